// peer_reduce.cu — in-place sum of one fp32 buffer over the GPUs of a node,
// over peer memory: every rank's buffer is mapped into every process (CUDA
// IPC), rank r adds chunk r of all buffers in rank order and stores the sum
// into chunk r of every buffer. One kernel per call; the result is bitwise
// identical on every rank and from run to run (a fixed summation order, unlike
// a ring all-reduce whose order depends on the ring).
//
// Synchronisation (flags in a small per-rank communication block, sequence
// numbers as in the TV slab exchange): at the start every CTA announces
// `arrive = seq` to all ranks and waits for all ranks' announcements (each
// rank's earlier work on its stream, e.g. the backward that filled the
// buffer, is then complete); at the end the last CTA of each rank announces
// `done = seq` and waits for everyone's, so that when the kernel completes all
// ranks' stores into this rank's buffer have landed and no rank still reads
// it. Waits are bounded: on expiry the kernel sets QC_FAULT_PEER_WAIT in the
// reduction's fault word and returns.
#include "qc_common.cuh"

namespace qc {
namespace pr {

__device__ unsigned int g_pr_fault_word = 0;

constexpr uint64_t kDefaultLimitNs = 10000000000ull;
constexpr int kThreads = 512;

struct Comm {
    unsigned long long arrive[QC_MAX_PEER_RANKS];
    unsigned long long done[QC_MAX_PEER_RANKS];
    unsigned int count;  // CTAs of this rank's launch that finished storing
    unsigned int pad[31];
};

// Flags are raised as one system-scope fence followed by relaxed stores (one
// fence for all ranks' flags instead of one per flag).
__device__ __forceinline__ void st_relaxed_sys(unsigned long long *p, unsigned long long v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ bool wait_geq(const unsigned long long *f, unsigned long long seq,
                                         uint64_t limit) {
    if (ld_acquire_sys(f) >= seq) return true;
    const uint64_t t0 = global_timer_ns();
    while (true) {
        __nanosleep(64);
        if (ld_acquire_sys(f) >= seq) return true;
        if (global_timer_ns() - t0 > limit) return false;
    }
}
__device__ __forceinline__ float4 ld_cg4(const float *p) {
    float4 v;
    asm volatile("ld.global.cg.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p));
    return v;
}
__device__ __forceinline__ float ld_cg1(const float *p) {
    float v;
    asm volatile("ld.global.cg.f32 %0, [%1];" : "=f"(v) : "l"(p));
    return v;
}

// Sums float4 i of chunk [b4, e4) of the range that starts at float `base`
// (16-byte aligned) over the ranks in rank order and stores it into every
// rank's buffer; `n` is the float count the range's float4s cover. WORLD > 0:
// the rank count is a compile-time constant, so all WORLD x U loads of a
// thread are issued before the first add (U float4s per thread per iteration
// keep 8-16 NVLink reads in flight).
template <int WORLD>
__device__ __forceinline__ void sum_chunk(const qc_peer_group &g, long long base, long long b4, long long e4,
                                          long long n) {
    constexpr int U = WORLD <= 4 ? 4 : 2;
    const long long stride = (long long)gridDim.x * blockDim.x;
    long long i = b4 + (long long)blockIdx.x * blockDim.x + threadIdx.x;
    for (; i + (U - 1) * stride < e4; i += U * stride) {
        // the iteration's largest index; the smaller ones follow
        if (!QC_IN_BOUNDS(4 * (i + (U - 1) * stride) + 3, n, g_pr_fault_word)) break;
        float4 v[U][WORLD];
#pragma unroll
        for (int u = 0; u < U; ++u)
#pragma unroll
            for (int q = 0; q < WORLD; ++q) v[u][q] = ld_cg4(g.buf[q] + base + 4 * (i + u * stride));
#pragma unroll
        for (int u = 0; u < U; ++u) {
            float4 s = v[u][0];
#pragma unroll
            for (int q = 1; q < WORLD; ++q) {
                s.x += v[u][q].x;
                s.y += v[u][q].y;
                s.z += v[u][q].z;
                s.w += v[u][q].w;
            }
            const long long j = i + u * stride;
#pragma unroll
            for (int q = 0; q < WORLD; ++q) *reinterpret_cast<float4 *>(g.buf[q] + base + 4 * j) = s;
        }
    }
    for (; i < e4; i += stride) {
        if (!QC_IN_BOUNDS(4 * i + 3, n, g_pr_fault_word)) continue;
        float4 v[WORLD];
#pragma unroll
        for (int q = 0; q < WORLD; ++q) v[q] = ld_cg4(g.buf[q] + base + 4 * i);
        float4 s = v[0];
#pragma unroll
        for (int q = 1; q < WORLD; ++q) {
            s.x += v[q].x;
            s.y += v[q].y;
            s.z += v[q].z;
            s.w += v[q].w;
        }
#pragma unroll
        for (int q = 0; q < WORLD; ++q) *reinterpret_cast<float4 *>(g.buf[q] + base + 4 * i) = s;
    }
}

// Any rank count (a runtime loop over the ranks).
__device__ __forceinline__ void sum_chunk_any(const qc_peer_group &g, long long base, long long b4, long long e4,
                                              long long n) {
    const long long stride = (long long)gridDim.x * blockDim.x;
    for (long long i = b4 + (long long)blockIdx.x * blockDim.x + threadIdx.x; i < e4; i += stride) {
        if (!QC_IN_BOUNDS(4 * i + 3, n, g_pr_fault_word)) continue;
        float4 s = ld_cg4(g.buf[0] + base + 4 * i);
        for (int q = 1; q < g.world; ++q) {
            const float4 v = ld_cg4(g.buf[q] + base + 4 * i);
            s.x += v.x;
            s.y += v.y;
            s.z += v.z;
            s.w += v.w;
        }
        for (int q = 0; q < g.world; ++q) *reinterpret_cast<float4 *>(g.buf[q] + base + 4 * i) = s;
    }
}

// One float at index i of every buffer, summed in rank order and stored back.
__device__ __forceinline__ void sum_one(const qc_peer_group &g, long long i) {
    float s = ld_cg1(g.buf[0] + i);
    for (int q = 1; q < g.world; ++q) s += ld_cg1(g.buf[q] + i);
    for (int q = 0; q < g.world; ++q) g.buf[q][i] = s;
}

// Sums floats [off, off + n) of every buffer.
__global__ void __launch_bounds__(kThreads, 2) allreduce_kernel(qc_peer_group g, unsigned long long seq,
                                                             long long off, long long n) {
    Comm *self = static_cast<Comm *>(g.comm[g.rank]);
    const uint64_t limit = g.timeout_ns ? g.timeout_ns : kDefaultLimitNs;
    __shared__ int go;
    if (threadIdx.x == 0) {
        __threadfence_system();
        for (int q = 0; q < g.world; ++q)
            st_relaxed_sys(&static_cast<Comm *>(g.comm[q])->arrive[g.rank], seq);
        bool ok = true;
        for (int q = 0; q < g.world; ++q) ok = wait_geq(&self->arrive[q], seq, limit) && ok;
        if (!ok) atomicOr(&g_pr_fault_word, QC_FAULT_PEER_WAIT);
        go = ok ? 1 : 0;
    }
    __syncthreads();
    if (go) {
        // floats before the range's first 16-byte boundary, then float4s,
        // then the floats after the last whole float4
        const long long head = (off % 4 == 0) ? 0 : (4 - off % 4 < n ? 4 - off % 4 : n);
        const long long base = off + head;
        const long long n4 = (n - head) / 4;
        // this rank's chunk of the float4s; the last rank takes the remainder
        const long long per = n4 / g.world;
        const long long b4 = per * g.rank;
        const long long e4 = g.rank == g.world - 1 ? n4 : b4 + per;
        switch (g.world) {
            case 2: sum_chunk<2>(g, base, b4, e4, 4 * n4); break;
            case 4: sum_chunk<4>(g, base, b4, e4, 4 * n4); break;
            case 8: sum_chunk<8>(g, base, b4, e4, 4 * n4); break;
            default: sum_chunk_any(g, base, b4, e4, 4 * n4); break;
        }
        if (g.rank == g.world - 1 && blockIdx.x == 0) {
            if (threadIdx.x < head) sum_one(g, off + threadIdx.x);
            for (long long i = base + 4 * n4 + threadIdx.x; i < off + n; i += blockDim.x) sum_one(g, i);
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        if (atomicAdd(&self->count, 1u) == gridDim.x - 1) {
            self->count = 0;  // the next call on this stream starts after this grid
            __threadfence_system();
            for (int q = 0; q < g.world; ++q)
                st_relaxed_sys(&static_cast<Comm *>(g.comm[q])->done[g.rank], seq);
            bool ok = true;
            for (int q = 0; q < g.world; ++q) ok = wait_geq(&self->done[q], seq, limit) && ok;
            if (!ok) atomicOr(&g_pr_fault_word, QC_FAULT_PEER_WAIT);
        }
    }
}

}  // namespace pr

int pr_fault_word(unsigned int *word, int clear) {
    unsigned int w = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&w, pr::g_pr_fault_word, sizeof(w));
    if (e == cudaSuccess && clear) {
        const unsigned int zero = 0;
        e = cudaMemcpyToSymbol(pr::g_pr_fault_word, &zero, sizeof(zero));
    }
    QC_CUDA_TRY(e, "cudaMemcpyFromSymbol(all-reduce fault word)");
    *word = w;
    return 0;
}

}  // namespace qc

extern "C" {

size_t peer_allreduce_comm_bytes(void) { return sizeof(qc::pr::Comm); }

int peer_allreduce_sum_f32_cuda(const qc_peer_group *g, unsigned long long seq, long long n,
                                cudaStream_t stream) {
    return peer_allreduce_sum_f32_range_cuda(g, seq, 0, n, 0, stream);
}

int peer_allreduce_sum_f32_range_cuda(const qc_peer_group *g, unsigned long long seq, long long offset,
                                      long long n, int max_ctas, cudaStream_t stream) {
    QC_NVTX("quantem::peer_allreduce");
    QC_RETURN_IF(g == nullptr, QC_ERR_INVALID_ARGUMENT, "peer_allreduce: null group");
    QC_RETURN_IF(g->world < 1 || g->world > QC_MAX_PEER_RANKS || g->rank < 0 ||
                     g->rank >= g->world,
                 QC_ERR_INVALID_ARGUMENT, "peer_allreduce: rank %d of %d", g->rank, g->world);
    QC_RETURN_IF(seq == 0, QC_ERR_INVALID_ARGUMENT, "peer_allreduce: seq starts at 1");
    QC_RETURN_IF(n < 0 || offset < 0 || max_ctas < 0, QC_ERR_INVALID_ARGUMENT,
                 "peer_allreduce: negative offset, size or CTA count");
    for (int q = 0; q < g->world; ++q) {
        QC_RETURN_IF(g->comm[q] == nullptr || g->buf[q] == nullptr, QC_ERR_INVALID_ARGUMENT,
                     "peer_allreduce: rank %d's buffer or communication block missing", q);
        QC_RETURN_IF(reinterpret_cast<uintptr_t>(g->buf[q]) % 16 != 0, QC_ERR_INVALID_ARGUMENT,
                     "peer_allreduce: buffers must be 16-byte aligned");
    }
    if (g->world == 1) return 0;
    int sms = 0;
    if (int st = qc::device_sm_count(&sms)) return st;
    const long long per4 = n / 4 / g->world + 1;
    long long grid = (per4 + qc::pr::kThreads - 1) / qc::pr::kThreads;
    const long long cap = max_ctas > 0 ? (long long)max_ctas : 2LL * sms;
    if (grid > cap) grid = cap;
    if (grid < 1) grid = 1;
    qc::pr::allreduce_kernel<<<(unsigned)grid, qc::pr::kThreads, 0, stream>>>(*g, seq, offset, n);
    QC_CHECK_LAUNCH("peer allreduce_kernel launch");
    return 0;
}

int peer_allreduce_fault_word(int device, unsigned int *word, int clear) {
    int prev = 0;
    QC_CUDA_TRY(cudaGetDevice(&prev), "cudaGetDevice");
    QC_CUDA_TRY(cudaSetDevice(device), "cudaSetDevice");
    unsigned int w = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&w, qc::pr::g_pr_fault_word, sizeof(w));
    if (e == cudaSuccess && clear) {
        const unsigned int zero = 0;
        e = cudaMemcpyToSymbol(qc::pr::g_pr_fault_word, &zero, sizeof(zero));
    }
    cudaSetDevice(prev);
    QC_CUDA_TRY(e, "cudaMemcpyFromSymbol(allreduce fault word)");
    if (word) *word = w;
    return 0;
}

}  // extern "C"
