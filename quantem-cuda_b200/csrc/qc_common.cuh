// qc_common.cuh — helpers shared by the sm_100a translation units: status
// plumbing for the C ABI, and thin inline-PTX wrappers for the Blackwell
// features the kernels use (mbarrier, TMA tiled loads, vector reductions,
// programmatic dependent launch).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <nvtx3/nvToolsExt.h>
#include <stdint.h>

#include "quantem_cuda_b200.h"

namespace qc {

// ── host-side status ──────────────────────────────────────────────────────
// Records `msg` as this thread's last error and returns `status` unchanged.
int set_error(int status, const char *fmt, ...);
// Converts a CUDA runtime error into a status (0 stays 0) with context.
int check_cuda(cudaError_t err, const char *what);

#define QC_RETURN_IF(cond, status, ...)                                                        \
    do {                                                                                       \
        if (cond) return ::qc::set_error((status), __VA_ARGS__);                               \
    } while (0)

#define QC_CUDA_TRY(call, what)                                                                \
    do {                                                                                       \
        int _st = ::qc::check_cuda((call), (what));                                            \
        if (_st) return _st;                                                                   \
    } while (0)

// Launch-time check after a <<<>>> launch: cudaPeekAtLastError, no sync
// (the reference's CUDA_CHECK_KERNEL, csrc/common.cuh:26-33, as a status).
#define QC_CHECK_LAUNCH(what) QC_CUDA_TRY(cudaPeekAtLastError(), (what))

// Number of SMs of the current device (cached per device).
int device_sm_count(int *sms);

// NVTX range over a C-ABI entry point, so that a profiler timeline shows each
// call by name next to its kernels (NVTX costs nothing without a tool).
struct NvtxRange {
    explicit NvtxRange(const char *name) { nvtxRangePushA(name); }
    ~NvtxRange() { nvtxRangePop(); }
    NvtxRange(const NvtxRange &) = delete;
    NvtxRange &operator=(const NvtxRange &) = delete;
};
#define QC_NVTX(name) ::qc::NvtxRange qc_nvtx_range_(name)

// ── device-side PTX wrappers ──────────────────────────────────────────────
__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}

// Makes mbarrier initialisation visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Waits for the phase of `bar` with the given parity to complete, for at most
// `limit_ns` nanoseconds. Returns false if it gave up.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity,
                                                  uint64_t limit_ns) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (global_timer_ns() - t0 > limit_ns) return false;
    }
}

// TMA: 3-D tiled bulk copy global -> shared, completion signalled on `bar`
// (complete_tx). No multicast. x must be a multiple of 4 fp32 elements.
__device__ __forceinline__ void tma_load_3d(void *smem_dst, const CUtensorMap *map, int x, int y,
                                            int z, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_addr(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ void prefetch_tensor_map(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Vector fp32 reduction to global memory (sm_90+): one L2 atomic op for 16 B.
__device__ __forceinline__ void red_add_v4(float *addr, float4 v) {
    asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(addr), "f"(v.x), "f"(v.y),
                 "f"(v.z), "f"(v.w)
                 : "memory");
}

// Programmatic dependent launch: the dependent grid may start its prologue;
// griddep_wait() blocks until all prerequisite grids completed and flushed.
__device__ __forceinline__ void griddep_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void griddep_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

__device__ __forceinline__ float4 ldg4(const float *p) {
    return __ldg(reinterpret_cast<const float4 *>(p));
}

// Bounds checks of the debug build (-DQC_DEBUG_BOUNDS): true when
// 0 <= i < n; otherwise sets QC_FAULT_BOUNDS in `word` and returns false, and
// the caller skips (or redirects) the access. The release build compiles them
// out.
__device__ __forceinline__ bool in_bounds_checked(long long i, long long n, unsigned int *word) {
    if (i >= 0 && i < n) return true;
    atomicOr(word, QC_FAULT_BOUNDS);
    return false;
}
#ifdef QC_DEBUG_BOUNDS
#define QC_IN_BOUNDS(i, n, word) (::qc::in_bounds_checked((long long)(i), (long long)(n), &(word)))
#else
#define QC_IN_BOUNDS(i, n, word) true
#endif

// Fault words of the kernel families compiled in other translation units
// (each reads the current device's word, clearing it if `clear`).
int kp_fault_word(unsigned int *word, int clear);
int pr_fault_word(unsigned int *word, int clear);

}  // namespace qc
