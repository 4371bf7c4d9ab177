// tv_sweep.cu — 3-D total-variation losses and gradients for sm_100a.
//
// Reference semantics: csrc/cuda/core/tv_loss.cu (six kernels, one per
// variant × {loss, gradient}); operator layer src/quantem/cuda/core/_ops.py.
//
// All three variants share one structure. For a voxel v at (d, h, w) let the
// forward differences be dd = v[d+1]-v, dh = v[h+1]-v, dw = v[w+1]-v, each
// present only where the neighbour exists. Each variant defines a per-voxel
// "flux" F = (Fd, Fh, Fw) from those differences, and its gradient is the
// backward divergence of F:
//
//   grad(v) = gmul · Σ_axis ( F_axis(voxel − e_axis) − F_axis(v) )
//
//   squared  F_axis = diff_axis                       gmul = 2g     loss Σ diff²
//   L1       F_axis = g_axis · sign(diff_axis)        gmul = 1      loss_axis Σ |diff|
//   iso      F_axis = diff_axis / s (corner valid)    gmul = g/N    loss Σ s,
//            s = sqrt(dd² + dh² + dw² + eps); a corner is valid when all three
//            neighbours exist (tv_loss.cu:64, :167-188).
//
// This reproduces the reference's gradient kernels term by term
// (tv_loss.cu:320-330 for squared, :462-473 for L1, :165-188 for iso) while
// letting one sweep produce loss and gradient together.
//
// Fast path (W % 4 == 0, 16-byte aligned pointers): a warp-specialised CTA
// marches along D through a column of 16×128 (H×W) tiles. One producer warp
// streams each plane tile plus a one-voxel halo (18 rows × 136 columns; the
// left halo is 4 columns wide because a TMA box must start on a 16-byte
// boundary) into a 4-stage shared-memory ring with cp.async.bulk.tensor; four
// consumer warps each own 4 rows × 128 columns (4 consecutive columns per
// lane), keep the previous plane's Fd in registers, and take in-plane
// neighbours from shared memory and warp shuffles. Each voxel is read from HBM
// once per sweep (halo rows/columns are shared with neighbouring tiles, which
// the chunk-major schedule processes at the same time, so they hit L2).
//
// Reductions are deterministic: each CTA writes fp64 partial sums to a
// caller-owned workspace slot, and a one-CTA finalize kernel, launched with
// programmatic dependent launch, sums the slots in fixed order.
#include <stdio.h>

#include <mutex>

#include "qc_common.cuh"

namespace qc {
namespace tv {

// Set (bit 0) by a TMA-ring wait that gave up instead of hanging.
__device__ unsigned int g_tv_fault_word = 0;

constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s per barrier wait

constexpr int kMaxPartials = 2048;  // CTA partial-sum slots in the workspace
constexpr int kAccSlots = 3;        // L1 keeps one sum per axis

// ── per-variant arithmetic ───────────────────────────────────────────────

__device__ __forceinline__ float sgnf(float x) {
    // torch's convention for d|x|/dx: sign(0) = 0 (tv_loss.cu:434-436).
    return (float)((x > 0.0f) - (x < 0.0f));
}

struct Gains {
    float gmul;      // multiplies the divergence
    float gd, gh, gw;  // L1 per-axis gains folded into F
};

// Loss terms and flux at a voxel with value v and +1 neighbours (nd, nh, nw);
// vd/vh/vw say whether each neighbour exists. `own` gates the loss.
template <int V, bool LOSS, bool GRAD>
__device__ __forceinline__ void voxel_flux(float v, float nd, float nh, float nw, bool vd, bool vh,
                                           bool vw, bool own, float eps, const Gains &gn,
                                           float &Fd, float &Fh, float &Fw, float &l0, float &l1,
                                           float &l2) {
    const float dd = nd - v, dh = nh - v, dw = nw - v;
    if constexpr (V == QC_TV_SQ) {
        if (LOSS && own) {
            float s = vd ? dd * dd : 0.f;
            s += vh ? dh * dh : 0.f;
            s += vw ? dw * dw : 0.f;
            l0 += s;
        }
        if (GRAD) {
            Fd = vd ? dd : 0.f;
            Fh = vh ? dh : 0.f;
            Fw = vw ? dw : 0.f;
        }
    } else if constexpr (V == QC_TV_L1) {
        if (LOSS && own) {
            l0 += vd ? fabsf(dd) : 0.f;
            l1 += vh ? fabsf(dh) : 0.f;
            l2 += vw ? fabsf(dw) : 0.f;
        }
        if (GRAD) {
            Fd = vd ? gn.gd * sgnf(dd) : 0.f;
            Fh = vh ? gn.gh * sgnf(dh) : 0.f;
            Fw = vw ? gn.gw * sgnf(dw) : 0.f;
        }
    } else {  // QC_TV_ISO
        const bool ok = vd && vh && vw;
        const float x = dd * dd + dh * dh + dw * dw + eps;
        if (LOSS && own) l0 += ok ? sqrtf(x) : 0.f;
        if (GRAD) {
            const float inv = rsqrtf(x);
            Fd = ok ? dd * inv : 0.f;
            Fh = ok ? dh * inv : 0.f;
            Fw = ok ? dw * inv : 0.f;
        }
    }
}

// Fh of the voxel one row up (h-1): `up` = v[h-1]; for iso the corner at
// (h-1) also needs v[d+1][h-1] (`up_nd`) and v[h-1][w+1] (`up_nw`).
template <int V>
__device__ __forceinline__ float flux_from_up(float v, float up, float up_nd, float up_nw,
                                              bool has_up, bool vd, bool vw_up, float eps,
                                              const Gains &gn) {
    if constexpr (V == QC_TV_SQ) {
        return has_up ? v - up : 0.f;
    } else if constexpr (V == QC_TV_L1) {
        return has_up ? gn.gh * sgnf(v - up) : 0.f;
    } else {
        const float dd = up_nd - up, dh = v - up, dw = up_nw - up;
        const bool ok = has_up && vd && vw_up;
        const float inv = rsqrtf(dd * dd + dh * dh + dw * dw + eps);
        return ok ? dh * inv : 0.f;
    }
}

// Fw of the voxel one column left (w-1): `lf` = v[w-1]; for iso the corner at
// (w-1) also needs v[d+1][w-1] (`lf_nd`) and v[h+1][w-1] (`lf_nh`).
template <int V>
__device__ __forceinline__ float flux_from_left(float v, float lf, float lf_nd, float lf_nh,
                                                bool has_left, bool vd, bool vh, float eps,
                                                const Gains &gn) {
    if constexpr (V == QC_TV_SQ) {
        return has_left ? v - lf : 0.f;
    } else if constexpr (V == QC_TV_L1) {
        return has_left ? gn.gw * sgnf(v - lf) : 0.f;
    } else {
        const float dd = lf_nd - lf, dh = lf_nh - lf, dw = v - lf;
        const bool ok = has_left && vd && vh;
        const float inv = rsqrtf(dd * dd + dh * dh + dw * dw + eps);
        return ok ? dw * inv : 0.f;
    }
}

template <int V>
__device__ __forceinline__ Gains load_gains(const float *g, float scale) {
    Gains gn{1.f, 0.f, 0.f, 0.f};
    if (g == nullptr) return gn;
    if constexpr (V == QC_TV_SQ) {
        gn.gmul = 2.0f * (__ldg(g) * scale);
    } else if constexpr (V == QC_TV_ISO) {
        gn.gmul = __ldg(g) * scale;
    } else {
        gn.gd = __ldg(g) * scale;
        gn.gh = __ldg(g + 1) * scale;
        gn.gw = __ldg(g + 2) * scale;
    }
    return gn;
}

// ── work plan shared by both paths ───────────────────────────────────────

struct Plan {
    int B, Dp, H, W;
    int d_lo, d_hi;          // owned planes [d_lo, d_hi) in every batch slice
    int has_prev, has_next;  // plane d_lo-1 / d_hi is a real neighbour
    int n_ht, n_wt;          // tiles per plane
    int n_cols;              // B * n_ht * n_wt
    int dchunk;              // planes per work unit
    int n_chunks;
    long long n_units;       // n_chunks * n_cols, chunk-major
    float eps;
    float scale;             // multiplies the gradient (and, on the host side, the sum)
};

struct Unit {
    int n, h0, w0;
    int d_start, d_end;  // owned planes of the unit
    int first, last;     // planes the unit loads (halo planes included)
};

template <bool GRAD>
__device__ __forceinline__ Unit decode_unit(const Plan &pl, long long u, int tile_h, int tile_w) {
    Unit U;
    const long long chunk = u / pl.n_cols;
    const int col = (int)(u - chunk * pl.n_cols);
    const int per_b = pl.n_ht * pl.n_wt;
    U.n = col / per_b;
    const int r = col - U.n * per_b;
    U.h0 = (r / pl.n_wt) * tile_h;
    U.w0 = (r % pl.n_wt) * tile_w;
    U.d_start = pl.d_lo + (int)chunk * pl.dchunk;
    U.d_end = min(U.d_start + pl.dchunk, pl.d_hi);
    const bool prev_exists = (U.d_start > pl.d_lo) || pl.has_prev;
    const bool next_exists = (U.d_end < pl.d_hi) || pl.has_next;
    U.first = (GRAD && prev_exists) ? U.d_start - 1 : U.d_start;
    U.last = next_exists ? U.d_end : U.d_end - 1;
    return U;
}

// ── fast path: TMA ring + warp-specialised D-march ───────────────────────

constexpr int kTileW = 128;                        // owned columns per tile
constexpr int kHaloW = 4;                          // halo columns each side
constexpr int kBoxW = kTileW + 2 * kHaloW;         // 136
constexpr int kRowsPerWarp = 4;
constexpr int kConsumerWarps = 4;
constexpr int kTileH = kRowsPerWarp * kConsumerWarps;  // 16
constexpr int kBoxH = kTileH + 2;                  // 18
constexpr int kStages = 4;
constexpr uint32_t kBoxBytes = kBoxW * kBoxH * 4;  // 9792
constexpr int kStageFloats = 2464;                 // 9856 B: keeps each stage 128-B aligned
constexpr int kSweepThreads = (kConsumerWarps + 1) * 32;
static_assert(kStageFloats * 4 >= (int)kBoxBytes, "stage too small");
static_assert((kStageFloats * 4) % 128 == 0, "stage alignment");

struct SweepSmem {
    float stage[kStages][kStageFloats];
    uint64_t full[kStages];
    uint64_t empty[kStages];
    double red[kConsumerWarps][kAccSlots];
    int abort;
};
static_assert(sizeof(SweepSmem) + 128 <= 48 * 1024, "sweep smem must fit without opt-in");

__device__ __forceinline__ bool aborted(const SweepSmem &sm) {
    return *reinterpret_cast<const volatile int *>(&sm.abort) != 0;
}

__device__ __forceinline__ float4 lds4(const float *s, int row, int col) {
    return *reinterpret_cast<const float4 *>(s + row * kBoxW + col);
}
__device__ __forceinline__ float lds1(const float *s, int row, int col) {
    return s[row * kBoxW + col];
}

template <int V, bool LOSS, bool GRAD>
__global__ void __launch_bounds__(kSweepThreads) tv_sweep_tma_kernel(
    const __grid_constant__ CUtensorMap map, const float *__restrict__ g,
    float *__restrict__ grad, double *__restrict__ partials, const Plan pl) {
    // TMA destinations must be 128-byte aligned: align the ring explicitly
    // (the launch requests sizeof(SweepSmem) + 128 bytes).
    extern __shared__ __align__(128) unsigned char smem_raw[];
    SweepSmem &sm = *reinterpret_cast<SweepSmem *>(smem_raw + ((128u - (smem_addr(smem_raw) & 127u)) & 127u));
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&sm.full[s], 1);
            mbar_init(&sm.empty[s], kConsumerWarps);
        }
        sm.abort = 0;
        fence_mbar_init();
    }
    __syncthreads();

    double acc0 = 0.0, acc1 = 0.0, acc2 = 0.0;

    if (warp == kConsumerWarps) {
        // ── producer warp: one lane issues every TMA load ──
        if (lane == 0) {
            prefetch_tensor_map(&map);
            long long seq = 0;
            long long last_seq[kStages] = {-1, -1, -1, -1};
            for (long long u = blockIdx.x; u < pl.n_units && !aborted(sm); u += gridDim.x) {
                const Unit U = decode_unit<GRAD>(pl, u, kTileH, kTileW);
                const int zbase = U.n * pl.Dp;
                for (int p = U.first; p <= U.last; ++p, ++seq) {
                    const int s = (int)(seq % kStages);
                    if (seq >= kStages) {
                        const uint32_t par = (uint32_t)(((seq / kStages) - 1) & 1);
                        if (!mbar_wait_bounded(&sm.empty[s], par, kWaitLimitNs)) {
                            atomicOr(&g_tv_fault_word, 1u);
                            sm.abort = 1;
                            break;
                        }
                    }
                    mbar_arrive_expect_tx(&sm.full[s], kBoxBytes);
                    tma_load_3d(sm.stage[s], &map, U.w0 - kHaloW, U.h0 - 1, zbase + p, &sm.full[s]);
                    last_seq[s] = seq;
                }
            }
            // Never leave a bulk copy in flight into shared memory that is about
            // to be released: wait (bounded) for the last load of every stage.
            for (int s = 0; s < kStages; ++s) {
                if (last_seq[s] < 0) continue;
                const uint32_t par = (uint32_t)((last_seq[s] / kStages) & 1);
                if (!mbar_wait_bounded(&sm.full[s], par, kWaitLimitNs))
                    atomicOr(&g_tv_fault_word, 1u);
            }
        }
    } else {
        // ── consumer warps ──
        const Gains gn = load_gains<V>(g, pl.scale);
        const int r0 = warp * kRowsPerWarp;  // first tile row of this warp's strip
        const int scol = kHaloW + 4 * lane;  // smem column of this lane's first voxel
        float Fd_prev[kRowsPerWarp][4];
        long long seq = 0;

        for (long long u = blockIdx.x; u < pl.n_units; u += gridDim.x) {
            const Unit U = decode_unit<GRAD>(pl, u, kTileH, kTileW);
            const int wcol = U.w0 + 4 * lane;  // global column of the lane's first voxel
            const bool col_in = wcol < pl.W;   // W % 4 == 0: 4 voxels all in or all out
#pragma unroll
            for (int i = 0; i < kRowsPerWarp; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) Fd_prev[i][j] = 0.f;

            const long long q0 = seq;
            {
                const int s0 = (int)(q0 % kStages);
                if (!mbar_wait_bounded(&sm.full[s0], (uint32_t)((q0 / kStages) & 1),
                                       kWaitLimitNs)) {
                    atomicOr(&g_tv_fault_word, 1u);
                    sm.abort = 1;
                }
            }
            if (aborted(sm)) break;

            for (int p = U.first; p < U.d_end; ++p) {
                const long long qc = q0 + (p - U.first);
                const bool has_nxt = (p + 1) <= U.last;
                const float *Sc = sm.stage[qc % kStages];
                const float *Sn = Sc;
                if (has_nxt) {
                    const long long qn = qc + 1;
                    const int sn = (int)(qn % kStages);
                    if (!mbar_wait_bounded(&sm.full[sn], (uint32_t)((qn / kStages) & 1),
                                           kWaitLimitNs)) {
                        atomicOr(&g_tv_fault_word, 1u);
                        sm.abort = 1;
                    }
                    Sn = sm.stage[sn];
                }
                if (aborted(sm)) break;
                const bool owned = p >= U.d_start;
                float l0 = 0.f, l1 = 0.f, l2 = 0.f;

                // Row above the strip (tile row r0-1 is smem row r0).
                float4 up = make_float4(0.f, 0.f, 0.f, 0.f), up_nd = up;
                float up_right = 0.f;
                if (GRAD) {
                    up = lds4(Sc, r0, scol);
                    if (V == QC_TV_ISO) {
                        up_nd = lds4(Sn, r0, scol);
                        up_right = __shfl_down_sync(0xffffffffu, up.x, 1);
                        if (lane == 31) up_right = lds1(Sc, r0, scol + 4);
                    }
                }
                float Fh_up[4];
                float4 cur = lds4(Sc, r0 + 1, scol);
                const int hbase = U.h0 + r0;

#pragma unroll
                for (int i = 0; i < kRowsPerWarp; ++i) {
                    const int h = hbase + i;
                    const int srow = r0 + 1 + i;  // smem row of tile row r0+i
                    const float4 down = lds4(Sc, srow + 1, scol);
                    const float4 nxt = has_nxt ? lds4(Sn, srow, scol) : make_float4(0.f, 0.f, 0.f, 0.f);
                    float right = __shfl_down_sync(0xffffffffu, cur.x, 1);
                    if (lane == 31) right = lds1(Sc, srow, scol + 4);

                    const float cv[4] = {cur.x, cur.y, cur.z, cur.w};
                    const float nv[4] = {nxt.x, nxt.y, nxt.z, nxt.w};
                    const float dv[4] = {down.x, down.y, down.z, down.w};
                    const float rv[4] = {cur.y, cur.z, cur.w, right};
                    const bool row_in = h < pl.H;
                    const bool vh = h + 1 < pl.H;
                    float Fd[4], Fh[4], Fw[4];
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const bool vw = wcol + j + 1 < pl.W;
                        voxel_flux<V, LOSS, GRAD>(cv[j], nv[j], dv[j], rv[j], has_nxt, vh, vw,
                                                  owned && row_in && col_in, pl.eps, gn, Fd[j],
                                                  Fh[j], Fw[j], l0, l1, l2);
                    }

                    if (GRAD) {
                        // Fh one row up: from the halo row for the strip's first
                        // row, else carried from the previous row.
                        if (i == 0) {
                            const float uv[4] = {up.x, up.y, up.z, up.w};
                            const float und[4] = {up_nd.x, up_nd.y, up_nd.z, up_nd.w};
                            const float unw[4] = {up.y, up.z, up.w, up_right};
#pragma unroll
                            for (int j = 0; j < 4; ++j)
                                Fh_up[j] = flux_from_up<V>(cv[j], uv[j], und[j], unw[j], h >= 1,
                                                           has_nxt, wcol + j + 1 < pl.W, pl.eps,
                                                           gn);
                        }
                        // Fw one column left of the lane's first voxel.
                        float lf = __shfl_up_sync(0xffffffffu, cur.w, 1);
                        if (lane == 0) lf = lds1(Sc, srow, scol - 1);
                        float lf_nd = 0.f, lf_nh = 0.f;
                        if (V == QC_TV_ISO) {
                            lf_nd = __shfl_up_sync(0xffffffffu, nxt.w, 1);
                            lf_nh = __shfl_up_sync(0xffffffffu, down.w, 1);
                            if (lane == 0) {
                                lf_nd = has_nxt ? lds1(Sn, srow, scol - 1) : 0.f;
                                lf_nh = lds1(Sc, srow + 1, scol - 1);
                            }
                        }
                        const float Fw_left0 = flux_from_left<V>(cv[0], lf, lf_nd, lf_nh,
                                                                 wcol >= 1, has_nxt, vh, pl.eps, gn);
                        const float Fw_left[4] = {Fw_left0, Fw[0], Fw[1], Fw[2]};
                        float gv[4];
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            gv[j] = gn.gmul * ((Fd_prev[i][j] - Fd[j]) + (Fh_up[j] - Fh[j]) +
                                               (Fw_left[j] - Fw[j]));
                            Fd_prev[i][j] = Fd[j];
                            Fh_up[j] = Fh[j];
                        }
                        if (owned && row_in && col_in) {
                            const size_t idx =
                                (((size_t)U.n * pl.Dp + p) * pl.H + h) * (size_t)pl.W + wcol;
                            __stcs(reinterpret_cast<float4 *>(grad + idx),
                                   make_float4(gv[0], gv[1], gv[2], gv[3]));
                        }
                    }
                    cur = down;
                }
                if (LOSS) {
                    acc0 += (double)l0;
                    if (V == QC_TV_L1) {
                        acc1 += (double)l1;
                        acc2 += (double)l2;
                    }
                }
                // Release plane p's stage.
                __syncwarp();
                if (lane == 0) mbar_arrive(&sm.empty[qc % kStages]);
            }
            if (aborted(sm)) break;
            if (U.last == U.d_end) {
                // The +1 halo plane was only ever a "next" plane: release it too.
                const long long ql = q0 + (U.last - U.first);
                __syncwarp();
                if (lane == 0) mbar_arrive(&sm.empty[ql % kStages]);
            }
            seq = q0 + (U.last - U.first + 1);
        }
    }

    griddep_launch_dependents();

    if (LOSS) {
        if (warp < kConsumerWarps) {
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) {
                acc0 += __shfl_xor_sync(0xffffffffu, acc0, off);
                acc1 += __shfl_xor_sync(0xffffffffu, acc1, off);
                acc2 += __shfl_xor_sync(0xffffffffu, acc2, off);
            }
            if (lane == 0) {
                sm.red[warp][0] = acc0;
                sm.red[warp][1] = acc1;
                sm.red[warp][2] = acc2;
            }
        }
        __syncthreads();
        if (threadIdx.x < kAccSlots) {
            double t = 0.0;
            for (int w = 0; w < kConsumerWarps; ++w) t += sm.red[w][threadIdx.x];
            partials[(size_t)blockIdx.x * kAccSlots + threadIdx.x] = t;
        }
    }
}

// ── generic path (any W, any alignment) ─────────────────────────────────

constexpr int kGenTileW = 32, kGenTileH = 8;
constexpr int kGenThreads = kGenTileW * kGenTileH;

template <int V, bool LOSS, bool GRAD>
__global__ void __launch_bounds__(kGenThreads) tv_sweep_generic_kernel(
    const float *__restrict__ vol, const float *__restrict__ g, float *__restrict__ grad,
    double *__restrict__ partials, const Plan pl) {
    const Gains gn = load_gains<V>(g, pl.scale);
    const int tx = threadIdx.x % kGenTileW, ty = threadIdx.x / kGenTileW;
    const size_t plane = (size_t)pl.H * pl.W;
    double acc0 = 0.0, acc1 = 0.0, acc2 = 0.0;

    for (long long u = blockIdx.x; u < pl.n_units; u += gridDim.x) {
        const Unit U = decode_unit<GRAD>(pl, u, kGenTileH, kGenTileW);
        const int h = U.h0 + ty, w = U.w0 + tx;
        const bool in = h < pl.H && w < pl.W;
        const float *vb = vol + (size_t)U.n * pl.Dp * plane;
        auto at = [&](int p, int hh, int ww) -> float {
            return __ldg(vb + (size_t)p * plane + (size_t)hh * pl.W + ww);
        };
        const bool vh = h + 1 < pl.H, vw = w + 1 < pl.W;
        float Fd_prev = 0.f;
        for (int p = U.first; p < U.d_end; ++p) {
            const bool has_nxt = (p + 1) <= U.last;
            const bool owned = p >= U.d_start;
            float l0 = 0.f, l1 = 0.f, l2 = 0.f;
            float Fd = 0.f, Fh = 0.f, Fw = 0.f;
            if (in) {
                const float v = at(p, h, w);
                const float nd = has_nxt ? at(p + 1, h, w) : 0.f;
                const float nh = vh ? at(p, h + 1, w) : 0.f;
                const float nw = vw ? at(p, h, w + 1) : 0.f;
                voxel_flux<V, LOSS, GRAD>(v, nd, nh, nw, has_nxt, vh, vw, owned, pl.eps, gn, Fd,
                                          Fh, Fw, l0, l1, l2);
                if (GRAD && owned) {
                    float Fh_up = 0.f, Fw_left = 0.f;
                    if (h >= 1) {
                        const float up = at(p, h - 1, w);
                        const float up_nd = (V == QC_TV_ISO && has_nxt) ? at(p + 1, h - 1, w) : 0.f;
                        const float up_nw = (V == QC_TV_ISO && vw) ? at(p, h - 1, w + 1) : 0.f;
                        Fh_up = flux_from_up<V>(v, up, up_nd, up_nw, true, has_nxt, vw, pl.eps, gn);
                    }
                    if (w >= 1) {
                        const float lf = at(p, h, w - 1);
                        const float lf_nd = (V == QC_TV_ISO && has_nxt) ? at(p + 1, h, w - 1) : 0.f;
                        const float lf_nh = (V == QC_TV_ISO && vh) ? at(p, h + 1, w - 1) : 0.f;
                        Fw_left = flux_from_left<V>(v, lf, lf_nd, lf_nh, true, has_nxt, vh, pl.eps, gn);
                    }
                    const float gv =
                        gn.gmul * ((Fd_prev - Fd) + (Fh_up - Fh) + (Fw_left - Fw));
                    grad[(size_t)U.n * pl.Dp * plane + (size_t)p * plane + (size_t)h * pl.W + w] = gv;
                }
            }
            Fd_prev = Fd;
            if (LOSS) {
                acc0 += (double)l0;
                acc1 += (double)l1;
                acc2 += (double)l2;
            }
        }
    }

    griddep_launch_dependents();

    if (LOSS) {
        __shared__ double red[kGenThreads / 32][kAccSlots];
        const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            acc0 += __shfl_xor_sync(0xffffffffu, acc0, off);
            acc1 += __shfl_xor_sync(0xffffffffu, acc1, off);
            acc2 += __shfl_xor_sync(0xffffffffu, acc2, off);
        }
        if (lane == 0) {
            red[warp][0] = acc0;
            red[warp][1] = acc1;
            red[warp][2] = acc2;
        }
        __syncthreads();
        if (threadIdx.x < kAccSlots) {
            double t = 0.0;
            for (int w = 0; w < kGenThreads / 32; ++w) t += red[w][threadIdx.x];
            partials[(size_t)blockIdx.x * kAccSlots + threadIdx.x] = t;
        }
    }
}

// ── finalize: fixed-order sum of the CTA partials ────────────────────────

constexpr int kFinThreads = 256;

__global__ void __launch_bounds__(kFinThreads) tv_finalize_kernel(const double *__restrict__ partials,
                                                                  int n_partials, int n_acc,
                                                                  float *__restrict__ acc,
                                                                  float scale, int overwrite) {
    griddep_wait();  // the sweep grid has completed and its writes are visible
    __shared__ double red[kAccSlots][kFinThreads];
    for (int a = 0; a < n_acc; ++a) {
        double t = 0.0;
        for (int i = threadIdx.x; i < n_partials; i += kFinThreads)
            t += partials[(size_t)i * kAccSlots + a];
        red[a][threadIdx.x] = t;
    }
    __syncthreads();
    for (int s = kFinThreads / 2; s > 0; s >>= 1) {
        if (threadIdx.x < s)
            for (int a = 0; a < n_acc; ++a) red[a][threadIdx.x] += red[a][threadIdx.x + s];
        __syncthreads();
    }
    if (threadIdx.x < n_acc) {
        const float v = (float)(red[threadIdx.x][0] * (double)scale);
        acc[threadIdx.x] = overwrite ? v : acc[threadIdx.x] + v;
    }
}

// ── host side ────────────────────────────────────────────────────────────

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *,
                                  const cuuint64_t *, const cuuint64_t *, const cuuint32_t *,
                                  const cuuint32_t *, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int get_encode_fn(EncodeTiledFn *fn) {
    static std::once_flag once;
    static EncodeTiledFn cached = nullptr;
    static cudaError_t err = cudaSuccess;
    static cudaDriverEntryPointQueryResult qres = cudaDriverEntryPointSuccess;
    std::call_once(once, [] {
        void *p = nullptr;
        err = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &qres);
        cached = reinterpret_cast<EncodeTiledFn>(p);
    });
    if (err != cudaSuccess) return check_cuda(err, "cudaGetDriverEntryPoint(cuTensorMapEncodeTiled)");
    if (cached == nullptr || qres != cudaDriverEntryPointSuccess)
        return set_error(QC_ERR_NO_DEVICE, "cuTensorMapEncodeTiled is not available from the driver");
    *fn = cached;
    return 0;
}

// Chooses the D-chunk of the chunk-major units. Time is modelled, in units of
// one plane per CTA, as the larger of the critical path (rounds of units, each
// chunk + halo planes long) and the bandwidth bound (all plane loads spread
// over the CTAs it takes to saturate HBM, taken as 60% of the resident ones).
void choose_chunking(Plan &pl, int max_ctas, int halo_planes) {
    const int Dn = pl.d_hi - pl.d_lo;
    const double sat = 0.6 * max_ctas;
    double best = 1e300;
    int best_dc = Dn, prev_dc = -1;
    for (int nch = 1; nch <= Dn; ++nch) {
        const int dc = (Dn + nch - 1) / nch;
        if (dc == prev_dc) continue;
        prev_dc = dc;
        const int real_nch = (Dn + dc - 1) / dc;
        const long long U = (long long)real_nch * pl.n_cols;
        const long long rounds = (U + max_ctas - 1) / max_ctas;
        const double path = (double)rounds * (dc + halo_planes);
        const double bw = (double)U * (dc + halo_planes) / sat;
        const double cost = path > bw ? path : bw;
        if (cost < best * 0.999) {
            best = cost;
            best_dc = dc;
        }
        if (U > 64LL * max_ctas) break;
    }
    pl.dchunk = best_dc;
    pl.n_chunks = (Dn + best_dc - 1) / best_dc;
    pl.n_units = (long long)pl.n_chunks * pl.n_cols;
}

template <int V, bool LOSS, bool GRAD>
int launch_variant(bool use_tma, const float *vol, const float *g, float *grad, double *partials,
                   Plan pl, int *grid_out, cudaStream_t stream) {
    int sms = 0;
    if (int st = device_sm_count(&sms)) return st;
    if (use_tma) {
        EncodeTiledFn encode = nullptr;
        if (int st = get_encode_fn(&encode)) return st;
        CUtensorMap map;
        const cuuint64_t dims[3] = {(cuuint64_t)pl.W, (cuuint64_t)pl.H,
                                    (cuuint64_t)pl.B * (cuuint64_t)pl.Dp};
        const cuuint64_t strides[2] = {(cuuint64_t)pl.W * 4, (cuuint64_t)pl.W * pl.H * 4};
        const cuuint32_t box[3] = {kBoxW, kBoxH, 1};
        const cuuint32_t estr[3] = {1, 1, 1};
        CUresult cr = encode(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float *>(vol),
                             dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                             CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (cr != CUDA_SUCCESS)
            return set_error(QC_ERR_TENSOR_MAP, "cuTensorMapEncodeTiled failed (CUresult %d) for "
                             "W=%d H=%d planes=%lld", (int)cr, pl.W, pl.H,
                             (long long)pl.B * pl.Dp);
        auto kern = tv_sweep_tma_kernel<V, LOSS, GRAD>;
        const size_t smem = sizeof(SweepSmem) + 128;  // below 48 KB: no opt-in needed
        int occ = 0;
        QC_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kSweepThreads, smem),
                    "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
        int max_ctas = occ * sms;
        if (max_ctas > kMaxPartials) max_ctas = kMaxPartials;
        if (max_ctas < 1) max_ctas = 1;
        pl.n_ht = (pl.H + kTileH - 1) / kTileH;
        pl.n_wt = (pl.W + kTileW - 1) / kTileW;
        pl.n_cols = pl.B * pl.n_ht * pl.n_wt;
        choose_chunking(pl, max_ctas, 1 + (GRAD ? 1 : 0));
        const long long rounds = (pl.n_units + max_ctas - 1) / max_ctas;
        const int grid = (int)((pl.n_units + rounds - 1) / rounds);
        kern<<<grid, kSweepThreads, smem, stream>>>(map, g, grad, partials, pl);
        QC_CHECK_LAUNCH("tv_sweep_tma_kernel launch");
        *grid_out = grid;
    } else {
        auto kern = tv_sweep_generic_kernel<V, LOSS, GRAD>;
        int occ = 0;
        QC_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kGenThreads, 0),
                    "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
        int max_ctas = occ * sms;
        if (max_ctas > kMaxPartials) max_ctas = kMaxPartials;
        if (max_ctas < 1) max_ctas = 1;
        pl.n_ht = (pl.H + kGenTileH - 1) / kGenTileH;
        pl.n_wt = (pl.W + kGenTileW - 1) / kGenTileW;
        pl.n_cols = pl.B * pl.n_ht * pl.n_wt;
        choose_chunking(pl, max_ctas, 1 + (GRAD ? 1 : 0));
        const long long rounds = (pl.n_units + max_ctas - 1) / max_ctas;
        const int grid = (int)((pl.n_units + rounds - 1) / rounds);
        kern<<<grid, kGenThreads, 0, stream>>>(vol, g, grad, partials, pl);
        QC_CHECK_LAUNCH("tv_sweep_generic_kernel launch");
        *grid_out = grid;
    }
    return 0;
}

template <int V>
int dispatch_mode(int flags, bool use_tma, const float *vol, const float *g, float *grad,
                  double *partials, const Plan &pl, int *grid, cudaStream_t stream) {
    const bool L = flags & QC_TV_LOSS, G = flags & QC_TV_GRAD;
    if (L && G) return launch_variant<V, true, true>(use_tma, vol, g, grad, partials, pl, grid, stream);
    if (L) return launch_variant<V, true, false>(use_tma, vol, g, grad, partials, pl, grid, stream);
    return launch_variant<V, false, true>(use_tma, vol, g, grad, partials, pl, grid, stream);
}

size_t workspace_bytes() { return (size_t)kMaxPartials * kAccSlots * sizeof(double); }

int run(int variant, int flags, const float *vol, const float *g, float *acc, float *grad, int B,
        int Dp, int H, int W, int d_lo, int d_hi, int has_prev, int has_next, float eps,
        float acc_scale, void *ws, size_t ws_bytes, cudaStream_t stream) {
    const bool want_loss = flags & QC_TV_LOSS, want_grad = flags & QC_TV_GRAD;
    QC_RETURN_IF(variant < QC_TV_SQ || variant > QC_TV_L1, QC_ERR_INVALID_ARGUMENT,
                 "tv: unknown variant %d", variant);
    QC_RETURN_IF(!want_loss && !want_grad, QC_ERR_INVALID_ARGUMENT,
                 "tv: flags must request QC_TV_LOSS and/or QC_TV_GRAD");
    QC_RETURN_IF(B < 0 || Dp < 0 || H < 0 || W < 0, QC_ERR_INVALID_ARGUMENT,
                 "tv: negative shape [%d, %d, %d, %d]", B, Dp, H, W);
    QC_RETURN_IF(d_lo < 0 || d_hi > Dp || d_lo > d_hi, QC_ERR_INVALID_ARGUMENT,
                 "tv: owned planes [%d, %d) outside [0, %d)", d_lo, d_hi, Dp);
    QC_RETURN_IF(has_prev && d_lo < 1, QC_ERR_INVALID_ARGUMENT,
                 "tv: has_prev needs a halo plane below d_lo");
    QC_RETURN_IF(has_next && d_hi > Dp - 1, QC_ERR_INVALID_ARGUMENT,
                 "tv: has_next needs a halo plane at d_hi");
    QC_RETURN_IF((long long)H * W >= (1LL << 31), QC_ERR_INVALID_ARGUMENT,
                 "tv: H*W must be < 2^31");
    const int n_acc = variant == QC_TV_L1 ? 3 : 1;
    const bool empty = B == 0 || H == 0 || W == 0 || d_hi == d_lo;
    if (want_loss) {
        QC_RETURN_IF(acc == nullptr, QC_ERR_INVALID_ARGUMENT, "tv: null acc");
        QC_RETURN_IF(ws == nullptr || ws_bytes < workspace_bytes(), QC_ERR_WORKSPACE_TOO_SMALL,
                     "tv: workspace of %zu bytes is below the %zu required", ws_bytes,
                     workspace_bytes());
    }
    if (want_grad) {
        QC_RETURN_IF(grad == nullptr, QC_ERR_INVALID_ARGUMENT, "tv: null grad");
        QC_RETURN_IF(g == nullptr, QC_ERR_INVALID_ARGUMENT, "tv: null upstream gradient");
    }
    QC_RETURN_IF(!empty && vol == nullptr, QC_ERR_INVALID_ARGUMENT, "tv: null volume");

    if (empty) {
        if (want_loss && (flags & QC_TV_ACC_OVERWRITE))
            QC_CUDA_TRY(cudaMemsetAsync(acc, 0, n_acc * sizeof(float), stream), "cudaMemsetAsync(acc)");
        return 0;
    }

    Plan pl{};
    pl.B = B;
    pl.Dp = Dp;
    pl.H = H;
    pl.W = W;
    pl.d_lo = d_lo;
    pl.d_hi = d_hi;
    pl.has_prev = has_prev ? 1 : 0;
    pl.has_next = has_next ? 1 : 0;
    pl.eps = eps;
    pl.scale = acc_scale;

    const bool aligned = (reinterpret_cast<uintptr_t>(vol) % 16 == 0) &&
                         (!want_grad || reinterpret_cast<uintptr_t>(grad) % 16 == 0);
    const bool use_tma = (W % 4 == 0) && aligned && ((long long)B * Dp < (1LL << 31));

    double *partials = reinterpret_cast<double *>(ws);
    int grid = 0;
    int st = 0;
    switch (variant) {
        case QC_TV_SQ: st = dispatch_mode<QC_TV_SQ>(flags, use_tma, vol, g, grad, partials, pl, &grid, stream); break;
        case QC_TV_ISO: st = dispatch_mode<QC_TV_ISO>(flags, use_tma, vol, g, grad, partials, pl, &grid, stream); break;
        default: st = dispatch_mode<QC_TV_L1>(flags, use_tma, vol, g, grad, partials, pl, &grid, stream); break;
    }
    if (st) return st;

    if (want_loss) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(1);
        cfg.blockDim = dim3(kFinThreads);
        cfg.dynamicSmemBytes = 0;
        cfg.stream = stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        QC_CUDA_TRY(cudaLaunchKernelEx(&cfg, tv_finalize_kernel, (const double *)partials, grid, n_acc,
                                       acc, acc_scale, (flags & QC_TV_ACC_OVERWRITE) ? 1 : 0),
                    "tv_finalize_kernel launch");
    }
    return 0;
}

}  // namespace tv
}  // namespace qc

// ── C ABI ─────────────────────────────────────────────────────────────────

extern "C" {

size_t tv_loss_3d_workspace_bytes(int, int, int, int) { return qc::tv::workspace_bytes(); }

int tv_loss_3d_slab_cuda(int variant, int flags, const float *d_vol, const float *d_g, float *d_acc,
                         float *d_grad_vol, int B, int Dp, int H, int W, int d_lo, int d_hi,
                         int has_prev, int has_next, float eps, float acc_scale, void *d_workspace,
                         size_t workspace_bytes, cudaStream_t stream) {
    return qc::tv::run(variant, flags, d_vol, d_g, d_acc, d_grad_vol, B, Dp, H, W, d_lo, d_hi,
                       has_prev, has_next, eps, acc_scale, d_workspace, workspace_bytes, stream);
}

int tv_loss_iso_3d_cuda(const float *d_vol, float *d_acc, int B, int D, int H, int W, float eps,
                        void *d_workspace, size_t workspace_bytes, cudaStream_t stream) {
    return qc::tv::run(QC_TV_ISO, QC_TV_LOSS, d_vol, nullptr, d_acc, nullptr, B, D, H, W, 0, D, 0,
                       0, eps, 1.0f, d_workspace, workspace_bytes, stream);
}

int tv_loss_iso_3d_grad_cuda(const float *d_vol, const float *d_g_scaled, float *d_grad_vol,
                             int B, int D, int H, int W, float eps, cudaStream_t stream) {
    return qc::tv::run(QC_TV_ISO, QC_TV_GRAD, d_vol, d_g_scaled, nullptr, d_grad_vol, B, D, H, W,
                       0, D, 0, 0, eps, 1.0f, nullptr, 0, stream);
}

int tv_loss_sq_3d_cuda(const float *d_vol, float *d_acc, int B, int D, int H, int W,
                       void *d_workspace, size_t workspace_bytes, cudaStream_t stream) {
    return qc::tv::run(QC_TV_SQ, QC_TV_LOSS, d_vol, nullptr, d_acc, nullptr, B, D, H, W, 0, D, 0,
                       0, 0.f, 1.0f, d_workspace, workspace_bytes, stream);
}

int tv_loss_sq_3d_grad_cuda(const float *d_vol, const float *d_g, float *d_grad_vol, int B, int D,
                            int H, int W, cudaStream_t stream) {
    return qc::tv::run(QC_TV_SQ, QC_TV_GRAD, d_vol, d_g, nullptr, d_grad_vol, B, D, H, W, 0, D, 0,
                       0, 0.f, 1.0f, nullptr, 0, stream);
}

int tv_loss_l1_3d_cuda(const float *d_vol, float *d_acc, int B, int D, int H, int W,
                       void *d_workspace, size_t workspace_bytes, cudaStream_t stream) {
    return qc::tv::run(QC_TV_L1, QC_TV_LOSS, d_vol, nullptr, d_acc, nullptr, B, D, H, W, 0, D, 0,
                       0, 0.f, 1.0f, d_workspace, workspace_bytes, stream);
}

int tv_loss_l1_3d_grad_cuda(const float *d_vol, const float *d_g, float *d_grad_vol, int B, int D,
                            int H, int W, cudaStream_t stream) {
    return qc::tv::run(QC_TV_L1, QC_TV_GRAD, d_vol, d_g, nullptr, d_grad_vol, B, D, H, W, 0, D, 0,
                       0, 0.f, 1.0f, nullptr, 0, stream);
}

int tv_loss_iso_3d_fwd_grad_cuda(const float *d_vol, const float *d_g_scaled, float *d_acc,
                                 float *d_grad_vol, int B, int D, int H, int W, float eps,
                                 void *d_workspace, size_t workspace_bytes, cudaStream_t stream) {
    return qc::tv::run(QC_TV_ISO, QC_TV_LOSS | QC_TV_GRAD, d_vol, d_g_scaled, d_acc, d_grad_vol, B,
                       D, H, W, 0, D, 0, 0, eps, 1.0f, d_workspace, workspace_bytes, stream);
}

int tv_loss_sq_3d_fwd_grad_cuda(const float *d_vol, const float *d_g, float *d_acc,
                                float *d_grad_vol, int B, int D, int H, int W, void *d_workspace,
                                size_t workspace_bytes, cudaStream_t stream) {
    return qc::tv::run(QC_TV_SQ, QC_TV_LOSS | QC_TV_GRAD, d_vol, d_g, d_acc, d_grad_vol, B, D, H,
                       W, 0, D, 0, 0, 0.f, 1.0f, d_workspace, workspace_bytes, stream);
}

int tv_loss_l1_3d_fwd_grad_cuda(const float *d_vol, const float *d_g, float *d_acc,
                                float *d_grad_vol, int B, int D, int H, int W, void *d_workspace,
                                size_t workspace_bytes, cudaStream_t stream) {
    return qc::tv::run(QC_TV_L1, QC_TV_LOSS | QC_TV_GRAD, d_vol, d_g, d_acc, d_grad_vol, B, D, H,
                       W, 0, D, 0, 0, 0.f, 1.0f, d_workspace, workspace_bytes, stream);
}

int quantem_cuda_device_fault_word(int device, unsigned int *word, int clear) {
    int prev = 0;
    QC_CUDA_TRY(cudaGetDevice(&prev), "cudaGetDevice");
    QC_CUDA_TRY(cudaSetDevice(device), "cudaSetDevice");
    unsigned int w = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&w, qc::tv::g_tv_fault_word, sizeof(w));
    if (e == cudaSuccess && clear) {
        const unsigned int zero = 0;
        e = cudaMemcpyToSymbol(qc::tv::g_tv_fault_word, &zero, sizeof(zero));
    }
    cudaSetDevice(prev);
    QC_CUDA_TRY(e, "cudaMemcpyFromSymbol(fault word)");
    if (word) *word = w;
    return 0;
}

}  // extern "C"
