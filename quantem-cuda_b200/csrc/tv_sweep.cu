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
// letting one sweep produce loss and gradient together, each difference being
// evaluated once and used by both voxels it touches.
//
// Fast path (W % 4 == 0, 16-byte aligned pointers). A CTA marches along D
// through a column of (R·NW) × 128 (H × W) tiles. One producer warp streams
// each plane tile with a one-voxel halo — (R·NW + 2) rows × 136 columns; the
// left halo is 4 columns wide because a TMA box must start on a 16-byte
// boundary — into an S-stage shared-memory ring with cp.async.bulk.tensor
// (no multicast). NW consumer warps each own R consecutive rows × 128 columns
// (4 columns per lane, moved as float4). Per plane a consumer thread:
//   * keeps Fd of the previous plane in registers (R × 4 values),
//   * carries Fh from row to row down its strip, computing Fh of the row
//     above the strip once (1 extra row per R),
//   * takes Fw of the column to its left from the neighbouring lane by
//     shuffle; the tile's left halo column is computed once per plane with
//     the warp's lanes standing for rows, then broadcast to lane 0.
// Square roots use the MUFU approximations (sqrt/rsqrt.approx, relative error
// ~2^-23), which keeps the kernel free of the IEEE slow path's branches.
//
// Each voxel is read from HBM once per sweep: halo rows and columns are shared
// with neighbouring tiles, which the chunk-major schedule runs at the same
// time, so they hit L2.
//
// Reductions are deterministic: each CTA writes fp64 partial sums to a
// caller-owned workspace slot, and a one-CTA finalize kernel, launched with
// programmatic dependent launch, sums the slots in fixed order.
#include <stdio.h>

#include <atomic>
#include <mutex>
#include <type_traits>

#include "qc_common.cuh"

namespace qc {
namespace tv {

// Set by a wait that gave up instead of hanging: QC_FAULT_TMA_WAIT by the
// TMA ring, QC_FAULT_PEER_WAIT by a wait for another rank.
__device__ unsigned int g_tv_fault_word = 0;

constexpr uint64_t kWaitLimitNs = 2000000000ull;       // 2 s per barrier wait
constexpr uint64_t kPeerWaitLimitNs = 10000000000ull;  // default bound of a wait for another rank

constexpr int kMaxPartials = 2048;  // CTA partial-sum slots in the workspace
constexpr int kMaxDevices = 64;     // per-device host-side caches
constexpr int kAccSlots = 3;        // L1 keeps one sum per axis

// Several terms of one volume in one sweep ("mixed" variants, V = kMix |
// mask): mask bit 0 the squared term, bit 1 the isotropic term, bit 2 the L1
// term. The gradient is linear in the terms' fluxes, so one divergence of the
// gain-weighted sum of fluxes gives the summed gradient; the loss slots are
// [Σ sq, Σ iso, Σ|Δd|, Σ|Δh|, Σ|Δw|].
constexpr int kMix = 8;
constexpr int kMixSlots = 5;
constexpr int kMaxSlots = kMixSlots;
__host__ __device__ constexpr bool is_mix(int V) { return V >= kMix; }
__host__ __device__ constexpr bool has_sq(int V) { return V == QC_TV_SQ || (V >= kMix && (V & 1)); }
__host__ __device__ constexpr bool has_iso(int V) { return V == QC_TV_ISO || (V >= kMix && (V & 2)); }
__host__ __device__ constexpr bool has_l1(int V) { return V == QC_TV_L1 || (V >= kMix && (V & 4)); }
// loss slots a CTA writes (the workspace stride of its partial sums)
__host__ __device__ constexpr int slots_of(int V) { return V >= kMix ? kMixSlots : kAccSlots; }

// ── per-variant arithmetic ───────────────────────────────────────────────

__device__ __forceinline__ float sqrt_approx(float x) {
    float y;
    asm("sqrt.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ float rsqrt_approx(float x) {
    float y;
    asm("rsqrt.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// dd² + dh² + dw² + eps with one fixed FMA chain, used by every path (scalar,
// paired, halo) so that a corner evaluates to the same bits wherever it is
// computed.
__device__ __forceinline__ float iso_x(float dd, float dh, float dw, float eps) {
    return __fmaf_rn(dw, dw, __fmaf_rn(dh, dh, __fmaf_rn(dd, dd, eps)));
}

// g·sign(x) with sign(0) = 0: torch's convention for d|x|/dx (tv_loss.cu:434-436).
__device__ __forceinline__ float gsign(float g, float x) {
    return x > 0.f ? g : (x < 0.f ? -g : 0.f);
}

struct Gains {
    float gmul;        // multiplies the divergence
    float gd, gh, gw;  // L1 per-axis gains folded into F
    float gsq2, giso;  // mixed variants: 2·g of the squared term, g of the isotropic term
};

// Loss terms and flux at a voxel with value v and +1 neighbours (nd, nh, nw);
// vd/vh/vw say whether each neighbour exists. `own` gates the loss.
template <int V, bool LOSS, bool GRAD>
__device__ __forceinline__ void voxel_flux(float v, float nd, float nh, float nw, bool vd, bool vh,
                                           bool vw, bool own, float eps, const Gains &gn,
                                           float &Fd, float &Fh, float &Fw, float *l) {
    float &l0 = l[0], &l1 = l[1], &l2 = l[2];
    const float dd = vd ? nd - v : 0.f;
    const float dh = vh ? nh - v : 0.f;
    const float dw = vw ? nw - v : 0.f;
    if constexpr (is_mix(V)) {
        float fd = 0.f, fh = 0.f, fw = 0.f;
        if constexpr (has_sq(V)) {
            if (LOSS && own) l[0] += __fmaf_rn(dw, dw, __fmaf_rn(dh, dh, dd * dd));
            if (GRAD) {
                fd = gn.gsq2 * dd;
                fh = gn.gsq2 * dh;
                fw = gn.gsq2 * dw;
            }
        }
        if constexpr (has_iso(V)) {
            const bool ok = vd && vh && vw;
            const float x = iso_x(dd, dh, dw, eps);
            if (LOSS) l[1] += (ok && own) ? sqrt_approx(x) : 0.f;
            if (GRAD) {
                const float inv = ok ? gn.giso * rsqrt_approx(x) : 0.f;
                fd = __fmaf_rn(dd, inv, fd);
                fh = __fmaf_rn(dh, inv, fh);
                fw = __fmaf_rn(dw, inv, fw);
            }
        }
        if constexpr (has_l1(V)) {
            if (LOSS && own) {
                l[2] += fabsf(dd);
                l[3] += fabsf(dh);
                l[4] += fabsf(dw);
            }
            if (GRAD) {
                fd += gsign(gn.gd, dd);
                fh += gsign(gn.gh, dh);
                fw += gsign(gn.gw, dw);
            }
        }
        if (GRAD) {
            Fd = fd;
            Fh = fh;
            Fw = fw;
        }
    } else if constexpr (V == QC_TV_SQ) {
        if (LOSS) {
            const float s = __fmaf_rn(dw, dw, __fmaf_rn(dh, dh, dd * dd));
            l0 += own ? s : 0.f;
        }
        if (GRAD) {
            Fd = dd;
            Fh = dh;
            Fw = dw;
        }
    } else if constexpr (V == QC_TV_L1) {
        if (LOSS && own) {
            l0 += fabsf(dd);
            l1 += fabsf(dh);
            l2 += fabsf(dw);
        }
        if (GRAD) {
            Fd = gsign(gn.gd, dd);
            Fh = gsign(gn.gh, dh);
            Fw = gsign(gn.gw, dw);
        }
    } else {  // QC_TV_ISO
        const bool ok = vd && vh && vw;
        const float x = iso_x(dd, dh, dw, eps);
        if (LOSS) l0 += (ok && own) ? sqrt_approx(x) : 0.f;
        if (GRAD) {
            const float inv = ok ? rsqrt_approx(x) : 0.f;
            Fd = dd * inv;
            Fh = dh * inv;
            Fw = dw * inv;
        }
    }
}

// Fh of the voxel one row up (h-1): `up` = v[h-1]; for iso the corner at
// (h-1) also needs v[d+1][h-1] (`up_nd`) and v[h-1][w+1] (`up_nw`).
template <int V>
__device__ __forceinline__ float flux_from_up(float v, float up, float up_nd, float up_nw,
                                              bool has_up, bool vd, bool vw_up, float eps,
                                              const Gains &gn) {
    const float dh = has_up ? v - up : 0.f;
    if constexpr (is_mix(V)) {
        float f = 0.f;
        if constexpr (has_sq(V)) f = gn.gsq2 * dh;
        if constexpr (has_iso(V)) {
            const bool ok = has_up && vd && vw_up;
            const float dd = up_nd - up, dw = up_nw - up;
            const float inv = ok ? gn.giso * rsqrt_approx(iso_x(dd, dh, dw, eps)) : 0.f;
            f = __fmaf_rn(dh, inv, f);
        }
        if constexpr (has_l1(V)) f += gsign(gn.gh, dh);
        return f;
    } else if constexpr (V == QC_TV_SQ) {
        return dh;
    } else if constexpr (V == QC_TV_L1) {
        return gsign(gn.gh, dh);
    } else {
        const bool ok = has_up && vd && vw_up;
        const float dd = up_nd - up, dw = up_nw - up;
        const float inv = ok ? rsqrt_approx(iso_x(dd, dh, dw, eps)) : 0.f;
        return dh * inv;
    }
}

// Fw of the voxel one column left (w-1): `lf` = v[w-1]; for iso the corner at
// (w-1) also needs v[d+1][w-1] (`lf_nd`) and v[h+1][w-1] (`lf_nh`).
template <int V>
__device__ __forceinline__ float flux_from_left(float v, float lf, float lf_nd, float lf_nh,
                                                bool has_left, bool vd, bool vh, float eps,
                                                const Gains &gn) {
    const float dw = has_left ? v - lf : 0.f;
    if constexpr (is_mix(V)) {
        float f = 0.f;
        if constexpr (has_sq(V)) f = gn.gsq2 * dw;
        if constexpr (has_iso(V)) {
            const bool ok = has_left && vd && vh;
            const float dd = lf_nd - lf, dh = lf_nh - lf;
            const float inv = ok ? gn.giso * rsqrt_approx(iso_x(dd, dh, dw, eps)) : 0.f;
            f = __fmaf_rn(dw, inv, f);
        }
        if constexpr (has_l1(V)) f += gsign(gn.gw, dw);
        return f;
    } else if constexpr (V == QC_TV_SQ) {
        return dw;
    } else if constexpr (V == QC_TV_L1) {
        return gsign(gn.gw, dw);
    } else {
        const bool ok = has_left && vd && vh;
        const float dd = lf_nd - lf, dh = lf_nh - lf;
        const float inv = ok ? rsqrt_approx(iso_x(dd, dh, dw, eps)) : 0.f;
        return dw * inv;
    }
}

template <int V>
__device__ __forceinline__ Gains load_gains(const float *g, float scale) {
    Gains gn{1.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (g == nullptr) return gn;
    if constexpr (is_mix(V)) {
        // g = [g_sq, g_iso, g_d, g_h, g_w], the upstream gradients of the
        // reported losses; `scale` is the isotropic loss's own factor (1/N
        // for the mean), so only g_iso takes it. The divergence gain stays 1.
        gn.gsq2 = 2.0f * __ldg(g);
        gn.giso = __ldg(g + 1) * scale;
        gn.gd = __ldg(g + 2);
        gn.gh = __ldg(g + 3);
        gn.gw = __ldg(g + 4);
    } else if constexpr (V == QC_TV_SQ) {
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
    float *acc_atomic;       // non-null: each CTA adds scale·(its sums) here with fp32
                             // atomics instead of writing a workspace partial
};

// A CTA's sum of loss slot `slot` (threadIdx.x < slots_of(V)): into the
// workspace for the fixed-order finalize, or (reference-signature entries,
// which have no workspace) added to the caller's accumulator atomically, as
// the reference's loss kernels do (tv_loss.cu:95, :273, :404-408).
template <int V>
__device__ __forceinline__ void store_cta_sum(const Plan &pl, double *partials, int slot, double t) {
    if (pl.acc_atomic != nullptr) {
        if (slot < (V == QC_TV_L1 ? 3 : 1)) atomicAdd(pl.acc_atomic + slot, (float)(t * (double)pl.scale));
    } else {
        partials[(size_t)blockIdx.x * slots_of(V) + slot] = t;
    }
}

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

// ── cross-rank flags over peer memory ─────────────────────────────────────
//
// One communication block per rank, in memory its peers have mapped. Flags
// hold the sequence number of the last call that set them; a waiter compares
// with >= so a flag that has moved on to a later call still releases it.
// Data goes into a peer's block with plain stores, then (one thread per CTA,
// after a CTA barrier) one system-scope fence and the flags as relaxed stores;
// the waiter loads a flag with acquire semantics.

struct PeerComm {
    unsigned long long ready[2];   // [s]: neighbour on side s (0 = rank-1, 1 = rank+1) lets
                                   // this rank store into that neighbour's halo for the call
    unsigned long long filled[2];  // [s]: neighbour on side s has filled this rank's halo s
    unsigned int arrive;           // CTAs of this rank's exchange launch done storing
    unsigned int pad0[7];
    unsigned long long red_flag[QC_MAX_PEER_RANKS];   // [q]: rank q's totals are in the slot
    double partials[2][QC_MAX_PEER_RANKS][QC_TV_MAX_PEER_SUMS];  // [call & 1][q][sum]
};

// Flag stores. A group of flags that publishes earlier stores is written as
// one system-scope fence followed by relaxed stores, so that raising k flags
// costs one fence (st.release would fence again before every flag).
__device__ __forceinline__ void st_relaxed_sys(unsigned long long *p, unsigned long long v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ double ld_relaxed_sys_f64(const double *p) {
    double v;
    asm volatile("ld.relaxed.sys.global.f64 %0, [%1];" : "=d"(v) : "l"(p) : "memory");
    return v;
}

// Waits until *flag >= seq, for at most limit_ns. Returns false if it gave up.
__device__ __forceinline__ bool wait_flag_geq(const unsigned long long *flag, unsigned long long seq,
                                              uint64_t limit_ns) {
    if (ld_acquire_sys(flag) >= seq) return true;
    const uint64_t t0 = global_timer_ns();
    while (true) {
        __nanosleep(64);
        if (ld_acquire_sys(flag) >= seq) return true;
        if (global_timer_ns() - t0 > limit_ns) return false;
    }
}

__device__ __forceinline__ uint64_t peer_limit(const qc_tv_peers &p) {
    return p.timeout_ns ? p.timeout_ns : kPeerWaitLimitNs;
}

// Halo exchange done by the sweep kernel itself (D-slabs over peer memory):
// every CTA stores its share of this rank's two boundary planes into the
// neighbours' halo planes at the start of the kernel, and the producer of a
// unit that reads a halo plane waits for the neighbour's `filled` flag just
// before issuing that plane's copy. seq == 0 disables it.
struct HaloXchg {
    PeerComm *self, *prev, *next;  // communication blocks (prev / next null at the ends)
    float *prev_slab, *next_slab;  // the neighbours' slabs, mapped here
    const float *vol;              // this rank's slab (the planes to send)
    int prev_dp, next_dp;
    unsigned long long seq;
    uint64_t limit_ns;
};

// The exchange's first half, run by every thread of every CTA of the sweep:
// tell the neighbours this rank's halos may be overwritten (all earlier work
// on the stream has completed), wait until they say the same, store this
// CTA's share of the boundary planes into their halos, and let the last CTA
// raise their `filled` flags. `go` is a shared-memory int of the caller.
__device__ __forceinline__ void halo_push_prologue(const HaloXchg &xc, int B, int Dp,
                                                   long long plane, int *go) {
    if (threadIdx.x == 0) {
        // nothing of this grid precedes these flags: the work they announce
        // (earlier kernels on the stream) completed before the grid started
        if (xc.prev) st_relaxed_sys(&xc.prev->ready[1], xc.seq);
        if (xc.next) st_relaxed_sys(&xc.next->ready[0], xc.seq);
        bool ok = true;
        if (xc.prev) ok = wait_flag_geq(&xc.self->ready[0], xc.seq, xc.limit_ns) && ok;
        if (xc.next) ok = wait_flag_geq(&xc.self->ready[1], xc.seq, xc.limit_ns) && ok;
        if (!ok) atomicOr(&g_tv_fault_word, QC_FAULT_PEER_WAIT);
        *go = ok ? 1 : 0;
    }
    __syncthreads();
    if (*go) {
        // float4 items: side (to rank-1, to rank+1) × batch slice × plane / 4
        const long long per = plane / 4, per_side = (long long)B * per;
        const long long stride = (long long)gridDim.x * blockDim.x;
        for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < 2 * per_side;
             i += stride) {
            const int side = i >= per_side;
            if (side == 0 ? xc.prev == nullptr : xc.next == nullptr) continue;
            const long long j = i - side * per_side;
            const long long b = j / per, e = j - b * per;
            const long long src = (long long)b * Dp + (side == 0 ? 1 : Dp - 2);
            const long long dst = side == 0 ? (long long)b * xc.prev_dp + xc.prev_dp - 1
                                            : (long long)b * xc.next_dp;
            float *d = side == 0 ? xc.prev_slab : xc.next_slab;
#ifdef QC_DEBUG_BOUNDS
            const int ddp = side == 0 ? xc.prev_dp : xc.next_dp;
            if (!QC_IN_BOUNDS(src * plane + e * 4 + 3, (long long)B * Dp * plane, g_tv_fault_word) ||
                !QC_IN_BOUNDS(dst * plane + e * 4 + 3, (long long)B * ddp * plane, g_tv_fault_word))
                continue;
#endif
            *reinterpret_cast<float4 *>(d + dst * plane + e * 4) = ldg4(xc.vol + src * plane + e * 4);
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        if (atomicAdd(&xc.self->arrive, 1u) == gridDim.x - 1) {
            xc.self->arrive = 0;  // the next exchange on this stream starts after this grid
            __threadfence_system();
            if (xc.prev) st_relaxed_sys(&xc.prev->filled[1], xc.seq);
            if (xc.next) st_relaxed_sys(&xc.next->filled[0], xc.seq);
        }
    }
}

// ── fast path: TMA ring + warp-specialised D-march ───────────────────────

constexpr int kTileW = 128;                 // owned columns per tile
constexpr int kHaloW = 4;                   // halo columns each side
constexpr int kBoxW = kTileW + 2 * kHaloW;  // 136

template <int R_, int NW_, int S_, int MINB_>
struct Geom {
    static constexpr int R = R_;        // rows per consumer warp
    static constexpr int NW = NW_;      // consumer warps
    static constexpr int S = S_;        // ring stages
    static constexpr int MinB = MINB_;  // CTAs per SM the register budget is sized for
    static constexpr int TileH = R * NW;
    static constexpr int BoxH = TileH + 2;
    static constexpr uint32_t BoxBytes = kBoxW * BoxH * 4;
    static constexpr int StageFloats = (int)(((BoxBytes + 127) / 128) * 32);  // 128-B aligned
    static constexpr int Threads = (NW + 1) * 32;
};

template <class G>
struct SweepSmem {
    float stage[G::S][G::StageFloats];
    uint64_t full[G::S];
    uint64_t empty[G::S];
    double red[G::NW][kMaxSlots];
    int abort;
    int xgo;
};

template <class G>
__device__ __forceinline__ bool aborted(const SweepSmem<G> &sm) {
    return *reinterpret_cast<const volatile int *>(&sm.abort) != 0;
}

__device__ __forceinline__ float4 lds4(const float *s, int row, int col) {
    return *reinterpret_cast<const float4 *>(s + row * kBoxW + col);
}
__device__ __forceinline__ float lds1(const float *s, int row, int col) {
    return s[row * kBoxW + col];
}
__device__ __forceinline__ float comp(const float4 &v, int j) {
    return j == 0 ? v.x : (j == 1 ? v.y : (j == 2 ? v.z : v.w));
}

// g·sign(d) with sign(0) = 0, as a sign transfer: g with its sign bit flipped
// where d < 0 (one logic op) and a zero test.
__device__ __forceinline__ float gsign_fast(float g, float d) {
    const float f = __int_as_float((__float_as_int(d) & 0x80000000) ^ __float_as_int(g));
    return d != 0.f ? f : 0.f;
}

// ── packed fp32 pairs ─────────────────────────────────────────────────────
// sm_100 executes two fp32 adds/multiplies/FMAs per instruction on a 64-bit
// register pair (add/sub/mul/fma.rn.f32x2). A lane's 4 voxels arrive from
// shared memory as two such pairs, (v0, v1) and (v2, v3); arithmetic that is
// the same for all four runs on the pairs, and only the views shifted by one
// column need packing moves.
typedef unsigned long long f2;

__device__ __forceinline__ f2 pk2(float lo, float hi) {
    f2 r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ float lo2(f2 v) {
    float a, b;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
    return a;
}
__device__ __forceinline__ float hi2(f2 v) {
    float a, b;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
    return b;
}
__device__ __forceinline__ f2 add2(f2 a, f2 b) {
    f2 r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ f2 sub2(f2 a, f2 b) {
    f2 r;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ f2 mul2(f2 a, f2 b) {
    f2 r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ f2 fma2(f2 a, f2 b, f2 c) {
    f2 r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}
__device__ __forceinline__ ulonglong2 lds_pairs(const float *s, int row, int col) {
    return *reinterpret_cast<const ulonglong2 *>(s + row * kBoxW + col);
}
// Gradient stores bypass L1 (no line allocated): 5% faster L1 sweeps than
// evict-first (.cs) or default stores on B200, iso and sq unchanged.
__device__ __forceinline__ void st_grad_pairs(float *p, f2 a, f2 b) {
    asm volatile("st.global.L1::no_allocate.v2.b64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b) : "memory");
}

// Loss terms and fluxes of one row of a lane's 4 voxels as pairs (c01, c23),
// with edge-replicated neighbours as in row_flux4 below. The loss
// accumulators are pairs (a01, a23) for SQ/iso, scalars for L1.
template <int V, bool LOSS, bool GRAD>
__device__ __forceinline__ void row_flux_pairs(const ulonglong2 &c, const ulonglong2 &n,
                                               const ulonglong2 &dn, float right, f2 eps01,
                                               f2 eps23, bool s3_ok, const Gains &gn,
                                               ulonglong2 &Fd, ulonglong2 &Fh, ulonglong2 &Fw,
                                               f2 &acc01, f2 &acc23, f2 &bcc01, f2 &bcc23,
                                               float &r0, float &r1, float &r2) {
    const f2 dd01 = sub2(n.x, c.x), dd23 = sub2(n.y, c.y);
    const f2 dh01 = sub2(dn.x, c.x), dh23 = sub2(dn.y, c.y);
    const f2 w01 = pk2(hi2(c.x), lo2(c.y)), w23 = pk2(hi2(c.y), right);
    const f2 dw01 = sub2(w01, c.x), dw23 = sub2(w23, c.y);
    if constexpr (is_mix(V)) {
        // squared loss pairs in acc, isotropic loss pairs in bcc, L1 sums in
        // r0..r2; the flux is the gain-weighted sum of the terms' fluxes
        f2 fd01 = 0ull, fd23 = 0ull, fh01 = 0ull, fh23 = 0ull, fw01 = 0ull, fw23 = 0ull;
        if constexpr (has_sq(V)) {
            if (LOSS) {
                acc01 = fma2(dd01, dd01, acc01);
                acc01 = fma2(dh01, dh01, acc01);
                acc01 = fma2(dw01, dw01, acc01);
                acc23 = fma2(dd23, dd23, acc23);
                acc23 = fma2(dh23, dh23, acc23);
                acc23 = fma2(dw23, dw23, acc23);
            }
            if (GRAD) {
                const f2 g2 = pk2(gn.gsq2, gn.gsq2);
                fd01 = mul2(dd01, g2);
                fd23 = mul2(dd23, g2);
                fh01 = mul2(dh01, g2);
                fh23 = mul2(dh23, g2);
                fw01 = mul2(dw01, g2);
                fw23 = mul2(dw23, g2);
            }
        }
        if constexpr (has_iso(V)) {
            const f2 x01 = fma2(dw01, dw01, fma2(dh01, dh01, fma2(dd01, dd01, eps01)));
            const f2 x23 = fma2(dw23, dw23, fma2(dh23, dh23, fma2(dd23, dd23, eps23)));
            const f2 r01 = pk2(rsqrt_approx(lo2(x01)), rsqrt_approx(hi2(x01)));
            const f2 r23 = pk2(rsqrt_approx(lo2(x23)), rsqrt_approx(hi2(x23)));
            if (LOSS) {
                const f2 s01 = mul2(x01, r01), s23 = mul2(x23, r23);
                bcc01 = add2(bcc01, s01);
                bcc23 = add2(bcc23, s3_ok ? s23 : pk2(lo2(s23), 0.f));
            }
            if (GRAD) {
                const f2 gi = pk2(gn.giso, gn.giso);
                const f2 q01 = mul2(r01, gi), q23 = mul2(r23, gi);
                fd01 = fma2(dd01, q01, fd01);
                fd23 = fma2(dd23, q23, fd23);
                fh01 = fma2(dh01, q01, fh01);
                fh23 = fma2(dh23, q23, fh23);
                fw01 = fma2(dw01, q01, fw01);
                fw23 = fma2(dw23, q23, fw23);
            }
        }
        if constexpr (has_l1(V)) {
            const float dd[4] = {lo2(dd01), hi2(dd01), lo2(dd23), hi2(dd23)};
            const float dh[4] = {lo2(dh01), hi2(dh01), lo2(dh23), hi2(dh23)};
            const float dw[4] = {lo2(dw01), hi2(dw01), lo2(dw23), hi2(dw23)};
            if (LOSS) {
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    r0 += fabsf(dd[j]);
                    r1 += fabsf(dh[j]);
                    r2 += fabsf(dw[j]);
                }
            }
            if (GRAD) {
                fd01 = add2(fd01, pk2(gsign_fast(gn.gd, dd[0]), gsign_fast(gn.gd, dd[1])));
                fd23 = add2(fd23, pk2(gsign_fast(gn.gd, dd[2]), gsign_fast(gn.gd, dd[3])));
                fh01 = add2(fh01, pk2(gsign_fast(gn.gh, dh[0]), gsign_fast(gn.gh, dh[1])));
                fh23 = add2(fh23, pk2(gsign_fast(gn.gh, dh[2]), gsign_fast(gn.gh, dh[3])));
                fw01 = add2(fw01, pk2(gsign_fast(gn.gw, dw[0]), gsign_fast(gn.gw, dw[1])));
                fw23 = add2(fw23, pk2(gsign_fast(gn.gw, dw[2]), gsign_fast(gn.gw, dw[3])));
            }
        }
        if (GRAD) {
            Fd = make_ulonglong2(fd01, fd23);
            Fh = make_ulonglong2(fh01, fh23);
            Fw = make_ulonglong2(fw01, fw23);
        }
    } else if constexpr (V == QC_TV_SQ) {
        if (LOSS) {
            acc01 = fma2(dd01, dd01, acc01);
            acc01 = fma2(dh01, dh01, acc01);
            acc01 = fma2(dw01, dw01, acc01);
            acc23 = fma2(dd23, dd23, acc23);
            acc23 = fma2(dh23, dh23, acc23);
            acc23 = fma2(dw23, dw23, acc23);
        }
        if (GRAD) {
            Fd = make_ulonglong2(dd01, dd23);
            Fh = make_ulonglong2(dh01, dh23);
            Fw = make_ulonglong2(dw01, dw23);
        }
    } else if constexpr (V == QC_TV_L1) {
        const float dd[4] = {lo2(dd01), hi2(dd01), lo2(dd23), hi2(dd23)};
        const float dh[4] = {lo2(dh01), hi2(dh01), lo2(dh23), hi2(dh23)};
        const float dw[4] = {lo2(dw01), hi2(dw01), lo2(dw23), hi2(dw23)};
        if (LOSS) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                r0 += fabsf(dd[j]);
                r1 += fabsf(dh[j]);
                r2 += fabsf(dw[j]);
            }
        }
        if (GRAD) {
            Fd = make_ulonglong2(pk2(gsign_fast(gn.gd, dd[0]), gsign_fast(gn.gd, dd[1])),
                                 pk2(gsign_fast(gn.gd, dd[2]), gsign_fast(gn.gd, dd[3])));
            Fh = make_ulonglong2(pk2(gsign_fast(gn.gh, dh[0]), gsign_fast(gn.gh, dh[1])),
                                 pk2(gsign_fast(gn.gh, dh[2]), gsign_fast(gn.gh, dh[3])));
            Fw = make_ulonglong2(pk2(gsign_fast(gn.gw, dw[0]), gsign_fast(gn.gw, dw[1])),
                                 pk2(gsign_fast(gn.gw, dw[2]), gsign_fast(gn.gw, dw[3])));
        }
    } else {
        const f2 x01 = fma2(dw01, dw01, fma2(dh01, dh01, fma2(dd01, dd01, eps01)));
        const f2 x23 = fma2(dw23, dw23, fma2(dh23, dh23, fma2(dd23, dd23, eps23)));
        const f2 r01 = pk2(rsqrt_approx(lo2(x01)), rsqrt_approx(hi2(x01)));
        const f2 r23 = pk2(rsqrt_approx(lo2(x23)), rsqrt_approx(hi2(x23)));
        if (LOSS) {
            const f2 s01 = mul2(x01, r01), s23 = mul2(x23, r23);
            acc01 = add2(acc01, s01);
            acc23 = add2(acc23, s3_ok ? s23 : pk2(lo2(s23), 0.f));
        }
        if (GRAD) {
            Fd = make_ulonglong2(mul2(dd01, r01), mul2(dd23, r23));
            Fh = make_ulonglong2(mul2(dh01, r01), mul2(dh23, r23));
            Fw = make_ulonglong2(mul2(dw01, r01), mul2(dw23, r23));
        }
    }
}

// Loss terms and flux of the 4 voxels of one row of a lane (fast path).
// Missing +D/+H/+W neighbours have already been replaced by the voxel itself
// (edge replication) and out-of-volume voxels read as zero, so every invalid
// squared or L1 term is an exact zero difference and needs no mask. For iso a
// corner without all three neighbours carries eps = +inf: rsqrt(+inf) = 0
// zeroes its flux, and its loss (s = x·rsqrt(x), not finite) is dropped by the
// caller's row-level select or, for the 4th voxel, by s3_ok.
template <int V, bool LOSS, bool GRAD>
__device__ __forceinline__ void row_flux4(const float4 &c, const float4 &n, const float4 &dn,
                                          float right, float eps_row, float eps3, bool s3_ok,
                                          const Gains &gn, float Fd[4], float Fh[4], float Fw[4],
                                          float &r0, float &r1, float &r2) {
    const float cv[4] = {c.x, c.y, c.z, c.w};
    const float nv[4] = {n.x, n.y, n.z, n.w};
    const float hv[4] = {dn.x, dn.y, dn.z, dn.w};
    const float wv[4] = {c.y, c.z, c.w, right};
    static_assert(!(is_mix(V) && LOSS), "row_flux4 gives the mixed variants' flux only");
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float dd = nv[j] - cv[j], dh = hv[j] - cv[j], dw = wv[j] - cv[j];
        if constexpr (is_mix(V)) {
            if (GRAD) {
                float fd = 0.f, fh = 0.f, fw = 0.f;
                if constexpr (has_sq(V)) {
                    fd = gn.gsq2 * dd;
                    fh = gn.gsq2 * dh;
                    fw = gn.gsq2 * dw;
                }
                if constexpr (has_iso(V)) {
                    const float r = gn.giso * rsqrt_approx(iso_x(dd, dh, dw, j == 3 ? eps3 : eps_row));
                    fd = __fmaf_rn(dd, r, fd);
                    fh = __fmaf_rn(dh, r, fh);
                    fw = __fmaf_rn(dw, r, fw);
                }
                if constexpr (has_l1(V)) {
                    fd += gsign_fast(gn.gd, dd);
                    fh += gsign_fast(gn.gh, dh);
                    fw += gsign_fast(gn.gw, dw);
                }
                Fd[j] = fd;
                Fh[j] = fh;
                Fw[j] = fw;
            }
        } else if constexpr (V == QC_TV_SQ) {
            if (LOSS) r0 = __fmaf_rn(dw, dw, __fmaf_rn(dh, dh, __fmaf_rn(dd, dd, r0)));
            if (GRAD) {
                Fd[j] = dd;
                Fh[j] = dh;
                Fw[j] = dw;
            }
        } else if constexpr (V == QC_TV_L1) {
            if (LOSS) {
                r0 += fabsf(dd);
                r1 += fabsf(dh);
                r2 += fabsf(dw);
            }
            if (GRAD) {
                Fd[j] = gsign_fast(gn.gd, dd);
                Fh[j] = gsign_fast(gn.gh, dh);
                Fw[j] = gsign_fast(gn.gw, dw);
            }
        } else {
            const float x = iso_x(dd, dh, dw, j == 3 ? eps3 : eps_row);
            const float r = rsqrt_approx(x);
            if (LOSS) {
                const float sv = x * r;
                r0 += (j < 3 || s3_ok) ? sv : 0.f;
            }
            if (GRAD) {
                Fd[j] = dd * r;
                Fh[j] = dh * r;
                Fw[j] = dw * r;
            }
        }
    }
}

template <int V, bool LOSS, bool GRAD, class G>
__global__ void __launch_bounds__(G::Threads, G::MinB) tv_sweep_tma_kernel(
    const __grid_constant__ CUtensorMap map, const float *__restrict__ g,
    float *__restrict__ grad, double *__restrict__ partials, const Plan pl, const HaloXchg xc) {
    constexpr int R = G::R, NW = G::NW, S = G::S;
    // TMA destinations must be 128-byte aligned: align the ring explicitly
    // (the launch requests sizeof(SweepSmem) + 128 bytes).
    extern __shared__ __align__(128) unsigned char smem_raw[];
    SweepSmem<G> &sm = *reinterpret_cast<SweepSmem<G> *>(
        smem_raw + ((128u - (smem_addr(smem_raw) & 127u)) & 127u));
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&sm.full[s], 1);
            mbar_init(&sm.empty[s], NW);
        }
        sm.abort = 0;
        fence_mbar_init();
    }
    __syncthreads();
    // Launched with programmatic stream serialization: the set-up above may
    // run while the previous kernel in the stream is finishing; nothing
    // global is read or written before that kernel has completed.
    griddep_wait();
    if (xc.seq != 0) halo_push_prologue(xc, pl.B, pl.Dp, (long long)pl.H * pl.W, &sm.xgo);

    double acc0 = 0.0, acc1 = 0.0, acc2 = 0.0, acc3 = 0.0, acc4 = 0.0;

    if (warp == NW) {
        // ── producer warp: one lane issues every TMA load ──
        if (lane == 0) {
            prefetch_tensor_map(&map);
            int seq = 0;
            int last_seq[S];
#pragma unroll
            for (int s = 0; s < S; ++s) last_seq[s] = -1;
            for (long long u = blockIdx.x; u < pl.n_units && !aborted(sm); u += gridDim.x) {
                const Unit U = decode_unit<GRAD>(pl, u, G::TileH, kTileW);
                const int zbase = U.n * pl.Dp;
                for (int p = U.first; p <= U.last; ++p, ++seq) {
                    const int s = seq % S;
                    if (xc.seq != 0 && ((p == pl.d_lo - 1 && pl.has_prev) || (p == pl.d_hi && pl.has_next))) {
                        // a halo plane: wait until the neighbour has stored it here
                        if (!wait_flag_geq(&xc.self->filled[p == pl.d_hi ? 1 : 0], xc.seq, xc.limit_ns))
                            atomicOr(&g_tv_fault_word, QC_FAULT_PEER_WAIT);
                        asm volatile("fence.proxy.async.global;" ::: "memory");
                    }
                    if (seq >= S) {
                        const uint32_t par = (uint32_t)(((seq / S) - 1) & 1);
                        if (!mbar_wait_bounded(&sm.empty[s], par, kWaitLimitNs)) {
                            atomicOr(&g_tv_fault_word, QC_FAULT_TMA_WAIT);
                            sm.abort = 1;
                            break;
                        }
                    }
                    mbar_arrive_expect_tx(&sm.full[s], G::BoxBytes);
                    tma_load_3d(sm.stage[s], &map, U.w0 - kHaloW, U.h0 - 1, zbase + p, &sm.full[s]);
#pragma unroll
                    for (int q = 0; q < S; ++q)
                        if (q == s) last_seq[q] = seq;
                }
            }
            // Never leave a bulk copy in flight into shared memory that is about
            // to be released: wait (bounded) for the last load of every stage.
#pragma unroll
            for (int s = 0; s < S; ++s) {
                if (last_seq[s] < 0) continue;
                const uint32_t par = (uint32_t)((last_seq[s] / S) & 1);
                if (!mbar_wait_bounded(&sm.full[s], par, kWaitLimitNs))
                    atomicOr(&g_tv_fault_word, QC_FAULT_TMA_WAIT);
            }
        }
    } else {
        // ── consumer warps ──
        const Gains gn = load_gains<V>(g, pl.scale);
        const int r0 = warp * R;             // first tile row of this warp's strip
        const int scol = kHaloW + 4 * lane;  // smem column of this lane's first voxel
        const size_t plane_elems = (size_t)pl.H * pl.W;
        const float kInf = __int_as_float(0x7f800000);
        f2 Fd_prev[R][2];  // Fd of the previous plane, as pairs
        int seq = 0;

        for (long long u = blockIdx.x; u < pl.n_units; u += gridDim.x) {
            const Unit U = decode_unit<GRAD>(pl, u, G::TileH, kTileW);
            const int wcol = U.w0 + 4 * lane;  // global column of the lane's first voxel
            const int hbase = U.h0 + r0;       // global row of the strip's first row
            // Per-unit lane facts (constant along D). W % 4 == 0, so a lane's 4
            // voxels are all inside or all outside, and only the 4th can lack
            // its +W neighbour.
            const bool lane_in = wcol < pl.W;
            const bool last_quad = wcol + 4 == pl.W;
            const bool has_up = hbase >= 1;
            const float eps_lane = lane_in ? pl.eps : kInf;
            // Lanes stand for rows when computing the left halo column.
            const int hrow = r0 + (lane < R ? lane : R - 1);  // tile row
            const bool hrow_vh = U.h0 + hrow + 1 < pl.H;
            const bool halo_left = U.w0 >= 1;
            float *gbase = grad + (((size_t)U.n * pl.Dp) * pl.H + hbase) * (size_t)pl.W + wcol;

#pragma unroll
            for (int i = 0; i < R; ++i) Fd_prev[i][0] = Fd_prev[i][1] = 0ull;

            const int q0 = seq;
            if (!mbar_wait_bounded(&sm.full[q0 % S], (uint32_t)((q0 / S) & 1), kWaitLimitNs)) {
                atomicOr(&g_tv_fault_word, QC_FAULT_TMA_WAIT);
                sm.abort = 1;
            }
            if (aborted(sm)) break;

            for (int p = U.first; p < U.d_end; ++p) {
                const int qc = q0 + (p - U.first);
                const bool has_nxt = (p + 1) <= U.last;
                const float *Sc = sm.stage[qc % S];
                const float *Sn = Sc;
                if (has_nxt) {
                    const int qn = qc + 1;
                    if (!mbar_wait_bounded(&sm.full[qn % S], (uint32_t)((qn / S) & 1),
                                           kWaitLimitNs)) {
                        atomicOr(&g_tv_fault_word, QC_FAULT_TMA_WAIT);
                        sm.abort = 1;
                    }
                    Sn = sm.stage[qn % S];
                }
                if (aborted(sm)) break;
                const bool owned = p >= U.d_start;
                const float eps_step = has_nxt ? eps_lane : kInf;
                float l0 = 0.f, l1 = 0.f, l2 = 0.f;

                if (!owned) {
                    // Halo plane below the chunk: only Fd is needed, for the
                    // first owned plane's backward difference (plane p+1 exists).
                    if (GRAD) {
                        float4 cur = lds4(Sc, r0 + 1, scol);
#pragma unroll
                        for (int i = 0; i < R; ++i) {
                            const bool row_ok = hbase + i + 1 < pl.H;
                            const float4 down = lds4(Sc, r0 + i + 2, scol);
                            const float4 nxt = lds4(Sn, r0 + i + 1, scol);
                            float right = __shfl_down_sync(0xffffffffu, cur.x, 1);
                            if (lane == 31) right = lds1(Sc, r0 + i + 1, scol + 4);
                            if (last_quad) right = cur.w;
                            const float4 dn = row_ok ? down : cur;
                            const float eps_row = row_ok ? eps_step : kInf;
                            float Fd[4], Fh[4], Fw[4], d0 = 0.f, d1 = 0.f, d2 = 0.f;
                            row_flux4<V, false, true>(cur, nxt, dn, right, eps_row,
                                                      last_quad ? kInf : eps_row, false, gn, Fd,
                                                      Fh, Fw, d0, d1, d2);
                            Fd_prev[i][0] = pk2(Fd[0], Fd[1]);
                            Fd_prev[i][1] = pk2(Fd[2], Fd[3]);
                            cur = down;
                        }
                    }
                } else {
                    // Left halo column (global column w0-1), lanes as rows.
                    float fw_halo = 0.f;
                    if (GRAD) {
                        const float lf = lds1(Sc, hrow + 1, kHaloW - 1);
                        const float v0 = lds1(Sc, hrow + 1, kHaloW);
                        float lf_nd = 0.f, lf_nh = 0.f;
                        if (has_iso(V)) {
                            lf_nd = lds1(Sn, hrow + 1, kHaloW - 1);
                            lf_nh = lds1(Sc, hrow + 2, kHaloW - 1);
                        }
                        fw_halo = flux_from_left<V>(v0, lf, lf_nd, lf_nh, halo_left, has_nxt,
                                                    hrow_vh, pl.eps, gn);
                    }
                    float4 cur = lds4(Sc, r0 + 1, scol);
                    // Row above the strip (tile row r0-1 is smem row r0); at the
                    // top of the volume it is replaced by the strip's first row.
                    float Fh_up[4] = {0.f, 0.f, 0.f, 0.f};
                    if (GRAD) {
                        const float4 up = has_up ? lds4(Sc, r0, scol) : cur;
                        if constexpr (V == QC_TV_ISO || is_mix(V)) {
                            const float4 up_nd = has_nxt ? lds4(Sn, r0, scol) : up;
                            float up_right = __shfl_down_sync(0xffffffffu, up.x, 1);
                            if (lane == 31) up_right = lds1(Sc, r0, scol + 4);
                            if (last_quad) up_right = up.w;
                            const float e_up = has_up ? eps_step : kInf;
                            float Fd_u[4], Fw_u[4], d0 = 0.f, d1 = 0.f, d2 = 0.f;
                            row_flux4<V, false, true>(up, up_nd, cur, up_right, e_up,
                                                      last_quad ? kInf : e_up, false, gn, Fd_u,
                                                      Fh_up, Fw_u, d0, d1, d2);
                        } else if constexpr (V == QC_TV_SQ) {
                            Fh_up[0] = cur.x - up.x;
                            Fh_up[1] = cur.y - up.y;
                            Fh_up[2] = cur.z - up.z;
                            Fh_up[3] = cur.w - up.w;
                        } else {
                            Fh_up[0] = gsign_fast(gn.gh, cur.x - up.x);
                            Fh_up[1] = gsign_fast(gn.gh, cur.y - up.y);
                            Fh_up[2] = gsign_fast(gn.gh, cur.z - up.z);
                            Fh_up[3] = gsign_fast(gn.gh, cur.w - up.w);
                        }
                    }

                    float *gp = gbase + (size_t)p * plane_elems;
                    f2 la01 = 0ull, la23 = 0ull;  // paired loss sums of this plane (+0.0f pairs)
                    f2 lb01 = 0ull, lb23 = 0ull;  // mixed variants: the isotropic term's pairs
                    f2 up01 = pk2(Fh_up[0], Fh_up[1]), up23 = pk2(Fh_up[2], Fh_up[3]);
                    // The strip's rows, specialised on whether every row has its
                    // +H neighbour (all strips but the one holding row H-1): then
                    // no per-row validity selects are needed. Without a next plane
                    // (has_nxt false) Sn is Sc, so `nxt` reads the voxel itself.
                    auto rows = [&](auto full_tag) {
                        constexpr bool FULL = decltype(full_tag)::value;
                        ulonglong2 curp = lds_pairs(Sc, r0 + 1, scol);
                        const f2 e01_full = pk2(eps_step, eps_step);
                        const f2 e23_full = pk2(eps_step, last_quad ? kInf : eps_step);
                        const bool loss_lane = has_nxt && lane_in;
#pragma unroll
                        for (int i = 0; i < R; ++i) {
                            const int h = hbase + i;
                            const bool row_ok = FULL || h + 1 < pl.H;  // row has a +H neighbour
                            const ulonglong2 down = lds_pairs(Sc, r0 + i + 2, scol);
                            const ulonglong2 nxt = lds_pairs(Sn, r0 + i + 1, scol);
                            float right = __shfl_down_sync(0xffffffffu, lo2(curp.x), 1);
                            if (lane == 31) right = lds1(Sc, r0 + i + 1, scol + 4);
                            // iso: the missing +W neighbour of the volume's last column
                            // is irrelevant (its corner carries eps = inf)
                            if (V != QC_TV_ISO && last_quad) right = hi2(curp.y);
                            // iso: a row without +H neighbour carries eps = inf, so the
                            // zero-filled row below can stand in for the replicated one
                            const ulonglong2 dn = (V == QC_TV_ISO || row_ok) ? down : curp;
                            f2 e01 = e01_full, e23 = e23_full;
                            if (!FULL && !row_ok) e01 = e23 = pk2(kInf, kInf);
                            ulonglong2 Fd, Fh, Fw;
                            f2 q01 = 0ull, q23 = 0ull, b01 = 0ull, b23 = 0ull;
                            row_flux_pairs<V, LOSS, GRAD>(curp, nxt, dn, right, e01, e23, !last_quad, gn,
                                                          Fd, Fh, Fw, q01, q23, b01, b23, l0, l1, l2);
                            if (LOSS) {
                                if constexpr (is_mix(V)) {
                                    if constexpr (has_sq(V)) {
                                        la01 = add2(la01, q01);
                                        la23 = add2(la23, q23);
                                    }
                                    if constexpr (has_iso(V)) {
                                        if (loss_lane && row_ok) {
                                            lb01 = add2(lb01, b01);
                                            lb23 = add2(lb23, b23);
                                        }
                                    }
                                } else if constexpr (V == QC_TV_ISO) {
                                    if (loss_lane && row_ok) {
                                        la01 = add2(la01, q01);
                                        la23 = add2(la23, q23);
                                    }
                                } else if constexpr (V == QC_TV_SQ) {
                                    la01 = add2(la01, q01);
                                    la23 = add2(la23, q23);
                                }
                            }
                            if (GRAD) {
                                const float fw_from_lane = __shfl_up_sync(0xffffffffu, hi2(Fw.y), 1);
                                const float fw_from_halo = __shfl_sync(0xffffffffu, fw_halo, i);
                                const float Fw_left0 = lane == 0 ? fw_from_halo : fw_from_lane;
                                const f2 wl01 = pk2(Fw_left0, lo2(Fw.x));
                                const f2 wl23 = pk2(hi2(Fw.x), lo2(Fw.y));
                                const f2 gm = pk2(gn.gmul, gn.gmul);
                                // gmul · ((Fd_prev − Fd) + (Fh_up − Fh) + (Fw_left − Fw))
                                const f2 g01 = mul2(gm, add2(add2(sub2(Fd_prev[i][0], Fd.x), sub2(up01, Fh.x)),
                                                             sub2(wl01, Fw.x)));
                                const f2 g23 = mul2(gm, add2(add2(sub2(Fd_prev[i][1], Fd.y), sub2(up23, Fh.y)),
                                                             sub2(wl23, Fw.y)));
#ifdef QC_DEBUG_BOUNDS
                                float *dst = gp + (size_t)i * pl.W;
                                if (lane_in && (FULL || h < pl.H) &&
                                    QC_IN_BOUNDS((dst - grad) + 3,
                                                 (long long)pl.B * pl.Dp * pl.H * (long long)pl.W,
                                                 g_tv_fault_word))
                                    st_grad_pairs(dst, g01, g23);
#else
                                if (lane_in && (FULL || h < pl.H)) st_grad_pairs(gp + (size_t)i * pl.W, g01, g23);
#endif
                                Fd_prev[i][0] = Fd.x;
                                Fd_prev[i][1] = Fd.y;
                                up01 = Fh.x;
                                up23 = Fh.y;
                            }
                            curp = down;
                        }
                    };
                    if (hbase + R < pl.H)
                        rows(std::true_type{});
                    else
                        rows(std::false_type{});
                    if (LOSS) {
                        if constexpr (is_mix(V)) {
                            // slots: sq, iso, then the L1 axes (l0..l2)
                            if constexpr (has_sq(V))
                                acc0 += (double)((lo2(la01) + hi2(la01)) + (lo2(la23) + hi2(la23)));
                            if constexpr (has_iso(V))
                                acc1 += (double)((lo2(lb01) + hi2(lb01)) + (lo2(lb23) + hi2(lb23)));
                        } else {
                            l0 += (lo2(la01) + hi2(la01)) + (lo2(la23) + hi2(la23));
                        }
                    }
                }
                if (LOSS) {
                    if constexpr (is_mix(V)) {
                        if constexpr (has_l1(V)) {
                            acc2 += (double)l0;
                            acc3 += (double)l1;
                            acc4 += (double)l2;
                        }
                    } else {
                        acc0 += (double)l0;
                        if (V == QC_TV_L1) {
                            acc1 += (double)l1;
                            acc2 += (double)l2;
                        }
                    }
                }
                // Release plane p's stage.
                __syncwarp();
                if (lane == 0) mbar_arrive(&sm.empty[qc % S]);
            }
            if (aborted(sm)) break;
            if (U.last == U.d_end) {
                // The +1 halo plane was only ever a "next" plane: release it too.
                const int ql = q0 + (U.last - U.first);
                __syncwarp();
                if (lane == 0) mbar_arrive(&sm.empty[ql % S]);
            }
            seq = q0 + (U.last - U.first + 1);
        }
    }

    griddep_launch_dependents();

    if (LOSS) {
        if (warp < NW) {
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) {
                acc0 += __shfl_xor_sync(0xffffffffu, acc0, off);
                acc1 += __shfl_xor_sync(0xffffffffu, acc1, off);
                acc2 += __shfl_xor_sync(0xffffffffu, acc2, off);
                if constexpr (is_mix(V)) {
                    acc3 += __shfl_xor_sync(0xffffffffu, acc3, off);
                    acc4 += __shfl_xor_sync(0xffffffffu, acc4, off);
                }
            }
            if (lane == 0) {
                sm.red[warp][0] = acc0;
                sm.red[warp][1] = acc1;
                sm.red[warp][2] = acc2;
                if constexpr (is_mix(V)) {
                    sm.red[warp][3] = acc3;
                    sm.red[warp][4] = acc4;
                }
            }
        }
        __syncthreads();
        if (threadIdx.x < slots_of(V)) {
            double t = 0.0;
            for (int w = 0; w < NW; ++w) t += sm.red[w][threadIdx.x];
            store_cta_sum<V>(pl, partials, threadIdx.x, t);
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
    double acc[kMaxSlots] = {0.0, 0.0, 0.0, 0.0, 0.0};

    for (long long u = blockIdx.x; u < pl.n_units; u += gridDim.x) {
        const Unit U = decode_unit<GRAD>(pl, u, kGenTileH, kGenTileW);
        const int h = U.h0 + ty, w = U.w0 + tx;
        const bool in = h < pl.H && w < pl.W;
        const float *vb = vol + (size_t)U.n * pl.Dp * plane;
        const long long total = (long long)pl.B * pl.Dp * (long long)plane;
        auto at = [&](int p, int hh, int ww) -> float {
            const long long i = (long long)U.n * pl.Dp * (long long)plane + (long long)p * plane +
                                (long long)hh * pl.W + ww;
            return QC_IN_BOUNDS(i, total, g_tv_fault_word) ? __ldg(vol + i) : 0.f;
        };
        const bool vh = h + 1 < pl.H, vw = w + 1 < pl.W;
        float Fd_prev = 0.f;
        for (int p = U.first; p < U.d_end; ++p) {
            const bool has_nxt = (p + 1) <= U.last;
            const bool owned = p >= U.d_start;
            float l[kMaxSlots] = {0.f, 0.f, 0.f, 0.f, 0.f};
            float Fd = 0.f, Fh = 0.f, Fw = 0.f;
            if (in) {
                const float v = at(p, h, w);
                const float nd = has_nxt ? at(p + 1, h, w) : 0.f;
                const float nh = vh ? at(p, h + 1, w) : 0.f;
                const float nw = vw ? at(p, h, w + 1) : 0.f;
                voxel_flux<V, LOSS, GRAD>(v, nd, nh, nw, has_nxt, vh, vw, owned, pl.eps, gn, Fd,
                                          Fh, Fw, l);
                if (GRAD && owned) {
                    float Fh_up = 0.f, Fw_left = 0.f;
                    if (h >= 1) {
                        const float up = at(p, h - 1, w);
                        const float up_nd = (has_iso(V) && has_nxt) ? at(p + 1, h - 1, w) : 0.f;
                        const float up_nw = (has_iso(V) && vw) ? at(p, h - 1, w + 1) : 0.f;
                        Fh_up = flux_from_up<V>(v, up, up_nd, up_nw, true, has_nxt, vw, pl.eps, gn);
                    }
                    if (w >= 1) {
                        const float lf = at(p, h, w - 1);
                        const float lf_nd = (has_iso(V) && has_nxt) ? at(p + 1, h, w - 1) : 0.f;
                        const float lf_nh = (has_iso(V) && vh) ? at(p, h + 1, w - 1) : 0.f;
                        Fw_left = flux_from_left<V>(v, lf, lf_nd, lf_nh, true, has_nxt, vh, pl.eps, gn);
                    }
                    const float gv =
                        gn.gmul * ((Fd_prev - Fd) + (Fh_up - Fh) + (Fw_left - Fw));
                    const long long gi = (long long)U.n * pl.Dp * (long long)plane +
                                         (long long)p * plane + (long long)h * pl.W + w;
                    if (QC_IN_BOUNDS(gi, total, g_tv_fault_word)) grad[gi] = gv;
                }
            }
            Fd_prev = Fd;
            if (LOSS) {
#pragma unroll
                for (int a = 0; a < slots_of(V); ++a) acc[a] += (double)l[a];
            }
        }
    }

    griddep_launch_dependents();

    if (LOSS) {
        __shared__ double red[kGenThreads / 32][kMaxSlots];
        const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
        for (int a = 0; a < slots_of(V); ++a) {
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) acc[a] += __shfl_xor_sync(0xffffffffu, acc[a], off);
            if (lane == 0) red[warp][a] = acc[a];
        }
        __syncthreads();
        if (threadIdx.x < slots_of(V)) {
            double t = 0.0;
            for (int w = 0; w < kGenThreads / 32; ++w) t += red[w][threadIdx.x];
            store_cta_sum<V>(pl, partials, threadIdx.x, t);
        }
    }
}

// ── finalize: fixed-order sum of the CTA partials ────────────────────────

constexpr int kFinThreads = 256;

// Per-slot multipliers of the finalized sums (the isotropic mean's 1/N).
struct FinScales {
    float s[kMaxSlots];
};

__global__ void __launch_bounds__(kFinThreads) tv_finalize_kernel(const double *__restrict__ partials,
                                                                  int n_partials, int n_acc,
                                                                  int stride,
                                                                  float *__restrict__ acc,
                                                                  const FinScales scales,
                                                                  int overwrite) {
    griddep_wait();  // the sweep grid has completed and its writes are visible
    griddep_launch_dependents();  // the next sweep may start its set-up
    __shared__ double red[kMaxSlots][kFinThreads];
    // CTA i's sums start at partials[i * stride] (stride: the sweep's slot
    // count, 3 for a single term, 5 for a mixed sweep)
    for (int a = 0; a < n_acc; ++a) {
        double t = 0.0;
        for (int i = threadIdx.x; i < n_partials; i += kFinThreads)
            t += partials[(size_t)i * stride + a];
        red[a][threadIdx.x] = t;
    }
    __syncthreads();
    for (int s = kFinThreads / 2; s > 0; s >>= 1) {
        if (threadIdx.x < s)
            for (int a = 0; a < n_acc; ++a) red[a][threadIdx.x] += red[a][threadIdx.x + s];
        __syncthreads();
    }
    if (threadIdx.x < n_acc) {
        const float v = (float)(red[threadIdx.x][0] * (double)scales.s[threadIdx.x]);
        acc[threadIdx.x] = overwrite ? v : acc[threadIdx.x] + v;
    }
}

// The finalize of D-sharded losses: for each term (one loss's CTA partials),
// the fixed-order total of this rank's partials; all of this rank's totals go
// into slot [seq & 1][rank] of every rank's block, and after all ranks' flags
// show `seq`, every rank adds the slots in rank order. A slot is rewritten two
// calls later at the earliest, and a rank gets there only after every rank
// has finished reading it (its own call seq+1 waited for all). Several losses
// of one step share a single finalize, i.e. a single wait for the other ranks.
struct FinTerm {
    const double *partials;
    int n_partials, n_acc;
    float *acc;
    float scale;
    int overwrite;
};
struct FinTerms {
    FinTerm t[QC_TV_MAX_PEER_SUMS];
    int n;
};

__global__ void __launch_bounds__(kFinThreads) tv_finalize_peer_kernel(const FinTerms terms,
                                                                       qc_tv_peers peers,
                                                                       unsigned long long seq) {
    griddep_wait();
    __shared__ double red[kFinThreads];
    __shared__ double tot[QC_TV_MAX_PEER_SUMS];
    __shared__ int gave_up;
    if (threadIdx.x == 0) gave_up = 0;
    int n_sums = 0;
    for (int k = 0; k < terms.n; ++k) {
        const FinTerm &tm = terms.t[k];
        for (int a = 0; a < tm.n_acc; ++a, ++n_sums) {
            double t = 0.0;
            for (int i = threadIdx.x; i < tm.n_partials; i += kFinThreads)
                t += tm.partials[(size_t)i * kAccSlots + a];
            red[threadIdx.x] = t;
            __syncthreads();
            for (int s = kFinThreads / 2; s > 0; s >>= 1) {
                if (threadIdx.x < s) red[threadIdx.x] += red[threadIdx.x + s];
                __syncthreads();
            }
            if (threadIdx.x == 0) tot[n_sums] = red[0];
            __syncthreads();
        }
    }
    const int slot = (int)(seq & 1ull);
    if (threadIdx.x < n_sums) {
        const double v = tot[threadIdx.x];
        for (int q = 0; q < peers.world; ++q)
            static_cast<PeerComm *>(peers.comm[q])->partials[slot][peers.rank][threadIdx.x] = v;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        for (int q = 0; q < peers.world; ++q)
            st_relaxed_sys(&static_cast<PeerComm *>(peers.comm[q])->red_flag[peers.rank], seq);
    }
    PeerComm *self = static_cast<PeerComm *>(peers.comm[peers.rank]);
    if (threadIdx.x < peers.world) {
        if (!wait_flag_geq(&self->red_flag[threadIdx.x], seq, peer_limit(peers))) {
            atomicOr(&gave_up, 1);
            atomicOr(&g_tv_fault_word, QC_FAULT_PEER_WAIT);
        }
    }
    __syncthreads();
    if (threadIdx.x < n_sums) {
        double t = 0.0;
        for (int q = 0; q < peers.world; ++q)
            t += ld_relaxed_sys_f64(&self->partials[slot][q][threadIdx.x]);
        tot[threadIdx.x] = t;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int j = 0;
        for (int k = 0; k < terms.n; ++k) {
            const FinTerm &tm = terms.t[k];
            for (int a = 0; a < tm.n_acc; ++a, ++j) {
                const float v = gave_up ? __int_as_float(0x7fc00000) : (float)(tot[j] * (double)tm.scale);
                tm.acc[a] = tm.overwrite ? v : tm.acc[a] + v;
            }
        }
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

// Chooses the D-chunk of the chunk-major units. Each CTA runs its units one
// after another, so the time is modelled as rounds × (chunk + halo planes),
// rounds = ceil(units / resident CTAs); ties go to the larger chunk (fewer
// halo planes re-read from HBM).
void choose_chunking(Plan &pl, int max_ctas, int halo_planes) {
    const int Dn = pl.d_hi - pl.d_lo;
    long long best = -1;
    int best_dc = Dn, prev_dc = -1;
    for (int nch = 1; nch <= Dn; ++nch) {
        const int dc = (Dn + nch - 1) / nch;
        if (dc == prev_dc) continue;
        prev_dc = dc;
        const int real_nch = (Dn + dc - 1) / dc;
        const long long U = (long long)real_nch * pl.n_cols;
        const long long rounds = (U + max_ctas - 1) / max_ctas;
        const long long cost = rounds * (dc + halo_planes);
        if (best < 0 || cost < best) {
            best = cost;
            best_dc = dc;
        }
        if (U > 64LL * max_ctas) break;
    }
    pl.dchunk = best_dc;
    pl.n_chunks = (Dn + best_dc - 1) / best_dc;
    pl.n_units = (long long)pl.n_chunks * pl.n_cols;
}

// Fast-path geometry per variant: rows per consumer warp, consumer warps, ring
// stages and the CTAs per SM that registers are budgeted for, chosen by timing
// geometries on a B200 ([4, 256^3]): the L1 sweep, whose sign transfers need
// the most registers, runs 16-row tiles at 4 CTAs per SM (8% faster than
// 32-row tiles at 3); iso and sq keep 32-row tiles. QC_TV_R, QC_TV_NW, QC_TV_S
// and QC_TV_MINB override all three at build time.
template <int V>
struct FastGeomFor {
#ifdef QC_TV_R
    using type = Geom<QC_TV_R, QC_TV_NW, QC_TV_S, QC_TV_MINB>;
#else
    using type = Geom<8, 4, 3, 3>;
#endif
};
#ifndef QC_TV_R
template <>
struct FastGeomFor<QC_TV_L1> {
    using type = Geom<4, 4, 4, 4>;
};
#endif
// Mixed sweeps carry several terms' fluxes and loss sums per voxel: 16-row
// tiles with the register budget of 3 CTAs per SM.
// QC_TV_MIX_R, QC_TV_MIX_NW, QC_TV_MIX_S and QC_TV_MIX_MINB override it at
// build time.
template <int V>
struct MixGeom {
#ifdef QC_TV_MIX_R
    using type = Geom<QC_TV_MIX_R, QC_TV_MIX_NW, QC_TV_MIX_S, QC_TV_MIX_MINB>;
#else
    using type = Geom<4, 4, 4, 3>;
#endif
};

template <int V, bool LOSS, bool GRAD>
int launch_variant(bool use_tma, const float *vol, const float *g, float *grad, double *partials,
                   Plan pl, const HaloXchg &xc, int *grid_out, cudaStream_t stream) {
    int sms = 0;
    if (int st = device_sm_count(&sms)) return st;
    if (use_tma) {
        using G = typename std::conditional<is_mix(V), typename MixGeom<V>::type,
                                            typename FastGeomFor<V>::type>::type;
        EncodeTiledFn encode = nullptr;
        if (int st = get_encode_fn(&encode)) return st;
        // The tensor map is encoded through the driver API, which needs a
        // current context on this thread; a thread that has made no runtime
        // call yet (autograd's backward thread, a fresh host thread) has none.
        // cudaSetDevice on the current device binds its primary context.
        int dev = 0;
        QC_CUDA_TRY(cudaGetDevice(&dev), "cudaGetDevice");
        QC_CUDA_TRY(cudaSetDevice(dev), "cudaSetDevice");
        CUtensorMap map;
        const cuuint64_t dims[3] = {(cuuint64_t)pl.W, (cuuint64_t)pl.H,
                                    (cuuint64_t)pl.B * (cuuint64_t)pl.Dp};
        const cuuint64_t strides[2] = {(cuuint64_t)pl.W * 4, (cuuint64_t)pl.W * pl.H * 4};
        const cuuint32_t box[3] = {kBoxW, G::BoxH, 1};
        const cuuint32_t estr[3] = {1, 1, 1};
        CUresult cr = encode(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float *>(vol),
                             dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                             CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
        if (cr != CUDA_SUCCESS)
            return set_error(QC_ERR_TENSOR_MAP, "cuTensorMapEncodeTiled failed (CUresult %d) for "
                             "W=%d H=%d planes=%lld", (int)cr, pl.W, pl.H,
                             (long long)pl.B * pl.Dp);
        auto kern = tv_sweep_tma_kernel<V, LOSS, GRAD, G>;
        const size_t smem = sizeof(SweepSmem<G>) + 128;
        // Above 48 KB of dynamic shared memory needs an opt-in, a per-device
        // function attribute; it and the occupancy it allows are looked up
        // once per device (host-side cost off the per-call path).
        static std::atomic<int> occ_cache[kMaxDevices];
        int occ = (dev >= 0 && dev < kMaxDevices) ? occ_cache[dev].load(std::memory_order_relaxed) : 0;
        if (occ <= 0) {
            QC_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem),
                        "cudaFuncSetAttribute(tv_sweep_tma_kernel)");
            QC_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, G::Threads, smem),
                        "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
            if (dev >= 0 && dev < kMaxDevices && occ > 0) occ_cache[dev].store(occ, std::memory_order_relaxed);
        }
        int max_ctas = occ * sms;
        if (max_ctas > kMaxPartials) max_ctas = kMaxPartials;
        if (max_ctas < 1) max_ctas = 1;
        pl.n_ht = (pl.H + G::TileH - 1) / G::TileH;
        pl.n_wt = (pl.W + kTileW - 1) / kTileW;
        pl.n_cols = pl.B * pl.n_ht * pl.n_wt;
        choose_chunking(pl, max_ctas, 1 + (GRAD ? 1 : 0));
        const long long rounds = (pl.n_units + max_ctas - 1) / max_ctas;
        const int grid = (int)((pl.n_units + rounds - 1) / rounds);
        // programmatic dependent launch: the CTAs start (barrier set-up,
        // tensor-map prefetch) while the previous kernel drains; measured
        // 1.4% faster on a two-sweep step ([4, 256^3], iso then L1)
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(grid);
        cfg.blockDim = dim3(G::Threads);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        QC_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, map, g, grad, partials, pl, xc),
                    "tv_sweep_tma_kernel launch");
        *grid_out = grid;
    } else {
        auto kern = tv_sweep_generic_kernel<V, LOSS, GRAD>;
        int dev = 0;
        QC_CUDA_TRY(cudaGetDevice(&dev), "cudaGetDevice");
        static std::atomic<int> occ_cache[kMaxDevices];
        int occ = (dev >= 0 && dev < kMaxDevices) ? occ_cache[dev].load(std::memory_order_relaxed) : 0;
        if (occ <= 0) {
            QC_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kGenThreads, 0),
                        "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
            if (dev >= 0 && dev < kMaxDevices && occ > 0) occ_cache[dev].store(occ, std::memory_order_relaxed);
        }
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
                  double *partials, const Plan &pl, const HaloXchg &xc, int *grid,
                  cudaStream_t stream) {
    const bool L = flags & QC_TV_LOSS, G = flags & QC_TV_GRAD;
    if (L && G) return launch_variant<V, true, true>(use_tma, vol, g, grad, partials, pl, xc, grid, stream);
    if (L) return launch_variant<V, true, false>(use_tma, vol, g, grad, partials, pl, xc, grid, stream);
    return launch_variant<V, false, true>(use_tma, vol, g, grad, partials, pl, xc, grid, stream);
}

int launch_halo_exchange(const qc_tv_peers *peers, unsigned long long seq, float *d_slab, int B,
                         int Dp, int H, int W, cudaStream_t stream);

// Scratch of the deterministic reduction: one slot row per CTA partial.
size_t workspace_bytes_for(int variant) {
    return (size_t)kMaxPartials * slots_of(variant) * sizeof(double);
}
size_t workspace_bytes() { return (size_t)kMaxPartials * kMaxSlots * sizeof(double); }

// Mixed-term variants with a compiled sweep: sq+iso, sq+L1, iso+L1, all three.
bool mix_supported(int variant) {
    return variant == (kMix | 3) || variant == (kMix | 5) || variant == (kMix | 6) ||
           variant == (kMix | 7);
}

int run(int variant, int flags, const float *vol, const float *g, float *acc, float *grad, int B,
        int Dp, int H, int W, int d_lo, int d_hi, int has_prev, int has_next, float eps,
        float acc_scale, void *ws, size_t ws_bytes, cudaStream_t stream,
        const qc_tv_peers *peers = nullptr, unsigned long long seq = 0,
        unsigned long long halo_seq = 0, int *n_partials_out = nullptr,
        bool atomic_acc = false) {
    QC_NVTX(variant == QC_TV_SQ    ? "quantem::tv_sq"
            : variant == QC_TV_ISO ? "quantem::tv_iso"
            : variant == QC_TV_L1  ? "quantem::tv_l1"
                                   : "quantem::tv_mix");
    // n_partials_out != nullptr: launch the sweep only (its CTA partials stay
    // in ws, *n_partials_out of them) for a later tv_loss_3d_peer_finalize_cuda.
    const bool sweep_only = n_partials_out != nullptr;
    if (sweep_only) *n_partials_out = 0;
    const bool want_loss = flags & QC_TV_LOSS, want_grad = flags & QC_TV_GRAD;
    const bool mixed = is_mix(variant);
    QC_RETURN_IF((variant < QC_TV_SQ || variant > QC_TV_L1) && !mix_supported(variant),
                 QC_ERR_INVALID_ARGUMENT, "tv: unknown variant %d", variant);
    QC_RETURN_IF(mixed && (flags & (QC_TV_LOSS | QC_TV_GRAD)) != (QC_TV_LOSS | QC_TV_GRAD),
                 QC_ERR_INVALID_ARGUMENT, "tv: a mixed sweep computes losses and gradient together");
    QC_RETURN_IF(mixed && (peers != nullptr || n_partials_out != nullptr || atomic_acc),
                 QC_ERR_INVALID_ARGUMENT, "tv: mixed sweeps are single-GPU, deterministic-workspace only");
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
    const int n_acc = mixed ? kMixSlots : (variant == QC_TV_L1 ? 3 : 1);
    const bool empty = B == 0 || H == 0 || W == 0 || d_hi == d_lo;
    QC_RETURN_IF(atomic_acc && (peers != nullptr || sweep_only || (flags & QC_TV_ACC_OVERWRITE)),
                 QC_ERR_INVALID_ARGUMENT, "tv: atomic accumulation is for single-GPU acc += calls");
    if (want_loss) {
        QC_RETURN_IF(acc == nullptr, QC_ERR_INVALID_ARGUMENT, "tv: null acc");
    }
    if (want_loss && !atomic_acc) {
        QC_RETURN_IF(ws == nullptr || ws_bytes < workspace_bytes_for(variant),
                     QC_ERR_WORKSPACE_TOO_SMALL,
                     "tv: workspace of %zu bytes is below the %zu required", ws_bytes,
                     workspace_bytes_for(variant));
    }
    if (want_grad) {
        QC_RETURN_IF(grad == nullptr, QC_ERR_INVALID_ARGUMENT, "tv: null grad");
        QC_RETURN_IF(g == nullptr, QC_ERR_INVALID_ARGUMENT, "tv: null upstream gradient");
    }
    QC_RETURN_IF(!empty && vol == nullptr, QC_ERR_INVALID_ARGUMENT, "tv: null volume");

    if (empty && peers == nullptr && !sweep_only) {
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
    // a mixed sweep: acc_scale multiplies its isotropic sum (slot 1) and the
    // isotropic gradient term, the other gains come from d_g unscaled
    pl.scale = acc_scale;
    pl.acc_atomic = (atomic_acc && want_loss) ? acc : nullptr;

    const bool aligned = (reinterpret_cast<uintptr_t>(vol) % 16 == 0) &&
                         (!want_grad || reinterpret_cast<uintptr_t>(grad) % 16 == 0);
    const bool use_tma = (W % 4 == 0) && aligned && ((long long)B * Dp < (1LL << 31));

    double *partials = atomic_acc ? nullptr : reinterpret_cast<double *>(ws);
    int grid = 0;
    int st = 0;
    HaloXchg xc{};
    if (halo_seq != 0 && peers != nullptr && peers->world > 1) {
        if (use_tma && !empty) {
            // the sweep kernel stores the boundary planes and waits for the halos itself
            const int r = peers->rank;
            xc.self = static_cast<PeerComm *>(peers->comm[r]);
            xc.prev = r > 0 ? static_cast<PeerComm *>(peers->comm[r - 1]) : nullptr;
            xc.next = r < peers->world - 1 ? static_cast<PeerComm *>(peers->comm[r + 1]) : nullptr;
            xc.prev_slab = peers->prev_slab;
            xc.next_slab = peers->next_slab;
            xc.prev_dp = peers->prev_dp;
            xc.next_dp = peers->next_dp;
            xc.vol = vol;
            xc.seq = halo_seq;
            xc.limit_ns = peers->timeout_ns ? peers->timeout_ns : kPeerWaitLimitNs;
        } else {
            st = launch_halo_exchange(peers, halo_seq, const_cast<float *>(vol), B, Dp, H, W, stream);
            if (st) return st;
        }
    }
    if (empty) {
        // a rank that owns no planes still takes part in the cross-rank sum
    } else switch (variant) {
        case QC_TV_SQ: st = dispatch_mode<QC_TV_SQ>(flags, use_tma, vol, g, grad, partials, pl, xc, &grid, stream); break;
        case QC_TV_ISO: st = dispatch_mode<QC_TV_ISO>(flags, use_tma, vol, g, grad, partials, pl, xc, &grid, stream); break;
        case QC_TV_L1: st = dispatch_mode<QC_TV_L1>(flags, use_tma, vol, g, grad, partials, pl, xc, &grid, stream); break;
        case kMix | 3: st = launch_variant<kMix | 3, true, true>(use_tma, vol, g, grad, partials, pl, xc, &grid, stream); break;
        case kMix | 5: st = launch_variant<kMix | 5, true, true>(use_tma, vol, g, grad, partials, pl, xc, &grid, stream); break;
        case kMix | 6: st = launch_variant<kMix | 6, true, true>(use_tma, vol, g, grad, partials, pl, xc, &grid, stream); break;
        default: st = launch_variant<kMix | 7, true, true>(use_tma, vol, g, grad, partials, pl, xc, &grid, stream); break;
    }
    if (st) return st;

    if (sweep_only) {
        *n_partials_out = want_loss ? grid : 0;
        return 0;
    }
    if (want_loss && !atomic_acc) {
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
        if (peers != nullptr) {
            FinTerms terms{};
            terms.n = 1;
            terms.t[0] = FinTerm{partials, grid, n_acc, acc, acc_scale,
                                 (flags & QC_TV_ACC_OVERWRITE) ? 1 : 0};
            QC_CUDA_TRY(cudaLaunchKernelEx(&cfg, tv_finalize_peer_kernel, terms, *peers, seq),
                        "tv_finalize_peer_kernel launch");
        } else {
            FinScales sc;
            for (int a = 0; a < kMaxSlots; ++a) sc.s[a] = mixed ? (a == 1 ? acc_scale : 1.0f) : acc_scale;
            QC_CUDA_TRY(cudaLaunchKernelEx(&cfg, tv_finalize_kernel, (const double *)partials, grid,
                                           n_acc, slots_of(variant), acc, sc,
                                           (flags & QC_TV_ACC_OVERWRITE) ? 1 : 0),
                        "tv_finalize_kernel launch");
        }
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

// The reference's loss launchers (csrc/ops/core.h:16-22, :40-45, :62-67):
// acc += Σ with each CTA's sum added by an fp32 atomic, as the reference's
// kernels do; no workspace, not bitwise reproducible run to run.
int tv_loss_iso_3d_cuda(const float *d_vol, float *d_acc, int B, int D, int H, int W, float eps,
                        cudaStream_t stream) {
    return qc::tv::run(QC_TV_ISO, QC_TV_LOSS, d_vol, nullptr, d_acc, nullptr, B, D, H, W, 0, D, 0,
                       0, eps, 1.0f, nullptr, 0, stream, nullptr, 0, 0, nullptr, true);
}

int tv_loss_sq_3d_cuda(const float *d_vol, float *d_acc, int B, int D, int H, int W,
                       cudaStream_t stream) {
    return qc::tv::run(QC_TV_SQ, QC_TV_LOSS, d_vol, nullptr, d_acc, nullptr, B, D, H, W, 0, D, 0,
                       0, 0.f, 1.0f, nullptr, 0, stream, nullptr, 0, 0, nullptr, true);
}

int tv_loss_l1_3d_cuda(const float *d_vol, float *d_acc, int B, int D, int H, int W,
                       cudaStream_t stream) {
    return qc::tv::run(QC_TV_L1, QC_TV_LOSS, d_vol, nullptr, d_acc, nullptr, B, D, H, W, 0, D, 0,
                       0, 0.f, 1.0f, nullptr, 0, stream, nullptr, 0, 0, nullptr, true);
}

// Deterministic forms: CTA sums go to the caller's workspace and one
// finalize kernel adds them in a fixed order (bitwise reproducible).
int tv_loss_iso_3d_ws_cuda(const float *d_vol, float *d_acc, int B, int D, int H, int W, float eps,
                           void *d_workspace, size_t workspace_bytes, cudaStream_t stream) {
    return qc::tv::run(QC_TV_ISO, QC_TV_LOSS, d_vol, nullptr, d_acc, nullptr, B, D, H, W, 0, D, 0,
                       0, eps, 1.0f, d_workspace, workspace_bytes, stream);
}

int tv_loss_iso_3d_grad_cuda(const float *d_vol, const float *d_g_scaled, float *d_grad_vol,
                             int B, int D, int H, int W, float eps, cudaStream_t stream) {
    return qc::tv::run(QC_TV_ISO, QC_TV_GRAD, d_vol, d_g_scaled, nullptr, d_grad_vol, B, D, H, W,
                       0, D, 0, 0, eps, 1.0f, nullptr, 0, stream);
}

int tv_loss_sq_3d_ws_cuda(const float *d_vol, float *d_acc, int B, int D, int H, int W,
                          void *d_workspace, size_t workspace_bytes, cudaStream_t stream) {
    return qc::tv::run(QC_TV_SQ, QC_TV_LOSS, d_vol, nullptr, d_acc, nullptr, B, D, H, W, 0, D, 0,
                       0, 0.f, 1.0f, d_workspace, workspace_bytes, stream);
}

int tv_loss_sq_3d_grad_cuda(const float *d_vol, const float *d_g, float *d_grad_vol, int B, int D,
                            int H, int W, cudaStream_t stream) {
    return qc::tv::run(QC_TV_SQ, QC_TV_GRAD, d_vol, d_g, nullptr, d_grad_vol, B, D, H, W, 0, D, 0,
                       0, 0.f, 1.0f, nullptr, 0, stream);
}

int tv_loss_l1_3d_ws_cuda(const float *d_vol, float *d_acc, int B, int D, int H, int W,
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

int tv_loss_mix_3d_fwd_grad_cuda(int terms, int flags, const float *d_vol, const float *d_g,
                                 float *d_acc, float *d_grad_vol, int B, int D, int H, int W,
                                 float eps, float iso_scale, void *d_workspace,
                                 size_t workspace_bytes, cudaStream_t stream) {
    QC_RETURN_IF(terms != (QC_TV_TERM_SQ | QC_TV_TERM_ISO) && terms != (QC_TV_TERM_SQ | QC_TV_TERM_L1) &&
                     terms != (QC_TV_TERM_ISO | QC_TV_TERM_L1) &&
                     terms != (QC_TV_TERM_SQ | QC_TV_TERM_ISO | QC_TV_TERM_L1),
                 QC_ERR_INVALID_ARGUMENT,
                 "tv_loss_mix_3d_fwd_grad_cuda: terms 0x%x must name two or three of "
                 "QC_TV_TERM_SQ, QC_TV_TERM_ISO, QC_TV_TERM_L1",
                 (unsigned)terms);
    QC_RETURN_IF(flags & ~QC_TV_ACC_OVERWRITE, QC_ERR_INVALID_ARGUMENT,
                 "tv_loss_mix_3d_fwd_grad_cuda: flags may only hold QC_TV_ACC_OVERWRITE");
    return qc::tv::run(qc::tv::kMix | terms, QC_TV_LOSS | QC_TV_GRAD | flags, d_vol, d_g, d_acc,
                       d_grad_vol, B, D, H, W, 0, D, 0, 0, eps, iso_scale, d_workspace,
                       workspace_bytes, stream);
}

int quantem_cuda_device_fault_word(int device, unsigned int *word, int clear) {
    int prev = 0;
    QC_CUDA_TRY(cudaGetDevice(&prev), "cudaGetDevice");
    QC_CUDA_TRY(cudaSetDevice(device), "cudaSetDevice");
    unsigned int w = 0, wk = 0, wp = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&w, qc::tv::g_tv_fault_word, sizeof(w));
    if (e == cudaSuccess && clear) {
        const unsigned int zero = 0;
        e = cudaMemcpyToSymbol(qc::tv::g_tv_fault_word, &zero, sizeof(zero));
    }
    int st = e == cudaSuccess ? qc::kp_fault_word(&wk, clear) : 0;
    if (e == cudaSuccess && st == 0) st = qc::pr_fault_word(&wp, clear);
    cudaSetDevice(prev);
    QC_CUDA_TRY(e, "cudaMemcpyFromSymbol(fault word)");
    if (st) return st;
    if (word) *word = w | wk | wp;
    return 0;
}

}  // extern "C"

// ── isotropic single sweep for callers that cannot allocate ────────────────
//
// Some callers of this library cannot call cudaMalloc (or any allocating
// routine) where they compute the loss: applications whose device memory is
// owned up front by a single allocator (a framework's caching allocator, an
// arena sized to a fixed budget) that another cudaMalloc would defeat or fail
// against, and embedded or real-time hosts that allocate only at start-up.
// For them the workspace of the deterministic reduction lives in this file
// instead: a statically allocated device array, present on every GPU that
// loads the library until the process exits. The entry still launches the
// sweep and finalize kernels like every other entry point; it only avoids
// allocating.

namespace qc {
namespace tv {

// 2048 CTA partial-sum slots × 3 fp64 = 48 KiB: the most the sweep planner
// uses for any volume shape (it caps the grid at kMaxPartials CTAs).
static __device__ __align__(256) double g_static_partials[kMaxPartials * kAccSlots];
static_assert(sizeof(g_static_partials) >= (size_t)kMaxPartials * kAccSlots * sizeof(double),
              "the static scratch must hold the planner's largest grid");

// Device address of g_static_partials on the current device. The host-side
// name is only a stand-in for the array, so it is translated once per device,
// with that device current, on the entry's first call there. The address is
// kept for the life of the process: after cudaDeviceReset the module is
// reloaded and the cached address is stale, so the entry must not be used
// across a device reset.
int static_partials_address(double **out) {
    static std::mutex mu;
    static double *addr[kMaxDevices] = {nullptr};
    int dev = 0;
    QC_CUDA_TRY(cudaGetDevice(&dev), "cudaGetDevice");
    std::lock_guard<std::mutex> lock(mu);
    if (dev >= 0 && dev < kMaxDevices && addr[dev] != nullptr) {
        *out = addr[dev];
        return 0;
    }
    double *p = nullptr;
    QC_CUDA_TRY(cudaGetSymbolAddress(reinterpret_cast<void **>(&p), g_static_partials),
                "cudaGetSymbolAddress(static TV scratch)");
    if (dev >= 0 && dev < kMaxDevices) addr[dev] = p;
    *out = p;
    return 0;
}

}  // namespace tv
}  // namespace qc

extern "C" int tv_loss_iso_3d_fwd_grad_noalloc_cuda(const float *d_vol, const float *d_g_scaled,
                                                    float *d_acc, float *d_grad_vol, int B, int D,
                                                    int H, int W, float eps, cudaStream_t stream) {
    // Shapes the sweep cannot index are refused before any CUDA call; every
    // other shape fits the static scratch (static_assert above).
    QC_RETURN_IF(B < 0 || D < 0 || H < 0 || W < 0, QC_ERR_INVALID_ARGUMENT,
                 "tv_loss_iso_3d_fwd_grad_noalloc_cuda: negative shape [%d, %d, %d, %d]", B, D, H, W);
    QC_RETURN_IF((long long)H * W >= (1LL << 31) || (long long)B * D >= (1LL << 31),
                 QC_ERR_INVALID_ARGUMENT,
                 "tv_loss_iso_3d_fwd_grad_noalloc_cuda: [%d, %d, %d, %d] exceeds the largest volume "
                 "(H*W and B*D below 2^31)",
                 B, D, H, W);
    double *scratch = nullptr;
    if (int st = qc::tv::static_partials_address(&scratch)) return st;
    return qc::tv::run(QC_TV_ISO, QC_TV_LOSS | QC_TV_GRAD, d_vol, d_g_scaled, d_acc, d_grad_vol, B,
                       D, H, W, 0, D, 0, 0, eps, 1.0f, scratch, sizeof(qc::tv::g_static_partials),
                       stream);
}

// ── D-slabs over peer memory: halo exchange and the C ABI ─────────────────

namespace qc {
namespace tv {

constexpr int kHaloThreads = 256;

// Stores this rank's boundary planes into its neighbours' halos (plane 1 into
// rank-1's plane prev_dp-1, plane Dp-2 into rank+1's plane 0) and waits for
// theirs. Every CTA first tells both neighbours that this rank's halos may be
// overwritten (everything earlier on this stream, the sweeps that read the
// old halos included, has completed), then waits for the same word from the
// neighbours it stores into, so no CTA depends on another CTA being resident.
// The last CTA to finish storing raises the neighbours' `filled` flags and
// waits for this rank's own.
__global__ void __launch_bounds__(kHaloThreads) tv_halo_exchange_kernel(
    qc_tv_peers peers, unsigned long long seq, const float *__restrict__ slab, int B, int Dp,
    long long plane, int vec4) {
    const bool has_prev = peers.rank > 0, has_next = peers.rank < peers.world - 1;
    PeerComm *self = static_cast<PeerComm *>(peers.comm[peers.rank]);
    PeerComm *prevc = has_prev ? static_cast<PeerComm *>(peers.comm[peers.rank - 1]) : nullptr;
    PeerComm *nextc = has_next ? static_cast<PeerComm *>(peers.comm[peers.rank + 1]) : nullptr;
    const uint64_t limit = peer_limit(peers);
    __shared__ int go;
    if (threadIdx.x == 0) {
        if (has_prev) st_relaxed_sys(&prevc->ready[1], seq);
        if (has_next) st_relaxed_sys(&nextc->ready[0], seq);
        bool ok = true;
        if (has_prev) ok = wait_flag_geq(&self->ready[0], seq, limit) && ok;
        if (has_next) ok = wait_flag_geq(&self->ready[1], seq, limit) && ok;
        if (!ok) atomicOr(&g_tv_fault_word, QC_FAULT_PEER_WAIT);
        go = ok ? 1 : 0;
    }
    __syncthreads();
    if (go) {
        // work items: side (prev, next) × batch slice × plane elements (or float4s)
        const long long per = vec4 ? plane / 4 : plane;
        const long long per_side = (long long)B * per;
        const long long n = per_side * 2;
        const long long stride = (long long)gridDim.x * blockDim.x;
        for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
            const int side = i >= per_side;
            if (side == 0 ? !has_prev : !has_next) continue;
            const long long j = i - side * per_side;
            const long long b = j / per, e = j - b * per;
            const long long src_plane = (long long)b * Dp + (side == 0 ? 1 : Dp - 2);
            const long long dst_plane = side == 0 ? (long long)b * peers.prev_dp + peers.prev_dp - 1
                                                  : (long long)b * peers.next_dp;
            float *dst = side == 0 ? peers.prev_slab : peers.next_slab;
            const int ddp = side == 0 ? peers.prev_dp : peers.next_dp;
            const long long last = vec4 ? e * 4 + 3 : e;
            if (!QC_IN_BOUNDS(src_plane * plane + last, (long long)B * Dp * plane, g_tv_fault_word) ||
                !QC_IN_BOUNDS(dst_plane * plane + last, (long long)B * ddp * plane, g_tv_fault_word))
                continue;
            if (vec4) {
                const float4 v = ldg4(slab + src_plane * plane + e * 4);
                *reinterpret_cast<float4 *>(dst + dst_plane * plane + e * 4) = v;
            } else {
                dst[dst_plane * plane + e] = __ldg(slab + src_plane * plane + e);
            }
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        const unsigned int before = atomicAdd(&self->arrive, 1u);
        if (before == gridDim.x - 1) {
            self->arrive = 0;  // the next exchange on this stream starts after this grid
            __threadfence_system();
            if (has_prev) st_relaxed_sys(&prevc->filled[1], seq);
            if (has_next) st_relaxed_sys(&nextc->filled[0], seq);
            bool ok = true;
            if (has_prev) ok = wait_flag_geq(&self->filled[0], seq, limit) && ok;
            if (has_next) ok = wait_flag_geq(&self->filled[1], seq, limit) && ok;
            if (!ok) atomicOr(&g_tv_fault_word, QC_FAULT_PEER_WAIT);
            // the sweeps read the halos with TMA (the async proxy)
            asm volatile("fence.proxy.async.global;" ::: "memory");
        }
    }
}

int check_peers(const qc_tv_peers *p, unsigned long long seq) {
    QC_RETURN_IF(p == nullptr, QC_ERR_INVALID_ARGUMENT, "tv peers: null peers");
    QC_RETURN_IF(p->world < 1 || p->world > QC_MAX_PEER_RANKS, QC_ERR_INVALID_ARGUMENT,
                 "tv peers: world %d outside [1, %d]", p->world, QC_MAX_PEER_RANKS);
    QC_RETURN_IF(p->rank < 0 || p->rank >= p->world, QC_ERR_INVALID_ARGUMENT,
                 "tv peers: rank %d outside [0, %d)", p->rank, p->world);
    QC_RETURN_IF(seq == 0, QC_ERR_INVALID_ARGUMENT, "tv peers: seq starts at 1");
    for (int q = 0; q < p->world; ++q)
        QC_RETURN_IF(p->comm[q] == nullptr, QC_ERR_INVALID_ARGUMENT,
                     "tv peers: null communication block of rank %d", q);
    return 0;
}

int launch_halo_exchange(const qc_tv_peers *peers, unsigned long long seq, float *d_slab, int B,
                         int Dp, int H, int W, cudaStream_t stream) {
    QC_NVTX("quantem::tv_halo_exchange");
    if (int st = check_peers(peers, seq)) return st;
    const bool has_prev = peers->rank > 0, has_next = peers->rank < peers->world - 1;
    QC_RETURN_IF(B < 0 || H < 0 || W < 0, QC_ERR_INVALID_ARGUMENT,
                 "tv_slab_halo_exchange_cuda: negative shape");
    QC_RETURN_IF(Dp < 3, QC_ERR_INVALID_ARGUMENT,
                 "tv_slab_halo_exchange_cuda: a slab needs a halo on each side and an owned "
                 "plane (Dp = %d)", Dp);
    QC_RETURN_IF(has_prev && (peers->prev_slab == nullptr || peers->prev_dp < 3),
                 QC_ERR_INVALID_ARGUMENT, "tv_slab_halo_exchange_cuda: rank-1's slab missing");
    QC_RETURN_IF(has_next && (peers->next_slab == nullptr || peers->next_dp < 3),
                 QC_ERR_INVALID_ARGUMENT, "tv_slab_halo_exchange_cuda: rank+1's slab missing");
    QC_RETURN_IF(d_slab == nullptr, QC_ERR_INVALID_ARGUMENT, "tv_slab_halo_exchange_cuda: null slab");
    if (peers->world == 1) return 0;
    const long long plane = (long long)H * W;
    const bool vec4 = plane % 4 == 0 && reinterpret_cast<uintptr_t>(d_slab) % 16 == 0 &&
                      (!has_prev || reinterpret_cast<uintptr_t>(peers->prev_slab) % 16 == 0) &&
                      (!has_next || reinterpret_cast<uintptr_t>(peers->next_slab) % 16 == 0);
    const long long items = 2LL * B * (vec4 ? plane / 4 : plane);
    int sms = 0;
    if (int st = qc::device_sm_count(&sms)) return st;
    long long grid = (items + kHaloThreads - 1) / kHaloThreads;
    if (grid > 2LL * sms) grid = 2LL * sms;
    if (grid < 1) grid = 1;
    tv_halo_exchange_kernel<<<(unsigned)grid, kHaloThreads, 0, stream>>>(*peers, seq, d_slab, B, Dp,
                                                                          plane, vec4 ? 1 : 0);
    QC_CHECK_LAUNCH("tv_halo_exchange_kernel launch");
    return 0;
}

}  // namespace tv
}  // namespace qc

extern "C" {

size_t tv_peer_comm_bytes(void) { return sizeof(qc::tv::PeerComm); }

int tv_slab_halo_exchange_cuda(const qc_tv_peers *peers, unsigned long long seq, float *d_slab,
                               int B, int Dp, int H, int W, cudaStream_t stream) {
    return qc::tv::launch_halo_exchange(peers, seq, d_slab, B, Dp, H, W, stream);
}

int tv_loss_3d_slab_peer_cuda(const qc_tv_peers *peers, unsigned long long halo_seq,
                              unsigned long long seq, int variant, int flags, const float *d_vol,
                              const float *d_g, float *d_acc, float *d_grad_vol, int B, int Dp,
                              int H, int W, int d_lo, int d_hi, int has_prev, int has_next,
                              float eps, float acc_scale, void *d_workspace,
                              size_t workspace_bytes, cudaStream_t stream) {
    using namespace qc::tv;
    if (int st = check_peers(peers, seq)) return st;
    if (halo_seq != 0) {
        const bool prev = peers->rank > 0, next = peers->rank < peers->world - 1;
        QC_RETURN_IF(d_lo != 1 || d_hi != Dp - 1 || (int)prev != (has_prev ? 1 : 0) ||
                         (int)next != (has_next ? 1 : 0),
                     QC_ERR_INVALID_ARGUMENT,
                     "tv_loss_3d_slab_peer_cuda: exchanging halos needs the slab layout (owned "
                     "planes [1, Dp-1), neighbours exactly where the ranks have them)");
        QC_RETURN_IF(Dp < 3, QC_ERR_INVALID_ARGUMENT,
                     "tv_loss_3d_slab_peer_cuda: a slab needs a halo on each side and an owned plane");
        QC_RETURN_IF((prev && (peers->prev_slab == nullptr || peers->prev_dp < 3)) ||
                         (next && (peers->next_slab == nullptr || peers->next_dp < 3)),
                     QC_ERR_INVALID_ARGUMENT, "tv_loss_3d_slab_peer_cuda: a neighbour's slab is missing");
    }
    QC_RETURN_IF(!(flags & QC_TV_LOSS), QC_ERR_INVALID_ARGUMENT,
                 "tv_loss_3d_slab_peer_cuda: flags must include QC_TV_LOSS (use "
                 "tv_loss_3d_slab_cuda for the gradient alone)");
    return run(variant, flags, d_vol, d_g, d_acc, d_grad_vol, B, Dp, H, W, d_lo, d_hi, has_prev,
               has_next, eps, acc_scale, d_workspace, workspace_bytes, stream, peers, seq, halo_seq);
}

}  // extern "C"

extern "C" int tv_loss_3d_slab_sweep_cuda(const qc_tv_peers *peers, unsigned long long halo_seq,
                                          int variant, int flags, const float *d_vol,
                                          const float *d_g, float *d_grad_vol, int B, int Dp,
                                          int H, int W, int d_lo, int d_hi, int has_prev,
                                          int has_next, float eps, float acc_scale,
                                          void *d_workspace, size_t workspace_bytes,
                                          int *n_partials, cudaStream_t stream) {
    using namespace qc::tv;
    QC_RETURN_IF(n_partials == nullptr, QC_ERR_INVALID_ARGUMENT,
                 "tv_loss_3d_slab_sweep_cuda: null n_partials");
    if (halo_seq != 0) {
        if (int st = check_peers(peers, 1)) return st;
        QC_RETURN_IF(d_lo != 1 || d_hi != Dp - 1, QC_ERR_INVALID_ARGUMENT,
                     "tv_loss_3d_slab_sweep_cuda: exchanging halos needs the slab layout "
                     "(owned planes [1, Dp-1))");
        QC_RETURN_IF((peers->rank > 0 && peers->prev_slab == nullptr) ||
                         (peers->rank < peers->world - 1 && peers->next_slab == nullptr),
                     QC_ERR_INVALID_ARGUMENT, "tv_loss_3d_slab_sweep_cuda: a neighbour's slab is missing");
    }
    // a dummy acc satisfies run()'s argument checks; the sweep never writes it
    static float unused_acc;
    return run(variant, flags, d_vol, d_g, &unused_acc, d_grad_vol, B, Dp, H, W, d_lo, d_hi,
               has_prev, has_next, eps, acc_scale, d_workspace, workspace_bytes, stream,
               halo_seq != 0 ? peers : nullptr, 0, halo_seq, n_partials);
}

extern "C" int tv_loss_3d_peer_finalize_cuda(const qc_tv_peers *peers, unsigned long long seq,
                                             const qc_tv_term *terms, int n_terms,
                                             cudaStream_t stream) {
    using namespace qc::tv;
    QC_NVTX("quantem::tv_peer_finalize");
    if (int st = check_peers(peers, seq)) return st;
    QC_RETURN_IF(terms == nullptr || n_terms < 1 || n_terms > QC_TV_MAX_PEER_SUMS,
                 QC_ERR_INVALID_ARGUMENT, "tv_loss_3d_peer_finalize_cuda: %d terms", n_terms);
    FinTerms ft{};
    int sums = 0;
    for (int k = 0; k < n_terms; ++k) {
        const qc_tv_term &t = terms[k];
        QC_RETURN_IF(t.acc == nullptr || t.n_acc < 1 || t.n_acc > kAccSlots || t.n_partials < 0 ||
                         t.n_partials > kMaxPartials || (t.n_partials > 0 && t.workspace == nullptr),
                     QC_ERR_INVALID_ARGUMENT, "tv_loss_3d_peer_finalize_cuda: bad term %d", k);
        sums += t.n_acc;
        ft.t[k] = FinTerm{static_cast<const double *>(t.workspace), t.n_partials, t.n_acc, t.acc,
                          t.acc_scale, t.overwrite ? 1 : 0};
    }
    QC_RETURN_IF(sums > QC_TV_MAX_PEER_SUMS, QC_ERR_INVALID_ARGUMENT,
                 "tv_loss_3d_peer_finalize_cuda: %d sums exceed %d", sums, QC_TV_MAX_PEER_SUMS);
    ft.n = n_terms;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(kFinThreads);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    QC_CUDA_TRY(cudaLaunchKernelEx(&cfg, tv_finalize_peer_kernel, ft, *peers, seq),
                "tv_finalize_peer_kernel launch");
    return 0;
}
