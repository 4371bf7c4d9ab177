// kplanes_tilted.cu — fused tilted K-Planes interpolation, forward and
// backward, for sm_100a.
//
// Reference semantics: csrc/cuda/core/ml/kplanes_tilted.cu:62-327 (kernels and
// launchers), src/quantem/cuda/core/ml/_ops.py:28-101 (op layer), and the
// pure-torch definition in tests/core/ml/test_kplanes_tilted.py:26-40:
//
//   r = R_t · p;  (gx, gy) per plane p: XY (rx, ry), ZX (rz, rx), YZ (ry, rz)
//   s_p = grid_sample(plane[t*3+p], (gx, gy), align_corners=True, border)
//   out[b, t*C + c] = s_0 · s_1 · s_2
//
// Mapping. A "group" of L = C/4 lanes handles one (point, rotation); each lane
// owns 4 consecutive channels and moves them with 16-byte loads, stores and
// vector reductions, so a C=32 corner row (128 B, one L2 line) is one
// instruction for 8 lanes. A warp holds 32/L groups, i.e. a tile of 32/L
// consecutive points, and loops over the T rotations for its tile. Looping
// Each (point, rotation) output row of C floats is written as whole lines.
//
// The tap arithmetic (unnormalise, clamp, floor, bilinear weights, border
// gradient mask) follows the operation order of the reference's make_tap
// (kplanes_tilted.cu:69-94). The rotation and the bilinear sums are written as
// explicit FMAs in the order nvcc gives the reference's plain expressions
// (a0*x0 + a1*x1 + ... contracts to fma(.., fma(a0, x0, a1*x1))), so forward
// values agree bit for bit with the reference kernel and with the CPU oracle,
// which uses the same explicit order.
//
// Backward. Plane gradients go out as red.global.add.v4.f32 (one L2 atomic op
// per 16 B instead of four); corners with zero bilinear weight are skipped.
// Coordinate gradients are reduced over the group's lanes with xor shuffles
// and mapped to dL/dr with the border masks; grad_pts takes three scalar
// reductions per (point, rotation); grad_R is accumulated in registers per
// group and reduced across the block once, one global reduction per entry.
#include "qc_common.cuh"

namespace qc {
namespace kp {

// QC_FAULT_BOUNDS from the debug build's checks (see check_tap).
__device__ unsigned int g_kp_fault_word = 0;

struct Tap {
    int cell[4];     // y*W + x of the (nw, ne, sw, se) corners, +1 sides clamped
    float w[4];      // bilinear weights; 0 exactly where a +1 side was clamped
    float tx, ty;    // fractional offsets
    float gxm, gym;  // d(ix)/d(gx), d(iy)/d(gy) with torch's border-clip mask
};

__device__ __forceinline__ Tap make_tap(float gx, float gy, int H, int W) {
    Tap t;
    const float wm1 = (float)(W - 1), hm1 = (float)(H - 1);
    float ix = (gx + 1.f) * 0.5f * wm1;
    float iy = (gy + 1.f) * 0.5f * hm1;
    // torch's clip_coordinates_set_grad: zero gradient at and beyond the border.
    t.gxm = (ix > 0.f && ix < wm1) ? 0.5f * wm1 : 0.f;
    t.gym = (iy > 0.f && iy < hm1) ? 0.5f * hm1 : 0.f;
    ix = fminf(fmaxf(ix, 0.f), wm1);
    iy = fminf(fmaxf(iy, 0.f), hm1);
    const int x0 = (int)ix, y0 = (int)iy;
    t.tx = ix - (float)x0;
    t.ty = iy - (float)y0;
    t.w[0] = (1.f - t.tx) * (1.f - t.ty);
    t.w[1] = t.tx * (1.f - t.ty);
    t.w[2] = (1.f - t.tx) * t.ty;
    t.w[3] = t.tx * t.ty;
    const int x1 = min(x0 + 1, W - 1), y1 = min(y0 + 1, H - 1);
    t.cell[0] = y0 * W + x0;
    t.cell[1] = y0 * W + x1;
    t.cell[2] = y1 * W + x0;
    t.cell[3] = y1 * W + x1;
    return t;
}

// Debug build: every corner index must lie in the plane; one that does not is
// recorded and redirected to cell 0 so that no access leaves the buffers.
__device__ __forceinline__ void check_tap(Tap &t, int H, int W) {
#ifdef QC_DEBUG_BOUNDS
#pragma unroll
    for (int k = 0; k < 4; ++k)
        if (!QC_IN_BOUNDS(t.cell[k], (long long)H * W, g_kp_fault_word)) t.cell[k] = 0;
#else
    (void)t;
    (void)H;
    (void)W;
#endif
}

// r = R_t·p as a0*x0 + a1*x1 + a2*x2 evaluated the way nvcc contracts that
// expression: the first product is fused around the second, then the third
// is fused on top — fma(a2, x2, fma(a0, x0, a1*x1)).
__device__ __forceinline__ float dot3(float a0, float x0, float a1, float x1, float a2, float x2) {
    return __fmaf_rn(a2, x2, __fmaf_rn(a0, x0, __fmul_rn(a1, x1)));
}

__device__ __forceinline__ void rotate(const float *Rt, float px, float py, float pz, float &rx,
                                       float &ry, float &rz) {
    rx = dot3(Rt[0], px, Rt[1], py, Rt[2], pz);
    ry = dot3(Rt[3], px, Rt[4], py, Rt[5], pz);
    rz = dot3(Rt[6], px, Rt[7], py, Rt[8], pz);
}

// w0*v0 + w1*v1 + w2*v2 + w3*v3 in the same contracted order:
// fma(w3, v3, fma(w2, v2, fma(w0, v0, w1*v1))).
__device__ __forceinline__ float bilerp(const float w[4], float v0, float v1, float v2, float v3) {
    return __fmaf_rn(w[3], v3, __fmaf_rn(w[2], v2, __fmaf_rn(w[0], v0, __fmul_rn(w[1], v1))));
}

// The tv-tap variant's tap k (1..3) samples at R_t·p + h·R_t[:, k-1]; the
// column offset is rounded on its own and then added, as the reference kernel
// stages h·R_t in shared memory before adding it (kplanes_tilted.cu:367-400).
__device__ __forceinline__ void tap_offsets(const float Rt[9], float h, float hc[9]) {
#pragma unroll
    for (int j = 0; j < 3; ++j)
#pragma unroll
        for (int i = 0; i < 3; ++i) hc[3 * j + i] = __fmul_rn(h, Rt[3 * i + j]);
}

__device__ __forceinline__ void tap_point(const float hc[9], int k, float rx, float ry, float rz,
                                          float &ax, float &ay, float &az) {
    if (k == 0) {
        ax = rx;
        ay = ry;
        az = rz;
    } else {
        ax = __fadd_rn(rx, hc[3 * (k - 1)]);
        ay = __fadd_rn(ry, hc[3 * (k - 1) + 1]);
        az = __fadd_rn(rz, hc[3 * (k - 1) + 2]);
    }
}

__device__ __forceinline__ void plane_coords(float rx, float ry, float rz, int p, float &gx,
                                             float &gy) {
    // p: 0 = XY (rx, ry), 1 = ZX (rz, rx), 2 = YZ (ry, rz).
    gx = p == 0 ? rx : (p == 1 ? rz : ry);
    gy = p == 0 ? ry : (p == 1 ? rx : rz);
}

// ── vectorised path: C == 4*L, L in {1, 2, 4, 8, 16, 32} ────────────────────
//
// Rotation-major grid: blockIdx.y is the rotation t and blockIdx.x picks a
// contiguous range of point tiles (a block's warps interleave within it; 4%
// faster in the backward than striding the whole range, measured on B200).
// Blocks are dispatched x-fastest, so the GPU works through the
// rotations one after another and only the three planes of about one rotation
// (and, backward, their three gradient planes) are live at a time: they stay
// in L2 instead of being re-read from (or, for the gradient reductions,
// read-modified-written in) HBM.

constexpr int kThreads = 256;

// Blocks per SM the backward's register budget is sized for (QC_KP_BWD_MINB
// overrides it at build time).
#ifndef QC_KP_BWD_MINB
#define QC_KP_BWD_MINB 2
#endif
constexpr int kBwdMinBlocks = QC_KP_BWD_MINB;

// Blocks per SM the forward's register budget is sized for: 5 (48 registers)
// measured 3% faster than 4 (64) and 7% faster than 6 (40, spilling) on B200;
// the four-tap forward keeps 4. QC_KP_FWD_MINB overrides it at build time.
#ifndef QC_KP_FWD_MINB
#define QC_KP_FWD_MINB 5
#endif
constexpr int kFwdMinBlocks = QC_KP_FWD_MINB;

// NT = 1: kplanes_tilted_fuse. NT = 4: kplanes_tilted_tv_fuse, the same
// interpolation at R_t·p and at the three offsets R_t·p + h·R_t[:, k-1], written
// to out[k] of a [4, B, T*C] output (tap 0 is bit-identical to NT = 1).
template <int L, int NT>
__device__ __forceinline__ void kpt_fwd_v4_body(const float *__restrict__ pts,
                                                const float *__restrict__ R,
                                                const float *__restrict__ grid,
                                                float *__restrict__ out, long long B, int T, int H,
                                                int W, float h) {
    constexpr int C = 4 * L;
    constexpr int G = 32 / L;  // points per warp tile
    const int t = blockIdx.y;
    float Rt[9];
#pragma unroll
    for (int k = 0; k < 9; ++k) Rt[k] = __ldg(R + 9 * t + k);
    float hc[9];
    if (NT > 1) tap_offsets(Rt, h, hc);

    const int lane = threadIdx.x & 31;
    const int grp = lane / L, c4 = 4 * (lane % L);
    const long long planeHWC = (long long)H * W * C;
    const float *g0 = grid + (long long)(3 * t) * planeHWC + c4;

    // this block's contiguous range of point tiles, its warps interleaved
    const long long n_tiles = (B + G - 1) / G;
    const long long per_block = (n_tiles + gridDim.x - 1) / gridDim.x;
    const long long tile_lo = (long long)blockIdx.x * per_block;
    const long long tile_hi = min(n_tiles, tile_lo + per_block);
    for (long long b0 = (tile_lo + (threadIdx.x >> 5)) * G; b0 < tile_hi * G;
         b0 += (long long)(blockDim.x >> 5) * G) {
        const long long b = b0 + grp;
        if (b >= B) continue;
        const float px = __ldg(pts + 3 * b), py = __ldg(pts + 3 * b + 1),
                    pz = __ldg(pts + 3 * b + 2);
        float rx, ry, rz;
        rotate(Rt, px, py, pz, rx, ry, rz);
#pragma unroll 1
        for (int k = 0; k < NT; ++k) {
            float ax, ay, az;
            tap_point(hc, k, rx, ry, rz, ax, ay, az);
            float4 s[3];
#pragma unroll
            for (int p = 0; p < 3; ++p) {
                float gx, gy;
                plane_coords(ax, ay, az, p, gx, gy);
                Tap tp = make_tap(gx, gy, H, W);
                check_tap(tp, H, W);
                const float *pc = g0 + p * planeHWC;
                const float4 v0 = ldg4(pc + tp.cell[0] * C), v1 = ldg4(pc + tp.cell[1] * C);
                const float4 v2 = ldg4(pc + tp.cell[2] * C), v3 = ldg4(pc + tp.cell[3] * C);
                s[p].x = bilerp(tp.w, v0.x, v1.x, v2.x, v3.x);
                s[p].y = bilerp(tp.w, v0.y, v1.y, v2.y, v3.y);
                s[p].z = bilerp(tp.w, v0.z, v1.z, v2.z, v3.z);
                s[p].w = bilerp(tp.w, v0.w, v1.w, v2.w, v3.w);
            }
            float4 o;
            o.x = __fmul_rn(__fmul_rn(s[0].x, s[1].x), s[2].x);
            o.y = __fmul_rn(__fmul_rn(s[0].y, s[1].y), s[2].y);
            o.z = __fmul_rn(__fmul_rn(s[0].z, s[1].z), s[2].z);
            o.w = __fmul_rn(__fmul_rn(s[0].w, s[1].w), s[2].w);
            __stcs(reinterpret_cast<float4 *>(out + ((long long)k * B + b) * (long long)(T * C) +
                                              t * C + c4),
                   o);
        }
    }
}

template <int L, int NT>
__global__ void __launch_bounds__(kThreads, NT == 1 ? kFwdMinBlocks : 4) kpt_fwd_v4_kernel(
    const float *__restrict__ pts, const float *__restrict__ R, const float *__restrict__ grid,
    float *__restrict__ out, long long B, int T, int H, int W, float h) {
    kpt_fwd_v4_body<L, NT>(pts, R, grid, out, B, T, H, W, h);
}

// Several levels of one multiscale encoding (planes of their own resolution,
// one rotation set) in one launch: blockIdx.z is the level. Blocks are
// dispatched level by level, so each level keeps the per-rotation L2
// residency of its own launch.
struct LevelTable {
    const float *grid[QC_KP_MAX_LEVELS];
    float *out[QC_KP_MAX_LEVELS];
    const float *gout[QC_KP_MAX_LEVELS];
    float *ggrid[QC_KP_MAX_LEVELS];
    int H[QC_KP_MAX_LEVELS], W[QC_KP_MAX_LEVELS];
};

template <int L>
__global__ void __launch_bounds__(kThreads, kFwdMinBlocks) kpt_fwd_levels_kernel(
    const float *__restrict__ pts, const float *__restrict__ R, const LevelTable tab, long long B,
    int T) {
    const int lv = blockIdx.z;
    kpt_fwd_v4_body<L, 1>(pts, R, tab.grid[lv], tab.out[lv], B, T, tab.H[lv], tab.W[lv], 0.f);
}


template <int L>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
    for (int off = L / 2; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    return v;
}

// Bilinear sample, ds/dix and ds/diy of one plane for this lane's 4 channels.
// (ds/dix = (1-ty)(v1-v0) + ty(v3-v2), ds/diy = (1-tx)(v2-v0) + tx(v3-v1); a
// clamped +1 corner only changes them where the border mask zeroes the result.)
template <int C>
__device__ __forceinline__ void sample_with_slopes(const float *pc, const Tap &tp, float4 &s,
                                                   float4 &dx, float4 &dy) {
    const float4 v0 = ldg4(pc + tp.cell[0] * C), v1 = ldg4(pc + tp.cell[1] * C);
    const float4 v2 = ldg4(pc + tp.cell[2] * C), v3 = ldg4(pc + tp.cell[3] * C);
    const float tx = tp.tx, ty = tp.ty;
    s = make_float4(bilerp(tp.w, v0.x, v1.x, v2.x, v3.x), bilerp(tp.w, v0.y, v1.y, v2.y, v3.y),
                    bilerp(tp.w, v0.z, v1.z, v2.z, v3.z), bilerp(tp.w, v0.w, v1.w, v2.w, v3.w));
    dx.x = (1.f - ty) * (v1.x - v0.x) + ty * (v3.x - v2.x);
    dx.y = (1.f - ty) * (v1.y - v0.y) + ty * (v3.y - v2.y);
    dx.z = (1.f - ty) * (v1.z - v0.z) + ty * (v3.z - v2.z);
    dx.w = (1.f - ty) * (v1.w - v0.w) + ty * (v3.w - v2.w);
    dy.x = (1.f - tx) * (v2.x - v0.x) + tx * (v3.x - v1.x);
    dy.y = (1.f - tx) * (v2.y - v0.y) + tx * (v3.y - v1.y);
    dy.z = (1.f - tx) * (v2.z - v0.z) + tx * (v3.z - v1.z);
    dy.w = (1.f - tx) * (v2.w - v0.w) + tx * (v3.w - v1.w);
}

// NT = 4 (tv taps): each tap's coordinate gradient dr_k reaches R_t twice —
// through R_t·p (dr_k ⊗ p, like the base op) and, for k >= 1, through the
// offset h·R_t[:, k-1] (h·dr_k into column k-1) — and reaches p through
// R_t^T dr_k; the taps' dr are summed before the point and R_t·p terms.
template <int L, int NT>
__device__ __forceinline__ void kpt_bwd_v4_body(
    const float *__restrict__ pts, const float *__restrict__ R, const float *__restrict__ grid,
    const float *__restrict__ gout, float *__restrict__ ggrid, float *__restrict__ gR,
    float *__restrict__ gpts, long long B, int T, int H, int W, int t0, float h) {
    constexpr int C = 4 * L;
    constexpr int G = 32 / L;
    constexpr int NWARP = kThreads / 32;
    __shared__ float sred[NWARP][9];
    const int t = t0 + blockIdx.y;
    float Rt[9];
#pragma unroll
    for (int k = 0; k < 9; ++k) Rt[k] = __ldg(R + 9 * t + k);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int grp = lane / L, lis = lane % L, c4 = 4 * lis;
    const long long planeHWC = (long long)H * W * C;
    const float *g0 = grid + (long long)(3 * t) * planeHWC + c4;
    float *gg0 = ggrid + (long long)(3 * t) * planeHWC + c4;
    float gr[9] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};  // this group's dL/dR_t
    float hc[9];
    if (NT > 1) tap_offsets(Rt, h, hc);

    // this block's contiguous range of point tiles, its warps interleaved
    const long long n_tiles = (B + G - 1) / G;
    const long long per_block = (n_tiles + gridDim.x - 1) / gridDim.x;
    const long long tile_lo = (long long)blockIdx.x * per_block;
    const long long tile_hi = min(n_tiles, tile_lo + per_block);
    for (long long b0 = (tile_lo + (threadIdx.x >> 5)) * G; b0 < tile_hi * G;
         b0 += (long long)(blockDim.x >> 5) * G) {
        const long long b_raw = b0 + grp;
        const bool active = b_raw < B;
        const long long b = active ? b_raw : B - 1;  // keep addresses valid; contributions zeroed
        const float px = __ldg(pts + 3 * b), py = __ldg(pts + 3 * b + 1),
                    pz = __ldg(pts + 3 * b + 2);
        float rx, ry, rz;
        rotate(Rt, px, py, pz, rx, ry, rz);
        float sx = 0.f, sy = 0.f, sz = 0.f;  // Σ over taps of dL/dr
#pragma unroll 1
        for (int kt = 0; kt < NT; ++kt) {
        float ax, ay, az;
        tap_point(hc, kt, rx, ry, rz, ax, ay, az);
        float4 go = __ldcs(reinterpret_cast<const float4 *>(
            gout + ((long long)kt * B + b) * (long long)(T * C) + t * C + c4));
        if (!active) go = make_float4(0.f, 0.f, 0.f, 0.f);

        Tap tap[3];
        float4 s[3], dx[3], dy[3];
#pragma unroll
        for (int p = 0; p < 3; ++p) {
            float gx, gy;
            plane_coords(ax, ay, az, p, gx, gy);
            tap[p] = make_tap(gx, gy, H, W);
            check_tap(tap[p], H, W);
            sample_with_slopes<C>(g0 + p * planeHWC, tap[p], s[p], dx[p], dy[p]);
        }

        float dgx[3], dgy[3];
#pragma unroll
        for (int p = 0; p < 3; ++p) {
            const float4 sa = s[(p + 1) % 3], sb = s[(p + 2) % 3];
            float4 other;
            other.x = sa.x * sb.x * go.x;
            other.y = sa.y * sb.y * go.y;
            other.z = sa.z * sb.z * go.z;
            other.w = sa.w * sb.w * go.w;
            float *gpc = gg0 + p * planeHWC;
            if (active) {
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const float wk = tap[p].w[k];
                    if (wk != 0.f)
                        red_add_v4(gpc + tap[p].cell[k] * C,
                                   make_float4(other.x * wk, other.y * wk, other.z * wk, other.w * wk));
                }
            }
            dgx[p] = other.x * dx[p].x + other.y * dx[p].y + other.z * dx[p].z + other.w * dx[p].w;
            dgy[p] = other.x * dy[p].x + other.y * dy[p].y + other.z * dy[p].z + other.w * dy[p].w;
        }
#pragma unroll
        for (int p = 0; p < 3; ++p) {
            dgx[p] = group_sum<L>(dgx[p]);
            dgy[p] = group_sum<L>(dgy[p]);
        }
        // Back to the rotated point: XY=(rx,ry), ZX=(rz,rx), YZ=(ry,rz).
        const float drx = dgx[0] * tap[0].gxm + dgy[1] * tap[1].gym;
        const float dry = dgy[0] * tap[0].gym + dgx[2] * tap[2].gxm;
        const float drz = dgx[1] * tap[1].gxm + dgy[2] * tap[2].gym;
        if (NT == 1) {
            sx = drx;
            sy = dry;
            sz = drz;
        } else {
            sx += drx;
            sy += dry;
            sz += drz;
            if (kt > 0 && active && lis == 0) {
                // the offset h·R_t[:, kt-1]: dL/dR_t[i, kt-1] += h · dr_i
                gr[kt - 1] += h * drx;
                gr[3 + kt - 1] += h * dry;
                gr[6 + kt - 1] += h * drz;
            }
        }
        }  // taps
        if (active && lis == 0) {
            // dL/dp += R_t^T dr (the point's T rotations run in different blocks)
            atomicAdd(gpts + 3 * b, Rt[0] * sx + Rt[3] * sy + Rt[6] * sz);
            atomicAdd(gpts + 3 * b + 1, Rt[1] * sx + Rt[4] * sy + Rt[7] * sz);
            atomicAdd(gpts + 3 * b + 2, Rt[2] * sx + Rt[5] * sy + Rt[8] * sz);
            // dL/dR_t[i, j] += dr_i * p_j, kept in registers
            gr[0] += sx * px; gr[1] += sx * py; gr[2] += sx * pz;
            gr[3] += sy * px; gr[4] += sy * py; gr[5] += sy * pz;
            gr[6] += sz * px; gr[7] += sz * py; gr[8] += sz * pz;
        }
    }

    // grad_R: groups of the warp (lanes 0, L, 2L, ...) then warps of the block,
    // then one reduction per entry per block.
#pragma unroll
    for (int k = 0; k < 9; ++k) {
        float v = gr[k];
#pragma unroll
        for (int off = L; off < 32; off <<= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
        if (lane == 0) sred[warp][k] = v;
    }
    __syncthreads();
    if (threadIdx.x < 9) {
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < NWARP; ++w) v += sred[w][threadIdx.x];
        if (v != 0.f) atomicAdd(gR + 9 * t + threadIdx.x, v);
    }
}

template <int L, int NT>
__global__ void __launch_bounds__(kThreads, kBwdMinBlocks) kpt_bwd_v4_kernel(
    const float *__restrict__ pts, const float *__restrict__ R, const float *__restrict__ grid,
    const float *__restrict__ gout, float *__restrict__ ggrid, float *__restrict__ gR,
    float *__restrict__ gpts, long long B, int T, int H, int W, int t0, float h) {
    kpt_bwd_v4_body<L, NT>(pts, R, grid, gout, ggrid, gR, gpts, B, T, H, W, t0, h);
}

// Backward of kpt_fwd_levels_kernel: blockIdx.z is the level; gR and gpts
// take the sum over the levels (they share the points and the rotations).
template <int L>
__global__ void __launch_bounds__(kThreads, kBwdMinBlocks) kpt_bwd_levels_kernel(
    const float *__restrict__ pts, const float *__restrict__ R, const LevelTable tab,
    float *__restrict__ gR, float *__restrict__ gpts, long long B, int T) {
    const int lv = blockIdx.z;
    kpt_bwd_v4_body<L, 1>(pts, R, tab.grid[lv], tab.gout[lv], tab.ggrid[lv], gR, gpts, B, T,
                          tab.H[lv], tab.W[lv], 0, 0.f);
}


// ── generic path: any C (scalar channels, one warp per point) ─────────────

template <int NT>
__global__ void __launch_bounds__(kThreads) kpt_fwd_generic_kernel(
    const float *__restrict__ pts, const float *__restrict__ R, const float *__restrict__ grid,
    float *__restrict__ out, long long B, int T, int C, int H, int W, float h) {
    extern __shared__ float sR[];
    for (int i = threadIdx.x; i < T * 9; i += blockDim.x) sR[i] = R[i];
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const long long planeHWC = (long long)H * W * C;
    const long long warp0 = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const long long nwarps = ((long long)gridDim.x * blockDim.x) >> 5;
    for (long long b = warp0; b < B; b += nwarps) {
        const float px = pts[3 * b], py = pts[3 * b + 1], pz = pts[3 * b + 2];
        for (int t = 0; t < T; ++t) {
            float rx, ry, rz;
            rotate(sR + 9 * t, px, py, pz, rx, ry, rz);
            float hc[9];
            if (NT > 1) tap_offsets(sR + 9 * t, h, hc);
            for (int k = 0; k < NT; ++k) {
                float ax, ay, az;
                tap_point(hc, k, rx, ry, rz, ax, ay, az);
                Tap tp[3];
#pragma unroll
                for (int p = 0; p < 3; ++p) {
                    float gx, gy;
                    plane_coords(ax, ay, az, p, gx, gy);
                    tp[p] = make_tap(gx, gy, H, W);
                    check_tap(tp[p], H, W);
                }
                for (int c = lane; c < C; c += 32) {
                    float s[3];
#pragma unroll
                    for (int p = 0; p < 3; ++p) {
                        const float *pc = grid + (long long)(3 * t + p) * planeHWC + c;
                        s[p] = bilerp(tp[p].w, __ldg(pc + (long long)tp[p].cell[0] * C),
                                      __ldg(pc + (long long)tp[p].cell[1] * C),
                                      __ldg(pc + (long long)tp[p].cell[2] * C),
                                      __ldg(pc + (long long)tp[p].cell[3] * C));
                    }
                    out[((long long)k * B + b) * (long long)(T * C) + (long long)t * C + c] =
                        __fmul_rn(__fmul_rn(s[0], s[1]), s[2]);
                }
            }
        }
    }
}

template <int NT>
__global__ void __launch_bounds__(kThreads) kpt_bwd_generic_kernel(
    const float *__restrict__ pts, const float *__restrict__ R, const float *__restrict__ grid,
    const float *__restrict__ gout, float *__restrict__ ggrid, float *__restrict__ gR,
    float *__restrict__ gpts, long long B, int T, int C, int H, int W, int t0, int t1, float h) {
    extern __shared__ float smem[];
    float *sR = smem;
    float *sgR = smem + 9 * T;
    for (int i = threadIdx.x; i < T * 9; i += blockDim.x) {
        sR[i] = R[i];
        sgR[i] = 0.f;
    }
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const long long planeHWC = (long long)H * W * C;
    const long long warp0 = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const long long nwarps = ((long long)gridDim.x * blockDim.x) >> 5;
    for (long long b = warp0; b < B; b += nwarps) {
        const float px = pts[3 * b], py = pts[3 * b + 1], pz = pts[3 * b + 2];
        float gpx = 0.f, gpy = 0.f, gpz = 0.f;
        for (int t = t0; t < t1; ++t) {
            const float *Rt = sR + 9 * t;
            float rx, ry, rz;
            rotate(Rt, px, py, pz, rx, ry, rz);
            float hc[9];
            if (NT > 1) tap_offsets(Rt, h, hc);
            for (int kt = 0; kt < NT; ++kt) {
            float ax, ay, az;
            tap_point(hc, kt, rx, ry, rz, ax, ay, az);
            Tap tp[3];
#pragma unroll
            for (int p = 0; p < 3; ++p) {
                float gx, gy;
                plane_coords(ax, ay, az, p, gx, gy);
                tp[p] = make_tap(gx, gy, H, W);
                    check_tap(tp[p], H, W);
            }
            float dgx[3] = {0.f, 0.f, 0.f}, dgy[3] = {0.f, 0.f, 0.f};
            for (int c = lane; c < C; c += 32) {
                const float go = gout[((long long)kt * B + b) * (long long)(T * C) + (long long)t * C + c];
                float v[3][4], s[3];
#pragma unroll
                for (int p = 0; p < 3; ++p) {
                    const float *pc = grid + (long long)(3 * t + p) * planeHWC + c;
#pragma unroll
                    for (int k = 0; k < 4; ++k) v[p][k] = __ldg(pc + (long long)tp[p].cell[k] * C);
                    s[p] = bilerp(tp[p].w, v[p][0], v[p][1], v[p][2], v[p][3]);
                }
#pragma unroll
                for (int p = 0; p < 3; ++p) {
                    const float other = s[(p + 1) % 3] * s[(p + 2) % 3] * go;
                    float *gpc = ggrid + (long long)(3 * t + p) * planeHWC + c;
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const float val = other * tp[p].w[k];
                        if (val != 0.f) atomicAdd(gpc + (long long)tp[p].cell[k] * C, val);
                    }
                    const float tx = tp[p].tx, ty = tp[p].ty;
                    dgx[p] += other * ((1.f - ty) * (v[p][1] - v[p][0]) + ty * (v[p][3] - v[p][2]));
                    dgy[p] += other * ((1.f - tx) * (v[p][2] - v[p][0]) + tx * (v[p][3] - v[p][1]));
                }
            }
#pragma unroll
            for (int p = 0; p < 3; ++p) {
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) {
                    dgx[p] += __shfl_xor_sync(0xffffffffu, dgx[p], off);
                    dgy[p] += __shfl_xor_sync(0xffffffffu, dgy[p], off);
                }
            }
            const float drx = dgx[0] * tp[0].gxm + dgy[1] * tp[1].gym;
            const float dry = dgy[0] * tp[0].gym + dgx[2] * tp[2].gxm;
            const float drz = dgx[1] * tp[1].gxm + dgy[2] * tp[2].gym;
            gpx += Rt[0] * drx + Rt[3] * dry + Rt[6] * drz;
            gpy += Rt[1] * drx + Rt[4] * dry + Rt[7] * drz;
            gpz += Rt[2] * drx + Rt[5] * dry + Rt[8] * drz;
            if (lane == 0) {
                float *sg = sgR + 9 * t;
                atomicAdd(sg + 0, drx * px);
                atomicAdd(sg + 1, drx * py);
                atomicAdd(sg + 2, drx * pz);
                atomicAdd(sg + 3, dry * px);
                atomicAdd(sg + 4, dry * py);
                atomicAdd(sg + 5, dry * pz);
                atomicAdd(sg + 6, drz * px);
                atomicAdd(sg + 7, drz * py);
                atomicAdd(sg + 8, drz * pz);
                if (NT > 1 && kt > 0) {
                    atomicAdd(sg + kt - 1, h * drx);
                    atomicAdd(sg + 3 + kt - 1, h * dry);
                    atomicAdd(sg + 6 + kt - 1, h * drz);
                }
            }
            }  // taps
        }
        if (lane == 0) {
            gpts[3 * b] += gpx;
            gpts[3 * b + 1] += gpy;
            gpts[3 * b + 2] += gpz;
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < T * 9; i += blockDim.x)
        if (sgR[i] != 0.f) atomicAdd(gR + i, sgR[i]);
}

// ── plane layout conversion [P, C, HW] <-> [P, HW, C] ─────────────────────

constexpr int kTT = 32;  // transpose tile

// dst[p][j][i] = src[p][i][j] for a [P, R, S] -> [P, S, R] transpose.
__global__ void __launch_bounds__(kTT * 8) transpose_kernel(const float *__restrict__ src,
                                                          float *__restrict__ dst, int Rn, int Sn) {
    __shared__ float tile[kTT][kTT + 1];
    const long long base = (long long)blockIdx.z * Rn * Sn;
    const int i0 = blockIdx.y * kTT, j0 = blockIdx.x * kTT;
    for (int k = threadIdx.y; k < kTT; k += 8) {
        const int i = i0 + k, j = j0 + threadIdx.x;
        if (i < Rn && j < Sn) tile[k][threadIdx.x] = __ldcs(src + base + (long long)i * Sn + j);
    }
    __syncthreads();
    for (int k = threadIdx.y; k < kTT; k += 8) {
        const int j = j0 + k, i = i0 + threadIdx.x;
        if (i < Rn && j < Sn) dst[base + (long long)j * Rn + i] = tile[threadIdx.x][k];
    }
}

// Fast form for R % 4 == 0, S % 4 == 0 and 16-byte aligned pointers: tiles of
// 32 rows (channels) × 128 columns (cells), 16-byte loads and stores on both
// sides. The shared tile keeps element (c, x) at c·132 + (x ^ 4·((c/4) % 8)):
// float4 groups stay together for the row-wise side, and the column-wise side
// (lanes reading 4 consecutive rows of 8 columns) hits 32 distinct banks.
constexpr int kTC = 32, kTS = 128, kTStride = kTS + 4;

__device__ __forceinline__ int tswz(int c, int x) {
    return c * kTStride + (x ^ (((c >> 2) & 7) << 2));
}

// TO_CL: [P, R, S] -> [P, S, R]; otherwise [P, S, R] -> [P, R, S].
template <bool TO_CL>
__global__ void __launch_bounds__(256) transpose_tile_kernel(const float *__restrict__ src,
                                                            float *__restrict__ dst, int R, int S) {
    __shared__ __align__(16) float tile[kTC * kTStride];
    const long long base = (long long)blockIdx.z * R * S;
    const int s0 = blockIdx.x * kTS, c0 = blockIdx.y * kTC;
    const int t = threadIdx.x;
    if (TO_CL) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int f = t + 256 * k;
            const int c = f >> 5, x = (f & 31) * 4;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (c0 + c < R && s0 + x < S)
                v = __ldcs(reinterpret_cast<const float4 *>(src + base + (long long)(c0 + c) * S + s0 + x));
            *reinterpret_cast<float4 *>(&tile[tswz(c, x)]) = v;
        }
        __syncthreads();
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int f = t + 256 * k;
            const int j = f >> 3, c = 4 * (f & 7);
            if (s0 + j < S && c0 + c < R) {
                const float4 v = make_float4(tile[tswz(c, j)], tile[tswz(c + 1, j)],
                                             tile[tswz(c + 2, j)], tile[tswz(c + 3, j)]);
                *reinterpret_cast<float4 *>(dst + base + (long long)(s0 + j) * R + c0 + c) = v;
            }
        }
    } else {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int f = t + 256 * k;
            const int j = f >> 3, c = 4 * (f & 7);
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (s0 + j < S && c0 + c < R)
                v = __ldcs(reinterpret_cast<const float4 *>(src + base + (long long)(s0 + j) * R + c0 + c));
            tile[tswz(c, j)] = v.x;
            tile[tswz(c + 1, j)] = v.y;
            tile[tswz(c + 2, j)] = v.z;
            tile[tswz(c + 3, j)] = v.w;
        }
        __syncthreads();
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int f = t + 256 * k;
            const int c = f >> 5, x = (f & 31) * 4;
            if (c0 + c < R && s0 + x < S)
                *reinterpret_cast<float4 *>(dst + base + (long long)(c0 + c) * S + s0 + x) =
                    *reinterpret_cast<const float4 *>(&tile[tswz(c, x)]);
        }
    }
}

int launch_transpose_fast(const float *src, float *dst, int P, int R, int S, bool to_cl,
                          cudaStream_t stream) {
    const dim3 grid((S + kTS - 1) / kTS, (R + kTC - 1) / kTC, P);
    QC_RETURN_IF(grid.y > 65535, QC_ERR_INVALID_ARGUMENT, "transpose: channel extent too large");
    if (to_cl)
        transpose_tile_kernel<true><<<grid, 256, 0, stream>>>(src, dst, R, S);
    else
        transpose_tile_kernel<false><<<grid, 256, 0, stream>>>(src, dst, R, S);
    QC_CHECK_LAUNCH("transpose_tile_kernel launch");
    return 0;
}

int launch_transpose(const float *src, float *dst, int P, int Rn, int Sn, cudaStream_t stream) {
    QC_RETURN_IF(P < 0 || Rn < 0 || Sn < 0, QC_ERR_INVALID_ARGUMENT, "transpose: negative shape");
    if ((long long)P * Rn * Sn == 0) return 0;
    QC_RETURN_IF(src == nullptr || dst == nullptr, QC_ERR_INVALID_ARGUMENT, "transpose: null pointer");
    QC_RETURN_IF(P > 65535, QC_ERR_INVALID_ARGUMENT, "transpose: more than 65535 planes");
    const dim3 grid((Sn + kTT - 1) / kTT, (Rn + kTT - 1) / kTT, P);
    QC_RETURN_IF(grid.y > 65535, QC_ERR_INVALID_ARGUMENT, "transpose: row extent too large");
    transpose_kernel<<<grid, dim3(kTT, 8), 0, stream>>>(src, dst, Rn, Sn);
    QC_CHECK_LAUNCH("transpose_kernel launch");
    return 0;
}

// ── launch plumbing ───────────────────────────────────────────────────────

int check_shapes(const char *who, long B, int T, int C, int H, int W) {
    QC_RETURN_IF(B < 0 || T < 0 || C < 0 || H < 0 || W < 0, QC_ERR_INVALID_ARGUMENT,
                 "%s: negative shape (B=%ld T=%d C=%d H=%d W=%d)", who, B, T, C, H, W);
    QC_RETURN_IF((long long)C * H * W >= (1LL << 31), QC_ERR_INVALID_ARGUMENT,
                 "%s: C*H*W must be < 2^31 (32-bit per-plane offsets)", who);
    QC_RETURN_IF(T > 4096, QC_ERR_INVALID_ARGUMENT, "%s: T=%d exceeds 4096", who, T);
    return 0;
}

int grid_size(long long work_warps, int *grid) {
    int sms = 0;
    if (int st = device_sm_count(&sms)) return st;
    const long long warps_per_block = kThreads / 32;
    long long blocks = (work_warps + warps_per_block - 1) / warps_per_block;
    const long long cap = (long long)sms * 64;  // persistent: enough waves to balance
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    *grid = (int)blocks;
    return 0;
}

// Blocks per rotation for the rotation-major grids: about two waves of
// resident blocks (so that one rotation's blocks fill the GPU before the next
// rotation starts), never more than the point tiles.
int rotation_grid_x(long long work_warps, int blocks_per_sm, int *gx) {
    int sms = 0;
    if (int st = device_sm_count(&sms)) return st;
    const long long warps_per_block = kThreads / 32;
    long long need = (work_warps + warps_per_block - 1) / warps_per_block;
    long long cap = 2LL * sms * blocks_per_sm;
    long long x = need < cap ? need : cap;
    if (x < 1) x = 1;
    *gx = (int)x;
    return 0;
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

template <int L, int NT>
int fwd_v4(const float *pts, const float *R, const float *grid, float *out, long long B, int T,
           int H, int W, float h, cudaStream_t stream) {
    constexpr int G = 32 / L;
    int gx = 0;
    if (int st = rotation_grid_x((B + G - 1) / G, 8, &gx)) return st;
    QC_RETURN_IF(T > 65535, QC_ERR_INVALID_ARGUMENT, "kplanes: T=%d exceeds 65535", T);
    kpt_fwd_v4_kernel<L, NT><<<dim3(gx, T), kThreads, 0, stream>>>(pts, R, grid, out, B, T, H, W, h);
    QC_CHECK_LAUNCH("kpt_fwd_v4_kernel launch");
    return 0;
}

template <int L, int NT>
int bwd_v4(const float *pts, const float *R, const float *grid, const float *gout, float *ggrid,
           float *gR, float *gpts, long long B, int T, int H, int W, int t0, int t1, float h,
           cudaStream_t stream) {
    constexpr int G = 32 / L;
    int gx = 0;
    if (int st = rotation_grid_x((B + G - 1) / G, kBwdMinBlocks, &gx)) return st;
    QC_RETURN_IF(t1 - t0 > 65535, QC_ERR_INVALID_ARGUMENT, "kplanes: %d rotations exceed 65535",
                 t1 - t0);
    kpt_bwd_v4_kernel<L, NT><<<dim3(gx, t1 - t0), kThreads, 0, stream>>>(
        pts, R, grid, gout, ggrid, gR, gpts, B, T, H, W, t0, h);
    QC_CHECK_LAUNCH("kpt_bwd_v4_kernel launch");
    return 0;
}

template <int L>
int fwd_levels(const float *pts, const float *R, const LevelTable &tab, int n, long long B, int T,
               cudaStream_t stream) {
    constexpr int G = 32 / L;
    int gx = 0;
    if (int st = rotation_grid_x((B + G - 1) / G, 8, &gx)) return st;
    QC_RETURN_IF(T > 65535, QC_ERR_INVALID_ARGUMENT, "kplanes: T=%d exceeds 65535", T);
    kpt_fwd_levels_kernel<L><<<dim3(gx, T, n), kThreads, 0, stream>>>(pts, R, tab, B, T);
    QC_CHECK_LAUNCH("kpt_fwd_levels_kernel launch");
    return 0;
}

template <int L>
int bwd_levels(const float *pts, const float *R, const LevelTable &tab, int n, float *gR,
               float *gpts, long long B, int T, cudaStream_t stream) {
    constexpr int G = 32 / L;
    int gx = 0;
    if (int st = rotation_grid_x((B + G - 1) / G, kBwdMinBlocks, &gx)) return st;
    QC_RETURN_IF(T > 65535, QC_ERR_INVALID_ARGUMENT, "kplanes: T=%d exceeds 65535", T);
    kpt_bwd_levels_kernel<L><<<dim3(gx, T, n), kThreads, 0, stream>>>(pts, R, tab, gR, gpts, B, T);
    QC_CHECK_LAUNCH("kpt_bwd_levels_kernel launch");
    return 0;
}

template <int NT>
int forward(const char *who, const float *d_pts, const float *d_R, const float *d_grid,
            float *d_out, long B, int T, int C, int H, int W, float h, cudaStream_t stream) {
    QC_NVTX(NT == 1 ? "quantem::kplanes_fwd" : "quantem::kplanes_tv_fwd");
    if (int st = check_shapes(who, B, T, C, H, W)) return st;
    if (B == 0 || T == 0 || C == 0) return 0;
    QC_RETURN_IF(H == 0 || W == 0, QC_ERR_INVALID_ARGUMENT, "%s: empty plane", who);
    QC_RETURN_IF(!d_pts || !d_R || !d_grid || !d_out, QC_ERR_INVALID_ARGUMENT, "%s: null pointer",
                 who);
    const bool vec = (C % 4 == 0) && C <= 128 && aligned16(d_grid) && aligned16(d_out);
    if (vec) {
        switch (C / 4) {
            case 1: return fwd_v4<1, NT>(d_pts, d_R, d_grid, d_out, B, T, H, W, h, stream);
            case 2: return fwd_v4<2, NT>(d_pts, d_R, d_grid, d_out, B, T, H, W, h, stream);
            case 4: return fwd_v4<4, NT>(d_pts, d_R, d_grid, d_out, B, T, H, W, h, stream);
            case 8: return fwd_v4<8, NT>(d_pts, d_R, d_grid, d_out, B, T, H, W, h, stream);
            case 16: return fwd_v4<16, NT>(d_pts, d_R, d_grid, d_out, B, T, H, W, h, stream);
            case 32: return fwd_v4<32, NT>(d_pts, d_R, d_grid, d_out, B, T, H, W, h, stream);
            default: break;
        }
    }
    int blocks = 0;
    if (int st = grid_size(B, &blocks)) return st;
    kpt_fwd_generic_kernel<NT><<<blocks, kThreads, 9 * T * sizeof(float), stream>>>(
        d_pts, d_R, d_grid, d_out, B, T, C, H, W, h);
    QC_CHECK_LAUNCH("kpt_fwd_generic_kernel launch");
    return 0;
}

template <int NT>
int backward(const char *who, const float *d_pts, const float *d_R, const float *d_grid,
             const float *d_gout, float *d_ggrid, float *d_gR, float *d_gpts, long B, int T,
             int C, int H, int W, int t_begin, int t_end, float h, cudaStream_t stream) {
    QC_NVTX(NT == 1 ? "quantem::kplanes_bwd" : "quantem::kplanes_tv_bwd");
    if (int st = check_shapes(who, B, T, C, H, W)) return st;
    QC_RETURN_IF(t_begin < 0 || t_end > T || t_begin > t_end, QC_ERR_INVALID_ARGUMENT,
                 "%s: rotations [%d, %d) outside [0, %d)", who, t_begin, t_end, T);
    if (B == 0 || t_begin == t_end || C == 0) return 0;
    QC_RETURN_IF(H == 0 || W == 0, QC_ERR_INVALID_ARGUMENT, "%s: empty plane", who);
    QC_RETURN_IF(!d_pts || !d_R || !d_grid || !d_gout || !d_ggrid || !d_gR || !d_gpts,
                 QC_ERR_INVALID_ARGUMENT, "%s: null pointer", who);
    const bool vec = (C % 4 == 0) && C <= 128 && aligned16(d_grid) && aligned16(d_gout) &&
                     aligned16(d_ggrid);
    const int t0 = t_begin, t1 = t_end;
    if (vec) {
        switch (C / 4) {
            case 1: return bwd_v4<1, NT>(d_pts, d_R, d_grid, d_gout, d_ggrid, d_gR, d_gpts, B, T, H, W, t0, t1, h, stream);
            case 2: return bwd_v4<2, NT>(d_pts, d_R, d_grid, d_gout, d_ggrid, d_gR, d_gpts, B, T, H, W, t0, t1, h, stream);
            case 4: return bwd_v4<4, NT>(d_pts, d_R, d_grid, d_gout, d_ggrid, d_gR, d_gpts, B, T, H, W, t0, t1, h, stream);
            case 8: return bwd_v4<8, NT>(d_pts, d_R, d_grid, d_gout, d_ggrid, d_gR, d_gpts, B, T, H, W, t0, t1, h, stream);
            case 16: return bwd_v4<16, NT>(d_pts, d_R, d_grid, d_gout, d_ggrid, d_gR, d_gpts, B, T, H, W, t0, t1, h, stream);
            case 32: return bwd_v4<32, NT>(d_pts, d_R, d_grid, d_gout, d_ggrid, d_gR, d_gpts, B, T, H, W, t0, t1, h, stream);
            default: break;
        }
    }
    int blocks = 0;
    if (int st = grid_size(B, &blocks)) return st;
    kpt_bwd_generic_kernel<NT><<<blocks, kThreads, 18 * T * sizeof(float), stream>>>(
        d_pts, d_R, d_grid, d_gout, d_ggrid, d_gR, d_gpts, B, T, C, H, W, t0, t1, h);
    QC_CHECK_LAUNCH("kpt_bwd_generic_kernel launch");
    return 0;
}

// Checks of the level tables (host arrays of device pointers and sizes).
int check_levels(const char *who, int n, const void *a, const void *b, const int *H, const int *W,
                 long B, int T, int C) {
    QC_RETURN_IF(n < 1 || n > QC_KP_MAX_LEVELS, QC_ERR_INVALID_ARGUMENT,
                 "%s: %d levels, need 1..%d", who, n, QC_KP_MAX_LEVELS);
    QC_RETURN_IF(a == nullptr || b == nullptr || H == nullptr || W == nullptr,
                 QC_ERR_INVALID_ARGUMENT, "%s: null level table", who);
    for (int l = 0; l < n; ++l)
        if (int st = check_shapes(who, B, T, C, H[l], W[l])) return st;
    return 0;
}

int forward_levels(const float *d_pts, const float *d_R, int n, const float *const *grids,
                   float *const *outs, const int *H, const int *W, long B, int T, int C,
                   cudaStream_t stream) {
    QC_NVTX("quantem::kplanes_fwd_levels");
    const char *who = "kplanes_tilted_fuse_levels_cuda";
    if (int st = check_levels(who, n, grids, outs, H, W, B, T, C)) return st;
    if (B == 0 || T == 0 || C == 0) return 0;
    bool vec = (C % 4 == 0) && C <= 128;
    for (int l = 0; l < n; ++l) {
        QC_RETURN_IF(H[l] == 0 || W[l] == 0, QC_ERR_INVALID_ARGUMENT, "%s: empty plane at level %d", who, l);
        QC_RETURN_IF(!grids[l] || !outs[l], QC_ERR_INVALID_ARGUMENT, "%s: null pointer at level %d", who, l);
        vec = vec && aligned16(grids[l]) && aligned16(outs[l]);
    }
    QC_RETURN_IF(!d_pts || !d_R, QC_ERR_INVALID_ARGUMENT, "%s: null pointer", who);
    if (!vec) {  // per-level launches of the general kernels
        for (int l = 0; l < n; ++l)
            if (int st = forward<1>(who, d_pts, d_R, grids[l], outs[l], B, T, C, H[l], W[l], 0.f, stream))
                return st;
        return 0;
    }
    LevelTable tab{};
    for (int l = 0; l < n; ++l) {
        tab.grid[l] = grids[l];
        tab.out[l] = outs[l];
        tab.H[l] = H[l];
        tab.W[l] = W[l];
    }
    switch (C / 4) {
        case 1: return fwd_levels<1>(d_pts, d_R, tab, n, B, T, stream);
        case 2: return fwd_levels<2>(d_pts, d_R, tab, n, B, T, stream);
        case 4: return fwd_levels<4>(d_pts, d_R, tab, n, B, T, stream);
        case 8: return fwd_levels<8>(d_pts, d_R, tab, n, B, T, stream);
        case 16: return fwd_levels<16>(d_pts, d_R, tab, n, B, T, stream);
        case 32: return fwd_levels<32>(d_pts, d_R, tab, n, B, T, stream);
        default: break;
    }
    for (int l = 0; l < n; ++l)
        if (int st = forward<1>(who, d_pts, d_R, grids[l], outs[l], B, T, C, H[l], W[l], 0.f, stream))
            return st;
    return 0;
}

int backward_levels(const float *d_pts, const float *d_R, int n, const float *const *grids,
                    const float *const *gouts, float *const *ggrids, const int *H, const int *W,
                    float *d_gR, float *d_gpts, long B, int T, int C, cudaStream_t stream) {
    QC_NVTX("quantem::kplanes_bwd_levels");
    const char *who = "kplanes_tilted_fuse_levels_grad_cuda";
    if (int st = check_levels(who, n, grids, gouts, H, W, B, T, C)) return st;
    QC_RETURN_IF(ggrids == nullptr, QC_ERR_INVALID_ARGUMENT, "%s: null level table", who);
    if (B == 0 || T == 0 || C == 0) return 0;
    bool vec = (C % 4 == 0) && C <= 128;
    for (int l = 0; l < n; ++l) {
        QC_RETURN_IF(H[l] == 0 || W[l] == 0, QC_ERR_INVALID_ARGUMENT, "%s: empty plane at level %d", who, l);
        QC_RETURN_IF(!grids[l] || !gouts[l] || !ggrids[l], QC_ERR_INVALID_ARGUMENT,
                     "%s: null pointer at level %d", who, l);
        vec = vec && aligned16(grids[l]) && aligned16(gouts[l]) && aligned16(ggrids[l]);
    }
    QC_RETURN_IF(!d_pts || !d_R || !d_gR || !d_gpts, QC_ERR_INVALID_ARGUMENT, "%s: null pointer", who);
    const bool fast = vec && (C / 4 == 1 || C / 4 == 2 || C / 4 == 4 || C / 4 == 8 || C / 4 == 16 ||
                              C / 4 == 32);
    if (!fast) {
        for (int l = 0; l < n; ++l)
            if (int st = backward<1>(who, d_pts, d_R, grids[l], gouts[l], ggrids[l], d_gR, d_gpts, B, T, C,
                                     H[l], W[l], 0, T, 0.f, stream))
                return st;
        return 0;
    }
    LevelTable tab{};
    for (int l = 0; l < n; ++l) {
        tab.grid[l] = grids[l];
        tab.gout[l] = gouts[l];
        tab.ggrid[l] = ggrids[l];
        tab.H[l] = H[l];
        tab.W[l] = W[l];
    }
    switch (C / 4) {
        case 1: return bwd_levels<1>(d_pts, d_R, tab, n, d_gR, d_gpts, B, T, stream);
        case 2: return bwd_levels<2>(d_pts, d_R, tab, n, d_gR, d_gpts, B, T, stream);
        case 4: return bwd_levels<4>(d_pts, d_R, tab, n, d_gR, d_gpts, B, T, stream);
        case 8: return bwd_levels<8>(d_pts, d_R, tab, n, d_gR, d_gpts, B, T, stream);
        case 16: return bwd_levels<16>(d_pts, d_R, tab, n, d_gR, d_gpts, B, T, stream);
        default: return bwd_levels<32>(d_pts, d_R, tab, n, d_gR, d_gpts, B, T, stream);
    }
}

}  // namespace kp

int kp_fault_word(unsigned int *word, int clear) {
    unsigned int w = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&w, kp::g_kp_fault_word, sizeof(w));
    if (e == cudaSuccess && clear) {
        const unsigned int zero = 0;
        e = cudaMemcpyToSymbol(kp::g_kp_fault_word, &zero, sizeof(zero));
    }
    QC_CUDA_TRY(e, "cudaMemcpyFromSymbol(K-Planes fault word)");
    *word = w;
    return 0;
}

}  // namespace qc

extern "C" {

int kplanes_tilted_fuse_cuda(const float *d_pts, const float *d_R, const float *d_grid,
                             float *d_out, long B, int T, int C, int H, int W,
                             cudaStream_t stream) {
    return qc::kp::forward<1>("kplanes_tilted_fuse_cuda", d_pts, d_R, d_grid, d_out, B, T, C, H,
                              W, 0.f, stream);
}

int kplanes_tilted_tv_fuse_cuda(const float *d_pts, const float *d_R, const float *d_grid,
                                float *d_out, long B, int T, int C, int H, int W, float h,
                                cudaStream_t stream) {
    return qc::kp::forward<4>("kplanes_tilted_tv_fuse_cuda", d_pts, d_R, d_grid, d_out, B, T, C,
                              H, W, h, stream);
}

int kplanes_tilted_fuse_grad_rotations_cuda(const float *d_pts, const float *d_R,
                                            const float *d_grid, const float *d_gout,
                                            float *d_ggrid, float *d_gR, float *d_gpts, long B,
                                            int T, int C, int H, int W, int t_begin, int t_end,
                                            cudaStream_t stream) {
    return qc::kp::backward<1>("kplanes_tilted_fuse_grad_cuda", d_pts, d_R, d_grid, d_gout,
                               d_ggrid, d_gR, d_gpts, B, T, C, H, W, t_begin, t_end, 0.f, stream);
}

int kplanes_tilted_tv_fuse_grad_cuda(const float *d_pts, const float *d_R, const float *d_grid,
                                     const float *d_gout, float *d_ggrid, float *d_gR,
                                     float *d_gpts, long B, int T, int C, int H, int W, float h,
                                     cudaStream_t stream) {
    return qc::kp::backward<4>("kplanes_tilted_tv_fuse_grad_cuda", d_pts, d_R, d_grid, d_gout,
                               d_ggrid, d_gR, d_gpts, B, T, C, H, W, 0, T < 0 ? 0 : T, h,
                               stream);
}

int kplanes_tilted_fuse_grad_cuda(const float *d_pts, const float *d_R, const float *d_grid,
                                  const float *d_gout, float *d_ggrid, float *d_gR, float *d_gpts,
                                  long B, int T, int C, int H, int W, cudaStream_t stream) {
    return kplanes_tilted_fuse_grad_rotations_cuda(d_pts, d_R, d_grid, d_gout, d_ggrid, d_gR,
                                                   d_gpts, B, T, C, H, W, 0, T < 0 ? 0 : T,
                                                   stream);
}

int kplanes_tilted_fuse_levels_cuda(const float *d_pts, const float *d_R, int n_levels,
                                    const float *const *grids, float *const *outs, const int *H,
                                    const int *W, long B, int T, int C, cudaStream_t stream) {
    return qc::kp::forward_levels(d_pts, d_R, n_levels, grids, outs, H, W, B, T, C, stream);
}

int kplanes_tilted_fuse_levels_grad_cuda(const float *d_pts, const float *d_R, int n_levels,
                                         const float *const *grids, const float *const *gouts,
                                         float *const *ggrids, const int *H, const int *W,
                                         float *d_gR, float *d_gpts, long B, int T, int C,
                                         cudaStream_t stream) {
    return qc::kp::backward_levels(d_pts, d_R, n_levels, grids, gouts, ggrids, H, W, d_gR, d_gpts,
                                   B, T, C, stream);
}

int kplanes_planes_to_channels_last_cuda(const float *d_src, float *d_dst, int P, int C, int H,
                                         int W, cudaStream_t stream) {
    QC_RETURN_IF(P < 0 || C < 0 || H < 0 || W < 0, QC_ERR_INVALID_ARGUMENT,
                 "kplanes_planes_to_channels_last_cuda: negative shape");
    QC_RETURN_IF((long long)H * W >= (1LL << 31), QC_ERR_INVALID_ARGUMENT,
                 "kplanes_planes_to_channels_last_cuda: H*W too large");
    const int S = H * W;
    if ((long long)P * C * S == 0) return 0;
    QC_RETURN_IF(P > 65535, QC_ERR_INVALID_ARGUMENT, "transpose: more than 65535 planes");
    if (C % 4 == 0 && S % 4 == 0 && qc::kp::aligned16(d_src) && qc::kp::aligned16(d_dst))
        return qc::kp::launch_transpose_fast(d_src, d_dst, P, C, S, true, stream);
    return qc::kp::launch_transpose(d_src, d_dst, P, C, S, stream);
}

int kplanes_planes_from_channels_last_cuda(const float *d_src, float *d_dst, int P, int C, int H,
                                           int W, cudaStream_t stream) {
    QC_RETURN_IF(P < 0 || C < 0 || H < 0 || W < 0, QC_ERR_INVALID_ARGUMENT,
                 "kplanes_planes_from_channels_last_cuda: negative shape");
    QC_RETURN_IF((long long)H * W >= (1LL << 31), QC_ERR_INVALID_ARGUMENT,
                 "kplanes_planes_from_channels_last_cuda: H*W too large");
    const int S = H * W;
    if ((long long)P * C * S == 0) return 0;
    QC_RETURN_IF(P > 65535, QC_ERR_INVALID_ARGUMENT, "transpose: more than 65535 planes");
    if (C % 4 == 0 && S % 4 == 0 && qc::kp::aligned16(d_src) && qc::kp::aligned16(d_dst))
        return qc::kp::launch_transpose_fast(d_src, d_dst, P, C, S, false, stream);
    return qc::kp::launch_transpose(d_src, d_dst, P, S, C, stream);
}

}  // extern "C"
