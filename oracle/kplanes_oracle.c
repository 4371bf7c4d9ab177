/* kplanes_oracle.c — CPU oracle for the fused tilted K-Planes interpolation.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the oracle the CUDA
 * kernels are tested against; nothing in the product links, loads or calls it. Only the tests,
 * the smoke check and the CPU-baseline leg of the benchmark use it.
 *
 * It restates the reference kernels of quantem-cuda
 * (csrc/cuda/core/ml/kplanes_tilted.cu):
 *   make_tap            :69-94    unnormalise ((g+1)·0.5·(size-1)), border mask,
 *                                 clamp, floor, bilinear weights, clamped +1 corner
 *   rotate              :96-102   r = R_t·p
 *   forward             :104-139  out[b, t*C+c] = Π_p Σ_k w_k·plane[t*3+p][c][cell_k]
 *   backward            :141-281  ggrid += w_k·s_{p+1}·s_{p+2}·go;
 *                                 dL/dr via ds/dix, ds/diy and the border masks;
 *                                 gR_t += dr ⊗ p;  gpts += R_tᵀ·dr
 *   tv taps             :329-612  the same at R_t·p and at R_t·p + h·R_t[:, k-1]
 *                                 (k = 1..3; h·R_t rounded, then added), output
 *                                 [4, N, T*C]; backward adds h·dr_k to column
 *                                 k-1 of gR_t for taps k >= 1
 * with the plane read in its parameter layout [3T, C, H, W] (the reference's
 * op layer permutes to channels-last only for the GPU; _ops.py:21-25).
 *
 * The forward is fp32 with every multiply-add written as fmaf() in the order
 * nvcc contracts the reference's expressions (measured on the GPU: a0*x0 +
 * a1*x1 + a2*x2 becomes fma(a2, x2, fma(a0, x0, a1*x1)), and likewise for the
 * four-term bilinear sum), so it reproduces the reference kernel's forward
 * values bit for bit on any host. Gradients accumulate in fp64.
 */
#include <math.h>
#include <stddef.h>
#include <stdlib.h>
#include <string.h>

typedef struct {
    int cell[4];
    float w[4];
    float tx, ty, gxm, gym;
} OTap;

static OTap otap(float gx, float gy, int H, int W) {
    OTap t;
    const float wm1 = (float)(W - 1), hm1 = (float)(H - 1);
    float ix = (gx + 1.f) * 0.5f * wm1;
    float iy = (gy + 1.f) * 0.5f * hm1;
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
    const int x1 = x0 + 1 < W - 1 ? x0 + 1 : W - 1;
    const int y1 = y0 + 1 < H - 1 ? y0 + 1 : H - 1;
    t.cell[0] = y0 * W + x0;
    t.cell[1] = y0 * W + x1;
    t.cell[2] = y1 * W + x0;
    t.cell[3] = y1 * W + x1;
    return t;
}

/* a0*x0 + a1*x1 + a2*x2 as an fp32 GPU evaluates the reference's expression
 * after contraction: fma(a2, x2, fma(a0, x0, a1*x1)). */
static float odot3(float a0, float x0, float a1, float x1, float a2, float x2) {
    return fmaf(a2, x2, fmaf(a0, x0, a1 * x1));
}

static void orotate(const float *Rt, float px, float py, float pz, float r[3]) {
    r[0] = odot3(Rt[0], px, Rt[1], py, Rt[2], pz);
    r[1] = odot3(Rt[3], px, Rt[4], py, Rt[5], pz);
    r[2] = odot3(Rt[6], px, Rt[7], py, Rt[8], pz);
}

static void ocoords(const float r[3], int p, float *gx, float *gy) {
    /* p: 0 = XY (rx, ry), 1 = ZX (rz, rx), 2 = YZ (ry, rz) */
    static const int ix[3] = {0, 2, 1}, iy[3] = {1, 0, 2};
    *gx = r[ix[p]];
    *gy = r[iy[p]];
}

/* w0*v0 + w1*v1 + w2*v2 + w3*v3, contracted the same way:
 * fma(w3, v3, fma(w2, v2, fma(w0, v0, w1*v1))). */
static float obilerp(const float w[4], float v0, float v1, float v2, float v3) {
    return fmaf(w[3], v3, fmaf(w[2], v2, fmaf(w[0], v0, w[1] * v1)));
}

/* Sample point of tap k: r itself (k = 0) or r + h·R_t[:, k-1]. */
static void otap_point(const float *Rt, const float r[3], int k, float h, float a[3]) {
    for (int i = 0; i < 3; ++i) {
        if (k == 0) {
            a[i] = r[i];
        } else {
            const float off = h * Rt[3 * i + (k - 1)];
            a[i] = r[i] + off;
        }
    }
}

/* ntap = 1: pts [N,3], R [T,3,3], plane [3T,C,H,W] -> out [N, T*C].
 * ntap = 4: out [4, N, T*C], tap k at R_t·p (+ h·R_t[:, k-1]). */
static void kp_fwd(const float *pts, const float *R, const float *plane, float *out, long N,
                   int T, int C, int H, int W, int ntap, float h) {
    const size_t HW = (size_t)H * W, planeCHW = (size_t)C * HW;
#pragma omp parallel for schedule(dynamic, 256)
    for (long b = 0; b < N; ++b) {
        const float px = pts[3 * b], py = pts[3 * b + 1], pz = pts[3 * b + 2];
        for (int t = 0; t < T; ++t)
        for (int k = 0; k < ntap; ++k) {
            float r0[3], r[3];
            orotate(R + 9 * t, px, py, pz, r0);
            otap_point(R + 9 * t, r0, k, h, r);
            OTap tp[3];
            for (int p = 0; p < 3; ++p) {
                float gx, gy;
                ocoords(r, p, &gx, &gy);
                tp[p] = otap(gx, gy, H, W);
            }
            for (int c = 0; c < C; ++c) {
                float prod = 1.f;
                for (int p = 0; p < 3; ++p) {
                    const float *pc = plane + (size_t)(3 * t + p) * planeCHW + (size_t)c * HW;
                    prod *= obilerp(tp[p].w, pc[tp[p].cell[0]], pc[tp[p].cell[1]],
                                    pc[tp[p].cell[2]], pc[tp[p].cell[3]]);
                }
                out[((size_t)k * N + b) * T * C + (size_t)t * C + c] = prod;
            }
        }
    }
}

void oracle_kplanes_fwd(const float *pts, const float *R, const float *plane, float *out, long N,
                        int T, int C, int H, int W) {
    kp_fwd(pts, R, plane, out, N, T, C, H, W, 1, 0.f);
}

void oracle_kplanes_tv_fwd(const float *pts, const float *R, const float *plane, float *out,
                           long N, int T, int C, int H, int W, float h) {
    kp_fwd(pts, R, plane, out, N, T, C, H, W, 4, h);
}

/* Gradients of Σ out·gout. gpts [N,3], gR [T,3,3], gplane [3T,C,H,W] are
 * overwritten. */
static void kp_bwd(const float *pts, const float *R, const float *plane, const float *gout,
                   float *gpts, float *gR, float *gplane, long N, int T, int C, int H, int W,
                   int ntap, float h) {
    const size_t HW = (size_t)H * W, planeCHW = (size_t)C * HW;
    const size_t P = (size_t)3 * T * planeCHW;
    double *acc = (double *)calloc(P > 0 ? P : 1, sizeof(double));
    double gR_acc[9 * 4096];
    memset(gR_acc, 0, sizeof(double) * 9 * (size_t)T);

#pragma omp parallel
    {
        double *gR_loc = (double *)calloc(9 * (size_t)T, sizeof(double));
#pragma omp for schedule(dynamic, 256)
        for (long b = 0; b < N; ++b) {
            const float px = pts[3 * b], py = pts[3 * b + 1], pz = pts[3 * b + 2];
            double gp[3] = {0.0, 0.0, 0.0};
            for (int t = 0; t < T; ++t)
            for (int kt = 0; kt < ntap; ++kt) {
                const float *Rt = R + 9 * t;
                float r0[3], r[3];
                orotate(Rt, px, py, pz, r0);
                otap_point(Rt, r0, kt, h, r);
                OTap tp[3];
                for (int p = 0; p < 3; ++p) {
                    float gx, gy;
                    ocoords(r, p, &gx, &gy);
                    tp[p] = otap(gx, gy, H, W);
                }
                double dgx[3] = {0, 0, 0}, dgy[3] = {0, 0, 0};
                for (int c = 0; c < C; ++c) {
                    const float go = gout[((size_t)kt * N + b) * T * C + (size_t)t * C + c];
                    float v[3][4], s[3];
                    for (int p = 0; p < 3; ++p) {
                        const float *pc = plane + (size_t)(3 * t + p) * planeCHW + (size_t)c * HW;
                        for (int k = 0; k < 4; ++k) v[p][k] = pc[tp[p].cell[k]];
                        s[p] = obilerp(tp[p].w, v[p][0], v[p][1], v[p][2], v[p][3]);
                    }
                    for (int p = 0; p < 3; ++p) {
                        const double other = (double)s[(p + 1) % 3] * s[(p + 2) % 3] * go;
                        double *gq = acc + (size_t)(3 * t + p) * planeCHW + (size_t)c * HW;
                        for (int k = 0; k < 4; ++k) {
                            const double val = other * tp[p].w[k];
                            if (val != 0.0) {
#pragma omp atomic update
                                gq[tp[p].cell[k]] += val;
                            }
                        }
                        const double tx = tp[p].tx, ty = tp[p].ty;
                        dgx[p] += other * ((1.0 - ty) * ((double)v[p][1] - v[p][0]) +
                                           ty * ((double)v[p][3] - v[p][2]));
                        dgy[p] += other * ((1.0 - tx) * ((double)v[p][2] - v[p][0]) +
                                           tx * ((double)v[p][3] - v[p][1]));
                    }
                }
                const double drx = dgx[0] * tp[0].gxm + dgy[1] * tp[1].gym;
                const double dry = dgy[0] * tp[0].gym + dgx[2] * tp[2].gxm;
                const double drz = dgx[1] * tp[1].gxm + dgy[2] * tp[2].gym;
                gp[0] += Rt[0] * drx + Rt[3] * dry + Rt[6] * drz;
                gp[1] += Rt[1] * drx + Rt[4] * dry + Rt[7] * drz;
                gp[2] += Rt[2] * drx + Rt[5] * dry + Rt[8] * drz;
                double *g9 = gR_loc + 9 * t;
                g9[0] += drx * px;
                g9[1] += drx * py;
                g9[2] += drx * pz;
                g9[3] += dry * px;
                g9[4] += dry * py;
                g9[5] += dry * pz;
                g9[6] += drz * px;
                g9[7] += drz * py;
                g9[8] += drz * pz;
                if (kt > 0) {
                    g9[kt - 1] += (double)h * drx;
                    g9[3 + kt - 1] += (double)h * dry;
                    g9[6 + kt - 1] += (double)h * drz;
                }
            }
            gpts[3 * b] = (float)gp[0];
            gpts[3 * b + 1] = (float)gp[1];
            gpts[3 * b + 2] = (float)gp[2];
        }
#pragma omp critical
        for (int i = 0; i < 9 * T; ++i) gR_acc[i] += gR_loc[i];
        free(gR_loc);
    }
    for (int i = 0; i < 9 * T; ++i) gR[i] = (float)gR_acc[i];
    for (size_t i = 0; i < P; ++i) gplane[i] = (float)acc[i];
    free(acc);
}

void oracle_kplanes_bwd(const float *pts, const float *R, const float *plane, const float *gout,
                        float *gpts, float *gR, float *gplane, long N, int T, int C, int H,
                        int W) {
    kp_bwd(pts, R, plane, gout, gpts, gR, gplane, N, T, C, H, W, 1, 0.f);
}

void oracle_kplanes_tv_bwd(const float *pts, const float *R, const float *plane,
                           const float *gout, float *gpts, float *gR, float *gplane, long N, int T,
                           int C, int H, int W, float h) {
    kp_bwd(pts, R, plane, gout, gpts, gR, gplane, N, T, C, H, W, 4, h);
}
