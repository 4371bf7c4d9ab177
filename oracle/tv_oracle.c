/* tv_oracle.c — CPU oracle for the 3-D total-variation losses and gradients.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the oracle the CUDA
 * kernels are tested against; nothing in the product links, loads or calls it. Only the tests,
 * the smoke check and the CPU-baseline leg of the benchmark use it.
 *
 * It restates, term by term, the reference kernels in
 * csrc/cuda/core/tv_loss.cu (quantem-cuda), deliberately in the reference's own
 * formulation (per-corner / per-voxel sums) rather than the divergence form
 * the CUDA kernels use, so that it checks the restructuring:
 *   iso loss      tv_loss.cu:64-78     Σ_corners sqrt(dd²+dh²+dw²+eps)
 *   iso gradient  tv_loss.cu:125-191   four corners per voxel, 1/sqrt
 *   sq loss       tv_loss.cu:237-258   Σ_axes Σ diff², full ranges
 *   sq gradient   tv_loss.cu:312-331   2g·Σ[(v-prev) - (next-v)]
 *   L1 loss       tv_loss.cu:371-383   per-axis Σ|diff|
 *   L1 gradient   tv_loss.cu:434-474   Σ g_axis·(sgn(v-prev) - sgn(next-v)), sgn(0)=0
 * Differences and per-term arithmetic are fp32 like the reference; sums are
 * accumulated in fp64 per (batch, plane) and combined in fixed order, so the
 * result is deterministic for any thread count.
 */
#include <math.h>
#include <stddef.h>
#include <stdlib.h>

#define AT(n, d, h, w) vol[((((size_t)(n) * D + (d)) * H + (h)) * W) + (w)]

static float sgnf_ref(float x) { return (float)((x > 0.0f) - (x < 0.0f)); }

/* out[0] = Σ iso corners (raw sum, not the mean). */
void oracle_tv_iso_loss(const float *vol, int B, int D, int H, int W, float eps, double *out) {
    const long long S = (long long)B * D;
    double *part = (double *)calloc((size_t)(S > 0 ? S : 1), sizeof(double));
#pragma omp parallel for schedule(dynamic, 1)
    for (long long z = 0; z < S; ++z) {
        const int n = (int)(z / D), i = (int)(z % D);
        double acc = 0.0;
        if (i < D - 1) {
            for (int j = 0; j < H - 1; ++j)
                for (int k = 0; k < W - 1; ++k) {
                    const float v = AT(n, i, j, k);
                    const float dd = AT(n, i + 1, j, k) - v;
                    const float dh = AT(n, i, j + 1, k) - v;
                    const float dw = AT(n, i, j, k + 1) - v;
                    acc += (double)sqrtf(dd * dd + dh * dh + dw * dw + eps);
                }
        }
        part[z] = acc;
    }
    double t = 0.0;
    for (long long z = 0; z < S; ++z) t += part[z];
    free(part);
    out[0] = t;
}

static float corner_inv(const float *vol, int n, int i, int j, int k, int D, int H, int W,
                        float eps, float *dd, float *dh, float *dw) {
    const float v = AT(n, i, j, k);
    *dd = AT(n, i + 1, j, k) - v;
    *dh = AT(n, i, j + 1, k) - v;
    *dw = AT(n, i, j, k + 1) - v;
    return 1.0f / sqrtf(*dd * *dd + *dh * *dh + *dw * *dw + eps);
}

/* grad = g_scaled · ∂(Σ iso corners)/∂vol; zero when D, H or W < 2. */
void oracle_tv_iso_grad(const float *vol, float g_scaled, float *grad, int B, int D, int H, int W,
                        float eps) {
    const long long S = (long long)B * D;
#pragma omp parallel for schedule(dynamic, 1)
    for (long long z = 0; z < S; ++z) {
        const int n = (int)(z / D), a = (int)(z % D);
        for (int b = 0; b < H; ++b)
            for (int c = 0; c < W; ++c) {
                float acc = 0.0f, dd, dh, dw, inv;
                if (D >= 2 && H >= 2 && W >= 2) {
                    if (a < D - 1 && b < H - 1 && c < W - 1) {
                        inv = corner_inv(vol, n, a, b, c, D, H, W, eps, &dd, &dh, &dw);
                        acc += -(dd + dh + dw) * inv;
                    }
                    if (a >= 1 && b < H - 1 && c < W - 1) {
                        inv = corner_inv(vol, n, a - 1, b, c, D, H, W, eps, &dd, &dh, &dw);
                        acc += dd * inv;
                    }
                    if (a < D - 1 && b >= 1 && c < W - 1) {
                        inv = corner_inv(vol, n, a, b - 1, c, D, H, W, eps, &dd, &dh, &dw);
                        acc += dh * inv;
                    }
                    if (a < D - 1 && b < H - 1 && c >= 1) {
                        inv = corner_inv(vol, n, a, b, c - 1, D, H, W, eps, &dd, &dh, &dw);
                        acc += dw * inv;
                    }
                }
                grad[(((size_t)n * D + a) * H + b) * W + c] = g_scaled * acc;
            }
    }
}

/* out[0] = sq sum (mode 0); out[0..2] = per-axis L1 sums (mode 1). */
static void axis_sums(const float *vol, int B, int D, int H, int W, int l1, double *out) {
    const long long S = (long long)B * D;
    double *part = (double *)calloc((size_t)(S > 0 ? 3 * S : 3), sizeof(double));
#pragma omp parallel for schedule(dynamic, 1)
    for (long long z = 0; z < S; ++z) {
        const int n = (int)(z / D), a = (int)(z % D);
        double sd = 0.0, sh = 0.0, sw = 0.0;
        for (int b = 0; b < H; ++b)
            for (int c = 0; c < W; ++c) {
                const float v = AT(n, a, b, c);
                if (a < D - 1) {
                    const float x = AT(n, a + 1, b, c) - v;
                    sd += l1 ? (double)fabsf(x) : (double)(x * x);
                }
                if (b < H - 1) {
                    const float x = AT(n, a, b + 1, c) - v;
                    sh += l1 ? (double)fabsf(x) : (double)(x * x);
                }
                if (c < W - 1) {
                    const float x = AT(n, a, b, c + 1) - v;
                    sw += l1 ? (double)fabsf(x) : (double)(x * x);
                }
            }
        part[3 * z] = sd;
        part[3 * z + 1] = sh;
        part[3 * z + 2] = sw;
    }
    double td = 0.0, th = 0.0, tw = 0.0;
    for (long long z = 0; z < S; ++z) {
        td += part[3 * z];
        th += part[3 * z + 1];
        tw += part[3 * z + 2];
    }
    free(part);
    if (l1) {
        out[0] = td;
        out[1] = th;
        out[2] = tw;
    } else {
        out[0] = td + th + tw;
    }
}

void oracle_tv_sq_loss(const float *vol, int B, int D, int H, int W, double *out) {
    axis_sums(vol, B, D, H, W, 0, out);
}

void oracle_tv_l1_loss(const float *vol, int B, int D, int H, int W, double *out) {
    axis_sums(vol, B, D, H, W, 1, out);
}

void oracle_tv_sq_grad(const float *vol, float g, float *grad, int B, int D, int H, int W) {
    const long long S = (long long)B * D;
#pragma omp parallel for schedule(dynamic, 1)
    for (long long z = 0; z < S; ++z) {
        const int n = (int)(z / D), a = (int)(z % D);
        for (int b = 0; b < H; ++b)
            for (int c = 0; c < W; ++c) {
                const float v = AT(n, a, b, c);
                float acc = 0.0f;
                if (a < D - 1) acc -= AT(n, a + 1, b, c) - v;
                if (a >= 1) acc += v - AT(n, a - 1, b, c);
                if (b < H - 1) acc -= AT(n, a, b + 1, c) - v;
                if (b >= 1) acc += v - AT(n, a, b - 1, c);
                if (c < W - 1) acc -= AT(n, a, b, c + 1) - v;
                if (c >= 1) acc += v - AT(n, a, b, c - 1);
                grad[(((size_t)n * D + a) * H + b) * W + c] = g * 2.0f * acc;
            }
    }
}

void oracle_tv_l1_grad(const float *vol, const float *g3, float *grad, int B, int D, int H,
                       int W) {
    const float gd = g3[0], gh = g3[1], gw = g3[2];
    const long long S = (long long)B * D;
#pragma omp parallel for schedule(dynamic, 1)
    for (long long z = 0; z < S; ++z) {
        const int n = (int)(z / D), a = (int)(z % D);
        for (int b = 0; b < H; ++b)
            for (int c = 0; c < W; ++c) {
                const float v = AT(n, a, b, c);
                float acc = 0.0f;
                if (a < D - 1) acc -= gd * sgnf_ref(AT(n, a + 1, b, c) - v);
                if (a >= 1) acc += gd * sgnf_ref(v - AT(n, a - 1, b, c));
                if (b < H - 1) acc -= gh * sgnf_ref(AT(n, a, b + 1, c) - v);
                if (b >= 1) acc += gh * sgnf_ref(v - AT(n, a, b - 1, c));
                if (c < W - 1) acc -= gw * sgnf_ref(AT(n, a, b, c + 1) - v);
                if (c >= 1) acc += gw * sgnf_ref(v - AT(n, a, b, c - 1));
                grad[(((size_t)n * D + a) * H + b) * W + c] = acc;
            }
    }
}

#ifdef _OPENMP
#include <omp.h>
#endif

/* Threads used by the parallel loops above (<= 0 leaves the OpenMP default). */
void oracle_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

int oracle_get_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}
