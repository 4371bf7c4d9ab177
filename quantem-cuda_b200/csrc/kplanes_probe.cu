// kplanes_probe.cu — the K-Planes kernels' memory traffic without their
// arithmetic, to measure the L2-side ceiling of their access pattern.
//
// Each (point, rotation) pair of the tilted K-Planes kernels touches 12
// channel rows of C = 32 floats (3 planes x 4 bilinear corners, one 128-byte
// L2 line each) at data-dependent cells: the forward gathers them and writes
// one 128-byte output row; the backward gathers them again, adds one
// 128-byte vector reduction per corner into the plane gradient, reads one
// 128-byte upstream-gradient row and adds 3 scalars to the point gradient.
// These kernels replay exactly that traffic with hashed cells (uniform over
// the plane, like rotated random points) and the same lane mapping (8 lanes
// x float4 per pair), so the time they take is what the memory system allows
// for the pattern, with no arithmetic or dependency in the way.
#include "qc_common.cuh"

namespace qc {
namespace kprobe {

constexpr int C = 32, L = 8, G = 32 / L;
constexpr int kBlocksPerSm = 4;
constexpr int kMaxSms = 512;  // the sink is sized for this many SMs

__device__ __forceinline__ uint32_t hash32(uint32_t x) {
    x ^= x >> 16;
    x *= 0x7feb352du;
    x ^= x >> 15;
    x *= 0x846ca68bu;
    x ^= x >> 16;
    return x;
}

// MODE: QC_KP_PROBE_GATHER, _REDUCE, _BACKWARD, _FORWARD (see the header).
template <int MODE>
__global__ void __launch_bounds__(256) probe_kernel(const float *__restrict__ planes,
                                                    float *__restrict__ grad, const float *__restrict__ gout,
                                                    float *__restrict__ out, float *__restrict__ gpts,
                                                    float *__restrict__ sink, long long pairs, long long npts,
                                                    int H, int W) {
    const int lane = threadIdx.x & 31, grp = lane / L, c4 = 4 * (lane % L);
    const long long HW = (long long)H * W;
    const uint32_t span = (uint32_t)((H - 1) * W - 1);  // cell, cell+1, cell+W, cell+W+1 < H*W
    const bool gathers = MODE != QC_KP_PROBE_REDUCE;
    const bool reduces = MODE == QC_KP_PROBE_REDUCE || MODE == QC_KP_PROBE_BACKWARD;
    float acc = 0.f;
    const long long gw = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const long long nw = ((long long)gridDim.x * blockDim.x) >> 5;
    for (long long b0 = gw * G; b0 < pairs; b0 += nw * G) {
        const long long b = b0 + grp;
        if (b >= pairs) continue;
        float4 go = make_float4(1.f, 1.f, 1.f, 1.f);
        if (MODE == QC_KP_PROBE_BACKWARD) go = __ldcs(reinterpret_cast<const float4 *>(gout + b * C + c4));
        float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int p = 0; p < 3; ++p) {
            const uint32_t cell = hash32((uint32_t)(b * 3 + p)) % span;
            const long long base = (p * HW + cell) * C + c4;
            const long long off[4] = {base, base + C, base + (long long)W * C, base + (long long)(W + 1) * C};
            if (gathers) {
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const float4 v = ldg4(planes + off[k]);
                    s.x += v.x;
                    s.y += v.y;
                    s.z += v.z;
                    s.w += v.w;
                }
            }
            if (reduces) {
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    red_add_v4(grad + off[k], make_float4(s.x * go.x, s.y * go.y, s.z * go.z, s.w * go.w + 1.f));
            }
        }
        if (MODE == QC_KP_PROBE_BACKWARD && (lane % L) == 0) {
            const long long q = (long long)(hash32((uint32_t)b ^ 0x9e3779b9u) % (uint32_t)npts);
            atomicAdd(gpts + 3 * q, s.x);
            atomicAdd(gpts + 3 * q + 1, s.y);
            atomicAdd(gpts + 3 * q + 2, s.z);
        }
        if (MODE == QC_KP_PROBE_FORWARD) __stcs(reinterpret_cast<float4 *>(out + b * C + c4), s);
        acc += s.x + s.y + s.z + s.w;
    }
    sink[(long long)blockIdx.x * blockDim.x + threadIdx.x] = acc;
}

}  // namespace kprobe
}  // namespace qc

extern "C" int kplanes_l2_probe_cuda(int mode, const float *d_planes, float *d_grad, const float *d_gout,
                                     float *d_out, float *d_gpts, float *d_sink, long long pairs,
                                     long long npts, int H, int W, cudaStream_t stream) {
    using namespace qc::kprobe;
    QC_RETURN_IF(mode < QC_KP_PROBE_GATHER || mode > QC_KP_PROBE_FORWARD, QC_ERR_INVALID_ARGUMENT,
                 "kplanes_l2_probe_cuda: unknown mode %d", mode);
    QC_RETURN_IF(pairs < 1 || npts < 1 || H < 2 || W < 2 || (long long)H * W >= (1LL << 31),
                 QC_ERR_INVALID_ARGUMENT, "kplanes_l2_probe_cuda: bad sizes");
    QC_RETURN_IF(d_planes == nullptr || d_grad == nullptr || d_gout == nullptr || d_out == nullptr ||
                     d_gpts == nullptr || d_sink == nullptr,
                 QC_ERR_INVALID_ARGUMENT, "kplanes_l2_probe_cuda: null buffer");
    int sms = 0;
    if (int st = qc::device_sm_count(&sms)) return st;
    // d_sink holds kplanes_l2_probe_sink_floats() floats: one per thread
    const int blocks = kBlocksPerSm * (sms < kMaxSms ? sms : kMaxSms);
    switch (mode) {
        case QC_KP_PROBE_GATHER:
            probe_kernel<QC_KP_PROBE_GATHER><<<blocks, 256, 0, stream>>>(d_planes, d_grad, d_gout, d_out, d_gpts,
                                                                         d_sink, pairs, npts, H, W);
            break;
        case QC_KP_PROBE_REDUCE:
            probe_kernel<QC_KP_PROBE_REDUCE><<<blocks, 256, 0, stream>>>(d_planes, d_grad, d_gout, d_out, d_gpts,
                                                                         d_sink, pairs, npts, H, W);
            break;
        case QC_KP_PROBE_BACKWARD:
            probe_kernel<QC_KP_PROBE_BACKWARD><<<blocks, 256, 0, stream>>>(d_planes, d_grad, d_gout, d_out,
                                                                           d_gpts, d_sink, pairs, npts, H, W);
            break;
        default:
            probe_kernel<QC_KP_PROBE_FORWARD><<<blocks, 256, 0, stream>>>(d_planes, d_grad, d_gout, d_out,
                                                                          d_gpts, d_sink, pairs, npts, H, W);
            break;
    }
    QC_CHECK_LAUNCH("kplanes_l2_probe_cuda launch");
    return 0;
}

extern "C" size_t kplanes_l2_probe_sink_floats(void) {
    return (size_t)qc::kprobe::kBlocksPerSm * qc::kprobe::kMaxSms * 256;
}
