// pybind_core.cpp — the `quantem.cuda._core` extension: a torch-free binding
// of the C ABI (include/quantem_cuda_b200.h). Tensors cross as integer device
// pointers (tensor.data_ptr()), shapes as ints and the stream as the integer
// torch.cuda.current_stream().cuda_stream, exactly like the reference's
// `_core` (csrc/bindings.cpp:22-28, csrc/bindings/core.cpp:101-148,
// csrc/bindings/core/ml.cpp:89-128). A non-zero status raises RuntimeError,
// which is what the reference's std::runtime_error becomes in Python.
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

#include "quantem_cuda_b200.h"

namespace py = pybind11;

namespace {

void check(int status) {
    if (status != 0)
        throw std::runtime_error(std::string(quantem_cuda_status_string(status)) + ": " +
                                 quantem_cuda_last_error());
}

template <typename T>
T *ptr(uintptr_t v) {
    return reinterpret_cast<T *>(v);
}

cudaStream_t stream_of(uintptr_t v) { return reinterpret_cast<cudaStream_t>(v); }

qc_peer_group make_group(int rank, int world, unsigned long long timeout_ns,
                         const std::vector<uintptr_t> &comm, const std::vector<uintptr_t> &buf) {
    if (world < 1 || world > QC_MAX_PEER_RANKS || (int)comm.size() != world ||
        (int)buf.size() != world)
        throw std::invalid_argument("PeerGroup: need 1 <= world <= " +
                                    std::to_string(QC_MAX_PEER_RANKS) +
                                    " and one communication block and buffer per rank");
    qc_peer_group g{};
    g.rank = rank;
    g.world = world;
    g.timeout_ns = timeout_ns;
    for (int q = 0; q < world; ++q) {
        g.comm[q] = ptr<void>(comm[q]);
        g.buf[q] = ptr<float>(buf[q]);
    }
    return g;
}

qc_tv_peers make_peers(int rank, int world, unsigned long long timeout_ns,
                       const std::vector<uintptr_t> &comm, uintptr_t prev_slab, int prev_dp,
                       uintptr_t next_slab, int next_dp) {
    if (world < 1 || world > QC_MAX_PEER_RANKS || (int)comm.size() != world)
        throw std::invalid_argument("TvPeers: need 1 <= world <= " +
                                    std::to_string(QC_MAX_PEER_RANKS) +
                                    " and one communication block per rank");
    qc_tv_peers p{};
    p.rank = rank;
    p.world = world;
    p.timeout_ns = timeout_ns;
    for (int q = 0; q < world; ++q) p.comm[q] = ptr<void>(comm[q]);
    p.prev_slab = ptr<float>(prev_slab);
    p.prev_dp = prev_dp;
    p.next_slab = ptr<float>(next_slab);
    p.next_dp = next_dp;
    return p;
}

}  // namespace

PYBIND11_MODULE(_core, m) {
    m.doc() = "quantem-cuda B200 kernels (raw-pointer API; use quantem.cuda.* instead)";
    m.attr("__cudart_version__") = quantem_cuda_cudart_version();

    // ── TV ──
    m.def("tv_loss_3d_workspace_bytes", &tv_loss_3d_workspace_bytes, py::arg("B"), py::arg("D"),
          py::arg("H"), py::arg("W"));

    // The reference's TV bindings, same names, arguments and argument names
    // (csrc/bindings/core.cpp:101-148): loss sums accumulate into acc with
    // fp32 atomics, as the reference's kernels do.
    m.def(
        "tv_loss_iso_3d_cuda",
        [](uintptr_t vol, uintptr_t acc, int B, int D, int H, int W, float eps, uintptr_t stream) {
            check(tv_loss_iso_3d_cuda(ptr<const float>(vol), ptr<float>(acc), B, D, H, W, eps,
                                      stream_of(stream)));
        },
        "Isotropic 3-D TV forward. vol_ptr: fp32 [B,D,H,W]; acc_ptr: pre-zeroed one-element fp32 "
        "accumulator (unnormalised corner sum added).",
        py::arg("vol_ptr"), py::arg("acc_ptr"), py::arg("B"), py::arg("D"), py::arg("H"),
        py::arg("W"), py::arg("eps"), py::arg("stream_ptr"));

    m.def(
        "tv_loss_iso_3d_grad_cuda",
        [](uintptr_t vol, uintptr_t g, uintptr_t grad, int B, int D, int H, int W, float eps,
           uintptr_t stream) {
            check(tv_loss_iso_3d_grad_cuda(ptr<const float>(vol), ptr<const float>(g),
                                           ptr<float>(grad), B, D, H, W, eps, stream_of(stream)));
        },
        "Backward of tv_loss_iso_3d; g_scaled_ptr = upstream / N (device scalar); grad_vol fully "
        "written.",
        py::arg("vol_ptr"), py::arg("g_scaled_ptr"), py::arg("grad_vol_ptr"), py::arg("B"),
        py::arg("D"), py::arg("H"), py::arg("W"), py::arg("eps"), py::arg("stream_ptr"));

    m.def(
        "tv_loss_sq_3d_cuda",
        [](uintptr_t vol, uintptr_t acc, int B, int D, int H, int W, uintptr_t stream) {
            check(tv_loss_sq_3d_cuda(ptr<const float>(vol), ptr<float>(acc), B, D, H, W,
                                     stream_of(stream)));
        },
        "Squared-anisotropic 3-D TV forward; acc_ptr: pre-zeroed one-element accumulator.",
        py::arg("vol_ptr"), py::arg("acc_ptr"), py::arg("B"), py::arg("D"), py::arg("H"),
        py::arg("W"), py::arg("stream_ptr"));

    m.def(
        "tv_loss_sq_3d_grad_cuda",
        [](uintptr_t vol, uintptr_t g, uintptr_t grad, int B, int D, int H, int W,
           uintptr_t stream) {
            check(tv_loss_sq_3d_grad_cuda(ptr<const float>(vol), ptr<const float>(g),
                                          ptr<float>(grad), B, D, H, W, stream_of(stream)));
        },
        "Backward of tv_loss_sq_3d; g_ptr = raw upstream grad (x2 in the kernel); grad_vol fully "
        "written.",
        py::arg("vol_ptr"), py::arg("g_ptr"), py::arg("grad_vol_ptr"), py::arg("B"), py::arg("D"),
        py::arg("H"), py::arg("W"), py::arg("stream_ptr"));

    m.def(
        "tv_loss_l1_3d_cuda",
        [](uintptr_t vol, uintptr_t acc, int B, int D, int H, int W, uintptr_t stream) {
            check(tv_loss_l1_3d_cuda(ptr<const float>(vol), ptr<float>(acc), B, D, H, W,
                                     stream_of(stream)));
        },
        "L1-anisotropic 3-D TV forward; acc_ptr: pre-zeroed 3-element accumulator (d, h, w).",
        py::arg("vol_ptr"), py::arg("acc_ptr"), py::arg("B"), py::arg("D"), py::arg("H"),
        py::arg("W"), py::arg("stream_ptr"));

    m.def(
        "tv_loss_l1_3d_grad_cuda",
        [](uintptr_t vol, uintptr_t g, uintptr_t grad, int B, int D, int H, int W,
           uintptr_t stream) {
            check(tv_loss_l1_3d_grad_cuda(ptr<const float>(vol), ptr<const float>(g),
                                          ptr<float>(grad), B, D, H, W, stream_of(stream)));
        },
        "Backward of tv_loss_l1_3d; g_ptr: 3 per-axis upstream grads (d, h, w); sign(0) = 0.",
        py::arg("vol_ptr"), py::arg("g_ptr"), py::arg("grad_vol_ptr"), py::arg("B"), py::arg("D"),
        py::arg("H"), py::arg("W"), py::arg("stream_ptr"));

    // Deterministic forms of the three sums (fixed-order reduction through a
    // caller-owned workspace of tv_loss_3d_workspace_bytes() bytes).
    m.def(
        "tv_loss_iso_3d_ws_cuda",
        [](uintptr_t vol, uintptr_t acc, int B, int D, int H, int W, float eps, uintptr_t ws,
           size_t ws_bytes, uintptr_t stream) {
            check(tv_loss_iso_3d_ws_cuda(ptr<const float>(vol), ptr<float>(acc), B, D, H, W, eps,
                                         ptr<void>(ws), ws_bytes, stream_of(stream)));
        },
        py::arg("vol_ptr"), py::arg("acc_ptr"), py::arg("B"), py::arg("D"), py::arg("H"),
        py::arg("W"), py::arg("eps"), py::arg("ws_ptr"), py::arg("ws_bytes"), py::arg("stream_ptr"));

    m.def(
        "tv_loss_sq_3d_ws_cuda",
        [](uintptr_t vol, uintptr_t acc, int B, int D, int H, int W, uintptr_t ws, size_t ws_bytes,
           uintptr_t stream) {
            check(tv_loss_sq_3d_ws_cuda(ptr<const float>(vol), ptr<float>(acc), B, D, H, W,
                                        ptr<void>(ws), ws_bytes, stream_of(stream)));
        },
        py::arg("vol_ptr"), py::arg("acc_ptr"), py::arg("B"), py::arg("D"), py::arg("H"),
        py::arg("W"), py::arg("ws_ptr"), py::arg("ws_bytes"), py::arg("stream_ptr"));

    m.def(
        "tv_loss_l1_3d_ws_cuda",
        [](uintptr_t vol, uintptr_t acc, int B, int D, int H, int W, uintptr_t ws, size_t ws_bytes,
           uintptr_t stream) {
            check(tv_loss_l1_3d_ws_cuda(ptr<const float>(vol), ptr<float>(acc), B, D, H, W,
                                        ptr<void>(ws), ws_bytes, stream_of(stream)));
        },
        py::arg("vol_ptr"), py::arg("acc_ptr"), py::arg("B"), py::arg("D"), py::arg("H"),
        py::arg("W"), py::arg("ws_ptr"), py::arg("ws_bytes"), py::arg("stream_ptr"));

    m.def(
        "tv_loss_3d_slab_cuda",
        [](int variant, int flags, uintptr_t vol, uintptr_t g, uintptr_t acc, uintptr_t grad,
           int B, int Dp, int H, int W, int d_lo, int d_hi, int has_prev, int has_next, float eps,
           float acc_scale, uintptr_t ws, size_t ws_bytes, uintptr_t stream) {
            check(tv_loss_3d_slab_cuda(variant, flags, ptr<const float>(vol), ptr<const float>(g),
                                       ptr<float>(acc), ptr<float>(grad), B, Dp, H, W, d_lo, d_hi,
                                       has_prev, has_next, eps, acc_scale, ptr<void>(ws), ws_bytes,
                                       stream_of(stream)));
        },
        py::arg("variant"), py::arg("flags"), py::arg("vol_ptr"), py::arg("g_ptr"),
        py::arg("acc_ptr"), py::arg("grad_vol_ptr"), py::arg("B"), py::arg("Dp"), py::arg("H"),
        py::arg("W"), py::arg("d_lo"), py::arg("d_hi"), py::arg("has_prev"), py::arg("has_next"),
        py::arg("eps"), py::arg("acc_scale"), py::arg("ws_ptr"), py::arg("ws_bytes"),
        py::arg("stream_ptr"));

    m.def(
        "tv_loss_mix_3d_fwd_grad_cuda",
        [](int terms, int flags, uintptr_t vol, uintptr_t g, uintptr_t acc, uintptr_t grad, int B,
           int D, int H, int W, float eps, float iso_scale, uintptr_t ws, size_t ws_bytes,
           uintptr_t stream) {
            check(tv_loss_mix_3d_fwd_grad_cuda(terms, flags, ptr<const float>(vol),
                                               ptr<const float>(g), ptr<float>(acc),
                                               ptr<float>(grad), B, D, H, W, eps, iso_scale,
                                               ptr<void>(ws), ws_bytes, stream_of(stream)));
        },
        "Two or three TV terms in one sweep: g = [g_sq, g_iso, g_d, g_h, g_w], acc = [sq, "
        "iso_scale*iso, l1_d, l1_h, l1_w], grad = the weighted sum of the terms' gradients.",
        py::arg("terms"), py::arg("flags"), py::arg("vol_ptr"), py::arg("g_ptr"), py::arg("acc_ptr"),
        py::arg("grad_vol_ptr"), py::arg("B"), py::arg("D"), py::arg("H"), py::arg("W"),
        py::arg("eps"), py::arg("iso_scale"), py::arg("ws_ptr"), py::arg("ws_bytes"),
        py::arg("stream_ptr"));
    m.attr("TV_TERM_SQ") = QC_TV_TERM_SQ;
    m.attr("TV_TERM_ISO") = QC_TV_TERM_ISO;
    m.attr("TV_TERM_L1") = QC_TV_TERM_L1;

    m.attr("TV_SQ") = QC_TV_SQ;
    m.attr("TV_ISO") = QC_TV_ISO;
    m.attr("TV_L1") = QC_TV_L1;
    m.attr("TV_LOSS") = QC_TV_LOSS;
    m.attr("TV_GRAD") = QC_TV_GRAD;
    m.attr("TV_ACC_OVERWRITE") = QC_TV_ACC_OVERWRITE;

    // ── K-Planes ──
    m.def(
        "kplanes_tilted_fuse_cuda",
        [](uintptr_t pts, uintptr_t r, uintptr_t grid, uintptr_t out, long B, int T, int C, int H,
           int W, uintptr_t stream) {
            check(kplanes_tilted_fuse_cuda(ptr<const float>(pts), ptr<const float>(r),
                                           ptr<const float>(grid), ptr<float>(out), B, T, C, H, W,
                                           stream_of(stream)));
        },
        "Fused TILTED K-Planes interpolation (one level). grid_ptr: fp32 [3T,H,W,C] "
        "channels-last; out_ptr: fp32 [B,T*C], fully written.",
        py::arg("pts_ptr"), py::arg("r_ptr"), py::arg("grid_ptr"), py::arg("out_ptr"), py::arg("B"),
        py::arg("T"), py::arg("C"), py::arg("H"), py::arg("W"), py::arg("stream_ptr"));

    m.def(
        "kplanes_tilted_fuse_grad_cuda",
        [](uintptr_t pts, uintptr_t r, uintptr_t grid, uintptr_t gout, uintptr_t ggrid,
           uintptr_t gr, uintptr_t gpts, long B, int T, int C, int H, int W, uintptr_t stream) {
            check(kplanes_tilted_fuse_grad_cuda(ptr<const float>(pts), ptr<const float>(r),
                                                ptr<const float>(grid), ptr<const float>(gout),
                                                ptr<float>(ggrid), ptr<float>(gr), ptr<float>(gpts),
                                                B, T, C, H, W, stream_of(stream)));
        },
        "Backward of kplanes_tilted_fuse. ggrid [3T,H,W,C], gr [T,3,3] and gpts [B,3] are "
        "accumulated into (pre-zero them).",
        py::arg("pts_ptr"), py::arg("r_ptr"), py::arg("grid_ptr"), py::arg("gout_ptr"),
        py::arg("ggrid_ptr"), py::arg("gr_ptr"), py::arg("gpts_ptr"), py::arg("B"), py::arg("T"),
        py::arg("C"), py::arg("H"), py::arg("W"), py::arg("stream_ptr"));

    m.def(
        "kplanes_tilted_tv_fuse_cuda",
        [](uintptr_t pts, uintptr_t r, uintptr_t grid, uintptr_t out, long B, int T, int C, int H,
           int W, float h, uintptr_t stream) {
            check(kplanes_tilted_tv_fuse_cuda(ptr<const float>(pts), ptr<const float>(r),
                                              ptr<const float>(grid), ptr<float>(out), B, T, C, H,
                                              W, h, stream_of(stream)));
        },
        "Four-tap tilted K-Planes: out [4, B, T*C] at R.x and R.x + h*R[:, k-1].",
        py::arg("pts_ptr"), py::arg("r_ptr"), py::arg("grid_ptr"), py::arg("out_ptr"), py::arg("B"),
        py::arg("T"), py::arg("C"), py::arg("H"), py::arg("W"), py::arg("h"),
        py::arg("stream_ptr"));

    m.def(
        "kplanes_tilted_tv_fuse_grad_cuda",
        [](uintptr_t pts, uintptr_t r, uintptr_t grid, uintptr_t gout, uintptr_t ggrid,
           uintptr_t gr, uintptr_t gpts, long B, int T, int C, int H, int W, float h,
           uintptr_t stream) {
            check(kplanes_tilted_tv_fuse_grad_cuda(
                ptr<const float>(pts), ptr<const float>(r), ptr<const float>(grid),
                ptr<const float>(gout), ptr<float>(ggrid), ptr<float>(gr), ptr<float>(gpts), B, T,
                C, H, W, h, stream_of(stream)));
        },
        "Backward of kplanes_tilted_tv_fuse. gout [4, B, T*C]; ggrid, gr, gpts accumulated into.",
        py::arg("pts_ptr"), py::arg("r_ptr"), py::arg("grid_ptr"), py::arg("gout_ptr"),
        py::arg("ggrid_ptr"), py::arg("gr_ptr"), py::arg("gpts_ptr"), py::arg("B"), py::arg("T"),
        py::arg("C"), py::arg("H"), py::arg("W"), py::arg("h"), py::arg("stream_ptr"));

    m.def(
        "kplanes_tilted_fuse_levels_cuda",
        [](uintptr_t pts, uintptr_t r, const std::vector<uintptr_t> &grids,
           const std::vector<uintptr_t> &outs, const std::vector<int> &H, const std::vector<int> &W,
           long B, int T, int C, uintptr_t stream) {
            const size_t n = grids.size();
            if (outs.size() != n || H.size() != n || W.size() != n)
                throw std::invalid_argument("kplanes_tilted_fuse_levels_cuda: one grid, output, H and W per level");
            std::vector<const float *> g(n);
            std::vector<float *> o(n);
            for (size_t l = 0; l < n; ++l) {
                g[l] = ptr<const float>(grids[l]);
                o[l] = ptr<float>(outs[l]);
            }
            check(kplanes_tilted_fuse_levels_cuda(ptr<const float>(pts), ptr<const float>(r), (int)n,
                                                  g.data(), o.data(), H.data(), W.data(), B, T, C,
                                                  stream_of(stream)));
        },
        "Several levels of a multiscale tilted K-Planes encoding in one launch.",
        py::arg("pts_ptr"), py::arg("r_ptr"), py::arg("grid_ptrs"), py::arg("out_ptrs"), py::arg("H"),
        py::arg("W"), py::arg("B"), py::arg("T"), py::arg("C"), py::arg("stream_ptr"));

    m.def(
        "kplanes_tilted_fuse_levels_grad_cuda",
        [](uintptr_t pts, uintptr_t r, const std::vector<uintptr_t> &grids,
           const std::vector<uintptr_t> &gouts, const std::vector<uintptr_t> &ggrids,
           const std::vector<int> &H, const std::vector<int> &W, uintptr_t gr, uintptr_t gpts, long B,
           int T, int C, uintptr_t stream) {
            const size_t n = grids.size();
            if (gouts.size() != n || ggrids.size() != n || H.size() != n || W.size() != n)
                throw std::invalid_argument(
                    "kplanes_tilted_fuse_levels_grad_cuda: one grid, upstream gradient, plane gradient, "
                    "H and W per level");
            std::vector<const float *> g(n), go(n);
            std::vector<float *> gg(n);
            for (size_t l = 0; l < n; ++l) {
                g[l] = ptr<const float>(grids[l]);
                go[l] = ptr<const float>(gouts[l]);
                gg[l] = ptr<float>(ggrids[l]);
            }
            check(kplanes_tilted_fuse_levels_grad_cuda(ptr<const float>(pts), ptr<const float>(r), (int)n,
                                                       g.data(), go.data(), gg.data(), H.data(), W.data(),
                                                       ptr<float>(gr), ptr<float>(gpts), B, T, C,
                                                       stream_of(stream)));
        },
        "Backward of kplanes_tilted_fuse_levels_cuda: ggrids per level, gr and gpts summed over levels "
        "(all accumulated into).",
        py::arg("pts_ptr"), py::arg("r_ptr"), py::arg("grid_ptrs"), py::arg("gout_ptrs"),
        py::arg("ggrid_ptrs"), py::arg("H"), py::arg("W"), py::arg("gr_ptr"), py::arg("gpts_ptr"),
        py::arg("B"), py::arg("T"), py::arg("C"), py::arg("stream_ptr"));
    m.attr("KP_MAX_LEVELS") = QC_KP_MAX_LEVELS;

    m.def(
        "kplanes_tilted_fuse_grad_rotations_cuda",
        [](uintptr_t pts, uintptr_t r, uintptr_t grid, uintptr_t gout, uintptr_t ggrid,
           uintptr_t gr, uintptr_t gpts, long B, int T, int C, int H, int W, int t_begin,
           int t_end, uintptr_t stream) {
            check(kplanes_tilted_fuse_grad_rotations_cuda(
                ptr<const float>(pts), ptr<const float>(r), ptr<const float>(grid),
                ptr<const float>(gout), ptr<float>(ggrid), ptr<float>(gr), ptr<float>(gpts), B, T,
                C, H, W, t_begin, t_end, stream_of(stream)));
        },
        "kplanes_tilted_fuse_grad_cuda restricted to rotations [t_begin, t_end).",
        py::arg("pts_ptr"), py::arg("r_ptr"), py::arg("grid_ptr"), py::arg("gout_ptr"),
        py::arg("ggrid_ptr"), py::arg("gr_ptr"), py::arg("gpts_ptr"), py::arg("B"), py::arg("T"),
        py::arg("C"), py::arg("H"), py::arg("W"), py::arg("t_begin"), py::arg("t_end"),
        py::arg("stream_ptr"));

    m.def(
        "kplanes_planes_to_channels_last_cuda",
        [](uintptr_t src, uintptr_t dst, int P, int C, int H, int W, uintptr_t stream) {
            check(kplanes_planes_to_channels_last_cuda(ptr<const float>(src), ptr<float>(dst), P, C,
                                                       H, W, stream_of(stream)));
        },
        py::arg("src_ptr"), py::arg("dst_ptr"), py::arg("P"), py::arg("C"), py::arg("H"),
        py::arg("W"), py::arg("stream_ptr"));

    m.def(
        "kplanes_planes_from_channels_last_cuda",
        [](uintptr_t src, uintptr_t dst, int P, int C, int H, int W, uintptr_t stream) {
            check(kplanes_planes_from_channels_last_cuda(ptr<const float>(src), ptr<float>(dst), P,
                                                         C, H, W, stream_of(stream)));
        },
        py::arg("src_ptr"), py::arg("dst_ptr"), py::arg("P"), py::arg("C"), py::arg("H"),
        py::arg("W"), py::arg("stream_ptr"));

    m.def(
        "kplanes_l2_probe_cuda",
        [](int mode, uintptr_t planes, uintptr_t grad, uintptr_t gout, uintptr_t out, uintptr_t gpts,
           uintptr_t sink, long long pairs, long long npts, int H, int W, uintptr_t stream) {
            check(kplanes_l2_probe_cuda(mode, ptr<const float>(planes), ptr<float>(grad),
                                        ptr<const float>(gout), ptr<float>(out), ptr<float>(gpts),
                                        ptr<float>(sink), pairs, npts, H, W, stream_of(stream)));
        },
        "Diagnostic: the K-Planes kernels' memory traffic (C = 32) without their arithmetic.",
        py::arg("mode"), py::arg("planes_ptr"), py::arg("grad_ptr"), py::arg("gout_ptr"),
        py::arg("out_ptr"), py::arg("gpts_ptr"), py::arg("sink_ptr"), py::arg("pairs"),
        py::arg("npts"), py::arg("H"), py::arg("W"), py::arg("stream_ptr"));
    m.def("kplanes_l2_probe_sink_floats", &kplanes_l2_probe_sink_floats);
    m.attr("KP_PROBE_GATHER") = QC_KP_PROBE_GATHER;
    m.attr("KP_PROBE_REDUCE") = QC_KP_PROBE_REDUCE;
    m.attr("KP_PROBE_BACKWARD") = QC_KP_PROBE_BACKWARD;
    m.attr("KP_PROBE_FORWARD") = QC_KP_PROBE_FORWARD;

    m.def(
        "device_fault_word",
        [](int device, bool clear) {
            unsigned int w = 0;
            check(quantem_cuda_device_fault_word(device, &w, clear ? 1 : 0));
            return w;
        },
        py::arg("device"), py::arg("clear") = false);

    // ── peer memory and the D-slab exchange over it ──
    m.attr("MAX_PEER_RANKS") = QC_MAX_PEER_RANKS;
    m.attr("FAULT_TMA_WAIT") = QC_FAULT_TMA_WAIT;
    m.attr("FAULT_PEER_WAIT") = QC_FAULT_PEER_WAIT;
    m.def("tv_peer_comm_bytes", &tv_peer_comm_bytes);
    m.def(
        "peer_alloc",
        [](size_t bytes) {
            void *p = nullptr;
            check(quantem_cuda_peer_alloc(bytes, &p));
            return reinterpret_cast<uintptr_t>(p);
        },
        py::arg("bytes"));
    m.def("peer_free", [](uintptr_t p) { check(quantem_cuda_peer_free(ptr<void>(p))); },
          py::arg("ptr"));
    m.def(
        "ipc_handle",
        [](uintptr_t p) {
            char h[QC_IPC_HANDLE_BYTES];
            check(quantem_cuda_ipc_handle(ptr<void>(p), h));
            return py::bytes(h, QC_IPC_HANDLE_BYTES);
        },
        py::arg("ptr"));
    m.def(
        "ipc_open",
        [](py::bytes handle) {
            std::string h = handle;
            if (h.size() != QC_IPC_HANDLE_BYTES)
                throw std::invalid_argument("ipc_open: handle must be " +
                                            std::to_string(QC_IPC_HANDLE_BYTES) + " bytes");
            void *p = nullptr;
            check(quantem_cuda_ipc_open(h.data(), &p));
            return reinterpret_cast<uintptr_t>(p);
        },
        py::arg("handle"));
    m.def("ipc_close", [](uintptr_t p) { check(quantem_cuda_ipc_close(ptr<void>(p))); },
          py::arg("ptr"));

    py::class_<qc_peer_group>(m, "PeerGroup")
        .def(py::init(&make_group), py::arg("rank"), py::arg("world"), py::arg("timeout_ns"),
             py::arg("comm"), py::arg("buf"))
        .def_readonly("rank", &qc_peer_group::rank)
        .def_readonly("world", &qc_peer_group::world);
    m.def("peer_allreduce_comm_bytes", &peer_allreduce_comm_bytes);
    m.def(
        "peer_allreduce_sum_f32_cuda",
        [](const qc_peer_group &g, unsigned long long seq, long long n, uintptr_t stream) {
            check(peer_allreduce_sum_f32_cuda(&g, seq, n, stream_of(stream)));
        },
        py::arg("group"), py::arg("seq"), py::arg("n"), py::arg("stream_ptr"));
    m.def(
        "peer_allreduce_sum_f32_range_cuda",
        [](const qc_peer_group &g, unsigned long long seq, long long offset, long long n, int max_ctas,
           uintptr_t stream) {
            check(peer_allreduce_sum_f32_range_cuda(&g, seq, offset, n, max_ctas, stream_of(stream)));
        },
        py::arg("group"), py::arg("seq"), py::arg("offset"), py::arg("n"), py::arg("max_ctas"),
        py::arg("stream_ptr"));
    m.def(
        "peer_allreduce_fault_word",
        [](int device, bool clear) {
            unsigned int w = 0;
            check(peer_allreduce_fault_word(device, &w, clear ? 1 : 0));
            return w;
        },
        py::arg("device"), py::arg("clear") = false);

    py::class_<qc_tv_peers>(m, "TvPeers")
        .def(py::init(&make_peers), py::arg("rank"), py::arg("world"), py::arg("timeout_ns"),
             py::arg("comm"), py::arg("prev_slab"), py::arg("prev_dp"), py::arg("next_slab"),
             py::arg("next_dp"))
        .def_readonly("rank", &qc_tv_peers::rank)
        .def_readonly("world", &qc_tv_peers::world)
        .def_readonly("timeout_ns", &qc_tv_peers::timeout_ns);

    m.def(
        "tv_slab_halo_exchange_cuda",
        [](const qc_tv_peers &peers, unsigned long long seq, uintptr_t slab, int B, int Dp, int H,
           int W, uintptr_t stream) {
            check(tv_slab_halo_exchange_cuda(&peers, seq, ptr<float>(slab), B, Dp, H, W,
                                             stream_of(stream)));
        },
        py::arg("peers"), py::arg("seq"), py::arg("slab_ptr"), py::arg("B"), py::arg("Dp"),
        py::arg("H"), py::arg("W"), py::arg("stream_ptr"));

    m.def(
        "tv_loss_3d_slab_sweep_cuda",
        [](py::object peers, unsigned long long halo_seq, int variant, int flags, uintptr_t vol,
           uintptr_t g, uintptr_t grad, int B, int Dp, int H, int W, int d_lo, int d_hi,
           int has_prev, int has_next, float eps, float scale, uintptr_t ws, size_t ws_bytes,
           uintptr_t stream) {
            const qc_tv_peers *pp = peers.is_none() ? nullptr : peers.cast<const qc_tv_peers *>();
            int n = 0;
            check(tv_loss_3d_slab_sweep_cuda(pp, halo_seq, variant, flags, ptr<const float>(vol),
                                             ptr<const float>(g), ptr<float>(grad), B, Dp, H, W,
                                             d_lo, d_hi, has_prev, has_next, eps, scale,
                                             ptr<void>(ws), ws_bytes, &n, stream_of(stream)));
            return n;
        },
        "One loss's sweep without its finalize; returns the number of CTA partials in ws.",
        py::arg("peers"), py::arg("halo_seq"), py::arg("variant"), py::arg("flags"),
        py::arg("vol_ptr"), py::arg("g_ptr"), py::arg("grad_ptr"), py::arg("B"), py::arg("Dp"),
        py::arg("H"), py::arg("W"), py::arg("d_lo"), py::arg("d_hi"), py::arg("has_prev"),
        py::arg("has_next"), py::arg("eps"), py::arg("acc_scale"), py::arg("ws_ptr"),
        py::arg("ws_bytes"), py::arg("stream_ptr"));

    m.def(
        "tv_loss_3d_peer_finalize_cuda",
        [](const qc_tv_peers &peers, unsigned long long seq, py::list terms, uintptr_t stream) {
            std::vector<qc_tv_term> ts;
            for (auto item : terms) {
                auto t = item.cast<py::tuple>();
                if (t.size() != 6)
                    throw std::invalid_argument(
                        "term = (ws_ptr, n_partials, n_acc, acc_ptr, acc_scale, overwrite)");
                qc_tv_term q{};
                q.workspace = ptr<const void>(t[0].cast<uintptr_t>());
                q.n_partials = t[1].cast<int>();
                q.n_acc = t[2].cast<int>();
                q.acc = ptr<float>(t[3].cast<uintptr_t>());
                q.acc_scale = t[4].cast<float>();
                q.overwrite = t[5].cast<bool>() ? 1 : 0;
                ts.push_back(q);
            }
            check(tv_loss_3d_peer_finalize_cuda(&peers, seq, ts.data(), (int)ts.size(),
                                                stream_of(stream)));
        },
        "Rank-ordered global sums of several sweeps' partials with one cross-rank wait.",
        py::arg("peers"), py::arg("seq"), py::arg("terms"), py::arg("stream_ptr"));

    m.def(
        "tv_loss_3d_slab_peer_cuda",
        [](const qc_tv_peers &peers, unsigned long long halo_seq, unsigned long long seq,
           int variant, int flags, uintptr_t vol, uintptr_t g, uintptr_t acc, uintptr_t grad,
           int B, int Dp, int H, int W, int d_lo, int d_hi, int has_prev, int has_next, float eps,
           float scale, uintptr_t ws, size_t ws_bytes, uintptr_t stream) {
            check(tv_loss_3d_slab_peer_cuda(&peers, halo_seq, seq, variant, flags,
                                            ptr<const float>(vol), ptr<const float>(g),
                                            ptr<float>(acc), ptr<float>(grad), B, Dp, H, W, d_lo,
                                            d_hi, has_prev, has_next, eps, scale, ptr<void>(ws),
                                            ws_bytes, stream_of(stream)));
        },
        py::arg("peers"), py::arg("halo_seq"), py::arg("seq"), py::arg("variant"), py::arg("flags"),
        py::arg("vol_ptr"),
        py::arg("g_ptr"), py::arg("acc_ptr"), py::arg("grad_ptr"), py::arg("B"), py::arg("Dp"),
        py::arg("H"), py::arg("W"), py::arg("d_lo"), py::arg("d_hi"), py::arg("has_prev"),
        py::arg("has_next"), py::arg("eps"), py::arg("acc_scale"), py::arg("ws_ptr"),
        py::arg("ws_bytes"), py::arg("stream_ptr"));
}
