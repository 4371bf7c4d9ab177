/* quantem_cuda_b200.h — C ABI of the B200 (sm_100a) kernels for quantem-cuda's
 * data-parallel hot path: the 3-D total-variation losses and the fused tilted
 * K-Planes interpolation.
 *
 * Every entry point is `extern "C"`, takes raw device pointers, plain integer
 * shapes and a CUDA stream, and never allocates device memory: buffers belong
 * to the caller. All launches are asynchronous on `stream`. An entry point
 * returns 0 on success; otherwise a CUDA runtime error code (1..9999) or one of
 * the QC_ERR_* codes below, and `quantem_cuda_last_error()` returns a message
 * for the calling thread. Launch-time errors are reported at the call; errors
 * raised while a kernel runs surface at the caller's next synchronisation,
 * exactly as in the reference's launchers (csrc/common.cuh:26-33).
 *
 * Layouts (all fp32, C-contiguous):
 *   TV volume           [B, D, H, W]      (B flattens any leading dims)
 *   K-Planes points     [N, 3]            (the reference calls N "B")
 *   K-Planes rotations  [T, 3, 3]         row-major
 *   K-Planes grid       [3T, H, W, C]     channels-last, plane index t*3 + {XY, ZX, YZ}
 *   K-Planes output     [N, T*C]          out[b, t*C + c]
 *
 * Differences from the reference launchers (csrc/ops/core.h, csrc/ops/core/ml.h):
 * each returns an int status instead of throwing std::runtime_error. The
 * entries that replace a reference launcher keep its name and its argument
 * list; everything else (deterministic *_ws_cuda loss forms, single sweeps,
 * D-slabs, peer memory) is an addition under a new name.
 */
#ifndef QUANTEM_CUDA_B200_H
#define QUANTEM_CUDA_B200_H

#include <stddef.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ── status ─────────────────────────────────────────────────────────────── */

#define QC_OK 0
#define QC_ERR_INVALID_ARGUMENT 10001    /* bad shape, null pointer, size overflow */
#define QC_ERR_WORKSPACE_TOO_SMALL 10002 /* workspace_bytes below the required size */
#define QC_ERR_NO_DEVICE 10003           /* no CUDA device / driver entry point missing */
#define QC_ERR_TENSOR_MAP 10004          /* cuTensorMapEncodeTiled rejected the layout */

/* Message describing the last non-zero status returned on this thread. */
const char *quantem_cuda_last_error(void);

/* Human-readable name of a status code. */
const char *quantem_cuda_status_string(int status);

/* CUDART_VERSION the library was compiled against (e.g. 12090).
 * Replaces the reference's `_core.__cudart_version__` (csrc/bindings.cpp:24). */
int quantem_cuda_cudart_version(void);

/* Reads (and, if `clear` != 0, resets) the device-side fault word of `device`:
 * the OR of every kernel family's bits. Kernels that wait (on a TMA barrier, on
 * another rank) give up after a bounded time and set a bit here instead of
 * hanging; the library built with QC_DEBUG_BOUNDS (libquantem_cuda_b200_debug.so)
 * also sets QC_FAULT_BOUNDS when a computed index falls outside its buffer and
 * skips that access. 0 means nothing happened. Synchronises the device. */
int quantem_cuda_device_fault_word(int device, unsigned int *word, int clear);

/* ── 3-D total variation ────────────────────────────────────────────────── */

/* Bytes of scratch the deterministic TV loss entry points (*_ws_cuda, the
 * single-sweep *_fwd_grad_cuda, tv_loss_3d_slab_cuda) need for a
 * [B, D, H, W] volume. */
size_t tv_loss_3d_workspace_bytes(int B, int D, int H, int W);

/* The reference's three loss launchers, same arguments in the same order
 * (csrc/ops/core.h:16-22, :40-45, :62-67; bound in Python as
 * csrc/bindings/core.cpp:101-148). acc is pre-zeroed by the caller and
 * receives acc += Σ; as in the reference, every CTA adds its sum with an fp32
 * atomic, so the last bits can differ from run to run. The *_ws_cuda forms
 * below compute the same sums deterministically. */

/* Isotropic TV: acc[0] += Σ_b Σ_corners sqrt(dd² + dh² + dw² + eps), corners
 * [0,D-2]×[0,H-2]×[0,W-2]. Replaces tv_loss_iso_3d_cuda
 * (reference csrc/ops/core.h:16-22, csrc/cuda/core/tv_loss.cu:98-121). */
int tv_loss_iso_3d_cuda(const float *d_vol, float *d_acc, int B, int D, int H, int W, float eps,
                        cudaStream_t stream);

/* Squared-anisotropic TV: acc[0] += Σ_b Σ_axes Σ (forward difference)², each axis
 * over its full complementary range. Replaces tv_loss_sq_3d_cuda
 * (reference csrc/ops/core.h:40-45, tv_loss.cu:276-294). */
int tv_loss_sq_3d_cuda(const float *d_vol, float *d_acc, int B, int D, int H, int W,
                       cudaStream_t stream);

/* L1-anisotropic TV: acc[axis] += Σ_b Σ |forward difference along axis|, axis
 * order (D, H, W). Replaces tv_loss_l1_3d_cuda (reference csrc/ops/core.h:62-67,
 * tv_loss.cu:411-429). */
int tv_loss_l1_3d_cuda(const float *d_vol, float *d_acc, int B, int D, int H, int W,
                       cudaStream_t stream);

/* The same three sums, deterministic: each CTA writes an fp64 partial into a
 * caller-owned scratch buffer (`workspace`, at least
 * tv_loss_3d_workspace_bytes() bytes, contents need no initialisation) and
 * one finalize kernel adds the partials in a fixed order, so acc receives the
 * same bits on every run. Calls that share one workspace must be ordered on
 * the GPU (one stream, or events). No counterpart in the reference, whose
 * sums are atomic (tv_loss.cu:95, :273, :404-408). */
int tv_loss_iso_3d_ws_cuda(const float *d_vol, float *d_acc, int B, int D, int H, int W, float eps,
                           void *d_workspace, size_t workspace_bytes, cudaStream_t stream);
int tv_loss_sq_3d_ws_cuda(const float *d_vol, float *d_acc, int B, int D, int H, int W,
                          void *d_workspace, size_t workspace_bytes, cudaStream_t stream);
int tv_loss_l1_3d_ws_cuda(const float *d_vol, float *d_acc, int B, int D, int H, int W,
                          void *d_workspace, size_t workspace_bytes, cudaStream_t stream);

/* Gradient of the isotropic sum times *d_g_scaled (upstream / N); grad_vol is
 * fully written (zero when a dim is < 2). Replaces tv_loss_iso_3d_grad_cuda
 * (reference csrc/ops/core.h:27-34, tv_loss.cu:194-218). */
int tv_loss_iso_3d_grad_cuda(const float *d_vol, const float *d_g_scaled, float *d_grad_vol,
                             int B, int D, int H, int W, float eps, cudaStream_t stream);

/* 2·g·∇ of the squared sum; grad_vol fully written. Replaces
 * tv_loss_sq_3d_grad_cuda (reference csrc/ops/core.h:50-56, tv_loss.cu:334-352). */
int tv_loss_sq_3d_grad_cuda(const float *d_vol, const float *d_g, float *d_grad_vol, int B, int D,
                            int H, int W, cudaStream_t stream);

/* Σ_axis g[axis]·∇ of the per-axis L1 sums, sign(0) = 0; grad_vol fully
 * written. Replaces tv_loss_l1_3d_grad_cuda (reference csrc/ops/core.h:72-78,
 * tv_loss.cu:477-495). */
int tv_loss_l1_3d_grad_cuda(const float *d_vol, const float *d_g, float *d_grad_vol, int B, int D,
                            int H, int W, cudaStream_t stream);

/* Single-sweep forward + gradient: one HBM pass reads the volume once and
 * writes both the loss (acc += Σ, deterministic as in the *_ws_cuda entries,
 * same workspace) and the gradient
 * (as the *_grad_cuda entries, scaled by the device scalar(s) at d_g). No
 * reference counterpart: the reference runs the loss and gradient kernels as
 * two passes (tv_loss.cu:47-96 then :140-192, and likewise for sq and L1). */
int tv_loss_iso_3d_fwd_grad_cuda(const float *d_vol, const float *d_g_scaled, float *d_acc,
                                 float *d_grad_vol, int B, int D, int H, int W, float eps,
                                 void *d_workspace, size_t workspace_bytes, cudaStream_t stream);
int tv_loss_sq_3d_fwd_grad_cuda(const float *d_vol, const float *d_g, float *d_acc,
                                float *d_grad_vol, int B, int D, int H, int W, void *d_workspace,
                                size_t workspace_bytes, cudaStream_t stream);
int tv_loss_l1_3d_fwd_grad_cuda(const float *d_vol, const float *d_g, float *d_acc,
                                float *d_grad_vol, int B, int D, int H, int W, void *d_workspace,
                                size_t workspace_bytes, cudaStream_t stream);

/* Several TV terms of one volume in one sweep: the volume is read once, each
 * term's loss sums are accumulated, and one gradient — the gain-weighted sum
 * of the terms' gradients — is written. No counterpart in the reference,
 * which runs one loss kernel and one gradient kernel per term; a caller that
 * regularises with two or three terms (isotropic + L1, squared + isotropic)
 * reads the volume once instead of once per term.
 *   terms: two or three of QC_TV_TERM_SQ, QC_TV_TERM_ISO, QC_TV_TERM_L1
 *   flags: 0 (acc += ...) or QC_TV_ACC_OVERWRITE (acc = ...)
 *   d_acc: 5 device floats, the losses [Σsq, iso_scale·Σiso, Σ|Δd|, Σ|Δh|,
 *          Σ|Δw|] (iso_scale = 1/N gives the isotropic mean); slots of terms
 *          not requested receive 0 (or are left as they were)
 *   d_g:   5 device floats, the upstream gradient of each of those losses:
 *          the gradient written is g_sq·∇Σsq + g_iso·iso_scale·∇Σiso +
 *          Σ_axis g_axis·∇Σ|Δ_axis|
 * Deterministic (fixed-order reduction through the workspace, at least
 * tv_loss_3d_workspace_bytes() bytes). */
#define QC_TV_TERM_SQ 1
#define QC_TV_TERM_ISO 2
#define QC_TV_TERM_L1 4
int tv_loss_mix_3d_fwd_grad_cuda(int terms, int flags, const float *d_vol, const float *d_g,
                                 float *d_acc, float *d_grad_vol, int B, int D, int H, int W,
                                 float eps, float iso_scale, void *d_workspace,
                                 size_t workspace_bytes, cudaStream_t stream);

/* tv_loss_iso_3d_fwd_grad_cuda without a workspace, for callers that cannot
 * call cudaMalloc where they compute the loss: applications whose device
 * memory is owned up front by one allocator or a fixed budget, and hosts that
 * allocate only at start-up. No counterpart in the reference. The reduction
 * scratch is a 48 KiB array statically allocated in the library's device code
 * (every GPU that loads the library holds it until exit); it covers every
 * volume shape, since the planner never uses more CTAs than it has slots.
 * Shapes beyond the largest volume (H*W or B*D at or above 2^31) are refused
 * with QC_ERR_INVALID_ARGUMENT. The entry allocates nothing, but it still
 * launches kernels, and its first call on a device also does host-side set-up
 * (it looks up the array's device address with that device current, sets
 * kernel attributes, may load the module): make that first call before any
 * stream capture. Do not use it across a cudaDeviceReset (the looked-up
 * address is kept). Every call shares the array, which keeps the previous
 * call's partial sums (nothing in it needs to start at zero): calls that
 * overlap on the GPU (other streams, other threads) race. */
int tv_loss_iso_3d_fwd_grad_noalloc_cuda(const float *d_vol, const float *d_g_scaled, float *d_acc,
                                         float *d_grad_vol, int B, int D, int H, int W, float eps,
                                         cudaStream_t stream);

/* General D-slab form behind all TV entries, used directly by the sharded
 * (multi-GPU) path. The volume holds Dp physical planes per batch slice; planes
 * [d_lo, d_hi) are owned. has_prev / has_next say whether plane d_lo-1 / d_hi is
 * a real neighbour (a halo received from another rank) rather than the edge of
 * the global volume. Loss terms anchored at owned planes are summed, and the
 * gradient of owned planes is written (planes outside [d_lo, d_hi) are left
 * untouched).
 *   variant: QC_TV_SQ, QC_TV_ISO, QC_TV_L1
 *   flags:   QC_TV_LOSS and/or QC_TV_GRAD, optionally QC_TV_ACC_OVERWRITE
 *            (acc = scale·Σ instead of acc += scale·Σ)
 *   d_g:     device scalar (sq, iso) or 3-vector (L1) multiplying the gradient
 *   acc_scale multiplies both the stored sum and the gradient (the isotropic
 *            op passes 1/N, folding the mean into the kernel). */
#define QC_TV_SQ 0
#define QC_TV_ISO 1
#define QC_TV_L1 2
#define QC_TV_LOSS 1
#define QC_TV_GRAD 2
#define QC_TV_ACC_OVERWRITE 4
int tv_loss_3d_slab_cuda(int variant, int flags, const float *d_vol, const float *d_g, float *d_acc,
                         float *d_grad_vol, int B, int Dp, int H, int W, int d_lo, int d_hi,
                         int has_prev, int has_next, float eps, float acc_scale, void *d_workspace,
                         size_t workspace_bytes, cudaStream_t stream);

/* ── D-slabs over peer memory (one process per GPU, GPUs of one node) ──────
 *
 * No counterpart in the reference, which is single-GPU. Each rank keeps its
 * slab [B, Dp, H, W] (planes 1..Dp-2 owned, halos 0 and Dp-1) and a small
 * communication block in memory allocated with quantem_cuda_peer_alloc and
 * mapped into its neighbours with CUDA IPC. The halo exchange and the
 * cross-rank loss reduction are kernels that store into the peers' memory
 * over NVLink and signal with release/acquire flags, so a step issues no
 * library collective and never synchronises the host.
 *
 * Every rank makes the same sequence of calls. `seq` numbers the calls of one
 * entry point (the halo exchange and the reduction keep separate counters):
 * 1 for the first call, +1 for each later call, the same on every rank. Waits
 * on another rank give up after `timeout_ns` (0: 10 s), set
 * QC_FAULT_PEER_WAIT in the device fault word and (for the reduction) store
 * NaN in the loss, so a rank that stops never hangs the others. */
#define QC_MAX_PEER_RANKS 8
#define QC_TV_MAX_PEER_SUMS 8 /* loss sums one cross-rank finalize carries (iso 1 + L1 3 + sq 1 fit) */
#define QC_IPC_HANDLE_BYTES 64
#define QC_FAULT_TMA_WAIT 0x1u  /* a kernel gave up waiting for its own TMA copies */
#define QC_FAULT_PEER_WAIT 0x2u /* a kernel gave up waiting for another rank */
#define QC_FAULT_BOUNDS 0x4u    /* debug builds (QC_DEBUG_BOUNDS): an index out of range was skipped */

typedef struct qc_tv_peers {
    int rank;                          /* this rank, 0 <= rank < world */
    int world;                         /* ranks in the D split, <= QC_MAX_PEER_RANKS */
    unsigned long long timeout_ns;     /* bound on every wait for another rank (0: 10 s) */
    void *comm[QC_MAX_PEER_RANKS];     /* every rank's communication block, mapped in this
                                          process (comm[rank] is this rank's own) */
    float *prev_slab;                  /* rank-1's slab mapped here (NULL on rank 0) */
    float *next_slab;                  /* rank+1's slab mapped here (NULL on the last rank) */
    int prev_dp;                       /* Dp of rank-1's slab */
    int next_dp;                       /* Dp of rank+1's slab */
} qc_tv_peers;

/* Device memory that other processes can map: cudaMalloc, zero-filled before
 * returning (synchronous). Free with quantem_cuda_peer_free. */
int quantem_cuda_peer_alloc(size_t bytes, void **d_ptr);
int quantem_cuda_peer_free(void *d_ptr);
/* CUDA IPC handle (QC_IPC_HANDLE_BYTES bytes) of a quantem_cuda_peer_alloc
 * allocation, and its mapping in another process (with peer access enabled). */
int quantem_cuda_ipc_handle(void *d_ptr, void *handle_out);
int quantem_cuda_ipc_open(const void *handle, void **d_ptr);
int quantem_cuda_ipc_close(void *d_ptr);

/* Bytes of one rank's communication block (flags and reduction slots). */
size_t tv_peer_comm_bytes(void);

/* Fills the halo planes of d_slab [B, Dp, H, W] (this rank's own slab, which
 * its neighbours have mapped): plane 1 goes into rank-1's plane prev_dp-1 and
 * plane Dp-2 into rank+1's plane 0, each after that neighbour has signalled
 * that its earlier work on the stream is done; returns (on the GPU) once both
 * neighbours' planes have arrived here. The sweeps that read the halos must be
 * on the same stream as the next exchange. */
int tv_slab_halo_exchange_cuda(const qc_tv_peers *peers, unsigned long long seq, float *d_slab,
                               int B, int Dp, int H, int W, cudaStream_t stream);

/* tv_loss_3d_slab_cuda with the loss summed over all ranks inside the
 * finalize kernel: each rank's fixed-order fp64 total goes to every rank's
 * communication block, and every rank adds the totals in rank order, so d_acc
 * holds the same bits on every rank. flags must include QC_TV_LOSS; `seq`
 * numbers the reductions. If halo_seq != 0 the call first exchanges the halos
 * (what tv_slab_halo_exchange_cuda does with that sequence number; d_vol is
 * then this rank's slab with owned planes [1, Dp-1)): on the TMA path the
 * sweep kernel itself stores the boundary planes into the neighbours at its
 * start and waits for each halo plane just before it loads it, so the
 * exchange costs no separate launch and overlaps the interior of the sweep. */
int tv_loss_3d_slab_peer_cuda(const qc_tv_peers *peers, unsigned long long halo_seq,
                              unsigned long long seq, int variant, int flags, const float *d_vol,
                              const float *d_g, float *d_acc, float *d_grad_vol, int B, int Dp,
                              int H, int W, int d_lo, int d_hi, int has_prev, int has_next,
                              float eps, float acc_scale, void *d_workspace,
                              size_t workspace_bytes, cudaStream_t stream);

/* Two-phase form, for several losses of one step with a single cross-rank
 * wait: tv_loss_3d_slab_sweep_cuda launches one loss's sweep (gradient written
 * as usual; with QC_TV_LOSS its CTA partial sums stay in d_workspace, their
 * count in *n_partials), and tv_loss_3d_peer_finalize_cuda then turns the
 * partials of up to QC_TV_MAX_PEER_SUMS sums (each term's workspace must stay
 * untouched until then) into the rank-ordered global sums, one wait for all
 * terms. peers may be NULL in the sweep call when halo_seq is 0. */
typedef struct qc_tv_term {
    const void *workspace; /* the sweep's workspace */
    int n_partials;        /* as returned by the sweep */
    int n_acc;             /* 1 (sq, iso) or 3 (L1) */
    float *acc;            /* device sums, n_acc floats */
    float acc_scale;       /* multiplies the global sums */
    int overwrite;         /* acc = scale·Σ (else acc += scale·Σ) */
} qc_tv_term;

int tv_loss_3d_slab_sweep_cuda(const qc_tv_peers *peers, unsigned long long halo_seq, int variant,
                               int flags, const float *d_vol, const float *d_g,
                               float *d_grad_vol, int B, int Dp, int H, int W, int d_lo, int d_hi,
                               int has_prev, int has_next, float eps, float acc_scale,
                               void *d_workspace, size_t workspace_bytes, int *n_partials,
                               cudaStream_t stream);
int tv_loss_3d_peer_finalize_cuda(const qc_tv_peers *peers, unsigned long long seq,
                                  const qc_tv_term *terms, int n_terms, cudaStream_t stream);

/* ── sum of one fp32 buffer over the GPUs of a node, over peer memory ──────
 *
 * No counterpart in the reference. Every rank's buffer (n floats, allocated
 * with quantem_cuda_peer_alloc) and communication block
 * (peer_allreduce_comm_bytes) are mapped into every process. One kernel:
 * rank r adds chunk r of all buffers in rank order and stores the sum into
 * chunk r of every buffer, so after the call every buffer holds the sum,
 * bitwise identical on every rank and run to run. `seq` numbers the calls
 * (1, 2, ...; the same on every rank). Waits on other ranks are bounded
 * (timeout_ns, 0: 10 s) and set QC_FAULT_PEER_WAIT in the word that
 * peer_allreduce_fault_word reads. */
typedef struct qc_peer_group {
    int rank;
    int world;
    unsigned long long timeout_ns;
    void *comm[QC_MAX_PEER_RANKS];  /* every rank's communication block, mapped here */
    float *buf[QC_MAX_PEER_RANKS];  /* every rank's buffer, mapped here (buf[rank] own) */
} qc_peer_group;

size_t peer_allreduce_comm_bytes(void);
int peer_allreduce_sum_f32_cuda(const qc_peer_group *group, unsigned long long seq, long long n,
                                cudaStream_t stream);
/* The same sum over floats [offset, offset + n) of every buffer only (any
 * offset; the caller keeps offset + n within every rank's buffer, whose size
 * the group does not record), in one launch of at most max_ctas CTAs (0: two
 * per SM). A small
 * max_ctas lets the sum of one range run beside other work on the GPU, e.g.
 * the backward of the rotations whose gradients fill the next range. Calls
 * share `seq` numbering with peer_allreduce_sum_f32_cuda. */
int peer_allreduce_sum_f32_range_cuda(const qc_peer_group *group, unsigned long long seq,
                                      long long offset, long long n, int max_ctas, cudaStream_t stream);
int peer_allreduce_fault_word(int device, unsigned int *word, int clear);

/* ── tilted K-Planes ────────────────────────────────────────────────────── */

/* out[b, t*C + c] = Π_{p∈XY,ZX,YZ} bilinear(grid[t*3+p], (R_t·pts_b) pair p), with
 * grid_sample(align_corners=True, padding_mode="border") semantics; out fully
 * written. Replaces kplanes_tilted_fuse_cuda (reference csrc/ops/core/ml.h:17-24,
 * csrc/cuda/core/ml/kplanes_tilted.cu:289-302). Requires C*H*W < 2^31. */
int kplanes_tilted_fuse_cuda(const float *d_pts, const float *d_R, const float *d_grid,
                             float *d_out, long B, int T, int C, int H, int W,
                             cudaStream_t stream);

/* Backward: ggrid [3T,H,W,C], gR [T,3,3] and gpts [N,3] are accumulated into
 * (caller pre-zeroes for a plain gradient). Coordinate gradients are zero where
 * the border clip engaged. Replaces kplanes_tilted_fuse_grad_cuda (reference
 * csrc/ops/core/ml.h:26-40, kplanes_tilted.cu:304-327). */
int kplanes_tilted_fuse_grad_cuda(const float *d_pts, const float *d_R, const float *d_grid,
                                  const float *d_gout, float *d_ggrid, float *d_gR, float *d_gpts,
                                  long B, int T, int C, int H, int W, cudaStream_t stream);

/* The backward restricted to rotations [t_begin, t_end): accumulates the
 * gradient of those rotations' planes (grid planes 3*t_begin .. 3*t_end-1) and
 * rows of gR, and their share of gpts; the other outputs are not touched.
 * Summing the calls over a partition of [0, T) gives the full backward (up to
 * the order of the gpts additions). No counterpart in the reference: it lets a
 * multi-GPU caller start reducing one rotation's plane gradient across ranks
 * while the next rotation's backward runs. */
int kplanes_tilted_fuse_grad_rotations_cuda(const float *d_pts, const float *d_R,
                                            const float *d_grid, const float *d_gout,
                                            float *d_ggrid, float *d_gR, float *d_gpts, long B,
                                            int T, int C, int H, int W, int t_begin, int t_end,
                                            cudaStream_t stream);

/* Several levels of one multiscale tilted K-Planes encoding (the caller's
 * loop over resolutions: one rotation set, one point set, the planes of each
 * level at their own H x W, all with C channels) in one launch each way.
 * `grids`, `outs`, `gouts`, `ggrids`, `H` and `W` are HOST arrays of
 * n_levels entries (1 <= n_levels <= QC_KP_MAX_LEVELS) holding device
 * pointers and sizes; level l is exactly kplanes_tilted_fuse_cuda /
 * kplanes_tilted_fuse_grad_cuda on grids[l] (channels-last [3T, H[l], W[l], C],
 * outs[l] and gouts[l] [N, T*C]). The backward accumulates each level's plane
 * gradient into ggrids[l] and the sum over levels into gR and gpts. No
 * counterpart in the reference (its caller, quantem's multiscale K-Planes
 * encoder, calls the single-level op once per level). */
#define QC_KP_MAX_LEVELS 8
int kplanes_tilted_fuse_levels_cuda(const float *d_pts, const float *d_R, int n_levels,
                                    const float *const *grids, float *const *outs, const int *H,
                                    const int *W, long B, int T, int C, cudaStream_t stream);
int kplanes_tilted_fuse_levels_grad_cuda(const float *d_pts, const float *d_R, int n_levels,
                                         const float *const *grids, const float *const *gouts,
                                         float *const *ggrids, const int *H, const int *W,
                                         float *d_gR, float *d_gpts, long B, int T, int C,
                                         cudaStream_t stream);

/* Tilted K-Planes at four taps for finite-difference TV regularisation:
 * out[k, b, t*C + c] samples at R_t·p (k = 0, bit-identical to
 * kplanes_tilted_fuse_cuda) and at R_t·p + h·R_t[:, k-1] (k = 1, 2, 3); out is
 * [4, N, T*C], fully written. Replaces kplanes_tilted_tv_fuse_cuda (reference
 * csrc/ops/core/ml.h:51-62, csrc/cuda/core/ml/kplanes_tilted.cu:329-425). */
int kplanes_tilted_tv_fuse_cuda(const float *d_pts, const float *d_R, const float *d_grid,
                                float *d_out, long B, int T, int C, int H, int W, float h,
                                cudaStream_t stream);

/* Backward of the four-tap form: gout is [4, N, T*C]; ggrid, gR and gpts are
 * accumulated into as in kplanes_tilted_fuse_grad_cuda. R_t receives both the
 * R_t·p term of every tap and, for taps 1..3, h·dL/dr in column k-1. Replaces
 * kplanes_tilted_tv_fuse_grad_cuda (reference csrc/ops/core/ml.h:64-77,
 * kplanes_tilted.cu:427-612). */
int kplanes_tilted_tv_fuse_grad_cuda(const float *d_pts, const float *d_R, const float *d_grid,
                                     const float *d_gout, float *d_ggrid, float *d_gR,
                                     float *d_gpts, long B, int T, int C, int H, int W, float h,
                                     cudaStream_t stream);

/* Diagnostic, no counterpart in the reference: the memory traffic of the
 * K-Planes kernels at C = 32 without their arithmetic, to measure the L2-side
 * ceiling of their access pattern. `pairs` (point, rotation) pairs each touch
 * 12 channel rows of 128 B at hashed cells of three [H, W, 32] planes:
 *   QC_KP_PROBE_GATHER    gathers them;
 *   QC_KP_PROBE_REDUCE    adds a red.global.add.v4.f32 per 16 B into d_grad;
 *   QC_KP_PROBE_BACKWARD  gathers, reduces, reads a 128-B row of d_gout and adds
 *                         3 floats to d_gpts (the backward's traffic);
 *   QC_KP_PROBE_FORWARD   gathers and writes a 128-B row of d_out (the forward's).
 * Buffers: d_planes and d_grad 3*H*W*32 floats, d_gout and d_out pairs*32,
 * d_gpts npts*3, d_sink kplanes_l2_probe_sink_floats() floats. */
#define QC_KP_PROBE_GATHER 0
#define QC_KP_PROBE_REDUCE 1
#define QC_KP_PROBE_BACKWARD 2
#define QC_KP_PROBE_FORWARD 3
int kplanes_l2_probe_cuda(int mode, const float *d_planes, float *d_grad, const float *d_gout,
                          float *d_out, float *d_gpts, float *d_sink, long long pairs,
                          long long npts, int H, int W, cudaStream_t stream);
size_t kplanes_l2_probe_sink_floats(void);

/* Plane layout conversion [P, C, H, W] -> [P, H, W, C] and back. Replaces the
 * torch permute+contiguous of the reference's op layer
 * (src/quantem/cuda/core/ml/_ops.py:21-25, :82). src and dst must not overlap. */
int kplanes_planes_to_channels_last_cuda(const float *d_src, float *d_dst, int P, int C, int H,
                                         int W, cudaStream_t stream);
int kplanes_planes_from_channels_last_cuda(const float *d_src, float *d_dst, int P, int C, int H,
                                           int W, cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* QUANTEM_CUDA_B200_H */
