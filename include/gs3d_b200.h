/*
 * gs3d_b200.h — C ABI of the B200 (sm_100a) 3D Gaussian Splatting rasterizer.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream handle
 * (cudaStream_t passed as void*; NULL means the legacy default stream) and returns an
 * int status (GS_OK or a GS_ERR_* code). On failure gs_last_error() returns a message
 * for the calling thread. No entry point allocates device memory except where stated;
 * scratch memory ("workspace") is supplied by the caller and sized by the *_workspace_size
 * queries. All work is enqueued asynchronously on `stream`.
 *
 * Tensor layouts are those of the reference pybind11 module `custom_rasterizer_cuda`
 * (csrc/bindings.cpp:141-151): row-major fp32, int32 for ids / ranges / counts.
 *   mu[N,3]  q[N,4] (w,x,y,z)  s[N,3] (log-scale)  R[3,3] (world->camera, row-major)  t[3]
 *   mean2d[N,2]  cov2d[N,3] = (a,b,c) of [[a,b],[b,c]]  depths[N]  colors[N,3]
 *   albedo[N,3] (SH DC)  k_j[N,15,3] (SH degrees 1..3, coefficient-major then RGB)
 *   img[H,W,3]  final_T[H,W]  n_contrib[H,W]  tile_ranges[T,2]  with T = ceil(W/16)*ceil(H/16)
 */
#ifndef GS3D_B200_H
#define GS3D_B200_H

#include <stddef.h>

#if defined(__GNUC__)
#define GS_API __attribute__((visibility("default")))
#else
#define GS_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define GS_OK 0
#define GS_ERR_INVALID_ARG 1   /* bad size, null pointer or misaligned buffer */
#define GS_ERR_CUDA 2          /* a CUDA runtime call or launch failed */
#define GS_ERR_CAPACITY 3      /* pair count M exceeded the caller's capacity */
#define GS_ERR_DEVICE 4        /* a device-side check failed (see gs_device_error_bits) */

/* Message describing the last error raised on the calling thread ("" if none). */
GS_API const char* gs_last_error(void);
/* Library version string. */
GS_API const char* gs_version(void);

/*
 * Projection forward. Replaces `project` (csrc/bindings.cpp:12-29, kernel
 * csrc/forward/projection.cu:12-107). Gaussians with camera-space z <= 0.2 get zeros in
 * all three outputs, as the reference's zero-initialised outputs do.
 */
GS_API int gs_project(int N, const float* mu, const float* q, const float* s, const float* R,
               const float* t, float fx, float fy, float cx, float cy, float* mean2d,
               float* cov2d, float* depths, void* stream);

/*
 * Spherical-harmonic colour forward, degrees 0..3. Replaces `SH`
 * (csrc/bindings.cpp:32-46, kernel csrc/forward/SH.cu:57-93). `cam_pos` is a DEVICE
 * pointer to 3 floats; unlike the reference no host copy of it is made.
 */
GS_API int gs_sh_forward(int N, const float* cam_pos, const float* mu, const float* albedo,
                  const float* k_j, float* colors, void* stream);

/*
 * Bytes of caller-provided workspace gs_rasterize needs for N Gaussians, an H x W image
 * and room for `pair_capacity` (tile, Gaussian) pairs.
 */
GS_API size_t gs_rasterize_workspace_size(int N, int H, int W, long long pair_capacity);

/*
 * Tile binning, depth/tile sort, tile ranges and the front-to-back alpha blend.
 * Replaces `rasterize` (csrc/bindings.cpp:50-70, host csrc/forward/rasterize.cu:284-486).
 * Outputs: img[H,W,3], sorted_ids[pair_capacity] (the first M are valid), tile_ranges[T,2]
 * (empty tiles (0,0)), final_T[H,W], n_contrib[H,W].
 * The pair count M is written to *pair_count_dev (a device int inside or outside the
 * workspace) and, when pair_count_host is non-NULL (pinned host memory), copied there
 * asynchronously; when `m_ready_event` (a cudaEvent_t) is non-NULL it is recorded right
 * after that copy, so a caller can learn M long before the blend finishes.
 * If M > pair_capacity every pair-dependent kernel does nothing and the caller must call
 * again with pair_capacity >= M (the status is still GS_OK: the overflow is only known
 * on the device). N == 0 or M == 0 produce zero images, final_T = 1, n_contrib = 0 and
 * zero ranges, as the reference does (rasterize.cu:306-319).
 */
GS_API int gs_rasterize(int N, int H, int W, const float* depths, const float* mean2d,
                 const float* cov2d, const float* colors, const float* alpha, void* workspace,
                 size_t workspace_bytes, long long pair_capacity, float* img, int* sorted_ids,
                 int* tile_ranges, float* final_T, int* n_contrib, int* pair_count_dev,
                 int* pair_count_host, void* m_ready_event, void* stream);

/*
 * gs_rasterize without a workspace, for callers that cannot allocate device memory when they
 * render (a plugin given only its input and output buffers, a process whose device memory is
 * reserved by another allocator, a per-frame path that must not hit cudaMalloc's device
 * synchronisation). No counterpart in the reference: it adds an allocation-free way in.
 * Binning/sort scratch comes from a 16 MiB array compiled into the library (held on every
 * device that loads it); calls whose layout for (N, H, W, pair_capacity) does not fit return
 * GS_ERR_CAPACITY before any GPU work. The first call on a device looks the array's address up
 * (cudaGetSymbolAddress), so make it before any stream capture, and do not call it again after
 * cudaDeviceReset in the same process (the cached address would be stale). Calls share the
 * array: GPU work of overlapping calls races and must be serialised by the caller. Outputs as
 * gs_rasterize; nothing is allocated. `pair_count_dev` is REQUIRED (a device int; NULL is
 * GS_ERR_INVALID_ARG): it receives M, and when M > pair_capacity the call writes none of img,
 * final_T, n_contrib, tile_ranges or sorted_ids (status GS_OK, the overflow is only known on
 * the device), so the caller must read M and call again with pair_capacity >= M.
 */
GS_API int gs_rasterize_noalloc(int N, int H, int W, const float* depths, const float* mean2d,
                                const float* cov2d, const float* colors, const float* alpha,
                                long long pair_capacity, float* img, int* sorted_ids,
                                int* tile_ranges, float* final_T, int* n_contrib,
                                int* pair_count_dev, void* stream);

/* Bytes of workspace gs_rasterize_backward needs for N Gaussians. */
GS_API size_t gs_rasterize_backward_workspace_size(int N);

/*
 * Backward of the alpha blend. Replaces `backwards_rasterization`
 * (csrc/bindings.cpp:72-100, kernel csrc/backward/rasterize_backward.cu:6-236).
 * Gradient outputs are ACCUMULATED (atomic adds) and must be zeroed by the caller:
 * g_mean2d[N,2], g_cov2d[N,3] (dL/dSigma2, not dL/dconic), g_colors[N,3], g_alpha[N].
 * `sorted_ids` holds the tile-sorted Gaussian ids addressed by tile_ranges; out-of-range
 * ids are skipped, as in the reference.
 */
GS_API int gs_rasterize_backward(int N, int H, int W, const float* grad_img, const float* mean2d,
                          const float* cov2d, const float* colors, const float* alpha,
                          const int* sorted_ids, const int* tile_ranges, const float* final_T,
                          const int* n_contrib, void* workspace, size_t workspace_bytes,
                          float* g_mean2d, float* g_cov2d, float* g_colors, float* g_alpha,
                          void* stream);

/*
 * Backward of the SH colour. Replaces `backwards_SH` (csrc/bindings.cpp:102-116, kernel
 * csrc/backward/delight_backward.cu:107-174). Outputs are overwritten (not accumulated).
 */
GS_API int gs_sh_backward(int N, const float* grad_colors, const float* mu, const float* albedo,
                   const float* k_j, const float* cam_pos, float* g_albedo, float* g_k_j,
                   float* g_mu, void* stream);

/*
 * Backward of the projection. Replaces `backwards_projection` (csrc/bindings.cpp:118-139,
 * kernel csrc/backward/projection_backward.cu:11-140). Outputs are overwritten; culled
 * Gaussians (z <= 0.2) get zeros.
 */
GS_API int gs_project_backward(int N, const float* g_mean2d, const float* g_cov2d, const float* mu,
                        const float* q, const float* s, const float* R, const float* t,
                        float fx, float fy, float cx, float cy, float* g_mu, float* g_q,
                        float* g_s, void* stream);

/*
 * Fused render path (what RasterizeFunction runs): the six reference ops of one view in two
 * calls. The reference wrapper chains project -> SH -> rasterize and their backwards
 * (gaussian_splatting/rasterizer/rasterize.py:43-117); these give the same outputs without
 * writing mean2d / cov2d / depths / colours to memory.
 *
 * gs_render_forward: opacity[N] (post-sigmoid), cam_pos = -R^T t (device, 3 floats, as the
 * wrapper computes it). Outputs as gs_rasterize plus radii[N], the wrapper's screen radii
 * 3 sqrt(max(mid + sqrt(max(((a-c)/2)^2 + b^2, 0.1)), 0)) (rasterize.py:49-53). The workspace
 * (gs_render_workspace_size) must be kept for gs_render_backward, which reads the forward's
 * blend records from it.
 * gs_render_backward: gradients of every parameter (g_opacity w.r.t. the post-sigmoid
 * opacity) and, when g_mean2d is non-NULL, dL/dmean2d. With accumulate = 0 the outputs are
 * overwritten; otherwise the gradients are added to them. When the three stat_* buffers [N] are
 * given, the reference trainer's densification statistics are updated in the same pass
 * (gaussian_splatting/utils/adc.py:58-87): n = |dL/dmean2d * (stat_scale_x, stat_scale_y)|,
 * and where n > 0, stat_norm_sum += n, stat_count += 1, stat_max = max(stat_max, n).
 * accum_wait_event / accum_done_event (cudaEvent_t or NULL): the kernel that writes the gradient
 * and statistic buffers waits for the first and the second is recorded after it, so that views
 * rendered concurrently on several streams can accumulate into the same buffers. flags: 0 or
 * GS_RENDER_CONCURRENT.
 */
/* gs_render_forward flags. GS_RENDER_TIGHT_BINS: bin each splat only into the tiles of its
 * reference rectangle that hold a pixel of its opacity-test extent box (the region where
 * o exp(power) >= 1/255 can hold, inflated). The image, final_T and every gradient of
 * gs_render_backward are unchanged, because the dropped pairs fail the opacity test at every
 * pixel of their tile; M is smaller, so sorted_ids, tile_ranges and n_contrib (a list position)
 * differ from the reference's. Without the flag all outputs match the reference's. */
#define GS_RENDER_TIGHT_BINS 1u
/* GS_RENDER_CONCURRENT (gs_render_forward and gs_render_backward): the caller overlaps several
 * views on different streams. The blend kernels then run with more pixels per thread (2 forward,
 * 4 backward instead of 1 and 2): fewer instructions per pixel, which raises throughput when
 * other kernels share the SMs, at the cost of a longer kernel when it runs alone. The forward
 * outputs are identical; the gradients differ only in the order of their float sums. */
#define GS_RENDER_CONCURRENT 2u

GS_API size_t gs_render_workspace_size(int N, int H, int W, long long pair_capacity);
GS_API int gs_render_forward(int N, int H, int W, const float* mu, const float* q, const float* s,
                             const float* opacity, const float* albedo, const float* k_j,
                             const float* R, const float* t, const float* cam_pos, float fx,
                             float fy, float cx, float cy, void* workspace,
                             size_t workspace_bytes, long long pair_capacity, float* img,
                             int* sorted_ids, int* tile_ranges, float* final_T, int* n_contrib,
                             float* radii, int* pair_count_host, void* m_ready_event,
                             unsigned flags, void* stream);
GS_API size_t gs_render_backward_workspace_size(int N);
GS_API int gs_render_backward(int N, int H, int W, const float* grad_img, const float* mu,
                              const float* q, const float* s, const float* albedo,
                              const float* k_j, const float* R, const float* t,
                              const float* cam_pos, float fx, float fy, float cx, float cy,
                              const void* fwd_workspace, long long pair_capacity,
                              const int* sorted_ids, const int* tile_ranges,
                              const float* final_T, const int* n_contrib, void* workspace,
                              size_t workspace_bytes, float* g_mu, float* g_q, float* g_s,
                              float* g_opacity, float* g_albedo, float* g_k_j, float* g_mean2d,
                              int accumulate, float* stat_norm_sum, float* stat_count,
                              float* stat_max, float stat_scale_x, float stat_scale_y,
                              void* accum_wait_event, void* accum_done_event, unsigned flags,
                              void* stream);

/*
 * gs_render_backward in two halves, for a batch of views whose gradients are summed (the
 * training step). gs_render_backward_blend runs one view's blend backward and leaves its
 * per-Gaussian sums in `workspace` (gs_render_backward_workspace_size(N) bytes, one per view,
 * kept until the second half has read it). gs_render_backward_gaussians then runs the SH and
 * projection backward of up to GS_MAX_VIEWS_PER_CALL views in one pass over the Gaussians:
 * each parameter, gradient and statistic element is read and written once per call instead of
 * once per view. The views are summed in array order after the buffers' own values
 * (accumulate = 1) or after zero (accumulate = 0), with the same rounding as one
 * gs_render_backward per view accumulating into the buffers in that order; so calls over
 * consecutive groups of views (the later ones with accumulate = 1) give the same bits as one
 * call over all of them. Statistics as gs_render_backward, per view with its own scales.
 */
#define GS_MAX_VIEWS_PER_CALL 16
typedef struct gs_view_sums {
  const void* workspace;  /* the view's gs_render_backward_blend workspace */
  size_t workspace_bytes; /* its size, at least gs_render_backward_workspace_size(N) */
  const float* R;         /* [3, 3] device, the view's camera as in gs_render_forward */
  const float* t;         /* [3] device */
  const float* cam_pos;   /* [3] device */
  float fx, fy, cx, cy;
  float stat_scale_x, stat_scale_y;
} gs_view_sums;
GS_API int gs_render_backward_blend(int N, int H, int W, const float* grad_img,
                                    const void* fwd_workspace, long long pair_capacity,
                                    const int* sorted_ids, const int* tile_ranges,
                                    const float* final_T, const int* n_contrib, void* workspace,
                                    size_t workspace_bytes, unsigned flags, void* stream);
GS_API int gs_render_backward_gaussians(int N, int n_views, const gs_view_sums* views,
                                        const float* mu, const float* q, const float* s,
                                        const float* albedo, const float* k_j, float* g_mu,
                                        float* g_q, float* g_s, float* g_opacity,
                                        float* g_albedo, float* g_k_j, int accumulate,
                                        float* stat_norm_sum, float* stat_count,
                                        float* stat_max, void* stream);

/*
 * Fused photometric loss of the training step (no counterpart in the reference's extension;
 * the reference trainer computes it with torchmetrics, gaussian_splatting/utils/loss.py:12-33):
 * loss = (1 - lambda) * mean|img - target| + lambda * (1 - SSIM) over [H, W, 3] images, with
 * the reference's SSIM semantics (torchmetrics structural_similarity_index_measure, data_range
 * 1.0, on the images clamped to [0, 1]): 11x11 Gaussian window (sigma 1.5), C1 = 0.01^2,
 * C2 = 0.03^2, variances clamped at 0, mean over the channels and the (H-10) x (W-10) interior
 * (torchmetrics reflect-pads by 5 and crops the same border, so the padding never reaches the
 * value). H and W must be at least 11. The L1 term uses the unclamped images.
 * The forward writes the scalar loss (and the mean SSIM when ssim_value is non-NULL) to device
 * memory and leaves per-pixel derivative maps in the workspace for the backward, which writes
 * grad_img = dL/dimg scaled by *grad_loss (a device scalar).
 */
GS_API size_t gs_l1_ssim_workspace_size(int H, int W);
GS_API int gs_l1_ssim_forward(int H, int W, const float* img, const float* target,
                              float lambda_dssim, void* workspace, size_t workspace_bytes,
                              float* loss, float* ssim_value, void* stream);
GS_API int gs_l1_ssim_backward(int H, int W, const float* img, const float* target,
                               float lambda_dssim, const void* workspace, size_t workspace_bytes,
                               const float* grad_loss, float* grad_img, void* stream);

/*
 * One Adam step (torch.optim.Adam semantics, amsgrad off, no weight decay; the reference's
 * trainer builds torch.optim.Adam(params, eps=1e-15), gaussian_splatting/utils/optim.py:31) over
 * n_groups <= 8 parameter tensors in one launch. Group k has sizes[k] elements at params[k]
 * and learning rate lrs[k] (host arrays); its gradients and moments are the slice starting at
 * sizes[0] + ... + sizes[k-1] of the flat device buffers grad, exp_avg and exp_avg_sq. `step` is
 * the 1-based step count used for bias correction; 1 - beta1, 1 - beta2 and the bias corrections
 * are formed in double on the host, as torch forms them from Python floats. clamp_min /
 * clamp_max (host arrays of n_groups floats, or NULL; -inf / +inf leave a side open): each
 * group's updated parameters become min(max(p, clamp_min[k]), clamp_max[k]) in the same pass,
 * the clamps the reference trainer applies right after optimizer.step() to the opacity logits
 * and log-scales (scripts/train.py:171-178). No counterpart in the reference's extension (its
 * trainer calls torch's optimizer).
 */
GS_API int gs_adam_step(int n_groups, float* const* params, const long long* sizes,
                        const float* lrs, const float* grad, float* exp_avg, float* exp_avg_sq,
                        double beta1, double beta2, double eps, long long step,
                        const float* clamp_min, const float* clamp_max, void* stream);

/*
 * The multi-GPU optimizer step of the view-parallel training step (no counterpart in the
 * reference, which trains on one GPU): reduce-scatter of the gradient bucket, Adam on this
 * rank's shard, all-gather of the parameters, SUM / MAX reductions of the densification
 * statistics, in one kernel per rank over NVLink. Every rank calls it with the same layout;
 * the buffers are symmetric (same size on every rank, mapped into every peer). With the *_mc
 * multicast pointers (NVSwitch) the reductions and broadcasts run as multimem operations in
 * the switch; otherwise the *_peers device arrays (one pointer per rank) are used for peer
 * loads and stores. Rank r owns elements [r * shard, (r + 1) * shard) of bucket and params:
 * gradients at [0, n_param) (parameter groups of group_sizes, learning rates lrs, gradient
 * scaled by grad_scale), SUM-reduced statistics at [stats_offset, stats_offset + n_stats), and
 * elements [r * max_shard, ...) of the MAX-reduced statistic (n_max non-negative floats).
 * exp_avg / exp_avg_sq hold this rank's shard of the Adam moments (shard floats each).
 * clamp_min / clamp_max: per-group clamps of the updated parameters, as in gs_adam_step.
 * signal_pads is a device array of each rank's signal pad (signal_slots zeroed uint32 words);
 * barrier waits are bounded and a timeout sets a device error bit (gs_device_error_bits).
 */
typedef struct gs_shard_buffers {
  int world, rank;
  long long shard, n_param, stats_offset, n_stats, max_shard, n_max;
  float* bucket;
  float* bucket_mc;
  void* const* bucket_peers;
  float* params;
  float* params_mc;
  void* const* params_peers;
  float* maxbuf;
  float* max_mc;
  void* const* max_peers;
  void* const* signal_pads;
  long long signal_slots;
  /* optional (may be NULL): 4 device words that receive, in globaltimer nanoseconds, the
     earliest CTA start, the latest end of the opening barrier, of the data loop and of the
     closing barrier (initialise to {~0, 0, 0, 0}) */
  unsigned long long* phase_ns;
  /* limit of each barrier wait in nanoseconds of GPU global time (0: 5 s); a wait that runs
     out sets bit 8 of gs_device_error_bits and the kernel returns */
  unsigned long long wait_ns;
} gs_shard_buffers;

GS_API int gs_sharded_adam_step(const gs_shard_buffers* buffers, float* exp_avg,
                                float* exp_avg_sq, int n_groups, const long long* group_sizes,
                                const float* lrs, double beta1, double beta2, double eps,
                                long long step, float grad_scale, const float* clamp_min,
                                const float* clamp_max, void* stream);

/*
 * Adaptive density control (the reference trainer's clone / split / prune / opacity reset,
 * gaussian_splatting/utils/adc.py:330-392, which the reference runs as torch ops with host
 * syncs) in two calls; no counterpart in the reference's extension.
 * gs_adc_plan classifies the N Gaussians from log-scales s[N,3], opacity logits alpha[N],
 * the densification statistics (grad_accum[N], denom[N], max_radii[N]) and the thresholds
 * (percent_dense_extent = percent_dense * extent and big_extent = 0.1 * extent, both rounded
 * to float as torch compares them; max_screen_size < 0: no screen-size rule; densify: the
 * reference's allow_densify and N < max_gaussians; prune: allow_densify). It writes five totals
 * to totals_host (pinned): kept originals, kept clones, split Gaussians, kept children per copy,
 * clones before pruning; and records done_event after the copy.
 * gs_adc_apply (same N and workspace, the first four totals on the host) writes the new set of
 * totals[0] + totals[1] + 2 * totals[3] Gaussians in the reference's order (kept originals,
 * kept clones, kept first children, kept second children; each in index order): params and
 * out_params are host arrays of the six device pointers mu[.,3], q[.,4], s[.,3], alpha[.,1],
 * A[.,3], k_j[.,15,3]; the optional Adam moments in the same layout are copied for originals
 * and zeroed for new Gaussians; z holds 2 * totals[2] unit normals [.,3] (rows [0, n) for the
 * first child of each split Gaussian in index order, [n, 2n) for the second); reset_opacity
 * caps alpha at logit(0.01) and zeroes its moments.
 */
GS_API size_t gs_adc_workspace_size(int N);
GS_API int gs_adc_plan(int N, const float* s, const float* alpha, const float* grad_accum,
                       const float* denom, const float* max_radii, float grad_threshold,
                       float percent_dense_extent, float big_extent, float min_opacity,
                       float max_screen_size, int densify, int prune, void* workspace,
                       size_t workspace_bytes, long long* totals_host, void* done_event,
                       void* stream);
GS_API int gs_adc_apply(int N, const void* workspace, size_t workspace_bytes,
                        const long long* totals, const float* const* params,
                        const float* const* exp_avg, const float* const* exp_avg_sq,
                        const float* z, int reset_opacity, float* const* out_params,
                        float* const* out_exp_avg, float* const* out_exp_avg_sq, void* stream);

/*
 * Densification statistics of one rendered view: the reference trainer's
 * accumulate_densification_stats (gaussian_splatting/utils/adc.py:58-80) in one launch. For each
 * Gaussian i with screen-space mean gradient (g[i*grad_stride], g[i*grad_stride+1]),
 * n = |(gx * scale_x, gy * scale_y)|; where n > 0, norm_sum[i] += n and count[i] += 1;
 * norm_max[i] = max(norm_max[i], n) when norm_max is non-NULL.
 */
GS_API int gs_densify_stats(int N, const float* mean2d_grad, int grad_stride, float scale_x,
                            float scale_y, float* norm_sum, float* count, float* norm_max,
                            void* stream);

/*
 * CUDA event helpers for m_ready_event (cudaEvent_t values passed as void*): create an event
 * with timing disabled, block the calling thread until it completes, destroy it.
 */
GS_API int gs_event_create(void** event);
GS_API int gs_event_synchronize(void* event);
GS_API int gs_event_destroy(void* event);

/*
 * Stage timing for profiling: while `events` (n cudaEvent_t handles, NULL entries allowed) is
 * installed, gs_render_forward / gs_render_backward record events[k] on their stream at stage
 * boundaries: 0 forward start, 1 after preprocess, 2 after the depth sort, 3 after pair
 * duplication, 4 after the tile sort, 5 after tile ranges, 6 after the blend, 7 backward start
 * (after the accumulator clear), 8 after the blend backward, 10 before and 9 after the
 * per-Gaussian backward (gs_render_backward, or gs_render_backward_gaussians for several views;
 * gs_render_backward_blend records 7 and 8). The setting is process-wide; events = NULL or
 * n = 0 removes it. Timed events come from gs_event_create_timed and are read with
 * gs_event_elapsed_ms.
 */
GS_API int gs_set_stage_events(void* const* events, int n);
GS_API int gs_event_create_timed(void** event);
GS_API int gs_event_elapsed_ms(void* start, void* end, float* ms);

/* Number of kernels this library has launched in this process (all devices, all threads). */
GS_API unsigned long long gs_kernel_launches(void);

/*
 * Device-side error bits recorded by the kernels of earlier calls on this device since
 * the last gs_clear_device_errors() (1 = a look-back wait gave up, 2 = pair capacity
 * exceeded, 4 = an index out of range, 8 = a cross-GPU barrier wait of gs_sharded_adam_step
 * gave up, 16 = a wait for a tile copy of the tensor memory accelerator gave up).
 * Synchronises the device.
 */
GS_API int gs_device_error_bits(unsigned* bits);
GS_API int gs_clear_device_errors(void);

#ifdef __cplusplus
}
#endif

#endif /* GS3D_B200_H */
