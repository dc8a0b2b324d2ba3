/*
 * gsx-b200: the C ABI of a B200-native (sm_100a) backend for the GSX Gaussian-splatting library.
 *
 * Plain C, plain pointers and sizes, no C++ or framework types.  All tensor arguments are DEVICE
 * pointers on the context's GPU, laid out exactly as GSX's tensors (row-major "CHW" contract of
 * gsx/include/gsx/gsx-core.h): Gaussian fields [N,3] / [N,4] / [N] / [N,k,3], images [3,H,W].
 * `stream` is a cudaStream_t (NULL = legacy default stream); every call is asynchronous on it
 * unless stated otherwise, and its outputs are ready on that stream when it returns, the same
 * contract as GSX's major stream (gsx/include/gsx/gsx-base.h:94-109).
 *
 * Every function returns 0 on success or a gsx_error_code value (gsx-base.h:68-84); the message
 * of the last failure on the calling thread is available from gsx_b200_last_error().  Nothing
 * ever falls back to the CPU: without a usable sm_100 device, calls fail.
 *
 * Each entry point names the reference interface it replaces (paths are inside the reference
 * project Adversarr/gsx).
 */
#ifndef GSX_B200_H
#define GSX_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define GSX_B200_API __attribute__((visibility("default")))
#else
#define GSX_B200_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum {
    GSX_B200_SUCCESS = 0,
    GSX_B200_OUT_OF_MEMORY = 1,
    GSX_B200_INVALID_ARGUMENT = 2,
    GSX_B200_OUT_OF_RANGE = 3,
    GSX_B200_INVALID_STATE = 4,
    GSX_B200_NOT_SUPPORTED = 5,
    GSX_B200_UNKNOWN = 255
};

enum { GSX_B200_FORWARD_INFERENCE = 0, GSX_B200_FORWARD_TRAIN = 1 };

/* element types (the values of gsx_data_type, gsx-core.h:8-14) */
enum { GSX_B200_DATA_F32 = 0, GSX_B200_DATA_U8 = 8, GSX_B200_DATA_I32 = 12 };

/* Pinhole camera: world->camera rotation (quaternion x, y, z, w) and translation, as
 * gsx_camera_pose (gsx-base.h:211-216) plus gsx_camera_intrinsics fx, fy, cx, cy, width, height. */
typedef struct gsx_b200_camera {
    int32_t width;
    int32_t height;
    float fx, fy, cx, cy;
    float rot_xyzw[4];
    float transl[3];
    float near_plane;
    float far_plane;
} gsx_b200_camera;

/* Gaussian parameters (the GS container fields of gsx-core.h:179-373).  sh1/sh2/sh3 may be NULL
 * when sh_degree is below 1/2/3. */
typedef struct gsx_b200_gaussians {
    int64_t count;
    const float *mean3d;   /* [N,3] */
    const float *rotation; /* [N,4] xyzw, need not be normalised */
    const float *logscale; /* [N,3] */
    const float *opacity;  /* [N] pre-sigmoid */
    const float *sh0;      /* [N,3] */
    const float *sh1;      /* [N,3,3] */
    const float *sh2;      /* [N,5,3] */
    const float *sh3;      /* [N,7,3] */
} gsx_b200_gaussians;

/* Parameter-gradient outputs, same shapes as gsx_b200_gaussians.  Written, not accumulated. */
typedef struct gsx_b200_gaussian_grads {
    float *mean3d;
    float *rotation;
    float *logscale;
    float *opacity;
    float *sh0;
    float *sh1;
    float *sh2;
    float *sh3;
} gsx_b200_gaussian_grads;

typedef struct gsx_b200_context gsx_b200_context;

/* Message of the last failing call on this thread ("" if none).  Static storage per thread. */
GSX_B200_API const char *gsx_b200_last_error(void);

/* Library version string. */
GSX_B200_API const char *gsx_b200_version(void);

/* Context = one render context (replaces gsx_cuda_render_context, gsx-cuda/render.c:35-80, and its
 * per-primitive/tile/instance/bucket scratch blobs, fastgs/buffer_utils.h:51-176).  It owns all
 * scratch on `device`, grown on demand, never shrunk.  Not thread-safe; one caller thread. */
GSX_B200_API int gsx_b200_context_create(int device, gsx_b200_context **out_ctx);
GSX_B200_API int gsx_b200_context_destroy(gsx_b200_context *ctx);

/*
 * Forward render into out_rgb (device [3,H,W] f32), background composed.
 * Replaces gsx_cuda_fastgs_forward_launch (gsx-cuda/render-kernels.cu:122-247) followed by
 * gsx_cuda_render_compose_background_to_chw_f32_kernel_launch (render-kernels.cu:72-96), i.e. the
 * body of gsx_cuda_renderer_render (gsx-cuda/render.c:1314-1423).
 * TRAIN retains the intermediates for one gsx_b200_render_backward on the same context; the
 * Gaussian buffers must stay unchanged until then.  One host synchronisation per call (to size
 * the instance buffers).
 */
GSX_B200_API int gsx_b200_render_forward(gsx_b200_context *ctx, const gsx_b200_gaussians *gaussians, int sh_degree,
                            const gsx_b200_camera *camera, const float background[3], int forward_type,
                            float *out_rgb, void *stream);

/*
 * Band render: rows [row_begin, row_end) of the full frame that `camera` describes, written as a
 * [3, row_end - row_begin, width] image.  Every projection, frustum clip, tile test and pixel position
 * uses full-frame coordinates, so the band is bit-identical to the same rows of
 * gsx_b200_render_forward; only the band's tiles are binned, sorted and blended.  row_begin must be a
 * multiple of 16 (a tile row) and row_begin < row_end <= height.  out_bf16 != 0
 * writes bf16 (round-to-nearest-even of the f32 result) instead of f32.  A TRAIN band is retained for
 * gsx_b200_render_backward like a full frame, whose grad_rgb is then the band's [3, rows, width].
 * The frame-split path of a large frame over several GPUs: rank r renders one band (no exchange).
 */
GSX_B200_API int gsx_b200_render_forward_rows(gsx_b200_context *ctx, const gsx_b200_gaussians *gaussians, int sh_degree,
                                 const gsx_b200_camera *camera, int row_begin, int row_end,
                                 const float background[3], int forward_type, void *out, int out_bf16,
                                 void *stream);

/*
 * Backward of the last TRAIN forward on ctx: grad_rgb (device [3,H,W]) -> parameter gradients.
 * Replaces gsx_cuda_fastgs_backward_launch (gsx-cuda/render-kernels.cu:249-343), i.e. the body of
 * gsx_cuda_renderer_backward (gsx-cuda/render.c:1425-1571).  Gradients are written for every
 * Gaussian (zero where culled); no prior zeroing needed.  Fails with GSX_B200_INVALID_STATE when
 * no TRAIN forward is retained (render.c:1434-1436).
 */
/*
 * Work estimate per tile row of the full frame, for splitting a large frame into bands of equal work
 * (no reference counterpart; the frame split of large-frame inference): host_row_costs[r] (n_rows =
 * ceil(height / 16) entries) receives, for every Gaussian the preprocess's conservative screen cull
 * keeps, the number of tile columns of its cull rectangle, added to each tile row the rectangle covers.
 * Integer sums: every rank computing it for the same inputs gets the same array, so every rank derives
 * the same bands without exchanging anything.  Waits for the stream (the array is host memory).
 */
GSX_B200_API int gsx_b200_render_row_costs(gsx_b200_context *ctx, const gsx_b200_gaussians *gaussians,
                                           const gsx_b200_camera *camera, uint32_t *host_row_costs, int32_t n_rows,
                                           void *stream);

GSX_B200_API int gsx_b200_render_backward(gsx_b200_context *ctx, const float *grad_rgb, const gsx_b200_gaussian_grads *grads,
                             void *stream);

/* Counts of the last forward (visible Gaussians, instances, buckets).  Synchronises the stream. */
GSX_B200_API int gsx_b200_render_stats(gsx_b200_context *ctx, uint64_t *n_visible, uint64_t *n_instances, uint64_t *n_buckets,
                          void *stream);

/* Device pointers to the last forward's intermediates, for parity checks:
 * keys (u64, sorted), values (u32, sorted), ranges (uint2 per tile), offsets (u32 [N+1], the
 * exclusive prefix of the per-Gaussian tile counts), tile_max (u32 per tile), pixel state
 * (float4 per pixel: composed rgb + n_contrib bits). */
typedef struct gsx_b200_render_view {
    const uint64_t *keys;
    const uint32_t *values;
    const uint32_t *ranges;
    const uint32_t *offsets;
    const uint32_t *tile_max;
    const float *pixel_state;
    uint64_t n_instances;
    int32_t n_tiles;
    int32_t grid_width;
} gsx_b200_render_view;
GSX_B200_API int gsx_b200_render_get_view(gsx_b200_context *ctx, gsx_b200_render_view *out_view);

/* Synchronise the stream and report device-side failures of previous calls on ctx (bounded
 * lookback waits that timed out, capacity overflows) as GSX_B200_UNKNOWN; clears them. */
GSX_B200_API int gsx_b200_context_check(gsx_b200_context *ctx, void *stream);

/*
 * Bind the density-control statistics of gsx_render_forward_request / gsx_render_backward_request
 * (gsx-render.h:123-124,143-144): device [N] f32 accumulators, each NULL to leave it unbound; they stay
 * bound until the next call.  TRAIN forwards add 1 to visible_counter[i] and raise
 * max_screen_radius[i] to the Gaussian's screen radius (ceil of 3 sigma of the larger eigenvalue of
 * its dilated 2-D covariance) for every Gaussian that touches a tile; backwards add the norm of the
 * screen-space mean gradient scaled by (W/2, H/2) to grad_acc[i], and the norm of the per-pixel
 * absolute gradient, scaled the same way, to absgrad_acc[i].  The reference's CUDA backend fills
 * none of them; the semantics are those of its Metal backend (gsx-metal/kernels/render.metal:425-439,
 * render_backward.metal:700-714).  N must cover the Gaussian count of every later call.
 */
GSX_B200_API int gsx_b200_render_bind_aux(gsx_b200_context *ctx, float *visible_counter, float *max_screen_radius,
                             float *grad_acc, float *absgrad_acc);

/*
 * How a TRAIN forward's state is kept for its backward (gsx_render_forward_request.borrow_train_state,
 * gsx-render.h; gsx-cuda/render.c:481-756).
 * RETAINED (default): the context keeps the forward's intermediates and the Gaussian pointers; the
 *   caller must not change the Gaussians between the TRAIN forward and its backward (or must pass
 *   private copies, as GSX's cloned train state does).  No extra work per step.
 * BORROWED: the reference's borrowed state.  The forward also records a 64-bit fingerprint of the
 *   Gaussian fields; the backward fingerprints them again (one read of the fields and one wait for the
 *   stream) and, if they changed, re-runs the TRAIN forward on the current fields before the backward,
 *   so the gradients are those of the current inputs, as the reference's refresh gives them.  The
 *   re-run writes a private image (not the caller's out_rgb) and leaves the density-control statistics
 *   alone.  Switching the mode drops a retained forward.
 */
enum { GSX_B200_TRAIN_STATE_RETAINED = 0, GSX_B200_TRAIN_STATE_BORROWED = 1 };
GSX_B200_API int gsx_b200_context_set_train_state(gsx_b200_context *ctx, int mode);
/* Number of borrowed-state refreshes (re-run TRAIN forwards) ctx has done. */
GSX_B200_API int gsx_b200_context_train_refreshes(gsx_b200_context *ctx, uint64_t *out_count);

/* Number of kernels ctx has launched since it was created (a host-side count, for benchmarks). */
GSX_B200_API int gsx_b200_context_launch_count(gsx_b200_context *ctx, uint64_t *out_count);

/* Per-stage device timing of the render pipeline with CUDA events on the launching stream (the
 * reference's session timing syncs the stream at every stage instead, gsx-runtime.c:619-680).
 * enable != 0 starts recording (up to 256 launches per stage), enable == 0 stops.  Stages:
 * 0 preprocess+scan, 1 key emission, 2 radix sort, 3 tile ranges, 4 blend forward, 5 blend backward,
 * 6 preprocess backward. */
#define GSX_B200_STAGE_COUNT 7
GSX_B200_API int gsx_b200_context_set_profiling(gsx_b200_context *ctx, int enable);
/* Synchronises, writes per-stage total milliseconds and launch counts since the last read
 * (arrays of GSX_B200_STAGE_COUNT), and resets them. */
GSX_B200_API int gsx_b200_context_read_profile(gsx_b200_context *ctx, float *total_ms, int32_t *launches);

/*
 * Fused image loss on [planes, H, W] f32 CHW planes (planes = outer * channels), one launch.
 * mode bit 0: accumulate the loss map; bit 1: accumulate the gradient; bit 2: include L1;
 * bit 3: overwrite instead of accumulate (loss_map and grad are written as if they held zeros).
 * With bit 2: loss_map = (loss_map + l1_scale*|p-t|) then SSIM as below; grad += sign(p-t)*l1_grad_scale.
 * SSIM: loss_map += ssim_scale*(1-ssim) (SET to 0 within 5 pixels of the border);
 *       grad += SSIM gradient scaled by ssim_grad_scale.
 * loss_sum (device f32, may be NULL) receives the sum of the loss-map values this call wrote.
 * Replaces the L1 and SSIM launches of gsx-cuda/loss.c:414-685
 * (gsx_cuda_loss_ssim_chw_f32_forward/backward_kernel_launch, loss-ssim-kernels.cu:360-480, and the
 * L1 kernels of loss-pointwise-kernels.cu:43-89) with one kernel and no partial-derivative scratch.
 */
GSX_B200_API int gsx_b200_loss_l1_ssim(int mode, const float *prediction, const float *target, float *loss_map, float *grad,
                          float *loss_sum, int64_t planes, int32_t height, int32_t width, float l1_scale,
                          float ssim_scale, float l1_grad_scale, float ssim_grad_scale, void *stream);

/* Pointwise losses on n elements: op 0 L1 forward (out += scale*|p-t|), 1 L1 backward
 * (out += sign(p-t)*scale), 2 MSE forward (out += scale*(p-t)^2), 3 MSE backward (out += 2(p-t)*scale).
 * Replaces gsx-cuda/loss-pointwise-kernels.cu:7-89. */
GSX_B200_API int gsx_b200_loss_pointwise(int op, const float *prediction, const float *target, float *out, uint64_t n, float scale,
                            void *stream);

/* One Adam parameter group (gsx_optim_param_group_desc, gsx-optim.h:60-71, plus its moment state).
 * inv_bias_correction1/2 = 1 / (1 - beta^t) computed by the caller in double (gsx-cuda/optim.c:776-778). */
typedef struct gsx_b200_adam_group {
    float *parameter;
    const float *gradient;
    float *first_moment;
    float *second_moment;
    uint64_t count;
    float learning_rate, beta1, beta2, epsilon, weight_decay, max_grad;
    double inv_bias_correction1, inv_bias_correction2;
} gsx_b200_adam_group;

/* All groups (up to 16) in ONE launch.  Replaces the per-group loop of gsx_cuda_optim_step_selected
 * (gsx-cuda/optim.c:746-803) over gsx_cuda_adam_step_f32_kernel_launch (gsx-cuda-kernels.cu:595-640). */
GSX_B200_API int gsx_b200_adam_step(const gsx_b200_adam_group *groups, int32_t group_count, void *stream);

/*
 * Stable sort of `count` (u64 key, u32 value) pairs by key bits [begin_bit, end_bit), onesweep LSD
 * radix sort.  keys/values are sorted in place (the alternate buffers are context scratch).
 * Replaces the two cub::DeviceRadixSort::SortPairs calls of fastgs/forward.cu:155-161,214-220.
 */
GSX_B200_API int gsx_b200_sort_pairs(gsx_b200_context *ctx, uint64_t *keys, uint32_t *values, uint64_t count, int32_t begin_bit,
                        int32_t end_bit, void *stream);

/*
 * The same stable sort, for callers that cannot allocate device memory.  It has no counterpart in
 * the reference: it exists because some hosts own every device allocation themselves (GSX hands all
 * memory out of caller-owned arenas, and a plugin host that budgets GPU memory forbids hidden
 * cudaMalloc calls).  keys/values are sorted in place; nothing is allocated: the scratch (alternate
 * buffers, digit histograms, lookback table, one status word) is one file-scope device array of
 * about 14 MiB that every GPU which loads this library keeps until the process exits.  count above
 * GSX_B200_NOALLOC_SORT_MAX_PAIRS is rejected with GSX_B200_OUT_OF_RANGE.  The first call on a
 * device looks up the array's device address (once per device, with that device current).  Each
 * call clears the status word, sorts, and reads the status word back, so it returns only once the
 * sort has finished on `stream`; a timed-out lookback wait returns GSX_B200_UNKNOWN.  All calls
 * share the one array: calls that overlap on the GPU (other streams or other host threads on the
 * same device) race, so serialise them.
 */
#define GSX_B200_NOALLOC_SORT_MAX_PAIRS (1u << 20)
GSX_B200_API int gsx_b200_sort_pairs_noalloc(uint64_t *keys, uint32_t *values, uint64_t count, int32_t begin_bit,
                                             int32_t end_bit, void *stream);

/*
 * Buffer helpers behind the GSX backend-buffer interface (gsx/src/gsx-impl.h:302-458), used by the
 * GSX provider in gsx_b200/provider/.
 * gsx_b200_fill_pattern: repeats a 1/2/4/8-byte pattern over size_bytes of device memory at dst
 * (size a multiple of the pattern, dst aligned to it); replaces the backend's fill_tensor
 * (gsx-impl.h:349-353, gsx-cuda/buffer.c).
 * gsx_b200_count_nonfinite_f32: ADDS the number of NaN/Inf values among n floats at x to the
 * device word device_count (clear it first); backs check_finite_tensor (gsx-impl.h:377-381).
 */
GSX_B200_API int gsx_b200_fill_pattern(void *dst, uint64_t size_bytes, const void *pattern, uint32_t pattern_bytes, void *stream);
GSX_B200_API int gsx_b200_count_nonfinite_f32(const float *x, uint64_t n, uint32_t *device_count, void *stream);

/*
 * Dataloader layout conversion: an interleaved HWC image of pixel_count pixels (channels 3: RGB;
 * channels 1: an alpha or inverse-depth plane), u8 or f32 (src_type GSX_B200_DATA_U8 / _F32), to a
 * planar CHW f32 tensor [channels, H, W] at dst, values unchanged (no 1/255 scaling).  Replaces the
 * CUDA async dataloader's layout kernels (gsx-cuda/async_dl.cu:45-160, called after the staging
 * upload at :205-262); results equal the CPU packer gsx_dataloader_pack_hwc_to_chw /
 * pack_hw_to_chw (gsx-data-impl.h:212-260) with f32 output, for every pixel count.  Device pointers;
 * f32 buffers 4-byte aligned; 16-byte aligned buffers take the vector path.
 */
GSX_B200_API int gsx_b200_hwc_to_chw_f32(const void *src, int src_type, int channels, uint64_t pixel_count, float *dst,
                                         void *stream);

/*
 * Structural operations of density control (device pointers, on `stream`).
 * gsx_b200_gather_rows: dst row r = src row index[r] (rows of row_bytes bytes, out_rows rows, src has
 * src_rows rows); an index outside [0, src_rows) sets *device_out_of_range to 1 (when non-NULL) and
 * leaves that row of dst untouched.  Replaces gsx_cuda_gather_rows_kernel_launch
 * (gsx-cuda/gsx-cuda-kernels.cu:642-675), behind gather_tensor and the optimizer's permute/gather.
 * gsx_b200_clamp_inplace: x[i] = lo if x[i] < lo, hi if x[i] > hi (NaN kept) for f32, i32 or u8
 * (gsx-cuda/buffer.c:1985-2060).  gsx_b200_iota_i32: dst[i] = i.
 */
GSX_B200_API int gsx_b200_gather_rows(const void *src, uint64_t src_rows, uint64_t row_bytes, const int32_t *index,
                                      uint64_t out_rows, void *dst, uint32_t *device_out_of_range, void *stream);
GSX_B200_API int gsx_b200_clamp_inplace(void *x, int data_type, uint64_t n, const void *min_value, const void *max_value,
                                        void *stream);
GSX_B200_API int gsx_b200_iota_i32(int32_t *dst, uint64_t n, void *stream);

/*
 * The refine pass of GSX's default density control (gsx-cuda/adc.cu:707-946), as device stages the
 * host sequences around gsx_gs_gather / gsx_optim_gather.  scratch holds
 * gsx_b200_adc_scratch_words(n) words.
 * gsx_b200_adc_select_growth: modes[i] (0 none, 1 duplicate, 2 split; adc.cu:428-476) for n
 * Gaussians and the ordered list of candidates (mode != 0) in candidates[]; device_counts[0] = the
 * candidate count, device_counts[1] = the splits among the first `budget` candidates.
 * gsx_b200_adc_apply_split: the split mutation (adc.cu:541-705) of grown rows count_before + g for
 * the first grow_count candidates whose mode is split (modes indexed by source row).
 * gsx_b200_adc_select_keep: the ordered list of rows the prune pass keeps (adc.cu:499-539) in keep[],
 * its length in *device_count; flags[n] is scratch.
 */
/*
 * Data-parallel training over NVLink: the gradient all-reduce and Adam fused into one kernel per rank
 * (no counterpart in the reference, which runs one view per process and no exchange; it replaces the
 * ncclAllReduce + full Adam that the data-parallel extension of gsx-runtime.c:1413-1536 would issue).
 * Rank `rank` of `world` owns the flat elements [shard_begin, shard_end): it averages them over
 * grads[0..world-1] (sum in rank order, times 1/world), applies Adam with the shard-local moments
 * (first/second_moment[k] belongs to element shard_begin + k) and stores the updated values into
 * params[0..world-1].  params[r] / grads[r] are rank r's flat buffers mapped into this process
 * (gsx_b200_ipc_open; this rank's own buffers for r == rank), 16-byte aligned.  segments cut the shard
 * into runs of one parameter role (Adam hyper-parameters per run), bounds multiples of 4 elements.
 * The kernel never waits: all ranks' gradients must be complete before it runs, and no rank may read
 * its parameters until every rank's call has finished (the host orders both with collectives).
 */
#define GSX_B200_DP_MAX_RANKS 8
#define GSX_B200_DP_MAX_SEGMENTS 8
#define GSX_B200_IPC_HANDLE_BYTES 64
typedef struct gsx_b200_dp_segment {
    uint64_t begin, end;
    float learning_rate, beta1, beta2, epsilon, weight_decay, max_grad;
    double inv_bias_correction1, inv_bias_correction2;
} gsx_b200_dp_segment;
GSX_B200_API int gsx_b200_dp_reduce_adam_gather(int world, int rank, float *const *params, const float *const *grads,
                                                float *first_moment, float *second_moment, uint64_t shard_begin,
                                                uint64_t shard_end, const gsx_b200_dp_segment *segments, int n_segments,
                                                void *stream);
/*
 * The same step over NVLink SHARP (NVSwitch multicast, no counterpart in the reference).  mc_grads and
 * mc_params are multicast addresses bound to every rank's flat gradient / parameter buffer; params is
 * this rank's own parameter buffer.  The shard's gradients are summed inside the switch
 * (multimem.ld_reduce), averaged, run through Adam with the shard-local moments, and the result is
 * written to every rank's parameter buffer with one multicast store: per rank and direction only
 * 1/world of the bytes cross NVLink.  The switch's summation order may differ from rank order (the
 * average agrees with the peer-load form to rounding); replicas stay identical.  Same ordering contract
 * as gsx_b200_dp_reduce_adam_gather: no waits inside, collectives around it on the host.
 */
GSX_B200_API int gsx_b200_dp_nvls_reduce_adam_broadcast(int world, float *mc_params, const float *mc_grads,
                                                        const float *params, float *first_moment, float *second_moment,
                                                        uint64_t shard_begin, uint64_t shard_end,
                                                        const gsx_b200_dp_segment *segments, int n_segments, void *stream);
/* Device buffers that other processes can map: cudaMalloc / cudaFree, the 64-byte CUDA IPC handle of a
 * buffer from gsx_b200_device_alloc, and mapping / unmapping another process's buffer by its handle. */
GSX_B200_API int gsx_b200_device_alloc(uint64_t bytes, void **out);
GSX_B200_API int gsx_b200_device_free(void *ptr);
GSX_B200_API int gsx_b200_ipc_handle(void *base, void *out_handle);
GSX_B200_API int gsx_b200_ipc_open(const void *handle, void **out);
GSX_B200_API int gsx_b200_ipc_close(void *ptr);

GSX_B200_API uint64_t gsx_b200_adc_scratch_words(uint64_t n);
GSX_B200_API int gsx_b200_adc_select_growth(uint64_t n, const float *grad_acc, const float *visible_counter,
                                            const float *logscale, float grad_threshold, float scale_threshold,
                                            float scene_scale, uint64_t budget, uint8_t *modes, int32_t *candidates,
                                            uint32_t *scratch, uint32_t *device_counts, void *stream);
GSX_B200_API int gsx_b200_adc_apply_split(uint64_t grow_count, const int32_t *sources, const uint8_t *modes,
                                          uint64_t count_before, uint64_t seed, uint64_t global_step, float *mean3d,
                                          float *logscale, float *opacity, const float *rotation, void *stream);
GSX_B200_API int gsx_b200_adc_select_keep(uint64_t n, const float *opacity, const float *logscale, const float *rotation,
                                          const float *max_screen_radius, uint64_t count_before_growth, int prune_large,
                                          float opacity_threshold, float max_world_scale, float max_screen_scale,
                                          float scene_scale, uint8_t *flags, int32_t *keep, uint32_t *scratch,
                                          uint32_t *device_count, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* GSX_B200_H */
