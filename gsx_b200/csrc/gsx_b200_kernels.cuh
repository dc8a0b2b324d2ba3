/*
 * Shared device-side definitions for the gsx-b200 sm_100a kernels.
 *
 * HBM layout of the per-frame render state (all owned by a gsx_b200_context):
 *   per primitive (capacity N):
 *     rec      PrimRec[N]   48 B: {mean2d.xy, conic.xy} {conic.z, opacity, rgb.rg} {rgb.b, depth, bx, by}
 *     counts   u32[N]       exact tile-overlap count (0 = culled); block_sums u32[N/256+1]
 *     tile_masks u32[N]     which tiles of the bounding rectangle (row-major, rectangles <= 32 tiles) overlap
 *     offsets  u32[N+1]     exclusive prefix of the counts (written by the emission kernel)
 *     grad_acc float4[3N]   per-primitive 2-D gradient accumulators of the blend backward
 *   per instance (capacity I): keys u64[2I], values u32[2I] (double-buffered radix sort)
 *   per tile (T):   ranges uint2[T], bucket_offsets u32[T] (inclusive), tile_max u32[T]
 *   per pixel (P):  pix float4[P] = {composed rgb, n_contrib bits}
 *   per bucket (B <= I/32 + T): bucket_tile u32[B], snap float4[256 B] (colour and transmittance
 *                   before each 32-instance bucket, per pixel of the tile)
 */
#ifndef GSX_B200_KERNELS_CUH
#define GSX_B200_KERNELS_CUH

#include <cuda_runtime.h>
#include <stdint.h>

#include "gsx_detmath.h"

#include <utility>

/* Programmatic dependent launch (sm_90+): a kernel launched with gsx_launch_pdl may start while the
 * kernel before it in the stream is finishing (its CTAs become resident as the previous kernel's last
 * CTAs leave, and its launch overhead is hidden); it must call gsx_pdl_wait() before it touches anything
 * the previous kernel reads or writes.  A kernel calls gsx_pdl_trigger() to let the next one launch
 * early.  Both are no-ops for kernels launched without the attribute. */
__device__ __forceinline__ void gsx_pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void gsx_pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
cudaError_t gsx_launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                           Args &&...args)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

#define GSX_TILE 16
#define GSX_TILE_PIXELS 256
#define GSX_SEQ_TILES 8
#define GSX_SPIN_LIMIT (1u << 22)
#define GSX_SEG_MAX 16384 /* largest tile (instances) sorted in shared memory by k_tilesort.cu */

/* device-side error flags (bitwise-or into ctx->dev_flags[0]) */
#define GSX_FLAG_LOOKBACK_TIMEOUT 1u
#define GSX_FLAG_INSTANCE_OVERFLOW 2u
#define GSX_FLAG_BUCKET_OVERFLOW 4u

struct __align__(16) PrimRec {
    float4 a; /* mean2d.x, mean2d.y, conic.x, conic.y */
    float4 b; /* conic.z, opacity, rgb.r, rgb.g  (rgb unclamped) */
    float4 c; /* rgb.b, depth, bounds x (x0 | x1 << 16), bounds y (y0 | y1 << 16) as bits */
};

struct CameraParams {
    float w2c[12];
    float cam_pos[3];
    float fx, fy, cx, cy;
    float width_f, height_f;
    float near_plane, far_plane;
    int width, height;
    int grid_w, grid_h;
    /* frustum clamp of the EWA Jacobian in normalised image coordinates (kernels_forward.cuh:324-327),
     * divided once on the host (IEEE, identical bits to a device division) */
    float clip_l, clip_r, clip_t, clip_b;
    /* band rendering: the image is rows [16 trow0, 16 trow0 + height) of a full frame of height
     * height_f; every projection, tile test and pixel position uses full-frame coordinates, only
     * the tile rows kept (grid_h from trow0) and the output rows are the band's.  0 = full frame. */
    int trow0;
    /* 1 + the largest squared clamped normalised coordinate (x: max(clip_l^2, clip_r^2), y likewise):
     * bounds the squared row norm of the EWA Jacobian over (fx or fy / depth)^2, for the preprocess's
     * conservative screen cull */
    float cull_jx, cull_jy;
};

/* Decoupled-lookback status word: 2-bit flag in the top bits, 30-bit count below. */
#define GSX_LB_EMPTY 0u
#define GSX_LB_AGG 1u
#define GSX_LB_INC 2u
#define GSX_LB_SHIFT 30
#define GSX_LB_MASK ((1u << GSX_LB_SHIFT) - 1u)

__device__ __forceinline__ uint32_t gsx_ld_acquire(const uint32_t *p)
{
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void gsx_st_release(uint32_t *p, uint32_t v)
{
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

/* Relaxed (fence-free) device-scope accesses for decoupled-lookback status words whose value is
 * self-contained (no other data is published through them). */
__device__ __forceinline__ uint32_t gsx_ld_relaxed(const uint32_t *p)
{
    uint32_t v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void gsx_st_relaxed(uint32_t *p, uint32_t v)
{
    asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint64_t gsx_ld_acquire64(const unsigned long long *p)
{
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void gsx_st_release64(unsigned long long *p, unsigned long long v)
{
    asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

/* fastgs/kernels_forward.cuh:71-106 (will_primitive_contribute), identical arithmetic to the
 * oracle's orc_tile_contributes.  `mx, my` is mean2d - 0.5. */
__device__ __forceinline__ bool gsx_tile_contributes(float mx, float my, float cx, float cy, float cz, unsigned tx,
                                                     unsigned ty, float power_threshold)
{
    const float rminx = (float)(tx * GSX_TILE), rminy = (float)(ty * GSX_TILE);
    const float rmaxx = (float)((tx + 1) * GSX_TILE - 1), rmaxy = (float)((ty + 1) * GSX_TILE - 1);
    const float x_min_diff = rminx - mx;
    const float x_left = x_min_diff > 0.0f ? 1.0f : 0.0f;
    const float not_in_x = x_left + (mx > rmaxx ? 1.0f : 0.0f);
    const float y_min_diff = rminy - my;
    const float y_above = y_min_diff > 0.0f ? 1.0f : 0.0f;
    const float not_in_y = y_above + (my > rmaxy ? 1.0f : 0.0f);
    if(not_in_y + not_in_x == 0.0f) return true;
    const float ccx = x_left != 0.0f ? rminx : rmaxx;
    const float ccy = y_above != 0.0f ? rminy : rmaxy;
    const float diffx = mx - ccx, diffy = my - ccy;
    const float dx = copysignf((float)(GSX_TILE - 1), x_min_diff);
    const float dy = copysignf((float)(GSX_TILE - 1), y_min_diff);
    const float tx_ = not_in_y * gsx_saturatef((dx * cx * diffx + dx * cy * diffy) / (dx * cx * dx));
    const float ty_ = not_in_x * gsx_saturatef((dy * cy * diffx + dy * cz * diffy) / (dy * cz * dy));
    const float px = ccx + tx_ * dx, py = ccy + ty_ * dy;
    const float ddx = mx - px, ddy = my - py;
    const float power = 0.5f * (cx * ddx * ddx + cz * ddy * ddy) + cy * ddx * ddy;
    return power <= power_threshold;
}

/* ---- kernel launchers (each .cu file owns its kernels; these are host-side entry points) ---- */
struct RenderScratch;

cudaError_t gsx_launch_preprocess(const float *mean3d, const float *rotation, const float *logscale,
                                  const float *opacity, const float *sh0, const float *sh1, const float *sh2,
                                  const float *sh3, int sh_degree, int64_t n, const CameraParams &cam, PrimRec *rec,
                                  uint32_t *counts, uint32_t *tile_masks, uint32_t *block_sums, float *visible_counter,
                                  float *max_screen_radius, cudaStream_t stream);
/* per tile row of the (full-frame) camera, an integer estimate of the instances it holds */
cudaError_t gsx_launch_band_cost(const float *mean3d, const float *logscale, int64_t n, const CameraParams &cam,
                                 uint32_t *row_cost, cudaStream_t stream);
cudaError_t gsx_launch_emit(int64_t n, const PrimRec *rec, const uint32_t *counts, const uint32_t *tile_masks,
                            const uint32_t *block_offsets,
                            uint32_t *offsets, int grid_w, int trow0, int n_tiles, unsigned long long *keys, uint32_t *vals,
                            uint64_t capacity,
                            uint32_t *flags, uint32_t *hist, int n_digits, uint32_t *tile_count, cudaStream_t stream);
cudaError_t gsx_launch_sort_passes(unsigned long long *keys_a, uint32_t *vals_a, unsigned long long *keys_b,
                                   uint32_t *vals_b, uint64_t count, const int *positions, const int *shifts,
                                   const int *widths, int npasses, const uint32_t *hist, void *scratch,
                                   size_t scratch_bytes, uint32_t *flags, int *out_result_in_b, cudaStream_t stream);
size_t gsx_sort_scratch_bytes(uint64_t capacity);
cudaError_t gsx_launch_sort_pairs(unsigned long long *keys_a, uint32_t *vals_a, unsigned long long *keys_b,
                                  uint32_t *vals_b, uint64_t count, int begin_bit, int end_bit, void *scratch,
                                  size_t scratch_bytes, uint32_t *flags, int *out_result_in_b, cudaStream_t stream);
#define GSX_SORT_CLASSES 5 /* per-tile sort size classes of k_tilesort.cu */
#define GSX_TILE_SUBCOUNTERS 32 /* instance counters per tile (emission, binning); a multiple of 4 */
/* sub-counter s of tile t, sub-counter-major: one tile's counters sit n_tiles words apart (different
 * cache lines and L2 slices, so the atomics of a crowded tile spread), and a warp's 32 tiles read one
 * counter index with one coalesced access */
#define GSX_SUBCOUNTER(t, s, n_tiles) ((size_t)(s) * (size_t)(n_tiles) + (size_t)(t))
size_t gsx_tile_scan_aux_words(int n_tiles);
cudaError_t gsx_launch_tile_scan(uint32_t *tile_count, int n_tiles, uint2 *ranges, uint32_t *bucket_offsets,
                                 uint32_t *class_tiles, uint32_t *block_aux, uint32_t *words_out, cudaStream_t stream);
/* side: GSX_SORT_CLASSES - 1 streams; ev: GSX_SORT_CLASSES events (fork and join) */
cudaError_t gsx_launch_tile_bin(const unsigned long long *keys, const uint32_t *vals, const uint32_t *d_total,
                                uint64_t max_n, int n_tiles, uint32_t *tile_end, unsigned long long *sort_keys, cudaStream_t stream);
cudaError_t gsx_launch_tile_sort(uint64_t n, int n_tiles, const uint2 *ranges, const uint32_t *class_tiles,
                                 const uint32_t *class_counts, const unsigned long long *sort_keys,
                                 unsigned long long *keys_out, uint32_t *vals_out, cudaStream_t stream,
                                 cudaStream_t const *side, cudaEvent_t const *ev);
/* out_rgb: [3, height, width] f32, or bf16 (round to nearest even) when out_bf16; row0 = first pixel
 * row of the band in the full frame (a multiple of 16, 0 for a full frame) */
/* tile_lists / class_sizes (may be NULL): the tile scan's class lists (classes 0..4 end to end, then
 * the empty tiles) and the device class sizes; CTAs then take tiles from the largest class down.
 * TRAIN: tile_order [n_tiles * 256] receives each tile's pixel ranks by decreasing last-contributor
 * bucket, bucket_active [buckets] the number of pixels the backward walks in each bucket. */
cudaError_t gsx_launch_blend_forward(int width, int height, int row0, int grid_w, int n_tiles, const uint2 *ranges,
                                     const uint32_t *bucket_offsets, const uint32_t *vals, const PrimRec *rec,
                                     const float bg[3], void *out_rgb, bool out_bf16, float4 *pix, uint32_t *tile_max,
                                     float4 *snap, uint32_t *bucket_tile, bool train, const uint32_t *tile_lists,
                                     const uint32_t *class_sizes, uint8_t *tile_order, uint16_t *bucket_active,
                                     cudaStream_t stream);
/* Blend backward of a TRAIN forward: orders the buckets by the number of pixels they walk
 * (bucket_active, tile_order from the forward; bucket_order [buckets] and sort_state
 * [gsx_bucket_sort_state_words()] are scratch), then the reverse blend into grad_acc */
size_t gsx_bucket_sort_state_words();
cudaError_t gsx_launch_blend_backward(int width, int height, int row0, int grid_w, const uint2 *ranges,
                                      const uint32_t *bucket_offsets, const uint32_t *bucket_tile,
                                      uint64_t bucket_capacity, int n_tiles, const uint16_t *bucket_active,
                                      const uint8_t *tile_order, uint32_t *bucket_order, uint32_t *sort_state,
                                      const uint32_t *vals, const PrimRec *rec, const float4 *pix, const float4 *snap,
                                      const float *grad_rgb, float4 *grad_acc, bool abs_grad, cudaStream_t stream);
cudaError_t gsx_launch_preprocess_backward(const float *mean3d, const float *rotation, const float *logscale,
                                           const float *sh1, const float *sh2, const float *sh3, int sh_degree,
                                           int64_t n, const CameraParams &cam, const uint32_t *counts,
                                           float4 *grad_acc, float *g_mean3d, float *g_rotation, float *g_logscale,
                                           float *g_opacity, float *g_sh0, float *g_sh1, float *g_sh2, float *g_sh3,
                                           float *grad_norm_acc, float *absgrad_norm_acc,
                                           cudaStream_t stream);

cudaError_t gsx_launch_fingerprint(const float *const *fields, const uint64_t *counts, int n_fields, unsigned long long *out,
                                   cudaStream_t stream);

#define GSX_ADAM_MAX_GROUPS 16
struct AdamGroupDev {
    float *param;
    const float *grad;
    float *m1;
    float *m2;
    uint64_t n;
    uint64_t first_block;
    float lr, beta1, beta2, eps, weight_decay, max_grad;
    double inv_c1, inv_c2;
};
struct AdamTable {
    AdamGroupDev g[GSX_ADAM_MAX_GROUPS];
    int count;
};
cudaError_t gsx_launch_adam(AdamTable &table, cudaStream_t stream);

/* One Adam element update, gsx-cuda/gsx-cuda-kernels.cu:279-321 (max_grad clamp, decoupled weight
 * decay, bias corrections in double).  Written with round-to-nearest intrinsics so that no
 * multiply-add contraction happens whatever the translation unit's -fmad setting: any kernel that
 * calls it gives the standalone Adam kernel's bits (and the oracle's). */
__device__ __forceinline__ float gsx_adam_one(float p, float g, float &m1, float &m2, const AdamGroupDev &G)
{
    if(G.max_grad > 0.0f) {
        if(g > G.max_grad) g = G.max_grad;
        else if(g < -G.max_grad) g = -G.max_grad;
    }
    const float a = __fadd_rn(__fmul_rn(G.beta1, m1), __fmul_rn(__fsub_rn(1.0f, G.beta1), g));
    const float b = __fadd_rn(__fmul_rn(G.beta2, m2), __fmul_rn(__fmul_rn(__fsub_rn(1.0f, G.beta2), g), g));
    const float ah = (float)((double)a * G.inv_c1);
    const float bh = (float)((double)b * G.inv_c2);
    m1 = a;
    m2 = b;
    if(G.weight_decay > 0.0f) p = __fsub_rn(p, __fmul_rn(__fmul_rn(G.lr, G.weight_decay), p));
    return __fsub_rn(p, __fmul_rn(G.lr, ah / __fadd_rn(sqrtf(bh), G.eps)));
}

cudaError_t gsx_launch_l1_ssim(int mode, const float *pred, const float *target, float *loss_map, float *grad,
                               float *loss_sum, int planes, int height, int width, float l1_scale, float ssim_scale,
                               float l1_grad_scale, float ssim_grad_scale, cudaStream_t stream);
cudaError_t gsx_launch_pointwise_loss(int op, const float *pred, const float *target, float *out, size_t n, float scale,
                                      cudaStream_t stream);

#endif /* GSX_B200_KERNELS_CUH */
