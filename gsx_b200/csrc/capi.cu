/*
 * C ABI of gsx-b200 (include/gsx_b200.h): context and scratch management, and the orchestration
 * of the render forward/backward pipeline on one stream.
 *
 * Forward: preprocess (+ one-CTA scan of block totals) -> emit keys (+ in-block scan into offsets)
 * -> tile scan -> binning (queued behind the one read-back of the instance total, largest tile and
 * size-class counts) -> per-tile depth sort (grids from the read-back) -> blend+compose.
 * Backward: blend backward -> preprocess backward.
 * Scratch grows on demand with cudaMalloc (outside any stream capture) and is never shrunk.
 */
#include "../../include/gsx_b200.h"
#include "gsx_b200_kernels.cuh"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>


namespace {

constexpr int kProfileSlots = 256;
thread_local std::string g_last_error;

int fail(int code, const std::string &msg)
{
    g_last_error = msg;
    return code;
}

int cuda_fail(cudaError_t e, const char *what)
{
    return fail(e == cudaErrorMemoryAllocation ? GSX_B200_OUT_OF_MEMORY : GSX_B200_UNKNOWN,
                std::string(what) + ": " + cudaGetErrorString(e));
}

#define GSX_CUDA_TRY(expr, what)                      \
    do {                                              \
        cudaError_t e__ = (expr);                     \
        if(e__ != cudaSuccess) return cuda_fail(e__, what); \
    } while(0)

struct DevBuf {
    void *ptr = nullptr;
    size_t bytes = 0;
};

int ensure(DevBuf &b, size_t bytes, bool zero = false)
{
    if(b.bytes >= bytes && b.ptr != nullptr) return 0;
    if(b.ptr) cudaFree(b.ptr);
    b.ptr = nullptr;
    b.bytes = 0;
    size_t grow = bytes + bytes / 4 + 256;
    cudaError_t e = cudaMalloc(&b.ptr, grow);
    if(e != cudaSuccess) {
        (void)cudaGetLastError();
        b.ptr = nullptr;
        return fail(GSX_B200_OUT_OF_MEMORY, std::string("cudaMalloc failed: ") + cudaGetErrorString(e));
    }
    b.bytes = grow;
    if(zero) {
        e = cudaMemset(b.ptr, 0, grow);
        if(e != cudaSuccess) return cuda_fail(e, "cudaMemset");
    }
    return 0;
}

void release(DevBuf &b)
{
    if(b.ptr) cudaFree(b.ptr);
    b.ptr = nullptr;
    b.bytes = 0;
}

CameraParams make_camera(const gsx_b200_camera &c, int row_begin, int row_end)
{
    /* gsx-cuda/render.c:870-921: normalised quaternion -> row-major R, camera centre -R^T t */
    CameraParams p;
    float qx = c.rot_xyzw[0], qy = c.rot_xyzw[1], qz = c.rot_xyzw[2], qw = c.rot_xyzw[3];
    const float nsq = qx * qx + qy * qy + qz * qz + qw * qw;
    if(nsq > 1.0e-20f) {
        const float inv = 1.0f / sqrtf(nsq);
        qx *= inv;
        qy *= inv;
        qz *= inv;
        qw *= inv;
    } else {
        qx = qy = qz = 0.0f;
        qw = 1.0f;
    }
    float r[9];
    r[0] = 1.0f - 2.0f * (qy * qy + qz * qz);
    r[1] = 2.0f * (qx * qy - qw * qz);
    r[2] = 2.0f * (qx * qz + qw * qy);
    r[3] = 2.0f * (qx * qy + qw * qz);
    r[4] = 1.0f - 2.0f * (qx * qx + qz * qz);
    r[5] = 2.0f * (qy * qz - qw * qx);
    r[6] = 2.0f * (qx * qz - qw * qy);
    r[7] = 2.0f * (qy * qz + qw * qx);
    r[8] = 1.0f - 2.0f * (qx * qx + qy * qy);
    const float *t = c.transl;
    const float w[12] = { r[0], r[1], r[2], t[0], r[3], r[4], r[5], t[1], r[6], r[7], r[8], t[2] };
    memcpy(p.w2c, w, sizeof(w));
    p.cam_pos[0] = -(r[0] * t[0] + r[3] * t[1] + r[6] * t[2]);
    p.cam_pos[1] = -(r[1] * t[0] + r[4] * t[1] + r[7] * t[2]);
    p.cam_pos[2] = -(r[2] * t[0] + r[5] * t[1] + r[8] * t[2]);
    p.fx = c.fx;
    p.fy = c.fy;
    p.cx = c.cx;
    p.cy = c.cy;
    p.width_f = (float)c.width;
    p.height_f = (float)c.height;
    p.near_plane = c.near_plane;
    p.far_plane = c.far_plane;
    p.width = c.width;
    p.height = row_end - row_begin;
    p.grid_w = (c.width + GSX_TILE - 1) / GSX_TILE;
    p.grid_h = (p.height + GSX_TILE - 1) / GSX_TILE;
    p.trow0 = row_begin / GSX_TILE;
    p.clip_l = (-0.15f * p.width_f - p.cx) / p.fx;
    p.clip_r = (1.15f * p.width_f - p.cx) / p.fx;
    p.clip_t = (-0.15f * p.height_f - p.cy) / p.fy;
    p.clip_b = (1.15f * p.height_f - p.cy) / p.fy;
    p.cull_jx = 1.0f + fmaxf(p.clip_l * p.clip_l, p.clip_r * p.clip_r);
    p.cull_jy = 1.0f + fmaxf(p.clip_t * p.clip_t, p.clip_b * p.clip_b);
    return p;
}

} // namespace

struct gsx_b200_context {
    int device = 0;
    /* per primitive */
    DevBuf rec, offsets, counts, tile_masks, block_sums, grad_acc;
    int64_t prim_cap = 0;
    /* per instance; hist = per-digit-position key histograms written by the emission kernel */
    DevBuf keys, vals, sort_scratch, hist;
    uint64_t inst_cap = 0;
    uint32_t *host_hist = nullptr; /* pinned copy of hist */
    /* per tile / pixel / bucket */
    DevBuf ranges, bucket_offsets, tile_max, pix, bucket_tile, snap, tile_count, class_tiles, tile_aux;
    /* TRAIN: per tile the pixel order by last contributor, per bucket the pixels its backward walks,
     * and the backward's bucket order and its counting-sort state */
    DevBuf tile_order, bucket_active, bucket_order, bucket_sort;
    DevBuf row_cost; /* per tile row work estimate (gsx_b200_render_row_costs) */
    /* small device words: [0] sticky flags, [1] the emission's overflow bit; from the tile scan: [2] instance total, [3] largest tile,
     * [4..8] tiles per per-tile-sort size class */
    DevBuf words;
    uint32_t *host_words = nullptr; /* pinned: [0] instance total, [1] flags, [2] largest tile, [3..7] class sizes,
                                     * [16..19] two input fingerprints (u64) */
    bool global_sort = false;       /* the last forward needed the global radix sort (a tile > GSX_SEG_MAX) */
    /* side streams and fork/join events of the per-tile sort's size classes (created on first use) */
    cudaStream_t side[GSX_SORT_CLASSES - 1] = {};
    cudaEvent_t side_ev[GSX_SORT_CLASSES] = {};
    bool side_created = false;
    /* recorded after the forward's read-back copies: the host waits on it, not on the stream, so the
     * kernels queued behind the copies keep the GPU busy meanwhile */
    cudaEvent_t readback_ev = nullptr;
    uint64_t launches = 0; /* kernels launched by this context (host-side count) */
    /* retained forward state */
    bool has_train = false;
    /* borrowed train state (gsx_b200_context_set_train_state): what a refresh needs to re-render, and
     * the inputs' fingerprints at the forward ([0]) and at the backward ([1]) */
    int train_state = GSX_B200_TRAIN_STATE_RETAINED;
    gsx_b200_camera saved_camera{};
    int saved_rows[2] = { 0, 0 };
    float saved_bg[3] = { 0.0f, 0.0f, 0.0f };
    DevBuf fingerprint, refresh_rgb;
    uint64_t refreshes = 0;
    /* bound ADC auxiliary accumulators (device [N] f32, NULL = not bound) */
    float *aux_visible = nullptr, *aux_radius = nullptr, *aux_grad = nullptr, *aux_absgrad = nullptr;
    gsx_b200_gaussians g{};
    int sh_degree = 0;
    CameraParams cam{};
    uint64_t n_instances = 0;
    uint64_t bucket_cap = 0;
    int n_tiles = 0;
    int keys_in_b = 0;
    /* per-stage event timing (gsx_b200_context_set_profiling) */
    bool profiling = false;
    cudaEvent_t ev[GSX_B200_STAGE_COUNT][kProfileSlots][2];
    int ev_count[GSX_B200_STAGE_COUNT] = {};
    bool ev_created = false;
};

namespace {

struct StageTimer {
    gsx_b200_context *ctx;
    int stage;
    cudaStream_t stream;
    int slot;
    StageTimer(gsx_b200_context *c, int s, cudaStream_t st) : ctx(c), stage(s), stream(st), slot(-1)
    {
        if(ctx->profiling && ctx->ev_count[stage] < kProfileSlots) {
            slot = ctx->ev_count[stage]++;
            cudaEventRecord(ctx->ev[stage][slot][0], stream);
        }
    }
    ~StageTimer()
    {
        if(slot >= 0) cudaEventRecord(ctx->ev[stage][slot][1], stream);
    }
};

} // namespace

/* Records `msg` as this thread's last error and returns `code` (for entry points defined in other
 * translation units of the library). */
int gsx_internal_fail(int code, const char *msg) { return fail(code, msg); }

extern "C" {

const char *gsx_b200_last_error(void) { return g_last_error.c_str(); }

const char *gsx_b200_version(void) { return "gsx-b200 0.1 (sm_100a)"; }

int gsx_b200_context_create(int device, gsx_b200_context **out_ctx)
{
    if(out_ctx == nullptr) return fail(GSX_B200_INVALID_ARGUMENT, "out_ctx must be non-null");
    *out_ctx = nullptr;
    int count = 0;
    GSX_CUDA_TRY(cudaGetDeviceCount(&count), "cudaGetDeviceCount");
    if(device < 0 || device >= count) return fail(GSX_B200_OUT_OF_RANGE, "device index out of range");
    cudaDeviceProp prop;
    GSX_CUDA_TRY(cudaGetDeviceProperties(&prop, device), "cudaGetDeviceProperties");
    if(prop.major < 10) return fail(GSX_B200_NOT_SUPPORTED, "gsx-b200 requires an sm_100 (Blackwell) device");
    GSX_CUDA_TRY(cudaSetDevice(device), "cudaSetDevice");
    gsx_b200_context *ctx = new gsx_b200_context();
    ctx->device = device;
    if(int rc = ensure(ctx->words, 64, true)) {
        delete ctx;
        return rc;
    }
    if(cudaMallocHost(&ctx->host_words, 128) != cudaSuccess) {
        release(ctx->words);
        delete ctx;
        return fail(GSX_B200_OUT_OF_MEMORY, "cudaMallocHost failed");
    }
    memset(ctx->host_words, 0, 128);
    if(cudaMallocHost(&ctx->host_hist, 8 * 256 * sizeof(uint32_t)) != cudaSuccess) {
        cudaFreeHost(ctx->host_words);
        release(ctx->words);
        delete ctx;
        return fail(GSX_B200_OUT_OF_MEMORY, "cudaMallocHost failed");
    }
    *out_ctx = ctx;
    return 0;
}

int gsx_b200_context_destroy(gsx_b200_context *ctx)
{
    if(ctx == nullptr) return 0;
    cudaSetDevice(ctx->device);
    cudaDeviceSynchronize();
    DevBuf *all[] = { &ctx->rec, &ctx->offsets, &ctx->counts, &ctx->tile_masks, &ctx->block_sums, &ctx->grad_acc, &ctx->keys, &ctx->vals,
                      &ctx->sort_scratch, &ctx->ranges, &ctx->bucket_offsets, &ctx->tile_max, &ctx->pix,
                      &ctx->bucket_tile, &ctx->snap, &ctx->tile_count, &ctx->class_tiles, &ctx->tile_aux, &ctx->words, &ctx->hist,
                      &ctx->fingerprint, &ctx->refresh_rgb, &ctx->tile_order, &ctx->bucket_active, &ctx->bucket_order,
                      &ctx->bucket_sort, &ctx->row_cost };
    for(DevBuf *b : all) release(*b);
    if(ctx->ev_created)
        for(int s = 0; s < GSX_B200_STAGE_COUNT; ++s)
            for(int k = 0; k < kProfileSlots; ++k) {
                cudaEventDestroy(ctx->ev[s][k][0]);
                cudaEventDestroy(ctx->ev[s][k][1]);
            }
    if(ctx->readback_ev) cudaEventDestroy(ctx->readback_ev);
    if(ctx->side_created) {
        for(int k = 0; k < GSX_SORT_CLASSES - 1; ++k) cudaStreamDestroy(ctx->side[k]);
        for(int k = 0; k < GSX_SORT_CLASSES; ++k) cudaEventDestroy(ctx->side_ev[k]);
    }
    if(ctx->host_words) cudaFreeHost(ctx->host_words);
    if(ctx->host_hist) cudaFreeHost(ctx->host_hist);
    delete ctx;
    return 0;
}

namespace {

/* fingerprint of the retained Gaussian inputs (ctx->g) into ctx->fingerprint word `slot` */
int launch_fingerprint(gsx_b200_context *ctx, int slot, cudaStream_t stream)
{
    if(int rc = ensure(ctx->fingerprint, 2 * sizeof(unsigned long long))) return rc;
    const gsx_b200_gaussians &g = ctx->g;
    const uint64_t n = (uint64_t)g.count;
    const float *fields[8] = { g.mean3d, g.rotation, g.logscale, g.opacity, g.sh0,
                               ctx->sh_degree >= 1 ? g.sh1 : nullptr, ctx->sh_degree >= 2 ? g.sh2 : nullptr,
                               ctx->sh_degree >= 3 ? g.sh3 : nullptr };
    const uint64_t counts[8] = { 3 * n, 4 * n, 3 * n, n, 3 * n, 9 * n, 15 * n, 21 * n };
    GSX_CUDA_TRY(gsx_launch_fingerprint(fields, counts, 8, (unsigned long long *)ctx->fingerprint.ptr + slot, stream),
                 "fingerprint launch");
    ctx->launches += 5 + (uint64_t)ctx->sh_degree;
    return 0;
}

int render_forward_impl(gsx_b200_context *ctx, const gsx_b200_gaussians *g, int sh_degree, const gsx_b200_camera *camera,
                        int row_begin, int row_end, const float background[3], int forward_type, void *out_rgb,
                        bool out_bf16, void *stream_)
{
    if(ctx == nullptr || g == nullptr || camera == nullptr || out_rgb == nullptr)
        return fail(GSX_B200_INVALID_ARGUMENT, "ctx, gaussians, camera and out_rgb must be non-null");
    if(sh_degree < 0 || sh_degree > 3) return fail(GSX_B200_OUT_OF_RANGE, "sh_degree must be in [0, 3]");
    if(forward_type != GSX_B200_FORWARD_INFERENCE && forward_type != GSX_B200_FORWARD_TRAIN)
        return fail(GSX_B200_OUT_OF_RANGE, "forward_type must be INFERENCE or TRAIN");
    if(camera->width <= 0 || camera->height <= 0) return fail(GSX_B200_INVALID_ARGUMENT, "camera size must be positive");
    if(row_begin < 0 || row_begin % GSX_TILE != 0 || row_end <= row_begin || row_end > camera->height)
        return fail(GSX_B200_OUT_OF_RANGE, "rows must satisfy 0 <= row_begin < row_end <= height, row_begin a multiple of 16");
    if(!(camera->near_plane > 0.0f) || !(camera->far_plane > camera->near_plane))
        return fail(GSX_B200_INVALID_ARGUMENT, "near_plane must be positive and below far_plane");
    if(g->count < 0 || g->count > (int64_t)INT32_MAX) return fail(GSX_B200_OUT_OF_RANGE, "gaussian count out of range");
    if(g->count > 0 && (g->mean3d == nullptr || g->rotation == nullptr || g->logscale == nullptr ||
                        g->opacity == nullptr || g->sh0 == nullptr))
        return fail(GSX_B200_INVALID_ARGUMENT, "gaussian field pointers must be non-null");
    if((sh_degree >= 1 && g->sh1 == nullptr) || (sh_degree >= 2 && g->sh2 == nullptr) || (sh_degree >= 3 && g->sh3 == nullptr))
        return fail(GSX_B200_INVALID_ARGUMENT, "higher-order SH tensors required by sh_degree are missing");
    if(((uintptr_t)g->rotation & 15u) != 0) return fail(GSX_B200_INVALID_ARGUMENT, "rotation must be 16-byte aligned");
    GSX_CUDA_TRY(cudaSetDevice(ctx->device), "cudaSetDevice");
    cudaStream_t stream = (cudaStream_t)stream_;
    const CameraParams cam = make_camera(*camera, row_begin, row_end);
    const int n_tiles = cam.grid_w * cam.grid_h;
    const int64_t n = g->count;
    const size_t P = (size_t)cam.width * (size_t)cam.height;
    const float bg[3] = { background ? background[0] : 0.0f, background ? background[1] : 0.0f,
                          background ? background[2] : 0.0f };
    ctx->has_train = false;

    /* per-primitive scratch */
    const int64_t pblocks = (n + 255) / 256;
    if(n > ctx->prim_cap) {
        if(int rc = ensure(ctx->rec, sizeof(PrimRec) * (size_t)n)) return rc;
        if(int rc = ensure(ctx->grad_acc, sizeof(float4) * 3 * (size_t)n, true)) return rc;
        ctx->prim_cap = (int64_t)(ctx->rec.bytes / sizeof(PrimRec));
        if((int64_t)(ctx->grad_acc.bytes / (3 * sizeof(float4))) < ctx->prim_cap)
            ctx->prim_cap = (int64_t)(ctx->grad_acc.bytes / (3 * sizeof(float4)));
    }
    if(int rc = ensure(ctx->offsets, sizeof(uint32_t) * (size_t)(n + 1))) return rc;
    if(int rc = ensure(ctx->counts, sizeof(uint32_t) * (size_t)(n + 1))) return rc;
    if(int rc = ensure(ctx->tile_masks, sizeof(uint32_t) * (size_t)(n + 1))) return rc;
    if(int rc = ensure(ctx->block_sums, sizeof(uint32_t) * (size_t)(pblocks + 1))) return rc;
    if(int rc = ensure(ctx->ranges, sizeof(uint2) * (size_t)n_tiles)) return rc;
    if(int rc = ensure(ctx->bucket_offsets, sizeof(uint32_t) * (size_t)n_tiles)) return rc;
    if(int rc = ensure(ctx->tile_max, sizeof(uint32_t) * (size_t)n_tiles)) return rc;
    if(int rc = ensure(ctx->pix, sizeof(float4) * P)) return rc;
    uint32_t *words = (uint32_t *)ctx->words.ptr;
    uint32_t *offsets = (uint32_t *)ctx->offsets.ptr;
    uint32_t *counts = (uint32_t *)ctx->counts.ptr;
    uint32_t *tile_masks = (uint32_t *)ctx->tile_masks.ptr;
    uint32_t *block_sums = (uint32_t *)ctx->block_sums.ptr;

    /* preprocess -> block-total scan -> emission into the current instance capacity (each instance
     * takes its rank in its tile) -> tile scan (ranges, bucket prefix, total, largest tile) -> ONE
     * read-back (instance total, largest tile, size-class counts), behind which the binning is already
     * queued (it reads the total on the device), so the GPU bins while the host waits; if the
     * capacity was too small the emission is repeated into grown buffers (rare: capacity keeps 25%
     * headroom).  Then the per-tile depth sort, or, when a tile holds more instances than shared memory
     * sorts, the global radix sort of the tile|depth keys (the binning's output is then unused). */
    int tile_bits = 0;
    while((1 << tile_bits) < n_tiles) ++tile_bits;
    const int end_bit = 32 + tile_bits;
    if(int rc = ensure(ctx->tile_count, sizeof(uint32_t) * GSX_TILE_SUBCOUNTERS * (size_t)n_tiles)) return rc;
    if(int rc = ensure(ctx->class_tiles, sizeof(uint32_t) * (size_t)n_tiles)) return rc;
    if(int rc = ensure(ctx->tile_aux, sizeof(uint32_t) * gsx_tile_scan_aux_words(n_tiles))) return rc;
    if(ctx->readback_ev == nullptr)
        GSX_CUDA_TRY(cudaEventCreateWithFlags(&ctx->readback_ev, cudaEventDisableTiming), "cudaEventCreate");
    uint32_t *tile_count = (uint32_t *)ctx->tile_count.ptr;
    uint32_t *class_tiles = (uint32_t *)ctx->class_tiles.ptr;
    uint64_t total = 0;
    uint32_t max_tile = 0;
    auto clear_counters = [&]() -> int {
        /* the emission's capacity-overflow bit lives in its own word (words[1]), cleared per pass: an
         * overflow is expected on the pass before a capacity retry.  words[0] keeps the sticky flags
         * (lookback timeouts) until gsx_b200_context_check reads them. */
        GSX_CUDA_TRY(cudaMemsetAsync(words + 1, 0, sizeof(uint32_t), stream), "memset");
        GSX_CUDA_TRY(cudaMemsetAsync(tile_count, 0, sizeof(uint32_t) * GSX_TILE_SUBCOUNTERS * (size_t)n_tiles, stream),
                     "memset");
        return 0;
    };
    bool counters_clear = false; /* cleared before the preprocess, so the kernels from the preprocess to
                                  * the tile scan follow each other directly (programmatic dependent launch) */
    auto emit_into_capacity = [&](uint64_t cap) -> int {
        /* capacity in pairs; ensure() only reallocates when the request exceeds what is held, and
         * inst_cap is the exact floor of what is held, so a steady workload never reallocates */
        if(cap == 0) cap = 1;
        if(int rc = ensure(ctx->keys, sizeof(unsigned long long) * 2 * (size_t)cap)) return rc;
        if(int rc = ensure(ctx->vals, sizeof(uint32_t) * 2 * (size_t)cap)) return rc;
        ctx->inst_cap = ctx->keys.bytes / (2 * sizeof(unsigned long long));
        const uint64_t vcap = ctx->vals.bytes / (2 * sizeof(uint32_t));
        if(vcap < ctx->inst_cap) ctx->inst_cap = vcap;
        if(!counters_clear)
            if(int rc = clear_counters()) return rc;
        counters_clear = false;
        {
            StageTimer st(ctx, 1, stream);
            GSX_CUDA_TRY(gsx_launch_emit(n, (const PrimRec *)ctx->rec.ptr, counts, tile_masks, block_sums, offsets,
                                         cam.grid_w, cam.trow0, n_tiles, (unsigned long long *)ctx->keys.ptr, (uint32_t *)ctx->vals.ptr,
                                         ctx->inst_cap, words + 1, nullptr, 0, tile_count, stream),
                         "emit launch");
            ctx->launches += n > 0 ? 1 : 0;
        }
        StageTimer st3(ctx, 3, stream);
        GSX_CUDA_TRY(gsx_launch_tile_scan(tile_count, n_tiles, (uint2 *)ctx->ranges.ptr,
                                          (uint32_t *)ctx->bucket_offsets.ptr, class_tiles,
                                          (uint32_t *)ctx->tile_aux.ptr, words + 2, stream),
                     "tile scan launch");
        ctx->launches += n_tiles > 0 ? 3 : 0;
        if(n > 0)
            GSX_CUDA_TRY(cudaMemcpyAsync(ctx->host_words, block_sums + pblocks, sizeof(uint32_t), cudaMemcpyDeviceToHost, stream),
                         "D2H");
        else
            ctx->host_words[0] = 0;
        GSX_CUDA_TRY(cudaMemcpyAsync(ctx->host_words + 2, words + 3, (1 + GSX_SORT_CLASSES) * sizeof(uint32_t),
                                     cudaMemcpyDeviceToHost, stream),
                     "D2H");
        GSX_CUDA_TRY(cudaEventRecord(ctx->readback_ev, stream), "cudaEventRecord");
        /* binning for the per-tile sort: keys/values of the emission -> (depth, primitive) keys in the
         * second half of the key buffer, count read on the device (words[2], the tile scan's total) */
        {
            const uint64_t kc = ctx->keys.bytes / (2 * sizeof(unsigned long long));
            unsigned long long *ka = (unsigned long long *)ctx->keys.ptr;
            GSX_CUDA_TRY(gsx_launch_tile_bin(ka, (const uint32_t *)ctx->vals.ptr, words + 2, ctx->inst_cap, n_tiles, tile_count, ka + kc,
                                             stream),
                         "tile bin launch");
            ctx->launches += 1;
        }
        return 0;
    };
    if(n > 0) {
        if(int rc = clear_counters()) return rc;
        counters_clear = true;
        {
            StageTimer st0(ctx, 0, stream);
            GSX_CUDA_TRY(gsx_launch_preprocess(g->mean3d, g->rotation, g->logscale, g->opacity, g->sh0, g->sh1, g->sh2,
                                               g->sh3, sh_degree, n, cam, (PrimRec *)ctx->rec.ptr, counts, tile_masks,
                                               block_sums, forward_type == GSX_B200_FORWARD_TRAIN ? ctx->aux_visible : nullptr,
                                               forward_type == GSX_B200_FORWARD_TRAIN ? ctx->aux_radius : nullptr, stream),
                         "preprocess launch");
            ctx->launches += 2;
        }
        if(int rc = emit_into_capacity(ctx->inst_cap)) return rc;
        GSX_CUDA_TRY(cudaEventSynchronize(ctx->readback_ev), "forward read-back");
        total = ctx->host_words[0];
        if(total > ctx->inst_cap) {
            if(int rc = emit_into_capacity(total + total / 4 + 1024)) return rc;
            GSX_CUDA_TRY(cudaEventSynchronize(ctx->readback_ev), "forward read-back");
        }
        max_tile = ctx->host_words[2];
    } else {
        GSX_CUDA_TRY(cudaMemsetAsync(offsets, 0, sizeof(uint32_t), stream), "memset");
        if(int rc = emit_into_capacity(ctx->inst_cap)) return rc;
        GSX_CUDA_TRY(cudaEventSynchronize(ctx->readback_ev), "forward read-back");
    }
    ctx->n_instances = total;
    const uint64_t bucket_cap = (total + 31) / 32 + (uint64_t)n_tiles;
    if(forward_type == GSX_B200_FORWARD_TRAIN) {
        /* bucket snapshots, the bucket -> tile table, the per-tile pixel order and the per-bucket pixel
         * counts exist for the backward only */
        if(int rc = ensure(ctx->bucket_tile, sizeof(uint32_t) * (size_t)bucket_cap)) return rc;
        if(int rc = ensure(ctx->snap, sizeof(float4) * GSX_TILE_PIXELS * (size_t)bucket_cap)) return rc;
        if(int rc = ensure(ctx->bucket_active, sizeof(uint16_t) * (size_t)bucket_cap)) return rc;
        if(int rc = ensure(ctx->tile_order, (size_t)GSX_TILE_PIXELS * (size_t)n_tiles)) return rc;
    }
    const uint64_t kcap = ctx->keys.bytes / (2 * sizeof(unsigned long long));
    unsigned long long *keys_a = (unsigned long long *)ctx->keys.ptr;
    unsigned long long *keys_b = keys_a + kcap;
    uint32_t *vals_a = (uint32_t *)ctx->vals.ptr;
    uint32_t *vals_b = vals_a + ctx->vals.bytes / (2 * sizeof(uint32_t));
    int in_b = 0;
    ctx->global_sort = false;
    if(total > 0) {
        StageTimer st(ctx, 2, stream);
        if(max_tile <= (uint32_t)GSX_SEG_MAX) {
            if(!ctx->side_created) {
                for(int k = 0; k < GSX_SORT_CLASSES - 1; ++k)
                    GSX_CUDA_TRY(cudaStreamCreateWithFlags(&ctx->side[k], cudaStreamNonBlocking), "cudaStreamCreate");
                for(int k = 0; k < GSX_SORT_CLASSES; ++k)
                    GSX_CUDA_TRY(cudaEventCreateWithFlags(&ctx->side_ev[k], cudaEventDisableTiming), "cudaEventCreate");
                ctx->side_created = true;
            }
            GSX_CUDA_TRY(gsx_launch_tile_sort(total, n_tiles, (const uint2 *)ctx->ranges.ptr, class_tiles, ctx->host_words + 3,
                                              keys_b, keys_a, vals_a, stream, ctx->side, ctx->side_ev),
                         "tile sort launch");
            for(int c = 0; c < GSX_SORT_CLASSES; ++c) ctx->launches += ctx->host_words[3 + c] ? 1 : 0;
        } else {
            /* a tile too large for shared memory: stable global radix sort of the tile|depth keys
             * (emitted in primitive order, so equal depths stay in primitive order) */
            ctx->global_sort = true;
            if(int rc = ensure(ctx->sort_scratch, gsx_sort_scratch_bytes(total + 1))) return rc;
            GSX_CUDA_TRY(gsx_launch_sort_pairs(keys_a, vals_a, keys_b, vals_b, total, 0, end_bit, ctx->sort_scratch.ptr,
                                               ctx->sort_scratch.bytes, words, &in_b, stream),
                         "sort launch");
            ctx->launches += 1 + (uint64_t)((end_bit + 7) / 8);
        }
    }
    const uint32_t *vals = in_b ? vals_b : vals_a;
    /* Largest-tiles-first order for the blend when the grid is only a few waves (about 740 CTAs of
     * 256 threads are resident at once on 148 SMs): there the last wave's long tiles decide the time.
     * With many waves the raster order wins, as neighbouring tiles share instance records in L2. */
    int sms = 148;
    (void)cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, ctx->device);
    const bool lpt = n_tiles <= sms * 5 * 8;
    {
    StageTimer st4(ctx, 4, stream);
    GSX_CUDA_TRY(gsx_launch_blend_forward(cam.width, cam.height, row_begin, cam.grid_w, n_tiles, (const uint2 *)ctx->ranges.ptr,
                                          (const uint32_t *)ctx->bucket_offsets.ptr, vals, (const PrimRec *)ctx->rec.ptr, bg,
                                          out_rgb, out_bf16, (float4 *)ctx->pix.ptr, (uint32_t *)ctx->tile_max.ptr,
                                          (float4 *)ctx->snap.ptr, (uint32_t *)ctx->bucket_tile.ptr,
                                          forward_type == GSX_B200_FORWARD_TRAIN, lpt ? class_tiles : nullptr, words + 4,
                                          (uint8_t *)ctx->tile_order.ptr, (uint16_t *)ctx->bucket_active.ptr, stream),
                 "blend launch");
    ctx->launches += n_tiles > 0 ? 1 : 0;
    }
    ctx->keys_in_b = in_b;
    ctx->bucket_cap = bucket_cap;
    ctx->n_tiles = n_tiles;
    ctx->cam = cam;
    if(forward_type == GSX_B200_FORWARD_TRAIN) {
        ctx->has_train = true;
        ctx->g = *g;
        ctx->sh_degree = sh_degree;
        if(ctx->train_state == GSX_B200_TRAIN_STATE_BORROWED) {
            /* keep what a refresh re-renders with, and fingerprint the borrowed inputs */
            ctx->saved_camera = *camera;
            ctx->saved_rows[0] = row_begin;
            ctx->saved_rows[1] = row_end;
            memcpy(ctx->saved_bg, bg, sizeof(bg));
            if(int rc = launch_fingerprint(ctx, 0, stream)) {
                ctx->has_train = false;
                return rc;
            }
        }
    }
    return 0;
}

/* Borrowed train state: the backward of the CURRENT inputs, as gsx-cuda/render.c:662-756 refreshes a
 * borrowed TRAIN state.  The inputs are fingerprinted again; if they differ from the forward's, the TRAIN
 * forward is re-run on them (into a private image, without touching the density-control statistics)
 * before the backward uses the retained state.  Unchanged inputs cost one read of the fields and one
 * host wait. */
int refresh_borrowed(gsx_b200_context *ctx, cudaStream_t stream)
{
    if(ctx->g.count == 0) return 0;
    if(int rc = launch_fingerprint(ctx, 1, stream)) return rc;
    unsigned long long *h = reinterpret_cast<unsigned long long *>(ctx->host_words + 16);
    GSX_CUDA_TRY(cudaMemcpyAsync(h, ctx->fingerprint.ptr, 2 * sizeof(unsigned long long), cudaMemcpyDeviceToHost, stream),
                 "D2H");
    GSX_CUDA_TRY(cudaStreamSynchronize(stream), "fingerprint read-back");
    if(h[0] == h[1]) return 0;
    const gsx_b200_gaussians g = ctx->g;
    const gsx_b200_camera cam = ctx->saved_camera;
    const int r0 = ctx->saved_rows[0], r1 = ctx->saved_rows[1];
    float bg[3];
    memcpy(bg, ctx->saved_bg, sizeof(bg));
    const size_t P = (size_t)cam.width * (size_t)(r1 - r0);
    if(int rc = ensure(ctx->refresh_rgb, 3 * sizeof(float) * P)) return rc;
    float *keep_visible = ctx->aux_visible, *keep_radius = ctx->aux_radius;
    ctx->aux_visible = nullptr;
    ctx->aux_radius = nullptr;
    const int rc = render_forward_impl(ctx, &g, ctx->sh_degree, &cam, r0, r1, bg, GSX_B200_FORWARD_TRAIN,
                                       ctx->refresh_rgb.ptr, false, stream);
    ctx->aux_visible = keep_visible;
    ctx->aux_radius = keep_radius;
    if(rc == 0) ++ctx->refreshes;
    return rc;
}

} // namespace

int gsx_b200_render_forward(gsx_b200_context *ctx, const gsx_b200_gaussians *g, int sh_degree,
                            const gsx_b200_camera *camera, const float background[3], int forward_type, float *out_rgb,
                            void *stream)
{
    if(camera == nullptr) return fail(GSX_B200_INVALID_ARGUMENT, "camera must be non-null");
    return render_forward_impl(ctx, g, sh_degree, camera, 0, camera->height, background, forward_type, out_rgb, false,
                               stream);
}

int gsx_b200_render_forward_rows(gsx_b200_context *ctx, const gsx_b200_gaussians *g, int sh_degree,
                                 const gsx_b200_camera *camera, int row_begin, int row_end, const float background[3],
                                 int forward_type, void *out_rgb, int out_bf16, void *stream)
{
    if(camera == nullptr) return fail(GSX_B200_INVALID_ARGUMENT, "camera must be non-null");
    return render_forward_impl(ctx, g, sh_degree, camera, row_begin, row_end, background, forward_type, out_rgb,
                               out_bf16 != 0, stream);
}

int gsx_b200_render_row_costs(gsx_b200_context *ctx, const gsx_b200_gaussians *g, const gsx_b200_camera *camera,
                              uint32_t *host_row_costs, int32_t n_rows, void *stream_)
{
    if(ctx == nullptr || g == nullptr || camera == nullptr || host_row_costs == nullptr)
        return fail(GSX_B200_INVALID_ARGUMENT, "ctx, gaussians, camera and host_row_costs must be non-null");
    if(camera->width <= 0 || camera->height <= 0) return fail(GSX_B200_INVALID_ARGUMENT, "camera size must be positive");
    const CameraParams cam = make_camera(*camera, 0, camera->height);
    if(n_rows != cam.grid_h) return fail(GSX_B200_INVALID_ARGUMENT, "n_rows must be the frame's tile rows, ceil(height / 16)");
    if(cam.grid_h > 1024) return fail(GSX_B200_OUT_OF_RANGE, "at most 1024 tile rows");
    if(g->count > 0 && (g->mean3d == nullptr || g->logscale == nullptr))
        return fail(GSX_B200_INVALID_ARGUMENT, "mean3d and logscale must be non-null");
    GSX_CUDA_TRY(cudaSetDevice(ctx->device), "cudaSetDevice");
    cudaStream_t stream = (cudaStream_t)stream_;
    if(int rc = ensure(ctx->row_cost, sizeof(uint32_t) * 1024)) return rc;
    GSX_CUDA_TRY(gsx_launch_band_cost(g->mean3d, g->logscale, g->count, cam, (uint32_t *)ctx->row_cost.ptr, stream),
                 "row cost launch");
    ctx->launches += g->count > 0 ? 1 : 0;
    GSX_CUDA_TRY(cudaMemcpyAsync(host_row_costs, ctx->row_cost.ptr, sizeof(uint32_t) * (size_t)n_rows,
                                 cudaMemcpyDeviceToHost, stream),
                 "D2H");
    GSX_CUDA_TRY(cudaStreamSynchronize(stream), "sync");
    return 0;
}

int gsx_b200_render_backward(gsx_b200_context *ctx, const float *grad_rgb, const gsx_b200_gaussian_grads *gr,
                             void *stream_)
{
    if(ctx == nullptr || grad_rgb == nullptr || gr == nullptr)
        return fail(GSX_B200_INVALID_ARGUMENT, "ctx, grad_rgb and grads must be non-null");
    if(!ctx->has_train) return fail(GSX_B200_INVALID_STATE, "backward requires a retained TRAIN forward on the same context");
    const int64_t n = ctx->g.count;
    if(n > 0 && (gr->mean3d == nullptr || gr->rotation == nullptr || gr->logscale == nullptr || gr->opacity == nullptr ||
                 gr->sh0 == nullptr))
        return fail(GSX_B200_INVALID_ARGUMENT, "gradient pointers must be non-null");
    if((ctx->sh_degree >= 1 && gr->sh1 == nullptr) || (ctx->sh_degree >= 2 && gr->sh2 == nullptr) ||
       (ctx->sh_degree >= 3 && gr->sh3 == nullptr))
        return fail(GSX_B200_INVALID_ARGUMENT, "higher-order SH gradient tensors required by sh_degree are missing");
    if(((uintptr_t)gr->rotation & 15u) != 0) return fail(GSX_B200_INVALID_ARGUMENT, "rotation gradient must be 16-byte aligned");
    GSX_CUDA_TRY(cudaSetDevice(ctx->device), "cudaSetDevice");
    cudaStream_t stream = (cudaStream_t)stream_;
    if(n == 0) return 0;
    if(ctx->train_state == GSX_B200_TRAIN_STATE_BORROWED)
        if(int rc = refresh_borrowed(ctx, stream)) return rc;
    const unsigned long long *keys_a = (const unsigned long long *)ctx->keys.ptr;
    (void)keys_a;
    const uint32_t *vals_a = (const uint32_t *)ctx->vals.ptr;
    const uint32_t *vals = ctx->keys_in_b ? vals_a + ctx->vals.bytes / (2 * sizeof(uint32_t)) : vals_a;
    if(ctx->n_instances > 0) {
        StageTimer st(ctx, 5, stream);
        if(int rc = ensure(ctx->bucket_order, sizeof(uint32_t) * (size_t)ctx->bucket_cap)) return rc;
        if(int rc = ensure(ctx->bucket_sort, sizeof(uint32_t) * gsx_bucket_sort_state_words())) return rc;
        GSX_CUDA_TRY(gsx_launch_blend_backward(ctx->cam.width, ctx->cam.height, ctx->cam.trow0 * GSX_TILE, ctx->cam.grid_w,
                                               (const uint2 *)ctx->ranges.ptr, (const uint32_t *)ctx->bucket_offsets.ptr,
                                               (const uint32_t *)ctx->bucket_tile.ptr, ctx->bucket_cap, ctx->n_tiles,
                                               (const uint16_t *)ctx->bucket_active.ptr, (const uint8_t *)ctx->tile_order.ptr,
                                               (uint32_t *)ctx->bucket_order.ptr, (uint32_t *)ctx->bucket_sort.ptr, vals,
                                               (const PrimRec *)ctx->rec.ptr, (const float4 *)ctx->pix.ptr,
                                               (const float4 *)ctx->snap.ptr, grad_rgb, (float4 *)ctx->grad_acc.ptr,
                                               ctx->aux_absgrad != nullptr, stream),
                     "blend backward launch");
        ctx->launches += 3;
    }
    StageTimer st6(ctx, 6, stream);
    GSX_CUDA_TRY(gsx_launch_preprocess_backward(ctx->g.mean3d, ctx->g.rotation, ctx->g.logscale, ctx->g.sh1, ctx->g.sh2,
                                                ctx->g.sh3, ctx->sh_degree, n, ctx->cam, (const uint32_t *)ctx->counts.ptr,
                                                (float4 *)ctx->grad_acc.ptr, gr->mean3d, gr->rotation, gr->logscale,
                                                gr->opacity, gr->sh0, gr->sh1, gr->sh2, gr->sh3, ctx->aux_grad,
                                                ctx->aux_absgrad, stream),
                 "preprocess backward launch");
    ctx->launches += 1;
    return 0;
}

int gsx_b200_render_bind_aux(gsx_b200_context *ctx, float *visible_counter, float *max_screen_radius, float *grad_acc,
                             float *absgrad_acc)
{
    if(ctx == nullptr) return fail(GSX_B200_INVALID_ARGUMENT, "ctx must be non-null");
    ctx->aux_visible = visible_counter;
    ctx->aux_radius = max_screen_radius;
    ctx->aux_grad = grad_acc;
    ctx->aux_absgrad = absgrad_acc;
    return 0;
}

int gsx_b200_context_set_train_state(gsx_b200_context *ctx, int mode)
{
    if(ctx == nullptr) return fail(GSX_B200_INVALID_ARGUMENT, "ctx must be non-null");
    if(mode != GSX_B200_TRAIN_STATE_RETAINED && mode != GSX_B200_TRAIN_STATE_BORROWED)
        return fail(GSX_B200_OUT_OF_RANGE, "mode must be GSX_B200_TRAIN_STATE_RETAINED or _BORROWED");
    if(mode != ctx->train_state) ctx->has_train = false; /* a retained forward belongs to the mode it ran in */
    ctx->train_state = mode;
    return 0;
}

int gsx_b200_context_train_refreshes(gsx_b200_context *ctx, uint64_t *out_count)
{
    if(ctx == nullptr || out_count == nullptr) return fail(GSX_B200_INVALID_ARGUMENT, "ctx and out_count must be non-null");
    *out_count = ctx->refreshes;
    return 0;
}

int gsx_b200_context_launch_count(gsx_b200_context *ctx, uint64_t *out_count)
{
    if(ctx == nullptr || out_count == nullptr) return fail(GSX_B200_INVALID_ARGUMENT, "ctx and out_count must be non-null");
    *out_count = ctx->launches;
    return 0;
}

int gsx_b200_render_stats(gsx_b200_context *ctx, uint64_t *n_visible, uint64_t *n_instances, uint64_t *n_buckets,
                          void *stream_)
{
    if(ctx == nullptr) return fail(GSX_B200_INVALID_ARGUMENT, "ctx must be non-null");
    cudaStream_t stream = (cudaStream_t)stream_;
    GSX_CUDA_TRY(cudaSetDevice(ctx->device), "cudaSetDevice");
    GSX_CUDA_TRY(cudaStreamSynchronize(stream), "sync");
    if(n_instances) *n_instances = ctx->n_instances;
    if(n_buckets) {
        uint32_t b = 0;
        if(ctx->n_tiles > 0)
            GSX_CUDA_TRY(cudaMemcpy(&b, (uint32_t *)ctx->bucket_offsets.ptr + ctx->n_tiles - 1, 4, cudaMemcpyDeviceToHost), "D2H");
        *n_buckets = b;
    }
    if(n_visible) {
        /* visible = primitives with a non-zero tile count (host pass over offsets; debug use) */
        *n_visible = 0;
        const int64_t n = ctx->g.count;
        if(n > 0 && ctx->has_train) {
            uint32_t *h = new uint32_t[(size_t)n + 1];
            cudaError_t e = cudaMemcpy(h, ctx->offsets.ptr, sizeof(uint32_t) * (size_t)(n + 1), cudaMemcpyDeviceToHost);
            if(e != cudaSuccess) {
                delete[] h;
                return cuda_fail(e, "D2H");
            }
            uint64_t v = 0;
            for(int64_t i = 0; i < n; ++i) v += h[i + 1] != h[i];
            delete[] h;
            *n_visible = v;
        }
    }
    return 0;
}

int gsx_b200_render_get_view(gsx_b200_context *ctx, gsx_b200_render_view *v)
{
    if(ctx == nullptr || v == nullptr) return fail(GSX_B200_INVALID_ARGUMENT, "ctx and out_view must be non-null");
    const uint64_t kcap = ctx->keys.bytes / (2 * sizeof(unsigned long long));
    const uint64_t vcap = ctx->vals.bytes / (2 * sizeof(uint32_t));
    v->keys = (const uint64_t *)ctx->keys.ptr + (ctx->keys_in_b ? kcap : 0);
    v->values = (const uint32_t *)ctx->vals.ptr + (ctx->keys_in_b ? vcap : 0);
    v->ranges = (const uint32_t *)ctx->ranges.ptr;
    v->offsets = (const uint32_t *)ctx->offsets.ptr;
    v->tile_max = (const uint32_t *)ctx->tile_max.ptr;
    v->pixel_state = (const float *)ctx->pix.ptr;
    v->n_instances = ctx->n_instances;
    v->n_tiles = ctx->n_tiles;
    v->grid_width = ctx->cam.grid_w;
    return 0;
}

int gsx_b200_context_check(gsx_b200_context *ctx, void *stream_)
{
    if(ctx == nullptr) return fail(GSX_B200_INVALID_ARGUMENT, "ctx must be non-null");
    cudaStream_t stream = (cudaStream_t)stream_;
    GSX_CUDA_TRY(cudaSetDevice(ctx->device), "cudaSetDevice");
    uint32_t flags = 0;
    GSX_CUDA_TRY(cudaMemcpyAsync(ctx->host_words + 1, ctx->words.ptr, 4, cudaMemcpyDeviceToHost, stream), "D2H");
    GSX_CUDA_TRY(cudaStreamSynchronize(stream), "sync");
    flags = ctx->host_words[1];
    if(flags != 0) {
        GSX_CUDA_TRY(cudaMemsetAsync(ctx->words.ptr, 0, 4, stream), "memset");
        GSX_CUDA_TRY(cudaStreamSynchronize(stream), "sync");
        std::string m = "device-side failure:";
        if(flags & GSX_FLAG_LOOKBACK_TIMEOUT) m += " lookback wait timed out;";
        if(flags & GSX_FLAG_INSTANCE_OVERFLOW) m += " instance capacity overflow;";
        if(flags & GSX_FLAG_BUCKET_OVERFLOW) m += " bucket capacity overflow;";
        return fail(GSX_B200_UNKNOWN, m);
    }
    return 0;
}

int gsx_b200_context_set_profiling(gsx_b200_context *ctx, int enable)
{
    if(ctx == nullptr) return fail(GSX_B200_INVALID_ARGUMENT, "ctx must be non-null");
    GSX_CUDA_TRY(cudaSetDevice(ctx->device), "cudaSetDevice");
    if(enable && !ctx->ev_created) {
        for(int s = 0; s < GSX_B200_STAGE_COUNT; ++s)
            for(int k = 0; k < kProfileSlots; ++k) {
                GSX_CUDA_TRY(cudaEventCreate(&ctx->ev[s][k][0]), "cudaEventCreate");
                GSX_CUDA_TRY(cudaEventCreate(&ctx->ev[s][k][1]), "cudaEventCreate");
            }
        ctx->ev_created = true;
    }
    ctx->profiling = enable != 0;
    return 0;
}

int gsx_b200_context_read_profile(gsx_b200_context *ctx, float *total_ms, int32_t *launches)
{
    if(ctx == nullptr || total_ms == nullptr || launches == nullptr)
        return fail(GSX_B200_INVALID_ARGUMENT, "ctx, total_ms and launches must be non-null");
    GSX_CUDA_TRY(cudaSetDevice(ctx->device), "cudaSetDevice");
    for(int s = 0; s < GSX_B200_STAGE_COUNT; ++s) {
        float sum = 0.0f;
        for(int k = 0; k < ctx->ev_count[s]; ++k) {
            GSX_CUDA_TRY(cudaEventSynchronize(ctx->ev[s][k][1]), "cudaEventSynchronize");
            float ms = 0.0f;
            GSX_CUDA_TRY(cudaEventElapsedTime(&ms, ctx->ev[s][k][0], ctx->ev[s][k][1]), "cudaEventElapsedTime");
            sum += ms;
        }
        total_ms[s] = sum;
        launches[s] = ctx->ev_count[s];
        ctx->ev_count[s] = 0;
    }
    return 0;
}

int gsx_b200_loss_l1_ssim(int mode, const float *prediction, const float *target, float *loss_map, float *grad,
                          float *loss_sum, int64_t planes, int32_t height, int32_t width, float l1_scale, float ssim_scale,
                          float l1_grad_scale, float ssim_grad_scale, void *stream)
{
    if(prediction == nullptr || target == nullptr) return fail(GSX_B200_INVALID_ARGUMENT, "prediction and target must be non-null");
    if((mode & 1) && loss_map == nullptr) return fail(GSX_B200_INVALID_ARGUMENT, "loss_map required by mode");
    if((mode & 2) && grad == nullptr) return fail(GSX_B200_INVALID_ARGUMENT, "grad required by mode");
    const int base_mode = mode & 7;
    if((mode & ~15) != 0 || (base_mode != 1 && base_mode != 2 && base_mode != 3 && base_mode != 5 && base_mode != 7))
        return fail(GSX_B200_OUT_OF_RANGE, "mode must be 1, 2, 3, 5 or 7, optionally with the overwrite bit 8");
    if(planes <= 0 || height <= 0 || width <= 0) return fail(GSX_B200_INVALID_ARGUMENT, "image shape must be positive");
    if(planes > INT32_MAX) return fail(GSX_B200_OUT_OF_RANGE, "too many planes");
    GSX_CUDA_TRY(gsx_launch_l1_ssim(mode, prediction, target, loss_map, grad, loss_sum, (int)planes, height, width, l1_scale,
                                    ssim_scale, l1_grad_scale, ssim_grad_scale, (cudaStream_t)stream),
                 "l1_ssim launch");
    return 0;
}

int gsx_b200_loss_pointwise(int op, const float *prediction, const float *target, float *out, uint64_t n, float scale,
                            void *stream)
{
    if(op < 0 || op > 3) return fail(GSX_B200_OUT_OF_RANGE, "op must be in [0, 3]");
    if(n > 0 && (prediction == nullptr || target == nullptr || out == nullptr))
        return fail(GSX_B200_INVALID_ARGUMENT, "pointers must be non-null");
    GSX_CUDA_TRY(gsx_launch_pointwise_loss(op, prediction, target, out, (size_t)n, scale, (cudaStream_t)stream),
                 "pointwise loss launch");
    return 0;
}

int gsx_b200_adam_step(const gsx_b200_adam_group *groups, int32_t group_count, void *stream)
{
    if(group_count < 0 || group_count > 16) return fail(GSX_B200_OUT_OF_RANGE, "group_count must be in [0, 16]");
    if(group_count > 0 && groups == nullptr) return fail(GSX_B200_INVALID_ARGUMENT, "groups must be non-null");
    AdamTable t;
    memset(&t, 0, sizeof(t));
    t.count = group_count;
    for(int i = 0; i < group_count; ++i) {
        const gsx_b200_adam_group &g = groups[i];
        if(g.count > 0 && (g.parameter == nullptr || g.gradient == nullptr || g.first_moment == nullptr || g.second_moment == nullptr))
            return fail(GSX_B200_INVALID_ARGUMENT, "adam group pointers must be non-null");
        t.g[i].param = g.parameter;
        t.g[i].grad = g.gradient;
        t.g[i].m1 = g.first_moment;
        t.g[i].m2 = g.second_moment;
        t.g[i].n = g.count;
        t.g[i].lr = g.learning_rate;
        t.g[i].beta1 = g.beta1;
        t.g[i].beta2 = g.beta2;
        t.g[i].eps = g.epsilon;
        t.g[i].weight_decay = g.weight_decay;
        t.g[i].max_grad = g.max_grad;
        t.g[i].inv_c1 = g.inv_bias_correction1;
        t.g[i].inv_c2 = g.inv_bias_correction2;
    }
    GSX_CUDA_TRY(gsx_launch_adam(t, (cudaStream_t)stream), "adam launch");
    return 0;
}

int gsx_b200_sort_pairs(gsx_b200_context *ctx, uint64_t *keys, uint32_t *values, uint64_t count, int32_t begin_bit,
                        int32_t end_bit, void *stream_)
{
    if(ctx == nullptr || (count > 0 && (keys == nullptr || values == nullptr)))
        return fail(GSX_B200_INVALID_ARGUMENT, "ctx, keys and values must be non-null");
    if(begin_bit < 0 || end_bit > 64 || begin_bit > end_bit) return fail(GSX_B200_OUT_OF_RANGE, "bit range must satisfy 0 <= begin <= end <= 64");
    if(count >= (1ull << 30)) return fail(GSX_B200_OUT_OF_RANGE, "count must be below 2^30");
    if(count == 0 || begin_bit == end_bit) return 0;
    GSX_CUDA_TRY(cudaSetDevice(ctx->device), "cudaSetDevice");
    cudaStream_t stream = (cudaStream_t)stream_;
    /* alternate buffers come from the context's instance scratch (invalidates a retained forward) */
    ctx->has_train = false;
    if(int rc = ensure(ctx->keys, sizeof(unsigned long long) * (size_t)count)) return rc;
    if(int rc = ensure(ctx->vals, sizeof(uint32_t) * (size_t)count)) return rc;
    if(int rc = ensure(ctx->sort_scratch, gsx_sort_scratch_bytes(count))) return rc;
    int in_b = 0;
    GSX_CUDA_TRY(gsx_launch_sort_pairs((unsigned long long *)keys, values, (unsigned long long *)ctx->keys.ptr,
                                       (uint32_t *)ctx->vals.ptr, count, begin_bit, end_bit, ctx->sort_scratch.ptr,
                                       ctx->sort_scratch.bytes, (uint32_t *)ctx->words.ptr, &in_b, stream),
                 "sort launch");
    if(in_b) {
        GSX_CUDA_TRY(cudaMemcpyAsync(keys, ctx->keys.ptr, sizeof(uint64_t) * count, cudaMemcpyDeviceToDevice, stream), "copy");
        GSX_CUDA_TRY(cudaMemcpyAsync(values, ctx->vals.ptr, sizeof(uint32_t) * count, cudaMemcpyDeviceToDevice, stream), "copy");
    }
    return 0;
}

} /* extern "C" */
