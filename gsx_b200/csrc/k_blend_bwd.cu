/*
 * Reverse-mode blend: one warp per 32-instance bucket, one instance per lane, walking the
 * tile's 256 pixels with per-pixel state handed lane to lane.
 *
 * Follows fastgs/kernels_backward.cuh:484-730 (blend_backward_cu2, after Taming-3DGS) for the
 * gradient rules: the state of each pixel starts from the forward snapshot taken before the
 * bucket (colour, transmittance) and from the composed image; fragments at or beyond the pixel's
 * last contributor are skipped; sigma is clamped at 0 (no 1/255 skip in the backward), alpha at
 * 0.999 with no opacity gradient when saturated, and (1 - alpha) is floored at 1e-4 in the
 * division.  Buckets at or beyond the tile's maximum contributor are skipped.
 *
 * B200 choices: the four 2-D gradient groups of an instance are accumulated in registers over all
 * 256 pixels and flushed with two 16-byte vector atomics (red.global.add.v4.f32) plus one scalar
 * atomic, instead of 9-11 scalar atomics; the grid is sized from the bucket capacity and buckets
 * past the device-side bucket count exit immediately (no host round trip for the count).
 */
#include "gsx_b200_kernels.cuh"

namespace {

constexpr int kWarps = 8;
constexpr int kThreads = 32 * kWarps;

__global__ void __launch_bounds__(kThreads) blend_backward_kernel(
    int width, int height, int grid_w, int n_tiles, const uint2 *__restrict__ ranges,
    const uint32_t *__restrict__ bucket_offsets, const uint32_t *__restrict__ bucket_tile,
    const uint32_t *__restrict__ vals, const PrimRec *__restrict__ rec, const float4 *__restrict__ pix,
    const uint32_t *__restrict__ tile_max, const float4 *__restrict__ snap, const float *__restrict__ grad_rgb,
    float4 *__restrict__ grad_acc)
{
    __shared__ float4 s_up[kWarps][32]; /* grad r, g, b, last contributor bits */
    __shared__ float4 s_lo[kWarps][32]; /* colour after (r, g, b), transmittance before bucket */
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t bucket = blockIdx.x * kWarps + warp;
    const uint32_t n_buckets = bucket_offsets[n_tiles - 1];
    if(bucket >= n_buckets) return;
    const uint32_t tile = bucket_tile[bucket];
    const uint2 range = ranges[tile];
    const int n_inst = (int)(range.y - range.x);
    const uint32_t first = tile == 0 ? 0u : bucket_offsets[tile - 1];
    const int tb = (int)(bucket - first);
    if((uint32_t)tb * 32u >= tile_max[tile]) return;
    const int tpi = tb * 32 + lane;
    const bool valid_prim = tpi < n_inst;

    uint32_t prim = 0;
    float mx = 0.0f, my = 0.0f, cx = 0.0f, cy = 0.0f, cz = 0.0f, op = 0.0f;
    float colr = 0.0f, colg = 0.0f, colb = 0.0f, fr = 0.0f, fg = 0.0f, fb = 0.0f;
    if(valid_prim) {
        prim = vals[range.x + tpi];
        const PrimRec r = rec[prim];
        mx = r.a.x - 0.5f;
        my = r.a.y - 0.5f;
        cx = r.a.z;
        cy = r.a.w;
        cz = r.b.x;
        op = r.b.y;
        colr = fmaxf(r.b.z, 0.0f);
        colg = fmaxf(r.b.w, 0.0f);
        colb = fmaxf(r.c.x, 0.0f);
        fr = r.b.z >= 0.0f ? 1.0f : 0.0f;
        fg = r.b.w >= 0.0f ? 1.0f : 0.0f;
        fb = r.c.x >= 0.0f ? 1.0f : 0.0f;
    }
    const int tx0 = (int)(tile % (uint32_t)grid_w) * GSX_TILE, ty0 = (int)(tile / (uint32_t)grid_w) * GSX_TILE;
    const size_t P = (size_t)width * (size_t)height;
    const float4 *bsnap = snap + (size_t)bucket * GSX_TILE_PIXELS;

    float g_mx = 0.0f, g_my = 0.0f, g_cx = 0.0f, g_cy = 0.0f, g_cz = 0.0f, g_op = 0.0f;
    float g_r = 0.0f, g_g = 0.0f, g_b = 0.0f;
    /* per-pixel state travelling along the lanes */
    float pgr = 0.0f, pgg = 0.0f, pgb = 0.0f, par = 0.0f, pag = 0.0f, pab = 0.0f, pT = 0.0f;
    uint32_t plast = 0;

    for(int i = 0; i < GSX_TILE_PIXELS + 31; ++i) {
        if((i & 31) == 0 && i < GSX_TILE_PIXELS) {
            const int p = i + lane;
            const int qx = tx0 + (p & (GSX_TILE - 1)), qy = ty0 + (p >> 4);
            float4 up = make_float4(0.0f, 0.0f, 0.0f, 0.0f), lo = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if(qx < width && qy < height) {
                const size_t idx = (size_t)qy * (size_t)width + (size_t)qx;
                const float4 s = bsnap[p];
                const float4 img = pix[idx];
                up = make_float4(grad_rgb[idx], grad_rgb[P + idx], grad_rgb[2 * P + idx], img.w);
                lo = make_float4(img.x - s.x, img.y - s.y, img.z - s.z, s.w);
            }
            s_up[warp][lane] = up;
            s_lo[warp][lane] = lo;
            __syncwarp();
        }
        pgr = __shfl_up_sync(0xffffffffu, pgr, 1);
        pgg = __shfl_up_sync(0xffffffffu, pgg, 1);
        pgb = __shfl_up_sync(0xffffffffu, pgb, 1);
        plast = __shfl_up_sync(0xffffffffu, plast, 1);
        par = __shfl_up_sync(0xffffffffu, par, 1);
        pag = __shfl_up_sync(0xffffffffu, pag, 1);
        pab = __shfl_up_sync(0xffffffffu, pab, 1);
        pT = __shfl_up_sync(0xffffffffu, pT, 1);
        if(lane == 0 && i < GSX_TILE_PIXELS) {
            const float4 up = s_up[warp][i & 31];
            const float4 lo = s_lo[warp][i & 31];
            pgr = up.x;
            pgg = up.y;
            pgb = up.z;
            plast = __float_as_uint(up.w);
            par = lo.x;
            pag = lo.y;
            pab = lo.z;
            pT = lo.w;
        }
        const int idx = i - lane;
        if(idx < 0 || idx >= GSX_TILE_PIXELS) continue;
        const int qx = tx0 + (idx & (GSX_TILE - 1)), qy = ty0 + (idx >> 4);
        if(!valid_prim || qx >= width || qy >= height || (uint32_t)tpi >= plast) continue;
        const float dx = mx - (float)qx, dy = my - (float)qy;
        const float dxx = dx * dx, dxy = dx * dy, dyy = dy * dy;
        const float sig = fmaxf(0.5f * (cx * dxx + cz * dyy) + cy * dxy, 0.0f);
        const float a_pre = op * __expf(-sig);
        const float alpha = fminf(a_pre, 0.999f);
        const bool sat = a_pre >= 0.999f;
        const float wgt = pT * alpha;
        g_r += wgt * (pgr * fr);
        g_g += wgt * (pgg * fg);
        g_b += wgt * (pgb * fb);
        par -= wgt * colr;
        pag -= wgt * colg;
        pab -= wgt * colb;
        const float cdg = colr * pgr + colg * pgg + colb * pgb;
        const float adg = par * pgr + pag * pgg + pab * pgb;
        const float oma = 1.0f - alpha;
        const float dl_dalpha = pT * cdg - adg * (1.0f / fmaxf(oma, 1e-4f));
        const float part = sat ? 0.0f : alpha * dl_dalpha;
        g_cx += -0.5f * part * dxx;
        g_cy += -part * dxy;
        g_cz += -0.5f * part * dyy;
        g_mx -= part * (cx * dx + cy * dy);
        g_my -= part * (cy * dx + cz * dy);
        g_op += part;
        pT *= oma;
    }
    if(valid_prim) {
        float4 *acc = grad_acc + (size_t)prim * 3;
        atomicAdd(acc + 0, make_float4(g_mx, g_my, g_cx, g_cy));
        atomicAdd(acc + 1, make_float4(g_cz, g_op * (1.0f - op), g_r, g_g));
        atomicAdd(&acc[2].x, g_b);
    }
}

} // namespace

cudaError_t gsx_launch_blend_backward(int width, int height, int grid_w, const uint2 *ranges,
                                      const uint32_t *bucket_offsets, const uint32_t *bucket_tile,
                                      uint64_t bucket_capacity, int n_tiles, const uint32_t *vals, const PrimRec *rec,
                                      const float4 *pix, const uint32_t *tile_max, const float4 *snap,
                                      const float *grad_rgb, float4 *grad_acc, int64_t n, cudaStream_t stream)
{
    (void)n;
    if(bucket_capacity == 0 || n_tiles <= 0) return cudaSuccess;
    const uint64_t blocks = (bucket_capacity + kWarps - 1) / kWarps;
    blend_backward_kernel<<<(unsigned)blocks, kThreads, 0, stream>>>(width, height, grid_w, n_tiles, ranges,
                                                                      bucket_offsets, bucket_tile, vals, rec, pix,
                                                                      tile_max, snap, grad_rgb, grad_acc);
    return cudaGetLastError();
}
