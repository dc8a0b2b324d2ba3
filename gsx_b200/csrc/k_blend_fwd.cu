/*
 * Front-to-back alpha blend of one 16x16 tile per CTA (256 threads, one pixel each), fused with
 * the background compose.
 *
 * Follows fastgs/kernels_forward.cuh:595-736 (blend_cu<false>) and render-kernels.cu:13-36:
 * alpha = min(opacity * exp(-sigma), 0.999), fragments with sigma < 0 or alpha < 1/255 skipped,
 * the pixel stops after the fragment that takes transmittance below 1e-4, a (colour,
 * transmittance) snapshot per pixel before every 32-instance bucket for the backward pass, and
 * out = colour + (1 - alpha) * background.
 *
 * B200 choices: batches of 256 instances are staged in shared memory as two float4 + one float
 * per instance (half-conic and clamped colour precomputed at staging, both exact transforms);
 * the whole-tile early exit is a __syncthreads_count vote; sigma > 5.6 is rejected before the
 * exponential (exp(-5.6) < 1/255, so such fragments can never pass the alpha test: the decision
 * is identical).  Compiled with -fmad=false; the fragment arithmetic uses explicit fmaf exactly
 * as the oracle's orc_blend_forward, so RGB is bit-identical to it.
 */
#include "gsx_b200_kernels.cuh"

namespace {

constexpr int kThreads = GSX_TILE_PIXELS;

__global__ void __launch_bounds__(kThreads) blend_forward_kernel(
    int width, int height, int grid_w, const uint2 *__restrict__ ranges, const uint32_t *__restrict__ bucket_offsets,
    const uint32_t *__restrict__ vals, const PrimRec *__restrict__ rec, float3 bg, float *__restrict__ out_rgb,
    float4 *__restrict__ pix, uint32_t *__restrict__ tile_max, float4 *__restrict__ snap)
{
    __shared__ float4 s_a[kThreads];
    __shared__ float4 s_b[kThreads];
    __shared__ float s_c[kThreads];
    __shared__ uint32_t s_max[kThreads / 32];
    const int tile = blockIdx.x;
    const int tx = tile % grid_w, ty = tile / grid_w;
    const int lx = threadIdx.x & (GSX_TILE - 1), ly = threadIdx.x >> 4;
    const int px = tx * GSX_TILE + lx, py = ty * GSX_TILE + ly;
    const bool inside = px < width && py < height;
    const float pxf = (float)px + 0.5f, pyf = (float)py + 0.5f;
    const uint2 range = ranges[tile];
    uint32_t bucket = tile == 0 ? 0u : bucket_offsets[tile - 1];

    float cr = 0.0f, cg = 0.0f, cb = 0.0f, T = 1.0f;
    uint32_t npos = 0, ncon = 0;
    bool done = !inside;
    const int total = (int)(range.y - range.x);
    for(int start = 0; start < total; start += kThreads) {
        if(__syncthreads_count(done) == kThreads) break;
        const int fetch = start + (int)threadIdx.x;
        if(fetch < total) {
            const PrimRec r = rec[vals[range.x + fetch]];
            s_a[threadIdx.x] = make_float4(r.a.x, r.a.y, 0.5f * r.a.z, r.a.w);
            s_b[threadIdx.x] = make_float4(0.5f * r.b.x, r.b.y, fmaxf(r.b.z, 0.0f), fmaxf(r.b.w, 0.0f));
            s_c[threadIdx.x] = fmaxf(r.c.x, 0.0f);
        }
        __syncthreads();
        const int batch = total - start < kThreads ? total - start : kThreads;
        int j = 0;
        for(; !done && j < batch; ++j) {
            if((j & 31) == 0) {
                snap[(size_t)bucket * kThreads + threadIdx.x] = make_float4(cr, cg, cb, T);
                ++bucket;
            }
            ++npos;
            const float4 a = s_a[j];
            const float dx = a.x - pxf, dy = a.y - pyf;
            const float4 b = s_b[j];
            const float sigma = fmaf(dx, fmaf(a.z, dx, a.w * dy), (b.x * dy) * dy);
            if(sigma < 0.0f || sigma > 5.6f) continue;
            const float g = gsx_expf_inrange(-sigma);
            const float alpha = fminf(b.y * g, 0.999f);
            if(alpha < 1.0f / 255.0f) continue;
            const float w = T * alpha;
            cr = fmaf(w, b.z, cr);
            cg = fmaf(w, b.w, cg);
            cb = fmaf(w, s_c[j], cb);
            T = T * (1.0f - alpha);
            ncon = npos;
            if(T < 1e-4f) done = true;
        }
        for(j = (j + 31) & ~31; j < batch; j += 32) {
            snap[(size_t)bucket * kThreads + threadIdx.x] = make_float4(cr, cg, cb, T);
            ++bucket;
        }
    }
    if(inside) {
        const size_t P = (size_t)width * (size_t)height;
        const size_t idx = (size_t)py * (size_t)width + (size_t)px;
        const float a = 1.0f - T;
        const float tr = 1.0f - a;
        const float o0 = cr + tr * bg.x, o1 = cg + tr * bg.y, o2 = cb + tr * bg.z;
        out_rgb[idx] = o0;
        out_rgb[P + idx] = o1;
        out_rgb[2 * P + idx] = o2;
        pix[idx] = make_float4(o0, o1, o2, __uint_as_float(ncon));
    }
    uint32_t m = ncon;
#pragma unroll
    for(int d = 16; d > 0; d >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, d));
    if((threadIdx.x & 31) == 0) s_max[threadIdx.x >> 5] = m;
    __syncthreads();
    if(threadIdx.x == 0) {
        uint32_t mm = 0;
#pragma unroll
        for(int w = 0; w < kThreads / 32; ++w) mm = max(mm, s_max[w]);
        tile_max[tile] = mm;
    }
}

} // namespace

cudaError_t gsx_launch_blend_forward(int width, int height, int grid_w, int n_tiles, const uint2 *ranges,
                                     const uint32_t *bucket_offsets, const uint32_t *vals, const PrimRec *rec,
                                     const float bg[3], float *out_rgb, float4 *pix, uint32_t *tile_max, float4 *snap,
                                     cudaStream_t stream)
{
    if(n_tiles <= 0) return cudaSuccess;
    blend_forward_kernel<<<(unsigned)n_tiles, kThreads, 0, stream>>>(
        width, height, grid_w, ranges, bucket_offsets, vals, rec, make_float3(bg[0], bg[1], bg[2]), out_rgb, pix,
        tile_max, snap);
    return cudaGetLastError();
}
