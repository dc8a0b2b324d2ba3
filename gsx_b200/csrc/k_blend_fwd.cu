/*
 * Front-to-back alpha blend of one 16x16 tile per CTA (256 threads, one pixel each), fused with
 * the background compose.
 *
 * Follows fastgs/kernels_forward.cuh:595-736 (blend_cu<false>) and render-kernels.cu:13-36:
 * alpha = min(opacity * exp(-sigma), 0.999), fragments with sigma < 0 or alpha < 1/255 skipped,
 * the pixel stops after the fragment that takes transmittance below 1e-4, a (colour,
 * transmittance) snapshot per pixel before every 32-instance bucket for the backward pass
 * (TRAIN forwards only, an INFERENCE forward has no backward; skipped for a pixel already finished,
 * whose backward never reaches the bucket), and out = colour + (1 - alpha) * background.  TRAIN
 * forwards also order each tile's pixels by last contributor and count, per bucket, the pixels the
 * backward has to walk.
 *
 * B200 organisation: each warp owns an 8x4 pixel block of the tile.  After a round of up to 512
 * instances is staged in shared memory (long rounds keep the warps, whose lists differ in length,
 * from waiting on each other at barriers), every warp builds the ordered list of staged instances
 * whose opacity-aware footprint can reach its block: the exact minimum of the instance's
 * quadratic form over the block's pixel-centre rectangle is compared with ln(255 * opacity) plus
 * a safety margin (the conic is bounded by the +0.3 dilation, so the float rounding of a pixel's
 * sigma is far below the margin).  Only listed instances are evaluated per pixel; an instance not
 * listed can never pass the per-pixel alpha test, so the result is unchanged.  Compiled with
 * -fmad=false; the per-pixel arithmetic uses explicit fmaf exactly as the oracle's
 * orc_blend_forward, so RGB is bit-identical to it.
 */
#include "gsx_b200_kernels.cuh"

#include <cuda_bf16.h>

namespace {

constexpr int kThreads = GSX_TILE_PIXELS;
constexpr int kWarps = kThreads / 32;
constexpr int kChunk = 512; /* instances staged per round: 2 per thread */
constexpr int kKeyMax = 511; /* last-contributor bucket keys above this share one bin */

struct FwdSmem {
    float4 a[kChunk]; /* mean2d.x, mean2d.y, conic.x / 2, conic.y */
    float4 b[kChunk]; /* conic.z / 2, opacity, clamped r, g */
    float4 c[kChunk]; /* clamped b, cull threshold, 1/conic.x, 1/conic.z */
    uint16_t list[kWarps][kChunk];
};

/* A pair of f32 in one 64-bit register for Blackwell's packed FP32 instructions (.rn.f32x2): one
 * issue does both halves, each rounded exactly as the scalar instruction, so results stay
 * bit-identical to the scalar (and oracle) arithmetic. */
typedef unsigned long long f2;

__device__ __forceinline__ f2 pk(float lo, float hi)
{
    f2 r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void upk(f2 v, float &lo, float &hi) { asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v)); }
__device__ __forceinline__ f2 sub2(f2 a, f2 b)
{
    f2 r;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ f2 mul2(f2 a, f2 b)
{
    f2 r;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
__device__ __forceinline__ f2 fma2(f2 a, f2 b, f2 c)
{
    f2 r;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
    return r;
}

/* gsx_expf_inrange on a pair, operation for operation (bit-identical results) for x in
 * [-87.33, 0]: with m = rint(-x log2 e) = -n (rint and the product are sign-symmetric),
 * r = fma(m, ln2_hi, x) = fma(-n, ln2_hi, x), the same degree-7 polynomial, times 2^n. */
__device__ __forceinline__ f2 expf_inrange2(f2 x)
{
    const f2 nlog2e = pk(-1.44269502162933349609f, -1.44269502162933349609f);
    float y0, y1;
    upk(mul2(x, nlog2e), y0, y1);
    const float m0 = rintf(y0), m1 = rintf(y1);
    const f2 m = pk(m0, m1);
    f2 r = fma2(m, pk(0.693145751953125f, 0.693145751953125f), x);
    r = fma2(m, pk(1.42860682030941723212e-06f, 1.42860682030941723212e-06f), r);
    f2 p = pk(1.98412698412698412698e-04f, 1.98412698412698412698e-04f);
    p = fma2(p, r, pk(1.38888888888888888889e-03f, 1.38888888888888888889e-03f));
    p = fma2(p, r, pk(8.33333333333333333333e-03f, 8.33333333333333333333e-03f));
    p = fma2(p, r, pk(4.16666666666666666667e-02f, 4.16666666666666666667e-02f));
    p = fma2(p, r, pk(1.66666666666666666667e-01f, 1.66666666666666666667e-01f));
    p = fma2(p, r, pk(0.5f, 0.5f));
    p = fma2(p, r, pk(1.0f, 1.0f));
    p = fma2(p, r, pk(1.0f, 1.0f));
    const f2 sc = pk(__uint_as_float((uint32_t)(127 - (int)m0) << 23), __uint_as_float((uint32_t)(127 - (int)m1) << 23));
    return mul2(p, sc);
}

/* minimum of q(d) = hcx dx^2 + cy dx dy + hcz dy^2, d = m - p, over p in [x0,x1] x [y0,y1] */
__device__ __forceinline__ float rect_min_power(float mx, float my, float hcx, float cy, float hcz, float icx, float icz,
                                                float x0, float x1, float y0, float y1)
{
    if(mx >= x0 && mx <= x1 && my >= y0 && my <= y1) return 0.0f;
    const float dy_lo = my - y1, dy_hi = my - y0, dx_lo = mx - x1, dx_hi = mx - x0;
    float best = 3.0e38f;
#pragma unroll
    for(int e = 0; e < 2; ++e) {
        const float dx = e == 0 ? dx_hi : dx_lo; /* edges x = x0, x = x1 */
        const float dy = fminf(fmaxf(-cy * dx * icz, dy_lo), dy_hi);
        best = fminf(best, hcx * dx * dx + cy * dx * dy + hcz * dy * dy);
    }
#pragma unroll
    for(int e = 0; e < 2; ++e) {
        const float dy = e == 0 ? dy_hi : dy_lo; /* edges y = y0, y = y1 */
        const float dx = fminf(fmaxf(-cy * dy * icx, dx_lo), dx_hi);
        best = fminf(best, hcx * dx * dx + cy * dx * dy + hcz * dy * dy);
    }
    return best;
}

template <bool kTrain, bool kBF16>
__global__ void __launch_bounds__(kThreads, kTrain ? 5 : 1) blend_forward_kernel(
    int width, int height, int row0, int grid_w, const uint2 *__restrict__ ranges, const uint32_t *__restrict__ bucket_offsets,
    const uint32_t *__restrict__ vals, const PrimRec *__restrict__ rec, float3 bg, void *__restrict__ out_rgb,
    float4 *__restrict__ pix, uint32_t *__restrict__ tile_max, float4 *__restrict__ snap, uint32_t *__restrict__ bucket_tile,
    const uint32_t *__restrict__ tile_lists, const uint32_t *__restrict__ class_sizes, uint8_t *__restrict__ tile_order,
    uint16_t *__restrict__ bucket_active)
{
    extern __shared__ __align__(16) unsigned char smem_raw[];
    FwdSmem &S = *reinterpret_cast<FwdSmem *>(smem_raw);
    __shared__ uint32_t s_max[kWarps];
    /* CTAs take tiles largest size class first (the tile scan's lists: classes 0..4 end to end, then
     * the empty tiles), so the long tiles start in the first wave and the short ones fill the tail */
    int tile = blockIdx.x;
    if(tile_lists != nullptr) {
        uint32_t cnt[GSX_SORT_CLASSES], off = 0;
#pragma unroll
        for(int c = 0; c < GSX_SORT_CLASSES; ++c) {
            cnt[c] = class_sizes[c];
            off += cnt[c];
        }
        uint32_t rem = blockIdx.x, at = off; /* at: start of the empty-tile list */
        bool found = false;
#pragma unroll
        for(int c = GSX_SORT_CLASSES - 1; c >= 0; --c) {
            at -= cnt[c];
            if(!found && rem < cnt[c]) {
                tile = (int)tile_lists[at + rem];
                found = true;
            }
            if(!found) rem -= cnt[c];
        }
        if(!found) tile = (int)tile_lists[off + rem];
    }
    const int tx = tile % grid_w, ty = tile / grid_w;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int lx = (warp & 1) * 8 + (lane & 7), ly = (warp >> 1) * 4 + (lane >> 3);
    const int prank = ly * GSX_TILE + lx; /* pixel rank in the tile: snapshot slot */
    const int px = tx * GSX_TILE + lx, py = ty * GSX_TILE + ly;
    const bool inside = px < width && py < height;
    /* arithmetic in full-frame pixel coordinates (a band starts at row row0) */
    const float pxf = (float)px + 0.5f, pyf = (float)(py + row0) + 0.5f;
    const float rx0 = (float)(tx * GSX_TILE + (warp & 1) * 8) + 0.5f, rx1 = rx0 + 7.0f;
    const float ry0 = (float)(ty * GSX_TILE + (warp >> 1) * 4 + row0) + 0.5f, ry1 = ry0 + 3.0f;
    const uint2 range = ranges[tile];
    uint32_t bucket = 0;
    if(kTrain) {
        bucket = tile == 0 ? 0u : bucket_offsets[tile - 1];
        for(uint32_t b = bucket + threadIdx.x; b < bucket_offsets[tile]; b += kThreads) bucket_tile[b] = (uint32_t)tile;
    }

    float cr = 0.0f, cg = 0.0f, cb = 0.0f, T = 1.0f;
    uint32_t ncon = 0;
    bool done = !inside;
    const int total = (int)(range.y - range.x);
    for(int start = 0; start < total; start += kChunk) {
        if(__syncthreads_count(done) == kThreads) break;
        const int batch = total - start < kChunk ? total - start : kChunk;
#pragma unroll
        for(int q = 0; q < kChunk / kThreads; ++q) {
            const int e = q * kThreads + (int)threadIdx.x;
            if(e < batch) {
                const PrimRec r = rec[vals[range.x + start + e]];
                const float thr = __logf(r.b.y * 255.0f);
                S.a[e] = make_float4(r.a.x, r.a.y, 0.5f * r.a.z, r.a.w);
                S.b[e] = make_float4(0.5f * r.b.x, r.b.y, fmaxf(r.b.z, 0.0f), fmaxf(r.b.w, 0.0f));
                S.c[e] = make_float4(fmaxf(r.c.x, 0.0f), thr + 0.05f + 1e-3f * fabsf(thr), 1.0f / r.a.z, 1.0f / r.b.x);
            }
        }
        __syncthreads();
        /* ordered list of the staged instances that can reach this warp's 8x4 block */
        int cnt = 0;
        if(__any_sync(0xffffffffu, !done)) {
#pragma unroll 1
            for(int k = 0; k * 32 < batch; ++k) {
                const int e = k * 32 + lane;
                bool pass = false;
                if(e < batch) {
                    const float4 a = S.a[e], b = S.b[e], c = S.c[e];
                    pass = rect_min_power(a.x, a.y, a.z, a.w, b.x, c.z, c.w, rx0, rx1, ry0, ry1) <= c.y;
                }
                const unsigned m = __ballot_sync(0xffffffffu, pass);
                if(pass) S.list[warp][cnt + __popc(m & ((1u << lane) - 1u))] = (uint16_t)e;
                cnt += __popc(m);
            }
        }
        __syncwarp();
        int li = 0;
        for(int kb = 0; kb * 32 < batch; ++kb) {
            if(kTrain) {
                /* a finished pixel (or one outside the image) has its last contributor before this
                 * bucket: the backward never reads its snapshot here */
                if(!done) snap[(size_t)bucket * kThreads + prank] = make_float4(cr, cg, cb, T);
                ++bucket;
            }
            const int bend = (kb + 1) * 32;
            /* two listed instances per iteration: geometry and exp on packed pairs, then the
             * blend applied in order (the second only if the first did not finish the pixel) */
            while(li < cnt) {
                const int e0 = S.list[warp][li];
                if(e0 >= bend) break;
                const bool has1 = li + 1 < cnt && S.list[warp][li + 1] < bend;
                const int e1 = has1 ? S.list[warp][li + 1] : e0;
                li += has1 ? 2 : 1;
                if(done) continue;
                const float4 a0 = S.a[e0], a1 = S.a[e1];
                const float4 b0 = S.b[e0], b1 = S.b[e1];
                const f2 dx = sub2(pk(a0.x, a1.x), pk(pxf, pxf)), dy = sub2(pk(a0.y, a1.y), pk(pyf, pyf));
                float s0, s1;
                upk(fma2(dx, fma2(pk(a0.z, a1.z), dx, mul2(pk(a0.w, a1.w), dy)), mul2(mul2(pk(b0.x, b1.x), dy), dy)), s0,
                    s1);
                const bool ok0 = !(s0 < 0.0f || s0 > 5.6f);
                const bool ok1 = has1 && !(s1 < 0.0f || s1 > 5.6f);
                if(!ok0 && !ok1) continue;
                float g0, g1;
                upk(expf_inrange2(pk(ok0 ? -s0 : 0.0f, ok1 ? -s1 : 0.0f)), g0, g1);
                float q0, q1;
                upk(mul2(pk(b0.y, b1.y), pk(g0, g1)), q0, q1);
                const float alpha0 = fminf(q0, 0.999f);
                if(ok0 && alpha0 >= 1.0f / 255.0f) {
                    const float w = T * alpha0;
                    cr = fmaf(w, b0.z, cr);
                    cg = fmaf(w, b0.w, cg);
                    cb = fmaf(w, S.c[e0].x, cb);
                    T = T * (1.0f - alpha0);
                    ncon = (uint32_t)(start + e0 + 1);
                    if(T < 1e-4f) done = true;
                }
                const float alpha1 = fminf(q1, 0.999f);
                if(ok1 && !done && alpha1 >= 1.0f / 255.0f) {
                    const float w = T * alpha1;
                    cr = fmaf(w, b1.z, cr);
                    cg = fmaf(w, b1.w, cg);
                    cb = fmaf(w, S.c[e1].x, cb);
                    T = T * (1.0f - alpha1);
                    ncon = (uint32_t)(start + e1 + 1);
                    if(T < 1e-4f) done = true;
                }
            }
        }
    }
    if(inside) {
        const size_t P = (size_t)width * (size_t)height;
        const size_t idx = (size_t)py * (size_t)width + (size_t)px;
        const float a = 1.0f - T;
        const float tr = 1.0f - a;
        const float o0 = cr + tr * bg.x, o1 = cg + tr * bg.y, o2 = cb + tr * bg.z;
        if(kBF16) {
            /* f32 accumulation, one rounding (to nearest even) at the store */
            __nv_bfloat16 *o = static_cast<__nv_bfloat16 *>(out_rgb);
            o[idx] = __float2bfloat16_rn(o0);
            o[P + idx] = __float2bfloat16_rn(o1);
            o[2 * P + idx] = __float2bfloat16_rn(o2);
        } else {
            float *o = static_cast<float *>(out_rgb);
            o[idx] = o0;
            o[P + idx] = o1;
            o[2 * P + idx] = o2;
        }
        pix[idx] = make_float4(o0, o1, o2, __uint_as_float(ncon));
    }
    uint32_t m = ncon;
#pragma unroll
    for(int d = 16; d > 0; d >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, d));
    if(lane == 0) s_max[warp] = m;
    __syncthreads();
    if(threadIdx.x == 0) {
        uint32_t mm = 0;
#pragma unroll
        for(int w = 0; w < kWarps; ++w) mm = max(mm, s_max[w]);
        tile_max[tile] = mm;
    }
    if(kTrain) {
        /* For the backward: the tile's pixels ordered by decreasing last-contributor bucket
         * (key = ceil(last / 32), capped at kKeyMax), and per bucket b of the tile the number of pixels
         * whose last contributor lies beyond the bucket's start (key > b): the pixels the backward
         * walks for that bucket are the first count(b) of the order.  A counting sort in shared
         * memory (the instance lists are dead by now); the order within one key is arbitrary. */
        static_assert((kKeyMax + 1) == 2 * kThreads, "two key bins per thread");
        uint32_t *s_cnt = reinterpret_cast<uint32_t *>(&S.list[0][0]); /* kKeyMax + 1 bins */
        uint32_t *s_warp = s_cnt + (kKeyMax + 1);                    /* kWarps partial sums */
        const uint32_t key = inside ? min((ncon + 31u) / 32u, (uint32_t)kKeyMax) : 0u;
        for(int k = threadIdx.x; k <= kKeyMax; k += kThreads) s_cnt[k] = 0u;
        __syncthreads();
        atomicAdd(&s_cnt[key], 1u);
        __syncthreads();
        /* descending exclusive scan: s_cnt[k] <- number of pixels with a key above k; thread t owns
         * bins 2t and 2t + 1 */
        const int k0 = 2 * (int)threadIdx.x, k1 = k0 + 1;
        const uint32_t h0 = s_cnt[k0], h1 = s_cnt[k1];
        /* suffix sums over threads: reverse the thread order into an inclusive prefix scan */
        uint32_t v = h0 + h1, incl = v;
#pragma unroll
        for(int d = 1; d < 32; d <<= 1) {
            const uint32_t x = __shfl_down_sync(0xffffffffu, incl, d);
            if(lane + d < 32) incl += x;
        }
        if(lane == 0) s_warp[warp] = incl;
        __syncthreads();
        uint32_t above = incl - v; /* bins beyond this thread's pair, within the warp */
        for(int w = warp + 1; w < kWarps; ++w) above += s_warp[w];
        __syncthreads();
        s_cnt[k0] = above + h1;
        s_cnt[k1] = above;
        __syncthreads();
        /* count(b) = pixels with key > min(b, kKeyMax - 1): conservative for the capped keys */
        const uint32_t b0 = tile == 0 ? 0u : bucket_offsets[tile - 1], nb = bucket_offsets[tile] - b0;
        for(uint32_t b = threadIdx.x; b < nb; b += kThreads)
            bucket_active[b0 + b] = (uint16_t)s_cnt[b < (uint32_t)kKeyMax ? b : (uint32_t)kKeyMax - 1u];
        __syncthreads();
        /* position: pixels with a larger key first, then a slot within the key */
        const uint32_t pos = atomicAdd(&s_cnt[key], 1u);
        tile_order[(size_t)tile * kThreads + pos] = (uint8_t)prank;
    }
}

} // namespace

cudaError_t gsx_launch_blend_forward(int width, int height, int row0, int grid_w, int n_tiles, const uint2 *ranges,
                                     const uint32_t *bucket_offsets, const uint32_t *vals, const PrimRec *rec,
                                     const float bg[3], void *out_rgb, bool out_bf16, float4 *pix, uint32_t *tile_max,
                                     float4 *snap, uint32_t *bucket_tile, bool train, const uint32_t *tile_lists,
                                     const uint32_t *class_sizes, uint8_t *tile_order, uint16_t *bucket_active,
                                     cudaStream_t stream)
{
    if(n_tiles <= 0) return cudaSuccess;
    static bool attr_done[4][256];
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if(err != cudaSuccess) return err;
    const int variant = (train ? 2 : 0) + (out_bf16 ? 1 : 0);
    auto kern = train ? (out_bf16 ? blend_forward_kernel<true, true> : blend_forward_kernel<true, false>)
                      : (out_bf16 ? blend_forward_kernel<false, true> : blend_forward_kernel<false, false>);
    if(dev < 0 || dev >= 256 || !attr_done[variant][dev]) {
        err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(FwdSmem));
        if(err != cudaSuccess) return err;
        if(dev >= 0 && dev < 256) attr_done[variant][dev] = true;
    }
    kern<<<(unsigned)n_tiles, kThreads, sizeof(FwdSmem), stream>>>(width, height, row0, grid_w, ranges, bucket_offsets, vals,
                                                                   rec, make_float3(bg[0], bg[1], bg[2]), out_rgb, pix,
                                                                   tile_max, snap, bucket_tile, tile_lists, class_sizes,
                                                                   tile_order, bucket_active);
    return cudaGetLastError();
}
