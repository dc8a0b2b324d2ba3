/*
 * Reverse-mode blend.  Gradient rules of fastgs/kernels_backward.cuh:484-730 (blend_backward_cu2,
 * after Taming-3DGS): every pixel of the tile starts each 32-instance bucket from the forward
 * snapshot (colour and transmittance before the bucket) and the composed image; fragments at or
 * beyond the pixel's last contributor are skipped; sigma is clamped at 0 (no 1/255 skip in the
 * backward), alpha at 0.999 with no opacity gradient when saturated, (1 - alpha) floored at 1e-4
 * in the division; buckets at or beyond the tile's maximum contributor are skipped.
 *
 * B200 organisation (a different work decomposition from the reference's warp-per-bucket):
 *   - a warp owns FOUR consecutive buckets (of the global bucket list, possibly from different
 *     tiles); each bucket is an 8-lane segment and each lane owns 4 consecutive instances, so a
 *     pixel's state walks 8 lanes instead of 32 (ramp of 7 steps instead of 31) and every state
 *     hand-off (8 shuffles) is amortised over 4 fragment evaluations per lane;
 *   - each segment prefetches its pixels' inputs (snapshot, composed colour, last contributor,
 *     upstream gradient) 32 pixels ahead into shared memory with cp.async, and its first lane
 *     feeds them into the chain, so segments from different tiles coexist in one warp;
 *   - per pixel, (colour still to come) . (upstream gradient) is carried as one scalar (each
 *     fragment lowers it by w * colour . gradient), so the hand-off is 6 values, not 8;
 *   - the factors that are constant per instance (conic on the mean terms, colour clamp mask,
 *     -1/2 on the conic terms, 1 - opacity) are applied once at the end, and each instance's
 *     accumulators are flushed with two 16-byte vector atomics plus one scalar atomic.
 */
#include "gsx_b200_kernels.cuh"


namespace {

constexpr int kWarps = 8;
constexpr int kThreads = 32 * kWarps;
constexpr int kPerLane = 4;

/* A pair of f32 in one 64-bit register: Blackwell's packed FP32 instructions (add/sub/mul/fma
 * .rn.f32x2) do both lanes of a pair in one issue, with the same IEEE rounding as two scalar ops. */
typedef unsigned long long f2;

__device__ __forceinline__ f2 pk(float lo, float hi)
{
    f2 r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void upk(f2 v, float &lo, float &hi) { asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v)); }
__device__ __forceinline__ f2 add2(f2 a, f2 b)
{
    f2 r;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
    return r;
}
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

/* two consecutive instances of a lane, field by field (lo = the earlier instance); conic terms
 * scaled by -log2(e), lop = log2(opacity), colours clamped at 0 */
struct FragPair {
    f2 mx, my, nhcx, ncy, nhcz, lop, r, g, b;
};

struct PixIn {
    float4 snap; /* forward colour and transmittance before the bucket */
    float4 img;  /* composed rgb, last-contributor bits */
    float4 grad; /* upstream dL/drgb (x, y, z) */
};

struct SegStage {
    PixIn buf[2][32];
    float4 pad;
};

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem)
{
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.ca.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}

__device__ __forceinline__ void cp_async4(void *smem, const void *gmem)
{
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(s), "l"(gmem) : "memory");
}

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }

/* 2^x and 1/x on the special-function unit (approximate: the backward is compared with tolerance) */
__device__ __forceinline__ float fast_exp2(float x)
{
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ float fast_rcp(float x)
{
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

template <int N>
__device__ __forceinline__ void cp_async_wait()
{
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ f2 abs2(f2 a) { return a & 0x7fffffff7fffffffull; }

/* Buckets grouped by the number of pixels they walk (bucket_active, from the TRAIN forward): a counting
 * sort, descending, of the buckets with at least one pixel to walk, so that the four buckets of a warp
 * walk about as many pixels each.  bucket_sort_state: [0, 257) histogram, [257, 514) cursors, [514]
 * number of listed buckets; zeroed before the histogram. */
constexpr int kCountBins = GSX_TILE_PIXELS + 1;

/* each CTA owns one contiguous chunk of the bucket list (neighbouring tiles stay together inside a
 * count) */
__device__ __forceinline__ void bucket_chunk(uint32_t n_buckets, uint32_t &b0, uint32_t &b1)
{
    const uint32_t chunk = (n_buckets + gridDim.x - 1) / gridDim.x;
    b0 = blockIdx.x * chunk;
    b1 = min(n_buckets, b0 + chunk);
}

__global__ void __launch_bounds__(256) bucket_hist_kernel(const uint32_t *__restrict__ bucket_offsets, int n_tiles,
                                                          const uint16_t *__restrict__ bucket_active,
                                                          uint32_t *__restrict__ state)
{
    __shared__ uint32_t h[kCountBins];
    for(int k = threadIdx.x; k < kCountBins; k += 256) h[k] = 0u;
    __syncthreads();
    uint32_t b0, b1;
    bucket_chunk(bucket_offsets[n_tiles - 1], b0, b1);
    for(uint32_t b = b0 + threadIdx.x; b < b1; b += 256u) atomicAdd(&h[bucket_active[b]], 1u);
    __syncthreads();
    for(int k = threadIdx.x; k < kCountBins; k += 256)
        if(h[k]) atomicAdd(&state[k], h[k]);
}

__global__ void __launch_bounds__(256) bucket_scatter_kernel(const uint32_t *__restrict__ bucket_offsets, int n_tiles,
                                                             const uint16_t *__restrict__ bucket_active,
                                                             uint32_t *__restrict__ state, uint32_t *__restrict__ order)
{
    /* start[c] = buckets with a count above c (descending order), for c = 1..256; thread t owns c = t + 1 */
    __shared__ uint32_t start[kCountBins];
    __shared__ uint32_t h[kCountBins];
    __shared__ uint32_t s_warp[8];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t v = state[threadIdx.x + 1];
    uint32_t incl = v;
#pragma unroll
    for(int d = 1; d < 32; d <<= 1) {
        const uint32_t x = __shfl_down_sync(0xffffffffu, incl, d);
        if(lane + d < 32) incl += x;
    }
    if(lane == 0) s_warp[warp] = incl;
    for(int k = threadIdx.x; k < kCountBins; k += 256) h[k] = 0u;
    __syncthreads();
    uint32_t above = incl - v;
    for(int w = warp + 1; w < 8; ++w) above += s_warp[w];
    if(blockIdx.x == 0 && threadIdx.x == 0) state[2 * kCountBins] = s_warp[0] + s_warp[1] + s_warp[2] + s_warp[3] +
                                                                   s_warp[4] + s_warp[5] + s_warp[6] + s_warp[7];
    /* this CTA's buckets per count (shared-memory atomics), then ONE global reservation per count */
    uint32_t b0, b1;
    bucket_chunk(bucket_offsets[n_tiles - 1], b0, b1);
    for(uint32_t b = b0 + threadIdx.x; b < b1; b += 256u) {
        const uint32_t c = bucket_active[b];
        if(c) atomicAdd(&h[c], 1u);
    }
    __syncthreads();
    {
        const int c = threadIdx.x + 1;
        start[c] = h[c] ? above + atomicAdd(&state[kCountBins + c], h[c]) : 0u;
        h[c] = 0u;
    }
    __syncthreads();
    for(uint32_t b = b0 + threadIdx.x; b < b1; b += 256u) {
        const uint32_t c = bucket_active[b];
        if(c) order[start[c] + atomicAdd(&h[c], 1u)] = b;
    }
}

/* kAbs: also accumulate sum over pixels of |d loss / d mean2d| per component (the absolute
 * screen-space gradient behind GSX's gs_absgrad_acc), into grad_acc[3i+2].yz */
template <bool kAbs>
__global__ void __launch_bounds__(kThreads, 2) blend_backward_kernel(
    int width, int height, int row0, int grid_w, const uint2 *__restrict__ ranges,
    const uint32_t *__restrict__ bucket_offsets, const uint32_t *__restrict__ bucket_tile,
    const uint32_t *__restrict__ bucket_order, const uint32_t *__restrict__ sort_state,
    const uint16_t *__restrict__ bucket_active, const uint8_t *__restrict__ tile_order,
    const uint32_t *__restrict__ vals, const PrimRec *__restrict__ rec, const float4 *__restrict__ pix,
    const float4 *__restrict__ snap, const float *__restrict__ grad_rgb, float4 *__restrict__ grad_acc)
{
    extern __shared__ __align__(16) unsigned char smem_raw[];
    /* per warp, per segment: 2 x 32 PixIn + one float4 of padding, so the four segment heads read
     * different banks */
    SegStage *s_in = reinterpret_cast<SegStage *>(smem_raw);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int sub = lane & 7;
    /* the warp's four buckets: consecutive entries of the bucket order (grouped by pixel count) */
    const uint32_t n_listed = sort_state[2 * kCountBins];
    const uint32_t slot = ((uint32_t)blockIdx.x * kWarps + warp) * 4u + (uint32_t)(lane >> 3);
    const bool seg_active = slot < n_listed;
    if(__ballot_sync(0xffffffffu, seg_active) == 0) return;
    uint32_t tile = 0, bucket = 0;
    int n_inst = 0, tb = 0, n_pix = 0;
    uint32_t inst0 = 0;
    if(seg_active) {
        bucket = bucket_order[slot];
        tile = bucket_tile[bucket];
        const uint2 range = ranges[tile];
        inst0 = range.x;
        n_inst = (int)(range.y - range.x);
        tb = (int)(bucket - (tile == 0 ? 0u : bucket_offsets[tile - 1]));
        n_pix = (int)bucket_active[bucket];
    }
    /* the pixels a segment walks: the first n_pix of its tile's order (last contributor beyond the
     * bucket's start); the warp runs until its longest segment is done */
    const int steps = __reduce_max_sync(0xffffffffu, (unsigned)n_pix) + 7;
    const uint8_t *order = tile_order + (size_t)tile * GSX_TILE_PIXELS;

    /* this lane's four instances, as two pairs */
    FragPair f[kPerLane / 2];
    uint32_t prim[kPerLane];
    int tpi[kPerLane];
    float fv[kPerLane][9];
#pragma unroll
    for(int k = 0; k < kPerLane; ++k) {
        tpi[k] = tb * 32 + sub * kPerLane + k;
        prim[k] = 0xffffffffu;
#pragma unroll
        for(int q = 0; q < 9; ++q) fv[k][q] = 0.0f;
        fv[k][5] = -126.0f; /* log2 opacity of an empty slot: alpha underflows to 0 */
        if(seg_active && tpi[k] < n_inst) {
            prim[k] = vals[inst0 + tpi[k]];
            const PrimRec r = rec[prim[k]];
            constexpr float kNL2E = -1.4426950408889634f;
            fv[k][0] = r.a.x - 0.5f;
            fv[k][1] = r.a.y - 0.5f;
            fv[k][2] = (0.5f * kNL2E) * r.a.z;
            fv[k][3] = kNL2E * r.a.w;
            fv[k][4] = (0.5f * kNL2E) * r.b.x;
            fv[k][5] = __log2f(r.b.y);
            fv[k][6] = fmaxf(r.b.z, 0.0f);
            fv[k][7] = fmaxf(r.b.w, 0.0f);
            fv[k][8] = fmaxf(r.c.x, 0.0f);
        } else {
            tpi[k] = 0x7fffffff; /* never below a last-contributor count */
        }
    }
#pragma unroll
    for(int j = 0; j < kPerLane / 2; ++j) {
        const float *lo = fv[2 * j], *hi = fv[2 * j + 1];
        f[j] = FragPair{ pk(lo[0], hi[0]), pk(lo[1], hi[1]), pk(lo[2], hi[2]), pk(lo[3], hi[3]), pk(lo[4], hi[4]),
                         pk(lo[5], hi[5]), pk(lo[6], hi[6]), pk(lo[7], hi[7]), pk(lo[8], hi[8]) };
    }
    /* accumulators per pair: mean (sum part * d), conic (sum part * d d^T), raw opacity, colour */
    f2 a_mx[kPerLane / 2], a_my[kPerLane / 2], a_cx[kPerLane / 2], a_cy[kPerLane / 2], a_cz[kPerLane / 2];
    f2 a_op[kPerLane / 2], a_r[kPerLane / 2], a_g[kPerLane / 2], a_b[kPerLane / 2];
    f2 a_ax[kPerLane / 2], a_ay[kPerLane / 2];
#pragma unroll
    for(int j = 0; j < kPerLane / 2; ++j) a_mx[j] = a_my[j] = a_cx[j] = a_cy[j] = a_cz[j] = a_op[j] = a_r[j] = a_g[j] = a_b[j] = 0ull;
#pragma unroll
    for(int j = 0; j < kPerLane / 2; ++j) a_ax[j] = a_ay[j] = 0ull;

    const int tx0 = (int)(tile % (uint32_t)grid_w) * GSX_TILE, ty0 = (int)(tile / (uint32_t)grid_w) * GSX_TILE;
    const size_t P = (size_t)width * (size_t)height;
    const float4 *bsnap = snap + (size_t)bucket * GSX_TILE_PIXELS;
    const int seg = lane >> 3;
    PixIn(*stage)[32] = s_in[warp * 4 + seg].buf;

    /* the 8 lanes of a segment prefetch the inputs of 32 list positions (snapshot, composed colour +
     * last contributor, upstream gradient, and the pixel's rank in the tile) into shared memory, one
     * batch ahead, with cp.async */
    /* each lane takes 4 consecutive list positions of a batch, whose ranks it reads as one 32-bit word
     * of the order one batch ahead of their prefetch (so the gather never waits on that read) */
    const uint32_t *order4 = reinterpret_cast<const uint32_t *>(order);
    uint32_t ranks = seg_active ? order4[sub] : 0u;
    auto prefetch = [&](int batch) {
        PixIn *dst = stage[batch & 1];
        const uint32_t mine = ranks;
        if(seg_active && (batch + 1) * 32 < n_pix) ranks = order4[(batch + 1) * 8 + sub];
#pragma unroll
        for(int q = 0; q < 4; ++q) {
            const int pl = sub * 4 + q, j = batch * 32 + pl;
            if(j < n_pix) {
                const int p = (int)((mine >> (8 * q)) & 255u);
                const int qx = tx0 + (p & (GSX_TILE - 1)), qy = ty0 + (p >> 4);
                const size_t idx = (size_t)qy * (size_t)width + (size_t)qx;
                cp_async16(&dst[pl].snap, bsnap + p);
                cp_async16(&dst[pl].img, pix + idx);
                cp_async4(&dst[pl].grad.x, grad_rgb + idx);
                cp_async4(&dst[pl].grad.y, grad_rgb + P + idx);
                cp_async4(&dst[pl].grad.z, grad_rgb + 2 * P + idx);
                dst[pl].grad.w = __int_as_float(p);
            }
        }
        cp_async_commit();
    };
    prefetch(0);

    /* per-pixel state travelling along the 8 lanes of a segment: upstream gradient, last
     * contributor, transmittance, and nadg = -(colour still to come) . (upstream gradient), kept as one
     * scalar because every fragment raises it by w * (colour . gradient) */
    float gr = 0.0f, gg = 0.0f, gb = 0.0f, nadg = 0.0f, T = 0.0f;
    int last = 0, rank = 0;
    for(int i = 0; i < steps; ++i) {
        if((i & 31) == 0 && i < steps - 7) {
            __syncwarp();
            if(i + 32 < steps - 7) {
                prefetch((i >> 5) + 1);
                cp_async_wait<1>();
            } else {
                cp_async_wait<0>();
            }
            __syncwarp();
        }
        gr = __shfl_up_sync(0xffffffffu, gr, 1);
        gg = __shfl_up_sync(0xffffffffu, gg, 1);
        gb = __shfl_up_sync(0xffffffffu, gb, 1);
        nadg = __shfl_up_sync(0xffffffffu, nadg, 1);
        T = __shfl_up_sync(0xffffffffu, T, 1);
        last = __shfl_up_sync(0xffffffffu, last, 1);
        rank = __shfl_up_sync(0xffffffffu, rank, 1);
        const int pos = i - sub; /* this lane's list position */
        const bool valid = pos >= 0 && pos < n_pix;
        if(sub == 0) {
            /* segment head: this bucket's inputs for list position i */
            last = 0;
            if(valid) {
                const PixIn &in = stage[(i >> 5) & 1][i & 31];
                const float4 sn = in.snap, img = in.img;
                gr = in.grad.x;
                gg = in.grad.y;
                gb = in.grad.z;
                rank = __float_as_int(in.grad.w);
                last = (int)__float_as_uint(img.w);
                nadg = (sn.x - img.x) * gr + (sn.y - img.y) * gg + (sn.z - img.z) * gb;
                T = sn.w;
            }
        }
        if(!valid) continue;
        const int qx = tx0 + (rank & (GSX_TILE - 1)), qy = ty0 + (rank >> 4);
        /* full-frame pixel coordinates (a band starts at row row0) */
        const f2 fx2 = pk((float)qx, (float)qx), fy2 = pk((float)(qy + row0), (float)(qy + row0));
        const f2 gr2 = pk(gr, gr), gg2 = pk(gg, gg), gb2 = pk(gb, gb);
        {
#pragma unroll
            for(int j = 0; j < kPerLane / 2; ++j) {
                /* independent per instance: geometry, alpha, colour . gradient (packed pairs).
                 * opacity * exp(-sigma) = 2^(-sigma log2 e + log2 opacity); sigma >= 0 for the
                 * positive-definite conic up to rounding, where the reference's clamp at 0 moves
                 * alpha by ~1e-7 relative, so it is not applied */
                const f2 dx = sub2(f[j].mx, fx2), dy = sub2(f[j].my, fy2);
                const f2 dxx = mul2(dx, dx), dxy = mul2(dx, dy), dyy = mul2(dy, dy);
                float e0, e1;
                upk(add2(fma2(f[j].nhcx, dxx, fma2(f[j].nhcz, dyy, mul2(f[j].ncy, dxy))), f[j].lop), e0, e1);
                const float ap0 = fast_exp2(e0), ap1 = fast_exp2(e1);
                const float al0 = tpi[2 * j] < last ? fminf(ap0, 0.999f) : 0.0f;
                const float al1 = tpi[2 * j + 1] < last ? fminf(ap1, 0.999f) : 0.0f;
                const f2 cdg = fma2(f[j].r, gr2, fma2(f[j].g, gg2, mul2(f[j].b, gb2)));
                float c0, c1;
                upk(cdg, c0, c1);
                float oma0, oma1;
                upk(sub2(pk(1.0f, 1.0f), pk(al0, al1)), oma0, oma1);
                /* sequential along the pixel's chain: transmittance and -(colour still to come).g;
                 * alpha <= 0.999 keeps 1 - alpha >= 1e-3, above the reference's 1e-4 floor */
                const float T0 = T, w0 = T * al0;
                const float nadg0 = fmaf(w0, c0, nadg);
                const float T1 = T0 * oma0, w1 = T1 * al1;
                nadg = fmaf(w1, c1, nadg0);
                T = T1 * oma1;
                const f2 dl = fma2(pk(nadg0, nadg), pk(fast_rcp(oma0), fast_rcp(oma1)), mul2(pk(T0, T1), cdg));
                const f2 part = mul2(pk(ap0 >= 0.999f ? 0.0f : al0, ap1 >= 0.999f ? 0.0f : al1), dl);
                const f2 w = pk(w0, w1);
                a_r[j] = fma2(w, gr2, a_r[j]);
                a_g[j] = fma2(w, gg2, a_g[j]);
                a_b[j] = fma2(w, gb2, a_b[j]);
                a_cx[j] = fma2(part, dxx, a_cx[j]);
                a_cy[j] = fma2(part, dxy, a_cy[j]);
                a_cz[j] = fma2(part, dyy, a_cz[j]);
                a_mx[j] = fma2(part, dx, a_mx[j]);
                a_my[j] = fma2(part, dy, a_my[j]);
                a_op[j] = add2(a_op[j], part);
                if constexpr(kAbs) {
                    /* |part (conic . d)| per component; the conic terms are held scaled by -log2 e
                     * (x: -log2e/2), so this is log2 e times the value, rescaled at the flush */
                    const f2 tx = fma2(f[j].nhcx, add2(dx, dx), mul2(f[j].ncy, dy));
                    const f2 ty = fma2(f[j].ncy, dx, mul2(f[j].nhcz, add2(dy, dy)));
                    const f2 ap = abs2(part);
                    a_ax[j] = fma2(ap, abs2(tx), a_ax[j]);
                    a_ay[j] = fma2(ap, abs2(ty), a_ay[j]);
                }
            }
        }
    }
    float u_mx[kPerLane], u_my[kPerLane], u_cx[kPerLane], u_cy[kPerLane], u_cz[kPerLane], u_op[kPerLane];
    float u_r[kPerLane], u_g[kPerLane], u_b[kPerLane], u_ax[kPerLane], u_ay[kPerLane];
#pragma unroll
    for(int j = 0; j < kPerLane / 2; ++j) {
        upk(a_mx[j], u_mx[2 * j], u_mx[2 * j + 1]);
        upk(a_my[j], u_my[2 * j], u_my[2 * j + 1]);
        upk(a_cx[j], u_cx[2 * j], u_cx[2 * j + 1]);
        upk(a_cy[j], u_cy[2 * j], u_cy[2 * j + 1]);
        upk(a_cz[j], u_cz[2 * j], u_cz[2 * j + 1]);
        upk(a_op[j], u_op[2 * j], u_op[2 * j + 1]);
        upk(a_r[j], u_r[2 * j], u_r[2 * j + 1]);
        upk(a_g[j], u_g[2 * j], u_g[2 * j + 1]);
        upk(a_b[j], u_b[2 * j], u_b[2 * j + 1]);
        upk(a_ax[j], u_ax[2 * j], u_ax[2 * j + 1]);
        upk(a_ay[j], u_ay[2 * j], u_ay[2 * j + 1]);
    }
#pragma unroll
    for(int k = 0; k < kPerLane; ++k) {
        if(prim[k] == 0xffffffffu) continue;
        const PrimRec r = rec[prim[k]];
        const float fr = r.b.z >= 0.0f ? 1.0f : 0.0f, fg = r.b.w >= 0.0f ? 1.0f : 0.0f, fb = r.c.x >= 0.0f ? 1.0f : 0.0f;
        float4 *acc = grad_acc + (size_t)prim[k] * 3;
        /* sum(part * (conic . d)) = conic . sum(part * d): the mean gradient is finished here */
        const float cx = r.a.z, cy = r.a.w, cz = r.b.x;
        const float gmx = fmaf(cx, u_mx[k], cy * u_my[k]), gmy = fmaf(cy, u_mx[k], cz * u_my[k]);
        atomicAdd(acc + 0, make_float4(-gmx, -gmy, -0.5f * u_cx[k], -u_cy[k]));
        atomicAdd(acc + 1, make_float4(-0.5f * u_cz[k], u_op[k] * (1.0f - r.b.y), u_r[k] * fr, u_g[k] * fg));
        if constexpr(kAbs) {
            constexpr float kLn2 = 0.6931471805599453f; /* 1 / log2(e) */
            atomicAdd(acc + 2, make_float4(u_b[k] * fb, kLn2 * u_ax[k], kLn2 * u_ay[k], 0.0f));
        } else {
            atomicAdd(&acc[2].x, u_b[k] * fb);
        }
    }
}

} // namespace

size_t gsx_bucket_sort_state_words() { return 2 * kCountBins + 1; }

cudaError_t gsx_launch_blend_backward(int width, int height, int row0, int grid_w, const uint2 *ranges,
                                      const uint32_t *bucket_offsets, const uint32_t *bucket_tile,
                                      uint64_t bucket_capacity, int n_tiles, const uint16_t *bucket_active,
                                      const uint8_t *tile_order, uint32_t *bucket_order, uint32_t *sort_state,
                                      const uint32_t *vals, const PrimRec *rec, const float4 *pix, const float4 *snap,
                                      const float *grad_rgb, float4 *grad_acc, bool abs_grad, cudaStream_t stream)
{
    if(bucket_capacity == 0 || n_tiles <= 0) return cudaSuccess;
    /* the bucket order: histogram of the pixel counts, then the scatter (both read the bucket count
     * on the device; grids sized by the capacity, grid-stride loops) */
    cudaError_t err = cudaMemsetAsync(sort_state, 0, sizeof(uint32_t) * gsx_bucket_sort_state_words(), stream);
    if(err != cudaSuccess) return err;
    uint64_t sblocks = (bucket_capacity + 255) / 256;
    if(sblocks > 148 * 8) sblocks = 148 * 8;
    bucket_hist_kernel<<<(unsigned)sblocks, 256, 0, stream>>>(bucket_offsets, n_tiles, bucket_active, sort_state);
    bucket_scatter_kernel<<<(unsigned)sblocks, 256, 0, stream>>>(bucket_offsets, n_tiles, bucket_active, sort_state,
                                                                 bucket_order);
    const uint64_t per_block = (uint64_t)kWarps * 4;
    const uint64_t blocks = (bucket_capacity + per_block - 1) / per_block;
    const size_t smem = sizeof(SegStage) * kWarps * 4;
    static bool attr_done[2][256];
    int dev = 0;
    err = cudaGetDevice(&dev);
    if(err != cudaSuccess) return err;
    auto kernel = abs_grad ? blend_backward_kernel<true> : blend_backward_kernel<false>;
    if(dev < 0 || dev >= 256 || !attr_done[abs_grad][dev]) {
        err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if(err != cudaSuccess) return err;
        if(dev >= 0 && dev < 256) attr_done[abs_grad][dev] = true;
    }
    kernel<<<(unsigned)blocks, kThreads, smem, stream>>>(width, height, row0, grid_w, ranges, bucket_offsets, bucket_tile,
                                                         bucket_order, sort_state, bucket_active, tile_order, vals, rec,
                                                         pix, snap, grad_rgb, grad_acc);
    return cudaGetLastError();
}
