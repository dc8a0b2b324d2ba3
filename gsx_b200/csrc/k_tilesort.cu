/*
 * Tile binning + per-tile depth sort: the (tile, depth) instance order without a global radix sort.
 *
 * The reference sorts twice with CUB (fastgs/forward.cu:155-161, depth keys over the visible
 * primitives; :214-220, a stable 16-bit tile sort over the instances), then extracts per-tile ranges
 * (kernels_forward.cuh:558-577) and 32-instance bucket counts (:579-593, forward.cu:250-256).  The
 * result is: instances grouped by tile, each tile's instances by increasing depth; equal depths
 * (frequent: 32-bit depths of millions of Gaussians collide) in primitive order here.
 *
 * B200 organisation, exploiting that a tile holds few instances (hundreds to a few thousand):
 *   1. the emission kernel counts the instances of every tile (atomic adds);
 *   2. tile_scan_kernel (one CTA) turns the counts into tile ranges [start, end), the inclusive
 *      bucket prefix, the instance total and the largest tile;
 *   3. bin_kernel moves every instance into a slot of its tile's range (taken by counting the
 *      tile's count back down: arbitrary order) as a 64-bit sort key depth_bits << 32 | primitive;
 *   4. segsort_kernel (one CTA per tile) radix-sorts the tile's (depth, primitive) keys in shared
 *      memory and writes the final tile|depth keys and primitive values: the order is fully
 *      determined.  Five size classes (up to 512, 1024, 2048, 4096 and 16384 instances), each launched
 *      over its own compact tile list (so a CTA's work follows its tile's size) and on its own
 *      stream, so that the classes run side by side.
 * The host falls back to the global radix sort when the largest tile exceeds GSX_SEG_MAX instances.
 */
#include "gsx_b200_kernels.cuh"

namespace {

constexpr int kScanThreads = 1024;
constexpr int kBinThreads = 256;
/* per-tile sort size classes: (threads, items per thread), capacity = threads * items */
constexpr int kClasses = 5;
constexpr int kClassThreads[kClasses] = { 256, 256, 256, 512, 1024 };
constexpr int kClassItems[kClasses] = { 2, 4, 8, 8, 16 };
constexpr uint32_t kClassMax[kClasses] = { 512, 1024, 2048, 4096, 16384 };
static_assert(kClassMax[0] == 512 && kClassMax[1] == 1024 && kClassMax[2] == 2048 && kClassMax[3] == 4096,
              "size_class() spells these bounds out for device code");

__device__ __forceinline__ int size_class(uint32_t n)
{
    return n <= 512u ? 0 : n <= 1024u ? 1 : n <= 2048u ? 2 : n <= 4096u ? 3 : 4; /* kClassMax */
}

/* words_out[0] = instance total, words_out[1] = largest tile count, words_out[2 + c] = number of
 * non-empty tiles of size class c (kClassMax[c-1] < n <= kClassMax[c]); class_tiles[] lists the
 * tile ids class by class, each class in increasing tile order */
__global__ void __launch_bounds__(kScanThreads) tile_scan_kernel(const uint32_t *__restrict__ tile_count, int n_tiles,
                                                                 uint2 *__restrict__ ranges,
                                                                 uint32_t *__restrict__ bucket_offsets,
                                                                 uint32_t *__restrict__ class_tiles,
                                                                 uint32_t *__restrict__ words_out)
{
    constexpr int kV = 2 + kClasses; /* scanned values: instances, buckets, one count per class */
    __shared__ uint32_t s_v[kV][kScanThreads / 32], s_m[kScanThreads / 32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int per = (n_tiles + kScanThreads - 1) / kScanThreads;
    const int t0 = threadIdx.x * per;
    uint32_t loc[kV], lm = 0;
#pragma unroll
    for(int v = 0; v < kV; ++v) loc[v] = 0u;
    for(int t = t0; t < t0 + per && t < n_tiles; ++t) {
        const uint32_t c = tile_count[t];
        loc[0] += c;
        loc[1] += (c + 31u) / 32u;
        lm = max(lm, c);
        if(c) loc[2 + size_class(c)] += 1u;
    }
    uint32_t inc[kV];
#pragma unroll
    for(int v = 0; v < kV; ++v) inc[v] = loc[v];
    uint32_t im = lm;
#pragma unroll
    for(int d = 1; d < 32; d <<= 1) {
#pragma unroll
        for(int v = 0; v < kV; ++v) {
            const uint32_t x = __shfl_up_sync(0xffffffffu, inc[v], d);
            if(lane >= d) inc[v] += x;
        }
        im = max(im, __shfl_xor_sync(0xffffffffu, im, d));
    }
    if(lane == 31)
#pragma unroll
        for(int v = 0; v < kV; ++v) s_v[v][warp] = inc[v];
    if(lane == 0) s_m[warp] = im;
    __syncthreads();
    uint32_t run[kV], tot[kV], mm = 0;
#pragma unroll
    for(int v = 0; v < kV; ++v) {
        uint32_t o = 0, t = 0;
        for(int w = 0; w < kScanThreads / 32; ++w) {
            o += w < warp ? s_v[v][w] : 0u;
            t += s_v[v][w];
        }
        run[v] = o + inc[v] - loc[v];
        tot[v] = t;
    }
    for(int w = 0; w < kScanThreads / 32; ++w) mm = max(mm, s_m[w]);
    uint32_t cbase = 0;
#pragma unroll
    for(int c = 0; c < kClasses; ++c) {
        run[2 + c] += cbase; /* class c's list starts after the smaller classes' lists */
        cbase += tot[2 + c];
    }
    for(int t = t0; t < t0 + per && t < n_tiles; ++t) {
        const uint32_t c = tile_count[t];
        /* empty tiles keep [0, 0), as the reference's memset ranges */
        ranges[t] = c ? make_uint2(run[0], run[0] + c) : make_uint2(0u, 0u);
        run[0] += c;
        run[1] += (c + 31u) / 32u;
        bucket_offsets[t] = run[1];
        if(c) {
            const int k = size_class(c);
#pragma unroll
            for(int q = 0; q < kClasses; ++q)
                if(q == k) class_tiles[run[2 + q]++] = (uint32_t)t;
        }
    }
    if(threadIdx.x == 0) {
        words_out[0] = tot[0];
        words_out[1] = mm;
#pragma unroll
        for(int c = 0; c < kClasses; ++c) words_out[2 + c] = tot[2 + c];
    }
}

/* each instance takes a slot of its tile by counting the tile's instance count back down (the scan
 * has consumed the counts; they end at zero) */
__global__ void __launch_bounds__(kBinThreads) bin_kernel(const unsigned long long *__restrict__ keys,
                                                          const uint32_t *__restrict__ vals, uint64_t n,
                                                          const uint2 *__restrict__ ranges, uint32_t *__restrict__ tile_count,
                                                          unsigned long long *__restrict__ sort_keys)
{
    const uint64_t i = (uint64_t)blockIdx.x * kBinThreads + threadIdx.x;
    if(i >= n) return;
    const unsigned long long k = keys[i];
    const uint32_t tile = (uint32_t)(k >> 32);
    const uint32_t slot = atomicSub(&tile_count[tile], 1u) - 1u;
    sort_keys[ranges[tile].x + slot] = (k << 32) | (unsigned long long)vals[i];
}

/* One CTA per tile (blockIdx -> tile directly, or through `tile_list`) holding kMinN < n <=
 * kThreads_ * kItems instances: stable LSD radix sort of the 64-bit keys depth << 32 | primitive in
 * shared memory, 8-bit digits (warp-level multisplit in (item, lane) order, per-warp digit counters
 * scanned in warp order), passes whose digit is the same for every key skipped.  The first attempt
 * sorts the 4 depth bytes only; runs of equal depth (in arbitrary binning order) are then put in
 * primitive order in place, or, if one is longer than 32, the tile is reloaded and sorted on all 8
 * bytes, primitive bytes first. */
template <int kThreads_, int kItems>
__global__ void __launch_bounds__(kThreads_) segsort_kernel(const uint2 *__restrict__ ranges,
                                                            const uint32_t *__restrict__ tile_list,
                                                            const unsigned long long *__restrict__ sort_keys,
                                                            unsigned long long *__restrict__ keys_out,
                                                            uint32_t *__restrict__ vals_out)
{
    constexpr int kW = kThreads_ / 32;
    constexpr int kN = kThreads_ * kItems;
    extern __shared__ __align__(16) unsigned long long s_key[]; /* kN */
    uint32_t *s_wh = reinterpret_cast<uint32_t *>(s_key + kN);  /* kW * 256: per-warp digit counters, then their exclusive prefix */
    uint32_t *s_dbase = s_wh + kW * 256;                        /* 256: exclusive prefix of the block's digit counts */
    uint32_t *s_misc = s_dbase + 256;                           /* 32: per-warp digit totals; [8] = pass is the identity */
    const int tile = (int)tile_list[blockIdx.x];
    const uint2 r = ranges[tile];
    const int n = (int)(r.y - r.x);
    if(n <= 0 || n > kN) return;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const unsigned lt = (1u << lane) - 1u;
    for(int attempt = 0; attempt < 2; ++attempt) {
        /* element e of the current order sits at s_key[e]; thread (warp, lane) owns
         * e = warp * 32 * kItems + it * 32 + lane */
        for(int e = threadIdx.x; e < n; e += kThreads_) s_key[e] = sort_keys[r.x + e];
        if(threadIdx.x == 0) s_misc[8] = 0u;
        __syncthreads();
        for(int shift = attempt == 0 ? 32 : 0; shift < 64; shift += 8) {
            unsigned long long k[kItems];
            uint32_t dg[kItems], rank[kItems];
#pragma unroll
            for(int it = 0; it < kItems; ++it) {
                const int e = warp * 32 * kItems + it * 32 + lane;
                k[it] = e < n ? s_key[e] : 0ull;
                dg[it] = e < n ? (uint32_t)(k[it] >> shift) & 255u : 256u;
            }
            for(int j = threadIdx.x; j < kW * 256; j += kThreads_) s_wh[j] = 0u;
            __syncthreads();
            uint32_t *wh = s_wh + warp * 256;
#pragma unroll
            for(int it = 0; it < kItems; ++it) {
                const unsigned peers = __match_any_sync(0xffffffffu, dg[it]);
                const int leader = __ffs(peers) - 1;
                uint32_t base = 0;
                if(lane == leader && dg[it] < 256u) {
                    base = wh[dg[it]];
                    wh[dg[it]] = base + (uint32_t)__popc(peers);
                }
                rank[it] = __shfl_sync(0xffffffffu, base, leader) + (uint32_t)__popc(peers & lt);
            }
            __syncthreads();
            /* digit d (thread d < 256): exclusive over warps (in place) and block count, then an
             * exclusive scan over digits */
            uint32_t cnt = 0;
            if(threadIdx.x < 256) {
                for(int w = 0; w < kW; ++w) {
                    const uint32_t c = s_wh[w * 256 + threadIdx.x];
                    s_wh[w * 256 + threadIdx.x] = cnt;
                    cnt += c;
                }
                if(cnt == (uint32_t)n) s_misc[8] = 1u; /* every key has this digit */
            }
            uint32_t incl = cnt;
#pragma unroll
            for(int d = 1; d < 32; d <<= 1) {
                const uint32_t x = __shfl_up_sync(0xffffffffu, incl, d);
                if(lane >= d) incl += x;
            }
            if(threadIdx.x < 256 && lane == 31) s_misc[warp] = incl;
            __syncthreads();
            const bool identity = s_misc[8] != 0u;
            if(threadIdx.x < 256) {
                uint32_t wo = 0;
                for(int w = 0; w < warp; ++w) wo += s_misc[w];
                s_dbase[threadIdx.x] = wo + incl - cnt;
            }
            __syncthreads();
            if(!identity) {
#pragma unroll
                for(int it = 0; it < kItems; ++it)
                    if(dg[it] < 256u) s_key[s_dbase[dg[it]] + s_wh[warp * 256 + dg[it]] + rank[it]] = k[it];
            }
            if(threadIdx.x == 0) s_misc[8] = 0u;
            __syncthreads();
        }
        if(attempt == 1) break;
        /* runs of equal depth are still in the arbitrary binning order: the thread at a run's start
         * orders a run of up to 32 keys in place (insertion); any longer run sends the whole tile
         * through the full 8-byte sort instead */
        int long_run = 0;
        for(int e = threadIdx.x; e + 1 < n; e += kThreads_) {
            const uint32_t d = (uint32_t)(s_key[e] >> 32);
            if((e == 0 || (uint32_t)(s_key[e - 1] >> 32) != d) && (uint32_t)(s_key[e + 1] >> 32) == d) {
                int end = e + 2;
                while(end < n && end - e <= 32 && (uint32_t)(s_key[end] >> 32) == d) ++end;
                if(end - e > 32) {
                    long_run = 1;
                    continue;
                }
                for(int a = e + 1; a < end; ++a) {
                    const unsigned long long v = s_key[a];
                    int b = a - 1;
                    while(b >= e && s_key[b] > v) {
                        s_key[b + 1] = s_key[b];
                        --b;
                    }
                    s_key[b + 1] = v;
                }
            }
        }
        if(!__syncthreads_or(long_run)) break;
    }
    const unsigned long long thi = (unsigned long long)tile << 32;
    for(int e = threadIdx.x; e < n; e += kThreads_) {
        const unsigned long long s = s_key[e];
        keys_out[r.x + e] = thi | (s >> 32);
        vals_out[r.x + e] = (uint32_t)s;
    }
}

constexpr size_t segsort_smem(int threads, int items) { return (size_t)8 * threads * items + (size_t)4 * ((threads / 32) * 256 + 256 + 32); }


} // namespace

cudaError_t gsx_launch_tile_scan(const uint32_t *tile_count, int n_tiles, uint2 *ranges, uint32_t *bucket_offsets,
                                 uint32_t *class_tiles, uint32_t *words_out, cudaStream_t stream)
{
    if(n_tiles <= 0) return cudaSuccess;
    tile_scan_kernel<<<1, kScanThreads, 0, stream>>>(tile_count, n_tiles, ranges, bucket_offsets, class_tiles, words_out);
    return cudaGetLastError();
}

int gsx_tile_sort_classes() { return kClasses; }

namespace {

template <int C>
cudaError_t launch_class(const uint2 *ranges, const uint32_t *list, uint32_t count, const unsigned long long *sort_keys,
                         unsigned long long *keys_out, uint32_t *vals_out, int dev, cudaStream_t stream)
{
    static bool attr_done[256];
    constexpr int T = kClassThreads[C], I = kClassItems[C];
    static_assert((uint32_t)(T * I) == kClassMax[C], "class capacity");
    auto kern = segsort_kernel<T, I>;
    const size_t smem = segsort_smem(T, I);
    if(count == 0) return cudaSuccess;
    if(smem > 48 * 1024 && (dev < 0 || dev >= 256 || !attr_done[dev])) {
        const cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if(err != cudaSuccess) return err;
        if(dev >= 0 && dev < 256) attr_done[dev] = true;
    }
    kern<<<count, T, smem, stream>>>(ranges, list, sort_keys, keys_out, vals_out);
    return cudaGetLastError();
}

} // namespace

cudaError_t gsx_launch_tile_sort(const unsigned long long *keys, const uint32_t *vals, uint64_t n, int n_tiles,
                                 const uint2 *ranges, uint32_t *tile_count, const uint32_t *class_tiles,
                                 const uint32_t *class_counts, unsigned long long *sort_keys, unsigned long long *keys_out,
                                 uint32_t *vals_out, cudaStream_t stream, cudaStream_t const *side, cudaEvent_t const *ev)
{
    static_assert(kClassMax[kClasses - 1] == GSX_SEG_MAX, "the largest class covers up to GSX_SEG_MAX");
    static_assert(kClasses == GSX_SORT_CLASSES, "class count");
    if(n == 0 || n_tiles <= 0) return cudaSuccess;
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if(err != cudaSuccess) return err;
    bin_kernel<<<(unsigned)((n + kBinThreads - 1) / kBinThreads), kBinThreads, 0, stream>>>(keys, vals, n, ranges,
                                                                                          tile_count, sort_keys);
    err = cudaGetLastError();
    if(err != cudaSuccess) return err;
    /* fork: class c > 0 runs on side[c - 1] after the binning, class 0 on the caller's stream; join */
    err = cudaEventRecord(ev[0], stream);
    if(err != cudaSuccess) return err;
    cudaError_t (*launchers[kClasses])(const uint2 *, const uint32_t *, uint32_t, const unsigned long long *,
                                       unsigned long long *, uint32_t *, int, cudaStream_t) = {
        launch_class<0>, launch_class<1>, launch_class<2>, launch_class<3>, launch_class<4> };
    const uint32_t *list = class_tiles;
    for(int c = 0; c < kClasses; ++c) {
        cudaStream_t st = stream;
        if(c > 0 && class_counts[c] > 0) {
            st = side[c - 1];
            err = cudaStreamWaitEvent(st, ev[0], 0);
            if(err != cudaSuccess) return err;
        }
        err = launchers[c](ranges, list, class_counts[c], sort_keys, keys_out, vals_out, dev, st);
        if(err != cudaSuccess) return err;
        if(c > 0 && class_counts[c] > 0) {
            err = cudaEventRecord(ev[c], st);
            if(err == cudaSuccess) err = cudaStreamWaitEvent(stream, ev[c], 0);
            if(err != cudaSuccess) return err;
        }
        list += class_counts[c];
    }
    return cudaSuccess;
}
