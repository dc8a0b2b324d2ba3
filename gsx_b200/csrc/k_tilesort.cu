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
 *   1. the emission kernel counts the instances of every tile (atomic adds on GSX_TILE_SUBCOUNTERS
 *      counters per tile, chosen by instance index, to spread the atomics of crowded tiles);
 *   2. the tile scan (three short launches, one thread per tile) turns the counts into tile ranges
 *      [start, end), the inclusive bucket prefix, the instance total and the largest tile, the
 *      per-class tile lists, and every sub-counter into the absolute end of its slice of the range;
 *   3. bin_kernel moves every instance into a slot of its tile's range (taken by counting its
 *      sub-counter's end back down: arbitrary order) as a 64-bit sort key depth_bits << 32 | primitive;
 *      it reads the instance count from the device, so the host launches it before waiting for the
 *      forward's one read-back and the GPU bins while the host decides the sort;
 *   4. segsort_kernel (one CTA per tile) radix-sorts the tile's (depth, primitive) keys in shared
 *      memory and writes the final tile|depth keys and primitive values: the order is fully
 *      determined.  Five size classes (up to 512, 1024, 2048, 4096 and 16384 instances), each launched
 *      over its own compact tile list (so a CTA's work follows its tile's size) and on its own
 *      stream, so that the classes run side by side.
 * The host falls back to the global radix sort when the largest tile exceeds GSX_SEG_MAX instances.
 */
#include "gsx_b200_kernels.cuh"

namespace {

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

/* Tile scan, three launches (one thread per tile, 256 tiles per CTA):
 *   tile_reduce_kernel: per CTA, the sums of (instances, buckets, tiles per size class) and the
 *     largest tile -> block_aux[block * kAux + v] (the empty tiles form one more list, after the
 *     classes, so that the blend can visit the lists from the largest class down to the empty tiles);
 *   block_scan_aux_kernel (one CTA): exclusive scan of those over the CTAs; the class lists are laid
 *     end to end, class by class; words_out[0] = instance total, [1] = largest tile,
 *     [2 + c] = tiles of size class c;
 *   tile_write_kernel: ranges [start, end) (empty tiles [0, 0)), the inclusive bucket prefix, the
 *     class lists (each class in increasing tile order), and every sub-counter turned into the
 *     absolute end position of its slice of the tile's range. */
constexpr int kTileThreads = 256;
constexpr int kLists = kClasses + 1;  /* the size classes' tile lists, then the list of empty tiles */
constexpr int kAux = 2 + kLists + 1;   /* instances, buckets, tiles per list, max */

__device__ __forceinline__ uint32_t tile_total(const uint32_t *__restrict__ sub, int t, int n_tiles,
                                               uint32_t part[GSX_TILE_SUBCOUNTERS])
{
#pragma unroll
    for(int q = 0; q < GSX_TILE_SUBCOUNTERS; ++q) part[q] = sub[GSX_SUBCOUNTER(t, q, n_tiles)];
    uint32_t c = 0;
#pragma unroll
    for(int k = 0; k < GSX_TILE_SUBCOUNTERS; ++k) c += part[k];
    return c;
}

__global__ void __launch_bounds__(kTileThreads) tile_reduce_kernel(const uint32_t *__restrict__ sub, int n_tiles,
                                                                   uint32_t *__restrict__ block_aux)
{
    gsx_pdl_wait();
    gsx_pdl_trigger();
    __shared__ uint32_t s[kTileThreads / 32][kAux];
    const int t = blockIdx.x * kTileThreads + threadIdx.x;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t v[kAux];
#pragma unroll
    for(int q = 0; q < kAux; ++q) v[q] = 0u;
    if(t < n_tiles) {
        uint32_t part[GSX_TILE_SUBCOUNTERS];
        const uint32_t c = tile_total(sub, t, n_tiles, part);
        v[0] = c;
        v[1] = (c + 31u) / 32u;
        v[2 + (c ? size_class(c) : kClasses)] = 1u;
        v[kAux - 1] = c;
    }
#pragma unroll
    for(int q = 0; q < kAux; ++q) v[q] = q == kAux - 1 ? __reduce_max_sync(0xffffffffu, v[q]) : __reduce_add_sync(0xffffffffu, v[q]);
    if(lane == 0)
#pragma unroll
        for(int q = 0; q < kAux; ++q) s[warp][q] = v[q];
    __syncthreads();
    if(threadIdx.x < kAux) {
        uint32_t acc = 0;
        for(int w = 0; w < kTileThreads / 32; ++w)
            acc = threadIdx.x == kAux - 1 ? max(acc, s[w][threadIdx.x]) : acc + s[w][threadIdx.x];
        block_aux[(size_t)blockIdx.x * kAux + threadIdx.x] = acc;
    }
}

/* one CTA of 1024 threads, at most 1024 tile blocks (262144 tiles) */
__global__ void __launch_bounds__(1024) block_scan_aux_kernel(uint32_t *__restrict__ block_aux, int n_blocks,
                                                              uint32_t *__restrict__ words_out)
{
    gsx_pdl_wait();
    gsx_pdl_trigger();
    __shared__ uint32_t s_w[32][kAux];
    __shared__ uint32_t s_tot[kAux];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int b = threadIdx.x;
    uint32_t v[kAux], inc[kAux];
#pragma unroll
    for(int q = 0; q < kAux; ++q) inc[q] = v[q] = b < n_blocks ? block_aux[(size_t)b * kAux + q] : 0u;
#pragma unroll
    for(int d = 1; d < 32; d <<= 1)
#pragma unroll
        for(int q = 0; q < kAux - 1; ++q) {
            const uint32_t x = __shfl_up_sync(0xffffffffu, inc[q], d);
            if(lane >= d) inc[q] += x;
        }
    inc[kAux - 1] = __reduce_max_sync(0xffffffffu, v[kAux - 1]);
    if(lane == 31)
#pragma unroll
        for(int q = 0; q < kAux - 1; ++q) s_w[warp][q] = inc[q];
    if(lane == 0) s_w[warp][kAux - 1] = inc[kAux - 1];
    __syncthreads();
    uint32_t off[kAux];
#pragma unroll
    for(int q = 0; q < kAux; ++q) off[q] = 0u;
    for(int w = 0; w < 32; ++w)
#pragma unroll
        for(int q = 0; q < kAux - 1; ++q) off[q] += w < warp ? s_w[w][q] : 0u;
    if(threadIdx.x < kAux) {
        uint32_t acc = 0;
        for(int w = 0; w < 32; ++w) acc = threadIdx.x == kAux - 1 ? max(acc, s_w[w][threadIdx.x]) : acc + s_w[w][threadIdx.x];
        s_tot[threadIdx.x] = acc;
    }
    __syncthreads();
    if(b < n_blocks) {
        /* exclusive offsets; class c's list starts after the lists of the smaller classes */
        uint32_t cbase = 0;
#pragma unroll
        for(int q = 0; q < kAux - 1; ++q) {
            uint32_t e = off[q] + inc[q] - v[q];
            if(q >= 2) {
                e += cbase;
                cbase += s_tot[q];
            }
            block_aux[(size_t)b * kAux + q] = e;
        }
    }
    if(threadIdx.x == 0) {
        words_out[0] = s_tot[0];
        words_out[1] = s_tot[kAux - 1];
#pragma unroll
        for(int c = 0; c < kClasses; ++c) words_out[2 + c] = s_tot[2 + c];
    }
}

__global__ void __launch_bounds__(kTileThreads) tile_write_kernel(uint32_t *__restrict__ sub, int n_tiles,
                                                                  const uint32_t *__restrict__ block_aux,
                                                                  uint2 *__restrict__ ranges, uint32_t *__restrict__ bucket_offsets,
                                                                  uint32_t *__restrict__ class_tiles)
{
    gsx_pdl_wait();
    gsx_pdl_trigger();
    __shared__ uint32_t s[kTileThreads / 32][kAux - 1];
    const int t = blockIdx.x * kTileThreads + threadIdx.x;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const unsigned lt = (1u << lane) - 1u;
    uint32_t part[GSX_TILE_SUBCOUNTERS];
    uint32_t c = 0;
    if(t < n_tiles) c = tile_total(sub, t, n_tiles, part);
    const int cls = t < n_tiles ? (c ? size_class(c) : kClasses) : -1;
    /* in-warp exclusive prefixes: instances and buckets by shuffles, class memberships by ballots */
    uint32_t vi = c, vb = (c + 31u) / 32u;
    uint32_t ii = vi, ib = vb;
#pragma unroll
    for(int d = 1; d < 32; d <<= 1) {
        const uint32_t xi = __shfl_up_sync(0xffffffffu, ii, d), xb = __shfl_up_sync(0xffffffffu, ib, d);
        if(lane >= d) {
            ii += xi;
            ib += xb;
        }
    }
    uint32_t cpos = 0, cmask[kLists];
#pragma unroll
    for(int k = 0; k < kLists; ++k) {
        cmask[k] = __ballot_sync(0xffffffffu, cls == k);
        if(cls == k) cpos = (uint32_t)__popc(cmask[k] & lt);
    }
    if(lane == 31) {
        s[warp][0] = ii;
        s[warp][1] = ib;
    }
    if(lane < kLists) s[warp][2 + lane] = (uint32_t)__popc(cmask[lane]);
    __syncthreads();
    if(t >= n_tiles) return;
    uint32_t oi = block_aux[(size_t)blockIdx.x * kAux + 0], ob = block_aux[(size_t)blockIdx.x * kAux + 1];
    for(int w = 0; w < warp; ++w) {
        oi += s[w][0];
        ob += s[w][1];
    }
    const uint32_t start = oi + ii - vi;
    ranges[t] = c ? make_uint2(start, start + c) : make_uint2(0u, 0u);
    bucket_offsets[t] = ob + ib;
    uint32_t run = start;
#pragma unroll
    for(int q = 0; q < GSX_TILE_SUBCOUNTERS; ++q) {
        run += part[q];
        sub[GSX_SUBCOUNTER(t, q, n_tiles)] = run;
    }
    if(cls >= 0) {
        uint32_t pos = block_aux[(size_t)blockIdx.x * kAux + 2 + cls] + cpos;
        for(int w = 0; w < warp; ++w) pos += s[w][2 + cls];
        class_tiles[pos] = (uint32_t)t;
    }
}

/* each instance takes a slot of its tile by counting its sub-counter's end position back down (the
 * scan turned the counts into end positions) */
/* the instance count comes from the device (the tile scan's total), so the launch needs no host
 * round trip: the grid covers the emission capacity and the CTAs past the total exit at once */
__global__ void __launch_bounds__(kBinThreads) bin_kernel(const unsigned long long *__restrict__ keys,
                                                          const uint32_t *__restrict__ vals,
                                                          const uint32_t *__restrict__ d_total, uint64_t max_n,
                                                          int n_tiles, uint32_t *__restrict__ tile_end,
                                                          unsigned long long *__restrict__ sort_keys)
{
    const uint64_t i = (uint64_t)blockIdx.x * kBinThreads + threadIdx.x;
    const uint64_t n = *d_total;
    if(i >= n || i >= max_n) return;
    const unsigned long long k = keys[i];
    const uint32_t tile = (uint32_t)(k >> 32);
    const uint32_t slot = atomicSub(&tile_end[GSX_SUBCOUNTER(tile, i & (GSX_TILE_SUBCOUNTERS - 1), n_tiles)], 1u) - 1u;
    sort_keys[slot] = (k << 32) | (unsigned long long)vals[i];
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
        /* asynchronous 8-byte copies, all of the thread's keys in flight together (a load-then-store
         * loop waits out one memory round trip per item: 16 in a row for the largest class) */
        for(int e = threadIdx.x; e < n; e += kThreads_) {
            const unsigned dst = (unsigned)__cvta_generic_to_shared(s_key + e);
            asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(dst), "l"(sort_keys + r.x + e) : "memory");
        }
        asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
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

size_t gsx_tile_scan_aux_words(int n_tiles) { return (size_t)((n_tiles + kTileThreads - 1) / kTileThreads) * kAux; }

cudaError_t gsx_launch_tile_scan(uint32_t *tile_count, int n_tiles, uint2 *ranges, uint32_t *bucket_offsets,
                                 uint32_t *class_tiles, uint32_t *block_aux, uint32_t *words_out, cudaStream_t stream)
{
    if(n_tiles <= 0) return cudaSuccess;
    const int blocks = (n_tiles + kTileThreads - 1) / kTileThreads;
    if(blocks > 1024) return cudaErrorInvalidValue;
    cudaError_t e = gsx_launch_pdl(tile_reduce_kernel, dim3(blocks), dim3(kTileThreads), 0, stream, tile_count, n_tiles,
                                   block_aux);
    if(e == cudaSuccess)
        e = gsx_launch_pdl(block_scan_aux_kernel, dim3(1), dim3(1024), 0, stream, block_aux, blocks, words_out);
    if(e == cudaSuccess)
        e = gsx_launch_pdl(tile_write_kernel, dim3(blocks), dim3(kTileThreads), 0, stream, tile_count, n_tiles,
                           (const uint32_t *)block_aux, ranges, bucket_offsets, class_tiles);
    return e;
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

cudaError_t gsx_launch_tile_bin(const unsigned long long *keys, const uint32_t *vals, const uint32_t *d_total,
                                uint64_t max_n, int n_tiles, uint32_t *tile_end, unsigned long long *sort_keys,
                                cudaStream_t stream)
{
    if(max_n == 0 || n_tiles <= 0) return cudaSuccess;
    bin_kernel<<<(unsigned)((max_n + kBinThreads - 1) / kBinThreads), kBinThreads, 0, stream>>>(keys, vals, d_total, max_n,
                                                                                              n_tiles, tile_end, sort_keys);
    return cudaGetLastError();
}

cudaError_t gsx_launch_tile_sort(uint64_t n, int n_tiles, const uint2 *ranges, const uint32_t *class_tiles,
                                 const uint32_t *class_counts, const unsigned long long *sort_keys,
                                 unsigned long long *keys_out, uint32_t *vals_out, cudaStream_t stream,
                                 cudaStream_t const *side, cudaEvent_t const *ev)
{
    static_assert(kClassMax[kClasses - 1] == GSX_SEG_MAX, "the largest class covers up to GSX_SEG_MAX");
    static_assert(kClasses == GSX_SORT_CLASSES, "class count");
    if(n == 0 || n_tiles <= 0) return cudaSuccess;
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
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
