/*
 * Emission of one 64-bit key (tile_id << 32 | depth bits) and one 32-bit primitive index per
 * (visible Gaussian, touched tile), in primitive order and, per primitive, row-major tile order.
 *
 * Follows fastgs/kernels_forward.cuh:453-556 (create_instances_cu) for which tiles are emitted
 * (the same exact overlap test as the preprocess count), but writes the combined tile|depth key
 * so that one stable LSD radix sort yields the reference's (tile, then depth) order
 * (forward.cu:155-161 depth sort followed by the stable 16-bit tile sort at :214-220).
 * With tile counters it also counts the instances of every tile (for the tile binning of
 * k_tilesort.cu) on GSX_TILE_SUBCOUNTERS counters per tile, picked by the instance's index, so that
 * the atomics of a crowded tile spread over several addresses; without them it counts, per 8-bit
 * digit position of the emitted keys, a 256-bin histogram from which the host plans the global
 * radix-sort passes (passes whose digit is the same for every key are skipped).
 * Tile rows are band-relative; the overlap tests use full-frame tile rows (trow0 + row).
 * Compiled with -fmad=false (bit-identical overlap decisions with the preprocess and the oracle).
 */
#include "gsx_b200_kernels.cuh"

namespace {

constexpr int kThreads = 256;
constexpr int kCoopLanes = 6; /* up to this many small-rectangle lanes, the warp emits them together */

__global__ void __launch_bounds__(kThreads, 5) emit_kernel(int64_t n, const PrimRec *__restrict__ rec,
                                                        const uint32_t *__restrict__ counts,
                                                        const uint32_t *__restrict__ tile_masks,
                                                        const uint32_t *__restrict__ block_offsets,
                                                        uint32_t *__restrict__ offsets, unsigned grid_w, unsigned trow0, unsigned n_tiles,
                                                        unsigned long long *__restrict__ keys, uint32_t *__restrict__ vals,
                                                        uint64_t capacity, uint32_t *__restrict__ flags,
                                                        uint32_t *__restrict__ hist, int n_digits,
                                                        uint32_t *__restrict__ tile_count)
{
    gsx_pdl_wait();
    gsx_pdl_trigger();
    __shared__ uint32_t s_warp[kThreads / 32];
    __shared__ uint32_t s_hist[8][256];
    const int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x;
    /* every load that does not depend on another is issued here, together: the block's offset pair,
     * the Gaussian's tile count and its overlap mask.  Only the record load below waits on them, so a
     * block costs two memory round trips instead of three (with 5 CTAs per SM: band emission 0.193 ->
     * 0.163 ms, config-3 emission 0.090 -> 0.078 ms) */
    const uint32_t boff0 = block_offsets[blockIdx.x], boff1 = block_offsets[blockIdx.x + 1];
    uint32_t cnt = i < n ? counts[i] : 0u;
    const uint32_t mask_in = i < n ? tile_masks[i] : 0u;
    if(n_digits == 0 && boff1 == boff0) {
        /* no instance in this block (every Gaussian culled): offsets only */
        if(i < n) offsets[i] = boff0;
        if(i == n - 1) offsets[n] = boff0;
        return;
    }
    for(int j = threadIdx.x; j < n_digits * 256; j += kThreads) (&s_hist[0][0])[j] = 0u;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    /* exclusive position = block offset + in-block exclusive scan of the counts */
    uint32_t incl = cnt;
#pragma unroll
    for(int d = 1; d < 32; d <<= 1) {
        const uint32_t t = __shfl_up_sync(0xffffffffu, incl, d);
        if(lane >= d) incl += t;
    }
    if(lane == 31) s_warp[warp] = incl;
    __syncthreads();
    uint32_t woff = 0;
#pragma unroll
    for(int k = 0; k < kThreads / 32; ++k) woff += k < warp ? s_warp[k] : 0u;
    const uint32_t start = boff0 + woff + incl - cnt;
    if(i < n) offsets[i] = start;
    if(i == n - 1) offsets[n] = start + cnt;
    const bool warp_busy = __ballot_sync(0xffffffffu, cnt != 0) != 0;
    if(warp_busy) {
    float msx = 0.0f, msy = 0.0f, cx = 0.0f, cy = 0.0f, cz = 0.0f, pt = 0.0f;
    unsigned bx0 = 0, bw = 0, by0 = 0, tmax = 0;
    unsigned long long dbits = 0;
    if(cnt != 0) {
        const PrimRec r = rec[i];
        msx = r.a.x - 0.5f;
        msy = r.a.y - 0.5f;
        cx = r.a.z;
        cy = r.a.w;
        cz = r.b.x;
        pt = gsx_logf(r.b.y * 255.0f);
        dbits = (unsigned long long)__float_as_uint(r.c.y);
        const unsigned bx = __float_as_uint(r.c.z), by = __float_as_uint(r.c.w);
        bx0 = bx & 0xffffu;
        bw = (bx >> 16) - bx0;
        by0 = by & 0xffffu;
        tmax = bw * ((by >> 16) - by0);
        if((uint64_t)start + cnt > capacity) {
            atomicOr(flags, GSX_FLAG_INSTANCE_OVERFLOW);
            cnt = 0;
            tmax = 0;
        }
    }
    uint32_t wpos = start;
    const unsigned lt_mask = (1u << lane) - 1u;
    /* rectangles of up to 32 tiles: the preprocess already ran the exact overlap test and left the
     * overlap mask.  A warp with few such lanes (a band of a large frame: most Gaussians culled) emits
     * one Gaussian at a time, lane k taking tile k of its rectangle, instead of walking tiles lane by
     * lane with the rest of the warp idle */
    {
        const unsigned m_own = tmax > 0 && tmax <= 32u ? mask_in : 0u;
        unsigned small = __ballot_sync(0xffffffffu, tmax > 0 && tmax <= 32u);
        if(__popc(small) > kCoopLanes) {
            /* many such lanes: each lane walks its own mask (fewer instructions than the broadcasts) */
            unsigned m = m_own;
            while(m) {
                const unsigned k = (unsigned)__ffs(m) - 1u;
                m &= m - 1u;
                const unsigned tx = bx0 + k % bw, ty = by0 + k / bw;
                const unsigned t = ty * grid_w + tx;
                const unsigned long long key = ((unsigned long long)t << 32) | dbits;
                keys[wpos] = key;
                vals[wpos] = (uint32_t)i;
                if(tile_count) atomicAdd(&tile_count[GSX_SUBCOUNTER(t, wpos & (GSX_TILE_SUBCOUNTERS - 1), n_tiles)], 1u);
                ++wpos;
                for(int q = 0; q < n_digits; ++q) atomicAdd(&s_hist[q][(uint32_t)(key >> (8 * q)) & 0xffu], 1u);
            }
            small = 0u;
        }
        while(small) {
            const int L = __ffs(small) - 1;
            small &= small - 1u;
            const unsigned m = __shfl_sync(0xffffffffu, m_own, L);
            const unsigned lbx0 = __shfl_sync(0xffffffffu, bx0, L), lbw = __shfl_sync(0xffffffffu, bw, L);
            const unsigned lby0 = __shfl_sync(0xffffffffu, by0, L);
            const unsigned long long ldb = __shfl_sync(0xffffffffu, dbits, L);
            const uint32_t lpos = __shfl_sync(0xffffffffu, wpos, L);
            const uint32_t lidx = (uint32_t)__shfl_sync(0xffffffffu, (long long)i, L);
            if((m >> lane) & 1u) {
                const unsigned k = (unsigned)lane;
                const unsigned tx = lbx0 + k % lbw, ty = lby0 + k / lbw;
                const unsigned t = ty * grid_w + tx;
                const uint32_t p = lpos + (uint32_t)__popc(m & lt_mask);
                const unsigned long long key = ((unsigned long long)t << 32) | ldb;
                keys[p] = key;
                vals[p] = lidx;
                if(tile_count) atomicAdd(&tile_count[GSX_SUBCOUNTER(t, p & (GSX_TILE_SUBCOUNTERS - 1), n_tiles)], 1u);
                for(int q = 0; q < n_digits; ++q) atomicAdd(&s_hist[q][(uint32_t)(key >> (8 * q)) & 0xffu], 1u);
            }
        }
        if(tmax <= 32u) tmax = 0; /* done: neither the sequential nor the cooperative pass below runs */
    }
    const unsigned nseq = tmax < GSX_SEQ_TILES ? tmax : GSX_SEQ_TILES;
    for(unsigned k = 0; k < nseq; ++k) {
        const unsigned tx = bx0 + k % bw, ty = by0 + k / bw;
        if(gsx_tile_contributes(msx, msy, cx, cy, cz, tx, trow0 + ty, pt)) {
            const unsigned t = ty * grid_w + tx;
            const unsigned long long key = ((unsigned long long)t << 32) | dbits;
            keys[wpos] = key;
            vals[wpos] = (uint32_t)i;
            if(tile_count) atomicAdd(&tile_count[GSX_SUBCOUNTER(t, wpos & (GSX_TILE_SUBCOUNTERS - 1), n_tiles)], 1u);
            ++wpos;
            for(int p = 0; p < n_digits; ++p) atomicAdd(&s_hist[p][(uint32_t)(key >> (8 * p)) & 0xffu], 1u);
        }
    }
    unsigned coop = __ballot_sync(0xffffffffu, tmax > GSX_SEQ_TILES);
    while(coop) {
        const int L = __ffs(coop) - 1;
        coop &= coop - 1u;
        const unsigned lbx0 = __shfl_sync(0xffffffffu, bx0, L), lbw = __shfl_sync(0xffffffffu, bw, L);
        const unsigned lby0 = __shfl_sync(0xffffffffu, by0, L), ltmax = __shfl_sync(0xffffffffu, tmax, L);
        const float lmx = __shfl_sync(0xffffffffu, msx, L), lmy = __shfl_sync(0xffffffffu, msy, L);
        const float lcx = __shfl_sync(0xffffffffu, cx, L), lcy = __shfl_sync(0xffffffffu, cy, L);
        const float lcz = __shfl_sync(0xffffffffu, cz, L), lpt = __shfl_sync(0xffffffffu, pt, L);
        const unsigned long long ldb = __shfl_sync(0xffffffffu, dbits, L);
        uint32_t lpos = __shfl_sync(0xffffffffu, wpos, L);
        const uint32_t lidx = (uint32_t)__shfl_sync(0xffffffffu, (long long)i, L);
        for(unsigned base = GSX_SEQ_TILES; base < ltmax; base += 32u) {
            const unsigned k = base + (unsigned)lane;
            const unsigned tx = lbx0 + k % lbw, ty = lby0 + k / lbw;
            const bool c = k < ltmax && gsx_tile_contributes(lmx, lmy, lcx, lcy, lcz, tx, trow0 + ty, lpt);
            const unsigned ballot = __ballot_sync(0xffffffffu, c);
            if(c) {
                const uint32_t p = lpos + (uint32_t)__popc(ballot & lt_mask);
                const unsigned t = ty * grid_w + tx;
                const unsigned long long key = ((unsigned long long)t << 32) | ldb;
                keys[p] = key;
                vals[p] = lidx;
                if(tile_count) atomicAdd(&tile_count[GSX_SUBCOUNTER(t, p & (GSX_TILE_SUBCOUNTERS - 1), n_tiles)], 1u);
                for(int q = 0; q < n_digits; ++q) atomicAdd(&s_hist[q][(uint32_t)(key >> (8 * q)) & 0xffu], 1u);
            }
            lpos += (uint32_t)__popc(ballot);
        }
    }
    }
    /* per-digit-position histograms of the emitted keys, for the radix sort's pass planning */
    __syncthreads();
    for(int j = threadIdx.x; j < n_digits * 256; j += kThreads) {
        const uint32_t v = (&s_hist[0][0])[j];
        if(v) atomicAdd(&hist[j], v);
    }
}

} // namespace

cudaError_t gsx_launch_emit(int64_t n, const PrimRec *rec, const uint32_t *counts, const uint32_t *tile_masks,
                            const uint32_t *block_offsets,
                            uint32_t *offsets, int grid_w, int trow0, int n_tiles, unsigned long long *keys, uint32_t *vals,
                            uint64_t capacity,
                            uint32_t *flags, uint32_t *hist, int n_digits, uint32_t *tile_count, cudaStream_t stream)
{
    if(n <= 0) return cudaSuccess;
    const int64_t blocks = (n + kThreads - 1) / kThreads;
    return gsx_launch_pdl(emit_kernel, dim3((unsigned)blocks), dim3(kThreads), 0, stream, n, rec, counts, tile_masks,
                          block_offsets, offsets, (unsigned)grid_w, (unsigned)trow0, (unsigned)n_tiles, keys, vals, capacity,
                          flags, hist, n_digits, tile_count);
}
