/*
 * Stable LSD radix sort of (u64 key, u32 value) pairs, 8-bit digits, one "onesweep" kernel per
 * digit pass (chained-scan digit binning with decoupled lookback, after Adinets & Merrill,
 * "Onesweep: A Faster Least Significant Digit Radix Sort for GPUs", 2022), preceded by a single
 * upfront histogram kernel that counts every pass's digits in one read of the keys.
 *
 * This replaces the reference's two CUB sorts (fastgs/forward.cu:155-161, 32-bit depth keys over
 * visible primitives, then :214-220, stable 16-bit tile keys over instances): one sort of the
 * combined tile|depth key gives the same (tile, depth) order.  Only bits [begin_bit, end_bit) are
 * sorted (for the render keys: 32 depth bits plus ceil(log2(tiles)) tile bits).
 *
 * Per pass, each block takes a dynamically numbered tile of 4096 pairs (8 per thread of 512, in a
 * warp-striped arrangement), ranks them with warp-level multisplit (__match_any_sync), publishes
 * per-digit counts to the lookback table, resolves its global digit offsets by looking back at
 * predecessor tiles (bounded spin: on timeout it sets GSX_FLAG_LOOKBACK_TIMEOUT and carries on
 * rather than hang), and scatters through shared memory so global writes are digit-contiguous.
 */
#include "gsx_b200_kernels.cuh"

namespace {

constexpr int kThreads = 512;
constexpr int kWarps = kThreads / 32;
constexpr int kItems = 8;
constexpr int kTile = kThreads * kItems; /* 4096 */
constexpr int kRadix = 256;
constexpr int kHistBlocks = 148 * 4;
constexpr uint32_t kValMask = (1u << 30) - 1u;
constexpr uint32_t kAgg = 1u << 30;
constexpr uint32_t kInc = 2u << 30;

__device__ __forceinline__ uint32_t digit_of(unsigned long long key, int shift, uint32_t mask)
{
    return (uint32_t)(key >> shift) & mask;
}

__global__ void __launch_bounds__(kThreads) histogram_kernel(const unsigned long long *__restrict__ keys, uint64_t n,
                                                             int begin_bit, int end_bit, int passes,
                                                             uint32_t *__restrict__ hist)
{
    __shared__ uint32_t s_hist[8][kRadix];
    for(int j = threadIdx.x; j < 8 * kRadix; j += kThreads) (&s_hist[0][0])[j] = 0u;
    __syncthreads();
    for(uint64_t i = (uint64_t)blockIdx.x * kThreads + threadIdx.x; i < n; i += (uint64_t)gridDim.x * kThreads) {
        const unsigned long long k = keys[i];
        for(int p = 0; p < passes; ++p) {
            const int shift = begin_bit + 8 * p;
            const int bits = end_bit - shift < 8 ? end_bit - shift : 8;
            atomicAdd(&s_hist[p][digit_of(k, shift, (1u << bits) - 1u)], 1u);
        }
    }
    __syncthreads();
    for(int j = threadIdx.x; j < passes * kRadix; j += kThreads) {
        const uint32_t v = (&s_hist[0][0])[j];
        if(v) atomicAdd(&hist[j], v);
    }
}

/* block-wide exclusive scan of one value per thread (256 threads) */
__device__ __forceinline__ uint32_t block_exclusive_scan(uint32_t v, uint32_t *s_warp, uint32_t *total)
{
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint32_t incl = v;
#pragma unroll
    for(int d = 1; d < 32; d <<= 1) {
        const uint32_t t = __shfl_up_sync(0xffffffffu, incl, d);
        if(lane >= d) incl += t;
    }
    __syncthreads();
    if(lane == 31) s_warp[warp] = incl;
    __syncthreads();
    uint32_t woff = 0, tot = 0;
#pragma unroll
    for(int w = 0; w < kWarps; ++w) {
        const uint32_t s = s_warp[w];
        woff += w < warp ? s : 0u;
        tot += s;
    }
    if(total) *total = tot;
    return woff + incl - v;
}

__global__ void __launch_bounds__(kThreads) onesweep_kernel(const unsigned long long *__restrict__ keys_in,
                                                            const uint32_t *__restrict__ vals_in,
                                                            unsigned long long *__restrict__ keys_out,
                                                            uint32_t *__restrict__ vals_out, uint64_t n, int shift,
                                                            uint32_t mask, const uint32_t *__restrict__ hist,
                                                            uint32_t *__restrict__ lookback, uint32_t *__restrict__ tile_counter,
                                                            uint32_t *__restrict__ flags)
{
    extern __shared__ __align__(16) unsigned char smem[];
    unsigned long long *s_keys = reinterpret_cast<unsigned long long *>(smem);               /* kTile * 8 */
    uint32_t *s_vals = reinterpret_cast<uint32_t *>(smem + kTile * 8);                       /* kTile * 4 */
    uint32_t *s_whist = reinterpret_cast<uint32_t *>(smem + kTile * 12);                     /* kWarps * 256 */
    uint32_t *s_digit_base = s_whist + kWarps * kRadix;                                      /* 256: global base */
    uint32_t *s_block_excl = s_digit_base + kRadix;                                          /* 256 */
    uint32_t *s_misc = s_block_excl + kRadix;                                                /* 32 */
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;

    if(threadIdx.x == 0) s_misc[kWarps] = atomicAdd(tile_counter, 1u);
    for(int j = threadIdx.x; j < kWarps * kRadix; j += kThreads) s_whist[j] = 0u;
    __syncthreads();
    const uint32_t tile = s_misc[kWarps];
    const uint64_t tile_base = (uint64_t)tile * kTile;

    /* load (warp-striped) */
    unsigned long long k[kItems];
    uint32_t v[kItems], dg[kItems], rank[kItems];
    const uint64_t wbase = tile_base + (uint64_t)warp * (32 * kItems) + lane;
#pragma unroll
    for(int it = 0; it < kItems; ++it) {
        const uint64_t idx = wbase + (uint64_t)it * 32;
        if(idx < n) {
            k[it] = keys_in[idx];
            v[it] = vals_in[idx];
            dg[it] = digit_of(k[it], shift, mask);
        } else {
            k[it] = 0ull;
            v[it] = 0u;
            dg[it] = kRadix; /* not a bin: never counted or written */
        }
    }
    /* warp-level multisplit ranking, in (item, lane) order = input order */
    const unsigned lt = (1u << lane) - 1u;
    uint32_t *wh = s_whist + warp * kRadix;
#pragma unroll
    for(int it = 0; it < kItems; ++it) {
        const unsigned peers = __match_any_sync(0xffffffffu, dg[it]);
        const int leader = __ffs(peers) - 1;
        uint32_t base = 0;
        if(lane == leader && dg[it] < kRadix) {
            base = wh[dg[it]];
            wh[dg[it]] = base + (uint32_t)__popc(peers);
        }
        base = __shfl_sync(0xffffffffu, base, leader);
        rank[it] = base + (uint32_t)__popc(peers & lt);
        __syncwarp();
    }
    __syncthreads();

    /* per digit (threads 0..255, thread d = digit d): block count, exclusive over warps */
    const int d = threadIdx.x;
    const bool is_digit = d < kRadix;
    uint32_t count = 0;
    if(is_digit) {
#pragma unroll
        for(int w = 0; w < kWarps; ++w) {
            const uint32_t c = s_whist[w * kRadix + d];
            s_whist[w * kRadix + d] = count;
            count += c;
        }
    }
    /* global base of digit d = exclusive scan of the pass histogram */
    const uint32_t hbase = block_exclusive_scan(is_digit ? hist[d] : 0u, s_misc, nullptr);
    const uint32_t bexcl = block_exclusive_scan(count, s_misc, nullptr);
    if(is_digit) s_block_excl[d] = bexcl;

    /* decoupled lookback for digit d */
    uint32_t *my_status = lookback + (uint64_t)tile * kRadix + d;
    uint32_t prefix = 0;
    if(!is_digit) {
    } else if(tile == 0) {
        gsx_st_relaxed(my_status, kInc | count);
    } else {
        gsx_st_relaxed(my_status, kAgg | count);
        int64_t j = (int64_t)tile - 1;
        unsigned spins = 0;
        while(j >= 0) {
            const uint32_t st = gsx_ld_relaxed(lookback + (uint64_t)j * kRadix + d);
            const uint32_t fl = st & ~kValMask;
            if(fl == 0u) {
                if(++spins > GSX_SPIN_LIMIT) {
                    atomicOr(flags, GSX_FLAG_LOOKBACK_TIMEOUT);
                    break;
                }
                continue;
            }
            prefix += st & kValMask;
            if(fl == kInc) break;
            --j;
        }
        gsx_st_relaxed(my_status, kInc | (prefix + count));
    }
    if(is_digit) s_digit_base[d] = hbase + prefix;
    __syncthreads();

    /* stage into shared memory in block-sorted order */
#pragma unroll
    for(int it = 0; it < kItems; ++it) {
        if(dg[it] < kRadix) {
            const uint32_t pos = s_block_excl[dg[it]] + s_whist[warp * kRadix + dg[it]] + rank[it];
            s_keys[pos] = k[it];
            s_vals[pos] = v[it];
        }
    }
    __syncthreads();
    const uint64_t remaining = n - tile_base;
    const uint32_t valid = remaining < (uint64_t)kTile ? (uint32_t)remaining : (uint32_t)kTile;
    for(uint32_t j = threadIdx.x; j < valid; j += kThreads) {
        const unsigned long long key = s_keys[j];
        const uint32_t dj = digit_of(key, shift, mask);
        const uint64_t out = (uint64_t)s_digit_base[dj] + (j - s_block_excl[dj]);
        keys_out[out] = key;
        vals_out[out] = s_vals[j];
    }
}

constexpr size_t kSmemBytes = (size_t)kTile * 12 + (size_t)kWarps * kRadix * 4 + 2 * kRadix * 4 + 32 * 4;

bool g_attr_set[256];

cudaError_t ensure_onesweep_attr()
{
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if(err != cudaSuccess) return err;
    if(dev >= 0 && dev < 256 && g_attr_set[dev]) return cudaSuccess;
    err = cudaFuncSetAttribute(onesweep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
    if(err == cudaSuccess && dev >= 0 && dev < 256) g_attr_set[dev] = true;
    return err;
}

} // namespace

size_t gsx_sort_scratch_bytes(uint64_t capacity)
{
    const uint64_t tiles = (capacity + kTile - 1) / kTile;
    /* 8 passes max: hist 8*256, counters 8 (+pad), lookback 8 * tiles * 256 (u32 each) */
    return (size_t)(8 * kRadix + 64 + 8 * tiles * kRadix) * 4;
}

cudaError_t gsx_launch_sort_pairs(unsigned long long *keys_a, uint32_t *vals_a, unsigned long long *keys_b,
                                  uint32_t *vals_b, uint64_t count, int begin_bit, int end_bit, void *scratch,
                                  size_t scratch_bytes, uint32_t *flags, int *out_result_in_b, cudaStream_t stream)
{
    *out_result_in_b = 0;
    if(count == 0 || end_bit <= begin_bit) return cudaSuccess;
    if(count >= (1ull << 30) || begin_bit < 0 || end_bit > 64) return cudaErrorInvalidValue;
    const int passes = (end_bit - begin_bit + 7) / 8;
    if(passes > 8) return cudaErrorInvalidValue;
    const uint64_t tiles = (count + kTile - 1) / kTile;
    const size_t need = (size_t)(8 * kRadix + 64 + (uint64_t)passes * tiles * kRadix) * 4;
    if(scratch_bytes < need) return cudaErrorInvalidValue;
    uint32_t *hist = reinterpret_cast<uint32_t *>(scratch);
    uint32_t *counters = hist + 8 * kRadix;
    uint32_t *lookback = counters + 64;
    cudaError_t err = cudaMemsetAsync(scratch, 0, need, stream);
    if(err != cudaSuccess) return err;
    err = ensure_onesweep_attr();
    if(err != cudaSuccess) return err;
    uint64_t hblocks = (count + kThreads - 1) / kThreads;
    if(hblocks > kHistBlocks) hblocks = kHistBlocks;
    histogram_kernel<<<(unsigned)hblocks, kThreads, 0, stream>>>(keys_a, count, begin_bit, end_bit, passes, hist);
    unsigned long long *kin = keys_a, *kout = keys_b;
    uint32_t *vin = vals_a, *vout = vals_b;
    for(int p = 0; p < passes; ++p) {
        const int shift = begin_bit + 8 * p;
        const int bits = end_bit - shift < 8 ? end_bit - shift : 8;
        onesweep_kernel<<<(unsigned)tiles, kThreads, kSmemBytes, stream>>>(
            kin, vin, kout, vout, count, shift, (1u << bits) - 1u, hist + p * kRadix,
            lookback + (uint64_t)p * tiles * kRadix, counters + p, flags);
        unsigned long long *tk = kin;
        kin = kout;
        kout = tk;
        uint32_t *tv = vin;
        vin = vout;
        vout = tv;
    }
    *out_result_in_b = passes & 1;
    return cudaGetLastError();
}

/* Digit passes chosen by the caller (the render pipeline skips passes whose digit is the same for
 * every key; its emission kernel produced the per-position histograms).  hist holds 256 counters
 * per digit position; pass i sorts the digit at bit `shifts[i]`, `widths[i]` bits wide, using
 * hist + positions[i] * 256.  scratch holds the tile counters and lookback tables. */
cudaError_t gsx_launch_sort_passes(unsigned long long *keys_a, uint32_t *vals_a, unsigned long long *keys_b,
                                   uint32_t *vals_b, uint64_t count, const int *positions, const int *shifts,
                                   const int *widths, int npasses, const uint32_t *hist, void *scratch,
                                   size_t scratch_bytes, uint32_t *flags, int *out_result_in_b, cudaStream_t stream)
{
    *out_result_in_b = 0;
    if(count == 0 || npasses == 0) return cudaSuccess;
    if(count >= (1ull << 30) || npasses > 8) return cudaErrorInvalidValue;
    const uint64_t tiles = (count + kTile - 1) / kTile;
    const size_t need = (size_t)(64 + (uint64_t)npasses * tiles * kRadix) * 4;
    if(scratch_bytes < need) return cudaErrorInvalidValue;
    uint32_t *counters = reinterpret_cast<uint32_t *>(scratch);
    uint32_t *lookback = counters + 64;
    cudaError_t err = cudaMemsetAsync(scratch, 0, need, stream);
    if(err != cudaSuccess) return err;
    err = ensure_onesweep_attr();
    if(err != cudaSuccess) return err;
    unsigned long long *kin = keys_a, *kout = keys_b;
    uint32_t *vin = vals_a, *vout = vals_b;
    for(int p = 0; p < npasses; ++p) {
        onesweep_kernel<<<(unsigned)tiles, kThreads, kSmemBytes, stream>>>(
            kin, vin, kout, vout, count, shifts[p], (1u << widths[p]) - 1u, hist + positions[p] * kRadix,
            lookback + (uint64_t)p * tiles * kRadix, counters + p, flags);
        unsigned long long *tk = kin;
        kin = kout;
        kout = tk;
        uint32_t *tv = vin;
        vin = vout;
        vout = tv;
    }
    *out_result_in_b = npasses & 1;
    return cudaGetLastError();
}

/* ------------------------------------------------------------------------------------------------
 * Allocation-free variant (gsx_b200_sort_pairs_noalloc, include/gsx_b200.h).
 *
 * Some callers must not allocate device memory on their own: a host that hands every buffer out of
 * its own arenas and accounts for all device memory (GSX's backend model), or a plugin host with a
 * fixed GPU memory budget that forbids hidden cudaMalloc calls.  For them the sort's scratch (the
 * alternate key/value buffers, the digit histograms, the lookback table and one status word) lives
 * in one file-scope device array sized for GSX_B200_NOALLOC_SORT_MAX_PAIRS pairs.  Every GPU that
 * loads this library holds the array until the process exits.  All calls share it: calls that
 * overlap on the GPU (different streams, or different host threads on the same device) race and
 * must be serialised by the caller.  Each call clears the status word first and reads it back after
 * the sort (so the call waits for its stream), returning GSX_B200_UNKNOWN if the bounded lookback
 * wait gave up.
 */
#include "../../include/gsx_b200.h"

#include <mutex>

int gsx_internal_fail(int code, const char *msg);

namespace {

constexpr uint64_t kNoAllocPairs = GSX_B200_NOALLOC_SORT_MAX_PAIRS;
constexpr size_t kNoAllocKeysBytes = (size_t)kNoAllocPairs * sizeof(unsigned long long);
constexpr size_t kNoAllocValsBytes = (size_t)kNoAllocPairs * sizeof(uint32_t);
constexpr size_t kNoAllocSortBytes = (size_t)(8 * kRadix + 64 + 8 * ((kNoAllocPairs + kTile - 1) / kTile) * kRadix) * 4;
constexpr size_t kNoAllocFlagBytes = 256;
constexpr size_t kNoAllocBytes = kNoAllocKeysBytes + kNoAllocValsBytes + kNoAllocSortBytes + kNoAllocFlagBytes;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

std::mutex g_noalloc_mutex;
unsigned char *g_noalloc_ptr[256];

} // namespace

extern "C" int gsx_b200_sort_pairs_noalloc(uint64_t *keys, uint32_t *values, uint64_t count, int32_t begin_bit,
                                           int32_t end_bit, void *stream_)
{
    if(count > 0 && (keys == nullptr || values == nullptr))
        return gsx_internal_fail(GSX_B200_INVALID_ARGUMENT, "keys and values must be non-null");
    if(begin_bit < 0 || end_bit > 64 || begin_bit > end_bit)
        return gsx_internal_fail(GSX_B200_OUT_OF_RANGE, "bit range must satisfy 0 <= begin <= end <= 64");
    if(count > kNoAllocPairs)
        return gsx_internal_fail(GSX_B200_OUT_OF_RANGE,
                                 "gsx_b200_sort_pairs_noalloc: count exceeds GSX_B200_NOALLOC_SORT_MAX_PAIRS (1048576)");
    if(count == 0 || begin_bit == end_bit) return GSX_B200_SUCCESS;
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if(err != cudaSuccess) return gsx_internal_fail(GSX_B200_UNKNOWN, cudaGetErrorString(err));
    if(dev < 0 || dev >= 256) return gsx_internal_fail(GSX_B200_OUT_OF_RANGE, "device ordinal out of range");
    unsigned char *base = nullptr;
    {
        /* once per device, with that device current: the array's device address (the host-side
         * name of the array is not a device address) */
        std::lock_guard<std::mutex> lock(g_noalloc_mutex);
        if(g_noalloc_ptr[dev] == nullptr) {
            void *p = nullptr;
            err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
            if(err != cudaSuccess) return gsx_internal_fail(GSX_B200_UNKNOWN, cudaGetErrorString(err));
            g_noalloc_ptr[dev] = static_cast<unsigned char *>(p);
        }
        base = g_noalloc_ptr[dev];
    }
    cudaStream_t stream = (cudaStream_t)stream_;
    unsigned long long *keys_b = reinterpret_cast<unsigned long long *>(base);
    uint32_t *vals_b = reinterpret_cast<uint32_t *>(base + kNoAllocKeysBytes);
    void *scratch = base + kNoAllocKeysBytes + kNoAllocValsBytes;
    uint32_t *flags = reinterpret_cast<uint32_t *>(base + kNoAllocKeysBytes + kNoAllocValsBytes + kNoAllocSortBytes);
    int in_b = 0;
    /* the status word keeps the previous call's value: clear it.  The launcher clears the
     * histograms, tile counters and lookback table itself. */
    err = cudaMemsetAsync(flags, 0, sizeof(uint32_t), stream);
    if(err == cudaSuccess)
        err = gsx_launch_sort_pairs(reinterpret_cast<unsigned long long *>(keys), values, keys_b, vals_b, count,
                                    begin_bit, end_bit, scratch, kNoAllocSortBytes, flags, &in_b, stream);
    if(err == cudaSuccess && in_b) {
        err = cudaMemcpyAsync(keys, keys_b, sizeof(uint64_t) * count, cudaMemcpyDeviceToDevice, stream);
        if(err == cudaSuccess)
            err = cudaMemcpyAsync(values, vals_b, sizeof(uint32_t) * count, cudaMemcpyDeviceToDevice, stream);
    }
    /* read the status word back (a copy into pageable host memory: returns once the sort is done) */
    uint32_t status = 0;
    if(err == cudaSuccess) err = cudaMemcpyAsync(&status, flags, sizeof(uint32_t), cudaMemcpyDeviceToHost, stream);
    if(err == cudaSuccess) err = cudaStreamSynchronize(stream);
    if(err != cudaSuccess) return gsx_internal_fail(GSX_B200_UNKNOWN, cudaGetErrorString(err));
    if(status & GSX_FLAG_LOOKBACK_TIMEOUT)
        return gsx_internal_fail(GSX_B200_UNKNOWN,
                                 "gsx_b200_sort_pairs_noalloc: a decoupled-lookback wait timed out; the output order is invalid");
    return GSX_B200_SUCCESS;
}
