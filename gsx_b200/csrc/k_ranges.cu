/*
 * Tile ranges and bucket bookkeeping over the sorted instance keys.
 *
 * Follows fastgs/kernels_forward.cuh:558-577 (extract_instance_ranges_cu: [start, end) per tile,
 * empty tiles stay [0, 0)) and :579-593 + forward.cu:250-256 (32-instance buckets per tile and their
 * inclusive prefix).  The per-bucket tile index is written by the blend forward kernel, as in the
 * reference (kernels_forward.cuh:637-644).
 */
#include "gsx_b200_kernels.cuh"

namespace {

constexpr int kThreads = 256;
constexpr int kScanThreads = 1024;

__global__ void __launch_bounds__(kThreads) ranges_kernel(const unsigned long long *__restrict__ keys, uint64_t n,
                                                          uint2 *__restrict__ ranges)
{
    const uint64_t i = (uint64_t)blockIdx.x * kThreads + threadIdx.x;
    if(i >= n) return;
    const uint32_t t = (uint32_t)(keys[i] >> 32);
    if(i == 0 || (uint32_t)(keys[i - 1] >> 32) != t) ranges[t].x = (uint32_t)i;
    if(i + 1 == n || (uint32_t)(keys[i + 1] >> 32) != t) ranges[t].y = (uint32_t)(i + 1);
}

__global__ void __launch_bounds__(kScanThreads) bucket_scan_kernel(const uint2 *__restrict__ ranges, int n_tiles,
                                                                   uint32_t *__restrict__ bucket_offsets,
                                                                   uint32_t *__restrict__ bucket_tile,
                                                                   uint64_t bucket_capacity, uint32_t *__restrict__ flags)
{
    __shared__ uint32_t s_warp[kScanThreads / 32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int per = (n_tiles + kScanThreads - 1) / kScanThreads;
    const int t0 = threadIdx.x * per;
    uint32_t local = 0;
    for(int t = t0; t < t0 + per && t < n_tiles; ++t) {
        const uint2 r = ranges[t];
        local += (r.y - r.x + 31u) / 32u;
    }
    uint32_t incl = local;
#pragma unroll
    for(int d = 1; d < 32; d <<= 1) {
        const uint32_t v = __shfl_up_sync(0xffffffffu, incl, d);
        if(lane >= d) incl += v;
    }
    if(lane == 31) s_warp[warp] = incl;
    __syncthreads();
    uint32_t woff = 0;
    for(int w = 0; w < warp; ++w) woff += s_warp[w];
    uint32_t run = woff + incl - local;
    for(int t = t0; t < t0 + per && t < n_tiles; ++t) {
        const uint2 r = ranges[t];
        run += (r.y - r.x + 31u) / 32u;
        bucket_offsets[t] = run;
    }
    if(threadIdx.x == kScanThreads - 1 && (uint64_t)run > bucket_capacity) atomicOr(flags, GSX_FLAG_BUCKET_OVERFLOW);
    (void)bucket_tile;
}

} // namespace

cudaError_t gsx_launch_tile_ranges(const unsigned long long *keys, uint64_t count, int n_tiles, uint2 *ranges,
                                   uint32_t *bucket_offsets, uint32_t *bucket_tile, uint64_t bucket_capacity,
                                   uint32_t *flags, cudaStream_t stream)
{
    cudaError_t err = cudaMemsetAsync(ranges, 0, sizeof(uint2) * (size_t)n_tiles, stream);
    if(err != cudaSuccess) return err;
    if(count > 0) {
        ranges_kernel<<<(unsigned)((count + kThreads - 1) / kThreads), kThreads, 0, stream>>>(keys, count, ranges);
    }
    bucket_scan_kernel<<<1, kScanThreads, 0, stream>>>(ranges, n_tiles, bucket_offsets, bucket_tile, bucket_capacity, flags);
    return cudaGetLastError();
}
