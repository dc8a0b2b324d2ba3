/*
 * Density control (GSX's default ADC) and the structural tensor operations it needs, on the device.
 *
 *   - gsx_b200_gather_rows: out[r] = x[index[r]] for rows of row_bytes bytes; an out-of-range index
 *     raises a device flag and leaves its row untouched (gsx-cuda/gsx-cuda-kernels.cu:323-345, the
 *     kernel behind gather_tensor, buffer.c:1120-1220, and the optimizer's permute/gather,
 *     optim.c:846-1140).  Rows move as 16-byte vectors when sizes and addresses allow it.
 *   - gsx_b200_clamp_inplace: v < lo -> lo, else v > hi -> hi, NaN passes (gsx-cuda-kernels.cu:440-470).
 *   - the refine pass of the default ADC (gsx-cuda/adc.cu:707-946): growth modes per Gaussian
 *     (duplicate predicate, adc.cu:428-476), the ordered candidate list (thrust::copy_if there), the
 *     split mutation of grown rows (adc.cu:541-705) and the ordered keep list of the prune pass
 *     (adc.cu:499-539).  Selections are a deterministic three-launch compaction (per-block counts,
 *     one-CTA scan of the block counts, ordered scatter) so the lists come out in index order like
 *     the reference's stable copy_if.
 *
 * Compiled with contraction on (-fmad=true), as the reference's CUDA code is; the transcendental
 * functions are CUDA's expf / logf / sqrtf, as in the reference kernels.
 */
#include <cfloat>

#include "../../include/gsx_b200.h"
#include "gsx_b200_kernels.cuh"

int gsx_internal_fail(int code, const char *msg);

namespace {

constexpr int kThreads = 256;
constexpr int kItems = 4;                      /* elements per thread in the selections */
constexpr int kTile = kThreads * kItems;       /* elements per selection block */
constexpr uint8_t kGrowNone = 0, kGrowDuplicate = 1, kGrowSplit = 2;

unsigned grid_for(uint64_t work)
{
    const uint64_t b = (work + kThreads - 1) / kThreads;
    return (unsigned)(b < 148ull * 16 ? (b ? b : 1) : 148ull * 16);
}

/* ------------------------------------------------------------------------------------------ */
/* row gather */

template <typename W>
__global__ void __launch_bounds__(kThreads) gather_rows_kernel(const W *__restrict__ src, W *__restrict__ dst,
                                                               uint64_t words_per_row, uint64_t out_rows,
                                                               const int32_t *__restrict__ index, uint64_t src_rows,
                                                               uint32_t *__restrict__ bad)
{
    const uint64_t total = out_rows * words_per_row;
    for(uint64_t w = (uint64_t)blockIdx.x * kThreads + threadIdx.x; w < total; w += (uint64_t)gridDim.x * kThreads) {
        const uint64_t r = w / words_per_row, k = w - r * words_per_row;
        const int32_t s = __ldg(index + r);
        if(s < 0 || (uint64_t)s >= src_rows) {
            if(bad != nullptr && k == 0) atomicExch(bad, 1u);
            continue;
        }
        dst[w] = src[(uint64_t)s * words_per_row + k];
    }
}

/* ------------------------------------------------------------------------------------------ */
/* clamp */

template <typename T>
__global__ void __launch_bounds__(kThreads) clamp_kernel(T *__restrict__ x, uint64_t n, T lo, T hi)
{
    for(uint64_t i = (uint64_t)blockIdx.x * kThreads + threadIdx.x; i < n; i += (uint64_t)gridDim.x * kThreads) {
        T v = x[i];
        if(v < lo) v = lo;
        else if(v > hi) v = hi;
        x[i] = v;
    }
}

__global__ void iota_kernel(int32_t *__restrict__ dst, uint64_t n)
{
    for(uint64_t i = (uint64_t)blockIdx.x * kThreads + threadIdx.x; i < n; i += (uint64_t)gridDim.x * kThreads) dst[i] = (int32_t)i;
}

/* ------------------------------------------------------------------------------------------ */
/* ordered selection: flags (u8, nonzero = selected) -> indices in increasing order */

__device__ __forceinline__ float max3_scale(const float *logscale, uint64_t i)
{
    const float sx = expf(logscale[i * 3 + 0]), sy = expf(logscale[i * 3 + 1]), sz = expf(logscale[i * 3 + 2]);
    float m = sx;
    if(sy > m) m = sy;
    if(sz > m) m = sz;
    return m;
}

/* block count of the elements whose flag is set, for a block of kTile elements */
__device__ __forceinline__ void block_count(const uint8_t (&f)[kItems], uint32_t *block_counts)
{
    __shared__ uint32_t s_warp[kThreads / 32];
    uint32_t c = 0;
#pragma unroll
    for(int k = 0; k < kItems; ++k) c += f[k] != 0 ? 1u : 0u;
    c = __reduce_add_sync(0xffffffffu, c);
    if((threadIdx.x & 31) == 0) s_warp[threadIdx.x >> 5] = c;
    __syncthreads();
    if(threadIdx.x == 0) {
        uint32_t t = 0;
#pragma unroll
        for(int w = 0; w < kThreads / 32; ++w) t += s_warp[w];
        block_counts[blockIdx.x] = t;
    }
}

/* growth modes of gsx-cuda/adc.cu:428-476: visible counter <= 0 or gradient mean <= threshold: none;
 * otherwise split when the largest scale exceeds scale_threshold * scene_scale, else duplicate */
__global__ void __launch_bounds__(kThreads) grow_modes_kernel(uint64_t n, const float *__restrict__ grad_acc,
                                                              const float *__restrict__ visible_counter,
                                                              const float *__restrict__ logscale, float grad_threshold,
                                                              float split_scale, uint8_t *__restrict__ modes,
                                                              uint32_t *__restrict__ block_counts)
{
    uint8_t f[kItems];
#pragma unroll
    for(int k = 0; k < kItems; ++k) {
        const uint64_t i = (uint64_t)blockIdx.x * kTile + (uint64_t)k * kThreads + threadIdx.x;
        uint8_t m = kGrowNone;
        if(i < n) {
            const float counter = visible_counter != nullptr ? visible_counter[i] : 1.0f;
            if(counter > 0.0f) {
                const float grad = grad_acc[i] / (counter > 1.0f ? counter : 1.0f);
                if(grad > grad_threshold) m = max3_scale(logscale, i) > split_scale ? kGrowSplit : kGrowDuplicate;
            }
            modes[i] = m;
        }
        f[k] = m;
    }
    block_count(f, block_counts);
}

/* keep predicate of gsx-cuda/adc.cu:499-539 */
__global__ void __launch_bounds__(kThreads) keep_flags_kernel(uint64_t n, const float *__restrict__ opacity,
                                                              const float *__restrict__ logscale,
                                                              const float *__restrict__ rotation,
                                                              const float *__restrict__ max_screen_radius,
                                                              uint64_t count_before_growth, bool prune_large,
                                                              float opacity_threshold, float max_world_scale,
                                                              float max_screen_scale, float scene_scale,
                                                              uint8_t *__restrict__ flags, uint32_t *__restrict__ block_counts)
{
    uint8_t f[kItems];
#pragma unroll
    for(int k = 0; k < kItems; ++k) {
        const uint64_t i = (uint64_t)blockIdx.x * kTile + (uint64_t)k * kThreads + threadIdx.x;
        uint8_t keep = 0;
        if(i < n) {
            const float op = 1.0f / (1.0f + expf(-opacity[i]));
            const bool not_transparent = op > opacity_threshold;
            const float q0 = rotation[i * 4 + 0], q1 = rotation[i * 4 + 1], q2 = rotation[i * 4 + 2], q3 = rotation[i * 4 + 3];
            const bool not_degenerate = fabsf(q0) + fabsf(q1) + fabsf(q2) + fabsf(q3) > FLT_EPSILON;
            bool k_ok = not_transparent && not_degenerate;
            if(prune_large) {
                bool not_large_ws = true, not_large_ss = true;
                if(max_world_scale > 0.0f) not_large_ws = max3_scale(logscale, i) < max_world_scale * scene_scale;
                if(max_screen_scale > 0.0f && max_screen_radius != nullptr && i < count_before_growth)
                    not_large_ss = max_screen_radius[i] < max_screen_scale;
                k_ok = k_ok && not_large_ws && not_large_ss;
            }
            keep = k_ok ? 1 : 0;
            flags[i] = keep;
        }
        f[k] = keep;
    }
    block_count(f, block_counts);
}

/* exclusive scan of nb block counts in place (one CTA); block_counts[nb] = total */
__global__ void __launch_bounds__(1024) scan_blocks_kernel(uint32_t *__restrict__ block_counts, uint64_t nb)
{
    __shared__ uint32_t s_w[32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint64_t per = (nb + 1023) / 1024;
    const uint64_t b0 = (uint64_t)threadIdx.x * per;
    uint32_t local = 0;
    for(uint64_t b = b0; b < b0 + per && b < nb; ++b) local += block_counts[b];
    uint32_t incl = local;
#pragma unroll
    for(int d = 1; d < 32; d <<= 1) {
        const uint32_t t = __shfl_up_sync(0xffffffffu, incl, d);
        if(lane >= d) incl += t;
    }
    if(lane == 31) s_w[warp] = incl;
    __syncthreads();
    uint32_t woff = 0, tot = 0;
    for(int k = 0; k < 32; ++k) {
        woff += k < warp ? s_w[k] : 0u;
        tot += s_w[k];
    }
    uint32_t run = woff + incl - local;
    for(uint64_t b = b0; b < b0 + per && b < nb; ++b) {
        const uint32_t v = block_counts[b];
        block_counts[b] = run;
        run += v;
    }
    if(threadIdx.x == 0) block_counts[nb] = tot;
}

/* ordered scatter of the selected indices; with split_count, also counts the splits among the first
 * `budget` selected entries (the ones the growth step keeps) */
__global__ void __launch_bounds__(kThreads) scatter_kernel(uint64_t n, const uint8_t *__restrict__ flags,
                                                           const uint32_t *__restrict__ block_offsets,
                                                           int32_t *__restrict__ out, uint64_t budget,
                                                           uint32_t *__restrict__ split_count)
{
    __shared__ uint32_t s_warp[kThreads / 32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    /* thread t owns elements base + t*kItems .. +kItems-1 (contiguous, so the order is kept) */
    const uint64_t base = (uint64_t)blockIdx.x * kTile + (uint64_t)threadIdx.x * kItems;
    uint8_t f[kItems];
    uint32_t c = 0;
#pragma unroll
    for(int k = 0; k < kItems; ++k) {
        f[k] = base + k < n ? flags[base + k] : 0;
        c += f[k] != 0 ? 1u : 0u;
    }
    uint32_t incl = c;
#pragma unroll
    for(int d = 1; d < 32; d <<= 1) {
        const uint32_t t = __shfl_up_sync(0xffffffffu, incl, d);
        if(lane >= d) incl += t;
    }
    if(lane == 31) s_warp[warp] = incl;
    __syncthreads();
    uint32_t woff = 0;
#pragma unroll
    for(int w = 0; w < kThreads / 32; ++w) woff += w < warp ? s_warp[w] : 0u;
    uint32_t pos = block_offsets[blockIdx.x] + woff + incl - c;
    uint32_t splits = 0;
#pragma unroll
    for(int k = 0; k < kItems; ++k) {
        if(f[k] != 0) {
            out[pos] = (int32_t)(base + k);
            if(split_count != nullptr && pos < budget && f[k] == kGrowSplit) ++splits;
            ++pos;
        }
    }
    if(split_count != nullptr) {
        splits = __reduce_add_sync(0xffffffffu, splits);
        if(lane == 0 && splits) atomicAdd(split_count, splits);
    }
}

/* ------------------------------------------------------------------------------------------ */
/* split mutation of gsx-cuda/adc.cu:541-705 */

__device__ __forceinline__ uint32_t mix32(uint32_t x)
{
    x ^= x >> 16;
    x *= 0x7feb352du;
    x ^= x >> 15;
    x *= 0x846ca68bu;
    x ^= x >> 16;
    return x;
}

/* the reference's per-(grow index, lane) variate: a logistic sample from a hashed uniform */
__device__ __forceinline__ float split_variate(uint64_t seed, uint64_t global_step, uint64_t grow_index, uint32_t lane)
{
    const uint32_t key = (uint32_t)(seed ^ (global_step * 0x9e3779b97f4a7c15ull));
    const uint32_t h = mix32(key ^ (uint32_t)grow_index ^ (lane * 0x9e3779b9u + 0x85ebca6bu));
    float u = ((float)h + 1.0f) / 4294967297.0f;
    if(u <= 1e-6f) u = 1e-6f;
    if(u >= 1.0f - 1e-6f) u = 1.0f - 1e-6f;
    return logf(u / (1.0f - u));
}

__global__ void __launch_bounds__(kThreads) split_kernel(uint64_t grow_count, const int32_t *__restrict__ sources,
                                                         const uint8_t *__restrict__ modes, uint64_t count_before,
                                                         uint64_t seed, uint64_t global_step, float *__restrict__ mean3d,
                                                         float *__restrict__ logscale, float *__restrict__ opacity,
                                                         const float *__restrict__ rotation)
{
    for(uint64_t g = (uint64_t)blockIdx.x * kThreads + threadIdx.x; g < grow_count; g += (uint64_t)gridDim.x * kThreads) {
        const uint64_t src = (uint64_t)sources[g];
        if(src >= count_before || modes[src] != kGrowSplit) continue;
        const uint64_t dst = count_before + g;
        const float sx = expf(logscale[src * 3 + 0]), sy = expf(logscale[src * 3 + 1]), sz = expf(logscale[src * 3 + 2]);
        float so = 1.0f / (1.0f + expf(-opacity[src]));
        float r[6];
#pragma unroll
        for(uint32_t l = 0; l < 6; ++l) r[l] = split_variate(seed, global_step, g, l);
        float qx = rotation[src * 4 + 0], qy = rotation[src * 4 + 1], qz = rotation[src * 4 + 2], qw = rotation[src * 4 + 3];
        const float qn = sqrtf(qx * qx + qy * qy + qz * qz + qw * qw);
        if(qn > 1e-8f) {
            const float inv = 1.0f / qn;
            qx *= inv;
            qy *= inv;
            qz *= inv;
            qw *= inv;
        }
        const float m00 = 1.0f - 2.0f * (qy * qy + qz * qz), m01 = 2.0f * (qx * qy - qw * qz), m02 = 2.0f * (qx * qz + qw * qy);
        const float m10 = 2.0f * (qx * qy + qw * qz), m11 = 1.0f - 2.0f * (qx * qx + qz * qz), m12 = 2.0f * (qy * qz - qw * qx);
        const float m20 = 2.0f * (qx * qz - qw * qy), m21 = 2.0f * (qy * qz + qw * qx), m22 = 1.0f - 2.0f * (qx * qx + qy * qy);
        const float t1x = r[0] * (sx + 1e-5f), t1y = r[1] * (sy + 1e-5f), t1z = r[2] * (sz + 1e-5f);
        const float t2x = r[3] * (sx + 1e-5f), t2y = r[4] * (sy + 1e-5f), t2z = r[5] * (sz + 1e-5f);
        const float o1x = m00 * t1x + m01 * t1y + m02 * t1z, o1y = m10 * t1x + m11 * t1y + m12 * t1z,
                    o1z = m20 * t1x + m21 * t1y + m22 * t1z;
        const float o2x = m00 * t2x + m01 * t2y + m02 * t2z, o2y = m10 * t2x + m11 * t2y + m12 * t2z,
                    o2z = m20 * t2x + m21 * t2y + m22 * t2z;
        if(so < 0.0f) so = 0.0f;
        if(so > 1.0f - 1e-6f) so = 1.0f - 1e-6f;
        float sp = 1.0f - sqrtf(1.0f - so);
        if(sp <= 1e-6f) sp = 1e-6f;
        if(sp >= 1.0f - 1e-6f) sp = 1.0f - 1e-6f;
        const float nlx = logf(sx / 1.6f), nly = logf(sy / 1.6f), nlz = logf(sz / 1.6f);
        const float nop = logf(sp / (1.0f - sp));
        const float mx = mean3d[src * 3 + 0], my = mean3d[src * 3 + 1], mz = mean3d[src * 3 + 2];
        mean3d[dst * 3 + 0] = mx + o1x;
        mean3d[dst * 3 + 1] = my + o1y;
        mean3d[dst * 3 + 2] = mz + o1z;
        logscale[dst * 3 + 0] = nlx;
        logscale[dst * 3 + 1] = nly;
        logscale[dst * 3 + 2] = nlz;
        opacity[dst] = nop;
        mean3d[src * 3 + 0] = mx + o2x;
        mean3d[src * 3 + 1] = my + o2y;
        mean3d[src * 3 + 2] = mz + o2z;
        logscale[src * 3 + 0] = nlx;
        logscale[src * 3 + 1] = nly;
        logscale[src * 3 + 2] = nlz;
        opacity[src] = nop;
    }
}

int launch_status()
{
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? GSX_B200_SUCCESS : gsx_internal_fail(GSX_B200_UNKNOWN, cudaGetErrorString(e));
}

bool aligned(const void *p, unsigned a) { return ((uintptr_t)p % a) == 0; }

} // namespace

extern "C" int gsx_b200_gather_rows(const void *src, uint64_t src_rows, uint64_t row_bytes, const int32_t *index,
                                    uint64_t out_rows, void *dst, uint32_t *device_out_of_range, void *stream_)
{
    if(out_rows == 0 || row_bytes == 0) return GSX_B200_SUCCESS;
    if(src == nullptr || dst == nullptr || index == nullptr)
        return gsx_internal_fail(GSX_B200_INVALID_ARGUMENT, "src, dst and index must be non-null");
    cudaStream_t stream = (cudaStream_t)stream_;
    if(row_bytes % 16 == 0 && aligned(src, 16) && aligned(dst, 16)) {
        const uint64_t w = row_bytes / 16;
        gather_rows_kernel<uint4><<<grid_for(out_rows * w), kThreads, 0, stream>>>(
            static_cast<const uint4 *>(src), static_cast<uint4 *>(dst), w, out_rows, index, src_rows, device_out_of_range);
    } else if(row_bytes % 4 == 0 && aligned(src, 4) && aligned(dst, 4)) {
        const uint64_t w = row_bytes / 4;
        gather_rows_kernel<uint32_t><<<grid_for(out_rows * w), kThreads, 0, stream>>>(
            static_cast<const uint32_t *>(src), static_cast<uint32_t *>(dst), w, out_rows, index, src_rows,
            device_out_of_range);
    } else {
        gather_rows_kernel<uint8_t><<<grid_for(out_rows * row_bytes), kThreads, 0, stream>>>(
            static_cast<const uint8_t *>(src), static_cast<uint8_t *>(dst), row_bytes, out_rows, index, src_rows,
            device_out_of_range);
    }
    return launch_status();
}

extern "C" int gsx_b200_clamp_inplace(void *x, int data_type, uint64_t n, const void *min_value, const void *max_value,
                                      void *stream_)
{
    if(n == 0) return GSX_B200_SUCCESS;
    if(x == nullptr || min_value == nullptr || max_value == nullptr)
        return gsx_internal_fail(GSX_B200_INVALID_ARGUMENT, "x, min_value and max_value must be non-null");
    cudaStream_t stream = (cudaStream_t)stream_;
    switch(data_type) {
    case GSX_B200_DATA_F32:
        clamp_kernel<float><<<grid_for(n), kThreads, 0, stream>>>(static_cast<float *>(x), n, *static_cast<const float *>(min_value),
                                                                  *static_cast<const float *>(max_value));
        break;
    case GSX_B200_DATA_I32:
        clamp_kernel<int32_t><<<grid_for(n), kThreads, 0, stream>>>(static_cast<int32_t *>(x), n,
                                                                    *static_cast<const int32_t *>(min_value),
                                                                    *static_cast<const int32_t *>(max_value));
        break;
    case GSX_B200_DATA_U8:
        clamp_kernel<uint8_t><<<grid_for(n), kThreads, 0, stream>>>(static_cast<uint8_t *>(x), n,
                                                                    *static_cast<const uint8_t *>(min_value),
                                                                    *static_cast<const uint8_t *>(max_value));
        break;
    default:
        return gsx_internal_fail(GSX_B200_NOT_SUPPORTED, "clamp supports f32, i32 and u8");
    }
    return launch_status();
}

extern "C" int gsx_b200_iota_i32(int32_t *dst, uint64_t n, void *stream_)
{
    if(n == 0) return GSX_B200_SUCCESS;
    if(dst == nullptr) return gsx_internal_fail(GSX_B200_INVALID_ARGUMENT, "dst must be non-null");
    iota_kernel<<<grid_for(n), kThreads, 0, (cudaStream_t)stream_>>>(dst, n);
    return launch_status();
}

extern "C" uint64_t gsx_b200_adc_scratch_words(uint64_t n) { return (n + kTile - 1) / kTile + 1; }

extern "C" int gsx_b200_adc_select_growth(uint64_t n, const float *grad_acc, const float *visible_counter,
                                          const float *logscale, float grad_threshold, float scale_threshold,
                                          float scene_scale, uint64_t budget, uint8_t *modes, int32_t *candidates,
                                          uint32_t *scratch, uint32_t *device_counts, void *stream_)
{
    if(n == 0) return GSX_B200_SUCCESS;
    if(n > (uint64_t)INT32_MAX) return gsx_internal_fail(GSX_B200_OUT_OF_RANGE, "gaussian count exceeds int32");
    if(grad_acc == nullptr || logscale == nullptr || modes == nullptr || candidates == nullptr || scratch == nullptr ||
       device_counts == nullptr)
        return gsx_internal_fail(GSX_B200_INVALID_ARGUMENT, "growth selection pointers must be non-null");
    cudaStream_t stream = (cudaStream_t)stream_;
    const uint64_t nb = (n + kTile - 1) / kTile;
    cudaError_t e = cudaMemsetAsync(device_counts + 1, 0, sizeof(uint32_t), stream);
    if(e != cudaSuccess) return gsx_internal_fail(GSX_B200_UNKNOWN, cudaGetErrorString(e));
    grow_modes_kernel<<<(unsigned)nb, kThreads, 0, stream>>>(n, grad_acc, visible_counter, logscale, grad_threshold,
                                                             scale_threshold * scene_scale, modes, scratch);
    scan_blocks_kernel<<<1, 1024, 0, stream>>>(scratch, nb);
    scatter_kernel<<<(unsigned)nb, kThreads, 0, stream>>>(n, modes, scratch, candidates, budget, device_counts + 1);
    e = cudaMemcpyAsync(device_counts, scratch + nb, sizeof(uint32_t), cudaMemcpyDeviceToDevice, stream);
    if(e != cudaSuccess) return gsx_internal_fail(GSX_B200_UNKNOWN, cudaGetErrorString(e));
    return launch_status();
}

extern "C" int gsx_b200_adc_apply_split(uint64_t grow_count, const int32_t *sources, const uint8_t *modes,
                                        uint64_t count_before, uint64_t seed, uint64_t global_step, float *mean3d,
                                        float *logscale, float *opacity, const float *rotation, void *stream_)
{
    if(grow_count == 0) return GSX_B200_SUCCESS;
    if(sources == nullptr || modes == nullptr || mean3d == nullptr || logscale == nullptr || opacity == nullptr ||
       rotation == nullptr)
        return gsx_internal_fail(GSX_B200_INVALID_ARGUMENT, "split pointers must be non-null");
    split_kernel<<<grid_for(grow_count), kThreads, 0, (cudaStream_t)stream_>>>(grow_count, sources, modes, count_before, seed,
                                                                               global_step, mean3d, logscale, opacity,
                                                                               rotation);
    return launch_status();
}

extern "C" int gsx_b200_adc_select_keep(uint64_t n, const float *opacity, const float *logscale, const float *rotation,
                                        const float *max_screen_radius, uint64_t count_before_growth, int prune_large,
                                        float opacity_threshold, float max_world_scale, float max_screen_scale,
                                        float scene_scale, uint8_t *flags, int32_t *keep, uint32_t *scratch,
                                        uint32_t *device_count, void *stream_)
{
    if(n == 0) return GSX_B200_SUCCESS;
    if(n > (uint64_t)INT32_MAX) return gsx_internal_fail(GSX_B200_OUT_OF_RANGE, "gaussian count exceeds int32");
    if(opacity == nullptr || logscale == nullptr || rotation == nullptr || flags == nullptr || keep == nullptr ||
       scratch == nullptr || device_count == nullptr)
        return gsx_internal_fail(GSX_B200_INVALID_ARGUMENT, "keep selection pointers must be non-null");
    cudaStream_t stream = (cudaStream_t)stream_;
    const uint64_t nb = (n + kTile - 1) / kTile;
    keep_flags_kernel<<<(unsigned)nb, kThreads, 0, stream>>>(n, opacity, logscale, rotation, max_screen_radius,
                                                             count_before_growth, prune_large != 0, opacity_threshold,
                                                             max_world_scale, max_screen_scale, scene_scale, flags, scratch);
    scan_blocks_kernel<<<1, 1024, 0, stream>>>(scratch, nb);
    scatter_kernel<<<(unsigned)nb, kThreads, 0, stream>>>(n, flags, scratch, keep, 0, nullptr);
    const cudaError_t e = cudaMemcpyAsync(device_count, scratch + nb, sizeof(uint32_t), cudaMemcpyDeviceToDevice, stream);
    if(e != cudaSuccess) return gsx_internal_fail(GSX_B200_UNKNOWN, cudaGetErrorString(e));
    return launch_status();
}
