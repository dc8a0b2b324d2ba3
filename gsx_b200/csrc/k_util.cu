/*
 * Small buffer kernels behind the GSX backend-buffer interface (gsx-impl.h:349-353 fill_tensor and
 * :377-381 check_finite_tensor), used by the GSX provider (gsx_b200/provider/).
 */
#include "../../include/gsx_b200.h"
#include "gsx_b200_kernels.cuh"

int gsx_internal_fail(int code, const char *msg);

namespace {

constexpr int kThreads = 256;

/* dst[i] = pattern for n 8-byte words (the pattern already repeated to 8 bytes) */
__global__ void __launch_bounds__(kThreads) fill8_kernel(unsigned long long *__restrict__ dst, uint64_t n,
                                                          unsigned long long pattern)
{
    for(uint64_t i = (uint64_t)blockIdx.x * kThreads + threadIdx.x; i < n; i += (uint64_t)gridDim.x * kThreads) dst[i] = pattern;
}

/* byte-granular tail: dst[i] = byte (i mod 8) of the 8-byte pattern, starting at phase */
__global__ void fill_tail_kernel(unsigned char *__restrict__ dst, uint64_t n, unsigned long long pattern, unsigned phase)
{
    const uint64_t i = (uint64_t)blockIdx.x * kThreads + threadIdx.x;
    if(i < n) dst[i] = (unsigned char)(pattern >> (8u * ((phase + (unsigned)i) & 7u)));
}

__global__ void __launch_bounds__(kThreads) count_nonfinite_kernel(const float *__restrict__ x, uint64_t n,
                                                                    uint32_t *__restrict__ count)
{
    uint32_t local = 0;
    for(uint64_t i = (uint64_t)blockIdx.x * kThreads + threadIdx.x; i < n; i += (uint64_t)gridDim.x * kThreads) {
        const uint32_t b = __float_as_uint(x[i]);
        local += (b & 0x7f800000u) == 0x7f800000u ? 1u : 0u;
    }
    local = __reduce_add_sync(0xffffffffu, local);
    if((threadIdx.x & 31) == 0 && local) atomicAdd(count, local);
}

/* splitmix64 finaliser: a bijective 64-bit mix */
__device__ __forceinline__ unsigned long long mix64(unsigned long long z)
{
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

/* out += sum over i of mix64(word_i ^ (salt + i * golden)): changing any word (or moving it) changes
 * its term, so the sum changes unless two 64-bit mixes collide */
__global__ void __launch_bounds__(kThreads) fingerprint_kernel(const uint32_t *__restrict__ x, uint64_t n,
                                                                unsigned long long salt, unsigned long long *out)
{
    unsigned long long acc = 0;
    for(uint64_t i = (uint64_t)blockIdx.x * kThreads + threadIdx.x; i < n; i += (uint64_t)gridDim.x * kThreads)
        acc += mix64((unsigned long long)__ldg(x + i) ^ (salt + i * 0x9e3779b97f4a7c15ull));
    for(int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if((threadIdx.x & 31) == 0) atomicAdd(out, acc);
}

unsigned grid_for(uint64_t n)
{
    const uint64_t b = (n + kThreads - 1) / kThreads;
    return (unsigned)(b < 148ull * 16 ? (b ? b : 1) : 148ull * 16);
}

} // namespace

extern "C" int gsx_b200_fill_pattern(void *dst, uint64_t size_bytes, const void *pattern, uint32_t pattern_bytes, void *stream_)
{
    if(size_bytes == 0) return GSX_B200_SUCCESS;
    if(dst == nullptr || pattern == nullptr) return gsx_internal_fail(GSX_B200_INVALID_ARGUMENT, "dst and pattern must be non-null");
    if(pattern_bytes != 1 && pattern_bytes != 2 && pattern_bytes != 4 && pattern_bytes != 8)
        return gsx_internal_fail(GSX_B200_INVALID_ARGUMENT, "pattern_bytes must be 1, 2, 4 or 8");
    if(size_bytes % pattern_bytes != 0)
        return gsx_internal_fail(GSX_B200_INVALID_ARGUMENT, "size_bytes must be a multiple of pattern_bytes");
    if(((uintptr_t)dst % pattern_bytes) != 0) return gsx_internal_fail(GSX_B200_INVALID_ARGUMENT, "dst is not aligned to the pattern");
    cudaStream_t stream = (cudaStream_t)stream_;
    const unsigned char *pb = static_cast<const unsigned char *>(pattern);
    unsigned long long word = 0;
    for(unsigned k = 0; k < 8; ++k) word |= (unsigned long long)pb[k % pattern_bytes] << (8u * k);
    unsigned char *p = static_cast<unsigned char *>(dst);
    /* head bytes up to an 8-byte boundary, 8-byte body, tail bytes; the pattern phase follows the
     * byte offset from dst (pattern_bytes divides 8, so phase = offset mod 8 keeps it aligned) */
    const uint64_t head = ((8u - ((uintptr_t)p & 7u)) & 7u) < size_bytes ? ((8u - ((uintptr_t)p & 7u)) & 7u) : size_bytes;
    if(head) fill_tail_kernel<<<1, kThreads, 0, stream>>>(p, head, word, 0u);
    const uint64_t body = (size_bytes - head) / 8u;
    if(body) {
        /* the body starts at byte offset `head`, so its words begin at pattern phase head mod 8 */
        const unsigned sh = (unsigned)(head & 7u) * 8u;
        const unsigned long long rot = sh ? (word >> sh) | (word << (64u - sh)) : word;
        fill8_kernel<<<grid_for(body), kThreads, 0, stream>>>(reinterpret_cast<unsigned long long *>(p + head), body, rot);
    }
    const uint64_t tail = size_bytes - head - body * 8u;
    if(tail) fill_tail_kernel<<<1, kThreads, 0, stream>>>(p + head + body * 8u, tail, word, (unsigned)((head + body * 8u) & 7u));
    const cudaError_t err = cudaGetLastError();
    if(err != cudaSuccess) return gsx_internal_fail(GSX_B200_UNKNOWN, cudaGetErrorString(err));
    return GSX_B200_SUCCESS;
}

extern "C" int gsx_b200_count_nonfinite_f32(const float *x, uint64_t n, uint32_t *device_count, void *stream_)
{
    if(n == 0) return GSX_B200_SUCCESS;
    if(x == nullptr || device_count == nullptr) return gsx_internal_fail(GSX_B200_INVALID_ARGUMENT, "x and device_count must be non-null");
    count_nonfinite_kernel<<<grid_for(n), kThreads, 0, (cudaStream_t)stream_>>>(x, n, device_count);
    const cudaError_t err = cudaGetLastError();
    if(err != cudaSuccess) return gsx_internal_fail(GSX_B200_UNKNOWN, cudaGetErrorString(err));
    return GSX_B200_SUCCESS;
}

/* 64-bit fingerprint of the Gaussian fields (mean3d, rotation, logscale, opacity, sh0, and sh1..sh3
 * up to sh_degree) into *out (device): one streaming pass, used to detect inputs changed between a
 * borrowed TRAIN forward and its backward. */
cudaError_t gsx_launch_fingerprint(const float *const *fields, const uint64_t *counts, int n_fields, unsigned long long *out,
                                   cudaStream_t stream)
{
    cudaError_t e = cudaMemsetAsync(out, 0, sizeof(unsigned long long), stream);
    for(int f = 0; f < n_fields && e == cudaSuccess; ++f) {
        if(fields[f] == nullptr || counts[f] == 0) continue;
        fingerprint_kernel<<<grid_for(counts[f]), kThreads, 0, stream>>>(reinterpret_cast<const uint32_t *>(fields[f]),
                                                                         counts[f], 0x51ed270b27a1f5c3ull * (f + 1), out);
        e = cudaGetLastError();
    }
    return e;
}
