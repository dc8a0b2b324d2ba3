/*
 * Image layout conversion on the step's input side: an interleaved HWC image (u8 or f32, 3 channels
 * or 1) to a planar CHW f32 tensor, values unchanged (no 1/255 scaling).  Same result as the
 * reference's CPU packer gsx_dataloader_pack_hwc_to_chw / pack_hw_to_chw (gsx-data-impl.h:174-260,
 * f32 output) and its CUDA dataloader kernels (gsx-cuda/async_dl.cu:45-101).  Those CUDA kernels
 * run one thread per element on a grid clamped to 65535 blocks of 256 with no stride loop
 * (async_dl.cu:103-130), so they convert only the first 16,776,960 elements (a 3840x2160 RGB image
 * has 24,883,200); this kernel converts every pixel.
 *
 * HBM-bound byte work: per pixel 3 (u8) or 12 (f32) bytes in and 12 bytes out.  Each thread moves a
 * group of pixels with 16-byte loads and stores: 16 pixels of u8 RGB (three 16-byte loads, four
 * float4 stores per plane) or 4 pixels of f32 RGB (three float4 loads, one float4 store per plane).
 * A group that is ragged (the image's last pixels) or not 16-byte aligned falls back to element
 * loads and stores.
 */
#include "../../include/gsx_b200.h"
#include "gsx_b200_kernels.cuh"

int gsx_internal_fail(int code, const char *msg);

namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ float u8_at(const uint4 *v, int b)
{
    const uint32_t w = (&v->x)[(b >> 2) & 3];
    return (float)((w >> (8 * (b & 3))) & 0xffu);
}

/* u8 HWC RGB -> f32 CHW, 16 pixels per thread */
__global__ void __launch_bounds__(kThreads) rgb_u8_kernel(const uint8_t *__restrict__ src, float *__restrict__ dst,
                                                          uint64_t P, bool vec)
{
    const uint64_t groups = (P + 15) / 16;
    for(uint64_t gi = (uint64_t)blockIdx.x * kThreads + threadIdx.x; gi < groups; gi += (uint64_t)gridDim.x * kThreads) {
        const uint64_t p0 = gi * 16;
        if(vec && p0 + 16 <= P) {
            const uint4 *s = reinterpret_cast<const uint4 *>(src + p0 * 3);
            uint4 in[3];
            in[0] = __ldcs(s);
            in[1] = __ldcs(s + 1);
            in[2] = __ldcs(s + 2);
#pragma unroll
            for(int c = 0; c < 3; ++c) {
                float4 *d = reinterpret_cast<float4 *>(dst + (uint64_t)c * P + p0);
#pragma unroll
                for(int q = 0; q < 4; ++q) {
                    float v[4];
#pragma unroll
                    for(int k = 0; k < 4; ++k) {
                        const int b = (4 * q + k) * 3 + c; /* byte within the 48-byte group */
                        v[k] = u8_at(&in[b >> 4], b & 15);
                    }
                    __stcs(d + q, make_float4(v[0], v[1], v[2], v[3]));
                }
            }
        } else {
            for(uint64_t p = p0; p < p0 + 16 && p < P; ++p)
                for(int c = 0; c < 3; ++c) dst[(uint64_t)c * P + p] = (float)src[p * 3 + c];
        }
    }
}

/* f32 HWC RGB -> f32 CHW, 4 pixels per thread */
__global__ void __launch_bounds__(kThreads) rgb_f32_kernel(const float *__restrict__ src, float *__restrict__ dst,
                                                           uint64_t P, bool vec)
{
    const uint64_t groups = (P + 3) / 4;
    for(uint64_t gi = (uint64_t)blockIdx.x * kThreads + threadIdx.x; gi < groups; gi += (uint64_t)gridDim.x * kThreads) {
        const uint64_t p0 = gi * 4;
        if(vec && p0 + 4 <= P) {
            const float4 *s = reinterpret_cast<const float4 *>(src + p0 * 3);
            const float4 a = __ldcs(s), b = __ldcs(s + 1), c = __ldcs(s + 2);
            /* a = r0 g0 b0 r1, b = g1 b1 r2 g2, c = b2 r3 g3 b3 */
            __stcs(reinterpret_cast<float4 *>(dst + p0), make_float4(a.x, a.w, b.z, c.y));
            __stcs(reinterpret_cast<float4 *>(dst + P + p0), make_float4(a.y, b.x, b.w, c.z));
            __stcs(reinterpret_cast<float4 *>(dst + 2 * P + p0), make_float4(a.z, b.y, c.x, c.w));
        } else {
            for(uint64_t p = p0; p < p0 + 4 && p < P; ++p)
                for(int c = 0; c < 3; ++c) dst[(uint64_t)c * P + p] = src[p * 3 + c];
        }
    }
}

/* u8 HW -> f32, 16 pixels per thread */
__global__ void __launch_bounds__(kThreads) plane_u8_kernel(const uint8_t *__restrict__ src, float *__restrict__ dst,
                                                            uint64_t P, bool vec)
{
    const uint64_t groups = (P + 15) / 16;
    for(uint64_t gi = (uint64_t)blockIdx.x * kThreads + threadIdx.x; gi < groups; gi += (uint64_t)gridDim.x * kThreads) {
        const uint64_t p0 = gi * 16;
        if(vec && p0 + 16 <= P) {
            const uint4 in = __ldcs(reinterpret_cast<const uint4 *>(src + p0));
            float4 *d = reinterpret_cast<float4 *>(dst + p0);
#pragma unroll
            for(int q = 0; q < 4; ++q)
                __stcs(d + q, make_float4(u8_at(&in, 4 * q), u8_at(&in, 4 * q + 1), u8_at(&in, 4 * q + 2), u8_at(&in, 4 * q + 3)));
        } else {
            for(uint64_t p = p0; p < p0 + 16 && p < P; ++p) dst[p] = (float)src[p];
        }
    }
}

unsigned grid_for(uint64_t groups)
{
    const uint64_t b = (groups + kThreads - 1) / kThreads;
    return (unsigned)(b < 148ull * 16 ? (b ? b : 1) : 148ull * 16);
}

bool aligned16(const void *p) { return ((uintptr_t)p & 15u) == 0; }

} // namespace

extern "C" int gsx_b200_hwc_to_chw_f32(const void *src, int src_type, int channels, uint64_t pixel_count, float *dst,
                                       void *stream_)
{
    if(pixel_count == 0) return GSX_B200_SUCCESS;
    if(src == nullptr || dst == nullptr) return gsx_internal_fail(GSX_B200_INVALID_ARGUMENT, "src and dst must be non-null");
    if(src_type != GSX_B200_DATA_U8 && src_type != GSX_B200_DATA_F32)
        return gsx_internal_fail(GSX_B200_NOT_SUPPORTED, "src_type must be GSX_B200_DATA_U8 or GSX_B200_DATA_F32");
    if(channels != 1 && channels != 3) return gsx_internal_fail(GSX_B200_INVALID_ARGUMENT, "channels must be 1 or 3");
    if(((uintptr_t)dst & 3u) != 0 || (src_type == GSX_B200_DATA_F32 && ((uintptr_t)src & 3u) != 0))
        return gsx_internal_fail(GSX_B200_INVALID_ARGUMENT, "f32 buffers must be 4-byte aligned");
    cudaStream_t stream = (cudaStream_t)stream_;
    /* planes 1 and 2 start 16-byte aligned only when the plane size is a multiple of 4 floats */
    const bool planes_ok = aligned16(dst) && (channels == 1 || pixel_count % 4 == 0);
    if(channels == 1 && src_type == GSX_B200_DATA_F32) {
        const cudaError_t e = cudaMemcpyAsync(dst, src, pixel_count * sizeof(float), cudaMemcpyDeviceToDevice, stream);
        return e == cudaSuccess ? GSX_B200_SUCCESS : gsx_internal_fail(GSX_B200_UNKNOWN, cudaGetErrorString(e));
    }
    if(channels == 1) {
        const bool vec = planes_ok && aligned16(src);
        plane_u8_kernel<<<grid_for((pixel_count + 15) / 16), kThreads, 0, stream>>>(static_cast<const uint8_t *>(src), dst,
                                                                                    pixel_count, vec);
    } else if(src_type == GSX_B200_DATA_U8) {
        const bool vec = planes_ok && aligned16(src);
        rgb_u8_kernel<<<grid_for((pixel_count + 15) / 16), kThreads, 0, stream>>>(static_cast<const uint8_t *>(src), dst,
                                                                                  pixel_count, vec);
    } else {
        const bool vec = planes_ok && aligned16(src);
        rgb_f32_kernel<<<grid_for((pixel_count + 3) / 4), kThreads, 0, stream>>>(static_cast<const float *>(src), dst,
                                                                                 pixel_count, vec);
    }
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? GSX_B200_SUCCESS : gsx_internal_fail(GSX_B200_UNKNOWN, cudaGetErrorString(e));
}
