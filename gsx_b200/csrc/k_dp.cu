/*
 * Data-parallel gradient exchange fused with Adam, over NVLink peer memory.
 *
 * The reference's multi-view training (one view per GPU) averages the per-view gradients with an
 * all-reduce and then runs Adam on every rank over every parameter (gsx-runtime.c:1413-1536 per rank;
 * the exchange is the data-parallel extension of that loop).  Here each rank owns one contiguous shard
 * of the flat parameter space and, in ONE kernel:
 *   - reads the shard's gradients from every rank's gradient buffer (peer loads over NVLink; its own
 *     from local memory) and averages them (sum in rank order, times 1/world),
 *   - applies Adam to the shard with shard-local moments (the moments are sharded: each rank keeps
 *     1/world of them),
 *   - stores the updated shard into every rank's parameter buffer (peer stores).
 * That is a reduce-scatter, the optimizer and an all-gather with no intermediate buffers: each rank
 * moves 2 (world-1)/world of the gradient bytes over NVLink in each direction (its stores plus the
 * replies to the other ranks' loads of its gradients), like a ring all-reduce, and runs Adam on
 * 1/world of the parameters instead of all of them.  Measured on two B200s: 168 MB per direction in
 * 0.255 ms, 660 GB/s per direction, at the link rate of a plain peer copy; issuing the stores through
 * the copy engines in pipelined chunks instead was slower (0.31-0.43 ms).  No waits inside the
 * kernel: the host orders it between two collectives (all ranks' backward done before; every rank's
 * parameters complete after).
 * The element update is gsx_adam_one, the same arithmetic as the single-GPU Adam kernel.
 */
#include "../../include/gsx_b200.h"
#include "gsx_b200_kernels.cuh"

#include <cstring>

int gsx_internal_fail(int code, const char *msg);

namespace {

constexpr int kThreads = 256;
constexpr int kChunk = 2048; /* elements per CTA */

struct DpTable {
    const float *grads[GSX_B200_DP_MAX_RANKS];
    float *params[GSX_B200_DP_MAX_RANKS];
    float *m1, *m2; /* shard-local, index = flat index - shard_begin */
    uint64_t shard_begin;
    int world, rank, count;
    float inv_world;
    AdamGroupDev g[GSX_B200_DP_MAX_SEGMENTS]; /* n = segment end, first_block = first CTA; param/grad unused */
    uint64_t begin[GSX_B200_DP_MAX_SEGMENTS];
};

template <int W>
__global__ void __launch_bounds__(kThreads) dp_adam_kernel(const __grid_constant__ DpTable t)
{
    int si = 0;
    while(si + 1 < t.count && (uint64_t)blockIdx.x >= t.g[si + 1].first_block) ++si;
    const AdamGroupDev &G = t.g[si];
    const uint64_t start = t.begin[si] + ((uint64_t)blockIdx.x - G.first_block) * kChunk;
    const uint64_t end = start + kChunk < G.n ? start + kChunk : G.n;
    const int world = W > 0 ? W : t.world;
    /* segment bounds are multiples of 4 elements and every buffer is 16-byte aligned */
    for(uint64_t i = start + 4 * (uint64_t)threadIdx.x; i < end; i += 4 * kThreads) {
        float4 gv[W > 0 ? W : GSX_B200_DP_MAX_RANKS];
#pragma unroll
        for(int r = 0; r < (W > 0 ? W : GSX_B200_DP_MAX_RANKS); ++r)
            if(r < world) gv[r] = *reinterpret_cast<const float4 *>(t.grads[r] + i);
        float4 g = gv[0];
#pragma unroll
        for(int r = 1; r < (W > 0 ? W : GSX_B200_DP_MAX_RANKS); ++r) {
            if(r < world) {
                g.x = __fadd_rn(g.x, gv[r].x);
                g.y = __fadd_rn(g.y, gv[r].y);
                g.z = __fadd_rn(g.z, gv[r].z);
                g.w = __fadd_rn(g.w, gv[r].w);
            }
        }
        g.x = __fmul_rn(g.x, t.inv_world);
        g.y = __fmul_rn(g.y, t.inv_world);
        g.z = __fmul_rn(g.z, t.inv_world);
        g.w = __fmul_rn(g.w, t.inv_world);
        const uint64_t j = i - t.shard_begin;
        float4 p = *reinterpret_cast<const float4 *>(t.params[t.rank] + i);
        float4 a = *reinterpret_cast<const float4 *>(t.m1 + j);
        float4 b = *reinterpret_cast<const float4 *>(t.m2 + j);
        p.x = gsx_adam_one(p.x, g.x, a.x, b.x, G);
        p.y = gsx_adam_one(p.y, g.y, a.y, b.y, G);
        p.z = gsx_adam_one(p.z, g.z, a.z, b.z, G);
        p.w = gsx_adam_one(p.w, g.w, a.w, b.w, G);
        *reinterpret_cast<float4 *>(t.m1 + j) = a;
        *reinterpret_cast<float4 *>(t.m2 + j) = b;
#pragma unroll
        for(int r = 0; r < (W > 0 ? W : GSX_B200_DP_MAX_RANKS); ++r)
            if(r < world) *reinterpret_cast<float4 *>(t.params[r] + i) = p;
    }
    /* no fence: the peer stores are complete when the kernel completes, and the host orders every
     * rank's next read of its parameters after that (a collective on each rank's stream); a
     * system-scope fence per thread here cost 40% of the kernel's time */
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

/* NVLink SHARP (NVLS) form of the same step.  mc_grads / mc_params are multicast addresses of the
 * ranks' flat gradient / parameter buffers (one NVSwitch multicast object each):
 * multimem.ld_reduce returns the sum of the element over every rank's buffer, reduced inside the
 * switch, and multimem.st writes one value into every rank's buffer.  Per rank and direction only the
 * shard's bytes cross NVLink (1/world of the gradients in, 1/world of the parameters out), instead of
 * 2 (world - 1)/world of them.  The switch's summation order is its own, so the average can differ from
 * the rank-order sum of the peer-load kernel by rounding; every rank still receives the one value its
 * owner computed, so the replicas stay identical. */
struct NvlsTable {
    const float *mc_grads;
    float *mc_params;
    const float *params; /* this rank's own parameter buffer (plain loads) */
    float *m1, *m2;
    uint64_t shard_begin;
    int count;
    float inv_world;
    AdamGroupDev g[GSX_B200_DP_MAX_SEGMENTS];
    uint64_t begin[GSX_B200_DP_MAX_SEGMENTS];
};

__device__ __forceinline__ float4 multimem_ld_reduce_add(const float *mc)
{
    float4 v;
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(mc)
                 : "memory");
    return v;
}

__device__ __forceinline__ void multimem_st(float *mc, float4 v)
{
    asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc), "f"(v.x), "f"(v.y), "f"(v.z),
                 "f"(v.w)
                 : "memory");
}

__global__ void __launch_bounds__(kThreads) dp_nvls_adam_kernel(const __grid_constant__ NvlsTable t)
{
    int si = 0;
    while(si + 1 < t.count && (uint64_t)blockIdx.x >= t.g[si + 1].first_block) ++si;
    const AdamGroupDev &G = t.g[si];
    const uint64_t start = t.begin[si] + ((uint64_t)blockIdx.x - G.first_block) * kChunk;
    const uint64_t end = start + kChunk < G.n ? start + kChunk : G.n;
    for(uint64_t i = start + 4 * (uint64_t)threadIdx.x; i < end; i += 4 * kThreads) {
        float4 g = multimem_ld_reduce_add(t.mc_grads + i);
        g.x = __fmul_rn(g.x, t.inv_world);
        g.y = __fmul_rn(g.y, t.inv_world);
        g.z = __fmul_rn(g.z, t.inv_world);
        g.w = __fmul_rn(g.w, t.inv_world);
        const uint64_t j = i - t.shard_begin;
        float4 p = *reinterpret_cast<const float4 *>(t.params + i);
        float4 a = *reinterpret_cast<const float4 *>(t.m1 + j);
        float4 b = *reinterpret_cast<const float4 *>(t.m2 + j);
        p.x = gsx_adam_one(p.x, g.x, a.x, b.x, G);
        p.y = gsx_adam_one(p.y, g.y, a.y, b.y, G);
        p.z = gsx_adam_one(p.z, g.z, a.z, b.z, G);
        p.w = gsx_adam_one(p.w, g.w, a.w, b.w, G);
        *reinterpret_cast<float4 *>(t.m1 + j) = a;
        *reinterpret_cast<float4 *>(t.m2 + j) = b;
        multimem_st(t.mc_params + i, p);
    }
}

/* segments -> per-segment Adam parameters and CTA ranges; returns the CTA count, or -1 on bad input */
int64_t fill_segments(AdamGroupDev *g, uint64_t *begin, int &count, uint64_t shard_begin, uint64_t shard_end,
                      const gsx_b200_dp_segment *segments, int n_segments)
{
    uint64_t blocks = 0;
    count = 0;
    for(int s = 0; s < n_segments; ++s) {
        const gsx_b200_dp_segment &S = segments[s];
        if(S.begin > S.end || S.begin < shard_begin || S.end > shard_end || S.begin % 4 != 0 || S.end % 4 != 0) return -1;
        if(S.end == S.begin) continue;
        AdamGroupDev &G = g[count];
        memset(&G, 0, sizeof(G));
        G.n = S.end;
        G.lr = S.learning_rate;
        G.beta1 = S.beta1;
        G.beta2 = S.beta2;
        G.eps = S.epsilon;
        G.weight_decay = S.weight_decay;
        G.max_grad = S.max_grad;
        G.inv_c1 = S.inv_bias_correction1;
        G.inv_c2 = S.inv_bias_correction2;
        G.first_block = blocks;
        begin[count] = S.begin;
        blocks += (S.end - S.begin + kChunk - 1) / kChunk;
        ++count;
    }
    return (int64_t)blocks;
}

} // namespace

extern "C" int gsx_b200_dp_nvls_reduce_adam_broadcast(int world, float *mc_params, const float *mc_grads,
                                                      const float *params, float *first_moment, float *second_moment,
                                                      uint64_t shard_begin, uint64_t shard_end,
                                                      const gsx_b200_dp_segment *segments, int n_segments, void *stream_)
{
    if(world < 1) return gsx_internal_fail(GSX_B200_OUT_OF_RANGE, "world must be positive");
    if(n_segments < 0 || n_segments > GSX_B200_DP_MAX_SEGMENTS)
        return gsx_internal_fail(GSX_B200_OUT_OF_RANGE, "n_segments must be in [0, GSX_B200_DP_MAX_SEGMENTS]");
    if(mc_params == nullptr || mc_grads == nullptr || params == nullptr ||
       (n_segments > 0 && (segments == nullptr || first_moment == nullptr || second_moment == nullptr)))
        return gsx_internal_fail(GSX_B200_INVALID_ARGUMENT, "multicast addresses, parameters, moments and segments must be non-null");
    if(!aligned16(mc_params) || !aligned16(mc_grads) || !aligned16(params) || !aligned16(first_moment) ||
       !aligned16(second_moment))
        return gsx_internal_fail(GSX_B200_INVALID_ARGUMENT, "buffers must be 16-byte aligned");
    if(shard_begin % 4 != 0 || shard_end < shard_begin)
        return gsx_internal_fail(GSX_B200_INVALID_ARGUMENT, "the shard must start on a multiple of 4 elements");
    NvlsTable t;
    memset(&t, 0, sizeof(t));
    t.mc_grads = mc_grads;
    t.mc_params = mc_params;
    t.params = params;
    t.m1 = first_moment;
    t.m2 = second_moment;
    t.shard_begin = shard_begin;
    t.inv_world = 1.0f / (float)world;
    const int64_t blocks = fill_segments(t.g, t.begin, t.count, shard_begin, shard_end, segments, n_segments);
    if(blocks < 0) return gsx_internal_fail(GSX_B200_INVALID_ARGUMENT, "segments must lie in the shard on multiples of 4 elements");
    if(blocks == 0) return GSX_B200_SUCCESS;
    dp_nvls_adam_kernel<<<(unsigned)blocks, kThreads, 0, (cudaStream_t)stream_>>>(t);
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? GSX_B200_SUCCESS : gsx_internal_fail(GSX_B200_UNKNOWN, cudaGetErrorString(e));
}

extern "C" int gsx_b200_dp_reduce_adam_gather(int world, int rank, float *const *params, const float *const *grads,
                                              float *first_moment, float *second_moment, uint64_t shard_begin,
                                              uint64_t shard_end, const gsx_b200_dp_segment *segments, int n_segments,
                                              void *stream_)
{
    if(world < 1 || world > GSX_B200_DP_MAX_RANKS || rank < 0 || rank >= world)
        return gsx_internal_fail(GSX_B200_OUT_OF_RANGE, "world must be in [1, GSX_B200_DP_MAX_RANKS] and 0 <= rank < world");
    if(n_segments < 0 || n_segments > GSX_B200_DP_MAX_SEGMENTS)
        return gsx_internal_fail(GSX_B200_OUT_OF_RANGE, "n_segments must be in [0, GSX_B200_DP_MAX_SEGMENTS]");
    if(params == nullptr || grads == nullptr || (n_segments > 0 && (segments == nullptr || first_moment == nullptr ||
                                                                    second_moment == nullptr)))
        return gsx_internal_fail(GSX_B200_INVALID_ARGUMENT, "pointer tables, moments and segments must be non-null");
    if(shard_begin % 4 != 0 || shard_end < shard_begin)
        return gsx_internal_fail(GSX_B200_INVALID_ARGUMENT, "the shard must start on a multiple of 4 elements");
    DpTable t;
    memset(&t, 0, sizeof(t));
    for(int r = 0; r < world; ++r) {
        if(params[r] == nullptr || grads[r] == nullptr || !aligned16(params[r]) || !aligned16(grads[r]))
            return gsx_internal_fail(GSX_B200_INVALID_ARGUMENT, "every rank's parameter and gradient buffer must be 16-byte aligned");
        t.params[r] = params[r];
        t.grads[r] = grads[r];
    }
    if(!aligned16(first_moment) || !aligned16(second_moment))
        return gsx_internal_fail(GSX_B200_INVALID_ARGUMENT, "moments must be 16-byte aligned");
    t.m1 = first_moment;
    t.m2 = second_moment;
    t.shard_begin = shard_begin;
    t.world = world;
    t.rank = rank;
    t.inv_world = 1.0f / (float)world;
    uint64_t blocks = 0;
    for(int s = 0; s < n_segments; ++s) {
        const gsx_b200_dp_segment &S = segments[s];
        if(S.begin > S.end || S.begin < shard_begin || S.end > shard_end || S.begin % 4 != 0 || S.end % 4 != 0)
            return gsx_internal_fail(GSX_B200_INVALID_ARGUMENT, "segments must lie in the shard on multiples of 4 elements");
        if(S.end == S.begin) continue;
        AdamGroupDev &G = t.g[t.count];
        G.n = S.end;
        G.lr = S.learning_rate;
        G.beta1 = S.beta1;
        G.beta2 = S.beta2;
        G.eps = S.epsilon;
        G.weight_decay = S.weight_decay;
        G.max_grad = S.max_grad;
        G.inv_c1 = S.inv_bias_correction1;
        G.inv_c2 = S.inv_bias_correction2;
        G.first_block = blocks;
        t.begin[t.count] = S.begin;
        blocks += (S.end - S.begin + kChunk - 1) / kChunk;
        ++t.count;
    }
    if(blocks == 0) return GSX_B200_SUCCESS;
    cudaStream_t stream = (cudaStream_t)stream_;
    switch(world) {
    case 1: dp_adam_kernel<1><<<(unsigned)blocks, kThreads, 0, stream>>>(t); break;
    case 2: dp_adam_kernel<2><<<(unsigned)blocks, kThreads, 0, stream>>>(t); break;
    case 4: dp_adam_kernel<4><<<(unsigned)blocks, kThreads, 0, stream>>>(t); break;
    case 8: dp_adam_kernel<8><<<(unsigned)blocks, kThreads, 0, stream>>>(t); break;
    default: dp_adam_kernel<0><<<(unsigned)blocks, kThreads, 0, stream>>>(t); break;
    }
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? GSX_B200_SUCCESS : gsx_internal_fail(GSX_B200_UNKNOWN, cudaGetErrorString(e));
}

extern "C" int gsx_b200_device_alloc(uint64_t bytes, void **out)
{
    if(out == nullptr) return gsx_internal_fail(GSX_B200_INVALID_ARGUMENT, "out must be non-null");
    *out = nullptr;
    const cudaError_t e = cudaMalloc(out, bytes ? bytes : 16);
    if(e == cudaErrorMemoryAllocation) return gsx_internal_fail(GSX_B200_OUT_OF_MEMORY, "cudaMalloc failed");
    if(e != cudaSuccess) return gsx_internal_fail(GSX_B200_UNKNOWN, cudaGetErrorString(e));
    return GSX_B200_SUCCESS;
}

extern "C" int gsx_b200_device_free(void *ptr)
{
    const cudaError_t e = cudaFree(ptr);
    return e == cudaSuccess ? GSX_B200_SUCCESS : gsx_internal_fail(GSX_B200_UNKNOWN, cudaGetErrorString(e));
}

extern "C" int gsx_b200_ipc_handle(void *base, void *out_handle)
{
    static_assert(sizeof(cudaIpcMemHandle_t) == GSX_B200_IPC_HANDLE_BYTES, "IPC handle size");
    if(base == nullptr || out_handle == nullptr) return gsx_internal_fail(GSX_B200_INVALID_ARGUMENT, "base and out_handle must be non-null");
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, base);
    if(e != cudaSuccess) return gsx_internal_fail(GSX_B200_UNKNOWN, cudaGetErrorString(e));
    memcpy(out_handle, &h, sizeof(h));
    return GSX_B200_SUCCESS;
}

extern "C" int gsx_b200_ipc_open(const void *handle, void **out)
{
    if(handle == nullptr || out == nullptr) return gsx_internal_fail(GSX_B200_INVALID_ARGUMENT, "handle and out must be non-null");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    const cudaError_t e = cudaIpcOpenMemHandle(out, h, cudaIpcMemLazyEnablePeerAccess);
    if(e != cudaSuccess) return gsx_internal_fail(GSX_B200_UNKNOWN, cudaGetErrorString(e));
    return GSX_B200_SUCCESS;
}

extern "C" int gsx_b200_ipc_close(void *ptr)
{
    const cudaError_t e = cudaIpcCloseMemHandle(ptr);
    return e == cudaSuccess ? GSX_B200_SUCCESS : gsx_internal_fail(GSX_B200_UNKNOWN, cudaGetErrorString(e));
}
