/*
 * Single-launch Adam over every parameter group (all GSX parameter roles in one kernel).
 *
 * Per-element arithmetic follows gsx-cuda/gsx-cuda-kernels.cu:279-321 exactly (optional gradient
 * clamp, fp32 moments, fp64 multiply by the host-computed 1/(1-beta^t) of gsx-cuda/optim.c:776-793,
 * decoupled weight decay applied only when > 0, p -= lr * m_hat / (sqrt(v_hat) + eps)).  The
 * reference launches one kernel per group (optim.c:746-803); here a table of up to 16 groups
 * travels in the kernel parameters and each 4096-element chunk of the concatenated index space is
 * one CTA, using 16-byte vector loads and stores where the group is 16-byte aligned.
 * Compiled with -fmad=false so results are bit-identical to the reference formula and the oracle.
 */
#include "gsx_b200_kernels.cuh"

namespace {

constexpr int kThreads = 256;
constexpr int kChunk = 4096;

__global__ void __launch_bounds__(kThreads) adam_kernel(const __grid_constant__ AdamTable table)
{
    int gi = 0;
    while(gi + 1 < table.count && (uint64_t)blockIdx.x >= table.g[gi + 1].first_block) ++gi;
    const AdamGroupDev &G = table.g[gi];
    const uint64_t start = ((uint64_t)blockIdx.x - G.first_block) * kChunk;
    const uint64_t end = start + kChunk < G.n ? start + kChunk : G.n;
    const bool vec = ((reinterpret_cast<uintptr_t>(G.param) | reinterpret_cast<uintptr_t>(G.grad) |
                       reinterpret_cast<uintptr_t>(G.m1) | reinterpret_cast<uintptr_t>(G.m2)) & 15u) == 0;
    if(vec) {
        const uint64_t vend = start + ((end - start) & ~(uint64_t)3);
        for(uint64_t i = start + 4 * threadIdx.x; i < vend; i += 4 * kThreads) {
            float4 p = *reinterpret_cast<const float4 *>(G.param + i);
            const float4 g = __ldcs(reinterpret_cast<const float4 *>(G.grad + i));
            float4 a = *reinterpret_cast<const float4 *>(G.m1 + i);
            float4 b = *reinterpret_cast<const float4 *>(G.m2 + i);
            p.x = gsx_adam_one(p.x, g.x, a.x, b.x, G);
            p.y = gsx_adam_one(p.y, g.y, a.y, b.y, G);
            p.z = gsx_adam_one(p.z, g.z, a.z, b.z, G);
            p.w = gsx_adam_one(p.w, g.w, a.w, b.w, G);
            *reinterpret_cast<float4 *>(G.param + i) = p;
            *reinterpret_cast<float4 *>(G.m1 + i) = a;
            *reinterpret_cast<float4 *>(G.m2 + i) = b;
        }
        for(uint64_t i = vend + threadIdx.x; i < end; i += kThreads) {
            float a = G.m1[i], b = G.m2[i];
            G.param[i] = gsx_adam_one(G.param[i], G.grad[i], a, b, G);
            G.m1[i] = a;
            G.m2[i] = b;
        }
    } else {
        for(uint64_t i = start + threadIdx.x; i < end; i += kThreads) {
            float a = G.m1[i], b = G.m2[i];
            G.param[i] = gsx_adam_one(G.param[i], G.grad[i], a, b, G);
            G.m1[i] = a;
            G.m2[i] = b;
        }
    }
}

} // namespace

cudaError_t gsx_launch_adam(AdamTable &table, cudaStream_t stream)
{
    uint64_t blocks = 0;
    int live = 0;
    AdamTable t = table;
    t.count = 0;
    for(int i = 0; i < table.count; ++i) {
        if(table.g[i].n == 0) continue;
        t.g[live] = table.g[i];
        t.g[live].first_block = blocks;
        blocks += (table.g[i].n + kChunk - 1) / kChunk;
        ++live;
    }
    t.count = live;
    if(blocks == 0) return cudaSuccess;
    if(blocks > 0x7fffffffull) return cudaErrorInvalidValue;
    adam_kernel<<<(unsigned)blocks, kThreads, 0, stream>>>(t);
    return cudaGetLastError();
}
