/*
 * Per-Gaussian preprocess: projection, EWA covariance, screen bounds, exact tile count, SH colour.
 *
 * Follows fastgs/kernels_forward.cuh:179-438 (preprocess_cu) for the projection, EWA covariance,
 * opacity-aware screen bounds and SH colour, and :109-175 for the exact tile count.  Differences
 * in structure (not in results):
 *   - no atomic compaction of visible primitives into the output: each CTA writes its primitives'
 *     tile counts and the totals of its 256-primitive blocks; a one-CTA scan over the block totals and
 *     the emission kernel's in-block scan turn them into exclusive offsets in primitive order, so
 *     emission is deterministic (the CTA's internal packing of cull survivors only picks which lane
 *     computes which primitive);
 *   - the [N,3] fields are staged through shared memory so every global load is a coalesced,
 *     contiguous warp access;
 *   - everything the later stages need is packed into one 48-byte PrimRec per primitive.
 * Compiled with -fmad=false: the arithmetic matches the oracle (oracle/gsx_oracle.c) bit for bit.
 */
#include "gsx_b200_kernels.cuh"

namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ int f2i_rd(float v)
{
    const float f = floorf(v);
    if(!(f == f)) return 0;
    if(f >= 2147483647.0f) return 2147483647;
    if(f <= -2147483648.0f) return (int)(-2147483647 - 1);
    return (int)f;
}

__device__ __forceinline__ int f2i_ru(float v)
{
    const float f = ceilf(v);
    if(!(f == f)) return 0;
    if(f >= 2147483647.0f) return 2147483647;
    if(f <= -2147483648.0f) return (int)(-2147483647 - 1);
    return (int)f;
}

__device__ __forceinline__ void sh_color(const float *__restrict__ sh0, const float *__restrict__ sh1,
                                         const float *__restrict__ sh2, const float *__restrict__ sh3, const float m[3],
                                         const float cam[3], int64_t i, int bases, float out[3])
{
#pragma unroll
    for(int c = 0; c < 3; ++c) out[c] = 0.5f + 0.28209479177387814f * sh0[i * 3 + c];
    if(bases > 1) {
        const float dx = m[0] - cam[0], dy = m[1] - cam[1], dz = m[2] - cam[2];
        const float inv = 1.0f / sqrtf(dx * dx + dy * dy + dz * dz);
        const float x = dx * inv, y = dy * inv, z = dz * inv;
        const float *c1 = sh1 + i * 9;
        for(int c = 0; c < 3; ++c) {
            out[c] = out[c] + (-0.48860251190291987f * y) * c1[0 * 3 + c] + (0.48860251190291987f * z) * c1[1 * 3 + c]
                + (-0.48860251190291987f * x) * c1[2 * 3 + c];
        }
        if(bases > 4) {
            const float xx = x * x, yy = y * y, zz = z * z, xy = x * y, xz = x * z, yz = y * z;
            const float *c2 = sh2 + i * 15;
            for(int c = 0; c < 3; ++c) {
                out[c] = out[c] + (1.0925484305920792f * xy) * c2[0 * 3 + c] + (-1.0925484305920792f * yz) * c2[1 * 3 + c]
                    + (0.94617469575755997f * zz - 0.31539156525251999f) * c2[2 * 3 + c]
                    + (-1.0925484305920792f * xz) * c2[3 * 3 + c]
                    + (0.54627421529603959f * xx - 0.54627421529603959f * yy) * c2[4 * 3 + c];
            }
            if(bases > 9) {
                const float *c3 = sh3 + i * 21;
                for(int c = 0; c < 3; ++c) {
                    out[c] = out[c] + (0.59004358992664352f * y * (-3.0f * xx + yy)) * c3[0 * 3 + c]
                        + (2.8906114426405538f * xy * z) * c3[1 * 3 + c]
                        + (0.45704579946446572f * y * (1.0f - 5.0f * zz)) * c3[2 * 3 + c]
                        + (0.3731763325901154f * z * (5.0f * zz - 3.0f)) * c3[3 * 3 + c]
                        + (0.45704579946446572f * x * (1.0f - 5.0f * zz)) * c3[4 * 3 + c]
                        + (1.4453057213202769f * z * (xx - yy)) * c3[5 * 3 + c]
                        + (0.59004358992664352f * x * (-xx + 3.0f * yy)) * c3[6 * 3 + c];
                }
            }
        }
    }
}

/* Gaussians per CTA: kGroup blocks of kThreads.  A CTA stages its rows, runs a cheap conservative
 * screen cull over all of them and packs the survivors, then runs the full path in rounds of
 * kThreads survivors: off-screen Gaussians (42-52% in the benchmark views, 80-90% for a quarter-frame
 * band) cost the cull only, and the full path runs on dense warps.  Each warp's full path is a long
 * dependent chain, so the CTA's duration is the number of rounds, not the number of live lanes.
 * 1024 Gaussians per CTA (26 KB of staging) and 48 registers let 5 CTAs share an SM; 2048 per CTA
 * (53 KB) held 4: config-3 preprocess 0.144 -> 0.137 ms. */
constexpr int kGroup = 4;
constexpr int kRows = kThreads * kGroup;
static_assert((kRows * 3) % (4 * kThreads) == 0, "16-byte staging chunks split evenly over the threads");

/* 16-byte global -> shared copy; bytes < 16 reads that many and zero-fills the rest */
__device__ __forceinline__ void cp_async16_zfill(void *smem, const void *gmem, unsigned bytes)
{
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.ca.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem), "r"(bytes) : "memory");
}

struct PrepSmem {
    float m[kRows * 3];
    float s[kRows * 3];
    uint16_t list[kRows];
    uint32_t bsum[kGroup];
    uint32_t warp_sum[kThreads / 32];
    int nsurv;
};

__global__ void __launch_bounds__(kThreads, 5) preprocess_kernel(
    const float *__restrict__ mean3d, const float *__restrict__ rotation, const float *__restrict__ logscale,
    const float *__restrict__ opacity_raw, const float *__restrict__ sh0, const float *__restrict__ sh1,
    const float *__restrict__ sh2, const float *__restrict__ sh3, int bases, int64_t n, CameraParams cam,
    PrimRec *__restrict__ rec, uint32_t *__restrict__ counts, uint32_t *__restrict__ tile_masks,
    uint32_t *__restrict__ block_sums, int64_t n_blocks, float *__restrict__ vis_counter, float *__restrict__ max_radius)
{
    gsx_pdl_trigger(); /* the block-total scan may launch once every CTA has started */
    extern __shared__ __align__(16) unsigned char smem_raw[];
    PrepSmem &S = *reinterpret_cast<PrepSmem *>(smem_raw);
    float *const s_m = S.m;
    float *const s_s = S.s;
    const int lane = threadIdx.x & 31;
    const int64_t base = (int64_t)blockIdx.x * kRows;
    {
        /* staging of the CTA's [kRows,3] mean and log-scale rows: 16-byte asynchronous copies, all in
         * flight at once (a load-then-store loop waits out one memory latency per iteration); the
         * copy past the end of the arrays is zero-filled.  Unaligned arrays take the plain loop. */
        const int64_t avail = (n - base) * 3;
        const float *gm = mean3d + base * 3, *gs = logscale + base * 3;
        if(((reinterpret_cast<uintptr_t>(mean3d) | reinterpret_cast<uintptr_t>(logscale)) & 15u) == 0) {
#pragma unroll
            for(int q = 0; q < kRows * 3 / 4 / kThreads; ++q) {
                const int c = q * kThreads + (int)threadIdx.x; /* 16-byte chunk */
                const int64_t left = avail - 4 * (int64_t)c;
                const unsigned bytes = left >= 4 ? 16u : left > 0 ? (unsigned)left * 4u : 0u;
                cp_async16_zfill(s_m + 4 * c, bytes ? gm + 4 * c : mean3d, bytes);
                cp_async16_zfill(s_s + 4 * c, bytes ? gs + 4 * c : logscale, bytes);
            }
            asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
        } else {
            for(int j = threadIdx.x; j < kRows * 3; j += kThreads) {
                const bool ok = j < avail;
                s_m[j] = ok ? mean3d[base * 3 + j] : 0.0f;
                s_s[j] = ok ? logscale[base * 3 + j] : 0.0f;
            }
        }
        if(threadIdx.x < kGroup) S.bsum[threadIdx.x] = 0u;
        if(threadIdx.x == 0) S.nsurv = 0;
        __syncthreads();
    }
    /* conservative screen cull: the largest footprint the full path could give (3.34 sigma of the
     * largest scale through the steepest clamped Jacobian, with the dilation, 1% and 2 px of margin;
     * approximate arithmetic is fine inside the margin) missing the frame's columns or the band's rows
     * means no tile: count 0 and mask 0, the full path's outputs.  Gaussians it keeps go through the
     * unchanged full path. */
    {
        const float *w = cam.w2c;
        const float xmax = (float)(GSX_TILE * cam.grid_w);
        const float ytop = (float)(GSX_TILE * cam.trow0), ybot = (float)(GSX_TILE * (cam.trow0 + cam.grid_h));
#pragma unroll 1
        for(int k = 0; k < kGroup; ++k) {
            const int r = k * kThreads + (int)threadIdx.x;
            const int64_t i0 = base + r;
            if(i0 >= n) continue;
            const float mx = s_m[r * 3 + 0], my = s_m[r * 3 + 1], mz = s_m[r * 3 + 2];
            const float d = w[8] * mx + w[9] * my + w[10] * mz + w[11];
            bool keep = !(d < cam.near_plane || d > cam.far_plane);
            if(keep) {
                const float inv = __frcp_rn(d);
                const float cxp = (w[0] * mx + w[1] * my + w[2] * mz + w[3]) * inv * cam.fx + cam.cx;
                const float cyp = (w[4] * mx + w[5] * my + w[6] * mz + w[7]) * inv * cam.fy + cam.cy;
                const float ls = fmaxf(fmaxf(s_s[r * 3 + 0], s_s[r * 3 + 1]), s_s[r * 3 + 2]);
                const float var = __expf(2.0f * ls) * 1.01f;
                const float j1 = cam.fx * inv, j2 = cam.fy * inv;
                const float rx = 3.34f * sqrtf(j1 * j1 * cam.cull_jx * var + 0.31f) + 2.0f;
                const float ry = 3.34f * sqrtf(j2 * j2 * cam.cull_jy * var + 0.31f) + 2.0f;
                if(cxp + rx < 0.0f || cxp - rx > xmax || cyp + ry < ytop || cyp - ry > ybot) keep = false;
            }
            if(keep) {
                S.list[atomicAdd(&S.nsurv, 1)] = (uint16_t)r;
            } else {
                counts[i0] = 0u;
                tile_masks[i0] = 0u;
            }
        }
        __syncthreads();
    }
    const int nsurv = S.nsurv;
#pragma unroll 1
    for(int round = 0; round * kThreads < nsurv; ++round) {
    const int idx = round * kThreads + (int)threadIdx.x;
    const bool has = idx < nsurv;
    const int li = has ? (int)S.list[idx] : 0; /* this lane's row in the CTA */
    const int64_t i = base + li;
    bool active = has;
    float m[3] = { 0.0f, 0.0f, 0.0f };
    float depth = 0.0f, op = 0.0f, m2x = 0.0f, m2y = 0.0f, conx = 0.0f, cony = 0.0f, conz = 0.0f, pt = 0.0f;
    unsigned bx0 = 0, bx1 = 0, by0 = 0, by1 = 0;
    float srad = 0.0f;
    const float *w = cam.w2c;
    if(active) {
        m[0] = s_m[li * 3 + 0];
        m[1] = s_m[li * 3 + 1];
        m[2] = s_m[li * 3 + 2];
        depth = w[8] * m[0] + w[9] * m[1] + w[10] * m[2] + w[11];
        if(depth < cam.near_plane || depth > cam.far_plane) active = false;
    }
    if(active) {
        op = gsx_sigmoidf(opacity_raw[i]);
        if(op < 1.0f / 255.0f) active = false;
    }
    if(active) {
        float var[3];
#pragma unroll
        for(int k = 0; k < 3; ++k) {
            const float s = gsx_expf(s_s[li * 3 + k]);
            var[k] = s * s;
        }
        const float4 q = *reinterpret_cast<const float4 *>(rotation + i * 4);
        const float qx = q.x, qy = q.y, qz = q.z, qr = q.w;
        const float qrr = qr * qr, qxx_raw = qx * qx, qyy_raw = qy * qy, qzz_raw = qz * qz;
        const float qn = qrr + qxx_raw + qyy_raw + qzz_raw;
        if(qn < 1e-8f) {
            active = false;
        } else {
            const float qxx = 2.0f * qxx_raw / qn, qyy = 2.0f * qyy_raw / qn, qzz = 2.0f * qzz_raw / qn;
            const float qxy = 2.0f * qx * qy / qn, qxz = 2.0f * qx * qz / qn, qyz = 2.0f * qy * qz / qn;
            const float qrx = 2.0f * qr * qx / qn, qry = 2.0f * qr * qy / qn, qrz = 2.0f * qr * qz / qn;
            const float R[9] = { 1.0f - (qyy + qzz), qxy - qrz, qry + qxz,
                                 qrz + qxy, 1.0f - (qxx + qzz), qyz - qrx,
                                 qxz - qry, qrx + qyz, 1.0f - (qxx + qyy) };
            const float RS[9] = { R[0] * var[0], R[1] * var[1], R[2] * var[2],
                                  R[3] * var[0], R[4] * var[1], R[5] * var[2],
                                  R[6] * var[0], R[7] * var[1], R[8] * var[2] };
            const float c11 = RS[0] * R[0] + RS[1] * R[1] + RS[2] * R[2];
            const float c12 = RS[0] * R[3] + RS[1] * R[4] + RS[2] * R[5];
            const float c13 = RS[0] * R[6] + RS[1] * R[7] + RS[2] * R[8];
            const float c22 = RS[3] * R[3] + RS[4] * R[4] + RS[5] * R[5];
            const float c23 = RS[3] * R[6] + RS[4] * R[7] + RS[5] * R[8];
            const float c33 = RS[6] * R[6] + RS[7] * R[7] + RS[8] * R[8];
            const float x = (w[0] * m[0] + w[1] * m[1] + w[2] * m[2] + w[3]) / depth;
            const float y = (w[4] * m[0] + w[5] * m[1] + w[6] * m[2] + w[7]) / depth;
            const float clip_l = cam.clip_l, clip_r = cam.clip_r, clip_t = cam.clip_t, clip_b = cam.clip_b;
            const float tx = fmaxf(clip_l, fminf(x, clip_r));
            const float ty = fmaxf(clip_t, fminf(y, clip_b));
            const float j11 = cam.fx / depth, j13 = -j11 * tx, j22 = cam.fy / depth, j23 = -j22 * ty;
            const float a1x = j11 * w[0] + j13 * w[8], a1y = j11 * w[1] + j13 * w[9], a1z = j11 * w[2] + j13 * w[10];
            const float a2x = j22 * w[4] + j23 * w[8], a2y = j22 * w[5] + j23 * w[9], a2z = j22 * w[6] + j23 * w[10];
            const float b1x = a1x * c11 + a1y * c12 + a1z * c13, b1y = a1x * c12 + a1y * c22 + a1z * c23,
                        b1z = a1x * c13 + a1y * c23 + a1z * c33;
            const float b2x = a2x * c11 + a2y * c12 + a2z * c13, b2y = a2x * c12 + a2y * c22 + a2z * c23,
                        b2z = a2x * c13 + a2y * c23 + a2z * c33;
            float cov_x = b1x * a1x + b1y * a1y + b1z * a1z;
            const float cov_y = b1x * a2x + b1y * a2y + b1z * a2z;
            float cov_z = b2x * a2x + b2y * a2y + b2z * a2z;
            cov_x += 0.3f;
            cov_z += 0.3f;
            const float det = cov_x * cov_z - cov_y * cov_y;
            if(det < 1e-8f) {
                active = false;
            } else {
                if(max_radius != nullptr) {
                    /* screen radius of gsx-metal/kernels/render.metal:432-438: 3 sigma of the larger
                     * eigenvalue of the dilated 2-D covariance, rounded up */
                    const float mid = 0.5f * (cov_x + cov_z);
                    const float disc = sqrtf(fmaxf(0.1f, mid * mid - det));
                    srad = ceilf(3.0f * sqrtf(fmaxf(mid + disc, mid - disc)));
                }
                conx = cov_z / det;
                cony = -cov_y / det;
                conz = cov_x / det;
                m2x = x * cam.fx + cam.cx;
                m2y = y * cam.fy + cam.cy;
                pt = gsx_logf(op * 255.0f);
                const float ptf = sqrtf(2.0f * pt);
                const float ex = fmaxf(ptf * sqrtf(cov_x) - 0.5f, 0.0f);
                const float ey = fmaxf(ptf * sqrtf(cov_z) - 0.5f, 0.0f);
                const unsigned gw = (unsigned)cam.grid_w, gh = (unsigned)cam.grid_h;
                int v;
                v = f2i_rd((m2x - ex) / 16.0f); bx0 = (unsigned)(v > 0 ? v : 0); bx0 = bx0 > gw ? gw : bx0;
                v = f2i_ru((m2x + ex) / 16.0f); bx1 = (unsigned)(v > 0 ? v : 0); bx1 = bx1 > gw ? gw : bx1;
                /* tile rows in full-frame units clamped to the band [trow0, trow0 + gh), stored band-relative */
                const int t0 = cam.trow0, t1 = cam.trow0 + (int)gh;
                v = f2i_rd((m2y - ey) / 16.0f); v = v < t0 ? t0 : (v > t1 ? t1 : v); by0 = (unsigned)(v - t0);
                v = f2i_ru((m2y + ey) / 16.0f); v = v < t0 ? t0 : (v > t1 ? t1 : v); by1 = (unsigned)(v - t0);
                if((bx1 - bx0) * (by1 - by0) == 0) active = false;
            }
        }
    }

    /* exact tile count: the first GSX_SEQ_TILES tiles of the rectangle per thread, the rest
     * warp-cooperatively (all lanes converged here; no early return above). */
    const unsigned bw = bx1 - bx0;
    const unsigned tmax = active ? bw * (by1 - by0) : 0u;
    const float msx = m2x - 0.5f, msy = m2y - 0.5f;
    unsigned cnt = 0, tmask = 0;
    const unsigned nseq = tmax < GSX_SEQ_TILES ? tmax : GSX_SEQ_TILES;
    for(unsigned k = 0; k < nseq; ++k) {
        if(gsx_tile_contributes(msx, msy, conx, cony, conz, bx0 + k % bw, (unsigned)cam.trow0 + by0 + k / bw, pt)) {
            ++cnt;
            tmask |= 1u << k;
        }
    }
    unsigned coop = __ballot_sync(0xffffffffu, tmax > GSX_SEQ_TILES);
    while(coop) {
        const int L = __ffs(coop) - 1;
        coop &= coop - 1u;
        const unsigned lbx0 = __shfl_sync(0xffffffffu, bx0, L), lbw = __shfl_sync(0xffffffffu, bw, L);
        const unsigned lby0 = __shfl_sync(0xffffffffu, by0, L), ltmax = __shfl_sync(0xffffffffu, tmax, L);
        const float lmx = __shfl_sync(0xffffffffu, msx, L), lmy = __shfl_sync(0xffffffffu, msy, L);
        const float lcx = __shfl_sync(0xffffffffu, conx, L), lcy = __shfl_sync(0xffffffffu, cony, L);
        const float lcz = __shfl_sync(0xffffffffu, conz, L), lpt = __shfl_sync(0xffffffffu, pt, L);
        unsigned sum = 0, first = 0;
        for(unsigned base = GSX_SEQ_TILES; base < ltmax; base += 32u) {
            const unsigned k = base + (unsigned)lane;
            const bool c = k < ltmax && gsx_tile_contributes(lmx, lmy, lcx, lcy, lcz, lbx0 + k % lbw,
                                                             (unsigned)cam.trow0 + lby0 + k / lbw, lpt);
            const unsigned b = __ballot_sync(0xffffffffu, c);
            if(base == GSX_SEQ_TILES) first = b;
            sum += (unsigned)__popc(b);
        }
        if(lane == L) {
            cnt += sum;
            if(ltmax <= 32u) tmask |= first << GSX_SEQ_TILES;
        }
    }
    if(cnt == 0) active = false;

    if(active) {
        float col[3];
        sh_color(sh0, sh1, sh2, sh3, m, cam.cam_pos, i, bases, col);
        PrimRec r;
        r.a = make_float4(m2x, m2y, conx, cony);
        r.b = make_float4(conz, op, col[0], col[1]);
        r.c = make_float4(col[2], depth, __uint_as_float(bx0 | (bx1 << 16)), __uint_as_float(by0 | (by1 << 16)));
        rec[i] = r;
        /* TRAIN auxiliary accumulators of a visible (tile-touching) Gaussian,
         * gsx-metal/kernels/render.metal:425-439 */
        if(vis_counter != nullptr) vis_counter[i] += 1.0f;
        if(max_radius != nullptr) max_radius[i] = fmaxf(max_radius[i], srad);
    }

    if(has) {
        counts[i] = cnt;
        tile_masks[i] = tmask;
        if(cnt) atomicAdd(&S.bsum[li / kThreads], cnt);
    }
    } /* rounds */
    __syncthreads();
    /* totals of the 256-Gaussian blocks the emission kernel scans */
    if(threadIdx.x < kGroup) {
        const int64_t b = (int64_t)blockIdx.x * kGroup + threadIdx.x;
        if(b < n_blocks) block_sums[b] = S.bsum[threadIdx.x];
    }
    (void)lane;
}

/* exclusive scan of the per-block totals (one CTA); block_sums[nb] receives the grand total.
 * The totals are walked in chunks of 4096: every thread reads and writes 4 consecutive words (one
 * coalesced 16-byte access per warp lane), and the next chunk's load is in flight while the current
 * chunk is scanned.  (Giving each thread its own contiguous run of nb/1024 totals made every load of a
 * warp touch 32 cache lines, one dependent round trip per element: 0.1 ms at 39k blocks.) */
__device__ __forceinline__ uint4 load_chunk(const uint32_t *__restrict__ p, int idx, int nb)
{
    if(idx + 3 < nb) return *reinterpret_cast<const uint4 *>(p + idx);
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if(idx < nb) v.x = p[idx];
    if(idx + 1 < nb) v.y = p[idx + 1];
    if(idx + 2 < nb) v.z = p[idx + 2];
    return v;
}

__global__ void __launch_bounds__(1024) block_scan_kernel(uint32_t *__restrict__ block_sums, int nb)
{
    gsx_pdl_wait();
    gsx_pdl_trigger();
    __shared__ uint32_t s_w[2][32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    constexpr int kChunk = 4 * 1024;
    const bool vec = (reinterpret_cast<uintptr_t>(block_sums) & 15u) == 0;
    uint32_t carry = 0;
    int idx = 4 * (int)threadIdx.x;
    uint4 v = idx < nb ? (vec ? load_chunk(block_sums, idx, nb)
                              : make_uint4(block_sums[idx], idx + 1 < nb ? block_sums[idx + 1] : 0u,
                                           idx + 2 < nb ? block_sums[idx + 2] : 0u, idx + 3 < nb ? block_sums[idx + 3] : 0u))
                       : make_uint4(0u, 0u, 0u, 0u);
    for(int base = 0, it = 0; base < nb; base += kChunk, ++it) {
        const uint4 cur = v;
        const int nidx = idx + kChunk;
        if(nidx < nb)
            v = vec ? load_chunk(block_sums, nidx, nb)
                    : make_uint4(block_sums[nidx], nidx + 1 < nb ? block_sums[nidx + 1] : 0u,
                                 nidx + 2 < nb ? block_sums[nidx + 2] : 0u, nidx + 3 < nb ? block_sums[nidx + 3] : 0u);
        else
            v = make_uint4(0u, 0u, 0u, 0u); /* past the end: adds nothing to the next chunk's total */
        const uint32_t local = cur.x + cur.y + cur.z + cur.w;
        uint32_t incl = local;
#pragma unroll
        for(int d = 1; d < 32; d <<= 1) {
            const uint32_t t = __shfl_up_sync(0xffffffffu, incl, d);
            if(lane >= d) incl += t;
        }
        uint32_t *const w = s_w[it & 1]; /* alternating buffers: one barrier per chunk */
        if(lane == 31) w[warp] = incl;
        __syncthreads();
        uint32_t woff = 0, tot = 0;
#pragma unroll 8
        for(int k = 0; k < 32; ++k) {
            const uint32_t x = w[k];
            woff += k < warp ? x : 0u;
            tot += x;
        }
        const uint32_t e0 = carry + woff + incl - local;
        const uint4 out = make_uint4(e0, e0 + cur.x, e0 + cur.x + cur.y, e0 + cur.x + cur.y + cur.z);
        if(vec && idx + 3 < nb) {
            *reinterpret_cast<uint4 *>(block_sums + idx) = out;
        } else {
            if(idx < nb) block_sums[idx] = out.x;
            if(idx + 1 < nb) block_sums[idx + 1] = out.y;
            if(idx + 2 < nb) block_sums[idx + 2] = out.z;
            if(idx + 3 < nb) block_sums[idx + 3] = out.w;
        }
        carry += tot;
        idx = nidx;
    }
    if(threadIdx.x == 0) block_sums[nb] = carry;
}

} // namespace

namespace {

/* Per tile row of the full frame, an estimate of the instances it will hold: every Gaussian that the
 * preprocess's conservative screen cull keeps adds the number of tile columns of its cull rectangle to
 * each tile row the rectangle covers (integer atomics, so every rank that computes it gets the same
 * array).  The frame split of large-frame inference cuts the rows where the running sum crosses
 * k/world of the total, so the bands carry about equal work. */
constexpr int kCostRows = 1024;

__global__ void __launch_bounds__(kThreads) band_cost_kernel(const float *__restrict__ mean3d,
                                                             const float *__restrict__ logscale, int64_t n,
                                                             CameraParams cam, uint32_t *__restrict__ row_cost)
{
    __shared__ uint32_t s_cost[kCostRows];
    const int rows = cam.grid_h;
    for(int r = threadIdx.x; r < rows; r += kThreads) s_cost[r] = 0u;
    __syncthreads();
    const float *w = cam.w2c;
    for(int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < n; i += (int64_t)gridDim.x * kThreads) {
        const float mx = mean3d[i * 3 + 0], my = mean3d[i * 3 + 1], mz = mean3d[i * 3 + 2];
        const float d = w[8] * mx + w[9] * my + w[10] * mz + w[11];
        if(d < cam.near_plane || d > cam.far_plane) continue;
        const float inv = __frcp_rn(d);
        const float cxp = (w[0] * mx + w[1] * my + w[2] * mz + w[3]) * inv * cam.fx + cam.cx;
        const float cyp = (w[4] * mx + w[5] * my + w[6] * mz + w[7]) * inv * cam.fy + cam.cy;
        const float ls = fmaxf(fmaxf(logscale[i * 3 + 0], logscale[i * 3 + 1]), logscale[i * 3 + 2]);
        const float var = __expf(2.0f * ls) * 1.01f;
        const float j1 = cam.fx * inv, j2 = cam.fy * inv;
        const float rx = 3.34f * sqrtf(j1 * j1 * cam.cull_jx * var + 0.31f) + 2.0f;
        const float ry = 3.34f * sqrtf(j2 * j2 * cam.cull_jy * var + 0.31f) + 2.0f;
        const int x0 = max(0, (int)floorf((cxp - rx) * (1.0f / GSX_TILE)));
        const int x1 = min(cam.grid_w - 1, (int)floorf((cxp + rx) * (1.0f / GSX_TILE)));
        const int y0 = max(0, (int)floorf((cyp - ry) * (1.0f / GSX_TILE)));
        const int y1 = min(rows - 1, (int)floorf((cyp + ry) * (1.0f / GSX_TILE)));
        if(x1 < x0 || y1 < y0) continue;
        for(int r = y0; r <= y1; ++r) atomicAdd(&s_cost[r], (uint32_t)(x1 - x0 + 1));
    }
    __syncthreads();
    for(int r = threadIdx.x; r < rows; r += kThreads)
        if(s_cost[r]) atomicAdd(&row_cost[r], s_cost[r]);
}

} // namespace

cudaError_t gsx_launch_band_cost(const float *mean3d, const float *logscale, int64_t n, const CameraParams &cam,
                                 uint32_t *row_cost, cudaStream_t stream)
{
    if(cam.grid_h > kCostRows) return cudaErrorInvalidValue;
    cudaError_t e = cudaMemsetAsync(row_cost, 0, sizeof(uint32_t) * (size_t)cam.grid_h, stream);
    if(e != cudaSuccess || n == 0) return e;
    int64_t blocks = (n + kThreads - 1) / kThreads;
    if(blocks > 148 * 8) blocks = 148 * 8;
    band_cost_kernel<<<(unsigned)blocks, kThreads, 0, stream>>>(mean3d, logscale, n, cam, row_cost);
    return cudaGetLastError();
}

cudaError_t gsx_launch_preprocess(const float *mean3d, const float *rotation, const float *logscale,
                                  const float *opacity, const float *sh0, const float *sh1, const float *sh2,
                                  const float *sh3, int sh_degree, int64_t n, const CameraParams &cam, PrimRec *rec,
                                  uint32_t *counts, uint32_t *tile_masks, uint32_t *block_sums, float *visible_counter,
                                  float *max_screen_radius, cudaStream_t stream)
{
    if(n <= 0) return cudaSuccess;
    const int64_t blocks = (n + kThreads - 1) / kThreads;
    const int64_t ctas = (n + kRows - 1) / kRows;
    static bool attr_done[256];
    int dev = 0;
    cudaError_t err = cudaGetDevice(&dev);
    if(err != cudaSuccess) return err;
    if(dev < 0 || dev >= 256 || !attr_done[dev]) {
        err = cudaFuncSetAttribute(preprocess_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(PrepSmem));
        if(err != cudaSuccess) return err;
        if(dev >= 0 && dev < 256) attr_done[dev] = true;
    }
    preprocess_kernel<<<(unsigned)ctas, kThreads, sizeof(PrepSmem), stream>>>(
        mean3d, rotation, logscale, opacity, sh0, sh1, sh2, sh3, (sh_degree + 1) * (sh_degree + 1), n, cam, rec, counts,
        tile_masks, block_sums, blocks, visible_counter, max_screen_radius);
    cudaError_t e = cudaGetLastError();
    if(e != cudaSuccess) return e;
    return gsx_launch_pdl(block_scan_kernel, dim3(1), dim3(1024), 0, stream, block_sums, (int)blocks);
}
