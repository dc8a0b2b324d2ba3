/*
 * Per-Gaussian backward through the projection: 2-D gradients (mean2d, conic, raw opacity,
 * colour) to the GSX parameter gradients (mean3d, rotation xyzw, logscale, opacity, SH).
 *
 * Follows fastgs/kernels_backward.cuh:127-422 (preprocess_backward_cu: conic -> cov2d -> cov3d ->
 * (scale, quaternion) and mean3d, with the frustum-clamp mask on the Jacobian) and :40-125 (SH
 * colour backward).  Every primitive's gradients are written with `=` (0 for culled ones), so the
 * caller's gradient tensors need no zeroing beforehand (the reference zeroes them first and
 * accumulates, render.c:1459-1516).  The 2-D accumulators are reset to zero after being read, so
 * the next backward starts clean without a memset.
 */
#include "gsx_b200_kernels.cuh"

namespace {

constexpr int kThreads = 256;

__global__ void __launch_bounds__(kThreads, 4) preprocess_backward_kernel(
    const float *__restrict__ mean3d, const float *__restrict__ rotation, const float *__restrict__ logscale,
    const float *__restrict__ sh1, const float *__restrict__ sh2, const float *__restrict__ sh3, int bases, int64_t n,
    CameraParams cam, const uint32_t *__restrict__ counts, float4 *__restrict__ grad_acc, float *__restrict__ g_mean3d,
    float *__restrict__ g_rotation, float *__restrict__ g_logscale, float *__restrict__ g_opacity,
    float *__restrict__ g_sh0, float *__restrict__ g_sh1, float *__restrict__ g_sh2, float *__restrict__ g_sh3,
    float *__restrict__ grad_norm_acc, float *__restrict__ absgrad_norm_acc)
{
    __shared__ __align__(16) float s_m[kThreads * 3];  /* staged mean3d rows, then gradient mean3d rows */
    __shared__ __align__(16) float s_s[kThreads * 3];  /* staged logscale rows, then gradient logscale rows */
    __shared__ float s_c[kThreads * 3];  /* gradient sh0 rows */
    const int64_t base = (int64_t)blockIdx.x * kThreads;
    const int64_t i = base + threadIdx.x;
    const int64_t avail = (n - base) * 3;
    /* every independent load of this thread is issued up front (the kernel is latency-bound) */
    const bool in_range = i < n;
    const uint32_t cnt = in_range ? counts[i] : 0u;
    float4 A0 = make_float4(0.0f, 0.0f, 0.0f, 0.0f), A1 = A0, A2 = A0, q = A0;
    if(in_range) {
        const float4 *acc_in = grad_acc + (size_t)i * 3;
        A0 = acc_in[0];
        A1 = acc_in[1];
        A2 = acc_in[2];
        q = *reinterpret_cast<const float4 *>(rotation + i * 4);
    }
    if(((reinterpret_cast<uintptr_t>(mean3d) | reinterpret_cast<uintptr_t>(logscale)) & 15u) == 0) {
        /* 16-byte asynchronous copies of the block's rows, all in flight together (zero-filled past the
         * end); the row of a thread is then read from shared memory.  The load-then-store loop it
         * replaces waited out its loads one iteration at a time: config-3 step 0.1425 -> 0.119 ms */
        if(threadIdx.x < kThreads * 3 / 4) {
            const int c = (int)threadIdx.x;
            const int64_t left = avail - 4 * (int64_t)c;
            const unsigned bytes = left >= 4 ? 16u : left > 0 ? (unsigned)left * 4u : 0u;
            const unsigned sm = (unsigned)__cvta_generic_to_shared(s_m + 4 * c);
            const unsigned ss = (unsigned)__cvta_generic_to_shared(s_s + 4 * c);
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(sm), "l"(bytes ? mean3d + base * 3 + 4 * c : mean3d), "r"(bytes) : "memory");
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(ss), "l"(bytes ? logscale + base * 3 + 4 * c : logscale), "r"(bytes) : "memory");
        }
        asm volatile("cp.async.commit_group;" ::: "memory");
        for(int j = threadIdx.x; j < kThreads * 3; j += kThreads) s_c[j] = 0.0f;
        asm volatile("cp.async.wait_group 0;" ::: "memory");
    } else {
        for(int j = threadIdx.x; j < kThreads * 3; j += kThreads) {
            const bool ok = j < avail;
            s_m[j] = ok ? mean3d[base * 3 + j] : 0.0f;
            s_s[j] = ok ? logscale[base * 3 + j] : 0.0f;
            s_c[j] = 0.0f;
        }
    }
    __syncthreads();
    const float m0 = s_m[threadIdx.x * 3 + 0], m1 = s_m[threadIdx.x * 3 + 1], m2 = s_m[threadIdx.x * 3 + 2];
    const float ls0 = s_s[threadIdx.x * 3 + 0], ls1 = s_s[threadIdx.x * 3 + 1], ls2 = s_s[threadIdx.x * 3 + 2];
    float gm[3] = { 0.0f, 0.0f, 0.0f }, gs[3] = { 0.0f, 0.0f, 0.0f };
    const bool visible = in_range && cnt != 0;
    if(i < n && !visible) {
        *reinterpret_cast<float4 *>(g_rotation + i * 4) = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        g_opacity[i] = 0.0f;
        if(bases > 1) for(int k = 0; k < 9; ++k) g_sh1[i * 9 + k] = 0.0f;
        if(bases > 4) for(int k = 0; k < 15; ++k) g_sh2[i * 15 + k] = 0.0f;
        if(bases > 9) for(int k = 0; k < 21; ++k) g_sh3[i * 21 + k] = 0.0f;
    }
    if(visible) {
    float4 *acc = grad_acc + (size_t)i * 3;
    acc[0] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    acc[1] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    acc[2] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    const float dm2x = A0.x, dm2y = A0.y, dcx = A0.z, dcy = A0.w, dcz = A1.x;
    const float gc[3] = { A1.z, A1.w, A2.x };
    g_opacity[i] = A1.y;
    if(grad_norm_acc != nullptr || absgrad_norm_acc != nullptr) {
        /* ADC statistics, gsx-metal/kernels/render_backward.metal:700-714: screen-space mean gradient
         * scaled to normalised device units (x W/2, y H/2 of the full frame), its norm and the norm
         * of the per-pixel absolute gradient (grad_acc[3i+2].yz, written by the blend backward) */
        const float sx = 0.5f * cam.width_f, sy = 0.5f * cam.height_f;
        if(grad_norm_acc != nullptr) {
            const float gx = dm2x * sx, gy = dm2y * sy;
            grad_norm_acc[i] += sqrtf(gx * gx + gy * gy);
        }
        if(absgrad_norm_acc != nullptr) {
            const float ax = A2.y * sx, ay = A2.z * sy;
            absgrad_norm_acc[i] += sqrtf(ax * ax + ay * ay);
        }
    }

    /* SH colour backward */
    float dmc0 = 0.0f, dmc1 = 0.0f, dmc2 = 0.0f;
#pragma unroll
    for(int c = 0; c < 3; ++c) s_c[threadIdx.x * 3 + c] = 0.28209479177387814f * gc[c];
    if(bases > 1) {
        const float xr = m0 - cam.cam_pos[0], yr = m1 - cam.cam_pos[1], zr = m2 - cam.cam_pos[2];
        const float nsq = xr * xr + yr * yr + zr * zr;
        const float inv = rsqrtf(nsq);
        const float x = xr * inv, y = yr * inv, z = zr * inv;
        float gdx[3], gdy[3], gdz[3];
        const float *c1 = sh1 + i * 9;
        for(int c = 0; c < 3; ++c) {
            g_sh1[i * 9 + 0 * 3 + c] = (-0.48860251190291987f * y) * gc[c];
            g_sh1[i * 9 + 1 * 3 + c] = (0.48860251190291987f * z) * gc[c];
            g_sh1[i * 9 + 2 * 3 + c] = (-0.48860251190291987f * x) * gc[c];
            gdx[c] = -0.48860251190291987f * c1[2 * 3 + c];
            gdy[c] = -0.48860251190291987f * c1[0 * 3 + c];
            gdz[c] = 0.48860251190291987f * c1[1 * 3 + c];
        }
        if(bases > 4) {
            const float xx = x * x, yy = y * y, zz = z * z, xy = x * y, xz = x * z, yz = y * z;
            const float *c2 = sh2 + i * 15;
            for(int c = 0; c < 3; ++c) {
                g_sh2[i * 15 + 0 * 3 + c] = (1.0925484305920792f * xy) * gc[c];
                g_sh2[i * 15 + 1 * 3 + c] = (-1.0925484305920792f * yz) * gc[c];
                g_sh2[i * 15 + 2 * 3 + c] = (0.94617469575755997f * zz - 0.31539156525251999f) * gc[c];
                g_sh2[i * 15 + 3 * 3 + c] = (-1.0925484305920792f * xz) * gc[c];
                g_sh2[i * 15 + 4 * 3 + c] = (0.54627421529603959f * xx - 0.54627421529603959f * yy) * gc[c];
                gdx[c] += 1.0925484305920792f * y * c2[0 * 3 + c] - 1.0925484305920792f * z * c2[3 * 3 + c]
                    + 1.0925484305920792f * x * c2[4 * 3 + c];
                gdy[c] += 1.0925484305920792f * x * c2[0 * 3 + c] - 1.0925484305920792f * z * c2[1 * 3 + c]
                    - 1.0925484305920792f * y * c2[4 * 3 + c];
                gdz[c] += -1.0925484305920792f * y * c2[1 * 3 + c] + 1.8923493915151202f * z * c2[2 * 3 + c]
                    - 1.0925484305920792f * x * c2[3 * 3 + c];
            }
            if(bases > 9) {
                const float *c3 = sh3 + i * 21;
                for(int c = 0; c < 3; ++c) {
                    g_sh3[i * 21 + 0 * 3 + c] = (0.59004358992664352f * y * (-3.0f * xx + yy)) * gc[c];
                    g_sh3[i * 21 + 1 * 3 + c] = (2.8906114426405538f * xy * z) * gc[c];
                    g_sh3[i * 21 + 2 * 3 + c] = (0.45704579946446572f * y * (1.0f - 5.0f * zz)) * gc[c];
                    g_sh3[i * 21 + 3 * 3 + c] = (0.3731763325901154f * z * (5.0f * zz - 3.0f)) * gc[c];
                    g_sh3[i * 21 + 4 * 3 + c] = (0.45704579946446572f * x * (1.0f - 5.0f * zz)) * gc[c];
                    g_sh3[i * 21 + 5 * 3 + c] = (1.4453057213202769f * z * (xx - yy)) * gc[c];
                    g_sh3[i * 21 + 6 * 3 + c] = (0.59004358992664352f * x * (-xx + 3.0f * yy)) * gc[c];
                    gdx[c] += -3.5402615395598609f * xy * c3[0 * 3 + c] + 2.8906114426405538f * yz * c3[1 * 3 + c]
                        + (0.45704579946446572f - 2.2852289973223288f * zz) * c3[4 * 3 + c]
                        + 2.8906114426405538f * xz * c3[5 * 3 + c]
                        + (-1.7701307697799304f * xx + 1.7701307697799304f * yy) * c3[6 * 3 + c];
                    gdy[c] += (-1.7701307697799304f * xx + 1.7701307697799304f * yy) * c3[0 * 3 + c]
                        + 2.8906114426405538f * xz * c3[1 * 3 + c]
                        + (0.45704579946446572f - 2.2852289973223288f * zz) * c3[2 * 3 + c]
                        - 2.8906114426405538f * yz * c3[5 * 3 + c] + 3.5402615395598609f * xy * c3[6 * 3 + c];
                    gdz[c] += 2.8906114426405538f * xy * c3[1 * 3 + c] - 4.5704579946446566f * yz * c3[2 * 3 + c]
                        + (5.597644988851731f * zz - 1.1195289977703462f) * c3[3 * 3 + c]
                        - 4.5704579946446566f * xz * c3[4 * 3 + c]
                        + (1.4453057213202769f * xx - 1.4453057213202769f * yy) * c3[5 * 3 + c];
                }
            }
        }
        const float gd0 = gdx[0] * gc[0] + gdx[1] * gc[1] + gdx[2] * gc[2];
        const float gd1 = gdy[0] * gc[0] + gdy[1] * gc[1] + gdy[2] * gc[2];
        const float gd2 = gdz[0] * gc[0] + gdz[1] * gc[1] + gdz[2] * gc[2];
        const float xx = xr * xr, yy = yr * yr, zz = zr * zr, xy = xr * yr, xz = xr * zr, yz = yr * zr;
        const float s3 = rsqrtf(nsq * nsq * nsq);
        dmc0 = ((yy + zz) * gd0 - xy * gd1 - xz * gd2) * s3;
        dmc1 = (-xy * gd0 + (xx + zz) * gd1 - yz * gd2) * s3;
        dmc2 = (-xz * gd0 - yz * gd1 + (xx + yy) * gd2) * s3;
    }

    const float *w = cam.w2c;
    const float depth = w[8] * m0 + w[9] * m1 + w[10] * m2 + w[11];
    const float x = (w[0] * m0 + w[1] * m1 + w[2] * m2 + w[3]) / depth;
    const float y = (w[4] * m0 + w[5] * m1 + w[6] * m2 + w[7]) / depth;
    float s[3], var[3];
#pragma unroll
    for(int k = 0; k < 3; ++k) {
        s[k] = __expf(k == 0 ? ls0 : (k == 1 ? ls1 : ls2));
        var[k] = s[k] * s[k];
    }
    const float qx = q.x, qy = q.y, qz = q.z, qr = q.w;
    const float qn = qr * qr + qx * qx + qy * qy + qz * qz;
    const float iqn = 1.0f / qn;
    const float qxx = 2.0f * qx * qx * iqn, qyy = 2.0f * qy * qy * iqn, qzz = 2.0f * qz * qz * iqn;
    const float qxy = 2.0f * qx * qy * iqn, qxz = 2.0f * qx * qz * iqn, qyz = 2.0f * qy * qz * iqn;
    const float qrx = 2.0f * qr * qx * iqn, qry = 2.0f * qr * qy * iqn, qrz = 2.0f * qr * qz * iqn;
    const float R[9] = { 1.0f - (qyy + qzz), qxy - qrz, qry + qxz, qrz + qxy, 1.0f - (qxx + qzz), qyz - qrx,
                         qxz - qry, qrx + qyz, 1.0f - (qxx + qyy) };
    float cov[3][3];
#pragma unroll
    for(int a = 0; a < 3; ++a)
#pragma unroll
        for(int b = 0; b < 3; ++b)
            cov[a][b] = R[a * 3 + 0] * var[0] * R[b * 3 + 0] + R[a * 3 + 1] * var[1] * R[b * 3 + 1] + R[a * 3 + 2] * var[2] * R[b * 3 + 2];
    const float cl = cam.clip_l, cr = cam.clip_r, ct = cam.clip_t, cb = cam.clip_b;
    const float tx = fmaxf(cl, fminf(x, cr)), ty = fmaxf(ct, fminf(y, cb));
    const float j11 = cam.fx / depth, j13 = -j11 * tx, j22 = cam.fy / depth, j23 = -j22 * ty;
    const float a1[3] = { j11 * w[0] + j13 * w[8], j11 * w[1] + j13 * w[9], j11 * w[2] + j13 * w[10] };
    const float a2[3] = { j22 * w[4] + j23 * w[8], j22 * w[5] + j23 * w[9], j22 * w[6] + j23 * w[10] };
    float b1[3], b2[3];
#pragma unroll
    for(int k = 0; k < 3; ++k) {
        b1[k] = a1[0] * cov[0][k] + a1[1] * cov[1][k] + a1[2] * cov[2][k];
        b2[k] = a2[0] * cov[0][k] + a2[1] * cov[1][k] + a2[2] * cov[2][k];
    }
    const float Aa = b1[0] * a1[0] + b1[1] * a1[1] + b1[2] * a1[2] + 0.3f;
    const float Bb = b1[0] * a2[0] + b1[1] * a2[1] + b1[2] * a2[2];
    const float Cc = b2[0] * a2[0] + b2[1] * a2[1] + b2[2] * a2[2] + 0.3f;
    const float det = Aa * Cc - Bb * Bb;
    const float idet = 1.0f / det;
    const float idet2 = idet * idet;
    const float dc2x = idet2 * (Bb * Cc * dcy - Cc * Cc * dcx - Bb * Bb * dcz);
    const float dc2y = idet2 * (Bb * Cc * dcx - 0.5f * (Aa * Cc + Bb * Bb) * dcy + Aa * Bb * dcz);
    const float dc2z = idet2 * (Aa * Bb * dcy - Bb * Bb * dcx - Aa * Aa * dcz);
    float dcov3[3][3];
#pragma unroll
    for(int a = 0; a < 3; ++a)
#pragma unroll
        for(int b = 0; b < 3; ++b) dcov3[a][b] = a1[a] * a1[b] * dc2x + (a1[a] * a2[b] + a1[b] * a2[a]) * dc2y + a2[a] * a2[b] * dc2z;
    float djw1[3], djw2[3];
#pragma unroll
    for(int k = 0; k < 3; ++k) {
        djw1[k] = 2.0f * (b1[k] * dc2x + b2[k] * dc2y);
        djw2[k] = 2.0f * (b1[k] * dc2y + b2[k] * dc2z);
    }
    const float dj11 = w[0] * djw1[0] + w[1] * djw1[1] + w[2] * djw1[2];
    const float dj22 = w[4] * djw2[0] + w[5] * djw2[1] + w[6] * djw2[2];
    const float dj13 = w[8] * djw1[0] + w[9] * djw1[1] + w[10] * djw1[2];
    const float dj23 = w[8] * djw2[0] + w[9] * djw2[1] + w[10] * djw2[2];
    const float dj13c = (x > cl && x < cr) ? dj13 : 0.0f;
    const float dj23c = (y > ct && y < cb) ? dj23 : 0.0f;
    const float h1 = dj11 - 2.0f * tx * dj13c, h2 = dj22 - 2.0f * ty * dj23c;
    const float idepth = 1.0f / depth;
    const float dcam0 = j11 * (dm2x - dj13c * idepth);
    const float dcam1 = j22 * (dm2y - dj23c * idepth);
    const float dcam2 = -j11 * (x * dm2x + h1 * idepth) - j22 * (y * dm2y + h2 * idepth);
    gm[0] = w[0] * dcam0 + w[4] * dcam1 + w[8] * dcam2 + dmc0;
    gm[1] = w[1] * dcam0 + w[5] * dcam1 + w[9] * dcam2 + dmc1;
    gm[2] = w[2] * dcam0 + w[6] * dcam1 + w[10] * dcam2 + dmc2;

    float dRS[9];
#pragma unroll
    for(int a = 0; a < 3; ++a)
#pragma unroll
        for(int b = 0; b < 3; ++b)
            dRS[a * 3 + b] = 2.0f * (dcov3[a][0] * R[0 * 3 + b] * s[b] + dcov3[a][1] * R[1 * 3 + b] * s[b] + dcov3[a][2] * R[2 * 3 + b] * s[b]);
#pragma unroll
    for(int b = 0; b < 3; ++b)
        gs[b] = (dRS[0 * 3 + b] * R[0 * 3 + b] + dRS[1 * 3 + b] * R[1 * 3 + b] + dRS[2 * 3 + b] * R[2 * 3 + b]) * s[b];
    float dR[9];
#pragma unroll
    for(int a = 0; a < 3; ++a)
#pragma unroll
        for(int b = 0; b < 3; ++b) dR[a * 3 + b] = dRS[a * 3 + b] * s[b];
    const float iq = rsqrtf(qn);
    const float w_ = qr * iq, x_ = qx * iq, y_ = qy * iq, z_ = qz * iq;
    const float dw = dR[1] * (-2.0f * z_) + dR[2] * (2.0f * y_) + dR[3] * (2.0f * z_) + dR[5] * (-2.0f * x_) + dR[6] * (-2.0f * y_) + dR[7] * (2.0f * x_);
    const float dx_ = dR[1] * (2.0f * y_) + dR[2] * (2.0f * z_) + dR[3] * (2.0f * y_) + dR[4] * (-4.0f * x_) + dR[5] * (-2.0f * w_)
        + dR[6] * (2.0f * z_) + dR[7] * (2.0f * w_) + dR[8] * (-4.0f * x_);
    const float dy_ = dR[0] * (-4.0f * y_) + dR[1] * (2.0f * x_) + dR[2] * (2.0f * w_) + dR[3] * (2.0f * x_) + dR[5] * (2.0f * z_)
        + dR[6] * (-2.0f * w_) + dR[7] * (2.0f * z_) + dR[8] * (-4.0f * y_);
    const float dz_ = dR[0] * (-4.0f * z_) + dR[1] * (-2.0f * w_) + dR[2] * (2.0f * x_) + dR[3] * (2.0f * w_) + dR[4] * (-4.0f * z_)
        + dR[5] * (2.0f * y_) + dR[6] * (2.0f * x_) + dR[7] * (2.0f * y_);
    const float dotq = w_ * dw + x_ * dx_ + y_ * dy_ + z_ * dz_;
    *reinterpret_cast<float4 *>(g_rotation + i * 4) =
        make_float4((dx_ - x_ * dotq) * iq, (dy_ - y_ * dotq) * iq, (dz_ - z_ * dotq) * iq, (dw - w_ * dotq) * iq);
    }
    /* coalesced write-out of the [256,3] gradient rows through shared memory */
    __syncthreads();
#pragma unroll
    for(int c = 0; c < 3; ++c) {
        s_m[threadIdx.x * 3 + c] = gm[c];
        s_s[threadIdx.x * 3 + c] = gs[c];
    }
    __syncthreads();
    for(int j = threadIdx.x; j < kThreads * 3; j += kThreads) {
        if(j < avail) {
            g_mean3d[base * 3 + j] = s_m[j];
            g_logscale[base * 3 + j] = s_s[j];
            g_sh0[base * 3 + j] = s_c[j];
        }
    }
}

} // namespace

cudaError_t gsx_launch_preprocess_backward(const float *mean3d, const float *rotation, const float *logscale,
                                           const float *sh1, const float *sh2, const float *sh3, int sh_degree,
                                           int64_t n, const CameraParams &cam, const uint32_t *counts,
                                           float4 *grad_acc, float *g_mean3d, float *g_rotation, float *g_logscale,
                                           float *g_opacity, float *g_sh0, float *g_sh1, float *g_sh2, float *g_sh3,
                                           float *grad_norm_acc, float *absgrad_norm_acc, cudaStream_t stream)
{
    if(n <= 0) return cudaSuccess;
    preprocess_backward_kernel<<<(unsigned)((n + kThreads - 1) / kThreads), kThreads, 0, stream>>>(
        mean3d, rotation, logscale, sh1, sh2, sh3, (sh_degree + 1) * (sh_degree + 1), n, cam, counts, grad_acc,
        g_mean3d, g_rotation, g_logscale, g_opacity, g_sh0, g_sh1, g_sh2, g_sh3, grad_norm_acc, absgrad_norm_acc);
    return cudaGetLastError();
}
