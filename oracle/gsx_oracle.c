/*
 * CPU ORACLE for the gsx-b200 hot path.  TEST INFRASTRUCTURE ONLY: the only callers are
 * tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg, and only as the checker.
 * Nothing in the product library links, loads or calls this file.
 *
 * It restates, in plain scalar C, the algorithm of the reference GSX CUDA backend
 * (Adversarr/gsx, the FastGS rasterizer under gsx/src/gsx-cuda/), citing the reference
 * file:line each function follows.  It is written under the arithmetic contract of
 * gsx_b200/csrc/gsx_detmath.h (no implicit FMA contraction: build with -ffp-contract=off;
 * exp/log from that header), so for the forward path it reproduces the CUDA kernels bit for bit.
 *
 * Pins: SSIM/L1/Adam are checked against the reference CPU backend built from the reference
 * sources (oracle/Makefile.ref); the render path against the reference's own known answers
 * (tests/test_oracle_pins.py) and, on the GPU box, against the reference CUDA backend.
 *
 * Deliberate deviation: depth ties between different Gaussians are
 * broken by primitive index.  The reference breaks them by atomic compaction order
 * (kernels_forward.cuh:433-436), which is nondeterministic.
 */
#include "../gsx_b200/csrc/gsx_detmath.h"
#ifdef _OPENMP
#include <omp.h>
#endif

#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORC_TILE 16
#define ORC_BLOCK (ORC_TILE * ORC_TILE)
#define ORC_SEQ_THRESHOLD 8

typedef struct orc_camera {
    float w2c[12];     /* row-major 3x4 world->camera */
    float cam_pos[3];  /* camera centre in world space */
    float fx, fy, cx, cy;
    int width, height;
    float near_plane, far_plane;
} orc_camera;

/* ---------------------------------------------------------------- pose
 * gsx/src/gsx-cuda/render.c:870-921 (quaternion xyzw -> row-major R, camera position -R^T t). */
void orc_pose_to_camera(const float q[4], const float t[3], float w2c[12], float cam_pos[3])
{
    float qx = q[0], qy = q[1], qz = q[2], qw = q[3];
    float norm_sq = qx * qx + qy * qy + qz * qz + qw * qw;
    float r[9];
    if(norm_sq > 1.0e-20f) {
        float inv = 1.0f / sqrtf(norm_sq);
        qx *= inv;
        qy *= inv;
        qz *= inv;
        qw *= inv;
    } else {
        qx = 0.0f;
        qy = 0.0f;
        qz = 0.0f;
        qw = 1.0f;
    }
    r[0] = 1.0f - 2.0f * (qy * qy + qz * qz);
    r[1] = 2.0f * (qx * qy - qw * qz);
    r[2] = 2.0f * (qx * qz + qw * qy);
    r[3] = 2.0f * (qx * qy + qw * qz);
    r[4] = 1.0f - 2.0f * (qx * qx + qz * qz);
    r[5] = 2.0f * (qy * qz - qw * qx);
    r[6] = 2.0f * (qx * qz - qw * qy);
    r[7] = 2.0f * (qy * qz + qw * qx);
    r[8] = 1.0f - 2.0f * (qx * qx + qy * qy);
    w2c[0] = r[0]; w2c[1] = r[1]; w2c[2] = r[2]; w2c[3] = t[0];
    w2c[4] = r[3]; w2c[5] = r[4]; w2c[6] = r[5]; w2c[7] = t[1];
    w2c[8] = r[6]; w2c[9] = r[7]; w2c[10] = r[8]; w2c[11] = t[2];
    cam_pos[0] = -(r[0] * t[0] + r[3] * t[1] + r[6] * t[2]);
    cam_pos[1] = -(r[1] * t[0] + r[4] * t[1] + r[7] * t[2]);
    cam_pos[2] = -(r[2] * t[0] + r[5] * t[1] + r[8] * t[2]);
}

/* saturating float->int conversions with the GPU's cvt.rmi/cvt.rpi semantics */
static int orc_f2i_rd(float v)
{
    float f = floorf(v);
    if(!(f == f)) return 0;
    if(f >= 2147483647.0f) return 2147483647;
    if(f <= -2147483648.0f) return (int)(-2147483647 - 1);
    return (int)f;
}

static int orc_f2i_ru(float v)
{
    float f = ceilf(v);
    if(!(f == f)) return 0;
    if(f >= 2147483647.0f) return 2147483647;
    if(f <= -2147483648.0f) return (int)(-2147483647 - 1);
    return (int)f;
}

/* ---------------------------------------------------------------- SH colour
 * fastgs/kernels_forward.cuh:30-68 (convert_sh_to_color), AoS [N,k,3] coefficient layout. */
static void orc_sh_color(const float *sh0, const float *sh1, const float *sh2, const float *sh3,
                         const float m[3], const float cam[3], int64_t i, int bases, float out[3])
{
    for(int c = 0; c < 3; ++c) out[c] = 0.5f + 0.28209479177387814f * sh0[i * 3 + c];
    if(bases > 1) {
        float dx = m[0] - cam[0], dy = m[1] - cam[1], dz = m[2] - cam[2];
        float inv = 1.0f / sqrtf(dx * dx + dy * dy + dz * dz);
        float x = dx * inv, y = dy * inv, z = dz * inv;
        const float *c1 = sh1 + i * 9;
        for(int c = 0; c < 3; ++c) {
            out[c] = out[c] + (-0.48860251190291987f * y) * c1[0 * 3 + c] + (0.48860251190291987f * z) * c1[1 * 3 + c]
                + (-0.48860251190291987f * x) * c1[2 * 3 + c];
        }
        if(bases > 4) {
            float xx = x * x, yy = y * y, zz = z * z, xy = x * y, xz = x * z, yz = y * z;
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

/* ---------------------------------------------------------------- tile overlap test
 * fastgs/kernels_forward.cuh:71-106 (will_primitive_contribute); `mean` is mean2d - 0.5. */
static int orc_tile_contributes(float mx, float my, float cx, float cy, float cz, unsigned tx, unsigned ty, float power_threshold)
{
    const float rminx = (float)(tx * ORC_TILE), rminy = (float)(ty * ORC_TILE);
    const float rmaxx = (float)((tx + 1) * ORC_TILE - 1), rmaxy = (float)((ty + 1) * ORC_TILE - 1);
    const float x_min_diff = rminx - mx;
    const float x_left = x_min_diff > 0.0f ? 1.0f : 0.0f;
    const float not_in_x = x_left + (mx > rmaxx ? 1.0f : 0.0f);
    const float y_min_diff = rminy - my;
    const float y_above = y_min_diff > 0.0f ? 1.0f : 0.0f;
    const float not_in_y = y_above + (my > rmaxy ? 1.0f : 0.0f);
    if(not_in_y + not_in_x == 0.0f) return 1;
    const float ccx = x_left != 0.0f ? rminx : rmaxx;
    const float ccy = y_above != 0.0f ? rminy : rmaxy;
    const float diffx = mx - ccx, diffy = my - ccy;
    const float dx = copysignf((float)(ORC_TILE - 1), x_min_diff);
    const float dy = copysignf((float)(ORC_TILE - 1), y_min_diff);
    const float tx_ = not_in_y * gsx_saturatef((dx * cx * diffx + dx * cy * diffy) / (dx * cx * dx));
    const float ty_ = not_in_x * gsx_saturatef((dy * cy * diffx + dy * cz * diffy) / (dy * cz * dy));
    const float px = ccx + tx_ * dx, py = ccy + ty_ * dy;
    const float ddx = mx - px, ddy = my - py;
    const float power = 0.5f * (cx * ddx * ddx + cz * ddy * ddy) + cy * ddx * ddy;
    return power <= power_threshold;
}

/* ---------------------------------------------------------------- preprocess
 * fastgs/kernels_forward.cuh:179-438 (preprocess_cu) and :109-175 (compute_exact_n_touched_tiles).
 * Outputs per primitive (zeros / untouched when culled):
 *   n_touched[N], bounds[N*4] (x_min, x_max, y_min, y_max in tiles), mean2d[N*2],
 *   conic_op[N*4] (conic x,y,z, sigmoid opacity), color[N*3] (unclamped), depth[N].
 * Returns the total instance count. */
static uint64_t orc_preprocess_impl(int64_t n, const float *mean3d, const float *rotation, const float *logscale,
                                    const float *opacity_raw, const float *sh0, const float *sh1, const float *sh2,
                                    const float *sh3, int sh_degree, const orc_camera *cam, uint32_t *n_touched,
                                    uint32_t *bounds, float *mean2d, float *conic_op, float *color, float *depth_out,
                                    float *screen_radius)
{
    const unsigned gw = (unsigned)((cam->width + ORC_TILE - 1) / ORC_TILE);
    const unsigned gh = (unsigned)((cam->height + ORC_TILE - 1) / ORC_TILE);
    const float *w = cam->w2c;
    const float W = (float)cam->width, H = (float)cam->height;
    const int bases = (sh_degree + 1) * (sh_degree + 1);
    uint64_t total = 0;
#pragma omp parallel for schedule(static, 4096) reduction(+ : total)
    for(int64_t i = 0; i < n; ++i) {
        n_touched[i] = 0;
        const float m[3] = { mean3d[i * 3 + 0], mean3d[i * 3 + 1], mean3d[i * 3 + 2] };
        const float depth = w[8] * m[0] + w[9] * m[1] + w[10] * m[2] + w[11];
        if(depth < cam->near_plane || depth > cam->far_plane) continue;
        const float op = gsx_sigmoidf(opacity_raw[i]);
        if(op < 1.0f / 255.0f) continue;
        float var[3];
        for(int k = 0; k < 3; ++k) {
            const float s = gsx_expf(logscale[i * 3 + k]);
            var[k] = s * s;
        }
        const float qx = rotation[i * 4 + 0], qy = rotation[i * 4 + 1], qz = rotation[i * 4 + 2], qr = rotation[i * 4 + 3];
        const float qrr = qr * qr, qxx_raw = qx * qx, qyy_raw = qy * qy, qzz_raw = qz * qz;
        const float qn = qrr + qxx_raw + qyy_raw + qzz_raw;
        if(qn < 1e-8f) continue;
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
        const float clip_l = (-0.15f * W - cam->cx) / cam->fx, clip_r = (1.15f * W - cam->cx) / cam->fx;
        const float clip_t = (-0.15f * H - cam->cy) / cam->fy, clip_b = (1.15f * H - cam->cy) / cam->fy;
        const float tx = fmaxf(clip_l, fminf(x, clip_r));
        const float ty = fmaxf(clip_t, fminf(y, clip_b));
        const float j11 = cam->fx / depth, j13 = -j11 * tx, j22 = cam->fy / depth, j23 = -j22 * ty;
        const float a1x = j11 * w[0] + j13 * w[8], a1y = j11 * w[1] + j13 * w[9], a1z = j11 * w[2] + j13 * w[10];
        const float a2x = j22 * w[4] + j23 * w[8], a2y = j22 * w[5] + j23 * w[9], a2z = j22 * w[6] + j23 * w[10];
        const float b1x = a1x * c11 + a1y * c12 + a1z * c13, b1y = a1x * c12 + a1y * c22 + a1z * c23, b1z = a1x * c13 + a1y * c23 + a1z * c33;
        const float b2x = a2x * c11 + a2y * c12 + a2z * c13, b2y = a2x * c12 + a2y * c22 + a2z * c23, b2z = a2x * c13 + a2y * c23 + a2z * c33;
        float cov_x = b1x * a1x + b1y * a1y + b1z * a1z;
        const float cov_y = b1x * a2x + b1y * a2y + b1z * a2z;
        float cov_z = b2x * a2x + b2y * a2y + b2z * a2z;
        cov_x += 0.3f;
        cov_z += 0.3f;
        const float det = cov_x * cov_z - cov_y * cov_y;
        if(det < 1e-8f) continue;
        const float conx = cov_z / det, cony = -cov_y / det, conz = cov_x / det;
        const float m2x = x * cam->fx + cam->cx, m2y = y * cam->fy + cam->cy;
        const float pt = gsx_logf(op * 255.0f);
        const float ptf = sqrtf(2.0f * pt);
        const float ex = fmaxf(ptf * sqrtf(cov_x) - 0.5f, 0.0f);
        const float ey = fmaxf(ptf * sqrtf(cov_z) - 0.5f, 0.0f);
        int v;
        unsigned bx0, bx1, by0, by1;
        v = orc_f2i_rd((m2x - ex) / 16.0f); bx0 = (unsigned)(v > 0 ? v : 0); if(bx0 > gw) bx0 = gw;
        v = orc_f2i_ru((m2x + ex) / 16.0f); bx1 = (unsigned)(v > 0 ? v : 0); if(bx1 > gw) bx1 = gw;
        v = orc_f2i_rd((m2y - ey) / 16.0f); by0 = (unsigned)(v > 0 ? v : 0); if(by0 > gh) by0 = gh;
        v = orc_f2i_ru((m2y + ey) / 16.0f); by1 = (unsigned)(v > 0 ? v : 0); if(by1 > gh) by1 = gh;
        const unsigned tmax = (bx1 - bx0) * (by1 - by0);
        if(tmax == 0) continue;
        const float msx = m2x - 0.5f, msy = m2y - 0.5f;
        const unsigned bw = bx1 - bx0;
        unsigned cnt = 0;
        for(unsigned k = 0; k < tmax; ++k) {
            if(orc_tile_contributes(msx, msy, conx, cony, conz, bx0 + k % bw, by0 + k / bw, pt)) ++cnt;
        }
        if(cnt == 0) continue;
        n_touched[i] = cnt;
        if(screen_radius) {
            /* gsx-metal/kernels/render.metal:432-438 */
            const float mid = 0.5f * (cov_x + cov_z);
            const float disc = sqrtf(fmaxf(0.1f, mid * mid - det));
            screen_radius[i] = ceilf(3.0f * sqrtf(fmaxf(mid + disc, mid - disc)));
        }
        bounds[i * 4 + 0] = bx0; bounds[i * 4 + 1] = bx1; bounds[i * 4 + 2] = by0; bounds[i * 4 + 3] = by1;
        mean2d[i * 2 + 0] = m2x; mean2d[i * 2 + 1] = m2y;
        conic_op[i * 4 + 0] = conx; conic_op[i * 4 + 1] = cony; conic_op[i * 4 + 2] = conz; conic_op[i * 4 + 3] = op;
        orc_sh_color(sh0, sh1, sh2, sh3, m, cam->cam_pos, i, bases, color + i * 3);
        depth_out[i] = depth;
        total += cnt;
    }
    return total;
}

uint64_t orc_preprocess(int64_t n, const float *mean3d, const float *rotation, const float *logscale, const float *opacity_raw,
                        const float *sh0, const float *sh1, const float *sh2, const float *sh3, int sh_degree,
                        const orc_camera *cam, uint32_t *n_touched, uint32_t *bounds, float *mean2d, float *conic_op,
                        float *color, float *depth_out)
{
    return orc_preprocess_impl(n, mean3d, rotation, logscale, opacity_raw, sh0, sh1, sh2, sh3, sh_degree, cam, n_touched,
                               bounds, mean2d, conic_op, color, depth_out, NULL);
}

/* The same, also writing the screen radius of every visible (tile-touching) Gaussian: the value a
 * TRAIN forward folds into gs_max_screen_radius (gsx-metal/kernels/render.metal:425-439; a visible
 * Gaussian is also the one that raises gs_visible_counter).  Culled Gaussians keep screen_radius[i]. */
uint64_t orc_preprocess_aux(int64_t n, const float *mean3d, const float *rotation, const float *logscale,
                            const float *opacity_raw, const float *sh0, const float *sh1, const float *sh2, const float *sh3,
                            int sh_degree, const orc_camera *cam, uint32_t *n_touched, uint32_t *bounds, float *mean2d,
                            float *conic_op, float *color, float *depth_out, float *screen_radius)
{
    return orc_preprocess_impl(n, mean3d, rotation, logscale, opacity_raw, sh0, sh1, sh2, sh3, sh_degree, cam, n_touched,
                               bounds, mean2d, conic_op, color, depth_out, screen_radius);
}

/* ---------------------------------------------------------------- instance emission + sort
 * fastgs/kernels_forward.cuh:453-556 (create_instances_cu) emits (tile, primitive) per touched tile
 * in row-major tile order; forward.cu:155-161,214-220 sort by depth then stably by tile.  The same
 * order is produced here by one stable sort of the 64-bit key (tile << 32 | depth bits) over
 * instances emitted in primitive-index order. */
typedef struct {
    uint64_t key;
    uint32_t val;
    uint64_t pos;
} orc_pair;

static int orc_pair_cmp(const void *a, const void *b)
{
    const orc_pair *x = (const orc_pair *)a, *y = (const orc_pair *)b;
    if(x->key != y->key) return x->key < y->key ? -1 : 1;
    return x->pos < y->pos ? -1 : (x->pos > y->pos ? 1 : 0);
}

/* Unsorted emission: keys/vals in primitive order (the exact buffer the GPU emits before sorting). */
void orc_emit(int64_t n, const uint32_t *n_touched, const uint32_t *bounds, const float *mean2d, const float *conic_op,
              const float *depth, int width, uint64_t *keys, uint32_t *vals)
{
    const unsigned gw = (unsigned)((width + ORC_TILE - 1) / ORC_TILE);
    uint64_t off = 0;
    for(int64_t i = 0; i < n; ++i) {
        if(n_touched[i] == 0) continue;
        const unsigned bx0 = bounds[i * 4 + 0], bx1 = bounds[i * 4 + 1], by0 = bounds[i * 4 + 2], by1 = bounds[i * 4 + 3];
        const unsigned bw = bx1 - bx0, tmax = bw * (by1 - by0);
        const float msx = mean2d[i * 2 + 0] - 0.5f, msy = mean2d[i * 2 + 1] - 0.5f;
        const float pt = gsx_logf(conic_op[i * 4 + 3] * 255.0f);
        const uint32_t dbits = gsx_float_to_bits(depth[i]);
        for(unsigned k = 0; k < tmax; ++k) {
            const unsigned tx = bx0 + k % bw, ty = by0 + k / bw;
            if(orc_tile_contributes(msx, msy, conic_op[i * 4 + 0], conic_op[i * 4 + 1], conic_op[i * 4 + 2], tx, ty, pt)) {
                keys[off] = ((uint64_t)(ty * gw + tx) << 32) | dbits;
                vals[off] = (uint32_t)i;
                ++off;
            }
        }
    }
}

/* Stable sort of (key, value) pairs by key: the contract of the GPU LSD radix sort. */
int orc_sort_pairs(uint64_t count, uint64_t *keys, uint32_t *vals)
{
    orc_pair *p = (orc_pair *)malloc(sizeof(orc_pair) * (count ? count : 1));
    if(p == NULL) return -1;
    for(uint64_t i = 0; i < count; ++i) {
        p[i].key = keys[i];
        p[i].val = vals[i];
        p[i].pos = i;
    }
    qsort(p, count, sizeof(orc_pair), orc_pair_cmp);
    for(uint64_t i = 0; i < count; ++i) {
        keys[i] = p[i].key;
        vals[i] = p[i].val;
    }
    free(p);
    return 0;
}

/* fastgs/kernels_forward.cuh:558-593: per-tile [start, end) over the sorted keys (zero if empty). */
void orc_tile_ranges(uint64_t count, const uint64_t *keys, int n_tiles, uint32_t *ranges)
{
    memset(ranges, 0, sizeof(uint32_t) * 2 * (size_t)n_tiles);
    for(uint64_t i = 0; i < count; ++i) {
        const uint32_t t = (uint32_t)(keys[i] >> 32);
        if(i == 0 || (uint32_t)(keys[i - 1] >> 32) != t) ranges[t * 2 + 0] = (uint32_t)i;
        if(i + 1 == count || (uint32_t)(keys[i + 1] >> 32) != t) ranges[t * 2 + 1] = (uint32_t)(i + 1);
    }
}

/* ---------------------------------------------------------------- blend forward
 * fastgs/kernels_forward.cuh:595-736 (blend_cu<false>) + render-kernels.cu:13-36 (background
 * compose).  The per-fragment arithmetic is written in the explicit-FMA form the GPU kernel uses:
 *   sigma = fma(dx, fma(0.5cx, dx, cy*dy), (0.5cz*dy)*dy),  w = T*alpha,  C = fma(w, colour, C).
 * Outputs: out_rgb CHW composed with the background, out_alpha = 1 - T, n_contrib per pixel,
 * tile_max[T] (max n_contrib in the tile). */
void orc_blend_forward(int width, int height, const uint32_t *ranges, const uint32_t *vals, const float *mean2d,
                       const float *conic_op, const float *color, const float bg[3], float *out_rgb, float *out_alpha,
                       uint32_t *n_contrib, uint32_t *tile_max)
{
    const int gw = (width + ORC_TILE - 1) / ORC_TILE, gh = (height + ORC_TILE - 1) / ORC_TILE;
    const size_t P = (size_t)width * (size_t)height;
    /* tiles are independent (every output is per pixel or per tile): parallel over tiles */
#pragma omp parallel for schedule(dynamic, 4)
    for(int tile = 0; tile < gw * gh; ++tile) {
        {
            const int ty = tile / gw, tx = tile % gw;
            const uint32_t r0 = ranges[tile * 2 + 0], r1 = ranges[tile * 2 + 1];
            uint32_t tmax = 0;
            for(int ly = 0; ly < ORC_TILE; ++ly) {
                for(int lx = 0; lx < ORC_TILE; ++lx) {
                    const int px = tx * ORC_TILE + lx, py = ty * ORC_TILE + ly;
                    if(px >= width || py >= height) continue;
                    const float pxf = (float)px + 0.5f, pyf = (float)py + 0.5f;
                    float C[3] = { 0.0f, 0.0f, 0.0f };
                    float T = 1.0f;
                    uint32_t npos = 0, ncon = 0;
                    for(uint32_t j = r0; j < r1; ++j) {
                        const uint32_t p = vals[j];
                        ++npos;
                        const float dx = mean2d[p * 2 + 0] - pxf, dy = mean2d[p * 2 + 1] - pyf;
                        const float hcx = 0.5f * conic_op[p * 4 + 0], cy = conic_op[p * 4 + 1], hcz = 0.5f * conic_op[p * 4 + 2];
                        const float sigma = fmaf(dx, fmaf(hcx, dx, cy * dy), (hcz * dy) * dy);
                        if(sigma < 0.0f) continue;
                        const float g = gsx_expf(-sigma);
                        const float alpha = fminf(conic_op[p * 4 + 3] * g, 0.999f);
                        if(alpha < 1.0f / 255.0f) continue;
                        const float wgt = T * alpha;
                        for(int c = 0; c < 3; ++c) C[c] = fmaf(wgt, fmaxf(color[p * 3 + c], 0.0f), C[c]);
                        T = T * (1.0f - alpha);
                        ncon = npos;
                        if(T < 1e-4f) break;
                    }
                    const size_t idx = (size_t)py * (size_t)width + (size_t)px;
                    const float a = 1.0f - T;
                    const float tr = 1.0f - a;
                    for(int c = 0; c < 3; ++c) out_rgb[c * P + idx] = C[c] + tr * bg[c];
                    out_alpha[idx] = a;
                    n_contrib[idx] = ncon;
                    if(ncon > tmax) tmax = ncon;
                }
            }
            tile_max[tile] = tmax;
        }
    }
}

/* ---------------------------------------------------------------- blend backward
 * fastgs/kernels_backward.cuh:484-730 (blend_backward_cu2).  For every bucket of 32 instances
 * below the tile's max contributor and every pixel, the state starts from the forward snapshot
 * (colour and transmittance before the bucket, kernels_forward.cuh:671-676) and walks the bucket
 * front to back with the reference's backward rules: no 1/255 skip, sigma clamped at 0, alpha
 * clamped at 0.999 with zero opacity gradient when saturated, (1-alpha) floored at 1e-4.
 * `image` is the composed output (colour + T*background), as the reference's retained image.
 * Outputs (accumulated with +=): d_mean2d[N*2], d_conic[N*3], d_opacity_raw[N], d_color[N*3]. */
static int orc_backward_consistent = 0;
void orc_set_backward_consistent(int v) { orc_backward_consistent = v; }

static void orc_blend_backward_tile(int tile, int width, int height, const uint32_t *ranges, const uint32_t *vals,
                                    const float *mean2d, const float *conic_op, const float *color, const float *image,
                                    const uint32_t *n_contrib, const uint32_t *tile_max, const float *grad_rgb,
                                    float *d_mean2d, float *d_conic, float *d_opacity_raw, float *d_color,
                                    float *d_mean2d_abs)
{
    const int gw = (width + ORC_TILE - 1) / ORC_TILE;
    const size_t P = (size_t)width * (size_t)height;
    {
        {
            const int ty = tile / gw, tx = tile % gw;
            const uint32_t r0 = ranges[tile * 2 + 0], r1 = ranges[tile * 2 + 1];
            const uint32_t n_inst = r1 - r0;
            for(int ly = 0; ly < ORC_TILE; ++ly) {
                for(int lx = 0; lx < ORC_TILE; ++lx) {
                    const int px = tx * ORC_TILE + lx, py = ty * ORC_TILE + ly;
                    if(px >= width || py >= height) continue;
                    const size_t idx = (size_t)py * (size_t)width + (size_t)px;
                    const float pxf = (float)px + 0.5f, pyf = (float)py + 0.5f;
                    const uint32_t last = n_contrib[idx];
                    const float g[3] = { grad_rgb[idx], grad_rgb[P + idx], grad_rgb[2 * P + idx] };
                    /* forward replay for the per-bucket snapshots */
                    float C[3] = { 0.0f, 0.0f, 0.0f };
                    float T = 1.0f;
                    int done = 0;
                    for(uint32_t b = 0; b * 32 < n_inst; ++b) {
                        const float snapC[3] = { C[0], C[1], C[2] };
                        const float snapT = T;
                        if(b * 32 < tile_max[tile]) {
                            float bT = snapT;
                            float after[3];
                            for(int c = 0; c < 3; ++c) after[c] = image[c * P + idx] - snapC[c];
                            for(uint32_t k = 0; k < 32 && b * 32 + k < n_inst; ++k) {
                                const uint32_t tpi = b * 32 + k;
                                const uint32_t p = vals[r0 + tpi];
                                if(tpi >= last) continue;
                                const float mx = mean2d[p * 2 + 0] - 0.5f, my = mean2d[p * 2 + 1] - 0.5f;
                                const float dx = mx - (float)px, dy = my - (float)py;
                                const float cx = conic_op[p * 4 + 0], cy = conic_op[p * 4 + 1], cz = conic_op[p * 4 + 2];
                                const float op = conic_op[p * 4 + 3];
                                float sig = 0.5f * (cx * dx * dx + cz * dy * dy) + cy * dx * dy;
                                if(orc_backward_consistent) {
                                    const float fdx = mean2d[p * 2 + 0] - pxf, fdy = mean2d[p * 2 + 1] - pyf;
                                    const float fs = fmaf(fdx, fmaf(0.5f * cx, fdx, cy * fdy), (0.5f * cz * fdy) * fdy);
                                    if(fs < 0.0f) continue;
                                    if(fminf(op * gsx_expf(-fs), 0.999f) < 1.0f / 255.0f) continue;
                                }
                                if(sig < 0.0f) sig = 0.0f;
                                const float gauss = expf(-sig);
                                const float a_pre = op * gauss;
                                const float alpha = fminf(a_pre, 0.999f);
                                const int sat = a_pre >= 0.999f;
                                const float wgt = bT * alpha;
                                float col[3], fac[3];
                                for(int c = 0; c < 3; ++c) {
                                    col[c] = fmaxf(color[p * 3 + c], 0.0f);
                                    fac[c] = color[p * 3 + c] >= 0.0f ? 1.0f : 0.0f;
                                }
                                const float cdg = col[0] * g[0] + col[1] * g[1] + col[2] * g[2];
                                for(int c = 0; c < 3; ++c) {
                                    d_color[p * 3 + c] += wgt * (g[c] * fac[c]);
                                    after[c] -= wgt * col[c];
                                }
                                const float adg = after[0] * g[0] + after[1] * g[1] + after[2] * g[2];
                                const float oma = 1.0f - alpha;
                                const float oma_safe = fmaxf(oma, 1e-4f);
                                const float dL_dalpha = bT * cdg - adg * (1.0f / oma_safe);
                                const float part = sat ? 0.0f : alpha * dL_dalpha;
                                d_conic[p * 3 + 0] += -0.5f * part * (dx * dx);
                                d_conic[p * 3 + 1] += -part * (dx * dy);
                                d_conic[p * 3 + 2] += -0.5f * part * (dy * dy);
                                d_mean2d[p * 2 + 0] -= part * (cx * dx + cy * dy);
                                d_mean2d[p * 2 + 1] -= part * (cy * dx + cz * dy);
                                if(d_mean2d_abs) {
                                    /* gsx-metal/kernels/render_backward.metal:361-366 */
                                    d_mean2d_abs[p * 2 + 0] += fabsf(part * (cx * dx + cy * dy));
                                    d_mean2d_abs[p * 2 + 1] += fabsf(part * (cy * dx + cz * dy));
                                }
                                d_opacity_raw[p] += part * (1.0f - op);
                                bT *= oma;
                            }
                        }
                        /* advance the forward replay across this bucket (forward rules) */
                        for(uint32_t k = 0; k < 32 && b * 32 + k < n_inst && !done; ++k) {
                            const uint32_t p = vals[r0 + b * 32 + k];
                            const float dx = mean2d[p * 2 + 0] - pxf, dy = mean2d[p * 2 + 1] - pyf;
                            const float hcx = 0.5f * conic_op[p * 4 + 0], cy = conic_op[p * 4 + 1], hcz = 0.5f * conic_op[p * 4 + 2];
                            const float sigma = fmaf(dx, fmaf(hcx, dx, cy * dy), (hcz * dy) * dy);
                            if(sigma < 0.0f) continue;
                            const float ga = gsx_expf(-sigma);
                            const float alpha = fminf(conic_op[p * 4 + 3] * ga, 0.999f);
                            if(alpha < 1.0f / 255.0f) continue;
                            const float wgt = T * alpha;
                            for(int c = 0; c < 3; ++c) C[c] = fmaf(wgt, fmaxf(color[p * 3 + c], 0.0f), C[c]);
                            T = T * (1.0f - alpha);
                            if(T < 1e-4f) done = 1;
                        }
                    }
                }
            }
        }
    }
}

/* Tiles in parallel; each thread accumulates into its own gradient arrays, summed in thread order
 * at the end (the summation order differs from a serial walk by rounding only). */
static void orc_blend_backward_impl(int width, int height, const uint32_t *ranges, const uint32_t *vals,
                                    const float *mean2d, const float *conic_op, const float *color, const float *image,
                                    const uint32_t *n_contrib, const uint32_t *tile_max, const float *grad_rgb,
                                    float *d_mean2d, float *d_conic, float *d_opacity_raw, float *d_color,
                                    float *d_mean2d_abs)
{
    const int n_tiles = ((width + ORC_TILE - 1) / ORC_TILE) * ((height + ORC_TILE - 1) / ORC_TILE);
    /* primitive count bound: the largest index referenced + 1 */
    int64_t n = 0;
    const uint64_t total = n_tiles > 0 ? ranges[(size_t)(n_tiles - 1) * 2 + 1] : 0;
    for(int t = 0; t < n_tiles; ++t)
        for(uint32_t j = ranges[t * 2]; j < ranges[t * 2 + 1]; ++j)
            if((int64_t)vals[j] + 1 > n) n = (int64_t)vals[j] + 1;
    (void)total;
    int nt = 1;
#ifdef _OPENMP
    nt = omp_get_max_threads();
#endif
    const size_t per = (size_t)n * (d_mean2d_abs ? 11 : 9);
    float *priv = nt > 1 && n > 0 ? (float *)calloc((size_t)nt * per, sizeof(float)) : NULL;
    if(priv == NULL) {
        for(int t = 0; t < n_tiles; ++t)
            orc_blend_backward_tile(t, width, height, ranges, vals, mean2d, conic_op, color, image, n_contrib, tile_max,
                                    grad_rgb, d_mean2d, d_conic, d_opacity_raw, d_color, d_mean2d_abs);
        return;
    }
#pragma omp parallel num_threads(nt)
    {
        int me = 0;
#ifdef _OPENMP
        me = omp_get_thread_num();
#endif
        float *b = priv + (size_t)me * per;
        float *pm = b, *pc = b + 2 * n, *po = b + 5 * n, *pcol = b + 6 * n, *pabs = d_mean2d_abs ? b + 9 * n : NULL;
#pragma omp for schedule(dynamic, 2)
        for(int t = 0; t < n_tiles; ++t)
            orc_blend_backward_tile(t, width, height, ranges, vals, mean2d, conic_op, color, image, n_contrib, tile_max,
                                    grad_rgb, pm, pc, po, pcol, pabs);
    }
    for(int k = 0; k < nt; ++k) {
        const float *b = priv + (size_t)k * per;
        for(int64_t i = 0; i < 2 * n; ++i) d_mean2d[i] += b[i];
        for(int64_t i = 0; i < 3 * n; ++i) d_conic[i] += b[2 * n + i];
        for(int64_t i = 0; i < n; ++i) d_opacity_raw[i] += b[5 * n + i];
        for(int64_t i = 0; i < 3 * n; ++i) d_color[i] += b[6 * n + i];
        if(d_mean2d_abs)
            for(int64_t i = 0; i < 2 * n; ++i) d_mean2d_abs[i] += b[9 * n + i];
    }
    free(priv);
}

void orc_blend_backward(int width, int height, const uint32_t *ranges, const uint32_t *vals, const float *mean2d,
                        const float *conic_op, const float *color, const float *image, const uint32_t *n_contrib,
                        const uint32_t *tile_max, const float *grad_rgb, float *d_mean2d, float *d_conic,
                        float *d_opacity_raw, float *d_color)
{
    orc_blend_backward_impl(width, height, ranges, vals, mean2d, conic_op, color, image, n_contrib, tile_max, grad_rgb,
                            d_mean2d, d_conic, d_opacity_raw, d_color, NULL);
}

/* The same, also accumulating the per-pixel absolute screen-space mean gradient per component
 * (d_mean2d_abs[N*2], added to), the input of gs_absgrad_acc. */
void orc_blend_backward_abs(int width, int height, const uint32_t *ranges, const uint32_t *vals, const float *mean2d,
                            const float *conic_op, const float *color, const float *image, const uint32_t *n_contrib,
                            const uint32_t *tile_max, const float *grad_rgb, float *d_mean2d, float *d_conic,
                            float *d_opacity_raw, float *d_color, float *d_mean2d_abs)
{
    orc_blend_backward_impl(width, height, ranges, vals, mean2d, conic_op, color, image, n_contrib, tile_max, grad_rgb,
                            d_mean2d, d_conic, d_opacity_raw, d_color, d_mean2d_abs);
}

/* ---------------------------------------------------------------- preprocess backward
 * fastgs/kernels_backward.cuh:127-422 (preprocess_backward_cu) and :40-125 (SH backward).
 * Writes (=) every primitive's parameter gradient; culled primitives (n_touched == 0) get 0.
 * d_opacity_raw_in is the blend backward's accumulated raw-opacity gradient (passed through). */
void orc_preprocess_backward(int64_t n, const float *mean3d, const float *rotation, const float *logscale, const float *sh1,
                             const float *sh2, const float *sh3, int sh_degree, const orc_camera *cam,
                             const uint32_t *n_touched, const float *d_mean2d, const float *d_conic, const float *d_color,
                             const float *d_opacity_in, float *g_mean3d, float *g_rotation, float *g_logscale,
                             float *g_opacity, float *g_sh0, float *g_sh1, float *g_sh2, float *g_sh3)
{
    const float *w = cam->w2c;
    const float W = (float)cam->width, H = (float)cam->height;
    const int bases = (sh_degree + 1) * (sh_degree + 1);
#pragma omp parallel for schedule(static, 4096)
    for(int64_t i = 0; i < n; ++i) {
        memset(g_mean3d + i * 3, 0, 12);
        memset(g_rotation + i * 4, 0, 16);
        memset(g_logscale + i * 3, 0, 12);
        g_opacity[i] = 0.0f;
        memset(g_sh0 + i * 3, 0, 12);
        if(g_sh1) memset(g_sh1 + i * 9, 0, 36);
        if(g_sh2) memset(g_sh2 + i * 15, 0, 60);
        if(g_sh3) memset(g_sh3 + i * 21, 0, 84);
        if(n_touched[i] == 0) continue;
        g_opacity[i] = d_opacity_in[i];
        const double m0 = mean3d[i * 3 + 0], m1 = mean3d[i * 3 + 1], m2 = mean3d[i * 3 + 2];
        const double gc[3] = { d_color[i * 3 + 0], d_color[i * 3 + 1], d_color[i * 3 + 2] };
        double dmc[3] = { 0.0, 0.0, 0.0 };
        for(int c = 0; c < 3; ++c) g_sh0[i * 3 + c] = (float)(0.28209479177387814 * gc[c]);
        if(bases > 1) {
            const double xr = m0 - cam->cam_pos[0], yr = m1 - cam->cam_pos[1], zr = m2 - cam->cam_pos[2];
            const double nrm = sqrt(xr * xr + yr * yr + zr * zr);
            const double x = xr / nrm, y = yr / nrm, z = zr / nrm;
            double gdx[3], gdy[3], gdz[3];
            const float *c1 = sh1 + i * 9;
            for(int c = 0; c < 3; ++c) {
                g_sh1[i * 9 + 0 * 3 + c] = (float)(-0.48860251190291987 * y * gc[c]);
                g_sh1[i * 9 + 1 * 3 + c] = (float)(0.48860251190291987 * z * gc[c]);
                g_sh1[i * 9 + 2 * 3 + c] = (float)(-0.48860251190291987 * x * gc[c]);
                gdx[c] = -0.48860251190291987 * c1[2 * 3 + c];
                gdy[c] = -0.48860251190291987 * c1[0 * 3 + c];
                gdz[c] = 0.48860251190291987 * c1[1 * 3 + c];
            }
            if(bases > 4) {
                const double xx = x * x, yy = y * y, zz = z * z, xy = x * y, xz = x * z, yz = y * z;
                const float *c2 = sh2 + i * 15;
                for(int c = 0; c < 3; ++c) {
                    g_sh2[i * 15 + 0 * 3 + c] = (float)(1.0925484305920792 * xy * gc[c]);
                    g_sh2[i * 15 + 1 * 3 + c] = (float)(-1.0925484305920792 * yz * gc[c]);
                    g_sh2[i * 15 + 2 * 3 + c] = (float)((0.94617469575755997 * zz - 0.31539156525251999) * gc[c]);
                    g_sh2[i * 15 + 3 * 3 + c] = (float)(-1.0925484305920792 * xz * gc[c]);
                    g_sh2[i * 15 + 4 * 3 + c] = (float)((0.54627421529603959 * xx - 0.54627421529603959 * yy) * gc[c]);
                    gdx[c] += 1.0925484305920792 * y * c2[0 * 3 + c] - 1.0925484305920792 * z * c2[3 * 3 + c]
                        + 1.0925484305920792 * x * c2[4 * 3 + c];
                    gdy[c] += 1.0925484305920792 * x * c2[0 * 3 + c] - 1.0925484305920792 * z * c2[1 * 3 + c]
                        - 1.0925484305920792 * y * c2[4 * 3 + c];
                    gdz[c] += -1.0925484305920792 * y * c2[1 * 3 + c] + 1.8923493915151202 * z * c2[2 * 3 + c]
                        - 1.0925484305920792 * x * c2[3 * 3 + c];
                }
                if(bases > 9) {
                    const float *c3 = sh3 + i * 21;
                    for(int c = 0; c < 3; ++c) {
                        g_sh3[i * 21 + 0 * 3 + c] = (float)(0.59004358992664352 * y * (-3.0 * xx + yy) * gc[c]);
                        g_sh3[i * 21 + 1 * 3 + c] = (float)(2.8906114426405538 * xy * z * gc[c]);
                        g_sh3[i * 21 + 2 * 3 + c] = (float)(0.45704579946446572 * y * (1.0 - 5.0 * zz) * gc[c]);
                        g_sh3[i * 21 + 3 * 3 + c] = (float)(0.3731763325901154 * z * (5.0 * zz - 3.0) * gc[c]);
                        g_sh3[i * 21 + 4 * 3 + c] = (float)(0.45704579946446572 * x * (1.0 - 5.0 * zz) * gc[c]);
                        g_sh3[i * 21 + 5 * 3 + c] = (float)(1.4453057213202769 * z * (xx - yy) * gc[c]);
                        g_sh3[i * 21 + 6 * 3 + c] = (float)(0.59004358992664352 * x * (-xx + 3.0 * yy) * gc[c]);
                        gdx[c] += -3.5402615395598609 * xy * c3[0 * 3 + c] + 2.8906114426405538 * yz * c3[1 * 3 + c]
                            + (0.45704579946446572 - 2.2852289973223288 * zz) * c3[4 * 3 + c]
                            + 2.8906114426405538 * xz * c3[5 * 3 + c]
                            + (-1.7701307697799304 * xx + 1.7701307697799304 * yy) * c3[6 * 3 + c];
                        gdy[c] += (-1.7701307697799304 * xx + 1.7701307697799304 * yy) * c3[0 * 3 + c]
                            + 2.8906114426405538 * xz * c3[1 * 3 + c]
                            + (0.45704579946446572 - 2.2852289973223288 * zz) * c3[2 * 3 + c]
                            - 2.8906114426405538 * yz * c3[5 * 3 + c] + 3.5402615395598609 * xy * c3[6 * 3 + c];
                        gdz[c] += 2.8906114426405538 * xy * c3[1 * 3 + c] - 4.5704579946446566 * yz * c3[2 * 3 + c]
                            + (5.597644988851731 * zz - 1.1195289977703462) * c3[3 * 3 + c]
                            - 4.5704579946446566 * xz * c3[4 * 3 + c]
                            + (1.4453057213202769 * xx - 1.4453057213202769 * yy) * c3[5 * 3 + c];
                    }
                }
            }
            const double gd[3] = { gdx[0] * gc[0] + gdx[1] * gc[1] + gdx[2] * gc[2],
                                   gdy[0] * gc[0] + gdy[1] * gc[1] + gdy[2] * gc[2],
                                   gdz[0] * gc[0] + gdz[1] * gc[1] + gdz[2] * gc[2] };
            const double xx = xr * xr, yy = yr * yr, zz = zr * zr, xy = xr * yr, xz = xr * zr, yz = yr * zr;
            const double n3 = nrm * nrm * nrm;
            dmc[0] = ((yy + zz) * gd[0] - xy * gd[1] - xz * gd[2]) / n3;
            dmc[1] = (-xy * gd[0] + (xx + zz) * gd[1] - yz * gd[2]) / n3;
            dmc[2] = (-xz * gd[0] - yz * gd[1] + (xx + yy) * gd[2]) / n3;
        }
        const double r1[4] = { w[0], w[1], w[2], w[3] }, r2[4] = { w[4], w[5], w[6], w[7] }, r3[4] = { w[8], w[9], w[10], w[11] };
        const double depth = r3[0] * m0 + r3[1] * m1 + r3[2] * m2 + r3[3];
        const double x = (r1[0] * m0 + r1[1] * m1 + r1[2] * m2 + r1[3]) / depth;
        const double y = (r2[0] * m0 + r2[1] * m1 + r2[2] * m2 + r2[3]) / depth;
        double s[3], var[3];
        for(int k = 0; k < 3; ++k) {
            s[k] = exp((double)logscale[i * 3 + k]);
            var[k] = s[k] * s[k];
        }
        const double qx = rotation[i * 4 + 0], qy = rotation[i * 4 + 1], qz = rotation[i * 4 + 2], qr = rotation[i * 4 + 3];
        const double qn = qr * qr + qx * qx + qy * qy + qz * qz;
        const double qxx = 2 * qx * qx / qn, qyy = 2 * qy * qy / qn, qzz = 2 * qz * qz / qn;
        const double qxy = 2 * qx * qy / qn, qxz = 2 * qx * qz / qn, qyz = 2 * qy * qz / qn;
        const double qrx = 2 * qr * qx / qn, qry = 2 * qr * qy / qn, qrz = 2 * qr * qz / qn;
        const double R[9] = { 1 - (qyy + qzz), qxy - qrz, qry + qxz, qrz + qxy, 1 - (qxx + qzz), qyz - qrx, qxz - qry, qrx + qyz, 1 - (qxx + qyy) };
        double cov[3][3];
        for(int a = 0; a < 3; ++a)
            for(int b = 0; b < 3; ++b) cov[a][b] = R[a * 3 + 0] * var[0] * R[b * 3 + 0] + R[a * 3 + 1] * var[1] * R[b * 3 + 1] + R[a * 3 + 2] * var[2] * R[b * 3 + 2];
        const double fx = cam->fx, fy = cam->fy;
        const double cl = (-0.15f * W - cam->cx) / cam->fx, cr = (1.15f * W - cam->cx) / cam->fx;
        const double ct = (-0.15f * H - cam->cy) / cam->fy, cb = (1.15f * H - cam->cy) / cam->fy;
        const double tx = fmax(cl, fmin(x, cr)), ty = fmax(ct, fmin(y, cb));
        const double j11 = fx / depth, j13 = -j11 * tx, j22 = fy / depth, j23 = -j22 * ty;
        const double a1[3] = { j11 * r1[0] + j13 * r3[0], j11 * r1[1] + j13 * r3[1], j11 * r1[2] + j13 * r3[2] };
        const double a2[3] = { j22 * r2[0] + j23 * r3[0], j22 * r2[1] + j23 * r3[1], j22 * r2[2] + j23 * r3[2] };
        double b1[3], b2[3];
        for(int k = 0; k < 3; ++k) {
            b1[k] = a1[0] * cov[0][k] + a1[1] * cov[1][k] + a1[2] * cov[2][k];
            b2[k] = a2[0] * cov[0][k] + a2[1] * cov[1][k] + a2[2] * cov[2][k];
        }
        const double A = b1[0] * a1[0] + b1[1] * a1[1] + b1[2] * a1[2] + 0.3;
        const double B = b1[0] * a2[0] + b1[1] * a2[1] + b1[2] * a2[2];
        const double Cc = b2[0] * a2[0] + b2[1] * a2[1] + b2[2] * a2[2] + 0.3;
        const double det = A * Cc - B * B;
        const double idet2 = 1.0 / (det * det);
        const double dcx = d_conic[i * 3 + 0], dcy = d_conic[i * 3 + 1], dcz = d_conic[i * 3 + 2];
        const double dc2x = idet2 * (B * Cc * dcy - Cc * Cc * dcx - B * B * dcz);
        const double dc2y = idet2 * (B * Cc * dcx - 0.5 * (A * Cc + B * B) * dcy + A * B * dcz);
        const double dc2z = idet2 * (A * B * dcy - B * B * dcx - A * A * dcz);
        double dcov3[3][3];
        for(int a = 0; a < 3; ++a)
            for(int b = 0; b < 3; ++b)
                dcov3[a][b] = a1[a] * a1[b] * dc2x + (a1[a] * a2[b] + a1[b] * a2[a]) * dc2y + a2[a] * a2[b] * dc2z;
        const double djw1[3] = { 2 * (b1[0] * dc2x + b2[0] * dc2y), 2 * (b1[1] * dc2x + b2[1] * dc2y), 2 * (b1[2] * dc2x + b2[2] * dc2y) };
        const double djw2[3] = { 2 * (b1[0] * dc2y + b2[0] * dc2z), 2 * (b1[1] * dc2y + b2[1] * dc2z), 2 * (b1[2] * dc2y + b2[2] * dc2z) };
        const double dj11 = r1[0] * djw1[0] + r1[1] * djw1[1] + r1[2] * djw1[2];
        const double dj22 = r2[0] * djw2[0] + r2[1] * djw2[1] + r2[2] * djw2[2];
        const double dj13 = r3[0] * djw1[0] + r3[1] * djw1[1] + r3[2] * djw1[2];
        const double dj23 = r3[0] * djw2[0] + r3[1] * djw2[1] + r3[2] * djw2[2];
        const double dtx = (x > cl && x < cr) ? 1.0 : 0.0, dty = (y > ct && y < cb) ? 1.0 : 0.0;
        const double dj13c = dj13 * dtx, dj23c = dj23 * dty;
        const double h1 = dj11 - 2.0 * tx * dj13c, h2 = dj22 - 2.0 * ty * dj23c;
        const double dm2x = d_mean2d[i * 2 + 0], dm2y = d_mean2d[i * 2 + 1];
        const double dcam[3] = { j11 * (dm2x - dj13c / depth), j22 * (dm2y - dj23c / depth),
                                 -j11 * (x * dm2x + h1 / depth) - j22 * (y * dm2y + h2 / depth) };
        for(int k = 0; k < 3; ++k) g_mean3d[i * 3 + k] = (float)(r1[k] * dcam[0] + r2[k] * dcam[1] + r3[k] * dcam[2] + dmc[k]);
        /* d cov3d -> d (R S): dRS = 2 dcov3 RS */
        double RS[9], dRS[9];
        for(int a = 0; a < 3; ++a)
            for(int b = 0; b < 3; ++b) RS[a * 3 + b] = R[a * 3 + b] * s[b];
        for(int a = 0; a < 3; ++a)
            for(int b = 0; b < 3; ++b) dRS[a * 3 + b] = 2.0 * (dcov3[a][0] * RS[0 * 3 + b] + dcov3[a][1] * RS[1 * 3 + b] + dcov3[a][2] * RS[2 * 3 + b]);
        for(int b = 0; b < 3; ++b)
            g_logscale[i * 3 + b] = (float)((dRS[0 * 3 + b] * R[0 * 3 + b] + dRS[1 * 3 + b] * R[1 * 3 + b] + dRS[2 * 3 + b] * R[2 * 3 + b]) * s[b]);
        double dR[9];
        for(int a = 0; a < 3; ++a)
            for(int b = 0; b < 3; ++b) dR[a * 3 + b] = dRS[a * 3 + b] * s[b];
        const double qnorm = sqrt(qn), iq = 1.0 / qnorm;
        const double w_ = qr * iq, x_ = qx * iq, y_ = qy * iq, z_ = qz * iq;
        const double dw = dR[1] * (-2 * z_) + dR[2] * (2 * y_) + dR[3] * (2 * z_) + dR[5] * (-2 * x_) + dR[6] * (-2 * y_) + dR[7] * (2 * x_);
        const double dx_ = dR[1] * (2 * y_) + dR[2] * (2 * z_) + dR[3] * (2 * y_) + dR[4] * (-4 * x_) + dR[5] * (-2 * w_) + dR[6] * (2 * z_) + dR[7] * (2 * w_) + dR[8] * (-4 * x_);
        const double dy_ = dR[0] * (-4 * y_) + dR[1] * (2 * x_) + dR[2] * (2 * w_) + dR[3] * (2 * x_) + dR[5] * (2 * z_) + dR[6] * (-2 * w_) + dR[7] * (2 * z_) + dR[8] * (-4 * y_);
        const double dz_ = dR[0] * (-4 * z_) + dR[1] * (-2 * w_) + dR[2] * (2 * x_) + dR[3] * (2 * w_) + dR[4] * (-4 * z_) + dR[5] * (2 * y_) + dR[6] * (2 * x_) + dR[7] * (2 * y_);
        const double dotq = w_ * dw + x_ * dx_ + y_ * dy_ + z_ * dz_;
        g_rotation[i * 4 + 0] = (float)((dx_ - x_ * dotq) * iq);
        g_rotation[i * 4 + 1] = (float)((dy_ - y_ * dotq) * iq);
        g_rotation[i * 4 + 2] = (float)((dz_ - z_ * dotq) * iq);
        g_rotation[i * 4 + 3] = (float)((dw - w_ * dotq) * iq);
    }
}

/* ---------------------------------------------------------------- losses
 * L1: gsx-cuda/loss-pointwise-kernels.cu:43-89 (loss_map += scale*|p-t|; grad += sign(p-t)*grad_scale).
 * SSIM: gsx-cpu/loss.c:397-556 in fp64 (11x11 Gaussian window sigma 1.5, zero padding, C1=0.01^2,
 * C2=0.03^2, 5-px border: loss_map set to 0 and partials zeroed), layout [outer, C, H, W]. */
void orc_l1_forward(int64_t n, const float *p, const float *t, float *loss_map, float scale)
{
    for(int64_t i = 0; i < n; ++i) loss_map[i] += scale * fabsf(p[i] - t[i]);
}

void orc_l1_backward(int64_t n, const float *p, const float *t, float *grad, float grad_scale)
{
    for(int64_t i = 0; i < n; ++i) {
        const float d = p[i] - t[i];
        const float s = d > 0.0f ? 1.0f : (d < 0.0f ? -1.0f : 0.0f);
        grad[i] += s * grad_scale;
    }
}

static double orc_gauss[11];
static void orc_init_gauss(void)
{
    double sum = 0.0;
    for(int k = 0; k < 11; ++k) {
        const double d = (double)(k - 5);
        orc_gauss[k] = exp(-(d * d) / (2.0 * 1.5 * 1.5));
        sum += orc_gauss[k];
    }
    for(int k = 0; k < 11; ++k) orc_gauss[k] /= sum;
}

/* loss_map may be NULL (no forward accumulation); grad may be NULL (no backward). */
int orc_ssim(int64_t outer, int channels, int height, int width, const float *p, const float *t, float *loss_map,
             float loss_scale, float *grad, float grad_scale)
{
    orc_init_gauss();
    const size_t plane = (size_t)height * (size_t)width;
    double *dmu = (double *)calloc(plane, sizeof(double));
    double *ds1 = (double *)calloc(plane, sizeof(double));
    double *ds12 = (double *)calloc(plane, sizeof(double));
    if(dmu == NULL || ds1 == NULL || ds12 == NULL) {
        free(dmu); free(ds1); free(ds12);
        return -1;
    }
    for(int64_t o = 0; o < outer; ++o) {
        for(int c = 0; c < channels; ++c) {
            const size_t base = ((size_t)o * (size_t)channels + (size_t)c) * plane;
            const float *P = p + base, *Tt = t + base;
            /* rows in parallel; every output and partial is per pixel */
#pragma omp parallel for schedule(static, 8)
            for(int y = 0; y < height; ++y) {
                for(int x = 0; x < width; ++x) {
                    double mu1 = 0, mu2 = 0, s11 = 0, s22 = 0, s12 = 0;
                    for(int ky = -5; ky <= 5; ++ky) {
                        const int yy = y + ky;
                        if(yy < 0 || yy >= height) continue;
                        for(int kx = -5; kx <= 5; ++kx) {
                            const int xx = x + kx;
                            if(xx < 0 || xx >= width) continue;
                            const double wgt = orc_gauss[ky + 5] * orc_gauss[kx + 5];
                            const double a = P[(size_t)yy * width + xx], b = Tt[(size_t)yy * width + xx];
                            mu1 += wgt * a; mu2 += wgt * b; s11 += wgt * a * a; s22 += wgt * b * b; s12 += wgt * a * b;
                        }
                    }
                    const double sg1 = s11 - mu1 * mu1, sg2 = s22 - mu2 * mu2, sg12 = s12 - mu1 * mu2;
                    const double A = mu1 * mu1 + mu2 * mu2 + 1e-4, B = sg1 + sg2 + 9e-4;
                    const double Cn = 2 * mu1 * mu2 + 1e-4, D = 2 * sg12 + 9e-4;
                    const double ssim = (Cn * D) / (A * B);
                    const size_t idx = (size_t)y * width + x;
                    const int border = y < 5 || y >= height - 5 || x < 5 || x >= width - 5;
                    if(loss_map) {
                        if(border) loss_map[base + idx] = 0.0f;
                        else loss_map[base + idx] += (float)((1.0 - ssim) * loss_scale);
                    }
                    if(border) {
                        dmu[idx] = ds1[idx] = ds12[idx] = 0.0;
                    } else {
                        const double ab = A * B;
                        dmu[idx] = (2 * mu2 * D) / ab - (2 * mu2 * Cn) / ab - (2 * mu1 * Cn * D) / (A * ab) + (2 * mu1 * Cn * D) / (ab * B);
                        ds1[idx] = -(Cn * D) / (ab * B);
                        ds12[idx] = (2 * Cn) / ab;
                    }
                }
            }
            if(grad) {
#pragma omp parallel for schedule(static, 8)
                for(int y = 0; y < height; ++y) {
                    for(int x = 0; x < width; ++x) {
                        double c0 = 0, c1 = 0, c2 = 0;
                        for(int ky = -5; ky <= 5; ++ky) {
                            const int yy = y + ky;
                            if(yy < 0 || yy >= height) continue;
                            for(int kx = -5; kx <= 5; ++kx) {
                                const int xx = x + kx;
                                if(xx < 0 || xx >= width) continue;
                                const double wgt = orc_gauss[ky + 5] * orc_gauss[kx + 5];
                                const size_t j = (size_t)yy * width + xx;
                                c0 += dmu[j] * wgt; c1 += ds1[j] * wgt; c2 += ds12[j] * wgt;
                            }
                        }
                        const size_t idx = (size_t)y * width + x;
                        const double g = -(c0 + 2.0 * (double)P[idx] * c1 + (double)Tt[idx] * c2) * (double)grad_scale;
                        grad[base + idx] += (float)g;
                    }
                }
            }
        }
    }
    free(dmu); free(ds1); free(ds12);
    return 0;
}

/* ---------------------------------------------------------------- Adam
 * gsx-cuda/gsx-cuda-kernels.cu:279-321 with the host-side fp64 bias corrections of
 * gsx-cuda/optim.c:776-793 (inv_c = 1 / (1 - beta^t) in double). */
void orc_adam(int64_t n, float *param, const float *grad, float *m1, float *m2, float beta1, float beta2, float lr,
              float weight_decay, float eps, float max_grad, double inv_c1, double inv_c2)
{
#pragma omp parallel for schedule(static, 65536)
    for(int64_t i = 0; i < n; ++i) {
        float g = grad[i];
        if(max_grad > 0.0f) {
            if(g > max_grad) g = max_grad;
            else if(g < -max_grad) g = -max_grad;
        }
        const float a = beta1 * m1[i] + (1.0f - beta1) * g;
        const float b = beta2 * m2[i] + (1.0f - beta2) * g * g;
        const float ah = (float)((double)a * inv_c1);
        const float bh = (float)((double)b * inv_c2);
        float pv = param[i];
        m1[i] = a;
        m2[i] = b;
        if(weight_decay > 0.0f) pv -= lr * weight_decay * pv;
        pv -= lr * (ah / (sqrtf(bh) + eps));
        param[i] = pv;
    }
}

/* exported for tests/test_oracle_pins.py: the deterministic exp/log the oracle and kernels share */
float orc_expf(float x) { return gsx_expf(x); }
float orc_logf(float x) { return gsx_logf(x); }
