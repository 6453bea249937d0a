/*
 * tgs_oracle.c -- CPU restatement of the tinygs training hot path.
 *
 * TEST INFRASTRUCTURE ONLY (see tgs_oracle.h).  Parity status: UNPINNED --
 * the reference has no golden vectors for this path and cannot be built in
 * this environment; each function below restates the reference source it
 * cites.  Paths are relative to the root of Adversarr/tinygs.
 *
 * Build: oracle/build_oracle.py (gcc -O2 -fopenmp -ffp-contract=off).
 */
#include "tgs_oracle.h"

#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define TILE 16
#define BLOCK 256
#define FRAGILE_REL 2e-5f

/* Timing samples only (bench.py's CPU baseline): the blend stages process
 * tiles t with t % g_tile_stride == 0 and skip the rest.  1 = every tile. */
static int g_tile_stride = 1;
void orc_set_tile_stride(int32_t stride) { g_tile_stride = stride > 0 ? stride : 1; }

/* Finite-difference checks only: a smooth variant of the fp32 forward (every
 * tile of the grid is touched, no alpha < 1/255 cut, no early termination),
 * of which the restated backward is the exact derivative. */
static int g_smooth = 0;
/* Width of the fp16 path's fragile band around the tile test's threshold,
 * relative to max(|threshold|, 1).  The oracle's half-precision inputs come
 * from IEEE fp32 arithmetic and the GPU's from fast-math fp32, which round
 * to different half values for a small fraction of Gaussians (one half ulp,
 * 2^-11 relative); tile decisions within a few half ulps of the threshold
 * can then differ. */
static float g_fragile_f16 = 2e-2f;
void orc_set_fragile_f16(float rel) { g_fragile_f16 = rel > 0.0f ? rel : 2e-2f; }
/* Optional per-pixel record of blend decisions near their thresholds (alpha
 * against 1/255 and against its cap, the transmittance stop at 1e-4), within
 * `g_pix_band` relative: the pixels whose value an end-to-end comparison
 * from the parameters cannot pin, since upstream last-bit differences of a
 * conic move such a decision.  One byte per pixel of the tiled plane. */
static uint8_t* g_pix_fragile = NULL;
static float g_pix_band = 0.0f;
void orc_set_pixel_fragile(uint8_t* buf, float band) {
    g_pix_fragile = buf;
    g_pix_band = band;
}
static inline int near_rel(float v, float thr, float band) { return fabsf(v - thr) <= band * fabsf(thr); }
void orc_set_smooth_forward(int32_t on) { g_smooth = on != 0; }

/* ---------------------------------------------------------------- helpers */

static inline float satf(float x) { return x > 0.f ? (x < 1.f ? x : 1.f) : 0.f; }
static inline float clampf(float x, float lo, float hi) { return fminf(fmaxf(x, lo), hi); }

/* 8x8-tiled physical index, tinygs/include/tinygs/common.hpp:389-408. */
static inline uint32_t tiled_index(uint32_t y, uint32_t x, uint32_t tiled_w) {
    return (((y >> 3) * tiled_w + (x >> 3)) << 6) + ((y & 7u) << 3) + (x & 7u);
}

static inline int near_threshold(float v, float thr) {
    float scale = fmaxf(fabsf(thr), 1e-6f);
    return fabsf(v - thr) <= FRAGILE_REL * scale;
}

static void set_threads(int32_t n_threads) {
#ifdef _OPENMP
    if (n_threads > 0) omp_set_num_threads(n_threads);
#else
    (void)n_threads;
#endif
}

/* IEEE 754 binary16, round to nearest even, written from the standard. */
static uint16_t f2h_double(double d) {
    uint16_t sign = signbit(d) ? 0x8000u : 0u;
    double a = fabs(d);
    if (isnan(d)) return (uint16_t)(sign | 0x7e00u);
    if (a >= 65520.0) return (uint16_t)(sign | 0x7c00u); /* rounds to inf */
    if (a < ldexp(1.0, -25)) {                         /* below half of min subnormal */
        if (a == ldexp(1.0, -25)) return sign;          /* tie to even -> 0 */
        return sign;
    }
    int e;
    double m = frexp(a, &e); /* a = m * 2^e, m in [0.5, 1) */
    int exp_h = e - 1;       /* a = (2m) * 2^(e-1) */
    if (exp_h < -14) {
        /* subnormal: units of 2^-24 */
        double q = ldexp(a, 24);
        double r = nearbyint(q); /* default rounding mode is RN-even */
        return (uint16_t)(sign | (uint16_t)r);
    }
    double frac = ldexp(2.0 * m - 1.0, 10); /* 10 fraction bits */
    double r = nearbyint(frac);
    uint32_t bits;
    if (r >= 1024.0) { /* mantissa overflow into next exponent */
        exp_h += 1;
        r = 0.0;
    }
    if (exp_h > 15) return (uint16_t)(sign | 0x7c00u);
    bits = ((uint32_t)(exp_h + 15) << 10) | (uint32_t)r;
    return (uint16_t)(sign | bits);
}

uint16_t orc_f2h(float f) { return f2h_double((double)f); }

float orc_h2f(uint16_t h) {
    uint32_t sign = (h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t man = h & 0x3ffu;
    float v;
    if (exp == 0) {
        v = ldexpf((float)man, -24);
    } else if (exp == 31) {
        v = man ? NAN : INFINITY;
    } else {
        v = ldexpf((float)(man | 0x400u), (int)exp - 25);
    }
    union { float f; uint32_t u; } c;
    c.f = v;
    c.u |= sign;
    return c.f;
}

/* Round toward -inf to binary16 (cuda __float2half_rd semantics). */
static uint16_t f2h_rd(double d) {
    uint16_t h = f2h_double(d);
    double back = (double)orc_h2f(h);
    if (isnan(d)) return h;
    if (back > d) {
        /* step one ulp toward -inf */
        if (h == 0x0000u) return 0x8001u;
        if (h & 0x8000u) return (uint16_t)(h + 1u);
        return (uint16_t)(h - 1u);
    }
    return h;
}

/* Half arithmetic emulated in double (exact for these inputs) then rounded. */
static inline uint16_t hmul(uint16_t a, uint16_t b) { return f2h_double((double)orc_h2f(a) * (double)orc_h2f(b)); }
static inline uint16_t hadd(uint16_t a, uint16_t b) { return f2h_double((double)orc_h2f(a) + (double)orc_h2f(b)); }
static inline uint16_t hsub(uint16_t a, uint16_t b) { return f2h_double((double)orc_h2f(a) - (double)orc_h2f(b)); }
static inline uint16_t hfma(uint16_t a, uint16_t b, uint16_t c) {
    return f2h_double(fma((double)orc_h2f(a), (double)orc_h2f(b), (double)orc_h2f(c)));
}
static inline uint16_t hneg(uint16_t a) { return (uint16_t)(a ^ 0x8000u); }
static inline uint16_t hdiv(uint16_t a, uint16_t b) { return f2h_double((double)orc_h2f(a) / (double)orc_h2f(b)); }
static inline uint16_t hmin(uint16_t a, uint16_t b) {
    float fa = orc_h2f(a), fb = orc_h2f(b);
    if (isnan(fa)) return b;
    if (isnan(fb)) return a;
    return fa < fb ? a : b;
}
static inline uint16_t hsat(uint16_t a) {
    float f = orc_h2f(a);
    if (!(f > 0.f)) return 0;
    if (f >= 1.f) return 0x3c00u;
    return a;
}
/* ex2.approx.f16x2 stand-in: correctly rounded 2^x (the hardware op is an
 * approximation; this is the single non-bit-exact step of the emulation). */
static inline uint16_t hex2(uint16_t a) { return f2h_double(exp2((double)orc_h2f(a))); }

/* c2w translation of the inverse of the row-major w2c, computed in double.
 * The reference takes c2w[3] of glm::inverse(w2c) (fastgs.cu:97-100). */
void orc_camera_position(const OrcCamera* cam, float out[3]) {
    const float* m = cam->w2c;
    double r[3][3], t[3];
    for (int i = 0; i < 3; ++i) {
        for (int j = 0; j < 3; ++j) r[i][j] = m[4 * i + j];
        t[i] = m[4 * i + 3];
    }
    /* general 3x3 inverse of the linear part, then -inv * t */
    double c00 = r[1][1] * r[2][2] - r[1][2] * r[2][1];
    double c01 = r[1][2] * r[2][0] - r[1][0] * r[2][2];
    double c02 = r[1][0] * r[2][1] - r[1][1] * r[2][0];
    double det = r[0][0] * c00 + r[0][1] * c01 + r[0][2] * c02;
    double inv[3][3];
    inv[0][0] = c00 / det;
    inv[0][1] = (r[0][2] * r[2][1] - r[0][1] * r[2][2]) / det;
    inv[0][2] = (r[0][1] * r[1][2] - r[0][2] * r[1][1]) / det;
    inv[1][0] = c01 / det;
    inv[1][1] = (r[0][0] * r[2][2] - r[0][2] * r[2][0]) / det;
    inv[1][2] = (r[0][2] * r[1][0] - r[0][0] * r[1][2]) / det;
    inv[2][0] = c02 / det;
    inv[2][1] = (r[0][1] * r[2][0] - r[0][0] * r[2][1]) / det;
    inv[2][2] = (r[0][0] * r[1][1] - r[0][1] * r[1][0]) / det;
    for (int i = 0; i < 3; ++i)
        out[i] = (float)(-(inv[i][0] * t[0] + inv[i][1] * t[1] + inv[i][2] * t[2]));
}

/* ------------------------------------------------------------- preprocess */

/* SH colour, fastgs_ours/kernels_forward.cuh:22-46 (constants are the real
 * spherical-harmonic normalisation factors of degrees 0..3). */
static void sh_to_color(const float* sh0, const float* rest, int active_bases,
                        const float pos[3], const float cam[3], float out[3]) {
    for (int c = 0; c < 3; ++c) out[c] = 0.5f + 0.28209479177387814f * sh0[c];
    if (active_bases <= 1) return;
    float dx = pos[0] - cam[0], dy = pos[1] - cam[1], dz = pos[2] - cam[2];
    float inv = 1.0f / sqrtf(dx * dx + dy * dy + dz * dz);
    float x = dx * inv, y = dy * inv, z = dz * inv;
    float b[15];
    b[0] = -0.48860251190291987f * y;
    b[1] = 0.48860251190291987f * z;
    b[2] = -0.48860251190291987f * x;
    int nb = 3;
    if (active_bases > 4) {
        float xx = x * x, yy = y * y, zz = z * z, xy = x * y, xz = x * z, yz = y * z;
        b[3] = 1.0925484305920792f * xy;
        b[4] = -1.0925484305920792f * yz;
        b[5] = 0.94617469575755997f * zz - 0.31539156525251999f;
        b[6] = -1.0925484305920792f * xz;
        b[7] = 0.54627421529603959f * xx - 0.54627421529603959f * yy;
        nb = 8;
        if (active_bases > 9) {
            b[8] = 0.59004358992664352f * y * (-3.0f * xx + yy);
            b[9] = 2.8906114426405538f * xy * z;
            b[10] = 0.45704579946446572f * y * (1.0f - 5.0f * zz);
            b[11] = 0.3731763325901154f * z * (5.0f * zz - 3.0f);
            b[12] = 0.45704579946446572f * x * (1.0f - 5.0f * zz);
            b[13] = 1.4453057213202769f * z * (xx - yy);
            b[14] = 0.59004358992664352f * x * (-xx + 3.0f * yy);
            nb = 15;
        }
    }
    for (int k = 0; k < nb; ++k)
        for (int c = 0; c < 3; ++c) out[c] += b[k] * rest[3 * k + c];
}

/* StopThePop tile test, fastgs_ours/kernels_forward.cuh:49-84.  Returns the
 * decision; *margin receives max_power - threshold. */
static int tile_test_f32(float mx, float my, const float conic[3], uint32_t tx,
                         uint32_t ty, float thr, float* margin) {
    float rminx = (float)(tx * TILE), rminy = (float)(ty * TILE);
    float rmaxx = (float)((tx + 1) * TILE - 1), rmaxy = (float)((ty + 1) * TILE - 1);
    float xmd = rminx - mx, ymd = rminy - my;
    float xl = xmd > 0.f ? 1.f : 0.f;
    float nix = xl + (mx > rmaxx ? 1.f : 0.f);
    float ya = ymd > 0.f ? 1.f : 0.f;
    float niy = ya + (my > rmaxy ? 1.f : 0.f);
    if (niy + nix == 0.f) {
        *margin = -INFINITY;
        return 1;
    }
    float ccx = rmaxx + xl * (rminx - rmaxx);
    float ccy = rmaxy + ya * (rminy - rmaxy);
    float dfx = mx - ccx, dfy = my - ccy;
    float dx = copysignf(15.f, xmd), dy = copysignf(15.f, ymd);
    float t0 = niy * satf((dx * conic[0] * dfx + dx * conic[1] * dfy) / (dx * conic[0] * dx));
    float t1 = nix * satf((dy * conic[1] * dfx + dy * conic[2] * dfy) / (dy * conic[2] * dy));
    float px = ccx + t0 * dx, py = ccy + t1 * dy;
    float ex = mx - px, ey = my - py;
    float p = 0.5f * (conic[0] * ex * ex + conic[2] * ey * ey) + conic[1] * ex * ey;
    *margin = p - thr;
    return p <= thr;
}

/* Half-precision tile test, fastgs_ours_fp16/kernels_forward.cuh:123-169. */
static int tile_test_f16(float mx, float my, uint16_t cx, uint16_t cy, uint16_t cz,
                         uint32_t tx, uint32_t ty, float thr, float* margin) {
    const uint16_t one = 0x3c00u, zero = 0u;
    const uint16_t ts = f2h_rd(15.0 / 16.0);
    uint16_t mdx = f2h_rd((double)((float)tx - mx * (1.0f / TILE)));
    uint16_t mdy = f2h_rd((double)((float)ty - my * (1.0f / TILE)));
    uint16_t Mdx = hadd(mdx, ts), Mdy = hadd(mdy, ts);
    /* unordered comparisons: true when either operand is NaN */
    float fmdx = orc_h2f(mdx), fmdy = orc_h2f(mdy), fMdx = orc_h2f(Mdx), fMdy = orc_h2f(Mdy);
    uint16_t xl = (isnan(fmdx) || fmdx > 0.f) ? one : zero;
    uint16_t ya = (isnan(fmdy) || fmdy > 0.f) ? one : zero;
    uint16_t xr = (isnan(fMdx) || fMdx < 0.f) ? one : zero;
    uint16_t yb = (isnan(fMdy) || fMdy < 0.f) ? one : zero;
    uint16_t nrx = hadd(xl, xr), nry = hadd(ya, yb);
    if (orc_h2f(nrx) == 0.f && orc_h2f(nry) == 0.f) {
        *margin = -INFINITY;
        return 1;
    }
    uint16_t dX = (uint16_t)((ts & 0x7fffu) | (mdx & 0x8000u));
    uint16_t dY = (uint16_t)((ts & 0x7fffu) | (mdy & 0x8000u));
    /* diff = -lerp(max_diff, min_diff, t) with lerp(v0,v1,t) = fma(t, v1, fma(-t, v0, v0)) */
    uint16_t difx = hneg(hfma(xl, mdx, hfma(hneg(xl), Mdx, Mdx)));
    uint16_t dify = hneg(hfma(ya, mdy, hfma(hneg(ya), Mdy, Mdy)));
    /* t_raw = (d*xy*diff_xx + d*yz*diff_yy) / (d*d*xz), lanes (x, y) */
    uint16_t numx = hadd(hmul(hmul(dX, cx), difx), hmul(hmul(dX, cy), dify));
    uint16_t numy = hadd(hmul(hmul(dY, cy), difx), hmul(hmul(dY, cz), dify));
    uint16_t denx = hmul(hmul(dX, dX), cx);
    uint16_t deny = hmul(hmul(dY, dY), cz);
    uint16_t trx = hdiv(numx, denx), try_ = hdiv(numy, deny);
    /* saturating multiply with the swapped not-in-range flags */
    uint16_t tX = hsat(hmul(trx, nry));
    uint16_t tY = hsat(hmul(try_, nrx));
    float ex = orc_h2f(hsub(difx, hmul(tX, dX))) * (float)TILE;
    float ey = orc_h2f(hsub(dify, hmul(tY, dY))) * (float)TILE;
    float fx = orc_h2f(cx), fy = orc_h2f(cy), fz = orc_h2f(cz);
    float p = 0.5f * (fx * ex * ex + fz * ey * ey) + fy * ex * ey;
    *margin = p - thr;
    return p <= thr;
}

typedef struct {
    int active1; /* survived depth/opacity/quaternion checks */
    int reach2;  /* reached the covariance stage (warp-level) */
} PreState;

void orc_preprocess(int64_t n, const float* means, const float* opacities,
                    const float* rotations, const float* scales,
                    const float* sh0, const float* sh_rest, int32_t sh_degree,
                    const OrcCamera* cam, int32_t fp16, OrcPrimitives* out,
                    float* dens, int32_t n_threads) {
    set_threads(n_threads);
    const float* r1 = cam->w2c;
    const float* r2 = cam->w2c + 4;
    const float* r3 = cam->w2c + 8;
    const float w = (float)cam->width, h = (float)cam->height;
    const uint32_t gw = (uint32_t)((cam->width + TILE - 1) / TILE);
    const uint32_t gh = (uint32_t)((cam->height + TILE - 1) / TILE);
    const int active_bases = (sh_degree + 1) * (sh_degree + 1);
    float campos[3];
    orc_camera_position(cam, campos);

    /* pass 1: the checks before the first warp-level exit (kernel lines
     * 229-271 fp32 / 300-349 fp16), needed to reproduce which warps carry on */
    int64_t n_warps = (n + 31) / 32;
    uint8_t* warp_alive = (uint8_t*)calloc((size_t)(n_warps > 0 ? n_warps : 1), 1);
    uint8_t* act = (uint8_t*)calloc((size_t)(n > 0 ? n : 1), 1);

#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        const float* m = means + 3 * i;
        float depth = r3[0] * m[0] + r3[1] * m[1] + r3[2] * m[2] + r3[3];
        int a = !(depth < cam->near_plane || depth > cam->far_plane);
        float op;
        if (fp16) {
            uint16_t raw_h = a ? orc_f2h(opacities[i]) : 0;
            op = 1.0f / (1.0f + expf(-orc_h2f(raw_h)));
        } else {
            op = 1.0f / (1.0f + expf(-opacities[i]));
        }
        if (op < 1.0f / 255.0f) a = 0;
        const float* q = rotations + 4 * i;
        float qn = 0.f;
        if (!fp16 || a) qn = q[0] * q[0] + q[1] * q[1] + q[2] * q[2] + q[3] * q[3];
        if (qn < 1e-8f) a = 0;
        act[i] = (uint8_t)a;
    }
    for (int64_t i = 0; i < n; ++i)
        if (act[i]) warp_alive[i / 32] = 1;

#pragma omp parallel for schedule(dynamic, 256)
    for (int64_t i = 0; i < n; ++i) {
        out->n_touched[i] = 0;
        out->fragile[i] = 0;
        if (!warp_alive[i / 32]) continue;
        const float* m = means + 3 * i;
        int active = act[i];
        uint8_t fragile = 0;
        float depth = r3[0] * m[0] + r3[1] * m[1] + r3[2] * m[2] + r3[3];
        if (near_threshold(depth, cam->near_plane) || near_threshold(depth, cam->far_plane)) fragile = 1;
        float opacity;
        uint16_t opacity_h = 0;
        if (fp16) {
            int a0 = !(depth < cam->near_plane || depth > cam->far_plane);
            uint16_t raw_h = a0 ? orc_f2h(opacities[i]) : 0;
            float f = 1.0f / (1.0f + expf(-orc_h2f(raw_h)));
            if (near_threshold(f, 1.0f / 255.0f)) fragile = 1;
            opacity_h = orc_f2h(f);
            opacity = f;
        } else {
            opacity = 1.0f / (1.0f + expf(-opacities[i]));
            if (near_threshold(opacity, 1.0f / 255.0f)) fragile = 1;
        }
        const float* s = scales + 3 * i;
        float v0 = expf(s[0]) * expf(s[0]), v1 = expf(s[1]) * expf(s[1]), v2 = expf(s[2]) * expf(s[2]);
        const float* q = rotations + 4 * i;
        float qr = q[0], qx = q[1], qy = q[2], qz = q[3];
        if (fp16 && !act[i]) {
            /* the fp16 kernel only loads the rotation for active lanes */
            int a0 = !(depth < cam->near_plane || depth > cam->far_plane);
            if (!a0 || opacity < 1.0f / 255.0f) { qr = qx = qy = qz = 0.f; }
        }
        float qrr = qr * qr, qxx_ = qx * qx, qyy_ = qy * qy, qzz_ = qz * qz;
        float qn = qrr + qxx_ + qyy_ + qzz_;
        float qxx = 2.0f * qxx_ / qn, qyy = 2.0f * qyy_ / qn, qzz = 2.0f * qzz_ / qn;
        float qxy = 2.0f * qx * qy / qn, qxz = 2.0f * qx * qz / qn, qyz = 2.0f * qy * qz / qn;
        float qrx = 2.0f * qr * qx / qn, qry = 2.0f * qr * qy / qn, qrz = 2.0f * qr * qz / qn;
        float R[3][3] = {{1.0f - (qyy + qzz), qxy - qrz, qry + qxz},
                         {qrz + qxy, 1.0f - (qxx + qzz), qyz - qrx},
                         {qxz - qry, qrx + qyz, 1.0f - (qxx + qyy)}};
        float var[3] = {v0, v1, v2};
        float RS[3][3];
        for (int a = 0; a < 3; ++a)
            for (int b = 0; b < 3; ++b) RS[a][b] = R[a][b] * var[b];
        float c11 = RS[0][0] * R[0][0] + RS[0][1] * R[0][1] + RS[0][2] * R[0][2];
        float c12 = RS[0][0] * R[1][0] + RS[0][1] * R[1][1] + RS[0][2] * R[1][2];
        float c13 = RS[0][0] * R[2][0] + RS[0][1] * R[2][1] + RS[0][2] * R[2][2];
        float c22 = RS[1][0] * R[1][0] + RS[1][1] * R[1][1] + RS[1][2] * R[1][2];
        float c23 = RS[1][0] * R[2][0] + RS[1][1] * R[2][1] + RS[1][2] * R[2][2];
        float c33 = RS[2][0] * R[2][0] + RS[2][1] * R[2][1] + RS[2][2] * R[2][2];

        float x = (r1[0] * m[0] + r1[1] * m[1] + r1[2] * m[2] + r1[3]) / depth;
        float y = (r2[0] * m[0] + r2[1] * m[1] + r2[2] * m[2] + r2[3]) / depth;
        float cl = (-0.15f * w - cam->cx) / cam->fx, cr = (1.15f * w - cam->cx) / cam->fx;
        float ct = (-0.15f * h - cam->cy) / cam->fy, cb = (1.15f * h - cam->cy) / cam->fy;
        float tx = clampf(x, cl, cr), ty = clampf(y, ct, cb);
        float j11 = cam->fx / depth, j13 = -j11 * tx, j22 = cam->fy / depth, j23 = -j22 * ty;
        float a1x = j11 * r1[0] + j13 * r3[0], a1y = j11 * r1[1] + j13 * r3[1], a1z = j11 * r1[2] + j13 * r3[2];
        float a2x = j22 * r2[0] + j23 * r3[0], a2y = j22 * r2[1] + j23 * r3[1], a2z = j22 * r2[2] + j23 * r3[2];
        float b1x = a1x * c11 + a1y * c12 + a1z * c13;
        float b1y = a1x * c12 + a1y * c22 + a1z * c23;
        float b1z = a1x * c13 + a1y * c23 + a1z * c33;
        float b2x = a2x * c11 + a2y * c12 + a2z * c13;
        float b2y = a2x * c12 + a2y * c22 + a2z * c23;
        float b2z = a2x * c13 + a2y * c23 + a2z * c33;
        float cov_a = b1x * a1x + b1y * a1y + b1z * a1z + 0.3f;
        float cov_b = b1x * a2x + b1y * a2y + b1z * a2z;
        float cov_c = b2x * a2x + b2y * a2y + b2z * a2z + 0.3f;
        float det = cov_a * cov_c - cov_b * cov_b;
        if (det < 1e-8f) active = 0;
        if (near_threshold(det, 1e-8f)) fragile = 1;
        float conic[3] = {cov_c / det, -cov_b / det, cov_a / det};
        if (dens) {
            float mid = 0.5f * (cov_a + cov_c);
            float l1 = mid + sqrtf(fmaxf(0.1f, mid * mid - det));
            float l2 = mid - sqrtf(fmaxf(0.1f, mid * mid - det));
            float rad = ceilf(3.f * sqrtf(fmaxf(l1, l2)));
            if (!isnan(rad)) dens[4 * i + 3] = fmaxf(dens[4 * i + 3], rad);
        }
        float mx = x * cam->fx + cam->cx, my = y * cam->fy + cam->cy;
        uint16_t hcx = 0, hcy = 0, hcz = 0;
        float thr;
        if (fp16) {
            hcx = orc_f2h(conic[0]);
            hcy = orc_f2h(conic[1]);
            hcz = orc_f2h(conic[2]);
            thr = logf(orc_h2f(opacity_h) * 255.0f);
        } else {
            thr = logf(opacity * 255.0f);
        }
        float fac = sqrtf(2.0f * thr);
        float ex = fmaxf(fac * sqrtf(cov_a) - 0.5f, 0.0f);
        float ey = fmaxf(fac * sqrtf(cov_c) - 0.5f, 0.0f);
        float bx0 = (mx - ex) / (float)TILE, bx1 = (mx + ex) / (float)TILE;
        float by0 = (my - ey) / (float)TILE, by1 = (my + ey) / (float)TILE;
        /* __float2int_rd / _ru; NaN maps to INT_MIN, then max(0, .) */
        long fx0 = isnan(bx0) ? 0 : (long)floorf(fmaxf(fminf(bx0, 2e9f), -2e9f));
        long fx1 = isnan(bx1) ? 0 : (long)ceilf(fmaxf(fminf(bx1, 2e9f), -2e9f));
        long fy0 = isnan(by0) ? 0 : (long)floorf(fmaxf(fminf(by0, 2e9f), -2e9f));
        long fy1 = isnan(by1) ? 0 : (long)ceilf(fmaxf(fminf(by1, 2e9f), -2e9f));
        uint32_t b0 = (uint32_t)(fx0 < 0 ? 0 : fx0); if (b0 > gw) b0 = gw;
        uint32_t b1 = (uint32_t)(fx1 < 0 ? 0 : fx1); if (b1 > gw) b1 = gw;
        uint32_t b2 = (uint32_t)(fy0 < 0 ? 0 : fy0); if (b2 > gh) b2 = gh;
        uint32_t b3 = (uint32_t)(fy1 < 0 ? 0 : fy1); if (b3 > gh) b3 = gh;
        if (fabsf(bx0 - roundf(bx0)) < 1e-4f || fabsf(bx1 - roundf(bx1)) < 1e-4f ||
            fabsf(by0 - roundf(by0)) < 1e-4f || fabsf(by1 - roundf(by1)) < 1e-4f)
            fragile = 1;
        if (g_smooth) { b0 = 0; b1 = gw; b2 = 0; b3 = gh; }
        uint32_t tile_count = (b1 - b0) * (b3 - b2);
        if (tile_count == 0) active = 0;
        if (!active) continue;
        uint32_t touched = 0;
        uint32_t bw = b1 - b0;
        float smx = mx - 0.5f, smy = my - 0.5f;
        for (uint32_t k = 0; k < tile_count; ++k) {
            uint32_t ty_ = b2 + k / bw, tx_ = b0 + k % bw;
            float margin;
            int c = fp16 ? tile_test_f16(smx, smy, hcx, hcy, hcz, tx_, ty_, thr, &margin)
                         : tile_test_f32(smx, smy, conic, tx_, ty_, thr, &margin);
            if (c || g_smooth) touched++;
            float tol = fp16 ? g_fragile_f16 * fmaxf(fabsf(thr), 1.f) : FRAGILE_REL * fmaxf(fabsf(thr), 1.f);
            if (isfinite(margin) && fabsf(margin) <= tol) fragile = 1;
        }
        out->fragile[i] = fragile;
        if (touched == 0) continue;
        out->n_touched[i] = touched;
        out->bounds[4 * i + 0] = (uint16_t)b0;
        out->bounds[4 * i + 1] = (uint16_t)b1;
        out->bounds[4 * i + 2] = (uint16_t)b2;
        out->bounds[4 * i + 3] = (uint16_t)b3;
        out->mean2d[2 * i + 0] = mx;
        out->mean2d[2 * i + 1] = my;
        float col[3];
        sh_to_color(sh0 + 3 * i, sh_rest + 45 * i, active_bases, m, campos, col);
        if (out->color) {
            out->color[3 * i + 0] = col[0];
            out->color[3 * i + 1] = col[1];
            out->color[3 * i + 2] = col[2];
        }
        union { float f; uint32_t u; } dk;
        dk.f = depth;
        out->depth_key[i] = dk.u;
        if (fp16) {
            if (out->prim_info) {
                uint8_t* rec = out->prim_info + 16 * i;
                memset(rec, 0, 16);
                uint16_t vals[4] = {hcx, hcy, hcz, opacity_h};
                memcpy(rec, vals, 8);
                for (int c = 0; c < 3; ++c) rec[8 + c] = (uint8_t)(satf(col[c]) * 255.0f);
            }
            if (out->conic_opacity) {
                out->conic_opacity[4 * i + 0] = orc_h2f(hcx);
                out->conic_opacity[4 * i + 1] = orc_h2f(hcy);
                out->conic_opacity[4 * i + 2] = orc_h2f(hcz);
                out->conic_opacity[4 * i + 3] = orc_h2f(opacity_h);
            }
        } else if (out->conic_opacity) {
            out->conic_opacity[4 * i + 0] = conic[0];
            out->conic_opacity[4 * i + 1] = conic[1];
            out->conic_opacity[4 * i + 2] = conic[2];
            out->conic_opacity[4 * i + 3] = opacity;
        }
    }
    free(warp_alive);
    free(act);
}

/* ---------------------------------------------------------------- binning */

typedef struct {
    uint32_t key;
    uint32_t idx;
} KeyIdx;

static int cmp_keyidx(const void* a, const void* b) {
    const KeyIdx* x = (const KeyIdx*)a;
    const KeyIdx* y = (const KeyIdx*)b;
    if (x->key != y->key) return x->key < y->key ? -1 : 1;
    return x->idx < y->idx ? -1 : (x->idx > y->idx ? 1 : 0);
}

/* Exact touched-tile count of every Gaussian recomputed from its stored
 * screen-space record (bounds, mean2d, conic + opacity or the fp16 record):
 * the decision the reference's create_instances_cu repeats
 * (fastgs_ours/kernels_forward.cuh:427-530, fp16 :517-631).  Gaussians with
 * n_touched == 0 in `prim` get 0. */
void orc_count_tiles(int64_t n, const OrcPrimitives* prim, const OrcCamera* cam, int32_t fp16,
                     uint32_t* out, uint8_t* fragile, float band, int32_t n_threads) {
    (void)cam;
    if (n_threads > 0) omp_set_num_threads(n_threads);
#pragma omp parallel for schedule(dynamic, 4096)
    for (int64_t i = 0; i < n; ++i) {
        out[i] = 0;
        if (fragile) fragile[i] = 0;
        if (prim->n_touched[i] == 0) continue;
        const uint16_t* b = prim->bounds + 4 * (size_t)i;
        uint32_t bw = (uint32_t)(b[1] - b[0]);
        uint32_t cnt = bw * (uint32_t)(b[3] - b[2]);
        float smx = prim->mean2d[2 * i] - 0.5f, smy = prim->mean2d[2 * i + 1] - 0.5f;
        float thr, conic[3] = {0.f, 0.f, 0.f};
        uint16_t hc[4] = {0, 0, 0, 0};
        if (fp16) {
            memcpy(hc, prim->prim_info + 16 * (size_t)i, 8);
            thr = logf(orc_h2f(hc[3]) * 255.0f);
        } else {
            const float* co = prim->conic_opacity + 4 * (size_t)i;
            conic[0] = co[0];
            conic[1] = co[1];
            conic[2] = co[2];
            thr = logf(co[3] * 255.0f);
        }
        uint32_t touched = 0;
        uint8_t fr = 0;
        for (uint32_t q = 0; q < cnt; ++q) {
            uint32_t ty = b[2] + q / bw, tx = b[0] + q % bw;
            float margin;
            int c = fp16 ? tile_test_f16(smx, smy, hc[0], hc[1], hc[2], tx, ty, thr, &margin)
                         : tile_test_f32(smx, smy, conic, tx, ty, thr, &margin);
            touched += c ? 1u : 0u;
            if (isfinite(margin) && fabsf(margin) <= band * fmaxf(fabsf(thr), 1.f)) fr = 1;
        }
        out[i] = touched;
        if (fragile) fragile[i] = fr;
    }
}

int64_t orc_binning(int64_t n, const OrcPrimitives* prim, const OrcCamera* cam,
                    int32_t fp16, uint32_t* inst_tile, uint32_t* inst_prim,
                    int64_t cap, uint32_t* ranges, uint32_t* sorted_visible,
                    uint32_t* n_visible) {
    const uint32_t gw = (uint32_t)((cam->width + TILE - 1) / TILE);
    const uint32_t gh = (uint32_t)((cam->height + TILE - 1) / TILE);
    const uint32_t n_tiles = gw * gh;
    int64_t nv = 0;
    for (int64_t i = 0; i < n; ++i) nv += prim->n_touched[i] > 0;
    KeyIdx* vis = (KeyIdx*)malloc(sizeof(KeyIdx) * (size_t)(nv > 0 ? nv : 1));
    int64_t k = 0;
    for (int64_t i = 0; i < n; ++i)
        if (prim->n_touched[i] > 0) {
            vis[k].key = prim->depth_key[i];
            vis[k].idx = (uint32_t)i;
            ++k;
        }
    /* depth order; ties by index (a deterministic member of the reference's
     * atomic-order tie set, fastgs_ours/kernels_forward.cuh:407-410) */
    qsort(vis, (size_t)nv, sizeof(KeyIdx), cmp_keyidx);
    if (n_visible) *n_visible = (uint32_t)nv;
    if (sorted_visible)
        for (int64_t j = 0; j < nv; ++j) sorted_visible[j] = vis[j].idx;
    int64_t total = 0;
    for (int64_t j = 0; j < nv; ++j) total += prim->n_touched[vis[j].idx];
    if (total > cap) {
        free(vis);
        return -1;
    }
    /* instance creation in depth order, kernels_forward.cuh:427-530; each
     * visible Gaussian writes its own slice (offsets = exclusive scan of the
     * touched-tile counts in depth order), so the loop runs in parallel */
    uint32_t* tmp_tile = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)(total > 0 ? total : 1));
    uint32_t* tmp_prim = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)(total > 0 ? total : 1));
    int64_t* offs = (int64_t*)malloc(sizeof(int64_t) * (size_t)(nv + 1));
    offs[0] = 0;
    for (int64_t j = 0; j < nv; ++j) offs[j + 1] = offs[j] + prim->n_touched[vis[j].idx];
    int64_t w = total;
#pragma omp parallel for schedule(dynamic, 1024)
    for (int64_t j = 0; j < nv; ++j) {
        uint32_t i = vis[j].idx;
        int64_t o = offs[j];
        const uint16_t* b = prim->bounds + 4 * (size_t)i;
        uint32_t bw = (uint32_t)(b[1] - b[0]);
        uint32_t cnt = bw * (uint32_t)(b[3] - b[2]);
        float smx = prim->mean2d[2 * i] - 0.5f, smy = prim->mean2d[2 * i + 1] - 0.5f;
        float thr;
        float conic[3] = {0.f, 0.f, 0.f};
        uint16_t hc[4] = {0, 0, 0, 0};
        if (fp16) {
            memcpy(hc, prim->prim_info + 16 * (size_t)i, 8);
            thr = logf(orc_h2f(hc[3]) * 255.0f);
        } else {
            const float* co = prim->conic_opacity + 4 * (size_t)i;
            conic[0] = co[0];
            conic[1] = co[1];
            conic[2] = co[2];
            thr = logf(co[3] * 255.0f);
        }
        uint32_t emitted = 0;
        for (uint32_t q = 0; q < cnt; ++q) {
            uint32_t ty = b[2] + q / bw, tx = b[0] + q % bw;
            float margin;
            int c = fp16 ? tile_test_f16(smx, smy, hc[0], hc[1], hc[2], tx, ty, thr, &margin)
                         : tile_test_f32(smx, smy, conic, tx, ty, thr, &margin);
            if ((c || g_smooth) && emitted < prim->n_touched[i]) {
                tmp_tile[o + emitted] = ty * gw + tx;
                tmp_prim[o + emitted] = i;
                ++emitted;
            }
        }
        /* keep the count consistent with n_touched even on a mismatch */
        while (emitted < prim->n_touched[i]) {
            tmp_tile[o + emitted] = 0xffffffffu;
            tmp_prim[o + emitted] = i;
            ++emitted;
        }
    }
    free(offs);
    /* stable counting sort by tile (fastgs_ours/forward.cu:206-217) */
    uint32_t* cnt = (uint32_t*)calloc(n_tiles + 1, sizeof(uint32_t));
    for (int64_t q = 0; q < w; ++q)
        if (tmp_tile[q] < n_tiles) cnt[tmp_tile[q] + 1]++;
    for (uint32_t t = 0; t < n_tiles; ++t) cnt[t + 1] += cnt[t];
    for (uint32_t t = 0; t < n_tiles; ++t) {
        ranges[2 * t] = cnt[t];
        ranges[2 * t + 1] = cnt[t + 1];
    }
    int64_t valid = cnt[n_tiles];
    for (int64_t q = 0; q < w; ++q) {
        uint32_t t = tmp_tile[q];
        if (t >= n_tiles) continue;
        uint32_t pos = cnt[t]++;
        inst_tile[pos] = t;
        inst_prim[pos] = tmp_prim[q];
    }
    free(cnt);
    free(tmp_tile);
    free(tmp_prim);
    free(vis);
    (void)gh;
    return valid;
}

int64_t orc_bucket_offsets(const uint32_t* ranges, int32_t n_tiles, uint32_t* bucket_offsets) {
    int64_t acc = 0;
    for (int32_t t = 0; t < n_tiles; ++t) {
        uint32_t c = ranges[2 * t + 1] - ranges[2 * t];
        acc += (c + 31) / 32;
        bucket_offsets[t] = (uint32_t)acc;
    }
    return acc;
}

/* position of pixel (lx, ly) of a 16x16 tile inside a bucket checkpoint
 * (2x2 arrangement of 8x8 sub-tiles), kernels_forward.cuh:650 */
static inline uint32_t ckpt_slot(uint32_t ly, uint32_t lx) { return tiled_index(ly, lx, 2); }

/* ------------------------------------------------------- blend forward f32 */

void orc_blend_forward_f32(const OrcCamera* cam, const uint32_t* ranges,
                           const uint32_t* inst_prim, const float* mean2d,
                           const float* conic_opacity, const float* color,
                           float* image, float* alpha, uint32_t* n_contrib,
                           uint32_t* tile_max_contrib,
                           const uint32_t* bucket_offsets, float* ckpt,
                           int32_t n_threads) {
    set_threads(n_threads);
    const uint32_t W = (uint32_t)cam->width, H = (uint32_t)cam->height;
    const uint32_t gw = (W + TILE - 1) / TILE, gh = (H + TILE - 1) / TILE;
    const uint32_t tw = (W + 7) >> 3, th = (H + 7) >> 3;
    const uint32_t plane = tw * th * 64;
    const int64_t n_tiles = (int64_t)gw * gh;
#pragma omp parallel for schedule(dynamic, 4)
    for (int64_t t = 0; t < n_tiles; ++t) {
        if (t % g_tile_stride != 0) continue;
        uint32_t gx = (uint32_t)(t % gw), gy = (uint32_t)(t / gw);
        uint32_t start = ranges[2 * t], end = ranges[2 * t + 1];
        uint32_t count = end - start;
        uint32_t nb = (count + 31) / 32;
        uint32_t boff = t == 0 ? 0 : bucket_offsets[t - 1];
        uint32_t tile_max = 0;
        /* number of buckets the block writes: it stops at the first 256-batch
         * in which every pixel is done (kernels_forward.cuh:630-632) */
        uint32_t max_ckpt = 0;
        for (uint32_t ly = 0; ly < TILE; ++ly)
            for (uint32_t lx = 0; lx < TILE; ++lx) {
                uint32_t px = gx * TILE + lx, py = gy * TILE + ly;
                int inside = px < W && py < H;
                float pxf = (float)px + 0.5f, pyf = (float)py + 0.5f;
                float cr = 0.f, cg = 0.f, cb = 0.f, T = 1.f;
                uint32_t npos = 0, ncon = 0;
                int done = !inside;
                uint32_t processed = 0; /* prims consumed before done */
                for (uint32_t j = 0; j < count && !done; ++j) {
                    if (ckpt && (j % 32) == 0) {
                        float* c = ckpt + 4 * ((size_t)(boff + j / 32) * BLOCK + ckpt_slot(ly, lx));
                        c[0] = cr; c[1] = cg; c[2] = cb; c[3] = T;
                    }
                    processed = j + 1;
                    npos++;
                    uint32_t p = inst_prim[start + j];
                    const float* co = conic_opacity + 4 * (size_t)p;
                    float dx = mean2d[2 * p] - pxf, dy = mean2d[2 * p + 1] - pyf;
                    float s = 0.5f * (co[0] * dx * dx + co[2] * dy * dy) + co[1] * dx * dy;
                    if (s < 0.f) continue;
                    float g = expf(-s);
                    float a = fminf(co[3] * g, 0.999f);
                    if (g_pix_fragile && inside &&
                        (near_rel(co[3] * g, 1.0f / 255.0f, g_pix_band) || near_rel(co[3] * g, 0.999f, g_pix_band) ||
                         near_rel(T * (1.0f - a), 1e-4f, g_pix_band)))
                        g_pix_fragile[tiled_index(py, px, tw)] = 1;
                    if (a < 1.0f / 255.0f && !g_smooth) continue;
                    float Tn = T * (1.0f - a);
                    if (Tn < 1e-4f && !g_smooth) {
                        done = 1;
                        continue;
                    }
                    const float* col = color + 3 * (size_t)p;
                    float w_ = T * a;
                    cr += w_ * fmaxf(col[0], 0.f);
                    cg += w_ * fmaxf(col[1], 0.f);
                    cb += w_ * fmaxf(col[2], 0.f);
                    T = Tn;
                    ncon = npos;
                }
                /* checkpoints after the pixel stopped hold its frozen state */
                if (ckpt && inside) {
                    for (uint32_t b = (processed + 31) / 32; b < nb; ++b) {
                        float* c = ckpt + 4 * ((size_t)(boff + b) * BLOCK + ckpt_slot(ly, lx));
                        c[0] = cr; c[1] = cg; c[2] = cb; c[3] = T;
                    }
                }
                if (!inside && ckpt) {
                    for (uint32_t b = 0; b < nb; ++b) {
                        float* c = ckpt + 4 * ((size_t)(boff + b) * BLOCK + ckpt_slot(ly, lx));
                        c[0] = 0.f; c[1] = 0.f; c[2] = 0.f; c[3] = 1.f;
                    }
                }
                (void)max_ckpt;
                if (inside) {
                    uint32_t pi = tiled_index(py, px, tw);
                    image[pi] = cr;
                    image[pi + plane] = cg;
                    image[pi + 2 * plane] = cb;
                    if (alpha) alpha[pi] = 1.0f - T;
                    n_contrib[pi] = ncon;
                }
                if (ncon > tile_max) tile_max = ncon;
            }
        tile_max_contrib[t] = tile_max;
    }
}

/* ------------------------------------------------------ blend backward f32 */

/* pixel order inside a tile for the backward sweep (kernels_backward.cuh:779-803) */
static inline void bwd_pixel(uint32_t idx, uint32_t* dx, uint32_t* dy) {
    uint32_t lt = idx >> 6, it = idx & 63u;
    *dx = (it & 7u) + (lt & 1u) * 8u;
    *dy = (it >> 3) + (lt >> 1) * 8u;
}

void orc_blend_backward_f32(const OrcCamera* cam, int64_t n,
                            const uint32_t* ranges, const uint32_t* inst_prim,
                            const float* mean2d, const float* conic_opacity,
                            const float* color, const float* image,
                            const float* grad_image, const uint32_t* n_contrib,
                            const uint32_t* tile_max_contrib,
                            const uint32_t* bucket_offsets, const float* ckpt,
                            float* grad_mean2d, float* absgrad_mean2d,
                            float* grad_conic, float* grad_opacity,
                            float* grad_color, int32_t n_threads) {
    set_threads(n_threads);
    const uint32_t W = (uint32_t)cam->width, H = (uint32_t)cam->height;
    const uint32_t gw = (W + TILE - 1) / TILE, gh = (H + TILE - 1) / TILE;
    const uint32_t tw = (W + 7) >> 3, th = (H + 7) >> 3;
    const uint32_t plane = tw * th * 64;
    const int64_t n_tiles = (int64_t)gw * gh;
    const int64_t n_inst = n_tiles > 0 ? ranges[2 * (n_tiles - 1) + 1] : 0;
    /* per-instance partial sums, reduced in instance order afterwards so the
     * result does not depend on the thread count */
    float* part = (float*)calloc((size_t)(n_inst > 0 ? n_inst : 1) * 11, sizeof(float));
#pragma omp parallel for schedule(dynamic, 2)
    for (int64_t t = 0; t < n_tiles; ++t) {
        if (t % g_tile_stride != 0) continue;
        uint32_t gx = (uint32_t)(t % gw), gy = (uint32_t)(t / gw);
        uint32_t start = ranges[2 * t], end = ranges[2 * t + 1];
        uint32_t count = end - start;
        uint32_t nb = (count + 31) / 32;
        uint32_t boff = t == 0 ? 0 : bucket_offsets[t - 1];
        for (uint32_t b = 0; b < nb; ++b) {
            if (b * 32 >= tile_max_contrib[t]) break;
            /* per-pixel running state at the start of this bucket */
            float Tpix[BLOCK], Ca[BLOCK][3], G[BLOCK][3];
            uint32_t last[BLOCK];
            int valid[BLOCK];
            for (uint32_t i = 0; i < BLOCK; ++i) {
                uint32_t dx, dy;
                bwd_pixel(i, &dx, &dy);
                uint32_t px = gx * TILE + dx, py = gy * TILE + dy;
                valid[i] = px < W && py < H;
                const float* c = ckpt + 4 * ((size_t)(boff + b) * BLOCK + i);
                if (valid[i]) {
                    uint32_t pi = tiled_index(py, px, tw);
                    Tpix[i] = c[3];
                    for (int k = 0; k < 3; ++k) {
                        Ca[i][k] = image[pi + k * plane] - c[k];
                        G[i][k] = grad_image[pi + k * plane];
                    }
                    last[i] = n_contrib[pi];
                } else {
                    Tpix[i] = 0.f;
                    for (int k = 0; k < 3; ++k) { Ca[i][k] = 0.f; G[i][k] = 0.f; }
                    last[i] = 0;
                }
            }
            for (uint32_t l = 0; l < 32; ++l) {
                uint32_t tp = b * 32 + l;
                if (tp >= count) break;
                uint32_t p = inst_prim[start + tp];
                const float* co = conic_opacity + 4 * (size_t)p;
                const float* cu = color + 3 * (size_t)p;
                float col[3] = {fmaxf(cu[0], 0.f), fmaxf(cu[1], 0.f), fmaxf(cu[2], 0.f)};
                float fac[3] = {cu[0] >= 0.f ? 1.f : 0.f, cu[1] >= 0.f ? 1.f : 0.f, cu[2] >= 0.f ? 1.f : 0.f};
                float mx = mean2d[2 * p] - 0.5f, my = mean2d[2 * p + 1] - 0.5f;
                float acc[11] = {0};
                for (uint32_t i = 0; i < BLOCK; ++i) {
                    uint32_t dx, dy;
                    bwd_pixel(i, &dx, &dy);
                    float pxf = (float)(gx * TILE + dx), pyf = (float)(gy * TILE + dy);
                    float ddx = mx - pxf, ddy = my - pyf;
                    float dxx = ddx * ddx, dxy = ddx * ddy, dyy = ddy * ddy;
                    float s = fmaxf(0.5f * (co[0] * dxx + co[2] * dyy) + co[1] * dxy, 0.f);
                    float g = expf(-s);
                    int skip = !valid[i] || tp >= last[i];
                    float a = skip ? 0.f : fminf(co[3] * g, 0.999f);
                    float T = Tpix[i];
                    float bw_ = T * a;
                    float om = 1.0f - a;
                    float cdg = col[0] * G[i][0] + col[1] * G[i][1] + col[2] * G[i][2];
                    for (int k = 0; k < 3; ++k) acc[7 + k] += bw_ * (G[i][k] * fac[k]);
                    for (int k = 0; k < 3; ++k) Ca[i][k] -= bw_ * col[k];
                    float cadg = Ca[i][0] * G[i][0] + Ca[i][1] * G[i][1] + Ca[i][2] * G[i][2];
                    float dLda = T * cdg - cadg / om;
                    float dop = a * dLda;
                    acc[10] += dop;
                    acc[4] += -0.5f * dop * dxx;
                    acc[5] += -0.5f * dop * dxy;
                    acc[6] += -0.5f * dop * dyy;
                    float gmx = dop * (co[0] * ddx + co[1] * ddy);
                    float gmy = dop * (co[1] * ddx + co[2] * ddy);
                    acc[0] -= gmx;
                    acc[1] -= gmy;
                    acc[2] += fabsf(gmx);
                    acc[3] += fabsf(gmy);
                    Tpix[i] = T * om;
                }
                float* dst = part + 11 * (size_t)(start + tp);
                for (int k = 0; k < 11; ++k) dst[k] = acc[k];
                /* opacity: partial sum times (1 - opacity) */
                dst[10] = acc[10] * (1.0f - co[3]);
            }
        }
    }
    for (int64_t q = 0; q < n_inst; ++q) {
        uint32_t p = inst_prim[q];
        const float* s = part + 11 * (size_t)q;
        grad_mean2d[2 * p] += s[0];
        grad_mean2d[2 * p + 1] += s[1];
        if (absgrad_mean2d) {
            absgrad_mean2d[2 * p] += s[2];
            absgrad_mean2d[2 * p + 1] += s[3];
        }
        grad_conic[p] += s[4];
        grad_conic[n + p] += s[5];
        grad_conic[2 * n + p] += s[6];
        grad_color[3 * p] += s[7];
        grad_color[3 * p + 1] += s[8];
        grad_color[3 * p + 2] += s[9];
        grad_opacity[p] += s[10];
    }
    free(part);
}

/* ------------------------------------------------------- blend forward f16 */

void orc_blend_forward_f16(const OrcCamera* cam, const uint32_t* ranges,
                           const uint32_t* inst_prim, const float* mean2d,
                           const uint8_t* prim_info, uint16_t* image,
                           uint16_t* alpha, uint16_t* n_contrib,
                           uint16_t* tile_max_contrib,
                           const uint32_t* bucket_offsets, uint16_t* ckpt,
                           int32_t n_threads) {
    set_threads(n_threads);
    const uint32_t W = (uint32_t)cam->width, H = (uint32_t)cam->height;
    const uint32_t gw = (W + TILE - 1) / TILE, gh = (H + TILE - 1) / TILE;
    const uint32_t tw = (W + 7) >> 3, th = (H + 7) >> 3;
    const uint32_t plane = tw * th * 64;
    const int64_t n_tiles = (int64_t)gw * gh;
    /* constants of fastgs_ours_fp16/kernels_forward.cuh:948-1039 */
    const uint16_t h_inv16 = orc_f2h(0.0625f), h16 = orc_f2h(16.0f);
    const uint16_t h_half = orc_f2h(0.5f), h_1_32 = orc_f2h(1.0f / 32.0f);
    const uint16_t h_scale = orc_f2h(255.0f), h_unscale = orc_f2h(1.0f / 255.0f);
    const uint16_t h_min_T = f2h_rd(1e-4f * 255.0f);
    const uint16_t h_max_a = orc_f2h(0.99f);
    const uint16_t h_log2e = orc_f2h(1.4426950409f);
    const uint16_t h_one = 0x3c00u;
#pragma omp parallel for schedule(dynamic, 4)
    for (int64_t t = 0; t < n_tiles; ++t) {
        if (t % g_tile_stride != 0) continue;
        uint32_t gx = (uint32_t)(t % gw), gy = (uint32_t)(t / gw);
        uint32_t start = ranges[2 * t], end = ranges[2 * t + 1];
        uint32_t count = end - start;
        uint32_t nb = (count + 31) / 32;
        uint32_t boff = t == 0 ? 0 : bucket_offsets[t - 1];
        uint16_t tile_max = 0;
        for (uint32_t ly = 0; ly < TILE; ++ly)
            for (uint32_t lx = 0; lx < TILE; ++lx) {
                uint32_t px = gx * TILE + lx, py = gy * TILE + ly;
                int inside = px < W && py < H;
                /* pixel offset inside the tile in tile units (1/16 + 1/32) */
                uint32_t ex = lx & ~1u;
                uint16_t off0x = hfma(h_inv16, orc_f2h((float)ex), h_1_32);
                uint16_t offx = (lx & 1u) ? hadd(h_inv16, off0x) : off0x;
                uint16_t offy = hfma(h_inv16, orc_f2h((float)ly), h_1_32);
                uint16_t cr = 0, cg = 0, cb = 0, T = h_scale;
                uint32_t ncon = 0;
                int unfinished = inside;
                uint32_t processed = 0;
                for (uint32_t j = 0; j < count && unfinished; ++j) {
                    if (ckpt && (j % 32) == 0) {
                        uint16_t* c = ckpt + 4 * ((size_t)(boff + j / 32) * BLOCK + ckpt_slot(ly, lx));
                        c[0] = cr; c[1] = cg; c[2] = cb; c[3] = T;
                    }
                    processed = j + 1;
                    uint32_t p = inst_prim[start + j];
                    const uint8_t* rec = prim_info + 16 * (size_t)p;
                    uint16_t hv[4];
                    memcpy(hv, rec, 8);
                    float mxf = mean2d[2 * p] / 16.0f - (float)gx;
                    float myf = mean2d[2 * p + 1] / 16.0f - (float)gy;
                    uint16_t mx = orc_f2h(mxf), my = orc_f2h(myf);
                    uint16_t cx = hmul(hv[0], h16), cy = hmul(hv[1], h16), cz = hmul(hv[2], h16);
                    uint16_t op = hv[3];
                    uint16_t dx = hsub(mx, offx), dy = hsub(my, offy);
                    uint16_t qx = hmul(dx, hmul(cx, dx));
                    uint16_t qz = hmul(dy, hmul(cz, dy));
                    uint16_t qy = hmul(dx, hmul(cy, dy));
                    uint16_t quad = hadd(qx, qz);
                    uint16_t sig = hmul(hfma(h_half, quad, qy), h16);
                    uint16_t gauss = hex2(hmul(hneg(sig), h_log2e));
                    uint16_t a = hmin(hmul(op, gauss), h_max_a);
                    uint16_t Tn = hfma(hneg(a), T, T);
                    if (g_pix_fragile && inside && unfinished &&
                        (near_rel(orc_h2f(Tn), orc_h2f(h_min_T), g_pix_band) ||
                         near_rel(orc_h2f(hmul(op, gauss)), orc_h2f(h_max_a), g_pix_band)))
                        g_pix_fragile[tiled_index(py, px, tw)] = 1;
                    int ok = Tn >= h_min_T; /* bit compare of positive halves */
                    int en = unfinished && ok;
                    uint16_t tah = hmul(hmul(T, a), h_unscale);
                    if (!en) tah = 0;
                    cr = hfma(orc_f2h((float)rec[8]), tah, cr);
                    cg = hfma(orc_f2h((float)rec[9]), tah, cg);
                    cb = hfma(orc_f2h((float)rec[10]), tah, cb);
                    if (en) T = Tn;
                    if (unfinished && ncon < 0xffffu) ncon++;
                    unfinished = unfinished && ok;
                    if ((j % 32) == 31 || j + 1 == count) {
                        if (ncon >= 0xffffu) unfinished = 0;
                    }
                }
                if (ckpt) {
                    uint32_t from = inside ? (processed + 31) / 32 : 0;
                    for (uint32_t b = from; b < nb; ++b) {
                        uint16_t* c = ckpt + 4 * ((size_t)(boff + b) * BLOCK + ckpt_slot(ly, lx));
                        c[0] = cr; c[1] = cg; c[2] = cb; c[3] = T;
                    }
                }
                uint16_t fr = hmul(cr, h_unscale), fg = hmul(cg, h_unscale), fb = hmul(cb, h_unscale);
                uint16_t Tu = hmul(T, h_unscale);
                if (inside) {
                    uint32_t pi = tiled_index(py, px, tw);
                    image[pi] = fr;
                    image[pi + plane] = fg;
                    image[pi + 2 * plane] = fb;
                    if (alpha) alpha[pi] = hsub(h_one, Tu);
                    n_contrib[pi] = (uint16_t)ncon;
                }
                if (ncon > tile_max) tile_max = (uint16_t)ncon;
            }
        tile_max_contrib[t] = tile_max;
    }
}

/* ------------------------------------------------------ blend backward f16 */

void orc_blend_backward_f16(const OrcCamera* cam, int64_t n,
                            const uint32_t* ranges, const uint32_t* inst_prim,
                            const float* mean2d, const uint8_t* prim_info,
                            const uint16_t* image, const uint16_t* grad_image,
                            const uint16_t* tile_max_contrib,
                            const uint32_t* bucket_offsets,
                            const uint16_t* ckpt, float* grad_mean2d,
                            float* absgrad_mean2d, float* grad_conic,
                            float* grad_opacity, float* grad_color,
                            int32_t n_threads) {
    set_threads(n_threads);
    (void)n;
    const uint32_t W = (uint32_t)cam->width, H = (uint32_t)cam->height;
    const uint32_t gw = (W + TILE - 1) / TILE, gh = (H + TILE - 1) / TILE;
    const uint32_t tw = (W + 7) >> 3, th = (H + 7) >> 3;
    const uint32_t plane = tw * th * 64;
    const int64_t n_tiles = (int64_t)gw * gh;
    const int64_t n_inst = n_tiles > 0 ? ranges[2 * (n_tiles - 1) + 1] : 0;
    float* part = (float*)calloc((size_t)(n_inst > 0 ? n_inst : 1) * 11, sizeof(float));
#pragma omp parallel for schedule(dynamic, 2)
    for (int64_t t = 0; t < n_tiles; ++t) {
        if (t % g_tile_stride != 0) continue;
        uint32_t gx = (uint32_t)(t % gw), gy = (uint32_t)(t / gw);
        uint32_t start = ranges[2 * t], end = ranges[2 * t + 1];
        uint32_t count = end - start;
        uint32_t nb = (count + 31) / 32;
        uint32_t boff = t == 0 ? 0 : bucket_offsets[t - 1];
        for (uint32_t b = 0; b < nb; ++b) {
            if (b * 32 >= tile_max_contrib[t]) break;
            float Tpix[BLOCK], Ca[BLOCK][3], G[BLOCK][3];
            int valid[BLOCK];
            for (uint32_t i = 0; i < BLOCK; ++i) {
                uint32_t dx, dy;
                bwd_pixel(i, &dx, &dy);
                uint32_t px = gx * TILE + dx, py = gy * TILE + dy;
                valid[i] = px < W && py < H;
                const uint16_t* c = ckpt + 4 * ((size_t)(boff + b) * BLOCK + i);
                if (valid[i]) {
                    uint32_t pi = tiled_index(py, px, tw);
                    Tpix[i] = orc_h2f(c[3]) * (1.0f / 255.0f);
                    for (int k = 0; k < 3; ++k) {
                        Ca[i][k] = orc_h2f(image[pi + k * plane]) * 255.0f - orc_h2f(c[k]);
                        G[i][k] = orc_h2f(grad_image[pi + k * plane]);
                    }
                } else {
                    Tpix[i] = 0.f;
                    for (int k = 0; k < 3; ++k) { Ca[i][k] = 0.f; G[i][k] = 0.f; }
                }
            }
            for (uint32_t l = 0; l < 32; ++l) {
                uint32_t tp = b * 32 + l;
                if (tp >= count || tp > 0xffffu) break;
                uint32_t p = inst_prim[start + tp];
                const uint8_t* rec = prim_info + 16 * (size_t)p;
                uint16_t hv[4];
                memcpy(hv, rec, 8);
                float ca = orc_h2f(hv[0]), cbv = orc_h2f(hv[1]), cc = orc_h2f(hv[2]);
                float op = orc_h2f(hv[3]);
                float col[3] = {(float)rec[8], (float)rec[9], (float)rec[10]};
                float mx = mean2d[2 * p] - 0.5f, my = mean2d[2 * p + 1] - 0.5f;
                float acc[11] = {0};
                for (uint32_t i = 0; i < BLOCK; ++i) {
                    uint32_t dx, dy;
                    bwd_pixel(i, &dx, &dy);
                    float ddx = mx - (float)(gx * TILE + dx);
                    float ddy = my - (float)(gy * TILE + dy);
                    float qxx = ca * ddx, qyx = cbv * ddx, qzy = cc * ddy, qyy = cbv * ddy;
                    float s = fmaxf(0.5f * (ddx * qxx + ddy * qzy) + ddx * qyy, 0.f);
                    float g = valid[i] ? expf(-s) : 0.f;
                    /* the fp16 kernels cap alpha at fp16(0.99) = 0.990234375 */
                    float a = fminf(op * g, orc_h2f(orc_f2h(0.99f)));
                    float T = Tpix[i];
                    float bw_ = T * a;
                    float om = 1.0f - a;
                    float cdg = col[0] * G[i][0] + col[1] * G[i][1] + col[2] * G[i][2];
                    for (int k = 0; k < 3; ++k) acc[7 + k] += bw_ * G[i][k];
                    for (int k = 0; k < 3; ++k) Ca[i][k] -= bw_ * col[k];
                    float cadg = Ca[i][0] * G[i][0] + Ca[i][1] * G[i][1] + Ca[i][2] * G[i][2];
                    float dop = a * (T * cdg - cadg / om); /* 255-scaled */
                    acc[10] += dop;
                    acc[4] += dop * ddx * ddx;
                    acc[5] += dop * ddx * ddy;
                    acc[6] += dop * ddy * ddy;
                    float gmx = dop * (qxx + qyy), gmy = dop * (qyx + qzy);
                    acc[0] += gmx;
                    acc[1] += gmy;
                    acc[2] += fabsf(gmx);
                    acc[3] += fabsf(gmy);
                    Tpix[i] = T * om;
                }
                float* dst = part + 11 * (size_t)(start + tp);
                const float inv = 1.0f / 255.0f;
                dst[0] = -acc[0] * inv;
                dst[1] = -acc[1] * inv;
                dst[2] = acc[2] * inv;
                dst[3] = acc[3] * inv;
                dst[4] = -0.5f * acc[4] * inv;
                dst[5] = -0.5f * acc[5] * inv;
                dst[6] = -0.5f * acc[6] * inv;
                dst[7] = acc[7];
                dst[8] = acc[8];
                dst[9] = acc[9];
                dst[10] = acc[10] * inv * (1.0f - op);
            }
        }
    }
    for (int64_t q = 0; q < n_inst; ++q) {
        uint32_t p = inst_prim[q];
        const float* s = part + 11 * (size_t)q;
        grad_mean2d[2 * p] += s[0];
        grad_mean2d[2 * p + 1] += s[1];
        if (absgrad_mean2d) {
            absgrad_mean2d[2 * p] += s[2];
            absgrad_mean2d[2 * p + 1] += s[3];
        }
        grad_conic[3 * p] += s[4];
        grad_conic[3 * p + 1] += s[5];
        grad_conic[3 * p + 2] += s[6];
        grad_color[3 * p] += s[7];
        grad_color[3 * p + 1] += s[8];
        grad_color[3 * p + 2] += s[9];
        grad_opacity[p] += s[10];
    }
    free(part);
}

/* ----------------------------------------------------- preprocess backward */

/* SH colour backward, fastgs_ours/kernels_backward.cuh:22-86: accumulates the
 * SH coefficient gradients and returns dL/dposition through the view dir. */
static void sh_backward(const float* rest, float* g_sh0, float* g_rest,
                        const float gc[3], const float pos[3], const float cam[3],
                        int active_bases, float out[3]) {
    for (int c = 0; c < 3; ++c) g_sh0[c] += 0.28209479177387814f * gc[c];
    out[0] = out[1] = out[2] = 0.f;
    if (active_bases <= 1) return;
    float xr = pos[0] - cam[0], yr = pos[1] - cam[1], zr = pos[2] - cam[2];
    float inv = 1.0f / sqrtf(xr * xr + yr * yr + zr * zr);
    float x = xr * inv, y = yr * inv, z = zr * inv;
    float b[15];
    float dbx[15] = {0}, dby[15] = {0}, dbz[15] = {0};
    b[0] = -0.48860251190291987f * y; dby[0] = -0.48860251190291987f;
    b[1] = 0.48860251190291987f * z;  dbz[1] = 0.48860251190291987f;
    b[2] = -0.48860251190291987f * x; dbx[2] = -0.48860251190291987f;
    int nb = 3;
    if (active_bases > 4) {
        float xx = x * x, yy = y * y, zz = z * z, xy = x * y, xz = x * z, yz = y * z;
        b[3] = 1.0925484305920792f * xy; dbx[3] = 1.0925484305920792f * y; dby[3] = 1.0925484305920792f * x;
        b[4] = -1.0925484305920792f * yz; dby[4] = -1.0925484305920792f * z; dbz[4] = -1.0925484305920792f * y;
        b[5] = 0.94617469575755997f * zz - 0.31539156525251999f; dbz[5] = 1.8923493915151202f * z;
        b[6] = -1.0925484305920792f * xz; dbx[6] = -1.0925484305920792f * z; dbz[6] = -1.0925484305920792f * x;
        b[7] = 0.54627421529603959f * xx - 0.54627421529603959f * yy; dbx[7] = 1.0925484305920792f * x; dby[7] = -1.0925484305920792f * y;
        nb = 8;
        if (active_bases > 9) {
            b[8] = 0.59004358992664352f * y * (-3.0f * xx + yy);
            dbx[8] = -3.5402615395598609f * xy;
            dby[8] = -1.7701307697799304f * xx + 1.7701307697799304f * yy;
            b[9] = 2.8906114426405538f * xy * z;
            dbx[9] = 2.8906114426405538f * yz; dby[9] = 2.8906114426405538f * xz; dbz[9] = 2.8906114426405538f * xy;
            b[10] = 0.45704579946446572f * y * (1.0f - 5.0f * zz);
            dby[10] = 0.45704579946446572f - 2.2852289973223288f * zz; dbz[10] = -4.5704579946446566f * yz;
            b[11] = 0.3731763325901154f * z * (5.0f * zz - 3.0f);
            dbz[11] = 5.597644988851731f * zz - 1.1195289977703462f;
            b[12] = 0.45704579946446572f * x * (1.0f - 5.0f * zz);
            dbx[12] = 0.45704579946446572f - 2.2852289973223288f * zz; dbz[12] = -4.5704579946446566f * xz;
            b[13] = 1.4453057213202769f * z * (xx - yy);
            dbx[13] = 2.8906114426405538f * xz; dby[13] = -2.8906114426405538f * yz;
            dbz[13] = 1.4453057213202769f * xx - 1.4453057213202769f * yy;
            b[14] = 0.59004358992664352f * x * (-xx + 3.0f * yy);
            dbx[14] = -1.7701307697799304f * xx + 1.7701307697799304f * yy; dby[14] = 3.5402615395598609f * xy;
            nb = 15;
        }
    }
    float gd[3] = {0.f, 0.f, 0.f};
    for (int k = 0; k < nb; ++k) {
        for (int c = 0; c < 3; ++c) g_rest[3 * k + c] += b[k] * gc[c];
        float dot = rest[3 * k] * gc[0] + rest[3 * k + 1] * gc[1] + rest[3 * k + 2] * gc[2];
        gd[0] += dbx[k] * dot;
        gd[1] += dby[k] * dot;
        gd[2] += dbz[k] * dot;
    }
    float xx = xr * xr, yy = yr * yr, zz = zr * zr, xy = xr * yr, xz = xr * zr, yz = yr * zr;
    float ns = xx + yy + zz;
    float r = 1.0f / sqrtf(ns * ns * ns);
    out[0] = ((yy + zz) * gd[0] - xy * gd[1] - xz * gd[2]) * r;
    out[1] = (-xy * gd[0] + (xx + zz) * gd[1] - yz * gd[2]) * r;
    out[2] = (-xz * gd[0] - yz * gd[1] + (xx + yy) * gd[2]) * r;
}

void orc_preprocess_backward(
    int64_t n, const float* means, const float* rotations, const float* scales,
    const float* sh_rest, int32_t sh_degree, const OrcCamera* cam,
    const uint32_t* n_touched, const float* grad_mean2d,
    const float* grad_conic, int32_t conic_soa, const float* absgrad_mean2d,
    const float* grad_color, float* g_means, float* g_rotations,
    float* g_scales, float* g_sh0, float* g_sh_rest, float* dens,
    int32_t n_threads) {
    set_threads(n_threads);
    const float* r1 = cam->w2c;
    const float* r2 = cam->w2c + 4;
    const float* r3 = cam->w2c + 8;
    const float w = (float)cam->width, h = (float)cam->height;
    const int active_bases = (sh_degree + 1) * (sh_degree + 1);
    float campos[3];
    orc_camera_position(cam, campos);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        if (n_touched[i] == 0) continue;
        const float* m = means + 3 * i;
        float dmc[3];
        sh_backward(sh_rest + 45 * i, g_sh0 + 3 * i, g_sh_rest + 45 * i, grad_color + 3 * i, m,
                    campos, active_bases, dmc);
        float depth = r3[0] * m[0] + r3[1] * m[1] + r3[2] * m[2] + r3[3];
        float x = (r1[0] * m[0] + r1[1] * m[1] + r1[2] * m[2] + r1[3]) / depth;
        float y = (r2[0] * m[0] + r2[1] * m[1] + r2[2] * m[2] + r2[3]) / depth;
        const float* s = scales + 3 * i;
        float es[3] = {expf(s[0]), expf(s[1]), expf(s[2])};
        float var[3] = {es[0] * es[0], es[1] * es[1], es[2] * es[2]};
        const float* q = rotations + 4 * i;
        float qr = q[0], qx = q[1], qy = q[2], qz = q[3];
        float qn = qr * qr + qx * qx + qy * qy + qz * qz;
        float qxx = 2.0f * qx * qx / qn, qyy = 2.0f * qy * qy / qn, qzz = 2.0f * qz * qz / qn;
        float qxy = 2.0f * qx * qy / qn, qxz = 2.0f * qx * qz / qn, qyz = 2.0f * qy * qz / qn;
        float qrx = 2.0f * qr * qx / qn, qry = 2.0f * qr * qy / qn, qrz = 2.0f * qr * qz / qn;
        float R[3][3] = {{1.0f - (qyy + qzz), qxy - qrz, qry + qxz},
                         {qrz + qxy, 1.0f - (qxx + qzz), qyz - qrx},
                         {qxz - qry, qrx + qyz, 1.0f - (qxx + qyy)}};
        float RS[3][3];
        for (int a = 0; a < 3; ++a)
            for (int b = 0; b < 3; ++b) RS[a][b] = R[a][b] * var[b];
        float c11 = RS[0][0] * R[0][0] + RS[0][1] * R[0][1] + RS[0][2] * R[0][2];
        float c12 = RS[0][0] * R[1][0] + RS[0][1] * R[1][1] + RS[0][2] * R[1][2];
        float c13 = RS[0][0] * R[2][0] + RS[0][1] * R[2][1] + RS[0][2] * R[2][2];
        float c22 = RS[1][0] * R[1][0] + RS[1][1] * R[1][1] + RS[1][2] * R[1][2];
        float c23 = RS[1][0] * R[2][0] + RS[1][1] * R[2][1] + RS[1][2] * R[2][2];
        float c33 = RS[2][0] * R[2][0] + RS[2][1] * R[2][1] + RS[2][2] * R[2][2];
        float cl = (-0.15f * w - cam->cx) / cam->fx, cr = (1.15f * w - cam->cx) / cam->fx;
        float ct = (-0.15f * h - cam->cy) / cam->fy, cb = (1.15f * h - cam->cy) / cam->fy;
        float tx = clampf(x, cl, cr), ty = clampf(y, ct, cb);
        float j11 = cam->fx / depth, j13 = -j11 * tx, j22 = cam->fy / depth, j23 = -j22 * ty;
        float a1[3] = {j11 * r1[0] + j13 * r3[0], j11 * r1[1] + j13 * r3[1], j11 * r1[2] + j13 * r3[2]};
        float a2[3] = {j22 * r2[0] + j23 * r3[0], j22 * r2[1] + j23 * r3[1], j22 * r2[2] + j23 * r3[2]};
        float b1[3] = {a1[0] * c11 + a1[1] * c12 + a1[2] * c13, a1[0] * c12 + a1[1] * c22 + a1[2] * c23,
                       a1[0] * c13 + a1[1] * c23 + a1[2] * c33};
        float b2[3] = {a2[0] * c11 + a2[1] * c12 + a2[2] * c13, a2[0] * c12 + a2[1] * c22 + a2[2] * c23,
                       a2[0] * c13 + a2[1] * c23 + a2[2] * c33};
        float A = b1[0] * a1[0] + b1[1] * a1[1] + b1[2] * a1[2] + 0.3f;
        float B = b1[0] * a2[0] + b1[1] * a2[1] + b1[2] * a2[2];
        float C = b2[0] * a2[0] + b2[1] * a2[1] + b2[2] * a2[2] + 0.3f;
        float aa = A * A, bb = B * B, cc = C * C, ac = A * C, ab = A * B, bc = B * C;
        float det = ac - bb;
        float dr = 1.0f / (det + 1e-8f);
        float dr2 = dr * dr;
        float gcx, gcy, gcz;
        if (conic_soa) {
            gcx = grad_conic[i]; gcy = grad_conic[n + i]; gcz = grad_conic[2 * n + i];
        } else {
            gcx = grad_conic[3 * i]; gcy = grad_conic[3 * i + 1]; gcz = grad_conic[3 * i + 2];
        }
        /* note: no factor 2 on the off-diagonal term, as in the reference
         * (fastgs_ours/kernels_backward.cuh:210-214) */
        float d2a = dr2 * (2.0f * bc * gcy - cc * gcx - bb * gcz);
        float d2b = dr2 * (bc * gcx - (ac + bb) * gcy + ab * gcz);
        float d2c = dr2 * (2.0f * ab * gcy - bb * gcx - aa * gcz);
        float d3[6] = {
            (a1[0] * a1[0]) * d2a + 2.0f * (a1[0] * a2[0]) * d2b + (a2[0] * a2[0]) * d2c,
            (a1[0] * a1[1]) * d2a + (a1[0] * a2[1] + a1[1] * a2[0]) * d2b + (a2[0] * a2[1]) * d2c,
            (a1[0] * a1[2]) * d2a + (a1[0] * a2[2] + a1[2] * a2[0]) * d2b + (a2[0] * a2[2]) * d2c,
            (a1[1] * a1[1]) * d2a + 2.0f * (a1[1] * a2[1]) * d2b + (a2[1] * a2[1]) * d2c,
            (a1[1] * a1[2]) * d2a + (a1[1] * a2[2] + a1[2] * a2[1]) * d2b + (a2[1] * a2[2]) * d2c,
            (a1[2] * a1[2]) * d2a + 2.0f * (a1[2] * a2[2]) * d2b + (a2[2] * a2[2]) * d2c};
        float dj1[3], dj2[3];
        for (int k = 0; k < 3; ++k) {
            dj1[k] = 2.0f * (b1[k] * d2a + b2[k] * d2b);
            dj2[k] = 2.0f * (b1[k] * d2b + b2[k] * d2c);
        }
        float dj11 = r1[0] * dj1[0] + r1[1] * dj1[1] + r1[2] * dj1[2];
        float dj22 = r2[0] * dj2[0] + r2[1] * dj2[1] + r2[2] * dj2[2];
        float dj13 = r3[0] * dj1[0] + r3[1] * dj1[1] + r3[2] * dj1[2];
        float dj23 = r3[0] * dj2[0] + r3[1] * dj2[1] + r3[2] * dj2[2];
        float dtx = (x > cl && x < cr) ? 1.0f : 0.0f;
        float dty = (y > ct && y < cb) ? 1.0f : 0.0f;
        float dj13c = dj13 * dtx, dj23c = dj23 * dty;
        float h1 = dj11 - 2.0f * tx * dj13c;
        float h2 = dj22 - 2.0f * ty * dj23c;
        float gmx = grad_mean2d[2 * i], gmy = grad_mean2d[2 * i + 1];
        float dcam[3] = {j11 * (gmx - dj13c / depth), j22 * (gmy - dj23c / depth),
                         -j11 * (x * gmx + h1 / depth) - j22 * (y * gmy + h2 / depth)};
        for (int k = 0; k < 3; ++k)
            g_means[3 * i + k] += (r1[k] * dcam[0] + r2[k] * dcam[1] + r3[k] * dcam[2]) + dmc[k];
        /* log-scale gradient: 2 * exp(s) * exp(s) * dL/dvariance */
        float dv[3];
        for (int k = 0; k < 3; ++k)
            dv[k] = R[0][k] * R[0][k] * d3[0] + R[1][k] * R[1][k] * d3[3] + R[2][k] * R[2][k] * d3[5] +
                    2.0f * (R[0][k] * R[1][k] * d3[1] + R[0][k] * R[2][k] * d3[2] + R[1][k] * R[2][k] * d3[4]);
        for (int k = 0; k < 3; ++k) g_scales[3 * i + k] += 2.0f * es[k] * es[k] * dv[k];
        /* rotation, kernels_backward.cuh:306-336 */
        float dR[3][3];
        for (int k = 0; k < 3; ++k) {
            dR[0][k] = 2.0f * (RS[0][k] * d3[0] + RS[1][k] * d3[1] + RS[2][k] * d3[2]);
            dR[1][k] = 2.0f * (RS[0][k] * d3[1] + RS[1][k] * d3[3] + RS[2][k] * d3[4]);
            dR[2][k] = 2.0f * (RS[0][k] * d3[2] + RS[1][k] * d3[4] + RS[2][k] * d3[5]);
        }
        float dqxx = -dR[1][1] - dR[2][2], dqyy = -dR[0][0] - dR[2][2], dqzz = -dR[0][0] - dR[1][1];
        float dqxy = dR[0][1] + dR[1][0], dqxz = dR[0][2] + dR[2][0], dqyz = dR[1][2] + dR[2][1];
        float dqrx = dR[2][1] - dR[1][2], dqry = dR[0][2] - dR[2][0], dqrz = dR[1][0] - dR[0][1];
        float hn = qxx * dqxx + qyy * dqyy + qzz * dqzz + qxy * dqxy + qxz * dqxz + qyz * dqyz +
                   qrx * dqrx + qry * dqry + qrz * dqrz;
        float den = qn * sqrtf(qn);
        float gq[4] = {2.0f * (qx * dqrx + qy * dqry + qz * dqrz - qr * hn) / den,
                       2.0f * (2.0f * qx * dqxx + qy * dqxy + qz * dqxz + qr * dqrx - qx * hn) / den,
                       2.0f * (2.0f * qy * dqyy + qx * dqxy + qz * dqyz + qr * dqry - qy * hn) / den,
                       2.0f * (2.0f * qz * dqzz + qx * dqxz + qy * dqyz + qr * dqrz - qz * hn) / den};
        for (int k = 0; k < 4; ++k) g_rotations[4 * i + k] += gq[k];
        if (dens) {
            float* d = dens + 4 * i;
            d[0] += 1.0f;
            float ux = gmx * (0.5f * w), uy = gmy * (0.5f * h);
            d[1] += sqrtf(ux * ux + uy * uy);
            if (absgrad_mean2d) {
                float vx = absgrad_mean2d[2 * i] * (0.5f * w), vy = absgrad_mean2d[2 * i + 1] * (0.5f * h);
                d[2] += sqrtf(vx * vx + vy * vy);
            }
        }
    }
}

/* ------------------------------------------------------------------ losses */

void orc_l1_f32(int32_t width, int32_t height, const float* pred,
                const float* target, float* loss_map, float* grad, float scale) {
    const uint32_t wp = ((uint32_t)width + 7u) & ~7u, hp = ((uint32_t)height + 7u) & ~7u;
    const int64_t total = (int64_t)wp * hp * 3;
    const float s = scale / (float)(width * height * 3);
    for (int64_t i = 0; i < total; ++i) {
        float p = satf(pred[i]);
        float d = p - target[i];
        if (loss_map) loss_map[i] = fmaf(fabsf(d), s, loss_map[i]);
        if (grad) grad[i] = fmaf(copysignf(1.0f, d), s, grad[i]);
    }
}

void orc_l1_f16(int32_t width, int32_t height, const uint16_t* pred,
                const uint16_t* target, uint16_t* loss_map, uint16_t* grad, float scale) {
    const uint32_t wp = ((uint32_t)width + 7u) & ~7u, hp = ((uint32_t)height + 7u) & ~7u;
    const int64_t total = (int64_t)wp * hp * 3;
    const float s = scale / (float)(width * height * 3);
    for (int64_t i = 0; i < total; ++i) {
        float p = satf(orc_h2f(pred[i]));
        float d = p - orc_h2f(target[i]);
        if (loss_map) loss_map[i] = orc_f2h(fmaf(fabsf(d), s, orc_h2f(loss_map[i])));
        if (grad) grad[i] = orc_f2h(fmaf(copysignf(1.0f, d), s, orc_h2f(grad[i])));
    }
}

static const float kGauss[11] = {0.001028380123898387f, 0.0075987582094967365f, 0.036000773310661316f,
                                 0.10936068743467331f,  0.21300552785396576f,   0.26601171493530273f,
                                 0.21300552785396576f,  0.10936068743467331f,   0.036000773310661316f,
                                 0.0075987582094967365f, 0.001028380123898387f};

/* SSIM core, fused_ssim.cu:55-442.  x, y: [H][W] row-major, already the
 * values the reference's convolutions see.  Writes the per-pixel (1 - ssim)
 * and the three backward sums S0..S2 (the Gaussian-window convolutions of
 * dssim/dmu1, dssim/dsigma1^2 and dssim/dsigma12), zero padding throughout.
 * The caller combines dL/dpred = S0 + 2*p*S1 + t*S2 (fused_ssim.cu:436). */
static void ssim_plane(int W, int H, const float* x, const float* y, float* one_minus_ssim,
                       float* S) {
    const float C1 = 0.01f * 0.01f, C2 = 0.03f * 0.03f;
    size_t np = (size_t)W * H;
    float* hx = (float*)malloc(sizeof(float) * np * 5);
    float* pd = (float*)malloc(sizeof(float) * np * 3);
    float* hp = (float*)malloc(sizeof(float) * np * 3);
    for (int r = 0; r < H; ++r)
        for (int c = 0; c < W; ++c) {
            float s[5] = {0, 0, 0, 0, 0};
            for (int d = 0; d < 11; ++d) {
                int cc = c + d - 5;
                float X = 0.f, Y = 0.f;
                if (cc >= 0 && cc < W) { X = x[(size_t)r * W + cc]; Y = y[(size_t)r * W + cc]; }
                float wv = kGauss[d];
                s[0] += X * wv; s[1] += (X * X) * wv; s[2] += Y * wv; s[3] += (Y * Y) * wv; s[4] += (X * Y) * wv;
            }
            for (int k = 0; k < 5; ++k) hx[((size_t)r * W + c) * 5 + k] = s[k];
        }
    for (int r = 0; r < H; ++r)
        for (int c = 0; c < W; ++c) {
            float o[5] = {0, 0, 0, 0, 0};
            for (int d = 0; d < 11; ++d) {
                int rr = r + d - 5;
                if (rr < 0 || rr >= H) continue;
                for (int k = 0; k < 5; ++k) o[k] += hx[((size_t)rr * W + c) * 5 + k] * kGauss[d];
            }
            float mu1 = o[0], mu2 = o[2];
            float m11 = mu1 * mu1, m22 = mu2 * mu2;
            float s1 = o[1] - m11, s2 = o[3] - m22, s12 = o[4] - mu1 * mu2;
            float A = m11 + m22 + C1, B = s1 + s2 + C2, Cc = 2.f * mu1 * mu2 + C1, D = 2.f * s12 + C2;
            size_t i = (size_t)r * W + c;
            one_minus_ssim[i] = 1.f - (Cc * D) / (A * B);
            pd[3 * i + 0] = (mu2 * 2.f * D) / (A * B) - (mu2 * 2.f * Cc) / (A * B) -
                            (mu1 * 2.f * Cc * D) / (A * A * B) + (mu1 * 2.f * Cc * D) / (A * B * B);
            pd[3 * i + 1] = (-Cc * D) / (A * B * B);
            pd[3 * i + 2] = (2.f * Cc) / (A * B);
        }
    for (int r = 0; r < H; ++r)
        for (int c = 0; c < W; ++c) {
            float s[3] = {0, 0, 0};
            for (int d = 0; d < 11; ++d) {
                int cc = c + d - 5;
                if (cc < 0 || cc >= W) continue;
                for (int k = 0; k < 3; ++k) s[k] += pd[((size_t)r * W + cc) * 3 + k] * kGauss[d];
            }
            for (int k = 0; k < 3; ++k) hp[((size_t)r * W + c) * 3 + k] = s[k];
        }
    for (int r = 0; r < H; ++r)
        for (int c = 0; c < W; ++c) {
            float s[3] = {0, 0, 0};
            for (int d = 0; d < 11; ++d) {
                int rr = r + d - 5;
                if (rr < 0 || rr >= H) continue;
                for (int k = 0; k < 3; ++k) s[k] += hp[((size_t)rr * W + c) * 3 + k] * kGauss[d];
            }
            for (int k = 0; k < 3; ++k) S[3 * ((size_t)r * W + c) + k] = s[k];
        }
    free(hx);
    free(pd);
    free(hp);
}

void orc_ssim_f32(int32_t width, int32_t height, const float* pred,
                  const float* target, float* loss_map, float* grad,
                  float scale, int32_t n_threads) {
    set_threads(n_threads);
    const uint32_t tw = ((uint32_t)width + 7u) >> 3, th = ((uint32_t)height + 7u) >> 3;
    const uint32_t plane = tw * th * 64;
    const float s = scale / (float)(width * height);
    size_t np = (size_t)width * height;
#pragma omp parallel for schedule(static)
    for (int ch = 0; ch < 3; ++ch) {
        float* x = (float*)malloc(sizeof(float) * np);
        float* y = (float*)malloc(sizeof(float) * np);
        float* l = (float*)malloc(sizeof(float) * np);
        float* S = (float*)malloc(sizeof(float) * np * 3);
        for (int r = 0; r < height; ++r)
            for (int c = 0; c < width; ++c) {
                uint32_t pi = tiled_index((uint32_t)r, (uint32_t)c, tw) + ch * plane;
                /* the fp32 forward stages both images as fp16 (fused_ssim.cu:97,137) */
                x[(size_t)r * width + c] = orc_h2f(orc_f2h(pred[pi]));
                y[(size_t)r * width + c] = orc_h2f(orc_f2h(target[pi]));
            }
        ssim_plane(width, height, x, y, l, S);
        for (int r = 0; r < height; ++r)
            for (int c = 0; c < width; ++c) {
                uint32_t pi = tiled_index((uint32_t)r, (uint32_t)c, tw) + ch * plane;
                size_t i = (size_t)r * width + c;
                if (loss_map) loss_map[pi] += l[i] * s;
                if (grad) {
                    /* the backward reads the fp32 pixels (fused_ssim.cu:319-322) */
                    float dL = S[3 * i] + (2.f * pred[pi]) * S[3 * i + 1] + target[pi] * S[3 * i + 2];
                    grad[pi] += -s * dL;
                }
            }
        free(x);
        free(y);
        free(l);
        free(S);
    }
}

void orc_ssim_f16(int32_t width, int32_t height, const uint16_t* pred,
                  const uint16_t* target, uint16_t* loss_map, uint16_t* grad,
                  float scale, int32_t n_threads) {
    set_threads(n_threads);
    const uint32_t tw = ((uint32_t)width + 7u) >> 3, th = ((uint32_t)height + 7u) >> 3;
    const uint32_t plane = tw * th * 64;
    const float s = scale / (float)(width * height);
    size_t np = (size_t)width * height;
#pragma omp parallel for schedule(static)
    for (int ch = 0; ch < 3; ++ch) {
        float* x = (float*)malloc(sizeof(float) * np);
        float* y = (float*)malloc(sizeof(float) * np);
        float* l = (float*)malloc(sizeof(float) * np);
        float* S = (float*)malloc(sizeof(float) * np * 3);
        for (int r = 0; r < height; ++r)
            for (int c = 0; c < width; ++c) {
                uint32_t pi = tiled_index((uint32_t)r, (uint32_t)c, tw) + ch * plane;
                x[(size_t)r * width + c] = orc_h2f(pred[pi]);
                y[(size_t)r * width + c] = orc_h2f(target[pi]);
            }
        ssim_plane(width, height, x, y, l, S);
        for (int r = 0; r < height; ++r)
            for (int c = 0; c < width; ++c) {
                uint32_t pi = tiled_index((uint32_t)r, (uint32_t)c, tw) + ch * plane;
                size_t i = (size_t)r * width + c;
                if (loss_map) loss_map[pi] = orc_f2h(fmaf(l[i], s, orc_h2f(loss_map[pi])));
                if (grad) {
                    float dL = S[3 * i] + (2.f * x[i]) * S[3 * i + 1] + y[i] * S[3 * i + 2];
                    grad[pi] = orc_f2h(fmaf(-s, dL, orc_h2f(grad[pi])));
                }
            }
        free(x);
        free(y);
        free(l);
        free(S);
    }
}

/* ------------------------------------------------------------------- adam */

void orc_adam(int64_t count, float* theta, const float* grad, float* m,
              float* v, float lr, float beta1, float beta2, float eps,
              float gradient_scale, float bias_correction1,
              float bias_correction2_sqrt, float max_grad_1,
              int32_t decay_kind, float decay) {
    /* element-wise, so the thread count does not change the result */
#pragma omp parallel for schedule(static) if (count > 65536)
    for (int64_t i = 0; i < count; ++i) {
        float th = theta[i];
        float g = gradient_scale * grad[i];
        if (decay_kind == 1) {
            float s = 1.0f / (1.0f + expf(-th));
            g = g + decay * (s * (1.0f - s));
        } else if (decay_kind == 2) {
            g = g + decay * expf(th);
        }
        if (max_grad_1 != 0.0f) g = copysignf(fminf(fabsf(g), max_grad_1), g);
        float t1 = 1.0f - beta1, t2 = 1.0f - beta2;
        float mm = fmaf(t1, g, fmaf(-t1, m[i], m[i]));
        float vv = fmaf(t2, g * g, fmaf(-t2, v[i], v[i]));
        float mh = mm / bias_correction1;
        float den = sqrtf(vv) / bias_correction2_sqrt + eps;
        th -= mh * lr / den;
        theta[i] = th;
        m[i] = mm;
        v[i] = vv;
    }
}

/* ------------------------------------------------------ densification */

#define PCG32_MULT 0x5851f42d4c957f2dULL

uint32_t orc_pcg32_next_uint(OrcPcg32* r) {
    const uint64_t old = r->state;
    r->state = old * PCG32_MULT + r->inc;
    const uint32_t xorshifted = (uint32_t)(((old >> 18u) ^ old) >> 27u);
    const uint32_t rot = (uint32_t)(old >> 59u);
    return (xorshifted >> rot) | (xorshifted << ((~rot + 1u) & 31u));
}

void orc_pcg32_seed(OrcPcg32* r, uint64_t initstate, uint64_t initseq) {
    r->state = 0u;
    r->inc = (initseq << 1u) | 1u;
    (void)orc_pcg32_next_uint(r);
    r->state += initstate;
    (void)orc_pcg32_next_uint(r);
}

/* [0, 1): 23 random mantissa bits under exponent 0, minus 1 */
float orc_pcg32_next_float(OrcPcg32* r) {
    union {
        uint32_t u;
        float f;
    } x;
    x.u = (orc_pcg32_next_uint(r) >> 9) | 0x3f800000u;
    return x.f - 1.0f;
}

/* jump ahead by delta draws: the LCG's affine map composed by squaring
 * (F. B. Brown, "Random number generation with arbitrary strides", 1994) */
void orc_pcg32_advance(OrcPcg32* r, uint64_t delta) {
    uint64_t cur_mult = PCG32_MULT, cur_plus = r->inc, acc_mult = 1u, acc_plus = 0u;
    while (delta > 0) {
        if (delta & 1u) {
            acc_mult *= cur_mult;
            acc_plus = acc_plus * cur_mult + cur_plus;
        }
        cur_plus = (cur_mult + 1u) * cur_plus;
        cur_mult *= cur_mult;
        delta >>= 1u;
    }
    r->state = acc_mult * r->state + acc_plus;
}

/* common.hpp:358-364 */
static inline float logistic_f(float x) { return 1.0f / (1.0f + expf(-x)); }
static inline float logit_f(float x) { return -logf(1.0f / clampf(x, 1e-9f, 1.0f - 1e-9f) - 1.0f); }

void orc_random_logistic(OrcPcg32* r, int64_t n, float* out) {
    const int64_t per = 4, block = 128;
    const int64_t work = (n + per - 1) / per;
    const int64_t threads = ((work + block - 1) / block) * block;
#pragma omp parallel for schedule(static) if (n > 65536)
    for (int64_t idx = 0; idx < n; ++idx) {
        OrcPcg32 g = *r;
        orc_pcg32_advance(&g, (uint64_t)((idx % threads) * per + idx / threads));
        out[idx] = logit_f(orc_pcg32_next_float(&g)) * 1.0f * 0.551328895f + 0.0f;
    }
    orc_pcg32_advance(r, (uint64_t)n);
}

static const int kSegW[6] = {3, 1, 4, 3, 3, 45};
static float* seg_of(OrcSet s, int k) {
    switch (k) {
        case 0: return s.means;
        case 1: return s.opacities;
        case 2: return s.rotations;
        case 3: return s.scales;
        case 4: return s.sh0;
        default: return s.sh_rest;
    }
}

static void zero_rows(OrcSet s, int64_t from, int64_t to) {
    for (int k = 0; k < 6; ++k) {
        float* p = seg_of(s, k);
        if (p != NULL && to > from) memset(p + from * kSegW[k], 0, sizeof(float) * (size_t)((to - from) * kSegW[k]));
    }
}

/* stable compaction of the rows with keep[i] != 0 */
static void compact_rows(OrcSet s, const uint8_t* keep, int64_t n) {
    for (int k = 0; k < 6; ++k) {
        float* p = seg_of(s, k);
        if (p == NULL) continue;
        const int w = kSegW[k];
        int64_t o = 0;
        for (int64_t i = 0; i < n; ++i)
            if (keep[i]) {
                if (o != i) memmove(p + o * w, p + i * w, sizeof(float) * (size_t)w);
                ++o;
            }
    }
}

int64_t orc_densify_step(int64_t n, int64_t capacity, OrcSet params, OrcSet grads, OrcSet exp_avg,
                         OrcSet exp_avg_sq, float* dens, const OrcDensifyConfig* cfg, int32_t step,
                         OrcPcg32* rng) {
    const int refine = step % cfg->refine_every == 0 && step >= cfg->start_refine && step <= cfg->end_refine;
    if (refine) {
        const int64_t n0 = n;
        /* duplicate (default.cu:151-296) */
        uint8_t* flag = (uint8_t*)calloc((size_t)(n0 > 0 ? n0 : 1), 1);
        int64_t grows = 0;
        if (n0 < cfg->max_num_gaussians) {
            const float grow_scale = cfg->duplicate_scale_threshold * cfg->scene_scale;
            const float grow_grad = cfg->duplicate_grad_threshold * cfg->grad_scaler;
            for (int64_t i = 0; i < n0; ++i) {
                const float* d = dens + 4 * i;
                const float accum = cfg->absgrad ? d[2] : d[1];
                const float grad = accum / fmaxf(d[0], 1.0f);
                if (grad > grow_grad && d[0] > 0.0f) {
                    const float* sc = params.scales + 3 * i;
                    const float mx = fmaxf(fmaxf(expf(sc[0]), expf(sc[1])), expf(sc[2]));
                    flag[i] = mx > grow_scale ? 2 : 1;
                    ++grows;
                }
            }
        }
        if (n0 + grows > capacity) {
            free(flag);
            return -1;
        }
        if (grows > 0) {
            float* rnd = (float*)malloc(sizeof(float) * (size_t)(6 * grows));
            orc_random_logistic(rng, 6 * grows, rnd);
            /* appended rows start as zeros (GPUGaussian3d::append, SimpleAdam::duplicate) */
            zero_rows(grads, n0, n0 + grows);
            zero_rows(exp_avg, n0, n0 + grows);
            zero_rows(exp_avg_sq, n0, n0 + grows);
            int64_t g = 0;
            for (int64_t src = 0; src < n0; ++src) {
                if (!flag[src]) continue;
                const int64_t dst = n0 + g;
                memcpy(params.rotations + 4 * dst, params.rotations + 4 * src, 4 * sizeof(float));
                memcpy(params.sh0 + 3 * dst, params.sh0 + 3 * src, 3 * sizeof(float));
                memcpy(params.sh_rest + 45 * dst, params.sh_rest + 45 * src, 45 * sizeof(float));
                if (flag[src] == 1) {
                    memcpy(params.means + 3 * dst, params.means + 3 * src, 3 * sizeof(float));
                    memcpy(params.scales + 3 * dst, params.scales + 3 * src, 3 * sizeof(float));
                    params.opacities[dst] = params.opacities[src];
                } else {
                    /* split: glm::mat3 built column by column from (w, x, y, z)
                     * (default.cu:268-276), applied as a column-major matrix */
                    const float* q = params.rotations + 4 * src;
                    const float r = q[0], x = q[1], y = q[2], z = q[3];
                    const float c0[3] = {1.f - 2.f * (y * y + z * z), 2.f * (x * y - r * z), 2.f * (x * z + r * y)};
                    const float c1[3] = {2.f * (x * y + r * z), 1.f - 2.f * (x * x + z * z), 2.f * (y * z - r * x)};
                    const float c2[3] = {2.f * (x * z - r * y), 2.f * (y * z + r * x), 1.f - 2.f * (x * x + y * y)};
                    const float* sc = params.scales + 3 * src;
                    const float act[3] = {expf(sc[0]), expf(sc[1]), expf(sc[2])};
                    const float new_op = 1.0f - sqrtf(1.0f - logistic_f(params.opacities[src]));
                    const float* r1 = rnd + 6 * g;
                    const float* r2 = rnd + 6 * g + 3;
                    float v1[3], v2[3];
                    for (int k = 0; k < 3; ++k) {
                        v1[k] = r1[k] * (act[k] + 1e-5f);
                        v2[k] = r2[k] * (act[k] + 1e-5f);
                    }
                    float* ms = params.means + 3 * src;
                    float* md = params.means + 3 * dst;
                    for (int k = 0; k < 3; ++k) {
                        const float off1 = c0[k] * v1[0] + c1[k] * v1[1] + c2[k] * v1[2];
                        const float off2 = c0[k] * v2[0] + c1[k] * v2[1] + c2[k] * v2[2];
                        md[k] = ms[k] + off1;
                        ms[k] = ms[k] + off2;
                    }
                    for (int k = 0; k < 3; ++k) {
                        const float ns = logf(act[k] / 1.6f);
                        params.scales[3 * dst + k] = ns;
                        params.scales[3 * src + k] = ns;
                    }
                    params.opacities[dst] = logit_f(new_op);
                    params.opacities[src] = logit_f(new_op);
                }
                ++g;
            }
            free(rnd);
        }
        free(flag);
        n = n0 + grows;
        /* prune (default.cu:298-345) */
        uint8_t* keep = (uint8_t*)malloc((size_t)(n > 0 ? n : 1));
        const float ss_thr = (float)(cfg->image_width > cfg->image_height ? cfg->image_width : cfg->image_height) *
                             cfg->max_screen_size;
        const int prune_large = step > cfg->reset_every;
        int64_t kept = 0;
        for (int64_t i = 0; i < n; ++i) {
            const float* sc = params.scales + 3 * i;
            const float mx = fmaxf(fmaxf(expf(sc[0]), expf(sc[1])), expf(sc[2]));
            const int not_large_ws = mx < cfg->pruning_scale_threshold * cfg->scene_scale;
            const int not_large_ss = i >= n0 || dens[4 * i + 3] < ss_thr;
            const int not_transparent = logistic_f(params.opacities[i]) > cfg->pruning_opacity_threshold;
            const float* q = params.rotations + 4 * i;
            const int not_degenerate = fabsf(q[0]) + fabsf(q[1]) + fabsf(q[2]) + fabsf(q[3]) > 1.1920929e-07f;
            keep[i] = (uint8_t)(not_transparent && ((not_large_ws && not_large_ss) || !prune_large) && not_degenerate);
            kept += keep[i];
        }
        if (kept > 0) {  /* StrategyBase::on_remove returns early on 0 (strategy.cpp:21) */
            compact_rows(params, keep, n);
            compact_rows(grads, keep, n);
            compact_rows(exp_avg, keep, n);
            compact_rows(exp_avg_sq, keep, n);
            n = kept;
        }
        free(keep);
        memset(dens, 0, sizeof(float) * 4 * (size_t)n);
    }
    if (cfg->reset_every > 0 && step % cfg->reset_every == 0 && step >= cfg->start_refine &&
        step < cfg->end_refine) {
        const float cap = 2.0f * cfg->pruning_opacity_threshold;
        for (int64_t i = 0; i < n; ++i) params.opacities[i] = logit_f(fminf(logistic_f(params.opacities[i]), cap));
        if (exp_avg.opacities) memset(exp_avg.opacities, 0, sizeof(float) * (size_t)n);
        if (exp_avg_sq.opacities) memset(exp_avg_sq.opacities, 0, sizeof(float) * (size_t)n);
    }
    return n;
}

/* ------------------------------------------------------------ Morton order */

typedef struct { uint32_t code, idx; } MortonPair;

static int morton_cmp(const void* a, const void* b) {
    const MortonPair* x = (const MortonPair*)a;
    const MortonPair* y = (const MortonPair*)b;
    if (x->code != y->code) return x->code < y->code ? -1 : 1;
    return x->idx < y->idx ? -1 : (x->idx > y->idx ? 1 : 0);
}

/* bit i of v (i < 10) to bit 3i */
static uint32_t spread10(uint32_t v) {
    uint32_t out = 0;
    for (int i = 0; i < 10; ++i) out |= ((v >> i) & 1u) << (3 * i);
    return out;
}

/* reorder(), tinygs/src/orchestrator.cu:26-100: bounding box of the means,
 * inverse extents 1 / max(max - min, 1e-8) (std::max semantics), 10-bit
 * quantisation of each normalised, clamped coordinate (x 1023, truncated),
 * the 30-bit Morton code (x -> bit 3i, y -> 3i+1, z -> 3i+2) and a stable
 * sort by code (CUB's radix sort is stable: equal codes keep index order). */
void orc_morton_order(int64_t n, const float* means, uint32_t* perm) {
    if (n <= 0) return;
    float lo[3] = {FLT_MAX, FLT_MAX, FLT_MAX}, hi[3] = {-FLT_MAX, -FLT_MAX, -FLT_MAX};
    for (int64_t i = 0; i < n; ++i)
        for (int c = 0; c < 3; ++c) {
            lo[c] = fminf(lo[c], means[3 * i + c]);
            hi[c] = fmaxf(hi[c], means[3 * i + c]);
        }
    float inv[3];
    for (int c = 0; c < 3; ++c) {
        float d = hi[c] - lo[c];
        float e = d < 1e-8f ? 1e-8f : d;
        inv[c] = 1.0f / e;
    }
    MortonPair* pairs = (MortonPair*)malloc(sizeof(MortonPair) * (size_t)n);
    for (int64_t i = 0; i < n; ++i) {
        uint32_t q[3];
        for (int c = 0; c < 3; ++c) {
            float v = (means[3 * i + c] - lo[c]) * inv[c];
            float u = fminf(fmaxf(v, 0.0f), 1.0f);
            float s = u * 1023.0f;
            q[c] = (uint32_t)s;
        }
        pairs[i].code = spread10(q[0]) | (spread10(q[1]) << 1) | (spread10(q[2]) << 2);
        pairs[i].idx = (uint32_t)i;
    }
    qsort(pairs, (size_t)n, sizeof(MortonPair), morton_cmp);
    for (int64_t i = 0; i < n; ++i) perm[i] = pairs[i].idx;
    free(pairs);
}
