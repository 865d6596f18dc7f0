/*
 * moe_oracle.c -- CPU restatement of the reference's MoE MUL_MAT_ID path.
 *
 * TEST INFRASTRUCTURE ONLY (parity checker and timed CPU baseline). The CUDA
 * product never links or calls this file. See moe_oracle.h for what each part
 * restates and how it is pinned.
 *
 * Build: oracle/Makefile (gcc -O3 -ffp-contract=off, pthreads). Contraction is
 * off so every float expression rounds exactly as written, which is what the
 * bit-exact activation-quantizer comparisons rely on.
 */
#include "moe_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

#define QK_K 256

/* ------------------------------------------------------------------------ */
/* block layouts (ggml-common.h formats; byte offsets written out explicitly) */
/* ------------------------------------------------------------------------ */
/*  Q4_0  18 B / 32 : d f16 @0, qs[16] @2 (lo nibble = elem j, hi = elem j+16)
 *  Q5_0  22 B / 32 : d f16 @0, qh u32 @2 (bit j = 5th bit of elem j), qs[16] @6
 *  Q8_0  34 B / 32 : d f16 @0, qs i8[32] @2
 *  Q8_1  36 B / 32 : d f16 @0, s f16 @2, qs i8[32] @4
 *  Q2_K  84 B /256 : scales[16] @0 (lo nib scale, hi nib min), qs[64] @16,
 *                    d f16 @80, dmin f16 @82
 *  Q3_K 110 B /256 : hmask[32] @0, qs[64] @32, scales[12] @96, d f16 @108
 *  Q4_K 144 B /256 : d f16 @0, dmin f16 @2, scales[12] @4, qs[128] @16
 *  Q5_K 176 B /256 : d @0, dmin @2, scales[12] @4, qh[32] @16, qs[128] @48
 *  Q6_K 210 B /256 : ql[128] @0, qh[64] @128, scales i8[16] @192, d f16 @208
 *  Q8_K 292 B /256 : d f32 @0, qs i8[256] @4, bsums i16[16] @260
 */

int orc_blck_size(int type) {
    switch (type) {
        case ORC_F32: case ORC_F16: return 1;
        case ORC_Q4_0: case ORC_Q5_0: case ORC_Q8_0: case ORC_Q8_1: return 32;
        case ORC_Q2_K: case ORC_Q3_K: case ORC_Q4_K: case ORC_Q5_K:
        case ORC_Q6_K: case ORC_Q8_K: return QK_K;
        default: return 0;
    }
}

int orc_type_size(int type) {
    switch (type) {
        case ORC_F32: return 4;
        case ORC_F16: return 2;
        case ORC_Q4_0: return 18;
        case ORC_Q5_0: return 22;
        case ORC_Q8_0: return 34;
        case ORC_Q8_1: return 36;
        case ORC_Q2_K: return 84;
        case ORC_Q3_K: return 110;
        case ORC_Q4_K: return 144;
        case ORC_Q5_K: return 176;
        case ORC_Q6_K: return 210;
        case ORC_Q8_K: return 292;
        default: return 0;
    }
}

size_t orc_row_size(int type, int64_t n) {
    const int bs = orc_blck_size(type);
    if (bs == 0 || n % bs) return 0;
    return (size_t)(n / bs) * (size_t)orc_type_size(type);
}

/* CPU type traits pairing, ggml-cpu.c:250-339 */
int orc_vec_dot_type(int type) {
    switch (type) {
        case ORC_Q4_0: case ORC_Q5_0: case ORC_Q8_0: return ORC_Q8_0;
        case ORC_Q2_K: case ORC_Q3_K: case ORC_Q4_K: case ORC_Q5_K: case ORC_Q6_K: return ORC_Q8_K;
        default: return -1;
    }
}

/* IEEE binary16 conversion, round to nearest even (own implementation) */
uint16_t orc_fp32_to_fp16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t exp  = (x >> 23) & 0xffu;
    uint32_t mant       = x & 0x7fffffu;
    if (exp == 0xffu) {
        return (uint16_t)(sign | 0x7c00u | (mant ? (0x200u | (mant >> 13)) : 0u));
    }
    const int32_t e = (int32_t)exp - 127 + 15;
    if (e >= 0x1f) return (uint16_t)(sign | 0x7c00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        mant |= 0x800000u;
        const int shift = 14 - e;
        uint32_t hm = mant >> shift;
        const uint32_t rem = mant & ((1u << shift) - 1u);
        const uint32_t halfway = 1u << (shift - 1);
        if (rem > halfway || (rem == halfway && (hm & 1u))) hm++;
        return (uint16_t)(sign | hm);
    }
    uint32_t h = sign | ((uint32_t)e << 10) | (mant >> 13);
    const uint32_t rem = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    return (uint16_t)h;
}

float orc_fp16_to_fp32(uint16_t h) {
    const uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t exp  = ((uint32_t)h >> 10) & 0x1fu;
    uint32_t mant = (uint32_t)h & 0x3ffu;
    uint32_t x;
    if (exp == 0x1fu) {
        x = sign | 0x7f800000u | (mant << 13);
    } else if (exp == 0) {
        if (mant == 0) {
            x = sign;
        } else {
            int e = -1;
            do { mant <<= 1; e++; } while (!(mant & 0x400u));
            mant &= 0x3ffu;
            x = sign | ((uint32_t)(127 - 15 - e) << 23) | (mant << 13);
        }
    } else {
        x = sign | ((exp + 127u - 15u) << 23) | (mant << 13);
    }
    float f;
    memcpy(&f, &x, 4);
    return f;
}

static inline uint16_t rd16(const uint8_t *p) { uint16_t v; memcpy(&v, p, 2); return v; }
static inline float    rdh(const uint8_t *p)  { return orc_fp16_to_fp32(rd16(p)); }
static inline void     wrh(uint8_t *p, float f) { uint16_t v = orc_fp32_to_fp16(f); memcpy(p, &v, 2); }

/* 16 packed 6-bit Q3_K scales -> signed values (stored value - 32).
 * Layout: low nibble of scale k<8 in byte k bits 0-3, k>=8 in byte k-8 bits
 * 4-7; the two high bits of scale k in byte 8+(k%4), bit pair k/4. */
static void q3k_scales(const uint8_t *s12, int sc[16]) {
    for (int k = 0; k < 16; ++k) {
        const int lo = k < 8 ? (s12[k] & 0xF) : (s12[k - 8] >> 4);
        const int hi = (s12[8 + (k % 4)] >> (2 * (k / 4))) & 3;
        sc[k] = (lo | (hi << 4)) - 32;
    }
}

/* Q4_K / Q5_K 6-bit scale/min pair j (0..7) from the 12 packed bytes */
static void k4_scale_min(int j, const uint8_t *q, int *d, int *m) {
    if (j < 4) {
        *d = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *d = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
        *m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

/* integer weight codes + per-element float affine, shared by dequant and the
 * exact dot. Fills for each element i: value = a[i] * q[i] - b[i] with a/b the
 * element's effective scale and offset (exact in double). */
static void block_affine(int type, const uint8_t *b, int q[QK_K], double sa[QK_K], double sb[QK_K]) {
    switch (type) {
        case ORC_Q4_0: {
            const double d = rdh(b);
            for (int j = 0; j < 16; ++j) {
                q[j]      = (b[2 + j] & 0xF) - 8;
                q[j + 16] = (b[2 + j] >> 4) - 8;
            }
            for (int i = 0; i < 32; ++i) { sa[i] = d; sb[i] = 0; }
        } break;
        case ORC_Q5_0: {
            const double d = rdh(b);
            uint32_t qh; memcpy(&qh, b + 2, 4);
            for (int j = 0; j < 16; ++j) {
                q[j]      = ((b[6 + j] & 0xF) | (((qh >> j) & 1u) << 4)) - 16;
                q[j + 16] = ((b[6 + j] >> 4) | (((qh >> (j + 16)) & 1u) << 4)) - 16;
            }
            for (int i = 0; i < 32; ++i) { sa[i] = d; sb[i] = 0; }
        } break;
        case ORC_Q8_0: {
            const double d = rdh(b);
            for (int i = 0; i < 32; ++i) { q[i] = (int8_t)b[2 + i]; sa[i] = d; sb[i] = 0; }
        } break;
        case ORC_Q2_K: {
            const double d = rdh(b + 80), dmin = rdh(b + 82);
            for (int n = 0; n < 2; ++n)
                for (int s = 0; s < 4; ++s)
                    for (int l = 0; l < 32; ++l) {
                        const int i = n * 128 + s * 32 + l;
                        const int sbi = i / 16;
                        q[i]  = (b[16 + n * 32 + l] >> (2 * s)) & 3;
                        sa[i] = d * (b[sbi] & 0xF);
                        sb[i] = dmin * (b[sbi] >> 4);
                    }
        } break;
        case ORC_Q3_K: {
            const double d = rdh(b + 108);
            int sc[16];
            q3k_scales(b + 96, sc);
            for (int n = 0; n < 2; ++n)
                for (int s = 0; s < 4; ++s)
                    for (int l = 0; l < 32; ++l) {
                        const int i = n * 128 + s * 32 + l;
                        const int hbit = (b[l] >> (n * 4 + s)) & 1;
                        q[i]  = ((b[32 + n * 32 + l] >> (2 * s)) & 3) - (hbit ? 0 : 4);
                        sa[i] = d * sc[i / 16];
                        sb[i] = 0;
                    }
        } break;
        case ORC_Q4_K:
        case ORC_Q5_K: {
            const double d = rdh(b), dmin = rdh(b + 2);
            const uint8_t *qs = b + (type == ORC_Q4_K ? 16 : 48);
            for (int c = 0; c < 4; ++c) {
                int d0, m0, d1, m1;
                k4_scale_min(2 * c, b + 4, &d0, &m0);
                k4_scale_min(2 * c + 1, b + 4, &d1, &m1);
                for (int l = 0; l < 32; ++l) {
                    int lo = qs[32 * c + l] & 0xF, hi = qs[32 * c + l] >> 4;
                    if (type == ORC_Q5_K) {
                        lo |= ((b[16 + l] >> (2 * c)) & 1) << 4;
                        hi |= ((b[16 + l] >> (2 * c + 1)) & 1) << 4;
                    }
                    q[64 * c + l] = lo;      sa[64 * c + l] = d * d0;      sb[64 * c + l] = dmin * m0;
                    q[64 * c + 32 + l] = hi; sa[64 * c + 32 + l] = d * d1; sb[64 * c + 32 + l] = dmin * m1;
                }
            }
        } break;
        case ORC_Q6_K: {
            const double d = rdh(b + 208);
            const int8_t *sc = (const int8_t *)(b + 192);
            for (int n = 0; n < 2; ++n)
                for (int l = 0; l < 32; ++l) {
                    const uint8_t *ql = b + 64 * n, *qh = b + 128 + 32 * n;
                    const int base = 128 * n;
                    q[base + l]      = ((ql[l] & 0xF)      | (((qh[l] >> 0) & 3) << 4)) - 32;
                    q[base + 32 + l] = ((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
                    q[base + 64 + l] = ((ql[l] >> 4)       | (((qh[l] >> 4) & 3) << 4)) - 32;
                    q[base + 96 + l] = ((ql[l + 32] >> 4)  | (((qh[l] >> 6) & 3) << 4)) - 32;
                }
            for (int i = 0; i < QK_K; ++i) { sa[i] = d * sc[i / 16]; sb[i] = 0; }
        } break;
        default: break;
    }
}

int orc_dequantize_row(int type, const void *src, float *dst, int64_t n) {
    const int bs = orc_blck_size(type), ts = orc_type_size(type);
    if (type == ORC_F32) { memcpy(dst, src, (size_t)n * 4); return 0; }
    if (bs == 0 || n % bs) return -1;
    const uint8_t *p = (const uint8_t *)src;
    int q[QK_K]; double sa[QK_K], sb[QK_K];
    for (int64_t ib = 0; ib < n / bs; ++ib, p += ts) {
        if (type == ORC_Q8_1) {
            const float d = rdh(p);
            for (int i = 0; i < 32; ++i) dst[ib * 32 + i] = d * (float)(int8_t)p[4 + i];
            continue;
        }
        if (type == ORC_Q8_K) {
            float d; memcpy(&d, p, 4);
            for (int i = 0; i < QK_K; ++i) dst[ib * QK_K + i] = d * (float)(int8_t)p[4 + i];
            continue;
        }
        block_affine(type, p, q, sa, sb);
        /* float evaluation in the same shape as ggml's dequantize_row_* */
        for (int i = 0; i < bs; ++i) {
            const float a = (float)sa[i], o = (float)sb[i];
            dst[ib * bs + i] = a * (float)q[i] - o;
        }
    }
    return 0;
}

/* ------------------------------------------------------------------------ */
/* quantizers                                                                */
/* ------------------------------------------------------------------------ */

/* ggml's nearest_int: round-half-even via the 1.5*2^23 magic constant */
static inline int nearest_int(float fval) {
    const float val = fval + 12582912.f;
    int i;
    memcpy(&i, &val, 4);
    return (i & 0x007fffff) - 0x00400000;
}

static inline int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

/* signed value with the largest magnitude (first occurrence wins) */
static float signed_absmax(const float *x, int n) {
    float amax = 0.0f, max = 0.0f;
    for (int j = 0; j < n; ++j) {
        const float v = x[j];
        if (amax < fabsf(v)) { amax = fabsf(v); max = v; }
    }
    return max;
}

static void quant_q4_0(const float *x, uint8_t *y) {   /* quantize_row_q4_0_ref */
    const float max = signed_absmax(x, 32);
    const float d = max / -8;
    const float id = d ? 1.0f / d : 0.0f;
    wrh(y, d);
    for (int j = 0; j < 16; ++j) {
        const float x0 = x[j] * id, x1 = x[16 + j] * id;
        const uint8_t xi0 = (uint8_t)clampi((int8_t)(x0 + 8.5f), -128, 15);
        const uint8_t xi1 = (uint8_t)clampi((int8_t)(x1 + 8.5f), -128, 15);
        y[2 + j] = (uint8_t)((xi0 & 0xF) | (xi1 << 4));
    }
}

static void quant_q5_0(const float *x, uint8_t *y) {   /* quantize_row_q5_0_ref */
    const float max = signed_absmax(x, 32);
    const float d = max / -16;
    const float id = d ? 1.0f / d : 0.0f;
    wrh(y, d);
    uint32_t qh = 0;
    for (int j = 0; j < 16; ++j) {
        const float x0 = x[j] * id, x1 = x[16 + j] * id;
        const uint8_t xi0 = (uint8_t)clampi((int8_t)(x0 + 16.5f), -128, 31);
        const uint8_t xi1 = (uint8_t)clampi((int8_t)(x1 + 16.5f), -128, 31);
        y[6 + j] = (uint8_t)((xi0 & 0x0F) | ((xi1 & 0x0F) << 4));
        qh |= ((xi0 & 0x10u) >> 4) << (j + 0);
        qh |= ((xi1 & 0x10u) >> 4) << (j + 16);
    }
    memcpy(y + 2, &qh, 4);
}

static void quant_q8_0(const float *x, uint8_t *y) {   /* quantize_row_q8_0_ref */
    float amax = 0.0f;
    for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(x[j]));
    const float d = amax / ((1 << 7) - 1);
    const float id = d ? 1.0f / d : 0.0f;
    wrh(y, d);
    for (int j = 0; j < 32; ++j) {
        const float x0 = x[j] * id;
        y[2 + j] = (uint8_t)(int8_t)roundf(x0);
    }
}

/* Q8_1 exactly as llama.cpp's CUDA quantize_q8_1: d = amax/127,
 * q = round(x/d), s = warp butterfly sum of x over the 32 lanes */
static void quant_q8_1(const float *x, uint8_t *y) {
    float amax = 0.0f;
    float v[32];
    for (int j = 0; j < 32; ++j) { amax = fmaxf(amax, fabsf(x[j])); v[j] = x[j]; }
    for (int off = 16; off >= 1; off >>= 1) {
        float t[32];
        for (int l = 0; l < 32; ++l) t[l] = v[l] + v[l ^ off];
        memcpy(v, t, sizeof(v));
    }
    const float sum = v[0];
    const float d = amax / 127;
    for (int j = 0; j < 32; ++j) {
        const int8_t q = amax == 0.0f ? 0 : (int8_t)roundf(x[j] / d);
        y[4 + j] = (uint8_t)q;
    }
    wrh(y, d);
    wrh(y + 2, sum);
}

static void quant_q8_K(const float *x, uint8_t *y) {   /* quantize_row_q8_K_ref */
    float max = 0, amax = 0;
    for (int j = 0; j < QK_K; ++j) {
        const float ax = fabsf(x[j]);
        if (ax > amax) { amax = ax; max = x[j]; }
    }
    int8_t *qs = (int8_t *)(y + 4);
    if (!amax) {
        const float z = 0.0f;
        memcpy(y, &z, 4);
        memset(y + 4, 0, QK_K + 32);   /* bsums zeroed too (upstream leaves them unset) */
        return;
    }
    const float iscale = -127.f / max;
    for (int j = 0; j < QK_K; ++j) {
        const int v = nearest_int(iscale * x[j]);
        qs[j] = (int8_t)(v < 127 ? v : 127);
    }
    for (int j = 0; j < QK_K / 16; ++j) {
        int sum = 0;
        for (int ii = 0; ii < 16; ++ii) sum += qs[j * 16 + ii];
        const int16_t s16 = (int16_t)sum;
        memcpy(y + 260 + 2 * j, &s16, 2);
    }
    const float d = 1 / iscale;
    memcpy(y, &d, 4);
}

/* ---- this project's min/max K-quant quantizers (format-exact, simple) --- */

/* asymmetric sub-block fit: value = d*sc*q - dmin*m, q in [0, qmax],
 * sc,m in [0, smax]; nsub sub-blocks of length sl */
static void fit_asym(const float *x, int nsub, int sl, int qmax, int smax,
                     float *d_out, float *dmin_out, int *sc, int *mn, int *q) {
    float scale[16], off[16], maxs = 0, maxm = 0;
    for (int s = 0; s < nsub; ++s) {
        float lo = 0.0f, hi = 0.0f;
        for (int l = 0; l < sl; ++l) {
            const float v = x[s * sl + l];
            if (v < lo) lo = v;
            if (v > hi) hi = v;
        }
        scale[s] = (hi - lo) / qmax;
        off[s] = -lo;
        if (scale[s] > maxs) maxs = scale[s];
        if (off[s] > maxm) maxm = off[s];
    }
    const float d = orc_fp16_to_fp32(orc_fp32_to_fp16(maxs / smax));
    const float dmin = orc_fp16_to_fp32(orc_fp32_to_fp16(maxm / smax));
    for (int s = 0; s < nsub; ++s) {
        sc[s] = d > 0 ? clampi(nearest_int(scale[s] / d), 0, smax) : 0;
        mn[s] = dmin > 0 ? clampi(nearest_int(off[s] / dmin), 0, smax) : 0;
        const float dl = d * sc[s], ml = dmin * mn[s];
        for (int l = 0; l < sl; ++l) {
            q[s * sl + l] = dl > 0 ? clampi(nearest_int((x[s * sl + l] + ml) / dl), 0, qmax) : 0;
        }
    }
    *d_out = d;
    *dmin_out = dmin;
}

/* symmetric sub-block fit: value = d*sc*q, q in [-qneg, qneg-1], sc signed
 * in [-smax-1, smax] */
static void fit_sym(const float *x, int nsub, int sl, int qneg, int smax,
                    float *d_out, int *sc, int *q) {
    float scale[16], maxs = 0;
    for (int s = 0; s < nsub; ++s) {
        scale[s] = signed_absmax(x + s * sl, sl) / -qneg;
        if (fabsf(scale[s]) > maxs) maxs = fabsf(scale[s]);
    }
    const float d = orc_fp16_to_fp32(orc_fp32_to_fp16(maxs / smax));
    for (int s = 0; s < nsub; ++s) {
        sc[s] = d > 0 ? clampi(nearest_int(scale[s] / d), -smax - 1, smax) : 0;
        const float dl = d * sc[s];
        for (int l = 0; l < sl; ++l) {
            q[s * sl + l] = dl != 0 ? clampi(nearest_int(x[s * sl + l] / dl), -qneg, qneg - 1) : 0;
        }
    }
    *d_out = d;
}

static void quant_q2_K(const float *x, uint8_t *y) {
    float d, dmin; int sc[16], mn[16], q[QK_K];
    fit_asym(x, 16, 16, 3, 15, &d, &dmin, sc, mn, q);
    memset(y, 0, 84);
    for (int s = 0; s < 16; ++s) y[s] = (uint8_t)(sc[s] | (mn[s] << 4));
    for (int i = 0; i < QK_K; ++i) {
        const int n = i / 128, s = (i % 128) / 32, l = i % 32;
        y[16 + n * 32 + l] |= (uint8_t)(q[i] << (2 * s));
    }
    wrh(y + 80, d);
    wrh(y + 82, dmin);
}

static void quant_q3_K(const float *x, uint8_t *y) {
    float d; int sc[16], q[QK_K];
    fit_sym(x, 16, 16, 4, 31, &d, sc, q);
    memset(y, 0, 110);
    for (int i = 0; i < QK_K; ++i) {
        const int n = i / 128, s = (i % 128) / 32, l = i % 32;
        const int u = q[i] + 4;                       /* 0..7 */
        y[32 + n * 32 + l] |= (uint8_t)((u & 3) << (2 * s));
        if (u & 4) y[l] |= (uint8_t)(1u << (n * 4 + s));
    }
    for (int k = 0; k < 16; ++k) {
        const int v = sc[k] + 32;                     /* 0..63 */
        if (k < 8) y[96 + k] |= (uint8_t)(v & 0xF);
        else       y[96 + k - 8] |= (uint8_t)((v & 0xF) << 4);
        y[96 + 8 + (k % 4)] |= (uint8_t)((v >> 4) << (2 * (k / 4)));
    }
    wrh(y + 108, d);
}

static void pack_k4_scales(const int *sc, const int *mn, uint8_t *q) {
    memset(q, 0, 12);
    for (int j = 0; j < 4; ++j) {
        q[j]     = (uint8_t)(sc[j] | ((sc[j + 4] >> 4) << 6));
        q[j + 4] = (uint8_t)(mn[j] | ((mn[j + 4] >> 4) << 6));
        q[j + 8] = (uint8_t)((sc[j + 4] & 0xF) | ((mn[j + 4] & 0xF) << 4));
    }
}

static void quant_q45_K(const float *x, uint8_t *y, int five) {
    float d, dmin; int sc[8], mn[8], q[QK_K];
    fit_asym(x, 8, 32, five ? 31 : 15, 63, &d, &dmin, sc, mn, q);
    memset(y, 0, five ? 176 : 144);
    wrh(y, d);
    wrh(y + 2, dmin);
    pack_k4_scales(sc, mn, y + 4);
    uint8_t *qs = y + (five ? 48 : 16);
    for (int c = 0; c < 4; ++c)
        for (int l = 0; l < 32; ++l) {
            const int lo = q[64 * c + l], hi = q[64 * c + 32 + l];
            qs[32 * c + l] = (uint8_t)((lo & 0xF) | ((hi & 0xF) << 4));
            if (five) {
                y[16 + l] |= (uint8_t)(((lo >> 4) & 1) << (2 * c));
                y[16 + l] |= (uint8_t)(((hi >> 4) & 1) << (2 * c + 1));
            }
        }
}

static void quant_q6_K(const float *x, uint8_t *y) {
    float d; int sc[16], q[QK_K];
    fit_sym(x, 16, 16, 32, 127, &d, sc, q);
    memset(y, 0, 210);
    for (int n = 0; n < 2; ++n)
        for (int l = 0; l < 32; ++l) {
            const int b = 128 * n;
            const int q1 = q[b + l] + 32, q2 = q[b + 32 + l] + 32;
            const int q3 = q[b + 64 + l] + 32, q4 = q[b + 96 + l] + 32;
            y[64 * n + l]      = (uint8_t)((q1 & 0xF) | ((q3 & 0xF) << 4));
            y[64 * n + 32 + l] = (uint8_t)((q2 & 0xF) | ((q4 & 0xF) << 4));
            y[128 + 32 * n + l] = (uint8_t)((q1 >> 4) | ((q2 >> 4) << 2) | ((q3 >> 4) << 4) | ((q4 >> 4) << 6));
        }
    for (int s = 0; s < 16; ++s) y[192 + s] = (uint8_t)(int8_t)sc[s];
    wrh(y + 208, d);
}

int orc_quantize_row(int type, const float *src, void *dst, int64_t n) {
    const int bs = orc_blck_size(type), ts = orc_type_size(type);
    if (bs == 0 || n % bs) return -1;
    uint8_t *y = (uint8_t *)dst;
    for (int64_t ib = 0; ib < n / bs; ++ib, y += ts) {
        const float *x = src + ib * bs;
        switch (type) {
            case ORC_Q4_0: quant_q4_0(x, y); break;
            case ORC_Q5_0: quant_q5_0(x, y); break;
            case ORC_Q8_0: quant_q8_0(x, y); break;
            case ORC_Q2_K: quant_q2_K(x, y); break;
            case ORC_Q3_K: quant_q3_K(x, y); break;
            case ORC_Q4_K: quant_q45_K(x, y, 0); break;
            case ORC_Q5_K: quant_q45_K(x, y, 1); break;
            case ORC_Q6_K: quant_q6_K(x, y); break;
            default: return -1;
        }
    }
    return 0;
}

int orc_quantize_act(int act_type, const float *src, void *dst, int64_t n) {
    const int bs = orc_blck_size(act_type), ts = orc_type_size(act_type);
    if (bs == 0 || n % bs) return -1;
    uint8_t *y = (uint8_t *)dst;
    for (int64_t ib = 0; ib < n / bs; ++ib, y += ts) {
        const float *x = src + ib * bs;
        switch (act_type) {
            case ORC_Q8_0: quant_q8_0(x, y); break;
            case ORC_Q8_1: quant_q8_1(x, y); break;
            case ORC_Q8_K: quant_q8_K(x, y); break;
            default: return -1;
        }
    }
    return 0;
}

/* ------------------------------------------------------------------------ */
/* vec_dot: llama.cpp generic CPU arithmetic                                 */
/* ------------------------------------------------------------------------ */

static float dot_legacy_q8_0(int type, int64_t n, const uint8_t *x, const uint8_t *y) {
    const int ts = orc_type_size(type);
    float sumf = 0;
    for (int64_t ib = 0; ib < n / 32; ++ib, x += ts, y += 34) {
        const int8_t *yq = (const int8_t *)(y + 2);
        int sumi = 0;
        if (type == ORC_Q4_0) {
            int s0 = 0, s1 = 0;
            for (int j = 0; j < 16; ++j) {
                s0 += ((x[2 + j] & 0x0F) - 8) * yq[j];
                s1 += ((x[2 + j] >> 4) - 8) * yq[j + 16];
            }
            sumi = s0 + s1;
            sumf += sumi * rdh(x) * rdh(y);
        } else if (type == ORC_Q5_0) {
            uint32_t qh; memcpy(&qh, x + 2, 4);
            int s0 = 0, s1 = 0;
            for (int j = 0; j < 16; ++j) {
                const uint8_t xh0 = (uint8_t)(((qh & (1u << j)) >> j) << 4);
                const uint8_t xh1 = (uint8_t)((qh & (1u << (j + 16))) >> (j + 12));
                const int32_t x0 = (int8_t)(((x[6 + j] & 0x0F) | xh0) - 16);
                const int32_t x1 = (int8_t)(((x[6 + j] >> 4) | xh1) - 16);
                s0 += x0 * yq[j];
                s1 += x1 * yq[j + 16];
            }
            sumi = s0 + s1;
            sumf += (rdh(x) * rdh(y)) * sumi;
        } else { /* Q8_0 */
            for (int j = 0; j < 32; ++j) sumi += (int8_t)x[2 + j] * yq[j];
            sumf += sumi * (rdh(x) * rdh(y));
        }
    }
    return sumf;
}

static inline float q8k_d(const uint8_t *y) { float d; memcpy(&d, y, 4); return d; }
static inline int16_t q8k_bsum(const uint8_t *y, int j) { int16_t v; memcpy(&v, y + 260 + 2 * j, 2); return v; }

static float dot_q2_K_q8_K(int64_t n, const uint8_t *x, const uint8_t *y) {
    float sumf = 0;
    for (int64_t i = 0; i < n / QK_K; ++i, x += 84, y += 292) {
        const uint8_t *q2 = x + 16, *sc = x;
        const int8_t *q8 = (const int8_t *)(y + 4);
        int summs = 0;
        for (int j = 0; j < 16; ++j) summs += q8k_bsum(y, j) * (sc[j] >> 4);
        const float dall = q8k_d(y) * rdh(x + 80);
        const float dmin = q8k_d(y) * rdh(x + 82);
        int isum = 0, is = 0;
        for (int k = 0; k < QK_K / 128; ++k) {
            int shift = 0;
            for (int j = 0; j < 4; ++j) {
                int d = sc[is++] & 0xF, isuml = 0;
                for (int l = 0; l < 16; ++l) isuml += q8[l] * ((q2[l] >> shift) & 3);
                isum += d * isuml;
                d = sc[is++] & 0xF; isuml = 0;
                for (int l = 16; l < 32; ++l) isuml += q8[l] * ((q2[l] >> shift) & 3);
                isum += d * isuml;
                shift += 2;
                q8 += 32;
            }
            q2 += 32;
        }
        sumf += dall * isum - dmin * summs;
    }
    return sumf;
}

/* shared tail of the Q3_K/Q4_K/Q5_K/Q6_K generic kernels: 8-lane int32
 * accumulators over 8-element groups, scaled per block into float sums[8] */
static float dot_aux8(int type, int64_t n, const uint8_t *x, const uint8_t *y) {
    const int ts = orc_type_size(type);
    float sums[8] = {0};
    float sumf = 0;
    int8_t aux8[QK_K];
    for (int64_t i = 0; i < n / QK_K; ++i, x += ts, y += 292) {
        int q[QK_K]; double sa[QK_K], sb[QK_K];
        block_affine(type, x, q, sa, sb);
        for (int e = 0; e < QK_K; ++e) aux8[e] = (int8_t)q[e];
        const int8_t *q8 = (const int8_t *)(y + 4);
        int32_t aux32[8] = {0};
        const int8_t *a = aux8;
        float d;
        if (type == ORC_Q3_K || type == ORC_Q6_K) {
            int scales[16];
            if (type == ORC_Q3_K) q3k_scales(x + 96, scales);
            else for (int s = 0; s < 16; ++s) scales[s] = ((const int8_t *)(x + 192))[s];
            for (int j = 0; j < QK_K / 16; ++j) {
                for (int h = 0; h < 2; ++h) {
                    for (int l = 0; l < 8; ++l) aux32[l] += scales[j] * (int16_t)(q8[l] * a[l]);
                    q8 += 8; a += 8;
                }
            }
            d = rdh(x + (type == ORC_Q3_K ? 108 : 208)) * q8k_d(y);
        } else {
            int sc[8], mn[8];
            for (int j = 0; j < 8; ++j) k4_scale_min(j, x + 4, &sc[j], &mn[j]);
            int sumi = 0;
            for (int j = 0; j < QK_K / 16; ++j) sumi += q8k_bsum(y, j) * mn[j / 2];
            /* block_affine returns unsigned codes for Q4_K/Q5_K already */
            for (int j = 0; j < QK_K / 32; ++j) {
                for (int h = 0; h < 4; ++h) {
                    for (int l = 0; l < 8; ++l) aux32[l] += sc[j] * (int16_t)(q8[l] * a[l]);
                    q8 += 8; a += 8;
                }
            }
            d = rdh(x) * q8k_d(y);
            const float dmin = rdh(x + 2) * q8k_d(y);
            sumf -= dmin * sumi;
        }
        for (int l = 0; l < 8; ++l) sums[l] += d * aux32[l];
    }
    for (int l = 0; l < 8; ++l) sumf += sums[l];
    return sumf;
}

/* exact value of sum(w*a) in double, any activation format */
static double act_value(int act_type, const uint8_t *a, int64_t i) {
    switch (act_type) {
        case ORC_Q8_0: { const uint8_t *b = a + (i / 32) * 34; return (double)rdh(b) * (int8_t)b[2 + i % 32]; }
        case ORC_Q8_1: { const uint8_t *b = a + (i / 32) * 36; return (double)rdh(b) * (int8_t)b[4 + i % 32]; }
        case ORC_Q8_K: { const uint8_t *b = a + (i / QK_K) * 292; return (double)q8k_d(b) * (int8_t)b[4 + i % QK_K]; }
        default: return 0;
    }
}

/* Value of a row dot in double. With Q8_1 activations this is what
 * llama.cpp's CUDA vec_dot_*_q8_1 computes (the functions the reference
 * kernel dispatches to, kernels/moe-cache.cu:46-47 for Q4_0 / Q5_0): the
 * integer dots are exact, and for Q4_0 / Q5_0 the weights' offset (8 or 16)
 * is taken off with the Q8_1 block's stored sum s -- the f16-rounded sum of
 * the UNquantized inputs that quantize_q8_1 writes -- as
 * d_w * (d_a * sum(q_w * q_a) - offset * s), not with the quantized inputs.
 * Every other pairing: sum(w * a) over the dequantized values. */
static double dot_exact(int type, int act_type, int64_t n, const uint8_t *x, const uint8_t *a) {
    const int bs = orc_blck_size(type), ts = orc_type_size(type);
    double s = 0;
    int q[QK_K]; double sa[QK_K], sb[QK_K];
    if (act_type == ORC_Q8_1 && (type == ORC_Q4_0 || type == ORC_Q5_0)) {
        const int off = type == ORC_Q4_0 ? 8 : 16;
        for (int64_t ib = 0; ib < n / 32; ++ib, x += ts) {
            block_affine(type, x, q, sa, sb);
            const uint8_t *ab = a + ib * 36;
            const double d_a = rdh(ab), s_a = rdh(ab + 2);
            int64_t sumi = 0;
            for (int i = 0; i < 32; ++i) sumi += (int64_t)(q[i] + off) * (int8_t)ab[4 + i];
            s += sa[0] * (d_a * (double)sumi - off * s_a);
        }
        return s;
    }
    for (int64_t ib = 0; ib < n / bs; ++ib, x += ts) {
        block_affine(type, x, q, sa, sb);
        for (int i = 0; i < bs; ++i) {
            const double w = sa[i] * q[i] - sb[i];
            s += w * act_value(act_type, a, ib * bs + i);
        }
    }
    return s;
}

int orc_vec_dot(int type, int act_type, int exact, int64_t n, const void *w, const void *a, float *out) {
    if (orc_blck_size(type) == 0 || n % orc_blck_size(type) || n % orc_blck_size(act_type)) return -1;
    const uint8_t *x = (const uint8_t *)w, *y = (const uint8_t *)a;
    if (exact) {
        if (act_type != ORC_Q8_0 && act_type != ORC_Q8_1 && act_type != ORC_Q8_K) return -1;
        *out = (float)dot_exact(type, act_type, n, x, y);
        return 0;
    }
    if (act_type != orc_vec_dot_type(type)) return -1;
    switch (type) {
        case ORC_Q4_0: case ORC_Q5_0: case ORC_Q8_0: *out = dot_legacy_q8_0(type, n, x, y); return 0;
        case ORC_Q2_K: *out = dot_q2_K_q8_K(n, x, y); return 0;
        case ORC_Q3_K: case ORC_Q4_K: case ORC_Q5_K: case ORC_Q6_K: *out = dot_aux8(type, n, x, y); return 0;
        default: return -1;
    }
}

/* ------------------------------------------------------------------------ */
/* MUL_MAT_ID                                                                */
/* ------------------------------------------------------------------------ */

typedef struct { int32_t i1, i2; } row_map;   /* (pick, token), ggml-cpu.c:1486 */

typedef struct {
    int type, act_type, exact;
    const void *const *experts;
    int64_t K, rows, ne11, n_used;
    size_t row_bytes, act_row;
    const uint8_t *wq;           /* quantized src1 [n_tok][ne11] rows of act_row */
    const int64_t *counts;       /* [E] */
    const row_map *rows_of;      /* [E][n_tok*n_used] */
    int64_t stride_map;
    float *dst;
    /* work items: (expert, row chunk) */
    const int64_t *item_e, *item_r0, *item_r1;
    int64_t n_items;
    int nth;
    int ith;
    int err;
} mmid_ctx;

static void *mmid_worker(void *arg) {
    mmid_ctx *c = (mmid_ctx *)arg;
    for (int64_t it = c->ith; it < c->n_items; it += c->nth) {
        const int64_t e = c->item_e[it];
        const uint8_t *src0 = (const uint8_t *)c->experts[e];
        for (int64_t m = 0; m < c->counts[e]; ++m) {
            const row_map rm = c->rows_of[e * c->stride_map + m];
            const int64_t i11 = rm.i1 % c->ne11, i12 = rm.i2;
            const uint8_t *col = c->wq + (i11 + i12 * c->ne11) * c->act_row;
            float *dcol = c->dst + (i12 * c->n_used + rm.i1) * c->rows;
            for (int64_t r = c->item_r0[it]; r < c->item_r1[it]; ++r) {
                if (orc_vec_dot(c->type, c->act_type, c->exact, c->K, src0 + r * c->row_bytes, col, &dcol[r]))
                    c->err = 1;
            }
        }
    }
    return NULL;
}

static int mmid_run(int type, int act_type, int exact, const void *const *experts, int64_t n_experts,
                    int64_t K, int64_t rows, size_t row_bytes, const uint8_t *wq, size_t act_row,
                    int64_t ne11, int64_t n_tok, const int32_t *ids, int64_t n_used,
                    float *dst, int n_threads) {
    /* group rows by expert (ggml-cpu.c:1677-1692) */
    const int64_t stride_map = n_tok * n_used;
    int64_t *counts = (int64_t *)calloc((size_t)n_experts, sizeof(int64_t));
    row_map *rows_of = (row_map *)malloc((size_t)(n_experts * stride_map) * sizeof(row_map) + 1);
    if (!counts || !rows_of) { free(counts); free(rows_of); return -2; }
    for (int64_t t = 0; t < n_tok; ++t)
        for (int64_t p = 0; p < n_used; ++p) {
            const int32_t e = ids[t * n_used + p];
            if (e < 0 || e >= n_experts) { free(counts); free(rows_of); return -3; }
            rows_of[e * stride_map + counts[e]] = (row_map){(int32_t)p, (int32_t)t};
            counts[e]++;
        }
    /* row chunks per expert (64-row chunks for the GEMV-shaped case) */
    const int64_t chunk = 64;
    int64_t n_items = 0;
    for (int64_t e = 0; e < n_experts; ++e) if (counts[e]) n_items += (rows + chunk - 1) / chunk;
    int64_t *ie = (int64_t *)malloc((size_t)(3 * n_items + 3) * sizeof(int64_t));
    int64_t *r0 = ie + n_items + 1, *r1 = r0 + n_items + 1;
    int64_t k = 0;
    for (int64_t e = 0; e < n_experts; ++e) {
        if (!counts[e]) continue;
        for (int64_t r = 0; r < rows; r += chunk) {
            ie[k] = e; r0[k] = r; r1[k] = r + chunk < rows ? r + chunk : rows; k++;
        }
    }
    if (n_threads < 1) n_threads = 1;
    if (n_threads > 256) n_threads = 256;
    mmid_ctx ctx[256];
    pthread_t th[256];
    int err = 0;
    for (int t = 0; t < n_threads; ++t) {
        ctx[t] = (mmid_ctx){type, act_type, exact, experts, K, rows, ne11, n_used, row_bytes, act_row,
                            wq, counts, rows_of, stride_map, dst, ie, r0, r1, n_items, n_threads, t, 0};
    }
    for (int t = 1; t < n_threads; ++t) pthread_create(&th[t], NULL, mmid_worker, &ctx[t]);
    mmid_worker(&ctx[0]);
    for (int t = 1; t < n_threads; ++t) pthread_join(th[t], NULL);
    for (int t = 0; t < n_threads; ++t) err |= ctx[t].err;
    free(ie); free(counts); free(rows_of);
    return err ? -4 : 0;
}

int orc_mul_mat_id(int type, int act_type, int exact, const void *const *experts, int64_t n_experts,
                   int64_t K, int64_t rows, size_t row_bytes, const float *src1, int64_t ne11,
                   int64_t n_tok, const int32_t *ids, int64_t n_used, float *dst, int n_threads) {
    const size_t act_row = orc_row_size(act_type, K);
    if (!act_row || !orc_row_size(type, K)) return -1;
    uint8_t *wq = (uint8_t *)malloc(act_row * (size_t)(n_tok * ne11) + 1);
    if (!wq) return -2;
    for (int64_t r = 0; r < n_tok * ne11; ++r) orc_quantize_act(act_type, src1 + r * K, wq + r * act_row, K);
    const int rc = mmid_run(type, act_type, exact, experts, n_experts, K, rows, row_bytes, wq, act_row,
                            ne11, n_tok, ids, n_used, dst, n_threads);
    free(wq);
    return rc;
}

int orc_mul_mat_id_q8_1(int type, const void *const *experts, int64_t n_experts, int64_t K, int64_t rows,
                        size_t row_bytes, const void *src1_q8_1, int64_t ne11, int64_t n_tok,
                        const int32_t *ids, int64_t n_used, float *dst, int n_threads) {
    const size_t act_row = orc_row_size(ORC_Q8_1, K);
    if (!act_row || !orc_row_size(type, K)) return -1;
    return mmid_run(type, ORC_Q8_1, 1, experts, n_experts, K, rows, row_bytes,
                    (const uint8_t *)src1_q8_1, act_row, ne11, n_tok, ids, n_used, dst, n_threads);
}

/* ------------------------------------------------------------------------ */
/* GLU, routing, layer                                                       */
/* ------------------------------------------------------------------------ */

static float silu(float x) { return x / (1.0f + expf(-x)); }

/* GLU epilogue of the reference kernel (kernels/moe-cache.cu:264-280):
 * result = up, gate_value = gate */
float orc_glu(int op, float gate, float up, float limit) {
    switch (op) {
        case ORC_GLU_SWIGLU: return up * silu(gate);
        case ORC_GLU_GEGLU: {
            const float c = 0.79788456080286535587989211986876f, a = 0.044715f;
            return up * (0.5f * gate * (1.0f + tanhf(c * gate * (1.0f + a * gate * gate))));
        }
        case ORC_GLU_SWIGLU_OAI: {
            const float alpha = 1.702f, lim = 7.0f;
            const float x = fminf(gate, lim);
            const float g = fmaxf(fminf(up, lim), -lim);
            return (x / (1.0f + expf(-x * alpha))) * (g + 1.0f);
        }
        case ORC_GLU_SWIGLU_CLAMP: {
            const float x = fminf(gate, limit);
            const float g = fmaxf(fminf(up, limit), -limit);
            return silu(x) * g;
        }
        default: return up * gate;
    }
}

int orc_topk_softmax(const float *logits, int64_t n_tok, int64_t n_experts, int64_t k, int norm_w,
                     int32_t *ids, float *weights) {
    if (k > n_experts || k < 1) return -1;
    for (int64_t t = 0; t < n_tok; ++t) {
        const float *l = logits + t * n_experts;
        int32_t *sel = ids + t * k;
        for (int64_t j = 0; j < k; ++j) {
            int32_t best = -1;
            for (int64_t e = 0; e < n_experts; ++e) {
                int taken = 0;
                for (int64_t q = 0; q < j; ++q) if (sel[q] == e) { taken = 1; break; }
                if (taken) continue;
                if (best < 0 || l[e] > l[best]) best = (int32_t)e;
            }
            sel[j] = best;
        }
        float mx = l[0];
        for (int64_t e = 1; e < n_experts; ++e) mx = fmaxf(mx, l[e]);
        double sum = 0;
        for (int64_t e = 0; e < n_experts; ++e) sum += expf(l[e] - mx);
        double wsum = 0;
        for (int64_t j = 0; j < k; ++j) {
            weights[t * k + j] = (float)(expf(l[sel[j]] - mx) / sum);
            wsum += weights[t * k + j];
        }
        if (norm_w)
            for (int64_t j = 0; j < k; ++j) weights[t * k + j] = (float)(weights[t * k + j] / wsum);
    }
    return 0;
}

int orc_moe_layer(const orc_layer *L, const float *x, const float *logits, int64_t n_tok, int act_mode,
                  int exact, float *out, int32_t *ids_out, float *w_out, int n_threads) {
    const int64_t H = L->H, F = L->F, k = L->k;
    int rc = orc_topk_softmax(logits, n_tok, L->n_experts, k, L->norm_w, ids_out, w_out);
    if (rc) return rc;
    float *g = (float *)malloc(sizeof(float) * (size_t)(n_tok * k * F));
    float *u = (float *)malloc(sizeof(float) * (size_t)(n_tok * k * F));
    float *d = (float *)malloc(sizeof(float) * (size_t)(n_tok * k * H));
    float *sh = (float *)malloc(sizeof(float) * (size_t)(n_tok * (F * 3 + H)));
    if (!g || !u || !d || !sh) { rc = -2; goto done; }
#define ACT(t) (act_mode == 1 ? ORC_Q8_1 : orc_vec_dot_type(t))
#define EX(t) (act_mode == 1 ? 1 : exact)
    rc = orc_mul_mat_id(L->type_gate, ACT(L->type_gate), EX(L->type_gate), L->gate, L->n_experts, H, F,
                        orc_row_size(L->type_gate, H), x, 1, n_tok, ids_out, k, g, n_threads);
    if (!rc) rc = orc_mul_mat_id(L->type_up, ACT(L->type_up), EX(L->type_up), L->up, L->n_experts, H, F,
                                 orc_row_size(L->type_up, H), x, 1, n_tok, ids_out, k, u, n_threads);
    if (rc) goto done;
    for (int64_t i = 0; i < n_tok * k * F; ++i) g[i] = orc_glu(L->glu_op, g[i], u[i], L->glu_limit);
    rc = orc_mul_mat_id(L->type_down, ACT(L->type_down), EX(L->type_down), L->down, L->n_experts, F, H,
                        orc_row_size(L->type_down, F), g, k, n_tok, ids_out, k, d, n_threads);
    if (rc) goto done;
    for (int64_t t = 0; t < n_tok; ++t)
        for (int64_t r = 0; r < H; ++r) {
            float acc = 0.0f;
            for (int64_t p = 0; p < k; ++p) {
                const float v = d[(t * k + p) * H + r] * w_out[t * k + p];
                acc = p == 0 ? v : acc + v;
            }
            out[t * H + r] = acc;
        }
    if (L->shared_type >= 0) {
        /* the shared expert's gate/up/down have the routed gate/up/down types */
        const int tg = L->type_gate, tu = L->type_up, td = L->type_down;
        const void *sg[1] = {L->shared_gate}, *su[1] = {L->shared_up}, *sd[1] = {L->shared_down};
        int32_t *zid = (int32_t *)calloc((size_t)n_tok, sizeof(int32_t));
        float *sgo = sh, *suo = sh + n_tok * F, *sdo = sh + 2 * n_tok * F;
        rc = orc_mul_mat_id(tg, ACT(tg), EX(tg), sg, 1, H, F, orc_row_size(tg, H), x, 1, n_tok, zid, 1, sgo, n_threads);
        if (!rc) rc = orc_mul_mat_id(tu, ACT(tu), EX(tu), su, 1, H, F, orc_row_size(tu, H), x, 1, n_tok, zid, 1, suo, n_threads);
        if (!rc) {
            for (int64_t i = 0; i < n_tok * F; ++i) sgo[i] = orc_glu(L->glu_op, sgo[i], suo[i], L->glu_limit);
            rc = orc_mul_mat_id(td, ACT(td), EX(td), sd, 1, F, H, orc_row_size(td, F), sgo, 1, n_tok, zid, 1, sdo, n_threads);
        }
        if (!rc)
            for (int64_t i = 0; i < n_tok * H; ++i) out[i] += sdo[i];
        free(zid);
    }
#undef ACT
#undef EX
done:
    free(g); free(u); free(d); free(sh);
    return rc;
}

/* ------------------------------------------------------------------------ */
/* synthetic weights (same counter-hash recipe as the device generator)      */
/* ------------------------------------------------------------------------ */
static inline uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

static inline float normal_at(uint64_t seed, uint64_t i) {
    const uint64_t h = mix64(seed ^ mix64(i));
    const float u1 = ((float)(h >> 40) + 0.5f) * (1.0f / 16777216.0f);
    const float u2 = (float)((h >> 16) & 0xFFFFFF) * (1.0f / 16777216.0f);
    return sqrtf(-2.0f * logf(u1)) * cosf(6.283185307179586f * u2);
}

typedef struct {
    int type; uint8_t *dst; int64_t row0, n_rows, n_cols; uint64_t seed; float sigma; int ith, nth;
} fill_ctx;

static void *fill_worker(void *arg) {
    fill_ctx *c = (fill_ctx *)arg;
    const size_t rs = orc_row_size(c->type, c->n_cols);
    float *x = (float *)malloc(sizeof(float) * (size_t)c->n_cols);
    for (int64_t r = c->ith; r < c->n_rows; r += c->nth) {
        const uint64_t base = (uint64_t)(c->row0 + r) * (uint64_t)c->n_cols;
        for (int64_t j = 0; j < c->n_cols; ++j) x[j] = c->sigma * normal_at(c->seed, base + (uint64_t)j);
        orc_quantize_row(c->type, x, c->dst + (size_t)r * rs, c->n_cols);
    }
    free(x);
    return NULL;
}

int orc_fill_quantized(int type, void *dst, int64_t row0, int64_t n_rows, int64_t n_cols, uint64_t seed,
                       float sigma, int n_threads) {
    if (!orc_row_size(type, n_cols)) return -1;
    if (n_threads < 1) n_threads = 1;
    if (n_threads > 256) n_threads = 256;
    fill_ctx ctx[256];
    pthread_t th[256];
    for (int t = 0; t < n_threads; ++t)
        ctx[t] = (fill_ctx){type, (uint8_t *)dst, row0, n_rows, n_cols, seed, sigma, t, n_threads};
    for (int t = 1; t < n_threads; ++t) pthread_create(&th[t], NULL, fill_worker, &ctx[t]);
    fill_worker(&ctx[0]);
    for (int t = 1; t < n_threads; ++t) pthread_join(th[t], NULL);
    return 0;
}
