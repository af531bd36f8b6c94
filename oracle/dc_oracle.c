/*
 * dc_oracle.c -- CPU restatement of the quantized matmul / decode attention arithmetic that
 * DenseCore reaches through ggml.  TEST INFRASTRUCTURE ONLY (the checker; never the product).
 * Interface and citations: dc_oracle.h.  Compile with -ffp-contract=off so no product/sum pair
 * is fused behind our back (the rounding steps below are part of the format definition).
 */
#include "dc_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ---------------- block layouts (GGUF / ggml, sizes = gguf.GGML_QUANT_SIZES) ---------------- */
#define QK8_0 32
#define QK_K 256
typedef struct { uint16_t d; int8_t qs[QK8_0]; } blk_q8_0;                       /* 34 B  */
typedef struct { uint16_t d, dmin; uint8_t scales[12]; uint8_t qs[QK_K / 2]; } blk_q4_K; /* 144 */
typedef struct { uint8_t ql[QK_K / 2]; uint8_t qh[QK_K / 4]; int8_t scales[QK_K / 16]; uint16_t d; } blk_q6_K; /* 210 */
typedef struct { float d; int8_t qs[QK_K]; int16_t bsums[QK_K / 16]; } blk_q8_K; /* 292 B */

_Static_assert(sizeof(blk_q8_0) == 34, "q8_0");
_Static_assert(sizeof(blk_q4_K) == 144, "q4_K");
_Static_assert(sizeof(blk_q6_K) == 210, "q6_K");
_Static_assert(sizeof(blk_q8_K) == 292, "q8_K");

/* ---------------- fp16 (IEEE binary16, round to nearest even) ---------------- */
uint16_t dco_fp32_to_fp16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) /* inf / nan */
        return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
    if (ax >= 0x477ff000u) /* rounds to >= 65520 -> inf */
        return (uint16_t)(sign | 0x7c00u);
    if (ax < 0x38800000u) { /* result is subnormal (or zero) in fp16 */
        /* value = ax_float; fp16 subnormal unit = 2^-24 */
        float a;
        memcpy(&a, &ax, 4);
        float scaled = a * 16777216.0f; /* exact: multiply by 2^24 */
        uint32_t q = (uint32_t)rintf(scaled);
        return (uint16_t)(sign | q);
    }
    uint32_t mant = ax & 0x7fffffu;
    int32_t exp = (int32_t)(ax >> 23) - 127 + 15;
    uint32_t h = ((uint32_t)exp << 10) | (mant >> 13);
    uint32_t rem = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1u;
    return (uint16_t)(sign | h);
}

float dco_fp16_to_fp32(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
    float out;
    if (e == 0) {
        out = ldexpf((float)m, -24);
        uint32_t b;
        memcpy(&b, &out, 4);
        b |= sign;
        memcpy(&out, &b, 4);
        return out;
    }
    uint32_t b = sign | (e == 31 ? (0xffu << 23) | (m << 13) : ((e - 15 + 127) << 23) | (m << 13));
    memcpy(&out, &b, 4);
    return out;
}

size_t dco_row_size(int type, int64_t k) {
    switch (type) {
        case DCO_Q8_0: return (size_t)(k / QK8_0) * sizeof(blk_q8_0);
        case DCO_Q4_K: return (size_t)(k / QK_K) * sizeof(blk_q4_K);
        case DCO_Q6_K: return (size_t)(k / QK_K) * sizeof(blk_q6_K);
        case DCO_Q8_K: return (size_t)(k / QK_K) * sizeof(blk_q8_K);
        case DCO_F16: return (size_t)k * 2;
        case DCO_F32: return (size_t)k * 4;
    }
    return 0;
}

/* ---------------- activation quantizers ---------------- */

/* Q8_0 (ggml quantize_row_q8_0 reference form): d = amax/127 stored fp16, id = 1/d,
 * q = roundf(x*id) (round half away from zero).  Called per activation row at
 * core/src/inference.cpp:889-892. */
void dco_quantize_row_q8_0(const float* x, void* vy, int64_t k) {
    blk_q8_0* y = (blk_q8_0*)vy;
    for (int64_t i = 0; i < k / QK8_0; i++) {
        const float* xb = x + i * QK8_0;
        float amax = 0.0f;
        for (int j = 0; j < QK8_0; j++) {
            float a = fabsf(xb[j]);
            if (a > amax) amax = a;
        }
        const float d = amax / 127.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        y[i].d = dco_fp32_to_fp16(d);
        for (int j = 0; j < QK8_0; j++) {
            const float v = xb[j] * id;
            y[i].qs[j] = (int8_t)roundf(v);
        }
    }
}

/* Q8_K (ggml quantize_row_q8_K reference form): per 256, `max` = the first element of largest
 * magnitude (sign kept); iscale = -127/max; q = min(127, nearest_even(iscale*x)); d = 1/iscale
 * stored f32; bsums = sums of each 16 q.  vec_dot_type of Q4_K/Q6_K (inference.cpp:970-983). */
void dco_quantize_row_q8_K(const float* x, void* vy, int64_t k) {
    blk_q8_K* y = (blk_q8_K*)vy;
    for (int64_t i = 0; i < k / QK_K; i++) {
        const float* xb = x + i * QK_K;
        float amax = 0.0f, max = 0.0f;
        for (int j = 0; j < QK_K; j++) {
            float a = fabsf(xb[j]);
            if (a > amax) { amax = a; max = xb[j]; }
        }
        if (amax == 0.0f) {
            memset(&y[i], 0, sizeof(blk_q8_K));
            continue;
        }
        const float iscale = -127.0f / max;
        for (int j = 0; j < QK_K; j++) {
            const float v = iscale * xb[j];
            int q = (int)rintf(v);
            y[i].qs[j] = (int8_t)(q < 127 ? q : 127);
        }
        for (int j = 0; j < QK_K / 16; j++) {
            int s = 0;
            for (int l = 0; l < 16; l++) s += y[i].qs[j * 16 + l];
            y[i].bsums[j] = (int16_t)s;
        }
        y[i].d = 1.0f / iscale;
    }
}

/* ---------------- weight quantizers (offline step; any valid encoding is acceptable) ----------
 * DenseCore's weights arrive pre-quantized from GGUF files (quantize.cpp, out of the hot path).
 * These simple min/max encoders produce valid Q4_K / Q6_K bytes for seeded synthetic weights;
 * the GPU weight encoder in the product follows the same arithmetic so tests can compare bytes. */

static void pack_q4_K_scales(uint8_t* q, const uint8_t* ls, const uint8_t* lm) {
    /* 12-byte packing of eight 6-bit scales and eight 6-bit mins (ggml get_scale_min_k4 inverse) */
    for (int j = 0; j < 8; j++) {
        if (j < 4) {
            q[j] = ls[j];
            q[j + 4] = lm[j];
        } else {
            q[j + 4] = (uint8_t)((ls[j] & 0xF) | ((lm[j] & 0xF) << 4));
            q[j - 4] |= (uint8_t)((ls[j] >> 4) << 6);
            q[j] |= (uint8_t)((lm[j] >> 4) << 6);
        }
    }
}

static void unpack_q4_K_scale(const uint8_t* q, int j, int* sc, int* m) {
    if (j < 4) {
        *sc = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
        *m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

static int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

void dco_quantize_row_q4_K(const float* x, void* vy, int64_t k) {
    blk_q4_K* y = (blk_q4_K*)vy;
    for (int64_t i = 0; i < k / QK_K; i++) {
        const float* xb = x + i * QK_K;
        float scale[8], mn[8], max_scale = 0.0f, max_min = 0.0f;
        for (int j = 0; j < 8; j++) {
            float lo = 0.0f, hi = 0.0f;
            for (int l = 0; l < 32; l++) {
                float v = xb[j * 32 + l];
                if (v < lo) lo = v;
                if (v > hi) hi = v;
            }
            scale[j] = (hi - lo) / 15.0f;
            mn[j] = lo < 0.0f ? -lo : 0.0f; /* +0, never -0 */
            if (scale[j] > max_scale) max_scale = scale[j];
            if (mn[j] > max_min) max_min = mn[j];
        }
        const float inv_s = max_scale > 0.0f ? 63.0f / max_scale : 0.0f;
        const float inv_m = max_min > 0.0f ? 63.0f / max_min : 0.0f;
        uint8_t ls[8], lm[8];
        for (int j = 0; j < 8; j++) {
            float a = inv_s * scale[j], b = inv_m * mn[j];
            ls[j] = (uint8_t)clampi((int)roundf(a), 0, 63);
            lm[j] = (uint8_t)clampi((int)roundf(b), 0, 63);
        }
        memset(y[i].scales, 0, 12);
        pack_q4_K_scales(y[i].scales, ls, lm);
        y[i].d = dco_fp32_to_fp16(max_scale / 63.0f);
        y[i].dmin = dco_fp32_to_fp16(max_min / 63.0f);
        const float d = dco_fp16_to_fp32(y[i].d), dmin = dco_fp16_to_fp32(y[i].dmin);
        uint8_t L[QK_K];
        for (int j = 0; j < 8; j++) {
            const float dl = d * (float)ls[j];
            const float dm = dmin * (float)lm[j];
            for (int l = 0; l < 32; l++) {
                int q = 0;
                if (dl != 0.0f) {
                    const float t = xb[j * 32 + l] + dm;
                    q = clampi((int)roundf(t / dl), 0, 15);
                }
                L[j * 32 + l] = (uint8_t)q;
            }
        }
        /* 32-byte groups: low nibbles = sub-block 2g, high nibbles = sub-block 2g+1 */
        for (int g = 0; g < 4; g++)
            for (int l = 0; l < 32; l++)
                y[i].qs[g * 32 + l] = (uint8_t)(L[64 * g + l] | (L[64 * g + 32 + l] << 4));
    }
}

void dco_quantize_row_q6_K(const float* x, void* vy, int64_t k) {
    blk_q6_K* y = (blk_q6_K*)vy;
    for (int64_t i = 0; i < k / QK_K; i++) {
        const float* xb = x + i * QK_K;
        float scale[16], max_scale = 0.0f;
        for (int s = 0; s < 16; s++) {
            float amax = 0.0f;
            for (int l = 0; l < 16; l++) {
                float a = fabsf(xb[s * 16 + l]);
                if (a > amax) amax = a;
            }
            scale[s] = amax / 31.0f;
            if (scale[s] > max_scale) max_scale = scale[s];
        }
        const float inv = max_scale > 0.0f ? 127.0f / max_scale : 0.0f;
        for (int s = 0; s < 16; s++) {
            float a = inv * scale[s];
            y[i].scales[s] = (int8_t)clampi((int)roundf(a), 0, 127);
        }
        y[i].d = dco_fp32_to_fp16(max_scale / 127.0f);
        const float d = dco_fp16_to_fp32(y[i].d);
        uint8_t L[QK_K];
        for (int s = 0; s < 16; s++) {
            const float dl = d * (float)y[i].scales[s];
            for (int l = 0; l < 16; l++) {
                int q = 0;
                if (dl != 0.0f) q = clampi((int)roundf(xb[s * 16 + l] / dl), -32, 31);
                L[s * 16 + l] = (uint8_t)(q + 32);
            }
        }
        /* two halves of 128: ql[h*64+i] holds element h*128+i (low) and h*128+64+i (high);
         * qh[h*32+i] holds the 2 high bits of elements h*128 + {0,32,64,96} + i */
        memset(y[i].qh, 0, sizeof(y[i].qh));
        for (int h = 0; h < 2; h++) {
            const uint8_t* Lh = L + 128 * h;
            for (int l = 0; l < 32; l++) {
                y[i].ql[h * 64 + l] = (uint8_t)((Lh[l] & 0xF) | ((Lh[l + 64] & 0xF) << 4));
                y[i].ql[h * 64 + 32 + l] = (uint8_t)((Lh[l + 32] & 0xF) | ((Lh[l + 96] & 0xF) << 4));
                y[i].qh[h * 32 + l] = (uint8_t)((Lh[l] >> 4) | ((Lh[l + 32] >> 4) << 2) |
                                                ((Lh[l + 64] >> 4) << 4) | ((Lh[l + 96] >> 4) << 6));
            }
        }
    }
}

/* q6 value (0..63) of element e (0..255) of a Q6_K block */
static int q6_at(const blk_q6_K* b, int e) {
    const int h = e / 128, r = e % 128;
    const int grp = r / 32, l = r % 32; /* grp 0..3 -> ql byte (l or l+32), nibble (lo or hi) */
    const uint8_t qlb = b->ql[h * 64 + (grp & 1) * 32 + l];
    const int lo = (grp < 2) ? (qlb & 0xF) : (qlb >> 4);
    const int hi = (b->qh[h * 32 + l] >> (2 * grp)) & 3;
    return lo | (hi << 4);
}

/* q4 value (0..15) of element e of a Q4_K block */
static int q4_at(const blk_q4_K* b, int e) {
    const int g = e / 64, r = e % 64;
    const uint8_t v = b->qs[g * 32 + (r % 32)];
    return r < 32 ? (v & 0xF) : (v >> 4);
}

void dco_dequantize_row(int type, const void* vx, float* y, int64_t k) {
    if (type == DCO_Q8_0) {
        const blk_q8_0* x = (const blk_q8_0*)vx;
        for (int64_t i = 0; i < k / QK8_0; i++) {
            const float d = dco_fp16_to_fp32(x[i].d);
            for (int j = 0; j < QK8_0; j++) y[i * QK8_0 + j] = d * (float)x[i].qs[j];
        }
    } else if (type == DCO_Q8_K) {
        const blk_q8_K* x = (const blk_q8_K*)vx;
        for (int64_t i = 0; i < k / QK_K; i++)
            for (int j = 0; j < QK_K; j++) y[i * QK_K + j] = x[i].d * (float)x[i].qs[j];
    } else if (type == DCO_Q4_K) {
        const blk_q4_K* x = (const blk_q4_K*)vx;
        for (int64_t i = 0; i < k / QK_K; i++) {
            const float d = dco_fp16_to_fp32(x[i].d), dmin = dco_fp16_to_fp32(x[i].dmin);
            for (int e = 0; e < QK_K; e++) {
                int sc, m;
                unpack_q4_K_scale(x[i].scales, e / 32, &sc, &m);
                const float dl = d * (float)sc, ml = dmin * (float)m;
                y[i * QK_K + e] = dl * (float)q4_at(&x[i], e) - ml;
            }
        }
    } else if (type == DCO_Q6_K) {
        const blk_q6_K* x = (const blk_q6_K*)vx;
        for (int64_t i = 0; i < k / QK_K; i++) {
            const float d = dco_fp16_to_fp32(x[i].d);
            for (int e = 0; e < QK_K; e++) {
                const float dl = d * (float)x[i].scales[e / 16];
                y[i * QK_K + e] = dl * (float)(q6_at(&x[i], e) - 32);
            }
        }
    }
}

/* ---------------- vec_dot (ggml vec_dot_* scalar reference structure) ---------------- */

static float vec_dot_q8_0(int n, const blk_q8_0* w, const blk_q8_0* x) {
    float sumf = 0.0f;
    for (int b = 0; b < n / QK8_0; b++) {
        int sumi = 0;
        for (int j = 0; j < QK8_0; j++) sumi += (int)w[b].qs[j] * (int)x[b].qs[j];
        const float dd = dco_fp16_to_fp32(w[b].d) * dco_fp16_to_fp32(x[b].d);
        sumf += (float)sumi * dd;
    }
    return sumf;
}

/* per super-block: isum = sum_j sc_j * dot_j (dot over 32 unsigned nibbles x q8),
 * msum = sum_j m_j * (bsum_{2j} + bsum_{2j+1});
 * sumf += (d_w * d_x) * isum - (dmin_w * d_x) * msum */
static void q4_K_ints(const blk_q4_K* w, const blk_q8_K* x, int32_t* sub, int32_t* msum) {
    int32_t ms = 0;
    for (int j = 0; j < 8; j++) {
        int sc, m;
        unpack_q4_K_scale(w->scales, j, &sc, &m);
        int dot = 0;
        for (int l = 0; l < 32; l++) dot += q4_at(w, j * 32 + l) * (int)x->qs[j * 32 + l];
        sub[j] = sc * dot;
        ms += m * ((int)x->bsums[2 * j] + (int)x->bsums[2 * j + 1]);
    }
    *msum = ms;
}

static float vec_dot_q4_K(int n, const blk_q4_K* w, const blk_q8_K* x) {
    float sumf = 0.0f;
    for (int b = 0; b < n / QK_K; b++) {
        int32_t sub[8], msum, isum = 0;
        q4_K_ints(&w[b], &x[b], sub, &msum);
        for (int j = 0; j < 8; j++) isum += sub[j];
        const float d = dco_fp16_to_fp32(w[b].d) * x[b].d;
        const float dmin = dco_fp16_to_fp32(w[b].dmin) * x[b].d;
        sumf += d * (float)isum;
        sumf -= dmin * (float)msum;
    }
    return sumf;
}

static void q6_K_ints(const blk_q6_K* w, const blk_q8_K* x, int32_t* sub16) {
    for (int s = 0; s < 16; s++) {
        int dot = 0;
        for (int l = 0; l < 16; l++) dot += (q6_at(w, s * 16 + l) - 32) * (int)x->qs[s * 16 + l];
        sub16[s] = dot;
    }
}

static float vec_dot_q6_K(int n, const blk_q6_K* w, const blk_q8_K* x) {
    float sumf = 0.0f;
    for (int b = 0; b < n / QK_K; b++) {
        int32_t sub[16], isum = 0;
        q6_K_ints(&w[b], &x[b], sub);
        for (int s = 0; s < 16; s++) isum += (int)w[b].scales[s] * sub[s];
        const float d = dco_fp16_to_fp32(w[b].d) * x[b].d;
        sumf += d * (float)isum;
    }
    return sumf;
}

void dco_vec_dot(int type, int n, float* s, const void* w, const void* xq) {
    switch (type) {
        case DCO_Q8_0: *s = vec_dot_q8_0(n, (const blk_q8_0*)w, (const blk_q8_0*)xq); break;
        case DCO_Q4_K: *s = vec_dot_q4_K(n, (const blk_q4_K*)w, (const blk_q8_K*)xq); break;
        case DCO_Q6_K: *s = vec_dot_q6_K(n, (const blk_q6_K*)w, (const blk_q8_K*)xq); break;
        default: *s = 0.0f;
    }
}

void dco_block_dots(int type, int n, const void* vw, const void* vx, int32_t* out, int32_t* out2) {
    if (type == DCO_Q8_0) {
        const blk_q8_0 *w = (const blk_q8_0*)vw, *x = (const blk_q8_0*)vx;
        for (int b = 0; b < n / QK8_0; b++) {
            int sumi = 0;
            for (int j = 0; j < QK8_0; j++) sumi += (int)w[b].qs[j] * (int)x[b].qs[j];
            out[b] = sumi;
        }
    } else if (type == DCO_Q4_K) {
        const blk_q4_K* w = (const blk_q4_K*)vw;
        const blk_q8_K* x = (const blk_q8_K*)vx;
        for (int b = 0; b < n / QK_K; b++) q4_K_ints(&w[b], &x[b], out + 8 * b, out2 + b);
    } else if (type == DCO_Q6_K) {
        const blk_q6_K* w = (const blk_q6_K*)vw;
        const blk_q8_K* x = (const blk_q8_K*)vx;
        for (int b = 0; b < n / QK_K; b++) q6_K_ints(&w[b], &x[b], out + 16 * b);
    }
}

/* ---------------- AVX2 restatement of vec_dot_q4_K (CPU baseline) --------------------------
 * The same integer sums and the same float operations in the same order as vec_dot_q4_K, so the
 * result is bit-identical: per pair group g the 32 nibble bytes hold sub-block 2g (low nibbles,
 * activation bytes 64g..64g+31) and 2g+1 (high nibbles, 64g+32..64g+63); maddubs multiplies the
 * unsigned nibbles by the signed activation bytes into int16 pairs (|pair| <= 3810, no saturation)
 * and madd scales them by the sub-block's 6-bit scale into int32. */
#if defined(__x86_64__)
#include <immintrin.h>
__attribute__((target("avx2,fma"))) static float vec_dot_q4_K_avx2(int n, const blk_q4_K* w, const blk_q8_K* x) {
    const __m256i m4 = _mm256_set1_epi8(0x0F);
    float sumf = 0.0f;
    for (int b = 0; b < n / QK_K; b++) {
        int sc[8], mn[8];
        for (int j = 0; j < 8; j++) unpack_q4_K_scale(w[b].scales, j, &sc[j], &mn[j]);
        __m256i acc = _mm256_setzero_si256();
        for (int g = 0; g < 4; g++) {
            const __m256i q = _mm256_loadu_si256((const __m256i*)(w[b].qs + 32 * g));
            const __m256i lo = _mm256_and_si256(q, m4);
            const __m256i hi = _mm256_and_si256(_mm256_srli_epi16(q, 4), m4);
            const __m256i xl = _mm256_loadu_si256((const __m256i*)(x[b].qs + 64 * g));
            const __m256i xh = _mm256_loadu_si256((const __m256i*)(x[b].qs + 64 * g + 32));
            const __m256i pl = _mm256_madd_epi16(_mm256_maddubs_epi16(lo, xl), _mm256_set1_epi16((short)sc[2 * g]));
            const __m256i ph = _mm256_madd_epi16(_mm256_maddubs_epi16(hi, xh), _mm256_set1_epi16((short)sc[2 * g + 1]));
            acc = _mm256_add_epi32(acc, _mm256_add_epi32(pl, ph));
        }
        __m128i t = _mm_add_epi32(_mm256_castsi256_si128(acc), _mm256_extracti128_si256(acc, 1));
        t = _mm_add_epi32(t, _mm_shuffle_epi32(t, 0x4E));
        t = _mm_add_epi32(t, _mm_shuffle_epi32(t, 0xB1));
        const int32_t isum = _mm_cvtsi128_si32(t);
        int32_t ms = 0;
        for (int j = 0; j < 8; j++) ms += mn[j] * ((int)x[b].bsums[2 * j] + (int)x[b].bsums[2 * j + 1]);
        const float d = dco_fp16_to_fp32(w[b].d) * x[b].d;
        const float dmin = dco_fp16_to_fp32(w[b].dmin) * x[b].d;
        sumf += d * (float)isum;
        sumf -= dmin * (float)ms;
    }
    return sumf;
}
static int have_avx2(void) { return __builtin_cpu_supports("avx2"); }

/* ---------------- AVX-512 VNNI restatement of vec_dot_q4_K (the CPU baseline where the host has
 * it; the vpdpbusd pattern of the reference's own best-ISA integer GEMV,
 * core/src/kernels/cpu_int4.cpp:279-410) ----------------------------------------------------
 * Per pair group g one 64-byte vector holds the low nibbles (sub-block 2g) then the high nibbles
 * (sub-block 2g+1), matching activation bytes 64g..64g+63; vpdpbusd forms unsigned x signed byte
 * products summed by fours into 16 int32 lanes (lanes 0-7: sub-block 2g, 8-15: 2g+1), which are
 * scaled by the two 6-bit sub-block scales (vpmulld) and accumulated.  The integer sum, the min
 * term and the float operations are those of vec_dot_q4_K, in the same order: bit-identical. */
__attribute__((target("avx512f,avx512bw,avx512vnni,fma"))) static float vec_dot_q4_K_vnni(int n, const blk_q4_K* w,
                                                                                           const blk_q8_K* x) {
    const __m256i m4 = _mm256_set1_epi8(0x0F);
    float sumf = 0.0f;
    for (int b = 0; b < n / QK_K; b++) {
        int sc[8], mn[8];
        for (int j = 0; j < 8; j++) unpack_q4_K_scale(w[b].scales, j, &sc[j], &mn[j]);
        __m512i acc = _mm512_setzero_si512();
        for (int g = 0; g < 4; g++) {
            const __m256i q = _mm256_loadu_si256((const __m256i*)(w[b].qs + 32 * g));
            const __m256i lo = _mm256_and_si256(q, m4);
            const __m256i hi = _mm256_and_si256(_mm256_srli_epi16(q, 4), m4);
            const __m512i qq = _mm512_inserti64x4(_mm512_castsi256_si512(lo), hi, 1);
            const __m512i xx = _mm512_loadu_si512((const void*)(x[b].qs + 64 * g));
            const __m512i dot = _mm512_dpbusd_epi32(_mm512_setzero_si512(), qq, xx);
            const __m512i scv = _mm512_inserti64x4(_mm512_castsi256_si512(_mm256_set1_epi32(sc[2 * g])),
                                                   _mm256_set1_epi32(sc[2 * g + 1]), 1);
            acc = _mm512_add_epi32(acc, _mm512_mullo_epi32(dot, scv));
        }
        const int32_t isum = _mm512_reduce_add_epi32(acc);
        int32_t ms = 0;
        for (int j = 0; j < 8; j++) ms += mn[j] * ((int)x[b].bsums[2 * j] + (int)x[b].bsums[2 * j + 1]);
        const float d = dco_fp16_to_fp32(w[b].d) * x[b].d;
        const float dmin = dco_fp16_to_fp32(w[b].dmin) * x[b].d;
        sumf += d * (float)isum;
        sumf -= dmin * (float)ms;
    }
    return sumf;
}
static int have_vnni(void) {
    return __builtin_cpu_supports("avx512f") && __builtin_cpu_supports("avx512bw") &&
           __builtin_cpu_supports("avx512vnni");
}
#else
static float vec_dot_q4_K_avx2(int n, const blk_q4_K* w, const blk_q8_K* x) { return vec_dot_q4_K(n, w, x); }
static float vec_dot_q4_K_vnni(int n, const blk_q4_K* w, const blk_q8_K* x) { return vec_dot_q4_K(n, w, x); }
static int have_avx2(void) { return 0; }
static int have_vnni(void) { return 0; }
#endif

/* ---------------- threaded row-sliced GEMV/GEMM (cb_gemv_custom, inference.cpp:896-924) ----- */
typedef struct {
    int type, simd;
    const uint8_t* w;
    size_t row_stride;
    int64_t n_rows, k, m, r0, r1;
    const uint8_t* xq;
    float* y;
} mm_job;

static void* mm_worker(void* p) {
    mm_job* j = (mm_job*)p;
    const size_t xrow = dco_row_size(j->type == DCO_Q8_0 ? DCO_Q8_0 : DCO_Q8_K, j->k);
    for (int64_t r = j->r0; r < j->r1; r++)
        for (int64_t i = 0; i < j->m; i++) {
            float* dst = &j->y[i * j->n_rows + r];
            if (j->simd == DCO_ISA_VNNI)
                *dst = vec_dot_q4_K_vnni((int)j->k, (const blk_q4_K*)(j->w + r * j->row_stride),
                                         (const blk_q8_K*)(j->xq + i * xrow));
            else if (j->simd == DCO_ISA_AVX2)
                *dst = vec_dot_q4_K_avx2((int)j->k, (const blk_q4_K*)(j->w + r * j->row_stride),
                                         (const blk_q8_K*)(j->xq + i * xrow));
            else
                dco_vec_dot(j->type, (int)j->k, dst, j->w + r * j->row_stride, j->xq + i * xrow);
        }
    return NULL;
}

static void mul_mat_threads(int type, int simd, const void* w, size_t row_stride, int64_t n_rows,
                            int64_t k, const void* xq, int64_t m, float* y, int nthreads);

void dco_mul_mat(int type, const void* w, size_t row_stride, int64_t n_rows, int64_t k,
                 const void* xq, int64_t m, float* y, int nthreads) {
    mul_mat_threads(type, 0, w, row_stride, n_rows, k, xq, m, y, nthreads);
}

int dco_simd_isa(void) { return have_vnni() ? DCO_ISA_VNNI : (have_avx2() ? DCO_ISA_AVX2 : 0); }

int dco_mul_mat_simd(int type, const void* w, size_t row_stride, int64_t n_rows, int64_t k,
                     const void* xq, int64_t m, float* y, int nthreads, int isa) {
    const int best = dco_simd_isa();
    int use = isa == 0 ? best : isa;
    if (type != DCO_Q4_K || (use == DCO_ISA_VNNI && !have_vnni()) || (use == DCO_ISA_AVX2 && !have_avx2())) use = 0;
    mul_mat_threads(type, use, w, row_stride, n_rows, k, xq, m, y, nthreads);
    return use;
}

static void mul_mat_threads(int type, int simd, const void* w, size_t row_stride, int64_t n_rows,
                            int64_t k, const void* xq, int64_t m, float* y, int nthreads) {
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    pthread_t th[256];
    mm_job jobs[256];
    const int64_t per = (n_rows + nthreads - 1) / nthreads;
    for (int t = 0; t < nthreads; t++) {
        int64_t r0 = t * per, r1 = r0 + per;
        if (r1 > n_rows) r1 = n_rows;
        if (r0 > n_rows) r0 = n_rows;
        jobs[t] = (mm_job){type, simd, (const uint8_t*)w, row_stride, n_rows, k, m, r0, r1,
                           (const uint8_t*)xq, y};
        if (t > 0) pthread_create(&th[t], NULL, mm_worker, &jobs[t]);
    }
    mm_worker(&jobs[0]);
    for (int t = 1; t < nthreads; t++) pthread_join(th[t], NULL);
}

/* ---------------- paged fp16 KV (kv_cache.cpp:353-370) and decode attention ----------------
 * Element (block, layer, slot, head, dim) lives at
 *   ((block * n_layer + layer) * 16 + slot) * hkv * d + head * d + dim.
 * Decode attention follows the flash path (inference.cpp:1519-1573) made per sequence: query
 * head h reads KV head h / (hq/hkv); keys 0..ctx_len-1 of its own block table; scale = the
 * caller's (1/sqrt(head_dim) in the engine); softmax in double precision. */
#define KV_BLOCK 16

static size_t kv_index(int blk, int n_layer, int layer, int slot, int hkv, int d, int head) {
    return (((size_t)blk * n_layer + layer) * KV_BLOCK + slot) * (size_t)hkv * d + (size_t)head * d;
}

typedef struct {
    const float* q;
    const uint16_t *k, *v;
    int n_layer, layer;
    const int32_t* bt;
    int mbs;
    const int32_t* ctx;
    int n_seqs, hq, hkv, d;
    float scale;
    float* out;
    int t, nt;
} attn_job;

static void* attn_worker(void* p) {
    attn_job* J = (attn_job*)p;
    const int rep = J->hq / J->hkv;
    double* sc = NULL;
    size_t sc_cap = 0;
    double acc[1024];
    for (int w = J->t; w < J->n_seqs * J->hq; w += J->nt) {
        const int s = w / J->hq, h = w % J->hq, kvh = h / rep;
        const int L = J->ctx[s];
        if ((size_t)L > sc_cap) {
            free(sc);
            sc_cap = (size_t)L + 64;
            sc = (double*)malloc(sc_cap * sizeof(double));
        }
        const float* qh = J->q + ((size_t)s * J->hq + h) * J->d;
        double mx = -1e300;
        for (int t = 0; t < L; t++) {
            const int blk = J->bt[(size_t)s * J->mbs + t / KV_BLOCK];
            const uint16_t* kr = J->k + kv_index(blk, J->n_layer, J->layer, t % KV_BLOCK, J->hkv, J->d, kvh);
            double dot = 0.0;
            for (int i = 0; i < J->d; i++) dot += (double)qh[i] * (double)dco_fp16_to_fp32(kr[i]);
            sc[t] = dot * (double)J->scale;
            if (sc[t] > mx) mx = sc[t];
        }
        double den = 0.0;
        for (int i = 0; i < J->d; i++) acc[i] = 0.0;
        for (int t = 0; t < L; t++) {
            const double pr = exp(sc[t] - mx);
            den += pr;
            const int blk = J->bt[(size_t)s * J->mbs + t / KV_BLOCK];
            const uint16_t* vr = J->v + kv_index(blk, J->n_layer, J->layer, t % KV_BLOCK, J->hkv, J->d, kvh);
            for (int i = 0; i < J->d; i++) acc[i] += pr * (double)dco_fp16_to_fp32(vr[i]);
        }
        float* o = J->out + ((size_t)s * J->hq + h) * J->d;
        for (int i = 0; i < J->d; i++) o[i] = L > 0 ? (float)(acc[i] / den) : 0.0f;
    }
    free(sc);
    return NULL;
}

void dco_paged_attn_decode(const float* q, const uint16_t* k_arena, const uint16_t* v_arena,
                           int n_layer, int layer, const int32_t* block_tables,
                           int max_blocks_per_seq, const int32_t* ctx_lens, int n_seqs, int hq,
                           int hkv, int d, float scale, float* out, int nthreads) {
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    if (d > 1024) return;
    pthread_t th[256];
    attn_job jobs[256];
    for (int t = 0; t < nthreads; t++) {
        jobs[t] = (attn_job){q, k_arena, v_arena, n_layer, layer, block_tables, max_blocks_per_seq,
                             ctx_lens, n_seqs, hq, hkv, d, scale, out, t, nthreads};
        if (t > 0) pthread_create(&th[t], NULL, attn_worker, &jobs[t]);
    }
    attn_worker(&jobs[0]);
    for (int t = 1; t < nthreads; t++) pthread_join(th[t], NULL);
}

/* PagedKVCache::WriteKSlot / WriteVSlot (kv_cache.cpp:566-598): f32 -> fp16 per slot */
void dco_kv_append(const float* k, const float* v, uint16_t* k_arena, uint16_t* v_arena,
                   int n_layer, int layer, const int32_t* block_tables, int max_blocks_per_seq,
                   const int32_t* seq_ids, const int32_t* positions, int n_tok, int hkv, int d) {
    for (int i = 0; i < n_tok; i++) {
        const int s = seq_ids[i], pos = positions[i];
        const int blk = block_tables[(size_t)s * max_blocks_per_seq + pos / KV_BLOCK];
        const size_t base = kv_index(blk, n_layer, layer, pos % KV_BLOCK, hkv, d, 0);
        for (int e = 0; e < hkv * d; e++) {
            k_arena[base + e] = dco_fp32_to_fp16(k[(size_t)i * hkv * d + e]);
            v_arena[base + e] = dco_fp32_to_fp16(v[(size_t)i * hkv * d + e]);
        }
    }
}
