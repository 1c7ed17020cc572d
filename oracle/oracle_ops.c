/*
 * CPU ORACLE — test infrastructure only (see oracle.h).  Op-level restatement.
 *
 * Every function names the reference lines it follows.  Paths are relative
 * to the reference project root.  Compiled with -ffp-contract=off.
 */
#include "oracle.h"

#include <float.h>
#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------ */
/* fp16 <-> fp32                                                             */
/* ------------------------------------------------------------------------ */

/* Follows ref_fp16_to_fp32, Singularity/tests/test_and_bench_a5.cpp:150-176. */
float orc_fp16_to_fp32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t exp = (h >> 10) & 0x1Fu;
    const uint32_t mant = h & 0x03FFu;
    uint32_t bits;
    if (exp == 0) {
        if (mant == 0) {
            bits = sign;
        } else {
            uint32_t m = mant;
            uint32_t e = 127u - 14u;
            while ((m & 0x0400u) == 0) {
                m <<= 1;
                --e;
            }
            m &= 0x03FFu;
            bits = sign | (e << 23) | (m << 13);
        }
    } else if (exp == 31u) {
        bits = sign | 0x7F800000u | (mant << 13);
    } else {
        bits = sign | ((exp + (127u - 15u)) << 23) | (mant << 13);
    }
    float out;
    memcpy(&out, &bits, sizeof out);
    return out;
}

/* Round-to-nearest-even binary32 -> binary16, written from the IEEE-754
 * rules.  It replaces the hardware conversion the reference calls through
 * singularity_f32_to_f16_row_a5 (Singularity/src/asm/singularity_asm_kernels.h:146),
 * which is VFPv4 vcvt.f16.f32 in the default (RNE) mode. */
uint16_t orc_fp32_to_fp16(float f) {
    uint32_t x;
    memcpy(&x, &f, sizeof x);
    const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    const uint32_t ax = x & 0x7FFFFFFFu;
    if (ax > 0x7F800000u) {                 /* NaN: quiet, keep top payload bits */
        return (uint16_t)(sign | 0x7E00u | ((ax >> 13) & 0x03FFu));
    }
    if (ax == 0x7F800000u) return (uint16_t)(sign | 0x7C00u);
    const int e = (int)(ax >> 23) - 127;
    if (e >= -14) {
        if (e > 15) return (uint16_t)(sign | 0x7C00u);
        const uint32_t m = ax & 0x007FFFFFu;
        uint32_t h = ((uint32_t)(e + 15) << 10) | (m >> 13);
        const uint32_t rem = m & 0x1FFFu;
        if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1u;   /* may carry into inf */
        return (uint16_t)(sign | h);
    }
    /* Subnormal half (or zero): value / 2^-24 rounded to nearest even. */
    const int shift = -1 - e;                 /* 13 + (-14 - e) */
    if (shift > 25) return sign;
    const uint32_t m = (ax & 0x007FFFFFu) | 0x00800000u;
    uint32_t h = m >> shift;
    const uint32_t rem = m & ((1u << shift) - 1u);
    const uint32_t half = 1u << (shift - 1);
    if (rem > half || (rem == half && (h & 1u))) h += 1u;
    return (uint16_t)(sign | h);
}

void orc_fp32_to_fp16_row(const float* x, uint16_t* y, int64_t n) {
    for (int64_t i = 0; i < n; ++i) y[i] = orc_fp32_to_fp16(x[i]);
}

void orc_fp16_to_fp32_row(const uint16_t* x, float* y, int64_t n) {
    for (int64_t i = 0; i < n; ++i) y[i] = orc_fp16_to_fp32(x[i]);
}

/* ------------------------------------------------------------------------ */
/* Block layouts                                                             */
/* ------------------------------------------------------------------------ */

/* Singularity/src/asm/singularity_asm_kernels.h:32-43 */
typedef struct { uint16_t d; uint8_t qs[16]; } __attribute__((packed)) blk_q4_0;
typedef struct { uint16_t d; int8_t qs[32]; } __attribute__((packed)) blk_q8_0;
/* Public GGUF K-quant layouts (ggml-common.h; IDs at Sutra/src/llm_backends.cpp:3399-3401). */
typedef struct { uint16_t d; uint16_t dmin; uint8_t scales[12]; uint8_t qs[128]; } __attribute__((packed)) blk_q4_k;
typedef struct { uint8_t ql[128]; uint8_t qh[64]; int8_t scales[16]; uint16_t d; } __attribute__((packed)) blk_q6_k;
typedef struct { float d; int8_t qs[256]; int16_t bsums[16]; } __attribute__((packed)) blk_q8_k;

_Static_assert(sizeof(blk_q4_0) == ORC_Q4_0_BYTES, "q4_0");
_Static_assert(sizeof(blk_q8_0) == ORC_Q8_0_BYTES, "q8_0");
_Static_assert(sizeof(blk_q4_k) == ORC_Q4_K_BYTES, "q4_k");
_Static_assert(sizeof(blk_q6_k) == ORC_Q6_K_BYTES, "q6_k");
_Static_assert(sizeof(blk_q8_k) == ORC_Q8_K_BYTES, "q8_k");

size_t orc_row_bytes(int type, int k) {
    switch (type) {
    case ORC_F32: return (size_t)k * 4;
    case ORC_F16: return (size_t)k * 2;
    case ORC_Q4_0: return (size_t)(k / 32) * ORC_Q4_0_BYTES;
    case ORC_Q8_0: return (size_t)(k / 32) * ORC_Q8_0_BYTES;
    case ORC_Q4_K: return (size_t)(k / 256) * ORC_Q4_K_BYTES;
    case ORC_Q6_K: return (size_t)(k / 256) * ORC_Q6_K_BYTES;
    case ORC_Q8_K: return (size_t)(k / 256) * ORC_Q8_K_BYTES;
    default: return 0;
    }
}

int orc_vec_dot_type(int wtype) {
    return (wtype == ORC_Q4_K || wtype == ORC_Q6_K) ? ORC_Q8_K : ORC_Q8_0;
}

/* ------------------------------------------------------------------------ */
/* Activation quantizers                                                     */
/* ------------------------------------------------------------------------ */

/* Follows ref_quantize_row_q8_0, Singularity/tests/test_and_bench_a5.cpp:223-245:
 * d = amax*(1/127) rounded to fp16, id = 127/amax, q = trunc(x*id ± 0.5)
 * clamped to ±127. */
void orc_quantize_row_q8_0(const float* x, void* vy, int k) {
    const int nb = k >> 5;
    blk_q8_0* y = (blk_q8_0*)vy;
    for (int b = 0; b < nb; ++b) {
        const float* xb = x + b * 32;
        float amax = 0.0f;
        for (int j = 0; j < 32; ++j) {
            const float av = xb[j] < 0.0f ? -xb[j] : xb[j];
            if (av > amax) amax = av;
        }
        const float d = amax * (1.0f / 127.0f);
        const float id = (amax != 0.0f) ? (127.0f / amax) : 0.0f;
        y[b].d = orc_fp32_to_fp16(d);
        for (int j = 0; j < 32; ++j) {
            const float scaled = xb[j] * id;
            const int32_t q = (int32_t)(scaled >= 0.0f ? (scaled + 0.5f) : (scaled - 0.5f));
            y[b].qs[j] = (int8_t)(q < -127 ? -127 : (q > 127 ? 127 : q));
        }
    }
}

/* Round to nearest, ties to even (the default FP environment). */
static inline int orc_nearest_int(float v) { return (int)rintf(v); }

/* ggml's quantize_row_q8_K_ref (llama.cpp, version unpinned; not in the
 * reference tree): per 256 values, max = the value of largest magnitude,
 * iscale = -127/max, q = nearest_int(iscale*x) capped at 127, d = 1/iscale,
 * bsums = sums of 16-value groups.  All-zero blocks give d = 0, q = 0,
 * bsums = 0. */
void orc_quantize_row_q8_k(const float* x, void* vy, int k) {
    const int nb = k / 256;
    blk_q8_k* y = (blk_q8_k*)vy;
    for (int b = 0; b < nb; ++b) {
        const float* xb = x + (size_t)b * 256;
        float max = 0.0f, amax = 0.0f;
        for (int j = 0; j < 256; ++j) {
            const float ax = fabsf(xb[j]);
            if (ax > amax) { amax = ax; max = xb[j]; }
        }
        if (amax == 0.0f) {
            memset(&y[b], 0, sizeof y[b]);
            continue;
        }
        const float iscale = -127.0f / max;
        for (int j = 0; j < 256; ++j) {
            const int v = orc_nearest_int(iscale * xb[j]);
            y[b].qs[j] = (int8_t)(v > 127 ? 127 : v);
        }
        for (int g = 0; g < 16; ++g) {
            int s = 0;
            for (int j = 0; j < 16; ++j) s += y[b].qs[g * 16 + j];
            y[b].bsums[g] = (int16_t)s;
        }
        y[b].d = 1.0f / iscale;
    }
}

/* ------------------------------------------------------------------------ */
/* Block dot products                                                        */
/* ------------------------------------------------------------------------ */

/* Follows ref_vec_dot_q4_0_q8_0, Singularity/tests/test_and_bench_a5.cpp:184-203. */
void orc_block_dots_q4_0_q8_0(int n, const void* vx, const void* vy, int32_t* out) {
    const blk_q4_0* x = (const blk_q4_0*)vx;
    const blk_q8_0* y = (const blk_q8_0*)vy;
    for (int b = 0; b < (n >> 5); ++b) {
        int32_t sumi = 0;
        for (int j = 0; j < 16; ++j) {
            const int32_t v0 = (int32_t)(x[b].qs[j] & 0x0Fu) - 8;
            const int32_t v1 = (int32_t)(x[b].qs[j] >> 4) - 8;
            sumi += v0 * (int32_t)y[b].qs[j] + v1 * (int32_t)y[b].qs[j + 16];
        }
        out[b] = sumi;
    }
}

float orc_vec_dot_q4_0_q8_0(int n, const void* vx, const void* vy) {
    const blk_q4_0* x = (const blk_q4_0*)vx;
    const blk_q8_0* y = (const blk_q8_0*)vy;
    float sumf = 0.0f;
    for (int b = 0; b < (n >> 5); ++b) {
        int32_t sumi;
        orc_block_dots_q4_0_q8_0(32, &x[b], &y[b], &sumi);
        const float dx = orc_fp16_to_fp32(x[b].d);
        const float dy = orc_fp16_to_fp32(y[b].d);
        sumf += (dx * dy) * (float)sumi;
    }
    return sumf;
}

/* Follows ref_vec_dot_q8_0_q8_0, Singularity/tests/test_and_bench_a5.cpp:205-221. */
void orc_block_dots_q8_0_q8_0(int n, const void* vx, const void* vy, int32_t* out) {
    const blk_q8_0* x = (const blk_q8_0*)vx;
    const blk_q8_0* y = (const blk_q8_0*)vy;
    for (int b = 0; b < (n >> 5); ++b) {
        int32_t sumi = 0;
        for (int j = 0; j < 32; ++j) sumi += (int32_t)x[b].qs[j] * (int32_t)y[b].qs[j];
        out[b] = sumi;
    }
}

float orc_vec_dot_q8_0_q8_0(int n, const void* vx, const void* vy) {
    const blk_q8_0* x = (const blk_q8_0*)vx;
    const blk_q8_0* y = (const blk_q8_0*)vy;
    float sumf = 0.0f;
    for (int b = 0; b < (n >> 5); ++b) {
        int32_t sumi;
        orc_block_dots_q8_0_q8_0(32, &x[b], &y[b], &sumi);
        const float dx = orc_fp16_to_fp32(x[b].d);
        const float dy = orc_fp16_to_fp32(y[b].d);
        sumf += (dx * dy) * (float)sumi;
    }
    return sumf;
}

/* Q4_K 6-bit scale/min unpacking (ggml get_scale_min_k4; the same packing is
 * documented in gguf-py quants.py Q4_K.get_scale_min). */
static void q4k_scale_min(const uint8_t* s, uint8_t sc[8], uint8_t m[8]) {
    for (int j = 0; j < 4; ++j) {
        sc[j] = s[j] & 63;
        m[j] = s[j + 4] & 63;
    }
    for (int j = 4; j < 8; ++j) {
        sc[j] = (uint8_t)((s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4));
        m[j] = (uint8_t)((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
    }
}

/* Q4_K element e of a super-block: sub-block j = e/32; nibble from
 * qs[(e/64)*32 + e%32], low half for (e/32) even, high half for odd. */
static inline int q4k_q(const blk_q4_k* x, int e) {
    const uint8_t byte = x->qs[(e >> 6) * 32 + (e & 31)];
    return ((e >> 5) & 1) ? (byte >> 4) : (byte & 0x0F);
}

/* Q6_K element e = h*128 + g*32 + l: low 4 bits from
 * ql[h*64 + (g&1)*32 + l] >> 4*(g>>1), high 2 bits from qh[h*32 + l] >> 2g;
 * value q - 32. */
static inline int q6k_q(const blk_q6_k* x, int e) {
    const int h = e >> 7, g = (e >> 5) & 3, l = e & 31;
    const int lo = (x->ql[h * 64 + (g & 1) * 32 + l] >> (4 * (g >> 1))) & 0x0F;
    const int hi = (x->qh[h * 32 + l] >> (2 * g)) & 0x03;
    return (lo | (hi << 4)) - 32;
}

/* Q4_K · Q8_K (ggml vec_dot_q4_K_q8_K, restated).  Per super-block the
 * integer parts are exact: isum = Σ_j sc_j·Σ q·y, msum = Σ_j m_j·(bsum_2j +
 * bsum_2j+1).  fp32 order: sumf += (d_x·d_y)·isum; sumf -= (dmin_x·d_y)·msum. */
void orc_block_dots_q4_k_q8_k(int n, const void* vx, const void* vy, int32_t* isum, int32_t* msum) {
    const blk_q4_k* x = (const blk_q4_k*)vx;
    const blk_q8_k* y = (const blk_q8_k*)vy;
    for (int b = 0; b < n / 256; ++b) {
        uint8_t sc[8], m[8];
        q4k_scale_min(x[b].scales, sc, m);
        int32_t is = 0, ms = 0;
        for (int j = 0; j < 8; ++j) {
            int32_t dot = 0;
            for (int l = 0; l < 32; ++l) dot += q4k_q(&x[b], j * 32 + l) * (int32_t)y[b].qs[j * 32 + l];
            is += (int32_t)sc[j] * dot;
            ms += (int32_t)m[j] * ((int32_t)y[b].bsums[2 * j] + (int32_t)y[b].bsums[2 * j + 1]);
        }
        isum[b] = is;
        msum[b] = ms;
    }
}

float orc_vec_dot_q4_k_q8_k(int n, const void* vx, const void* vy) {
    const blk_q4_k* x = (const blk_q4_k*)vx;
    const blk_q8_k* y = (const blk_q8_k*)vy;
    float sumf = 0.0f;
    for (int b = 0; b < n / 256; ++b) {
        int32_t is, ms;
        orc_block_dots_q4_k_q8_k(256, &x[b], &y[b], &is, &ms);
        const float d = orc_fp16_to_fp32(x[b].d) * y[b].d;
        const float dmin = orc_fp16_to_fp32(x[b].dmin) * y[b].d;
        sumf += d * (float)is;
        sumf -= dmin * (float)ms;
    }
    return sumf;
}

/* Q6_K · Q8_K (ggml vec_dot_q6_K_q8_K, restated): isum = Σ_g sc_g·Σ q·y over
 * 16-value groups (exact); sumf += (d_x·d_y)·isum. */
void orc_block_dots_q6_k_q8_k(int n, const void* vx, const void* vy, int32_t* isum) {
    const blk_q6_k* x = (const blk_q6_k*)vx;
    const blk_q8_k* y = (const blk_q8_k*)vy;
    for (int b = 0; b < n / 256; ++b) {
        int32_t is = 0;
        for (int g = 0; g < 16; ++g) {
            int32_t dot = 0;
            for (int l = 0; l < 16; ++l) dot += q6k_q(&x[b], g * 16 + l) * (int32_t)y[b].qs[g * 16 + l];
            is += (int32_t)x[b].scales[g] * dot;
        }
        isum[b] = is;
    }
}

float orc_vec_dot_q6_k_q8_k(int n, const void* vx, const void* vy) {
    const blk_q6_k* x = (const blk_q6_k*)vx;
    const blk_q8_k* y = (const blk_q8_k*)vy;
    float sumf = 0.0f;
    for (int b = 0; b < n / 256; ++b) {
        int32_t is;
        orc_block_dots_q6_k_q8_k(256, &x[b], &y[b], &is);
        const float d = orc_fp16_to_fp32(x[b].d) * y[b].d;
        sumf += d * (float)is;
    }
    return sumf;
}

/* ------------------------------------------------------------------------ */
/* Dequantization (one row)                                                  */
/* ------------------------------------------------------------------------ */

/* Q4_0 / Q8_0 follow the embedding dequant in
 * Singularity/src/core/cortex_a5_engine.cpp:1073-1105; Q4_K / Q6_K follow the
 * public layouts (gguf-py quants.py Q4_K/Q6_K.dequantize_blocks):
 * Q4_K y = (d·sc)·q − dmin·m,  Q6_K y = (d·sc)·q. */
void orc_dequantize_row(int type, const void* vx, float* y, int k) {
    switch (type) {
    case ORC_F32: memcpy(y, vx, (size_t)k * 4); break;
    case ORC_F16: orc_fp16_to_fp32_row((const uint16_t*)vx, y, k); break;
    case ORC_Q4_0: {
        const blk_q4_0* x = (const blk_q4_0*)vx;
        for (int b = 0; b < k / 32; ++b) {
            const float d = orc_fp16_to_fp32(x[b].d);
            for (int j = 0; j < 16; ++j) {
                y[b * 32 + j] = (float)((int32_t)(x[b].qs[j] & 0x0Fu) - 8) * d;
                y[b * 32 + j + 16] = (float)((int32_t)(x[b].qs[j] >> 4) - 8) * d;
            }
        }
        break;
    }
    case ORC_Q8_0: {
        const blk_q8_0* x = (const blk_q8_0*)vx;
        for (int b = 0; b < k / 32; ++b) {
            const float d = orc_fp16_to_fp32(x[b].d);
            for (int j = 0; j < 32; ++j) y[b * 32 + j] = (float)x[b].qs[j] * d;
        }
        break;
    }
    case ORC_Q4_K: {
        const blk_q4_k* x = (const blk_q4_k*)vx;
        for (int b = 0; b < k / 256; ++b) {
            uint8_t sc[8], m[8];
            q4k_scale_min(x[b].scales, sc, m);
            const float d = orc_fp16_to_fp32(x[b].d), dmin = orc_fp16_to_fp32(x[b].dmin);
            for (int e = 0; e < 256; ++e) {
                const int j = e >> 5;
                const float ds = d * (float)sc[j];
                const float dm = dmin * (float)m[j];
                y[b * 256 + e] = ds * (float)q4k_q(&x[b], e) - dm;
            }
        }
        break;
    }
    case ORC_Q6_K: {
        const blk_q6_k* x = (const blk_q6_k*)vx;
        for (int b = 0; b < k / 256; ++b) {
            const float d = orc_fp16_to_fp32(x[b].d);
            for (int e = 0; e < 256; ++e) {
                const float ds = d * (float)x[b].scales[e >> 4];
                y[b * 256 + e] = ds * (float)q6k_q(&x[b], e);
            }
        }
        break;
    }
    default: memset(y, 0, (size_t)k * 4); break;
    }
}

/* ------------------------------------------------------------------------ */
/* Elementwise ops                                                           */
/* ------------------------------------------------------------------------ */

/* Follows ref_rmsnorm_f32, Singularity/tests/test_and_bench_a5.cpp:247-258. */
void orc_rmsnorm(const float* x, const float* w, float* out, int n, float eps) {
    volatile float ss = 0.0f;
    for (int i = 0; i < n; ++i) ss = ss + x[i] * x[i];
    const float mean_sq = (ss / (float)n) + eps;
    const float inv_rms = 1.0f / sqrtf(mean_sq);
    for (int i = 0; i < n; ++i) out[i] = (x[i] * inv_rms) * w[i];
}

/* RMSNorm as ggml's CPU backend computes it (llama.cpp
 * ggml_compute_forward_rms_norm_f32, version unpinned, not vendored): the
 * squares are rounded to fp32 and summed in double, mean = (float)(sum / n),
 * scale = 1/sqrtf(mean + eps), out = (x·scale)·w (the weight is a separate
 * ggml_mul).  The double sum makes the result independent of summation
 * order, so a parallel reduction reproduces it bit for bit. */
void orc_rmsnorm_ggml(const float* x, const float* w, float* out, int n, float eps) {
    double sum = 0.0;
    for (int i = 0; i < n; ++i) sum += (double)(x[i] * x[i]);
    const float mean = (float)(sum / (double)n);
    const float scale = 1.0f / sqrtf(mean + eps);
    for (int i = 0; i < n; ++i) out[i] = (x[i] * scale) * w[i];
}

/* Follows ref_softmax_f32, Singularity/tests/test_and_bench_a5.cpp:260-278. */
void orc_softmax(const float* x, float* out, int n) {
    float max_val = x[0];
    for (int i = 1; i < n; ++i)
        if (x[i] > max_val) max_val = x[i];
    float sum = 0.0f;
    for (int i = 0; i < n; ++i) {
        const float e = expf(x[i] - max_val);
        out[i] = e;
        sum += e;
    }
    const float inv_sum = 1.0f / sum;
    for (int i = 0; i < n; ++i) out[i] *= inv_sum;
}

/* Follows ref_rope_f32, Singularity/tests/test_and_bench_a5.cpp:280-293
 * (adjacent pairs, GGUF "normal" rope mode used for llama). */
void orc_rope_pairs(float* x, const float* cos_sin, int head_dim, int n_heads) {
    for (int h = 0; h < n_heads; ++h) {
        float* xh = x + h * head_dim;
        for (int i = 0; i < head_dim; i += 2) {
            const float x0 = xh[i], x1 = xh[i + 1];
            const float c = cos_sin[i], s = cos_sin[i + 1];
            xh[i] = x0 * c - x1 * s;
            xh[i + 1] = x0 * s + x1 * c;
        }
    }
}

/* singularity_silu_mul_f32_a5 semantics (prototype
 * Singularity/src/asm/singularity_asm_kernels.h:120-124, call
 * Singularity/src/core/cortex_a5_engine.cpp:1277): hb = silu(hb)·hb2, with
 * silu(x) = x / (1 + exp(−x)). */
void orc_silu_mul(float* hb, const float* hb2, int n) {
    for (int i = 0; i < n; ++i) {
        const float x = hb[i];
        const float s = x / (1.0f + expf(-x));
        hb[i] = s * hb2[i];
    }
}

/* Standard θ^(−2i/hd) table; Singularity's Qwen2 branch
 * (Singularity/src/core/cortex_a5_engine.cpp:777-786) uses this frequency
 * formula; its non-Qwen branch (:787-796) ignores rope_freq_base and is not
 * followed. */
void orc_rope_table(float theta, int head_dim, int p0, int n_pos, float* out) {
    for (int p = 0; p < n_pos; ++p) {
        for (int i = 0; i < head_dim / 2; ++i) {
            const double freq = pow((double)theta, -2.0 * (double)i / (double)head_dim);
            const double ang = (double)(p0 + p) * freq;
            out[(size_t)p * head_dim + 2 * i] = (float)cos(ang);
            out[(size_t)p * head_dim + 2 * i + 1] = (float)sin(ang);
        }
    }
}

/* ------------------------------------------------------------------------ */
/* Device-order arithmetic                                                   */
/* The same operations as above evaluated in the GPU kernels' order, so the  */
/* model forward can be checked bit for bit.  Each is checked against its    */
/* reference-order counterpart within tolerance by the tests.                */
/* ------------------------------------------------------------------------ */

/* exp(x): Cody-Waite reduction x = n·ln2 + r, degree-7 Taylor polynomial of
 * e^r by Horner's rule, scaling by 2^n from exponent bits; one rounded
 * operation per step (built with -ffp-contract=off). */
float orc_expf_dev(float x) {
    if (!(x == x)) return x;
    if (x > 88.7228394f) return INFINITY;
    if (x < -103.972084f) return 0.0f;
    const float t = x * 1.44269502f;
    const float n = (t + 12582912.0f) - 12582912.0f;
    float r = x - n * 0.693145751953125f;
    r = r - n * 1.42860677e-06f;
    float p = 1.98412698e-04f;
    p = p * r + 1.38888889e-03f;
    p = p * r + 8.33333333e-03f;
    p = p * r + 4.16666667e-02f;
    p = p * r + 1.66666667e-01f;
    p = p * r + 0.5f;
    p = p * r + 1.0f;
    p = p * r + 1.0f;
    int ni = (int)n;
    float s2 = 1.0f;
    if (ni > 127) {
        ni -= 1;
        s2 = 2.0f;
    } else if (ni < -126) {
        ni += 64;
        s2 = 5.42101086e-20f;
    }
    uint32_t bits = (uint32_t)(ni + 127) << 23;
    float s1;
    memcpy(&s1, &bits, 4);
    return (p * s1) * s2;
}

void orc_silu_mul_dev(float* hb, const float* hb2, int n) {
    for (int i = 0; i < n; ++i) {
        const float x = hb[i];
        hb[i] = (x / (1.0f + orc_expf_dev(-x))) * hb2[i];
    }
}

/* ---- tiled GEMV order ------------------------------------------------------
 * The tile GEMV kernels (dp4a for small batches, int8 mma for larger ones)
 * share one evaluation order per (row, token), independent of the batch:
 *   units u = 32-weight blocks (Q4_0, Q8_0) or 256-weight super-blocks
 *   (Q4_K, Q6_K), nu per row; S = orc_tile_splits() ranges of L = ceil(nu/S)
 *   units, R_w = [w·L, min((w+1)·L, nu)); inside R_w four partial sums a_q
 *   take the units with u mod 4 == q in increasing u; the range's sum is
 *   (a_0 + a_1) + (a_2 + a_3); the row's value is ((S_0 + S_1) + S_2) + ...
 * A unit adds its exact integer dot scaled as the reference does:
 *   Q4_0/Q8_0: acc + (d_w·d_x)·isum;  Q6_K: acc + (d_w·d_x)·isum;
 *   Q4_K: (acc + (d·d_x)·isum) − (dmin·d_x)·msum. */
int orc_tile_splits(int wtype, int k) {
    const int nu = (wtype == ORC_Q4_K || wtype == ORC_Q6_K) ? k / 256 : k / 32;
    int s = 1;
    while (s < 8 && 2 * s * 4 <= nu) s *= 2;
    return s;
}

static float tile_unit(int wtype, const uint8_t* wrow, const uint8_t* xrow, int u, float acc) {
    switch (wtype) {
    case ORC_Q4_0: {
        const blk_q4_0* x = (const blk_q4_0*)wrow + u;
        const blk_q8_0* y = (const blk_q8_0*)xrow + u;
        int32_t s;
        orc_block_dots_q4_0_q8_0(32, x, y, &s);
        return acc + (orc_fp16_to_fp32(x->d) * orc_fp16_to_fp32(y->d)) * (float)s;
    }
    case ORC_Q8_0: {
        const blk_q8_0* x = (const blk_q8_0*)wrow + u;
        const blk_q8_0* y = (const blk_q8_0*)xrow + u;
        int32_t s;
        orc_block_dots_q8_0_q8_0(32, x, y, &s);
        return acc + (orc_fp16_to_fp32(x->d) * orc_fp16_to_fp32(y->d)) * (float)s;
    }
    case ORC_Q4_K: {
        const blk_q4_k* x = (const blk_q4_k*)wrow + u;
        const blk_q8_k* y = (const blk_q8_k*)xrow + u;
        int32_t is, ms;
        orc_block_dots_q4_k_q8_k(256, x, y, &is, &ms);
        acc = acc + (orc_fp16_to_fp32(x->d) * y->d) * (float)is;
        return acc - (orc_fp16_to_fp32(x->dmin) * y->d) * (float)ms;
    }
    default: {
        const blk_q6_k* x = (const blk_q6_k*)wrow + u;
        const blk_q8_k* y = (const blk_q8_k*)xrow + u;
        int32_t is;
        orc_block_dots_q6_k_q8_k(256, x, y, &is);
        return acc + (orc_fp16_to_fp32(x->d) * y->d) * (float)is;
    }
    }
}

float orc_tile_row_dot(int wtype, const void* wrow, int k, const void* xq) {
    const int nu = (wtype == ORC_Q4_K || wtype == ORC_Q6_K) ? k / 256 : k / 32;
    const int S = orc_tile_splits(wtype, k);
    const int L = (nu + S - 1) / S;
    float total = 0.0f;
    for (int w = 0; w < S; ++w) {
        const int u0 = w * L < nu ? w * L : nu, u1 = (w + 1) * L < nu ? (w + 1) * L : nu;
        float a[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        for (int u = u0; u < u1; ++u) a[u & 3] = tile_unit(wtype, (const uint8_t*)wrow, (const uint8_t*)xq, u, a[u & 3]);
        const float sw = (a[0] + a[1]) + (a[2] + a[3]);
        total = w == 0 ? sw : total + sw;
    }
    return total;
}

typedef struct {
    int wtype, k;
    const uint8_t* w;
    size_t row_bytes;
    const void* xq;
    float* y;
    int64_t r0, r1;
} mmd_job;

static void* mmd_worker(void* arg) {
    const mmd_job* j = (const mmd_job*)arg;
    for (int64_t r = j->r0; r < j->r1; ++r)
        j->y[r] = orc_tile_row_dot(j->wtype, j->w + (size_t)r * j->row_bytes, j->k, j->xq);
    return NULL;
}

void orc_matmul_dev(int wtype, const void* w, int64_t n_rows, int k, const void* xq, float* y, int swiglu,
                    int n_threads) {
    orc_matmul_dev_strided(wtype, w, n_rows, orc_row_bytes(wtype, k), k, xq, y, swiglu, n_threads);
}

void orc_matmul_dev_strided(int wtype, const void* w, int64_t n_rows, size_t row_stride, int k, const void* xq,
                            float* y, int swiglu, int n_threads) {
    if (n_threads < 1) n_threads = 1;
    if (n_threads > 256) n_threads = 256;
    if ((int64_t)n_threads > n_rows) n_threads = (int)n_rows;
    mmd_job jobs[256];
    pthread_t th[256];
    for (int t = 0; t < n_threads; ++t) {
        jobs[t].wtype = wtype;
        jobs[t].k = k;
        jobs[t].w = (const uint8_t*)w;
        jobs[t].row_bytes = row_stride;
        jobs[t].xq = xq;
        jobs[t].y = y;
        jobs[t].r0 = n_rows * t / n_threads;
        jobs[t].r1 = n_rows * (t + 1) / n_threads;
    }
    for (int t = 1; t < n_threads; ++t) pthread_create(&th[t], NULL, mmd_worker, &jobs[t]);
    mmd_worker(&jobs[0]);
    for (int t = 1; t < n_threads; ++t) pthread_join(th[t], NULL);
}

/* Split-K decode attention in the device kernels' order: positions in chunks
 * of 128; per chunk and head, the score of a position is eight fmaf chains
 * over hd/8 dims each (chain i over dims [i·B, i·B + B) then
 * [hd/2 + i·B, hd/2 + i·B + B), B = hd/16), combined by the 8-lane
 * butterfly (xor 4, 2, 1), times 1/sqrt(hd); m = the
 * chunk max; e = exp_dev(s − m); the chunk sum is ((W0 + W1) + W2) + W3, W_w
 * the 32-lane butterfly (xor 16..1) over positions 32w..32w+31 (0 past the
 * end); P·V per dim keeps four sums a_r of e·v by fmaf over the positions
 * i ≡ r (mod 4) in order, then (a0 + a1) + (a2 + a3); chunks combined with
 * exp_dev(m_s − M). */
static float butterfly(float* v, int n) {
    float t[32];
    for (int o = n / 2; o > 0; o >>= 1) {
        for (int l = 0; l < n; ++l) t[l] = v[l] + v[l ^ o];
        for (int l = 0; l < n; ++l) v[l] = t[l];
    }
    return v[0];
}

void orc_attn_decode_dev(const float* q, const uint16_t* kc, const uint16_t* vc, int64_t kv_stride, int n_pos,
                         int n_heads, int n_kv_heads, int hd, float* out) {
    const int G = n_heads / n_kv_heads;
    const int P = 128, B = hd / 16;
    const float scale = 1.0f / sqrtf((float)hd);
    const int n_split = (n_pos + P - 1) / P;
    float* sc = (float*)malloc(sizeof(float) * P);
    float* ms = (float*)malloc(sizeof(float) * (size_t)n_split);
    float* ls = (float*)malloc(sizeof(float) * (size_t)n_split);
    float* os = (float*)malloc(sizeof(float) * (size_t)n_split * hd);
    float* kt = (float*)malloc(sizeof(float) * (size_t)hd);
    for (int h = 0; h < n_heads; ++h) {
        const int kvh = h / G;
        const float* qh = q + (size_t)h * hd;
        for (int s = 0; s < n_split; ++s) {
            const int t0 = s * P, n = (n_pos - t0 < P) ? n_pos - t0 : P;
            float m = -FLT_MAX;
            for (int i = 0; i < n; ++i) {
                orc_fp16_to_fp32_row(kc + (size_t)(t0 + i) * kv_stride + (size_t)kvh * hd, kt, hd);
                /* lane l: dims [B*l, B*l+B) then [hd/2 + B*l, hd/2 + B*l + B) */
                float a[8];
                for (int l = 0; l < 8; ++l) {
                    a[l] = 0.0f;
                    for (int j = 0; j < 2; ++j)
                        for (int d = j * (hd / 2) + B * l; d < j * (hd / 2) + B * (l + 1); ++d)
                            a[l] = fmaf(qh[d], kt[d], a[l]);
                }
                sc[i] = butterfly(a, 8) * scale;
                m = fmaxf(m, sc[i]);
            }
            float W[4];
            for (int w = 0; w < 4; ++w) {
                float v[32];
                for (int l = 0; l < 32; ++l) {
                    const int i = 32 * w + l;
                    v[l] = i < n ? orc_expf_dev(sc[i] - m) : 0.0f;
                }
                W[w] = butterfly(v, 32);
            }
            for (int i = 0; i < n; ++i) sc[i] = orc_expf_dev(sc[i] - m);
            ms[s] = m;
            ls[s] = ((W[0] + W[1]) + W[2]) + W[3];
            for (int d = 0; d < hd; ++d) {
                float a[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                for (int i = 0; i < n; ++i) {
                    const float v = orc_fp16_to_fp32(vc[(size_t)(t0 + i) * kv_stride + (size_t)kvh * hd + d]);
                    a[i & 3] = fmaf(sc[i], v, a[i & 3]);
                }
                os[(size_t)s * hd + d] = (a[0] + a[1]) + (a[2] + a[3]);
            }
        }
        float M = -FLT_MAX;
        for (int s = 0; s < n_split; ++s) M = fmaxf(M, ms[s]);
        float L = 0.0f;
        for (int s = 0; s < n_split; ++s)
            if (ls[s] > 0.0f) L = L + orc_expf_dev(ms[s] - M) * ls[s];
        const float invL = 1.0f / L;
        for (int d = 0; d < hd; ++d) {
            float v = 0.0f;
            for (int s = 0; s < n_split; ++s)
                if (ls[s] > 0.0f) v = v + orc_expf_dev(ms[s] - M) * os[(size_t)s * hd + d];
            out[(size_t)h * hd + d] = v * invL;
        }
    }
    free(sc); free(ms); free(ls); free(os); free(kt);
}

/* ------------------------------------------------------------------------ */
/* Quantized matmul (row-parallel)                                           */
/* ------------------------------------------------------------------------ */

typedef struct {
    int wtype;
    const uint8_t* w;
    size_t row_bytes;
    int k;
    const void* xq;
    float* y;
    int64_t r0, r1;
} mm_job;

/* Follows matmul_quantized, Singularity/src/core/cortex_a5_engine.cpp:997-1027:
 * one vec_dot per output row. */
static void* mm_worker(void* arg) {
    const mm_job* j = (const mm_job*)arg;
    for (int64_t r = j->r0; r < j->r1; ++r) {
        const void* row = j->w + (size_t)r * j->row_bytes;
        float v = 0.0f;
        switch (j->wtype) {
        case ORC_Q4_0: v = orc_vec_dot_q4_0_q8_0(j->k, row, j->xq); break;
        case ORC_Q8_0: v = orc_vec_dot_q8_0_q8_0(j->k, row, j->xq); break;
        case ORC_Q4_K: v = orc_vec_dot_q4_k_q8_k(j->k, row, j->xq); break;
        case ORC_Q6_K: v = orc_vec_dot_q6_k_q8_k(j->k, row, j->xq); break;
        default: break;
        }
        j->y[r] = v;
    }
    return NULL;
}

void orc_matmul(int wtype, const void* w, int64_t n_rows, int k, const void* xq, float* y, int n_threads) {
    orc_matmul_strided(wtype, w, n_rows, orc_row_bytes(wtype, k), k, xq, y, n_threads);
}

/* orc_matmul over rows row_stride bytes apart (a column slice of a wider
 * matrix: its rows start row_stride bytes apart and hold k values). */
void orc_matmul_strided(int wtype, const void* w, int64_t n_rows, size_t row_stride, int k, const void* xq, float* y,
                        int n_threads) {
    if (n_threads < 1) n_threads = 1;
    if (n_threads > 256) n_threads = 256;
    if ((int64_t)n_threads > n_rows) n_threads = (int)n_rows;
    mm_job jobs[256];
    pthread_t th[256];
    const size_t rb = row_stride;
    for (int t = 0; t < n_threads; ++t) {
        jobs[t].wtype = wtype;
        jobs[t].w = (const uint8_t*)w;
        jobs[t].row_bytes = rb;
        jobs[t].k = k;
        jobs[t].xq = xq;
        jobs[t].y = y;
        jobs[t].r0 = n_rows * t / n_threads;
        jobs[t].r1 = n_rows * (t + 1) / n_threads;
    }
    if (n_threads == 1) {
        mm_worker(&jobs[0]);
        return;
    }
    for (int t = 1; t < n_threads; ++t) pthread_create(&th[t], NULL, mm_worker, &jobs[t]);
    mm_worker(&jobs[0]);
    for (int t = 1; t < n_threads; ++t) pthread_join(th[t], NULL);
}

/* ------------------------------------------------------------------------ */
/* Attention and KV shift                                                    */
/* ------------------------------------------------------------------------ */

/* Follows the GQA attention loop, Singularity/src/core/cortex_a5_engine.cpp:1205-1254:
 * score_t = (Σ_i q_i·k_t,i)·(1/√hd) summed in order; softmax over t;
 * out_i = Σ_t a_t·v_t,i summed in order.  q-head h reads kv head
 * min(h / (n_heads/n_kv), n_kv−1) (:1061-1064, :1250-1253). */
void orc_attn_decode(const float* q, const uint16_t* kc, const uint16_t* vc, int64_t kv_stride,
                     int n_pos, int n_heads, int n_kv_heads, int hd, float* out) {
    int gqa = 1;
    while (gqa * n_kv_heads < n_heads) ++gqa;
    const float att_scale = 1.0f / sqrtf((float)hd);
    float* att = (float*)malloc(sizeof(float) * (size_t)(n_pos > 0 ? n_pos : 1));
    float* tmp = (float*)malloc(sizeof(float) * (size_t)hd);
    for (int h = 0; h < n_heads; ++h) {
        int kvh = h / gqa;
        if (kvh > n_kv_heads - 1) kvh = n_kv_heads - 1;
        const float* qh = q + (size_t)h * hd;
        for (int t = 0; t < n_pos; ++t) {
            orc_fp16_to_fp32_row(kc + (size_t)t * kv_stride + (size_t)kvh * hd, tmp, hd);
            float score = 0.0f;
            for (int i = 0; i < hd; ++i) score += qh[i] * tmp[i];
            att[t] = score * att_scale;
        }
        if (n_pos > 0) orc_softmax(att, att, n_pos);
        float* oh = out + (size_t)h * hd;
        for (int i = 0; i < hd; ++i) oh[i] = 0.0f;
        for (int t = 0; t < n_pos; ++t) {
            orc_fp16_to_fp32_row(vc + (size_t)t * kv_stride + (size_t)kvh * hd, tmp, hd);
            const float a = att[t];
            for (int i = 0; i < hd; ++i) oh[i] += a * tmp[i];
        }
    }
    free(tmp);
    free(att);
}

/* KV shift (Milda/src/engine.cpp:1642-1675: llama_memory_seq_rm then
 * llama_memory_seq_add(−n_discard); the cache re-applies RoPE to the kept
 * K by the position delta).  Each kept K row is rotated by the delta angle:
 * fp16 → fp32, x0·c − x1·s / x0·s + x1·c, RNE → fp16.  V is unchanged. */
void orc_kv_shift_k(uint16_t* kc, int64_t kv_stride, int n_pos, int n_kv_heads, int hd,
                    int delta, float theta) {
    float* cs = (float*)malloc(sizeof(float) * (size_t)hd);
    orc_rope_table(theta, hd, delta, 1, cs);
    for (int t = 0; t < n_pos; ++t) {
        for (int h = 0; h < n_kv_heads; ++h) {
            uint16_t* row = kc + (size_t)t * kv_stride + (size_t)h * hd;
            for (int i = 0; i < hd; i += 2) {
                const float x0 = orc_fp16_to_fp32(row[i]);
                const float x1 = orc_fp16_to_fp32(row[i + 1]);
                const float c = cs[i], s = cs[i + 1];
                row[i] = orc_fp32_to_fp16(x0 * c - x1 * s);
                row[i + 1] = orc_fp32_to_fp16(x0 * s + x1 * c);
            }
        }
    }
    free(cs);
}

/* ------------------------------------------------------------------------ */
/* Quantized KV cache (llama.cpp cache types)                                */
/* ------------------------------------------------------------------------ */

/* Milda asks llama.cpp for a Q8_0 K and V cache by default
 * (Milda/include/milda/engine.hpp:85-86, mapped at Milda/src/engine.cpp:74-87
 * and set at :1195-1196) with flash attention on (engine.hpp:91,
 * engine.cpp:1197).  llama.cpp (absent from the reference tree) stores each
 * cached row with its type's quantizer, pairs a quantized K row with the
 * query quantized to the K type's dot type (Q8_0 for Q8_0 K) and scores with
 * that type's block dot, and dequantizes V rows (d·q) before the weighted
 * sum.  Restated here with the reference's own ops: Q8_0 quantization and
 * the Q8_0·Q8_0 dot of Singularity/tests/test_and_bench_a5.cpp:205-245, the
 * Q8_0 dequantization of Singularity/src/core/cortex_a5_engine.cpp:1090-1105,
 * and the softmax and order of the fp16 attention above
 * (cortex_a5_engine.cpp:1205-1254). */

static size_t kv_row_bytes(int type, int hd) { return orc_row_bytes(type, hd); }

/* ggml's quantize_row_q4_0_ref (llama.cpp's Q4_0 cache type; the same
 * formula as the library's GGUF weight quantizer, pinned to gguf-py): the
 * value of largest magnitude (first such), d = max/−8, id = 1/d, code =
 * min(15, trunc(x·id + 8.5)), element j low nibble and j+16 high nibble of
 * byte j. */
void orc_quantize_row_q4_0(const float* x, void* vy, int k) {
    blk_q4_0* y = (blk_q4_0*)vy;
    for (int b = 0; b < k / 32; ++b) {
        const float* xb = x + b * 32;
        float amax = 0.0f, max = 0.0f;
        for (int j = 0; j < 32; ++j) {
            const float v = xb[j];
            const float av = v < 0.0f ? -v : v;
            if (amax < av) {
                amax = av;
                max = v;
            }
        }
        const float d = max / -8.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        y[b].d = orc_fp32_to_fp16(d);
        for (int j = 0; j < 16; ++j) {
            const float x0 = xb[j] * id, x1 = xb[16 + j] * id;
            int q0 = (int)(int8_t)(x0 + 8.5f), q1 = (int)(int8_t)(x1 + 8.5f);
            q0 = q0 < 15 ? q0 : 15;
            q1 = q1 < 15 ? q1 : 15;
            y[b].qs[j] = (uint8_t)(q0 | (q1 << 4));
        }
    }
}

void orc_kv_store_row(int type, const float* x, void* row, int n) {
    if (type == ORC_Q8_0) orc_quantize_row_q8_0(x, row, n);
    else if (type == ORC_Q4_0) orc_quantize_row_q4_0(x, row, n);
    else orc_fp32_to_fp16_row(x, (uint16_t*)row, n);
}

void orc_kv_store_rows(int type, const float* x, void* rows, int64_t n_rows, int n) {
    const size_t rb = kv_row_bytes(type, n);
    for (int64_t r = 0; r < n_rows; ++r) orc_kv_store_row(type, x + (size_t)r * n, (uint8_t*)rows + (size_t)r * rb, n);
}

void orc_attn_decode_typed(const float* q, const void* kc, int ktype, size_t k_stride, const void* vc,
                           int vtype, size_t v_stride, int n_pos, int n_heads, int n_kv_heads, int hd,
                           float* out) {
    int gqa = 1;
    while (gqa * n_kv_heads < n_heads) ++gqa;
    const float att_scale = 1.0f / sqrtf((float)hd);
    const size_t krb = kv_row_bytes(ktype, hd), vrb = kv_row_bytes(vtype, hd);
    const uint8_t* kb = (const uint8_t*)kc;
    const uint8_t* vb = (const uint8_t*)vc;
    float* att = (float*)malloc(sizeof(float) * (size_t)(n_pos > 0 ? n_pos : 1));
    float* tmp = (float*)malloc(sizeof(float) * (size_t)hd);
    blk_q8_0* qq = (blk_q8_0*)malloc(sizeof(blk_q8_0) * (size_t)(hd / 32));
    for (int h = 0; h < n_heads; ++h) {
        int kvh = h / gqa;
        if (kvh > n_kv_heads - 1) kvh = n_kv_heads - 1;
        const float* qh = q + (size_t)h * hd;
        if (ktype == ORC_Q8_0 || ktype == ORC_Q4_0) orc_quantize_row_q8_0(qh, qq, hd);
        for (int t = 0; t < n_pos; ++t) {
            const uint8_t* krow = kb + (size_t)t * k_stride + (size_t)kvh * krb;
            float score = 0.0f;
            if (ktype == ORC_Q8_0) {
                score = orc_vec_dot_q8_0_q8_0(hd, krow, qq);
            } else if (ktype == ORC_Q4_0) {
                score = orc_vec_dot_q4_0_q8_0(hd, krow, qq);
            } else {
                orc_fp16_to_fp32_row((const uint16_t*)krow, tmp, hd);
                for (int i = 0; i < hd; ++i) score += qh[i] * tmp[i];
            }
            att[t] = score * att_scale;
        }
        if (n_pos > 0) orc_softmax(att, att, n_pos);
        float* oh = out + (size_t)h * hd;
        for (int i = 0; i < hd; ++i) oh[i] = 0.0f;
        for (int t = 0; t < n_pos; ++t) {
            orc_dequantize_row(vtype, vb + (size_t)t * v_stride + (size_t)kvh * vrb, tmp, hd);
            const float a = att[t];
            for (int i = 0; i < hd; ++i) oh[i] += a * tmp[i];
        }
    }
    free(qq);
    free(tmp);
    free(att);
}

/* The KV shift's K re-rotation on a typed cache: each kept row is
 * dequantized, rotated by the delta angle as in orc_kv_shift_k and stored
 * back with the type's quantizer (llama.cpp rotates a quantized K through an
 * fp32 copy and writes it back through the type's quantizer). */
void orc_kv_shift_k_typed(void* kc, int ktype, size_t k_stride, int n_pos, int n_kv_heads, int hd, int delta,
                          float theta) {
    float* cs = (float*)malloc(sizeof(float) * (size_t)hd);
    float* x = (float*)malloc(sizeof(float) * (size_t)hd);
    float* y = (float*)malloc(sizeof(float) * (size_t)hd);
    const size_t rb = kv_row_bytes(ktype, hd);
    orc_rope_table(theta, hd, delta, 1, cs);
    for (int t = 0; t < n_pos; ++t) {
        for (int h = 0; h < n_kv_heads; ++h) {
            uint8_t* row = (uint8_t*)kc + (size_t)t * k_stride + (size_t)h * rb;
            orc_dequantize_row(ktype, row, x, hd);
            for (int i = 0; i < hd; i += 2) {
                const float c = cs[i], s = cs[i + 1];
                y[i] = x[i] * c - x[i + 1] * s;
                y[i + 1] = x[i] * s + x[i + 1] * c;
            }
            orc_kv_store_row(ktype, y, row, hd);
        }
    }
    free(y);
    free(x);
    free(cs);
}
