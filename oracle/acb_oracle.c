/*
 * acb_oracle.c -- CPU oracle (test infrastructure only; see acb_oracle.h).
 *
 * Each function names the reference call site whose ggml-CPU arithmetic it restates.
 * Built with -O2 -ffp-contract=off so that no multiply-add is fused behind our back.
 */
#include "acb_oracle.h"
#include "../hbd-acestep.cpp_b200/csrc/acb_exp.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#    include <omp.h>
#endif

/* ------------------------------------------------------------------------------------------ */
/* scalar conversions (IEEE binary16 / bfloat16; ggml_fp16_t and ggml_bf16_t storage)         */
/* ------------------------------------------------------------------------------------------ */

static inline uint32_t f2u(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    return u;
}

static inline float u2f(uint32_t u) {
    float f;
    memcpy(&f, &u, 4);
    return f;
}

float orc_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t) (h & 0x8000) << 16;
    uint32_t exp  = (h >> 10) & 0x1f;
    uint32_t man  = h & 0x3ff;
    if (exp == 0) {
        if (man == 0) {
            return u2f(sign);
        }
        /* subnormal: value = man * 2^-24 (exact in float) */
        float v = (float) man * 5.9604644775390625e-8f;
        return sign ? -v : v;
    }
    if (exp == 31) {
        return u2f(sign | 0x7f800000u | (man << 13));
    }
    return u2f(sign | ((exp + 112) << 23) | (man << 13));
}

uint16_t orc_f32_to_f16(float f) {
    uint32_t x    = f2u(f);
    uint32_t sign = (x >> 16) & 0x8000;
    uint32_t ax   = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) { /* inf / nan */
        return (uint16_t) (sign | 0x7c00 | (ax > 0x7f800000u ? 0x200 : 0));
    }
    if (ax >= 0x477ff000u) { /* rounds to >= 65520 -> inf */
        return (uint16_t) (sign | 0x7c00);
    }
    if (ax < 0x38800000u) { /* below the smallest normal half: subnormal or zero */
        /* value / 2^-24 rounded to nearest even integer */
        float    v = u2f(ax) * 16777216.0f; /* exact scaling by 2^24 */
        /* round half to even via the 2^23 trick (v < 1024) */
        float    r = (v + 8388608.0f) - 8388608.0f;
        uint32_t m = (uint32_t) r;
        return (uint16_t) (sign | m); /* m == 1024 carries into the exponent field correctly */
    }
    /* normal: rebias exponent, round mantissa 23 -> 10 bits, nearest even */
    uint32_t e    = ((ax >> 23) - 112) << 10;
    uint32_t man  = ax & 0x7fffffu;
    uint32_t h    = e | (man >> 13);
    uint32_t rem  = man & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) {
        h += 1; /* may carry into the exponent: still correct */
    }
    return (uint16_t) (sign | h);
}

float orc_bf16_to_f32(uint16_t h) {
    return u2f((uint32_t) h << 16);
}

uint16_t orc_f32_to_bf16(float f) {
    uint32_t u = f2u(f);
    if ((u & 0x7fffffffu) > 0x7f800000u) { /* nan: keep quiet */
        return (uint16_t) ((u >> 16) | 64);
    }
    return (uint16_t) ((u + (0x7fff + ((u >> 16) & 1))) >> 16);
}

/* ------------------------------------------------------------------------------------------ */
/* block formats (public GGUF layouts)                                                         */
/*   Q8_0: f16 d, int8 qs[32]                                         34 B / 32               */
/*   Q4_K: f16 d, f16 dmin, u8 scales[12] (6-bit packed), u8 qs[128]  144 B / 256             */
/*   Q6_K: u8 ql[128], u8 qh[64], int8 scales[16], f16 d              210 B / 256             */
/*   Q8_K: f32 d, int8 qs[256], int16 bsums[16]                       292 B / 256             */
/* ------------------------------------------------------------------------------------------ */

int64_t orc_block_elems(int type) {
    switch (type) {
        case ORC_Q8_0:
            return 32;
        case ORC_Q4_K:
        case ORC_Q6_K:
        case ORC_Q8_K:
            return 256;
        case ORC_F32:
        case ORC_F16:
        case ORC_BF16:
            return 1;
        default:
            return 0;
    }
}

int64_t orc_block_bytes(int type) {
    switch (type) {
        case ORC_Q8_0:
            return 34;
        case ORC_Q4_K:
            return 144;
        case ORC_Q6_K:
            return 210;
        case ORC_Q8_K:
            return 292;
        case ORC_F32:
            return 4;
        case ORC_F16:
        case ORC_BF16:
            return 2;
        default:
            return 0;
    }
}

int64_t orc_row_bytes(int type, int64_t n) {
    int64_t be = orc_block_elems(type);
    if (be <= 0 || n % be != 0) {
        return -1;
    }
    return n / be * orc_block_bytes(type);
}

static inline uint16_t rd16(const uint8_t * p) {
    return (uint16_t) (p[0] | (p[1] << 8));
}

/* Q4_K 6-bit scale/min unpack for sub-block j (0..7) of the 12-byte table. */
static inline void q4k_scale_min(int j, const uint8_t * q, int * sc, int * m) {
    if (j < 4) {
        *sc = q[j] & 63;
        *m  = q[j + 4] & 63;
    } else {
        *sc = (q[j + 4] & 0x0f) | ((q[j - 4] >> 6) << 4);
        *m  = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

/* Q6_K element j (0..255) of a block as a signed 6-bit value in [-32, 31]. */
static inline int q6k_value(const uint8_t * blk, int j) {
    const uint8_t * ql   = blk;
    const uint8_t * qh   = blk + 128;
    int             half = j >> 7, c = (j >> 5) & 3, l = j & 31;
    int             lo   = (c & 1) ? ql[half * 64 + 32 + l] : ql[half * 64 + l];
    lo                   = (c & 2) ? (lo >> 4) : (lo & 0x0f);
    int hi               = (qh[half * 32 + l] >> (2 * c)) & 3;
    return (lo | (hi << 4)) - 32;
}

/* Q4_K element j (0..255): returns the 4-bit q and the sub-block index (0..7). */
static inline int q4k_value(const uint8_t * blk, int j, int * sub) {
    const uint8_t * qs = blk + 16;
    int             g = j >> 6, hi = (j >> 5) & 1, l = j & 31;
    *sub              = 2 * g + hi;
    uint8_t b         = qs[g * 32 + l];
    return hi ? (b >> 4) : (b & 0x0f);
}

int orc_dequant_row(int type, const void * src, float * dst, int64_t n) {
    const uint8_t * p = (const uint8_t *) src;
    if (orc_row_bytes(type, n) < 0) {
        return -1;
    }
    switch (type) {
        case ORC_F32:
            memcpy(dst, src, (size_t) n * 4);
            return 0;
        case ORC_F16:
            for (int64_t i = 0; i < n; i++) {
                dst[i] = orc_f16_to_f32(rd16(p + 2 * i));
            }
            return 0;
        case ORC_BF16:
            for (int64_t i = 0; i < n; i++) {
                dst[i] = orc_bf16_to_f32(rd16(p + 2 * i));
            }
            return 0;
        case ORC_Q8_0:
            /* element = d * q (one rounding; exact for |q| <= 127 and f16 d) */
            for (int64_t b = 0; b < n / 32; b++) {
                const uint8_t * blk = p + b * 34;
                float           d   = orc_f16_to_f32(rd16(blk));
                for (int j = 0; j < 32; j++) {
                    dst[b * 32 + j] = d * (float) (int8_t) blk[2 + j];
                }
            }
            return 0;
        case ORC_Q4_K:
            /* element = (d*sc)*q - (dmin*m): two products, then one subtraction */
            for (int64_t b = 0; b < n / 256; b++) {
                const uint8_t * blk  = p + b * 144;
                float           d    = orc_f16_to_f32(rd16(blk));
                float           dmin = orc_f16_to_f32(rd16(blk + 2));
                float           d1[8], m1[8];
                for (int s = 0; s < 8; s++) {
                    int sc, m;
                    q4k_scale_min(s, blk + 4, &sc, &m);
                    d1[s] = d * (float) sc;
                    m1[s] = dmin * (float) m;
                }
                for (int j = 0; j < 256; j++) {
                    int   sub;
                    int   q        = q4k_value(blk, j, &sub);
                    float prod     = d1[sub] * (float) q;
                    dst[b * 256 + j] = prod - m1[sub];
                }
            }
            return 0;
        case ORC_Q6_K:
            /* element = (d*sc)*q: the product d*sc first, then times q (rounds once more) */
            for (int64_t b = 0; b < n / 256; b++) {
                const uint8_t * blk = p + b * 210;
                const int8_t *  sc  = (const int8_t *) (blk + 192);
                float           d   = orc_f16_to_f32(rd16(blk + 208));
                for (int j = 0; j < 256; j++) {
                    float ds         = d * (float) sc[j >> 4];
                    dst[b * 256 + j] = ds * (float) q6k_value(blk, j);
                }
            }
            return 0;
        case ORC_Q8_K:
            for (int64_t b = 0; b < n / 256; b++) {
                const uint8_t * blk = p + b * 292;
                float           d;
                memcpy(&d, blk, 4);
                for (int j = 0; j < 256; j++) {
                    dst[b * 256 + j] = d * (float) (int8_t) blk[4 + j];
                }
            }
            return 0;
        default:
            return -1;
    }
}

/* Q8_0 activation quantizer: d = amax/127, id = 1/d, q = roundf(x*id) (half away from 0).
 * Same arithmetic as gguf-py Q8_0.quantize_blocks (quants.py:381-394). */
void orc_quantize_row_q8_0(const float * x, void * dst, int64_t n) {
    uint8_t * p = (uint8_t *) dst;
    for (int64_t b = 0; b < n / 32; b++) {
        const float * xb   = x + b * 32;
        float         amax = 0.0f;
        for (int j = 0; j < 32; j++) {
            float a = fabsf(xb[j]);
            if (a > amax) {
                amax = a;
            }
        }
        float    d  = amax / 127.0f;
        float    id = d != 0.0f ? 1.0f / d : 0.0f;
        uint16_t dh = orc_f32_to_f16(d);
        p[b * 34]     = (uint8_t) (dh & 0xff);
        p[b * 34 + 1] = (uint8_t) (dh >> 8);
        for (int j = 0; j < 32; j++) {
            float v              = xb[j] * id;
            p[b * 34 + 2 + j]    = (uint8_t) (int8_t) roundf(v);
        }
    }
}

/* round half to even for |v| < 2^22 (the float magic-number trick) */
static inline int nearest_int(float v) {
    float    t = v + 12582912.0f;
    uint32_t u = f2u(t);
    return (int) (u & 0x007fffff) - 0x00400000;
}

/* Q8_K activation quantizer (vec-dot type of Q4_K / Q6_K): per 256 block the signed value of
 * largest magnitude `max`, iscale = -127/max, q = min(127, nearest_int(iscale*x)),
 * d = 1/iscale, bsums = sums of 16-element groups. */
void orc_quantize_row_q8_K(const float * x, void * dst, int64_t n) {
    uint8_t * p = (uint8_t *) dst;
    for (int64_t b = 0; b < n / 256; b++) {
        const float * xb  = x + b * 256;
        uint8_t *     blk = p + b * 292;
        float         mx = 0.0f, amax = 0.0f;
        for (int j = 0; j < 256; j++) {
            float a = fabsf(xb[j]);
            if (a > amax) {
                amax = a;
                mx   = xb[j];
            }
        }
        int8_t * qs = (int8_t *) (blk + 4);
        int16_t  bs[16];
        if (amax == 0.0f) {
            float z = 0.0f;
            memcpy(blk, &z, 4);
            memset(qs, 0, 256);
            memset(bs, 0, sizeof(bs));
            memcpy(blk + 260, bs, 32);
            continue;
        }
        float iscale = -127.0f / mx;
        for (int j = 0; j < 256; j++) {
            int v = nearest_int(iscale * xb[j]);
            qs[j] = (int8_t) (v < 127 ? v : 127);
        }
        for (int g = 0; g < 16; g++) {
            int s = 0;
            for (int j = 0; j < 16; j++) {
                s += qs[g * 16 + j];
            }
            bs[g] = (int16_t) s;
        }
        memcpy(blk + 260, bs, 32);
        float d = 1.0f / iscale;
        memcpy(blk, &d, 4);
    }
}

/* Valid Q4_K blocks: per 32-element sub-block, scale = (max-min)/15 and min offset, both
 * encoded as 6-bit multiples of per-block f16 super-scales. */
void orc_quantize_row_q4_K(const float * x, void * dst, int64_t n) {
    uint8_t * p = (uint8_t *) dst;
    for (int64_t b = 0; b < n / 256; b++) {
        const float * xb  = x + b * 256;
        uint8_t *     blk = p + b * 144;
        float         scl[8], mns[8];
        float         max_scale = 0.0f, max_min = 0.0f;
        for (int s = 0; s < 8; s++) {
            float lo = xb[s * 32], hi = xb[s * 32];
            for (int j = 1; j < 32; j++) {
                float v = xb[s * 32 + j];
                lo      = v < lo ? v : lo;
                hi      = v > hi ? v : hi;
            }
            if (lo > 0.0f) {
                lo = 0.0f;
            }
            scl[s] = (hi - lo) / 15.0f;
            mns[s] = -lo;
            if (scl[s] > max_scale) {
                max_scale = scl[s];
            }
            if (mns[s] > max_min) {
                max_min = mns[s];
            }
        }
        float    d     = max_scale / 63.0f;
        float    dmin  = max_min / 63.0f;
        uint16_t dh    = orc_f32_to_f16(d);
        uint16_t dmh   = orc_f32_to_f16(dmin);
        float    dq    = orc_f16_to_f32(dh);
        float    dminq = orc_f16_to_f32(dmh);
        int      ls[8], lm[8];
        for (int s = 0; s < 8; s++) {
            int a = dq > 0.0f ? (int) lroundf(scl[s] / dq) : 0;
            int c = dminq > 0.0f ? (int) lroundf(mns[s] / dminq) : 0;
            ls[s] = a < 0 ? 0 : (a > 63 ? 63 : a);
            lm[s] = c < 0 ? 0 : (c > 63 ? 63 : c);
        }
        blk[0] = (uint8_t) (dh & 0xff);
        blk[1] = (uint8_t) (dh >> 8);
        blk[2] = (uint8_t) (dmh & 0xff);
        blk[3] = (uint8_t) (dmh >> 8);
        uint8_t * sc = blk + 4;
        for (int j = 0; j < 4; j++) {
            sc[j]     = (uint8_t) ((ls[j] & 63) | ((ls[j + 4] >> 4) << 6));
            sc[j + 4] = (uint8_t) ((lm[j] & 63) | ((lm[j + 4] >> 4) << 6));
            sc[j + 8] = (uint8_t) ((ls[j + 4] & 0x0f) | ((lm[j + 4] & 0x0f) << 4));
        }
        uint8_t * qs = blk + 16;
        memset(qs, 0, 128);
        for (int s = 0; s < 8; s++) {
            float ds = dq * (float) ls[s];
            float dm = dminq * (float) lm[s];
            for (int j = 0; j < 32; j++) {
                int q = ds > 0.0f ? (int) lroundf((xb[s * 32 + j] + dm) / ds) : 0;
                q     = q < 0 ? 0 : (q > 15 ? 15 : q);
                int g = s >> 1;
                if (s & 1) {
                    qs[g * 32 + j] |= (uint8_t) (q << 4);
                } else {
                    qs[g * 32 + j] |= (uint8_t) q;
                }
            }
        }
    }
}

/* Valid Q6_K blocks: per 16-element group an int8 scale of a per-block f16 super-scale. */
void orc_quantize_row_q6_K(const float * x, void * dst, int64_t n) {
    uint8_t * p = (uint8_t *) dst;
    for (int64_t b = 0; b < n / 256; b++) {
        const float * xb  = x + b * 256;
        uint8_t *     blk = p + b * 210;
        float         gs[16];
        float         max_abs_scale = 0.0f;
        for (int g = 0; g < 16; g++) {
            float amax = 0.0f;
            for (int j = 0; j < 16; j++) {
                float a = fabsf(xb[g * 16 + j]);
                amax    = a > amax ? a : amax;
            }
            gs[g] = amax / 31.0f;
            if (gs[g] > max_abs_scale) {
                max_abs_scale = gs[g];
            }
        }
        float    d  = max_abs_scale / 127.0f;
        uint16_t dh = orc_f32_to_f16(d);
        float    dq = orc_f16_to_f32(dh);
        int8_t * sc = (int8_t *) (blk + 192);
        for (int g = 0; g < 16; g++) {
            int s = dq > 0.0f ? (int) lroundf(gs[g] / dq) : 0;
            sc[g] = (int8_t) (s > 127 ? 127 : s);
        }
        blk[208] = (uint8_t) (dh & 0xff);
        blk[209] = (uint8_t) (dh >> 8);
        uint8_t * ql = blk;
        uint8_t * qh = blk + 128;
        memset(ql, 0, 128);
        memset(qh, 0, 64);
        for (int j = 0; j < 256; j++) {
            float ds = dq * (float) sc[j >> 4];
            int   q  = ds > 0.0f ? (int) lroundf(xb[j] / ds) : 0;
            q        = q < -32 ? -32 : (q > 31 ? 31 : q);
            int u    = q + 32;
            int half = j >> 7, c = (j >> 5) & 3, l = j & 31;
            int li   = half * 64 + ((c & 1) ? 32 : 0) + l;
            if (c & 2) {
                ql[li] |= (uint8_t) ((u & 0x0f) << 4);
            } else {
                ql[li] |= (uint8_t) (u & 0x0f);
            }
            qh[half * 32 + l] |= (uint8_t) (((u >> 4) & 3) << (2 * c));
        }
    }
}

/* ------------------------------------------------------------------------------------------ */
/* ops                                                                                         */
/* ------------------------------------------------------------------------------------------ */

void orc_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) {
        omp_set_num_threads(n);
    }
#else
    (void) n;
#endif
}

int orc_get_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* ggml_get_rows on a quantized/plain table (qwen3-enc.h:390, qwen3-lm.h:464,626). */
int orc_get_rows(int type, const void * table, int64_t n_rows, int64_t cols, const int32_t * ids, int64_t n_ids,
                 float * out) {
    int64_t rb = orc_row_bytes(type, cols);
    if (rb < 0) {
        return -1;
    }
    int bad = 0;
#pragma omp parallel for reduction(| : bad) schedule(static)
    for (int64_t i = 0; i < n_ids; i++) {
        int32_t id = ids[i];
        if (id < 0 || id >= n_rows) {
            bad |= 1;
            continue;
        }
        orc_dequant_row(type, (const uint8_t *) table + (size_t) id * rb, out + i * cols, cols);
    }
    return bad ? -1 : 0;
}

/* ggml_rms_norm followed by ggml_mul(w) (qwen3-enc.h:114-120; dit-graph.h:24-30). */
static inline void rms_norm_row(const float * x, const float * w, float * y, int64_t cols, float eps) {
    double sum = 0.0;
    for (int64_t i = 0; i < cols; i++) {
        sum += (double) (x[i] * x[i]);
    }
    float mean  = (float) (sum / (double) cols);
    float scale = 1.0f / sqrtf(mean + eps);
    for (int64_t i = 0; i < cols; i++) {
        float v = x[i] * scale;
        y[i]    = w ? v * w[i] : v;
    }
}

void orc_rms_norm(const float * x, const float * w, float * y, int64_t rows, int64_t cols, float eps) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; r++) {
        rms_norm_row(x + r * cols, w, y + r * cols, cols, eps);
    }
}

/* RoPE cache as ggml builds it for mode NEOX with freq_scale 1, ext_factor 0, attn_factor 1
 * (the arguments passed at qwen3-enc.h:172-173, qwen3-lm.h:378-379, dit-graph.h:195-197):
 * theta_scale = powf(base, -2/D); theta starts at pos and is multiplied by theta_scale
 * after each pair. */
void orc_rope_cache(float * cache, const int32_t * pos, int64_t n_pos, int head_dim, float base) {
    const float theta_scale = powf(base, -2.0f / (float) head_dim);
    for (int64_t p = 0; p < n_pos; p++) {
        float   theta = (float) pos[p];
        float * c     = cache + p * head_dim;
        for (int i = 0; i < head_dim / 2; i++) {
            c[2 * i]     = cosf(theta);
            c[2 * i + 1] = sinf(theta);
            theta *= theta_scale;
        }
    }
}

/* Per-head q/k RMSNorm * w then NeoX rotation of (i, i + D/2)
 * (qwen3-enc.h:164-174; qwen3-lm.h:371-379; dit-graph.h:181-197). */
void orc_qk_norm_rope(const float * x, int64_t x_tok_stride, float * y, int64_t y_tok_stride, int64_t n_tok,
                      int n_heads, int head_dim, const float * w, float eps, const float * rope) {
    const int half = head_dim / 2;
#pragma omp parallel for schedule(static)
    for (int64_t t = 0; t < n_tok; t++) {
        float tmp[1024];
        for (int h = 0; h < n_heads; h++) {
            const float * xs = x + t * x_tok_stride + (int64_t) h * head_dim;
            float *       ys = y + t * y_tok_stride + (int64_t) h * head_dim;
            rms_norm_row(xs, w, tmp, head_dim, eps);
            if (!rope) {
                memcpy(ys, tmp, sizeof(float) * head_dim);
                continue;
            }
            const float * c = rope + t * head_dim;
            for (int i = 0; i < half; i++) {
                float cs = c[2 * i], sn = c[2 * i + 1];
                float x0 = tmp[i], x1 = tmp[i + half];
                float a = x0 * cs, b = x1 * sn;
                float e = x0 * sn, f = x1 * cs;
                ys[i]        = a - b;
                ys[i + half] = e + f;
            }
        }
    }
}

/* ggml_swiglu / ggml_swiglu_split (qwen3-enc.h:217,221; dit-graph.h:259,264):
 * silu(g) = g / (1 + exp(-g)), times u. exp is acb_expf (acb_exp.h), the library's own
 * exponential: ggml-CPU's vectorised exp is not available here, so the oracle fixes one exp that
 * the kernels share bit for bit. */
void orc_swiglu(const float * g, int64_t g_stride, const float * u, int64_t u_stride, float * out, int64_t rows,
                int64_t F) {
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; r++) {
        const float * gr = g + r * g_stride;
        const float * ur = u + r * u_stride;
        float *       o  = out + r * F;
        for (int64_t i = 0; i < F; i++) {
            float s = gr[i] / (1.0f + acb_expf(-gr[i]));
            o[i]    = s * ur[i];
        }
    }
}

/* dit_ggml_rms_norm_weighted + dit_ggml_adaln (dit-graph.h:24-30, 54-64):
 * one_plus_s = scale + 1; y = n * one_plus_s; y = y + shift (three graph nodes). */
void orc_adaln(const float * x, const float * w, float eps, const float * scale, const float * shift,
               int64_t vec_stride, float * y, int64_t samples, int64_t rows_per_sample, int64_t H) {
#pragma omp parallel for collapse(2) schedule(static)
    for (int64_t s = 0; s < samples; s++) {
        for (int64_t r = 0; r < rows_per_sample; r++) {
            const float * sc = scale + s * vec_stride;
            const float * sh = shift + s * vec_stride;
            const float * xr = x + (s * rows_per_sample + r) * H;
            float *       yr = y + (s * rows_per_sample + r) * H;
            if (w) {
                rms_norm_row(xr, w, yr, H, eps);
            } else if (yr != xr) {
                memcpy(yr, xr, sizeof(float) * H);
            }
            for (int64_t i = 0; i < H; i++) {
                float ops = sc[i] + 1.0f;
                float v   = yr[i] * ops;
                yr[i]     = v + sh[i];
            }
        }
    }
}

/* dit_ggml_gated_add (dit-graph.h:70-76): out = r + o * gate. */
void orc_gated_residual(const float * r, const float * o, const float * gate, int64_t vec_stride, float * out,
                        int64_t samples, int64_t rows_per_sample, int64_t H) {
#pragma omp parallel for collapse(2) schedule(static)
    for (int64_t s = 0; s < samples; s++) {
        for (int64_t t = 0; t < rows_per_sample; t++) {
            const float * g   = gate + s * vec_stride;
            int64_t       off = (s * rows_per_sample + t) * H;
            for (int64_t i = 0; i < H; i++) {
                float v      = o[off + i] * g[i];
                out[off + i] = r[off + i] + v;
            }
        }
    }
}

/* ---- quantized mul_mat (ggml_mul_mat at every linear: qwen3-enc.h:86-88; dit-graph.h:36-49) ---- */

/* The quantised dot products. Each block's term is formed in float exactly as ggml forms it
 * (integer block dot, then (float)isum * (d_w * d_x), each product rounded), and the terms are
 * added in double with one rounding to float at the end. ggml's own float order over the
 * blocks depends on its SIMD width and cannot be known here; a double sum of float terms is
 * exact whenever the terms span fewer than ~20 binades, so it gives the same float in any
 * order and every GPU partition of the sum reproduces it. */
static float dot_q8_0_q8_0(const uint8_t * w, const uint8_t * xq, int64_t nb) {
    double sumf = 0.0;
    for (int64_t b = 0; b < nb; b++) {
        const uint8_t * wb   = w + b * 34;
        const uint8_t * xb   = xq + b * 34;
        int             sumi = 0;
        for (int j = 0; j < 32; j++) {
            sumi += (int) (int8_t) wb[2 + j] * (int) (int8_t) xb[2 + j];
        }
        float dd = orc_f16_to_f32(rd16(wb)) * orc_f16_to_f32(rd16(xb));
        sumf += (double) ((float) sumi * dd);
    }
    return (float) sumf;
}

static float dot_q4_K_q8_K(const uint8_t * w, const uint8_t * xq, int64_t nb) {
    double sumf = 0.0;
    for (int64_t b = 0; b < nb; b++) {
        const uint8_t * wb = w + b * 144;
        const uint8_t * xb = xq + b * 292;
        const int8_t *  q8 = (const int8_t *) (xb + 4);
        int16_t         bs[16];
        memcpy(bs, xb + 260, 32);
        float dx;
        memcpy(&dx, xb, 4);
        int isum = 0, imin = 0;
        for (int s = 0; s < 8; s++) {
            int sc, m;
            q4k_scale_min(s, wb + 4, &sc, &m);
            int dot = 0;
            for (int l = 0; l < 32; l++) {
                int sub;
                int q = q4k_value(wb, s * 32 + l, &sub);
                dot += q * q8[s * 32 + l];
            }
            isum += sc * dot;
            imin += m * (bs[2 * s] + bs[2 * s + 1]);
        }
        float d    = orc_f16_to_f32(rd16(wb)) * dx;
        float dmin = orc_f16_to_f32(rd16(wb + 2)) * dx;
        sumf += (double) (d * (float) isum);
        sumf -= (double) (dmin * (float) imin);
    }
    return (float) sumf;
}

static float dot_q6_K_q8_K(const uint8_t * w, const uint8_t * xq, int64_t nb) {
    double sumf = 0.0;
    for (int64_t b = 0; b < nb; b++) {
        const uint8_t * wb = w + b * 210;
        const uint8_t * xb = xq + b * 292;
        const int8_t *  q8 = (const int8_t *) (xb + 4);
        const int8_t *  sc = (const int8_t *) (wb + 192);
        float           dx;
        memcpy(&dx, xb, 4);
        int isum = 0;
        for (int g = 0; g < 16; g++) {
            int dot = 0;
            for (int l = 0; l < 16; l++) {
                dot += q6k_value(wb, g * 16 + l) * q8[g * 16 + l];
            }
            isum += sc[g] * dot;
        }
        float d = orc_f16_to_f32(rd16(wb + 208)) * dx;
        sumf += (double) (d * (float) isum);
    }
    return (float) sumf;
}

/* The same Q8_0 x Q8_0 products for a tile of up to 4 activation rows x 4 weight rows: each block
 * of 32 is loaded once for four dot products (the integer dots, the float terms and their double
 * sums are exactly those of dot_q8_0_q8_0, so the results are identical; only the host's cache
 * traffic and instruction count drop). The AVX2 form sign-extends to 16 bits and uses
 * multiply-add pairs: exact for every int8 value. */
#if defined(__AVX2__)
#    include <immintrin.h>
static inline __m256i q8_lo16(const uint8_t * p) {
    return _mm256_cvtepi8_epi16(_mm_loadu_si128((const __m128i *) p));
}
static inline int hsum_i32(__m256i v) {
    __m128i s = _mm_add_epi32(_mm256_castsi256_si128(v), _mm256_extracti128_si256(v, 1));
    s         = _mm_add_epi32(s, _mm_shuffle_epi32(s, 0x4e));
    s         = _mm_add_epi32(s, _mm_shuffle_epi32(s, 0xb1));
    return _mm_cvtsi128_si32(s);
}
#endif

static void tile_q8_0(const uint8_t * w, int64_t rb, const uint8_t * xq, int64_t xrb, int64_t nb, int mt, int nt,
                      float * y, int64_t ldy) {
    double acc[4][4];
    memset(acc, 0, sizeof(acc));
    for (int64_t b = 0; b < nb; b++) {
        float dw[4];
        for (int j = 0; j < nt; j++) {
            dw[j] = orc_f16_to_f32(rd16(w + j * rb + b * 34));
        }
#if defined(__AVX2__)
        __m256i w16[4][2];
        for (int j = 0; j < nt; j++) {
            const uint8_t * wb = w + j * rb + b * 34 + 2;
            w16[j][0]          = q8_lo16(wb);
            w16[j][1]          = q8_lo16(wb + 16);
        }
#endif
        for (int i = 0; i < mt; i++) {
            const uint8_t * xb = xq + i * xrb + b * 34;
            const float     dx = orc_f16_to_f32(rd16(xb));
#if defined(__AVX2__)
            const __m256i x0 = q8_lo16(xb + 2), x1 = q8_lo16(xb + 18);
#endif
            for (int j = 0; j < nt; j++) {
#if defined(__AVX2__)
                const int sumi =
                    hsum_i32(_mm256_add_epi32(_mm256_madd_epi16(x0, w16[j][0]), _mm256_madd_epi16(x1, w16[j][1])));
#else
                const uint8_t * wb   = w + j * rb + b * 34;
                int             sumi = 0;
                for (int e = 0; e < 32; e++) {
                    sumi += (int) (int8_t) wb[2 + e] * (int) (int8_t) xb[2 + e];
                }
#endif
                const float dd = dw[j] * dx;
                acc[i][j] += (double) ((float) sumi * dd);
            }
        }
    }
    for (int i = 0; i < mt; i++) {
        for (int j = 0; j < nt; j++) {
            y[i * ldy + j] = (float) acc[i][j];
        }
    }
}

static int g_mm_mode = ORC_MM_GGML;

void orc_set_mul_mat_mode(int mode) {
    g_mm_mode = mode == ORC_MM_EXACT ? ORC_MM_EXACT : ORC_MM_GGML;
}

int orc_get_mul_mat_mode(void) {
    return g_mm_mode;
}

/* ORC_MM_EXACT: every weight row dequantised once, f32 activation, double accumulation. */
static int mul_mat_exact(int wtype, const uint8_t * w, int64_t rb, int64_t N, int64_t K, const float * x, int64_t M,
                         float * y) {
    float * wd = (float *) malloc(sizeof(float) * (size_t) (N * K));
    if (!wd) {
        return -1;
    }
    int bad = 0;
#pragma omp parallel for schedule(static) reduction(| : bad)
    for (int64_t n = 0; n < N; n++) {
        bad |= orc_dequant_row(wtype, w + n * rb, wd + n * K, K) != 0;
    }
    if (bad) {
        free(wd);
        return -1;
    }
#pragma omp parallel for collapse(2) schedule(static)
    for (int64_t m = 0; m < M; m++) {
        for (int64_t n = 0; n < N; n++) {
            const float * xr  = x + m * K;
            const float * wr  = wd + n * K;
            double        acc = 0.0;
            for (int64_t k = 0; k < K; k++) {
                acc += (double) wr[k] * (double) xr[k];
            }
            y[m * N + n] = (float) acc;
        }
    }
    free(wd);
    return 0;
}

int orc_mul_mat(int wtype, const void * W, int64_t N, int64_t K, const float * x, int64_t M, float * y) {
    int64_t rb = orc_row_bytes(wtype, K);
    if (rb < 0) {
        return -1;
    }
    const uint8_t * w = (const uint8_t *) W;
    if (g_mm_mode == ORC_MM_EXACT) {
        return mul_mat_exact(wtype, w, rb, N, K, x, M, y);
    }
    if (wtype == ORC_Q8_0 || wtype == ORC_Q4_K || wtype == ORC_Q6_K) {
        int     vt  = wtype == ORC_Q8_0 ? ORC_Q8_0 : ORC_Q8_K;
        int64_t xrb = orc_row_bytes(vt, K);
        if (xrb < 0) {
            return -1;
        }
        uint8_t * xq = (uint8_t *) malloc((size_t) (M * xrb));
        for (int64_t m = 0; m < M; m++) {
            if (vt == ORC_Q8_0) {
                orc_quantize_row_q8_0(x + m * K, xq + m * xrb, K);
            } else {
                orc_quantize_row_q8_K(x + m * K, xq + m * xrb, K);
            }
        }
        if (wtype == ORC_Q8_0) {
            const int64_t mtiles = (M + 3) / 4, ntiles = (N + 3) / 4;
#pragma omp parallel for collapse(2) schedule(static)
            for (int64_t tm = 0; tm < mtiles; tm++) {
                for (int64_t tn = 0; tn < ntiles; tn++) {
                    const int mt = (int) (M - 4 * tm < 4 ? M - 4 * tm : 4);
                    const int nt = (int) (N - 4 * tn < 4 ? N - 4 * tn : 4);
                    tile_q8_0(w + 4 * tn * rb, rb, xq + 4 * tm * xrb, xrb, K / 32, mt, nt, y + 4 * tm * N + 4 * tn, N);
                }
            }
            free(xq);
            return 0;
        }
#pragma omp parallel for collapse(2) schedule(static)
        for (int64_t m = 0; m < M; m++) {
            for (int64_t n = 0; n < N; n++) {
                const uint8_t * wr = w + n * rb;
                const uint8_t * xr = xq + m * xrb;
                float           v;
                if (wtype == ORC_Q8_0) {
                    v = dot_q8_0_q8_0(wr, xr, K / 32);
                } else if (wtype == ORC_Q4_K) {
                    v = dot_q4_K_q8_K(wr, xr, K / 256);
                } else {
                    v = dot_q6_K_q8_K(wr, xr, K / 256);
                }
                y[m * N + n] = v;
            }
        }
        free(xq);
        return 0;
    }
    if (wtype == ORC_F32 || wtype == ORC_F16 || wtype == ORC_BF16) {
        /* F16/BF16 weights: the activation is converted to the weight type first. */
#pragma omp parallel for collapse(2) schedule(static)
        for (int64_t m = 0; m < M; m++) {
            for (int64_t n = 0; n < N; n++) {
                const float * xr  = x + m * K;
                double        acc = 0.0;
                for (int64_t k = 0; k < K; k++) {
                    float wv, xv = xr[k];
                    if (wtype == ORC_F32) {
                        wv = ((const float *) w)[n * K + k];
                    } else if (wtype == ORC_F16) {
                        wv = orc_f16_to_f32(rd16(w + 2 * (n * K + k)));
                        xv = orc_f16_to_f32(orc_f32_to_f16(xv));
                    } else {
                        wv = orc_bf16_to_f32(rd16(w + 2 * (n * K + k)));
                        xv = orc_bf16_to_f32(orc_f32_to_bf16(xv));
                    }
                    acc += (double) (wv * xv);
                }
                y[m * N + n] = (float) acc;
            }
        }
        return 0;
    }
    return -1;
}

/* ---- attention (qwen3_attn_f32, qwen3-enc.h:101-112; dit_attn_f32, dit-graph.h:123-134) ---- */

static inline float kv_at(const void * base, int kv_type, int64_t idx) {
    if (kv_type == ORC_F16) {
        return orc_f16_to_f32(((const uint16_t *) base)[idx]);
    }
    return ((const float *) base)[idx];
}

void orc_attention(const float * q, int64_t q_tok_stride, const void * k, const void * v, int kv_type,
                   int64_t kv_tok_stride, int64_t kv_head_stride, const float * mask, float * out,
                   int64_t out_tok_stride, int64_t Sq, int64_t Skv, int Hq, int Hkv, int D, float scale) {
    const int grp = Hq / Hkv;
    const int f16 = kv_type == ORC_F16;
#pragma omp parallel for collapse(2) schedule(dynamic, 4)
    for (int64_t i = 0; i < Sq; i++) {
        for (int h = 0; h < Hq; h++) {
            float * s   = (float *) malloc(sizeof(float) * (size_t) Skv);
            float   qv[512];
            int     hk  = h / grp;
            for (int d = 0; d < D; d++) {
                float x = q[i * q_tok_stride + (int64_t) h * D + d];
                qv[d]   = f16 ? orc_f16_to_f32(orc_f32_to_f16(x)) : x;
            }
            /* scores = K . q, then soft_max_ext: x*scale + mask. On the f16 cache the dot is
             * summed in float in one fixed order (every product of two f16 values is exact):
             * eight sequential sums over 16 dimensions each, added as
             * ((s0+s1)+(s2+s3))+((s4+s5)+(s6+s7)) -- the order of the decode kernels. The f32
             * path sums in double. The P.V sums accumulate in double and round once (on the f16
             * cache every product is exact, so the sum is exact in any order unless its terms
             * span ~24 binades); the exponential is acb_expf. */
            float mx = -INFINITY;
            for (int64_t j = 0; j < Skv; j++) {
                float sv;
                if (f16 && D == 128) {
                    float part[8];
                    for (int c = 0; c < 8; c++) {
                        float acc = 0.0f;
                        for (int d = 16 * c; d < 16 * c + 16; d++) {
                            float kk = kv_at(k, kv_type, j * kv_tok_stride + (int64_t) hk * kv_head_stride + d);
                            acc      = acc + kk * qv[d];
                        }
                        part[c] = acc;
                    }
                    sv = (((part[0] + part[1]) + (part[2] + part[3])) + ((part[4] + part[5]) + (part[6] + part[7]))) *
                         scale;
                } else {
                    double acc = 0.0;
                    for (int d = 0; d < D; d++) {
                        float kk = kv_at(k, kv_type, j * kv_tok_stride + (int64_t) hk * kv_head_stride + d);
                        acc += f16 ? (double) (kk * qv[d]) : (double) kk * (double) qv[d];
                    }
                    sv = (float) acc * scale;
                }
                if (mask) {
                    sv = sv + mask[i * Skv + j];
                }
                s[j] = sv;
                mx   = sv > mx ? sv : mx;
            }
            double sum = 0.0;
            for (int64_t j = 0; j < Skv; j++) {
                float e = (mx == -INFINITY) ? 0.0f : acb_expf(s[j] - mx);
                s[j]    = e;
                sum += (double) e;
            }
            float inv = sum > 0.0 ? (float) (1.0 / sum) : 0.0f;
            for (int64_t j = 0; j < Skv; j++) {
                float p = s[j] * inv;
                s[j]    = f16 ? orc_f16_to_f32(orc_f32_to_f16(p)) : p;
            }
            float * o = out + i * out_tok_stride + (int64_t) h * D;
            for (int d = 0; d < D; d++) {
                double acc = 0.0;
                for (int64_t j = 0; j < Skv; j++) {
                    float vv = kv_at(v, kv_type, j * kv_tok_stride + (int64_t) hk * kv_head_stride + d);
                    acc += f16 ? (double) (vv * s[j]) : (double) vv * (double) s[j];
                }
                o[d] = (float) acc;
            }
            free(s);
        }
    }
}

/* ggml_timestep_embedding (dit-graph.h:93): [cos(t*f_j) | sin(t*f_j)], f_j = exp(-ln(P) j/half). */
void orc_timestep_embedding(float t, int dim, int max_period, float * out) {
    int half = dim / 2;
    for (int j = 0; j < half; j++) {
        float freq    = expf(-logf((float) max_period) * (float) j / (float) half);
        float arg     = t * freq;
        out[j]        = cosf(arg);
        out[j + half] = sinf(arg);
    }
    if (dim % 2) {
        out[dim - 1] = 0.0f;
    }
}

/* ---- Philox noise (src/philox.h) ---- */

/* One round: two 32x32->64 products of the even words, the odd words and the key XORed into the
 * high halves (philox.h:37-47). Round multipliers and Weyl key increments (philox.h:16-19) are the
 * published Philox4x32 constants. */
void orc_philox4x32_10(const uint32_t ctr[4], uint32_t k0, uint32_t k1, uint32_t out[4]) {
    uint32_t c0 = ctr[0], c1 = ctr[1], c2 = ctr[2], c3 = ctr[3];
    for (int r = 0; r < 10; r++) {
        if (r) {
            k0 += 0x9E3779B9u;
            k1 += 0xBB67AE85u;
        }
        const uint64_t p0 = (uint64_t) 0xD2511F53u * c0;
        const uint64_t p1 = (uint64_t) 0xCD9E8D57u * c2;
        const uint32_t n0 = (uint32_t) (p1 >> 32) ^ c1 ^ k0;
        const uint32_t n2 = (uint32_t) (p0 >> 32) ^ c3 ^ k1;
        c0 = n0;
        c1 = (uint32_t) p1;
        c2 = n2;
        c3 = (uint32_t) p0;
    }
    out[0] = c0;
    out[1] = c1;
    out[2] = c2;
    out[3] = c3;
}

/* Only the first output of the first Box-Muller pair is kept (philox.h:85-91, 130-136): a uniform
 * u in (0, 1] from word 0 and an angle in (0, 2 pi) from word 1, both as x * 2^-32 + half a step
 * in float; normal = sqrt(-2 ln u) * sin(angle). */
void orc_philox_randn(int64_t seed, int64_t n, int bf16_round, float * out) {
    const float inv32 = 2.3283064365386963e-10f;   /* 2^-32 */
    const float inv32_2pi = 1.4629180792671596e-09f; /* 2 pi 2^-32 */
    const uint32_t k0 = (uint32_t) (uint64_t) seed, k1 = (uint32_t) ((uint64_t) seed >> 32);
#pragma omp parallel for schedule(static) if (n > 65536)
    for (int64_t k = 0; k < n; k++) {
        const uint32_t ctr[4] = { 0u, 0u, (uint32_t) (uint64_t) k, (uint32_t) ((uint64_t) k >> 32) };
        uint32_t       w[4];
        orc_philox4x32_10(ctr, k0, k1, w);
        const float u = (float) w[0] * inv32 + inv32 * 0.5f;
        const float v = (float) w[1] * inv32_2pi + inv32_2pi * 0.5f;
        const float z = sqrtf(-2.0f * logf(u)) * sinf(v);
        out[k] = bf16_round ? orc_bf16_to_f32(orc_f32_to_bf16(z)) : z;
    }
}

/* ---- FSQ (src/fsq-detok.h:14-29, src/fsq-tok.h:42-60) ---- */

static const int orc_fsq_levels[6] = { 8, 8, 8, 5, 5, 5 };

/* fsq_decode_index: dimension d's level (index / prod(L_<d)) % L_d mapped to level / ((L-1)/2) - 1 */
void orc_fsq_decode_index(int index, float * out6) {
    int stride = 1;
    for (int d = 0; d < 6; d++) {
        int   L      = orc_fsq_levels[d];
        float half_L = (float) (L - 1) / 2.0f;
        out6[d]      = (float) ((index / stride) % L) / half_L - 1.0f;
        stride *= L;
    }
}

/* fsq_encode_index: level floor((L-1) * (tanh(x) + 1) / 2 + 0.5) clamped to [0, L-1], flat index
 * with dimension 0 fastest */
int orc_fsq_encode_index(const float * raw6) {
    int index = 0, mult = 1;
    for (int d = 0; d < 6; d++) {
        int   L    = orc_fsq_levels[d];
        float t    = tanhf(raw6[d]);
        int   code = (int) floorf((float) (L - 1) * (t + 1.0f) / 2.0f + 0.5f);
        if (code < 0) {
            code = 0;
        }
        if (code >= L) {
            code = L - 1;
        }
        index += code * mult;
        mult *= L;
    }
    return index;
}

/* ---- LM sampling (sample_top_k_p, src/sampling.h:30-133) ---- */

typedef struct {
    int   id;
    float prob;
} orc_tok_prob;

static int cmp_desc_f32(const void * a, const void * b) {
    float x = *(const float *) a, y = *(const float *) b;
    return (x < y) - (x > y);
}

/* descending probability; equal probabilities by ascending id (the reference's std::sort leaves
 * their order unspecified) */
static int cmp_tok_prob(const void * a, const void * b) {
    const orc_tok_prob * x = (const orc_tok_prob *) a;
    const orc_tok_prob * y = (const orc_tok_prob *) b;
    if (x->prob != y->prob) {
        return x->prob > y->prob ? -1 : 1;
    }
    return (x->id > y->id) - (x->id < y->id);
}

/* temperature -> top_k -> top_p -> softmax -> multinomial on logits[V] (modified in place, as the
 * reference does); u is the draw of std::uniform_real_distribution<float>(0, sum)'s canonical
 * variate, so r = u * sum. Returns the sampled index. */
int orc_sample_top_k_p(float * logits, int V, float temperature, float top_p, int top_k, float u) {
    if (temperature <= 0.0f) {
        int best = 0;
        for (int i = 1; i < V; i++) {
            if (logits[i] > logits[best]) {
                best = i;
            }
        }
        return best;
    }
    float inv_temp = 1.0f / temperature;
    for (int i = 0; i < V; i++) {
        logits[i] *= inv_temp;
    }
    if (top_k > 0 && top_k < V) {
        float * tmp = (float *) malloc(sizeof(float) * (size_t) V);
        memcpy(tmp, logits, sizeof(float) * (size_t) V);
        qsort(tmp, (size_t) V, sizeof(float), cmp_desc_f32);
        float threshold = tmp[top_k - 1];
        free(tmp);
        for (int i = 0; i < V; i++) {
            if (logits[i] < threshold) {
                logits[i] = -INFINITY;
            }
        }
    }
    if (top_p > 0.0f && top_p < 1.0f) {
        float max_logit = -INFINITY;
        for (int i = 0; i < V; i++) {
            if (logits[i] > max_logit) {
                max_logit = logits[i];
            }
        }
        float sum_exp = 0.0f;
        for (int i = 0; i < V; i++) {
            sum_exp += expf(logits[i] - max_logit);
        }
        float          inv_sum = 1.0f / sum_exp;
        float          cutoff  = max_logit - 16.0f;
        orc_tok_prob * buf     = (orc_tok_prob *) malloc(sizeof(orc_tok_prob) * (size_t) V);
        int            K       = 0;
        for (int i = 0; i < V; i++) {
            if (logits[i] >= cutoff) {
                buf[K].id   = i;
                buf[K].prob = expf(logits[i] - max_logit) * inv_sum;
                K++;
            } else {
                logits[i] = -INFINITY;
            }
        }
        if (K > 0) {
            qsort(buf, (size_t) K, sizeof(orc_tok_prob), cmp_tok_prob);
            float cum = 0.0f;
            for (int i = 0; i < K; i++) {
                if (i > 0 && cum >= top_p) {
                    logits[buf[i].id] = -INFINITY;
                }
                cum += buf[i].prob;
            }
        }
        free(buf);
    }
    float max_val = -INFINITY;
    for (int i = 0; i < V; i++) {
        if (logits[i] > max_val) {
            max_val = logits[i];
        }
    }
    float sum = 0.0f;
    for (int i = 0; i < V; i++) {
        logits[i] = expf(logits[i] - max_val);
        sum += logits[i];
    }
    float r   = u * (sum - 0.0f) + 0.0f;
    float acc = 0.0f;
    for (int i = 0; i < V; i++) {
        acc += logits[i];
        if (acc >= r) {
            return i;
        }
    }
    return 0;
}
