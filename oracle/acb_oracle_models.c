/*
 * acb_oracle_models.c -- CPU oracle of the encoder / LM / DiT forwards (test infrastructure
 * only; see acb_oracle_models.h for the reference functions each one restates).
 */
#include "acb_oracle_models.h"
#include "../hbd-acestep.cpp_b200/csrc/acb_exp.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

static float * fbuf(int64_t n) {
    return (float *) calloc((size_t) (n > 0 ? n : 1), sizeof(float));
}

/* y[M][nrows] = rows [row0, row0+nrows) of W applied to x[M][K] (ggml_mul_mat). */
static int linear_rows(const orc_tensor * w, int64_t row0, int64_t nrows, const float * x, int64_t M, float * y) {
    int64_t rb = orc_row_bytes(w->type, w->K);
    if (rb < 0 || row0 + nrows > w->N) {
        return -1;
    }
    return orc_mul_mat(w->type, (const uint8_t *) w->data + row0 * rb, nrows, w->K, x, M, y);
}

static int linear(const orc_tensor * w, const float * x, int64_t M, float * y) {
    return linear_rows(w, 0, w->N, x, M, y);
}

/* ggml_add of an F32 bias broadcast along rows (dit_ggml_linear_bias, dit-graph.h:43-49). */
static void add_bias(float * y, int64_t M, int64_t N, const orc_tensor * b) {
    const float * bv = (const float *) b->data;
    int64_t       nb = b->K * b->N;
    for (int64_t m = 0; m < M; m++) {
        for (int64_t n = 0; n < N; n++) {
            y[m * N + n] = y[m * N + n] + bv[n % nb];
        }
    }
}

static void add_inplace(float * h, const float * o, int64_t n) {
    for (int64_t i = 0; i < n; i++) {
        h[i] = h[i] + o[i];
    }
}

/* ggml_silu with the library's exponential (acb_exp.h), like every SiLU of the oracle */
static inline float silu(float x) {
    return x / (1.0f + acb_expf(-x));
}

/* ---------------------------------------------------------------------------------------- */
/* Qwen3 layer (qwen3_build_layer, qwen3-enc.h:227-246; qw3lm_build_attn, qwen3-lm.h:327-424) */
/* ---------------------------------------------------------------------------------------- */

typedef struct {
    /* f32 K/V of the current tokens (encoder), or an f16 cache (LM) */
    orc_kv *        kv;
    int             layer;
    int             set0;        /* LM: first kv set */
    int             set_per_tok; /* 0: all tokens in set0 (prefill), 1: token i in set0+i (decode) */
    const int32_t * pos;         /* position of each token */
} attn_ctx;

/* One layer over S rows. Encoder (ac->kv NULL): the rows are B sequences of S / B rows, attention
 * within each sequence under the additive mask_enc [S/B][S/B] (NULL: none). */
static int qwen3_layer(const orc_qwen3 * m, const orc_qwen3_layer * ly, float * hidden, int S, const float * rope,
                       const attn_ctx * ac, const float * mask_enc, int B) {
    const int H = m->H, D = m->D, Nh = m->Nh, Nkv = m->Nkv, F = m->F;
    const int qd = Nh * D, kvd = Nkv * D, qkvd = qd + 2 * kvd;
    float *   norm = fbuf((int64_t) S * H);
    float *   qkv  = fbuf((int64_t) S * qkvd);
    float *   q    = fbuf((int64_t) S * qd);
    float *   k    = fbuf((int64_t) S * kvd);
    float *   v    = fbuf((int64_t) S * kvd);
    float *   att  = fbuf((int64_t) S * qd);
    float *   o    = fbuf((int64_t) S * H);
    float *   gu   = fbuf((int64_t) S * 2 * F);
    float *   act  = fbuf((int64_t) S * F);
    int       rc   = 0;

    orc_rms_norm(hidden, (const float *) ly->attn_norm.data, norm, S, H, m->eps);
    if (ly->qkv.data) {
        rc |= linear(&ly->qkv, norm, S, qkv);
    } else {
        /* separate projections: same row-wise products, written into the fused layout */
        float * t = fbuf((int64_t) S * qd);
        rc |= linear(&ly->q, norm, S, t);
        for (int s = 0; s < S; s++) {
            memcpy(qkv + (int64_t) s * qkvd, t + (int64_t) s * qd, sizeof(float) * qd);
        }
        rc |= linear(&ly->k, norm, S, t);
        for (int s = 0; s < S; s++) {
            memcpy(qkv + (int64_t) s * qkvd + qd, t + (int64_t) s * kvd, sizeof(float) * kvd);
        }
        rc |= linear(&ly->v, norm, S, t);
        for (int s = 0; s < S; s++) {
            memcpy(qkv + (int64_t) s * qkvd + qd + kvd, t + (int64_t) s * kvd, sizeof(float) * kvd);
        }
        free(t);
    }
    orc_qk_norm_rope(qkv, qkvd, q, qd, S, Nh, D, (const float *) ly->q_norm.data, m->eps, rope);
    orc_qk_norm_rope(qkv + qd, qkvd, k, kvd, S, Nkv, D, (const float *) ly->k_norm.data, m->eps, rope);
    for (int s = 0; s < S; s++) {
        memcpy(v + (int64_t) s * kvd, qkv + (int64_t) s * qkvd + qd + kvd, sizeof(float) * kvd);
    }
    const float scale = 1.0f / sqrtf((float) D);
    if (!ac->kv) {
        const int Ss = S / B;
        for (int b = 0; b < B; b++) {
            const int64_t r = (int64_t) b * Ss;
            orc_attention(q + r * qd, qd, k + r * kvd, v + r * kvd, ORC_F32, kvd, D, mask_enc, att + r * qd, qd, Ss, Ss,
                          Nh, Nkv, D, scale);
        }
    } else {
        orc_kv *      kv  = ac->kv;
        const int64_t hs  = (int64_t) kv->max_seq * D;            /* head stride */
        const int64_t ss  = (int64_t) Nkv * hs;                    /* set stride */
        const int64_t ls  = (int64_t) kv->n_sets * ss;             /* layer stride */
        uint16_t *    kl  = kv->k + ac->layer * ls;
        uint16_t *    vl  = kv->v + ac->layer * ls;
        /* ggml_cpy f32 -> f16 of the new K/V rows into the cache (qwen3-lm.h:396-406) */
        for (int s = 0; s < S; s++) {
            int     set = ac->set0 + (ac->set_per_tok ? s : 0);
            int64_t p   = ac->pos[s];
            for (int h = 0; h < Nkv; h++) {
                for (int d = 0; d < D; d++) {
                    int64_t idx = set * ss + h * hs + p * D + d;
                    kl[idx]     = orc_f32_to_f16(k[(int64_t) s * kvd + h * D + d]);
                    vl[idx]     = orc_f32_to_f16(v[(int64_t) s * kvd + h * D + d]);
                }
            }
        }
        if (!ac->set_per_tok) {
            /* prefill: causal over [0, pos[S-1]] of one set */
            int     kv_len = ac->pos[S - 1] + 1;
            float * mask   = fbuf((int64_t) S * kv_len);
            for (int i = 0; i < S; i++) {
                for (int j = 0; j < kv_len; j++) {
                    mask[(int64_t) i * kv_len + j] = (j <= ac->pos[i]) ? 0.0f : -INFINITY;
                }
            }
            orc_attention(q, qd, kl + ac->set0 * ss, vl + ac->set0 * ss, ORC_F16, D, hs, mask, att, qd, S, kv_len,
                          Nh, Nkv, D, scale);
            free(mask);
        } else {
            for (int s = 0; s < S; s++) {
                int set    = ac->set0 + s;
                int kv_len = ac->pos[s] + 1;
                orc_attention(q + (int64_t) s * qd, qd, kl + set * ss, vl + set * ss, ORC_F16, D, hs, NULL,
                              att + (int64_t) s * qd, qd, 1, kv_len, Nh, Nkv, D, scale);
            }
        }
    }
    rc |= linear(&ly->o, att, S, o);
    add_inplace(hidden, o, (int64_t) S * H);

    orc_rms_norm(hidden, (const float *) ly->post_norm.data, norm, S, H, m->eps);
    if (ly->gate_up.data) {
        rc |= linear(&ly->gate_up, norm, S, gu);
    } else {
        float * t = fbuf((int64_t) S * F);
        rc |= linear(&ly->gate, norm, S, t);
        for (int s = 0; s < S; s++) {
            memcpy(gu + (int64_t) s * 2 * F, t + (int64_t) s * F, sizeof(float) * F);
        }
        rc |= linear(&ly->up, norm, S, t);
        for (int s = 0; s < S; s++) {
            memcpy(gu + (int64_t) s * 2 * F + F, t + (int64_t) s * F, sizeof(float) * F);
        }
        free(t);
    }
    orc_swiglu(gu, 2 * F, gu + F, 2 * F, act, S, F);
    rc |= linear(&ly->down, act, S, o);
    add_inplace(hidden, o, (int64_t) S * H);

    free(norm);
    free(qkv);
    free(q);
    free(k);
    free(v);
    free(att);
    free(o);
    free(gu);
    free(act);
    return rc ? -1 : 0;
}

int orc_qwen3_layers_ex(const orc_qwen3 * m, float * hidden, int B, int S, int l0, int l1, int causal, int window,
                        float * out) {
    if (l0 < 0 || l1 > m->n_layers || l0 > l1 || B <= 0 || S <= 0) {
        return -1;
    }
    const int R    = B * S;
    int32_t * pos  = (int32_t *) malloc(sizeof(int32_t) * R);
    float *   rope = fbuf((int64_t) R * m->D);
    float *   mask = causal ? fbuf((int64_t) S * S) : NULL;
    /* the bidirectional sliding window of the even layers: |i - j| <= window (cond-enc.h:298-312) */
    float *   slide = (!causal && window > 0) ? fbuf((int64_t) S * S) : NULL;
    for (int i = 0; i < S; i++) {
        for (int j = 0; j < S; j++) {
            if (mask) {
                mask[(int64_t) i * S + j] = (j <= i) ? 0.0f : -INFINITY;
            }
            if (slide) {
                slide[(int64_t) i * S + j] = abs(i - j) <= window ? 0.0f : -INFINITY;
            }
        }
    }
    for (int i = 0; i < R; i++) {
        pos[i] = i % S;
    }
    orc_rope_cache(rope, pos, R, m->D, m->rope_theta);
    attn_ctx ac = { 0 };
    int      rc = 0;
    for (int l = l0; l < l1 && rc == 0; l++) {
        const float * lm = causal ? mask : (slide && l % 2 == 0 ? slide : NULL);
        rc               = qwen3_layer(m, &m->layers[l], hidden, R, rope, &ac, lm, B);
    }
    if (out) {
        orc_rms_norm(hidden, (const float *) m->final_norm.data, out, R, m->H, m->eps);
    }
    free(pos);
    free(rope);
    free(mask);
    free(slide);
    return rc;
}

int orc_qwen3_layers(const orc_qwen3 * m, float * hidden, int S, int l0, int l1, int causal, float * out) {
    return orc_qwen3_layers_ex(m, hidden, 1, S, l0, l1, causal, 0, out);
}

int orc_qwen3_encode(const orc_qwen3 * m, const int32_t * ids, int S, float * out) {
    float * hidden = fbuf((int64_t) S * m->H);
    if (orc_get_rows(m->embed.type, m->embed.data, m->embed.N, m->H, ids, S, hidden) != 0) {
        free(hidden);
        return -1;
    }
    const int rc = orc_qwen3_layers(m, hidden, S, 0, m->n_layers, 1, out);
    free(hidden);
    return rc;
}

static int lm_head(const orc_qwen3 * m, const float * h, int M, float * logits, int lm_offset, int lm_count) {
    if (lm_count > 0) {
        return linear_rows(&m->embed, lm_offset, lm_count, h, M, logits);
    }
    return linear(&m->embed, h, M, logits);
}

int orc_qw3lm_prefill(const orc_qwen3 * m, orc_kv * kv, int set, int kv_pos, const int32_t * ids, int n,
                      float * logits, int lm_offset, int lm_count, float * hidden_out) {
    const int H = m->H;
    if (kv_pos + n > kv->max_seq || set < 0 || set >= kv->n_sets) {
        return -1;
    }
    float * hidden = fbuf((int64_t) n * H);
    if (orc_get_rows(m->embed.type, m->embed.data, m->embed.N, H, ids, n, hidden) != 0) {
        free(hidden);
        return -1;
    }
    int32_t * pos  = (int32_t *) malloc(sizeof(int32_t) * n);
    float *   rope = fbuf((int64_t) n * m->D);
    for (int i = 0; i < n; i++) {
        pos[i] = kv_pos + i;
    }
    orc_rope_cache(rope, pos, n, m->D, m->rope_theta);
    attn_ctx ac = { kv, 0, set, 0, pos };
    int      rc = 0;
    for (int l = 0; l < m->n_layers && rc == 0; l++) {
        ac.layer = l;
        rc       = qwen3_layer(m, &m->layers[l], hidden, n, rope, &ac, NULL, 1);
    }
    float * fin = fbuf((int64_t) n * H);
    orc_rms_norm(hidden, (const float *) m->final_norm.data, fin, n, H, m->eps);
    if (hidden_out) {
        memcpy(hidden_out, fin, sizeof(float) * (size_t) n * H);
    }
    if (rc == 0 && logits) {
        rc = lm_head(m, fin + (int64_t) (n - 1) * H, 1, logits, lm_offset, lm_count);
    }
    free(fin);
    free(hidden);
    free(pos);
    free(rope);
    return rc;
}

int orc_qw3lm_decode(const orc_qwen3 * m, orc_kv * kv, int set0, const int32_t * kv_pos, const int32_t * ids, int N,
                     float * logits, int lm_offset, int lm_count) {
    const int H = m->H;
    for (int i = 0; i < N; i++) {
        if (kv_pos[i] + 1 > kv->max_seq || set0 + i >= kv->n_sets) {
            return -1;
        }
    }
    float * hidden = fbuf((int64_t) N * H);
    if (orc_get_rows(m->embed.type, m->embed.data, m->embed.N, H, ids, N, hidden) != 0) {
        free(hidden);
        return -1;
    }
    float * rope = fbuf((int64_t) N * m->D);
    orc_rope_cache(rope, kv_pos, N, m->D, m->rope_theta);
    attn_ctx ac = { kv, 0, set0, 1, kv_pos };
    int      rc = 0;
    for (int l = 0; l < m->n_layers && rc == 0; l++) {
        ac.layer = l;
        rc       = qwen3_layer(m, &m->layers[l], hidden, N, rope, &ac, NULL, 1);
    }
    float * fin = fbuf((int64_t) N * H);
    orc_rms_norm(hidden, (const float *) m->final_norm.data, fin, N, H, m->eps);
    if (rc == 0) {
        rc = lm_head(m, fin, N, logits, lm_offset, lm_count);
    }
    free(fin);
    free(hidden);
    free(rope);
    return rc;
}

/* ---------------------------------------------------------------------------------------- */
/* DiT (dit-graph.h)                                                                         */
/* ---------------------------------------------------------------------------------------- */

int orc_dit_timestep(const orc_dit * m, const orc_dit_temb * te, float t, float * temb, float * tproj) {
    const int H = m->H;
    float     sinus[256];
    float *   h  = fbuf(H);
    float *   h2 = fbuf(H);
    int       rc = 0;
    orc_timestep_embedding(t * 1000.0f, 256, 10000, sinus); /* ggml_scale then embedding (:87-90) */
    rc |= linear(&te->l1_w, sinus, 1, h);
    add_bias(h, 1, H, &te->l1_b);
    for (int i = 0; i < H; i++) {
        h[i] = silu(h[i]);
    }
    rc |= linear(&te->l2_w, h, 1, temb);
    add_bias(temb, 1, H, &te->l2_b);
    for (int i = 0; i < H; i++) {
        h2[i] = silu(temb[i]);
    }
    rc |= linear(&te->tp_w, h2, 1, tproj);
    add_bias(tproj, 1, 6 * H, &te->tp_b);
    free(h);
    free(h2);
    return rc ? -1 : 0;
}

/* dit_ggml_build_layer (dit-graph.h:367-450). hidden [N][S][H], enc [N][enc_S][H]. */
static int dit_layer(const orc_dit * m, const orc_dit_layer * ly, float * hidden, const float * enc, int N, int S,
                     int enc_S, const float * tproj, const float * rope, const int * real_S, const int * real_enc_S) {
    const int     H = m->H, D = m->D, Nh = m->Nh, Nkv = m->Nkv, F = m->F;
    const int     qd = Nh * D, kvd = Nkv * D, qkvd = qd + 2 * kvd;
    const int64_t R  = (int64_t) N * S;
    int           rc = 0;

    /* adaln = scale_shift_table + tproj, six [H] vectors */
    float *       ada = fbuf(6 * H);
    const float * sst = (const float *) ly->scale_shift.data;
    for (int i = 0; i < 6 * H; i++) {
        ada[i] = sst[i] + tproj[i];
    }
    const float *shift_sa = ada, *scale_sa = ada + H, *gate_sa = ada + 2 * H;
    const float *shift_ff = ada + 3 * H, *scale_ff = ada + 4 * H, *gate_ff = ada + 5 * H;

    float * norm = fbuf(R * H);
    float * qkv  = fbuf(R * qkvd);
    float * q    = fbuf(R * qd);
    float * k    = fbuf(R * kvd);
    float * v    = fbuf(R * kvd);
    float * att  = fbuf(R * qd);
    float * o    = fbuf(R * H);

    /* self-attention with adaLN and gated residual */
    orc_adaln(hidden, (const float *) ly->sa_norm.data, m->eps, scale_sa, shift_sa, 0, norm, 1, R, H);
    rc |= linear(&ly->sa_qkv, norm, R, qkv);
    for (int b = 0; b < N; b++) {
        float * qb = qkv + (int64_t) b * S * qkvd;
        orc_qk_norm_rope(qb, qkvd, q + (int64_t) b * S * qd, qd, S, Nh, D, (const float *) ly->sa_q_norm.data,
                         m->eps, rope);
        orc_qk_norm_rope(qb + qd, qkvd, k + (int64_t) b * S * kvd, kvd, S, Nkv, D,
                         (const float *) ly->sa_k_norm.data, m->eps, rope);
        for (int s = 0; s < S; s++) {
            memcpy(v + ((int64_t) b * S + s) * kvd, qb + (int64_t) s * qkvd + qd + kvd, sizeof(float) * kvd);
        }
    }
    /* self-attention mask of sequence b (dit-sampler.h:253-282): sa_mask_sw on the sliding layers
     * (window and padding), sa_mask_pad on the full ones (padding only) */
    float *     mask = NULL;
    int         win  = m->sliding_window;
    const int   swa  = ly->layer_type == 0 && win > 0 && S > win;
    const float scale = 1.0f / sqrtf((float) D);
    if (swa || real_S) {
        mask = fbuf((int64_t) S * S);
    }
    for (int b = 0; b < N; b++) {
        if (mask) {
            const int rs = real_S ? real_S[b] : S;
            for (int i = 0; i < S; i++) {
                for (int j = 0; j < S; j++) {
                    int dist                  = i > j ? i - j : j - i;
                    int ok                    = i < rs && j < rs && (!swa || dist <= win);
                    mask[(int64_t) i * S + j] = ok ? 0.0f : -INFINITY;
                }
            }
        }
        orc_attention(q + (int64_t) b * S * qd, qd, k + (int64_t) b * S * kvd, v + (int64_t) b * S * kvd, ORC_F32,
                      kvd, D, mask, att + (int64_t) b * S * qd, qd, S, S, Nh, Nkv, D, scale);
    }
    free(mask);
    rc |= linear(&ly->sa_o, att, R, o);
    orc_gated_residual(hidden, o, gate_sa, 0, hidden, 1, R, H);

    /* cross-attention: q rows of ca_qkv on hidden, k||v rows on enc; q/k norm, no rope */
    if (enc) {
        const int64_t Re  = (int64_t) N * enc_S;
        float *       kvb = fbuf(Re * 2 * kvd);
        float *       ke  = fbuf(Re * kvd);
        float *       ve  = fbuf(Re * kvd);
        orc_rms_norm(hidden, (const float *) ly->ca_norm.data, norm, R, H, m->eps);
        rc |= linear_rows(&ly->ca_qkv, 0, qd, norm, R, att);
        orc_qk_norm_rope(att, qd, q, qd, R, Nh, D, (const float *) ly->ca_q_norm.data, m->eps, NULL);
        rc |= linear_rows(&ly->ca_qkv, qd, 2 * kvd, enc, Re, kvb);
        orc_qk_norm_rope(kvb, 2 * kvd, ke, kvd, Re, Nkv, D, (const float *) ly->ca_k_norm.data, m->eps, NULL);
        for (int64_t r = 0; r < Re; r++) {
            memcpy(ve + r * kvd, kvb + r * 2 * kvd + kvd, sizeof(float) * kvd);
        }
        /* cross-attention mask (dit-sampler.h:288-304): condition rows ki < real_enc_S[b] */
        float * cmask = real_enc_S ? fbuf((int64_t) S * enc_S) : NULL;
        for (int b = 0; b < N; b++) {
            if (cmask) {
                for (int i = 0; i < S; i++) {
                    for (int j = 0; j < enc_S; j++) {
                        cmask[(int64_t) i * enc_S + j] = j < real_enc_S[b] ? 0.0f : -INFINITY;
                    }
                }
            }
            orc_attention(q + (int64_t) b * S * qd, qd, ke + (int64_t) b * enc_S * kvd, ve + (int64_t) b * enc_S * kvd,
                          ORC_F32, kvd, D, cmask, att + (int64_t) b * S * qd, qd, S, enc_S, Nh, Nkv, D, scale);
        }
        free(cmask);
        rc |= linear(&ly->ca_o, att, R, o);
        add_inplace(hidden, o, R * H);
        free(kvb);
        free(ke);
        free(ve);
    }

    /* FFN with adaLN and gated residual */
    float * gu  = fbuf(R * 2 * F);
    float * act = fbuf(R * F);
    orc_adaln(hidden, (const float *) ly->mlp_norm.data, m->eps, scale_ff, shift_ff, 0, norm, 1, R, H);
    rc |= linear(&ly->gate_up, norm, R, gu);
    orc_swiglu(gu, 2 * F, gu + F, 2 * F, act, R, F);
    rc |= linear(&ly->down, act, R, o);
    orc_gated_residual(hidden, o, gate_ff, 0, hidden, 1, R, H);

    free(gu);
    free(act);
    free(ada);
    free(norm);
    free(qkv);
    free(q);
    free(k);
    free(v);
    free(att);
    free(o);
    return rc ? -1 : 0;
}

int orc_dit_forward(const orc_dit * m, const float * input, const float * enc_in, int N, int T, int enc_S, float t,
                    float t_r, float * velocity, int n_layers_run) {
    return orc_dit_forward_masked(m, input, enc_in, N, T, enc_S, t, t_r, velocity, n_layers_run, NULL, NULL);
}

/* One evaluation in three parts, so that a caller can run the layers in slices (the CPU
 * baseline times real layers of a full-depth evaluation a few at a time). */
struct orc_dit_state {
    int       N, T, S, enc_S, rc;
    int *     real_S;
    int *     real_enc_S;
    float *   temb;
    float *   tproj;
    float *   hidden;
    float *   enc;
    float *   rope;
};

orc_dit_state * orc_dit_begin(const orc_dit * m, const float * input, const float * enc_in, int N, int T, int enc_S,
                              float t, float t_r, const int * real_S, const int * real_enc_S) {
    const int H = m->H, P = m->P;
    if (T % P != 0) {
        return NULL;
    }
    const int       S = T / P;
    const int64_t   R = (int64_t) N * S;
    orc_dit_state * st = (orc_dit_state *) calloc(1, sizeof(orc_dit_state));
    st->N = N, st->T = T, st->S = S, st->enc_S = enc_S;
    if (real_S) {
        st->real_S = (int *) malloc(sizeof(int) * N);
        memcpy(st->real_S, real_S, sizeof(int) * N);
    }
    if (real_enc_S) {
        st->real_enc_S = (int *) malloc(sizeof(int) * N);
        memcpy(st->real_enc_S, real_enc_S, sizeof(int) * N);
    }
    int rc = 0;
    /* timestep embeddings: t and t - t_r, summed (dit-graph.h:537-562) */
    st->temb       = fbuf(H);
    st->tproj      = fbuf(6 * H);
    float * temb_r = fbuf(H);
    float * tprojr = fbuf(6 * H);
    rc |= orc_dit_timestep(m, &m->te, t, st->temb, st->tproj);
    rc |= orc_dit_timestep(m, &m->te_r, t - t_r, temb_r, tprojr);
    for (int i = 0; i < H; i++) {
        st->temb[i] = st->temb[i] + temb_r[i];
    }
    for (int i = 0; i < 6 * H; i++) {
        st->tproj[i] = st->tproj[i] + tprojr[i];
    }
    free(temb_r);
    free(tprojr);

    /* proj_in on the patchified input: [N][S][in_ch*P] is a reshape of [N][T][in_ch] */
    st->hidden = fbuf(R * H);
    rc |= linear(&m->proj_in_w, input, R, st->hidden);
    add_bias(st->hidden, R, H, &m->proj_in_b);

    /* condition embedder */
    st->enc = fbuf((int64_t) N * enc_S * H);
    rc |= linear(&m->cond_w, enc_in, (int64_t) N * enc_S, st->enc);
    add_bias(st->enc, (int64_t) N * enc_S, H, &m->cond_b);

    /* positions 0..S-1 per batch element */
    int32_t * pos = (int32_t *) malloc(sizeof(int32_t) * S);
    st->rope      = fbuf((int64_t) S * m->D);
    for (int i = 0; i < S; i++) {
        pos[i] = i;
    }
    orc_rope_cache(st->rope, pos, S, m->D, m->rope_theta);
    free(pos);
    st->rc = rc;
    return st;
}

int orc_dit_run_layers(const orc_dit * m, orc_dit_state * st, int l0, int l1) {
    if (!st || l0 < 0 || l1 > m->n_layers) {
        return -1;
    }
    for (int l = l0; l < l1 && st->rc == 0; l++) {
        st->rc |= dit_layer(m, &m->layers[l], st->hidden, st->enc, st->N, st->S, st->enc_S, st->tproj, st->rope,
                            st->real_S, st->real_enc_S);
    }
    return st->rc ? -1 : 0;
}

int orc_dit_finish(const orc_dit * m, orc_dit_state * st, float * velocity) {
    const int     H = m->H, P = m->P;
    const int64_t R = (int64_t) st->N * st->S;
    int           rc = st->rc;
    /* output adaLN + proj_out (dit-graph.h:588-612) */
    const float * oss       = (const float *) m->out_ss.data;
    float *       out_shift = fbuf(H);
    float *       out_scale = fbuf(H);
    for (int i = 0; i < H; i++) {
        out_shift[i] = oss[i] + st->temb[i];
        out_scale[i] = oss[H + i] + st->temb[i];
    }
    float * norm = fbuf(R * H);
    orc_adaln(st->hidden, (const float *) m->norm_out.data, m->eps, out_scale, out_shift, 0, norm, 1, R, H);
    rc |= linear(&m->proj_out_w, norm, R, velocity);
    add_bias(velocity, R, (int64_t) m->out_ch * P, &m->proj_out_b);
    free(out_shift);
    free(out_scale);
    free(norm);
    return rc ? -1 : 0;
}

void orc_dit_state_free(orc_dit_state * st) {
    if (!st) {
        return;
    }
    free(st->real_S);
    free(st->real_enc_S);
    free(st->temb);
    free(st->tproj);
    free(st->hidden);
    free(st->enc);
    free(st->rope);
    free(st);
}

int orc_dit_forward_masked(const orc_dit * m, const float * input, const float * enc_in, int N, int T, int enc_S,
                           float t, float t_r, float * velocity, int n_layers_run, const int * real_S,
                           const int * real_enc_S) {
    orc_dit_state * st = orc_dit_begin(m, input, enc_in, N, T, enc_S, t, t_r, real_S, real_enc_S);
    if (!st) {
        return -1;
    }
    const int nl = n_layers_run < 0 || n_layers_run > m->n_layers ? m->n_layers : n_layers_run;
    int       rc = orc_dit_run_layers(m, st, 0, nl);
    rc |= orc_dit_finish(m, st, velocity);
    orc_dit_state_free(st);
    return rc ? -1 : 0;
}
