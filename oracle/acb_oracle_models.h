/*
 * acb_oracle_models.h -- CPU oracle of the three model forwards whose per-layer op-chain the
 * CUDA path replaces. TEST INFRASTRUCTURE ONLY (see acb_oracle.h).
 *
 *   orc_qwen3_encode   qwen3_forward          (src/qwen3-enc.h:373-448)
 *   orc_qw3lm_prefill  qw3lm_forward          (src/qwen3-lm.h:429-549)
 *   orc_qw3lm_decode   qw3lm_forward_batch    (src/qwen3-lm.h:557-823)
 *   orc_dit_forward    dit_ggml_build_graph   (src/dit-graph.h:466-619), one evaluation
 *
 * Weights are given as orc_tensor views of raw GGUF tensor bytes. A linear weight is N rows
 * of K elements (ggml [K, N]); fused Q||K||V and gate||up are row concatenations, exactly as
 * gf_load_qkv_fused / gf_load_pair_fused build them (src/gguf-weights.h:281-354).
 */
#ifndef ACB_ORACLE_MODELS_H
#define ACB_ORACLE_MODELS_H

#include "acb_oracle.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    int          type;
    const void * data;
    int64_t      K; /* elements per row (ne0) */
    int64_t      N; /* rows (ne1) */
} orc_tensor;

typedef struct {
    orc_tensor attn_norm; /* F32 [H] */
    orc_tensor qkv;       /* [H -> (Nh + 2 Nkv) D]; data NULL: use q, k, v below */
    orc_tensor q_norm;    /* F32 [D] */
    orc_tensor k_norm;    /* F32 [D] */
    orc_tensor o;         /* [Nh D -> H] */
    orc_tensor post_norm; /* F32 [H] */
    orc_tensor gate_up;   /* [H -> 2 F]; data NULL: use gate, up below */
    orc_tensor down;      /* [F -> H] */
    orc_tensor q, k, v;   /* unfused projections (types differ, as gf_load_qkv_fused refuses) */
    orc_tensor gate, up;
} orc_qwen3_layer;

typedef struct {
    int                     n_layers, H, F, Nh, Nkv, D, V;
    float                   rope_theta, eps;
    orc_tensor              embed;      /* [H, V]: V rows of H */
    orc_tensor              final_norm; /* F32 [H] */
    const orc_qwen3_layer * layers;
} orc_qwen3;

/* KV cache: f16, layout [L][n_sets][Nkv][max_seq][D] (per layer the reference's 4-D
 * [D, max_seq, Nkv, n_sets] tensor, qwen3-lm.h:173-224). */
typedef struct {
    uint16_t * k;
    uint16_t * v;
    int        n_sets;
    int        max_seq;
} orc_kv;

/* Text-encoder forward: ids[S] -> out[S][H] (post final norm), causal, f32 attention. */
int orc_qwen3_encode(const orc_qwen3 * m, const int32_t * ids, int S, float * out);

/* qwen3_build_layers (src/qwen3-enc.h:249-262) over layers [l0, l1) from given hidden states
 * (in place, [S][H]), positions 0..S-1, causal or unmasked attention; out (optional) receives
 * the final RMSNorm of the result. The encoder callers that start from a projection
 * (cond_ggml_forward) and per-layer parity checks use it. */
int orc_qwen3_layers(const orc_qwen3 * m, float * hidden, int S, int l0, int l1, int causal, float * out);

/* orc_qwen3_layers over B independent sequences of S rows each (hidden [B*S][H], positions
 * 0..S-1 in every sequence, attention within a sequence), and with window > 0 on a bidirectional
 * stack the sliding-window mask |i - j| <= window on the even layers (the lyric and timbre
 * encoders, src/cond-enc.h:203-212, 263-272). B > 1 is the reference's loop of one graph per
 * group (fsq-tok.h:208-223, fsq-detok.h:193-205) done as one call: every linear is row-wise. */
int orc_qwen3_layers_ex(const orc_qwen3 * m, float * hidden, int B, int S, int l0, int l1, int causal, int window,
                        float * out);

/* LM prefill of n tokens into kv set `set` starting at position kv_pos; writes the f16 K/V,
 * returns the logits of the last token in logits[V] (or lm rows [lm_offset, lm_offset+lm_count)
 * when lm_count > 0). If hidden_out is non-NULL it receives the final-normed hidden rows
 * [n][H]. */
int orc_qw3lm_prefill(const orc_qwen3 * m, orc_kv * kv, int set, int kv_pos, const int32_t * ids, int n,
                      float * logits, int lm_offset, int lm_count, float * hidden_out);

/* Batched one-token decode: token ids[N] for consecutive sets set0..set0+N-1 whose current
 * positions are kv_pos[N]; logits [N][out_V]. */
int orc_qw3lm_decode(const orc_qwen3 * m, orc_kv * kv, int set0, const int32_t * kv_pos, const int32_t * ids, int N,
                     float * logits, int lm_offset, int lm_count);

typedef struct {
    orc_tensor l1_w, l1_b; /* [256 -> H], F32 [H] */
    orc_tensor l2_w, l2_b; /* [H -> H], F32 [H] */
    orc_tensor tp_w, tp_b; /* [H -> 6H], F32 [6H] */
} orc_dit_temb;

typedef struct {
    orc_tensor sa_norm;            /* F32 [H] */
    orc_tensor sa_qkv;             /* [H -> (Nh + 2 Nkv) D] */
    orc_tensor sa_q_norm, sa_k_norm;
    orc_tensor sa_o;               /* [Nh D -> H] */
    orc_tensor ca_norm;            /* F32 [H] */
    orc_tensor ca_qkv;             /* [H -> (Nh + 2 Nkv) D]: q rows from hidden, k||v rows from enc */
    orc_tensor ca_q_norm, ca_k_norm;
    orc_tensor ca_o;               /* [Nh D -> H] */
    orc_tensor mlp_norm;           /* F32 [H] */
    orc_tensor gate_up;            /* [H -> 2 F] */
    orc_tensor down;               /* [F -> H] */
    orc_tensor scale_shift;        /* F32 [6][H] */
    int        layer_type;         /* 0 = sliding window, 1 = full (dit.h:399) */
} orc_dit_layer;

typedef struct {
    int                   n_layers, H, F, Nh, Nkv, D, in_ch, out_ch, P, sliding_window, H_enc;
    float                 rope_theta, eps;
    orc_dit_temb          te, te_r;
    orc_tensor            proj_in_w; /* F32 [in_ch*P -> H], input index j = p*in_ch + ic */
    orc_tensor            proj_in_b; /* F32 [H] */
    orc_tensor            cond_w;    /* [H_enc -> H] */
    orc_tensor            cond_b;    /* F32 [H] */
    const orc_dit_layer * layers;
    orc_tensor            norm_out;   /* F32 [H] */
    orc_tensor            out_ss;     /* F32 [2][H]: shift, scale */
    orc_tensor            proj_out_w; /* F32 [H -> out_ch*P], output index j = p*out_ch + oc */
    orc_tensor            proj_out_b; /* F32 [out_ch] */
} orc_dit;

/* One DiT evaluation: input [N][T][in_ch], enc [N][enc_S][H_enc] -> velocity [N][T][out_ch].
 * All frames and encoder rows are real (no padding masks). n_layers_run < 0 runs every layer;
 * otherwise only the first n_layers_run layers (the CPU-baseline sample). */
int orc_dit_forward(const orc_dit * m, const float * input, const float * enc, int N, int T, int enc_S, float t,
                    float t_r, float * velocity, int n_layers_run);

/* orc_dit_forward with the padding masks of dit_ggml_generate (dit-sampler.h:244-304): sequence b
 * has real_S[b] real patch positions (self-attention: query and key both real, and inside the
 * window on the sliding layers) and real_enc_S[b] real condition rows (cross-attention keys).
 * Either array may be NULL (every position real). A query row with no admitted key (a padded
 * position) gets a zero attention output: the masked keys are skipped and the empty sum gives 0,
 * as ggml's flash attention does. */
int orc_dit_forward_masked(const orc_dit * m, const float * input, const float * enc, int N, int T, int enc_S,
                           float t, float t_r, float * velocity, int n_layers_run, const int * real_S,
                           const int * real_enc_S);

/* The evaluation of orc_dit_forward_masked in parts: begin (timestep embeddings, proj_in, the
 * condition embedder), layers [l0, l1) on the carried hidden state, finish (output adaLN and
 * proj_out). Used to time full-depth evaluations a slice of layers at a time. */
typedef struct orc_dit_state orc_dit_state;
orc_dit_state * orc_dit_begin(const orc_dit * m, const float * input, const float * enc, int N, int T, int enc_S,
                              float t, float t_r, const int * real_S, const int * real_enc_S);
int             orc_dit_run_layers(const orc_dit * m, orc_dit_state * st, int l0, int l1);
int             orc_dit_finish(const orc_dit * m, orc_dit_state * st, float * velocity);
void            orc_dit_state_free(orc_dit_state * st);

/* Timestep projection of one embedder (dit-graph.h:81-117): temb[H], tproj[6H]. */
int orc_dit_timestep(const orc_dit * m, const orc_dit_temb * te, float t, float * temb, float * tproj);

#ifdef __cplusplus
}
#endif
#endif
