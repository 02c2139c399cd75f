/*
 * acb_models.h -- model-level C ABI of libacb: the GGUF reader and the Qwen3 causal LM with its
 * f16 KV cache, with the same entry points, argument meaning and ownership as acestep.cpp's
 * header-only drivers (src/gguf-weights.h, src/qwen3-lm.h), backed by the sm_100a kernels of
 * acb.h. Differences from the reference are limited to error reporting: every function returns
 * an acb_status where the reference calls exit(1) or returns silently.
 */
#ifndef ACB_MODELS_H
#define ACB_MODELS_H

#include "acb.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ---- GGUF (replaces gf_load / gf_close / gf_get_*, src/gguf-weights.h:48-155,357-390) ---- */

typedef struct acb_gguf acb_gguf;

/* mmap + parse + per-tensor truncation check (gguf-weights.h:74-155). */
ACB_API acb_status   acb_gguf_open(const char * path, acb_gguf ** out);
ACB_API void         acb_gguf_close(acb_gguf * g);                              /* gf_close :48 */
ACB_API int64_t      acb_gguf_n_tensors(const acb_gguf * g);
ACB_API int64_t      acb_gguf_find_tensor(const acb_gguf * g, const char * name); /* -1 if absent */
ACB_API acb_status   acb_gguf_tensor_info(const acb_gguf * g, int64_t idx, const char ** name, int * type,
                                          int * n_dims, int64_t * ne4, const void ** data, size_t * nbytes);
ACB_API uint32_t     acb_gguf_get_u32(const acb_gguf * g, const char * key);     /* gf_get_u32 :357 */
ACB_API float        acb_gguf_get_f32(const acb_gguf * g, const char * key);     /* gf_get_f32 :367 */
ACB_API const char * acb_gguf_get_str(const acb_gguf * g, const char * key);     /* gf_get_str :377 */
ACB_API int          acb_gguf_get_bool(const acb_gguf * g, const char * key);    /* gf_get_bool :387 */
ACB_API const char * acb_last_error(void); /* message of the last failed load in this thread */

/* ---- Qwen3 causal LM (replaces src/qwen3-lm.h) ---------------------------------------------- */

typedef struct acb_qw3lm acb_qw3lm;

/* Qwen3LMConfig (qwen3-lm.h:15-27), filled from acestep.config_json like qw3lm_load_config. */
typedef struct {
    int   vocab_size;
    int   hidden_size;
    int   intermediate_size;
    int   n_heads;
    int   n_kv_heads;
    int   head_dim;
    int   n_layers;
    float rope_theta;
    float rms_norm_eps;
    int   tie_embeddings;
    int   max_seq_len;
} acb_qw3lm_config;

/* qw3lm_load (qwen3-lm.h:242): weights in their GGUF types (Q||K||V and gate||up fused when
 * the types match), norms promoted to F32, a zeroed f16 KV cache of n_kv_sets sets of
 * max_seq_len positions (max_seq_len <= 0 keeps the config's 8192). `device` is the CUDA
 * ordinal the model lives on. */
ACB_API acb_status acb_qw3lm_load(const char * gguf_path, int max_seq_len, int n_kv_sets, int device,
                                  acb_qw3lm ** out);
ACB_API acb_status acb_qw3lm_get_config(const acb_qw3lm * m, acb_qw3lm_config * cfg);
ACB_API size_t     acb_qw3lm_weight_bytes(const acb_qw3lm * m);

/* qw3lm_forward (qwen3-lm.h:429): prefill n_tokens into kv_set from its current position;
 * logits (host, [vocab_size]) of the last token. ACB_ERR_OUT_OF_RANGE if the cache would
 * overflow or an id is outside the vocabulary. */
ACB_API acb_status acb_qw3lm_forward(acb_qw3lm * m, const int32_t * token_ids, int n_tokens, int kv_set,
                                     float * logits);

/* qw3lm_forward_batch (qwen3-lm.h:557): one token per sequence for N consecutive kv sets
 * (kv_sets[i] == kv_sets[0] + i, the reference's assumption at :709); logits (host) [N][out_V]
 * with out_V = lm_count when lm_count > 0 and a partial head for lm_offset was built, else the
 * full vocabulary. */
ACB_API acb_status acb_qw3lm_forward_batch(acb_qw3lm * m, const int32_t * token_ids, const int32_t * kv_sets, int N,
                                           float * logits, int lm_offset, int lm_count);

ACB_API void       acb_qw3lm_reset_kv(acb_qw3lm * m, int kv_set);            /* qw3lm_reset_kv :227 */
ACB_API acb_status acb_qw3lm_copy_kv(acb_qw3lm * m, int src, int dst);       /* qw3lm_copy_kv :233 */
ACB_API acb_status acb_qw3lm_build_partial_head(acb_qw3lm * m, int lm_offset); /* :290 */
ACB_API int        acb_qw3lm_kv_pos(const acb_qw3lm * m, int kv_set);
ACB_API void       acb_qw3lm_free(acb_qw3lm * m);                             /* qw3lm_free :826 */

/* Greedy (temperature 0) decode of n_steps tokens for N consecutive kv sets, entirely on the
 * device: the step (embedding gather, every layer, full-vocabulary head, argmax) is captured
 * once as a CUDA graph and replayed, each step's argmax feeding the next step's gather.
 * last_ids[N] are the tokens to feed first (at the sets' current positions); tokens_out
 * [N][n_steps] and margins_out [N][n_steps] (top1 - top2 logit, optional) are host arrays.
 * gpu_ms (optional) receives the device time of the replay loop. Replaces the temperature-0
 * path of the phase-2 decode loop (src/pipeline-lm.cpp:427-523). */
ACB_API acb_status acb_qw3lm_generate_greedy(acb_qw3lm * m, const int32_t * last_ids, int set0, int N, int n_steps,
                                             int32_t * tokens_out, float * margins_out, float * gpu_ms);

#ifdef __cplusplus
}
#endif
#endif
