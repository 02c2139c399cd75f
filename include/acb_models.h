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

/* Cancellation callback, polled between steps of a long call (denoise steps, dit-sampler.h:409-413;
 * VAE tiles, vae.h:496): nonzero stops the call with ACB_ERR_CANCELLED. */
typedef int (*acb_cancel_fn)(void * data);

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

/* ---- Qwen3 encoder stack (replaces src/qwen3-enc.h) ------------------------------------------ */

typedef struct acb_qwen3_enc acb_qwen3_enc;

/* Qwen3Config (qwen3-enc.h:27-37) plus the embedding table's row count. */
typedef struct {
    int   hidden_size;
    int   intermediate_size;
    int   n_heads;
    int   n_kv_heads;
    int   head_dim;
    int   n_layers;
    float rope_theta;
    float rms_norm_eps;
    int   is_causal;
    int   vocab_size;
} acb_qwen3_config;

/* qwen3_load_text_encoder (qwen3-enc.h:319-367): tensors embed_tokens.weight, norm.weight and
 * layers.N.* (no "model." prefix), config 1024/3072/16/8/128/28 layers, rope theta 1e6,
 * eps 1e-6, causal -- the reference's constants; a GGUF carrying acestep.config_json may
 * override them (the shipped text encoder's config holds the same values). Every linear is
 * dequantised once to a resident f16 copy (bf16 for BF16 weights; Q||K||V and gate||up stacked
 * into one matrix) for the tensor-core GEMM, whose activations are quantised like ggml's
 * quantised mul_mat (acb_act_quant); the embedding table and norms keep their GGUF / F32
 * forms. `device` is the CUDA ordinal the model lives on. */
ACB_API acb_status acb_qwen3_load_text_encoder(const char * gguf_path, int device, acb_qwen3_enc ** out);
ACB_API acb_status acb_qwen3_get_config(const acb_qwen3_enc * m, acb_qwen3_config * cfg);
/* Arithmetic of the linears and attention: exact (the default, nonzero) forms every product of
 * the reference's dequantised operands from hi/lo f16 splits, tracking the reference CPU build to
 * fp32 summation order at 3x the tensor work; fast (0) uses single f16 operands. */
ACB_API acb_status acb_qwen3_set_exact(acb_qwen3_enc * m, int exact);
ACB_API size_t     acb_qwen3_weight_bytes(const acb_qwen3_enc * m); /* device bytes of all weights */

/* qwen3_forward (qwen3-enc.h:373-448): token ids (host, [S]) -> last-layer hidden states after
 * the final RMSNorm (host, caller-allocated [S][hidden_size] f32). ACB_ERR_OUT_OF_RANGE when an
 * id is outside the embedding table. */
ACB_API acb_status acb_qwen3_forward(acb_qwen3_enc * m, const int32_t * token_ids, int S, float * output);

/* The same forward on device buffers (ids [S] int32, out [S][hidden_size] f32), enqueued on
 * `stream` without a host synchronisation. The chain for each S is captured once as a CUDA
 * graph over the model's own scratch, so calls on one model must not overlap. Ids are not
 * range-checked on the host here; acb_qwen3_forward is the checked entry point. */
ACB_API acb_status acb_qwen3_forward_device(acb_qwen3_enc * m, const int32_t * d_ids, int S, float * d_out,
                                            acb_stream_t stream);
/* Kernel launches of the last forward of this stack (the nodes of its captured graph); 0 before the
 * first. No reference counterpart: an accounting query. */
ACB_API int        acb_qwen3_forward_kernels(const acb_qwen3_enc * m);

/* qwen3_build_layers (qwen3-enc.h:249-262) over layers [layer_begin, layer_end) from caller
 * hidden states (device, [S][hidden_size] f32; the condition encoders' entry, cond-enc.h:171,
 * which start from a projection instead of token ids), positions 0..S-1 and the model's own
 * masking; d_out receives the resulting hidden states, or their final RMSNorm when final_norm
 * is nonzero. Enqueued on `stream`, no graph, no host synchronisation. */
ACB_API acb_status acb_qwen3_forward_hidden(acb_qwen3_enc * m, const float * d_hidden, int S, int layer_begin,
                                            int layer_end, int final_norm, float * d_out, acb_stream_t stream);

/* qwen3_embed_lookup (qwen3-enc.h:453-480): embedding rows (host ids [S] -> host [S][H] f32). */
ACB_API acb_status acb_qwen3_embed_lookup(acb_qwen3_enc * m, const int32_t * token_ids, int S, float * output);
ACB_API void       acb_qwen3_free(acb_qwen3_enc * m); /* qwen3_free :483 */

/* ---- condition encoder (replaces src/cond-enc.h) --------------------------------------------- */

typedef struct acb_cond acb_cond;

/* Sizes of a loaded condition encoder: the packed output width, the two input widths, the stacks'
 * depths and whether the timbre stack prepends its learned CLS token (XL models, the GGUF key
 * acestep.encoder_hidden_size present). */
typedef struct {
    int hidden_size;   /* 2048: width of the packed encoder states */
    int text_dim;      /* 1024: text_projector input (Qwen3-Embedding states) */
    int lyric_dim;     /* 1024: lyric embed_tokens input */
    int timbre_dim;    /* 64: timbre embed_tokens input (VAE latent channels) */
    int lyric_layers;  /* 8 */
    int timbre_layers; /* 4 */
    int window;        /* 128: |i - j| <= window on the even layers of both stacks */
    int timbre_cls;    /* 1 when the timbre stack prepends its CLS token */
} acb_cond_config;

/* cond_ggml_load (cond-enc.h:86-164) from the DiT GGUF: encoder.lyric_encoder.* (8 layers),
 * encoder.timbre_encoder.* (4 layers, special_token when acestep.encoder_hidden_size > 0),
 * encoder.text_projector.weight and null_condition_emb. Linears become resident 16-bit copies
 * for the tensor-core GEMM as in acb_qwen3_load_text_encoder. */
ACB_API acb_status acb_cond_load(const char * gguf_path, int device, acb_cond ** out);
ACB_API acb_status acb_cond_get_config(const acb_cond * m, acb_cond_config * cfg);
/* exact (default) / fast arithmetic of every linear and attention, as acb_qwen3_set_exact. */
ACB_API acb_status acb_cond_set_exact(acb_cond * m, int exact);
/* cond_ggml_forward (cond-enc.h:171-381). Host f32 inputs, rows contiguous: text_hidden
 * [S_text][1024], lyric_embed [S_lyric][1024], timbre_feats [S_ref][64] (NULL or S_ref 0: no
 * timbre). enc_hidden (caller-allocated, (S_lyric + (timbre ? 1 : 0) + S_text) * hidden_size
 * floats) receives the packed states [lyric | timbre row 0 | text projection]; *out_enc_S their
 * row count. S_lyric >= 1 and S_text >= 1 as in the reference. */
ACB_API acb_status acb_cond_forward(acb_cond * m, const float * text_hidden, int S_text, const float * lyric_embed,
                                    int S_lyric, const float * timbre_feats, int S_ref, float * enc_hidden,
                                    int * out_enc_S);
/* The same on device buffers, enqueued on `stream` (no host synchronisation; calls on one model
 * must not overlap). */
ACB_API acb_status acb_cond_forward_device(acb_cond * m, const float * d_text_hidden, int S_text,
                                           const float * d_lyric_embed, int S_lyric, const float * d_timbre_feats,
                                           int S_ref, float * d_enc_hidden, int * out_enc_S, acb_stream_t stream);
/* null_condition_emb as f32 [hidden_size] (host): the unconditional row of classifier-free
 * guidance (CondGGML.null_cond_emb). */
ACB_API acb_status acb_cond_null_embedding(acb_cond * m, float * out);
ACB_API void       acb_cond_free(acb_cond * m); /* cond_ggml_free :383 */

/* ---- VAE decoder (replaces src/vae.h) --------------------------------------------------------- */

typedef struct acb_vae acb_vae;

/* vae_ggml_load (vae.h:167-259): decoder.* of an acestep-vae GGUF (BF16 weight_g / weight_v,
 * biases, snake alpha / beta). Weight normalisation is fused at load as the reference does it and
 * the weights kept in f16; channels and strides come from the tensor shapes (channel counts must
 * be multiples of 64). */
ACB_API acb_status acb_vae_load(const char * gguf_path, int device, acb_vae ** out);
ACB_API int        acb_vae_upsample(const acb_vae * m); /* audio samples per latent frame (1920) */
/* vae_ggml_decode (vae.h:442-459): latent [T_latent][64] (host, time-major as the DiT writes it)
 * -> audio_out [2][T_audio] (host: channel 0 then channel 1), T_audio = T_latent * upsample <=
 * max_T_audio. Convolutions run as tcgen05 GEMMs on f16 operands (ggml's conv_1d casts the
 * activation to the f16 weights), snake activations in f32. */
ACB_API acb_status acb_vae_decode(acb_vae * m, const float * latent, int T_latent, float * audio_out,
                                  int max_T_audio, int * out_T_audio);
/* vae_ggml_decode_tiled (vae.h:467-565): the same windows (chunk_size frames plus overlap of
 * context each side, reference defaults 256 / 64), trims and layout; cancel is polled per tile. */
ACB_API acb_status acb_vae_decode_tiled(acb_vae * m, const float * latent, int T_latent, float * audio_out,
                                        int max_T_audio, int chunk_size, int overlap, acb_cancel_fn cancel,
                                        void * cancel_data, int * out_T_audio);
/* Device buffers: d_latent [T_latent][64] -> d_audio [2][T_latent * upsample]; synchronises. */
ACB_API acb_status acb_vae_decode_device(acb_vae * m, const float * d_latent, int T_latent, float * d_audio,
                                         acb_stream_t stream);
ACB_API void       acb_vae_free(acb_vae * m); /* vae_ggml_free :567 */

/* ---- FSQ detokenizer and tokenizer (replace src/fsq-detok.h, src/fsq-tok.h) ------------------ */

/* The FSQ alphabet: 6 dimensions of {8, 8, 8, 5, 5, 5} levels, 64000 codes. Host helpers with the
 * reference's arithmetic: fsq_decode_index (fsq-detok.h:18-29) and fsq_encode_index
 * (fsq-tok.h:42-60). */
ACB_API void acb_fsq_decode_index(int index, float * out6);
ACB_API int  acb_fsq_encode_index(const float * raw6);

typedef struct acb_detok acb_detok;

/* detok_ggml_load (fsq-detok.h:70-122): tokenizer.quantizer.project_out.*, detokenizer.* (2-layer
 * bidirectional stack, special_tokens [5][2048], proj_out 2048 -> 64) from the DiT GGUF. */
ACB_API acb_status acb_detok_load(const char * gguf_path, int device, acb_detok ** out);
ACB_API acb_status acb_detok_set_exact(acb_detok * m, int exact);
/* detok_ggml_decode (fsq-detok.h:128-212): codes [T_5Hz] (host) -> context_out [T_5Hz * 5][64]
 * (host, caller-allocated). Every code is decoded in one batch (5 frames per code, attention
 * within a code's frames). ACB_ERR_OUT_OF_RANGE for a negative code. */
ACB_API acb_status acb_detok_decode(acb_detok * m, const int * codes, int T_5Hz, float * context_out);
/* The same on device buffers (codes int32 [T_5Hz], out f32 [T_5Hz * 5][64]), enqueued on stream;
 * a negative code gives a zero row and ACB_DEVERR_CODE_RANGE in the model's device flag, which
 * acb_detok_decode checks. */
ACB_API acb_status acb_detok_decode_device(acb_detok * m, const int32_t * d_codes, int T_5Hz, float * d_out,
                                           acb_stream_t stream);
ACB_API void       acb_detok_free(acb_detok * m); /* detok_ggml_free :215 */

typedef struct acb_tok acb_tok;

/* tok_ggml_load (fsq-tok.h:63-126): tokenizer.audio_acoustic_proj.*, tokenizer.attention_pooler.*
 * (embed, special_token, 2-layer stack, norm) and tokenizer.quantizer.project_in.*. */
ACB_API acb_status acb_tok_load(const char * gguf_path, int device, acb_tok ** out);
ACB_API acb_status acb_tok_set_exact(acb_tok * m, int exact);
/* tok_ggml_encode (fsq-tok.h:133-238): latents [T_25Hz][64] (host) padded to a multiple of 5 with
 * the first rows of silence_latent ([>= 4][64], required when T_25Hz % 5 != 0) -> codes_out
 * [(T_25Hz + 4) / 5] (host); *out_T_5Hz receives the count. All groups run as one batch. */
ACB_API acb_status acb_tok_encode(acb_tok * m, const float * latents, int T_25Hz, int * codes_out,
                                  const float * silence_latent, int * out_T_5Hz);
/* The same on device buffers: latents f32 [T_5Hz * 5][64] already padded, codes int32 [T_5Hz]. */
ACB_API acb_status acb_tok_encode_device(acb_tok * m, const float * d_latents, int T_5Hz, int32_t * d_codes,
                                         acb_stream_t stream);
ACB_API void       acb_tok_free(acb_tok * m); /* tok_ggml_free :241 */

/* ---- ACE-Step DiT (replaces src/dit.h, src/dit-graph.h, src/dit-sampler.h) ------------------- */

typedef struct acb_dit acb_dit;

/* DiTGGMLConfig (dit.h) from the GGUF keys acestep-dit.* / acestep.*, plus the condition width
 * (condition_embedder input) and whether null_condition_emb (CFG) is present. */
typedef struct {
    int   n_layers;
    int   hidden_size;
    int   intermediate_size;
    int   n_heads;
    int   n_kv_heads;
    int   head_dim;
    int   in_channels;
    int   out_channels;
    int   patch_size;
    int   sliding_window;
    float rope_theta;
    float rms_norm_eps;
    int   enc_hidden_size;
    int   has_null_condition;
} acb_dit_config;

/* dit_ggml_load (dit.h:256-420): decoder.* tensors, proj_in / proj_out pre-permuted to F32 at
 * load, every linear dequantised once to a resident 16-bit copy ([hi|lo|hi] f16 for quantised and
 * F32 weights, see acb_act_quant_ex) for the tensor-core GEMM. */
ACB_API acb_status acb_dit_load(const char * gguf_path, int device, acb_dit ** out);
/* dit_ggml_load with an adapter (dit.h:421-428, adapter_merge): the LoRA at adapter_path (a PEFT
 * directory with adapter_model.safetensors and adapter_config.json, or one safetensors file) is
 * merged into the decoder weights at load with user scale adapter_scale, before the resident
 * copies are built: base dequantised, + bf16(alpha/rank * scale * B.A), requantised to its GGUF
 * type on the device (Q8_0 with ggml's quantiser; Q4_K / Q6_K with this library's encoders, which
 * choose their scales differently from ggml's search). A LyCORIS LoKr file (lycoris_<path> modules,
 * adapter_merge_lokr) merges base + bf16(kron(w1 * alpha/rank, W2)) * scale, or with a
 * dora_scale vector the weight decomposition of acb_lokr_delta_add. adapter_path NULL is
 * acb_dit_load; ACB_ERR_FORMAT when no pair or module matches a weight. */
ACB_API acb_status acb_dit_load_ex(const char * gguf_path, int device, const char * adapter_path,
                                   float adapter_scale, acb_dit ** out);
ACB_API acb_status acb_dit_get_config(const acb_dit * m, acb_dit_config * cfg);
ACB_API size_t     acb_dit_weight_bytes(const acb_dit * m);
/* exact (default, nonzero): hi/lo split products, tracking the reference CPU build to fp32
 * summation order at 3x tensor work; fast (0): single f16 operands. */
ACB_API acb_status acb_dit_set_exact(acb_dit * m, int exact);

/* One DiT evaluation (dit_ggml_build_graph + compute, dit-graph.h:466-619) on device buffers:
 * input [N][T][in_channels] (context channels then xt), enc [N][enc_S][enc_hidden_size] ->
 * velocity [N][T][out_channels]; t and t_r the two timesteps (time_embed_r sees t - t_r).
 * n_layers_run < 0 runs every layer, else only the first n_layers_run (then the output stage).
 * All frames and condition rows are real (no padding masks). Synchronises `stream`. */
ACB_API acb_status acb_dit_forward(acb_dit * m, const float * d_input, const float * d_enc, int N, int T, int enc_S,
                                   float t, float t_r, float * d_velocity, int n_layers_run, acb_stream_t stream);

/* Padding for the acb_dit_set_condition / acb_dit_eval path (dit-sampler.h:244-304): host arrays of
 * the slots' real patch positions (self-attention queries and keys) and real condition rows
 * (cross-attention keys), one value per sequence of the last acb_dit_set_condition (NULL: all
 * real). acb_dit_set_condition and acb_dit_forward reset both to "all real". Enqueued on stream. */
ACB_API acb_status acb_dit_set_lengths(acb_dit * m, const int * real_S, const int * real_enc_S, acb_stream_t stream);
/* The two halves of acb_dit_forward for callers that run their own step loop (e.g. sequences
 * sharded over GPUs): set_condition embeds enc [N][enc_S][enc_hidden_size] (device) and caches
 * every layer's cross-attention K/V for N sequences of T frames; eval runs one evaluation of
 * input [N][T][in_channels] (device) with tt = {t, t_r} (device floats) into velocity, as one
 * CUDA graph per shape (captured on first use), enqueued on `stream` without synchronising. */
ACB_API acb_status acb_dit_set_condition(acb_dit * m, const float * d_enc, int N, int T, int enc_S,
                                         acb_stream_t stream);
ACB_API acb_status acb_dit_eval(acb_dit * m, const float * d_input, const float * tt, float * d_velocity,
                                acb_stream_t stream);
/* Kernel launches in the last captured evaluation graph (0 before the first acb_dit_eval). */
ACB_API int        acb_dit_eval_kernels(const acb_dit * m);
/* Kernel launches of this library in the last denoise step run by the generate / job drivers:
 * the nodes of its step graph(s) (evaluation, guidance, solver) plus a DCW launch; the STORK4
 * step's adaptive launches and the NCCL exchange are not counted. 0 before the first step. No
 * reference counterpart: an accounting query. */
ACB_API int        acb_dit_step_kernels(const acb_dit * m);

/* dit_ggml_generate (dit-sampler.h:132-711) with the Euler solver, host arrays as in the reference:
 * noise [N][T][out_channels], context_latents [N][T][in_channels - out_channels], enc_hidden
 * [N][enc_S][enc_hidden_size], schedule[num_steps] -> output [N][T][out_channels] (the x0
 * prediction of the last step). guidance_scale > 1 with a null condition runs batched CFG
 * (2N sequences per evaluation) with APG. Each step is one CUDA graph (captured on first use per
 * shape); gpu_ms (optional) receives the device time of the step loop. The full argument list
 * (padding masks, cancellation, cover mode, the SDE solver) is acb_dit_generate_ex. */
ACB_API acb_status acb_dit_generate(acb_dit * m, const float * noise, const float * context_latents,
                                    const float * enc_hidden, int enc_S, int T, int N, int num_steps,
                                    const float * schedule, float * output, float guidance_scale, float * gpu_ms);
/* Solvers (the registry keys of solvers/solver-registry.h:30-33: "euler", "dpm3m", "sde"). */
enum { ACB_SOLVER_EULER = 0, ACB_SOLVER_DPM3M = 1, ACB_SOLVER_SDE = 2, ACB_SOLVER_STORK4 = 3 };

/* ---- STORK4 solver (replaces src/solvers/solver-stork.h) ------------------------------------- */

/* The ROCK4 tables STORK4 runs on (Abdulle 2002; the reference compiles them in as STORK4_MS,
 * STORK4_FPA, STORK4_FPB, STORK4_RECF in solver-stork4-constants.h): ms[ms_len] increasing degrees,
 * fpa[ms_len][6] and fpb[ms_len][4] finishing coefficients, recf[recf_len] recurrence
 * coefficients. The library keeps its own copy. */
typedef struct {
    const int *    ms;
    int            ms_len;
    const double * fpa;
    const double * fpb;
    const double * recf;
    int            recf_len;
} acb_stork4_tables;

typedef struct acb_stork4 acb_stork4;

/* STORK4 state for latents of n floats on the current device (solver_stork4_step,
 * solver-stork.h:270-315; SolverState's velocity history and step index): substeps <= 0 takes the
 * reference's 10. */
ACB_API acb_status acb_stork4_create(const acb_stork4_tables * tables, int64_t n, int substeps, acb_stork4 ** out);
/* One step on device buffers: xt [n] in place from vt [n] (the guided velocity) between t_curr and
 * t_prev. Step 0 is Euler; later steps take velocity derivatives from the history (orders 2 / 1 / 0
 * by the reference's stability guards), run the ROCK4 sub stepping (one fused pass per attempt,
 * the sub step count halved while the result is not finite) or fall back to Euler. Synchronises
 * `stream` (the adaptive choice is made on the host). */
ACB_API acb_status acb_stork4_step(acb_stork4 * st, float * xt, const float * vt, float t_curr, float t_prev,
                                   acb_stream_t stream);
ACB_API void       acb_stork4_reset(acb_stork4 * st);
ACB_API int        acb_stork4_step_index(const acb_stork4 * st);
ACB_API void       acb_stork4_free(acb_stork4 * st);

/* The ROCK4 tables for the "stork4" solver of acb_dit_generate_ex / acb_dit_generate_sharded /
 * acb_dit_job_begin (copied; without them that solver returns ACB_ERR_UNSUPPORTED). */
ACB_API acb_status acb_dit_set_stork4_tables(acb_dit * m, const acb_stork4_tables * tables);
/* acb_dit_generate with dit_ggml_generate's solver choice (dit-sampler.h:391-398, 608-611): Euler or
 * DPM++ 3M (acb_dit_dpm3m on the velocity after guidance, its history on the device; the last
 * step is the x0 prediction for every solver). Other solver values: ACB_ERR_INVALID_ARG. */
ACB_API acb_status acb_dit_generate_solver(acb_dit * m, const float * noise, const float * context_latents,
                                           const float * enc_hidden, int enc_S, int T, int N, int num_steps,
                                           const float * schedule, float * output, float guidance_scale, int solver,
                                           float * gpu_ms);
/* Host noise source of the SDE solver: n N(0,1) samples of the stream seeded with `seed` into out.
 * The reference's is philox_randn(seed, out, n, true) (src/philox.h: Philox4x32-10, rounded to
 * bf16). With no source (NULL) the library draws that same stream on the device inside the step
 * (acb_dit_sde_philox), with no host fill and no copy. */
typedef void (*acb_randn_fn)(int64_t seed, float * out, int n, void * data);
/* dit_ggml_generate (src/dit-sampler.h:132-711) argument for argument, host arrays as in the
 * reference:
 *   noise [N][T][Oc], context_latents [N][T][in_ch - Oc], enc_hidden [N][enc_S][enc_hidden_size],
 *   schedule[num_steps] -> output [N][T][Oc] (x0 of the last step), guidance_scale (> 1 with a
 *   null condition: batched CFG with APG);
 *   context_switch / cover_steps / enc_switch / real_enc_S_switch: cover mode (:414-449): from
 *   step cover_steps on, every slot's context is context_switch and the conditional slots'
 *   condition is enc_switch with lengths real_enc_S_switch (the unconditional slots keep theirs);
 *   cancel(cancel_data): polled before every step; nonzero stops with ACB_ERR_CANCELLED (at most
 *   two steps are queued on the GPU, so it takes effect within two steps);
 *   real_S[N] / real_enc_S[N]: padding masks (:244-304; NULL: no padding);
 *   seeds[N] + randn / randn_data: the SDE solver's per-step noise (seed_b + step + 1): randn
 *   NULL draws it on the device (the reference's philox_randn stream), else on the host;
 *   use_batch_cfg: accepted, both values run the batched graph (results equal up to summation order);
 *   dcw_scaler / dcw_high_scaler / dcw_mode: DCW after every ODE step but the last (either scaler
 *   > 0; modes "low" (also NULL or unknown), "high", "double", "pix"; acb_dit_dcw), not with SDE;
 *   solver_name: "euler" (also NULL / ""), "dpm3m", "sde", "stork4" (after
 *   acb_dit_set_stork4_tables; before it ACB_ERR_UNSUPPORTED); any other name falls back to Euler,
 *   as solver_lookup's caller does;
 *   gpu_ms (optional): device time of the step loop.
 * Returns ACB_OK where the reference returns 0. */
ACB_API acb_status acb_dit_generate_ex(acb_dit * m, const float * noise, const float * context_latents,
                                       const float * enc_hidden, int enc_S, int T, int N, int num_steps,
                                       const float * schedule, float * output, float guidance_scale,
                                       const float * context_switch, int cover_steps, acb_cancel_fn cancel,
                                       void * cancel_data, const int * real_S, const int * real_enc_S,
                                       const float * enc_switch, const int * real_enc_S_switch, const int64_t * seeds,
                                       int use_batch_cfg, float dcw_scaler, float dcw_high_scaler,
                                       const char * dcw_mode, const char * solver_name, int stork_substeps,
                                       acb_randn_fn randn, void * randn_data, float * gpu_ms);
ACB_API void       acb_dit_free(acb_dit * m);

/* ---- several GPUs (one process per GPU) ------------------------------------------------------
 * The reference runs one GPU per process (ace-server pins workers with CUDA_VISIBLE_DEVICES,
 * tools/ace-server.cpp:2095-2120) and has no collectives. These entry points let a C/C++ host shard
 * one DiT job over the GPUs of a node: every rank holds a full copy of the weights and evaluates
 * its own sequences; NCCL (libnccl.so.2, opened at run time) moves the per-step velocity between
 * the two ranks of a split CFG pair and gathers the finished latents. Every wait on peers is
 * bounded by the communicator's timeout: on expiry the communicator is aborted and the call
 * returns ACB_ERR_TIMEOUT. */
typedef struct acb_comm acb_comm;
/* 128-byte NCCL unique id, made on one rank and handed to the others by the host's own channel. */
ACB_API acb_status acb_comm_unique_id(void * id128);
ACB_API acb_status acb_comm_init(const void * id128, int world, int rank, int device, int timeout_ms, acb_comm ** out);
ACB_API int        acb_comm_rank(const acb_comm * c);
ACB_API int        acb_comm_world(const acb_comm * c);
ACB_API void       acb_comm_free(acb_comm * c);

/* Which tracks rank `rank` of `world` evaluates in a job of n_tracks (host logic only): when world
 * divides n_tracks, the whole track pairs [track0, track0 + n_local) (half = -1, no exchange during
 * the steps); with CFG and world == 2 * n_tracks, one half of track rank / 2 (half 0 conditional,
 * 1 unconditional) whose other half is on rank `peer` (one velocity exchange per step). Otherwise
 * ACB_ERR_UNSUPPORTED. */
ACB_API acb_status acb_dit_shard_plan(int n_tracks, int cfg, int world, int rank, int * track0, int * n_local,
                                      int * half, int * peer);
/* dit_ggml_generate sharded over the communicator's ranks. Every rank passes the whole job's host
 * arrays (as acb_dit_generate_ex) and receives every track's x0 in output [N][T][out_channels]. */
ACB_API acb_status acb_dit_generate_sharded(acb_dit * m, acb_comm * comm, const float * noise,
                                            const float * context_latents, const float * enc_hidden, int enc_S, int T,
                                            int N, int num_steps, const float * schedule, float * output,
                                            float guidance_scale, const float * context_switch, int cover_steps,
                                            acb_cancel_fn cancel, void * cancel_data, const int * real_S,
                                            const int * real_enc_S, const float * enc_switch,
                                            const int * real_enc_S_switch, const int64_t * seeds,
                                            const char * solver_name, acb_randn_fn randn, void * randn_data,
                                            float * gpu_ms);
/* The same job one step at a time, for hosts that drive the schedule themselves: begin (comm may be
 * NULL: the whole job on this GPU), then step k with (t_curr, t_next) -- last != 0 for the final
 * x0 step; host_out (optional) receives this rank's xt after the step, or x0 after the last --,
 * then end (output: every track's x0; gpu_ms: device time from the first step). Steps run on
 * acb_dit_stream(m). */
ACB_API acb_status   acb_dit_job_begin(acb_dit * m, acb_comm * comm, const float * noise, const float * context_latents,
                                       const float * enc_hidden, int enc_S, int T, int N, float guidance_scale,
                                       const float * context_switch, int cover_steps, acb_cancel_fn cancel,
                                       void * cancel_data, const int * real_S, const int * real_enc_S,
                                       const float * enc_switch, const int * real_enc_S_switch, const int64_t * seeds,
                                       const char * solver_name, acb_randn_fn randn, void * randn_data);
ACB_API acb_status   acb_dit_job_step(acb_dit * m, int step, float t_curr, float t_next, int last, float * host_out);
ACB_API acb_status   acb_dit_job_end(acb_dit * m, float * output, float * gpu_ms);
ACB_API acb_stream_t acb_dit_stream(const acb_dit * m);

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

/* The phase-2 decode step of src/pipeline-lm.cpp:455-497 with its sampling on the device: one
 * acb_qw3lm_forward_batch over n_active sets (2 * n_active with use_cfg: the conditional sets
 * first, then the unconditional ones, the reference's layout), then for each active sequence the
 * targeted CFG lu + cfg_scale * (lc - lu) over its [eos_idx] + [code_offset, code_offset + n_codes)
 * logit columns (columns of the out_V row), the compaction and sample_top_k_p (acb_sample_top_k_p)
 * with u[a] (host) the canonical uniform of that sequence's generator. sampled[a] (host) receives
 * the compact index: 0 for EOS, 1 + c for audio code c. Only n_active ints leave the device. */
ACB_API acb_status acb_qw3lm_forward_batch_sample(acb_qw3lm * m, const int32_t * token_ids,
                                                  const int32_t * kv_sets, int n_active, int use_cfg,
                                                  float cfg_scale, int lm_offset, int lm_count, int eos_idx,
                                                  int code_offset, int n_codes, float temperature, float top_p,
                                                  int top_k, const float * u, int32_t * sampled);

ACB_API void       acb_qw3lm_reset_kv(acb_qw3lm * m, int kv_set);            /* qw3lm_reset_kv :227 */
ACB_API acb_status acb_qw3lm_copy_kv(acb_qw3lm * m, int src, int dst);       /* qw3lm_copy_kv :233 */
ACB_API acb_status acb_qw3lm_build_partial_head(acb_qw3lm * m, int lm_offset); /* :290 */
ACB_API int        acb_qw3lm_kv_pos(const acb_qw3lm * m, int kv_set);
/* 1 when single-sequence decode runs as the persistent step (acb_lm_decode_step):
 * acb_qw3lm_forward_batch with N = 1 and the full head (one launch per call), and
 * acb_qw3lm_generate_greedy with N = 1 (up to 64 tokens per launch); 0 when it runs the per-op
 * graph (shape outside the persistent kernel, e.g. K-quant weights, or ACB_LM_PERSIST=0 in the
 * environment at load). No counterpart in the reference. */
ACB_API int        acb_qw3lm_persistent_decode(const acb_qw3lm * m);
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
