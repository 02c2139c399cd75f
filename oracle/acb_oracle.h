/*
 * acb_oracle.h -- CPU oracle for the acestep.cpp per-layer op-chain.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the checker that the CUDA path is compared
 * against; it is never linked into, loaded by, or called from the product library
 * (libacb.so). Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use it.
 *
 * It restates, in plain C, the arithmetic that the reference's ggml-CPU build performs for
 * the ops emitted by src/qwen3-enc.h, src/qwen3-lm.h and src/dit-graph.h (the ggml source is
 * an empty submodule in the reference mount, so the semantics are taken from the reference's
 * call sites and the public GGUF/ggml format definitions, and pinned against gguf-py 0.19.0
 * where that package covers the arithmetic: Q8_0 quantize, Q8_0/Q4_K/Q6_K dequantize).
 *
 * Float rules followed everywhere (built with -ffp-contract=off):
 *   - rms_norm sums x*x (float product) in double, mean = (float)(sum/n),
 *     scale = 1.0f/sqrtf(mean+eps), y = x*scale, then the separate ggml_mul by the weight;
 *   - each ggml graph node rounds to float once (no fused multiply-add across nodes);
 *   - RoPE angles come from a host-built table: theta = pos, then theta *= base^(-2/D)
 *     once per pair, cos/sin in float (ggml rope cache order);
 *   - quantized mul_mat first quantizes the activation row to the weight's vec-dot type
 *     (Q8_0 for Q8_0 weights, Q8_K for Q4_K/Q6_K), integer block dot products, float
 *     per-block scaling, blocks summed in order.
 */
#ifndef ACB_ORACLE_H
#define ACB_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* GGUF tensor type ids (public GGUF format). */
enum {
    ORC_F32  = 0,
    ORC_F16  = 1,
    ORC_Q8_0 = 8,
    ORC_Q4_K = 12,
    ORC_Q6_K = 14,
    ORC_Q8_K = 15,
    ORC_BF16 = 30,
};

/* ---- scalar conversions ---- */
float    orc_f16_to_f32(uint16_t h);
uint16_t orc_f32_to_f16(float f);  /* round to nearest even */
float    orc_bf16_to_f32(uint16_t h);
uint16_t orc_f32_to_bf16(float f); /* round to nearest even, NaN kept quiet */

/* ---- block formats ---- */
int64_t orc_block_elems(int type);           /* elements per block (1 for plain types) */
int64_t orc_block_bytes(int type);           /* bytes per block */
int64_t orc_row_bytes(int type, int64_t n);  /* bytes of a row of n elements, -1 if n not a block multiple */

/* Dequantize one row of n elements. Returns 0, or -1 for an unsupported type / bad n. */
int orc_dequant_row(int type, const void * src, float * dst, int64_t n);

/* Activation quantizers used by the quantized mul_mat. */
void orc_quantize_row_q8_0(const float * x, void * dst, int64_t n);
void orc_quantize_row_q8_K(const float * x, void * dst, int64_t n); /* 292 B / 256 */

/* Encoders that produce valid Q4_K / Q6_K blocks for synthetic weights. They are not
 * ggml's quantizers (those are search-based); only the dequantized values matter. */
void orc_quantize_row_q4_K(const float * x, void * dst, int64_t n);
void orc_quantize_row_q6_K(const float * x, void * dst, int64_t n);

/* ---- ops ---- */

/* out[i] = dequant(table[ids[i]]). Returns -1 if any id is out of range (nothing written
 * for that row), else 0. */
int orc_get_rows(int type, const void * table, int64_t n_rows, int64_t cols, const int32_t * ids,
                 int64_t n_ids, float * out);

/* y = rms_norm(x) * w (w may be NULL: plain rms_norm). x/y [rows][cols]. */
void orc_rms_norm(const float * x, const float * w, float * y, int64_t rows, int64_t cols, float eps);

/* RoPE table: cache[p][i][0..1] = cos/sin of pos[p] * base^(-2i/D) (iterative), i < D/2. */
void orc_rope_cache(float * cache, const int32_t * pos, int64_t n_pos, int head_dim, float base);

/* Per-head RMSNorm (weight w[head_dim], may be NULL) then NeoX rotation (rope may be NULL).
 * x/y: [n_tok][n_heads][head_dim] with token stride tok_stride (elements).
 * rope: [n_tok][head_dim/2][2] (one table row per token). */
void orc_qk_norm_rope(const float * x, int64_t x_tok_stride, float * y, int64_t y_tok_stride, int64_t n_tok,
                      int n_heads, int head_dim, const float * w, float eps, const float * rope);

/* out[r][i] = silu(g[r][i]) * u[r][i]; g and u rows have strides g_stride/u_stride. */
void orc_swiglu(const float * g, int64_t g_stride, const float * u, int64_t u_stride, float * out, int64_t rows,
                int64_t F);

/* y[s][t][:] = rms_norm(x)*w (w may be NULL: no norm, x taken as already normalised)
 *              * (1 + scale[s]) + shift[s]; vec_stride 0 = one vector for all samples. */
void orc_adaln(const float * x, const float * w, float eps, const float * scale, const float * shift,
               int64_t vec_stride, float * y, int64_t samples, int64_t rows_per_sample, int64_t H);

/* out = r + o * gate[s] (gate raw, no sigmoid); vec_stride as above. */
void orc_gated_residual(const float * r, const float * o, const float * gate, int64_t vec_stride, float * out,
                        int64_t samples, int64_t rows_per_sample, int64_t H);

/* y[m][n] = sum_k W[n][k] * x[m][k] with ggml-CPU quantized mul_mat semantics.
 * W: N rows of K elements in wtype (Q8_0, Q4_K, Q6_K, BF16, F16, F32). */
int orc_mul_mat(int wtype, const void * W, int64_t N, int64_t K, const float * x, int64_t M, float * y);

/* Arithmetic of orc_mul_mat, process-wide:
 *   ORC_MM_GGML  (default) ggml-CPU semantics: the activation is quantised to the weight's
 *                vec-dot type (Q8_0 / Q8_K) or rounded to F16 / BF16 before the dot products;
 *   ORC_MM_EXACT dequantised weights times the unrounded f32 activation, accumulated in double.
 * EXACT measures how far the reference's own activation quantisation sits from exact
 * arithmetic; GGML is the reference every parity bar is taken against. */
enum { ORC_MM_GGML = 0, ORC_MM_EXACT = 1 };
void orc_set_mul_mat_mode(int mode);
int  orc_get_mul_mat_mode(void);

/* Attention with ggml-CPU semantics of qwen3_attn_f32 (qwen3-enc.h:101-112).
 * q [Sq][Hq][D] f32; k/v in kv_type (F32 or F16): element (token j, head h, d) at
 * j*kv_tok_stride + h*kv_head_stride + d;
 * mask [Sq][Skv] f32 additive (NULL = none), out [Sq][Hq][D] f32. GQA: head h uses kv head
 * h / (Hq/Hkv). For F16 K/V, q and the normalised probabilities are rounded to f16 before
 * their dot products (the mul_mat vec-dot type of an F16 operand). */
void orc_attention(const float * q, int64_t q_tok_stride, const void * k, const void * v, int kv_type,
                   int64_t kv_tok_stride, int64_t kv_head_stride, const float * mask, float * out,
                   int64_t out_tok_stride, int64_t Sq, int64_t Skv, int Hq, int Hkv, int D, float scale);

/* Sinusoidal timestep embedding (ggml_timestep_embedding, dim even): out[dim]. */
void orc_timestep_embedding(float t, int dim, int max_period, float * out);

/* Philox4x32-10 (Salmon et al., "Parallel random numbers: as easy as 1, 2, 3", SC'11) of one
 * 128-bit counter under a 64-bit key, as src/philox.h:30-82 computes it. */
void orc_philox4x32_10(const uint32_t ctr[4], uint32_t k0, uint32_t k1, uint32_t out[4]);
/* philox_randn (src/philox.h:130-136): out[k] = the first Box-Muller normal of counter
 * {0, 0, k_lo, k_hi} under key = seed, rounded through bfloat16 when bf16_round. */
void orc_philox_randn(int64_t seed, int64_t n, int bf16_round, float * out);

/* FSQ alphabet {8,8,8,5,5,5}: fsq_decode_index (src/fsq-detok.h:18-29) and fsq_encode_index
 * (src/fsq-tok.h:42-60, libm tanhf). */
void orc_fsq_decode_index(int index, float * out6);
int  orc_fsq_encode_index(const float * raw6);

/* sample_top_k_p (src/sampling.h:30-133) on logits[V] in place; u = the canonical uniform of the
 * reference's std::uniform_real_distribution<float>(0, sum) draw. Equal probabilities in the top_p
 * sort are ordered by ascending id. */
int orc_sample_top_k_p(float * logits, int V, float temperature, float top_p, int top_k, float u);

/* Thread control for the CPU baseline (0 = OpenMP default). */
void orc_set_threads(int n);
int  orc_get_threads(void);

#ifdef __cplusplus
}
#endif
#endif
