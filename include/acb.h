/*
 * acb.h -- C ABI of libacb, the B200 (sm_100a) implementation of acestep.cpp's per-layer
 * transformer op-chain.
 *
 * Conventions
 *   - Every entry point returns an acb_status (0 = ACB_OK) and never exits the process.
 *   - Tensor arguments are device pointers with explicit element strides; nothing here takes
 *     a framework tensor type. Host arguments are marked "host".
 *   - `stream` is a cudaStream_t (NULL = the legacy default stream). All kernels are enqueued
 *     asynchronously; a launch failure is reported as ACB_ERR_CUDA.
 *   - Type ids are the GGUF/ggml tensor type ids (acb_type), so GGUF blocks are consumed
 *     byte-for-byte with no repacking.
 *   - Layouts use ggml order translated to row-major: a ggml activation [H, S] is rows[S][H];
 *     a ggml weight [K, N] is N rows of K elements with quant blocks running along K.
 *   - `err_flag` (optional device int) receives a bitwise OR of ACB_DEVERR_* bits when a
 *     kernel meets an out-of-range index; the offending row is written as zeros and nothing is
 *     read out of bounds.
 *
 * Each function names the reference interface (file:line in acestep.cpp) whose ggml graph node
 * it replaces.
 */
#ifndef ACB_H
#define ACB_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#    define ACB_API __attribute__((visibility("default")))
#else
#    define ACB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st * acb_stream_t; /* == cudaStream_t */

typedef enum {
    ACB_OK               = 0,
    ACB_ERR_INVALID_ARG  = 1, /* null pointer, bad size, bad stride */
    ACB_ERR_UNSUPPORTED  = 2, /* type / shape combination not implemented */
    ACB_ERR_CUDA         = 3, /* a CUDA runtime call or kernel launch failed */
    ACB_ERR_OUT_OF_RANGE = 4, /* id, position or kv length beyond its table */
    ACB_ERR_OOM          = 5, /* device or host allocation failed */
    ACB_ERR_IO           = 6, /* file open / map / read failed */
    ACB_ERR_FORMAT       = 7, /* malformed or truncated GGUF, missing tensor */
    ACB_ERR_DEVICE       = 8, /* a kernel reported an error through its device flag */
    ACB_ERR_CANCELLED    = 9, /* the caller's cancel callback asked to stop (the reference returns -1) */
    ACB_ERR_TIMEOUT      = 10, /* a bounded wait on peer GPUs gave up (the communicator is aborted) */
} acb_status;

typedef enum {
    ACB_TYPE_F32  = 0,
    ACB_TYPE_F16  = 1,
    ACB_TYPE_Q8_0 = 8,
    ACB_TYPE_Q4_K = 12,
    ACB_TYPE_Q6_K = 14,
    ACB_TYPE_Q8_K = 15,
    ACB_TYPE_I32  = 26,
    ACB_TYPE_BF16 = 30,
    /* not a GGUF type: Q8_0 weights repacked by acb_q8_0_to_tiles for the tensor-core GEMV */
    ACB_TYPE_Q8_0_TILES = 1008,
} acb_type;

enum {
    ACB_DEVERR_ID_RANGE  = 1, /* get_rows id outside [0, n_rows) */
    ACB_DEVERR_POS_RANGE = 2, /* rope / kv position outside [0, max_pos) */
    ACB_DEVERR_TIMEOUT   = 4, /* a bounded device-side wait gave up */
    ACB_DEVERR_CODE_RANGE = 8, /* a negative FSQ code (acb_fsq_project_out) */
};

/* ---- library ------------------------------------------------------------------------------ */

ACB_API int          acb_version(void);                  /* (major << 16) | (minor << 8) | patch */
ACB_API const char * acb_status_string(int status);      /* static string */
ACB_API int          acb_last_cuda_error(void);          /* cudaError_t of the last ACB_ERR_CUDA */
ACB_API int64_t      acb_row_bytes(int type, int64_t n); /* bytes of a row of n elements, -1 if invalid */

/* RoPE table for mode NEOX (freq_scale 1, ext_factor 0, attn_factor 1), host memory:
 * table[p][2i] = cos(theta_i(p)), table[p][2i+1] = sin(theta_i(p)), i < head_dim/2, where
 * theta_0 = p and theta_{i+1} = theta_i * base^(-2/head_dim) in float (the ggml rope cache).
 * Replaces the angle computation inside ggml_rope_ext(..., mode 2, ...) at
 * src/qwen3-enc.h:172-173, src/qwen3-lm.h:378-379,666-667, src/dit-graph.h:195-197. */
ACB_API acb_status acb_rope_table_host(float * table, int max_pos, int head_dim, float base);

/* ---- row ops (config 2a-2d of the op-chain) ------------------------------------------------ */

/* y[r] = rms_norm(x[r], eps) * w (w NULL: plain rms_norm). x/y types F32, BF16 or F16.
 * Replaces ggml_rms_norm + ggml_mul: qwen3_rms_norm (src/qwen3-enc.h:114-120),
 * dit_ggml_rms_norm_weighted (src/dit-graph.h:24-30). */
ACB_API acb_status acb_rms_norm(const void * x, int x_type, int64_t x_stride, const float * w, void * y, int y_type,
                        int64_t y_stride, int64_t rows, int cols, float eps, acb_stream_t stream);

/* Per-head RMSNorm * norm_w followed by NeoX RoPE, gathered from and scattered to strided
 * layouts (also the f16 KV-cache write). Source element (t, h, d) is
 * src[t*src_tok_stride + h*head_dim + d]; destination element is
 * dst[t*dst_tok_stride + h*dst_head_stride + pos[t]*dst_pos_stride + d].
 * norm_w NULL skips the norm; rope_table NULL skips the rotation (pos may then be NULL when
 * dst_pos_stride is 0). rope_table is [max_pos][head_dim] from acb_rope_table_host, on device.
 * head_dim must be a multiple of 64 and at most 256. dst_type F32, F16 or BF16.
 * Replaces the q/k-norm + ggml_rope_ext + ggml_cpy(->f16 cache) chain of
 * qwen3_build_self_attn (src/qwen3-enc.h:159-174), qw3lm_build_attn (src/qwen3-lm.h:366-406),
 * qw3lm_forward_batch (src/qwen3-lm.h:654-703) and dit_ggml_build_self_attn
 * (src/dit-graph.h:175-198). */
ACB_API acb_status acb_qk_norm_rope(const void * src, int src_type, int64_t src_tok_stride, void * dst, int dst_type,
                            int64_t dst_tok_stride, int64_t dst_head_stride, int64_t dst_pos_stride, int64_t n_tok,
                            int n_heads, int head_dim, const float * norm_w, float eps, const int32_t * pos,
                            const float * rope_table, int max_pos, int * err_flag, acb_stream_t stream);

/* acb_qk_norm_rope into the exact operand planes of the split-precision attention, for the q
 * heads and the k heads of a fused qkv row in one launch: heads [0, n_q_heads) are normalised
 * with q_norm_w, heads [n_q_heads, n_q_heads + n_k_heads) with k_norm_w (src head h at column
 * h*128), then rotated when a rope table is given; dst[t][h*128 + d] = f16(v) and
 * dst[lo_offset + same] = f16(v - hi), v the fp32 result. head_dim 128; src f32 or f16. One
 * pass instead of f32 results followed by acb_act_quant_ex(..., ACB_LAYOUT_PLANES). */
ACB_API acb_status acb_qk_norm_rope_planes(const void * src, int src_type, int64_t src_tok_stride, uint16_t * dst,
                                           int64_t dst_tok_stride, int64_t lo_offset, int64_t n_tok, int n_q_heads,
                                           const float * q_norm_w, int n_k_heads, const float * k_norm_w,
                                           int head_dim, float eps, const int32_t * pos, const float * rope_table,
                                           int max_pos, int * err_flag, acb_stream_t stream);

/* out[r][i] = silu(g[r][i]) * u[r][i], silu(v) = v / (1 + exp(-v)). g = gu + r*gu_stride,
 * u = g + up_offset (fused [gate(F) | up(F)] rows: up_offset = F, gu_stride = 2F).
 * Replaces ggml_swiglu / ggml_swiglu_split (src/qwen3-enc.h:217,221; src/dit-graph.h:259,264). */
ACB_API acb_status acb_swiglu(const void * gu, int gu_type, int64_t gu_stride, int64_t up_offset, void * out, int out_type,
                      int64_t out_stride, int64_t rows, int64_t F, acb_stream_t stream);

/* y = n * (1 + scale[s]) + shift[s] with n = rms_norm(x)*norm_w (norm_w NULL: n = x).
 * x/y [samples][rows_per_sample][H]; scale/shift F32 device vectors, vec_stride 0 = one vector
 * for every sample, H = one per sample. Replaces dit_ggml_rms_norm_weighted + dit_ggml_adaln
 * (src/dit-graph.h:24-30, 54-64, 405-406, 438-439, 603-604). */
ACB_API acb_status acb_adaln_modulate(const void * x, int x_type, const float * norm_w, float eps, const float * scale,
                              const float * shift, int64_t vec_stride, void * y, int y_type, int64_t samples,
                              int64_t rows_per_sample, int H, acb_stream_t stream);

/* out = r + o * gate[s] (gate raw, no sigmoid); layouts as acb_adaln_modulate; out may alias r.
 * Replaces dit_ggml_gated_add (src/dit-graph.h:70-76, 420, 445). */
ACB_API acb_status acb_gated_residual(const void * r, const void * o, int io_type, const float * gate, int64_t vec_stride,
                              void * out, int64_t samples, int64_t rows_per_sample, int H, acb_stream_t stream);

/* out[i][:] = dequant(table[ids[i]][:]) for table rows of `cols` elements in table_type
 * (F32, F16, BF16, Q8_0, Q4_K, Q6_K); out_type F32, BF16 or F16. Bit-exact with the ggml
 * dequantizers. Replaces ggml_get_rows (src/qwen3-enc.h:390,465; src/qwen3-lm.h:464,626). */
ACB_API acb_status acb_get_rows(const void * table, int table_type, int64_t n_rows, int64_t cols, const int32_t * ids,
                        int64_t n_ids, void * out, int out_type, int64_t out_stride, int * err_flag,
                        acb_stream_t stream);

/* Quantise f32 rows [rows][K] (device) into GGUF blocks at dst (device): Q8_0 with ggml's
 * reference quantiser arithmetic (d = amax/127 as f16, q = roundf(x/d)); Q4_K and Q6_K with
 * min/max encoders that produce valid blocks. Used to build synthetic weights and to requantise
 * on device (the reference requantises on the host in src/adapter-merge.h:357-472). */
ACB_API acb_status acb_quantize(const float * x, int64_t rows, int64_t K, int type, void * dst, acb_stream_t stream);

/* LoRA delta (src/adapter-merge.h:482-672, PEFT merge_and_unload): w[n][k] += bf16(scaling *
 * sum_r B[n][r] * A[r][k]) on f32 rows w [N][K] (the dequantised base), A [rank][K] and B [N][rank]
 * f32 already rounded to bf16 (so each product is exact); the products are added in double and
 * rounded to f32 once, multiplied by scaling, rounded to bf16 and added. rank <= 1024. */
ACB_API acb_status acb_lora_delta_add(float * w, int64_t N, int64_t K, const float * A, const float * B, int rank,
                                      float scaling, acb_stream_t stream);
/* LyCORIS LoKr delta (src/adapter-merge.h:674-958 with the merge of :357-472) on f32 rows w [N][K]
 * (the dequantised base), N = a*c, K = b*d: delta[i*c + k][j*d + l] = fl32(w1s[i][j] * w2[k][l])
 * with w1s [a][b] = w1 * (alpha / rank) and w2 [c][d] (the factor product w2_a . w2_b, or w2) in
 * f32, rounded to bf16. Without dora_scale: w += bf16(delta) * user_scale. With dora_scale [N]
 * (weight decomposition): m = w + bf16(delta), w = m * s per row, s = dora_scale[n] / (|m| + 2^-7)
 * and, for user_scale != 1, s = s * user_scale + (1 - user_scale); |m| from the row's f32 squares
 * summed in double. */
ACB_API acb_status acb_lokr_delta_add(float * w, int64_t N, int64_t K, const float * w1s, int a, int b,
                                      const float * w2, int c, int d, float user_scale, const float * dora_scale,
                                      acb_stream_t stream);
/* f32 rows back into a GGUF type: Q8_0 / Q4_K / Q6_K (acb_quantize), BF16 / F16 (nearest even), F32
 * (copy). The requantisation step of the adapter merge. */
ACB_API acb_status acb_requant(const float * x, int64_t rows, int64_t K, int type, void * dst, acb_stream_t stream);

/* ---- dense path (configs 1, 4, 5): tensor-core GEMM ---------------------------------------- */

enum {
    ACB_FLAG_F16    = 2, /* acb_gemm_bf16 / acb_attn_prefill: the tensor-core operands are f16, not bf16 */
    ACB_FLAG_GEMM_A = 4, /* acb_attn_tc with o_type Q8_0 / F16 / BF16: write the output projection's
                            exact operand [hi | hi | lo] (hi at column c, again at Nh*128 + c, lo at
                            2*Nh*128 + c; o_ts >= 3*Nh*128) instead of one 16-bit copy */
};

/* Activation operand of a tensor-core linear, with the arithmetic of ggml-CPU's quantised
 * mul_mat: each f32 row of x [rows][x_stride] is quantised like ggml's from_float for the
 * weight's vec-dot type and the dequantised values d*q are written rounded to f16, so that a
 * GEMM of f16 operands reproduces the reference's products up to f16 rounding:
 *   vec_type ACB_TYPE_Q8_0 (weights Q8_0): per 32, d = amax/127 stored as f16, q = round(x/d);
 *   vec_type ACB_TYPE_Q8_K (weights Q4_K / Q6_K): per 256, the signed value of largest magnitude
 *            mx (first index), iscale = -127/mx, q = min(127, round-half-even(iscale*x)),
 *            d = 1/iscale;
 *   vec_type ACB_TYPE_F16 / ACB_TYPE_BF16 (weights of that type): x rounded to that type.
 * y_type is ACB_TYPE_BF16 for vec_type BF16, else ACB_TYPE_F16. K a multiple of 32 (256 for
 * Q8_K). Replaces the activation quantisation inside ggml_mul_mat (src/qwen3-enc.h:86-88,
 * src/dit-graph.h:36-49) at M = tokens. */
ACB_API acb_status acb_act_quant(const float * x, int64_t x_stride, int64_t rows, int64_t K, int vec_type, void * y,
                                 int y_type, int64_t y_stride, acb_stream_t stream);

/* acb_act_quant of h = silu(g) * u (the ggml_swiglu arithmetic of acb_swiglu) over fused rows:
 * g = gu + r*gu_stride, u = g + up_offset, F columns; the activation of the down projection. */
ACB_API acb_status acb_act_quant_swiglu(const float * gu, int64_t gu_stride, int64_t up_offset, int64_t rows,
                                        int64_t F, int vec_type, void * y, int y_type, int64_t y_stride,
                                        acb_stream_t stream);

/* Operand layouts of acb_act_quant_ex. The exact layouts split every value v (each dequantised
 * operand has at most 18 significant bits: an f16 or f32 scale times a small integer) into
 * hi = f16(v) and lo = f16(v - hi), which represent it exactly, so that one GEMM over K' = 3K,
 * A' = [hi|hi|lo] times B' = [hi|lo|hi], sums hi.hi + hi.lo + lo.hi: every product of the
 * reference's dequantised operands to within 2^-22 relative, accumulated in fp32. */
enum {
    ACB_LAYOUT_PLAIN  = 0, /* y[m][k] = operand value */
    ACB_LAYOUT_GEMM_A = 1, /* y[m][0..3K) = [hi | hi | lo], y_stride >= 3K */
    ACB_LAYOUT_GEMM_B = 2, /* y[m][0..3K) = [hi | lo | hi] (weights), y_stride >= 3K */
    ACB_LAYOUT_PLANES = 3, /* hi at y[m][k], lo at y[lo_offset + m*y_stride + k] (attention operands) */
};

/* acb_act_quant / acb_act_quant_swiglu (up_offset > 0: h = silu(x) * x[up_offset + .]) with an
 * output layout. */
ACB_API acb_status acb_act_quant_ex(const float * x, int64_t x_stride, int64_t up_offset, int64_t rows, int64_t K,
                                    int vec_type, int layout, void * y, int y_type, int64_t y_stride,
                                    int64_t lo_offset, acb_stream_t stream);

/* RMSNorm of each row (times norm_w when given), optionally adaLN-modulated (y = n * (1 + scale)
 * + shift, scale/shift f32 vectors of one sample every rows_per_sample rows, vec_stride apart),
 * then quantised exactly as acb_act_quant_ex does (vec_type, layout PLAIN / GEMM_A / PLANES).
 * Replaces ggml_rms_norm + ggml_mul [+ ggml_mul(1 + scale) + ggml_add(shift)] feeding a
 * ggml_mul_mat (src/dit-graph.h:150-157, 250-258, src/qwen3-enc.h:80-90) in one pass; results
 * are bit-identical to acb_rms_norm / acb_adaln_modulate (f32 output) followed by
 * acb_act_quant_ex. Without norm_w the adaLN form applies no normalisation (as
 * acb_adaln_modulate). K a multiple of 32 (256 for Q8_K), at most 4096. */
ACB_API acb_status acb_norm_quant(const float * x, int64_t x_stride, int64_t rows, int64_t K, const float * norm_w,
                                  float eps, const float * scale, const float * shift, int64_t vec_stride,
                                  int64_t rows_per_sample, int vec_type, int layout, void * y, int y_type,
                                  int64_t y_stride, int64_t lo_offset, acb_stream_t stream);

/* Vec-dot type of a weight type (ggml's type_traits_cpu[].vec_dot_type): Q8_0 for Q8_0, Q8_K
 * for Q4_K / Q6_K, the type itself for F16 / BF16 / F32 (F32: the activation stays f32; the
 * exact layouts split it, a plain operand rounds it to f16); -1 for other types. */
ACB_API int acb_vec_dot_type(int weight_type);

/* C[m][n] = epi(sum_k A[m][k] B[n][k]) on the 5th-generation tensor cores (tcgen05.mma, TMEM
 * accumulators, TMA-fed 128-byte-swizzled tiles): A [M][lda] and B [N][ldb] bf16 row-major, or
 * f16 with ACB_FLAG_F16 (K contiguous, K a multiple of 64, rows 16-byte aligned), fp32
 * accumulation, C f32, bf16 or f16 [M][ldc]. Epilogue, applied in order: + bias[n] (f32,
 * optional); then with res (f32 [M][ldr], may alias an f32 C): C = res + acc, or with gate (f32,
 * row m uses gate[(m / rows_per_sample) * gate_stride + n]): C = res + acc * gate, the DiT gated
 * residual. B holds the weights dequantised once (acb_get_rows with identity ids; f16 for
 * quantised and F16 weights, bf16 for BF16 weights) and A comes from acb_act_quant, which
 * together give ggml's quantised mul_mat up to f16 rounding. Replaces ggml_mul_mat at M = tokens
 * in dit_ggml_linear(_bias) (src/dit-graph.h:36-49), the DiT layer's projections
 * (dit-graph.h:159-172, 258-268, 298-314) with dit_ggml_gated_add (:70-76) fused, and the
 * encoder's prefill linears (src/qwen3-enc.h:86-88). */
ACB_API acb_status acb_gemm_bf16(const void * A, int64_t lda, const void * B, int64_t ldb, int64_t M, int64_t N,
                                 int64_t K, void * C, int c_type, int64_t ldc, const float * bias, const float * res,
                                 int64_t ldr, const float * gate, int64_t gate_stride, int64_t rows_per_sample,
                                 int flags, int * err_flag, acb_stream_t stream);

/* acb_gemm_bf16 with a split-K workspace: when the output tiles of an M x N GEMM would leave
 * most SMs idle (few tokens, e.g. the text encoder's 256), K is split across CTAs that write f32
 * partial tiles to `workspace` ([splits][M][N], 16-byte aligned), and a second kernel sums them
 * in split order (deterministic) and applies the epilogue. acb_gemm_workspace_bytes gives the
 * bytes needed at these sizes (0: no split is used); a smaller or NULL workspace runs unsplit.
 * Calls sharing one workspace must not overlap. */
/* The gate/up projection of a feed-forward block with SwiGLU and the down projection's activation
 * quantisation fused into its epilogue: Y = from_float(silu(A.Bg^T [+ bg]) * (A.Bu^T [+ bu])),
 * B = [Bg (F rows) | Bu (F rows)] stacked [2F][ldb] (bias, if given, [2F] in the same order),
 * quantised as acb_act_quant_ex does for vec_type Q8_0, F16 or BF16 (layout PLAIN [M][F] or
 * GEMM_A [M][3F] hi|hi|lo), y_type F16 (BF16 for vec_type BF16), ldy elements per row. Replaces
 * the two ggml_mul_mat, ggml_swiglu and the down mul_mat's from_float of dit_ggml_build_layer
 * (src/dit-graph.h:259-268) and the encoder FFN (src/qwen3-enc.h:217-223); bit-identical to
 * acb_gemm_tc (f32 out) + acb_act_quant_ex(..., up_offset = F, ...). F a multiple of 128. */
ACB_API acb_status acb_gemm_swiglu_quant(const void * A, int64_t lda, const void * B, int64_t ldb, int64_t M,
                                         int64_t F, int64_t K, const float * bias, int vec_type, int layout,
                                         void * Y, int y_type, int64_t ldy, int flags, int * err_flag,
                                         acb_stream_t stream);

/* The fused q/k/v projection of an attention block with everything up to the attention operands
 * in its epilogue: C = A . B^T with B = [Wq (n_q_heads*128 rows) | Wk | Wv (n_kv_heads*128 rows
 * each)] stacked, then per q / k head RMSNorm (q_norm_w / k_norm_w, NULL: none) and, with a rope
 * table, NeoX RoPE at pos[m] (ggml_rms_norm + ggml_mul + ggml_rope_ext of src/dit-graph.h:176-205,
 * src/qwen3-enc.h:165-184), written as f16 into qk [M][qk_ld] (q heads then k heads; with qk_lo
 * nonzero as exact hi / lo planes, lo qk_lo elements further); v heads go transposed into vt
 * [(b*n_kv_heads + h)*128 + d][vt_ld] at column t for row m = b*seq_len + t (lo plane vt_lo
 * further when nonzero). Bit-identical to acb_gemm_tc (f32 out) + acb_qk_norm_rope_planes +
 * acb_attn_vt. Head counts even; n_kv_heads 0 is the q projection alone (vt unused: the
 * cross-attention query of src/dit-graph.h:300-316). Rows with a position outside [0, max_pos)
 * are written as zeros and flag ACB_DEVERR_POS_RANGE. */
ACB_API acb_status acb_gemm_qkv_planes(const void * A, int64_t lda, const void * B, int64_t ldb, int64_t M, int64_t K,
                                       int n_q_heads, int n_kv_heads, const float * q_norm_w, const float * k_norm_w,
                                       float eps, const int32_t * pos, const float * rope_table, int max_pos,
                                       int64_t seq_len, uint16_t * qk, int64_t qk_ld, int64_t qk_lo, uint16_t * vt,
                                       int64_t vt_ld, int64_t vt_lo, int flags, int * err_flag, acb_stream_t stream);

ACB_API size_t     acb_gemm_workspace_bytes(int64_t M, int64_t N, int64_t K);

/* Unsplit GEMMs with M > 128 run on CTA pairs (clusters of two, tcgen05 cta_group::2, 256 x 256
 * output tiles, each CTA loading half of the B tile). Returns how many pairs fit on this device
 * at once (0: the pair kernel is off, e.g. ACB_GEMM_PAIR=0 in the environment). No reference
 * counterpart: a query of this library's tiling. */
ACB_API int        acb_gemm_pair_clusters(int f16);
ACB_API acb_status acb_gemm_tc(const void * A, int64_t lda, const void * B, int64_t ldb, int64_t M, int64_t N,
                               int64_t K, void * C, int c_type, int64_t ldc, const float * bias, const float * res,
                               int64_t ldr, const float * gate, int64_t gate_stride, int64_t rows_per_sample,
                               int flags, void * workspace, size_t workspace_bytes, int * err_flag,
                               acb_stream_t stream);

/* 1-D convolution as an implicit GEMM on the same tensor-core kernel (ggml_conv_1d = im2col +
 * mul_mat, src/vae.h:279-295, without the im2col buffer):
 *   Y[t][n] = epi( sum_{k, c} X[t + k*dilation - pad][c] * W[n][k*C_in + c] ),
 * X [T][ldx] bf16 / f16 (ACB_FLAG_F16) rows of C_in channels, rows outside [0, T) read as 0 (the
 * TMA bounds fill), W [N][kernel*C_in] in the same type, stride 1 (T_out = T when 2*pad =
 * (kernel-1)*dilation). Epilogue, workspace, flags and Y types as acb_gemm_tc. C_in a multiple of
 * 64 (one 64-channel slice of one tap per k-tile). */
ACB_API acb_status acb_conv1d_tc(const void * X, int64_t ldx, int64_t T, int C_in, const void * W, int64_t N,
                                 int kernel, int dilation, int pad, void * Y, int y_type, int64_t ldy,
                                 const float * bias, const float * res, int64_t ldr, int flags, void * workspace,
                                 size_t workspace_bytes, int * err_flag, acb_stream_t stream);

/* Attention over whole sequences (flash tiling on tensor cores, fp32 softmax and
 * accumulation), head_dim 128, GQA head h -> kv head h / (Nh/Nkv):
 *   O[b,i,h] = softmax_j(Q[b,i,h].K[b,j,h'] * scale + mask) V[b,j,h']
 * Q/K/V bf16 (f16 with ACB_FLAG_F16; the probabilities then meet V in the same type) with
 * element strides per batch (*_bs) and per token (*_ts); heads are contiguous
 * 128-element runs within a token row (so Q, K and V may be column views of one fused QKV
 * row). mask: 0 none, 1 causal (key j <= i + causal_off), 2 sliding window (|i - j| <= window).
 * O is f32, bf16 or f16. Replaces ggml_flash_attn_ext / qwen3_attn_f32 / dit_attn_f32 at prefill
 * (src/qwen3-enc.h:186-199; src/dit-graph.h:218-231 self-attention with the sliding-window and
 * padding masks of dit-sampler.h:253-282, and 339-352 cross-attention). */
ACB_API acb_status acb_attn_prefill(const void * q, int64_t q_bs, int64_t q_ts, const void * k, int64_t k_bs,
                                    int64_t k_ts, const void * v, int64_t v_bs, int64_t v_ts, void * o, int o_type,
                                    int64_t o_bs, int64_t o_ts, int batch, int Sq, int Skv, int Nh, int Nkv,
                                    int head_dim, int mask, int window, int causal_off, float scale, int flags,
                                    acb_stream_t stream);

/* acb_attn_prefill with f32-accurate arithmetic: q, k and v point at f16 hi planes whose lo
 * planes (lo = f16(x - hi), ACB_LAYOUT_PLANES of acb_act_quant_ex) sit q_lo / k_lo / v_lo
 * elements further; Q.K and P.V are formed as hi.hi + hi.lo + lo.hi on the tensor cores, which
 * reproduces the reference CPU build's f32 attention (qwen3_attn_f32, src/qwen3-enc.h:101-112;
 * dit_attn_f32, src/dit-graph.h:123-134) to about 2^-22 relative per product. */
ACB_API acb_status acb_attn_prefill_split(const void * q, int64_t q_bs, int64_t q_ts, const void * k, int64_t k_bs,
                                          int64_t k_ts, const void * v, int64_t v_bs, int64_t v_ts, void * o,
                                          int o_type, int64_t o_bs, int64_t o_ts, int batch, int Sq, int Skv, int Nh,
                                          int Nkv, int head_dim, int mask, int window, int causal_off, float scale,
                                          int flags, int64_t q_lo, int64_t k_lo, int64_t v_lo, acb_stream_t stream);

/* Attention on the 5th-generation tensor cores (tcgen05.mma into TMEM, TMA-fed 128-byte-swizzled
 * tiles, one softmax thread per query row): the same results as acb_attn_prefill for sequences
 * stored batch after batch. q [batch*Sq][q_ts] and k [batch*Skv][k_ts] f16 (head h at column
 * h*128; q_ts, k_ts multiples of 8); V is given transposed, vt [batch][Nkv][128][vt_ld] f16
 * (acb_attn_vt, vt_ld >= Skv, a multiple of 8); o [batch*Sq][o_ts] f32, bf16 or f16, or o_type
 * Q8_0: the output projection's activation operand (every 32 output columns quantised as one
 * Q8_0 block the way ggml's from_float does, stored as f16 d*q; with ACB_FLAG_GEMM_A as the exact
 * [hi|hi|lo] operand) -- the ggml_mul_mat(attn_o, .) input of src/dit-graph.h:236, 356 and
 * src/qwen3-enc.h:201, identical to an f32 output followed by acb_act_quant_ex. With q_lo / k_lo
 * / vt_lo nonzero every operand has an f16 lo plane that many elements further and the products
 * are lo.hi + hi.lo + hi.hi: f32-accurate attention. Masks as acb_attn_prefill. */
ACB_API acb_status acb_attn_tc(const void * q, int64_t q_ts, const void * k, int64_t k_ts, const void * vt,
                               int64_t vt_ld, void * o, int o_type, int64_t o_ts, int batch, int Sq, int Skv, int Nh,
                               int Nkv, int head_dim, int mask, int window, int causal_off, float scale, int flags,
                               int64_t q_lo, int64_t k_lo, int64_t vt_lo, int * err_flag, acb_stream_t stream);
/* acb_attn_tc with the padding masks of dit_ggml_generate (src/dit-sampler.h:244-304): for batch
 * element b only keys j < kv_len[b] take part (with the window or causal mask on top), and query
 * rows i >= q_len[b] are written as zeros (all their keys are masked: the empty sum of ggml's
 * flash attention). q_len / kv_len are device int arrays [batch], read when the kernel runs (so a
 * captured graph follows their current contents), or NULL for no padding. The DiT passes
 * q_len = kv_len = real_S for self-attention and kv_len = real_enc_S for cross-attention. */
ACB_API acb_status acb_attn_tc_masked(const void * q, int64_t q_ts, const void * k, int64_t k_ts, const void * vt,
                                      int64_t vt_ld, void * o, int o_type, int64_t o_ts, int batch, int Sq, int Skv,
                                      int Nh, int Nkv, int head_dim, int mask, int window, int causal_off, float scale,
                                      int flags, int64_t q_lo, int64_t k_lo, int64_t vt_lo, const int * q_len,
                                      const int * kv_len, int * err_flag, acb_stream_t stream);
/* V (f32 or f16; element (b, t, hk, d) at b*v_bs + t*v_ts + hk*128 + d) to the transposed f16
 * operand of acb_attn_tc: vt[((b*Nkv + hk)*128 + d)*vt_ld + t]; with lo_offset nonzero also the lo
 * plane f16(v - hi) at lo_offset elements further. */
ACB_API acb_status acb_attn_vt(const void * v, int v_type, int64_t v_bs, int64_t v_ts, int batch, int S, int Nkv,
                               int head_dim, void * vt, int64_t vt_ld, int64_t lo_offset, acb_stream_t stream);

/* ---- DiT step kernels (configs 4 and 5) ------------------------------------------------------ */

/* tt = {t, t_r} on the device: out[0][:] = ggml_timestep_embedding(t*1000, dim, max_period),
 * out[1][:] = the same of (t - t_r)*1000 (dit_ggml_build_temb, src/dit-graph.h:81-117). */
ACB_API acb_status acb_dit_sinusoid(const float * tt, int dim, int max_period, float * out, acb_stream_t stream);
/* y = x / (1 + exp(-x)) (ggml_silu). */
ACB_API acb_status acb_silu(const float * x, float * y, int64_t n, acb_stream_t stream);
/* Modulation vectors of one step (src/dit-graph.h:383-400, 591-606): ada[l] = sst[l] +
 * (tproj2[0] + tproj2[1]) for each layer's six [H] vectors (sst [n_layers][6H]); out_ss[0] =
 * oss[0] + (temb2[0] + temb2[1]) (shift), out_ss[1] = oss[1] + ... (scale). */
ACB_API acb_status acb_dit_modulation(const float * sst, const float * tproj2, const float * temb2, const float * oss,
                                      int n_layers, int H, float * ada, float * out_ss, acb_stream_t stream);
/* Noisy latent xt [N][T][Oc] into the xt channels of the DiT input [Ng][T][ctx_ch + Oc]; slot b
 * takes sample b % N (src/dit-sampler.h:466-479). */
ACB_API acb_status acb_dit_pack_xt(const float * xt, float * input, int N, int Ng, int T, int Oc, int ctx_ch,
                                   acb_stream_t stream);
/* APG guidance (apg_forward, src/dit-sampler.h:73-122) for N samples [T][Oc] in double:
 * running_avg [N][T][Oc] doubles (first != 0 starts it), momentum -0.75 and norm threshold 2.5
 * in the reference. vt = cond + (guidance_scale - 1) * orthogonal part. */
ACB_API acb_status acb_dit_apg(const float * cond, const float * uncond, double * running_avg, int first,
                               float momentum, float guidance_scale, float norm_threshold, int N, int T, int Oc,
                               float * vt, acb_stream_t stream);
/* tt = {t_curr, t_r, t_next}: xt -= vt * (t_curr - t_next) (solver-euler.h:8-18), or with last != 0
 * out = xt - vt * t_curr (the x0 prediction, dit-sampler.h:596-604). */
ACB_API acb_status acb_dit_euler(float * xt, const float * vt, const float * tt, int last, float * out, int64_t n,
                                 acb_stream_t stream);
/* DCW, Differential Correction in the Wavelet domain (src/dit-sampler.h:613-666, src/dwt-haar.h),
 * in place on xt [n_tracks][T][C] right after an ODE solver step (not after the last step, not
 * for SDE): denoised = xt - vt * t_next; for the wavelet modes the orthonormal Haar transform of
 * frame pairs (2j, 2j+1) along T (zero padding on odd T), the low band moved by s_low * (xL - yL)
 * (ACB_DCW_LOW, DOUBLE) and the high band by s_high * (xH - yH) (HIGH, DOUBLE), then the inverse;
 * ACB_DCW_PIX: xt += s_low * (xt - denoised). Every op one f32 rounding. The caller passes the
 * step's effective scales (low: t_curr * dcw_scaler; high: (1 - t_curr) * dcw_scaler; double:
 * those two with dcw_high_scaler for the high band; pix: dcw_scaler) and skips the call when they
 * are zero, as the reference returns before its transform. */
enum { ACB_DCW_LOW = 0, ACB_DCW_HIGH = 1, ACB_DCW_DOUBLE = 2, ACB_DCW_PIX = 3 };
ACB_API acb_status acb_dit_dcw(float * xt, const float * vt, int n_tracks, int T, int C, float t_next, int mode,
                               float s_low, float s_high, acb_stream_t stream);
/* DPM++ 3M step, the "dpm3m" solver (src/solvers/solver-dpm.h:14-50; registry solver-registry.h:32):
 * tt = {t_curr, t_r, t_next}, dt = t_curr - t_next; history = velocities stored so far, capped at 2
 * (the step index for steps 0, 1, then 2). history 0: xt -= vt*dt; 1: xt -= (1.5 vt - 0.5 prev)*dt;
 * 2: xt -= (23/12 vt - 16/12 prev + 5/12 prev_prev)*dt. Then prev_prev_vt <- prev_vt and prev_vt <- vt,
 * in place (both [n] f32, caller-owned; their contents are ignored while history says they are
 * empty). The last step of a schedule is acb_dit_euler with last != 0, as for every solver. */
ACB_API acb_status acb_dit_dpm3m(float * xt, const float * vt, float * prev_vt, float * prev_prev_vt, int history,
                                 const float * tt, int64_t n, acb_stream_t stream);
/* SDE ancestral step, the "sde" solver (src/solvers/solver-sde.h:17-38): tt = {t_curr, t_r, t_next};
 * xt = t_next * noise + (1 - t_next) * (xt - vt * t_curr). noise [n] f32 is the caller's: the
 * reference draws, for batch item b at step s, N(0,1) from Philox seeded with seed_b + s + 1 and
 * rounds it to bf16 (philox.h:113-126, the values torch.randn gives in bf16 on a CUDA generator
 * with that seed). The last step of a schedule is acb_dit_euler with last != 0. */
ACB_API acb_status acb_dit_sde(float * xt, const float * vt, const float * noise, const float * tt, int64_t n,
                               acb_stream_t stream);
/* acb_dit_sde with the noise drawn inline: for track b (of n_tracks, n_per elements each) the
 * noise is the bf16 Philox stream seeded with step_seeds[b] (device [n_tracks], the caller's
 * seed_b + step + 1, solver-sde.h:28-31) -- the values acb_philox_randn(step_seeds[b], .., 1)
 * writes. tt = {t_curr, t_r, t_next} on the device, as for acb_dit_sde. */
ACB_API acb_status acb_dit_sde_philox(float * xt, const float * vt, const int64_t * step_seeds, const float * tt,
                                      int n_tracks, int64_t n_per, acb_stream_t stream);

/* ---- seeded noise (src/philox.h) ------------------------------------------------------------- */

/* philox_randn (src/philox.h:130-136) on the device: out[k] (k < n, device f32) = the first
 * Box-Muller normal of Philox4x32-10 of counter {0, 0, k} under key = seed, rounded through bf16
 * when bf16_round (the reference always rounds: the values torch.randn gives in bf16 on a CUDA
 * generator seeded with `seed`). Replaces the host fills of the initial noise
 * (pipeline-synth-ops.cpp:761-770) and the SDE noise (solver-sde.h:28-31). The integer rounds are
 * exact; the float tail uses CUDA's logf/sinf, so at most 1 in 1000 values differs from the
 * reference's host stream by one bf16 step. */
ACB_API acb_status acb_philox_randn(int64_t seed, float * out, int64_t n, int bf16_round, acb_stream_t stream);
/* The raw Philox4x32-10 words of counters {0, 0, first + i} (i < n) under key = seed: out
 * [n][4] u32 on the device, 16-byte aligned (philox.h:50-82, 95-107). */
ACB_API acb_status acb_philox_bits(int64_t seed, int64_t first, int64_t n, uint32_t * out, acb_stream_t stream);

/* ---- FSQ and sequence packing (the condition encoder and the FSQ (de)tokenizer) ------------- */

/* out[g][n] = project_out(fsq_decode_index(codes[g]))[n] + bias[n] for G codes: the flat index is
 * split into the 6 FSQ levels {8,8,8,5,5,5} (fsq_decode_index, src/fsq-detok.h:18-29: level /
 * ((L-1)/2) - 1), rounded to the weight type and multiplied by w [N][6] (BF16, F16 or F32, the
 * tokenizer.quantizer.project_out weight), products added in double and rounded once, then the
 * f32 bias (NULL: none) -- ggml_mul_mat + ggml_add of src/fsq-detok.h:150-160, batched over every
 * code. A negative code writes a zero row and sets ACB_DEVERR_CODE_RANGE. */
ACB_API acb_status acb_fsq_project_out(const int32_t * codes, int G, const void * w, int w_type, int N,
                                       const float * bias, float * out, int64_t ldo, int * err_flag,
                                       acb_stream_t stream);
/* codes[g] = fsq_encode_index(raw[g][0..5] + bias): tanh, level floor((L-1)(t+1)/2 + 0.5) clamped
 * to [0, L-1], flat index with dimension 0 fastest (src/fsq-tok.h:42-60, 196-199). raw rows ld
 * floats apart; bias f32 [6] or NULL. */
ACB_API acb_status acb_fsq_quantize(const float * raw, int64_t ld, const float * bias, int G, int32_t * codes,
                                    acb_stream_t stream);
/* out[g*P + p][:] = a[g][:] + b[p][:] (f32 rows of H, H and the strides multiples of 4, pointers
 * 16-byte aligned): ggml_add(ggml_repeat(embedded, special), special), src/fsq-detok.h:165-169. */
ACB_API acb_status acb_rows_repeat_add(const float * a, int64_t lda, const float * b, int64_t ldb, int G, int P,
                                       int H, float * out, int64_t ldo, acb_stream_t stream);
/* out[g*(P+1)][:] = head[:], out[g*(P+1) + 1 + p][:] = src[g*P + p][:]: a learned token prepended
 * to each group of P rows (ggml_concat(cls, x, 1), src/fsq-tok.h:181-184, src/cond-enc.h:256-259).
 * Alignment as acb_rows_repeat_add. */
ACB_API acb_status acb_rows_prepend(const float * head, const float * src, int64_t lds, int G, int P, int H,
                                    float * out, int64_t ldo, acb_stream_t stream);

/* ---- VAE decoder ops (src/vae.h) -------------------------------------------------------------- */

/* y [T][ldy] f16 = f16(snake(x)) with the snake x + sin(x*e^a)^2 * e^-b (vae_snake, src/vae.h:
 * 267-276: exp_alpha = e^a, inv_beta = e^-b per channel, five separately rounded f32 ops; NULL:
 * no snake, a plain cast). f16 is the operand type ggml_conv_1d gives the activation (its im2col
 * takes the f16 weights' type); acb_conv1d_tc reads y in place of the im2col. C, x_stride, ldy
 * multiples of 8, x and y 16-byte aligned. */
ACB_API acb_status acb_vae_snake_f16(const float * x, int64_t x_stride, int64_t T, int C, const float * exp_alpha,
                                     const float * inv_beta, void * y, int64_t ldy, acb_stream_t stream);
/* The output conv: snake, then C -> 2 channels, kernel 7, pad 3, no bias; w f16 [2][7][C];
 * y planar [2][T]. */
ACB_API acb_status acb_vae_out_conv(const float * x, int64_t T, int C, const float * exp_alpha,
                                    const float * inv_beta, const void * w, float * y, acb_stream_t stream);

/* ---- LM token sampling ------------------------------------------------------------------------ */

/* sample_top_k_p (src/sampling.h:30-133) for `rows` sequences on the device, one CTA each, with the
 * phase-2 targeted CFG and compaction in front (src/pipeline-lm.cpp:474-497). Row r's sampled row
 * is x[c] for c < Vc = (col0 >= 0) + span_len: column col0 first (the EOS logit), then columns
 * span_off .. span_off + span_len - 1 (the audio codes; col0 = -1, span_off 0, span_len V for a
 * whole row); with uncond (rows uld floats apart) x = u + cfg_scale * (x - u) first. Then
 * temperature (<= 0: greedy, first maximum), top_k (0: off), top_p (outside (0, 1): off) and the
 * multinomial draw r = u[r] * sum with u[r] the canonical uniform that the reference's
 * std::uniform_real_distribution<float>(0, sum) takes from the sequence's mt19937
 * (std::generate_canonical<float, 24>; unused and may be NULL when greedy). idx[r] receives the
 * index c in the compacted row. work: acb_sample_work_bytes(rows, Vc) bytes of device scratch.
 * Reductions run in a fixed order (deterministic); the reference's single-thread sums round
 * differently, which can change a draw only when r or top_p falls within rounding of a boundary.
 * Equal probabilities at the top_p boundary are all kept. */
ACB_API size_t     acb_sample_work_bytes(int rows, int Vc);
ACB_API acb_status acb_sample_top_k_p(const float * logits, int64_t ld, const float * uncond, int64_t uld,
                                      float cfg_scale, int col0, int64_t span_off, int span_len, int rows,
                                      float temperature, float top_p, int top_k, const float * u, float * work,
                                      int32_t * idx, acb_stream_t stream);

/* ---- decode path (configs 3 and 5) --------------------------------------------------------- */

enum {
    ACB_PRO_X          = 0, /* activation x[m][k] = x[m*x_stride + k] */
    ACB_PRO_RMSNORM    = 1, /* x = rms_norm(h[m]) * norm_w (h = x argument) */
    ACB_PRO_SUM_SPLITS = 2, /* x[m][k] = (float) sum_s xd[(m*n_split + s)*K + k]: x points at DOUBLE
                               partials xd (acb_attn_decode's), added in double, rounded once */
    ACB_PRO_SWIGLU     = 3, /* x[m][k] = silu(g[m][k]) * g[m][K + k], g rows of 2K at x_stride */
};
enum {
    ACB_EPI_STORE = 0, /* y = W.x */
    ACB_EPI_ADD   = 1, /* y = res + W.x (ggml_add(hidden, out); y may alias res) */
};
enum {
    ACB_FLAG_PDL = 1, /* launch with programmatic dependent launch (the kernel waits on its
                         predecessor with griddepcontrol.wait before reading activations) */
};

/* Weight-streaming GEMV for M = 1..8 rows: y[m][n] = sum_k W[n][k] * x[m][k] for W = N rows of K
 * elements in Q8_0, Q4_K or Q6_K (K a multiple of 256; W 16-byte aligned and readable up to the
 * next 16-byte boundary past its last row). The activation is quantised in-kernel to the
 * weight's ggml vec-dot type (Q8_0 / Q8_K) and dotted with integer arithmetic, exactly like
 * ggml-CPU's quantised mul_mat: each block's term is (float)isum * (d_w * d_x) rounded to float,
 * and a row's terms are added in double and rounded to float once, so the result does not
 * depend on how the kernel partitions the row; `prologue` fuses the producer of x and
 * `epilogue` the residual add. Replaces ggml_mul_mat at every decode linear (src/qwen3-lm.h:639-651, 747-755) together
 * with the ggml_rms_norm/ggml_mul before it (qwen3-lm.h:636,741), ggml_swiglu
 * (qwen3-enc.h:217) and ggml_add after it (qwen3-lm.h:730,738). */
/* Repack GGUF Q8_0 rows [N][K] (N a multiple of 16) into 16-row tiles for acb_gemv with w_type
 * ACB_TYPE_Q8_0_TILES: per tile and 32-column block, 512 bytes of int8 weights in the order of the
 * A operand of an int8 mma.m16n8k32 followed by the 16 rows' f16 scales -- the same byte count as
 * the GGUF rows, and the same values. No reference counterpart (an on-device layout). */
ACB_API acb_status acb_q8_0_to_tiles(const void * src, void * dst, int64_t N, int64_t K, acb_stream_t stream);
ACB_API acb_status acb_gemv(const void * W, int w_type, int64_t N, int64_t K, int M, int prologue, const float * x,
                            int64_t x_stride, const float * norm_w, float eps, int n_split, float * y,
                            int64_t y_stride, int epilogue, const float * res, int64_t res_stride, int flags,
                            int * err_flag, acb_stream_t stream);

/* Fused QKV post-processing for the KV-cache path, head_dim 128: for every token t and every
 * head of the fused [q(Nh) | k(Nkv) | v(Nkv)] row (f32, token stride qkv_stride): q heads ->
 * RMSNorm*q_norm + NeoX RoPE -> q_out (f32); k heads -> RMSNorm*k_norm + RoPE -> f16 k_cache;
 * v heads -> f16 v_cache. Cache element (set, h, p, d) is at ((set*Nkv + h)*max_seq + p)*128 + d
 * (the reference's 4-D [D, max_seq, Nkv, n_sets] tensor); token t uses set
 * set0 + t*set_per_tok and position pos[t]. Replaces qw3lm_build_attn's q/k-norm, rope and
 * ggml_cpy into the cache (src/qwen3-lm.h:366-406; batched: 654-703). */
ACB_API acb_status acb_qkv_post(const float * qkv, int64_t qkv_stride, int64_t n_tok, int Nh, int Nkv, int head_dim,
                                const float * q_norm, const float * k_norm, float eps, const int32_t * pos,
                                const float * rope_table, int max_pos, float * q_out, int64_t q_stride,
                                uint16_t * k_cache, uint16_t * v_cache, int max_seq, int set0, int set_per_tok,
                                int flags, int * err_flag, acb_stream_t stream);

/* Number of KV splits acb_attn_decode uses for n_tok sequences of Nkv heads on this device. */
ACB_API int acb_attn_decode_splits(int n_tok, int Nkv);

/* One-token attention for n_tok sequences over the f16 cache, kv_len = pos[t] + 1, with
 * ggml-CPU semantics (q and normalised probabilities rounded to f16, softmax sum in double):
 *   s_j = (sum_d q16_d k16_jd) * scale in float, in one fixed order: eight sequential sums of 16
 *         dimensions added as ((s0+s1)+(s2+s3))+((s4+s5)+(s6+s7)) (products of f16 are exact)
 *   p_j = f16( acb_expf(s_j - max) * (float)(1 / sum_j acb_expf(s_j - max)) )
 *   o_d = (float) sum_j p_j v16_jd, sum in double
 * so the result is the same for any split count. Scratch (device, caller-owned): scores
 * [n_tok][Nh][max_seq] f32, smax [n_tok][Nh][n_split] f32, part [n_tok][n_split][Nh*128] double
 * split partials. With out (and tickets, int [n_tok][Nkv], zeroed before first use and
 * returned to zero by every call) the last split CTA of each (token, kv head) adds the partials
 * in double into out[t*out_stride + h*128 + d]; with out NULL the partials are left for the
 * O-projection's ACB_PRO_SUM_SPLITS prologue.
 * Replaces ggml_flash_attn_ext / qwen3_attn_f32 on the cache view (src/qwen3-lm.h:705-723). */
ACB_API acb_status acb_attn_decode(const float * q, int64_t q_stride, int n_tok, int Nh, int Nkv, int head_dim,
                                   const int32_t * pos, const uint16_t * k_cache, const uint16_t * v_cache,
                                   int max_seq, int set0, int set_per_tok, float scale, int n_split, float * scores,
                                   float * smax, double * part, float * out, int64_t out_stride, int * tickets,
                                   int flags, acb_stream_t stream);

/* Largest `rows` acb_argmax takes. The scratch starts with one counter per possible row (a fixed
 * 4 KB, whatever the call's shape), followed by the per-CTA partials. */
#define ACB_ARGMAX_MAX_ROWS 1024

/* Device scratch (bytes) acb_argmax needs for `rows` rows of V logits. */
ACB_API size_t acb_argmax_scratch_bytes(int rows, int64_t V);

/* Greedy sampling on device: ids[r] = argmax_v logits[r*stride + v] (lowest index on ties),
 * margin[r] = top1 - top2 (optional), pos_advance[r] += 1 (optional: advances the next step's
 * positions without a host round trip). With hist (requires pos_advance and hist_base) the
 * token is also recorded at hist[r*hist_stride + pos_advance[r] - hist_base[r]] (and its margin
 * in mhist when given) before the position advances. `scratch` is a 16-byte aligned device
 * buffer of acb_argmax_scratch_bytes(rows, V) bytes whose first 4 KB (the counters) are zeroed
 * before its first use; every call returns the counters to zero, so one buffer sized for the
 * largest (rows, V) serves calls of any smaller shape in any order. Calls that share a scratch
 * buffer must not overlap on the GPU. rows <= ACB_ARGMAX_MAX_ROWS. Replaces the temperature-0
 * branch of sample_top_k_p (src/sampling.h:30-34). */
ACB_API acb_status acb_argmax(const float * logits, int64_t stride, int64_t V, int rows, int32_t * ids, float * margin,
                              int32_t * pos_advance, int32_t * hist, float * mhist, int64_t hist_stride,
                              const int32_t * hist_base, void * scratch, int flags, acb_stream_t stream);

/* acb_argmax for callers that cannot allocate device memory when they sample: a host whose own
 * pool owns the whole device and forbids allocations it did not make, or a decode thread that
 * must never call cudaMalloc because it can synchronise the device. No counterpart in the
 * reference (which samples on the host). Same arguments and results as acb_argmax without
 * `scratch`: the scratch is a fixed array in the library's device memory (64.25 KB), sized for
 * ACB_ARGMAX_NOALLOC_MAX_ROWS rows of any vocabulary, which every device that loads the
 * library holds until the process exits. More rows return ACB_ERR_UNSUPPORTED (message in
 * acb_last_error) without launching anything. Nothing is allocated by the call. The first call
 * on each device looks up the array's device address and clears its counters with an
 * asynchronous memset on the caller's stream, so make that first call outside any stream
 * capture; afterwards calls of any shape, in any order, leave the array reusable. All calls on
 * a device share the array: calls that overlap on the GPU (different streams, no ordering) race
 * and must be serialised by the caller. The device address is cached per device ordinal for the
 * life of the process: do not use this entry point again after cudaDeviceReset. */
#define ACB_ARGMAX_NOALLOC_MAX_ROWS 32
ACB_API acb_status acb_argmax_noalloc(const float * logits, int64_t stride, int64_t V, int rows, int32_t * ids,
                                      float * margin, int32_t * pos_advance, int32_t * hist, float * mhist,
                                      int64_t hist_stride, const int32_t * hist_base, int flags, acb_stream_t stream);

/* ---- whole batch-1 decode step in one persistent launch ------------------------------------
 * One Qwen3 LM decode step for one sequence (qw3lm_forward_batch with N = 1,
 * src/qwen3-lm.h:557-823, and the temperature-0 sampler, src/sampling.h:30-34) as a single
 * cooperative kernel with one CTA per SM: token gather, every layer (RMSNorm -> QKV GEMV ->
 * q/k-norm + RoPE + f16 cache write -> f16-cache attention -> o GEMV + residual -> RMSNorm ->
 * gate|up GEMV -> SwiGLU -> down GEMV + residual), final RMSNorm, the head GEMV and the argmax.
 * Each CTA's weight bytes stream through its shared-memory ring without a break across layers;
 * stages that need the whole previous vector wait at a bounded grid-wide barrier. Arithmetic per
 * op is that of the separate kernels (acb_gemv on ACB_TYPE_Q8_0_TILES, acb_qkv_post,
 * acb_attn_decode, acb_argmax). */
typedef struct acb_decode_layer {
    const void *  qkv;       /* Q8_0_TILES [Nh*D + 2*Nkv*D][H]: q rows, k rows, v rows */
    const void *  o;         /* Q8_0_TILES [H][Nh*D] */
    const void *  gate_up;   /* Q8_0_TILES [2F][H]: gate rows, then up rows */
    const void *  down;      /* Q8_0_TILES [H][F] */
    const float * attn_norm; /* [H] */
    const float * post_norm; /* [H] */
    const float * q_norm;    /* [D] or NULL */
    const float * k_norm;    /* [D] or NULL */
    uint16_t *    k_cache;   /* f16 [n_sets][Nkv][max_seq][D] of this layer */
    uint16_t *    v_cache;
} acb_decode_layer;

typedef struct acb_decode_step {
    const acb_decode_layer * layers; /* device array [n_layers] */
    int           n_layers, hidden, ffn, n_heads, n_kv_heads, head_dim; /* head_dim 128; Nh/Nkv in {1,2,4} */
    float         eps, attn_scale;
    int           max_seq, max_pos, kv_set;
    const void *  embed;      /* Q8_0 GGUF rows [embed_rows][H] (token gather) */
    int64_t       embed_rows;
    const void *  head;       /* Q8_0_TILES [vocab][H] */
    int64_t       vocab;      /* multiple of 16 */
    const float * final_norm; /* [H] */
    const float * rope;       /* [max_pos][D]: (cos, sin) of pair i at 2i, 2i+1 */
    int32_t *     ids;        /* [1] token of this step; the next token when greedy */
    int32_t *     pos;        /* [1] kv position of this step; += 1 when greedy */
    float *       logits;     /* [vocab] */
    int           greedy;     /* 1: argmax -> ids[0], margin, history, pos[0] += 1 */
    int           n_steps;    /* greedy tokens decoded by this launch (each step feeds the last argmax;
                                 <= 1: one step); history holds every step, ids / pos / margin the last */
    float *       margin;     /* [1] top1 - top2, or NULL */
    int32_t *     hist;       /* token history [max_seq] at pos - hist_base[0], or NULL */
    float *       mhist;      /* margin history, or NULL */
    const int32_t * hist_base;
    void *        scratch;    /* acb_lm_decode_scratch_bytes, zeroed before first use; every
                                 successful step leaves its counters at zero */
    int *         err;        /* ACB_DEVERR_* bits */
} acb_decode_step;

/* Device scratch the step needs (0 when the shape is unsupported: see acb_last_error). */
ACB_API size_t acb_lm_decode_scratch_bytes(const acb_decode_step * step);
/* Enqueue one step. ACB_ERR_UNSUPPORTED for shapes outside the kernel (head_dim != 128,
 * Nh/Nkv not in {1,2,4}, a width above 12288 or not a multiple of 32, N not a multiple of 16)
 * or a device that cannot hold one CTA per SM; the caller keeps its per-op path for those.
 * After a step that raised a device error the scratch must be zeroed again. */
ACB_API acb_status acb_lm_decode_step(const acb_decode_step * step, acb_stream_t stream);

/* ---- bounded device-side wait ---------------------------------------------------------------
 * Holds `stream` on the device until the 32-bit word at `flag` is >= `value` (unsigned compare,
 * system-scope acquire loads), so later work on the stream sees what the producer wrote before
 * raising it. The producer can be the host (a flag in mapped pinned memory), a peer GPU (P2P /
 * IPC memory) or work on another stream that is already running; never a kernel that could be
 * scheduled only after this one on the same GPU. After limit_ns nanoseconds (1 ns .. 10 s) of
 * waiting it gives up: ACB_DEVERR_TIMEOUT is OR-ed into *err_flag (may be NULL), the stream goes
 * on and the context stays usable, so a producer that never comes is reported instead of hanging
 * the GPU. It is the same bounded poll as the persistent decode step's grid barrier. No
 * counterpart in the reference. */
ACB_API acb_status acb_stream_wait_flag(const uint32_t * flag, uint32_t value, uint64_t limit_ns, int * err_flag,
                                        acb_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif
