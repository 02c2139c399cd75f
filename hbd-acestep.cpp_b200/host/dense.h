// dense.h -- the tensor-core linear shared by the prefill-shaped drivers (text encoder, DiT):
// ggml_mul_mat(W, x) at M = tokens (src/qwen3-enc.h:86-88, src/dit-graph.h:36-49) over a
// resident 16-bit copy of W, with the activation quantised the way ggml's quantised mul_mat
// does it (acb_act_quant_ex).
//
// Two arithmetic modes share one weight copy:
//   exact  quantised weights are stored as [hi | lo | hi] f16 along K (hi + lo == the dequantised
//          value) and the activation as [hi | hi | lo]; one GEMM over 3K then forms every
//          product of the reference's dequantised operands to ~2^-22 and accumulates in fp32,
//          so results track the reference CPU build to fp32 summation order;
//   fast   the GEMM reads only the hi columns (K): f16 operands, 3x less tensor work, f16
//          rounding of both operands.
// F16 and BF16 weights are exact in one pass (ggml rounds the activation to the weight type).
#pragma once

#include <cuda_runtime.h>

#include <vector>

#include "../../include/acb.h"
#include "weights.h"

namespace acb {

struct DenseLinear {
    uint16_t * w     = nullptr;  // [N][ldw] 16-bit
    int64_t    ldw   = 0;        // K, or 3K when split
    int        N     = 0;
    int        K     = 0;
    int        vec   = -1;     // ggml vec-dot type of the source weights
    int        op    = 0;      // ACB_FLAG_F16 or 0 (bf16 operands)
    bool       split = false;  // weights stored as [hi | lo | hi]

    int act_type() const { return op ? ACB_TYPE_F16 : ACB_TYPE_BF16; }

    // 16-bit elements of the stored copy of `parts` stacked by rows
    static size_t elems(const std::vector<DevTensor *> & parts);
};

// Build the resident copy of `parts` stacked by row concatenation (gf_load_qkv_fused /
// gf_load_pair_fused, src/gguf-weights.h:281-354) at dst. ids: device int32 0..max rows-1;
// tmp: device f32 scratch of max N*K floats. Enqueued on st.
acb_status dense_build(DenseLinear & L, const std::vector<DevTensor *> & parts, uint16_t * dst, const int32_t * ids,
                       float * tmp, cudaStream_t st);

// Scratch of one dense call: the quantised activation and the split-K workspace.
struct DenseScratch {
    void *  xq       = nullptr;  // >= rows * 3K 16-bit elements
    void *  ws       = nullptr;
    size_t  ws_bytes = 0;
    int *   err      = nullptr;
};

// Row normalisation applied to x inside the activation producer (acb_norm_quant): RMSNorm times
// w, then, with scale/shift, the adaLN modulation n * (1 + scale) + shift (one vector pair every
// rows_per_sample rows, vec_stride apart).
struct NormSpec {
    const float * w               = nullptr;
    float         eps             = 0.0f;
    const float * scale           = nullptr;
    const float * shift           = nullptr;
    int64_t       vec_stride      = 0;
    int64_t       rows_per_sample = 1;
};

// C[M][N] = epi(x . W^T): x f32 [M][xs] (with up_off > 0: silu(x) * x[up_off + .], the SwiGLU
// input of a down projection); bias f32 [N] optional; res/gate as acb_gemm_tc.
acb_status dense_forward(const DenseLinear & L, bool exact, const float * x, int64_t xs, int64_t up_off, int M,
                         void * C, int c_type, int64_t ldc, const float * bias, const float * res, int64_t ldr,
                         const float * gate, int64_t gate_stride, int64_t rows_per_sample, const DenseScratch & s,
                         cudaStream_t st, const NormSpec * norm = nullptr);

// The activation operand of L for x (normalised first by `norm` when given) into s.xq, as
// dense_forward produces it; *width = its row length (K, or 3K in the exact split layout).
acb_status dense_operand(const DenseLinear & L, bool exact, const float * x, int64_t xs, int M, const DenseScratch & s,
                         cudaStream_t st, const NormSpec * norm, int64_t * width);

// How a fused producer (the attention epilogue, acb_attn_tc) writes L's activation operand into
// s.xq itself: its o_type, flags (ACB_FLAG_GEMM_A for the exact layout) and row width. False when
// only acb_act_quant_ex can produce it (Q8_K blocks span 256 columns).
bool dense_operand_spec(const DenseLinear & L, bool exact, int * o_type, int * flags, int64_t * width);

// C = epi(xq . W^T) for an activation operand that a fused producer already wrote to s.xq.
acb_status dense_forward_operand(const DenseLinear & L, bool exact, int M, void * C, int c_type, int64_t ldc,
                                 const float * bias, const float * res, int64_t ldr, const float * gate,
                                 int64_t gate_stride, int64_t rows_per_sample, const DenseScratch & s,
                                 cudaStream_t st);

// Rows from which the q/k/v projection runs with the QKV epilogue (acb_gemm_qkv_planes; fewer rows
// take the split-K GEMM and the separate norm / transpose passes). ACB_QKV_FUSE_MIN_ROWS in the
// environment (read once) overrides the default.
int qkv_fuse_min_rows();

// Rows from which the feed-forward block runs its gate/up GEMM with the SwiGLU epilogue (the
// fused form needs whole waves of 256-row tiles to pay off; fewer rows take the split-K path).
// ACB_FFN_FUSE_MIN_ROWS overrides the default.
int ffn_fuse_min_rows();

// Feed-forward block out = epi(down(swiglu(gate_up(x)))) (ggml_swiglu between the two
// projections, src/dit-graph.h:259-268, src/qwen3-enc.h:217-223): x f32 [M][xs] (normalised
// first by `norm` when given), out f32 [M][ldo] with res / gate as acb_gemm_tc. gu_buf holds
// max(M * 2F f32, M * 3F 16-bit) bytes: the f32 gate/up product, or, when the gate/up GEMM
// fuses SwiGLU and the down projection's quantisation into its epilogue, that operand.
acb_status dense_ffn(const DenseLinear & Lgu, const DenseLinear & Ldown, bool exact, const float * x, int64_t xs,
                     int M, float * out, int64_t ldo, const float * res, int64_t ldr, const float * gate,
                     int64_t gate_stride, int64_t rows_per_sample, void * gu_buf, const DenseScratch & s,
                     cudaStream_t st, const NormSpec * norm = nullptr);

}  // namespace acb
