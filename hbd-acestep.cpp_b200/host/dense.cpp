// dense.cpp -- tensor-core linears with the reference's quantised mul_mat arithmetic.
#include "dense.h"

#include <cstdlib>

#include "host_common.h"

namespace acb {

// Weights whose values are not exact in one 16-bit operand: quantised blocks (f16/f32 scale
// times an integer) and F32.
static bool splits_weights(int vec) {
    return vec == ACB_TYPE_Q8_0 || vec == ACB_TYPE_Q8_K || vec == ACB_TYPE_F32;
}

size_t DenseLinear::elems(const std::vector<DevTensor *> & parts) {
    size_t n = 0;
    for (const DevTensor * t : parts) {
        n += (size_t) t->N * (size_t) t->K;
    }
    return parts.empty() ? 0 : n * (splits_weights(acb_vec_dot_type(parts[0]->type)) ? 3 : 1);
}

static int env_rows(const char * name, int fallback) {
    const char * e = std::getenv(name);
    return e && *e ? std::atoi(e) : fallback;
}

int qkv_fuse_min_rows() {
    static const int v = env_rows("ACB_QKV_FUSE_MIN_ROWS", 1024);
    return v;
}

int ffn_fuse_min_rows() {
    static const int v = env_rows("ACB_FFN_FUSE_MIN_ROWS", 1024);
    return v;
}

acb_status dense_build(DenseLinear & L, const std::vector<DevTensor *> & parts, uint16_t * dst, const int32_t * ids,
                       float * tmp, cudaStream_t st) {
    if (parts.empty()) {
        return ACB_ERR_INVALID_ARG;
    }
    const int vt = acb_vec_dot_type(parts[0]->type);
    if (vt < 0) {
        set_last_error("weight type without a tensor-core path");
        return ACB_ERR_UNSUPPORTED;
    }
    for (const DevTensor * t : parts) {
        if (acb_vec_dot_type(t->type) != vt || t->K != parts[0]->K) {
            set_last_error("stacked projections with different vec-dot types or widths");
            return ACB_ERR_UNSUPPORTED;
        }
    }
    const int64_t K = parts[0]->K;
    L.w             = dst;
    L.vec           = vt;
    L.op            = vt == ACB_TYPE_BF16 ? 0 : ACB_FLAG_F16;
    L.K             = (int) K;
    L.split         = splits_weights(vt);
    L.ldw           = L.split ? 3 * K : K;
    int64_t rows    = 0;
    for (const DevTensor * t : parts) {
        uint16_t * d = dst + rows * L.ldw;
        if (L.split) {
            // exact f32 dequantisation, then the [hi | lo | hi] split of every value
            ACB_TRY(acb_get_rows(t->data, t->type, t->N, K, ids, t->N, tmp, ACB_TYPE_F32, K, nullptr,
                                 (acb_stream_t) st));
            ACB_TRY(acb_act_quant_ex(tmp, K, 0, t->N, K, ACB_TYPE_F16, ACB_LAYOUT_GEMM_B, d, ACB_TYPE_F16, L.ldw, 0,
                                     (acb_stream_t) st));
        } else {
            ACB_TRY(acb_get_rows(t->data, t->type, t->N, K, ids, t->N, d, L.act_type(), K, nullptr,
                                 (acb_stream_t) st));
        }
        rows += t->N;
    }
    L.N = (int) rows;
    return ACB_OK;
}

acb_status dense_forward(const DenseLinear & L, bool exact, const float * x, int64_t xs, int64_t up_off, int M,
                         void * C, int c_type, int64_t ldc, const float * bias, const float * res, int64_t ldr,
                         const float * gate, int64_t gate_stride, int64_t rows_per_sample, const DenseScratch & s,
                         cudaStream_t st, const NormSpec * norm) {
    const bool    three  = exact && L.split;
    const int64_t Kp     = three ? 3 * (int64_t) L.K : L.K;
    const int     layout = three ? ACB_LAYOUT_GEMM_A : ACB_LAYOUT_PLAIN;
    if (norm) {
        if (up_off != 0) {
            return ACB_ERR_INVALID_ARG;
        }
        ACB_TRY(acb_norm_quant(x, xs, M, L.K, norm->w, norm->eps, norm->scale, norm->shift, norm->vec_stride,
                               norm->rows_per_sample, L.vec, layout, s.xq, L.act_type(), Kp, 0, (acb_stream_t) st));
    } else {
        ACB_TRY(acb_act_quant_ex(x, xs, up_off, M, L.K, L.vec, layout, s.xq, L.act_type(), Kp, 0, (acb_stream_t) st));
    }
    return acb_gemm_tc(s.xq, Kp, L.w, L.ldw, M, L.N, Kp, C, c_type, ldc, bias, res, ldr, gate, gate_stride,
                       rows_per_sample, ACB_FLAG_PDL | L.op, s.ws, s.ws_bytes, s.err, (acb_stream_t) st);
}

acb_status dense_operand(const DenseLinear & L, bool exact, const float * x, int64_t xs, int M, const DenseScratch & s,
                         cudaStream_t st, const NormSpec * norm, int64_t * width) {
    const bool    three  = exact && L.split;
    const int64_t Kp     = three ? 3 * (int64_t) L.K : L.K;
    const int     layout = three ? ACB_LAYOUT_GEMM_A : ACB_LAYOUT_PLAIN;
    *width               = Kp;
    if (norm) {
        return acb_norm_quant(x, xs, M, L.K, norm->w, norm->eps, norm->scale, norm->shift, norm->vec_stride,
                              norm->rows_per_sample, L.vec, layout, s.xq, L.act_type(), Kp, 0, (acb_stream_t) st);
    }
    return acb_act_quant_ex(x, xs, 0, M, L.K, L.vec, layout, s.xq, L.act_type(), Kp, 0, (acb_stream_t) st);
}

bool dense_operand_spec(const DenseLinear & L, bool exact, int * o_type, int * flags, int64_t * width) {
    if (L.vec != ACB_TYPE_Q8_0 && L.vec != ACB_TYPE_F16 && L.vec != ACB_TYPE_BF16 && L.vec != ACB_TYPE_F32) {
        return false;
    }
    const bool three = exact && L.split;
    *o_type          = L.vec == ACB_TYPE_Q8_0 ? ACB_TYPE_Q8_0 : (L.vec == ACB_TYPE_BF16 ? ACB_TYPE_BF16 : ACB_TYPE_F16);
    *flags           = three ? ACB_FLAG_GEMM_A : 0;
    *width           = three ? 3 * (int64_t) L.K : L.K;
    return true;
}

acb_status dense_forward_operand(const DenseLinear & L, bool exact, int M, void * C, int c_type, int64_t ldc,
                                 const float * bias, const float * res, int64_t ldr, const float * gate,
                                 int64_t gate_stride, int64_t rows_per_sample, const DenseScratch & s,
                                 cudaStream_t st) {
    const int64_t Kp = (exact && L.split) ? 3 * (int64_t) L.K : L.K;
    return acb_gemm_tc(s.xq, Kp, L.w, L.ldw, M, L.N, Kp, C, c_type, ldc, bias, res, ldr, gate, gate_stride,
                       rows_per_sample, ACB_FLAG_PDL | L.op, s.ws, s.ws_bytes, s.err, (acb_stream_t) st);
}

acb_status dense_ffn(const DenseLinear & Lgu, const DenseLinear & Ldown, bool exact, const float * x, int64_t xs,
                     int M, float * out, int64_t ldo, const float * res, int64_t ldr, const float * gate,
                     int64_t gate_stride, int64_t rows_per_sample, void * gu_buf, const DenseScratch & s,
                     cudaStream_t st, const NormSpec * norm) {
    const int64_t F         = Ldown.K;
    const bool    down3     = exact && Ldown.split;
    const int     vt        = Ldown.vec;
    const bool    fusable   = Lgu.N == 2 * F && F % 128 == 0 && M >= ffn_fuse_min_rows() &&
                         (vt == ACB_TYPE_Q8_0 || vt == ACB_TYPE_F16 || vt == ACB_TYPE_BF16) &&
                         Lgu.op == Ldown.op;
    if (!fusable) {
        ACB_TRY(dense_forward(Lgu, exact, x, xs, 0, M, gu_buf, ACB_TYPE_F32, 2 * F, nullptr, nullptr, 0, nullptr, 0, 0,
                              s, st, norm));
        return dense_forward(Ldown, exact, static_cast<const float *>(gu_buf), 2 * F, F, M, out, ACB_TYPE_F32, ldo,
                             nullptr, res, ldr, gate, gate_stride, rows_per_sample, s, st);
    }
    // activation of the gate/up projection
    const bool    three  = exact && Lgu.split;
    const int64_t Kp     = three ? 3 * (int64_t) Lgu.K : Lgu.K;
    const int     layout = three ? ACB_LAYOUT_GEMM_A : ACB_LAYOUT_PLAIN;
    if (norm) {
        ACB_TRY(acb_norm_quant(x, xs, M, Lgu.K, norm->w, norm->eps, norm->scale, norm->shift, norm->vec_stride,
                               norm->rows_per_sample, Lgu.vec, layout, s.xq, Lgu.act_type(), Kp, 0, (acb_stream_t) st));
    } else {
        ACB_TRY(acb_act_quant_ex(x, xs, 0, M, Lgu.K, Lgu.vec, layout, s.xq, Lgu.act_type(), Kp, 0, (acb_stream_t) st));
    }
    // gate/up GEMM with SwiGLU and the down projection's quantisation in its epilogue
    const int64_t Kd = down3 ? 3 * F : F;
    ACB_TRY(acb_gemm_swiglu_quant(s.xq, Kp, Lgu.w, Lgu.ldw, M, F, Kp, nullptr, vt,
                                  down3 ? ACB_LAYOUT_GEMM_A : ACB_LAYOUT_PLAIN, gu_buf, Ldown.act_type(), Kd,
                                  ACB_FLAG_PDL | Lgu.op, s.err, (acb_stream_t) st));
    return acb_gemm_tc(gu_buf, Kd, Ldown.w, Ldown.ldw, M, Ldown.N, Kd, out, ACB_TYPE_F32, ldo, nullptr, res, ldr, gate,
                       gate_stride, rows_per_sample, ACB_FLAG_PDL | Ldown.op, s.ws, s.ws_bytes, s.err,
                       (acb_stream_t) st);
}

}  // namespace acb
