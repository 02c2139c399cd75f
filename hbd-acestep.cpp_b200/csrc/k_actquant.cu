// k_actquant.cu -- activation operand of the tensor-core linears with ggml-CPU's quantised
// mul_mat arithmetic (the from_float step of ggml_mul_mat for Q8_0 / Q4_K / Q6_K / F16 / BF16
// weights, reached from src/qwen3-enc.h:86-88 and src/dit-graph.h:36-49).
//
// One warp per 256-element chunk of a row; lane l holds elements [8l, 8l+8) in registers
// (two 16-byte loads). Q8_0 blocks of 32 are four consecutive lanes (two xor shuffles for the
// block max); a Q8_K block of 256 is the whole warp (five shuffles carrying value and index,
// so the first element of largest magnitude wins as in the sequential reference). The
// dequantised values d*q are written as f16 with one 16-byte store per lane. The SwiGLU variant
// computes silu(g)*u from fused [gate | up] rows first (ggml_swiglu followed by the down
// projection's quantisation, src/qwen3-enc.h:217-223, src/dit-graph.h:259-268).
#include "common.cuh"

namespace acb {

constexpr int kAqWarps = 8;

__device__ __forceinline__ void load8(const float * p, bool vec, float * v) {
    if (vec) {
        const float4 a = *reinterpret_cast<const float4 *>(p);
        const float4 b = *reinterpret_cast<const float4 *>(p + 4);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
        v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    } else {
#pragma unroll
        for (int e = 0; e < 8; e++) {
            v[e] = p[e];
        }
    }
}

// 8 values of a lane as 16-bit operands at dst (vector store when allowed)
template <int OT> __device__ __forceinline__ void store8(void * dst, const float * o, bool vec) {
    using et = typename io<OT>::t;
    et * yr  = reinterpret_cast<et *>(dst);
    if (vec) {
        vec16<OT> pk;
#pragma unroll
        for (int e = 0; e < 8; e++) {
            pk.v[e] = io<OT>::from_f(o[e]);
        }
        *reinterpret_cast<uint4 *>(yr) = pk.u;
    } else {
#pragma unroll
        for (int e = 0; e < 8; e++) {
            yr[e] = io<OT>::from_f(o[e]);
        }
    }
}

template <int OT, int LAYOUT>
__device__ __forceinline__ void split_store(typename io<OT>::t * yr, const float * o, int64_t K, int64_t lo_off,
                                            bool vec_out);

// ggml's from_float of one lane's 8 consecutive values (v) to the dequantised operand values
// (o): Q8_0 blocks of 32 are four consecutive lanes, a Q8_K block of 256 is the whole warp
// (all 32 lanes must call it together); F16 / BF16 / F32 pass the values through.
template <int VT> __device__ __forceinline__ void quant8(const float * v, int lane, float * o) {
    if (VT == ACB_TYPE_Q8_0) {
        float amax = 0.0f;
#pragma unroll
        for (int e = 0; e < 8; e++) {
            amax = fmaxf(amax, fabsf(v[e]));
        }
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
        const float d  = __fdiv_rn(amax, 127.0f);
        const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        const float dh = __half2float(__float2half_rn(d));  // the block stores d as f16
#pragma unroll
        for (int e = 0; e < 8; e++) {
            // through an int, as the block stores it: a rounded -0.x is +0
            o[e] = __fmul_rn(dh, (float) (int) roundf(__fmul_rn(v[e], id)));
        }
    } else if (VT == ACB_TYPE_Q8_K) {
        float amax = 0.0f, mx = 0.0f;
        int   idx  = 0x7fffffff;
#pragma unroll
        for (int e = 0; e < 8; e++) {
            const float a = fabsf(v[e]);
            if (a > amax) {  // first index of the largest magnitude within the lane
                amax = a;
                mx   = v[e];
                idx  = lane * 8 + e;
            }
        }
#pragma unroll
        for (int s = 1; s < 32; s <<= 1) {
            const float oa = __shfl_xor_sync(0xffffffffu, amax, s);
            const float om = __shfl_xor_sync(0xffffffffu, mx, s);
            const int   oi = __shfl_xor_sync(0xffffffffu, idx, s);
            if (oa > amax || (oa == amax && oi < idx)) {
                amax = oa;
                mx   = om;
                idx  = oi;
            }
        }
        if (amax == 0.0f) {
#pragma unroll
            for (int e = 0; e < 8; e++) {
                o[e] = 0.0f;
            }
        } else {
            const float iscale = __fdiv_rn(-127.0f, mx);
            const float d      = __fdiv_rn(1.0f, iscale);
#pragma unroll
            for (int e = 0; e < 8; e++) {
                int q = __float2int_rn(__fmul_rn(iscale, v[e]));
                q     = q < 127 ? q : 127;
                o[e]  = __fmul_rn(d, (float) q);
            }
        }
    } else {
#pragma unroll
        for (int e = 0; e < 8; e++) {
            o[e] = v[e];
        }
    }
}


template <int VT, bool SWIGLU, int LAYOUT>
__global__ void __launch_bounds__(kAqWarps * 32)
    act_quant_kernel(const float * __restrict__ x, int64_t xs, int64_t up_off, int64_t rows, int64_t K,
                     void * __restrict__ y, int64_t ys, int64_t lo_off, bool vec_in, bool vec_out) {
    const int     lane   = threadIdx.x & 31;
    const int64_t chunks = (K + 255) / 256;
    const int64_t item   = (int64_t) blockIdx.x * kAqWarps + (threadIdx.x >> 5);
    if (item >= rows * chunks) {
        return;
    }
    const int64_t r     = item / chunks;
    const int64_t c0    = (item - r * chunks) * 256 + lane * 8;
    const bool    valid = c0 < K;  // K is a multiple of 32: a lane is all in or all out
    const float * xr    = x + r * xs + c0;
    float         v[8];
    if (valid) {
        load8(xr, vec_in, v);
        if (SWIGLU) {
            float u[8];
            load8(xr + up_off, vec_in, u);
#pragma unroll
            for (int e = 0; e < 8; e++) {
                v[e] = silu_times(v[e], u[e]);
            }
        }
    } else {
#pragma unroll
        for (int e = 0; e < 8; e++) {
            v[e] = 0.0f;
        }
    }

    float o[8];
    quant8<VT>(v, lane, o);
    if (!valid) {
        return;
    }
    constexpr int OT = VT == ACB_TYPE_BF16 ? ACB_TYPE_BF16 : ACB_TYPE_F16;
    using et         = typename io<OT>::t;
    et * yr          = reinterpret_cast<et *>(y) + r * ys + c0;
    if constexpr (LAYOUT == ACB_LAYOUT_PLAIN) {
        store8<OT>(yr, o, vec_out);
    } else {
        split_store<OT, LAYOUT>(yr, o, K, lo_off, vec_out);
    }
}

template <int OT, int LAYOUT>
__device__ __forceinline__ void split_store(typename io<OT>::t * yr, const float * o, int64_t K, int64_t lo_off,
                                            bool vec_out) {
    // exact split: hi = f16(v), lo = f16(v - hi); v - hi is exact in f32, and for values of at
    // most 22 significant bits (every dequantised operand here has <= 18) hi + lo == v exactly
    float hi[8], lo[8];
#pragma unroll
    for (int e = 0; e < 8; e++) {
        hi[e] = io<OT>::to_f(io<OT>::from_f(o[e]));
        lo[e] = __fsub_rn(o[e], hi[e]);
    }
    if (LAYOUT == ACB_LAYOUT_GEMM_A) {  // [hi | hi | lo] along K
        store8<OT>(yr, hi, vec_out);
        store8<OT>(yr + K, hi, vec_out);
        store8<OT>(yr + 2 * K, lo, vec_out);
    } else if (LAYOUT == ACB_LAYOUT_GEMM_B) {  // [hi | lo | hi] along K
        store8<OT>(yr, hi, vec_out);
        store8<OT>(yr + K, lo, vec_out);
        store8<OT>(yr + 2 * K, hi, vec_out);
    } else {  // ACB_LAYOUT_PLANES: hi here, lo at lo_off elements further
        store8<OT>(yr, hi, vec_out);
        store8<OT>(yr + lo_off, lo, vec_out);
    }
}


// RMSNorm (+ weight) [+ adaLN modulate] of a row followed by the quantisation above, in one pass:
// ggml_rms_norm -> ggml_mul(w) [-> ggml_mul(1 + scale) -> ggml_add(shift)] and then the
// from_float of the next ggml_mul_mat (src/dit-graph.h:150-157, 250-258; src/qwen3-enc.h:80-90),
// with every product and sum rounded as those separate graph nodes round them. One CTA per row,
// one warp per 256-element chunk (lane l holds elements [256w + 8l, +8) in registers); the
// row's sum of squares (double) is combined across warps through shared memory in warp order.
// Without a weight, the adaLN form skips the normalisation (as acb_adaln_modulate does).
template <int VT, int LAYOUT, bool ADALN>
__global__ void __launch_bounds__(512)
    norm_quant_kernel(const float * __restrict__ x, int64_t xs, int64_t K, const float * __restrict__ w,
                      float eps, const float * __restrict__ scale, const float * __restrict__ shift, int64_t vs,
                      int64_t rps, void * __restrict__ y, int64_t ys, int64_t lo_off, bool vec_in, bool vec_out) {
    __shared__ double part[16];
    const int     lane  = threadIdx.x & 31, wid = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int64_t r     = blockIdx.x;
    const int64_t c0    = (int64_t) wid * 256 + lane * 8;
    const bool    valid = c0 < K;  // K is a multiple of 32: a lane is all in or all out
    float         v[8];
    if (valid) {
        load8(x + r * xs + c0, vec_in, v);
    } else {
#pragma unroll
        for (int e = 0; e < 8; e++) {
            v[e] = 0.0f;
        }
    }
    const bool do_norm = !ADALN || w != nullptr;
    float      sc      = 1.0f;
    if (do_norm) {
        double ss = 0.0;
#pragma unroll
        for (int e = 0; e < 8; e++) {
            ss += (double) __fmul_rn(v[e], v[e]);
        }
        ss = warp_sum(ss);
        if (lane == 0) {
            part[wid] = ss;
        }
        __syncthreads();
        double t = 0.0;
        for (int i = 0; i < nw; i++) {
            t += part[i];
        }
        sc = rms_scale(t, (int) K, eps);
    }
    const int64_t smp = ADALN ? r / rps : 0;
    float         f[8], wv[8], a[8], b[8];
    if (valid) {
        // the weight and modulation vectors: 16-byte loads when aligned (vec_in covers them)
        if (w) {
            load8(w + c0, vec_in, wv);
        }
        if (ADALN) {
            load8(scale + smp * vs + c0, vec_in, a);
            load8(shift + smp * vs + c0, vec_in, b);
        }
    }
#pragma unroll
    for (int e = 0; e < 8; e++) {
        float t = v[e];
        if (valid) {
            if (do_norm) {
                t = __fmul_rn(t, sc);
                if (w) {
                    t = __fmul_rn(t, wv[e]);
                }
            }
            if (ADALN) {
                t = __fadd_rn(__fmul_rn(t, __fadd_rn(a[e], 1.0f)), b[e]);
            }
        }
        f[e] = t;
    }
    float o[8];
    quant8<VT>(f, lane, o);
    if (!valid) {
        return;
    }
    constexpr int OT = VT == ACB_TYPE_BF16 ? ACB_TYPE_BF16 : ACB_TYPE_F16;
    using et         = typename io<OT>::t;
    et * yr          = reinterpret_cast<et *>(y) + r * ys + c0;
    if constexpr (LAYOUT == ACB_LAYOUT_PLAIN) {
        store8<OT>(yr, o, vec_out);
    } else {
        split_store<OT, LAYOUT>(yr, o, K, lo_off, vec_out);
    }
}

}  // namespace acb

using namespace acb;

extern "C" int acb_vec_dot_type(int weight_type) {
    switch (weight_type) {
        case ACB_TYPE_Q8_0:
            return ACB_TYPE_Q8_0;
        case ACB_TYPE_Q4_K:
        case ACB_TYPE_Q6_K:
            return ACB_TYPE_Q8_K;
        case ACB_TYPE_F16:
            return ACB_TYPE_F16;
        case ACB_TYPE_BF16:
            return ACB_TYPE_BF16;
        case ACB_TYPE_F32:
            return ACB_TYPE_F32;
        default:
            return -1;
    }
}

template <int VT, bool SWIGLU>
static void launch_layout(int layout, dim3 grid, cudaStream_t st, const float * x, int64_t xs, int64_t up_off,
                          int64_t rows, int64_t K, void * y, int64_t ys, int64_t lo_off, bool vin, bool vout) {
#define ACB_AQL(L) \
    act_quant_kernel<VT, SWIGLU, L><<<grid, kAqWarps * 32, 0, st>>>(x, xs, up_off, rows, K, y, ys, lo_off, vin, vout)
    switch (layout) {
        case ACB_LAYOUT_GEMM_A:
            ACB_AQL(ACB_LAYOUT_GEMM_A);
            break;
        case ACB_LAYOUT_GEMM_B:
            ACB_AQL(ACB_LAYOUT_GEMM_B);
            break;
        case ACB_LAYOUT_PLANES:
            ACB_AQL(ACB_LAYOUT_PLANES);
            break;
        default:
            ACB_AQL(ACB_LAYOUT_PLAIN);
    }
#undef ACB_AQL
}

template <bool SWIGLU>
static acb_status launch_act_quant(const float * x, int64_t x_stride, int64_t up_off, int64_t rows, int64_t K,
                                   int vec_type, int layout, void * y, int y_type, int64_t y_stride, int64_t lo_off,
                                   cudaStream_t st) {
    const int want_y = vec_type == ACB_TYPE_BF16 ? ACB_TYPE_BF16 : ACB_TYPE_F16;
    if (y_type != want_y || K % 32 != 0 || (vec_type == ACB_TYPE_Q8_K && K % 256 != 0) || layout < 0 || layout > 3) {
        return ACB_ERR_UNSUPPORTED;
    }
    if ((layout == ACB_LAYOUT_GEMM_A || layout == ACB_LAYOUT_GEMM_B) && y_stride < 3 * K) {
        return ACB_ERR_INVALID_ARG;
    }
    if (rows == 0) {
        return ACB_OK;
    }
    const bool vin  = (x_stride % 4 == 0) && (up_off % 4 == 0) && (reinterpret_cast<uintptr_t>(x) % 16 == 0);
    const bool vout = (y_stride % 8 == 0) && (K % 8 == 0) && (lo_off % 8 == 0) &&
                      (reinterpret_cast<uintptr_t>(y) % 16 == 0);
    const int64_t items = rows * ((K + 255) / 256);
    const dim3    grid((unsigned) ((items + kAqWarps - 1) / kAqWarps));
    switch (vec_type) {
        case ACB_TYPE_Q8_0:
            launch_layout<ACB_TYPE_Q8_0, SWIGLU>(layout, grid, st, x, x_stride, up_off, rows, K, y, y_stride, lo_off,
                                                 vin, vout);
            break;
        case ACB_TYPE_Q8_K:
            launch_layout<ACB_TYPE_Q8_K, SWIGLU>(layout, grid, st, x, x_stride, up_off, rows, K, y, y_stride, lo_off,
                                                 vin, vout);
            break;
        case ACB_TYPE_F16:
            launch_layout<ACB_TYPE_F16, SWIGLU>(layout, grid, st, x, x_stride, up_off, rows, K, y, y_stride, lo_off,
                                                vin, vout);
            break;
        case ACB_TYPE_F32:
            launch_layout<ACB_TYPE_F32, SWIGLU>(layout, grid, st, x, x_stride, up_off, rows, K, y, y_stride, lo_off,
                                                vin, vout);
            break;
        case ACB_TYPE_BF16:
            launch_layout<ACB_TYPE_BF16, SWIGLU>(layout, grid, st, x, x_stride, up_off, rows, K, y, y_stride, lo_off,
                                                 vin, vout);
            break;
        default:
            return ACB_ERR_UNSUPPORTED;
    }
    return launch_status();
}

extern "C" acb_status acb_act_quant(const float * x, int64_t x_stride, int64_t rows, int64_t K, int vec_type, void * y,
                                    int y_type, int64_t y_stride, acb_stream_t stream) {
    if (!x || !y || rows < 0 || K <= 0 || x_stride < K || y_stride < K) {
        return ACB_ERR_INVALID_ARG;
    }
    return launch_act_quant<false>(x, x_stride, 0, rows, K, vec_type, ACB_LAYOUT_PLAIN, y, y_type, y_stride, 0,
                                   (cudaStream_t) stream);
}

extern "C" acb_status acb_act_quant_swiglu(const float * gu, int64_t gu_stride, int64_t up_offset, int64_t rows,
                                           int64_t F, int vec_type, void * y, int y_type, int64_t y_stride,
                                           acb_stream_t stream) {
    if (!gu || !y || rows < 0 || F <= 0 || up_offset < F || gu_stride < up_offset + F || y_stride < F) {
        return ACB_ERR_INVALID_ARG;
    }
    return launch_act_quant<true>(gu, gu_stride, up_offset, rows, F, vec_type, ACB_LAYOUT_PLAIN, y, y_type, y_stride,
                                  0, (cudaStream_t) stream);
}

extern "C" acb_status acb_act_quant_ex(const float * x, int64_t x_stride, int64_t up_offset, int64_t rows, int64_t K,
                                       int vec_type, int layout, void * y, int y_type, int64_t y_stride,
                                       int64_t lo_offset, acb_stream_t stream) {
    if (!x || !y || rows < 0 || K <= 0 || y_stride < K || up_offset < 0 ||
        (up_offset > 0 && (up_offset < K || x_stride < up_offset + K)) || (up_offset == 0 && x_stride < K)) {
        return ACB_ERR_INVALID_ARG;
    }
    if (layout == ACB_LAYOUT_PLANES && lo_offset == 0) {
        return ACB_ERR_INVALID_ARG;
    }
    if (up_offset > 0) {
        return launch_act_quant<true>(x, x_stride, up_offset, rows, K, vec_type, layout, y, y_type, y_stride,
                                      lo_offset, (cudaStream_t) stream);
    }
    return launch_act_quant<false>(x, x_stride, 0, rows, K, vec_type, layout, y, y_type, y_stride, lo_offset,
                                   (cudaStream_t) stream);
}

namespace {

template <int VT, bool ADALN>
void launch_nq_layout(int layout, dim3 grid, dim3 block, cudaStream_t st, const float * x, int64_t xs, int64_t K,
                      const float * w, float eps, const float * scale, const float * shift, int64_t vs, int64_t rps,
                      void * y, int64_t ys, int64_t lo_off, bool vin, bool vout) {
#define ACB_NQL(L)                                                                                                \
    norm_quant_kernel<VT, L, ADALN><<<grid, block, 0, st>>>(x, xs, K, w, eps, scale, shift, vs, rps, y, ys, lo_off, \
                                                            vin, vout)
    switch (layout) {
        case ACB_LAYOUT_GEMM_A:
            ACB_NQL(ACB_LAYOUT_GEMM_A);
            break;
        case ACB_LAYOUT_PLANES:
            ACB_NQL(ACB_LAYOUT_PLANES);
            break;
        default:
            ACB_NQL(ACB_LAYOUT_PLAIN);
    }
#undef ACB_NQL
}

template <bool ADALN>
acb_status launch_norm_quant(int vec_type, int layout, const float * x, int64_t xs, int64_t rows, int64_t K,
                             const float * w, float eps, const float * scale, const float * shift, int64_t vs,
                             int64_t rps, void * y, int64_t ys, int64_t lo_off, cudaStream_t st) {
    const bool vin = (xs % 4 == 0) && (reinterpret_cast<uintptr_t>(x) % 16 == 0) &&
                     (reinterpret_cast<uintptr_t>(w) % 16 == 0) && (reinterpret_cast<uintptr_t>(scale) % 16 == 0) &&
                     (reinterpret_cast<uintptr_t>(shift) % 16 == 0) && vs % 4 == 0;
    const bool vout =
        (ys % 8 == 0) && (K % 8 == 0) && (lo_off % 8 == 0) && (reinterpret_cast<uintptr_t>(y) % 16 == 0);
    const dim3 grid((unsigned) rows);
    const dim3 block((unsigned) (((K + 255) / 256) * 32));
#define ACB_NQV(V) \
    launch_nq_layout<V, ADALN>(layout, grid, block, st, x, xs, K, w, eps, scale, shift, vs, rps, y, ys, lo_off, vin, vout)
    switch (vec_type) {
        case ACB_TYPE_Q8_0:
            ACB_NQV(ACB_TYPE_Q8_0);
            break;
        case ACB_TYPE_Q8_K:
            ACB_NQV(ACB_TYPE_Q8_K);
            break;
        case ACB_TYPE_F16:
            ACB_NQV(ACB_TYPE_F16);
            break;
        case ACB_TYPE_F32:
            ACB_NQV(ACB_TYPE_F32);
            break;
        case ACB_TYPE_BF16:
            ACB_NQV(ACB_TYPE_BF16);
            break;
        default:
            return ACB_ERR_UNSUPPORTED;
    }
#undef ACB_NQV
    return launch_status();
}

}  // namespace

extern "C" acb_status acb_norm_quant(const float * x, int64_t x_stride, int64_t rows, int64_t K, const float * norm_w,
                                     float eps, const float * scale, const float * shift, int64_t vec_stride,
                                     int64_t rows_per_sample, int vec_type, int layout, void * y, int y_type,
                                     int64_t y_stride, int64_t lo_offset, acb_stream_t stream) {
    if (!x || !y || rows < 0 || K <= 0 || x_stride < K || y_stride < K || (!scale != !shift) || vec_stride < 0 ||
        (scale && rows_per_sample <= 0)) {
        return ACB_ERR_INVALID_ARG;
    }
    if (layout == ACB_LAYOUT_PLANES && lo_offset == 0) {
        return ACB_ERR_INVALID_ARG;
    }
    const int want_y = vec_type == ACB_TYPE_BF16 ? ACB_TYPE_BF16 : ACB_TYPE_F16;
    if (y_type != want_y || K % 32 != 0 || K > 4096 || (vec_type == ACB_TYPE_Q8_K && K % 256 != 0) ||
        layout == ACB_LAYOUT_GEMM_B || layout < 0 || layout > 3) {
        return ACB_ERR_UNSUPPORTED;
    }
    if (layout == ACB_LAYOUT_GEMM_A && y_stride < 3 * K) {
        return ACB_ERR_INVALID_ARG;
    }
    if (rows == 0) {
        return ACB_OK;
    }
    cudaStream_t st = (cudaStream_t) stream;
    if (scale) {
        return launch_norm_quant<true>(vec_type, layout, x, x_stride, rows, K, norm_w, eps, scale, shift, vec_stride,
                                       rows_per_sample, y, y_stride, lo_offset, st);
    }
    return launch_norm_quant<false>(vec_type, layout, x, x_stride, rows, K, norm_w, eps, nullptr, nullptr, 0, 1, y,
                                    y_stride, lo_offset, st);
}
