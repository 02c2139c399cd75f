// k_elementwise.cu -- streaming elementwise ops: SwiGLU and the DiT gated residual.
//
// Both are pure HBM streams. A CTA covers a contiguous run of 16-byte vectors of one row
// (gridDim.y walks rows), every load is a 16-byte streaming load issued before any math, and
// the result is written with a streaming store. silu uses the IEEE float division and CUDA's
// expf; the gated residual keeps ggml's two separately rounded nodes (o*gate, then r + .).
#include "common.cuh"

namespace acb {

// silu(g) * u for an output of type TO. A bf16 output keeps 8 mantissa bits, so the fast exp and
// divide intrinsics (a few f32 ulps) round to the same bf16 value as g / (1 + expf(-g)) except
// within a few ulps of a rounding boundary (then one bf16 step apart); they take the kernel from
// issue-bound to HBM-bound. Other outputs keep the correctly rounded chain.
template <int TO> __device__ __forceinline__ float silu_mul(float g, float u) {
    if constexpr (TO == ACB_TYPE_BF16) {
        return __fmul_rn(__fdividef(g, __fadd_rn(1.0f, __expf(-g))), u);
    } else {
        return silu_times(g, u);
    }
}

template <int TI, int TO, int U>
__global__ void __launch_bounds__(256) swiglu_vec_kernel(const void * __restrict__ gu, int64_t gu_stride,
                                                         int64_t up_off, void * __restrict__ out, int64_t out_stride,
                                                         int64_t rows, int64_t vpr) {
    using VI        = vec16<TI>;
    constexpr int N = VI::N;
    using ei        = typename io<TI>::t;
    using eo        = typename io<TO>::t;
    for (int64_t r = blockIdx.y; r < rows; r += gridDim.y) {
        const ei * g = reinterpret_cast<const ei *>(gu) + r * gu_stride;
        const ei * u = g + up_off;
        eo *       o = reinterpret_cast<eo *>(out) + r * out_stride;
        const int64_t v0 = ((int64_t) blockIdx.x * blockDim.x) * U + threadIdx.x;
        VI gv[U], uv[U];
#pragma unroll
        for (int k = 0; k < U; k++) {
            const int64_t vi = v0 + (int64_t) k * blockDim.x;
            if (vi < vpr) {
                gv[k].load_stream(g + vi * N);
                uv[k].load_stream(u + vi * N);
            }
        }
#pragma unroll
        for (int k = 0; k < U; k++) {
            const int64_t vi = v0 + (int64_t) k * blockDim.x;
            if (vi < vpr) {
                union {
                    eo    e[N];
                    uint4 q[(N * sizeof(eo) + 15) / 16];
                    uint2 h;
                } res;
#pragma unroll
                for (int j = 0; j < N; j++) {
                    res.e[j] = io<TO>::from_f(silu_mul<TO>(gv[k].get(j), uv[k].get(j)));
                }
                eo * dst = o + vi * N;
                if constexpr (N * sizeof(eo) == 8) {
                    __stcs(reinterpret_cast<uint2 *>(dst), res.h);
                } else {
#pragma unroll
                    for (int q = 0; q < (int) (N * sizeof(eo) / 16); q++) {
                        __stcs(reinterpret_cast<uint4 *>(dst) + q, res.q[q]);
                    }
                }
            }
        }
    }
}

template <int TI, int TO>
__global__ void __launch_bounds__(256) swiglu_scalar_kernel(const void * __restrict__ gu, int64_t gu_stride,
                                                            int64_t up_off, void * __restrict__ out,
                                                            int64_t out_stride, int64_t rows, int64_t F) {
    using ei = typename io<TI>::t;
    using eo = typename io<TO>::t;
    for (int64_t r = blockIdx.y; r < rows; r += gridDim.y) {
        const ei * g = reinterpret_cast<const ei *>(gu) + r * gu_stride;
        eo *       o = reinterpret_cast<eo *>(out) + r * out_stride;
        for (int64_t i = (int64_t) blockIdx.x * blockDim.x + threadIdx.x; i < F; i += (int64_t) gridDim.x * blockDim.x) {
            o[i] = io<TO>::from_f(silu_mul<0>(io<TI>::to_f(g[i]), io<TI>::to_f(g[up_off + i])));
        }
    }
}

template <int TI, int TO>
static acb_status launch_swiglu(const void * gu, int64_t gs, int64_t uo, void * out, int64_t os, int64_t rows,
                                int64_t F, cudaStream_t st) {
    constexpr int N  = vec16<TI>::N;
    constexpr int U  = 2;
    const int     si = (int) sizeof(typename io<TI>::t), so = (int) sizeof(typename io<TO>::t);
    const bool    vec = F % N == 0 && reinterpret_cast<uintptr_t>(gu) % 16 == 0 &&
                     reinterpret_cast<uintptr_t>(out) % 16 == 0 && (gs * si) % 16 == 0 && (uo * si) % 16 == 0 &&
                     (os * so) % 16 == 0 && N * so >= 8;
    const unsigned gy = (unsigned) (rows < 65535 ? rows : 65535);
    if (vec) {
        const int64_t vpr = F / N;
        const dim3    grid((unsigned) ((vpr + 256 * U - 1) / (256 * U)), gy);
        swiglu_vec_kernel<TI, TO, U><<<grid, 256, 0, st>>>(gu, gs, uo, out, os, rows, vpr);
    } else {
        const dim3 grid((unsigned) ((F + 255) / 256 < 64 ? (F + 255) / 256 : 64), gy);
        swiglu_scalar_kernel<TI, TO><<<grid, 256, 0, st>>>(gu, gs, uo, out, os, rows, F);
    }
    return launch_status();
}

// ---- gated residual: out = r + o * gate[s] --------------------------------------------------
template <int T, int U>
__global__ void __launch_bounds__(256) gated_vec_kernel(const void * __restrict__ r, const void * __restrict__ o,
                                                        const float * __restrict__ gate, int64_t vs,
                                                        void * __restrict__ out, int64_t rows, int64_t rps,
                                                        int64_t H) {
    using V         = vec16<T>;
    constexpr int N = V::N;
    using e         = typename io<T>::t;
    const int64_t vpr = H / N;
    for (int64_t row = blockIdx.y; row < rows; row += gridDim.y) {
        const e *     rr = reinterpret_cast<const e *>(r) + row * H;
        const e *     oo = reinterpret_cast<const e *>(o) + row * H;
        e *           dd = reinterpret_cast<e *>(out) + row * H;
        const float * g  = gate + (row / rps) * vs;
        const int64_t v0 = ((int64_t) blockIdx.x * blockDim.x) * U + threadIdx.x;
        V             rv[U], ov[U];
#pragma unroll
        for (int k = 0; k < U; k++) {
            const int64_t vi = v0 + (int64_t) k * blockDim.x;
            if (vi < vpr) {
                rv[k].load_stream(rr + vi * N);
                ov[k].load_stream(oo + vi * N);
            }
        }
#pragma unroll
        for (int k = 0; k < U; k++) {
            const int64_t vi = v0 + (int64_t) k * blockDim.x;
            if (vi < vpr) {
                V res;
#pragma unroll
                for (int j = 0; j < N; j += 4) {
                    const float4 gv = __ldg(reinterpret_cast<const float4 *>(g + vi * N + j));
                    const float  ga[4] = { gv.x, gv.y, gv.z, gv.w };
#pragma unroll
                    for (int q = 0; q < 4; q++) {
                        res.set(j + q, __fadd_rn(rv[k].get(j + q), __fmul_rn(ov[k].get(j + q), ga[q])));
                    }
                }
                res.store_stream(dd + vi * N);
            }
        }
    }
}

template <int T>
__global__ void __launch_bounds__(256) gated_scalar_kernel(const void * __restrict__ r, const void * __restrict__ o,
                                                           const float * __restrict__ gate, int64_t vs,
                                                           void * __restrict__ out, int64_t rows, int64_t rps,
                                                           int64_t H) {
    using e = typename io<T>::t;
    for (int64_t row = blockIdx.y; row < rows; row += gridDim.y) {
        const float * g = gate + (row / rps) * vs;
        for (int64_t i = (int64_t) blockIdx.x * blockDim.x + threadIdx.x; i < H; i += (int64_t) gridDim.x * blockDim.x) {
            const float rv = io<T>::to_f(reinterpret_cast<const e *>(r)[row * H + i]);
            const float ov = io<T>::to_f(reinterpret_cast<const e *>(o)[row * H + i]);
            reinterpret_cast<e *>(out)[row * H + i] = io<T>::from_f(__fadd_rn(rv, __fmul_rn(ov, g[i])));
        }
    }
}

template <int T>
static acb_status launch_gated(const void * r, const void * o, const float * gate, int64_t vs, void * out,
                               int64_t rows, int64_t rps, int64_t H, cudaStream_t st) {
    constexpr int N  = vec16<T>::N;
    constexpr int U  = 2;
    const int     sz = (int) sizeof(typename io<T>::t);
    const bool    vec = H % N == 0 && reinterpret_cast<uintptr_t>(r) % 16 == 0 &&
                     reinterpret_cast<uintptr_t>(o) % 16 == 0 && reinterpret_cast<uintptr_t>(out) % 16 == 0 &&
                     reinterpret_cast<uintptr_t>(gate) % 16 == 0 && (H * sz) % 16 == 0 && vs % 4 == 0;
    const unsigned gy = (unsigned) (rows < 65535 ? rows : 65535);
    if (vec) {
        const int64_t vpr = H / N;
        const dim3    grid((unsigned) ((vpr + 256 * U - 1) / (256 * U)), gy);
        gated_vec_kernel<T, U><<<grid, 256, 0, st>>>(r, o, gate, vs, out, rows, rps, H);
    } else {
        const dim3 grid((unsigned) ((H + 255) / 256 < 64 ? (H + 255) / 256 : 64), gy);
        gated_scalar_kernel<T><<<grid, 256, 0, st>>>(r, o, gate, vs, out, rows, rps, H);
    }
    return launch_status();
}

}  // namespace acb

using namespace acb;

extern "C" acb_status acb_swiglu(const void * gu, int gu_type, int64_t gu_stride, int64_t up_offset, void * out,
                                 int out_type, int64_t out_stride, int64_t rows, int64_t F, acb_stream_t stream) {
    if (!gu || !out || rows < 0 || F <= 0 || out_stride < F) {
        return ACB_ERR_INVALID_ARG;
    }
    if (rows == 0) {
        return ACB_OK;
    }
    cudaStream_t st = (cudaStream_t) stream;
#define ACB_SW(A, B)                                                                       \
    if (gu_type == A && out_type == B) {                                                   \
        return launch_swiglu<A, B>(gu, gu_stride, up_offset, out, out_stride, rows, F, st); \
    }
    ACB_SW(ACB_TYPE_F32, ACB_TYPE_F32)
    ACB_SW(ACB_TYPE_F32, ACB_TYPE_BF16)
    ACB_SW(ACB_TYPE_BF16, ACB_TYPE_BF16)
    ACB_SW(ACB_TYPE_BF16, ACB_TYPE_F32)
    ACB_SW(ACB_TYPE_F16, ACB_TYPE_F16)
#undef ACB_SW
    return ACB_ERR_UNSUPPORTED;
}

extern "C" acb_status acb_gated_residual(const void * r, const void * o, int io_type, const float * gate,
                                         int64_t vec_stride, void * out, int64_t samples, int64_t rows_per_sample,
                                         int H, acb_stream_t stream) {
    if (!r || !o || !gate || !out || samples < 0 || rows_per_sample < 0 || H <= 0 || vec_stride < 0) {
        return ACB_ERR_INVALID_ARG;
    }
    const int64_t rows = samples * rows_per_sample;
    if (rows == 0) {
        return ACB_OK;
    }
    cudaStream_t st = (cudaStream_t) stream;
    switch (io_type) {
        case ACB_TYPE_F32:
            return launch_gated<ACB_TYPE_F32>(r, o, gate, vec_stride, out, rows, rows_per_sample, H, st);
        case ACB_TYPE_BF16:
            return launch_gated<ACB_TYPE_BF16>(r, o, gate, vec_stride, out, rows, rows_per_sample, H, st);
        case ACB_TYPE_F16:
            return launch_gated<ACB_TYPE_F16>(r, o, gate, vec_stride, out, rows, rows_per_sample, H, st);
        default:
            return ACB_ERR_UNSUPPORTED;
    }
}
