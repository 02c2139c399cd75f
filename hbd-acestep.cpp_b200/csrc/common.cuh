// common.cuh -- shared device helpers for libacb (sm_100a only).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/acb.h"
#include "acb_exp.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#    error "libacb is built for sm_100a only"
#endif

namespace acb {

constexpr int kWarp = 32;

// Records the CUDA error of the last failed call (acb_last_cuda_error).
void set_last_cuda_error(cudaError_t e);

inline acb_status launch_status() {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        set_last_cuda_error(e);
        return ACB_ERR_CUDA;
    }
    return ACB_OK;
}

inline bool is_io_type(int t) {
    return t == ACB_TYPE_F32 || t == ACB_TYPE_BF16 || t == ACB_TYPE_F16;
}

inline int type_size(int t) {
    return t == ACB_TYPE_F32 ? 4 : 2;
}

// ---- scalar I/O conversions (round to nearest even on store) ----

template <int T> struct io;

template <> struct io<ACB_TYPE_F32> {
    using t                                       = float;
    static __device__ __forceinline__ float to_f(float v) { return v; }
    static __device__ __forceinline__ float from_f(float v) { return v; }
};

template <> struct io<ACB_TYPE_BF16> {
    using t = __nv_bfloat16;
    static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
    static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
};

template <> struct io<ACB_TYPE_F16> {
    using t = __half;
    static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
    static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
};

// 16-byte vector of an I/O type: N = 4 (f32) or 8 (bf16/f16) elements.
template <int T> struct vec16 {
    using e                  = typename io<T>::t;
    static constexpr int N   = 16 / sizeof(e);
    union {
        uint4 u;
        e     v[N];
    };
    __device__ __forceinline__ void load(const void * p) { u = *reinterpret_cast<const uint4 *>(p); }
    __device__ __forceinline__ void load_nc(const void * p) { u = __ldg(reinterpret_cast<const uint4 *>(p)); }
    __device__ __forceinline__ void load_stream(const void * p) {
        u = __ldcs(reinterpret_cast<const uint4 *>(p));
    }
    __device__ __forceinline__ void store(void * p) const { *reinterpret_cast<uint4 *>(p) = u; }
    __device__ __forceinline__ void store_stream(void * p) const { __stcs(reinterpret_cast<uint4 *>(p), u); }
    __device__ __forceinline__ float get(int i) const { return io<T>::to_f(v[i]); }
    __device__ __forceinline__ void set(int i, float f) { v[i] = io<T>::from_f(f); }
};

__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        v += __shfl_xor_sync(0xffffffffu, v, o);
    }
    return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        v += __shfl_xor_sync(0xffffffffu, v, o);
    }
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    }
    return v;
}

// ggml_rms_norm scale: sum of float squares accumulated in double, mean rounded to float,
// 1/sqrt in IEEE float (the division and sqrt are correctly rounded under -prec-div/-prec-sqrt).
// ggml_swiglu element: silu(g) * u with silu(g) = g / (1 + exp(-g)), IEEE division, each node
// rounded once, exp = acb_expf (every SwiGLU in the library uses this one definition, and the
// same exp as any host program that includes acb_exp.h).
__device__ __forceinline__ float silu_f(float g) {
    return __fdiv_rn(g, __fadd_rn(1.0f, acb_expf(-g)));
}

__device__ __forceinline__ float silu_times(float g, float u) {
    const float s = silu_f(g);
    return __fmul_rn(s, u);
}

// The VAE's snake activation x + sin(x * e^a)^2 * e^-b (src/vae.h:267-276, ggml_mul, ggml_sin,
// ggml_sqr, ggml_mul, ggml_add: each node rounded once); ea = e^a, ib = e^-b per channel. One
// definition for the standalone kernel and the GEMM epilogue that fuses it.
__device__ __forceinline__ float snake_f(float x, float ea, float ib) {
    const float ax = __fmul_rn(x, ea);
    const float s  = sinf(ax);
    return __fadd_rn(x, __fmul_rn(__fmul_rn(s, s), ib));
}

__device__ __forceinline__ float rms_scale(double sumsq, int n, float eps) {
    float mean = (float) (sumsq / (double) n);
    return 1.0f / sqrtf(__fadd_rn(mean, eps));
}

// rms_scale for a power-of-two count NN: the mean is sumsq * 2^-k, which equals sumsq / NN
// exactly in double (a power-of-two scaling of a sum of float squares stays normal), so the scale
// is bit-identical to rms_scale's without a double division (per-head norms run it in every lane).
template <int NN> __device__ __forceinline__ float rms_scale_pow2(double sumsq, float eps) {
    static_assert(NN > 0 && (NN & (NN - 1)) == 0, "power of two");
    const float mean = (float) (sumsq * (1.0 / (double) NN));
    return 1.0f / sqrtf(__fadd_rn(mean, eps));
}

__device__ __forceinline__ uint16_t ld_u16(const uint8_t * p) {
    return (uint16_t) (p[0] | (p[1] << 8));
}

__device__ __forceinline__ float f16_bits_to_f(uint16_t h) {
    return __half2float(__ushort_as_half(h));
}

inline int num_sms() {
    static int n = 0;
    if (n == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) {
            n = 148;
        }
    }
    return n;
}

}  // namespace acb
