// k_vae.cu -- the AutoencoderOobleck decoder's non-GEMM ops (src/vae.h:267-369). Its convolutions
// run on the tensor-core GEMM (acb_conv1d_tc, an implicit GEMM: TMA reads each tap's rows of the
// f16 activation directly, with zero fill outside [0, T)), whose epilogue also applies the next
// snake; what remains here:
//
//   acb_vae_snake_f16     y[t][c] = f16(snake(x[t][c])): the snake activation x + sin(x*e^a)^2 *
//                         e^-b (vae_snake, :267-276, five separately rounded f32 ops), rounded to
//                         the f16 operand type ggml_conv_1d gives the activation (its im2col takes
//                         the weights' type). Without e^a a plain cast (the first conv's input).
//   acb_vae_out_conv      the last conv (C -> 2 channels, k = 7, no bias) with its snake, as a
//                         direct convolution: 2 outputs per sample are too few for a GEMM tile.
//                         Output planar [2][T] (ggml's [T, 2] with T contiguous).
#include "common.cuh"

namespace acb {
namespace {

// one thread per 8 consecutive channels of one row; C a multiple of 8
__global__ void snake_f16_kernel(const float * __restrict__ x, int64_t xs, int64_t T, int C,
                                 const float * __restrict__ ea, const float * __restrict__ ib,
                                 __half * __restrict__ y, int64_t ldy) {
    const int     groups = C / 8;
    const int64_t idx    = (int64_t) blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= T * groups) {
        return;
    }
    const int64_t t  = idx / groups;
    const int     c0 = (int) (idx - t * groups) * 8;
    const float4  a  = *reinterpret_cast<const float4 *>(x + t * xs + c0);
    const float4  b  = *reinterpret_cast<const float4 *>(x + t * xs + c0 + 4);
    const float   v[8] = { a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w };
    union {
        uint4  u;
        __half h[8];
    } o;
#pragma unroll
    for (int e = 0; e < 8; e++) {
        o.h[e] = __float2half_rn(ea ? snake_f(v[e], __ldg(ea + c0 + e), __ldg(ib + c0 + e)) : v[e]);
    }
    *reinterpret_cast<uint4 *>(y + t * ldy + c0) = o.u;
}

// Final conv, C channels -> 2, k = 7, pad 3, with the snake. A CTA of 8 warps covers 128 samples:
// the snake'd inputs of samples [t0 - 3, t0 + 131), rounded to f16 (the conv's operand type) and
// kept as f32, are staged in shared memory once; a warp computes one sample at a time with its
// lanes across channel quads (one 16-byte shared read per tap, no bank conflicts), f32 products
// and sums, reduced over the lanes. With C <= 128 every lane holds its quads' 14 weight vectors
// in registers (REGW); wider layers read them from shared memory.
constexpr int kOutTile = 128, kOutThreads = 256;

template <bool REGW>
__global__ void __launch_bounds__(kOutThreads) out_conv_kernel(const float * __restrict__ x, int64_t T, int C,
                                                               const float * __restrict__ ea,
                                                               const float * __restrict__ ib,
                                                               const __half * __restrict__ w,  // [2][7][C]
                                                               float * __restrict__ y) {
    extern __shared__ __align__(16) float oc_smem[];  // [kOutTile + 6][C] inputs, [14][C] weights
    float *          xs  = oc_smem;
    float *          wsm = oc_smem + (kOutTile + 6) * C;
    __shared__ float res[2][kOutTile];
    const int64_t    t0 = (int64_t) blockIdx.x * kOutTile;
    const int        cq = C / 4;
    for (int i = threadIdx.x; i < (kOutTile + 6) * cq; i += blockDim.x) {
        const int     r  = i / cq, c = (i - r * cq) * 4;
        const int64_t ts = t0 - 3 + r;
        float4        o  = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (ts >= 0 && ts < T) {
            const float4 v = *reinterpret_cast<const float4 *>(x + ts * C + c);
            o.x            = __half2float(__float2half_rn(snake_f(v.x, __ldg(ea + c), __ldg(ib + c))));
            o.y            = __half2float(__float2half_rn(snake_f(v.y, __ldg(ea + c + 1), __ldg(ib + c + 1))));
            o.z            = __half2float(__float2half_rn(snake_f(v.z, __ldg(ea + c + 2), __ldg(ib + c + 2))));
            o.w            = __half2float(__float2half_rn(snake_f(v.w, __ldg(ea + c + 3), __ldg(ib + c + 3))));
        }
        *reinterpret_cast<float4 *>(xs + r * C + c) = o;
    }
    for (int i = threadIdx.x; i < 14 * C; i += blockDim.x) {
        wsm[i] = __half2float(w[i]);
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float4    wr[14];  // REGW: this lane's quad (lane) of the 2 x 7 weight rows
    if constexpr (REGW) {
#pragma unroll
        for (int j = 0; j < 14; j++) {
            wr[j] = lane < cq ? *reinterpret_cast<const float4 *>(wsm + j * C + 4 * lane) : make_float4(0, 0, 0, 0);
        }
    }
    for (int s = warp; s < kOutTile; s += kOutThreads / 32) {
        float a0 = 0.0f, a1 = 0.0f;
        if constexpr (REGW) {
            if (lane < cq) {
#pragma unroll
                for (int k = 0; k < 7; k++) {
                    const float4 xv = *reinterpret_cast<const float4 *>(xs + (s + k) * C + 4 * lane);
                    a0 = fmaf(xv.x, wr[k].x, a0);
                    a0 = fmaf(xv.y, wr[k].y, a0);
                    a0 = fmaf(xv.z, wr[k].z, a0);
                    a0 = fmaf(xv.w, wr[k].w, a0);
                    a1 = fmaf(xv.x, wr[7 + k].x, a1);
                    a1 = fmaf(xv.y, wr[7 + k].y, a1);
                    a1 = fmaf(xv.z, wr[7 + k].z, a1);
                    a1 = fmaf(xv.w, wr[7 + k].w, a1);
                }
            }
        } else {
            for (int k = 0; k < 7; k++) {
                for (int q = lane; q < cq; q += 32) {
                    const float4 xv = *reinterpret_cast<const float4 *>(xs + (s + k) * C + 4 * q);
                    const float4 w0 = *reinterpret_cast<const float4 *>(wsm + k * C + 4 * q);
                    const float4 w1 = *reinterpret_cast<const float4 *>(wsm + (7 + k) * C + 4 * q);
                    a0              = fmaf(xv.x, w0.x, fmaf(xv.y, w0.y, fmaf(xv.z, w0.z, fmaf(xv.w, w0.w, a0))));
                    a1              = fmaf(xv.x, w1.x, fmaf(xv.y, w1.y, fmaf(xv.z, w1.z, fmaf(xv.w, w1.w, a1))));
                }
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            a0 += __shfl_xor_sync(0xffffffffu, a0, o);
            a1 += __shfl_xor_sync(0xffffffffu, a1, o);
        }
        if (lane == 0) {
            res[0][s] = a0;
            res[1][s] = a1;
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < 2 * kOutTile; i += blockDim.x) {
        const int     ch = i / kOutTile, s = i - ch * kOutTile;
        const int64_t t  = t0 + s;
        if (t < T) {
            y[ch * T + t] = res[ch][s];
        }
    }
}

}  // namespace
}  // namespace acb

using namespace acb;

extern "C" acb_status acb_vae_snake_f16(const float * x, int64_t x_stride, int64_t T, int C, const float * exp_alpha,
                                        const float * inv_beta, void * y, int64_t ldy, acb_stream_t stream) {
    if (!x || !y || T <= 0 || C <= 0 || x_stride < C || ldy < C || (exp_alpha && !inv_beta)) {
        return ACB_ERR_INVALID_ARG;
    }
    if (C % 8 || x_stride % 4 || ldy % 8 || (reinterpret_cast<uintptr_t>(x) & 15) ||
        (reinterpret_cast<uintptr_t>(y) & 15)) {
        return ACB_ERR_UNSUPPORTED;
    }
    const int64_t n = T * (C / 8);
    snake_f16_kernel<<<(unsigned) ((n + 255) / 256), 256, 0, (cudaStream_t) stream>>>(
        x, x_stride, T, C, exp_alpha, inv_beta, reinterpret_cast<__half *>(y), ldy);
    return launch_status();
}

extern "C" acb_status acb_vae_out_conv(const float * x, int64_t T, int C, const float * exp_alpha,
                                       const float * inv_beta, const void * w, float * y, acb_stream_t stream) {
    if (!x || !w || !y || !exp_alpha || !inv_beta || T <= 0 || C <= 0) {
        return ACB_ERR_INVALID_ARG;
    }
    const size_t smem = (size_t) (kOutTile + 6 + 14) * C * 4;
    if (C % 4 || smem > 200 * 1024 || (reinterpret_cast<uintptr_t>(x) & 15)) {
        return ACB_ERR_UNSUPPORTED;
    }
    const bool regw = C <= 128;
    void (*kern)(const float *, int64_t, int, const float *, const float *, const __half *, float *) =
        regw ? out_conv_kernel<true> : out_conv_kernel<false>;
    if (smem > 48 * 1024) {
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);
    }
    kern<<<(unsigned) ((T + kOutTile - 1) / kOutTile), kOutThreads, smem, (cudaStream_t) stream>>>(
        x, T, C, exp_alpha, inv_beta, reinterpret_cast<const __half *>(w), y);
    return launch_status();
}
