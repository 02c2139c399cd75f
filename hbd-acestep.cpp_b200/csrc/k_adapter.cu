// k_adapter.cu -- LoRA merge arithmetic on the device (src/adapter-merge.h:357-472, 482-672):
//
//   acb_lora_delta_add  w[n][k] += bf16( fl32( scaling * fl32( sum_r B[n][r] * A[r][k] ) ) )
//                       the delta of PEFT merge_and_unload / the reference's merge graph: A and B
//                       arrive already rounded to bf16 (PEFT casts them), so every product is
//                       exact in f32; the products are added in double and rounded once (the
//                       library's canonical rule, independent of how the sum is split), then
//                       scaled, rounded to bf16 (diff.to(base.dtype)) and added to the
//                       dequantised base in f32.
//   acb_requant         f32 rows back to the base tensor's GGUF type: Q8_0 / Q4_K / Q6_K through
//                       acb_quantize, BF16 / F16 rounded to nearest even, F32 copied.
//
//   acb_lokr_delta_add  LyCORIS LoKr (src/adapter-merge.h:674-958, merge :357-472): the delta is the
//                       Kronecker product kron(w1s, W2), element (i*c + k, j*d + l) =
//                       fl32(w1s[i][j] * W2[k][l]) (w1s = w1 * alpha / rank, both f32 from the
//                       caller), rounded to bf16; then either w += bf16(delta) * user_scale, or
//                       with a DoRA magnitude vector (LyCORIS apply_weight_decompose) per output row
//                       m = w + bf16(delta), w = m * s with s = ds / (|m| + eps) (eps = bf16
//                       epsilon, 2^-7) and, for user_scale != 1, s = s * user_scale + (1 - user_scale);
//                       |m| is the square root of the row's f32 squares summed in double.
//
// One thread per output element; the CTA's 256 threads share a row n (B's r values in shared
// memory) and read A's rows with coalesced 32-bit loads. The DoRA form takes a CTA per row.
#include "common.cuh"

namespace acb {
namespace {

constexpr int kMaxLoraRank = 1024;

__global__ void __launch_bounds__(256) lora_delta_add_kernel(float * __restrict__ w, int64_t K,
                                                             const float * __restrict__ A,
                                                             const float * __restrict__ B, int rank, float scaling) {
    __shared__ float bs[kMaxLoraRank];
    const int64_t n = blockIdx.y;
    for (int j = threadIdx.x; j < rank; j += blockDim.x) {
        bs[j] = B[n * rank + j];
    }
    __syncthreads();
    const int64_t k = (int64_t) blockIdx.x * blockDim.x + threadIdx.x;
    if (k >= K) {
        return;
    }
    double acc = 0.0;
    for (int j = 0; j < rank; j++) {
        acc = __dadd_rn(acc, (double) __fmul_rn(bs[j], A[(int64_t) j * K + k]));
    }
    const float d  = __fmul_rn(__double2float_rn(acc), scaling);
    const float db = __bfloat162float(__float2bfloat16_rn(d));
    float *     p  = w + n * K + k;
    *p             = __fadd_rn(*p, db);
}

__device__ __forceinline__ float lokr_delta_bf16(const float * __restrict__ w1s, const float * __restrict__ w2, int64_t n,
                                                 int64_t k, int b, int c, int d) {
    const int64_t i = n / c, kk = n - i * c, j = k / d, l = k - j * d;
    const float   v = __fmul_rn(w1s[i * b + j], w2[kk * d + l]);
    return __bfloat162float(__float2bfloat16_rn(v));
}

__global__ void __launch_bounds__(256) lokr_delta_add_kernel(float * __restrict__ w, int64_t row0, int64_t K,
                                                             const float * __restrict__ w1s,
                                                             const float * __restrict__ w2, int b, int c, int d,
                                                             float user_scale) {
    const int64_t n = row0 + blockIdx.y;
    const int64_t k = (int64_t) blockIdx.x * blockDim.x + threadIdx.x;
    if (k >= K) {
        return;
    }
    float * p = w + n * K + k;
    *p        = __fadd_rn(*p, __fmul_rn(lokr_delta_bf16(w1s, w2, n, k, b, c, d), user_scale));
}

// DoRA: a CTA per output row (grid-stride over the rows)
__global__ void __launch_bounds__(256) lokr_dora_kernel(float * __restrict__ w, int64_t N, int64_t K,
                                                        const float * __restrict__ w1s,
                                                        const float * __restrict__ w2, int b, int c, int d,
                                                        float user_scale, const float * __restrict__ ds) {
    __shared__ double red[8];
    __shared__ float  scale_s;
    const float       eps = 0.0078125f;  // torch.finfo(torch.bfloat16).eps
    for (int64_t n = blockIdx.x; n < N; n += gridDim.x) {
        float * row = w + n * K;
        double  ss  = 0.0;
        for (int64_t k = threadIdx.x; k < K; k += blockDim.x) {
            const float m = __fadd_rn(row[k], lokr_delta_bf16(w1s, w2, n, k, b, c, d));
            row[k]        = m;
            ss += (double) __fmul_rn(m, m);
        }
        ss = warp_sum(ss);
        if ((threadIdx.x & 31) == 0) {
            red[threadIdx.x >> 5] = ss;
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            double t = 0.0;
            for (int i = 0; i < (int) (blockDim.x >> 5); i++) {
                t += red[i];
            }
            const float rn = __fadd_rn(sqrtf((float) t), eps);
            float       sc = __fdiv_rn(ds[n], rn);
            if (user_scale != 1.0f) {
                sc = __fadd_rn(__fmul_rn(sc, user_scale), __fsub_rn(1.0f, user_scale));
            }
            scale_s = sc;
        }
        __syncthreads();
        const float sc = scale_s;
        for (int64_t k = threadIdx.x; k < K; k += blockDim.x) {
            row[k] = __fmul_rn(row[k], sc);
        }
        __syncthreads();  // red / scale_s are rewritten by the next row
    }
}

template <int TO>
__global__ void to16_kernel(const float * __restrict__ x, int64_t n, void * __restrict__ y) {
    const int64_t i = (int64_t) blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) {
        reinterpret_cast<typename io<TO>::t *>(y)[i] = io<TO>::from_f(x[i]);
    }
}

}  // namespace
}  // namespace acb

using namespace acb;

extern "C" acb_status acb_lora_delta_add(float * w, int64_t N, int64_t K, const float * A, const float * B, int rank,
                                         float scaling, acb_stream_t stream) {
    if (!w || !A || !B || N <= 0 || K <= 0 || rank <= 0) {
        return ACB_ERR_INVALID_ARG;
    }
    if (rank > kMaxLoraRank || N > 65535LL * 65535LL) {
        return ACB_ERR_UNSUPPORTED;
    }
    // grid.y is limited to 65535 rows per launch
    for (int64_t n0 = 0; n0 < N; n0 += 65535) {
        const int64_t nn = N - n0 < 65535 ? N - n0 : 65535;
        const dim3    grid((unsigned) ((K + 255) / 256), (unsigned) nn);
        lora_delta_add_kernel<<<grid, 256, 0, (cudaStream_t) stream>>>(w + n0 * K, K, A, B + n0 * rank, rank,
                                                                       scaling);
        const acb_status s = launch_status();
        if (s != ACB_OK) {
            return s;
        }
    }
    return ACB_OK;
}

extern "C" acb_status acb_lokr_delta_add(float * w, int64_t N, int64_t K, const float * w1s, int a, int b,
                                         const float * w2, int c, int d, float user_scale, const float * dora_scale,
                                         acb_stream_t stream) {
    if (!w || !w1s || !w2 || N <= 0 || K <= 0 || a <= 0 || b <= 0 || c <= 0 || d <= 0 || (int64_t) a * c != N ||
        (int64_t) b * d != K) {
        return ACB_ERR_INVALID_ARG;
    }
    cudaStream_t s = (cudaStream_t) stream;
    if (dora_scale) {
        const int64_t nb = N < 148 * 8 ? N : 148 * 8;
        lokr_dora_kernel<<<(unsigned) nb, 256, 0, s>>>(w, N, K, w1s, w2, b, c, d, user_scale, dora_scale);
        return launch_status();
    }
    for (int64_t n0 = 0; n0 < N; n0 += 65535) {  // grid.y is limited to 65535 rows per launch
        const int64_t nn = N - n0 < 65535 ? N - n0 : 65535;
        lokr_delta_add_kernel<<<dim3((unsigned) ((K + 255) / 256), (unsigned) nn), 256, 0, s>>>(w, n0, K, w1s, w2, b,
                                                                                                c, d, user_scale);
        const acb_status st = launch_status();
        if (st != ACB_OK) {
            return st;
        }
    }
    return ACB_OK;
}

extern "C" acb_status acb_requant(const float * x, int64_t rows, int64_t K, int type, void * dst,
                                  acb_stream_t stream) {
    if (!x || !dst || rows <= 0 || K <= 0) {
        return ACB_ERR_INVALID_ARG;
    }
    const int64_t n = rows * K;
    cudaStream_t  s = (cudaStream_t) stream;
    switch (type) {
        case ACB_TYPE_Q8_0:
        case ACB_TYPE_Q4_K:
        case ACB_TYPE_Q6_K:
            return acb_quantize(x, rows, K, type, dst, stream);
        case ACB_TYPE_BF16:
            to16_kernel<ACB_TYPE_BF16><<<(unsigned) ((n + 255) / 256), 256, 0, s>>>(x, n, dst);
            return launch_status();
        case ACB_TYPE_F16:
            to16_kernel<ACB_TYPE_F16><<<(unsigned) ((n + 255) / 256), 256, 0, s>>>(x, n, dst);
            return launch_status();
        case ACB_TYPE_F32:
            return cudaMemcpyAsync(dst, x, (size_t) n * 4, cudaMemcpyDeviceToDevice, s) == cudaSuccess
                       ? ACB_OK
                       : ACB_ERR_CUDA;
        default:
            return ACB_ERR_UNSUPPORTED;
    }
}
