// k_fsq.cu -- the small ops around the FSQ tokenizer / detokenizer stacks and the condition
// encoder's sequence packing, batched over every 5 Hz group at once (the reference runs one graph
// per group, src/fsq-tok.h:208-223, src/fsq-detok.h:193-205).
//
//   acb_fsq_project_out  codes -> fsq_decode_index -> project_out (K = 6) + bias
//                        (src/fsq-detok.h:18-29, 150-160)
//   acb_fsq_quantize     project_in output + bias -> tanh -> per-dimension level -> flat index
//                        (src/fsq-tok.h:42-60, 196-199)
//   acb_rows_repeat_add  out[g*P + p] = a[g] + b[p]: ggml_add(ggml_repeat(embedded, special), special)
//                        (src/fsq-detok.h:165-169)
//   acb_rows_prepend     out[g*(P+1)] = head, out[g*(P+1) + 1 + p] = src[g*P + p]: the CLS concat
//                        (src/fsq-tok.h:181-184, src/cond-enc.h:256-259)
//
// All four are HBM-bound row copies; one thread per output element (float4 where rows allow).
#include "common.cuh"

namespace acb {
namespace {

constexpr int kFsqDims           = 6;
__constant__ int c_fsq_levels[6] = { 8, 8, 8, 5, 5, 5 };  // FSQ_LEVELS, src/fsq-detok.h:15

// One output row g of project_out: the 6 decoded levels rounded to the weight type (ggml converts
// the activation to the weight's vec-dot type), each product exact or rounded once in f32, the six
// added in double and rounded once (ggml_vec_dot_{bf16,f16,f32} below one SIMD step), then the
// f32 bias add (ggml_add).
template <int WT>
__global__ void fsq_project_out_kernel(const int32_t * __restrict__ codes, int G, const void * __restrict__ w, int N,
                                       const float * __restrict__ bias, float * __restrict__ out, int64_t ldo,
                                       int * err) {
    const int nb = (N + 127) / 128;  // blocks per row
    const int g  = (int) (blockIdx.x / nb);
    const int n  = (int) (blockIdx.x % nb) * 128 + threadIdx.x;
    if (g >= G || n >= N) {
        return;
    }
    const int code = codes[g];
    if (code < 0) {
        if (n == 0 && err) {
            atomicOr(err, ACB_DEVERR_CODE_RANGE);
        }
        out[(int64_t) g * ldo + n] = 0.0f;
        return;
    }
    float x[kFsqDims];
    int   stride = 1;
#pragma unroll
    for (int d = 0; d < kFsqDims; d++) {
        const int   L      = c_fsq_levels[d];
        const int   lvl    = (code / stride) % L;
        const float half_L = __fdiv_rn((float) (L - 1), 2.0f);
        x[d]               = __fadd_rn(__fdiv_rn((float) lvl, half_L), -1.0f);
        stride *= L;
    }
    double acc = 0.0;
#pragma unroll
    for (int d = 0; d < kFsqDims; d++) {
        float wv, xv;
        if constexpr (WT == ACB_TYPE_BF16) {
            wv = __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(w)[(int64_t) n * kFsqDims + d]);
            xv = __bfloat162float(__float2bfloat16_rn(x[d]));
        } else if constexpr (WT == ACB_TYPE_F16) {
            wv = __half2float(reinterpret_cast<const __half *>(w)[(int64_t) n * kFsqDims + d]);
            xv = __half2float(__float2half_rn(x[d]));
        } else {
            wv = reinterpret_cast<const float *>(w)[(int64_t) n * kFsqDims + d];
            xv = x[d];
        }
        acc = __dadd_rn(acc, (double) __fmul_rn(wv, xv));
    }
    float v = __double2float_rn(acc);
    if (bias) {
        v = __fadd_rn(v, bias[n]);
    }
    out[(int64_t) g * ldo + n] = v;
}

__global__ void fsq_quantize_kernel(const float * __restrict__ raw, int64_t ld, const float * __restrict__ bias, int G,
                                    int32_t * __restrict__ codes) {
    const int g = blockIdx.x * blockDim.x + threadIdx.x;
    if (g >= G) {
        return;
    }
    int index = 0, mult = 1;
#pragma unroll
    for (int d = 0; d < kFsqDims; d++) {
        const int L = c_fsq_levels[d];
        float     v = raw[(int64_t) g * ld + d];
        if (bias) {
            v = __fadd_rn(v, bias[d]);
        }
        const float t = tanhf(v);
        // floor((L-1) * (t+1) / 2 + 0.5), each operation rounded on its own as in the C source
        const float s    = __fadd_rn(__fdiv_rn(__fmul_rn((float) (L - 1), __fadd_rn(t, 1.0f)), 2.0f), 0.5f);
        int         code = (int) floorf(s);
        code             = code < 0 ? 0 : (code >= L ? L - 1 : code);
        index += code * mult;
        mult *= L;
    }
    codes[g] = index;
}

__global__ void rows_repeat_add_kernel(const float * __restrict__ a, int64_t lda, const float * __restrict__ b,
                                       int64_t ldb, int G, int P, int H4, float * __restrict__ out, int64_t ldo) {
    const int64_t row = blockIdx.y;  // g * P + p
    const int     c   = blockIdx.x * blockDim.x + threadIdx.x;
    if (row >= (int64_t) G * P || c >= H4) {
        return;
    }
    const int64_t g  = row / P, p = row % P;
    const float4  av = reinterpret_cast<const float4 *>(a + g * lda)[c];
    const float4  bv = reinterpret_cast<const float4 *>(b + p * ldb)[c];
    reinterpret_cast<float4 *>(out + row * ldo)[c] =
        make_float4(__fadd_rn(av.x, bv.x), __fadd_rn(av.y, bv.y), __fadd_rn(av.z, bv.z), __fadd_rn(av.w, bv.w));
}

__global__ void rows_prepend_kernel(const float * __restrict__ head, const float * __restrict__ src, int64_t lds,
                                    int G, int P, int H4, float * __restrict__ out, int64_t ldo) {
    const int64_t row = blockIdx.y;  // g * (P + 1) + j
    const int     c   = blockIdx.x * blockDim.x + threadIdx.x;
    if (row >= (int64_t) G * (P + 1) || c >= H4) {
        return;
    }
    const int64_t g = row / (P + 1), j = row % (P + 1);
    const float * s = j == 0 ? head : src + (g * P + j - 1) * lds;
    reinterpret_cast<float4 *>(out + row * ldo)[c] = reinterpret_cast<const float4 *>(s)[c];
}

bool aligned16(const void * p) {
    return (reinterpret_cast<uintptr_t>(p) & 15) == 0;
}

}  // namespace
}  // namespace acb

using namespace acb;

extern "C" acb_status acb_fsq_project_out(const int32_t * codes, int G, const void * w, int w_type, int N,
                                          const float * bias, float * out, int64_t ldo, int * err_flag,
                                          acb_stream_t stream) {
    if (!codes || !w || !out || G < 0 || N <= 0 || ldo < N) {
        return ACB_ERR_INVALID_ARG;
    }
    if (G == 0) {
        return ACB_OK;
    }
    if ((int64_t) G * ((N + 127) / 128) > 2147483647LL) {
        return ACB_ERR_UNSUPPORTED;
    }
    const dim3   grid((unsigned) (G * ((N + 127) / 128)));
    cudaStream_t s = (cudaStream_t) stream;
    switch (w_type) {
        case ACB_TYPE_BF16:
            fsq_project_out_kernel<ACB_TYPE_BF16><<<grid, 128, 0, s>>>(codes, G, w, N, bias, out, ldo, err_flag);
            break;
        case ACB_TYPE_F16:
            fsq_project_out_kernel<ACB_TYPE_F16><<<grid, 128, 0, s>>>(codes, G, w, N, bias, out, ldo, err_flag);
            break;
        case ACB_TYPE_F32:
            fsq_project_out_kernel<ACB_TYPE_F32><<<grid, 128, 0, s>>>(codes, G, w, N, bias, out, ldo, err_flag);
            break;
        default:
            return ACB_ERR_UNSUPPORTED;
    }
    return launch_status();
}

extern "C" acb_status acb_fsq_quantize(const float * raw, int64_t ld, const float * bias, int G, int32_t * codes,
                                       acb_stream_t stream) {
    if (!raw || !codes || G < 0 || ld < 6) {
        return ACB_ERR_INVALID_ARG;
    }
    if (G == 0) {
        return ACB_OK;
    }
    fsq_quantize_kernel<<<(G + 127) / 128, 128, 0, (cudaStream_t) stream>>>(raw, ld, bias, G, codes);
    return launch_status();
}

extern "C" acb_status acb_rows_repeat_add(const float * a, int64_t lda, const float * b, int64_t ldb, int G, int P,
                                          int H, float * out, int64_t ldo, acb_stream_t stream) {
    if (!a || !b || !out || G < 0 || P <= 0 || H <= 0) {
        return ACB_ERR_INVALID_ARG;
    }
    if (H % 4 || lda % 4 || ldb % 4 || ldo % 4 || !aligned16(a) || !aligned16(b) || !aligned16(out) || P > 65535) {
        return ACB_ERR_UNSUPPORTED;
    }
    if (G == 0) {
        return ACB_OK;
    }
    const int64_t rows = (int64_t) G * P;
    if (rows > 65535) {
        // grid.y is limited to 65535: split the rows into chunks of whole groups
        const int gchunk = 65535 / P;
        for (int g0 = 0; g0 < G; g0 += gchunk) {
            const int gn = G - g0 < gchunk ? G - g0 : gchunk;
            const acb_status st = acb_rows_repeat_add(a + (int64_t) g0 * lda, lda, b, ldb, gn, P, H,
                                                      out + (int64_t) g0 * P * ldo, ldo, stream);
            if (st != ACB_OK) {
                return st;
            }
        }
        return ACB_OK;
    }
    const int  H4 = H / 4;
    const dim3 grid((unsigned) ((H4 + 127) / 128), (unsigned) rows);
    rows_repeat_add_kernel<<<grid, 128, 0, (cudaStream_t) stream>>>(a, lda, b, ldb, G, P, H4, out, ldo);
    return launch_status();
}

extern "C" acb_status acb_rows_prepend(const float * head, const float * src, int64_t lds, int G, int P, int H,
                                       float * out, int64_t ldo, acb_stream_t stream) {
    if (!head || !out || G < 0 || P < 0 || H <= 0 || (P > 0 && !src)) {
        return ACB_ERR_INVALID_ARG;
    }
    if (H % 4 || lds % 4 || ldo % 4 || !aligned16(head) || (src && !aligned16(src)) || !aligned16(out) ||
        P >= 65535) {
        return ACB_ERR_UNSUPPORTED;
    }
    if (G == 0) {
        return ACB_OK;
    }
    const int64_t rows = (int64_t) G * (P + 1);
    if (rows > 65535) {
        const int gchunk = 65535 / (P + 1);
        for (int g0 = 0; g0 < G; g0 += gchunk) {
            const int gn = G - g0 < gchunk ? G - g0 : gchunk;
            const acb_status st = acb_rows_prepend(head, src ? src + (int64_t) g0 * P * lds : nullptr, lds, gn, P,
                                                   H, out + (int64_t) g0 * (P + 1) * ldo, ldo, stream);
            if (st != ACB_OK) {
                return st;
            }
        }
        return ACB_OK;
    }
    const int  H4 = H / 4;
    const dim3 grid((unsigned) ((H4 + 127) / 128), (unsigned) rows);
    rows_prepend_kernel<<<grid, 128, 0, (cudaStream_t) stream>>>(head, src, lds, G, P, H4, out, ldo);
    return launch_status();
}
