// k_attn_decode.cu -- the attention part of one batched decode step (qw3lm_forward_batch,
// src/qwen3-lm.h:633-733): fused QKV post-processing into the f16 KV cache, split-KV attention
// over the cache, and the greedy argmax that feeds the next step's embedding gather.
//
// Attention reproduces ggml-CPU's qwen3_attn_f32 on an f16 cache (src/qwen3-enc.h:101-112):
//   s_j = (f16(q) . k_j) * scale    f32, in one fixed order: eight sequential sums of 16
//                                   dimensions, added as ((s0+s1)+(s2+s3))+((s4+s5)+(s6+s7))
//   p_j = f16( exp(s_j - max) * (float)(1/sum) )         sum of exp in double, exp = acb_expf
//   o   = (float) sum_j p_j v_j                          double accumulation of exact products
// The score order is the same in every kernel that scores keys (and in the oracle); products of
// two f16 values are exact in float and their double sum is exact unless the terms span ~24
// binades, so every split count and lane order gives the same P.V floats. The normalised probabilities are rounded before the PV
// product, so the step runs in two passes over split chunks of the cache: pass 1 writes scores
// and per-split maxima, pass 2 normalises and forms per-split partial outputs (double), and
// the last split CTA of each head adds the partials and rounds once.
#include "common.cuh"
#include "ptx.cuh"

namespace acb {

struct KvLayout {
    uint16_t * k;  // f16 cache [n_sets][Nkv][max_seq][D]
    uint16_t * v;
    int        max_seq;
    int        set0;
    int        set_per_tok;  // token i uses set set0 + i*set_per_tok
};

__device__ __forceinline__ int64_t kv_index(const KvLayout & kv, int Nkv, int D, int set, int h, int p) {
    return (((int64_t) set * Nkv + h) * kv.max_seq + p) * D;
}

template <int PDL>
__device__ __forceinline__ void dep_wait() {
    if (PDL) {
        ptx::grid_dep_wait();
    }
}

// ---- fused QKV post: q -> norm+rope -> q_out (f32); k -> norm+rope -> cache; v -> cache -------
// one warp per (token, head of Nh + 2 Nkv); D = 128 (E = 2 elements per lane per half)
template <int E, int PDL>
__global__ void __launch_bounds__(256) qkv_post_kernel(const float * __restrict__ qkv, int64_t qkv_stride,
                                                       int64_t n_tok, int Nh, int Nkv,
                                                       const float * __restrict__ q_norm,
                                                       const float * __restrict__ k_norm, float eps,
                                                       const int32_t * __restrict__ pos,
                                                       const float * __restrict__ rope, int max_pos,
                                                       float * __restrict__ q_out, int64_t q_stride, KvLayout kv,
                                                       int * __restrict__ err) {
    constexpr int D    = 64 * E;
    constexpr int HALF = D / 2;
    dep_wait<PDL>();
    ptx::grid_dep_launch();
    const int     lane  = threadIdx.x & 31;
    const int     nh    = Nh + 2 * Nkv;
    const int64_t item  = (int64_t) blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (item >= n_tok * nh) {
        return;
    }
    const int64_t t = item / nh;
    const int     h = (int) (item - t * nh);
    const int     p = __ldg(pos + t);
    if (p < 0 || p >= max_pos || p >= kv.max_seq) {
        if (lane == 0 && err) {
            atomicOr(err, ACB_DEVERR_POS_RANGE);
        }
        return;
    }
    const float * s = qkv + t * qkv_stride + (int64_t) h * D + lane * E;
    float         a[E], b[E];
#pragma unroll
    for (int e = 0; e < E; e++) {
        a[e] = s[e];
        b[e] = s[HALF + e];
    }
    const int     kind = h < Nh ? 0 : (h < Nh + Nkv ? 1 : 2);
    const float * w    = kind == 0 ? q_norm : k_norm;
    if (kind < 2) {
        if (w) {
            double ss = 0.0;
#pragma unroll
            for (int e = 0; e < E; e++) {
                ss += (double) __fmul_rn(a[e], a[e]);
                ss += (double) __fmul_rn(b[e], b[e]);
            }
            ss             = warp_sum(ss);
            const float sc = rms_scale_pow2<D>(ss, eps);
#pragma unroll
            for (int e = 0; e < E; e++) {
                a[e] = __fmul_rn(__fmul_rn(a[e], sc), __ldg(w + lane * E + e));
                b[e] = __fmul_rn(__fmul_rn(b[e], sc), __ldg(w + HALF + lane * E + e));
            }
        }
        const float * c = rope + (int64_t) p * D + 2 * lane * E;
#pragma unroll
        for (int e = 0; e < E; e++) {
            const float cs = __ldg(c + 2 * e), sn = __ldg(c + 2 * e + 1);
            const float x0 = a[e], x1 = b[e];
            a[e]           = __fsub_rn(__fmul_rn(x0, cs), __fmul_rn(x1, sn));
            b[e]           = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, cs));
        }
    }
    if (kind == 0) {
        float * d = q_out + t * q_stride + (int64_t) h * D + lane * E;
#pragma unroll
        for (int e = 0; e < E; e++) {
            d[e]        = a[e];
            d[HALF + e] = b[e];
        }
    } else {
        const int  set = kv.set0 + (int) t * kv.set_per_tok;
        const int  hk  = kind == 1 ? h - Nh : h - Nh - Nkv;
        uint16_t * d   = (kind == 1 ? kv.k : kv.v) + kv_index(kv, Nkv, D, set, hk, p) + lane * E;
#pragma unroll
        for (int e = 0; e < E; e++) {
            d[e]        = __half_as_ushort(__float2half_rn(a[e]));
            d[HALF + e] = __half_as_ushort(__float2half_rn(b[e]));
        }
    }
}

// ---- pass 1: scores of one (token, kv head, split) for the G q heads of the group ---------------
// block = 128 threads (4 warps); lane owns 4 of the 128 head elements; one key per warp step.
template <int G, int PDL>
__global__ void __launch_bounds__(128) attn_scores_kernel(const float * __restrict__ q, int64_t q_stride, int Nh,
                                                          int Nkv, const int32_t * __restrict__ pos, KvLayout kv,
                                                          float scale, int n_split, float * __restrict__ scores,
                                                          int64_t s_stride, float * __restrict__ smax) {
    constexpr int D = 128;
    dep_wait<PDL>();
    ptx::grid_dep_launch();
    const int   split = blockIdx.x, hk = blockIdx.y, t = blockIdx.z;
    const int   lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int   kv_len = __ldg(pos + t) + 1;
    if (kv_len <= 0 || kv_len > kv.max_seq) {
        return;  // position out of range: acb_qkv_post has already flagged it
    }
    const int   chunk  = (kv_len + n_split - 1) / n_split;
    const int   j0     = split * chunk;
    const int   j1     = min(kv_len, j0 + chunk);
    const int   set    = kv.set0 + t * kv.set_per_tok;
    __shared__ float wmax[4][G];
    // 8 lanes per key: lane owns dims [16*sub, 16*sub+16) of key slot ks; q of the group's heads,
    // rounded to f16 (the vec-dot type of the f16 cache)
    const int sub = lane & 7, ks = lane >> 3;
    float     qv[G][16];
#pragma unroll
    for (int g = 0; g < G; g++) {
        const float4 * qp = reinterpret_cast<const float4 *>(q + (int64_t) t * q_stride + (int64_t) (hk * G + g) * D +
                                                             16 * sub);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const float4 v   = qp[i];
            qv[g][4 * i]     = __half2float(__float2half_rn(v.x));
            qv[g][4 * i + 1] = __half2float(__float2half_rn(v.y));
            qv[g][4 * i + 2] = __half2float(__float2half_rn(v.z));
            qv[g][4 * i + 3] = __half2float(__float2half_rn(v.w));
        }
    }
    float mx[G];
#pragma unroll
    for (int g = 0; g < G; g++) {
        mx[g] = -INFINITY;
    }
    const uint16_t * kb = kv.k + kv_index(kv, Nkv, D, set, hk, 0);
    constexpr int    U  = 2;  // key groups in flight per lane
    for (int jb = j0 + warp * 4; jb < j1; jb += 16 * U) {
        uint4 raw[U][2];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int j = jb + 16 * u + ks;
            if (j < j1) {
                const uint4 * src = reinterpret_cast<const uint4 *>(kb + (int64_t) j * D + 16 * sub);
                raw[u][0]         = src[0];
                raw[u][1]         = src[1];
            }
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int j = jb + 16 * u + ks;
            float     kf[16];
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const __half2 * hp = reinterpret_cast<const __half2 *>(&raw[u][h]);
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const float2 f      = __half22float2(hp[e]);
                    kf[8 * h + 2 * e]     = f.x;
                    kf[8 * h + 2 * e + 1] = f.y;
                }
            }
#pragma unroll
            for (int g = 0; g < G; g++) {
                float acc = 0.0f;
#pragma unroll
                for (int e = 0; e < 16; e++) {
                    acc = __fadd_rn(acc, __fmul_rn(kf[e], qv[g][e]));  // the product is exact
                }
                acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 1));
                acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 2));
                acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 4));
                const float sv = __fmul_rn(acc, scale);
                if (j < j1) {
                    if (sub == 0) {
                        scores[(int64_t) t * Nh * s_stride + (int64_t) (hk * G + g) * s_stride + j] = sv;
                    }
                    mx[g] = fmaxf(mx[g], sv);
                }
            }
        }
    }
#pragma unroll
    for (int g = 0; g < G; g++) {
        mx[g] = warp_max(mx[g]);
    }
    if (lane == 0) {
#pragma unroll
        for (int g = 0; g < G; g++) {
            wmax[warp][g] = mx[g];
        }
    }
    __syncthreads();
    if (threadIdx.x < G) {
        const int g = threadIdx.x;
        float     m = fmaxf(fmaxf(wmax[0][g], wmax[1][g]), fmaxf(wmax[2][g], wmax[3][g]));
        smax[((int64_t) t * Nh + hk * G + g) * n_split + split] = m;
    }
}

// ---- pass 2: global normaliser, f16 probabilities of this split's chunk, partial P.V ----------
template <int G, int PDL>
__global__ void __launch_bounds__(128) attn_pv_kernel(const float * __restrict__ scores, int64_t s_stride,
                                                      const float * __restrict__ smax, int Nh, int Nkv,
                                                      const int32_t * __restrict__ pos, KvLayout kv, int n_split,
                                                      double * __restrict__ part, float * __restrict__ out,
                                                      int64_t out_stride, int * __restrict__ tickets) {
    constexpr int D = 128;
    dep_wait<PDL>();
    ptx::grid_dep_launch();
    const int split = blockIdx.x, hk = blockIdx.y, t = blockIdx.z;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int kv_len = __ldg(pos + t) + 1;
    if (kv_len <= 0 || kv_len > kv.max_seq) {
        return;
    }
    const int chunk  = (kv_len + n_split - 1) / n_split;
    const int j0     = split * chunk;
    const int j1     = min(kv_len, j0 + chunk);
    const int set    = kv.set0 + t * kv.set_per_tok;
    __shared__ double red[4][G];
    __shared__ float  sM[G], sInv[G];

    // global max and double sum of exp(s - max) over the whole row; every loop keeps a batch of
    // loads in flight (a chain of dependent L2 round trips would dominate the kernel)
    float M[G];
#pragma unroll
    for (int g = 0; g < G; g++) {
        M[g] = -INFINITY;
    }
    for (int i0 = 0; i0 < n_split; i0 += 8) {
        float v[G][8];
#pragma unroll
        for (int g = 0; g < G; g++) {
            const float * sm = smax + ((int64_t) t * Nh + hk * G + g) * n_split;
#pragma unroll
            for (int u = 0; u < 8; u++) {
                v[g][u] = sm[min(i0 + u, n_split - 1)];  // clamped: a repeated maximum changes nothing
            }
        }
#pragma unroll
        for (int g = 0; g < G; g++) {
#pragma unroll
            for (int u = 0; u < 8; u++) {
                M[g] = fmaxf(M[g], v[g][u]);
            }
        }
    }
    double ssum[G];
#pragma unroll
    for (int g = 0; g < G; g++) {
        ssum[g] = 0.0;
    }
    constexpr int US = 8;
    for (int j0 = threadIdx.x; j0 < kv_len; j0 += 128 * US) {
        float v[G][US];
#pragma unroll
        for (int g = 0; g < G; g++) {
            const float * sr = scores + (int64_t) t * Nh * s_stride + (int64_t) (hk * G + g) * s_stride;
#pragma unroll
            for (int u = 0; u < US; u++) {
                v[g][u] = sr[min(j0 + 128 * u, kv_len - 1)];  // clamped: added only if in range
            }
        }
#pragma unroll
        for (int g = 0; g < G; g++) {
#pragma unroll
            for (int u = 0; u < US; u++) {
                if (j0 + 128 * u < kv_len) {
                    ssum[g] += (double) acb_expf(__fsub_rn(v[g][u], M[g]));
                }
            }
        }
    }
#pragma unroll
    for (int g = 0; g < G; g++) {
        const double sg = warp_sum(ssum[g]);
        if (lane == 0) {
            red[warp][g] = sg;
        }
    }
    __syncthreads();
    if (threadIdx.x < G) {
        const int    g = threadIdx.x;
        const double S = (red[0][g] + red[1][g]) + (red[2][g] + red[3][g]);
        sM[g]          = M[g];
        sInv[g]        = S > 0.0 ? (float) (1.0 / S) : 0.0f;
    }
    __syncthreads();

    // partial output over this chunk: lane owns 4 of the D elements, warps take blocks of 32 keys.
    // The probabilities of a block are computed once (lane l: key jb + l, every q head of the
    // group) and handed to the other lanes by shuffles.
    double acc[G][4];
#pragma unroll
    for (int g = 0; g < G; g++) {
#pragma unroll
        for (int e = 0; e < 4; e++) {
            acc[g][e] = 0.0;
        }
    }
    const uint16_t * vb = kv.v + kv_index(kv, Nkv, D, set, hk, 0);
    const float *    sb = scores + (int64_t) t * Nh * s_stride + (int64_t) (hk * G) * s_stride;
    constexpr int    U  = 8;  // V rows in flight per lane
    for (int jb = j0 + 32 * warp; jb < j1; jb += 32 * 4) {
        const int n  = min(32, j1 - jb);
        const int jl = min(jb + lane, j1 - 1);  // clamped: lanes past the chunk carry p = 0
        float     pl[G];
#pragma unroll
        for (int g = 0; g < G; g++) {
            const float pe = __fmul_rn(acb_expf(__fsub_rn(sb[(int64_t) g * s_stride + jl], sM[g])), sInv[g]);
            pl[g]          = lane < n ? __half2float(__float2half_rn(pe)) : 0.0f;
        }
        for (int u0 = 0; u0 < n; u0 += U) {
            uint2 raw[U];
#pragma unroll
            for (int u = 0; u < U; u++) {
                const int j = jb + min(u0 + u, n - 1);  // clamped: used only below n
                raw[u]      = *reinterpret_cast<const uint2 *>(vb + (int64_t) j * D + lane * 4);
            }
#pragma unroll
            for (int u = 0; u < U; u++) {
                if (u0 + u < n) {  // uniform over the warp
                    const float2 f01 = __half22float2(*reinterpret_cast<const __half2 *>(&raw[u].x));
                    const float2 f23 = __half22float2(*reinterpret_cast<const __half2 *>(&raw[u].y));
                    const double v0 = f01.x, v1 = f01.y, v2 = f23.x, v3 = f23.y;  // shared by the G heads
#pragma unroll
                    for (int g = 0; g < G; g++) {
                        const double pp = (double) __shfl_sync(0xffffffffu, pl[g], u0 + u);
                        // p * v is exact (two f16 values): the fused multiply-add rounds only the sum
                        acc[g][0] = fma(pp, v0, acc[g][0]);
                        acc[g][1] = fma(pp, v1, acc[g][1]);
                        acc[g][2] = fma(pp, v2, acc[g][2]);
                        acc[g][3] = fma(pp, v3, acc[g][3]);
                    }
                }
            }
        }
    }
    // reduce the 4 warps through shared memory, then write the split partial [t][split][Nh*D]
    __shared__ double4 wacc[4][G][32];
#pragma unroll
    for (int g = 0; g < G; g++) {
        wacc[warp][g][lane] = make_double4(acc[g][0], acc[g][1], acc[g][2], acc[g][3]);
    }
    __syncthreads();
    for (int g = warp; g < G; g += 4) {
        double4 r = wacc[0][g][lane];
#pragma unroll
        for (int w = 1; w < 4; w++) {
            const double4 o = wacc[w][g][lane];
            r.x += o.x;
            r.y += o.y;
            r.z += o.z;
            r.w += o.w;
        }
        double * dst = part + ((int64_t) t * n_split + split) * Nh * D + (int64_t) (hk * G + g) * D + lane * 4;
        reinterpret_cast<double2 *>(dst)[0] = make_double2(r.x, r.y);
        reinterpret_cast<double2 *>(dst)[1] = make_double2(r.z, r.w);
    }
    __threadfence();
    if (!out) {
        return;
    }
    // the last split CTA of this (token, kv head) sums the partials in split order
    __shared__ bool last;
    __syncthreads();
    if (threadIdx.x == 0) {
        const int tk = atomicAdd(tickets + t * Nkv + hk, 1);
        last         = (tk == n_split - 1);
    }
    __syncthreads();
    if (!last) {
        return;
    }
    __threadfence();
    for (int idx = threadIdx.x; idx < G * 64; idx += blockDim.x) {
        const int     g   = idx >> 6, l = idx & 63;
        const int64_t off = (int64_t) (hk * G + g) * D + l * 2;
        double2       a   = make_double2(0.0, 0.0);
        for (int s = 0; s < n_split; s++) {
            const double2 b = __ldcg(reinterpret_cast<const double2 *>(part + ((int64_t) t * n_split + s) * Nh * D + off));
            a.x += b.x;
            a.y += b.y;
        }
        *reinterpret_cast<float2 *>(out + (int64_t) t * out_stride + off) = make_float2((float) a.x, (float) a.y);
    }
    if (threadIdx.x == 0) {
        tickets[t * Nkv + hk] = 0;
    }
}

template <typename Kern, typename... Args>
static acb_status launch_ex(Kern k, dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim            = grid;
    cfg.blockDim           = block;
    cfg.dynamicSmemBytes   = smem;
    cfg.stream             = st;
    cudaLaunchAttribute attr[1];
    attr[0].id                                         = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs                                          = pdl ? attr : nullptr;
    cfg.numAttrs                                       = pdl ? 1 : 0;
    cudaError_t e                                      = cudaLaunchKernelEx(&cfg, k, args...);
    if (e != cudaSuccess) {
        set_last_cuda_error(e);
        return ACB_ERR_CUDA;
    }
    return ACB_OK;
}

}  // namespace acb

using namespace acb;

extern "C" acb_status acb_qkv_post(const float * qkv, int64_t qkv_stride, int64_t n_tok, int Nh, int Nkv,
                                   int head_dim, const float * q_norm, const float * k_norm, float eps,
                                   const int32_t * pos, const float * rope_table, int max_pos, float * q_out,
                                   int64_t q_stride, uint16_t * k_cache, uint16_t * v_cache, int max_seq, int set0,
                                   int set_per_tok, int flags, int * err_flag, acb_stream_t stream) {
    if (!qkv || !pos || !rope_table || !q_out || !k_cache || !v_cache || n_tok < 0 || Nh <= 0 || Nkv <= 0 ||
        max_pos <= 0 || max_seq <= 0 || set0 < 0) {
        return ACB_ERR_INVALID_ARG;
    }
    if (head_dim != 128) {
        return ACB_ERR_UNSUPPORTED;
    }
    if (n_tok == 0) {
        return ACB_OK;
    }
    KvLayout      kv    = { k_cache, v_cache, max_seq, set0, set_per_tok };
    const int64_t items = n_tok * (Nh + 2 * Nkv);
    const dim3    grid((unsigned) ((items + 7) / 8));
    const bool    pdl = flags & 1;
    if (pdl) {
        return launch_ex(qkv_post_kernel<2, 1>, grid, dim3(256), 0, (cudaStream_t) stream, true, qkv, qkv_stride,
                         n_tok, Nh, Nkv, q_norm, k_norm, eps, pos, rope_table, max_pos, q_out, q_stride, kv,
                         err_flag);
    }
    return launch_ex(qkv_post_kernel<2, 0>, grid, dim3(256), 0, (cudaStream_t) stream, false, qkv, qkv_stride, n_tok,
                     Nh, Nkv, q_norm, k_norm, eps, pos, rope_table, max_pos, q_out, q_stride, kv, err_flag);
}

extern "C" int acb_attn_decode_splits(int n_tok, int Nkv) {
    const int per = num_sms() / (n_tok * Nkv > 0 ? n_tok * Nkv : 1);
    return per < 1 ? 1 : (per > 32 ? 32 : per);
}

extern "C" acb_status acb_attn_decode(const float * q, int64_t q_stride, int n_tok, int Nh, int Nkv, int head_dim,
                                      const int32_t * pos, const uint16_t * k_cache, const uint16_t * v_cache,
                                      int max_seq, int set0, int set_per_tok, float scale, int n_split,
                                      float * scores, float * smax, double * part, float * out, int64_t out_stride,
                                      int * tickets, int flags, acb_stream_t stream) {
    if (!q || !pos || !k_cache || !v_cache || !scores || !smax || !part || n_tok <= 0 || Nh <= 0 || Nkv <= 0 ||
        n_split < 1 || max_seq <= 0 || (out && !tickets)) {
        return ACB_ERR_INVALID_ARG;
    }
    if (head_dim != 128 || Nh % Nkv != 0 || Nh / Nkv > 8) {
        return ACB_ERR_UNSUPPORTED;
    }
    KvLayout     kv   = { (uint16_t *) k_cache, (uint16_t *) v_cache, max_seq, set0, set_per_tok };
    const int    G    = Nh / Nkv;
    const dim3   grid((unsigned) n_split, (unsigned) Nkv, (unsigned) n_tok);
    cudaStream_t st   = (cudaStream_t) stream;
    const bool   pdl  = flags & 1;
    acb_status   rc   = ACB_OK;
#define ACB_ATT(GG)                                                                                                \
    if (G == GG) {                                                                                                 \
        rc = pdl ? launch_ex(attn_scores_kernel<GG, 1>, grid, dim3(128), 0, st, true, q, q_stride, Nh, Nkv, pos, kv, \
                             scale, n_split, scores, (int64_t) max_seq, smax)                                      \
                 : launch_ex(attn_scores_kernel<GG, 0>, grid, dim3(128), 0, st, false, q, q_stride, Nh, Nkv, pos, kv, \
                             scale, n_split, scores, (int64_t) max_seq, smax);                                     \
        if (rc != ACB_OK) {                                                                                        \
            return rc;                                                                                             \
        }                                                                                                          \
        return pdl ? launch_ex(attn_pv_kernel<GG, 1>, grid, dim3(128), 0, st, true, (const float *) scores,        \
                               (int64_t) max_seq, (const float *) smax, Nh, Nkv, pos, kv, n_split, part, out, \
                               out_stride, tickets)                                                                \
                   : launch_ex(attn_pv_kernel<GG, 0>, grid, dim3(128), 0, st, false, (const float *) scores,       \
                               (int64_t) max_seq, (const float *) smax, Nh, Nkv, pos, kv, n_split, part, out, \
                               out_stride, tickets);                                                               \
    }
    ACB_ATT(1)
    ACB_ATT(2)
    ACB_ATT(4)
    ACB_ATT(8)
#undef ACB_ATT
    return ACB_ERR_UNSUPPORTED;
}
