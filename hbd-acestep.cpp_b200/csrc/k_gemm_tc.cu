// k_gemm_tc.cu -- tensor-core GEMM for the dense prefill / DiT linears (src/dit-graph.h:36-49 and
// every ggml_mul_mat of dit_ggml_build_layer at M = tokens):
//     C[m][n] = epilogue( sum_k A[m][k] * B[n][k] ),  A, B bf16 or f16 K-major, fp32 accumulation.
//
// sm_100a design (one persistent CTA per SM, 6 warps, no clusters, no multicast):
//   warp 0      TMA producer: A tile 128x64 and B tile 256x64 per stage (128-byte swizzle) into a
//               4-stage ring (48 KB per stage), completion on an mbarrier per stage;
//   warp 1      allocates 512 TMEM columns (two 128x256 fp32 accumulators), one elected thread
//               issues tcgen05.mma (M=128, N=256, K=16; kind::f16 with bf16 or f16 inputs) and releases
//               ring stages / publishes finished accumulators with tcgen05.commit;
//   warps 2..5  epilogue: tcgen05.ld 32 columns at a time from their TMEM lane quarter, fused
//               bias / residual / DiT gated residual, f32, bf16 or f16 stores; the accumulator is
//               handed back so the MMA of the next tile overlaps this epilogue.
// Every mbarrier wait is bounded; on a timeout the kernel records ACB_DEVERR_TIMEOUT, stops, and
// still frees its TMEM.
#include <cuda.h>


#include "common.cuh"
#include "ptx.cuh"
#include "tc.cuh"

namespace acb {

constexpr int kBM = 128, kBN = 256, kBK = 64, kStages = 4;
constexpr int kATile = kBM * kBK * 2;  // 16 KB
constexpr int kBTile = kBN * kBK * 2;  // 32 KB
constexpr int kStageBytes = kATile + kBTile;
constexpr int kGemmThreads = 192;
constexpr int kTmemCols    = 512;

enum { EPI_PLAIN = 0, EPI_BIAS = 1, EPI_RES = 2, EPI_GATED_RES = 4 };

struct GemmArgs {
    int64_t       M, N, K;
    void *        C;
    int           c_type;  // ACB_TYPE_F32, ACB_TYPE_BF16 or ACB_TYPE_F16
    int64_t       ldc;
    const float * bias;    // [N] or null
    int           epi;     // bit set of EPI_*
    const float * res;     // f32 [M][ldr] (may alias C when C is f32)
    int64_t       ldr;
    const float * gate;    // f32 [samples][gate_stride], EPI_GATED_RES: C = res + acc * gate
    int64_t       gate_stride;
    int64_t       rows_per_sample;
    int *         err;
    int           splits;  // split-K factor; > 1: raw partials to ws, epilogue by splitk_reduce_kernel
    int           kps;     // k-tiles per split
    float *       ws;      // [splits][M][N] f32 partial accumulators
};

// 32 accumulator columns of one row to a 16-bit C (vector stores when whole and aligned)
template <int T>
__device__ __forceinline__ void store_row16(void * C, int64_t off, const float * v, bool full_cols, int left) {
    using et = typename io<T>::t;
    et * dst = reinterpret_cast<et *>(C) + off;
    if (full_cols && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
#pragma unroll
        for (int j = 0; j < 32; j += 8) {
            vec16<T> pk;
#pragma unroll
            for (int e = 0; e < 8; e++) {
                pk.v[e] = io<T>::from_f(v[j + e]);
            }
            *reinterpret_cast<uint4 *>(dst + j) = pk.u;
        }
    } else {
        for (int j = 0; j < 32 && j < left; j++) {
            dst[j] = io<T>::from_f(v[j]);
        }
    }
}

// ---- the kernel ------------------------------------------------------------------------------------
template <bool F16>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const GemmArgs g) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t * smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t * ring = smem;  // kStages * kStageBytes, 1024-aligned tiles
    uint64_t * full       = reinterpret_cast<uint64_t *>(smem + kStages * kStageBytes);
    uint64_t * empty      = full + kStages;
    uint64_t * tmem_full  = empty + kStages;
    uint64_t * tmem_empty = tmem_full + 2;
    uint32_t * tmem_slot  = reinterpret_cast<uint32_t *>(tmem_empty + 2);
    __shared__ volatile int abort_flag;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t m_tiles = (g.M + kBM - 1) / kBM, n_tiles = (g.N + kBN - 1) / kBN;
    const int64_t tiles   = m_tiles * n_tiles;
    const int64_t n_work  = tiles * g.splits;
    const int     k_tiles = (int) (g.K / kBK);

    if (threadIdx.x == 0) {
        abort_flag = 0;
        for (int s = 0; s < kStages; s++) {
            ptx::mbar_init(&full[s], 1);
            ptx::mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; a++) {
            ptx::mbar_init(&tmem_full[a], 1);
            ptx::mbar_init(&tmem_empty[a], 4);  // one arrival per epilogue warp
        }
        ptx::fence_mbar_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         ptx::smem_u32(tmem_slot)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    ptx::grid_dep_wait();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            int it = 0;  // global k-stage counter
            for (int64_t w = blockIdx.x; w < n_work && !abort_flag; w += gridDim.x) {
                const int64_t t  = w % tiles;
                const int     sp = (int) (w / tiles);
                const int m0 = (int) ((t % m_tiles) * kBM), n0 = (int) ((t / m_tiles) * kBN);
                const int kt1 = min(k_tiles, (sp + 1) * g.kps);
                for (int kt = sp * g.kps; kt < kt1; kt++, it++) {
                    const int s = it % kStages;
                    if (it >= kStages && !ptx::mbar_wait(&empty[s], ((it / kStages) - 1) & 1)) {
                        flag_timeout(g.err);
                        abort_flag = 1;
                        break;
                    }
                    uint8_t * st = ring + (size_t) s * kStageBytes;
                    ptx::mbar_arrive_expect_tx(&full[s], kStageBytes);
                    tma_load_2d(st, &tmA, kt * kBK, m0, &full[s]);
                    tma_load_2d(st + kATile, &tmB, kt * kBK, n0, &full[s]);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_kind_f16(kBM, kBN, F16);
            int                it    = 0;
            int                tile  = 0;
            for (int64_t w = blockIdx.x; w < n_work && !abort_flag; w += gridDim.x, tile++) {
                const int acc = tile & 1;
                if (tile >= 2 && !ptx::mbar_wait(&tmem_empty[acc], ((tile >> 1) - 1) & 1)) {
                    flag_timeout(g.err);
                    abort_flag = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t tmem_d = tmem_base + (uint32_t) (acc * kBN);
                const int      kt0    = (int) (w / tiles) * g.kps;
                const int      kt1    = min(k_tiles, kt0 + g.kps);
                for (int kt = kt0; kt < kt1; kt++, it++) {
                    const int s = it % kStages;
                    if (!ptx::mbar_wait(&full[s], (it / kStages) & 1)) {
                        flag_timeout(g.err);
                        abort_flag = 1;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a0 = ptx::smem_u32(ring + (size_t) s * kStageBytes);
                    const uint32_t b0 = a0 + kATile;
#pragma unroll
                    for (int kk = 0; kk < kBK / 16; kk++) {
                        umma_f16kind(tmem_d, smem_desc_sw128(a0 + kk * 32), smem_desc_sw128(b0 + kk * 32), idesc,
                                  (kt != kt0 || kk != 0) ? 1u : 0u);
                    }
                    umma_commit(&empty[s]);  // frees the stage once these MMAs have read it
                }
                umma_commit(&tmem_full[acc]);  // accumulator complete
            }
        }
    } else {
        // epilogue: warp w reads TMEM lanes 32*(w%4) .. +31 = tile rows
        const int q    = warp & 3;
        const int row_in_tile = q * 32 + lane;
        int       tile = 0;
        for (int64_t w = blockIdx.x; w < n_work; w += gridDim.x, tile++) {
            const int acc = tile & 1;
            if (!ptx::mbar_wait(&tmem_full[acc], (tile >> 1) & 1)) {
                if (lane == 0) {
                    flag_timeout(g.err);
                }
                abort_flag = 1;
                break;
            }
            tc_fence_after();
            const int64_t t  = w % tiles;
            const int64_t m  = (t % m_tiles) * kBM + row_in_tile;
            const int64_t n0 = (t / m_tiles) * kBN;
            const bool    part = g.splits > 1;  // raw partial of split w / tiles
            float *       pdst = part ? g.ws + ((w / tiles) * g.M + m) * g.N : nullptr;
            const float * gate_row = (!part && (g.epi & EPI_GATED_RES))
                                         ? g.gate + (m < g.M ? (m / g.rows_per_sample) : 0) * g.gate_stride
                                         : nullptr;
#pragma unroll 1
            for (int c = 0; c < kBN / 32; c++) {
                uint32_t r[32];
                tmem_ld32(tmem_base + ((uint32_t) (q * 32) << 16) + (uint32_t) (acc * kBN + c * 32), r);
                const int64_t nc = n0 + c * 32;
                if (m < g.M && nc < g.N) {
                float v[32];
#pragma unroll
                for (int j = 0; j < 32; j++) {
                    v[j] = __uint_as_float(r[j]);
                }
                const bool full_cols = nc + 32 <= g.N;
                if (part) {
                    float * dst = pdst + nc;
                    if (full_cols && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
#pragma unroll
                        for (int j = 0; j < 32; j += 4) {
                            *reinterpret_cast<float4 *>(dst + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
                        }
                    } else {
                        for (int j = 0; j < 32 && nc + j < g.N; j++) {
                            dst[j] = v[j];
                        }
                    }
                } else {  // final tile: epilogue and store
                if (g.bias) {
#pragma unroll
                    for (int j = 0; j < 32; j++) {
                        if (full_cols || nc + j < g.N) {
                            v[j] = __fadd_rn(v[j], g.bias[nc + j]);
                        }
                    }
                }
                if (g.epi & (EPI_RES | EPI_GATED_RES)) {
                    const float * rr = g.res + m * g.ldr + nc;
#pragma unroll
                    for (int j = 0; j < 32; j++) {
                        if (full_cols || nc + j < g.N) {
                            const float o = (g.epi & EPI_GATED_RES) ? __fmul_rn(v[j], gate_row[nc + j]) : v[j];
                            v[j]          = __fadd_rn(rr[j], o);
                        }
                    }
                }
                if (g.c_type == ACB_TYPE_F32) {
                    float * dst = reinterpret_cast<float *>(g.C) + m * g.ldc + nc;
                    if (full_cols && (reinterpret_cast<uintptr_t>(dst) & 15) == 0) {
#pragma unroll
                        for (int j = 0; j < 32; j += 4) {
                            *reinterpret_cast<float4 *>(dst + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
                        }
                    } else {
                        for (int j = 0; j < 32 && nc + j < g.N; j++) {
                            dst[j] = v[j];
                        }
                    }
                } else if (g.c_type == ACB_TYPE_BF16) {
                    store_row16<ACB_TYPE_BF16>(g.C, m * g.ldc + nc, v, full_cols, (int) (g.N - nc));
                } else {
                    store_row16<ACB_TYPE_F16>(g.C, m * g.ldc + nc, v, full_cols, (int) (g.N - nc));
                }
                }  // final tile
                }  // valid row and column chunk
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                ptx::mbar_arrive(&tmem_empty[acc]);
            }
        }
    }
    ptx::grid_dep_launch();
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols));
    }
}

// Split-K second pass: C = epilogue(sum over splits of the partials, in split order), four
// consecutive columns per thread. Deterministic: every element is summed in the same order.
__global__ void __launch_bounds__(256) splitk_reduce_kernel(const GemmArgs g) {
    ptx::grid_dep_wait();
    const int64_t nq  = g.N / 4;
    const int64_t idx = (int64_t) blockIdx.x * blockDim.x + threadIdx.x;
    if (idx < g.M * nq) {
        const int64_t m = idx / nq, n = (idx - m * nq) * 4;
        float4        a = *reinterpret_cast<const float4 *>(g.ws + m * g.N + n);
        float         v[4] = { a.x, a.y, a.z, a.w };
        for (int sp = 1; sp < g.splits; sp++) {
            const float4 b = *reinterpret_cast<const float4 *>(g.ws + (sp * g.M + m) * g.N + n);
            v[0] = __fadd_rn(v[0], b.x);
            v[1] = __fadd_rn(v[1], b.y);
            v[2] = __fadd_rn(v[2], b.z);
            v[3] = __fadd_rn(v[3], b.w);
        }
#pragma unroll
        for (int j = 0; j < 4; j++) {
            if (g.bias) {
                v[j] = __fadd_rn(v[j], g.bias[n + j]);
            }
            if (g.epi & (EPI_RES | EPI_GATED_RES)) {
                const float o = (g.epi & EPI_GATED_RES)
                                    ? __fmul_rn(v[j], g.gate[(m / g.rows_per_sample) * g.gate_stride + n + j])
                                    : v[j];
                v[j] = __fadd_rn(g.res[m * g.ldr + n + j], o);
            }
        }
        if (g.c_type == ACB_TYPE_F32) {
            float * d = reinterpret_cast<float *>(g.C) + m * g.ldc + n;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                d[j] = v[j];
            }
        } else if (g.c_type == ACB_TYPE_BF16) {
            __nv_bfloat16 * d = reinterpret_cast<__nv_bfloat16 *>(g.C) + m * g.ldc + n;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                d[j] = __float2bfloat16_rn(v[j]);
            }
        } else {
            __half * d = reinterpret_cast<__half *>(g.C) + m * g.ldc + n;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                d[j] = __float2half_rn(v[j]);
            }
        }
    }
    ptx::grid_dep_launch();
}

// Split-K factor for an M x N x K GEMM: only when the output tiles leave most SMs idle; every
// split keeps at least 4 k-tiles (256 of K) so its pipeline fill stays amortised.
static int choose_splits(int64_t M, int64_t N, int64_t K, int * kps) {
    const int64_t tiles   = ((M + kBM - 1) / kBM) * ((N + kBN - 1) / kBN);
    const int     k_tiles = (int) (K / kBK);
    const int     sms     = num_sms();
    *kps                  = k_tiles;
    if (tiles * 2 > sms || k_tiles < 8 || N % 4 != 0) {
        return 1;
    }
    int sp = (int) (sms / tiles);
    sp     = sp < k_tiles / 4 ? sp : k_tiles / 4;
    sp     = sp < 16 ? sp : 16;
    if (sp < 2) {
        return 1;
    }
    *kps = (k_tiles + sp - 1) / sp;
    return (k_tiles + *kps - 1) / *kps;
}

// bf16/f16 row-major [rows][ld] (K contiguous), box = box_rows x 64 elements, 128-byte swizzle
static bool make_map(CUtensorMap * m, const void * base, int64_t rows, int64_t K, int64_t ld, int box_rows,
                     bool f16) {
    return make_map_2d(m, base, f16, K, rows, ld, kBK, box_rows);
}

}  // namespace acb

using namespace acb;

extern "C" size_t acb_gemm_workspace_bytes(int64_t M, int64_t N, int64_t K) {
    if (M <= 0 || N <= 0 || K <= 0 || K % kBK != 0) {
        return 0;
    }
    int       kps = 0;
    const int sp  = choose_splits(M, N, K, &kps);
    return sp > 1 ? (size_t) sp * (size_t) M * (size_t) N * 4 : 0;
}

extern "C" acb_status acb_gemm_tc(const void * A, int64_t lda, const void * B, int64_t ldb, int64_t M, int64_t N,
                                  int64_t K, void * C, int c_type, int64_t ldc, const float * bias, const float * res,
                                  int64_t ldr, const float * gate, int64_t gate_stride, int64_t rows_per_sample,
                                  int flags, void * workspace, size_t workspace_bytes, int * err_flag,
                                  acb_stream_t stream) {
    if (!A || !B || !C || M <= 0 || N <= 0 || K <= 0 || lda < K || ldb < K || ldc < N) {
        return ACB_ERR_INVALID_ARG;
    }
    if (K % kBK != 0 || (lda * 2) % 16 != 0 || (ldb * 2) % 16 != 0 || reinterpret_cast<uintptr_t>(A) % 16 != 0 ||
        reinterpret_cast<uintptr_t>(B) % 16 != 0) {
        return ACB_ERR_UNSUPPORTED;
    }
    if (c_type != ACB_TYPE_F32 && c_type != ACB_TYPE_BF16 && c_type != ACB_TYPE_F16) {
        return ACB_ERR_UNSUPPORTED;
    }
    if (gate && (!res || rows_per_sample <= 0)) {
        return ACB_ERR_INVALID_ARG;
    }
    GemmArgs g        = {};
    g.M               = M;
    g.N               = N;
    g.K               = K;
    g.C               = C;
    g.c_type          = c_type;
    g.ldc             = ldc;
    g.bias            = bias;
    g.epi             = (bias ? EPI_BIAS : 0) | (gate ? EPI_GATED_RES : (res ? EPI_RES : 0));
    g.res             = res;
    g.ldr             = ldr;
    g.gate            = gate;
    g.gate_stride     = gate_stride;
    g.rows_per_sample = rows_per_sample > 0 ? rows_per_sample : 1;
    g.err             = err_flag;
    g.splits          = 1;
    g.kps             = (int) (K / kBK);
    {
        int       kps = 0;
        const int sp  = choose_splits(M, N, K, &kps);
        if (sp > 1 && workspace && reinterpret_cast<uintptr_t>(workspace) % 16 == 0 &&
            workspace_bytes >= (size_t) sp * (size_t) M * (size_t) N * 4) {
            g.splits = sp;
            g.kps    = kps;
            g.ws     = reinterpret_cast<float *>(workspace);
        }
    }
    const bool  f16 = (flags & ACB_FLAG_F16) != 0;
    CUtensorMap ta, tb;
    if (!make_map(&ta, A, M, K, lda, kBM, f16) || !make_map(&tb, B, N, K, ldb, kBN, f16)) {
        return ACB_ERR_CUDA;
    }
    const int64_t work = ((M + kBM - 1) / kBM) * ((N + kBN - 1) / kBN) * g.splits;
    const int     grid = (int) (work < num_sms() ? work : num_sms());
    const size_t  smem = (size_t) kStages * kStageBytes + 1024 + 256;
    void (*kern)(const CUtensorMap, const CUtensorMap, const GemmArgs) =
        f16 ? gemm_tc_kernel<true> : gemm_tc_kernel<false>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim            = dim3((unsigned) grid);
    cfg.blockDim           = dim3(kGemmThreads);
    cfg.dynamicSmemBytes   = smem;
    cfg.stream             = (cudaStream_t) stream;
    cudaLaunchAttribute attr[1];
    attr[0].id                                         = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs                                          = (flags & ACB_FLAG_PDL) ? attr : nullptr;
    cfg.numAttrs                                       = (flags & ACB_FLAG_PDL) ? 1 : 0;
    cudaError_t e                                      = cudaLaunchKernelEx(&cfg, kern, ta, tb, g);
    if (e == cudaSuccess && g.splits > 1) {
        // the reduction always waits on the GEMM through griddepcontrol.wait
        const int64_t n_thr = M * (N / 4);
        cfg.gridDim         = dim3((unsigned) ((n_thr + 255) / 256));
        cfg.blockDim        = dim3(256);
        cfg.dynamicSmemBytes = 0;
        cfg.attrs           = attr;
        cfg.numAttrs        = 1;
        e                   = cudaLaunchKernelEx(&cfg, splitk_reduce_kernel, g);
    }
    if (e != cudaSuccess) {
        set_last_cuda_error(e);
        return ACB_ERR_CUDA;
    }
    return ACB_OK;
}

extern "C" acb_status acb_gemm_bf16(const void * A, int64_t lda, const void * B, int64_t ldb, int64_t M, int64_t N,
                                    int64_t K, void * C, int c_type, int64_t ldc, const float * bias, const float * res,
                                    int64_t ldr, const float * gate, int64_t gate_stride, int64_t rows_per_sample,
                                    int flags, int * err_flag, acb_stream_t stream) {
    return acb_gemm_tc(A, lda, B, ldb, M, N, K, C, c_type, ldc, bias, res, ldr, gate, gate_stride, rows_per_sample,
                       flags, nullptr, 0, err_flag, stream);
}
