// k_getrows.cu -- embedding gather with in-register dequantisation (ggml_get_rows).
//
// One warp per gathered row. A quantised row (Q8_0 / Q4_K / Q6_K blocks) is first copied into
// shared memory with coalesced 16-byte loads (GGUF rows of these types are 16-byte multiples
// at the BASELINE widths; 4- and 1-byte loads cover other widths), then every lane dequantises
// whole 16-byte output vectors from shared memory and writes them with streaming stores.
// Dequantisation rounds exactly like the ggml / gguf-py dequantisers:
//   Q8_0: d*q          Q4_K: (d*sc)*q - (dmin*m)          Q6_K: (d*sc)*q
#include "common.cuh"

namespace acb {

struct qdesc {
    int blk_elems;
    int blk_bytes;
};

__host__ __device__ inline qdesc qinfo(int t) {
    switch (t) {
        case ACB_TYPE_Q8_0:
            return { 32, 34 };
        case ACB_TYPE_Q4_K:
            return { 256, 144 };
        case ACB_TYPE_Q6_K:
            return { 256, 210 };
        case ACB_TYPE_F32:
            return { 1, 4 };
        case ACB_TYPE_F16:
        case ACB_TYPE_BF16:
            return { 1, 2 };
        default:
            return { 0, 0 };
    }
}

// Dequantise element e of a row held in shared memory.
template <int QT> __device__ __forceinline__ float deq(const uint8_t * row, int e);

template <> __device__ __forceinline__ float deq<ACB_TYPE_Q8_0>(const uint8_t * row, int e) {
    const uint8_t * b = row + (e >> 5) * 34;
    return __fmul_rn(f16_bits_to_f(ld_u16(b)), (float) (int8_t) b[2 + (e & 31)]);
}

template <> __device__ __forceinline__ float deq<ACB_TYPE_Q4_K>(const uint8_t * row, int e) {
    const uint8_t * b   = row + (e >> 8) * 144;
    const int       j   = e & 255;
    const int       g   = j >> 6, hi = (j >> 5) & 1, l = j & 31;
    const int       sub = 2 * g + hi;
    const uint8_t * sc  = b + 4;
    int             s, m;
    if (sub < 4) {
        s = sc[sub] & 63;
        m = sc[sub + 4] & 63;
    } else {
        s = (sc[sub + 4] & 0x0f) | ((sc[sub - 4] >> 6) << 4);
        m = (sc[sub + 4] >> 4) | ((sc[sub] >> 6) << 4);
    }
    const uint8_t qb = b[16 + g * 32 + l];
    const int     q  = hi ? (qb >> 4) : (qb & 0x0f);
    const float   d1 = __fmul_rn(f16_bits_to_f(ld_u16(b)), (float) s);
    const float   m1 = __fmul_rn(f16_bits_to_f(ld_u16(b + 2)), (float) m);
    return __fsub_rn(__fmul_rn(d1, (float) q), m1);
}

template <> __device__ __forceinline__ float deq<ACB_TYPE_Q6_K>(const uint8_t * row, int e) {
    const uint8_t * b    = row + (e >> 8) * 210;
    const int       j    = e & 255;
    const int       half = j >> 7, c = (j >> 5) & 3, l = j & 31;
    int             lo   = b[half * 64 + ((c & 1) ? 32 : 0) + l];
    lo                   = (c & 2) ? (lo >> 4) : (lo & 0x0f);
    const int hi         = (b[128 + half * 32 + l] >> (2 * c)) & 3;
    const int q          = (lo | (hi << 4)) - 32;
    const float ds       = __fmul_rn(f16_bits_to_f(ld_u16(b + 208)), (float) (int8_t) b[192 + (j >> 4)]);
    return __fmul_rn(ds, (float) q);
}

// Dequantise the NO consecutive elements v*NO .. v*NO+NO-1 of a row held in shared memory.
template <int QT, int NO> __device__ __forceinline__ void deq_vec(const uint8_t * row, int v, float * f) {
#pragma unroll
    for (int j = 0; j < NO; j++) {
        f[j] = deq<QT>(row, v * NO + j);
    }
}

// Q8_0: the NO elements share one block (NO divides 32); its f16 scale is one 2-byte load and
// the int8 quants NO/2 2-byte loads (a block starts at an even offset, 34 bytes per block).
template <> __device__ __forceinline__ void deq_vec<ACB_TYPE_Q8_0, 4>(const uint8_t * row, int v, float * f) {
    const uint8_t * b = row + (v >> 3) * 34;
    const float     d = f16_bits_to_f(*reinterpret_cast<const uint16_t *>(b));
    const uint16_t * q = reinterpret_cast<const uint16_t *>(b + 2 + (v & 7) * 4);
    const uint16_t  q0 = q[0], q1 = q[1];
    f[0]               = __fmul_rn(d, (float) (int8_t) (q0 & 0xff));
    f[1]               = __fmul_rn(d, (float) (int8_t) (q0 >> 8));
    f[2]               = __fmul_rn(d, (float) (int8_t) (q1 & 0xff));
    f[3]               = __fmul_rn(d, (float) (int8_t) (q1 >> 8));
}

template <> __device__ __forceinline__ void deq_vec<ACB_TYPE_Q8_0, 8>(const uint8_t * row, int v, float * f) {
    const uint8_t * b = row + (v >> 2) * 34;
    const float     d = f16_bits_to_f(*reinterpret_cast<const uint16_t *>(b));
    const uint16_t * q = reinterpret_cast<const uint16_t *>(b + 2 + (v & 3) * 8);
#pragma unroll
    for (int j = 0; j < 4; j++) {
        const uint16_t w = q[j];
        f[2 * j]         = __fmul_rn(d, (float) (int8_t) (w & 0xff));
        f[2 * j + 1]     = __fmul_rn(d, (float) (int8_t) (w >> 8));
    }
}

template <int QT, int TO>
__global__ void __launch_bounds__(256) get_rows_q_kernel(const uint8_t * __restrict__ table, int64_t n_rows,
                                                         int64_t row_bytes, int cols, const int32_t * __restrict__ ids,
                                                         int64_t n_ids, void * __restrict__ out, int64_t out_stride,
                                                         int * __restrict__ err, int smem_row, int load_w) {
    extern __shared__ __align__(16) uint8_t smem[];
    using eo              = typename io<TO>::t;
    constexpr int NO      = 16 / sizeof(eo);
    const int     lane    = threadIdx.x & 31;
    const int     wid     = threadIdx.x >> 5;
    const int64_t i       = (int64_t) blockIdx.x * (blockDim.x >> 5) + wid;
    if (i >= n_ids) {
        return;
    }
    uint8_t *     srow = smem + (int64_t) wid * smem_row;
    eo *          orow = reinterpret_cast<eo *>(out) + i * out_stride;
    const int32_t id   = __ldg(ids + i);
    const int     nvo  = cols / NO;
    if (id < 0 || id >= n_rows) {
        if (lane == 0 && err) {
            atomicOr(err, ACB_DEVERR_ID_RANGE);
        }
        for (int v = lane; v < nvo; v += 32) {
            reinterpret_cast<uint4 *>(orow)[v] = make_uint4(0, 0, 0, 0);
        }
        return;
    }
    const uint8_t * g = table + (int64_t) id * row_bytes;
    if (load_w == 16) {
        for (int64_t k = lane; k < row_bytes / 16; k += 32) {
            reinterpret_cast<uint4 *>(srow)[k] = __ldg(reinterpret_cast<const uint4 *>(g) + k);
        }
    } else if (load_w == 4) {
        for (int64_t k = lane; k < row_bytes / 4; k += 32) {
            reinterpret_cast<uint32_t *>(srow)[k] = __ldg(reinterpret_cast<const uint32_t *>(g) + k);
        }
    } else {
        for (int64_t k = lane; k < row_bytes; k += 32) {
            srow[k] = g[k];
        }
    }
    __syncwarp();
    for (int v = lane; v < nvo; v += 32) {
        union {
            eo    e[NO];
            uint4 u;
        } r;
        float f[NO];
        deq_vec<QT, NO>(srow, v, f);
#pragma unroll
        for (int j = 0; j < NO; j++) {
            r.e[j] = io<TO>::from_f(f[j]);
        }
        __stcs(reinterpret_cast<uint4 *>(orow) + v, r.u);
    }
}

// Plain-type tables (F32 / F16 / BF16): convert element by element.
template <int TI, int TO>
__global__ void __launch_bounds__(256) get_rows_plain_kernel(const void * __restrict__ table, int64_t n_rows,
                                                             int cols, const int32_t * __restrict__ ids,
                                                             int64_t n_ids, void * __restrict__ out,
                                                             int64_t out_stride, int * __restrict__ err) {
    using ei           = typename io<TI>::t;
    using eo           = typename io<TO>::t;
    const int     lane = threadIdx.x & 31;
    const int64_t i    = (int64_t) blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (i >= n_ids) {
        return;
    }
    const int32_t id   = __ldg(ids + i);
    eo *          orow = reinterpret_cast<eo *>(out) + i * out_stride;
    if (id < 0 || id >= n_rows) {
        if (lane == 0 && err) {
            atomicOr(err, ACB_DEVERR_ID_RANGE);
        }
        for (int c = lane; c < cols; c += 32) {
            orow[c] = io<TO>::from_f(0.0f);
        }
        return;
    }
    const ei * src = reinterpret_cast<const ei *>(table) + (int64_t) id * cols;
    for (int c = lane; c < cols; c += 32) {
        orow[c] = io<TO>::from_f(io<TI>::to_f(src[c]));
    }
}

template <int QT, int TO>
static acb_status launch_q(const void * table, int64_t n_rows, int64_t cols, const int32_t * ids, int64_t n_ids,
                           void * out, int64_t os, int * err, cudaStream_t st) {
    const qdesc   q         = qinfo(QT);
    const int64_t row_bytes = cols / q.blk_elems * q.blk_bytes;
    const int     smem_row  = (int) ((row_bytes + 15) / 16 * 16);
    int           warps     = 8;
    while (warps > 1 && (int64_t) warps * smem_row > 96 * 1024) {
        warps >>= 1;
    }
    const int64_t smem = (int64_t) warps * smem_row;
    if (smem > 220 * 1024) {
        return ACB_ERR_UNSUPPORTED;
    }
    const uintptr_t base   = reinterpret_cast<uintptr_t>(table);
    const int       load_w = (base % 16 == 0 && row_bytes % 16 == 0) ? 16 : ((base % 4 == 0 && row_bytes % 4 == 0) ? 4 : 1);
    auto            kern   = get_rows_q_kernel<QT, TO>;
    if (smem > 48 * 1024) {
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);
    }
    const dim3 grid((unsigned) ((n_ids + warps - 1) / warps));
    kern<<<grid, warps * 32, (size_t) smem, st>>>((const uint8_t *) table, n_rows, row_bytes, (int) cols, ids, n_ids,
                                                  out, os, err, smem_row, load_w);
    return launch_status();
}

template <int TI, int TO>
static acb_status launch_plain(const void * table, int64_t n_rows, int64_t cols, const int32_t * ids, int64_t n_ids,
                               void * out, int64_t os, int * err, cudaStream_t st) {
    const dim3 grid((unsigned) ((n_ids + 7) / 8));
    get_rows_plain_kernel<TI, TO><<<grid, 256, 0, st>>>(table, n_rows, (int) cols, ids, n_ids, out, os, err);
    return launch_status();
}

template <int TO>
static acb_status dispatch_table(int tt, const void * table, int64_t n_rows, int64_t cols, const int32_t * ids,
                                 int64_t n_ids, void * out, int64_t os, int * err, cudaStream_t st) {
    constexpr int NO = 16 / sizeof(typename io<TO>::t);
    const bool    qvec = cols % NO == 0 && reinterpret_cast<uintptr_t>(out) % 16 == 0 &&
                      (os * (int64_t) sizeof(typename io<TO>::t)) % 16 == 0;
    switch (tt) {
        case ACB_TYPE_Q8_0:
            return qvec ? launch_q<ACB_TYPE_Q8_0, TO>(table, n_rows, cols, ids, n_ids, out, os, err, st)
                        : ACB_ERR_UNSUPPORTED;
        case ACB_TYPE_Q4_K:
            return qvec ? launch_q<ACB_TYPE_Q4_K, TO>(table, n_rows, cols, ids, n_ids, out, os, err, st)
                        : ACB_ERR_UNSUPPORTED;
        case ACB_TYPE_Q6_K:
            return qvec ? launch_q<ACB_TYPE_Q6_K, TO>(table, n_rows, cols, ids, n_ids, out, os, err, st)
                        : ACB_ERR_UNSUPPORTED;
        case ACB_TYPE_F32:
            return launch_plain<ACB_TYPE_F32, TO>(table, n_rows, cols, ids, n_ids, out, os, err, st);
        case ACB_TYPE_F16:
            return launch_plain<ACB_TYPE_F16, TO>(table, n_rows, cols, ids, n_ids, out, os, err, st);
        case ACB_TYPE_BF16:
            return launch_plain<ACB_TYPE_BF16, TO>(table, n_rows, cols, ids, n_ids, out, os, err, st);
        default:
            return ACB_ERR_UNSUPPORTED;
    }
}

}  // namespace acb

using namespace acb;

extern "C" acb_status acb_get_rows(const void * table, int table_type, int64_t n_rows, int64_t cols,
                                   const int32_t * ids, int64_t n_ids, void * out, int out_type, int64_t out_stride,
                                   int * err_flag, acb_stream_t stream) {
    if (!table || !ids || !out || n_rows <= 0 || cols <= 0 || n_ids < 0 || out_stride < cols) {
        return ACB_ERR_INVALID_ARG;
    }
    const qdesc q = qinfo(table_type);
    if (q.blk_elems == 0) {
        return ACB_ERR_UNSUPPORTED;
    }
    if (cols % q.blk_elems != 0) {
        return ACB_ERR_INVALID_ARG;
    }
    if (n_ids == 0) {
        return ACB_OK;
    }
    cudaStream_t st = (cudaStream_t) stream;
    switch (out_type) {
        case ACB_TYPE_F32:
            return dispatch_table<ACB_TYPE_F32>(table_type, table, n_rows, cols, ids, n_ids, out, out_stride, err_flag,
                                                st);
        case ACB_TYPE_BF16:
            return dispatch_table<ACB_TYPE_BF16>(table_type, table, n_rows, cols, ids, n_ids, out, out_stride,
                                                 err_flag, st);
        case ACB_TYPE_F16:
            return dispatch_table<ACB_TYPE_F16>(table_type, table, n_rows, cols, ids, n_ids, out, out_stride, err_flag,
                                                st);
        default:
            return ACB_ERR_UNSUPPORTED;
    }
}
