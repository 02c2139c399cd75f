// k_argmax.cu -- greedy sampling on device (the temperature-0 branch of sample_top_k_p,
// src/sampling.h:30-34): argmax over a logits row with the lowest index winning ties, plus the
// top1 - top2 margin.
//
// A row (217,472 logits = 870 KB at the BASELINE vocabulary) is split over ~50 CTAs, each
// streaming its chunk with 16-byte loads (four in flight per thread) and reducing to a
// (best, index, second) triple. Partials go to caller-provided scratch; the CTA that finishes
// last (ticket counter, which it resets for the next launch) merges them and writes the token,
// so the whole sampling step is one launch and can sit inside a CUDA graph.
#include <mutex>
#include <string>

#include "common.cuh"
#include "best.cuh"
#include "ptx.cuh"

namespace acb {

__device__ Best block_best(Best s) {
    __shared__ float sb1[32], sb2[32];
    __shared__ int   si1[32];
    const int        lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        best_merge(s, __shfl_xor_sync(0xffffffffu, s.b1, o), __shfl_xor_sync(0xffffffffu, s.b2, o),
                   __shfl_xor_sync(0xffffffffu, s.i1, o));
    }
    if (lane == 0) {
        sb1[warp] = s.b1;
        sb2[warp] = s.b2;
        si1[warp] = s.i1;
    }
    __syncthreads();
    Best r = { sb1[0], sb2[0], si1[0] };
    for (int w = 1; w < (int) (blockDim.x >> 5); w++) {
        best_merge(r, sb1[w], sb2[w], si1[w]);
    }
    return r;
}

// scratch layout: int ticket[ticket_rows] (padded to 256 bytes) at offset 0, then
// float4 part[rows][nblk] (b1, b2, i1 bits, -). The tickets sit at the same offset for every
// shape, so a buffer reused across (rows, V) never finds a stale partial where a counter lives.
template <int PDL>
__global__ void __launch_bounds__(256) argmax_kernel(const float * __restrict__ logits, int64_t stride, int64_t V,
                                                     int64_t chunk, int32_t * __restrict__ ids,
                                                     float * __restrict__ margin, int32_t * __restrict__ pos_advance,
                                                     int32_t * __restrict__ hist, float * __restrict__ mhist,
                                                     int64_t hist_stride, const int32_t * __restrict__ hist_base,
                                                     float4 * __restrict__ part, int * __restrict__ ticket) {
    if (PDL) {
        ptx::grid_dep_wait();
    }
    ptx::grid_dep_launch();
    const int     row  = blockIdx.y;
    const int     nblk = gridDim.x;
    const float * l    = logits + (int64_t) row * stride;
    const int64_t c0   = (int64_t) blockIdx.x * chunk;
    const int64_t c1   = c0 + chunk < V ? c0 + chunk : V;
    Best          s    = { -INFINITY, -INFINITY, 0x7fffffff };
    const bool    vec  = ((reinterpret_cast<uintptr_t>(l + c0) & 15) == 0) && (chunk % 4 == 0);
    if (vec) {
        const int64_t nv = (c1 - c0) / 4;
        const float4 * lv = reinterpret_cast<const float4 *>(l + c0);
        for (int64_t v0 = threadIdx.x; v0 < nv; v0 += 4 * blockDim.x) {
            float4 t[4];
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int64_t vi = v0 + (int64_t) u * blockDim.x;
                t[u]             = vi < nv ? __ldg(lv + vi) : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
            }
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int i = (int) (c0 + 4 * (v0 + (int64_t) u * blockDim.x));
                if (v0 + (int64_t) u * blockDim.x < nv) {
                    best_push(s, t[u].x, i);
                    best_push(s, t[u].y, i + 1);
                    best_push(s, t[u].z, i + 2);
                    best_push(s, t[u].w, i + 3);
                }
            }
        }
        for (int64_t i = c0 + nv * 4 + threadIdx.x; i < c1; i += blockDim.x) {
            best_push(s, l[i], (int) i);
        }
    } else {
        for (int64_t i = c0 + threadIdx.x; i < c1; i += blockDim.x) {
            best_push(s, l[i], (int) i);
        }
    }
    const Best b = block_best(s);
    __shared__ bool last;
    if (threadIdx.x == 0) {
        part[(int64_t) row * nblk + blockIdx.x] = make_float4(b.b1, b.b2, __int_as_float(b.i1), 0.0f);
        __threadfence();
        const int t = atomicAdd(ticket + row, 1);
        last        = (t == nblk - 1);
    }
    __syncthreads();
    if (!last) {
        return;
    }
    // last CTA of this row: merge every partial (L2 loads, bypassing L1)
    __threadfence();
    Best r = { -INFINITY, -INFINITY, 0x7fffffff };
    for (int k = threadIdx.x; k < nblk; k += blockDim.x) {
        const float4 p = __ldcg(part + (int64_t) row * nblk + k);
        best_merge(r, p.x, p.y, __float_as_int(p.z));
    }
    const Best f = block_best(r);
    if (threadIdx.x == 0) {
        ticket[row] = 0;
        ids[row]    = f.i1;
        if (margin) {
            margin[row] = f.b1 - f.b2;
        }
        if (pos_advance) {
            if (hist && hist_base) {
                const int64_t step             = pos_advance[row] - hist_base[row];
                hist[row * hist_stride + step] = f.i1;
                if (mhist) {
                    mhist[row * hist_stride + step] = f.b1 - f.b2;
                }
            }
            pos_advance[row] += 1;
        }
    }
}

static int argmax_blocks(int64_t V) {
    int64_t n = (V + 4095) / 4096;
    return (int) (n < 1 ? 1 : (n > 128 ? 128 : n));
}

static size_t ticket_bytes(int ticket_rows) {
    return ((size_t) ticket_rows * sizeof(int) + 255) / 256 * 256;
}

static acb_status launch_argmax(const float * logits, int64_t stride, int64_t V, int rows, int32_t * ids,
                                float * margin, int32_t * pos_advance, int32_t * hist, float * mhist,
                                int64_t hist_stride, const int32_t * hist_base, void * scratch, int ticket_rows,
                                int flags, cudaStream_t stream) {
    const int nblk  = argmax_blocks(V);
    int64_t   chunk = (V + nblk - 1) / nblk;
    chunk           = (chunk + 3) / 4 * 4;
    int *     ticket = reinterpret_cast<int *>(scratch);
    float4 *  part   = reinterpret_cast<float4 *>(reinterpret_cast<unsigned char *>(scratch) + ticket_bytes(ticket_rows));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim            = dim3((unsigned) nblk, (unsigned) rows);
    cfg.blockDim           = dim3(256);
    cfg.stream             = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id                                         = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    const bool pdl                                     = flags & 1;
    cfg.attrs                                          = pdl ? attr : nullptr;
    cfg.numAttrs                                       = pdl ? 1 : 0;
    cudaError_t e = pdl ? cudaLaunchKernelEx(&cfg, argmax_kernel<1>, logits, stride, V, chunk, ids, margin,
                                             pos_advance, hist, mhist, hist_stride, hist_base, part, ticket)
                        : cudaLaunchKernelEx(&cfg, argmax_kernel<0>, logits, stride, V, chunk, ids, margin,
                                             pos_advance, hist, mhist, hist_stride, hist_base, part, ticket);
    if (e != cudaSuccess) {
        set_last_cuda_error(e);
        return ACB_ERR_CUDA;
    }
    return ACB_OK;
}

}  // namespace acb

using namespace acb;

extern "C" size_t acb_argmax_scratch_bytes(int rows, int64_t V) {
    if (rows <= 0 || V <= 0) {
        return 0;
    }
    return ticket_bytes(ACB_ARGMAX_MAX_ROWS) + (size_t) rows * argmax_blocks(V) * sizeof(float4);
}

extern "C" acb_status acb_argmax(const float * logits, int64_t stride, int64_t V, int rows, int32_t * ids,
                                 float * margin, int32_t * pos_advance, int32_t * hist, float * mhist,
                                 int64_t hist_stride, const int32_t * hist_base, void * scratch, int flags,
                                 acb_stream_t stream) {
    if (!logits || !ids || !scratch || V <= 0 || V > INT32_MAX || rows <= 0 || rows > ACB_ARGMAX_MAX_ROWS ||
        stride < V || (hist && (!pos_advance || !hist_base))) {
        return ACB_ERR_INVALID_ARG;
    }
    if (reinterpret_cast<uintptr_t>(scratch) % 16 != 0) {
        return ACB_ERR_INVALID_ARG;
    }
    return launch_argmax(logits, stride, V, rows, ids, margin, pos_advance, hist, mhist, hist_stride, hist_base,
                         scratch, ACB_ARGMAX_MAX_ROWS, flags, (cudaStream_t) stream);
}

// ---- variant with library-owned scratch (no allocation by the caller or the library) ------------
//
// For callers that cannot allocate device memory at the point where they sample: a host that
// hands the whole device to its own memory pool (and forbids allocations behind its back), or a
// latency-critical decode thread that must not call cudaMalloc because it can synchronise the
// device. The scratch lives in a fixed array in this module's device memory instead; every
// device that loads the library holds it (ACB_ARGMAX_NOALLOC_MAX_ROWS rows) until the process
// exits.
namespace acb {
constexpr int    kNoallocRows  = ACB_ARGMAX_NOALLOC_MAX_ROWS;
constexpr size_t kNoallocTicketBytes = ((size_t) kNoallocRows * sizeof(int) + 255) / 256 * 256;
constexpr size_t kNoallocBytes       = kNoallocTicketBytes + (size_t) kNoallocRows * 128 * sizeof(float4);
static __device__ __align__(256) unsigned char g_argmax_scratch[kNoallocBytes];

// Device address of g_argmax_scratch per device ordinal. In host code the array's name is only a
// host-side stand-in, so the address is looked up once per device, with that device current.
static void *     g_scratch_addr[64];
static std::mutex g_scratch_mu;

void set_last_error(const std::string & e);

static acb_status noalloc_scratch(void ** out, cudaStream_t stream) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        set_last_error("acb_argmax_noalloc: no current CUDA device");
        return ACB_ERR_CUDA;
    }
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    if (!g_scratch_addr[dev]) {
        void *      p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_argmax_scratch);
        if (e != cudaSuccess || !p) {
            set_last_cuda_error(e);
            set_last_error("acb_argmax_noalloc: cudaGetSymbolAddress failed");
            return ACB_ERR_CUDA;
        }
        // The array is zero when the module loads; clearing the ticket counters once more on the
        // caller's stream orders the clear before this call's kernel whatever kind of stream
        // (blocking, non-blocking, per-thread default) the caller uses.
        e = cudaMemsetAsync(p, 0, kNoallocTicketBytes, stream);
        if (e != cudaSuccess) {
            set_last_cuda_error(e);
            set_last_error("acb_argmax_noalloc: clearing the scratch counters failed");
            return ACB_ERR_CUDA;
        }
        g_scratch_addr[dev] = p;
    }
    *out = g_scratch_addr[dev];
    return ACB_OK;
}
}  // namespace acb

extern "C" acb_status acb_argmax_noalloc(const float * logits, int64_t stride, int64_t V, int rows, int32_t * ids,
                                         float * margin, int32_t * pos_advance, int32_t * hist, float * mhist,
                                         int64_t hist_stride, const int32_t * hist_base, int flags,
                                         acb_stream_t stream) {
    if (!logits || !ids || V <= 0 || V > INT32_MAX || rows <= 0 || stride < V ||
        (hist && (!pos_advance || !hist_base))) {
        return ACB_ERR_INVALID_ARG;
    }
    if (rows > kNoallocRows) {
        set_last_error("acb_argmax_noalloc: rows exceeds ACB_ARGMAX_NOALLOC_MAX_ROWS (" +
                       std::to_string(kNoallocRows) + "); use acb_argmax with caller scratch");
        return ACB_ERR_UNSUPPORTED;
    }
    void *     scratch = nullptr;
    acb_status st      = noalloc_scratch(&scratch, (cudaStream_t) stream);
    if (st != ACB_OK) {
        return st;
    }
    return launch_argmax(logits, stride, V, rows, ids, margin, pos_advance, hist, mhist, hist_stride, hist_base,
                         scratch, kNoallocRows, flags, (cudaStream_t) stream);
}
