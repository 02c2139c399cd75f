// k_sample.cu -- LM token sampling on the device: sample_top_k_p (src/sampling.h:30-133) with the
// targeted CFG combine and the EOS + audio-code compaction of the phase-2 loop in front of it
// (src/pipeline-lm.cpp:470-500), one CTA per sequence.
//
// Per row: (1) build the compacted row x[c] (optional CFG x = u + cfg * (x - u)), scaled by
// 1 / temperature; temperature <= 0 is greedy (first maximum). (2) top_k: the k-th largest value by
// a 4-pass MSB-first radix select over order-preserving 32-bit keys; values below it become -inf.
// (3) top_p: full-row softmax (max, sum of exp), tokens below max - 16 become -inf, and the
// nucleus is found by a probability-weighted radix select: a token with probability q is kept when
// the probability mass strictly above q is below top_p (the shift-right cumulative sum of the
// sorted list). Bin masses are 2^-48 fixed-point integers, so the selection does not depend on the
// order of the block's atomics. (4) softmax of the survivors and the multinomial draw r = u * sum
// with the caller's uniform u (the mt19937 draw stays on the host): the first index whose running
// sum reaches r, from per-thread contiguous chunks and a fixed-order scan.
//
// Every reduction has a fixed order, so a row's result depends only on its inputs. The reference
// adds in index order on one CPU thread; sums here are grouped differently, which can move the
// choice only when r (or top_p) falls within rounding of a boundary.
#include "common.cuh"

namespace acb {
namespace {

constexpr int kSThreads = 1024;
constexpr int kSWarps   = kSThreads / 32;
constexpr int kSReps    = 8;  // histogram replicas (warp w uses replica w % 8)

struct SampleArgs {
    const float *   logits;
    int64_t         ld;
    const float *   uncond;
    int64_t         uld;
    float           cfg;
    int             col0;  // compact column 0 reads this column (-1: none)
    int64_t         off;   // then span columns starting here
    int             span;
    int             Vc;
    float           temp;
    float           top_p;
    int             top_k;
    const float *   u;
    float *         work;
    int64_t         wld;
    int32_t *       idx;
};

__device__ __forceinline__ uint32_t fkey(float f) {
    const uint32_t b = __float_as_uint(f);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ float kval(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// block-wide max of v (every thread gets it)
__device__ float block_max(float v, float * red) {
    for (int o = 16; o > 0; o >>= 1) {
        v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    }
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) {
        red[w] = v;
    }
    __syncthreads();
    v = l < kSWarps ? red[l] : -INFINITY;
    for (int o = 16; o > 0; o >>= 1) {
        v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    }
    return v;
}

// block-wide f32 sum in a fixed order: lanes by xor butterfly, then warps 0..31 the same way
__device__ float block_sum(float v, float * red) {
    for (int o = 16; o > 0; o >>= 1) {
        v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    }
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) {
        red[w] = v;
    }
    __syncthreads();
    v = l < kSWarps ? red[l] : 0.0f;
    for (int o = 16; o > 0; o >>= 1) {
        v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    }
    return v;
}

// Shared scratch of the selection passes.
struct SelSmem {
    unsigned long long hist[kSReps][256];
    unsigned long long bins[256];
    unsigned long long above;
    int                bin, found;
};

// The smallest key T such that every element with key >= T has less than `target` mass strictly
// above it (among the elements), by four MSB-first passes over 8 key bits. kv(c) gives element c's
// key and mass (mass 0: the element does not take part). With mass 1 and target k this is the k-th
// largest key (top_k); with fixed-point probabilities and target top_p the nucleus boundary. 0 when
// the whole mass is below target (everything kept).
template <class KV>
__device__ uint32_t select_threshold(int Vc, KV kv, unsigned long long target, SelSmem & sm) {
    uint32_t           prefix = 0, mask = 0;
    unsigned long long above  = 0;
    const int          w = threadIdx.x >> 5, l = threadIdx.x & 31;
    for (int shift = 24; shift >= 0; shift -= 8) {
        for (int i = threadIdx.x; i < kSReps * 256; i += kSThreads) {
            (&sm.hist[0][0])[i] = 0ull;
        }
        __syncthreads();
        unsigned long long * h = sm.hist[w % kSReps];
        for (int c = threadIdx.x; c < Vc; c += kSThreads) {
            uint32_t           key;
            unsigned long long m;
            kv(c, key, m);
            if (m && (key & mask) == prefix) {
                atomicAdd(&h[(key >> shift) & 255u], m);
            }
        }
        __syncthreads();
        if (threadIdx.x < 256) {
            unsigned long long s = 0;
#pragma unroll
            for (int r = 0; r < kSReps; r++) {
                s += sm.hist[r][threadIdx.x];
            }
            sm.bins[threadIdx.x] = s;
        }
        __syncthreads();
        if (w == 0) {
            // lane l holds bins 255 - 8l down to 248 - 8l: an inclusive scan over lanes runs over
            // the bins from the top
            unsigned long long ls = 0;
#pragma unroll
            for (int j = 0; j < 8; j++) {
                ls += sm.bins[255 - 8 * l - j];
            }
            unsigned long long inc = ls;
            for (int o = 1; o < 32; o <<= 1) {
                const unsigned long long t = __shfl_up_sync(0xffffffffu, inc, o);
                if (l >= o) {
                    inc += t;
                }
            }
            const unsigned long long exc = inc - ls;
            const bool               hit = above + exc < target && above + inc >= target;
            if (hit) {
                unsigned long long s = above + exc;
                for (int j = 0; j < 8; j++) {
                    const int b = 255 - 8 * l - j;
                    if (s + sm.bins[b] >= target) {
                        sm.bin   = b;
                        sm.above = s;
                        break;
                    }
                    s += sm.bins[b];
                }
            }
            const unsigned any = __ballot_sync(0xffffffffu, hit);
            if (l == 0) {
                sm.found = any != 0;
            }
        }
        __syncthreads();
        const bool found = sm.found;
        const int  b     = sm.bin;
        above            = sm.above;
        __syncthreads();  // sm is rewritten by the next pass
        if (!found) {
            return prefix;  // the range's whole mass stays below target: keep all of it
        }
        prefix |= (uint32_t) b << shift;
        mask |= 255u << shift;
    }
    return prefix;
}

__global__ void __launch_bounds__(kSThreads) sample_kernel(const SampleArgs a) {
    __shared__ SelSmem sm;
    __shared__ float   red[kSWarps];
    __shared__ float   red2[kSWarps];
    __shared__ int     ired[kSWarps];
    __shared__ float   sm_excl[kSThreads];
    const int          row = blockIdx.x;
    const int          Vc  = a.Vc;
    const float *      lg  = a.logits + row * a.ld;
    const float *      un  = a.uncond ? a.uncond + row * a.uld : nullptr;
    float *            x   = a.work + row * a.wld;
    const bool         greedy   = !(a.temp > 0.0f);
    const float        inv_temp = greedy ? 1.0f : __fdiv_rn(1.0f, a.temp);

    // (1) the compacted, CFG-combined, temperature-scaled row
    for (int c = threadIdx.x; c < Vc; c += kSThreads) {
        const int64_t col = a.col0 >= 0 ? (c == 0 ? (int64_t) a.col0 : a.off + c - 1) : a.off + c;
        float         v   = lg[col];
        if (un) {
            const float u = un[col];
            v             = __fadd_rn(u, __fmul_rn(a.cfg, __fsub_rn(v, u)));
        }
        x[c] = greedy ? v : __fmul_rn(v, inv_temp);
    }
    __syncthreads();
    if (greedy) {  // std::max_element: the first maximum
        float bv = -INFINITY;
        int   bi = 0x7fffffff;
        for (int c = threadIdx.x; c < Vc; c += kSThreads) {
            const float v = x[c];
            if (v > bv) {
                bv = v;
                bi = c;
            }
        }
        const float m = block_max(bv, red);
        int         i = bv == m ? bi : 0x7fffffff;
        for (int o = 16; o > 0; o >>= 1) {
            i = min(i, __shfl_xor_sync(0xffffffffu, i, o));
        }
        if ((threadIdx.x & 31) == 0) {
            ired[threadIdx.x >> 5] = i;
        }
        __syncthreads();
        if (threadIdx.x < 32) {
            i = ired[threadIdx.x];
            for (int o = 16; o > 0; o >>= 1) {
                i = min(i, __shfl_xor_sync(0xffffffffu, i, o));
            }
            if (threadIdx.x == 0) {
                a.idx[row] = i == 0x7fffffff ? 0 : i;
            }
        }
        return;
    }

    // (2) top_k: values below the k-th largest become -inf
    if (a.top_k > 0 && a.top_k < Vc) {
        const uint32_t T = select_threshold(
            Vc, [&](int c, uint32_t & key, unsigned long long & m) { key = fkey(x[c]); m = 1ull; },
            (unsigned long long) a.top_k, sm);
        const float thr = kval(T);
        for (int c = threadIdx.x; c < Vc; c += kSThreads) {
            if (x[c] < thr) {
                x[c] = -INFINITY;
            }
        }
        __syncthreads();
    }

    // (3) top_p: softmax over the row, cut at max - 16, nucleus by probability mass
    if (a.top_p > 0.0f && a.top_p < 1.0f) {
        float mx = -INFINITY;
        for (int c = threadIdx.x; c < Vc; c += kSThreads) {
            mx = fmaxf(mx, x[c]);
        }
        mx      = block_max(mx, red);
        float s = 0.0f;
        for (int c = threadIdx.x; c < Vc; c += kSThreads) {
            s = __fadd_rn(s, expf(__fsub_rn(x[c], mx)));
        }
        s                   = block_sum(s, red2);
        const float inv_sum = __fdiv_rn(1.0f, s);
        const float cutoff  = __fsub_rn(mx, 16.0f);
        for (int c = threadIdx.x; c < Vc; c += kSThreads) {
            if (x[c] < cutoff) {
                x[c] = -INFINITY;
            }
        }
        __syncthreads();
        // probability mass in units of 2^-48 (exact integer sums in any order)
        auto pk = [&](int c, uint32_t & key, unsigned long long & m) {
            const float v = x[c];
            if (v == -INFINITY) {
                key = 0;
                m   = 0;
                return;
            }
            const float p = __fmul_rn(expf(__fsub_rn(v, mx)), inv_sum);
            key           = __float_as_uint(p);
            m             = (unsigned long long) __fmul_rz(p, 281474976710656.0f);
        };
        const unsigned long long target = (unsigned long long) ((double) a.top_p * 281474976710656.0);
        const uint32_t           T      = select_threshold(Vc, pk, target > 0 ? target : 1ull, sm);
        for (int c = threadIdx.x; c < Vc; c += kSThreads) {
            uint32_t           key;
            unsigned long long m;
            pk(c, key, m);
            if (m && key < T) {
                x[c] = -INFINITY;
            }
        }
        __syncthreads();
    }

    // (4) softmax of the survivors and the multinomial draw: the first index whose running sum
    // reaches r = u * sum, over per-thread contiguous chunks
    float mx = -INFINITY;
    for (int c = threadIdx.x; c < Vc; c += kSThreads) {
        mx = fmaxf(mx, x[c]);
    }
    mx           = block_max(mx, red);
    const int C  = (Vc + kSThreads - 1) / kSThreads;
    const int c0 = min(Vc, threadIdx.x * C), c1 = min(Vc, c0 + C);
    float     cs = 0.0f;
    for (int c = c0; c < c1; c++) {
        cs = __fadd_rn(cs, expf(__fsub_rn(x[c], mx)));
    }
    // exclusive scan of the chunk sums in thread order (warp scans, then the warp totals)
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    float     inc = cs;
    for (int o = 1; o < 32; o <<= 1) {
        const float t = __shfl_up_sync(0xffffffffu, inc, o);
        if (l >= o) {
            inc = __fadd_rn(t, inc);
        }
    }
    __syncthreads();
    if (l == 31) {
        red[w] = inc;
    }
    __syncthreads();
    if (w == 0) {
        float wi = red[l];
        for (int o = 1; o < 32; o <<= 1) {
            const float t = __shfl_up_sync(0xffffffffu, wi, o);
            if (l >= o) {
                wi = __fadd_rn(t, wi);
            }
        }
        red2[l] = wi;  // inclusive over warps
    }
    __syncthreads();
    // every thread's exclusive prefix in one array: thread t's chunk covers (excl[t], excl[t + 1]],
    // the last one up to the total, so the intervals tile (0, total] without rounding gaps
    const float wbase = w == 0 ? 0.0f : red2[w - 1];
    const float prev  = __shfl_up_sync(0xffffffffu, inc, 1);  // monotone in thread order
    const float excl  = l == 0 ? wbase : __fadd_rn(wbase, prev);
    sm_excl[threadIdx.x] = excl;
    __syncthreads();
    const float total = __fadd_rn(sm_excl[kSThreads - 1], threadIdx.x == kSThreads - 1 ? cs : 0.0f);
    if (threadIdx.x == kSThreads - 1) {
        ired[0] = __float_as_int(total);
    }
    __syncthreads();
    const float r    = __fmul_rn(a.u[row], __int_as_float(ired[0]));
    const float incl = threadIdx.x + 1 < kSThreads ? sm_excl[threadIdx.x + 1] : __int_as_float(ired[0]);
    __syncthreads();
    if (threadIdx.x == 0) {
        ired[1] = 0;  // r <= 0 (u = 0): the first element already reaches it
    }
    __syncthreads();
    if (c0 < c1 && excl < r && r <= incl) {
        // the running sum from this chunk's start, as the reference adds it; if rounding keeps it
        // short of r the crossing is this chunk's last token with mass
        float acc = excl;
        int   hit = -1, last = c0;
        for (int c = c0; c < c1; c++) {
            const float e = expf(__fsub_rn(x[c], mx));
            if (e > 0.0f) {
                last = c;
            }
            acc = __fadd_rn(acc, e);
            if (acc >= r) {
                hit = c;
                break;
            }
        }
        ired[1] = hit >= 0 ? hit : last;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        a.idx[row] = ired[1];
    }
}

}  // namespace
}  // namespace acb

using namespace acb;

extern "C" size_t acb_sample_work_bytes(int rows, int Vc) {
    return rows > 0 && Vc > 0 ? (size_t) rows * (size_t) Vc * 4 : 0;
}

extern "C" acb_status acb_sample_top_k_p(const float * logits, int64_t ld, const float * uncond, int64_t uld,
                                         float cfg_scale, int col0, int64_t span_off, int span_len, int rows,
                                         float temperature, float top_p, int top_k, const float * u, float * work,
                                         int32_t * idx, acb_stream_t stream) {
    if (!logits || !work || !idx || rows <= 0 || span_len < 0 || span_off < 0 || (temperature > 0.0f && !u)) {
        return ACB_ERR_INVALID_ARG;
    }
    const int Vc = (col0 >= 0 ? 1 : 0) + span_len;
    if (Vc <= 0 || ld < span_off + span_len || (col0 >= 0 && col0 >= ld) || (uncond && uld < ld)) {
        return ACB_ERR_INVALID_ARG;
    }
    SampleArgs a;
    a.logits = logits;
    a.ld     = ld;
    a.uncond = uncond;
    a.uld    = uld;
    a.cfg    = cfg_scale;
    a.col0   = col0;
    a.off    = span_off;
    a.span   = span_len;
    a.Vc     = Vc;
    a.temp   = temperature;
    a.top_p  = top_p;
    a.top_k  = top_k;
    a.u      = u;
    a.work   = work;
    a.wld    = Vc;
    a.idx    = idx;
    sample_kernel<<<rows, kSThreads, 0, (cudaStream_t) stream>>>(a);
    return launch_status();
}
