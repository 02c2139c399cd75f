// k_gemv.cu -- weight-streaming GEMV for batch-1..8 decode: y[m][n] = sum_k W[n][k] x[m][k]
// with W in GGUF Q8_0 / Q4_K / Q6_K blocks (quantised mul_mat of every decode linear,
// src/qwen3-lm.h:639-651,755).
//
// Design (HBM-bound; the weight bytes are the roofline):
//   - persistent CTAs, one per SM; each owns a contiguous row range and streams it through a
//     3-4 stage shared-memory ring filled by 1-D bulk copies (TMA engine) issued by a producer
//     warp; 8 consumer warps compute from shared memory (one output row per warp at a time);
//   - the activation is quantised inside the kernel exactly like ggml-CPU's quantised mul_mat
//     (Q8_0 blocks for Q8_0 weights, Q8_K for K-quants), and the dot products are integer
//     dp4a sums scaled per block, so each block's contribution equals the CPU's;
//   - a row's block terms are added in double and rounded to float once: the double sum of
//     float terms is exact unless they span ~20 binades, so the float result does not depend
//     on how lanes, warps and CTAs split the row (the oracle and the persistent decode step
//     give the same bits);
//   - fused prologues build the activation from its producer's output (RMSNorm*w, the sum of
//     attention split partials, or SwiGLU of a gate|up row); the epilogue optionally adds a
//     residual (ggml_add(hidden, out));
//   - programmatic dependent launch: weight prefetch is issued before griddepcontrol.wait, so
//     the next linear's weights stream while the previous kernel drains.
#include "common.cuh"
#include "ptx.cuh"

namespace acb {

enum { PRO_X = 0, PRO_RMSNORM = 1, PRO_SUM_SPLITS = 2, PRO_SWIGLU = 3 };
enum { EPI_STORE = 0, EPI_ADD = 1 };

constexpr int kConsumerWarps = 16;
constexpr int kThreads       = (kConsumerWarps + 1) * 32;
constexpr int kHdr           = 256;  // shared-memory header bytes (barriers, reduction)

struct GemvParams {
    const uint8_t * W;
    int64_t         N;
    int             K;
    int64_t         row_bytes;
    int             M;
    int             prologue;
    const float *   x;
    int64_t         x_stride;
    const float *   norm_w;
    float           eps;
    int             n_split;
    float *         y;
    int64_t         y_stride;
    int             epilogue;
    const float *   res;
    int64_t         res_stride;
    int             rows_per_cta;  // multiple of align_rows
    int             chunk_rows;    // rows per pipeline stage
    int             stage_bytes;   // 16-byte multiple >= chunk_rows * row_bytes
    int             stages;
    int *           err;
};

// ---- activation value of element k of row m under the prologue ------------------------------
// (raw loads first, `act_finish` after, so a round of loads is in flight at once)
template <int PRO> struct ActRaw {
    float a, b;
};

template <int PRO> __device__ __forceinline__ ActRaw<PRO> act_load(const GemvParams & p, int m, int k) {
    ActRaw<PRO>   r{ 0.0f, 0.0f };
    const float * row = p.x + (int64_t) m * p.x_stride;
    if (PRO == PRO_SUM_SPLITS) {
        // partials in double (the attention's split partials): summed, then rounded once
        const double * rd = reinterpret_cast<const double *>(p.x) + (int64_t) m * p.x_stride;
        double         s  = 0.0;
        for (int i = 0; i < p.n_split; i++) {
            s += rd[(int64_t) i * p.K + k];
        }
        r.a = (float) s;
    } else if (PRO == PRO_SWIGLU) {
        r.a = row[k];
        r.b = row[p.K + k];
    } else if (PRO == PRO_RMSNORM) {
        r.a = row[k];
        r.b = p.norm_w ? __ldg(p.norm_w + k) : 1.0f;
    } else {
        r.a = row[k];
    }
    return r;
}

template <int PRO> __device__ __forceinline__ float act_finish(const GemvParams & p, ActRaw<PRO> r, float sc) {
    if (PRO == PRO_RMSNORM) {
        const float v = __fmul_rn(r.a, sc);
        return p.norm_w ? __fmul_rn(v, r.b) : v;
    }
    if (PRO == PRO_SWIGLU) {
        return silu_times(r.a, r.b);
    }
    return r.a;
}

// RMSNorm scale of activation row m (PRO_RMSNORM), computed by the 256 consumer threads.
__device__ float rms_scale_block(const GemvParams & p, int m, double * red) {
    const int tid = threadIdx.x;
    double    ss  = 0.0;
    const float * row = p.x + (int64_t) m * p.x_stride;
    if ((p.K & 3) == 0 && (reinterpret_cast<uintptr_t>(row) & 15) == 0) {
        for (int k = tid * 4; k < p.K; k += kConsumerWarps * 32 * 4) {
            const float4 h = *reinterpret_cast<const float4 *>(row + k);
            ss += (double) __fmul_rn(h.x, h.x);
            ss += (double) __fmul_rn(h.y, h.y);
            ss += (double) __fmul_rn(h.z, h.z);
            ss += (double) __fmul_rn(h.w, h.w);
        }
    } else {
        for (int k = tid; k < p.K; k += kConsumerWarps * 32) {
            const float h = row[k];
            ss += (double) __fmul_rn(h, h);
        }
    }
    ss = warp_sum(ss);
    if ((tid & 31) == 0) {
        red[tid >> 5] = ss;
    }
    asm volatile("bar.sync 1, %0;" ::"r"(kConsumerWarps * 32));
    double t = 0.0;
    for (int w = 0; w < kConsumerWarps; w++) {
        t += red[w];
    }
    asm volatile("bar.sync 1, %0;" ::"r"(kConsumerWarps * 32));
    return rms_scale(t, p.K, p.eps);
}

// ---- activation quantisers (into shared memory) ----------------------------------------------
// 32 consecutive activation values of row m starting at k0 (16-byte loads when aligned).
template <int PRO>
__device__ __forceinline__ void act_block32(const GemvParams & p, int m, int k0, float sc, bool vec, float * v) {
    const float * row = p.x + (int64_t) m * p.x_stride;
    if (PRO == PRO_SUM_SPLITS) {
        const double * rd = reinterpret_cast<const double *>(p.x) + (int64_t) m * p.x_stride + k0;
        double         a[32];
#pragma unroll
        for (int e = 0; e < 32; e++) {
            a[e] = 0.0;
        }
        for (int s = 0; s < p.n_split; s++) {
#pragma unroll
            for (int e = 0; e < 32; e++) {
                a[e] += rd[(int64_t) s * p.K + e];
            }
        }
#pragma unroll
        for (int e = 0; e < 32; e++) {
            v[e] = (float) a[e];
        }
        return;
    }
    if (vec) {
        float4 a[8], b[8];
#pragma unroll
        for (int i = 0; i < 8; i++) {
            a[i] = *reinterpret_cast<const float4 *>(row + k0 + 4 * i);
        }
        if (PRO == PRO_SWIGLU) {
#pragma unroll
            for (int i = 0; i < 8; i++) {
                b[i] = *reinterpret_cast<const float4 *>(row + p.K + k0 + 4 * i);
            }
        } else if (PRO == PRO_RMSNORM && p.norm_w) {
#pragma unroll
            for (int i = 0; i < 8; i++) {
                b[i] = __ldg(reinterpret_cast<const float4 *>(p.norm_w + k0 + 4 * i));
            }
        }
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const float aa[4] = { a[i].x, a[i].y, a[i].z, a[i].w };
            const float bb[4] = { b[i].x, b[i].y, b[i].z, b[i].w };
#pragma unroll
            for (int e = 0; e < 4; e++) {
                ActRaw<PRO> r{ aa[e], (PRO == PRO_RMSNORM && !p.norm_w) ? 1.0f : bb[e] };
                v[4 * i + e] = act_finish<PRO>(p, r, sc);
            }
        }
    } else {
#pragma unroll
        for (int e = 0; e < 32; e++) {
            v[e] = act_finish<PRO>(p, act_load<PRO>(p, m, k0 + e), sc);
        }
    }
}

// Q8_0: qs int8 [M][K], d (f16-rounded, as float) [M][K/32]. One consumer thread quantises one
// whole 32-element block (no cross-lane reductions on the critical path).
template <int PRO>
__device__ void quantize_q8_0(const GemvParams & p, int8_t * xq, float * xd, double * red) {
    const int  tid = threadIdx.x;
    const int  nb  = p.K / 32;
    const bool vec = (p.x_stride % 4 == 0) && ((reinterpret_cast<uintptr_t>(p.x) & 15) == 0) &&
                     (p.norm_w == nullptr || (reinterpret_cast<uintptr_t>(p.norm_w) & 15) == 0);
    for (int m = 0; m < p.M; m++) {
        const float sc = PRO == PRO_RMSNORM ? rms_scale_block(p, m, red) : 1.0f;
        for (int b = tid; b < nb; b += kConsumerWarps * 32) {
            float v[32];
            act_block32<PRO>(p, m, b * 32, sc, vec, v);
            float amax = 0.0f;
#pragma unroll
            for (int e = 0; e < 32; e++) {
                amax = fmaxf(amax, fabsf(v[e]));
            }
            const float d  = amax / 127.0f;
            const float id = d != 0.0f ? 1.0f / d : 0.0f;
            uint32_t    w[8];
#pragma unroll
            for (int i = 0; i < 8; i++) {
                uint32_t u = 0;
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const int q = (int) roundf(__fmul_rn(v[4 * i + e], id));
                    u |= ((uint32_t) (q & 0xff)) << (8 * e);
                }
                w[i] = u;
            }
            uint4 * dst = reinterpret_cast<uint4 *>(xq + (int64_t) m * p.K + b * 32);
            dst[0]      = make_uint4(w[0], w[1], w[2], w[3]);
            dst[1]      = make_uint4(w[4], w[5], w[6], w[7]);
            xd[m * nb + b] = __half2float(__float2half_rn(d));
        }
    }
}

// Q8_K: qs int8 [M][K], d float [M][K/256], bsums int [M][K/16]. Eight consumer threads share
// a 256-element block, one 32-element part each; the signed maximum (first index on ties) is
// combined over the eight with shuffles.
template <int PRO>
__device__ void quantize_q8_K(const GemvParams & p, int8_t * xq, float * xd, int * xbs, double * red) {
    const int  tid  = threadIdx.x;
    const int  part = tid & 7;
    const int  nsb  = p.K / 256;
    const bool vec  = (p.x_stride % 4 == 0) && ((reinterpret_cast<uintptr_t>(p.x) & 15) == 0) &&
                     (p.norm_w == nullptr || (reinterpret_cast<uintptr_t>(p.norm_w) & 15) == 0);
    const int  rounds = (nsb + (kConsumerWarps * 4) - 1) / (kConsumerWarps * 4);
    for (int m = 0; m < p.M; m++) {
        const float sc = PRO == PRO_RMSNORM ? rms_scale_block(p, m, red) : 1.0f;
        for (int r = 0; r < rounds; r++) {
            const int  sb    = r * kConsumerWarps * 4 + (tid >> 3);
            const bool valid = sb < nsb;
            float      v[32];
            if (valid) {
                act_block32<PRO>(p, m, sb * 256 + part * 32, sc, vec, v);
            } else {
#pragma unroll
                for (int e = 0; e < 32; e++) {
                    v[e] = 0.0f;
                }
            }
            float amax = 0.0f, mx = 0.0f;
            int   idx  = 0x7fffffff;
#pragma unroll
            for (int e = 0; e < 32; e++) {
                const float a = fabsf(v[e]);
                if (a > amax) {  // first index of the largest magnitude wins
                    amax = a;
                    mx   = v[e];
                    idx  = part * 32 + e;
                }
            }
#pragma unroll
            for (int o = 1; o < 8; o <<= 1) {
                const float oa = __shfl_xor_sync(0xffffffffu, amax, o);
                const float om = __shfl_xor_sync(0xffffffffu, mx, o);
                const int   oi = __shfl_xor_sync(0xffffffffu, idx, o);
                if (oa > amax || (oa == amax && oi < idx)) {
                    amax = oa;
                    mx   = om;
                    idx  = oi;
                }
            }
            if (!valid) {
                continue;
            }
            uint32_t w[8];
            int      s0 = 0, s1 = 0;
            const float iscale = amax == 0.0f ? 0.0f : -127.0f / mx;
#pragma unroll
            for (int i = 0; i < 8; i++) {
                uint32_t u = 0;
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    int q = 0;
                    if (amax != 0.0f) {
                        q = __float2int_rn(__fmul_rn(iscale, v[4 * i + e]));
                        q = q < 127 ? q : 127;
                    }
                    if (i < 4) {
                        s0 += q;
                    } else {
                        s1 += q;
                    }
                    u |= ((uint32_t) (q & 0xff)) << (8 * e);
                }
                w[i] = u;
            }
            uint4 * dst = reinterpret_cast<uint4 *>(xq + (int64_t) m * p.K + sb * 256 + part * 32);
            dst[0]      = make_uint4(w[0], w[1], w[2], w[3]);
            dst[1]      = make_uint4(w[4], w[5], w[6], w[7]);
            xbs[m * (p.K / 16) + sb * 16 + part * 2]     = s0;
            xbs[m * (p.K / 16) + sb * 16 + part * 2 + 1] = s1;
            if (part == 0) {
                xd[m * nsb + sb] = amax == 0.0f ? 0.0f : 1.0f / iscale;
            }
        }
    }
}

// ---- per-row dot products from a shared-memory weight row ------------------------------------
template <int MT>
__device__ __forceinline__ void dot_q8_0(const uint8_t * wrow, const GemvParams & p, const int8_t * xq,
                                         const float * xd, double * acc) {
    const int lane = threadIdx.x & 31;
    const int np   = p.K / 64;  // block pairs (68 bytes, 4-byte aligned)
    for (int pr = lane; pr < np; pr += 32) {
        const uint32_t * w32 = reinterpret_cast<const uint32_t *>(wrow + 68 * pr);
        uint32_t         w[17];
#pragma unroll
        for (int j = 0; j < 17; j++) {
            w[j] = w32[j];
        }
        const float d0 = f16_bits_to_f((uint16_t) (w[0] & 0xffff));
        const float d1 = f16_bits_to_f((uint16_t) (w[8] >> 16));
        int         q0[8];
#pragma unroll
        for (int j = 0; j < 8; j++) {
            q0[j] = (int) __byte_perm(w[j], w[j + 1], 0x5432);
        }
#pragma unroll
        for (int m = 0; m < MT; m++) {
            if (m < p.M) {
                const int4 * xv = reinterpret_cast<const int4 *>(xq + (int64_t) m * p.K + 64 * pr);
                const int4   a = xv[0], b = xv[1], c = xv[2], e = xv[3];
                int          s0 = 0, s1 = 0;
                s0 = __dp4a(q0[0], a.x, s0);
                s0 = __dp4a(q0[1], a.y, s0);
                s0 = __dp4a(q0[2], a.z, s0);
                s0 = __dp4a(q0[3], a.w, s0);
                s0 = __dp4a(q0[4], b.x, s0);
                s0 = __dp4a(q0[5], b.y, s0);
                s0 = __dp4a(q0[6], b.z, s0);
                s0 = __dp4a(q0[7], b.w, s0);
                s1 = __dp4a((int) w[9], c.x, s1);
                s1 = __dp4a((int) w[10], c.y, s1);
                s1 = __dp4a((int) w[11], c.z, s1);
                s1 = __dp4a((int) w[12], c.w, s1);
                s1 = __dp4a((int) w[13], e.x, s1);
                s1 = __dp4a((int) w[14], e.y, s1);
                s1 = __dp4a((int) w[15], e.z, s1);
                s1 = __dp4a((int) w[16], e.w, s1);
                const float * dx = xd + m * (p.K / 32) + 2 * pr;
                acc[m] += (double) __fmul_rn((float) s0, __fmul_rn(d0, dx[0]));
                acc[m] += (double) __fmul_rn((float) s1, __fmul_rn(d1, dx[1]));
            }
        }
    }
}

// Q4_K: lane = (superblock slot lane/8, sub-block lane%8); the integer sums of the 8 sub-blocks
// of a superblock are combined exactly before the float scaling.
template <int MT>
__device__ __forceinline__ void dot_q4_K(const uint8_t * wrow, const GemvParams & p, const int8_t * xq,
                                         const float * xd, const int * xbs, double * acc) {
    const int lane = threadIdx.x & 31;
    const int sub  = lane & 7;
    const int nsb  = p.K / 256;
    for (int sb0 = 0; sb0 < nsb; sb0 += 4) {
        const int  sb    = sb0 + (lane >> 3);
        const bool valid = sb < nsb;
        const uint8_t * blk = wrow + (int64_t) (valid ? sb : 0) * 144;
        int             scv = 0, mnv = 0;
        uint32_t        qw[8];
        float           d = 0.0f, dmin = 0.0f;
        if (valid) {
            d                  = f16_bits_to_f(ld_u16(blk));
            dmin               = f16_bits_to_f(ld_u16(blk + 2));
            const uint8_t * sc = blk + 4;
            if (sub < 4) {
                scv = sc[sub] & 63;
                mnv = sc[sub + 4] & 63;
            } else {
                scv = (sc[sub + 4] & 0x0f) | ((sc[sub - 4] >> 6) << 4);
                mnv = (sc[sub + 4] >> 4) | ((sc[sub] >> 6) << 4);
            }
            const uint4 * q4 = reinterpret_cast<const uint4 *>(blk + 16 + (sub >> 1) * 32);
            const uint4   u0 = q4[0], u1 = q4[1];
            const int     sh = 4 * (sub & 1);
            qw[0]            = (u0.x >> sh) & 0x0F0F0F0Fu;
            qw[1]            = (u0.y >> sh) & 0x0F0F0F0Fu;
            qw[2]            = (u0.z >> sh) & 0x0F0F0F0Fu;
            qw[3]            = (u0.w >> sh) & 0x0F0F0F0Fu;
            qw[4]            = (u1.x >> sh) & 0x0F0F0F0Fu;
            qw[5]            = (u1.y >> sh) & 0x0F0F0F0Fu;
            qw[6]            = (u1.z >> sh) & 0x0F0F0F0Fu;
            qw[7]            = (u1.w >> sh) & 0x0F0F0F0Fu;
        }
#pragma unroll
        for (int m = 0; m < MT; m++) {
            if (m < p.M) {
                int isum = 0, imin = 0;
                if (valid) {
                    const int4 * xv  = reinterpret_cast<const int4 *>(xq + (int64_t) m * p.K + sb * 256 + sub * 32);
                    const int4   a   = xv[0], b = xv[1];
                    int          dot = 0;
                    dot              = __dp4a((int) qw[0], a.x, dot);
                    dot              = __dp4a((int) qw[1], a.y, dot);
                    dot              = __dp4a((int) qw[2], a.z, dot);
                    dot              = __dp4a((int) qw[3], a.w, dot);
                    dot              = __dp4a((int) qw[4], b.x, dot);
                    dot              = __dp4a((int) qw[5], b.y, dot);
                    dot              = __dp4a((int) qw[6], b.z, dot);
                    dot              = __dp4a((int) qw[7], b.w, dot);
                    const int * bs   = xbs + m * (p.K / 16) + sb * 16 + 2 * sub;
                    isum             = scv * dot;
                    imin             = mnv * (bs[0] + bs[1]);
                }
#pragma unroll
                for (int o = 1; o < 8; o <<= 1) {
                    isum += __shfl_xor_sync(0xffffffffu, isum, o);
                    imin += __shfl_xor_sync(0xffffffffu, imin, o);
                }
                if (valid && sub == 0) {
                    const float dx = xd[m * nsb + sb];
                    acc[m] += (double) __fmul_rn(__fmul_rn(d, dx), (float) isum);
                    acc[m] -= (double) __fmul_rn(__fmul_rn(dmin, dx), (float) imin);
                }
            }
        }
    }
}

// Q6_K: lane = (superblock slot lane/16, 16-element group lane%16). Unsigned 6-bit values are
// dotted and the -32 offset removed with the activation's 16-element sum (exact integers).
template <int MT>
__device__ __forceinline__ void dot_q6_K(const uint8_t * wrow, const GemvParams & p, const int8_t * xq,
                                         const float * xd, const int * xbs, double * acc) {
    const int lane = threadIdx.x & 31;
    const int g    = lane & 15;
    const int nsb  = p.K / 256;
    const int half = g >> 3, c = (g >> 1) & 3, l0 = (g & 1) * 16;
    for (int sb0 = 0; sb0 < nsb; sb0 += 2) {
        const int       sb    = sb0 + (lane >> 4);
        const bool      valid = sb < nsb;
        const uint8_t * blk   = wrow + (int64_t) (valid ? sb : 0) * 210;
        uint32_t        vw[4];
        int             scv = 0;
        float           d   = 0.0f;
        if (valid) {
            const uint16_t * ql = reinterpret_cast<const uint16_t *>(blk + half * 64 + (c & 1) * 32 + l0);
            const uint16_t * qh = reinterpret_cast<const uint16_t *>(blk + 128 + half * 32 + l0);
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const uint32_t lo4 = (uint32_t) ql[2 * j] | ((uint32_t) ql[2 * j + 1] << 16);
                const uint32_t hi4 = (uint32_t) qh[2 * j] | ((uint32_t) qh[2 * j + 1] << 16);
                const uint32_t lo  = (c & 2) ? ((lo4 >> 4) & 0x0F0F0F0Fu) : (lo4 & 0x0F0F0F0Fu);
                const uint32_t hi  = ((hi4 >> (2 * c)) & 0x03030303u) << 4;
                vw[j]              = lo | hi;
            }
            scv = (int) (int8_t) blk[192 + g];
            d   = f16_bits_to_f(ld_u16(blk + 208));
        }
#pragma unroll
        for (int m = 0; m < MT; m++) {
            if (m < p.M) {
                int isum = 0;
                if (valid) {
                    const int4 a   = *reinterpret_cast<const int4 *>(xq + (int64_t) m * p.K + sb * 256 + g * 16);
                    int        dot = 0;
                    dot            = __dp4a((int) vw[0], a.x, dot);
                    dot            = __dp4a((int) vw[1], a.y, dot);
                    dot            = __dp4a((int) vw[2], a.z, dot);
                    dot            = __dp4a((int) vw[3], a.w, dot);
                    isum           = scv * (dot - 32 * xbs[m * (p.K / 16) + sb * 16 + g]);
                }
#pragma unroll
                for (int o = 1; o < 16; o <<= 1) {
                    isum += __shfl_xor_sync(0xffffffffu, isum, o);
                }
                if (valid && g == 0) {
                    acc[m] += (double) __fmul_rn(__fmul_rn(d, xd[m * nsb + sb]), (float) isum);
                }
            }
        }
    }
}

template <int QT, int MT, int PRO>
__global__ void __launch_bounds__(kThreads, 1) gemv_kernel(const GemvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // shared layout: [barriers][reduction][x quants][x scales][x bsums][stages]
    // header: full[8] @0, empty[8] @64, reduction doubles[8] @128, activation from 256
    uint64_t * full  = reinterpret_cast<uint64_t *>(smem);
    uint64_t * empty = full + 8;
    double *   red   = reinterpret_cast<double *>(smem + 128);
    int8_t *   xq    = reinterpret_cast<int8_t *>(smem + kHdr);
    const int  xq_bytes = (MT * p.K + 15) / 16 * 16;
    float *    xd       = reinterpret_cast<float *>(smem + kHdr + xq_bytes);
    const int  nscale   = QT == ACB_TYPE_Q8_0 ? p.K / 32 : p.K / 256;
    const int  xd_bytes = (MT * nscale * 4 + 15) / 16 * 16;
    int *      xbs      = reinterpret_cast<int *>(smem + kHdr + xq_bytes + xd_bytes);
    const int  bs_bytes = QT == ACB_TYPE_Q8_0 ? 0 : (MT * (p.K / 16) * 4 + 15) / 16 * 16;
    const int  st_off   = (kHdr + xq_bytes + xd_bytes + bs_bytes + 127) / 128 * 128;
    uint8_t *  stages   = smem + st_off;

    const int64_t row0   = (int64_t) blockIdx.x * p.rows_per_cta;
    const int64_t row1   = row0 + p.rows_per_cta < p.N ? row0 + p.rows_per_cta : p.N;
    const int     nrows  = row1 > row0 ? (int) (row1 - row0) : 0;
    const int     nchunk = (nrows + p.chunk_rows - 1) / p.chunk_rows;

    if (threadIdx.x == 0) {
        for (int s = 0; s < p.stages; s++) {
            ptx::mbar_init(&full[s], 1);
            ptx::mbar_init(&empty[s], kConsumerWarps);
        }
        ptx::fence_mbar_init();
    }
    __syncthreads();
    ptx::grid_dep_launch();

    if (warp == kConsumerWarps) {
        // producer: stream this CTA's rows (independent of the previous kernel's output)
        if (lane == 0) {
            const uint64_t pol = ptx::policy_evict_first();
            for (int i = 0; i < nchunk; i++) {
                const int s = i % p.stages;
                if (i >= p.stages && !ptx::mbar_wait(&empty[s], ((i / p.stages) - 1) & 1)) {
                    if (p.err) {
                        atomicOr(p.err, ACB_DEVERR_TIMEOUT);
                    }
                    break;
                }
                const int64_t r     = row0 + (int64_t) i * p.chunk_rows;
                const int     rows  = (int) ((row1 - r) < p.chunk_rows ? (row1 - r) : p.chunk_rows);
                const uint32_t bytes = (uint32_t) (((int64_t) rows * p.row_bytes + 15) / 16 * 16);
                ptx::mbar_arrive_expect_tx(&full[s], bytes);
                ptx::bulk_g2s_stream(stages + (int64_t) s * p.stage_bytes, p.W + r * p.row_bytes, bytes, &full[s],
                                     pol);
            }
        }
        return;
    }

    // consumers: activation prologue once the previous kernel's output is visible
    ptx::grid_dep_wait();
    if (QT == ACB_TYPE_Q8_0) {
        quantize_q8_0<PRO>(p, xq, xd, red);
    } else {
        quantize_q8_K<PRO>(p, xq, xd, xbs, red);
    }
    asm volatile("bar.sync 1, %0;" ::"r"(kConsumerWarps * 32));

    for (int i = 0; i < nchunk; i++) {
        const int s = i % p.stages;
        if (!ptx::mbar_wait(&full[s], (i / p.stages) & 1)) {
            if (lane == 0 && p.err) {
                atomicOr(p.err, ACB_DEVERR_TIMEOUT);
            }
            return;
        }
        const int64_t   r     = row0 + (int64_t) i * p.chunk_rows;
        const int       rows  = (int) ((row1 - r) < p.chunk_rows ? (row1 - r) : p.chunk_rows);
        const uint8_t * stage = stages + (int64_t) s * p.stage_bytes;
        for (int rr = warp; rr < rows; rr += kConsumerWarps) {
            double acc[MT];
#pragma unroll
            for (int m = 0; m < MT; m++) {
                acc[m] = 0.0;
            }
            const uint8_t * wrow = stage + (int64_t) rr * p.row_bytes;
            if (QT == ACB_TYPE_Q8_0) {
                dot_q8_0<MT>(wrow, p, xq, xd, acc);
            } else if (QT == ACB_TYPE_Q4_K) {
                dot_q4_K<MT>(wrow, p, xq, xd, xbs, acc);
            } else {
                dot_q6_K<MT>(wrow, p, xq, xd, xbs, acc);
            }
#pragma unroll
            for (int m = 0; m < MT; m++) {
                if (m < p.M) {
                    // lanes that hold terms: every lane (Q8_0), lanes 0/8/16/24 (Q4_K: one per
                    // superblock slot), lanes 0/16 (Q6_K); the others hold zero
                    double t = acc[m];
                    if (QT == ACB_TYPE_Q8_0) {
                        t = warp_sum(t);
                    } else {
                        if (QT == ACB_TYPE_Q4_K) {
                            t += __shfl_xor_sync(0xffffffffu, t, 8);
                        }
                        t += __shfl_xor_sync(0xffffffffu, t, 16);
                    }
                    const float v = (float) t;
                    if (lane == 0) {
                        const int64_t n  = r + rr;
                        float *       yp = p.y + (int64_t) m * p.y_stride + n;
                        *yp = p.epilogue == EPI_ADD ? __fadd_rn(p.res[(int64_t) m * p.res_stride + n], v) : v;
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) {
            ptx::mbar_arrive(&empty[s]);
        }
    }
}

// ---- Q8_0 repacked into 16-row MMA tiles (ACB_TYPE_Q8_0_TILES) ------------------------------
// Tile t (rows 16t .. 16t+15), K-block b (32 columns) is 544 bytes: 512 bytes of int8 weights in
// the order of the A operand of mma.m16n8k32 (lane l = 4g + q holds rows g and g+8, columns
// 4q..4q+3 and 16+4q..16+4q+3, 16 bytes) followed by eight words (d[16t+g] | d[16t+g+8] << 16) of
// f16 block scales. Tiles are stored tile-major, blocks in K order: the same bytes as Q8_0 rows.
constexpr int kTileBytes = 544;

__device__ __forceinline__ void mma_s8_16832(const uint4 & a, int b0, int b1, int * c) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%12,%13};"
        : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
        : "r"(a.x), "r"(a.y), "r"(a.z), "r"(a.w), "r"(b0), "r"(b1), "r"(0), "r"(0), "r"(0), "r"(0));
}

// One warp per (tile, 544-byte block): repack from GGUF Q8_0 rows.
__global__ void __launch_bounds__(256) q8_0_to_tiles_kernel(const uint8_t * __restrict__ src, uint8_t * __restrict__ dst,
                                                            int64_t n_tiles, int nb) {
    const int     lane = threadIdx.x & 31;
    const int64_t item = (int64_t) blockIdx.x * 8 + (threadIdx.x >> 5);
    if (item >= n_tiles * nb) {
        return;
    }
    const int64_t t = item / nb;
    const int     b = (int) (item - t * nb);
    const int     g = lane >> 2, q = lane & 3;
    const int64_t rb = (int64_t) nb * 34;
    auto          qs = [&](int r, int k) -> uint32_t {  // 4 int8 of row r at columns k..k+3 of block b
        const uint8_t * blk = src + (16 * t + r) * rb + (int64_t) b * 34 + 2;
        return (uint32_t) blk[k] | ((uint32_t) blk[k + 1] << 8) | ((uint32_t) blk[k + 2] << 16) |
               ((uint32_t) blk[k + 3] << 24);
    };
    uint8_t * o = dst + item * kTileBytes;
    reinterpret_cast<uint4 *>(o)[lane] = make_uint4(qs(g, 4 * q), qs(g + 8, 4 * q), qs(g, 16 + 4 * q), qs(g + 8, 16 + 4 * q));
    if (lane < 8) {
        const uint8_t * d0 = src + (16 * t + lane) * rb + (int64_t) b * 34;
        const uint8_t * d1 = src + (16 * t + lane + 8) * rb + (int64_t) b * 34;
        reinterpret_cast<uint32_t *>(o + 512)[lane] = (uint32_t) d0[0] | ((uint32_t) d0[1] << 8) |
                                                      ((uint32_t) d1[0] << 16) | ((uint32_t) d1[1] << 24);
    }
}

// Tensor-core GEMV over tiled Q8_0 weights: each CTA streams a contiguous range of tiles through
// the shared-memory ring in stages of bs K-blocks (whole tiles when K <= 2048); warp w takes
// blocks w, w+16, ... of a stage and issues one mma.m16n8k32 (int8, int32 sums exact) per block,
// scaling each block's sums by d_w * d_x (ggml's vec_dot_q8_0_q8_0 arithmetic per block) and
// adding the terms in double; at the end of a tile the 16 warps' partials are added in double
// and rounded to float once.
template <int MT, int PRO>
__global__ void __launch_bounds__(kThreads, 1) gemv_tiles_kernel(const GemvParams p, int bs) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint64_t * full  = reinterpret_cast<uint64_t *>(smem);
    uint64_t * empty = full + 8;
    double *   red   = reinterpret_cast<double *>(smem + 128);
    int8_t *   xq    = reinterpret_cast<int8_t *>(smem + kHdr);
    const int  nb       = p.K / 32;
    const int  xq_bytes = (MT * p.K + 15) / 16 * 16;
    float *    xd       = reinterpret_cast<float *>(smem + kHdr + xq_bytes);
    const int  xd_bytes = (MT * nb * 4 + 15) / 16 * 16;
    double *   tred     = reinterpret_cast<double *>(smem + kHdr + xq_bytes + xd_bytes);  // [16 warps][32][4]
    const int  st_off   = (kHdr + xq_bytes + xd_bytes + kConsumerWarps * 32 * 4 * 8 + 127) / 128 * 128;
    uint8_t *  stages   = smem + st_off;

    const int64_t n_tiles = p.N / 16;
    const int64_t t0      = (int64_t) blockIdx.x * p.rows_per_cta;  // rows_per_cta holds tiles per CTA here
    const int64_t t1      = t0 + p.rows_per_cta < n_tiles ? t0 + p.rows_per_cta : n_tiles;
    const int     parts   = nb / bs;
    const int     nstage  = t1 > t0 ? (int) ((t1 - t0) * parts) : 0;
    const int     sbytes  = bs * kTileBytes;

    if (threadIdx.x == 0) {
        for (int s = 0; s < p.stages; s++) {
            ptx::mbar_init(&full[s], 1);
            ptx::mbar_init(&empty[s], kConsumerWarps);
        }
        ptx::fence_mbar_init();
    }
    __syncthreads();
    ptx::grid_dep_launch();

    if (warp == kConsumerWarps) {
        if (lane == 0) {
            const uint64_t pol = ptx::policy_evict_first();
            const uint8_t * src = p.W + t0 * (int64_t) nb * kTileBytes;
            for (int i = 0; i < nstage; i++) {
                const int s = i % p.stages;
                if (i >= p.stages && !ptx::mbar_wait(&empty[s], ((i / p.stages) - 1) & 1)) {
                    if (p.err) {
                        atomicOr(p.err, ACB_DEVERR_TIMEOUT);
                    }
                    break;
                }
                ptx::mbar_arrive_expect_tx(&full[s], (uint32_t) sbytes);
                ptx::bulk_g2s_stream(stages + (int64_t) s * p.stage_bytes, src + (int64_t) i * sbytes,
                                     (uint32_t) sbytes, &full[s], pol);
            }
        }
        return;
    }

    ptx::grid_dep_wait();
    quantize_q8_0<PRO>(p, xq, xd, red);
    asm volatile("bar.sync 1, %0;" ::"r"(kConsumerWarps * 32));

    const int g = lane >> 2, q = lane & 3;
    // this lane's batch column of the B operand (n = g) and of the accumulators (n = 2q, 2q + 1)
    const int8_t * xb  = xq + (int64_t) (g < MT ? g : 0) * p.K;
    const bool     bok = g < p.M;
    double         acc[4] = { 0.0, 0.0, 0.0, 0.0 };  // (row g, n 2q), (g, 2q+1), (g+8, 2q), (g+8, 2q+1)
    for (int i = 0; i < nstage; i++) {
        const int s = i % p.stages;
        if (!ptx::mbar_wait(&full[s], (i / p.stages) & 1)) {
            if (lane == 0 && p.err) {
                atomicOr(p.err, ACB_DEVERR_TIMEOUT);
            }
            return;
        }
        const int       part  = i % parts;
        const uint8_t * stage = stages + (int64_t) s * p.stage_bytes;
        for (int bl = warp; bl < bs; bl += kConsumerWarps) {
            const int     b  = part * bs + bl;
            const uint4   a  = *reinterpret_cast<const uint4 *>(stage + bl * kTileBytes + lane * 16);
            const uint32_t dw = *reinterpret_cast<const uint32_t *>(stage + bl * kTileBytes + 512 + g * 4);
            const int     b0 = bok ? *reinterpret_cast<const int *>(xb + 32 * b + 4 * q) : 0;
            const int     b1 = bok ? *reinterpret_cast<const int *>(xb + 32 * b + 16 + 4 * q) : 0;
            int           c[4];
            mma_s8_16832(a, b0, b1, c);
            const float dr[2] = { f16_bits_to_f((uint16_t) (dw & 0xffff)), f16_bits_to_f((uint16_t) (dw >> 16)) };
#pragma unroll
            for (int j = 0; j < 2; j++) {
                const int n = 2 * q + j;
                if (n < p.M) {
                    const float dx = xd[n * nb + b];
#pragma unroll
                    for (int r = 0; r < 2; r++) {
                        acc[2 * r + j] += (double) __fmul_rn((float) c[2 * r + j], __fmul_rn(dr[r], dx));
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) {
            ptx::mbar_arrive(&empty[s]);
        }
        if (part == parts - 1) {
            // tile complete: add the 16 warps' partials in warp order and store
            reinterpret_cast<double2 *>(tred + (warp * 32 + lane) * 4)[0] = make_double2(acc[0], acc[1]);
            reinterpret_cast<double2 *>(tred + (warp * 32 + lane) * 4)[1] = make_double2(acc[2], acc[3]);
            asm volatile("bar.sync 1, %0;" ::"r"(kConsumerWarps * 32));
            if (warp == 0) {
                double v[4] = { 0.0, 0.0, 0.0, 0.0 };
                for (int w = 0; w < kConsumerWarps; w++) {
                    const double2 t0 = reinterpret_cast<const double2 *>(tred + (w * 32 + lane) * 4)[0];
                    const double2 t1 = reinterpret_cast<const double2 *>(tred + (w * 32 + lane) * 4)[1];
                    v[0] += t0.x;
                    v[1] += t0.y;
                    v[2] += t1.x;
                    v[3] += t1.y;
                }
                const int64_t tile = t0 + i / parts;
#pragma unroll
                for (int r = 0; r < 2; r++) {
#pragma unroll
                    for (int j = 0; j < 2; j++) {
                        const int n = 2 * q + j;
                        if (n < p.M) {
                            const int64_t row = tile * 16 + g + 8 * r;
                            float *       yp  = p.y + (int64_t) n * p.y_stride + row;
                            const float   val = (float) v[2 * r + j];
                            *yp = p.epilogue == EPI_ADD ? __fadd_rn(p.res[(int64_t) n * p.res_stride + row], val) : val;
                        }
                    }
                }
            }
            asm volatile("bar.sync 1, %0;" ::"r"(kConsumerWarps * 32));
            acc[0] = acc[1] = acc[2] = acc[3] = 0.0;
        }
    }
}

template <int MT, int PRO>
static acb_status launch_gemv_tiles(GemvParams p, bool pdl, cudaStream_t st) {
    const int     sms     = num_sms();
    const int     nb      = p.K / 32;
    const int64_t n_tiles = p.N / 16;
    // K-blocks per stage: the largest divisor of nb up to 64 (whole tiles for K <= 2048)
    int bs = 1;
    for (int d = 1; d <= 64 && d <= nb; d++) {
        if (nb % d == 0) {
            bs = d;
        }
    }
    const int64_t per_cta = (n_tiles + sms - 1) / sms;
    const int     grid    = (int) ((n_tiles + per_cta - 1) / per_cta);
    p.rows_per_cta        = (int) per_cta;  // tiles per CTA
    p.stage_bytes         = bs * kTileBytes;
    const int xq_bytes = (MT * p.K + 15) / 16 * 16;
    const int xd_bytes = (MT * nb * 4 + 15) / 16 * 16;
    const int st_off   = (kHdr + xq_bytes + xd_bytes + kConsumerWarps * 32 * 4 * 8 + 127) / 128 * 128;
    const int64_t nstage = per_cta * (nb / bs);
    int           stages = nstage < 6 ? (int) nstage : 6;
    const int64_t smem_cap = nstage > 4 ? 200 * 1024 : 110 * 1024;
    while (stages > 1 && st_off + (int64_t) stages * p.stage_bytes > smem_cap) {
        stages--;
    }
    p.stages = stages < 1 ? 1 : stages;
    const int64_t smem = st_off + (int64_t) p.stages * p.stage_bytes;
    if (smem > 220 * 1024) {
        return ACB_ERR_UNSUPPORTED;
    }
    auto kern = gemv_tiles_kernel<MT, PRO>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim            = dim3((unsigned) grid);
    cfg.blockDim           = dim3(kThreads);
    cfg.dynamicSmemBytes   = (size_t) smem;
    cfg.stream             = st;
    cudaLaunchAttribute attr[1];
    attr[0].id                                         = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs                                          = pdl ? attr : nullptr;
    cfg.numAttrs                                       = pdl ? 1 : 0;
    cudaError_t e                                      = cudaLaunchKernelEx(&cfg, kern, p, bs);
    if (e != cudaSuccess) {
        set_last_cuda_error(e);
        return ACB_ERR_CUDA;
    }
    return ACB_OK;
}

template <int PRO>
static acb_status dispatch_tiles_mp(const GemvParams & p, bool pdl, cudaStream_t st) {
    if (p.M <= 1) {
        return launch_gemv_tiles<1, PRO>(p, pdl, st);
    }
    if (p.M <= 2) {
        return launch_gemv_tiles<2, PRO>(p, pdl, st);
    }
    if (p.M <= 4) {
        return launch_gemv_tiles<4, PRO>(p, pdl, st);
    }
    return launch_gemv_tiles<8, PRO>(p, pdl, st);
}

static acb_status dispatch_tiles(const GemvParams & p, bool pdl, cudaStream_t st) {
    switch (p.prologue) {
        case PRO_RMSNORM:
            return dispatch_tiles_mp<PRO_RMSNORM>(p, pdl, st);
        case PRO_SUM_SPLITS:
            return dispatch_tiles_mp<PRO_SUM_SPLITS>(p, pdl, st);
        case PRO_SWIGLU:
            return dispatch_tiles_mp<PRO_SWIGLU>(p, pdl, st);
        default:
            return dispatch_tiles_mp<PRO_X>(p, pdl, st);
    }
}

template <int QT, int MT, int PRO>
static acb_status launch_gemv(GemvParams p, bool pdl, cudaStream_t st) {
    const int sms = num_sms();
    // rows must start on 16-byte boundaries for the bulk copies
    int align = 1;
    while ((p.row_bytes * align) % 16 != 0) {
        align++;
    }
    // ~32 KB stages, 3-4 deep, leaving room for a second CTA of the next kernel (PDL)
    int chunk = (int) (32768 / p.row_bytes);
    chunk     = chunk < 1 ? 1 : chunk;
    chunk     = (chunk + align - 1) / align * align;
    int64_t per_cta = (p.N + sms - 1) / sms;
    per_cta         = (per_cta + align - 1) / align * align;
    if (chunk > per_cta) {
        chunk = (int) per_cta;
    }
    p.rows_per_cta = (int) per_cta;
    p.chunk_rows   = chunk;
    p.stage_bytes  = (int) (((int64_t) chunk * p.row_bytes + 15) / 16 * 16);
    const int nscale   = QT == ACB_TYPE_Q8_0 ? p.K / 32 : p.K / 256;
    const int xq_bytes = (MT * p.K + 15) / 16 * 16;
    const int xd_bytes = (MT * nscale * 4 + 15) / 16 * 16;
    const int bs_bytes = QT == ACB_TYPE_Q8_0 ? 0 : (MT * (p.K / 16) * 4 + 15) / 16 * 16;
    const int st_off   = (kHdr + xq_bytes + xd_bytes + bs_bytes + 127) / 128 * 128;
    const int64_t chunks_per_cta = (per_cta + chunk - 1) / chunk;
    // deep rings for long row ranges (bytes in flight cover the loaded-HBM latency), shallow
    // ones for short ranges so a CTA of the next kernel can co-reside
    int stages = chunks_per_cta < 6 ? (int) chunks_per_cta : 6;
    const int64_t smem_cap = chunks_per_cta > 4 ? 200 * 1024 : 110 * 1024;
    while (stages > 1 && st_off + (int64_t) stages * p.stage_bytes > smem_cap) {
        stages--;
    }
    p.stages = stages < 1 ? 1 : stages;
    const int64_t smem = st_off + (int64_t) p.stages * p.stage_bytes;
    if (smem > 220 * 1024) {
        return ACB_ERR_UNSUPPORTED;
    }
    const int grid = (int) ((p.N + per_cta - 1) / per_cta);
    auto      kern = gemv_kernel<QT, MT, PRO>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);

    cudaLaunchConfig_t cfg = {};
    cfg.gridDim            = dim3((unsigned) grid);
    cfg.blockDim           = dim3(kThreads);
    cfg.dynamicSmemBytes   = (size_t) smem;
    cfg.stream             = st;
    cudaLaunchAttribute attr[1];
    attr[0].id                                         = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs                                          = pdl ? attr : nullptr;
    cfg.numAttrs                                       = pdl ? 1 : 0;
    cudaError_t e                                      = cudaLaunchKernelEx(&cfg, kern, p);
    if (e != cudaSuccess) {
        set_last_cuda_error(e);
        return ACB_ERR_CUDA;
    }
    return ACB_OK;
}

template <int QT, int PRO>
static acb_status dispatch_mp(const GemvParams & p, bool pdl, cudaStream_t st) {
    if (p.M <= 1) {
        return launch_gemv<QT, 1, PRO>(p, pdl, st);
    }
    if (p.M <= 2) {
        return launch_gemv<QT, 2, PRO>(p, pdl, st);
    }
    if (p.M <= 4) {
        return launch_gemv<QT, 4, PRO>(p, pdl, st);
    }
    return launch_gemv<QT, 8, PRO>(p, pdl, st);
}

// ---- BF16 / F16 weights (the unquantised GGUFs convert.py writes) -------------------------------
// ggml converts the activation to the weight's type and multiplies in f32: a bf16 x bf16 or
// f16 x f16 product is exact in f32, so the products are added in double and rounded to f32 once
// -- the same canonical rule as the quantised rows, independent of how a row is split. The block's
// 512 threads first write every activation row (prologue applied, rounded to the weight type) to
// shared memory; then each warp takes kHalfRowsPerWarp weight rows, its lanes streaming 16-byte
// runs of 8 weights, with a double butterfly at the end of each row.
constexpr int kHalfRowsPerWarp = 4;

template <int WT, int MT, int PRO>
__global__ void __launch_bounds__(kConsumerWarps * 32) gemv_half_kernel(const GemvParams p) {
    extern __shared__ __align__(16) uint8_t gh_smem[];
    using et        = typename io<WT>::t;
    et *      xs    = reinterpret_cast<et *>(gh_smem);  // [MT][K]
    __shared__ double red[kConsumerWarps];
    const int tid   = threadIdx.x;
    const int warp  = tid >> 5, lane = tid & 31;
    ptx::grid_dep_wait();
    const bool vec = (p.x_stride % 4 == 0) && ((reinterpret_cast<uintptr_t>(p.x) & 15) == 0) &&
                     (p.norm_w == nullptr || (reinterpret_cast<uintptr_t>(p.norm_w) & 15) == 0);
    for (int m = 0; m < p.M; m++) {
        const float sc = PRO == PRO_RMSNORM ? rms_scale_block(p, m, red) : 1.0f;
        for (int b = tid; b < p.K / 32; b += kConsumerWarps * 32) {
            float v[32];
            act_block32<PRO>(p, m, b * 32, sc, vec, v);
            et * d = xs + (int64_t) m * p.K + b * 32;
#pragma unroll
            for (int e = 0; e < 32; e++) {
                d[e] = io<WT>::from_f(v[e]);
            }
        }
    }
    __syncthreads();
    const int64_t row0 = ((int64_t) blockIdx.x * kConsumerWarps + warp) * kHalfRowsPerWarp;
    for (int r = 0; r < kHalfRowsPerWarp; r++) {
        const int64_t n = row0 + r;
        if (n >= p.N) {
            break;
        }
        const et * wr = reinterpret_cast<const et *>(p.W + n * p.row_bytes);
        double     acc[MT];
#pragma unroll
        for (int m = 0; m < MT; m++) {
            acc[m] = 0.0;
        }
        for (int k = lane * 8; k < p.K; k += 256) {
            union {
                uint4 u;
                et    e[8];
            } w;
            w.u = __ldcs(reinterpret_cast<const uint4 *>(wr + k));
            float wf[8];
#pragma unroll
            for (int e = 0; e < 8; e++) {
                wf[e] = io<WT>::to_f(w.e[e]);
            }
#pragma unroll
            for (int m = 0; m < MT; m++) {
                if (m < p.M) {
                    union {
                        uint4 u;
                        et    e[8];
                    } x;
                    x.u = *reinterpret_cast<const uint4 *>(xs + (int64_t) m * p.K + k);
#pragma unroll
                    for (int e = 0; e < 8; e++) {
                        acc[m] += (double) __fmul_rn(wf[e], io<WT>::to_f(x.e[e]));
                    }
                }
            }
        }
#pragma unroll
        for (int m = 0; m < MT; m++) {
            acc[m] = warp_sum(acc[m]);
        }
        if (lane == 0) {
            for (int m = 0; m < p.M; m++) {
                float v = (float) acc[m];
                if (p.epilogue == EPI_ADD) {
                    v = __fadd_rn(p.res[(int64_t) m * p.res_stride + n], v);
                }
                p.y[(int64_t) m * p.y_stride + n] = v;
            }
        }
    }
    ptx::grid_dep_launch();
}

template <int WT, int MT, int PRO>
static acb_status launch_half(const GemvParams & p, bool pdl, cudaStream_t st) {
    const size_t smem = (size_t) p.M * p.K * 2;
    auto         kern = gemv_half_kernel<WT, MT, PRO>;
    if (smem > 48 * 1024 && cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem) !=
                                cudaSuccess) {
        return ACB_ERR_UNSUPPORTED;
    }
    const int64_t rows_per_cta = (int64_t) kConsumerWarps * kHalfRowsPerWarp;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim            = dim3((unsigned) ((p.N + rows_per_cta - 1) / rows_per_cta));
    cfg.blockDim           = dim3(kConsumerWarps * 32);
    cfg.dynamicSmemBytes   = smem;
    cfg.stream             = st;
    cudaLaunchAttribute attr[1];
    attr[0].id                                         = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs                                          = pdl ? attr : nullptr;
    cfg.numAttrs                                       = pdl ? 1 : 0;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, p);
    if (e != cudaSuccess) {
        set_last_cuda_error(e);
        return ACB_ERR_CUDA;
    }
    return ACB_OK;
}

template <int WT, int PRO>
static acb_status dispatch_half_mp(const GemvParams & p, bool pdl, cudaStream_t st) {
    if (p.M <= 1) {
        return launch_half<WT, 1, PRO>(p, pdl, st);
    }
    if (p.M <= 2) {
        return launch_half<WT, 2, PRO>(p, pdl, st);
    }
    if (p.M <= 4) {
        return launch_half<WT, 4, PRO>(p, pdl, st);
    }
    return launch_half<WT, 8, PRO>(p, pdl, st);
}

template <int WT>
static acb_status dispatch_half(const GemvParams & p, bool pdl, cudaStream_t st) {
    switch (p.prologue) {
        case PRO_RMSNORM:
            return dispatch_half_mp<WT, PRO_RMSNORM>(p, pdl, st);
        case PRO_SUM_SPLITS:
            return dispatch_half_mp<WT, PRO_SUM_SPLITS>(p, pdl, st);
        case PRO_SWIGLU:
            return dispatch_half_mp<WT, PRO_SWIGLU>(p, pdl, st);
        default:
            return dispatch_half_mp<WT, PRO_X>(p, pdl, st);
    }
}

template <int QT>
static acb_status dispatch_m(const GemvParams & p, bool pdl, cudaStream_t st) {
    switch (p.prologue) {
        case PRO_RMSNORM:
            return dispatch_mp<QT, PRO_RMSNORM>(p, pdl, st);
        case PRO_SUM_SPLITS:
            return dispatch_mp<QT, PRO_SUM_SPLITS>(p, pdl, st);
        case PRO_SWIGLU:
            return dispatch_mp<QT, PRO_SWIGLU>(p, pdl, st);
        default:
            return dispatch_mp<QT, PRO_X>(p, pdl, st);
    }
}

}  // namespace acb

using namespace acb;

extern "C" acb_status acb_gemv(const void * W, int w_type, int64_t N, int64_t K, int M, int prologue, const float * x,
                               int64_t x_stride, const float * norm_w, float eps, int n_split, float * y,
                               int64_t y_stride, int epilogue, const float * res, int64_t res_stride, int flags,
                               int * err_flag, acb_stream_t stream) {
    if (!W || !x || !y || N <= 0 || K <= 0 || M <= 0 || M > 8 || y_stride < N) {
        return ACB_ERR_INVALID_ARG;
    }
    if (prologue < PRO_X || prologue > PRO_SWIGLU || (prologue == PRO_SUM_SPLITS && n_split < 1)) {
        return ACB_ERR_INVALID_ARG;
    }
    if (epilogue == EPI_ADD && !res) {
        return ACB_ERR_INVALID_ARG;
    }
    if (reinterpret_cast<uintptr_t>(W) % 16 != 0) {
        return ACB_ERR_INVALID_ARG;
    }
    GemvParams p = {};
    p.W          = (const uint8_t *) W;
    p.N          = N;
    p.K          = (int) K;
    p.M          = M;
    p.prologue   = prologue;
    p.x          = x;
    p.x_stride   = x_stride;
    p.norm_w     = norm_w;
    p.eps        = eps;
    p.n_split    = n_split;
    p.y          = y;
    p.y_stride   = y_stride;
    p.epilogue   = epilogue;
    p.res        = res;
    p.res_stride = res_stride;
    p.err        = err_flag;
    const bool   pdl = (flags & 1) != 0;
    cudaStream_t st  = (cudaStream_t) stream;
    switch (w_type) {
        case ACB_TYPE_Q8_0:
            if (K % 256 != 0) {
                return ACB_ERR_UNSUPPORTED;
            }
            p.row_bytes = K / 32 * 34;
            return dispatch_m<ACB_TYPE_Q8_0>(p, pdl, st);
        case ACB_TYPE_Q8_0_TILES:
            if (K % 256 != 0 || N % 16 != 0) {
                return ACB_ERR_UNSUPPORTED;
            }
            p.row_bytes = K / 32 * 34;
            return dispatch_tiles(p, pdl, st);
        case ACB_TYPE_Q4_K:
            if (K % 256 != 0) {
                return ACB_ERR_UNSUPPORTED;
            }
            p.row_bytes = K / 256 * 144;
            return dispatch_m<ACB_TYPE_Q4_K>(p, pdl, st);
        case ACB_TYPE_Q6_K:
            if (K % 256 != 0) {
                return ACB_ERR_UNSUPPORTED;
            }
            p.row_bytes = K / 256 * 210;
            return dispatch_m<ACB_TYPE_Q6_K>(p, pdl, st);
        case ACB_TYPE_BF16:
        case ACB_TYPE_F16:
            if (K % 256 != 0 || (size_t) M * K * 2 > 200 * 1024) {
                return ACB_ERR_UNSUPPORTED;
            }
            p.row_bytes = K * 2;
            return w_type == ACB_TYPE_BF16 ? dispatch_half<ACB_TYPE_BF16>(p, pdl, st)
                                           : dispatch_half<ACB_TYPE_F16>(p, pdl, st);
        default:
            return ACB_ERR_UNSUPPORTED;
    }
}

extern "C" acb_status acb_q8_0_to_tiles(const void * src, void * dst, int64_t N, int64_t K, acb_stream_t stream) {
    if (!src || !dst || N <= 0 || K <= 0) {
        return ACB_ERR_INVALID_ARG;
    }
    if (N % 16 != 0 || K % 32 != 0 || reinterpret_cast<uintptr_t>(dst) % 16 != 0) {
        return ACB_ERR_UNSUPPORTED;
    }
    const int64_t items = (N / 16) * (K / 32);
    q8_0_to_tiles_kernel<<<(unsigned) ((items + 7) / 8), 256, 0, (cudaStream_t) stream>>>(
        reinterpret_cast<const uint8_t *>(src), reinterpret_cast<uint8_t *>(dst), N / 16, (int) (K / 32));
    return launch_status();
}
