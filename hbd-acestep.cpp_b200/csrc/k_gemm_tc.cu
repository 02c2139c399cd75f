// k_gemm_tc.cu -- tensor-core GEMM for the dense prefill / DiT linears (src/dit-graph.h:36-49 and
// every ggml_mul_mat of dit_ggml_build_layer at M = tokens):
//     C[m][n] = epilogue( sum_k A[m][k] * B[n][k] ),  A, B bf16 or f16 K-major, fp32 accumulation.
//
// sm_100a design (persistent, 6 warps, no multicast loads). Two variants of one kernel:
//   single CTA  work tile 128x256: A 128x64 + B 256x64 per stage (48 KB), 4-stage ring;
//   CTA pair    work tile 256x256 on a cluster of two CTAs (tcgen05 cta_group::2): each CTA loads
//               its own 128 rows of A and its half (128 rows) of B per stage (32 KB), 6-stage ring;
//               the leader CTA issues M=256 MMAs that read B from both CTAs' shared memory and
//               write each CTA's 128 rows into that CTA's TMEM. Per SM this moves 2/3 of the
//               shared-memory bytes of the single-CTA tile for the same tensor work.
//   warp 0      TMA producer (128-byte swizzle), completion on an mbarrier per stage (the
//               leader's, for a pair: both CTAs' bytes count there);
//   warp 1      allocates 512 TMEM columns (two 128x256 fp32 accumulators); one elected thread
//               (the leader's, for a pair) issues tcgen05.mma (K=16, kind::f16, bf16 or f16
//               inputs) and releases ring stages / publishes finished accumulators with
//               tcgen05.commit (to both CTAs of a pair);
//   warps 2..5  epilogue: tcgen05.ld 32 columns at a time from their TMEM lane quarter, fused
//               bias / residual / DiT gated residual, f32, bf16 or f16 stores; the accumulator is
//               handed back (to the leader, for a pair) so the next tile's MMA overlaps it.
// Every mbarrier wait is bounded; on a timeout the kernel records ACB_DEVERR_TIMEOUT, stops, and
// still frees its TMEM (both CTAs of a pair meet at a cluster barrier first).
#include <cuda.h>

#include <cstdlib>

#include "common.cuh"
#include "ptx.cuh"
#include "tc.cuh"

namespace acb {

constexpr int kBN = 256, kBK = 64;
constexpr int kGemmThreads = 192;
constexpr int kTmemCols    = 512;
constexpr int kStgPitch    = 36;                       // floats per staged row (16-byte aligned, conflict-free)
constexpr int kStgBytes    = 4 * 32 * kStgPitch * 4;   // one 32 x 32 f32 block per epilogue warp

template <bool PAIR> struct GemmCfg {
    static constexpr int      kTileM  = PAIR ? 256 : 128;  // output rows per work tile
    static constexpr int      kRowsB  = PAIR ? 128 : 256;  // B rows loaded per CTA
    static constexpr int      kATile  = 128 * kBK * 2;     // 16 KB
    static constexpr int      kBTile  = kRowsB * kBK * 2;
    static constexpr int      kStage  = kATile + kBTile;
    static constexpr int      kStages = PAIR ? 6 : 4;
    static constexpr uint32_t kTx     = (PAIR ? 2 : 1) * kStage;  // bytes landing per stage
    static constexpr size_t   kSmem   = (size_t) kStages * kStage + kStgBytes + 1024 + 256;
};

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
    // SwiGLU epilogue (swiglu != 0): B is [gate rows F | up rows F]; output tile t covers features
    // [128 nt, 128 nt + 128) (accumulator columns 0..127 gate, 128..255 up); C receives the
    // down projection's activation operand: silu(gate) * up quantised as vec type sw_vt, layout
    // sw_layout (PLAIN [M][F] or GEMM_A [M][3F]), 16-bit, ldc elements per row
    int           swiglu, sw_vt, sw_layout;
    int64_t       F;
    // QKV epilogue (qkv != 0): output columns are nq q heads, nk k heads, then nk v heads of 128;
    // q/k heads get RMSNorm (qn / kn) and, with a rope table, NeoX RoPE at pos[m], and go to the
    // f16 planes qk [M][qk_ld] (hi; lo qk_lo elements further when nonzero); v heads go transposed
    // to vt[((b*nk + hv)*128 + d)*vt_ld + t] (m = b*seq + t; lo vt_lo further when nonzero)
    int             qkv, nq, nk, max_pos;
    const float *   qn;
    const float *   kn;
    float           eps;
    const int32_t * pos;
    const float *   rope;
    int64_t         seq;
    uint16_t *      qk;
    int64_t         qk_ld, qk_lo;
    uint16_t *      vt;
    int64_t         vt_ld, vt_lo;
    int           group_m;  // tile order: groups of group_m m-tiles, n-tiles outer within a group, m inner
    int           splits;  // split-K factor; > 1: raw partials to ws, epilogue by splitk_reduce_kernel
    int           kps;     // k-tiles per split
    float *       ws;      // [splits][M][N] f32 partial accumulators
    // implicit 1-D convolution (conv_c != 0): A's tensor map covers the activation [M][conv_c] and
    // k-tile kt reads tap (kt*64) / conv_c, channels (kt*64) % conv_c of rows m + tap*conv_dil -
    // conv_pad (rows outside [0, M) arrive as zeros from the TMA bounds fill)
    int           conv_c, conv_dil, conv_pad;
};

// A's coordinates of k-tile kt for a tile starting at row ma (plain GEMM or implicit convolution)
__device__ __forceinline__ void a_coords(const GemmArgs & g, int kt, int ma, int & x, int & y) {
    x = kt * kBK;
    y = ma;
    if (g.conv_c) {
        const int tap = x / g.conv_c;
        x -= tap * g.conv_c;
        y += tap * g.conv_dil - g.conv_pad;
    }
}

// up to 4 consecutive columns of one row: one vector access when all 4 are in range and aligned.
// Values travel in a float4 and every index is static, so nothing is placed in local memory.
__device__ __forceinline__ float f4_get(const float4 & v, int j) {
    return j == 0 ? v.x : j == 1 ? v.y : j == 2 ? v.z : v.w;
}

template <int T> __device__ __forceinline__ void store_cols(void * C, int64_t off, float4 v, int ncol) {
    using et = typename io<T>::t;
    et * dst = reinterpret_cast<et *>(C) + off;
    if (ncol == 4 && (reinterpret_cast<uintptr_t>(dst) & (4 * sizeof(et) - 1)) == 0) {
        if constexpr (T == ACB_TYPE_F32) {
            *reinterpret_cast<float4 *>(dst) = v;
        } else {
            union {
                uint2 u;
                et    e[4];
            } pk;
            pk.e[0]                          = io<T>::from_f(v.x);
            pk.e[1]                          = io<T>::from_f(v.y);
            pk.e[2]                          = io<T>::from_f(v.z);
            pk.e[3]                          = io<T>::from_f(v.w);
            *reinterpret_cast<uint2 *>(dst) = pk.u;
        }
    } else {
#pragma unroll
        for (int j = 0; j < 4; j++) {
            if (j < ncol) {
                dst[j] = io<T>::from_f(f4_get(v, j));
            }
        }
    }
}

__device__ __forceinline__ float4 load_cols(const float * src, int ncol) {
    if (ncol == 4 && (reinterpret_cast<uintptr_t>(src) & 15) == 0) {
        return *reinterpret_cast<const float4 *>(src);
    }
    return make_float4(ncol > 0 ? src[0] : 0.0f, ncol > 1 ? src[1] : 0.0f, ncol > 2 ? src[2] : 0.0f,
                       ncol > 3 ? src[3] : 0.0f);
}

// C[off .. off+ncol) = v in C's type
__device__ __forceinline__ void store_c(const GemmArgs & g, int64_t off, float4 v, int ncol) {
    if (g.c_type == ACB_TYPE_F32) {
        store_cols<ACB_TYPE_F32>(g.C, off, v, ncol);
    } else if (g.c_type == ACB_TYPE_BF16) {
        store_cols<ACB_TYPE_BF16>(g.C, off, v, ncol);
    } else {
        store_cols<ACB_TYPE_F16>(g.C, off, v, ncol);
    }
}

// The residual of one 32 x 32 chunk as this lane reads it in the plain epilogue (rows it*4 + sub,
// columns cc .. cc+3), loaded ahead of the chunk's stores: res may alias C, so loads issued inside
// the store loop would each wait for the previous store (one memory round trip per 4 rows).
__device__ __forceinline__ void load_res_chunk(const GemmArgs & g, int64_t m_base, int64_t nc, int sub, int cc,
                                               float4 (&rv)[8]) {
    const int64_t n    = nc + cc;
    const int     ncol = (nc < g.N && n < g.N) ? (g.N - n < 4 ? (int) (g.N - n) : 4) : 0;
#pragma unroll
    for (int it = 0; it < 8; it++) {
        const int64_t m = m_base + it * 4 + sub;
        rv[it]          = (m < g.M && ncol > 0) ? load_cols(g.res + m * g.ldr + n, ncol) : make_float4(0, 0, 0, 0);
    }
}

// SwiGLU epilogue of one warp: its 32 rows (m_base + lane) of the tile, features f0 .. f0+127.
// Per 32-feature group: silu(gate) * up (ggml_swiglu, the unfused acb_act_quant_swiglu
// arithmetic), then one Q8_0 block per row (d = amax / 127 stored as f16, q = round(y / d)) or a
// plain 16-bit rounding, then the 16-bit operand planes (GEMM_A: hi at f, hi at F + f, lo at 2F +
// f; PLAIN: hi at f), staged through shared memory so each row segment is written whole.
__device__ __forceinline__ void swiglu_epilogue(const GemmArgs & g, uint32_t tacc, int64_t m_base, int64_t f0,
                                                int lane, float * stg) {
    const int64_t m  = m_base + lane;
    const bool    bf = g.sw_vt == ACB_TYPE_BF16;
    uint32_t *    sw = reinterpret_cast<uint32_t *>(stg);  // [32 rows][20 words]: 16 words of row data
#pragma unroll 1
    for (int c = 0; c < 4; c++) {
        uint32_t rg[32], ru[32];
        tmem_ld32(tacc + (uint32_t) (c * 32), rg);
        tmem_ld32(tacc + (uint32_t) (128 + c * 32), ru);
        if (m_base >= g.M) {
            continue;  // warp-uniform
        }
        const int64_t f = f0 + c * 32;
        float         y[32];
#pragma unroll
        for (int j = 0; j < 32; j++) {
            float gv = __uint_as_float(rg[j]), uv = __uint_as_float(ru[j]);
            if (g.bias) {
                gv = __fadd_rn(gv, g.bias[f + j]);
                uv = __fadd_rn(uv, g.bias[g.F + f + j]);
            }
            y[j] = silu_times(gv, uv);
        }
        if (g.sw_vt == ACB_TYPE_Q8_0) {
            float amax = 0.0f;
#pragma unroll
            for (int j = 0; j < 32; j++) {
                amax = fmaxf(amax, fabsf(y[j]));
            }
            const float d  = __fdiv_rn(amax, 127.0f);
            const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
            const float dh = __half2float(__float2half_rn(d));  // the block stores d as f16
#pragma unroll
            for (int j = 0; j < 32; j++) {
                y[j] = __fmul_rn(dh, (float) (int) roundf(__fmul_rn(y[j], id)));
            }
        }
        const int nplanes = g.sw_layout == ACB_LAYOUT_GEMM_A ? 2 : 1;
        for (int pl = 0; pl < nplanes; pl++) {
            // this row's 32 values of the plane as 16 packed words
#pragma unroll
            for (int j = 0; j < 32; j += 8) {
                uint32_t wv[4];
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const float a = y[j + 2 * e], b = y[j + 2 * e + 1];
                    if (bf) {
                        __nv_bfloat162 hb = __floats2bfloat162_rn(a, b);
                        if (pl == 1) {
                            const float2 hf2 = __bfloat1622float2(hb);
                            hb               = __floats2bfloat162_rn(__fsub_rn(a, hf2.x), __fsub_rn(b, hf2.y));
                        }
                        wv[e] = *reinterpret_cast<uint32_t *>(&hb);
                    } else {
                        __half2 hh = __floats2half2_rn(a, b);
                        if (pl == 1) {
                            const float2 hf2 = __half22float2(hh);
                            hh               = __floats2half2_rn(__fsub_rn(a, hf2.x), __fsub_rn(b, hf2.y));
                        }
                        wv[e] = *reinterpret_cast<uint32_t *>(&hh);
                    }
                }
                *reinterpret_cast<uint4 *>(sw + lane * 20 + j / 2) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
            }
            __syncwarp();
            // 8 rows per pass, 4 lanes x 16 bytes per row
#pragma unroll
            for (int it = 0; it < 4; it++) {
                const int     rr = it * 8 + (lane >> 2), part = lane & 3;
                const int64_t mr = m_base + rr;
                if (mr < g.M) {
                    const uint4 v   = *reinterpret_cast<const uint4 *>(sw + rr * 20 + part * 4);
                    uint16_t *  dst = reinterpret_cast<uint16_t *>(g.C) + mr * g.ldc + f + part * 8;
                    if (pl == 0) {
                        *reinterpret_cast<uint4 *>(dst) = v;
                        if (g.sw_layout == ACB_LAYOUT_GEMM_A) {
                            *reinterpret_cast<uint4 *>(dst + g.F) = v;
                        }
                    } else {
                        *reinterpret_cast<uint4 *>(dst + 2 * g.F) = v;
                    }
                }
            }
            __syncwarp();
        }
    }
    (void) m;
}

// (m-tile, n-tile) of tile t: tiles run in groups of group_m m-tiles; within a group the m-tile
// varies fastest, so a wave of resident CTAs touches a compact block of A rows and B rows
__device__ __forceinline__ void tile_mn(int64_t t, int64_t m_tiles, int64_t n_tiles, int group_m, int64_t & mt,
                                        int64_t & nt) {
    const int64_t gsz = (int64_t) group_m * n_tiles;
    const int64_t grp = t / gsz, idx = t - grp * gsz;
    const int64_t m0  = grp * group_m;
    const int64_t gm  = m_tiles - m0 < group_m ? m_tiles - m0 : group_m;
    mt                = m0 + idx % gm;
    nt                = idx / gm;
}

// 32 values per row of this warp's 32 rows (lane = row m_base + lane, values v) as f16 at
// base + m*ld + col: the high parts, or with LO the low parts f16(v - f16(v)); staged through
// shared memory (20 words per row) so that each row's 64 bytes are written by 4 lanes.
template <bool LO>
__device__ __forceinline__ void put_rows32_f16(uint32_t * sw, int lane, const float * v, uint16_t * base, int64_t ld,
                                               int64_t m_base, int64_t M, int64_t col) {
#pragma unroll
    for (int j = 0; j < 32; j += 8) {
        uint32_t wv[4];
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const float a = v[j + 2 * e], b = v[j + 2 * e + 1];
            __half2     hh = __floats2half2_rn(a, b);
            if (LO) {
                const float2 f2 = __half22float2(hh);
                hh              = __floats2half2_rn(__fsub_rn(a, f2.x), __fsub_rn(b, f2.y));
            }
            wv[e] = *reinterpret_cast<uint32_t *>(&hh);
        }
        *reinterpret_cast<uint4 *>(sw + lane * 20 + j / 2) = make_uint4(wv[0], wv[1], wv[2], wv[3]);
    }
    __syncwarp();
#pragma unroll
    for (int it = 0; it < 4; it++) {
        const int     rr = it * 8 + (lane >> 2), part = lane & 3;
        const int64_t mr = m_base + rr;
        if (mr < M) {
            *reinterpret_cast<uint4 *>(base + mr * ld + col + part * 8) =
                *reinterpret_cast<const uint4 *>(sw + rr * 20 + part * 4);
        }
    }
    __syncwarp();
}

// QKV epilogue of one warp: rows m_base + lane, output columns n0 .. n0 + 255 = two heads. For a q
// or k head: RMSNorm with the sum of squares in the association order of the one-warp-per-head
// kernel (lane l's partial ((a[2l]^2 + a[2l+1]^2) + b[2l]^2) + b[2l+1]^2 in double, a = dims
// 0..63, b = 64..127, then the xor-butterfly tree), so the result is bit-identical to
// acb_qk_norm_rope_planes over the f32 product; then NeoX RoPE and the hi/lo planes. A v head
// goes to the transposed planes, 32 tokens per store (one dim).
__device__ __forceinline__ void qkv_epilogue(const GemmArgs & g, uint32_t tacc, int64_t m_base, int64_t n0, int lane,
                                             float * stg) {
    const int64_t m  = m_base + lane;
    uint32_t *    sw = reinterpret_cast<uint32_t *>(stg);
    int           p  = 0;
    if (g.rope && m < g.M) {
        p = __ldg(g.pos + m);
        if (p < 0 || p >= g.max_pos) {
            if (g.err) {
                atomicOr(g.err, ACB_DEVERR_POS_RANGE);
            }
            p = -1;  // this row is written as zeros
        }
    }
#pragma unroll 1
    for (int hh = 0; hh < 2; hh++) {
        const int      hd  = (int) (n0 / 128) + hh;
        const uint32_t tc0 = tacc + (uint32_t) (hh * 128);
        if (hd < g.nq + g.nk) {
            const float * w = hd < g.nq ? g.qn : g.kn;
            float         sc = 1.0f;
            if (w) {
                uint32_t ra[32], rb[32];
                double   t[16];
                tmem_ld32(tc0 + 0, ra);   // dims 0..31   (lanes 0..15 of the per-head kernel)
                tmem_ld32(tc0 + 64, rb);  // dims 64..95
#pragma unroll
                for (int l = 0; l < 16; l++) {
                    const float a0 = __uint_as_float(ra[2 * l]), a1 = __uint_as_float(ra[2 * l + 1]);
                    const float b0 = __uint_as_float(rb[2 * l]), b1 = __uint_as_float(rb[2 * l + 1]);
                    double      s  = (double) __fmul_rn(a0, a0);
                    s += (double) __fmul_rn(a1, a1);
                    s += (double) __fmul_rn(b0, b0);
                    s += (double) __fmul_rn(b1, b1);
                    t[l] = s;
                }
                tmem_ld32(tc0 + 32, ra);  // dims 32..63  (lanes 16..31)
                tmem_ld32(tc0 + 96, rb);  // dims 96..127
#pragma unroll
                for (int l = 0; l < 16; l++) {
                    const float a0 = __uint_as_float(ra[2 * l]), a1 = __uint_as_float(ra[2 * l + 1]);
                    const float b0 = __uint_as_float(rb[2 * l]), b1 = __uint_as_float(rb[2 * l + 1]);
                    double      s  = (double) __fmul_rn(a0, a0);
                    s += (double) __fmul_rn(a1, a1);
                    s += (double) __fmul_rn(b0, b0);
                    s += (double) __fmul_rn(b1, b1);
                    t[l] = t[l] + s;  // butterfly level 16: lane l + lane l + 16
                }
#pragma unroll
                for (int o = 8; o > 0; o >>= 1) {
#pragma unroll
                    for (int l = 0; l < o; l++) {
                        t[l] = t[l] + t[l + o];
                    }
                }
                sc = rms_scale_pow2<128>(t[0], g.eps);
            }
#pragma unroll 1
            for (int c = 0; c < 2; c++) {
                uint32_t ra[32], rb[32];
                tmem_ld32(tc0 + (uint32_t) (32 * c), ra);
                tmem_ld32(tc0 + (uint32_t) (64 + 32 * c), rb);
                float a[32], b[32];
#pragma unroll
                for (int j = 0; j < 32; j++) {
                    a[j] = __uint_as_float(ra[j]);
                    b[j] = __uint_as_float(rb[j]);
                    if (w) {
                        a[j] = __fmul_rn(__fmul_rn(a[j], sc), __ldg(w + 32 * c + j));
                        b[j] = __fmul_rn(__fmul_rn(b[j], sc), __ldg(w + 64 + 32 * c + j));
                    }
                }
                if (g.rope && p >= 0) {
                    const float * cr = g.rope + (int64_t) p * 128 + 64 * c;  // cos/sin of dims 32c ..
#pragma unroll
                    for (int j = 0; j < 32; j += 2) {
                        const float4 cs = __ldg(reinterpret_cast<const float4 *>(cr + 2 * j));
#pragma unroll
                        for (int e = 0; e < 2; e++) {
                            const float cv = e ? cs.z : cs.x, sv = e ? cs.w : cs.y;
                            const float x0 = a[j + e], x1 = b[j + e];
                            a[j + e]       = __fsub_rn(__fmul_rn(x0, cv), __fmul_rn(x1, sv));
                            b[j + e]       = __fadd_rn(__fmul_rn(x0, sv), __fmul_rn(x1, cv));
                        }
                    }
                }
                if (p < 0) {
#pragma unroll
                    for (int j = 0; j < 32; j++) {
                        a[j] = 0.0f;
                        b[j] = 0.0f;
                    }
                }
                const int64_t col = (int64_t) hd * 128 + 32 * c;
                put_rows32_f16<false>(sw, lane, a, g.qk, g.qk_ld, m_base, g.M, col);
                put_rows32_f16<false>(sw, lane, b, g.qk, g.qk_ld, m_base, g.M, col + 64);
                if (g.qk_lo) {
                    put_rows32_f16<true>(sw, lane, a, g.qk + g.qk_lo, g.qk_ld, m_base, g.M, col);
                    put_rows32_f16<true>(sw, lane, b, g.qk + g.qk_lo, g.qk_ld, m_base, g.M, col + 64);
                }
            }
        } else {
            const int     hv = hd - g.nq - g.nk;
            const int64_t bb = m / g.seq, tt = m - bb * g.seq;
            uint16_t *    dst = g.vt + ((bb * g.nk + hv) * 128) * g.vt_ld + tt;
#pragma unroll 1
            for (int c = 0; c < 4; c++) {
                uint32_t r[32];
                tmem_ld32(tc0 + (uint32_t) (32 * c), r);
                if (m < g.M) {
#pragma unroll 4
                    for (int j = 0; j < 32; j++) {
                        const float   x  = __uint_as_float(r[j]);
                        const __half  hi = __float2half_rn(x);
                        const int64_t o  = (int64_t) (32 * c + j) * g.vt_ld;
                        dst[o]           = __half_as_ushort(hi);
                        if (g.vt_lo) {
                            dst[g.vt_lo + o] = __half_as_ushort(__float2half_rn(__fsub_rn(x, __half2float(hi))));
                        }
                    }
                }
            }
        }
    }
}

// ---- the kernel ------------------------------------------------------------------------------------
template <bool F16, bool PAIR>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const GemmArgs g) {
    using Cf = GemmCfg<PAIR>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t * smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t * ring = smem;  // kStages * kStage, 1024-aligned tiles (same offsets in both CTAs of a pair)
    float *    stage_base = reinterpret_cast<float *>(smem + Cf::kStages * Cf::kStage);
    uint64_t * full       = reinterpret_cast<uint64_t *>(smem + Cf::kStages * Cf::kStage + kStgBytes);
    uint64_t * empty      = full + Cf::kStages;
    uint64_t * tmem_full  = empty + Cf::kStages;
    uint64_t * tmem_empty = tmem_full + 2;
    uint32_t * tmem_slot  = reinterpret_cast<uint32_t *>(tmem_empty + 2);
    __shared__ volatile int abort_flag;

    const int      warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank   = PAIR ? cluster_ctarank() : 0;
    const bool     leader = rank == 0;
    const int64_t  unit    = PAIR ? (blockIdx.x >> 1) : blockIdx.x;  // work-issuing unit: CTA or CTA pair
    const int64_t  n_units = PAIR ? (gridDim.x >> 1) : gridDim.x;
    const int64_t m_tiles = (g.M + Cf::kTileM - 1) / Cf::kTileM;
    const int64_t n_tiles = g.swiglu ? g.F / 128 : (g.N + kBN - 1) / kBN;
    const int64_t tiles   = m_tiles * n_tiles;
    const int64_t n_work  = tiles * g.splits;
    const int     k_tiles = (int) (g.K / kBK);

    if (threadIdx.x == 0) {
        abort_flag = 0;
        for (int s = 0; s < Cf::kStages; s++) {
            ptx::mbar_init(&full[s], 1);
            ptx::mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; a++) {
            ptx::mbar_init(&tmem_full[a], 1);
            ptx::mbar_init(&tmem_empty[a], PAIR ? 8 : 4);  // one arrival per epilogue warp (of both CTAs)
        }
        ptx::fence_mbar_init();
        tma_prefetch_desc(&tmA);
        tma_prefetch_desc(&tmB);
    }
    if (warp == 1) {
        if constexpr (PAIR) {
            asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                             ptx::smem_u32(tmem_slot)),
                         "r"(kTmemCols));
            asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
        } else {
            asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                             ptx::smem_u32(tmem_slot)),
                         "r"(kTmemCols));
            asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
        }
    }
    ptx::grid_dep_wait();
    tc_fence_before();
    if constexpr (PAIR) {
        cluster_sync_all();  // barrier inits of both CTAs visible before any cross-CTA signal
    } else {
        __syncthreads();
    }
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            int it = 0;  // global k-stage counter
            for (int64_t w = unit; w < n_work && !abort_flag; w += n_units) {
                const int64_t t  = w % tiles;
                const int     sp = (int) (w / tiles);
                int64_t mt, nt;
                tile_mn(t, m_tiles, n_tiles, g.group_m, mt, nt);
                const int ma = (int) (mt * Cf::kTileM) + (int) rank * 128;  // this CTA's A rows
                // this CTA's B rows (SwiGLU: 128 gate rows and the matching 128 up rows per tile)
                const int nb = g.swiglu ? (int) (nt * 128) + (int) rank * (int) g.F
                                        : (int) (nt * kBN) + (int) rank * Cf::kRowsB;
                const int kt1 = min(k_tiles, (sp + 1) * g.kps);
                for (int kt = sp * g.kps; kt < kt1; kt++, it++) {
                    const int s = it % Cf::kStages;
                    if (it >= Cf::kStages && !ptx::mbar_wait(&empty[s], ((it / Cf::kStages) - 1) & 1)) {
                        flag_timeout(g.err);
                        abort_flag = 1;
                        break;
                    }
                    uint8_t * st = ring + (size_t) s * Cf::kStage;
                    int       ax, ay;
                    a_coords(g, kt, ma, ax, ay);
                    if constexpr (PAIR) {
                        const uint32_t fb = mapa_shared(ptx::smem_u32(&full[s]), 0);
                        if (leader) {
                            ptx::mbar_arrive_expect_tx(&full[s], Cf::kTx);
                        }
                        tma_load_2d_pair(st, &tmA, ax, ay, fb);
                        tma_load_2d_pair(st + Cf::kATile, &tmB, kt * kBK, nb, fb);
                    } else {
                        ptx::mbar_arrive_expect_tx(&full[s], Cf::kTx);
                        tma_load_2d(st, &tmA, ax, ay, &full[s]);
                        if (g.swiglu) {  // two 128-row boxes: gate rows, then up rows
                            tma_load_2d(st + Cf::kATile, &tmB, kt * kBK, nb, &full[s]);
                            tma_load_2d(st + Cf::kATile + 128 * kBK * 2, &tmB, kt * kBK, nb + (int) g.F, &full[s]);
                        } else {
                            tma_load_2d(st + Cf::kATile, &tmB, kt * kBK, nb, &full[s]);
                        }
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && leader) {
            constexpr uint32_t idesc = idesc_kind_f16(Cf::kTileM, kBN, F16);
            int                it    = 0;
            int                tile  = 0;
            for (int64_t w = unit; w < n_work && !abort_flag; w += n_units, tile++) {
                const int acc = tile & 1;
                if (tile >= 2 && !mbar_wait_cluster(&tmem_empty[acc], ((tile >> 1) - 1) & 1)) {
                    flag_timeout(g.err);
                    abort_flag = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t tmem_d = tmem_base + (uint32_t) (acc * kBN);
                const int      kt0    = (int) (w / tiles) * g.kps;
                const int      kt1    = min(k_tiles, kt0 + g.kps);
                for (int kt = kt0; kt < kt1; kt++, it++) {
                    const int s = it % Cf::kStages;
                    if (!ptx::mbar_wait(&full[s], (it / Cf::kStages) & 1)) {
                        flag_timeout(g.err);
                        abort_flag = 1;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a0 = ptx::smem_u32(ring + (size_t) s * Cf::kStage);
                    const uint32_t b0 = a0 + Cf::kATile;
#pragma unroll
                    for (int kk = 0; kk < kBK / 16; kk++) {
                        const uint32_t accumulate = (kt != kt0 || kk != 0) ? 1u : 0u;
                        if constexpr (PAIR) {
                            umma_f16kind_pair(tmem_d, smem_desc_sw128(a0 + kk * 32), smem_desc_sw128(b0 + kk * 32),
                                              idesc, accumulate);
                        } else {
                            umma_f16kind(tmem_d, smem_desc_sw128(a0 + kk * 32), smem_desc_sw128(b0 + kk * 32), idesc,
                                         accumulate);
                        }
                    }
                    // frees the stage (in both CTAs) once these MMAs have read it
                    if constexpr (PAIR) {
                        umma_commit_pair(&empty[s]);
                    } else {
                        umma_commit(&empty[s]);
                    }
                }
                if constexpr (PAIR) {  // accumulator complete
                    umma_commit_pair(&tmem_full[acc]);
                } else {
                    umma_commit(&tmem_full[acc]);
                }
            }
        }
    } else {
        // epilogue: warp w reads TMEM lanes 32*(w%4) .. +31 = tile rows. Each 32x32 chunk of raw
        // accumulators goes through this warp's staging block in shared memory so that global
        // reads and writes are whole 128-byte row segments (8 lanes x 4 columns per row).
        const int q     = warp & 3;
        float *   stg   = stage_base + q * 32 * kStgPitch;
        const int sub   = lane >> 3;       // row offset within a group of 4 rows
        const int cc    = (lane & 7) * 4;  // column offset within the chunk
        int       tile  = 0;
        // plain residual epilogue: each chunk's residual is in registers before its stores, the
        // first chunk's loaded while the tile's MMAs still run
        const bool pre = !g.swiglu && !g.qkv && g.splits == 1 && g.epi == (g.epi & (EPI_BIAS | EPI_RES)) &&
                         (g.epi & EPI_RES);
        float4     rv[8], rvn[8];
        for (int64_t w = unit; w < n_work; w += n_units, tile++) {
            const int acc = tile & 1;
            const int64_t t      = w % tiles;
            int64_t mt, nt;
            tile_mn(t, m_tiles, n_tiles, g.group_m, mt, nt);
            const int64_t m_base = mt * Cf::kTileM + (int64_t) rank * 128 + q * 32;
            if (pre) {
                load_res_chunk(g, m_base, nt * kBN, sub, cc, rv);
            }
            if (!ptx::mbar_wait(&tmem_full[acc], (tile >> 1) & 1)) {
                if (lane == 0) {
                    flag_timeout(g.err);
                }
                abort_flag = 1;
                break;
            }
            tc_fence_after();
            if (g.swiglu) {
                swiglu_epilogue(g, tmem_base + ((uint32_t) (q * 32) << 16) + (uint32_t) (acc * kBN), m_base,
                                nt * 128, lane, stg);
            } else if (g.qkv) {
                qkv_epilogue(g, tmem_base + ((uint32_t) (q * 32) << 16) + (uint32_t) (acc * kBN), m_base, nt * kBN,
                             lane, stg);
            } else {
            const int64_t n0     = nt * kBN;
            const bool    part   = g.splits > 1;  // raw partial of split w / tiles
            float *       pws    = part ? g.ws + (w / tiles) * g.M * g.N : nullptr;
#pragma unroll 1
            for (int c = 0; c < kBN / 32; c++) {
                if (pre && c + 1 < kBN / 32) {
                    load_res_chunk(g, m_base, n0 + (c + 1) * 32, sub, cc, rvn);
                }
                uint32_t r[32];
                tmem_ld32(tmem_base + ((uint32_t) (q * 32) << 16) + (uint32_t) (acc * kBN + c * 32), r);
                const int64_t nc = n0 + c * 32;
                if (nc >= g.N || m_base >= g.M) {
                    if (pre) {
#pragma unroll
                        for (int it = 0; it < 8; it++) {
                            rv[it] = rvn[it];
                        }
                    }
                    continue;  // warp-uniform: the whole chunk is outside C
                }
#pragma unroll
                for (int j = 0; j < 32; j += 4) {
                    *reinterpret_cast<float4 *>(stg + lane * kStgPitch + j) =
                        make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]), __uint_as_float(r[j + 2]),
                                    __uint_as_float(r[j + 3]));
                }
                __syncwarp();
                const int64_t n    = nc + cc;
                const int     ncol = n < g.N ? (g.N - n < 4 ? (int) (g.N - n) : 4) : 0;
                if (pre) {
                    // bias + prefetched residual (rv[it] is row it*4 + sub of this chunk)
#pragma unroll
                    for (int it = 0; it < 8; it++) {
                        const int64_t m = m_base + it * 4 + sub;
                        if (m < g.M && ncol > 0) {
                            float4 v = *reinterpret_cast<const float4 *>(stg + (it * 4 + sub) * kStgPitch + cc);
                            if (g.bias) {
                                const float4 bv = load_cols(g.bias + n, ncol);
                                v.x             = __fadd_rn(v.x, bv.x);
                                v.y             = __fadd_rn(v.y, bv.y);
                                v.z             = __fadd_rn(v.z, bv.z);
                                v.w             = __fadd_rn(v.w, bv.w);
                            }
                            v.x = __fadd_rn(rv[it].x, v.x);
                            v.y = __fadd_rn(rv[it].y, v.y);
                            v.z = __fadd_rn(rv[it].z, v.z);
                            v.w = __fadd_rn(rv[it].w, v.w);
                            store_c(g, m * g.ldc + n, v, ncol);
                        }
                        rv[it] = rvn[it];
                    }
                    __syncwarp();
                    continue;
                }
#pragma unroll 2
                for (int it = 0; it < 8; it++) {
                    const int     rr = it * 4 + sub;
                    const int64_t m  = m_base + rr;
                    if (m >= g.M || ncol == 0) {
                        continue;
                    }
                    float4 v = *reinterpret_cast<const float4 *>(stg + rr * kStgPitch + cc);
                    if (part) {
                        store_cols<ACB_TYPE_F32>(pws, m * g.N + n, v, ncol);
                        continue;
                    }
                    if (g.bias) {
                        const float4 bv = load_cols(g.bias + n, ncol);
                        v.x             = __fadd_rn(v.x, bv.x);
                        v.y             = __fadd_rn(v.y, bv.y);
                        v.z             = __fadd_rn(v.z, bv.z);
                        v.w             = __fadd_rn(v.w, bv.w);
                    }
                    if (g.epi & (EPI_RES | EPI_GATED_RES)) {
                        const float4 rs = load_cols(g.res + m * g.ldr + n, ncol);
                        if (g.epi & EPI_GATED_RES) {
                            const float4 gv = load_cols(g.gate + (m / g.rows_per_sample) * g.gate_stride + n, ncol);
                            v.x             = __fmul_rn(v.x, gv.x);
                            v.y             = __fmul_rn(v.y, gv.y);
                            v.z             = __fmul_rn(v.z, gv.z);
                            v.w             = __fmul_rn(v.w, gv.w);
                        }
                        v.x = __fadd_rn(rs.x, v.x);
                        v.y = __fadd_rn(rs.y, v.y);
                        v.z = __fadd_rn(rs.z, v.z);
                        v.w = __fadd_rn(rs.w, v.w);
                    }
                    store_c(g, m * g.ldc + n, v, ncol);
                }
                __syncwarp();
            }
            }  // plain / split epilogue
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                if (leader) {
                    ptx::mbar_arrive(&tmem_empty[acc]);
                } else {  // the pair's accumulators are handed back to the leader's MMA thread
                    mbar_arrive_cluster(mapa_shared(ptx::smem_u32(&tmem_empty[acc]), 0));
                }
            }
        }
    }
    ptx::grid_dep_launch();
    tc_fence_before();
    if constexpr (PAIR) {
        cluster_sync_all();  // no MMA, load or arrival of either CTA still targets the other
    } else {
        __syncthreads();
    }
    if (warp == 1) {
        tc_fence_after();
        if constexpr (PAIR) {
            asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols));
        } else {
            asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols));
        }
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
    const int64_t tiles   = ((M + 127) / 128) * ((N + kBN - 1) / kBN);
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

// Clusters of two CTAs that can be resident at once for the pair kernel (0: pairs off). Cached
// per operand type; ACB_GEMM_PAIR=0 in the environment turns the pair kernel off.
// Tile-order group (m-tiles per group); ACB_GEMM_GROUP in the environment overrides it.
static int group_m_for(int64_t m_tiles) {
    static int env = -1;
    if (env < 0) {
        const char * e = getenv("ACB_GEMM_GROUP");
        env            = e ? atoi(e) : 0;
    }
    const int gm = env > 0 ? env : (int) m_tiles;
    return gm < 1 ? 1 : (gm > m_tiles ? (int) m_tiles : gm);
}

static int pair_clusters(bool f16) {
    static int n[2] = { -1, -1 };
    int &      c    = n[f16 ? 1 : 0];
    if (c < 0) {
        c                 = 0;
        const char * env = getenv("ACB_GEMM_PAIR");
        if (env && env[0] == '0') {
            return c;
        }
        void (*kern)(const CUtensorMap, const CUtensorMap, const GemmArgs) =
            f16 ? gemm_tc_kernel<true, true> : gemm_tc_kernel<false, true>;
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) GemmCfg<true>::kSmem) !=
            cudaSuccess) {
            cudaGetLastError();
            return c;
        }
        cudaLaunchConfig_t  cfg = {};
        cudaLaunchAttribute a;
        a.id                 = cudaLaunchAttributeClusterDimension;
        a.val.clusterDim.x   = 2;
        a.val.clusterDim.y   = 1;
        a.val.clusterDim.z   = 1;
        cfg.gridDim          = dim3(2 * (unsigned) num_sms());
        cfg.blockDim         = dim3(kGemmThreads);
        cfg.dynamicSmemBytes = GemmCfg<true>::kSmem;
        cfg.attrs            = &a;
        cfg.numAttrs         = 1;
        int k                = 0;
        if (cudaOccupancyMaxActiveClusters(&k, kern, &cfg) == cudaSuccess && k > 0) {
            c = k;
        } else {
            cudaGetLastError();
        }
    }
    return c;
}

}  // namespace acb

using namespace acb;

extern "C" int acb_gemm_pair_clusters(int f16) {
    return pair_clusters(f16 != 0);
}

extern "C" size_t acb_gemm_workspace_bytes(int64_t M, int64_t N, int64_t K) {
    if (M <= 0 || N <= 0 || K <= 0 || K % kBK != 0) {
        return 0;
    }
    int       kps = 0;
    const int sp  = choose_splits(M, N, K, &kps);
    return sp > 1 ? (size_t) sp * (size_t) M * (size_t) N * 4 : 0;
}

// acb_gemm_tc and acb_conv1d_tc: a_cols = the columns of A's tensor map (K, or the channel count
// of an implicit convolution, whose conv_* fields are already set in g0)
static acb_status gemm_tc_launch(GemmArgs g0, const void * A, int64_t lda, int64_t a_cols, const void * B,
                                 int64_t ldb, int64_t M, int64_t N, int64_t K, void * C, int c_type, int64_t ldc,
                                 const float * bias, const float * res, int64_t ldr, const float * gate,
                                 int64_t gate_stride, int64_t rows_per_sample, int flags, void * workspace,
                                 size_t workspace_bytes, int * err_flag, acb_stream_t stream);

extern "C" acb_status acb_gemm_tc(const void * A, int64_t lda, const void * B, int64_t ldb, int64_t M, int64_t N,
                                  int64_t K, void * C, int c_type, int64_t ldc, const float * bias, const float * res,
                                  int64_t ldr, const float * gate, int64_t gate_stride, int64_t rows_per_sample,
                                  int flags, void * workspace, size_t workspace_bytes, int * err_flag,
                                  acb_stream_t stream) {
    if (!A || !B || !C || M <= 0 || N <= 0 || K <= 0 || lda < K || ldb < K || ldc < N) {
        return ACB_ERR_INVALID_ARG;
    }
    return gemm_tc_launch(GemmArgs{}, A, lda, K, B, ldb, M, N, K, C, c_type, ldc, bias, res, ldr, gate, gate_stride,
                          rows_per_sample, flags, workspace, workspace_bytes, err_flag, stream);
}

extern "C" acb_status acb_conv1d_tc(const void * X, int64_t ldx, int64_t T, int C_in, const void * W, int64_t N,
                                    int kernel, int dilation, int pad, void * Y, int y_type, int64_t ldy,
                                    const float * bias, const float * res, int64_t ldr, int flags, void * workspace,
                                    size_t workspace_bytes, int * err_flag, acb_stream_t stream) {
    if (!X || !W || !Y || T <= 0 || C_in <= 0 || N <= 0 || kernel <= 0 || dilation <= 0 || pad < 0 ||
        ldx < C_in || ldy < N) {
        return ACB_ERR_INVALID_ARG;
    }
    if (C_in % kBK != 0) {
        return ACB_ERR_UNSUPPORTED;
    }
    // rows reached by the taps stay within int range for the TMA coordinates
    if (T + (int64_t) (kernel - 1) * dilation > INT32_MAX / 2 || (int64_t) kernel * C_in > INT32_MAX / 2) {
        return ACB_ERR_UNSUPPORTED;
    }
    GemmArgs g0 = {};
    g0.conv_c   = C_in;
    g0.conv_dil = dilation;
    g0.conv_pad = pad;
    const int64_t K = (int64_t) kernel * C_in;
    return gemm_tc_launch(g0, X, ldx, C_in, W, K, T, N, K, Y, y_type, ldy, bias, res, ldr, nullptr, 0, 1, flags,
                          workspace, workspace_bytes, err_flag, stream);
}

static acb_status gemm_tc_launch(GemmArgs g0, const void * A, int64_t lda, int64_t a_cols, const void * B,
                                 int64_t ldb, int64_t M, int64_t N, int64_t K, void * C, int c_type, int64_t ldc,
                                 const float * bias, const float * res, int64_t ldr, const float * gate,
                                 int64_t gate_stride, int64_t rows_per_sample, int flags, void * workspace,
                                 size_t workspace_bytes, int * err_flag, acb_stream_t stream) {
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
    GemmArgs g        = g0;
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
    const bool f16 = (flags & ACB_FLAG_F16) != 0;
    // CTA pairs when the single-CTA tiling needs no split (enough 256x256 tiles to fill the GPU)
    const int  clusters = g.splits == 1 && M > 128 ? pair_clusters(f16) : 0;
    const bool pair     = clusters > 0;
    CUtensorMap ta, tb;
    if (!make_map(&ta, A, M, a_cols, lda, 128, f16) || !make_map(&tb, B, N, K, ldb, pair ? 128 : kBN, f16)) {
        return ACB_ERR_CUDA;
    }
    g.group_m              = group_m_for(pair ? (M + 255) / 256 : (M + 127) / 128);
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim           = dim3(kGemmThreads);
    cfg.stream             = (cudaStream_t) stream;
    cudaLaunchAttribute attr[2];
    int                 na = 0;
    if (pair) {
        attr[na].id               = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = 2;
        attr[na].val.clusterDim.y = 1;
        attr[na].val.clusterDim.z = 1;
        na++;
    }
    cudaLaunchAttribute & pdl = attr[na];
    pdl.id                                         = cudaLaunchAttributeProgrammaticStreamSerialization;
    pdl.val.programmaticStreamSerializationAllowed = 1;
    if (flags & ACB_FLAG_PDL) {
        na++;
    }
    cfg.attrs    = na ? attr : nullptr;
    cfg.numAttrs = na;
    cudaError_t e;
    if (pair) {
        const int64_t work = ((M + 255) / 256) * ((N + kBN - 1) / kBN);
        cfg.gridDim          = dim3((unsigned) (2 * (work < clusters ? work : clusters)));
        cfg.dynamicSmemBytes = GemmCfg<true>::kSmem;
        e = cudaLaunchKernelEx(&cfg, f16 ? gemm_tc_kernel<true, true> : gemm_tc_kernel<false, true>, ta, tb, g);
    } else {
        const int64_t work = ((M + 127) / 128) * ((N + kBN - 1) / kBN) * g.splits;
        void (*kern)(const CUtensorMap, const CUtensorMap, const GemmArgs) =
            f16 ? gemm_tc_kernel<true, false> : gemm_tc_kernel<false, false>;
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) GemmCfg<false>::kSmem);
        cfg.gridDim          = dim3((unsigned) (work < num_sms() ? work : num_sms()));
        cfg.dynamicSmemBytes = GemmCfg<false>::kSmem;
        e                    = cudaLaunchKernelEx(&cfg, kern, ta, tb, g);
    }
    if (e == cudaSuccess && g.splits > 1) {
        // the reduction always waits on the GEMM through griddepcontrol.wait
        const int64_t n_thr = M * (N / 4);
        cfg.gridDim         = dim3((unsigned) ((n_thr + 255) / 256));
        cfg.blockDim        = dim3(256);
        cfg.dynamicSmemBytes = 0;
        cfg.attrs           = &pdl;
        cfg.numAttrs        = 1;
        e                   = cudaLaunchKernelEx(&cfg, splitk_reduce_kernel, g);
    }
    if (e != cudaSuccess) {
        set_last_cuda_error(e);
        return ACB_ERR_CUDA;
    }
    return ACB_OK;
}

extern "C" acb_status acb_gemm_swiglu_quant(const void * A, int64_t lda, const void * B, int64_t ldb, int64_t M,
                                            int64_t F, int64_t K, const float * bias, int vec_type, int layout,
                                            void * Y, int y_type, int64_t ldy, int flags, int * err_flag,
                                            acb_stream_t stream) {
    if (!A || !B || !Y || M <= 0 || F <= 0 || K <= 0 || lda < K || ldb < K) {
        return ACB_ERR_INVALID_ARG;
    }
    if (F % 128 != 0 || K % kBK != 0 || (lda * 2) % 16 != 0 || (ldb * 2) % 16 != 0 ||
        reinterpret_cast<uintptr_t>(A) % 16 != 0 || reinterpret_cast<uintptr_t>(B) % 16 != 0 ||
        reinterpret_cast<uintptr_t>(Y) % 16 != 0 || ldy % 8 != 0) {
        return ACB_ERR_UNSUPPORTED;
    }
    if ((vec_type != ACB_TYPE_Q8_0 && vec_type != ACB_TYPE_F16 && vec_type != ACB_TYPE_BF16) ||
        (layout != ACB_LAYOUT_PLAIN && layout != ACB_LAYOUT_GEMM_A) ||
        y_type != (vec_type == ACB_TYPE_BF16 ? ACB_TYPE_BF16 : ACB_TYPE_F16)) {
        return ACB_ERR_UNSUPPORTED;
    }
    if (ldy < (layout == ACB_LAYOUT_GEMM_A ? 3 * F : F)) {
        return ACB_ERR_INVALID_ARG;
    }
    GemmArgs g        = {};
    g.M               = M;
    g.N               = 2 * F;
    g.K               = K;
    g.C               = Y;
    g.c_type          = y_type;
    g.ldc             = ldy;
    g.bias            = bias;
    g.rows_per_sample = 1;
    g.err             = err_flag;
    g.splits          = 1;
    g.kps             = (int) (K / kBK);
    g.swiglu          = 1;
    g.sw_vt           = vec_type;
    g.sw_layout       = layout;
    g.F               = F;
    const bool f16      = (flags & ACB_FLAG_F16) != 0;
    const int  clusters = M > 128 ? pair_clusters(f16) : 0;
    const bool pair     = clusters > 0;
    CUtensorMap ta, tb;
    if (!make_map(&ta, A, M, K, lda, 128, f16) || !make_map(&tb, B, 2 * F, K, ldb, 128, f16)) {
        return ACB_ERR_CUDA;
    }
    g.group_m              = group_m_for(pair ? (M + 255) / 256 : (M + 127) / 128);
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim           = dim3(kGemmThreads);
    cfg.stream             = (cudaStream_t) stream;
    cudaLaunchAttribute attr[2];
    int                 na = 0;
    if (pair) {
        attr[na].id               = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = 2;
        attr[na].val.clusterDim.y = 1;
        attr[na].val.clusterDim.z = 1;
        na++;
    }
    if (flags & ACB_FLAG_PDL) {
        attr[na].id                                         = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        na++;
    }
    cfg.attrs    = na ? attr : nullptr;
    cfg.numAttrs = na;
    cudaError_t e;
    if (pair) {
        const int64_t work = ((M + 255) / 256) * (F / 128);
        cfg.gridDim          = dim3((unsigned) (2 * (work < clusters ? work : clusters)));
        cfg.dynamicSmemBytes = GemmCfg<true>::kSmem;
        e = cudaLaunchKernelEx(&cfg, f16 ? gemm_tc_kernel<true, true> : gemm_tc_kernel<false, true>, ta, tb, g);
    } else {
        const int64_t work = ((M + 127) / 128) * (F / 128);
        void (*kern)(const CUtensorMap, const CUtensorMap, const GemmArgs) =
            f16 ? gemm_tc_kernel<true, false> : gemm_tc_kernel<false, false>;
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) GemmCfg<false>::kSmem);
        cfg.gridDim          = dim3((unsigned) (work < num_sms() ? work : num_sms()));
        cfg.dynamicSmemBytes = GemmCfg<false>::kSmem;
        e                    = cudaLaunchKernelEx(&cfg, kern, ta, tb, g);
    }
    if (e != cudaSuccess) {
        set_last_cuda_error(e);
        return ACB_ERR_CUDA;
    }
    return ACB_OK;
}

extern "C" acb_status acb_gemm_qkv_planes(const void * A, int64_t lda, const void * B, int64_t ldb, int64_t M,
                                          int64_t K, int n_q_heads, int n_kv_heads, const float * q_norm_w,
                                          const float * k_norm_w, float eps, const int32_t * pos,
                                          const float * rope_table, int max_pos, int64_t seq_len, uint16_t * qk,
                                          int64_t qk_ld, int64_t qk_lo, uint16_t * vt, int64_t vt_ld, int64_t vt_lo,
                                          int flags, int * err_flag, acb_stream_t stream) {
    if (!A || !B || !qk || (n_kv_heads > 0 && !vt) || M <= 0 || K <= 0 || lda < K || ldb < K || n_q_heads <= 0 ||
        n_kv_heads < 0 || seq_len <= 0 || M % seq_len != 0 || qk_ld < (int64_t) (n_q_heads + n_kv_heads) * 128 ||
        (n_kv_heads > 0 && vt_ld < seq_len) || qk_lo < 0 || vt_lo < 0) {
        return ACB_ERR_INVALID_ARG;
    }
    if (rope_table && (!pos || max_pos <= 0)) {
        return ACB_ERR_INVALID_ARG;
    }
    if (n_q_heads % 2 || n_kv_heads % 2 || K % kBK != 0 || (lda * 2) % 16 != 0 || (ldb * 2) % 16 != 0 ||
        reinterpret_cast<uintptr_t>(A) % 16 != 0 || reinterpret_cast<uintptr_t>(B) % 16 != 0 ||
        reinterpret_cast<uintptr_t>(qk) % 16 != 0 || qk_ld % 8 != 0 || qk_lo % 8 != 0 ||
        reinterpret_cast<uintptr_t>(rope_table) % 16 != 0) {
        return ACB_ERR_UNSUPPORTED;
    }
    const int64_t N   = (int64_t) (n_q_heads + 2 * n_kv_heads) * 128;
    GemmArgs      g   = {};
    g.M               = M;
    g.N               = N;
    g.K               = K;
    g.C               = qk;
    g.c_type          = ACB_TYPE_F16;
    g.ldc             = qk_ld;
    g.rows_per_sample = 1;
    g.err             = err_flag;
    g.splits          = 1;
    g.kps             = (int) (K / kBK);
    g.qkv             = 1;
    g.nq              = n_q_heads;
    g.nk              = n_kv_heads;
    g.qn              = q_norm_w;
    g.kn              = k_norm_w;
    g.eps             = eps;
    g.pos             = pos;
    g.rope            = rope_table;
    g.max_pos         = max_pos;
    g.seq             = seq_len;
    g.qk              = qk;
    g.qk_ld           = qk_ld;
    g.qk_lo           = qk_lo;
    g.vt              = vt;
    g.vt_ld           = vt_ld;
    g.vt_lo           = vt_lo;
    const bool f16      = (flags & ACB_FLAG_F16) != 0;
    const int  clusters = M > 128 ? pair_clusters(f16) : 0;
    const bool pair     = clusters > 0;
    CUtensorMap ta, tb;
    if (!make_map(&ta, A, M, K, lda, 128, f16) || !make_map(&tb, B, N, K, ldb, pair ? 128 : kBN, f16)) {
        return ACB_ERR_CUDA;
    }
    g.group_m              = group_m_for(pair ? (M + 255) / 256 : (M + 127) / 128);
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim           = dim3(kGemmThreads);
    cfg.stream             = (cudaStream_t) stream;
    cudaLaunchAttribute attr[2];
    int                 na = 0;
    if (pair) {
        attr[na].id               = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = 2;
        attr[na].val.clusterDim.y = 1;
        attr[na].val.clusterDim.z = 1;
        na++;
    }
    if (flags & ACB_FLAG_PDL) {
        attr[na].id                                         = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        na++;
    }
    cfg.attrs    = na ? attr : nullptr;
    cfg.numAttrs = na;
    cudaError_t e;
    if (pair) {
        const int64_t work = ((M + 255) / 256) * (N / kBN);
        cfg.gridDim          = dim3((unsigned) (2 * (work < clusters ? work : clusters)));
        cfg.dynamicSmemBytes = GemmCfg<true>::kSmem;
        e = cudaLaunchKernelEx(&cfg, f16 ? gemm_tc_kernel<true, true> : gemm_tc_kernel<false, true>, ta, tb, g);
    } else {
        const int64_t work = ((M + 127) / 128) * (N / kBN);
        void (*kern)(const CUtensorMap, const CUtensorMap, const GemmArgs) =
            f16 ? gemm_tc_kernel<true, false> : gemm_tc_kernel<false, false>;
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) GemmCfg<false>::kSmem);
        cfg.gridDim          = dim3((unsigned) (work < num_sms() ? work : num_sms()));
        cfg.dynamicSmemBytes = GemmCfg<false>::kSmem;
        e                    = cudaLaunchKernelEx(&cfg, kern, ta, tb, g);
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
