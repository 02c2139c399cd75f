// k_attn_prefill.cu -- attention over whole sequences for the text encoder (causal,
// src/qwen3-enc.h:186-199) and the DiT (self-attention with the even layers' sliding window,
// cross-attention to the condition; src/dit-graph.h:218-231, 339-352):
//     O[b,i,h,:] = softmax_j( Q[b,i,h,:] . K[b,j,h/G,:] * scale + mask(i,j) ) V[b,j,h/G,:]
// Flash-attention tiling with bf16 or f16 tensor-core MMAs (mma.sync m16n8k16, fp32 accumulation):
// a CTA owns 128 queries of one (batch, head); eight warps own 16 query rows each with their Q
// fragments in registers; 64-key K/V blocks stream through a cp.async double buffer (rows padded
// to 272 bytes so ldmatrix is conflict-free); the softmax is online in fp32 (exp2 with the scale
// folded into log2 e); blocks wholly outside a causal or sliding-window mask are skipped.
#include "common.cuh"
#include "ptx.cuh"

namespace acb {

constexpr int kAttnD    = 128;
constexpr int kAttnBQ   = 128;  // queries per CTA: 8 warps of 16 rows
constexpr int kAttnBK   = 64;
constexpr int kAttnPad  = kAttnD + 8;  // bf16 elements per smem row
constexpr int kAttnThreads = kAttnBQ * 2;

enum { MASK_NONE = 0, MASK_CAUSAL = 1, MASK_WINDOW = 2 };

struct AttnArgs {
    const __nv_bfloat16 * q;
    const __nv_bfloat16 * k;
    const __nv_bfloat16 * v;
    void *                o;
    int                   o_type;
    int64_t               q_bs, q_ts;  // element strides: batch, token (head stride = D)
    int64_t               k_bs, k_ts;
    int64_t               v_bs, v_ts;
    int64_t               o_bs, o_ts;
    int                   Sq, Skv, Nh, Nkv;
    int                   mask;
    int                   window;      // MASK_WINDOW: |i - j| <= window
    int                   causal_off;  // MASK_CAUSAL: key j allowed when j <= i + causal_off
    float                 scale_log2;  // scale * log2(e)
    int64_t               q_lo, k_lo, v_lo;  // SPLIT: element offsets of the lo planes
};

__device__ __forceinline__ void cp_async16(void * dst, const void * src, bool pred) {
    const int n = pred ? 16 : 0;  // zero-fill when out of range
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(ptx::smem_u32(dst)), "l"(src), "r"(n)
                 : "memory");
}

__device__ __forceinline__ void cp_async_commit() {
    asm volatile("cp.async.commit_group;" ::: "memory");
}

template <int N> __device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t & r0, uint32_t & r1, uint32_t & r2, uint32_t & r3, const void * p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(ptx::smem_u32(p)));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t & r0, uint32_t & r1, uint32_t & r2, uint32_t & r3, const void * p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(ptx::smem_u32(p)));
}

// m16n8k16 with fp32 accumulation; A and B both bf16, or both f16
template <bool F16> __device__ __forceinline__ void mma16(float * c, const uint32_t * a, uint32_t b0, uint32_t b1) {
    if (F16) {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    } else {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
            : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
    }
}

template <bool F16> __device__ __forceinline__ uint32_t pack16(float lo, float hi) {
    if (F16) {
        __half2 h = __floats2half2_rn(lo, hi);
        return *reinterpret_cast<uint32_t *>(&h);
    }
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&h);
}

// load a [ROWS][128] 16-bit tile (rows row0.., clipped to nrows) into padded smem
template <int ROWS>
__device__ __forceinline__ void load_tile(__nv_bfloat16 * sm, const __nv_bfloat16 * g, int64_t ts, int row0,
                                          int nrows) {
    for (int c = threadIdx.x; c < ROWS * 16; c += kAttnThreads) {
        const int  r  = c >> 4, col = (c & 15) * 8;
        const bool ok = row0 + r < nrows;
        cp_async16(sm + r * kAttnPad + col, g + (int64_t) (ok ? row0 + r : 0) * ts + col, ok);
    }
}

// SPLIT: every operand is given as f16 hi and lo planes (hi + lo == the f32 value) and each
// product is formed as hi.hi + hi.lo + lo.hi, which reproduces f32 attention to ~2^-22; the
// probabilities are split the same way before P.V.
template <int MASK, bool F16, bool SPLIT>
__global__ void __launch_bounds__(kAttnThreads) attn_prefill_kernel(const AttnArgs a) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    constexpr int   kQTile = kAttnBQ * kAttnPad;       // elements of the padded query tile
    constexpr int   kKTile = kAttnBK * kAttnPad;       // elements of one padded key/value tile
    __nv_bfloat16 * sQ = reinterpret_cast<__nv_bfloat16 *>(smem_raw);
    __nv_bfloat16 * sK = sQ + kQTile;                  // 2 buffers
    __nv_bfloat16 * sV = sK + 2 * kKTile;              // 2 buffers
    __nv_bfloat16 * sQl = sV + 2 * kKTile;             // SPLIT only: lo planes
    __nv_bfloat16 * sKl = sQl + kQTile;
    __nv_bfloat16 * sVl = sKl + 2 * kKTile;

    const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int hk   = h / (a.Nh / a.Nkv);
    const int q0   = qt * kAttnBQ;

    ptx::grid_dep_wait();
    const __nv_bfloat16 * Qg = a.q + (int64_t) b * a.q_bs + (int64_t) h * kAttnD;
    const __nv_bfloat16 * Kg = a.k + (int64_t) b * a.k_bs + (int64_t) hk * kAttnD;
    const __nv_bfloat16 * Vg = a.v + (int64_t) b * a.v_bs + (int64_t) hk * kAttnD;

    // key-block range allowed by the mask for this query tile
    int kb_lo = 0, kb_hi = (a.Skv + kAttnBK - 1) / kAttnBK;
    if (MASK == MASK_CAUSAL) {
        const int last_q = min(q0 + kAttnBQ, a.Sq) - 1 + a.causal_off;
        kb_hi            = min(kb_hi, last_q / kAttnBK + 1);
    } else if (MASK == MASK_WINDOW) {
        kb_lo = max(0, (q0 - a.window) / kAttnBK);
        kb_hi = min(kb_hi, (min(q0 + kAttnBQ, a.Sq) - 1 + a.window) / kAttnBK + 1);
    }

    load_tile<kAttnBQ>(sQ, Qg + (int64_t) 0, a.q_ts, q0, a.Sq);
    if (SPLIT) {
        load_tile<kAttnBQ>(sQl, Qg + a.q_lo, a.q_ts, q0, a.Sq);
    }
    if (kb_lo < kb_hi) {
        load_tile<kAttnBK>(sK, Kg, a.k_ts, kb_lo * kAttnBK, a.Skv);
        load_tile<kAttnBK>(sV, Vg, a.v_ts, kb_lo * kAttnBK, a.Skv);
        if (SPLIT) {
            load_tile<kAttnBK>(sKl, Kg + a.k_lo, a.k_ts, kb_lo * kAttnBK, a.Skv);
            load_tile<kAttnBK>(sVl, Vg + a.v_lo, a.v_ts, kb_lo * kAttnBK, a.Skv);
        }
    }
    cp_async_commit();

    float    o[16][4];
    float    m_i[2] = { -INFINITY, -INFINITY }, l_i[2] = { 0.0f, 0.0f };
    uint32_t qf[8][4];
#pragma unroll
    for (int n = 0; n < 16; n++) {
#pragma unroll
        for (int e = 0; e < 4; e++) {
            o[n][e] = 0.0f;
        }
    }
    const int row_a = q0 + warp * 16 + (lane >> 2);  // this thread's two query rows: row_a, row_a + 8

    for (int kb = kb_lo; kb < kb_hi; kb++) {
        const int buf = (kb - kb_lo) & 1;
        if (kb + 1 < kb_hi) {
            load_tile<kAttnBK>(sK + (buf ^ 1) * kKTile, Kg, a.k_ts, (kb + 1) * kAttnBK, a.Skv);
            load_tile<kAttnBK>(sV + (buf ^ 1) * kKTile, Vg, a.v_ts, (kb + 1) * kAttnBK, a.Skv);
            if (SPLIT) {
                load_tile<kAttnBK>(sKl + (buf ^ 1) * kKTile, Kg + a.k_lo, a.k_ts, (kb + 1) * kAttnBK, a.Skv);
                load_tile<kAttnBK>(sVl + (buf ^ 1) * kKTile, Vg + a.v_lo, a.v_ts, (kb + 1) * kAttnBK, a.Skv);
            }
        }
        cp_async_commit();
        cp_async_wait<1>();
        __syncthreads();
        if (!SPLIT && kb == kb_lo) {
#pragma unroll
            for (int ks = 0; ks < 8; ks++) {
                const __nv_bfloat16 * p = sQ + (warp * 16 + (lane & 15)) * kAttnPad + ks * 16 + (lane >> 4) * 8;
                ldsm_x4(qf[ks][0], qf[ks][1], qf[ks][2], qf[ks][3], p);
            }
        }
        const __nv_bfloat16 * Kb  = sK + buf * kAttnBK * kAttnPad;
        const __nv_bfloat16 * Vb  = sV + buf * kAttnBK * kAttnPad;
        const __nv_bfloat16 * Kbl = sKl + buf * kAttnBK * kAttnPad;
        const __nv_bfloat16 * Vbl = sVl + buf * kAttnBK * kAttnPad;

        // S = Q K^T for 16 rows x 64 keys
        float s[8][4];
#pragma unroll
        for (int n = 0; n < 8; n++) {
#pragma unroll
            for (int e = 0; e < 4; e++) {
                s[n][e] = 0.0f;
            }
        }
#pragma unroll
        for (int ks = 0; ks < 8; ks++) {
            uint32_t qh[4], ql[4];
            if (SPLIT) {  // Q fragments re-read per key block (registers go to the split products)
                const int off = (warp * 16 + (lane & 15)) * kAttnPad + ks * 16 + (lane >> 4) * 8;
                ldsm_x4(qh[0], qh[1], qh[2], qh[3], sQ + off);
                ldsm_x4(ql[0], ql[1], ql[2], ql[3], sQl + off);
            }
#pragma unroll
            for (int np = 0; np < 4; np++) {  // pairs of 8-key n-tiles
                uint32_t b0, b1, b2, b3;
                const int key = np * 16 + (lane & 7) + ((lane >> 4) << 3);
                const int d   = ks * 16 + ((lane >> 3) & 1) * 8;
                ldsm_x4(b0, b1, b2, b3, Kb + key * kAttnPad + d);
                if (SPLIT) {
                    uint32_t c0, c1, c2, c3;
                    ldsm_x4(c0, c1, c2, c3, Kbl + key * kAttnPad + d);
                    mma16<F16>(s[2 * np], ql, b0, b1);
                    mma16<F16>(s[2 * np + 1], ql, b2, b3);
                    mma16<F16>(s[2 * np], qh, c0, c1);
                    mma16<F16>(s[2 * np + 1], qh, c2, c3);
                    mma16<F16>(s[2 * np], qh, b0, b1);
                    mma16<F16>(s[2 * np + 1], qh, b2, b3);
                } else {
                    mma16<F16>(s[2 * np], qf[ks], b0, b1);
                    mma16<F16>(s[2 * np + 1], qf[ks], b2, b3);
                }
            }
        }
        // scale (in log2 units), mask, online softmax
        const int kbase = kb * kAttnBK;
        float     mx[2] = { -INFINITY, -INFINITY };
#pragma unroll
        for (int n = 0; n < 8; n++) {
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int j   = kbase + n * 8 + (lane & 3) * 2 + (e & 1);
                const int i   = row_a + (e >> 1) * 8;
                bool      ok  = j < a.Skv;
                if (MASK == MASK_CAUSAL) {
                    ok = ok && j <= i + a.causal_off;
                } else if (MASK == MASK_WINDOW) {
                    ok = ok && (i > j ? i - j : j - i) <= a.window;
                }
                const float v = ok ? s[n][e] * a.scale_log2 : -INFINITY;
                s[n][e]       = v;
                mx[e >> 1]    = fmaxf(mx[e >> 1], v);
            }
        }
#pragma unroll
        for (int r = 0; r < 2; r++) {
            mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
            mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
        }
        float m_new[2], alpha[2], rs[2] = { 0.0f, 0.0f };
#pragma unroll
        for (int r = 0; r < 2; r++) {
            m_new[r] = fmaxf(m_i[r], mx[r]);
            alpha[r] = m_new[r] == -INFINITY ? 1.0f : exp2f(m_i[r] - m_new[r]);
        }
        uint32_t pf[4][4];  // P as 16-bit A fragments: 4 key steps of 16
        uint32_t pl[SPLIT ? 4 : 1][4];  // SPLIT: lo parts of P
#pragma unroll
        for (int n = 0; n < 8; n++) {
            float p[4];
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const float mr = m_new[e >> 1];
                p[e]           = mr == -INFINITY ? 0.0f : exp2f(s[n][e] - mr);
                rs[e >> 1] += p[e];
            }
            // C-fragment (rows r, r+8; cols 2c, 2c+1) -> A-fragment halves of key step n/2
            pf[n >> 1][(n & 1) * 2 + 0] = pack16<F16>(p[0], p[1]);
            pf[n >> 1][(n & 1) * 2 + 1] = pack16<F16>(p[2], p[3]);
            if (SPLIT) {
                float l[4];
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    l[e] = __fsub_rn(p[e], __half2float(__float2half_rn(p[e])));
                }
                pl[SPLIT ? (n >> 1) : 0][(n & 1) * 2 + 0] = pack16<F16>(l[0], l[1]);
                pl[SPLIT ? (n >> 1) : 0][(n & 1) * 2 + 1] = pack16<F16>(l[2], l[3]);
            }
        }
#pragma unroll
        for (int r = 0; r < 2; r++) {
            rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 1);
            rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 2);
            l_i[r] = l_i[r] * alpha[r] + rs[r];
            m_i[r] = m_new[r];
        }
#pragma unroll
        for (int n = 0; n < 16; n++) {
            o[n][0] *= alpha[0];
            o[n][1] *= alpha[0];
            o[n][2] *= alpha[1];
            o[n][3] *= alpha[1];
        }
        // O += P V
#pragma unroll
        for (int ks = 0; ks < 4; ks++) {
            // A fragment order for m16k16: {rows r: k0-7, rows r+8: k0-7, rows r: k8-15, rows r+8: k8-15}
            const uint32_t af[4] = { pf[ks][0], pf[ks][1], pf[ks][2], pf[ks][3] };
#pragma unroll
            for (int np = 0; np < 8; np++) {  // pairs of 8-wide d tiles
                uint32_t b0, b1, b2, b3;
                const int key = ks * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
                const int d   = np * 16 + (lane >> 4) * 8;
                ldsm_x4_t(b0, b1, b2, b3, Vb + key * kAttnPad + d);
                if (SPLIT) {
                    uint32_t c0, c1, c2, c3;
                    ldsm_x4_t(c0, c1, c2, c3, Vbl + key * kAttnPad + d);
                    const uint32_t lf[4] = { pl[SPLIT ? ks : 0][0], pl[SPLIT ? ks : 0][1], pl[SPLIT ? ks : 0][2],
                                             pl[SPLIT ? ks : 0][3] };
                    mma16<F16>(o[2 * np], lf, b0, b1);
                    mma16<F16>(o[2 * np + 1], lf, b2, b3);
                    mma16<F16>(o[2 * np], af, c0, c1);
                    mma16<F16>(o[2 * np + 1], af, c2, c3);
                }
                mma16<F16>(o[2 * np], af, b0, b1);
                mma16<F16>(o[2 * np + 1], af, b2, b3);
            }
        }
        __syncthreads();
    }
    cp_async_wait<0>();

    // normalise and store rows row_a and row_a + 8
#pragma unroll
    for (int r = 0; r < 2; r++) {
        const int i = row_a + r * 8;
        if (i >= a.Sq) {
            continue;
        }
        const float inv = l_i[r] > 0.0f ? 1.0f / l_i[r] : 0.0f;
        const int64_t base = (int64_t) b * a.o_bs + (int64_t) i * a.o_ts + (int64_t) h * kAttnD;
#pragma unroll
        for (int n = 0; n < 16; n++) {
            const int   d  = n * 8 + (lane & 3) * 2;
            const float v0 = o[n][2 * r] * inv, v1 = o[n][2 * r + 1] * inv;
            if (a.o_type == ACB_TYPE_F32) {
                float * dst = reinterpret_cast<float *>(a.o) + base + d;
                *reinterpret_cast<float2 *>(dst) = make_float2(v0, v1);
            } else if (a.o_type == ACB_TYPE_BF16) {
                __nv_bfloat16 * dst = reinterpret_cast<__nv_bfloat16 *>(a.o) + base + d;
                *reinterpret_cast<__nv_bfloat162 *>(dst) = __floats2bfloat162_rn(v0, v1);
            } else {
                __half * dst = reinterpret_cast<__half *>(a.o) + base + d;
                *reinterpret_cast<__half2 *>(dst) = __floats2half2_rn(v0, v1);
            }
        }
    }
    ptx::grid_dep_launch();
}

}  // namespace acb

using namespace acb;

static acb_status attn_launch(const void * q, int64_t q_bs, int64_t q_ts, const void * k, int64_t k_bs, int64_t k_ts,
                              const void * v, int64_t v_bs, int64_t v_ts, void * o, int o_type, int64_t o_bs,
                              int64_t o_ts, int batch, int Sq, int Skv, int Nh, int Nkv, int head_dim, int mask,
                              int window, int causal_off, float scale, int flags, bool split, int64_t q_lo,
                              int64_t k_lo, int64_t v_lo, acb_stream_t stream) {
    if (!q || !k || !v || !o || batch <= 0 || Sq <= 0 || Skv <= 0 || Nh <= 0 || Nkv <= 0 || Nh % Nkv != 0) {
        return ACB_ERR_INVALID_ARG;
    }
    if (head_dim != kAttnD || (o_type != ACB_TYPE_F32 && o_type != ACB_TYPE_BF16 && o_type != ACB_TYPE_F16) ||
        mask < 0 || mask > 2) {
        return ACB_ERR_UNSUPPORTED;
    }
    if ((q_ts | k_ts | v_ts | q_bs | k_bs | v_bs | q_lo | k_lo | v_lo) % 8 != 0 ||
        reinterpret_cast<uintptr_t>(q) % 16 || reinterpret_cast<uintptr_t>(k) % 16 ||
        reinterpret_cast<uintptr_t>(v) % 16) {
        return ACB_ERR_UNSUPPORTED;  // 16-byte cp.async rows
    }
    AttnArgs a   = {};
    a.q          = (const __nv_bfloat16 *) q;
    a.k          = (const __nv_bfloat16 *) k;
    a.v          = (const __nv_bfloat16 *) v;
    a.o          = o;
    a.o_type     = o_type;
    a.q_bs       = q_bs;
    a.q_ts       = q_ts;
    a.k_bs       = k_bs;
    a.k_ts       = k_ts;
    a.v_bs       = v_bs;
    a.v_ts       = v_ts;
    a.o_bs       = o_bs;
    a.o_ts       = o_ts;
    a.Sq         = Sq;
    a.Skv        = Skv;
    a.Nh         = Nh;
    a.Nkv        = Nkv;
    a.mask       = mask;
    a.window     = window;
    a.causal_off = causal_off;
    a.scale_log2 = scale * 1.4426950408889634f;
    a.q_lo       = q_lo;
    a.k_lo       = k_lo;
    a.v_lo       = v_lo;
    const size_t smem = (size_t) ((split ? 2 : 1) * kAttnBQ + (split ? 8 : 4) * kAttnBK) * kAttnPad * 2;
    const dim3   grid((unsigned) ((Sq + kAttnBQ - 1) / kAttnBQ), (unsigned) Nh, (unsigned) batch);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim            = grid;
    cfg.blockDim           = dim3(kAttnThreads);
    cfg.dynamicSmemBytes   = smem;
    cfg.stream             = (cudaStream_t) stream;
    cudaLaunchAttribute attr[1];
    attr[0].id                                         = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs                                          = (flags & ACB_FLAG_PDL) ? attr : nullptr;
    cfg.numAttrs                                       = (flags & ACB_FLAG_PDL) ? 1 : 0;
    const bool f16 = split || (flags & ACB_FLAG_F16) != 0;
    void (*kern)(const AttnArgs) = nullptr;
#define ACB_PICK(M)                                                                                      \
    kern = split ? attn_prefill_kernel<M, true, true>                                                    \
                 : (f16 ? attn_prefill_kernel<M, true, false> : attn_prefill_kernel<M, false, false>)
    if (mask == MASK_CAUSAL) {
        ACB_PICK(MASK_CAUSAL);
    } else if (mask == MASK_WINDOW) {
        ACB_PICK(MASK_WINDOW);
    } else {
        ACB_PICK(MASK_NONE);
    }
#undef ACB_PICK
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a);
    if (e != cudaSuccess) {
        set_last_cuda_error(e);
        return ACB_ERR_CUDA;
    }
    return ACB_OK;
}

extern "C" acb_status acb_attn_prefill(const void * q, int64_t q_bs, int64_t q_ts, const void * k, int64_t k_bs,
                                       int64_t k_ts, const void * v, int64_t v_bs, int64_t v_ts, void * o,
                                       int o_type, int64_t o_bs, int64_t o_ts, int batch, int Sq, int Skv, int Nh,
                                       int Nkv, int head_dim, int mask, int window, int causal_off, float scale,
                                       int flags, acb_stream_t stream) {
    return attn_launch(q, q_bs, q_ts, k, k_bs, k_ts, v, v_bs, v_ts, o, o_type, o_bs, o_ts, batch, Sq, Skv, Nh, Nkv,
                       head_dim, mask, window, causal_off, scale, flags, false, 0, 0, 0, stream);
}

extern "C" acb_status acb_attn_prefill_split(const void * q, int64_t q_bs, int64_t q_ts, const void * k, int64_t k_bs,
                                             int64_t k_ts, const void * v, int64_t v_bs, int64_t v_ts, void * o,
                                             int o_type, int64_t o_bs, int64_t o_ts, int batch, int Sq, int Skv,
                                             int Nh, int Nkv, int head_dim, int mask, int window, int causal_off,
                                             float scale, int flags, int64_t q_lo, int64_t k_lo, int64_t v_lo,
                                             acb_stream_t stream) {
    if (q_lo == 0 || k_lo == 0 || v_lo == 0) {
        return ACB_ERR_INVALID_ARG;
    }
    return attn_launch(q, q_bs, q_ts, k, k_bs, k_ts, v, v_bs, v_ts, o, o_type, o_bs, o_ts, batch, Sq, Skv, Nh, Nkv,
                       head_dim, mask, window, causal_off, scale, flags, true, q_lo, k_lo, v_lo, stream);
}
