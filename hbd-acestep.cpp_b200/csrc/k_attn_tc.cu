// k_attn_tc.cu -- attention over whole sequences on the 5th-generation tensor cores, for the text
// encoder (src/qwen3-enc.h:186-199) and the DiT (src/dit-graph.h:218-231 self-attention with the
// sliding window of the even layers, 339-352 cross-attention):
//     O[b,i,h,:] = softmax_j( Q[b,i,h,:] . K[b,j,h/G,:] * scale + mask(i,j) ) V[b,j,h/G,:]
//
// One CTA per (128 queries, head, batch), 10 warps; the 512 TMEM columns hold two S/P buffers, the
// O accumulator and Q (P and Q are the A operands of the two products, two f16 per 32-bit column),
// so the tensor cores read only K and V from shared memory, and every MMA is N = 128 wide (the
// narrower N = 64 form runs at about two thirds of the tensor rate):
//   warp 0      TMA, two threads: key blocks of 128, K [128][128] and V^T [128][128], into separate
//               rings (a K stage is released as soon as its scores are computed, a V stage after
//               P.V; neither stream waits on the other), 128-byte swizzled K-major tiles;
//   warp 1      one thread issues tcgen05.mma with A from TMEM: S = Q.K^T (M=128 queries, N=128
//               keys) into one of the two S/P buffers, and O += P.V (M=128, N=128 head dims); S for
//               block i+2 is issued right after P.V of block i (the tensor pipe runs them in order,
//               so S(i+2) overwrites the P(i) it aliases only after P.V(i) has read it);
//   warps 2..9  softmax, two threads per query row (its TMEM lane; warps w and w+4 share a lane
//               quarter): each first copies its half of the row's Q into TMEM, then per block
//               takes 64 of the 128 key columns: scores from TMEM, the mask only on blocks that
//               cross a boundary, the block max combined by the pair through shared memory, one
//               FFMA and one ex2 per score (scale folded into log2 e); the reference max moves
//               (and the O row is rescaled, each thread its 64 columns) only when the block max
//               exceeds it by more than 2^8, so P <= 256; P written over the block's S as f16; at
//               the end O divided by the row sum and stored.
// Padding (dit_ggml_generate's masks, dit-sampler.h:244-304): per batch element, only keys below
// kv_len[b] take part (key blocks past it are not loaded) and query rows from q_len[b] on are
// written as zeros -- a row whose keys are all masked has an empty sum, which ggml's flash
// attention turns into a zero output.
// SPLIT: every operand comes as f16 hi and lo planes (hi + lo = the f32 value) and each product is
// lo.hi + hi.lo + hi.hi, P split the same way -- f32-accurate attention (the reference CPU build's
// qwen3_attn_f32 / dit_attn_f32). Every wait is bounded; on a timeout the kernel records
// ACB_DEVERR_TIMEOUT, stops, and still frees its TMEM.
#include <cuda.h>

#include "common.cuh"
#include "ptx.cuh"
#include "tc.cuh"

namespace acb {

constexpr int kTcBQ      = 128;  // queries per CTA = TMEM lanes
constexpr int kTcBK      = 128;  // keys per block
constexpr int kTcD       = 128;  // head dim
constexpr int kTcThreads = 320;  // TMA warp, MMA warp, 8 softmax warps

enum { TC_MASK_NONE = 0, TC_MASK_CAUSAL = 1, TC_MASK_WINDOW = 2 };

struct AttnTcArgs {
    void *  o;
    int     o_type;
    int64_t o_ts;  // O element (b, i, h, d) at (b*Sq + i)*o_ts + h*128 + d
    int     Sq, Skv, Nh, Nkv;
    int     window, causal_off;
    float   scale_log2;
    int *   err;
    int     gemm_a;  // 16-bit output as [hi | hi | lo] planes Nh*128 columns apart
    int64_t o_k;     // Nh*128
    const int * q_len;   // [batch] real query rows, or NULL (all Sq)
    const int * kv_len;  // [batch] real keys, or NULL (all Skv)
};

template <bool SPLIT> struct TcLayout {
    static constexpr int NP    = SPLIT ? 2 : 1;       // operand planes
    static constexpr int KB    = NP * 2 * 16384;      // K block: plane x d-chunk x [128 keys][64 d]
    static constexpr int VB    = NP * 2 * 16384;      // V^T block: plane x key-chunk x [128 d][64 keys]
    static constexpr int NK    = SPLIT ? 2 : 3;       // K ring stages
    static constexpr int NV    = SPLIT ? 1 : 2;       // V ring stages
    static constexpr int QB    = NP * 2 * 16384;      // Q tile: plane x d-chunk x [128 q][64 d]
    static constexpr int TOTAL = NK * KB + NV * VB;   // 192 KB split, 160 KB otherwise
    static_assert(QB <= VB, "the Q tile is staged in V stage 0");
    // TMEM columns (512 allocated): two S/P buffers of 128 columns (S fp32; after the softmax, P
    // as f16 pairs: hi plane in the first 64 columns, lo plane in the next 64), O at 256..383,
    // Q planes (64 columns each: two f16 per column) from 384
    static constexpr uint32_t TO = 256, TQ = 384;
};

// 2^x on the special-function unit (relative error ~2^-22; -inf -> +0, denormal results flush to 0)
__device__ __forceinline__ float ex2_fast(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// lazy rescaling: the reference max of a row moves only when a block max exceeds it by more than
// this many powers of two
constexpr float kRescaleLog2 = 8.0f;

__device__ __forceinline__ bool tc_wait(uint64_t * bar, uint32_t parity, volatile int * abort_flag, int * err) {
    if (*abort_flag) {
        return false;
    }
    if (!ptx::mbar_wait(bar, parity)) {
        *abort_flag = 1;
        if (err) {
            atomicOr(err, ACB_DEVERR_TIMEOUT);
        }
        return false;
    }
    return true;
}

// D (TMEM) += A (TMEM: lane = row, two f16 of K per 32-bit column) x B (shared-memory descriptor)
__device__ __forceinline__ void umma_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
        "r"(tmem_a), "l"(b), "r"(idesc), "r"(acc));
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t * r) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
            taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}

template <int MASK, bool SPLIT>
__global__ void __launch_bounds__(kTcThreads, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap mq, const __grid_constant__ CUtensorMap mql,
                   const __grid_constant__ CUtensorMap mk, const __grid_constant__ CUtensorMap mkl,
                   const __grid_constant__ CUtensorMap mv, const __grid_constant__ CUtensorMap mvl,
                   const AttnTcArgs a) {
    using Lay = TcLayout<SPLIT>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t * smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t * sK   = smem;
    uint8_t * sV   = sK + Lay::NK * Lay::KB;
    uint64_t * q_full   = reinterpret_cast<uint64_t *>(sV + Lay::NV * Lay::VB);
    uint64_t * q_tma    = q_full + 1;  // the Q tile has landed in V stage 0
    uint64_t * k_full   = q_tma + 1;
    uint64_t * k_empty  = k_full + Lay::NK;
    uint64_t * v_full   = k_empty + Lay::NK;
    uint64_t * v_empty  = v_full + Lay::NV;
    uint64_t * s_full   = v_empty + Lay::NV;
    uint64_t * p_full   = s_full + 2;   // [2]: P of block i is published on p_full[i & 1] (a softmax
                                        // warp may run one block ahead of the slowest)
    uint64_t * pv_done  = p_full + 2;   // [2]: P.V of block i completes on pv_done[i & 1]
    uint64_t * o_done   = pv_done + 2;  // the last P.V has completed
    uint64_t * xbar     = o_done + 1;   // [4]: softmax pair exchange, one per TMEM lane quarter
    uint32_t * tmem_slot = reinterpret_cast<uint32_t *>(xbar + 4);
    __shared__ volatile int abort_flag;
    __shared__ float        xchg[2 * 2 * kTcBQ];  // softmax pair exchange: [parity][half][row]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int hk = h / (a.Nh / a.Nkv);
    const int q0 = qt * kTcBQ;

    // key blocks that the mask leaves for this query tile
    int kb_lo = 0, kb_hi = (a.Skv + kTcBK - 1) / kTcBK;
    if (MASK == TC_MASK_CAUSAL) {
        const int last_q = min(q0 + kTcBQ, a.Sq) - 1 + a.causal_off;
        kb_hi            = min(kb_hi, max(0, last_q / kTcBK + 1));
    } else if (MASK == TC_MASK_WINDOW) {
        kb_lo = max(0, (q0 - a.window) / kTcBK);
        kb_hi = min(kb_hi, (min(q0 + kTcBQ, a.Sq) - 1 + a.window) / kTcBK + 1);
    }

    if (threadIdx.x == 0) {
        abort_flag = 0;
        ptx::mbar_init(q_full, 8);  // one arrival per softmax warp once its Q columns are in TMEM
        ptx::mbar_init(q_tma, 1);
        for (int s = 0; s < Lay::NK; s++) {
            ptx::mbar_init(&k_full[s], 1);
            ptx::mbar_init(&k_empty[s], 1);
        }
        for (int s = 0; s < Lay::NV; s++) {
            ptx::mbar_init(&v_full[s], 1);
            ptx::mbar_init(&v_empty[s], 1);
        }
        ptx::mbar_init(&s_full[0], 1);
        ptx::mbar_init(&s_full[1], 1);
        ptx::mbar_init(&p_full[0], 8);  // one arrival per softmax warp
        ptx::mbar_init(&p_full[1], 8);
        ptx::mbar_init(&pv_done[0], 1);
        ptx::mbar_init(&pv_done[1], 1);
        ptx::mbar_init(o_done, 1);
        for (int x = 0; x < 4; x++) {
            ptx::mbar_init(&xbar[x], 2);  // the two warps of a pair
        }
        ptx::fence_mbar_init();
        tma_prefetch_desc(&mq);
        tma_prefetch_desc(&mk);
        tma_prefetch_desc(&mv);
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(ptx::smem_u32(tmem_slot)),
                     "r"(512));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    ptx::grid_dep_wait();
    // padding: the real keys and query rows of this batch element (read after the dependency
    // wait, like every input)
    const int klen = a.kv_len ? max(0, min(__ldg(a.kv_len + b), a.Skv)) : a.Skv;
    const int qlen = a.q_len ? max(0, min(__ldg(a.q_len + b), a.Sq)) : a.Sq;
    kb_hi          = min(kb_hi, (klen + kTcBK - 1) / kTcBK);
    const int nblk = (kb_hi > kb_lo && q0 < qlen) ? kb_hi - kb_lo : 0;
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t tO   = tmem + Lay::TO;
    const uint32_t tQ   = tmem + Lay::TQ;

    if (warp == 0) {
        // two independent producer threads: lane 0 streams K blocks (a stage frees as soon as its
        // scores are computed), lane 16 streams V^T blocks (a stage frees after its P.V)
        if (lane == 0 && nblk > 0) {
            for (int i = 0; i < nblk; i++) {
                const int key0 = (kb_lo + i) * kTcBK;
                const int sk   = i % Lay::NK;
                if (i >= Lay::NK && !tc_wait(&k_empty[sk], ((i / Lay::NK) - 1) & 1, &abort_flag, a.err)) {
                    break;
                }
                uint8_t * kst = sK + sk * Lay::KB;
                ptx::mbar_arrive_expect_tx(&k_full[sk], Lay::KB);
                for (int p = 0; p < Lay::NP; p++) {
                    for (int c = 0; c < 2; c++) {
                        tma_load_2d(kst + (p * 2 + c) * 16384, p ? &mkl : &mk, hk * kTcD + c * 64, b * a.Skv + key0,
                                    &k_full[sk]);
                    }
                }
            }
        } else if (lane == 16 && nblk > 0) {
            // the Q tile (both planes, 64 KB split / 32 KB) goes through V stage 0 on its way to TMEM
            ptx::mbar_arrive_expect_tx(q_tma, Lay::QB);
            for (int p = 0; p < Lay::NP; p++) {
                for (int c = 0; c < 2; c++) {
                    tma_load_2d(sV + (p * 2 + c) * 16384, p ? &mql : &mq, h * kTcD + c * 64, b * a.Sq + q0, q_tma);
                }
            }
            const bool q_copied = tc_wait(q_full, 0, &abort_flag, a.err);
            for (int i = 0; q_copied && i < nblk; i++) {
                const int key0 = (kb_lo + i) * kTcBK;
                const int sv   = i % Lay::NV;
                if (i >= Lay::NV && !tc_wait(&v_empty[sv], ((i / Lay::NV) - 1) & 1, &abort_flag, a.err)) {
                    break;
                }
                uint8_t * vst = sV + sv * Lay::VB;
                ptx::mbar_arrive_expect_tx(&v_full[sv], Lay::VB);
                for (int p = 0; p < Lay::NP; p++) {
                    for (int c = 0; c < 2; c++) {
                        tma_load_2d(vst + (p * 2 + c) * 16384, p ? &mvl : &mv, key0 + c * 64, (b * a.Nkv + hk) * kTcD,
                                    &v_full[sv]);
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && nblk > 0 && tc_wait(q_full, 0, &abort_flag, a.err)) {
            tc_fence_after();
            constexpr uint32_t idesc_s = idesc_kind_f16(128, kTcBK, true);
            constexpr uint32_t idesc_o = idesc_kind_f16(128, kTcD, true);
            // products (A plane, B plane): lo.hi + hi.lo + hi.hi (small terms first), or hi.hi
            constexpr int      n_prod = SPLIT ? 3 : 1;
            const int          pa[3]  = { SPLIT ? 1 : 0, 0, 0 };
            const int          pb[3]  = { 0, SPLIT ? 1 : 0, 0 };
            auto issue_s = [&](int i) -> bool {
                const int sk = i % Lay::NK;
                if (!tc_wait(&k_full[sk], (i / Lay::NK) & 1, &abort_flag, a.err)) {
                    return false;
                }
                tc_fence_after();
                const uint32_t st  = ptx::smem_u32(sK + sk * Lay::KB);
                const uint32_t tS  = tmem + (uint32_t) ((i & 1) * 128);
                uint32_t       acc = 0;
                for (int pr = 0; pr < n_prod; pr++) {
#pragma unroll
                    for (int kk = 0; kk < kTcD / 16; kk++) {
                        const int      c   = kk >> 2;
                        const uint32_t off = (uint32_t) ((kk & 3) * 32);
                        umma_ts(tS, tQ + (uint32_t) (pa[pr] * 64 + kk * 8),
                                smem_desc_sw128(st + (pb[pr] * 2 + c) * 16384 + off), idesc_s, acc);
                        acc = 1;
                    }
                }
                umma_commit(&s_full[i & 1]);
                umma_commit(&k_empty[sk]);  // this K block is consumed
                return true;
            };
            bool ok = issue_s(0) && (nblk < 2 || issue_s(1));
            for (int i = 0; ok && i < nblk; i++) {
                if (!tc_wait(&p_full[i & 1], (i >> 1) & 1, &abort_flag, a.err)) {
                    break;
                }
                const int sv = i % Lay::NV;
                if (!tc_wait(&v_full[sv], (i / Lay::NV) & 1, &abort_flag, a.err)) {
                    break;
                }
                tc_fence_after();
                const uint32_t vt  = ptx::smem_u32(sV + sv * Lay::VB);
                const uint32_t tP  = tmem + (uint32_t) ((i & 1) * 128);  // P aliases this block's S buffer
                uint32_t       acc = i > 0 ? 1u : 0u;
                for (int pr = 0; pr < n_prod; pr++) {
#pragma unroll
                    for (int kk = 0; kk < kTcBK / 16; kk++) {
                        const int      c   = kk >> 2;
                        const uint32_t off = (uint32_t) ((kk & 3) * 32);
                        umma_ts(tO, tP + (uint32_t) (pa[pr] * 64 + kk * 8),
                                smem_desc_sw128(vt + (pb[pr] * 2 + c) * 16384 + off), idesc_o, acc);
                        acc = 1;
                    }
                }
                umma_commit(&pv_done[i & 1]);
                umma_commit(&v_empty[sv]);  // this V block is consumed
                if (i + 1 == nblk) {
                    umma_commit(o_done);
                }
                if (i + 2 < nblk) {
                    ok = issue_s(i + 2);
                }
            }
        }
    } else {
        // softmax: two threads per query row. Warp w (2..9) reads TMEM lane quarter w % 4; half
        // hf = (w - 2) / 4 owns head dims [64 hf, 64 hf + 64) of Q and O and key columns
        // [32 hf, 32 hf + 32) of each block. The pair (same quarter, hence the same TMEM lanes)
        // exchanges row values through TMEM and meets at mbarrier xbar[quarter] (bounded waits,
        // so an abort cannot leave one warp waiting).
        const int      qq    = warp & 3;
        const int      hf    = (warp - 2) >> 2;
        const int      row   = qq * 32 + lane;
        const int      iq    = q0 + row;  // query index within the sequence
        const uint32_t lanes = (uint32_t) (qq * 32) << 16;
        float          m = -INFINITY, l = 0.0f;
        bool           ok = true;
        // this row's Q (dims [64 hf, 64 hf + 64) of each plane) from the swizzled TMA tile in V stage
        // 0 into TMEM, 32 columns per plane (16-byte unit u of row r sits at unit u ^ (r % 8))
        if (nblk == 0) {
            // no key block: nothing to stage (the output rows are zero)
        } else if (__all_sync(0xffffffffu, tc_wait(q_tma, 0, &abort_flag, a.err))) {
#pragma unroll
            for (int p = 0; p < Lay::NP; p++) {
                const uint8_t * src = sV + (p * 2 + hf) * 16384 + row * 128;
                uint32_t        v[32];
#pragma unroll
                for (int u = 0; u < 8; u++) {
                    const uint4 t = *reinterpret_cast<const uint4 *>(src + ((u ^ (row & 7)) << 4));
                    v[4 * u]      = t.x;
                    v[4 * u + 1]  = t.y;
                    v[4 * u + 2]  = t.z;
                    v[4 * u + 3]  = t.w;
                }
                tmem_st32(tQ + lanes + (uint32_t) (p * 64 + hf * 32), v);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                ptx::mbar_arrive(q_full);
            }
        } else {
            ok = false;
        }
        // publish v for `phase`, wait for the partner (bounded), return its value
        auto pair_xchg = [&](int phase, float v, float * other) -> bool {
            xchg[((phase & 1) * 2 + hf) * kTcBQ + row] = v;
            __syncwarp();
            if (lane == 0) {
                ptx::mbar_arrive(&xbar[qq]);
            }
            if (!__all_sync(0xffffffffu, tc_wait(&xbar[qq], phase & 1, &abort_flag, a.err))) {
                return false;
            }
            *other = xchg[((phase & 1) * 2 + (hf ^ 1)) * kTcBQ + row];
            return true;
        };
        // P.V(k) has completed: pv_done[k & 1], phase k >> 1 (waited in order, one phase at a time)
        int  pv_seen0 = 0, pv_seen1 = 0;  // phases of pv_done[0] / pv_done[1] waited
        auto wait_pv  = [&](int k) -> bool {
            const int bb = k & 1, ph = k >> 1;
            int &     seen = bb ? pv_seen1 : pv_seen0;
            if (seen > ph) {
                return true;
            }
            if (!__all_sync(0xffffffffu, tc_wait(&pv_done[bb], ph & 1, &abort_flag, a.err))) {
                return false;
            }
            seen = ph + 1;
            tc_fence_after();
            return true;
        };
        for (int i = 0; i < nblk; i++) {
            // every exit is warp-uniform (tcgen05.ld / st are warp-collective) and pair-uniform
            if (!__all_sync(0xffffffffu, tc_wait(&s_full[i & 1], (i >> 1) & 1, &abort_flag, a.err))) {
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t tS = tmem + lanes + (uint32_t) ((i & 1) * 128);
            uint32_t       r[64];
            tmem_ld32(tS + (uint32_t) (hf * 64), r);
            tmem_ld32(tS + (uint32_t) (hf * 64 + 32), r + 32);
            const int key0 = (kb_lo + i) * kTcBK + hf * 64;
            // the mask, only on a block that crosses a boundary for this row
            bool need = key0 + 64 > klen;
            if (MASK == TC_MASK_CAUSAL) {
                need = need || key0 + 63 > iq + a.causal_off;
            } else if (MASK == TC_MASK_WINDOW) {
                need = need || key0 < iq - a.window || key0 + 63 > iq + a.window;
            }
            if (need) {
#pragma unroll
                for (int c = 0; c < 64; c++) {
                    const int j  = key0 + c;
                    bool      in = j < klen;
                    if (MASK == TC_MASK_CAUSAL) {
                        in = in && j <= iq + a.causal_off;
                    } else if (MASK == TC_MASK_WINDOW) {
                        in = in && (iq > j ? iq - j : j - iq) <= a.window;
                    }
                    if (!in) {
                        r[c] = __float_as_uint(-INFINITY);
                    }
                }
            }
            float mt[8];
#pragma unroll
            for (int c = 0; c < 8; c++) {
                mt[c] = fmaxf(fmaxf(fmaxf(__uint_as_float(r[c]), __uint_as_float(r[c + 8])),
                                    fmaxf(__uint_as_float(r[c + 16]), __uint_as_float(r[c + 24]))),
                              fmaxf(fmaxf(__uint_as_float(r[c + 32]), __uint_as_float(r[c + 40])),
                                    fmaxf(__uint_as_float(r[c + 48]), __uint_as_float(r[c + 56]))));
            }
            const float mh = fmaxf(fmaxf(fmaxf(mt[0], mt[1]), fmaxf(mt[2], mt[3])),
                                   fmaxf(fmaxf(mt[4], mt[5]), fmaxf(mt[6], mt[7])));
            // the pair exchange also orders both threads' reads of this S buffer before either
            // overwrites it with P
            float mo;
            if (!pair_xchg(i, mh, &mo)) {
                ok = false;
                break;
            }
            // running reference max (log2 domain); moves only when exceeded by > 2^kRescaleLog2.
            // Both threads of a row apply the same rule to the same values.
            const float mb    = fmaxf(mh, mo) * a.scale_log2;
            float       alpha = 1.0f;
            bool        resc  = false;
            if (m == -INFINITY) {
                m = mb;  // no mass accumulated yet: O is still zero
            } else if (mb > m + kRescaleLog2) {
                alpha = ex2_fast(m - mb);
                m     = mb;
                resc  = true;
            }
            const float nm = -m;
            float       ps[4] = { 0.0f, 0.0f, 0.0f, 0.0f };
#pragma unroll
            for (int c = 0; c < 64; c++) {
                const float p = m == -INFINITY ? 0.0f : ex2_fast(fmaf(__uint_as_float(r[c]), a.scale_log2, nm));
                r[c]          = __float_as_uint(p);
                ps[c & 3] += p;
            }
            const float ls = (ps[0] + ps[1]) + (ps[2] + ps[3]);
            // P of this half as f16 pairs: hi into r[0..31], lo = f16(p - hi) into r[32..63]
#pragma unroll
            for (int e = 0; e < 32; e++) {
                const float   p0 = __uint_as_float(r[2 * e]), p1 = __uint_as_float(r[2 * e + 1]);
                const __half2 hh = __floats2half2_rn(p0, p1);
                if (SPLIT) {
                    const float2  f2 = __half22float2(hh);
                    const __half2 ll = __floats2half2_rn(p0 - f2.x, p1 - f2.y);
                    r[2 * e + 1]     = *reinterpret_cast<const uint32_t *>(&ll);  // slot 2e+1 is read above
                }
                r[2 * e] = *reinterpret_cast<const uint32_t *>(&hh);
            }
            uint32_t ph[32], pl[32];
#pragma unroll
            for (int e = 0; e < 32; e++) {
                ph[e] = r[2 * e];
                pl[e] = r[2 * e + 1];
            }
            // P.V(i-2) has completed (S(i), already seen, follows it in the in-order tensor pipe):
            // record it, so that every pv_done barrier is waited at most one phase behind
            if (i >= 2 && !wait_pv(i - 2)) {
                ok = false;
                break;
            }
            if (__any_sync(0xffffffffu, resc)) {
                // rescaling O needs P.V(i-1) finished; otherwise P(i) goes out without waiting
                if (!wait_pv(i - 1)) {
                    ok = false;
                    break;
                }
#pragma unroll 1
                for (int c = 0; c < 2; c++) {
                    uint32_t       o[32];
                    const uint32_t col = (uint32_t) (hf * 64 + c * 32);
                    tmem_ld32(tO + lanes + col, o);
#pragma unroll
                    for (int e = 0; e < 32; e++) {
                        o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
                    }
                    tmem_st32(tO + lanes + col, o);
                }
            }
            l = l * alpha + ls;
            // P into this block's S buffer: keys [64 hf, 64 hf + 64) are columns [32 hf, 32 hf + 32)
            // of the hi plane (columns 0..63) and of the lo plane (64..127)
            tmem_st32(tS + (uint32_t) (hf * 32), ph);
            if (SPLIT) {
                tmem_st32(tS + (uint32_t) (64 + hf * 32), pl);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                ptx::mbar_arrive(&p_full[i & 1]);
            }
        }
        if (ok && nblk > 0) {
            ok = __all_sync(0xffffffffu, tc_wait(o_done, 0, &abort_flag, a.err));
            tc_fence_after();
        }
        // row sum of both halves (exchange slot nblk & 1 is free: the last exchange used the other)
        float lo_sum = 0.0f;
        if (ok) {
            ok = pair_xchg(nblk, l, &lo_sum);
        }
        const float lt  = ok ? l + lo_sum : 0.0f;
        const float inv = (ok && lt > 0.0f && iq < qlen) ? 1.0f / lt : 0.0f;
        // O rows through this warp's staging block in the (now idle) K ring, then written as whole
        // row segments: f32, or 16-bit (Q8_0: each 32 columns one block of the output projection's
        // quantised operand, ggml from_float: d = amax / 127 stored as f16, q = round(y / d))
        const int sw  = warp - 2;  // 0..7: rows 32 (w % 4) .. +31, columns 64 hf .. +63
        uint8_t * stg = sK + sw * 9216;
        const bool f32o = a.o_type == ACB_TYPE_F32, bfo = a.o_type == ACB_TYPE_BF16;
#pragma unroll 1
        for (int c = 0; c < 2; c++) {
            uint32_t o[32];
            if (nblk > 0 && ok) {
                tmem_ld32(tO + lanes + (uint32_t) (hf * 64 + c * 32), o);
            } else {
#pragma unroll
                for (int e = 0; e < 32; e++) {
                    o[e] = 0u;
                }
            }
            float y[32];
#pragma unroll
            for (int e = 0; e < 32; e++) {
                y[e] = __uint_as_float(o[e]) * inv;
            }
            if (f32o) {  // [32 rows][64 f32 + 4 pad]
#pragma unroll
                for (int e = 0; e < 32; e += 4) {
                    *reinterpret_cast<float4 *>(stg + lane * 272 + (c * 32 + e) * 4) =
                        make_float4(y[e], y[e + 1], y[e + 2], y[e + 3]);
                }
                continue;
            }
            if (a.o_type == ACB_TYPE_Q8_0) {
                float amax = 0.0f;
#pragma unroll
                for (int e = 0; e < 32; e++) {
                    amax = fmaxf(amax, fabsf(y[e]));
                }
                const float d  = __fdiv_rn(amax, 127.0f);
                const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
                const float dh = __half2float(__float2half_rn(d));
#pragma unroll
                for (int e = 0; e < 32; e++) {
                    y[e] = __fmul_rn(dh, (float) (int) roundf(__fmul_rn(y[e], id)));
                }
            }
            // hi plane [32 rows][64 x 16-bit + 8 pad] at 0, lo plane at 4608
#pragma unroll
            for (int e = 0; e < 32; e += 8) {
                uint32_t hw[4], lw[4];
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const float v0 = y[e + 2 * j], v1 = y[e + 2 * j + 1];
                    if (bfo) {
                        __nv_bfloat162 bb = __floats2bfloat162_rn(v0, v1);
                        const float2   f2 = __bfloat1622float2(bb);
                        __nv_bfloat162 ll = __floats2bfloat162_rn(__fsub_rn(v0, f2.x), __fsub_rn(v1, f2.y));
                        hw[j]             = *reinterpret_cast<uint32_t *>(&bb);
                        lw[j]             = *reinterpret_cast<uint32_t *>(&ll);
                    } else {
                        __half2      hh = __floats2half2_rn(v0, v1);
                        const float2 f2 = __half22float2(hh);
                        __half2      ll = __floats2half2_rn(__fsub_rn(v0, f2.x), __fsub_rn(v1, f2.y));
                        hw[j]           = *reinterpret_cast<uint32_t *>(&hh);
                        lw[j]           = *reinterpret_cast<uint32_t *>(&ll);
                    }
                }
                const int off = lane * 144 + (c * 32 + e) * 2;
                *reinterpret_cast<uint4 *>(stg + off)        = make_uint4(hw[0], hw[1], hw[2], hw[3]);
                *reinterpret_cast<uint4 *>(stg + 4608 + off) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
            }
        }
        __syncwarp();
        const int64_t row0 = (int64_t) b * a.Sq + q0 + qq * 32;  // global row of this warp's first row
        const int     rmax = a.Sq - (q0 + qq * 32);               // rows of this warp inside the sequence
        const int64_t col0 = (int64_t) h * kTcD + hf * 64;
        if (f32o) {
            // 16 lanes x 16 bytes per row, 2 rows per pass
#pragma unroll 4
            for (int it = 0; it < 16; it++) {
                const int rr = it * 2 + (lane >> 4), cc = (lane & 15) * 4;
                if (rr < rmax) {
                    *reinterpret_cast<float4 *>(reinterpret_cast<float *>(a.o) + (row0 + rr) * a.o_ts + col0 + cc) =
                        *reinterpret_cast<const float4 *>(stg + rr * 272 + cc * 4);
                }
            }
        } else {
            // 8 lanes x 16 bytes per row, 4 rows per pass; GEMM_A: hi twice, then lo
            const int nplanes = a.gemm_a ? 3 : 1;
            for (int pl = 0; pl < nplanes; pl++) {
                const int src_off = pl == 2 ? 4608 : 0;
                const int64_t dc  = col0 + (int64_t) pl * a.o_k;
#pragma unroll 4
                for (int it = 0; it < 8; it++) {
                    const int rr = it * 4 + (lane >> 3), cc = (lane & 7) * 8;
                    if (rr < rmax) {
                        *reinterpret_cast<uint4 *>(reinterpret_cast<uint16_t *>(a.o) + (row0 + rr) * a.o_ts + dc + cc) =
                            *reinterpret_cast<const uint4 *>(stg + src_off + rr * 144 + cc * 2);
                    }
                }
            }
        }
    }
    ptx::grid_dep_launch();
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512));
    }
}

// V (f32 or f16, element (b, t, hk, d) at b*v_bs + t*v_ts + hk*128 + d) to V^T planes:
// vt[((b*Nkv + hk)*128 + d)*vt_ld + t] = f16(v) and, with lo_off, vt[lo_off + same] = f16(v - hi).
// A 32-token x 32-dim tile per block, transposed through shared memory.
template <int TI>
__global__ void __launch_bounds__(256) vt_planes_kernel(const void * __restrict__ v, int64_t v_bs, int64_t v_ts,
                                                        int S, int Nkv, uint16_t * __restrict__ vt, int64_t vt_ld,
                                                        int64_t lo_off) {
    __shared__ float tile[32][33];
    const int t0 = blockIdx.x * 32, dc = blockIdx.y, bh = blockIdx.z;  // bh = b*Nkv + hk; dc = 32-dim chunk
    const int b = bh / Nkv, hk = bh - b * Nkv;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 8 rows per pass
    using ei    = typename io<TI>::t;
    const ei * src = reinterpret_cast<const ei *>(v) + (int64_t) b * v_bs + (int64_t) hk * kTcD + dc * 32;
    for (int r = ty; r < 32; r += 8) {
        const int t = t0 + r;
        tile[r][tx] = t < S ? io<TI>::to_f(src[(int64_t) t * v_ts + tx]) : 0.0f;
    }
    __syncthreads();
    for (int r = ty; r < 32; r += 8) {
        const int t = t0 + tx;
        if (t < S) {
            const float   x   = tile[tx][r];
            const __half  hi  = __float2half_rn(x);
            const int64_t idx = ((int64_t) bh * kTcD + dc * 32 + r) * vt_ld + t;
            vt[idx]           = __half_as_ushort(hi);
            if (lo_off) {
                vt[lo_off + idx] = __half_as_ushort(__float2half_rn(x - __half2float(hi)));
            }
        }
    }
}

}  // namespace acb

using namespace acb;

extern "C" acb_status acb_attn_vt(const void * v, int v_type, int64_t v_bs, int64_t v_ts, int batch, int S, int Nkv,
                                  int head_dim, void * vt, int64_t vt_ld, int64_t lo_offset, acb_stream_t stream) {
    if (!v || !vt || batch <= 0 || S <= 0 || Nkv <= 0 || vt_ld < S || lo_offset < 0) {
        return ACB_ERR_INVALID_ARG;
    }
    if (head_dim != kTcD || (v_type != ACB_TYPE_F32 && v_type != ACB_TYPE_F16)) {
        return ACB_ERR_UNSUPPORTED;
    }
    const dim3 grid((unsigned) ((S + 31) / 32), kTcD / 32, (unsigned) (batch * Nkv));
    if (v_type == ACB_TYPE_F32) {
        vt_planes_kernel<ACB_TYPE_F32><<<grid, 256, 0, (cudaStream_t) stream>>>(
            v, v_bs, v_ts, S, Nkv, reinterpret_cast<uint16_t *>(vt), vt_ld, lo_offset);
    } else {
        vt_planes_kernel<ACB_TYPE_F16><<<grid, 256, 0, (cudaStream_t) stream>>>(
            v, v_bs, v_ts, S, Nkv, reinterpret_cast<uint16_t *>(vt), vt_ld, lo_offset);
    }
    return launch_status();
}

extern "C" acb_status acb_attn_tc_masked(const void * q, int64_t q_ts, const void * k, int64_t k_ts,
                                         const void * vt, int64_t vt_ld, void * o, int o_type, int64_t o_ts, int batch,
                                         int Sq, int Skv, int Nh, int Nkv, int head_dim, int mask, int window,
                                         int causal_off, float scale, int flags, int64_t q_lo, int64_t k_lo,
                                         int64_t vt_lo, const int * q_len, const int * kv_len, int * err_flag,
                                         acb_stream_t stream) {
    if (!q || !k || !vt || !o || batch <= 0 || Sq <= 0 || Skv <= 0 || Nh <= 0 || Nkv <= 0 || Nh % Nkv != 0 ||
        vt_ld < Skv) {
        return ACB_ERR_INVALID_ARG;
    }
    if (head_dim != kTcD || mask < 0 || mask > 2 ||
        (o_type != ACB_TYPE_F32 && o_type != ACB_TYPE_BF16 && o_type != ACB_TYPE_F16 && o_type != ACB_TYPE_Q8_0)) {
        return ACB_ERR_UNSUPPORTED;
    }
    const bool gemm_a = (flags & ACB_FLAG_GEMM_A) != 0;
    if (gemm_a && (o_type == ACB_TYPE_F32 || o_ts < 3 * (int64_t) Nh * kTcD)) {
        return ACB_ERR_INVALID_ARG;
    }
    const bool split = q_lo != 0 || k_lo != 0 || vt_lo != 0;
    if (split && (q_lo == 0 || k_lo == 0 || vt_lo == 0)) {
        return ACB_ERR_INVALID_ARG;
    }
    // TMA: 16-byte aligned bases and row strides; outputs of 16-byte units
    if ((q_ts | k_ts | vt_ld | q_lo | k_lo | vt_lo) % 8 != 0 || o_ts % 8 != 0 ||
        reinterpret_cast<uintptr_t>(q) % 16 || reinterpret_cast<uintptr_t>(k) % 16 ||
        reinterpret_cast<uintptr_t>(vt) % 16 || reinterpret_cast<uintptr_t>(o) % 16) {
        return ACB_ERR_UNSUPPORTED;
    }
    const uint16_t * q16 = reinterpret_cast<const uint16_t *>(q);
    const uint16_t * k16 = reinterpret_cast<const uint16_t *>(k);
    const uint16_t * v16 = reinterpret_cast<const uint16_t *>(vt);
    CUtensorMap      mq, mql, mk, mkl, mv, mvl;
    const int64_t    kc = (int64_t) Nkv * kTcD;
    bool ok = make_map_2d(&mq, q16, true, (int64_t) Nh * kTcD, (int64_t) batch * Sq, q_ts, 64, kTcBQ) &&
              make_map_2d(&mk, k16, true, kc, (int64_t) batch * Skv, k_ts, 64, kTcBK) &&
              make_map_2d(&mv, v16, true, Skv, (int64_t) batch * Nkv * kTcD, vt_ld, 64, kTcD);
    if (split) {
        ok = ok && make_map_2d(&mql, q16 + q_lo, true, (int64_t) Nh * kTcD, (int64_t) batch * Sq, q_ts, 64, kTcBQ) &&
             make_map_2d(&mkl, k16 + k_lo, true, kc, (int64_t) batch * Skv, k_ts, 64, kTcBK) &&
             make_map_2d(&mvl, v16 + vt_lo, true, Skv, (int64_t) batch * Nkv * kTcD, vt_ld, 64, kTcD);
    } else {
        mql = mq;
        mkl = mk;
        mvl = mv;
    }
    if (!ok) {
        return ACB_ERR_CUDA;
    }
    AttnTcArgs a = {};
    a.o          = o;
    a.o_type     = o_type;
    a.o_ts       = o_ts;
    a.Sq         = Sq;
    a.Skv        = Skv;
    a.Nh         = Nh;
    a.Nkv        = Nkv;
    a.window     = window;
    a.causal_off = causal_off;
    a.scale_log2 = scale * 1.4426950408889634f;
    a.err        = err_flag;
    a.gemm_a     = gemm_a ? 1 : 0;
    a.o_k        = (int64_t) Nh * kTcD;
    a.q_len      = q_len;
    a.kv_len     = kv_len;
    const size_t smem = (size_t) (split ? TcLayout<true>::TOTAL : TcLayout<false>::TOTAL) + 1024 + 256;
    void (*kern)(const CUtensorMap, const CUtensorMap, const CUtensorMap, const CUtensorMap, const CUtensorMap,
                 const CUtensorMap, const AttnTcArgs) = nullptr;
#define ACB_TC_PICK(M) kern = split ? attn_tc_kernel<M, true> : attn_tc_kernel<M, false>
    if (mask == TC_MASK_CAUSAL) {
        ACB_TC_PICK(TC_MASK_CAUSAL);
    } else if (mask == TC_MASK_WINDOW) {
        ACB_TC_PICK(TC_MASK_WINDOW);
    } else {
        ACB_TC_PICK(TC_MASK_NONE);
    }
#undef ACB_TC_PICK
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim            = dim3((unsigned) ((Sq + kTcBQ - 1) / kTcBQ), (unsigned) Nh, (unsigned) batch);
    cfg.blockDim           = dim3(kTcThreads);
    cfg.dynamicSmemBytes   = smem;
    cfg.stream             = (cudaStream_t) stream;
    cudaLaunchAttribute attr[1];
    attr[0].id                                         = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs                                          = (flags & ACB_FLAG_PDL) ? attr : nullptr;
    cfg.numAttrs                                       = (flags & ACB_FLAG_PDL) ? 1 : 0;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, mq, mql, mk, mkl, mv, mvl, a);
    if (e != cudaSuccess) {
        set_last_cuda_error(e);
        return ACB_ERR_CUDA;
    }
    return ACB_OK;
}

extern "C" acb_status acb_attn_tc(const void * q, int64_t q_ts, const void * k, int64_t k_ts, const void * vt,
                                  int64_t vt_ld, void * o, int o_type, int64_t o_ts, int batch, int Sq, int Skv,
                                  int Nh, int Nkv, int head_dim, int mask, int window, int causal_off, float scale,
                                  int flags, int64_t q_lo, int64_t k_lo, int64_t vt_lo, int * err_flag,
                                  acb_stream_t stream) {
    return acb_attn_tc_masked(q, q_ts, k, k_ts, vt, vt_ld, o, o_type, o_ts, batch, Sq, Skv, Nh, Nkv, head_dim, mask,
                              window, causal_off, scale, flags, q_lo, k_lo, vt_lo, nullptr, nullptr, err_flag, stream);
}
