// k_decode_persist.cu -- one batch-1 greedy decode step of the Qwen3 LM (qw3lm_forward_batch with
// N = 1, src/qwen3-lm.h:557-823, plus the temperature-0 sampler, src/sampling.h:30-34) as a
// single persistent kernel.
//
// Why: at batch 1 every linear is a GEMV that moves a few MB; as separate launches each pays
// a fill/drain of a few microseconds, and a 28-layer step issues ~200 of them. Here one CTA
// per SM (cooperative launch) runs the whole step:
//   - warp 8 of every CTA is a producer that streams ALL of the CTA's weight tiles for the
//     step (each layer's qkv, o, gate|up, down slices, then the head slice) through a ring of
//     35 KB shared-memory slots with 1-D bulk copies. Weights do not depend on activations, so
//     the stream never waits for a layer boundary, only for a free slot;
//   - warps 0-7 are consumers: before each GEMV they build the quantised activation in shared
//     memory (RMSNorm * w, the SwiGLU vector or the attention output, then Q8_0 blocks), then run a dp4a
//     GEMV over their range of Q8_0 tiles (ACB_TYPE_Q8_0_TILES): one activation column makes
//     the int8 MMA of k_gemv.cu a poor fit, and eight independent blocks per warp and stage
//     keep the shared-memory ring draining at HBM rate;
//   - a stage whose input is a whole vector written by other CTAs starts after a grid-wide
//     barrier: one counter in global memory, release-add by each CTA, acquire-poll with a time
//     limit. Six barriers per layer (after qkv, scores, attention, o, gate|up, down);
//   - attention (f16 cache): CTA (kv head h, split s) normalises and rotates its q heads (and,
//     when its split holds the new position, the new k and v, written to the cache), writes
//     scores and the split maximum; after a barrier it forms the f16 probabilities with the
//     global maximum and double sum, its partial P.V, and the last split CTA of the head adds
//     the partials in split order (ticket counter);
//   - the head GEMV keeps a running (best, second, index) per output row lane; CTAs merge
//     theirs, and the last CTA to finish (ticket) writes the token, its margin and history,
//     advances the position and returns the counters to zero for the next step.
// Every wait is bounded. A CTA that gives up sets ACB_DEVERR_TIMEOUT and the barrier word's
// abort bit; every CTA then leaves at its next barrier, and each producer waits for its own
// copies in flight before its CTA exits.
//
// Arithmetic per op is that of the per-op kernels: activation quantisation of quantize_q8_0,
// exact integer dot products per Q8_0 block scaled by d_w * d_x (dp4a here, the int8 MMA of
// gemv_tiles_kernel there), q/k-norm + RoPE of qkv_post_kernel, the two-pass f16-cache softmax
// of attn_scores_kernel / attn_pv_kernel, the argmax of argmax_kernel. Every sum whose order
// the partition decides (8 consumer warps, 4 lanes per row, split count, tile ranges) is formed
// in double from float terms and rounded to float once, so this kernel, the per-op graph and
// the CPU oracle produce the same floats and the same greedy tokens.
#include <cstdlib>
#include <string>

#include "best.cuh"
#include "common.cuh"
#include "ptx.cuh"

namespace acb {

void set_last_error(const std::string & e);

namespace {

constexpr int      kPdWarps       = 8;   // consumer warps
constexpr int      kPdThreads     = (kPdWarps + 1) * 32;
constexpr int      kPdCons        = kPdWarps * 32;
constexpr int      kPdTileBlk     = 544;  // one 16-row x 32-column block of ACB_TYPE_Q8_0_TILES
constexpr int      kPdStageBlocks = 64;
constexpr int      kPdSlot        = kPdStageBlocks * kPdTileBlk;  // 34816 bytes: one K=2048 tile
constexpr int      kPdMaxSlots    = 16;
constexpr int      kPdBpw         = kPdStageBlocks / kPdWarps;  // blocks per warp per stage
constexpr int      kPdMaxK        = 12288;
constexpr int      kPdMaxSplit    = 32;
constexpr int      kPdD           = 128;
constexpr unsigned kAbortBit      = 0x80000000u;
constexpr uint64_t kBarrierNs     = 2000000000ull;  // grid barrier time limit

// shared-memory map (bytes)
constexpr int kSmFull   = 0;     // uint64 full[16]
constexpr int kSmEmpty  = 128;   // uint64 empty[16]
constexpr int kSmRed    = 256;   // double [16][4]
constexpr int kSmMisc   = 768;   // float inv[4], float max[4], int flags (up to byte 808)
constexpr int kSmGate   = 1024;  // float [256] gate rows of this CTA's SwiGLU tiles; residual rows
constexpr int kSmAct    = 2048;  // int8 xq[kPdMaxK] + f16 xd[kPdMaxK/32]; attention scratch
constexpr int kSmTredG  = kSmAct + kPdMaxK + kPdMaxK / 32 * 2;  // double [8 tiles][8 warps][16 rows]
constexpr int kSmRing   = (kSmTredG + kPdWarps * kPdWarps * 16 * 8 + 127) / 128 * 128;
// attention scratch inside the activation region
constexpr int kAtQ      = 0;      // float [G][128] f16-rounded q
constexpr int kAtKp     = 2048;   // float [128] the new k (f16-rounded)
constexpr int kAtAcc    = 2560;   // double4 [8 warps][32] (P.V partials; the combine uses 256)
constexpr int kAtMax    = 10752;  // float [16][G]
static_assert(kAtMax + 16 * 4 * 4 <= kPdMaxK + kPdMaxK / 32 * 2, "attention scratch fits the activation region");

extern __shared__ __align__(128) uint8_t pd_smem[];

// shared-memory regions at constant offsets (no registers held for them)
__device__ __forceinline__ uint64_t * sm_full() { return reinterpret_cast<uint64_t *>(pd_smem + kSmFull); }
__device__ __forceinline__ uint64_t * sm_empty() { return reinterpret_cast<uint64_t *>(pd_smem + kSmEmpty); }
__device__ __forceinline__ double * sm_red() { return reinterpret_cast<double *>(pd_smem + kSmRed); }
__device__ __forceinline__ double * sm_tredd() { return reinterpret_cast<double *>(pd_smem + kSmTredG); }
__device__ __forceinline__ float * sm_misc() { return reinterpret_cast<float *>(pd_smem + kSmMisc); }
__device__ __forceinline__ volatile int * sm_abort() { return reinterpret_cast<volatile int *>(pd_smem + kSmMisc + 32); }
__device__ __forceinline__ volatile int * sm_last() { return reinterpret_cast<volatile int *>(pd_smem + kSmMisc + 36); }
__device__ __forceinline__ uint8_t * sm_act() { return pd_smem + kSmAct; }
__device__ __forceinline__ float * sm_gate() { return reinterpret_cast<float *>(pd_smem + kSmGate); }
__device__ __forceinline__ int8_t * sm_xq() { return reinterpret_cast<int8_t *>(pd_smem + kSmAct); }
// activation block scales: f16 values (the scale is rounded to f16 by the quantiser), stored as f16
__device__ __forceinline__ __half * sm_xd() { return reinterpret_cast<__half *>(pd_smem + kSmAct + kPdMaxK); }
__device__ __forceinline__ uint8_t * sm_ring() { return pd_smem + kSmRing; }

struct PdParams {
    acb_decode_step s;
    int             n_ctas, n_split, slots;
    int             bs_h, bs_q, bs_f;  // K-blocks per ring stage at K = hidden, Nh*D, ffn
    int64_t         prefetch;          // L2 prefetch distance (bytes) ahead of the ring stage
    float *         hidden;
    float *         qkv;
    float *         scores;  // [Nh][max_seq]
    float *         smax;    // [Nh][kPdMaxSplit]
    double *        part;    // [kPdMaxSplit][Nh][D]
    float *         att;     // [Nh*D]
    float *         gu;      // [F] silu(gate) * up
    float4 *        bpart;   // [n_ctas]
    unsigned *      bar;
    int *           done;
    int *           tickets;  // [Nkv]
};

struct ScratchMap {
    size_t hidden, qkv, scores, smax, part, att, gu, bpart, total;
};

ScratchMap scratch_map(const acb_decode_step & s, int n_ctas) {
    auto     al = [](size_t v) { return (v + 255) / 256 * 256; };
    ScratchMap m{};
    size_t   o = 256;  // bar, done, tickets[Nkv]
    const size_t qd = (size_t) s.n_heads * s.head_dim, kvd = (size_t) s.n_kv_heads * s.head_dim;
    m.hidden = o;
    o        = al(o + 4 * (size_t) s.hidden);
    m.qkv    = o;
    o        = al(o + 4 * (qd + 2 * kvd));
    m.scores = o;
    o        = al(o + 4 * (size_t) s.n_heads * s.max_seq);
    m.smax   = o;
    o        = al(o + 4 * (size_t) s.n_heads * kPdMaxSplit);
    m.part   = o;
    o        = al(o + 8 * (size_t) kPdMaxSplit * qd);
    m.att    = o;
    o        = al(o + 4 * qd);
    m.gu     = o;
    o        = al(o + 4 * 2 * (size_t) s.ffn);
    m.bpart  = o;
    o        = al(o + 16 * (size_t) n_ctas);
    m.total  = o;
    return m;
}

__device__ __forceinline__ void cons_sync() {
    asm volatile("bar.sync 1, %0;" ::"r"(kPdCons) : "memory");
}


__device__ __forceinline__ float f16r(float v) {
    return __half2float(__float2half_rn(v));
}

// Balanced tile range of CTA c for GEMV number gi; the assignment rotates with gi so that the
// CTAs holding one more tile differ from GEMV to GEMV.
__device__ __forceinline__ void pd_range(int64_t n_tiles, int gi, int c, int G, int64_t & t0, int64_t & t1) {
    const int v = (c + (int) (((int64_t) gi * 37) % G)) % G;
    t0          = (int64_t) v * n_tiles / G;
    t1          = (int64_t) (v + 1) * n_tiles / G;
}

// ---- producer: the CTA's whole weight stream of the step -----------------------------------
// Byte range of this CTA's tiles of stream segment k of the step: per layer l, segments 5 l +
// {qkv, o, gate rows, up rows, down}; 5 n_layers is the head. Tiles of a range are contiguous,
// blocks in K order. The gate and up pieces of the gate|up weight take the same tile range (a
// CTA owns whole rows of the SwiGLU). gi is the GEMV index that rotates the assignment.
__device__ void pd_segment(const PdParams & P, int k, const uint8_t *& ptr, int64_t & bytes, int & K, int & bs) {
    const acb_decode_step & S  = P.s;
    const int               qd = S.n_heads * S.head_dim;
    const uint8_t *         W;
    int64_t                 n_rows, row0 = 0;
    int                     gi;
    if (k == 5 * S.n_layers) {
        W      = (const uint8_t *) S.head;
        n_rows = S.vocab;
        K      = S.hidden;
        bs     = P.bs_h;
        gi     = 4 * S.n_layers;
    } else {
        const int                l = k / 5;
        const acb_decode_layer & L = S.layers[l];
        switch (k - 5 * l) {
            case 0:
                W      = (const uint8_t *) L.qkv;
                n_rows = qd + 2 * S.n_kv_heads * S.head_dim;
                K      = S.hidden;
                bs     = P.bs_h;
                gi     = 4 * l;
                break;
            case 1:
                W      = (const uint8_t *) L.o;
                n_rows = S.hidden;
                K      = qd;
                bs     = P.bs_q;
                gi     = 4 * l + 1;
                break;
            case 2:
            case 3:
                W      = (const uint8_t *) L.gate_up;
                n_rows = S.ffn;
                row0   = (k - 5 * l == 3) ? S.ffn : 0;
                K      = S.hidden;
                bs     = P.bs_h;
                gi     = 4 * l + 2;
                break;
            default:
                W      = (const uint8_t *) L.down;
                n_rows = S.hidden;
                K      = S.ffn;
                bs     = P.bs_f;
                gi     = 4 * l + 3;
                break;
        }
    }
    int64_t t0, t1;
    pd_range(n_rows / 16, gi, blockIdx.x, P.n_ctas, t0, t1);
    const int64_t tile_bytes = (int64_t) (K / 32) * kPdTileBlk;
    ptr                      = W + (row0 / 16 + t0) * tile_bytes;
    bytes                    = (t1 - t0) * tile_bytes;
}

// The producer thread: ring stages in consumption order, and ahead of them L2 prefetches of
// the same byte stream (P.prefetch bytes ahead of the stage being issued), so that HBM keeps
// streaming while the consumers sit at a grid barrier or in a prologue.
__device__ void pd_producer(const PdParams & P) {
    uint64_t *     full    = sm_full();
    uint64_t *     empty   = sm_empty();
    uint8_t *      ring    = sm_ring();
    volatile int * s_abort = sm_abort();
    const acb_decode_step & S     = P.s;
    const uint64_t          pol   = ptx::policy_evict_first();
    const int               nseg  = (5 * S.n_layers + 1) * max(1, S.n_steps);  // every step streams all weights
    uint32_t                it    = 0;
    bool                    ok    = true;
    // prefetch cursor
    int             pk = 0, pK, pbs;
    int64_t         po = 0, pb, pref = 0, loaded = 0;
    const uint8_t * pp;
    const int       per = 5 * S.n_layers + 1;
    pd_segment(P, 0, pp, pb, pK, pbs);
    for (int k = 0; k < nseg && ok; k++) {
        const uint8_t * W;
        int64_t         seg_bytes;
        int             K, bs;
        pd_segment(P, k % per, W, seg_bytes, K, bs);
        const uint32_t bytes = (uint32_t) bs * kPdTileBlk;
        for (int64_t off = 0; off < seg_bytes && ok; off += bytes) {
            while (pref < loaded + P.prefetch && pk < nseg) {
                if (po >= pb) {
                    if (++pk < nseg) {
                        pd_segment(P, pk % per, pp, pb, pK, pbs);
                        po = 0;
                    }
                    continue;
                }
                const uint32_t n = (uint32_t) min((int64_t) 32768, pb - po);
                ptx::bulk_prefetch_l2(pp + po, n);
                po += n;
                pref += n;
            }
            const int s = (int) (it % (uint32_t) P.slots);
            if (it >= (uint32_t) P.slots) {
                const uint32_t par = ((it / (uint32_t) P.slots) - 1) & 1;
                uint32_t       n   = 0;
                while (!ptx::mbar_try_wait(&empty[s], par)) {
                    if (*s_abort) {
                        ok = false;
                        break;
                    }
                    if (++n > (1u << 24)) {
                        if (S.err) {
                            atomicOr(S.err, ACB_DEVERR_TIMEOUT);
                        }
                        atomicOr(P.bar, kAbortBit);
                        ok = false;
                        break;
                    }
                }
                if (!ok) {
                    break;
                }
            }
            ptx::mbar_arrive_expect_tx(&full[s], bytes);
            ptx::bulk_g2s_stream(ring + (size_t) s * kPdSlot, W + off, bytes, &full[s], pol);
            it++;
            loaded += bytes;
        }
    }
    if (!ok) {
        // the consumers stopped: wait (bounded) for the copies this thread still has in flight
        const uint32_t first = it > (uint32_t) P.slots ? it - (uint32_t) P.slots : 0;
        for (uint32_t i = first; i < it; i++) {
            ptx::mbar_wait(&full[i % (uint32_t) P.slots], (i / (uint32_t) P.slots) & 1);
        }
    }
}

// ---- consumer pieces --------------------------------------------------------------------------
struct PdCtx {
    uint32_t it;     // ring stage counter (the producer's issue order)
    unsigned epoch;  // grid barriers passed
};

// Grid-wide barrier over the consumers of every CTA. Returns false when the step is aborted.
__device__ bool pd_grid_sync(const PdParams & P, PdCtx & x) {
    cons_sync();
    x.epoch++;
    if (threadIdx.x == 0) {
        const unsigned target = x.epoch * (unsigned) P.n_ctas;
        __threadfence();
        unsigned v = *sm_abort() ? (atomicOr(P.bar, kAbortBit) | kAbortBit) : atomicAdd(P.bar, 1u) + 1u;
        if (!(v & kAbortBit) && v < target) {
            const bool done = ptx::poll_bounded<false>(
                P.bar, kBarrierNs, [target](unsigned w) { return (w & kAbortBit) || (w & ~kAbortBit) >= target; },
                v);
            if (!done) {
                if (P.s.err) {
                    atomicOr(P.s.err, ACB_DEVERR_TIMEOUT);
                }
                atomicOr(P.bar, kAbortBit);
                v |= kAbortBit;
            }
        }
        if (v & kAbortBit) {
            *sm_abort() = 1;
        }
        __threadfence();
    }
    cons_sync();
    return *sm_abort() == 0;
}

// Wait for ring stage s; false once the step is aborted (then the caller skips the stage's
// work but keeps every named barrier, so all consumer warps reach the next grid barrier).
__device__ __forceinline__ bool pd_wait_full(const PdParams & P, PdCtx & x, int s, uint32_t par) {
    if (*sm_abort()) {
        return false;
    }
    if (ptx::mbar_wait(&sm_full()[s], par)) {
        return true;
    }
    if ((threadIdx.x & 31) == 0) {
        if (P.s.err) {
            atomicOr(P.s.err, ACB_DEVERR_TIMEOUT);
        }
        atomicOr(P.bar, kAbortBit);
        *sm_abort() = 1;
    }
    return false;
}

enum { ACT_X = 0, ACT_RMS = 1, ACT_EMBED = 3 };

// Activation of K elements -> Q8_0 blocks in shared memory (quantize_q8_0 arithmetic). Thread t
// owns float4 chunks t, t + 512, ...; the 8 chunks of a 32-element block sit in 8 adjacent lanes.
// All loads (activation and norm gains) are issued before the first use.
// Chunks c0 .. c0 + NCH - 1 of every thread; the RMSNorm modes take all chunks in one call.
template <int MODE, int NCH>
__device__ void pd_act_quant_n(const PdParams & P, PdCtx & x, const float * src, const float * w,
                               const uint8_t * erow, int K, float * raw_out, int c0 = 0, bool last = true) {
    const int tid = threadIdx.x, lane = tid & 31;
    const int nf  = K / 4;
    float4    v[NCH], ww[NCH];
#pragma unroll
    for (int i = 0; i < NCH; i++) {
        // loads at a clamped index, then a select (predicated loads cost registers)
        const int f  = tid + (c0 + i) * kPdCons;
        const int fc = min(f, nf - 1);
        ww[i]        = make_float4(1.0f, 1.0f, 1.0f, 1.0f);
        if ((MODE == ACT_RMS || MODE == ACT_EMBED) && w) {
            ww[i] = __ldg(reinterpret_cast<const float4 *>(w) + fc);
        }
        {
            const int f = fc;
            if (MODE == ACT_EMBED) {
                const uint8_t * b = erow + (f >> 3) * 34;
                const float     d = f16_bits_to_f(ld_u16(b));
                const int8_t *  q = reinterpret_cast<const int8_t *>(b + 2 + (f & 7) * 4);
                v[i] = make_float4(__fmul_rn(d, (float) q[0]), __fmul_rn(d, (float) q[1]), __fmul_rn(d, (float) q[2]),
                                   __fmul_rn(d, (float) q[3]));
                if (raw_out) {
                    reinterpret_cast<float4 *>(raw_out)[f] = v[i];
                }
            } else {
                v[i] = __ldcg(reinterpret_cast<const float4 *>(src) + f);
            }
        }
        if (f >= nf) {
            v[i] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
    }
    if (MODE == ACT_RMS || MODE == ACT_EMBED) {
        double ss = 0.0;
#pragma unroll
        for (int i = 0; i < NCH; i++) {
            ss += (double) __fmul_rn(v[i].x, v[i].x);
            ss += (double) __fmul_rn(v[i].y, v[i].y);
            ss += (double) __fmul_rn(v[i].z, v[i].z);
            ss += (double) __fmul_rn(v[i].w, v[i].w);
        }
        ss = warp_sum(ss);
        if (lane == 0) {
            sm_red()[tid >> 5] = ss;
        }
        cons_sync();
        double t = 0.0;
        for (int i = 0; i < kPdWarps; i++) {
            t += sm_red()[i];
        }
        const float sc = rms_scale(t, K, P.s.eps);
#pragma unroll
        for (int i = 0; i < NCH; i++) {
            v[i].x = __fmul_rn(v[i].x, sc);
            v[i].y = __fmul_rn(v[i].y, sc);
            v[i].z = __fmul_rn(v[i].z, sc);
            v[i].w = __fmul_rn(v[i].w, sc);
            if (w) {
                v[i].x = __fmul_rn(v[i].x, ww[i].x);
                v[i].y = __fmul_rn(v[i].y, ww[i].y);
                v[i].z = __fmul_rn(v[i].z, ww[i].z);
                v[i].w = __fmul_rn(v[i].w, ww[i].w);
            }
        }
    }
#pragma unroll
    for (int i = 0; i < NCH; i++) {
        if ((c0 + i) * kPdCons >= nf) {
            break;  // uniform over the CTA
        }
        const int f    = tid + (c0 + i) * kPdCons;
        float     amax = fmaxf(fmaxf(fabsf(v[i].x), fabsf(v[i].y)), fmaxf(fabsf(v[i].z), fabsf(v[i].w)));
        amax           = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
        amax           = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
        amax           = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
        if (f < nf) {
            const float d  = amax / 127.0f;
            const float id = d != 0.0f ? 1.0f / d : 0.0f;
            const int   q0 = (int) roundf(__fmul_rn(v[i].x, id));
            const int   q1 = (int) roundf(__fmul_rn(v[i].y, id));
            const int   q2 = (int) roundf(__fmul_rn(v[i].z, id));
            const int   q3 = (int) roundf(__fmul_rn(v[i].w, id));
            // words of a block stored in the order 0,4,1,5,2,6,3,7: the GEMV lane q reads its
            // words q and 4 + q as one 8-byte load
            const int w = f & 7;
            reinterpret_cast<uint32_t *>(sm_xq())[(f & ~7) + ((w & 3) << 1) + (w >> 2)] =
                (uint32_t) (q0 & 0xff) | ((uint32_t) (q1 & 0xff) << 8) | ((uint32_t) (q2 & 0xff) << 16) |
                ((uint32_t) (q3 & 0xff) << 24);
            if ((f & 7) == 0) {
                sm_xd()[f >> 3] = __float2half_rn(d);
            }
        }
    }
    if (last) {
        cons_sync();
    }
}

template <int MODE>
__device__ __forceinline__ void pd_act_quant(const PdParams & P, PdCtx & x, const float * src, const float * w,
                                             const uint8_t * erow, int K, float * raw_out) {
    if (K <= kPdCons * 8) {
        pd_act_quant_n<MODE, 2>(P, x, src, w, erow, K, raw_out);
    } else if (K <= kPdCons * 16) {
        pd_act_quant_n<MODE, 4>(P, x, src, w, erow, K, raw_out);
    } else if (K <= kPdCons * 24 || MODE != ACT_X) {
        pd_act_quant_n<MODE, 6>(P, x, src, w, erow, K, raw_out);  // RMSNorm widths are at most 6144
    } else {
        // wide plain activations in two batches of six chunks (one register set of the
        // six-chunk form; a twelve-chunk form would spill)
        pd_act_quant_n<MODE, 6>(P, x, src, w, erow, K, raw_out, 0, false);
        pd_act_quant_n<MODE, 6>(P, x, src, w, erow, K, raw_out, 6, true);
    }
}

// EPI_GATE keeps the rows in shared memory; EPI_UP writes silu(gate) * up of the same rows
enum { EPI_STORE = 0, EPI_ADD = 1, EPI_HEAD = 2, EPI_GATE = 3, EPI_UP = 4 };

// Integer partial sums of one 16-row x 32-column tile block for one activation column. Lane
// 4g + q holds bytes 4q..4q+3 and 16+4q..16+4q+3 of rows g and g + 8 (the tile order) and the
// activation words q and 4 + q (xw); two dp4a per row give its partial sum over those 8 columns.
__device__ __forceinline__ void pd_isum(const uint4 & a, uint2 xw, int & s0, int & s1) {
    s0 = __dp4a((int) a.z, (int) xw.y, __dp4a((int) a.x, (int) xw.x, 0));
    s1 = __dp4a((int) a.w, (int) xw.y, __dp4a((int) a.y, (int) xw.x, 0));
}

// Four blocks' partial sums of one row over the 4 lanes q of the row -> lane q holds the whole
// integer sum of block q (a transposing butterfly: 3 shuffles instead of 4 x 2).
__device__ __forceinline__ int pd_transpose4(int v0, int v1, int v2, int v3, int q) {
    const bool hi2 = q & 2, hi1 = q & 1;
    int        x0  = hi2 ? v2 : v0;
    int        x1  = hi2 ? v3 : v1;
    x0 += __shfl_xor_sync(0xffffffffu, hi2 ? v0 : v2, 2);
    x1 += __shfl_xor_sync(0xffffffffu, hi2 ? v1 : v3, 2);
    int z = hi1 ? x1 : x0;
    z += __shfl_xor_sync(0xffffffffu, hi1 ? x0 : x1, 1);
    return z;
}

// Blocks u0..u0+3 of a warp's stage share: lane q turns block u0 + q's integer sums (rows g,
// g + 8) into their float terms (float)isum * (d_w * d_x) and adds them in double. Sums of
// blocks that are not there are zero (their terms add 0).
__device__ __forceinline__ void pd_quad(const int s0[4], const int s1[4], const uint32_t dw[4], const float dx[4],
                                        int q, double & acc0, double & acc2, bool use) {
    const int      t0 = pd_transpose4(s0[0], s0[1], s0[2], s0[3], q);
    const int      t1 = pd_transpose4(s1[0], s1[1], s1[2], s1[3], q);
    const uint32_t w  = q == 0 ? dw[0] : (q == 1 ? dw[1] : (q == 2 ? dw[2] : dw[3]));
    const float    d  = q == 0 ? dx[0] : (q == 1 ? dx[1] : (q == 2 ? dx[2] : dx[3]));
    const float    dl = f16_bits_to_f((uint16_t) (w & 0xffff));
    const float    dh = f16_bits_to_f((uint16_t) (w >> 16));
    if (use) {
        acc0 += (double) __fmul_rn((float) t0, __fmul_rn(dl, d));
        acc2 += (double) __fmul_rn((float) t1, __fmul_rn(dh, d));
    }
}

// Q8_0 tile GEMV over this CTA's tile range for one activation column: warp w takes 8
// consecutive K-blocks of every stage (pd_block), its lanes' partials are added over the 4
// lanes of a row, and the 8 warps' partials of a tile are added in warp order by one warp.
// Residual row of the reducer lane (lane < 16) of warp w for EPI_ADD GEMV gi: y[(t0 + w) * 16 +
// lane]. Requested a whole stage ahead of the GEMV (the rows last changed two barriers earlier),
// so the epilogue finds it in a register.
__device__ __forceinline__ float pd_residual(const PdParams & P, int64_t n_rows, int gi, const float * y) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    int64_t   t0, t1;
    pd_range(n_rows / 16, gi, blockIdx.x, P.n_ctas, t0, t1);
    return (lane < 16 && t0 + warp < t1) ? __ldcg(y + (t0 + warp) * 16 + lane) : 0.0f;
}

template <int EPI>
__device__ __forceinline__ bool pd_gemv(const PdParams & P, PdCtx & x, int64_t n_rows, int K, int bs, int gi, float * y,
                                        Best & best, float resv = 0.0f) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, q = lane & 3;
    int64_t   t0, t1;
    pd_range(n_rows / 16, gi, blockIdx.x, P.n_ctas, t0, t1);
    const int        nb  = K / 32;
    const uint32_t * xq4 = reinterpret_cast<const uint32_t *>(sm_xq());
    if (EPI == EPI_UP) {
        cons_sync();  // the gate GEMV's reducers are done with the partials buffer
    }
    // tiles in groups of (up to) 8: every warp leaves its partials of each tile of the group in
    // shared memory, one named barrier, then warp j adds tile j's partials in warp order
    for (int64_t tg = t0; tg < t1; tg += kPdWarps) {
        const int nt = (int) min((int64_t) kPdWarps, t1 - tg);
        for (int j = 0; j < nt; j++) {
        double acc0 = 0.0, acc2 = 0.0;  // rows g and g + 8: this lane's share of the block terms
        for (int b0 = 0; b0 < nb; b0 += bs) {
            const int       s    = (int) (x.it % (uint32_t) P.slots);
            const bool      have = pd_wait_full(P, x, s, (x.it / (uint32_t) P.slots) & 1);
            const uint8_t * st   = sm_ring() + (size_t) s * kPdSlot;
            // warp w takes nbw consecutive blocks of the stage; every shared-memory operand of
            // its blocks is loaded first. Lane 4g + q holds bytes 4q..4q+3 and 16+4q..16+4q+3 of
            // rows g and g + 8 (the tile order); its two dp4a pairs give those rows' partial sums
            // over its 8 columns; per four blocks the 4 lanes of a row exchange them so that each
            // lane holds one block's whole integer sum and adds that block's float term.
            const int nbw = (bs + kPdWarps - 1) / kPdWarps, bw0 = warp * nbw;
            if (nbw == kPdBpw && bw0 + kPdBpw <= bs && (b0 & 3) == 0) {
                // all of this warp's blocks are in the stage: constant offsets (the f16 scales of
                // blocks bb.. are read as 8-byte aligned quads: bb is a multiple of 4)
                const uint8_t * sp = st + bw0 * kPdTileBlk;
                const int       bb = b0 + bw0;
                uint4           a[kPdBpw];
                uint32_t        dw[kPdBpw];
                uint2           xw[kPdBpw];
#pragma unroll
                for (int u = 0; u < kPdBpw; u++) {
                    a[u]  = *reinterpret_cast<const uint4 *>(sp + u * kPdTileBlk + lane * 16);
                    dw[u] = *reinterpret_cast<const uint32_t *>(sp + u * kPdTileBlk + 512 + g * 4);
                    xw[u] = *reinterpret_cast<const uint2 *>(xq4 + 8 * (bb + u) + 2 * q);
                }
                float dx[kPdBpw];
#pragma unroll
                for (int u = 0; u < kPdBpw; u += 4) {
                    const uint2   d4 = *reinterpret_cast<const uint2 *>(sm_xd() + bb + u);
                    const float2  lo = __half22float2(*reinterpret_cast<const __half2 *>(&d4.x));
                    const float2  hi = __half22float2(*reinterpret_cast<const __half2 *>(&d4.y));
                    dx[u]           = lo.x;
                    dx[u + 1]       = lo.y;
                    dx[u + 2]       = hi.x;
                    dx[u + 3]       = hi.y;
                }
                // the shuffles inside run on every lane; the terms are added only with the stage
#pragma unroll
                for (int u0 = 0; u0 < kPdBpw; u0 += 4) {
                    int s0[4], s1[4];
#pragma unroll
                    for (int u = 0; u < 4; u++) {
                        pd_isum(a[u0 + u], xw[u0 + u], s0[u], s1[u]);
                    }
                    pd_quad(s0, s1, dw + u0, dx + u0, q, acc0, acc2, have);
                }
            } else {
                // ragged stage: indices past it are clamped to its last block (loads stay
                // unconditional: a predicated load sequence costs registers) and their sums zeroed
#pragma unroll
                for (int u0 = 0; u0 < kPdBpw; u0 += 4) {
                    int      s0[4], s1[4];
                    uint32_t dw[4];
                    float    dx[4];
#pragma unroll
                    for (int u = 0; u < 4; u++) {
                        const int   bl = min(bw0 + u0 + u, bs - 1);
                        const int   b  = b0 + bl;
                        const uint4 a  = *reinterpret_cast<const uint4 *>(st + bl * kPdTileBlk + lane * 16);
                        dw[u]          = *reinterpret_cast<const uint32_t *>(st + bl * kPdTileBlk + 512 + g * 4);
                        const uint2 xw = *reinterpret_cast<const uint2 *>(xq4 + 8 * b + 2 * q);
                        dx[u]          = __half2float(sm_xd()[b]);
                        pd_isum(a, xw, s0[u], s1[u]);
                        if (!(u0 + u < nbw && bw0 + u0 + u < bs)) {
                            s0[u] = 0;
                            s1[u] = 0;
                        }
                    }
                    pd_quad(s0, s1, dw, dx, q, acc0, acc2, have);
                }
            }
            __syncwarp();
            if (lane == 0 && have) {
                ptx::mbar_arrive(&sm_empty()[s]);
            }
            x.it++;
        }
        acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
        acc2 += __shfl_xor_sync(0xffffffffu, acc2, 1);
        acc0 += __shfl_xor_sync(0xffffffffu, acc0, 2);
        acc2 += __shfl_xor_sync(0xffffffffu, acc2, 2);
        if (q == 0) {
            double * tr = sm_tredd() + (j * kPdWarps + warp) * 16;
            tr[g]       = acc0;
            tr[g + 8]   = acc2;
        }
        }
        cons_sync();
        if (warp < nt && lane < 16) {
            const int64_t t  = tg + warp;
            const double * tr = sm_tredd() + warp * kPdWarps * 16;
            double         vd = 0.0;
#pragma unroll
            for (int w = 0; w < kPdWarps; w++) {
                vd += tr[w * 16 + lane];
            }
            const float v = (float) vd;
            const int64_t row = t * 16 + lane;
            if (EPI == EPI_ADD) {
                y[row] = __fadd_rn(t - t0 < kPdWarps ? resv : __ldcg(y + row), v);
            } else if (EPI == EPI_GATE) {
                sm_gate()[(t - t0) * 16 + lane] = v;
            } else if (EPI == EPI_UP) {
                y[row] = silu_times(sm_gate()[(t - t0) * 16 + lane], v);
            } else {
                y[row] = v;
            }
            if (EPI == EPI_HEAD) {
                best_push(best, v, (int) row);
            }
        }
        if (tg + kPdWarps < t1) {
            cons_sync();  // the next group reuses the partials buffer
        }
    }
    return *sm_abort() == 0;
}

// q/k RMSNorm (per head, D = 128) and NeoX RoPE of one head by one warp (qkv_post_kernel with
// E = 2): lane owns elements 2*lane + e (a) and 64 + 2*lane + e (b).
__device__ __forceinline__ void pd_norm_rope(const float * src, const float * w, float eps, const float * rope_row,
                                             float a[2], float b[2]) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int e = 0; e < 2; e++) {
        a[e] = __ldcg(src + lane * 2 + e);
        b[e] = __ldcg(src + 64 + lane * 2 + e);
    }
    if (w) {
        double ss = 0.0;
#pragma unroll
        for (int e = 0; e < 2; e++) {
            ss += (double) __fmul_rn(a[e], a[e]);
            ss += (double) __fmul_rn(b[e], b[e]);
        }
        ss             = warp_sum(ss);
        const float sc = rms_scale_pow2<kPdD>(ss, eps);
#pragma unroll
        for (int e = 0; e < 2; e++) {
            a[e] = __fmul_rn(__fmul_rn(a[e], sc), __ldg(w + lane * 2 + e));
            b[e] = __fmul_rn(__fmul_rn(b[e], sc), __ldg(w + 64 + lane * 2 + e));
        }
    }
    const float * cs = rope_row + 4 * lane;
#pragma unroll
    for (int e = 0; e < 2; e++) {
        const float c = __ldg(cs + 2 * e), s = __ldg(cs + 2 * e + 1);
        const float x0 = a[e], x1 = b[e];
        a[e]           = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
        b[e]           = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
    }
}

// Split count of the attention at kv length n: one split per 64 keys, at most one CTA per
// (kv head, split) and kPdMaxSplit. Both passes of a step derive the same value.
__device__ __forceinline__ int pd_splits(const PdParams & P, int n) {
    return min(P.n_split, max(1, (n + 63) / 64));
}

// L2 prefetch of the K and V rows (positions before p) of this CTA's attention split, issued at
// the start of the layer: the cache rows do not depend on the step, and fetching them from HBM
// after the QKV barrier would put an HBM round trip on the critical path twice.
template <int G>
__device__ __forceinline__ void pd_kv_prefetch(const PdParams & P, const acb_decode_layer & L, int p) {
    const acb_decode_step & S = P.s;
    const int               kv_len = p + 1, ns = pd_splits(P, kv_len), c = blockIdx.x;
    if (threadIdx.x != 0 || c >= S.n_kv_heads * ns) {
        return;
    }
    const int     h = c / ns, sp = c % ns, chunk = (kv_len + ns - 1) / ns;
    const int     j0 = sp * chunk, j1 = min(p, j0 + chunk);  // position p is written this step
    const int64_t base = (((int64_t) S.kv_set * S.n_kv_heads + h) * S.max_seq + j0) * kPdD;
    if (j1 > j0) {
        const uint32_t bytes = (uint32_t) (j1 - j0) * kPdD * 2;
        ptx::bulk_prefetch_l2(L.k_cache + base, bytes);
        ptx::bulk_prefetch_l2(L.v_cache + base, bytes);
    }
}

// Attention pass 1 for CTA (kv head h, split s): q heads of the group, the new k/v (by the
// split that holds position p), scores of the split's keys and the split maximum. The split's
// first keys are requested before the q/k work so that their latency overlaps it; key p reads
// the new k from shared memory.
template <int G>
__device__ void pd_attn_scores(const PdParams & P, PdCtx & x, const acb_decode_layer & L, int p) {
    const acb_decode_step & S = P.s;
    const int               c = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int               kv_len = p + 1, ns = pd_splits(P, kv_len);
    if (c >= S.n_kv_heads * ns) {
        return;
    }
    const int     h = c / ns, sp = c % ns, Nh = S.n_heads, Nkv = S.n_kv_heads;
    const int     chunk = (kv_len + ns - 1) / ns;
    const int     j0 = sp * chunk, j1 = min(kv_len, j0 + chunk);
    const int64_t base = ((int64_t) S.kv_set * Nkv + h) * S.max_seq * kPdD;
    uint16_t *    kb   = L.k_cache + base;
    uint16_t *    vb   = L.v_cache + base;
    float *       qf   = reinterpret_cast<float *>(sm_act() + kAtQ);
    float *       kp   = reinterpret_cast<float *>(sm_act() + kAtKp);
    float *       wmax = reinterpret_cast<float *>(sm_act() + kAtMax);
    const float * rope = S.rope + (int64_t) p * kPdD;
    // 8 lanes per key: lane owns dims [16 sub, 16 sub + 16) of key slot ks (attn_scores_kernel);
    // U groups of 4 keys per warp in flight
    constexpr int U   = 2;
    const int     sub = lane & 7, ks = lane >> 3;
    uint4         raw[U][2];
    auto          load_keys = [&](int jb) {
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int     j   = min(jb + kPdWarps * 4 * u + ks, j1 - 1);  // clamped: scored only if in range
            const uint4 * src = reinterpret_cast<const uint4 *>(kb + (int64_t) j * kPdD + 16 * sub);
            raw[u][0]         = __ldcg(src);
            raw[u][1]         = __ldcg(src + 1);
        }
    };
    int jb = j0 + warp * 4;
    load_keys(jb);
    const bool own_p = p >= j0 && p < j1;
    if (warp < G) {
        float a[2], b[2];
        pd_norm_rope(P.qkv + (int64_t) (h * G + warp) * kPdD, L.q_norm, S.eps, rope, a, b);
#pragma unroll
        for (int e = 0; e < 2; e++) {
            qf[warp * kPdD + 2 * lane + e]      = f16r(a[e]);
            qf[warp * kPdD + 64 + 2 * lane + e] = f16r(b[e]);
        }
    } else if (warp == G && own_p) {
        float a[2], b[2];
        pd_norm_rope(P.qkv + (int64_t) (Nh + h) * kPdD, L.k_norm, S.eps, rope, a, b);
        uint16_t * d = kb + (int64_t) p * kPdD;
#pragma unroll
        for (int e = 0; e < 2; e++) {
            const __half ha = __float2half_rn(a[e]), hb = __float2half_rn(b[e]);
            d[2 * lane + e]       = __half_as_ushort(ha);
            d[64 + 2 * lane + e]  = __half_as_ushort(hb);
            kp[2 * lane + e]      = __half2float(ha);
            kp[64 + 2 * lane + e] = __half2float(hb);
        }
    } else if (warp == G + 1 && own_p) {
        const float * src = P.qkv + (int64_t) (Nh + Nkv + h) * kPdD;
        uint16_t *    d   = vb + (int64_t) p * kPdD;
        float         v[4];
#pragma unroll
        for (int e = 0; e < 2; e++) {
            v[e]     = __ldcg(src + 2 * lane + e);
            v[2 + e] = __ldcg(src + 64 + 2 * lane + e);
        }
#pragma unroll
        for (int e = 0; e < 2; e++) {
            d[2 * lane + e]      = __half_as_ushort(__float2half_rn(v[e]));
            d[64 + 2 * lane + e] = __half_as_ushort(__float2half_rn(v[2 + e]));
        }
        // read back by pass 2 through L2 after the grid barrier, whose fence publishes it
    }
    cons_sync();
    float qv[G][16];
#pragma unroll
    for (int g = 0; g < G; g++) {
#pragma unroll
        for (int e = 0; e < 16; e++) {
            qv[g][e] = qf[g * kPdD + 16 * sub + e];
        }
    }
    float mx[G];
#pragma unroll
    for (int g = 0; g < G; g++) {
        mx[g] = -INFINITY;
    }
    for (;;) {
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int j = jb + kPdWarps * 4 * u + ks;
            float     kf[16];
            if (j == p) {
#pragma unroll
                for (int e = 0; e < 16; e++) {
                    kf[e] = kp[16 * sub + e];
                }
            } else {
#pragma unroll
                for (int hh = 0; hh < 2; hh++) {
                    const __half2 * hp = reinterpret_cast<const __half2 *>(&raw[u][hh]);
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        const float2 f        = __half22float2(hp[e]);
                        kf[8 * hh + 2 * e]     = f.x;
                        kf[8 * hh + 2 * e + 1] = f.y;
                    }
                }
            }
#pragma unroll
            for (int g = 0; g < G; g++) {
                // the score order of attn_scores_kernel: 16 dimensions per lane in sequence, then
                // the xor-1/2/4 tree over the key's 8 lanes (products of f16 values are exact)
                float acc = 0.0f;
#pragma unroll
                for (int e = 0; e < 16; e++) {
                    acc = __fadd_rn(acc, __fmul_rn(kf[e], qv[g][e]));
                }
                acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 1));
                acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 2));
                acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, 4));
                const float sv = __fmul_rn(acc, S.attn_scale);
                if (j < j1) {
                    if (sub == 0) {
                        P.scores[(int64_t) (h * G + g) * S.max_seq + j] = sv;
                    }
                    mx[g] = fmaxf(mx[g], sv);
                }
            }
        }
        jb += kPdWarps * 4 * U;
        if (jb >= j1) {
            break;
        }
        load_keys(jb);
    }
#pragma unroll
    for (int g = 0; g < G; g++) {
        mx[g] = warp_max(mx[g]);
    }
    if (lane == 0) {
#pragma unroll
        for (int g = 0; g < G; g++) {
            wmax[warp * G + g] = mx[g];
        }
    }
    cons_sync();
    if (threadIdx.x < G) {
        float m = -INFINITY;
        for (int w = 0; w < kPdWarps; w++) {
            m = fmaxf(m, wmax[w * G + threadIdx.x]);
        }
        P.smax[(int64_t) (h * G + threadIdx.x) * kPdMaxSplit + sp] = m;
    }
}

// Attention pass 2 for CTA (h, s): global max and double sum of the group's rows, f16
// probabilities of the split's keys, partial P.V; the last split CTA of the head adds the
// partials in split order into the attention output. Every loop over memory keeps its loads
// in flight together (a dependent chain of L2 round trips would dominate the step).
template <int G>
__device__ void pd_attn_pv(const PdParams & P, PdCtx & x, const acb_decode_layer & L, int p) {
    const acb_decode_step & S = P.s;
    const int               c = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int               kv_len = p + 1, ns = pd_splits(P, kv_len);
    if (c >= S.n_kv_heads * ns) {
        return;
    }
    constexpr int WPH = kPdWarps / G;  // warps per q head
    constexpr int UV  = 16;            // keys in flight per warp
    const int     h = c / ns, sp = c % ns, Nh = S.n_heads;
    const int     chunk = (kv_len + ns - 1) / ns;
    const int     j0 = sp * chunk, j1 = min(kv_len, j0 + chunk);
    const uint16_t * vb = L.v_cache + ((int64_t) S.kv_set * S.n_kv_heads + h) * S.max_seq * kPdD;
    // warp w serves q head g = w / WPH over keys j0 + (w % WPH) + WPH u; lane owns 4 dims.
    // Its first UV keys (V rows and scores) are requested now: they do not depend on the max.
    const int     g  = warp / WPH, wi = warp % WPH, hq = h * G + g;
    const float * sr = P.scores + (int64_t) hq * S.max_seq;
    // lane l < UV also loads the score of key u = l of the batch: the batch's probabilities are
    // computed once (one per lane) and handed to the other lanes by shuffles
    uint2         vr[UV];
    float         sv;
    auto          load_pv = [&](int jb) {
#pragma unroll
        for (int u = 0; u < UV; u++) {
            const int j = max(j0, min(jb + WPH * u, j1 - 1));  // clamped: used only if in range
            vr[u]       = __ldcg(reinterpret_cast<const uint2 *>(vb + (int64_t) j * kPdD + lane * 4));
        }
        sv = __ldcg(sr + max(j0, min(jb + WPH * (lane % UV), j1 - 1)));
    };
    int jb = j0 + wi;
    load_pv(jb);
    // the first batch of the softmax-sum scores does not depend on the max either
    constexpr int US = 8;
    float         ts[G][US];
#pragma unroll
    for (int gg = 0; gg < G; gg++) {
        const float * r = P.scores + (int64_t) (h * G + gg) * S.max_seq;
#pragma unroll
        for (int u = 0; u < US; u++) {
            ts[gg][u] = __ldcg(r + min(tid + u * kPdCons, kv_len - 1));  // clamped: summed only if in range
        }
    }
    float * sM = sm_misc() + 4;
    if (warp < G) {
        float m = lane < ns ? __ldcg(P.smax + (int64_t) (h * G + warp) * kPdMaxSplit + lane) : -INFINITY;
        m       = warp_max(m);
        if (lane == 0) {
            sM[warp] = m;
        }
    }
    cons_sync();
    float M[G];
#pragma unroll
    for (int gg = 0; gg < G; gg++) {
        M[gg] = sM[gg];
    }
    // sum of expf(s - M) in double over each whole row: thread t takes j = t + 256 i
#pragma unroll
    for (int gg = 0; gg < G; gg++) {
        const float * r = P.scores + (int64_t) (h * G + gg) * S.max_seq;
        double        s = 0.0;
        for (int j = tid; j < kv_len; j += US * kPdCons) {
            float t[US];
#pragma unroll
            for (int u = 0; u < US; u++) {
                t[u] = j == tid ? ts[gg][u] : __ldcg(r + min(j + u * kPdCons, kv_len - 1));
            }
#pragma unroll
            for (int u = 0; u < US; u++) {
                if (j + u * kPdCons < kv_len) {
                    s += (double) acb_expf(__fsub_rn(t[u], M[gg]));
                }
            }
        }
        s = warp_sum(s);
        if (lane == 0) {
            sm_red()[warp * 4 + gg] = s;
        }
    }
    cons_sync();
    if (tid < G) {
        double t = 0.0;
        for (int w = 0; w < kPdWarps; w++) {
            t += sm_red()[w * 4 + tid];
        }
        sm_misc()[tid] = t > 0.0 ? (float) (1.0 / t) : 0.0f;
    }
    cons_sync();
    const float Mg = M[g], ig = sm_misc()[g];
    double4     acc = make_double4(0.0, 0.0, 0.0, 0.0);
    for (;;) {
        const float pl = f16r(__fmul_rn(acb_expf(__fsub_rn(sv, Mg)), ig));  // key jb + WPH * (lane % UV)
#pragma unroll
        for (int u = 0; u < UV; u++) {
            const int    j  = jb + WPH * u;
            const double pp = (double) __shfl_sync(0xffffffffu, pl, u);  // every lane takes part
            if (j < j1) {
                const float2 f01 = __half22float2(*reinterpret_cast<const __half2 *>(&vr[u].x));
                const float2 f23 = __half22float2(*reinterpret_cast<const __half2 *>(&vr[u].y));
                // p * v is exact (two f16 values): the fused multiply-add rounds only the sum
                acc.x = fma(pp, (double) f01.x, acc.x);
                acc.y = fma(pp, (double) f01.y, acc.y);
                acc.z = fma(pp, (double) f23.x, acc.z);
                acc.w = fma(pp, (double) f23.y, acc.w);
            }
        }
        jb += WPH * UV;
        if (jb >= j1) {
            break;
        }
        load_pv(jb);
    }
    double4 * wacc = reinterpret_cast<double4 *>(sm_act() + kAtAcc);
    wacc[warp * 32 + lane] = acc;
    cons_sync();
    if (wi == 0) {
        double4 r = wacc[warp * 32 + lane];
        for (int w = 1; w < WPH; w++) {
            const double4 o = wacc[(warp + w) * 32 + lane];
            r.x += o.x;
            r.y += o.y;
            r.z += o.z;
            r.w += o.w;
        }
        double2 * dst = reinterpret_cast<double2 *>(P.part + ((int64_t) sp * Nh + hq) * kPdD + lane * 4);
        __stcg(dst, make_double2(r.x, r.y));
        __stcg(dst + 1, make_double2(r.z, r.w));
        __threadfence();
    }
    cons_sync();
    if (tid == 0) {
        const int tk = atomicAdd(P.tickets + h, 1);
        *sm_last()    = (tk == ns - 1);
    }
    cons_sync();
    if (!*sm_last()) {
        return;
    }
    // last split CTA of the head: thread (q, g, l) adds splits [q ns / Q, (q + 1) ns / Q) in
    // double, then the Q partial sums are added in double and rounded to float once
    __threadfence();
    constexpr int Q    = kPdWarps / G;  // split ranges (G * 32 * Q == 256)
    constexpr int QMAX = (kPdMaxSplit + Q - 1) / Q;
    const int     q    = tid / (G * 32), gl = tid % (G * 32);
    const int     s0   = q * ns / Q, s1 = (q + 1) * ns / Q;
    const int64_t off  = (int64_t) (h * G) * kPdD + gl * 4;
    double4       a    = make_double4(0.0, 0.0, 0.0, 0.0);
    {
        // every partial of the range requested at once (one L2 round trip on the critical path)
        double2 v[QMAX][2];
#pragma unroll
        for (int i = 0; i < QMAX; i++) {
            const int       si  = min(s0 + i, ns - 1);  // clamped: added only if in the range
            const double2 * src = reinterpret_cast<const double2 *>(P.part + (int64_t) si * Nh * kPdD + off);
            v[i][0]             = __ldcg(src);
            v[i][1]             = __ldcg(src + 1);
        }
#pragma unroll
        for (int i = 0; i < QMAX; i++) {
            if (s0 + i < s1) {
                a.x += v[i][0].x;
                a.y += v[i][0].y;
                a.z += v[i][1].x;
                a.w += v[i][1].y;
            }
        }
    }
    wacc[tid] = a;  // the block reduction above is complete (cons_sync after the ticket)
    cons_sync();
    if (tid < G * 32) {
        double4 r = wacc[tid];
        for (int qq = 1; qq < Q; qq++) {
            const double4 o = wacc[qq * G * 32 + tid];
            r.x += o.x;
            r.y += o.y;
            r.z += o.z;
            r.w += o.w;
        }
        __stcg(reinterpret_cast<float4 *>(P.att + off), make_float4((float) r.x, (float) r.y, (float) r.z, (float) r.w));
        if (tid == 0) {
            P.tickets[h] = 0;
        }
    }
}

template <int G>
__global__ void __launch_bounds__(kPdThreads, 1) lm_decode_kernel(const PdParams P) {
    const acb_decode_step & S = P.s;
    const int               tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    PdCtx                   x;
    x.it      = 0;
    x.epoch   = 0;

    // step inputs: every CTA reads the same values and takes the same exit
    const int n_steps = max(1, S.n_steps);
    const int id0 = __ldcg(S.ids), p0 = __ldcg(S.pos);
    const int p_last  = p0 + n_steps - 1;
    if (id0 < 0 || id0 >= S.embed_rows || p0 < 0 || p_last >= S.max_seq || p_last >= S.max_pos) {
        if (blockIdx.x == 0 && tid == 0 && S.err) {
            atomicOr(S.err, (id0 < 0 || id0 >= S.embed_rows) ? ACB_DEVERR_ID_RANGE : ACB_DEVERR_POS_RANGE);
        }
        return;
    }
    if (tid == 0) {
        for (int s = 0; s < P.slots; s++) {
            ptx::mbar_init(&sm_full()[s], 1);
            ptx::mbar_init(&sm_empty()[s], kPdWarps);
        }
        *sm_abort() = 0;
        *sm_last()  = 0;
        ptx::fence_mbar_init();
    }
    __syncthreads();
    if (warp == kPdWarps) {
        if (lane == 0) {
            pd_producer(P);
        }
        return;
    }

    const int qd = S.n_heads * S.head_dim, qkvd = qd + 2 * S.n_kv_heads * S.head_dim;
    bool      ok = true;
    int       id = id0;
    for (int tok = 0; tok < n_steps; tok++) {
    const int p    = p0 + tok;
    Best      best = { -INFINITY, -INFINITY, 0x7fffffff };
    for (int l = 0; l < S.n_layers && ok; l++) {
        const acb_decode_layer & L = S.layers[l];
        if (l == 0) {
            const uint8_t * erow = (const uint8_t *) S.embed + (int64_t) id * (S.hidden / 32 * 34);
            pd_act_quant<ACT_EMBED>(P, x, nullptr, L.attn_norm, erow, S.hidden, blockIdx.x == 0 ? P.hidden : nullptr);
        } else {
            pd_act_quant<ACT_RMS>(P, x, P.hidden, L.attn_norm, nullptr, S.hidden, nullptr);
        }
        pd_kv_prefetch<G>(P, L, p);
        ok = pd_gemv<EPI_STORE>(P, x, qkvd, S.hidden, P.bs_h, 4 * l, P.qkv, best) && pd_grid_sync(P, x);
        if (!ok) {
            break;
        }
        const float res_o = pd_residual(P, S.hidden, 4 * l + 1, P.hidden);
        pd_attn_scores<G>(P, x, L, p);
        if (!pd_grid_sync(P, x)) {
            break;
        }
        pd_attn_pv<G>(P, x, L, p);
        if (!pd_grid_sync(P, x)) {
            break;
        }
        pd_act_quant<ACT_X>(P, x, P.att, nullptr, nullptr, qd, nullptr);
        ok = pd_gemv<EPI_ADD>(P, x, S.hidden, qd, P.bs_q, 4 * l + 1, P.hidden, best, res_o) && pd_grid_sync(P, x);
        if (!ok) {
            break;
        }
        const float res_d = pd_residual(P, S.hidden, 4 * l + 3, P.hidden);
        pd_act_quant<ACT_RMS>(P, x, P.hidden, L.post_norm, nullptr, S.hidden, nullptr);
        ok = pd_gemv<EPI_GATE>(P, x, S.ffn, S.hidden, P.bs_h, 4 * l + 2, nullptr, best) &&
             pd_gemv<EPI_UP>(P, x, S.ffn, S.hidden, P.bs_h, 4 * l + 2, P.gu, best) && pd_grid_sync(P, x);
        if (!ok) {
            break;
        }
        pd_act_quant<ACT_X>(P, x, P.gu, nullptr, nullptr, S.ffn, nullptr);
        ok = pd_gemv<EPI_ADD>(P, x, S.hidden, S.ffn, P.bs_f, 4 * l + 3, P.hidden, best, res_d) && pd_grid_sync(P, x);
    }
    if (!ok) {
        return;
    }
    pd_act_quant<ACT_RMS>(P, x, P.hidden, S.final_norm, nullptr, S.hidden, nullptr);
    if (!pd_gemv<EPI_HEAD>(P, x, S.vocab, S.hidden, P.bs_h, 4 * S.n_layers, S.logits, best)) {
        return;
    }
    // CTA best -> partial
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        best_merge(best, __shfl_xor_sync(0xffffffffu, best.b1, o), __shfl_xor_sync(0xffffffffu, best.b2, o),
                   __shfl_xor_sync(0xffffffffu, best.i1, o));
    }
    float4 * wb = reinterpret_cast<float4 *>(sm_act());
    if (lane == 0) {
        wb[warp] = make_float4(best.b1, best.b2, __int_as_float(best.i1), 0.0f);
    }
    cons_sync();
    const bool last_step = tok + 1 == n_steps;
    if (tid == 0) {
        Best r = { -INFINITY, -INFINITY, 0x7fffffff };
        for (int w = 0; w < kPdWarps; w++) {
            const float4 v = wb[w];
            best_merge(r, v.x, v.y, __float_as_int(v.z));
        }
        __stcg(P.bpart + blockIdx.x, make_float4(r.b1, r.b2, __int_as_float(r.i1), 0.0f));
        if (last_step) {
            __threadfence();
            const int tk = atomicAdd(P.done, 1);
            *sm_last()    = (tk == P.n_ctas - 1);
        }
    }
    if (!last_step) {
        // a following step of the same launch: after a grid barrier every CTA merges the CTA
        // partials in CTA order (the same triple everywhere), CTA 0 records the token
        if (!pd_grid_sync(P, x)) {
            return;
        }
        if (warp == 0) {
            Best r = { -INFINITY, -INFINITY, 0x7fffffff };
            for (int k = lane; k < P.n_ctas; k += 32) {
                const float4 v = __ldcg(P.bpart + k);
                best_merge(r, v.x, v.y, __float_as_int(v.z));
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                best_merge(r, __shfl_xor_sync(0xffffffffu, r.b1, o), __shfl_xor_sync(0xffffffffu, r.b2, o),
                           __shfl_xor_sync(0xffffffffu, r.i1, o));
            }
            if (lane == 0) {
                *sm_last() = r.i1;  // the next token, for the whole CTA
                if (blockIdx.x == 0 && S.hist && S.hist_base) {
                    const int step = p - S.hist_base[0];
                    S.hist[step]   = r.i1;
                    if (S.mhist) {
                        S.mhist[step] = r.b1 - r.b2;
                    }
                }
            }
        }
        cons_sync();
        id = *sm_last();
        cons_sync();  // every thread has the token before sm_last is written again
        continue;
    }
    cons_sync();
    if (!*sm_last() || warp != 0) {
        return;
    }
    __threadfence();
    Best r = { -INFINITY, -INFINITY, 0x7fffffff };
    for (int k = lane; k < P.n_ctas; k += 32) {
        const float4 v = __ldcg(P.bpart + k);
        best_merge(r, v.x, v.y, __float_as_int(v.z));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        best_merge(r, __shfl_xor_sync(0xffffffffu, r.b1, o), __shfl_xor_sync(0xffffffffu, r.b2, o),
                   __shfl_xor_sync(0xffffffffu, r.i1, o));
    }
    if (lane == 0) {
        if (S.greedy) {
            S.ids[0] = r.i1;
            if (S.margin) {
                S.margin[0] = r.b1 - r.b2;
            }
            if (S.hist && S.hist_base) {
                const int step = p - S.hist_base[0];
                S.hist[step]   = r.i1;
                if (S.mhist) {
                    S.mhist[step] = r.b1 - r.b2;
                }
            }
            S.pos[0] = p + 1;
        }
        // every CTA has passed its last barrier: the counters return to zero for the next step
        *P.done = 0;
        *P.bar  = 0;
    }
    }
}

int blocks_per_stage(int K) {
    const int nb = K / 32;
    int       bs = 1;
    for (int d = 1; d <= kPdStageBlocks && d <= nb; d++) {
        if (nb % d == 0) {
            bs = d;
        }
    }
    return bs;
}

const char * check_shape(const acb_decode_step & s) {
    if (s.head_dim != kPdD) {
        return "head_dim must be 128";
    }
    if (s.n_layers <= 0 || s.n_kv_heads <= 0 || s.n_heads % s.n_kv_heads != 0) {
        return "bad layer or head counts";
    }
    const int G = s.n_heads / s.n_kv_heads;
    if (G != 1 && G != 2 && G != 4) {
        return "q heads per kv head must be 1, 2 or 4";
    }
    if (s.n_kv_heads > 48) {
        return "too many kv heads";
    }
    const int qd = s.n_heads * kPdD;
    for (int k : { s.hidden, s.ffn, qd }) {
        if (k <= 0 || k % 32 != 0 || k > kPdMaxK) {
            return "hidden, ffn and Nh*D must be multiples of 32 up to 12288";
        }
    }
    if (s.hidden > kPdCons * 24) {
        return "hidden must be at most 6144";
    }
    if (s.hidden % 16 != 0 || s.vocab <= 0 || s.vocab % 16 != 0 || s.vocab > 0x7fffffffLL) {
        return "row counts must be multiples of 16";
    }
    if (s.max_seq <= 0 || s.max_pos <= 0) {
        return "bad max_seq / max_pos";
    }
    return nullptr;
}

int num_ctas() {
    return num_sms();
}

}  // namespace
}  // namespace acb

using namespace acb;

extern "C" size_t acb_lm_decode_scratch_bytes(const acb_decode_step * step) {
    if (!step) {
        return 0;
    }
    if (const char * why = check_shape(*step)) {
        set_last_error(std::string("acb_lm_decode: ") + why);
        return 0;
    }
    return scratch_map(*step, num_ctas()).total;
}

extern "C" acb_status acb_lm_decode_step(const acb_decode_step * step, acb_stream_t stream) {
    if (!step || !step->layers || !step->embed || !step->head || !step->final_norm || !step->rope || !step->ids ||
        !step->pos || !step->logits || !step->scratch) {
        return ACB_ERR_INVALID_ARG;
    }
    if (const char * why = check_shape(*step)) {
        set_last_error(std::string("acb_lm_decode: ") + why);
        return ACB_ERR_UNSUPPORTED;
    }
    if (step->greedy && step->hist && !step->hist_base) {
        return ACB_ERR_INVALID_ARG;
    }
    if ((reinterpret_cast<uintptr_t>(step->head) & 15) || (reinterpret_cast<uintptr_t>(step->scratch) & 255)) {
        return ACB_ERR_INVALID_ARG;
    }
    static int max_optin = 0;
    if (max_optin == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&max_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    }
    PdParams P{};
    P.s       = *step;
    P.n_ctas  = num_ctas();
    P.n_split = std::min(kPdMaxSplit, std::max(1, P.n_ctas / step->n_kv_heads));
    P.slots   = std::min(kPdMaxSlots, (max_optin - kSmRing) / kPdSlot);
    if (P.slots < 4) {
        set_last_error("acb_lm_decode: not enough shared memory for the weight ring");
        return ACB_ERR_UNSUPPORTED;
    }
    P.bs_h = blocks_per_stage(step->hidden);
    P.bs_q = blocks_per_stage(step->n_heads * kPdD);
    P.bs_f = blocks_per_stage(step->ffn);
    {
        // prefetch distance: about one layer of this CTA's weights (ACB_PD_PREFETCH_KB overrides)
        const char * env = std::getenv("ACB_PD_PREFETCH_KB");
        P.prefetch       = env ? (int64_t) std::atoi(env) * 1024 : (int64_t) 384 * 1024;
    }
    const ScratchMap m = scratch_map(*step, P.n_ctas);
    uint8_t *        sc = static_cast<uint8_t *>(step->scratch);
    P.bar     = reinterpret_cast<unsigned *>(sc);
    P.done    = reinterpret_cast<int *>(sc + 4);
    P.tickets = reinterpret_cast<int *>(sc + 16);
    P.hidden  = reinterpret_cast<float *>(sc + m.hidden);
    P.qkv     = reinterpret_cast<float *>(sc + m.qkv);
    P.scores  = reinterpret_cast<float *>(sc + m.scores);
    P.smax    = reinterpret_cast<float *>(sc + m.smax);
    P.part    = reinterpret_cast<double *>(sc + m.part);
    P.att     = reinterpret_cast<float *>(sc + m.att);
    P.gu      = reinterpret_cast<float *>(sc + m.gu);
    P.bpart   = reinterpret_cast<float4 *>(sc + m.bpart);

    const int  G     = step->n_heads / step->n_kv_heads;
    const int  smem  = kSmRing + P.slots * kPdSlot;
    void *     kern  = G == 1 ? (void *) lm_decode_kernel<1> : (G == 2 ? (void *) lm_decode_kernel<2> : (void *) lm_decode_kernel<4>);
    cudaError_t e    = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    int         occ  = 0;
    if (e == cudaSuccess) {
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kPdThreads, (size_t) smem);
    }
    if (e != cudaSuccess) {
        set_last_cuda_error(e);
        return ACB_ERR_CUDA;
    }
    if (occ < 1) {
        set_last_error("acb_lm_decode: one CTA per SM does not fit");
        return ACB_ERR_UNSUPPORTED;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim            = dim3((unsigned) P.n_ctas);
    cfg.blockDim           = dim3(kPdThreads);
    cfg.dynamicSmemBytes   = (size_t) smem;
    cfg.stream             = (cudaStream_t) stream;
    cudaLaunchAttribute attr[1];
    attr[0].id              = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs               = attr;
    cfg.numAttrs            = 1;
    void * args[]           = { &P };
    e                       = cudaLaunchKernelExC(&cfg, kern, args);
    if (e != cudaSuccess) {
        set_last_cuda_error(e);
        return ACB_ERR_CUDA;
    }
    return ACB_OK;
}
