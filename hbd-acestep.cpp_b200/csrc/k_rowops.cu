// k_rowops.cu -- row-wise ops of the op-chain: RMSNorm (+weight), adaLN modulate (with the
// fused RMSNorm), per-head q/k RMSNorm + NeoX RoPE with strided / KV-cache destinations.
//
// All three are HBM-bound: a CTA owns a row at a time (a warp takes a few heads), the row is
// loaded once with vector loads into registers, reduced with shuffles, and written once. The
// sum of squares is accumulated in double (the ggml-CPU rule), which makes the normalisation
// scale identical to the CPU's; products and sums that ggml performs as separate graph nodes
// are kept separately rounded (__fmul_rn / __fadd_rn) so no multiply-add is contracted.
#include <type_traits>

#include "common.cuh"

namespace acb {

// ---- vector store of N floats into an I/O type (N*size = 8, 16 or 32 bytes) ---------------
template <int TO, int N> __device__ __forceinline__ void store_n(void * p, const float * f) {
    using e = typename io<TO>::t;
    constexpr int B = N * (int) sizeof(e);
    static_assert(B == 8 || B == 16 || B == 32, "store width");
    union {
        uint4 u[B >= 16 ? B / 16 : 1];
        uint2 h;
        e     v[N];
    } s;
#pragma unroll
    for (int i = 0; i < N; i++) {
        s.v[i] = io<TO>::from_f(f[i]);
    }
    if constexpr (B == 8) {
        *reinterpret_cast<uint2 *>(p) = s.h;
    } else {
#pragma unroll
        for (int i = 0; i < B / 16; i++) {
            reinterpret_cast<uint4 *>(p)[i] = s.u[i];
        }
    }
}

template <int N> __device__ __forceinline__ void load_w(const float * w, float * out) {
#pragma unroll
    for (int i = 0; i < N; i += 4) {
        float4 t   = __ldg(reinterpret_cast<const float4 *>(w + i));
        out[i]     = t.x;
        out[i + 1] = t.y;
        out[i + 2] = t.z;
        out[i + 3] = t.w;
    }
}

// ---- RMSNorm / adaLN: a CTA per row at a time, grid-stride with one row of lookahead -------
// MODE 0: y = rms_norm(x)*w (w may be null)
// MODE 1: y = (w ? rms_norm(x)*w : x) * (1 + scale) + shift
// A row is spread over the CTA (V 16-byte vectors per thread, vector i*blockDim + tid). The grid
// is as many CTAs as fit on the SMs at once; each walks rows r, r + grid, ... and loads the next
// row while it reduces, scales and stores the current one, so HBM reads never stop for the
// reduction or for launching a new CTA. The double sum of squares is reduced with warp shuffles,
// then over the warps' sums in warp order.
template <int TI, int TO, int V, int MODE>
__global__ void __launch_bounds__(512) row_norm_cta_kernel(const void * __restrict__ x, int64_t xs,
                                                            const float * __restrict__ w, void * __restrict__ y,
                                                            int64_t ys, int64_t rows, int cols, float eps,
                                                            const float * __restrict__ scale,
                                                            const float * __restrict__ shift, int64_t vec_stride,
                                                            int64_t rows_per_sample) {
    using VI          = vec16<TI>;
    constexpr int N   = VI::N;
    using ei          = typename io<TI>::t;
    using eo          = typename io<TO>::t;
    __shared__ double red[2][32];  // two slots: a fast warp may start the next row's sum early
    const int     tid     = threadIdx.x;
    const int     nt      = blockDim.x;
    const int     nvec    = cols / N;
    const bool    do_norm = (MODE == 0) || (w != nullptr);
    const int64_t stride  = gridDim.x;

    VI cur[V], nxt[V];
    int64_t row = blockIdx.x;
    if (row >= rows) {
        return;
    }
    {
        const char * xr = reinterpret_cast<const char *>(x) + row * xs * (int64_t) sizeof(ei);
#pragma unroll
        for (int i = 0; i < V; i++) {
            const int vi = tid + i * nt;
            if (vi < nvec) {
                cur[i].load_stream(xr + (int64_t) vi * 16);
            }
        }
    }
    for (int it = 0; row < rows; row += stride, it ^= 1) {
        const int64_t nrow = row + stride;
        if (nrow < rows) {
            const char * xr = reinterpret_cast<const char *>(x) + nrow * xs * (int64_t) sizeof(ei);
#pragma unroll
            for (int i = 0; i < V; i++) {
                const int vi = tid + i * nt;
                if (vi < nvec) {
                    nxt[i].load_stream(xr + (int64_t) vi * 16);
                }
            }
        }
        float sc = 1.0f;
        if (do_norm) {
            double ss = 0.0;
#pragma unroll
            for (int i = 0; i < V; i++) {
                if (tid + i * nt < nvec) {
#pragma unroll
                    for (int j = 0; j < N; j++) {
                        const float f = cur[i].get(j);
                        ss += (double) __fmul_rn(f, f);
                    }
                }
            }
            ss = warp_sum(ss);
            if ((tid & 31) == 0) {
                red[it][tid >> 5] = ss;
            }
            __syncthreads();
            double t = 0.0;
            for (int k = 0; k < (nt >> 5); k++) {  // every thread sums the warps' sums in warp order
                t += red[it][k];
            }
            sc = rms_scale(t, cols, eps);
        }
        const float * scl = nullptr;
        const float * shf = nullptr;
        if (MODE == 1) {
            const int64_t smp = row / rows_per_sample;
            scl               = scale + smp * vec_stride;
            shf               = shift + smp * vec_stride;
        }
        char * yr = reinterpret_cast<char *>(y) + row * ys * (int64_t) sizeof(eo);
#pragma unroll
        for (int i = 0; i < V; i++) {
            const int vi = tid + i * nt;
            if (vi < nvec) {
                float o[N];
                float wv[N];
                if (w) {
                    load_w<N>(w + (int64_t) vi * N, wv);
                }
#pragma unroll
                for (int j = 0; j < N; j++) {
                    float f = cur[i].get(j);
                    if (do_norm) {
                        f = __fmul_rn(f, sc);
                        if (w) {
                            f = __fmul_rn(f, wv[j]);
                        }
                    }
                    o[j] = f;
                }
                if (MODE == 1) {
                    float a[N], b[N];
                    load_w<N>(scl + (int64_t) vi * N, a);
                    load_w<N>(shf + (int64_t) vi * N, b);
#pragma unroll
                    for (int j = 0; j < N; j++) {
                        o[j] = __fadd_rn(__fmul_rn(o[j], __fadd_rn(a[j], 1.0f)), b[j]);
                    }
                }
                store_n<TO, N>(yr + (int64_t) vi * N * (int64_t) sizeof(eo), o);
            }
        }
#pragma unroll
        for (int i = 0; i < V; i++) {
            cur[i] = nxt[i];
        }
    }
}

// Fallback for unaligned / odd-width rows: scalar loads, two passes over the row.
template <int TI, int TO, int MODE>
__global__ void __launch_bounds__(256) row_norm_scalar_kernel(const void * __restrict__ x, int64_t xs,
                                                              const float * __restrict__ w, void * __restrict__ y,
                                                              int64_t ys, int64_t rows, int cols, float eps,
                                                              const float * __restrict__ scale,
                                                              const float * __restrict__ shift, int64_t vec_stride,
                                                              int64_t rows_per_sample) {
    using ei           = typename io<TI>::t;
    using eo           = typename io<TO>::t;
    const int     lane = threadIdx.x & 31;
    const int64_t row  = (int64_t) blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= rows) {
        return;
    }
    const ei * xr      = reinterpret_cast<const ei *>(x) + row * xs;
    eo *       yr      = reinterpret_cast<eo *>(y) + row * ys;
    const bool do_norm = (MODE == 0) || (w != nullptr);
    double     ss      = 0.0;
    if (do_norm) {
        for (int i = lane; i < cols; i += 32) {
            float f = io<TI>::to_f(xr[i]);
            ss += (double) __fmul_rn(f, f);
        }
        ss = warp_sum(ss);
    }
    const float   sc = do_norm ? rms_scale(ss, cols, eps) : 1.0f;
    const int64_t s  = MODE == 1 ? row / rows_per_sample : 0;
    for (int i = lane; i < cols; i += 32) {
        float f = io<TI>::to_f(xr[i]);
        if (do_norm) {
            f = __fmul_rn(f, sc);
            if (w) {
                f = __fmul_rn(f, w[i]);
            }
        }
        if (MODE == 1) {
            f = __fadd_rn(__fmul_rn(f, __fadd_rn(scale[s * vec_stride + i], 1.0f)), shift[s * vec_stride + i]);
        }
        yr[i] = io<TO>::from_f(f);
    }
}

template <int TI, int TO, int MODE>
static acb_status launch_row_norm(const void * x, int64_t xs, const float * w, void * y, int64_t ys, int64_t rows,
                                  int cols, float eps, const float * scale, const float * shift, int64_t vs,
                                  int64_t rps, cudaStream_t st) {
    constexpr int NI    = vec16<TI>::N;
    const int     warps = 8;
    const dim3    grid((unsigned) ((rows + warps - 1) / warps));
    const int     si = (int) sizeof(typename io<TI>::t), so = (int) sizeof(typename io<TO>::t);
    const bool    aligned = cols % NI == 0 && (reinterpret_cast<uintptr_t>(x) % 16) == 0 &&
                         (reinterpret_cast<uintptr_t>(y) % 16) == 0 && (xs * si) % 16 == 0 && (ys * so) % 16 == 0 &&
                         (w == nullptr || reinterpret_cast<uintptr_t>(w) % 16 == 0) &&
                         (MODE == 0 || ((reinterpret_cast<uintptr_t>(scale) % 16) == 0 &&
                                        (reinterpret_cast<uintptr_t>(shift) % 16) == 0 && vs % 4 == 0)) &&
                         (NI * so) >= 8;
    const int nvec = cols / NI;
    // vectors per thread: 4 for f32 rows, 2 for 16-bit rows (8 elements a vector, whose per-column
    // weight / scale / shift floats would otherwise cost registers and occupancy)
    constexpr int V = NI == 4 ? 4 : 2;
    if (aligned && nvec <= V * 512) {
        // a row per CTA at a time: 32..512 threads; as many CTAs as are resident at once (per
        // block size, cached)
        const int threads = ((nvec + V * 32 - 1) / (V * 32)) * 32;
        static int resident[17];
        int &      res = resident[threads / 32];
        if (res == 0) {
            int per_sm = 0;
            if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, row_norm_cta_kernel<TI, TO, V, MODE>, threads,
                                                              0) != cudaSuccess ||
                per_sm < 1) {
                per_sm = 1;
            }
            res = per_sm * num_sms();
        }
        const int64_t nb = rows < res ? rows : res;
        row_norm_cta_kernel<TI, TO, V, MODE><<<dim3((unsigned) nb), threads, 0, st>>>(x, xs, w, y, ys, rows, cols,
                                                                                   eps, scale, shift, vs, rps);
    } else {
        row_norm_scalar_kernel<TI, TO, MODE><<<grid, warps * 32, 0, st>>>(x, xs, w, y, ys, rows, cols, eps, scale,
                                                                          shift, vs, rps);
    }
    return launch_status();
}

template <int MODE>
static acb_status dispatch_row_norm(int ti, int to, const void * x, int64_t xs, const float * w, void * y,
                                    int64_t ys, int64_t rows, int cols, float eps, const float * scale,
                                    const float * shift, int64_t vs, int64_t rps, cudaStream_t st) {
#define ACB_RN(A, B)                                                                                          \
    if (ti == A && to == B) {                                                                                 \
        return launch_row_norm<A, B, MODE>(x, xs, w, y, ys, rows, cols, eps, scale, shift, vs, rps, st);      \
    }
    ACB_RN(ACB_TYPE_F32, ACB_TYPE_F32)
    ACB_RN(ACB_TYPE_F32, ACB_TYPE_BF16)
    ACB_RN(ACB_TYPE_F32, ACB_TYPE_F16)
    ACB_RN(ACB_TYPE_BF16, ACB_TYPE_BF16)
    ACB_RN(ACB_TYPE_BF16, ACB_TYPE_F32)
    ACB_RN(ACB_TYPE_F16, ACB_TYPE_F16)
    ACB_RN(ACB_TYPE_F16, ACB_TYPE_F32)
#undef ACB_RN
    return ACB_ERR_UNSUPPORTED;
}

// ---- per-head q/k RMSNorm + NeoX RoPE ------------------------------------------------------
// E consecutive elements of an I/O type as floats: one 4-, 8- or 16-byte access when VEC (the
// caller checked the alignment), else E scalar accesses.
template <int T, int E, bool VEC> __device__ __forceinline__ void ld_run(const void * p, float * f) {
    using e         = typename io<T>::t;
    constexpr int B = E * (int) sizeof(e);
    if constexpr (VEC && (B == 4 || B == 8 || B == 16)) {
        using W = std::conditional_t<B == 16, uint4, std::conditional_t<B == 8, uint2, uint32_t>>;
        union {
            W u;
            e v[E];
        } r;
        r.u = *reinterpret_cast<const W *>(p);
#pragma unroll
        for (int i = 0; i < E; i++) {
            f[i] = io<T>::to_f(r.v[i]);
        }
    } else {
#pragma unroll
        for (int i = 0; i < E; i++) {
            f[i] = io<T>::to_f(reinterpret_cast<const e *>(p)[i]);
        }
    }
}

template <int T, int E, bool VEC> __device__ __forceinline__ void st_run(void * p, const float * f) {
    using e         = typename io<T>::t;
    constexpr int B = E * (int) sizeof(e);
    if constexpr (VEC && (B == 4 || B == 8 || B == 16)) {
        using W = std::conditional_t<B == 16, uint4, std::conditional_t<B == 8, uint2, uint32_t>>;
        union {
            W u;
            e v[E];
        } r;
#pragma unroll
        for (int i = 0; i < E; i++) {
            r.v[i] = io<T>::from_f(f[i]);
        }
        *reinterpret_cast<W *>(p) = r.u;
    } else {
#pragma unroll
        for (int i = 0; i < E; i++) {
            reinterpret_cast<e *>(p)[i] = io<T>::from_f(f[i]);
        }
    }
}

// One warp per HPW consecutive (token, head) items. Lane l owns E = D/64 consecutive elements of
// the first half starting at l*E and the matching elements of the second half, so each NeoX pair
// (i, i+D/2) lives in one lane. The warp issues the loads of all its heads (positions, head
// vectors, norm weights, then the rope rows, which wait only on the positions) before the first
// use, so a head of 256-512 bytes does not cost a round trip of its own.
template <int TI, int TO, int E, int HPW, bool VEC>
__global__ void __launch_bounds__(256) qk_norm_rope_kernel(
    const void * __restrict__ src, int64_t sts, void * __restrict__ dst, int64_t dts, int64_t dhs, int64_t dps,
    int64_t n_tok, int n_heads, const float * __restrict__ w, float eps, const int32_t * __restrict__ pos,
    const float * __restrict__ rope, int max_pos, int * __restrict__ err) {
    using ei            = typename io<TI>::t;
    using eo            = typename io<TO>::t;
    constexpr int D     = 64 * E;
    constexpr int HALF  = D / 2;
    const int     lane  = threadIdx.x & 31;
    const int64_t items = n_tok * n_heads;
    const int64_t item0 = ((int64_t) blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * HPW;
    if (item0 >= items) {
        return;
    }
    // (token, head) of each item: one division per warp, then steps of one head; items past the
    // end repeat the first item so that their loads stay in bounds
    int64_t tk[HPW];
    int     hd[HPW];
    {
        int64_t t = item0 / n_heads;
        int     h = (int) (item0 - t * n_heads);
#pragma unroll
        for (int k = 0; k < HPW; k++) {
            const bool in = item0 + k < items;
            tk[k]         = in ? t : tk[0];
            hd[k]         = in ? h : hd[0];
            if (++h == n_heads) {
                h = 0;
                t++;
            }
        }
    }
    int p[HPW];
#pragma unroll
    for (int k = 0; k < HPW; k++) {
        p[k] = pos ? __ldg(pos + tk[k]) : 0;
    }
    float a[HPW][E], b[HPW][E];
#pragma unroll
    for (int k = 0; k < HPW; k++) {
        const ei * s = reinterpret_cast<const ei *>(src) + tk[k] * sts + (int64_t) hd[k] * D + lane * E;
        ld_run<TI, E, VEC>(s, a[k]);
        ld_run<TI, E, VEC>(s + HALF, b[k]);
    }
    float wa[E], wb[E];
    if (w) {
        ld_run<ACB_TYPE_F32, E, VEC>(w + lane * E, wa);
        ld_run<ACB_TYPE_F32, E, VEC>(w + HALF + lane * E, wb);
    }
    float cs[HPW][E], sn[HPW][E];
    if (rope) {
#pragma unroll
        for (int k = 0; k < HPW; k++) {
            const bool    ok = !pos || (p[k] >= 0 && p[k] < max_pos);
            const float * c  = rope + (int64_t) (ok ? p[k] : 0) * D + 2 * lane * E;
            float         r[2 * E];
            if (ok) {
                ld_run<ACB_TYPE_F32, 2 * E, VEC>(c, r);
            } else {
#pragma unroll
                for (int e = 0; e < 2 * E; e++) {
                    r[e] = 0.0f;
                }
            }
#pragma unroll
            for (int e = 0; e < E; e++) {
                cs[k][e] = r[2 * e];
                sn[k][e] = r[2 * e + 1];
            }
        }
    }
    // the heads' sums of squares are reduced side by side (same butterfly per head), so their
    // shuffle and division latencies overlap instead of adding up
    float sc[HPW];
    if (w) {
        double ss[HPW];
#pragma unroll
        for (int k = 0; k < HPW; k++) {
            ss[k] = 0.0;
#pragma unroll
            for (int e = 0; e < E; e++) {
                ss[k] += (double) __fmul_rn(a[k][e], a[k][e]);
            }
#pragma unroll
            for (int e = 0; e < E; e++) {
                ss[k] += (double) __fmul_rn(b[k][e], b[k][e]);
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
            for (int k = 0; k < HPW; k++) {
                ss[k] += __shfl_xor_sync(0xffffffffu, ss[k], o);
            }
        }
#pragma unroll
        for (int k = 0; k < HPW; k++) {
            sc[k] = rms_scale_pow2<D>(ss[k], eps);
        }
    }
#pragma unroll
    for (int k = 0; k < HPW; k++) {
        if (item0 + k >= items) {
            break;
        }
        if (pos && (p[k] < 0 || p[k] >= max_pos)) {
            if (lane == 0 && err) {
                atomicOr(err, ACB_DEVERR_POS_RANGE);
            }
            continue;
        }
        if (w) {
#pragma unroll
            for (int e = 0; e < E; e++) {
                a[k][e] = __fmul_rn(__fmul_rn(a[k][e], sc[k]), wa[e]);
                b[k][e] = __fmul_rn(__fmul_rn(b[k][e], sc[k]), wb[e]);
            }
        }
        if (rope) {
#pragma unroll
            for (int e = 0; e < E; e++) {
                const float x0 = a[k][e], x1 = b[k][e];
                a[k][e]        = __fsub_rn(__fmul_rn(x0, cs[k][e]), __fmul_rn(x1, sn[k][e]));
                b[k][e]        = __fadd_rn(__fmul_rn(x0, sn[k][e]), __fmul_rn(x1, cs[k][e]));
            }
        }
        eo * d = reinterpret_cast<eo *>(dst) + tk[k] * dts + (int64_t) hd[k] * dhs + (int64_t) p[k] * dps + lane * E;
        st_run<TO, E, VEC>(d, a[k]);
        st_run<TO, E, VEC>(d + HALF, b[k]);
    }
}

// 128-wide heads, a warp per token: the half-warps take two heads at a time, lane l16 = lane & 15
// owning elements 8*l16 .. 8*l16 + 7 (16- or 32-byte accesses). The NeoX partner of element i < 64
// is i + 64, eight lanes away (a shuffle), and every head of the token shares the lane's norm
// weights and rope rows, which are loaded once per token instead of once per head. All heads'
// loads are issued before the first reduction. Same arithmetic as qk_norm_rope_kernel: the sum of
// squares in double (16-lane butterfly), (x * scale) * w, then the rotation.
template <int TI, int TO>
__global__ void __launch_bounds__(256) qk_tok_kernel(const void * __restrict__ src, int64_t sts,
                                                     void * __restrict__ dst, int64_t dts, int64_t dhs, int64_t dps,
                                                     int64_t n_tok, int n_heads, const float * __restrict__ w,
                                                     float eps, const int32_t * __restrict__ pos,
                                                     const float * __restrict__ rope, int max_pos,
                                                     int * __restrict__ err) {
    using ei          = typename io<TI>::t;
    using eo          = typename io<TO>::t;
    constexpr int D   = 128;
    constexpr int U   = 4;  // head pairs per pass: 8 heads' loads in flight per warp
    const int     lane = threadIdx.x & 31;
    const int64_t t    = (int64_t) blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (t >= n_tok) {
        return;
    }
    const int  sub   = lane >> 4;
    const int  l16   = lane & 15;
    const bool first = l16 < 8;
    const int  p     = pos ? __ldg(pos + t) : 0;
    if (pos && (p < 0 || p >= max_pos)) {
        if (lane == 0 && err) {
            atomicOr(err, ACB_DEVERR_POS_RANGE);
        }
        return;
    }
    float wv[8];
    if (w) {
        ld_run<ACB_TYPE_F32, 4, true>(w + 8 * l16, wv);
        ld_run<ACB_TYPE_F32, 4, true>(w + 8 * l16 + 4, wv + 4);
    }
    float cs[8], sn[8];
    if (rope) {
        const float * c = rope + (int64_t) p * D + 16 * (l16 & 7);  // (cos, sin) of pairs 8*(l16&7) ..
        float         r[16];
#pragma unroll
        for (int q = 0; q < 4; q++) {
            ld_run<ACB_TYPE_F32, 4, true>(c + 4 * q, r + 4 * q);
        }
#pragma unroll
        for (int e = 0; e < 8; e++) {
            cs[e] = r[2 * e];
            sn[e] = first ? -r[2 * e + 1] : r[2 * e + 1];
        }
    }
    const int npairs = (n_heads + 1) / 2;
    for (int base = 0; base < npairs; base += U) {
        // phase by phase over the U head pairs, so that their loads, shuffle chains, square roots
        // and divisions overlap (pairs past the end hold zeros and store nothing)
        float x[U][8];
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int h = 2 * (base + u) + sub;
            if (base + u < npairs && h < n_heads) {
                const ei * s = reinterpret_cast<const ei *>(src) + t * sts + (int64_t) h * D + 8 * l16;
                if constexpr (sizeof(ei) == 2) {
                    ld_run<TI, 8, true>(s, x[u]);
                } else {
                    ld_run<TI, 4, true>(s, x[u]);
                    ld_run<TI, 4, true>(s + 4, x[u] + 4);
                }
            } else {
#pragma unroll
                for (int e = 0; e < 8; e++) {
                    x[u][e] = 0.0f;
                }
            }
        }
        if (w) {
            // the four heads' sums of squares by a transposed reduction over the 16 lanes: after
            // the exchanges at distances 8 and 4 each lane holds one head's partial (head
            // 2*bit3 + bit2 of its lane index) and finishes it with two more, so there are five
            // double shuffles and one square root and division per lane instead of sixteen and
            // four
            double v[U];
#pragma unroll
            for (int u = 0; u < U; u++) {
                v[u] = 0.0;
#pragma unroll
                for (int e = 0; e < 8; e++) {
                    v[u] += (double) __fmul_rn(x[u][e], x[u][e]);
                }
            }
            const bool   b8 = (lane & 8) != 0, b4 = (lane & 4) != 0;
            const double r0 = __shfl_xor_sync(0xffffffffu, b8 ? v[0] : v[2], 8);
            const double r1 = __shfl_xor_sync(0xffffffffu, b8 ? v[1] : v[3], 8);
            const double w0 = (b8 ? v[2] : v[0]) + r0;
            const double w1 = (b8 ? v[3] : v[1]) + r1;
            double       z  = (b4 ? w1 : w0) + __shfl_xor_sync(0xffffffffu, b4 ? w0 : w1, 4);
            z += __shfl_xor_sync(0xffffffffu, z, 2);
            z += __shfl_xor_sync(0xffffffffu, z, 1);
            const float mine = rms_scale_pow2<D>(z, eps);
#pragma unroll
            for (int u = 0; u < U; u++) {
                const float sc = __shfl_sync(0xffffffffu, mine, (lane & 19) | (u << 2));
#pragma unroll
                for (int e = 0; e < 8; e++) {
                    x[u][e] = __fmul_rn(__fmul_rn(x[u][e], sc), wv[e]);
                }
            }
        }
        if (rope) {
            // first half: x0*c - x1*s with x1 the partner; second half: x0*s + x1*c with x0 the
            // partner -- both own*c + partner*s' with s' = -s in the first half (exact negation)
#pragma unroll
            for (int u = 0; u < U; u++) {
#pragma unroll
                for (int e = 0; e < 8; e++) {
                    const float o = __shfl_xor_sync(0xffffffffu, x[u][e], 8);
                    x[u][e]       = __fadd_rn(__fmul_rn(x[u][e], cs[e]), __fmul_rn(o, sn[e]));
                }
            }
        }
#pragma unroll
        for (int u = 0; u < U; u++) {
            const int h = 2 * (base + u) + sub;
            if (base + u < npairs && h < n_heads) {
                eo * d = reinterpret_cast<eo *>(dst) + t * dts + (int64_t) h * dhs + (int64_t) p * dps + 8 * l16;
                if constexpr (sizeof(eo) == 2) {
                    st_run<TO, 8, true>(d, x[u]);
                } else {
                    st_run<TO, 4, true>(d, x[u]);
                    st_run<TO, 4, true>(d + 4, x[u] + 4);
                }
            }
        }
    }
}

// q/k RMSNorm (+ NeoX RoPE) of 128-wide heads into exact hi/lo f16 planes: one warp per
// (token, head); heads [0, nq) use wq, heads [nq, nq + nk) use wk. Lane l holds elements
// (2l, 2l+1) of each half (8-byte loads), so each NeoX pair (i, i + 64) is in one lane.
template <int TI>
__global__ void __launch_bounds__(256) qk_planes_kernel(const void * __restrict__ src, int64_t sts,
                                                        uint16_t * __restrict__ dst, int64_t dts, int64_t lo_off,
                                                        int64_t n_tok, int nq, int nk, const float * __restrict__ wq,
                                                        const float * __restrict__ wk, float eps,
                                                        const int32_t * __restrict__ pos,
                                                        const float * __restrict__ rope, int max_pos,
                                                        int * __restrict__ err) {
    using ei           = typename io<TI>::t;
    const int     lane = threadIdx.x & 31;
    const int     nh   = nq + nk;
    const int64_t item = (int64_t) blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (item >= n_tok * nh) {
        return;
    }
    const int64_t t = item / nh;
    const int     h = (int) (item - t * nh);
    int           p = 0;
    if (rope) {
        p = __ldg(pos + t);
        if (p < 0 || p >= max_pos) {
            if (lane == 0 && err) {
                atomicOr(err, ACB_DEVERR_POS_RANGE);
            }
            return;
        }
    }
    const ei * s = reinterpret_cast<const ei *>(src) + t * sts + (int64_t) h * 128 + lane * 2;
    float      a[2], b[2];
    if constexpr (TI == ACB_TYPE_F32) {
        const float2 x = *reinterpret_cast<const float2 *>(s), y = *reinterpret_cast<const float2 *>(s + 64);
        a[0] = x.x;
        a[1] = x.y;
        b[0] = y.x;
        b[1] = y.y;
    } else {
#pragma unroll
        for (int e = 0; e < 2; e++) {
            a[e] = io<TI>::to_f(s[e]);
            b[e] = io<TI>::to_f(s[64 + e]);
        }
    }
    const float * w = h < nq ? wq : wk;
    if (w) {
        double ss = (double) __fmul_rn(a[0], a[0]);
        ss += (double) __fmul_rn(a[1], a[1]);
        ss += (double) __fmul_rn(b[0], b[0]);
        ss += (double) __fmul_rn(b[1], b[1]);
        ss             = warp_sum(ss);
        const float sc = rms_scale_pow2<128>(ss, eps);
#pragma unroll
        for (int e = 0; e < 2; e++) {
            a[e] = __fmul_rn(__fmul_rn(a[e], sc), __ldg(w + lane * 2 + e));
            b[e] = __fmul_rn(__fmul_rn(b[e], sc), __ldg(w + 64 + lane * 2 + e));
        }
    }
    if (rope) {
        const float4 c  = __ldg(reinterpret_cast<const float4 *>(rope + (int64_t) p * 128 + 4 * lane));
        const float  cs[2] = { c.x, c.z }, sn[2] = { c.y, c.w };
#pragma unroll
        for (int e = 0; e < 2; e++) {
            const float x0 = a[e], x1 = b[e];
            a[e]           = __fsub_rn(__fmul_rn(x0, cs[e]), __fmul_rn(x1, sn[e]));
            b[e]           = __fadd_rn(__fmul_rn(x0, sn[e]), __fmul_rn(x1, cs[e]));
        }
    }
    uint16_t *    d  = dst + t * dts + (int64_t) h * 128 + lane * 2;
    const __half2 ah = __floats2half2_rn(a[0], a[1]), bh = __floats2half2_rn(b[0], b[1]);
    const float2  af = __half22float2(ah), bf = __half22float2(bh);
    const __half2 al = __floats2half2_rn(__fsub_rn(a[0], af.x), __fsub_rn(a[1], af.y));
    const __half2 bl = __floats2half2_rn(__fsub_rn(b[0], bf.x), __fsub_rn(b[1], bf.y));
    *reinterpret_cast<__half2 *>(d)               = ah;
    *reinterpret_cast<__half2 *>(d + 64)          = bh;
    *reinterpret_cast<__half2 *>(d + lo_off)      = al;
    *reinterpret_cast<__half2 *>(d + lo_off + 64) = bl;
}

template <int TI, int TO, int E, int HPW>
static void launch_qk_e(bool vec, dim3 grid, const void * src, int64_t sts, void * dst, int64_t dts, int64_t dhs,
                        int64_t dps, int64_t n_tok, int n_heads, const float * w, float eps, const int32_t * pos,
                        const float * rope, int max_pos, int * err, cudaStream_t st) {
    if constexpr (E > 1) {  // a single element per lane has nothing to vectorise
        if (vec) {
            qk_norm_rope_kernel<TI, TO, E, HPW, true><<<grid, 256, 0, st>>>(src, sts, dst, dts, dhs, dps, n_tok,
                                                                            n_heads, w, eps, pos, rope, max_pos, err);
            return;
        }
    }
    qk_norm_rope_kernel<TI, TO, E, HPW, false>
        <<<grid, 256, 0, st>>>(src, sts, dst, dts, dhs, dps, n_tok, n_heads, w, eps, pos, rope, max_pos, err);
}

template <int TI, int TO>
static acb_status launch_qk(const void * src, int64_t sts, void * dst, int64_t dts, int64_t dhs, int64_t dps,
                            int64_t n_tok, int n_heads, int D, const float * w, float eps, const int32_t * pos,
                            const float * rope, int max_pos, int * err, cudaStream_t st) {
    if (D != 64 && D != 128 && D != 256) {
        return ACB_ERR_UNSUPPORTED;
    }
    const int64_t items = n_tok * n_heads;
    // heads per warp: 0.5-2 KB of loads in flight per warp; 8 warps per CTA
    const int  hpw = D == 256 ? 2 : 4;
    const dim3 grid((unsigned) ((items + 8LL * hpw - 1) / (8LL * hpw)));
    // each lane's E = D/64 consecutive elements as one access when every run is aligned to its size
    const int  E  = D / 64;
    const int  si = (int) sizeof(typename io<TI>::t), so = (int) sizeof(typename io<TO>::t);
    auto       al = [](const void * q, int b) { return (reinterpret_cast<uintptr_t>(q) % (uintptr_t) b) == 0; };
    const bool vec = E > 1 && al(src, E * si) && al(dst, E * so) && sts % E == 0 && dts % E == 0 && dhs % E == 0 &&
                     dps % E == 0 && (!w || al(w, E * 4)) && (!rope || al(rope, 2 * E * 4));
    const bool tokv = D == 128 && al(src, 8 * si) && al(dst, 8 * so) && sts % 8 == 0 && dts % 8 == 0 &&
                      dhs % 8 == 0 && dps % 8 == 0 && (!w || al(w, 16)) && (!rope || al(rope, 16));
    if (tokv) {
        qk_tok_kernel<TI, TO><<<(unsigned) ((n_tok + 7) / 8), 256, 0, st>>>(src, sts, dst, dts, dhs, dps, n_tok,
                                                                           n_heads, w, eps, pos, rope, max_pos, err);
        return launch_status();
    }
    switch (D) {
        case 64:
            launch_qk_e<TI, TO, 1, 4>(false, grid, src, sts, dst, dts, dhs, dps, n_tok, n_heads, w, eps, pos, rope,
                                      max_pos, err, st);
            break;
        case 128:
            launch_qk_e<TI, TO, 2, 4>(vec, grid, src, sts, dst, dts, dhs, dps, n_tok, n_heads, w, eps, pos, rope,
                                      max_pos, err, st);
            break;
        default:
            launch_qk_e<TI, TO, 4, 2>(vec, grid, src, sts, dst, dts, dhs, dps, n_tok, n_heads, w, eps, pos, rope,
                                      max_pos, err, st);
            break;
    }
    return launch_status();
}

}  // namespace acb

using namespace acb;

extern "C" acb_status acb_rms_norm(const void * x, int x_type, int64_t x_stride, const float * w, void * y,
                                   int y_type, int64_t y_stride, int64_t rows, int cols, float eps,
                                   acb_stream_t stream) {
    if (!x || !y || rows < 0 || cols <= 0 || x_stride < cols || y_stride < cols) {
        return ACB_ERR_INVALID_ARG;
    }
    if (rows == 0) {
        return ACB_OK;
    }
    return dispatch_row_norm<0>(x_type, y_type, x, x_stride, w, y, y_stride, rows, cols, eps, nullptr, nullptr, 0, 1,
                                (cudaStream_t) stream);
}

extern "C" acb_status acb_adaln_modulate(const void * x, int x_type, const float * norm_w, float eps,
                                         const float * scale, const float * shift, int64_t vec_stride, void * y,
                                         int y_type, int64_t samples, int64_t rows_per_sample, int H,
                                         acb_stream_t stream) {
    if (!x || !y || !scale || !shift || samples < 0 || rows_per_sample < 0 || H <= 0 || vec_stride < 0) {
        return ACB_ERR_INVALID_ARG;
    }
    if (samples * rows_per_sample == 0) {
        return ACB_OK;
    }
    return dispatch_row_norm<1>(x_type, y_type, x, H, norm_w, y, H, samples * rows_per_sample, H, eps, scale, shift,
                                vec_stride, rows_per_sample, (cudaStream_t) stream);
}

extern "C" acb_status acb_qk_norm_rope(const void * src, int src_type, int64_t src_tok_stride, void * dst,
                                       int dst_type, int64_t dst_tok_stride, int64_t dst_head_stride,
                                       int64_t dst_pos_stride, int64_t n_tok, int n_heads, int head_dim,
                                       const float * norm_w, float eps, const int32_t * pos,
                                       const float * rope_table, int max_pos, int * err_flag,
                                       acb_stream_t stream) {
    if (!src || !dst || n_tok < 0 || n_heads <= 0 || head_dim <= 0) {
        return ACB_ERR_INVALID_ARG;
    }
    if ((rope_table || dst_pos_stride != 0) && (!pos || max_pos <= 0)) {
        return ACB_ERR_INVALID_ARG;
    }
    if (head_dim % 64 != 0 || head_dim > 256) {
        return ACB_ERR_UNSUPPORTED;
    }
    if (n_tok == 0) {
        return ACB_OK;
    }
    cudaStream_t st = (cudaStream_t) stream;
#define ACB_QK(A, B)                                                                                             \
    if (src_type == A && dst_type == B) {                                                                        \
        return launch_qk<A, B>(src, src_tok_stride, dst, dst_tok_stride, dst_head_stride, dst_pos_stride, n_tok, \
                               n_heads, head_dim, norm_w, eps, pos, rope_table, max_pos, err_flag, st);          \
    }
    ACB_QK(ACB_TYPE_F32, ACB_TYPE_F32)
    ACB_QK(ACB_TYPE_F32, ACB_TYPE_F16)
    ACB_QK(ACB_TYPE_F32, ACB_TYPE_BF16)
    ACB_QK(ACB_TYPE_BF16, ACB_TYPE_BF16)
    ACB_QK(ACB_TYPE_BF16, ACB_TYPE_F32)
    ACB_QK(ACB_TYPE_BF16, ACB_TYPE_F16)
    ACB_QK(ACB_TYPE_F16, ACB_TYPE_F16)
#undef ACB_QK
    return ACB_ERR_UNSUPPORTED;
}

extern "C" acb_status acb_qk_norm_rope_planes(const void * src, int src_type, int64_t src_tok_stride, uint16_t * dst,
                                              int64_t dst_tok_stride, int64_t lo_offset, int64_t n_tok, int n_q_heads,
                                              const float * q_norm_w, int n_k_heads, const float * k_norm_w,
                                              int head_dim, float eps, const int32_t * pos, const float * rope_table,
                                              int max_pos, int * err_flag, acb_stream_t stream) {
    const int nh = n_q_heads + n_k_heads;
    if (!src || !dst || n_tok < 0 || n_q_heads < 0 || n_k_heads < 0 || nh <= 0 || lo_offset <= 0 ||
        src_tok_stride < (int64_t) nh * head_dim || dst_tok_stride < (int64_t) nh * head_dim) {
        return ACB_ERR_INVALID_ARG;
    }
    if (rope_table && (!pos || max_pos <= 0)) {
        return ACB_ERR_INVALID_ARG;
    }
    if (head_dim != 128 || (src_type != ACB_TYPE_F32 && src_type != ACB_TYPE_F16)) {
        return ACB_ERR_UNSUPPORTED;
    }
    // 8-byte source loads and 4-byte plane stores
    const int es = src_type == ACB_TYPE_F32 ? 4 : 2;
    if (reinterpret_cast<uintptr_t>(src) % (2 * es) || (src_tok_stride * es) % (2 * es) ||
        reinterpret_cast<uintptr_t>(dst) % 4 || dst_tok_stride % 2 || lo_offset % 2) {
        return ACB_ERR_UNSUPPORTED;
    }
    if (n_tok == 0) {
        return ACB_OK;
    }
    const int64_t items = n_tok * nh;
    const dim3    grid((unsigned) ((items + 7) / 8));
    cudaStream_t  st = (cudaStream_t) stream;
    if (src_type == ACB_TYPE_F32) {
        qk_planes_kernel<ACB_TYPE_F32><<<grid, 256, 0, st>>>(src, src_tok_stride, dst, dst_tok_stride, lo_offset, n_tok,
                                                             n_q_heads, n_k_heads, q_norm_w, k_norm_w, eps, pos,
                                                             rope_table, max_pos, err_flag);
    } else {
        qk_planes_kernel<ACB_TYPE_F16><<<grid, 256, 0, st>>>(src, src_tok_stride, dst, dst_tok_stride, lo_offset, n_tok,
                                                             n_q_heads, n_k_heads, q_norm_w, k_norm_w, eps, pos,
                                                             rope_table, max_pos, err_flag);
    }
    return launch_status();
}
