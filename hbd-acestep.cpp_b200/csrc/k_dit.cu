// k_dit.cu -- the small per-step kernels of the DiT denoiser around its layer chain
// (src/dit-graph.h:81-117 timestep embedding, :383-400 and :591-606 modulation vectors;
// src/dit-sampler.h:44-122 APG guidance, :327-339 and :466-479 input packing, :596-604 and
// src/solvers/solver-euler.h:8-18 the Euler step and the final x0). Every input that changes per
// step (t, t_r) is read from device memory, so a whole denoise step can be one CUDA graph.
#include <algorithm>

#include "common.cuh"

namespace acb {

// ggml_timestep_embedding of t*1000 (row 0) and (t - t_r)*1000 (row 1): dim/2 frequencies
// exp(-ln(max_period) * j / half), [cos | sin].
__global__ void dit_sinusoid_kernel(const float * __restrict__ tt, int dim, int max_period, float * __restrict__ out) {
    const int row = blockIdx.x, half = dim / 2;
    const float t = row == 0 ? tt[0] : __fsub_rn(tt[0], tt[1]);
    const float a = __fmul_rn(t, 1000.0f);
    for (int j = threadIdx.x; j < half; j += blockDim.x) {
        const float freq = expf(__fdiv_rn(__fmul_rn(-logf((float) max_period), (float) j), (float) half));
        const float arg  = __fmul_rn(a, freq);
        out[row * dim + j]        = cosf(arg);
        out[row * dim + j + half] = sinf(arg);
    }
    if ((dim & 1) && threadIdx.x == 0) {
        out[row * dim + dim - 1] = 0.0f;
    }
}

__global__ void silu_kernel(const float * __restrict__ x, float * __restrict__ y, int64_t n) {
    const int64_t i = (int64_t) blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) {
        const float v = x[i];
        y[i]          = silu_f(v);
    }
}

// tproj = tproj_t + tproj_r; ada[l] = scale_shift_table[l] + tproj (six [H] vectors per layer);
// temb = temb_t + temb_r; out_shift = oss[0] + temb, out_scale = oss[1] + temb.
__global__ void dit_modulation_kernel(const float * __restrict__ sst, const float * __restrict__ tproj2,
                                      const float * __restrict__ temb2, const float * __restrict__ oss, int L, int H,
                                      float * __restrict__ ada, float * __restrict__ out_ss) {
    const int64_t i  = (int64_t) blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t H6 = 6 * (int64_t) H;
    if (i < L * H6) {
        const int64_t j = i % H6;
        ada[i]          = __fadd_rn(sst[i], __fadd_rn(tproj2[j], tproj2[H6 + j]));
    }
    if (i < H) {
        const float temb = __fadd_rn(temb2[i], temb2[H + i]);
        out_ss[i]        = __fadd_rn(oss[i], temb);      // shift
        out_ss[H + i]    = __fadd_rn(oss[H + i], temb);  // scale
    }
}

// The noisy latent into the xt channels of the DiT input [Ng][T][in_ch] (context channels are
// written once); slot b takes sample b % N (batched CFG: conditional then unconditional slots).
__global__ void dit_pack_xt_kernel(const float * __restrict__ xt, float * __restrict__ input, int N, int Ng, int T,
                                   int Oc, int ctx_ch) {
    const int64_t i     = (int64_t) blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t total = (int64_t) Ng * T * Oc;
    if (i >= total) {
        return;
    }
    const int64_t c  = i % Oc;
    const int64_t bt = i / Oc;  // slot * T + frame
    const int64_t b  = bt / T, t = bt - b * T;
    input[bt * (ctx_ch + Oc) + ctx_ch + c] = xt[((b % N) * T + t) * Oc + c];
}

// APG (adaptive projected guidance) for one (sample, channel), in double over all T frames:
// diff = cond - uncond; running average ra = diff (first step) or diff + momentum * ra; diff =
// ra clipped to L2 norm <= threshold over T; parallel/orthogonal split of diff against cond;
// v = cond + (scale - 1) * orthogonal.
constexpr int kApgThreads = 256;

__device__ double block_sum_d(double v, double * red) {
    v = warp_sum(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) {
        red[w] = v;
    }
    __syncthreads();
    double s = 0.0;
    if (threadIdx.x == 0) {
        for (int i = 0; i < kApgThreads / 32; i++) {
            s += red[i];
        }
        red[32] = s;
    }
    __syncthreads();
    return red[32];
}

__global__ void __launch_bounds__(kApgThreads)
    dit_apg_kernel(const float * __restrict__ cond, const float * __restrict__ uncond, double * __restrict__ ra,
                   int first, double momentum, double scale, double threshold, int T, int Oc, float * __restrict__ vt) {
    __shared__ double red[33];
    const int     c    = blockIdx.x, b = blockIdx.y;
    const int64_t base = (int64_t) b * T * Oc + c;
    double        n2   = 0.0;
    for (int t = threadIdx.x; t < T; t += kApgThreads) {
        const int64_t idx = base + (int64_t) t * Oc;
        const double  d   = (double) cond[idx] - (double) uncond[idx];
        const double  r   = first ? d : d + momentum * ra[idx];
        ra[idx]           = r;
        n2 += r * r;
    }
    n2              = block_sum_d(n2, red);
    const double nr = sqrt(n2 > 0.0 ? n2 : 0.0);
    const double s  = (threshold > 0.0 && nr > 1e-60) ? fmin(1.0, threshold / nr) : 1.0;
    double       v2 = 0.0, dot = 0.0;
    for (int t = threadIdx.x; t < T; t += kApgThreads) {
        const int64_t idx = base + (int64_t) t * Oc;
        const double  v1  = (double) cond[idx];
        v2 += v1 * v1;
    }
    v2               = block_sum_d(v2, red);
    const double inv = v2 > 1e-60 ? 1.0 / sqrt(v2) : 0.0;
    for (int t = threadIdx.x; t < T; t += kApgThreads) {
        const int64_t idx = base + (int64_t) t * Oc;
        const double  d   = s < 1.0 ? ra[idx] * s : ra[idx];
        dot += d * ((double) cond[idx] * inv);
    }
    dot = block_sum_d(dot, red);
    for (int t = threadIdx.x; t < T; t += kApgThreads) {
        const int64_t idx  = base + (int64_t) t * Oc;
        const double  d    = s < 1.0 ? ra[idx] * s : ra[idx];
        const double  v1n  = (double) cond[idx] * inv;
        const double  orth = d - dot * v1n;
        vt[idx]            = (float) ((double) cond[idx] + (scale - 1.0) * orth);
    }
}

// Euler step xt -= vt * (t_curr - t_next), or at the last step out = xt - vt * t_curr.
__global__ void dit_euler_kernel(float * __restrict__ xt, const float * __restrict__ vt, const float * __restrict__ tt,
                                 int last, float * __restrict__ out, int64_t n) {
    const int64_t i = (int64_t) blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) {
        return;
    }
    if (last) {
        out[i] = __fsub_rn(xt[i], __fmul_rn(vt[i], tt[0]));
    } else {
        const float dt = __fsub_rn(tt[0], tt[2]);
        xt[i]          = __fsub_rn(xt[i], __fmul_rn(vt[i], dt));
    }
}

// DPM++ 3M step (src/solvers/solver-dpm.h:14-50): a third-order Adams-Bashforth step on the
// velocity with two stored velocities, second order with one, Euler with none; then the history
// moves down (prev_prev <- prev, prev <- vt). Every element is independent, so the shift happens
// in place in the same pass. Products and sums are rounded one by one in the reference's order.
__global__ void dit_dpm3m_kernel(float * __restrict__ xt, const float * __restrict__ vt, float * __restrict__ prev,
                                 float * __restrict__ prev_prev, int history, const float * __restrict__ tt,
                                 int64_t n) {
    const int64_t i = (int64_t) blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) {
        return;
    }
    constexpr float c0 = 23.0f / 12.0f, c1 = 16.0f / 12.0f, c2 = 5.0f / 12.0f;
    const float     dt = __fsub_rn(tt[0], tt[2]);
    const float     v  = vt[i];
    float           ve = v;
    const float     p1 = prev[i];
    if (history >= 2) {
        ve = __fadd_rn(__fsub_rn(__fmul_rn(c0, v), __fmul_rn(c1, p1)), __fmul_rn(c2, prev_prev[i]));
    } else if (history == 1) {
        ve = __fsub_rn(__fmul_rn(1.5f, v), __fmul_rn(0.5f, p1));
    }
    xt[i]        = __fsub_rn(xt[i], __fmul_rn(ve, dt));
    prev_prev[i] = p1;
    prev[i]      = v;
}

// SDE ancestral step (src/solvers/solver-sde.h:17-38): predict x0 = xt - vt * t_curr, then renoise
// to the next time, xt = t_next * noise + (1 - t_next) * x0, each product and sum rounded in the
// reference's order. The noise is an input (the reference draws it per batch item on the host).
__global__ void dit_sde_kernel(float * __restrict__ xt, const float * __restrict__ vt,
                               const float * __restrict__ noise, const float * __restrict__ tt, int64_t n) {
    const int64_t i = (int64_t) blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) {
        return;
    }
    const float t_curr = tt[0], t_next = tt[2];
    const float x0     = __fsub_rn(xt[i], __fmul_rn(vt[i], t_curr));
    xt[i]              = __fadd_rn(__fmul_rn(t_next, noise[i]), __fmul_rn(__fsub_rn(1.0f, t_next), x0));
}

}  // namespace acb

using namespace acb;

// DCW (src/dit-sampler.h:613-666, src/dwt-haar.h) after an ODE solver step: denoised = xt - vt *
// t_next; modes 0 low / 1 high / 2 double move the Haar bands of xt (frames 2j, 2j+1 along T,
// zero-padded on odd T) away from the denoised sample's by s_low / s_high, then invert; mode 3
// (pix) moves xt itself by s_low. One thread per (track, frame pair, channel) -- pix: per element.
__global__ void dit_dcw_kernel(float * __restrict__ xt, const float * __restrict__ vt, int T, int C, int Tl,
                               int64_t n_items, float t_next, int mode, float s_low, float s_high) {
    const int64_t idx = (int64_t) blockIdx.x * blockDim.x + threadIdx.x;
    if (idx >= n_items) {
        return;
    }
    if (mode == ACB_DCW_PIX) {
        const float den = __fsub_rn(xt[idx], __fmul_rn(vt[idx], t_next));
        xt[idx]         = __fadd_rn(xt[idx], __fmul_rn(s_low, __fsub_rn(xt[idx], den)));
        return;
    }
    const float   r     = 0.70710678118654752440f;
    const int64_t c     = idx % C;
    const int64_t q     = idx / C;
    const int64_t tl    = q % Tl;
    const int64_t b     = q / Tl;
    const int64_t i0    = ((b * T) + 2 * tl) * C + c;
    const bool    has_b = 2 * tl + 1 < T;
    const int64_t i1    = i0 + C;
    const float   xa = xt[i0], xb = has_b ? xt[i1] : 0.0f;
    const float   da = __fsub_rn(xa, __fmul_rn(vt[i0], t_next));
    const float   db = has_b ? __fsub_rn(xb, __fmul_rn(vt[i1], t_next)) : 0.0f;
    float xL = has_b ? __fmul_rn(__fadd_rn(xa, xb), r) : __fmul_rn(xa, r);
    float xH = has_b ? __fmul_rn(__fsub_rn(xa, xb), r) : __fmul_rn(xa, r);
    const float yL = has_b ? __fmul_rn(__fadd_rn(da, db), r) : __fmul_rn(da, r);
    const float yH = has_b ? __fmul_rn(__fsub_rn(da, db), r) : __fmul_rn(da, r);
    if (mode != ACB_DCW_HIGH && s_low != 0.0f) {
        xL = __fadd_rn(xL, __fmul_rn(s_low, __fsub_rn(xL, yL)));
    }
    if (mode != ACB_DCW_LOW && s_high != 0.0f) {
        xH = __fadd_rn(xH, __fmul_rn(s_high, __fsub_rn(xH, yH)));
    }
    xt[i0] = __fmul_rn(__fadd_rn(xL, xH), r);
    if (has_b) {
        xt[i1] = __fmul_rn(__fsub_rn(xL, xH), r);
    }
}

static unsigned blocks_for(int64_t n, int threads) {
    return (unsigned) ((n + threads - 1) / threads);
}

extern "C" acb_status acb_dit_sinusoid(const float * tt, int dim, int max_period, float * out, acb_stream_t stream) {
    if (!tt || !out || dim <= 0 || max_period <= 0) {
        return ACB_ERR_INVALID_ARG;
    }
    dit_sinusoid_kernel<<<2, 128, 0, (cudaStream_t) stream>>>(tt, dim, max_period, out);
    return launch_status();
}

extern "C" acb_status acb_silu(const float * x, float * y, int64_t n, acb_stream_t stream) {
    if (!x || !y || n < 0) {
        return ACB_ERR_INVALID_ARG;
    }
    if (n == 0) {
        return ACB_OK;
    }
    silu_kernel<<<blocks_for(n, 256), 256, 0, (cudaStream_t) stream>>>(x, y, n);
    return launch_status();
}

extern "C" acb_status acb_dit_modulation(const float * sst, const float * tproj2, const float * temb2,
                                         const float * oss, int n_layers, int H, float * ada, float * out_ss,
                                         acb_stream_t stream) {
    if (!sst || !tproj2 || !temb2 || !oss || !ada || !out_ss || n_layers <= 0 || H <= 0) {
        return ACB_ERR_INVALID_ARG;
    }
    const int64_t n = std::max<int64_t>((int64_t) n_layers * 6 * H, H);
    dit_modulation_kernel<<<blocks_for(n, 256), 256, 0, (cudaStream_t) stream>>>(sst, tproj2, temb2, oss, n_layers, H,
                                                                                  ada, out_ss);
    return launch_status();
}

extern "C" acb_status acb_dit_pack_xt(const float * xt, float * input, int N, int Ng, int T, int Oc, int ctx_ch,
                                      acb_stream_t stream) {
    if (!xt || !input || N <= 0 || Ng < N || T <= 0 || Oc <= 0 || ctx_ch < 0) {
        return ACB_ERR_INVALID_ARG;
    }
    const int64_t n = (int64_t) Ng * T * Oc;
    dit_pack_xt_kernel<<<blocks_for(n, 256), 256, 0, (cudaStream_t) stream>>>(xt, input, N, Ng, T, Oc, ctx_ch);
    return launch_status();
}

extern "C" acb_status acb_dit_apg(const float * cond, const float * uncond, double * running_avg, int first,
                                  float momentum, float guidance_scale, float norm_threshold, int N, int T, int Oc,
                                  float * vt, acb_stream_t stream) {
    if (!cond || !uncond || !running_avg || !vt || N <= 0 || T <= 0 || Oc <= 0) {
        return ACB_ERR_INVALID_ARG;
    }
    dit_apg_kernel<<<dim3((unsigned) Oc, (unsigned) N), kApgThreads, 0, (cudaStream_t) stream>>>(
        cond, uncond, running_avg, first, (double) momentum, (double) guidance_scale, (double) norm_threshold, T, Oc,
        vt);
    return launch_status();
}

extern "C" acb_status acb_dit_euler(float * xt, const float * vt, const float * tt, int last, float * out, int64_t n,
                                    acb_stream_t stream) {
    if (!xt || !vt || !tt || (last && !out) || n < 0) {
        return ACB_ERR_INVALID_ARG;
    }
    if (n == 0) {
        return ACB_OK;
    }
    dit_euler_kernel<<<blocks_for(n, 256), 256, 0, (cudaStream_t) stream>>>(xt, vt, tt, last, out, n);
    return launch_status();
}

extern "C" acb_status acb_dit_dcw(float * xt, const float * vt, int n_tracks, int T, int C, float t_next, int mode,
                                  float s_low, float s_high, acb_stream_t stream) {
    if (!xt || !vt || n_tracks <= 0 || T <= 0 || C <= 0 || mode < ACB_DCW_LOW || mode > ACB_DCW_PIX) {
        return ACB_ERR_INVALID_ARG;
    }
    const int     Tl = (T + 1) / 2;
    const int64_t n  = mode == ACB_DCW_PIX ? (int64_t) n_tracks * T * C : (int64_t) n_tracks * Tl * C;
    dit_dcw_kernel<<<blocks_for(n, 256), 256, 0, (cudaStream_t) stream>>>(xt, vt, T, C, Tl, n, t_next, mode, s_low,
                                                                          s_high);
    return launch_status();
}

extern "C" acb_status acb_dit_dpm3m(float * xt, const float * vt, float * prev_vt, float * prev_prev_vt, int history,
                                    const float * tt, int64_t n, acb_stream_t stream) {
    if (!xt || !vt || !prev_vt || !prev_prev_vt || !tt || history < 0 || n < 0) {
        return ACB_ERR_INVALID_ARG;
    }
    if (n == 0) {
        return ACB_OK;
    }
    dit_dpm3m_kernel<<<blocks_for(n, 256), 256, 0, (cudaStream_t) stream>>>(xt, vt, prev_vt, prev_prev_vt, history,
                                                                             tt, n);
    return launch_status();
}

extern "C" acb_status acb_dit_sde(float * xt, const float * vt, const float * noise, const float * tt, int64_t n,
                                  acb_stream_t stream) {
    if (!xt || !vt || !noise || !tt || n < 0) {
        return ACB_ERR_INVALID_ARG;
    }
    if (n == 0) {
        return ACB_OK;
    }
    dit_sde_kernel<<<blocks_for(n, 256), 256, 0, (cudaStream_t) stream>>>(xt, vt, noise, tt, n);
    return launch_status();
}
