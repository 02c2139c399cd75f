// k_philox.cu -- the reference's seeded noise (src/philox.h) as device kernels, and the SDE step
// (src/solvers/solver-sde.h:17-38) that draws its fresh noise inline.
//
// The reference fills noise on the host, one Philox counter per element (philox_randn), for the
// initial latents (pipeline-synth-ops.cpp:761-770) and for every SDE step (solver-sde.h:28-31),
// and copies it to the device. Here every element is computed where it is consumed: one thread
// per element, ten 32-bit multiply-high rounds plus a log, a sine and a square root, no state and
// no memory traffic but the output. The SDE step folds the noise into the update, so a step moves
// 12 bytes per element (xt, vt in; xt out) instead of 16 plus a host fill and a copy.
#include <algorithm>

#include "common.cuh"
#include "philox.cuh"

namespace acb {
namespace {

__global__ void philox_randn_kernel(uint64_t seed, float * __restrict__ out, int64_t n, bool round_bf16) {
    for (int64_t k = (int64_t) blockIdx.x * blockDim.x + threadIdx.x; k < n; k += (int64_t) gridDim.x * blockDim.x) {
        out[k] = philox::randn(seed, (uint64_t) k, round_bf16);
    }
}

__global__ void philox_bits_kernel(uint64_t seed, uint64_t first, int64_t n, uint4 * __restrict__ out) {
    for (int64_t i = (int64_t) blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t) gridDim.x * blockDim.x) {
        out[i] = philox::words(seed, first + (uint64_t) i);
    }
}

// xt[b][i] = t_next * noise_b[i] + (1 - t_next) * (xt[b][i] - vt[b][i] * t_curr), noise_b the bf16
// stream of step_seeds[b] (the caller's seed_b + step + 1); the arithmetic is acb_dit_sde's.
__global__ void dit_sde_philox_kernel(float * __restrict__ xt, const float * __restrict__ vt,
                                      const int64_t * __restrict__ step_seeds, const float * __restrict__ tt,
                                      int64_t n_per) {
    const int     b    = blockIdx.y;
    const int64_t base = (int64_t) b * n_per;
    const uint64_t seed = (uint64_t) step_seeds[b];
    const float   t_curr = tt[0], t_next = tt[2];
    for (int64_t i = (int64_t) blockIdx.x * blockDim.x + threadIdx.x; i < n_per; i += (int64_t) gridDim.x * blockDim.x) {
        const float noise = philox::randn(seed, (uint64_t) i, true);
        const float x0    = __fsub_rn(xt[base + i], __fmul_rn(vt[base + i], t_curr));
        xt[base + i]      = __fadd_rn(__fmul_rn(t_next, noise), __fmul_rn(__fsub_rn(1.0f, t_next), x0));
    }
}

// one wave of 256-thread blocks, 8 resident per SM, grid-stride beyond it
constexpr int kThreads = 256;

int grid_for(int64_t n) {
    static int sms = 0;
    if (sms == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0) {
            sms = 148;
        }
    }
    const int64_t need = (n + kThreads - 1) / kThreads;
    return (int) std::max<int64_t>(1, std::min<int64_t>(need, (int64_t) sms * 8));
}

}  // namespace
}  // namespace acb

using namespace acb;

extern "C" acb_status acb_philox_randn(int64_t seed, float * out, int64_t n, int bf16_round, acb_stream_t stream) {
    if (n < 0 || (n > 0 && !out)) {
        return ACB_ERR_INVALID_ARG;
    }
    if (n == 0) {
        return ACB_OK;
    }
    philox_randn_kernel<<<grid_for(n), kThreads, 0, (cudaStream_t) stream>>>((uint64_t) seed, out, n, bf16_round != 0);
    return launch_status();
}

extern "C" acb_status acb_philox_bits(int64_t seed, int64_t first, int64_t n, uint32_t * out, acb_stream_t stream) {
    if (n < 0 || first < 0 || (n > 0 && !out) || (reinterpret_cast<uintptr_t>(out) & 15)) {
        return ACB_ERR_INVALID_ARG;
    }
    if (n == 0) {
        return ACB_OK;
    }
    philox_bits_kernel<<<grid_for(n), kThreads, 0, (cudaStream_t) stream>>>((uint64_t) seed, (uint64_t) first, n,
                                                                            reinterpret_cast<uint4 *>(out));
    return launch_status();
}

extern "C" acb_status acb_dit_sde_philox(float * xt, const float * vt, const int64_t * step_seeds, const float * tt,
                                         int n_tracks, int64_t n_per, acb_stream_t stream) {
    if (!xt || !vt || !step_seeds || !tt || n_tracks <= 0 || n_tracks > 65535 || n_per < 0) {
        return ACB_ERR_INVALID_ARG;
    }
    if (n_per == 0) {
        return ACB_OK;
    }
    const int gx = std::max(1, grid_for(n_per) / n_tracks);
    dit_sde_philox_kernel<<<dim3(gx, n_tracks), kThreads, 0, (cudaStream_t) stream>>>(xt, vt, step_seeds, tt, n_per);
    return launch_status();
}
