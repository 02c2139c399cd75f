// philox.cuh -- the reference's seeded N(0, 1) noise (src/philox.h) on the device.
//
// Element k of the stream seeded with `seed` is the first Box-Muller normal of Philox4x32-10
// (Salmon, Moraes, Dror, Shaw: "Parallel random numbers: as easy as 1, 2, 3", SC'11) of the
// counter {0, 0, k_lo, k_hi} under the key {seed_lo, seed_hi}, rounded to bfloat16
// (philox.h:95-107, 130-136): one counter per element, so any element is computed on its own and
// a thread needs no state. The integer rounds are exact; the Box-Muller arithmetic is written with
// explicitly rounded operations (nvcc must not fuse its multiply-adds, the reference's CPU code does
// not), and the transcendental calls are CUDA's logf / sinf / sqrt, which agree with the host libm
// to a few ulp -- after the bfloat16 rounding the streams differ in at most 1 element in 1000,
// by one bfloat16 step.
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

namespace acb {
namespace philox {

// the published Philox4x32 round multipliers and Weyl key increments (philox.h:16-19)
constexpr uint32_t kMul0 = 0xD2511F53u, kMul1 = 0xCD9E8D57u;
constexpr uint32_t kWeyl0 = 0x9E3779B9u, kWeyl1 = 0xBB67AE85u;
// word -> (0, 1]: w * 2^-32 + 2^-33; word -> (0, 2 pi): w * 2 pi 2^-32 + pi 2^-32 (philox.h:22-23, 85-91)
constexpr float kInv32 = 2.3283064365386963e-10f, kInv32Half = kInv32 * 0.5f;
constexpr float kInv32Tau = 1.4629180792671596e-09f, kInv32TauHalf = kInv32Tau * 0.5f;

__device__ __forceinline__ uint4 rounds10(uint4 c, uint32_t k0, uint32_t k1) {
#pragma unroll
    for (int r = 0; r < 10; r++) {
        if (r) {
            k0 += kWeyl0;
            k1 += kWeyl1;
        }
        const uint32_t lo0 = kMul0 * c.x, hi0 = __umulhi(kMul0, c.x);
        const uint32_t lo1 = kMul1 * c.z, hi1 = __umulhi(kMul1, c.z);
        c = make_uint4(hi1 ^ c.y ^ k0, lo1, hi0 ^ c.w ^ k1, lo0);
    }
    return c;
}

// counter {0, 0, k_lo, k_hi} under key = seed
__device__ __forceinline__ uint4 words(uint64_t seed, uint64_t k) {
    return rounds10(make_uint4(0u, 0u, (uint32_t) k, (uint32_t) (k >> 32)), (uint32_t) seed, (uint32_t) (seed >> 32));
}

__device__ __forceinline__ float normal(uint32_t w0, uint32_t w1) {
    const float u = __fadd_rn(__fmul_rn(__uint2float_rn(w0), kInv32), kInv32Half);
    const float a = __fadd_rn(__fmul_rn(__uint2float_rn(w1), kInv32Tau), kInv32TauHalf);
    return __fmul_rn(__fsqrt_rn(__fmul_rn(-2.0f, logf(u))), sinf(a));
}

// round to nearest even through bfloat16 (the values are never NaN)
__device__ __forceinline__ float bf16_round(float z) {
    return __bfloat162float(__float2bfloat16_rn(z));
}

__device__ __forceinline__ float randn(uint64_t seed, uint64_t k, bool round_bf16) {
    const uint4 w = words(seed, k);
    const float z = normal(w.x, w.y);
    return round_bf16 ? bf16_round(z) : z;
}

}  // namespace philox
}  // namespace acb
