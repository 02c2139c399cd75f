// k_stork.cu -- the STORK4 solver's device arithmetic (src/solvers/solver-stork.h): velocity
// derivatives from the step history and one ROCK4 sub-stepping pass, each a single pass over the
// latent.
//
//   stork4_derivs       dv = (v_prev - vt) / h1, d2v from the three-point formula in double
//                       (_stork_compute_derivatives, solver-stork.h:72-127), and the double sums of
//                       squares of vt, dv, d2v that its stability guards compare (fixed-order
//                       block partials, so the sums do not depend on scheduling)
//   stork4_substep      the Chebyshev recurrence over mdeg sub steps and the 4-stage finishing
//                       procedure (_rock4_substep, solver-stork.h:160-268) with every stage kept in
//                       registers: each element reads xt, vt, dv, d2v once and writes its result
//                       once, where the reference streams three n-long buffers per sub step. The
//                       per-sub-step scalars (computed on the host exactly as the reference does)
//                       come in a small table; a non-finite result sets *nonfinite.
// Every operation is a separately rounded f32 (or, for d2v, f64) operation in the reference's
// order.
#include "common.cuh"

namespace acb {
namespace {

constexpr int kStThreads = 256;

__device__ __forceinline__ float taylor(int order, float diff, float half_diff2, float v, float dv, float d2v) {
    if (order >= 2) {
        return __fadd_rn(__fadd_rn(v, __fmul_rn(diff, dv)), __fmul_rn(half_diff2, d2v));
    }
    if (order == 1) {
        return __fadd_rn(v, __fmul_rn(diff, dv));
    }
    return v;
}

__global__ void stork_derivs_kernel(const float * __restrict__ vt, const float * __restrict__ v1, float h1,
                                    const float * __restrict__ v2, float h2, int want2, int64_t n,
                                    float * __restrict__ dv, float * __restrict__ d2v, double * __restrict__ part) {
    __shared__ double red[3][kStThreads / 32];
    const double h1d = (double) h1, h2d = (double) h2;
    const double coeff = 2.0 / (h1d * h2d * (h1d + h2d));
    double       s0 = 0.0, s1 = 0.0, s2 = 0.0;
    for (int64_t i = (int64_t) blockIdx.x * kStThreads + threadIdx.x; i < n; i += (int64_t) gridDim.x * kStThreads) {
        const float v = vt[i];
        const float d = __fdiv_rn(__fsub_rn(v1[i], v), h1);
        dv[i]         = d;
        s0            = __dadd_rn(s0, __dmul_rn((double) v, (double) v));
        s1            = __dadd_rn(s1, __dmul_rn((double) d, (double) d));
        if (want2) {
            const double t = __dadd_rn(__dsub_rn(__dmul_rn((double) v2[i], h1d), __dmul_rn((double) v1[i], h1d + h2d)),
                                       __dmul_rn((double) v, h2d));
            const float  e = __double2float_rn(__dmul_rn(coeff, t));
            d2v[i]         = e;
            s2             = __dadd_rn(s2, __dmul_rn((double) e, (double) e));
        }
    }
    for (int o = 16; o > 0; o >>= 1) {
        s0 = __dadd_rn(s0, __shfl_xor_sync(0xffffffffu, s0, o));
        s1 = __dadd_rn(s1, __shfl_xor_sync(0xffffffffu, s1, o));
        s2 = __dadd_rn(s2, __shfl_xor_sync(0xffffffffu, s2, o));
    }
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (l == 0) {
        red[0][w] = s0;
        red[1][w] = s1;
        red[2][w] = s2;
    }
    __syncthreads();
    if (threadIdx.x < 3) {
        double s = 0.0;
        for (int k = 0; k < kStThreads / 32; k++) {
            s = __dadd_rn(s, red[threadIdx.x][k]);
        }
        part[(size_t) blockIdx.x * 3 + threadIdx.x] = s;
    }
}

__global__ void stork_sum_kernel(const double * __restrict__ part, int nblk, double * __restrict__ sums) {
    if (threadIdx.x < 3) {
        double s = 0.0;
        for (int b = 0; b < nblk; b++) {
            s = __dadd_rn(s, part[(size_t) b * 3 + threadIdx.x]);
        }
        sums[threadIdx.x] = s;
    }
}

// The scalars outside the recurrence table (coef[j] = {temp1, temp2, temp3, diff} of sub step j):
// sub step 1's temp1, and the finishing stages' Taylor offsets and final weights.
struct StorkFin {
    float t1_first;  // -dt * RECF[mr]
    float diff[4];   // finishing stages' Taylor offsets
    float fpb[4];
};

__global__ void stork_substep_kernel(const float * __restrict__ xt, const float * __restrict__ vt,
                                     const float * __restrict__ dvp, const float * __restrict__ d2vp, int order,
                                     const float4 * __restrict__ coef, int mdeg, const StorkFin fin, int64_t n,
                                     float * __restrict__ out, int * __restrict__ nonfinite) {
    const int64_t i = (int64_t) blockIdx.x * kStThreads + threadIdx.x;
    if (i >= n) {
        return;
    }
    const float x  = xt[i];
    const float v  = vt[i];
    const float dv = order >= 1 ? dvp[i] : 0.0f;
    const float d2 = order >= 2 ? d2vp[i] : 0.0f;
    // sub step 1: Y_1 = xt + temp1 * vt, Y_0 = xt
    float y1 = __fadd_rn(x, __fmul_rn(fin.t1_first, v));
    float y2 = x;
    for (int j = 2; j <= mdeg; j++) {
        const float4 c    = coef[j];
        const float  half = __fmul_rn(__fmul_rn(0.5f, c.w), c.w);
        const float  vel  = taylor(order, c.w, half, v, dv, d2);
        const float  y = __fadd_rn(__fadd_rn(__fmul_rn(c.x, vel), __fmul_rn(c.y, y1)), __fmul_rn(c.z, y2));
        y2             = y1;
        y1             = y;
    }
    float f[4];
#pragma unroll
    for (int k = 0; k < 4; k++) {
        const float d = fin.diff[k];
        f[k]          = taylor(order, d, __fmul_rn(__fmul_rn(0.5f, d), d), v, dv, d2);
    }
    float r = __fadd_rn(y1, __fmul_rn(fin.fpb[0], f[0]));
    r       = __fadd_rn(r, __fmul_rn(fin.fpb[1], f[1]));
    r       = __fadd_rn(r, __fmul_rn(fin.fpb[2], f[2]));
    r       = __fadd_rn(r, __fmul_rn(fin.fpb[3], f[3]));
    out[i]  = r;
    if (!isfinite(r)) {
        atomicOr(nonfinite, 1);
    }
}

}  // namespace
}  // namespace acb

namespace acb {

// Launchers used by host/stork.cpp (declared in host/stork.h).
acb_status stork4_derivs(const float * vt, const float * v1, float h1, const float * v2, float h2, int want2,
                         int64_t n, float * dv, float * d2v, double * part, int nblk, double * sums,
                         cudaStream_t s) {
    stork_derivs_kernel<<<nblk, kStThreads, 0, s>>>(vt, v1, h1, v2, h2, want2, n, dv, d2v, part);
    stork_sum_kernel<<<1, 32, 0, s>>>(part, nblk, sums);
    return launch_status();
}

acb_status stork4_substep(const float * xt, const float * vt, const float * dv, const float * d2v, int order,
                          const float * coef4, int mdeg, float t1_first, const float * diff4, const float * fpb4,
                          int64_t n, float * out, int * nonfinite, cudaStream_t s) {
    StorkFin fin;
    fin.t1_first = t1_first;
    for (int k = 0; k < 4; k++) {
        fin.diff[k] = diff4[k];
        fin.fpb[k]  = fpb4[k];
    }
    const int64_t nb = (n + kStThreads - 1) / kStThreads;
    if (nb > 2147483647LL) {
        return ACB_ERR_UNSUPPORTED;
    }
    stork_substep_kernel<<<(unsigned) nb, kStThreads, 0, s>>>(xt, vt, dv, d2v, order,
                                                                reinterpret_cast<const float4 *>(coef4), mdeg, fin,
                                                                n, out, nonfinite);
    return launch_status();
}

}  // namespace acb
