// stork.h -- device launchers of the STORK4 solver (csrc/k_stork.cu) for host/stork.cpp.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/acb.h"

namespace acb {

// dv, d2v (want2) and the double sums of squares {vt, dv, d2v} into sums[3]; part: nblk * 3 doubles
acb_status stork4_derivs(const float * vt, const float * v1, float h1, const float * v2, float h2, int want2,
                         int64_t n, float * dv, float * d2v, double * part, int nblk, double * sums, cudaStream_t s);
// one ROCK4 pass: coef4 device float4 [mdeg + 1] ({temp1, temp2, temp3, diff} of sub step j at j),
// finishing Taylor offsets diff4 and weights fpb4 (host), result in out, *nonfinite |= 1 when any
// element is not finite
acb_status stork4_substep(const float * xt, const float * vt, const float * dv, const float * d2v, int order,
                          const float * coef4, int mdeg, float t1_first, const float * diff4, const float * fpb4,
                          int64_t n, float * out, int * nonfinite, cudaStream_t s);

}  // namespace acb
