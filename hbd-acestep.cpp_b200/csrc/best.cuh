// best.cuh -- running (best, second, index) triple of a greedy argmax: the lowest index wins
// ties, and the second value is the runner-up in the multiset (equal to the best on a tie), so
// any merge order gives the same triple.
#pragma once

namespace acb {

struct Best {
    float b1;
    float b2;
    int   i1;
};

__device__ __forceinline__ void best_push(Best & s, float v, int i) {
    if (v > s.b1) {
        s.b2 = s.b1;
        s.b1 = v;
        s.i1 = i;
    } else if (v > s.b2) {
        s.b2 = v;
    }
}

__device__ __forceinline__ void best_merge(Best & s, float ob1, float ob2, int oi) {
    if (ob1 > s.b1 || (ob1 == s.b1 && oi < s.i1)) {
        s.b2 = fmaxf(s.b1, ob2);
        s.b1 = ob1;
        s.i1 = oi;
    } else {
        s.b2 = fmaxf(s.b2, ob1);
    }
}

}  // namespace acb
