// k_quantize.cu -- on-device quantisation of f32 rows into GGUF blocks.
//   Q8_0: d = amax/127, q = roundf(x * (1/d)) (ggml's reference Q8_0 quantiser; gguf-py
//         documents its numpy port as bit-exact with it)
//   Q4_K: per 32-element sub-block scale (max-min)/15 and offset -min, both as 6-bit
//         multiples of f16 super-scales (max/63)
//   Q6_K: per 16-element group scale amax/31 as an int8 multiple of an f16 super-scale (max/127)
// The K-quant encoders are simple min/max encoders producing valid blocks (ggml's own K-quant
// quantisers are search-based); they exist to make synthetic weights. One thread per block.
#include "common.cuh"

namespace acb {

__device__ __forceinline__ void st_u16(uint8_t * p, uint16_t v) {
    p[0] = (uint8_t) (v & 0xff);
    p[1] = (uint8_t) (v >> 8);
}

// one warp per 32-element block: lane j owns element j
__global__ void quant_q8_0_kernel(const float * __restrict__ x, int64_t nblk, uint8_t * __restrict__ dst) {
    const int64_t b    = (int64_t) blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int     lane = threadIdx.x & 31;
    if (b >= nblk) {
        return;
    }
    const float v    = x[b * 32 + lane];
    const float amax = warp_max(fabsf(v));
    const float d    = amax / 127.0f;
    const float id   = d != 0.0f ? 1.0f / d : 0.0f;
    uint8_t *   o    = dst + b * 34;  // 2-byte aligned
    if (lane == 0) {
        *reinterpret_cast<uint16_t *>(o) = __half_as_ushort(__float2half_rn(d));
    }
    o[2 + lane] = (uint8_t) (int8_t) roundf(__fmul_rn(v, id));
}

__global__ void quant_q4_K_kernel(const float * __restrict__ x, int64_t nblk, uint8_t * __restrict__ dst) {
    const int64_t b = (int64_t) blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= nblk) {
        return;
    }
    const float * xb  = x + b * 256;
    uint8_t *     blk = dst + b * 144;
    float         scl[8], mns[8];
    float         max_scale = 0.0f, max_min = 0.0f;
    for (int s = 0; s < 8; s++) {
        float lo = xb[s * 32], hi = xb[s * 32];
        for (int j = 1; j < 32; j++) {
            const float v = xb[s * 32 + j];
            lo            = v < lo ? v : lo;
            hi            = v > hi ? v : hi;
        }
        if (lo > 0.0f) {
            lo = 0.0f;
        }
        scl[s] = __fdiv_rn(__fsub_rn(hi, lo), 15.0f);
        mns[s] = -lo;
        if (scl[s] > max_scale) {
            max_scale = scl[s];
        }
        if (mns[s] > max_min) {
            max_min = mns[s];
        }
    }
    const float    d     = __fdiv_rn(max_scale, 63.0f);
    const float    dmin  = __fdiv_rn(max_min, 63.0f);
    const uint16_t dh    = __half_as_ushort(__float2half_rn(d));
    const uint16_t dmh   = __half_as_ushort(__float2half_rn(dmin));
    const float    dq    = __half2float(__ushort_as_half(dh));
    const float    dminq = __half2float(__ushort_as_half(dmh));
    int            ls[8], lm[8];
    for (int s = 0; s < 8; s++) {
        const int a = dq > 0.0f ? (int) lroundf(__fdiv_rn(scl[s], dq)) : 0;
        const int c = dminq > 0.0f ? (int) lroundf(__fdiv_rn(mns[s], dminq)) : 0;
        ls[s]       = a < 0 ? 0 : (a > 63 ? 63 : a);
        lm[s]       = c < 0 ? 0 : (c > 63 ? 63 : c);
    }
    st_u16(blk, dh);
    st_u16(blk + 2, dmh);
    uint8_t * sc = blk + 4;
    for (int j = 0; j < 4; j++) {
        sc[j]     = (uint8_t) ((ls[j] & 63) | ((ls[j + 4] >> 4) << 6));
        sc[j + 4] = (uint8_t) ((lm[j] & 63) | ((lm[j + 4] >> 4) << 6));
        sc[j + 8] = (uint8_t) ((ls[j + 4] & 0x0f) | ((lm[j + 4] & 0x0f) << 4));
    }
    uint8_t * qs = blk + 16;
    for (int g = 0; g < 4; g++) {
        const float ds0 = __fmul_rn(dq, (float) ls[2 * g]), dm0 = __fmul_rn(dminq, (float) lm[2 * g]);
        const float ds1 = __fmul_rn(dq, (float) ls[2 * g + 1]), dm1 = __fmul_rn(dminq, (float) lm[2 * g + 1]);
        for (int j = 0; j < 32; j++) {
            int q0 = ds0 > 0.0f ? (int) lroundf(__fdiv_rn(__fadd_rn(xb[64 * g + j], dm0), ds0)) : 0;
            int q1 = ds1 > 0.0f ? (int) lroundf(__fdiv_rn(__fadd_rn(xb[64 * g + 32 + j], dm1), ds1)) : 0;
            q0     = q0 < 0 ? 0 : (q0 > 15 ? 15 : q0);
            q1     = q1 < 0 ? 0 : (q1 > 15 ? 15 : q1);
            qs[g * 32 + j] = (uint8_t) (q0 | (q1 << 4));
        }
    }
}

__global__ void quant_q6_K_kernel(const float * __restrict__ x, int64_t nblk, uint8_t * __restrict__ dst) {
    const int64_t b = (int64_t) blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= nblk) {
        return;
    }
    const float * xb  = x + b * 256;
    uint8_t *     blk = dst + b * 210;
    float         gs[16];
    float         mx = 0.0f;
    for (int g = 0; g < 16; g++) {
        float amax = 0.0f;
        for (int j = 0; j < 16; j++) {
            amax = fmaxf(amax, fabsf(xb[g * 16 + j]));
        }
        gs[g] = __fdiv_rn(amax, 31.0f);
        mx    = gs[g] > mx ? gs[g] : mx;
    }
    const float    d  = __fdiv_rn(mx, 127.0f);
    const uint16_t dh = __half_as_ushort(__float2half_rn(d));
    const float    dq = __half2float(__ushort_as_half(dh));
    int8_t *       sc = (int8_t *) (blk + 192);
    for (int g = 0; g < 16; g++) {
        const int s = dq > 0.0f ? (int) lroundf(__fdiv_rn(gs[g], dq)) : 0;
        sc[g]       = (int8_t) (s > 127 ? 127 : s);
    }
    st_u16(blk + 208, dh);
    uint8_t * ql = blk;
    uint8_t * qh = blk + 128;
    for (int i = 0; i < 128; i++) {
        ql[i] = 0;
    }
    for (int i = 0; i < 64; i++) {
        qh[i] = 0;
    }
    for (int j = 0; j < 256; j++) {
        const float ds = __fmul_rn(dq, (float) sc[j >> 4]);
        int         q  = ds > 0.0f ? (int) lroundf(__fdiv_rn(xb[j], ds)) : 0;
        q              = q < -32 ? -32 : (q > 31 ? 31 : q);
        const int u    = q + 32;
        const int half = j >> 7, c = (j >> 5) & 3, l = j & 31;
        const int li   = half * 64 + ((c & 1) ? 32 : 0) + l;
        ql[li] |= (c & 2) ? (uint8_t) ((u & 0x0f) << 4) : (uint8_t) (u & 0x0f);
        qh[half * 32 + l] |= (uint8_t) (((u >> 4) & 3) << (2 * c));
    }
}

}  // namespace acb

using namespace acb;

extern "C" acb_status acb_quantize(const float * x, int64_t rows, int64_t K, int type, void * dst,
                                   acb_stream_t stream) {
    if (!x || !dst || rows < 0 || K <= 0) {
        return ACB_ERR_INVALID_ARG;
    }
    const int64_t be = type == ACB_TYPE_Q8_0 ? 32 : 256;
    if (type != ACB_TYPE_Q8_0 && type != ACB_TYPE_Q4_K && type != ACB_TYPE_Q6_K) {
        return ACB_ERR_UNSUPPORTED;
    }
    if (K % be != 0) {
        return ACB_ERR_INVALID_ARG;
    }
    const int64_t nblk = rows * (K / be);
    if (nblk == 0) {
        return ACB_OK;
    }
    const dim3   grid((unsigned) ((nblk + 127) / 128));
    cudaStream_t st = (cudaStream_t) stream;
    if (type == ACB_TYPE_Q8_0) {
        quant_q8_0_kernel<<<dim3((unsigned) ((nblk + 7) / 8)), 256, 0, st>>>(x, nblk, (uint8_t *) dst);
    } else if (type == ACB_TYPE_Q4_K) {
        quant_q4_K_kernel<<<grid, 128, 0, st>>>(x, nblk, (uint8_t *) dst);
    } else {
        quant_q6_K_kernel<<<grid, 128, 0, st>>>(x, nblk, (uint8_t *) dst);
    }
    return launch_status();
}
