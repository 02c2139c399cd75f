// vae.cpp -- the AutoencoderOobleck audio decoder (src/vae.h) on libacb kernels: latents
// [T][64] -> stereo audio [2][T * 1920].
//
//   conv1 (64 -> C0, k 7)                         f16 cast, implicit-GEMM conv + bias -> x (f32)
//   5 blocks: snake -> ConvTranspose (s, k 2s)    snake (f16), 3-tap implicit-GEMM conv (below)
//             3 res units (dilation 1, 3, 9):       + bias -> x
//               snake -> conv k7 -> snake ->      snake (f16), k7 conv + bias -> h (f32), snake
//               conv k1 -> + x                    (f16), k1 conv: x += v + bias (in place)
//   snake -> conv2 (C -> 2, k 7, no bias)         direct kernel, planar output
// Every convolution with more than two output channels is one tcgen05 GEMM (f16 operands, f32
// accumulation) reading its taps straight from the f16 activation (acb_conv1d_tc, no im2col):
// ggml's conv_1d casts the activation to the f16 weight type, so the operands are those of the
// reference. The snakes run as their own full-occupancy pass (acb_vae_snake_f16): folded into the
// GEMM epilogue the sine made the four epilogue warps the bottleneck (36.8 instead of 20.4 ms for
// 30 s of audio).
// ConvTranspose1d with kernel 2s, stride s, padding s/2 (s even): output row s*q + r takes input
// rows q-1 and q (r < s/2) or q and q+1 (r >= s/2), so it is a 3-tap convolution over the input
// with s*OC output columns, phase-major ([T_in][s*OC] is the upsampled [T_in*s][OC]): the weights
// are laid out W3[r*OC + oc][(j+1)*IC + ic] = w[ic][oc][k] for the tap k that phase r takes from
// input row q + j (zero where a phase takes nothing from that row). The two contributions of
// ggml_col2im_1d are summed inside the GEMM's f32 accumulation instead of after it.
// Weight normalisation is fused at load exactly as vae_fuse_wn / vae_fuse_wn_ct do (f32,
// sequential sum of squares), the weights rounded to f16 as the reference stores them. Channel
// counts and strides come from the tensor shapes (the shipped model: 2048 -> 1024 -> 512 -> 256 ->
// 128 -> 128, strides 10, 6, 4, 4, 2). Tiled decoding (vae_ggml_decode_tiled) keeps the
// reference's windows and trims.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <memory>
#include <string>
#include <vector>

#include "../../include/acb_models.h"
#include "gguf.h"
#include "host_common.h"
#include "weights.h"

using namespace acb;

namespace {

struct Conv {  // a convolution as a GEMM: B [N][Kp] f16 (Kp = kernel * C_in), bias f32 [N]
    int    N = 0, Kp = 0, cin = 0, kernel = 1, dil = 1;
    DevBuf w, b;
};

struct Snake {  // e^alpha and e^-beta, f32 [C]
    DevBuf ea, ib;
};

struct ResUnit {
    Snake s1, s2;
    Conv  c1, c2;
};

struct Block {
    int     in_ch = 0, out_ch = 0, stride = 0, kernel = 0;
    Snake   sn;       // the snake in front of the transposed conv
    Conv    ct;       // 3-tap form: B [stride * out_ch][3 * in_ch]
    DevBuf  ctb;      // bias tiled over the stride phases [stride * out_ch]
    ResUnit ru[3];
};

float bf16f(const uint8_t * p, int64_t i) {
    uint16_t h;
    memcpy(&h, p + 2 * i, 2);
    return host_bf16_to_f32(h);
}

// a GGUF tensor as f32 values (BF16, F16 or F32 storage)
bool read_f32(const GGUFFile & gf, const std::string & name, std::vector<float> & out, int64_t * ne = nullptr) {
    const GGUFTensor * t = gf.find(name);
    if (!t) {
        set_last_error("VAE tensor '" + name + "' not found");
        return false;
    }
    int64_t n = 1;
    for (int d = 0; d < t->n_dims; d++) {
        n *= t->ne[d];
        if (ne) {
            ne[d] = t->ne[d];
        }
    }
    out.resize((size_t) n);
    for (int64_t i = 0; i < n; i++) {
        if (t->type == ACB_TYPE_BF16) {
            out[(size_t) i] = bf16f(t->data, i);
        } else if (t->type == ACB_TYPE_F16) {
            uint16_t h;
            memcpy(&h, t->data + 2 * i, 2);
            out[(size_t) i] = host_f16_to_f32(h);
        } else if (t->type == ACB_TYPE_F32) {
            memcpy(&out[(size_t) i], t->data + 4 * i, 4);
        } else {
            set_last_error("VAE tensor '" + name + "' has an unsupported type");
            return false;
        }
    }
    return true;
}

// weight_norm over dim 0 (vae_fuse_wn, vae.h:64-93; vae_fuse_wn_ct, :100-128): w[d][i] = v[d][i] * g[d] / (|v[d]| + 1e-12),
// the norm from a sequential f32 sum of squares
std::vector<float> fuse_wn(const std::vector<float> & g, const std::vector<float> & v, int64_t dim0) {
    const int64_t      fan = (int64_t) v.size() / dim0;
    std::vector<float> w(v.size());
    for (int64_t d = 0; d < dim0; d++) {
        float nsq = 0.0f;
        for (int64_t i = 0; i < fan; i++) {
            const float vv = v[(size_t) (d * fan + i)];
            const float sq = vv * vv;
            nsq            = nsq + sq;
        }
        const float s = g[(size_t) d] / (sqrtf(nsq) + 1e-12f);
        for (int64_t i = 0; i < fan; i++) {
            w[(size_t) (d * fan + i)] = v[(size_t) (d * fan + i)] * s;
        }
    }
    return w;
}

acb_status upload_f32(DevBuf & b, const std::vector<float> & h) {
    ACB_TRY(b.alloc(h.size() * 4, false));
    return cudaMemcpy(b.p, h.data(), h.size() * 4, cudaMemcpyHostToDevice) == cudaSuccess ? ACB_OK : ACB_ERR_CUDA;
}

// f32 host values -> f16 device buffer (rounded to nearest even on the device)
acb_status upload_f16(DevBuf & b, const std::vector<float> & h, DevBuf & tmp) {
    ACB_TRY(b.alloc(h.size() * 2, false));
    if (tmp.bytes < h.size() * 4) {
        ACB_TRY(tmp.alloc(h.size() * 4, false));
    }
    if (cudaMemcpy(tmp.p, h.data(), h.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    ACB_TRY(acb_requant(tmp.as<float>(), 1, (int64_t) h.size(), ACB_TYPE_F16, b.p, nullptr));
    return cudaDeviceSynchronize() == cudaSuccess ? ACB_OK : ACB_ERR_CUDA;
}

acb_status load_snake(const GGUFFile & gf, const std::string & pfx, Snake & s, int * C) {
    std::vector<float> a, b;
    if (!read_f32(gf, pfx + ".alpha", a) || !read_f32(gf, pfx + ".beta", b) || a.size() != b.size()) {
        return ACB_ERR_FORMAT;
    }
    for (size_t i = 0; i < a.size(); i++) {  // vae_load_snake / vae_load_snake_inv (:131-152)
        a[i] = expf(a[i]);
        b[i] = 1.0f / expf(b[i]);
    }
    *C = (int) a.size();
    ACB_TRY(upload_f32(s.ea, a));
    return upload_f32(s.ib, b);
}

// Conv1d [OC][IC][K] (GGUF ne = [K, IC, OC]) -> B[oc][k*IC + ic]
acb_status load_conv(const GGUFFile & gf, const std::string & pfx, Conv & c, int dil, bool bias, DevBuf & tmp) {
    std::vector<float> g, v, b;
    int64_t            ne[4] = { 1, 1, 1, 1 };
    if (!read_f32(gf, pfx + ".weight_g", g) || !read_f32(gf, pfx + ".weight_v", v, ne)) {
        return ACB_ERR_FORMAT;
    }
    const int64_t K = ne[0], IC = ne[1], OC = ne[2];
    if ((int64_t) g.size() != OC || K * IC * OC != (int64_t) v.size()) {
        set_last_error("VAE conv '" + pfx + "' has unexpected shapes");
        return ACB_ERR_FORMAT;
    }
    const std::vector<float> w = fuse_wn(g, v, OC);
    std::vector<float>       p((size_t) (OC * K * IC));
    for (int64_t oc = 0; oc < OC; oc++) {
        for (int64_t ic = 0; ic < IC; ic++) {
            for (int64_t k = 0; k < K; k++) {
                p[(size_t) (oc * K * IC + k * IC + ic)] = w[(size_t) ((oc * IC + ic) * K + k)];
            }
        }
    }
    c.N = (int) OC, c.cin = (int) IC, c.kernel = (int) K, c.Kp = (int) (K * IC), c.dil = dil;
    ACB_TRY(upload_f16(c.w, p, tmp));
    if (bias) {
        if (!read_f32(gf, pfx + ".bias", b) || (int64_t) b.size() != OC) {
            return ACB_ERR_FORMAT;
        }
        ACB_TRY(upload_f32(c.b, b));
    }
    return ACB_OK;
}

}  // namespace

struct acb_vae {
    int          device = 0;
    cudaStream_t st     = nullptr;
    int          latent = 64, up = 1;  // input channels, total upsampling
    Conv         c1;
    Block        blk[5];
    Snake        sn;           // final snake
    int          c_last = 0;   // channels into conv2
    DevBuf       c2w;          // [2][7][c_last] f16
    DevBuf       x, h, a16, ws, err, lat, out;

    ~acb_vae() {
        cudaSetDevice(device);
        if (st) {
            cudaStreamDestroy(st);
        }
    }

    acb_status grow(DevBuf & b, size_t bytes) {
        if (b.bytes >= bytes) {
            return ACB_OK;
        }
        // the split-K workspace starts zeroed; the other buffers are written before they are read
        return b.alloc(bytes, &b == &ws) == ACB_OK ? ACB_OK : ACB_ERR_OOM;
    }

    // one convolution over the f16 activation X [T][c.cin]: y [T][ldy] f32 = conv + bias (+ res)
    acb_status conv(const Conv & c, const void * X, int64_t T, int pad, float * y, int64_t ldy, const float * bias,
                    const float * res) {
        return acb_conv1d_tc(X, c.cin, T, c.cin, c.w.p, c.N, c.kernel, c.dil, pad, y, ACB_TYPE_F32, ldy, bias, res,
                             ldy, ACB_FLAG_F16, ws.p, ws.bytes, err.as<int>(), (acb_stream_t) st);
    }

    acb_status reserve(int64_t T0);
    acb_status run(const float * d_latent, int64_t T0, float * d_audio);
};

acb_status acb_vae::reserve(int64_t T0) {
    int64_t T = T0, mx = T0 * std::max(c1.N, latent);
    size_t  wsb = acb_gemm_workspace_bytes(T0, c1.N, c1.Kp);
    for (const Block & b : blk) {
        wsb = std::max(wsb, acb_gemm_workspace_bytes(T, b.ct.N, b.ct.Kp));
        T *= b.stride;
        mx = std::max(mx, T * (int64_t) b.out_ch);
        for (const ResUnit & r : b.ru) {
            wsb = std::max({ wsb, acb_gemm_workspace_bytes(T, r.c1.N, r.c1.Kp),
                             acb_gemm_workspace_bytes(T, r.c2.N, r.c2.Kp) });
        }
    }
    ACB_TRY(grow(x, (size_t) mx * 4));
    ACB_TRY(grow(h, (size_t) mx * 4));
    ACB_TRY(grow(a16, (size_t) mx * 2));
    ACB_TRY(grow(ws, std::max(wsb, (size_t) 256)));
    return ACB_OK;
}

// vae_ggml_build_graph (vae.h:344-369) on device buffers: d_latent [T0][latent] f32 ->
// d_audio [2][T0 * up] f32. a16 holds the f16 operand of the next conv.
acb_status acb_vae::run(const float * d_latent, int64_t T0, float * d_audio) {
    const acb_stream_t as = (acb_stream_t) st;
    int64_t            T  = T0;
    float *            xp = x.as<float>();
    float *            hp = h.as<float>();
    void *             A  = a16.p;
    // conv1, no snake in front: its input is the latent cast to f16
    ACB_TRY(acb_vae_snake_f16(d_latent, latent, T, latent, nullptr, nullptr, A, latent, as));
    ACB_TRY(conv(c1, A, T, c1.kernel / 2, xp, c1.N, c1.b.as<float>(), nullptr));
    int C = c1.N;
    for (Block & b : blk) {
        const int64_t sN = (int64_t) b.stride * b.out_ch;
        // snake -> ConvTranspose1d as the 3-tap phase-major convolution: [T][s*OC] = [T*s][OC]
        ACB_TRY(acb_vae_snake_f16(xp, C, T, C, b.sn.ea.as<float>(), b.sn.ib.as<float>(), A, C, as));
        ACB_TRY(conv(b.ct, A, T, 1, xp, sN, b.ctb.as<float>(), nullptr));
        T *= b.stride;
        C = b.out_ch;
        for (ResUnit & u : b.ru) {
            ACB_TRY(acb_vae_snake_f16(xp, C, T, C, u.s1.ea.as<float>(), u.s1.ib.as<float>(), A, C, as));
            ACB_TRY(conv(u.c1, A, T, (u.c1.kernel / 2) * u.c1.dil, hp, C, u.c1.b.as<float>(), nullptr));
            ACB_TRY(acb_vae_snake_f16(hp, C, T, C, u.s2.ea.as<float>(), u.s2.ib.as<float>(), A, C, as));
            ACB_TRY(conv(u.c2, A, T, 0, xp, C, u.c2.b.as<float>(), xp));  // + skip, in place
        }
    }
    return acb_vae_out_conv(xp, T, C, sn.ea.as<float>(), sn.ib.as<float>(), c2w.p, d_audio, as);
}

extern "C" acb_status acb_vae_load(const char * gguf_path, int device, acb_vae ** out) {
    if (!gguf_path || !out) {
        return ACB_ERR_INVALID_ARG;
    }
    *out = nullptr;
    if (cudaSetDevice(device) != cudaSuccess) {
        set_last_error("cannot select CUDA device");
        return ACB_ERR_CUDA;
    }
    GGUFFile gf;
    if (!gf.open(gguf_path)) {
        set_last_error(gf.error());
        return gf.error().rfind("cannot open", 0) == 0 ? ACB_ERR_IO : ACB_ERR_FORMAT;
    }
    std::unique_ptr<acb_vae> m(new acb_vae());
    m->device = device;
    if (cudaStreamCreateWithFlags(&m->st, cudaStreamNonBlocking) != cudaSuccess || m->err.alloc(4) != ACB_OK) {
        return ACB_ERR_CUDA;
    }
    DevBuf tmp;
    ACB_TRY(load_conv(gf, "decoder.conv1", m->c1, 1, true, tmp));
    m->latent = m->c1.cin;
    int C     = m->c1.N;
    m->up     = 1;
    static const int dil[3] = { 1, 3, 9 };
    for (int i = 0; i < 5; i++) {
        Block &           b = m->blk[i];
        const std::string p = "decoder.block." + std::to_string(i);
        int               sc = 0;
        ACB_TRY(load_snake(gf, p + ".snake1", b.sn, &sc));
        // ConvTranspose1d [IC][OC][K] (GGUF ne = [K, OC, IC]), weight norm over IC (vae_fuse_wn_ct)
        std::vector<float> g, v, bias;
        int64_t            ne[4] = { 1, 1, 1, 1 };
        if (!read_f32(gf, p + ".conv_t1.weight_g", g) || !read_f32(gf, p + ".conv_t1.weight_v", v, ne) ||
            !read_f32(gf, p + ".conv_t1.bias", bias)) {
            return ACB_ERR_FORMAT;
        }
        const int64_t K = ne[0], OC = ne[1], IC = ne[2];
        if (IC != C || sc != C || (int64_t) g.size() != IC || (int64_t) bias.size() != OC || K % 2 != 0) {
            set_last_error("VAE block " + std::to_string(i) + " shapes do not chain");
            return ACB_ERR_FORMAT;
        }
        const std::vector<float> w = fuse_wn(g, v, IC);  // [IC][OC][K]
        const int64_t            s = K / 2;
        if (s % 2 != 0) {
            set_last_error("VAE block " + std::to_string(i) + ": odd stride (the 3-tap form needs padding s/2)");
            return ACB_ERR_UNSUPPORTED;
        }
        // W3[r*OC + oc][(j+1)*IC + ic] = w[ic][oc][k]: phase r takes tap k from input row q + j
        std::vector<float> pw((size_t) (s * OC * 3 * IC), 0.0f);
        for (int64_t r = 0; r < s; r++) {
            const int64_t kj[3] = { r < s / 2 ? r + 3 * s / 2 : -1, r + s / 2, r >= s / 2 ? r - s / 2 : -1 };
            for (int64_t oc = 0; oc < OC; oc++) {
                float * row = &pw[(size_t) ((r * OC + oc) * 3 * IC)];
                for (int j = 0; j < 3; j++) {
                    if (kj[j] < 0) {
                        continue;
                    }
                    for (int64_t ic = 0; ic < IC; ic++) {
                        row[j * IC + ic] = w[(size_t) ((ic * OC + oc) * K + kj[j])];
                    }
                }
            }
        }
        b.in_ch = (int) IC, b.out_ch = (int) OC, b.kernel = (int) K, b.stride = (int) s;
        b.ct.N = (int) (s * OC), b.ct.Kp = (int) (3 * IC), b.ct.cin = (int) IC, b.ct.kernel = 3, b.ct.dil = 1;
        ACB_TRY(upload_f16(b.ct.w, pw, tmp));
        std::vector<float> tb((size_t) (s * OC));
        for (int64_t r = 0; r < s; r++) {
            std::copy(bias.begin(), bias.end(), tb.begin() + r * OC);
        }
        ACB_TRY(upload_f32(b.ctb, tb));
        C = (int) OC;
        m->up *= b.stride;
        for (int r = 0; r < 3; r++) {
            ResUnit &         u  = b.ru[r];
            const std::string rp = p + ".res_unit" + std::to_string(r + 1);
            int               c1 = 0, c2 = 0;
            ACB_TRY(load_snake(gf, rp + ".snake1", u.s1, &c1));
            ACB_TRY(load_snake(gf, rp + ".snake2", u.s2, &c2));
            ACB_TRY(load_conv(gf, rp + ".conv1", u.c1, dil[r], true, tmp));
            ACB_TRY(load_conv(gf, rp + ".conv2", u.c2, 1, true, tmp));
            if (c1 != C || c2 != C || u.c1.N != C || u.c1.cin != C || u.c2.N != C || u.c2.cin != C ||
                u.c1.kernel % 2 != 1 || u.c2.kernel != 1) {
                set_last_error("VAE res unit shapes do not chain");
                return ACB_ERR_FORMAT;
            }
        }
    }
    int sc = 0;
    ACB_TRY(load_snake(gf, "decoder.snake1", m->sn, &sc));
    {
        std::vector<float> g, v;
        int64_t            ne[4] = { 1, 1, 1, 1 };
        if (!read_f32(gf, "decoder.conv2.weight_g", g) || !read_f32(gf, "decoder.conv2.weight_v", v, ne)) {
            return ACB_ERR_FORMAT;
        }
        const int64_t K = ne[0], IC = ne[1], OC = ne[2];
        if (OC != 2 || K != 7 || IC != C || sc != C) {
            set_last_error("VAE output conv shapes do not match");
            return ACB_ERR_FORMAT;
        }
        const std::vector<float> w = fuse_wn(g, v, OC);
        std::vector<float>       pw((size_t) (OC * K * IC));  // [2][7][C]
        for (int64_t oc = 0; oc < OC; oc++) {
            for (int64_t ic = 0; ic < IC; ic++) {
                for (int64_t k = 0; k < K; k++) {
                    pw[(size_t) ((oc * K + k) * IC + ic)] = w[(size_t) ((oc * IC + ic) * K + k)];
                }
            }
        }
        ACB_TRY(upload_f16(m->c2w, pw, tmp));
    }
    m->c_last = C;
    // every conv's input channel count must be a multiple of 64 (one k-tile of the GEMM holds one
    // 64-channel slice of one tap): the shipped channel counts are multiples of 128
    bool ok = C % 8 == 0 && m->c1.cin % 64 == 0 && m->c1.N % 8 == 0;
    for (const Block & b : m->blk) {
        ok = ok && b.ct.cin % 64 == 0 && b.out_ch % 8 == 0;
        for (const ResUnit & r : b.ru) {
            ok = ok && r.c1.cin % 64 == 0 && r.c2.cin % 64 == 0;
        }
    }
    if (!ok) {
        set_last_error("VAE channel counts must be multiples of 64");
        return ACB_ERR_UNSUPPORTED;
    }
    *out = m.release();
    return ACB_OK;
}

extern "C" int acb_vae_upsample(const acb_vae * m) {
    return m ? m->up : 0;
}

extern "C" acb_status acb_vae_decode_device(acb_vae * m, const float * d_latent, int T_latent, float * d_audio,
                                            acb_stream_t stream) {
    if (!m || !d_latent || !d_audio || T_latent <= 0) {
        return ACB_ERR_INVALID_ARG;
    }
    if (cudaSetDevice(m->device) != cudaSuccess || cudaStreamSynchronize((cudaStream_t) stream) != cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    ACB_TRY(m->reserve(T_latent));
    ACB_TRY(m->run(d_latent, T_latent, d_audio));
    return cudaStreamSynchronize(m->st) == cudaSuccess ? ACB_OK : ACB_ERR_CUDA;
}

// vae_ggml_decode (vae.h:442-459): host latent [T][latent] -> host audio [2][T * up]
extern "C" acb_status acb_vae_decode(acb_vae * m, const float * latent, int T_latent, float * audio_out,
                                     int max_T_audio, int * out_T_audio) {
    if (!m || !latent || !audio_out || T_latent <= 0) {
        return ACB_ERR_INVALID_ARG;
    }
    const int64_t Ta = (int64_t) T_latent * m->up;
    if (Ta > max_T_audio) {
        set_last_error("T_audio exceeds max_T_audio");
        return ACB_ERR_OUT_OF_RANGE;
    }
    if (cudaSetDevice(m->device) != cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    ACB_TRY(m->reserve(T_latent));
    cudaMemsetAsync(m->err.p, 0, 4, m->st);
    if (m->lat.bytes < (size_t) T_latent * m->latent * 4) {
        ACB_TRY(m->lat.alloc((size_t) T_latent * m->latent * 4, false));
    }
    if (m->out.bytes < (size_t) Ta * 2 * 4) {
        ACB_TRY(m->out.alloc((size_t) Ta * 2 * 4, false));
    }
    if (cudaMemcpyAsync(m->lat.p, latent, (size_t) T_latent * m->latent * 4, cudaMemcpyHostToDevice, m->st) !=
        cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    ACB_TRY(m->run(m->lat.as<float>(), T_latent, m->out.as<float>()));
    if (cudaMemcpyAsync(audio_out, m->out.p, (size_t) Ta * 2 * 4, cudaMemcpyDeviceToHost, m->st) != cudaSuccess ||
        cudaStreamSynchronize(m->st) != cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    int flag = 0;
    cudaMemcpy(&flag, m->err.p, 4, cudaMemcpyDeviceToHost);
    if (flag) {
        set_last_error("device error flag " + std::to_string(flag));
        return ACB_ERR_DEVICE;
    }
    if (out_T_audio) {
        *out_T_audio = (int) Ta;
    }
    return ACB_OK;
}

// vae_ggml_decode_tiled (vae.h:467-565): windows of chunk_size latent frames with `overlap`
// frames of context on each side, each decoded on its own and trimmed to its core, cores
// concatenated; audio_out holds channel 0 for T_audio samples, then channel 1.
extern "C" acb_status acb_vae_decode_tiled(acb_vae * m, const float * latent, int T_latent, float * audio_out,
                                           int max_T_audio, int chunk_size, int overlap, acb_cancel_fn cancel,
                                           void * cancel_data, int * out_T_audio) {
    if (!m || !latent || !audio_out || T_latent <= 0 || chunk_size <= 0 || overlap < 0) {
        return ACB_ERR_INVALID_ARG;
    }
    while (chunk_size - 2 * overlap <= 0 && overlap > 0) {
        overlap /= 2;
    }
    if (T_latent <= chunk_size) {
        return acb_vae_decode(m, latent, T_latent, audio_out, max_T_audio, out_T_audio);
    }
    if (cudaSetDevice(m->device) != cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    const int stride = chunk_size - 2 * overlap;
    const int steps  = (T_latent + stride - 1) / stride;
    const int wmax   = std::min(T_latent, chunk_size + 2 * overlap);
    ACB_TRY(m->reserve(wmax));
    if (m->lat.bytes < (size_t) wmax * m->latent * 4) {
        ACB_TRY(m->lat.alloc((size_t) wmax * m->latent * 4, false));
    }
    if (m->out.bytes < (size_t) wmax * m->up * 2 * 4) {
        ACB_TRY(m->out.alloc((size_t) wmax * m->up * 2 * 4, false));
    }
    cudaMemsetAsync(m->err.p, 0, 4, m->st);
    std::vector<float> ch1;  // channel 1 of the cores, placed after channel 0 at the end
    float              upf = 0.0f;
    int                pos = 0;
    for (int i = 0; i < steps; i++) {
        if (cancel && cancel(cancel_data)) {
            set_last_error("cancelled at tile " + std::to_string(i));
            return ACB_ERR_CANCELLED;
        }
        const int core0 = i * stride, core1 = std::min(core0 + stride, T_latent);
        const int w0 = std::max(core0 - overlap, 0), w1 = std::min(core1 + overlap, T_latent);
        const int wl = w1 - w0;
        if (cudaMemcpyAsync(m->lat.p, latent + (size_t) w0 * m->latent, (size_t) wl * m->latent * 4,
                            cudaMemcpyHostToDevice, m->st) != cudaSuccess) {
            return ACB_ERR_CUDA;
        }
        ACB_TRY(m->run(m->lat.as<float>(), wl, m->out.as<float>()));
        const int tile_T = wl * m->up;
        if (i == 0) {
            upf = (float) tile_T / (float) wl;
        }
        const int trim0 = (int) roundf((float) (core0 - w0) * upf);
        const int trim1 = (int) roundf((float) (w1 - core1) * upf);
        const int end   = trim1 > 0 ? tile_T - trim1 : tile_T;
        const int len   = end - trim0;
        if (len <= 0) {
            continue;
        }
        if (pos + len > max_T_audio) {
            set_last_error("tiled output exceeds max_T_audio");
            return ACB_ERR_OUT_OF_RANGE;
        }
        ch1.resize((size_t) (pos + len));
        if (cudaMemcpyAsync(audio_out + pos, m->out.as<float>() + trim0, (size_t) len * 4, cudaMemcpyDeviceToHost,
                            m->st) != cudaSuccess ||
            cudaMemcpyAsync(ch1.data() + pos, m->out.as<float>() + tile_T + trim0, (size_t) len * 4,
                            cudaMemcpyDeviceToHost, m->st) != cudaSuccess ||
            cudaStreamSynchronize(m->st) != cudaSuccess) {
            return ACB_ERR_CUDA;
        }
        pos += len;
    }
    int flag = 0;
    cudaMemcpy(&flag, m->err.p, 4, cudaMemcpyDeviceToHost);
    if (flag) {
        set_last_error("device error flag " + std::to_string(flag));
        return ACB_ERR_DEVICE;
    }
    memcpy(audio_out + pos, ch1.data(), (size_t) pos * 4);
    if (out_T_audio) {
        *out_T_audio = pos;
    }
    return ACB_OK;
}

extern "C" void acb_vae_free(acb_vae * m) {
    delete m;
}
