// cond_enc.cpp -- the condition encoder (src/cond-enc.h) and the FSQ detokenizer / tokenizer
// (src/fsq-detok.h, src/fsq-tok.h) on libacb kernels.
//
// All three are Qwen3 encoder stacks (enc_stack.h) fed by projections:
//   condition   lyric  [S_l][1024] -> Linear+bias -> 8 layers (window 128 on even layers) -> norm
//               timbre [S_r][64]   -> Linear+bias (-> CLS prepended) -> 4 layers -> norm -> row 0
//               text   [S_t][1024] -> Linear
//               packed into [lyric | timbre row | text] rows of 2048 (cond-enc.h:350-374)
//   detok       codes [G] -> FSQ levels -> project_out (K = 6) + bias -> embed + bias
//               -> + special_tokens [5] -> 2 layers -> norm -> proj_out + bias   [5G][64]
//   tok         latents [5G][64] -> proj + bias -> embed + bias -> CLS prepended to each group
//               -> 2 layers -> norm -> CLS row -> project_in + bias -> FSQ index  [G]
// The reference runs the FSQ models one 5-frame group per graph; here every group of a call is one
// batch (B = G sequences of 5 or 6 rows, attention within a group), so each linear is a single
// tensor-core GEMM over all groups' rows.
//
// Stack sizes are read from the tensor shapes (the reference's constants, cond-enc.h:18-44,
// fsq-detok.h:32-44, fsq-tok.h:71-80, are what the shipped GGUFs hold).
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <memory>
#include <string>
#include <utility>
#include <vector>

#include "../../include/acb_models.h"
#include "dense.h"
#include "enc_stack.h"
#include "gguf.h"
#include "host_common.h"
#include "weights.h"

using namespace acb;

namespace {

constexpr int kFsqGroup = 5;  // pool window: 25 Hz frames per 5 Hz code (fsq-tok.h:136)
constexpr int kFsqDims  = 6;

// One ggml_mul_mat(W, x) (+ bias) per linear on the tensor cores (dense.h), every W a resident
// 16-bit copy, sharing one activation / split-K scratch.
struct Linears {
    DevBuf                     w16, xq, ws, err;
    std::vector<DenseLinear *> all;
    int                        cap  = 0;
    int64_t                    kmax = 0;

    acb_status build(const std::vector<std::pair<DenseLinear *, DevTensor *>> & items, cudaStream_t st) {
        size_t  total = 0;
        int64_t maxn = 0, maxnk = 0;
        for (const auto & it : items) {
            total += (DenseLinear::elems({ it.second }) * 2 + 255) & ~size_t(255);
            maxn  = std::max(maxn, it.second->N);
            maxnk = std::max(maxnk, it.second->N * it.second->K);
            kmax  = std::max(kmax, it.second->K);
        }
        DevBuf ids, tmp;
        if (w16.alloc(total, false) != ACB_OK || ids.alloc((size_t) maxn * 4, false) != ACB_OK ||
            tmp.alloc((size_t) maxnk * 4, false) != ACB_OK || err.alloc(4) != ACB_OK) {
            set_last_error("linear weight allocation failed");
            return ACB_ERR_OOM;
        }
        std::vector<int32_t> idv((size_t) maxn);
        for (int64_t r = 0; r < maxn; r++) {
            idv[(size_t) r] = (int32_t) r;
        }
        if (cudaMemcpy(ids.p, idv.data(), idv.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess) {
            return ACB_ERR_CUDA;
        }
        uint8_t * p = w16.as<uint8_t>();
        for (const auto & it : items) {
            ACB_TRY(dense_build(*it.first, { it.second }, reinterpret_cast<uint16_t *>(p), ids.as<int32_t>(),
                                tmp.as<float>(), st));
            p += (DenseLinear::elems({ it.second }) * 2 + 255) & ~size_t(255);
            if (cudaStreamSynchronize(st) != cudaSuccess) {  // tmp is reused by the next matrix
                return ACB_ERR_CUDA;
            }
            all.push_back(it.first);
        }
        return ACB_OK;
    }

    acb_status reserve(int M) {
        if (M <= cap) {
            return ACB_OK;
        }
        const int n   = std::max(M, 256);
        size_t    wsb = 0;
        for (int m = 128; m < n + 128; m += 128) {
            for (const DenseLinear * L : all) {
                for (int64_t km : { (int64_t) 1, (int64_t) 3 }) {
                    wsb = std::max(wsb, acb_gemm_workspace_bytes(std::min(m, n), L->N, km * L->K));
                }
            }
        }
        if (xq.alloc((size_t) n * 3 * kmax * 2, false) != ACB_OK || ws.alloc(wsb, true) != ACB_OK) {  // zeroed split-K tickets
            cap = 0;
            set_last_error("linear scratch allocation failed");
            return ACB_ERR_OOM;
        }
        cap = n;
        return ACB_OK;
    }

    // y[M][N] (rows ldy apart) = x[M][K] (rows xs apart) . W^T + bias
    acb_status run(const DenseLinear & L, bool exact, const float * x, int64_t xs, int M, float * y, int64_t ldy,
                   const float * bias, cudaStream_t st) {
        ACB_TRY(reserve(M));
        const DenseScratch s{ xq.p, ws.p, ws.bytes, err.as<int>() };
        return dense_forward(L, exact, x, xs, 0, M, y, ACB_TYPE_F32, ldy, bias, nullptr, 0, nullptr, 0, 0, s, st);
    }
};

// f32 device copy of a small tensor (biases, learned tokens) whatever its GGUF type: F32 / BF16 /
// F16 through load_f32 on the host, quantised rows dequantised on the device (ggml_cast to F32).
struct F32Tensor {
    DevTensor * t = nullptr;
    DevBuf      own;
    int64_t     K = 0, N = 0;

    const float * data() const { return own.p ? own.as<float>() : (t ? (const float *) t->data : nullptr); }

    acb_status finish(cudaStream_t st) {  // after the arena upload
        if (!t) {
            return ACB_ERR_FORMAT;
        }
        K = t->K;
        N = t->N;
        if (t->type == ACB_TYPE_F32) {
            return ACB_OK;
        }
        DevBuf ids;
        ACB_TRY(own.alloc((size_t) K * N * 4, false));
        ACB_TRY(ids.alloc((size_t) N * 4, false));
        std::vector<int32_t> idv((size_t) N);
        for (int64_t r = 0; r < N; r++) {
            idv[(size_t) r] = (int32_t) r;
        }
        if (cudaMemcpy(ids.p, idv.data(), idv.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess) {
            return ACB_ERR_CUDA;
        }
        ACB_TRY(acb_get_rows(t->data, t->type, N, K, ids.as<int32_t>(), N, own.p, ACB_TYPE_F32, K, nullptr,
                             (acb_stream_t) st));
        return cudaStreamSynchronize(st) == cudaSuccess ? ACB_OK : ACB_ERR_CUDA;
    }
};

// Qwen3Config of the stack under `prefix` from its tensor shapes (head_dim from q_norm).
bool stack_config(const GGUFFile & gf, const std::string & prefix, acb_qwen3_config & c) {
    c              = acb_qwen3_config{};
    c.rope_theta   = 1000000.0f;
    c.rms_norm_eps = 1e-6f;
    c.is_causal    = 0;
    while (gf.find(prefix + "layers." + std::to_string(c.n_layers) + ".input_layernorm.weight")) {
        c.n_layers++;
    }
    const GGUFTensor * norm = gf.find(prefix + "norm.weight");
    const GGUFTensor * qn   = gf.find(prefix + "layers.0.self_attn.q_norm.weight");
    const GGUFTensor * q    = gf.find(prefix + "layers.0.self_attn.q_proj.weight");
    const GGUFTensor * k    = gf.find(prefix + "layers.0.self_attn.k_proj.weight");
    const GGUFTensor * g    = gf.find(prefix + "layers.0.mlp.gate_proj.weight");
    if (c.n_layers == 0 || !norm || !qn || !q || !k || !g || qn->ne[0] <= 0) {
        return false;
    }
    c.hidden_size       = (int) norm->ne[0];
    c.head_dim          = (int) qn->ne[0];
    c.n_heads           = (int) (q->ne[1] / c.head_dim);
    c.n_kv_heads        = (int) (k->ne[1] / c.head_dim);
    c.intermediate_size = (int) g->ne[1];
    return true;
}

struct StackDeleter {
    void operator()(acb_qwen3_enc * m) const { acb_qwen3_free(m); }
};
using StackPtr = std::unique_ptr<acb_qwen3_enc, StackDeleter>;

acb_status open_gguf(GGUFFile & gf, const char * path) {
    if (!gf.open(path)) {
        set_last_error(gf.error());
        return gf.error().rfind("cannot open", 0) == 0 ? ACB_ERR_IO : ACB_ERR_FORMAT;
    }
    return ACB_OK;
}

acb_status load_stack(GGUFFile & gf, const std::string & prefix, int window, int device, StackPtr & out) {
    acb_qwen3_config c;
    if (!stack_config(gf, prefix, c)) {
        set_last_error("encoder stack '" + prefix + "' missing or misshapen");
        return ACB_ERR_FORMAT;
    }
    acb_qwen3_enc * m = nullptr;
    ACB_TRY(enc_stack_load(gf, prefix, c, window, false, device, &m));
    out.reset(m);
    return ACB_OK;
}

// a device buffer that only grows
acb_status grow(DevBuf & b, size_t bytes) {
    if (b.bytes >= bytes) {
        return ACB_OK;
    }
    if (b.alloc(bytes, false) != ACB_OK) {
        set_last_error("scratch allocation failed");
        return ACB_ERR_OOM;
    }
    return ACB_OK;
}

// read and clear the device error flags of a call; ACB_ERR_DEVICE when one is set
acb_status check_flags(cudaStream_t st, std::initializer_list<int *> flags) {
    int any = 0;
    for (int * f : flags) {
        int v = 0;
        if (f && (cudaMemcpyAsync(&v, f, 4, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
                  cudaStreamSynchronize(st) != cudaSuccess || cudaMemsetAsync(f, 0, 4, st) != cudaSuccess)) {
            return ACB_ERR_CUDA;
        }
        any |= v;
    }
    if (cudaStreamSynchronize(st) != cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    if (any) {
        set_last_error("device error flag " + std::to_string(any));
        return ACB_ERR_DEVICE;
    }
    return ACB_OK;
}

}  // namespace

// ---- condition encoder -------------------------------------------------------------------------

struct acb_cond {
    int             device = 0;
    cudaStream_t    st     = nullptr;
    bool            exact  = true;
    acb_cond_config cfg{};
    StackPtr        lyric, timbre;
    WeightArena     arena;
    DenseLinear     lyric_in, timbre_in, text_proj;
    F32Tensor       lyric_b, timbre_b, cls, null_emb;
    Linears         lin;
    DevBuf          tbuf, tout, in_text, in_lyric, in_timbre, out;

    ~acb_cond() {
        cudaSetDevice(device);
        lyric.reset();
        timbre.reset();
        if (st) {
            cudaStreamDestroy(st);
        }
    }

    acb_status forward(const float * text, int S_text, const float * lyr, int S_lyric, const float * tim, int S_ref,
                       float * enc, cudaStream_t s);
};

acb_status acb_cond::forward(const float * text, int S_text, const float * lyr, int S_lyric, const float * tim,
                             int S_ref, float * enc, cudaStream_t s) {
    const int  H          = cfg.hidden_size;
    const bool has_timbre = tim && S_ref > 0;
    // lyric: Linear + bias into the stack's input, 8 layers + norm straight into rows [0, S_lyric)
    float * h = enc_stack_input(lyric.get(), 1, S_lyric, s);
    if (!h) {
        return ACB_ERR_OOM;
    }
    ACB_TRY(lin.run(lyric_in, exact, lyr, cfg.lyric_dim, S_lyric, h, H, lyric_b.data(), s));
    ACB_TRY(enc_stack_run(lyric.get(), 1, S_lyric, enc, H, s));
    // timbre: Linear + bias (after the CLS row for XL models), 4 layers + norm, first row
    if (has_timbre) {
        const int S_t = S_ref + (cfg.timbre_cls ? 1 : 0);
        float *   th  = enc_stack_input(timbre.get(), 1, S_t, s);
        if (!th) {
            return ACB_ERR_OOM;
        }
        if (cfg.timbre_cls) {
            ACB_TRY(grow(tbuf, (size_t) S_ref * H * 4));
            ACB_TRY(lin.run(timbre_in, exact, tim, cfg.timbre_dim, S_ref, tbuf.as<float>(), H, timbre_b.data(), s));
            ACB_TRY(acb_rows_prepend(cls.data(), tbuf.as<float>(), H, 1, S_ref, H, th, H, (acb_stream_t) s));
        } else {
            ACB_TRY(lin.run(timbre_in, exact, tim, cfg.timbre_dim, S_ref, th, H, timbre_b.data(), s));
        }
        ACB_TRY(grow(tout, (size_t) S_t * H * 4));
        ACB_TRY(enc_stack_run(timbre.get(), 1, S_t, tout.as<float>(), H, s));
        if (cudaMemcpyAsync(enc + (size_t) S_lyric * H, tout.p, (size_t) H * 4, cudaMemcpyDeviceToDevice, s) !=
            cudaSuccess) {
            return ACB_ERR_CUDA;
        }
    }
    // text projection (no bias) into the last S_text rows
    float * tp = enc + (size_t) (S_lyric + (has_timbre ? 1 : 0)) * H;
    return lin.run(text_proj, exact, text, cfg.text_dim, S_text, tp, H, nullptr, s);
}

extern "C" acb_status acb_cond_load(const char * gguf_path, int device, acb_cond ** out) {
    if (!gguf_path || !out) {
        return ACB_ERR_INVALID_ARG;
    }
    *out = nullptr;
    if (cudaSetDevice(device) != cudaSuccess) {
        set_last_error("cannot select CUDA device");
        return ACB_ERR_CUDA;
    }
    GGUFFile gf;
    ACB_TRY(open_gguf(gf, gguf_path));
    std::unique_ptr<acb_cond> m(new acb_cond());
    m->device = device;
    if (cudaStreamCreateWithFlags(&m->st, cudaStreamNonBlocking) != cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    const int W = 128;  // sliding window of the even layers (cond-enc.h:298, 325)
    ACB_TRY(load_stack(gf, "encoder.lyric_encoder.", W, device, m->lyric));
    ACB_TRY(load_stack(gf, "encoder.timbre_encoder.", W, device, m->timbre));
    acb_cond_config & c = m->cfg;
    acb_qwen3_config  lc, tc;
    acb_qwen3_get_config(m->lyric.get(), &lc);
    acb_qwen3_get_config(m->timbre.get(), &tc);
    c.hidden_size   = lc.hidden_size;
    c.lyric_layers  = lc.n_layers;
    c.timbre_layers = tc.n_layers;
    c.window        = W;
    c.timbre_cls    = gf.get_u32("acestep.encoder_hidden_size") > 0 ? 1 : 0;  // cond-enc.h:104-106

    WeightArena stage;
    DevTensor * lw = stage.load(gf, "encoder.lyric_encoder.embed_tokens.weight");
    DevTensor * tw = stage.load(gf, "encoder.timbre_encoder.embed_tokens.weight");
    DevTensor * pw = stage.load(gf, "encoder.text_projector.weight");
    m->lyric_b.t   = m->arena.load_f32(gf, "encoder.lyric_encoder.embed_tokens.bias");
    m->timbre_b.t  = m->arena.load_f32(gf, "encoder.timbre_encoder.embed_tokens.bias");
    m->null_emb.t  = m->arena.load_f32(gf, "null_condition_emb");
    if (c.timbre_cls) {
        m->cls.t = m->arena.load_f32(gf, "encoder.timbre_encoder.special_token");
    }
    if (!lw || !tw || !pw || !m->lyric_b.t || !m->timbre_b.t || !m->null_emb.t || (c.timbre_cls && !m->cls.t)) {
        set_last_error(!stage.error.empty() ? stage.error : m->arena.error);
        return ACB_ERR_FORMAT;
    }
    const int H  = c.hidden_size;
    c.lyric_dim  = (int) lw->K;
    c.timbre_dim = (int) tw->K;
    c.text_dim   = (int) pw->K;
    if (lw->N != H || tw->N != H || pw->N != H || tc.hidden_size != H || m->lyric_b.t->K * m->lyric_b.t->N != H ||
        m->timbre_b.t->K * m->timbre_b.t->N != H || m->null_emb.t->K * m->null_emb.t->N != H ||
        (c.timbre_cls && m->cls.t->K * m->cls.t->N != H)) {
        set_last_error("condition encoder tensor shapes do not agree");
        return ACB_ERR_FORMAT;
    }
    ACB_TRY(m->arena.upload(m->st));
    ACB_TRY(stage.upload(m->st));
    ACB_TRY(m->lyric_b.finish(m->st));
    ACB_TRY(m->timbre_b.finish(m->st));
    ACB_TRY(m->null_emb.finish(m->st));
    if (c.timbre_cls) {
        ACB_TRY(m->cls.finish(m->st));
    }
    ACB_TRY(m->lin.build({ { &m->lyric_in, lw }, { &m->timbre_in, tw }, { &m->text_proj, pw } }, m->st));
    if (cudaStreamSynchronize(m->st) != cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    *out = m.release();
    return ACB_OK;
}

extern "C" acb_status acb_cond_get_config(const acb_cond * m, acb_cond_config * cfg) {
    if (!m || !cfg) {
        return ACB_ERR_INVALID_ARG;
    }
    *cfg = m->cfg;
    return ACB_OK;
}

extern "C" acb_status acb_cond_set_exact(acb_cond * m, int exact) {
    if (!m) {
        return ACB_ERR_INVALID_ARG;
    }
    m->exact = exact != 0;
    acb_qwen3_set_exact(m->lyric.get(), exact);
    acb_qwen3_set_exact(m->timbre.get(), exact);
    return ACB_OK;
}

extern "C" acb_status acb_cond_forward_device(acb_cond * m, const float * d_text_hidden, int S_text,
                                              const float * d_lyric_embed, int S_lyric, const float * d_timbre_feats,
                                              int S_ref, float * d_enc_hidden, int * out_enc_S, acb_stream_t stream) {
    if (!m || !d_text_hidden || !d_lyric_embed || !d_enc_hidden || S_text <= 0 || S_lyric <= 0 || S_ref < 0) {
        return ACB_ERR_INVALID_ARG;
    }
    if (cudaSetDevice(m->device) != cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    const bool has_timbre = d_timbre_feats && S_ref > 0;
    ACB_TRY(m->forward(d_text_hidden, S_text, d_lyric_embed, S_lyric, d_timbre_feats, S_ref, d_enc_hidden,
                       (cudaStream_t) stream));
    if (out_enc_S) {
        *out_enc_S = S_lyric + (has_timbre ? 1 : 0) + S_text;
    }
    return ACB_OK;
}

extern "C" acb_status acb_cond_forward(acb_cond * m, const float * text_hidden, int S_text, const float * lyric_embed,
                                       int S_lyric, const float * timbre_feats, int S_ref, float * enc_hidden,
                                       int * out_enc_S) {
    if (!m || !text_hidden || !lyric_embed || !enc_hidden || S_text <= 0 || S_lyric <= 0 || S_ref < 0) {
        return ACB_ERR_INVALID_ARG;
    }
    if (cudaSetDevice(m->device) != cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    const acb_cond_config & c          = m->cfg;
    const bool              has_timbre = timbre_feats && S_ref > 0;
    const int               S_total    = S_lyric + (has_timbre ? 1 : 0) + S_text;
    cudaStream_t            s          = m->st;
    ACB_TRY(grow(m->in_text, (size_t) S_text * c.text_dim * 4));
    ACB_TRY(grow(m->in_lyric, (size_t) S_lyric * c.lyric_dim * 4));
    ACB_TRY(grow(m->out, (size_t) S_total * c.hidden_size * 4));
    if (has_timbre) {
        ACB_TRY(grow(m->in_timbre, (size_t) S_ref * c.timbre_dim * 4));
    }
    if (cudaMemcpyAsync(m->in_text.p, text_hidden, (size_t) S_text * c.text_dim * 4, cudaMemcpyHostToDevice, s) !=
            cudaSuccess ||
        cudaMemcpyAsync(m->in_lyric.p, lyric_embed, (size_t) S_lyric * c.lyric_dim * 4, cudaMemcpyHostToDevice, s) !=
            cudaSuccess ||
        (has_timbre && cudaMemcpyAsync(m->in_timbre.p, timbre_feats, (size_t) S_ref * c.timbre_dim * 4,
                                       cudaMemcpyHostToDevice, s) != cudaSuccess)) {
        return ACB_ERR_CUDA;
    }
    ACB_TRY(m->forward(m->in_text.as<float>(), S_text, m->in_lyric.as<float>(), S_lyric,
                       has_timbre ? m->in_timbre.as<float>() : nullptr, S_ref, m->out.as<float>(), s));
    if (cudaMemcpyAsync(enc_hidden, m->out.p, (size_t) S_total * c.hidden_size * 4, cudaMemcpyDeviceToHost, s) !=
        cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    ACB_TRY(check_flags(s, { m->lin.err.as<int>(), enc_stack_err(m->lyric.get()), enc_stack_err(m->timbre.get()) }));
    if (out_enc_S) {
        *out_enc_S = S_total;
    }
    return ACB_OK;
}

extern "C" acb_status acb_cond_null_embedding(acb_cond * m, float * out) {
    if (!m || !out) {
        return ACB_ERR_INVALID_ARG;
    }
    if (cudaSetDevice(m->device) != cudaSuccess ||
        cudaMemcpy(out, m->null_emb.data(), (size_t) m->cfg.hidden_size * 4, cudaMemcpyDeviceToHost) != cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    return ACB_OK;
}

extern "C" void acb_cond_free(acb_cond * m) {
    delete m;
}

// ---- FSQ host helpers --------------------------------------------------------------------------

static const int kFsqLevels[kFsqDims] = { 8, 8, 8, 5, 5, 5 };  // FSQ_LEVELS, fsq-detok.h:15

extern "C" void acb_fsq_decode_index(int index, float * out6) {
    int stride = 1;
    for (int d = 0; d < kFsqDims; d++) {
        const int   L      = kFsqLevels[d];
        const float half_L = (float) (L - 1) / 2.0f;
        out6[d]            = (float) ((index / stride) % L) / half_L - 1.0f;
        stride *= L;
    }
}

extern "C" int acb_fsq_encode_index(const float * raw6) {
    int index = 0, mult = 1;
    for (int d = 0; d < kFsqDims; d++) {
        const int   L    = kFsqLevels[d];
        const float t    = tanhf(raw6[d]);
        int         code = (int) floorf((float) (L - 1) * (t + 1.0f) / 2.0f + 0.5f);
        code             = code < 0 ? 0 : (code >= L ? L - 1 : code);
        index += code * mult;
        mult *= L;
    }
    return index;
}

// ---- FSQ detokenizer ---------------------------------------------------------------------------

struct acb_detok {
    int          device = 0;
    cudaStream_t st     = nullptr;
    bool         exact  = true;
    int          H = 0, C = 0;  // stack width, output channels (64)
    StackPtr     stack;
    WeightArena  arena;
    DevTensor *  po_w = nullptr;  // project_out [2048][6], BF16 / F16 / F32
    F32Tensor    po_b, emb_b, out_b, special;
    DenseLinear  embed, proj_out;
    Linears      lin;
    DevBuf       q, e, y, codes, out, err;

    ~acb_detok() {
        cudaSetDevice(device);
        stack.reset();
        if (st) {
            cudaStreamDestroy(st);
        }
    }

    acb_status decode(const int32_t * d_codes, int G, float * d_out, cudaStream_t s) {
        float * h = enc_stack_input(stack.get(), G, kFsqGroup, s);
        if (!h) {
            return ACB_ERR_OOM;
        }
        ACB_TRY(grow(q, (size_t) G * H * 4));
        ACB_TRY(grow(e, (size_t) G * H * 4));
        ACB_TRY(grow(y, (size_t) G * kFsqGroup * H * 4));
        ACB_TRY(acb_fsq_project_out(d_codes, G, po_w->data, po_w->type, H, po_b.data(), q.as<float>(), H,
                                    err.as<int>(), (acb_stream_t) s));
        ACB_TRY(lin.run(embed, exact, q.as<float>(), H, G, e.as<float>(), H, emb_b.data(), s));
        ACB_TRY(acb_rows_repeat_add(e.as<float>(), H, special.data(), H, G, kFsqGroup, H, h, H, (acb_stream_t) s));
        ACB_TRY(enc_stack_run(stack.get(), G, kFsqGroup, y.as<float>(), H, s));
        return lin.run(proj_out, exact, y.as<float>(), H, G * kFsqGroup, d_out, C, out_b.data(), s);
    }
};

extern "C" acb_status acb_detok_load(const char * gguf_path, int device, acb_detok ** out) {
    if (!gguf_path || !out) {
        return ACB_ERR_INVALID_ARG;
    }
    *out = nullptr;
    if (cudaSetDevice(device) != cudaSuccess) {
        set_last_error("cannot select CUDA device");
        return ACB_ERR_CUDA;
    }
    GGUFFile gf;
    ACB_TRY(open_gguf(gf, gguf_path));
    std::unique_ptr<acb_detok> m(new acb_detok());
    m->device = device;
    if (cudaStreamCreateWithFlags(&m->st, cudaStreamNonBlocking) != cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    ACB_TRY(load_stack(gf, "detokenizer.", 0, device, m->stack));
    acb_qwen3_config sc;
    acb_qwen3_get_config(m->stack.get(), &sc);
    m->H = sc.hidden_size;
    WeightArena stage;
    m->po_w       = m->arena.load(gf, "tokenizer.quantizer.project_out.weight");
    m->po_b.t     = m->arena.load_f32(gf, "tokenizer.quantizer.project_out.bias");
    DevTensor * ew = stage.load(gf, "detokenizer.embed_tokens.weight");
    m->emb_b.t    = m->arena.load_f32(gf, "detokenizer.embed_tokens.bias");
    m->special.t  = m->arena.load_f32(gf, "detokenizer.special_tokens");
    DevTensor * ow = stage.load(gf, "detokenizer.proj_out.weight");
    m->out_b.t    = m->arena.load_f32(gf, "detokenizer.proj_out.bias");
    if (!m->po_w || !m->po_b.t || !ew || !m->emb_b.t || !m->special.t || !ow || !m->out_b.t) {
        set_last_error(!stage.error.empty() ? stage.error : m->arena.error);
        return ACB_ERR_FORMAT;
    }
    const int H = m->H;
    m->C        = (int) ow->N;
    if (m->po_w->K != kFsqDims || m->po_w->N != H || ew->K != H || ew->N != H || ow->K != H ||
        m->special.t->K != H || m->special.t->N != kFsqGroup || m->out_b.t->K * m->out_b.t->N != m->C ||
        m->po_b.t->K * m->po_b.t->N != H || m->emb_b.t->K * m->emb_b.t->N != H) {
        set_last_error("detokenizer tensor shapes do not agree");
        return ACB_ERR_FORMAT;
    }
    if (m->po_w->type != ACB_TYPE_BF16 && m->po_w->type != ACB_TYPE_F16 && m->po_w->type != ACB_TYPE_F32) {
        set_last_error("project_out weight type not supported");
        return ACB_ERR_UNSUPPORTED;
    }
    ACB_TRY(m->arena.upload(m->st));
    ACB_TRY(stage.upload(m->st));
    for (F32Tensor * t : { &m->po_b, &m->emb_b, &m->special, &m->out_b }) {
        ACB_TRY(t->finish(m->st));
    }
    ACB_TRY(m->lin.build({ { &m->embed, ew }, { &m->proj_out, ow } }, m->st));
    ACB_TRY(m->err.alloc(4));
    if (cudaStreamSynchronize(m->st) != cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    *out = m.release();
    return ACB_OK;
}

extern "C" acb_status acb_detok_set_exact(acb_detok * m, int exact) {
    if (!m) {
        return ACB_ERR_INVALID_ARG;
    }
    m->exact = exact != 0;
    return acb_qwen3_set_exact(m->stack.get(), exact);
}

extern "C" acb_status acb_detok_decode_device(acb_detok * m, const int32_t * d_codes, int T_5Hz, float * d_out,
                                              acb_stream_t stream) {
    if (!m || !d_codes || !d_out || T_5Hz <= 0) {
        return ACB_ERR_INVALID_ARG;
    }
    if (cudaSetDevice(m->device) != cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    return m->decode(d_codes, T_5Hz, d_out, (cudaStream_t) stream);
}

extern "C" acb_status acb_detok_decode(acb_detok * m, const int * codes, int T_5Hz, float * context_out) {
    if (!m || !codes || !context_out || T_5Hz <= 0) {
        return ACB_ERR_INVALID_ARG;
    }
    for (int g = 0; g < T_5Hz; g++) {
        if (codes[g] < 0) {
            set_last_error("negative FSQ code");
            return ACB_ERR_OUT_OF_RANGE;
        }
    }
    if (cudaSetDevice(m->device) != cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    cudaStream_t s  = m->st;
    const size_t ob = (size_t) T_5Hz * kFsqGroup * m->C * 4;
    ACB_TRY(grow(m->codes, (size_t) T_5Hz * 4));
    ACB_TRY(grow(m->out, ob));
    if (cudaMemcpyAsync(m->codes.p, codes, (size_t) T_5Hz * 4, cudaMemcpyHostToDevice, s) != cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    ACB_TRY(m->decode(m->codes.as<int32_t>(), T_5Hz, m->out.as<float>(), s));
    if (cudaMemcpyAsync(context_out, m->out.p, ob, cudaMemcpyDeviceToHost, s) != cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    return check_flags(s, { m->err.as<int>(), m->lin.err.as<int>(), enc_stack_err(m->stack.get()) });
}

extern "C" void acb_detok_free(acb_detok * m) {
    delete m;
}

// ---- FSQ tokenizer -----------------------------------------------------------------------------

struct acb_tok {
    int          device = 0;
    cudaStream_t st     = nullptr;
    bool         exact  = true;
    int          H = 0, C = 0;  // stack width, latent channels (64)
    StackPtr     stack;
    WeightArena  arena;
    F32Tensor    proj_b, emb_b, cls, in_b;
    DenseLinear  proj, embed, project_in;
    Linears      lin;
    DevBuf       p, e, y, raw, lat, codes;

    ~acb_tok() {
        cudaSetDevice(device);
        stack.reset();
        if (st) {
            cudaStreamDestroy(st);
        }
    }

    acb_status encode(const float * d_lat, int G, int32_t * d_codes, cudaStream_t s) {
        const int S = kFsqGroup + 1;  // CLS + 5 frames
        float *   h = enc_stack_input(stack.get(), G, S, s);
        if (!h) {
            return ACB_ERR_OOM;
        }
        const int R = G * kFsqGroup;
        ACB_TRY(grow(p, (size_t) R * H * 4));
        ACB_TRY(grow(e, (size_t) R * H * 4));
        ACB_TRY(grow(y, (size_t) G * S * H * 4));
        ACB_TRY(grow(raw, (size_t) G * 8 * 4));
        ACB_TRY(lin.run(proj, exact, d_lat, C, R, p.as<float>(), H, proj_b.data(), s));
        ACB_TRY(lin.run(embed, exact, p.as<float>(), H, R, e.as<float>(), H, emb_b.data(), s));
        ACB_TRY(acb_rows_prepend(cls.data(), e.as<float>(), H, G, kFsqGroup, H, h, H, (acb_stream_t) s));
        ACB_TRY(enc_stack_run(stack.get(), G, S, y.as<float>(), H, s));
        // project_in over the CLS rows only (every S-th row), bias + tanh + levels in one kernel
        ACB_TRY(lin.run(project_in, exact, y.as<float>(), (int64_t) S * H, G, raw.as<float>(), 8, nullptr, s));
        return acb_fsq_quantize(raw.as<float>(), 8, in_b.data(), G, d_codes, (acb_stream_t) s);
    }
};

extern "C" acb_status acb_tok_load(const char * gguf_path, int device, acb_tok ** out) {
    if (!gguf_path || !out) {
        return ACB_ERR_INVALID_ARG;
    }
    *out = nullptr;
    if (cudaSetDevice(device) != cudaSuccess) {
        set_last_error("cannot select CUDA device");
        return ACB_ERR_CUDA;
    }
    GGUFFile gf;
    ACB_TRY(open_gguf(gf, gguf_path));
    std::unique_ptr<acb_tok> m(new acb_tok());
    m->device = device;
    if (cudaStreamCreateWithFlags(&m->st, cudaStreamNonBlocking) != cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    ACB_TRY(load_stack(gf, "tokenizer.attention_pooler.", 0, device, m->stack));
    acb_qwen3_config sc;
    acb_qwen3_get_config(m->stack.get(), &sc);
    m->H = sc.hidden_size;
    WeightArena stage;
    DevTensor * pw = stage.load(gf, "tokenizer.audio_acoustic_proj.weight");
    m->proj_b.t    = m->arena.load_f32(gf, "tokenizer.audio_acoustic_proj.bias");
    DevTensor * ew = stage.load(gf, "tokenizer.attention_pooler.embed_tokens.weight");
    m->emb_b.t     = m->arena.load_f32(gf, "tokenizer.attention_pooler.embed_tokens.bias");
    m->cls.t       = m->arena.load_f32(gf, "tokenizer.attention_pooler.special_token");
    DevTensor * iw = stage.load(gf, "tokenizer.quantizer.project_in.weight");
    m->in_b.t      = m->arena.load_f32(gf, "tokenizer.quantizer.project_in.bias");
    if (!pw || !m->proj_b.t || !ew || !m->emb_b.t || !m->cls.t || !iw || !m->in_b.t) {
        set_last_error(!stage.error.empty() ? stage.error : m->arena.error);
        return ACB_ERR_FORMAT;
    }
    const int H = m->H;
    m->C        = (int) pw->K;
    if (pw->N != H || ew->K != H || ew->N != H || iw->K != H || iw->N != kFsqDims ||
        m->cls.t->K * m->cls.t->N != H || m->proj_b.t->K * m->proj_b.t->N != H ||
        m->emb_b.t->K * m->emb_b.t->N != H || m->in_b.t->K * m->in_b.t->N != kFsqDims) {
        set_last_error("tokenizer tensor shapes do not agree");
        return ACB_ERR_FORMAT;
    }
    ACB_TRY(m->arena.upload(m->st));
    ACB_TRY(stage.upload(m->st));
    for (F32Tensor * t : { &m->proj_b, &m->emb_b, &m->cls, &m->in_b }) {
        ACB_TRY(t->finish(m->st));
    }
    ACB_TRY(m->lin.build({ { &m->proj, pw }, { &m->embed, ew }, { &m->project_in, iw } }, m->st));
    if (cudaStreamSynchronize(m->st) != cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    *out = m.release();
    return ACB_OK;
}

extern "C" acb_status acb_tok_set_exact(acb_tok * m, int exact) {
    if (!m) {
        return ACB_ERR_INVALID_ARG;
    }
    m->exact = exact != 0;
    return acb_qwen3_set_exact(m->stack.get(), exact);
}

extern "C" acb_status acb_tok_encode_device(acb_tok * m, const float * d_latents, int T_5Hz, int32_t * d_codes,
                                            acb_stream_t stream) {
    if (!m || !d_latents || !d_codes || T_5Hz <= 0) {
        return ACB_ERR_INVALID_ARG;
    }
    if (cudaSetDevice(m->device) != cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    return m->encode(d_latents, T_5Hz, d_codes, (cudaStream_t) stream);
}

extern "C" acb_status acb_tok_encode(acb_tok * m, const float * latents, int T_25Hz, int * codes_out,
                                     const float * silence_latent, int * out_T_5Hz) {
    if (!m || !latents || !codes_out || T_25Hz <= 0) {
        return ACB_ERR_INVALID_ARG;
    }
    const int pad = (kFsqGroup - T_25Hz % kFsqGroup) % kFsqGroup;  // fsq-tok.h:140-149
    if (pad > 0 && !silence_latent) {
        set_last_error("silence_latent is required to pad the latents to a multiple of 5 frames");
        return ACB_ERR_INVALID_ARG;
    }
    if (cudaSetDevice(m->device) != cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    const int    G  = (T_25Hz + pad) / kFsqGroup;
    const size_t fb = (size_t) m->C * 4;  // bytes per frame
    cudaStream_t s  = m->st;
    ACB_TRY(grow(m->lat, (size_t) G * kFsqGroup * fb));
    ACB_TRY(grow(m->codes, (size_t) G * 4));
    if (cudaMemcpyAsync(m->lat.p, latents, (size_t) T_25Hz * fb, cudaMemcpyHostToDevice, s) != cudaSuccess ||
        (pad > 0 && cudaMemcpyAsync(m->lat.as<uint8_t>() + (size_t) T_25Hz * fb, silence_latent, (size_t) pad * fb,
                                    cudaMemcpyHostToDevice, s) != cudaSuccess)) {
        return ACB_ERR_CUDA;
    }
    ACB_TRY(m->encode(m->lat.as<float>(), G, m->codes.as<int32_t>(), s));
    if (cudaMemcpyAsync(codes_out, m->codes.p, (size_t) G * 4, cudaMemcpyDeviceToHost, s) != cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    ACB_TRY(check_flags(s, { m->lin.err.as<int>(), enc_stack_err(m->stack.get()) }));
    if (out_T_5Hz) {
        *out_T_5Hz = G;
    }
    return ACB_OK;
}

extern "C" void acb_tok_free(acb_tok * m) {
    delete m;
}
