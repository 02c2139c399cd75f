// qwen3_lm.cpp -- the Qwen3 causal LM of acestep.cpp (src/qwen3-lm.h) on libacb kernels.
//
// One decode step for N sequences is a fixed chain per layer:
//   GEMV qkv   (prologue RMSNorm * input_layernorm)                  -> qkv rows
//   qkv_post   (q/k RMSNorm + NeoX RoPE, k/v -> f16 cache)           -> q rows, cache
//   attention  (split-KV scores, f16 probabilities, split partials)  -> partials
//   GEMV o     (prologue: sum of split partials; epilogue: + hidden) -> hidden
//   GEMV gate|up (prologue RMSNorm * post_attention_layernorm)       -> gate|up rows
//   GEMV down  (prologue SwiGLU; epilogue: + hidden)                 -> hidden
// then the head GEMV (prologue RMSNorm * model.norm). Every launch after the first uses
// programmatic dependent launch, and the whole step is captured once per shape as a CUDA
// graph. Prefill runs the same chain with all tokens in one KV set (causal by position).
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "../../include/acb_models.h"
#include "gguf.h"
#include "host_common.h"
#include "weights.h"

using namespace acb;

namespace {

struct LMLayer {
    DevTensor *attn_norm = nullptr, *post_norm = nullptr, *q_norm = nullptr, *k_norm = nullptr;
    DevTensor *qkv = nullptr, *qk = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *o = nullptr;
    DevTensor *gate_up = nullptr, *gate = nullptr, *up = nullptr, *down = nullptr;
};

constexpr int kPrefillChunk = 256;  // tokens per prefill pass
constexpr int kMaxSets      = 32;   // QW3LM_MAX_KV_SETS (qwen3-lm.h:29)

}  // namespace

struct acb_qw3lm {
    acb_qw3lm_config     c{};
    int                  device = 0;
    cudaStream_t         st     = nullptr;
    WeightArena          arena;
    DevTensor *          embed      = nullptr;
    DevTensor *          final_norm = nullptr;
    std::vector<LMLayer> layers;
    DevBuf               head2;
    DevTensor            head2_t;
    DevBuf               head_tiles;  // the LM head (tied embedding) repacked for the tensor-core GEMV
    DevTensor            head_tiles_t;
    int                  head2_off = -1;
    int                  n_sets    = 1;
    std::vector<int>     kv_pos;
    DevBuf               kc, vc, rope;
    size_t               layer_elems = 0;
    int                  cap_tok     = 0;
    int                  max_split   = 1;
    DevBuf hidden, qkv, q, scores, smax, part, att, tickets, gu, logits, ids, pos, err, hist_base, hist, mhist, amax;
    DevBuf samp_work, samp_u, samp_idx;  // device sampling (acb_qw3lm_forward_batch_sample)
    int32_t *                           h_ids = nullptr;
    int32_t *                           h_pos = nullptr;
    std::map<long long, cudaGraphExec_t> graphs;
    // single-sequence decode as one persistent launch (acb_lm_decode_step), when the shape allows
    bool            persist = false;
    DevBuf          pd_layers, pd_scratch;
    acb_decode_step pd{};

    ~acb_qw3lm() {
        cudaSetDevice(device);
        for (auto & kv : graphs) {
            cudaGraphExecDestroy(kv.second);
        }
        if (h_ids) {
            cudaFreeHost(h_ids);
        }
        if (h_pos) {
            cudaFreeHost(h_pos);
        }
        if (st) {
            cudaStreamDestroy(st);
        }
    }

    int qd() const { return c.n_heads * c.head_dim; }
    int kvd() const { return c.n_kv_heads * c.head_dim; }
    int qkvd() const { return qd() + 2 * kvd(); }
    int splits(int n) const { return std::min(acb_attn_decode_splits(n, c.n_kv_heads), max_split); }
};

namespace {

acb_status gemv_rows(acb_qw3lm * m, const DevTensor * W, int64_t row0, int64_t nrows, int M, int pro, const float * x,
                     int64_t xs, const float * nw, int nsplit, float * y, int64_t ys, int epi, const float * res,
                     int64_t rs) {
    const int64_t rb = W->row_bytes();
    for (int c0 = 0; c0 < M; c0 += 8) {
        const int        mc = std::min(8, M - c0);
        const acb_status s  = acb_gemv((const uint8_t *) W->data + row0 * rb, W->type, nrows, W->K, mc, pro,
                                      x + (int64_t) c0 * xs, xs, nw, m->c.rms_norm_eps, nsplit, y + (int64_t) c0 * ys,
                                      ys, epi, res ? res + (int64_t) c0 * rs : nullptr, rs, ACB_FLAG_PDL,
                                      m->err.as<int>(), (acb_stream_t) m->st);
        if (s != ACB_OK) {
            return s;
        }
    }
    return ACB_OK;
}

// Layers for n tokens whose embeddings are in m->hidden and positions in m->pos.
acb_status enqueue_layers(acb_qw3lm * m, int n, int set0, int set_per_tok) {
    const acb_qw3lm_config & c = m->c;
    const int H = c.hidden_size, F = c.intermediate_size, D = c.head_dim;
    const int qd = m->qd(), kvd = m->kvd(), qkvd = m->qkvd();
    float *   hid = m->hidden.as<float>();
    float *   qkv = m->qkv.as<float>();
    for (int l = 0; l < c.n_layers; l++) {
        const LMLayer & L  = m->layers[l];
        const float *   an = (const float *) L.attn_norm->data;
        if (L.qkv) {
            ACB_TRY(gemv_rows(m, L.qkv, 0, qkvd, n, ACB_PRO_RMSNORM, hid, H, an, 0, qkv, qkvd, ACB_EPI_STORE, nullptr, 0));
        } else if (L.qk) {
            ACB_TRY(gemv_rows(m, L.qk, 0, qd + kvd, n, ACB_PRO_RMSNORM, hid, H, an, 0, qkv, qkvd, ACB_EPI_STORE, nullptr, 0));
            ACB_TRY(gemv_rows(m, L.v, 0, kvd, n, ACB_PRO_RMSNORM, hid, H, an, 0, qkv + qd + kvd, qkvd, ACB_EPI_STORE,
                              nullptr, 0));
        } else {
            ACB_TRY(gemv_rows(m, L.q, 0, qd, n, ACB_PRO_RMSNORM, hid, H, an, 0, qkv, qkvd, ACB_EPI_STORE, nullptr, 0));
            ACB_TRY(gemv_rows(m, L.k, 0, kvd, n, ACB_PRO_RMSNORM, hid, H, an, 0, qkv + qd, qkvd, ACB_EPI_STORE, nullptr, 0));
            ACB_TRY(gemv_rows(m, L.v, 0, kvd, n, ACB_PRO_RMSNORM, hid, H, an, 0, qkv + qd + kvd, qkvd, ACB_EPI_STORE,
                              nullptr, 0));
        }
        uint16_t * kc = m->kc.as<uint16_t>() + (size_t) l * m->layer_elems;
        uint16_t * vc = m->vc.as<uint16_t>() + (size_t) l * m->layer_elems;
        ACB_TRY(acb_qkv_post(qkv, qkvd, n, c.n_heads, c.n_kv_heads, D, (const float *) L.q_norm->data,
                             (const float *) L.k_norm->data, c.rms_norm_eps, m->pos.as<int32_t>(), m->rope.as<float>(),
                             c.max_seq_len, m->q.as<float>(), qd, kc, vc, c.max_seq_len, set0, set_per_tok, ACB_FLAG_PDL,
                             m->err.as<int>(), (acb_stream_t) m->st));
        const int ns = m->splits(n);
        ACB_TRY(acb_attn_decode(m->q.as<float>(), qd, n, c.n_heads, c.n_kv_heads, D, m->pos.as<int32_t>(), kc, vc,
                                c.max_seq_len, set0, set_per_tok, 1.0f / sqrtf((float) D), ns, m->scores.as<float>(),
                                m->smax.as<float>(), m->part.as<double>(), m->att.as<float>(), qd,
                                m->tickets.as<int>(), ACB_FLAG_PDL, (acb_stream_t) m->st));
        ACB_TRY(gemv_rows(m, L.o, 0, H, n, ACB_PRO_X, m->att.as<float>(), qd, nullptr, 0, hid, H, ACB_EPI_ADD, hid, H));
        const float * pn = (const float *) L.post_norm->data;
        float *       gu = m->gu.as<float>();
        if (L.gate_up) {
            ACB_TRY(gemv_rows(m, L.gate_up, 0, 2 * F, n, ACB_PRO_RMSNORM, hid, H, pn, 0, gu, 2 * F, ACB_EPI_STORE, nullptr, 0));
        } else {
            ACB_TRY(gemv_rows(m, L.gate, 0, F, n, ACB_PRO_RMSNORM, hid, H, pn, 0, gu, 2 * F, ACB_EPI_STORE, nullptr, 0));
            ACB_TRY(gemv_rows(m, L.up, 0, F, n, ACB_PRO_RMSNORM, hid, H, pn, 0, gu + F, 2 * F, ACB_EPI_STORE, nullptr, 0));
        }
        ACB_TRY(gemv_rows(m, L.down, 0, H, n, ACB_PRO_SWIGLU, gu, 2 * F, nullptr, 0, hid, H, ACB_EPI_ADD, hid, H));
    }
    return ACB_OK;
}

acb_status check_err(acb_qw3lm * m) {
    int e = 0;
    if (cudaMemcpy(&e, m->err.p, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    if (e != 0) {
        cudaMemset(m->err.p, 0, sizeof(int));
        if (m->persist) {
            cudaMemset(m->pd_scratch.p, 0, m->pd_scratch.bytes);  // counters of an aborted step
        }
        set_last_error("device error flag " + std::to_string(e));
        return ACB_ERR_DEVICE;
    }
    return ACB_OK;
}

acb_status sync(acb_qw3lm * m) {
    const cudaError_t e = cudaStreamSynchronize(m->st);
    if (e != cudaSuccess) {
        set_last_error(cudaGetErrorString(e));
        return ACB_ERR_CUDA;
    }
    return check_err(m);
}

const DevTensor * head_for(acb_qw3lm * m, int lm_offset, int lm_count, int * out_v) {
    if (lm_count > 0 && m->head2_off == lm_offset && m->head2_t.N == lm_count) {
        *out_v = lm_count;
        return &m->head2_t;
    }
    *out_v = m->c.vocab_size;
    return m->head_tiles_t.valid() ? &m->head_tiles_t : m->embed;
}

// The persistent single-sequence step needs every linear in tensor-core tiles with fused qkv and
// gate|up rows, a Q8_0 embedding and its tiled head copy; otherwise the per-op graph runs.
// ACB_LM_PERSIST=0 keeps the per-op graph (for comparisons).
void setup_persistent(acb_qw3lm * m) {
    const char * env = std::getenv("ACB_LM_PERSIST");
    if (env && std::strcmp(env, "0") == 0) {
        return;
    }
    const acb_qw3lm_config & c = m->c;
    if (!m->head_tiles_t.valid() || m->embed->type != ACB_TYPE_Q8_0) {
        return;
    }
    std::vector<acb_decode_layer> ls(c.n_layers);
    for (int l = 0; l < c.n_layers; l++) {
        const LMLayer & L = m->layers[l];
        for (const DevTensor * t : { L.qkv, L.o, L.gate_up, L.down }) {
            if (!t || t->type != ACB_TYPE_Q8_0_TILES || (reinterpret_cast<uintptr_t>(t->data) & 15)) {
                return;
            }
        }
        acb_decode_layer & d = ls[l];
        d.qkv                = L.qkv->data;
        d.o                  = L.o->data;
        d.gate_up            = L.gate_up->data;
        d.down               = L.down->data;
        d.attn_norm          = (const float *) L.attn_norm->data;
        d.post_norm          = (const float *) L.post_norm->data;
        d.q_norm             = L.q_norm ? (const float *) L.q_norm->data : nullptr;
        d.k_norm             = L.k_norm ? (const float *) L.k_norm->data : nullptr;
        d.k_cache            = m->kc.as<uint16_t>() + (size_t) l * m->layer_elems;
        d.v_cache            = m->vc.as<uint16_t>() + (size_t) l * m->layer_elems;
    }
    acb_decode_step & p = m->pd;
    p.n_layers          = c.n_layers;
    p.hidden            = c.hidden_size;
    p.ffn               = c.intermediate_size;
    p.n_heads           = c.n_heads;
    p.n_kv_heads        = c.n_kv_heads;
    p.head_dim          = c.head_dim;
    p.eps               = c.rms_norm_eps;
    p.attn_scale        = 1.0f / sqrtf((float) c.head_dim);
    p.max_seq           = c.max_seq_len;
    p.max_pos           = c.max_seq_len;
    p.embed             = m->embed->data;
    p.embed_rows        = m->embed->N;
    p.head              = m->head_tiles_t.data;
    p.vocab             = m->head_tiles_t.N;
    p.final_norm        = (const float *) m->final_norm->data;
    p.rope              = m->rope.as<float>();
    p.ids               = m->ids.as<int32_t>();
    p.pos               = m->pos.as<int32_t>();
    p.logits            = m->logits.as<float>();
    p.err               = m->err.as<int>();
    const size_t sb     = acb_lm_decode_scratch_bytes(&p);
    if (sb == 0 || m->pd_layers.alloc(ls.size() * sizeof(acb_decode_layer), false) != ACB_OK ||
        m->pd_scratch.alloc(sb) != ACB_OK) {
        return;
    }
    if (cudaMemcpy(m->pd_layers.p, ls.data(), ls.size() * sizeof(acb_decode_layer), cudaMemcpyHostToDevice) !=
        cudaSuccess) {
        return;
    }
    p.layers   = m->pd_layers.as<acb_decode_layer>();
    p.scratch  = m->pd_scratch.p;
    m->persist = true;
}

// One persistent launch for kv set `set` (ids/pos already on the device): one step, or n_steps
// greedy steps that feed each argmax to the next.
acb_status persistent_step(acb_qw3lm * m, int set, bool greedy, int n_steps = 1) {
    acb_decode_step p = m->pd;
    p.kv_set          = set;
    p.greedy          = greedy ? 1 : 0;
    p.n_steps         = greedy ? n_steps : 1;
    if (greedy) {
        p.hist      = m->hist.as<int32_t>();
        p.mhist     = m->mhist.as<float>();
        p.hist_base = m->hist_base.as<int32_t>();
    }
    return acb_lm_decode_step(&p, (acb_stream_t) m->st);
}

// step graph: [embed gather] [layers] [head] (+ argmax/advance when greedy)
acb_status enqueue_step(acb_qw3lm * m, int N, int set0, const DevTensor * head, int out_v, bool greedy) {
    ACB_TRY(acb_get_rows(m->embed->data, m->embed->type, m->embed->N, m->embed->K, m->ids.as<int32_t>(), N,
                         m->hidden.p, ACB_TYPE_F32, m->c.hidden_size, m->err.as<int>(), (acb_stream_t) m->st));
    ACB_TRY(enqueue_layers(m, N, set0, 1));
    ACB_TRY(gemv_rows(m, head, 0, out_v, N, ACB_PRO_RMSNORM, m->hidden.as<float>(), m->c.hidden_size,
                      (const float *) m->final_norm->data, 0, m->logits.as<float>(), out_v, ACB_EPI_STORE, nullptr, 0));
    if (greedy) {
        ACB_TRY(acb_argmax(m->logits.as<float>(), out_v, out_v, N, m->ids.as<int32_t>(), nullptr, m->pos.as<int32_t>(),
                           m->hist.as<int32_t>(), m->mhist.as<float>(), m->c.max_seq_len, m->hist_base.as<int32_t>(),
                           m->amax.p, ACB_FLAG_PDL, (acb_stream_t) m->st));
    }
    return ACB_OK;
}

acb_status run_graph(acb_qw3lm * m, long long key, int N, int set0, const DevTensor * head, int out_v, bool greedy,
                     bool with_upload) {
    auto it = m->graphs.find(key);
    if (it == m->graphs.end()) {
        cudaGraph_t g = nullptr;
        if (cudaStreamBeginCapture(m->st, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
            return ACB_ERR_CUDA;
        }
        acb_status s = ACB_OK;
        if (with_upload) {
            cudaMemcpyAsync(m->ids.p, m->h_ids, sizeof(int32_t) * N, cudaMemcpyHostToDevice, m->st);
            cudaMemcpyAsync(m->pos.p, m->h_pos, sizeof(int32_t) * N, cudaMemcpyHostToDevice, m->st);
        }
        s                   = enqueue_step(m, N, set0, head, out_v, greedy);
        const cudaError_t e = cudaStreamEndCapture(m->st, &g);
        if (s != ACB_OK || e != cudaSuccess) {
            if (g) {
                cudaGraphDestroy(g);
            }
            cudaGetLastError();
            return s != ACB_OK ? s : ACB_ERR_CUDA;
        }
        cudaGraphExec_t ge = nullptr;
        if (cudaGraphInstantiate(&ge, g, 0) != cudaSuccess) {
            cudaGraphDestroy(g);
            return ACB_ERR_CUDA;
        }
        cudaGraphDestroy(g);
        it = m->graphs.emplace(key, ge).first;
    }
    if (cudaGraphLaunch(it->second, m->st) != cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    return ACB_OK;
}

}  // namespace

extern "C" acb_status acb_qw3lm_load(const char * gguf_path, int max_seq_len, int n_kv_sets, int device,
                                     acb_qw3lm ** out) {
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
    auto m    = new acb_qw3lm();
    m->device = device;
    // 0.6B defaults, then acestep.config_json (qw3lm_load_config, qwen3-lm.h:124-160)
    acb_qw3lm_config & c = m->c;
    c                    = { 217204, 1024, 3072, 16, 8, 128, 28, 1000000.0f, 1e-6f, 1, 8192 };
    const char * j       = gf.get_str("acestep.config_json");
    if (j && j[0]) {
        c.vocab_size        = json_int(j, "vocab_size", c.vocab_size);
        c.hidden_size       = json_int(j, "hidden_size", c.hidden_size);
        c.intermediate_size = json_int(j, "intermediate_size", c.intermediate_size);
        c.n_heads           = json_int(j, "num_attention_heads", c.n_heads);
        c.n_kv_heads        = json_int(j, "num_key_value_heads", c.n_kv_heads);
        c.head_dim          = json_int(j, "head_dim", c.head_dim);
        c.n_layers          = json_int(j, "num_hidden_layers", c.n_layers);
        c.rope_theta        = json_float(j, "rope_theta", c.rope_theta);
        c.rms_norm_eps      = json_float(j, "rms_norm_eps", c.rms_norm_eps);
        c.tie_embeddings    = json_bool(j, "tie_word_embeddings", true) ? 1 : 0;
    }
    if (max_seq_len > 0) {
        c.max_seq_len = max_seq_len;
    }
    m->n_sets = n_kv_sets > 0 ? n_kv_sets : 1;
    auto bad  = [&](acb_status s, const std::string & msg) {
        set_last_error(msg);
        delete m;
        return s;
    };
    if (c.n_layers <= 0 || c.n_layers > 64 || m->n_sets > kMaxSets || c.head_dim != 128 ||
        c.n_heads % c.n_kv_heads != 0) {
        return bad(ACB_ERR_UNSUPPORTED, "unsupported LM configuration");
    }
    if (cudaStreamCreateWithFlags(&m->st, cudaStreamNonBlocking) != cudaSuccess) {
        return bad(ACB_ERR_CUDA, "stream creation failed");
    }

    WeightArena & A = m->arena;
    m->embed        = A.load(gf, "model.embed_tokens.weight");
    m->final_norm   = A.load_f32(gf, "model.norm.weight");
    m->layers.resize(c.n_layers);
    for (int i = 0; i < c.n_layers; i++) {
        const std::string p = "model.layers." + std::to_string(i);
        LMLayer &         L = m->layers[i];
        L.attn_norm         = A.load_f32(gf, p + ".input_layernorm.weight");
        L.post_norm         = A.load_f32(gf, p + ".post_attention_layernorm.weight");
        const std::string q = p + ".self_attn.q_proj.weight", k = p + ".self_attn.k_proj.weight",
                          v = p + ".self_attn.v_proj.weight";
        L.qkv               = A.load_fused(gf, { q, k, v });
        if (!L.qkv) {
            L.qk = A.load_fused(gf, { q, k });
            if (L.qk) {
                L.v = A.load(gf, v);
            } else {
                L.q = A.load(gf, q);
                L.k = A.load(gf, k);
                L.v = A.load(gf, v);
            }
        }
        L.o       = A.load(gf, p + ".self_attn.o_proj.weight");
        L.q_norm  = A.load_f32(gf, p + ".self_attn.q_norm.weight");
        L.k_norm  = A.load_f32(gf, p + ".self_attn.k_norm.weight");
        L.gate_up = A.load_fused(gf, { p + ".mlp.gate_proj.weight", p + ".mlp.up_proj.weight" });
        if (!L.gate_up) {
            L.gate = A.load(gf, p + ".mlp.gate_proj.weight");
            L.up   = A.load(gf, p + ".mlp.up_proj.weight");
        }
        L.down = A.load(gf, p + ".mlp.down_proj.weight");
        const bool ok = L.attn_norm && L.post_norm && L.o && L.q_norm && L.k_norm && L.down &&
                        (L.qkv || (L.qk && L.v) || (L.q && L.k && L.v)) && (L.gate_up || (L.gate && L.up));
        if (!ok) {
            return bad(ACB_ERR_FORMAT, A.error.empty() ? "missing layer tensor" : A.error);
        }
    }
    if (!m->embed || !m->final_norm) {
        return bad(ACB_ERR_FORMAT, A.error);
    }
    if (m->embed->K != c.hidden_size || m->embed->N < c.vocab_size) {
        return bad(ACB_ERR_FORMAT, "embed_tokens shape does not match the config");
    }
    {
        acb_status s = A.upload(m->st);
        if (s != ACB_OK) {
            return bad(s, A.error);
        }
    }
    {
        // Q8_0 linears (N a multiple of 16) repacked in place into the tensor-core GEMV's tiles;
        // the embedding keeps its GGUF rows for get_rows and gets a tiled copy for the head
        size_t big = 0;
        auto   tileable = [](const DevTensor * t) { return t && t->type == ACB_TYPE_Q8_0 && t->N % 16 == 0; };
        std::vector<DevTensor *> lin;
        for (LMLayer & L : m->layers) {
            for (DevTensor * t : { L.qkv, L.qk, L.q, L.k, L.v, L.o, L.gate_up, L.gate, L.up, L.down }) {
                if (tileable(t)) {
                    lin.push_back(t);
                    big = std::max(big, (size_t) t->N * (size_t) t->row_bytes());
                }
            }
        }
        DevBuf tmp;
        if (!lin.empty() && tmp.alloc(big, false) != ACB_OK) {
            return bad(ACB_ERR_OOM, "repack buffer allocation failed");
        }
        for (DevTensor * t : lin) {
            const size_t bytes = (size_t) t->N * (size_t) t->row_bytes();
            if (cudaMemcpyAsync(tmp.p, t->data, bytes, cudaMemcpyDeviceToDevice, m->st) != cudaSuccess) {
                return bad(ACB_ERR_CUDA, "repack copy failed");
            }
            acb_status s = acb_q8_0_to_tiles(tmp.p, t->data, t->N, t->K, (acb_stream_t) m->st);
            if (s != ACB_OK) {
                return bad(s, "repack failed");
            }
            t->type = ACB_TYPE_Q8_0_TILES;
        }
        if (tileable(m->embed) && m->embed->N >= c.vocab_size) {
            const int64_t n = (int64_t) c.vocab_size / 16 * 16;
            if (n == c.vocab_size && m->head_tiles.alloc((size_t) n * m->embed->row_bytes(), false) == ACB_OK) {
                acb_status s = acb_q8_0_to_tiles(m->embed->data, m->head_tiles.p, n, m->embed->K, (acb_stream_t) m->st);
                if (s != ACB_OK) {
                    return bad(s, "head repack failed");
                }
                m->head_tiles_t      = *m->embed;
                m->head_tiles_t.type = ACB_TYPE_Q8_0_TILES;
                m->head_tiles_t.data = m->head_tiles.p;
                m->head_tiles_t.N    = n;
            }
        }
        if (cudaStreamSynchronize(m->st) != cudaSuccess) {
            return bad(ACB_ERR_CUDA, "repack failed");
        }
    }

    // KV cache [L][n_sets][Nkv][max_seq][D] f16, zeroed (qw3lm_alloc_kv_cache, qwen3-lm.h:173-224)
    const int D = c.head_dim, S = c.max_seq_len;
    m->layer_elems = (size_t) m->n_sets * c.n_kv_heads * S * D;
    if (m->kc.alloc(m->layer_elems * c.n_layers * 2) || m->vc.alloc(m->layer_elems * c.n_layers * 2)) {
        return bad(ACB_ERR_OOM, "KV cache allocation failed");
    }
    m->kv_pos.assign(m->n_sets, 0);
    {
        std::vector<float> tab((size_t) S * D);
        acb_rope_table_host(tab.data(), S, D, c.rope_theta);
        if (m->rope.alloc(tab.size() * 4, false)) {
            return bad(ACB_ERR_OOM, "rope table allocation failed");
        }
        cudaMemcpy(m->rope.p, tab.data(), tab.size() * 4, cudaMemcpyHostToDevice);
    }
    // scratch for up to cap_tok tokens per pass
    m->cap_tok    = std::max(kPrefillChunk, kMaxSets);
    m->max_split  = 32;
    size_t part_n = 0;
    for (int n = 1; n <= m->cap_tok; n++) {
        part_n = std::max(part_n, (size_t) n * m->splits(n));
    }
    const size_t T = (size_t) m->cap_tok;
    bool         f = false;
    f |= m->hidden.alloc(T * c.hidden_size * 4) != ACB_OK;
    f |= m->qkv.alloc(T * m->qkvd() * 4) != ACB_OK;
    f |= m->q.alloc(T * m->qd() * 4) != ACB_OK;
    f |= m->scores.alloc(T * c.n_heads * (size_t) S * 4) != ACB_OK;
    f |= m->smax.alloc(T * c.n_heads * m->max_split * 4) != ACB_OK;
    f |= m->part.alloc(part_n * m->qd() * 8) != ACB_OK;  // double split partials
    f |= m->att.alloc(T * m->qd() * 4) != ACB_OK;
    f |= m->tickets.alloc(T * c.n_kv_heads * 4) != ACB_OK;  // zeroed; every attention call leaves it zero
    f |= m->gu.alloc(T * 2 * c.intermediate_size * 4) != ACB_OK;
    f |= m->logits.alloc((size_t) kMaxSets * c.vocab_size * 4) != ACB_OK;
    f |= m->ids.alloc(T * 4) != ACB_OK;
    f |= m->pos.alloc(T * 4) != ACB_OK;
    f |= m->err.alloc(16) != ACB_OK;
    f |= m->hist_base.alloc(kMaxSets * 4) != ACB_OK;
    f |= m->hist.alloc((size_t) kMaxSets * S * 4) != ACB_OK;
    f |= m->mhist.alloc((size_t) kMaxSets * S * 4) != ACB_OK;
    f |= m->amax.alloc(acb_argmax_scratch_bytes(kMaxSets, c.vocab_size)) != ACB_OK;  // zeroed
    f |= cudaMallocHost(&m->h_ids, T * 4) != cudaSuccess;
    f |= cudaMallocHost(&m->h_pos, T * 4) != cudaSuccess;
    if (f) {
        return bad(ACB_ERR_OOM, "scratch allocation failed");
    }
    setup_persistent(m);
    *out = m;
    return ACB_OK;
}

extern "C" acb_status acb_qw3lm_get_config(const acb_qw3lm * m, acb_qw3lm_config * cfg) {
    if (!m || !cfg) {
        return ACB_ERR_INVALID_ARG;
    }
    *cfg = m->c;
    return ACB_OK;
}

extern "C" size_t acb_qw3lm_weight_bytes(const acb_qw3lm * m) {
    return m ? m->arena.bytes() : 0;
}

extern "C" int acb_qw3lm_kv_pos(const acb_qw3lm * m, int kv_set) {
    return (m && kv_set >= 0 && kv_set < m->n_sets) ? m->kv_pos[kv_set] : -1;
}

extern "C" int acb_qw3lm_persistent_decode(const acb_qw3lm * m) {
    return m && m->persist ? 1 : 0;
}

extern "C" void acb_qw3lm_reset_kv(acb_qw3lm * m, int kv_set) {
    if (m && kv_set >= 0 && kv_set < m->n_sets) {
        m->kv_pos[kv_set] = 0;  // positions beyond kv_pos are never read
    }
}

extern "C" acb_status acb_qw3lm_copy_kv(acb_qw3lm * m, int src, int dst) {
    if (!m || src < 0 || dst < 0 || src >= m->n_sets || dst >= m->n_sets) {
        return ACB_ERR_INVALID_ARG;
    }
    cudaSetDevice(m->device);
    const size_t set_elems = (size_t) m->c.n_kv_heads * m->c.max_seq_len * m->c.head_dim;
    for (int l = 0; l < m->c.n_layers; l++) {
        const size_t base = (size_t) l * m->layer_elems;
        cudaMemcpyAsync(m->kc.as<uint16_t>() + base + dst * set_elems, m->kc.as<uint16_t>() + base + src * set_elems,
                        set_elems * 2, cudaMemcpyDeviceToDevice, m->st);
        cudaMemcpyAsync(m->vc.as<uint16_t>() + base + dst * set_elems, m->vc.as<uint16_t>() + base + src * set_elems,
                        set_elems * 2, cudaMemcpyDeviceToDevice, m->st);
    }
    m->kv_pos[dst] = m->kv_pos[src];
    return sync(m);
}

extern "C" acb_status acb_qw3lm_build_partial_head(acb_qw3lm * m, int lm_offset) {
    if (!m) {
        return ACB_ERR_INVALID_ARG;
    }
    const int V = m->c.vocab_size, count = V - lm_offset;
    if (count <= 0 || count >= V) {
        return ACB_ERR_INVALID_ARG;
    }
    cudaSetDevice(m->device);
    const int64_t rb = m->embed->row_bytes();
    if (m->head2.alloc((size_t) count * rb + 512)) {
        return ACB_ERR_OOM;
    }
    cudaMemcpy(m->head2.p, (const uint8_t *) m->embed->data + (size_t) lm_offset * rb, (size_t) count * rb,
               cudaMemcpyDeviceToDevice);
    m->head2_t      = *m->embed;
    m->head2_t.data = m->head2.p;
    m->head2_t.N    = count;
    m->head2_off    = lm_offset;
    return ACB_OK;
}

extern "C" acb_status acb_qw3lm_forward(acb_qw3lm * m, const int32_t * token_ids, int n_tokens, int kv_set,
                                        float * logits) {
    if (!m || !token_ids || n_tokens <= 0 || kv_set < 0 || kv_set >= m->n_sets) {
        return ACB_ERR_INVALID_ARG;
    }
    const acb_qw3lm_config & c = m->c;
    if (m->kv_pos[kv_set] + n_tokens > c.max_seq_len) {
        set_last_error("kv_len exceeds max_seq");
        return ACB_ERR_OUT_OF_RANGE;
    }
    for (int i = 0; i < n_tokens; i++) {
        if (token_ids[i] < 0 || token_ids[i] >= m->embed->N) {
            return ACB_ERR_OUT_OF_RANGE;
        }
    }
    cudaSetDevice(m->device);
    const int H = c.hidden_size;
    for (int c0 = 0; c0 < n_tokens; c0 += kPrefillChunk) {
        const int n = std::min(kPrefillChunk, n_tokens - c0);
        ACB_TRY(sync(m));  // pinned staging is reused
        for (int i = 0; i < n; i++) {
            m->h_ids[i] = token_ids[c0 + i];
            m->h_pos[i] = m->kv_pos[kv_set] + c0 + i;
        }
        cudaMemcpyAsync(m->ids.p, m->h_ids, sizeof(int32_t) * n, cudaMemcpyHostToDevice, m->st);
        cudaMemcpyAsync(m->pos.p, m->h_pos, sizeof(int32_t) * n, cudaMemcpyHostToDevice, m->st);
        ACB_TRY(acb_get_rows(m->embed->data, m->embed->type, m->embed->N, m->embed->K, m->ids.as<int32_t>(), n,
                             m->hidden.p, ACB_TYPE_F32, H, m->err.as<int>(), (acb_stream_t) m->st));
        ACB_TRY(enqueue_layers(m, n, kv_set, 0));
        if (c0 + n == n_tokens && logits) {
            ACB_TRY(gemv_rows(m, m->head_tiles_t.valid() ? &m->head_tiles_t : m->embed, 0, c.vocab_size, 1, ACB_PRO_RMSNORM, m->hidden.as<float>() + (size_t) (n - 1) * H,
                              H, (const float *) m->final_norm->data, 0, m->logits.as<float>(), c.vocab_size,
                              ACB_EPI_STORE, nullptr, 0));
            cudaMemcpyAsync(logits, m->logits.p, sizeof(float) * c.vocab_size, cudaMemcpyDeviceToHost, m->st);
        }
    }
    ACB_TRY(sync(m));
    m->kv_pos[kv_set] += n_tokens;
    return ACB_OK;
}

// One decode step for N consecutive sets; the logits [N][*out_v] stay in m->logits and the sets'
// positions advance once the step has been enqueued.
static acb_status forward_batch_dev(acb_qw3lm * m, const int32_t * token_ids, const int32_t * kv_sets, int N,
                                    int lm_offset, int lm_count, int * out_v_ret) {
    if (!m || !token_ids || !kv_sets || N <= 0 || N > kMaxSets) {
        return ACB_ERR_INVALID_ARG;
    }
    const int set0 = kv_sets[0];
    for (int i = 0; i < N; i++) {
        if (kv_sets[i] != set0 + i || kv_sets[i] < 0 || kv_sets[i] >= m->n_sets) {
            set_last_error("kv_sets must be consecutive and in range");
            return ACB_ERR_INVALID_ARG;
        }
        if (m->kv_pos[kv_sets[i]] + 1 > m->c.max_seq_len) {
            set_last_error("kv_len exceeds max_seq");
            return ACB_ERR_OUT_OF_RANGE;
        }
        if (token_ids[i] < 0 || token_ids[i] >= m->embed->N) {
            return ACB_ERR_OUT_OF_RANGE;
        }
    }
    cudaSetDevice(m->device);
    int               out_v = 0;
    const DevTensor * head  = head_for(m, lm_offset, lm_count, &out_v);
    ACB_TRY(sync(m));
    for (int i = 0; i < N; i++) {
        m->h_ids[i] = token_ids[i];
        m->h_pos[i] = m->kv_pos[set0 + i];
    }
    if (N == 1 && m->persist && head == &m->head_tiles_t) {
        cudaMemcpyAsync(m->ids.p, m->h_ids, sizeof(int32_t), cudaMemcpyHostToDevice, m->st);
        cudaMemcpyAsync(m->pos.p, m->h_pos, sizeof(int32_t), cudaMemcpyHostToDevice, m->st);
        ACB_TRY(persistent_step(m, set0, false));
    } else {
        const long long key =
            ((long long) N << 40) | ((long long) set0 << 32) | ((long long) (head == m->embed ? 0 : 1) << 31);
        ACB_TRY(run_graph(m, key, N, set0, head, out_v, false, true));
    }
    for (int i = 0; i < N; i++) {
        m->kv_pos[set0 + i]++;
    }
    *out_v_ret = out_v;
    return ACB_OK;
}

extern "C" acb_status acb_qw3lm_forward_batch(acb_qw3lm * m, const int32_t * token_ids, const int32_t * kv_sets,
                                              int N, float * logits, int lm_offset, int lm_count) {
    if (!logits) {
        return ACB_ERR_INVALID_ARG;
    }
    int out_v = 0;
    ACB_TRY(forward_batch_dev(m, token_ids, kv_sets, N, lm_offset, lm_count, &out_v));
    cudaMemcpyAsync(logits, m->logits.p, sizeof(float) * (size_t) N * out_v, cudaMemcpyDeviceToHost, m->st);
    return sync(m);
}

extern "C" acb_status acb_qw3lm_forward_batch_sample(acb_qw3lm * m, const int32_t * token_ids,
                                                     const int32_t * kv_sets, int n_active, int use_cfg,
                                                     float cfg_scale, int lm_offset, int lm_count, int eos_idx,
                                                     int code_offset, int n_codes, float temperature, float top_p,
                                                     int top_k, const float * u, int32_t * sampled) {
    if (!m || !sampled || n_active <= 0 || n_codes < 0 || (temperature > 0.0f && !u)) {
        return ACB_ERR_INVALID_ARG;
    }
    const int N     = use_cfg ? 2 * n_active : n_active;
    int       out_v = 0;
    ACB_TRY(forward_batch_dev(m, token_ids, kv_sets, N, lm_offset, lm_count, &out_v));
    if (eos_idx < 0 || eos_idx >= out_v || code_offset < 0 || code_offset + n_codes > out_v) {
        set_last_error("EOS / audio-code columns outside the logit row");
        return ACB_ERR_INVALID_ARG;
    }
    const int    Vc = 1 + n_codes;
    const size_t wb = acb_sample_work_bytes(n_active, Vc);
    if ((m->samp_work.bytes < wb && m->samp_work.alloc(wb, false) != ACB_OK) ||
        (!m->samp_u.p && m->samp_u.alloc((size_t) kMaxSets * 4, false) != ACB_OK) ||
        (!m->samp_idx.p && m->samp_idx.alloc((size_t) kMaxSets * 4, false) != ACB_OK)) {
        set_last_error("sampling scratch allocation failed");
        return ACB_ERR_OOM;
    }
    if (u && cudaMemcpyAsync(m->samp_u.p, u, sizeof(float) * n_active, cudaMemcpyHostToDevice, m->st) !=
                 cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    const float * lg = m->logits.as<float>();
    ACB_TRY(acb_sample_top_k_p(lg, out_v, use_cfg ? lg + (size_t) n_active * out_v : nullptr, out_v, cfg_scale,
                               eos_idx, code_offset, n_codes, n_active, temperature, top_p, top_k,
                               u ? m->samp_u.as<float>() : nullptr, m->samp_work.as<float>(),
                               m->samp_idx.as<int32_t>(), (acb_stream_t) m->st));
    cudaMemcpyAsync(sampled, m->samp_idx.p, sizeof(int32_t) * n_active, cudaMemcpyDeviceToHost, m->st);
    return sync(m);
}

extern "C" acb_status acb_qw3lm_generate_greedy(acb_qw3lm * m, const int32_t * last_ids, int set0, int N,
                                                int n_steps, int32_t * tokens_out, float * margins_out,
                                                float * gpu_ms) {
    if (!m || !last_ids || N <= 0 || N > kMaxSets || n_steps <= 0 || set0 < 0 || set0 + N > m->n_sets) {
        return ACB_ERR_INVALID_ARG;
    }
    for (int i = 0; i < N; i++) {
        if (m->kv_pos[set0 + i] + n_steps > m->c.max_seq_len) {
            set_last_error("kv_len exceeds max_seq");
            return ACB_ERR_OUT_OF_RANGE;
        }
        if (last_ids[i] < 0 || last_ids[i] >= m->embed->N) {
            return ACB_ERR_OUT_OF_RANGE;
        }
    }
    cudaSetDevice(m->device);
    ACB_TRY(sync(m));
    for (int i = 0; i < N; i++) {
        m->h_ids[i] = last_ids[i];
        m->h_pos[i] = m->kv_pos[set0 + i];
    }
    cudaMemcpyAsync(m->ids.p, m->h_ids, sizeof(int32_t) * N, cudaMemcpyHostToDevice, m->st);
    cudaMemcpyAsync(m->pos.p, m->h_pos, sizeof(int32_t) * N, cudaMemcpyHostToDevice, m->st);
    cudaMemcpyAsync(m->hist_base.p, m->h_pos, sizeof(int32_t) * N, cudaMemcpyHostToDevice, m->st);
    ACB_TRY(sync(m));
    const long long key = ((long long) N << 40) | ((long long) set0 << 32) | (1ll << 30);
    cudaEvent_t     e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    cudaEventRecord(e0, m->st);
    acb_status s = ACB_OK;
    int               hv    = 0;
    const DevTensor * ghead = head_for(m, 0, 0, &hv);
    const bool        pers  = N == 1 && m->persist;
    if (pers) {
        // up to 64 tokens per launch (each launch ends with the counters back at zero)
        for (int k = 0; k < n_steps && s == ACB_OK; k += 64) {
            s = persistent_step(m, set0, true, std::min(64, n_steps - k));
        }
    } else {
        for (int k = 0; k < n_steps && s == ACB_OK; k++) {
            s = run_graph(m, key, N, set0, ghead, hv, true, false);
        }
    }
    cudaEventRecord(e1, m->st);
    if (s == ACB_OK) {
        s = sync(m);
    }
    if (s == ACB_OK && gpu_ms) {
        cudaEventElapsedTime(gpu_ms, e0, e1);
    }
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    if (s != ACB_OK) {
        return s;
    }
    const size_t S = (size_t) m->c.max_seq_len;
    for (int i = 0; i < N; i++) {
        if (tokens_out) {
            cudaMemcpy(tokens_out + (size_t) i * n_steps, m->hist.as<int32_t>() + i * S, sizeof(int32_t) * n_steps,
                       cudaMemcpyDeviceToHost);
        }
        if (margins_out) {
            cudaMemcpy(margins_out + (size_t) i * n_steps, m->mhist.as<float>() + i * S, sizeof(float) * n_steps,
                       cudaMemcpyDeviceToHost);
        }
        m->kv_pos[set0 + i] += n_steps;
    }
    return ACB_OK;
}

extern "C" void acb_qw3lm_free(acb_qw3lm * m) {
    delete m;
}
