// qwen3_enc.cpp -- the Qwen3 encoder stack of acestep.cpp (src/qwen3-enc.h) on libacb kernels.
//
// Prefill over a whole prompt is GEMM-shaped, so every linear is a tensor-core GEMM (dense.h)
// over a resident 16-bit copy of the weights with the activation quantised like ggml's
// quantised mul_mat. In the default exact mode products are formed from hi/lo f16 splits of the
// reference's own dequantised operands and attention likewise (acb_attn_prefill_split), so the
// result tracks the reference CPU build to fp32 summation order; fast mode uses single f16
// operands. One forward for S tokens, per layer:
//   RMSNorm * input_layernorm                h (f32)       -> xn (f32)
//   quantise + GEMM  Q||K||V                 xn            -> qkv (f32 exact / f16 fast)
//   q/k RMSNorm + NeoX RoPE (2 launches)     qkv columns   -> in place (exact) / q, k (fast)
//   hi/lo planes of Q||K||V (exact)          qkv           -> planes
//   flash attention, causal                  q, k, v views -> att (f32)
//   quantise + GEMM  o_proj, epilogue + h    att           -> h (in place)
//   RMSNorm * post_attention_layernorm       h             -> xn
//   quantise + GEMM  gate||up                xn            -> gu (f32 [S][2F])
//   SwiGLU + quantise + GEMM down, + h       gu            -> h (in place)
// then the final RMSNorm into f32 output. The chain for each (S, mode) is captured once as a
// CUDA graph (tensor-core launches with programmatic dependent launch) and replayed.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "../../include/acb_models.h"
#include "dense.h"
#include "enc_stack.h"
#include "gguf.h"
#include "host_common.h"
#include "weights.h"

using namespace acb;

namespace {

struct EncLayer {
    DevTensor * attn_norm = nullptr, *post_norm = nullptr, *q_norm = nullptr, *k_norm = nullptr;
    DenseLinear qkv, o, gu, down;
};

constexpr int kPdl = ACB_FLAG_PDL;

}  // namespace

struct acb_qwen3_enc {
    int                   device = 0;
    acb_qwen3_config      c{};
    int                   window = 0;  // non-causal stacks: |i - j| <= window on even layers (cond-enc.h:203-208)
    WeightArena           arena;  // embedding table (GGUF type) and F32 norms
    DevBuf                w16;    // every linear, 16-bit
    DevTensor *           embed = nullptr, *final_norm = nullptr;
    std::vector<EncLayer> layers;
    cudaStream_t          st    = nullptr;
    bool                  exact = true;

    // scratch for up to cap rows; positions restart every `period` rows (0: row index)
    int                            cap = 0, period = 0;
    DevBuf                         ids, pos, rope, h, xn, xq, qkv, qkv32, planes, vtb, q, k, att, gu, out, err, ws;
    int                            s_ld = 0;  // V^T row length: the sequence length rounded up to 8
    std::map<int, cudaGraphExec_t> graphs;  // one per S * 2 + exact
    std::map<int, int>             graph_kernels;  // their kernel nodes
    int                            last_kernels = 0;  // kernel launches of the last forward

    ~acb_qwen3_enc() {
        cudaSetDevice(device);
        drop_graphs();
        if (st) {
            cudaStreamDestroy(st);
        }
    }

    void drop_graphs() {
        for (auto & kv : graphs) {
            cudaGraphExecDestroy(kv.second);
        }
        graphs.clear();
        graph_kernels.clear();
    }

    int nqkv() const { return (c.n_heads + 2 * c.n_kv_heads) * c.head_dim; }

    // room for R rows in sequences of S rows; period: S for a batch of sequences, 0 for one
    acb_status reserve(int R, int S, int period);
    acb_status reserve(int S) { return reserve(S, S, 0); }
    DenseScratch scratch() { return DenseScratch{ xq.p, ws.p, ws.bytes, err.as<int>() }; }
    // layers [l0, l1) over B sequences of S rows in h (positions 0..S-1 in each)
    acb_status enqueue_layers(int B, int S, int l0, int l1, cudaStream_t s);
    acb_status enqueue_layers(int S, int l0, int l1, cudaStream_t s) { return enqueue_layers(1, S, l0, l1, s); }
    acb_status enqueue(int S, cudaStream_t s);
    acb_status run(int S, cudaStream_t s);
};

acb_status acb_qwen3_enc::reserve(int R, int S, int per) {
    const size_t KD = (size_t) c.n_kv_heads * c.head_dim;
    if (R <= cap) {
        // V^T of ceil(cap / S) sequences of round8(S) columns, hi and lo planes
        const int    ld   = (S + 7) / 8 * 8;
        const size_t vneed = (size_t) 2 * KD * ld * 2 * ((cap + S - 1) / S);
        if (vneed > vtb.bytes) {
            drop_graphs();
            if (vtb.alloc(vneed) != ACB_OK) {
                cap = 0;
                set_last_error("encoder scratch allocation failed");
                return ACB_ERR_OOM;
            }
        }
        s_ld = ld;
        if (per != period) {
            // the positions of a captured graph (one sequence: rows 0..S-1) do not depend on the period
            std::vector<int32_t> p((size_t) cap);
            for (int i = 0; i < cap; i++) {
                p[(size_t) i] = per > 0 ? i % per : i;
            }
            if (cudaMemcpy(pos.p, p.data(), p.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess) {
                return ACB_ERR_CUDA;
            }
            period = per;
        }
        return ACB_OK;
    }
    drop_graphs();
    const int    n  = std::max({ R, cap, 256 });
    const size_t H  = (size_t) c.hidden_size, F = (size_t) c.intermediate_size;
    const size_t QD = (size_t) c.n_heads * c.head_dim;
    const size_t XQ = std::max({ H, QD, F });
    bool         bad = false;
    bad |= ids.alloc((size_t) n * 4) != ACB_OK;
    bad |= pos.alloc((size_t) n * 4, false) != ACB_OK;
    bad |= h.alloc((size_t) n * H * 4) != ACB_OK;
    bad |= xn.alloc((size_t) n * H * 4) != ACB_OK;
    bad |= xq.alloc((size_t) n * XQ * 3 * 2) != ACB_OK;
    bad |= qkv.alloc((size_t) n * nqkv() * 2) != ACB_OK;
    bad |= qkv32.alloc((size_t) n * nqkv() * 4) != ACB_OK;
    bad |= planes.alloc((size_t) n * (QD + KD) * 2 * 2) != ACB_OK;
    s_ld = (S + 7) / 8 * 8;
    bad |= vtb.alloc((size_t) 2 * KD * s_ld * 2 * ((n + S - 1) / S)) != ACB_OK;
    bad |= q.alloc((size_t) n * QD * 2) != ACB_OK;
    bad |= k.alloc((size_t) n * KD * 2) != ACB_OK;
    bad |= att.alloc((size_t) n * QD * 4) != ACB_OK;
    bad |= gu.alloc((size_t) n * 2 * F * 4) != ACB_OK;
    bad |= out.alloc((size_t) n * H * 4) != ACB_OK;
    bad |= rope.alloc((size_t) n * c.head_dim * 4, false) != ACB_OK;
    {
        // split-K workspace: the largest need over the four linears at every M tile count <= n
        size_t wsb = 0;
        for (int m = 128; m < n + 128; m += 128) {
            const int64_t M = std::min(m, n);
            for (int64_t km : { (int64_t) 1, (int64_t) 3 }) {
                wsb = std::max({ wsb, acb_gemm_workspace_bytes(M, nqkv(), km * H),
                                 acb_gemm_workspace_bytes(M, H, km * QD), acb_gemm_workspace_bytes(M, 2 * F, km * H),
                                 acb_gemm_workspace_bytes(M, H, km * F) });
            }
        }
        bad |= ws.alloc(wsb, true) != ACB_OK;  // the split-K ticket area starts at zero
    }
    if (!err.p) {
        bad |= err.alloc(4) != ACB_OK;
    }
    if (bad) {
        cap = 0;
        set_last_error("encoder scratch allocation failed");
        return ACB_ERR_OOM;
    }
    std::vector<int32_t> p((size_t) n);
    for (int i = 0; i < n; i++) {
        p[(size_t) i] = per > 0 ? i % per : i;  // positions 0..S-1 of every sequence (qwen3-enc.h:418-424)
    }
    std::vector<float> tab((size_t) n * c.head_dim);
    acb_rope_table_host(tab.data(), n, c.head_dim, c.rope_theta);
    if (cudaMemcpy(pos.p, p.data(), p.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(rope.p, tab.data(), tab.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    cap    = n;
    period = per;
    return ACB_OK;
}

// Layers [l0, l1) over the hidden states in `h` (qwen3_build_layers, qwen3-enc.h:249-262): B
// sequences of S rows each, attention within each sequence.
acb_status acb_qwen3_enc::enqueue_layers(int B, int S, int l0, int l1, cudaStream_t s) {
    const int          H = c.hidden_size, Nh = c.n_heads, Nkv = c.n_kv_heads, D = c.head_dim;
    const int          QD = Nh * D, KD = Nkv * D, NQKV = nqkv();
    const float        eps   = c.rms_norm_eps;
    const float        scale = 1.0f / sqrtf((float) D);
    const acb_stream_t as    = (acb_stream_t) s;
    const DenseScratch sc    = scratch();
    int *              e     = err.as<int>();
    float *            hp    = h.as<float>();
    const int          R     = B * S;
    for (int l = l0; l < l1; l++) {
        const EncLayer & L = layers[(size_t) l];
        // causal (text encoder), or bidirectional with the sliding window on even layers
        const int mask = c.is_causal ? 1 : ((window > 0 && l % 2 == 0 && S > window + 1) ? 2 : 0);
        // attention output straight into the output projection's operand when possible
        int        ao_type = ACB_TYPE_F32, ao_flags = 0;
        int64_t    ao_ts   = QD;
        void *     ao      = att.p;
        const bool fuse_o  = dense_operand_spec(L.o, exact, &ao_type, &ao_flags, &ao_ts);
        if (fuse_o) {
            ao = sc.xq;
        } else {
            ao_type  = ACB_TYPE_F32;
            ao_flags = 0;
            ao_ts    = QD;
        }
        // input_layernorm inside the qkv projection's activation producer
        NormSpec ns_in;
        ns_in.w   = (const float *) L.attn_norm->data;
        ns_in.eps = eps;
        if (Nh % 2 == 0 && Nkv % 2 == 0 && R >= qkv_fuse_min_rows()) {
            // qkv projection with q/k RMSNorm + RoPE and the V transpose in its epilogue
            const int64_t W  = QD + KD;
            const int64_t lo = exact ? (int64_t) cap * W : 0;
            const int64_t vl = exact ? (int64_t) B * KD * s_ld : 0;
            uint16_t *    hi = planes.as<uint16_t>();
            int64_t       Kp = 0;
            ACB_TRY(dense_operand(L.qkv, exact, hp, H, R, sc, s, &ns_in, &Kp));
            ACB_TRY(acb_gemm_qkv_planes(sc.xq, Kp, L.qkv.w, L.qkv.ldw, R, Kp, Nh, Nkv, (const float *) L.q_norm->data,
                                        (const float *) L.k_norm->data, eps, pos.as<int32_t>(), rope.as<float>(), cap,
                                        S, hi, W, lo, vtb.as<uint16_t>(), s_ld, vl, kPdl | L.qkv.op, e, as));
            ACB_TRY(acb_attn_tc(hi, W, hi + QD, W, vtb.p, s_ld, ao, ao_type, ao_ts, B, S, S, Nh, Nkv, D, mask, window, 0,
                                scale, kPdl | ao_flags, lo, lo, vl, e, as));
        } else if (exact) {
            float * q32 = qkv32.as<float>();
            ACB_TRY(dense_forward(L.qkv, true, hp, H, 0, R, q32, ACB_TYPE_F32, NQKV, nullptr, nullptr, 0, nullptr, 0,
                                  0, sc, s, &ns_in));
            // q/k norm + rope straight into hi/lo planes of Q||K, and V^T planes, for the
            // tensor-core attention
            const int64_t W  = QD + KD;
            const int64_t lo = (int64_t) cap * W;
            const int64_t vl = (int64_t) B * KD * s_ld;
            uint16_t *    hi = planes.as<uint16_t>();
            ACB_TRY(acb_qk_norm_rope_planes(q32, ACB_TYPE_F32, NQKV, hi, W, lo, R, Nh, (const float *) L.q_norm->data,
                                            Nkv, (const float *) L.k_norm->data, D, eps, pos.as<int32_t>(),
                                            rope.as<float>(), cap, e, as));
            ACB_TRY(acb_attn_vt(q32 + QD + KD, ACB_TYPE_F32, (int64_t) S * NQKV, NQKV, B, S, Nkv, D, vtb.p, s_ld, vl,
                                as));
            ACB_TRY(acb_attn_tc(hi, W, hi + QD, W, vtb.p, s_ld, ao, ao_type, ao_ts, B, S, S, Nh, Nkv, D, mask, window, 0,
                                scale, kPdl | ao_flags, lo, lo, vl, e, as));
        } else {
            ACB_TRY(dense_forward(L.qkv, false, hp, H, 0, R, qkv.p, ACB_TYPE_F16, NQKV, nullptr, nullptr, 0, nullptr, 0,
                                  0, sc, s, &ns_in));
            ACB_TRY(acb_qk_norm_rope(qkv.p, ACB_TYPE_F16, NQKV, q.p, ACB_TYPE_F16, QD, D, 0, R, Nh, D,
                                     (const float *) L.q_norm->data, eps, pos.as<int32_t>(), rope.as<float>(), cap, e,
                                     as));
            ACB_TRY(acb_qk_norm_rope(qkv.as<uint16_t>() + QD, ACB_TYPE_F16, NQKV, k.p, ACB_TYPE_F16, KD, D, 0, R, Nkv,
                                     D, (const float *) L.k_norm->data, eps, pos.as<int32_t>(), rope.as<float>(), cap,
                                     e, as));
            ACB_TRY(acb_attn_vt(qkv.as<uint16_t>() + QD + KD, ACB_TYPE_F16, (int64_t) S * NQKV, NQKV, B, S, Nkv, D,
                                vtb.p, s_ld, 0, as));
            ACB_TRY(acb_attn_tc(q.p, QD, k.p, KD, vtb.p, s_ld, ao, ao_type, ao_ts, B, S, S, Nh, Nkv, D, mask, window, 0,
                                scale, kPdl | ao_flags, 0, 0, 0, e, as));
        }
        if (fuse_o) {  // the attention wrote the output projection's operand
            ACB_TRY(dense_forward_operand(L.o, exact, R, hp, ACB_TYPE_F32, H, nullptr, hp, H, nullptr, 0, 0, sc, s));
        } else {
            ACB_TRY(dense_forward(L.o, exact, att.as<float>(), QD, 0, R, hp, ACB_TYPE_F32, H, nullptr, hp, H, nullptr, 0,
                                  0, sc, s));
        }
        // post_attention_layernorm inside the gate/up projection's producer
        NormSpec ns_post;
        ns_post.w   = (const float *) L.post_norm->data;
        ns_post.eps = eps;
        ACB_TRY(dense_ffn(L.gu, L.down, exact, hp, H, R, hp, H, hp, H, nullptr, 0, 0, gu.p, sc, s, &ns_post));
    }
    return ACB_OK;
}

// The whole forward for S tokens whose ids are already in `ids`; result in `out`.
acb_status acb_qwen3_enc::enqueue(int S, cudaStream_t s) {
    const int          H  = c.hidden_size;
    const acb_stream_t as = (acb_stream_t) s;
    ACB_TRY(acb_get_rows(embed->data, embed->type, embed->N, H, ids.as<int32_t>(), S, h.p, ACB_TYPE_F32, H,
                         err.as<int>(), as));
    ACB_TRY(enqueue_layers(S, 0, c.n_layers, s));
    return acb_rms_norm(h.p, ACB_TYPE_F32, H, (const float *) final_norm->data, out.p, ACB_TYPE_F32, H, S, H,
                        c.rms_norm_eps, as);
}

// Replay (capturing on first use) the graph for S on stream s.
acb_status acb_qwen3_enc::run(int S, cudaStream_t s) {
    const int key = S * 2 + (exact ? 1 : 0);
    auto      it  = graphs.find(key);
    if (it == graphs.end()) {
        cudaGraph_t g = nullptr;
        if (cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
            return ACB_ERR_CUDA;
        }
        const acb_status  es = enqueue(S, st);
        const cudaError_t ce = cudaStreamEndCapture(st, &g);
        if (es != ACB_OK || ce != cudaSuccess) {
            if (g) {
                cudaGraphDestroy(g);
            }
            set_last_error("encoder graph capture failed");
            return es != ACB_OK ? es : ACB_ERR_CUDA;
        }
        graph_kernels[key]   = graph_kernel_nodes(g);
        cudaGraphExec_t   ex = nullptr;
        const cudaError_t ie = cudaGraphInstantiate(&ex, g, 0);
        cudaGraphDestroy(g);
        if (ie != cudaSuccess) {
            set_last_error("encoder graph instantiation failed");
            return ACB_ERR_CUDA;
        }
        it = graphs.emplace(key, ex).first;
    }
    last_kernels = graph_kernels[key];
    return cudaGraphLaunch(it->second, s) == cudaSuccess ? ACB_OK : ACB_ERR_CUDA;
}

// ---- C ABI ---------------------------------------------------------------------------------------

namespace acb {

// A Qwen3 layer stack whose tensors are `prefix`layers.{i}.* and `prefix`norm.weight (with
// `prefix`embed_tokens.weight when with_embed): the text encoder (prefix "", qwen3-enc.h:319-360) and
// the stacks of the condition encoder and the FSQ (de)tokenizer (cond-enc.h:97-135,
// fsq-tok.h:86-112, fsq-detok.h:83-110), which share qwen3_load_layer.
acb_status enc_stack_load(GGUFFile & gf, const std::string & prefix, const acb_qwen3_config & cfg, int window,
                          bool with_embed, int device, acb_qwen3_enc ** out) {
    *out = nullptr;
    if (cudaSetDevice(device) != cudaSuccess) {
        set_last_error("cannot select CUDA device");
        return ACB_ERR_CUDA;
    }
    std::unique_ptr<acb_qwen3_enc> m(new acb_qwen3_enc());
    m->device            = device;
    m->window            = window;
    acb_qwen3_config & c = m->c;
    c                    = cfg;
    auto bad = [&](acb_status s, const std::string & msg) {
        set_last_error(msg);
        return s;
    };
    const int H = c.hidden_size, F = c.intermediate_size, D = c.head_dim;
    if (c.n_layers <= 0 || c.n_layers > 64 || D != 128 || c.n_kv_heads <= 0 || c.n_heads % c.n_kv_heads != 0 ||
        H % 256 != 0 || F % 256 != 0) {
        return bad(ACB_ERR_UNSUPPORTED, "unsupported encoder configuration");
    }
    if (cudaStreamCreateWithFlags(&m->st, cudaStreamNonBlocking) != cudaSuccess) {
        return bad(ACB_ERR_CUDA, "stream creation failed");
    }

    // Resident tensors: embedding and norms. Linears go through a staging arena that is freed
    // once their 16-bit copies exist.
    WeightArena & A     = m->arena;
    auto          stage = std::make_unique<WeightArena>();
    m->embed            = with_embed ? A.load(gf, prefix + "embed_tokens.weight") : nullptr;
    m->final_norm       = A.load_f32(gf, prefix + "norm.weight");
    struct Raw {
        std::vector<DevTensor *> qkv, gu;
        DevTensor *              o = nullptr, *down = nullptr;
    };
    std::vector<Raw> raw((size_t) c.n_layers);
    m->layers.resize((size_t) c.n_layers);
    const int QD = c.n_heads * D, KD = c.n_kv_heads * D;
    for (int i = 0; i < c.n_layers; i++) {
        const std::string p = prefix + "layers." + std::to_string(i);
        EncLayer &        L = m->layers[(size_t) i];
        Raw &             R = raw[(size_t) i];
        L.attn_norm         = A.load_f32(gf, p + ".input_layernorm.weight");
        L.post_norm         = A.load_f32(gf, p + ".post_attention_layernorm.weight");
        L.q_norm            = A.load_f32(gf, p + ".self_attn.q_norm.weight");
        L.k_norm            = A.load_f32(gf, p + ".self_attn.k_norm.weight");
        R.qkv  = { stage->load(gf, p + ".self_attn.q_proj.weight"), stage->load(gf, p + ".self_attn.k_proj.weight"),
                   stage->load(gf, p + ".self_attn.v_proj.weight") };
        R.o    = stage->load(gf, p + ".self_attn.o_proj.weight");
        R.gu   = { stage->load(gf, p + ".mlp.gate_proj.weight"), stage->load(gf, p + ".mlp.up_proj.weight") };
        R.down = stage->load(gf, p + ".mlp.down_proj.weight");
        bool ok = L.attn_norm && L.post_norm && L.q_norm && L.k_norm && R.o && R.down;
        for (DevTensor * t : R.qkv) {
            ok = ok && t && t->K == H;
        }
        for (DevTensor * t : R.gu) {
            ok = ok && t && t->K == H && t->N == F;
        }
        if (!ok) {
            return bad(ACB_ERR_FORMAT, !A.error.empty()      ? A.error :
                                       !stage->error.empty() ? stage->error :
                                                               "missing or misshapen layer tensor");
        }
        if (R.qkv[0]->N != QD || R.qkv[1]->N != KD || R.qkv[2]->N != KD || R.o->K != QD || R.o->N != H ||
            R.down->K != F || R.down->N != H || L.q_norm->K != D || L.k_norm->K != D || L.attn_norm->K != H) {
            return bad(ACB_ERR_FORMAT, "layer tensor shapes do not match the config");
        }
    }
    if ((with_embed && !m->embed) || !m->final_norm) {
        return bad(ACB_ERR_FORMAT, A.error.empty() ? "missing embedding or final norm" : A.error);
    }
    if (m->embed && m->embed->K != H) {
        return bad(ACB_ERR_FORMAT, "embed_tokens shape does not match the config");
    }
    c.vocab_size = m->embed ? (int) m->embed->N : 0;
    ACB_TRY(A.upload(m->st));
    ACB_TRY(stage->upload(m->st));

    // 16-bit copies ([hi | lo | hi] for quantised weights), every matrix on a 256-byte boundary
    size_t total = 0;
    for (const Raw & R : raw) {
        for (const std::vector<DevTensor *> & parts : { R.qkv, std::vector<DevTensor *>{ R.o }, R.gu,
                                                         std::vector<DevTensor *>{ R.down } }) {
            total += (DenseLinear::elems(parts) * 2 + 255) & ~size_t(255);
        }
    }
    if (m->w16.alloc(total, false) != ACB_OK) {
        return bad(ACB_ERR_OOM, "16-bit weight allocation failed");
    }
    DevBuf        idbuf, tmp;
    const int64_t max_rows = std::max<int64_t>({ (int64_t) QD, (int64_t) F, (int64_t) H });
    if (idbuf.alloc((size_t) max_rows * 4, false) != ACB_OK ||
        tmp.alloc((size_t) max_rows * std::max(H, std::max(F, QD)) * 4, false) != ACB_OK) {
        return bad(ACB_ERR_OOM, "conversion scratch allocation failed");
    }
    {
        std::vector<int32_t> idv((size_t) max_rows);
        for (int64_t r = 0; r < max_rows; r++) {
            idv[(size_t) r] = (int32_t) r;
        }
        if (cudaMemcpy(idbuf.p, idv.data(), idv.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess) {
            return bad(ACB_ERR_CUDA, "id upload failed");
        }
    }
    uint8_t * p = m->w16.as<uint8_t>();
    for (int i = 0; i < c.n_layers; i++) {
        EncLayer & L     = m->layers[(size_t) i];
        Raw &      R     = raw[(size_t) i];
        auto       place = [&](DenseLinear & D, const std::vector<DevTensor *> & parts) -> acb_status {
            ACB_TRY(dense_build(D, parts, reinterpret_cast<uint16_t *>(p), idbuf.as<int32_t>(), tmp.as<float>(),
                                m->st));
            p += (DenseLinear::elems(parts) * 2 + 255) & ~size_t(255);
            // the conversion scratch is reused by the next matrix
            return cudaStreamSynchronize(m->st) == cudaSuccess ? ACB_OK : ACB_ERR_CUDA;
        };
        ACB_TRY(place(L.qkv, R.qkv));
        ACB_TRY(place(L.o, { R.o }));
        ACB_TRY(place(L.gu, R.gu));
        ACB_TRY(place(L.down, { R.down }));
    }
    if (cudaStreamSynchronize(m->st) != cudaSuccess) {
        return bad(ACB_ERR_CUDA, "weight conversion failed");
    }
    stage.reset();
    ACB_TRY(m->reserve(256));
    *out = m.release();
    return ACB_OK;
}

float * enc_stack_input(acb_qwen3_enc * m, int B, int S, cudaStream_t s) {
    if (B <= 0 || S <= 0 || (int64_t) B * S > (1 << 30)) {
        set_last_error("encoder batch shape out of range");
        return nullptr;
    }
    // the positions are rewritten synchronously: nothing may still read them
    if (cudaStreamSynchronize(s) != cudaSuccess || cudaStreamSynchronize(m->st) != cudaSuccess) {
        return nullptr;
    }
    return m->reserve(B * S, S, B > 1 ? S : 0) == ACB_OK ? m->h.as<float>() : nullptr;
}

acb_status enc_stack_run(acb_qwen3_enc * m, int B, int S, float * d_out, int64_t ldo, cudaStream_t s) {
    ACB_TRY(m->enqueue_layers(B, S, 0, m->c.n_layers, s));
    const int H = m->c.hidden_size;
    return acb_rms_norm(m->h.p, ACB_TYPE_F32, H, (const float *) m->final_norm->data, d_out, ACB_TYPE_F32, ldo,
                        (int64_t) B * S, H, m->c.rms_norm_eps, (acb_stream_t) s);
}

int * enc_stack_err(acb_qwen3_enc * m) {
    return m->err.as<int>();
}

}  // namespace acb

extern "C" acb_status acb_qwen3_load_text_encoder(const char * gguf_path, int device, acb_qwen3_enc ** out) {
    if (!gguf_path || !out) {
        return ACB_ERR_INVALID_ARG;
    }
    *out = nullptr;
    GGUFFile gf;
    if (!gf.open(gguf_path)) {
        set_last_error(gf.error());
        return gf.error().rfind("cannot open", 0) == 0 ? ACB_ERR_IO : ACB_ERR_FORMAT;
    }
    acb_qwen3_config c = { 1024, 3072, 16, 8, 128, 28, 1000000.0f, 1e-6f, 1, 0 };  // qwen3-enc.h:327-337
    const char *     j = gf.get_str("acestep.config_json");
    if (j && j[0]) {
        c.hidden_size       = json_int(j, "hidden_size", c.hidden_size);
        c.intermediate_size = json_int(j, "intermediate_size", c.intermediate_size);
        c.n_heads           = json_int(j, "num_attention_heads", c.n_heads);
        c.n_kv_heads        = json_int(j, "num_key_value_heads", c.n_kv_heads);
        c.head_dim          = json_int(j, "head_dim", c.head_dim);
        c.n_layers          = json_int(j, "num_hidden_layers", c.n_layers);
        c.rope_theta        = json_float(j, "rope_theta", c.rope_theta);
        c.rms_norm_eps      = json_float(j, "rms_norm_eps", c.rms_norm_eps);
    }
    return enc_stack_load(gf, "", c, 0, true, device, out);
}

extern "C" acb_status acb_qwen3_set_exact(acb_qwen3_enc * m, int exact) {
    if (!m) {
        return ACB_ERR_INVALID_ARG;
    }
    m->exact = exact != 0;
    return ACB_OK;
}

extern "C" acb_status acb_qwen3_get_config(const acb_qwen3_enc * m, acb_qwen3_config * cfg) {
    if (!m || !cfg) {
        return ACB_ERR_INVALID_ARG;
    }
    *cfg = m->c;
    return ACB_OK;
}

extern "C" size_t acb_qwen3_weight_bytes(const acb_qwen3_enc * m) {
    return m ? m->arena.bytes() + m->w16.bytes : 0;
}

extern "C" acb_status acb_qwen3_forward_device(acb_qwen3_enc * m, const int32_t * d_ids, int S, float * d_out,
                                               acb_stream_t stream) {
    if (!m || !d_ids || !d_out || S <= 0) {
        return ACB_ERR_INVALID_ARG;
    }
    if (cudaSetDevice(m->device) != cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    ACB_TRY(m->reserve(S));
    cudaStream_t s = (cudaStream_t) stream;
    if (cudaMemcpyAsync(m->ids.p, d_ids, (size_t) S * 4, cudaMemcpyDeviceToDevice, s) != cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    ACB_TRY(m->run(S, s));
    const size_t ob = (size_t) S * m->c.hidden_size * 4;
    return cudaMemcpyAsync(d_out, m->out.p, ob, cudaMemcpyDeviceToDevice, s) == cudaSuccess ? ACB_OK : ACB_ERR_CUDA;
}

extern "C" int acb_qwen3_forward_kernels(const acb_qwen3_enc * m) {
    return m ? m->last_kernels : 0;
}

extern "C" acb_status acb_qwen3_forward_hidden(acb_qwen3_enc * m, const float * d_hidden, int S, int layer_begin,
                                               int layer_end, int final_norm, float * d_out, acb_stream_t stream) {
    if (!m || !d_hidden || !d_out || S <= 0 || layer_begin < 0 || layer_end > m->c.n_layers ||
        layer_begin > layer_end) {
        return ACB_ERR_INVALID_ARG;
    }
    if (cudaSetDevice(m->device) != cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    ACB_TRY(m->reserve(S));
    cudaStream_t s  = (cudaStream_t) stream;
    const size_t hb = (size_t) S * m->c.hidden_size * 4;
    if (cudaMemcpyAsync(m->h.p, d_hidden, hb, cudaMemcpyDeviceToDevice, s) != cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    ACB_TRY(m->enqueue_layers(S, layer_begin, layer_end, s));
    if (final_norm) {
        const int H = m->c.hidden_size;
        return acb_rms_norm(m->h.p, ACB_TYPE_F32, H, (const float *) m->final_norm->data, d_out, ACB_TYPE_F32, H, S, H,
                            m->c.rms_norm_eps, stream);
    }
    return cudaMemcpyAsync(d_out, m->h.p, hb, cudaMemcpyDeviceToDevice, s) == cudaSuccess ? ACB_OK : ACB_ERR_CUDA;
}

static acb_status check_ids(const acb_qwen3_enc * m, const int32_t * ids, int S) {
    for (int i = 0; i < S; i++) {
        if (ids[i] < 0 || ids[i] >= m->c.vocab_size) {
            set_last_error("token id outside the embedding table");
            return ACB_ERR_OUT_OF_RANGE;
        }
    }
    return ACB_OK;
}

extern "C" acb_status acb_qwen3_forward(acb_qwen3_enc * m, const int32_t * token_ids, int S, float * output) {
    if (!m || !token_ids || !output || S <= 0) {
        return ACB_ERR_INVALID_ARG;
    }
    ACB_TRY(check_ids(m, token_ids, S));
    if (cudaSetDevice(m->device) != cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    ACB_TRY(m->reserve(S));
    if (cudaMemcpyAsync(m->ids.p, token_ids, (size_t) S * 4, cudaMemcpyHostToDevice, m->st) != cudaSuccess ||
        cudaMemsetAsync(m->err.p, 0, 4, m->st) != cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    ACB_TRY(m->run(S, m->st));
    int          dev_err = 0;
    const size_t ob      = (size_t) S * m->c.hidden_size * 4;
    if (cudaMemcpyAsync(output, m->out.p, ob, cudaMemcpyDeviceToHost, m->st) != cudaSuccess ||
        cudaMemcpyAsync(&dev_err, m->err.p, 4, cudaMemcpyDeviceToHost, m->st) != cudaSuccess ||
        cudaStreamSynchronize(m->st) != cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    if (dev_err) {
        set_last_error("device error flag " + std::to_string(dev_err));
        return ACB_ERR_DEVICE;
    }
    return ACB_OK;
}

extern "C" acb_status acb_qwen3_embed_lookup(acb_qwen3_enc * m, const int32_t * token_ids, int S, float * output) {
    if (!m || !token_ids || !output || S <= 0) {
        return ACB_ERR_INVALID_ARG;
    }
    ACB_TRY(check_ids(m, token_ids, S));
    if (cudaSetDevice(m->device) != cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    ACB_TRY(m->reserve(S));
    const int H = m->c.hidden_size;
    if (cudaMemcpyAsync(m->ids.p, token_ids, (size_t) S * 4, cudaMemcpyHostToDevice, m->st) != cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    ACB_TRY(acb_get_rows(m->embed->data, m->embed->type, m->embed->N, H, m->ids.as<int32_t>(), S, m->out.p,
                         ACB_TYPE_F32, H, nullptr, (acb_stream_t) m->st));
    if (cudaMemcpyAsync(output, m->out.p, (size_t) S * H * 4, cudaMemcpyDeviceToHost, m->st) != cudaSuccess ||
        cudaStreamSynchronize(m->st) != cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    return ACB_OK;
}

extern "C" void acb_qwen3_free(acb_qwen3_enc * m) {
    delete m;
}
