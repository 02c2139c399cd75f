// dit.cpp -- the ACE-Step DiT flow-matching denoiser (src/dit.h, src/dit-graph.h,
// src/dit-sampler.h) on libacb kernels.
//
// One evaluation for Ng sequences of S = T / P patches (R = Ng * S rows):
//   timestep embeddings t and t - t_r -> temb, tproj; modulation vectors for every layer
//   proj_in (patchify is a reshape of [Ng][T][in_ch]) + bias                 -> h (f32 [R][H])
//   per layer (dit_ggml_build_layer, dit-graph.h:367-450):
//     adaLN(h, self_attn_norm, scale_sa, shift_sa) -> Q||K||V -> q/k norm + RoPE -> self
//       attention (sliding window on even layers) -> o_proj, epilogue h += o * gate_sa
//     RMSNorm(h, cross_attn_norm) -> q_proj -> q norm -> cross attention over the condition's
//       K/V (computed once per condition and cached per layer) -> o_proj, epilogue h += o
//     adaLN(h, mlp_norm, scale_ff, shift_ff) -> gate||up -> SwiGLU -> down, h += o * gate_ff
//   adaLN(h, norm_out, out_scale, out_shift) -> proj_out + bias -> velocity [Ng][T][out_ch]
// Linears are tensor-core GEMMs (dense.h; exact mode by default). The generate loop
// (dit_ggml_generate) runs each denoise step -- embeddings, every layer, CFG/APG, the solver
// update -- as one captured CUDA graph; the host only uploads t for the step (and, for the SDE
// solver, the step's fresh noise). Padding: per-slot real patch positions (sa_len) and real
// condition rows (ca_len) live in device arrays that the attention kernels read when they run.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <tuple>
#include <vector>

#include "../../include/acb_models.h"
#include "comm.h"
#include "adapter.h"
#include "dense.h"
#include "gguf.h"
#include "host_common.h"
#include "weights.h"

using namespace acb;

namespace {

struct DiTLayerW {
    DevTensor * sa_norm = nullptr, *sa_q_norm = nullptr, *sa_k_norm = nullptr;
    DevTensor * ca_norm = nullptr, *ca_q_norm = nullptr, *ca_k_norm = nullptr, *mlp_norm = nullptr;
    DenseLinear sa_qkv, sa_o, ca_q, ca_kv, ca_o, gu, down;
};

struct TembW {
    DenseLinear l1, l2, tp;
    DevTensor * b1 = nullptr, *b2 = nullptr, *btp = nullptr;
};

constexpr int kPdl = ACB_FLAG_PDL;

}  // namespace

struct DiTRun;

struct acb_dit {
    int            device = 0;
    acb_dit_config c{};
    cudaStream_t   st    = nullptr;
    bool           exact = true;

    WeightArena            arena;  // norms, biases, tables (F32), null condition
    DevBuf                 w16;    // every linear, 16-bit
    TembW                  te, te_r;
    DenseLinear            proj_in, cond, proj_out;
    DevTensor *            proj_in_b = nullptr, *cond_b = nullptr, *norm_out = nullptr, *oss = nullptr;
    DevTensor *            null_emb = nullptr;
    DevBuf                 proj_out_b;  // bias [out_ch] repeated over the P patch positions
    DevBuf                 sst;         // [L][6H]
    std::vector<DiTLayerW> layers;

    // per-shape scratch
    int    Ng = 0, S = 0, enc_S = 0;
    DevBuf tt, sinus, th1, th2, temb2, tproj2, ada, out_ss;
    DevBuf input, h, xn, xq, qkv32, qkv16, planes, vtb, q16, k16, att, gu, vel, pos, rope, ws, err;
    DevBuf enc_in, enc_h, kv32, kvcache;  // condition: raw [Ng][enc_S][H_enc], embedded, per-layer K / V^T planes
    DevBuf sa_len, ca_len;                // [Ng] real patch positions / condition rows per slot
    // cached condition of one layer: K hi, K lo ([Ng*enc_S][KD] each), V^T hi, V^T lo
    // ([Ng][Nkv][128][enc_ld] each)
    size_t k_plane = 0, vt_plane = 0, kv_layer_elems = 0;
    int    s_ld = 0, enc_ld = 0;  // V^T row lengths: sequence / condition rows rounded up to 8
    int    eval_kernels   = 0;            // kernel launches of one captured evaluation
    // generate
    DevBuf                          xt, vt, out, ra;
    DevBuf                          hist1, hist2;  // DPM++ 3M velocity history (previous, the one before)
    DevBuf                          noise;         // SDE with a host noise source: the step's fresh noise [N][T][out_ch]
    DevBuf                          step_seeds;    // SDE on the device generator: seed_b + step + 1 per track
    DevBuf                          vpair, xall;   // sharded: [cond, uncond] velocities; gathered x0
    std::unique_ptr<DiTRun>         job;           // the step-level job (acb_dit_job_*)
    acb_stork4_tables               stork_tab{};   // the caller's ROCK4 tables (acb_dit_set_stork4_tables)
    std::vector<int>                stork_ms;
    std::vector<double>             stork_fpa, stork_fpb, stork_recf;
    std::map<std::tuple<int, int, int, int, int, uint32_t>, cudaGraphExec_t> graphs;
    std::map<std::tuple<int, int, int, int, int, uint32_t>, int> graph_kernels;  // kernel nodes per graph
    int step_kernels = 0;  // kernel launches of the last denoise step run (its step graph(s))

    ~acb_dit();

    void drop_graphs() {
        for (auto & kv : graphs) {
            cudaGraphExecDestroy(kv.second);
        }
        graphs.clear();
    }

    int qd() const { return c.n_heads * c.head_dim; }
    int kvd() const { return c.n_kv_heads * c.head_dim; }
    int nqkv() const { return qd() + 2 * kvd(); }

    DenseScratch scratch() { return DenseScratch{ xq.p, ws.p, ws.bytes, err.as<int>() }; }

    acb_status reserve(int Ng_, int T, int enc_S_);
    acb_status timestep(cudaStream_t s);
    acb_status condition(cudaStream_t s);
    acb_status evaluate(int n_layers_run, cudaStream_t s);
    acb_status layer(int l, cudaStream_t s);
    // per-slot lengths for the Ng slots: real_S / real_enc_S of the first n slots (NULL: all real),
    // repeated over the slots after them (the CFG twins); enqueued on s
    acb_status set_lengths(const int * real_S, const int * real_enc_S, int n, cudaStream_t s);
};

acb_status acb_dit::set_lengths(const int * real_S, const int * real_enc_S, int n, cudaStream_t s) {
    if (Ng <= 0 || n <= 0) {
        return ACB_ERR_INVALID_ARG;
    }
    std::vector<int> v(2 * (size_t) Ng);
    for (int b = 0; b < Ng; b++) {
        v[(size_t) b]      = real_S ? std::max(0, std::min(real_S[b % n], S)) : S;
        v[(size_t) Ng + b] = real_enc_S ? std::max(0, std::min(real_enc_S[b % n], enc_S)) : enc_S;
    }
    // pageable source: the call returns once the values are staged, so v may go out of scope
    if (cudaMemcpyAsync(sa_len.p, v.data(), (size_t) Ng * 4, cudaMemcpyHostToDevice, s) != cudaSuccess ||
        cudaMemcpyAsync(ca_len.p, v.data() + Ng, (size_t) Ng * 4, cudaMemcpyHostToDevice, s) != cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    return ACB_OK;
}

// ---- scratch ---------------------------------------------------------------------------------------

acb_status acb_dit::reserve(int Ng_, int T, int enc_S_) {
    const int S_ = T / c.patch_size;
    if (Ng_ == Ng && S_ == S && enc_S_ == enc_S) {
        return ACB_OK;
    }
    drop_graphs();
    Ng = Ng_, S = S_, enc_S = enc_S_;
    const size_t R = (size_t) Ng * S, Re = (size_t) Ng * enc_S;
    const size_t H = c.hidden_size, F = c.intermediate_size, QD = qd(), KD = kvd(), NQKV = nqkv();
    const size_t in_ch = c.in_channels, P = c.patch_size, Oc = c.out_channels;
    const size_t XQ = 3 * std::max({ H, F, QD, in_ch * P, (size_t) c.enc_hidden_size, (size_t) 256 });
    bool         bad = false;
    auto         A   = [&](DevBuf & b, size_t bytes, bool zero = false) { bad |= b.alloc(bytes, zero) != ACB_OK; };
    A(tt, 64, true);
    A(sinus, 2 * 256 * 4);
    A(th1, 2 * H * 4);
    A(th2, 2 * H * 4);
    A(temb2, 2 * H * 4);
    A(tproj2, 2 * 6 * H * 4);
    A(ada, (size_t) c.n_layers * 6 * H * 4);
    A(out_ss, 2 * H * 4);
    A(input, R * in_ch * P * 4, true);
    A(h, R * H * 4);
    A(xn, R * H * 4);
    A(xq, std::max(R, Re) * XQ * 2);
    A(qkv32, R * NQKV * 4);
    A(qkv16, R * NQKV * 2);
    s_ld   = (S + 7) / 8 * 8;
    enc_ld = (enc_S + 7) / 8 * 8;
    A(planes, 2 * R * (QD + KD) * 2);
    A(vtb, 2 * (size_t) Ng * KD * s_ld * 2);
    A(q16, R * QD * 2);
    A(k16, R * KD * 2);
    A(att, R * QD * 4);
    A(gu, R * 2 * F * 4);
    A(vel, R * Oc * P * 4);
    A(enc_in, Re * c.enc_hidden_size * 4);
    A(enc_h, Re * H * 4);
    A(kv32, Re * 2 * KD * 4);
    k_plane        = Re * KD;
    vt_plane       = (size_t) Ng * KD * enc_ld;
    kv_layer_elems = 2 * (k_plane + vt_plane);
    A(kvcache, (size_t) c.n_layers * kv_layer_elems * 2);
    A(sa_len, (size_t) Ng * 4);
    A(ca_len, (size_t) Ng * 4);
    if (!err.p) {
        A(err, 4, true);
    }
    {
        // split-K workspace: the largest need over every linear at these row counts (x3 for exact)
        size_t  wsb = 0;
        int64_t Ms[3] = { (int64_t) R, (int64_t) Re, 1 };
        for (int64_t M : Ms) {
            for (int64_t km : { (int64_t) 1, (int64_t) 3 }) {
                for (auto nk : { std::make_pair(NQKV, H), std::make_pair(H, QD), std::make_pair(2 * F, H),
                                 std::make_pair(H, F), std::make_pair(2 * KD, H), std::make_pair(H, in_ch * P),
                                 std::make_pair(Oc * P, H), std::make_pair(H, (size_t) c.enc_hidden_size),
                                 std::make_pair(6 * H, H), std::make_pair(H, H), std::make_pair(H, (size_t) 256) }) {
                    wsb = std::max(wsb, acb_gemm_workspace_bytes(M, (int64_t) nk.first, km * (int64_t) nk.second));
                }
            }
        }
        A(ws, wsb, true);  // the split-K ticket area starts at zero
    }
    // positions 0..S-1 per sequence and the rope table
    {
        std::vector<int32_t> p(R);
        for (size_t i = 0; i < R; i++) {
            p[i] = (int32_t) (i % (size_t) S);
        }
        std::vector<float> tab((size_t) S * c.head_dim);
        acb_rope_table_host(tab.data(), S, c.head_dim, c.rope_theta);
        A(pos, R * 4);
        A(rope, tab.size() * 4);
        if (!bad && (cudaMemcpy(pos.p, p.data(), R * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
                     cudaMemcpy(rope.p, tab.data(), tab.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess)) {
            bad = true;
        }
    }
    if (bad) {
        Ng = S = enc_S = 0;
        set_last_error("DiT scratch allocation failed");
        return ACB_ERR_OOM;
    }
    // no padding until a caller sets lengths (blocking copies: the buffers are new)
    std::vector<int> v((size_t) Ng, S), ve((size_t) Ng, enc_S);
    if (cudaMemcpy(sa_len.p, v.data(), (size_t) Ng * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(ca_len.p, ve.data(), (size_t) Ng * 4, cudaMemcpyHostToDevice) != cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    return ACB_OK;
}

// ---- timestep embedding (dit_ggml_build_temb, dit-graph.h:81-117) -----------------------------------

acb_status acb_dit::timestep(cudaStream_t s) {
    const int          H  = c.hidden_size;
    const acb_stream_t as = (acb_stream_t) s;
    const DenseScratch sc = scratch();
    ACB_TRY(acb_dit_sinusoid(tt.as<float>(), 256, 10000, sinus.as<float>(), as));
    for (int r = 0; r < 2; r++) {
        const TembW & E   = r == 0 ? te : te_r;
        float *       x0  = sinus.as<float>() + r * 256;
        float *       a1  = th1.as<float>() + r * H;
        float *       a2  = th2.as<float>() + r * H;
        float *       emb = temb2.as<float>() + r * H;
        ACB_TRY(dense_forward(E.l1, exact, x0, 256, 0, 1, a1, ACB_TYPE_F32, H, (const float *) E.b1->data, nullptr, 0,
                              nullptr, 0, 0, sc, s));
        ACB_TRY(acb_silu(a1, a2, H, as));
        ACB_TRY(dense_forward(E.l2, exact, a2, H, 0, 1, emb, ACB_TYPE_F32, H, (const float *) E.b2->data, nullptr, 0,
                              nullptr, 0, 0, sc, s));
        ACB_TRY(acb_silu(emb, a2, H, as));
        ACB_TRY(dense_forward(E.tp, exact, a2, H, 0, 1, tproj2.as<float>() + r * 6 * H, ACB_TYPE_F32, 6 * H,
                              (const float *) E.btp->data, nullptr, 0, nullptr, 0, 0, sc, s));
    }
    return acb_dit_modulation(sst.as<float>(), tproj2.as<float>(), temb2.as<float>(), (const float *) oss->data,
                              c.n_layers, H, ada.as<float>(), out_ss.as<float>(), as);
}

// ---- condition: embedder and every layer's cross-attention K/V (constant across steps) -----------

acb_status acb_dit::condition(cudaStream_t s) {
    const int          H = c.hidden_size, KD = kvd(), D = c.head_dim;
    const int          Re = Ng * enc_S;
    const acb_stream_t as = (acb_stream_t) s;
    const DenseScratch sc = scratch();
    ACB_TRY(dense_forward(cond, exact, enc_in.as<float>(), c.enc_hidden_size, 0, Re, enc_h.p, ACB_TYPE_F32, H,
                          (const float *) cond_b->data, nullptr, 0, nullptr, 0, 0, sc, s));
    for (int l = 0; l < c.n_layers; l++) {
        const DiTLayerW & L  = layers[(size_t) l];
        float *           kv = kv32.as<float>();
        ACB_TRY(dense_forward(L.ca_kv, exact, enc_h.as<float>(), H, 0, Re, kv, ACB_TYPE_F32, 2 * KD, nullptr, nullptr,
                              0, nullptr, 0, 0, sc, s));
        // k RMSNorm (no rope for cross-attention, dit-graph.h:317-331), in place
        ACB_TRY(acb_qk_norm_rope(kv, ACB_TYPE_F32, 2 * KD, kv, ACB_TYPE_F32, 2 * KD, D, 0, Re, c.n_kv_heads, D,
                                 (const float *) L.ca_k_norm->data, c.rms_norm_eps, nullptr, nullptr, 0, err.as<int>(),
                                 as));
        uint16_t * kh = kvcache.as<uint16_t>() + (size_t) l * kv_layer_elems;
        ACB_TRY(acb_act_quant_ex(kv, 2 * KD, 0, Re, KD, ACB_TYPE_F16, ACB_LAYOUT_PLANES, kh, ACB_TYPE_F16, KD,
                                 (int64_t) k_plane, as));
        ACB_TRY(acb_attn_vt(kv + KD, ACB_TYPE_F32, (int64_t) enc_S * 2 * KD, 2 * KD, Ng, enc_S, c.n_kv_heads, D,
                            kh + 2 * k_plane, enc_ld, (int64_t) vt_plane, as));
    }
    return ACB_OK;
}

// ---- one layer (dit_ggml_build_layer, dit-graph.h:367-450) ----------------------------------------

acb_status acb_dit::layer(int l, cudaStream_t s) {
    const DiTLayerW &  L = layers[(size_t) l];
    const int          H = c.hidden_size, D = c.head_dim, Nh = c.n_heads, Nkv = c.n_kv_heads;
    const int          QD = qd(), KD = kvd(), NQKV = nqkv();
    const int          R = Ng * S;
    const float        eps   = c.rms_norm_eps;
    const float        scale = 1.0f / sqrtf((float) D);
    const acb_stream_t as    = (acb_stream_t) s;
    const DenseScratch sc    = scratch();
    int *              e     = err.as<int>();
    float *            hp    = h.as<float>();
    const float *      a     = ada.as<float>() + (size_t) l * 6 * H;
    const float *shift_sa = a, *scale_sa = a + H, *gate_sa = a + 2 * H;
    const float *shift_ff = a + 3 * H, *scale_ff = a + 4 * H, *gate_ff = a + 5 * H;
    // sliding window on even layers when the sequence is longer than the window (dit-sampler.h:253-282)
    const bool swa  = (l % 2 == 0) && c.sliding_window > 0 && S > c.sliding_window;
    const int  mask = swa ? 2 : 0;

    // attention output: straight into the output projection's operand (s.xq) when the epilogue can
    // quantise it, else f32 for acb_act_quant_ex
    int     ao_type = ACB_TYPE_F32, ao_flags = 0;
    int64_t ao_ts   = QD;
    void *  ao      = att.p;
    const bool fuse_o = dense_operand_spec(L.sa_o, exact, &ao_type, &ao_flags, &ao_ts);
    if (fuse_o) {
        ao = sc.xq;
    } else {
        ao_type = ACB_TYPE_F32;
        ao_flags = 0;
        ao_ts    = QD;
    }
    // self-attention: adaLN (norm1, shift/scale_msa) inside the qkv projection's activation producer
    NormSpec ns_sa;
    ns_sa.w               = (const float *) L.sa_norm->data;
    ns_sa.eps             = eps;
    ns_sa.scale           = scale_sa;
    ns_sa.shift           = shift_sa;
    ns_sa.rows_per_sample = R;
    if (Nh % 2 == 0 && Nkv % 2 == 0 && R >= qkv_fuse_min_rows()) {
        // qkv projection with q/k RMSNorm + RoPE and the V transpose in its epilogue: the hi (and,
        // exact, lo) planes of Q||K and of V^T for the tensor-core attention
        const int64_t W  = QD + KD;
        const int64_t lo = exact ? (int64_t) R * W : 0;
        uint16_t *    hi = planes.as<uint16_t>();
        const int64_t vl = exact ? (int64_t) Ng * KD * s_ld : 0;
        int64_t       Kp = 0;
        ACB_TRY(dense_operand(L.sa_qkv, exact, hp, H, R, sc, s, &ns_sa, &Kp));
        ACB_TRY(acb_gemm_qkv_planes(sc.xq, Kp, L.sa_qkv.w, L.sa_qkv.ldw, R, Kp, Nh, Nkv,
                                    (const float *) L.sa_q_norm->data, (const float *) L.sa_k_norm->data, eps,
                                    pos.as<int32_t>(), rope.as<float>(), S, S, hi, W, lo, vtb.as<uint16_t>(), s_ld, vl,
                                    kPdl | L.sa_qkv.op, e, as));
        ACB_TRY(acb_attn_tc_masked(hi, W, hi + QD, W, vtb.p, s_ld, ao, ao_type, ao_ts, Ng, S, S, Nh, Nkv, D, mask,
                                   c.sliding_window, 0, scale, kPdl | ao_flags, lo, lo, vl, sa_len.as<int>(),
                                   sa_len.as<int>(), e, as));
    } else if (exact) {
        float * q32 = qkv32.as<float>();
        ACB_TRY(dense_forward(L.sa_qkv, true, hp, H, 0, R, q32, ACB_TYPE_F32, NQKV, nullptr, nullptr, 0, nullptr, 0, 0,
                              sc, s, &ns_sa));
        // q/k RMSNorm + RoPE straight into hi/lo planes of Q||K, and V transposed into hi/lo
        // planes, for the tensor-core attention
        const int64_t W  = QD + KD;
        const int64_t lo = (int64_t) R * W;
        uint16_t *    hi = planes.as<uint16_t>();
        const int64_t vl = (int64_t) Ng * KD * s_ld;
        ACB_TRY(acb_qk_norm_rope_planes(q32, ACB_TYPE_F32, NQKV, hi, W, lo, R, Nh, (const float *) L.sa_q_norm->data,
                                        Nkv, (const float *) L.sa_k_norm->data, D, eps, pos.as<int32_t>(),
                                        rope.as<float>(), S, e, as));
        ACB_TRY(acb_attn_vt(q32 + QD + KD, ACB_TYPE_F32, (int64_t) S * NQKV, NQKV, Ng, S, Nkv, D, vtb.p, s_ld, vl, as));
        ACB_TRY(acb_attn_tc_masked(hi, W, hi + QD, W, vtb.p, s_ld, ao, ao_type, ao_ts, Ng, S, S, Nh, Nkv, D, mask,
                                   c.sliding_window, 0, scale, kPdl | ao_flags, lo, lo, vl, sa_len.as<int>(),
                                   sa_len.as<int>(), e, as));
    } else {
        uint16_t * q16p = qkv16.as<uint16_t>();
        ACB_TRY(dense_forward(L.sa_qkv, false, hp, H, 0, R, q16p, ACB_TYPE_F16, NQKV, nullptr, nullptr, 0, nullptr, 0,
                              0, sc, s, &ns_sa));
        ACB_TRY(acb_qk_norm_rope(q16p, ACB_TYPE_F16, NQKV, q16.p, ACB_TYPE_F16, QD, D, 0, R, Nh, D,
                                 (const float *) L.sa_q_norm->data, eps, pos.as<int32_t>(), rope.as<float>(), S, e,
                                 as));
        ACB_TRY(acb_qk_norm_rope(q16p + QD, ACB_TYPE_F16, NQKV, k16.p, ACB_TYPE_F16, KD, D, 0, R, Nkv, D,
                                 (const float *) L.sa_k_norm->data, eps, pos.as<int32_t>(), rope.as<float>(), S, e,
                                 as));
        ACB_TRY(acb_attn_vt(q16p + QD + KD, ACB_TYPE_F16, (int64_t) S * NQKV, NQKV, Ng, S, Nkv, D, vtb.p, s_ld, 0, as));
        ACB_TRY(acb_attn_tc_masked(q16.p, QD, k16.p, KD, vtb.p, s_ld, ao, ao_type, ao_ts, Ng, S, S, Nh, Nkv, D, mask,
                                   c.sliding_window, 0, scale, kPdl | ao_flags, 0, 0, 0, sa_len.as<int>(),
                                   sa_len.as<int>(), e, as));
    }
    if (fuse_o) {  // the attention wrote the output projection's operand
        ACB_TRY(dense_forward_operand(L.sa_o, exact, R, hp, ACB_TYPE_F32, H, nullptr, hp, H, gate_sa, 0, R, sc, s));
    } else {
        ACB_TRY(dense_forward(L.sa_o, exact, att.as<float>(), QD, 0, R, hp, ACB_TYPE_F32, H, nullptr, hp, H, gate_sa, 0,
                              R, sc, s));
    }

    // cross-attention over the cached condition K/V; norm2 inside the q projection's producer
    NormSpec ns_ca;
    ns_ca.w   = (const float *) L.ca_norm->data;
    ns_ca.eps = eps;
    // the query's RMSNorm (q_norm) into the attention operand planes: in the q projection's epilogue
    // (from 1024 rows), else through f32
    const bool cq_fused = Nh % 2 == 0 && R >= qkv_fuse_min_rows();
    float *    cq       = qkv32.as<float>();
    if (cq_fused) {
        int64_t Kp = 0;
        ACB_TRY(dense_operand(L.ca_q, exact, hp, H, R, sc, s, &ns_ca, &Kp));
        ACB_TRY(acb_gemm_qkv_planes(sc.xq, Kp, L.ca_q.w, L.ca_q.ldw, R, Kp, Nh, 0, (const float *) L.ca_q_norm->data,
                                    nullptr, eps, nullptr, nullptr, 0, R, planes.as<uint16_t>(), QD,
                                    exact ? (int64_t) R * QD : 0, nullptr, 0, 0, kPdl | L.ca_q.op, e, as));
    } else {
        ACB_TRY(dense_forward(L.ca_q, exact, hp, H, 0, R, cq, ACB_TYPE_F32, QD, nullptr, nullptr, 0, nullptr, 0, 0, sc,
                              s, &ns_ca));
    }
    int     co_type = ACB_TYPE_F32, co_flags = 0;
    int64_t co_ts   = QD;
    void *  co      = att.p;
    const bool fuse_co = dense_operand_spec(L.ca_o, exact, &co_type, &co_flags, &co_ts);
    if (fuse_co) {
        co = sc.xq;
    } else {
        co_type  = ACB_TYPE_F32;
        co_flags = 0;
        co_ts    = QD;
    }
    const uint16_t * k_hi  = kvcache.as<uint16_t>() + (size_t) l * kv_layer_elems;
    const uint16_t * vt_hi = k_hi + 2 * k_plane;
    if (exact) {
        const int64_t lo = (int64_t) R * QD;
        uint16_t *    qh = planes.as<uint16_t>();
        if (!cq_fused) {
            ACB_TRY(acb_qk_norm_rope_planes(cq, ACB_TYPE_F32, QD, qh, QD, lo, R, Nh, (const float *) L.ca_q_norm->data,
                                            0, nullptr, D, eps, nullptr, nullptr, 0, e, as));
        }
        ACB_TRY(acb_attn_tc_masked(qh, QD, k_hi, KD, vt_hi, enc_ld, co, co_type, co_ts, Ng, S, enc_S, Nh, Nkv, D, 0,
                                   0, 0, scale, kPdl | co_flags, lo, (int64_t) k_plane, (int64_t) vt_plane, nullptr,
                                   ca_len.as<int>(), e, as));
    } else {
        uint16_t * q16p = cq_fused ? planes.as<uint16_t>() : q16.as<uint16_t>();
        if (!cq_fused) {
            ACB_TRY(acb_qk_norm_rope(cq, ACB_TYPE_F32, QD, q16.p, ACB_TYPE_F16, QD, D, 0, R, Nh, D,
                                     (const float *) L.ca_q_norm->data, eps, nullptr, nullptr, 0, e, as));
        }
        ACB_TRY(acb_attn_tc_masked(q16p, QD, k_hi, KD, vt_hi, enc_ld, co, co_type, co_ts, Ng, S, enc_S, Nh, Nkv, D,
                                   0, 0, 0, scale, kPdl | co_flags, 0, 0, 0, nullptr, ca_len.as<int>(), e, as));
    }
    if (fuse_co) {
        ACB_TRY(dense_forward_operand(L.ca_o, exact, R, hp, ACB_TYPE_F32, H, nullptr, hp, H, nullptr, 0, 0, sc, s));
    } else {
        ACB_TRY(dense_forward(L.ca_o, exact, att.as<float>(), QD, 0, R, hp, ACB_TYPE_F32, H, nullptr, hp, H, nullptr, 0,
                              0, sc, s));
    }

    // FFN: adaLN (norm3, shift/scale_mlp) inside the gate/up projection's producer
    NormSpec ns_ff = ns_sa;
    ns_ff.w        = (const float *) L.mlp_norm->data;
    ns_ff.scale    = scale_ff;
    ns_ff.shift    = shift_ff;
    return dense_ffn(L.gu, L.down, exact, hp, H, R, hp, H, hp, H, gate_ff, 0, R, gu.p, sc, s, &ns_ff);
}

// ---- one evaluation: input [Ng][T][in_ch] in `input` -> velocity in `vel` ---------------------------

acb_status acb_dit::evaluate(int n_layers_run, cudaStream_t s) {
    const int          H = c.hidden_size, R = Ng * S, KP = c.in_channels * c.patch_size;
    const DenseScratch sc = scratch();
    ACB_TRY(timestep(s));
    ACB_TRY(dense_forward(proj_in, exact, input.as<float>(), KP, 0, R, h.p, ACB_TYPE_F32, H,
                          (const float *) proj_in_b->data, nullptr, 0, nullptr, 0, 0, sc, s));
    const int nl = n_layers_run < 0 || n_layers_run > c.n_layers ? c.n_layers : n_layers_run;
    for (int l = 0; l < nl; l++) {
        ACB_TRY(layer(l, s));
    }
    const float * o = out_ss.as<float>();
    NormSpec      ns;
    ns.w               = (const float *) norm_out->data;
    ns.eps             = c.rms_norm_eps;
    ns.scale           = o + H;
    ns.shift           = o;
    ns.rows_per_sample = R;
    const int NO = c.out_channels * c.patch_size;
    return dense_forward(proj_out, exact, h.as<float>(), H, 0, R, vel.p, ACB_TYPE_F32, NO, proj_out_b.as<float>(),
                         nullptr, 0, nullptr, 0, 0, sc, s, &ns);
}

// ---- loading (dit_ggml_load, src/dit.h:256-420) -----------------------------------------------------

namespace {

// GGUF conv weight [H][ch][P] (ggml ne = [P, ch, H]) to a pre-permuted F32 GEMM weight:
// proj_in  rows h, element j = p*ch + c  (dit_load_proj_in_w, dit.h:142-195);
// proj_out rows j = p*ch + c, element h  (dit_load_proj_out_w, dit.h:197-252).
bool conv_to_f32(const GGUFFile & gf, const std::string & name, int H, int ch, int P, bool out_side,
                 std::vector<float> & dst) {
    const GGUFTensor * t = gf.find(name);
    if (!t || t->ne[0] * t->ne[1] * t->ne[2] * t->ne[3] != (int64_t) H * ch * P) {
        return false;
    }
    auto rd = [&](int64_t i) -> float {
        const uint8_t * p = static_cast<const uint8_t *>(t->data);
        uint16_t        v;
        switch (t->type) {
            case ACB_TYPE_F32: {
                float f;
                memcpy(&f, p + 4 * i, 4);
                return f;
            }
            case ACB_TYPE_F16:
                memcpy(&v, p + 2 * i, 2);
                return host_f16_to_f32(v);
            case ACB_TYPE_BF16:
                memcpy(&v, p + 2 * i, 2);
                return host_bf16_to_f32(v);
            default:
                return NAN;
        }
    };
    if (t->type != ACB_TYPE_F32 && t->type != ACB_TYPE_F16 && t->type != ACB_TYPE_BF16) {
        return false;
    }
    dst.resize((size_t) H * ch * P);
    for (int hh = 0; hh < H; hh++) {
        for (int cc = 0; cc < ch; cc++) {
            for (int p = 0; p < P; p++) {
                const float v = rd((int64_t) hh * P * ch + (int64_t) cc * P + p);
                if (out_side) {
                    dst[((size_t) p * ch + cc) * H + hh] = v;
                } else {
                    dst[(size_t) hh * ch * P + (size_t) p * ch + cc] = v;
                }
            }
        }
    }
    return true;
}

}  // namespace

extern "C" acb_status acb_dit_load(const char * gguf_path, int device, acb_dit ** out) {
    return acb_dit_load_ex(gguf_path, device, nullptr, 1.0f, out);
}

extern "C" acb_status acb_dit_load_ex(const char * gguf_path, int device, const char * adapter_path,
                                      float adapter_scale, acb_dit ** out) {
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
    std::unique_ptr<acb_dit> m(new acb_dit());
    m->device         = device;
    acb_dit_config & c = m->c;
    c.n_layers          = (int) gf.get_u32("acestep-dit.block_count");
    c.hidden_size       = (int) gf.get_u32("acestep-dit.embedding_length");
    c.intermediate_size = (int) gf.get_u32("acestep-dit.feed_forward_length");
    c.n_heads           = (int) gf.get_u32("acestep-dit.attention.head_count");
    c.n_kv_heads        = (int) gf.get_u32("acestep-dit.attention.head_count_kv");
    c.head_dim          = (int) gf.get_u32("acestep-dit.attention.key_length");
    c.in_channels       = (int) gf.get_u32("acestep.in_channels");
    c.out_channels      = (int) gf.get_u32("acestep.audio_acoustic_hidden_dim");
    c.patch_size        = (int) gf.get_u32("acestep.patch_size");
    c.sliding_window    = (int) gf.get_u32("acestep.sliding_window");
    c.rope_theta        = gf.get_f32("acestep-dit.rope.freq_base");
    c.rms_norm_eps      = gf.get_f32("acestep-dit.attention.layer_norm_rms_epsilon");
    auto bad = [&](acb_status s, const std::string & msg) {
        set_last_error(msg);
        return s;
    };
    // dit.h:289-296: every field must be present
    if (!c.n_layers || !c.hidden_size || !c.intermediate_size || !c.n_heads || !c.n_kv_heads || !c.head_dim ||
        !c.in_channels || !c.out_channels || !c.patch_size || !c.sliding_window || c.rope_theta <= 0.0f ||
        c.rms_norm_eps <= 0.0f) {
        return bad(ACB_ERR_FORMAT, "incomplete DiT config in GGUF");
    }
    const int H = c.hidden_size, F = c.intermediate_size, D = c.head_dim;
    if (D != 128 || c.n_heads % c.n_kv_heads != 0 || H % 256 != 0 || F % 256 != 0 || c.n_layers > 128 ||
        (c.in_channels * c.patch_size) % 64 != 0 || c.out_channels <= 0 || c.in_channels <= c.out_channels) {
        return bad(ACB_ERR_UNSUPPORTED, "unsupported DiT configuration");
    }
    if (cudaStreamCreateWithFlags(&m->st, cudaStreamNonBlocking) != cudaSuccess) {
        return bad(ACB_ERR_CUDA, "stream creation failed");
    }

    WeightArena & A     = m->arena;
    auto          stage = std::make_unique<WeightArena>();
    auto          req   = [&](DevTensor * t) { return t != nullptr; };
    bool          ok    = true;
    // timestep embedders
    struct TembRaw {
        DevTensor *l1 = nullptr, *l2 = nullptr, *tp = nullptr;
    } tr[2];
    for (int r = 0; r < 2; r++) {
        const std::string p = r == 0 ? "decoder.time_embed" : "decoder.time_embed_r";
        TembW &           E = r == 0 ? m->te : m->te_r;
        tr[r].l1            = stage->load(gf, p + ".linear_1.weight");
        tr[r].l2            = stage->load(gf, p + ".linear_2.weight");
        tr[r].tp            = stage->load(gf, p + ".time_proj.weight");
        E.b1                = A.load_f32(gf, p + ".linear_1.bias");
        E.b2                = A.load_f32(gf, p + ".linear_2.bias");
        E.btp               = A.load_f32(gf, p + ".time_proj.bias");
        ok = ok && req(tr[r].l1) && req(tr[r].l2) && req(tr[r].tp) && req(E.b1) && req(E.b2) && req(E.btp);
    }
    // proj_in / proj_out, pre-permuted on the host
    const int          P = c.patch_size, in_ch = c.in_channels, Oc = c.out_channels;
    std::vector<float> pin, pout;
    if (!conv_to_f32(gf, "decoder.proj_in.1.weight", H, in_ch, P, false, pin) ||
        !conv_to_f32(gf, "decoder.proj_out.1.weight", H, Oc, P, true, pout)) {
        return bad(ACB_ERR_FORMAT, "decoder.proj_in / proj_out weight missing or of an unsupported type");
    }
    DevTensor * pin_t  = stage->add_host(ACB_TYPE_F32, (int64_t) in_ch * P, H, pin.data(), pin.size() * 4);
    DevTensor * pout_t = stage->add_host(ACB_TYPE_F32, H, (int64_t) Oc * P, pout.data(), pout.size() * 4);
    m->proj_in_b       = A.load_f32(gf, "decoder.proj_in.1.bias");
    DevTensor * pob    = A.load_f32(gf, "decoder.proj_out.1.bias");
    DevTensor * cond_w = stage->load(gf, "decoder.condition_embedder.weight");
    m->cond_b          = A.load_f32(gf, "decoder.condition_embedder.bias");
    m->norm_out        = A.load_f32(gf, "decoder.norm_out.weight");
    m->oss             = A.load_f32(gf, "decoder.scale_shift_table");
    m->null_emb        = gf.find("null_condition_emb") ? A.load_f32(gf, "null_condition_emb") : nullptr;
    ok = ok && req(m->proj_in_b) && req(pob) && req(cond_w) && req(m->cond_b) && req(m->norm_out) && req(m->oss);
    if (!ok) {
        return bad(ACB_ERR_FORMAT, !A.error.empty() ? A.error : stage->error);
    }
    c.enc_hidden_size = (int) cond_w->K;
    if (cond_w->N != H || pob->K * pob->N != Oc || m->oss->K * m->oss->N != 2 * H || c.enc_hidden_size % 256 != 0) {
        return bad(ACB_ERR_FORMAT, "DiT input/output tensor shapes do not match the config");
    }
    // layers
    struct LRaw {
        std::vector<DevTensor *> sa_qkv, ca_q, ca_kv, gu;
        DevTensor *              sa_o = nullptr, *ca_o = nullptr, *down = nullptr, *sst = nullptr;
    };
    std::vector<LRaw> raw((size_t) c.n_layers);
    m->layers.resize((size_t) c.n_layers);
    const int QD = c.n_heads * D, KD = c.n_kv_heads * D;
    for (int i = 0; i < c.n_layers; i++) {
        const std::string p = "decoder.layers." + std::to_string(i);
        DiTLayerW &       L = m->layers[(size_t) i];
        LRaw &            R = raw[(size_t) i];
        L.sa_norm           = A.load_f32(gf, p + ".self_attn_norm.weight");
        L.sa_q_norm         = A.load_f32(gf, p + ".self_attn.q_norm.weight");
        L.sa_k_norm         = A.load_f32(gf, p + ".self_attn.k_norm.weight");
        L.ca_norm           = A.load_f32(gf, p + ".cross_attn_norm.weight");
        L.ca_q_norm         = A.load_f32(gf, p + ".cross_attn.q_norm.weight");
        L.ca_k_norm         = A.load_f32(gf, p + ".cross_attn.k_norm.weight");
        L.mlp_norm          = A.load_f32(gf, p + ".mlp_norm.weight");
        R.sst               = stage->load_f32(gf, p + ".scale_shift_table");
        R.sa_qkv = { stage->load(gf, p + ".self_attn.q_proj.weight"), stage->load(gf, p + ".self_attn.k_proj.weight"),
                     stage->load(gf, p + ".self_attn.v_proj.weight") };
        R.sa_o   = stage->load(gf, p + ".self_attn.o_proj.weight");
        R.ca_q   = { stage->load(gf, p + ".cross_attn.q_proj.weight") };
        R.ca_kv  = { stage->load(gf, p + ".cross_attn.k_proj.weight"), stage->load(gf, p + ".cross_attn.v_proj.weight") };
        R.ca_o   = stage->load(gf, p + ".cross_attn.o_proj.weight");
        R.gu     = { stage->load(gf, p + ".mlp.gate_proj.weight"), stage->load(gf, p + ".mlp.up_proj.weight") };
        R.down   = stage->load(gf, p + ".mlp.down_proj.weight");
        bool lok = L.sa_norm && L.sa_q_norm && L.sa_k_norm && L.ca_norm && L.ca_q_norm && L.ca_k_norm && L.mlp_norm &&
                   R.sst && R.sa_o && R.ca_o && R.down;
        for (auto * v : { &R.sa_qkv, &R.ca_q, &R.ca_kv, &R.gu }) {
            for (DevTensor * t : *v) {
                lok = lok && t && t->K == H;
            }
        }
        if (!lok) {
            return bad(ACB_ERR_FORMAT, !A.error.empty()      ? A.error :
                                       !stage->error.empty() ? stage->error :
                                                               "missing or misshapen DiT layer tensor");
        }
        if (R.sa_qkv[0]->N != QD || R.sa_qkv[1]->N != KD || R.sa_qkv[2]->N != KD || R.ca_q[0]->N != QD ||
            R.ca_kv[0]->N != KD || R.ca_kv[1]->N != KD || R.gu[0]->N != F || R.gu[1]->N != F || R.sa_o->K != QD ||
            R.sa_o->N != H || R.ca_o->K != QD || R.ca_o->N != H || R.down->K != F || R.down->N != H ||
            R.sst->K * R.sst->N != 6 * H || L.sa_q_norm->K != D) {
            return bad(ACB_ERR_FORMAT, "DiT layer tensor shapes do not match the config");
        }
    }
    ACB_TRY(A.upload(m->st));
    ACB_TRY(stage->upload(m->st));
    if (adapter_path) {
        // LoRA merged into the staged decoder weights before their resident copies exist
        int merged = 0;
        const acb_status as = adapter_merge(adapter_path, adapter_scale, *stage, m->st, &merged);
        if (as != ACB_OK) {
            const std::string why = acb_last_error();
            return bad(as, why);
        }
    }

    // proj_out bias repeated over the patch positions (ggml_add broadcast of [out_ch] over out_ch*P)
    {
        if (m->proj_out_b.alloc((size_t) Oc * P * 4, false) != ACB_OK) {
            return bad(ACB_ERR_OOM, "bias allocation failed");
        }
        for (int p = 0; p < P; p++) {
            cudaMemcpy(m->proj_out_b.as<float>() + p * Oc, pob->data, (size_t) Oc * 4, cudaMemcpyDeviceToDevice);
        }
        if (m->sst.alloc((size_t) c.n_layers * 6 * H * 4, false) != ACB_OK) {
            return bad(ACB_ERR_OOM, "modulation table allocation failed");
        }
        for (int i = 0; i < c.n_layers; i++) {
            cudaMemcpy(m->sst.as<float>() + (size_t) i * 6 * H, raw[(size_t) i].sst->data, (size_t) 6 * H * 4,
                       cudaMemcpyDeviceToDevice);
        }
    }

    // 16-bit copies of every linear
    std::vector<std::pair<DenseLinear *, std::vector<DevTensor *>>> lins;
    for (int r = 0; r < 2; r++) {
        TembW & E = r == 0 ? m->te : m->te_r;
        lins.push_back({ &E.l1, { tr[r].l1 } });
        lins.push_back({ &E.l2, { tr[r].l2 } });
        lins.push_back({ &E.tp, { tr[r].tp } });
    }
    lins.push_back({ &m->proj_in, { pin_t } });
    lins.push_back({ &m->proj_out, { pout_t } });
    lins.push_back({ &m->cond, { cond_w } });
    for (int i = 0; i < c.n_layers; i++) {
        DiTLayerW & L = m->layers[(size_t) i];
        LRaw &      R = raw[(size_t) i];
        lins.push_back({ &L.sa_qkv, R.sa_qkv });
        lins.push_back({ &L.sa_o, { R.sa_o } });
        lins.push_back({ &L.ca_q, R.ca_q });
        lins.push_back({ &L.ca_kv, R.ca_kv });
        lins.push_back({ &L.ca_o, { R.ca_o } });
        lins.push_back({ &L.gu, R.gu });
        lins.push_back({ &L.down, { R.down } });
    }
    size_t  total = 0;
    int64_t max_rows = 0, max_elems = 0;
    for (auto & lp : lins) {
        total += (DenseLinear::elems(lp.second) * 2 + 255) & ~size_t(255);
        for (DevTensor * t : lp.second) {
            max_rows  = std::max(max_rows, t->N);
            max_elems = std::max(max_elems, t->N * t->K);
        }
    }
    DevBuf idbuf, tmp;
    if (m->w16.alloc(total, false) != ACB_OK || idbuf.alloc((size_t) max_rows * 4, false) != ACB_OK ||
        tmp.alloc((size_t) max_elems * 4, false) != ACB_OK) {
        return bad(ACB_ERR_OOM, "16-bit weight allocation failed");
    }
    {
        std::vector<int32_t> idv((size_t) max_rows);
        for (int64_t r = 0; r < max_rows; r++) {
            idv[(size_t) r] = (int32_t) r;
        }
        cudaMemcpy(idbuf.p, idv.data(), idv.size() * 4, cudaMemcpyHostToDevice);
    }
    uint8_t * wp = m->w16.as<uint8_t>();
    for (auto & lp : lins) {
        ACB_TRY(dense_build(*lp.first, lp.second, reinterpret_cast<uint16_t *>(wp), idbuf.as<int32_t>(),
                            tmp.as<float>(), m->st));
        wp += (DenseLinear::elems(lp.second) * 2 + 255) & ~size_t(255);
        if (cudaStreamSynchronize(m->st) != cudaSuccess) {  // tmp is reused by the next matrix
            return bad(ACB_ERR_CUDA, "weight conversion failed");
        }
    }
    stage.reset();
    c.has_null_condition = m->null_emb ? 1 : 0;
    *out                 = m.release();
    return ACB_OK;
}

// ---- C ABI ---------------------------------------------------------------------------------------

extern "C" acb_status acb_dit_get_config(const acb_dit * m, acb_dit_config * cfg) {
    if (!m || !cfg) {
        return ACB_ERR_INVALID_ARG;
    }
    *cfg = m->c;
    return ACB_OK;
}

extern "C" acb_status acb_dit_set_exact(acb_dit * m, int exact) {
    if (!m) {
        return ACB_ERR_INVALID_ARG;
    }
    if (m->exact != (exact != 0)) {
        m->exact = exact != 0;
        m->drop_graphs();
    }
    return ACB_OK;
}

extern "C" size_t acb_dit_weight_bytes(const acb_dit * m) {
    return m ? m->arena.bytes() + m->w16.bytes : 0;
}

extern "C" acb_status acb_dit_forward(acb_dit * m, const float * d_input, const float * d_enc, int N, int T, int enc_S,
                                      float t, float t_r, float * d_velocity, int n_layers_run, acb_stream_t stream) {
    if (!m || !d_input || !d_enc || !d_velocity || N <= 0 || T <= 0 || enc_S <= 0 || T % m->c.patch_size != 0) {
        return ACB_ERR_INVALID_ARG;
    }
    if (cudaSetDevice(m->device) != cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    ACB_TRY(m->reserve(N, T, enc_S));
    cudaStream_t  s  = (cudaStream_t) stream;
    const float   tv[3] = { t, t_r, 0.0f };
    const size_t  nin = (size_t) N * T * m->c.in_channels * 4;
    const size_t  nen = (size_t) N * enc_S * m->c.enc_hidden_size * 4;
    if (cudaMemcpyAsync(m->tt.p, tv, sizeof(tv), cudaMemcpyHostToDevice, s) != cudaSuccess ||
        cudaMemcpyAsync(m->input.p, d_input, nin, cudaMemcpyDeviceToDevice, s) != cudaSuccess ||
        cudaMemcpyAsync(m->enc_in.p, d_enc, nen, cudaMemcpyDeviceToDevice, s) != cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    ACB_TRY(m->set_lengths(nullptr, nullptr, N, s));
    ACB_TRY(m->condition(s));
    ACB_TRY(m->evaluate(n_layers_run, s));
    const size_t nv = (size_t) N * T * m->c.out_channels * 4;
    if (cudaMemcpyAsync(d_velocity, m->vel.p, nv, cudaMemcpyDeviceToDevice, s) != cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    // tt must outlive the async copy: synchronise before returning the stack array
    return cudaStreamSynchronize(s) == cudaSuccess ? ACB_OK : ACB_ERR_CUDA;
}

extern "C" acb_status acb_dit_set_condition(acb_dit * m, const float * d_enc, int N, int T, int enc_S,
                                            acb_stream_t stream) {
    if (!m || !d_enc || N <= 0 || T <= 0 || enc_S <= 0 || T % m->c.patch_size != 0) {
        return ACB_ERR_INVALID_ARG;
    }
    if (cudaSetDevice(m->device) != cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    ACB_TRY(m->reserve(N, T, enc_S));
    cudaStream_t s   = (cudaStream_t) stream;
    const size_t nen = (size_t) N * enc_S * m->c.enc_hidden_size * 4;
    if (cudaMemcpyAsync(m->enc_in.p, d_enc, nen, cudaMemcpyDeviceToDevice, s) != cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    ACB_TRY(m->set_lengths(nullptr, nullptr, N, s));
    return m->condition(s);
}

extern "C" acb_status acb_dit_set_lengths(acb_dit * m, const int * real_S, const int * real_enc_S,
                                          acb_stream_t stream) {
    if (!m || m->Ng <= 0) {
        return ACB_ERR_INVALID_ARG;
    }
    if (cudaSetDevice(m->device) != cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    return m->set_lengths(real_S, real_enc_S, m->Ng, (cudaStream_t) stream);
}

extern "C" acb_status acb_dit_eval(acb_dit * m, const float * d_input, const float * tt, float * d_velocity,
                                   acb_stream_t stream) {
    if (!m || !d_input || !tt || !d_velocity || m->Ng <= 0) {
        return ACB_ERR_INVALID_ARG;
    }
    if (cudaSetDevice(m->device) != cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    cudaStream_t  s   = (cudaStream_t) stream;
    const int     T   = m->S * m->c.patch_size;
    const size_t  nin = (size_t) m->Ng * T * m->c.in_channels * 4;
    const size_t  nv  = (size_t) m->Ng * T * m->c.out_channels * 4;
    // the evaluation chain for this shape is one graph over the model's buffers
    const auto key = std::make_tuple(m->Ng * 100000 + T, m->enc_S, 2, 0, m->exact ? 1 : 0, 0u);
    auto       it  = m->graphs.find(key);
    if (it == m->graphs.end()) {
        cudaGraph_t g = nullptr;
        if (cudaStreamBeginCapture(m->st, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
            return ACB_ERR_CUDA;
        }
        const acb_status  es = m->evaluate(-1, m->st);
        const cudaError_t ce = cudaStreamEndCapture(m->st, &g);
        if (es != ACB_OK || ce != cudaSuccess) {
            if (g) {
                cudaGraphDestroy(g);
            }
            set_last_error("DiT evaluation graph capture failed");
            return es != ACB_OK ? es : ACB_ERR_CUDA;
        }
        size_t n_nodes = 0;  // every node of the evaluation graph is one of this library's kernels
        cudaGraphGetNodes(g, nullptr, &n_nodes);
        m->eval_kernels      = (int) n_nodes;
        cudaGraphExec_t   ex = nullptr;
        const cudaError_t ie = cudaGraphInstantiate(&ex, g, 0);
        cudaGraphDestroy(g);
        if (ie != cudaSuccess) {
            return ACB_ERR_CUDA;
        }
        it = m->graphs.emplace(key, ex).first;
    }
    if (cudaMemcpyAsync(m->tt.p, tt, 2 * sizeof(float), cudaMemcpyDeviceToDevice, s) != cudaSuccess ||
        cudaMemcpyAsync(m->input.p, d_input, nin, cudaMemcpyDeviceToDevice, s) != cudaSuccess ||
        cudaGraphLaunch(it->second, s) != cudaSuccess ||
        cudaMemcpyAsync(d_velocity, m->vel.p, nv, cudaMemcpyDeviceToDevice, s) != cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    return ACB_OK;
}

namespace {

// The arguments of dit_ggml_generate (src/dit-sampler.h:132-158) that this library implements.
struct GenArgs {
    const float *   noise = nullptr, *context = nullptr, *enc = nullptr;
    int             enc_S = 0, T = 0, N = 0, num_steps = 0;
    const float *   schedule = nullptr;
    float *         output   = nullptr;
    float           guidance = 1.0f;
    const float *   context_switch = nullptr;
    int             cover_steps    = -1;
    acb_cancel_fn   cancel         = nullptr;
    void *          cancel_data    = nullptr;
    const int *     real_S = nullptr, *real_enc_S = nullptr;
    const float *   enc_switch        = nullptr;
    const int *     real_enc_S_switch = nullptr;
    const int64_t * seeds             = nullptr;
    int             solver            = ACB_SOLVER_EULER;
    int             stork_substeps    = 10;
    int             dcw_mode          = -1;  // ACB_DCW_* or -1: no DCW
    float           dcw_scaler = 0.0f, dcw_high_scaler = 0.0f;
    acb_randn_fn    randn             = nullptr;
    void *          randn_data        = nullptr;
    float *         gpu_ms            = nullptr;
};

}  // namespace

// One denoise run on this model: the whole job (tracks [0, N)), or this rank's share of a sharded
// job -- whole track pairs (half = -1), or one CFG half of one track (half = 0 conditional, 1
// unconditional) whose partner rank holds the other half. Host argument pointers are the job's;
// the run reads the tracks [track0, track0 + n) of them.
struct DiTRun {
    acb_dit *   m      = nullptr;
    acb_comm *  comm   = nullptr;
    GenArgs     g;
    int         track0 = 0, n = 0;  // local tracks
    int         half   = -1;        // -1 whole pairs; 0 / 1 one half of track track0
    int         peer   = -1;        // the partner rank in half mode
    bool        do_cfg = false;
    int         Ng     = 0;         // local slots
    int         T = 0, Oc = 0, in_ch = 0, ctx_ch = 0, He = 0, enc_S = 0;
    size_t      n_per  = 0, n_tot = 0;
    std::vector<float> nul;
    std::vector<int>   re_now, re_first;
    std::vector<float> tv, fresh;
    std::vector<int64_t> seedv;  // SDE on the device generator: this step's seeds
    bool        switched = false, began = false;
    cudaStream_t s = nullptr;
    cudaEvent_t  e0 = nullptr, e1 = nullptr, done[2] = { nullptr, nullptr };
    int          steps_run = 0;
    acb_stork4 * stork     = nullptr;  // the STORK4 state of this run (solver stork4)
    int          last_kernels = 0;     // kernel nodes of the graph get_graph returned last

    ~DiTRun() {
        for (cudaEvent_t e : { e0, e1, done[0], done[1] }) {
            if (e) {
                cudaEventDestroy(e);
            }
        }
        acb_stork4_free(stork);
    }

    const float * ctx_of(const float * c) const { return c + (size_t) track0 * T * ctx_ch; }
    const float * enc_of(const float * e) const { return e + (size_t) track0 * enc_S * He; }

    bool upload_context(const float * ctx) {
        std::vector<float> in((size_t) Ng * T * in_ch, 0.0f);
        for (int b = 0; b < Ng; b++) {
            const int src = b % n;
            for (int t = 0; t < T; t++) {
                memcpy(&in[((size_t) b * T + t) * in_ch], &ctx_of(ctx)[((size_t) src * T + t) * ctx_ch],
                       (size_t) ctx_ch * 4);
            }
        }
        return cudaMemcpyAsync(m->input.p, in.data(), in.size() * 4, cudaMemcpyHostToDevice, s) == cudaSuccess &&
               cudaStreamSynchronize(s) == cudaSuccess;
    }

    // slot b < n is track b's conditional slot (or, in half mode, the one slot of this half)
    bool slot_is_null(int b) const { return half >= 0 ? half == 1 : b >= n; }

    bool upload_enc(const float * e) {
        std::vector<float> enc((size_t) Ng * enc_S * He);
        for (int b = 0; b < Ng; b++) {
            float * dst = &enc[(size_t) b * enc_S * He];
            if (slot_is_null(b)) {
                for (int r = 0; r < enc_S; r++) {
                    memcpy(dst + (size_t) r * He, nul.data(), (size_t) He * 4);
                }
            } else {
                memcpy(dst, enc_of(e) + (size_t) (b % n) * enc_S * He, (size_t) enc_S * He * 4);
            }
        }
        return cudaMemcpyAsync(m->enc_in.p, enc.data(), enc.size() * 4, cudaMemcpyHostToDevice, s) == cudaSuccess &&
               cudaStreamSynchronize(s) == cudaSuccess;
    }

    // padding (dit-sampler.h:244-304): every slot takes its track's lengths; the conditional slots
    // follow a cover switch, the unconditional ones keep the first lengths
    acb_status upload_lengths() {
        std::vector<int> rs((size_t) Ng), re((size_t) Ng);
        for (int b = 0; b < Ng; b++) {
            const int tr   = b % n;
            rs[(size_t) b] = g.real_S ? g.real_S[track0 + tr] : m->S;
            re[(size_t) b] = slot_is_null(b) ? re_first[(size_t) tr] : re_now[(size_t) tr];
        }
        return m->set_lengths(rs.data(), re.data(), Ng, s);
    }

    acb_status begin(acb_dit * model, acb_comm * c, const GenArgs & args, int t0, int nloc, int h, int pr);
    acb_status get_graph(int first, int last, int hist, int part, cudaGraphExec_t * ex);
    acb_status step(int step, float t_curr, float t_next, bool last, float * host_out);
    acb_status finish(float * host_out, bool gather);
};

acb_status DiTRun::begin(acb_dit * model, acb_comm * c, const GenArgs & args, int t0, int nloc, int h, int pr) {
    m = model, comm = c, g = args, track0 = t0, n = nloc, half = h, peer = pr;
    const bool dpm = g.solver == ACB_SOLVER_DPM3M, sde = g.solver == ACB_SOLVER_SDE;
    const bool stk = g.solver == ACB_SOLVER_STORK4;
    if (!m || !g.noise || !g.context || !g.enc || g.N <= 0 || g.T <= 0 || g.enc_S <= 0 || n <= 0 ||
        g.T % m->c.patch_size != 0 ||
        (g.solver != ACB_SOLVER_EULER && g.solver != ACB_SOLVER_DPM3M && g.solver != ACB_SOLVER_SDE && !stk) ||
        (sde && !g.seeds) || (half >= 0 && (n != 1 || !comm))) {
        return ACB_ERR_INVALID_ARG;
    }
    if (stk && m->stork_ms.empty()) {
        set_last_error("the stork4 solver needs the ROCK4 tables (acb_dit_set_stork4_tables)");
        return ACB_ERR_UNSUPPORTED;
    }
    if (cudaSetDevice(m->device) != cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    const acb_dit_config & cf = m->c;
    T = g.T, enc_S = g.enc_S, Oc = cf.out_channels, in_ch = cf.in_channels, ctx_ch = in_ch - Oc;
    He = cf.enc_hidden_size;
    // CFG batching (dit-sampler.h:167-171): conditional slots [0, n), unconditional [n, 2n); in half
    // mode this rank evaluates one of them
    do_cfg = g.guidance > 1.0f && m->null_emb;
    if (half >= 0 && !do_cfg) {
        set_last_error("a rank per CFG half needs guidance > 1 and a null condition");
        return ACB_ERR_INVALID_ARG;
    }
    Ng = half >= 0 ? 1 : (do_cfg ? 2 * n : n);
    ACB_TRY(m->reserve(Ng, T, enc_S));
    s     = m->st;
    n_per = (size_t) T * Oc, n_tot = n_per * n;
    const size_t pair = half >= 0 ? 2 * n_per : 0;  // [cond, uncond] velocities of the track
    bool bad = m->xt.bytes < n_tot * 4 || m->vt.bytes < n_tot * 4 || m->out.bytes < n_tot * 4 ||
               m->ra.bytes < n_tot * 8 || (dpm && (m->hist1.bytes < n_tot * 4 || m->hist2.bytes < n_tot * 4)) ||
               (sde && g.randn && m->noise.bytes < n_tot * 4) || (sde && m->step_seeds.bytes < (size_t) n * 8) ||
               m->vpair.bytes < pair * 4;
    if (bad) {
        m->drop_graphs();  // the graphs hold these addresses
        if (m->xt.alloc(n_tot * 4) != ACB_OK || m->vt.alloc(n_tot * 4) != ACB_OK || m->out.alloc(n_tot * 4) != ACB_OK ||
            m->ra.alloc(n_tot * 8) != ACB_OK ||
            (dpm && (m->hist1.alloc(n_tot * 4) != ACB_OK || m->hist2.alloc(n_tot * 4) != ACB_OK)) ||
            (sde && g.randn && m->noise.alloc(n_tot * 4) != ACB_OK) ||
            (sde && m->step_seeds.alloc((size_t) n * 8) != ACB_OK) || (pair && m->vpair.alloc(pair * 4) != ACB_OK)) {
            set_last_error("DiT generate buffers allocation failed");
            return ACB_ERR_OOM;
        }
    }
    if (do_cfg) {
        // null_condition_emb broadcast over enc_S rows for the unconditional slots (:345-385)
        if (m->null_emb->type != ACB_TYPE_F32 || m->null_emb->K * m->null_emb->N != He) {
            set_last_error("null_condition_emb has an unexpected shape");
            return ACB_ERR_FORMAT;
        }
        nul.resize((size_t) He);
        cudaMemcpy(nul.data(), m->null_emb->data, (size_t) He * 4, cudaMemcpyDeviceToHost);
    }
    re_now.assign((size_t) n, enc_S);
    if (g.real_enc_S) {
        re_now.assign(g.real_enc_S + track0, g.real_enc_S + track0 + n);
    }
    re_first = re_now;
    if (!upload_context(g.context) || !upload_enc(g.enc) ||
        cudaMemcpyAsync(m->xt.p, g.noise + (size_t) track0 * n_per, n_tot * 4, cudaMemcpyHostToDevice, s) !=
            cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    ACB_TRY(upload_lengths());
    ACB_TRY(m->condition(s));
    if (stk) {
        acb_stork4_free(stork);
        stork = nullptr;
        ACB_TRY(acb_stork4_create(&m->stork_tab, (int64_t) n_tot, g.stork_substeps, &stork));
    }
    fresh.assign(sde && g.randn ? n_tot : 0, 0.0f);
    seedv.assign(sde ? n : 0, 0);
    tv.assign(3, 0.0f);
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    cudaEventCreateWithFlags(&done[0], cudaEventDisableTiming);
    cudaEventCreateWithFlags(&done[1], cudaEventDisableTiming);
    switched = false, began = true, steps_run = 0;
    return ACB_OK;
}

// Step graphs, one per (shape, cfg, mode, first, last, solver, history, part): part 0 is the whole
// step (pack xt, evaluate, guidance, solver); in half mode part 1 is pack + evaluate and part 2
// guidance + solver, with the exchange of the velocity between them.
acb_status DiTRun::get_graph(int first, int last, int hist, int part, cudaGraphExec_t * ex) {
    const bool dpm = g.solver == ACB_SOLVER_DPM3M, sde = g.solver == ACB_SOLVER_SDE;
    uint32_t   gbits = 0;  // the guidance scale is baked into the captured APG launch
    memcpy(&gbits, &g.guidance, 4);
    const int  sde_dev = sde && !g.randn ? 1 : 0;  // SDE noise drawn inside the graph
    const int  stepk = ((((g.solver * 3 + hist) * 4 + first * 2 + last) * 4 + part) * 3 + (half + 1)) * 2 + sde_dev;
    const auto key   = std::make_tuple(Ng * 100000 + T, enc_S, do_cfg ? 1 : 0, stepk, m->exact ? 1 : 0, gbits);
    auto       it    = m->graphs.find(key);
    if (it != m->graphs.end()) {
        *ex = it->second;
        last_kernels = m->graph_kernels[key];
        return ACB_OK;
    }
    cudaGraph_t gr = nullptr;
    if (cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    acb_status st = ACB_OK;
    if (part != 2) {
        st = acb_dit_pack_xt(m->xt.as<float>(), m->input.as<float>(), n, Ng, T, Oc, ctx_ch, (acb_stream_t) s);
        if (st == ACB_OK) {
            st = m->evaluate(-1, s);
        }
    }
    if (part != 1) {
        const float * v = m->vel.as<float>();
        if (st == ACB_OK && do_cfg) {
            // guidance on [cond, uncond]: the two halves of the slots, or (half mode) of the pair
            // buffer the exchange filled
            const float * vc = half >= 0 ? m->vpair.as<float>() : v;
            st = acb_dit_apg(vc, vc + n_tot, m->ra.as<double>(), first, -0.75f, g.guidance, 2.5f, n, T, Oc,
                             m->vt.as<float>(), (acb_stream_t) s);
            v  = m->vt.as<float>();
        }
        float * vv = const_cast<float *>(v);
        if (g.solver == ACB_SOLVER_STORK4 && !last) {
            // the STORK4 step runs after the graph (its sub step count adapts on the host)
        } else if (st == ACB_OK && dpm && !last) {
            st = acb_dit_dpm3m(m->xt.as<float>(), vv, m->hist1.as<float>(), m->hist2.as<float>(), hist,
                               m->tt.as<float>(), (int64_t) n_tot, (acb_stream_t) s);
        } else if (st == ACB_OK && sde && !last && sde_dev) {
            st = acb_dit_sde_philox(m->xt.as<float>(), vv, m->step_seeds.as<int64_t>(), m->tt.as<float>(), n,
                                    (int64_t) n_per, (acb_stream_t) s);
        } else if (st == ACB_OK && sde && !last) {
            st = acb_dit_sde(m->xt.as<float>(), vv, m->noise.as<float>(), m->tt.as<float>(), (int64_t) n_tot,
                             (acb_stream_t) s);
        } else if (st == ACB_OK) {
            st = acb_dit_euler(m->xt.as<float>(), vv, m->tt.as<float>(), last, m->out.as<float>(), (int64_t) n_tot,
                               (acb_stream_t) s);
        }
    }
    const cudaError_t ce = cudaStreamEndCapture(s, &gr);
    if (st != ACB_OK || ce != cudaSuccess) {
        if (gr) {
            cudaGraphDestroy(gr);
        }
        set_last_error("DiT step graph capture failed");
        return st != ACB_OK ? st : ACB_ERR_CUDA;
    }
    const int         nk = graph_kernel_nodes(gr);
    const cudaError_t ie = cudaGraphInstantiate(ex, gr, 0);
    cudaGraphDestroy(gr);
    if (ie != cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    m->graphs.emplace(key, *ex);
    m->graph_kernels[key] = nk;
    last_kernels          = nk;
    return ACB_OK;
}

acb_status DiTRun::step(int k, float t_curr, float t_next, bool last, float * host_out) {
    if (!began) {
        return ACB_ERR_INVALID_ARG;
    }
    const bool dpm = g.solver == ACB_SOLVER_DPM3M, sde = g.solver == ACB_SOLVER_SDE;
    // at most two steps in flight, so that a cancellation (polled before every step, like
    // dit-sampler.h:409-413) takes effect within two steps
    if (steps_run >= 2 && cudaEventSynchronize(done[steps_run & 1]) != cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    if (g.cancel && g.cancel(g.cancel_data)) {
        cudaStreamSynchronize(s);
        set_last_error("cancelled at step " + std::to_string(k));
        return ACB_ERR_CANCELLED;
    }
    // cover mode (dit-sampler.h:414-449): from cover_steps on, the other context (every slot) and,
    // for the conditional slots, the other condition and its lengths
    if (g.context_switch && g.cover_steps >= 0 && k >= g.cover_steps && !switched) {
        switched = true;
        if (cudaStreamSynchronize(s) != cudaSuccess || !upload_context(g.context_switch)) {
            return ACB_ERR_CUDA;
        }
        if (g.enc_switch) {
            if (g.real_enc_S_switch) {
                re_now.assign(g.real_enc_S_switch + track0, g.real_enc_S_switch + track0 + n);
            }
            if (!upload_enc(g.enc_switch) || upload_lengths() != ACB_OK || m->condition(s) != ACB_OK) {
                return ACB_ERR_CUDA;
            }
        }
    }
    const int first = k == 0 ? 1 : 0, lst = last ? 1 : 0, hist = dpm ? (k < 2 ? k : 2) : 0;
    // SDE: the fresh noise of every track from its seed (solver-sde.h:28-31: seed_b + step + 1),
    // from the caller's noise source on the host, else drawn on the device inside the step
    if (sde && !last && g.randn) {
        for (int b = 0; b < n; b++) {
            g.randn(g.seeds[track0 + b] + k + 1, fresh.data() + (size_t) b * n_per, (int) n_per, g.randn_data);
        }
        if (cudaMemcpyAsync(m->noise.p, fresh.data(), n_tot * 4, cudaMemcpyHostToDevice, s) != cudaSuccess) {
            return ACB_ERR_CUDA;
        }
    } else if (sde && !last) {
        for (int b = 0; b < n; b++) {
            seedv[b] = g.seeds[track0 + b] + k + 1;
        }
        // pageable source: staged by the call, like the timesteps below
        if (cudaMemcpyAsync(m->step_seeds.p, seedv.data(), (size_t) n * 8, cudaMemcpyHostToDevice, s) !=
            cudaSuccess) {
            return ACB_ERR_CUDA;
        }
    }
    // t_curr, t_r = t_curr (dit-sampler.h:431-436), t_next; pageable source: staged by the call
    tv[0] = t_curr, tv[1] = t_curr, tv[2] = last ? 0.0f : t_next;
    if (steps_run == 0) {
        cudaEventRecord(e0, s);
    }
    if (cudaMemcpyAsync(m->tt.p, tv.data(), 3 * sizeof(float), cudaMemcpyHostToDevice, s) != cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    int launched = 0;  // this library's kernels in this step
    if (half < 0) {
        cudaGraphExec_t ex = nullptr;
        ACB_TRY(get_graph(first, lst, hist, 0, &ex));
        launched = last_kernels;
        if (cudaGraphLaunch(ex, s) != cudaSuccess) {
            return ACB_ERR_CUDA;
        }
    } else {
        // evaluate this half, swap velocities with the partner, then guidance + solver on the
        // [cond, uncond] pair (both ranks of the pair hold the same xt and take the same step)
        cudaGraphExec_t ea = nullptr, eb = nullptr;
        ACB_TRY(get_graph(first, lst, hist, 1, &ea));
        launched = last_kernels;
        ACB_TRY(get_graph(first, lst, hist, 2, &eb));
        launched += last_kernels;
        float * mine  = m->vpair.as<float>() + (size_t) half * n_per;
        float * other = m->vpair.as<float>() + (size_t) (1 - half) * n_per;
        if (cudaGraphLaunch(ea, s) != cudaSuccess ||
            cudaMemcpyAsync(mine, m->vel.p, n_per * 4, cudaMemcpyDeviceToDevice, s) != cudaSuccess) {
            return ACB_ERR_CUDA;
        }
        ACB_TRY(comm_exchange(comm, peer, mine, other, n_per * 4, s));
        if (cudaGraphLaunch(eb, s) != cudaSuccess) {
            return ACB_ERR_CUDA;
        }
    }
    if (stork && !last) {
        const float * v = do_cfg ? m->vt.as<float>() : m->vel.as<float>();
        ACB_TRY(acb_stork4_step(stork, m->xt.as<float>(), v, t_curr, t_next, (acb_stream_t) s));
    }
    if (g.dcw_mode >= 0 && !last && !sde) {
        // DCW after the solver step (dit-sampler.h:613-666) with this step's effective scales; a
        // zero scale leaves xt as it is (the reference returns before its transform)
        const int   md = g.dcw_mode;
        const float hi = md == ACB_DCW_DOUBLE ? g.dcw_high_scaler : g.dcw_scaler;
        const float sl = md == ACB_DCW_PIX ? g.dcw_scaler : t_curr * g.dcw_scaler;
        const float sh = (1.0f - t_curr) * hi;
        const bool  run = md == ACB_DCW_HIGH ? sh != 0.0f : md == ACB_DCW_DOUBLE ? (sl != 0.0f || sh != 0.0f)
                                                                                 : sl != 0.0f;
        if (run) {
            const float * v = do_cfg ? m->vt.as<float>() : m->vel.as<float>();
            ACB_TRY(acb_dit_dcw(m->xt.as<float>(), v, n, T, Oc, t_next, md, sl, sh, (acb_stream_t) s));
            launched++;
        }
    }
    m->step_kernels = launched;
    if (host_out && cudaMemcpyAsync(host_out, last ? m->out.p : m->xt.p, n_tot * 4, cudaMemcpyDeviceToHost, s) !=
                        cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    if (cudaEventRecord(done[steps_run & 1], s) != cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    steps_run++;
    return ACB_OK;
}

// x0 of the run's tracks (the last step's prediction) to host_out: this rank's tracks, or with
// `gather` every rank's, all-gathered in rank order (track order) over the communicator.
acb_status DiTRun::finish(float * host_out, bool gather) {
    if (!began) {
        return ACB_ERR_INVALID_ARG;
    }
    began = false;
    cudaEventRecord(e1, s);
    const float * src = m->out.as<float>();
    size_t        cnt = n_tot;
    if (gather && comm) {
        const int w = comm_world(comm);
        if (half >= 0) {
            // both ranks of a pair hold the track's x0: gather every rank's copy, keep even ranks'
            if (m->xall.bytes < (size_t) w * n_tot * 4) {
                ACB_TRY(m->xall.alloc((size_t) w * n_tot * 4));
            }
            ACB_TRY(comm_all_gather(comm, m->out.p, m->xall.p, n_tot * 4, s));
            ACB_TRY(comm_wait(comm, s));
            std::vector<float> all((size_t) w * n_tot);
            if (cudaMemcpy(all.data(), m->xall.p, all.size() * 4, cudaMemcpyDeviceToHost) != cudaSuccess) {
                return ACB_ERR_CUDA;
            }
            for (int r = 0; r < w; r += 2) {
                memcpy(host_out + (size_t) (r / 2) * n_tot, all.data() + (size_t) r * n_tot, n_tot * 4);
            }
            src = nullptr;
        } else {
            if (m->xall.bytes < (size_t) w * n_tot * 4) {
                ACB_TRY(m->xall.alloc((size_t) w * n_tot * 4));
            }
            ACB_TRY(comm_all_gather(comm, m->out.p, m->xall.p, n_tot * 4, s));
            ACB_TRY(comm_wait(comm, s));
            src = m->xall.as<float>();
            cnt = (size_t) w * n_tot;
        }
    }
    int dev_err = 0;
    if ((src && cudaMemcpyAsync(host_out, src, cnt * 4, cudaMemcpyDeviceToHost, s) != cudaSuccess) ||
        cudaMemcpyAsync(&dev_err, m->err.p, 4, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess) {
        return ACB_ERR_CUDA;
    }
    if (g.gpu_ms) {
        cudaEventElapsedTime(g.gpu_ms, e0, e1);
    }
    if (dev_err) {
        set_last_error("device error flag " + std::to_string(dev_err));
        return ACB_ERR_DEVICE;
    }
    return ACB_OK;
}

acb_dit::~acb_dit() {
    cudaSetDevice(device);
    job.reset();
    drop_graphs();
    if (st) {
        cudaStreamDestroy(st);
    }
}

namespace {

acb_status run_schedule(DiTRun & r, const GenArgs & g) {
    for (int k = 0; k < g.num_steps; k++) {
        const bool last = k == g.num_steps - 1;
        ACB_TRY(r.step(k, g.schedule[k], last ? 0.0f : g.schedule[k + 1], last, nullptr));
    }
    return ACB_OK;
}

acb_status generate_impl(acb_dit * m, const GenArgs & g) {
    if (!m || !g.schedule || !g.output || g.num_steps <= 0) {
        return ACB_ERR_INVALID_ARG;
    }
    DiTRun r;
    ACB_TRY(r.begin(m, nullptr, g, 0, g.N, -1, -1));
    const acb_status st = run_schedule(r, g);
    if (st != ACB_OK) {
        cudaStreamSynchronize(m->st);
        return st;
    }
    return r.finish(g.output, false);
}

}  // namespace

extern "C" acb_status acb_dit_generate(acb_dit * m, const float * noise, const float * context_latents,
                                       const float * enc_hidden, int enc_S, int T, int N, int num_steps,
                                       const float * schedule, float * output, float guidance_scale, float * gpu_ms) {
    return acb_dit_generate_solver(m, noise, context_latents, enc_hidden, enc_S, T, N, num_steps, schedule, output,
                                   guidance_scale, ACB_SOLVER_EULER, gpu_ms);
}

extern "C" acb_status acb_dit_generate_solver(acb_dit * m, const float * noise, const float * context_latents,
                                              const float * enc_hidden, int enc_S, int T, int N, int num_steps,
                                              const float * schedule, float * output, float guidance_scale,
                                              int solver, float * gpu_ms) {
    if (solver != ACB_SOLVER_EULER && solver != ACB_SOLVER_DPM3M) {
        return ACB_ERR_INVALID_ARG;  // the SDE solver needs per-track seeds: acb_dit_generate_ex
    }
    GenArgs g;
    g.noise     = noise;
    g.context   = context_latents;
    g.enc       = enc_hidden;
    g.enc_S     = enc_S;
    g.T         = T;
    g.N         = N;
    g.num_steps = num_steps;
    g.schedule  = schedule;
    g.output    = output;
    g.guidance  = guidance_scale;
    g.solver    = solver;
    g.gpu_ms    = gpu_ms;
    return generate_impl(m, g);
}

extern "C" acb_status acb_dit_generate_ex(acb_dit * m, const float * noise, const float * context_latents,
                                          const float * enc_hidden, int enc_S, int T, int N, int num_steps,
                                          const float * schedule, float * output, float guidance_scale,
                                          const float * context_switch, int cover_steps, acb_cancel_fn cancel,
                                          void * cancel_data, const int * real_S, const int * real_enc_S,
                                          const float * enc_switch, const int * real_enc_S_switch,
                                          const int64_t * seeds, int use_batch_cfg, float dcw_scaler,
                                          float dcw_high_scaler, const char * dcw_mode, const char * solver_name,
                                          int stork_substeps, acb_randn_fn randn, void * randn_data, float * gpu_ms) {
    (void) use_batch_cfg;   // both settings run the batched graph: HBM is not the constraint here
    int solver = ACB_SOLVER_EULER;  // solver_lookup: NULL or "" is euler; an unknown name falls back to it
    if (solver_name && std::strcmp(solver_name, "dpm3m") == 0) {
        solver = ACB_SOLVER_DPM3M;
    } else if (solver_name && std::strcmp(solver_name, "sde") == 0) {
        solver = ACB_SOLVER_SDE;
    } else if (solver_name && std::strcmp(solver_name, "stork4") == 0) {
        solver = ACB_SOLVER_STORK4;
    }
    GenArgs g;
    g.noise             = noise;
    g.context           = context_latents;
    g.enc               = enc_hidden;
    g.enc_S             = enc_S;
    g.T                 = T;
    g.N                 = N;
    g.num_steps         = num_steps;
    g.schedule          = schedule;
    g.output            = output;
    g.guidance          = guidance_scale;
    g.context_switch    = context_switch;
    g.cover_steps       = cover_steps;
    g.cancel            = cancel;
    g.cancel_data       = cancel_data;
    g.real_S            = real_S;
    g.real_enc_S        = real_enc_S;
    g.enc_switch        = enc_switch;
    g.real_enc_S_switch = real_enc_S_switch;
    g.seeds             = seeds;
    g.solver            = solver;
    g.stork_substeps    = stork_substeps > 0 ? stork_substeps : 10;
    g.randn             = randn;
    g.randn_data        = randn_data;
    g.gpu_ms            = gpu_ms;
    if (dcw_scaler > 0.0f || dcw_high_scaler > 0.0f) {  // the mode names of dit-sampler.h:632-640
        g.dcw_mode        = ACB_DCW_LOW;  // also an unknown or missing name
        g.dcw_scaler      = dcw_scaler;
        g.dcw_high_scaler = dcw_high_scaler;
        if (dcw_mode && std::strcmp(dcw_mode, "high") == 0) {
            g.dcw_mode = ACB_DCW_HIGH;
        } else if (dcw_mode && std::strcmp(dcw_mode, "double") == 0) {
            g.dcw_mode = ACB_DCW_DOUBLE;
        } else if (dcw_mode && std::strcmp(dcw_mode, "pix") == 0) {
            g.dcw_mode = ACB_DCW_PIX;
        }
    }
    return generate_impl(m, g);
}

extern "C" acb_status acb_dit_set_stork4_tables(acb_dit * m, const acb_stork4_tables * t) {
    if (!m || !t || !t->ms || t->ms_len <= 0 || !t->fpa || !t->fpb || !t->recf || t->recf_len <= 0) {
        return ACB_ERR_INVALID_ARG;
    }
    m->stork_ms.assign(t->ms, t->ms + t->ms_len);
    m->stork_fpa.assign(t->fpa, t->fpa + (size_t) t->ms_len * 6);
    m->stork_fpb.assign(t->fpb, t->fpb + (size_t) t->ms_len * 4);
    m->stork_recf.assign(t->recf, t->recf + t->recf_len);
    m->stork_tab = acb_stork4_tables{ m->stork_ms.data(), t->ms_len, m->stork_fpa.data(), m->stork_fpb.data(),
                                      m->stork_recf.data(), t->recf_len };
    return ACB_OK;
}

// ---- sharded jobs (one process per GPU) ------------------------------------------------------

extern "C" acb_status acb_dit_shard_plan(int n_tracks, int cfg, int world, int rank, int * track0, int * n_local,
                                         int * half, int * peer) {
    if (n_tracks <= 0 || world <= 0 || rank < 0 || rank >= world || !track0 || !n_local || !half || !peer) {
        return ACB_ERR_INVALID_ARG;
    }
    if (n_tracks % world == 0) {
        // whole track pairs: no exchange during the steps
        *n_local = n_tracks / world;
        *track0  = rank * *n_local;
        *half    = -1;
        *peer    = -1;
        return ACB_OK;
    }
    if (cfg && world == 2 * n_tracks) {
        // one CFG half per rank: ranks 2t (conditional) and 2t + 1 (unconditional) share track t
        *n_local = 1;
        *track0  = rank / 2;
        *half    = rank % 2;
        *peer    = rank ^ 1;
        return ACB_OK;
    }
    set_last_error("acb_dit_shard_plan: " + std::to_string(n_tracks) + " tracks do not shard over " +
                   std::to_string(world) + " ranks (a divisor of the track count, or two ranks per track with CFG)");
    return ACB_ERR_UNSUPPORTED;
}

namespace {

int solver_id(const char * name, acb_status * st) {
    *st = ACB_OK;
    if (name && std::strcmp(name, "dpm3m") == 0) {
        return ACB_SOLVER_DPM3M;
    }
    if (name && std::strcmp(name, "sde") == 0) {
        return ACB_SOLVER_SDE;
    }
    if (name && std::strcmp(name, "stork4") == 0) {
        return ACB_SOLVER_STORK4;
    }
    return ACB_SOLVER_EULER;  // solver_lookup's fallback for unknown names
}

}  // namespace

extern "C" acb_status acb_dit_job_begin(acb_dit * m, acb_comm * comm, const float * noise, const float * context_latents,
                                        const float * enc_hidden, int enc_S, int T, int N, float guidance_scale,
                                        const float * context_switch, int cover_steps, acb_cancel_fn cancel,
                                        void * cancel_data, const int * real_S, const int * real_enc_S,
                                        const float * enc_switch, const int * real_enc_S_switch,
                                        const int64_t * seeds, const char * solver_name, acb_randn_fn randn,
                                        void * randn_data) {
    if (!m) {
        return ACB_ERR_INVALID_ARG;
    }
    acb_status st     = ACB_OK;
    const int  solver = solver_id(solver_name, &st);
    ACB_TRY(st);
    int t0 = 0, nl = N, half = -1, peer = -1;
    if (comm) {
        const bool cfg = guidance_scale > 1.0f && m->null_emb;
        ACB_TRY(acb_dit_shard_plan(N, cfg ? 1 : 0, comm_world(comm), comm_rank(comm), &t0, &nl, &half, &peer));
    }
    GenArgs g;
    g.noise             = noise;
    g.context           = context_latents;
    g.enc               = enc_hidden;
    g.enc_S             = enc_S;
    g.T                 = T;
    g.N                 = N;
    g.guidance          = guidance_scale;
    g.context_switch    = context_switch;
    g.cover_steps       = cover_steps;
    g.cancel            = cancel;
    g.cancel_data       = cancel_data;
    g.real_S            = real_S;
    g.real_enc_S        = real_enc_S;
    g.enc_switch        = enc_switch;
    g.real_enc_S_switch = real_enc_S_switch;
    g.seeds             = seeds;
    g.solver            = solver;
    g.randn             = randn;
    g.randn_data        = randn_data;
    m->job.reset(new DiTRun());
    const acb_status b = m->job->begin(m, comm, g, t0, nl, half, peer);
    if (b != ACB_OK) {
        m->job.reset();
    }
    return b;
}

extern "C" acb_status acb_dit_job_step(acb_dit * m, int step, float t_curr, float t_next, int last, float * host_out) {
    if (!m || !m->job || step < 0) {
        return ACB_ERR_INVALID_ARG;
    }
    return m->job->step(step, t_curr, t_next, last != 0, host_out);
}

extern "C" acb_status acb_dit_job_end(acb_dit * m, float * output, float * gpu_ms) {
    if (!m || !m->job || !output) {
        return ACB_ERR_INVALID_ARG;
    }
    m->job->g.gpu_ms      = gpu_ms;
    const acb_status st   = m->job->finish(output, m->job->comm != nullptr);
    m->job.reset();
    return st;
}

extern "C" acb_stream_t acb_dit_stream(const acb_dit * m) {
    return m ? (acb_stream_t) m->st : nullptr;
}

extern "C" acb_status acb_dit_generate_sharded(acb_dit * m, acb_comm * comm, const float * noise,
                                               const float * context_latents, const float * enc_hidden, int enc_S,
                                               int T, int N, int num_steps, const float * schedule, float * output,
                                               float guidance_scale, const float * context_switch, int cover_steps,
                                               acb_cancel_fn cancel, void * cancel_data, const int * real_S,
                                               const int * real_enc_S, const float * enc_switch,
                                               const int * real_enc_S_switch, const int64_t * seeds,
                                               const char * solver_name, acb_randn_fn randn, void * randn_data,
                                               float * gpu_ms) {
    if (!m || !comm || !schedule || !output || num_steps <= 0) {
        return ACB_ERR_INVALID_ARG;
    }
    ACB_TRY(acb_dit_job_begin(m, comm, noise, context_latents, enc_hidden, enc_S, T, N, guidance_scale, context_switch,
                              cover_steps, cancel, cancel_data, real_S, real_enc_S, enc_switch, real_enc_S_switch,
                              seeds, solver_name, randn, randn_data));
    GenArgs g       = m->job->g;
    g.num_steps     = num_steps;
    g.schedule      = schedule;
    const acb_status st = run_schedule(*m->job, g);
    if (st != ACB_OK) {
        cudaStreamSynchronize(m->st);
        m->job.reset();
        return st;
    }
    return acb_dit_job_end(m, output, gpu_ms);
}

extern "C" int acb_dit_eval_kernels(const acb_dit * m) {
    return m ? m->eval_kernels : 0;
}

extern "C" int acb_dit_step_kernels(const acb_dit * m) {
    return m ? m->step_kernels : 0;
}

extern "C" void acb_dit_free(acb_dit * m) {
    delete m;
}
