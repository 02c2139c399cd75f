"""Tiny seeded Qwen3 LMs written as GGUF files (reference tensor names, acestep.config_json),
with the identical raw tensors handed to the oracle. Weights are quantised on the CPU by the
oracle's encoders so the CPU-only tests need no device."""
import json

import numpy as np

import oracle as O

TINY = dict(vocab_size=1000, hidden_size=256, intermediate_size=512, num_hidden_layers=2, num_attention_heads=4,
            num_key_value_heads=2, head_dim=128, rope_theta=1000000.0, rms_norm_eps=1e-6, tie_word_embeddings=True)


def policy_all(qt):
    return lambda name, layer, L: qt


def policy_q4_k_m(name, layer, L):
    """tools/quantize.cpp Q4_K_M: base Q4_K, v/down bumped to Q6_K in i < L/9, i >= L-L/7, i%3==0; embed Q6_K."""
    if "embed_tokens" in name:
        return O.Q6_K
    if ("v_proj" in name or "down_proj" in name) and layer >= 0:
        if layer < L // 9 or layer >= L - L // 7 or layer % 3 == 0:
            return O.Q6_K
    return O.Q4_K


def make_tensors(cfg, policy, seed=0, std=0.02, embed_std=None, prefix="model."):
    """prefix "model." gives the LM's tensor names, "" the text encoder's."""
    rng = np.random.default_rng(seed)
    H, F, L = cfg["hidden_size"], cfg["intermediate_size"], cfg["num_hidden_layers"]
    Nh, Nkv, D, V = cfg["num_attention_heads"], cfg["num_key_value_heads"], cfg["head_dim"], cfg["vocab_size"]
    out = {}

    def mat(name, N, K, layer, s=std):
        qt = policy(name, layer, L)
        w = rng.standard_normal((N, K), dtype=np.float32)
        w *= np.float32(s)
        out[name] = (qt, O.quantize(w, qt), K, N)

    def gain(name, n):
        out[name] = (O.F32, (1.0 + 0.01 * rng.standard_normal(n)).astype(np.float32), n, 1)

    mat(f"{prefix}embed_tokens.weight", V, H, -1, embed_std or std)
    gain(f"{prefix}norm.weight", H)
    for i in range(L):
        p = f"{prefix}layers.{i}"
        gain(f"{p}.input_layernorm.weight", H)
        gain(f"{p}.post_attention_layernorm.weight", H)
        mat(f"{p}.self_attn.q_proj.weight", Nh * D, H, i)
        mat(f"{p}.self_attn.k_proj.weight", Nkv * D, H, i)
        mat(f"{p}.self_attn.v_proj.weight", Nkv * D, H, i)
        mat(f"{p}.self_attn.o_proj.weight", H, Nh * D, i)
        gain(f"{p}.self_attn.q_norm.weight", D)
        gain(f"{p}.self_attn.k_norm.weight", D)
        mat(f"{p}.mlp.gate_proj.weight", F, H, i)
        mat(f"{p}.mlp.up_proj.weight", F, H, i)
        mat(f"{p}.mlp.down_proj.weight", H, F, i)
    return out


def write_gguf(path, cfg, tensors, arch="acestep-lm"):
    import gguf
    w = gguf.GGUFWriter(path, arch)
    w.add_string("acestep.config_json", json.dumps(cfg))
    for name, (qt, raw, K, N) in tensors.items():
        if qt == O.F32:
            w.add_tensor(name, raw.reshape(-1) if N == 1 else raw)
        else:
            w.add_tensor(name, raw, raw_dtype=gguf.GGMLQuantizationType(qt))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


def oracle_model(cfg, tensors, prefix="model."):
    return O.qwen3_from_gguf_tensors(cfg, tensors, prefix)


def oracle_greedy(m, prompt, n_steps, set_=0):
    """Reference greedy loop: prefill, feed argmax, decode one token at a time. Returns the
    argmax after each of the n_steps decode steps (and its top1 - top2 margin)."""
    lg = m.prefill(prompt, set_=set_)
    nxt = int(np.argmax(lg))
    toks, margins = [], []
    for _ in range(n_steps):
        lg = m.decode(np.array([nxt], np.int32), set0=set_)[0]
        nxt = int(np.argmax(lg))
        srt = np.sort(lg)
        toks.append(nxt)
        margins.append(float(srt[-1] - srt[-2]))
    return toks, margins
