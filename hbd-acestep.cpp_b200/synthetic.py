"""Synthetic GGUF models for benchmarks and parity tests (no checkpoints exist offline).

Weights are N(0, 0.02) and norm gains 1 + N(0, 0.01) (F32), drawn from a seeded torch
generator on the GPU and quantised on the device by libacb's acb_quantize; files are written
with gguf-py's GGUFWriter using the reference's tensor names (model.layers.{i}.self_attn.q_proj.
weight, ...) and its `acestep.config_json` key, so acb_qw3lm_load reads them exactly like a
converted checkpoint. Quantisation mixes follow tools/quantize.cpp:51-63,98-171 of the
reference (Q4_K_M: Q4_K base, v_proj/down_proj bumped to Q6_K in layers i < L/9,
i >= L - L/7 or i % 3 == 0, embed_tokens Q6_K).
"""
from __future__ import annotations

import json

import numpy as np

import acb

Q8_0, Q4_K, Q6_K, F32 = acb.Q8_0, acb.Q4_K, acb.Q6_K, acb.F32

QWEN3_1_7B = dict(vocab_size=217472, hidden_size=2048, intermediate_size=6144, num_hidden_layers=28,
                  num_attention_heads=16, num_key_value_heads=8, head_dim=128, rope_theta=1000000.0,
                  rms_norm_eps=1e-6, tie_word_embeddings=True)
QWEN3_EMBED_0_6B = dict(vocab_size=151936, hidden_size=1024, intermediate_size=3072, num_hidden_layers=28,
                        num_attention_heads=16, num_key_value_heads=8, head_dim=128, rope_theta=1000000.0,
                        rms_norm_eps=1e-6)
QWEN3_4B = dict(vocab_size=217472, hidden_size=2560, intermediate_size=9728, num_hidden_layers=36,
                num_attention_heads=32, num_key_value_heads=8, head_dim=128, rope_theta=1000000.0,
                rms_norm_eps=1e-6, tie_word_embeddings=True)


def policy_q8_0(name: str, layer: int, n_layers: int) -> int:
    return Q8_0


def policy_q4_k_m(name: str, layer: int, n_layers: int) -> int:
    if "embed_tokens" in name:
        return Q6_K
    if ("v_proj" in name or "down_proj" in name) and layer >= 0:
        L = n_layers
        if layer < L // 9 or layer >= L - L // 7 or layer % 3 == 0:
            return Q6_K
    return Q4_K


def quantize_on_device(w, qtype: int):
    """w: float32 CUDA tensor [N, K] -> uint8 numpy [N, row_bytes] of GGUF blocks."""
    import torch
    N, K = w.shape
    rb = acb.lib().acb_row_bytes(qtype, K)
    out = torch.empty((N, rb), dtype=torch.uint8, device=w.device)
    acb._check("acb_quantize", acb.lib().acb_quantize(w.data_ptr(), N, K, qtype, out.data_ptr(),
                                                       acb._stream(None)))
    return out.cpu().numpy()


def lm_tensors(cfg: dict, policy=policy_q8_0, seed: int = 0, device: str = "cuda", prefix: str = "model."):
    """Yields (name, qtype, raw uint8 [N, row_bytes] or float32 array, ggml K) in file order.
    prefix "model." gives the LM's names (src/qwen3-lm.h), "" the text encoder's (src/qwen3-enc.h)."""
    import torch
    g = torch.Generator(device=device).manual_seed(seed)
    H, F, L = cfg["hidden_size"], cfg["intermediate_size"], cfg["num_hidden_layers"]
    Nh, Nkv, D, V = cfg["num_attention_heads"], cfg["num_key_value_heads"], cfg["head_dim"], cfg["vocab_size"]

    def mat(name, N, K, layer):
        qt = policy(name, layer, L)
        w = torch.randn((N, K), generator=g, device=device) * 0.02
        return name, qt, quantize_on_device(w, qt), K

    def gain(name, n):
        v = (1.0 + 0.01 * torch.randn(n, generator=g, device=device)).cpu().numpy().astype(np.float32)
        return name, F32, v, n

    yield mat(f"{prefix}embed_tokens.weight", V, H, -1)
    yield gain(f"{prefix}norm.weight", H)
    for i in range(L):
        p = f"{prefix}layers.{i}"
        yield gain(f"{p}.input_layernorm.weight", H)
        yield gain(f"{p}.post_attention_layernorm.weight", H)
        yield mat(f"{p}.self_attn.q_proj.weight", Nh * D, H, i)
        yield mat(f"{p}.self_attn.k_proj.weight", Nkv * D, H, i)
        yield mat(f"{p}.self_attn.v_proj.weight", Nkv * D, H, i)
        yield mat(f"{p}.self_attn.o_proj.weight", H, Nh * D, i)
        yield gain(f"{p}.self_attn.q_norm.weight", D)
        yield gain(f"{p}.self_attn.k_norm.weight", D)
        yield mat(f"{p}.mlp.gate_proj.weight", F, H, i)
        yield mat(f"{p}.mlp.up_proj.weight", F, H, i)
        yield mat(f"{p}.mlp.down_proj.weight", H, F, i)


def write_lm_gguf(path: str, cfg: dict, policy=policy_q8_0, seed: int = 0, device: str = "cuda",
                  keep: dict | None = None, prefix: str = "model.", arch: str = "acestep-lm") -> int:
    """Write a Qwen3 LM GGUF (arch acestep-lm; prefix "" and arch "qwen3" for a text encoder).
    If `keep` is a dict, the raw tensors are stored in it by name (for oracle comparisons on
    small models). Returns the file's tensor-data bytes."""
    import gguf
    w = gguf.GGUFWriter(path, arch)
    w.add_string("acestep.config_json", json.dumps(cfg))
    total = 0
    for name, qt, raw, K in lm_tensors(cfg, policy, seed, device, prefix):
        if qt == F32:
            w.add_tensor(name, raw)
        else:
            w.add_tensor(name, raw, raw_dtype=gguf.GGMLQuantizationType(qt))
        total += raw.nbytes
        if keep is not None:
            keep[name] = (qt, raw, K)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return total
