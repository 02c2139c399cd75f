"""CPU: pin the oracle against the committed golden fixtures before trusting it.

quant_golden.npz comes from gguf-py 0.19.0 (bit-exact Q8_0 quantize per gguf/quants.py:378-394,
and the Q8_0 / Q4_K / Q6_K dequantizers); lm_golden.npz holds logits from the reference's own
fp32 PyTorch restatement of the Qwen3 LM forward (tests/debug-lm-logits.py:7-136) on a tiny
seeded model. Both were produced by tests/golden/make_golden.py.
"""
import json
import os

import numpy as np
import pytest

import oracle as O
from helpers import assert_bitexact, cos_sim, max_rel

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def qg():
    return np.load(os.path.join(GOLD, "quant_golden.npz"))


def test_q8_0_quantize_matches_gguf_py(qg):
    ours = O.quantize(qg["x"], O.Q8_0)
    assert np.array_equal(ours, qg["q8_0_bytes"])


@pytest.mark.parametrize("name,qt,K", [("q8_0", O.Q8_0, 512), ("q4_k", O.Q4_K, 512), ("q6_k", O.Q6_K, 512)])
def test_dequant_matches_gguf_py(qg, name, qt, K):
    deq = O.dequantize(qg[f"{name}_bytes"], qt, K)
    assert_bitexact(deq, qg[f"{name}_deq"].astype(np.float32), name)


def test_f16_conversions_exhaustive():
    L = O.lib()
    bits = np.arange(65536, dtype=np.uint16)
    ours = np.array([L.orc_f16_to_f32(int(b)) for b in bits], dtype=np.float32)
    ref = bits.view(np.float16).astype(np.float32)
    same = (ours.view(np.uint32) == ref.view(np.uint32)) | (np.isnan(ours) & np.isnan(ref))
    assert same.all()
    rng = np.random.default_rng(1)
    v = np.concatenate([rng.standard_normal(20000).astype(np.float32) * s for s in (1e-7, 1e-3, 1, 1e3, 6e4)])
    v = np.concatenate([v, np.array([65504, 65519, 65520, -65520, 6e-8, 2.9e-8, 3.0e-8, 0.0, -0.0], np.float32)])
    ours16 = np.array([L.orc_f32_to_f16(float(t)) for t in v], dtype=np.uint16)
    with np.errstate(over="ignore"):
        assert np.array_equal(ours16, v.astype(np.float16).view(np.uint16))


def test_k_quant_encoders_make_valid_blocks():
    rng = np.random.default_rng(2)
    x = (rng.standard_normal((8, 1024)) * 0.02).astype(np.float32)
    for qt, tol in ((O.Q4_K, 0.08), (O.Q6_K, 0.02)):
        raw = O.quantize(x, qt)
        from gguf import quants, GGMLQuantizationType as T
        ref = quants.dequantize(raw, T.Q4_K if qt == O.Q4_K else T.Q6_K).astype(np.float32)
        assert_bitexact(O.dequantize(raw, qt, 1024), ref, "k-quant")
        assert max_rel(ref, x) < tol


def test_q8_K_activation_quant_roundtrip():
    rng = np.random.default_rng(3)
    x = rng.standard_normal((4, 512)).astype(np.float32)
    raw = O.quantize(x, O.Q8_K)
    back = O.dequantize(raw, O.Q8_K, 512)
    assert max_rel(back, x) < 1.0 / 127 + 1e-6
    # bsums are the 16-element sums of the int8 values
    blk = raw.reshape(-1, 292)
    qs = blk[:, 4:260].view(np.int8).astype(np.int32).reshape(-1, 16, 16).sum(-1)
    bs = blk[:, 260:292].copy().view(np.int16).astype(np.int32)
    assert np.array_equal(qs, bs)


def _lm_weights(z, cfg, qtype=O.F32):
    W = {k[2:]: z[k].astype(np.float32) for k in z.files if k.startswith("w:")}

    def t(a, qt=qtype):
        a = np.ascontiguousarray(a, np.float32)
        K = a.shape[-1]
        return (qt, O.quantize(a, qt), K, a.size // K)

    def f32(a):
        return t(a, O.F32)

    w = {"embed": t(W["model.embed_tokens.weight"]), "final_norm": f32(W["model.norm.weight"])}
    for i in range(cfg["num_hidden_layers"]):
        p = f"model.layers.{i}"
        w[f"layers.{i}.attn_norm"] = f32(W[p + ".input_layernorm.weight"])
        w[f"layers.{i}.post_norm"] = f32(W[p + ".post_attention_layernorm.weight"])
        w[f"layers.{i}.qkv"] = t(np.concatenate([W[p + ".self_attn.q_proj.weight"], W[p + ".self_attn.k_proj.weight"],
                                                  W[p + ".self_attn.v_proj.weight"]]))
        w[f"layers.{i}.o"] = t(W[p + ".self_attn.o_proj.weight"])
        w[f"layers.{i}.q_norm"] = f32(W[p + ".self_attn.q_norm.weight"])
        w[f"layers.{i}.k_norm"] = f32(W[p + ".self_attn.k_norm.weight"])
        w[f"layers.{i}.gate_up"] = t(np.concatenate([W[p + ".mlp.gate_proj.weight"], W[p + ".mlp.up_proj.weight"]]))
        w[f"layers.{i}.down"] = t(W[p + ".mlp.down_proj.weight"])
    oc = dict(n_layers=cfg["num_hidden_layers"], H=cfg["hidden_size"], F=cfg["intermediate_size"],
              Nh=cfg["num_attention_heads"], Nkv=cfg["num_key_value_heads"], D=cfg["head_dim"],
              V=cfg["vocab_size"], rope_theta=cfg["rope_theta"], eps=cfg["rms_norm_eps"])
    return oc, w, W


def test_oracle_lm_matches_reference_pytorch_logits():
    z = np.load(os.path.join(GOLD, "lm_golden.npz"))
    cfg = json.loads(str(z["config_json"]))
    oc, w, W = _lm_weights(z, cfg)
    m = O.OracleQwen3(oc, w)
    ref = z["logits"]
    # f32 attention path (the encoder graph, qwen3_forward): differs from torch fp32 only by
    # summation order
    hid = m.encode(z["prompt"])
    lg = W["model.embed_tokens.weight"] @ hid[-1]
    assert cos_sim(lg, ref) > 0.9999999 and max_rel(lg, ref) < 1e-6
    # LM prefill path with the f16 KV cache (q and probabilities rounded to f16, ggml-CPU)
    m.alloc_kv(1, 64)
    lg2 = m.prefill(z["prompt"])
    assert cos_sim(lg2, ref) > 0.99999 and max_rel(lg2, ref) < 1e-3
    assert int(lg2.argmax()) == int(ref.argmax())


def test_oracle_lm_q8_0_close_to_reference():
    z = np.load(os.path.join(GOLD, "lm_golden.npz"))
    cfg = json.loads(str(z["config_json"]))
    oc, w, _ = _lm_weights(z, cfg, O.Q8_0)
    m = O.OracleQwen3(oc, w)
    m.alloc_kv(1, 64)
    lg = m.prefill(z["prompt"])
    assert cos_sim(lg, z["logits"]) > 0.999


def test_oracle_decode_matches_prefill():
    """One-token batched decode after a prefill equals the prefill of the longer prompt."""
    z = np.load(os.path.join(GOLD, "lm_golden.npz"))
    cfg = json.loads(str(z["config_json"]))
    oc, w, _ = _lm_weights(z, cfg, O.Q8_0)
    prompt = z["prompt"]
    a = O.OracleQwen3(oc, w)
    a.alloc_kv(2, 64)
    a.prefill(prompt[:-1], set_=0)
    a.prefill(prompt[:-3], set_=1)
    dec = a.decode(np.array([prompt[-1], prompt[-3]], np.int32), set0=0)
    b = O.OracleQwen3(oc, w)
    b.alloc_kv(1, 64)
    full = b.prefill(prompt)
    assert cos_sim(dec[0], full) > 0.999999


def test_mul_mat_exact_mode_is_dequantised_float_product():
    """ORC_MM_EXACT: dequantised weights times the unrounded activation (double accumulation);
    ORC_MM_GGML stays the default and differs by the activation quantisation."""
    rng = np.random.default_rng(11)
    N, K, M = 40, 512, 3
    x = rng.standard_normal((M, K)).astype(np.float32)
    assert O.get_mul_mat_mode() == O.MM_GGML
    for qt in (O.Q8_0, O.Q4_K, O.Q6_K, O.BF16):
        W = O.quantize((rng.standard_normal((N, K)) * 0.02).astype(np.float32), qt)
        ref = x.astype(np.float64) @ O.dequantize(W, qt, K).astype(np.float64).T
        with O.mul_mat_mode(O.MM_EXACT):
            y = O.mul_mat(qt, W, N, K, x)
        assert np.abs(y - ref).max() <= 1e-6 * np.abs(ref).max()
        g = O.mul_mat(qt, W, N, K, x)
        assert np.abs(g - ref).max() > 0  # the ggml mode rounds the activation
    assert O.get_mul_mat_mode() == O.MM_GGML
