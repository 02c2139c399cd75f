"""Generate the committed golden fixtures under tests/golden/.

Run in the build container (it needs gguf-py and, for the LM fixture, the reference checkout):

    python tests/golden/make_golden.py [--reference /path/to/acestep.cpp]

Fixtures:
  quant_golden.npz  gguf-py 0.19.0 Q8_0 quantize of seeded rows, and gguf-py dequantize of
                    Q8_0 / Q4_K / Q6_K blocks (the blocks themselves are stored too, so the check
                    needs no quantizer). gguf-py's Q8_0 path is documented as bit-exact with
                    ggml-quants.c (gguf/quants.py:378-394).
  philox_golden.npz the reference's own Philox noise (src/philox.h, through tests/test-philox.cpp
                    compiled into oracle/_ref/ by `make -C oracle ref REFERENCE=...`): for each
                    seed its first 8192 bf16 values as uint16 bits, and the SHA-256 of the full
                    192000-value dump (64 channels x 25 Hz x 120 s, the reference test's size).
  lm_golden.npz     a tiny seeded Qwen3 causal LM (F32 weights stored as float16-representable
                    values) and the first-token-position logits of a prompt computed by the
                    reference's own fp32 PyTorch restatement test_pytorch_logits
                    (tests/debug-lm-logits.py:7-136), imported from the reference checkout.
"""
from __future__ import annotations

import argparse
import importlib.util
import json
import os
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def make_quant(rng) -> dict:
    from gguf import quants, GGMLQuantizationType as T

    x = (rng.standard_normal((16, 512)) * 0.02).astype(np.float32)
    x[3, :] = 0.0  # all-zero block row: d = 0 path
    x[5, 7] = 1.0  # outlier
    q8 = quants.quantize(x, T.Q8_0)
    out = {"x": x, "q8_0_bytes": q8, "q8_0_deq": quants.dequantize(q8, T.Q8_0).astype(np.float32)}
    # Q4_K / Q6_K: random but valid block bytes (every bit pattern is a valid block; only the
    # f16 super-scales are forced finite and modest)
    for name, qt, bb in (("q4_k", T.Q4_K, 144), ("q6_k", T.Q6_K, 210)):
        blocks = rng.integers(0, 256, size=(16 * 2, bb), dtype=np.uint8)
        d = (np.abs(rng.standard_normal(16 * 2)) * 1e-3 + 1e-4).astype(np.float16).view(np.uint8).reshape(-1, 2)
        if qt == T.Q4_K:
            blocks[:, 0:2] = d
            dm = (np.abs(rng.standard_normal(16 * 2)) * 1e-3).astype(np.float16).view(np.uint8).reshape(-1, 2)
            blocks[:, 2:4] = dm
        else:
            blocks[:, 208:210] = d
        raw = blocks.reshape(16, 2 * bb)
        out[f"{name}_bytes"] = raw
        out[f"{name}_deq"] = quants.dequantize(raw, qt).astype(np.float32)
    return out


def tiny_lm(rng) -> tuple[dict, dict]:
    cfg = dict(hidden_size=64, intermediate_size=128, num_hidden_layers=2, num_attention_heads=4,
               num_key_value_heads=2, head_dim=16, vocab_size=96, rope_theta=1000000.0, rms_norm_eps=1e-6,
               tie_word_embeddings=True)
    H, F, L = cfg["hidden_size"], cfg["intermediate_size"], cfg["num_hidden_layers"]
    Nh, Nkv, D, V = cfg["num_attention_heads"], cfg["num_key_value_heads"], cfg["head_dim"], cfg["vocab_size"]

    def w(*shape, s=0.08):
        return (rng.standard_normal(shape) * s).astype(np.float16).astype(np.float32)

    def g(n):
        return (1.0 + rng.standard_normal(n) * 0.1).astype(np.float16).astype(np.float32)

    W = {"model.embed_tokens.weight": w(V, H, s=1.0), "model.norm.weight": g(H)}
    for i in range(L):
        p = f"model.layers.{i}"
        W[f"{p}.input_layernorm.weight"] = g(H)
        W[f"{p}.post_attention_layernorm.weight"] = g(H)
        W[f"{p}.self_attn.q_proj.weight"] = w(Nh * D, H)
        W[f"{p}.self_attn.k_proj.weight"] = w(Nkv * D, H)
        W[f"{p}.self_attn.v_proj.weight"] = w(Nkv * D, H)
        W[f"{p}.self_attn.o_proj.weight"] = w(H, Nh * D)
        W[f"{p}.self_attn.q_norm.weight"] = g(D)
        W[f"{p}.self_attn.k_norm.weight"] = g(D)
        W[f"{p}.mlp.gate_proj.weight"] = w(F, H)
        W[f"{p}.mlp.up_proj.weight"] = w(F, H)
        W[f"{p}.mlp.down_proj.weight"] = w(H, F)
    return cfg, W


def make_lm(rng, reference: str) -> dict:
    import torch
    from safetensors.torch import save_file

    path = os.path.join(reference, "tests", "debug-lm-logits.py")
    spec = importlib.util.spec_from_file_location("debug_lm_logits", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)

    cfg, W = tiny_lm(rng)
    prompt = rng.integers(0, cfg["vocab_size"], size=24).astype(np.int64)
    with tempfile.TemporaryDirectory() as d:
        with open(os.path.join(d, "config.json"), "w") as f:
            json.dump(cfg, f)
        save_file({k: torch.from_numpy(v) for k, v in W.items()}, os.path.join(d, "model.safetensors"))
        logits = mod.test_pytorch_logits(d, prompt.tolist())
    out = {"config_json": np.array(json.dumps(cfg)), "prompt": prompt.astype(np.int32),
           "logits": np.asarray(logits, dtype=np.float32)}
    for k, v in W.items():
        out["w:" + k] = v.astype(np.float16)
    return out


PHILOX_SEEDS = [42, 0, 1, -1, 123456789, 2**32 + 5, 2**40 + 7, 9223372036854775807, -9223372036854775808]
PHILOX_FULL = 64 * 25 * 120


def make_philox(reference: str) -> dict:
    import hashlib
    import subprocess
    oracle_dir = os.path.join(HERE, "..", "..", "oracle")
    subprocess.run(["make", "-s", "-C", oracle_dir, "ref", f"REFERENCE={os.path.abspath(reference)}"], check=True)
    exe = os.path.join(oracle_dir, "_ref", "test-philox")
    bits, digests = [], []
    with tempfile.TemporaryDirectory() as td:
        dump = os.path.join(td, "noise.f32")
        for seed in PHILOX_SEEDS:
            subprocess.run([exe, str(seed), str(PHILOX_FULL), dump], check=True, capture_output=True)
            v = np.fromfile(dump, dtype=np.float32)
            assert v.size == PHILOX_FULL and not (v.view(np.uint32) & 0xFFFF).any()  # bf16-representable
            bits.append((v[:8192].view(np.uint32) >> 16).astype(np.uint16))
            digests.append(hashlib.sha256(v.tobytes()).hexdigest())
    return {"seeds": np.array(PHILOX_SEEDS, dtype=np.int64), "bf16_bits": np.stack(bits),
            "full_n": np.int64(PHILOX_FULL), "full_sha256": np.array(digests)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("ACB_REFERENCE"),
                    help="checkout of the reference project (or set ACB_REFERENCE)")
    ap.add_argument("--only", choices=["quant", "lm", "philox"], action="append",
                    help="write only these fixtures (default: all)")
    a = ap.parse_args()
    if not a.reference:
        ap.error("give the reference checkout with --reference or ACB_REFERENCE")
    only = set(a.only or ["quant", "lm", "philox"])
    rng = np.random.default_rng(20261201)
    quant = make_quant(rng)  # drawn first in every run, so the LM fixture sees the same rng state
    if "quant" in only:
        np.savez_compressed(os.path.join(HERE, "quant_golden.npz"), **quant)
    if "lm" in only:
        np.savez_compressed(os.path.join(HERE, "lm_golden.npz"), **make_lm(rng, a.reference))
    if "philox" in only:
        np.savez_compressed(os.path.join(HERE, "philox_golden.npz"), **make_philox(a.reference))
    print("wrote", sorted(os.listdir(HERE)))


if __name__ == "__main__":
    main()
