"""GPU: models in the unquantised layout the reference's converter writes (`convert.py`,
`add_metadata` and `add_tensors_from_sf`: tensors in sorted name order, BF16 sources as BF16, F16
as F16, F32 sources truncated to BF16 -- 1-D norms, biases and tables included -- the
`acestep-*` architecture names, the llama-style keys, `acestep.config_json` in compact form), loaded
through the C ABI and compared with the oracle on the same tensors (1-D tensors promoted to F32
as gf_load_tensor_f32 does):

- the LM (BF16 weights, tied head): prefill logits bit-identical and 24 greedy tokens identical
  (the BF16 decode GEMV adds the exact bf16 products in double, the canonical rule);
- the text encoder: row cosine >= 0.9999, max_rel <= 1e-2;
- the DiT (BF16 weights, scale/shift tables and null condition stored BF16): one CFG generate at
  the DiT bars.
The writer below restates the converter's rules (the layout is the format); nothing runs the
reference's script."""
import json
import os

import numpy as np
import pytest

import acb
import oracle as O
from helpers import assert_bitexact, cos_sim, max_rel

pytestmark = pytest.mark.gpu


def _to_bf16_truncate(a: np.ndarray) -> np.ndarray:
    """convert.py's F32 -> BF16: drop the low 16 bits (truncation, not rounding)."""
    return (np.ascontiguousarray(a, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)


def write_convert_style(path, arch, cfg, tensors, f16_names=(), model_type="lm", extra=None):
    """tensors: name -> float32 array in PyTorch shape. Returns {name: (qtype, raw, K, shape)} as
    stored (BF16 bits, or F16 for f16_names)."""
    import gguf
    w = gguf.GGUFWriter(path, arch)
    for key, fn in (("num_hidden_layers", w.add_block_count), ("hidden_size", w.add_embedding_length),
                    ("intermediate_size", w.add_feed_forward_length), ("num_attention_heads", w.add_head_count),
                    ("num_key_value_heads", w.add_head_count_kv), ("head_dim", w.add_key_length),
                    ("vocab_size", w.add_vocab_size), ("rms_norm_eps", w.add_layer_norm_rms_eps)):
        if key in cfg:
            fn(cfg[key])
    if cfg.get("rope_theta"):
        w.add_rope_freq_base(float(cfg["rope_theta"]))
    if model_type == "lm" and cfg.get("tie_word_embeddings"):
        w.add_bool("acestep.tie_word_embeddings", True)
    for k, v in (extra or {}).items():
        w.add_uint32(f"acestep.{k}", v)
    w.add_string("acestep.config_json", json.dumps(cfg, separators=(",", ":")))
    stored = {}
    for name in sorted(tensors):
        a = np.asarray(tensors[name], dtype=np.float32)
        K = a.shape[-1]
        if name in f16_names:
            raw = a.astype(np.float16)
            w.add_tensor(name, raw)
            stored[name] = (acb.F16, raw.view(np.uint16), K, a.shape)
        else:
            raw = _to_bf16_truncate(a)
            w.add_tensor(name, raw, raw_dtype=gguf.GGMLQuantizationType.BF16)
            stored[name] = (acb.BF16, raw, K, a.shape)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return stored


def _f32(entry):
    qt, raw, K, shape = entry
    if qt == acb.BF16:
        return O.bf16_bits_to_f32(raw).reshape(shape)
    if qt == acb.F16:
        return raw.view(np.float16).astype(np.float32).reshape(shape)
    return np.asarray(raw, np.float32).reshape(shape)


def _qwen3_f32_tensors(cfg, rng, prefix, embed=True):
    H, F, L = cfg["hidden_size"], cfg["intermediate_size"], cfg["num_hidden_layers"]
    Nh, Nkv, D = cfg["num_attention_heads"], cfg["num_key_value_heads"], cfg["head_dim"]
    t = {}
    if embed:
        t[f"{prefix}embed_tokens.weight"] = rng.standard_normal((cfg["vocab_size"], H)) * 0.5
    t[f"{prefix}norm.weight"] = 1 + 0.01 * rng.standard_normal(H)
    for i in range(L):
        p = f"{prefix}layers.{i}"
        t[f"{p}.input_layernorm.weight"] = 1 + 0.01 * rng.standard_normal(H)
        t[f"{p}.post_attention_layernorm.weight"] = 1 + 0.01 * rng.standard_normal(H)
        t[f"{p}.self_attn.q_proj.weight"] = rng.standard_normal((Nh * D, H)) * 0.02
        t[f"{p}.self_attn.k_proj.weight"] = rng.standard_normal((Nkv * D, H)) * 0.02
        t[f"{p}.self_attn.v_proj.weight"] = rng.standard_normal((Nkv * D, H)) * 0.02
        t[f"{p}.self_attn.o_proj.weight"] = rng.standard_normal((H, Nh * D)) * 0.02
        t[f"{p}.self_attn.q_norm.weight"] = 1 + 0.01 * rng.standard_normal(D)
        t[f"{p}.self_attn.k_norm.weight"] = 1 + 0.01 * rng.standard_normal(D)
        t[f"{p}.mlp.gate_proj.weight"] = rng.standard_normal((F, H)) * 0.02
        t[f"{p}.mlp.up_proj.weight"] = rng.standard_normal((F, H)) * 0.02
        t[f"{p}.mlp.down_proj.weight"] = rng.standard_normal((H, F)) * 0.02
    return t


def _view4(stored):
    """(qtype, raw [N][K], K, N) per tensor for the oracle's Qwen3 model, 1-D tensors as F32."""
    out = {}
    for name, (qt, raw, K, shape) in stored.items():
        N = int(np.prod(shape)) // K
        if len(shape) == 1:
            out[name] = (O.F32, _f32((qt, raw, K, shape)), K, 1)
        else:
            out[name] = (qt, np.ascontiguousarray(raw).reshape(N, K), K, N)
    return out


def test_lm_bf16_convert_layout(cuda, tmp_path):
    import lm_fixtures as F
    cfg = dict(F.TINY)
    rng = np.random.default_rng(61)
    t = _qwen3_f32_tensors(cfg, rng, "model.")
    path = str(tmp_path / "lm-BF16.gguf")
    stored = write_convert_style(path, "acestep-lm", cfg, t)
    m = acb.QW3LM(path, max_seq_len=128, n_kv_sets=1)
    assert not m.persistent_decode()  # BF16 weights take the per-op graph
    ora = F.oracle_model(cfg, _view4(stored))
    ora.alloc_kv(1, 128)
    prompt = rng.integers(0, cfg["vocab_size"], 40).astype(np.int32)
    lg = m.forward(prompt, kv_set=0)
    lr = ora.prefill(prompt, set_=0)
    assert_bitexact(lg, lr, "BF16 prefill logits")
    first = int(np.argmax(lr))
    toks, _, _ = m.generate_greedy([first], 0, 24)
    nxt, otoks = first, []
    for _ in range(24):
        nxt = int(np.argmax(ora.decode(np.array([nxt], np.int32), set0=0)[0]))
        otoks.append(nxt)
    assert toks[0].tolist() == otoks
    m.close()


def test_text_encoder_bf16_convert_layout(cuda, tmp_path):
    import lm_fixtures as F
    cfg = dict(F.TINY, num_hidden_layers=3)
    rng = np.random.default_rng(62)
    t = _qwen3_f32_tensors(cfg, rng, "")
    path = str(tmp_path / "Qwen3-Embedding-BF16.gguf")
    stored = write_convert_style(path, "acestep-text-enc", cfg, t, model_type="text-enc")
    enc = acb.Qwen3Encoder(path)
    ora = O.qwen3_from_gguf_tensors(cfg, _view4(stored), prefix="")
    ids = rng.integers(0, cfg["vocab_size"], 70).astype(np.int32)
    got = enc.forward(ids)
    ref = ora.encode(ids)
    for r in range(ids.size):
        c, e = cos_sim(got[r], ref[r]), max_rel(got[r], ref[r])
        assert c >= 0.9999 and e <= 1e-2, (r, c, e)
    enc.close()


def _dit_f32_tensors(cfg, rng):
    H, F, L = cfg["hidden_size"], cfg["intermediate_size"], cfg["n_layers"]
    Nh, Nkv, D = cfg["n_heads"], cfg["n_kv_heads"], cfg["head_dim"]
    in_ch, oc, P, He = cfg["in_channels"], cfg["out_channels"], cfg["patch_size"], cfg["enc_hidden_size"]
    m = lambda *s: rng.standard_normal(s) * 0.02
    g = lambda n: 1 + 0.01 * rng.standard_normal(n)
    t = {}
    for te in ("decoder.time_embed", "decoder.time_embed_r"):
        t[f"{te}.linear_1.weight"], t[f"{te}.linear_1.bias"] = m(H, 256), m(H)
        t[f"{te}.linear_2.weight"], t[f"{te}.linear_2.bias"] = m(H, H), m(H)
        t[f"{te}.time_proj.weight"], t[f"{te}.time_proj.bias"] = m(6 * H, H), m(6 * H)
    t["decoder.proj_in.1.weight"], t["decoder.proj_in.1.bias"] = m(H, in_ch, P), m(H)
    t["decoder.condition_embedder.weight"], t["decoder.condition_embedder.bias"] = m(H, He), m(H)
    for i in range(L):
        p = f"decoder.layers.{i}"
        for a in ("self_attn", "cross_attn"):
            t[f"{p}.{a}.q_proj.weight"] = m(Nh * D, H)
            t[f"{p}.{a}.k_proj.weight"] = m(Nkv * D, H)
            t[f"{p}.{a}.v_proj.weight"] = m(Nkv * D, H)
            t[f"{p}.{a}.o_proj.weight"] = m(H, Nh * D)
            t[f"{p}.{a}.q_norm.weight"], t[f"{p}.{a}.k_norm.weight"] = g(D), g(D)
        t[f"{p}.self_attn_norm.weight"], t[f"{p}.cross_attn_norm.weight"] = g(H), g(H)
        t[f"{p}.mlp_norm.weight"] = g(H)
        t[f"{p}.mlp.gate_proj.weight"], t[f"{p}.mlp.up_proj.weight"] = m(F, H), m(F, H)
        t[f"{p}.mlp.down_proj.weight"] = m(H, F)
        t[f"{p}.scale_shift_table"] = rng.standard_normal((1, 6, H)) * 0.05
    t["decoder.norm_out.weight"] = g(H)
    t["decoder.scale_shift_table"] = rng.standard_normal((1, 2, H)) * 0.05
    t["decoder.proj_out.1.weight"], t["decoder.proj_out.1.bias"] = m(H, oc, P), m(oc)
    t["null_condition_emb"] = rng.standard_normal((1, 1, He))
    return t


def test_dit_bf16_convert_layout(cuda, tmp_path):
    cfg = dict(n_layers=2, hidden_size=256, intermediate_size=512, n_heads=4, n_kv_heads=2, head_dim=128,
               in_channels=64, out_channels=32, patch_size=2, sliding_window=16, rope_theta=1000000.0,
               rms_norm_eps=1e-6, enc_hidden_size=256)
    hf = dict(num_hidden_layers=2, hidden_size=256, intermediate_size=512, num_attention_heads=4,
              num_key_value_heads=2, head_dim=128, rope_theta=1000000.0, rms_norm_eps=1e-6, in_channels=64,
              audio_acoustic_hidden_dim=32, patch_size=2, sliding_window=16)
    rng = np.random.default_rng(63)
    t = _dit_f32_tensors(cfg, rng)
    path = str(tmp_path / "acestep-v15-turbo-BF16.gguf")
    stored = write_convert_style(path, "acestep-dit", hf, t, model_type="dit",
                                 extra={k: hf[k] for k in ("in_channels", "audio_acoustic_hidden_dim", "patch_size",
                                                           "sliding_window")})
    ov = {n: ((O.F32, _f32(e).reshape(-1), e[2], e[3]) if len(e[3]) == 1 else e) for n, e in stored.items()}
    od = O.dit_from_gguf_tensors(cfg, ov)
    null = _f32(stored["null_condition_emb"]).reshape(-1)
    dit = acb.DiT(path)
    N, T, enc_S, Oc = 2, 48, 20, cfg["out_channels"]
    noise = rng.standard_normal((N, T, Oc)).astype(np.float32)
    ctx = rng.standard_normal((N, T, cfg["in_channels"] - Oc)).astype(np.float32)
    enc = rng.standard_normal((N, enc_S, cfg["enc_hidden_size"])).astype(np.float32)
    got, _ = dit.generate_ex(noise, ctx, enc, acb.turbo_schedule(4), guidance_scale=3.0)
    ref = O.dit_generate(od, noise, ctx, enc, null, acb.turbo_schedule(4), 3.0)
    for b in range(N):
        c, e = cos_sim(got[b], ref[b]), max_rel(got[b], ref[b])
        assert c >= 0.9999 and e <= 1e-2, (b, c, e)
    dit.close()
