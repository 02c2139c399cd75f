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

Q8_0, Q4_K, Q6_K, F32, BF16 = acb.Q8_0, acb.Q4_K, acb.Q6_K, acb.F32, acb.BF16

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


def policy_bf16(name: str, layer: int, n_layers: int) -> int:
    """Every matrix BF16, as convert.py stores an unquantised model (the reference's text encoder)."""
    return BF16


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
        if qt == BF16:  # bits of the round-to-nearest-even bf16 values, [N][2K] bytes
            return name, qt, w.to(torch.bfloat16).view(torch.int16).cpu().numpy().view(np.uint8), K
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


# ---- DiT (src/dit.h) ---------------------------------------------------------------------------

ACESTEP_DIT_2B = dict(n_layers=24, hidden_size=2048, intermediate_size=6144, n_heads=16, n_kv_heads=8, head_dim=128,
                      in_channels=192, out_channels=64, patch_size=2, sliding_window=128, rope_theta=1000000.0,
                      rms_norm_eps=1e-6, enc_hidden_size=2048)


def dit_tensors(cfg: dict, qtype: int = Q8_0, seed: int = 0, device: str = "cuda", null_condition: bool = True):
    """Yields (name, qtype, raw, K, shape) of a DiT GGUF in file order, the reference's names and
    the quantize tool's choices (tools/quantize.cpp:97-125): 2-D linears in `qtype`, norms,
    biases, scale_shift_table and null_condition_emb F32, the conv proj_in / proj_out BF16 (their
    innermost dimension, the patch size, is not a block multiple). raw is uint8 [N, row_bytes]
    for quantised tensors, float32 / bf16 bits otherwise; shape is the numpy (PyTorch) shape."""
    import torch
    g = torch.Generator(device=device).manual_seed(seed)
    H, F, L = cfg["hidden_size"], cfg["intermediate_size"], cfg["n_layers"]
    Nh, Nkv, D = cfg["n_heads"], cfg["n_kv_heads"], cfg["head_dim"]
    in_ch, oc, P, He = cfg["in_channels"], cfg["out_channels"], cfg["patch_size"], cfg["enc_hidden_size"]

    def mat(name, N, K, std=0.02):
        w = torch.randn((N, K), generator=g, device=device) * std
        return name, qtype, quantize_on_device(w, qtype), K, (N, K)

    def vec(name, shape, base=0.0, std=0.02):
        v = (base + std * torch.randn(shape, generator=g, device=device)).cpu().numpy().astype(np.float32)
        return name, F32, v, shape[-1], shape

    def conv_bf16(name, shape):
        w = (torch.randn(shape, generator=g, device=device) * 0.02).to(torch.bfloat16)
        return name, acb.BF16, w.view(torch.int16).cpu().numpy().view(np.uint16), shape[-1], shape

    for te in ("decoder.time_embed", "decoder.time_embed_r"):
        yield mat(f"{te}.linear_1.weight", H, 256)
        yield vec(f"{te}.linear_1.bias", (H,))
        yield mat(f"{te}.linear_2.weight", H, H)
        yield vec(f"{te}.linear_2.bias", (H,))
        yield mat(f"{te}.time_proj.weight", 6 * H, H)
        yield vec(f"{te}.time_proj.bias", (6 * H,))
    yield conv_bf16("decoder.proj_in.1.weight", (H, in_ch, P))
    yield vec("decoder.proj_in.1.bias", (H,))
    yield mat("decoder.condition_embedder.weight", H, He)
    yield vec("decoder.condition_embedder.bias", (H,))
    for i in range(L):
        p = f"decoder.layers.{i}"
        yield vec(f"{p}.self_attn_norm.weight", (H,), 1.0, 0.01)
        yield mat(f"{p}.self_attn.q_proj.weight", Nh * D, H)
        yield mat(f"{p}.self_attn.k_proj.weight", Nkv * D, H)
        yield mat(f"{p}.self_attn.v_proj.weight", Nkv * D, H)
        yield mat(f"{p}.self_attn.o_proj.weight", H, Nh * D)
        yield vec(f"{p}.self_attn.q_norm.weight", (D,), 1.0, 0.01)
        yield vec(f"{p}.self_attn.k_norm.weight", (D,), 1.0, 0.01)
        yield vec(f"{p}.cross_attn_norm.weight", (H,), 1.0, 0.01)
        yield mat(f"{p}.cross_attn.q_proj.weight", Nh * D, H)
        yield mat(f"{p}.cross_attn.k_proj.weight", Nkv * D, H)
        yield mat(f"{p}.cross_attn.v_proj.weight", Nkv * D, H)
        yield mat(f"{p}.cross_attn.o_proj.weight", H, Nh * D)
        yield vec(f"{p}.cross_attn.q_norm.weight", (D,), 1.0, 0.01)
        yield vec(f"{p}.cross_attn.k_norm.weight", (D,), 1.0, 0.01)
        yield vec(f"{p}.mlp_norm.weight", (H,), 1.0, 0.01)
        yield mat(f"{p}.mlp.gate_proj.weight", F, H)
        yield mat(f"{p}.mlp.up_proj.weight", F, H)
        yield mat(f"{p}.mlp.down_proj.weight", H, F)
        yield vec(f"{p}.scale_shift_table", (1, 6, H), 0.0, 0.05)
    yield vec("decoder.norm_out.weight", (H,), 1.0, 0.01)
    yield vec("decoder.scale_shift_table", (1, 2, H), 0.0, 0.05)
    yield conv_bf16("decoder.proj_out.1.weight", (H, oc, P))
    yield vec("decoder.proj_out.1.bias", (oc,))
    if null_condition:
        yield vec("null_condition_emb", (He,), 0.0, 1.0)


# Condition encoder and FSQ models (src/cond-enc.h, src/fsq-tok.h, src/fsq-detok.h): the
# reference's sizes, and a small stand-in for parity tests against the oracle.
ACESTEP_COND = dict(hidden_size=2048, intermediate_size=6144, n_heads=16, n_kv_heads=8, head_dim=128,
                    lyric_layers=8, timbre_layers=4, tok_layers=2, detok_layers=2, text_dim=1024, lyric_dim=1024,
                    latent_dim=64)
COND_TINY = dict(hidden_size=256, intermediate_size=512, n_heads=4, n_kv_heads=2, head_dim=128, lyric_layers=2,
                 timbre_layers=2, tok_layers=2, detok_layers=2, text_dim=256, lyric_dim=256, latent_dim=64)


def _block_of(qtype: int) -> int:
    return {Q8_0: 32, Q4_K: 256, Q6_K: 256}.get(qtype, 1)


def cond_tensors(ccfg: dict, qtype: int = Q8_0, seed: int = 0, device: str = "cuda", timbre_cls: bool = False):
    """Yields (name, qtype, raw, K, shape) of the encoder.*, tokenizer.* and detokenizer.* tensors of
    a DiT GGUF with the quantize tool's choices (tools/quantize.cpp:97-171): 2-D tensors whose
    innermost size is a block multiple in `qtype` (the detokenizer's special_tokens [1, 5, H]
    included), the rest BF16 (project_out [H, 6], and the 64-wide inputs under K-quants); 1-D
    tensors (norms, biases, the [H] learned tokens) F32."""
    import torch
    g = torch.Generator(device=device).manual_seed(seed)
    H, F, Nh, Nkv, D = (ccfg[k] for k in ("hidden_size", "intermediate_size", "n_heads", "n_kv_heads", "head_dim"))

    def mat(name, shape, std=0.02):
        K = shape[-1]
        rows = int(np.prod(shape[:-1]))
        w = torch.randn((rows, K), generator=g, device=device) * std
        if K % _block_of(qtype) == 0:
            return name, qtype, quantize_on_device(w, qtype), K, shape
        b = w.to(torch.bfloat16).view(torch.int16).cpu().numpy().view(np.uint16).reshape(shape)
        return name, acb.BF16, b, K, shape

    def vec(name, n, base=0.0, std=0.02):
        v = (base + std * torch.randn(n, generator=g, device=device)).cpu().numpy().astype(np.float32)
        return name, F32, v, n, (n,)

    def stack(prefix, L):
        for i in range(L):
            p = f"{prefix}layers.{i}"
            yield vec(f"{p}.input_layernorm.weight", H, 1.0, 0.01)
            yield vec(f"{p}.post_attention_layernorm.weight", H, 1.0, 0.01)
            yield mat(f"{p}.self_attn.q_proj.weight", (Nh * D, H))
            yield mat(f"{p}.self_attn.k_proj.weight", (Nkv * D, H))
            yield mat(f"{p}.self_attn.v_proj.weight", (Nkv * D, H))
            yield mat(f"{p}.self_attn.o_proj.weight", (H, Nh * D))
            yield vec(f"{p}.self_attn.q_norm.weight", D, 1.0, 0.01)
            yield vec(f"{p}.self_attn.k_norm.weight", D, 1.0, 0.01)
            yield mat(f"{p}.mlp.gate_proj.weight", (F, H))
            yield mat(f"{p}.mlp.up_proj.weight", (F, H))
            yield mat(f"{p}.mlp.down_proj.weight", (H, F))
        yield vec(f"{prefix}norm.weight", H, 1.0, 0.01)

    C = ccfg["latent_dim"]
    yield mat("encoder.lyric_encoder.embed_tokens.weight", (H, ccfg["lyric_dim"]))
    yield vec("encoder.lyric_encoder.embed_tokens.bias", H)
    yield from stack("encoder.lyric_encoder.", ccfg["lyric_layers"])
    yield mat("encoder.timbre_encoder.embed_tokens.weight", (H, C))
    yield vec("encoder.timbre_encoder.embed_tokens.bias", H)
    yield from stack("encoder.timbre_encoder.", ccfg["timbre_layers"])
    if timbre_cls:
        yield vec("encoder.timbre_encoder.special_token", H, 0.0, 1.0)
    yield mat("encoder.text_projector.weight", (H, ccfg["text_dim"]))
    yield mat("tokenizer.audio_acoustic_proj.weight", (H, C))
    yield vec("tokenizer.audio_acoustic_proj.bias", H)
    yield mat("tokenizer.attention_pooler.embed_tokens.weight", (H, H))
    yield vec("tokenizer.attention_pooler.embed_tokens.bias", H)
    yield vec("tokenizer.attention_pooler.special_token", H, 0.0, 1.0)
    yield from stack("tokenizer.attention_pooler.", ccfg["tok_layers"])
    # project_in drives the FSQ levels: a larger spread so that every level occurs
    yield mat("tokenizer.quantizer.project_in.weight", (6, H), 0.05)
    yield vec("tokenizer.quantizer.project_in.bias", 6, 0.0, 0.2)
    yield mat("tokenizer.quantizer.project_out.weight", (H, 6), 0.5)
    yield vec("tokenizer.quantizer.project_out.bias", H)
    yield mat("detokenizer.embed_tokens.weight", (H, H))
    yield vec("detokenizer.embed_tokens.bias", H)
    yield mat("detokenizer.special_tokens", (1, 5, H), 1.0)
    yield from stack("detokenizer.", ccfg["detok_layers"])
    yield mat("detokenizer.proj_out.weight", (C, H))
    yield vec("detokenizer.proj_out.bias", C)


def write_dit_gguf(path: str, cfg: dict, qtype: int = Q8_0, seed: int = 0, device: str = "cuda",
                   keep: dict | None = None, null_condition: bool = True, cond: dict | None = None,
                   timbre_cls: bool = False, decoder: bool = True) -> int:
    """Write a DiT GGUF with the reference's metadata keys (dit.h:276-287). If `keep` is a dict,
    the raw tensors are stored in it as name -> (qtype, raw, K, shape). `cond` (a COND_TINY-like
    dict) adds the condition encoder and FSQ tensors; timbre_cls writes the XL models'
    acestep.encoder_hidden_size key and timbre special_token; decoder False leaves the
    decoder.* tensors out (only null_condition_emb stays)."""
    import gguf
    w = gguf.GGUFWriter(path, "acestep-dit")
    a = "acestep-dit"
    w.add_uint32(f"{a}.block_count", cfg["n_layers"])
    w.add_uint32(f"{a}.embedding_length", cfg["hidden_size"])
    w.add_uint32(f"{a}.feed_forward_length", cfg["intermediate_size"])
    w.add_uint32(f"{a}.attention.head_count", cfg["n_heads"])
    w.add_uint32(f"{a}.attention.head_count_kv", cfg["n_kv_heads"])
    w.add_uint32(f"{a}.attention.key_length", cfg["head_dim"])
    w.add_float32(f"{a}.rope.freq_base", cfg["rope_theta"])
    w.add_float32(f"{a}.attention.layer_norm_rms_epsilon", cfg["rms_norm_eps"])
    w.add_uint32("acestep.in_channels", cfg["in_channels"])
    w.add_uint32("acestep.audio_acoustic_hidden_dim", cfg["out_channels"])
    w.add_uint32("acestep.patch_size", cfg["patch_size"])
    w.add_uint32("acestep.sliding_window", cfg["sliding_window"])
    if timbre_cls:
        w.add_uint32("acestep.encoder_hidden_size", cfg["enc_hidden_size"])
    total = 0

    def all_tensors():
        for t in dit_tensors(cfg, qtype, seed, device, null_condition):
            if decoder or not t[0].startswith("decoder."):
                yield t
        if cond is not None:
            yield from cond_tensors(cond, qtype, seed + 7, device, timbre_cls)

    for name, qt, raw, K, shape in all_tensors():
        if qt == F32:
            w.add_tensor(name, raw)
        elif qt == acb.BF16:
            w.add_tensor(name, raw.view(np.uint8).reshape(*shape[:-1], shape[-1] * 2),
                         raw_dtype=gguf.GGMLQuantizationType.BF16)
        else:
            w.add_tensor(name, raw, raw_dtype=gguf.GGMLQuantizationType(qt))
        total += raw.nbytes
        if keep is not None:
            keep[name] = (qt, raw, K, shape)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return total


# ---- VAE decoder (src/vae.h) ---------------------------------------------------------------------

ACESTEP_VAE = dict(latent=64, c0=2048, in_ch=[2048, 1024, 512, 256, 128], out_ch=[1024, 512, 256, 128, 128],
                   strides=[10, 6, 4, 4, 2])
VAE_TINY = dict(latent=64, c0=256, in_ch=[256, 128, 128, 64, 64], out_ch=[128, 128, 64, 64, 64],
                strides=[10, 6, 4, 4, 2])


def vae_tensors(vcfg: dict, seed: int = 0):
    """Yields (name, numpy float32 array in PyTorch shape) of an AutoencoderOobleck decoder with the
    reference's GGUF names (vae.h:229-255): weight-normalised convs (weight_g [OC,1,1], weight_v),
    biases, snake alpha / beta [1, C, 1]. Stored BF16 by write_vae_gguf, as convert.py does.
    Conditioned like a trained residual decoder, so that rounding differences stay small at the
    output: residual branches end in a small gain (conv2 weight_g 0.1-0.3) and the snake's
    periodic term is damped (beta around 1, e^-beta around 0.37). With unit gains everywhere a
    1e-6 input perturbation moved the output by 2e-2 at this depth."""
    rng = np.random.default_rng(seed)

    def wn(pfx, shape, dim0, g=(0.6, 1.2)):
        yield f"{pfx}.weight_g", rng.uniform(g[0], g[1], (dim0, 1, 1)).astype(np.float32)
        yield f"{pfx}.weight_v", rng.standard_normal(shape).astype(np.float32)

    def snake(pfx, C):
        yield f"{pfx}.alpha", (0.2 * rng.standard_normal((1, C, 1))).astype(np.float32)
        yield f"{pfx}.beta", (1.0 + 0.2 * rng.standard_normal((1, C, 1))).astype(np.float32)

    c0, L = vcfg["c0"], vcfg["latent"]
    yield from wn("decoder.conv1", (c0, L, 7), c0)
    yield "decoder.conv1.bias", (0.05 * rng.standard_normal(c0)).astype(np.float32)
    for i, (ic, oc, s) in enumerate(zip(vcfg["in_ch"], vcfg["out_ch"], vcfg["strides"])):
        p = f"decoder.block.{i}"
        yield from snake(f"{p}.snake1", ic)
        yield from wn(f"{p}.conv_t1", (ic, oc, 2 * s), ic)
        yield f"{p}.conv_t1.bias", (0.05 * rng.standard_normal(oc)).astype(np.float32)
        for r in range(1, 4):
            rp = f"{p}.res_unit{r}"
            yield from snake(f"{rp}.snake1", oc)
            yield from wn(f"{rp}.conv1", (oc, oc, 7), oc)
            yield f"{rp}.conv1.bias", (0.05 * rng.standard_normal(oc)).astype(np.float32)
            yield from snake(f"{rp}.snake2", oc)
            yield from wn(f"{rp}.conv2", (oc, oc, 1), oc, g=(0.1, 0.3))
            yield f"{rp}.conv2.bias", (0.05 * rng.standard_normal(oc)).astype(np.float32)
    cl = vcfg["out_ch"][-1]
    yield from snake("decoder.snake1", cl)
    yield from wn("decoder.conv2", (2, cl, 7), 2)


def write_vae_gguf(path: str, vcfg: dict, seed: int = 0, keep: dict | None = None) -> int:
    """An acestep-vae GGUF with every tensor BF16 (rounded to nearest even). keep receives
    name -> bf16 bits (numpy uint16, PyTorch shape)."""
    import gguf
    w = gguf.GGUFWriter(path, "acestep-vae")
    total = 0
    for name, a in vae_tensors(vcfg, seed):
        u = a.view(np.uint32)  # finite values: u + 0x8000 stays below 2^32
        bits = ((u + (np.uint32(0x7FFF) + ((u >> 16) & np.uint32(1)))) >> 16).astype(np.uint16)
        w.add_tensor(name, bits.view(np.uint8).reshape(*a.shape[:-1], a.shape[-1] * 2),
                     raw_dtype=gguf.GGMLQuantizationType.BF16)
        total += bits.nbytes
        if keep is not None:
            keep[name] = bits
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return total
