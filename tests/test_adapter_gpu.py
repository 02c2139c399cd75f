"""GPU: LoRA merge at load (src/adapter-merge.h) against the oracle's restatement.

- kernel level: dequantise -> acb_lora_delta_add -> acb_requant gives the oracle's merged bytes
  bit for bit (Q8_0 and BF16 bases; A / B given in F32 and BF16);
- model level: acb_dit_load_ex with a PEFT directory (adapter_model.safetensors with
  base_model.model.layers.* keys, adapter_config.json lora_alpha) and with a ComfyUI single file
  (diffusion_model.* keys, lora_down / lora_up, per-tensor alpha scalars) generates what the
  oracle generates from the merged tensors, at the DiT bars (cosine >= 0.9999, max_rel <= 1e-2),
  and differs from the unmerged model;
- a LoKr payload is refused with ACB_ERR_UNSUPPORTED.
Safetensors files are written here by a small writer of the format (8-byte header length, JSON
header, data)."""
import json
import os
import struct

import numpy as np
import pytest

import acb
import oracle as O
from helpers import cos_sim, max_rel

pytestmark = pytest.mark.gpu

DIT = dict(n_layers=2, hidden_size=256, intermediate_size=512, n_heads=4, n_kv_heads=2, head_dim=128,
           in_channels=64, out_channels=32, patch_size=2, sliding_window=16, rope_theta=1000000.0,
           rms_norm_eps=1e-6, enc_hidden_size=256)


def write_safetensors(path, tensors, metadata=None):
    """tensors: name -> (dtype "F32" / "BF16" / "F16", numpy array of that storage)."""
    header, blobs, off = {}, [], 0
    for name, (dt, arr) in tensors.items():
        b = np.ascontiguousarray(arr).tobytes()
        header[name] = {"dtype": dt, "shape": list(arr.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    if metadata:
        header["__metadata__"] = metadata
    h = json.dumps(header).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def _bf16(a):
    return O.f32_to_bf16_bits(np.asarray(a, np.float32))


@pytest.mark.parametrize("qt", [acb.Q8_0, acb.BF16])
def test_lora_merge_kernels_bitexact(cuda, qt):
    import torch
    rng = np.random.default_rng(5 + qt)
    N, K, r = 384, 512, 16
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    raw = O.quantize(w, qt) if qt != acb.BF16 else _bf16(w)
    entry = (qt, raw, K, (N, K))
    A = (rng.standard_normal((r, K)) * 0.05).astype(np.float32)
    B = (rng.standard_normal((N, r)) * 0.05).astype(np.float32)
    scaling = O.lora_scaling(32, r, 0.7)
    _, ref_raw, _ = O.lora_merge(entry, A, B, scaling)
    d_raw = torch.from_numpy(np.ascontiguousarray(raw).view(np.uint8).copy()).cuda()
    ids = torch.arange(N, dtype=torch.int32, device="cuda")
    tmp = torch.empty((N, K), dtype=torch.float32, device="cuda")
    acb._check("acb_get_rows", acb.lib().acb_get_rows(d_raw.data_ptr(), qt, N, K, ids.data_ptr(), N, tmp.data_ptr(),
                                                      acb.F32, K, None, acb._stream(None)))
    dA = torch.from_numpy(O.round_bf16(A)).cuda()
    dB = torch.from_numpy(O.round_bf16(B)).cuda()
    acb._check("acb_lora_delta_add", acb.lib().acb_lora_delta_add(tmp.data_ptr(), N, K, dA.data_ptr(), dB.data_ptr(),
                                                                  r, float(scaling), acb._stream(None)))
    out = torch.empty_like(d_raw)
    acb._check("acb_requant", acb.lib().acb_requant(tmp.data_ptr(), N, K, qt, out.data_ptr(), acb._stream(None)))
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    want = np.ascontiguousarray(ref_raw).view(np.uint8).reshape(-1)
    assert np.array_equal(got.reshape(-1), want)


TARGETS = [("layers.0.self_attn.q_proj", 512, 256), ("layers.0.self_attn.v_proj", 256, 256),
           ("layers.1.cross_attn.o_proj", 256, 512), ("layers.1.mlp.down_proj", 256, 512)]


def _adapter_factors(rng, r):
    return {t: ((rng.standard_normal((r, K)) * 0.2).astype(np.float32),
                (rng.standard_normal((N, r)) * 0.2).astype(np.float32)) for t, N, K in TARGETS}


def _merged_keep(keep, factors, alphas, r, scale):
    out = dict(keep)
    for t, (A, B) in factors.items():
        name = f"decoder.{t}.weight"
        qt, raw, K, shape = keep[name]
        _, mraw, _ = O.lora_merge((qt, raw, K, shape), A, B, O.lora_scaling(alphas[t], r, scale))
        out[name] = (qt, np.ascontiguousarray(mraw).reshape(raw.shape), K, shape)
    return out


def _run(dit, rng_seed):
    rng = np.random.default_rng(rng_seed)
    N, T, enc_S, Oc = 2, 48, 20, DIT["out_channels"]
    noise = rng.standard_normal((N, T, Oc)).astype(np.float32)
    ctx = rng.standard_normal((N, T, DIT["in_channels"] - Oc)).astype(np.float32)
    enc = rng.standard_normal((N, enc_S, DIT["enc_hidden_size"])).astype(np.float32)
    return noise, ctx, enc


@pytest.fixture(scope="module")
def dit_file(tmp_path_factory, cuda):
    import synthetic
    path = os.path.join(str(tmp_path_factory.mktemp("dit")), "dit.gguf")
    keep = {}
    synthetic.write_dit_gguf(path, DIT, synthetic.Q8_0, seed=71, device="cuda", keep=keep)
    return path, keep


def _check_generate(path, adapter, scale, keep_merged, keep):
    dit = acb.DiT(path, adapter=adapter, adapter_scale=scale)
    noise, ctx, enc = _run(dit, 3)
    got, _ = dit.generate_ex(noise, ctx, enc, acb.turbo_schedule(4), guidance_scale=3.0)
    dit.close()
    null = keep["null_condition_emb"][1].astype(np.float32)
    ref = O.dit_generate(O.dit_from_gguf_tensors(DIT, keep_merged), noise, ctx, enc, null, acb.turbo_schedule(4), 3.0)
    base = O.dit_generate(O.dit_from_gguf_tensors(DIT, keep), noise, ctx, enc, null, acb.turbo_schedule(4), 3.0)
    for b in range(noise.shape[0]):
        c, e = cos_sim(got[b], ref[b]), max_rel(got[b], ref[b])
        assert c >= 0.9999 and e <= 1e-2, (b, c, e)
    assert max_rel(ref, base) > 1e-2  # the adapter changes the model


def test_dit_peft_directory(dit_file, tmp_path):
    path, keep = dit_file
    rng = np.random.default_rng(11)
    r, alpha, scale = 8, 16, 0.8
    fac = _adapter_factors(rng, r)
    d = tmp_path / "peft"
    d.mkdir()
    tens = {}
    for i, (t, (A, B)) in enumerate(fac.items()):
        if i % 2 == 0:  # BF16 storage for half of them
            tens[f"base_model.model.{t}.lora_A.weight"] = ("BF16", _bf16(A))
            tens[f"base_model.model.{t}.lora_B.weight"] = ("BF16", _bf16(B))
        else:
            tens[f"base_model.model.{t}.lora_A.default.weight"] = ("F32", A)
            tens[f"base_model.model.{t}.lora_B.default.weight"] = ("F32", B)
    write_safetensors(str(d / "adapter_model.safetensors"), tens, {"format": "pt"})
    (d / "adapter_config.json").write_text(json.dumps({"r": r, "lora_alpha": alpha, "target_modules": ["q_proj"]}))
    merged = _merged_keep(keep, fac, {t: alpha for t in fac}, r, scale)
    _check_generate(path, str(d), scale, merged, keep)


def test_dit_comfyui_file_with_alpha_scalars(dit_file, tmp_path):
    path, keep = dit_file
    rng = np.random.default_rng(12)
    r = 4
    fac = _adapter_factors(rng, r)
    alphas = {t: float(2 + i) for i, t in enumerate(fac)}
    tens = {}
    for t, (A, B) in fac.items():
        tens[f"diffusion_model.{t}.lora_down.weight"] = ("F32", A)
        tens[f"diffusion_model.{t}.lora_up.weight"] = ("F32", B)
        tens[f"diffusion_model.{t}.alpha"] = ("F32", np.array(alphas[t], dtype=np.float32).reshape(()))
    f = str(tmp_path / "lora_comfy.safetensors")
    write_safetensors(f, tens)
    merged = _merged_keep(keep, fac, alphas, r, 1.0)
    _check_generate(path, f, 1.0, merged, keep)


def test_lokr_refused(dit_file, tmp_path):
    path, _ = dit_file
    f = str(tmp_path / "lokr.safetensors")
    write_safetensors(f, {"layers.0.self_attn.q_proj.lokr_w1": ("F32", np.ones((4, 4), np.float32))})
    with pytest.raises(acb.AcbError) as e:
        acb.DiT(path, adapter=f)
    assert e.value.status == 2
