"""GPU: LoRA merge at load (src/adapter-merge.h) against the oracle's restatement.

- kernel level: dequantise -> acb_lora_delta_add -> acb_requant gives the oracle's merged bytes
  bit for bit (Q8_0 and BF16 bases; A / B given in F32 and BF16);
- model level: acb_dit_load_ex with a PEFT directory (adapter_model.safetensors with
  base_model.model.layers.* keys, adapter_config.json lora_alpha) and with a ComfyUI single file
  (diffusion_model.* keys, lora_down / lora_up, per-tensor alpha scalars) generates what the
  oracle generates from the merged tensors, at the DiT bars (cosine >= 0.9999, max_rel <= 1e-2),
  and differs from the unmerged model;
- LyCORIS LoKr (adapter_merge_lokr): the Kronecker delta with factorised and monolithic second
  factors and the DoRA weight decomposition, bit for bit at kernel level (acb_lokr_delta_add) and
  at the DiT bars through acb_dit_load_ex with a lycoris_* file; a LoKr payload with no usable
  module is refused with ACB_ERR_FORMAT.
Safetensors files are written here by a small writer of the format (8-byte header length, JSON
header, data)."""
import ctypes as C
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


def test_lokr_without_usable_module_refused(dit_file, tmp_path):
    path, _ = dit_file
    f = str(tmp_path / "lokr.safetensors")
    # a LoKr marker but no lycoris_ module with w1, w2 and alpha: nothing merges
    write_safetensors(f, {"layers.0.self_attn.q_proj.lokr_w1": ("F32", np.ones((4, 4), np.float32))})
    with pytest.raises(acb.AcbError) as e:
        acb.DiT(path, adapter=f)
    assert e.value.status == 7


@pytest.mark.parametrize("qt,form,dora,user", [(acb.Q8_0, "factor", False, 0.8), (acb.Q8_0, "mono", True, 0.8),
                                               (acb.BF16, "factor", True, 1.0), (acb.BF16, "mono", False, 1.0)])
def test_lokr_kernels_bitexact(cuda, qt, form, dora, user):
    import torch
    rng = np.random.default_rng(40 + qt + (form == "mono") + 2 * dora)
    a, b, c, d, r = 4, 8, 96, 64, 8
    N, K = a * c, b * d
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    raw = O.quantize(w, qt) if qt != acb.BF16 else _bf16(w)
    entry = (qt, raw, K, (N, K))
    w1 = (rng.standard_normal((a, b)) * 0.1).astype(np.float32)
    if form == "factor":
        w1s, W2 = O.lokr_factors(w1, 16.0, r, w2a=(rng.standard_normal((c, r)) * 0.1).astype(np.float32),
                                 w2b=(rng.standard_normal((r, d)) * 0.1).astype(np.float32))
    else:
        w1s, W2 = O.lokr_factors(w1, 16.0, r, w2=(rng.standard_normal((c, d)) * 0.05).astype(np.float32))
    ds = (1.0 + 0.1 * rng.standard_normal(N)).astype(np.float32) * np.float32(0.1) if dora else None
    _, ref_raw, _ = O.lokr_merge(entry, w1s, W2, user, ds)
    d_raw = torch.from_numpy(np.ascontiguousarray(raw).view(np.uint8).copy()).cuda()
    ids = torch.arange(N, dtype=torch.int32, device="cuda")
    tmp = torch.empty((N, K), dtype=torch.float32, device="cuda")
    acb._check("acb_get_rows", acb.lib().acb_get_rows(d_raw.data_ptr(), qt, N, K, ids.data_ptr(), N, tmp.data_ptr(),
                                                      acb.F32, K, None, acb._stream(None)))
    d1, d2 = torch.from_numpy(w1s).cuda(), torch.from_numpy(W2).cuda()
    dds = torch.from_numpy(ds).cuda() if dora else None
    fn = acb.lib().acb_lokr_delta_add
    fn.restype = C.c_int
    fn.argtypes = [C.c_void_p, C.c_int64, C.c_int64, C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_int, C.c_int,
                   C.c_float, C.c_void_p, C.c_void_p]
    acb._check("acb_lokr_delta_add", fn(tmp.data_ptr(), N, K, d1.data_ptr(), a, b, d2.data_ptr(), c, d, user,
                                        dds.data_ptr() if dora else None, acb._stream(None)))
    out = torch.empty_like(d_raw)
    acb._check("acb_requant", acb.lib().acb_requant(tmp.data_ptr(), N, K, qt, out.data_ptr(), acb._stream(None)))
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy().reshape(-1), np.ascontiguousarray(ref_raw).view(np.uint8).reshape(-1))


# (target, a, b, form): factorised modules of rank 4, monolithic ones of linear_dim 6
LOKR = [("layers.0.self_attn.q_proj", 4, 4, "factor"), ("layers.0.self_attn.v_proj", 2, 4, "mono"),
        ("layers.1.cross_attn.o_proj", 4, 8, "factor"), ("layers.1.mlp.down_proj", 2, 2, "mono")]


def test_dit_lokr_file(dit_file, tmp_path):
    path, keep = dit_file
    rng = np.random.default_rng(13)
    shapes = {t: (N, K) for t, N, K in TARGETS}
    tens, merged, user, lin_dim = {}, dict(keep), 0.9, 6
    for i, (t, a, b, form) in enumerate(LOKR):
        N, K = shapes[t]
        c, d = N // a, K // b
        key = "lycoris_" + t.replace(".", "_")
        w1 = (rng.standard_normal((a, b)) * 0.5).astype(np.float32)
        alpha = float(3 + i)
        tens[f"{key}.lokr_w1"] = ("F32", w1)
        tens[f"{key}.alpha"] = ("F32", np.array(alpha, dtype=np.float32).reshape(()))
        if form == "factor":
            w2a = (rng.standard_normal((c, 4)) * 0.3).astype(np.float32)
            w2b = (rng.standard_normal((4, d)) * 0.3).astype(np.float32)
            tens[f"{key}.lokr_w2_a"] = ("F32", w2a)
            tens[f"{key}.lokr_w2_b"] = ("BF16", _bf16(w2b))  # read as f32 without a second rounding
            w1s, W2 = O.lokr_factors(w1, alpha, 4, w2a=w2a, w2b=O.round_bf16(w2b))
        else:
            w2 = (rng.standard_normal((c, d)) * 0.1).astype(np.float32)
            tens[f"{key}.lokr_w2"] = ("F32", w2)
            w1s, W2 = O.lokr_factors(w1, alpha, lin_dim, w2=w2)
        ds = None
        if i == 2:  # one module with a DoRA magnitude vector
            ds = (np.abs(rng.standard_normal(N)) + 0.5).astype(np.float32)
            tens[f"{key}.dora_scale"] = ("F32", ds.reshape(N, 1))
        name = f"decoder.{t}.weight"
        qt, raw, K_, shape = keep[name]
        _, mraw, _ = O.lokr_merge((qt, raw, K_, shape), w1s, W2, user, ds)
        merged[name] = (qt, np.ascontiguousarray(mraw).reshape(raw.shape), K_, shape)
    f = str(tmp_path / "lokr.safetensors")
    write_safetensors(f, tens, {"lokr_config": json.dumps({"linear_dim": lin_dim, "factor": -1})})
    _check_generate(path, f, user, merged, keep)
