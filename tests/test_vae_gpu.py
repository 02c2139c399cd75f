"""GPU: the AutoencoderOobleck decoder (src/vae.h) through the C ABI against the oracle's
restatement, at the floating-point bar (cosine >= 0.9999, max_rel <= 1e-2 per channel).

The device convolutions are tcgen05 GEMMs with f32 accumulation over f16 operands (the
reference's operand types); the oracle sums the same f16 products in float64, so the two agree
to accumulation-order rounding, not bit for bit.
- tiny decoder (VAE_TINY): 1, 6 and 7 latent frames; tiled decoding with small windows; the
  device-buffer entry equals the host entry bit for bit; a cancel callback stops tiling;
- the shipped shape (ACESTEP_VAE: 2048 -> 1024 -> 512 -> 256 -> 128 -> 128, 1920x) on 3 frames;
- a channel count off the GEMM's 64-multiple is refused at load with ACB_ERR_UNSUPPORTED."""
import numpy as np
import pytest

import acb
import oracle as O
from helpers import cos_sim, max_rel

pytestmark = pytest.mark.gpu


def _close(got, ref, what=""):
    assert got.shape == ref.shape, (what, got.shape, ref.shape)
    for ch in range(2):
        c, e = cos_sim(got[ch], ref[ch]), max_rel(got[ch], ref[ch])
        assert c >= 0.9999 and e <= 1e-2, (what, ch, c, e)


@pytest.fixture(scope="module")
def tiny(tmp_path_factory, cuda):
    import synthetic
    path = str(tmp_path_factory.mktemp("vae") / "vae_tiny.gguf")
    keep = {}
    synthetic.write_vae_gguf(path, synthetic.VAE_TINY, seed=3, keep=keep)
    vae = acb.VAE(path)
    yield vae, O.OracleVAE(keep)
    vae.close()


@pytest.mark.parametrize("T", [1, 6, 7])
def test_vae_decode_tiny(tiny, T):
    vae, ov = tiny
    assert vae.up == ov.up == 1920
    lat = np.random.default_rng(10 + T).standard_normal((T, 64)).astype(np.float32)
    _close(vae.decode(lat), ov.decode(lat), f"T={T}")


def test_vae_decode_tiled_tiny(tiny):
    vae, ov = tiny
    lat = np.random.default_rng(21).standard_normal((13, 64)).astype(np.float32)
    got = vae.decode_tiled(lat, chunk_size=8, overlap=2)
    ref = ov.decode_tiled(lat, chunk_size=8, overlap=2)
    _close(got, ref, "tiled")
    # overlap larger than half the chunk is halved until a core remains (vae.h:477-479)
    _close(vae.decode_tiled(lat, chunk_size=6, overlap=4), ov.decode_tiled(lat, chunk_size=6, overlap=4), "halved")


def test_vae_decode_device_matches_host(tiny):
    import torch
    vae, _ = tiny
    lat = np.random.default_rng(22).standard_normal((5, 64)).astype(np.float32)
    host = vae.decode(lat)
    d_lat = torch.from_numpy(lat).cuda()
    d_out = torch.empty((2, 5 * vae.up), dtype=torch.float32, device="cuda")
    vae.decode_device(d_lat, d_out)
    torch.cuda.synchronize()
    assert np.array_equal(d_out.cpu().numpy(), host)


def test_vae_tiled_cancel(tiny):
    vae, _ = tiny
    lat = np.random.default_rng(23).standard_normal((13, 64)).astype(np.float32)
    calls = []

    def cancel():
        calls.append(1)
        return len(calls) >= 2  # stop before the second tile

    with pytest.raises(acb.AcbError) as e:
        vae.decode_tiled(lat, chunk_size=8, overlap=2, cancel=cancel)
    assert e.value.status == 9 and len(calls) == 2


def test_vae_decode_shipped_shape(tmp_path, cuda):
    import synthetic
    path = str(tmp_path / "vae.gguf")
    keep = {}
    synthetic.write_vae_gguf(path, synthetic.ACESTEP_VAE, seed=4, keep=keep)
    vae = acb.VAE(path)
    ov = O.OracleVAE(keep)
    lat = np.random.default_rng(24).standard_normal((3, 64)).astype(np.float32)
    _close(vae.decode(lat), ov.decode(lat), "shipped")
    vae.close()


def test_vae_channels_not_multiple_of_64_refused(tmp_path, cuda):
    import synthetic
    cfg = dict(synthetic.VAE_TINY)
    cfg["out_ch"] = list(cfg["out_ch"][:-1]) + [72]
    path = str(tmp_path / "vae72.gguf")
    synthetic.write_vae_gguf(path, cfg, seed=5)
    with pytest.raises(acb.AcbError) as e:
        acb.VAE(path)
    assert e.value.status == 2


@pytest.mark.parametrize("T,C,N,kernel,dil,res", [(300, 128, 192, 7, 3, True), (5, 64, 256, 7, 9, False),
                                                  (1000, 256, 128, 7, 1, True), (129, 64, 64, 3, 1, False)])
def test_conv1d_tc_implicit_gemm(cuda, T, C, N, kernel, dil, res):
    """acb_conv1d_tc against float64 sums of the same f16 products (f32 accumulation on the device:
    max_rel <= 1e-5); taps reaching outside [0, T) read zeros."""
    import torch
    rng = np.random.default_rng(T + C)
    x = rng.standard_normal((T, C)).astype(np.float16)
    w = (rng.standard_normal((N, kernel, C)) * 0.1).astype(np.float16)  # [N][k*C + c]
    bias = rng.standard_normal(N).astype(np.float32)
    r = rng.standard_normal((T, N)).astype(np.float32)
    pad = (kernel // 2) * dil
    xp = np.zeros((T + 2 * pad, C))
    xp[pad:pad + T] = x.astype(np.float64)
    ref = np.zeros((T, N))
    for k in range(kernel):
        ref += xp[k * dil:k * dil + T] @ w[:, k, :].astype(np.float64).T
    ref = ref.astype(np.float32) + bias
    if res:
        ref = r + ref
    dx, dw = torch.from_numpy(x).cuda(), torch.from_numpy(w.reshape(N, -1)).cuda()
    db, dr = torch.from_numpy(bias).cuda(), torch.from_numpy(r).cuda()
    y = torch.empty((T, N), dtype=torch.float32, device="cuda")
    wsb = acb.lib().acb_gemm_workspace_bytes(T, N, kernel * C)
    ws = torch.zeros(max(wsb, 256) // 4, dtype=torch.float32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    acb._check("acb_conv1d_tc", acb.lib().acb_conv1d_tc(
        dx.data_ptr(), C, T, C, dw.data_ptr(), N, kernel, dil, pad, y.data_ptr(), acb.F32, N, db.data_ptr(),
        dr.data_ptr() if res else None, N, 2, ws.data_ptr(), ws.numel() * 4, err.data_ptr(), acb._stream(None)))
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert max_rel(y.cpu().numpy(), ref) <= 1e-5
