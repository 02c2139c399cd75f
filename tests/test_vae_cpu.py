"""CPU: the oracle's VAE decoder restatement (src/vae.h:64-369) pinned against PyTorch's own
definition of the AutoencoderOobleck decoder: torch.nn.functional conv1d / conv_transpose1d and
the weight_norm formula g * v / |v| in float64, with the reference's operand precision applied
(f16 weights, f16-cast conv inputs). This checks the oracle's padding, dilation, stride, crop,
layout and weight-norm axis (dim 0 of [OC, IC, K] for convs, of [IC, OC, K] for the transposed
convs) independently of the restatement. Tolerance: cosine >= 0.9999, max_rel <= 1e-2 (the
floating-point bar of the decoder's output)."""
import numpy as np
import pytest

import oracle as O
from helpers import cos_sim, max_rel

torch = pytest.importorskip("torch")
F = torch.nn.functional


@pytest.fixture(scope="module")
def tiny(tmp_path_factory):
    import synthetic
    keep = {}
    synthetic.write_vae_gguf(str(tmp_path_factory.mktemp("vae") / "vae.gguf"), synthetic.VAE_TINY, seed=3, keep=keep)
    return keep


def _torch_decoder(keep, latent):
    f = lambda n: torch.from_numpy(O.bf16_bits_to_f32(keep[n]).reshape(keep[n].shape)).double()
    h16 = lambda t: t.half().double()

    def wn(p):
        g, v = f(p + ".weight_g"), f(p + ".weight_v")
        return h16(v * g / v.pow(2).sum(dim=(1, 2), keepdim=True).sqrt())

    def snake(x, p):
        return x + torch.sin(x * f(p + ".alpha").exp()).pow(2) / f(p + ".beta").exp()

    x = torch.from_numpy(latent).double().T[None]
    x = F.conv1d(h16(x), wn("decoder.conv1"), f("decoder.conv1.bias"), padding=3)
    i = 0
    while f"decoder.block.{i}.conv_t1.weight_v" in keep:
        p = f"decoder.block.{i}"
        x = snake(x, p + ".snake1")
        w = wn(p + ".conv_t1")
        s = w.shape[2] // 2
        x = F.conv_transpose1d(h16(x), w, f(p + ".conv_t1.bias"), stride=s, padding=(w.shape[2] - s) // 2)
        for r, d in zip(range(1, 4), (1, 3, 9)):
            q = f"{p}.res_unit{r}"
            h = F.conv1d(h16(snake(x, q + ".snake1")), wn(q + ".conv1"), f(q + ".conv1.bias"), padding=3 * d,
                         dilation=d)
            x = x + F.conv1d(h16(snake(h, q + ".snake2")), wn(q + ".conv2"), f(q + ".conv2.bias"))
        i += 1
    x = snake(x, "decoder.snake1")
    return F.conv1d(h16(x), wn("decoder.conv2"), None, padding=3)[0].numpy()


def test_oracle_vae_matches_torch_definition(tiny):
    lat = np.random.default_rng(1).standard_normal((6, 64)).astype(np.float32)
    ov = O.OracleVAE(tiny)
    got = ov.decode(lat)
    ref = _torch_decoder(tiny, lat)
    assert got.shape == ref.shape == (2, 6 * ov.up)
    c, e = cos_sim(got, ref), max_rel(got, ref)
    assert c >= 0.9999 and e <= 1e-2, (c, e)


def test_oracle_weight_norm_axis_and_sum(tiny):
    """The fused weight is g * v / (|v| + 1e-12) per dim-0 slice, the norm from a sequential f32 sum."""
    v = O.bf16_bits_to_f32(tiny["decoder.block.0.conv_t1.weight_v"]).reshape(tiny["decoder.block.0.conv_t1.weight_v"].shape)
    g = O.bf16_bits_to_f32(tiny["decoder.block.0.conv_t1.weight_g"]).reshape(-1)
    w = O.OracleVAE._wn(g, v)
    ref = v.astype(np.float64) * (g[:, None, None] / np.sqrt((v.astype(np.float64) ** 2).sum(axis=(1, 2)))[:, None, None])
    assert max_rel(w, ref) <= 1e-5
    nsq = np.float32(0)
    row = v[0].ravel()
    for t in row:  # the reference's loop, term by term
        nsq = np.float32(nsq + np.float32(t * t))
    s = np.float32(g[0] / np.float32(np.sqrt(nsq) + np.float32(1e-12)))
    assert np.array_equal(w[0].ravel(), (row * s).astype(np.float32))


def test_oracle_tiled_short_input_is_plain_decode(tiny):
    lat = np.random.default_rng(2).standard_normal((5, 64)).astype(np.float32)
    ov = O.OracleVAE(tiny)
    assert np.array_equal(ov.decode_tiled(lat, chunk_size=8, overlap=2), ov.decode(lat))


def test_oracle_tiled_length_and_core_trims(tiny):
    """Cores of chunk - 2*overlap latent frames, each up-sampled: the output covers every frame once."""
    lat = np.random.default_rng(3).standard_normal((13, 64)).astype(np.float32)
    ov = O.OracleVAE(tiny)
    out = ov.decode_tiled(lat, chunk_size=8, overlap=2)
    assert out.shape == (2, 13 * ov.up)
    # the first core (frames 0-3) sees frames 0-5: same as decoding those 6 frames, trimmed
    first = ov.decode(lat[:6])[:, :4 * ov.up]
    assert np.array_equal(out[:, :4 * ov.up], first)
