"""GPU: the library's own multi-GPU path (acb_comm + acb_dit_generate_sharded), the C++ entry a
host such as ace-synth calls to shard one DiT job over the GPUs of a node (one process per GPU).

- A communicator whose peer never joins: the bounded, non-blocking NCCL init gives up after the
  timeout with ACB_ERR_TIMEOUT (host-side wait, nothing runs on the GPU; one GPU is enough).
- Two GPUs (skipped with fewer): two spawned ranks share a tiny DiT job, once as whole track pairs
  (no exchange during the steps) and once as one CFG half per rank (the velocity crosses NVLink
  every step); every rank gets every track's x0, which must match the oracle's generate at the
  DiT bars (cosine >= 0.9999, max_rel <= 1e-2 per track).
NCCL's NVLink multicast (NVLS) is switched off in these tests.
"""
import os
import time

import numpy as np
import pytest

import acb
import oracle as O
from helpers import cos_sim, max_rel

pytestmark = pytest.mark.gpu

DIT_TINY = dict(n_layers=2, hidden_size=256, intermediate_size=512, n_heads=4, n_kv_heads=2, head_dim=128,
                in_channels=64, out_channels=32, patch_size=2, sliding_window=16, rope_theta=1000000.0,
                rms_norm_eps=1e-6, enc_hidden_size=256)


def test_comm_init_times_out_without_peer(cuda):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    uid = acb.Comm.unique_id()
    t0 = time.time()
    with pytest.raises(acb.AcbError) as e:
        acb.Comm(uid, world=2, rank=0, device=0, timeout_ms=3000)  # rank 1 never comes
    assert e.value.status == 10, e.value
    assert time.time() - t0 < 60
    assert b"timeout" in acb.lib().acb_last_error()


def _rank(rank, world, uid, path, inputs, q):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import torch
    torch.cuda.set_device(rank)
    comm = acb.Comm(uid, world=world, rank=rank, device=rank, timeout_ms=60000)
    dit = acb.DiT(path, device=rank)
    out = {}
    for name, (noise, ctx, enc, kw) in inputs.items():
        x0, ms = acb.dit_generate_sharded(dit, comm, noise, ctx, enc, acb.turbo_schedule(4), guidance_scale=3.0, **kw)
        out[name] = x0
    dit.close()
    comm.close()
    q.put((rank, out))


@pytest.mark.skipif("not __import__('torch').cuda.is_available() or __import__('torch').cuda.device_count() < 2")
def test_dit_generate_sharded_two_gpus(cuda, tmp_path):
    import torch.multiprocessing as mp

    import synthetic
    cfg = DIT_TINY
    keep = {}
    path = os.path.join(str(tmp_path), "dit.gguf")
    synthetic.write_dit_gguf(path, cfg, synthetic.Q8_0, seed=31, device="cuda", keep=keep)
    od = O.dit_from_gguf_tensors(cfg, keep)
    null = keep["null_condition_emb"][1].astype(np.float32)
    rng = np.random.default_rng(32)
    T, enc_S, Oc = 80, 24, cfg["out_channels"]

    def job(N):
        return (rng.standard_normal((N, T, Oc)).astype(np.float32),
                rng.standard_normal((N, T, cfg["in_channels"] - Oc)).astype(np.float32),
                rng.standard_normal((N, enc_S, cfg["enc_hidden_size"])).astype(np.float32))

    inputs = {"pairs": job(2) + (dict(real_S=[40, 27], real_enc_S=[24, 11]),),  # one track pair per rank
              "halves": job(1) + (dict(),)}  # one CFG half per rank, exchange every step
    uid = acb.Comm.unique_id()
    ctx_mp = mp.get_context("spawn")
    q = ctx_mp.Queue()
    procs = [ctx_mp.Process(target=_rank, args=(r, 2, uid, path, inputs, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for name, (noise, ctx, enc, kw) in inputs.items():
        ref = O.dit_generate(od, noise, ctx, enc, null, acb.turbo_schedule(4), 3.0, **kw)
        for r in range(2):
            x0 = got[r][name]
            for b in range(ref.shape[0]):
                c, e = cos_sim(x0[b], ref[b]), max_rel(x0[b], ref[b])
                assert c >= 0.9999 and e <= 1e-2, (name, r, b, c, e)
        assert np.array_equal(got[0][name], got[1][name])  # every rank holds the same gathered result
