"""CPU: the host logic of the sharded jobs with two gloo ranks (world_size 2, 127.0.0.1).

bench.py runs config 4's DiT sharded over the ranks (each evaluates a block of the 2N CFG slots
and every rank then holds all velocities in slot order) and config 5's LM one sequence per rank
(token streams gathered at the end); both report the slowest rank's time. These are the same
helpers (multi.py), exercised here with gloo on the CPU: which slots a rank owns, the gather
order that the APG pairing (conditional slots 0..N-1, unconditional N..2N-1) relies on, and the
max-over-ranks time. The product's own sharding plan (acb_dit_shard_plan, the C++ host logic
behind acb_dit_generate_sharded and the acb_dit_job_* API) is checked the same way: every rank
asks the library for its share, the ranks gather the shares, and together they must cover every
(track, CFG half) exactly once, with split pairs on partner ranks."""
import os
import socket

import pytest

import multi


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        n_tracks, T, C = 4, 3, 2
        slots = multi.dit_slots(2 * n_tracks, world, rank)
        assert slots == list(range(rank * 4, rank * 4 + 4))
        tracks, uncond = multi.slot_tracks(slots, n_tracks)
        # each slot's "velocity" encodes (slot, track, cond) so the gathered order can be checked
        vel = torch.stack([torch.full((T, C), 100.0 * j + 10.0 * tr + (1.0 if u else 0.0))
                           for j, tr, u in zip(slots, tracks, uncond)])
        allv = multi.gather_rows(vel, world)
        assert allv.shape == (2 * n_tracks, T, C)
        for j in range(2 * n_tracks):
            tr, u = j % n_tracks, j >= n_tracks
            assert float(allv[j, 0, 0]) == 100.0 * j + 10.0 * tr + (1.0 if u else 0.0)
        # APG pairs conditional track i (slot i) with its unconditional twin (slot N + i)
        cond, unc = allv[:n_tracks], allv[n_tracks:]
        assert torch.all((unc - cond)[:, 0, 0] == 100.0 * n_tracks + 1.0)
        # the sharded LM: one token stream per rank, gathered in rank order
        toks = torch.arange(5, dtype=torch.int64)[None] + 1000 * rank
        got = multi.gather_rows(toks, world)
        assert got.shape == (world, 5) and got[1, 0].item() == 1000 and got[0, 4].item() == 4
        # the job's time is the slowest rank's, on every rank
        assert multi.max_over_ranks(1.5 + rank, world) == 1.5 + (world - 1)
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_dit_slots_and_errors():
    assert multi.dit_slots(8, 1, 0) == list(range(8))
    assert multi.dit_slots(8, 8, 5) == [5]
    assert multi.slot_tracks([2, 5], 4) == ([2, 1], [False, True])
    with pytest.raises(ValueError):
        multi.dit_slots(8, 3, 0)


def test_two_gloo_ranks():
    import torch.multiprocessing as mp
    mp.spawn(_rank_main, args=(2, _free_port()), nprocs=2, join=True)


def _plan_rank(rank, world, port, n_tracks, cfg, q):
    import torch
    import torch.distributed as dist
    import acb
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        t0, nl, half, peer = acb.dit_shard_plan(n_tracks, cfg, world, rank)
        mine = torch.tensor([t0, nl, half, peer], dtype=torch.int64)
        parts = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(parts, mine)
        if rank == 0:
            q.put([p.tolist() for p in parts])
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("n_tracks,cfg,world", [(4, 1, 2), (1, 1, 2), (8, 1, 2), (2, 0, 2)])
def test_product_shard_plan_over_gloo_ranks(n_tracks, cfg, world):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    mp.spawn(_plan_rank, args=(world, _free_port(), n_tracks, cfg, q), nprocs=world, join=True)
    plans = q.get()
    seen = {}
    for r, (t0, nl, half, peer) in enumerate(plans):
        for t in range(t0, t0 + nl):
            for h in ((0, 1) if (half < 0 and cfg) else ((0,) if half < 0 else (half,))):
                assert (t, h) not in seen, (t, h, plans)
                seen[(t, h)] = r
        if half >= 0:  # a split pair: the partner holds the other half of the same track
            assert plans[peer][0] == t0 and plans[peer][2] == 1 - half and plans[peer][3] == r
    halves = (0, 1) if cfg else (0,)
    assert set(seen) == {(t, h) for t in range(n_tracks) for h in halves}


def test_product_shard_plan_rejects_uneven_jobs():
    import acb
    with pytest.raises(acb.AcbError) as e:
        acb.dit_shard_plan(3, 1, 2, 0)  # 3 tracks over 2 ranks: neither whole pairs nor halves
    assert e.value.status == 2
    assert acb.dit_shard_plan(4, 1, 8, 7) == (3, 1, 1, 6)
    assert acb.dit_shard_plan(4, 1, 4, 1) == (1, 1, -1, -1)
