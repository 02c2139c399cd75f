#!/usr/bin/env python3
"""Benchmark of the B200 op-chain (one JSON line on rank 0).

Headline (workload `dit`, every N): BASELINE config 4, the DiT denoiser -- 24 layers, hidden
2048, Q8_0 weights, 4 tracks x CFG 2 = 8 sequences of 750 tokens (1500 latent frames, patch 2),
512 condition rows, the turbo schedule with Euler steps and APG guidance. A step is one denoise
step of the whole 8-sequence job; the sequences are sharded over the GPUs (strong scaling) and
each step all-gathers the velocities (NCCL) before APG. The metric is denoise steps/s, in the
exact arithmetic mode (products of the reference's dequantised operands from hi/lo f16 splits);
the fast mode (single f16 operands) is reported beside it.

Sub-results at N=1: config 1 (text encoder forwards/s), config 3 (LM decode tok/s) and config 2:
the isolated fused-op microbench at DiT/LM row shapes, in both f32 and bf16 I/O. One step runs,
per I/O type:
  (a) RMSNorm over 8192 rows of 2048
  (b) per-head q/k RMSNorm + NeoX RoPE on [B=4, T=1024, H=16, D=128], positions 0..T-1, theta 1e6
  (c) SwiGLU on gate/up [8192, 6144] (fused [8192, 12288] rows)
  (d) adaLN modulate x*(1+scale)+shift, then the gated residual, x [8, 750, 2048], per-sample
      shift/scale/gate [8, 2048]
  (e) get_rows of 8192 random ids from a [217472 x 2048] Q8_0 table
The metric is HBM GB/s over algorithmic bytes (every input read once, every output written
once). Inputs are N(0,1) from a fixed seed, resident in HBM; the per-step working set (1.7 GB)
is far above the 126 MB L2 and every buffer is touched once per step, so nothing is served from
L2 across iterations.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Multi-GPU: launched under torch.distributed.run, one process per GPU; timing is the max over ranks
of the CUDA-event time.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "hbd-acestep.cpp_b200"))

HBM_FALLBACK_GBS = 6650.0


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return {"hbm_gbs": HBM_FALLBACK_GBS, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


# ---- workload: BASELINE config 2 --------------------------------------------------------------

RMS_ROWS, RMS_COLS = 8192, 2048
QK_B, QK_T, QK_H, QK_D = 4, 1024, 16, 128
SW_ROWS, SW_F = 8192, 6144
AD_S, AD_T, AD_H = 8, 750, 2048
GR_V, GR_H, GR_N = 217472, 2048, 8192
EPS, THETA = 1e-6, 1e6


def op_bytes(io: str) -> dict:
    """Algorithmic bytes per launch (inputs read once + outputs written once)."""
    s = 4 if io == "f32" else 2
    return {
        "rms_norm": RMS_ROWS * RMS_COLS * s * 2 + RMS_COLS * 4,
        "qk_norm_rope": QK_B * QK_T * QK_H * QK_D * s * 2 + QK_D * 4 + QK_B * QK_T * 4 + QK_T * QK_D * 4,
        "swiglu": SW_ROWS * SW_F * s * 3,
        "adaln_modulate": AD_S * AD_T * AD_H * s * 2 + 2 * AD_S * AD_H * 4,
        "gated_residual": AD_S * AD_T * AD_H * s * 3 + AD_S * AD_H * 4,
        "get_rows": GR_N * (GR_H // 32 * 34) + GR_N * 4 + GR_N * GR_H * s,
    }


class OpsWorkload:
    """Device buffers for one config-2 step in one I/O type, and the C-ABI calls over them."""

    def __init__(self, io: str, dev, table, seed: int):
        import torch
        import acb

        self.io = io
        self.acb = acb
        dt = torch.float32 if io == "f32" else torch.bfloat16
        g = torch.Generator(device=dev).manual_seed(seed)

        def rn(*shape, scale=1.0):
            return (torch.randn(*shape, generator=g, device=dev) * scale).to(dt)

        self.x_rms = rn(RMS_ROWS, RMS_COLS)
        self.w_rms = (1 + 0.01 * torch.randn(RMS_COLS, generator=g, device=dev)).float()
        self.y_rms = torch.empty_like(self.x_rms)
        self.x_qk = rn(QK_B * QK_T, QK_H * QK_D)
        self.w_qk = (1 + 0.01 * torch.randn(QK_D, generator=g, device=dev)).float()
        self.pos = torch.arange(QK_T, dtype=torch.int32, device=dev).repeat(QK_B)
        self.rope = acb.rope_table(QK_T, QK_D, THETA).to(dev)
        self.y_qk = torch.empty((QK_B * QK_T, QK_H, QK_D), dtype=dt, device=dev)
        self.gu = rn(SW_ROWS, 2 * SW_F)
        self.y_sw = torch.empty((SW_ROWS, SW_F), dtype=dt, device=dev)
        self.x_ad = rn(AD_S, AD_T, AD_H)
        self.scale = (0.1 * torch.randn(AD_S, AD_H, generator=g, device=dev)).float()
        self.shift = (0.1 * torch.randn(AD_S, AD_H, generator=g, device=dev)).float()
        self.gate = torch.randn(AD_S, AD_H, generator=g, device=dev).float()
        self.y_ad = torch.empty_like(self.x_ad)
        self.o_ad = rn(AD_S, AD_T, AD_H)
        self.out_gr = torch.empty_like(self.x_ad)
        self.table = table
        self.ids = torch.randint(0, GR_V, (GR_N,), dtype=torch.int32, device=dev, generator=g)
        self.y_rows = torch.empty((GR_N, GR_H), dtype=dt, device=dev)
        self.bytes = op_bytes(io)

    def ops(self):
        a = self.acb
        return [
            ("rms_norm", lambda: a.rms_norm(self.x_rms, self.w_rms, EPS, out=self.y_rms)),
            ("qk_norm_rope", lambda: a.qk_norm_rope(self.x_qk, QK_H, QK_D, self.w_qk, EPS, self.pos, self.rope,
                                                    out=self.y_qk, dst_tok_stride=QK_H * QK_D,
                                                    dst_head_stride=QK_D)),
            ("swiglu", lambda: a.swiglu(self.gu, SW_F, out=self.y_sw)),
            ("adaln_modulate", lambda: a.adaln_modulate(self.x_ad, None, EPS, self.scale, self.shift, out=self.y_ad)),
            ("gated_residual", lambda: a.gated_residual(self.x_ad, self.o_ad, self.gate, out=self.out_gr)),
            ("get_rows", lambda: a.get_rows(self.table, a.Q8_0, GR_V, GR_H, self.ids, out=self.y_rows)),
        ]

    # e2e: the same calls with host inputs/outputs copied in and out each step
    def host_mirror(self):
        import torch
        ins = [self.x_rms, self.x_qk, self.gu, self.x_ad, self.o_ad, self.ids]
        outs = [self.y_rms, self.y_qk, self.y_sw, self.y_ad, self.out_gr, self.y_rows]
        self.h_in = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True).copy_(t) for t in ins]
        self.h_out = [torch.empty(t.shape, dtype=t.dtype, pin_memory=True) for t in outs]
        self.d_in, self.d_out = ins, outs
        self.h2d = sum(t.numel() * t.element_size() for t in ins)
        self.d2h = sum(t.numel() * t.element_size() for t in outs)

    def e2e_step(self):
        for h, d in zip(self.h_in, self.d_in):
            d.copy_(h, non_blocking=True)
        for _, f in self.ops():
            f()
        for h, d in zip(self.h_out, self.d_out):
            h.copy_(d, non_blocking=True)


def make_q8_table(dev, seed):
    """[217472 x 2048] Q8_0 table, built on the device: random int8 quants, f16 scales of a
    N(0,1)/127-sized row."""
    import torch
    g = torch.Generator(device=dev).manual_seed(seed)
    raw = torch.randint(0, 256, (GR_V, GR_H // 32 * 34), dtype=torch.uint8, device=dev, generator=g)
    d = (torch.rand((GR_V, GR_H // 32), device=dev, generator=g) * 0.02 + 0.005).to(torch.float16)
    raw.view(GR_V, GR_H // 32, 34)[:, :, 0:2] = d.view(torch.uint8).view(GR_V, GR_H // 32, 2)
    return raw


# ---- clocks --------------------------------------------------------------------------------

class ClockSampler:
    """nvidia-smi samples (200 ms) of SM clock and throttle reasons during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except (OSError, FileNotFoundError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 8:
                continue
            try:
                sm.append(float(parts[0]))
                mx.append(float(parts[1]))
            except ValueError:
                continue
            for n, v in zip(names, parts[4:8]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---- CPU baseline (oracle) -----------------------------------------------------------------

def cpu_ops_sample(frac: int = 8, threads: int | None = None) -> tuple[float, dict]:
    """Time the oracle (the CPU restatement of the reference's ggml-CPU arithmetic) on 1/frac of
    the rows of every config-2 op, f32 I/O. Returns (GB/s over algorithmic bytes, info)."""
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    if threads:
        O.set_threads(threads)
    rng = np.random.default_rng(0)
    r = lambda *s: rng.standard_normal(s).astype(np.float32)
    x_rms, w_rms = r(RMS_ROWS // frac, RMS_COLS), np.ones(RMS_COLS, np.float32)
    x_qk = r(QK_B * QK_T // frac, QK_H, QK_D)
    rope = O.rope_cache(np.arange(QK_B * QK_T // frac, dtype=np.int32) % QK_T, QK_D, THETA)
    gu = r(SW_ROWS // frac, 2 * SW_F)
    g, u = np.ascontiguousarray(gu[:, :SW_F]), np.ascontiguousarray(gu[:, SW_F:])
    x_ad, o_ad = r(AD_S, AD_T // frac, AD_H), r(AD_S, AD_T // frac, AD_H)
    sc, sh, gt = r(AD_S, AD_H) * 0.1, r(AD_S, AD_H) * 0.1, r(AD_S, AD_H)
    n_tab = GR_V // frac
    table = O.quantize(r(n_tab, GR_H) * 0.02, O.Q8_0)
    ids = rng.integers(0, n_tab, GR_N // frac).astype(np.int32)
    t0 = time.perf_counter()
    O.rms_norm(x_rms, w_rms, EPS)
    O.qk_norm_rope(x_qk, np.ones(QK_D, np.float32), EPS, rope)
    O.swiglu(g, u)
    O.adaln(x_ad, None, EPS, sc, sh)
    O.gated_residual(x_ad, o_ad, gt)
    O.get_rows(O.Q8_0, table, GR_H, ids)
    dt = time.perf_counter() - t0
    nbytes = sum(op_bytes("f32").values()) / frac
    return nbytes / dt / 1e9, {"cores": O.get_threads(), "seconds": dt,
                               "sample": f"1/{frac} of the rows of every config-2 op, f32 I/O, one pass"}


# ---- main ----------------------------------------------------------------------------------

def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def cpu_dit_tensors(cfg, seed):
    """DiT weights made on the host for the reference arm, with the reference's tensor names and
    quantize-tool types (Q8_0 linears, F32 norms / biases / tables, BF16 conv projections), without
    any GPU or this repository's library: Q8_0 blocks are random int8 values in [-127, 127] with
    one f16 scale (3.3e-4, the scale of N(0, 0.02) rows); vectors N(base, std). The CPU arm's
    timing does not depend on the values."""
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    rng = np.random.default_rng(seed)
    H, F, L = cfg["hidden_size"], cfg["intermediate_size"], cfg["n_layers"]
    Nh, Nkv, D = cfg["n_heads"], cfg["n_kv_heads"], cfg["head_dim"]
    in_ch, oc, P, He = cfg["in_channels"], cfg["out_channels"], cfg["patch_size"], cfg["enc_hidden_size"]
    out = {}
    d16 = np.frombuffer(np.float16(3.3e-4).tobytes(), np.uint8)

    def mat(name, N, K):
        raw = np.empty((N, K // 32, 34), np.uint8)
        raw[:, :, 0:2] = d16
        raw[:, :, 2:] = rng.integers(-127, 128, size=(N, K // 32, 32), dtype=np.int8).view(np.uint8)
        out[name] = (O.Q8_0, raw.reshape(N, K // 32 * 34), K, (N, K))

    def vec(name, shape, base=0.0, std=0.02):
        out[name] = (O.F32, (base + std * rng.standard_normal(shape, dtype=np.float32)).astype(np.float32),
                     shape[-1], shape)

    def conv_bf16(name, shape):
        out[name] = (O.BF16, O.f32_to_bf16_bits(0.02 * rng.standard_normal(shape, dtype=np.float32)), shape[-1], shape)

    for te in ("decoder.time_embed", "decoder.time_embed_r"):
        mat(f"{te}.linear_1.weight", H, 256)
        vec(f"{te}.linear_1.bias", (H,))
        mat(f"{te}.linear_2.weight", H, H)
        vec(f"{te}.linear_2.bias", (H,))
        mat(f"{te}.time_proj.weight", 6 * H, H)
        vec(f"{te}.time_proj.bias", (6 * H,))
    conv_bf16("decoder.proj_in.1.weight", (H, in_ch, P))
    vec("decoder.proj_in.1.bias", (H,))
    mat("decoder.condition_embedder.weight", H, He)
    vec("decoder.condition_embedder.bias", (H,))
    for i in range(L):
        p = f"decoder.layers.{i}"
        for a in ("self_attn", "cross_attn"):
            mat(f"{p}.{a}.q_proj.weight", Nh * D, H)
            mat(f"{p}.{a}.k_proj.weight", Nkv * D, H)
            mat(f"{p}.{a}.v_proj.weight", Nkv * D, H)
            mat(f"{p}.{a}.o_proj.weight", H, Nh * D)
            vec(f"{p}.{a}.q_norm.weight", (D,), 1.0, 0.01)
            vec(f"{p}.{a}.k_norm.weight", (D,), 1.0, 0.01)
        vec(f"{p}.self_attn_norm.weight", (H,), 1.0, 0.01)
        vec(f"{p}.cross_attn_norm.weight", (H,), 1.0, 0.01)
        vec(f"{p}.mlp_norm.weight", (H,), 1.0, 0.01)
        mat(f"{p}.mlp.gate_proj.weight", F, H)
        mat(f"{p}.mlp.up_proj.weight", F, H)
        mat(f"{p}.mlp.down_proj.weight", H, F)
        vec(f"{p}.scale_shift_table", (1, 6, H), 0.0, 0.05)
    vec("decoder.norm_out.weight", (H,), 1.0, 0.01)
    vec("decoder.scale_shift_table", (1, 2, H), 0.0, 0.05)
    conv_bf16("decoder.proj_out.1.weight", (H, oc, P))
    vec("decoder.proj_out.1.bias", (oc,))
    vec("null_condition_emb", (He,), 0.0, 1.0)
    return out


DIT_2B = dict(n_layers=24, hidden_size=2048, intermediate_size=6144, n_heads=16, n_kv_heads=8, head_dim=128,
              in_channels=192, out_channels=64, patch_size=2, sliding_window=128, rope_theta=1000000.0,
              rms_norm_eps=1e-6, enc_hidden_size=2048)


def run_reference(args):
    """Reference arm on the headline's metric and config (config 4 DiT denoise steps/s). The
    reference's ggml-CPU build cannot be compiled here (its ggml submodule is empty), so the CPU
    oracle -- the port of its DiT arithmetic: Q8_0 x Q8_0-quantised integer block dots, f32
    attention, rounding per graph node -- runs on all host threads. No GPU and none of this
    repository's CUDA library is touched: the weights are made on the host (cpu_dit_tensors).

    Work: full-depth evaluations of one CFG pair (2 of the step's 8 sequences of 750 tokens, 512
    condition rows), run a slice of consecutive layers per timed step so that the run ends in a few
    minutes; the hidden state carries from slice to slice, and after layer 23 the output
    projection closes the evaluation and the next begins. Each step's unit is the fraction of a
    denoise step it did (layers / 24 x 2 / 8 sequences); value = the fractions summed over the K
    timed steps / their total time. The layer count per slice comes from one warm-up layer
    (about 5 s per slice). Under torchrun only rank 0 runs."""
    ws, rank, _ = dist_env()
    if rank != 0:
        return
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    O.set_threads(len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1))
    cfg = dict(DIT_2B)
    L = cfg["n_layers"]
    t0 = time.perf_counter()
    keep = cpu_dit_tensors(cfg, seed=21)
    od = O.dit_from_gguf_tensors(cfg, keep)
    t_setup = time.perf_counter() - t0
    rng = np.random.default_rng(1)
    T, enc_S = DIT_T, DIT_ENC_S
    x = rng.standard_normal((2, T, cfg["in_channels"]), dtype=np.float32)
    e = rng.standard_normal((2, enc_S, cfg["enc_hidden_size"]), dtype=np.float32)
    frac_per_layer = (1.0 / L) * (2.0 / (2 * DIT_TRACKS))
    state = {"layer": 0, "open": False}

    def slice_(n):
        """Run the next n layers of the evaluation chain; returns the denoise-step fraction done."""
        if not state["open"]:
            od.begin(x, e, 0.75, 0.75)
            state["open"] = True
        l0 = state["layer"]
        l1 = min(L, l0 + n)
        od.run_layers(l0, l1)
        state["layer"] = l1
        if l1 == L:
            od.finish()
            state.update(layer=0, open=False)
        return (l1 - l0) * frac_per_layer

    # warm-up: one layer sets the slice length, then W-1 slices at that length
    t0 = time.perf_counter()
    slice_(1)
    t_layer = time.perf_counter() - t0
    n_l = int(max(1, min(L, round(5.0 / max(t_layer, 1e-3)))))
    for _ in range(max(0, args.warmup - 1)):
        slice_(n_l)
    fr, dts = [], []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        f = slice_(n_l)
        dts.append(time.perf_counter() - t0)
        fr.append(f)
    val = sum(fr) / sum(dts)
    ms_step = 1e3 * sum(dts) / len(dts)
    cores = O.get_threads()
    line = {"metric": "DiT denoise steps/s (config 4: 24 layers, hidden 2048, Q8_0, 4 tracks x CFG 2 = 8 "
                      "sequences of 750 tokens, 512 condition rows, turbo Euler + APG)",
            "value": round(val, 6), "unit": "step/s", "impl": "reference", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 1), "higher_is_better": True, "scaling": "strong",
            "dtype": "int8 dot products (Q8_0 x Q8_0-quantised activations), f32 elsewhere", "data": "synthetic",
            "config": {"workload": "config4_dit2b_q8_0_turbo_cfg", "tracks": DIT_TRACKS, "sequences": 2 * DIT_TRACKS,
                       "frames": T, "enc_rows": enc_S, "layers": L},
            "cpu_baseline": {"value": round(val, 6), "unit": "step/s", "cores": cores, "kind": "port",
                             "sample": f"each timed step: {n_l} consecutive layers of a full-depth 24-layer evaluation "
                                       f"of one CFG pair (2 of 8 sequences), hidden state carried between steps; "
                                       f"{args.steps} steps = {sum(fr):.4f} denoise steps of work in "
                                       f"{sum(dts):.1f} s (weights made on the host in {t_setup:.0f} s)"},
            "e2e": {"value": round(val, 6), "unit": "step/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "step_fraction": round(fr[0], 6),
            "note": "reference ggml-CPU build unavailable (ggml submodule absent); the oracle port of its "
                    "arithmetic is timed instead, on the host cores only"}
    print(json.dumps(line), flush=True)


def run_ours(args):
    import torch
    import acb

    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    acb.lib()
    stream = torch.cuda.current_stream()

    if args.workloads == "lm5":
        r = run_lm5(dev, rank, ws, gen_len=args.lm5_gen)
        if rank == 0:
            print(json.dumps(dict(r, data="synthetic", dtype="int8-dot/f32 (Q8_K-quantised activations)")),
                  flush=True)
        if ws > 1:
            torch.distributed.destroy_process_group()
        return
    if args.workloads == "gemv":
        print(json.dumps(run_gemv_shapes(dev)), flush=True)
        return
    if args.workloads == "dit1":
        # profiling target: the per-GPU evaluation of config 4 at 8 GPUs (one 750-token sequence)
        import tempfile

        import numpy as np

        import synthetic
        cfg = dict(synthetic.ACESTEP_DIT_2B)
        path = os.path.join(tempfile.gettempdir(), "acb_bench_dit1.gguf")
        synthetic.write_dit_gguf(path, cfg, synthetic.Q8_0, seed=21, device=str(dev))
        dit = acb.DiT(path, device=dev.index or 0)
        os.remove(path)
        rng = np.random.default_rng(3)
        n_seq = int(os.environ.get("ACB_DIT1_SEQ", "1"))
        x = torch.from_numpy(rng.standard_normal((n_seq, DIT_T, cfg["in_channels"])).astype(np.float32)).to(dev)
        e = torch.from_numpy(rng.standard_normal((n_seq, DIT_ENC_S, cfg["enc_hidden_size"])).astype(np.float32)).to(dev)
        out = torch.empty((n_seq, DIT_T, cfg["out_channels"]), device=dev)
        tt = torch.tensor([0.8, 0.8], device=dev)
        dit.set_condition(e, DIT_T)
        for _ in range(3):
            dit.eval(x, tt, out)
        torch.cuda.synchronize()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record()
        for _ in range(10):
            dit.eval(x, tt, out)
        ev1.record()
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
        dit.eval(x, tt, out)
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
        print(json.dumps({"workload": "dit1", "sequences": n_seq, "ms_per_eval": ev0.elapsed_time(ev1) / 10,
                          "kernels_per_eval": dit.eval_kernels()}), flush=True)
        dit.close()
        return
    if args.workloads == "gemm_exact":
        # profiling target: three launches of the DiT's dominant kernel (exact gate|up), nothing else
        import torch as _t
        A = _t.randn(6000, 6144, device=dev).to(_t.float16)
        B = (_t.randn(12288, 6144, device=dev) * 0.02).to(_t.float16)
        C = _t.empty(6000, 12288, device=dev, dtype=_t.float32)
        for _ in range(3):
            acb.gemm_bf16(A, B, out=C)
        _t.cuda.synchronize()
        print(json.dumps({"workload": "gemm_exact gate|up", "launches": 3}), flush=True)
        return
    if args.workloads.startswith("gemm"):
        which = args.workloads.split(":")[1].split("+") if ":" in args.workloads else None
        print(json.dumps(run_gemm_shapes(dev, which=which)), flush=True)
        return
    if args.workloads.startswith("attn"):
        which = args.workloads.split(":")[1].split("+") if ":" in args.workloads else None
        print(json.dumps(run_attn_shapes(dev, which=which)), flush=True)
        return
    if args.workloads == "ditmodes":
        r = run_dit(dev, rank, want_cpu=not args.no_cpu_baseline)
        if rank == 0:
            print(json.dumps(dict(r, n_gpus=ws, data="synthetic", dtype="f16 operands (Q8_0-quantised activations)")),
                  flush=True)
        return
    if args.workloads == "condlog":
        r = run_cond_logged(dev, rank)
        if rank == 0:
            print(json.dumps(dict(r, n_gpus=ws, data="synthetic", dtype="f16 hi/lo operands, fp32 accumulation")),
                  flush=True)
        return
    if args.workloads == "ditlog":
        r = run_dit_logged(dev, rank)
        if rank == 0:
            print(json.dumps(dict(r, n_gpus=ws, data="synthetic", dtype="f16 hi/lo operands, fp32 accumulation")),
                  flush=True)
        return
    if args.workloads == "vae":
        r = run_vae(dev, rank, want_cpu=not args.no_cpu_baseline)
        if rank == 0:
            print(json.dumps(dict(r, n_gpus=ws, data="synthetic", dtype="f16 operands, f32 accumulation")),
                  flush=True)
        return
    if args.workloads == "noise":
        r = run_noise(dev, rank, want_cpu=not args.no_cpu_baseline)
        if rank == 0:
            print(json.dumps(dict(r, n_gpus=ws, data="synthetic", dtype="u32 rounds, f32 Box-Muller")), flush=True)
        return
    if args.workloads == "enc":
        r = run_enc(dev, rank, want_cpu=not args.no_cpu_baseline)
        if rank == 0:
            print(json.dumps(dict(r, n_gpus=ws, data="synthetic", dtype="f16 operands (Q8_0-quantised activations)")),
                  flush=True)
        return
    if args.workloads.split(",") == ["lm"]:
        # LM-only run (profiling): one line with the decode result
        lm = run_lm(dev, rank, want_cpu=not args.no_cpu_baseline, prompt_len=args.lm_prompt, gen_len=args.lm_gen)
        if rank == 0:
            print(json.dumps(dict(lm, n_gpus=ws, data="synthetic", dtype="int8-dot/f32")), flush=True)
        return

    wl = args.workloads.split(",")
    if "dit" not in wl:
        # config-2 headline (legacy layout): ops line with the LM / encoder results attached
        line = run_ops_line(args, dev, rank, ws, local, stream)
        if "lm" in wl and ws == 1:
            line["lm_decode"] = run_lm(dev, rank, want_cpu=not args.no_cpu_baseline, prompt_len=args.lm_prompt,
                                       gen_len=args.lm_gen)
        if "enc" in wl and ws == 1:
            line["text_encoder"] = run_enc(dev, rank, want_cpu=not args.no_cpu_baseline)
    else:
        line = run_dit_job(args, dev, rank, ws, local, stream)
        if ws == 1:
            # the other configs on one GPU, as sub-results
            if "ops" in wl:
                import copy
                a2 = copy.copy(args)
                a2.steps, a2.warmup = 300, 20
                line["fused_ops"] = run_ops_line(a2, dev, rank, ws, local, stream)
            if "lm" in wl:
                torch.cuda.empty_cache()
                line["lm_decode"] = run_lm(dev, rank, want_cpu=not args.no_cpu_baseline, prompt_len=args.lm_prompt,
                                           gen_len=args.lm_gen)
            if "enc" in wl:
                torch.cuda.empty_cache()
                line["text_encoder"] = run_enc(dev, rank, want_cpu=not args.no_cpu_baseline)
            if "vae" in wl:
                torch.cuda.empty_cache()
                line["vae_decode"] = run_vae(dev, rank, want_cpu=not args.no_cpu_baseline)
            if "ditlog" in wl:
                torch.cuda.empty_cache()
                line["dit_logged_case"] = run_dit_logged(dev, rank)
            if "condlog" in wl:
                torch.cuda.empty_cache()
                line["cond_logged_case"] = run_cond_logged(dev, rank)
            if "noise" in wl:
                torch.cuda.empty_cache()
                line["philox_noise"] = run_noise(dev, rank, want_cpu=not args.no_cpu_baseline)
        if "lm5" in wl:
            # config 5's LM shards one sequence per GPU: run at every N (all ranks take part)
            torch.cuda.empty_cache()
            line["lm5_decode"] = run_lm5(dev, rank, ws)
        if "dit5" in wl:
            # config 5's DiT leg (16 sequences, track pairs per GPU): every N
            torch.cuda.empty_cache()
            line["dit5"] = run_dit5_job(args, dev, rank, ws, local, stream)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if ws > 1:
        torch.distributed.destroy_process_group()


def run_ops_line(args, dev, rank, ws, local, stream):
    """Config 2 (the fused-op microbench): one line dict (every rank runs a replica)."""
    import torch
    table = make_q8_table(dev, 1234 + rank)
    wls = [OpsWorkload("f32", dev, table, 100 + rank), OpsWorkload("bf16", dev, table, 200 + rank)]
    ops = [(w.io, name, f, w.bytes[name]) for w in wls for name, f in w.ops()]
    step_bytes = sum(b for *_, b in ops)

    def barrier():
        if ws > 1:
            torch.distributed.barrier()

    for _ in range(args.warmup):
        for *_, f, _b in ops:
            f()
    torch.cuda.synchronize()

    # timed region: K steps, events around every launch (on torch's current stream, which is
    # the stream the kernels are enqueued on)
    evs = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in ops]
           for _ in range(args.steps)]
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    clk = ClockSampler(local)
    barrier()
    torch.cuda.synchronize()
    clk.start()
    time.sleep(0.3)
    # a ~2 ms spin on the stream first, so that the host's launches (ctypes calls from Python,
    # slower than these 20-90 us kernels are short) queue up ahead of the GPU and the events
    # time the kernels back to back rather than the host's launch gaps
    torch.cuda._sleep(4_000_000)
    t_start.record(stream)
    for k in range(args.steps):
        for (ea, eb), (_io, _n, f, _b) in zip(evs[k], ops):
            ea.record(stream)
            f()
            eb.record(stream)
    t_end.record(stream)
    torch.cuda.synchronize()
    barrier()
    clocks = clk.stop()
    ms = t_start.elapsed_time(t_end)
    if ws > 1:
        t = torch.tensor([ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    per_op = {}
    for i, (io, name, _f, b) in enumerate(ops):
        d = [evs[k][i][0].elapsed_time(evs[k][i][1]) for k in range(args.steps)]
        per_op[f"{name}.{io}"] = {"ms": statistics.mean(d), "GB/s": b / (statistics.mean(d) * 1e-3) / 1e9,
                                  "bytes": b}
    value = ws * step_bytes * args.steps / (ms * 1e-3) / 1e9
    n_launch = len(ops) * args.steps

    # e2e through the C ABI with host buffers (pinned), copies inside the timed region
    for w in wls:
        w.host_mirror()
    h2d = sum(w.h2d for w in wls)
    d2h = sum(w.d2h for w in wls)
    e2e_steps = max(2, min(args.steps // 100, 10))
    for w in wls:
        w.e2e_step()
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        for w in wls:
            w.e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    e_ms = e0.elapsed_time(e1)
    if ws > 1:
        t = torch.tensor([e_ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        e_ms = float(t.item())
    e2e_val = ws * step_bytes * e2e_steps / (e_ms * 1e-3) / 1e9

    peaks, peak_kind = measured_peaks()
    dom = max(per_op.items(), key=lambda kv: kv[1]["ms"])
    roof = {"kernel": dom[0], "bound": "hbm", "achieved": round(dom[1]["GB/s"], 1),
            "peak": peaks["hbm_gbs"], "peak_kind": peak_kind, "unit": "GB/s",
            "frac": round(dom[1]["GB/s"] / peaks["hbm_gbs"], 4),
            "frac_of_8TBs": round(dom[1]["GB/s"] / 8000.0, 4), "traffic": TRAFFIC.get(dom[0])}

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline:
        v, info = cpu_ops_sample(8)
        cpu = {"value": round(v, 3), "unit": "GB/s", "cores": info["cores"], "kind": "port",
               "sample": info["sample"]}

    line = {"metric": "fused-op HBM GB/s (config 2 op-chain, algorithmic bytes)", "value": round(value, 2),
            "unit": "GB/s", "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 5), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "config2_fused_ops", "io": ["f32", "bf16"],
                       "ops": ["rms_norm 8192x2048", "qk_norm_rope 4x1024x16x128", "swiglu 8192x6144",
                               "adaln_modulate 8x750x2048", "gated_residual 8x750x2048",
                               "get_rows 8192 of 217472x2048 q8_0"],
                       "bytes_per_step": step_bytes,
                       "l2": "working set 1.7 GB per step > 126 MB L2, each buffer touched once per step",
                       "parallelism": f"replica{ws}" if ws > 1 else "single"},
            "roofline": roof, "per_op": {k: {"ms": round(v["ms"], 5), "GB/s": round(v["GB/s"], 1)}
                                         for k, v in per_op.items()},
            "e2e": {"value": round(e2e_val, 3), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "steps": e2e_steps},
            "gpu_launches": n_launch, "clocks": clocks, "cpu_baseline": cpu}
    del wls, ops, evs
    torch.cuda.empty_cache()
    return line


# DRAM traffic per launch from ncu captures (profiles/); None until captured.
TRAFFIC: dict = {}


# ---- GEMV shapes of one config-3 decode step (per-launch CUDA events) -------------------------

GEMV_SHAPES = [("o_proj", 2048, 2048), ("qkv", 4096, 2048), ("gate_up", 12288, 2048), ("down", 2048, 6144),
               ("lm_head", 217472, 2048)]


def run_gemv_shapes(dev, reps=20):
    """Q8_0 GEMV (M=1) at every linear shape of the 1.7B decode step, each timed alone (events
    around `reps` back-to-back launches; 3 warm-up launches first; weights > L2 only for the
    head, so the small shapes are partly L2-served here)."""
    import torch

    import acb
    out = {"metric": "Q8_0 GEMV GB/s per decode shape (M=1)", "shapes": {}}
    for name, N, K in GEMV_SHAPES:
        rb = K // 32 * 34
        W = torch.randint(0, 256, (N * rb + 256,), dtype=torch.uint8, device=dev)
        W[: N * rb].view(N, K // 32, 34)[:, :, 0:2] = torch.tensor([0x00, 0x14], dtype=torch.uint8, device=dev)
        x = torch.randn(1, K, device=dev)
        y = torch.empty(1, N, device=dev)
        nbytes = N * rb + K * 4 + N * 4
        res = {"N": N, "K": K}
        Wt = acb.q8_0_to_tiles(W, N, K) if N % 16 == 0 else None
        for form, WW, wt in (("gguf", W, acb.Q8_0), ("tiles", Wt, acb.Q8_0_TILES)):
            if WW is None:
                continue
            for _ in range(3):
                acb.gemv(WW, wt, N, K, x, y=y)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(reps):
                acb.gemv(WW, wt, N, K, x, y=y)
            e1.record()
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) / reps * 1e3
            res[form] = {"us": round(us, 2), "GB/s": round(nbytes / us / 1e3, 1)}
        out["shapes"][name] = res
        del W, Wt
    return out


# ---- tcgen05 GEMM at the DiT layer shapes (M = 8 sequences x 750 tokens) -----------------------

GEMM_SHAPES = [("sa_qkv", 6000, 4096, 2048), ("sa_o", 6000, 2048, 2048), ("gate_up", 6000, 12288, 2048),
               ("down", 6000, 2048, 6144)]


def run_gemm_shapes(dev, reps=20, which=None):
    """acb_gemm_tc per DiT linear shape, CUDA events around `reps` launches after 3 warm-ups:
    bf16 operands over K, and the exact mode's f16 operands over K' = 3K (hi/lo splits). TFLOP/s
    of tensor work against the measured bf16 peak."""
    import torch

    import acb
    peaks, kind = measured_peaks()
    out = {"metric": "tcgen05 GEMM TFLOP/s per DiT shape (tensor work)", "peak_tflops": peaks["bf16_tflops"],
           "peak_kind": kind, "shapes": {}}
    for name, M, N, K in GEMM_SHAPES:
        if which and name not in which:
            continue
        res = {"M": M, "N": N, "K": K}
        for mode, dt, Kp in (("bf16", torch.bfloat16, K), ("f16_exact3K", torch.float16, 3 * K)):
            A = torch.randn(M, Kp, device=dev).to(dt)
            B = (torch.randn(N, Kp, device=dev) * 0.02).to(dt)
            C = torch.empty(M, N, device=dev, dtype=torch.float32)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(3):
                acb.gemm_bf16(A, B, out=C)
            e1.record()
            torch.cuda.synchronize()
            # enough launches for ~150 ms of steady-state work (clocks settle under the power cap)
            reps = max(20, int(150.0 / max(e0.elapsed_time(e1) / 3, 1e-3)))
            e0.record()
            for _ in range(reps):
                acb.gemm_bf16(A, B, out=C)
            e1.record()
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) / reps * 1e3
            tf = 2.0 * M * N * Kp / (us * 1e-6) / 1e12
            res[mode] = {"us": round(us, 1), "TFLOP/s": round(tf, 1), "frac": round(tf / peaks["bf16_tflops"], 3)}
            # the same product through cuBLAS (torch.matmul, 16-bit output), for comparison only
            Cl = torch.empty(M, N, device=dev, dtype=dt)
            for _ in range(3):
                torch.matmul(A, B.T, out=Cl)
            e0.record()
            for _ in range(reps):
                torch.matmul(A, B.T, out=Cl)
            e1.record()
            torch.cuda.synchronize()
            us_l = e0.elapsed_time(e1) / reps * 1e3
            res[mode]["cublas_TFLOP/s"] = round(2.0 * M * N * Kp / (us_l * 1e-6) / 1e12, 1)
            del A, B, C, Cl
        out["shapes"][name] = res
    return out


ATTN_SHAPES = [("dit_self_window", 8, 750, 750, 2, 128), ("dit_self_full", 8, 750, 750, 0, 0),
               ("dit_cross", 8, 750, 512, 0, 0), ("enc_causal", 1, 256, 256, 1, 0)]


def run_attn_shapes(dev, reps=10, which=None):
    """acb_attn_prefill (mma.sync; f16 operands, and hi/lo planes of the exact mode) and acb_attn_tc
    (tcgen05; the same two operand forms) per attention shape of configs 1 and 4 (16 q heads, 8 kv heads, D 128), CUDA events around
    `reps` launches after 3 warm-ups; algorithmic TFLOP/s (QK^T and PV over the unmasked pairs)."""
    import torch

    import acb
    out = {"metric": "prefill/DiT attention algorithmic TFLOP/s per shape", "shapes": {}}
    Nh, Nkv, D = 16, 8, 128
    for name, B, Sq, Skv, mask, win in ATTN_SHAPES:
        if which and name not in which:
            continue
        g = torch.Generator(device=dev).manual_seed(Sq + Skv)
        q = torch.randn(B, Sq, Nh * D, device=dev, generator=g)
        k = torch.randn(B, Skv, Nkv * D, device=dev, generator=g)
        v = torch.randn(B, Skv, Nkv * D, device=dev, generator=g)
        planes = [acb.act_quant_ex(t.reshape(-1, t.shape[-1]), t.shape[-1], acb.F16, acb.LAYOUT_PLANES)
                  for t in (q, k, v)]
        hi = [p[: p.shape[0] // 2].view(t.shape) for p, t in zip(planes, (q, k, v))]
        lo = [t.numel() for t in (q, k, v)]
        o = torch.empty(B, Sq, Nh * D, device=dev)
        vt_h, vld, _ = acb.attn_vt(hi[2], Nkv)
        vt_s, _, vlo = acb.attn_vt(v, Nkv, lo=True)
        qf, kf = planes[0], planes[1]
        pairs = sum(min(Skv, i + win + 1) - max(0, i - win) for i in range(Sq)) if mask == 2 else \
            (Sq * (Sq + 1) // 2 if mask == 1 else Sq * Skv)
        fl = 4.0 * D * Nh * B * pairs
        res = {"B": B, "Sq": Sq, "Skv": Skv, "mask": mask}
        for mode in ("f16", "split", "tc_f16", "tc_split"):
            def call():
                if mode == "f16":
                    acb.attn_prefill(hi[0], hi[1], hi[2], Nh, Nkv, mask=mask, window=win, out=o)
                elif mode == "split":
                    acb.attn_prefill_split(hi[0], hi[1], hi[2], lo[0], lo[1], lo[2], Nh, Nkv, mask=mask,
                                           window=win, out=o)
                elif mode == "tc_f16":
                    acb.attn_tc(qf[: B * Sq], kf[: B * Skv], vt_h, vld, Nh, Nkv, Sq, Skv, B, mask=mask, window=win,
                                out=o.view(B * Sq, -1))
                else:
                    acb.attn_tc(qf[: B * Sq], kf[: B * Skv], vt_s, vld, Nh, Nkv, Sq, Skv, B, mask=mask, window=win,
                                out=o.view(B * Sq, -1), q_lo=lo[0], k_lo=lo[1], vt_lo=vlo)
            for _ in range(3):
                call()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(reps):
                call()
            e1.record()
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) / reps * 1e3
            res[mode] = {"us": round(us, 1), "TFLOP/s": round(fl / (us * 1e-6) / 1e12, 1)}
        out["shapes"][name] = res
    return out


# ---- workload: BASELINE config 3 (Qwen3-1.7B-shaped LM, greedy decode, batch 1) ----------------

LM_PROMPT, LM_GEN = 512, 1024


def lm_weight_bytes(cfg) -> int:
    """Weight bytes streamed per decoded token (every linear + the tied head), Q8_0."""
    H, F, L = cfg["hidden_size"], cfg["intermediate_size"], cfg["num_hidden_layers"]
    Nh, Nkv, D, V = cfg["num_attention_heads"], cfg["num_key_value_heads"], cfg["head_dim"], cfg["vocab_size"]
    q8 = lambda n, k: n * (k // 32) * 34
    per_layer = q8((Nh + 2 * Nkv) * D, H) + q8(H, Nh * D) + q8(2 * F, H) + q8(H, F) + (2 * H + 2 * D) * 4
    return L * per_layer + q8(V, H) + H * 4


def run_lm(dev, rank, warm_tokens=16, want_cpu=True, gguf_dir=None, prompt_len=LM_PROMPT, gen_len=LM_GEN):
    """Config 3 on this GPU: returns the lm_decode result dict."""
    import tempfile

    import numpy as np
    import torch

    import acb
    import synthetic

    cfg = dict(synthetic.QWEN3_1_7B)
    d = gguf_dir or tempfile.gettempdir()
    path = os.path.join(d, f"acb_bench_lm17_q8_0_r{rank}.gguf")
    keep = {} if want_cpu else None
    t0 = time.time()
    synthetic.write_lm_gguf(path, cfg, synthetic.policy_q8_0, seed=42, device=str(dev), keep=keep)
    t_gen = time.time() - t0
    m = acb.QW3LM(path, max_seq_len=8192, n_kv_sets=1, device=dev.index or 0)
    persist = m.persistent_decode()
    rng = np.random.default_rng(7)
    prompt = rng.integers(0, cfg["vocab_size"], size=prompt_len).astype(np.int32)
    t0 = time.time()
    lg = m.forward(prompt, kv_set=0)
    t_prefill = time.time() - t0
    first = int(np.argmax(lg))
    # warm-up (captures the step graph), then the timed stretch of the 1024 generated tokens
    toks_w, _, _ = m.generate_greedy([first], 0, warm_tokens)
    n_timed = gen_len - warm_tokens
    torch.cuda.profiler.start()  # profiler range = the timed decode loop (no effect without a profiler)
    toks, _, gpu_ms = m.generate_greedy([int(toks_w[0, -1])], 0, n_timed)
    torch.cuda.profiler.stop()
    tok_s = n_timed / (gpu_ms * 1e-3)
    wb = lm_weight_bytes(cfg)
    # KV bytes read per token at the average context of the timed stretch (K and V, f16)
    avg_ctx = prompt_len + warm_tokens + n_timed / 2
    kv_b = int(avg_ctx * cfg["num_hidden_layers"] * cfg["num_key_value_heads"] * cfg["head_dim"] * 2 * 2)
    per_tok_bytes = wb + kv_b
    # e2e through the reference-facing API: host ids in, host logits out, host argmax
    nxt = int(toks[0, -1])
    e2e_n = 32
    t0 = time.perf_counter()
    for _ in range(e2e_n):
        lg = m.forward_batch(np.array([nxt], np.int32), [0])
        nxt = int(np.argmax(lg[0]))
    e2e_s = time.perf_counter() - t0
    V = cfg["vocab_size"]
    # dominant kernel: the head-shaped GEMV (217472 x 2048 Q8_0, M=1), timed alone with events
    head = torch.randint(0, 256, (V * 2176 + 256,), dtype=torch.uint8, device=dev)
    head.view(-1)[: V * 2176].view(V, 64, 34)[:, :, 0:2] = torch.tensor([0x00, 0x14], dtype=torch.uint8,
                                                                        device=dev)  # d = 2^-10 (f16 0x1400)
    x = torch.randn(1, 2048, device=dev)
    y = torch.empty(1, V, device=dev)
    for _ in range(3):
        acb.gemv(head, acb.Q8_0, V, 2048, x, y=y)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 20
    e0.record()
    for _ in range(reps):
        acb.gemv(head, acb.Q8_0, V, 2048, x, y=y)
    e1.record()
    torch.cuda.synchronize()
    head_ms = e0.elapsed_time(e1) / reps
    head_bytes = V * 2176 + 2048 * 4 + V * 4
    peaks, kind = measured_peaks()
    # greedy identity (the same token stream for the first 256 tokens): the
    # timed path's tokens against the per-op graph (ACB_LM_PERSIST=0) and the CPU oracle on the
    # same weights, from the same prompt
    n_cmp = min(256, gen_len)
    ours = np.concatenate([toks_w[0], toks[0]])[:n_cmp]
    lead = lambda a, b: int(next((i for i, (x, y) in enumerate(zip(a, b)) if x != y), min(len(a), len(b))))
    ident = {"tokens": n_cmp, "path_timed": "persistent" if persist else "per-op graph"}
    if persist:
        os.environ["ACB_LM_PERSIST"] = "0"
        try:
            m2 = acb.QW3LM(path, max_seq_len=8192, n_kv_sets=1, device=dev.index or 0)
        finally:
            del os.environ["ACB_LM_PERSIST"]
        m2.forward(prompt, kv_set=0)
        a, _, _ = m2.generate_greedy([first], 0, n_cmp)
        m2.close()
        ident["per_op_graph_identical"] = lead(a[0].tolist(), ours.tolist())
    cpu_decode = None
    if want_cpu:
        otoks, first_o, cpu_decode = cpu_lm_greedy(cfg, keep, prompt, n_cmp)
        ident["oracle_first_token_equal"] = bool(first_o == first)
        ident["identical_to_oracle"] = lead(otoks, ours.tolist()) if first_o == first else 0
    step_gbs = per_tok_bytes * tok_s / 1e9
    res = {
        "metric": "LM decode tok/s (config 3: Qwen3-1.7B shape, Q8_0, batch 1, greedy)",
        "value": round(tok_s, 2), "unit": "tok/s", "higher_is_better": True,
        "ms_per_token": round(gpu_ms / n_timed, 4),
        "config": {"workload": "config3_lm17_q8_0_decode", "prompt": prompt_len, "generated": gen_len,
                   "timed_tokens": n_timed, "kv_cache": "f16 max_seq 8192", "weights_MB": round(wb / 1e6, 1),
                   "setup_s": {"gguf_write": round(t_gen, 1), "prefill": round(t_prefill, 2)}},
        "hbm": {"bytes_per_token": per_tok_bytes, "achieved_GBs": round(per_tok_bytes * tok_s / 1e9, 1),
                "frac_of_measured": round(per_tok_bytes * tok_s / 1e9 / peaks["hbm_gbs"], 4),
                "bound_us_per_token": round(per_tok_bytes / (peaks["hbm_gbs"] * 1e3), 1),
                "ratio_to_bound": round((gpu_ms / n_timed * 1e3) / (per_tok_bytes / (peaks["hbm_gbs"] * 1e3)), 3)},
        "path": "persistent (acb_lm_decode_step, up to 64 greedy tokens per launch)" if persist else "per-op graph",
        "roofline": ({"kernel": "lm_decode_kernel (whole step: weights + KV cache bytes per token)", "bound": "hbm",
                      "achieved": round(step_gbs, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                      "frac": round(step_gbs / peaks["hbm_gbs"], 4), "traffic": None} if persist else
                     {"kernel": "gemv_kernel<Q8_0,M=1> 217472x2048 (LM-head shape)", "bound": "hbm",
                      "achieved": round(head_bytes / (head_ms * 1e-3) / 1e9, 1), "peak": peaks["hbm_gbs"],
                      "unit": "GB/s", "frac": round(head_bytes / (head_ms * 1e-3) / 1e9 / peaks["hbm_gbs"], 4),
                      "traffic": None}),
        "head_gemv_alone": {"kernel": "gemv_kernel<Q8_0,M=1> 217472x2048", "GBs": round(head_bytes / (head_ms * 1e-3) / 1e9, 1)},
        "greedy_identity": ident,
        "e2e": {"value": round(e2e_n / e2e_s, 2), "unit": "tok/s", "h2d_bytes_per_step": 8,
                "d2h_bytes_per_step": V * 4, "path": "acb_qw3lm_forward_batch + host argmax"},
        "tokens_head": toks[0, :8].tolist(),
    }
    if cpu_decode:
        res["cpu_baseline"] = cpu_decode
    m.close()
    del keep
    try:
        os.remove(path)
    except OSError:
        pass
    return res


# ---- workload: BASELINE config 5's LM (Qwen3-4B shape, Q4_K_M, one sequence per GPU) ------------

LM5_PROMPT, LM5_GEN = 1024, 2048


def run_lm5(dev, rank, ws, prompt_len=LM5_PROMPT, gen_len=LM5_GEN, warm_tokens=16):
    """Config 5's LM on every rank: the Qwen3-4B shape quantised with the Q4_K_M policy of
    tools/quantize.cpp (Q4_K base, v/down bumped to Q6_K in the listed layers, Q6_K embedding =
    tied head), a 1024-token random prompt and 2048 greedy tokens per sequence, one independent
    sequence per GPU (weak scaling, no exchange during decode). The ranks' token streams are
    gathered over NCCL at the end. Time: the library's CUDA events around the device greedy loop,
    max over ranks; value = all ranks' tokens / that time."""
    import tempfile

    import numpy as np
    import torch

    import acb
    import synthetic

    cfg = dict(synthetic.QWEN3_4B)
    V = cfg["vocab_size"]
    path = os.path.join(tempfile.gettempdir(), "acb_bench_lm4b_q4_k_m.gguf")
    t0 = time.time()
    if rank == 0:
        synthetic.write_lm_gguf(path, cfg, synthetic.policy_q4_k_m, seed=45, device=str(dev))
    if ws > 1:
        torch.distributed.barrier()
    t_gen = time.time() - t0
    m = acb.QW3LM(path, max_seq_len=prompt_len + gen_len + 64, n_kv_sets=1, device=dev.index or 0)
    wb = m.weight_bytes()
    rng = np.random.default_rng(70 + rank)
    prompt = rng.integers(0, V, size=prompt_len).astype(np.int32)
    t0 = time.time()
    lg = m.forward(prompt, kv_set=0)
    t_prefill = time.time() - t0
    toks_w, _, _ = m.generate_greedy([int(np.argmax(lg))], 0, warm_tokens)
    n_timed = gen_len - warm_tokens
    if ws > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    torch.cuda.profiler.start()  # profiler range = the timed decode loop (no effect without a profiler)
    toks, _, gpu_ms = m.generate_greedy([int(toks_w[0, -1])], 0, n_timed)
    torch.cuda.profiler.stop()
    import multi
    ids = torch.from_numpy(np.concatenate([toks_w[0], toks[0]]).astype(np.int64)).to(dev)
    gathered = multi.gather_rows(ids[None], ws)  # the final token-id gather of the sharded job
    ms = multi.max_over_ranks(gpu_ms, ws, dev)
    persist = m.persistent_decode()
    m.close()
    if ws > 1:
        torch.distributed.barrier()
    if rank == 0:
        try:
            os.remove(path)
        except OSError:
            pass
    peaks, _ = measured_peaks()
    avg_ctx = prompt_len + warm_tokens + n_timed / 2
    kv_b = int(avg_ctx * cfg["num_hidden_layers"] * cfg["num_key_value_heads"] * cfg["head_dim"] * 2 * 2)
    per_tok = wb + kv_b
    ms_tok = ms / n_timed
    return {
        "metric": "LM decode tok/s (config 5 LM: Qwen3-4B shape, Q4_K_M, one sequence per GPU, greedy)",
        "value": round(ws * n_timed / (ms * 1e-3), 2), "unit": "tok/s", "n_gpus": ws, "scaling": "weak",
        "ms_per_token": round(ms_tok, 4),
        "config": {"workload": "config5_lm4b_q4_k_m_decode", "prompt": prompt_len, "generated": gen_len,
                   "timed_tokens_per_gpu": n_timed, "weights_MB": round(wb / 1e6, 1),
                   "path": "persistent step" if persist else "per-op graph (Q4_K / Q6_K GEMVs)",
                   "setup_s": {"gguf_write": round(t_gen, 1), "prefill": round(t_prefill, 2)}},
        "hbm": {"bytes_per_token": per_tok, "bound_us_per_token": round(per_tok / (peaks["hbm_gbs"] * 1e3), 1),
                "ratio_to_bound": round(ms_tok * 1e3 / (per_tok / (peaks["hbm_gbs"] * 1e3)), 3),
                "achieved_GBs_per_gpu": round(per_tok / (ms_tok * 1e-3) / 1e9, 1)},
        "tokens_gathered": int(gathered.numel()),
        "tokens_head_rank0": toks_w[0, :4].tolist(),
        "cpu_baseline": None,
        "note": "no CPU sample for this sub-result (the 4B K-quant oracle needs minutes per token); "
                "config 3's line carries the decode CPU baseline",
    }


ENC_S = 256


def enc_flops(cfg, S) -> int:
    """Algorithmic FLOPs of one encoder forward: every linear (2*S*N*K) plus causal attention
    (QK^T and PV over the S(S+1)/2 unmasked pairs, 2*D flops each, per head)."""
    H, F, L = cfg["hidden_size"], cfg["intermediate_size"], cfg["num_hidden_layers"]
    Nh, Nkv, D = cfg["num_attention_heads"], cfg["num_key_value_heads"], cfg["head_dim"]
    lin = (Nh + 2 * Nkv) * D * H + H * Nh * D + 2 * F * H + H * F
    att = 2 * (2 * D) * Nh * (S * (S + 1) // 2)
    return L * (2 * S * lin + att)


def run_enc(dev, rank, want_cpu=True, S=ENC_S, reps=50):
    """Config 1 on this GPU: the Qwen3-0.6B-shaped text encoder, 256 tokens, Q8_0 weights."""
    import tempfile

    import numpy as np
    import torch

    import acb
    import synthetic

    cfg = dict(synthetic.QWEN3_EMBED_0_6B)
    path = os.path.join(tempfile.gettempdir(), f"acb_bench_enc06_q8_0_r{rank}.gguf")
    keep = {} if want_cpu else None
    synthetic.write_lm_gguf(path, cfg, synthetic.policy_q8_0, seed=3, device=str(dev), keep=keep, prefix="",
                            arch="qwen3")
    enc = acb.Qwen3Encoder(path, device=dev.index or 0)
    ids = np.random.default_rng(11).integers(0, cfg["vocab_size"], S).astype(np.int32)
    d_ids = torch.from_numpy(ids).to(dev)
    d_out = torch.empty((S, cfg["hidden_size"]), dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream()
    for _ in range(5):
        enc.forward_device(d_ids, d_out, stream)
    torch.cuda.synchronize()
    # the 0.9 GB of f16 weights exceed the 126 MB L2: back-to-back forwards stream them from HBM
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.profiler.start()  # profiler range = the timed forwards (no effect without a profiler)
    e0.record(stream)
    for _ in range(reps):
        enc.forward_device(d_ids, d_out, stream)
    e1.record(stream)
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    ms = e0.elapsed_time(e1) / reps
    n_kernels = enc.forward_kernels()  # nodes of the forward's captured graph
    fl = enc_flops(cfg, S)
    # e2e: host ids in, host hidden states out (acb_qwen3_forward, the qwen3_forward drop-in)
    out = enc.forward(ids)
    t0 = time.perf_counter()
    e2e_n = 20
    for _ in range(e2e_n):
        out = enc.forward(ids)
    e2e_s = (time.perf_counter() - t0) / e2e_n
    peaks, kind = measured_peaks()
    res = {
        "metric": "text-encoder forwards/s (config 1: Qwen3-0.6B shape, Q8_0 weights, 256 tokens)",
        "value": round(1e3 / ms, 2), "unit": "forward/s", "higher_is_better": True, "ms_per_forward": round(ms, 4),
        "tokens_per_s": round(S * 1e3 / ms, 1),
        "config": {"workload": "config1_text_encoder_q8_0", "tokens": S, "layers": cfg["num_hidden_layers"],
                   "weights": "Q8_0 in the GGUF, resident f16 copies; activations quantised like ggml (Q8_0)",
                   "weight_bytes_device": enc.weight_bytes()},
        "roofline": {"kernel": "whole forward (tcgen05 GEMMs dominate)", "bound": "tensor",
                     "achieved": round(fl / (ms * 1e-3) / 1e12, 1), "peak": peaks["bf16_tflops"],
                     "peak_kind": kind, "unit": "TFLOP/s",
                     "frac": round(fl / (ms * 1e-3) / 1e12 / peaks["bf16_tflops"], 4),
                     "flops_per_forward": fl, "traffic": None},
        "e2e": {"value": round(1.0 / e2e_s, 2), "unit": "forward/s", "h2d_bytes_per_step": S * 4,
                "d2h_bytes_per_step": S * cfg["hidden_size"] * 4, "path": "acb_qwen3_forward"},
        "gpu_launches_per_forward": n_kernels,
    }
    if want_cpu:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as O
        tensors = {n: (qt, raw, K, raw.shape[0] if raw.ndim > 1 else 1) for n, (qt, raw, K) in keep.items()}
        om = O.qwen3_from_gguf_tensors(cfg, tensors, prefix="")
        t0 = time.perf_counter()
        ref = om.encode(ids)
        dt = time.perf_counter() - t0
        res["cpu_baseline"] = {"value": round(1.0 / dt, 4), "unit": "forward/s", "cores": O.get_threads(),
                               "kind": "port", "sample": "one full oracle forward (ggml-CPU mul_mat semantics), "
                                                         "same weights and ids"}
        num = (out.astype(np.float64) * ref).sum(1)
        den = np.linalg.norm(out, axis=1) * np.linalg.norm(ref, axis=1)
        res["parity_vs_oracle"] = {"min_row_cosine": round(float((num / den).min()), 8)}
    enc.close()
    del keep
    try:
        os.remove(path)
    except OSError:
        pass
    return res


# latent frames: 86.8 s of 48 kHz stereo audio (1920 samples per frame), the length the reference
# logs its tiled decode at (tests/CUDA0-Q8_0.log:216-222: 3 tiles of chunk 1024 / overlap 64)
VAE_T = 2170


def run_cond_logged(dev, rank, reps=10):
    """The conditioning the reference logs on its own GPU (tests/CUDA0-Q8_0.log:406-433): the BF16
    Qwen3-0.6B text encoder on 70 caption tokens, the lyric embedding lookup of 167 tokens, and the
    Q8_0 condition encoder (lyric 8 layers with the 128 sliding window, timbre 4 layers on one
    reference row, text projection) packed into enc_S = 238 rows; 15.9 ms warm there on an RTX PRO
    6000. Timed here as the three host calls of acb_qwen3_forward, acb_qwen3_embed_lookup and
    acb_cond_forward (host buffers in and out)."""
    import tempfile

    import numpy as np

    import acb
    import synthetic

    tcfg = dict(synthetic.QWEN3_EMBED_0_6B)
    tpath = os.path.join(tempfile.gettempdir(), f"acb_bench_textenc_bf16_r{rank}.gguf")
    synthetic.write_lm_gguf(tpath, tcfg, synthetic.policy_bf16, seed=3, device=str(dev), prefix="", arch="qwen3")
    cpath = os.path.join(tempfile.gettempdir(), f"acb_bench_cond_q8_0_r{rank}.gguf")
    synthetic.write_dit_gguf(cpath, dict(synthetic.ACESTEP_DIT_2B), synthetic.Q8_0, seed=21, device=str(dev),
                             cond=dict(synthetic.ACESTEP_COND), decoder=False)
    enc = acb.Qwen3Encoder(tpath, device=dev.index or 0)
    cond = acb.CondEncoder(cpath, device=dev.index or 0)
    os.remove(tpath)
    os.remove(cpath)
    rng = np.random.default_rng(42)
    text_ids = rng.integers(0, tcfg["vocab_size"], 70).astype(np.int32)
    lyric_ids = rng.integers(0, tcfg["vocab_size"], 167).astype(np.int32)
    timbre = rng.standard_normal((1, synthetic.ACESTEP_COND["latent_dim"])).astype(np.float32)

    def chain():
        return cond.forward(enc.forward(text_ids), enc.embed_lookup(lyric_ids), timbre)

    for _ in range(3):
        out = chain()
    times = []
    for _ in range(reps):
        t0 = time.perf_counter()
        out = chain()
        times.append((time.perf_counter() - t0) * 1e3)
    enc.close()
    cond.close()
    ms = float(np.median(times))
    return {
        "metric": "conditioning ms (the reference's logged case: text encoder 70 tokens + lyric 167 -> enc_S 238)",
        "value": round(ms, 3), "unit": "ms", "higher_is_better": False,
        "config": {"workload": "cond_logged_case", "text_tokens": 70, "lyric_tokens": 167, "timbre_rows": 1,
                   "enc_rows": int(out.shape[0]), "text_encoder": "Qwen3-0.6B shape, BF16",
                   "cond_encoder": "lyric 8L + timbre 4L, Q8_0", "mode": "exact"},
        "e2e": {"value": round(ms, 3), "unit": "ms",
                "path": "acb_qwen3_forward + acb_qwen3_embed_lookup + acb_cond_forward (host buffers)",
                "h2d_bytes_per_step": int(text_ids.nbytes + lyric_ids.nbytes + timbre.nbytes),
                "d2h_bytes_per_step": int(out.nbytes)},
        "reference_published": "15.9 ms warm on an RTX PRO 6000, ggml-CUDA (tests/CUDA0-Q8_0.log:433; "
                               "other hardware, context only)",
        "finite": bool(np.isfinite(out).all()),
    }


def vae_flops(vcfg, T) -> int:
    """Multiply-adds x 2 of the decoder's convolutions for T latent frames (src/vae.h:344-369)."""
    fl = 2 * T * vcfg["c0"] * 7 * vcfg["latent"]
    t = T
    for ic, oc, s in zip(vcfg["in_ch"], vcfg["out_ch"], vcfg["strides"]):
        fl += 2 * t * ic * 2 * s * oc  # ConvTranspose (GEMM into 2s columns per input step)
        t *= s
        fl += 3 * 2 * t * (7 * oc * oc + oc * oc)  # res units: k7 conv + k1 conv
    return fl + 2 * t * 2 * 7 * vcfg["out_ch"][-1]


def run_vae(dev, rank, want_cpu=True, T=VAE_T, reps=10):
    """The VAE decoder (the shipped AutoencoderOobleck shape, BF16 GGUF, random weights) on 86.8 s of
    audio: device-resident timing of one untiled decode, and the pipeline's host call
    (vae_ggml_decode_tiled with its default chunk 1024 / overlap 64: three windows) end to end."""
    import tempfile

    import numpy as np
    import torch

    import acb
    import synthetic

    vcfg = dict(synthetic.ACESTEP_VAE)
    path = os.path.join(tempfile.gettempdir(), f"acb_bench_vae_r{rank}.gguf")
    keep = {} if want_cpu else None
    synthetic.write_vae_gguf(path, vcfg, seed=4, keep=keep)
    vae = acb.VAE(path, device=dev.index or 0)
    os.remove(path)
    lat = np.random.default_rng(5).standard_normal((T, vcfg["latent"])).astype(np.float32)
    d_lat = torch.from_numpy(lat).to(dev)
    d_out = torch.empty((2, T * vae.up), dtype=torch.float32, device=dev)
    for _ in range(3):
        vae.decode_device(d_lat, d_out)
    torch.cuda.synchronize()
    # activations of 1-4 GB per layer at the last block: every pass streams them from HBM
    ms_all = []
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        vae.decode_device(d_lat, d_out)
        e1.record()
        torch.cuda.synchronize()
        ms_all.append(e0.elapsed_time(e1))
    ms = float(np.median(ms_all))
    audio_s = T * vae.up / 48000.0
    out = vae.decode_tiled(lat, chunk_size=1024, overlap=64)
    t0 = time.perf_counter()
    e2e_n = 5
    for _ in range(e2e_n):
        out = vae.decode_tiled(lat, chunk_size=1024, overlap=64)
    e2e_s = (time.perf_counter() - t0) / e2e_n
    fl = vae_flops(vcfg, T)
    peaks, kind = measured_peaks()
    res = {
        "metric": "VAE decode throughput (audio seconds per second; AutoencoderOobleck, 86.8 s of 48 kHz stereo)",
        "value": round(audio_s / (ms * 1e-3), 1), "unit": "audio_s/s", "higher_is_better": True,
        "ms_per_decode": round(ms, 3),
        "config": {"workload": "vae_decode_86s", "latent_frames": T, "audio_samples": T * vae.up,
                   "channels": [vcfg["c0"]] + vcfg["out_ch"], "strides": vcfg["strides"],
                   "weights": "BF16 in the GGUF, weight-norm fused at load into f16 (as the reference)"},
        "roofline": {"kernel": "whole decode (tcgen05 implicit-GEMM convs dominate)", "bound": "tensor",
                     "achieved": round(fl / (ms * 1e-3) / 1e12, 1), "peak": peaks["bf16_tflops"],
                     "peak_kind": kind, "unit": "TFLOP/s",
                     "frac": round(fl / (ms * 1e-3) / 1e12 / peaks["bf16_tflops"], 4),
                     "flops_per_decode": fl, "traffic": None},
        "e2e": {"value": round(audio_s / e2e_s, 1), "unit": "audio_s/s", "h2d_bytes_per_step": lat.nbytes,
                "d2h_bytes_per_step": int(out.nbytes), "path": "acb_vae_decode_tiled (chunk 1024, overlap 64)",
                "ms_per_call": round(e2e_s * 1e3, 2),
                "reference_published": "427.6 ms for the same length and tiling on an RTX PRO 6000 "
                                       "(tests/CUDA0-Q8_0.log:222; other hardware, context only)"},
        "gpu_launches_per_decode": 2 + 5 * (2 + 3 * 4) + 1,
    }
    if want_cpu:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as O
        ov = O.OracleVAE(keep)
        n = 3  # bounded sample: 3 latent frames (0.12 s of audio)
        t0 = time.perf_counter()
        ref = ov.decode(lat[:n])
        dt = time.perf_counter() - t0
        res["cpu_baseline"] = {"value": round(n * vae.up / 48000.0 / dt, 4), "unit": "audio_s/s",
                               "cores": O.get_threads(), "kind": "port",
                               "sample": "oracle decode of the first 3 latent frames, same weights"}
        got = vae.decode(lat[:n])
        res["parity_vs_oracle"] = {"cosine": round(float((got.ravel().astype(np.float64) @ ref.ravel()) /
                                                         (np.linalg.norm(got) * np.linalg.norm(ref))), 8)}
    vae.close()
    return res


NOISE_N = 1 << 26  # 64 Mi values, 256 MiB of output: twice the L2


def run_noise(dev, rank, want_cpu=True, reps=20):
    """The reference's seeded noise (src/philox.h philox_randn: Philox4x32-10 + Box-Muller, bf16):
    device fill of 64 Mi values, and end to end the host fill that the pipeline makes per
    generate (pipeline-synth-ops.cpp:761-770: 4 tracks x 2170 frames x 64 channels) through
    acb_philox_randn + a copy into pinned host memory. CPU arm: the reference's own
    tests/test-philox binary (oracle/_ref, compiled from its sources) when present, else the
    oracle port (bit-identical to it)."""
    import subprocess
    import tempfile

    import numpy as np
    import torch

    import acb

    out = torch.empty(NOISE_N, dtype=torch.float32, device=dev)
    for i in range(3):
        acb.philox_randn(i, NOISE_N, out=out)
    torch.cuda.synchronize()
    ms_all = []
    for i in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        acb.philox_randn(100 + i, NOISE_N, out=out)
        e1.record()
        torch.cuda.synchronize()
        ms_all.append(e0.elapsed_time(e1))
    ms = float(np.median(ms_all))
    vps = NOISE_N / (ms * 1e-3)
    n_e2e = 4 * 2170 * 64
    host = torch.empty(n_e2e, dtype=torch.float32).pin_memory()
    buf = torch.empty(n_e2e, dtype=torch.float32, device=dev)
    for i in range(3):
        acb.philox_randn(i, n_e2e, out=buf)
        host.copy_(buf, non_blocking=True)
    torch.cuda.synchronize()
    e2e_reps = 50
    t0 = time.perf_counter()
    for i in range(e2e_reps):
        acb.philox_randn(1000 + i, n_e2e, out=buf)
        host.copy_(buf, non_blocking=True)
        torch.cuda.synchronize()
    e2e_s = (time.perf_counter() - t0) / e2e_reps
    peaks, kind = measured_peaks()
    gbs = NOISE_N * 4 / (ms * 1e-3) / 1e9
    res = {
        "metric": "seeded noise values per second (philox_randn: Philox4x32-10 + Box-Muller, bf16-rounded)",
        "value": round(vps / 1e9, 2), "unit": "Gvalues/s", "higher_is_better": True, "ms_per_fill": round(ms, 4),
        "config": {"workload": "philox_randn_64Mi", "values": NOISE_N, "l2": "output 256 MiB > L2"},
        "roofline": {"kernel": "philox_randn_kernel", "bound": "alu (10 multiply-high rounds + log/sin/sqrt per "
                     "value; 4 bytes written)", "achieved": round(gbs, 1), "peak": peaks["hbm_gbs"],
                     "peak_kind": kind, "unit": "GB/s written", "frac": round(gbs / peaks["hbm_gbs"], 4),
                     "bytes_per_fill": NOISE_N * 4, "traffic": None},
        "e2e": {"value": round(n_e2e / e2e_s / 1e9, 3), "unit": "Gvalues/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": n_e2e * 4, "ms_per_call": round(e2e_s * 1e3, 3),
                "path": "acb_philox_randn + copy to pinned host: one generate's initial noise, 4 x 2170 x 64"},
        "gpu_launches_per_fill": 1,
    }
    if want_cpu:
        n = 1 << 22
        exe = os.path.join(ROOT, "oracle", "_ref", "test-philox")
        if os.access(exe, os.X_OK):
            with tempfile.TemporaryDirectory() as td:
                t0 = time.perf_counter()
                subprocess.run([exe, "42", str(n), os.path.join(td, "n.f32")], check=True, capture_output=True)
                dt = time.perf_counter() - t0
            cpu = {"kind": "reference", "sample": f"the reference's tests/test-philox, {n} values, one thread "
                                                  "(process start and a 16 MiB file write included)"}
        else:
            sys.path.insert(0, os.path.join(ROOT, "oracle"))
            import oracle as O
            before = O.get_threads()
            O.set_threads(1)
            t0 = time.perf_counter()
            O.philox_randn(42, n)
            dt = time.perf_counter() - t0
            O.set_threads(before)
            cpu = {"kind": "port", "sample": f"oracle philox_randn, {n} values, one thread"}
        res["cpu_baseline"] = dict(cpu, value=round(n / dt / 1e9, 4), unit="Gvalues/s", cores=1)
    return res


DIT_TRACKS, DIT_T, DIT_ENC_S, DIT_STEPS, DIT_GUIDANCE = 4, 1500, 512, 8, 3.0


def run_dit_logged(dev, rank, reps=5):
    """The DiT generation the reference logs on its own GPU (tests/CUDA0-Q8_0.log:156-205): one
    track, T = 2170 latent frames (1085 tokens), enc_S = 238, the turbo model's 8 Euler steps at
    shift 3 with guidance 1.0 (no CFG: pipeline-synth.cpp:236-261), Q8_0 weights; 268.2 ms there on
    an RTX PRO 6000. Timed here through acb_dit_generate_ex (dit_ggml_generate's call: host noise,
    context and condition in, host latents out) and by the library's own device clock."""
    import tempfile

    import numpy as np

    import acb
    import synthetic

    cfg = dict(synthetic.ACESTEP_DIT_2B)
    T, enc_S, Oc = 2170, 238, cfg["out_channels"]
    path = os.path.join(tempfile.gettempdir(), f"acb_bench_ditlog_r{rank}.gguf")
    synthetic.write_dit_gguf(path, cfg, synthetic.Q8_0, seed=21, device=str(dev))
    dit = acb.DiT(path, device=dev.index or 0)
    os.remove(path)
    rng = np.random.default_rng(42)
    noise = rng.standard_normal((1, T, Oc)).astype(np.float32)
    ctx = rng.standard_normal((1, T, cfg["in_channels"] - Oc)).astype(np.float32)
    enc = rng.standard_normal((1, enc_S, cfg["enc_hidden_size"])).astype(np.float32)
    sched = acb.turbo_schedule(8, 3.0)
    for _ in range(2):
        dit.generate_ex(noise, ctx, enc, sched, guidance_scale=1.0)
    wall, dev_ms = [], []
    for _ in range(reps):
        t0 = time.perf_counter()
        out, ms = dit.generate_ex(noise, ctx, enc, sched, guidance_scale=1.0)
        wall.append((time.perf_counter() - t0) * 1e3)
        dev_ms.append(ms)
    dit.close()
    e2e_ms, gpu_ms = float(np.median(wall)), float(np.median(dev_ms))
    return {
        "metric": "DiT generation ms (the reference's logged case: 1 track, 1085 tokens, enc_S 238, turbo 8 steps)",
        "value": round(gpu_ms, 2), "unit": "ms", "higher_is_better": False,
        "config": {"workload": "dit_logged_case", "tracks": 1, "frames": T, "tokens": T // 2, "enc_rows": enc_S,
                   "steps": 8, "shift": 3.0, "guidance": 1.0, "weights": "Q8_0 (synthetic)", "mode": "exact"},
        "e2e": {"value": round(e2e_ms, 2), "unit": "ms", "path": "acb_dit_generate_ex",
                "h2d_bytes_per_step": int(noise.nbytes + ctx.nbytes + enc.nbytes),
                "d2h_bytes_per_step": int(out.nbytes)},
        "reference_published": "268.2 ms on an RTX PRO 6000, ggml-CUDA, Q8_0 (tests/CUDA0-Q8_0.log:205; "
                               "other hardware, context only)",
        "x0_finite": bool(np.isfinite(out).all()),
    }


def dit_step_flops(cfg, Ng, S, enc_S) -> int:
    """Algorithmic FLOPs of one DiT evaluation over Ng sequences: every linear (2*rows*N*K; the
    condition K/V projections counted once per step as the reference computes them) plus self
    attention (windowed on even layers) and cross attention (QK^T and PV, 2*D flops each)."""
    H, F, L = cfg["hidden_size"], cfg["intermediate_size"], cfg["n_layers"]
    Nh, Nkv, D = cfg["n_heads"], cfg["n_kv_heads"], cfg["head_dim"]
    R, Re = Ng * S, Ng * enc_S
    QD, KD = Nh * D, Nkv * D
    per_layer = 2 * R * (H * (QD + 2 * KD) + QD * H + H * QD + QD * H + H * 2 * F + F * H) + 2 * Re * H * 2 * KD
    win = cfg["sliding_window"]
    pairs_full = S * S
    pairs_win = sum(min(S, i + win + 1) - max(0, i - win) for i in range(S)) if S > win else S * S
    att = 0
    for l in range(L):
        att += 4 * D * Nh * Ng * (pairs_win if l % 2 == 0 else pairs_full) + 4 * D * Nh * Ng * S * enc_S
    io = 2 * R * (cfg["in_channels"] * cfg["patch_size"] * H + H * cfg["out_channels"] * cfg["patch_size"])
    io += 2 * Re * cfg["enc_hidden_size"] * H
    return L * per_layer + att + io


def run_dit(dev, rank, want_cpu=True, reps=2, modes=("exact", "fast")):
    """Config 4 on this GPU: DiT 24 layers, 4 tracks x CFG 2 (8 sequences), 1500 frames, 512
    condition rows, 8 turbo Euler steps with APG; steps/s of the device step loop."""
    import tempfile

    import numpy as np

    import acb
    import synthetic

    cfg = dict(synthetic.ACESTEP_DIT_2B)
    path = os.path.join(tempfile.gettempdir(), f"acb_bench_dit2b_q8_0_r{rank}.gguf")
    keep = {} if want_cpu else None
    t0 = time.time()
    synthetic.write_dit_gguf(path, cfg, synthetic.Q8_0, seed=21, device=str(dev), keep=keep)
    t_gen = time.time() - t0
    dit = acb.DiT(path, device=dev.index or 0)
    rng = np.random.default_rng(17)
    N, T, enc_S, Oc = DIT_TRACKS, DIT_T, DIT_ENC_S, cfg["out_channels"]
    noise = rng.standard_normal((N, T, Oc)).astype(np.float32)
    ctx = rng.standard_normal((N, T, cfg["in_channels"] - Oc)).astype(np.float32)
    enc = rng.standard_normal((N, enc_S, cfg["enc_hidden_size"])).astype(np.float32)
    sched = acb.turbo_schedule(DIT_STEPS)
    Ng, S = 2 * N, T // cfg["patch_size"]
    fl = dit_step_flops(cfg, Ng, S, enc_S)
    peaks, kind = measured_peaks()
    res = {"metric": "DiT denoise steps/s (config 4: 24 layers, hidden 2048, Q8_0, 4 tracks x CFG 2, 750 tokens, "
                     "512 condition rows, turbo 8 Euler steps with APG)",
           "unit": "step/s", "higher_is_better": True,
           "config": {"workload": "config4_dit2b_q8_0_turbo8_cfg", "tracks": N, "sequences": Ng, "frames": T,
                      "tokens": S, "enc_rows": enc_S, "steps": DIT_STEPS, "guidance": DIT_GUIDANCE,
                      "weight_bytes_device": dit.weight_bytes(), "gguf_write_s": round(t_gen, 1)},
           "flops_per_step": fl}
    for mode in modes:
        dit.set_exact(mode == "exact")
        dit.generate(noise, ctx, enc, sched, guidance_scale=DIT_GUIDANCE)  # captures the step graphs
        ms = []
        import torch
        if mode == modes[0]:
            torch.cuda.profiler.start()  # profiler range = the first mode's timed generates
        for _ in range(reps):
            _, m = dit.generate(noise, ctx, enc, sched, guidance_scale=DIT_GUIDANCE)
            ms.append(m)
        if mode == modes[0]:
            torch.cuda.profiler.stop()
        step_ms = min(ms) / DIT_STEPS
        t1 = time.perf_counter()
        x0, _ = dit.generate(noise, ctx, enc, sched, guidance_scale=DIT_GUIDANCE)
        e2e_s = time.perf_counter() - t1
        res[mode] = {
            "value": round(1e3 / step_ms, 3), "ms_per_step": round(step_ms, 3),
            "tensor_work_multiplier": 3 if mode == "exact" else 1,
            "roofline": {"kernel": "whole denoise step (tcgen05 GEMMs dominate)", "bound": "tensor",
                         "achieved": round(fl / (step_ms * 1e-3) / 1e12, 1), "peak": peaks["bf16_tflops_sustained"],
                         "peak_kind": kind + " sustained", "unit": "TFLOP/s",
                         "frac": round(fl / (step_ms * 1e-3) / 1e12 / peaks["bf16_tflops_sustained"], 4),
                         "traffic": None},
            "e2e": {"value": round(DIT_STEPS / e2e_s, 3), "unit": "step/s",
                    "h2d_bytes_per_step": (noise.nbytes + ctx.nbytes + enc.nbytes) // DIT_STEPS,
                    "d2h_bytes_per_step": x0.nbytes // DIT_STEPS, "path": "acb_dit_generate_solver (host arrays, Euler)"},
        }
    res["value"] = res[modes[0]]["value"]
    if want_cpu:
        res["cpu_baseline"] = cpu_dit_sample(cfg, keep, N, T, enc_S)
    dit.close()
    del keep
    try:
        os.remove(path)
    except OSError:
        pass
    return res


def make_comm(ws, rank, local):
    """The library's NCCL communicator (acb_comm) for the sharded DiT job: rank 0 makes the unique
    id, torch.distributed hands it to the other ranks."""
    import torch

    import acb
    if ws == 1:
        return None
    obj = [acb.Comm.unique_id() if rank == 0 else None]
    torch.distributed.broadcast_object_list(obj, src=0)
    return acb.Comm(obj[0], world=ws, rank=rank, device=local, timeout_ms=120000)


def run_dit_job(args, dev, rank, ws, local, stream):
    """The headline: config 4 denoise steps/s for the whole 8-sequence job (4 tracks x CFG 2),
    sharded over the ranks by the library itself (acb_dit_job_* over acb_comm, the C ABI a C++ host
    uses): whole track pairs per rank at 1, 2 and 4 GPUs (no exchange during the steps), one CFG
    half per rank at 8 GPUs (the partner ranks swap the step's velocity over NCCL). A step of the
    turbo schedule is one timed unit; the 8-step schedule is cycled (APG restarts with every
    cycle). Time: CUDA events on the model's stream, max over ranks."""
    import tempfile

    import numpy as np
    import torch

    import acb
    import synthetic

    import multi

    cfg = dict(synthetic.ACESTEP_DIT_2B)
    N, T, enc_S, Oc = DIT_TRACKS, DIT_T, DIT_ENC_S, cfg["out_channels"]
    Ng, S, ctx_ch = 2 * N, T // cfg["patch_size"], cfg["in_channels"] - Oc
    t0_, n_loc_tr, half, _ = acb.dit_shard_plan(N, 1, ws, rank)
    n_loc = 1 if half >= 0 else 2 * n_loc_tr  # sequences this rank evaluates

    def barrier():
        if ws > 1:
            torch.distributed.barrier()

    # one synthetic checkpoint for all ranks: rank 0 writes it, everyone loads it
    path = os.path.join(tempfile.gettempdir(), "acb_bench_dit2b_q8_0.gguf")
    keep = {} if (rank == 0 and ws == 1 and not args.no_cpu_baseline) else None
    if rank == 0:
        synthetic.write_dit_gguf(path, cfg, synthetic.Q8_0, seed=21, device=str(dev), keep=keep)
    barrier()
    dit = acb.DiT(path, device=local)
    barrier()
    if rank == 0:
        os.remove(path)
    comm = make_comm(ws, rank, local)

    rng = np.random.default_rng(17)
    noise = rng.standard_normal((N, T, Oc)).astype(np.float32)
    ctx = rng.standard_normal((N, T, ctx_ch)).astype(np.float32)
    enc = rng.standard_normal((N, enc_S, cfg["enc_hidden_size"])).astype(np.float32)
    sched = acb.turbo_schedule(DIT_STEPS)
    L = acb.lib()
    C = __import__("ctypes")
    ms_stream = torch.cuda.ExternalStream(L.acb_dit_stream(dit.h), device=dev)

    def job_begin():
        acb._check("acb_dit_job_begin", L.acb_dit_job_begin(
            dit.h, comm.h if comm else None, noise.ctypes.data, ctx.ctypes.data, enc.ctypes.data, enc_S, T, N,
            float(DIT_GUIDANCE), None, -1, None, None, None, None, None, None, None, b"euler", None, None))

    def step(k, h_out=None):
        i = k % DIT_STEPS
        last = i == DIT_STEPS - 1
        acb._check("acb_dit_job_step", L.acb_dit_job_step(
            dit.h, i, float(sched[i]), float(sched[i + 1]) if not last else 0.0, int(last),
            C.c_void_p(h_out.data_ptr()) if h_out is not None else None))

    def timed(K, **kw):
        barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(ms_stream)
        for k in range(K):
            step(k, **kw)
        e1.record(ms_stream)
        torch.cuda.synchronize()
        barrier()
        return multi.max_over_ranks(e0.elapsed_time(e1), ws, dev)

    peaks, kind = measured_peaks()
    fl = dit_step_flops(cfg, Ng, S, enc_S)
    out = {}
    x0_all = np.empty((N, T, Oc), np.float32)
    for mode in ("fast", "exact"):  # the headline mode last
        dit.set_exact(mode == "exact")
        job_begin()
        for k in range(max(args.warmup, 3)):
            step(k)
        K = args.steps if mode == "exact" else min(args.steps, DIT_STEPS)
        clk = ClockSampler(local) if mode == "exact" else None
        if clk:
            clk.start()
            time.sleep(0.3)
        ms = timed(K)
        clocks = clk.stop() if clk else None
        if mode == "exact":
            # end to end: the same steps through the C ABI with this rank's step result (xt, or x0 at
            # the last step) read back to pinned host memory every step (the step's t values go up
            # from the host inside every acb_dit_job_step)
            n_tr_loc = 1 if half >= 0 else n_loc_tr
            h_out = torch.empty((n_tr_loc, T, Oc), dtype=torch.float32, pin_memory=True)
            e2e_k = DIT_STEPS
            e2e_ms = timed(e2e_k, h_out=h_out)
        acb._check("acb_dit_job_end", L.acb_dit_job_end(dit.h, x0_all.ctypes.data, None))
        step_ms = ms / K
        out[mode] = {"value": round(K / (ms * 1e-3), 3), "ms_per_step": round(step_ms, 3), "steps": K,
                     "clocks": clocks,
                     "roofline": {"kernel": "whole denoise step (tcgen05 GEMMs dominate)", "bound": "tensor",
                                  "achieved": round(fl / ws / (step_ms * 1e-3) / 1e12, 1),
                                  "peak": peaks["bf16_tflops_sustained"], "peak_kind": kind + " sustained",
                                  "unit": "TFLOP/s",
                                  "frac": round(fl / ws / (step_ms * 1e-3) / 1e12 / peaks["bf16_tflops_sustained"], 4),
                                  "traffic": None, "tensor_work_multiplier": 3 if mode == "exact" else 1}}
    dom = dominant_gemm(dev, n_loc * S, 2 * cfg["intermediate_size"], cfg["hidden_size"], peaks, kind)
    ex = out["exact"]
    launches = dit.step_kernels()  # the step graph(s) of the last timed step: evaluation, APG, Euler
    line = {"metric": "DiT denoise steps/s (config 4: 24 layers, hidden 2048, Q8_0, 4 tracks x CFG 2 = 8 "
                      "sequences of 750 tokens, 512 condition rows, turbo Euler + APG)",
            "value": ex["value"], "unit": "step/s", "n_gpus": ws, "steps": ex["steps"], "warmup": max(args.warmup, 3),
            "ms_per_step": ex["ms_per_step"], "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "f16 hi/lo split operands (exact products of Q8_0 weights and Q8_0-quantised activations), "
                     "fp32 accumulation",
            "data": "synthetic (random N(0,0.02) weights in Q8_0, N(0,1) latents and condition, seeded)",
            "config": {"workload": "config4_dit2b_q8_0_turbo_cfg", "tracks": N, "sequences": Ng,
                       "sequences_per_gpu": n_loc, "frames": T, "tokens": S, "enc_rows": enc_S,
                       "schedule": "turbo shift 3, 8 steps (cycled)", "guidance": DIT_GUIDANCE,
                       "parallelism": ("one CFG half per GPU, NCCL velocity exchange per step (acb_dit_job_*)"
                                       if half >= 0 else f"track pairs per GPU ({n_loc_tr}), no per-step exchange "
                                       "(acb_dit_job_*)") if ws > 1 else "single",
                       "l2": "weights 9.4 GB and activations > 126 MB L2: every step streams from HBM",
                       "flops_per_step": fl},
            "roofline": dom["roofline"], "step_roofline": ex["roofline"], "dominant_kernel": dom["detail"],
            "clocks": ex["clocks"],
            "e2e": {"value": round(e2e_k / (e2e_ms * 1e-3), 3), "unit": "step/s", "h2d_bytes_per_step": 12,
                    "d2h_bytes_per_step": int(h_out.numel() * 4),
                    "path": "acb_dit_job_step with the step's times from the host and its result to pinned host "
                            "memory every step"},
            "gpu_launches": launches * ex["steps"],
            "x0_finite": bool(np.isfinite(x0_all).all()),
            "fast_mode": {k: out["fast"][k] for k in ("value", "ms_per_step", "roofline")}}
    if keep is not None:
        line["cpu_baseline"] = cpu_dit_sample(cfg, keep, N, T, enc_S)
    dit.close()
    if comm:
        comm.close()
    del keep
    torch.cuda.empty_cache()
    return line


# DRAM bytes of one exact-mode gate|up launch (M=6000, N=12288, K'=6144 f16 operands, f32 output),
# dram__bytes_read.sum + dram__bytes_write.sum from ncu: profiles/gemm_exact_gate_up_ncu.md
GEMM_EXACT_GATE_UP_DRAM = 1277940992 + 278831104


def dominant_gemm(dev, M, N, K, peaks, kind):
    """The dominant kernel of the DiT step (gemm_tc_kernel, 83% of the step: the gate|up shape at
    this rank's rows), exact mode (f16 hi/lo operands over K' = 3K), f32 output, timed alone with
    CUDA events on the launching stream over ~150 ms of back-to-back launches. achieved =
    algorithmic FLOPs 2*M*N*K per launch / the average launch time, against the measured bf16 burst
    peak (the kernel is timed alone); the tensor pipe does 3x that work."""
    import torch

    import acb
    A = torch.randn(M, 3 * K, device=dev).to(torch.float16)
    B = (torch.randn(N, 3 * K, device=dev) * 0.02).to(torch.float16)
    C = torch.empty(M, N, device=dev, dtype=torch.float32)
    st = torch.cuda.current_stream()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    for _ in range(3):
        acb.gemm_bf16(A, B, out=C)
    e0.record(st)
    for _ in range(3):
        acb.gemm_bf16(A, B, out=C)
    e1.record(st)
    torch.cuda.synchronize()
    reps = max(20, int(150.0 / max(e0.elapsed_time(e1) / 3, 1e-3)))
    e0.record(st)
    for _ in range(reps):
        acb.gemm_bf16(A, B, out=C)
    e1.record(st)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) / reps * 1e3
    alg = 2.0 * M * N * K
    ach = alg / (us * 1e-6) / 1e12
    traffic = GEMM_EXACT_GATE_UP_DRAM if (M, N, K) == (6000, 12288, 2048) else None
    del A, B, C
    return {"roofline": {"kernel": f"gemm_tc_kernel<f16, pair> exact mode, gate|up M={M} N={N} K={K} (K'={3 * K})",
                         "bound": "tensor", "achieved": round(ach, 1), "peak": peaks["bf16_tflops"],
                         "peak_kind": kind + " burst", "unit": "TFLOP/s", "frac": round(ach / peaks["bf16_tflops"], 4),
                         "traffic": traffic, "algorithmic_bytes": int(2 * (M + N) * 3 * K + 4 * M * N),
                         "tensor_work_multiplier": 3},
            "detail": {"us_per_launch": round(us, 1), "launches_timed": reps,
                       "tensor_work_TFLOP/s": round(3 * ach, 1),
                       "tensor_frac_of_burst": round(3 * ach / peaks["bf16_tflops"], 4)}}


DIT5_TRACKS, DIT5_STEPS, DIT5_TIMED = 8, 50, 10


def run_dit5_job(args, dev, rank, ws, local, stream):
    """Config 5's DiT leg: the config-4 DiT on the sft schedule (50 steps, shift 1,
    pipeline-synth-ops.cpp:289-309) for 8 tracks x CFG 2 = 16 sequences. Every rank owns whole
    track pairs (track r*8/N .. (r+1)*8/N - 1 with its unconditional twin), so guidance needs no
    exchange during the steps (one pair per GPU at 8 GPUs); the x0 of every track is gathered over
    NCCL at the end, outside the timed region. Timed: DIT5_TIMED consecutive steps of the schedule
    after warm-up steps, CUDA events, max over ranks; value = steps of the whole 16-sequence job per
    second (strong scaling)."""
    import tempfile

    import numpy as np
    import torch

    import acb
    import synthetic

    import multi

    cfg = dict(synthetic.ACESTEP_DIT_2B)
    N, T, enc_S, Oc = DIT5_TRACKS, DIT_T, DIT_ENC_S, cfg["out_channels"]
    S, ctx_ch = T // cfg["patch_size"], cfg["in_channels"] - Oc
    if N % ws:
        raise SystemExit(f"config 5 DiT: {N} tracks do not shard over {ws} ranks")
    nt = N // ws
    mine = list(range(rank * nt, (rank + 1) * nt))
    slots = mine + [N + t for t in mine]  # local order: conditional tracks, then their twins

    def barrier():
        if ws > 1:
            torch.distributed.barrier()

    path = os.path.join(tempfile.gettempdir(), "acb_bench_dit2b_q8_0_c5.gguf")
    if rank == 0:
        synthetic.write_dit_gguf(path, cfg, synthetic.Q8_0, seed=21, device=str(dev))
    barrier()
    dit = acb.DiT(path, device=local)
    import gguf
    null = np.array([t for t in gguf.GGUFReader(path).tensors if t.name == "null_condition_emb"][0].data,
                    dtype=np.float32).reshape(-1)
    barrier()
    if rank == 0:
        os.remove(path)
    rng = np.random.default_rng(55)
    noise = rng.standard_normal((N, T, Oc)).astype(np.float32)
    ctx = rng.standard_normal((N, T, ctx_ch)).astype(np.float32)
    enc = rng.standard_normal((N, enc_S, cfg["enc_hidden_size"])).astype(np.float32)
    enc_loc = np.stack([np.broadcast_to(null, enc.shape[1:]) if j >= N else enc[j] for j in slots])
    dit.set_condition(torch.from_numpy(np.ascontiguousarray(enc_loc)).to(dev), T)
    tracks = torch.tensor([j % N for j in slots], device=dev)
    inp = torch.zeros((2 * nt, T, cfg["in_channels"]), device=dev)
    inp[:, :, :ctx_ch] = torch.from_numpy(ctx).to(dev)[tracks]
    noise_d = torch.from_numpy(noise[mine]).to(dev)
    xt = noise_d.clone()
    vel = torch.empty((2 * nt, T, Oc), device=dev)
    vt = torch.empty((nt, T, Oc), device=dev)
    x0 = torch.empty((nt, T, Oc), device=dev)
    ra = torch.empty((nt, T, Oc), dtype=torch.float64, device=dev)
    sched = acb.turbo_schedule(DIT5_STEPS, shift=1.0)  # shift 1: t_i = 1 - i/50
    tts = torch.tensor([[t, t, sched[i + 1] if i + 1 < DIT5_STEPS else 0.0] for i, t in enumerate(sched)],
                       dtype=torch.float32, device=dev)
    loc_tr = torch.arange(nt, device=dev).repeat(2)

    def step(k, h_tt=None, h_out=None):
        i = k % DIT5_STEPS
        tt = tts[i]
        if h_tt is not None:
            tt = h_tt[1]
            tt.copy_(h_tt[0][i], non_blocking=True)
        inp[:, :, ctx_ch:] = xt[loc_tr]
        dit.eval(inp, tt, vel)
        acb.dit_apg(vel[:nt], vel[nt:], ra, i == 0, DIT_GUIDANCE, vt)
        last = i == DIT5_STEPS - 1
        acb.dit_euler(xt, vt, tt, last, out=x0)
        if last:
            xt.copy_(noise_d)
        if h_out is not None:
            h_out.copy_(x0 if last else xt, non_blocking=True)

    def timed(K, **kw):
        barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for k in range(K):
            step(k, **kw)
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
        return multi.max_over_ranks(e0.elapsed_time(e1), ws, dev)

    for k in range(max(args.warmup, 3)):
        step(k)
    K = DIT5_TIMED
    ms = timed(K)
    h_tts = torch.empty((DIT5_STEPS, 3), dtype=torch.float32, pin_memory=True).copy_(tts)
    d_tt = torch.empty(3, dtype=torch.float32, device=dev)
    h_out = torch.empty((nt, T, Oc), dtype=torch.float32, pin_memory=True)
    e2e_ms = timed(K, h_tt=(h_tts, d_tt), h_out=h_out)
    # the whole generate's result: every rank's x0 gathered (NCCL, outside the timed region)
    for k in range(DIT5_STEPS):
        step(k)
    x0_all = multi.gather_rows(x0, ws)
    peaks, kind = measured_peaks()
    fl = dit_step_flops(cfg, 2 * N, S, enc_S)
    step_ms = ms / K
    ach = fl / (step_ms * 1e-3) / 1e12
    res = {"metric": "DiT denoise steps/s (config 5 DiT: sft 50 steps, shift 1, 8 tracks x CFG 2 = 16 sequences "
                     "of 750 tokens)",
           "value": round(K / (ms * 1e-3), 3), "unit": "step/s", "n_gpus": ws, "steps": K,
           "ms_per_step": round(step_ms, 3), "higher_is_better": True, "scaling": "strong",
           "config": {"workload": "config5_dit2b_q8_0_sft50_cfg", "tracks": N, "sequences": 2 * N,
                      "tracks_per_gpu": nt, "frames": T, "enc_rows": enc_S,
                      "schedule": "sft, shift 1, 50 steps (timed: steps 3..12 of the cycle)",
                      "parallelism": f"track pairs per GPU ({nt}), no per-step exchange; x0 gathered at the end"
                                     if ws > 1 else "single", "flops_per_step": fl},
           "roofline": {"kernel": "whole denoise step (tcgen05 GEMMs dominate)", "bound": "tensor",
                        "achieved": round(ach / ws, 1), "peak": peaks["bf16_tflops_sustained"],
                        "peak_kind": kind + " sustained", "unit": "TFLOP/s",
                        "frac": round(ach / ws / peaks["bf16_tflops_sustained"], 4), "traffic": None,
                        "tensor_work_multiplier": 3},
           "e2e": {"value": round(K / (e2e_ms * 1e-3), 3), "unit": "step/s", "h2d_bytes_per_step": 12,
                   "d2h_bytes_per_step": nt * T * Oc * 4,
                   "path": "acb_dit_eval + acb_dit_apg + acb_dit_euler with per-step pinned host copies"},
           "x0_gathered": list(x0_all.shape), "x0_finite": bool(torch.isfinite(x0_all).all().item()),
           "cpu_baseline": None,
           "note": "the CPU reference arm times config 4's step; one config-5 step is the same work for 16 sequences"}
    dit.close()
    torch.cuda.empty_cache()
    return res


def cpu_dit_sample(cfg, keep, N, T, enc_S):
    """Oracle DiT on the host cores (bounded sample, the reference arm's method): one CFG pair of
    sequences evaluated with 0 and with 1 layer; a step of the 2N-sequence job is
    (t0 + n_layers * (t1 - t0)) * N (every layer and every pair does the same work)."""
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    od = O.dit_from_gguf_tensors(cfg, keep)
    rng = np.random.default_rng(1)
    x = rng.standard_normal((2, T, cfg["in_channels"])).astype(np.float32)
    e = rng.standard_normal((2, enc_S, cfg["enc_hidden_size"])).astype(np.float32)
    t0 = time.perf_counter()
    od.forward(x, e, 0.5, 0.5, n_layers_run=0)
    t_base = time.perf_counter() - t0
    t0 = time.perf_counter()
    od.forward(x, e, 0.5, 0.5, n_layers_run=1)
    t_one = time.perf_counter() - t0
    step = (t_base + cfg["n_layers"] * max(t_one - t_base, 0.0)) * N
    return {"value": round(1.0 / step, 6), "unit": "step/s", "cores": O.get_threads(), "kind": "port",
            "sample": f"oracle evaluations of one CFG pair with 0 and 1 layers ({t_base:.1f} s, {t_one:.1f} s), "
                      f"extrapolated to {cfg['n_layers']} layers x {N} pairs"}


def cpu_lm_greedy(cfg, keep, prompt, n_tokens):
    """The CPU oracle on the same weights: prefill of the whole prompt, then n_tokens greedy
    one-token steps (each streams every weight, like the GPU step). Returns the oracle's tokens,
    its first argmax and the cpu_baseline record (the decode steps timed on all host threads)."""
    import numpy as np
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    tensors = {}
    for name, (qt, raw, K) in keep.items():
        N = raw.shape[0] if raw.ndim > 1 else 1
        tensors[name] = (qt, raw, K, N)
    m = O.qwen3_from_gguf_tensors(cfg, tensors)
    m.alloc_kv(1, len(prompt) + n_tokens + 1)
    t0 = time.perf_counter()
    lg = m.prefill(prompt)
    t_pre = time.perf_counter() - t0
    first = int(np.argmax(lg))
    nxt, toks = first, []
    t0 = time.perf_counter()
    for _ in range(n_tokens):
        lg = m.decode(np.array([nxt], np.int32))[0]
        nxt = int(np.argmax(lg))
        toks.append(nxt)
    dt = time.perf_counter() - t0
    rec = {"value": round(n_tokens / dt, 3), "unit": "tok/s", "cores": O.get_threads(), "kind": "port",
           "sample": f"oracle greedy decode of {n_tokens} tokens after the {len(prompt)}-token prompt "
                     f"(prefill {t_pre:.1f} s, not counted), same Q8_0 weights"}
    return toks, first, rec


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=16, help="timed DiT denoise steps (the headline unit)")
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--lm-prompt", type=int, default=LM_PROMPT)
    ap.add_argument("--lm-gen", type=int, default=LM_GEN)
    ap.add_argument("--lm5-gen", type=int, default=LM5_GEN, help="config 5 LM tokens (profiling runs use fewer)")
    ap.add_argument("--workloads", default="dit,ops,lm,enc,vae,ditlog,condlog,noise,lm5,dit5",
                    help="comma list: dit (config 4, the headline line, every N), ops (config 2), lm (config 3 "
                         "decode), enc (config 1 text encoder), vae (the audio decoder on 86.8 s), ditlog (the DiT "
                         "generation the reference logs: 1 track, turbo, no CFG), condlog (the conditioning it logs) -- "
                         "those six at "
                         "N=1 as sub-results -- and lm5 "
                         "(config 5's 4B Q4_K_M LM, one sequence per GPU, at every N), dit5 (config 5's DiT leg, "
                         "track pairs per GPU, at every N); without dit, ops is the "
                         "headline; or one of gemv / gemm / enc / vae / ditlog / condlog / ditmodes / lm5 alone")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
