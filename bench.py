"""Training-throughput benchmark: the f32 decoder-LM training step on B200.

Workload: the medium decoder LM (12 layers, d_model 1024, 16 heads, FFN 4096,
vocab 32768, seq 1024) at a fixed global batch of 64 sequences (65,536
tokens per step), f32-grade contractions (split-f16 binary16 hi/lo operand
pairs by default, 3xTF32 with --contractions tf32x3), f32 master weights and
AdamW;
synthetic uniform tokens from a seed, N(0, 0.02) weights.  One step is
forward + backward (+ NCCL gradient allreduce across ranks) + AdamW.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

N > 1 runs under torchrun (one process per GPU): each rank takes 64/N
sequences (strong scaling), gradients are summed with NCCL.  Rank 0 prints one
JSON line.  `value` times device-resident token batches with CUDA events on
the model's stream (max over ranks); `e2e` times the public host API
(et_b200_lm_step_v1: host ids/targets copied in, loss copied out) the same
way.  `--impl reference` times the reference's own CPU implementation of the
same step on this host's cores by sampled per-operation timing.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "train tokens/s (fwd+bwd+opt, f32) at 1/2/4/8 B200"
UNIT = "tokens/s"
WORKLOAD = "medium decoder LM L12 d1024 H16 F4096 V32768 T1024, global batch 64"
GLOBAL_BATCH = 64
SHAPE = dict(layers=12, d_model=1024, heads=16, ffn=4096, vocabulary=32768, seq_len=1024)


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text())
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
            "fallback": True}


class ClockSampler:
    """nvidia-smi clock/throttle samples every 200 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None
        self.path = Path(tempfile.gettempdir()) / f"et_b200_clocks_{gpu}_{os.getpid()}.csv"

    def __enter__(self):
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.fh, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.fh.close()

    def summary(self) -> dict:
        try:
            rows = [r.split(",") for r in self.path.read_text().strip().splitlines()]
        except Exception:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        rows = [[c.strip() for c in r] for r in rows if len(r) >= 9]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(rows)}


def dist_env():
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


# DRAM bytes per algorithmic GFLOP of the pair GEMM, measured by ncu
# (dram__bytes_read.sum + dram__bytes_write.sum) on the profiling case's
# FFN-up backward launches: split-f16 dX 84.0 + 5.2 MB and dW 84.0 + 3.5 MB
# for 34.36 GFLOP each; 3xTF32 (FFN-up and FFN-down forward) 109.7 MB and
# 171.7 MB.
GEMM_DRAM_MB_PER_GFLOP = {"f16x3": (84.0 + 5.2 + 84.0 + 3.5) / (2 * 34.36),
                          "tf32x3": (109.7 + 171.7) / (2 * 34.36)}


def roofline_entry(gemm: dict, gemm_tflops: float, peak_t: float, peaks: dict,
                   clocks: dict, f16: bool) -> dict:
    """The dominant kernel class (every linear GEMM of the timed steps).

    achieved = algorithmic 2*M*N*K FLOP / CUDA-event time; peak = the measured
    bf16 sustained rate.  Both f32-grade modes issue three tensor-core MMAs per
    algorithmic FMA: split-f16 (binary16 hi/lo pairs, kind::f16) at the
    bf16/f16 rate, whose ceiling is 8,192 FLOP/clk/SM at the clock the SMs ran,
    and 3xTF32 (kind::tf32) at half of it (4,096).
    """
    per_launch_flop = gemm["flop"] / max(gemm["launches"], 1)
    sm_mhz = clocks.get("sm_mhz")
    per_clk = 8192 if f16 else 4096
    ceiling = per_clk * 148 * sm_mhz * 1e6 / 1e12 if sm_mhz else None
    kind = "kind::f16, split-f16 pairs" if f16 else "kind::tf32"
    return {
        "bound": "tensor", "kernel": f"linear GEMM (tcgen05.mma.cta_group::2 {kind}, 3 passes)",
        "achieved": round(gemm_tflops, 2), "peak": peak_t, "unit": "TFLOP/s",
        "frac": round(gemm_tflops / peak_t, 4) if peak_t else None,
        "peak_source": "MEASURED_PEAKS.json bf16_tflops_sustained (of measured)"
        if not peaks.get("fallback") else "fallback",
        "tensor_mma_per_algorithmic_flop": 3,
        "tensor_issue_tflops": round(3 * gemm_tflops, 1),
        "frac_tensor_issue_of_measured_bf16": round(3 * gemm_tflops / peak_t, 4) if peak_t else None,
        "mma_ceiling_at_median_clock_tflops": round(ceiling, 1) if ceiling else None,
        "frac_of_mma_ceiling_at_clock": round(3 * gemm_tflops / ceiling, 4) if ceiling else None,
        "flop_per_launch": per_launch_flop,
        "avg_launch_ms": gemm["ms"] / max(gemm["launches"], 1),
        "traffic": round(per_launch_flop / 1e9 *
                         GEMM_DRAM_MB_PER_GFLOP["f16x3" if f16 else "tf32x3"] * 1e6),
        "traffic_unit": "bytes per launch",
        "traffic_source": "ncu DRAM bytes of the profiling-case GEMM launches per algorithmic "
                          "FLOP, scaled to the average launch",
    }


# ----------------------------------------------------------------- B200 arm

def time_steps(etb, shape, precision, global_tokens, dev, stream_of, steps, warmup, rank, world,
               barrier) -> float:
    """ms per step (max over ranks) of a fresh model in `precision` over the
    device-resident batches `dev`."""
    import torch
    import torch.distributed as dist

    model = etb.LanguageModel(shape, precision=precision, global_tokens=global_tokens)
    model.init(20261201)
    if world > 1:
        uid = [etb.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        model.enable_data_parallel(uid[0], rank, world)
    stream = torch.cuda.ExternalStream(model.stream())
    loss = torch.zeros(1, device="cuda")
    for i in range(warmup):
        model.step_device(dev[i % len(dev)][0].data_ptr(), dev[i % len(dev)][1].data_ptr(),
                          loss.data_ptr())
    barrier()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for i in range(steps):
        ids, tg = dev[i % len(dev)]
        model.step_device(ids.data_ptr(), tg.data_ptr(), loss.data_ptr())
    stop.record(stream)
    barrier()
    ms = start.elapsed_time(stop) / steps
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = t.item()
    model.close()
    return ms


def run_b200(args) -> None:
    import torch
    import torch.distributed as dist

    import eshkol_transformer_b200 as etb

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        # NCCL's communicator-init log (one "comm ... rank r nRanks n" line per
        # rank and communicator, on stderr) shows how many ranks joined
        os.environ.setdefault("NCCL_DEBUG", "INFO")
        os.environ.setdefault("NCCL_DEBUG_SUBSYS", "INIT")
        os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")
        dist.init_process_group("nccl", init_method="env://",
                                timeout=__import__("datetime").timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    if GLOBAL_BATCH % world:
        raise SystemExit("global batch 64 must divide across ranks")
    batch = GLOBAL_BATCH // world
    shape = etb.ModelShape(batch=batch, **SHAPE)
    tokens_rank = batch * shape.seq_len
    global_tokens = GLOBAL_BATCH * shape.seq_len
    f16 = args.contractions == "f16x3"
    precision = etb.PRECISION_F16X3 if f16 else etb.PRECISION_TF32X3
    model = etb.LanguageModel(shape, precision=precision, global_tokens=global_tokens)
    model.init(20261201)
    if world > 1:
        uid = [etb.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        model.enable_data_parallel(uid[0], rank, world)
    stream = torch.cuda.ExternalStream(model.stream())
    # distinct token batches per step, resident in HBM before timing
    nbuf = 4
    batches = [etb.synthetic_batch(1000 + 97 * i + rank, batch, shape.seq_len, shape.vocabulary)
               for i in range(nbuf)]
    dev = [(torch.from_numpy(a).cuda(), torch.from_numpy(b).cuda()) for a, b in batches]
    loss = torch.zeros(1, device="cuda")

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    for i in range(args.warmup):
        model.step_device(dev[i % nbuf][0].data_ptr(), dev[i % nbuf][1].data_ptr(), loss.data_ptr())
    barrier()
    model.profile(True)
    launches0 = etb.launch_count()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        barrier()
        start.record(stream)
        for i in range(args.steps):
            ids, tg = dev[i % nbuf]
            model.step_device(ids.data_ptr(), tg.data_ptr(), loss.data_ptr())
        stop.record(stream)
        barrier()
    launches = etb.launch_count() - launches0
    ms = start.elapsed_time(stop)
    prof = model.profile_read()
    model.profile(False)
    ms_max = ms
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_max = t.item()
    value = global_tokens * args.steps / (ms_max / 1e3)

    # e2e through the public host API: host ids/targets in, loss out
    host = [(np.ascontiguousarray(a), np.ascontiguousarray(b)) for a, b in batches]
    barrier()
    e2e_start = torch.cuda.Event(enable_timing=True)
    e2e_stop = torch.cuda.Event(enable_timing=True)
    e2e_steps = max(1, min(args.steps, 5))
    e2e_start.record(stream)
    t0 = time.perf_counter()
    losses = []
    for i in range(e2e_steps):
        a, b = host[i % nbuf]
        losses.append(model.step(a, b))
    e2e_stop.record(stream)
    barrier()
    wall = time.perf_counter() - t0
    e2e_ms = max(e2e_start.elapsed_time(e2e_stop), wall * 1e3)
    if world > 1:
        t = torch.tensor([e2e_ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = t.item()
    e2e_value = global_tokens * e2e_steps / (e2e_ms / 1e3)

    model.close()
    # the config's named contraction mode (3xTF32) on the same box and ranks,
    # fewer steps: reported beside the headline, not as it
    tf32x3 = None
    if f16 and not args.no_tf32x3:
        tf32x3 = time_steps(etb, shape, etb.PRECISION_TF32X3, global_tokens, dev, stream_of=None,
                            steps=max(2, min(args.steps, 3)), warmup=2, rank=rank, world=world,
                            barrier=barrier)

    peaks = measured_peaks()
    gemm = prof["gemm"]
    gemm_tflops = gemm["flop"] / (gemm["ms"] / 1e3) / 1e12 if gemm["ms"] else 0.0
    peak_t = peaks.get("bf16_tflops_sustained", 1400.0)
    attn_b = prof["attention_backward"]
    attn_tflops = attn_b["flop"] / (attn_b["ms"] / 1e3) / 1e12 if attn_b["ms"] else 0.0
    total_prof_ms = sum(v["ms"] for v in prof.values())
    hbm = peaks.get("hbm_gbs", 6650.0)

    def hbm_entry(name):
        c = prof[name]
        if not c["ms"]:
            return None
        gbs = c["bytes"] / (c["ms"] / 1e3) / 1e9
        return {"achieved_gbs": round(gbs, 1), "frac": round(gbs / hbm, 4),
                "bytes_per_step": c["bytes"] / args.steps,
                "ms_per_step": round(c["ms"] / args.steps, 3)}
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic uniform tokens (seeded), N(0,0.02) random-init weights",
        "config": {"workload": WORKLOAD, "global_batch": GLOBAL_BATCH,
                   "seq_len": shape.seq_len, "tokens_per_step": global_tokens,
                   "contractions": ("split-f16 tcgen05 (binary16 hi/lo pairs with per-tensor "
                                    "power-of-two scales, 3 products; f32-grade)" if f16
                                    else "3xTF32 tcgen05 (f32-grade)"),
                   "parallelism": f"dp{world}",
                   "l2": "activations (GBs per step) exceed the 126 MB L2; no flush needed"},
        "gpu_launches": launches,
        "roofline": roofline_entry(gemm, gemm_tflops, peak_t, peaks, clocks.summary(), f16),
        "attention_backward": {"achieved_tflops": round(attn_tflops, 2),
                               "ms_per_step": round(attn_b["ms"] / args.steps, 3)},
        "hbm_frac": {"peak_gbs": hbm, "peak_source": "MEASURED_PEAKS.json hbm_gbs (of measured)"
                     if not peaks.get("fallback") else "fallback",
                     "cross_entropy": hbm_entry("cross_entropy"),
                     "adamw": hbm_entry("adamw"), "adamw_check": hbm_entry("adamw_check")},
        "profile_ms_per_step": {k: round(v["ms"] / args.steps, 3) for k, v in prof.items()},
        "profile_share": {k: round(v["ms"] / total_prof_ms, 4) for k, v in prof.items()}
        if total_prof_ms else {},
        "e2e": {"value": round(e2e_value, 1), "unit": UNIT,
                "h2d_bytes_per_step": 2 * 8 * tokens_rank, "d2h_bytes_per_step": 4,
                "steps": e2e_steps, "final_loss": losses[-1]},
        "clocks": clocks.summary(),
    }
    if tf32x3 is not None:
        line["config"]["tf32x3_ms_per_step"] = round(tf32x3, 3)
        line["config"]["tf32x3_tokens_per_s"] = round(global_tokens / (tf32x3 / 1e3), 1)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(kind="port", budget_s=args.cpu_budget)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# ----------------------------------------------------------------- CPU arm

def cpu_baseline(kind: str = "port", budget_s: float = 20.0) -> dict:
    """The CPU implementation of one training step of the workload, timed per
    operation on a token sample and scaled to tokens/s by the step's
    operation counts (a full step takes hours on the CPU).

    kind "port": the oracle restatement (OpenMP over the host cores).
    kind "reference": the reference's own C code only (oracle/_ref), serial
    as the reference is -- see reference_step_sample.
    """
    if kind == "reference":
        return reference_step_sample()
    from oracle import oracle as orc

    threads = os.cpu_count() or 1
    L, d, H, F, V, T = (SHAPE[k] for k in ("layers", "d_model", "heads", "ffn", "vocabulary",
                                         "seq_len"))
    Dh = d // H
    S = 64  # token sample for the contractions
    rows = S
    t = {}

    def timed(name, fn, repeat=1):
        t0 = time.perf_counter()
        for _ in range(repeat):
            fn()
        t[name] = (time.perf_counter() - t0) / repeat

    x = orc.fill_normal(1, 1, rows * F)
    dy = orc.fill_normal(1, 2, rows * F)

    def linear_pair(din, dout):
        xi = x[:rows * din].reshape(1, rows, din)
        w = orc.fill_normal(1, 3, dout * din, 0, 0.02).reshape(dout, din)
        b = np.zeros(dout, np.float32)
        g = dy[:rows * dout].reshape(1, rows, dout)
        return lambda: (orc.linear_forward(xi, w, b), orc.linear_backward(xi, w, g))

    timed("qkv", linear_pair(d, 3 * d))
    timed("out", linear_pair(d, d))
    timed("up", linear_pair(d, F))
    timed("down", linear_pair(F, d))
    # tied head at a smaller sample (largest contraction), scaled to S
    Sh = max(4, S // 4)
    xh = x[:Sh * d].reshape(1, Sh, d)
    wh = orc.fill_normal(1, 4, V * d, 0, 0.02).reshape(V, d)
    gh = orc.fill_normal(1, 5, Sh * V).reshape(1, Sh, V)
    t0 = time.perf_counter()
    orc.linear_forward(xh, wh)
    orc.linear_backward(xh, wh, gh, with_bias=False)
    head = (time.perf_counter() - t0) * S / Sh
    # attention at the full sequence length for one (sequence, head), scaled
    shp = (1, 1, 1, T, T, Dh)
    q = orc.fill_normal(2, 1, T * Dh).reshape(1, 1, T, Dh)
    pos = np.arange(T, dtype=np.int64).reshape(1, T)
    mask = np.ones((1, T, T), np.uint8)
    t0 = time.perf_counter()
    orc.attention_forward(shp, q, q, q, pos, pos, mask)
    orc.attention_backward(shp, q, q, q, pos, pos, mask, q)
    att_per_token = (time.perf_counter() - t0) * H / T
    # LN / GELU / CE / AdamW per element, sampled
    xl = orc.fill_normal(3, 1, rows * d).reshape(1, rows, d)
    gam = np.ones(d, np.float32)
    t0 = time.perf_counter()
    orc.layer_norm_forward(xl, gam, gam, 1e-5)
    orc.layer_norm_backward(xl, gam, 1e-5, xl)
    ln = time.perf_counter() - t0
    u = x[:rows * F]
    t0 = time.perf_counter()
    orc.gelu_forward(u)
    orc.gelu_backward(u, u)
    gelu = time.perf_counter() - t0
    lg = orc.fill_normal(3, 2, rows * V).reshape(1, rows, V)
    tg = orc.fill_tokens(3, 3, rows, V).reshape(1, rows)
    t0 = time.perf_counter()
    orc.ce_forward(lg, tg)
    orc.ce_backward(lg, tg, np.ones((1, rows), np.float32))
    ce = time.perf_counter() - t0
    n_params = 12 * (4 * d * d + 2 * d * F) + V * d
    pa = orc.fill_normal(4, 1, 1 << 20)
    m = np.zeros_like(pa)
    v = np.zeros_like(pa)
    t0 = time.perf_counter()
    orc.adamw_step(pa, pa, m, v, orc.adamw_options(1e-3, 0.9, 0.999, 1e-8, 0.01), 1)
    adam = (time.perf_counter() - t0) * n_params / (1 << 20)
    per_token = ((t["qkv"] + t["out"] + t["up"] + t["down"] + 2 * ln + gelu) * L + head + ln
                 + ce) / S + att_per_token * L + adam / (GLOBAL_BATCH * T)
    return {"value": round(1.0 / per_token, 3), "unit": UNIT, "cores": threads, "kind": "port",
            "sample": (f"per-op timing on {S} tokens of the {WORKLOAD} step (tied head on {Sh} "
                       f"tokens, attention on one (sequence, head) at T={T}, AdamW on 2^20 "
                       f"parameters) scaled by the step's operation counts")}


_REF_O2_READY = False


def reference_step_sample(S: int = 16, Ta: int = 256) -> dict:
    """The reference's own C code (compiled unmodified into oracle/_ref) timed
    per operation on one host core, then scaled to one step of the workload.

    * the N2 runners: QKV / output / FFN linears and the tied head (forward
      and backward), LayerNorm forward/backward (3 per layer-step: 2 per
      layer + the final one), GELU forward/backward, embedding
      forward/backward -- on S tokens;
    * A2 through its provider's invoke_call: rope.forward on Q and K,
      causal-attention.forward, causal-attention.backward, rope.backward on
      dQ and dK, at [1 sequence, 2 heads, T=Ta] (validate_call, whose cost is
      O(T^3 Dh^2), is not part of a step and is not timed), scaled by
      (T/Ta)^2 and heads/2;
    * L2 through its provider's invoke_call: indexed-cross-entropy forward
      and backward over S rows of V logits;
    * O2 through its API: an I2 gradient-plan accumulation, the AdamW step and
      zero_grad over one 2^20-element parameter, scaled to the model's count.
    The step time is extrapolated from these samples ("extrapolated": true).
    """
    import ctypes as C

    from eshkol_transformer_b200 import k1
    from oracle import oracle as orc

    global _REF_O2_READY
    ref = orc.ref()
    if ref is None:
        raise SystemExit("oracle/_ref/libref.so is not built (the reference's C sources)")
    L, d, H, F, V, T = (SHAPE[k] for k in ("layers", "d_model", "heads", "ffn", "vocabulary",
                                         "seq_len"))
    Dh = d // H
    p = lambda a: a.ctypes.data_as(C.c_void_p)
    sz = C.c_size_t
    secs = {}

    def timed(name, fn):
        t0 = time.perf_counter()
        rc = fn()
        secs[name] = time.perf_counter() - t0
        return rc

    x = orc.fill_normal(1, 1, S * F)
    dy = orc.fill_normal(1, 2, S * F)

    def linear(name, din, dout, bias=True, tokens=S):
        xi = np.ascontiguousarray(x[:tokens * din])
        w = orc.fill_normal(1, 3, dout * din, 0, 0.02)
        b = np.zeros(dout, np.float32)
        g = np.ascontiguousarray(dy[:tokens * dout]) if tokens * dout <= dy.size else \
            orc.fill_normal(1, 5, tokens * dout)
        y = np.empty(tokens * dout, np.float32)
        dx, dw, db = np.empty_like(xi), np.empty_like(w), np.empty(dout, np.float32)
        timed(name, lambda: (
            ref.ref_n2_linear_forward(sz(1), sz(tokens), sz(din), sz(dout), p(xi), p(w),
                                      p(b) if bias else None, p(y)),
            ref.ref_n2_linear_backward(sz(1), sz(tokens), sz(din), sz(dout), p(xi), p(w), p(g),
                                       1 if bias else 0, p(dx), p(dw),
                                       p(db) if bias else None)))

    linear("qkv", d, 3 * d)
    linear("out", d, d)
    linear("up", d, F)
    linear("down", F, d)
    Sh = max(2, S // 4)  # the tied head is the largest contraction
    linear("head", d, V, bias=False, tokens=Sh)
    secs["head"] *= S / Sh
    xl = np.ascontiguousarray(x[:S * d])
    gam, bet = np.ones(d, np.float32), np.zeros(d, np.float32)
    yl, dxl = np.empty_like(xl), np.empty_like(xl)
    dgam, dbet = np.empty(d, np.float32), np.empty(d, np.float32)
    eps = C.c_float(1e-5)
    timed("layer_norm", lambda: (
        ref.ref_n2_layer_norm_forward(sz(1), sz(S), sz(d), p(xl), p(gam), p(bet), eps, p(yl)),
        ref.ref_n2_layer_norm_backward(sz(1), sz(S), sz(d), p(xl), p(gam), eps, p(xl), p(dxl),
                                       p(dgam), p(dbet))))
    u = np.ascontiguousarray(x[:S * F])
    gu, du = np.empty_like(u), np.empty_like(u)
    timed("gelu", lambda: (ref.ref_n2_gelu(sz(1), sz(S), sz(F), p(u), None, p(gu)),
                           ref.ref_n2_gelu(sz(1), sz(S), sz(F), p(u), p(u), p(du))))
    ids = orc.fill_tokens(3, 1, S, V)
    emb = orc.fill_normal(3, 4, V * d, 0, 0.02)
    ye, dwe = np.empty(S * d, np.float32), np.empty(V * d, np.float32)
    timed("embedding", lambda: (
        ref.ref_n2_embedding_forward(sz(1), sz(S), sz(V), sz(d), p(ids), p(emb), p(ye)),
        ref.ref_n2_embedding_backward(sz(1), sz(S), sz(V), sz(d), p(ids), p(xl), p(dwe))))
    # A2: rope + attention forward/backward through invoke_call
    a2 = k1.provider(ref, "et_a2_kernel_provider_v1")
    Ha = 2
    q, kk, vv, go = (orc.fill_normal(2, i, Ha * Ta * Dh).reshape(1, Ha, Ta, Dh)
                     for i in range(4))
    pos = np.arange(Ta, dtype=np.int64).reshape(1, Ta)
    keep = np.ones((1, Ta, Ta), np.uint8)
    inv = np.array([np.float32(1.0 / 10000.0 ** (2 * i / Dh)) for i in range(Dh // 2)],
                   np.float32)
    rshape = (1, Ha, Ta, Dh)
    qr, kr, o = (np.empty(rshape, np.float32) for _ in range(3))
    dq, dk, dv, dqr, dkr = (np.empty(rshape, np.float32) for _ in range(5))
    ashape = (1, Ha, Ha, Ta, Ta, Dh)
    calls = [
        k1.KernelCall("kernel.rope", "rope.forward", rshape, [q, pos, inv], [qr]),
        k1.KernelCall("kernel.rope", "rope.forward", rshape, [kk, pos, inv], [kr]),
        k1.KernelCall("kernel.causal-attention", "causal-attention.forward", ashape,
                      [qr, kr, vv, pos, pos, keep], [o]),
        k1.KernelCall("kernel.causal-attention", "causal-attention.backward", ashape,
                      [qr, kr, vv, pos, pos, keep, go], [dq, dk, dv]),
        k1.KernelCall("kernel.rope", "rope.backward", rshape, [dq, pos, inv], [dqr]),
        k1.KernelCall("kernel.rope", "rope.backward", rshape, [dk, pos, inv], [dkr]),
    ]
    timed("attention", lambda: [a2.invoke_call(C.pointer(c.call)) for c in calls])
    att_per_token = secs["attention"] * (T / Ta) ** 2 * (H / Ha) / T
    # L2: cross-entropy forward + backward through invoke_call
    l2 = k1.provider(ref, "et_l2_indexed_cross_entropy_provider_v1")
    lg = orc.fill_normal(3, 2, S * V).reshape(1, S, V)
    tg = orc.fill_tokens(3, 3, S, V).reshape(1, S)
    up = np.full((1, S), 1.0 / (GLOBAL_BATCH * T), np.float32)
    loss, grad = np.empty((1, S), np.float32), np.empty((1, S, V), np.float32)
    ce_calls = [k1.KernelCall("kernel.indexed-cross-entropy", "indexed-cross-entropy.forward",
                              (1, S, V), [lg, tg], [loss]),
                k1.KernelCall("kernel.indexed-cross-entropy", "indexed-cross-entropy.backward",
                              (1, S, V), [lg, tg, up], [grad])]
    timed("cross_entropy", lambda: [l2.invoke_call(C.pointer(c.call)) for c in ce_calls])
    # O2 through its API (one optimizer per process: the harness keeps it)
    n_o2 = 1 << 20
    if not _REF_O2_READY:
        init = orc.fill_normal(4, 1, n_o2).view(np.uint32)
        bits = [orc.bits(v) for v in (1e-3, 0.9, 0.999, 1e-8, 0.01)]
        if ref.ref_o2_create(p(init), sz(n_o2), *[C.c_uint32(b) for b in bits]) != 0:
            raise SystemExit("the reference's O2 optimizer could not be built")
        _REF_O2_READY = True
    grad_bits = orc.fill_normal(4, 2, n_o2, 0.0, 1e-3).view(np.uint32)
    rc = timed("adamw", lambda: (ref.ref_o2_accumulate(p(grad_bits), C.c_uint32(0x3f800000)),
                                 ref.ref_o2_step(), ref.ref_o2_zero_grad()))
    if any(rc):
        raise SystemExit(f"the reference's O2 step failed: {rc}")
    n_params = L * (4 * d * d + 2 * d * F) + V * d
    tokens = GLOBAL_BATCH * T
    per_token = ((secs["qkv"] + secs["out"] + secs["up"] + secs["down"]
                  + 2 * secs["layer_norm"] + secs["gelu"]) * L
                 + secs["head"] + secs["layer_norm"] + secs["cross_entropy"]
                 + secs["embedding"]) / S + att_per_token * L \
        + secs["adamw"] * n_params / n_o2 / tokens
    step_s = per_token * tokens
    return {"value": round(1.0 / per_token, 4), "unit": UNIT, "cores": 1, "kind": "reference",
            "extrapolated": True, "step_s": round(step_s, 1),
            "per_op_sample_s": {k: round(v, 4) for k, v in secs.items()},
            "sample": (f"the reference's own C code on one core: N2 linears, LayerNorm, GELU and "
                       f"embedding on {S} tokens (tied head on {Sh}), A2 rope + attention "
                       f"forward/backward via invoke_call at 1 sequence x {Ha} heads x T={Ta}, "
                       f"L2 cross-entropy via invoke_call on {S} rows, O2 accumulate + step + "
                       f"zero_grad on 2^20 parameters; scaled to the {WORKLOAD} step by its "
                       f"operation counts (attention by (T/{Ta})^2)")}


def run_reference(args) -> None:
    rank, world, _ = dist_env()
    if rank != 0:
        return
    t0 = time.perf_counter()
    for _ in range(args.warmup if args.warmup < 2 else 1):
        reference_step_sample()
    samples = [reference_step_sample() for _ in range(max(1, args.steps))]
    value = statistics.median(s["value"] for s in samples)
    base = samples[0]
    ms_per_step = GLOBAL_BATCH * SHAPE["seq_len"] / value * 1e3
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_per_step, 1),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded)",
        "config": {"workload": WORKLOAD, "global_batch": GLOBAL_BATCH,
                   "seq_len": SHAPE["seq_len"], "parallelism": "host CPU, 1 core (serial C)"},
        "extrapolated": True,
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": base["cores"],
                         "kind": base["kind"], "sample": base["sample"], "extrapolated": True},
        "per_op_sample_s": base["per_op_sample_s"],
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "wall_s": round(time.perf_counter() - t0, 1)}), flush=True)


# ----------------------------------------------------------------- attention sweep

SWEEP = dict(batch=4, heads=16, head_dims=(64, 128), seq_lens=(512, 1024, 2048, 4096, 8192, 16384))


def contraction_label(pairs16: bool, single: bool) -> str:
    """The attention contraction scheme of a sweep shape: binary16 operands
    (head_dim 128, head_dim 64 from 768^2 or on request) or TF32, three
    products of operand pairs (f32-grade) or one (TF32 mode)."""
    if single:
        return ("binary16 with per-tensor scales (kind::f16, 1 product)" if pairs16
                else "TF32 (kind::tf32, 1 product)")
    return "binary16 pairs (kind::f16)" if pairs16 else "3xTF32 pairs (kind::tf32)"


def attention_sweep(args) -> None:
    """Causal attention with RoPE, forward and backward, over the sweep's
    shapes (batch 4, 16 heads, head_dim 64 / 128, T = 512 ... 16384, seeded
    N(0, 1) Q/K/V/dO) through et_b200_attention_*_v1; one JSON line per
    shape.  Algorithmic FLOP: forward 2 B H T^2 Dh (the causal half of two
    GEMMs), backward 4 B H T^2 Dh (four); bytes: each tensor read or written
    once (forward Q, K, V, O; backward Q, K, V, O, dO, dQ, dK, dV).  The
    reference's A2 provider (oracle/_ref, one core, invoke_call only) is
    timed at T <= 2048 on one sequence and two heads and scaled by B H / 2;
    beyond 2048 its time is extrapolated by (T / 2048)^2 and marked."""
    import torch

    import eshkol_transformer_b200 as etb

    torch.cuda.set_device(0)
    peaks = measured_peaks()
    bf16 = peaks.get("bf16_tflops", 1590.0)
    hbm = peaks.get("hbm_gbs", 6650.0)
    ref_cache = {}
    contraction = {"default": etb.ATTENTION_DEFAULT, "pairs16": etb.ATTENTION_BWD_PAIRS16,
                   "tf32": etb.ATTENTION_TF32}[args.attention_contraction]
    head_dims = args.sweep_head_dims or SWEEP["head_dims"]
    seq_lens = args.sweep_seq_lens or SWEEP["seq_lens"]
    for Dh in head_dims:
        for T in seq_lens:
            B, H = SWEEP["batch"], SWEEP["heads"]
            g = torch.Generator(device="cuda").manual_seed(T * 1000 + Dh)
            q, k, v, do = (torch.randn(B, H, T, Dh, device="cuda", generator=g)
                           for _ in range(4))
            pos = torch.arange(T, dtype=torch.int64, device="cuda").repeat(B, 1).contiguous()
            c, s_ = etb.rope_tables(T, Dh)
            cos, sin = torch.from_numpy(c).cuda(), torch.from_numpy(s_).cuda()
            att = etb.Attention(B, H, H, T, T, Dh, pos, pos, None, cos, sin,
                                contraction=contraction)
            o = torch.empty_like(q)
            m = torch.empty(B, H, T, device="cuda")
            l = torch.empty(B, H, T, device="cuda")
            dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
            iters = max(2, min(20, int(2e12 / (4.0 * B * H * T * T * Dh))))
            for _ in range(2):
                att.forward(q, k, v, o, m, l)
                att.backward(q, k, v, o, do, m, l, dq, dk, dv)
            torch.cuda.synchronize()
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
            with ClockSampler(0) as clocks:
                ev[0].record()
                for _ in range(iters):
                    att.forward(q, k, v, o, m, l)
                ev[1].record()
                for _ in range(iters):
                    att.backward(q, k, v, o, do, m, l, dq, dk, dv)
                ev[2].record()
                torch.cuda.synchronize()
            fwd_ms = ev[0].elapsed_time(ev[1]) / iters
            bwd_ms = ev[1].elapsed_time(ev[2]) / iters
            f_flop = 2.0 * B * H * T * T * Dh
            b_flop = 4.0 * B * H * T * T * Dh
            t_bytes = 4.0 * B * H * T * Dh
            pairs16 = Dh == 128 or (Dh == 64 and (contraction == etb.ATTENTION_BWD_PAIRS16
                                                  or T * T >= 768 * 768))
            single = contraction == etb.ATTENTION_TF32
            line = {
                "metric": "attn fwd/bwd % roofline", "workload": "causal attention + RoPE",
                "batch": B, "heads": H, "seq_len": T, "head_dim": Dh,
                "dtype": "tf32" if single else "f32",
                # the forward takes binary16 operands wherever the backward does
                "contractions": {
                    "forward": contraction_label(pairs16, single),
                    "backward": contraction_label(pairs16, single)},
                "fwd_ms": round(fwd_ms, 4), "bwd_ms": round(bwd_ms, 4),
                "fwd_tflops": round(f_flop / fwd_ms / 1e9, 2),
                "bwd_tflops": round(b_flop / bwd_ms / 1e9, 2),
                "fwd_frac_of_measured_bf16": round(f_flop / fwd_ms / 1e9 / bf16, 4),
                "bwd_frac_of_measured_bf16": round(b_flop / bwd_ms / 1e9 / bf16, 4),
                "fwd_frac_of_tf32_rate": round(2 * f_flop / fwd_ms / 1e9 / bf16, 4),
                "bwd_frac_of_tf32_rate": round(2 * b_flop / bwd_ms / 1e9 / bf16, 4),
                "fwd_gbs": round(4 * t_bytes / fwd_ms / 1e6, 1),
                "bwd_gbs": round(8 * t_bytes / bwd_ms / 1e6, 1),
                "hbm_frac_bwd": round(8 * t_bytes / bwd_ms / 1e6 / hbm, 4),
                "iters": iters, "clocks": clocks.summary(),
                "tensor_core_backward": Dh in (32, 64, 128),
            }
            if not args.no_cpu_baseline:
                line["reference_cpu"] = reference_attention_seconds(B, H, T, Dh, ref_cache)
            print(json.dumps(line), flush=True)
            del q, k, v, do, o, dq, dk, dv, att
            torch.cuda.empty_cache()


def reference_attention_seconds(B, H, T, Dh, cache) -> dict:
    """The reference's A2 provider (invoke_call; rope fwd on Q, K, attention
    forward and backward, rope bwd on dQ, dK) on one core for one sequence
    and two heads at min(T, 2048), scaled by B H / 2 and, above 2048, by
    (T / 2048)^2 (marked extrapolated)."""
    import ctypes as C

    from eshkol_transformer_b200 import k1
    from oracle import oracle as orc

    ref = orc.ref()
    if ref is None:
        return {"unavailable": "oracle/_ref/libref.so is not built"}
    Ta = min(T, 2048)
    if (Ta, Dh) not in cache:
        a2 = k1.provider(ref, "et_a2_kernel_provider_v1")
        Ha = 2
        q, kk, vv, go = (orc.fill_normal(6, i, Ha * Ta * Dh).reshape(1, Ha, Ta, Dh)
                         for i in range(4))
        pos = np.arange(Ta, dtype=np.int64).reshape(1, Ta)
        keep = np.ones((1, Ta, Ta), np.uint8)
        inv = np.array([np.float32(1.0 / 10000.0 ** (2 * i / Dh)) for i in range(Dh // 2)],
                       np.float32)
        rs = (1, Ha, Ta, Dh)
        qr, kr, o, dq, dk, dv, dqr, dkr = (np.empty(rs, np.float32) for _ in range(8))
        asz = (1, Ha, Ha, Ta, Ta, Dh)
        fwd = [k1.KernelCall("kernel.rope", "rope.forward", rs, [q, pos, inv], [qr]),
               k1.KernelCall("kernel.rope", "rope.forward", rs, [kk, pos, inv], [kr]),
               k1.KernelCall("kernel.causal-attention", "causal-attention.forward", asz,
                             [qr, kr, vv, pos, pos, keep], [o])]
        bwd = [k1.KernelCall("kernel.causal-attention", "causal-attention.backward", asz,
                             [qr, kr, vv, pos, pos, keep, go], [dq, dk, dv]),
               k1.KernelCall("kernel.rope", "rope.backward", rs, [dq, pos, inv], [dqr]),
               k1.KernelCall("kernel.rope", "rope.backward", rs, [dk, pos, inv], [dkr])]
        t0 = time.perf_counter()
        for c in fwd:
            a2.invoke_call(C.pointer(c.call))
        t1 = time.perf_counter()
        for c in bwd:
            a2.invoke_call(C.pointer(c.call))
        t2 = time.perf_counter()
        cache[(Ta, Dh)] = (t1 - t0, t2 - t1, Ha)
    f, b, Ha = cache[(Ta, Dh)]
    scale = B * H / Ha * (T / Ta) ** 2
    return {"fwd_s": round(f * scale, 3), "bwd_s": round(b * scale, 3), "cores": 1,
            "sample": f"1 sequence x {Ha} heads at T={Ta}, scaled by B*H/{Ha}"
                      + (f" and (T/{Ta})^2" if T > Ta else ""),
            "extrapolated": T > Ta}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--cpu-budget", type=float, default=20.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-tf32x3", action="store_true",
                    help="skip the 3xTF32 step time reported beside a split-f16 run")
    ap.add_argument("--contractions", default="f16x3", choices=["f16x3", "tf32x3"],
                    help="f32-grade contraction scheme of the linear GEMMs (split-f16 pairs or "
                         "3xTF32)")
    ap.add_argument("--profile-case", action="store_true",
                    help="small case of the same kernels for ncu captures (2 layers, global "
                         "batch 4 = 4096 tokens; a few GB on the device); not a bench value")
    ap.add_argument("--attention-sweep", action="store_true",
                    help="causal attention + RoPE fwd/bwd over B4 H16 Dh{64,128} T 512..16384 "
                         "(one JSON line per shape); not the default bench line")
    ap.add_argument("--attention-contraction", choices=("default", "pairs16", "tf32"),
                    default="default",
                    help="sweep's contraction mode: default (f32-grade: 3xTF32 pairs; binary16 "
                         "pairs for the head_dim-128 backward), pairs16 (binary16 pairs in the "
                         "backward at head_dim 64 too) or tf32 (one product of TF32-grade "
                         "operands, the sweep's TF32 mode)")
    ap.add_argument("--sweep-head-dims", type=int, nargs="*", default=None,
                    help="sweep only these head_dims")
    ap.add_argument("--sweep-seq-lens", type=int, nargs="*", default=None,
                    help="sweep only these sequence lengths")
    args = ap.parse_args()
    if args.attention_sweep:
        attention_sweep(args)
        return
    if args.profile_case:
        global GLOBAL_BATCH, WORKLOAD
        SHAPE["layers"] = 2
        GLOBAL_BATCH = 4
        WORKLOAD = "ncu profiling case: medium-LM widths, 2 layers, global batch 4"
        args.no_cpu_baseline = True
    if args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
