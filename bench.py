"""Benchmark of the SSM-scan hot path on B200 (one process per GPU).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--op scan|ssd|decode] [--config 1|2]

Default workload (the BASELINE metric): the Mamba-1 selective scan forward +
backward of BASELINE config 2 -- batch 16, d_inner 5120, seqlen 4096,
d_state 16, one group, bf16 u/delta/z/B/C, fp32 A/D/delta_bias,
delta_softplus=True, dy ~ N(0,1) -- sharded by batch over the N ranks
(global batch 16, 16/N rows per rank), followed by the NCCL all-reduce of the
shared-parameter gradients (dA, dD, d delta_bias) as one flat fp32 bucket.

One step = forward + backward of the whole batch shard (+ the all-reduce when
N > 1).  The timed region is bracketed by a barrier and a device synchronise
on both sides and timed with CUDA events on the launching stream; the reported
time is the max over ranks.  Inputs are generated on the host from the config's
seeded distributions (synthetic data), then moved to HBM; every input tensor is
larger than the 126 MB L2, so no flush is needed between steps.

Rank 0 prints one JSON line (see the keys below).  ``--impl reference`` times
the reference's CPU implementation of the same op (the oracle restatement of
``cv/path_scan.py:579-605`` + the ``scan.py:311-320`` epilogue, fp32, autograd
forward + backward) on the host cores, on a bounded sample of the same
workload, and prints the same line with ``"impl": "reference"``.
"""

from __future__ import annotations

import argparse
import json
import os
import pathlib
import statistics
import subprocess
import sys
import time

import torch

ROOT = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

CONFIGS = {
    1: dict(batch=8, dim=1536, length=2048, dstate=16, groups=1, seed=1001),
    2: dict(batch=16, dim=5120, length=4096, dstate=16, groups=1, seed=1002),
}
SSD_CONFIG = dict(batch=8, length=8192, nheads=80, headdim=64, dstate=128, ngroups=8, chunk=256,
                  seed=1003)
DECODE_CONFIG = dict(batch=256, nheads=80, headdim=64, dstate=128, ngroups=8, seed=1004)
# the reference's largest timed ss2d shape (measured/path_scan.json "b1_d96_56x56")
SS2D_CONFIG = dict(batch=1, channels=96, groups=1, dstate=16, height=56, width=56, seed=1005)
# the gated RMSNorm after the SSD scan at BASELINE config 3's layer shape
# (rows = B*L = 8*8192, d_inner = 80*64, groups of d_inner / ngroups)
GNORM_CONFIG = dict(rows=65536, features=5120, group_size=640, norm_before_gate=False, seed=1007)
# the convolution in front of the scan at BASELINE config 2's layer shape
CONV_CONFIG = dict(batch=16, channels=5120, length=4096, width=4, activation="silu", seed=1006)


def _peaks():
    try:
        return json.loads((ROOT / "MEASURED_PEAKS.json").read_text()), "measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def _dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


class Clocks:
    """nvidia-smi sampling (every 200 ms) during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for name, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(name)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------- scan op --

def _scan_inputs(cfg, batch_lo, batch_hi, device):
    from metal_kernelops_b200.workloads import selective_scan_inputs
    # generate the full config on the host (seeded), keep this rank's rows
    full = selective_scan_inputs(cfg["batch"], cfg["dim"], cfg["length"], cfg["dstate"],
                                 cfg["groups"], seed=cfg["seed"], act_dtype=torch.bfloat16) \
        if cfg["batch"] * cfg["dim"] * cfg["length"] <= 50_000_000 else None
    if full is None:
        full = _scan_inputs_rows(cfg, batch_lo, batch_hi)
    else:
        full = {k: (v[batch_lo:batch_hi] if k in ("u", "delta", "z", "dout", "B", "C") else v)
                for k, v in full.items()}
    return full


def _scan_inputs_rows(cfg, lo, hi):
    """Large configs: generate per batch row with a row-derived seed so every
    rank sees the same global tensor without materialising it whole."""
    from metal_kernelops_b200.workloads import selective_scan_rows
    return selective_scan_rows(cfg["dim"], cfg["length"], cfg["dstate"], cfg["groups"], cfg["seed"],
                               lo, hi, act_dtype=torch.bfloat16)


def _config(args):
    cfg = dict(CONFIGS[args.config])
    if args.shape:
        cfg["batch"], cfg["dim"], cfg["length"] = (int(v) for v in args.shape.split(","))
    return cfg


def _scan_config(args, cfg, world):
    """The workload description both arms print (so the driver sees one config)."""
    per = batch_slice_len(cfg["batch"], world)
    return {"workload": f"mamba1 selective scan fwd+bwd, BASELINE config {args.config}",
            "global_batch": cfg["batch"], "batch_per_gpu": per, "dim": cfg["dim"],
            "seq_len": cfg["length"], "dstate": cfg["dstate"], "groups": cfg["groups"],
            "parallelism": f"dp{world} (batch shard)", "l2": "inputs > L2 (126 MB), no flush"}


def batch_slice_len(batch, world):
    """Rows of rank 0 (the largest shard) when ``batch`` is split over ``world``."""
    return -(-batch // world)


def _scan_alg_bytes(b, d, l, n, g, s_a=2):
    fwd = 4 * s_a * b * d * l + 2 * s_a * b * g * n * l
    bwd = 7 * s_a * b * d * l + 4 * s_a * b * g * n * l
    return fwd, bwd


def run_scan(args, world, rank, device):
    import torch.distributed as dist
    import metal_kernelops_b200 as mk  # noqa: F401  (registers the ops)

    from metal_kernelops_b200.parallel import ParamGradBucket, batch_slice
    cfg = _config(args)
    rows = batch_slice(cfg["batch"], rank, world)
    lo, hi = rows.start, rows.stop
    per = hi - lo
    host = _scan_inputs(cfg, lo, hi, device)
    dev = {k: v.to(device) for k, v in host.items()}
    u, delta, A, B, C, D, z, bias, dout = (dev[k] for k in
                                           ("u", "delta", "A", "B", "C", "D", "z", "delta_bias", "dout"))
    ops = torch.ops.b200ssm
    bucket = ParamGradBucket([A.shape, D.shape, bias.shape], device)
    from metal_kernelops_b200.scan import checkpoint_numel
    saved_bytes = 4 * checkpoint_numel(per, cfg["dim"], cfg["length"], cfg["dstate"], 2, True, args.lean)

    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]

    def step(i=None):
        e = ev[i] if i is not None else None
        if e:
            e[0].record()
        y, ck = ops.selective_scan_fwd(u, delta, A, B, C, D, z, bias, True, True, args.lean)
        if e:
            e[1].record()
        du, dd, dA, dB, dC, dD, dz, db = ops.selective_scan_bwd(dout, u, delta, A, B, C, D, z, bias,
                                                                ck, True, args.lean)
        if e:
            e[2].record()
        if world > 1:
            bucket.reduce([dA, dD, db])
        if e:
            e[3].record()
        return y

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    # start the clock sampler before the barrier, so that no rank enters the
    # timed region while another is still setting it up
    clocks = Clocks(torch.cuda.current_device()) if rank == 0 else None
    if clocks:
        clocks.start()
        time.sleep(0.3)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for i in range(args.steps):
        step(i)
    t1.record()
    torch.cuda.synchronize()
    ck_info = clocks.stop() if clocks else None
    ms = t0.elapsed_time(t1)
    fwd_ms = sum(e[0].elapsed_time(e[1]) for e in ev) / args.steps
    bwd_ms = sum(e[1].elapsed_time(e[2]) for e in ev) / args.steps
    ar_ms = sum(e[2].elapsed_time(e[3]) for e in ev) / args.steps
    if world > 1:
        t = torch.tensor([ms, fwd_ms, bwd_ms, ar_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, fwd_ms, bwd_ms, ar_ms = t.tolist()
        dist.barrier()

    # end to end through the public API: pinned host inputs -> H2D, fwd+bwd via
    # autograd, D2H of the parameter gradients, every step.  Batch rows are
    # independent (the parameter gradients add), so each step runs as
    # micro-batches: a copy stream fills one of two device buffer sets from
    # pinned memory while the compute stream scans the other, and the step's
    # parameter gradients are summed, all-reduced and copied into that step's
    # own pinned host buffers.  The host reads them after the timed steps
    # rather than waiting for each, so the next step's input copies queue
    # behind the previous step's compute (the dependencies are device events).
    from metal_kernelops_b200 import scan as scan_mod
    scan_mod.set_lean_backward(args.lean)
    pinned = {k: v.pin_memory() for k, v in host.items()}
    e2e_steps = max(1, min(args.steps, 5))
    names = ("u", "delta", "A", "B", "C", "D", "z", "delta_bias")
    batched = ("u", "delta", "z", "dout", "B", "C")
    nmb = next(m for m in (4, 2, 1) if per % m == 0)
    rows_mb = per // nmb
    chunks = [{k: (pinned[k][j * rows_mb:(j + 1) * rows_mb] if k in batched else pinned[k]) for k in pinned}
              for j in range(nmb)]
    bufs = [{k: torch.empty(v.shape, dtype=v.dtype, device=device) for k, v in chunks[0].items()}
            for _ in range(2)]
    copy_stream = torch.cuda.Stream(device=device)
    copy_done = [torch.cuda.Event() for _ in range(2)]
    free = [torch.cuda.Event() for _ in range(2)]
    for ev in free:
        ev.record()

    results = [[torch.empty(t.shape, dtype=torch.float32).pin_memory() for t in (A, D, bias)]
               for _ in range(e2e_steps + 1)]

    def e2e_step(slot_base, out):
        acc = None
        for j in range(nmb):
            slot = (slot_base + j) % 2
            copy_stream.wait_event(free[slot])
            with torch.cuda.stream(copy_stream):
                for k, v in chunks[j].items():
                    bufs[slot][k].copy_(v, non_blocking=True)
                copy_done[slot].record(copy_stream)
            torch.cuda.current_stream().wait_event(copy_done[slot])
            d = bufs[slot]
            leaves = [d[k].detach().requires_grad_(True) for k in names]
            y = mk.selective_scan(*leaves[:5], D=leaves[5], z=leaves[6], delta_bias=leaves[7],
                                  delta_softplus=True)
            gr = torch.autograd.grad(y, leaves, d["dout"])
            part = [gr[2], gr[5], gr[7]]
            acc = part if acc is None else [a_ + p_ for a_, p_ in zip(acc, part)]
            free[slot].record()
        reduced = bucket.reduce(acc)
        for r, o in zip(reduced, out):
            o.copy_(r.reshape(o.shape), non_blocking=True)

    e2e_step(0, results[-1])
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    s0 = torch.cuda.Event(enable_timing=True)
    s1 = torch.cuda.Event(enable_timing=True)
    s0.record()
    for i in range(e2e_steps):
        e2e_step(i * nmb, results[i])
    s1.record()
    torch.cuda.synchronize()
    e2e_ms = s0.elapsed_time(s1) / e2e_steps
    # the host reads every step's result
    assert all(bool(torch.isfinite(o).all()) for res in results[:e2e_steps] for o in res)
    if world > 1:
        t = torch.tensor([e2e_ms], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = t.item()
    # whole-job bytes per step (every rank copies its own shard)
    h2d = world * sum(v.numel() * v.element_size() for v in host.values())
    d2h = world * (A.numel() + 2 * A.shape[0]) * 4

    if rank != 0:
        return None
    b, d, l, n, g = per, cfg["dim"], cfg["length"], cfg["dstate"], cfg["groups"]
    units = cfg["batch"] * d * l if world > 1 else b * d * l
    ms_step = ms / args.steps
    value = units / (ms_step / 1e3)
    peaks, peak_kind = _peaks()
    fwd_b, bwd_b = _scan_alg_bytes(b, d, l, n, g)
    bwd_gbs = bwd_b / (bwd_ms / 1e3) / 1e9
    fwd_gbs = fwd_b / (fwd_ms / 1e3) / 1e9
    step_gbs = (fwd_b + bwd_b) / ((fwd_ms + bwd_ms) / 1e3) / 1e9
    # The compute floor the kernels sit against: one MUFU ex2 per element-state
    # in the forward and two in the backward (the sub-block replay from the
    # saved states, and the adjoint, which recomputes the decays), at 16 per
    # clock per SM and the SM clock sampled under load.
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    mhz = (ck_info or {}).get("sm_mhz") or 1965.0
    ex2_per_s = sms * 16 * mhz * 1e6
    es = b * d * l * n
    fwd_floor, bwd_floor = es / ex2_per_s * 1e3, 2 * es / ex2_per_s * 1e3
    mufu = {"pipe": "XU (MUFU ex2), 16 per clock per SM", "sm_mhz": mhz,
            "ex2_per_element_state": {"fwd": 1, "bwd": 2},
            "fwd_floor_ms": fwd_floor, "bwd_floor_ms": bwd_floor,
            "fwd_frac": fwd_floor / fwd_ms, "bwd_frac": bwd_floor / bwd_ms}
    return {
        "metric": "selective-scan fwd+bwd B*L*D elems/s",
        "value": value,
        "unit": "elem/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_step,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16 storage, fp32 compute",
        "data": "synthetic (seeded, BASELINE config distributions)",
        "config": _scan_config(args, cfg, world),
        "breakdown_ms": {"fwd": fwd_ms, "bwd": bwd_ms, "allreduce": ar_ms},
        "saved_for_backward": {"mode": "lean (states every 16 steps)" if args.lean else
                               "states every 4 steps + scan output",
                               "bytes": saved_bytes},
        "roofline": {"bound": "hbm", "kernel": "selective_scan bwd (bwd2_tma_kernel + reduce)",
                     "achieved": bwd_gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": bwd_gbs / peaks["hbm_gbs"], "peak_source": peak_kind,
                     "traffic": _traffic("selective_scan_bwd"),
                     "alg_bytes_per_launch": bwd_b,
                     "fwd": {"achieved": fwd_gbs, "frac": fwd_gbs / peaks["hbm_gbs"]},
                     "fwd_bwd": {"achieved": step_gbs, "frac": step_gbs / peaks["hbm_gbs"]},
                     "mufu_floor": mufu},
        "e2e": {"value": units / (e2e_ms / 1e3), "unit": "elem/s", "ms_per_step": e2e_ms,
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "path": ("metal_kernelops_b200.selective_scan + autograd, pinned host buffers, "
                         f"{nmb} micro-batches per step, H2D on a second stream overlapping compute, "
                         "D2H of each step's gradients into pinned buffers read after the timed steps")},
        "gpu_launches": 3 * args.steps,
        "clocks": ck_info,
    }


def _traffic(kernel):
    """Per-launch DRAM bytes of the kernel from the committed ncu summary, if any."""
    f = ROOT / "profiles" / "traffic.txt"
    try:
        for line in f.read_text().splitlines():
            k, _, v = line.partition(":")
            if k.strip() == kernel:
                return float(v.split()[0])
    except Exception:
        pass
    return None


# ------------------------------------------------------------ SSD / decode --

def _timed(fn, steps, warmup, world, dist):
    """Run fn warmup + steps times; CUDA-event device time per step (max over ranks)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(steps):
        fn()
    t1.record()
    torch.cuda.synchronize()
    ms = t0.elapsed_time(t1) / steps
    if world > 1:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = t.item()
    return ms


def run_ssd(args, world, rank, device, shape=None):
    """Mamba-2 SSD chunk scan fwd+bwd, B8 L8192 H80 P64 N128
    G8 chunk 256, bf16 x/B/C, fp32 dt/A/D, dt_softplus; batch sharded, with the
    shared-parameter gradients (dA, dD, d dt_bias) summed over the ranks by one
    all-reduce of a flat fp32 bucket inside every timed step."""
    import torch.distributed as dist
    import metal_kernelops_b200  # noqa: F401
    from metal_kernelops_b200.parallel import ParamGradBucket, batch_slice
    from metal_kernelops_b200.workloads import ssd_inputs
    cfg = dict(SSD_CONFIG)
    if shape:   # batch,length[,nheads,headdim,dstate,ngroups]
        vals = [int(v) for v in shape.split(",")]
        for k, v in zip(("batch", "length", "nheads", "headdim", "dstate", "ngroups"), vals):
            cfg[k] = v
    rows = batch_slice(cfg["batch"], rank, world)
    host = ssd_inputs(cfg["batch"], cfg["length"], cfg["nheads"], cfg["headdim"], cfg["dstate"],
                      cfg["ngroups"], seed=cfg["seed"])
    for k in ("x", "dt", "B", "C", "dy"):
        host[k] = host[k][rows].contiguous()
    dev = {k: v.to(device) for k, v in host.items()}
    del host
    ops = torch.ops.b200ssm
    bucket = ParamGradBucket([dev["A"].shape, dev["D"].shape, dev["dt_bias"].shape], device)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    split = {"fwd": 0.0, "bwd": 0.0, "allreduce": 0.0, "n": 0}

    def step(record=False):
        if record:
            ev[0].record()
        y, fin, saved = ops.chunk_scan_fwd(dev["x"], dev["dt"], dev["A"], dev["B"], dev["C"], dev["D"],
                                           None, dev["dt_bias"], None, cfg["chunk"], True, True)
        if record:
            ev[1].record()
        g = ops.chunk_scan_bwd(dev["dy"], None, dev["x"], dev["dt"], dev["A"], dev["B"], dev["C"], dev["D"],
                               None, dev["dt_bias"], None, saved, cfg["chunk"], True)
        if record:
            ev[2].record()
        if world > 1:
            bucket.reduce([g[2], g[5], g[7]])
        if record:
            ev[3].record()

    ms = _timed(step, args.steps, args.warmup, world, dist)
    # one more step with events between the phases (outside the timed region)
    step(record=True)
    torch.cuda.synchronize()
    brk = {"fwd": ev[0].elapsed_time(ev[1]), "bwd": ev[1].elapsed_time(ev[2]),
           "allreduce": ev[2].elapsed_time(ev[3])}
    if world > 1:
        t = torch.tensor([brk["fwd"], brk["bwd"], brk["allreduce"]], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        brk = dict(zip(("fwd", "bwd", "allreduce"), t.tolist()))
    del dev, bucket
    if rank != 0:
        return None
    units = cfg["batch"] * cfg["length"] * cfg["nheads"] * cfg["headdim"]
    b = rows.stop - rows.start
    L, H, P, N, G, Q = (cfg[k] for k in ("length", "nheads", "headdim", "dstate", "ngroups", "chunk"))
    nc = L // Q
    # causal-minimal algorithmic flops, forward + backward: per chunk the C B^T
    # products of each group and the masked (Q x Q) x (Q x P) products plus the
    # chunk-state terms of each head
    flops = b * nc * (3 * G * Q * Q * N + H * (3 * Q * Q * P + 12 * Q * N * P))
    alg_bytes = b * L * (H * P * 2 * 4 + 2 * G * N * 2 * 2 + H * 4 * 2) + b * H * P * N * 4
    peaks, kind = _peaks()
    tflops = flops / (ms / 1e3) / 1e12
    return {
        "metric": "mamba2 SSD chunk scan fwd+bwd B*L*H*P elems/s", "value": units / (ms / 1e3),
        "unit": "elem/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "bf16 storage, fp32 compute", "data": "synthetic (seeded, BASELINE config 3)",
        "config": {"workload": "mamba2 SSD chunk scan fwd+bwd, " + ("shape override" if shape else "BASELINE config 3"), **cfg,
                   "batch_per_gpu": b, "parallelism": f"dp{world} (batch shard)",
                   "l2": "x 671 MB > L2, no flush"},
        "breakdown_ms": brk,
        "roofline": {"bound": "tensor", "achieved": tflops, "peak": peaks["bf16_tflops"],
                     "unit": "TFLOP/s", "frac": tflops / peaks["bf16_tflops"], "peak_source": kind,
                     "alg_flops_per_step": flops,
                     "hbm_frac": alg_bytes / (ms / 1e3) / 1e9 / peaks["hbm_gbs"],
                     "traffic": _traffic("ssd_step")},
        # states, outputs (forward); dstates, grads, parameter reduce (backward)
        "gpu_launches": 5 * args.steps,
    }


def run_decode(args, world, rank, device):
    """Mamba-2 decode update, B256 H80 P64 N128 G8, fp32 state,
    bf16 x/B/C, in place (out_state=state), no grad; one step = one token."""
    import torch.distributed as dist
    from metal_kernelops_b200.cv import mamba2_state_update
    from metal_kernelops_b200.parallel import batch_slice
    from metal_kernelops_b200.workloads import decode_inputs
    cfg = dict(DECODE_CONFIG)
    rows = batch_slice(cfg["batch"], rank, world)
    host = decode_inputs(cfg["batch"], cfg["nheads"], cfg["headdim"], cfg["dstate"], cfg["ngroups"],
                         seed=cfg["seed"])
    for k in ("state", "x", "dt", "B", "C"):
        host[k] = host[k][rows].contiguous()
    dev = {k: v.to(device) for k, v in host.items()}
    del host
    state = dev["state"]

    def step():
        with torch.no_grad():
            mamba2_state_update(state, dev["x"], dev["dt"], dev["A"], dev["B"], dev["C"], D=dev["D"],
                                dt_bias=dev["dt_bias"], dt_softplus=True, out_state=state)

    ms = _timed(step, args.steps, args.warmup, world, dist)
    del dev, state
    if rank != 0:
        return None
    b = rows.stop - rows.start
    H, P, N, G = cfg["nheads"], cfg["headdim"], cfg["dstate"], cfg["ngroups"]
    units = cfg["batch"] * H * P * N
    alg_bytes = b * H * P * N * 8 + b * H * P * (2 + 4) + b * G * N * 2 * 2 + b * H * 4
    gbs = alg_bytes / (ms / 1e3) / 1e9
    peaks, kind = _peaks()
    return {
        "metric": "mamba2 decode state update state elems/s", "value": units / (ms / 1e3),
        "unit": "elem/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "fp32 state, bf16 x/B/C", "data": "synthetic (seeded, BASELINE config 4)",
        "config": {"workload": "mamba2 decode update, BASELINE config 4 (in place)", **cfg,
                   "batch_per_gpu": b, "parallelism": f"dp{world} (batch shard)",
                   "l2": "state 671 MB > L2, no flush"},
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": gbs / peaks["hbm_gbs"], "peak_source": kind,
                     "alg_bytes_per_launch": alg_bytes, "traffic": _traffic("decode_step")},
        "gpu_launches": args.steps,
    }


def run_ss2d(args, world, rank, device):
    """VMamba four-path 2D scan fwd+bwd, fp32 as in the reference,
    at the reference's largest timed shape (b1 d96 56x56, 16 states) unless
    --shape batch,channels,height,width overrides it; batch sharded."""
    import torch.distributed as dist
    from metal_kernelops_b200.parallel import batch_slice
    from metal_kernelops_b200.workloads import ss2d_inputs
    cfg = dict(SS2D_CONFIG)
    if args.shape:
        cfg["batch"], cfg["channels"], cfg["height"], cfg["width"] = (int(v) for v in args.shape.split(","))
    rows = batch_slice(cfg["batch"], rank, world)
    u, dt, A, B, C = ss2d_inputs(cfg["batch"], cfg["channels"], cfg["groups"], cfg["dstate"],
                                 cfg["height"], cfg["width"], seed=cfg["seed"])
    u, dt, B, C = (t[rows].contiguous().to(device) for t in (u, dt, B, C))
    A = A.to(device)
    g = torch.Generator().manual_seed(cfg["seed"] + 1)
    dy = torch.randn(u.shape, generator=g).to(device)
    ops = torch.ops.b200ssm

    def fwd():
        return ops.ss2d_scan_fwd(u, dt, A, B, C, 1.0, True)

    def step():
        y, ck = fwd()
        ops.ss2d_scan_bwd(dy, u, dt, A, B, C, ck, 1.0)

    ms = _timed(step, args.steps, args.warmup, world, dist)
    fwd_ms = _timed(fwd, args.steps, args.warmup, world, dist)
    if rank != 0:
        return None
    b = rows.stop - rows.start
    C_, G, N, H, W = (cfg[k] for k in ("channels", "groups", "dstate", "height", "width"))
    L = H * W
    units = cfg["batch"] * C_ * L
    alg_bytes = b * (32 * C_ * L + 24 * G * N * L)
    gbs = alg_bytes / (ms / 1e3) / 1e9
    peaks, kind = _peaks()
    return {
        "metric": "ss2d four-path scan fwd+bwd B*C*H*W elems/s", "value": units / (ms / 1e3),
        "unit": "elem/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "fp32", "data": "synthetic (seeded, reference verifier distributions)",
        "config": {"workload": "VMamba ss2d four-path scan fwd+bwd", **cfg,
                   "parallelism": f"dp{world} (batch shard)"},
        "breakdown_ms": {"fwd": fwd_ms, "bwd": ms - fwd_ms},
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": gbs / peaks["hbm_gbs"], "peak_source": kind,
                     "alg_bytes_per_step": alg_bytes, "traffic": None},
        "gpu_launches": 22 * args.steps,
    }


def run_conv1d(args, world, rank, device):
    """Causal depthwise conv1d fwd+bwd, bf16, K=4, SiLU, at the
    Mamba-1 layer shape of BASELINE config 2 (x = (16, 5120, 4096)) unless
    --shape batch,channels,length overrides it; batch sharded.  HBM-bound:
    forward reads x and writes out, backward reads x and dout and writes dx."""
    import torch.distributed as dist
    from metal_kernelops_b200.parallel import batch_slice
    cfg = dict(CONV_CONFIG)
    if args.shape:
        cfg["batch"], cfg["channels"], cfg["length"] = (int(v) for v in args.shape.split(","))
    rows = batch_slice(cfg["batch"], rank, world)
    b = rows.stop - rows.start
    g = torch.Generator(device=device).manual_seed(cfg["seed"] + rank)
    x = torch.randn(b, cfg["channels"], cfg["length"], generator=g, device=device).to(torch.bfloat16)
    dout = torch.randn(b, cfg["channels"], cfg["length"], generator=g, device=device).to(torch.bfloat16)
    w = torch.randn(cfg["channels"], cfg["width"], generator=g, device=device) * 0.5
    bias = torch.randn(cfg["channels"], generator=g, device=device)
    ops = torch.ops.b200ssm

    def fwd():
        return ops.causal_conv1d_fwd(x, w, bias, None, True, False)

    def step():
        fwd()
        ops.causal_conv1d_bwd(dout, x, w, bias, None, True)

    ms = _timed(step, args.steps, args.warmup, world, dist)
    fwd_ms = _timed(fwd, args.steps, args.warmup, world, dist)
    if rank != 0:
        return None
    n = cfg["batch"] * cfg["channels"] * cfg["length"]
    alg_bytes = b * cfg["channels"] * cfg["length"] * 2 * 5
    gbs = alg_bytes / (ms / 1e3) / 1e9
    fwd_gbs = b * cfg["channels"] * cfg["length"] * 2 * 2 / (fwd_ms / 1e3) / 1e9
    peaks, kind = _peaks()
    return {
        "metric": "causal conv1d fwd+bwd B*C*L elems/s", "value": n / (ms / 1e3),
        "unit": "elem/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "bf16 storage, fp32 compute", "data": "synthetic (seeded normal)",
        "config": {"workload": "causal conv1d fwd+bwd (K=4, SiLU) at the config-2 layer shape", **cfg,
                   "parallelism": f"dp{world} (batch shard)", "l2": "x 671 MB > L2"},
        "breakdown_ms": {"fwd": fwd_ms, "bwd": ms - fwd_ms},
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": gbs / peaks["hbm_gbs"], "peak_source": kind,
                     "fwd_frac": fwd_gbs / peaks["hbm_gbs"],
                     "alg_bytes_per_step": alg_bytes, "traffic": None},
        "gpu_launches": 3 * args.steps,
    }


def run_gnorm(args, world, rank, device):
    """Gated RMSNorm fwd+bwd, bf16, gate before the norm, no bias,
    at the Mamba-2 layer shape of BASELINE config 3; rows sharded.  HBM-bound:
    forward reads x, z and writes out; backward reads x, z, dy and writes dx, dz."""
    import torch.distributed as dist
    from metal_kernelops_b200.parallel import batch_slice
    cfg = dict(GNORM_CONFIG)
    if args.shape:
        cfg["rows"], cfg["features"], cfg["group_size"] = (int(v) for v in args.shape.split(","))
    rows = batch_slice(cfg["rows"], rank, world)
    n = rows.stop - rows.start
    g = torch.Generator(device=device).manual_seed(cfg["seed"] + rank)
    x = torch.randn(n, cfg["features"], generator=g, device=device).to(torch.bfloat16)
    z = torch.randn(n, cfg["features"], generator=g, device=device).to(torch.bfloat16)
    dy = torch.randn(n, cfg["features"], generator=g, device=device).to(torch.bfloat16)
    w = torch.randn(cfg["features"], generator=g, device=device)
    ops = torch.ops.b200ssm
    gate = 2 if cfg["norm_before_gate"] else 1

    def fwd():
        return ops.gated_rmsnorm_fwd(x, w, None, z, 1e-5, cfg["group_size"], gate, True)

    def step():
        _, rstd = fwd()
        ops.gated_rmsnorm_bwd(dy, x, w, None, z, rstd, 1e-5, cfg["group_size"], gate)

    ms = _timed(step, args.steps, args.warmup, world, dist)
    fwd_ms = _timed(fwd, args.steps, args.warmup, world, dist)
    if rank != 0:
        return None
    elems = n * cfg["features"]
    alg_bytes = elems * 2 * 8
    gbs = alg_bytes / (ms / 1e3) / 1e9
    peaks, kind = _peaks()
    return {
        "metric": "gated RMSNorm fwd+bwd rows*features elems/s",
        "value": cfg["rows"] * cfg["features"] / (ms / 1e3),
        "unit": "elem/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "bf16 storage, fp32 compute", "data": "synthetic (seeded normal)",
        "config": {"workload": "gated RMSNorm fwd+bwd at the config-3 layer shape", **cfg,
                   "parallelism": f"dp{world} (row shard)", "l2": "x 671 MB > L2"},
        "breakdown_ms": {"fwd": fwd_ms, "bwd": ms - fwd_ms},
        "roofline": {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": gbs / peaks["hbm_gbs"], "peak_source": kind,
                     "fwd_frac": elems * 2 * 3 / (fwd_ms / 1e3) / 1e9 / peaks["hbm_gbs"],
                     "alg_bytes_per_step": alg_bytes, "traffic": None},
        "gpu_launches": 3 * args.steps,
    }


BLOCK_CONFIG = dict(batch=8, length=8192, d_model=2560, nheads=80, headdim=64, dstate=128, ngroups=8,
                    conv=4, chunk=256, seed=1008)


def run_block(args, world, rank, device):
    """One Mamba-2 layer, fwd + bwd + SGD step, bf16 autocast, at the shape of
    BASELINE config 3 (d_inner = 80 x 64, state 128, 8 groups, 8 x 8192
    tokens): in_proj (cuBLAS) -> causal conv1d + SiLU -> SSD chunk scan ->
    gated RMSNorm -> out_proj (cuBLAS), the block of the reference's
    integration verifier (benchmarks/verify_cv_integration.py:37-74) at layer
    size, with the in-projection output split once (as Mamba-2 layer code
    does) where the verifier slices it three times.  Batch sharded; the metric
    is tokens per second."""
    import torch.distributed as dist
    from metal_kernelops_b200.cv import causal_conv1d_fn, mamba2_chunk_scan, rmsnorm_gated
    from metal_kernelops_b200.parallel import batch_slice
    cfg = dict(BLOCK_CONFIG)
    if args.shape:
        cfg["batch"], cfg["length"] = (int(v) for v in args.shape.split(",")[:2])
    rows = batch_slice(cfg["batch"], rank, world)
    b = rows.stop - rows.start
    H, P, N, G, L = cfg["nheads"], cfg["headdim"], cfg["dstate"], cfg["ngroups"], cfg["length"]
    inner, gn = H * P, G * N
    torch.manual_seed(cfg["seed"])
    in_proj = torch.nn.Linear(cfg["d_model"], 2 * inner + 2 * gn + H, device=device)
    out_proj = torch.nn.Linear(inner, cfg["d_model"], device=device)
    conv_w = torch.nn.Parameter(torch.randn(inner + 2 * gn, cfg["conv"], device=device) * .3)
    conv_b = torch.nn.Parameter(torch.randn(inner + 2 * gn, device=device) * .1)
    a_log = torch.nn.Parameter(torch.rand(H, device=device) * 2.7)
    d_skip = torch.nn.Parameter(torch.ones(H, device=device))
    dt_bias = torch.nn.Parameter(torch.randn(H, device=device) * .2 - 4.0)
    norm_w = torch.nn.Parameter(torch.ones(inner, device=device))
    params = list(in_proj.parameters()) + list(out_proj.parameters()) + [conv_w, conv_b, a_log, d_skip,
                                                                          dt_bias, norm_w]
    opt = torch.optim.SGD(params, lr=1e-4)
    x = torch.randn(b, L, cfg["d_model"], device=device, generator=torch.Generator(device=device).manual_seed(
        cfg["seed"] + rank)).to(torch.bfloat16)

    def step():
        with torch.autocast("cuda", dtype=torch.bfloat16):
            zxbcdt = in_proj(x)
            # one split (its backward is one concatenation) rather than three
            # slices (three zero-filled full-width gradients summed)
            z, xbc, dt = torch.split(zxbcdt, [inner, inner + 2 * gn, H], dim=-1)
            xbc = causal_conv1d_fn(xbc.transpose(1, 2), conv_w, conv_b, activation="silu").transpose(1, 2)
            xs = xbc[..., :inner].reshape(b, L, H, P)
            B = xbc[..., inner:inner + gn].reshape(b, L, G, N)
            C = xbc[..., inner + gn:].reshape(b, L, G, N)
            y, _ = mamba2_chunk_scan(xs, dt, -torch.exp(a_log), B, C, chunk_size=cfg["chunk"], D=d_skip,
                                     dt_bias=dt_bias, dt_softplus=True)
            y = rmsnorm_gated(y.reshape(b, L, inner), norm_w, z=z, group_size=inner // G, norm_before_gate=False)
            loss = out_proj(y).float().square().mean()
        loss.backward()
        if world > 1:
            for prm in params:
                dist.all_reduce(prm.grad)
        opt.step()
        opt.zero_grad(set_to_none=True)

    ms = _timed(step, args.steps, args.warmup, world, dist)
    if rank != 0:
        return None
    tokens = cfg["batch"] * L
    flops_gemm = 6 * tokens * (cfg["d_model"] * (2 * inner + 2 * gn + H) + inner * cfg["d_model"])
    return {
        "metric": "Mamba-2 layer fwd+bwd+SGD tokens/s", "value": tokens / (ms / 1e3),
        "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "bf16 autocast (fp32 master weights)", "data": "synthetic (seeded normal), random-init weights",
        "config": {"workload": "Mamba-2 layer at BASELINE config 3 shape", **cfg,
                   "parallelism": f"dp{world} (batch shard, gradient all-reduce)"},
        "projection_gemm_tflop_per_step": flops_gemm / 1e12,
        "gpu_launches": None,
    }


def cpu_baseline_scan(cfg, threads, budget_s=15.0):
    """The oracle (reference CPU code restated) on a bounded sample: one batch
    row, a slice of channels, the full sequence; fwd + bwd with autograd.

    The reference steps the sequence in Python, one autograd op per step, so
    its rate grows with the channels per step until memory traffic takes over
    (on 8 host cores: 13 k elem/s at 64 channels, 131 k at 1024, 57 k at a
    full 5120-channel row, which takes 6 minutes).  512 channels keeps one
    pass within the budget while sitting near the best rate."""
    from metal_kernelops_b200.workloads import selective_scan_inputs
    from oracle.ssm_oracle import selective_scan_ref
    torch.set_num_threads(threads)
    channels = 512
    inp = selective_scan_inputs(1, channels, cfg["length"], cfg["dstate"], cfg["groups"],
                                seed=cfg["seed"], act_dtype=torch.float32)
    names = ("u", "delta", "A", "B", "C", "D", "z", "delta_bias")
    done, units, t_start = 0, 0, time.perf_counter()
    while True:
        leaves = [inp[k].clone().requires_grad_(True) for k in names]
        y = selective_scan_ref(*leaves[:5], D=leaves[5], z=leaves[6], delta_bias=leaves[7],
                               delta_softplus=True, stepping="index")
        torch.autograd.grad(y, leaves, inp["dout"])
        done += 1
        units += channels * cfg["length"]
        if time.perf_counter() - t_start > budget_s or done >= 3:
            break
    el = time.perf_counter() - t_start
    return {"value": units / el, "unit": "elem/s", "cores": threads, "kind": "port",
            "sample": f"1 batch row x {channels} channels x {cfg['length']} steps "
                      f"(dstate {cfg['dstate']}), the reference's per-step stepping, "
                      f"fp32 fwd+bwd via autograd, {done} pass(es), {el:.1f} s",
            "sample_fraction": channels / (cfg["batch"] * cfg["dim"])}


def cpu_baseline_ssd(threads, budget_s=40.0):
    """The reference's CPU path for the SSD chunk scan -- its torch composition
    (``cv/mamba2_chunk.py:447-533, :652-678``, restated in the oracle), fp32,
    forward + backward by autograd -- on one batch row of config 3 at the full
    sequence length (rows are independent, so the rate is that of the whole
    batch)."""
    from metal_kernelops_b200.workloads import ssd_inputs
    from oracle.ssm_oracle import mamba2_chunk_scan_composition
    torch.set_num_threads(threads)
    c = SSD_CONFIG
    inp = ssd_inputs(1, c["length"], c["nheads"], c["headdim"], c["dstate"], c["ngroups"], seed=c["seed"],
                     dtype=torch.float32)
    names = ("x", "dt", "A", "B", "C", "D", "dt_bias")
    done, t_start = 0, time.perf_counter()
    while True:
        lv = {k: inp[k].clone().requires_grad_(True) for k in names}
        y, _ = mamba2_chunk_scan_composition(lv["x"], lv["dt"], lv["A"], lv["B"], lv["C"], c["chunk"],
                                             D=lv["D"], dt_bias=lv["dt_bias"], dt_softplus=True)
        torch.autograd.grad((y * inp["dy"]).sum(), list(lv.values()))
        done += 1
        if time.perf_counter() - t_start > budget_s / 2 or done >= 2:
            break
    el = time.perf_counter() - t_start
    units = done * c["length"] * c["nheads"] * c["headdim"]
    return {"value": units / el, "unit": "elem/s", "cores": threads, "kind": "port",
            "sample": f"1 of {c['batch']} batch rows x {c['length']} steps (full sequence), "
                      f"reference torch composition, fp32 fwd+bwd via autograd, {done} pass(es), {el:.1f} s",
            "sample_fraction": 1.0 / c["batch"]}


def cpu_baseline_decode(threads, steps=4):
    """The reference's decode update on the CPU (``cv/mamba2_state.py:822-849``,
    restated in the oracle), fp32, at the full config-4 shape, for a few
    steps (the metric is a per-step rate)."""
    from metal_kernelops_b200.workloads import decode_inputs
    from oracle.ssm_oracle import mamba2_state_update_ref
    torch.set_num_threads(threads)
    c = DECODE_CONFIG
    d = decode_inputs(c["batch"], c["nheads"], c["headdim"], c["dstate"], c["ngroups"], seed=c["seed"],
                      dtype=torch.float32)
    st = d["state"]
    t_start = time.perf_counter()
    for _ in range(steps):
        _, st = mamba2_state_update_ref(st, d["x"], d["dt"], d["A"], d["B"], d["C"], D=d["D"],
                                        dt_bias=d["dt_bias"], dt_softplus=True)
    el = time.perf_counter() - t_start
    units = steps * c["batch"] * c["nheads"] * c["headdim"] * c["dstate"]
    return {"value": units / el, "unit": "elem/s", "cores": threads, "kind": "port",
            "sample": f"{steps} decode steps at the full config-4 shape, fp32, {el:.1f} s",
            "sample_fraction": steps / 1024}


SUB_KEYS = ("metric", "value", "unit", "ms_per_step", "dtype", "config", "breakdown_ms", "roofline",
            "gpu_launches", "cpu_baseline")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--op", default="scan", choices=["scan", "ssd", "decode", "ss2d", "conv1d", "gnorm", "block"])
    ap.add_argument("--config", type=int, default=2, choices=[1, 2])
    ap.add_argument("--shape", default=None,
                    help="override of the config (profiling runs, other shapes): scan batch,dim,seqlen; "
                         "ssd batch,length[,nheads,headdim,dstate,ngroups]")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra-ops", action="store_true",
                    help="scan line only (no ssd / decode sub-objects)")
    ap.add_argument("--lean", action="store_true",
                    help="scan: the memory-lean backward (states saved every 16 steps, the rest recomputed)")
    args = ap.parse_args()
    world, rank, local = _dist()
    threads = len(os.sched_getaffinity(0))

    if args.impl == "reference":
        if rank != 0:
            return
        cfg = CONFIGS[args.config]
        vals = []
        for _ in range(args.warmup + args.steps):
            vals.append(cpu_baseline_scan(cfg, threads, budget_s=5.0))
        timed = vals[args.warmup:]
        v = statistics.median(x["value"] for x in timed)
        units = cfg["batch"] * cfg["dim"] * cfg["length"]
        line = {
            "impl": "reference", "metric": "selective-scan fwd+bwd B*L*D elems/s", "value": v,
            "unit": "elem/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": units / v * 1e3, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
            "config": _scan_config(args, cfg, args.gpus),
            "host": f"{threads} host CPU threads (the reference has no CUDA path)",
            # each step times a sample of the workload; the step time is the
            # sample's rate applied to the whole configuration
            "extrapolated_from_fraction": timed[0]["sample_fraction"],
            "cpu_baseline": {**timed[0], "value": v},
            "e2e": {"value": v, "unit": "elem/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }
        print(json.dumps(line), flush=True)
        return

    if world > 1:
        from metal_kernelops_b200.parallel import init_process_group
        torch.cuda.set_device(local)
        init_process_group("nccl", timeout_s=300, device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    device = torch.device("cuda", torch.cuda.current_device())
    want_cpu = world == 1 and not args.no_cpu_baseline

    if args.op == "scan":
        line = run_scan(args, world, rank, device)
        if rank == 0 and want_cpu:
            line["cpu_baseline"] = cpu_baseline_scan(CONFIGS[args.config], threads)
        if not args.no_extra_ops and not args.shape:
            # the other two hot-path kernel groups at their BASELINE configs,
            # same N, same timing rules (every rank takes part in both)
            torch.cuda.empty_cache()
            for name, fn, base in (("ssd", run_ssd, cpu_baseline_ssd), ("decode", run_decode, cpu_baseline_decode)):
                sub = fn(args, world, rank, device)
                torch.cuda.empty_cache()
                if rank == 0:
                    if want_cpu:
                        sub["cpu_baseline"] = base(threads)
                    line[name] = {k: sub[k] for k in SUB_KEYS if k in sub}
                    line["gpu_launches"] += sub["gpu_launches"]
    elif args.op == "ssd":
        line = run_ssd(args, world, rank, device, shape=args.shape)
        if rank == 0 and want_cpu:
            line["cpu_baseline"] = cpu_baseline_ssd(threads)
    elif args.op == "decode":
        line = run_decode(args, world, rank, device)
        if rank == 0 and want_cpu:
            line["cpu_baseline"] = cpu_baseline_decode(threads)
    else:
        line = {"ss2d": run_ss2d, "conv1d": run_conv1d, "gnorm": run_gnorm,
                "block": run_block}[args.op](args, world, rank, device)
    # no kernel gave up on a bounded wait during any of the timed work (the
    # ops' status words; raises if one did, so no number is printed)
    import metal_kernelops_b200 as mk
    mk.check_errors()
    if rank == 0 and line is not None:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
