"""Batch-sharded data parallelism on CPU with gloo (world size 2).

Each rank runs the CPU oracle on its batch shard, sums the shared-parameter
gradients with the package's single-bucket all-reduce, and must reproduce the
single-process gradients of the whole batch: for the Mamba-1 selective scan
(dA, dD, d delta_bias) and for the Mamba-2 SSD chunk scan (dA, dD, d dt_bias).
A third test checks failure detection on the host: one rank exits before the
collective, and the other rank's all-reduce ends with an error within the
process-group timeout instead of hanging.

Workers are spawned processes that hand their results back through files in
a temporary directory (no queue or pipe shared with the parent), and the
parent joins every worker with a deadline.
"""

import multiprocessing as mp
import os
import pathlib
import socket
import tempfile

import torch

from metal_kernelops_b200.parallel import ParamGradBucket, batch_slice, shard_batch

PARAMS = ("A", "D", "delta_bias")
SSD_PARAMS = ("A", "D", "dt_bias")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _spawn(target, world, *args, deadline=180):
    """Run ``target(rank, world, port, outdir, *args)`` on ``world`` spawned
    processes; returns {rank: object the rank saved} and the exit codes."""
    port = _free_port()
    ctx = mp.get_context("spawn")
    with tempfile.TemporaryDirectory() as tmp:
        procs = [ctx.Process(target=target, args=(r, world, port, tmp, *args)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=deadline)
        codes = []
        for p in procs:
            if p.is_alive():
                p.kill()
                p.join(timeout=10)
            codes.append(p.exitcode)
        out = {}
        for r in range(world):
            f = pathlib.Path(tmp) / f"{r}.pt"
            if f.exists():
                out[r] = torch.load(f)
        return out, codes


def _init(rank, world, port, timeout_s=60):
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))
    return dist


def _inputs():
    from oracle import ssm_oracle as orc
    inp = orc.selective_scan_inputs(4, 6, 20, 5, 2, seed=77, act_dtype=torch.float64)
    return {k: v.double() for k, v in inp.items()}


def _worker(rank, world, port, outdir):
    from oracle import ssm_oracle as orc
    dist = _init(rank, world, port)
    inp = _inputs()
    u, delta, z, dout, B, C = shard_batch([inp[k] for k in ("u", "delta", "z", "dout", "B", "C")],
                                          rank, world)
    params = {k: inp[k].clone().requires_grad_(True) for k in PARAMS}
    y = orc.selective_scan_ref(u, delta, params["A"], B, C, D=params["D"], z=z,
                               delta_bias=params["delta_bias"], delta_softplus=True)
    grads = torch.autograd.grad(y, [params[k] for k in PARAMS], dout)
    bucket = ParamGradBucket([g.shape for g in grads], "cpu", dtype=torch.float64)
    torch.save([r.clone() for r in bucket.reduce(grads)], pathlib.Path(outdir) / f"{rank}.pt")
    dist.destroy_process_group()


def test_batch_slices_cover_the_batch():
    for batch in (1, 2, 7, 16):
        for world in (1, 2, 3, 8):
            rows = []
            for r in range(world):
                s = batch_slice(batch, r, world)
                rows.extend(range(s.start, s.stop))
            assert rows == list(range(batch))


def test_gloo_data_parallel_matches_single_process():
    from oracle import ssm_oracle as orc
    results, codes = _spawn(_worker, 2)
    assert codes == [0, 0], codes
    inp = _inputs()
    params = {k: inp[k].clone().requires_grad_(True) for k in PARAMS}
    y = orc.selective_scan_ref(inp["u"], inp["delta"], params["A"], inp["B"], inp["C"],
                               D=params["D"], z=inp["z"], delta_bias=params["delta_bias"],
                               delta_softplus=True)
    full = torch.autograd.grad(y, [params[k] for k in PARAMS], inp["dout"])
    for r in (0, 1):
        for got, want in zip(results[r], full):
            assert torch.allclose(got, want, rtol=1e-12, atol=1e-12)


def _ssd_inputs():
    from oracle import ssm_oracle as orc
    inp = orc.ssd_inputs(3, 40, 4, 8, 16, 2, seed=78, dtype=torch.float64)
    return {k: v.double() for k, v in inp.items()}


def _ssd_worker(rank, world, port, outdir):
    from oracle import ssm_oracle as orc
    dist = _init(rank, world, port)
    inp = _ssd_inputs()
    x, dt, B, C, dy = shard_batch([inp[k] for k in ("x", "dt", "B", "C", "dy")], rank, world)
    params = {k: inp[k].clone().requires_grad_(True) for k in SSD_PARAMS}
    y, _ = orc.mamba2_chunk_scan_ref(x, dt, params["A"], B, C, 16, D=params["D"],
                                     dt_bias=params["dt_bias"], dt_softplus=True)
    grads = torch.autograd.grad(y, [params[k] for k in SSD_PARAMS], dy)
    bucket = ParamGradBucket([g.shape for g in grads], "cpu", dtype=torch.float64)
    torch.save([r.clone() for r in bucket.reduce(grads)], pathlib.Path(outdir) / f"{rank}.pt")
    dist.destroy_process_group()


def test_gloo_ssd_data_parallel_matches_single_process():
    """The SSD chunk scan sharded by batch (3 rows over 2 ranks: 2 + 1): the
    bucketed all-reduce of dA, dD and d dt_bias equals the gradients of the
    whole batch in one process."""
    from oracle import ssm_oracle as orc
    results, codes = _spawn(_ssd_worker, 2)
    assert codes == [0, 0], codes
    inp = _ssd_inputs()
    params = {k: inp[k].clone().requires_grad_(True) for k in SSD_PARAMS}
    y, _ = orc.mamba2_chunk_scan_ref(inp["x"], inp["dt"], params["A"], inp["B"], inp["C"], 16,
                                     D=params["D"], dt_bias=params["dt_bias"], dt_softplus=True)
    full = torch.autograd.grad(y, [params[k] for k in SSD_PARAMS], inp["dy"])
    for r in (0, 1):
        for got, want in zip(results[r], full):
            assert torch.allclose(got, want, rtol=1e-12, atol=1e-12)


def _dying_worker(rank, world, port, outdir):
    dist = _init(rank, world, port, timeout_s=3)
    if rank == 1:
        os._exit(0)           # leaves between steps, before the collective
    bucket = ParamGradBucket([torch.Size([8])], "cpu")
    try:
        bucket.reduce([torch.ones(8)])
        msg = "no error"
    except Exception as exc:  # noqa: BLE001
        msg = f"error: {type(exc).__name__}"
    torch.save(msg, pathlib.Path(outdir) / f"{rank}.pt")
    del dist


def test_lost_rank_is_detected_by_timeout():
    results, _ = _spawn(_dying_worker, 2, deadline=120)
    assert 0 in results, "the surviving rank did not report"
    assert results[0].startswith("error"), results[0]
