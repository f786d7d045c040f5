"""Batch-sharded data parallelism on CPU with gloo (world size 2).

Each rank runs the CPU oracle on its batch shard, sums the shared-parameter
gradients with the package's single-bucket all-reduce, and must reproduce the
single-process gradients of the whole batch.  A second test checks failure
detection on the host: one rank exits before the collective, and the other
rank's all-reduce ends with an error within the process-group timeout instead
of hanging.
"""

import multiprocessing as mp
import os
import socket

import torch

from metal_kernelops_b200.parallel import ParamGradBucket, batch_slice, shard_batch

PARAMS = ("A", "D", "delta_bias")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    from oracle import ssm_oracle as orc
    inp = orc.selective_scan_inputs(4, 6, 20, 5, 2, seed=77, act_dtype=torch.float64)
    return {k: v.double() for k, v in inp.items()}


def _worker(rank, world, port, q):
    import torch.distributed as dist
    from oracle import ssm_oracle as orc
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    inp = _inputs()
    u, delta, z, dout, B, C = shard_batch([inp[k] for k in ("u", "delta", "z", "dout", "B", "C")],
                                          rank, world)
    params = {k: inp[k].clone().requires_grad_(True) for k in PARAMS}
    y = orc.selective_scan_ref(u, delta, params["A"], B, C, D=params["D"], z=z,
                               delta_bias=params["delta_bias"], delta_softplus=True)
    grads = torch.autograd.grad(y, [params[k] for k in PARAMS], dout)
    bucket = ParamGradBucket([g.shape for g in grads], "cpu", dtype=torch.float64)
    q.put((rank, [r.clone() for r in bucket.reduce(grads)]))
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
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    inp = _inputs()
    params = {k: inp[k].clone().requires_grad_(True) for k in PARAMS}
    y = orc.selective_scan_ref(inp["u"], inp["delta"], params["A"], inp["B"], inp["C"],
                               D=params["D"], z=inp["z"], delta_bias=params["delta_bias"],
                               delta_softplus=True)
    full = torch.autograd.grad(y, [params[k] for k in PARAMS], inp["dout"])
    for r in (0, 1):
        for got, want in zip(results[r], full):
            assert torch.allclose(got, want, rtol=1e-12, atol=1e-12)


def _dying_worker(rank, world, port, q):
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=3))
    if rank == 1:
        os._exit(0)           # leaves between steps, before the collective
    bucket = ParamGradBucket([torch.Size([8])], "cpu")
    try:
        bucket.reduce([torch.ones(8)])
        q.put("no error")
    except Exception as exc:  # noqa: BLE001
        q.put(f"error: {type(exc).__name__}")


def test_lost_rank_is_detected_by_timeout():
    port = _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_dying_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    msg = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert msg.startswith("error"), msg
