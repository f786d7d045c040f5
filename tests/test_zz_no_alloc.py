"""The allocation-free decode backward, ``ssm_state_update_bwd_noalloc``.

Some callers cannot allocate device memory where they run the backward (their
device memory is planned up front and owned by another runtime, or the
allocator must not be touched at that point).  For them the library offers a
variant of the decode backward whose scratch is a fixed array inside the
library instead of a workspace the caller allocates.  These tests call it
through the C ABI, several times in a row on problems of different sizes and
options, and check that:

* every call returns exactly the gradients of the regular entry point
  (``ssm_state_update_bwd``), run with a workspace pre-filled with NaN -- both
  run the same deterministic kernels, so the results are equal bit for bit,
  and nothing a previous call left in the shared array leaks into the next;
* the calls change neither torch's allocated-bytes counter nor the device's
  free memory (``cudaMemGetInfo``): nothing is allocated;
* a problem whose scratch does not fit the array is refused with a clear
  error instead of running.

This file is named to be collected last, so that a run stopping at the first
failure has already run every other test.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu


def _problem(batch, nheads, headdim, dstate, ngroups, seed, d_per_head=False, use_d=True,
             dt_per_row=False):
    g = torch.Generator().manual_seed(seed)
    t = {
        "state": torch.randn(batch, nheads, headdim, dstate, generator=g),
        "x": torch.randn(batch, nheads, headdim, generator=g),
        "dt": torch.randn(*((batch, nheads, headdim) if dt_per_row else (batch, nheads)), generator=g),
        "A": -torch.rand(nheads, generator=g) - 0.05,
        "B": torch.randn(batch, ngroups, dstate, generator=g),
        "C": torch.randn(batch, ngroups, dstate, generator=g),
        "z": torch.randn(batch, nheads, headdim, generator=g),
        "dt_bias": torch.randn(nheads, generator=g) * 0.1,
        "dy": torch.randn(batch, nheads, headdim, generator=g),
        "dnew": torch.randn(batch, nheads, headdim, dstate, generator=g),
    }
    if use_d:
        t["D"] = torch.randn(*((nheads, headdim) if d_per_head else (nheads,)), generator=g)
    t = {k: v.to("cuda").contiguous() for k, v in t.items()}
    t["_options"] = (d_per_head, dt_per_row)
    return t


def _params(nat, t, out):
    batch, nheads, headdim, dstate = t["state"].shape
    p = nat.StateUpdateParams()
    p.batch, p.nheads, p.headdim, p.dstate, p.ngroups = batch, nheads, headdim, dstate, t["B"].shape[1]
    p.dtype = nat.SSM_F32
    d_per_head, dt_per_row = t["_options"]
    p.flags = (nat.HAS_BIAS | nat.SOFTPLUS | nat.HAS_Z | nat.HAS_DY | nat.HAS_DSTATE |
               (nat.HAS_D if "D" in t else 0) | (nat.D_PER_HEAD if d_per_head else 0) |
               (nat.DT_PER_ROW if dt_per_row else 0))
    for k in ("state", "x", "dt", "A", "B", "C", "D", "z", "dt_bias", "dy", "dnew"):
        if k in t:
            setattr(p, k, t[k].data_ptr())
    for k, v in out.items():
        setattr(p, k, v.data_ptr())
    return p


def _outputs(t):
    like = {"grad_state": "state", "dx": "x", "ddt": "dt", "dA": "A", "dB": "B", "dC": "C",
            "dz": "z", "ddt_bias": "A"}
    if "D" in t:
        like["dD"] = "D"
    return {k: torch.full_like(t[v], float("nan")) for k, v in like.items()}


def _reference(nat, t):
    """The workspace entry point, with its workspace filled with NaN first."""
    lib = nat.lib()
    out = _outputs(t)
    p = _params(nat, t, out)
    need = nat._SZ()
    assert lib.ssm_state_update_sizes(p, need) == nat.SSM_OK
    work = torch.full((max(need.value, 4) // 4,), float("nan"), dtype=torch.float32, device="cuda")
    p.workspace, p.workspace_bytes = work.data_ptr(), work.numel() * 4
    nat.check(lib.ssm_state_update_bwd(p, nat.stream_of(t["state"])), "ssm_state_update_bwd")
    torch.cuda.synchronize()
    return out, need.value


def test_noalloc_matches_workspace_backward_on_calls_in_a_row():
    from metal_kernelops_b200 import _native as nat
    lib = nat.lib()
    # large (D per head and channel) -> small with other options (no D, dt per
    # row) -> the large one again: each reads back only scratch it wrote itself
    problems = [
        _problem(4, 16, 64, 128, 4, seed=5, d_per_head=True),
        _problem(2, 6, 16, 32, 3, seed=6, use_d=False, dt_per_row=True),
        _problem(4, 16, 64, 128, 4, seed=7, d_per_head=True),
    ]
    refs = []
    for t in problems:
        ref, need = _reference(nat, t)
        assert 0 < need <= (8 << 20)
        refs.append(ref)

    # the first call in this context looks the array up (and may load the
    # library's kernels); the memory checks cover the calls after it
    warm = _outputs(problems[1])
    nat.check(lib.ssm_state_update_bwd_noalloc(_params(nat, problems[1], warm), nat.stream_of(warm["dx"])),
              "ssm_state_update_bwd_noalloc")
    torch.cuda.synchronize()

    outs = [_outputs(t) for t in problems]
    calls = [_params(nat, t, o) for t, o in zip(problems, outs)]   # no workspace given
    torch.cuda.synchronize()
    allocated, (free, _) = torch.cuda.memory_allocated(), torch.cuda.mem_get_info()
    for t, q in zip(problems, calls):
        nat.check(lib.ssm_state_update_bwd_noalloc(q, nat.stream_of(t["state"])), "ssm_state_update_bwd_noalloc")
        torch.cuda.synchronize()
    assert torch.cuda.memory_allocated() == allocated
    assert torch.cuda.mem_get_info()[0] == free
    for i, (out, ref) in enumerate(zip(outs, refs)):
        assert set(out) == set(ref)
        for k in out:
            assert torch.equal(out[k], ref[k]), (i, k)


def test_noalloc_refuses_problems_beyond_its_scratch():
    """A problem needing more scratch than the fixed array is refused before
    any launch; the workspace entry point still runs it."""
    from metal_kernelops_b200 import _native as nat
    lib = nat.lib()
    t = _problem(batch=96, nheads=80, headdim=64, dstate=128, ngroups=8, seed=6)
    out = _outputs(t)
    p = _params(nat, t, out)
    need = nat._SZ()
    assert lib.ssm_state_update_sizes(p, need) == nat.SSM_OK
    assert need.value > (8 << 20)
    stream = nat.stream_of(t["state"])
    status = lib.ssm_state_update_bwd_noalloc(p, stream)
    assert status == nat.SSM_ERR_UNSUPPORTED
    assert b"fixed array" in lib.ssm_last_error()
    work = torch.empty(need.value, dtype=torch.uint8, device="cuda")
    p.workspace, p.workspace_bytes = work.data_ptr(), work.numel()
    nat.check(lib.ssm_state_update_bwd(p, stream), "ssm_state_update_bwd")
    torch.cuda.synchronize()
    assert all(torch.isfinite(v).all() for v in out.values())
