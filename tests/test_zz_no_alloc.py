"""The allocation-free decode backward, ``ssm_state_update_bwd_noalloc``.

Some callers cannot allocate device memory where they run the backward (their
device memory is planned up front and owned by another runtime, or the
allocator must not be touched at that point).  For them the library offers a
variant of the decode backward whose scratch is a fixed array inside the
library instead of a workspace the caller allocates.  These tests call it
through the C ABI and check, on two calls in a row, that it returns the same
gradients as the regular entry point (``ssm_state_update_bwd`` with a
workspace), within the fp32 tolerance of the decode tests; and that a problem
whose scratch does not fit the array is refused with a clear error instead of
running.

This file is named to be collected last, so that a run stopping at the first
failure has already run every other test.
"""

import pytest
import torch

from oracle import ssm_oracle as orc

pytestmark = pytest.mark.gpu

TOL = 1e-5   # fp32 tolerance of the decode tests


def _problem(batch, nheads, headdim, dstate, ngroups, seed=5):
    g = torch.Generator().manual_seed(seed)
    dev = "cuda"
    t = {
        "state": torch.randn(batch, nheads, headdim, dstate, generator=g),
        "x": torch.randn(batch, nheads, headdim, generator=g),
        "dt": torch.randn(batch, nheads, generator=g),
        "A": -torch.rand(nheads, generator=g) - 0.05,
        "B": torch.randn(batch, ngroups, dstate, generator=g),
        "C": torch.randn(batch, ngroups, dstate, generator=g),
        "D": torch.randn(nheads, generator=g),
        "z": torch.randn(batch, nheads, headdim, generator=g),
        "dt_bias": torch.randn(nheads, generator=g) * 0.1,
        "dy": torch.randn(batch, nheads, headdim, generator=g),
        "dnew": torch.randn(batch, nheads, headdim, dstate, generator=g),
    }
    return {k: v.to(dev).contiguous() for k, v in t.items()}


def _params(nat, t, out):
    batch, nheads, headdim, dstate = t["state"].shape
    p = nat.StateUpdateParams()
    p.batch, p.nheads, p.headdim, p.dstate, p.ngroups = batch, nheads, headdim, dstate, t["B"].shape[1]
    p.dtype = nat.SSM_F32
    p.flags = (nat.HAS_BIAS | nat.SOFTPLUS | nat.HAS_D | nat.HAS_Z | nat.HAS_DY | nat.HAS_DSTATE)
    for k in ("state", "x", "dt", "A", "B", "C", "D", "z", "dt_bias", "dy", "dnew"):
        setattr(p, k, t[k].data_ptr())
    for k, v in out.items():
        setattr(p, k, v.data_ptr())
    return p


def _outputs(t):
    f = lambda like: torch.empty_like(like)  # noqa: E731
    return {"grad_state": f(t["state"]), "dx": f(t["x"]), "ddt": f(t["dt"]), "dA": f(t["A"]),
            "dB": f(t["B"]), "dC": f(t["C"]), "dD": f(t["D"]), "dz": f(t["z"]),
            "ddt_bias": f(t["A"])}


def test_noalloc_matches_workspace_backward_twice():
    from metal_kernelops_b200 import _native as nat
    lib = nat.lib()
    t = _problem(batch=4, nheads=16, headdim=64, dstate=128, ngroups=4)
    stream = nat.stream_of(t["state"])

    ref = _outputs(t)
    p = _params(nat, t, ref)
    need = nat._SZ()
    assert lib.ssm_state_update_sizes(p, need) == nat.SSM_OK
    work = torch.empty(need.value, dtype=torch.uint8, device="cuda")
    p.workspace, p.workspace_bytes = work.data_ptr(), work.numel()
    nat.check(lib.ssm_state_update_bwd(p, stream), "ssm_state_update_bwd")

    runs = []
    for _ in range(2):
        out = _outputs(t)
        q = _params(nat, t, out)        # no workspace given
        nat.check(lib.ssm_state_update_bwd_noalloc(q, stream), "ssm_state_update_bwd_noalloc")
        runs.append(out)
    torch.cuda.synchronize()
    for out in runs:
        for k in ref:
            assert orc.norm_rel(out[k].cpu(), ref[k].cpu()) <= TOL, k


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
