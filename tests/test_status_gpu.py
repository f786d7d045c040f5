"""Kernel-side failures reach the caller (GPU).

Kernels that wait on an mbarrier (the tensor-core SSD pipeline, the conv1d
bulk-copy ring) give up after a bounded number of polls and write a code into
the call's status word (``params.status``), which every op of the package
passes; ``check_errors()`` reads the words and raises.  The failure is made on
purpose by the library's self-test kernel: a wait, limited to a few polls, on
an mbarrier that nothing arrives at, with no copy in flight.  It must return,
set the status, raise through ``check_errors``, and leave the context usable
for the next real call.
"""

import pytest
import torch

from oracle import ssm_oracle as orc

pytestmark = pytest.mark.gpu


def _ssd_small():
    import metal_kernelops_b200.cv as cv
    t = orc.ssd_inputs(1, 200, 2, 64, 128, 1, dtype=torch.bfloat16)
    d = {k: v.cuda().requires_grad_(v.is_floating_point()) for k, v in t.items()}
    y, fin = cv.mamba2_chunk_scan(d["x"], d["dt"], d["A"], d["B"], d["C"], 256, D=d["D"],
                                  dt_bias=d["dt_bias"], dt_softplus=True)
    g = torch.autograd.grad((y.float() * d["dy"].float()).sum(), [d[k] for k in ("x", "dt", "B", "C")])
    yr, _ = orc.mamba2_chunk_scan_ref(*(t[k].double() for k in ("x", "dt", "A", "B", "C")), 256,
                                      D=t["D"].double(), dt_bias=t["dt_bias"].double(), dt_softplus=True)
    assert orc.max_rel(y.detach().float().cpu(), yr) <= 2e-2
    return g


def test_bounded_wait_that_runs_out_is_reported_and_the_context_survives():
    from metal_kernelops_b200 import _native as nat
    import metal_kernelops_b200 as mk
    mk.check_errors()                       # nothing pending
    nat.selftest_bounded_wait(polls=8)
    word = nat._status_buffer(torch.device("cuda", torch.cuda.current_device()))
    torch.cuda.synchronize()
    assert word[nat.STATUS_SLOTS.index("selftest")].item() == 99   # SSM_KERR_SELFTEST
    with pytest.raises(RuntimeError, match="selftest"):
        mk.check_errors()
    mk.check_errors()                       # read and cleared
    # the per-device flag is untouched by the self-test, and real calls still run
    assert nat.lib().ssm_take_kernel_error() == 0
    _ssd_small()
    torch.cuda.synchronize()
    mk.check_errors()
    assert nat.lib().ssm_take_kernel_error() == 0


def test_selftest_rejects_bad_arguments():
    from metal_kernelops_b200 import _native as nat
    lib = nat.lib()
    assert lib.ssm_selftest_bounded_wait(None, 8, None) == nat.SSM_ERR_INVALID
    word = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert lib.ssm_selftest_bounded_wait(word.data_ptr(), 0, None) == nat.SSM_ERR_INVALID
    torch.cuda.synchronize()
    assert word.item() == 0


def test_every_op_passes_its_status_word():
    """A normal run of the waiting ops leaves every status word at zero."""
    import metal_kernelops_b200 as mk
    from metal_kernelops_b200 import _native as nat
    from metal_kernelops_b200.cv import causal_conv1d_fn
    _ssd_small()
    x = torch.randn(2, 64, 9000, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    w = torch.randn(64, 4, device="cuda", requires_grad=True)
    out = causal_conv1d_fn(x, w, None, activation="silu")
    torch.autograd.grad(out.float().sum(), [x, w])
    torch.cuda.synchronize()
    word = nat._status_buffer(torch.device("cuda", torch.cuda.current_device()))
    assert not word.any()
    mk.check_errors()
