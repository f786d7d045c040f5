"""VMamba four-path 2D selective scan on the GPU vs the fp64 oracle.

Mirrors the reference's verifier (benchmarks/verify_path_scan.py): forward and
all five gradients on its shapes, degenerate extents, both merge modes, the
cumulative-sum ordering known answer, the state limit, strided inputs, plus the
golden fixtures made from the reference's own ``ss2d_scan_reference``.  Error
metric: norm-relative (the verifier's ``relative``); float32 tolerances are the
verifier's, 1e-5 forward and 1e-4 gradients; bfloat16 activations 2e-2.
"""

import pytest
import torch

from oracle import ssm_oracle as orc

pytestmark = pytest.mark.gpu

NAMES = ("u", "dt", "A", "B", "C")


def _mod():
    from metal_kernelops_b200.cv import path_scan
    return path_scan


def _rel(got, want):
    got, want = got.detach(), want.detach()
    den = float(want.norm())
    if den == 0.0:
        return 0.0 if float(got.norm()) == 0.0 else float("inf")
    return float((got - want).norm()) / den


def _check(args, merge="sum", tol=1e-5, gtol=1e-4, dtype=torch.float32, seed=0):
    m = _mod()
    want = orc.ss2d_scan_ref(*[t.double() for t in args], merge=merge)
    dev = [t.to("cuda", dtype if i != 2 else torch.float32) for i, t in enumerate(args)]
    got = m.ss2d_scan(*dev, merge=merge)
    assert tuple(got.shape) == tuple(want.shape)
    assert got.dtype == dtype
    assert torch.isfinite(got).all()
    assert _rel(got.double().cpu(), want) < tol
    g = torch.Generator().manual_seed(seed)
    cot = torch.randn(want.shape, generator=g, dtype=torch.float64)
    leaves = [t.double().clone().requires_grad_(True) for t in args]
    ref = torch.autograd.grad(orc.ss2d_scan_ref(*leaves, merge=merge), leaves, cot)
    dl = [t.clone().requires_grad_(True) for t in dev]
    fast = torch.autograd.grad(m.ss2d_scan(*dl, merge=merge), dl, cot.to("cuda", dtype))
    for name, a, b in zip(NAMES, fast, ref):
        assert a.shape == b.shape, name
        assert _rel(a.double().cpu(), b) < gtol, (name, _rel(a.double().cpu(), b))


SHAPES = {
    "fb_1x3x3x2_5x7": ((1, 3, 3, 2, 5, 7), "sum"),
    "fb_2x16x1x8_8x8": ((2, 16, 1, 8, 8, 8), "sum"),
    "fb_2x8x2x4_6x5": ((2, 8, 2, 4, 6, 5), "sum"),
    "per_channel_groups": ((1, 4, 4, 3, 3, 5), "sum"),
    "one_channel": ((1, 1, 1, 3, 3, 3), "sum"),
    "sixteen_states": ((1, 8, 1, 16, 9, 11), "sum"),
    "thirty_two_states": ((1, 4, 2, 32, 5, 7), "sum"),
    "five_states": ((1, 6, 2, 5, 13, 3), "sum"),
    "mean_merge": ((1, 4, 1, 3, 4, 5), "mean"),
    "single_pixel": ((1, 4, 1, 3, 1, 1), "sum"),
    "single_row": ((1, 4, 1, 3, 1, 7), "sum"),
    "single_column": ((1, 4, 1, 3, 7, 1), "sum"),
    "wide_map": ((1, 5, 1, 16, 3, 45), "sum"),
}


@pytest.mark.parametrize("idx", range(len(SHAPES)), ids=list(SHAPES))
def test_forward_backward(idx):
    shape, merge = list(SHAPES.values())[idx]
    _check(orc.ss2d_inputs(*shape, seed=40 + idx), merge=merge)


def _four_calls(args, merge):
    """The four paths as four calls of this package's Mamba-1 ``selective_scan``
    on permuted copies (the reference verifier's baseline,
    verify_path_scan.py:323-358), merged (p0 + p2) + (p1 + p3)."""
    from metal_kernelops_b200 import selective_scan
    u, dt, A, B, C = args
    batch, channels, height, width = u.shape
    groups, states = B.shape[1], A.shape[1]
    length = height * width
    fu, fdt = u.reshape(batch, channels, length), dt.reshape(batch, channels, length)
    fb, fc = B.reshape(batch, groups, states, length), C.reshape(batch, groups, states, length)
    out = []
    for order in orc.ss2d_path_orders(height, width):
        order = order.to(u.device)
        y = selective_scan(fu.index_select(-1, order), fdt.index_select(-1, order), A,
                           fb.index_select(-1, order), fc.index_select(-1, order))
        out.append(torch.zeros_like(y).index_copy(-1, order, y))
    total = (out[0] + out[2]) + (out[1] + out[3])
    return (total * 0.25 if merge == "mean" else total).reshape(u.shape)


@pytest.mark.parametrize("shape,merge", [((1, 2, 1, 4, 160, 155), "mean"),
                                         ((1, 96, 1, 16, 56, 56), "sum"),
                                         ((4, 192, 2, 16, 28, 28), "sum")],
                         ids=["map_above_smem_limit", "vmamba_56x56", "vmamba_28x28_b4"])
def test_against_four_scan_calls(shape, merge):
    """Maps too large for the fp64 oracle's autograd: forward and every gradient
    against four calls of the (separately parity-tested) Mamba-1 scan on
    permuted copies.  The two differ only in summation order."""
    m = _mod()
    args = [t.cuda() for t in orc.ss2d_inputs(*shape, seed=17)]
    g = torch.Generator().manual_seed(18)
    cot = torch.randn(shape[0], shape[1], shape[4], shape[5], generator=g).cuda()
    la = [t.clone().requires_grad_(True) for t in args]
    lb = [t.clone().requires_grad_(True) for t in args]
    ya = m.ss2d_scan(*la, merge=merge)
    yb = _four_calls(lb, merge)
    assert _rel(ya.double(), yb.double()) < 1e-5
    ga = torch.autograd.grad(ya, la, cot)
    gb = torch.autograd.grad(yb, lb, cot)
    for name, a, b in zip(NAMES, ga, gb):
        assert _rel(a.double(), b.double()) < 1e-4, name


@pytest.mark.parametrize("name", ["zero_height", "zero_width", "no_channels", "no_states", "batch_of_zero"])
def test_degenerate_shapes(name):
    shape = {"zero_height": (1, 4, 1, 3, 0, 5), "zero_width": (1, 4, 1, 3, 5, 0),
             "no_channels": (2, 0, 0, 4, 3, 3), "no_states": (1, 4, 1, 0, 3, 3),
             "batch_of_zero": (0, 4, 1, 3, 3, 3)}[name]
    m = _mod()
    args = [t.cuda().requires_grad_(True) for t in orc.ss2d_inputs(*shape, seed=3)]
    y = m.ss2d_scan(*args)
    assert tuple(y.shape) == (shape[0], shape[1], shape[4], shape[5])
    assert float(y.abs().sum()) == 0.0
    grads = torch.autograd.grad(y.sum(), args, allow_unused=True)
    for g, t in zip(grads, args):
        assert g is None or float(g.abs().sum()) == 0.0


@pytest.mark.parametrize("case", ["fb_1x3x3x2_5x7", "fb_2x16x1x8_8x8", "fb_2x8x2x4_6x5", "five_states",
                                  "mean_merge", "single_row", "single_column", "thirty_two_states"])
def test_golden(golden, case):
    """The reference's own ss2d_scan_reference outputs (fp64), reproduced in fp32."""
    m = _mod()
    c = golden("path_scan")[case]
    dev = [c["inputs"][k].float().cuda().requires_grad_(True) for k in NAMES]
    y = m.ss2d_scan(*dev, merge=c["merge"])
    assert _rel(y.double().detach().cpu(), c["y"]) < 1e-5
    grads = torch.autograd.grad(y, dev, c["dy"].float().cuda())
    for k, g in zip(NAMES, grads):
        assert _rel(g.double().cpu(), c["grads"][k]) < 1e-4, k


def test_order_cumsum_kat():
    m = _mod()
    for height, width in ((4, 3), (1, 6), (6, 1), (5, 5), (17, 33)):
        length = height * width
        g = torch.Generator().manual_seed(height * 31 + width)
        values = torch.randn(1, 1, length, generator=g)
        expected = torch.zeros(1, 1, length, dtype=torch.float64)
        for order in orc.ss2d_path_orders(height, width):
            seq = values[0, 0].double().index_select(0, order).cumsum(0)
            back = torch.empty_like(seq)
            back[order] = seq
            expected[0, 0] += back
        shape = (1, 1, height, width)
        got = m.ss2d_scan(values.reshape(shape).cuda(), torch.ones(shape, device="cuda"),
                          torch.zeros((1, 1), device="cuda"),
                          torch.ones((1, 1, 1, height, width), device="cuda"),
                          torch.ones((1, 1, 1, height, width), device="cuda"))
        assert _rel(got.double().cpu(), expected.reshape(shape)) < 1e-6


def test_path_orders_match_oracle():
    m = _mod()
    for h, w in ((4, 3), (1, 6), (5, 5)):
        for a, b in zip(m.path_orders(h, w), orc.ss2d_path_orders(h, w)):
            assert torch.equal(a.cpu(), b)


def test_state_limit():
    m = _mod()
    args = [t.cuda() for t in orc.ss2d_inputs(1, 4, 1, 64, 3, 3, seed=3)]
    with pytest.raises(ValueError, match="32"):
        m.ss2d_scan(*args)


def test_contract_errors():
    m = _mod()
    u, dt, A, B, C = [t.cuda() for t in orc.ss2d_inputs(1, 4, 2, 3, 3, 3, seed=3)]
    with pytest.raises(ValueError):
        m.ss2d_scan(u, dt, A, B, C, merge="max")
    with pytest.raises(ValueError):
        m.ss2d_scan(u[0], dt, A, B, C)
    with pytest.raises(ValueError):
        m.ss2d_scan(u, dt, A, B[:, :, :, :2], C)
    bad_b = torch.randn(1, 3, 3, 3, 3, device="cuda")
    with pytest.raises(ValueError):
        m.ss2d_scan(u, dt, A, bad_b, bad_b)
    with pytest.raises(ValueError):
        m.ss2d_scan(u.cpu(), dt, A, B, C)


def test_noncontiguous():
    m = _mod()
    g = torch.Generator().manual_seed(91)
    su = torch.randn(2, 4, 5, 6, generator=g)
    sdt = torch.rand(2, 4, 5, 6, generator=g) * 0.2 + 0.05
    sa = -(torch.rand(3, 4, generator=g) + 0.1)
    sb = torch.randn(2, 2, 3, 5, 6, generator=g)
    sc = torch.randn(2, 2, 3, 5, 6, generator=g)
    args = [su.transpose(2, 3), sdt.transpose(2, 3), sa.transpose(0, 1), sb.transpose(3, 4), sc.transpose(3, 4)]
    assert not any(t.is_contiguous() for t in args)
    want = orc.ss2d_scan_ref(*[t.double() for t in args])
    got = m.ss2d_scan(*[t.cuda() for t in args])
    assert _rel(got.double().cpu(), want) < 1e-5


def test_bfloat16_activations():
    _check(orc.ss2d_inputs(2, 16, 2, 16, 14, 14, seed=5), tol=2e-2, gtol=2e-2, dtype=torch.bfloat16)


def test_vmamba_stage_forward_vs_oracle():
    """The reference's largest timed shape (batch 1, 96 channels, 16 states,
    56x56), forward against the fp64 oracle."""
    m = _mod()
    args = orc.ss2d_inputs(1, 96, 1, 16, 56, 56, seed=11)
    with torch.no_grad():
        want = orc.ss2d_scan_ref(*[t.double() for t in args])
        got = m.ss2d_scan(*[t.cuda() for t in args])
    assert _rel(got.double().cpu(), want) < 1e-5


def test_deterministic():
    m = _mod()
    args = [t.cuda() for t in orc.ss2d_inputs(2, 32, 2, 16, 20, 24, seed=21)]
    runs = []
    for _ in range(3):
        leaves = [t.clone().requires_grad_(True) for t in args]
        y = m.ss2d_scan(*leaves)
        runs.append((y.detach(),) + torch.autograd.grad(y.square().sum(), leaves))
    for vals in zip(*runs):
        assert all(torch.equal(vals[0], v) for v in vals[1:])
