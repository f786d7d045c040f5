"""Gated RMSNorm on the GPU vs the fp64 oracle.

Mirrors the reference's verifier (benchmarks/verify_gated_norm.py): its
correctness cases (:79-97) for the forward and its gradient cases (:121-131) in
float32, float16 and bfloat16, the non-contiguous, empty and narrow inputs
(:255-300), plus the golden fixtures made from the reference's own
``rmsnorm_gated_reference``.  Limits are the verifier's: forward |err| fp32
2e-5, fp16 5e-3, bf16 4e-2 -- for 16-bit outputs plus half an output ulp of
|ref| (2^-9 bf16, 2^-11 fp16), since rounding an output of magnitude 8-16 to
bf16 alone errs by up to 0.03; gradients norm-relative fp32 1e-6 (1e-5 for the
widest groups, whose fp32 sums run over 16 K-40 K terms), fp16 2e-3, bf16 2e-2.
"""

import pytest
import torch

from oracle import ssm_oracle as orc

pytestmark = pytest.mark.gpu

FWD = {torch.float32: 2e-5, torch.float16: 5e-3, torch.bfloat16: 4e-2}
HALF_ULP = {torch.float32: 0.0, torch.float16: 2.0 ** -11, torch.bfloat16: 2.0 ** -9}
GRAD = {torch.float32: 1e-6, torch.float16: 2e-3, torch.bfloat16: 2e-2}


def _fwd_ok(out, ref, dtype):
    err = (out.double().cpu() - ref).abs()
    return bool((err <= FWD[dtype] + HALF_ULP[dtype] * ref.abs()).all())


def _gn():
    from metal_kernelops_b200.cv import gated_norm
    return gated_norm


def _make(shape, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(*shape, generator=g).to("cuda", dtype)


FWD_CASES = [  # shape, group_size, bias, gate, norm_before_gate, eps
    ((512, 300), None, True, True, True, 1e-5),
    ((512, 300), 60, True, True, True, 1e-5),
    ((512, 300), 100, True, True, True, 1e-6),
    ((512, 300), 150, True, True, False, 1e-5),
    ((512, 300), None, False, True, True, 1e-5),
    ((512, 300), None, True, False, True, 1e-5),
    ((512, 300), 60, True, True, False, 1e-5),
    ((512, 300), None, True, True, True, 1.0),
    ((4, 8, 300), 100, True, True, True, 1e-5),
    ((3, 5, 7, 128), 32, True, True, True, 1e-5),
    ((1, 64), 16, True, True, False, 1e-5),
    ((7, 4096), 1024, True, True, True, 1e-5),
    ((2, 3, 8192), None, True, True, True, 1e-5),
    ((64, 16384), 4096, True, True, True, 1e-5),
    ((16, 32768), None, True, True, True, 1e-5),
    ((8, 40000), 20000, True, True, False, 1e-5),
    ((256, 5120), 640, True, True, False, 1e-5),       # Mamba-2 layer (d_inner / ngroups)
]


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("idx", range(len(FWD_CASES)))
def test_forward(idx, dtype):
    shape, group, bias, gate, before, eps = FWD_CASES[idx]
    gn = _gn()
    x = _make(shape, dtype, 1)
    w = _make(shape[-1:], dtype, 2)
    b = _make(shape[-1:], dtype, 3) if bias else None
    z = _make(shape, dtype, 4) if gate else None
    out = gn.rmsnorm_gated(x, w, b, z, eps=eps, group_size=group, norm_before_gate=before)
    ref = orc.rmsnorm_gated_ref(*(t.double().cpu() if t is not None else None for t in (x, w, b, z)),
                                eps=eps, group_size=group, norm_before_gate=before)
    assert out.dtype == dtype and out.shape == x.shape
    assert _fwd_ok(out, ref, dtype)


GRAD_CASES = [  # shape, group_size, bias, gate, norm_before_gate
    ((256, 300), None, True, True, True),
    ((256, 300), 60, True, True, True),
    ((256, 300), 100, True, True, False),
    ((256, 300), None, False, True, True),
    ((256, 300), None, True, False, True),
    ((4, 6, 128), 32, True, True, False),
    ((8, 4096), 1024, True, True, True),
    ((16, 32768), None, True, True, True),
    ((8, 40000), 20000, True, True, False),
    ((512, 5120), 640, True, True, False),
]


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("idx", range(len(GRAD_CASES)))
def test_gradients(idx, dtype):
    shape, group, bias, gate, before = GRAD_CASES[idx]
    gn = _gn()
    x = _make(shape, dtype, 11).requires_grad_(True)
    w = _make(shape[-1:], dtype, 12).requires_grad_(True)
    b = _make(shape[-1:], dtype, 13).requires_grad_(True) if bias else None
    z = _make(shape, dtype, 14).requires_grad_(True) if gate else None
    out = gn.rmsnorm_gated(x, w, b, z, group_size=group, norm_before_gate=before)
    dy = _make(shape, dtype, 15)
    leaves = [t for t in (x, w, b, z) if t is not None]
    got = torch.autograd.grad(out, leaves, dy)
    ref_leaves = [t.detach().double().cpu().requires_grad_(True) for t in leaves]
    it = iter(ref_leaves)
    rx, rw = next(it), next(it)
    rb = next(it) if bias else None
    rz = next(it) if gate else None
    ref = orc.rmsnorm_gated_ref(rx, rw, rb, rz, group_size=group, norm_before_gate=before)
    want = torch.autograd.grad(ref, ref_leaves, dy.double().cpu())
    wide = (group or shape[-1]) > 16384
    tol = 1e-5 if (dtype == torch.float32 and wide) else GRAD[dtype]
    for t, g_, r_ in zip(leaves, got, want):
        assert g_.dtype == t.dtype
        rel = float((g_.double().cpu() - r_).norm() / (r_.norm() + 1e-30))
        assert rel <= tol, rel


GOLDEN = ["whole_axis", "group_60", "group_100_eps", "group_150_before", "no_bias", "no_gate",
          "group_60_before", "eps_one", "batched_3d", "batched_4d", "narrow", "wide_group"]


@pytest.mark.parametrize("case", GOLDEN)
def test_golden(golden, case):
    """The reference's own rmsnorm_gated_reference outputs (fp64), in fp32."""
    gn = _gn()
    c = golden("gated_norm")[case]
    names = [k for k in ("x", "weight", "bias", "z") if c["inputs"][k] is not None]
    dev = {k: c["inputs"][k].float().cuda().requires_grad_(True) for k in names}
    out = gn.rmsnorm_gated(dev["x"], dev["weight"], dev.get("bias"), dev.get("z"), eps=c["eps"],
                           group_size=c["group_size"], norm_before_gate=c["norm_before_gate"])
    assert float((out.double().detach().cpu() - c["out"]).abs().max()) <= 2e-5
    grads = torch.autograd.grad(out, [dev[k] for k in names], c["dy"].float().cuda())
    for k, g_ in zip(names, grads):
        want = c["grads"][k]
        assert float((g_.double().cpu() - want).norm() / want.norm()) <= 1e-6, k


def test_edge_cases():
    gn = _gn()
    base = torch.randn(64, 129, device="cuda")
    for x in (base.t(), torch.randn(64, 258, device="cuda")[:, ::2]):
        assert not x.is_contiguous()
        w = torch.randn(x.shape[-1], device="cuda")
        xg, wg = x.detach().clone().requires_grad_(True), w.detach().clone().requires_grad_(True)
        out = gn.rmsnorm_gated(xg, wg)
        ref = orc.rmsnorm_gated_ref(x.double().cpu(), w.double().cpu())
        assert float((out.double().detach().cpu() - ref).abs().max()) < 2e-5
        dy = torch.randn_like(out)
        gx, gw = torch.autograd.grad(out, (xg, wg), dy)
        rx, rw = x.double().cpu().requires_grad_(True), w.double().cpu().requires_grad_(True)
        rgx, rgw = torch.autograd.grad(orc.rmsnorm_gated_ref(rx, rw), (rx, rw), dy.double().cpu())
        assert float((gx.double().cpu() - rgx).norm() / rgx.norm()) < 1e-6
    for shape in ((0, 300), (5, 0), (0,), (2, 0, 7)):
        x = torch.empty(*shape, device="cuda")
        w = torch.empty(shape[-1] if shape else 0, device="cuda")
        out = gn.rmsnorm_gated(x, w)
        assert out.shape == x.shape and out.numel() == 0 and out.dtype == x.dtype
    for features in (1, 2, 31, 33):
        x = torch.randn(4, features, device="cuda")
        w = torch.randn(features, device="cuda")
        ref = orc.rmsnorm_gated_ref(x.double().cpu(), w.double().cpu())
        assert float((gn.rmsnorm_gated(x, w).double().cpu() - ref).abs().max()) < 2e-5
    with pytest.raises(ValueError):
        gn.rmsnorm_gated(torch.randn(4, 30, device="cuda"), torch.randn(30, device="cuda"), group_size=7)
    with pytest.raises(ValueError):
        gn.rmsnorm_gated(torch.randn(4, 30, device="cuda"), torch.randn(31, device="cuda"))
    with pytest.raises(ValueError):
        gn.rmsnorm_gated(torch.randn(4, 30), torch.randn(30))


def test_deterministic():
    gn = _gn()
    x = _make((1024, 5120), torch.bfloat16, 21)
    z = _make((1024, 5120), torch.bfloat16, 22)
    w = _make((5120,), torch.float32, 23)
    b = _make((5120,), torch.float32, 24)
    runs = []
    for _ in range(3):
        leaves = [t.clone().requires_grad_(True) for t in (x, w, b, z)]
        out = gn.rmsnorm_gated(leaves[0], leaves[1], leaves[2], leaves[3], group_size=640, norm_before_gate=False)
        runs.append((out.detach(),) + torch.autograd.grad(out.float().square().sum(), leaves))
    for vals in zip(*runs):
        assert all(torch.equal(vals[0], v) for v in vals[1:])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("norm_before_gate", [False, True])
def test_column_slices(dtype, norm_before_gate):
    """x and z as column slices of wider projection outputs (the Mamba-2 layer's
    z is such a slice) are read through their row strides, not copied: forward
    and every gradient equal the call on contiguous copies bit for bit when the
    rows keep 16-byte alignment, and match the fp64 oracle when they do not."""
    gn = _gn()
    rows, feat, group = 96, 640, 320
    for extra, exact in ((64, True), (3, False)):
        wide_x = _make((rows, feat + extra), dtype, 71)
        wide_z = _make((rows, 2 * feat + extra), dtype, 72)
        w = _make((feat,), torch.float32, 73)
        dy = _make((rows, feat), dtype, 74)
        runs = []
        for contiguous in (False, True):
            x = wide_x[:, extra // 2:extra // 2 + feat].detach()
            z = wide_z[:, feat:2 * feat].detach()
            if contiguous:
                x, z = x.contiguous(), z.contiguous()
            x.requires_grad_(True)
            z.requires_grad_(True)
            wl = w.clone().requires_grad_(True)
            out = gn.rmsnorm_gated(x, wl, z=z, group_size=group, norm_before_gate=norm_before_gate)
            out.backward(dy)
            runs.append([t.detach().clone() for t in (out, x.grad, z.grad, wl.grad)])
        if exact:
            for a_, b_ in zip(*runs):
                assert torch.equal(a_, b_)
        else:
            x = wide_x[:, extra // 2:extra // 2 + feat]
            z = wide_z[:, feat:2 * feat]
            ref = orc.rmsnorm_gated_ref(x.double().cpu(), w.double().cpu(), z=z.double().cpu(),
                                        group_size=group, norm_before_gate=norm_before_gate)
            assert _fwd_ok(runs[0][0], ref, dtype)
