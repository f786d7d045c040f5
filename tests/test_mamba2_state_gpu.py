"""Mamba-2 decode state update: CUDA kernels vs the fp64 oracle (GPU).

Mirrors the reference's verifier (benchmarks/verify_mamba2_state.py): the
17-case option matrix (:552-570) with its tolerances (fp32 1e-5, fp16 5e-3;
bf16 held to the north-star 2e-2 where the verifier allows 3e-2; forward
max|err| <= tol * max(scale, 1), gradients norm-relative),
the aliasing/``out_state`` contract and error cases (:196-264), one-output
adjoints (:169-193) and bit-determinism over 3 runs (:267-302).
"""

import pytest
import torch

from oracle import ssm_oracle as orc

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-5, torch.float16: 5e-3, torch.bfloat16: 2e-2}
NAMES = ("state", "x", "dt", "A", "B", "C", "D", "z", "dt_bias")


def _mk():
    from metal_kernelops_b200.cv import mamba2_state_update
    return mamba2_state_update


def build(batch, nheads, dim, dstate, groups, dt_per_head=False, d_kind="head", use_z=True,
          use_bias=True, dtype=torch.float32, state_scale=1.0, seed=7):
    g = torch.Generator().manual_seed(seed)
    inputs = [
        torch.randn(batch, nheads, dim, dstate, generator=g) * state_scale,
        torch.randn(batch, nheads, dim, generator=g),
        (torch.rand(batch, nheads, dim, generator=g) if dt_per_head
         else torch.rand(batch, nheads, generator=g)) * 0.2,
        -torch.rand(nheads, generator=g) - 0.05,
        torch.randn(batch, groups, dstate, generator=g),
        torch.randn(batch, groups, dstate, generator=g),
        {"none": None, "head": torch.randn(nheads, generator=g),
         "head_dim": torch.randn(nheads, dim, generator=g)}[d_kind],
        torch.randn(batch, nheads, dim, generator=g) if use_z else None,
        torch.randn(nheads, generator=g) * 0.1 if use_bias else None,
    ]
    return [None if t is None else t.to(dtype) for t in inputs]


CASES = [
    ("decode-f32", torch.float32, (1, 16, 128, 128, 1), dict(use_bias=True), True),
    ("decode-batched", torch.float32, (4, 8, 64, 64, 2), {}, False),
    ("zero-state", torch.float32, (2, 4, 32, 64, 1), dict(state_scale=0.0), False),
    ("carried-state", torch.float32, (3, 8, 16, 64, 2), {}, False),
    ("gqa-4", torch.float32, (2, 16, 32, 64, 4), {}, False),
    ("mha", torch.float32, (2, 6, 8, 16, 6), {}, False),
    ("dt-per-head", torch.float32, (2, 4, 16, 32, 2), dict(dt_per_head=False), False),
    ("dt-per-element", torch.float32, (2, 4, 16, 32, 2), dict(dt_per_head=True), False),
    ("head-dim-D", torch.float32, (2, 4, 16, 32, 2), dict(d_kind="head_dim"), False),
    ("no-D", torch.float32, (2, 4, 16, 32, 2), dict(d_kind="none"), False),
    ("no-gate", torch.float32, (2, 4, 16, 32, 2), dict(use_z=False), False),
    ("bias-softplus", torch.float32, (2, 4, 16, 32, 2), {}, True),
    ("softplus-no-bias", torch.float32, (2, 4, 16, 32, 2), dict(use_bias=False), True),
    ("dstate-1", torch.float32, (2, 4, 8, 1, 1), {}, False),
    ("f16", torch.float16, (2, 4, 16, 32, 2), {}, False),
    ("bf16", torch.bfloat16, (2, 4, 16, 32, 2), {}, False),
    ("bf16-decode", torch.bfloat16, (1, 16, 128, 128, 1), {}, False),
    ("odd-dstate", torch.float32, (2, 4, 5, 7, 2), {}, True),
    ("dstate-256", torch.float32, (1, 4, 8, 256, 1), {}, True),
]


@pytest.mark.parametrize("tag,dtype,shape,kw,softplus", CASES, ids=[c[0] for c in CASES])
def test_case(tag, dtype, shape, kw, softplus):
    upd = _mk()
    inputs = build(*shape, dtype=dtype, **kw)
    g = torch.Generator().manual_seed(99)
    wy = torch.randn(*shape[:3], generator=g, dtype=torch.float64) * 0.5
    ws = torch.randn(*shape[:4], generator=g, dtype=torch.float64) * 0.5
    truth = [None if t is None else t.double().requires_grad_(True) for t in inputs]
    want_y, want_s = orc.mamba2_state_update_ref(*truth, dt_softplus=softplus)
    ((want_y * wy).sum() + (want_s * ws).sum()).backward()
    got = [None if t is None else t.cuda().requires_grad_(True) for t in inputs]
    y, s = upd(*got, dt_softplus=softplus)
    ((y * wy.cuda().to(dtype)).sum() + (s * ws.cuda().to(dtype)).sum()).backward()
    fwd_err = max((y.detach().cpu().double() - want_y.detach()).abs().max().item(),
                  (s.detach().cpu().double() - want_s.detach()).abs().max().item())
    scale = max(want_y.abs().max().item(), want_s.abs().max().item())
    assert fwd_err <= TOL[dtype] * max(scale, 1.0), f"forward {fwd_err:.3e}"
    for name, a, b in zip(NAMES, got, truth):
        if b is None:
            continue
        assert a.grad is not None and a.grad.dtype == dtype, name
        err = (a.grad.cpu().double() - b.grad).norm().item() / max(b.grad.norm().item(), 1e-12)
        assert err <= TOL[dtype], f"d{name} {err:.3e}"


@pytest.mark.parametrize("case", ["decode", "batched", "dt_per_element", "head_dim_D",
                                  "no_options", "dstate_1"])
def test_golden_fixture(golden, case):
    upd = _mk()
    c = golden("mamba2_state")[case]
    inp = {k: v.float().cuda().requires_grad_(True) for k, v in c["inputs"].items()}
    y, s = upd(*[inp.get(k) for k in NAMES], dt_softplus=c["softplus"])
    assert orc.max_rel(y.cpu(), c["y"]) <= 1e-5
    assert orc.max_rel(s.cpu(), c["new_state"]) <= 1e-5
    ((y * c["wy"].float().cuda()).sum() + (s * c["ws"].float().cuda()).sum()).backward()
    for k, want in c["grads"].items():
        assert orc.norm_rel(inp[k].grad.cpu(), want) <= 1e-5, k


def test_contract():
    upd = _mk()
    state, x, dt, A, B, C, D, z, bias = [t.cuda() for t in build(2, 4, 6, 16, 2)]
    kept = state.clone()
    y, new_state = upd(state, x, dt, A, B, C, D, z, bias)
    assert torch.equal(state, kept)
    assert new_state.data_ptr() != state.data_ptr()
    out = torch.empty_like(state)
    _, staged = upd(state, x, dt, A, B, C, D, z, bias, out_state=out)
    assert torch.equal(out, new_state)
    assert staged.untyped_storage().data_ptr() == out.untyped_storage().data_ptr()
    assert torch.equal(state, kept)
    buf = state.clone()
    _, upd_ = upd(buf, x, dt, A, B, C, D, z, bias, out_state=buf)
    assert torch.equal(buf, new_state)
    assert upd_.untyped_storage().data_ptr() == buf.untyped_storage().data_ptr()
    # strided x/z give the same result
    wx = torch.randn(2, 4, 12, device="cuda")
    wz = torch.randn(2, 4, 12, device="cuda")
    a1 = upd(state, wx[:, :, ::2], dt, A, B, C, D, wz[:, :, ::2], bias)
    a2 = upd(state, wx[:, :, ::2].contiguous(), dt, A, B, C, D, wz[:, :, ::2].contiguous(), bias)
    assert torch.equal(a1[0], a2[0]) and torch.equal(a1[1], a2[1])


def test_in_place_with_grad():
    """``out_state`` aliasing ``state`` while other inputs need grad: the
    backward still sees the entering state."""
    upd = _mk()
    inputs = build(2, 4, 6, 16, 2)
    state = inputs[0].cuda()
    rest = [None if t is None else t.cuda().requires_grad_(True) for t in inputs[1:]]
    y, s = upd(state, *rest, out_state=state)
    (y.sum() + s.sum()).backward()
    truth = [inputs[0].double()] + [None if t is None else t.double().requires_grad_(True)
                                    for t in inputs[1:]]
    wy, wsr = orc.mamba2_state_update_ref(*truth)
    (wy.sum() + wsr.sum()).backward()
    for name, a, b in zip(NAMES[1:], rest, truth[1:]):
        if b is not None:
            assert orc.norm_rel(a.grad.cpu(), b.grad) <= 1e-5, name


def test_errors():
    upd = _mk()
    state, x, dt, A, B, C, D, z, bias = [t.cuda() for t in build(2, 4, 6, 16, 2)]
    with pytest.raises(ValueError):
        upd(*(t.cpu() for t in (state, x, dt, A, B, C)))
    with pytest.raises(ValueError):
        upd(state, x, dt, A, torch.randn(2, 3, 16, device="cuda"), torch.randn(2, 3, 16, device="cuda"))
    with pytest.raises(ValueError):
        upd(state, x, dt, A, B, C, out_state=torch.empty_like(x))
    with pytest.raises(ValueError):
        upd(state.int(), x.int(), dt.int(), A, B.int(), C.int())
    with pytest.raises(ValueError):
        upd(state, x, dt, A, B, C, out_state=torch.empty_like(state).requires_grad_(True))


@pytest.mark.parametrize("use_y,use_state", [(True, False), (False, True)])
def test_one_output_adjoint(use_y, use_state):
    upd = _mk()
    inputs = build(2, 4, 6, 16, 2)
    wy = torch.randn(2, 4, 6, dtype=torch.float64)
    wsw = torch.randn(2, 4, 6, 16, dtype=torch.float64)

    def loss(y, s, dev):
        tot = 0
        if use_y:
            tot = tot + (y * wy.to(dev, y.dtype)).sum()
        if use_state:
            tot = tot + (s * wsw.to(dev, s.dtype)).sum()
        return tot

    truth = [None if t is None else t.double().requires_grad_(True) for t in inputs]
    loss(*orc.mamba2_state_update_ref(*truth), "cpu").backward()
    got = [None if t is None else t.cuda().requires_grad_(True) for t in inputs]
    loss(*upd(*got), "cuda").backward()
    for name, a, b in zip(NAMES, got, truth):
        if b is None or b.grad is None:
            continue
        assert orc.norm_rel(a.grad.cpu(), b.grad) <= 1e-5, name


@pytest.mark.parametrize("shape", [(4, 8, 64, 64, 2), (1, 16, 128, 128, 1)])
def test_determinism(shape):
    upd = _mk()
    inputs = [None if t is None else t.cuda().requires_grad_(True) for t in build(*shape)]
    wy = torch.randn(*shape[:3], device="cuda")
    wsw = torch.randn(*shape[:4], device="cuda")
    runs = []
    for _ in range(3):
        for t in inputs:
            if t is not None:
                t.grad = None
        y, s = upd(*inputs)
        ((y * wy).sum() + (s * wsw).sum()).backward()
        runs.append([t.grad.clone() for t in inputs if t is not None])
    for vals in zip(*runs):
        assert all(torch.equal(vals[0], v) for v in vals[1:])


def test_config4_step_in_place():
    """Config 4 (B256 H80 P64 N128 G8, fp32 state, bf16 x/B/C): one in-place
    step vs the oracle on a slice of rows, plus a 4-step loop equal to 4 calls
    of the functional path."""
    upd = _mk()
    inp = orc.decode_inputs(256, 80, 64, 128, 8)
    dev = {k: v.cuda() for k, v in inp.items()}
    state = dev["state"].clone()
    y, s = upd(state, dev["x"], dev["dt"], dev["A"], dev["B"], dev["C"], D=dev["D"],
               dt_bias=dev["dt_bias"], dt_softplus=True, out_state=state)
    assert s.data_ptr() == state.data_ptr()
    b = slice(10, 12)
    want_y, want_s = orc.mamba2_state_update_ref(
        inp["state"][b].double(), inp["x"][b].double(), inp["dt"][b].double(), inp["A"].double(),
        inp["B"][b].double(), inp["C"][b].double(), D=inp["D"].double(),
        dt_bias=inp["dt_bias"].double(), dt_softplus=True)
    scale = max(want_y.abs().max().item(), want_s.abs().max().item())
    assert (s[b].cpu().double() - want_s).abs().max().item() <= 1e-5 * max(scale, 1)
    assert (y[b].float().cpu().double() - want_y).abs().max().item() <= 1e-5 * max(scale, 1)


@pytest.mark.parametrize("io", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape,use_z", [((3, 8, 16, 64, 2), True), ((2, 4, 5, 7, 2), False)],
                         ids=["vec", "odd-dstate"])
def test_io_dtype_matches_widened_inputs(io, shape, use_z):
    """16-bit x, B, C, z against an fp32 state are read as they are (no
    widening copies); widening bf16/fp16 to fp32 is exact, so the results equal
    the call on pre-widened inputs bit for bit."""
    upd = _mk()
    st, x, dt, A, B, C, D, z, bias = build(*shape, use_z=use_z)
    x, B, C = (t.to(io) for t in (x, B, C))
    z = z.to(io) if z is not None else None
    cu = [None if t is None else t.cuda() for t in (st, x, dt, A, B, C, D, z, bias)]
    wide = [None if t is None else t.float() for t in cu]
    with torch.no_grad():
        y1, s1 = upd(*cu, dt_softplus=True)
        y2, s2 = upd(*wide, dt_softplus=True)
    assert y1.dtype == torch.float32 and s1.dtype == torch.float32
    assert torch.equal(y1, y2) and torch.equal(s1, s2)
