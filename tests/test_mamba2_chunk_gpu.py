"""Mamba-2 SSD chunk scan: CUDA kernels vs the fp64 oracle (GPU).

Mirrors the reference's verifier (benchmarks/verify_mamba2_chunk.py): the
forward option matrix over 4 shapes x chunk {1, 4, 16, 64} x 3 dtypes with
every option on (:113-147), defaults and single options (:150-179), the
``ssd_minimal_discrete`` known-answer cross-check (:182-234), layout /
strided / ``initial_states`` spellings and shape errors (:237-266), and the
gradients of all 9 inputs against fp64 autograd (:269-290).  Metric:
max|err| / max|ref|; tolerances fp32 1e-5, fp16 2e-3, bf16 2e-2.
"""

import pytest
import torch
import torch.nn.functional as F

from oracle import ssm_oracle as orc

pytestmark = pytest.mark.gpu

TOL = {torch.float32: 1e-5, torch.float16: 2e-3, torch.bfloat16: 2e-2}
NAMES = ("x", "dt", "A", "B", "C", "D", "z", "dt_bias", "initial_states")


def _scan():
    from metal_kernelops_b200.cv import mamba2_chunk_scan
    return mamba2_chunk_scan


def _problem(batch, length, nheads, headdim, ngroups, dstate, seed=0, dtype=torch.float32):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(batch, length, nheads, headdim, generator=g)
    dt = torch.randn(batch, length, nheads, generator=g)
    A = -torch.exp(torch.rand(nheads, generator=g))
    B = torch.randn(batch, length, ngroups, dstate, generator=g)
    C = torch.randn(batch, length, ngroups, dstate, generator=g)
    return [t.to(dtype) for t in (x, dt, A, B, C)]


def _options(batch, length, nheads, headdim, dstate, seed=1):
    g = torch.Generator().manual_seed(seed)
    return dict(
        D=torch.randn(nheads, generator=g),
        z=torch.randn(batch, length, nheads, headdim, generator=g),
        dt_bias=torch.randn(nheads, generator=g) * 0.1,
        initial_states=torch.randn(batch, nheads, headdim, dstate, generator=g) * 0.1,
    )


SHAPES = [(2, 13, 4, 6, 2, 5), (1, 16, 4, 4, 1, 4), (2, 9, 4, 3, 4, 3), (1, 5, 2, 2, 1, 3)]


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("chunk", [1, 4, 16, 64])
@pytest.mark.parametrize("si", range(len(SHAPES)))
def test_forward_matrix(si, chunk, dtype):
    scan = _scan()
    batch, length, nheads, headdim, ngroups, dstate = SHAPES[si]
    args = [t.to("cuda", dtype) for t in _problem(*SHAPES[si], seed=si, dtype=dtype)]
    opts = {k: v.to("cuda", dtype) for k, v in
            _options(batch, length, nheads, headdim, dstate, seed=si + 10).items()}
    cpu = [t.cpu().double() for t in args]
    copt = {k: v.cpu().double() for k, v in opts.items()}
    y_ref, s_ref = orc.mamba2_chunk_scan_ref(*cpu, D=copt["D"], z=copt["z"], dt_bias=copt["dt_bias"],
                                             dt_softplus=True, initial_states=copt["initial_states"])
    y, s = scan(*args, chunk, D=opts["D"], z=opts["z"], dt_bias=opts["dt_bias"], dt_softplus=True,
                initial_states=opts["initial_states"])
    assert y.dtype == dtype and s.dtype == dtype
    assert orc.max_rel(y.float().cpu(), y_ref) <= TOL[dtype]
    assert orc.max_rel(s.float().cpu(), s_ref) <= TOL[dtype]


def test_defaults_and_single_options():
    scan = _scan()
    args = [t.cuda() for t in _problem(2, 9, 4, 6, 2, 5, seed=7)]
    cpu = [t.cpu().double() for t in args]
    opts = {k: v.cuda() for k, v in _options(2, 9, 4, 6, 5, seed=17).items()}
    y_ref, s_ref = orc.mamba2_chunk_scan_ref(*cpu)
    y, s = scan(*args, 4)
    assert orc.max_rel(y.cpu(), y_ref) <= 1e-5 and orc.max_rel(s.cpu(), s_ref) <= 1e-5
    y_ref, _ = orc.mamba2_chunk_scan_ref(*cpu, D=opts["D"].cpu().double())
    y, _ = scan(*args, 4, D=opts["D"])
    assert orc.max_rel(y.cpu(), y_ref) <= 1e-5
    dp = torch.randn(4, 6, generator=torch.Generator().manual_seed(3), dtype=torch.float64)
    y_ref, _ = orc.mamba2_chunk_scan_ref(*cpu, D=dp)
    y, _ = scan(*args, 4, D=dp.float().cuda())
    assert orc.max_rel(y.cpu(), y_ref) <= 1e-5
    y_ref, _ = orc.mamba2_chunk_scan_ref(*cpu, dt_bias=opts["dt_bias"].cpu().double())
    y, _ = scan(*args, 4, dt_bias=opts["dt_bias"])
    assert orc.max_rel(y.cpu(), y_ref) <= 1e-5
    y_ref, s_ref = orc.mamba2_chunk_scan_ref(*cpu, initial_states=opts["initial_states"].cpu().double())
    y, s = scan(*args, 4, initial_states=opts["initial_states"])
    assert orc.max_rel(y.cpu(), y_ref) <= 1e-5 and orc.max_rel(s.cpu(), s_ref) <= 1e-5


def test_ssd_minimal_known_answer():
    scan = _scan()
    g = lambda s: torch.Generator().manual_seed(s)  # noqa: E731
    b, l, h, p, ng, n = 1, 16, 2, 3, 1, 4
    x = torch.randn(b, l, h, p, generator=g(5), dtype=torch.float64)
    dt = F.softplus(torch.randn(b, l, h, generator=g(6), dtype=torch.float64) - 2)
    A = -torch.exp(torch.rand(h, generator=g(7), dtype=torch.float64))
    B = torch.randn(b, l, ng, n, generator=g(8), dtype=torch.float64)
    C = torch.randn(b, l, ng, n, generator=g(9), dtype=torch.float64)
    init = torch.randn(b, h, p, n, generator=g(10), dtype=torch.float64) * 0.1
    y_min, s_min = orc.ssd_minimal_discrete(x * dt.unsqueeze(-1), A * dt, B, C, 4, init[:, None])
    y, s = scan(*(t.float().cuda() for t in (x, dt, A, B, C)), 4, initial_states=init.float().cuda())
    assert orc.max_rel(y.cpu(), y_min) <= 1e-5
    assert orc.max_rel(s.cpu(), s_min) <= 1e-5


@pytest.mark.parametrize("case", ["ragged", "gqa1", "mha", "short"])
def test_golden_fixture(golden, case):
    """The reference's own outputs and gradients (tests/golden)."""
    scan = _scan()
    c = golden("mamba2_chunk")[case]
    inp = {k: v.float().cuda().requires_grad_(True) for k, v in c["inputs"].items()}
    y, s = scan(inp["x"], inp["dt"], inp["A"], inp["B"], inp["C"], 4, D=inp["D"], z=inp["z"],
                dt_bias=inp["dt_bias"], dt_softplus=True, initial_states=inp["initial_states"])
    assert orc.max_rel(y.cpu(), c["y"]) <= 1e-5
    assert orc.max_rel(s.cpu(), c["final_state"]) <= 1e-5
    loss = (y * c["wy"].float().cuda()).sum() + (s * c["ws"].float().cuda()).sum()
    grads = torch.autograd.grad(loss, [inp[k] for k in NAMES])
    for k, gr in zip(NAMES, grads):
        assert orc.max_rel(gr.cpu(), c["grads"][k]) <= 1e-5, k


def test_layout():
    scan = _scan()
    args = _problem(2, 13, 4, 6, 2, 5, seed=11)
    for dtype in (torch.float32, torch.float16, torch.bfloat16):
        y, s = scan(*[t.to("cuda", dtype) for t in args], 5)
        assert y.dtype == dtype and s.dtype == dtype
        assert y.shape == (2, 13, 4, 6) and s.shape == (2, 4, 6, 5)
    dev = [t.cuda() for t in args]
    wide = torch.zeros(2, 13, 4, 12, device="cuda")
    wide[:, :, :, ::2] = dev[0]
    ys, ss = scan(wide[:, :, :, ::2], *dev[1:], 5)
    yp, sp = scan(*dev, 5)
    assert torch.equal(ys, yp) and torch.equal(ss, sp)
    s0 = torch.randn(2, 4, 6, 5, generator=torch.Generator().manual_seed(12)).cuda()
    ya, _ = scan(*dev, 5, initial_states=s0)
    yb, _ = scan(*dev, 5, initial_states=s0.transpose(-1, -2))
    yc, _ = scan(*dev, 5, initial_states=s0[:, None])
    assert torch.equal(ya, yb) and torch.equal(ya, yc)
    with pytest.raises(ValueError):
        scan(*dev, 5, initial_states=torch.zeros(2, 4, 5, 5, device="cuda"))


@pytest.mark.parametrize("chunk", [1, 8, 64])
def test_gradients_all_inputs(chunk):
    """Gradients of all 9 inputs vs fp64 autograd of the recurrence
    (verify_mamba2_chunk.py:269-290)."""
    scan = _scan()
    batch, length, nheads, headdim, ngroups, dstate = 2, 21, 4, 4, 2, 5
    args = _problem(batch, length, nheads, headdim, ngroups, dstate, seed=13)
    opts = _options(batch, length, nheads, headdim, dstate, seed=14)

    def run(device, dtype, fn):
        x, dt, A, B, C = (t.to(device=device, dtype=dtype).requires_grad_(True) for t in args)
        D = opts["D"].to(device, dtype).requires_grad_(True)
        z = opts["z"].to(device, dtype).requires_grad_(True)
        bias = opts["dt_bias"].to(device, dtype).requires_grad_(True)
        init = opts["initial_states"].to(device, dtype).requires_grad_(True)
        y, s = fn(x, dt, A, B, C, chunk, D=D, z=z, dt_bias=bias, dt_softplus=True, initial_states=init)
        loss = (y * y).sum() + (s * s).sum()
        return torch.autograd.grad(loss, (x, dt, A, B, C, D, z, bias, init))

    fast = run("cuda", torch.float32, scan)
    slow = run("cpu", torch.float64, orc.mamba2_chunk_scan_ref)
    for name, gf, gs in zip(NAMES, fast, slow):
        assert orc.max_rel(gf.cpu(), gs) <= 1e-5, name


def test_gradients_per_head_D_and_half():
    scan = _scan()
    args = _problem(1, 70, 4, 8, 2, 16, seed=21)
    Dp = torch.randn(4, 8, generator=torch.Generator().manual_seed(2))
    for dtype, tol in ((torch.float32, 1e-5), (torch.bfloat16, 3e-2)):
        leaves = [t.to("cuda", dtype).requires_grad_(True) for t in args] + \
                 [Dp.to("cuda", dtype).requires_grad_(True)]
        y, s = scan(*leaves[:5], 16, D=leaves[5], dt_softplus=True)
        g = torch.autograd.grad(y.float().square().sum() + s.float().square().sum(), leaves)
        ref = [t.to(dtype).double().requires_grad_(True) for t in args] + \
              [Dp.to(dtype).double().requires_grad_(True)]
        yr, sr = orc.mamba2_chunk_scan_ref(*ref[:5], D=ref[5], dt_softplus=True)
        gr = torch.autograd.grad(yr.square().sum() + sr.square().sum(), ref)
        for a, b in zip(g, gr):
            assert orc.norm_rel(a.float().cpu(), b) <= tol


def test_deterministic_backward():
    scan = _scan()
    args = [t.cuda().requires_grad_(True) for t in _problem(2, 100, 8, 16, 2, 32, seed=4)]
    runs = []
    for _ in range(3):
        y, s = scan(*args, 32, dt_softplus=True)
        runs.append(torch.autograd.grad(y.sum() + s.sum(), args))
    for vals in zip(*runs):
        assert all(torch.equal(vals[0], v) for v in vals[1:])


def test_config3_prefix_full_size():
    """Config 3 shape at full size (B8 L8192 H80 P64 N128 G8, bf16): the
    output on a batch row / one group's heads / the first 512 steps matches the
    oracle (the scan is causal and heads of a group are independent given
    B, C), and a run on that prefix gives the prefix's final state."""
    scan = _scan()
    inp = orc.ssd_inputs(8, 8192, 80, 64, 128, 8)
    dev = {k: v.cuda() for k, v in inp.items()}
    y, s = scan(dev["x"], dev["dt"], dev["A"], dev["B"], dev["C"], 256, D=dev["D"],
                dt_bias=dev["dt_bias"], dt_softplus=True)
    assert torch.isfinite(y.float()).all() and torch.isfinite(s.float()).all()
    b, L, hs = 5, 512, slice(10, 20)      # group 1 holds heads 10..19
    sl = dict(x=inp["x"][b:b + 1, :L, hs], dt=inp["dt"][b:b + 1, :L, hs], A=inp["A"][hs],
              B=inp["B"][b:b + 1, :L, 1:2], C=inp["C"][b:b + 1, :L, 1:2], D=inp["D"][hs],
              dt_bias=inp["dt_bias"][hs])
    yr, sr = orc.mamba2_chunk_scan_ref(sl["x"].double(), sl["dt"].double(), sl["A"].double(),
                                       sl["B"].double(), sl["C"].double(), D=sl["D"].double(),
                                       dt_bias=sl["dt_bias"].double(), dt_softplus=True)
    assert orc.max_rel(y[b:b + 1, :L, hs].float().cpu(), yr) <= 2e-2
    yp, sp = scan(*(sl[k].cuda() for k in ("x", "dt", "A", "B", "C")), 256, D=sl["D"].cuda(),
                  dt_bias=sl["dt_bias"].cuda(), dt_softplus=True)
    assert orc.max_rel(sp.float().cpu(), sr) <= 2e-2
