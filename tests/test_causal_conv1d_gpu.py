"""Causal depthwise conv1d on the GPU vs the fp64 oracle.

Mirrors the reference's verifier (benchmarks/verify_causal_conv1d.py): its
forward/gradient cases (:171-182) and update cases (:185-193) at their sizes,
its semantic checks (:454-583), step parity of the decode kernel against the
full forward (:586-617), plus the golden fixtures made from the reference's own
``causal_conv1d_ref``.  Metric: norm-relative error (the verifier's
``rel_error``); limits are the verifier's: values fp32 1e-6, fp16 3e-3,
gradients fp32 1e-5, fp16 3e-2; bfloat16 2e-2 / 3e-2.
"""

import pytest
import torch

from oracle import ssm_oracle as orc

pytestmark = pytest.mark.gpu

VALUE = {torch.float32: 1e-6, torch.float16: 3e-3, torch.bfloat16: 2e-2}
GRAD = {torch.float32: 1e-5, torch.float16: 3e-2, torch.bfloat16: 3e-2}


def _cc():
    from metal_kernelops_b200.cv import causal_conv1d
    return causal_conv1d


def _rel(got, want):
    got, want = got.detach().double().cpu(), want.detach().double().cpu()
    den = float(want.norm())
    if den == 0.0:
        return 0.0 if float(got.norm()) == 0.0 else float("inf")
    return float((got - want).norm()) / den


def _make(shape, dtype, seed, scale=1.0, device="cuda"):
    g = torch.Generator().manual_seed(seed)
    return (torch.randn(shape, generator=g, dtype=torch.float64) * scale).to(device, dtype)


CASES = [  # name, batch, channels, length, K, activation, initial state, dtype
    ("decode-1x2048", 1, 2048, 1, 4, "silu", True, torch.float32),
    ("decode-8x2048", 8, 2048, 1, 4, "silu", True, torch.float32),
    ("decode-16x1536-fp16", 16, 1536, 1, 4, "silu", True, torch.float16),
    ("short-2x256x16", 2, 256, 16, 4, "silu", False, torch.float32),
    ("prefill-1x768x4096", 1, 768, 4096, 4, "silu", True, torch.float32),
    ("prefill-8x512x2048", 8, 512, 2048, 4, "silu", False, torch.float32),
    ("prefill-16x768x1024-fp16", 16, 768, 1024, 4, "silu", True, torch.float16),
    ("narrow-4x128x200-k8", 4, 128, 200, 8, None, False, torch.float32),
    ("k1-2x64x33", 2, 64, 33, 1, None, True, torch.float32),
    ("prefill-4x256x1000-bf16", 4, 256, 1000, 4, "silu", True, torch.bfloat16),
    ("odd-length-3x40x777", 3, 40, 777, 3, "silu", True, torch.float32),
    ("long-rows-1x4x50000", 1, 4, 50000, 4, "silu", True, torch.float32),
]


@pytest.mark.parametrize("case", CASES, ids=[c[0] for c in CASES])
def test_forward_and_gradients(case):
    name, b, c, l, k, act, has_state, dtype = case
    cc = _cc()
    w = _make((c, 1, k), dtype, 1, 0.5)
    bias = _make((c,), dtype, 2)
    x = _make((b, c, l), dtype, 3)
    state = _make((b, c, k - 1), dtype, 4) if has_state else None
    leaves = [t.clone().requires_grad_(True) if t is not None else None for t in (x, w, bias, state)]
    out, final = cc.causal_conv1d_fn(leaves[0], leaves[1], leaves[2], act, leaves[3], True)
    ref_leaves = [t.double().cpu().requires_grad_(True) if t is not None else None for t in (x, w, bias, state)]
    rout, rfinal = orc.causal_conv1d_ref(ref_leaves[0], ref_leaves[1], ref_leaves[2], act, ref_leaves[3], True)
    assert out.dtype == dtype and final.shape == rfinal.shape
    assert _rel(out, rout) <= VALUE[dtype], _rel(out, rout)
    assert _rel(final, rfinal) <= VALUE[dtype]
    g = torch.Generator().manual_seed(5)
    dout = torch.randn(out.shape, generator=g, dtype=torch.float64)
    dfinal = torch.randn(final.shape, generator=g, dtype=torch.float64)
    used = [i for i, t in enumerate(leaves) if t is not None]
    fast = torch.autograd.grad((out.double() * dout.cuda()).sum() + (final.double() * dfinal.cuda()).sum(),
                               [leaves[i] for i in used], allow_unused=True)
    slow = torch.autograd.grad((rout * dout).sum() + (rfinal * dfinal).sum(),
                               [ref_leaves[i] for i in used], allow_unused=True)
    for i, a, r in zip(used, fast, slow):
        a = a if a is not None else torch.zeros_like(leaves[i])
        r = r if r is not None else torch.zeros_like(ref_leaves[i])
        assert a.dtype == leaves[i].dtype
        assert _rel(a, r) <= GRAD[dtype], (("x", "weight", "bias", "initial_state")[i], _rel(a, r))


GOLDEN = ["decode_1x128", "short_2x64x16", "prefill_1x8x300", "prefill_2x8x129",
          "narrow_2x8x200_k8", "k1_2x16x33", "k2_3x8x5", "short_below_taps"]


@pytest.mark.parametrize("case", GOLDEN)
def test_golden(golden, case):
    """The reference's own causal_conv1d_ref outputs (fp64), reproduced in fp32."""
    cc = _cc()
    c = golden("causal_conv1d")[case]
    inp = c["inputs"]
    names = [k for k in ("x", "weight", "bias", "initial_state") if inp[k] is not None]
    dev = {k: inp[k].float().cuda().requires_grad_(True) for k in names}
    out, final = cc.causal_conv1d_fn(dev["x"], dev["weight"], dev["bias"], c["activation"],
                                     dev.get("initial_state"), True)
    assert _rel(out, c["out"]) <= 1e-6
    assert _rel(final, c["final"]) <= 1e-6
    grads = torch.autograd.grad((out * c["dout"].float().cuda()).sum() + (final * c["dfinal"].float().cuda()).sum(),
                                [dev[k] for k in names], allow_unused=True)
    for k, gr in zip(names, grads):
        gr = gr if gr is not None else torch.zeros_like(dev[k])
        assert _rel(gr, c["grads"][k]) <= 1e-5, k


UPDATES = ["update_1x256x1", "update_8x64x1", "update_1x128x4", "update_wide_state",
           "update_q_beyond_state", "update_k1"]


@pytest.mark.parametrize("case", UPDATES)
def test_update_golden(golden, case):
    cc = _cc()
    c = golden("causal_conv1d")[case]
    inp = c["inputs"]
    state = inp["state"].float().cuda()
    out = cc.causal_conv1d_update(inp["x"].float().cuda(), state, inp["weight"].float().cuda(),
                                  inp["bias"].float().cuda(), c["activation"])
    assert _rel(out, c["out"]) <= 1e-6
    assert _rel(state, c["new_state"]) <= 1e-7


@pytest.mark.parametrize("case", [
    ("update-64x2048x1", 64, 2048, 1, 4, "silu", 3, torch.float32),
    ("update-1x2048x4", 1, 2048, 4, 4, "silu", 3, torch.float32),
    ("update-8x2048x1-wide", 8, 2048, 1, 4, "silu", 8, torch.float32),
    ("update-16x1536x1-fp16", 16, 1536, 1, 4, "silu", 3, torch.float16),
    ("update-4x512x2-bf16", 4, 512, 2, 4, None, 5, torch.bfloat16),
], ids=lambda c: c[0])
def test_update_cases(case):
    name, b, c, q, k, act, cols, dtype = case
    cc = _cc()
    w = _make((c, 1, k), dtype, 11, 0.5)
    bias = _make((c,), dtype, 12)
    x = _make((b, c, q), dtype, 13)
    state = _make((b, c, cols), dtype, 14)
    ref_state = state.double().cpu()
    want = orc.causal_conv1d_update_ref(x.double().cpu(), ref_state, w.double().cpu(), bias.double().cpu(), act)
    out = cc.causal_conv1d_update(x, state, w, bias, act)
    assert out.dtype == dtype
    assert _rel(out, want) <= VALUE[dtype]
    assert _rel(state, ref_state) <= VALUE[dtype]


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
def test_step_parity(dtype):
    """Token-by-token and chunked decode reproduce the full forward and its
    final state (verify_causal_conv1d.py:586-617)."""
    cc = _cc()
    tol = VALUE[dtype] if dtype == torch.float16 else 1e-6
    for b, c, l in ((2, 64, 9), (1, 256, 17), (3, 32, 4)):
        w = _make((c, 1, 4), dtype, 51, 0.5)
        bias = _make((c,), dtype, 52)
        x = _make((b, c, l), dtype, 53)
        state = _make((b, c, 3), dtype, 54)
        full, final = cc.causal_conv1d_fn(x, w, bias, "silu", state, True)
        st = state.clone()
        steps = torch.stack([cc.causal_conv1d_update(x[..., t], st, w, bias, "silu") for t in range(l)], dim=-1)
        assert _rel(steps, full) <= tol and _rel(st, final) <= tol
        st = state.clone()
        chunks = torch.cat([cc.causal_conv1d_update(x[..., i:i + 3], st, w, bias, "silu")
                            for i in range(0, l, 3)], dim=-1)
        assert _rel(chunks, full) <= tol and _rel(st, final) <= tol


def test_semantics():
    """The reference verifier's semantic checks (verify_causal_conv1d.py:454-583)."""
    cc = _cc()
    # empty sequence: no convolution, the state passes through
    w = _make((8, 1, 4), torch.float32, 31)
    state = _make((2, 8, 3), torch.float32, 32)
    out, final = cc.causal_conv1d_fn(torch.empty(2, 8, 0, device="cuda"), w, None, "silu", state, True)
    assert tuple(out.shape) == (2, 8, 0) and torch.equal(final, state)
    buf = _make((2, 8, 3), torch.float32, 33)
    before = buf.clone()
    cc.causal_conv1d_update(torch.empty(2, 8, 0, device="cuda"), buf, w)
    assert torch.equal(buf, before)
    # one token without a state sees only the last tap
    x = _make((1, 4, 1), torch.float32, 34)
    w = _make((4, 1, 4), torch.float32, 35, 0.5)
    assert _rel(cc.causal_conv1d_fn(x, w, None, None), x * w[:, 0, 3].view(1, 4, 1)) < 1e-6
    # K = 1: a scaled copy, empty final state
    w = _make((4, 1, 1), torch.float32, 36, 0.5)
    x = _make((2, 4, 7), torch.float32, 37)
    out, final = cc.causal_conv1d_fn(x, w, None, None, None, True)
    assert _rel(out, x * w[:, 0, 0].view(1, 4, 1)) < 1e-6 and tuple(final.shape) == (2, 4, 0)
    # non-contiguous and strided inputs
    w = _make((16, 1, 4), torch.float32, 38, 0.5)
    tr = _make((2, 40, 16), torch.float32, 39).transpose(1, 2)
    assert _rel(cc.causal_conv1d_fn(tr, w, None, "silu"),
                orc.causal_conv1d_ref(tr.cpu().double(), w.cpu().double(), None, "silu")) < 1e-6
    sl = _make((2, 16, 64), torch.float32, 40)[..., 1::2]
    assert _rel(cc.causal_conv1d_fn(sl, w, None, None),
                orc.causal_conv1d_ref(sl.cpu().double(), w.cpu().double(), None, None)) < 1e-6
    # (C, 1, K) and (C, K) weights are the same convolution
    x = _make((2, 16, 40), torch.float32, 42)
    assert torch.equal(cc.causal_conv1d_fn(x, w, None, "silu"), cc.causal_conv1d_fn(x, w[:, 0, :], None, "silu"))
    # a state that is a slice of a larger cache is read and written in place
    cache = _make((2, 16, 9), torch.float32, 43)
    view = cache[..., :3]
    x = _make((2, 16), torch.float32, 44)
    expected = cache.double().cpu().clone()
    before = cache.clone()
    want = orc.causal_conv1d_update_ref(x.double().cpu().unsqueeze(-1), expected[..., :3], w.double().cpu(),
                                        None, "silu").squeeze(-1)
    out = cc.causal_conv1d_update(x, view, w, None, "silu")
    assert out.shape == (2, 16)
    assert not torch.equal(cache[..., :3], before[..., :3]) and torch.equal(cache[..., 3:], before[..., 3:])
    assert _rel(out, want) < 1e-6 and _rel(cache[..., :3], expected[..., :3]) < 1e-6
    # decode carries no autograd
    with pytest.raises(RuntimeError):
        cc.causal_conv1d_update(_make((2, 16), torch.float32, 46).requires_grad_(True),
                                _make((2, 16, 3), torch.float32, 47), w)
    # mixed dtypes: result in x.dtype, gradients in each input's dtype
    wm = _make((8, 1, 4), torch.float32, 52, 0.5).requires_grad_(True)
    xm = _make((2, 8, 12), torch.float16, 53).requires_grad_(True)
    out = cc.causal_conv1d_fn(xm, wm, None, "silu")
    out.float().sum().backward()
    ref = orc.causal_conv1d_ref(xm.detach().cpu().double(), wm.detach().cpu().double(), None, "silu")
    assert out.dtype == torch.float16 and xm.grad.dtype == torch.float16 and wm.grad.dtype == torch.float32
    assert _rel(out, ref) < 3e-3


def test_contract_errors():
    cc = _cc()
    x = _make((2, 8, 16), torch.float32, 1)
    w = _make((8, 1, 4), torch.float32, 2)
    with pytest.raises(NotImplementedError):
        cc.causal_conv1d_fn(x, w, None, "relu")
    with pytest.raises(ValueError):
        cc.causal_conv1d_fn(x, _make((8, 2, 4), torch.float32, 3))
    with pytest.raises(ValueError):
        cc.causal_conv1d_fn(x[0], w)
    with pytest.raises(ValueError):
        cc.causal_conv1d_fn(x, _make((4, 1, 4), torch.float32, 3))
    with pytest.raises(ValueError):
        cc.causal_conv1d_fn(x, w, _make((4,), torch.float32, 3))
    with pytest.raises(ValueError):
        cc.causal_conv1d_fn(x, w, None, None, _make((2, 8, 2), torch.float32, 3))
    with pytest.raises(ValueError):
        cc.causal_conv1d_update(x[..., :1], _make((2, 8, 2), torch.float32, 3), w)
    with pytest.raises(ValueError):
        cc.causal_conv1d_update(x[..., :1], _make((2, 3, 8), torch.float32, 3).transpose(1, 2), w)
    with pytest.raises(ValueError):
        cc.causal_conv1d_fn(x.cpu(), w.cpu())


def test_deterministic():
    cc = _cc()
    x = _make((4, 96, 3000), torch.bfloat16, 61)
    w = _make((96, 1, 4), torch.float32, 62, 0.5)
    bias = _make((96,), torch.float32, 63)
    st = _make((4, 96, 3), torch.bfloat16, 64)
    runs = []
    for _ in range(3):
        leaves = [t.clone().requires_grad_(True) for t in (x, w, bias, st)]
        out = cc.causal_conv1d_fn(*leaves[:3], "silu", leaves[3])
        runs.append((out.detach(),) + torch.autograd.grad(out.float().square().sum(), leaves))
    for vals in zip(*runs):
        assert all(torch.equal(vals[0], v) for v in vals[1:])


CL_CASES = [  # name, batch, channels, length, K, activation, dtype, extra columns of the wider rows
    ("cl-bf16-2x256x1000-k4", 2, 256, 1000, 4, "silu", torch.bfloat16, 40),
    ("cl-f32-3x40x777-k3", 3, 40, 777, 3, "silu", torch.float32, 4),
    ("cl-unaligned-f32-2x40x300-k4", 2, 40, 300, 4, "silu", torch.float32, 6),  # 12-byte offset: copied
    ("cl-f16-1x128x70-k8", 1, 128, 70, 8, None, torch.float16, 8),
    ("cl-f32-2x64x33-k1", 2, 64, 33, 1, None, torch.float32, 0),
    ("cl-bf16-4x136x3-k4", 4, 136, 3, 4, "silu", torch.bfloat16, 16),       # shorter than the taps
    ("cl-bf16-2x512x1100-k2", 2, 512, 1100, 2, "silu", torch.bfloat16, 64),   # runs across row blocks
]


@pytest.mark.parametrize("case", CL_CASES, ids=[c[0] for c in CL_CASES])
def test_channel_last(case):
    """x as the transpose of a column slice of wider (batch, length, columns)
    rows -- a Mamba block's in-projection output -- is read in place by the
    channel-last kernels: out equals the contiguous call bit for bit (same tap
    order and activation), dx too where that call takes the bulk path (the
    unaligned-row path's 16-bit SiLU' rounds differently), and every value and
    gradient matches the fp64 oracle."""
    name, b, c, l, k, act, dtype, extra = case
    cc = _cc()
    w = _make((c, 1, k), dtype, 11, 0.5)
    bias = _make((c,), dtype, 12)
    wide = _make((b, l, c + extra), dtype, 13)
    g = torch.Generator().manual_seed(14)
    dout = torch.randn((b, c, l), generator=g, dtype=torch.float64)
    runs = []
    for contiguous in (False, True):
        x = wide[:, :, extra // 2:extra // 2 + c].transpose(1, 2).detach()
        if contiguous:
            x = x.contiguous()
        x.requires_grad_(True)
        wl, bl = w.clone().requires_grad_(True), bias.clone().requires_grad_(True)
        out = cc.causal_conv1d_fn(x, wl, bl, act)
        if not contiguous:                          # channel-last result unless the slice is misaligned
            assert (out.stride(1) == 1) == ((extra // 2 * wide.element_size()) % 8 == 0)
        grads = torch.autograd.grad((out.double() * dout.cuda()).sum(), [x, wl, bl])
        runs.append((out.detach(), *grads))
    assert torch.equal(runs[0][0], runs[1][0])
    if (l * wide.element_size()) % 16 == 0:
        assert torch.equal(runs[0][1], runs[1][1])
    x64 = wide[:, :, extra // 2:extra // 2 + c].transpose(1, 2).double().cpu().requires_grad_(True)
    w64, b64 = w.double().cpu().requires_grad_(True), bias.double().cpu().requires_grad_(True)
    rout = orc.causal_conv1d_ref(x64, w64, b64, act)
    rgrads = torch.autograd.grad((rout * dout).sum(), [x64, w64, b64])
    assert _rel(runs[0][0], rout) <= VALUE[dtype]
    for name_, a, r in zip(("x", "weight", "bias"), runs[0][1:], rgrads):
        assert _rel(a, r) <= GRAD[dtype], (name_, _rel(a, r))
