"""Pin the CPU oracle to the reference's own outputs (CPU only).

The fixtures in ``tests/golden`` were produced by running the reference's
functions (``tests/golden/make_golden.py``); here the restatement in
``oracle/ssm_oracle.py`` must reproduce them, so the GPU parity tests, which
compare against the oracle, are anchored to the reference itself.
"""

import pytest
import torch
import torch.nn.functional as F

from oracle import ssm_oracle as orc

EXACT = 1e-12   # fp64 restatement vs fp64 reference: same arithmetic up to op order


def _close(got, want, tol=EXACT):
    assert got.shape == want.shape
    assert orc.max_rel(got, want) <= tol, orc.max_rel(got, want)


@pytest.mark.parametrize("case", ["config0", "grouped", "per_channel_groups", "thirty_two_states"])
def test_selective_scan_forward_and_grads(golden, case):
    c = golden("selective_scan")[case]
    inp = c["inputs"]
    names = ("u", "delta", "A", "B", "C", "D", "z", "delta_bias")
    leaves = {k: inp[k].clone().requires_grad_(True) for k in names}
    y = orc.selective_scan_ref(leaves["u"], leaves["delta"], leaves["A"], leaves["B"],
                               leaves["C"], D=leaves["D"], z=leaves["z"],
                               delta_bias=leaves["delta_bias"], delta_softplus=True)
    _close(y, c["y"])
    grads = torch.autograd.grad(y, [leaves[k] for k in names], inp["dout"])
    for k, g in zip(names, grads):
        _close(g, c["grads"][k])


@pytest.mark.parametrize("case", ["config0", "grouped"])
def test_stepwise_matches_reference_loop(golden, case):
    c = golden("selective_scan")[case]
    inp = c["inputs"]
    dt = F.softplus(inp["delta"] + inp["delta_bias"][..., None])
    y = orc.selective_scan_stepwise(inp["u"], dt, inp["A"], inp["B"], inp["C"])
    _close(y, c["y_stepwise_scan"])
    # and the functional scan agrees with the loop (reference probe: 4.4e-16)
    y2 = orc.scan_functional(inp["u"], dt, inp["A"], inp["B"], inp["C"])
    _close(y2, c["y_stepwise_scan"])


@pytest.mark.parametrize("case", ["config0", "grouped"])
def test_stepping_modes_identical(golden, case):
    """The reference's per-step indexing (timed as the CPU baseline) and the
    unbind stepping (parity) give the same output and gradients bit for bit."""
    c = golden("selective_scan")[case]
    inp = c["inputs"]
    names = ("u", "delta", "A", "B", "C", "D", "z", "delta_bias")
    runs = []
    for stepping in ("index", "unbind"):
        leaves = {k: inp[k].clone().requires_grad_(True) for k in names}
        y = orc.selective_scan_ref(leaves["u"], leaves["delta"], leaves["A"], leaves["B"], leaves["C"],
                                   D=leaves["D"], z=leaves["z"], delta_bias=leaves["delta_bias"],
                                   delta_softplus=True, stepping=stepping)
        runs.append((y,) + torch.autograd.grad(y, [leaves[k] for k in names], inp["dout"]))
    for a, b in zip(*runs):
        assert torch.equal(a, b)


def test_cumsum_kat(golden):
    c = golden("selective_scan")["cumsum_kat"]
    u = c["u"]
    y = orc.scan_functional(u, torch.ones_like(u), torch.zeros(1, 1, dtype=u.dtype),
                            torch.ones(1, 1, 1, u.shape[-1], dtype=u.dtype),
                            torch.ones(1, 1, 1, u.shape[-1], dtype=u.dtype))
    _close(y, c["y"])
    _close(y, u.cumsum(-1))


@pytest.mark.parametrize("case", ["ragged", "gqa1", "mha", "short"])
def test_ssd_reference(golden, case):
    c = golden("mamba2_chunk")[case]
    inp = c["inputs"]
    names = ("x", "dt", "A", "B", "C", "D", "z", "dt_bias", "initial_states")
    leaves = {k: inp[k].clone().requires_grad_(True) for k in names}
    y, s = orc.mamba2_chunk_scan_ref(leaves["x"], leaves["dt"], leaves["A"], leaves["B"],
                                     leaves["C"], D=leaves["D"], z=leaves["z"],
                                     dt_bias=leaves["dt_bias"], dt_softplus=True,
                                     initial_states=leaves["initial_states"])
    _close(y, c["y"])
    _close(s, c["final_state"])
    grads = torch.autograd.grad((y * c["wy"]).sum() + (s * c["ws"]).sum(),
                                [leaves[k] for k in names])
    for k, g in zip(names, grads):
        _close(g, c["grads"][k])


@pytest.mark.parametrize("case", ["ragged", "gqa1", "mha", "short"])
def test_ssd_composition_restatement(golden, case):
    c = golden("mamba2_chunk")[case]
    f32 = {k: v.float() for k, v in c["inputs"].items()}
    y, s = orc.mamba2_chunk_scan_composition(
        f32["x"], f32["dt"], f32["A"], f32["B"], f32["C"], 4, D=f32["D"], z=f32["z"],
        dt_bias=f32["dt_bias"], dt_softplus=True, initial_states=f32["initial_states"])
    _close(y, c["y_composition_f32"], 1e-6)
    _close(s, c["final_composition_f32"], 1e-6)
    # the composition itself matches the fp64 recurrence to fp32 accuracy
    _close(y, c["y"], 1e-5)


def test_ssd_defaults(golden):
    c = golden("mamba2_chunk")["defaults"]
    inp = c["inputs"]
    y, s = orc.mamba2_chunk_scan_ref(inp["x"], inp["dt"], inp["A"], inp["B"], inp["C"])
    _close(y, c["y"])
    _close(s, c["final_state"])


def test_ssd_minimal_cross_check():
    """``ssd_minimal_discrete`` agrees with the recurrence
    (verify_mamba2_chunk.py:182-234)."""
    g = lambda s: torch.Generator().manual_seed(s)  # noqa: E731
    b, l, h, p, ng, n = 1, 16, 2, 3, 1, 4
    x = torch.randn(b, l, h, p, generator=g(5), dtype=torch.float64)
    dt = F.softplus(torch.randn(b, l, h, generator=g(6), dtype=torch.float64) - 2)
    A = -torch.exp(torch.rand(h, generator=g(7), dtype=torch.float64))
    B = torch.randn(b, l, ng, n, generator=g(8), dtype=torch.float64)
    C = torch.randn(b, l, ng, n, generator=g(9), dtype=torch.float64)
    init = torch.randn(b, h, p, n, generator=g(10), dtype=torch.float64) * 0.1
    y_min, s_min = orc.ssd_minimal_discrete(x * dt.unsqueeze(-1), A * dt, B, C, 4, init[:, None])
    y_ref, s_ref = orc.mamba2_chunk_scan_ref(x, dt, A, B, C, 4, initial_states=init)
    assert orc.max_rel(y_min, y_ref) < 1e-10
    assert orc.max_rel(s_min, s_ref) < 1e-10


@pytest.mark.parametrize("case", ["decode", "batched", "dt_per_element", "head_dim_D",
                                  "no_options", "dstate_1"])
def test_decode_reference(golden, case):
    c = golden("mamba2_state")[case]
    inp = c["inputs"]
    names = ("state", "x", "dt", "A", "B", "C", "D", "z", "dt_bias")
    leaves = {k: (inp[k].clone().requires_grad_(True) if k in inp else None) for k in names}
    y, s = orc.mamba2_state_update_ref(*[leaves[k] for k in names], dt_softplus=c["softplus"])
    _close(y, c["y"])
    _close(s, c["new_state"])
    present = [k for k in names if leaves[k] is not None]
    grads = torch.autograd.grad((y * c["wy"]).sum() + (s * c["ws"]).sum(),
                                [leaves[k] for k in present])
    for k, gr in zip(present, grads):
        _close(gr, c["grads"][k])


def test_finite_differences_selective_scan():
    """fp64 central differences of the oracle (verify_path_scan.py:191-215)."""
    inp = orc.selective_scan_inputs(1, 2, 5, 3, 1, seed=13, act_dtype=torch.float64)
    inp = {k: v.double() for k, v in inp.items()}
    names = ("u", "delta", "A", "B", "C", "D", "z", "delta_bias")

    def f(**kw):
        return orc.selective_scan_ref(kw["u"], kw["delta"], kw["A"], kw["B"], kw["C"],
                                      D=kw["D"], z=kw["z"], delta_bias=kw["delta_bias"],
                                      delta_softplus=True).sum()

    leaves = {k: inp[k].clone().requires_grad_(True) for k in names}
    grads = torch.autograd.grad(f(**leaves), [leaves[k] for k in names])
    step = 1e-6
    for k, gr in zip(names, grads):
        for pick in range(min(3, inp[k].numel())):
            plus = {kk: v.clone() for kk, v in inp.items()}
            minus = {kk: v.clone() for kk, v in inp.items()}
            plus[k].reshape(-1)[pick] += step
            minus[k].reshape(-1)[pick] -= step
            num = (float(f(**plus)) - float(f(**minus))) / (2 * step)
            ana = float(gr.reshape(-1)[pick])
            assert abs(num - ana) <= 1e-6 * max(1.0, abs(num)), (k, pick, num, ana)


# ---------------------------------------------------------------------------
# VMamba four-path scan (cv/path_scan.py)
# ---------------------------------------------------------------------------

SS2D_CASES = ["fb_1x3x3x2_5x7", "fb_2x16x1x8_8x8", "fb_2x8x2x4_6x5", "five_states",
              "mean_merge", "single_row", "single_column", "thirty_two_states"]
SS2D_NAMES = ("u", "dt", "A", "B", "C")


@pytest.mark.parametrize("case", SS2D_CASES)
def test_ss2d_reference(golden, case):
    c = golden("path_scan")[case]
    leaves = [c["inputs"][k].clone().requires_grad_(True) for k in SS2D_NAMES]
    y = orc.ss2d_scan_ref(*leaves, merge=c["merge"])
    _close(y, c["y"])
    grads = torch.autograd.grad(y, leaves, c["dy"])
    for k, g in zip(SS2D_NAMES, grads):
        _close(g, c["grads"][k])


def test_ss2d_path_orders(golden):
    for (h, w), want in golden("path_scan")["orders"].items():
        got = orc.ss2d_path_orders(h, w)
        assert all(torch.equal(a, b) for a, b in zip(got, want)), (h, w)


def test_ss2d_order_cumsum_kat():
    """A = 0, dt = 1, B = C = 1 turns every path into a cumulative sum along
    its order (verify_path_scan.py:125-159); expected values from plain index
    lists."""
    for height, width in ((4, 3), (1, 6), (6, 1), (5, 5)):
        length = height * width
        g = torch.Generator().manual_seed(height * 31 + width)
        values = torch.randn(1, 1, length, generator=g, dtype=torch.float64)
        expected = torch.zeros_like(values)
        orders = [[h * width + w for h in range(height) for w in range(width)],
                  [h * width + w for w in range(width) for h in range(height)]]
        orders += [o[::-1] for o in orders]
        for order in orders:
            idx = torch.tensor(order)
            seq = values[0, 0].index_select(0, idx).cumsum(0)
            back = torch.empty_like(seq)
            back[idx] = seq
            expected[0, 0] += back
        shape = (1, 1, height, width)
        got = orc.ss2d_scan_ref(values.reshape(shape), torch.ones(shape, dtype=torch.float64),
                                torch.zeros(1, 1, dtype=torch.float64),
                                torch.ones(1, 1, 1, height, width, dtype=torch.float64),
                                torch.ones(1, 1, 1, height, width, dtype=torch.float64))
        _close(got, expected.reshape(shape), 1e-12)


def test_ss2d_matches_stepwise_loop():
    """The four-path oracle equals the triple-loop scan run on each permuted
    sequence (verify_path_scan.py:162-188)."""
    u, dt, A, B, C = orc.ss2d_inputs(2, 4, 2, 3, 3, 4, seed=7, dtype=torch.float64)
    batch, channels, height, width = u.shape
    length = height * width
    fu, fdt = u.reshape(batch, channels, length), dt.reshape(batch, channels, length)
    fb, fc = B.reshape(batch, 2, 3, length), C.reshape(batch, 2, 3, length)
    restored = []
    for order in orc.ss2d_path_orders(height, width):
        seq = orc.selective_scan_stepwise(fu.index_select(-1, order), fdt.index_select(-1, order), A,
                                          fb.index_select(-1, order).contiguous(),
                                          fc.index_select(-1, order).contiguous())
        restored.append(fu.new_zeros(batch, channels, length).index_copy(-1, order, seq))
    want = ((restored[0] + restored[2]) + (restored[1] + restored[3])).reshape(u.shape)
    _close(orc.ss2d_scan_ref(u, dt, A, B, C), want, 1e-12)


@pytest.mark.parametrize("merge", ["sum", "mean"])
def test_ss2d_finite_differences(merge):
    """fp64 central differences on a 2x2 map (verify_path_scan.py:191-215)."""
    args = orc.ss2d_inputs(1, 2, 1, 2, 2, 2, seed=13, dtype=torch.float64)
    f = lambda *a: orc.ss2d_scan_ref(*a, merge=merge)  # noqa: E731
    leaves = [t.clone().requires_grad_(True) for t in args]
    analytic = torch.autograd.grad(f(*leaves), leaves, torch.ones_like(leaves[0]))
    step = 1e-6
    for i in range(len(args)):
        for pick in range(min(3, args[i].numel())):
            plus = [t.clone() for t in args]
            minus = [t.clone() for t in args]
            plus[i].reshape(-1)[pick] += step
            minus[i].reshape(-1)[pick] -= step
            num = (float(f(*plus).sum()) - float(f(*minus).sum())) / (2 * step)
            ana = float(analytic[i].reshape(-1)[pick])
            assert abs(num - ana) <= 1e-6 * max(abs(num), 1e-9) + 1e-9, (i, pick, num, ana)


# ---------------------------------------------------------------------------
# causal depthwise conv1d (cv/causal_conv1d.py)
# ---------------------------------------------------------------------------

CONV_CASES = ["decode_1x128", "short_2x64x16", "prefill_1x8x300", "prefill_2x8x129",
              "narrow_2x8x200_k8", "k1_2x16x33", "k2_3x8x5", "short_below_taps"]
CONV_UPDATES = ["update_1x256x1", "update_8x64x1", "update_1x128x4", "update_wide_state",
                "update_q_beyond_state", "update_k1"]


@pytest.mark.parametrize("case", CONV_CASES)
def test_causal_conv1d_reference(golden, case):
    c = golden("causal_conv1d")[case]
    inp = c["inputs"]
    names = [k for k in ("x", "weight", "bias", "initial_state") if inp[k] is not None]
    leaves = {k: inp[k].clone().requires_grad_(True) for k in names}
    out, final = orc.causal_conv1d_ref(leaves["x"], leaves["weight"], leaves["bias"], c["activation"],
                                       leaves.get("initial_state"), True)
    _close(out, c["out"])
    _close(final, c["final"])
    grads = torch.autograd.grad((out * c["dout"]).sum() + (final * c["dfinal"]).sum(),
                                [leaves[k] for k in names], allow_unused=True)
    for k, g in zip(names, grads):
        _close(g if g is not None else torch.zeros_like(leaves[k]), c["grads"][k])


@pytest.mark.parametrize("case", CONV_UPDATES)
def test_causal_conv1d_update_reference(golden, case):
    c = golden("causal_conv1d")[case]
    inp = c["inputs"]
    state = inp["state"].clone()
    out = orc.causal_conv1d_update_ref(inp["x"], state, inp["weight"], inp["bias"], c["activation"])
    _close(out, c["out"])
    assert torch.equal(state, c["new_state"])


def test_causal_conv1d_steps_match_full():
    """Token-by-token and chunked decode reproduce the full-sequence forward and
    its final state (verify_causal_conv1d.py:586-617), on the oracle."""
    g = torch.Generator().manual_seed(51)
    for batch, channels, length in ((2, 64, 9), (1, 16, 17), (3, 32, 4)):
        w = torch.randn(channels, 1, 4, generator=g, dtype=torch.float64) * 0.5
        bias = torch.randn(channels, generator=g, dtype=torch.float64)
        x = torch.randn(batch, channels, length, generator=g, dtype=torch.float64)
        state = torch.randn(batch, channels, 3, generator=g, dtype=torch.float64)
        full, final = orc.causal_conv1d_ref(x, w, bias, "silu", state, True)
        st = state.clone()
        steps = torch.cat([orc.causal_conv1d_update_ref(x[..., t:t + 1], st, w, bias, "silu")
                           for t in range(length)], dim=-1)
        _close(steps, full, 1e-12)
        _close(st, final, 0.0)
        st = state.clone()
        chunks = torch.cat([orc.causal_conv1d_update_ref(x[..., i:i + 3], st, w, bias, "silu")
                            for i in range(0, length, 3)], dim=-1)
        _close(chunks, full, 1e-12)
        _close(st, final, 0.0)


def test_causal_conv1d_finite_differences():
    """fp64 central differences of all four inputs (verify_causal_conv1d.py:620-658)."""
    g = torch.Generator().manual_seed(7)
    x = torch.randn(2, 3, 7, generator=g, dtype=torch.float64)
    w = torch.randn(3, 1, 4, generator=g, dtype=torch.float64)
    bias = torch.randn(3, generator=g, dtype=torch.float64)
    state = torch.randn(2, 3, 3, generator=g, dtype=torch.float64)
    args = [x, w, bias, state]
    leaves = [t.clone().requires_grad_(True) for t in args]
    out, final = orc.causal_conv1d_ref(leaves[0], leaves[1], leaves[2], "silu", leaves[3], True)
    so, sf = torch.randn(out.shape, generator=g, dtype=torch.float64), torch.randn(final.shape, generator=g, dtype=torch.float64)
    analytic = torch.autograd.grad((out * so).sum() + (final * sf).sum(), leaves)

    def loss(a):
        o, f = orc.causal_conv1d_ref(a[0], a[1], a[2], "silu", a[3], True)
        return float((o * so).sum() + (f * sf).sum())

    eps = 1e-6
    for i, t in enumerate(args):
        num = torch.zeros_like(t)
        for k in range(t.numel()):
            plus = [a.clone() for a in args]
            minus = [a.clone() for a in args]
            plus[i].view(-1)[k] += eps
            minus[i].view(-1)[k] -= eps
            num.view(-1)[k] = (loss(plus) - loss(minus)) / (2 * eps)
        assert float((num - analytic[i]).norm() / analytic[i].norm()) < 1e-7, i


# ---------------------------------------------------------------------------
# gated RMSNorm (cv/gated_norm.py)
# ---------------------------------------------------------------------------

GN_CASES = ["whole_axis", "group_60", "group_100_eps", "group_150_before", "no_bias", "no_gate",
            "group_60_before", "eps_one", "batched_3d", "batched_4d", "narrow", "wide_group"]


@pytest.mark.parametrize("case", GN_CASES)
def test_gated_norm_reference(golden, case):
    c = golden("gated_norm")[case]
    inp = c["inputs"]
    names = [k for k in ("x", "weight", "bias", "z") if inp[k] is not None]
    leaves = {k: inp[k].clone().requires_grad_(True) for k in names}
    out = orc.rmsnorm_gated_ref(leaves["x"], leaves["weight"], leaves.get("bias"), leaves.get("z"),
                                eps=c["eps"], group_size=c["group_size"],
                                norm_before_gate=c["norm_before_gate"])
    _close(out, c["out"])
    grads = torch.autograd.grad(out, [leaves[k] for k in names], c["dy"])
    for k, g in zip(names, grads):
        _close(g, c["grads"][k])


@pytest.mark.parametrize("before", [True, False])
def test_gated_norm_finite_differences(before):
    """fp64 central differences of the oracle (verify_gated_norm.py:173-220)."""
    g = torch.Generator().manual_seed(17)
    x = torch.randn(3, 12, generator=g, dtype=torch.float64)
    w = torch.randn(12, generator=g, dtype=torch.float64)
    b = torch.randn(12, generator=g, dtype=torch.float64)
    z = torch.randn(3, 12, generator=g, dtype=torch.float64)
    args = [x, w, b, z]
    f = lambda a: orc.rmsnorm_gated_ref(a[0], a[1], a[2], a[3], group_size=4,  # noqa: E731
                                        norm_before_gate=before).square().sum()
    leaves = [t.clone().requires_grad_(True) for t in args]
    analytic = torch.autograd.grad(f(leaves), leaves)
    eps = 1e-6
    for i, t in enumerate(args):
        for k in range(0, t.numel(), 5):
            plus = [a.clone() for a in args]
            minus = [a.clone() for a in args]
            plus[i].view(-1)[k] += eps
            minus[i].view(-1)[k] -= eps
            num = (float(f(plus)) - float(f(minus))) / (2 * eps)
            ana = float(analytic[i].view(-1)[k])
            assert abs(num - ana) <= 1e-6 * max(1.0, abs(num)), (i, k, num, ana)
