"""Mamba-1 selective scan: CUDA kernels vs the fp64 oracle (GPU).

Oracle: ``oracle.selective_scan_ref`` (the reference's ``_scan_reference`` of
cv/path_scan.py:579-605 wrapped in the epilogue of scan.py:311-320), evaluated
in float64 on the same rounded inputs, with autograd for the gradients.
Metrics follow the reference's verifiers: forward max|err|/max|ref|,
gradients norm-relative.  Tolerances: fp32 forward
1e-5, fp32 gradients 1e-4, bf16/fp16 inputs 2e-2.
"""

import pytest
import torch

from oracle import ssm_oracle as orc

pytestmark = pytest.mark.gpu

FWD_TOL = {torch.float32: 1e-5, torch.bfloat16: 2e-2, torch.float16: 2e-2}
GRAD_TOL = {torch.float32: 1e-4, torch.bfloat16: 2e-2, torch.float16: 2e-2}
NAMES = ("u", "delta", "A", "B", "C", "D", "z", "delta_bias")


def _mk():
    import metal_kernelops_b200 as mk
    return mk


def _run_pair(inp, dtype, opts=("D", "z", "delta_bias"), softplus=True, grads=True):
    """Run the CUDA op and the fp64 oracle on the same rounded inputs."""
    mk = _mk()
    use = {k: inp[k] for k in NAMES if k in ("u", "delta", "A", "B", "C") or k in opts}
    dev = {k: v.cuda().requires_grad_(grads) for k, v in use.items()}
    ref = {k: v.double().requires_grad_(grads) for k, v in use.items()}
    y = mk.selective_scan(dev["u"], dev["delta"], dev["A"], dev["B"], dev["C"], D=dev.get("D"),
                          z=dev.get("z"), delta_bias=dev.get("delta_bias"),
                          delta_softplus=softplus)
    yr = orc.selective_scan_ref(ref["u"], ref["delta"], ref["A"], ref["B"], ref["C"],
                                D=ref.get("D"), z=ref.get("z"), delta_bias=ref.get("delta_bias"),
                                delta_softplus=softplus)
    assert y.dtype == inp["u"].dtype and y.shape == inp["u"].shape
    assert torch.isfinite(y).all()
    err = orc.max_rel(y.float().cpu(), yr)
    assert err <= FWD_TOL[dtype], f"forward rel {err:.3e}"
    if not grads:
        return
    dout = inp["dout"]
    keys = list(use)
    g = torch.autograd.grad(y, [dev[k] for k in keys], dout.cuda())
    gr = torch.autograd.grad(yr, [ref[k] for k in keys], dout.double())
    for k, a, b in zip(keys, g, gr):
        assert a.dtype == dev[k].dtype, k
        e = orc.norm_rel(a.float().cpu(), b)
        assert e <= GRAD_TOL[dtype], f"d{k} rel {e:.3e}"


@pytest.mark.parametrize("shape", [
    (2, 8, 64, 16, 1),      # config 0
    (2, 8, 24, 5, 2),       # grouped, odd dstate
    (1, 4, 9, 3, 4),        # one channel per group
    (1, 4, 11, 32, 2),      # 32 states
    (1, 6, 37, 64, 3),      # 64 states
    (3, 16, 63, 8, 4),      # L not a multiple of the chunk
    (1, 1, 1, 16, 1),       # single step, single channel
    (2, 130, 100, 16, 1),   # several channel tiles, ragged last tile
    (1, 64, 300, 4, 2),     # dstate 4, many chunks
    (1, 16384, 40, 16, 1),  # 16384 rows: backward launch shape 8 states x 2 lanes
    (2, 12800, 37, 16, 2),  # 25600 rows: forward and backward 8 x 2, ragged chunk
])
def test_fp32_parity(shape):
    b, d, l, n, g = shape
    inp = orc.selective_scan_inputs(b, d, l, n, g, seed=11 + l)
    _run_pair(inp, torch.float32)


@pytest.mark.parametrize("opts,softplus", [
    ((), False), (("D",), False), (("z",), True), (("delta_bias",), False),
    (("delta_bias",), True), (("D", "z"), False),
])
def test_option_matrix(opts, softplus):
    inp = orc.selective_scan_inputs(2, 12, 45, 16, 2, seed=5)
    if not softplus:
        # without the softplus, delta must itself be a positive step size, as in
        # the reference's verifier inputs (dt = 0.05 + 0.2 * U, verify_path_scan.py:72)
        inp["delta"] = inp["delta"].abs() * 0.4 + 0.05
        inp["delta_bias"] = inp["delta_bias"].abs() * 0.01
    _run_pair(inp, torch.float32, opts=opts, softplus=softplus)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_half_parity(dtype):
    inp = orc.selective_scan_inputs(2, 40, 150, 16, 1, seed=21, act_dtype=dtype)
    _run_pair(inp, dtype)


@pytest.mark.parametrize("case", ["config0", "grouped", "per_channel_groups", "thirty_two_states"])
def test_golden_fixture(golden, case):
    """The reference's own outputs (tests/golden) reproduced from fp32 inputs."""
    mk = _mk()
    c = golden("selective_scan")[case]
    inp = {k: v.float() for k, v in c["inputs"].items()}
    dev = {k: inp[k].cuda().requires_grad_(True) for k in NAMES}
    y = mk.selective_scan(dev["u"], dev["delta"], dev["A"], dev["B"], dev["C"], D=dev["D"],
                          z=dev["z"], delta_bias=dev["delta_bias"], delta_softplus=True)
    assert orc.max_rel(y.cpu(), c["y"]) <= 1e-5
    g = torch.autograd.grad(y, [dev[k] for k in NAMES], inp["dout"].cuda())
    for k, a in zip(NAMES, g):
        assert orc.norm_rel(a.cpu(), c["grads"][k]) <= 1e-4, k


def test_cumsum_kat(golden):
    mk = _mk()
    c = golden("selective_scan")["cumsum_kat"]
    u = c["u"].float().cuda()
    L = u.shape[-1]
    y = mk.scan_cuda(u, torch.ones_like(u), torch.zeros(1, 1, device="cuda"),
                     torch.ones(1, 1, 1, L, device="cuda"), torch.ones(1, 1, 1, L, device="cuda"))
    assert orc.max_rel(y.cpu(), c["y"]) <= 1e-6


def test_degenerate_shapes():
    mk = _mk()
    for b, d, l, n, g in [(0, 4, 5, 3, 1), (1, 4, 0, 3, 1), (2, 0, 5, 3, 1)]:
        inp = orc.selective_scan_inputs(max(b, 1), max(d, 1), max(l, 1), n, 1, seed=3)
        u = torch.zeros(b, d, l, device="cuda", requires_grad=True)
        dt = torch.zeros(b, d, l, device="cuda", requires_grad=True)
        A = torch.zeros(d, n, device="cuda", requires_grad=True)
        B = torch.zeros(b, g if d else 1, n, l, device="cuda", requires_grad=True)
        C = torch.zeros_like(B, requires_grad=True)
        y = mk.selective_scan(u, dt, A, B, C)
        assert y.shape == (b, d, l)
        grads = torch.autograd.grad(y.sum(), [u, dt, A, B, C], allow_unused=True)
        assert all(gr is None or (gr == 0).all() for gr in grads)
        del inp


def test_deterministic_backward():
    mk = _mk()
    inp = orc.selective_scan_inputs(2, 256, 200, 16, 1, seed=9)
    dev = {k: inp[k].cuda().requires_grad_(True) for k in NAMES}
    runs = []
    for _ in range(3):
        y = mk.selective_scan(dev["u"], dev["delta"], dev["A"], dev["B"], dev["C"], D=dev["D"],
                              z=dev["z"], delta_bias=dev["delta_bias"], delta_softplus=True)
        runs.append(torch.autograd.grad(y, [dev[k] for k in NAMES], inp["dout"].cuda()))
    for k, *vals in zip(NAMES, *runs):
        assert all(torch.equal(vals[0], v) for v in vals[1:]), k


def test_inference_saves_nothing():
    mk = _mk()
    inp = orc.selective_scan_inputs(1, 8, 40, 16, 1, seed=4)
    with torch.no_grad():
        y = mk.selective_scan(*(inp[k].cuda() for k in ("u", "delta", "A", "B", "C")),
                              D=inp["D"].cuda(), delta_softplus=True)
    assert y.shape == (1, 8, 40)


def _slice_oracle(inp, rows, ch, dout):
    """fp64 oracle of the channels ``ch`` over the batch rows ``rows``
    (channels are independent given B and C): y and every input gradient."""
    sl = {"u": inp["u"][rows, ch], "delta": inp["delta"][rows, ch], "A": inp["A"][ch],
          "B": inp["B"][rows], "C": inp["C"][rows], "D": inp["D"][ch],
          "z": inp["z"][rows, ch], "delta_bias": inp["delta_bias"][ch]}
    ref = {k: v.double().requires_grad_(True) for k, v in sl.items()}
    yr = orc.selective_scan_ref(ref["u"], ref["delta"], ref["A"], ref["B"], ref["C"], D=ref["D"],
                                z=ref["z"], delta_bias=ref["delta_bias"], delta_softplus=True)
    gr = torch.autograd.grad(yr, [ref[k] for k in NAMES], dout[rows, ch].double())
    return yr.detach(), dict(zip(NAMES, gr))


def _full_size_check(inp, ch, prefix_row, prefix_len, lean=False):
    """Forward and backward of a full-size bf16 problem on the GPU, then:

    * y, du, ddelta, dz of the channels ``ch`` over every batch row, and the
      shared-parameter gradients dA, dD, d delta_bias of those channels (the
      values the multi-GPU all-reduce sums), against the fp64 oracle of that
      channel slice over all rows;
    * dB and dC -- sums over every channel -- through a second backward of the
      same forward whose upstream gradient is zero except on batch row
      ``prefix_row`` for its first ``prefix_len`` steps: the scan is causal, so
      those gradients equal the oracle's on that row's prefix over all
      channels, and every other gradient entry is zero."""
    mk = _mk()
    from metal_kernelops_b200 import scan as scan_mod
    dev = {k: inp[k].cuda().requires_grad_(True) for k in NAMES}
    prev = scan_mod.set_lean_backward(lean)
    try:
        y = mk.selective_scan(dev["u"], dev["delta"], dev["A"], dev["B"], dev["C"], D=dev["D"],
                              z=dev["z"], delta_bias=dev["delta_bias"], delta_softplus=True)
    finally:
        scan_mod.set_lean_backward(prev)
    assert torch.isfinite(y).all()
    g = torch.autograd.grad(y, [dev[k] for k in NAMES], inp["dout"].cuda(), retain_graph=True)
    grads = dict(zip(NAMES, g))
    for k, v in grads.items():
        assert torch.isfinite(v.float()).all(), k
    rows = slice(0, inp["u"].shape[0])
    yr, gr = _slice_oracle(inp, rows, ch, inp["dout"])
    assert orc.max_rel(y[rows, ch].float().cpu(), yr) <= 2e-2
    for k in ("u", "delta", "z"):
        assert orc.norm_rel(grads[k][rows, ch].float().cpu(), gr[k]) <= 2e-2, k
    for k in ("A", "D", "delta_bias"):
        assert orc.norm_rel(grads[k][ch].float().cpu(), gr[k]) <= 2e-2, k

    mask = torch.zeros_like(inp["dout"])
    b, t = prefix_row, prefix_len
    mask[b, :, :t] = inp["dout"][b, :, :t]
    g2 = dict(zip(NAMES, torch.autograd.grad(y, [dev[k] for k in NAMES], mask.cuda())))
    pre = {k: (v[b:b + 1, ..., :t] if k in ("u", "delta", "z", "B", "C") else v) for k, v in inp.items()}
    pre["dout"] = inp["dout"][b:b + 1, :, :t]
    _, gp = _slice_oracle(pre, slice(0, 1), slice(None), pre["dout"])
    for k in ("B", "C", "u", "delta", "z"):
        got = g2[k][b:b + 1, ..., :t].float().cpu()
        assert orc.norm_rel(got, gp[k]) <= 2e-2, f"prefix d{k}"
        rest = g2[k].float().clone()
        rest[b, ..., :t] = 0
        assert not rest.any(), f"d{k} outside the prefix"


def test_config1_full_size_slices():
    """BASELINE config 1 at full size (B8 D1536 L2048 N16, bf16, seed 1001)."""
    inp = orc.selective_scan_inputs(8, 1536, 2048, 16, 1, seed=1001, act_dtype=torch.bfloat16)
    _full_size_check(inp, slice(100, 132), prefix_row=3, prefix_len=512)


@pytest.fixture(scope="module")
def config2_inputs():
    from metal_kernelops_b200.workloads import selective_scan_rows
    return selective_scan_rows(5120, 4096, 16, 1, 1002, 0, 16)


@pytest.mark.parametrize("lean", [False, True], ids=["saved_states", "lean"])
def test_config2_full_size_slices(config2_inputs, lean):
    """BASELINE config 2 -- the bench's headline workload -- at full size
    (B16 D5120 L4096 N16, bf16) on exactly the inputs ``bench.py`` times
    (``workloads.selective_scan_rows``, seed 1002): the launch shape, the
    saved-state layout and the partial reductions of the timed kernels, in
    both backward modes (states saved every 4 steps; the lean mode's states
    every 16 steps with the rest recomputed)."""
    _full_size_check(config2_inputs, slice(2000, 2032), prefix_row=5, prefix_len=256, lean=lean)


def test_errors():
    mk = _mk()
    inp = orc.selective_scan_inputs(1, 4, 8, 3, 1, seed=2)
    cu = {k: v.cuda() for k, v in inp.items()}
    with pytest.raises(ValueError):   # groups must divide dim
        mk.selective_scan(cu["u"], cu["delta"], cu["A"], cu["B"].repeat(1, 3, 1, 1),
                          cu["C"].repeat(1, 3, 1, 1))
    with pytest.raises(ValueError):   # float64 is not a kernel dtype
        mk.selective_scan(cu["u"].double(), cu["delta"], cu["A"], cu["B"], cu["C"])
    big = torch.zeros(1, 4, 8, device="cuda")
    with pytest.raises(ValueError):   # dstate above the supported maximum
        mk.selective_scan(big, big, torch.zeros(4, 65, device="cuda"),
                          torch.zeros(1, 1, 65, 8, device="cuda"), torch.zeros(1, 1, 65, 8, device="cuda"))


@pytest.mark.parametrize("shape,dtype", [
    ((1, 8, 2000, 16, 1), torch.float32),     # one channel tile: 32 segments per pass
    ((2, 24, 1999, 16, 3), torch.float32),    # ragged last chunk and segment, 3 groups
    ((1, 4, 515, 32, 1), torch.float32),      # 32 states
    ((1, 40, 1500, 16, 1), torch.bfloat16),
])
def test_sequence_segments(shape, dtype):
    """Small batch x dim with long sequences: the kernels cut the sequence into
    segments (a summary pass, a combine over segments, then every segment from
    its entering state / adjoint).  Same oracle and tolerances as above."""
    b, d, l, n, g = shape
    inp = orc.selective_scan_inputs(b, d, l, n, g, seed=70 + l, act_dtype=dtype)
    _run_pair(inp, dtype)
    # bare scan: without the softplus the raw delta must stay positive, or
    # exp(delta * A) overflows over a long sequence (in the oracle too)
    bare = dict(inp, delta=(inp["delta"].float().abs() * 0.1 + 1e-3).to(dtype))
    _run_pair(bare, dtype, opts=(), softplus=False)


@pytest.mark.parametrize("shape,dtype,opts", [
    ((2, 64, 256, 16, 1), torch.bfloat16, ("D", "z", "delta_bias")),
    ((6, 4096, 128, 16, 1), torch.bfloat16, ("D", "z", "delta_bias")),    # 8 states x 2 lanes
    ((1, 40, 1496, 16, 1), torch.bfloat16, ("D", "z", "delta_bias")),     # segments, ragged chunk
    ((2, 24, 1000, 16, 3), torch.float32, ("D", "delta_bias")),                # ragged chunk, 3 groups
    ((3, 96, 640, 8, 2), torch.float16, ("z",)),
    ((2, 32, 512, 32, 1), torch.float32, ("D", "z", "delta_bias")),
    ((2, 16, 256, 64, 1), torch.bfloat16, ("D", "z", "delta_bias")),
    ((2, 128, 272, 4, 4), torch.float32, ("D", "z", "delta_bias")),
    # the two-channel dstate-16 backward: a last channel tile of 8 channels (one
    # lane's pair may be half valid), segments, a ragged last chunk
    ((1, 8200, 1992, 16, 1), torch.bfloat16, ("D", "z", "delta_bias")),
    ((2, 8200, 776, 16, 2), torch.float32, ("D", "delta_bias")),
    ((2, 4096, 256, 16, 1), torch.float16, ("D", "z", "delta_bias")),
])
def test_tma_and_plain_staging_identical(shape, dtype, opts):
    """Rows that are 16-byte aligned run the TMA-staged kernels; the
    plain-staging kernels run the same arithmetic, so y and every gradient
    are equal bit for bit between the two.  One exception: at dstate 16 with
    8 states x 2 lanes per channel (from 8192 rows) the TMA backward holds two
    channels of 4 states per lane, so its sums over channels (dB, dC) and over
    states (du, ddelta, hence d delta_bias) associate differently, and it
    forms dh a x as (dh a) x (dA) -- those agree to fp32 rounding, carried into
    the activation dtype; y, dD and dz stay bit-identical."""
    mk = _mk()
    from metal_kernelops_b200 import scan as scan_mod
    b, d, l, n, g = shape
    inp = orc.selective_scan_inputs(b, d, l, n, g, seed=300 + l, act_dtype=dtype)
    use = {k: inp[k] for k in NAMES if k in ("u", "delta", "A", "B", "C") or k in opts}
    runs = []
    for tma in (True, False):
        prev = scan_mod.set_tma_staging(tma)
        try:
            dev = {k: v.cuda().requires_grad_(True) for k, v in use.items()}
            y = mk.selective_scan(dev["u"], dev["delta"], dev["A"], dev["B"], dev["C"], D=dev.get("D"),
                                  z=dev.get("z"), delta_bias=dev.get("delta_bias"), delta_softplus=True)
            gr = torch.autograd.grad(y, list(dev.values()), inp["dout"].cuda())
            runs.append([y.detach()] + list(gr))
        finally:
            scan_mod.set_tma_staging(prev)
    two_channel = n == 16 and b * d >= 8192
    regrouped = ("u", "delta", "A", "B", "C", "delta_bias")
    for name, a, b_ in zip(("y",) + tuple(use), *runs):
        if two_channel and name in regrouped:
            assert orc.norm_rel(a.float().cpu(), b_.float().cpu()) <= (1e-6 if a.dtype == torch.float32 else 1e-4), name
        else:
            assert torch.equal(a, b_), name


def test_backward_first_cuda_call_on_a_fresh_thread():
    """torch runs backward passes on its own autograd thread, and the scan's
    backward may be the first CUDA call made there, before any CUDA context is
    current on that thread.  The C-ABI backward, called from a brand-new
    thread with every buffer prepared on the main thread, must run (the TMA
    path encodes its tensor maps only after making the device's context
    current) and equal the same call made on the main thread bit for bit."""
    import threading
    from metal_kernelops_b200 import _native as nat
    from metal_kernelops_b200 import scan as scan_mod
    inp = orc.selective_scan_inputs(2, 64, 256, 16, 1, seed=21, act_dtype=torch.bfloat16)
    dev = {k: inp[k].cuda() for k in NAMES + ("dout",)}
    y, ck = torch.ops.b200ssm.selective_scan_fwd(dev["u"], dev["delta"], dev["A"], dev["B"], dev["C"],
                                                 dev["D"], dev["z"], dev["delta_bias"], True, True)

    def prepared():
        p = scan_mod._params(dev["u"], dev["delta"], dev["A"], dev["B"], dev["C"], dev["D"], dev["z"],
                             dev["delta_bias"], True)
        _, ws_bytes = scan_mod._sizes(p)
        out = {k: torch.empty_like(dev["u"]) for k in ("du", "ddelta", "dz")}
        out.update({"dA": torch.empty_like(dev["A"]), "dB": torch.empty(dev["B"].shape, device="cuda"),
                    "dC": torch.empty(dev["C"].shape, device="cuda"), "dD": torch.empty_like(dev["D"]),
                    "ddelta_bias": torch.empty_like(dev["delta_bias"])})
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
        p.checkpoints, p.dout = ck.data_ptr(), dev["dout"].data_ptr()
        for k, v in out.items():
            setattr(p, k, v.data_ptr())
        p.workspace, p.workspace_bytes = ws.data_ptr(), ws.numel()
        return p, out, ws

    p_main, out_main, ws_main = prepared()
    stream = nat.stream_of(dev["u"])
    nat.check(nat.lib().ssm_selective_scan_bwd(p_main, stream), "main thread")
    p_thr, out_thr, ws_thr = prepared()
    torch.cuda.synchronize()
    status = {}
    th = threading.Thread(target=lambda: status.setdefault("s", nat.lib().ssm_selective_scan_bwd(p_thr, stream)))
    th.start()
    th.join()
    assert status["s"] == nat.SSM_OK, nat.lib().ssm_last_error()
    torch.cuda.synchronize()
    for k in out_main:
        assert torch.equal(out_main[k], out_thr[k]), k


@pytest.mark.parametrize("shape,dtype,plain", [
    ((6, 4096, 128, 16, 1), torch.bfloat16, False),    # TMA path, 8 states x 2 lanes
    ((2, 64, 256, 16, 1), torch.bfloat16, False),      # TMA path, segments
    ((2, 24, 1000, 16, 3), torch.float32, False),      # ragged last chunk
    ((2, 64, 250, 16, 1), torch.bfloat16, True),       # plain path (unaligned rows)
    ((2, 32, 512, 32, 1), torch.float32, True),        # plain path, 32 states
    ((1, 8200, 1992, 16, 1), torch.bfloat16, False),   # two-channel backward, segments, partial tile
])
def test_lean_backward_matches_saved_states(shape, dtype, plain):
    """The lean mode saves the state entering every 16-step chunk only and
    replays the rest in the backward with the same arithmetic: every gradient
    but dz equals the default mode's bit for bit; dz (from the recomputed
    scan output, summed in another order) agrees to the activation dtype's
    rounding; the saved buffer is a quarter of the states and no output."""
    mk = _mk()
    from metal_kernelops_b200 import scan as scan_mod
    b, d, l, n, g = shape
    inp = orc.selective_scan_inputs(b, d, l, n, g, seed=400 + l, act_dtype=dtype)
    runs, saved = [], []
    prev_tma = scan_mod.set_tma_staging(not plain)
    try:
        for lean in (False, True):
            prev = scan_mod.set_lean_backward(lean)
            try:
                dev = {k: inp[k].cuda().requires_grad_(True) for k in NAMES}
                y = mk.selective_scan(dev["u"], dev["delta"], dev["A"], dev["B"], dev["C"], D=dev["D"],
                                      z=dev["z"], delta_bias=dev["delta_bias"], delta_softplus=True)
                gr = torch.autograd.grad(y, list(dev.values()), inp["dout"].cuda())
                runs.append(dict(zip(("y",) + NAMES, [y.detach()] + list(gr))))
                _, ck = torch.ops.b200ssm.selective_scan_fwd(dev["u"], dev["delta"], dev["A"], dev["B"], dev["C"],
                                                             dev["D"], dev["z"], dev["delta_bias"], True, True, lean)
                saved.append(ck.numel())
            finally:
                scan_mod.set_lean_backward(prev)
    finally:
        scan_mod.set_tma_staging(prev_tma)
    full, lean_ = runs
    for k in ("y",) + NAMES:
        if k == "z":
            assert orc.norm_rel(lean_[k].float().cpu(), full[k].float().cpu()) <= 1e-2 if dtype != torch.float32 \
                else orc.norm_rel(lean_[k].cpu(), full[k].cpu()) <= 1e-6, k
        else:
            assert torch.equal(lean_[k], full[k]), k
    assert saved[1] < saved[0] / 3
