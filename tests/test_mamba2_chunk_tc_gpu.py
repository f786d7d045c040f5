"""Mamba-2 SSD chunk scan, tensor-core path (tcgen05 / TMEM), vs the fp64 oracle.

The tensor-core kernels serve bf16/f16 inputs with d_head a multiple of 8 up to
64, or 128 or 256, and d_state a multiple of 8 up to 128 (tiles of the
Mamba-2 layer shape of BASELINE config 3, d_head 64 and d_state 128, which
smaller heads fill with zeros and wider heads split into 64-column virtual
heads); they round each GEMM operand to
the input dtype and accumulate in fp32.  These tests check them the way the
reference's verifier checks its fast path (benchmarks/verify_mamba2_chunk.py):
forward outputs and final state over ragged lengths, group sizes and every
option against the fp64 sequential recurrence (max|err| / max|ref|: bf16 2e-2,
f16 2e-3), all nine gradients against fp64 autograd (norm-relative: bf16 2e-2,
the north-star bf16 limit, f16 5e-3), a gradient slice of the full config-3
problem against the fp64 oracle, agreement with the CUDA-core kernels at the
full config-3 size, bit-identical reruns, and that no kernel gave up on a
bounded wait.
"""

import pytest
import torch

from oracle import ssm_oracle as orc

pytestmark = pytest.mark.gpu

P, N = 64, 128
TOL_FWD = {torch.bfloat16: 2e-2, torch.float16: 2e-3}
TOL_GRAD = {torch.bfloat16: 2e-2, torch.float16: 5e-3}
NAMES = ("x", "dt", "A", "B", "C", "D", "z", "dt_bias", "initial_states")


def _mod():
    from metal_kernelops_b200.cv import mamba2_chunk
    return mamba2_chunk


def _inputs(batch, length, nheads, ngroups, seed, dtype, d_per_head=False, p=P, n=N):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(batch, length, nheads, p, generator=g)
    dt = torch.randn(batch, length, nheads, generator=g) - 1.0
    A = -(torch.rand(nheads, generator=g) * 4 + 0.5)
    B = torch.randn(batch, length, ngroups, n, generator=g)
    C = torch.randn(batch, length, ngroups, n, generator=g)
    D = torch.randn(nheads, p, generator=g) if d_per_head else torch.randn(nheads, generator=g)
    z = torch.randn(batch, length, nheads, p, generator=g)
    bias = torch.randn(nheads, generator=g) * 0.5
    init = torch.randn(batch, nheads, p, n, generator=g) * 0.2
    vals = dict(x=x, dt=dt, A=A, B=B, C=C, D=D, z=z, dt_bias=bias, initial_states=init)
    # x, B, C, z, dt in the run dtype; the oracle sees the same rounded values
    for k in ("x", "dt", "B", "C", "z"):
        vals[k] = vals[k].to(dtype)
    return vals


def _run(vals, device, cast, fn, opts, grad=False):
    t = {k: (v.to(device) if k in ("x", "dt", "B", "C", "z") else v.to(device, cast))
         for k, v in vals.items()}
    if cast == torch.float64:
        t = {k: v.double() for k, v in t.items()}
    if grad:
        t = {k: v.requires_grad_(True) for k, v in t.items()}
    kw = {k: t[k] for k in opts}
    y, s = fn(t["x"], t["dt"], t["A"], t["B"], t["C"], 256, dt_softplus=True, **kw)
    return t, y, s


SHAPES = [(1, 128, 2, 1), (2, 300, 4, 2), (1, 1000, 8, 2), (2, 77, 6, 3)]
OPTS = [(), ("D", "z", "dt_bias", "initial_states")]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("oi", range(len(OPTS)))
@pytest.mark.parametrize("si", range(len(SHAPES)))
def test_tc_forward(si, oi, dtype):
    m = _mod()
    vals = _inputs(*SHAPES[si], seed=100 + si, dtype=dtype)
    opts = OPTS[oi]
    _, y, s = _run(vals, "cuda", torch.float32, m.mamba2_chunk_scan, opts)
    _, yr, sr = _run(vals, "cpu", torch.float64, orc.mamba2_chunk_scan_ref, opts)
    assert y.dtype == dtype
    assert orc.max_rel(y.float().cpu(), yr) <= TOL_FWD[dtype]
    assert orc.max_rel(s.float().cpu(), sr) <= TOL_FWD[dtype]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("shape", [(2, 300, 4, 2), (1, 129, 4, 4)])
def test_tc_gradients_all_inputs(shape, dtype):
    m = _mod()
    vals = _inputs(*shape, seed=7, dtype=dtype)
    g = torch.Generator().manual_seed(8)
    wy = torch.randn(shape[0], shape[1], shape[2], P, generator=g)
    ws = torch.randn(shape[0], shape[2], P, N, generator=g)
    opts = ("D", "z", "dt_bias", "initial_states")

    def grads(device, cast, fn):
        t, y, s = _run(vals, device, cast, fn, opts, grad=True)
        loss = (y.to(cast) * wy.to(device, cast)).sum() + (s.to(cast) * ws.to(device, cast)).sum()
        return torch.autograd.grad(loss, [t[k] for k in NAMES])

    fast = grads("cuda", torch.float32, m.mamba2_chunk_scan)
    slow = grads("cpu", torch.float64, orc.mamba2_chunk_scan_ref)
    for name, gf, gs in zip(NAMES, fast, slow):
        assert orc.norm_rel(gf.float().cpu(), gs) <= TOL_GRAD[dtype], name


def test_tc_gradients_per_head_p_D_no_softplus():
    m = _mod()
    dtype = torch.bfloat16
    vals = _inputs(1, 200, 4, 2, seed=9, dtype=dtype, d_per_head=True)
    vals["dt"] = (vals["dt"].float().abs() * 0.05 + 0.01).to(dtype)
    keys = ("x", "dt", "A", "B", "C", "D")

    def grads(device, cast, fn):
        t = {k: vals[k].to(device) if k in ("x", "dt", "B", "C") else vals[k].to(device, cast) for k in keys}
        if cast == torch.float64:
            t = {k: v.double() for k, v in t.items()}
        t = {k: v.requires_grad_(True) for k, v in t.items()}
        y, s = fn(t["x"], t["dt"], t["A"], t["B"], t["C"], 64, D=t["D"])
        loss = y.to(cast).square().sum() + s.to(cast).square().sum()
        return y, s, torch.autograd.grad(loss, [t[k] for k in keys])

    y, s, fast = grads("cuda", torch.float32, m.mamba2_chunk_scan)
    yr, sr, slow = grads("cpu", torch.float64, orc.mamba2_chunk_scan_ref)
    assert orc.max_rel(y.float().detach().cpu(), yr.detach()) <= TOL_FWD[dtype]
    for name, gf, gs in zip(keys, fast, slow):
        assert orc.norm_rel(gf.float().cpu(), gs) <= TOL_GRAD[dtype], name


def test_tc_deterministic_and_no_kernel_error():
    m = _mod()
    from metal_kernelops_b200 import _native as nat
    vals = _inputs(2, 700, 8, 2, seed=11, dtype=torch.bfloat16)
    runs = []
    for _ in range(3):
        t, y, s = _run(vals, "cuda", torch.float32, m.mamba2_chunk_scan, ("D", "dt_bias"), grad=True)
        gr = torch.autograd.grad(y.float().sum() + s.float().sum(), [t[k] for k in ("x", "dt", "A", "B", "C")])
        runs.append((y.detach(), s.detach()) + tuple(gr))
    for vals_ in zip(*runs):
        assert all(torch.equal(vals_[0], v) for v in vals_[1:])
    torch.cuda.synchronize()
    assert nat.lib().ssm_take_kernel_error() == 0


def test_tc_and_cuda_cores_agree_at_config3():
    """BASELINE config 3 at full size (B8 L8192 H80 P64 N128 G8, bf16): the
    tensor-core forward and backward agree with the CUDA-core kernels (which
    are exact to fp32 rounding) within the bf16 tolerances."""
    m = _mod()
    inp = orc.ssd_inputs(8, 8192, 80, 64, 128, 8)
    dev = {k: v.cuda() for k, v in inp.items()}

    def run(tensor_cores):
        prev = m.set_tensor_cores(tensor_cores)
        try:
            leaves = [dev[k].clone().requires_grad_(True) for k in ("x", "dt", "A", "B", "C", "D", "dt_bias")]
            x, dt, A, B, C, D, bias = leaves
            y, s = m.mamba2_chunk_scan(x, dt, A, B, C, 256, D=D, dt_bias=bias, dt_softplus=True)
            g = torch.autograd.grad((y.float() * dev["dy"].float()).sum(), leaves)
            return [y.detach().float(), s.detach().float()] + [t.float() for t in g]
        finally:
            m.set_tensor_cores(prev)

    fast = run(True)
    exact = run(False)
    names = ("y", "final", "dx", "ddt", "dA", "dB", "dC", "dD", "ddt_bias")
    for name, a, b in zip(names, fast, exact):
        assert torch.isfinite(a).all(), name
        tol = 2e-2
        err = (orc.max_rel(a.cpu(), b.cpu()) if name in ("y", "final")
               else orc.norm_rel(a.cpu(), b.cpu()))
        assert err <= tol, (name, err)
    from metal_kernelops_b200 import _native as nat
    assert nat.lib().ssm_take_kernel_error() == 0


def test_config3_gradient_slice_vs_oracle():
    """BASELINE config 3 at full size (B8 L8192 H80 P64 N128 G8, bf16, the
    bench's inputs) through the tensor-core kernels, with the upstream
    gradient kept only on batch row 5, the first 512 steps and the ten heads
    of group 3 (zero elsewhere).  Rows and groups are independent and the scan
    is causal, so y on that slice and every gradient -- dx, d dt, dB, dC and the
    shared dA, dD, d dt_bias of those heads -- equal the fp64 oracle run on the
    slice alone, and every other gradient entry is zero."""
    m = _mod()
    inp = orc.ssd_inputs(8, 8192, 80, 64, 128, 8)
    r, t, g = 5, 512, 3
    heads = slice(10 * g, 10 * g + 10)
    keys = ("x", "dt", "A", "B", "C", "D", "dt_bias")
    dev = {k: inp[k].cuda().requires_grad_(True) for k in keys}
    y, _ = m.mamba2_chunk_scan(dev["x"], dev["dt"], dev["A"], dev["B"], dev["C"], 256, D=dev["D"],
                               dt_bias=dev["dt_bias"], dt_softplus=True)
    assert m.last_path() == "cuda"
    dy = torch.zeros_like(inp["dy"])
    dy[r, :t, heads] = inp["dy"][r, :t, heads]
    got = dict(zip(keys, torch.autograd.grad(y, [dev[k] for k in keys], dy.cuda())))

    sl = {"x": inp["x"][r:r + 1, :t, heads], "dt": inp["dt"][r:r + 1, :t, heads], "A": inp["A"][heads],
          "B": inp["B"][r:r + 1, :t, g:g + 1], "C": inp["C"][r:r + 1, :t, g:g + 1], "D": inp["D"][heads],
          "dt_bias": inp["dt_bias"][heads]}
    ref = {k: v.double().requires_grad_(True) for k, v in sl.items()}
    yr, _ = orc.mamba2_chunk_scan_ref(ref["x"], ref["dt"], ref["A"], ref["B"], ref["C"], 256, D=ref["D"],
                                      dt_bias=ref["dt_bias"], dt_softplus=True)
    assert orc.max_rel(y[r:r + 1, :t, heads].detach().float().cpu(), yr) <= 2e-2
    want = dict(zip(keys, torch.autograd.grad(yr, [ref[k] for k in keys],
                                              dy[r:r + 1, :t, heads].double())))
    where = {"x": (slice(r, r + 1), slice(0, t), heads), "dt": (slice(r, r + 1), slice(0, t), heads),
             "B": (slice(r, r + 1), slice(0, t), slice(g, g + 1)),
             "C": (slice(r, r + 1), slice(0, t), slice(g, g + 1)),
             "A": (heads,), "D": (heads,), "dt_bias": (heads,)}
    for k in keys:
        gk = got[k].float()
        assert orc.norm_rel(gk[where[k]].cpu(), want[k]) <= 2e-2, k
        rest = gk.clone()
        rest[where[k]] = 0
        assert not rest.any(), f"d{k} outside the slice"
    from metal_kernelops_b200 import _native as nat
    assert nat.lib().ssm_take_kernel_error() == 0


@pytest.mark.parametrize("length", [300, 296])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_tc_token_strided_inputs(dtype, length):
    """x, B and C as column slices of one wider (batch, length, columns)
    buffer -- the Mamba-2 layer's convolution output -- are read through their
    token strides by the tensor maps and the x-row loads, not copied: y, the
    final state and every gradient equal the call on dense copies bit for bit.
    Length 296 (a multiple of 8) takes the whole-tile tensor maps, 300 the
    8-row-group ones."""
    mod = _mod()
    b, h, g = 2, 8, 2
    inner, gn, pad = h * P, g * N, 24
    gen = torch.Generator().manual_seed(77)
    wide = (torch.randn(b, length, inner + 2 * gn + pad, generator=gen)).to("cuda", dtype)
    dt = (torch.randn(b, length, h, generator=gen) - 1.0).to("cuda", dtype)
    A = -(torch.rand(h, generator=gen) * 4 + 0.5).cuda()
    D = torch.randn(h, generator=gen).cuda()
    bias = (torch.randn(h, generator=gen) * 0.5).cuda()
    dy = torch.randn(b, length, h, P, generator=gen).to("cuda", dtype)
    runs = []
    for dense in (False, True):
        x = wide[..., :inner].reshape(b, length, h, P).detach()
        B = wide[..., inner:inner + gn].reshape(b, length, g, N).detach()
        C = wide[..., inner + gn:inner + 2 * gn].reshape(b, length, g, N).detach()
        if dense:
            x, B, C = x.contiguous(), B.contiguous(), C.contiguous()
        leaves = [t.requires_grad_(True) for t in (x, B, C)]
        y, fin = mod.mamba2_chunk_scan(leaves[0], dt, A, leaves[1], leaves[2], chunk_size=64, D=D,
                                       dt_bias=bias, dt_softplus=True)
        grads = torch.autograd.grad((y.float() * dy.float()).sum() + fin.float().sum(), leaves)
        runs.append((y.detach(), fin.detach(), *grads))
    assert mod.last_path() == "cuda"
    for a_, b_ in zip(*runs):
        assert torch.equal(a_, b_)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_tc_whole_tile_maps_match_row_group_maps(dtype):
    """The two ways of copying a tile agree.  A length that is a multiple of 8
    (296) copies each 128-row tile with one whole-tile box, zero-filling the
    rows past the end; a ragged length (300) copies it in 8-row groups.  With
    the same first 296 rows and dy zero on rows 296-299, the two runs give the
    same y, dx, dB, dC and d dt on rows 0-295 (the rows past 296 of the longer
    run only meet zeros there), and the same parameter gradients."""
    mod = _mod()
    b, h, g = 2, 8, 2
    vals = _inputs(b, 300, h, g, seed=41, dtype=dtype)
    x, dt, A, B, C, D, bias = (vals[k].cuda() for k in ("x", "dt", "A", "B", "C", "D", "dt_bias"))
    gen = torch.Generator().manual_seed(42)
    dy = torch.randn(b, 300, h, P, generator=gen).to("cuda", dtype)
    dy[:, 296:] = 0
    runs = []
    for L in (300, 296):
        leaves = [t[:, :L].contiguous().requires_grad_(True) for t in (x, dt, B, C)]
        params = [t.clone().requires_grad_(True) for t in (A, D, bias)]
        y, _ = mod.mamba2_chunk_scan(leaves[0], leaves[1], params[0], leaves[2], leaves[3], chunk_size=128,
                                     D=params[1], dt_bias=params[2], dt_softplus=True)
        assert mod.last_path() == "cuda"
        grads = torch.autograd.grad((y.float() * dy[:, :L].float()).sum(), leaves + params)
        runs.append(([y.detach()[:, :296]] + [t[:, :296] for t in grads[:4]], grads[4:]))
    for name, a_, b_ in zip(("y", "dx", "ddt", "dB", "dC"), runs[0][0], runs[1][0]):
        assert torch.equal(a_, b_), name
    for name, a_, b_ in zip(("dA", "dD", "ddt_bias"), runs[0][1], runs[1][1]):
        torch.testing.assert_close(a_, b_, rtol=1e-5, atol=1e-5, msg=name)


# head shapes other than 64 x 128: zero-filled tiles (d_head < 64, d_state < 128)
# and 64-column virtual heads (d_head 128, 256); (d_head, d_state, heads, groups)
WIDE = [(64, 64, 4, 2), (32, 128, 4, 2), (128, 128, 4, 2), (32, 64, 6, 3), (128, 64, 2, 1),
        (256, 128, 2, 2), (16, 16, 4, 4), (40, 72, 3, 1)]


@pytest.mark.parametrize("wi", range(len(WIDE)))
def test_tc_other_head_shapes_forward_and_gradients(wi):
    """Every option (gate, D per head or per column, bias, initial state, a
    d_state gradient) against the fp64 oracle; the tensor-core path must be the
    one that ran (a CUDA-core fallback would pass the same checks)."""
    m = _mod()
    dtype = torch.bfloat16
    p, n, heads, groups = WIDE[wi]
    assert m.tc_shape(p, n)
    d_per_head = wi % 2 == 1
    vals = _inputs(2, 300, heads, groups, seed=300 + wi, dtype=dtype, d_per_head=d_per_head, p=p, n=n)
    g = torch.Generator().manual_seed(301 + wi)
    wy = torch.randn(2, 300, heads, p, generator=g)
    ws = torch.randn(2, heads, p, n, generator=g)
    opts = ("D", "z", "dt_bias", "initial_states")

    def grads(device, cast, fn):
        t, y, s = _run(vals, device, cast, fn, opts, grad=True)
        loss = (y.to(cast) * wy.to(device, cast)).sum() + (s.to(cast) * ws.to(device, cast)).sum()
        return y.detach(), s.detach(), torch.autograd.grad(loss, [t[k] for k in NAMES])

    y, s, fast = grads("cuda", torch.float32, m.mamba2_chunk_scan)
    yr, sr, slow = grads("cpu", torch.float64, orc.mamba2_chunk_scan_ref)
    assert y.shape == (2, 300, heads, p) and s.shape == (2, heads, p, n)
    assert orc.max_rel(y.float().cpu(), yr) <= TOL_FWD[dtype]
    assert orc.max_rel(s.float().cpu(), sr) <= TOL_FWD[dtype]
    for name, gf, gs in zip(NAMES, fast, slow):
        assert gf.shape == gs.shape, name
        assert orc.norm_rel(gf.float().cpu(), gs) <= TOL_GRAD[dtype], name


def test_tc_other_head_shapes_take_the_tensor_cores():
    """The shapes above run on the tensor cores: forcing the CUDA-core kernels
    gives results within rounding but not bit-identical to them (the two paths
    round GEMM operands differently), while two tensor-core runs are."""
    m = _mod()
    vals = _inputs(1, 200, 4, 2, seed=77, dtype=torch.bfloat16, p=128, n=64)
    _, y1, _ = _run(vals, "cuda", torch.float32, m.mamba2_chunk_scan, ("D", "dt_bias"))
    _, y2, _ = _run(vals, "cuda", torch.float32, m.mamba2_chunk_scan, ("D", "dt_bias"))
    prev = m.set_tensor_cores(False)
    try:
        _, yc, _ = _run(vals, "cuda", torch.float32, m.mamba2_chunk_scan, ("D", "dt_bias"))
    finally:
        m.set_tensor_cores(prev)
    assert torch.equal(y1, y2)
    assert not torch.equal(y1, yc)
    assert orc.max_rel(y1.float().cpu(), yc.float().cpu()) <= 2e-2


def _split_problem(seed):
    """A problem whose state kernels need more than one wave (4 rows x 80 heads
    > 2 per SM x 148 SMs), so the library splits the batch over two streams."""
    return _inputs(4, 384, 80, 8, seed=seed, dtype=torch.bfloat16)


def _fwd_bwd(m, vals):
    t, y, s = _run(vals, "cuda", torch.float32, m.mamba2_chunk_scan, ("D", "dt_bias"), grad=True)
    gr = torch.autograd.grad(y.float().square().sum() + s.float().sum(), [t[k] for k in ("x", "dt", "A", "B", "C")])
    return [y.detach(), s.detach()] + list(gr)


def test_split_batch_follows_the_callers_stream():
    """The batch halves fork from and join back into the stream the call is
    made on: run on a side torch stream, results equal the default stream's
    bit for bit and are complete when that stream is synchronised."""
    m = _mod()
    vals = _split_problem(501)
    ref = _fwd_bwd(m, vals)
    torch.cuda.synchronize()
    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        got = _fwd_bwd(m, vals)
    st.synchronize()
    for a, b in zip(ref, got):
        assert torch.equal(a, b)


def test_split_batch_from_two_host_threads():
    """Two host threads, each on its own stream, run the split SSD at the same
    time (they share the library's side stream): each result equals the one
    computed alone."""
    import threading
    m = _mod()
    probs = [_split_problem(502), _split_problem(503)]
    alone = [_fwd_bwd(m, v) for v in probs]
    torch.cuda.synchronize()
    out, errs = [None, None], []

    def work(i):
        try:
            st = torch.cuda.Stream()
            with torch.cuda.stream(st):
                out[i] = _fwd_bwd(m, probs[i])
            st.synchronize()
        except Exception as exc:  # noqa: BLE001
            errs.append(exc)

    ths = [threading.Thread(target=work, args=(i,)) for i in range(2)]
    for th in ths:
        th.start()
    for th in ths:
        th.join()
    assert not errs, errs
    for i in range(2):
        for a, b in zip(alone[i], out[i]):
            assert torch.equal(a, b)


def test_forward_captures_into_a_cuda_graph():
    """The tensor-core forward can be captured into a CUDA graph (the batch is
    then not split: the capture stays on one stream) and the replay equals an
    eager call on new inputs copied into the captured buffers."""
    m = _mod()
    vals = _split_problem(504)
    dev = {k: (v.cuda() if k in ("x", "dt", "B", "C", "z") else v.cuda().float()) for k, v in vals.items()}
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(st):      # warm-up outside the capture
        m.mamba2_chunk_scan(dev["x"], dev["dt"], dev["A"], dev["B"], dev["C"], 256, D=dev["D"],
                            dt_bias=dev["dt_bias"], dt_softplus=True)
    torch.cuda.current_stream().wait_stream(st)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        y, s = m.mamba2_chunk_scan(dev["x"], dev["dt"], dev["A"], dev["B"], dev["C"], 256, D=dev["D"],
                                   dt_bias=dev["dt_bias"], dt_softplus=True)
    new = _split_problem(505)
    for k in ("x", "dt", "B", "C"):
        dev[k].copy_(new[k].cuda())
    g.replay()
    torch.cuda.synchronize()
    ye, se = m.mamba2_chunk_scan(dev["x"], dev["dt"], dev["A"], dev["B"], dev["C"], 256, D=dev["D"],
                                 dt_bias=dev["dt_bias"], dt_softplus=True)
    assert torch.equal(y, ye) and torch.equal(s, se)
    del g


def test_split_batch_with_virtual_heads_and_padded_states():
    """The batch split together with 64-column virtual heads (d_head 128) and a
    zero-filled state tile (d_state 64): forward and every gradient agree with
    the CUDA-core kernels (which share no code with the tensor-core path)."""
    m = _mod()
    vals = _inputs(4, 256, 40, 8, seed=506, dtype=torch.bfloat16, d_per_head=True, p=128, n=64)
    opts = ("D", "z", "dt_bias", "initial_states")

    def run():
        t, y, s = _run(vals, "cuda", torch.float32, m.mamba2_chunk_scan, opts, grad=True)
        gr = torch.autograd.grad(y.float().square().sum() + s.float().sum(), [t[k] for k in NAMES])
        return [y.detach(), s.detach()] + list(gr)

    tc = run()
    prev = m.set_tensor_cores(False)
    try:
        cc = run()
    finally:
        m.set_tensor_cores(prev)
    for name, a, b in zip(("y", "final") + NAMES, tc, cc):
        assert orc.norm_rel(a.float().cpu(), b.float().cpu()) <= 2e-2, name
