"""CPU restatement of the reference's SSM-scan definitions (TEST INFRASTRUCTURE).

This module is the parity oracle and the CPU baseline.  It is never imported by
``metal_kernelops_b200``.  Every function restates one definition of
dbydd/metal-kernelops 0.3.0 (paths relative to that project) in plain torch
so that it evaluates in float64 on the CPU and carries autograd where the
reference's does:

* ``selective_scan_stepwise``  <- ``src/metal_kernelops/reference.py:5-49``
  (the triple-loop recurrence; forward only, like the original)
* ``scan_functional``          <- ``src/metal_kernelops/cv/path_scan.py:579-605``
  (``_scan_reference``: the same recurrence, rebuilt per step so autograd works)
* ``selective_scan_ref``       <- ``src/metal_kernelops/scan.py:295-320``
  (bias, softplus, scan, ``+ u*D``, ``* silu(z)``) over ``scan_functional``
* ``mamba2_chunk_scan_ref``    <- ``src/metal_kernelops/cv/mamba2_chunk.py:681-723``
* ``mamba2_chunk_scan_composition`` <- ``cv/mamba2_chunk.py:447-533`` and
  ``:652-678`` (the chunked torch composition the reference runs off-MPS; it is
  the reference's CPU path and therefore the timed CPU baseline for SSD)
* ``mamba2_state_update_ref``  <- ``src/metal_kernelops/cv/mamba2_state.py:822-849``
* ``ss2d_scan_ref``            <- ``src/metal_kernelops/cv/path_scan.py:608-639``
  (``ss2d_scan_reference``: four index-arithmetic path orders over
  ``scan_functional``, merged as (p0 + p2) + (p1 + p3))
* ``causal_conv1d_ref``        <- ``src/metal_kernelops/cv/causal_conv1d.py:480-518``
  (explicit taps over ``cat(initial_state, x)``, bias, SiLU, final state)
* ``causal_conv1d_update_ref`` <- ``src/metal_kernelops/cv/causal_conv1d.py:657-670``
  (``_update_aten``: the decode step against a rolling state, in place)
* ``rmsnorm_gated_ref``        <- ``src/metal_kernelops/cv/gated_norm.py:689-720``
  (``rmsnorm_gated_reference``: mamba's ``rms_norm_ref`` in float64)
* ``ssd_minimal_discrete``     <- ``benchmarks/verify_mamba2_chunk.py:185-216``
  (the published ``ssd_minimal_discrete`` listing of state-spaces/mamba, used
  by the reference as a known-answer cross-check)

The seeded input generators (hot-path configurations 0-4 and the reference
verifiers' distributions) live in ``metal_kernelops_b200.workloads`` and are
re-exported here for the tests.
"""

from __future__ import annotations


import torch
import torch.nn.functional as F

# seeded workload generators (BASELINE distributions); they live with the
# package so that bench.py's GPU arm does not import this module
from metal_kernelops_b200.workloads import (  # noqa: F401
    decode_inputs, selective_scan_inputs, ss2d_inputs, ssd_inputs)

__all__ = [
    "selective_scan_stepwise",
    "scan_functional",
    "selective_scan_ref",
    "mamba2_chunk_scan_ref",
    "mamba2_chunk_scan_composition",
    "mamba2_state_update_ref",
    "ssd_minimal_discrete",
    "causal_conv1d_ref",
    "rmsnorm_gated_ref",
    "causal_conv1d_update_ref",
    "ss2d_path_orders",
    "ss2d_scan_ref",
    "ss2d_inputs",
    "max_rel",
    "norm_rel",
    "selective_scan_inputs",
    "ssd_inputs",
    "decode_inputs",
]


# ---------------------------------------------------------------------------
# error metrics used by the reference's verifiers
# ---------------------------------------------------------------------------

def max_rel(got, want):
    """max|got - want| / max|want| (``benchmarks/verify_mamba2_chunk.py:67-73``)."""
    got = got.detach().double().cpu()
    want = want.detach().double().cpu()
    if want.numel() == 0:
        return 0.0
    scale = want.abs().max().item()
    return (got - want).abs().max().item() / max(scale, 1e-30)


def norm_rel(got, want):
    """||got - want|| / ||want||, 0 when both are zero
    (``benchmarks/verify_path_scan.py:61-66``)."""
    got = got.detach().double().cpu()
    want = want.detach().double().cpu()
    denom = float(want.norm())
    if denom == 0.0:
        return 0.0 if float(got.norm()) == 0.0 else float("inf")
    return float((got - want).norm()) / denom


# ---------------------------------------------------------------------------
# Mamba-1 selective scan
# ---------------------------------------------------------------------------

def selective_scan_stepwise(u, dt, A, B, C):
    """Per-(t, b, channel) loop, forward only (``reference.py:5-49``).

    x_t = exp(dt_t * A) * x_{t-1} + dt_t * B_t * u_t ;  y_t = <x_t, C_t>
    u, dt: (batch, dim, length); A: (dim, dstate); B, C: (batch, groups, dstate, length).
    """
    batch, dim, length = u.shape
    groups, dstate = B.shape[1], A.shape[1]
    if dim % groups:
        raise ValueError("dim must be divisible by groups")
    width = dim // groups
    y = torch.zeros_like(u)
    state = torch.zeros(batch, dim, dstate, dtype=u.dtype)
    for t in range(length):
        for b in range(batch):
            for ch in range(dim):
                g = ch // width
                decay = torch.exp(A[ch] * dt[b, ch, t])
                state[b, ch] = decay * state[b, ch] + dt[b, ch, t] * u[b, ch, t] * B[b, g, :, t]
                y[b, ch, t] = torch.dot(state[b, ch], C[b, g, :, t])
    return y


def scan_functional(u, dt, A, B, C, stepping="unbind"):
    """Differentiable stepwise scan (``cv/path_scan.py:579-605``).

    The state is rebuilt every step instead of written in place, so autograd
    can differentiate it.  Vectorised over (batch, channel, state).

    ``stepping="index"`` takes each step's slices exactly as the reference
    does (``x[:, :, t]`` on the inputs, B and C of the step expanded to the
    channels per step); autograd then builds a full-size zero gradient per
    step and slice, which is the reference's own cost and what the timed CPU
    baseline measures.  ``stepping="unbind"`` (the parity default) takes the
    same per-step values from ``unbind``, whose backward is one stack, so long
    sequences stay linear in time; the arithmetic is identical.
    """
    batch, dim, length = u.shape
    dstate = A.shape[1]
    groups = B.shape[1]
    width = dim // groups if groups else 0
    if length == 0 or dim == 0 or batch == 0:
        return u.new_zeros(batch, dim, length) + 0.0 * (u.sum() + dt.sum() + A.sum() + B.sum() + C.sum())
    if stepping == "index":
        step_of = lambda t: (dt[:, :, t], u[:, :, t],  # noqa: E731
                             B[:, :, :, t].repeat_interleave(width, dim=1),
                             C[:, :, :, t].repeat_interleave(width, dim=1))
    elif stepping == "unbind":
        dts, us, Bs, Cs = dt.unbind(-1), u.unbind(-1), B.unbind(-1), C.unbind(-1)
        step_of = lambda t: (dts[t], us[t], Bs[t].repeat_interleave(width, dim=1),  # noqa: E731
                             Cs[t].repeat_interleave(width, dim=1))
    else:
        raise ValueError(f"unknown stepping {stepping!r}")
    state = u.new_zeros(batch, dim, dstate)
    out = []
    for t in range(length):
        d_t, u_t, b_t, c_t = step_of(t)
        state = torch.exp(d_t.unsqueeze(-1) * A) * state + (d_t * u_t).unsqueeze(-1) * b_t
        out.append((state * c_t).sum(-1))
    return torch.stack(out, dim=-1)


def selective_scan_ref(u, dt, A, B, C, D=None, z=None, delta_bias=None,
                       delta_softplus=False, stepping="unbind"):
    """The full Mamba-1 op of ``scan.py:295-320`` over ``scan_functional``.

    bias add, softplus (torch's threshold-20 rule), scan, ``+ u*D``, ``* silu(z)``.
    """
    if delta_bias is not None:
        dt = dt + delta_bias[..., None]
    if delta_softplus:
        dt = F.softplus(dt)
    out = scan_functional(u, dt, A, B, C, stepping=stepping)
    if D is not None:
        out = out + u * D[..., None]
    if z is not None:
        out = out * F.silu(z)
    return out


# ---------------------------------------------------------------------------
# causal depthwise conv1d
# ---------------------------------------------------------------------------

def causal_conv1d_ref(x, weight, bias=None, activation=None, initial_state=None,
                      return_final_state=False):
    """Explicit-tap causal depthwise conv1d (``causal_conv1d_ref``,
    cv/causal_conv1d.py:480-518): arithmetic in ``weight.dtype``, result in
    ``x.dtype``, SiLU after the cast, final state = last K-1 columns of
    ``cat(initial_state, x)``.  Differentiable."""
    if weight.dim() == 3:
        weight = weight[:, 0, :]
    channels, width = weight.shape
    taps = width - 1
    length = x.shape[-1]
    out_dtype, compute = x.dtype, weight.dtype
    work = x.to(compute)
    if initial_state is not None:
        work = torch.cat([initial_state.to(compute), work], dim=-1)
    else:
        work = F.pad(work, (taps, 0))
    out = None
    for j in range(width):
        term = work[..., j:j + length] * weight[:, j].view(1, channels, 1)
        out = term if out is None else out + term
    if bias is not None:
        out = out + bias.to(compute).view(1, channels, 1)
    final = work[..., length:].to(out_dtype) if return_final_state else None
    out = out.to(out_dtype)
    if activation is not None:
        out = F.silu(out)
    return (out, final) if return_final_state else out


def causal_conv1d_update_ref(x, state, weight, bias=None, activation=None):
    """Decode step (``_update_aten``, cv/causal_conv1d.py:657-670): convolve
    ``cat(state, x)``, keep the last q outputs, and overwrite ``state`` in place
    with the last ``s`` columns.  x is (batch, channels, q)."""
    if weight.dim() == 3:
        weight = weight[:, 0, :]
    channels = weight.shape[0]
    length = x.shape[-1]
    compute = weight.dtype
    joined = torch.cat([state.to(compute), x.to(compute)], dim=-1)
    shift = bias.to(compute) if bias is not None else None
    out = F.conv1d(joined, weight.unsqueeze(1), shift, groups=channels)
    state.copy_(joined[..., -state.shape[-1]:])
    out = out[..., -length:]
    if activation is not None:
        out = F.silu(out)
    return out.to(x.dtype)


# ---------------------------------------------------------------------------
# gated RMSNorm
# ---------------------------------------------------------------------------

def rmsnorm_gated_ref(x, weight, bias=None, z=None, eps=1e-5, group_size=None,
                      norm_before_gate=True):
    """mamba's ``rms_norm_ref`` (``rmsnorm_gated_reference``,
    cv/gated_norm.py:689-720): gate before the mean or after the shift, biased
    mean over groups of ``group_size``, evaluated in the inputs' dtype (call it
    with float64 tensors).  Differentiable."""
    features = x.shape[-1]
    group = features if group_size is None else group_size
    xf = x
    if z is not None and not norm_before_gate:
        xf = xf * F.silu(z)
    grouped = xf.reshape(xf.shape[:-1] + (features // group, group))
    rstd = torch.rsqrt(grouped.square().mean(-1, keepdim=True) + eps)
    out = (grouped * rstd).reshape(xf.shape) * weight
    if bias is not None:
        out = out + bias
    if z is not None and norm_before_gate:
        out = out * F.silu(z)
    return out


# ---------------------------------------------------------------------------
# VMamba four-path 2D scan
# ---------------------------------------------------------------------------

def ss2d_path_orders(height, width):
    """Step -> flat pixel index of the four paths (``cv/path_scan.py:153-163``),
    built from explicit index lists: row-major, column-major, and their reverses."""
    row = [h * width + w for h in range(height) for w in range(width)]
    col = [h * width + w for w in range(width) for h in range(height)]
    return [torch.tensor(o, dtype=torch.long) for o in (row, col, row[::-1], col[::-1])]


def ss2d_scan_ref(u, dt, A, B, C, merge="sum"):
    """Four-path 2D selective scan (``ss2d_scan_reference``, path_scan.py:608-639).

    u, dt: (batch, channels, height, width); A: (channels, states);
    B, C: (batch, groups, states, height, width).  Each path permutes the
    flattened map, runs ``scan_functional``, and scatters back; the merge is
    (p0 + p2) + (p1 + p3), times 0.25 for ``merge="mean"``.
    """
    if merge not in ("sum", "mean"):
        raise ValueError(f"merge must be one of ('sum', 'mean'), got {merge!r}")
    batch, channels, height, width = u.shape
    groups, states = B.shape[1], A.shape[1]
    length = height * width
    su = u.reshape(batch, channels, length)
    sdt = dt.reshape(batch, channels, length)
    sb = B.reshape(batch, groups, states, length)
    sc = C.reshape(batch, groups, states, length)
    restored = []
    for order in ss2d_path_orders(height, width):
        y = scan_functional(su.index_select(-1, order), sdt.index_select(-1, order), A,
                            sb.index_select(-1, order), sc.index_select(-1, order))
        restored.append(su.new_zeros(batch, channels, length).index_copy(-1, order, y))
    total = (restored[0] + restored[2]) + (restored[1] + restored[3])
    if merge == "mean":
        total = total * 0.25
    return total.reshape(batch, channels, height, width)


# ---------------------------------------------------------------------------
# Mamba-2 SSD chunk scan
# ---------------------------------------------------------------------------

def _initial_canonical(initial, batch, nheads, headdim, dstate):
    """Accepted ``initial_states`` spellings (``cv/mamba2_chunk.py:426-438``)."""
    if initial is None:
        return None
    if initial.dim() == 5 and initial.shape[1] == 1:
        initial = initial[:, 0]
    if tuple(initial.shape) != (batch, nheads, headdim, dstate):
        if tuple(initial.shape) == (batch, nheads, dstate, headdim) and headdim != dstate:
            initial = initial.transpose(-1, -2)
        else:
            raise ValueError("initial_states has the wrong shape")
    return initial


def mamba2_chunk_scan_ref(x, dt, A, B, C, chunk_size=64, D=None, z=None,
                          dt_bias=None, dt_softplus=False, initial_states=None,
                          dtype=torch.float64):
    """Token-by-token SSD recurrence (``cv/mamba2_chunk.py:681-723``).

    ``chunk_size`` is accepted and ignored.  Returns ``(y, final_state)`` cast
    back to ``x.dtype``.
    """
    out_dtype = x.dtype
    x, dt, A, B, C = (t.to(dtype) for t in (x, dt, A, B, C))
    batch, length, nheads, headdim = x.shape
    ngroups, dstate = B.shape[2], B.shape[3]
    rep = nheads // ngroups
    Bh = B.repeat_interleave(rep, dim=2)
    Ch = C.repeat_interleave(rep, dim=2)
    if dt_bias is not None:
        dt = dt + dt_bias.to(dtype).view(1, 1, nheads)
    if dt_softplus:
        dt = F.softplus(dt)
    state = x.new_zeros(batch, nheads, headdim, dstate)
    init = _initial_canonical(initial_states, batch, nheads, headdim, dstate)
    if init is not None:
        state = init.to(dtype).clone()
    ys = []
    for t in range(length):
        d_t = dt[:, t]                                              # (b, h)
        state = state * torch.exp(d_t * A)[..., None, None] + \
            (d_t[..., None] * x[:, t])[..., :, None] * Bh[:, t][:, :, None, :]
        ys.append((state * Ch[:, t][:, :, None, :]).sum(-1))
    y = torch.stack(ys, dim=1) if length else x.new_zeros(batch, 0, nheads, headdim)
    if D is not None:
        Dd = D.to(dtype)
        y = y + x * (Dd.view(1, 1, nheads, 1) if Dd.dim() == 1 else Dd.view(1, 1, nheads, headdim))
    if z is not None:
        y = y * F.silu(z.to(dtype))
    return y.to(out_dtype), state.to(out_dtype)


def mamba2_chunk_scan_composition(x, dt, A, B, C, chunk_size=64, D=None, z=None,
                                  dt_bias=None, dt_softplus=False, initial_states=None):
    """The reference's chunked torch composition (``cv/mamba2_chunk.py:447-533``,
    ``:652-678``): fp32 discretisation, chunk states by matmul, a causal
    chunk-to-chunk decay matrix, intra- and inter-chunk outputs per group.
    Differentiable through autograd; this is the reference's CPU code path."""
    batch, length, nheads, headdim = x.shape
    ngroups, dstate = B.shape[2], B.shape[3]
    init = _initial_canonical(initial_states, batch, nheads, headdim, dstate)
    rep = nheads // ngroups
    q = min(chunk_size, length)
    nc = -(-length // q)
    padded = nc * q
    # discretisation, float32 (:447-462)
    d = dt.transpose(1, 2).to(torch.float32)
    if dt_bias is not None:
        d = d + dt_bias.to(torch.float32).view(1, nheads, 1)
    if dt_softplus:
        d = F.softplus(d)
    if padded > length:
        d = F.pad(d, (0, padded - length))
    d = d.reshape(batch, nheads, nc, q)
    dcs = torch.cumsum(d * A.to(torch.float32).view(1, nheads, 1, 1), dim=-1)
    if padded > length:
        pad = (0, 0, 0, 0, 0, padded - length)
        xp, Bp, Cp = F.pad(x, pad), F.pad(B, pad), F.pad(C, pad)
    else:
        xp, Bp, Cp = x, B, C
    # chunk states (:465-484): (b, h, c, n, p)
    w = (d * torch.exp(dcs[..., -1:] - dcs)).permute(0, 2, 3, 1).unsqueeze(-1)
    xw = xp.view(batch, nc, q, nheads, headdim) * w.to(x.dtype)
    xg = xw.view(batch, nc, q, ngroups, rep, headdim).permute(0, 3, 4, 1, 2, 5)
    Bg = Bp.view(batch, nc, q, ngroups, dstate).permute(0, 3, 1, 2, 4)
    states = torch.matmul(Bg.transpose(-1, -2).unsqueeze(2), xg)
    states = states.float().reshape(batch, nheads, nc, dstate, headdim)
    # chunk-to-chunk transfer (:487-505)
    total = dcs[..., -1]
    before = torch.cumsum(F.pad(total, (1, 0)), dim=-1)
    diff = before[..., :-1, None] - before[..., None, 1:]
    mask = torch.ones(nc, nc, dtype=torch.bool).tril(-1)
    decay = torch.exp(diff.masked_fill(~mask, float("-inf")))
    entering = torch.matmul(decay, states.reshape(batch, nheads, nc, dstate * headdim))
    if init is not None:
        carry = torch.exp(before[..., :-1]).unsqueeze(-1)
        entering = entering + carry * init.transpose(-1, -2).reshape(
            batch, nheads, headdim * dstate).unsqueeze(2)
    entering = entering.reshape(batch, nheads, nc, dstate, headdim)
    final = states[:, :, -1] + torch.exp(total[:, :, -1])[..., None, None] * entering[:, :, -1]
    final = final.transpose(-1, -2).contiguous()
    # outputs (:508-533)
    lower = torch.ones(q, q, dtype=torch.bool).tril()
    intra = torch.exp((dcs[..., :, None] - dcs[..., None, :]).masked_fill(~lower, float("-inf")))
    out_decay = torch.exp(dcs)
    parts = []
    for g in range(ngroups):
        hs = slice(g * rep, (g + 1) * rep)
        Cg = Cp[:, :, g].reshape(batch, nc, q, dstate).contiguous()
        Bgg = Bp[:, :, g].reshape(batch, nc, q, dstate).contiguous()
        cb = torch.matmul(Cg, Bgg.transpose(-1, -2)).float()
        scores = (intra[:, hs] * cb[:, None] * d[:, hs][..., None, :]).to(x.dtype)
        xh = xp[:, :, hs].view(batch, nc, q, rep, headdim).permute(0, 3, 1, 2, 4)
        out = torch.matmul(scores, xh)
        prev = torch.matmul(Cg[:, None].to(x.dtype), entering[:, hs].to(x.dtype))
        prev = prev * out_decay[:, hs][..., None].to(x.dtype)
        parts.append((out + prev).permute(0, 2, 3, 1, 4))
    y = parts[0] if ngroups == 1 else torch.cat(parts, dim=3)
    y = y.reshape(batch, padded, nheads, headdim)
    if D is not None:
        skip = D.to(x.dtype).view(1, 1, nheads, 1) if D.dim() == 1 else D.to(x.dtype).view(1, 1, nheads, headdim)
        y = y + xp * skip
    if z is not None:
        zp = F.pad(z, (0, 0, 0, 0, 0, padded - length)) if padded > length else z
        y = y * F.silu(zp)
    if padded > length:
        y = y[:, :length].contiguous()
    return y, final.to(x.dtype)


def _segsum(v):
    """Stable segment sum of the ``ssd_minimal`` listing: out[..., i, j] =
    sum_{j<k<=i} v[..., k] for j <= i, -inf above the diagonal."""
    size = v.size(-1)
    tri_strict = torch.ones(size, size, dtype=torch.bool).tril(-1)
    tri = torch.ones(size, size, dtype=torch.bool).tril()
    rep = v.unsqueeze(-1).expand(*v.shape, size).masked_fill(~tri_strict, 0)
    acc = torch.cumsum(rep, dim=-2)
    return acc.masked_fill(~tri, float("-inf"))


def ssd_minimal_discrete(X, A, B, C, block_len, initial_states=None):
    """``ssd_minimal_discrete`` as listed in ``verify_mamba2_chunk.py:185-216``.

    X: (b, l, h, p) already multiplied by dt; A: (b, l, h) = A*dt; B, C: (b, l, g, n)
    with g == h or g == 1.  Returns (y, final_state (b, h, p, n)).
    """
    batch, length, nheads, headdim = X.shape
    nc = length // block_len
    X = X.reshape(batch, nc, block_len, nheads, headdim)
    A = A.reshape(batch, nc, block_len, nheads).permute(0, 3, 1, 2)
    B = B.reshape(batch, nc, block_len, B.shape[2], B.shape[3])
    C = C.reshape(batch, nc, block_len, C.shape[2], C.shape[3])
    if B.shape[3] != nheads:
        B = B.expand(-1, -1, -1, nheads, -1)
        C = C.expand(-1, -1, -1, nheads, -1)
    A_cs = torch.cumsum(A, dim=-1)
    L = torch.exp(_segsum(A))
    Y_diag = torch.einsum("bclhn,bcshn,bhcls,bcshp->bclhp", C, B, L, X)
    decay_states = torch.exp(A_cs[:, :, :, -1:] - A_cs)
    states = torch.einsum("bclhn,bhcl,bclhp->bchpn", B, decay_states, X)
    if initial_states is None:
        initial_states = torch.zeros_like(states[:, :1])
    states = torch.cat([initial_states, states], dim=1)
    decay_chunk = torch.exp(_segsum(F.pad(A_cs[:, :, :, -1], (1, 0))))
    new_states = torch.einsum("bhzc,bchpn->bzhpn", decay_chunk, states)
    states, final_state = new_states[:, :-1], new_states[:, -1]
    Y_off = torch.einsum("bclhn,bchpn,bhcl->bclhp", C, states, torch.exp(A_cs))
    return (Y_diag + Y_off).reshape(batch, length, nheads, headdim), final_state


# ---------------------------------------------------------------------------
# Mamba-2 decode state update
# ---------------------------------------------------------------------------

def mamba2_state_update_ref(state, x, dt, A, B, C, D=None, z=None, dt_bias=None,
                            dt_softplus=False):
    """One decode step in closed form (``cv/mamba2_state.py:822-849``).

    Leaves ``state`` untouched; returns ``(y, new_state)``.
    """
    if dt.dim() == 2:
        dt = dt.unsqueeze(-1)
    if D is not None and D.dim() == 1:
        D = D.unsqueeze(-1)
    if dt_bias is not None:
        dt = dt + dt_bias[None, :, None]
    if dt_softplus:
        dt = F.softplus(dt)
    nheads, ngroups = state.shape[1], B.shape[1]
    rep = nheads // ngroups
    Bh = B.repeat_interleave(rep, dim=1)
    Ch = C.repeat_interleave(rep, dim=1)
    decay = torch.exp(A[None, :, None, None] * dt[..., None])
    new_state = decay * state + (dt * x)[..., None] * Bh[:, :, None, :]
    y = (new_state * Ch[:, :, None, :]).sum(-1)
    if D is not None:
        y = y + x * D
    if z is not None:
        y = y * F.silu(z)
    return y, new_state


# ---------------------------------------------------------------------------
# seeded inputs for the hot-path configurations
# ---------------------------------------------------------------------------

