"""Mamba-2 decode state update on the B200: drop-in for
``metal_kernelops.cv.mamba2_state`` (src/metal_kernelops/cv/mamba2_state.py).

One step of the recurrence a Mamba-2 layer runs per generated token::

    delta = softplus(dt + dt_bias)            (dt_softplus=True)
    a     = exp(A_h * delta)
    s'    = a * s + delta * x * B[g]          (g = h // (nheads / ngroups))
    y     = (sum_n s' * C[g] + D * x) * silu(z)

Layouts (reference :17-24): state (batch, nheads, dim, dstate); x, z
(batch, nheads, dim); dt (batch, nheads) or (batch, nheads, dim); A (nheads,);
B, C (batch, ngroups, dstate); D (nheads,) or (nheads, dim); dt_bias (nheads,).

Contract kept from the reference (:26-31, :565-598, :805-819): ``state`` is
never modified unless it is passed as ``out_state``; ``out_state`` is written
in place, must match ``state`` in shape and dtype, be contiguous and not require
grad; x, dt, B, C, z are cast to ``state.dtype`` and A, D, dt_bias to float32
(without grad, 16-bit x, B, C, z against a float32 state are widened inside
the kernel instead -- the same exact conversion, without the copies);
the backward computes in float32 and casts each gradient back to its input's
dtype; without any input requiring grad the kernel is called directly (the
decode-loop path).  ``ValueError`` on contract violations, CPU tensors
included.  Registered as ``b200ssm::state_update_fwd`` / ``_bwd`` custom ops on
the CUDA key.
"""

from __future__ import annotations

from typing import Optional

import torch

from .. import _native as nat

__all__ = ["mamba2_state_update"]

_DTYPES = (torch.float32, torch.float16, torch.bfloat16)


def _flags(dt, D, z, dt_bias, softplus):
    return ((nat.DT_PER_ROW if dt.dim() == 3 else 0) | (nat.HAS_BIAS if dt_bias is not None else 0)
            | (nat.HAS_D if D is not None else 0)
            | (nat.D_PER_HEAD if D is not None and D.dim() == 2 else 0)
            | (nat.HAS_Z if z is not None else 0) | (nat.SOFTPLUS if softplus else 0))


def _params(state, x, dt, A, B, C, D, z, dt_bias, softplus):
    p = nat.StateUpdateParams()
    p.batch, p.nheads, p.headdim, p.dstate = state.shape
    p.ngroups = B.shape[1]
    p.dtype = nat.dtype_code(state.dtype)
    p.flags = _flags(dt, D, z, dt_bias, softplus)
    p.state, p.x, p.dt, p.A, p.B, p.C = (t.data_ptr() for t in (state, x, dt, A, B, C))
    p.D = D.data_ptr() if D is not None else None
    p.z = z.data_ptr() if z is not None else None
    p.dt_bias = dt_bias.data_ptr() if dt_bias is not None else None
    return p


def _launch(state, x, dt, A, B, C, D, z, dt_bias, softplus, new_state):
    y = torch.empty(state.shape[:3], dtype=state.dtype, device=state.device)
    p = _params(state, x, dt, A, B, C, D, z, dt_bias, softplus)
    if x.dtype != state.dtype:      # x, B, C (and z) read in their own dtype
        p.flags |= nat.IO_DTYPE
        p.io_dtype = nat.dtype_code(x.dtype)
    p.new_state, p.y = new_state.data_ptr(), y.data_ptr()
    p.status = nat.status_word(state.device, "state_update")
    nat.check(nat.lib().ssm_state_update_fwd(p, nat.stream_of(state)), "mamba2_state_update")
    return y


@torch.library.custom_op("b200ssm::state_update_fwd", mutates_args=(), device_types="cuda")
def _fwd(state: torch.Tensor, x: torch.Tensor, dt: torch.Tensor, A: torch.Tensor,
         B: torch.Tensor, C: torch.Tensor, D: Optional[torch.Tensor], z: Optional[torch.Tensor],
         dt_bias: Optional[torch.Tensor], softplus: bool) -> tuple[torch.Tensor, torch.Tensor]:
    new_state = torch.empty_like(state)
    y = _launch(state, x, dt, A, B, C, D, z, dt_bias, softplus, new_state)
    return y, new_state


@_fwd.register_fake
def _(state, x, dt, A, B, C, D, z, dt_bias, softplus):
    return state.new_empty(state.shape[:3]), torch.empty_like(state)


@torch.library.custom_op("b200ssm::state_update_into", mutates_args=("out_state",),
                         device_types="cuda")
def _fwd_into(state: torch.Tensor, x: torch.Tensor, dt: torch.Tensor, A: torch.Tensor,
              B: torch.Tensor, C: torch.Tensor, D: Optional[torch.Tensor],
              z: Optional[torch.Tensor], dt_bias: Optional[torch.Tensor], softplus: bool,
              out_state: torch.Tensor) -> torch.Tensor:
    return _launch(state, x, dt, A, B, C, D, z, dt_bias, softplus, out_state)


@_fwd_into.register_fake
def _(state, x, dt, A, B, C, D, z, dt_bias, softplus, out_state):
    return state.new_empty(state.shape[:3])


@torch.library.custom_op("b200ssm::state_update_bwd", mutates_args=(), device_types="cuda")
def _bwd(state: torch.Tensor, x: torch.Tensor, dt: torch.Tensor, A: torch.Tensor,
         B: torch.Tensor, C: torch.Tensor, D: Optional[torch.Tensor], z: Optional[torch.Tensor],
         dt_bias: Optional[torch.Tensor], softplus: bool, dy: Optional[torch.Tensor],
         dnew: Optional[torch.Tensor]) -> list[torch.Tensor]:
    """All tensor inputs fp32 (widened by the caller)."""
    f32 = dict(dtype=torch.float32, device=state.device)
    batch, nheads, headdim, dstate = state.shape
    p = _params(state, x, dt, A, B, C, D, z, dt_bias, softplus)
    if dy is not None:
        p.flags |= nat.HAS_DY
        p.dy = dy.data_ptr()
    if dnew is not None:
        p.flags |= nat.HAS_DSTATE
        p.dnew = dnew.data_ptr()
    ws = nat._SZ()
    nat.check(nat.lib().ssm_state_update_sizes(p, ws), "mamba2_state_update backward")
    work = torch.empty(max(ws.value, 1), dtype=torch.uint8, device=state.device)
    g_state = torch.empty(state.shape, **f32)
    dx = torch.empty(x.shape, **f32)
    ddt = torch.empty(dt.shape, **f32)
    dA = torch.empty(nheads, **f32)
    dB = torch.empty(B.shape, **f32)
    dC = torch.empty(C.shape, **f32)
    dD = torch.empty(D.shape, **f32) if D is not None else state.new_empty(0, dtype=torch.float32)
    dz = torch.empty(x.shape, **f32) if z is not None else state.new_empty(0, dtype=torch.float32)
    dbias = torch.empty(nheads, **f32) if dt_bias is not None else state.new_empty(0, dtype=torch.float32)
    p.grad_state, p.dx, p.ddt, p.dA = g_state.data_ptr(), dx.data_ptr(), ddt.data_ptr(), dA.data_ptr()
    p.dB, p.dC = dB.data_ptr(), dC.data_ptr()
    p.dD = dD.data_ptr() if D is not None else None
    p.dz = dz.data_ptr() if z is not None else None
    p.ddt_bias = dbias.data_ptr() if dt_bias is not None else None
    p.workspace, p.workspace_bytes = work.data_ptr(), work.numel()
    p.status = nat.status_word(state.device, "state_update")
    nat.check(nat.lib().ssm_state_update_bwd(p, nat.stream_of(state)), "mamba2_state_update backward")
    return [g_state, dx, ddt, dA, dB, dC, dD, dz, dbias]


@_bwd.register_fake
def _(state, x, dt, A, B, C, D, z, dt_bias, softplus, dy, dnew):
    f = lambda t: t.new_empty(t.shape, dtype=torch.float32)  # noqa: E731
    e = state.new_empty(0, dtype=torch.float32)
    return [f(state), f(x), f(dt), f(A), f(B), f(C), f(D) if D is not None else e,
            f(x) if z is not None else e, f(A) if dt_bias is not None else e]


class _StateUpdate(torch.autograd.Function):
    """Autograd wrapper (reference ``_StateUpdate``, :640-756)."""

    @staticmethod
    def forward(ctx, state, x, dt, A, B, C, D, z, dt_bias, softplus):
        y, new_state = torch.ops.b200ssm.state_update_fwd(state, x, dt, A, B, C, D, z,
                                                          dt_bias, softplus)
        ctx.softplus = softplus
        ctx.set_materialize_grads(False)
        ctx.save_for_backward(state, x, dt, A, B, C, D, z, dt_bias)
        return y, new_state

    @staticmethod
    @torch.autograd.function.once_differentiable
    def backward(ctx, dy, dnew):
        state, x, dt, A, B, C, D, z, dt_bias = ctx.saved_tensors
        wide = lambda t: None if t is None else t.float().contiguous()  # noqa: E731
        grads = torch.ops.b200ssm.state_update_bwd(
            wide(state), wide(x), wide(dt), A, wide(B), wide(C), D, wide(z), dt_bias,
            ctx.softplus, wide(dy), wide(dnew))
        g_state, dx, ddt, dA, dB, dC, dD, dz, dbias = grads
        narrow = lambda g, ref: None if ref is None else g.to(ref.dtype)  # noqa: E731
        return (narrow(g_state, state), narrow(dx, x), narrow(ddt, dt), narrow(dA, A),
                narrow(dB, B), narrow(dC, C), narrow(dD, D), narrow(dz, z),
                narrow(dbias, dt_bias), None)


def _check(state, x, dt, A, B, C, D, z, dt_bias, out_state):
    # same contract and messages as the reference's _check (:565-598)
    if state.dim() != 4:
        raise ValueError(f"state must be (batch, nheads, dim, dstate), got {tuple(state.shape)}")
    batch, nheads, dim, dstate = state.shape
    if dstate < 1:
        raise ValueError("state must have a non-empty last dimension")
    expected = (batch, nheads, dim)
    for name, t in (("x", x), ("z", z)):
        if t is not None and tuple(t.shape) != expected:
            raise ValueError(f"{name} must be {expected}, got {tuple(t.shape)}")
    if tuple(dt.shape) not in ((batch, nheads), expected):
        raise ValueError(f"dt must be {(batch, nheads)} or {expected}, got {tuple(dt.shape)}")
    if tuple(A.shape) != (nheads,):
        raise ValueError(f"A must be {(nheads,)}, got {tuple(A.shape)}")
    if B.dim() != 3:
        raise ValueError(f"B must be (batch, ngroups, dstate), got {tuple(B.shape)}")
    groups = B.shape[1]
    if tuple(B.shape) != (batch, groups, dstate) or tuple(C.shape) != tuple(B.shape):
        raise ValueError(f"B and C must be {(batch, groups, dstate)}, got {tuple(B.shape)}, {tuple(C.shape)}")
    if groups < 1 or nheads % groups:
        raise ValueError(f"nheads ({nheads}) must be divisible by ngroups ({groups})")
    if D is not None and tuple(D.shape) not in ((nheads,), (nheads, dim)):
        raise ValueError(f"D must be {(nheads,)} or {(nheads, dim)}, got {tuple(D.shape)}")
    if dt_bias is not None and tuple(dt_bias.shape) != (nheads,):
        raise ValueError(f"dt_bias must be {(nheads,)}, got {tuple(dt_bias.shape)}")
    if out_state is not None:
        if out_state.device != state.device:
            raise ValueError("out_state must be on the same device as state")
        if tuple(out_state.shape) != tuple(state.shape) or out_state.dtype != state.dtype:
            raise ValueError("out_state must match state in shape and dtype")
        if not out_state.is_contiguous():
            raise ValueError("out_state must be contiguous")
        if out_state.requires_grad:
            raise ValueError("out_state is written in place and cannot require grad")


def mamba2_state_update(state, x, dt, A, B, C, D=None, z=None, dt_bias=None,
                        dt_softplus=False, out_state=None):
    """One Mamba-2 selective state update step on the GPU.

    Same arguments and return as the reference's ``mamba2_state_update``
    (cv/mamba2_state.py:759-819): returns ``(y, updated_state)``; without
    ``out_state`` the input ``state`` is untouched and ``updated_state`` is a
    fresh tensor, with it ``updated_state`` shares ``out_state``'s storage.
    """
    _check(state, x, dt, A, B, C, D, z, dt_bias, out_state)
    for name, t in (("state", state), ("x", x), ("dt", dt), ("A", A), ("B", B), ("C", C),
                    ("D", D), ("z", z), ("dt_bias", dt_bias)):
        if t is not None and t.device.type != "cuda":
            raise ValueError(f"mamba2_state_update runs CUDA kernels, {name} is on {t.device}")
        if t is not None and t.device != state.device:
            raise ValueError(f"{name} is on {t.device}, state is on {state.device}")
    if state.dtype not in _DTYPES:
        raise ValueError(f"state must be float32, float16 or bfloat16, got {state.dtype}")
    dtype = state.dtype
    needs_grad = torch.is_grad_enabled() and any(
        t is not None and t.requires_grad for t in (state, x, dt, A, B, C, D, z, dt_bias))
    # The forward kernel reads 16-bit x, B, C (and z) against an fp32 state
    # directly; everything else is brought to the state's dtype.
    io = (not needs_grad and dtype == torch.float32 and x.dtype in (torch.bfloat16, torch.float16)
          and B.dtype == x.dtype and C.dtype == x.dtype and (z is None or z.dtype == x.dtype))
    if io:
        dt = dt.to(dtype)
    else:
        x, dt, B, C = (t.to(dtype) for t in (x, dt, B, C))
        z = z.to(dtype) if z is not None else None
    A = A.float()
    D = D.float() if D is not None else None
    dt_bias = dt_bias.float() if dt_bias is not None else None
    x, dt, B, C, A = (t.contiguous() for t in (x, dt, B, C, A))
    z = z.contiguous() if z is not None else None
    D = D.contiguous() if D is not None else None
    dt_bias = dt_bias.contiguous() if dt_bias is not None else None
    state_c = state.contiguous()

    if not needs_grad:
        if out_state is None:
            return torch.ops.b200ssm.state_update_fwd(state_c, x, dt, A, B, C, D, z, dt_bias,
                                                      bool(dt_softplus))
        y = torch.ops.b200ssm.state_update_into(state_c, x, dt, A, B, C, D, z, dt_bias,
                                                bool(dt_softplus), out_state)
        return y, out_state
    if out_state is not None and \
            out_state.untyped_storage().data_ptr() == state.untyped_storage().data_ptr():
        state_c = state_c.clone()   # the backward needs the entering state
    y, new_state = _StateUpdate.apply(state_c, x, dt, A, B, C, D, z, dt_bias, bool(dt_softplus))
    if out_state is None:
        return y, new_state
    # Differentiable path with a destination: the backward keeps the entering
    # state it saved (a fresh tensor), and the destination receives a copy, so
    # aliasing `state` is safe whichever inputs require grad.  The copy is
    # recorded by autograd, so a loss on the returned state still reaches the
    # inputs.
    out_state.copy_(new_state)
    return y, out_state
