"""Causal depthwise conv1d on the B200: the convolution every Mamba block runs
before its scan.

Drop-in for ``metal_kernelops.cv.causal_conv1d`` (src/metal_kernelops/cv/
causal_conv1d.py of the reference), same names, arguments, layouts and error
convention:

* ``causal_conv1d_fn(x, weight, bias=None, activation=None, initial_state=None,
  return_final_state=False)`` -- prefill over a whole sequence, with autograd
  for x, weight, bias and initial_state (:610-690).
* ``causal_conv1d_update(x, state, weight, bias=None, activation=None)`` --
  decode: one or a few tokens against a rolling state updated in place; no
  autograd (:690-756).

With ``z = cat(initial_state, x)`` (zeros without a state) and K the weight
width: ``out[t] = act(bias + sum_j weight[:, j] * z[t + j])`` and
``final_state = z[..., L : L + K - 1]``; ``act`` is None or SiLU
(``"silu"``/``"swish"``).

Layouts: x ``(batch, channels, length)`` (any strides; made contiguous);
weight ``(channels, 1, K)`` or ``(channels, K)``; bias ``(channels,)``;
initial_state ``(batch, channels, K - 1)``; the decode state
``(batch, channels, s >= K - 1)`` with last stride 1 (a cache slice is read and
written through its strides).  x may be float32, bfloat16 or float16; the
arithmetic is float32 and the result comes back in ``x.dtype``.  K is 1..8.
CUDA tensors only.

On the device (``csrc/causal_conv1d.cu``): one forward kernel (16-byte vector
tiles, fused bias, SiLU and final state), one backward kernel that recomputes
the pre-activation from x and produces dx, the initial-state gradient and
per-CTA dweight/dbias partials, a fold of the partials per channel (fixed
order, bit-reproducible), and one decode kernel.
"""

from __future__ import annotations

from typing import Optional

import torch

from .. import _native as nat

__all__ = ["causal_conv1d_fn", "causal_conv1d_update"]

_ACTIVATIONS = (None, "silu", "swish")
_DTYPES = (torch.float32, torch.bfloat16, torch.float16)
MAX_WIDTH = 8
"""Widest kernel the CUDA kernels are built for."""


def _as_depthwise(weight):
    """(channels, 1, K) or (channels, K) -> (channels, K) (reference :414-429)."""
    if weight.dim() == 3:
        if weight.shape[1] != 1:
            raise ValueError("weight must be (channels, 1, K) for a depthwise convolution, "
                             f"got {tuple(weight.shape)}")
        weight = weight[:, 0, :]
    elif weight.dim() != 2:
        raise ValueError(f"weight must be (channels, 1, K) or (channels, K), got {tuple(weight.shape)}")
    if weight.shape[1] < 1:
        raise ValueError("the kernel width must be at least 1")
    return weight


def _check_activation(activation):
    if activation not in _ACTIVATIONS:
        raise NotImplementedError(f"activation must be one of {_ACTIVATIONS}, got {activation!r}")


def _check_device(name, t, ref):
    if t.device.type != "cuda":
        raise ValueError(f"causal_conv1d runs CUDA kernels, {name} is on {t.device}")
    if t.device != ref.device:
        raise ValueError(f"causal_conv1d: {name} is on {t.device}, x is on {ref.device}")
    if not t.is_floating_point():
        raise ValueError(f"causal_conv1d: {name} must be floating point, got {t.dtype}")


def _params(x, weight, bias, init, silu):
    batch, channels, length = x.shape
    p = nat.CausalConv1dParams()
    p.batch, p.channels, p.length, p.width = batch, channels, length, weight.shape[1]
    p.dtype = nat.dtype_code(x.dtype)
    p.flags = ((nat.HAS_BIAS if bias is not None else 0) | (nat.HAS_INIT if init is not None else 0)
               | (nat.CONV_SILU if silu else 0))
    p.x, p.weight = x.data_ptr(), weight.data_ptr()
    p.bias = bias.data_ptr() if bias is not None else None
    p.initial_state = init.data_ptr() if init is not None else None
    return p


@torch.library.custom_op("b200ssm::causal_conv1d_fwd", mutates_args=(), device_types="cuda")
def _fwd(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor],
         init: Optional[torch.Tensor], silu: bool, want_final: bool) -> tuple[torch.Tensor, torch.Tensor]:
    p = _params(x, weight, bias, init, silu)
    out = torch.empty_like(x)
    final = x.new_empty((x.shape[0], x.shape[1], weight.shape[1] - 1) if want_final else (0,))
    p.out = out.data_ptr()
    p.final_state = final.data_ptr() if want_final and final.numel() else None
    p.status = nat.status_word(x.device, "causal_conv1d")
    nat.check(nat.lib().ssm_causal_conv1d_fwd(p, nat.stream_of(x)), "causal_conv1d")
    return out, final


@_fwd.register_fake
def _(x, weight, bias, init, silu, want_final):
    return (torch.empty_like(x),
            x.new_empty((x.shape[0], x.shape[1], weight.shape[1] - 1) if want_final else (0,)))


@torch.library.custom_op("b200ssm::causal_conv1d_bwd", mutates_args=(), device_types="cuda")
def _bwd(dout: torch.Tensor, x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor],
         init: Optional[torch.Tensor], silu: bool
         ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    p = _params(x, weight, bias, init, silu)
    ws_bytes = nat._SZ()
    nat.check(nat.lib().ssm_causal_conv1d_sizes(p, ws_bytes), "causal_conv1d backward")
    dx = torch.empty_like(x)
    dweight = torch.empty(weight.shape, dtype=torch.float32, device=x.device)
    dbias = torch.empty(weight.shape[0] if bias is not None else 0, dtype=torch.float32, device=x.device)
    dinit = torch.empty_like(init) if init is not None else x.new_empty(0)
    ws = torch.empty(max(ws_bytes.value, 1), dtype=torch.uint8, device=x.device)
    p.dout, p.dx = dout.data_ptr(), dx.data_ptr()
    p.dweight = dweight.data_ptr()
    p.dbias = dbias.data_ptr() if bias is not None else None
    p.dinitial = dinit.data_ptr() if init is not None and dinit.numel() else None
    p.workspace, p.workspace_bytes = ws.data_ptr(), ws.numel()
    p.status = nat.status_word(x.device, "causal_conv1d")
    nat.check(nat.lib().ssm_causal_conv1d_bwd(p, nat.stream_of(x)), "causal_conv1d backward")
    return dx, dweight, dbias, dinit


@_bwd.register_fake
def _(dout, x, weight, bias, init, silu):
    f32 = dict(dtype=torch.float32)
    return (torch.empty_like(x), weight.new_empty(weight.shape, **f32),
            weight.new_empty(weight.shape[0] if bias is not None else 0, **f32),
            torch.empty_like(init) if init is not None else x.new_empty(0))


def _setup(ctx, inputs, output):
    x, weight, bias, init, silu, want_final = inputs
    ctx.save_for_backward(x, weight, bias, init)
    ctx.silu = silu
    ctx.set_materialize_grads(False)     # no zero-filled gradient for the final state


def _backward(ctx, dout, dfinal):
    x, weight, bias, init = ctx.saved_tensors
    if dout is None:
        return (None,) * 6
    dx, dweight, dbias, dinit = _bwd(dout.contiguous(), x, weight, bias, init, ctx.silu)
    return (dx, dweight, dbias if bias is not None else None,
            dinit if init is not None else None, None, None)


_fwd.register_autograd(_backward, setup_context=_setup)


# --------------------------------------------------------- channel-last path --
# x given as a (batch, channels, length) view of (batch, length, channels)
# memory -- the transpose of a Mamba block's input-projection output, possibly
# a column slice of it -- runs on kernels that read that layout directly, so
# the operand is never copied; the output comes back as the same kind of view.

def _cl_rows(t):
    """(batch, length, channels) tensor t usable by the channel-last kernels:
    unit channel stride, evenly spaced rows, 8-byte aligned."""
    b, length, c = t.shape
    es = t.element_size()
    if t.stride(2) != 1 or (c * es) % 8 or t.data_ptr() % 8:
        return False
    rs = t.stride(1) if length > 1 else c
    if rs < c or (rs * es) % 8:
        return False
    return b <= 1 or t.stride(0) == length * rs


def _params_cl(xt, weight, bias, silu):
    p = nat.CausalConv1dParams()
    p.batch, p.length, p.channels = xt.shape
    p.width = weight.shape[1]
    p.dtype = nat.dtype_code(xt.dtype)
    p.flags = nat.CHANNEL_LAST | (nat.HAS_BIAS if bias is not None else 0) | (nat.CONV_SILU if silu else 0)
    p.x, p.weight = xt.data_ptr(), weight.data_ptr()
    p.bias = bias.data_ptr() if bias is not None else None
    p.x_row_stride = xt.stride(1) if xt.shape[1] > 1 else 0
    return p


@torch.library.custom_op("b200ssm::causal_conv1d_cl_fwd", mutates_args=(), device_types="cuda")
def _fwd_cl(xt: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor], silu: bool) -> torch.Tensor:
    """xt: (batch, length, channels) with unit channel stride; the result is dense."""
    p = _params_cl(xt, weight, bias, silu)
    out = xt.new_empty(xt.shape)
    p.out = out.data_ptr()
    p.status = nat.status_word(xt.device, "causal_conv1d")
    nat.check(nat.lib().ssm_causal_conv1d_fwd(p, nat.stream_of(xt)), "causal_conv1d")
    return out


@_fwd_cl.register_fake
def _(xt, weight, bias, silu):
    return xt.new_empty(xt.shape)


@torch.library.custom_op("b200ssm::causal_conv1d_cl_bwd", mutates_args=(), device_types="cuda")
def _bwd_cl(dout: torch.Tensor, xt: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor],
            silu: bool) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    p = _params_cl(xt, weight, bias, silu)
    p.dout_row_stride = dout.stride(1) if dout.shape[1] > 1 else 0
    ws_bytes = nat._SZ()
    nat.check(nat.lib().ssm_causal_conv1d_sizes(p, ws_bytes), "causal_conv1d backward")
    dx = xt.new_empty(xt.shape)
    dweight = torch.empty(weight.shape, dtype=torch.float32, device=xt.device)
    dbias = torch.empty(weight.shape[0] if bias is not None else 0, dtype=torch.float32, device=xt.device)
    ws = torch.empty(max(ws_bytes.value, 1), dtype=torch.uint8, device=xt.device)
    p.dout, p.dx = dout.data_ptr(), dx.data_ptr()
    p.dweight = dweight.data_ptr()
    p.dbias = dbias.data_ptr() if bias is not None else None
    p.workspace, p.workspace_bytes = ws.data_ptr(), ws.numel()
    p.status = nat.status_word(xt.device, "causal_conv1d")
    nat.check(nat.lib().ssm_causal_conv1d_bwd(p, nat.stream_of(xt)), "causal_conv1d backward")
    return dx, dweight, dbias


@_bwd_cl.register_fake
def _(dout, xt, weight, bias, silu):
    f32 = dict(dtype=torch.float32)
    return (xt.new_empty(xt.shape), weight.new_empty(weight.shape, **f32),
            weight.new_empty(weight.shape[0] if bias is not None else 0, **f32))


def _setup_cl(ctx, inputs, output):
    xt, weight, bias, silu = inputs
    ctx.save_for_backward(xt, weight, bias)
    ctx.silu = silu


def _backward_cl(ctx, dout):
    xt, weight, bias = ctx.saved_tensors
    if not _cl_rows(dout):
        dout = dout.contiguous()
    dx, dweight, dbias = _bwd_cl(dout, xt, weight, bias, ctx.silu)
    return dx, dweight, dbias if bias is not None else None, None


_fwd_cl.register_autograd(_backward_cl, setup_context=_setup_cl)


def _final_state(x, init, taps):
    """The last ``taps`` columns of ``cat(init, x)`` (reference :468-477), through
    torch ops so that gradients reach x and init."""
    length = x.shape[-1]
    if length >= taps:
        return x[..., length - taps:].contiguous()
    head = init[..., length:] if init is not None else x.new_zeros(x.shape[:-1] + (taps - length,))
    return torch.cat([head, x], dim=-1)


def causal_conv1d_fn(x, weight, bias=None, activation=None, initial_state=None, return_final_state=False):
    """Causal depthwise conv1d over a whole sequence (reference :610-690).

    Returns ``(batch, channels, length)`` in ``x.dtype``, or ``(out,
    final_state)`` with ``final_state`` of shape ``(batch, channels, K - 1)``.
    """
    weight = _as_depthwise(weight)
    _check_activation(activation)
    if x.dim() != 3:
        raise ValueError(f"x must be (batch, channels, length), got {tuple(x.shape)}")
    channels, width = weight.shape
    if x.shape[1] != channels:
        raise ValueError(f"x has {x.shape[1]} channels, weight has {channels}")
    if bias is not None and (bias.dim() != 1 or bias.shape[0] != channels):
        raise ValueError(f"bias must be ({channels},), got {tuple(bias.shape)}")
    if initial_state is not None:
        expected = (x.shape[0], channels, width - 1)
        if tuple(initial_state.shape) != expected:
            raise ValueError(f"initial_state must be {expected}, got {tuple(initial_state.shape)}")
    for name, t in (("x", x), ("weight", weight), ("bias", bias), ("initial_state", initial_state)):
        if t is not None:
            _check_device(name, t, x)
    if x.dtype not in _DTYPES:
        raise ValueError(f"causal_conv1d computes float32/bfloat16/float16, x is {x.dtype}")
    if width > MAX_WIDTH:
        raise ValueError(f"causal_conv1d: kernel width must be at most {MAX_WIDTH}, got {width}")
    taps = width - 1
    silu = activation is not None
    if initial_state is None and x.numel() and x.shape[2] > 1 and _cl_rows(x.transpose(1, 2)):
        w32 = weight.float().contiguous()
        b32 = bias.float().contiguous() if bias is not None else None
        out = torch.ops.b200ssm.causal_conv1d_cl_fwd(x.transpose(1, 2), w32, b32, silu).transpose(1, 2)
        if return_final_state:
            return out, _final_state(x, None, taps)
        return out
    work = x.contiguous()
    # a width-1 kernel has no state: (batch, channels, 0) carries nothing
    init = initial_state.to(x.dtype).contiguous() if initial_state is not None and taps else None
    w32 = weight.float().contiguous()
    b32 = bias.float().contiguous() if bias is not None else None
    grads = torch.is_grad_enabled() and any(
        t is not None and t.requires_grad for t in (x, weight, bias, initial_state))
    if work.numel() == 0:
        out = work.new_empty(work.shape)
        if return_final_state:
            return out, _final_state(work, init, taps)
        return out
    if return_final_state and not grads:
        out, final = torch.ops.b200ssm.causal_conv1d_fwd(work, w32, b32, init, silu, True)
        return out, final
    out, _ = torch.ops.b200ssm.causal_conv1d_fwd(work, w32, b32, init, silu, False)
    if return_final_state:
        return out, _final_state(work, init, taps)
    return out


@torch.library.custom_op("b200ssm::causal_conv1d_update", mutates_args=("state",), device_types="cuda")
def _update(x: torch.Tensor, state: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor],
            silu: bool) -> torch.Tensor:
    batch, channels, length = x.shape
    out = torch.empty_like(x)
    p = nat.CausalConv1dUpdateParams()
    p.batch, p.channels, p.length, p.width = batch, channels, length, weight.shape[1]
    p.state_len = state.shape[-1]
    p.state_stride_batch, p.state_stride_channel = state.stride(0), state.stride(1)
    p.dtype = nat.dtype_code(x.dtype)
    p.flags = (nat.HAS_BIAS if bias is not None else 0) | (nat.CONV_SILU if silu else 0)
    p.state, p.x, p.weight = state.data_ptr(), x.data_ptr(), weight.data_ptr()
    p.bias = bias.data_ptr() if bias is not None else None
    p.out = out.data_ptr()
    p.status = nat.status_word(x.device, "causal_conv1d_update")
    nat.check(nat.lib().ssm_causal_conv1d_update(p, nat.stream_of(x)), "causal_conv1d_update")
    return out


@_update.register_fake
def _(x, state, weight, bias, silu):
    return torch.empty_like(x)


def causal_conv1d_update(x, state, weight, bias=None, activation=None):
    """Advance the causal convolution by ``q`` tokens, updating ``state`` in
    place with ``cat(state, x)[..., -s:]`` (reference :690-756).

    x is ``(batch, channels)`` or ``(batch, channels, q)``; the result has the
    rank of x.  Decode only: raises ``RuntimeError`` if anything requires grad.
    """
    weight = _as_depthwise(weight)
    _check_activation(activation)
    squeezed = x.dim() == 2
    if squeezed:
        x = x.unsqueeze(-1)
    if x.dim() != 3:
        raise ValueError(f"x must be (batch, channels) or (batch, channels, q), got {tuple(x.shape)}")
    channels, width = weight.shape
    taps = width - 1
    batch, xchannels, length = x.shape
    if xchannels != channels:
        raise ValueError(f"x has {xchannels} channels, weight has {channels}")
    if state.dim() != 3 or state.shape[0] != batch or state.shape[1] != channels:
        raise ValueError(f"state must be ({batch}, {channels}, s) with s >= {taps}, got {tuple(state.shape)}")
    span = state.shape[-1]
    if span < taps:
        raise ValueError(f"state must hold at least K-1 = {taps} columns, got {span}")
    if state.stride(-1) != 1:
        raise ValueError(f"state must have stride 1 in its last dimension, got {state.stride()}")
    if bias is not None and (bias.dim() != 1 or bias.shape[0] != channels):
        raise ValueError(f"bias must be ({channels},), got {tuple(bias.shape)}")
    if x.requires_grad or weight.requires_grad or state.requires_grad:
        raise RuntimeError("causal_conv1d_update is the decode path and carries no autograd")
    for name, t in (("x", x), ("state", state), ("weight", weight), ("bias", bias)):
        if t is not None:
            _check_device(name, t, x)
    if state.dtype not in _DTYPES:
        raise ValueError(f"causal_conv1d_update: state must be float32/bfloat16/float16, got {state.dtype}")
    if width > MAX_WIDTH:
        raise ValueError(f"causal_conv1d: kernel width must be at most {MAX_WIDTH}, got {width}")
    work = x.to(state.dtype).contiguous()
    if work.numel() == 0:
        out = x.new_empty(x.shape)
        return out.squeeze(-1) if squeezed else out
    b32 = bias.float().contiguous() if bias is not None else None
    out = torch.ops.b200ssm.causal_conv1d_update(work, state, weight.float().contiguous(), b32,
                                                 activation is not None)
    out = out.to(x.dtype)
    return out.squeeze(-1) if squeezed else out
