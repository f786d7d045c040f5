"""Gated RMSNorm on the B200: the normalisation Mamba-2 runs after its SSD scan.

Drop-in for ``metal_kernelops.cv.gated_norm.rmsnorm_gated`` (src/metal_kernelops/
cv/gated_norm.py:647-686): same signature, arguments, defaults, shape contract
and ``ValueError`` messages.  mamba_ssm's ``rms_norm_ref`` semantics: with
``gate = silu(z)``,

    x'  = x * gate                       if z is given and not norm_before_gate
    r   = rsqrt(mean(x'^2 over the group) + eps)
    y   = x' * r * weight + bias
    out = y * gate                       if z is given and norm_before_gate

the mean over the last ``group_size`` features (the whole axis when None).
All intermediates are float32; the result is in ``x.dtype``.  x (and z) may be
float32, bfloat16 or float16, any leading shape; weight and bias any float
dtype (their gradients come back in their own dtypes).  CUDA tensors only.

On the device (``csrc/gated_norm.cu``): one forward kernel (a warp per
(row, group) for groups of up to 1024 bf16 / 512 fp32 elements, a CTA
streaming each row twice for wider ones) that also saves the per-(row, group)
``rsqrt`` for the backward, one analytic backward kernel with deterministic
per-row-block dweight/dbias partials, and a fixed-order fold of the partials.
"""

from __future__ import annotations

from typing import Optional

import torch

from .. import _native as nat

__all__ = ["rmsnorm_gated"]

_DTYPES = (torch.float32, torch.bfloat16, torch.float16)
_GATE_NONE, _GATE_BEFORE, _GATE_AFTER = 0, 1, 2


def _params(x, weight, bias, z, eps, group, gate):
    rows, features = x.shape
    p = nat.GatedRmsNormParams()
    p.rows, p.features, p.group_size = rows, features, group
    p.dtype = nat.dtype_code(x.dtype)
    p.gate = gate
    p.flags = nat.HAS_BIAS if bias is not None else 0
    p.eps = eps
    p.x, p.weight = x.data_ptr(), weight.data_ptr()
    p.z = z.data_ptr() if z is not None else None
    # row strides (0: contiguous; a single row's stride is never used)
    p.x_row_stride = x.stride(0) if x.shape[0] > 1 else 0
    p.z_row_stride = z.stride(0) if z is not None and z.shape[0] > 1 else 0
    p.bias = bias.data_ptr() if bias is not None else None
    return p


@torch.library.custom_op("b200ssm::gated_rmsnorm_fwd", mutates_args=(), device_types="cuda")
def _fwd(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor], z: Optional[torch.Tensor],
         eps: float, group: int, gate: int, save: bool) -> tuple[torch.Tensor, torch.Tensor]:
    p = _params(x, weight, bias, z, eps, group, gate)
    out = torch.empty(x.shape, dtype=x.dtype, device=x.device)
    rstd = torch.empty((x.shape[0] * (x.shape[1] // group)) if save else 0, dtype=torch.float32,
                       device=x.device)
    p.out = out.data_ptr()
    p.rstd = rstd.data_ptr() if save and rstd.numel() else None
    p.status = nat.status_word(x.device, "gated_rmsnorm")
    nat.check(nat.lib().ssm_gated_rmsnorm_fwd(p, nat.stream_of(x)), "rmsnorm_gated")
    return out, rstd


@_fwd.register_fake
def _(x, weight, bias, z, eps, group, gate, save):
    return x.new_empty(x.shape), x.new_empty((x.shape[0] * (x.shape[1] // group)) if save else 0,
                                             dtype=torch.float32)


@torch.library.custom_op("b200ssm::gated_rmsnorm_bwd", mutates_args=(), device_types="cuda")
def _bwd(dy: torch.Tensor, x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor],
         z: Optional[torch.Tensor], rstd: torch.Tensor, eps: float, group: int,
         gate: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    p = _params(x, weight, bias, z, eps, group, gate)
    ws_bytes = nat._SZ()
    nat.check(nat.lib().ssm_gated_rmsnorm_sizes(p, ws_bytes), "rmsnorm_gated backward")
    dx = x.new_empty(x.shape)
    dz = z.new_empty(z.shape) if z is not None else x.new_empty(0)
    dw = torch.empty(x.shape[1], dtype=torch.float32, device=x.device)
    db = torch.empty(x.shape[1] if bias is not None else 0, dtype=torch.float32, device=x.device)
    ws = torch.empty(max(ws_bytes.value, 1), dtype=torch.uint8, device=x.device)
    p.rstd = rstd.data_ptr()
    p.dy, p.dx = dy.data_ptr(), dx.data_ptr()
    p.dz = dz.data_ptr() if z is not None else None
    p.dweight = dw.data_ptr()
    p.dbias = db.data_ptr() if bias is not None else None
    p.workspace, p.workspace_bytes = ws.data_ptr(), ws.numel()
    p.status = nat.status_word(x.device, "gated_rmsnorm")
    nat.check(nat.lib().ssm_gated_rmsnorm_bwd(p, nat.stream_of(x)), "rmsnorm_gated backward")
    return dx, dw, db, dz


@_bwd.register_fake
def _(dy, x, weight, bias, z, rstd, eps, group, gate):
    f32 = dict(dtype=torch.float32)
    return (x.new_empty(x.shape), x.new_empty(x.shape[1], **f32),
            x.new_empty(x.shape[1] if bias is not None else 0, **f32),
            z.new_empty(z.shape) if z is not None else x.new_empty(0))


def _setup(ctx, inputs, output):
    x, weight, bias, z, eps, group, gate, save = inputs
    _, rstd = output
    ctx.save_for_backward(x, weight, bias, z, rstd)
    ctx.eps, ctx.group, ctx.gate = eps, group, gate
    ctx.set_materialize_grads(False)     # no zero-filled gradient for rstd


def _backward(ctx, dout, drstd):
    x, weight, bias, z, rstd = ctx.saved_tensors
    if rstd.numel() == 0 and x.numel() != 0:
        raise RuntimeError("rmsnorm_gated: the forward did not save its statistics (save=False)")
    if dout is None:
        return (None,) * 8
    dx, dw, db, dz = _bwd(dout.contiguous(), x, weight, bias, z, rstd, ctx.eps, ctx.group, ctx.gate)
    return (dx, dw, db if bias is not None else None, dz if z is not None else None,
            None, None, None, None)


_fwd.register_autograd(_backward, setup_context=_setup)


def _rows(t, features):
    """t as (rows, features) with contiguous features: a view when its rows are
    evenly spaced and do not overlap (a column slice of a wider projection
    output, say), else a contiguous copy."""
    t2 = t.reshape(-1, features)
    if t2.stride(1) == 1 and (t2.shape[0] <= 1 or t2.stride(0) >= features):
        return t2
    return t2.contiguous()


def rmsnorm_gated(x, weight, bias=None, z=None, eps=1e-5, group_size=None, norm_before_gate=True):
    """Gated RMSNorm over the last axis, as in ``mamba_ssm``'s ``RMSNorm``
    (reference :647-686).

    Args:
        x: ``(..., features)``.
        weight: ``(features,)`` scale.
        bias: ``(features,)`` shift, added before the gate.
        z: same shape as ``x``; ``silu(z)`` multiplies the normalised output
            (``norm_before_gate=True``) or the input before normalisation.
        eps: added to the mean square before ``rsqrt``.
        group_size: features per normalisation group (None: the whole axis);
            must divide ``features``.
        norm_before_gate: whether the gate is applied after normalisation.

    Returns:
        ``(..., features)`` in ``x.dtype``.
    """
    if x.dim() < 1:
        raise ValueError("rmsnorm_gated needs a feature axis")
    features = x.shape[-1]
    if features == 0:
        return x.clone()
    group = features if group_size is None else int(group_size)
    if group <= 0 or features % group:
        raise ValueError(f"group_size {group} does not divide {features}")
    if weight.shape != (features,):
        raise ValueError(f"weight must be ({features},), got {tuple(weight.shape)}")
    if bias is not None and bias.shape != (features,):
        raise ValueError(f"bias must be ({features},), got {tuple(bias.shape)}")
    if z is not None and z.shape != x.shape:
        raise ValueError(f"z must match x {tuple(x.shape)}, got {tuple(z.shape)}")
    for name, t in (("x", x), ("weight", weight), ("bias", bias), ("z", z)):
        if t is None:
            continue
        if t.device.type != "cuda":
            raise ValueError(f"rmsnorm_gated runs CUDA kernels, {name} is on {t.device}")
        if t.device != x.device:
            raise ValueError(f"rmsnorm_gated: {name} is on {t.device}, x is on {x.device}")
    if x.dtype not in _DTYPES:
        raise ValueError(f"rmsnorm_gated computes float32/bfloat16/float16, x is {x.dtype}")
    if x.numel() == 0:
        return x.new_empty(x.shape)
    shape = x.shape
    x2 = _rows(x, features)
    z2 = _rows(z.to(x.dtype), features) if z is not None else None
    w32 = weight.float().contiguous()
    b32 = bias.float().contiguous() if bias is not None else None
    gate = _GATE_NONE if z is None else (_GATE_AFTER if norm_before_gate else _GATE_BEFORE)
    save = torch.is_grad_enabled() and any(t is not None and t.requires_grad for t in (x, weight, bias, z))
    out, _ = torch.ops.b200ssm.gated_rmsnorm_fwd(x2, w32, b32, z2, float(eps), group, gate, bool(save))
    return out.reshape(shape)
