"""Mamba-1 selective scan on the B200: the drop-in for ``metal_kernelops.scan``.

Public surface (same names, arguments, layouts and error convention as
src/metal_kernelops/scan.py:283-329 of the reference):

* ``selective_scan(u, dt, A, B, C, D=None, z=None, delta_bias=None,
  delta_softplus=False)`` and its alias ``selective_scan_fn`` -- the full op:
  bias add, softplus, the scan, ``+ u*D`` and ``* silu(z)``.  In the reference
  the epilogue is four extra torch ops (scan.py:311-319); here it is fused
  into the scan kernel, and so is its backward.
* ``scan_cuda(u, dt, A, B, C)`` -- the bare scan, the counterpart of the
  reference's ``scan_mps`` (scan.py:283-292).

Layouts (scan.py:299-306): u, dt, z (batch, dim, length); A (dim, dstate);
B, C (batch, groups, dstate, length) with groups dividing dim; D and
delta_bias (dim,).  u/dt/z may be float32, bfloat16 or float16 (dt and z are
cast to u's dtype); B and C float32/bfloat16/float16; A, D and delta_bias are
read as float32.  All arithmetic is float32.  Non-CUDA tensors raise
``ValueError`` (the reference raises the same for non-MPS tensors,
scan.py:285-286); there is no CPU path.

The ops are registered as ``torch.library`` custom ops on the CUDA dispatch
key (``b200ssm::selective_scan_fwd`` / ``_bwd``) with fake kernels and an
autograd formula, so they compose with autograd, ``torch.compile`` tracing and
CUDA graphs.
"""

from __future__ import annotations

from typing import Optional

import torch

from . import _native as nat

CHUNK = 16
"""Steps per chunk of the backward's reverse walk."""
SUB_BLOCK = 4
"""Steps between the states the forward saves for the backward."""

__all__ = ["CHUNK", "selective_scan", "selective_scan_fn", "scan_cuda", "set_tma_staging",
           "set_lean_backward"]

_plain_staging = False
_lean = False


def set_lean_backward(enabled: bool) -> bool:
    """Choose what the forward saves for the backward.  False (the default):
    the state entering every SUB_BLOCK steps and, with a gate, the scan output
    -- 4 * dstate / SUB_BLOCK + 2 bytes per (batch, channel, step) element at
    bf16 (18 at dstate 16).  True: only the state entering every CHUNK steps
    (4 at dstate 16); the backward replays the rest from it, at about a
    quarter more backward time.  Applies to calls made after it; each call's
    backward follows the mode of its own forward.  Returns the previous
    setting."""
    global _lean
    prev = _lean
    _lean = bool(enabled)
    return prev


def set_tma_staging(enabled: bool) -> bool:
    """Choose the kernels' tile staging: True (the default) lets every problem
    whose rows are 16-byte aligned run the TMA-staged kernels; False runs the
    plain-staging kernels everywhere.  Both compute the same results bit for
    bit.  Returns the previous setting."""
    global _plain_staging
    prev = not _plain_staging
    _plain_staging = not enabled
    return prev


def _params(u, delta, A, B, C, D, z, delta_bias, softplus, lean=False):
    batch, dim, length = u.shape
    flags = ((nat.HAS_D if D is not None else 0) | (nat.HAS_Z if z is not None else 0)
             | (nat.HAS_BIAS if delta_bias is not None else 0) | (nat.SOFTPLUS if softplus else 0)
             | (nat.SCAN_PLAIN if _plain_staging else 0) | (nat.SCAN_LEAN if lean else 0))
    p = nat.SelectiveScanParams()
    p.batch, p.dim, p.length = batch, dim, length
    p.groups, p.dstate = B.shape[1], A.shape[1]
    p.act_dtype = nat.dtype_code(u.dtype)
    p.bc_dtype = nat.dtype_code(B.dtype)
    p.flags = flags
    p.u, p.delta, p.A, p.B, p.C = (t.data_ptr() for t in (u, delta, A, B, C))
    p.D = D.data_ptr() if D is not None else None
    p.z = z.data_ptr() if z is not None else None
    p.delta_bias = delta_bias.data_ptr() if delta_bias is not None else None
    return p


def _sizes(p):
    ck, ws = nat._SZ(), nat._SZ()
    nat.check(nat.lib().ssm_selective_scan_sizes(p, ck, ws), "selective_scan")
    return ck.value, ws.value


@torch.library.custom_op("b200ssm::selective_scan_fwd", mutates_args=(), device_types="cuda")
def _fwd(u: torch.Tensor, delta: torch.Tensor, A: torch.Tensor, B: torch.Tensor,
         C: torch.Tensor, D: Optional[torch.Tensor], z: Optional[torch.Tensor],
         delta_bias: Optional[torch.Tensor], softplus: bool,
         save: bool, lean: bool = False) -> tuple[torch.Tensor, torch.Tensor]:
    p = _params(u, delta, A, B, C, D, z, delta_bias, softplus, lean)
    ck_bytes, _ = _sizes(p)
    fw = nat._SZ()
    nat.check(nat.lib().ssm_selective_scan_fwd_workspace(p, fw), "selective_scan")
    y = torch.empty_like(u)
    ckpt = torch.empty(ck_bytes // 4 if save else 0, dtype=torch.float32, device=u.device)
    ws = torch.empty(fw.value, dtype=torch.uint8, device=u.device) if fw.value else None
    p.y = y.data_ptr()
    p.checkpoints = ckpt.data_ptr() if save and ckpt.numel() else None
    if ws is not None:
        p.workspace, p.workspace_bytes = ws.data_ptr(), ws.numel()
    p.status = nat.status_word(u.device, "selective_scan")
    nat.check(nat.lib().ssm_selective_scan_fwd(p, nat.stream_of(u)), "selective_scan")
    return y, ckpt


def checkpoint_numel(batch: int, dim: int, length: int, dstate: int, act_size: int,
                     gated: bool, lean: bool = False) -> int:
    """fp32 elements of the forward's saved-for-backward buffer (the size
    ``ssm_selective_scan_sizes`` returns): the states entering every
    SUB_BLOCK-step block, then, with a gate, the scan output in the activation
    dtype, each padded to 256 bytes; in the lean mode the states entering
    every CHUNK-step chunk only."""
    every = CHUNK if lean else SUB_BLOCK
    states = batch * (-(-length // CHUNK)) * (CHUNK // every) * dim * dstate * 4
    ybytes = batch * dim * length * act_size if gated and not lean else 0
    return (-(-states // 256) * 256 + -(-ybytes // 256) * 256) // 4


@_fwd.register_fake
def _(u, delta, A, B, C, D, z, delta_bias, softplus, save, lean=False):
    batch, dim, length = u.shape
    n = checkpoint_numel(batch, dim, length, A.shape[1], u.element_size(), z is not None, lean) if save else 0
    return torch.empty_like(u), u.new_empty(n, dtype=torch.float32)


@torch.library.custom_op("b200ssm::selective_scan_bwd", mutates_args=(), device_types="cuda")
def _bwd(dout: torch.Tensor, u: torch.Tensor, delta: torch.Tensor, A: torch.Tensor,
         B: torch.Tensor, C: torch.Tensor, D: Optional[torch.Tensor], z: Optional[torch.Tensor],
         delta_bias: Optional[torch.Tensor], ckpt: torch.Tensor,
         softplus: bool, lean: bool = False) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor,
                                                      torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    p = _params(u, delta, A, B, C, D, z, delta_bias, softplus, lean)
    _, ws_bytes = _sizes(p)
    dev = u.device
    du = torch.empty_like(u)
    ddelta = torch.empty_like(u)
    dz = torch.empty_like(u) if z is not None else u.new_empty(0)
    dA = torch.empty(A.shape, dtype=torch.float32, device=dev)
    dB = torch.empty(B.shape, dtype=torch.float32, device=dev)
    dC = torch.empty(C.shape, dtype=torch.float32, device=dev)
    dD = torch.empty(u.shape[1], dtype=torch.float32, device=dev) if D is not None else u.new_empty(0)
    dbias = (torch.empty(u.shape[1], dtype=torch.float32, device=dev) if delta_bias is not None
             else u.new_empty(0))
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
    p.checkpoints = ckpt.data_ptr()
    p.dout = dout.data_ptr()
    p.du, p.ddelta = du.data_ptr(), ddelta.data_ptr()
    p.dz = dz.data_ptr() if z is not None else None
    p.dA, p.dB, p.dC = dA.data_ptr(), dB.data_ptr(), dC.data_ptr()
    p.dD = dD.data_ptr() if D is not None else None
    p.ddelta_bias = dbias.data_ptr() if delta_bias is not None else None
    p.workspace, p.workspace_bytes = ws.data_ptr(), ws.numel()
    p.status = nat.status_word(u.device, "selective_scan")
    nat.check(nat.lib().ssm_selective_scan_bwd(p, nat.stream_of(u)), "selective_scan backward")
    return du, ddelta, dA, dB, dC, dD, dz, dbias


@_bwd.register_fake
def _(dout, u, delta, A, B, C, D, z, delta_bias, ckpt, softplus, lean=False):
    f32 = dict(dtype=torch.float32)
    return (torch.empty_like(u), torch.empty_like(u), A.new_empty(A.shape, **f32),
            B.new_empty(B.shape, **f32), C.new_empty(C.shape, **f32),
            u.new_empty(u.shape[1] if D is not None else 0, **f32),
            torch.empty_like(u) if z is not None else u.new_empty(0),
            u.new_empty(u.shape[1] if delta_bias is not None else 0, **f32))


def _setup(ctx, inputs, output):
    u, delta, A, B, C, D, z, delta_bias, softplus, save = inputs[:10]
    _, ckpt = output
    ctx.save_for_backward(u, delta, A, B, C, D, z, delta_bias, ckpt)
    ctx.softplus = softplus
    ctx.lean = bool(inputs[10]) if len(inputs) > 10 else False
    # the saved-states output never receives a gradient: without this, autograd
    # would zero-fill a buffer of its size before every backward
    ctx.set_materialize_grads(False)
    ctx.flags = (D is not None, z is not None, delta_bias is not None)


def _backward(ctx, dy, dckpt):
    u, delta, A, B, C, D, z, delta_bias, ckpt = ctx.saved_tensors
    if ckpt.numel() == 0 and u.numel() != 0:
        raise RuntimeError("selective_scan: the forward did not save its states (save=False)")
    if dy is None:
        return (None,) * 11
    du, ddelta, dA, dB, dC, dD, dz, dbias = _bwd(
        dy.contiguous(), u, delta, A, B, C, D, z, delta_bias, ckpt, ctx.softplus, ctx.lean)
    has_d, has_z, has_b = ctx.flags
    return (du, ddelta, dA, dB.to(B.dtype), dC.to(C.dtype),
            dD if has_d else None, dz if has_z else None, dbias if has_b else None, None, None, None)


_fwd.register_autograd(_backward, setup_context=_setup)


_DTYPES = (torch.float32, torch.bfloat16, torch.float16)


def _prepare(u, dt, A, B, C, D, z, delta_bias, name):
    if u.dim() != 3:
        raise ValueError(f"u must be (batch, dim, length), got {tuple(u.shape)}")
    batch, dim, length = u.shape
    if tuple(dt.shape) != tuple(u.shape):
        raise ValueError(f"dt must be {tuple(u.shape)}, got {tuple(dt.shape)}")
    if A.dim() != 2 or A.shape[0] != dim:
        raise ValueError(f"A must be ({dim}, dstate), got {tuple(A.shape)}")
    dstate = A.shape[1]
    if B.dim() != 4 or tuple(C.shape) != tuple(B.shape) or B.shape[0] != batch \
            or B.shape[2] != dstate or B.shape[3] != length:
        raise ValueError(f"B and C must be ({batch}, groups, {dstate}, {length}), "
                         f"got {tuple(B.shape)} and {tuple(C.shape)}")
    groups = B.shape[1]
    if groups < 1 or dim % groups:
        raise ValueError(f"groups={groups} must divide dim={dim}")
    if z is not None and tuple(z.shape) != tuple(u.shape):
        raise ValueError(f"z must be {tuple(u.shape)}, got {tuple(z.shape)}")
    for k, t in (("D", D), ("delta_bias", delta_bias)):
        if t is not None and tuple(t.shape) != (dim,):
            raise ValueError(f"{k} must be ({dim},), got {tuple(t.shape)}")
    tensors = {"u": u, "dt": dt, "A": A, "B": B, "C": C, "D": D, "z": z, "delta_bias": delta_bias}
    for k, t in tensors.items():
        if t is not None and t.device.type != "cuda":
            raise ValueError(f"{name} runs CUDA kernels, {k} is on {t.device}")
        if t is not None and t.device != u.device:
            raise ValueError(f"{k} is on {t.device}, u is on {u.device}")
    if u.dtype not in _DTYPES:
        raise ValueError(f"{name} computes float32/bfloat16/float16 activations, got {u.dtype}")
    if B.dtype not in _DTYPES or C.dtype not in _DTYPES:
        raise ValueError(f"B and C must be float32/bfloat16/float16, got {B.dtype}, {C.dtype}")
    act = u.dtype
    u = u.contiguous()
    dt = dt.to(act).contiguous()
    z = z.to(act).contiguous() if z is not None else None
    C = C.to(B.dtype).contiguous()
    B = B.contiguous()
    A = A.float().contiguous()
    D = D.float().contiguous() if D is not None else None
    delta_bias = delta_bias.float().contiguous() if delta_bias is not None else None
    return u, dt, A, B, C, D, z, delta_bias


def selective_scan(u, dt, A, B, C, D=None, z=None, delta_bias=None, delta_softplus=False):
    """Fused selective scan matching the reference's ``selective_scan``
    (src/metal_kernelops/scan.py:295-320).

        dt'  = softplus(dt + delta_bias)       (bias / softplus optional)
        x_t  = exp(dt'_t * A) * x_{t-1} + dt'_t * B_t * u_t
        y_t  = <x_t, C_t> + u_t * D
        out  = y * silu(z)                     (gate optional)

    Returns ``(batch, dim, length)`` in ``u.dtype``.
    """
    u, dt, A, B, C, D, z, delta_bias = _prepare(u, dt, A, B, C, D, z, delta_bias, "selective_scan")
    save = torch.is_grad_enabled() and any(
        t is not None and t.requires_grad for t in (u, dt, A, B, C, D, z, delta_bias))
    y, _ = torch.ops.b200ssm.selective_scan_fwd(u, dt, A, B, C, D, z, delta_bias,
                                                bool(delta_softplus), bool(save), _lean)
    return y


selective_scan_fn = selective_scan


def scan_cuda(u, dt, A, B, C):
    """Bare scan ``y_t = <x_t, C_t>`` (no bias, softplus, skip or gate); the CUDA
    counterpart of the reference's ``scan_mps`` (scan.py:283-292)."""
    return selective_scan(u, dt, A, B, C)
