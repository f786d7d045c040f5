"""VMamba four-path 2D selective scan (``ss2d``) on the B200.

Drop-in for ``metal_kernelops.cv.path_scan`` (src/metal_kernelops/cv/path_scan.py
of the reference): same ``ss2d_scan(u, dt, A, B, C, merge="sum")`` and
``path_orders(height, width, device=None)``, same layouts, path orders, merge
modes and ``ValueError`` contract (:112-151, :546-576).

A ``(height, width)`` map is scanned along four paths with the Mamba-1
recurrence ``x_t = exp(dt_t A) x_{t-1} + dt_t B_t u_t``, ``y_t = <x_t, C_t>``:

======  ==========================
path    step of pixel ``(h, w)``
======  ==========================
0       ``h * W + w``   (row-major)
1       ``w * H + h``   (column-major)
2       ``L - 1 - (h * W + w)``
3       ``L - 1 - (w * H + h)``
======  ==========================

and the outputs are added per pixel as ``(p0 + p2) + (p1 + p3)`` (times 0.25
for ``merge="mean"``).  ``dt``, ``A``, ``B`` and ``C`` are shared by the four
paths, so their gradients add the four path contributions.

Layouts: u, dt ``(batch, channels, height, width)``; A ``(channels, states)``;
B, C ``(batch, groups, states, height, width)`` with ``groups`` dividing
``channels``.  float32 as in the reference, and also bfloat16/float16
activations (fp32 arithmetic).  At most ``MAX_STATES`` = 32 states, the
reference's limit.  Zero extents give the empty/zero result with zero
gradients.  CUDA tensors only; there is no CPU path.

On the device (``csrc/path_scan.cu``): one kernel writes the four path orders
of u, dt, B and C (each plane read once, all stores coalesced), the Mamba-1
selective-scan kernels run the four paths as one problem of 4 x channels rows,
and one kernel folds the four path outputs back per pixel.  The backward runs
the same way with the scan's backward kernels.
"""

from __future__ import annotations

import torch

from .. import _native as nat
from ..scan import checkpoint_numel

__all__ = ["MAX_STATES", "MERGE_MODES", "path_orders", "ss2d_scan"]

MERGE_MODES = ("sum", "mean")
"""How the four path outputs combine: elementwise sum, or their mean."""

MAX_STATES = 32
"""Widest state axis accepted (the reference's limit, path_scan.py:96)."""

_DTYPES = (torch.float32, torch.bfloat16, torch.float16)


def _check_merge(merge):
    if merge not in MERGE_MODES:
        raise ValueError(f"merge must be one of {MERGE_MODES}, got {merge!r}")


def _shape_contract(u, dt, A, B, C, where):
    """The reference's shape contract (path_scan.py:112-151), same messages."""
    if u.dim() != 4:
        raise ValueError(f"{where}: u must be (batch, channels, height, width), got {tuple(u.shape)}")
    batch, channels, height, width = u.shape
    if dt.shape != u.shape:
        raise ValueError(f"{where}: dt {tuple(dt.shape)} != u {tuple(u.shape)}")
    if A.dim() != 2:
        raise ValueError(f"{where}: A must be (channels, states), got {tuple(A.shape)}")
    if A.shape[0] != channels:
        raise ValueError(f"{where}: A has {A.shape[0]} rows for {channels} channels")
    if B.dim() != 5:
        raise ValueError(f"{where}: B must be (batch, groups, states, height, width), got {tuple(B.shape)}")
    if C.shape != B.shape:
        raise ValueError(f"{where}: C {tuple(C.shape)} != B {tuple(B.shape)}")
    if B.shape[0] != batch:
        raise ValueError(f"{where}: B batch {B.shape[0]} != u batch {batch}")
    if B.shape[2] != A.shape[1]:
        raise ValueError(f"{where}: B has {B.shape[2]} states, A has {A.shape[1]}")
    if tuple(B.shape[3:]) != (height, width):
        raise ValueError(f"{where}: B spatial {tuple(B.shape[3:])} != {(height, width)}")
    groups = B.shape[1]
    if channels and groups < 1:
        raise ValueError(f"{where}: {channels} channels need at least one group")
    if groups and channels % groups:
        raise ValueError(f"{where}: {channels} channels do not divide into {groups} groups; "
                         f"a channel would map to no group")
    return batch, channels, groups, A.shape[1], height, width


def path_orders(height, width, device=None):
    """Spatial index order of each of the four scan paths (path_scan.py:153-163).

    Entry ``p[i]`` of path ``k`` is the flat ``h * width + w`` index of the pixel
    at step ``i``; paths 2 and 3 are the reverses of paths 0 and 1.
    """
    row_major = torch.arange(height * width, device=device).reshape(height, width)
    flat = row_major.reshape(-1)
    column_major = row_major.transpose(0, 1).reshape(-1)
    return [flat, column_major, flat.flip(0), column_major.flip(0)]


def _zero_result(shape, tensors):
    """A zero result that still carries the gradient graph of ``tensors``."""
    zero = tensors[0].sum() * 0
    for tensor in tensors[1:]:
        zero = zero + tensor.sum() * 0
    return tensors[0].new_zeros(shape) + zero


def _params(u, dt, A, B, C, scale):
    batch, channels, height, width = u.shape
    p = nat.Ss2dScanParams()
    p.batch, p.channels, p.height, p.width = batch, channels, height, width
    p.groups, p.dstate = B.shape[1], A.shape[1]
    p.act_dtype = nat.dtype_code(u.dtype)
    p.bc_dtype = nat.dtype_code(B.dtype)
    p.scale = scale
    p.u, p.dt, p.A, p.B, p.C = (t.data_ptr() for t in (u, dt, A, B, C))
    return p


def _sizes(p):
    ck, fw, bw = nat._SZ(), nat._SZ(), nat._SZ()
    nat.check(nat.lib().ssm_ss2d_scan_sizes(p, ck, fw, bw), "ss2d_scan")
    return ck.value, fw.value, bw.value


@torch.library.custom_op("b200ssm::ss2d_scan_fwd", mutates_args=(), device_types="cuda")
def _fwd(u: torch.Tensor, dt: torch.Tensor, A: torch.Tensor, B: torch.Tensor, C: torch.Tensor,
         scale: float, save: bool) -> tuple[torch.Tensor, torch.Tensor]:
    p = _params(u, dt, A, B, C, scale)
    ck_bytes, fw_bytes, _ = _sizes(p)
    y = torch.empty_like(u)
    ckpt = torch.empty(ck_bytes // 4 if save else 0, dtype=torch.float32, device=u.device)
    ws = torch.empty(max(fw_bytes, 1), dtype=torch.uint8, device=u.device)
    p.y = y.data_ptr()
    p.checkpoints = ckpt.data_ptr() if save and ckpt.numel() else None
    p.workspace, p.workspace_bytes = ws.data_ptr(), ws.numel()
    p.status = nat.status_word(u.device, "ss2d_scan")
    nat.check(nat.lib().ssm_ss2d_scan_fwd(p, nat.stream_of(u)), "ss2d_scan")
    return y, ckpt


@_fwd.register_fake
def _(u, dt, A, B, C, scale, save):
    batch, channels, height, width = u.shape
    # the four paths run as one Mamba-1 problem of 4 x channels rows
    n = (checkpoint_numel(batch, 4 * channels, height * width, A.shape[1], u.element_size(), False)
         if save else 0)
    return torch.empty_like(u), u.new_empty(n, dtype=torch.float32)


@torch.library.custom_op("b200ssm::ss2d_scan_bwd", mutates_args=(), device_types="cuda")
def _bwd(dout: torch.Tensor, u: torch.Tensor, dt: torch.Tensor, A: torch.Tensor, B: torch.Tensor,
         C: torch.Tensor, ckpt: torch.Tensor, scale: float
         ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]:
    p = _params(u, dt, A, B, C, scale)
    _, _, bw_bytes = _sizes(p)
    dev = u.device
    du = torch.empty_like(u)
    ddt = torch.empty_like(u)
    dA = torch.empty(A.shape, dtype=torch.float32, device=dev)
    dB = torch.empty(B.shape, dtype=torch.float32, device=dev)
    dC = torch.empty(C.shape, dtype=torch.float32, device=dev)
    ws = torch.empty(max(bw_bytes, 1), dtype=torch.uint8, device=dev)
    p.checkpoints = ckpt.data_ptr() if ckpt.numel() else None
    p.dout = dout.data_ptr()
    p.du, p.ddt = du.data_ptr(), ddt.data_ptr()
    p.dA, p.dB, p.dC = dA.data_ptr(), dB.data_ptr(), dC.data_ptr()
    p.workspace, p.workspace_bytes = ws.data_ptr(), ws.numel()
    p.status = nat.status_word(u.device, "ss2d_scan")
    nat.check(nat.lib().ssm_ss2d_scan_bwd(p, nat.stream_of(u)), "ss2d_scan backward")
    return du, ddt, dA, dB, dC


@_bwd.register_fake
def _(dout, u, dt, A, B, C, ckpt, scale):
    f32 = dict(dtype=torch.float32)
    return (torch.empty_like(u), torch.empty_like(u), A.new_empty(A.shape, **f32),
            B.new_empty(B.shape, **f32), C.new_empty(C.shape, **f32))


def _setup(ctx, inputs, output):
    u, dt, A, B, C, scale, save = inputs
    _, ckpt = output
    ctx.save_for_backward(u, dt, A, B, C, ckpt)
    ctx.scale = scale
    ctx.set_materialize_grads(False)     # no zero-filled gradient for the saved states


def _backward(ctx, dy, dckpt):
    u, dt, A, B, C, ckpt = ctx.saved_tensors
    if ckpt.numel() == 0:
        raise RuntimeError("ss2d_scan: the forward did not save its states (save=False)")
    if dy is None:
        return (None,) * 7
    du, ddt, dA, dB, dC = _bwd(dy.contiguous(), u, dt, A, B, C, ckpt, ctx.scale)
    return du, ddt, dA, dB.to(B.dtype), dC.to(C.dtype), None, None


_fwd.register_autograd(_backward, setup_context=_setup)


def ss2d_scan(u, dt, A, B, C, merge="sum"):
    """Four-path 2D selective scan (reference ``ss2d_scan``, path_scan.py:546-576).

    Args:
        u, dt: (batch, channels, height, width)
        A: (channels, states), negative
        B, C: (batch, groups, states, height, width)
        merge: ``"sum"`` adds the four path outputs, ``"mean"`` divides by four.

    Returns:
        (batch, channels, height, width) contiguous output in ``u.dtype``.
    """
    _check_merge(merge)
    batch, channels, groups, states, height, width = _shape_contract(u, dt, A, B, C, "ss2d_scan")
    for name, tensor in (("u", u), ("dt", dt), ("A", A), ("B", B), ("C", C)):
        if tensor.device.type != "cuda":
            raise ValueError(f"ss2d_scan runs CUDA kernels, {name} is on {tensor.device}")
        if tensor.device != u.device:
            raise ValueError(f"ss2d_scan: {name} is on {tensor.device}, u is on {u.device}")
        if tensor.dtype not in _DTYPES:
            raise ValueError(f"ss2d_scan computes float32/bfloat16/float16, {name} is {tensor.dtype}")
    if states > MAX_STATES:
        raise ValueError(f"ss2d_scan: states must be at most {MAX_STATES}, got {states}")
    if u.numel() == 0 or B.numel() == 0:
        return _zero_result((batch, channels, height, width), (u, dt, A, B, C))
    act = u.dtype
    u = u.contiguous()
    dt = dt.to(act).contiguous()
    B = B.contiguous()
    C = C.to(B.dtype).contiguous()
    A = A.float().contiguous()
    save = torch.is_grad_enabled() and any(t.requires_grad for t in (u, dt, A, B, C))
    y, _ = torch.ops.b200ssm.ss2d_scan_fwd(u, dt, A, B, C, 0.25 if merge == "mean" else 1.0, bool(save))
    return y
