"""Mamba-2 chunked SSD scan on the B200: drop-in for
``metal_kernelops.cv.mamba2_chunk`` (src/metal_kernelops/cv/mamba2_chunk.py).

Computes ``mamba_chunk_scan_combined`` (reference :1-13)::

    dt_t  = softplus(dt_t + dt_bias)                      (dt_softplus)
    a_t   = exp(dt_t * A)                                 A negative, per head
    s_t   = a_t * s_{t-1} + dt_t * x_t (x) B_t            s (batch, head, d_head, d_state)
    y_t   = <C_t, s_t> + D * x_t
    y_t   = y_t * silu(z_t)
    final = s_{L-1}

Layout contract (reference :38-58): x, z (batch, length, nheads, d_head); dt
(batch, length, nheads); A (nheads,); B, C (batch, length, ngroups, d_state);
D (nheads,) or (nheads, d_head); dt_bias (nheads,); initial_states
(batch, nheads, d_head, d_state), also accepted transposed when
d_state != d_head and with a leading singleton chunk axis.  Returns
``(y, final_state)`` in ``x.dtype``.  The result does not depend on
``chunk_size``.  Errors are ``ValueError`` (reference ``_check`` :398-444);
tensors must be on a CUDA device (no CPU path).

Registered as ``b200ssm::chunk_scan_fwd`` / ``_bwd`` custom ops on the CUDA key,
with an autograd formula covering every differentiable input (the reference
gets its backward from autograd through its matmul composition).
"""

from __future__ import annotations

from typing import Optional

import torch

from .. import _native as nat

__all__ = ["mamba2_chunk_scan", "last_path", "set_tensor_cores", "tc_shape"]

_DTYPES = (torch.float32, torch.float16, torch.bfloat16)
_path = "none"
_tensor_cores = True


def tc_shape(d_head: int, d_state: int) -> bool:
    """Whether the tensor-core kernels serve this head shape (with bf16/f16
    inputs): d_head a multiple of 8 up to 64, or 128 or 256, and d_state a
    multiple of 8 up to 128.  Other shapes and fp32 inputs run the CUDA-core
    kernels."""
    pd = (8 <= d_head <= 64 and d_head % 8 == 0) or d_head in (128, 256)
    return pd and 8 <= d_state <= 128 and d_state % 8 == 0


def set_tensor_cores(enabled: bool) -> bool:
    """Allow (default) or forbid the tensor-core kernels, which serve bf16/f16
    inputs whose head shape :func:`tc_shape` accepts; forbidden, those inputs
    run the CUDA-core kernels like every other case.  Returns the previous
    setting.  The setting must not change between a forward and its
    backward."""
    global _tensor_cores
    prev, _tensor_cores = _tensor_cores, bool(enabled)
    return prev


def last_path():
    """Which implementation the last :func:`mamba2_chunk_scan` call ran
    (reference :389-395 reports "metal" or "composition"; here it is always
    "cuda")."""
    return _path


def _params(x, dt, A, B, C, D, z, dt_bias, init, chunk_size, softplus):
    p = nat.ChunkScanParams()
    p.batch, p.length, p.nheads, p.headdim = x.shape
    p.ngroups, p.dstate = B.shape[2], B.shape[3]
    p.chunk_size = chunk_size
    p.dtype = nat.dtype_code(x.dtype)
    p.dt_dtype = nat.dtype_code(dt.dtype)
    p.flags = ((nat.HAS_D if D is not None else 0)
               | (nat.D_PER_HEAD if D is not None and D.dim() == 2 else 0)
               | (nat.HAS_Z if z is not None else 0) | (nat.HAS_BIAS if dt_bias is not None else 0)
               | (nat.SOFTPLUS if softplus else 0) | (nat.HAS_INIT if init is not None else 0))
    # the tensor-core kernels move 16-byte rows: odd views take the CUDA-core path
    if not _tensor_cores or (x.device.type != "meta" and any(
            t is not None and t.data_ptr() % 16 for t in (x, B, C, z))):
        p.flags |= nat.CUDA_CORES
    # token strides (0 for one token: never used)
    p.x_token_stride = x.stride(1) if x.shape[1] > 1 else 0
    p.bc_token_stride = B.stride(1) if B.shape[1] > 1 else 0
    if x.device.type == "meta":
        return p
    p.x, p.dt, p.A, p.B, p.C = (t.data_ptr() for t in (x, dt, A, B, C))
    p.D = D.data_ptr() if D is not None else None
    p.z = z.data_ptr() if z is not None else None
    p.dt_bias = dt_bias.data_ptr() if dt_bias is not None else None
    p.initial_states = init.data_ptr() if init is not None else None
    return p


def _sizes(p):
    sv, ws = nat._SZ(), nat._SZ()
    nat.check(nat.lib().ssm_chunk_scan_sizes(p, sv, ws), "mamba2_chunk_scan")
    return sv.value, ws.value


@torch.library.custom_op("b200ssm::chunk_scan_fwd", mutates_args=(), device_types="cuda")
def _fwd(x: torch.Tensor, dt: torch.Tensor, A: torch.Tensor, B: torch.Tensor, C: torch.Tensor,
         D: Optional[torch.Tensor], z: Optional[torch.Tensor], dt_bias: Optional[torch.Tensor],
         init: Optional[torch.Tensor], chunk_size: int, softplus: bool,
         save: bool) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    p = _params(x, dt, A, B, C, D, z, dt_bias, init, chunk_size, softplus)
    saved_bytes, ws_bytes = _sizes(p)
    batch, length, nheads, headdim = x.shape
    y = x.new_empty(x.shape)
    final = torch.empty(batch, nheads, headdim, B.shape[3], dtype=torch.float32, device=x.device)
    saved = torch.empty(saved_bytes // 4, dtype=torch.float32, device=x.device)
    p.y, p.final_state, p.saved = y.data_ptr(), final.data_ptr(), saved.data_ptr()
    p.status = nat.status_word(x.device, "chunk_scan")
    nat.check(nat.lib().ssm_chunk_scan_fwd(p, nat.stream_of(x)), "mamba2_chunk_scan")
    return y, final, saved


@_fwd.register_fake
def _(x, dt, A, B, C, D, z, dt_bias, init, chunk_size, softplus, save):
    batch, length, nheads, headdim = x.shape
    saved_bytes, _ = _sizes(_params(x, dt, A, B, C, D, z, dt_bias, init, chunk_size, softplus))
    return (x.new_empty(x.shape), x.new_empty(batch, nheads, headdim, B.shape[3], dtype=torch.float32),
            x.new_empty(saved_bytes // 4, dtype=torch.float32))


@torch.library.custom_op("b200ssm::chunk_scan_bwd", mutates_args=(), device_types="cuda")
def _bwd(dy: torch.Tensor, dfinal: Optional[torch.Tensor], x: torch.Tensor, dt: torch.Tensor,
         A: torch.Tensor, B: torch.Tensor, C: torch.Tensor, D: Optional[torch.Tensor],
         z: Optional[torch.Tensor], dt_bias: Optional[torch.Tensor], init: Optional[torch.Tensor],
         saved: torch.Tensor, chunk_size: int, softplus: bool) -> list[torch.Tensor]:
    p = _params(x, dt, A, B, C, D, z, dt_bias, init, chunk_size, softplus)
    _, ws_bytes = _sizes(p)
    dev = x.device
    f32 = dict(dtype=torch.float32, device=dev)
    dx = x.new_empty(x.shape)
    ddt = torch.empty(dt.shape, **f32)
    dA = torch.empty(A.shape, **f32)
    dB = torch.empty(B.shape, **f32)
    dC = torch.empty(C.shape, **f32)
    # absent gradients: distinct empty tensors (custom-op returns may not alias)
    dD = torch.empty(D.shape if D is not None else (0,), **f32)
    dz = x.new_empty(x.shape) if z is not None else x.new_empty(0)
    dbias = torch.empty(A.shape if dt_bias is not None else (0,), **f32)
    dinit = torch.empty(init.shape if init is not None else (0,), **f32)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=dev)
    p.flags |= nat.HAS_DY
    p.dy = dy.data_ptr()
    if dfinal is not None:
        p.flags |= nat.HAS_DSTATE
        p.dfinal = dfinal.data_ptr()
    p.saved = saved.data_ptr()
    p.dx, p.ddt, p.dA, p.dB, p.dC = (t.data_ptr() for t in (dx, ddt, dA, dB, dC))
    p.dD = dD.data_ptr() if D is not None else None
    p.dz = dz.data_ptr() if z is not None else None
    p.ddt_bias = dbias.data_ptr() if dt_bias is not None else None
    p.dinitial = dinit.data_ptr() if init is not None else None
    p.workspace, p.workspace_bytes = ws.data_ptr(), ws.numel()
    p.status = nat.status_word(x.device, "chunk_scan")
    nat.check(nat.lib().ssm_chunk_scan_bwd(p, nat.stream_of(x)), "mamba2_chunk_scan backward")
    return [dx, ddt, dA, dB, dC, dD, dz, dbias, dinit]


@_bwd.register_fake
def _(dy, dfinal, x, dt, A, B, C, D, z, dt_bias, init, saved, chunk_size, softplus):
    f = lambda t: t.new_empty(t.shape, dtype=torch.float32)  # noqa: E731
    e = lambda: x.new_empty(0, dtype=torch.float32)  # noqa: E731
    return [x.new_empty(x.shape), f(dt), f(A), f(B), f(C), f(D) if D is not None else e(),
            x.new_empty(x.shape) if z is not None else x.new_empty(0),
            f(A) if dt_bias is not None else e(), f(init) if init is not None else e()]


def _setup(ctx, inputs, output):
    x, dt, A, B, C, D, z, dt_bias, init, chunk_size, softplus, save = inputs
    _, _, saved = output
    ctx.save_for_backward(x, dt, A, B, C, D, z, dt_bias, init, saved)
    ctx.chunk_size, ctx.softplus = chunk_size, softplus
    # unused outputs (the saved chunk states, an unused final state) arrive as
    # None instead of zero-filled buffers of their size
    ctx.set_materialize_grads(False)


def _backward(ctx, dy, dfinal, dsaved):
    x, dt, A, B, C, D, z, dt_bias, init, saved = ctx.saved_tensors
    if dy is None:
        dy = torch.zeros_like(x)
    dy = dy.contiguous()
    if dy.data_ptr() % 16:
        dy = dy.clone()
    grads = _bwd(dy, None if dfinal is None else dfinal.float().contiguous(),
                 x, dt, A, B, C, D, z, dt_bias, init, saved, ctx.chunk_size, ctx.softplus)
    dx, ddt, dA, dB, dC, dD, dz, dbias, dinit = grads
    return (dx, ddt.to(dt.dtype), dA, dB.to(B.dtype), dC.to(C.dtype),
            dD if D is not None else None, dz if z is not None else None,
            dbias if dt_bias is not None else None, dinit if init is not None else None,
            None, None, None)


_fwd.register_autograd(_backward, setup_context=_setup)


def _check(x, dt, A, B, C, D, z, dt_bias, initial_states, chunk_size):
    """Shape/dtype contract with the reference's messages (:398-444)."""
    if chunk_size < 1:
        raise ValueError(f"chunk_size must be positive, got {chunk_size}")
    if x.dim() != 4:
        raise ValueError(f"x must be (batch, length, nheads, d_head), got {tuple(x.shape)}")
    batch, length, nheads, headdim = x.shape
    if tuple(dt.shape) != (batch, length, nheads):
        raise ValueError(f"dt must be {(batch, length, nheads)}, got {tuple(dt.shape)}")
    if tuple(A.shape) != (nheads,):
        raise ValueError(f"A must be ({nheads},), got {tuple(A.shape)}")
    if B.dim() != 4 or tuple(C.shape) != tuple(B.shape):
        raise ValueError("B and C must both be (batch, length, ngroups, d_state), got "
                         f"{tuple(B.shape)} and {tuple(C.shape)}")
    if tuple(B.shape[:2]) != (batch, length):
        raise ValueError(f"B/C must start with {(batch, length)}, got {tuple(B.shape)}")
    ngroups, dstate = B.shape[2], B.shape[3]
    if ngroups < 1 or nheads % ngroups:
        raise ValueError(f"nheads={nheads} must be a multiple of ngroups={ngroups}")
    if z is not None and tuple(z.shape) != tuple(x.shape):
        raise ValueError(f"z must be {tuple(x.shape)}, got {tuple(z.shape)}")
    if D is not None and tuple(D.shape) not in ((nheads,), (nheads, headdim)):
        raise ValueError(f"D must be ({nheads},) or ({nheads}, {headdim}), got {tuple(D.shape)}")
    if dt_bias is not None and tuple(dt_bias.shape) != (nheads,):
        raise ValueError(f"dt_bias must be ({nheads},), got {tuple(dt_bias.shape)}")
    if initial_states is not None:
        if initial_states.dim() == 5 and initial_states.shape[1] == 1:
            initial_states = initial_states[:, 0]
        if tuple(initial_states.shape) != (batch, nheads, headdim, dstate):
            if (tuple(initial_states.shape) == (batch, nheads, dstate, headdim)
                    and headdim != dstate):
                initial_states = initial_states.transpose(-1, -2)
            else:
                raise ValueError(
                    "initial_states must be (batch, nheads, d_head, d_state) = "
                    f"{(batch, nheads, headdim, dstate)}, got {tuple(initial_states.shape)}")
    if x.dtype not in _DTYPES:
        raise ValueError(f"x must be float32, float16 or bfloat16, got {x.dtype}")
    for name, t in (("x", x), ("dt", dt), ("A", A), ("B", B), ("C", C), ("D", D), ("z", z),
                    ("dt_bias", dt_bias), ("initial_states", initial_states)):
        if t is not None and t.device.type != "cuda":
            raise ValueError(f"mamba2_chunk_scan runs CUDA kernels, {name} is on {t.device}")
        if t is not None and t.device != x.device:
            raise ValueError(f"{name} is on {t.device}, x is on {x.device}")
    return initial_states


def _token_rows(t):
    """(batch, length, heads, width) t that the tensor-core kernels can read
    through its token stride: heads and width packed, tokens evenly spaced in
    16-byte steps, batches length tokens apart, 16-byte aligned."""
    b, length, heads, width = t.shape
    if t.stride(3) != 1 or t.stride(2) != width or t.data_ptr() % 16:
        return False
    ts = t.stride(1) if length > 1 else heads * width
    if ts < heads * width or (ts * t.element_size()) % 16:
        return False
    return b <= 1 or t.stride(0) == length * ts


def mamba2_chunk_scan(x, dt, A, B, C, chunk_size=64, D=None, z=None, dt_bias=None,
                      dt_softplus=False, initial_states=None):
    """Exact Mamba-2 chunked SSD scan (reference cv/mamba2_chunk.py:617-678).

    Returns ``(y, final_state)``: ``y`` (batch, length, nheads, d_head) and
    ``final_state`` (batch, nheads, d_head, d_state), both in ``x.dtype``.
    """
    global _path
    initial_states = _check(x, dt, A, B, C, D, z, dt_bias, initial_states, chunk_size)
    dtype = x.dtype
    B = B.to(dtype)
    C = C.to(dtype)
    # the tensor-core path reads x and B / C through their token strides (column
    # slices of a wider projection or convolution output need no copy; B and C
    # share one stride); anything else is made dense
    tc = _tensor_cores and dtype in (torch.bfloat16, torch.float16) and tc_shape(x.shape[3], B.shape[3])
    if not (tc and _token_rows(x)):
        x = x.contiguous()
    if not (tc and _token_rows(B) and _token_rows(C) and B.stride() == C.stride()):
        B, C = B.contiguous(), C.contiguous()
    z = z.to(dtype).contiguous() if z is not None else None
    dt = (dt if dt.dtype in _DTYPES else dt.float()).contiguous()
    A = A.float().contiguous()
    D = D.float().contiguous() if D is not None else None
    dt_bias = dt_bias.float().contiguous() if dt_bias is not None else None
    init = initial_states.float().contiguous() if initial_states is not None else None
    save = torch.is_grad_enabled() and any(
        t is not None and t.requires_grad for t in (x, dt, A, B, C, D, z, dt_bias, init))
    _path = "cuda"
    y, final, _ = torch.ops.b200ssm.chunk_scan_fwd(x, dt, A, B, C, D, z, dt_bias, init,
                                                   int(chunk_size), bool(dt_softplus), bool(save))
    return y, final.to(dtype)
