"""ctypes binding of the in-tree C-ABI library ``libssm_b200.so``.

The structs mirror ``include/ssm_b200.h`` field for field.  There is no
fallback: if the library is missing or a CUDA tensor reaches an op without it,
the op raises.  The library itself loads without a GPU (it links only the CUDA
runtime), so the CPU test suite can check its exported symbols.
"""

from __future__ import annotations

import ctypes
import pathlib
import threading

import torch

LIB_PATH = pathlib.Path(__file__).resolve().parent / "libssm_b200.so"

SSM_OK, SSM_ERR_INVALID, SSM_ERR_UNSUPPORTED, SSM_ERR_CUDA, SSM_ERR_WORKSPACE = range(5)
SSM_F32, SSM_BF16, SSM_F16 = 0, 1, 2

HAS_D = 0x01
HAS_Z = 0x02
HAS_BIAS = 0x04
SOFTPLUS = 0x08
D_PER_HEAD = 0x10
DT_PER_ROW = 0x20
HAS_INIT = 0x40
HAS_DY = 0x80
HAS_DSTATE = 0x100
CUDA_CORES = 0x200
CONV_SILU = 0x400
IO_DTYPE = 0x800
CHANNEL_LAST = 0x1000
SCAN_PLAIN = 0x2000
SCAN_LEAN = 0x4000

EXPORTS = (
    "ssm_status_string", "ssm_last_error",
    "ssm_selective_scan_sizes", "ssm_selective_scan_fwd", "ssm_selective_scan_bwd",
    "ssm_selective_scan_fwd_workspace",
    "ssm_state_update_sizes", "ssm_state_update_fwd", "ssm_state_update_bwd",
    "ssm_state_update_bwd_noalloc",
    "ssm_chunk_scan_sizes", "ssm_chunk_scan_fwd", "ssm_chunk_scan_bwd",
    "ssm_take_kernel_error", "ssm_selftest_bounded_wait",
    "ssm_ss2d_scan_sizes", "ssm_ss2d_scan_fwd", "ssm_ss2d_scan_bwd",
    "ssm_causal_conv1d_sizes", "ssm_causal_conv1d_fwd", "ssm_causal_conv1d_bwd",
    "ssm_causal_conv1d_update",
    "ssm_gated_rmsnorm_sizes", "ssm_gated_rmsnorm_fwd", "ssm_gated_rmsnorm_bwd",
)

_I64, _I32, _U32, _P, _SZ = ctypes.c_int64, ctypes.c_int32, ctypes.c_uint32, ctypes.c_void_p, ctypes.c_size_t


class SelectiveScanParams(ctypes.Structure):
    _fields_ = [
        ("batch", _I64), ("dim", _I64), ("length", _I64), ("groups", _I64), ("dstate", _I64),
        ("act_dtype", _I32), ("bc_dtype", _I32), ("flags", _U32),
        ("u", _P), ("delta", _P), ("A", _P), ("B", _P), ("C", _P),
        ("D", _P), ("z", _P), ("delta_bias", _P),
        ("y", _P), ("checkpoints", _P),
        ("dout", _P), ("du", _P), ("ddelta", _P), ("dz", _P),
        ("dA", _P), ("dB", _P), ("dC", _P), ("dD", _P), ("ddelta_bias", _P),
        ("workspace", _P), ("workspace_bytes", _SZ),
        ("status", _P),
    ]


class StateUpdateParams(ctypes.Structure):
    _fields_ = [
        ("batch", _I64), ("nheads", _I64), ("headdim", _I64), ("dstate", _I64), ("ngroups", _I64),
        ("dtype", _I32), ("flags", _U32),
        ("state", _P), ("x", _P), ("dt", _P), ("A", _P), ("B", _P), ("C", _P),
        ("D", _P), ("z", _P), ("dt_bias", _P),
        ("new_state", _P), ("y", _P),
        ("dy", _P), ("dnew", _P),
        ("grad_state", _P), ("dx", _P), ("ddt", _P), ("dA", _P), ("dB", _P), ("dC", _P),
        ("dD", _P), ("dz", _P), ("ddt_bias", _P),
        ("workspace", _P), ("workspace_bytes", _SZ),
        ("io_dtype", _I32),
        ("status", _P),
    ]


class ChunkScanParams(ctypes.Structure):
    _fields_ = [
        ("batch", _I64), ("length", _I64), ("nheads", _I64), ("headdim", _I64),
        ("ngroups", _I64), ("dstate", _I64), ("chunk_size", _I64),
        ("dtype", _I32), ("dt_dtype", _I32), ("flags", _U32),
        ("x", _P), ("dt", _P), ("A", _P), ("B", _P), ("C", _P), ("D", _P), ("z", _P),
        ("dt_bias", _P), ("initial_states", _P),
        ("y", _P), ("final_state", _P),
        ("dy", _P), ("dfinal", _P),
        ("dx", _P), ("ddt", _P), ("dA", _P), ("dB", _P), ("dC", _P), ("dD", _P), ("dz", _P),
        ("ddt_bias", _P), ("dinitial", _P),
        ("saved", _P), ("workspace", _P), ("workspace_bytes", _SZ),
        ("x_token_stride", _I64), ("bc_token_stride", _I64),
        ("status", _P),
    ]


class Ss2dScanParams(ctypes.Structure):
    _fields_ = [
        ("batch", _I64), ("channels", _I64), ("height", _I64), ("width", _I64),
        ("groups", _I64), ("dstate", _I64),
        ("act_dtype", _I32), ("bc_dtype", _I32), ("scale", ctypes.c_float),
        ("u", _P), ("dt", _P), ("A", _P), ("B", _P), ("C", _P),
        ("y", _P), ("checkpoints", _P),
        ("dout", _P), ("du", _P), ("ddt", _P), ("dA", _P), ("dB", _P), ("dC", _P),
        ("workspace", _P), ("workspace_bytes", _SZ),
        ("status", _P),
    ]


class CausalConv1dParams(ctypes.Structure):
    _fields_ = [
        ("batch", _I64), ("channels", _I64), ("length", _I64), ("width", _I64),
        ("dtype", _I32), ("flags", _U32),
        ("x", _P), ("weight", _P), ("bias", _P), ("initial_state", _P),
        ("out", _P), ("final_state", _P),
        ("dout", _P), ("dx", _P), ("dweight", _P), ("dbias", _P), ("dinitial", _P),
        ("workspace", _P), ("workspace_bytes", _SZ),
        ("x_row_stride", _I64), ("dout_row_stride", _I64),
        ("status", _P),
    ]


class CausalConv1dUpdateParams(ctypes.Structure):
    _fields_ = [
        ("batch", _I64), ("channels", _I64), ("length", _I64), ("width", _I64), ("state_len", _I64),
        ("state_stride_batch", _I64), ("state_stride_channel", _I64),
        ("dtype", _I32), ("flags", _U32),
        ("state", _P), ("x", _P), ("weight", _P), ("bias", _P), ("out", _P),
        ("status", _P),
    ]


class GatedRmsNormParams(ctypes.Structure):
    _fields_ = [
        ("rows", _I64), ("features", _I64), ("group_size", _I64),
        ("dtype", _I32), ("gate", _I32), ("flags", _U32), ("eps", ctypes.c_float),
        ("x", _P), ("z", _P), ("weight", _P), ("bias", _P), ("out", _P), ("rstd", _P),
        ("dy", _P), ("dx", _P), ("dz", _P), ("dweight", _P), ("dbias", _P),
        ("workspace", _P), ("workspace_bytes", _SZ),
        ("x_row_stride", _I64), ("z_row_stride", _I64),
        ("status", _P),
    ]


_lib = None
_lock = threading.Lock()


def lib():
    """The loaded library; raises if it was not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"{LIB_PATH.name} is not built; run `python -m metal_kernelops_b200.build` "
                    "(there is no CPU fallback)")
            handle = ctypes.CDLL(str(LIB_PATH))
            handle.ssm_status_string.restype = ctypes.c_char_p
            handle.ssm_status_string.argtypes = [ctypes.c_int]
            handle.ssm_last_error.restype = ctypes.c_char_p
            handle.ssm_last_error.argtypes = []
            for name, struct in (("selective_scan", SelectiveScanParams),
                                 ("state_update", StateUpdateParams),
                                 ("chunk_scan", ChunkScanParams),
                                 ("ss2d_scan", Ss2dScanParams),
                                 ("causal_conv1d", CausalConv1dParams),
                                 ("gated_rmsnorm", GatedRmsNormParams)):
                for suffix in ("fwd", "bwd"):
                    fn = getattr(handle, f"ssm_{name}_{suffix}")
                    fn.restype = ctypes.c_int
                    fn.argtypes = [ctypes.POINTER(struct), ctypes.c_void_p]
            handle.ssm_selective_scan_sizes.argtypes = [
                ctypes.POINTER(SelectiveScanParams), ctypes.POINTER(_SZ), ctypes.POINTER(_SZ)]
            handle.ssm_state_update_sizes.argtypes = [
                ctypes.POINTER(StateUpdateParams), ctypes.POINTER(_SZ)]
            handle.ssm_chunk_scan_sizes.argtypes = [
                ctypes.POINTER(ChunkScanParams), ctypes.POINTER(_SZ), ctypes.POINTER(_SZ)]
            handle.ssm_causal_conv1d_sizes.argtypes = [ctypes.POINTER(CausalConv1dParams), ctypes.POINTER(_SZ)]
            handle.ssm_gated_rmsnorm_sizes.argtypes = [ctypes.POINTER(GatedRmsNormParams), ctypes.POINTER(_SZ)]
            handle.ssm_causal_conv1d_update.restype = ctypes.c_int
            handle.ssm_causal_conv1d_update.argtypes = [ctypes.POINTER(CausalConv1dUpdateParams), ctypes.c_void_p]
            handle.ssm_selective_scan_fwd_workspace.argtypes = [
                ctypes.POINTER(SelectiveScanParams), ctypes.POINTER(_SZ)]
            handle.ssm_ss2d_scan_sizes.argtypes = [
                ctypes.POINTER(Ss2dScanParams), ctypes.POINTER(_SZ), ctypes.POINTER(_SZ),
                ctypes.POINTER(_SZ)]
            handle.ssm_state_update_bwd_noalloc.restype = ctypes.c_int
            handle.ssm_state_update_bwd_noalloc.argtypes = [ctypes.POINTER(StateUpdateParams),
                                                            ctypes.c_void_p]
            for name in ("ssm_selective_scan_sizes", "ssm_state_update_sizes", "ssm_chunk_scan_sizes",
                         "ssm_ss2d_scan_sizes", "ssm_selective_scan_fwd_workspace",
                         "ssm_causal_conv1d_sizes", "ssm_gated_rmsnorm_sizes"):
                getattr(handle, name).restype = ctypes.c_int
            handle.ssm_take_kernel_error.restype = ctypes.c_int
            handle.ssm_take_kernel_error.argtypes = []
            handle.ssm_selftest_bounded_wait.restype = ctypes.c_int
            handle.ssm_selftest_bounded_wait.argtypes = [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_void_p]
            _lib = handle
    return _lib


class NativeError(RuntimeError):
    pass


def check(status: int, what: str) -> None:
    """Map a C-ABI status to the reference's error convention: contract
    violations are ``ValueError``, everything else ``RuntimeError``."""
    if status == SSM_OK:
        return
    L = lib()
    msg = L.ssm_last_error().decode() or L.ssm_status_string(status).decode()
    if status in (SSM_ERR_INVALID, SSM_ERR_UNSUPPORTED):
        raise ValueError(f"{what}: {msg}")
    raise NativeError(f"{what}: {msg} (status {status})")


_DTYPES = {torch.float32: SSM_F32, torch.bfloat16: SSM_BF16, torch.float16: SSM_F16}


def dtype_code(dtype: torch.dtype) -> int:
    return _DTYPES[dtype]


def ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def stream_of(t: torch.Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(t.device).cuda_stream)


# --------------------------------------------------------------- status words --
# One int32 device word per op family and device, zero-initialised once from
# the caching allocator and handed to every call of that op (params.status).
# A kernel that gives up on a bounded wait writes its code there; nothing is
# cleared until ``check_errors`` reads the words.  Reading is lazy -- one small
# device-to-host copy when the caller asks -- so the ops never synchronise.
STATUS_SLOTS = ("selective_scan", "state_update", "chunk_scan", "ss2d_scan", "causal_conv1d",
                "causal_conv1d_update", "gated_rmsnorm", "selftest")
_status = {}


def _status_buffer(device: torch.device) -> torch.Tensor:
    key = device.index if device.index is not None else torch.cuda.current_device()
    buf = _status.get(key)
    if buf is None:
        buf = torch.zeros(len(STATUS_SLOTS), dtype=torch.int32, device=torch.device("cuda", key))
        _status[key] = buf
    return buf


def status_word(device: torch.device, op: str) -> int:
    """Device address of ``op``'s status word on ``device`` (for params.status)."""
    buf = _status_buffer(device)
    return buf.data_ptr() + 4 * STATUS_SLOTS.index(op)


def check_errors(device=None) -> None:
    """Read the status words of ``device`` (every device used so far when
    None), clear them, and raise ``RuntimeError`` if a kernel gave up on a
    bounded wait since the last check.  Synchronises with those devices."""
    keys = list(_status) if device is None else [torch.device(device).index or 0]
    failed = []
    for key in keys:
        buf = _status.get(key)
        if buf is None:
            continue
        vals = buf.cpu().tolist()
        if any(vals):
            buf.zero_()
            failed += [f"{op} (code {v}) on cuda:{key}" for op, v in zip(STATUS_SLOTS, vals) if v]
    if failed:
        raise NativeError("a kernel gave up on a bounded wait; its outputs are invalid: " + ", ".join(failed))


def selftest_bounded_wait(device=None, polls: int = 16) -> None:
    """Launch the library's failure-path self-test on ``device``: a wait on an
    mbarrier that nothing completes, limited to ``polls`` polls, which gives
    up and writes its code into the self-test status word."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    with torch.cuda.device(dev):
        stream = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
        check(lib().ssm_selftest_bounded_wait(ctypes.c_void_p(status_word(dev, "selftest")),
                                              ctypes.c_uint32(polls), stream), "selftest_bounded_wait")
