"""Host-side checks that need no GPU: the C-ABI library loads and exports every
symbol ``include/ssm_b200.h`` declares, the ctypes structs match the header's
layout, and the Python layer enforces the reference's argument contract
(``ValueError`` for bad shapes and for tensors off the GPU -- there is no CPU
fallback)."""

import ctypes
import pathlib
import re

import pytest
import torch

ROOT = pathlib.Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "ssm_b200.h"


def _declared():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:int|const char\*)\s+(ssm_\w+)\s*\(", text, re.M)))


def test_library_exports_every_declared_symbol():
    from metal_kernelops_b200 import _native as nat
    lib = nat.lib()
    names = _declared()
    assert len(names) >= 11
    for name in names:
        assert hasattr(lib, name), name
    assert set(names) <= set(nat.EXPORTS) | {"ssm_status_string", "ssm_last_error"}
    assert lib.ssm_status_string(0) == b"ok"


def _STRUCTS(nat):
    return (("ssm_selective_scan_params", nat.SelectiveScanParams),
            ("ssm_state_update_params", nat.StateUpdateParams),
            ("ssm_chunk_scan_params", nat.ChunkScanParams),
            ("ssm_ss2d_scan_params", nat.Ss2dScanParams),
            ("ssm_causal_conv1d_params", nat.CausalConv1dParams),
            ("ssm_causal_conv1d_update_params", nat.CausalConv1dUpdateParams),
            ("ssm_gated_rmsnorm_params", nat.GatedRmsNormParams))


def test_struct_layouts_match_header():
    """Field order and count of the ctypes mirrors equal the C structs."""
    from metal_kernelops_b200 import _native as nat
    text = HEADER.read_text()
    for cname, struct in _STRUCTS(nat):
        body = re.search(r"typedef struct %s \{(.*?)\} %s;" % (cname, cname), text, re.S).group(1)
        body = re.sub(r"/\*.*?\*/", "", body, flags=re.S)
        fields = []
        for decl in body.split(";"):
            decl = decl.strip()
            if not decl:
                continue
            names = decl.split(None, 1)[1] if not decl.startswith("const") else decl.split(None, 2)[2]
            for n in names.split(","):
                fields.append(n.strip().lstrip("*").strip())
        assert [f for f, _ in struct._fields_] == fields, cname


def test_struct_offsets_match_c_compiler(tmp_path):
    """Every field offset and struct size of the ctypes mirrors equals what a C
    compiler makes of the header (gcc on a generated probe program)."""
    import shutil
    import subprocess
    from metal_kernelops_b200 import _native as nat
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("no C compiler")
    lines = ['#include <stdio.h>', '#include "ssm_b200.h"', "int main(void) {"]
    want = []
    for cname, struct in _STRUCTS(nat):
        lines.append(f'printf("%zu\\n", sizeof({cname}));')
        want.append(ctypes.sizeof(struct))
        for name, _ in struct._fields_:
            lines.append(f'printf("%zu\\n", offsetof({cname}, {name}));')
            want.append(getattr(struct, name).offset)
    lines += ["return 0;", "}"]
    src = tmp_path / "probe.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "probe"
    subprocess.run([gcc, "-I", str(HEADER.parent), str(src), "-o", str(exe)], check=True)
    got = [int(v) for v in subprocess.run([str(exe)], check=True, capture_output=True,
                                          text=True).stdout.split()]
    assert got == want


def test_invalid_arguments_rejected_by_abi():
    """The C ABI returns a status (no exception, no crash) for bad sizes."""
    from metal_kernelops_b200 import _native as nat
    lib = nat.lib()
    p = nat.SelectiveScanParams()
    p.batch, p.dim, p.length, p.groups, p.dstate = 1, 6, 4, 4, 16   # groups does not divide dim
    assert lib.ssm_selective_scan_fwd(p, None) == nat.SSM_ERR_INVALID
    assert b"divisible" in lib.ssm_last_error()
    p.groups, p.dstate = 1, 300
    assert lib.ssm_selective_scan_fwd(p, None) == nat.SSM_ERR_UNSUPPORTED
    q = nat.StateUpdateParams()
    q.batch, q.nheads, q.headdim, q.dstate, q.ngroups = 1, 6, 4, 8, 4
    assert lib.ssm_state_update_fwd(q, None) == nat.SSM_ERR_INVALID


@pytest.mark.parametrize("gated", [False, True])
@pytest.mark.parametrize("shape", [(2, 8, 64, 16, 2), (3, 24, 37, 4, 4), (1, 5, 1, 16, 2),
                                   (2, 16, 0, 16, 2), (4, 96, 3136, 16, 4)])
def test_checkpoint_numel_matches_library_size(shape, gated):
    """The fake-tensor size of the saved-for-backward buffer equals the size
    the library asks for (a host-only query), for the scan and for ss2d."""
    from metal_kernelops_b200 import _native as nat
    from metal_kernelops_b200.scan import checkpoint_numel
    batch, dim, length, dstate, esz = shape
    lib = nat.lib()
    p = nat.SelectiveScanParams()
    p.batch, p.dim, p.length, p.groups, p.dstate = batch, dim, length, 1, dstate
    p.act_dtype = p.bc_dtype = {4: nat.dtype_code(torch.float32), 2: nat.dtype_code(torch.bfloat16)}[esz]
    p.flags = nat.HAS_Z if gated else 0
    ck, ws = nat._SZ(), nat._SZ()
    assert lib.ssm_selective_scan_sizes(p, ck, ws) == nat.SSM_OK
    assert checkpoint_numel(batch, dim, length, dstate, esz, gated) * 4 == ck.value
    # the lean mode: states every 16 steps, no saved scan output
    p.flags |= nat.SCAN_LEAN
    assert lib.ssm_selective_scan_sizes(p, ck, ws) == nat.SSM_OK
    assert checkpoint_numel(batch, dim, length, dstate, esz, gated, lean=True) * 4 == ck.value
    if length:
        full = checkpoint_numel(batch, dim, length, dstate, esz, gated)
        assert ck.value < full * 4
    p.flags &= ~nat.SCAN_LEAN
    if length and length % 8 == 0 and not gated:   # ss2d: a (height, 8) map, four paths per channel
        q = nat.Ss2dScanParams()
        q.batch, q.channels, q.height, q.width, q.groups, q.dstate = batch, dim, length // 8, 8, 1, dstate
        q.act_dtype = q.bc_dtype = p.act_dtype
        q.scale = 1.0
        ck2, fw, bw = nat._SZ(), nat._SZ(), nat._SZ()
        assert lib.ssm_ss2d_scan_sizes(q, ck2, fw, bw) == nat.SSM_OK
        assert checkpoint_numel(batch, 4 * dim, length, dstate, esz, False) * 4 == ck2.value


@pytest.mark.parametrize("batch,dim,length,segmented", [
    (16, 5120, 4096, False),   # config 2: 1280 CTAs fill the GPU, one pass per channel tile
    (2, 5120, 4096, True),     # per-GPU work at 8 GPUs: the sequence is cut into segments
    (1, 8, 2000, True),        # one channel tile over a long sequence
    (1, 8, 100, False),        # too short to cut (fewer than 8 chunks)
])
def test_sequence_segment_planning(batch, dim, length, segmented):
    """The host plans sequence segments (and asks for forward scratch for
    them) only when the channel tiles leave most of the GPU idle.  Host-only:
    without a device the library plans for 148 SMs."""
    from metal_kernelops_b200 import _native as nat
    lib = nat.lib()
    p = nat.SelectiveScanParams()
    p.batch, p.dim, p.length, p.groups, p.dstate = batch, dim, length, 1, 16
    p.act_dtype = p.bc_dtype = nat.dtype_code(torch.bfloat16)
    fw = nat._SZ()
    assert lib.ssm_selective_scan_fwd_workspace(p, fw) == nat.SSM_OK
    assert (fw.value > 0) == segmented


def test_selective_scan_contract_on_cpu():
    import metal_kernelops_b200 as mk
    u = torch.zeros(1, 4, 8)
    A = torch.zeros(4, 3)
    B = torch.zeros(1, 1, 3, 8)
    with pytest.raises(ValueError, match="runs CUDA kernels"):
        mk.selective_scan(u, u, A, B, B)
    with pytest.raises(ValueError):
        mk.selective_scan(u, u[..., :7], A, B, B)
    with pytest.raises(ValueError):
        mk.selective_scan(u, u, A, B.repeat(1, 3, 1, 1), B.repeat(1, 3, 1, 1))
    with pytest.raises(ValueError):
        mk.selective_scan(u, u, A, B, B, D=torch.zeros(5))


def test_state_update_contract_on_cpu():
    from metal_kernelops_b200.cv import mamba2_state_update
    state = torch.zeros(2, 4, 6, 16)
    x = torch.zeros(2, 4, 6)
    dt = torch.zeros(2, 4)
    A = torch.zeros(4)
    B = torch.zeros(2, 2, 16)
    with pytest.raises(ValueError, match="runs CUDA kernels"):
        mamba2_state_update(state, x, dt, A, B, B)
    with pytest.raises(ValueError):
        mamba2_state_update(state, x, dt, A, torch.zeros(2, 3, 16), torch.zeros(2, 3, 16))
    with pytest.raises(ValueError):
        mamba2_state_update(state, x, dt, A, B, B, out_state=torch.zeros(2, 4, 6))


def test_chunk_scan_contract_on_cpu():
    from metal_kernelops_b200.cv import mamba2_chunk_scan
    x = torch.zeros(2, 13, 4, 6)
    dt = torch.zeros(2, 13, 4)
    A = torch.zeros(4)
    B = torch.zeros(2, 13, 2, 5)
    with pytest.raises(ValueError, match="runs CUDA kernels"):
        mamba2_chunk_scan(x, dt, A, B, B, 5)
    with pytest.raises(ValueError):
        mamba2_chunk_scan(x, dt, A, B, B, 5, initial_states=torch.zeros(2, 4, 5, 5))
    with pytest.raises(ValueError):
        mamba2_chunk_scan(x, dt, A, B, B, 0)
    with pytest.raises(ValueError):
        mamba2_chunk_scan(x, dt, A, torch.zeros(2, 13, 3, 5), torch.zeros(2, 13, 3, 5))


@pytest.mark.parametrize("headdim,dstate", [(64, 128), (64, 64), (32, 128), (128, 128), (256, 64), (16, 16),
                                            (40, 72), (96, 128), (64, 136), (64, 256), (12, 64)])
def test_chunk_scan_tensor_core_shapes_match_library(headdim, dstate):
    """`tc_shape` (which the Python wrapper uses to keep token-strided views)
    says exactly which head shapes the library runs on the tensor cores: for
    those, the saved-state buffer the library asks for is the tensor-core
    layout (one 16 KB state image per (batch, 64-column virtual head, 128-step
    chunk)); for the others it is the CUDA-core layout, the same as with
    SSM_CUDA_CORES forced.  Host-only query."""
    from metal_kernelops_b200 import _native as nat
    from metal_kernelops_b200.cv import tc_shape
    lib = nat.lib()

    def saved(flags):
        p = nat.ChunkScanParams()
        p.batch, p.length, p.nheads, p.headdim, p.ngroups, p.dstate = 2, 300, 4, headdim, 2, dstate
        p.chunk_size = 64
        p.dtype, p.dt_dtype = nat.dtype_code(torch.bfloat16), nat.dtype_code(torch.float32)
        p.flags = flags
        s, w = nat._SZ(), nat._SZ()
        assert lib.ssm_chunk_scan_sizes(p, s, w) == nat.SSM_OK
        return s.value

    virtual = headdim // 64 if headdim > 64 else 1
    tc_bytes = (2 * 4 * virtual * 3 * 16384 + 255) // 256 * 256
    if tc_shape(headdim, dstate):
        assert saved(0) == tc_bytes
        assert saved(nat.CUDA_CORES) != tc_bytes
    else:
        assert saved(0) == saved(nat.CUDA_CORES)
