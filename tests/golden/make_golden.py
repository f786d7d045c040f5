"""Generate the golden fixtures from the reference's own functions.

Run once in a container that holds the reference source tree:

    REFERENCE_SRC=<path to metal-kernelops>/src python tests/golden/make_golden.py [names...]

(names: selective_scan, mamba2_chunk, mamba2_state, path_scan, causal_conv1d,
gated_norm; default all)

It imports dbydd/metal-kernelops 0.3.0 and evaluates, on seeded CPU inputs,
the functions the hot path is defined by:

* ``metal_kernelops.reference.selective_scan``      (reference.py:5-49)
* ``metal_kernelops.cv.path_scan._scan_reference``  (cv/path_scan.py:579-605),
  wrapped in the epilogue of ``scan.selective_scan`` (scan.py:311-320), with
  autograd for the gradients
* ``metal_kernelops.cv.mamba2_chunk_scan_reference`` (cv/mamba2_chunk.py:681-723)
* ``metal_kernelops.cv.mamba2_chunk_scan``  (the CPU composition, :617-678)
* ``metal_kernelops.cv.mamba2_state_update_reference`` (cv/mamba2_state.py:822-849)
* ``metal_kernelops.cv.path_scan.ss2d_scan_reference`` (cv/path_scan.py:608-639)
  and ``path_orders`` (:153-163)
* ``metal_kernelops.cv.causal_conv1d.causal_conv1d_ref`` (cv/causal_conv1d.py:480-518)
  and ``_update_aten`` (:657-670)
* ``metal_kernelops.cv.gated_norm.rmsnorm_gated_reference`` (cv/gated_norm.py:689-720)

The outputs go to ``tests/golden/*.pt``.  The test suite never imports the
reference; it only reads these files.
"""

import os
import pathlib
import sys

import torch
import torch.nn.functional as F

HERE = pathlib.Path(__file__).resolve().parent
if not os.environ.get("REFERENCE_SRC"):
    sys.exit("set REFERENCE_SRC to the reference's src directory (the one holding metal_kernelops/)")
sys.path.insert(0, os.environ["REFERENCE_SRC"])

from metal_kernelops import reference as stepwise  # noqa: E402
from metal_kernelops.cv import mamba2_chunk_scan, mamba2_chunk_scan_reference  # noqa: E402
from metal_kernelops.cv import mamba2_state_update_reference  # noqa: E402
from metal_kernelops.cv.path_scan import _scan_reference  # noqa: E402
from metal_kernelops.cv.path_scan import path_orders, ss2d_scan_reference  # noqa: E402
from metal_kernelops.cv import causal_conv1d as _cc  # noqa: E402
from metal_kernelops.cv.gated_norm import rmsnorm_gated_reference  # noqa: E402

sys.path.insert(0, str(HERE.parent.parent))
from oracle.ssm_oracle import selective_scan_inputs, ss2d_inputs  # noqa: E402

torch.set_num_threads(8)


def _leaf(t):
    return None if t is None else t.detach().clone().requires_grad_(True)


def selective_scan_cases():
    """Mamba-1: config 0 plus grouped / odd-size variants, fp64."""
    cases = {}
    shapes = {
        "config0": (2, 8, 64, 16, 1),
        "grouped": (2, 8, 24, 5, 2),
        "per_channel_groups": (1, 4, 9, 3, 4),
        "thirty_two_states": (1, 4, 11, 32, 2),
    }
    for idx, (name, (b, d, l, n, g)) in enumerate(shapes.items()):
        inp = selective_scan_inputs(b, d, l, n, g, seed=1000 + idx, act_dtype=torch.float64)
        inp = {k: v.double() for k, v in inp.items()}
        # stepwise reference (forward only, as in the original)
        dt_eff = F.softplus(inp["delta"] + inp["delta_bias"][..., None])
        y_step = stepwise.selective_scan(inp["u"], dt_eff, inp["A"], inp["B"], inp["C"])
        # differentiable reference with the selective_scan epilogue
        names = ("u", "delta", "A", "B", "C", "D", "z", "delta_bias")
        leaves = {k: _leaf(inp[k]) for k in names}
        dt = leaves["delta"] + leaves["delta_bias"][..., None]
        dt = F.softplus(dt)
        out = _scan_reference(leaves["u"], dt, leaves["A"], leaves["B"], leaves["C"])
        out = out + leaves["u"] * leaves["D"][..., None]
        out = out * F.silu(leaves["z"])
        grads = torch.autograd.grad(out, [leaves[k] for k in names], inp["dout"])
        cases[name] = {
            "inputs": inp,
            "y_stepwise_scan": y_step,
            "y": out.detach(),
            "grads": dict(zip(names, grads)),
        }
    # cumsum known answer (verify_path_scan.py:125-159): A=0, dt=1, B=C=1
    g = torch.Generator().manual_seed(77)
    u = torch.randn(1, 1, 12, generator=g, dtype=torch.float64)
    y = _scan_reference(u, torch.ones_like(u), torch.zeros(1, 1, dtype=torch.float64),
                        torch.ones(1, 1, 1, 12, dtype=torch.float64),
                        torch.ones(1, 1, 1, 12, dtype=torch.float64))
    cases["cumsum_kat"] = {"u": u, "y": y}
    return cases


def _ssd_problem(batch, length, nheads, headdim, ngroups, dstate, seed):
    # same draw order as benchmarks/verify_mamba2_chunk.py:_problem/_options
    gen = torch.Generator().manual_seed(seed)
    x = torch.randn(batch, length, nheads, headdim, generator=gen)
    dt = torch.randn(batch, length, nheads, generator=gen)
    A = -torch.exp(torch.rand(nheads, generator=gen))
    B = torch.randn(batch, length, ngroups, dstate, generator=gen)
    C = torch.randn(batch, length, ngroups, dstate, generator=gen)
    gen = torch.Generator().manual_seed(seed + 10)
    opts = dict(
        D=torch.randn(nheads, generator=gen),
        z=torch.randn(batch, length, nheads, headdim, generator=gen),
        dt_bias=torch.randn(nheads, generator=gen) * 0.1,
        initial_states=torch.randn(batch, nheads, headdim, dstate, generator=gen) * 0.1,
    )
    return dict(x=x, dt=dt, A=A, B=B, C=C), opts


def ssd_cases():
    cases = {}
    shapes = {
        "ragged": (2, 13, 4, 6, 2, 5),
        "gqa1": (1, 16, 4, 4, 1, 4),
        "mha": (2, 9, 4, 3, 4, 3),
        "short": (1, 5, 2, 2, 1, 3),
    }
    names = ("x", "dt", "A", "B", "C", "D", "z", "dt_bias", "initial_states")
    for seed, (name, shape) in enumerate(shapes.items()):
        base, opts = _ssd_problem(*shape, seed=seed)
        inp = {k: v.double() for k, v in {**base, **opts}.items()}
        leaves = {k: _leaf(inp[k]) for k in names}
        y, s = mamba2_chunk_scan_reference(
            leaves["x"], leaves["dt"], leaves["A"], leaves["B"], leaves["C"],
            D=leaves["D"], z=leaves["z"], dt_bias=leaves["dt_bias"], dt_softplus=True,
            initial_states=leaves["initial_states"])
        gen = torch.Generator().manual_seed(seed + 50)
        wy = torch.randn(y.shape, generator=gen, dtype=torch.float64)
        ws = torch.randn(s.shape, generator=gen, dtype=torch.float64)
        grads = torch.autograd.grad((y * wy).sum() + (s * ws).sum(), [leaves[k] for k in names])
        # the reference's own CPU composition, fp32, chunk 4
        f32 = {k: v.float() for k, v in inp.items()}
        yc, sc = mamba2_chunk_scan(f32["x"], f32["dt"], f32["A"], f32["B"], f32["C"], 4,
                                   D=f32["D"], z=f32["z"], dt_bias=f32["dt_bias"],
                                   dt_softplus=True, initial_states=f32["initial_states"])
        cases[name] = {"inputs": inp, "y": y.detach(), "final_state": s.detach(),
                       "wy": wy, "ws": ws, "grads": dict(zip(names, grads)),
                       "y_composition_f32": yc, "final_composition_f32": sc}
    # defaults (no options), verify_mamba2_chunk.py:150-157
    base, _ = _ssd_problem(2, 9, 4, 6, 2, 5, seed=7)
    inp = {k: v.double() for k, v in base.items()}
    y, s = mamba2_chunk_scan_reference(inp["x"], inp["dt"], inp["A"], inp["B"], inp["C"])
    cases["defaults"] = {"inputs": inp, "y": y, "final_state": s}
    return cases


def decode_cases():
    cases = {}
    specs = {
        # name: batch, nheads, dim, dstate, groups, dt_per_row, d_kind, z, bias, softplus
        "decode": (1, 16, 8, 32, 1, False, "head", True, True, True),
        "batched": (4, 8, 4, 16, 2, False, "head", True, True, False),
        "dt_per_element": (2, 4, 6, 8, 2, True, "head", True, True, False),
        "head_dim_D": (2, 4, 6, 8, 2, False, "head_dim", True, True, False),
        "no_options": (2, 6, 4, 16, 6, False, "none", False, False, False),
        "dstate_1": (2, 4, 8, 1, 1, False, "head", True, True, True),
    }
    names = ("state", "x", "dt", "A", "B", "C", "D", "z", "dt_bias")
    for idx, (name, spec) in enumerate(specs.items()):
        b, h, p, n, g, per_row, d_kind, use_z, use_bias, softplus = spec
        gen = torch.Generator().manual_seed(7 + idx)
        inp = {
            "state": torch.randn(b, h, p, n, generator=gen),
            "x": torch.randn(b, h, p, generator=gen),
            "dt": (torch.rand(b, h, p, generator=gen) if per_row else
                   torch.rand(b, h, generator=gen)) * 0.2,
            "A": -torch.rand(h, generator=gen) - 0.05,
            "B": torch.randn(b, g, n, generator=gen),
            "C": torch.randn(b, g, n, generator=gen),
            "D": {"none": None, "head": torch.randn(h, generator=gen),
                  "head_dim": torch.randn(h, p, generator=gen)}[d_kind],
            "z": torch.randn(b, h, p, generator=gen) if use_z else None,
            "dt_bias": torch.randn(h, generator=gen) * 0.1 if use_bias else None,
        }
        inp = {k: (None if v is None else v.double()) for k, v in inp.items()}
        leaves = {k: _leaf(inp[k]) for k in names}
        y, s = mamba2_state_update_reference(*[leaves[k] for k in names], dt_softplus=softplus)
        wy = torch.randn(y.shape, generator=gen, dtype=torch.float64)
        ws = torch.randn(s.shape, generator=gen, dtype=torch.float64)
        present = [k for k in names if leaves[k] is not None]
        grads = torch.autograd.grad((y * wy).sum() + (s * ws).sum(), [leaves[k] for k in present])
        cases[name] = {"inputs": {k: v for k, v in inp.items() if v is not None},
                       "softplus": softplus, "y": y.detach(), "new_state": s.detach(),
                       "wy": wy, "ws": ws, "grads": dict(zip(present, grads))}
    return cases


def path_scan_cases():
    """VMamba four-path scan: the reference verifier's shapes
    (benchmarks/verify_path_scan.py:218-238), fp64, with gradients under a
    seeded cotangent, plus the path orders of a few maps."""
    shapes = {
        "fb_1x3x3x2_5x7": ((1, 3, 3, 2, 5, 7), "sum"),
        "fb_2x16x1x8_8x8": ((2, 16, 1, 8, 8, 8), "sum"),
        "fb_2x8x2x4_6x5": ((2, 8, 2, 4, 6, 5), "sum"),
        "five_states": ((1, 6, 2, 5, 13, 3), "sum"),
        "mean_merge": ((1, 4, 1, 3, 4, 5), "mean"),
        "single_row": ((1, 4, 1, 3, 1, 7), "sum"),
        "single_column": ((1, 4, 1, 3, 7, 1), "sum"),
        "thirty_two_states": ((1, 4, 2, 32, 5, 7), "sum"),
    }
    cases = {}
    for idx, (name, (shape, merge)) in enumerate(shapes.items()):
        args = ss2d_inputs(*shape, seed=500 + idx, dtype=torch.float64)
        leaves = [_leaf(t) for t in args]
        y = ss2d_scan_reference(*leaves, merge=merge)
        gen = torch.Generator().manual_seed(600 + idx)
        dy = torch.randn(y.shape, generator=gen, dtype=torch.float64)
        grads = torch.autograd.grad(y, leaves, dy)
        cases[name] = {"inputs": dict(zip(("u", "dt", "A", "B", "C"), args)), "merge": merge,
                       "y": y.detach(), "dy": dy, "grads": dict(zip(("u", "dt", "A", "B", "C"), grads))}
    cases["orders"] = {(h, w): path_orders(h, w) for h, w in ((4, 3), (1, 6), (6, 1), (5, 5), (3, 4))}
    return cases


def causal_conv1d_cases():
    """The reference verifier's forward/gradient cases (benchmarks/
    verify_causal_conv1d.py:171-182, with fewer channels so the fixture stays
    small) and update cases (:185-193), fp64."""
    cases = {}
    shapes = {  # name: batch, channels, length, K, activation, initial state
        "decode_1x128": (1, 128, 1, 4, "silu", True),
        "short_2x64x16": (2, 64, 16, 4, "silu", False),
        "prefill_1x8x300": (1, 8, 300, 4, "silu", True),
        "prefill_2x8x129": (2, 8, 129, 4, None, False),
        "narrow_2x8x200_k8": (2, 8, 200, 8, None, False),
        "k1_2x16x33": (2, 16, 33, 1, None, True),
        "k2_3x8x5": (3, 8, 5, 2, "silu", True),
        "short_below_taps": (2, 8, 2, 4, "silu", True),
    }
    for idx, (name, (b, c, l, k, act, has_state)) in enumerate(shapes.items()):
        g = torch.Generator().manual_seed(700 + idx)
        x = torch.randn(b, c, l, generator=g, dtype=torch.float64)
        w = torch.randn(c, 1, k, generator=g, dtype=torch.float64) * 0.5
        bias = torch.randn(c, generator=g, dtype=torch.float64)
        init = torch.randn(b, c, k - 1, generator=g, dtype=torch.float64) if has_state else None
        leaves = [_leaf(t) for t in (x, w, bias, init)]
        out, final = _cc.causal_conv1d_ref(leaves[0], leaves[1], leaves[2], act, leaves[3], True)
        dout = torch.randn(out.shape, generator=g, dtype=torch.float64)
        dfinal = torch.randn(final.shape, generator=g, dtype=torch.float64)
        present = [t for t in leaves if t is not None]
        grads = torch.autograd.grad((out * dout).sum() + (final * dfinal).sum(), present,
                                    allow_unused=True)
        names = [n for n, t in zip(("x", "weight", "bias", "initial_state"), leaves) if t is not None]
        cases[name] = {"inputs": {"x": x, "weight": w, "bias": bias, "initial_state": init},
                       "activation": act, "out": out.detach().clone(), "final": final.detach().clone(),
                       "dout": dout, "dfinal": dfinal,
                       "grads": {n: (gr.clone() if gr is not None else torch.zeros_like(t))
                                 for n, gr, t in zip(names, grads, present)}}
    updates = {  # name: batch, channels, q, K, activation, state columns
        "update_1x256x1": (1, 256, 1, 4, "silu", 3),
        "update_8x64x1": (8, 64, 1, 4, "silu", 3),
        "update_1x128x4": (1, 128, 4, 4, "silu", 3),
        "update_wide_state": (8, 64, 1, 4, "silu", 8),
        "update_q_beyond_state": (2, 16, 5, 4, None, 3),
        "update_k1": (2, 16, 1, 1, None, 0),
    }
    for idx, (name, (b, c, q, k, act, cols)) in enumerate(updates.items()):
        g = torch.Generator().manual_seed(800 + idx)
        x = torch.randn(b, c, q, generator=g, dtype=torch.float64)
        state = torch.randn(b, c, cols, generator=g, dtype=torch.float64)
        w = torch.randn(c, 1, k, generator=g, dtype=torch.float64) * 0.5
        bias = torch.randn(c, generator=g, dtype=torch.float64)
        st = state.clone()
        out = _cc._update_aten(x, st, w[:, 0, :], bias, act)
        cases[name] = {"inputs": {"x": x, "state": state, "weight": w, "bias": bias},
                       "activation": act, "out": out.clone(), "new_state": st}
    return cases


def gated_norm_cases():
    """The reference verifier's correctness cases (benchmarks/verify_gated_norm.py:
    79-97, 121-131), with fewer rows so the fixture stays small, fp64, with
    gradients under a seeded cotangent."""
    shapes = {  # name: shape, group_size, bias, gate, norm_before_gate, eps
        "whole_axis": ((4, 300), None, True, True, True, 1e-5),
        "group_60": ((4, 300), 60, True, True, True, 1e-5),
        "group_100_eps": ((4, 300), 100, True, True, True, 1e-6),
        "group_150_before": ((4, 300), 150, True, True, False, 1e-5),
        "no_bias": ((4, 300), None, False, True, True, 1e-5),
        "no_gate": ((4, 300), None, True, False, True, 1e-5),
        "group_60_before": ((4, 300), 60, True, True, False, 1e-5),
        "eps_one": ((4, 300), None, True, True, True, 1.0),
        "batched_3d": ((2, 3, 300), 100, True, True, True, 1e-5),
        "batched_4d": ((2, 3, 2, 128), 32, True, True, True, 1e-5),
        "narrow": ((1, 64), 16, True, True, False, 1e-5),
        "wide_group": ((2, 2048), 1024, True, True, True, 1e-5),
    }
    cases = {}
    for idx, (name, (shape, group, bias, gate, before, eps)) in enumerate(shapes.items()):
        g = torch.Generator().manual_seed(900 + idx)
        x = torch.randn(*shape, generator=g, dtype=torch.float64)
        w = torch.randn(shape[-1], generator=g, dtype=torch.float64)
        b = torch.randn(shape[-1], generator=g, dtype=torch.float64) if bias else None
        z = torch.randn(*shape, generator=g, dtype=torch.float64) if gate else None
        leaves = [_leaf(t) for t in (x, w, b, z)]
        out = rmsnorm_gated_reference(leaves[0], leaves[1], leaves[2], leaves[3], eps=eps,
                                      group_size=group, norm_before_gate=before)
        dy = torch.randn(out.shape, generator=g, dtype=torch.float64)
        present = [t for t in leaves if t is not None]
        names = [n for n, t in zip(("x", "weight", "bias", "z"), leaves) if t is not None]
        grads = torch.autograd.grad(out, present, dy)
        cases[name] = {"inputs": {"x": x, "weight": w, "bias": b, "z": z}, "group_size": group,
                       "norm_before_gate": before, "eps": eps, "out": out.detach().clone(),
                       "dy": dy, "grads": {n: gr.clone() for n, gr in zip(names, grads)}}
    return cases


MAKERS = {
    "selective_scan": selective_scan_cases,
    "mamba2_chunk": ssd_cases,
    "mamba2_state": decode_cases,
    "path_scan": path_scan_cases,
    "causal_conv1d": causal_conv1d_cases,
    "gated_norm": gated_norm_cases,
}


def main():
    wanted = sys.argv[1:] or list(MAKERS)
    for name in wanted:
        torch.save(MAKERS[name](), HERE / f"{name}.pt")
    for f in sorted(HERE.glob("*.pt")):
        print(f.name, f.stat().st_size)


if __name__ == "__main__":
    main()
