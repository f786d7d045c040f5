"""Seeded synthetic workloads with the hot-path configurations' shapes and
value distributions (BASELINE configs 0-4 and the reference verifiers).

Used by ``bench.py``, ``__graft_entry__.smoke()`` and the tests.  Everything is
generated in fp32 on the CPU with ``torch.Generator().manual_seed(seed)`` and
then cast, so every rank and every run sees the same tensors.
"""

from __future__ import annotations

import math

import torch

__all__ = ["selective_scan_inputs", "selective_scan_rows", "ssd_inputs", "decode_inputs", "ss2d_inputs"]


def _softplus_inv(v):
    return math.log(math.expm1(v))


def selective_scan_inputs(batch, dim, length, dstate, groups=1, seed=1000,
                          act_dtype=torch.float32, delta_std=0.5):
    """Config 0/1/2 distributions: u, z, B, C ~ N(0,1); delta ~ N(0, delta_std^2);
    delta_bias ~ U(log(e^0.001-1), log(e^0.1-1)); A[d, n] = -(n+1); D ~ N(0,1);
    dout ~ N(0,1).  Generated in fp32 on the CPU, then cast (activations and
    B/C to ``act_dtype``; A, D, delta_bias stay fp32)."""
    g = torch.Generator().manual_seed(seed)
    u = torch.randn(batch, dim, length, generator=g)
    delta = torch.randn(batch, dim, length, generator=g) * delta_std
    lo, hi = _softplus_inv(0.001), _softplus_inv(0.1)
    delta_bias = torch.rand(dim, generator=g) * (hi - lo) + lo
    A = -torch.arange(1, dstate + 1, dtype=torch.float32).repeat(dim, 1)
    B = torch.randn(batch, groups, dstate, length, generator=g)
    C = torch.randn(batch, groups, dstate, length, generator=g)
    D = torch.randn(dim, generator=g)
    z = torch.randn(batch, dim, length, generator=g)
    dout = torch.randn(batch, dim, length, generator=g)
    cast = lambda t: t.to(act_dtype)  # noqa: E731
    return dict(u=cast(u), delta=cast(delta), A=A, B=cast(B), C=cast(C), D=D,
                z=cast(z), delta_bias=delta_bias, dout=cast(dout))


def selective_scan_rows(dim, length, dstate, groups, seed, lo, hi, act_dtype=torch.bfloat16):
    """Batch rows ``lo:hi`` of a large selective-scan configuration (config 2:
    335 M elements per activation) without materialising the whole batch: row
    ``b`` comes from its own generator seeded ``seed * 1000 + b``, and the
    shared parameters A, D, delta_bias from ``seed``, so every rank (and every
    test) sees the same global tensors whatever slice it generates."""
    rows = [selective_scan_inputs(1, dim, length, dstate, groups, seed=seed * 1000 + b,
                                  act_dtype=act_dtype) for b in range(lo, hi)]
    out = {k: torch.cat([r[k] for r in rows]) for k in ("u", "delta", "z", "dout", "B", "C")}
    base = selective_scan_inputs(1, dim, 1, dstate, groups, seed=seed)
    for k in ("A", "D", "delta_bias"):
        out[k] = base[k]
    return out


def ssd_inputs(batch, length, nheads, headdim, dstate, ngroups, seed=1003,
               dtype=torch.bfloat16):
    """Config 3 distributions: x, B, C ~ N(0,1) in ``dtype``; raw dt fp32 ~ N(0,1)
    with dt_bias[h] = softplus^-1(u_h), u_h log-uniform on [0.001, 0.1] and
    dt_softplus=True; A = -U(1, 16) fp32; D ~ N(0,1) per head; dy ~ N(0,1)."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(batch, length, nheads, headdim, generator=g)
    dt = torch.randn(batch, length, nheads, generator=g)
    lu = torch.rand(nheads, generator=g) * (math.log(0.1) - math.log(0.001)) + math.log(0.001)
    dt_bias = torch.log(torch.expm1(torch.exp(lu)))
    A = -(torch.rand(nheads, generator=g) * 15 + 1)
    B = torch.randn(batch, length, ngroups, dstate, generator=g)
    C = torch.randn(batch, length, ngroups, dstate, generator=g)
    D = torch.randn(nheads, generator=g)
    dy = torch.randn(batch, length, nheads, headdim, generator=g)
    return dict(x=x.to(dtype), dt=dt, A=A, B=B.to(dtype), C=C.to(dtype), D=D,
                dt_bias=dt_bias, dy=dy.to(dtype))


def decode_inputs(batch, nheads, headdim, dstate, ngroups, seed=1004,
                  dtype=torch.bfloat16):
    """Config 4 distributions: fp32 state ~ N(0,1); x, B, C ~ N(0,1) in ``dtype``;
    dt and A as in config 3 (dt per head, dt_softplus=True); D ~ N(0,1)."""
    g = torch.Generator().manual_seed(seed)
    state = torch.randn(batch, nheads, headdim, dstate, generator=g)
    x = torch.randn(batch, nheads, headdim, generator=g)
    dt = torch.randn(batch, nheads, generator=g)
    lu = torch.rand(nheads, generator=g) * (math.log(0.1) - math.log(0.001)) + math.log(0.001)
    dt_bias = torch.log(torch.expm1(torch.exp(lu)))
    A = -(torch.rand(nheads, generator=g) * 15 + 1)
    B = torch.randn(batch, ngroups, dstate, generator=g)
    C = torch.randn(batch, ngroups, dstate, generator=g)
    D = torch.randn(nheads, generator=g)
    return dict(state=state, x=x.to(dtype), dt=dt, A=A, B=B.to(dtype), C=C.to(dtype),
                D=D, dt_bias=dt_bias)


def ss2d_inputs(batch, channels, groups, states, height, width, seed, dtype=torch.float32):
    """The reference verifier's distributions (benchmarks/verify_path_scan.py:69-84):
    u, B, C ~ N(0,1); dt ~ U(0.05, 0.25); A = -(U(0,1) + 0.1)."""
    g = torch.Generator().manual_seed(seed)
    shape = (batch, channels, height, width)
    u = torch.randn(shape, generator=g, dtype=dtype)
    dt = torch.rand(shape, generator=g, dtype=dtype) * 0.2 + 0.05
    A = -(torch.rand((channels, states), generator=g, dtype=dtype) + 0.1)
    B = torch.randn((batch, groups, states, height, width), generator=g, dtype=dtype)
    C = torch.randn((batch, groups, states, height, width), generator=g, dtype=dtype)
    return u, dt, A, B, C
