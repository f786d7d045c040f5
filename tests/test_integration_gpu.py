"""End-to-end blocks through the public ops, against the fp64 references.

The reference's integration verifier (benchmarks/verify_cv_integration.py:37-74,
:77-91, :99-125) builds a small Mamba-2 block (in_proj -> causal conv1d + SiLU
-> SSD chunk scan with D, dt_bias and softplus -> gated RMSNorm -> out_proj)
and a VMamba-style four-path block, runs them once through the CPU references
and once through the fused device ops, and compares the loss, every parameter
gradient and one SGD step.  Here the CPU side is the fp64 oracle and the device
side this package's CUDA ops; the limits are the verifier's (loss 5e-5,
gradients rtol 2e-4 / atol 2e-5) for fp32, and norm-relative 2e-2 for a bf16
block at the Mamba-2 head shape (head dim 64, state 128: the tensor-core SSD).
"""

import pytest
import torch
import torch.nn.functional as F

from oracle import ssm_oracle as orc

pytestmark = pytest.mark.gpu


def _cv():
    from metal_kernelops_b200 import cv
    return cv


class Mamba2Block(torch.nn.Module):
    """The verifier's Mamba-2 block; `reference=True` runs the oracle ops."""

    def __init__(self, d_model=24, heads=2, head_dim=6, d_state=5, conv=4, ngroups=1, chunk=8):
        super().__init__()
        self.heads, self.head_dim, self.d_state, self.ngroups, self.chunk = heads, head_dim, d_state, ngroups, chunk
        inner = heads * head_dim
        self.inner = inner
        bc = 2 * ngroups * d_state
        self.in_proj = torch.nn.Linear(d_model, 2 * inner + bc + heads)
        self.conv_weight = torch.nn.Parameter(torch.randn(inner + bc, 1, conv) * .3)
        self.conv_bias = torch.nn.Parameter(torch.randn(inner + bc) * .1)
        self.a_log = torch.nn.Parameter(torch.randn(heads) * .2)
        self.d_skip = torch.nn.Parameter(torch.ones(heads))
        self.dt_bias = torch.nn.Parameter(torch.randn(heads) * .2)
        self.norm_weight = torch.nn.Parameter(torch.ones(inner))
        self.out_proj = torch.nn.Linear(inner, d_model)

    def forward(self, x, reference=False):
        cv = None if reference else _cv()
        batch, length = x.shape[:2]
        gn = self.ngroups * self.d_state
        zxbcdt = self.in_proj(x)
        z = zxbcdt[..., :self.inner]
        xbc = zxbcdt[..., self.inner:2 * self.inner + 2 * gn]
        dt = zxbcdt[..., 2 * self.inner + 2 * gn:]
        conv = orc.causal_conv1d_ref if reference else cv.causal_conv1d_fn
        xbc = conv(xbc.transpose(1, 2), self.conv_weight.reshape(self.inner + 2 * gn, -1),
                   self.conv_bias, activation="silu").transpose(1, 2)
        x_ssm = xbc[..., :self.inner].reshape(batch, length, self.heads, self.head_dim)
        B = xbc[..., self.inner:self.inner + gn].reshape(batch, length, self.ngroups, self.d_state)
        C = xbc[..., self.inner + gn:].reshape(batch, length, self.ngroups, self.d_state)
        A = -torch.exp(self.a_log)
        scan = orc.mamba2_chunk_scan_ref if reference else cv.mamba2_chunk_scan
        y, _ = scan(x_ssm, dt, A, B, C, chunk_size=self.chunk, D=self.d_skip,
                    dt_bias=self.dt_bias, dt_softplus=True)
        y = y.reshape(batch, length, self.inner)
        if reference:
            y = orc.rmsnorm_gated_ref(y, self.norm_weight, z=z, group_size=self.inner // self.ngroups,
                                      norm_before_gate=False)
        else:
            y = cv.rmsnorm_gated(y, self.norm_weight, z=z, group_size=self.inner // self.ngroups,
                                 norm_before_gate=False)
        return self.out_proj(y).square().mean()


class PathBlock(torch.nn.Module):
    """The verifier's VMamba-style block around the four-path scan."""

    def __init__(self, channels=6, groups=2, states=4):
        super().__init__()
        self.groups, self.states = groups, states
        self.u = torch.nn.Conv2d(channels, channels, 3, padding=1)
        self.dt = torch.nn.Conv2d(channels, channels, 1)
        self.b = torch.nn.Conv2d(channels, groups * states, 1)
        self.c = torch.nn.Conv2d(channels, groups * states, 1)
        self.a = torch.nn.Parameter(-torch.rand(channels, states))

    def forward(self, x, reference=False):
        u = self.u(x)
        dt = F.softplus(self.dt(x))
        shape = (x.shape[0], self.groups, self.states, x.shape[2], x.shape[3])
        B = self.b(x).reshape(shape)
        C = self.c(x).reshape(shape)
        scan = orc.ss2d_scan_ref if reference else _cv().ss2d_scan
        return scan(u, dt, self.a, B, C, merge="sum").square().mean()


def _pair(make, seed):
    torch.manual_seed(seed)
    cpu = make().double()
    dev = make().cuda()
    dev.load_state_dict({k: v.float() for k, v in cpu.state_dict().items()})
    return cpu, dev


def _check_step(cpu, dev, x, loss_tol=5e-5, rtol=2e-4, atol=2e-5, dtype=torch.float32):
    cpu.zero_grad(set_to_none=True)
    dev.zero_grad(set_to_none=True)
    loss_c = cpu(x.double(), reference=True)
    with torch.autocast("cuda", dtype=dtype, enabled=dtype != torch.float32):
        loss_d = dev(x.cuda())
    loss_c.backward()
    loss_d.backward()
    torch.testing.assert_close(loss_d.detach().double().cpu(), loss_c.detach(), rtol=loss_tol, atol=loss_tol)
    for (name, a), (_, b) in zip(cpu.named_parameters(), dev.named_parameters()):
        assert b.grad is not None, name
        if dtype == torch.float32:
            torch.testing.assert_close(b.grad.double().cpu(), a.grad, rtol=rtol, atol=atol, msg=name)
        else:
            rel = float((b.grad.double().cpu() - a.grad).norm() / (a.grad.norm() + 1e-30))
            assert rel <= rtol, (name, rel)
    before = {n: p.detach().clone() for n, p in dev.named_parameters()}
    torch.optim.SGD(cpu.parameters(), lr=.03).step()
    torch.optim.SGD(dev.parameters(), lr=.03).step()
    assert all(not torch.equal(before[n], p) for n, p in dev.named_parameters())
    if dtype == torch.float32:
        for (name, a), (_, b) in zip(cpu.named_parameters(), dev.named_parameters()):
            torch.testing.assert_close(b.detach().double().cpu(), a.detach(), rtol=1e-4, atol=1e-5, msg=name)


def test_mamba2_block_verifier_shape():
    cpu, dev = _pair(Mamba2Block, 17)
    _check_step(cpu, dev, torch.randn(2, 19, 24))


def test_mamba2_block_grouped_longer():
    make = lambda: Mamba2Block(d_model=48, heads=4, head_dim=8, d_state=16, ngroups=2, chunk=32)  # noqa: E731
    cpu, dev = _pair(make, 18)
    _check_step(cpu, dev, torch.randn(2, 150, 48))


def test_mamba2_block_bf16_tensor_core_shape():
    """Head dim 64 and state 128 in bf16 autocast: the SSD runs on the tensor
    cores, conv1d and the norm in bf16 storage; against fp64 with the bf16
    norm-relative limit."""
    make = lambda: Mamba2Block(d_model=128, heads=4, head_dim=64, d_state=128, ngroups=1, chunk=64)  # noqa: E731
    cpu, dev = _pair(make, 19)
    _check_step(cpu, dev, torch.randn(2, 160, 128), loss_tol=2e-2, rtol=2e-2, dtype=torch.bfloat16)


def test_path_block_verifier_shape():
    cpu, dev = _pair(PathBlock, 20)
    _check_step(cpu, dev, torch.randn(2, 6, 9, 11))
