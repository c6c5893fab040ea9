"""GroupNorm -> SiLU fusion and the GroupNorm -> SiLU -> conv block
(nn.Sequential patch): parity with the unfused stock chain, fused path forced
(contest off) and through the contest, and the declines (live gradients,
non-affine GroupNorm, grouped conv, other Sequentials)."""
from __future__ import annotations

import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

import oracle

pytestmark = pytest.mark.gpu


def _np(t):
    return t.detach().float().cpu().numpy()


@pytest.fixture
def patched():
    import amd_tuned_torch
    from amd_tuned_torch import kernel_select
    kernel_select.reset()
    amd_tuned_torch.enable()
    yield amd_tuned_torch
    amd_tuned_torch.disable()
    kernel_select.reset()


def _block(conv_cls, C, Co, G, dt, dev, seed):
    torch.manual_seed(seed)
    m = nn.Sequential(nn.GroupNorm(G, C), nn.SiLU(), conv_cls(C, Co, 3, padding=1))
    with torch.no_grad():
        m[0].weight.uniform_(0.5, 1.5)
        m[0].bias.normal_(0, 0.1)
    return m.to(dev, dt).eval()


def _chain_ref(m, x):
    """fp32 CPU chain with the activation rounded to the input dtype once
    (the fused path's single rounding point)."""
    xf = x.float().cpu()
    h = F.silu(F.group_norm(xf, m[0].num_groups, m[0].weight.float().cpu(),
                            m[0].bias.float().cpu(), m[0].eps)).to(x.dtype).float()
    conv = F.conv3d if isinstance(m[2], nn.Conv3d) else F.conv2d
    return conv(h, m[2].weight.float().cpu(), m[2].bias.float().cpu(), padding=1)


@pytest.mark.parametrize("conv_cls,shape,Co,G,dt", [
    (nn.Conv3d, (1, 128, 6, 32, 32), 128, 32, torch.bfloat16),
    (nn.Conv3d, (2, 64, 4, 16, 24), 64, 8, torch.float16),
    (nn.Conv2d, (2, 64, 32, 48), 64, 32, torch.float16),
    (nn.Conv2d, (1, 128, 40, 40), 96, 16, torch.bfloat16),
])
@pytest.mark.parametrize("contest", [False, True])
def test_block_matches_chain(cuda, patched, monkeypatch, conv_cls, shape, Co, G, dt, contest):
    from amd_tuned_torch import kernel_select
    monkeypatch.setattr(kernel_select, "_ENABLED", contest)
    m = _block(conv_cls, shape[1], Co, G, dt, cuda, seed=sum(shape))
    x = torch.randn(*shape, generator=torch.Generator().manual_seed(1)).to(cuda, dt)
    with torch.no_grad():
        y = m(x)
    with torch.no_grad():
        ref = _chain_ref(m, x)
    assert tuple(y.shape) == tuple(ref.shape) and y.dtype == dt
    # Three ops: with the contest on, the unfused chain may win and it rounds
    # the activation twice (GroupNorm out, SiLU out) before the output's own
    # rounding, one bf16 ulp being 3.9e-3 -- the per-op 2e-3 bar holds for fp16.
    tol = 5e-3 if dt == torch.bfloat16 else 2e-3
    assert oracle.rel_l2(_np(y), ref.numpy()) <= tol


def test_fused_conv2d_block_repeated_calls(cuda, patched, monkeypatch):
    from amd_tuned_torch import kernel_select
    monkeypatch.setattr(kernel_select, "_ENABLED", False)
    m = _block(nn.Conv2d, 64, 64, 32, torch.float16, cuda, seed=9)
    x = torch.randn(2, 64, 16, 16, device=cuda, dtype=torch.float16)
    with torch.no_grad():
        ys = [m(x) for _ in range(3)]
    for y in ys[1:]:
        assert torch.equal(y, ys[0])


def test_fused_block_is_what_runs_with_contest_off(cuda, patched, monkeypatch):
    from amd_tuned_torch import conv_fusion_ops, kernel_select
    monkeypatch.setattr(kernel_select, "_ENABLED", False)
    calls = []
    orig = conv_fusion_ops._fused_block
    monkeypatch.setattr(conv_fusion_ops, "_fused_block",
                        lambda *a: calls.append(1) or orig(*a))
    m = _block(nn.Conv3d, 64, 64, 32, torch.bfloat16, cuda, seed=3)
    x = torch.randn(1, 64, 4, 16, 16, device=cuda, dtype=torch.bfloat16)
    with torch.no_grad():
        m(x)
    assert calls == [1]


def test_block_declines(cuda, patched, monkeypatch):
    from amd_tuned_torch import conv_fusion_ops
    calls = []
    orig = conv_fusion_ops._fused_block
    monkeypatch.setattr(conv_fusion_ops, "_fused_block",
                        lambda *a: calls.append(1) or orig(*a))
    x = torch.randn(1, 64, 4, 16, 16, device=cuda, dtype=torch.bfloat16)
    m = _block(nn.Conv3d, 64, 64, 32, torch.bfloat16, cuda, seed=4)
    y = m(x)                                   # gradients live (module params) -> stock chain
    assert y.requires_grad and calls == []
    m2 = nn.Sequential(nn.GroupNorm(32, 64, affine=False), nn.SiLU(),
                       nn.Conv3d(64, 64, 3, padding=1)).to(cuda, torch.bfloat16).eval()
    m3 = nn.Sequential(nn.GroupNorm(32, 64), nn.SiLU(),
                       nn.Conv3d(64, 64, 3, padding=1, groups=2)).to(cuda, torch.bfloat16).eval()
    m4 = nn.Sequential(nn.GroupNorm(32, 64), nn.ReLU(),
                       nn.Conv3d(64, 64, 3, padding=1)).to(cuda, torch.bfloat16).eval()
    with torch.no_grad():
        for mm in (m2, m3, m4):
            mm(x)
    assert calls == []


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16])
def test_group_norm_silu(cuda, dt):
    from amd_tuned_torch import conv_fusion_ops
    x = (torch.randn(2, 64, 8, 16, 16, generator=torch.Generator().manual_seed(5)) * 2).to(dt)
    w = torch.rand(64, generator=torch.Generator().manual_seed(6)).to(dt) + 0.5
    b = torch.randn(64, generator=torch.Generator().manual_seed(7)).to(dt) * 0.1
    y = conv_fusion_ops.group_norm_silu(x.to(cuda), 16, w.to(cuda), b.to(cuda), 1e-5)
    ref = F.silu(F.group_norm(x.float(), 16, w.float(), b.float(), 1e-5))
    assert oracle.rel_l2(_np(y), ref.numpy()) <= 2e-3
