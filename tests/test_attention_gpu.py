"""Parity of the 3xTF32 tcgen05 attention kernel (ko_attention_f32) with a float64 reference, through the C ABI.

The reference computes, per batch item and head, softmax(scale * q k^T) v in float64 on the CPU — the math of
mx.fast.scaled_dot_product_attention at fast_rfdetr/model.py:110, :119-120 and :238. Tolerance: normwise relative
error <= 1e-5 (max|gpu - ref| <= 1e-5 * max|ref|), the bar of the other fp32 kernels.
"""
from __future__ import annotations

import math

import pytest
import torch

from kernelopt_b200 import kernels as K

pytestmark = pytest.mark.gpu

REL = 1e-5


def reference(q, k, v, heads, scale):
    """float64 attention on CPU tensors [B, L, heads*hd] -> [B, L, heads*hd]."""
    b, n, w = q.shape
    hd = w // heads
    q, k, v = (t.double().reshape(b, n, heads, hd).transpose(1, 2) for t in (q, k, v))
    p = torch.softmax((q @ k.transpose(-1, -2)) * scale, dim=-1)
    return (p @ v).transpose(1, 2).reshape(b, n, w)


def check(g, ref, what):
    g = g.detach().cpu().double()
    err = (g - ref).abs().max().item()
    scale = ref.abs().max().item()
    assert torch.isfinite(g).all(), what
    assert err <= REL * scale, f"{what}: normwise error {err / scale:.3e} > {REL}"


@pytest.mark.parametrize("b,n,heads,hd", [(8, 401, 6, 64), (2, 1604, 6, 64), (4, 300, 8, 32), (3, 1, 6, 64),
                                          (2, 17, 2, 64), (2, 128, 3, 64), (2, 129, 3, 32), (1, 640, 1, 64)])
def test_attention_fused_qkv_layout(cuda, b, n, heads, hd):
    """q, k, v as column slices of one [B, L, 3*heads*hd] projection (the backbone's layout)."""
    g = torch.Generator().manual_seed(b * 1000 + n)
    w = heads * hd
    qkv = torch.randn(b, n, 3 * w, generator=g)
    ref = reference(qkv[..., :w], qkv[..., w:2 * w], qkv[..., 2 * w:], heads, 1 / math.sqrt(hd))
    d = qkv.to(cuda)
    out = K.attention(d[..., :w], d[..., w:2 * w], d[..., 2 * w:], heads, 1 / math.sqrt(hd))
    K.check_device_status(cuda)
    check(out, ref, f"b={b} n={n} heads={heads} hd={hd}")


def test_attention_separate_tensors_and_peaked_scores(cuda):
    """Separate q/k/v tensors (the decoder's layout) and large scores: softmax far from uniform."""
    g = torch.Generator().manual_seed(5)
    b, n, heads, hd = 2, 300, 8, 32
    q = 3 * torch.randn(b, n, heads * hd, generator=g)
    k = 3 * torch.randn(b, n, heads * hd, generator=g)
    v = torch.randn(b, n, heads * hd, generator=g)
    ref = reference(q, k, v, heads, 1 / math.sqrt(hd))
    out = K.attention(q.to(cuda), k.to(cuda), v.to(cuda), heads, 1 / math.sqrt(hd))
    check(out, ref, "peaked")


def test_attention_writes_into_out_and_rejects_bad_shapes(cuda):
    g = torch.Generator().manual_seed(6)
    q, k, v = (torch.randn(2, 50, 128, generator=g).to(cuda) for _ in range(3))
    out = torch.full((2, 50, 128), float("nan"), device=cuda)
    K.attention(q, k, v, 2, 0.125, out=out)
    check(out, reference(q.cpu(), k.cpu(), v.cpu(), 2, 0.125), "out=")
    with pytest.raises(ValueError):
        K.attention(q, k, v, 3, 0.125)          # head_dim 128/3
    with pytest.raises(ValueError):
        K.attention(q, k, v, 1, 0.125)          # head_dim 128
    with pytest.raises(ValueError):
        K.attention(q.cpu(), k, v, 2, 0.125)    # no CPU path
