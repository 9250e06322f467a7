"""Rel-pos flash attention kernel against a plain PyTorch fp32 restatement of
the reference's attention core (src/relpos_attention.cpp:214-302): scores
(q+u)k^T + rel_shift((q+v)p^T), key mask, softmax(scale * s), times v.

Inputs are exact f16/bf16 values; the kernel rounds q+u / q+v and the
probabilities to the operand type and accumulates in f32, so the bound is a
few operand ulps relative to the output magnitude (2e-2 for bf16, 5e-3 f16).
"""
import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def reference(qkv, ptab, centre, bu, bv, lens, H):
    import torch
    d = ptab.shape[1]
    dk = d // H
    out = torch.zeros(qkv.shape[0], d, dtype=torch.float32, device=qkv.device)
    off = 0
    for T in lens:
        x = qkv[off:off + T].float()
        q = x[:, :d].view(T, H, dk).transpose(0, 1)
        k = x[:, d:2 * d].view(T, H, dk).transpose(0, 1)
        v = x[:, 2 * d:].view(T, H, dk).transpose(0, 1)
        qu = q + bu.view(H, 1, dk)
        qv = q + bv.view(H, 1, dk)
        i = torch.arange(T, device=qkv.device)[:, None]
        j = torch.arange(T, device=qkv.device)[None, :]
        rows = centre - 1 - (i - j)                      # positional row of (i, j)
        p = ptab.float().view(-1, H, dk).transpose(0, 1)  # [H, NP, dk]
        bd_raw = qv @ p.transpose(1, 2)                   # [H, T, NP]
        bd = torch.gather(bd_raw, 2, rows.expand(H, T, T))
        s = (qu @ k.transpose(1, 2) + bd) / math.sqrt(dk)
        a = torch.softmax(s, dim=-1)
        out[off:off + T] = (a @ v).transpose(0, 1).reshape(T, d)
        off += T
    return out


@pytest.mark.parametrize("bf16", [False, True])
@pytest.mark.parametrize("dk,lens", [(128, [1, 7, 64, 100]), (64, [33, 16, 2]), (128, [437, 250]),
                                     (128, [1500])])
def test_relpos_attention_matches_torch(cuda, bf16, dk, lens):
    import torch
    import pkc
    H = 8 if dk == 128 else 4
    d = H * dk
    dt = torch.bfloat16 if bf16 else torch.float16
    g = torch.Generator().manual_seed(sum(lens) + dk)
    M = sum(lens)
    centre = max(lens) + 3  # any centre >= max length gives the same values
    qkv = (torch.randn(M, 3 * d, generator=g) * 0.6).to(dt).to(cuda)
    ptab = (torch.randn(2 * centre - 1, d, generator=g) * 0.6).to(dt).to(cuda)
    bu = (torch.randn(d, generator=g) * 0.05).to(cuda)
    bv = (torch.randn(d, generator=g) * 0.05).to(cuda)
    ctx = torch.zeros(M, d, dtype=dt, device=cuda)
    pkc.relpos_attention(qkv.data_ptr(), ptab.data_ptr(), centre, bu.data_ptr(), bv.data_ptr(), lens,
                         d, H, bf16=bf16, ctx=ctx.data_ptr())
    ref = reference(qkv, ptab, centre, bu, bv, lens, H)
    err = (ctx.float() - ref).abs().max().item() / ref.abs().max().item()
    assert err < (2e-2 if bf16 else 5e-3), err


@pytest.mark.parametrize("bf16", [False, True])
@pytest.mark.parametrize("dk,lens", [(128, [129, 65, 1, 191, 128, 64]), (64, [257, 63, 130])])
def test_relpos_attention_tile_edges(cuda, bf16, dk, lens):
    """Lengths one past / one short of the 128-row query tile and the 64-key tile."""
    test_relpos_attention_matches_torch(cuda, bf16, dk, lens)


@pytest.mark.parametrize("bf16", [False, True])
def test_relpos_attention_late_maximum(cuda, bf16):
    """Keys late in the utterance carry much larger scores than the first key
    tiles, so the running maximum of every row moves after P V has started
    accumulating: the rescale of the partial output must be exact."""
    import torch
    import pkc
    H, dk = 8, 128
    d = H * dk
    lens = [700, 300]
    dt = torch.bfloat16 if bf16 else torch.float16
    g = torch.Generator().manual_seed(77)
    M = sum(lens)
    centre = max(lens)
    qkv = torch.randn(M, 3 * d, generator=g) * 0.8
    # keys 0..383 small, keys 384.. of the first utterance three times larger
    qkv[384:700, d:2 * d] *= 3.0
    qkv = qkv.to(dt).to(cuda)
    ptab = (torch.randn(2 * centre - 1, d, generator=g) * 0.3).to(dt).to(cuda)
    bu = (torch.randn(d, generator=g) * 0.05).to(cuda)
    bv = (torch.randn(d, generator=g) * 0.05).to(cuda)
    ctx = torch.zeros(M, d, dtype=dt, device=cuda)
    pkc.relpos_attention(qkv.data_ptr(), ptab.data_ptr(), centre, bu.data_ptr(), bv.data_ptr(), lens,
                         d, H, bf16=bf16, ctx=ctx.data_ptr())
    ref = reference(qkv, ptab, centre, bu, bv, lens, H)
    err = (ctx.float() - ref).abs().max().item() / ref.abs().max().item()
    assert err < (2e-2 if bf16 else 5e-3), err
