"""Kernels of the f32-accurate path (f32 GGUF weights) against float64.

The split-f16 GEMM carries each f32 operand as hi = f16(v), lo = f16(v - hi)
and accumulates A_hi B_hi + A_hi B_lo + A_lo B_hi in f32, so a product keeps
~22 significant bits; the f32 attention computes scores, softmax (expf) and
P V in f32. Bound: 5e-5 per element (tests/parity.py's comparator; the
tensor core's f32 accumulation over K = 2560 alone reaches ~2e-5), far below
the 1e-3 the encoder must meet and ~50x tighter than a plain f16 GEMM.
"""
import numpy as np
import pytest

from parity import max_rel_err

pytestmark = pytest.mark.gpu

TOL = 5e-5


def split(t):
    """f32 tensor [R, K] -> f16 [R, 2K] rows [hi | lo]."""
    import torch
    hi = t.to(torch.float16)
    lo = (t - hi.float()).to(torch.float16)
    return torch.cat([hi, lo], dim=1).contiguous()


def unsplit(t, K):
    return t[:, :K].double() + t[:, K:2 * K].double()


@pytest.mark.parametrize("M,N,Ks", [(37, 256, 256), (128, 512, 1024), (300, 256, 2560), (1000, 1024, 512)])
@pytest.mark.parametrize("mode", ["store_f32", "resid", "silu_f32", "relu_split", "glu_f32"])
def test_split_gemm_matches_float64(cuda, M, N, Ks, mode):
    import torch
    import pkc
    g = torch.Generator(device=cuda).manual_seed(M * 7 + N + Ks)
    A = torch.randn(M, Ks, generator=g, device=cuda)
    W = torch.randn(N, Ks, generator=g, device=cuda) * 0.02
    bias = torch.randn(N, generator=g, device=cuda) * 0.1
    ref = A.double() @ W.double().T + bias.double()
    a, w = split(A), split(W)
    if mode == "store_f32":
        out = torch.zeros(M, N, device=cuda)
        pkc.gemm_split(a.data_ptr(), w.data_ptr(), M, N, Ks, epi=pkc.EPI_STORE_F32, alpha=0.5,
                       bias=bias.data_ptr(), out=out.data_ptr(), ldo=N)
        want, got = 0.5 * ref, out.double()
    elif mode == "resid":
        x = torch.randn(M, N, generator=g, device=cuda)
        want = x.double() + 0.5 * ref
        pkc.gemm_split(a.data_ptr(), w.data_ptr(), M, N, Ks, epi=pkc.EPI_RESID_F32, alpha=0.5,
                       bias=bias.data_ptr(), out=x.data_ptr(), ldo=N)
        got = x.double()
    elif mode == "silu_f32":
        out = torch.zeros(M, N, device=cuda)
        pkc.gemm_split(a.data_ptr(), w.data_ptr(), M, N, Ks, epi=pkc.EPI_STORE_H, act=pkc.ACT_SILU,
                       bias=bias.data_ptr(), out=out.data_ptr(), ldo=N, ofmt=pkc.OUT_F32)
        want, got = ref * torch.sigmoid(ref), out.double()
    elif mode == "relu_split":
        out = torch.zeros(M, 2 * N, dtype=torch.float16, device=cuda)
        pkc.gemm_split(a.data_ptr(), w.data_ptr(), M, N, Ks, epi=pkc.EPI_STORE_H, act=pkc.ACT_RELU,
                       bias=bias.data_ptr(), out=out.data_ptr(), ldo=2 * N, ofmt=pkc.OUT_SPLIT, split_ld=N)
        want, got = torch.relu(ref), unsplit(out, N)
    else:  # GLU over paired rows: within each 256-row tile, rows [0,128) value, [128,256) gate
        out = torch.zeros(M, N // 2, device=cuda)
        pkc.gemm_split(a.data_ptr(), w.data_ptr(), M, N, Ks, epi=pkc.EPI_GLU_H, bias=bias.data_ptr(),
                       out=out.data_ptr(), ldo=N // 2, ofmt=pkc.OUT_F32)
        r = ref.view(M, N // 256, 2, 128)
        want = (r[:, :, 0] * torch.sigmoid(r[:, :, 1])).reshape(M, N // 2)
        got = out.double()
    e = max_rel_err(got.cpu().numpy(), want.cpu().numpy())
    print(f"split GEMM {mode} M={M} N={N} K={Ks}: max rel err {e:.2e}")
    assert e < TOL, e


def attention_f64(qkv, ptab, centre, bu, bv, lens, H):
    """float64 restatement of the reference's attention core
    (src/relpos_attention.cpp:214-302), rel_shift as the row index
    centre - 1 - (i - j)."""
    import torch
    d = ptab.shape[1]
    dk = d // H
    out = torch.zeros(qkv.shape[0], d, dtype=torch.float64, device=qkv.device)
    off = 0
    for T in lens:
        x = qkv[off:off + T].double()
        q = x[:, :d].view(T, H, dk).transpose(0, 1)
        k = x[:, d:2 * d].view(T, H, dk).transpose(0, 1)
        v = x[:, 2 * d:].view(T, H, dk).transpose(0, 1)
        qu = q + bu.double().view(H, 1, dk)
        qv = q + bv.double().view(H, 1, dk)
        i = torch.arange(T, device=qkv.device)[:, None]
        j = torch.arange(T, device=qkv.device)[None, :]
        rows = centre - 1 - (i - j)
        p = ptab.double().view(-1, H, dk).transpose(0, 1)
        bd = torch.gather(qv @ p.transpose(1, 2), 2, rows.expand(H, T, T))
        a = torch.softmax((qu @ k.transpose(1, 2) + bd) / dk ** 0.5, dim=-1)
        out[off:off + T] = (a @ v).transpose(0, 1).reshape(T, d)
        off += T
    return out


@pytest.mark.parametrize("dk,lens", [(64, [126]), (64, [1, 33, 64, 65, 200]), (128, [437, 250, 17]), (128, [1500])])
def test_attention_f32_matches_float64(cuda, dk, lens):
    import torch
    import pkc
    H = 8
    d = H * dk
    g = torch.Generator(device=cuda).manual_seed(sum(lens) + dk)
    M = sum(lens)
    centre = max(lens) + 2
    qkv = torch.randn(M, 3 * d, generator=g, device=cuda) * 0.8
    ptab = torch.randn(2 * centre - 1, d, generator=g, device=cuda) * 0.6
    bu = torch.randn(d, generator=g, device=cuda) * 0.05
    bv = torch.randn(d, generator=g, device=cuda) * 0.05
    ctx = torch.zeros(M, 2 * d, dtype=torch.float16, device=cuda)
    pkc.relpos_attention_f32(qkv.data_ptr(), ptab.data_ptr(), centre, bu.data_ptr(), bv.data_ptr(), lens, d, H,
                             ctx=ctx.data_ptr())
    want = attention_f64(qkv, ptab, centre, bu, bv, lens, H)
    e = max_rel_err(unsplit(ctx, d).cpu().numpy(), want.cpu().numpy())
    print(f"f32 attention dk={dk} lens={lens}: max rel err {e:.2e}")
    assert e < TOL, e
