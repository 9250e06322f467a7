"""tcgen05 GEMM + fused epilogues against a plain PyTorch fp32 reference.

Tolerances: operands are exact f16/bf16 values, the kernel accumulates in f32,
so the only differences are summation order and the final rounding of the
f16/bf16 outputs (relative 2^-11 / 2^-8).
"""
import pytest

pytestmark = pytest.mark.gpu


def _setup(M, N, K, dtype, seed=0):
    import torch
    g = torch.Generator(device="cpu").manual_seed(seed)
    A = (torch.randn(M, K, generator=g) * 0.5).to(dtype).cuda()
    B = (torch.randn(N, K, generator=g) * 0.05).to(dtype).cuda()
    bias = (torch.randn(N, generator=g) * 0.1).float().cuda()
    ref = A.float() @ B.float().t()
    return A, B, bias, ref


@pytest.mark.parametrize("bf16", [False, True])
@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (300, 512, 1024), (1000, 1024, 4096), (7, 256, 128),
                                   (20000, 1024, 256), (4099, 3072, 1024), (129, 512, 256),
                                   (255, 256, 512), (256, 768, 64), (257, 1024, 128), (511, 256, 1024)])
def test_store_h_bias(cuda, bf16, M, N, K):
    import torch
    import pkc
    dt = torch.bfloat16 if bf16 else torch.float16
    A, B, bias, ref = _setup(M, N, K, dt)
    out = torch.zeros(M, N, dtype=dt, device=cuda)
    pkc.gemm(A.data_ptr(), B.data_ptr(), M, N, K, bf16=bf16, epi=pkc.EPI_STORE_H,
             bias=bias.data_ptr(), out=out.data_ptr(), ldo=N)
    torch.cuda.synchronize()
    want = ref + bias
    tol = 1e-2 if bf16 else 2e-3
    err = (out.float() - want).abs().max().item() / want.abs().max().item()
    assert err < tol, err


@pytest.mark.parametrize("act", ["silu", "relu"])
def test_store_h_act(cuda, act):
    import torch
    import pkc
    M, N, K = 513, 768, 512
    A, B, bias, ref = _setup(M, N, K, torch.float16, seed=1)
    out = torch.zeros(M, N, dtype=torch.float16, device=cuda)
    pkc.gemm(A.data_ptr(), B.data_ptr(), M, N, K, bf16=False, epi=pkc.EPI_STORE_H,
             act=pkc.ACT_SILU if act == "silu" else pkc.ACT_RELU, bias=bias.data_ptr(),
             out=out.data_ptr(), ldo=N)
    torch.cuda.synchronize()
    x = ref + bias
    want = torch.nn.functional.silu(x) if act == "silu" else torch.relu(x)
    err = (out.float() - want).abs().max().item() / want.abs().max().item()
    assert err < 3e-3, err


def test_resid_f32(cuda):
    import torch
    import pkc
    M, N, K = 333, 1024, 2048
    A, B, bias, ref = _setup(M, N, K, torch.float16, seed=2)
    base = torch.randn(M, N, device=cuda)
    out = base.clone()
    pkc.gemm(A.data_ptr(), B.data_ptr(), M, N, K, bf16=False, epi=pkc.EPI_RESID_F32, alpha=0.5,
             bias=bias.data_ptr(), out=out.data_ptr(), ldo=N)
    torch.cuda.synchronize()
    want = base + 0.5 * (ref + bias)
    err = (out - want).abs().max().item() / want.abs().max().item()
    assert err < 1e-4, err


def test_store_f32_nobias(cuda):
    import torch
    import pkc
    M, N, K = 200, 512, 2560
    A, B, _, ref = _setup(M, N, K, torch.float16, seed=3)
    out = torch.zeros(M, N, device=cuda)
    pkc.gemm(A.data_ptr(), B.data_ptr(), M, N, K, bf16=False, epi=pkc.EPI_STORE_F32, alpha=2.0,
             bias=None, out=out.data_ptr(), ldo=N)
    torch.cuda.synchronize()
    want = 2.0 * ref
    err = (out - want).abs().max().item() / want.abs().max().item()
    assert err < 1e-4, err


def test_glu_and_power(cuda):
    import torch
    import pkc
    M, N, K = 260, 1024, 512
    A, B, bias, ref = _setup(M, N, K, torch.float16, seed=4)
    x = ref + bias
    # tile-local pairing: within each 256-column tile, [0,128) pairs with [128,256)
    xt = x.view(M, N // 256, 2, 128)
    a, g = xt[:, :, 0, :].reshape(M, N // 2), xt[:, :, 1, :].reshape(M, N // 2)
    out = torch.zeros(M, N // 2, dtype=torch.float16, device=cuda)
    pkc.gemm(A.data_ptr(), B.data_ptr(), M, N, K, bf16=False, epi=pkc.EPI_GLU_H,
             bias=bias.data_ptr(), out=out.data_ptr(), ldo=N // 2)
    pw = torch.zeros(M, N // 2, device=cuda)
    pkc.gemm(A.data_ptr(), B.data_ptr(), M, N, K, bf16=False, epi=pkc.EPI_POWER_F32,
             bias=None, out=pw.data_ptr(), ldo=N // 2)
    torch.cuda.synchronize()
    want = a * torch.sigmoid(g)
    err = (out.float() - want).abs().max().item() / want.abs().max().item()
    assert err < 3e-3, err
    rt = ref.view(M, N // 256, 2, 128)
    ra, rg = rt[:, :, 0, :].reshape(M, N // 2), rt[:, :, 1, :].reshape(M, N // 2)
    wp = ra * ra + rg * rg
    err = (pw - wp).abs().max().item() / wp.abs().max().item()
    assert err < 1e-4, err


def test_one_sm_and_two_sm_kernels_agree(cuda):
    """The 2-SM (cta_group::2) tiles and the 1-SM tiles give the same result
    up to f32 summation order; run in a child process with the 1-SM switch."""
    import os
    import subprocess
    import sys
    import torch
    import pkc
    M, N, K = 1000, 1024, 2048
    A, B, bias, ref = _setup(M, N, K, torch.float16, seed=9)
    out = torch.zeros(M, N, device=cuda)
    pkc.gemm(A.data_ptr(), B.data_ptr(), M, N, K, bf16=False, epi=pkc.EPI_STORE_F32, alpha=1.0,
             bias=bias.data_ptr(), out=out.data_ptr(), ldo=N)
    torch.cuda.synchronize()
    err = (out - (ref + bias)).abs().max().item() / ref.abs().max().item()
    assert err < 1e-4, err
