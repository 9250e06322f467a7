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


def _chunk_stats(x):
    """per-row (mean, sum of squared deviations) of each 128-column chunk"""
    import torch
    M, N = x.shape
    c = x.view(M, N // 128, 128)
    mean = c.mean(dim=2)
    m2 = ((c - mean[..., None]) ** 2).sum(dim=2)
    return torch.stack([mean, m2], dim=-1)


@pytest.mark.parametrize("M,N,K", [(333, 1024, 2048), (1, 512, 256), (4099, 1024, 4096), (129, 256, 128)])
def test_resid_stats(cuda, M, N, K):
    """The residual GEMM's epilogue also writes the updated rows' statistics
    per 128-column chunk (the input of the LayerNorm fused into the next GEMM)."""
    import torch
    import pkc
    A, B, bias, ref = _setup(M, N, K, torch.float16, seed=11)
    base = torch.randn(M, N, device=cuda) + 3.0
    x = base.clone()
    stats = torch.full((M, N // 128, 2), float("nan"), device=cuda)
    pkc.gemm_resid_stats(A.data_ptr(), B.data_ptr(), M, N, K, bf16=False, alpha=0.5, bias=bias.data_ptr(),
                         x=x.data_ptr(), stats=stats.data_ptr())
    torch.cuda.synchronize()
    want = base + 0.5 * (ref + bias)
    assert (x - want).abs().max().item() / want.abs().max().item() < 1e-4
    ws = _chunk_stats(x)
    assert torch.isfinite(stats).all()
    assert (stats[..., 0] - ws[..., 0]).abs().max().item() < 1e-5 * max(1.0, ws[..., 0].abs().max().item())
    assert (stats[..., 1] - ws[..., 1]).abs().max().item() < 1e-4 * ws[..., 1].abs().max().item()


@pytest.mark.parametrize("bf16", [False, True])
@pytest.mark.parametrize("M,N,K,epi,act", [(300, 768, 256, "store", "none"), (4099, 3072, 1024, "store", "none"),
                                           (1, 256, 256, "store", "none"), (257, 2048, 512, "glu", "none"),
                                           (1000, 4096, 1024, "store", "silu"), (700, 1024, 512, "glu", "none")])
def test_gemm_layernorm_fused(cuda, bf16, M, N, K, epi, act):
    """LayerNorm(x; gamma, beta) * W^T + b with the normalisation done while
    the A operand is staged and gamma / beta folded into W and b (as the
    encoder loads them), against torch fp32 (LayerNorm with population
    variance, eps 1e-5, then the GEMM with W). Statistics come from the
    residual GEMM's epilogue, as in the encoder. The bound covers the f16 /
    bf16 roundings of xhat and of W diag(gamma)."""
    import torch
    import pkc
    dt = torch.bfloat16 if bf16 else torch.float16
    g = torch.Generator(device="cpu").manual_seed(M + N + K)
    x0 = (torch.randn(M, K, generator=g) * 2.0 + 0.7).cuda()
    gamma = (1.0 + 0.3 * torch.randn(K, generator=g)).cuda()
    beta = (0.2 * torch.randn(K, generator=g)).cuda()
    Bw = (torch.randn(N, K, generator=g) * 0.05).to(dt).cuda()
    bias = (torch.randn(N, generator=g) * 0.1).cuda()
    # x = x0 + 0 * (0 * 0^T) through the residual GEMM, which writes x's statistics
    Az = torch.zeros(M, 128, dtype=dt, device=cuda)
    Bz = torch.zeros(K, 128, dtype=dt, device=cuda)
    x = x0.clone()
    stats = torch.empty(M, K // 128, 2, device=cuda)
    pkc.gemm_resid_stats(Az.data_ptr(), Bz.data_ptr(), M, K, 128, bf16=bf16, x=x.data_ptr(),
                         stats=stats.data_ptr())
    ncols = N // 2 if epi == "glu" else N
    out = torch.zeros(M, ncols, dtype=dt, device=cuda)
    Wf = (Bw.float() * gamma[None, :]).to(dt)
    bf_ = (bias.double() + Bw.double() @ beta.double()).float()
    pkc.gemm_ln(x.data_ptr(), stats.data_ptr(), Wf.data_ptr(), M, N, K,
                bf16=bf16, epi=pkc.EPI_GLU_H if epi == "glu" else pkc.EPI_STORE_H,
                act=pkc.ACT_SILU if act == "silu" else pkc.ACT_NONE, bias=bf_.data_ptr(), out=out.data_ptr(),
                ldo=ncols)
    torch.cuda.synchronize()
    y = torch.nn.functional.layer_norm(x0, (K,), gamma, beta, eps=1e-5)
    z = y @ Bw.float().t() + bias
    if epi == "glu":
        zt = z.view(M, N // 256, 2, 128)
        a, gg = zt[:, :, 0, :].reshape(M, N // 2), zt[:, :, 1, :].reshape(M, N // 2)
        want = a * torch.sigmoid(gg)
    elif act == "silu":
        want = torch.nn.functional.silu(z)
    else:
        want = z
    tol = 2e-2 if bf16 else 4e-3
    err = (out.float() - want).abs().max().item() / want.abs().max().item()
    assert err < tol, err


def test_gemm_layernorm_rejects_bad_shapes(cuda):
    import torch
    import pkc
    x = torch.zeros(64, 96, device=cuda)
    st = torch.zeros(64, 1, 2, device=cuda)
    Bw = torch.zeros(256, 96, dtype=torch.float16, device=cuda)
    out = torch.zeros(64, 256, dtype=torch.float16, device=cuda)
    with pytest.raises(pkc.PkcError):   # K = 96 is not a multiple of 128
        pkc.gemm_ln(x.data_ptr(), st.data_ptr(), Bw.data_ptr(), 64, 256, 96, bf16=False, out=out.data_ptr(),
                    ldo=256)


_SPLITK_CHILD = r"""
import sys, numpy as np, torch
sys.path.insert(0, sys.argv[1])
import pkc
M, N, K, epi = (int(v) for v in sys.argv[2:6])
g = torch.Generator().manual_seed(M * 7 + N + K)
A = (torch.randn(M, K, generator=g) * 0.5).half().cuda()
B = (torch.randn(N, K, generator=g) * 0.05).half().cuda()
bias = (torch.randn(N, generator=g) * 0.1).cuda()
ncols = N // 2 if epi == pkc.EPI_GLU_H else N
f32 = epi in (pkc.EPI_RESID_F32, pkc.EPI_STORE_F32)
out = (torch.randn(M, ncols, generator=g).cuda() if f32 else torch.zeros(M, ncols, dtype=torch.half, device="cuda"))
pkc.gemm(A.data_ptr(), B.data_ptr(), M, N, K, bf16=False, epi=epi, alpha=0.5 if f32 else 1.0,
         bias=bias.data_ptr(), out=out.data_ptr(), ldo=ncols)
torch.cuda.synchronize()
np.save(sys.argv[6], out.float().cpu().numpy())
"""


@pytest.mark.parametrize("M,N,K,epi", [(3282, 1024, 1024, "resid"), (3282, 3072, 1024, "store"),
                                       (3282, 2048, 1024, "glu"), (3282, 1024, 4096, "resid"),
                                       (600, 1024, 2048, "f32")])
def test_stream_k_matches_whole_tiles(cuda, tmp_path, M, N, K, epi):
    """With PKC_GEMM_SPLITK=1, shapes whose whole-tile schedule leaves part of
    the last wave idle run stream-K (tiles split along K across CTA pairs,
    partial sums added by the finishing pair in pair order). Against the
    whole-tile kernel (the default; a child process each) the results differ
    only by f32 summation order; the same call twice is bitwise identical."""
    import os
    import subprocess
    import sys
    import numpy as np
    import pkc
    e = {"resid": pkc.EPI_RESID_F32, "store": pkc.EPI_STORE_H, "glu": pkc.EPI_GLU_H, "f32": pkc.EPI_STORE_F32}[epi]
    pydir = os.path.dirname(pkc.__file__)
    outs = {}
    for tag, env in (("sk", {"PKC_GEMM_SPLITK": "1"}), ("sk2", {"PKC_GEMM_SPLITK": "1"}), ("whole", {})):
        f = str(tmp_path / f"{tag}.npy")
        base = {k: v for k, v in os.environ.items() if k != "PKC_GEMM_SPLITK"}
        subprocess.run([sys.executable, "-c", _SPLITK_CHILD, pydir, str(M), str(N), str(K), str(e), f],
                       check=True, env={**base, **env}, timeout=300)
        outs[tag] = np.load(f)
    np.testing.assert_array_equal(outs["sk"], outs["sk2"])
    scale = np.abs(outs["whole"]).max()
    tol = 1e-5 if epi in ("resid", "f32") else 1e-3   # f16 outputs: a last-bit flip at most
    assert np.abs(outs["sk"] - outs["whole"]).max() <= tol * scale


@pytest.mark.parametrize("bf16", [False, True])
@pytest.mark.parametrize("M", [1, 2, 5, 16])
@pytest.mark.parametrize("epi", ["store_silu", "resid", "f32", "glu"])
def test_skinny_epilogues(cuda, bf16, M, epi):
    """M <= 16: the skinny CUDA-core GEMM (one warp per weight row, f32
    accumulation) with every epilogue the streaming encoder uses, against
    the fp32 reference; K = 2048 exercises several 16-byte chunks per lane."""
    import torch
    import pkc
    N, K = 1024, 2048
    dt = torch.bfloat16 if bf16 else torch.float16
    A, B, bias, ref = _setup(M, N, K, dt, seed=20 + M)
    x = ref + bias
    tol = 1e-2 if bf16 else 3e-3
    if epi == "store_silu":
        out = torch.zeros(M, N, dtype=dt, device=cuda)
        pkc.gemm(A.data_ptr(), B.data_ptr(), M, N, K, bf16=bf16, epi=pkc.EPI_STORE_H, act=pkc.ACT_SILU,
                 bias=bias.data_ptr(), out=out.data_ptr(), ldo=N)
        want, got = torch.nn.functional.silu(x), out.float()
    elif epi == "resid":
        base = torch.randn(M, N, device=cuda)
        out = base.clone()
        pkc.gemm(A.data_ptr(), B.data_ptr(), M, N, K, bf16=bf16, epi=pkc.EPI_RESID_F32, alpha=0.5,
                 bias=bias.data_ptr(), out=out.data_ptr(), ldo=N)
        want, got, tol = base + 0.5 * x, out, 1e-4
    elif epi == "f32":
        out = torch.zeros(M, N, device=cuda)
        pkc.gemm(A.data_ptr(), B.data_ptr(), M, N, K, bf16=bf16, epi=pkc.EPI_STORE_F32, alpha=2.0,
                 bias=bias.data_ptr(), out=out.data_ptr(), ldo=N)
        want, got, tol = 2.0 * x, out, 1e-4
    else:
        xt = x.view(M, N // 256, 2, 128)
        a, g = xt[:, :, 0, :].reshape(M, N // 2), xt[:, :, 1, :].reshape(M, N // 2)
        out = torch.zeros(M, N // 2, dtype=dt, device=cuda)
        pkc.gemm(A.data_ptr(), B.data_ptr(), M, N, K, bf16=bf16, epi=pkc.EPI_GLU_H, bias=bias.data_ptr(),
                 out=out.data_ptr(), ldo=N // 2)
        want, got = a * torch.sigmoid(g), out.float()
    torch.cuda.synchronize()
    err = (got - want).abs().max().item() / want.abs().max().item()
    assert err < tol, err


@pytest.mark.parametrize("epi", ["store_h", "resid_f32", "store_f32"])
def test_narrow_tiles_match_wide_tiles_bitwise(cuda, epi):
    """A GEMM whose 256-wide pair tiles would fill at most half of the SM pairs
    runs 256 x 128 pair tiles; a row's sums run in the same order in both, so
    the rows of a small-M call equal the same rows of a large-M call (wide
    tiles) bit for bit -- a clip's encoder output does not depend on how
    many clips share its batch."""
    import torch
    import pkc
    N, K, Ms, Mb = 1024, 1024, 700, 20000
    A, B, bias, _ = _setup(Mb, N, K, torch.float16, seed=5)
    e = {"store_h": pkc.EPI_STORE_H, "resid_f32": pkc.EPI_RESID_F32, "store_f32": pkc.EPI_STORE_F32}[epi]
    dt = torch.float16 if epi == "store_h" else torch.float32
    g = torch.Generator(device="cpu").manual_seed(6)
    x0 = torch.randn(Mb, N, generator=g).to(dt).to(cuda)
    outs = []
    for M in (Ms, Mb):
        out = x0[:M].clone()
        pkc.gemm(A.data_ptr(), B.data_ptr(), M, N, K, bf16=False, epi=e, alpha=0.5, bias=bias.data_ptr(),
                 out=out.data_ptr(), ldo=N)
        torch.cuda.synchronize()
        outs.append(out)
    assert torch.equal(outs[0], outs[1][:Ms])
