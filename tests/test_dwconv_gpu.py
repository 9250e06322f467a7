"""Conv module depthwise stage (k_dwconv_bn_silu, through the kernel-level
C-ABI entry pkc_conv_depthwise) against a plain PyTorch fp32 restatement of
the reference's nodes (src/conformer.cpp: 63-79 time mask, 112-124 depthwise
conv, 134-154 batch norm folded to scale / shift, SiLU):
y = silu((conv1d_dw(x; w, pad (K-1)/2) + b) * scale + shift), zeros outside
each utterance.

Inputs are exact f16 / bf16 values and the kernel accumulates in f32, so the
only difference is the final rounding to the operand type plus the fast
exponential of the SiLU: 1 ulp of the output type (2e-3 relative for f16,
1.6e-2 for bf16) against the output magnitude."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def reference(x, lens, w, b, scale, shift):
    import torch
    K, d = w.shape
    pad = (K - 1) // 2
    out = torch.zeros(x.shape[0], d, dtype=torch.float32, device=x.device)
    off = 0
    for T in lens:
        if T == 0:
            continue
        xi = x[off:off + T].float().t().unsqueeze(0)                 # [1, d, T]
        wk = w.t().unsqueeze(1).contiguous()                        # [d, 1, K]; tap k reads frame t - pad + k
        y = torch.nn.functional.conv1d(xi, wk, bias=b, padding=pad, groups=d)[0].t()
        y = y * scale + shift
        out[off:off + T] = y * torch.sigmoid(y)
        off += T
    return out


CASES = [
    # (d, K, lens)
    (1024, 9, [437, 250, 64, 63, 1, 2, 129]),
    (256, 9, [0, 5, 0, 300, 65]),
    (176, 9, [100, 33]),          # d not a multiple of the kernel's channel block
    (512, 7, [77, 128, 1]),
    (256, 5, [64, 3]),
    (128, 3, [200, 1, 64]),
]


@pytest.mark.parametrize("bf16", [False, True])
@pytest.mark.parametrize("d,K,lens", CASES)
def test_conv_depthwise_matches_torch(cuda, bf16, d, K, lens):
    import torch
    import pkc
    dt = torch.bfloat16 if bf16 else torch.float16
    g = torch.Generator().manual_seed(d * 31 + K + sum(lens))
    M = sum(lens)
    x = torch.randn(M, d, generator=g).to(dt).to(cuda)
    w = (torch.randn(K, d, generator=g) * 0.3).to(cuda)
    b = (torch.randn(d, generator=g) * 0.1).to(cuda)
    scale = (1.0 + 0.2 * torch.randn(d, generator=g)).to(cuda)
    shift = (0.1 * torch.randn(d, generator=g)).to(cuda)
    out = torch.full((M, d), float("nan"), dtype=dt, device=cuda)
    pkc.conv_depthwise(x.data_ptr(), lens, d, K, w.data_ptr(), b.data_ptr(), scale.data_ptr(), shift.data_ptr(),
                       bf16=bf16, out=out.data_ptr())
    torch.cuda.synchronize()
    ref = reference(x, lens, w, b, scale, shift)
    got = out.float()
    assert torch.isfinite(got).all()
    err = (got - ref).abs().max().item() / ref.abs().max().item()
    assert err < (1.6e-2 if bf16 else 2e-3), err


def test_conv_depthwise_many_items_and_no_bias(cuda):
    """400 utterances of 0..89 frames (empty ones included) and no bias."""
    import torch
    import pkc
    g = torch.Generator().manual_seed(7)
    lens = [int(v) for v in torch.randint(0, 90, (400,), generator=g)]
    d, K = 256, 9
    M = sum(lens)
    x = torch.randn(M, d, generator=g).half().to(cuda)
    w = (torch.randn(K, d, generator=g) * 0.3).to(cuda)
    scale = (1.0 + 0.2 * torch.randn(d, generator=g)).to(cuda)
    shift = (0.1 * torch.randn(d, generator=g)).to(cuda)
    out = torch.full((M, d), float("nan"), dtype=torch.float16, device=cuda)
    pkc.conv_depthwise(x.data_ptr(), lens, d, K, w.data_ptr(), 0, scale.data_ptr(), shift.data_ptr(),
                       bf16=False, out=out.data_ptr())
    torch.cuda.synchronize()
    ref = reference(x, lens, w, None, scale, shift)
    got = out.float()
    assert torch.isfinite(got).all()
    err = (got - ref).abs().max().item() / ref.abs().max().item()
    assert err < 2e-3, err
