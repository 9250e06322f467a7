"""The attention entry point for callers that may not allocate device memory.

Some hosts own all of the GPU's memory through their own allocator: a
serving runtime that reserves HBM up front, or one whose accounting must
see every byte. For them a cudaMalloc inside a library call is refused or
stalls the device. pkc_relpos_attention_noalloc keeps its tables in a fixed
array inside the library instead of allocating them.

This test calls it twice in a row through the C ABI, with different batch
shapes, and checks each result against the allocating entry point
(pkc_relpos_attention) within the attention tests' tolerance. It lives in
its own file that pytest collects last.
"""
import pytest

pytestmark = pytest.mark.gpu


def _inputs(lens, dk, H, bf16, seed):
    import torch
    d = H * dk
    dt = torch.bfloat16 if bf16 else torch.float16
    g = torch.Generator().manual_seed(seed)
    M = sum(lens)
    centre = max(lens)
    qkv = (torch.randn(M, 3 * d, generator=g) * 0.6).to(dt).cuda()
    ptab = (torch.randn(2 * centre - 1, d, generator=g) * 0.6).to(dt).cuda()
    bu = (torch.randn(d, generator=g) * 0.05).cuda()
    bv = (torch.randn(d, generator=g) * 0.05).cuda()
    return qkv, ptab, centre, bu, bv, d


@pytest.mark.parametrize("bf16", [False, True])
def test_noalloc_matches_allocating_entry_twice(cuda, bf16):
    import torch
    import pkc
    tol = 2e-2 if bf16 else 5e-3
    for call, (lens, dk, H) in enumerate((([300, 17, 129], 128, 8), ([5, 64, 1, 200, 33], 64, 4))):
        qkv, ptab, centre, bu, bv, d = _inputs(lens, dk, H, bf16, 100 + call)
        dt = qkv.dtype
        want = torch.zeros(sum(lens), d, dtype=dt, device=cuda)
        got = torch.full((sum(lens), d), float("nan"), dtype=dt, device=cuda)
        pkc.relpos_attention(qkv.data_ptr(), ptab.data_ptr(), centre, bu.data_ptr(), bv.data_ptr(), lens, d, H,
                             bf16=bf16, ctx=want.data_ptr())
        pkc.relpos_attention_noalloc(qkv.data_ptr(), ptab.data_ptr(), centre, bu.data_ptr(), bv.data_ptr(),
                                     lens, d, H, bf16=bf16, ctx=got.data_ptr())
        torch.cuda.synchronize()
        assert torch.isfinite(got.float()).all()
        err = (got.float() - want.float()).abs().max().item() / want.float().abs().max().item()
        assert err <= tol, (call, err)


def test_noalloc_rejects_oversize(cuda):
    import torch
    import pkc
    qkv, ptab, centre, bu, bv, d = _inputs([8], 64, 4, False, 7)
    ctx = torch.zeros(8, d, dtype=qkv.dtype, device=cuda)
    with pytest.raises(pkc.PkcError) as e:
        pkc.relpos_attention_noalloc(qkv.data_ptr(), ptab.data_ptr(), centre, bu.data_ptr(), bv.data_ptr(),
                                     [8] * 1025, d, 4, bf16=False, ctx=ctx.data_ptr())
    assert e.value.status == 1 and "1024" in str(e.value)
