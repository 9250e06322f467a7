"""The attention entry point for callers that may not allocate device memory.

Some hosts own all of the GPU's memory through their own allocator: a
serving runtime that reserves HBM up front, or one whose accounting must
see every byte. For them a cudaMalloc inside a library call is refused or
stalls the device. pkc_relpos_attention_noalloc keeps its tables in a fixed
array inside the library instead of allocating them.

These tests call it through the C ABI: twice in a row with different batch
shapes (the second call must not see the first call's tables), on a
non-default stream, and at its size limit. Each result is compared bit for
bit with the allocating entry point (pkc_relpos_attention, the same kernel
on the same tables) and against the plain PyTorch fp32 attention of
tests/test_attention_gpu.py within that test's bounds (5e-3 f16, 2e-2
bf16). The file is collected last.
"""
import pytest

from test_attention_gpu import reference

pytestmark = pytest.mark.gpu

# the entry point's fixed table: 20480 ints = offsets (B+1) + lengths (B) +
# 2 per 128-frame query tile + the error word
TABLE_INTS = 20480
QUERY_TILE = 128


def _inputs(lens, dk, H, bf16, seed, device):
    import torch
    d = H * dk
    dt = torch.bfloat16 if bf16 else torch.float16
    g = torch.Generator(device=device).manual_seed(seed)
    M = sum(lens)
    centre = max(lens)
    qkv = (torch.randn(M, 3 * d, generator=g, device=device) * 0.6).to(dt)
    ptab = (torch.randn(2 * centre - 1, d, generator=g, device=device) * 0.6).to(dt)
    bu = torch.randn(d, generator=g, device=device) * 0.05
    bv = torch.randn(d, generator=g, device=device) * 0.05
    return qkv, ptab, centre, bu, bv, d


def _both(lens, dk, H, bf16, seed, device, stream=0):
    import torch
    import pkc
    qkv, ptab, centre, bu, bv, d = _inputs(lens, dk, H, bf16, seed, device)
    want = torch.zeros(sum(lens), d, dtype=qkv.dtype, device=device)
    got = torch.full((sum(lens), d), float("nan"), dtype=qkv.dtype, device=device)
    pkc.relpos_attention(qkv.data_ptr(), ptab.data_ptr(), centre, bu.data_ptr(), bv.data_ptr(), lens, d, H,
                         bf16=bf16, ctx=want.data_ptr())
    torch.cuda.synchronize()
    pkc.relpos_attention_noalloc(qkv.data_ptr(), ptab.data_ptr(), centre, bu.data_ptr(), bv.data_ptr(),
                                 lens, d, H, bf16=bf16, ctx=got.data_ptr(), stream=stream)
    torch.cuda.synchronize()
    return (qkv, ptab, centre, bu, bv), got, want


@pytest.mark.parametrize("bf16", [False, True])
def test_noalloc_matches_allocating_entry_twice(cuda, bf16):
    tol = 2e-2 if bf16 else 5e-3
    for call, (lens, dk, H) in enumerate((([300, 17, 129], 128, 8), ([5, 64, 1, 200, 33], 64, 4))):
        (qkv, ptab, centre, bu, bv), got, want = _both(lens, dk, H, bf16, 100 + call, cuda)
        assert bool((got == want).all()), f"call {call}: differs from pkc_relpos_attention"
        ref = reference(qkv, ptab, centre, bu, bv, lens, H)
        err = (got.float() - ref).abs().max().item() / ref.abs().max().item()
        assert err <= tol, (call, err)


def test_noalloc_on_a_side_stream(cuda):
    import torch
    s = torch.cuda.Stream(cuda)
    _, got, want = _both([90, 260, 3], 128, 8, False, 5, cuda, stream=s.cuda_stream)
    assert bool((got == want).all())


def test_noalloc_at_the_tile_limit_and_one_past(cuda):
    """B = 1024 utterances: (20480 - 2 - 2B) / 2 = 9215 query tiles fit. 1023
    utterances of 9 tiles and one of 8 run and match the allocating entry;
    one tile more is refused before anything is launched (the buffers are
    real and large enough either way)."""
    import pkc
    import torch
    B = 1024
    cap = (TABLE_INTS - 2 - 2 * B) // 2
    lens = [9 * QUERY_TILE] * (B - 1) + [8 * QUERY_TILE]
    assert sum((n + QUERY_TILE - 1) // QUERY_TILE for n in lens) == cap
    (qkv, ptab, centre, bu, bv), got, want = _both(lens, 64, 4, False, 9, cuda)
    assert bool((got == want).all())
    lens[-1] = 9 * QUERY_TILE
    d = 256
    ctx = torch.zeros(sum(lens), d, dtype=qkv.dtype, device=cuda)
    qkv2 = torch.zeros(sum(lens), 3 * d, dtype=qkv.dtype, device=cuda)
    with pytest.raises(pkc.PkcError) as e:
        pkc.relpos_attention_noalloc(qkv2.data_ptr(), ptab.data_ptr(), centre, bu.data_ptr(), bv.data_ptr(),
                                     lens, d, 4, bf16=False, ctx=ctx.data_ptr())
    assert e.value.status == 1 and "query tiles" in str(e.value), str(e.value)


def test_noalloc_rejects_oversize(cuda):
    import torch
    import pkc
    qkv, ptab, centre, bu, bv, d = _inputs([8], 64, 4, False, 7, cuda)
    ctx = torch.zeros(8, d, dtype=qkv.dtype, device=cuda)
    with pytest.raises(pkc.PkcError) as e:
        pkc.relpos_attention_noalloc(qkv.data_ptr(), ptab.data_ptr(), centre, bu.data_ptr(), bv.data_ptr(),
                                     [8] * 1025, d, 4, bf16=False, ctx=ctx.data_ptr())
    assert e.value.status == 1 and "1024" in str(e.value)
