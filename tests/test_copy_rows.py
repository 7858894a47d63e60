"""The library's strided row copy (V slots of fused QKV tensors and gradients).

GPU: bit-equal to torch's copy for the layouts the ops use (a V slot of
[T, 3, H, D] / [B, N, 3, H, D] to and from separate tensors), rows of 64 B to
6 KB, ragged row counts, and layouts it hands back to torch (misaligned base,
rows that are not 16-byte multiples). CPU: the argument checks of the C ABI.
"""
import ctypes

import pytest
import torch

from flash_attn_prologue_b200 import _lib


def test_c_abi_argument_checks():
    lib = _lib.load()
    s3 = (ctypes.c_int64 * 3)(0, 0, 128)
    dims = (ctypes.c_int64 * 3)(1, 1, 4)
    p = ctypes.c_void_p(16)
    assert lib.flash_prologue_copy_rows(p, s3, p, s3, dims, 24, None) == _lib.ERR_ALIGNMENT
    assert lib.flash_prologue_copy_rows(p, s3, p, s3, None, 128, None) == _lib.ERR_INVALID_ARGUMENT
    assert lib.flash_prologue_copy_rows(p, s3, p, s3, (ctypes.c_int64 * 3)(1, 0, 4), 128, None) == _lib.OK
    # overlapping source and destination byte ranges are rejected before any launch:
    # 4 rows of 128 B at stride 128 from 4096 (bytes 4096..4607) against the same
    # layout from 4352 or from 3712
    base, s_row = ctypes.c_void_p(4096), (ctypes.c_int64 * 3)(0, 0, 128)
    for dst in (4096 + 256, 4096 - 384):
        assert lib.flash_prologue_copy_rows(base, s_row, ctypes.c_void_p(dst), s_row, dims, 128,
                                            None) == _lib.ERR_INVALID_ARGUMENT
    # a reversed stride reaches below the base: rows at 5120, 4992, 4864, 4736 (bytes 4736..5247)
    neg = (ctypes.c_int64 * 3)(0, 0, -128)
    assert lib.flash_prologue_copy_rows(ctypes.c_void_p(5120), neg, ctypes.c_void_p(4096 + 512), s_row, dims,
                                        128, None) == _lib.ERR_INVALID_ARGUMENT
    with pytest.raises(ValueError, match="CUDA"):
        _lib.copy_rows(torch.empty(4, 8), torch.empty(4, 8))


@pytest.mark.gpu
@pytest.mark.parametrize("T,H,D", [(1, 1, 32), (333, 16, 64), (4096, 4, 128), (77, 12, 256)])
def test_v_slot_round_trip(T, H, D):
    g = torch.Generator(device="cuda").manual_seed(T)
    qkv = torch.randn(T, 3, H, D, generator=g, device="cuda").to(torch.bfloat16)
    v = torch.empty(T, H, D, dtype=qkv.dtype, device="cuda")
    _lib.copy_rows(v, qkv[:, 2])
    assert torch.equal(v, qkv[:, 2])
    back = torch.zeros_like(qkv)
    _lib.copy_rows(back[:, 2], v)
    assert torch.equal(back[:, 2], v) and float(back[:, :2].abs().sum()) == 0.0


@pytest.mark.gpu
@pytest.mark.parametrize("B,N,H,D", [(2, 50, 8, 64), (3, 7, 1, 32), (1, 129, 16, 128)])
def test_batched_slot_to_bhnd(B, N, H, D):
    g = torch.Generator(device="cuda").manual_seed(N)
    qkv = torch.randn(B, N, 3, H, D, generator=g, device="cuda").to(torch.bfloat16)
    src = qkv[:, :, 2].permute(0, 2, 1, 3)          # [B, H, N, D] view, rows of D
    dst = torch.empty(B, H, N, D, dtype=qkv.dtype, device="cuda")
    _lib.copy_rows(dst, src)
    assert torch.equal(dst, src)
    grad = torch.zeros(B, N, 3, H, D, dtype=qkv.dtype, device="cuda")
    gv = torch.randn(B, N, H, D, generator=g, device="cuda").to(torch.bfloat16)
    _lib.copy_rows(grad[:, :, 2], gv)
    assert torch.equal(grad[:, :, 2], gv)


@pytest.mark.gpu
def test_layouts_handed_to_torch():
    base = torch.randn(1000, device="cuda").to(torch.bfloat16)
    src = base[1:1 + 6 * 40].view(6, 40)            # misaligned base pointer
    dst = torch.empty(6, 40, dtype=torch.bfloat16, device="cuda")
    _lib.copy_rows(dst, src)
    assert torch.equal(dst, src)
    odd = torch.randn(5, 7, 3, device="cuda")       # 12-byte rows
    out = torch.empty_like(odd)
    _lib.copy_rows(out, odd)
    assert torch.equal(out, odd)


@pytest.mark.gpu
def test_random_layouts_match_torch_copy():
    """Slices and permutations with the last dimension contiguous, merged or not."""
    g = torch.Generator().manual_seed(0)
    for trial in range(40):
        shape = [int(torch.randint(1, 9, (1,), generator=g)) for _ in range(3)] + \
                [int(torch.tensor([8, 16, 24, 32, 64])[torch.randint(0, 5, (1,), generator=g)])]
        slot = int(torch.randint(0, 3, (1,), generator=g))
        base = torch.randn(shape[0], shape[1], 3, shape[2], shape[3]).to(torch.bfloat16).cuda()
        src = base[:, :, slot]                           # a slot of a fused buffer
        perm = [0, 1, 2]
        if trial % 2:
            perm = [1, 0, 2] if trial % 4 == 1 else [2, 0, 1]
        src = src.permute(*perm, 3)
        dst = torch.empty(src.shape, dtype=src.dtype, device="cuda")
        if trial % 3 == 0:                                # a strided destination as well
            big = torch.zeros(*src.shape[:-1], 2 * src.shape[-1], dtype=src.dtype, device="cuda")
            dst = big[..., : src.shape[-1]]
        _lib.copy_rows(dst, src)
        assert torch.equal(dst, src), (trial, shape, perm)
