"""Host-side argument checks of the Python surface that run before any CUDA
call, on CPU tensors (no GPU needed): wrong shapes, dtypes and layouts raise
ValueError / TypeError the way the reference's callers would see them."""
import pytest
import torch

import fftsparse_b200 as F


def _qkv(L=2048, H=4, Hkv=2, dtype=torch.bfloat16):
    return (torch.zeros(1, H, L, 128, dtype=dtype), torch.zeros(1, Hkv, L, 128, dtype=dtype),
            torch.zeros(1, Hkv, L, 128, dtype=dtype))


def test_rope_pool_rejects_bad_arguments():
    L, D = 256, 128
    qp = torch.zeros(L, 4 * D, dtype=torch.bfloat16)
    kp = torch.zeros(L, 2 * D, dtype=torch.bfloat16)
    cs = torch.zeros(L, D, dtype=torch.bfloat16)
    with pytest.raises(ValueError):  # fp32 projection
        F.rope_pool(qp.float(), kp, None, 4, 2, cs, cs)
    with pytest.raises(ValueError):  # non-unit column stride
        F.rope_pool(qp.t().contiguous().t(), kp, None, 4, 2, cs, cs)
    with pytest.raises(ValueError):  # fewer columns than the heads need
        F.rope_pool(qp, kp, None, 5, 2, cs, cs)
    with pytest.raises(ValueError):  # row counts differ
        F.rope_pool(qp[:-1], kp, None, 4, 2, cs, cs)
    with pytest.raises(ValueError):  # cos and sin differ in shape
        F.rope_pool(qp, kp, None, 4, 2, cs, cs[:-1])


def test_block_mask_rejects_bad_arguments():
    q, k, _ = _qkv()
    with pytest.raises(ValueError):  # 3-D input
        F.fft_block_mask(q[0], k)
    with pytest.raises(TypeError):  # dtypes differ
        F.fft_block_mask(q, k.float())
    with pytest.raises(ValueError):  # H not a multiple of Hkv
        F.fft_block_mask(q[:, :3], k)
    N = 2048 // 128
    qb = torch.zeros(1, 4, N, 128, dtype=torch.bfloat16)
    kb = torch.zeros(1, 2, N, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError):  # pooled blocks of the wrong length
        F.fft_block_mask(q, k, pooled=(qb[:, :, :-1], kb))
    with pytest.raises(ValueError):  # pooled blocks in another dtype
        F.fft_block_mask(q, k, pooled=(qb.float(), kb.float()))


def test_prefill_keeps_reference_errors():
    q, k, v = _qkv()
    with pytest.raises(AssertionError):  # the reference's is_cuda assert (my_attn_v7.py:502)
        F.myattn_prefill(q, k, v, 0)
    with pytest.raises(ValueError):  # unknown selection mode (:210), raised while deriving parameters
        F.derive_mask_params(2048, correlation_selection_mode="bogus")


def test_sparse_attention_rejects_non_bf16():
    q, k, v = _qkv(dtype=torch.float32)
    bits = torch.zeros(1, 4, 16, 1, dtype=torch.int32)
    with pytest.raises(TypeError):
        F.sparse_attention(q, k, v, bits, 128)


def test_decode_rejects_bad_arguments():
    q = torch.zeros(1, 8, 128, dtype=torch.bfloat16)
    kc = torch.zeros(1, 2, 64, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError):  # more than one new token
        F.decode_attention(torch.zeros(1, 8, 2, 128, dtype=torch.bfloat16), kc, kc)
    with pytest.raises(TypeError):  # fp32 cache
        F.decode_attention(q, kc.float(), kc.float())
    with pytest.raises(ValueError):  # caches of different shapes
        F.decode_attention(q, kc, kc[:, :, :32])
    with pytest.raises(ValueError):  # batch mismatch
        F.decode_attention(torch.zeros(2, 8, 128, dtype=torch.bfloat16), kc, kc)
