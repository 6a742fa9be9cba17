"""GPU parity of ffts_decode_attn (decode attention over the un-expanded KV
cache) against a plain PyTorch fp32 evaluation of the caller's decode branch
(eval/LongBench/pred.py:306-322: softmax(q k^T / sqrt(D)) v over the
repeat_kv-expanded cache).  Tolerance (bf16 output): max |err| <= 2e-2 and
mean |err| <= 1e-3.  The file sorts after the kernel tests, so under -x they
run first."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def reference(q, k, v):
    """fp32, per GQA group (the same as attending the repeat_kv-expanded cache)."""
    B, H, D = q.shape
    Hkv = k.shape[1]
    qg = q.float().view(B, Hkv, H // Hkv, D)
    s = torch.einsum("bkgd,bkld->bkgl", qg, k.float()) / D ** 0.5
    return torch.einsum("bkgl,bkld->bkgd", s.softmax(-1), v.float()).reshape(B, H, D)


@pytest.mark.parametrize("B,H,Hkv,Lk,splits", [(1, 32, 8, 131072, None), (2, 28, 4, 65536 + 5, 37),
                                               (1, 4, 4, 77, 3), (1, 8, 1, 1000, 1), (1, 16, 1, 300, None)])
def test_decode_matches_fp32(B, H, Hkv, Lk, splits):
    import fftsparse_b200 as F
    F.load_library()
    g = torch.Generator().manual_seed(Lk + H)
    q = (torch.randn(B, H, 128, generator=g) * 2).bfloat16().cuda()
    k = torch.randn(B, Hkv, Lk, 128, generator=g).bfloat16().cuda()
    v = torch.randn(B, Hkv, Lk, 128, generator=g).bfloat16().cuda()
    got = F.decode_attention(q, k, v, splits=splits)
    ref = reference(q, k, v)
    err = (got.float() - ref).abs()
    assert float(err.max()) <= 2e-2 and float(err.mean()) <= 1e-3, (float(err.max()), float(err.mean()))


def test_decode_over_a_cache_slice_and_q_len_one():
    # a preallocated cache of capacity 4096 holding 2500 tokens; q as [B, H, 1, D]
    import fftsparse_b200 as F
    g = torch.Generator().manual_seed(7)
    cap, Lk = 4096, 2500
    kc = torch.randn(1, 2, cap, 128, generator=g).bfloat16().cuda()
    vc = torch.randn(1, 2, cap, 128, generator=g).bfloat16().cuda()
    q = torch.randn(1, 8, 1, 128, generator=g).bfloat16().cuda()
    got = F.decode_attention(q, kc[:, :, :Lk], vc[:, :, :Lk])
    ref = reference(q[:, :, 0], kc[:, :, :Lk], vc[:, :, :Lk])
    assert float((got.float() - ref).abs().max()) <= 2e-2


@pytest.mark.parametrize("mask_dtype", [torch.bfloat16, torch.float32])
def test_decode_with_padding_mask(mask_dtype):
    """A left-padded batch of two: HF's 4-D additive mask [B, 1, 1, kv_len] (0 for
    real keys, the dtype's minimum for padding, one spare column past Lk) is added
    to the scaled scores before the softmax, as the caller's decode branch adds
    attention_mask (eval/LongBench/pred.py:311-313)."""
    import fftsparse_b200 as F
    g = torch.Generator().manual_seed(11)
    B, H, Hkv, Lk = 2, 8, 2, 3000
    q = (torch.randn(B, H, 128, generator=g) * 2).bfloat16().cuda()
    k = torch.randn(B, Hkv, Lk, 128, generator=g).bfloat16().cuda()
    v = torch.randn(B, Hkv, Lk, 128, generator=g).bfloat16().cuda()
    pad = [0, 700]  # sequence 1 has 700 padding tokens on the left
    mask = torch.zeros(B, 1, 1, Lk + 1, dtype=mask_dtype)
    for b, p in enumerate(pad):
        mask[b, 0, 0, :p] = torch.finfo(mask_dtype).min
    mask = mask.cuda()
    got = F.decode_attention(q, k, v, attention_mask=mask)
    D = q.shape[2]
    qg = q.float().view(B, Hkv, H // Hkv, D)
    s = torch.einsum("bkgd,bkld->bkgl", qg, k.float()) / D ** 0.5 + mask[:, :, :, :Lk].float()
    ref = torch.einsum("bkgl,bkld->bkgd", s.softmax(-1), v.float()).reshape(B, H, D)
    err = (got.float() - ref).abs()
    assert float(err.max()) <= 2e-2 and float(err.mean()) <= 1e-3, (float(err.max()), float(err.mean()))
    # the padded keys really are excluded: the same as attending the unpadded keys only
    alone = F.decode_attention(q[1:], k[1:, :, pad[1]:].contiguous(), v[1:, :, pad[1]:].contiguous())
    assert float((got[1:].float() - alone.float()).abs().max()) <= 2e-2
