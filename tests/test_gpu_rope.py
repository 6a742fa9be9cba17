"""GPU parity of ffts_rope_pool: the rotated head-major q/k, the head-major v
and the pooled blocks equal the CPU oracle (C ffo_rope + canonical pooling) and
torch's own bf16 RoPE expression followed by ffts_pool, bit for bit; the mask
selected from the pooled blocks equals the mask selected from q and k."""
import pytest
import torch

from oracle import oracle as O
from tests.test_rope_oracle import rope_tables

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def F():
    import fftsparse_b200
    fftsparse_b200.load_library()
    return fftsparse_b200


@pytest.mark.parametrize("L,Hq,Hkv,bs,with_v", [(1000, 4, 2, 128, True), (4096, 8, 2, 64, True),
                                                 (333, 2, 1, 32, False), (131, 3, 3, 128, True)])
def test_rope_pool_matches_oracle_and_torch(F, L, Hq, Hkv, bs, with_v):
    D = 128
    g = torch.Generator().manual_seed(L * 7 + Hq)
    qkv = (torch.randn(L, (Hq + 2 * Hkv) * D + 64, generator=g) * 2).bfloat16()  # one fused product, strided
    cos, sin = rope_tables(L)
    srcs = (qkv[:, :Hq * D], qkv[:, Hq * D:(Hq + Hkv) * D], qkv[:, (Hq + Hkv) * D:(Hq + 2 * Hkv) * D])
    ref = O.rope_pool(srcs[0], srcs[1], srcs[2] if with_v else None, Hq, Hkv, cos, sin, bs)
    qkv_d, cos_d, sin_d = qkv.cuda(), cos.cuda(), sin.cuda()
    src_d = (qkv_d[:, :Hq * D], qkv_d[:, Hq * D:(Hq + Hkv) * D], qkv_d[:, (Hq + Hkv) * D:(Hq + 2 * Hkv) * D])
    got = F.rope_pool(src_d[0], src_d[1], src_d[2] if with_v else None, Hq, Hkv, cos_d, sin_d, bs)
    torch.cuda.synchronize()
    for name, r, x in zip(("q", "k", "v", "q_pooled", "k_pooled"), ref, got):
        if r is None:
            assert x is None
            continue
        assert torch.equal(x.cpu(), r), name
    # torch's bf16 expression on the GPU, then the pooling kernel
    for h, src, x, xb in ((Hq, src_d[0], got[0], got[3]), (Hkv, src_d[1], got[1], got[4])):
        xv = src.reshape(L, h, D).transpose(0, 1)[None]
        x1, x2 = xv[..., :D // 2], xv[..., D // 2:]
        t = xv * cos_d + torch.cat([-x2, x1], -1) * sin_d
        assert torch.equal(x, t)
        assert torch.equal(xb, F.pool_blocks(t, bs))


def test_mask_from_pooled_blocks_equals_mask_from_q_k(F):
    import bench
    D, L, Hq, Hkv = 128, 8192, 4, 2
    g = torch.Generator().manual_seed(3)
    qkv = torch.randn(L, (Hq + 2 * Hkv) * D, generator=g).bfloat16().cuda()
    cos, sin = (t.cuda() for t in rope_tables(L))
    q, k, v, qb, kb = F.rope_pool(qkv[:, :Hq * D], qkv[:, Hq * D:(Hq + Hkv) * D], qkv[:, (Hq + Hkv) * D:],
                                  Hq, Hkv, cos, sin)
    kw = bench.mask_kwargs(0.1)
    a = F.fft_block_mask(q, k, **kw)
    b = F.fft_block_mask(q, k, pooled=(qb, kb), **kw)
    assert torch.equal(a.bits, b.bits) and torch.equal(a.corr, b.corr)
    o1 = F.myattn_prefill(q, k, v, 0, **kw)
    o2 = F.myattn_prefill(q, k, v, 0, pooled=(qb, kb), **kw)
    assert torch.equal(o1, o2)
    with pytest.raises(ValueError):
        F.fft_block_mask(q, k, pooled=(qb[:, :, :-1], kb), **kw)


def test_rope_pool_rejects_bad_shapes(F):
    x = torch.zeros(64, 4 * 64, dtype=torch.bfloat16, device="cuda")
    cs = torch.zeros(64, 64, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):  # head_dim 64
        F.rope_pool(x, x, None, 2, 2, cs, cs)
