"""The oracle's restatement of the caller's rotary embedding (ffo_rope) against
HF transformers' own apply_rotary_pos_emb, the function the reference's
callers apply to q and k before myattn_prefill (eval/LongBench/pred.py:191-194),
bit for bit on the CPU; and oracle.rope_pool's pooled blocks against the
canonical pooling of the rotated tensors."""
import pytest
import torch

from oracle import oracle as O


def rope_tables(L, D=128, base=500000.0, dtype=torch.bfloat16):
    inv = 1.0 / (base ** (torch.arange(0, D, 2, dtype=torch.float32) / D))
    fr = torch.arange(L, dtype=torch.float32)[:, None] * inv[None]
    emb = torch.cat([fr, fr], -1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


@pytest.mark.parametrize("L,Hq,Hkv,scale", [(300, 4, 2, 1.0), (1000, 3, 1, 8.0), (129, 2, 2, 0.05)])
def test_rope_equals_hf_apply_rotary_pos_emb(L, Hq, Hkv, scale):
    hf = pytest.importorskip("transformers.models.llama.modeling_llama")
    D = 128
    g = torch.Generator().manual_seed(L + Hq)
    qkv = (torch.randn(L, (Hq + 2 * Hkv) * D + 32, generator=g) * scale).bfloat16()  # strided rows
    cos, sin = rope_tables(L)
    q_src, k_src = qkv[:, :Hq * D], qkv[:, Hq * D:(Hq + Hkv) * D]
    q_ref = q_src.reshape(L, Hq, D).transpose(0, 1)[None]
    k_ref = k_src.reshape(L, Hkv, D).transpose(0, 1)[None]
    qe, ke = hf.apply_rotary_pos_emb(q_ref, k_ref, cos[None], sin[None])
    assert torch.equal(O.rope(q_src, Hq, cos, sin), qe)
    assert torch.equal(O.rope(k_src, Hkv, cos, sin), ke)


@pytest.mark.parametrize("bs", [128, 64, 32])
def test_rope_pool_pools_the_rotated_tensors(bs):
    D, L, Hq, Hkv = 128, 1000, 2, 1
    g = torch.Generator().manual_seed(5)
    qkv = torch.randn(L, (Hq + 2 * Hkv) * D, generator=g).bfloat16()
    cos, sin = rope_tables(L)
    q, k, v, qb, kb = O.rope_pool(qkv[:, :Hq * D], qkv[:, Hq * D:(Hq + Hkv) * D], qkv[:, (Hq + Hkv) * D:],
                                  Hq, Hkv, cos, sin, bs)
    assert q.shape == (1, Hq, L, D) and k.shape == v.shape == (1, Hkv, L, D)
    assert torch.equal(v[0], qkv[:, (Hq + Hkv) * D:].reshape(L, Hkv, D).transpose(0, 1))
    assert torch.equal(qb, O.pool(q, bs)) and torch.equal(kb, O.pool(k, bs))
    assert qb.shape == (1, Hq, (L + bs - 1) // bs, D)
