"""Seeded synthetic prefill inputs for the FFTSparse hot path.

Shared by the CPU oracle, the parity tests and bench.py so that every consumer
sees identical q/k/v.  It is a workload generator, not part of the operator.

The reference measures on Q/K captured from Llama-3.1-8B
(eval/efficiency/capture_qk_real.py:69-114, layout [1, 32, L, 128] post-RoPE,
k already repeat_kv'd).  Those captures and the model weights are not available,
so this generator stands in for them with the same layout and GQA shape (32 q
heads over 8 kv heads) and injected structure so that every mask family fires:

  * attention sinks: +3 sigma on the first 4 key tokens,
  * vertical stripes: a +2 sigma shared key direction on every 512th token,
  * slash diagonals: q/k phase-aligned (through RoPE) at offsets 64 and 1024,

followed by HF-convention RoPE (rotate_half, theta_i = base^(-2i/D)).

Draw order (frozen; changing it changes every fixture):
  q~[1,Hq,L,D], k~[1,Hkv,L,D], v[1,Hkv,L,D]  ~ N(0,1) fp32
  s_sink, s_stripe, p_64, p_1024             each [Hkv, D], unit RMS
"""
from __future__ import annotations

import math

import torch

__all__ = ["make_inputs", "rope_cos_sin", "apply_rope", "expand_kv"]


def rope_cos_sin(positions: torch.Tensor, dim: int, base: float):
    """HF Llama rotary tables: cos/sin of shape [len(positions), dim] (fp32)."""
    inv_freq = 1.0 / (base ** (torch.arange(0, dim, 2, dtype=torch.float64) / dim))
    freqs = positions.to(torch.float64)[:, None] * inv_freq[None, :]
    emb = torch.cat([freqs, freqs], dim=-1)
    return emb.cos().to(torch.float32), emb.sin().to(torch.float32)


def _rotate_half(x: torch.Tensor) -> torch.Tensor:
    h = x.shape[-1] // 2
    return torch.cat([-x[..., h:], x[..., :h]], dim=-1)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x [..., L, D] rotated with per-position cos/sin [L, D] (HF rotate_half form)."""
    return x * cos + _rotate_half(x) * sin


def _unit_rms(g: torch.Generator, hkv: int, d: int) -> torch.Tensor:
    v = torch.randn(hkv, d, generator=g, dtype=torch.float32)
    return v / v.pow(2).mean(dim=-1, keepdim=True).sqrt()


def expand_kv(x: torch.Tensor, n_rep: int) -> torch.Tensor:
    """HF repeat_kv order: kv head g serves q heads g*n_rep .. g*n_rep+n_rep-1."""
    if n_rep == 1:
        return x
    b, hkv, l, d = x.shape
    return x[:, :, None].expand(b, hkv, n_rep, l, d).reshape(b, hkv * n_rep, l, d)


def make_inputs(seq_len: int, *, num_q_heads: int = 32, num_kv_heads: int = 8,
                head_dim: int = 128, dtype: torch.dtype = torch.bfloat16,
                seed: int = 0, rope_base: float = 500000.0, batch: int = 1,
                expand: bool = True, sink_tokens: int = 4, stripe_period: int = 512,
                slash_offsets=(64, 1024), device: str = "cpu"):
    """Return (q, k, v) as [batch, H, L, D] tensors on ``device``.

    With ``expand`` (the drop-in layout the reference's callers pass), k and v
    carry ``num_q_heads`` heads (repeat_kv'd); otherwise ``num_kv_heads``.
    Each batch element b uses seed ``seed + b``.  The random draws always come
    from a CPU generator (so every device sees the same values); only the RoPE
    arithmetic and the final cast run on ``device``.
    """
    L, Hq, Hkv, D = seq_len, num_q_heads, num_kv_heads, head_dim
    assert Hq % Hkv == 0
    rep = Hq // Hkv
    qs, ks, vs = [], [], []
    pos = torch.arange(L)
    cos, sin = rope_cos_sin(pos, D, rope_base)
    for b in range(batch):
        g = torch.Generator("cpu").manual_seed(seed + b)
        q = torch.randn(1, Hq, L, D, generator=g, dtype=torch.float32)
        k = torch.randn(1, Hkv, L, D, generator=g, dtype=torch.float32)
        v = torch.randn(1, Hkv, L, D, generator=g, dtype=torch.float32)
        s_sink = _unit_rms(g, Hkv, D)
        s_stripe = _unit_rms(g, Hkv, D)
        p = {off: _unit_rms(g, Hkv, D) for off in slash_offsets}

        k[0, :, :min(sink_tokens, L)] += 3.0 * s_sink[:, None, :]
        if L >= stripe_period:
            k[0, :, stripe_period - 1::stripe_period] += 2.0 * s_stripe[:, None, :]
        q_bias = 0.25 * (s_sink + s_stripe)
        for off in slash_offsets:
            q_bias = q_bias + 0.5 * p[off]
            c1, s1 = rope_cos_sin(torch.tensor([off]), D, rope_base)
            k[0] += (0.5 * apply_rope(p[off], c1, s1))[:, None, :]
        q[0] += q_bias.repeat_interleave(rep, dim=0)[:, None, :]

        if device != "cpu":
            q, k, v = q.to(device), k.to(device), v.to(device)
            cos, sin = cos.to(device), sin.to(device)
        q = apply_rope(q, cos, sin)
        k = apply_rope(k, cos, sin)
        qs.append(q)
        ks.append(k)
        vs.append(v)
        if device != "cpu":
            cos, sin = cos.cpu(), sin.cpu()
    q = torch.cat(qs).to(dtype)
    k = torch.cat(ks).to(dtype)
    v = torch.cat(vs).to(dtype)
    if expand:
        k = expand_kv(k, rep).contiguous()
        v = expand_kv(v, rep).contiguous()
    return q.contiguous(), k, v


if __name__ == "__main__":  # pragma: no cover - manual inspection helper
    q, k, v = make_inputs(4096, dtype=torch.float32)
    print(q.shape, k.shape, v.shape, float(q.std()), float(k.std()), math.isfinite(float(v.sum())))
