"""Python face of the CPU oracle.

TEST INFRASTRUCTURE: the checker for the parity tests, smoke() and bench.py's
cpu_baseline leg.  The product path (fftsparse_b200) never imports this.

* ``pool`` / ``block_mask`` call the C restatement in ffts_oracle.c (canonical
  arithmetic, bit-exact target for the CUDA kernels).
* ``sparse_attention`` is an fp32 torch-CPU restatement of the forward of
  block_sparse_attn_func as myattn_prefill calls it (my_attn_v7.py:775-786):
  causal, scale 1/sqrt(D), head h uses mask plane h (head_mask_type all 1,
  :772), rows with nothing selected give zeros.
* ``prefill_mask`` chains pooling and selection for [B, H, L, D] inputs.
* ``rope`` / ``rope_pool`` restate the caller's rotary embedding (C ffo_rope)
  and the fused RoPE + layout + pooling pass (ffts_rope_pool).
"""
from __future__ import annotations

import ctypes
import os
import sys

import numpy as np
import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
_REPO = os.path.dirname(_HERE)
if _REPO not in sys.path:
    sys.path.insert(0, _REPO)

from oracle import build as _build  # noqa: E402

_lib = None


def lib():
    global _lib
    if _lib is None:
        path = _build.build()
        L = ctypes.CDLL(path)
        L.ffo_pool.restype = ctypes.c_int
        L.ffo_pool.argtypes = [ctypes.c_void_p, ctypes.c_int] + [ctypes.c_int64] * 7 + [
            ctypes.c_int, ctypes.c_void_p]
        L.ffo_rope.restype = ctypes.c_int
        L.ffo_rope.argtypes = [ctypes.c_void_p] + [ctypes.c_int64] * 4 + [ctypes.c_void_p] * 2 + [
            ctypes.c_int64, ctypes.c_void_p]
        L.ffo_block_mask.restype = ctypes.c_int
        L.ffo_block_mask.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int,
                                     ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                     ctypes.c_int64, ctypes.c_void_p] + [ctypes.c_void_p] * 6
        _lib = L
    return _lib


def _dtype_code(dt: torch.dtype) -> int:
    if dt == torch.float32:
        return 0
    if dt == torch.bfloat16:
        return 1
    raise TypeError(f"oracle supports fp32/bf16, got {dt}")


def pool(x: torch.Tensor, block_size: int) -> torch.Tensor:
    """Canonical block mean of x [B, H, L, D] (CPU) -> [B, H, N, D] in x.dtype."""
    assert x.device.type == "cpu" and x.dim() == 4 and x.stride(-1) == 1
    B, H, L, D = x.shape
    N = (L + block_size - 1) // block_size
    out = torch.empty(B, H, N, D, dtype=x.dtype)
    rc = lib().ffo_pool(x.data_ptr(), _dtype_code(x.dtype), B, H, L, D, x.stride(0),
                        x.stride(1), x.stride(2), block_size, out.data_ptr())
    if rc != 0:
        raise ValueError(f"ffo_pool rejected shape (rc={rc})")
    return out


def rope(x: torch.Tensor, num_heads: int, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """The caller's rotary embedding (C restatement ffo_rope) of token-major bf16
    projections x [L, >= num_heads * D] (row stride x.stride(0)) with bf16 cos/sin
    [L, D] -> head-major [1, num_heads, L, D] bf16."""
    assert x.device.type == "cpu" and x.dtype == torch.bfloat16 and x.dim() == 2 and x.stride(1) == 1
    assert cos.dtype == sin.dtype == torch.bfloat16 and cos.stride() == sin.stride() and cos.stride(1) == 1
    L, D = cos.shape
    out = torch.empty(1, num_heads, L, D, dtype=torch.bfloat16)
    rc = lib().ffo_rope(x.data_ptr(), x.stride(0), L, num_heads, D, cos.data_ptr(), sin.data_ptr(),
                        cos.stride(0), out.data_ptr())
    if rc != 0:
        raise ValueError(f"ffo_rope rejected shape (rc={rc})")
    return out


def rope_pool(q_src, k_src, v_src, num_heads, num_kv_heads, cos, sin, block_size):
    """Checker of ffts_rope_pool: RoPE'd head-major q and k, head-major v, and the
    canonical block means of the RoPE'd q and k."""
    q = rope(q_src, num_heads, cos, sin)
    k = rope(k_src, num_kv_heads, cos, sin)
    L, D = cos.shape
    v = None if v_src is None else v_src[:, :num_kv_heads * D].reshape(L, num_kv_heads, D).transpose(0, 1)[None]
    return q, k, None if v is None else v.contiguous(), pool(q, block_size), pool(k, block_size)


def block_mask(qb: torch.Tensor, kb: torch.Tensor, params, dtype: torch.dtype):
    """Canonical selection from pooled qb [B,H,N,D], kb [B,Hkv,N,D].

    Returns dict with packed ``bits`` [B,H,N,W] (int32 view of uint32),
    ``row_count``, ``corr``, ``corr_sum`` [B,H,N], ``is_stripe``, ``stripe_var`` [B,H].
    """
    qf = qb.float().contiguous()
    kf = kb.float().contiguous()
    B, H, N, D = qf.shape
    Hkv = kf.shape[1]
    W = (N + 31) // 32
    cp = params.to_c()
    bits = torch.zeros(B, H, N, W, dtype=torch.int32)
    row_count = torch.zeros(B, H, N, dtype=torch.int32)
    corr = torch.zeros(B, H, N, dtype=torch.float32)
    corr_sum = torch.zeros(B, H, N, dtype=torch.float32)
    is_stripe = torch.zeros(B, H, dtype=torch.uint8)
    stripe_var = torch.zeros(B, H, dtype=torch.float32)
    rc = lib().ffo_block_mask(qf.data_ptr(), kf.data_ptr(), _dtype_code(dtype), B, H, Hkv, D,
                              ctypes.addressof(cp), bits.data_ptr(), row_count.data_ptr(),
                              corr.data_ptr(), corr_sum.data_ptr(), is_stripe.data_ptr(),
                              stripe_var.data_ptr())
    if rc != 0:
        raise ValueError(f"ffo_block_mask failed (rc={rc})")
    return {"bits": bits, "row_count": row_count, "corr": corr, "corr_sum": corr_sum,
            "is_stripe": is_stripe, "stripe_var": stripe_var}


def unpack_bits(bits: torch.Tensor, n: int) -> torch.Tensor:
    """[..., W] packed words -> bool [..., n]."""
    b = bits.to(torch.int64) & 0xFFFFFFFF
    shifts = torch.arange(32, dtype=torch.int64)
    expanded = ((b[..., :, None] >> shifts) & 1).to(torch.bool)
    return expanded.reshape(*bits.shape[:-1], -1)[..., :n]


def pack_bool(mask: torch.Tensor) -> torch.Tensor:
    """bool [..., n] -> packed int32 words [..., ceil(n/32)]."""
    n = mask.shape[-1]
    W = (n + 31) // 32
    m = np.zeros(mask.shape[:-1] + (W * 32,), dtype=np.uint8)
    m[..., :n] = mask.numpy().astype(np.uint8)
    packed = np.packbits(m, axis=-1, bitorder="little")  # [..., W*4] bytes
    return torch.from_numpy(np.ascontiguousarray(packed).view(np.int32).copy())


def prefill_mask(q: torch.Tensor, k: torch.Tensor, params):
    """Pool q/k ([B,H,L,D] / [B,Hkv,L,D], CPU) and run the canonical selection."""
    qb = pool(q, params.block_size)
    kb = pool(k, params.block_size)
    out = block_mask(qb, kb, params, q.dtype)
    out["qb"] = qb
    out["kb"] = kb
    return out


def sparse_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, mask: torch.Tensor,
                     block_size: int, causal: bool = True, heads=None, rows=None):
    """fp32 CPU block-sparse attention.

    q [B,H,L,D], k/v [B,Hkv,L,D] (any float dtype), mask bool [B,H,Nq,Nk].
    Returns fp32 [B, H, L, D] (only ``heads`` / query-block ``rows`` filled if given).
    """
    B, H, L, D = q.shape
    Hkv = k.shape[1]
    rep = H // Hkv
    out = torch.zeros(B, H, L, D, dtype=torch.float32)
    scale = 1.0 / (D ** 0.5)
    tok_blk = torch.arange(L) // block_size
    nq = mask.shape[2]
    for b in range(B):
        for h in (range(H) if heads is None else heads):
            qh = q[b, h].float()
            kh = k[b, h // rep].float()
            vh = v[b, h // rep].float()
            for i in (range(nq) if rows is None else rows):
                r0, r1 = i * block_size, min(L, (i + 1) * block_size)
                if r0 >= L:
                    continue
                sel = mask[b, h, i][tok_blk]
                allowed = sel[None, :].expand(r1 - r0, L)
                if causal:
                    allowed = allowed & (torch.arange(L)[None, :] <= torch.arange(r0, r1)[:, None])
                keys = allowed.any(dim=0).nonzero().flatten()
                if keys.numel() == 0:
                    continue
                s = (qh[r0:r1] @ kh[keys].T) * scale
                a = allowed[:, keys]
                s = s.masked_fill(~a, float("-inf"))
                any_row = a.any(dim=1, keepdim=True)
                p = torch.softmax(s.masked_fill(~any_row, 0.0), dim=-1) * any_row
                out[b, h, r0:r1] = p @ vh[keys]
    return out


def as_numpy_bits(bits: torch.Tensor) -> np.ndarray:
    return bits.numpy().view(np.uint32)
