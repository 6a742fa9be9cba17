"""Decode attention after the FFTSparse prefill (ffts_decode_attn).

The reference's callers switch to an eager decode branch once the prompt is
prefilled (eval/LongBench/pred.py:306-322): softmax(q k^T / sqrt(D)) v over
the repeat_kv-expanded cache, softmax in fp32.  ``decode_attention`` computes
the same for one new token per sequence, reading the cache un-expanded in the
head-major [B, Hkv, Lk, D] layout that ``rope_pool`` writes and an HF cache
stores (the KV-cache handoff needs no copy), with fp32 scores, softmax and
accumulation and a bf16 result.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _lib

_SM_COUNT = {}  # device index -> streaming multiprocessors (the split count aims at ~4 CTAs per SM)


def _sm_count(device: torch.device) -> int:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _SM_COUNT:
        _SM_COUNT[idx] = torch.cuda.get_device_properties(idx).multi_processor_count
    return _SM_COUNT[idx]


def decode_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                     splits: Optional[int] = None, out: Optional[torch.Tensor] = None,
                     attention_mask: Optional[torch.Tensor] = None) -> torch.Tensor:
    """q [B, H, 1, D] or [B, H, D]; k_cache / v_cache [B, Hkv, Lk, D] (bf16, unit
    stride over D, H % Hkv == 0, H / Hkv <= 16, D = 128).  Returns [B, H, D] bf16
    (or fills ``out``).

    ``attention_mask`` is the caller's additive mask for this step, as its decode
    branch adds it (eval/LongBench/pred.py:311-313): HF's [B, 1, 1, >= Lk] causal
    mask (its first Lk columns are used) or [B, Lk]; fp32 or bf16, 0 to keep a
    key and a large negative value (e.g. the dtype's minimum) to drop one, as
    left padding in a batch needs."""
    if q.dim() == 4:
        if q.shape[2] != 1:
            raise ValueError("decode_attention takes one new token per sequence (q_len 1)")
        q = q[:, :, 0]
    if q.dim() != 3 or k_cache.dim() != 4 or v_cache.dim() != 4:
        raise ValueError("q must be [B, H, D] (or [B, H, 1, D]) and the caches [B, Hkv, Lk, D]")
    for name, t in (("q", q), ("k_cache", k_cache), ("v_cache", v_cache)):
        if t.dtype != torch.bfloat16:
            raise TypeError(f"decode attention supports bfloat16 only (got {name} {t.dtype})")
        if t.stride(-1) != 1:
            raise ValueError(f"{name} must be contiguous in the head dimension")
    B, H, D = q.shape
    _, Hkv, Lk, _ = k_cache.shape
    if k_cache.shape[0] != B or v_cache.shape != k_cache.shape or k_cache.shape[3] != D:
        raise ValueError(f"caches {tuple(k_cache.shape)} / {tuple(v_cache.shape)} do not match q {tuple(q.shape)}")
    if splits is None:
        # splits that fill the SMs once (two CTAs per SM when a CTA holds at most 4
        # q-heads, else one: the kernel's shared-memory rings), each at least 64 keys
        G = H // Hkv
        per_sm = 2 if G <= 4 else 1
        ctas = B * Hkv * ((G + 7) // 8)
        splits = max(1, min((Lk + 63) // 64, per_sm * _sm_count(q.device) // ctas))
    if out is None:
        out = torch.empty(B, H, D, dtype=torch.bfloat16, device=q.device)
    mask_ptr, mask_dt, mask_sb = None, 0, 0
    if attention_mask is not None:
        m = attention_mask
        if m.dim() == 4:
            if m.shape[1] != 1 or m.shape[2] != 1:
                raise ValueError(f"a 4-D attention_mask must be [B, 1, 1, kv_len], got {tuple(m.shape)}")
            m = m[:, 0, 0]
        if m.dim() != 2 or m.shape[0] != B or m.shape[1] < Lk:
            raise ValueError(f"attention_mask {tuple(attention_mask.shape)} does not cover [B={B}, Lk={Lk}]")
        if m.dtype not in (torch.float32, torch.bfloat16):
            raise TypeError(f"attention_mask must be fp32 or bf16, got {m.dtype}")
        if m.device != q.device:
            raise ValueError("attention_mask must be on q's device")
        if m.stride(1) != 1:
            m = m.contiguous()
        attention_mask = m  # keep the tensor alive for the launch
        mask_ptr, mask_dt, mask_sb = m.data_ptr(), (_lib.DTYPE_BF16 if m.dtype == torch.bfloat16 else
                                                    _lib.DTYPE_F32), m.stride(0)
    lib = _lib.load()
    nbytes = int(lib.ffts_decode_workspace_bytes(B, H, Hkv, splits))
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=q.device)
    ks = _lib.i64_array([k_cache.stride(0), k_cache.stride(1), k_cache.stride(2)])
    vs = _lib.i64_array([v_cache.stride(0), v_cache.stride(1), v_cache.stride(2)])
    _lib.check(lib.ffts_decode_attn(q.data_ptr(), q.stride(0), q.stride(1), k_cache.data_ptr(), ks,
                                    v_cache.data_ptr(), vs, B, H, Hkv, Lk, D, splits, ws.data_ptr(), nbytes,
                                    out.data_ptr(), out.stride(0), out.stride(1), mask_ptr, mask_dt, mask_sb,
                                    torch.cuda.current_stream(q.device).cuda_stream))
    return out
