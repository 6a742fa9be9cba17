"""The FFTSparse prefill operator on B200.

``myattn_prefill`` keeps the signature, argument meaning, return layout and
error behaviour of the reference's ``myattn_prefill``
(attn_src/fft_attn/my_attn_v7.py:454-792) so that it drops into the model
patching code that calls it (eval/LongBench/pred.py:216,
eval/RULER/pred.py:89, eval/LVEval/pred.py:277,
eval/InfiniteBench/src/pred_infinitebench.py:336,
eval/efficiency/benchmark_attention_multilayer.py:308).

Every step runs in libfftsparse_b200.so on the current CUDA stream with no
host synchronisation:

  ffts_pool            block mean pooling of q and k          (ref :552-555)
  ffts_block_mask      the union of all block masks           (ref :532-641)
  ffts_sparse_attn_fwd block-sparse causal attention          (ref :763-786)

``fft_block_mask`` additionally exposes the selected block mask (the
reference's ``base_blockmask``) and the intermediate statistics.
``rope_pool`` (ffts_rope_pool) serves the caller's side: the RoPE its
attention forward applies before the call, the head-major layout and the
pooling of q and k in one pass, whose pooled blocks ``fft_block_mask`` and
``myattn_prefill`` accept (``pooled=``); ``qkv_rope_pool`` (ffts_qkv_rope_pool)
also folds the QKV projection GEMM in front of them.  ``corr_mask_fraction`` feeds the
reference's calibration hook.
"""
from __future__ import annotations

import sys
from dataclasses import dataclass
from typing import Optional

import torch

from . import _lib, trace
from .params import SEL_TOPK, derive_mask_params, MaskParams
from .status import device_status

__all__ = ["myattn_prefill", "myattn_prefill_host", "fft_block_mask", "sparse_attention", "pool_blocks", "BlockMask",
           "AttentionCache", "_attention_cache"]


class AttentionCache:
    """Kept for interface parity with my_attn_v7.py:23-47 (cu_seqlens and
    head_mask_type caches).  The B200 kernels need neither, so the cache is
    never consulted on the hot path."""

    def __init__(self):
        self._cu_seqlens = {}
        self._head_mask_type = {}

    def get_cu_seqlens(self, seq_len, device):
        key = (seq_len, str(device))
        if key not in self._cu_seqlens:
            self._cu_seqlens[key] = torch.tensor([0, seq_len], dtype=torch.int32, device=device)
        return self._cu_seqlens[key]

    def get_head_mask_type(self, num_heads, device):
        key = (num_heads, str(device))
        if key not in self._head_mask_type:
            self._head_mask_type[key] = torch.tensor([1] * num_heads, dtype=torch.int32, device=device)
        return self._head_mask_type[key]


_attention_cache = AttentionCache()

_DTYPES = {torch.float32: _lib.DTYPE_F32, torch.bfloat16: _lib.DTYPE_BF16}


def _stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _check_4d(name: str, t: torch.Tensor):
    if t.dim() != 4:
        raise ValueError(f"{name} must be [B, H, L, D], got shape {tuple(t.shape)}")
    if t.stride(-1) != 1:
        raise ValueError(f"{name} must be contiguous in the head dimension")


def pool_blocks(x: torch.Tensor, block_size: int) -> torch.Tensor:
    """Block mean of x [B, H, L, D] (ffts_pool) -> contiguous [B, H, N, D] in x.dtype."""
    _check_4d("x", x)
    if x.dtype not in _DTYPES:
        raise TypeError(f"pooling supports float32 and bfloat16, got {x.dtype}")
    lib = _lib.load()
    B, H, L, D = x.shape
    N = (L + block_size - 1) // block_size
    out = torch.empty(B, H, N, D, dtype=x.dtype, device=x.device)
    _lib.check(lib.ffts_pool(x.data_ptr(), _DTYPES[x.dtype], B, H, L, D, x.stride(0), x.stride(1),
                             x.stride(2), block_size, out.data_ptr(), _stream_ptr(x.device)))
    return out


def rope_pool(q_proj: torch.Tensor, k_proj: torch.Tensor, v_proj: Optional[torch.Tensor], num_heads: int,
              num_kv_heads: int, cos: torch.Tensor, sin: torch.Tensor, block_size: int = 128):
    """The caller's rotary embedding, head-major layout and the block pooling of
    q and k in one pass (ffts_rope_pool).

    q_proj [L, >= num_heads * 128], k_proj / v_proj [L, >= num_kv_heads * 128]:
    token-major bf16 projections (rows may be strided, e.g. column slices of one
    fused QKV product); v_proj may be None.  cos / sin: bf16 [L, 128] (HF's
    position embeddings for one sequence).  Returns (q, k, v, q_pooled,
    k_pooled): q [1, num_heads, L, 128] and k, v [1, num_kv_heads, L, 128]
    contiguous, q rotated as HF apply_rotary_pos_emb rotates it in bf16, and
    the pooled blocks that ``fft_block_mask(q, k, pooled=(q_pooled, k_pooled))``
    takes instead of pooling q and k again.
    """
    for name, t in (("q_proj", q_proj), ("k_proj", k_proj), ("v_proj", v_proj), ("cos", cos), ("sin", sin)):
        if t is None and name == "v_proj":
            continue
        if t.dim() != 2 or t.stride(1) != 1 or t.dtype != torch.bfloat16:
            raise ValueError(f"{name} must be a 2-D bf16 tensor with unit column stride")
    L, D = cos.shape
    if sin.shape != cos.shape or sin.stride() != cos.stride():
        raise ValueError("cos and sin must have the same shape and strides")
    if q_proj.shape[0] != L or k_proj.shape[0] != L or (v_proj is not None and v_proj.shape[0] != L):
        raise ValueError("projections and cos/sin must have the same number of rows")
    if q_proj.shape[1] < num_heads * D or k_proj.shape[1] < num_kv_heads * D or \
            (v_proj is not None and v_proj.shape[1] < num_kv_heads * D):
        raise ValueError("a projection has fewer columns than its heads need")
    dev = q_proj.device
    N = (L + block_size - 1) // block_size
    q = torch.empty(1, num_heads, L, D, dtype=torch.bfloat16, device=dev)
    k = torch.empty(1, num_kv_heads, L, D, dtype=torch.bfloat16, device=dev)
    v = None if v_proj is None else torch.empty(1, num_kv_heads, L, D, dtype=torch.bfloat16, device=dev)
    qb = torch.empty(1, num_heads, N, D, dtype=torch.bfloat16, device=dev)
    kb = torch.empty(1, num_kv_heads, N, D, dtype=torch.bfloat16, device=dev)
    lib = _lib.load()
    _lib.check(lib.ffts_rope_pool(
        q_proj.data_ptr(), q_proj.stride(0), k_proj.data_ptr(), k_proj.stride(0),
        None if v_proj is None else v_proj.data_ptr(), 0 if v_proj is None else v_proj.stride(0),
        L, num_heads, num_kv_heads, D, cos.data_ptr(), sin.data_ptr(), cos.stride(0), block_size,
        q.data_ptr(), k.data_ptr(), None if v is None else v.data_ptr(), qb.data_ptr(), kb.data_ptr(),
        _stream_ptr(dev)))
    return q, k, v, qb, kb


def qkv_rope_pool(hidden: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor], num_heads: int,
                  num_kv_heads: int, cos: torch.Tensor, sin: torch.Tensor, block_size: int = 128,
                  return_projection: bool = False, status: Optional[torch.Tensor] = None):
    """The caller's QKV projection with RoPE, the head-major layout and the q/k
    block pooling in the GEMM's epilogue (ffts_qkv_rope_pool).

    hidden [B, L, hidden_size] or [L, hidden_size] bf16 (unit column stride);
    weight [(num_heads + 2 num_kv_heads) * 128, hidden_size] bf16: the q_proj,
    k_proj and v_proj weights stacked row-wise (``torch.cat([q_proj.weight,
    k_proj.weight, v_proj.weight])``); bias: the stacked biases or None; cos /
    sin: bf16 [L, 128].  Returns (q, k, v, q_pooled, k_pooled) with q
    [B, num_heads, L, 128], k and v [B, num_kv_heads, L, 128], the pooled blocks
    [B, H, N, 128]; with ``return_projection`` also the bf16 projection
    [B, L, (num_heads + 2 num_kv_heads) * 128] before RoPE (what the three
    Linear calls return, up to the GEMM's summation order), of which the other
    outputs are exactly ``rope_pool``'s.  ``status`` as for ``sparse_attention``.
    """
    if hidden.dim() == 2:
        hidden = hidden.unsqueeze(0)
    for name, t in (("hidden", hidden), ("weight", weight), ("cos", cos), ("sin", sin)):
        if t.dtype != torch.bfloat16 or t.stride(-1) != 1:
            raise ValueError(f"{name} must be bf16 with unit column stride")
    if hidden.dim() != 3 or weight.dim() != 2:
        raise ValueError("hidden must be [B, L, hidden_size] (or [L, hidden_size]) and weight 2-D")
    B, L, K = hidden.shape
    D = 128
    heads = num_heads + 2 * num_kv_heads
    if weight.shape != (heads * D, K):
        raise ValueError(f"weight must be [{heads * D}, {K}] (q, k, v projections stacked), got {tuple(weight.shape)}")
    if bias is not None and (bias.shape != (heads * D,) or bias.dtype != torch.bfloat16 or not bias.is_contiguous()):
        raise ValueError(f"bias must be a contiguous bf16 [{heads * D}]")
    if cos.shape != (L, D) or sin.shape != cos.shape or sin.stride() != cos.stride():
        raise ValueError(f"cos and sin must both be [{L}, {D}] with the same strides")
    dev = hidden.device
    N = (L + block_size - 1) // block_size
    q = torch.empty(B, num_heads, L, D, dtype=torch.bfloat16, device=dev)
    k = torch.empty(B, num_kv_heads, L, D, dtype=torch.bfloat16, device=dev)
    v = torch.empty(B, num_kv_heads, L, D, dtype=torch.bfloat16, device=dev)
    qb = torch.empty(B, num_heads, N, D, dtype=torch.bfloat16, device=dev)
    kb = torch.empty(B, num_kv_heads, N, D, dtype=torch.bfloat16, device=dev)
    proj = torch.empty(B, L, heads * D, dtype=torch.bfloat16, device=dev) if return_projection else None
    own = None
    if status is None:
        own = device_status(dev)
        own.poll()
        status = own.word
    lib = _lib.load()
    ws_bytes = int(lib.ffts_qkv_workspace_bytes(L))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    _lib.check(lib.ffts_qkv_rope_pool(
        hidden.data_ptr(), B, L, K, hidden.stride(1), hidden.stride(0), weight.data_ptr(), weight.stride(0),
        None if bias is None else bias.data_ptr(), num_heads, num_kv_heads, D, cos.data_ptr(), sin.data_ptr(),
        cos.stride(0), block_size, q.data_ptr(), k.data_ptr(), v.data_ptr(), qb.data_ptr(), kb.data_ptr(),
        None if proj is None else proj.data_ptr(), 0 if proj is None else proj.stride(1), ws.data_ptr(), ws_bytes,
        status.data_ptr(), _stream_ptr(dev)))
    if own is not None:
        own.read_back()
    if return_projection:
        return q, k, v, qb, kb, proj
    return q, k, v, qb, kb


@dataclass
class BlockMask:
    """Result of the block-mask selection for a [B, H, L, D] prefill."""

    bits: torch.Tensor          # int32 [B, H, N, W] packed (bit j of row i = key block j kept)
    row_count: torch.Tensor     # int32 [B, H, N]
    corr: torch.Tensor          # fp32 [B, H, N] lag scores (corr_causal)
    corr_sum: torch.Tensor      # fp32 [B, H, N] raw lag sums (corr_causal_sum)
    is_stripe: torch.Tensor     # uint8 [B, H]
    stripe_var: torch.Tensor    # fp32 [B, H]
    params: MaskParams
    q_pooled: torch.Tensor
    k_pooled: torch.Tensor

    @property
    def n_blocks(self) -> int:
        return self.params.n_blocks

    def dense(self) -> torch.Tensor:
        """bool [B, H, N, N], the reference's ``base_blockmask`` layout."""
        lib = _lib.load()
        B, H, N, _ = self.bits.shape
        out = torch.empty(B, H, N, N, dtype=torch.uint8, device=self.bits.device)
        _lib.check(lib.ffts_unpack_mask(self.bits.data_ptr(), B, H, N, out.data_ptr(),
                                        _stream_ptr(self.bits.device)))
        return out.view(torch.bool)

    def csr(self):
        """(row_ptr int64 [B*H*N+1], col_idx int32 [nnz]): the kept key blocks of
        each query block in ascending order, rows in [B, H, N] order, built on the
        device from the packed bits (ffts_mask_row_ptr, ffts_mask_col_idx).  Reads
        the total count back once to size col_idx."""
        lib = _lib.load()
        dev = self.bits.device
        B, H, N, _ = self.bits.shape
        rows = B * H * N
        row_ptr = torch.empty(rows + 1, dtype=torch.int64, device=dev)
        _lib.check(lib.ffts_mask_row_ptr(self.row_count.data_ptr(), rows, row_ptr.data_ptr(), _stream_ptr(dev)))
        nnz = int(row_ptr[-1].item())
        col_idx = torch.empty(max(nnz, 1), dtype=torch.int32, device=dev)
        status = torch.zeros(1, dtype=torch.int32, device=dev)
        _lib.check(lib.ffts_mask_col_idx(self.bits.data_ptr(), rows, N, row_ptr.data_ptr(), col_idx.data_ptr(), nnz,
                                         status.data_ptr(), _stream_ptr(dev)))
        if int(status.item()) != 0:
            raise RuntimeError("block mask rows and row counts disagree (row_count does not match the bits)")
        return row_ptr, col_idx[:nnz]

    def density(self) -> float:
        """Kept fraction of the causal block pairs."""
        N = self.n_blocks
        causal = N * (N + 1) // 2
        return float(self.row_count.sum()) / (causal * self.row_count.shape[0] * self.row_count.shape[1])


def fft_block_mask(query_states: torch.Tensor, key_states: torch.Tensor, *, block_size: int = 128,
                   params: Optional[MaskParams] = None, pooled=None, **kwargs) -> BlockMask:
    """Select the FFTSparse block mask for q [B, H, L, D] and k [B, Hkv, L, D].

    ``kwargs`` are the mask arguments of myattn_prefill (sink_ratio,
    recent_ratio, local_span_ratio, enable_correlation_mask,
    correlation_selection_mode, ...).  ``pooled = (q_pooled, k_pooled)``, the
    [B, H, N, D] / [B, Hkv, N, D] block means already computed (rope_pool),
    skips the pooling pass.
    """
    q, k = query_states, key_states
    _check_4d("query_states", q)
    _check_4d("key_states", k)
    if q.dtype != k.dtype:
        raise TypeError("query and key dtypes differ")
    if q.dtype not in _DTYPES:
        raise TypeError(f"mask selection supports float32 and bfloat16, got {q.dtype}")
    B, H, L, D = q.shape
    Hkv = k.shape[1]
    if k.shape[0] != B or k.shape[2] != L or k.shape[3] != D or H % Hkv:
        raise ValueError(f"key_states {tuple(k.shape)} incompatible with query_states {tuple(q.shape)}")
    cp = None
    if params is None:
        params, cp = _cached_params(L, block_size, kwargs)
    lib = _lib.load()
    N = params.n_blocks
    if pooled is None:
        with trace.stage("3_mean_pool"):
            qb = pool_blocks(q, params.block_size)
            kb = pool_blocks(k, params.block_size)
    else:
        qb, kb = pooled
        if qb.shape != (B, H, N, D) or kb.shape != (B, Hkv, N, D) or qb.dtype != q.dtype or \
                kb.dtype != q.dtype or not (qb.is_contiguous() and kb.is_contiguous()):
            raise ValueError(f"pooled blocks must be contiguous [B, H, N, D] / [B, Hkv, N, D] with N = {N} "
                             f"in the input dtype")
    W = (N + 31) // 32
    dev = q.device
    bits = torch.empty(B, H, N, W, dtype=torch.int32, device=dev)
    row_count = torch.empty(B, H, N, dtype=torch.int32, device=dev)
    corr = torch.empty(B, H, N, dtype=torch.float32, device=dev)
    corr_sum = torch.empty(B, H, N, dtype=torch.float32, device=dev)
    is_stripe = torch.empty(B, H, dtype=torch.uint8, device=dev)
    stripe_var = torch.empty(B, H, dtype=torch.float32, device=dev)
    ws_bytes = int(lib.ffts_mask_workspace_bytes(B, H, N, D))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    if cp is None:
        cp = params.to_c()
    with trace.stage("4-9_select"):
        _lib.check(lib.ffts_block_mask(qb.data_ptr(), kb.data_ptr(), _DTYPES[q.dtype], B, H, Hkv, D,
                                       _lib.ctypes.addressof(cp), bits.data_ptr(), row_count.data_ptr(),
                                       corr.data_ptr(), corr_sum.data_ptr(), is_stripe.data_ptr(),
                                       stripe_var.data_ptr(), ws.data_ptr(), ws_bytes, _stream_ptr(dev)))
    return BlockMask(bits, row_count, corr, corr_sum, is_stripe, stripe_var, params, qb, kb)


_PARAM_CACHE = {}


def _cached_params(L: int, block_size: int, kwargs: dict):
    """derive_mask_params and its C struct, reused across calls with the same length
    and arguments (a prefill calls the operator once per layer with the same ones)."""
    try:
        key = (L, block_size, tuple(sorted(kwargs.items())))
        hit = _PARAM_CACHE.get(key)
    except TypeError:  # an unhashable argument: derive afresh
        key, hit = None, None
    if hit is None:
        params = derive_mask_params(L, block_size=block_size, **kwargs)
        hit = (params, params.to_c())
        if key is not None:
            if len(_PARAM_CACHE) > 256:
                _PARAM_CACHE.clear()
            _PARAM_CACHE[key] = hit
    return hit


def corr_mask_fraction(corr: torch.Tensor, params: MaskParams) -> float:
    """Kept fraction of the reference's correlation block mask, the value its
    calibration hook records under "corr" (my_attn_v7.py:713-717).

    The mask (create_correlation_block_mask, :160-227) keeps block (i, j) of a
    head when the lag i - j is a selected remote lag and j >= keep_sink.  The
    lags are selected from the fp32 lag scores ``corr`` [B, H, N] exactly as the
    reference selects them (:193-206): corr >= torch.quantile(remote scores,
    1 - topk_ratio) in top-k mode, corr / max(remote scores, 1e-6) >= threshold
    in threshold mode.  Lag t then contributes max(0, N - t - keep_sink) blocks;
    the fraction is over all B * H * N * N blocks.  Calibration only: it reads
    the scores back to the host.
    """
    N, rs, ks = params.n_blocks, params.remote_start, params.keep_sink
    B, H = corr.shape[0], corr.shape[1]
    if rs >= N:
        return 0.0
    remote = corr[..., rs:].float()
    if params.corr_mode == SEL_TOPK:
        # corr_quantile is 1 - topk_ratio rounded to fp32, as torch.quantile rounds it
        thr = torch.quantile(remote, params.corr_quantile, dim=-1, keepdim=True)
        sel = remote >= thr
    else:
        mx = remote.max(dim=-1, keepdim=True).values.clamp(min=1e-6)
        sel = (remote / mx) >= params.corr_threshold
    taus = torch.arange(rs, N, device=corr.device)
    per_lag = (N - taus - ks).clamp(min=0)
    kept = int((sel.to(torch.int64) * per_lag).sum().item())
    return kept / (B * H * N * N)


def _dense_causal_bits(B: int, H: int, N: int, device) -> torch.Tensor:
    W = (N + 31) // 32
    return torch.full((B, H, N, W), -1, dtype=torch.int32, device=device)


def sparse_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, bits: torch.Tensor,
                     block_size: int, causal: bool = True, out: Optional[torch.Tensor] = None,
                     status: Optional[torch.Tensor] = None, rows=None, peers=None) -> torch.Tensor:
    """Block-sparse attention (ffts_sparse_attn_fwd).

    q [B, H, L, D], k/v [B, Hkv, L, D] bf16; bits [B, H, N, W] packed mask.
    Returns (or fills) ``out`` of shape [B, L, H, D] bf16.  With ``rows = (lo, hi)``
    only query rows [lo, hi) are computed (lo a multiple of 128, hi a multiple of
    128 or L; ffts_sparse_attn_fwd_rows) and ``out`` has shape [B, hi - lo, H, D].
    With ``peers`` (device addresses of other GPUs' buffers laid out like ``out``,
    mapped into this process) every output row is also stored there by the
    kernel's epilogue (ffts_sparse_attn_fwd_push).

    ``status`` (int32 [1] on q's device) receives the code of a bounded wait that
    timed out; the caller then reads it.  Without it the device's own status word
    is used (fftsparse_b200.status): a time-out raises WaitTimeout at the first
    call after the failing kernel has completed, or at ``check_status()``.
    """
    for name, t in (("q", q), ("k", k), ("v", v)):
        _check_4d(name, t)
        if t.dtype != torch.bfloat16:
            raise TypeError(f"block-sparse attention supports bfloat16 inputs only (got {name} {t.dtype})")
    B, H, L, D = q.shape
    Hkv = k.shape[1]
    lo, hi = (0, L) if rows is None else (int(rows[0]), int(rows[1]))
    if out is None:
        out = torch.empty(B, hi - lo, H, D, dtype=torch.bfloat16, device=q.device)
    lib = _lib.load()
    qs = _lib.i64_array([q.stride(0), q.stride(1), q.stride(2)])
    ks = _lib.i64_array([k.stride(0), k.stride(1), k.stride(2)])
    vs = _lib.i64_array([v.stride(0), v.stride(1), v.stride(2)])
    os_ = _lib.i64_array([out.stride(0), out.stride(2), out.stride(1)])
    own = None
    if status is None:
        own = device_status(q.device)
        own.poll()  # an earlier call's time-out, if its read-back has landed
        status = own.word
    st = status.data_ptr()
    if peers:
        arr = (_lib.ctypes.c_void_p * len(peers))(*peers)
        _lib.check(lib.ffts_sparse_attn_fwd_push(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), B, H, Hkv, L, D, qs, ks, vs, bits.data_ptr(),
            block_size, int(bool(causal)), lo, hi, out.data_ptr(), os_, arr, len(peers), st,
            _stream_ptr(q.device)))
    elif rows is None:
        _lib.check(lib.ffts_sparse_attn_fwd(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), B, H, Hkv, L, D, qs, ks, vs, bits.data_ptr(),
            block_size, int(bool(causal)), out.data_ptr(), os_, st, _stream_ptr(q.device)))
    else:
        _lib.check(lib.ffts_sparse_attn_fwd_rows(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), B, H, Hkv, L, D, qs, ks, vs, bits.data_ptr(),
            block_size, int(bool(causal)), lo, hi, out.data_ptr(), os_, st, _stream_ptr(q.device)))
    if own is not None:
        own.read_back()
    return out


def myattn_prefill(
        query_states,
        key_states,
        value_states,
        layer_idx,
        block_size=128,
        is_causal=True,
        is_visual=False,
        sink_ratio=0.1,
        recent_ratio=0.1,
        local_span_ratio=0.1,
        enable_correlation_mask=True,
        correlation_selection_mode: str = "threshold",
        correlation_topk_ratio: float = 0.2,
        corr_threshold: float = 0.1,
        collect_corr_stats: bool = False,
        enable_column_mask: bool = True,
        column_topk_ratio: float = 0.1,
        column_start_exclude_ratio: float = 0.1,
        column_end_exclude_ratio: float = 0.2,
        enable_last_block_mask=True,
        last_block_threshold=0.01,
        diag_sample_ratio: float = 0.15,
        min_diag_samples: int = 5,
        max_diag_samples: int = 64,
        stripe_threshold: float = 0.3,
        qk_topk_ratio: float = 0.2,
        attention_vis_heads=(0,),
        attention_vis_dir=None,
        pooled=None,
):
    """Block-sparse prefill attention with FFT-correlation block selection.

    query_states [B, H, L, D]; key_states / value_states [B, H, L, D]
    (repeat_kv-expanded, as the reference's callers pass them) or
    [B, Hkv, L, D] with H % Hkv == 0.  Returns [B, L, H*D] in bf16.

    As in the reference, sequences shorter than 10 blocks use dense causal
    attention (my_attn_v7.py:506-519), ``last_block_threshold``, ``is_visual``,
    ``collect_corr_stats`` and the visualisation arguments are accepted and
    ignored, a non-CUDA input raises AssertionError (:502) and an unknown
    selection mode raises ValueError (:210).

    ``pooled`` (not in the reference's signature; default None) takes the
    (q_pooled, k_pooled) block means a caller already computed with rope_pool,
    so the selection skips its pooling pass.
    """
    assert query_states.is_cuda, "input tensors must be on CUDA"
    q, k, v = query_states, key_states, value_states
    L_q = q.shape[2]
    L_k = k.shape[2]
    if L_q != L_k:
        raise ValueError("prefill expects equal query and key lengths")
    mask_kwargs = dict(
        sink_ratio=sink_ratio, recent_ratio=recent_ratio, local_span_ratio=local_span_ratio,
        enable_correlation_mask=enable_correlation_mask,
        correlation_selection_mode=correlation_selection_mode,
        correlation_topk_ratio=correlation_topk_ratio, corr_threshold=corr_threshold,
        enable_column_mask=enable_column_mask, column_topk_ratio=column_topk_ratio,
        column_start_exclude_ratio=column_start_exclude_ratio,
        column_end_exclude_ratio=column_end_exclude_ratio,
        enable_last_block_mask=enable_last_block_mask, diag_sample_ratio=diag_sample_ratio,
        min_diag_samples=min_diag_samples, max_diag_samples=max_diag_samples,
        stripe_threshold=stripe_threshold, qk_topk_ratio=qk_topk_ratio)
    if trace.enabled():
        with trace.layer(layer_idx):
            return _prefill(q, k, v, block_size, is_causal, pooled, mask_kwargs)
    return _prefill(q, k, v, block_size, is_causal, pooled, mask_kwargs)


def _prefill(q, k, v, block_size, is_causal, pooled, mask_kwargs):
    B, H, L, D = q.shape
    if L < block_size * 10:  # the reference's min_blocks_needed (my_attn_v7.py:506)
        N = (L + block_size - 1) // block_size
        bits = _dense_causal_bits(B, H, N, q.device)
        with trace.stage("10_kernel"):
            out = sparse_attention(q, k, v, bits, block_size, causal=True)
        return out.view(B, L, H * D)

    mask = fft_block_mask(q, k, block_size=block_size, pooled=pooled, **mask_kwargs)

    collector = getattr(sys.modules[__name__], "_sparsity_collector", None)
    if collector is not None:
        N = mask.n_blocks
        if mask.params.corr_on:
            collector.setdefault("corr", []).append(corr_mask_fraction(mask.corr, mask.params))
        collector.setdefault("final", []).append(float(mask.row_count.sum()) / (B * H * N * N))

    with trace.stage("10_kernel"):
        out = sparse_attention(q, k, v, mask.bits, block_size, causal=is_causal)
    return out.view(B, L, H * D)


_HOST_STREAMS = {}


def _host_streams(device: torch.device):
    """(copy-in stream, copy-out stream) of ``device``, created once."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _HOST_STREAMS:
        _HOST_STREAMS[idx] = (torch.cuda.Stream(idx), torch.cuda.Stream(idx))
    return _HOST_STREAMS[idx]


def myattn_prefill_host(query_states, key_states, value_states, layer_idx, chunk_heads: int = 1,
                        out: Optional[torch.Tensor] = None, device=None, **kwargs):
    """``myattn_prefill`` on host buffers, with the copies overlapped with the work.

    query_states [B, H, L, D] and key_states / value_states [B, H or Hkv, L, D]
    are CPU tensors (pinned for the copies to overlap); ``kwargs`` are
    myattn_prefill's.  Returns ``out``, a pinned CPU [B, L, H*D] bf16 tensor
    (allocated when None), equal bit for bit to myattn_prefill on the same inputs
    on the device: the selection and the attention of a head read only that head
    (and its KV head).  Heads go in chunks of ``chunk_heads``, rounded to a
    multiple of the group size H / Hkv (default: one head, or one KV group of
    un-expanded K/V): chunk c+1 is copied in on one stream while chunk c is
    selected and attended on the current stream and chunk c-1's output columns
    are copied back on a third, so the layer takes about as long as its copies
    (small chunks keep the last chunk's work and read-back, which nothing
    overlaps, short).  The call returns once the work is queued; the result is complete when
    the current stream's work is (``torch.cuda.current_stream().synchronize()``).
    The calibration collector, when installed, records one entry per chunk.
    """
    q_h, k_h, v_h = query_states, key_states, value_states
    if kwargs.get("pooled") is not None:
        raise ValueError("myattn_prefill_host pools per head chunk itself; it takes no pooled=")
    for name, t in (("query_states", q_h), ("key_states", k_h), ("value_states", v_h)):
        if t.is_cuda or t.dim() != 4:
            raise ValueError(f"{name} must be a 4-D CPU tensor (use myattn_prefill for device tensors)")
    B, H, L, D = q_h.shape
    Hkv = k_h.shape[1]
    if H % Hkv or v_h.shape != k_h.shape or k_h.shape[0] != B or k_h.shape[2] != L or k_h.shape[3] != D:
        raise ValueError(f"key/value {tuple(k_h.shape)} / {tuple(v_h.shape)} incompatible with query {tuple(q_h.shape)}")
    G = H // Hkv
    hc = max(G, (chunk_heads // G) * G)
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    if out is None:
        out = torch.empty(B, L, H * D, dtype=q_h.dtype, pin_memory=True)
    elif out.shape != (B, L, H * D) or out.is_cuda or not out.is_contiguous():
        raise ValueError(f"out must be a contiguous CPU tensor of shape {(B, L, H * D)}")
    lib = _lib.load()
    comp = torch.cuda.current_stream(dev)
    s_in, s_out = _host_streams(dev)
    s_in.wait_stream(comp)  # device buffers allocated below belong to the current stream's order
    q_d = torch.empty(B, H, L, D, dtype=q_h.dtype, device=dev)
    k_d = torch.empty(B, Hkv, L, D, dtype=k_h.dtype, device=dev)
    v_d = torch.empty(B, Hkv, L, D, dtype=v_h.dtype, device=dev)
    chunks = [(h0, min(H, h0 + hc)) for h0 in range(0, H, hc)]
    arrived = []
    with torch.cuda.stream(s_in):
        for h0, h1 in chunks:
            for b in range(B):  # each [b, h0:h1] slice is contiguous on both sides
                q_d[b, h0:h1].copy_(q_h[b, h0:h1], non_blocking=True)
                k_d[b, h0 // G:h1 // G].copy_(k_h[b, h0 // G:h1 // G], non_blocking=True)
                v_d[b, h0 // G:h1 // G].copy_(v_h[b, h0 // G:h1 // G], non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(s_in)
            arrived.append(ev)
    row = H * D * out.element_size()
    for (h0, h1), ev in zip(chunks, arrived):
        comp.wait_event(ev)
        o = myattn_prefill(q_d[:, h0:h1], k_d[:, h0 // G:h1 // G], v_d[:, h0 // G:h1 // G], layer_idx, **kwargs)
        done = torch.cuda.Event()
        done.record(comp)
        s_out.wait_event(done)
        o.record_stream(s_out)
        width = (h1 - h0) * D * out.element_size()
        for b in range(B):
            _lib.check(lib.ffts_copy_2d(out[b].data_ptr() + h0 * D * out.element_size(), row,
                                        o[b].data_ptr(), width, width, L, s_out.cuda_stream))
    for t in (q_d, k_d, v_d):
        t.record_stream(s_in)
    comp.wait_stream(s_out)  # the current stream's completion covers the read-back
    return out
