"""Host-side derivation of the mask-selection parameters.

Every integer and threshold below is derived with the same Python/torch
arithmetic as ``myattn_prefill`` in attn_src/fft_attn/my_attn_v7.py, so that
the kernels see exactly the values the reference would use:

  keep_sink / keep_recent / local_window        :537-540
  correlation top-k gate                        :579-581
  exclude_tau / sink_tau_start                  :137-138 (batch_fft_cross_correlation)
  remote_start                                  :183-184, :585-586
  number of sampled diagonals                   :589-591
  sampled lags (torch.linspace(...).long())     :323-334
  column range and top-k count                  :622-634, :429-437
  last-row top-k                                :65

The result is a ctypes mirror of ``ffts_mask_params`` (include/fftsparse_b200.h).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from typing import List

import torch

MAX_DIAG_SAMPLES = 64
SEL_THRESHOLD = 0
SEL_TOPK = 1


class CMaskParams(ctypes.Structure):
    """ctypes layout of ``ffts_mask_params``."""

    _fields_ = [
        ("n_blocks", ctypes.c_int32),
        ("block_size", ctypes.c_int32),
        ("keep_sink", ctypes.c_int32),
        ("keep_recent", ctypes.c_int32),
        ("local_window", ctypes.c_int32),
        ("corr_on", ctypes.c_int32),
        ("corr_mode", ctypes.c_int32),
        ("corr_threshold", ctypes.c_float),
        ("corr_quantile", ctypes.c_float),
        ("exclude_tau", ctypes.c_int32),
        ("sink_tau_raw", ctypes.c_int32),
        ("remote_start", ctypes.c_int32),
        ("n_diag_samples", ctypes.c_int32),
        ("diag_taus", ctypes.c_int32 * MAX_DIAG_SAMPLES),
        ("stripe_all_diffuse", ctypes.c_int32),
        ("stripe_threshold", ctypes.c_float),
        ("qk_topk_ratio", ctypes.c_float),
        ("col_on", ctypes.c_int32),
        ("col_start", ctypes.c_int32),
        ("col_end", ctypes.c_int32),
        ("col_topk", ctypes.c_int32),
        ("last_on", ctypes.c_int32),
        ("last_topk", ctypes.c_int32),
    ]


@dataclass
class MaskParams:
    n_blocks: int
    block_size: int
    keep_sink: int
    keep_recent: int
    local_window: int
    corr_on: bool
    corr_mode: int
    corr_threshold: float
    corr_quantile: float
    exclude_tau: int
    sink_tau_raw: int
    remote_start: int
    diag_taus: List[int] = field(default_factory=list)
    stripe_all_diffuse: bool = False
    stripe_threshold: float = 0.3
    qk_topk_ratio: float = 0.2
    col_on: bool = True
    col_start: int = 0
    col_end: int = 0
    col_topk: int = 0
    last_on: bool = True
    last_topk: int = 0

    def to_c(self) -> CMaskParams:
        c = CMaskParams()
        for name, _ in CMaskParams._fields_:
            if name in ("diag_taus", "n_diag_samples"):
                continue
            value = getattr(self, name)
            setattr(c, name, int(value) if isinstance(value, bool) else value)
        c.n_diag_samples = len(self.diag_taus)
        for i, t in enumerate(self.diag_taus):
            c.diag_taus[i] = int(t)
        return c


def _f32(x: float) -> float:
    return float(torch.tensor(x, dtype=torch.float32))


def _sample_taus(n_blocks: int, remote_start: int, num_sample_diags: int) -> List[int]:
    """Lags sampled by compute_stripe_variance (my_attn_v7.py:323-334)."""
    max_tau = (n_blocks + remote_start) // 2
    num_available = max(1, max_tau - remote_start + 1)
    actual_num = min(num_sample_diags, num_available)
    if actual_num <= 1:
        return [remote_start]
    idx = torch.linspace(0, num_available - 1, actual_num).long()
    return [int(t) + remote_start for t in idx.tolist()]


def derive_mask_params(seq_len: int, *, block_size: int = 128, sink_ratio: float = 0.1,
                       recent_ratio: float = 0.1, local_span_ratio: float = 0.1,
                       enable_correlation_mask: bool = True,
                       correlation_selection_mode: str = "threshold",
                       correlation_topk_ratio: float = 0.2, corr_threshold: float = 0.1,
                       enable_column_mask: bool = True, column_topk_ratio: float = 0.1,
                       column_start_exclude_ratio: float = 0.1,
                       column_end_exclude_ratio: float = 0.2,
                       enable_last_block_mask: bool = True, diag_sample_ratio: float = 0.15,
                       min_diag_samples: int = 5, max_diag_samples: int = 64,
                       stripe_threshold: float = 0.3, qk_topk_ratio: float = 0.2,
                       **_ignored) -> MaskParams:
    """Mask-selection parameters for a self-attention prefill of ``seq_len`` tokens.

    Raises ValueError where the reference raises (unknown selection mode,
    my_attn_v7.py:210) or where it would fail to unpack the early-return of
    create_correlation_block_mask (remote_start >= N, :191 vs :568).
    """
    N = (seq_len + block_size - 1) // block_size
    keep_sink = max(1, int(N * sink_ratio))
    keep_recent = max(1, int(N * recent_ratio))
    local_span = max(2, int(N * local_span_ratio))
    local_window = local_span // 2
    correlation_top_k = max(1, int(N * correlation_topk_ratio))
    corr_on = bool(enable_correlation_mask) and N > correlation_top_k
    exclude_tau = local_window + 1
    sink_tau_raw = N - keep_sink - 5
    remote_start = max(local_window, keep_recent - 1) + 1
    if corr_on:
        if correlation_selection_mode not in ("threshold", "topk"):
            raise ValueError(f"Unknown selection_mode: {correlation_selection_mode}")
        if remote_start >= N:
            raise ValueError(
                "remote_start >= number of blocks: the reference's "
                "create_correlation_block_mask returns a bare mask here and the caller "
                "fails to unpack it (my_attn_v7.py:191, :568)")
    if max_diag_samples > MAX_DIAG_SAMPLES:
        raise ValueError(f"max_diag_samples > {MAX_DIAG_SAMPLES} is not supported")
    num_remote_diags = max(1, (N + remote_start) // 2 - remote_start + 1)
    num_diag_samples = int(num_remote_diags * diag_sample_ratio)
    num_diag_samples = max(min_diag_samples, min(num_diag_samples, max_diag_samples))
    stripe_all_diffuse = remote_start >= N - 1
    diag_taus = [] if stripe_all_diffuse else _sample_taus(N, remote_start, num_diag_samples)
    if len(diag_taus) > MAX_DIAG_SAMPLES:
        raise ValueError(f"more than {MAX_DIAG_SAMPLES} sampled diagonals")

    col_on = bool(enable_column_mask) and N > 1
    col_ratio_scale = min(1.0, (128.0 / N) ** 0.5)
    scaled_ratio = column_topk_ratio * col_ratio_scale
    col_start = max(1, int(N * column_start_exclude_ratio))
    col_end = N - max(1, int(N * column_end_exclude_ratio))
    if col_end > col_start:
        nvalid = col_end - col_start
        col_topk = min(max(1, int(nvalid * scaled_ratio)), nvalid)
    else:
        col_topk = 0

    return MaskParams(
        n_blocks=N, block_size=block_size, keep_sink=keep_sink, keep_recent=keep_recent,
        local_window=local_window, corr_on=corr_on,
        corr_mode=SEL_TOPK if correlation_selection_mode == "topk" else SEL_THRESHOLD,
        corr_threshold=_f32(corr_threshold), corr_quantile=_f32(1.0 - correlation_topk_ratio),
        exclude_tau=exclude_tau, sink_tau_raw=sink_tau_raw, remote_start=remote_start,
        diag_taus=diag_taus, stripe_all_diffuse=stripe_all_diffuse,
        stripe_threshold=_f32(stripe_threshold), qk_topk_ratio=_f32(qk_topk_ratio),
        col_on=col_on, col_start=col_start, col_end=col_end, col_topk=col_topk,
        last_on=bool(enable_last_block_mask), last_topk=min(128, N),
    )
