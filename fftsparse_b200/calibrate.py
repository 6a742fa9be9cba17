"""Target-sparsity calibration of the correlation selection, on the device.

Restates calibrate_from_qk (eval/efficiency/benchmark_attention_multilayer.py:
179-262).  The reference bisects the selection value (``correlation_topk_ratio``
in top-k mode, ``corr_threshold`` in threshold mode) over [0, 1] for up to 20
steps.  Each step runs the whole operator, attention included, on every layer
and reads the mean correlation-mask kept fraction back through the
``_sparsity_collector`` hook.  The step stops early once the fraction is
within 0.01 of the target.

Here the FFT lag scores, which do not depend on the searched value, are
selected once per layer (one ``fft_block_mask`` pass).  Every bisection step is
then a few tensor operations on the device:
- the lags each layer would select at the step's value (the reference's own
  torch.quantile / normalised-threshold rule, as ``corr_mask_fraction`` applies it);
- their kept fraction;
- the mean over the layers;
- the update of the search interval (``torch.where``, so no step waits for the host).

One read-back gives the chosen value. One more selection pass per layer at that
value gives the reported fractions, as the reference's closing ``measure`` does.
"""
from __future__ import annotations

from typing import Sequence, Tuple

import torch

from .prefill import corr_mask_fraction, fft_block_mask


def _kept_per_lag(N: int, rs: int, ks: int, device) -> torch.Tensor:
    taus = torch.arange(rs, N, device=device)
    return (N - taus - ks).clamp(min=0).to(torch.float64)


def calibrate_from_qk(layers: Sequence[Tuple[torch.Tensor, torch.Tensor]], target_sparsity: float, *,
                      correlation_selection_mode: str = "topk", steps: int = 20, tolerance: float = 0.01,
                      block_size: int = 128, **mask_kwargs):
    """Bisect the correlation selection value so that the mean correlation-mask
    kept fraction over ``layers`` (a sequence of (q [B, H, L, D], k [B, Hkv, L, D])
    pairs) comes within ``tolerance`` of ``target_sparsity``.

    ``mask_kwargs`` are the other myattn_prefill mask arguments.  Their
    ``correlation_topk_ratio`` / ``corr_threshold`` are ignored: in top-k mode
    the searched value is the top-k ratio (threshold 1.0), in threshold mode it
    is the threshold (top-k ratio 0.2), as the reference's ``measure`` sets them.
    Returns ``(best_value, corr_fraction, final_fraction)`` like the reference.
    """
    if correlation_selection_mode not in ("topk", "threshold"):
        raise ValueError(f"Unknown selection_mode: {correlation_selection_mode}")
    topk = correlation_selection_mode == "topk"
    kw = {k: v for k, v in mask_kwargs.items() if k not in ("correlation_topk_ratio", "corr_threshold")}
    kw.update(block_size=block_size, correlation_selection_mode=correlation_selection_mode)

    # the lag scores of every layer, selected once (a top-k ratio of 0 keeps the
    # correlation stage on whenever there is more than one block)
    scores = []
    for q, k in layers:
        sel_kw = dict(kw, correlation_topk_ratio=0.0 if topk else 0.2, corr_threshold=1.0)
        mask = fft_block_mask(q, k, **sel_kw)
        p = mask.params
        if p.corr_on:
            remote = mask.corr[..., p.remote_start:].float()
            scores.append((remote, _kept_per_lag(p.n_blocks, p.remote_start, p.keep_sink, remote.device),
                           p.n_blocks, float(remote.shape[0] * remote.shape[1] * p.n_blocks * p.n_blocks)))
    if not scores:
        raise ValueError("no layer has the correlation stage on")
    dev = scores[0][0].device
    f64 = torch.float64

    def mean_fraction(val: torch.Tensor) -> torch.Tensor:
        """Mean over the layers whose correlation stage is on at ``val`` (nan if none)."""
        total = torch.zeros((), dtype=f64, device=dev)
        count = torch.zeros((), dtype=f64, device=dev)
        for remote, per_lag, N, numel in scores:
            if topk:
                on = N > torch.clamp(torch.floor(N * val), min=1.0)  # N > max(1, int(N * ratio))
                thr = torch.quantile(remote, (1.0 - val).to(torch.float32), dim=-1, keepdim=True)
                sel = remote >= thr
            else:
                on = torch.ones((), dtype=torch.bool, device=dev)
                mx = remote.max(dim=-1, keepdim=True).values.clamp(min=1e-6)
                sel = (remote / mx) >= val.to(torch.float32)
            frac = (sel.to(f64) * per_lag).sum() / numel
            total = total + torch.where(on, frac, torch.zeros_like(frac))
            count = count + on.to(f64)
        return total / count

    lo = torch.zeros((), dtype=f64, device=dev)
    hi = torch.ones((), dtype=f64, device=dev)
    best = torch.full((), 0.5, dtype=f64, device=dev)
    done = torch.zeros((), dtype=torch.bool, device=dev)
    target = torch.tensor(float(target_sparsity), dtype=f64, device=dev)
    for _ in range(steps):
        mid = (lo + hi) / 2
        f = mean_fraction(mid)
        hit = (f - target).abs() < tolerance
        live = ~done
        best = torch.where(live, mid, best)  # the reference's best_val = mid on a hit and after a miss
        move = live & ~hit
        above = f > target
        # top-k: too many lags kept -> smaller ratio; threshold: too many -> larger threshold
        shrink_hi = above if topk else ~above
        hi = torch.where(move & shrink_hi, mid, hi)
        lo = torch.where(move & ~shrink_hi, mid, lo)
        done = done | hit
    best_value = float(best.item())

    corr_fracs, final_fracs = [], []
    for q, k in layers:
        sel_kw = dict(kw, correlation_topk_ratio=best_value if topk else 0.2,
                      corr_threshold=1.0 if topk else best_value)
        mask = fft_block_mask(q, k, **sel_kw)
        p = mask.params
        B, H, N = mask.row_count.shape
        if p.corr_on:
            corr_fracs.append(corr_mask_fraction(mask.corr, p))
        final_fracs.append(float(mask.row_count.sum()) / (B * H * N * N))
    nan = float("nan")
    corr_ret = sum(corr_fracs) / len(corr_fracs) if corr_fracs else nan
    final_ret = sum(final_fracs) / len(final_fracs) if final_fracs else nan
    return best_value, corr_ret, final_ret


__all__ = ["calibrate_from_qk"]
