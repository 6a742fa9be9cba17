"""Per-stage timing and NVTX ranges for the prefill operator.

The reference's timed variant records CUDA-event milliseconds per (layer, stage)
(attn_src/fft_attn/my_attn_v6_timed.py:26-41) for the stages at :506-657 and
prints a per-layer table with the mean over layers (:44-137).  This module keeps
that schema for the launches of this build.  Several of the reference's stages
are one launch here, so a fused stage carries the joined stage numbers:

    3_mean_pool   block means of q and k (pool_kernel; absent when the caller
                  passed ``pooled=`` from rope_pool / qkv_rope_pool)
    4-9_select    ffts_block_mask: prior bands (2), last-block rows (4), FFT
                  correlation (5), block scores (6), stripe variance (7),
                  q.k top-k (8) and column mask (9), as one C call
    10_kernel     block-sparse attention
    10_kernel+gather, 11_gather
                  the sharded prefill's attention with its peer-memory output
                  gather, or the NCCL all-gather after it (the reference runs on
                  one device and has no such stage)

``1_reshape_pad`` has no counterpart: every kernel reads [B, H, L, D] in place
and handles the ragged last block itself.

Recording is off by default and costs one global read per stage when off.  When
on, each stage records two CUDA events on the current stream; nothing
synchronises until ``times()`` or ``summary()`` reads them.  NVTX ranges named
``fftsparse/<stage>`` (layer in the payload message) are pushed around the same
stages when ``nvtx=True``; the C ABI also pushes one range per entry point, so
nsys shows both levels.  Set FFTS_TRACE=1 in the environment to switch recording
(events and NVTX) on at import.
"""
from __future__ import annotations

import contextlib
import os
import sys
from typing import Dict, List, Optional

import torch

STAGES = ("3_mean_pool", "4-9_select", "10_kernel", "10_kernel+gather", "11_gather")

_state = {"events": False, "nvtx": False}
_pending: List[tuple] = []          # (layer, stage, start_event, end_event)
_times: Dict[int, Dict[str, List[float]]] = {}
_layer: List[int] = [0]


def enable(events: bool = True, nvtx: bool = True) -> None:
    """Switch recording on: CUDA-event stage timing and/or NVTX ranges."""
    _state["events"] = bool(events)
    _state["nvtx"] = bool(nvtx)


def disable() -> None:
    _state["events"] = False
    _state["nvtx"] = False


def enabled() -> bool:
    return _state["events"] or _state["nvtx"]


def reset() -> None:
    """Forget every recorded time (pending events included)."""
    _pending.clear()
    _times.clear()


@contextlib.contextmanager
def layer(layer_idx: int):
    """Attribute the stages recorded inside to ``layer_idx``."""
    prev = _layer[0]
    _layer[0] = int(layer_idx)
    try:
        yield
    finally:
        _layer[0] = prev


class _Stage:
    __slots__ = ("name", "ev0", "ev1", "pushed")

    def __init__(self, name: str):
        self.name = name
        self.ev0 = self.ev1 = None
        self.pushed = False

    def __enter__(self):
        if _state["nvtx"]:
            torch.cuda.nvtx.range_push(f"fftsparse/{self.name} layer={_layer[0]}")
            self.pushed = True
        if _state["events"]:
            self.ev0 = torch.cuda.Event(enable_timing=True)
            self.ev1 = torch.cuda.Event(enable_timing=True)
            self.ev0.record()
        return self

    def __exit__(self, *exc):
        if self.ev0 is not None:
            self.ev1.record()
            _pending.append((_layer[0], self.name, self.ev0, self.ev1))
        if self.pushed:
            torch.cuda.nvtx.range_pop()
        return False


_NULL = contextlib.nullcontext()


def stage(name: str):
    """Context manager around one stage's launches (a no-op while recording is off)."""
    if not (_state["events"] or _state["nvtx"]):
        return _NULL
    return _Stage(name)


def _drain() -> None:
    if not _pending:
        return
    for _, _, _, ev1 in _pending:
        ev1.synchronize()
    for lay, name, ev0, ev1 in _pending:
        _times.setdefault(lay, {}).setdefault(name, []).append(float(ev0.elapsed_time(ev1)))
    _pending.clear()


def record(layer_idx: int, name: str, ms: float) -> None:
    """Add a time measured elsewhere (the reference's ``_record`` signature)."""
    _times.setdefault(int(layer_idx), {}).setdefault(name, []).append(float(ms))


def times() -> Dict[int, Dict[str, List[float]]]:
    """{layer: {stage: [ms per call]}}, after waiting for the recorded events."""
    _drain()
    return {lay: {s: list(v) for s, v in st.items()} for lay, st in _times.items()}


def _stage_order(tab) -> List[str]:
    seen = [s for s in STAGES if any(s in st for st in tab.values())]
    for st in tab.values():
        for s in st:
            if s not in seen:
                seen.append(s)
    return seen


def table(tab: Optional[Dict[int, Dict[str, List[float]]]] = None) -> dict:
    """Per-layer mean ms per stage, per-layer totals, and the per-stage mean over
    layers with and without layer 0 (its first call carries one-time set-up)."""
    tab = times() if tab is None else tab
    stages = _stage_order(tab)
    layers = sorted(tab)

    def mean(v):
        return sum(v) / len(v) if v else 0.0

    per_layer = {lay: {s: mean(tab[lay].get(s, [])) for s in stages} for lay in layers}
    totals = {lay: sum(per_layer[lay].values()) for lay in layers}

    def over(ls):
        return {s: (sum(per_layer[l][s] for l in ls) / len(ls) if ls else 0.0) for s in stages}

    rest = [l for l in layers if l != 0]
    return {"stages": stages, "per_layer": per_layer, "layer_total": totals,
            "mean": over(layers), "mean_excl_layer0": over(rest) if rest else None}


def summary(file=None) -> dict:
    """Print the per-layer stage table and return it (see ``table``)."""
    file = sys.stdout if file is None else file
    t = table()
    stages = t["stages"]
    head = "layer | " + " | ".join(f"{s:>12}" for s in stages) + " |        total"
    print(head, file=file)
    print("-" * len(head), file=file)
    for lay in sorted(t["per_layer"]):
        row = t["per_layer"][lay]
        print(f"{lay:>5} | " + " | ".join(f"{row[s]:12.4f}" for s in stages)
              + f" | {t['layer_total'][lay]:12.4f}", file=file)
    if t["per_layer"]:
        m = t["mean"]
        print(" mean | " + " | ".join(f"{m[s]:12.4f}" for s in stages)
              + f" | {sum(m.values()):12.4f}", file=file)
        if t["mean_excl_layer0"] is not None:
            m = t["mean_excl_layer0"]
            print("  >0  | " + " | ".join(f"{m[s]:12.4f}" for s in stages)
                  + f" | {sum(m.values()):12.4f}", file=file)
    return t


if os.environ.get("FFTS_TRACE", "") not in ("", "0"):
    enable()
