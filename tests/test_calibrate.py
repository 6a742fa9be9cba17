"""On-device calibration (fftsparse_b200.calibrate.calibrate_from_qk) against
the reference's bisection (eval/efficiency/benchmark_attention_multilayer.py:
179-262) restated as plain host code over the reference's measured quantity,
the mean correlation-mask kept fraction of the layers (corr_mask_fraction,
pinned to the reference's hook values by tests/test_collector.py).  The mask
selection runs on the CPU oracle here; the bisection under test is the same
tensor code the GPU runs."""
from types import SimpleNamespace

import pytest
import torch

import fftsparse_b200.calibrate as C
from fftsparse_b200.params import derive_mask_params
from fftsparse_b200.prefill import corr_mask_fraction
from oracle import oracle as O
from oracle.synth import make_inputs


def reference_bisection(fraction_of, target, topk, steps=20, tol=0.01):
    """calibrate_from_qk's loop (:233-253) over a value -> mean fraction function."""
    lo, hi, best = 0.0, 1.0, 0.5
    for _ in range(steps):
        mid = (lo + hi) / 2
        f = fraction_of(mid)
        if abs(f - target) < tol:
            best = mid
            break
        if (f > target) == topk:
            hi = mid
        else:
            lo = mid
        best = mid
    return best


def oracle_mask(q, k, block_size=128, **kw):
    params = derive_mask_params(q.shape[2], block_size=block_size, **kw)
    m = O.prefill_mask(q, k, params)
    return SimpleNamespace(params=params, corr=m["corr"], row_count=m["row_count"])


@pytest.fixture(scope="module")
def layers():
    out = []
    for seed, L in ((0, 8192), (1, 6144 + 40), (2, 8192)):
        q, k, _ = make_inputs(L, num_q_heads=4, num_kv_heads=2, dtype=torch.bfloat16, expand=False, seed=seed)
        out.append((q, k))
    return out


KW = dict(sink_ratio=0.01, recent_ratio=0.0, local_span_ratio=0.02, stripe_threshold=0.3, qk_topk_ratio=0.1)


@pytest.mark.parametrize("mode,target", [("topk", 0.05), ("topk", 0.2), ("threshold", 0.05), ("threshold", 0.3),
                                         ("topk", 0.9)])
def test_device_bisection_equals_reference_loop(monkeypatch, layers, mode, target):
    monkeypatch.setattr(C, "fft_block_mask", oracle_mask)
    topk = mode == "topk"
    corrs = [oracle_mask(q, k, correlation_selection_mode=mode, correlation_topk_ratio=0.0 if topk else 0.2,
                         **KW) for q, k in layers]

    def fraction_of(val):
        fr = []
        for (q, k), m in zip(layers, corrs):
            p = derive_mask_params(q.shape[2], block_size=128, correlation_selection_mode=mode,
                                   correlation_topk_ratio=val if topk else 0.2,
                                   corr_threshold=1.0 if topk else val, **KW)
            if p.corr_on:
                fr.append(corr_mask_fraction(m.corr, p))
        return sum(fr) / len(fr) if fr else float("nan")

    want = reference_bisection(fraction_of, target, topk)
    best, corr_ret, final_ret = C.calibrate_from_qk(layers, target, correlation_selection_mode=mode, **KW)
    assert best == want
    assert corr_ret == pytest.approx(fraction_of(best), abs=0, rel=1e-12)
    assert 0.0 < final_ret <= 1.0


def test_rejects_unknown_mode(layers):
    with pytest.raises(ValueError):
        C.calibrate_from_qk(layers, 0.1, correlation_selection_mode="bogus")
