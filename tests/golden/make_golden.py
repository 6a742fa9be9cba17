"""Generate the golden block-mask fixtures from the reference implementation.

Run in a container that holds the reference checkout, named by
FFTS_REFERENCE_ROOT:

    python tests/golden/make_golden.py

For each case it builds seeded synthetic inputs (oracle/synth.py), runs the
reference's own ``myattn_prefill`` (attn_src/fft_attn/my_attn_v7.py) on the
CPU through oracle/ref_import.py with lowest-index tie-breaking, and stores:

  mask       packed bits uint32 [B, H, N, W] of ``base_blockmask``
  corr       the reference's fp32 lag scores (batch_fft_cross_correlation)
  corr_sum   the reference's raw fp32 lag sums
  pooled_sha sha256 of the reference's pooled Q_b / K_b bytes
  input_sha  sha256 of the generated q / k bytes (detects generator drift)
  raw_topk_agrees  whether the mask is unchanged with torch.topk's own tie order
  pooled_diff  per sequence, how many pooled q / k elements of the reference
             differ from the canonical pooling (fp32 sum of the block's rows in
             order, divided by block_size, rounded once; oracle.pool).  torch's
             CPU mean sums a large tensor in a different order, which moves a
             rare rounding boundary by one ulp.

Batch-2 cases run the reference once per sequence (it supports batch 1 only,
my_attn_v7.py:521, :528) and stack the results.
"""
from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from oracle.synth import make_inputs  # noqa: E402

# Efficiency-script settings (eval/efficiency/1_run_eval_multilayer.sh:46-63, :72).
EFF = dict(sink_ratio=0.01, recent_ratio=0.0, local_span_ratio=0.02, enable_column_mask=True,
           column_topk_ratio=0.2, enable_last_block_mask=True, diag_sample_ratio=0.15,
           min_diag_samples=5, max_diag_samples=64, stripe_threshold=0.3)


def keep_ratio(r):
    """Keep ratio r -> topk mode with correlation_topk_ratio = qk_topk_ratio = r."""
    return dict(correlation_selection_mode="topk", correlation_topk_ratio=r, corr_threshold=1.0,
                qk_topk_ratio=r)


def threshold(t):
    return dict(correlation_selection_mode="threshold", corr_threshold=t,
                correlation_topk_ratio=0.2, qk_topk_ratio=0.3)


CASES = {
    # 8K, fp32, keep ratio 0.1
    "cfg1_topk": dict(L=8192, dtype="fp32", kw={**EFF, **keep_ratio(0.1)}),
    "cfg1_thr090": dict(L=8192, dtype="fp32", kw={**EFF, **threshold(0.9)}),
    # 32K, bf16, keep ratio 0.05
    "cfg2_topk": dict(L=32768, dtype="bf16", kw={**EFF, **keep_ratio(0.05)}),
    "cfg2_thr090": dict(L=32768, dtype="bf16", kw={**EFF, **threshold(0.9)}),
    # mixed stripe / diffuse heads (threshold inside the statistic's spread)
    "mixed_16k": dict(L=16384, dtype="bf16", kw={**EFF, **keep_ratio(0.1), "stripe_threshold": 0.011}),
    # every head diffuse: per-row QK top-k
    "diffuse_8k": dict(L=8192, dtype="bf16", kw={**EFF, **keep_ratio(0.2), "stripe_threshold": 0.0}),
    "diffuse_fp32": dict(L=4096, dtype="fp32", kw={**EFF, **keep_ratio(0.3), "stripe_threshold": 0.0}),
    # ragged length (partial last block), N not a power of two
    "ragged_8269": dict(L=8192 + 77, dtype="bf16", kw={**EFF, **keep_ratio(0.1)}),
    "ragged_12800_mixed": dict(L=12800 - 5, dtype="bf16",
                               kw={**EFF, **keep_ratio(0.1), "stripe_threshold": 0.012}),
    # block size 64 (BASELINE config 5 granularity)
    "bs64_4k": dict(L=4096, dtype="bf16", bs=64, kw={**EFF, **keep_ratio(0.05)}),
    "bs32_2k": dict(L=2048, dtype="bf16", bs=32, kw={**EFF, **keep_ratio(0.1)}),
    # the reference's own defaults (my_attn_v7.py:454-489)
    "defaults_4k": dict(L=4096, dtype="bf16", kw={}),
    "defaults_6k_fp32": dict(L=6144 + 3, dtype="fp32", kw={}),
    # switches
    "no_corr": dict(L=8192, dtype="bf16", kw={**EFF, **keep_ratio(0.1), "enable_correlation_mask": False}),
    "no_col_no_last": dict(L=8192, dtype="bf16",
                           kw={**EFF, **keep_ratio(0.1), "enable_column_mask": False,
                               "enable_last_block_mask": False}),
    "corr_gate_off": dict(L=2560, dtype="bf16", kw={**EFF, **keep_ratio(0.1), "correlation_topk_ratio": 0.95}),
    # smallest sparse case (N = 10) and wide recent window
    "n10": dict(L=1280, dtype="bf16", kw={**EFF, **keep_ratio(0.1)}),
    "recent_wide": dict(L=8192, dtype="bf16", kw={**EFF, **keep_ratio(0.1), "recent_ratio": 0.1,
                                                   "local_span_ratio": 0.1}),
    # batch of two sequences (seeds 0 and 1)
    "batch2": dict(L=4096 + 100, dtype="bf16", batch=2, kw={**EFF, **keep_ratio(0.1),
                                                             "stripe_threshold": 0.012}),
    # BASELINE config 3 as bench.py runs it: 128K tokens, 32 / 8 heads, bf16, keep ratio 0.05
    "cfg3_topk005_128k": dict(L=131072, dtype="bf16", kw={**EFF, **keep_ratio(0.05)}),
    # BASELINE config 5's attention shape: 2 x 65536 tokens, 28 / 4 heads, block 64, RoPE base 1e6
    "cfg5_qwen_bs64_2x64k": dict(L=65536, dtype="bf16", bs=64, batch=2, hq=28, hkv=4, rope_base=1e6,
                                 kw={**EFF, **keep_ratio(0.05)}),
}

DT = {"fp32": torch.float32, "bf16": torch.bfloat16}


def sha(t: torch.Tensor) -> str:
    t = t.contiguous()
    if t.dtype == torch.bfloat16:
        t = t.view(torch.int16)
    return hashlib.sha256(t.numpy().tobytes()).hexdigest()


def pack(mask: np.ndarray) -> np.ndarray:
    n = mask.shape[-1]
    W = (n + 31) // 32
    m = np.zeros(mask.shape[:-1] + (W * 32,), dtype=np.uint8)
    m[..., :n] = mask
    return np.packbits(m, axis=-1, bitorder="little").view(np.uint32)


def input_kwargs(spec):
    """make_inputs arguments of a case (head counts and RoPE base default to config 1-3's)."""
    return dict(dtype=DT[spec["dtype"]], batch=spec.get("batch", 1), num_q_heads=spec.get("hq", 32),
                num_kv_heads=spec.get("hkv", 8), rope_base=spec.get("rope_base", 500000.0))


def case_inputs(spec):
    return make_inputs(spec["L"], **input_kwargs(spec))


def main(names=None):
    from oracle import oracle as O
    from oracle.ref_import import reference_intermediates, run_reference

    manifest = {}
    for name, spec in CASES.items():
        if names and name not in names:
            continue
        bs = spec.get("bs", 128)
        kw = dict(spec["kw"], block_size=bs)
        q, k, v = case_inputs(spec)
        masks, corrs, sums, psha, pdiff = [], [], [], [], []
        raw_agree = True
        for b in range(q.shape[0]):
            qb, kb, vb = q[b:b + 1], k[b:b + 1], v[b:b + 1]
            m, _ = run_reference(qb, kb, vb, stable_topk=True, **kw)
            m_raw, _ = run_reference(qb, kb, vb, stable_topk=False, **kw)
            raw_agree &= bool(torch.equal(m, m_raw))
            inter = reference_intermediates(
                qb, kb, block_size=bs, sink_ratio=kw.get("sink_ratio", 0.1),
                recent_ratio=kw.get("recent_ratio", 0.1),
                local_span_ratio=kw.get("local_span_ratio", 0.1))
            masks.append(pack(m[0].numpy().astype(np.uint8)))
            corrs.append(inter["corr"].numpy())
            sums.append(inter["corr_sum"].numpy())
            psha.append(sha(inter["Qb"]) + ":" + sha(inter["Kb"]))
            diff = 0
            for x, ref in ((qb, inter["Qb"]), (kb, inter["Kb"])):
                canon = O.pool(x, bs)[0].permute(1, 0, 2)  # [N, H, D], the reference's layout
                diff += int((canon.float() != ref.float()).sum())
            pdiff.append(diff)
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), mask=np.stack(masks),
                            corr=np.stack(corrs).astype(np.float32),
                            corr_sum=np.stack(sums).astype(np.float32))
        manifest[name] = dict(L=spec["L"], dtype=spec["dtype"], block_size=bs,
                              batch=q.shape[0], kwargs=spec["kw"], input_sha=sha(q) + ":" + sha(k),
                              hq=q.shape[1], hkv=spec.get("hkv", 8), rope_base=spec.get("rope_base", 500000.0),
                              pooled_sha=psha, pooled_diff=pdiff, raw_topk_agrees=raw_agree,
                              density=float(np.mean([np.unpackbits(mm.view(np.uint8)).mean() for mm in masks])))
        print(name, "N=", (spec["L"] + bs - 1) // bs, "raw topk agrees:", raw_agree, flush=True)
    path = os.path.join(HERE, "manifest.json")
    old = json.load(open(path)) if (names and os.path.exists(path)) else {}
    old.update(manifest)
    with open(path, "w") as f:
        json.dump(old, f, indent=1, sort_keys=True)


if __name__ == "__main__":
    main(sys.argv[1:] or None)
