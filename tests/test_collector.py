"""The calibration hook (myattn_prefill's ``_sparsity_collector``) against the
values the reference's own hook records (my_attn_v7.py:713-720), read from
tests/golden/collector.json (tests/golden/make_collector_golden.py):

* "corr": corr_mask_fraction recounted from the reference's own lag scores
  (the golden ``corr``) equals the reference's correlation-mask fraction exactly;
* "final": the kept fraction of the golden ``base_blockmask`` equals the
  reference's final fraction exactly;
* a case with the correlation mask off records no "corr" value.
"""
import json
import os

import numpy as np
import pytest
import torch

from fftsparse_b200.params import derive_mask_params
from fftsparse_b200.prefill import corr_mask_fraction

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
COLLECTED = json.load(open(os.path.join(HERE, "collector.json")))
MANIFEST = json.load(open(os.path.join(HERE, "manifest.json")))


@pytest.mark.parametrize("name", sorted(COLLECTED))
def test_hook_values_equal_reference(name):
    spec = MANIFEST[name]
    fx = np.load(os.path.join(HERE, f"{name}.npz"))
    params = derive_mask_params(spec["L"], block_size=spec["block_size"], **spec["kwargs"])
    want = COLLECTED[name]
    B = spec["batch"]
    if params.corr_on:
        got = [corr_mask_fraction(torch.from_numpy(fx["corr"][b:b + 1]), params) for b in range(B)]
        assert got == want["corr"]
    else:
        assert want["corr"] == []
    N = params.n_blocks
    bits = fx["mask"]  # [B, H, N, W] packed, bit j of row i = key block j
    kept = [int(np.unpackbits(bits[b].view(np.uint8), bitorder="little").sum()) for b in range(B)]
    H = bits.shape[1]
    assert [kk / (H * N * N) for kk in kept] == want["final"]
