"""Pin the CPU oracle against the reference's own outputs (golden fixtures).

The fixtures were produced by tests/golden/make_golden.py, which runs the
reference's attn_src/fft_attn/my_attn_v7.py on the CPU.  These tests need no
GPU and no reference checkout.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.golden_cases import case_names, load_case, sha

CASES = case_names(large=False)
LARGE = case_names(large=True)


@pytest.mark.parametrize("name", CASES)
def test_inputs_match_fixture_generator(name):
    spec, q, k, v, params, fx = load_case(name)
    assert sha(q) + ":" + sha(k) == spec["input_sha"], "synthetic generator drifted"


@pytest.mark.parametrize("name", CASES)
def test_oracle_mask_bit_exact_vs_reference(name):
    spec, q, k, v, params, fx = load_case(name)
    out = O.prefill_mask(q, k, params)
    got = O.as_numpy_bits(out["bits"])
    want = fx["mask"]
    assert got.shape == want.shape
    mismatched_rows = int((got != want).any(-1).sum())
    assert mismatched_rows == 0, f"{mismatched_rows} rows differ from the reference mask"


@pytest.mark.parametrize("name", CASES)
def test_oracle_corr_within_tolerance(name):
    # FFT lag scores: |oracle - reference| <= 1e-4 * max|reference| (fp32 FFTs of
    # different factorisations agree to ~1e-6 relative).
    spec, q, k, v, params, fx = load_case(name)
    if not params.corr_on:
        pytest.skip("correlation mask disabled in this case")
    out = O.prefill_mask(q, k, params)
    ref = torch.from_numpy(fx["corr"])
    got = out["corr"]
    scale = max(1.0, float(ref.abs().max()))
    assert float((got - ref).abs().max()) <= 1e-4 * scale
    ref_sum = torch.from_numpy(fx["corr_sum"])
    scale = max(1.0, float(ref_sum.abs().max()))
    assert float((out["corr_sum"] - ref_sum).abs().max()) <= 1e-4 * scale


@pytest.mark.parametrize("name", LARGE)
def test_large_case_against_reference(name):
    """BASELINE config 3 (128K tokens, 32 / 8 heads, keep ratio 0.05) and config 5's
    attention shape (2 x 65536, 28 / 4 heads, block 64): the oracle's mask equals
    the reference's bit for bit and its lag scores are within 1e-4.  The pooled
    bytes are not compared here: at this size torch's CPU mean sums in another
    order, which the generator measured as a one-ulp change in a handful of the
    millions of pooled elements (manifest ``pooled_diff``); the masks agree anyway."""
    spec, q, k, v, params, fx = load_case(name)
    assert sha(q) + ":" + sha(k) == spec["input_sha"], "synthetic generator drifted"
    assert sum(spec["pooled_diff"]) <= 16
    out = O.prefill_mask(q, k, params)
    got = O.as_numpy_bits(out["bits"])
    assert got.shape == fx["mask"].shape
    mismatched_rows = int((got != fx["mask"]).any(-1).sum())
    assert mismatched_rows == 0, f"{mismatched_rows} rows differ from the reference mask"
    ref = torch.from_numpy(fx["corr"])
    assert float((out["corr"] - ref).abs().max()) <= 1e-4 * max(1.0, float(ref.abs().max()))


@pytest.mark.parametrize("name", [n for n in CASES if n.endswith(("topk", "8k", "16k"))])
def test_bf16_pooling_matches_reference_bytes(name):
    spec, q, k, v, params, fx = load_case(name)
    if spec["dtype"] != "bf16":
        pytest.skip("fp32 pooling differs from torch in the last ulp by design")
    qb = O.pool(q, params.block_size)
    kb = O.pool(k, params.block_size)
    got = [sha(qb[b].permute(1, 0, 2)) + ":" + sha(kb[b].permute(1, 0, 2)) for b in range(q.shape[0])]
    assert got == spec["pooled_sha"]


def test_fp32_pooling_close_to_mean():
    torch.manual_seed(0)
    x = torch.randn(1, 4, 1000, 128)
    got = O.pool(x, 128)
    pad = torch.nn.functional.pad(x, (0, 0, 0, 24))
    ref = pad.view(1, 4, 8, 128, 128).double().mean(dim=3).float()
    assert float((got - ref).abs().max()) < 1e-6


def test_pack_unpack_roundtrip():
    m = torch.rand(2, 3, 70, 70) > 0.5
    assert torch.equal(O.unpack_bits(O.pack_bool(m), 70), m)


def test_attention_oracle_dense_matches_sdpa():
    torch.manual_seed(0)
    q = torch.randn(1, 2, 300, 64)
    k = torch.randn(1, 2, 300, 64)
    v = torch.randn(1, 2, 300, 64)
    N = 3
    mask = torch.ones(1, 2, N, N, dtype=torch.bool)
    got = O.sparse_attention(q, k, v, mask, 128, causal=True)
    ref = torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=True)
    assert float((got - ref).abs().max()) < 1e-5


def test_attention_oracle_empty_rows_are_zero():
    q = torch.randn(1, 1, 256, 64)
    k = torch.randn(1, 1, 256, 64)
    v = torch.randn(1, 1, 256, 64)
    mask = torch.zeros(1, 1, 2, 2, dtype=torch.bool)
    mask[0, 0, 1, 0] = True
    got = O.sparse_attention(q, k, v, mask, 128, causal=True)
    assert float(got[0, 0, :128].abs().max()) == 0.0
    s = (q[0, 0, 128:] @ k[0, 0, :128].T) / 8.0
    ref = torch.softmax(s, -1) @ v[0, 0, :128]
    assert float((got[0, 0, 128:] - ref).abs().max()) < 1e-5
