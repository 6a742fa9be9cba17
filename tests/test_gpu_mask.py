"""GPU parity of pooling and block-mask selection (bit-exact) against the CPU
oracle and the reference's golden masks."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.golden_cases import case_names, load_case

pytestmark = pytest.mark.gpu


def _bits_equal(a: torch.Tensor, b: torch.Tensor) -> bool:
    if a.dtype == torch.bfloat16:
        a, b = a.view(torch.int16), b.view(torch.int16)
    elif a.dtype == torch.float32:
        a, b = a.view(torch.int32), b.view(torch.int32)
    return bool(torch.equal(a, b))


@pytest.fixture(scope="module")
def lib():
    import fftsparse_b200
    fftsparse_b200.load_library()
    return fftsparse_b200


@pytest.mark.parametrize("name", case_names())
def test_mask_bit_exact(lib, name):
    spec, q, k, v, params, fx = load_case(name)
    ref = O.prefill_mask(q, k, params)
    m = lib.fft_block_mask(q.cuda(), k.cuda(), params=params)
    torch.cuda.synchronize()
    assert _bits_equal(m.q_pooled.cpu(), ref["qb"]), "pooled q differs from the oracle"
    assert _bits_equal(m.k_pooled.cpu(), ref["kb"]), "pooled k differs from the oracle"
    assert torch.equal(m.is_stripe.cpu(), ref["is_stripe"])
    assert _bits_equal(m.stripe_var.cpu(), ref["stripe_var"])
    if params.corr_on:
        assert _bits_equal(m.corr_sum.cpu(), ref["corr_sum"]), "FFT lag sums differ from the oracle"
        assert _bits_equal(m.corr.cpu(), ref["corr"]), "lag scores differ from the oracle"
    bits = m.bits.cpu()
    assert torch.equal(bits, ref["bits"]), "mask differs from the oracle"
    assert (O.as_numpy_bits(bits) == fx["mask"]).all(), "mask differs from the reference fixture"
    assert torch.equal(m.row_count.cpu(), ref["row_count"])
    dense = m.dense().cpu()
    assert torch.equal(dense, O.unpack_bits(ref["bits"], params.n_blocks))


def test_gqa_unexpanded_kv_gives_same_mask(lib):
    spec, q, k, v, params, fx = load_case("cfg2_topk")
    k_kv = k[:, ::4].contiguous()  # repeat_kv order: kv head g serves q heads 4g..4g+3
    m_exp = lib.fft_block_mask(q.cuda(), k.cuda(), params=params)
    m_kv = lib.fft_block_mask(q.cuda(), k_kv.cuda(), params=params)
    assert torch.equal(m_exp.bits, m_kv.bits)


def test_strided_inputs(lib):
    spec, q, k, v, params, fx = load_case("ragged_8269")
    # [B, L, H, D] storage viewed as [B, H, L, D]
    qs = q.transpose(1, 2).contiguous().cuda().transpose(1, 2)
    ks = k.transpose(1, 2).contiguous().cuda().transpose(1, 2)
    m = lib.fft_block_mask(qs, ks, params=params)
    assert (O.as_numpy_bits(m.bits.cpu()) == fx["mask"]).all()


def test_pool_odd_shapes(lib):
    g = torch.Generator().manual_seed(3)
    for dtype in (torch.bfloat16, torch.float32):
        for (B, H, L, D, bs) in [(2, 3, 1000, 128, 128), (1, 2, 77, 64, 32), (1, 1, 4096, 256, 64)]:
            x = torch.randn(B, H, L, D, generator=g).to(dtype)
            got = lib.pool_blocks(x.cuda(), bs).cpu()
            assert _bits_equal(got, O.pool(x, bs)), (dtype, B, H, L, D, bs)


def test_block_mask_rejects_bad_workspace(lib):
    import ctypes
    from fftsparse_b200 import _lib
    spec, q, k, v, params, fx = load_case("n10")
    qb = lib.pool_blocks(q.cuda(), 128)
    kb = lib.pool_blocks(k.cuda(), 128)
    L = _lib.load()
    B, H, N, D = qb.shape
    bits = torch.empty(B, H, N, 1, dtype=torch.int32, device="cuda")
    cp = params.to_c()
    rc = L.ffts_block_mask(qb.data_ptr(), kb.data_ptr(), 1, B, H, H, D, ctypes.addressof(cp), bits.data_ptr(),
                           None, None, None, None, None, None, 0, torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.FFTS_E_WORKSPACE
    assert b"workspace" in L.ffts_last_error_string()


@pytest.mark.slow
def test_mask_bit_exact_128k(lib):
    """BASELINE config 3 shape (L = 131072, 32 heads, bf16), keep ratio 0.05, against the
    oracle (lag scores bit-exact), and with a stripe threshold that splits the heads into
    stripe and diffuse.  The same mask is compared with the reference's own
    (cfg3_topk005_128k fixture) in test_mask_bit_exact."""
    from oracle.synth import make_inputs
    from fftsparse_b200.params import derive_mask_params
    L = 131072
    q, k, v = make_inputs(L, dtype=torch.bfloat16)
    kw = dict(sink_ratio=0.01, recent_ratio=0.0, local_span_ratio=0.02, correlation_selection_mode="topk",
              correlation_topk_ratio=0.05, qk_topk_ratio=0.05, column_topk_ratio=0.2)
    params = derive_mask_params(L, **kw)
    ref = O.prefill_mask(q, k, params)
    m = lib.fft_block_mask(q.cuda(), k.cuda(), params=params)
    assert torch.equal(m.bits.cpu(), ref["bits"])
    assert _bits_equal(m.corr.cpu(), ref["corr"])
    # mixed stripe / diffuse heads at full size
    params2 = derive_mask_params(L, **dict(kw, stripe_threshold=float(ref["stripe_var"].median())))
    ref2 = O.block_mask(ref["qb"], ref["kb"], params2, torch.bfloat16)
    m2 = lib.fft_block_mask(q.cuda(), k.cuda(), params=params2)
    assert 0 < int(ref2["is_stripe"].sum()) < 32
    assert torch.equal(m2.bits.cpu(), ref2["bits"])


@pytest.mark.slow
def test_mask_bit_exact_n2048(lib):
    """N = 2048 blocks (L = 262144): FFT length 4096 takes the shared-memory FFT, the column pass
    64-row chunks and the stripe statistics groups of at most 4 lags; stripe and diffuse heads."""
    from oracle.synth import make_inputs
    from fftsparse_b200.params import derive_mask_params
    L = 262144
    q, k, v = make_inputs(L, num_q_heads=4, num_kv_heads=1, dtype=torch.bfloat16)
    del v
    kw = dict(sink_ratio=0.01, recent_ratio=0.0, local_span_ratio=0.02, correlation_selection_mode="topk",
              correlation_topk_ratio=0.05, qk_topk_ratio=0.05, column_topk_ratio=0.2)
    params = derive_mask_params(L, **kw)
    assert params.n_blocks == 2048
    ref = O.prefill_mask(q, k, params)
    m = lib.fft_block_mask(q.cuda(), k.cuda(), params=params)
    assert torch.equal(m.bits.cpu(), ref["bits"])
    assert _bits_equal(m.corr.cpu(), ref["corr"])
    params2 = derive_mask_params(L, **dict(kw, stripe_threshold=float(ref["stripe_var"].median())))
    ref2 = O.block_mask(ref["qb"], ref["kb"], params2, torch.bfloat16)
    m2 = lib.fft_block_mask(q.cuda(), k.cuda(), params=params2)
    assert 0 < int(ref2["is_stripe"].sum()) < 4
    assert torch.equal(m2.bits.cpu(), ref2["bits"])


@pytest.mark.parametrize("name", case_names())
def test_csr_equals_dense_mask(lib, name):
    """The device-built CSR list (ffts_mask_row_ptr / ffts_mask_col_idx) equals the
    row-major nonzeros of the reference's bool block mask, ascending per row."""
    spec, q, k, v, params, fx = load_case(name)
    m = lib.fft_block_mask(q.cuda(), k.cuda(), params=params)
    row_ptr, col_idx = m.csr()
    N = params.n_blocks
    dense = O.unpack_bits(torch.from_numpy(fx["mask"].view("int32")), N).reshape(-1, N)
    nz = dense.nonzero()
    want_ptr = torch.zeros(dense.shape[0] + 1, dtype=torch.int64)
    want_ptr[1:] = torch.cumsum(dense.sum(1), 0)
    assert torch.equal(row_ptr.cpu(), want_ptr)
    assert torch.equal(col_idx.cpu().long(), nz[:, 1])


def test_csr_rejects_inconsistent_counts(lib):
    spec, q, k, v, params, fx = load_case("n10")
    m = lib.fft_block_mask(q.cuda(), k.cuda(), params=params)
    m.row_count[0, 0, 3] += 1  # no longer the popcount of its row
    with pytest.raises(RuntimeError):
        m.csr()
