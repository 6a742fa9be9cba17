"""End-to-end parity of the drop-in ``myattn_prefill`` against the oracle
(canonical mask + fp32 block-sparse attention)."""
import pytest
import torch

from oracle import oracle as O
from tests.golden_cases import load_case

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib():
    import fftsparse_b200
    fftsparse_b200.load_library()
    return fftsparse_b200


@pytest.mark.parametrize("name", ["defaults_4k", "mixed_16k", "bs64_4k", "ragged_8269", "batch2"])
def test_prefill_matches_oracle(lib, name):
    spec, q, k, v, params, fx = load_case(name)
    if q.dtype != torch.bfloat16:
        pytest.skip("attention runs in bf16")
    kw = dict(spec["kwargs"], block_size=spec["block_size"])
    out = lib.myattn_prefill(q.cuda(), k.cuda(), v.cuda(), 0, **kw)
    torch.cuda.synchronize()
    B, H, L, D = q.shape
    assert out.shape == (B, L, H * D) and out.dtype == torch.bfloat16
    got = out.view(B, L, H, D).permute(0, 2, 1, 3).float().cpu()
    mask = O.unpack_bits(torch.from_numpy(fx["mask"].view("int32")), params.n_blocks)
    heads = [0, H - 1]
    N = params.n_blocks
    rows = sorted({0, 1, N // 2, N - 2, N - 1})
    ref = O.sparse_attention(q, k, v, mask, params.block_size, heads=heads, rows=rows)
    bs = params.block_size
    for h in heads:
        for i in rows:
            sl = slice(i * bs, min(L, (i + 1) * bs))
            err = (got[:, h, sl] - ref[:, h, sl]).abs()
            assert float(err.max()) <= 2e-2 and float(err.mean()) <= 1e-3, (h, i, float(err.max()))


def test_short_sequence_uses_dense_causal(lib):
    g = torch.Generator().manual_seed(4)
    q = torch.randn(1, 4, 1000, 128, generator=g).bfloat16()
    k = torch.randn(1, 4, 1000, 128, generator=g).bfloat16()
    v = torch.randn(1, 4, 1000, 128, generator=g).bfloat16()
    out = lib.myattn_prefill(q.cuda(), k.cuda(), v.cuda(), 0)
    ref = torch.nn.functional.scaled_dot_product_attention(q.float(), k.float(), v.float(), is_causal=True)
    got = out.view(1, 1000, 4, 128).permute(0, 2, 1, 3).float().cpu()
    err = (got - ref).abs()
    assert float(err.max()) <= 2e-2 and float(err.mean()) <= 1e-3


def test_cpu_input_raises_assertion(lib):
    x = torch.zeros(1, 1, 2048, 128, dtype=torch.bfloat16)
    with pytest.raises(AssertionError):
        lib.myattn_prefill(x, x, x, 0)


def test_unknown_mode_raises_value_error(lib):
    x = torch.zeros(1, 1, 2048, 128, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        lib.myattn_prefill(x, x, x, 0, correlation_selection_mode="nope")


def test_config5_shape(lib):
    """BASELINE config 5 head shape: 2 sequences, 28 q-heads over 4 KV heads (groups of 7),
    block 64, keep ratio 0.05, un-expanded k/v; L reduced to 8192."""
    import bench
    from fftsparse_b200.params import derive_mask_params
    from oracle.synth import make_inputs
    L = 8192
    q, k, v = make_inputs(L, num_q_heads=28, num_kv_heads=4, dtype=torch.bfloat16, expand=False, batch=2, seed=5,
                          rope_base=1e6)
    kw = dict(bench.mask_kwargs(0.05), block_size=64)
    params = derive_mask_params(L, **kw)
    m = lib.fft_block_mask(q.cuda(), k.cuda(), **kw)
    ref = O.prefill_mask(q, k, params)
    assert torch.equal(m.bits.cpu(), ref["bits"])
    out = lib.myattn_prefill(q.cuda(), k.cuda(), v.cuda(), 0, **kw)
    torch.cuda.synchronize()
    got = out.view(2, L, 28, 128).permute(0, 2, 1, 3).float().cpu()
    mask = O.unpack_bits(ref["bits"], params.n_blocks)
    heads, rows = [0, 6, 27], [0, 37, params.n_blocks - 1]
    exp = O.sparse_attention(q, k, v, mask, 64, heads=heads, rows=rows)
    for h in heads:
        for i in rows:
            sl = slice(i * 64, (i + 1) * 64)
            err = (got[:, h, sl] - exp[:, h, sl]).abs()
            assert float(err.max()) <= 2e-2 and float(err.mean()) <= 1e-3, (h, i, float(err.max()))
