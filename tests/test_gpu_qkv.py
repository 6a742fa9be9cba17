"""GPU parity of ffts_qkv_rope_pool, the QKV projection GEMM with RoPE, the
head-major layout and the q/k pooling in its epilogue.

The projection it computes (returned on request) is checked against an fp32
evaluation of x W^T (+ bias): every element within one bf16 rounding step of
it, and nearly all equal to its bf16 rounding.  Everything after the
projection is integer-exact work on bf16 values: the rotated head-major q/k,
the head-major v and the pooled blocks must equal, bit for bit, the CPU
oracle's RoPE + pooling (and the rope_pool kernel) applied to that projection.
"""
import pytest
import torch

from oracle import oracle as O
from tests.test_rope_oracle import rope_tables

pytestmark = pytest.mark.gpu

D = 128


@pytest.fixture(scope="module")
def F():
    import fftsparse_b200
    fftsparse_b200.load_library()
    return fftsparse_b200


def _inputs(B, L, K, Hq, Hkv, with_bias, seed):
    g = torch.Generator().manual_seed(seed)
    heads = Hq + 2 * Hkv
    x = torch.randn(B, L, K, generator=g).bfloat16()
    w = (torch.randn(heads * D, K, generator=g) * K ** -0.5).bfloat16()
    bias = (torch.randn(heads * D, generator=g) * 0.1).bfloat16() if with_bias else None
    return x, w, bias


def _bound(x, w, bias):
    """The fp32 product and a bound on a bf16 result's distance from it: one bf16
    step at the value (2^-7 relative, an upper bound on the ulp) plus 2^-16 of the
    sum of the terms' magnitudes (covers any fp32 summation order)."""
    xd, wd = x.cuda().float(), w.cuda().float()
    ref = torch.matmul(xd, wd.T)
    mag = torch.matmul(xd.abs(), wd.abs().T)
    if bias is not None:
        ref = ref + bias.cuda().float()
        mag = mag + bias.cuda().float().abs()
    return ref, ref.abs() * 2.0 ** -7 + mag * 2.0 ** -16


def _check_projection(proj, x, w, bias):
    """proj (bf16) against the fp32 product: within the bound everywhere, equal to
    the product's bf16 rounding for all but a sliver of elements (the fp32
    accumulation order differs from the reference evaluation's)."""
    ref, tol = _bound(x, w, bias)
    err = (proj.float() - ref).abs()
    assert bool((err <= tol).all()), float((err / tol).max())
    mismatch = (proj != ref.bfloat16()).float().mean().item()
    assert mismatch < 0.02, mismatch


CASES = [
    # B, L, K, Hq, Hkv, block_size, bias
    (1, 1000, 512, 4, 2, 128, False),    # ragged last tile and block
    (2, 777, 256, 3, 1, 64, True),       # two sequences; 5 heads = 2.5 column tiles
    (1, 300, 128, 1, 1, 16, True),       # two K steps, block 16
    (1, 513, 200, 2, 1, 32, False),      # K not a multiple of 64 (zero-filled tail)
    (1, 2048, 3584, 28, 4, 64, True),    # Qwen2.5-7B projection shape
]


@pytest.mark.parametrize("B,L,K,Hq,Hkv,bs,with_bias", CASES)
def test_qkv_rope_pool_equals_oracle_on_its_projection(F, B, L, K, Hq, Hkv, bs, with_bias):
    x, w, bias = _inputs(B, L, K, Hq, Hkv, with_bias, seed=L + K + Hq)
    cos, sin = rope_tables(L)
    xd, wd, cd, sd = x.cuda(), w.cuda(), cos.cuda(), sin.cuda()
    bd = None if bias is None else bias.cuda()
    q, k, v, qb, kb, proj = F.qkv_rope_pool(xd, wd, bd, Hq, Hkv, cd, sd, bs, return_projection=True)
    torch.cuda.synchronize()
    F.check_status()
    _check_projection(proj, x, w, bias)
    pc = proj.cpu()
    for b in range(B):
        srcs = (pc[b, :, :Hq * D], pc[b, :, Hq * D:(Hq + Hkv) * D], pc[b, :, (Hq + Hkv) * D:])
        ref = O.rope_pool(srcs[0], srcs[1], srcs[2], Hq, Hkv, cos, sin, bs)
        for name, r, got in zip(("q", "k", "v", "q_pooled", "k_pooled"), ref, (q, k, v, qb, kb)):
            assert torch.equal(got[b:b + 1].cpu(), r), (name, b)
    # without the projection output the kernel computes the same values
    again = F.qkv_rope_pool(xd, wd, bd, Hq, Hkv, cd, sd, bs)
    for a, g in zip(again, (q, k, v, qb, kb)):
        assert torch.equal(a, g)


def test_qkv_rope_pool_llama_shape_against_rope_pool_and_cublas(F):
    """Llama-3.1-8B projection shape (hidden 4096, 32 / 8 heads) at 8K tokens: the
    fused outputs equal rope_pool on the kernel's own projection, and that
    projection is within one bf16 step of cuBLAS's bf16 product."""
    B, L, K, Hq, Hkv, bs = 1, 8192, 4096, 32, 8, 128
    x, w, _ = _inputs(B, L, K, Hq, Hkv, False, seed=11)
    cos, sin = (t.cuda() for t in rope_tables(L))
    xd, wd = x.cuda(), w.cuda()
    q, k, v, qb, kb, proj = F.qkv_rope_pool(xd, wd, None, Hq, Hkv, cos, sin, bs, return_projection=True)
    ref = F.rope_pool(proj[0, :, :Hq * D], proj[0, :, Hq * D:(Hq + Hkv) * D], proj[0, :, (Hq + Hkv) * D:],
                      Hq, Hkv, cos, sin, bs)
    torch.cuda.synchronize()
    F.check_status()
    for name, r, got in zip(("q", "k", "v", "q_pooled", "k_pooled"), ref, (q, k, v, qb, kb)):
        assert torch.equal(got, r), name
    _check_projection(proj, x, w, None)
    cub = torch.matmul(xd[0], wd.T)  # cuBLAS, bf16 out
    _, tol = _bound(x[0], w, None)
    assert bool(((proj[0].float() - cub.float()).abs() <= 2 * tol).all())
    assert (proj[0] != cub).float().mean().item() < 0.02


def test_qkv_rope_pool_rejects_bad_arguments(F):
    x = torch.zeros(1, 256, 128, dtype=torch.bfloat16, device="cuda")
    cos, sin = (t.cuda() for t in rope_tables(256))
    with pytest.raises(ValueError):
        F.qkv_rope_pool(x, torch.zeros(3 * D, 64, dtype=torch.bfloat16, device="cuda"), None, 1, 1, cos, sin)
    w = torch.zeros(3 * D, 128, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):  # block_size 256 is outside what the epilogue pools
        F.qkv_rope_pool(x, w, None, 1, 1, cos, sin, 256)
    # through the C ABI: a workspace smaller than ffts_qkv_workspace_bytes(L) is refused, nothing runs
    from fftsparse_b200 import _lib
    lib = _lib.load()
    need = int(lib.ffts_qkv_workspace_bytes(256))
    assert need == 256 * D * 2 * 2
    outs = [torch.empty(1, 1, 256, D, dtype=torch.bfloat16, device="cuda") for _ in range(3)]
    pooled = [torch.empty(1, 1, 2, D, dtype=torch.bfloat16, device="cuda") for _ in range(2)]
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.ffts_qkv_rope_pool(x.data_ptr(), 1, 256, 128, 128, 256 * 128, w.data_ptr(), 128, None, 1, 1, D,
                                cos.data_ptr(), sin.data_ptr(), D, 128, *[t.data_ptr() for t in outs],
                                *[t.data_ptr() for t in pooled], None, 0, ws.data_ptr(), need - 16, None, stream)
    assert rc == _lib.FFTS_E_WORKSPACE
