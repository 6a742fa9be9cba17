"""The allocation-free mask selection entry point (ffts_block_mask_noalloc).

Some callers of this library may not allocate device memory while they run the
selection (an engine that owns all GPU memory through its own pool, or a plugin
hook where cudaMalloc could synchronise the device), so they cannot pass the
workspace ffts_block_mask asks for.  This entry point runs the same kernels on
a fixed scratch array inside the library.  These tests call it through the C
ABI and require results identical to ffts_block_mask (the selection is
bit-exact, so the tolerance is zero) on two calls in a row, the second one
running over the scratch the first one left behind.

The file is named to be collected last, so a failure here does not stop a
``-x`` run before every other test has run.
"""
import ctypes

import pytest
import torch

from oracle import oracle as O
from tests.golden_cases import load_case

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def F():
    import fftsparse_b200
    fftsparse_b200.load_library()
    return fftsparse_b200


def _outputs(B, H, N, dev):
    W = (N + 31) // 32
    return {
        "bits": torch.full((B, H, N, W), 0x5A5A5A5A, dtype=torch.int32, device=dev),
        "row_count": torch.full((B, H, N), -7, dtype=torch.int32, device=dev),
        "corr": torch.full((B, H, N), float("nan"), device=dev),
        "corr_sum": torch.full((B, H, N), float("nan"), device=dev),
        "is_stripe": torch.full((B, H), 9, dtype=torch.uint8, device=dev),
        "stripe_var": torch.full((B, H), float("nan"), device=dev),
    }


def _ptrs(o):
    return [o[k].data_ptr() for k in ("bits", "row_count", "corr", "corr_sum", "is_stripe", "stripe_var")]


def _run_both(F, name):
    from fftsparse_b200 import _lib
    lib = _lib.load()
    spec, q, k, v, params, fx = load_case(name)
    dev = torch.device("cuda")
    qb = F.pool_blocks(q.to(dev), params.block_size)
    kb = F.pool_blocks(k.to(dev), params.block_size)
    B, H, N, D = qb.shape
    Hkv = kb.shape[1]
    dtype = 1 if q.dtype == torch.bfloat16 else 0
    cp = params.to_c()
    stream = torch.cuda.current_stream().cuda_stream

    ref = _outputs(B, H, N, dev)
    ws_bytes = int(lib.ffts_mask_workspace_bytes(B, H, N, D))
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
    rc = lib.ffts_block_mask(qb.data_ptr(), kb.data_ptr(), dtype, B, H, Hkv, D, ctypes.addressof(cp),
                             *_ptrs(ref), ws.data_ptr(), ws_bytes, stream)
    assert rc == 0, lib.ffts_last_error_string()

    got = _outputs(B, H, N, dev)
    rc = lib.ffts_block_mask_noalloc(qb.data_ptr(), kb.data_ptr(), dtype, B, H, Hkv, D, ctypes.addressof(cp),
                                     *_ptrs(got), stream)
    assert rc == 0, lib.ffts_last_error_string()
    torch.cuda.synchronize()
    for key in ref:
        a, b = ref[key], got[key]
        if a.is_floating_point():
            a, b = a.view(torch.int32), b.view(torch.int32)
        assert torch.equal(a, b), f"{name}: {key} differs between ffts_block_mask and ffts_block_mask_noalloc"


def test_noalloc_matches_workspace_entry_point_on_two_calls(F):
    # first call: 32K tokens, 32 heads, all stripe heads (FFT lag path)
    _run_both(F, "cfg2_topk")
    # second call, different shape and diffuse heads, over the scratch left by the first
    _run_both(F, "mixed_16k")


def test_noalloc_call_allocates_nothing(F):
    """After a first call (which loads the library's code and scratch onto the
    device), a call takes no device memory: neither torch's allocator nor the
    device's free total moves."""
    from fftsparse_b200 import _lib
    lib = _lib.load()
    spec, q, k, v, params, fx = load_case("mixed_16k")
    dev = torch.device("cuda")
    qb = F.pool_blocks(q.to(dev), params.block_size)
    kb = F.pool_blocks(k.to(dev), params.block_size)
    B, H, N, D = qb.shape
    cp = params.to_c()
    stream = torch.cuda.current_stream().cuda_stream
    out = _outputs(B, H, N, dev)
    args = (qb.data_ptr(), kb.data_ptr(), 1, B, H, kb.shape[1], D, ctypes.addressof(cp), *_ptrs(out), stream)
    assert lib.ffts_block_mask_noalloc(*args) == 0, lib.ffts_last_error_string()
    torch.cuda.synchronize()
    torch_bytes = torch.cuda.memory_allocated(dev)
    free_before = torch.cuda.mem_get_info(dev)[0]
    assert lib.ffts_block_mask_noalloc(*args) == 0, lib.ffts_last_error_string()
    torch.cuda.synchronize()
    assert torch.cuda.memory_allocated(dev) == torch_bytes
    assert torch.cuda.mem_get_info(dev)[0] == free_before, "ffts_block_mask_noalloc allocated device memory"
    assert (O.as_numpy_bits(out["bits"].cpu()) == fx["mask"]).all()


def test_noalloc_rejects_shapes_beyond_its_scratch(F):
    from fftsparse_b200 import _lib
    from fftsparse_b200.params import derive_mask_params
    lib = _lib.load()
    dev = torch.device("cuda")
    B, H, D, L = 1, 32, 128, 4096 * 128  # N = 4096 blocks needs ~16.8 MB of scratch
    params = derive_mask_params(L, sink_ratio=0.01, recent_ratio=0.0, local_span_ratio=0.02)
    N = params.n_blocks
    qb = torch.zeros(B, H, N, D, dtype=torch.bfloat16, device=dev)
    out = _outputs(B, H, N, dev)
    before = out["bits"].clone()
    cp = params.to_c()
    rc = lib.ffts_block_mask_noalloc(qb.data_ptr(), qb.data_ptr(), 1, B, H, H, D, ctypes.addressof(cp),
                                     *_ptrs(out), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert rc == _lib.FFTS_E_WORKSPACE
    msg = lib.ffts_last_error_string().decode()
    assert "scratch" in msg and str(8 << 20) in msg
    assert torch.equal(out["bits"], before), "a rejected call must not launch any kernel"
