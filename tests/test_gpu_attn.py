"""GPU parity of the tcgen05 block-sparse attention kernel against the fp32 CPU
oracle.  Tolerance (bf16 inputs and output): max |err| <= 2e-2 and
mean |err| <= 1e-3."""
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
MEAN_ABS = 1e-3


@pytest.fixture(scope="module")
def lib():
    import fftsparse_b200
    fftsparse_b200.load_library()
    return fftsparse_b200


def random_mask(B, H, N, density, gen, diag=True):
    m = torch.rand(B, H, N, N, generator=gen) < density
    m &= torch.ones(N, N, dtype=torch.bool).tril()
    if diag:
        m |= torch.eye(N, dtype=torch.bool)
    return m


def run_case(lib, B, H, Hkv, L, bs, density, seed=0, causal=True, empty_rows=False, heads=None, rows=None):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, H, L, 128, generator=g).bfloat16()
    k = torch.randn(B, Hkv, L, 128, generator=g).bfloat16()
    v = torch.randn(B, Hkv, L, 128, generator=g).bfloat16()
    N = (L + bs - 1) // bs
    mask = random_mask(B, H, N, density, g, diag=not empty_rows)
    if empty_rows:
        mask[:, :, ::3] = False
    bits = O.pack_bool(mask)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = lib.sparse_attention(q.cuda(), k.cuda(), v.cuda(), bits.cuda(), bs, causal=causal, status=status)
    torch.cuda.synchronize()
    assert int(status.item()) == 0, "kernel reported a wait time-out"
    got = out.float().cpu().permute(0, 2, 1, 3)  # [B, H, L, D]
    ref = O.sparse_attention(q, k, v, mask, bs, causal=causal, heads=heads, rows=rows)
    if heads is not None or rows is not None:
        sel = torch.zeros(B, H, L, dtype=torch.bool)
        for h in (range(H) if heads is None else heads):
            for i in (range(N) if rows is None else rows):
                sel[:, h, i * bs:(i + 1) * bs] = True
        got, ref = got[sel], ref[sel]
    err = (got - ref).abs()
    assert float(err.max()) <= MAX_ABS, float(err.max())
    assert float(err.mean()) <= MEAN_ABS, float(err.mean())
    return got, ref


def test_tiny_single_tile(lib):
    run_case(lib, 1, 1, 1, 128, 128, 1.0)


def test_two_tiles_dense(lib):
    run_case(lib, 1, 2, 2, 256, 128, 1.0)


@pytest.mark.parametrize("bs", [128, 64, 32])
def test_random_masks(lib, bs):
    run_case(lib, 1, 4, 4, 2048, bs, 0.3, seed=bs)


def test_ragged_length(lib):
    run_case(lib, 1, 2, 2, 1000 + 37, 128, 0.5, seed=7)


def test_gqa_and_batch(lib):
    run_case(lib, 2, 8, 2, 1536, 128, 0.25, seed=11)


def test_empty_rows_are_zero(lib):
    got, ref = run_case(lib, 1, 2, 2, 1024, 128, 0.4, seed=5, empty_rows=True)
    assert float(ref[..., :128, :].abs().max()) == 0.0


def test_non_causal_flag(lib):
    run_case(lib, 1, 2, 2, 768, 128, 0.5, seed=9, causal=False)


def test_long_rows_subset(lib):
    # 8K tokens, 64 key tiles per row at most; check 2 heads x 6 query blocks.
    run_case(lib, 1, 4, 1, 8192, 128, 0.2, seed=13, heads=[0, 3], rows=[0, 1, 17, 40, 62, 63])


def test_dense_matches_sdpa(lib):
    g = torch.Generator().manual_seed(1)
    L = 2048 + 64
    q = torch.randn(1, 4, L, 128, generator=g).bfloat16().cuda()
    k = torch.randn(1, 4, L, 128, generator=g).bfloat16().cuda()
    v = torch.randn(1, 4, L, 128, generator=g).bfloat16().cuda()
    N = (L + 127) // 128
    bits = torch.full((1, 4, N, (N + 31) // 32), -1, dtype=torch.int32, device="cuda")
    out = lib.sparse_attention(q, k, v, bits, 128).float().permute(0, 2, 1, 3)
    ref = torch.nn.functional.scaled_dot_product_attention(q.float(), k.float(), v.float(), is_causal=True)
    err = (out - ref).abs()
    assert float(err.max()) <= MAX_ABS and float(err.mean()) <= MEAN_ABS


def test_output_layout_and_strides(lib):
    g = torch.Generator().manual_seed(2)
    B, H, L = 1, 4, 512
    base = torch.randn(B, L, H, 128, generator=g).bfloat16().cuda()
    q = base.transpose(1, 2)  # non-contiguous [B, H, L, D] view
    k = torch.randn(B, H, L, 128, generator=g).bfloat16().cuda()
    v = torch.randn(B, H, L, 128, generator=g).bfloat16().cuda()
    N = L // 128
    bits = torch.full((B, H, N, 1), -1, dtype=torch.int32, device="cuda")
    out = lib.sparse_attention(q, k, v, bits, 128)
    ref = lib.sparse_attention(q.contiguous(), k, v, bits, 128)
    assert torch.equal(out, ref)


def test_rejects_fp32(lib):
    x = torch.zeros(1, 1, 128, 128, device="cuda")
    bits = torch.full((1, 1, 1, 1), -1, dtype=torch.int32, device="cuda")
    with pytest.raises(TypeError):
        lib.sparse_attention(x, x, x, bits, 128)


def test_repeated_calls_are_deterministic(lib):
    # every run of the kernel must produce identical bits (guards against
    # pipeline races that only show up intermittently)
    g = torch.Generator().manual_seed(21)
    B, H, L, bs = 1, 8, 4096, 128
    q = torch.randn(B, H, L, 128, generator=g).bfloat16().cuda()
    k = torch.randn(B, H, L, 128, generator=g).bfloat16().cuda()
    v = torch.randn(B, H, L, 128, generator=g).bfloat16().cuda()
    N = L // bs
    mask = random_mask(B, H, N, 0.3, g)
    bits = O.pack_bool(mask).cuda()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    first = lib.sparse_attention(q, k, v, bits, bs, status=status)
    for _ in range(50):
        assert torch.equal(lib.sparse_attention(q, k, v, bits, bs, status=status), first)
    assert int(status.item()) == 0, "kernel reported a wait time-out"


@pytest.mark.slow
def test_max_tiles_subset(lib):
    # L = 262144: 4096 key tiles of 64, the largest tile bitmask the kernel takes; check 3 query blocks
    run_case(lib, 1, 2, 1, 262144, 128, 0.02, seed=17, heads=[1], rows=[0, 1000, 2047])


def test_row_range_equals_full_call(lib):
    # ffts_sparse_attn_fwd_rows computes exactly the rows of the whole call it covers
    g = torch.Generator().manual_seed(23)
    B, H, L, bs = 1, 4, 3000, 128
    q = torch.randn(B, H, L, 128, generator=g).bfloat16().cuda()
    k = torch.randn(B, 2, L, 128, generator=g).bfloat16().cuda()
    v = torch.randn(B, 2, L, 128, generator=g).bfloat16().cuda()
    N = (L + bs - 1) // bs
    bits = O.pack_bool(random_mask(B, H, N, 0.3, g)).cuda()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    full = lib.sparse_attention(q, k, v, bits, bs, status=status)
    for lo, hi in ((0, 1024), (1024, 2304), (2304, L)):
        part = lib.sparse_attention(q, k, v, bits, bs, status=status, rows=(lo, hi))
        assert part.shape == (B, hi - lo, H, 128)
        assert torch.equal(part, full[:, lo:hi])
    assert int(status.item()) == 0
    with pytest.raises(ValueError):
        lib.sparse_attention(q, k, v, bits, bs, rows=(100, 1024))  # not on a 128-row boundary


def test_push_to_peer_buffers_equals_own_output(lib):
    # ffts_sparse_attn_fwd_push: the epilogue also stores every output row into
    # each peer buffer (here two more buffers on this GPU, which the kernel
    # addresses the same way); ragged L, a row range, both output layouts
    g = torch.Generator().manual_seed(29)
    B, H, L, bs = 2, 4, 3000, 64
    q = torch.randn(B, H, L, 128, generator=g).bfloat16().cuda()
    k = torch.randn(B, 2, L, 128, generator=g).bfloat16().cuda()
    v = torch.randn(B, 2, L, 128, generator=g).bfloat16().cuda()
    N = (L + bs - 1) // bs
    bits = O.pack_bool(random_mask(B, H, N, 0.3, g)).cuda()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    full = lib.sparse_attention(q, k, v, bits, bs, status=status)
    # [B, L, H, D] output
    peers = [torch.full((B, L, H, 128), 7.0, dtype=torch.bfloat16, device="cuda") for _ in range(2)]
    own = lib.sparse_attention(q, k, v, bits, bs, status=status, peers=[p.data_ptr() for p in peers])
    assert torch.equal(own, full)
    for p in peers:
        assert torch.equal(p, full)
    # head-major [B, H, L, D] buffers (rows contiguous), rows [1024, L) of heads 1..2
    lo = 1024
    bufs = [torch.zeros(B, H, L, 128, dtype=torch.bfloat16, device="cuda") for _ in range(3)]
    pitch_h = L * 128 * 2
    out = bufs[0][:, 1:3, lo:].permute(0, 2, 1, 3)
    part = lib.sparse_attention(q[:, 1:3], k[:, :1], v[:, :1], bits[:, 1:3].contiguous(), bs, status=status,
                                out=out, rows=(lo, L),
                                peers=[b.data_ptr() + 1 * pitch_h + lo * 256 for b in bufs[1:]])
    torch.cuda.synchronize()
    ref = lib.sparse_attention(q[:, 1:3], k[:, :1], v[:, :1], bits[:, 1:3].contiguous(), bs, status=status)
    for b in bufs:
        assert torch.equal(b[:, 1:3, lo:], ref[:, lo:].permute(0, 2, 1, 3))
        assert not b[:, :, :lo].any() and not b[:, 0].any() and not b[:, 3].any()
    assert int(status.item()) == 0
    with pytest.raises(ValueError):
        lib.sparse_attention(q, k, v, bits, bs, peers=[0])  # a NULL peer buffer


@pytest.mark.parametrize("L,H,Hkv,bs", [(8000, 4, 2, 128), (6000, 4, 4, 64)])
def test_selected_mask_matches_flash_attn_on_gathered_blocks(lib, L, H, Hkv, bs):
    """Pins the sparse attention with a selected FFTSparse mask to flash_attn, the
    library behind the reference's block_sparse_attn_func.  Each (head, query
    block) becomes one varlen sequence whose keys are its kept key blocks gathered
    in ascending order: the diagonal block is always kept and comes last, so
    flash_attn's bottom-right causal alignment masks exactly the causal part of
    it.  Same bf16 tolerance as the fp32 comparisons."""
    try:
        from flash_attn import flash_attn_varlen_func
    except Exception as exc:  # noqa: BLE001 - any import failure means the wheel is unusable here
        pytest.skip(f"flash_attn cannot be imported: {exc}")
    import bench
    g = torch.Generator().manual_seed(L + bs)
    q = torch.randn(1, H, L, 128, generator=g).bfloat16().cuda()
    k = torch.randn(1, Hkv, L, 128, generator=g).bfloat16().cuda()
    v = torch.randn(1, Hkv, L, 128, generator=g).bfloat16().cuda()
    mask = lib.fft_block_mask(q, k, **dict(bench.mask_kwargs(0.1), block_size=bs))
    row_ptr, col_idx = (t.cpu() for t in mask.csr())
    out = lib.sparse_attention(q, k, v, mask.bits, bs)  # [1, L, H, D]
    N, G = mask.n_blocks, H // Hkv
    qi, ki, cu_q, cu_k, heads_q, heads_k = [], [], [0], [0], [], []
    for h in range(H):
        for i in range(N):
            r = h * N + i
            sel = col_idx[row_ptr[r]:row_ptr[r + 1]].long()
            sel = sel[sel <= i]  # the kernel cuts blocks above the diagonal
            assert int(sel[-1]) == i, "the diagonal block is always kept"
            rows = torch.arange(i * bs, min((i + 1) * bs, L))
            keys = torch.cat([torch.arange(j * bs, min((j + 1) * bs, L)) for j in sel.tolist()])
            qi.append(rows)
            ki.append(keys)
            heads_q.append(torch.full_like(rows, h))
            heads_k.append(torch.full_like(keys, h // G))
            cu_q.append(cu_q[-1] + rows.numel())
            cu_k.append(cu_k[-1] + keys.numel())
    qi, ki = torch.cat(qi).cuda(), torch.cat(ki).cuda()
    hq, hk = torch.cat(heads_q).cuda(), torch.cat(heads_k).cuda()
    qg = q[0][hq, qi].unsqueeze(1)  # [total_q, 1, D]
    kg, vg = k[0][hk, ki].unsqueeze(1), v[0][hk, ki].unsqueeze(1)
    cq = torch.tensor(cu_q, dtype=torch.int32, device="cuda")
    ck = torch.tensor(cu_k, dtype=torch.int32, device="cuda")
    try:
        ref = flash_attn_varlen_func(qg, kg, vg, cq, ck, bs, max(b - a for a, b in zip(cu_k, cu_k[1:])),
                                     causal=True)
    except RuntimeError as exc:
        pytest.skip(f"flash_attn has no kernel for this GPU: {exc}")
    got = out[0][qi, hq]  # [total_q, D] in the same (head, block, row) order
    err = (got.float() - ref[:, 0].float()).abs()
    assert float(err.max()) <= MAX_ABS, float(err.max())
    assert float(err.mean()) <= MEAN_ABS, float(err.mean())


def _gathered_pairs(row_ptr, col_idx, H, N, bs, pairs):
    """(query rows, kept key positions) of each (batch, head, query block) pair:
    the kept key blocks in ascending order, cut at the diagonal as the kernel does."""
    out = []
    for b, h, i in pairs:
        r = (b * H + h) * N + i
        sel = col_idx[row_ptr[r]:row_ptr[r + 1]].long()
        sel = sel[sel <= i]
        assert int(sel[-1]) == i, "the diagonal block is always kept"
        rows = torch.arange(i * bs, (i + 1) * bs)
        keys = torch.cat([torch.arange(j * bs, (j + 1) * bs) for j in sel.tolist()])
        out.append((rows, keys))
    return out


@pytest.mark.parametrize("B,L,H,Hkv,bs,rope_base", [(1, 131072, 32, 8, 128, 500000.0),
                                                     (2, 65536, 28, 4, 64, 1000000.0)])
def test_bench_shape_matches_fp32_and_flash_attn(lib, B, L, H, Hkv, bs, rope_base):
    """The BASELINE shapes at full size: config 3 as bench.py runs it (131072
    tokens, 32 query heads over 8 KV heads, block 128) and config 5's Qwen2.5-7B
    layer (2 x 65536 tokens, 28 over 4 heads, block 64), with the bench's synthetic
    inputs (K/V repeat_kv-expanded, as the reference's callers pass them), keep ratio
    0.05 and the FFTSparse-selected mask.  One head of every KV
    group of the last sequence is checked on 40 query blocks spread over the
    sequence, first and last included: the kernel's rows against a plain PyTorch
    fp32 evaluation, and against flash_attn (the library behind the reference's
    block_sparse_attn_func), on the same gathered key blocks.  The drop-in call
    returns the same bits as the kernel called on the selected mask."""
    import bench
    from fftsparse_b200.synthetic import make_inputs
    G = H // Hkv
    q, k, v = make_inputs(L, num_q_heads=H, num_kv_heads=Hkv, dtype=torch.bfloat16, device="cuda", batch=B,
                          rope_base=rope_base)
    kw = dict(bench.mask_kwargs(0.05), block_size=bs)
    mask = lib.fft_block_mask(q, k, **kw)
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = lib.sparse_attention(q, k, v, mask.bits, bs, status=status)  # [B, L, H, D]
    full = lib.myattn_prefill(q, k, v, 0, **kw)
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    assert torch.equal(full.view(B, L, H, 128), out)
    N = mask.n_blocks
    row_ptr, col_idx = (t.cpu() for t in mask.csr())
    b = B - 1
    kv_of = (lambda h: h // G) if k.shape[1] == Hkv else (lambda h: h)  # the bench passes expanded K/V
    heads = [g * G + (g % G) for g in range(Hkv)]  # one head per KV group, varying position in the group
    blocks = sorted({0, 1, 2, N // 2, N - 2, N - 1} | set(range(5, N, max(1, N // 34))))[:40]
    pairs = [(b, h, i) for h in heads for i in blocks]
    spans = _gathered_pairs(row_ptr, col_idx, H, N, bs, pairs)
    scale = 128 ** -0.5
    errs = []
    for (_, h, _), (rows, keys) in zip(pairs, spans):
        rows, keys = rows.cuda(), keys.cuda()
        s = (q[b, h, rows].float() @ k[b, kv_of(h), keys].float().T) * scale
        s = s.masked_fill(keys[None, :] > rows[:, None], float("-inf"))
        ref = torch.softmax(s, dim=-1) @ v[b, kv_of(h), keys].float()
        errs.append((out[b, rows, h].float() - ref).abs().flatten())
    err = torch.cat(errs)
    assert float(err.max()) <= MAX_ABS, float(err.max())
    assert float(err.mean()) <= MEAN_ABS, float(err.mean())
    try:
        from flash_attn import flash_attn_varlen_func
    except Exception:  # noqa: BLE001 - the fp32 comparison above stands on its own
        return
    qi = torch.cat([r for r, _ in spans]).cuda()
    ki = torch.cat([kk for _, kk in spans]).cuda()
    hq = torch.cat([torch.full((r.numel(),), h) for (_, h, _), (r, _) in zip(pairs, spans)]).cuda()
    hk = torch.cat([torch.full((kk.numel(),), kv_of(h)) for (_, h, _), (_, kk) in zip(pairs, spans)]).cuda()
    cu_q = torch.tensor([0] + [r.numel() for r, _ in spans]).cumsum(0).int().cuda()
    lens_k = [kk.numel() for _, kk in spans]
    cu_k = torch.tensor([0] + lens_k).cumsum(0).int().cuda()
    try:
        ref = flash_attn_varlen_func(q[b][hq, qi].unsqueeze(1), k[b][hk, ki].unsqueeze(1),
                                     v[b][hk, ki].unsqueeze(1), cu_q, cu_k, bs, max(lens_k), causal=True)
    except RuntimeError:
        return
    err = (out[b][qi, hq].float() - ref[:, 0].float()).abs()
    assert float(err.max()) <= MAX_ABS, float(err.max())
    assert float(err.mean()) <= MEAN_ABS, float(err.mean())
