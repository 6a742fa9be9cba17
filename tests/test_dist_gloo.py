"""Multi-process host logic of the KV-group sharded prefill, on CPU ranks (gloo).

The two CUDA entry points sharded_prefill calls are replaced by the CPU oracle
inside each rank, so these tests run the real host code and check what the
sharding adds: which heads a rank owns, the head-major
all-gather, equality with the unsharded result, and that a rank that dies
before the collective turns into an error on its peer instead of a hang.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from fftsparse_b200.dist import gather_heads, kv_group_shard, local_views, unit_shard


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_kv_group_shard_partitions_heads():
    for world in (1, 2, 4, 8):
        seen = []
        for r in range(world):
            s = kv_group_shard(32, 8, world, r)
            assert s.h_hi - s.h_lo == 32 // world
            assert (s.kv_hi - s.kv_lo) * 4 == s.h_hi - s.h_lo
            seen.extend(range(s.h_lo, s.h_hi))
        assert seen == list(range(32))
    with pytest.raises(ValueError):
        kv_group_shard(28, 4, 8, 0)  # 4 KV groups cannot split over 8 ranks


def test_unit_shard_sequences_by_kv_groups():
    # 2 sequences x 4 KV groups (28 q-heads) over 8 ranks, one unit each
    seen = set()
    for r in range(8):
        s = unit_shard(2, 28, 4, 8, r)
        assert s.b_hi - s.b_lo == 1 and s.kv_hi - s.kv_lo == 1 and s.heads == 7
        seen.add((s.b_lo, s.kv_lo))
    assert seen == {(b, g) for b in range(2) for g in range(4)}
    # KV groups split first when they divide over the ranks
    s = unit_shard(4, 8, 2, 2, 1)
    assert (s.b_lo, s.b_hi, s.kv_lo, s.kv_hi) == (0, -1, 1, 2)
    # one KV group: whole sequences per rank
    s = unit_shard(4, 4, 1, 2, 1)
    assert (s.b_lo, s.b_hi, s.h_lo, s.h_hi) == (2, 4, 0, 4)
    with pytest.raises(ValueError):
        unit_shard(3, 28, 4, 8, 0)  # 12 units over 8 ranks


def test_local_views_expanded_and_gqa():
    q = torch.randn(1, 8, 16, 4)
    k_exp = torch.randn(1, 8, 16, 4)
    k_kv = torch.randn(1, 2, 16, 4)
    s = kv_group_shard(8, 2, 2, 1)
    qs, ks, vs = local_views(q, k_exp, k_exp, s)
    assert torch.equal(qs, q[:, 4:8]) and torch.equal(ks, k_exp[:, 4:8])
    qs, ks, vs = local_views(q, k_kv, k_kv, s)
    assert torch.equal(ks, k_kv[:, 1:2])


def _patch_kernels_with_oracle():
    """Swap the two CUDA entry points sharded_prefill calls for oracle stand-ins,
    so the real host logic (shard choice, local views, output layout, gather)
    runs on CPU ranks."""
    from types import SimpleNamespace

    import fftsparse_b200.prefill as P
    from fftsparse_b200.params import derive_mask_params
    from oracle import oracle as O

    def fake_mask(q, k, block_size=128, **kw):
        params = derive_mask_params(q.shape[2], block_size=block_size, **kw)
        m = O.prefill_mask(q.contiguous(), k.contiguous(), params)
        return SimpleNamespace(bits=O.unpack_bits(m["bits"], params.n_blocks))

    def fake_attn(q, k, v, dense, bs, causal=True, out=None, status=None, rows=None):
        L = q.shape[2]
        lo, hi = (0, L) if rows is None else rows
        blocks = list(range(lo // bs, (hi + bs - 1) // bs))
        res = O.sparse_attention(q, k, v, dense, bs, causal=causal, rows=blocks).to(torch.bfloat16)  # [B, H, L, D]
        out.copy_(res[:, :, lo:hi].permute(0, 2, 1, 3))
        return out

    P.fft_block_mask = fake_mask
    P.sparse_attention = fake_attn


def _worker(rank, world, port, result_q, kw):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from fftsparse_b200.dist import sharded_prefill
        from oracle.synth import make_inputs
        _patch_kernels_with_oracle()
        q, k, v = make_inputs(1536, num_q_heads=8, num_kv_heads=2, dtype=torch.bfloat16, expand=False)
        out_full = sharded_prefill(q, k, v, 0, **kw)
        # each rank holding only its own heads (its columns of a QKV projection)
        s = kv_group_shard(8, 2, world, rank)
        ql, kl, vl = local_views(q, k, v, s)
        out_local = sharded_prefill(ql.contiguous(), kl.contiguous(), vl.contiguous(), 0,
                                    inputs_are_local=True, **kw)
        if rank == 0:
            result_q.put((out_full.view(torch.int16).numpy().tobytes(),
                          out_local.view(torch.int16).numpy().tobytes()))
    finally:
        dist.destroy_process_group()


def _worker_batch(rank, world, port, result_q, kw):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from fftsparse_b200.dist import sharded_prefill
        from oracle.synth import make_inputs
        _patch_kernels_with_oracle()
        # 2 sequences x 1 KV group: the ranks split by sequence
        q, k, v = make_inputs(1280, num_q_heads=4, num_kv_heads=1, dtype=torch.bfloat16, expand=False, batch=2)
        out_full = sharded_prefill(q, k, v, 0, **kw)
        s = unit_shard(2, 4, 1, world, rank)
        ql, kl, vl = local_views(q, k, v, s)
        out_local = sharded_prefill(ql.contiguous(), kl.contiguous(), vl.contiguous(), 0, inputs_are_local=True,
                                    global_batch=2, num_heads=4, num_kv_heads=1, **kw)
        if rank == 0:
            result_q.put((out_full.view(torch.int16).numpy().tobytes(),
                          out_local.view(torch.int16).numpy().tobytes()))
    finally:
        dist.destroy_process_group()


def test_sharded_by_sequence_world2():
    kw = dict(block_size=128, sink_ratio=0.01, recent_ratio=0.0, local_span_ratio=0.02,
              correlation_selection_mode="topk", correlation_topk_ratio=0.2, qk_topk_ratio=0.2)
    ctx = mp.get_context("spawn")
    q_out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_batch, args=(r, 2, port, q_out, kw)) for r in range(2)]
    for p in procs:
        p.start()
    got_full, got_local = q_out.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    import numpy as np

    from oracle import oracle as O
    from oracle.synth import make_inputs
    from fftsparse_b200.params import derive_mask_params
    q, k, v = make_inputs(1280, num_q_heads=4, num_kv_heads=1, dtype=torch.bfloat16, expand=False, batch=2)
    params = derive_mask_params(1280, **kw)
    m = O.prefill_mask(q, k, params)
    ref = O.sparse_attention(q, k, v, O.unpack_bits(m["bits"], params.n_blocks), 128).to(torch.bfloat16)
    for b in (got_full, got_local):
        got = torch.from_numpy(np.frombuffer(b, dtype=np.int16).copy()).view(torch.bfloat16).view(2, 4, 1280, 128)
        assert torch.equal(got, ref)


def test_sharded_equals_unsharded_world2():
    kw = dict(block_size=128, sink_ratio=0.01, recent_ratio=0.0, local_span_ratio=0.02,
              correlation_selection_mode="topk", correlation_topk_ratio=0.2, qk_topk_ratio=0.2,
              stripe_threshold=0.012)
    ctx = mp.get_context("spawn")
    q_out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q_out, kw)) for r in range(2)]
    for p in procs:
        p.start()
    got_full, got_local = q_out.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    import numpy as np

    def as_bf16(b):
        return torch.from_numpy(np.frombuffer(b, dtype=np.int16).copy()).view(torch.bfloat16).view(1, 8, 1536, 128)

    from oracle import oracle as O
    from oracle.synth import make_inputs
    from fftsparse_b200.params import derive_mask_params
    q, k, v = make_inputs(1536, num_q_heads=8, num_kv_heads=2, dtype=torch.bfloat16, expand=False)
    params = derive_mask_params(1536, **kw)
    m = O.prefill_mask(q, k, params)
    ref = O.sparse_attention(q, k, v, O.unpack_bits(m["bits"], params.n_blocks), 128).to(torch.bfloat16)
    assert torch.equal(as_bf16(got_full), ref)
    assert torch.equal(as_bf16(got_local), ref)


def _dying_worker(rank, world, port, result_q):
    from datetime import timedelta
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    if rank == 1:
        os._exit(3)  # leaves between steps, before the collective
    try:
        gather_heads(torch.zeros(1, 1, 4, 4), torch.zeros(1, 2, 4, 4))
        result_q.put("no error")
    except Exception as e:  # the peer's death surfaces as an error, not a hang
        result_q.put(type(e).__name__)


def test_dead_rank_raises_on_peer():
    ctx = mp.get_context("spawn")
    q_out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dying_worker, args=(r, 2, port, q_out)) for r in range(2)]
    for p in procs:
        p.start()
    res = q_out.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert res != "no error"


def test_row_chunks_cover_rows_with_equal_causal_work():
    from fftsparse_b200.dist import row_chunks
    L = 131072
    for parts in (2, 4, 8):
        ch = row_chunks(L, parts)
        assert ch[0][0] == 0 and ch[-1][1] == L and len(ch) == parts
        assert all(a[1] == b[0] for a, b in zip(ch, ch[1:]))          # contiguous
        assert all(lo % 128 == 0 for lo, _ in ch)                      # on tile-row boundaries
        work = [(hi * hi - lo * lo) / (L * L) for lo, hi in ch]      # causal work ~ rows squared
        assert max(work) - min(work) < 0.01
    assert row_chunks(L, 4) == [(0, 65536), (65536, 92672), (92672, 113536), (113536, 131072)]
    assert row_chunks(1000, 4) == [(0, 1000)]                          # short: one chunk
    assert row_chunks(L, 1) == [(0, L)]
