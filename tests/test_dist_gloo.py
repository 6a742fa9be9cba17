"""Multi-process host logic of the KV-group sharded prefill, on CPU ranks (gloo).

The CUDA kernels are replaced by the CPU oracle inside each rank, so these tests
check what the sharding adds: which heads a rank owns, the head-major
all-gather, equality with the unsharded result, and that a rank that dies
before the collective turns into an error on its peer instead of a hang.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from fftsparse_b200.dist import gather_heads, kv_group_shard, local_views


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


def test_local_views_expanded_and_gqa():
    q = torch.randn(1, 8, 16, 4)
    k_exp = torch.randn(1, 8, 16, 4)
    k_kv = torch.randn(1, 2, 16, 4)
    s = kv_group_shard(8, 2, 2, 1)
    qs, ks, vs = local_views(q, k_exp, k_exp, s)
    assert torch.equal(qs, q[:, 4:8]) and torch.equal(ks, k_exp[:, 4:8])
    qs, ks, vs = local_views(q, k_kv, k_kv, s)
    assert torch.equal(ks, k_kv[:, 1:2])


def _cpu_sharded_prefill(q, k, v, kw):
    """sharded_prefill's host logic with the oracle standing in for the kernels."""
    from oracle import oracle as O
    from fftsparse_b200.params import derive_mask_params
    world, rank = dist.get_world_size(), dist.get_rank()
    B, H, L, D = q.shape
    shard = kv_group_shard(H, k.shape[1], world, rank)
    ql, kl, vl = local_views(q, k, v, shard)
    params = derive_mask_params(L, **kw)
    m = O.prefill_mask(ql.contiguous(), kl.contiguous(), params)
    dense = O.unpack_bits(m["bits"], params.n_blocks)
    local = O.sparse_attention(ql, kl, vl, dense, params.block_size).to(torch.bfloat16)
    out = torch.empty(B, H, L, D, dtype=torch.bfloat16)
    return gather_heads(local, out)


def _worker(rank, world, port, result_q, kw):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle.synth import make_inputs
        q, k, v = make_inputs(1536, num_q_heads=8, num_kv_heads=2, dtype=torch.bfloat16, expand=False)
        out = _cpu_sharded_prefill(q, k, v, kw)
        if rank == 0:
            result_q.put(out.view(torch.int16).numpy().tobytes())
    finally:
        dist.destroy_process_group()


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
    got = q_out.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    import numpy as np
    got = torch.from_numpy(np.frombuffer(got, dtype=np.int16).copy()).view(torch.bfloat16).view(1, 8, 1536, 128)

    from oracle import oracle as O
    from oracle.synth import make_inputs
    from fftsparse_b200.params import derive_mask_params
    q, k, v = make_inputs(1536, num_q_heads=8, num_kv_heads=2, dtype=torch.bfloat16, expand=False)
    params = derive_mask_params(1536, **kw)
    m = O.prefill_mask(q, k, params)
    ref = O.sparse_attention(q, k, v, O.unpack_bits(m["bits"], params.n_blocks), 128).to(torch.bfloat16)
    assert torch.equal(got, ref)


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
