"""The copy-engine all-gather of the sharded prefill (dist.PeerGather) on two GPUs:
its output equals the NCCL all-gather path bit for bit, on consecutive calls
(both of its alternating buffers, and a reuse).  Skipped on a box with one GPU."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q_out):
    from datetime import timedelta

    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120), device_id=dev)
    try:
        import bench
        import fftsparse_b200 as F
        from fftsparse_b200.dist import PeerGather, row_chunks, sharded_prefill
        from fftsparse_b200.synthetic import make_inputs
        F.load_library()
        L = 8192
        assert len(row_chunks(L)) > 1
        q, k, v = make_inputs(L, num_q_heads=8, num_kv_heads=2, dtype=torch.bfloat16, device=str(dev),
                              expand=False)
        kw = bench.mask_kwargs(0.1)
        pg = PeerGather(8, L, 128, device=dev)
        ref = sharded_prefill(q, k, v, 0, **kw).clone()
        ok = True
        for _ in range(3):
            got = sharded_prefill(q, k, v, 0, gather=pg, **kw)
            torch.cuda.synchronize(dev)
            ok &= bool(torch.equal(got, ref))
        ok &= int(pg.status.item()) == 0
        dist.barrier()
        pg.close()
        q_out.put((rank, ok))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_peer_gather_equals_nccl_gather():
    ctx = mp.get_context("spawn")
    q_out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q_out)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q_out.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert results == {0: True, 1: True}
