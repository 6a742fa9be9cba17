"""The copy-engine all-gather of the sharded prefill (dist.PeerGather).

On two GPUs its output equals the NCCL all-gather path bit for bit, with the
pushes in the attention epilogue and on the copy engines, on consecutive calls
(both of its alternating buffers, and a reuse); skipped on a box with one GPU.  On one GPU: the row copy, flag store and bounded wait entry
points, including a wait that runs out on a flag nothing sets."""
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
        ref = sharded_prefill(q, k, v, 0, **kw).clone()
        ok = True
        for push in ("epilogue", "copy"):
            pg = PeerGather(8, L, 128, device=dev, push=push)
            for _ in range(3):
                got = sharded_prefill(q, k, v, 0, gather=pg, **kw)
                torch.cuda.synchronize(dev)
                ok &= bool(torch.equal(got, ref))
            ok &= int(pg.status.item()) == 0
            dist.barrier()
            pg.close()
            dist.barrier()
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


def _ptrs(*addrs):
    import ctypes
    return (ctypes.c_void_p * len(addrs))(*addrs)


def test_copy_rows_signal_wait_one_gpu():
    """The copy, flag-store and wait entry points on one GPU: a strided row copy
    to two destinations on two streams, an epoch stored into two flags, and a
    wait that sees it (status stays 0)."""
    from fftsparse_b200 import _lib
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream(dev).cuda_stream
    H, L, D = 3, 640, 128
    src = torch.randn(H, L, D, device=dev).to(torch.bfloat16)
    dst = [torch.zeros(H, L, D, dtype=torch.bfloat16, device=dev) for _ in range(2)]
    pitch, row = L * D * 2, D * 2
    lo, hi = 128, 512
    side = torch.cuda.Stream(device=dev)
    ready = torch.cuda.Event()
    ready.record(torch.cuda.current_stream(dev))
    # copy 0 on the current stream, copy 1 on a second stream that waits for `ready`
    _lib.check(lib.ffts_copy_rows(_ptrs(*[d.data_ptr() + lo * row for d in dst]), _ptrs(stream, side.cuda_stream),
                                  2, src.data_ptr() + lo * row, pitch, (hi - lo) * row, H, ready.cuda_event))
    flags = torch.zeros(2, dtype=torch.int32, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    _lib.check(lib.ffts_signal(_ptrs(flags.data_ptr(), flags.data_ptr() + 4), _ptrs(stream, side.cuda_stream), 2, 7))
    torch.cuda.current_stream(dev).wait_stream(side)
    _lib.check(lib.ffts_wait_flags(flags.data_ptr(), 2, 7, status.data_ptr(), stream))
    torch.cuda.synchronize(dev)
    for d in dst:
        assert torch.equal(d[:, lo:hi], src[:, lo:hi])
        assert not d[:, :lo].any() and not d[:, hi:].any()
    assert flags.tolist() == [7, 7]
    assert int(status.item()) == 0


def test_wait_flags_times_out_with_status():
    """A wait on a flag that nothing sets ends by itself (about 2 s of SM cycles)
    with status 5; the context stays usable afterwards."""
    from fftsparse_b200 import _lib
    lib = _lib.load()
    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream(dev).cuda_stream
    flags = torch.tensor([3, 0], dtype=torch.int32, device=dev)  # flag 1 never reaches epoch 3
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    _lib.check(lib.ffts_wait_flags(flags.data_ptr(), 2, 3, status.data_ptr(), stream))
    torch.cuda.synchronize(dev)
    assert int(status.item()) == 5
    x = torch.ones(4, device=dev)
    assert float((x + 1).sum().item()) == 8.0


def test_peer_gather_raises_when_a_peer_never_delivers():
    """PeerGather.run on one GPU (a one-rank group) with a second flag that no
    peer ever stores: the bounded flag wait ends with status 5, and the next run
    raises WaitTimeout before launching anything; once the flag set is whole
    again the calls go on."""
    import torch.distributed as dist

    import bench
    import fftsparse_b200 as F
    from fftsparse_b200.dist import PeerGather, kv_group_shard, local_views
    from fftsparse_b200.status import WaitTimeout
    from fftsparse_b200.synthetic import make_inputs
    F.load_library()
    dev = torch.device("cuda", 0)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{_free_port()}", rank=0, world_size=1)
    try:
        L = 2048
        q, k, v = make_inputs(L, num_q_heads=8, num_kv_heads=2, dtype=torch.bfloat16, device=str(dev), expand=False)
        shard = kv_group_shard(8, 2, 1, 0)
        ql, kl, vl = local_views(q, k, v, shard)
        mask = F.fft_block_mask(ql, kl, **bench.mask_kwargs(0.1))
        pg = PeerGather(8, L, 128, device=dev)
        ref = pg.run(ql, kl, vl, mask.bits, 128, True, shard).clone()
        pg.check()
        own_flags, pg.flags, pg.world = pg.flags, torch.zeros(2, dtype=torch.int32, device=dev), 2
        pg.run(ql, kl, vl, mask.bits, 128, True, shard)  # waits ~2 s for flag 1, then gives up
        torch.cuda.synchronize(dev)
        with pytest.raises(WaitTimeout) as exc:
            pg.run(ql, kl, vl, mask.bits, 128, True, shard)
        assert exc.value.code == 5
        pg.flags, pg.world = own_flags, 1
        got = pg.run(ql, kl, vl, mask.bits, 128, True, shard)
        pg.check()
        assert torch.equal(got, ref)
        pg.close()
    finally:
        dist.destroy_process_group()
