"""The TTFT decoder harness (bench.DecoderShape) split over two gloo CPU ranks:
attention by (sequence, KV group) unit, o_proj/MLP by token rows with one
all-gather of the hidden states per layer.  Two shapes: one sequence whose two
KV groups split over the ranks (config 4's split), and two sequences of one KV
group with block 64, which split by sequence (config 5's split).  The fused RoPE + pooling and the two attention entry
points are replaced by the CPU oracle inside each rank, which also checks that
the pooled blocks handed to the selection are those of the rotated q and k.
The last-position logits of the two-rank run equal the one-rank run's, bit for
bit."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

# (dims = H, HKV, D, HIDDEN, INTER, VOCAB; batch; sequence length; block size)
CASES = {"kv_groups": ((4, 2, 128, 256, 512, 1000), 1, 2048, 128),
         "sequences": ((2, 1, 128, 256, 512, 1000), 2, 1280, 64)}
LAYERS = 2


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _patch_with_oracle(mp=None):
    """Replace the CUDA entry points with oracle stand-ins; through ``mp`` (pytest's
    monkeypatch, undone after the test) in the test process, for good in a worker."""
    from types import SimpleNamespace

    import fftsparse_b200 as F
    import fftsparse_b200.prefill as P
    from fftsparse_b200.params import derive_mask_params
    from oracle import oracle as O

    def fake_mask(q, k, block_size=128, pooled=None, **kw):
        params = derive_mask_params(q.shape[2], block_size=block_size, **kw)
        if pooled is not None:  # the blocks rope_pool produced are the pooled rotated q and k
            assert torch.equal(pooled[0], O.pool(q.contiguous(), block_size))
            assert torch.equal(pooled[1], O.pool(k.contiguous(), block_size))
        m = O.prefill_mask(q.contiguous(), k.contiguous(), params)
        return SimpleNamespace(bits=O.unpack_bits(m["bits"], params.n_blocks))

    def fake_attn(q, k, v, dense, bs, causal=True, out=None, status=None, rows=None, peers=None):
        res = O.sparse_attention(q, k, v, dense, bs, causal=causal).to(torch.bfloat16)  # [B, H, L, D]
        out.copy_(res.permute(0, 2, 1, 3))
        return out

    def fake_prefill(q, k, v, layer_idx, block_size=128, pooled=None, **kw):
        m = fake_mask(q, k, block_size=block_size, pooled=pooled, **kw)
        B, H, Lq, D = q.shape
        out = torch.empty(B, Lq, H, D, dtype=torch.bfloat16)
        return fake_attn(q, k, v, m.bits, block_size, out=out).view(B, Lq, H * D)

    def fake_rope_pool(qp, kp, vp, h, hkv, cos, sin, block_size=128):
        return O.rope_pool(qp, kp, vp, h, hkv, cos, sin, block_size)

    def fake_qkv_rope_pool(x, w, bias, h, hkv, cos, sin, block_size=128, return_projection=False, status=None):
        # the projection per sequence, then the oracle's RoPE + layout + pooling
        assert bias is None and not return_projection
        D = cos.shape[1]
        outs = []
        for s in range(x.shape[0]):
            p = x[s] @ w.T
            outs.append(O.rope_pool(p[:, :h * D], p[:, h * D:(h + hkv) * D], p[:, (h + hkv) * D:], h, hkv, cos, sin,
                                    block_size))
        return tuple(torch.cat([o[j] for o in outs], 0) for j in range(5))

    put = mp.setattr if mp is not None else setattr
    put(P, "fft_block_mask", fake_mask)
    put(P, "sparse_attention", fake_attn)
    put(F, "myattn_prefill", fake_prefill)
    put(F, "rope_pool", fake_rope_pool)
    put(F, "qkv_rope_pool", fake_qkv_rope_pool)


def _run(world, rank, case, mp=None):
    import bench
    _patch_with_oracle(mp)
    dims, B, L, bs = CASES[case]
    kw = dict(bench.mask_kwargs(0.2), block_size=bs)
    model = bench.DecoderShape(LAYERS, torch.device("cpu"), world, rank, dims=dims, batch=B)
    ids = torch.randint(0, dims[-1], (B, L), generator=torch.Generator().manual_seed(0))
    with torch.no_grad():
        return model.forward(ids, kw).float()


def _worker(rank, world, port, result_q, case):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        logits = _run(world, rank, case)
        result_q.put((rank, logits.numpy().tobytes()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("case", sorted(CASES))
def test_decoder_two_ranks_equals_one(case, monkeypatch):
    ctx = mp.get_context("spawn")
    q_out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q_out, case)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q_out.get(timeout=600) for _ in range(2))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    ref = _run(1, 0, case, monkeypatch)
    assert ref.shape == (CASES[case][1], CASES[case][0][-1])
    for r in (0, 1):
        logits = torch.from_numpy(np.frombuffer(got[r], dtype=np.float32).copy()).view_as(ref)
        assert torch.isfinite(logits).all()
        # every output row of a GEMM is summed the same way whatever rows surround it
        assert torch.equal(logits, ref), (logits - ref).abs().max()
