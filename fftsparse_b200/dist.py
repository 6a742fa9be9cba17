"""(Sequence, KV-group) sharded FFTSparse prefill, one process per GPU.

The reference has no distributed path: multi-GPU use there is accelerate's
``device_map="auto"`` layer placement (eval/LongBench/pred.py:520).  Every step
of the operator is independent per head, and heads that share a key/value head
(a GQA group) also share its K/V tiles, so the unit of work is the
(sequence, KV group).  Each rank runs pooling, mask selection and attention
for its contiguous slice of KV groups with no communication, and one
all-gather assembles the head-major output [B, H, L, D] that o_proj consumes:
through peer memory, fused into the attention kernel's epilogue (PeerGather),
or as an NCCL all-gather (gather_heads).
When the KV groups are fewer than the ranks (2 sequences x
4 KV groups on 8 GPUs), the units are (sequence, KV group) pairs, ordered
sequence-major, and a rank owns a contiguous run of them.

Functions here take the full q/k/v (or any rank-local copy of them) and slice
the rank's heads as views; nothing is copied before the kernels run.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist

from . import trace
from .status import StatusWord


@dataclass(frozen=True)
class Shard:
    rank: int
    world: int
    kv_lo: int
    kv_hi: int
    h_lo: int
    h_hi: int
    b_lo: int = 0     # sequences [b_lo, b_hi); b_hi = -1 means every sequence
    b_hi: int = -1

    @property
    def heads(self) -> int:
        return self.h_hi - self.h_lo


def unit_shard(batch: int, num_heads: int, num_kv_heads: int, world: int, rank: int) -> Shard:
    """The (sequence, KV group) units owned by ``rank``.

    KV groups are split when they divide evenly over the ranks (every rank then
    takes all sequences).  Otherwise the batch * Hkv units, ordered sequence-major,
    are split into equal contiguous runs, each of which must be a block of KV groups
    within one sequence or a block of whole sequences."""
    if num_heads % num_kv_heads:
        raise ValueError(f"H={num_heads} is not a multiple of Hkv={num_kv_heads}")
    rep = num_heads // num_kv_heads
    if num_kv_heads % world == 0:
        per = num_kv_heads // world
        kv_lo, kv_hi = rank * per, (rank + 1) * per
        return Shard(rank, world, kv_lo, kv_hi, kv_lo * rep, kv_hi * rep)
    units = batch * num_kv_heads
    if units % world:
        raise ValueError(f"{batch} sequences x {num_kv_heads} KV groups cannot be split evenly over {world} ranks")
    per = units // world
    first = rank * per
    if per <= num_kv_heads and num_kv_heads % per == 0:
        b = first // num_kv_heads
        kv_lo = first % num_kv_heads
        return Shard(rank, world, kv_lo, kv_lo + per, kv_lo * rep, (kv_lo + per) * rep, b, b + 1)
    if per % num_kv_heads == 0:
        b = first // num_kv_heads
        return Shard(rank, world, 0, num_kv_heads, 0, num_heads, b, b + per // num_kv_heads)
    raise ValueError(f"{per} units per rank do not form whole KV-group blocks of {num_kv_heads}")


def kv_group_shard(num_heads: int, num_kv_heads: int, world: int, rank: int) -> Shard:
    """Contiguous slice of KV groups owned by ``rank`` (every sequence); requires Hkv % world == 0."""
    if num_kv_heads % world:
        raise ValueError(f"{num_kv_heads} KV groups cannot be split evenly over {world} ranks")
    return unit_shard(1, num_heads, num_kv_heads, world, rank)


def local_views(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, shard: Shard):
    """Views of the rank's sequences and heads: q [Bl, Hl, L, D]; k/v [Bl, Hkvl, L, D]
    (or the matching q-head slice when k/v are repeat_kv-expanded to H heads)."""
    H, Hk = q.shape[1], k.shape[1]
    bs = slice(shard.b_lo, None if shard.b_hi < 0 else shard.b_hi)
    qs = q[bs, shard.h_lo:shard.h_hi]
    if Hk == H:
        ks, vs = k[bs, shard.h_lo:shard.h_hi], v[bs, shard.h_lo:shard.h_hi]
    else:
        ks, vs = k[bs, shard.kv_lo:shard.kv_hi], v[bs, shard.kv_lo:shard.kv_hi]
    return qs, ks, vs


def gather_heads(local_out: torch.Tensor, full_out: torch.Tensor, group=None, shards=None) -> torch.Tensor:
    """All-gather the ranks' head-major shards [Bl, Hl, L, D] into [B, H, L, D].

    ``shards`` (one Shard per rank) places each rank's block; without it every rank
    holds all sequences and a contiguous run of heads in rank order.  One sequence
    split by heads gathers straight into the output with one ncclAllGather; other
    layouts gather rank-major and copy each block into place."""
    world = dist.get_world_size(group)
    if world == 1:
        full_out.copy_(local_out)
        return full_out
    B = full_out.shape[0]
    whole_batch = shards is None or all(s.b_lo == 0 and s.b_hi in (-1, B) for s in shards)
    if whole_batch and B == 1:
        dist.all_gather_into_tensor(full_out.view(-1), local_out.reshape(-1), group=group)
        return full_out
    tmp = torch.empty((world,) + tuple(local_out.shape), dtype=local_out.dtype, device=local_out.device)
    dist.all_gather_into_tensor(tmp.view(-1), local_out.reshape(-1), group=group)
    if shards is None:
        full_out.copy_(tmp.permute(1, 0, 2, 3, 4).reshape(full_out.shape))
        return full_out
    for r, sh in enumerate(shards):
        bsl = slice(sh.b_lo, None if sh.b_hi < 0 else sh.b_hi)
        full_out[bsl, sh.h_lo:sh.h_hi].copy_(tmp[r])
    return full_out


def row_chunks(L: int, parts: int = 4, tile: int = 128):
    """Query-row chunks [lo, hi) of about equal causal work (boundaries at
    L * sqrt(i / parts), on tile-row boundaries), in increasing row order; one
    chunk for short sequences."""
    if parts <= 1 or L < parts * 8 * tile:
        return [(0, L)]
    cuts = [0]
    for i in range(1, parts):
        c = int(round(L * (i / parts) ** 0.5 / tile)) * tile
        if cuts[-1] < c < L:
            cuts.append(c)
    cuts.append(L)
    return list(zip(cuts[:-1], cuts[1:]))


class PeerGather:
    """The all-gather of the sharded attention output over NVLink peer memory,
    overlapped with the attention itself.

    Created once per (heads, sequence length) by every rank of the group (it is
    collective).  Each rank holds two full head-major output buffers [1, H, L, D]
    and maps its peers' buffers and flag words through CUDA IPC.  NCCL's
    all-gather cannot overlap with the attention: it runs as SM kernels, and the
    attention kernel holds every SM's shared memory and TMEM.  Two ways to push
    the rank's heads into every peer's buffer instead:

    * ``push="epilogue"`` (default): one attention launch whose epilogue stores
      each finished output tile into the own buffer and, over NVLink, into every
      peer's (ffts_sparse_attn_fwd_push), so the transfer runs tile by tile
      alongside the math;
    * ``push="copy"``: the rows are computed in ``chunks`` row chunks of about
      equal causal work (row_chunks); after each chunk one copy stream per peer
      pushes those rows with cudaMemcpy2DAsync (the copy engines) while the SMs
      compute the next chunk.

    Then the call's epoch number is stored into each peer's flag after the
    pushes, and the calling stream waits (bounded) until every rank's flag
    reached the epoch.

    The two buffers alternate between calls, so the tensor a call returns stays
    valid until the call after next; consume it (o_proj) before that.  One
    sequence (B = 1), KV-group shards, bf16 output.  ``status`` (int32 [1]) is
    nonzero after a bounded wait of the attention kernel or of the flag wait
    timed out (code 5: a peer never delivered its rows); ``run`` raises
    WaitTimeout for it at the first call after the failing one has completed,
    and ``check()`` raises at once."""

    def __init__(self, num_heads: int, seq_len: int, head_dim: int = 128, group=None, device=None,
                 push: str = "epilogue", chunks: int = 4):
        from . import _lib

        if push not in ("epilogue", "copy"):
            raise ValueError(f"push must be 'epilogue' or 'copy', got {push!r}")
        self.push = push
        self.world = dist.get_world_size(group)
        # the epilogue stores to at most 15 peers; the wait kernel watches at most 32 flags
        limit = 16 if push == "epilogue" else 32
        if self.world > limit:
            raise ValueError(f"PeerGather(push={push!r}) supports at most {limit} ranks, got {self.world}")
        self.rank = dist.get_rank(group)
        self.H, self.L, self.D = num_heads, seq_len, head_dim
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.lib = _lib.load()
        self.bufs = [torch.empty(1, num_heads, seq_len, head_dim, dtype=torch.bfloat16, device=self.device)
                     for _ in range(2)]
        self.flags = torch.zeros(self.world, dtype=torch.int32, device=self.device)
        self.status_word = StatusWord(self.device)
        self.status = self.status_word.word
        torch.cuda.synchronize(self.device)

        def handle(t):
            h = (ctypes.c_ubyte * 64)()
            off = ctypes.c_int64()
            _lib.check(self.lib.ffts_ipc_handle(t.data_ptr(), h, ctypes.byref(off)))
            return bytes(h), off.value

        mine = [handle(b) for b in self.bufs] + [handle(self.flags)]
        everyone = [None] * self.world
        dist.all_gather_object(everyone, mine, group=group)
        self.peer_bufs = {}
        self.peer_flags = {}
        self._opened = []
        for p in range(self.world):
            if p == self.rank:
                continue
            ptrs = []
            for hb, off in everyone[p]:
                ptr = ctypes.c_void_p()
                _lib.check(self.lib.ffts_ipc_open((ctypes.c_ubyte * 64).from_buffer_copy(hb), off,
                                                  ctypes.byref(ptr)))
                ptrs.append(ptr.value)
                self._opened.append((ptr.value, off))
            self.peer_bufs[p] = ptrs[:2]
            self.peer_flags[p] = ptrs[2]
        peers = sorted(self.peer_bufs)
        # one copy stream per peer: one stream's copies run one after another, so
        # pushes to different peers on different streams use several copy engines
        self.streams = [torch.cuda.Stream(device=self.device) for _ in peers]
        self.chunks = row_chunks(seq_len, chunks)
        self.events = [torch.cuda.Event() for _ in self.chunks]
        n = max(1, len(peers))
        # destination bases per buffer slot and the peers' flag words for this rank
        self._dst = [(ctypes.c_void_p * n)(*[self.peer_bufs[p][slot] for p in peers]) for slot in range(2)]
        self._flags = (ctypes.c_void_p * n)(*[self.peer_flags[p] + 4 * self.rank for p in peers])
        self._streams = (ctypes.c_void_p * n)(*[st.cuda_stream for st in self.streams])
        self._npeers = len(peers)
        self._own_flag = (ctypes.c_void_p * 1)(self.flags.data_ptr() + 4 * self.rank)
        # epilogue pushes: every flag (the peers' words for this rank, then its own)
        # is stored by one kernel on the calling stream after the attention
        self._all_flags = (ctypes.c_void_p * (len(peers) + 1))(*list(self._flags)[:len(peers)],
                                                                self.flags.data_ptr() + 4 * self.rank)
        self.epoch = 0
        dist.barrier(group)  # every rank has mapped every buffer before the first push

    def run(self, ql, kl, vl, bits, block_size: int, causal: bool, shard: Shard, timing=None) -> torch.Tensor:
        """The rank's attention with its output pushed to every peer, then the flag
        exchange.  With a list ``timing`` (epilogue pushes), three timing events are
        appended per call: before the attention, after it, after the flag wait."""
        from . import _lib
        from .prefill import sparse_attention

        lib, dev, ct = self.lib, self.device, ctypes
        cur = torch.cuda.current_stream(dev)
        self.status_word.poll()  # a time-out of an earlier call, once its read-back has landed
        self.epoch += 1
        e, slot = self.epoch, self.epoch % 2
        buf = self.bufs[slot]
        L, D, Hl = self.L, self.D, shard.heads
        row_bytes = D * buf.element_size()
        pitch = L * row_bytes
        local = buf.data_ptr() + shard.h_lo * pitch
        bases = self._dst[slot]
        if self.push == "epilogue":
            evs = [torch.cuda.Event(enable_timing=True) for _ in range(3)] if timing is not None else None
            if evs:
                evs[0].record(cur)
            mine = buf[:, shard.h_lo:shard.h_hi].permute(0, 2, 1, 3)
            sparse_attention(ql, kl, vl, bits, block_size, causal=causal, out=mine, status=self.status,
                             peers=[b + shard.h_lo * pitch for b in bases[:self._npeers]])
            if evs:
                evs[1].record(cur)
            n = self._npeers + 1
            _lib.check(lib.ffts_signal(self._all_flags, (ct.c_void_p * n)(*([cur.cuda_stream] * n)), n, e))
            _lib.check(lib.ffts_wait_flags(self.flags.data_ptr(), self.world, e, self.status.data_ptr(),
                                           cur.cuda_stream))
            if evs:
                evs[2].record(cur)
                timing.append(evs)
            self.status_word.read_back(cur)
            return buf
        # the buffer used now was last read by this rank's pushes two calls ago
        for st in self.streams:
            cur.wait_stream(st)
        for (lo, hi), done in zip(self.chunks, self.events):
            sparse_attention(ql, kl, vl, bits, block_size, causal=causal, status=self.status,
                             out=buf[:, shard.h_lo:shard.h_hi, lo:hi].permute(0, 2, 1, 3), rows=(lo, hi))
            done.record(cur)
            off = shard.h_lo * pitch + lo * row_bytes
            dsts = (ct.c_void_p * max(1, self._npeers))(*[b + off for b in bases])
            _lib.check(lib.ffts_copy_rows(dsts, self._streams, self._npeers, local + lo * row_bytes, pitch,
                                          (hi - lo) * row_bytes, Hl, done.cuda_event))
        if self._npeers:
            _lib.check(lib.ffts_signal(self._flags, self._streams, self._npeers, e))
        _lib.check(lib.ffts_signal(self._own_flag, (ct.c_void_p * 1)(cur.cuda_stream), 1, e))
        _lib.check(lib.ffts_wait_flags(self.flags.data_ptr(), self.world, e, self.status.data_ptr(),
                                       cur.cuda_stream))
        self.status_word.read_back(cur)
        return buf

    def check(self) -> None:
        """Wait for the device and raise WaitTimeout if any call so far timed out."""
        self.status_word.check()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def close(self):
        """Unmap the peers' buffers (after every rank's last call has completed;
        ``with PeerGather(...) as pg:`` calls it on leaving the block)."""
        torch.cuda.synchronize(self.device)
        for ptr, off in self._opened:
            self.lib.ffts_ipc_close(ptr, off)
        self._opened = []


def sharded_prefill(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, layer_idx: int = 0, *,
                    group=None, out: Optional[torch.Tensor] = None, inputs_are_local: bool = False,
                    global_batch: Optional[int] = None, gather: Optional["PeerGather"] = None,
                    **kwargs) -> torch.Tensor:
    """FFTSparse prefill of the rank's KV groups followed by the output all-gather.

    Returns the head-major output [B, H, L, D] (bf16) on every rank.  The mask
    arguments are those of myattn_prefill.  With ``inputs_are_local`` the q/k/v
    given already hold only this rank's sequences and heads (its units, in rank
    order), as when each rank computes its own columns of the QKV projection;
    ``global_batch`` then gives the total number of sequences (default: the local
    count, no split by sequence), and a split by sequence also needs the global
    ``num_heads`` and ``num_kv_heads``.  With ``gather`` (a PeerGather of this
    group), one sequence split by KV group is gathered on the copy engines,
    overlapped with the attention, and the result is the gather's buffer (valid
    until the call after next) unless ``out`` is given.
    """
    from .prefill import fft_block_mask, sparse_attention

    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    B, H, L, D = q.shape
    if inputs_are_local:
        Bg = global_batch or B
        Hg = kwargs.pop("num_heads", None)
        n_kv = kwargs.pop("num_kv_heads", None)
        if Hg is None or n_kv is None:
            if Bg != B:
                raise ValueError("rank-local inputs split by sequence need num_heads and num_kv_heads")
            Hg = H * world
            n_kv = Hg if k.shape[1] == q.shape[1] else k.shape[1] * world
        shards = [unit_shard(Bg, Hg, n_kv, world, r) for r in range(world)]
        shard = shards[rank]
        B, H = Bg, Hg
        ql, kl, vl = q, k, v
    else:
        # KV groups: k's own head count, or (for repeat_kv-expanded k) num_kv_heads
        n_kv = kwargs.pop("num_kv_heads", None)
        if k.shape[1] != H or n_kv is None:
            n_kv = k.shape[1]
        shards = [unit_shard(B, H, n_kv, world, r) for r in range(world)]
        shard = shards[rank]
        ql, kl, vl = local_views(q, k, v, shard)
    block_size = kwargs.pop("block_size", 128)
    is_causal = kwargs.pop("is_causal", True)
    with trace.layer(layer_idx):
        mask = fft_block_mask(ql, kl, block_size=block_size, **kwargs)
        whole_batch = all(sh.b_lo == 0 and sh.b_hi in (-1, B) for sh in shards)
        if gather is not None and world > 1 and B == 1 and whole_batch:
            # the peer pushes run inside the attention launch and its copy-engine overlap
            with trace.stage("10_kernel+gather"):
                res = gather.run(ql, kl, vl, mask.bits, block_size, is_causal, shard)
            if out is not None:
                out.copy_(res)
                return out
            return res
        if out is None:
            out = torch.empty(B, H, L, D, dtype=torch.bfloat16, device=q.device)
        Bl = ql.shape[0]
        local = out if world == 1 else torch.empty(Bl, shard.heads, L, D, dtype=torch.bfloat16, device=q.device)
        # [Bl, Hl, L, D] storage, written through the kernel's [B, L, H, D] strides
        with trace.stage("10_kernel"):
            sparse_attention(ql, kl, vl, mask.bits, block_size, causal=is_causal, out=local.permute(0, 2, 1, 3))
        if world == 1:
            return out
        with trace.stage("11_gather"):  # no counterpart: the reference runs on one device
            return gather_heads(local, out, group, shards)
