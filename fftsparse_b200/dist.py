"""(Sequence, KV-group) sharded FFTSparse prefill over NCCL (one process per GPU).

The reference has no distributed path: multi-GPU use there is accelerate's
``device_map="auto"`` layer placement (eval/LongBench/pred.py:520).  Every step
of the operator is independent per head, and heads that share a key/value head
(a GQA group) also share its K/V tiles, so the unit of work is the
(sequence, KV group).  Each rank runs pooling, mask selection and attention
for its contiguous slice of KV groups with no communication, and one
all-gather assembles the head-major output [B, H, L, D] that o_proj consumes.
When the KV groups are fewer than the ranks (2 sequences x
4 KV groups on 8 GPUs), the units are (sequence, KV group) pairs, ordered
sequence-major, and a rank owns a contiguous run of them.

Functions here take the full q/k/v (or any rank-local copy of them) and slice
the rank's heads as views; nothing is copied before the kernels run.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist


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


def sharded_prefill(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, layer_idx: int = 0, *,
                    group=None, out: Optional[torch.Tensor] = None, inputs_are_local: bool = False,
                    global_batch: Optional[int] = None, **kwargs) -> torch.Tensor:
    """FFTSparse prefill of the rank's KV groups followed by the output all-gather.

    Returns the head-major output [B, H, L, D] (bf16) on every rank.  The mask
    arguments are those of myattn_prefill.  With ``inputs_are_local`` the q/k/v
    given already hold only this rank's sequences and heads (its units, in rank
    order), as when each rank computes its own columns of the QKV projection;
    ``global_batch`` then gives the total number of sequences (default: the local
    count, no split by sequence), and a split by sequence also needs the global
    ``num_heads`` and ``num_kv_heads``.
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
    mask = fft_block_mask(ql, kl, block_size=block_size, **kwargs)
    if out is None:
        out = torch.empty(B, H, L, D, dtype=torch.bfloat16, device=q.device)
    Bl = ql.shape[0]
    local = out if world == 1 else torch.empty(Bl, shard.heads, L, D, dtype=torch.bfloat16, device=q.device)
    # [Bl, Hl, L, D] storage, written through the kernel's [B, L, H, D] strides
    sparse_attention(ql, kl, vl, mask.bits, block_size, causal=is_causal, out=local.permute(0, 2, 1, 3))
    if world == 1:
        return out
    return gather_heads(local, out, group, shards)
