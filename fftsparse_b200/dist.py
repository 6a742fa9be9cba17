"""KV-group sharded FFTSparse prefill over NCCL (one process per GPU).

The reference has no distributed path: multi-GPU use there is accelerate's
``device_map="auto"`` layer placement (eval/LongBench/pred.py:520).  Every step
of the operator is independent per head, and heads that share a key/value head
(a GQA group) also share its K/V tiles, so the unit of work is the
(sequence, KV group).  Each rank runs pooling, mask selection and attention
for its contiguous slice of KV groups with no communication, and one
all-gather assembles the head-major output [B, H, L, D] that o_proj consumes.

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

    @property
    def heads(self) -> int:
        return self.h_hi - self.h_lo


def kv_group_shard(num_heads: int, num_kv_heads: int, world: int, rank: int) -> Shard:
    """Contiguous slice of KV groups owned by ``rank``; requires Hkv % world == 0."""
    if num_heads % num_kv_heads:
        raise ValueError(f"H={num_heads} is not a multiple of Hkv={num_kv_heads}")
    if num_kv_heads % world:
        raise ValueError(f"{num_kv_heads} KV groups cannot be split evenly over {world} ranks")
    per = num_kv_heads // world
    rep = num_heads // num_kv_heads
    kv_lo, kv_hi = rank * per, (rank + 1) * per
    return Shard(rank, world, kv_lo, kv_hi, kv_lo * rep, kv_hi * rep)


def local_views(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, shard: Shard):
    """Views of the rank's heads: q [B, Hl, L, D]; k/v [B, Hkvl, L, D] (or the
    matching q-head slice when k/v are repeat_kv-expanded to H heads)."""
    H, Hk = q.shape[1], k.shape[1]
    qs = q[:, shard.h_lo:shard.h_hi]
    if Hk == H:
        ks, vs = k[:, shard.h_lo:shard.h_hi], v[:, shard.h_lo:shard.h_hi]
    else:
        ks, vs = k[:, shard.kv_lo:shard.kv_hi], v[:, shard.kv_lo:shard.kv_hi]
    return qs, ks, vs


def gather_heads(local_out: torch.Tensor, full_out: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather head-major shards [B, Hl, L, D] into [B, H, L, D] (B == 1 uses one
    ncclAllGather straight into the output; B > 1 gathers rank-major then permutes)."""
    world = dist.get_world_size(group)
    B = local_out.shape[0]
    if world == 1:
        full_out.copy_(local_out)
        return full_out
    if B == 1:
        dist.all_gather_into_tensor(full_out.view(-1), local_out.reshape(-1), group=group)
        return full_out
    tmp = torch.empty((world,) + tuple(local_out.shape), dtype=local_out.dtype, device=local_out.device)
    dist.all_gather_into_tensor(tmp.view(-1), local_out.reshape(-1), group=group)
    full_out.copy_(tmp.permute(1, 0, 2, 3, 4).reshape(full_out.shape))
    return full_out


def sharded_prefill(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, layer_idx: int = 0, *,
                    group=None, out: Optional[torch.Tensor] = None, inputs_are_local: bool = False,
                    **kwargs) -> torch.Tensor:
    """FFTSparse prefill of the rank's KV groups followed by the output all-gather.

    Returns the head-major output [B, H, L, D] (bf16) on every rank.  The mask
    arguments are those of myattn_prefill.  With ``inputs_are_local`` the q/k/v
    given already hold only this rank's heads (its KV groups, in rank order), as
    when each rank computes its own columns of the QKV projection.
    """
    from .prefill import fft_block_mask, sparse_attention

    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    B, H, L, D = q.shape
    if inputs_are_local:
        kwargs.pop("num_kv_heads", None)
        H = H * world
        shard = kv_group_shard(H, k.shape[1] * world if k.shape[1] != q.shape[1] else H, world, rank)
        ql, kl, vl = q, k, v
    else:
        # KV groups: k's own head count, or (for repeat_kv-expanded k) num_kv_heads
        n_kv = kwargs.pop("num_kv_heads", None)
        if k.shape[1] != H or n_kv is None:
            n_kv = k.shape[1]
        shard = kv_group_shard(H, n_kv, world, rank)
        ql, kl, vl = local_views(q, k, v, shard)
    block_size = kwargs.pop("block_size", 128)
    is_causal = kwargs.pop("is_causal", True)
    mask = fft_block_mask(ql, kl, block_size=block_size, **kwargs)
    if out is None:
        out = torch.empty(B, H, L, D, dtype=torch.bfloat16, device=q.device)
    local = out if world == 1 else torch.empty(B, shard.heads, L, D, dtype=torch.bfloat16, device=q.device)
    # [B, Hl, L, D] storage, written through the kernel's [B, L, H, D] strides
    sparse_attention(ql, kl, vl, mask.bits, block_size, causal=is_causal, out=local.permute(0, 2, 1, 3))
    if world == 1:
        return out
    return gather_heads(local, out, group)
