"""Multi-GPU partitioning of the decode attention (one process per GPU).

Two partitions, neither present in the reference (which is single-GPU,
``scripts/run_lmeval.sh:2``):

* by KV head: rank r owns KV heads ``head_shard(Hkv, world, r)`` with their
  query heads; attention needs no exchange, and the per-rank outputs
  ``[B, Hq/world, D]`` are all-gathered once (in a tensor-parallel model this
  folds into the o_proj all-reduce);
* by context chunk (long contexts, or more GPUs than KV heads): rank r owns a
  contiguous range of 32-token tiles, emits split-KV partials (O, m, l), and
  the partials are all-gathered and merged with the log-sum-exp merge kernel.

The collectives are ``torch.distributed`` (NCCL over NVLink on the GPU box;
gloo in the CPU tests).  The merge function is a parameter so the exchange
logic can be tested on CPU ranks with the oracle merge.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def head_shard(n_kv_heads: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous KV-head range [lo, hi) of a rank; heads must divide evenly."""
    if n_kv_heads % world:
        raise ValueError(f"{n_kv_heads} KV heads do not split over {world} ranks")
    per = n_kv_heads // world
    return rank * per, (rank + 1) * per


def chunk_range(n_items: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous, near-equal range [lo, hi) of n_items (tiles) for a rank."""
    base, extra = divmod(n_items, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def gather_heads(out_local: torch.Tensor, group=None) -> torch.Tensor:
    """[..., Hq_local, D] per rank -> [..., Hq, D] in rank (head) order
    (allocating; HeadGather is the per-step form)."""
    return HeadGather(out_local, group)().flatten(-3, -2)


class HeadGather:
    """The per-step all-gather of the KV-head shards' attention outputs,
    with its buffer allocated once: one all_gather_into_tensor of the local
    [..., Hq_local, D] block into a [world, ..., Hq_local, D] buffer.
    ``heads()`` views it as [..., world, Hq_local, D] (query head
    r * Hq_local + j at [..., r, j, :]), with no copy."""

    def __init__(self, out_local: torch.Tensor, group=None):
        self.src = out_local
        self.group = group
        self.world = dist.get_world_size(group)
        # concatenated along dim 0 (the form every backend takes), viewed as
        # [world, ...]
        shape = tuple(out_local.shape)
        self.flat = out_local.new_empty((self.world * shape[0],) + shape[1:])
        self.buf = self.flat.view((self.world,) + shape)

    def __call__(self) -> torch.Tensor:
        """Gather; returns the [..., world, Hq_local, D] view of the buffer."""
        dist.all_gather_into_tensor(self.flat, self.src.contiguous(), group=self.group)
        return self.heads()

    def heads(self) -> torch.Tensor:
        nd = self.buf.dim()
        return self.buf.permute(*range(1, nd - 2), 0, nd - 2, nd - 1)


def merge_context_partials(po: torch.Tensor, pm: torch.Tensor, pl: torch.Tensor, dtype,
                           group=None, merge_fn=None) -> torch.Tensor:
    """All-gather each rank's split partials (po [B,Hq,s,D], pm/pl [B,Hq,s];
    the split count may differ per rank) and merge them into [B, Hq, D]."""
    world = dist.get_world_size(group)
    s_local = torch.tensor([po.shape[2]], dtype=torch.int64, device=po.device)
    sizes = [torch.zeros_like(s_local) for _ in range(world)]
    dist.all_gather(sizes, s_local, group=group)
    smax = int(max(x.item() for x in sizes))
    B, Hq, s, D = po.shape
    pad_o = po.new_zeros((B, Hq, smax, D))
    pad_m = pm.new_full((B, Hq, smax), float("-inf"))
    pad_l = pl.new_zeros((B, Hq, smax))
    pad_o[:, :, :s] = po
    pad_m[:, :, :s] = pm
    pad_l[:, :, :s] = pl
    go = [torch.empty_like(pad_o) for _ in range(world)]
    gm = [torch.empty_like(pad_m) for _ in range(world)]
    gl = [torch.empty_like(pad_l) for _ in range(world)]
    dist.all_gather(go, pad_o, group=group)
    dist.all_gather(gm, pad_m, group=group)
    dist.all_gather(gl, pad_l, group=group)
    po_all, pm_all, pl_all = torch.cat(go, 2), torch.cat(gm, 2), torch.cat(gl, 2)
    if merge_fn is None:
        from .attention import lse_merge
        merge_fn = lse_merge
    return merge_fn(po_all, pm_all, pl_all, dtype)
