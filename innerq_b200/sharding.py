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


def _pack(po, pm, pl):
    return torch.cat([po.reshape(-1), pm.reshape(-1), pl.reshape(-1)])


def _unpack(block, B, Hq, s, D):
    rows = B * Hq * s
    return (block[:rows * D].view(B, Hq, s, D), block[rows * D:rows * (D + 1)].view(B, Hq, s),
            block[rows * (D + 1):rows * (D + 2)].view(B, Hq, s))


def merge_context_partials(po: torch.Tensor, pm: torch.Tensor, pl: torch.Tensor, dtype,
                           group=None, merge_fn=None) -> torch.Tensor:
    """Gather every rank's split partials (po [B,Hq,s,D], pm/pl [B,Hq,s], the
    same split count s on every rank: pass n_splits explicitly) with ONE
    all-gather of a packed block per rank, then merge them into [B, Hq, D]:
    by merge_fn(po_all, pm_all, pl_all, dtype) when given (CPU ranks), else
    by the CUDA rank-block merge, which reads the gathered blocks in place."""
    world = dist.get_world_size(group)
    B, Hq, s, D = po.shape
    send = _pack(po, pm, pl)
    recv = send.new_empty((world * send.numel(),))
    dist.all_gather_into_tensor(recv, send, group=group)
    if merge_fn is not None:
        parts = [_unpack(recv[w * send.numel():(w + 1) * send.numel()], B, Hq, s, D)
                 for w in range(world)]
        return merge_fn(torch.cat([p[0] for p in parts], 2), torch.cat([p[1] for p in parts], 2),
                        torch.cat([p[2] for p in parts], 2), dtype)
    out = torch.empty((B, Hq, D), dtype=dtype, device=po.device)
    merge_rank_blocks(recv, world, send.numel(), B, Hq, s, out)
    return out


def merge_rank_blocks(recv: torch.Tensor, world: int, block: int, B: int, Hq: int, s: int,
                      out: torch.Tensor) -> torch.Tensor:
    """innerq_lse_merge_ranks over `world` gathered partials blocks."""
    from . import _lib
    from .store import dtype_code, stream_ptr
    _lib.call("innerq_lse_merge_ranks", recv.data_ptr(), world, block, B, Hq, s, out.shape[-1],
              dtype_code(out.dtype), out.data_ptr(), out.stride(0), out.stride(1), None,
              stream_ptr(recv.device))
    return out


class ContextMerge:
    """The per-layer exchange of a context-sharded layer, buffers allocated
    once: this rank's attention writes its split partials straight into
    ``po`` / ``pm`` / ``pl`` (views of one packed send block), ``__call__``
    gathers the blocks of all ranks of ``group`` with one
    all_gather_into_tensor and merges them into ``out`` with one launch."""

    def __init__(self, B: int, Hq: int, n_splits: int, device, group=None, D: int = 128):
        self.group = group
        self.world = dist.get_world_size(group)
        self.B, self.Hq, self.s, self.D = B, Hq, n_splits, D
        self.block = B * Hq * n_splits * (D + 2)
        self.send = torch.empty(self.block, dtype=torch.float32, device=device)
        self.recv = torch.empty(self.world * self.block, dtype=torch.float32, device=device)
        self.po, self.pm, self.pl = _unpack(self.send, B, Hq, n_splits, D)

    def __call__(self, out: torch.Tensor) -> torch.Tensor:
        dist.all_gather_into_tensor(self.recv, self.send, group=self.group)
        return merge_rank_blocks(self.recv, self.world, self.block, self.B, self.Hq, self.s, out)
