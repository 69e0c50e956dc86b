"""Multi-rank exchange logic on CPU gloo ranks (world size 2): KV-head shards
gathered, and context-chunk split partials gathered and log-sum-exp merged,
both equal to single-rank attention.  The per-rank compute is the oracle."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from innerq_b200.sharding import chunk_range, head_shard


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _data():
    rng = np.random.default_rng(0)
    q = rng.standard_normal((2, 8, 1, 64))
    k = rng.standard_normal((2, 2, 200, 64)) * 2
    v = rng.standard_normal((2, 2, 200, 64))
    return q, k, v


def _partials(q, k, v, lo, hi):
    """Unnormalised split partials (log2 domain) of tokens [lo, hi)."""
    rep = q.shape[1] // k.shape[1]
    kk = np.repeat(k, rep, axis=1)[:, :, lo:hi]
    vv = np.repeat(v, rep, axis=1)[:, :, lo:hi]
    x = np.einsum("bhqd,bhsd->bhs", q, kk) / np.sqrt(q.shape[-1]) / np.log(2)
    m = x.max(-1)
    p = np.exp2(x - m[..., None])
    return (torch.from_numpy(np.einsum("bhs,bhsd->bhd", p, vv)[:, :, None]),
            torch.from_numpy(m[..., None]), torch.from_numpy(p.sum(-1)[..., None]))


def _merge_np(po, pm, pl, dtype):
    M = pm.max(-1, keepdim=True).values
    w = torch.exp2(pm - M)
    return (po * w[..., None]).sum(2) / (pl * w).sum(-1)[..., None]


def _worker(rank, world, port, q_out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from innerq_b200.sharding import gather_heads, merge_context_partials
    from oracle.cache_ref import attention
    q, k, v = _data()
    # context sharding: each rank a contiguous token range (uneven on purpose)
    lo, hi = chunk_range(200, world, rank)
    po, pm, pl = _partials(q, k, v, lo, hi)
    merged = merge_context_partials(po, pm, pl, torch.float64, merge_fn=_merge_np)
    # head sharding: each rank its KV heads and their query heads
    h0, h1 = head_shard(2, world, rank)
    rep = q.shape[1] // k.shape[1]
    o_loc, _ = attention(q[:, h0 * rep:h1 * rep], k[:, h0:h1], v[:, h0:h1])
    gathered = gather_heads(torch.from_numpy(o_loc[:, :, 0]))
    if rank == 0:
        full, _ = attention(q, k, v)
        q_out.put((np.abs(merged.numpy() - full[:, :, 0]).max(),
                   np.abs(gathered.numpy() - full[:, :, 0]).max()))
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_merge_and_gather():
    ctx = mp.get_context("spawn")
    q_out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q_out)) for r in range(2)]
    for p in procs:
        p.start()
    e_merge, e_gather = q_out.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert e_merge < 1e-12 and e_gather < 1e-12


def test_ranges():
    assert head_shard(8, 4, 3) == (6, 8)
    with pytest.raises(ValueError):
        head_shard(8, 3, 0)
    spans = [chunk_range(1029, 8, r) for r in range(8)]
    assert spans[0][0] == 0 and spans[-1][1] == 1029
    assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    assert max(h - l for l, h in spans) - min(h - l for l, h in spans) <= 1
