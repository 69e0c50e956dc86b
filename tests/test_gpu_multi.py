"""Multi-GPU exchange over NCCL (needs 2 GPUs on one box; skipped otherwise).

Two ranks hold the same layer; each computes the split partials of its half
of the context tiles straight into its ContextMerge send block, one NCCL
all-gather exchanges the blocks and innerq_lse_merge_ranks merges them.  The
result must equal the single-GPU fused attention over the whole context.  The
KV-head all-gather (HeadGather) must reproduce the full head order."""
import ctypes
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q_out):
    import numpy as np
    import torch.distributed as dist

    from innerq_b200 import _lib
    from innerq_b200.attention import _workspace, build_args, decode_attention, plan
    from innerq_b200.cache import InnerqDynamicLayer
    from innerq_b200.sharding import ContextMerge, HeadGather, chunk_range
    from innerq_b200.store import stream_ptr
    from tests._util import cfg, synth_kv_dev

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev)
    try:
        kw = dict(k_bits=2, v_bits=2, key_flush_size=1, key_normalize=True, key_w_sink=32,
                  value_w_sink=32, key_w_recent=96, value_w_recent=96)
        layer = InnerqDynamicLayer(cfg(**kw), 0)
        k, v = synth_kv_dev(4, 8, 20000, seed=40, device=dev)
        layer.update(k, v)
        g = torch.Generator(device=dev).manual_seed(41)
        q = torch.randn((4, 64, 1, 128), device=dev, generator=g).half()
        full = decode_attention(q, layer.key_side, layer.value_side)
        n_tiles, _ = plan(build_args(q, layer.key_side, layer.value_side))
        lo, hi = chunk_range(n_tiles, world, rank)
        mg = ContextMerge(4, 64, 12, dev)
        args = build_args(q, layer.key_side, layer.value_side, n_splits=12, tile_range=(lo, hi))
        ws = _workspace(dev, _lib.load().innerq_decode_attn_workspace(ctypes.byref(args)))
        _lib.call("innerq_decode_attn_partials", ctypes.byref(args), mg.po.data_ptr(),
                  mg.pm.data_ptr(), mg.pl.data_ptr(), ws.data_ptr(), ws.numel(), stream_ptr(dev))
        merged = torch.empty_like(full)
        mg(merged)
        f, m = full.float(), merged.float()
        err_merge = ((m - f).abs().max() / f.abs().max()).item()
        # KV-head shards: rank r holds query heads [32 r, 32 r + 32)
        hg = HeadGather(full[:, 32 * rank:32 * (rank + 1)].contiguous())
        got = hg().flatten(-3, -2)
        err_heads = (got.float() - f).abs().max().item()
        if rank == 0:
            q_out.put((err_merge, err_heads))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_two_rank_nccl_context_merge_equals_one_gpu():
    ctx = mp.get_context("spawn")
    q_out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q_out)) for r in range(2)]
    for p in procs:
        p.start()
    err_merge, err_heads = q_out.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert err_merge < 2e-3, err_merge
    assert err_heads == 0.0
