"""Tensor-parallel host logic on CPU: world_size-2 gloo ranks.

Each rank takes its weight shard (oct_b200.tp.shard_weights), runs the binary64
block restatement with its heads / FFN share and sums the two row-parallel
partials with a gloo all-reduce; the result must equal the unsharded block.
This pins the sharding layout the GPU block consumes, with no GPU.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, family: int, queue) -> None:
    import torch
    import torch.distributed as dist
    from oct_b200 import tp
    from oracle import blocks as OB
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        if family == OB.GEMMA:
            cfg = OB.gemma_config(seq_len=32, hidden=128, heads=4, head_dim=32, ffn=256)
            ts = None
        else:
            cfg = OB.dit_config(seq_len=64, hidden=256, heads=4, ffn=256, grid_w=8)
            ts = [300.0]
        w = OB.random_weights(cfg, seed=3)
        x = np.random.default_rng(4).standard_normal((cfg.seq_len, cfg.hidden)).astype(np.float32)
        shard = tp.shard_weights(cfg.family, cfg.hidden, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.ffn, w, rank,
                                 world)
        rcfg = tp.rank_config(cfg, rank, world)

        def all_reduce(a):
            t = torch.from_numpy(np.ascontiguousarray(a))
            dist.all_reduce(t)
            return t.numpy()

        y_tp = OB.forward(rcfg, shard, x, ts, all_reduce)
        y_full = OB.forward(cfg, w, x, ts)
        queue.put((rank, float(np.max(np.abs(y_tp - y_full)) / np.max(np.abs(y_full)))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("family", [1, 2])
def test_tp_sharding_reproduces_the_full_block(family):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, family, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    errs = dict(q.get(timeout=5) for _ in range(2))
    assert max(errs.values()) < 1e-12, errs


def test_shard_shapes_and_divisibility():
    from oct_b200 import tp
    from oracle import blocks as OB
    cfg = OB.gemma_config(seq_len=16, hidden=64, heads=8, head_dim=16, ffn=128)
    w = OB.random_weights(cfg, 1)
    s = tp.shard_weights(cfg.family, cfg.hidden, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.ffn, w, 1, 4)
    assert s["wqkv"].shape == (64, (2 + 2) * 16) and s["wo"].shape == (32, 64)
    assert s["wgu"].shape == (64, 64) and s["wd"].shape == (32, 64)
    assert np.array_equal(s["wqkv"][:, 32:], w["wqkv"][:, 128:])  # replicated MQA K|V
    with pytest.raises(ValueError):
        tp.shard_weights(cfg.family, cfg.hidden, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.ffn, w, 0, 3)


def _sgemm_rank_main(rank: int, world: int, port: int, queue) -> None:
    """Column-parallel SGEMM host logic: shard B by columns, multiply locally with the
    oracle (binary64 accumulation), all-gather the slabs [w][m][n/w] over gloo and
    repack them to row-major C, as oct_b200_sgemm_tp_device does on the GPUs."""
    import torch
    import torch.distributed as dist
    from oct_b200 import tp
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        m, n, k = 37, 48, 29  # ragged m and k; n a multiple of 4 * world
        rng = np.random.default_rng(8)
        a = rng.uniform(-1, 1, (m, k)).astype(np.float32)  # replicated
        b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
        part = tp.shard_columns(b, rank, world)
        slab = torch.from_numpy(a.astype(np.float64) @ part.astype(np.float64))
        slabs = [torch.empty_like(slab) for _ in range(world)]
        dist.all_gather(slabs, slab)
        c = tp.gather_columns(torch.stack(slabs)).numpy()
        full = a.astype(np.float64) @ b.astype(np.float64)
        queue.put((rank, bool(np.array_equal(c, full)), part.shape))
    finally:
        dist.destroy_process_group()


def test_column_parallel_sgemm_layout_world2():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_sgemm_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = dict((r, (ok, shape)) for r, ok, shape in (q.get(timeout=5) for _ in range(2)))
    assert all(ok for ok, _ in res.values()), res
    assert all(shape == (29, 24) for _, shape in res.values())


def test_column_shard_helpers():
    from oct_b200 import tp
    b = np.arange(6 * 32, dtype=np.float32).reshape(6, 32)
    parts = [tp.shard_columns(b, r, 4) for r in range(4)]
    assert all(p.shape == (6, 8) and p.flags.c_contiguous for p in parts)
    assert np.array_equal(tp.gather_columns(np.stack(parts)), b)
    with pytest.raises(ValueError):
        tp.shard_columns(b, 0, 3)  # 32 is not a multiple of 12
    with pytest.raises(ValueError):
        tp.check_columns(40, 4)
