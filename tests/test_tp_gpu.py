"""Tensor-parallel block on 2 B200s (NCCL all-reduce inside the block forward).

Skipped when fewer than 2 GPUs are visible.  Each rank runs in its own process
on its own GPU, takes its weight shard (oct_b200.tp.shard_weights) and the
NCCL unique id that rank 0 created; both ranks must produce the full block
output, equal to the binary64 oracle within the block tolerance.
"""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
NORMWISE_TOL = 1e-4


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, family: int, queue) -> None:
    import torch
    import torch.distributed as dist
    from oct_b200 import reactor as R
    from oct_b200 import tp
    from oracle import blocks as OB
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rt = R.Runtime()
        ids = [R.nccl_unique_id(rt.lib) if rank == 0 else None]
        dist.broadcast_object_list(ids, src=0)
        if family == OB.GEMMA:
            cfg, ts = OB.gemma_config(seq_len=128, hidden=512, heads=4, head_dim=128, ffn=1024), None
        else:
            cfg, ts = OB.dit_config(seq_len=256, hidden=512, heads=4, ffn=1024, grid_w=16), [400.0]
        w = OB.random_weights(cfg, seed=21)
        x = np.random.default_rng(22).standard_normal((cfg.seq_len, cfg.hidden)).astype(np.float32)
        shard = tp.shard_weights(cfg.family, cfg.hidden, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.ffn, w, rank,
                                 world)
        rcfg = tp.rank_config(cfg, rank, world)
        fam = R.BLOCK_GEMMA if family == OB.GEMMA else R.BLOCK_DIT
        blk = rt.block(fam, hidden=rcfg.hidden, heads=rcfg.heads, kv_heads=rcfg.kv_heads, head_dim=rcfg.head_dim,
                       ffn=rcfg.ffn, seq_len=rcfg.seq_len, max_batch=1, eps=rcfg.eps, rope_base=rcfg.rope_base,
                       grid_w=rcfg.grid_w, rope_frame=rcfg.rope_frame, tp_rank=rank, tp_world=world,
                       nccl_id=ids[0])
        blk.set_weights(shard)
        y = blk.forward(x, 1, ts)
        blk.close()
        rt.close()
        ref = OB.forward(cfg, w, x, ts)
        queue.put((rank, float(np.max(np.abs(y - ref)) / np.max(np.abs(ref)))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("family", [1, 2])
def test_tp2_block_matches_oracle(family):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, family, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    errs = dict(q.get(timeout=5) for _ in range(2))
    assert max(errs.values()) <= NORMWISE_TOL, errs
