"""Tensor-parallel block on 2, 4 and 8 B200s (the fused peer-memory collective and
NCCL all-reduce inside the block forward).

Each world size is skipped when fewer GPUs are visible.  Each rank runs in its
own process on its own GPU, takes its weight shard (oct_b200.tp.shard_weights)
and the NCCL unique id that rank 0 created for each block; every rank must
produce the full block output, equal to the binary64 oracle within the block
tolerance (normwise <= 1e-4), the same on every rank and repeatable.  The
configurations have 8 query heads so that every world size divides them
(tp = 8 leaves one head per rank; the Gemma KV head is replicated).
"""
from __future__ import annotations

import hashlib
import os
import queue
import socket
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
NORMWISE_TOL = 1e-4
# (family, batch): Gemma at batch 1, DiT at batch 1 and 2
CASES = ((1, 1), (2, 1), (2, 2))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _case_config(family: int):
    from oracle import blocks as OB
    if family == OB.GEMMA:
        return OB.gemma_config(seq_len=128, hidden=1024, heads=8, head_dim=128, ffn=2048)
    return OB.dit_config(seq_len=256, hidden=1024, heads=8, ffn=2048, grid_w=16)


def _rank_main(rank: int, world: int, port: int, collective: str, queue) -> None:
    os.environ["OCT_B200_TP_COLLECTIVE"] = collective
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
        ids = [[R.nccl_unique_id(rt.lib) for _ in CASES] if rank == 0 else None]
        dist.broadcast_object_list(ids, src=0)
        out = []
        for i, (family, batch) in enumerate(CASES):
            cfg = _case_config(family)
            ts = [400.0, 90.0][:batch] if family == OB.DIT else None
            w = OB.random_weights(cfg, seed=21)
            x = np.random.default_rng(22).standard_normal((batch * cfg.seq_len, cfg.hidden)).astype(np.float32)
            shard = tp.shard_weights(cfg.family, cfg.hidden, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.ffn, w,
                                     rank, world)
            rcfg = tp.rank_config(cfg, rank, world)
            fam = R.BLOCK_GEMMA if family == OB.GEMMA else R.BLOCK_DIT
            blk = rt.block(fam, hidden=rcfg.hidden, heads=rcfg.heads, kv_heads=rcfg.kv_heads,
                           head_dim=rcfg.head_dim, ffn=rcfg.ffn, seq_len=rcfg.seq_len, max_batch=batch, eps=rcfg.eps,
                           rope_base=rcfg.rope_base, grid_w=rcfg.grid_w, rope_frame=rcfg.rope_frame, tp_rank=rank,
                           tp_world=world, nccl_id=ids[0][i])
            blk.set_weights(shard)
            y = blk.forward(x, batch, ts)
            again = blk.forward(x, batch, ts)  # a second forward reuses every buffer and flag
            blk.close()
            ok = rt.sync_status().ok
            ref = OB.forward(cfg, w, x, ts)
            err = float(np.max(np.abs(y - ref)) / np.max(np.abs(ref)))
            # a digest, not the array: a child cannot exit while a large queue item is unflushed
            out.append((err, bool(np.array_equal(y, again)) and ok, hashlib.sha256(y.tobytes()).hexdigest()))
        rt.close()
        queue.put((rank, out))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("collective", ["fused", "nccl"])
@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_block_matches_oracle(world, collective):
    """Both collectives: the fused peer-memory path (row scatter in the GEMM epilogue,
    owner-side reduce + push) and NCCL all-reduce; every rank must hold the same full
    output, equal to the oracle within the block tolerance."""
    import torch
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, collective, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = {}
    try:
        deadline = time.time() + 600
        while len(res) < world and time.time() < deadline:  # drain the queue before joining
            try:
                rank, r = q.get(timeout=2)
                res[rank] = r
            except queue.Empty:
                if any(p.exitcode not in (None, 0) for p in procs):
                    break
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert all(p.exitcode == 0 for p in procs) and len(res) == world, [p.exitcode for p in procs]
    for i, case in enumerate(CASES):
        errs = [res[r][i][0] for r in range(world)]
        print(f"world {world} {collective} case {case}: normwise {max(errs):.3e}")
        assert max(errs) <= NORMWISE_TOL, (case, errs)
        assert all(res[r][i][1] for r in range(world)), case  # repeatable, status clean
        assert len({res[r][i][2] for r in range(world)}) == 1, case  # replicated output
