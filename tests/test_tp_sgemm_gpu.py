"""Column-parallel SGEMM (oct_b200_sgemm_tp_device) on 2, 4 and 8 B200s.

Each world size is skipped when fewer GPUs are visible.  Each rank runs in its
own process on its own GPU with the same A and its column block of B
(oct_b200.tp.shard_columns), over both collectives (epilogue peer stores and
NCCL all-gather + repack).  Every rank must hold all of C:
  * equal to the binary64 product within the SGEMM bar (normwise <= 1e-5);
  * bit-identical on every rank, and its own column block bit-identical to a
    one-GPU 3xTF32 product of A and that block (the same kernel);
  * the library's own copy (out_result) equal to the caller's C, and a strided
    C (ldc > n) leaving the columns past n untouched;
  * repeated calls (the alternating output buffers) reproducible.
Shapes have ragged m and k.
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
NORMWISE_TOL = 1e-5
SHAPES = ((1000, 2048, 1023), (257, 1024, 640), (64, 256, 96))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, collective: int, queue) -> None:
    import torch
    import torch.distributed as dist
    from oct_b200 import reactor as R
    from oct_b200 import tp
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rt = R.Runtime()
        ids = [R.nccl_unique_id(rt.lib) if rank == 0 else None]
        dist.broadcast_object_list(ids, src=0)
        t = rt.tp_sgemm(rank, world, max_m=1024, max_n=2048, nccl_id=ids[0], collective=collective)
        out = {"collective": t.collective, "cases": []}
        for m, n, k in SHAPES:
            rng = np.random.default_rng(m + n + k)
            a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
            b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
            nr = n // world
            da = torch.from_numpy(a).cuda()
            db = torch.from_numpy(tp.shard_columns(b, rank, world)).cuda()
            dc = torch.full((m, n), float("nan"), device="cuda")
            res_ptr = t.run_device(da, db, dc, m, n, k)
            # strided C: ldc = n + 12, columns past n must stay as written
            ds = torch.full((m, n + 12), -7.0, device="cuda")
            second_ptr = t.run_device(da, db, ds, m, n, k, ldc=n + 12)
            again_ptr = t.run_device(da, db, None, m, n, k)  # the library's copy only
            status = t.sync()
            # read the library's copy exactly: an FMA product with the identity
            eye = torch.eye(n, device="cuda")
            lib_copy = torch.empty(m, n, device="cuda")
            rt.sgemm_device(again_ptr, eye, lib_copy, m, n, n, R.SGEMM_FMA)
            # this rank's column block on one GPU, the same 3xTF32 kernel
            own = torch.empty(m, nr, device="cuda")
            rt.sgemm_device(da, db, own, m, nr, k, R.SGEMM_TC_BK16)
            torch.cuda.synchronize()
            c = dc.cpu().numpy()
            ref = a.astype(np.float64) @ b.astype(np.float64)
            out["cases"].append({
                "err": float(np.max(np.abs(c - ref)) / np.max(np.abs(ref))),
                "digest": hashlib.sha256(c.tobytes()).hexdigest(),
                "own_block_equal": bool(torch.equal(dc[:, rank * nr:(rank + 1) * nr], own)),
                "strided_equal": bool(torch.equal(ds[:, :n], dc)) and bool((ds[:, n:] == -7.0).all()),
                "copy_equal": bool(torch.equal(lib_copy, dc)),
                "status": status,
                # consecutive calls alternate between two output buffers
                "distinct_buffers": res_ptr != second_ptr and res_ptr == again_ptr and res_ptr != 0,
            })
        t.close()
        rt.close()
        queue.put((rank, out))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("collective", [1, 2], ids=["peer", "nccl"])
@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_sgemm_matches_oracle(world, collective):
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
        while len(res) < world and time.time() < deadline:
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
    assert all(r["collective"] == collective for r in res.values()), res
    for i, shape in enumerate(SHAPES):
        cases = [res[r]["cases"][i] for r in range(world)]
        print(f"world {world} collective {collective} {shape}: normwise {max(c['err'] for c in cases):.3e}")
        assert max(c["err"] for c in cases) <= NORMWISE_TOL, (shape, cases)
        assert len({c["digest"] for c in cases}) == 1, shape  # every rank holds the same C
        for c in cases:
            assert c["own_block_equal"] and c["strided_equal"] and c["copy_equal"], (shape, c)
            assert c["status"] == 0 and c["distinct_buffers"], (shape, c)
