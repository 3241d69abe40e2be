"""Transformer-block parity on the B200 against the binary64 oracle (oracle/blocks.py).

Tolerance (<= 1e-4 per block output), written here:
  normwise relative error max|y - y64| / max|y64| <= 1e-4 for every block output,
  and relative L2 error ||y - y64|| / ||y64|| <= 1e-5.
Cases: reduced dims, the benchmark hidden / head / FFN dims with shorter
sequences, and the two benchmark configurations end to end (Gemma 4 x 1024 at
hidden 2048, DiT 2 x 4096 at hidden 3072; the oracle takes tens of seconds);
both through the device and the host entry points.  Weights include a
non-zero adaLN bias.
"""
from __future__ import annotations

import numpy as np
import pytest

from oct_b200 import reactor as R
from oracle import blocks as OB

pytestmark = pytest.mark.gpu
NORMWISE_TOL = 1e-4
L2_TOL = 1e-5

CASES = {
    "gemma_small": (OB.gemma_config(seq_len=128, hidden=512, heads=4, head_dim=128, ffn=1024), 2),
    "dit_small": (OB.dit_config(seq_len=256, hidden=512, heads=4, ffn=1024, grid_w=16), 2),
    "gemma_baseline_dims": (OB.gemma_config(seq_len=256), 1),
    "dit_baseline_dims": (OB.dit_config(seq_len=256, grid_w=16), 1),
    "dit_seq1024": (OB.dit_config(seq_len=1024, hidden=512, heads=4, ffn=1024, grid_w=32), 2),
    # 256-channel heads take the fused causal CTA-pair attention kernel: one and three query tiles
    "gemma_head256_seq128": (OB.gemma_config(seq_len=128, hidden=512, heads=2, head_dim=256, ffn=1024), 2),
    "gemma_head256_seq384": (OB.gemma_config(seq_len=384, hidden=512, heads=2, head_dim=256, ffn=1024), 2),
    # the benchmark block configurations themselves (Gemma 4 x 1024 at d 2048, DiT 2 x 4096 at d 3072)
    "gemma_baseline_config": (OB.gemma_config(), 4),
    "dit_baseline_config": (OB.dit_config(), 2),
}


def make_block(rt, cfg: OB.BlockConfig, batch: int):
    fam = R.BLOCK_GEMMA if cfg.family == OB.GEMMA else R.BLOCK_DIT
    return rt.block(fam, hidden=cfg.hidden, heads=cfg.heads, kv_heads=cfg.kv_heads, head_dim=cfg.head_dim,
                    ffn=cfg.ffn, seq_len=cfg.seq_len, max_batch=batch, eps=cfg.eps, rope_base=cfg.rope_base,
                    grid_w=cfg.grid_w, rope_frame=cfg.rope_frame)


def errors(y, ref):
    y = y.astype(np.float64).reshape(ref.shape)
    return (float(np.max(np.abs(y - ref)) / np.max(np.abs(ref))),
            float(np.linalg.norm(y - ref) / np.linalg.norm(ref)))


@pytest.mark.parametrize("name", list(CASES))
def test_block_matches_fp64_oracle(runtime, name):
    import torch
    cfg, batch = CASES[name]
    w = OB.random_weights(cfg, seed=11)
    rng = np.random.Generator(np.random.PCG64(12))
    x = rng.standard_normal((batch * cfg.seq_len, cfg.hidden), dtype=np.float32)
    ts = [500.0, 250.0][:batch] if cfg.family == OB.DIT else None
    blk = make_block(runtime, cfg, batch)
    try:
        blk.set_weights(w)
        dx = torch.from_numpy(x).cuda()
        dy = torch.full_like(dx, float("nan"))
        torch.cuda.synchronize()
        blk.forward_device(dx, dy, batch, ts)
        torch.cuda.synchronize()
        assert runtime.sync_status().ok
        y_dev = dy.cpu().numpy()
        y_host = blk.forward(x, batch, ts)
    finally:
        blk.close()
    ref = OB.forward(cfg, w, x, ts)
    nw, l2 = errors(y_dev, ref)
    print(f"{name}: normwise {nw:.3e}  relL2 {l2:.3e}")
    assert np.all(np.isfinite(y_dev))
    assert nw <= NORMWISE_TOL and l2 <= L2_TOL, (nw, l2)
    assert np.array_equal(y_host, y_dev)


def test_block_is_deterministic_and_batch_independent(runtime):
    """A sequence's output does not depend on which batch slot it occupies."""
    cfg, _ = CASES["gemma_small"]
    w = OB.random_weights(cfg, seed=5)
    rng = np.random.Generator(np.random.PCG64(6))
    x = rng.standard_normal((2 * cfg.seq_len, cfg.hidden), dtype=np.float32)
    blk = make_block(runtime, cfg, 2)
    try:
        blk.set_weights(w)
        y2 = blk.forward(x, 2)
        y1 = blk.forward(x[cfg.seq_len:], 1)
        again = blk.forward(x, 2)
    finally:
        blk.close()
    assert np.array_equal(y2[cfg.seq_len:], y1)
    assert np.array_equal(y2, again)


def test_dit_fused_and_materialized_attention_agree(runtime, monkeypatch):
    """The DiT block's fused attention kernel and its materialised path (scores
    in HBM, softmax kernel, two batched products) both meet the oracle bar."""
    import torch
    cfg, batch = CASES["dit_small"]
    w = OB.random_weights(cfg, seed=21)
    rng = np.random.Generator(np.random.PCG64(22))
    x = rng.standard_normal((batch * cfg.seq_len, cfg.hidden), dtype=np.float32)
    ts = [700.0, 100.0]
    outs = {}
    for mode in ("fused", "materialized"):
        monkeypatch.setenv("OCT_B200_DIT_ATTENTION", mode)
        blk = make_block(runtime, cfg, batch)
        try:
            blk.set_weights(w)
            outs[mode] = blk.forward(x, batch, ts)
        finally:
            blk.close()
        assert runtime.sync_status().ok
    ref = OB.forward(cfg, w, x, ts)
    for mode, y in outs.items():
        nw, l2 = errors(y, ref)
        print(f"dit {mode}: normwise {nw:.3e}  relL2 {l2:.3e}")
        assert nw <= NORMWISE_TOL and l2 <= L2_TOL, (mode, nw, l2)


@pytest.mark.parametrize("name", ["gemma_head256_seq384", "gemma_baseline_dims"])
def test_gemma_fused_and_materialized_attention_agree(runtime, monkeypatch, name):
    """The Gemma block's fused causal attention (CTA pair per 128-query tile, 256-channel heads)
    and its materialised path (scores in HBM, causal softmax kernel, two batched products) both
    meet the oracle bar."""
    cfg, batch = CASES[name]
    w = OB.random_weights(cfg, seed=23)
    rng = np.random.Generator(np.random.PCG64(24))
    x = rng.standard_normal((batch * cfg.seq_len, cfg.hidden), dtype=np.float32)
    outs = {}
    for mode in ("fused", "materialized"):
        monkeypatch.setenv("OCT_B200_GEMMA_ATTENTION", mode)
        blk = make_block(runtime, cfg, batch)
        try:
            blk.set_weights(w)
            outs[mode] = blk.forward(x, batch)
        finally:
            blk.close()
        assert runtime.sync_status().ok
    ref = OB.forward(cfg, w, x)
    for mode, y in outs.items():
        nw, l2 = errors(y, ref)
        print(f"{name} {mode}: normwise {nw:.3e}  relL2 {l2:.3e}")
        assert nw <= NORMWISE_TOL and l2 <= L2_TOL, (mode, nw, l2)
