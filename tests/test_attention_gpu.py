"""Fused attention kernel (attention.cu) against the binary64 oracle attention.

The kernel is the exact bidirectional attention of the Z-Image block
(`canonicalAttention`, internal/prometheus/zimage/canonical_reference.go:241-289),
called through the C ABI entry `oct_b200_attention_device` with the reference's
token-major [token][head][channel] layout.

Tolerance, written here: relative L2 error ||o - o64|| / ||o64|| <= 2e-6 and
normwise max|o - o64| / max|o64| <= 1e-5, and never more than 2x the error of a
plain fp32 CPU evaluation (numpy float32) of the same attention + 1e-7.
Cases cover one query tile, several heads and items, the DiT sequence length
(4096), scores large enough that the running max moves in every key block, and
a max that arrives in the last key block.
"""
from __future__ import annotations

import zlib

import numpy as np
import pytest

from oracle import blocks as OB

pytestmark = pytest.mark.gpu
L2_TOL = 2e-6
NORMWISE_TOL = 1e-5


def _inputs(items, seq, heads, seed, spread=1.0, rising=False):
    rng = np.random.Generator(np.random.PCG64(seed))
    shape = (items * seq, heads * 128)
    q = rng.standard_normal(shape, dtype=np.float32)
    k = rng.standard_normal(shape, dtype=np.float32) * np.float32(spread)
    v = rng.standard_normal(shape, dtype=np.float32)
    if rising:
        # key norms grow with position: the running max changes in the last block
        ramp = np.tile(np.linspace(0.25, 3.0, seq, dtype=np.float32), items)[:, None]
        k = (k * ramp).astype(np.float32)
    return q, k, v


def _oracle(q, k, v, items, seq, heads, scale):
    out = np.empty(q.shape, dtype=np.float64)
    for it in range(items):
        sl = slice(it * seq, (it + 1) * seq)
        out[sl] = OB.attention(q[sl].astype(np.float64).reshape(seq, heads, 128),
                               k[sl].astype(np.float64).reshape(seq, heads, 128),
                               v[sl].astype(np.float64).reshape(seq, heads, 128), float(scale), False)
    return out


def _fp32_cpu(q, k, v, items, seq, heads, scale):
    out = np.empty(q.shape, dtype=np.float32)
    for it in range(items):
        sl = slice(it * seq, (it + 1) * seq)
        for h in range(heads):
            hs = slice(h * 128, (h + 1) * 128)
            s = (q[sl, hs] @ k[sl, hs].T) * np.float32(scale)
            s = np.exp(s - s.max(axis=1, keepdims=True))
            s /= s.sum(axis=1, keepdims=True, dtype=np.float32)
            out[sl, hs] = s @ v[sl, hs]
    return out


def _errors(o, ref):
    o = o.astype(np.float64)
    return (float(np.linalg.norm(o - ref) / np.linalg.norm(ref)),
            float(np.max(np.abs(o - ref)) / np.max(np.abs(ref))))


CASES = {
    "one_tile": (1, 128, 1, {}),
    "items_heads": (2, 256, 3, {}),
    "seq1024_spread": (1, 1024, 2, {"spread": 4.0}),
    "late_max": (1, 512, 2, {"rising": True}),
    "dit_seq4096": (2, 4096, 1, {}),
}


@pytest.mark.parametrize("name", list(CASES))
def test_fused_attention_matches_oracle(runtime, name):
    import torch
    items, seq, heads, kw = CASES[name]
    q, k, v = _inputs(items, seq, heads, seed=zlib.crc32(name.encode()) % 1000, **kw)
    scale = np.float32(1.0) / np.sqrt(np.float32(128))
    dq, dk, dv = (torch.from_numpy(a).cuda() for a in (q, k, v))
    do = torch.full_like(dq, float("nan"))
    torch.cuda.synchronize()
    runtime.attention_device(dq, dk, dv, do, items, seq, heads, 128, float(scale))
    torch.cuda.synchronize()
    assert runtime.sync_status().ok
    o = do.cpu().numpy()
    assert np.all(np.isfinite(o))
    ref = _oracle(q, k, v, items, seq, heads, scale)
    l2, nw = _errors(o, ref)
    l2_cpu, nw_cpu = _errors(_fp32_cpu(q, k, v, items, seq, heads, scale), ref)
    print(f"{name}: relL2 {l2:.3e} (fp32 cpu {l2_cpu:.3e})  normwise {nw:.3e} (fp32 cpu {nw_cpu:.3e})")
    assert l2 <= L2_TOL and nw <= NORMWISE_TOL, (l2, nw)
    assert l2 <= 2 * l2_cpu + 1e-7, (l2, l2_cpu)


def test_fused_attention_is_deterministic_and_item_independent(runtime):
    import torch
    items, seq, heads = 2, 256, 2
    q, k, v = _inputs(items, seq, heads, seed=3)
    dq, dk, dv = (torch.from_numpy(a).cuda() for a in (q, k, v))
    o2 = torch.empty_like(dq)
    again = torch.empty_like(dq)
    o1 = torch.empty((seq, heads * 128), device="cuda")
    runtime.attention_device(dq, dk, dv, o2, items, seq, heads, 128)
    runtime.attention_device(dq, dk, dv, again, items, seq, heads, 128)
    runtime.attention_device(dq[seq:], dk[seq:], dv[seq:], o1, 1, seq, heads, 128)
    torch.cuda.synchronize()
    assert runtime.sync_status().ok
    assert torch.equal(o2, again)
    assert torch.equal(o2[seq:], o1)


def test_fused_attention_rejects_unsupported_shapes(runtime):
    import torch
    x = torch.zeros((192, 128), device="cuda")
    with pytest.raises(RuntimeError, match="detail=-7007"):
        runtime.attention_device(x, x, x, x, 1, 192, 1, 128)  # seq not a multiple of 128
    y = torch.zeros((128, 64), device="cuda")
    with pytest.raises(RuntimeError, match="detail=-7007"):
        runtime.attention_device(y, y, y, y, 1, 128, 1, 64)  # head_dim 64
