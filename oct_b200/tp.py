"""Tensor-parallel layout of the transformer block (host side).

Megatron-style split of one block over `world` GPUs, as the block ABI expects it
(include/prometheus_reactor.h, OctB200BlockConfig):
  * query heads (and the DiT's K/V heads) are split evenly; the Gemma MQA KV
    head is replicated on every rank;
  * the fused QKV weight is column-sharded (each rank keeps the columns of its
    heads), the out projection row-sharded;
  * the gate|up (W1|W3) weight is column-sharded within each half, the down
    (W2) weight row-sharded;
  * norms, the adaLN linear and the Q/K norm gains are replicated.
The two row-parallel products give partial sums that the block all-reduces
over NCCL; every rank ends with the full block output.

Works on numpy arrays and on torch tensors alike.
"""
from __future__ import annotations

from dataclasses import replace

GEMMA, DIT = 1, 2


def _cat_cols(parts):
    first = parts[0]
    if hasattr(first, "dim"):  # torch
        import torch
        return torch.cat(parts, dim=1).contiguous()
    import numpy as np
    return np.ascontiguousarray(np.concatenate(parts, axis=1))


def _rows(a, r0, r1):
    out = a[r0:r1]
    return out.contiguous() if hasattr(out, "contiguous") else out.copy()


def check_divisible(family: int, heads: int, ffn: int, world: int) -> None:
    if world < 1 or heads % world or ffn % world:
        raise ValueError(f"heads ({heads}) and ffn ({ffn}) must divide evenly over {world} ranks")


def rank_config(cfg, rank: int, world: int):
    """The per-rank block config: heads and ffn divided by world (oracle BlockConfig or a dict)."""
    check_divisible(cfg.family, cfg.heads, cfg.ffn, world)
    kv = cfg.kv_heads if cfg.family == GEMMA else cfg.heads // world
    return replace(cfg, heads=cfg.heads // world, ffn=cfg.ffn // world, kv_heads=kv)


def shard_weights(family: int, hidden: int, heads: int, kv_heads: int, head_dim: int, ffn: int, weights: dict,
                  rank: int, world: int) -> dict:
    """This rank's weight shard of a full block weight set (slot names of oracle/blocks.py)."""
    check_divisible(family, heads, ffn, world)
    hp, fp = heads // world, ffn // world
    h0, h1 = rank * hp * head_dim, (rank + 1) * hp * head_dim
    f0, f1 = rank * fp, (rank + 1) * fp
    out = dict(weights)
    wqkv = weights["wqkv"]
    if family == GEMMA:
        q = wqkv[:, h0:h1]
        kv = wqkv[:, heads * head_dim:(heads + 2 * kv_heads) * head_dim]  # replicated MQA K|V
        out["wqkv"] = _cat_cols([q, kv])
        gu_name, down_name = "wgu", "wd"
    else:
        d = heads * head_dim
        out["wqkv"] = _cat_cols([wqkv[:, h0:h1], wqkv[:, d + h0:d + h1], wqkv[:, 2 * d + h0:2 * d + h1]])
        gu_name, down_name = "w13", "w2"
    out["wo"] = _rows(weights["wo"], h0, h1)
    gu = weights[gu_name]
    out[gu_name] = _cat_cols([gu[:, f0:f1], gu[:, ffn + f0:ffn + f1]])
    out[down_name] = _rows(weights[down_name], f0, f1)
    return out


# ---------------------------------------------------------------- column-parallel SGEMM
def check_columns(n: int, world: int) -> int:
    """Columns per rank of the column-parallel SGEMM (oct_b200_sgemm_tp_device): n must
    be a multiple of 4 * world (whole 16-byte granules per rank)."""
    if world < 1 or n <= 0 or n % (4 * world):
        raise ValueError(f"n ({n}) must be a positive multiple of 4 * world ({4 * world})")
    return n // world


def shard_columns(b, rank: int, world: int):
    """This rank's column block B[:, r n/w .. (r+1) n/w) of a [k][n] operand, contiguous."""
    nr = check_columns(b.shape[1], world)
    part = b[:, rank * nr:(rank + 1) * nr]
    return part.contiguous() if hasattr(part, "contiguous") else part.copy()


def gather_columns(slabs):
    """Row-major C from the gathered slabs [world][m][n/w] -- what the library's
    repack kernel does after the all-gather: C[i, r n/w + j] = slabs[r][i][j]."""
    if hasattr(slabs, "dim"):  # torch [w][m][nr]
        w, m, nr = slabs.shape
        return slabs.permute(1, 0, 2).reshape(m, w * nr).contiguous()
    import numpy as np
    slabs = np.asarray(slabs)
    w, m, nr = slabs.shape
    return np.ascontiguousarray(slabs.transpose(1, 0, 2).reshape(m, w * nr))
