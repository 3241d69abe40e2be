"""Binary64 oracle of the two transformer blocks on the hot path (test infrastructure only).

Only tests/ and bench.py's CPU leg use this module, as the checker; the product
(libprometheus_reactor.so) never calls it.  It restates, step by step, the
reference's CPU block code in numpy float64 so every output of the CUDA block
can be compared against it (tolerance: <= 1e-4 relative per block output).

DiT block: `runCanonicalNoiseRefiner0` (internal/prometheus/zimage/canonical_reference.go:377-479)
  adaLN linear -> tanh(gates), scales + 1            (:358-381)
  RMSNorm eps 1e-5 (`canonicalNormRows`, :178-190; formula canonical_contract.go:91-105)
  modulation `canonicalScale` (:192-199)
  fused QKV linear, no bias (`canonicalLinear`, :156-175; split :404-413)
  per-head Q/K RMSNorm (:414-421)
  3-axis interleaved RoPE (`canonicalRope`, :212-239; `CanonicalRopeRotate`,
    canonical_contract.go:66-89: frequency = float32(theta^(-2p/width)), angle in fp32)
  exact softmax attention, scale 1/sqrt(head_dim) (`canonicalAttention`, :241-289)
  out projection -> RMSNorm -> gated residual (`canonicalAddGate`, :201-210)
  FFN norm -> modulation -> w1, w3 -> silu(w1)*w3 (:455-458) -> w2 -> RMSNorm -> gated residual.
  Extensions of the benchmark configs (unpinned by the reference, which has 4 x hidden and no
  shift): a 6 x hidden adaLN whose extra parts are additive shifts applied after
  each modulation, and a 256-d sinusoidal timestep embedding [cos | sin] with
  frequencies exp(-ln(10000) i / 128) computed here instead of read from a file.
  Image tokens sit on a grid_w-wide grid: coordinate (frame, token // grid_w, token % grid_w),
  as `CanonicalImageTokenCoordinate` (canonical_contract.go:53-64) does for its 32-wide grid.

Gemma block (decoder, pre-norm):
  RMSNorm (`cpuHeadRMSNorm` formula, gemma4e2b_m1_rtx.go:811-832) with gain g
  Q/K/V linear (`cpuMatmulRowMajor`, :795-809), MQA: every query head uses KV head 0
  half-split RoPE (`cpuGemma4e2bRope`, :834-861, without its BF16 storage rounding)
  raw scores q.k * (1/sqrt(head_dim)) (`cpuGemma4e2bRawScores`, :863-883), then the
  causal mask and softmax of a decoder, P.V, output projection, residual
  RMSNorm -> gate/up linear -> GeGLU gelu_tanh(gate) * up -> down linear -> residual.
  The reference stops at raw scores: the mask, softmax, P.V, out projection and
  GeGLU FFN are parity-unpinned by it; they follow the standard Gemma decoder.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np

GEMMA, DIT = 1, 2


@dataclass
class BlockConfig:
    family: int
    hidden: int
    heads: int
    kv_heads: int
    head_dim: int
    ffn: int
    seq_len: int
    eps: float
    rope_base: float
    grid_w: int = 0
    rope_frame: int = 0
    rope_axes: tuple = (32, 48, 48)
    qk_eps: float = 1e-5


def gemma_config(seq_len: int = 1024, hidden: int = 2048, heads: int = 8, head_dim: int = 256, ffn: int = 16384,
                 kv_heads: int = 1) -> BlockConfig:
    """The benchmark's Gemma-2B-shaped decoder block (4 x 1024 tokens, hidden 2048, 8 x 256 MQA, GeGLU 16384)."""
    return BlockConfig(GEMMA, hidden, heads, kv_heads, head_dim, ffn, seq_len, eps=1e-6, rope_base=10000.0)


def dit_config(seq_len: int = 4096, hidden: int = 3072, heads: int = 24, head_dim: int = 128, ffn: int = 8192,
               grid_w: int = 64, rope_frame: int = 33) -> BlockConfig:
    """The benchmark's Z-Image-style DiT block (2 x 4096 tokens = 64 x 64 latent patches, hidden 3072)."""
    return BlockConfig(DIT, hidden, heads, heads, head_dim, ffn, seq_len, eps=1e-5, rope_base=256.0,
                       grid_w=grid_w, rope_frame=rope_frame)


# ---------------------------------------------------------------- weights
GEMMA_SLOTS = ("norm1", "wqkv", "wo", "norm2", "wgu", "wd")
DIT_SLOTS = ("ada_w", "ada_b", "attn_norm1", "wqkv", "q_norm", "k_norm", "wo", "attn_norm2", "ffn_norm1", "w13",
             "w2", "ffn_norm2")


def weight_shapes(cfg: BlockConfig) -> dict[str, tuple]:
    d, h, kv, hd, f = cfg.hidden, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.ffn
    if cfg.family == GEMMA:
        return {"norm1": (d,), "wqkv": (d, (h + 2 * kv) * hd), "wo": (h * hd, d), "norm2": (d,),
                "wgu": (d, 2 * f), "wd": (f, d)}
    return {"ada_w": (256, 6 * d), "ada_b": (6 * d,), "attn_norm1": (d,), "wqkv": (d, 3 * h * hd),
            "q_norm": (hd,), "k_norm": (hd,), "wo": (h * hd, d), "attn_norm2": (d,), "ffn_norm1": (d,),
            "w13": (d, 2 * f), "w2": (f, d), "ffn_norm2": (d,)}


def random_weights(cfg: BlockConfig, seed: int) -> dict[str, np.ndarray]:
    """Benchmark init: linear weights and the adaLN bias N(0, 0.02); norm gains 1 + N(0, 0.02).

    The non-zero adaLN bias exercises `canonicalLinear`'s bias term
    (canonical_reference.go:163-164)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    out = {}
    for name, shape in weight_shapes(cfg).items():
        if name == "ada_b":
            out[name] = (0.02 * rng.standard_normal(shape)).astype(np.float32)
        elif len(shape) == 1:
            out[name] = (1.0 + 0.02 * rng.standard_normal(shape)).astype(np.float32)
        else:
            out[name] = (0.02 * rng.standard_normal(shape)).astype(np.float32)
    return out


# ---------------------------------------------------------------- pieces (float64)
def rmsnorm(x: np.ndarray, g: np.ndarray, eps: float) -> np.ndarray:
    x = x.astype(np.float64)
    inv = 1.0 / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + float(np.float32(eps)))
    return x * inv * g.astype(np.float64)


def timestep_embedding(t: float, dim: int = 256) -> np.ndarray:
    half = dim // 2
    freqs = np.exp(-math.log(10000.0) * np.arange(half, dtype=np.float64) / half)
    ang = float(t) * freqs
    return np.concatenate([np.cos(ang), np.sin(ang)])


def rope_half_split(x: np.ndarray, positions: np.ndarray, base: float) -> np.ndarray:
    """x [T, heads, hd]; rotate_half pairing (c, c + hd/2)."""
    hd = x.shape[-1]
    half = hd // 2
    inv = base ** (-np.arange(half, dtype=np.float64) * 2.0 / hd)
    ang = positions.astype(np.float64)[:, None] * inv[None, :]
    cos, sin = np.cos(ang)[:, None, :], np.sin(ang)[:, None, :]
    a, b = x[..., :half], x[..., half:]
    return np.concatenate([a * cos - b * sin, b * cos + a * sin], axis=-1)


def rope_3axis(x: np.ndarray, coords: np.ndarray, theta: float, axes=(32, 48, 48)) -> np.ndarray:
    """x [T, heads, hd]; coords [T, 3]; interleaved (even, odd) pairs per axis segment."""
    out = x.copy()
    base = 0
    for axis, width in enumerate(axes):
        p = np.arange(width // 2)
        freq = (1.0 / np.power(float(theta), 2.0 * p / width)).astype(np.float32)  # float32, as the reference
        ang = (coords[:, axis].astype(np.float32)[:, None] * freq[None, :]).astype(np.float64)
        cos = np.cos(ang).astype(np.float32).astype(np.float64)[:, None, :]
        sin = np.sin(ang).astype(np.float32).astype(np.float64)[:, None, :]
        e = x[..., base + 2 * p]
        o = x[..., base + 2 * p + 1]
        out[..., base + 2 * p] = e * cos - o * sin
        out[..., base + 2 * p + 1] = e * sin + o * cos
        base += width
    return out


def attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, scale: float, causal: bool) -> np.ndarray:
    """q [S, H, hd], k/v [S, KVH, hd] (KVH = 1 or H) -> [S, H*hd]."""
    S, H, hd = q.shape
    kvh = k.shape[1]
    out = np.empty((S, H, hd))
    mask = np.triu(np.ones((S, S), dtype=bool), k=1) if causal else None
    for h in range(H):
        kk = k[:, 0 if kvh == 1 else h, :]
        vv = v[:, 0 if kvh == 1 else h, :]
        s = (q[:, h, :] @ kk.T) * scale
        if mask is not None:
            s = np.where(mask, -np.inf, s)
        s = s - s.max(axis=1, keepdims=True)
        p = np.exp(s)
        p /= p.sum(axis=1, keepdims=True)
        out[:, h, :] = p @ vv
    return out.reshape(S, H * hd)


def gelu_tanh(x: np.ndarray) -> np.ndarray:
    return 0.5 * x * (1.0 + np.tanh(math.sqrt(2.0 / math.pi) * (x + 0.044715 * x ** 3)))


def silu(x: np.ndarray) -> np.ndarray:
    return x / (1.0 + np.exp(-x))


# ---------------------------------------------------------------- blocks
def _identity(a):
    return a


def gemma_forward(cfg: BlockConfig, w: dict, x: np.ndarray, all_reduce=_identity) -> np.ndarray:
    """x [B*S, d] float32 -> [B*S, d] float64.

    Under tensor parallelism cfg.heads / cfg.ffn are one rank's share, `w` its
    shard, and `all_reduce` sums the two row-parallel partial products."""
    d, H, KV, hd, F, S = cfg.hidden, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.ffn, cfg.seq_len
    W = {k: v.astype(np.float64) for k, v in w.items()}
    x64 = x.astype(np.float64)
    T = x.shape[0]
    out = np.empty_like(x64)
    for s0 in range(0, T, S):
        xs = x64[s0:s0 + S]
        h = rmsnorm(xs, W["norm1"], cfg.eps)
        qkv = h @ W["wqkv"]
        q = qkv[:, :H * hd].reshape(S, H, hd)
        k = qkv[:, H * hd:(H + KV) * hd].reshape(S, KV, hd)
        v = qkv[:, (H + KV) * hd:].reshape(S, KV, hd)
        pos = np.arange(S)
        q = rope_half_split(q, pos, cfg.rope_base)
        k = rope_half_split(k, pos, cfg.rope_base)
        o = attention(q, k, v, 1.0 / math.sqrt(hd), causal=True)
        x1 = xs + all_reduce(o @ W["wo"])
        h2 = rmsnorm(x1, W["norm2"], cfg.eps)
        gu = h2 @ W["wgu"]
        act = gelu_tanh(gu[:, :F]) * gu[:, F:]
        out[s0:s0 + S] = x1 + all_reduce(act @ W["wd"])
    return out


def dit_forward(cfg: BlockConfig, w: dict, x: np.ndarray, timesteps, all_reduce=_identity) -> np.ndarray:
    """x [B*S, d] float32, one timestep per batch item -> [B*S, d] float64 (TP as gemma_forward)."""
    d, H, hd, F, S = cfg.hidden, cfg.heads, cfg.head_dim, cfg.ffn, cfg.seq_len
    W = {k: v.astype(np.float64) for k, v in w.items()}
    x64 = x.astype(np.float64)
    out = np.empty_like(x64)
    tok = np.arange(S)
    coords = np.stack([np.full(S, cfg.rope_frame), tok // cfg.grid_w, tok % cfg.grid_w], axis=1)
    for b, t in enumerate(timesteps):
        xs = x64[b * S:(b + 1) * S]
        ada = timestep_embedding(t) @ W["ada_w"] + W["ada_b"]
        scale_a, gate_a, scale_m, gate_m, shift_a, shift_m = (ada[i * d:(i + 1) * d] for i in range(6))
        gate_a, gate_m = np.tanh(gate_a), np.tanh(gate_m)
        scale_a, scale_m = scale_a + 1.0, scale_m + 1.0
        mod = rmsnorm(xs, W["attn_norm1"], cfg.eps) * scale_a + shift_a
        qkv = mod @ W["wqkv"]
        q = qkv[:, :H * hd].reshape(S, H, hd)
        k = qkv[:, H * hd:2 * H * hd].reshape(S, H, hd)
        v = qkv[:, 2 * H * hd:].reshape(S, H, hd)
        q = rmsnorm(q, W["q_norm"], cfg.qk_eps)
        k = rmsnorm(k, W["k_norm"], cfg.qk_eps)
        q = rope_3axis(q, coords, cfg.rope_base, cfg.rope_axes)
        k = rope_3axis(k, coords, cfg.rope_base, cfg.rope_axes)
        o = attention(q, k, v, 1.0 / math.sqrt(hd), causal=False)
        n2 = rmsnorm(all_reduce(o @ W["wo"]), W["attn_norm2"], cfg.eps)
        res = xs + gate_a * n2
        fin = rmsnorm(res, W["ffn_norm1"], cfg.eps) * scale_m + shift_m
        h13 = fin @ W["w13"]
        hidden = silu(h13[:, :F]) * h13[:, F:]
        fo = rmsnorm(all_reduce(hidden @ W["w2"]), W["ffn_norm2"], cfg.eps)
        out[b * S:(b + 1) * S] = res + gate_m * fo
    return out


def forward(cfg: BlockConfig, w: dict, x: np.ndarray, timesteps=None, all_reduce=_identity) -> np.ndarray:
    if cfg.family == GEMMA:
        return gemma_forward(cfg, w, x, all_reduce)
    return dit_forward(cfg, w, x, timesteps, all_reduce)


def flops_per_forward(cfg: BlockConfig, batch: int) -> float:
    """Algorithmic flops of one block forward (causal attention counts the lower triangle)."""
    d, H, KV, hd, F, S = cfg.hidden, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.ffn, cfg.seq_len
    T = batch * S
    linear = 2.0 * T * d * ((H + 2 * KV) * hd) + 2.0 * T * (H * hd) * d + 2.0 * T * d * 2 * F + 2.0 * T * F * d
    pairs = S * (S + 1) / 2 if cfg.family == GEMMA else float(S * S)
    attn = batch * H * pairs * 4.0 * hd
    return linear + attn


# ---------------------------------------------------------------- Z-Image model-block executors
ZIMAGE_NOISE_NAMES = ("adaLN_modulation.0.bias", "adaLN_modulation.0.weight", "attention.k_norm.weight",
                      "attention.out.weight", "attention.q_norm.weight", "attention.qkv.weight",
                      "attention_norm1.weight", "attention_norm2.weight", "feed_forward.w1.weight",
                      "feed_forward.w2.weight", "feed_forward.w3.weight", "ffn_norm1.weight", "ffn_norm2.weight")
ZIMAGE_CONTEXT_NAMES = ZIMAGE_NOISE_NAMES[2:]


def zimage_weight_shapes(context: bool = False, width: int = 3840, heads: int = 30, head_dim: int = 128,
                         ffn: int = 10240) -> dict[str, tuple]:
    """The cache manifest's tensors in lexical order, linear weights [in][out]
    (canonicalLoadWeights, zimage/canonical_reference.go:51-80; reactor_vulkan_model_block.c:160-183)."""
    shapes = {"adaLN_modulation.0.bias": (4 * width,), "adaLN_modulation.0.weight": (256, 4 * width),
              "attention.k_norm.weight": (head_dim,), "attention.out.weight": (width, width),
              "attention.q_norm.weight": (head_dim,), "attention.qkv.weight": (width, 3 * width),
              "attention_norm1.weight": (width,), "attention_norm2.weight": (width,),
              "feed_forward.w1.weight": (width, ffn), "feed_forward.w2.weight": (ffn, width),
              "feed_forward.w3.weight": (width, ffn), "ffn_norm1.weight": (width,), "ffn_norm2.weight": (width,)}
    names = ZIMAGE_CONTEXT_NAMES if context else ZIMAGE_NOISE_NAMES
    return {n: shapes[n] for n in names}


def zimage_random_weights_f16(seed: int, context: bool = False) -> dict[str, np.ndarray]:
    """Random binary16 payloads: linear weights and the adaLN N(0, 0.02), gains 1 + N(0, 0.02)."""
    rng = np.random.Generator(np.random.PCG64(seed))
    out = {}
    for name, shape in zimage_weight_shapes(context).items():
        if len(shape) == 1 and not name.startswith("adaLN"):
            v = 1.0 + 0.02 * rng.standard_normal(shape)
        else:
            v = 0.02 * rng.standard_normal(shape)
        out[name] = v.astype(np.float16)
    return out


def bf16_values(x: np.ndarray) -> np.ndarray:
    """fp32 -> BF16 (round to nearest even) -> fp32, and the raw 16-bit payload."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    b = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32), b


def _canonical_rope_rows(x: np.ndarray, coords: np.ndarray, theta: float = 256.0) -> np.ndarray:
    return rope_3axis(x, coords, theta, (32, 48, 48))


def zimage_refiner_forward(w16: dict, x: np.ndarray, temb: np.ndarray | None, tokens: int, context: bool,
                           width: int = 3840, heads: int = 30, head_dim: int = 128, ffn: int = 10240) -> np.ndarray:
    """One Z-Image refiner block in binary64 from binary16 weights.

    Noise refiner: runCanonicalNoiseRefiner0 (zimage/canonical_reference.go:315-480): adaLN
    256 -> 4 x width with bias, gates tanh, scales + 1, no shift; image tokens on the 32-wide
    grid at frame 33 (canonical_contract.go:44-64).  Context refiner: runCanonicalContextRefiner
    (zimage/context_refiner_reference.go:229-299): the same block unmodulated, token t at
    (t + 1, 0, 0) (:151-174).  Both: RMSNorm eps 1e-5, sandwich norms, SwiGLU, residuals."""
    W = {k: v.astype(np.float64) for k, v in w16.items()}
    xs = x.astype(np.float64).reshape(tokens, width)
    eps = float(np.float32(1e-5))
    if context:
        scale_a = scale_m = gate_a = gate_m = 1.0
        coords = np.stack([np.arange(tokens) + 1, np.zeros(tokens), np.zeros(tokens)], axis=1)
    else:
        ada = temb.astype(np.float64) @ W["adaLN_modulation.0.weight"] + W["adaLN_modulation.0.bias"]
        scale_a, gate_a, scale_m, gate_m = (ada[i * width:(i + 1) * width] for i in range(4))
        gate_a, gate_m = np.tanh(gate_a), np.tanh(gate_m)
        scale_a, scale_m = scale_a + 1.0, scale_m + 1.0
        tok = np.arange(tokens)
        coords = np.stack([np.full(tokens, 33), tok // 32, tok % 32], axis=1)
    mod = rmsnorm(xs, W["attention_norm1.weight"], eps) * scale_a
    qkv = mod @ W["attention.qkv.weight"]
    q = qkv[:, :width].reshape(tokens, heads, head_dim)
    k = qkv[:, width:2 * width].reshape(tokens, heads, head_dim)
    v = qkv[:, 2 * width:].reshape(tokens, heads, head_dim)
    q = _canonical_rope_rows(rmsnorm(q, W["attention.q_norm.weight"], eps), coords)
    k = _canonical_rope_rows(rmsnorm(k, W["attention.k_norm.weight"], eps), coords)
    o = attention(q, k, v, 1.0 / math.sqrt(head_dim), causal=False)
    res = xs + gate_a * rmsnorm(o @ W["attention.out.weight"], W["attention_norm2.weight"], eps)
    fin = rmsnorm(res, W["ffn_norm1.weight"], eps) * scale_m
    hidden = silu(fin @ W["feed_forward.w1.weight"]) * (fin @ W["feed_forward.w3.weight"])
    return res + gate_m * rmsnorm(hidden @ W["feed_forward.w2.weight"], W["ffn_norm2.weight"], eps)
