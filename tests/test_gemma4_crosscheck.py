"""An independent check of the Gemma block oracle's pieces that the reference does
not pin, against the transformers Gemma4 modules (installed: transformers 5.5.0;
the reference pins the module family at 5.6.2,
tools/python/gemma/gemma4e2b_m1_reference.py:3-24).

The reference's own Gemma lane stops at the raw scores
(gemma4e2b_m1_rtx.go:863-883), so the oracle's causal softmax, P.V, GeGLU
feed-forward and the half-split RoPE convention follow the standard Gemma
decoder.  Here each is compared, with the same random weights, against the
transformers module that implements it:

  Gemma4RMSNorm             x * (mean(x^2) + eps)^-1/2 * weight (computed in fp32)
  Gemma4TextRotaryEmbedding + apply_rotary_pos_emb   rotate_half pairing (c, c + hd/2)
  eager_attention_forward   causal mask, softmax (fp32), P.V, MQA by repeat_kv
  Gemma4TextMLP             down(gelu_tanh(gate(x)) * up(x))

The Gemma4 decoder layer itself is not the benchmark's block: it adds q/k/v
norms and uses unit attention scaling, so the comparison is per piece.  Runs on
CPU, float64 where the module allows it.
"""
from __future__ import annotations

import math

import numpy as np
import pytest

from oracle import blocks as OB

torch = pytest.importorskip("torch")
gemma4 = pytest.importorskip("transformers.models.gemma4.modeling_gemma4")
from transformers.models.gemma4.configuration_gemma4 import Gemma4TextConfig  # noqa: E402

HIDDEN, HEADS, HEAD_DIM, FFN, SEQ = 256, 4, 64, 512, 48


def _config():
    return Gemma4TextConfig(
        hidden_size=HIDDEN, intermediate_size=FFN, num_hidden_layers=1, num_attention_heads=HEADS,
        num_key_value_heads=1, head_dim=HEAD_DIM, hidden_activation="gelu_pytorch_tanh", rms_norm_eps=1e-6,
        layer_types=["full_attention"], num_kv_shared_layers=0, attention_k_eq_v=False,
        rope_parameters={"full_attention": {"rope_type": "default", "rope_theta": 10000.0}},
        max_position_embeddings=4096, vocab_size=32, hidden_size_per_layer_input=0, vocab_size_per_layer_input=32)


@pytest.fixture(scope="module")
def parts():
    cfg = OB.gemma_config(seq_len=SEQ, hidden=HIDDEN, heads=HEADS, head_dim=HEAD_DIM, ffn=FFN)
    w = OB.random_weights(cfg, seed=31)
    x = np.random.default_rng(32).standard_normal((SEQ, HIDDEN))
    return cfg, w, x


def test_rmsnorm_matches_gemma4(parts):
    cfg, w, x = parts
    norm = gemma4.Gemma4RMSNorm(HIDDEN, eps=1e-6)
    with torch.no_grad():
        norm.weight.copy_(torch.from_numpy(w["norm1"].astype(np.float64)))
        got = norm.double()(torch.from_numpy(x)).numpy()
    want = OB.rmsnorm(x, w["norm1"], 1e-6)
    assert np.max(np.abs(got - want)) <= 2e-6 * np.max(np.abs(want))  # the module computes in fp32


def test_geglu_ffn_matches_gemma4_mlp(parts):
    cfg, w, x = parts
    mlp = gemma4.Gemma4TextMLP(_config(), layer_idx=0).double()
    wgu = w["wgu"].astype(np.float64)
    with torch.no_grad():
        mlp.gate_proj.weight.copy_(torch.from_numpy(wgu[:, :FFN].T.copy()))
        mlp.up_proj.weight.copy_(torch.from_numpy(wgu[:, FFN:].T.copy()))
        mlp.down_proj.weight.copy_(torch.from_numpy(w["wd"].astype(np.float64).T.copy()))
        got = mlp(torch.from_numpy(x)).numpy()
    gu = x @ wgu
    want = (OB.gelu_tanh(gu[:, :FFN]) * gu[:, FFN:]) @ w["wd"].astype(np.float64)
    assert np.max(np.abs(got - want)) <= 1e-12 * np.max(np.abs(want))


def test_half_split_rope_matches_gemma4_rotary(parts):
    cfg, w, x = parts
    rng = np.random.default_rng(33)
    q = rng.standard_normal((1, SEQ, HEADS, HEAD_DIM))
    rot = gemma4.Gemma4TextRotaryEmbedding(_config())
    pos = torch.arange(SEQ)[None, :]
    cos, sin = rot(torch.from_numpy(q), pos, layer_type="full_attention")
    got = gemma4.apply_rotary_pos_emb(torch.from_numpy(q), cos.double(), sin.double(), unsqueeze_dim=2).numpy()[0]
    want = OB.rope_half_split(q[0], np.arange(SEQ), 10000.0)
    # the module's inverse frequencies are fp32: angles agree to ~pos * 6e-8
    assert np.max(np.abs(got - want)) <= 5e-6 * np.max(np.abs(want))


def test_causal_mqa_attention_matches_gemma4_eager_attention(parts):
    rng = np.random.default_rng(34)
    q = rng.standard_normal((SEQ, HEADS, HEAD_DIM))
    k = rng.standard_normal((SEQ, 1, HEAD_DIM))
    v = rng.standard_normal((SEQ, 1, HEAD_DIM))
    scale = 1.0 / math.sqrt(HEAD_DIM)

    class Mod:
        num_key_value_groups = HEADS
        head_dim = HEAD_DIM
        training = False

    mask = torch.triu(torch.full((SEQ, SEQ), float("-inf"), dtype=torch.float64), diagonal=1)[None, None]
    tq, tk, tv = (torch.from_numpy(t).permute(1, 0, 2)[None].contiguous() for t in (q, k, v))
    out, _ = gemma4.eager_attention_forward(Mod(), tq, tk, tv, mask, scaling=scale)
    got = out[0].reshape(SEQ, HEADS * HEAD_DIM).numpy()
    want = OB.attention(q, k, v, scale, causal=True)
    assert np.max(np.abs(got - want)) <= 1e-6 * np.max(np.abs(want))  # softmax is taken in fp32
