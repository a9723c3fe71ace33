"""Seeded synthetic inputs for the MoE layer benchmark configurations.

The reference's weights (a private Gemma-4-26B-A4B QAT GGUF) are not available, so every
input is drawn from seeded distributions with the layer's exact shapes and formats:

* x: N(0,1) rows of n_embd, RMS-normalised (sum of squares in f64, eps 1e-6, as
  ``ops::rms_norm``, runtime/src/ops.rs:131-139), then rounded to bf16.
* router: bf16 N(0, 0.02), ``n_experts`` rows of ``n_embd`` (ggml dims [2816, 128], the
  layout of ``ffn_gate_inp.weight``, runtime/src/contract.rs:66).
* experts: Q4_0 in the reference's GGUF layout (runtime/src/model.rs:36-40):
  gate_up [n_experts][2*ff rows][n_embd/32 blocks of 18 B] (gate rows, then up rows) and
  down [n_experts][n_embd rows][ff/32 blocks]; block scale f16(|N(0,1)| * 0.01), nibble
  bytes uniform 0..255.

Shapes default to the target's contract (runtime/src/contract.rs:12-22): n_embd 2816,
ff 704, 128 experts, top-8.
"""
from __future__ import annotations

import numpy as np

N_EMBD = 2816
FF = 704
N_EXPERTS = 128
USED = 8
QK = 32
Q4_BLOCK = 18
Q8_BLOCK = 34

GATE_UP_BYTES = 2 * FF * (N_EMBD // QK) * Q4_BLOCK   # 2,230,272 per expert
DOWN_BYTES = N_EMBD * (FF // QK) * Q4_BLOCK          # 1,115,136 per expert
EXPERT_BYTES = GATE_UP_BYTES + DOWN_BYTES            # 3,345,408


def rng(seed: int) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64(seed))


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even f32 -> bf16, returned as uint16 bit patterns."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    rounding = ((b >> 16) & 1) + 0x7FFF
    out = ((b + rounding) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        out[nan] = 0x7FC0
    return out


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def rms_normalise(x: np.ndarray, eps: float = 1e-6) -> np.ndarray:
    x = np.asarray(x, dtype=np.float32)
    ss = np.sum(x.astype(np.float64) ** 2, axis=-1, keepdims=True)
    mean = (ss / x.shape[-1]).astype(np.float32)
    scale = np.float32(1.0) / np.sqrt(mean + np.float32(eps))
    return (x * scale).astype(np.float32)


def tokens(n_tok: int, seed: int, n_embd: int = N_EMBD) -> np.ndarray:
    """bf16 bits [n_tok, n_embd]: N(0,1), RMS-normalised."""
    g = rng(seed)
    x = g.standard_normal((n_tok, n_embd), dtype=np.float32)
    return f32_to_bf16_bits(rms_normalise(x))


def router(seed: int, n_experts: int = N_EXPERTS, n_embd: int = N_EMBD) -> np.ndarray:
    g = rng(seed)
    return f32_to_bf16_bits(g.standard_normal((n_experts, n_embd), dtype=np.float32) * np.float32(0.02))


def q4_rows(g: np.random.Generator, shape_blocks: tuple) -> np.ndarray:
    """Q4_0 blocks with f16(|N(0,1)|*0.01) scales and uniform nibble bytes; shape (..., 18)."""
    n = int(np.prod(shape_blocks))
    out = np.empty((n, Q4_BLOCK), np.uint8)
    d = (np.abs(g.standard_normal(n, dtype=np.float32)) * np.float32(0.01)).astype(np.float16)
    out[:, :2] = d.view(np.uint8).reshape(n, 2)
    out[:, 2:] = g.integers(0, 256, size=(n, 16), dtype=np.uint8)
    return out.reshape(*shape_blocks, Q4_BLOCK)


def experts(seed: int, n_experts: int = N_EXPERTS, n_embd: int = N_EMBD, ff: int = FF):
    """(gate_up, down) in the reference GGUF byte layout."""
    g = rng(seed)
    gate_up = q4_rows(g, (n_experts, 2 * ff, n_embd // QK))
    down = q4_rows(g, (n_experts, n_embd, ff // QK))
    return gate_up, down


def down_scales(seed: int | None, n_experts: int = N_EXPERTS) -> np.ndarray:
    """ffn_down_exps.scale: ones for the primary configs, U[0.5, 1.5) for the scaled variant."""
    if seed is None:
        return np.ones(n_experts, np.float32)
    return rng(seed).uniform(0.5, 1.5, n_experts).astype(np.float32)


def zipf_bias(seed: int, s: float = 1.1, n_experts: int = N_EXPERTS) -> np.ndarray:
    """Per-expert logit bias log(rank^-s) over a seeded random rank order, so that the bias
    alone would route with Zipf(s) probabilities (config 2's skewed prefill)."""
    g = rng(seed)
    rank = g.permutation(n_experts) + 1
    return (-s * np.log(rank.astype(np.float64))).astype(np.float32)


def hot_expert_bias(seed: int, n_tok: int, hot: np.ndarray, frac: float = 0.9, boost: float = 30.0,
                    n_experts: int = N_EXPERTS) -> np.ndarray:
    """Per-token bias [n_tok, n_experts] forcing `frac` of the tokens onto the `hot` experts
    (config 4's adversarial load). The boost is far above the logits' spread, so those tokens'
    top-8 is exactly the hot set."""
    g = rng(seed)
    b = np.zeros((n_tok, n_experts), np.float32)
    forced = g.random(n_tok) < frac
    b[np.ix_(forced, hot)] = np.float32(boost)
    return b


def config_inputs(config: int, n_tok: int | None = None, seed: int = 0, scaled_down: bool = False):
    """Inputs for BASELINE config 0..4. Returns a dict of numpy arrays.

    Seeds: tokens use `seed`, the router seed+1, experts seed+2, biases seed+3.
    """
    defaults = {0: 1, 1: 64, 2: 2048, 3: 16384, 4: 8192}
    n = defaults[config] if n_tok is None else n_tok
    d = {
        "x": tokens(n, seed),
        "w_router": router(seed + 1),
        "down_scale": down_scales(seed + 4 if scaled_down else None),
        "bias": None,
        "bias_stride": 0,
    }
    if config == 2:
        d["bias"] = zipf_bias(seed + 3)
    elif config == 4:
        d["bias"] = hot_expert_bias(seed + 3, n, np.arange(8, dtype=np.int64))
        d["bias_stride"] = N_EXPERTS
    return d
