"""Seeded synthetic models of the benchmark configurations.

The reference has no seeded initialiser, so weights are drawn on the host by
the documented counter-based generator of nutllm_b200/host/synth.cpp, one
stream per tensor, and the identical bytes feed every implementation:

  embeddings        stream 1            N(0, 0.02), fp32
  lm_head           stream 2            N(0, 0.02), fp32 (untied)
  prompt ids        token stream 3      uniform in [1, vocab - 1]
  layer l, proj j   stream 1000+8l+j    N(0, 0.02), quantised at load
                    (j = 0..6: query key value output gate up down, [out][in])
  norm gains        1.0
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from . import (INT4, INT8, PROJECTIONS, Config, LayerWeights, ModelWeights,
               QuantizedMatrix, synth_normal, synth_tokens)

SIGMA = 0.02


@dataclass(frozen=True)
class Workload:
    """One BASELINE configuration: model shape, quantisation and loop."""

    name: str
    config: tuple  # layers, heads, dim, head_dim, ffn, vocab, max_seq, eos, kv
    qtype: int
    prompt: int
    steps: int
    batch: int = 1

    def model_config(self) -> Config:
        return Config(*self.config)


# llama2.c checkpoints hard-wire eos_token = 1 (reference src/llama2.cpp:222).
WORKLOADS = {
    "tiny-int8": Workload("tiny-int8", (6, 6, 288, 48, 768, 512, 256, 1, 6),
                          INT8, 5, 16),
    "tinyllama-int4": Workload("tinyllama-int4",
                               (22, 32, 2048, 64, 5632, 32000, 2048, 1, 4),
                               INT4, 5, 16),
    "tinyllama-int8-long": Workload("tinyllama-int8-long",
                                    (22, 32, 2048, 64, 5632, 32000, 2048, 1, 4),
                                    INT8, 512, 256),
    "llama2-7b-int4": Workload("llama2-7b-int4",
                               (32, 32, 4096, 128, 11008, 32000, 2048, 1, 32),
                               INT4, 128, 128, batch=64),
}


def projection_shapes(c: Config) -> list[tuple[int, int]]:
    kv = c.kv_dim
    return [(c.dim, c.dim), (kv, c.dim), (kv, c.dim), (c.dim, c.dim),
            (c.ffn_dim, c.dim), (c.ffn_dim, c.dim), (c.dim, c.ffn_dim)]


def projection_fp32(c: Config, seed: int, layer: int, j: int) -> np.ndarray:
    rows, cols = projection_shapes(c)[j]
    return synth_normal(seed, 1000 + 8 * layer + j, rows * cols, SIGMA).reshape(rows, cols)


def embeddings_fp32(c: Config, seed: int) -> np.ndarray:
    return synth_normal(seed, 1, c.vocab_size * c.dim, SIGMA).reshape(c.vocab_size, c.dim)


def lm_head_fp32(c: Config, seed: int) -> np.ndarray:
    return synth_normal(seed, 2, c.vocab_size * c.dim, SIGMA).reshape(c.vocab_size, c.dim)


def prompt_ids(c: Config, seed: int, n: int, stream: int = 3) -> np.ndarray:
    return synth_tokens(seed, stream, n, 1, int(c.vocab_size) - 1)


def build_model(c: Config, qtype: int, seed: int, tied: bool = False) -> ModelWeights:
    """Seeded fp32 weights, quantised by the host quantiser."""
    layers = []
    ones = np.ones(c.dim, np.float32)
    for layer in range(c.layers):
        mats = [QuantizedMatrix.quantize(projection_fp32(c, seed, layer, j), qtype)
                for j in range(len(PROJECTIONS))]
        layers.append(LayerWeights(*mats, attention_norm=ones.copy(),
                                   ffn_norm=ones.copy()))
    return ModelWeights(config=Config(*[getattr(c, n) for n, _ in c._fields_]),
                        qtype=qtype, embeddings=embeddings_fp32(c, seed),
                        layers=layers, final_norm=ones.copy(),
                        lm_head=None if tied else lm_head_fp32(c, seed),
                        tied_embeddings=tied)


def quantised_layer_bytes(c: Config, qtype: int) -> int:
    """Storage of one layer's seven quantised projections: the weights
    (1 or 1/2 byte each) and one fp16 scale per block of 32."""
    n = sum(rows * cols for rows, cols in projection_shapes(c))
    return (n if qtype == INT8 else n // 2) + 2 * (n // 32)


def algorithmic_decode_bytes(c: Config, qtype: int, pos: int,
                             logits: bool = True) -> int:
    """HBM bytes one batch-1 decode pass at position `pos` must move: every
    quantised weight and scale once, the embedding row, the two norm vectors
    per layer, the KV history of positions 0..pos (K and V, fp32, written
    once and read once), and, when the pass produces logits, the final norm
    and the fp32 classifier."""
    b = (c.layers * quantised_layer_bytes(c, qtype) + c.dim * 4
         + 2 * c.layers * c.dim * 4 + c.layers * 2 * c.kv_dim * 4 * (pos + 1))
    if logits:
        b += c.vocab_size * c.dim * 4 + c.dim * 4
    return int(b)


def algorithmic_generation_bytes(c: Config, qtype: int, n_prompt: int,
                                 steps: int) -> int:
    """Bytes of one greedy generation run as a single device loop: passes at
    positions 0 .. n_prompt+steps-1, logits after passes n_prompt-1 ..
    n_prompt+steps-2 (the last pass decodes the last chosen token)."""
    total = 0
    for pos in range(n_prompt + steps):
        total += algorithmic_decode_bytes(
            c, qtype, pos, n_prompt - 1 <= pos <= n_prompt + steps - 2)
    return total


# Prompts of at least this many tokens are prefilled as GEMMs by default
# (the library's nut_model_set_prefill_threshold default).
GEMM_PREFILL_MIN = 64


def algorithmic_decode_launch_bytes(c: Config, qtype: int, n_prompt: int,
                                    steps: int) -> int:
    """Bytes of the persistent decode launch of one greedy generation.  With
    a prompt of GEMM_PREFILL_MIN tokens or more the prompt goes through the
    GEMM prefill first, and the launch reads the classifier for the prompt's
    last hidden state and then runs the passes at positions n_prompt ..
    n_prompt+steps-1 (logits after all but the last); shorter prompts run
    every pass in the launch (algorithmic_generation_bytes)."""
    if n_prompt < GEMM_PREFILL_MIN:
        return algorithmic_generation_bytes(c, qtype, n_prompt, steps)
    last = n_prompt - 1
    total = (algorithmic_decode_bytes(c, qtype, last, True)
             - algorithmic_decode_bytes(c, qtype, last, False))
    for pos in range(n_prompt, n_prompt + steps):
        total += algorithmic_decode_bytes(c, qtype, pos, pos <= n_prompt + steps - 2)
    return total
