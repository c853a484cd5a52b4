"""Seeded inputs of the BASELINE configurations (test infrastructure only).

* config 0: 28-layer model, 32-token uniform-random prompt, max cache 512,
  128 greedy decode steps.
* config 1: one decoder layer (layer 0 of the config-0 weights), hidden
  N(0,1) BF16 [1024], K/V cache [8, 512, 128] BF16 with positions 0-510 filled
  N(0,1), one decode step at position 511.
* config 2: isolated LM head, the config-0 embedding [151936, 1024] and a
  hidden N(0,1) BF16 [1024] taken as already normalised.
* config 3: config 0 with max cache 4096, 3584-token prompt, 256 steps.

All draws use ``numpy.random.default_rng([seed, stream])`` so every machine
regenerates identical inputs.
"""
from __future__ import annotations

import numpy as np
import torch

from .weights import HEAD_DIM, HIDDEN, N_KV, prompt_ids

CONFIG0 = dict(prompt_len=32, max_seq=512, steps=128)
CONFIG1 = dict(position=511, max_seq=512)
CONFIG3 = dict(prompt_len=3584, max_seq=4096, steps=256)


def _bf16_normal(seed: int, stream: int, shape) -> torch.Tensor:
    rng = np.random.default_rng([seed, stream])
    return torch.from_numpy(rng.standard_normal(size=shape, dtype=np.float32)).to(torch.bfloat16)


def config0_prompt(seed: int = 0) -> torch.Tensor:
    return prompt_ids(seed, CONFIG0["prompt_len"])


def config3_prompt(seed: int = 0) -> torch.Tensor:
    return prompt_ids(seed, CONFIG3["prompt_len"])


def config1_inputs(seed: int = 0) -> dict:
    pos = CONFIG1["position"]
    hidden = _bf16_normal(seed, 1001, (HIDDEN,))
    k_prefix = _bf16_normal(seed, 1002, (N_KV, pos, HEAD_DIM))
    v_prefix = _bf16_normal(seed, 1003, (N_KV, pos, HEAD_DIM))
    return dict(hidden=hidden, k_prefix=k_prefix, v_prefix=v_prefix, position=pos,
                max_seq=CONFIG1["max_seq"])


def config2_hidden(seed: int = 0) -> torch.Tensor:
    return _bf16_normal(seed, 2001, (HIDDEN,))


def sample_indices(n: int = 512, vocab: int = 151936, seed: int = 7) -> np.ndarray:
    """Fixed logit indices stored in the golden files."""
    rng = np.random.default_rng([seed, 99])
    return np.sort(rng.choice(vocab, size=n, replace=False)).astype(np.int64)
