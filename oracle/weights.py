"""Deterministic synthetic Qwen3-0.6B weights (test infrastructure only).

The real checkpoint is not available offline, so every configuration uses
random-init weights: linear/embedding weights ~ N(0, 0.02), RMSNorm weights
1.0 (the ``_init_weights`` recipe of HF Qwen3), rounded once to BF16. Those
BF16 values are "the identical weights": the GPU engine streams them as BF16 and
the FP32 oracles upcast them exactly.

Each tensor draws from its own ``numpy.random.default_rng([seed, index])``
stream (PCG64), which numpy guarantees to be reproducible across machines, so
the GPU box regenerates bit-identical weights without shipping 1.2 GB.

``perturb_norms`` replaces the all-ones norm weights with 1 + N(0, 0.1): the
tests use it so that a kernel applying the wrong norm vector cannot pass.

Order of the 11 per-layer tensors is the reference's ``LayerWeights`` order
(``config.cuh:77-89``, flattened in ``model.py:30-44``): input norm, q, k, v,
q_norm, k_norm, o, post-attention norm, gate, up, down.
"""
from __future__ import annotations

import os
from dataclasses import dataclass, field

import numpy as np
import torch

HIDDEN = 1024
INTER = 3072
N_Q = 16
N_KV = 8
HEAD_DIM = 128
Q_SIZE = N_Q * HEAD_DIM
KV_SIZE = N_KV * HEAD_DIM
VOCAB = 151936
N_LAYERS = 28
EPS = 1e-6
ROPE_THETA = 1.0e6

LAYER_FIELDS = (
    "input_norm", "q", "k", "v", "q_norm", "k_norm",
    "o", "post_norm", "gate", "up", "down",
)

LAYER_SHAPES = {
    "input_norm": (HIDDEN,),
    "q": (Q_SIZE, HIDDEN),
    "k": (KV_SIZE, HIDDEN),
    "v": (KV_SIZE, HIDDEN),
    "q_norm": (HEAD_DIM,),
    "k_norm": (HEAD_DIM,),
    "o": (HIDDEN, Q_SIZE),
    "post_norm": (HIDDEN,),
    "gate": (INTER, HIDDEN),
    "up": (INTER, HIDDEN),
    "down": (HIDDEN, INTER),
}

NORM_FIELDS = ("input_norm", "q_norm", "k_norm", "post_norm")


@dataclass
class QwenWeights:
    """BF16 weights on the CPU (or moved to a device with :meth:`to`)."""

    embed: torch.Tensor                      # [VOCAB, HIDDEN], tied with the LM head
    final_norm: torch.Tensor                 # [HIDDEN]
    layers: list = field(default_factory=list)  # list of dicts keyed by LAYER_FIELDS
    seed: int = 0
    vocab: int = VOCAB

    @property
    def n_layers(self) -> int:
        return len(self.layers)

    def flat_layer_list(self) -> list:
        """The 28*11 list the reference binding takes (``model.py:30-44``)."""
        out = []
        for lw in self.layers:
            out.extend(lw[f] for f in LAYER_FIELDS)
        return out

    def to(self, device) -> "QwenWeights":
        return QwenWeights(
            embed=self.embed.to(device),
            final_norm=self.final_norm.to(device),
            layers=[{k: v.to(device) for k, v in lw.items()} for lw in self.layers],
            seed=self.seed,
            vocab=self.vocab,
        )

    def checksum(self) -> float:
        """Cheap fingerprint used to detect generator drift between machines."""
        s = float(self.embed[:64].float().sum()) + float(self.embed[-64:].float().sum())
        for lw in self.layers[:2] + self.layers[-1:]:
            for f in ("q", "down", "input_norm"):
                s += float(lw[f].reshape(-1)[:4096].float().sum())
        return s


def _normal_bf16(seed: int, index: int, shape, std: float) -> torch.Tensor:
    rng = np.random.default_rng([seed, index])
    a = rng.standard_normal(size=shape, dtype=np.float32)
    a *= np.float32(std)
    return torch.from_numpy(a).to(torch.bfloat16)


def make_weights(seed: int = 0, n_layers: int = N_LAYERS, vocab: int = VOCAB,
                 std: float = 0.02, perturb_norms: bool = False,
                 threads: int | None = None) -> QwenWeights:
    """Generate the synthetic model. ~1.2 GB of BF16 at full size.

    Tensor ``i`` (embedding = 1, then 11 per layer in ``LAYER_FIELDS`` order,
    then the final norm) draws from ``default_rng([seed, i])``; the tensors are
    generated on a thread pool (numpy fills without holding the GIL).
    """
    from concurrent.futures import ThreadPoolExecutor

    jobs = [("embed", None, 1, (vocab, HIDDEN), False)]
    i = 1
    for li in range(n_layers):
        for f in LAYER_FIELDS:
            i += 1
            jobs.append((f, li, i, LAYER_SHAPES[f], f in NORM_FIELDS))
    jobs.append(("final_norm", None, i + 1, (HIDDEN,), True))

    def run(job):
        _, _, idx, shape, is_norm = job
        if is_norm:
            if perturb_norms:
                return (1.0 + _normal_bf16(seed, idx, shape, 0.1).float()).to(torch.bfloat16)
            return torch.ones(shape, dtype=torch.bfloat16)
        return _normal_bf16(seed, idx, shape, std)

    n = threads or min(16, os.cpu_count() or 1)
    with ThreadPoolExecutor(max_workers=n) as ex:
        tensors = list(ex.map(run, jobs))
    embed = tensors[0]
    final_norm = tensors[-1]
    layers = [dict() for _ in range(n_layers)]
    for job, t in zip(jobs[1:-1], tensors[1:-1]):
        layers[job[1]][job[0]] = t
    return QwenWeights(embed=embed, final_norm=final_norm, layers=layers, seed=seed, vocab=vocab)


def prompt_ids(seed: int, length: int, vocab: int = VOCAB) -> torch.Tensor:
    """Uniform random prompt ids, ``torch.randint`` with a seeded generator."""
    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, vocab, (length,), generator=g, dtype=torch.int64)


def rope_tables(max_seq: int, dtype=torch.float32):
    """cos/sin tables ``[max_seq, HEAD_DIM]``.

    Same construction as the reference driver (``model.py:47-53``) and HF's
    default rotary embedding (inv_freq = theta^(-2i/d), emb = cat(f, f)),
    computed in FP32 on the CPU, then cast to ``dtype`` (the reference passes
    BF16 tables).
    """
    dims = torch.arange(0, HEAD_DIM, 2, dtype=torch.int64).to(torch.float32)
    inv_freq = 1.0 / (ROPE_THETA ** (dims / HEAD_DIM))
    pos = torch.arange(max_seq, dtype=torch.float32)
    freqs = torch.outer(pos, inv_freq)
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)
