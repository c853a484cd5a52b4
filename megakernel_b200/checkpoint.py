"""Qwen3 checkpoint loading: safetensors files -> the tensors the decode path takes.

The reference loads ``Qwen/Qwen3-0.6B`` through Hugging Face and flattens each
decoder layer's 11 weights in ``LayerWeights`` order (``model.py:24-44``). This
module reads the same checkpoint straight from its safetensors file(s) -- a
single ``model.safetensors``, a sharded set with ``model.safetensors.index.json``,
or one ``.safetensors`` path -- using the Hugging Face tensor names:

    model.embed_tokens.weight                 [vocab, 1024]
    model.layers.{i}.input_layernorm.weight   [1024]
    model.layers.{i}.self_attn.{q,k,v}_proj.weight
    model.layers.{i}.self_attn.{q,k}_norm.weight
    model.layers.{i}.self_attn.o_proj.weight
    model.layers.{i}.post_attention_layernorm.weight
    model.layers.{i}.mlp.{gate,up,down}_proj.weight
    model.norm.weight                         [1024]
    lm_head.weight                            (absent when tied to the embedding)

Every tensor is returned as a contiguous BF16 tensor on ``device`` (CUDA
allocations are 256-byte aligned, which the bulk copies need), with the shapes
checked against the Qwen3-0.6B architecture.
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass, field

import torch

HIDDEN, INTER, HEAD_DIM, VOCAB = 1024, 3072, 128, 151936

# LayerWeights order (config.cuh:77-89, model.py:30-44): (HF name suffix, shape)
LAYER_FIELDS = [
    ("input_layernorm.weight", (HIDDEN,)),
    ("self_attn.q_proj.weight", (2048, HIDDEN)),
    ("self_attn.k_proj.weight", (1024, HIDDEN)),
    ("self_attn.v_proj.weight", (1024, HIDDEN)),
    ("self_attn.q_norm.weight", (HEAD_DIM,)),
    ("self_attn.k_norm.weight", (HEAD_DIM,)),
    ("self_attn.o_proj.weight", (HIDDEN, 2048)),
    ("post_attention_layernorm.weight", (HIDDEN,)),
    ("mlp.gate_proj.weight", (INTER, HIDDEN)),
    ("mlp.up_proj.weight", (INTER, HIDDEN)),
    ("mlp.down_proj.weight", (HIDDEN, INTER)),
]


@dataclass
class Qwen3Weights:
    embed: torch.Tensor
    lm_head: torch.Tensor          # the embedding itself when the checkpoint ties them
    final_norm: torch.Tensor
    layer_weights: list = field(default_factory=list)  # n_layers * 11, LayerWeights order
    n_layers: int = 0
    tied: bool = True
    config: dict = field(default_factory=dict)


def _files(path: str) -> list:
    if os.path.isfile(path):
        return [path]
    index = os.path.join(path, "model.safetensors.index.json")
    if os.path.exists(index):
        with open(index) as f:
            shards = sorted(set(json.load(f)["weight_map"].values()))
        return [os.path.join(path, s) for s in shards]
    single = os.path.join(path, "model.safetensors")
    if os.path.exists(single):
        return [single]
    found = sorted(f for f in os.listdir(path) if f.endswith(".safetensors"))
    if not found:
        raise FileNotFoundError(f"no .safetensors file under {path}")
    return [os.path.join(path, f) for f in found]


def load_qwen3(path: str, device="cuda", n_layers: int | None = None) -> Qwen3Weights:
    """Read a Qwen3-0.6B checkpoint (file or directory) onto ``device``.

    ``n_layers`` defaults to the number of decoder layers the checkpoint holds
    (28 for Qwen3-0.6B); a checkpoint missing a tensor, or holding one of the
    wrong shape, raises ``ValueError``.
    """
    from safetensors import safe_open

    device = torch.device(device)
    where = {}
    for fn in _files(path):
        with safe_open(fn, framework="pt", device="cpu") as f:
            for k in f.keys():
                where[k] = fn

    def get(name, shape):
        if name not in where:
            raise ValueError(f"checkpoint has no tensor {name}")
        with safe_open(where[name], framework="pt", device="cpu") as f:
            t = f.get_tensor(name)
        if tuple(t.shape) != tuple(shape):
            raise ValueError(f"{name} has shape {tuple(t.shape)}, expected {tuple(shape)}")
        return t.to(device=device, dtype=torch.bfloat16).contiguous()

    have = sorted({int(k.split(".")[2]) for k in where if k.startswith("model.layers.")})
    if n_layers is None:
        n_layers = len(have)
    if not 1 <= n_layers <= 28 or have[:n_layers] != list(range(n_layers)):
        raise ValueError(f"checkpoint layers {have[:4]}... do not cover layers 0..{n_layers - 1}")
    embed = get("model.embed_tokens.weight", (VOCAB, HIDDEN))
    tied = "lm_head.weight" not in where
    lm_head = embed if tied else get("lm_head.weight", (VOCAB, HIDDEN))
    final_norm = get("model.norm.weight", (HIDDEN,))
    layers = []
    for i in range(n_layers):
        for suffix, shape in LAYER_FIELDS:
            layers.append(get(f"model.layers.{i}.{suffix}", shape))
    cfg = {}
    cfg_path = os.path.join(path if os.path.isdir(path) else os.path.dirname(path), "config.json")
    if os.path.exists(cfg_path):
        with open(cfg_path) as f:
            cfg = json.load(f)
    return Qwen3Weights(embed=embed, lm_head=lm_head, final_norm=final_norm, layer_weights=layers,
                        n_layers=n_layers, tied=tied, config=cfg)


def save_qwen3(path: str, embed, final_norm, layer_weights, lm_head=None) -> None:
    """Write tensors in LayerWeights order under the Hugging Face names (the
    inverse of :func:`load_qwen3`; ``lm_head`` omitted = tied)."""
    from safetensors.torch import save_file

    t = {"model.embed_tokens.weight": embed, "model.norm.weight": final_norm}
    if lm_head is not None:
        t["lm_head.weight"] = lm_head
    n = len(layer_weights) // len(LAYER_FIELDS)
    for i in range(n):
        for j, (suffix, _) in enumerate(LAYER_FIELDS):
            t[f"model.layers.{i}.{suffix}"] = layer_weights[i * len(LAYER_FIELDS) + j]
    save_file({k: v.detach().to("cpu").contiguous() for k, v in t.items()}, path)
