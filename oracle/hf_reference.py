"""BASELINE oracle: Hugging Face Qwen3 in FP32 on the CPU (test infrastructure).

Third-party dependency: ``transformers`` 5.5.0 (``Qwen3ForCausalLM``,
``models/qwen3/modeling_qwen3.py``), the model path the reference drives in
``model.py:24-27`` (load), ``model.py:72-73`` (prefill) and ``model.py:163-167``
(decode). The reference does not pin a version; this build pins the installed
5.5.0 and records it in the golden fixtures.

The model is built from :class:`oracle.weights.QwenWeights`: the BF16 weights
are upcast to FP32 exactly, embeddings are tied (``HF:443``), attention is the
eager path. ``prefill`` returns HF's FP32 cache and ``to_kernel_cache`` lays it
out as the reference's ``[L, 8, max_seq, 128]`` BF16 cache (``model.py:79-87``).
"""
from __future__ import annotations

import os

import torch

from .weights import (EPS, HEAD_DIM, HIDDEN, INTER, N_KV, N_Q, ROPE_THETA, QwenWeights)


def hf_config(n_layers: int, vocab: int):
    from transformers import Qwen3Config
    return Qwen3Config(
        vocab_size=vocab, hidden_size=HIDDEN, intermediate_size=INTER,
        num_hidden_layers=n_layers, num_attention_heads=N_Q, num_key_value_heads=N_KV,
        head_dim=HEAD_DIM, rms_norm_eps=EPS, tie_word_embeddings=True,
        rope_parameters={"rope_type": "default", "rope_theta": ROPE_THETA},
        max_position_embeddings=40960, attention_bias=False, hidden_act="silu",
    )


def build_model(w: QwenWeights, threads: int | None = None):
    """FP32 eager ``Qwen3ForCausalLM`` holding exactly ``w``'s values."""
    from transformers import Qwen3ForCausalLM
    if threads:
        torch.set_num_threads(threads)
    cfg = hf_config(w.n_layers, w.vocab)
    cfg._attn_implementation = "eager"
    with torch.device("meta"):
        model = Qwen3ForCausalLM(cfg)
    sd = {"model.embed_tokens.weight": w.embed.float(), "model.norm.weight": w.final_norm.float()}
    names = {
        "input_norm": "input_layernorm.weight", "q": "self_attn.q_proj.weight",
        "k": "self_attn.k_proj.weight", "v": "self_attn.v_proj.weight",
        "q_norm": "self_attn.q_norm.weight", "k_norm": "self_attn.k_norm.weight",
        "o": "self_attn.o_proj.weight", "post_norm": "post_attention_layernorm.weight",
        "gate": "mlp.gate_proj.weight", "up": "mlp.up_proj.weight", "down": "mlp.down_proj.weight",
    }
    for i, lw in enumerate(w.layers):
        for f, n in names.items():
            sd[f"model.layers.{i}.{n}"] = lw[f].float()
    sd["lm_head.weight"] = sd["model.embed_tokens.weight"]
    model.load_state_dict(sd, strict=False, assign=True)
    model.lm_head.weight = model.model.embed_tokens.weight
    # the rotary inv_freq buffers are non-persistent: rebuild them on the CPU
    from transformers.models.qwen3.modeling_qwen3 import Qwen3RotaryEmbedding
    model.model.rotary_emb = Qwen3RotaryEmbedding(cfg, device="cpu")
    model.eval()
    return model


@torch.inference_mode()
def prefill(model, ids: torch.Tensor):
    """HF prefill of ``ids`` (``model.py:72-76``): returns (last logits FP32, cache)."""
    out = model(ids.view(1, -1), use_cache=True)
    return out.logits[0, -1].float(), out.past_key_values


@torch.inference_mode()
def step(model, cache, token: int):
    """One HF decode step (``model.py:163-167``): returns (logits FP32, cache)."""
    out = model(torch.tensor([[token]], dtype=torch.int64), past_key_values=cache, use_cache=True)
    return out.logits[0, -1].float(), out.past_key_values


def to_kernel_cache(cache, n_layers: int, max_seq: int, dtype=torch.bfloat16):
    """HF DynamicCache -> reference layout ``[L, 8, max_seq, 128]`` (``model.py:79-87``)."""
    k = torch.zeros((n_layers, N_KV, max_seq, HEAD_DIM), dtype=dtype)
    v = torch.zeros_like(k)
    for layer in range(n_layers):
        lk = cache.layers[layer].keys[0]
        lv = cache.layers[layer].values[0]
        t = lk.shape[1]
        k[layer, :, :t] = lk.to(dtype)
        v[layer, :, :t] = lv.to(dtype)
    return k, v


@torch.inference_mode()
def greedy_decode(model, ids: torch.Tensor, n_steps: int, forced: list | None = None,
                  keep_logits=None):
    """Prefill then ``n_steps`` decode steps.

    Step ``i`` feeds token ``t_i`` at position ``len(ids) + i``; ``t_0`` is the
    argmax of the prefill logits and ``t_{i+1}`` the argmax of step ``i``'s
    logits, unless ``forced`` gives the tokens (teacher forcing). Returns
    ``(tokens_fed, logits_per_step)``; ``keep_logits(i, logits)`` may reduce
    what is kept per step (default: keep everything).
    """
    logits, cache = prefill(model, ids)
    fed, kept = [], []
    tok = int(torch.argmax(logits))
    for i in range(n_steps):
        if forced is not None:
            tok = int(forced[i])
        fed.append(tok)
        logits, cache = step(model, cache, tok)
        kept.append(keep_logits(i, logits) if keep_logits else logits)
        tok = int(torch.argmax(logits))
    return fed, kept


def default_threads() -> int:
    return max(1, os.cpu_count() or 1)


@torch.inference_mode()
def single_layer(model, layer: int, hidden: torch.Tensor, k_prefix: torch.Tensor,
                 v_prefix: torch.Tensor, position: int) -> dict:
    """One HF ``Qwen3DecoderLayer`` decode step over a given cache prefix (config 1).

    hidden: [1024]; k_prefix/v_prefix: [8, position, 128] (their values are
    upcast to FP32). Returns the layer output, the attention block output
    (o_proj, before the residual add) and the new K (after norm + RoPE) / V.
    """
    from transformers import DynamicCache
    lay = model.model.layers[layer]
    cache = DynamicCache(config=model.config)
    cache.update(k_prefix.float()[None], v_prefix.float()[None], layer)
    x = hidden.float().view(1, 1, -1)
    pos_ids = torch.tensor([[position]], dtype=torch.int64)
    pe = model.model.rotary_emb(x, pos_ids)
    captured = {}

    def hook(_m, _inp, out):
        captured["attn"] = out[0].reshape(-1).clone()

    hd = lay.self_attn.register_forward_hook(hook)
    try:
        out = lay(x, attention_mask=None, position_ids=pos_ids, past_key_values=cache,
                  use_cache=True, cache_position=torch.tensor([position]), position_embeddings=pe)
    finally:
        hd.remove()
    out = out[0] if isinstance(out, tuple) else out
    k_all = cache.layers[layer].keys[0]
    v_all = cache.layers[layer].values[0]
    return {"out": out.reshape(-1).float(), "attn_o": captured["attn"].float(),
            "k_new": k_all[:, position].float(), "v_new": v_all[:, position].float()}
