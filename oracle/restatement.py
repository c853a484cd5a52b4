"""PyTorch-FP32 CPU restatement of the reference decode step (test infrastructure).

Follows the stage order and numerics of the reference megakernel
(``megakernel.cu:744-893``):

* residual stream and every activation in FP32 (``megakernel.cu:760-769``);
* BF16 weights upcast to FP32 and accumulated in FP32 (every GEMV stage);
* the new K/V are rounded to BF16 when appended to the cache and attention reads
  the BF16 cache for every key, the new one included
  (``megakernel.cu:613-620,279,300``);
* RoPE uses the caller's cos/sin table row at ``position``, first half only,
  rotate-half form (``megakernel.cu:512-513,550-555``);
* attention scale 1/sqrt(head_dim) (``megakernel.cu:266``), GQA with two Q heads
  per KV head (``megakernel.cu:246-248``).

With an FP32 cache and FP32 tables this is the same computation as HF's eager
Qwen3 path (``modeling_qwen3.py`` RMSNorm/RoPE/eager attention), which the CPU
tests check to ~1e-5.

Every function returns the intermediates the GPU tests compare stage by stage.
"""
from __future__ import annotations

import torch

from .weights import EPS, HEAD_DIM, HIDDEN, N_KV, N_Q, QwenWeights


def rmsnorm(r: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """``megakernel.cu:704-739`` / ``:148-182``: r * w * rsqrt(mean(r^2) + eps)."""
    ms = (r.double() ** 2).mean().float()
    return r * torch.rsqrt(ms + EPS) * w.float()


def head_norm_rope(x: torch.Tensor, w: torch.Tensor, cos_row: torch.Tensor,
                   sin_row: torch.Tensor) -> torch.Tensor:
    """Per-head RMSNorm over 128 then rotate-half RoPE (``megakernel.cu:516-560``).

    x: [heads, 128] FP32. cos_row/sin_row: [128] (only the first 64 entries are
    used, as in the reference).
    """
    ms = (x.double() ** 2).mean(dim=-1, keepdim=True).float()
    y = x * torch.rsqrt(ms + EPS) * w.float()
    half = HEAD_DIM // 2
    c = cos_row[:half].float()
    s = sin_row[:half].float()
    a, b = y[:, :half], y[:, half:]
    return torch.cat((a * c - b * s, b * c + a * s), dim=-1)


def attention(q: torch.Tensor, k_rows: torch.Tensor, v_rows: torch.Tensor) -> torch.Tensor:
    """Softmax(q K^T / sqrt(128)) V per Q head (``megakernel.cu:228-370``).

    q: [16,128]; k_rows/v_rows: [8, cache_len, 128] FP32 (already upcast).
    """
    rep = N_Q // N_KV
    k = k_rows.repeat_interleave(rep, dim=0)
    v = v_rows.repeat_interleave(rep, dim=0)
    s = torch.einsum("hd,htd->ht", q.double(), k.double()) / (HEAD_DIM ** 0.5)
    p = torch.softmax(s, dim=-1)
    return torch.einsum("ht,htd->hd", p, v.double()).float()


def decode_layer(lw: dict, r: torch.Tensor, layer: int, position: int, cache_len: int,
                 k_cache: torch.Tensor, v_cache: torch.Tensor,
                 cos_table: torch.Tensor, sin_table: torch.Tensor) -> dict:
    """One decoder layer; mutates ``k_cache``/``v_cache`` at ``[layer, :, position]``.

    Returns the stage outputs: ``x`` (input norm), ``q``/``k``/``v`` raw GEMV
    outputs, ``q_rot``/``k_rot``, ``attn``, ``r_mid`` (after o_proj + residual),
    ``x2`` (post norm), ``m`` (SwiGLU), ``r_out``.
    """
    out = {}
    x = rmsnorm(r, lw["input_norm"])                                  # :704-739
    q = lw["q"].float() @ x                                           # :633-701
    k = lw["k"].float() @ x
    v = lw["v"].float() @ x
    out.update(x=x, q=q, k=k, v=v)
    cos_row, sin_row = cos_table[position], sin_table[position]
    q_rot = head_norm_rope(q.view(N_Q, HEAD_DIM), lw["q_norm"], cos_row, sin_row)   # :516-560
    k_rot = head_norm_rope(k.view(N_KV, HEAD_DIM), lw["k_norm"], cos_row, sin_row)  # :565-616
    k_cache[layer, :, position] = k_rot.to(k_cache.dtype)                           # :613-614
    v_cache[layer, :, position] = v.view(N_KV, HEAD_DIM).to(v_cache.dtype)          # :618-620
    out.update(q_rot=q_rot, k_rot=k_rot)
    attn = attention(q_rot, k_cache[layer, :, :cache_len].float(),
                     v_cache[layer, :, :cache_len].float()).reshape(-1)            # :228-370
    r_mid = r + lw["o"].float() @ attn                                # :191-225
    x2 = rmsnorm(r_mid, lw["post_norm"])                              # :148-182
    g = lw["gate"].float() @ x2                                       # :100-142
    u = lw["up"].float() @ x2
    m = torch.nn.functional.silu(g) * u
    r_out = r_mid + lw["down"].float() @ m                            # :53-90
    out.update(attn=attn, r_mid=r_mid, x2=x2, m=m, r_out=r_out)
    return out


def lm_head(embed: torch.Tensor, final_norm: torch.Tensor, r: torch.Tensor):
    """Final norm + tied LM head (``megakernel.cu:870-886``) + argmax (``model.py:97``)."""
    x = rmsnorm(r, final_norm)
    logits = embed.float() @ x
    return x, logits


def decode_step(w: QwenWeights, token: int, position: int, k_cache: torch.Tensor,
                v_cache: torch.Tensor, cos_table: torch.Tensor, sin_table: torch.Tensor,
                cache_len: int | None = None, keep_layers: bool = False) -> dict:
    """Full single-token decode (``megakernel.cu:783-886``).

    ``cache_len`` defaults to ``position + 1`` (``pytorch_binding.cu:98``).
    Returns ``logits`` [V] FP32, ``token`` (first-occurrence argmax) and
    ``r_final``; with ``keep_layers`` also every layer's stage outputs.
    """
    if cache_len is None:
        cache_len = position + 1
    r = w.embed[token].float()                                        # :783-795
    layers = []
    for li, lw in enumerate(w.layers):
        o = decode_layer(lw, r, li, position, cache_len, k_cache, v_cache, cos_table, sin_table)
        r = o["r_out"]
        if keep_layers:
            layers.append(o)
    x, logits = lm_head(w.embed, w.final_norm, r)
    return {"logits": logits, "token": int(torch.argmax(logits)), "r_final": r,
            "x_final": x, "layers": layers}


def prefill_cache(w: QwenWeights, ids: torch.Tensor, max_seq: int, cache_dtype=torch.bfloat16):
    """Fill a ``[L, 8, max_seq, 128]`` cache by running :func:`decode_step` over a prompt.

    The GPU tests use HF prefill instead (as the reference does); this slower
    path exists for small self-contained CPU checks.
    """
    from .weights import rope_tables
    k = torch.zeros((w.n_layers, N_KV, max_seq, HEAD_DIM), dtype=cache_dtype)
    v = torch.zeros_like(k)
    cos, sin = rope_tables(max_seq, torch.float32)
    last = None
    for p, t in enumerate(ids.tolist()):
        last = decode_step(w, t, p, k, v, cos, sin)
    return k, v, last


def top2_margin(logits: torch.Tensor) -> float:
    t = torch.topk(logits.double(), 2).values
    return float(t[0] - t[1])


__all__ = [
    "rmsnorm", "head_norm_rope", "attention", "decode_layer", "lm_head",
    "decode_step", "prefill_cache", "top2_margin", "HIDDEN",
]
