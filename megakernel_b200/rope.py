"""RoPE cos/sin tables for the decode engine.

Same construction as the reference driver (``model.py:47-53``): inv_freq =
theta^(-2i/128) in FP32, angle = position * inv_freq, the 64 angles duplicated to
128 columns, cos/sin in FP32. The reference casts the tables to BF16; the
engine keeps them in FP32 by default (BF16 tables are still accepted through the
drop-in ``decode`` call), which keeps long-cache positions accurate.
"""
from __future__ import annotations

import torch

HEAD_DIM = 128
ROPE_THETA = 1.0e6


def rope_tables(max_seq: int, device=None, dtype=torch.float32):
    dims = torch.arange(0, HEAD_DIM, 2, dtype=torch.int64).to(torch.float32)
    inv_freq = 1.0 / (ROPE_THETA ** (dims / HEAD_DIM))
    pos = torch.arange(max_seq, dtype=torch.float32)
    freqs = torch.outer(pos, inv_freq)
    emb = torch.cat((freqs, freqs), dim=-1)
    cos = emb.cos().to(dtype)
    sin = emb.sin().to(dtype)
    if device is not None:
        cos, sin = cos.to(device), sin.to(device)
    return cos.contiguous(), sin.contiguous()
