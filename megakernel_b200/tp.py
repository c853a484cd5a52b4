"""Tensor-parallel decode over 2, 4 or 8 GPUs of one node (one process per GPU).

Rank r holds KV heads [r*8/G, (r+1)*8/G) (its KV-cache shard), a block of
SwiGLU rows and a block of vocabulary rows; the full weights stay where they are
(each rank reads only its rows). Every layer's two all-reduces of the hidden
state happen inside the persistent kernel: o_proj partials are added straight
into every GPU's counted accumulators over NVLink, the down-projection sums are
reduced on each GPU first and then forwarded by one CTA per GPU, and the greedy
token is the maximum over all GPUs' candidates. Every poll reads local memory;
every copy reads this GPU's own memory.

The only host-side collective is the set-up: each rank exports its engine's
workspace (CUDA IPC), the handles are all-gathered with ``torch.distributed``
(any backend), and each rank maps the others'.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from .engine import DecodeEngine


def exchange_handles(handle: bytes, group=None) -> list:
    """All-gather one 64-byte handle per rank (rank order)."""
    import torch.distributed as dist
    out = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, handle, group=group)
    return out


class TPDecodeEngine:
    """One rank of a tensor-parallel decode group. Every method must be called
    on every rank with the same arguments (SPMD)."""

    def __init__(self, embed, final_norm, layer_weights, k_shard, v_shard, cos=None, sin=None, lm_head=None,
                 group=None, use_graph: bool = True):
        import torch.distributed as dist
        self.rank = dist.get_rank(group)
        self.size = dist.get_world_size(group)
        self.engine = DecodeEngine(embed, final_norm, layer_weights, k_shard, v_shard, cos=cos, sin=sin,
                                   lm_head=lm_head, fused_down=True, use_graph=use_graph, tp_size=self.size)
        handles = exchange_handles(self.engine.ipc_handle(), group)
        lib = _lib.load()
        self._opened = []
        peers = []
        with torch.cuda.device(self.engine.device):
            for g, h in enumerate(handles):
                if g == self.rank:
                    peers.append(self.engine.workspace_ptr)
                    continue
                p = ctypes.c_void_p()
                _lib.check(lib.mkb_ipc_open(h, ctypes.byref(p)), "mkb_ipc_open")
                self._opened.append(p.value)
                peers.append(p.value)
        self.engine.attach_tp(self.rank, self.size, peers)
        torch.cuda.synchronize(self.engine.device)
        dist.barrier(group)

    @property
    def logits(self) -> torch.Tensor:
        """FP32 [151936]; this rank fills its vocabulary rows (vocab_range)."""
        return self.engine.logits

    def vocab_range(self) -> tuple:
        v = 151936
        return v * self.rank // self.size, v * (self.rank + 1) // self.size

    def step(self, token: int, position: int, stream=None) -> int:
        return self.engine.step(token, position, stream)

    def generate(self, token: int, position: int, n: int, out=None, stream=None, stop_token=None):
        return self.engine.generate(token, position, n, out=out, stream=stream, stop_token=stop_token)

    def prefill(self, ids, position: int = 0, stream=None) -> int:
        return self.engine.prefill(ids, position, stream)

    def status(self) -> list:
        return self.engine.status()

    def close(self):
        torch.cuda.synchronize(self.engine.device)
        lib = _lib.load()
        with torch.cuda.device(self.engine.device):
            for p in self._opened:
                lib.mkb_ipc_close(ctypes.c_void_p(p))
        self._opened = []
        self.engine.close()


def shard_cache(cache: torch.Tensor, rank: int, size: int) -> torch.Tensor:
    """Rank's KV-head shard [L, 8/size, S, 128] of a full [L, 8, S, 128] cache."""
    h = cache.shape[1] // size
    return cache[:, rank * h:(rank + 1) * h].contiguous()
