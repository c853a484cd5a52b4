"""Torch-facing wrappers over the C ABI (``libmkb200.so``).

* :class:`DecodeEngine` -- the resident engine (``mkb_engine_*``): device
  LayerWeights table, transposed down weights, workspace and the per-token CUDA
  graph are built once; :meth:`step` decodes one token through the public C
  call (host token in, host argmax out), :meth:`generate` runs an on-device
  greedy loop of ``n`` tokens in one persistent launch.
* :func:`decode_call` -- the explicit-argument launch (``mkb_decode``) used by
  the stage-level tests (single layer, isolated LM head).

Weights are the reference's tensors: BF16, ``[out, in]`` row-major, the 11
per-layer tensors in ``LayerWeights`` order (``model.py:30-44``). The KV cache
is the reference's ``[layers, 8, max_seq, 128]`` BF16 layout (``model.py:81-87``)
and stays owned by the caller; it is updated in place.
"""
from __future__ import annotations

import ctypes
from ctypes import byref, c_int, c_void_p

import torch

from . import _lib
from .rope import rope_tables

HIDDEN, INTER, VOCAB, N_KV, HEAD_DIM = 1024, 3072, 151936, 8, 128
LAYER_SHAPES = [
    (HIDDEN,), (2048, HIDDEN), (1024, HIDDEN), (1024, HIDDEN), (HEAD_DIM,), (HEAD_DIM,),
    (HIDDEN, 2048), (HIDDEN,), (INTER, HIDDEN), (INTER, HIDDEN), (HIDDEN, INTER),
]


def _require(cond: bool, msg: str):
    if not cond:
        raise ValueError(msg)


def check_tensor(t: torch.Tensor, name: str, shape=None, dtype=torch.bfloat16, device=None):
    _require(isinstance(t, torch.Tensor), f"{name} must be a tensor")
    _require(t.is_cuda, f"{name} must be a CUDA tensor")
    _require(t.dtype == dtype, f"{name} must be {dtype}, got {t.dtype}")
    _require(t.is_contiguous(), f"{name} must be contiguous")
    _require(t.data_ptr() % 16 == 0, f"{name} must be 16-byte aligned")
    if shape is not None:
        _require(tuple(t.shape) == tuple(shape), f"{name} must have shape {tuple(shape)}, got {tuple(t.shape)}")
    if device is not None:
        _require(t.device == device, f"{name} must be on {device}")


def check_model(embed, final_norm, layer_weights, k_cache, v_cache, lm_head=None, tp_size: int = 1):
    """Validation shared by every entry point (the reference checks nothing).
    With tensor parallelism the caches are the rank's shard of 8 / tp_size KV heads."""
    check_tensor(embed, "embed_weight", (VOCAB, HIDDEN))
    dev = embed.device
    check_tensor(final_norm, "final_norm_weight", (HIDDEN,), device=dev)
    if lm_head is not None:
        check_tensor(lm_head, "lm_head_weight", (VOCAB, HIDDEN), device=dev)
    _require(len(layer_weights) % 11 == 0 and 0 < len(layer_weights) // 11 <= 28,
             "layer_weights must hold 11 tensors per layer (LayerWeights order)")
    for i, t in enumerate(layer_weights):
        check_tensor(t, f"layer_weights[{i}]", LAYER_SHAPES[i % 11], device=dev)
    n_layers = len(layer_weights) // 11
    _require(tp_size in (1, 2, 4, 8), "tp_size must be 1, 2, 4 or 8")
    heads = N_KV // tp_size
    _require(k_cache.dim() == 4 and k_cache.shape[0] == n_layers and k_cache.shape[1] == heads
             and k_cache.shape[3] == HEAD_DIM, f"k_cache must be [layers, {heads}, max_seq, 128]")
    check_tensor(k_cache, "k_cache", device=dev)
    check_tensor(v_cache, "v_cache", tuple(k_cache.shape), device=dev)
    return n_layers, int(k_cache.shape[2])


def _stream_ptr(stream=None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return int(s.cuda_stream)


class DecodeEngine:
    """Resident batch-one decode engine over the reference's tensors."""

    def __init__(self, embed, final_norm, layer_weights, k_cache, v_cache, cos=None, sin=None,
                 lm_head=None, fused_down: bool = True, use_graph: bool = True, tp_size: int = 1):
        self.lib = _lib.load()
        self.n_layers, self.max_seq = check_model(embed, final_norm, layer_weights, k_cache, v_cache, lm_head,
                                                  tp_size)
        self.tp_size = tp_size
        dev = embed.device
        if cos is None:
            cos, sin = rope_tables(self.max_seq, dev, torch.float32)
        _require(cos.dtype in (torch.float32, torch.bfloat16) and sin.dtype == cos.dtype,
                 "cos/sin must both be FP32 or both BF16")
        check_tensor(cos, "cos_table", dtype=cos.dtype, device=dev)
        check_tensor(sin, "sin_table", tuple(cos.shape), dtype=cos.dtype, device=dev)
        _require(cos.dim() == 2 and cos.shape[1] == HEAD_DIM and cos.shape[0] >= self.max_seq,
                 "RoPE tables must be [>=max_seq, 128]")
        # keep every tensor alive as long as the engine
        self._keep = (embed, final_norm, list(layer_weights), k_cache, v_cache, cos, sin, lm_head)
        self.k_cache, self.v_cache = k_cache, v_cache
        self.logits = torch.empty(VOCAB, dtype=torch.float32, device=dev)
        self.device = dev
        ptrs = (c_void_p * len(layer_weights))(*[t.data_ptr() for t in layer_weights])
        self._ptrs = ptrs
        m = _lib.Model()
        m.embed = embed.data_ptr()
        m.lm_head = (lm_head if lm_head is not None else embed).data_ptr()
        m.final_norm = final_norm.data_ptr()
        m.layer_weights = ctypes.cast(ptrs, ctypes.POINTER(c_void_p))
        m.n_layers = self.n_layers
        m.cos_table = cos.data_ptr()
        m.sin_table = sin.data_ptr()
        m.rope_fp32 = 1 if cos.dtype == torch.float32 else 0
        m.k_cache = k_cache.data_ptr()
        m.v_cache = v_cache.data_ptr()
        m.max_seq = self.max_seq
        m.fused_down = 1 if fused_down else 0
        m.use_graph = 1 if use_graph else 0
        m.logits = self.logits.data_ptr()
        m.tp_size = tp_size
        h = c_void_p()
        with torch.cuda.device(dev):
            torch.cuda.synchronize()
            _lib.check(self.lib.mkb_engine_create(byref(m), byref(h)), "mkb_engine_create")
        self._h = h
        self.grid = self.lib.mkb_engine_grid(h)

    @property
    def workspace_ptr(self) -> int:
        return self.lib.mkb_engine_workspace(self._h)

    def step(self, token: int, position: int, stream=None) -> int:
        """Decode one token at ``position`` (cache_len = position + 1); returns the argmax id."""
        _require(0 <= token < VOCAB, "token_id out of range")
        _require(0 <= position < self.max_seq, "position out of range")
        out = c_int(-1)
        with torch.cuda.device(self.device):
            code = self.lib.mkb_engine_step(self._h, int(token), int(position), byref(out),
                                            c_void_p(_stream_ptr(stream)))
        _lib.check(code, "mkb_engine_step")
        return out.value

    def generate(self, token: int, position: int, n: int, out: torch.Tensor | None = None, stream=None,
                 stop_token: int | None = None):
        """Greedy-decode ``n`` tokens on the device in one launch; returns int32 ids [n].

        ``stop_token`` (e.g. the tokenizer's ``eos_token_id``) ends the launch after
        the first generated token equal to it, as the reference loop does
        (model.py:102-105); the ids after it read -1. A token that did not complete
        because of an in-kernel error also reads -1, and the next engine call raises."""
        _require(n >= 1 and 0 <= position and position + n <= self.max_seq, "generate range out of bounds")
        _require(stop_token is None or 0 <= stop_token < VOCAB, "stop_token out of range")
        if out is None:
            out = torch.empty(n, dtype=torch.int32, device=self.device)
        with torch.cuda.device(self.device):
            code = self.lib.mkb_engine_generate_until(self._h, int(token), int(position), int(n),
                                                      -1 if stop_token is None else int(stop_token),
                                                      c_void_p(out.data_ptr()), c_void_p(_stream_ptr(stream)))
        _lib.check(code, "mkb_engine_generate")
        return out

    def prefill(self, ids, position: int = 0, stream=None, batched: bool = False) -> int:
        """In-engine prefill of prompt ``ids`` at ``position``.. (model.py:72-87 did this
        with HF). ``batched=False``: one persistent launch of the decode kernel feeds
        the prompt token by token. ``batched=True``: every prompt token of a layer at
        once -- tcgen05 tensor-core GEMMs for the projections, causal attention on
        the tensor cores (mkb_engine_prefill_batched). Either way the K/V rows are
        appended and the return value is the argmax of the last prompt token, the
        first generated token; ``logits`` holds its logits."""
        ids = torch.as_tensor(ids, dtype=torch.int32).flatten()
        n = int(ids.numel())
        _require(n >= 1 and 0 <= position and position + n <= self.max_seq, "prefill range out of bounds")
        _require(bool(((ids >= 0) & (ids < VOCAB)).all()), "token_id out of range")
        dev_ids = ids.to(self.device)
        nxt = torch.empty(1, dtype=torch.int32, device=self.device)
        with torch.cuda.device(self.device):
            fn = self.lib.mkb_engine_prefill_batched if batched else self.lib.mkb_engine_prefill
            code = fn(self._h, c_void_p(dev_ids.data_ptr()), n, int(position), c_void_p(nxt.data_ptr()),
                      c_void_p(_stream_ptr(stream)))
        _lib.check(code, "mkb_engine_prefill")
        out = int(nxt.item())
        st = self.status()
        if st[0] != 0:
            raise RuntimeError(f"in-kernel error {st}")
        return out

    def status(self) -> list:
        return _lib.workspace_status(self.workspace_ptr)

    # ---- serve session: one persistent launch, tokens through pinned memory ----
    def serve_open(self, position: int, max_tokens: int, timeout_s: float = 1.0, stream=None):
        """Start a session of up to ``max_tokens`` tokens at ``position``.. (see
        mkb_engine_serve_open): each :meth:`serve_step` hands one input token to the
        running launch and returns its argmax, without a launch or a copy."""
        _require(max_tokens >= 1 and 0 <= position and position + max_tokens <= self.max_seq,
                 "serve range out of bounds")
        with torch.cuda.device(self.device):
            _lib.check(self.lib.mkb_engine_serve_open(self._h, int(position), int(max_tokens),
                                                      int(timeout_s * 1e9), c_void_p(_stream_ptr(stream))),
                       "mkb_engine_serve_open")

    def serve_step(self, token: int) -> int:
        _require(0 <= token < VOCAB, "token_id out of range")
        out = c_int(-1)
        _lib.check(self.lib.mkb_engine_serve_step(self._h, int(token), byref(out)), "mkb_engine_serve_step")
        return out.value

    def serve_close(self):
        _lib.check(self.lib.mkb_engine_serve_close(self._h), "mkb_engine_serve_close")

    def ipc_handle(self) -> bytes:
        """64 bytes that let another process on this node map this engine's workspace."""
        buf = ctypes.create_string_buffer(64)
        with torch.cuda.device(self.device):
            _lib.check(self.lib.mkb_ipc_export(c_void_p(self.workspace_ptr), buf), "mkb_ipc_export")
        return buf.raw

    def attach_tp(self, tp_rank: int, tp_size: int, peer_workspaces: list):
        """Join a tensor-parallel group (see mkb_engine_tp_attach); peer_workspaces are
        device addresses valid on this GPU, this engine's own at index tp_rank."""
        _require(tp_size == self.tp_size, "tp_size differs from the one the engine was built for")
        arr = (c_void_p * tp_size)(*peer_workspaces)
        with torch.cuda.device(self.device):
            _lib.check(self.lib.mkb_engine_tp_attach(self._h, int(tp_rank), int(tp_size), arr),
                       "mkb_engine_tp_attach")
        self.tp_rank = tp_rank

    def close(self):
        if getattr(self, "_h", None):
            torch.cuda.synchronize(self.device)
            self.lib.mkb_engine_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def build_layer_table(layer_weights, device) -> torch.Tensor:
    """Device ``LayerWeights[n]`` table (11 pointers per layer, config.cuh:77-89)."""
    ptrs = torch.tensor([t.data_ptr() for t in layer_weights], dtype=torch.int64)
    return ptrs.to(device)


def decode_call(**kw) -> int:
    """Launch ``mkb_decode`` with keyword fields of ``mkb_decode_args``.

    Tensor values are converted to their data pointers; ``stream`` selects the
    CUDA stream (default: current). Returns the CUDA error code.
    """
    lib = _lib.load()
    stream = kw.pop("stream", None)
    a = _lib.new_args()
    for k, v in kw.items():
        if isinstance(v, torch.Tensor):
            v = v.data_ptr()
        setattr(a, k, v)
    return lib.mkb_decode(byref(a), c_void_p(_stream_ptr(stream)))
