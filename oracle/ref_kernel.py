"""Drive the reference CUDA kernel built from its own sources (test infrastructure).

``oracle/_ref/libref_megakernel.so`` (see ``oracle/build_ref.py``) exports the
reference's ``launch_decode_kernel`` (megakernel.cu:898-994) and the
``ref_decode_call`` shim that repeats its binding's per-call work
(pytorch_binding.cu:62-126). Used by the GPU tests as a second parity anchor
and by ``bench.py --impl reference`` to time the reference kernel on this GPU.
"""
from __future__ import annotations

import ctypes
import os

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "_ref", "libref_megakernel.so")


def available() -> bool:
    return os.path.exists(LIB)


def load():
    if not available():
        raise FileNotFoundError(f"{LIB} not built (python oracle/build_ref.py)")
    lib = ctypes.CDLL(LIB)
    lib.ref_decode_call.restype = ctypes.c_int
    lib.ref_decode_call.argtypes = [ctypes.c_int] + [ctypes.c_void_p] * 8 + [
        ctypes.POINTER(ctypes.c_void_p), ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    return lib


class RefDecoder:
    """The reference's per-call decode (fresh scratch and table every call)."""

    def __init__(self, embed, final_norm, layer_weights, cos_bf16, sin_bf16, k_cache, v_cache):
        self.lib = load()
        self.embed, self.final_norm = embed, final_norm
        self.cos, self.sin = cos_bf16, sin_bf16
        self.k, self.v = k_cache, v_cache
        self.layers = layer_weights
        self.table = (ctypes.c_void_p * len(layer_weights))(*[t.data_ptr() for t in layer_weights])
        self.max_seq = int(k_cache.shape[2])

    def decode(self, token: int, position: int) -> torch.Tensor:
        dev = self.embed.device
        f32 = dict(dtype=torch.float32, device=dev)
        # the reference binding's 10 scratch tensors (pytorch_binding.cu:51-60)
        scratch = [torch.empty(1024, dtype=torch.bfloat16, device=dev), torch.empty(1024, **f32),
                   torch.empty(1024, **f32), torch.empty(2048, **f32), torch.empty(1024, **f32),
                   torch.empty(3072, **f32), torch.empty(151936, **f32), torch.empty(2048, **f32),
                   torch.empty(1024, **f32), torch.empty(1024, **f32)]
        ptrs = (ctypes.c_void_p * 10)(*[t.data_ptr() for t in scratch])
        code = self.lib.ref_decode_call(int(token), self.embed.data_ptr(), self.embed.data_ptr(),
                                        self.final_norm.data_ptr(), ctypes.cast(self.table, ctypes.c_void_p),
                                        self.cos.data_ptr(), self.sin.data_ptr(), self.k.data_ptr(),
                                        self.v.data_ptr(), ptrs, int(position), self.max_seq,
                                        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        if code != 0:
            raise RuntimeError(f"reference decode failed with CUDA error {code}")
        return scratch[6]


def load_launcher():
    """The reference's own ``launch_decode_kernel`` (megakernel.cu:898-927) from
    the library built from its sources."""
    lib = load()
    fn = lib.launch_decode_kernel
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_int] + [ctypes.c_void_p] * 18 + [ctypes.c_int] * 3 + [ctypes.c_void_p]
    return fn


def time_reference_resident(steps: int = 64, warmup: int = 5, seed: int = 0) -> dict:
    """Per-token time of the reference kernel alone: the device LayerWeights table
    and the scratch vectors are allocated once and kept, and the CUDA events
    bracket the launch only (no per-call cudaMalloc/cudaFree, no table copy).
    Host argmax between calls, outside the timed region."""
    from .weights import make_weights, rope_tables
    dev = torch.device("cuda", torch.cuda.current_device())
    w = make_weights(seed).to(dev)
    cos, sin = rope_tables(512, torch.bfloat16)
    cos, sin = cos.to(dev), sin.to(dev)
    k = torch.zeros((28, 8, 512, 128), dtype=torch.bfloat16, device=dev)
    v = torch.zeros_like(k)
    table = torch.tensor([t.data_ptr() for t in w.flat_layer_list()], dtype=torch.int64, device=dev)
    f32 = dict(dtype=torch.float32, device=dev)
    scratch = [torch.empty(1024, dtype=torch.bfloat16, device=dev), torch.empty(1024, **f32),
               torch.empty(1024, **f32), torch.empty(2048, **f32), torch.empty(1024, **f32),
               torch.empty(3072, **f32), torch.empty(151936, **f32), torch.empty(2048, **f32),
               torch.empty(1024, **f32), torch.empty(1024, **f32)]
    fn = load_launcher()
    stream = torch.cuda.current_stream()

    def call(tok, pos):
        code = fn(int(tok), w.embed.data_ptr(), w.embed.data_ptr(), w.final_norm.data_ptr(), table.data_ptr(),
                  cos.data_ptr(), sin.data_ptr(), k.data_ptr(), v.data_ptr(), *[t.data_ptr() for t in scratch],
                  int(pos), int(pos) + 1, 512, ctypes.c_void_p(stream.cuda_stream))
        if code != 0:
            raise RuntimeError(f"reference launch failed with CUDA error {code}")

    tok = 1
    for p in range(32 + warmup):
        call(tok, p)
        tok = int(torch.argmax(scratch[6]).item())
    times = []
    for i in range(steps):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        call(tok, 32 + warmup + i)
        e.record(stream)
        e.synchronize()
        times.append(s.elapsed_time(e))
        tok = int(torch.argmax(scratch[6]).item())
    ms = sum(times) / len(times)
    return {"us_per_token": ms * 1000.0, "tok_s": 1000.0 / ms, "steps": steps,
            "source": "reference megakernel.cu built from its sources for sm_100a (oracle/_ref): "
                      "launch_decode_kernel alone, table and scratch resident, CUDA events around the launch"}


def time_reference(steps: int = 64, warmup: int = 5, seed: int = 0) -> dict:
    """Per-token time of the reference kernel on this GPU, config 0 shapes.

    Same protocol as model.py:107-127: CUDA events around each decode call,
    host argmax between calls (the call includes the binding's table
    allocation and cudaFree, as in the published numbers).
    """
    from .weights import make_weights, rope_tables
    dev = torch.device("cuda", torch.cuda.current_device())
    w = make_weights(seed).to(dev)
    cos, sin = rope_tables(512, torch.bfloat16)
    cos, sin = cos.to(dev), sin.to(dev)
    k = torch.zeros((28, 8, 512, 128), dtype=torch.bfloat16, device=dev)
    v = torch.zeros_like(k)
    r = RefDecoder(w.embed, w.final_norm, w.flat_layer_list(), cos, sin, k, v)
    tok = 1
    for p in range(32 + warmup):
        tok = int(torch.argmax(r.decode(tok, p)).item())
    times = []
    for i in range(steps):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        logits = r.decode(tok, 32 + warmup + i)
        e.record()
        e.synchronize()
        times.append(s.elapsed_time(e))
        tok = int(torch.argmax(logits).item())
    ms = sum(times) / len(times)
    return {"us_per_token": ms * 1000.0, "tok_s": 1000.0 / ms, "steps": steps,
            "source": "reference megakernel.cu built from its sources for sm_100a (oracle/_ref), "
                      "timed per decode call as model.py:107-127 does"}
