"""ctypes binding of ``libmkb200.so`` (the C ABI in ``include/mkb200.h``).

The library is built in-tree by ``megakernel_b200.build``. Importing this
module without the built library raises: there is no fallback path.
"""
from __future__ import annotations

import ctypes
import os
from ctypes import (POINTER, Structure, c_float, c_int, c_int32, c_size_t, c_uint32,
                    c_ulonglong, c_void_p, c_char_p)

HERE = os.path.dirname(os.path.abspath(__file__))
# MKB200_LIB selects another build of the library (same ABI), e.g. a debug build.
LIB_PATH = os.environ.get("MKB200_LIB") or os.path.join(HERE, "libmkb200.so")

MKB_FLAG_LM_HEAD = 1
MKB_FLAG_SKIP_FINAL_NORM = 2
MKB_FLAG_ADVANCE_STEP = 4

ERROR_NAMES = {
    0: "ok",
    1: "timeout waiting for a grid transition",
    2: "timeout waiting for a shared-memory ring slot",
    3: "timeout waiting for the greedy token broadcast",
    4: "bad arguments (range or alignment) seen on the device",
    5: "a partial sum outside the counted fixed-point range (|x| >= 2^19 or NaN)",
}


class DecodeArgs(Structure):
    """Mirror of ``mkb_decode_args`` (field order and types must match)."""

    _fields_ = [
        ("embed", c_void_p),
        ("lm_head", c_void_p),
        ("final_norm", c_void_p),
        ("layers", c_void_p),
        ("down_t", c_void_p),
        ("cos_table", c_void_p),
        ("sin_table", c_void_p),
        ("rope_fp32", c_int),
        ("k_cache", c_void_p),
        ("v_cache", c_void_p),
        ("max_seq", c_int),
        ("layer_begin", c_int),
        ("layer_end", c_int),
        ("token", c_int),
        ("position", c_int),
        ("cache_len", c_int),
        ("step", c_void_p),
        ("n_tokens", c_int),
        ("flags", c_int),
        ("input_residual", c_void_p),
        ("logits", c_void_p),
        ("out_tokens", c_void_p),
        ("residual_out", c_void_p),
        ("q_out", c_void_p),
        ("k_out", c_void_p),
        ("v_out", c_void_p),
        ("mlp_out", c_void_p),
        ("workspace", c_void_p),
        ("grid", c_int),
        ("splits", c_int),
        ("timeout_ns", c_ulonglong),
        ("withhold_cta", c_int),
        ("trace", c_void_p),
        ("trace_cap", c_int),
        ("prompt_tokens", c_void_p),
        ("err_flag", c_void_p),
        ("stop_token", c_int),
        ("tp_rank", c_int),
        ("tp_size", c_int),
        ("peer_workspaces", c_void_p * 8),
        ("mailbox", c_void_p),
        ("result", c_void_p),
    ]


class Model(Structure):
    """Mirror of ``mkb_model``."""

    _fields_ = [
        ("embed", c_void_p),
        ("lm_head", c_void_p),
        ("final_norm", c_void_p),
        ("layer_weights", POINTER(c_void_p)),
        ("n_layers", c_int),
        ("cos_table", c_void_p),
        ("sin_table", c_void_p),
        ("rope_fp32", c_int),
        ("k_cache", c_void_p),
        ("v_cache", c_void_p),
        ("max_seq", c_int),
        ("fused_down", c_int),
        ("use_graph", c_int),
        ("logits", c_void_p),
        ("tp_size", c_int),
    ]


# (name, restype, argtypes) for every symbol declared in include/mkb200.h
SIGNATURES = [
    ("launch_decode_kernel", c_int,
     [c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
      c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
      c_void_p, c_int, c_int, c_int, c_void_p]),
    ("launch_decode_kernel_noalloc", c_int,
     [c_int, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
      c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
      c_void_p, c_int, c_int, c_int, c_void_p]),
    ("mkb_noalloc_status", c_int, [c_int, POINTER(c_uint32)]),
    ("mkb_decode_args_init", None, [POINTER(DecodeArgs)]),
    ("mkb_decode", c_int, [POINTER(DecodeArgs), c_void_p]),
    ("mkb_workspace_bytes", c_size_t, []),
    ("mkb_workspace_reset", c_int, [c_void_p, c_void_p]),
    ("mkb_workspace_status", c_int, [c_void_p, POINTER(c_uint32)]),
    ("mkb_workspace_tag_base", c_int, [c_void_p, POINTER(c_uint32), POINTER(c_uint32)]),
    ("mkb_default_workspace", c_int, [c_int, POINTER(c_void_p)]),
    ("mkb_error_name", c_char_p, [c_uint32]),
    ("mkb_transpose_down", c_int, [c_void_p, c_void_p, c_void_p]),
    ("mkb_engine_create", c_int, [POINTER(Model), POINTER(c_void_p)]),
    ("mkb_engine_step", c_int, [c_void_p, c_int, c_int, POINTER(c_int), c_void_p]),
    ("mkb_engine_generate", c_int, [c_void_p, c_int, c_int, c_int, c_void_p, c_void_p]),
    ("mkb_engine_generate_until", c_int, [c_void_p, c_int, c_int, c_int, c_int, c_void_p, c_void_p]),
    ("mkb_engine_serve_open", c_int, [c_void_p, c_int, c_int, c_ulonglong, c_void_p]),
    ("mkb_engine_serve_step", c_int, [c_void_p, c_int, POINTER(c_int)]),
    ("mkb_engine_serve_close", c_int, [c_void_p]),
    ("mkb_engine_prefill", c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p]),
    ("mkb_engine_prefill_batched", c_int, [c_void_p, c_void_p, c_int, c_int, c_void_p, c_void_p]),
    ("mkb_gemm_bf16_split", c_int, [c_void_p, c_void_p, c_void_p, c_void_p, c_int, c_int, c_int, c_void_p]),
    ("mkb_engine_logits", c_void_p, [c_void_p]),
    ("mkb_engine_workspace", c_void_p, [c_void_p]),
    ("mkb_engine_tp_attach", c_int, [c_void_p, c_int, c_int, POINTER(c_void_p)]),
    ("mkb_ipc_export", c_int, [c_void_p, ctypes.c_char_p]),
    ("mkb_ipc_open", c_int, [ctypes.c_char_p, POINTER(c_void_p)]),
    ("mkb_ipc_close", c_int, [c_void_p]),
    ("mkb_engine_grid", c_int, [c_void_p]),
    ("mkb_engine_destroy", None, [c_void_p]),
    ("mkb_plan_query", c_int, [c_int, c_int, POINTER(c_int32)]),
    ("mkb_plan_query_tp", c_int, [c_int, c_int, c_int, c_int, POINTER(c_int32)]),
    ("mkb_qkv_global_row", c_int, [c_int, c_int, c_int]),
    ("mkb_choose_splits", c_int, [c_int, c_int]),
    ("mkb_key_range", None, [c_int, c_int, c_int, POINTER(c_int32)]),
    ("mkb_attn_keys", c_int, [c_int, c_int, c_int, c_int, POINTER(c_int32)]),
    ("mkb_qkv_chunk_end", c_int, [c_int, c_int]),
    ("mkb_smem_bytes", c_size_t, []),
    ("mkb_version", c_int, []),
]

_lib = None


class MkbError(RuntimeError):
    pass


def load(path: str | None = None):
    """Load the shared library once; raises if it has not been built."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = path or LIB_PATH
    if not os.path.exists(p):
        raise MkbError(f"libmkb200.so not built at {p}; run megakernel_b200.build.build_all()")
    lib = ctypes.CDLL(p)
    for name, res, args in SIGNATURES:
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = lib
    return lib


def check(code: int, what: str = "") -> None:
    if code != 0:
        raise MkbError(f"{what}: CUDA error {code} ({cuda_error_name(code)})")


def cuda_error_name(code: int) -> str:
    try:
        import torch  # noqa: F401
        from torch.cuda import cudart  # type: ignore
        return str(cudart().cudaGetErrorString(code))
    except Exception:  # pragma: no cover - name lookup is best effort
        return f"cudaError {code}"


def new_args() -> DecodeArgs:
    a = DecodeArgs()
    load().mkb_decode_args_init(ctypes.byref(a))
    return a


def workspace_status(ws_ptr: int) -> list:
    out = (c_uint32 * 8)()
    check(load().mkb_workspace_status(c_void_p(ws_ptr), out), "mkb_workspace_status")
    return list(out)


def plan(grid: int, cta: int) -> dict:
    out = (c_int32 * 16)()
    if load().mkb_plan_query(grid, cta, out) != 0:
        raise ValueError("bad grid/cta")
    keys = ["qa", "qb", "in_bc", "h", "c", "oa", "ob", "ja", "jb", "da", "db", "va", "vb", "group_size"]
    return dict(zip(keys, list(out)[:14]))


def plan_tp(grid: int, cta: int, tp_rank: int, tp_size: int) -> dict:
    out = (c_int32 * 16)()
    if load().mkb_plan_query_tp(grid, cta, tp_rank, tp_size, out) != 0:
        raise ValueError("bad grid/cta/tp shape")
    keys = ["qa", "qb", "in_bc", "h", "c", "oa", "ob", "ja", "jb", "da", "db", "va", "vb", "group_size", "hl"]
    return dict(zip(keys, list(out)[:15]))


def key_range(cache_len: int, splits: int, c: int) -> tuple:
    out = (c_int32 * 2)()
    load().mkb_key_range(cache_len, splits, c, out)
    return out[0], out[1]
