"""Host-side checks that need no GPU: the C ABI library loads and exports every
declared symbol, the static work split covers every row exactly once, and the
Python entry points reject bad arguments before any CUDA call."""
import ctypes
import os
import re

import pytest
import torch

from megakernel_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
VOCAB = 151936


def declared_functions():
    src = open(os.path.join(ROOT, "include", "mkb200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    names = re.findall(r"\b([A-Za-z_][A-Za-z0-9_]*)\s*\(", src)
    skip = {"if", "for", "while", "sizeof", "return", "defined"}
    return sorted({n for n in names if n not in skip and (n.startswith("mkb_") or n.startswith("launch_decode_kernel"))})


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_functions()
    assert "launch_decode_kernel" in names and "mkb_engine_step" in names
    assert "launch_decode_kernel_noalloc" in names
    for n in names:
        assert hasattr(lib, n), n
    assert {s[0] for s in _lib.SIGNATURES} == set(names)


def test_shared_memory_and_workspace_sizes():
    lib = _lib.load()
    assert lib.mkb_smem_bytes() <= 232448
    assert lib.mkb_workspace_bytes() > 0 and lib.mkb_workspace_bytes() % 128 == 0


def _cover(ranges, n):
    seen = [0] * n
    for a, b in ranges:
        assert 0 <= a <= b <= n
        for i in range(a, b):
            seen[i] += 1
    return seen


@pytest.mark.parametrize("grid", [128, 144, 148, 160, 256])
def test_plan_covers_every_row_once(grid):
    plans = [_lib.plan(grid, c) for c in range(grid)]
    assert all(v == 1 for v in _cover([(p["qa"], p["qb"]) for p in plans], 4096))
    assert all(v == 1 for v in _cover([(p["ja"], p["jb"]) for p in plans], 3072))
    assert all(v == 1 for v in _cover([(p["da"], p["db"]) for p in plans], 1024))
    lm = [0] * 0
    va = sorted((p["va"], p["vb"]) for p in plans)
    assert va[0][0] == 0 and va[-1][1] == VOCAB
    assert all(va[i][1] == va[i + 1][0] for i in range(len(va) - 1))
    gs = plans[0]["group_size"]
    assert gs == grid // 8
    for h in range(8):
        grp = [p for p in plans if p["in_bc"] and p["h"] == h]
        assert len(grp) == gs
        assert all(v == 1 for v in _cover([(p["oa"], p["ob"]) for p in grp], 1024))
    # per-CTA bounds the kernel relies on (shared arrays of 32 SwiGLU rows, 5 down rows per chunk)
    assert max(p["jb"] - p["ja"] for p in plans) <= 32
    assert max(p["ob"] - p["oa"] for p in plans if p["in_bc"]) <= 1024
    del lm


def test_qkv_chunks_never_cross_matrices():
    lib = _lib.load()
    for qa, qb in [(0, 4096), (2040, 2070), (3060, 3100), (4090, 4096)]:
        r = qa
        while r < qb:
            e = lib.mkb_qkv_chunk_end(r, qb)
            assert r < e <= qb and e - r <= 16
            assert (r < 2048) == (e - 1 < 2048)
            assert (r < 3072) == (e - 1 < 3072)
            r = e


@pytest.mark.parametrize("cache_len", [1, 2, 33, 160, 384, 385, 512, 3585, 3840, 4096])
def test_attention_splits_cover_the_cache(cache_len):
    lib = _lib.load()
    for gs in (16, 18, 32):
        s = lib.mkb_choose_splits(cache_len, gs)
        assert 1 <= s <= min(gs, 32)
        if cache_len <= 384:
            assert s == 1
        parts = [_lib.key_range(cache_len, s, c) for c in range(gs)]
        if s == 1:
            assert all(p == (0, cache_len) for p in parts)
        else:
            assert all(v == 1 for v in _cover(parts[:s], cache_len))
            assert all(p[0] == p[1] for p in parts[s:])
            assert all(p[1] - p[0] >= 1 for p in parts[:s])


def test_engine_rejects_cpu_tensors():
    from megakernel_b200 import DecodeEngine
    e = torch.zeros((VOCAB, 1024), dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="CUDA"):
        DecodeEngine(e, torch.ones(1024, dtype=torch.bfloat16), [], torch.zeros(1), torch.zeros(1))


def test_extension_decode_rejects_bad_arguments():
    import megakernel_b200 as mk
    ext = mk.extension()
    e = torch.zeros((4, 4), dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        ext.decode(0, e, e, e, [e] * 308, e, e, e, e, 0, 512)


@pytest.mark.parametrize("grid", [128, 140, 148, 160, 256])
@pytest.mark.parametrize("cache_len", [1, 33, 64, 65, 100, 160, 384])
def test_cluster_pair_attention_halves_cover_the_cache(grid, cache_len):
    """Below the group split (caches up to 384 keys), a CTA attends over all keys,
    or, from kPairSplitKeys (65) on, when its cluster pair shares the KV head,
    over one half: the two halves of a pair tile [0, cache_len) exactly."""
    lib = _lib.load()
    for cta in range(0, grid, 2):
        outs, pairs = [], []
        for r in (0, 1):
            o = (ctypes.c_int32 * 2)()
            pairs.append(lib.mkb_attn_keys(cache_len, 1, grid, cta + r, o))
            outs.append((o[0], o[1]))
        assert pairs[0] == pairs[1]
        plan = _lib.plan(grid, cta)
        if plan["in_bc"] and grid // 8 % 2 == 0:
            assert pairs[0] == 1  # even group sizes put both CTAs of a pair on one head
        if pairs[0] and cache_len >= 65:
            assert outs[0][0] == 0 and outs[0][1] == outs[1][0] and outs[1][1] == cache_len
            assert outs[0][1] - outs[0][0] >= 1 and outs[1][1] - outs[1][0] >= 1
        else:
            assert outs == [(0, cache_len), (0, cache_len)]


def test_engine_prefill_rejects_bad_arguments():
    lib = _lib.load()
    ids = (ctypes.c_int * 4)(1, 2, 3, 4)
    assert lib.mkb_engine_prefill(None, ctypes.cast(ids, ctypes.c_void_p), 4, 0, None, None) != 0


def test_every_error_code_has_a_name():
    """Each ErrorCode of the kernel (mkb_config.cuh) has a name in the C ABI
    (mkb_error_name) and in the Python table; unknown codes say so."""
    src = open(os.path.join(ROOT, "megakernel_b200", "csrc", "mkb_config.cuh")).read()
    body = src[src.index("enum ErrorCode"):]
    body = body[:body.index("};")]
    codes = {name: int(val) for name, val in re.findall(r"\b(kErr\w+)\s*=\s*(\d+)", body)}
    assert codes["kErrNone"] == 0 and "kErrRange" in codes
    lib = _lib.load()
    for name, val in codes.items():
        c_name = lib.mkb_error_name(val).decode()
        assert c_name != "unknown", name
        assert _lib.ERROR_NAMES[val] == c_name, name
    assert lib.mkb_error_name(max(codes.values()) + 1).decode() == "unknown"


def test_decode_args_mirror_matches_the_header():
    """The ctypes mirror of mkb_decode_args lists the header's fields in order."""
    src = open(os.path.join(ROOT, "include", "mkb200.h")).read()
    body = src[src.index("typedef struct mkb_decode_args {"):src.index("} mkb_decode_args;")]
    body = re.sub(r"/\*.*?\*/", "", body, flags=re.S).split("{", 1)[1]
    names = []
    for decl in body.split(";"):
        decl = decl.strip()
        if not decl:
            continue
        head, _, rest = decl.rpartition(" ")
        # "int layer_begin, layer_end" declares several fields
        decl = re.sub(r"\[\d+\]$", "", decl)  # arrays: "void* peer_workspaces[8]"
        first = decl.split(",")
        names.append(re.findall(r"\**(\w+)$", first[0].strip())[0])
        names += [re.sub(r"^\*+", "", x.strip()) for x in first[1:]]
    assert names == [f[0] for f in _lib.DecodeArgs._fields_]
