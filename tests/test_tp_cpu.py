"""Tensor-parallel decode, host side, on the CPU: the work split over ranks
covers every row of every weight exactly once (and the KV heads map onto each
rank's cache shard), and the set-up's handle exchange runs over gloo ranks."""
import os
import socket

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from megakernel_b200 import _lib
from megakernel_b200.tp import exchange_handles

VOCAB, INTER, HIDDEN = 151936, 3072, 1024


@pytest.mark.parametrize("tp_size", [1, 2, 4, 8])
@pytest.mark.parametrize("grid", [144, 148])
def test_tp_split_covers_every_row_once(tp_size, grid):
    lib = _lib.load()
    qkv = [0] * 4096
    inter = [0] * INTER
    vocab = [0] * VOCAB
    heads = {}
    for r in range(tp_size):
        for cta in range(grid):
            p = _lib.plan_tp(grid, cta, r, tp_size)
            for lr in range(p["qa"], p["qb"]):
                qkv[lib.mkb_qkv_global_row(r, tp_size, lr)] += 1
            for j in range(p["ja"], p["jb"]):
                inter[j] += 1
            for v in range(p["va"], p["vb"]):
                vocab[v] += 1
            if p["in_bc"]:
                # a rank's CTAs attend only over its own heads, cache shard index h - first head
                assert r * 8 // tp_size <= p["h"] < (r + 1) * 8 // tp_size
                assert p["hl"] == p["h"] - r * 8 // tp_size
                heads.setdefault(p["h"], []).append((p["oa"], p["ob"]))
    assert qkv == [1] * 4096
    assert inter == [1] * INTER
    assert vocab == [1] * VOCAB
    assert sorted(heads) == list(range(8))
    for h, rows in heads.items():  # each head's group covers every o_proj row once
        cover = [0] * HIDDEN
        for a, b in rows:
            for i in range(a, b):
                cover[i] += 1
        assert cover == [1] * HIDDEN, h


def test_tp_qkv_rows_are_the_ranks_heads():
    """Rank r's local q/k/v segments are its heads' rows of Wq, Wk and Wv."""
    lib = _lib.load()
    for size in (2, 4, 8):
        hl = 8 // size
        for r in range(size):
            rows = [lib.mkb_qkv_global_row(r, size, i) for i in range(512 * hl)]
            h0 = r * hl
            assert rows[:256 * hl] == list(range(256 * h0, 256 * (h0 + hl)))
            assert rows[256 * hl:384 * hl] == list(range(2048 + 128 * h0, 2048 + 128 * (h0 + hl)))
            assert rows[384 * hl:] == list(range(3072 + 128 * h0, 3072 + 128 * (h0 + hl)))


def test_single_gpu_plan_is_unchanged():
    for cta in (0, 17, 143, 147):
        assert {k: v for k, v in _lib.plan_tp(148, cta, 0, 1).items() if k != "hl"} == _lib.plan(148, cta)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        mine = bytes([rank]) * 64
        out[rank] = exchange_handles(mine)
    finally:
        dist.destroy_process_group()


def test_handle_exchange_over_gloo_ranks():
    world = 2
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_worker, args=(world, _free_port(), out), nprocs=world, join=True)
    for rank in range(world):
        assert out[rank] == [bytes([0]) * 64, bytes([1]) * 64]
