"""launch_decode_kernel_noalloc against launch_decode_kernel.

Some callers cannot allocate device memory while they decode: a serving loop
that runs under a fixed memory budget, a host runtime that forbids allocation
after start-up, or code that must not synchronise the device (cudaMalloc and
cudaFree can). For them the no-allocation launcher keeps its synchronisation
workspace in a static device array of the library, set up on the first call.

The two launchers run the same kernel on identical inputs, and the kernel is
bit-deterministic (every cross-CTA sum is an integer add of counted fixed-point
words, every combine has a fixed order), so the check is equality: logits,
residual, the last layer's raw QKV and SwiGLU vector and the appended K/V rows,
on two calls in a row. It also checks that the second call changes no device
allocation (free device memory stays the same) and that the status word of the
static workspace reads 0 after each call.

This file sorts last so that a run stopping at the first failure has run every
other test first; it passes on its own as well.
"""
import ctypes

import pytest
import torch

import megakernel_b200 as mk
from megakernel_b200 import _lib
from megakernel_b200.engine import build_layer_table
from oracle import weights as W

pytestmark = pytest.mark.gpu
DEV = "cuda:0"
MAX_SEQ = 512
POS = 40
NAMES = [("res", 1024), ("q", 2048), ("k", 1024), ("v", 1024), ("mlp", 3072), ("logits", 151936)]


def _launch(fn, tok, pos, w, table, cos, sin, k, v, bufs):
    return fn(tok, w.embed.data_ptr(), w.embed.data_ptr(), w.final_norm.data_ptr(), table.data_ptr(),
              cos.data_ptr(), sin.data_ptr(), k.data_ptr(), v.data_ptr(), None, bufs["res"].data_ptr(), None,
              None, None, bufs["mlp"].data_ptr(), bufs["logits"].data_ptr(), bufs["q"].data_ptr(),
              bufs["k"].data_ptr(), bufs["v"].data_ptr(), pos, pos + 1, MAX_SEQ,
              ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


def _noalloc_status(lib):
    out = (ctypes.c_uint32 * 8)()
    _lib.check(lib.mkb_noalloc_status(0, out), "mkb_noalloc_status")
    return list(out)


def _inputs():
    w = W.make_weights(0).to(DEV)
    table = build_layer_table(w.flat_layer_list(), DEV)
    cos, sin = mk.rope_tables(MAX_SEQ, DEV, torch.bfloat16)
    g = torch.Generator(device=DEV).manual_seed(7)
    k0 = (torch.randn((28, 8, MAX_SEQ, 128), generator=g, device=DEV) * 0.5).to(torch.bfloat16)
    v0 = (torch.randn((28, 8, MAX_SEQ, 128), generator=g, device=DEV) * 0.5).to(torch.bfloat16)
    return w, table, cos, sin, k0, v0


def _arm(fn, k0, v0):
    f32 = dict(dtype=torch.float32, device=DEV)
    return dict(fn=fn, k=k0.clone(), v=v0.clone(), bufs={n: torch.zeros(s, **f32) for n, s in NAMES},
                keep={n: torch.zeros(s, **f32) for n, s in NAMES})


def test_noalloc_launcher_matches_allocating_launcher(cuda_device):
    lib = _lib.load()
    w, table, cos, sin, k0, v0 = _inputs()
    arms = {"alloc": _arm(lib.launch_decode_kernel, k0, v0), "noalloc": _arm(lib.launch_decode_kernel_noalloc, k0, v0)}
    tok = 1234
    for call in range(2):
        pos = POS + call
        for name, a in arms.items():
            torch.cuda.synchronize()
            free_before = torch.cuda.mem_get_info()[0]
            _lib.check(_launch(a["fn"], tok, pos, w, table, cos, sin, a["k"], a["v"], a["bufs"]), name)
            torch.cuda.synchronize()
            if name == "noalloc":
                assert _noalloc_status(lib)[0] == 0
                if call == 1:  # the first call did the one-time set-up
                    assert torch.cuda.mem_get_info()[0] == free_before
            for n, b in a["bufs"].items():
                a["keep"][n].copy_(b)
        ref, got = arms["alloc"]["keep"], arms["noalloc"]["keep"]
        for n, _ in NAMES:
            assert torch.equal(got[n], ref[n]), f"call {call}: {n} differs"
        assert torch.isfinite(ref["logits"]).all()
        assert torch.equal(arms["alloc"]["k"], arms["noalloc"]["k"]), f"call {call}: K cache"
        assert torch.equal(arms["alloc"]["v"], arms["noalloc"]["v"]), f"call {call}: V cache"
        assert not torch.equal(arms["noalloc"]["k"][:, :, pos], k0[:, :, pos])  # the row was appended
        tok = int(torch.argmax(ref["logits"]))


def test_noalloc_failure_is_visible_and_cleared_by_the_next_call(cuda_device):
    """A layer table with a misaligned weight is refused inside the kernel: the
    logits are NaN, the static workspace's status reads kErrBadArgs (4), and the
    next call, which clears the array, decodes normally."""
    lib = _lib.load()
    w, table, cos, sin, k0, v0 = _inputs()
    layers = w.flat_layer_list()
    shifted = torch.ones(1024 + 8, dtype=torch.bfloat16, device=DEV)
    bad = list(layers)
    bad[0] = shifted[1:1025]
    bad_table = build_layer_table(bad, DEV)
    arm = _arm(lib.launch_decode_kernel_noalloc, k0, v0)
    _lib.check(_launch(arm["fn"], 77, POS, w, bad_table, cos, sin, arm["k"], arm["v"], arm["bufs"]), "noalloc")
    torch.cuda.synchronize()
    assert _noalloc_status(lib)[0] == 4
    assert bool(torch.isnan(arm["bufs"]["logits"]).all())
    assert torch.equal(arm["k"], k0)
    ref = _arm(lib.launch_decode_kernel, k0, v0)
    _lib.check(_launch(arm["fn"], 77, POS, w, table, cos, sin, arm["k"], arm["v"], arm["bufs"]), "noalloc")
    _lib.check(_launch(ref["fn"], 77, POS, w, table, cos, sin, ref["k"], ref["v"], ref["bufs"]), "alloc")
    torch.cuda.synchronize()
    assert _noalloc_status(lib)[0] == 0
    assert torch.equal(arm["bufs"]["logits"], ref["bufs"]["logits"])
