"""launch_decode_kernel_noalloc (workspace in a static device array, no device
allocation at any call) against launch_decode_kernel (workspace allocated once
per device) over two calls in a row on identical inputs.

The file name sorts last so the check also runs after every other GPU test
(the static array's first-call set-up then happens late in the process); it
passes on its own as well. The two launchers run the same kernel, but its
grid-wide float atomics add partial sums in arrival order, and a last-bit
difference that flips the BF16 rounding of one appended K/V element carries
into every later layer. So the bound is the kernel's run-to-run spread, not
bit equality: logits, residual and the last layer's raw QKV within
2e-3 x max(1, max|x|) (a tenth of the HF parity bound), appended K/V within
4 BF16 ulp + 2e-3, the greedy token identical unless the top-2 margin is
below 4e-3, and every other cache slot bit-identical.
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


def _launch(fn, tok, pos, w, table, cos, sin, k, v, bufs):
    code = fn(tok, w.embed.data_ptr(), w.embed.data_ptr(), w.final_norm.data_ptr(), table.data_ptr(),
              cos.data_ptr(), sin.data_ptr(), k.data_ptr(), v.data_ptr(), None, bufs["res"].data_ptr(), None,
              None, None, bufs["mlp"].data_ptr(), bufs["logits"].data_ptr(), bufs["q"].data_ptr(),
              bufs["k"].data_ptr(), bufs["v"].data_ptr(), pos, pos + 1, MAX_SEQ,
              ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    return code


def test_noalloc_launcher_matches_allocating_launcher(cuda_device):
    lib = _lib.load()
    w = W.make_weights(0).to(cuda_device)
    table = build_layer_table(w.flat_layer_list(), DEV)
    cos, sin = mk.rope_tables(MAX_SEQ, DEV, torch.bfloat16)
    g = torch.Generator(device=DEV).manual_seed(7)
    k0 = (torch.randn((28, 8, MAX_SEQ, 128), generator=g, device=DEV) * 0.5).to(torch.bfloat16)
    v0 = (torch.randn((28, 8, MAX_SEQ, 128), generator=g, device=DEV) * 0.5).to(torch.bfloat16)
    arms = {}
    for name in ("alloc", "noalloc"):
        f32 = dict(dtype=torch.float32, device=DEV)
        bufs = {n: torch.zeros(s, **f32) for n, s in
                [("res", 1024), ("q", 2048), ("k", 1024), ("v", 1024), ("mlp", 3072), ("logits", 151936)]}
        arms[name] = dict(k=k0.clone(), v=v0.clone(), bufs=bufs, fn=(lib.launch_decode_kernel if name == "alloc"
                                                                    else lib.launch_decode_kernel_noalloc))
    tok = 1234
    for call in range(2):
        pos = POS + call
        outs = {}
        for name, a in arms.items():
            _lib.check(_launch(a["fn"], tok, pos, w, table, cos, sin, a["k"], a["v"], a["bufs"]), name)
            torch.cuda.synchronize()
            outs[name] = {n: b.clone() for n, b in a["bufs"].items()}
        ref, got = outs["alloc"], outs["noalloc"]
        for n in ("logits", "res", "q", "k", "v"):
            d = (got[n] - ref[n]).abs().max().item()
            bound = 2e-3 * max(1.0, ref[n].abs().max().item())
            assert d <= bound, f"call {call}: {n} differs by {d} (bound {bound})"
        top2 = torch.topk(ref["logits"], 2).values
        if float(top2[0] - top2[1]) >= 4e-3:
            assert int(torch.argmax(got["logits"])) == int(torch.argmax(ref["logits"]))
        ka, kb = arms["alloc"]["k"][:, :, pos].float(), arms["noalloc"]["k"][:, :, pos].float()
        va, vb = arms["alloc"]["v"][:, :, pos].float(), arms["noalloc"]["v"][:, :, pos].float()
        assert ((kb - ka).abs() <= ka.abs() * 2.0 ** -5 + 2e-3).all(), f"call {call}: appended K"
        assert ((vb - va).abs() <= va.abs() * 2.0 ** -5 + 2e-3).all(), f"call {call}: appended V"
        # nothing else in the caches moved
        for nm in ("k", "v"):
            rest_a = torch.cat([arms["alloc"][nm][:, :, :POS], arms["alloc"][nm][:, :, pos + 1:]], dim=2)
            rest_b = torch.cat([arms["noalloc"][nm][:, :, :POS], arms["noalloc"][nm][:, :, pos + 1:]], dim=2)
            assert torch.equal(rest_a, rest_b)
        tok = int(torch.argmax(ref["logits"]))
