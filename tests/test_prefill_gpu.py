"""Batched prefill (mkb_engine_prefill_batched): the tcgen05 GEMM on its own
against float64, and the whole prefill against HF's FP32 prefill (the BASELINE
oracle, model.py:72-87) and against the token-by-token in-engine prefill.

Tolerances: the GEMM splits its FP32 A operand into a BF16 high part and the
BF16 remainder, so products carry ~2^-16 relative error and the FP32 sums add
~K * 2^-24: max |err| <= 1e-4 * sqrt(K) * scale. The model-level bounds are the
HF parity bounds of the decode tests (logits 2e-2, cosine 0.999, K/V 2e-2)."""
import ctypes
import os

import pytest
import torch

import megakernel_b200 as mk
from megakernel_b200 import _lib
from oracle import configs as C
from oracle import hf_reference as H
from oracle import weights as W

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


def cosine(a, b):
    return torch.nn.functional.cosine_similarity(a.double(), b.double(), dim=0).item()


@pytest.mark.parametrize("m,n,k", [(128, 128, 64), (200, 256, 1024), (1, 384, 3072), (333, 128, 2048),
                                   (4096, 4096, 256), (4000, 1920, 128)])
def test_gemm_split_matches_float64(m, n, k, cuda_device):
    """The last two shapes give every persistent CTA three or four output tiles
    (both TMEM accumulators reused; 256- and 128-column tiles)."""
    g = torch.Generator(device=DEV).manual_seed(m + n + k)
    a = torch.randn((m, k), generator=g, device=DEV)
    a_hi = a.to(torch.bfloat16)
    a_lo = (a - a_hi.float()).to(torch.bfloat16)
    b = (torch.randn((n, k), generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    c = torch.full((m, n), float("nan"), dtype=torch.float32, device=DEV)
    code = _lib.load().mkb_gemm_bf16_split(a_hi.data_ptr(), a_lo.data_ptr(), b.data_ptr(), c.data_ptr(), m, n, k,
                                            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    _lib.check(code, "mkb_gemm_bf16_split")
    torch.cuda.synchronize()
    ref = (a_hi.double() + a_lo.double()) @ b.double().t()
    scale = ref.abs().max().item()
    err = (c.double() - ref).abs().max().item()
    assert err <= 1e-4 * (k ** 0.5) * max(scale, 1e-3), (err, scale)


@pytest.fixture(scope="module")
def w_cpu():
    return W.make_weights(0)


@pytest.fixture(scope="module")
def w_gpu(w_cpu, cuda_device):
    return w_cpu.to(cuda_device)


@pytest.fixture(scope="module")
def hf_model(w_cpu):
    return H.build_model(w_cpu, threads=os.cpu_count())


@pytest.mark.parametrize("n_prompt", [1, 32, 200, 400])
def test_batched_prefill_matches_hf(n_prompt, w_gpu, hf_model):
    ids = C.config0_prompt(0).view(-1)[:n_prompt] if n_prompt <= 32 else torch.randint(
        0, 151936, (n_prompt,), generator=torch.Generator().manual_seed(5))
    logits_hf, cache = H.prefill(hf_model, ids)
    kh, vh = H.to_kernel_cache(cache, 28, 512, torch.bfloat16)
    kg = torch.zeros((28, 8, 512, 128), dtype=torch.bfloat16, device=DEV)
    vg = torch.zeros_like(kg)
    eng = mk.DecodeEngine(w_gpu.embed, w_gpu.final_norm, w_gpu.flat_layer_list(), kg, vg)
    nxt = eng.prefill(ids, batched=True)
    lg = eng.logits.cpu()
    assert (lg - logits_hf).abs().max().item() <= 2e-2
    assert cosine(lg, logits_hf) > 0.999
    t2 = torch.topk(logits_hf.double(), 2).values
    if float(t2[0] - t2[1]) > 0.05:
        assert nxt == int(torch.argmax(logits_hf))
    for got, ref in ((kg[:, :, :n_prompt], kh[:, :, :n_prompt]), (vg[:, :, :n_prompt], vh[:, :, :n_prompt])):
        torch.testing.assert_close(got.float().cpu(), ref.float(), rtol=2e-2, atol=2e-2)
    assert not kg[:, :, n_prompt:].any()
    tok = int(torch.argmax(logits_hf))
    for i in range(3):  # decoding continues from the batched cache
        eng.step(tok, n_prompt + i)
        ref, cache = H.step(hf_model, cache, tok)
        lg = eng.logits.cpu()
        assert (lg - ref).abs().max().item() <= 2e-2 and cosine(lg, ref) > 0.999, f"step {i}"
        tok = int(torch.argmax(ref))
    assert eng.status()[0] == 0
    eng.close()


def test_batched_prefill_matches_token_by_token_prefill(w_gpu):
    """The batched and the token-by-token prefill agree closely (same BF16 cache
    rounding, FP32 residuals, ~2^-16 products) and continue the same way.

    The logits bound is half the HF bound. It leaves room for rounding: two
    batched builds that differ only in where the compiler fused one multiply-add
    of the q/k RMSNorm (layer 0's K/V identical to 2e-6) end 1.7e-3 apart in the
    logits after 28 random-weight layers, and 4.9e-3 vs 5.2e-3 from the
    token-by-token prefill."""
    ids = torch.randint(0, 151936, (150,), generator=torch.Generator().manual_seed(9))
    k1 = torch.zeros((28, 8, 256, 128), dtype=torch.bfloat16, device=DEV)
    v1, k2, v2 = torch.zeros_like(k1), torch.zeros_like(k1), torch.zeros_like(k1)
    e1 = mk.DecodeEngine(w_gpu.embed, w_gpu.final_norm, w_gpu.flat_layer_list(), k1, v1)
    e2 = mk.DecodeEngine(w_gpu.embed, w_gpu.final_norm, w_gpu.flat_layer_list(), k2, v2)
    n1 = e1.prefill(ids, batched=True)
    n2 = e2.prefill(ids)
    l1, l2 = e1.logits.cpu(), e2.logits.cpu()
    assert (l1 - l2).abs().max().item() <= 1e-2
    assert cosine(l1, l2) > 0.99999
    t2 = torch.topk(l2.double(), 2).values
    if float(t2[0] - t2[1]) > 5e-3:
        assert n1 == n2
    for got, ref in ((k1, k2), (v1, v2)):
        torch.testing.assert_close(got.float(), ref.float(), rtol=2e-2, atol=2e-2)
    e1.close()
    e2.close()


def test_batched_prefill_continues_at_unaligned_offsets(w_gpu):
    """Three batched prefills (100 tokens, 157 at position 100, 1 at position 257)
    into a 300-slot cache (not a multiple of the attention's 128-key tiles) equal
    one batched prefill of all 258 tokens: the earlier keys' V^T comes from the
    cache through v_transpose_kernel, over key blocks that the same prefill's
    QKV epilogue partly wrote."""
    ids = torch.randint(0, 151936, (258,), generator=torch.Generator().manual_seed(4))
    k1 = torch.zeros((28, 8, 300, 128), dtype=torch.bfloat16, device=DEV)
    v1, k2, v2 = torch.zeros_like(k1), torch.zeros_like(k1), torch.zeros_like(k1)
    e1 = mk.DecodeEngine(w_gpu.embed, w_gpu.final_norm, w_gpu.flat_layer_list(), k1, v1)
    e2 = mk.DecodeEngine(w_gpu.embed, w_gpu.final_norm, w_gpu.flat_layer_list(), k2, v2)
    e1.prefill(ids[:100], batched=True)
    e1.prefill(ids[100:257], position=100, batched=True)
    n1 = e1.prefill(ids[257:], position=257, batched=True)
    n2 = e2.prefill(ids, batched=True)
    assert (e1.logits - e2.logits).abs().max().item() <= 1e-3
    for got, ref in ((k1, k2), (v1, v2)):
        torch.testing.assert_close(got.float(), ref.float(), rtol=1.6e-2, atol=1e-3)
    assert not k1[:, :, 258:].any() and not v1[:, :, 258:].any()
    t2 = torch.topk(e2.logits.double(), 2).values
    if float(t2[0] - t2[1]) > 1e-3:
        assert n1 == n2
    assert e1.status()[0] == 0 and e2.status()[0] == 0
    e1.close()
    e2.close()


def test_batched_prefill_at_an_offset_continues_a_cache(w_gpu):
    """A second batched prefill at position 40 after a first one at 0 equals one
    batched prefill of the concatenated prompt (the causal attention reads the
    earlier rows from the cache)."""
    ids = torch.randint(0, 151936, (100,), generator=torch.Generator().manual_seed(3))
    k1 = torch.zeros((28, 8, 128, 128), dtype=torch.bfloat16, device=DEV)
    v1, k2, v2 = torch.zeros_like(k1), torch.zeros_like(k1), torch.zeros_like(k1)
    e1 = mk.DecodeEngine(w_gpu.embed, w_gpu.final_norm, w_gpu.flat_layer_list(), k1, v1)
    e2 = mk.DecodeEngine(w_gpu.embed, w_gpu.final_norm, w_gpu.flat_layer_list(), k2, v2)
    e1.prefill(ids[:40], batched=True)
    n1 = e1.prefill(ids[40:], position=40, batched=True)
    n2 = e2.prefill(ids, batched=True)
    assert (e1.logits - e2.logits).abs().max().item() <= 1e-3
    torch.testing.assert_close(k1.float(), k2.float(), rtol=1.6e-2, atol=1e-3)
    t2 = torch.topk(e2.logits.double(), 2).values
    if float(t2[0] - t2[1]) > 1e-3:
        assert n1 == n2
    e1.close()
    e2.close()
