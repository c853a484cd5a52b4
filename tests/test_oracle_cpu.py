"""The CPU oracle against Hugging Face Qwen3 and the committed golden fixtures.

These pin ``oracle.restatement`` (the checker of the GPU tests) to the
BASELINE oracle: HF ``Qwen3ForCausalLM`` FP32 on the CPU (transformers 5.5.0).
"""
import os

import numpy as np
import pytest
import torch

from oracle import configs as C
from oracle import hf_reference as H
from oracle import restatement as R
from oracle import weights as W

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.fixture(scope="module")
def full_weights():
    return W.make_weights(0)


def test_weights_are_reproducible(full_weights):
    g = np.load(os.path.join(GOLDEN, "config0.npz"))
    assert abs(full_weights.checksum() - float(g["checksum"])) < 1e-6
    again = W.make_weights(0, n_layers=1, threads=1)
    assert torch.equal(again.embed, full_weights.embed)
    assert torch.equal(again.layers[0]["gate"], full_weights.layers[0]["gate"])


def test_restatement_matches_hf_two_layers():
    """FP32 cache + FP32 RoPE: restatement == HF eager to ~1e-5 (teacher forced)."""
    w = W.make_weights(3, n_layers=2, perturb_norms=True)
    model = H.build_model(w, threads=os.cpu_count())
    ids = W.prompt_ids(3, 6)
    logits, cache = H.prefill(model, ids)
    k, v = H.to_kernel_cache(cache, 2, 32, torch.float32)
    cos, sin = W.rope_tables(32)
    tok = int(torch.argmax(logits))
    for i in range(3):
        o = R.decode_step(w, tok, 6 + i, k, v, cos, sin)
        hl, cache = H.step(model, cache, tok)
        assert (o["logits"] - hl).abs().max().item() < 1e-4
        tok = int(torch.argmax(hl))


def test_golden_config0_restatement(full_weights):
    """First decode steps of config 0 against the committed HF logits."""
    g = np.load(os.path.join(GOLDEN, "config0.npz"))
    model = H.build_model(full_weights, threads=os.cpu_count())
    ids = torch.from_numpy(g["prompt"])
    assert torch.equal(ids, C.config0_prompt(0))
    logits, cache = H.prefill(model, ids)
    assert int(torch.argmax(logits)) == int(g["prefill_argmax"])
    k, v = H.to_kernel_cache(cache, 28, 64, torch.float32)
    cos, sin = W.rope_tables(64)
    idx = torch.from_numpy(g["sample_idx"])
    for i in range(3):
        o = R.decode_step(full_weights, int(g["fed"][i]), 32 + i, k, v, cos, sin)
        ref = torch.from_numpy(g["sampled"][i])
        assert (o["logits"][idx] - ref).abs().max().item() < 2e-4
        assert o["token"] == int(g["argmax"][i])


def test_golden_config1_restatement():
    g = np.load(os.path.join(GOLDEN, "config1.npz"))
    w1 = W.make_weights(0, n_layers=1, perturb_norms=True)
    assert abs(w1.checksum() - float(g["checksum"])) < 1e-6
    c1 = C.config1_inputs(0)
    pos = c1["position"]
    k = torch.zeros(1, 8, 512, 128)
    v = torch.zeros_like(k)
    k[0, :, :pos] = c1["k_prefix"].float()
    v[0, :, :pos] = c1["v_prefix"].float()
    cos, sin = W.rope_tables(512)
    o = R.decode_layer(w1.layers[0], c1["hidden"].float(), 0, pos, pos + 1, k, v, cos, sin)
    assert (o["r_out"] - torch.from_numpy(g["out"])).abs().max().item() < 1e-4
    assert (o["k_rot"] - torch.from_numpy(g["k_new"])).abs().max().item() < 1e-5
    assert (o["v"].view(8, 128) - torch.from_numpy(g["v_new"])).abs().max().item() < 1e-5


def test_golden_config2_restatement(full_weights):
    g = np.load(os.path.join(GOLDEN, "config2.npz"))
    x = C.config2_hidden(0)
    logits = full_weights.embed.float() @ x.float()
    idx = torch.from_numpy(g["sample_idx"])
    assert (logits[idx].double() - torch.from_numpy(g["sampled"])).abs().max().item() < 1e-4
    assert int(torch.argmax(logits)) == int(g["argmax"])


def test_bf16_cache_semantics_stay_within_baseline_tolerance(full_weights):
    """The kernel's numerics (BF16 cache, FP32 activations) vs HF FP32: the
    BASELINE tolerance (max-abs 2e-2, cosine > 0.999) holds on the oracle side."""
    model = H.build_model(full_weights, threads=os.cpu_count())
    ids = C.config0_prompt(0)
    logits, cache = H.prefill(model, ids)
    k, v = H.to_kernel_cache(cache, 28, 64, torch.bfloat16)
    cos, sin = W.rope_tables(64)
    tok = int(torch.argmax(logits))
    for i in range(2):
        o = R.decode_step(full_weights, tok, 32 + i, k, v, cos, sin)
        hl, cache = H.step(model, cache, tok)
        d = (o["logits"] - hl).abs().max().item()
        cs = torch.nn.functional.cosine_similarity(o["logits"].double(), hl.double(), dim=0).item()
        assert d < 2e-2 and cs > 0.999
        tok = int(torch.argmax(hl))
