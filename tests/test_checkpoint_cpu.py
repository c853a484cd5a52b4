"""Checkpoint loading (safetensors -> LayerWeights order, model.py:24-44), on the CPU.

The real Qwen3-0.6B checkpoint is not available here, so the files are written by
the tests: once by Hugging Face's own ``save_pretrained`` (its tensor names and
tied-embedding convention) and once by ``save_qwen3``, from the seeded synthetic
weights of the oracle, with two decoder layers to keep the files small."""
import os

import pytest
import torch

from megakernel_b200.checkpoint import LAYER_FIELDS, load_qwen3, save_qwen3
from oracle import weights as W

KEYS = ["input_norm", "q", "k", "v", "q_norm", "k_norm", "o", "post_norm", "gate", "up", "down"]


@pytest.fixture(scope="module")
def w2():
    return W.make_weights(0, n_layers=2)


def _check(got, w):
    assert got.n_layers == w.n_layers
    assert torch.equal(got.embed, w.embed)
    assert torch.equal(got.final_norm, w.final_norm)
    assert len(got.layer_weights) == 11 * w.n_layers
    for i, lw in enumerate(w.layers):
        for j, k in enumerate(KEYS):
            t = got.layer_weights[11 * i + j]
            assert t.dtype == torch.bfloat16 and t.is_contiguous()
            assert torch.equal(t, lw[k]), (i, k)


def test_roundtrip_through_save_qwen3(tmp_path, w2):
    p = os.path.join(tmp_path, "model.safetensors")
    save_qwen3(p, w2.embed, w2.final_norm, w2.flat_layer_list())
    got = load_qwen3(str(tmp_path), device="cpu")
    _check(got, w2)
    assert got.tied and got.lm_head is got.embed


def test_hugging_face_save_pretrained_layout(tmp_path, w2):
    """A directory written by transformers' save_pretrained (BF16, tied head)."""
    from oracle import hf_reference as H
    model = H.build_model(w2).to(torch.bfloat16)
    model.save_pretrained(str(tmp_path), safe_serialization=True)
    got = load_qwen3(str(tmp_path), device="cpu")
    _check(got, w2)
    assert got.config.get("num_hidden_layers") == 2


def test_missing_or_misshaped_tensor_is_refused(tmp_path, w2):
    layers = w2.flat_layer_list()
    bad = list(layers)
    bad[1] = layers[1][:1024]  # q_proj with the wrong row count
    p = os.path.join(tmp_path, "model.safetensors")
    save_qwen3(p, w2.embed, w2.final_norm, bad)
    with pytest.raises(ValueError, match="q_proj"):
        load_qwen3(p, device="cpu")
    assert [f for f, _ in LAYER_FIELDS][1] == "self_attn.q_proj.weight"
