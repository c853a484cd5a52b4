"""Generate the golden fixtures from Hugging Face Qwen3 in FP32 on the CPU.

Run from the repository root (takes ~1 minute on 8 cores):

    python tests/golden/make_golden.py

Writes ``tests/golden/config{0,1,2}.npz``. The model is transformers 5.5.0's
``Qwen3ForCausalLM`` (the reference's model path, ``model.py:24-27,72-73,
163-167``) holding the seeded synthetic weights of ``oracle.weights``; the
fixtures pin the CPU restatement (``oracle.restatement``) and the GPU kernel.

config0: 32-token prompt (seed 0), HF prefill, 128 HF greedy steps. Per step:
the token fed, the argmax, the top-2 margin, the top-8 ids/values and the
logits at 512 fixed indices.
config1: one decoder layer (layer 0, perturbed norms so a misapplied norm vector
shows) at position 511 over a seeded N(0,1) BF16 cache prefix: the layer
output, the attention block output and the new K/V.
config2: the isolated LM head, logits = E @ x in float64 for a seeded BF16 x.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from oracle import configs as C  # noqa: E402
from oracle import hf_reference as H  # noqa: E402
from oracle import weights as W  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))


def versions():
    import transformers
    return np.array([transformers.__version__, torch.__version__, np.__version__])


def config0(w):
    model = H.build_model(w, threads=os.cpu_count())
    ids = C.config0_prompt(0)
    idx = C.sample_indices()
    steps = C.CONFIG0["steps"]
    rec = {"argmax": [], "margin": [], "top_ids": [], "top_vals": [], "sampled": [], "maxabs": []}

    def keep(_i, logits):
        l64 = logits.double()
        t = torch.topk(l64, 8)
        rec["argmax"].append(int(torch.argmax(logits)))
        rec["margin"].append(float(t.values[0] - t.values[1]))
        rec["top_ids"].append(t.indices.numpy())
        rec["top_vals"].append(t.values.numpy())
        rec["sampled"].append(logits[idx].numpy())
        rec["maxabs"].append(float(logits.abs().max()))
        return None

    pre_logits, _ = H.prefill(model, ids)
    fed, _ = H.greedy_decode(model, ids, steps, keep_logits=keep)
    np.savez_compressed(
        os.path.join(OUT, "config0.npz"), versions=versions(), checksum=np.float64(w.checksum()),
        prompt=ids.numpy(), fed=np.array(fed, dtype=np.int64), sample_idx=idx,
        prefill_argmax=np.int64(int(torch.argmax(pre_logits))),
        argmax=np.array(rec["argmax"], dtype=np.int64), margin=np.array(rec["margin"]),
        top_ids=np.stack(rec["top_ids"]), top_vals=np.stack(rec["top_vals"]),
        sampled=np.stack(rec["sampled"]).astype(np.float32), maxabs=np.array(rec["maxabs"]))
    return model


def config1():
    w1 = W.make_weights(0, n_layers=1, perturb_norms=True)
    model = H.build_model(w1, threads=os.cpu_count())
    c1 = C.config1_inputs(0)
    o = H.single_layer(model, 0, c1["hidden"], c1["k_prefix"], c1["v_prefix"], c1["position"])
    np.savez_compressed(
        os.path.join(OUT, "config1.npz"), versions=versions(), checksum=np.float64(w1.checksum()),
        out=o["out"].numpy(), attn_o=o["attn_o"].numpy(), k_new=o["k_new"].numpy(),
        v_new=o["v_new"].numpy(), hidden=c1["hidden"].float().numpy())


def config2(w):
    x = C.config2_hidden(0)
    logits = w.embed.double() @ x.double()
    idx = C.sample_indices()
    t = torch.topk(logits, 8)
    np.savez_compressed(
        os.path.join(OUT, "config2.npz"), versions=versions(), checksum=np.float64(w.checksum()),
        sample_idx=idx, sampled=logits[idx].numpy(), argmax=np.int64(int(torch.argmax(logits))),
        margin=np.float64(t.values[0] - t.values[1]), top_ids=t.indices.numpy(),
        top_vals=t.values.numpy(), checksum_logits=np.float64(logits.sum()))


if __name__ == "__main__":
    torch.manual_seed(0)
    weights = W.make_weights(0)
    config2(weights)
    config1()
    config0(weights)
    print("wrote", sorted(f for f in os.listdir(OUT) if f.endswith(".npz")))
