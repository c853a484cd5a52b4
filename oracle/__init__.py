"""CPU oracle for the batch-one Qwen3-0.6B decode path.

TEST INFRASTRUCTURE ONLY. Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import this
package, and only as the checker or the timed CPU baseline. The product path
(``megakernel_b200``) never imports it and has no CPU fallback.

Contents:

* ``weights``      -- deterministic synthetic Qwen3-0.6B weights (seeded numpy
                      PCG64 normals, rounded to BF16), in the reference's
                      ``LayerWeights`` order (``config.cuh:77-89``).
* ``restatement``  -- a PyTorch-FP32-on-CPU restatement of the reference decode
                      step (``megakernel.cu:744-893``), stage by stage, with the
                      reference's numerics (FP32 activations, BF16 KV cache,
                      caller-supplied RoPE tables).
* ``hf_reference`` -- the BASELINE oracle: Hugging Face ``Qwen3ForCausalLM``
                      (transformers 5.5.0, a third-party dependency that the
                      reference calls from ``model.py:24-27,72-73,163-167``) run
                      in FP32 on CPU with the same weights.

Parity pin: ``tests/golden/make_golden.py`` ran the HF model in this build
container and committed per-step logits samples and greedy tokens;
``tests/test_oracle_cpu.py`` checks the restatement against those fixtures and
against HF itself.
"""
