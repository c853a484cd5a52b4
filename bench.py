#!/usr/bin/env python
"""Batch-one Qwen3-0.6B decode benchmark on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl mkb|reference] [--config 0|2|3]

One step = one greedy decode token (batch 1) of the 28-layer Qwen3-0.6B
architecture with random-init BF16 weights (synthetic data), max cache 512, a
32-token prompt, positions 32.. (config 0). Prints ONE JSON line on rank 0.

``--config 2``: one step = one launch of the isolated LM head + argmax
(151936 x 1024 BF16 weight, hidden N(0,1) taken as normalised).
``--config 3``: config 0 with a 4096-slot cache, the 3584-token prompt prefilled
in-engine, 256 greedy steps at positions 3584.. (cache lengths 3585..3840).

* value: tokens/s of the on-device greedy loop (DecodeEngine.generate: one
  persistent launch decodes the K tokens, argmax feeding the next embedding),
  device-timed with CUDA events on the launching stream; with N GPUs each rank
  runs its own replica (prompt seed = rank) and value = all tokens / max time.
* e2e: the same metric through the public per-token call (mkb_engine_step):
  every step copies (token, position) host->device from pinned memory, replays
  the CUDA graph, and the kernel's last CTA stores the argmax id into the
  engine's pinned (mapped) host memory, which the host reads after the sync.
* roofline: decode_kernel's algorithmic bytes (every weight byte once per token
  + KV bytes read) / its measured launch duration, against the measured HBM peak.
* cpu_baseline: HF Qwen3 FP32 decode on this host's cores (oracle), rank 0, N=1.
* tp (N > 1): the same greedy loop with the model split over the N GPUs
  (tensor parallel: KV heads, SwiGLU rows and vocabulary rows per rank, the two
  hidden-state all-reduces per layer and the argmax inside the kernel over NVLink),
  one stream: per-token latency, device-timed, max over ranks.

``--impl reference`` times the reference's model path on the host CPU (HF
Qwen3ForCausalLM FP32, the comparison decode of model.py:139-180) for the same
config/metric, and, when ``oracle/_ref`` holds the reference CUDA kernel built
from its own sources, its per-token time on this GPU as an extra field.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

HIDDEN, INTER, VOCAB, LAYERS = 1024, 3072, 151936, 28
PROMPT, MAX_SEQ = 32, 512
WEIGHT_BYTES = LAYERS * (31_457_280 + 4_608) + 311_164_928 + 2_048 + 2_048   # 1,192,101,888
KV_BYTES_PER_POS = LAYERS * 8 * 128 * 2 * 2                                   # 114,688
LM_BYTES = 311_164_928 + HIDDEN * 4                                           # LM head weight + FP32 hidden
METRIC = "batch-1 decode tok/s (Qwen3-0.6B, 512-token cache)"


def args_parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["mkb", "reference"], default="mkb")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--config", type=int, choices=[0, 2, 3], default=0)
    ap.add_argument("--prefill", action="store_true", help="time the batched prefill (32 and 3584 tokens)")
    ap.add_argument("--prefill-once", type=int, default=0, metavar="N",
                    help="two batched prefills of N tokens and nothing else (for a profiler's launch list)")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


def max_over_ranks(values, world: int, device=None):
    """Element-wise maximum of per-rank timings (one collective on every rank;
    a no-op for one process). Returns plain floats on every rank."""
    t = torch.tensor([float(v) for v in values], dtype=torch.float64, device=device)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return [float(x) for x in t.tolist()]


def replica_throughput(world: int, steps: int, ms: float) -> float:
    """Whole-job tokens/s of `world` independent replicas that each decoded `steps`
    tokens, timed by the slowest rank (`ms`)."""
    return world * steps / (ms / 1000.0)


def end_to_end(eng, first: int, pos0: int, steps: int, warm: int, span: int):
    """Host wall-clock seconds for `steps` greedy tokens through the two public
    per-token surfaces, from token `first` at position `pos0`:

    - a serve session (mkb_engine_serve_open / _step / _close): one persistent
      launch; per token the host writes {seq, token} (8 B) into pinned mapped
      memory and reads {seq, argmax} (8 B) back; open and close are timed;
    - mkb_engine_step: 8 B copied in, one graph replay, the kernel stores the
      4 B argmax into pinned host memory.

    A session covers at most `span` positions; longer runs are timed over
    `span` tokens and scaled. Returns (serve_s, step_s)."""
    n_serve = min(steps, span)
    eng.serve_open(pos0, warm)
    t = first
    for _ in range(warm):
        t = eng.serve_step(t)
    eng.serve_close()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    eng.serve_open(pos0, n_serve)
    t = first
    for _ in range(n_serve):
        t = eng.serve_step(t)
    eng.serve_close()
    serve_s = (time.perf_counter() - t0) * steps / n_serve
    assert eng.status()[0] == 0, f"in-kernel error {eng.status()}"
    for i in range(warm):
        eng.step(first, pos0 + i)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    t = first
    for i in range(steps):
        t = eng.step(t, pos0 + (i % span))
    torch.cuda.synchronize()
    return serve_s, time.perf_counter() - t0


def e2e_fields(world: int, steps: int, serve_ms: float, step_ms: float) -> dict:
    """The bench line's `e2e` object: the serve session as the headline, the
    per-call mkb_engine_step beside it."""
    return {"value": replica_throughput(world, steps, serve_ms), "unit": "tok/s", "h2d_bytes_per_step": 8,
            "d2h_bytes_per_step": 8, "us_per_token": serve_ms * 1000.0 / steps,
            "api": "serve session (mkb_engine_serve_open / _step / _close): one persistent launch; per step the "
                   "host writes {seq, token} (8 B) into pinned mapped memory and reads {seq, argmax} (8 B) back; "
                   "open and close inside the timed region",
            "per_call_step": {"value": replica_throughput(world, steps, step_ms), "unit": "tok/s",
                              "us_per_token": step_ms * 1000.0 / steps, "h2d_bytes_per_step": 8,
                              "d2h_bytes_per_step": 4,
                              "api": "mkb_engine_step (8 B copied in from pinned memory, graph replay, the "
                                     "kernel stores the 4 B argmax into pinned host memory)"}}


def synthetic_weights(seed: int, device):
    """Random-init Qwen3-0.6B weights generated on the device (N(0, 0.02), norms 1)."""
    g = torch.Generator(device=device).manual_seed(seed)

    def lin(*shape):
        return (torch.randn(shape, generator=g, device=device, dtype=torch.float32) * 0.02).to(torch.bfloat16)

    ones = lambda n: torch.ones(n, dtype=torch.bfloat16, device=device)  # noqa: E731
    embed = lin(VOCAB, HIDDEN)
    layers = []
    for _ in range(LAYERS):
        layers += [ones(HIDDEN), lin(2048, HIDDEN), lin(1024, HIDDEN), lin(1024, HIDDEN), ones(128), ones(128),
                   lin(HIDDEN, 2048), ones(HIDDEN), lin(INTER, HIDDEN), lin(INTER, HIDDEN), lin(HIDDEN, INTER)]
    return embed, ones(HIDDEN), layers


class ClockSampler:
    """SM clock, power and clock-event reasons sampled every 5 ms (NVML, read only)
    while the timed region runs; falls back to nvidia-smi at 200 ms without NVML."""

    def __init__(self, index: int):
        self.index = index
        self.samples = []   # (sm_mhz, max_mhz, power_w, reasons)
        self.stop = threading.Event()
        self.thread = None
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            names = {pynvml.nvmlClocksEventReasonHwSlowdown: "hw_slowdown",
                     pynvml.nvmlClocksEventReasonHwThermalSlowdown: "hw_thermal_slowdown",
                     pynvml.nvmlClocksEventReasonSwThermalSlowdown: "sw_thermal_slowdown",
                     pynvml.nvmlClocksEventReasonSwPowerCap: "sw_power_cap"}
            mx = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)

            def run():
                while not self.stop.is_set():
                    try:
                        sm = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                        pw = pynvml.nvmlDeviceGetPowerUsage(h) / 1000.0
                        bits = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                        self.samples.append((sm, mx, pw, [n for b, n in names.items() if bits & b]))
                    except Exception:
                        pass
                    time.sleep(0.005)

            self.thread = threading.Thread(target=run, daemon=True)
            self.thread.start()
            return self
        except Exception:
            pass
        try:
            fields = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                      "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                      "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={fields}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.proc.stdout:
            p = [x.strip() for x in line.split(",")]
            if len(p) < 9:
                continue
            try:
                self.samples.append((float(p[1]), float(p[2]), float(p[3]),
                                     [n for n, v in zip(names, p[5:9]) if v.lower() == "active"]))
            except ValueError:
                continue

    def __exit__(self, *exc):
        self.stop.set()
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=2)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        reasons = sorted({r for s in self.samples for r in s[3]})
        return {"sm_mhz": statistics.median(s[0] for s in self.samples),
                "sm_max_mhz": max(s[1] for s in self.samples),
                "power_w_max": max(s[2] for s in self.samples), "reasons": reasons, "samples": len(self.samples)}


def measured_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def ncu_traffic():
    """DRAM bytes of one decode_kernel token from the committed ncu capture:
    (bytes at the captured cache length, that length, KV bytes per extra position)."""
    try:
        with open(os.path.join(ROOT, "profiles", "decode_kernel_traffic.json")) as f:
            d = json.load(f)
        return float(d["dram_bytes_per_token"]), int(d["cache_len"]), float(d["kv_bytes_per_position"])
    except Exception:
        return None


def cpu_baseline(steps_cap: int = 128, budget_s: float = 12.0):
    """HF Qwen3 FP32 decode on the host CPU (the oracle), bounded sample."""
    from oracle import configs as C
    from oracle import hf_reference as H
    from oracle import weights as W
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    w = W.make_weights(0)
    model = H.build_model(w, threads=threads)
    ids = C.config0_prompt(0)
    logits, cache = H.prefill(model, ids)
    tok = int(torch.argmax(logits))
    n, t0 = 0, time.perf_counter()
    while n < steps_cap:
        logits, cache = H.step(model, cache, tok)
        tok = int(torch.argmax(logits))
        n += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = time.perf_counter() - t0
    cpu = "unknown"
    try:
        for ln in open("/proc/cpuinfo"):
            if ln.startswith("model name"):
                cpu = ln.split(":", 1)[1].strip()
                break
    except Exception:
        pass
    return {"value": n / dt, "unit": "tok/s", "cores": threads, "kind": "reference",
            "sample": f"HF transformers Qwen3ForCausalLM FP32 eager, {n} greedy decode steps at positions "
                      f"32..{31 + n} after a 32-token prefill, {threads} threads, {cpu}"}


def run_reference(a, rank, world):
    if rank != 0:
        return
    if a.config != 0:
        print(json.dumps({"impl": "reference", "unavailable": "the reference arm is measured on config 0 only "
                          "(its CPU model path takes minutes per step at these sizes)"}), flush=True)
        return
    base = cpu_baseline(steps_cap=max(a.steps, 1), budget_s=60.0)
    line = {"impl": "reference", "metric": METRIC, "value": base["value"], "unit": "tok/s", "n_gpus": a.gpus,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": 1000.0 / base["value"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (random-init weights, random prompt ids)",
            "config": {"workload": "config0: Qwen3-0.6B batch-1 greedy decode, 32-token prompt, cache 512",
                       "model": "Qwen3-0.6B", "global_batch": 1, "seq_len": MAX_SEQ, "parallelism": "none (CPU)"},
            "cpu_baseline": base,
            "e2e": {"value": base["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    ref_gpu = reference_kernel_on_gpu(a)
    if ref_gpu is not None:
        line["reference_cuda_kernel_b200"] = ref_gpu
    print(json.dumps(line), flush=True)


def timed_region(local, fn):
    """Run fn() between CUDA events on the current stream with clocks sampled;
    returns (device ms, clock summary)."""
    stream = torch.cuda.current_stream()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        ev0.record(stream)
        out = fn()
        ev1.record(stream)
        torch.cuda.synchronize()
    return ev0.elapsed_time(ev1), clk.summary(), out


def profile_traffic(name):
    """DRAM bytes per launch of a committed ncu capture (profiles/<name>.json)."""
    try:
        with open(os.path.join(ROOT, "profiles", name)) as f:
            return json.load(f)
    except Exception:
        return None


def run_config2(a, rank, world, local):
    """Isolated LM head + argmax, one launch per step."""
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    import megakernel_b200 as mk
    from megakernel_b200 import _lib
    from megakernel_b200.engine import build_layer_table, decode_call
    g = torch.Generator(device=dev).manual_seed(2001 + rank)
    embed = (torch.randn((VOCAB, HIDDEN), generator=g, device=dev) * 0.02).to(torch.bfloat16)
    x = torch.randn(HIDDEN, generator=g, device=dev).to(torch.bfloat16).float()
    norm = torch.ones(HIDDEN, dtype=torch.bfloat16, device=dev)
    layer = [norm, embed[:2048], embed[:1024], embed[:1024], norm[:128], norm[:128], embed[:1024, :1024].contiguous(),
             norm, embed[:3072], embed[:3072], embed[:1024, :1024].contiguous()]
    table = build_layer_table(layer, dev)
    kv = torch.zeros((1, 8, 16, 128), dtype=torch.bfloat16, device=dev)
    cos, sin = mk.rope_tables(16, dev)
    logits = torch.empty(VOCAB, dtype=torch.float32, device=dev)
    tok = torch.empty(max(a.steps, 1), dtype=torch.int32, device=dev)
    common = dict(embed=embed, lm_head=embed, final_norm=norm, layers=table, cos_table=cos, sin_table=sin,
                  rope_fp32=1, k_cache=kv, v_cache=kv, max_seq=16, layer_begin=0, layer_end=0, token=0,
                  position=0, cache_len=1, flags=_lib.MKB_FLAG_LM_HEAD | _lib.MKB_FLAG_SKIP_FINAL_NORM,
                  logits=logits)
    steps, warm = max(1, a.steps), max(3, a.warmup)

    def launches(n):
        for i in range(n):
            _lib.check(decode_call(input_residual=x, out_tokens=tok[i:i + 1], **common), "mkb_decode")

    launches(warm)
    dev_ms, clocks, _ = timed_region(local, lambda: launches(steps))
    # steady-state stream: one launch that runs the LM head `steps` times over the same input
    n_pass = min(steps, 16 - 1)
    pass_ms, _, _ = timed_region(local, lambda: _lib.check(decode_call(
        input_residual=x, out_tokens=tok, n_tokens=n_pass, **{**common, "max_seq": 16}), "mkb_decode"))
    # e2e: hidden copied in from pinned memory, argmax copied back, per step
    xh = x.cpu().pin_memory()
    th = torch.empty(1, dtype=torch.int32).pin_memory()
    xd = torch.empty_like(x)
    stream = torch.cuda.current_stream()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for i in range(steps):
        xd.copy_(xh, non_blocking=True)
        _lib.check(decode_call(input_residual=xd, out_tokens=tok[:1], **common), "mkb_decode")
        th.copy_(tok[:1], non_blocking=True)
        stream.synchronize()
    e2e_s = time.perf_counter() - t0
    assert int(th.item()) == int(torch.argmax(embed.float() @ x).item())
    dev_ms, e2e_ms, pass_ms = max_over_ranks([dev_ms, e2e_s * 1000.0, pass_ms], world, dev)
    per_launch = LM_BYTES
    achieved = per_launch / (dev_ms / 1000.0 / steps) / 1e9
    peak, peak_kind = measured_peak()
    tr = profile_traffic("lm_head_traffic.json")
    if rank == 0:
        line = {"metric": "isolated LM-head GEMV + argmax launches/s (151936 x 1024 BF16)",
                "value": world * steps / (dev_ms / 1000.0), "unit": "launch/s", "n_gpus": world, "steps": steps,
                "warmup": warm, "ms_per_step": dev_ms / steps, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic (E ~ N(0,0.02) BF16, hidden ~ N(0,1) BF16 taken as normalised)",
                "config": {"workload": "config2: isolated LM head + argmax, 311 MB weight per launch",
                           "us_per_launch": dev_ms * 1000.0 / steps,
                           "us_per_pass_in_one_launch": pass_ms * 1000.0 / n_pass,
                           "l2": "inputs larger than L2: 311 MB weight per launch vs 126 MB L2"},
                "e2e": {"value": world * steps / (e2e_ms / 1000.0), "unit": "launch/s",
                        "h2d_bytes_per_step": HIDDEN * 4, "d2h_bytes_per_step": 4,
                        "us_per_launch": e2e_ms * 1000.0 / steps,
                        "api": "mkb_decode (hidden copied in, argmax copied out, stream synchronised per step)"},
                "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                             "frac": achieved / peak, "peak_source": peak_kind,
                             "traffic": tr["dram_bytes_per_launch"] if tr else None, "kernel": "decode_kernel",
                             "algorithmic_bytes_per_launch": per_launch,
                             "stream_frac_in_one_launch": per_launch / (pass_ms / 1000.0 / n_pass) / 1e9 / peak},
                "gpu_launches": steps, "clocks": clocks}
        print(json.dumps(line), flush=True)


LINEAR_PARAMS = LAYERS * (4096 * 1024 + 1024 * 2048 + 2 * 3072 * 1024 + 1024 * 3072)   # 440,401,920


def prefill_flops(n: int, pos0: int = 0) -> float:
    """Model FLOPs of a prefill of n tokens at positions pos0..: 2 per weight per
    token for the projections, 4 * 128 per (query, key) pair per head for QK^T
    and PV (causal), 2 per LM-head weight for the last token."""
    keys = n * pos0 + n * (n + 1) // 2
    return 2.0 * LINEAR_PARAMS * n + LAYERS * 16 * 512.0 * keys + 2.0 * 311_164_928 / 2


def prefill_once(n: int, local: int):
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    import megakernel_b200 as mk
    embed, final_norm, layers = synthetic_weights(1000, dev)
    k = torch.zeros((LAYERS, 8, 4096, 128), dtype=torch.bfloat16, device=dev)
    v = torch.zeros_like(k)
    eng = mk.DecodeEngine(embed, final_norm, layers, k, v)
    ids = torch.randint(0, VOCAB, (n,), generator=torch.Generator().manual_seed(1))
    for _ in range(2):
        eng.prefill(ids, batched=True)
    torch.cuda.synchronize()
    eng.close()


def run_prefill(a, rank, world, local):
    """Batched prefill (tcgen05 GEMMs, tensor-core attention) of a 32- and a
    3584-token prompt, against the token-by-token in-engine prefill."""
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    import megakernel_b200 as mk
    from ctypes import c_void_p
    from megakernel_b200 import _lib
    embed, final_norm, layers = synthetic_weights(1000, dev)
    k = torch.zeros((LAYERS, 8, 4096, 128), dtype=torch.bfloat16, device=dev)
    v = torch.zeros_like(k)
    eng = mk.DecodeEngine(embed, final_norm, layers, k, v, fused_down=True, use_graph=True)
    lib = _lib.load()
    nxt = torch.empty(1, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream()
    res = {}
    for n in (32, 3584):
        ids = torch.randint(0, VOCAB, (n,), generator=torch.Generator().manual_seed(n)).to(torch.int32).to(dev)

        def batched():
            _lib.check(lib.mkb_engine_prefill_batched(eng._h, c_void_p(ids.data_ptr()), n, 0, c_void_p(nxt.data_ptr()),
                                                      c_void_p(stream.cuda_stream)), "prefill_batched")

        def stepwise():
            _lib.check(lib.mkb_engine_prefill(eng._h, c_void_p(ids.data_ptr()), n, 0, c_void_p(nxt.data_ptr()),
                                              c_void_p(stream.cuda_stream)), "prefill")

        for _ in range(max(3, a.warmup)):
            batched()
        reps = 5 if n > 1000 else 20
        ms, clocks, _ = timed_region(local, lambda: [batched() for _ in range(reps)])
        ms /= reps
        st_ms, _, _ = timed_region(local, stepwise)
        assert eng.status()[0] == 0
        res[n] = {"ms": ms, "token_by_token_ms": st_ms, "clocks": clocks}
    peak, _ = measured_peak()
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            tf_peak, tf_kind = float(json.load(f)["bf16_tflops"]), "measured"
    except Exception:
        tf_peak, tf_kind = 1590.0, "fallback"
    n = 3584
    fl = prefill_flops(n)
    achieved = fl / (res[n]["ms"] / 1000.0) / 1e12
    if rank == 0:
        line = {"metric": "batched prefill tok/s (Qwen3-0.6B, 3584-token prompt)", "value": n / (res[n]["ms"] / 1000.0),
                "unit": "tok/s", "n_gpus": 1, "steps": 5, "warmup": max(3, a.warmup), "ms_per_step": res[n]["ms"],
                "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic (random-init BF16 weights N(0,0.02), random prompt ids)",
                "config": {"workload": "prefill of a 3584-token prompt into a 4096-slot cache (config 3's prompt), "
                                       "and of a 32-token prompt (config 0's)",
                           "ms_3584": res[n]["ms"], "token_by_token_ms_3584": res[n]["token_by_token_ms"],
                           "speedup_vs_token_by_token_3584": res[n]["token_by_token_ms"] / res[n]["ms"],
                           "ms_32": res[32]["ms"], "token_by_token_ms_32": res[32]["token_by_token_ms"]},
                "roofline": {"bound": "tensor", "achieved": achieved, "peak": tf_peak, "unit": "TFLOP/s",
                             "frac": achieved / tf_peak, "peak_source": tf_kind,
                             "flops_per_prefill": fl,
                             "note": "model FLOPs; the GEMMs run each activation as two BF16 parts, "
                                     "so the tensor cores execute about twice these FLOPs"},
                "gpu_launches": 28 * 7 + 2, "clocks": res[n]["clocks"]}
        print(json.dumps(line), flush=True)
    eng.close()


def run_config3(a, rank, world, local):
    """Long cache: 4096-slot cache, 3584-token prompt
    prefilled in-engine, 256 greedy steps in one persistent launch."""
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    import megakernel_b200 as mk
    prompt_len, max_seq = 3584, 4096
    steps = max(1, min(a.steps, max_seq - prompt_len))
    warm = max(3, a.warmup)
    embed, final_norm, layers = synthetic_weights(1000 + rank, dev)
    k = torch.zeros((LAYERS, 8, max_seq, 128), dtype=torch.bfloat16, device=dev)
    v = torch.zeros_like(k)
    eng = mk.DecodeEngine(embed, final_norm, layers, k, v, fused_down=True, use_graph=True)
    prompt = torch.randint(0, VOCAB, (prompt_len,), generator=torch.Generator().manual_seed(rank)).tolist()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    first = eng.prefill(prompt, batched=True)
    prefill_s = time.perf_counter() - t0
    out = torch.empty(steps, dtype=torch.int32, device=dev)
    eng.generate(first, prompt_len, warm, out=out[:warm])
    dev_ms, clocks, _ = timed_region(local, lambda: eng.generate(first, prompt_len, steps, out=out))
    assert eng.status()[0] == 0
    serve_s, step_s = end_to_end(eng, first, prompt_len, steps, warm, max_seq - prompt_len)
    dev_ms, serve_ms, step_ms = max_over_ranks([dev_ms, serve_s * 1000.0, step_s * 1000.0], world, dev)
    alg = sum(WEIGHT_BYTES + KV_BYTES_PER_POS * (prompt_len + i + 1) for i in range(steps))
    achieved = alg / (dev_ms / 1000.0) / 1e9
    peak, peak_kind = measured_peak()
    tr = ncu_traffic()
    traffic = None
    if tr is not None:
        tok_bytes, cl0, per_pos = tr
        traffic = sum(tok_bytes + per_pos * (prompt_len + i + 1 - cl0) for i in range(steps))
    line = {"metric": METRIC.replace("512", "4096"), "value": replica_throughput(world, steps, dev_ms),
            "unit": "tok/s", "n_gpus": world, "steps": steps, "warmup": warm, "ms_per_step": dev_ms / steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (random-init BF16 weights N(0,0.02), random prompt ids)",
            "config": {"workload": "config3: Qwen3-0.6B batch-1 greedy decode, 3584-token prompt, cache 4096, "
                                   "cache lengths 3585..3840", "model": "Qwen3-0.6B", "global_batch": world,
                       "seq_len": max_seq, "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                       "l2": "inputs larger than L2: 1.6 GB streamed per token vs 126 MB L2",
                       "us_per_token": dev_ms * 1000.0 / steps, "batched_prefill_s_3584_tokens": prefill_s,
                       "kv_share_of_bytes": sum(KV_BYTES_PER_POS * (prompt_len + i + 1) for i in range(steps)) / alg},
            "e2e": e2e_fields(world, steps, serve_ms, step_ms),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                         "peak_source": peak_kind, "traffic": traffic, "kernel": "decode_kernel",
                         "algorithmic_bytes_per_launch": alg},
            "gpu_launches": 1, "clocks": clocks}
    if rank == 0:
        print(json.dumps(line), flush=True)
    eng.close()


def reference_kernel_on_gpu(a):
    """The reference's own megakernel (built from its sources into oracle/_ref),
    timed per call on this GPU the way model.py:107-127 times it (its binding's
    per-call table allocation and cudaFree included)."""
    if not torch.cuda.is_available():
        return None
    try:
        from oracle import ref_kernel
        out = ref_kernel.time_reference(steps=min(a.steps, 64), warmup=a.warmup)
        # the same kernel without its binding's per-call allocation: table and
        # scratch resident, events around the launch only
        out["resident"] = ref_kernel.time_reference_resident(steps=min(a.steps, 64), warmup=a.warmup)
        return out
    except Exception as e:  # the reference kernel is optional context, never the product
        return {"unavailable": f"{type(e).__name__}: {e}"[:200]}


def main():
    a = args_parse()
    rank, world, local = dist_env()
    if a.impl == "reference":
        run_reference(a, rank, world)
        return
    if a.prefill_once:
        prefill_once(a.prefill_once, local)
        return
    if a.prefill:
        run_prefill(a, rank, world, local)
        return
    if a.config == 2:
        run_config2(a, rank, world, local)
        return
    if a.config == 3:
        run_config3(a, rank, world, local)
        return
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    import megakernel_b200 as mk

    # the same weights on every rank (the tensor-parallel run below shares them);
    # the replicas are independent streams through their own prompts
    embed, final_norm, layers = synthetic_weights(1000, dev)
    k = torch.zeros((LAYERS, 8, MAX_SEQ, 128), dtype=torch.bfloat16, device=dev)
    v = torch.zeros_like(k)
    eng = mk.DecodeEngine(embed, final_norm, layers, k, v, fused_down=True, use_graph=True)
    g = torch.Generator().manual_seed(rank)
    prompt = torch.randint(0, VOCAB, (PROMPT,), generator=g).tolist()
    # in-engine prefill of the prompt (positions 0..31, one launch)
    first = eng.prefill(prompt)
    span = MAX_SEQ - PROMPT
    steps, warm = max(1, a.steps), max(3, a.warmup)

    def greedy(n_tok):
        """n_tok greedy tokens in launches of <= span tokens from position 32; returns launches."""
        done, launches = 0, 0
        out = torch.empty(span, dtype=torch.int32, device=dev)
        while done < n_tok:
            n = min(span, n_tok - done)
            eng.generate(first, PROMPT, n, out=out)
            done += n
            launches += 1
        return launches

    greedy(warm)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        ev0.record(stream)
        launches = greedy(steps)
        ev1.record(stream)
        torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    dev_ms = ev0.elapsed_time(ev1)
    st = eng.status()
    assert st[0] == 0, f"in-kernel error {st}"

    serve_s, step_s = end_to_end(eng, first, PROMPT, steps, warm, span)
    dev_ms, serve_ms, step_ms = max_over_ranks([dev_ms, serve_s * 1000.0, step_s * 1000.0], world, dev)

    # algorithmic bytes of the timed launches (positions 32.. wrap every `span` tokens)
    alg = 0
    for i in range(steps):
        cl = PROMPT + (i % span) + 1
        alg += WEIGHT_BYTES + KV_BYTES_PER_POS * cl
    per_launch_bytes = alg / launches
    per_launch_s = dev_ms / 1000.0 / launches
    peak, peak_kind = measured_peak()
    achieved = per_launch_bytes / per_launch_s / 1e9
    toks_per_launch = steps / launches
    # ncu traffic of one captured token, scaled to this launch's cache lengths
    traffic = None
    tr = ncu_traffic()
    if tr is not None:
        tok_bytes, cl0, per_pos = tr
        traffic = sum(tok_bytes + per_pos * (PROMPT + (i % span) + 1 - cl0) for i in range(steps)) / launches
    if rank == 0:
        line = {
            "metric": METRIC, "value": replica_throughput(world, steps, dev_ms), "unit": "tok/s", "n_gpus": world,
            "steps": steps, "warmup": warm, "ms_per_step": dev_ms / steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic (random-init BF16 weights N(0,0.02), random prompt ids)",
            "config": {"workload": "config0: Qwen3-0.6B batch-1 greedy decode, 32-token prompt, cache 512",
                       "model": "Qwen3-0.6B", "global_batch": world, "seq_len": MAX_SEQ,
                       "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                       "l2": "inputs larger than L2: 1.19 GB of weights streamed per token vs 126 MB L2",
                       "us_per_token": dev_ms * 1000.0 / steps, "tokens_per_launch": toks_per_launch},
            "e2e": e2e_fields(world, steps, serve_ms, step_ms),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_source": peak_kind,
                         "traffic": traffic,
                         "kernel": "decode_kernel", "algorithmic_bytes_per_launch": per_launch_bytes},
            "gpu_launches": launches,
            "clocks": clk.summary(),
        }
        if world == 1 and not a.no_cpu_baseline:
            try:
                line["cpu_baseline"] = cpu_baseline()
            except Exception as e:
                line["cpu_baseline"] = {"unavailable": f"{type(e).__name__}: {e}"[:200]}
    eng.close()
    if world > 1:
        tp = tensor_parallel_run(rank, world, dev, embed, final_norm, layers, steps, warm, local)
        if rank == 0:
            line["tp"] = tp
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def tensor_parallel_run(rank, world, dev, embed, final_norm, layers, steps, warm, local):
    """One decode stream with the model split over `world` GPUs (megakernel_b200.tp):
    32-token prompt prefilled, then `steps` greedy tokens in one launch per rank,
    CUDA events on each rank, max over ranks."""
    import torch.distributed as dist
    from megakernel_b200.tp import TPDecodeEngine
    res, ok = {}, 1.0
    tpe = None
    try:
        h = 8 // world
        ks = torch.zeros((LAYERS, h, MAX_SEQ, 128), dtype=torch.bfloat16, device=dev)
        vs = torch.zeros_like(ks)
        tpe = TPDecodeEngine(embed, final_norm, layers, ks, vs)
        prompt = torch.randint(0, VOCAB, (PROMPT,), generator=torch.Generator().manual_seed(0)).tolist()
        first = tpe.prefill(prompt)
        n = min(steps, MAX_SEQ - PROMPT)
        out = torch.empty(n, dtype=torch.int32, device=dev)
        tpe.generate(first, PROMPT, min(warm, n), out=out[:min(warm, n)])
        torch.cuda.synchronize()
        dist.barrier()
        ms, clocks, _ = timed_region(local, lambda: tpe.generate(first, PROMPT, n, out=out))
        st = tpe.status()
        if st[0] != 0:
            raise RuntimeError(f"in-kernel error {st}")
        res = {"us_per_token": None, "tp_size": world, "tokens": n, "device_ms_local": ms, "clocks": clocks,
               "split": f"KV heads {h}/GPU, SwiGLU rows {3072 // world}/GPU, vocabulary rows {VOCAB // world}/GPU",
               "exchange": "in-kernel over NVLink: o_proj partials added into every GPU's counted accumulators, "
                           "down-projection sums reduced per GPU then forwarded (one CTA per GPU), argmax "
                           "candidates red.max into every GPU; local polling only"}
    except Exception as e:  # reported, never fatal for the replica measurement above
        ok = 0.0
        res = {"unavailable": f"{type(e).__name__}: {e}"[:300]}
    # the collective an NCCL form of the same split would need: an all_reduce of
    # the 4 KB hidden state, twice per layer (56 per token)
    ar_ms = 0.0
    try:
        x = torch.ones(1024, dtype=torch.float32, device=dev)
        for _ in range(10):
            dist.all_reduce(x)
        torch.cuda.synchronize()
        ar_ms, _, _ = timed_region(local, lambda: [dist.all_reduce(x) for _ in range(200)])
        ar_ms /= 200
    except Exception:
        ar_ms = 0.0
    flags = max_over_ranks([1.0 - ok, res.get("device_ms_local", 0.0), ar_ms], world, dev)
    res["nccl_allreduce_4kb_us"] = flags[2] * 1000.0 if flags[2] > 0 else None
    if flags[2] > 0:
        res["nccl_allreduce_per_token_us"] = flags[2] * 1000.0 * 2 * LAYERS
    if flags[0] > 0:
        res = res if "unavailable" in res else {"unavailable": "failed on another rank"}
    else:
        res["us_per_token"] = flags[1] * 1000.0 / res["tokens"]
        res["tok_s"] = res["tokens"] / (flags[1] / 1000.0)
        res["bytes_per_gpu_per_token"] = WEIGHT_BYTES / world
        res.pop("device_ms_local", None)
    if tpe is not None:
        try:
            tpe.close()
        except Exception:
            pass
    return res


if __name__ == "__main__":
    main()
