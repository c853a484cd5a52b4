"""Stage timeline of the decode kernel from its in-kernel ``%globaltimer`` stamps.

With a trace buffer, consumer thread 0 of every CTA stamps each cross-CTA wait
(begin/end), each publish, the sub-stage boundaries and the token start/LM-head
end/token end (codes in ``mkb_decode_args.trace``). Stamps are staged in shared
memory and cover layers 8-15 plus the token-level marks. This module launches
the kernel with such a buffer and reduces the stamps to per-stage wait and
compute times.

    python -m megakernel_b200.trace [--tokens N] [--position P] [--max-seq S] [--reference-layout]

runs config 0 shapes (synthetic weights, a 512-slot cache unless --max-seq says
otherwise) and prints the summary.
"""
from __future__ import annotations

import argparse
import statistics
from collections import defaultdict

import torch

from . import _lib
from .engine import build_layer_table, decode_call
from .rope import rope_tables

STAGE_NAMES = {0: "qkv", 1: "attn+o_proj", 2: "swiglu(+down)", 3: "down", 4: "lm_head",
               5: "split-combine", 6: "token", 7: "end", 8: "qkv:input", 9: "qkv:norm",
               10: "attn:head-prep", 11: "attn:softmax-v", 12: "attn:combine", 13: "swiglu:input+norm",
               14: "swiglu:gate-up", 15: "swiglu:down", 16: "ring-fill", 17: "slot-free", 18: "issue",
               19: "qkv:mma", 20: "qkv:stash+bar", 21: "attn:partials+bar", 22: "o_proj:mma",
               23: "o_proj:stash+bar", 24: "gate-up:mma", 25: "gate-up:stash+bar", 26: "swiglu:silu+send+bar",
               27: "down:own-rows", 28: "down:partner-wait"}
KIND_NAMES = {0: "pre-wait", 1: "wait", 2: "publish", 3: "mark"}


class TracedDecoder:
    """Explicit-argument launches of the decode kernel with a trace buffer."""

    def __init__(self, embed, final_norm, layer_weights, k_cache, v_cache, cos=None, sin=None,
                 fused: bool = True):
        dev = embed.device
        self.dev = dev
        self.embed, self.final_norm, self.k, self.v = embed, final_norm, k_cache, v_cache
        self.layers = list(layer_weights)
        self.n_layers = len(self.layers) // 11
        self.max_seq = int(k_cache.shape[2])
        if cos is None:
            cos, sin = rope_tables(self.max_seq, dev)
        self.cos, self.sin = cos, sin
        self.table = build_layer_table(self.layers, dev)
        self.down_t = None
        self._bufs = []
        if fused:
            lib = _lib.load()
            for li in range(self.n_layers):
                t = torch.empty((3072, 1024), dtype=torch.bfloat16, device=dev)
                _lib.check(lib.mkb_transpose_down(self.layers[li * 11 + 10].data_ptr(), t.data_ptr(), None),
                           "mkb_transpose_down")
                self._bufs.append(t)
            self.down_t = torch.tensor([b.data_ptr() for b in self._bufs], dtype=torch.int64, device=dev)
        self.logits = torch.empty(151936, dtype=torch.float32, device=dev)
        self.out = torch.empty(self.max_seq, dtype=torch.int32, device=dev)
        props = torch.cuda.get_device_properties(dev)
        self.grid = min(props.multi_processor_count, 256)

    def run(self, token: int, position: int, n_tokens: int = 1, cap: int = 2048, traced: bool = True):
        trace = torch.zeros((2 * self.grid, cap), dtype=torch.int64, device=self.dev)
        code = decode_call(embed=self.embed, lm_head=self.embed, final_norm=self.final_norm, layers=self.table,
                           down_t=(self.down_t.data_ptr() if self.down_t is not None else None),
                           cos_table=self.cos, sin_table=self.sin,
                           rope_fp32=1 if self.cos.dtype == torch.float32 else 0, k_cache=self.k,
                           v_cache=self.v, max_seq=self.max_seq, layer_begin=0, layer_end=self.n_layers,
                           token=token, position=position, cache_len=position + 1, n_tokens=n_tokens,
                           flags=_lib.MKB_FLAG_LM_HEAD, logits=self.logits, out_tokens=self.out,
                           grid=self.grid, trace=(trace.data_ptr() if traced else None), trace_cap=cap)
        _lib.check(code, "mkb_decode")
        torch.cuda.synchronize(self.dev)
        if not traced:
            return None
        recs = decode_records(trace.cpu())
        self.producer_records = recs[self.grid:]
        return recs[:self.grid]


def decode_records(trace: torch.Tensor):
    """[grid, cap] int64 -> per CTA list of (kind, stage, layer, token, t_ns)."""
    out = []
    for row in trace.tolist():
        recs = []
        for v in row:
            if v == 0:
                break
            u = v & ((1 << 64) - 1)
            code = u >> 48
            t = u & ((1 << 48) - 1)
            recs.append((code & 3, (code >> 2) & 31, (code >> 7) & 31, (code >> 12) & 15, t))
        out.append(recs)
    return out


def summarize(per_cta) -> dict:
    t0 = min(r[0][4] for r in per_cta if r)
    waits = defaultdict(list)      # stage -> wait durations (ns)
    compute = defaultdict(list)    # stage -> wait end (or previous publish) -> publish (ns)
    token_ns, lm_ns, layer_period = [], [], []
    for recs in per_cta:
        open_wait = {}
        last_ready = None
        a_pub = []
        tok_start = lm_start = None
        for kind, st, layer, tok, t in recs:
            key = (st, layer, tok)
            if kind == 0:
                open_wait[key] = t
            elif kind == 1:
                if key in open_wait:
                    waits[st].append(t - open_wait.pop(key))
                last_ready = t
                if st == 4:
                    lm_start = t
            elif kind == 2:
                if last_ready is not None:
                    compute[st].append(t - last_ready)
                last_ready = t
                if st == 0:
                    a_pub.append(t)
            elif kind == 3:
                if st == 6:
                    tok_start = t
                    last_ready = t
                elif st == 4 and lm_start is not None:
                    lm_ns.append(t - lm_start)
                elif st == 7 and tok_start is not None:
                    token_ns.append(t - tok_start)
        layer_period += [b - a for a, b in zip(a_pub, a_pub[1:])]
    # time between consecutive stamps of a CTA, labelled by the later stamp
    seg = defaultdict(list)
    for recs in per_cta:
        for prev, cur in zip(recs, recs[1:]):
            name = STAGE_NAMES.get(cur[1], f"mark{cur[1]}")
            label = f"{KIND_NAMES[cur[0]]}:{name}" if cur[0] != 3 else name
            seg[label].append(cur[4] - prev[4])
    # exchange latency: last publish of a stage over all CTAs -> each CTA's end of
    # the wait on that stage (DE of layer l feeds A of l+1 and the LM head; BC
    # feeds DE of the same layer)
    last_pub = defaultdict(int)
    for recs in per_cta:
        for kind, st, layer, tok, t in recs:
            if kind == 2 and st in (1, 2):
                last_pub[(st, layer, tok)] = max(last_pub[(st, layer, tok)], t)
    xlat = defaultdict(list)
    for recs in per_cta:
        for kind, st, layer, tok, t in recs:
            if kind != 1:
                continue
            src = (2, layer - 1, tok) if st == 0 else (1, layer, tok) if st == 2 else (2, layer, tok) if st == 4 else None
            if src in last_pub:
                xlat[st].append(t - last_pub[src])
    # stragglers: per (stage, layer, token) the publishing CTAs' spread and who is last
    pubs = defaultdict(list)
    for cta, recs in enumerate(per_cta):
        for kind, st, layer, tok, t in recs:
            if kind == 2 and st in (0, 1, 2):
                pubs[(st, layer, tok)].append((t, cta))
    spread = defaultdict(list)
    last_cta = defaultdict(lambda: defaultdict(int))
    for (st, layer, tok), v in pubs.items():
        ts = sorted(x[0] for x in v)
        spread[st].append(ts[-1] - ts[len(ts) // 2])
        last_cta[st][max(v)[1]] += 1
    med = lambda xs: statistics.median(xs) / 1000.0 if xs else None  # noqa: E731
    mean = lambda xs: statistics.fmean(xs) / 1000.0 if xs else None  # noqa: E731
    span = max(r[-1][4] for r in per_cta if r) - t0
    return {
        "span_us": span / 1000.0,
        "token_us_max": max(token_ns) / 1000.0 if token_ns else None,
        "layer_period_us_median": med(layer_period),
        "lm_head_us_median": med(lm_ns),
        "exchange_us_median": {STAGE_NAMES[k]: med(v) for k, v in xlat.items()},
        "publish_spread_us_median": {STAGE_NAMES[k]: med(v) for k, v in spread.items()},
        "last_publishers": {STAGE_NAMES[k]: sorted(v.items(), key=lambda kv: -kv[1])[:6] for k, v in last_cta.items()},
        "segments": {k: {"mean_us": statistics.fmean(v) / 1000.0, "median_us": statistics.median(v) / 1000.0,
                         "count": len(v)} for k, v in seg.items()},
        "stages": {STAGE_NAMES[s]: {"wait_us_mean": mean(waits[s]), "wait_us_median": med(waits[s]),
                                    "compute_us_mean": mean(compute[s]), "compute_us_median": med(compute[s])}
                   for s in sorted(set(waits) | set(compute))},
    }


def format_summary(s: dict) -> str:
    lines = [f"launch span {s['span_us']:.1f} us; per-token (max over CTAs) {s['token_us_max']}",
             f"layer period (median, QKV publish to QKV publish) {s['layer_period_us_median']} us; "
             f"LM head (median) {s['lm_head_us_median']} us",
             f"{'stage':16s} {'wait mean':>10s} {'wait med':>10s} {'compute mean':>13s} {'compute med':>12s}  (us)"]
    for name, d in s["stages"].items():
        f = lambda v: f"{v:10.3f}" if v is not None else f"{'-':>10s}"  # noqa: E731
        lines.append(f"{name:16s} {f(d['wait_us_mean'])} {f(d['wait_us_median'])} "
                     f"{f(d['compute_us_mean']):>13s} {f(d['compute_us_median']):>12s}")
    if s.get("exchange_us_median"):
        lines.append("exchange latency (last publish over all CTAs -> wait end), median: " +
                     ", ".join(f"{k} {v:.3f} us" for k, v in s["exchange_us_median"].items() if v is not None))
    if s.get("publish_spread_us_median"):
        lines.append("publish spread (last CTA - median CTA), median over layers: " +
                     ", ".join(f"{k} {v:.3f} us" for k, v in s["publish_spread_us_median"].items() if v is not None))
        for k, v in s["last_publishers"].items():
            lines.append(f"  last {k} publishers (cta: layers): " + ", ".join(f"{c}: {n}" for c, n in v))
    lines.append("segments (time since the CTA's previous stamp, labelled by the later stamp):")
    for k, d in sorted(s.get("segments", {}).items(), key=lambda kv: -kv[1]["mean_us"] * kv[1]["count"]):
        lines.append(f"  {k:28s} mean {d['mean_us']:8.3f} us  median {d['median_us']:8.3f} us  n={d['count']}")
    return "\n".join(lines)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--tokens", type=int, default=1)
    ap.add_argument("--position", type=int, default=32)
    ap.add_argument("--reference-layout", action="store_true")
    ap.add_argument("--repeat", type=int, default=3)
    ap.add_argument("--plain", action="store_true", help="launch without the trace buffer (for ncu)")
    ap.add_argument("--max-seq", type=int, default=512, help="cache slots (4096 for config-3 lengths)")
    a = ap.parse_args()
    dev = torch.device("cuda:0")
    g = torch.Generator(device=dev).manual_seed(1000)

    def lin(*shape):
        return (torch.randn(shape, generator=g, device=dev) * 0.02).to(torch.bfloat16)

    ones = lambda n: torch.ones(n, dtype=torch.bfloat16, device=dev)  # noqa: E731
    embed = lin(151936, 1024)
    layers = []
    for _ in range(28):
        layers += [ones(1024), lin(2048, 1024), lin(1024, 1024), lin(1024, 1024), ones(128), ones(128),
                   lin(1024, 2048), ones(1024), lin(3072, 1024), lin(3072, 1024), lin(1024, 3072)]
    assert 0 <= a.position and a.position + a.tokens <= a.max_seq, "positions past the cache"
    k = torch.randn((28, 8, a.max_seq, 128), generator=g, device=dev).to(torch.bfloat16)
    v = torch.randn((28, 8, a.max_seq, 128), generator=g, device=dev).to(torch.bfloat16)
    td = TracedDecoder(embed, ones(1024), layers, k, v, fused=not a.reference_layout)
    res = None
    for _ in range(a.repeat):
        recs = td.run(1, a.position, a.tokens, traced=not a.plain)
        res = summarize(recs) if recs is not None else None
    if res is None:
        print("plain launches done")
        return
    prod = getattr(td, "producer_records", None)
    if prod and any(prod):
        waits = []
        issues = []
        for recs in prod:
            tot, open_t = 0, None
            for kind, st, _l, _t, t in recs:
                if st == 17 and kind == 0:
                    open_t = t
                elif st == 17 and kind == 1 and open_t is not None:
                    tot += t - open_t
                    open_t = None
                elif st == 18:
                    issues.append(t)
            waits.append(tot)
        print(f"producer: slot-free waits per CTA per launch: mean {statistics.fmean(waits) / 1000:.1f} us, "
              f"max {max(waits) / 1000:.1f} us; chunks issued {len(issues)}")
    print(f"config0 shapes, position {a.position}, {a.tokens} token(s) per launch, "
          f"{'reference' if a.reference_layout else 'transposed'} down layout, grid {td.grid}")
    print(format_summary(res))


if __name__ == "__main__":
    main()
