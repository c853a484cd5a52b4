// Persistent single-launch batch-one Qwen3-0.6B decode kernel for sm_100a.
//
// Structure (one CTA per SM, 17 warps):
//   * warp 16 (producer) walks this CTA's fixed chunk schedule for the whole
//     launch and streams every weight byte (and the KV rows that do not depend
//     on the current token) into a 6 x 32 KB shared-memory ring with 1-D bulk
//     async copies (cp.async.bulk, completion on mbarriers). It never waits on
//     a grid transition (except a one-off acquire before re-reading KV rows in a
//     multi-token launch), so HBM keeps streaming while the consumers wait.
//   * warps 0-15 (consumers) run the stages of each layer and hand off between
//     CTAs through gpu-scope release/acquire counters in the workspace:
//        A  : input RMSNorm + QKV GEMV rows                        -> T_A
//        BC : q/k RMSNorm + RoPE + KV append, GQA decode attention,
//             o_proj partial of this KV head (red.add into acc_mid) -> T_BC
//        DE : post RMSNorm + gate/up SwiGLU rows + down-proj partial
//             over the same rows of the transposed down weight
//             (red.add into acc_down)                               -> T_DE
//        (reference-layout down weight: D writes the SwiGLU vector -> T_D,
//         E computes whole down rows and writes the residual       -> T_E)
//     then final RMSNorm + tied LM head + block/grid argmax.
// Every wait is bounded by DecodeParams::timeout_ns; on expiry the kernel
// records an error in Workspace::error, stops issuing copies, drains the ones in
// flight and returns, so the host gets a status instead of a hang.
//
// Reference: megakernel.cu:744-893 (decode_kernel) and the stage functions it
// calls (megakernel.cu:9-739); see the per-stage comments below.

#include <cfloat>
#include <climits>
#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "mkb_config.cuh"
#include "mkb_ptx.cuh"

namespace mkb {

struct __align__(128) Smem {
  uint8_t ring[kSlots][kSlotBytes];
  uint64_t full[kSlots];
  uint64_t empty[kSlots];
  float r[kHidden];      // residual entering the current layer
  float rmid[kHidden];   // residual after attention + o_proj
  union {
    float att[kConsumerWarps][2][kHeadDim + 4];  // per-warp attention partials
    float x[kInter];                             // SwiGLU vector (reference-layout down)
  } u;
  float q[2][kHeadDim];  // rotated, pre-scaled queries of this KV head's two Q heads
  float knew[kHeadDim];  // rotated new key (BF16-rounded)
  float vnew[kHeadDim];  // new value (BF16-rounded)
  float attn[2 * kHeadDim];
  float gu[2][32];
  float m[32];
  float dpart[8][4];
  float red[32];
  float best_v[kConsumerWarps];
  int best_i[kConsumerWarps];
  // Copy of the device LayerWeights table (+ the transposed down pointer) in
  // shared memory: grid-transition acquires invalidate L1, and these pointers
  // are needed on the critical path of every stage.
  const __nv_bfloat16* lwp[kMaxLayers][12];
  int token;
  int is_last;
  int abort;
};

constexpr size_t kSmemBytes = sizeof(Smem);
static_assert(kSmemBytes <= 232448, "shared memory budget exceeded");

// Upper bound on one hardware-suspended mbarrier wait; the enclosing loops
// re-check the abort flag and the overall timeout after each.
constexpr uint32_t kSuspendNs = 20000;

struct Ctl {
  Smem* sm;
  Workspace* ws;
  uint64_t timeout;
  int cta;
  unsigned long long* trace;  // this CTA's row of the trace buffer (or null)
  int trace_cap;
};

// Stage time stamp (consumer thread 0 only; no-op without a trace buffer).
struct Tracer {
  unsigned long long* row;
  int cap;
  int n;
  int who;  // the one thread that records
  __device__ __forceinline__ void mark(uint32_t kind, uint32_t stage, int layer, int tok) {
    if (row != nullptr && static_cast<int>(threadIdx.x) == who && n < cap) {
      const uint64_t code = kind | ((stage & 31u) << 2) | ((static_cast<uint32_t>(layer) & 31u) << 7) |
                            ((static_cast<uint32_t>(tok) & 15u) << 12);
      row[n++] = (code << 48) | (global_ns() & 0xffffffffffffull);
    }
  }
};

__device__ __forceinline__ bool aborted(const Ctl& c) {
  return *reinterpret_cast<volatile int*>(&c.sm->abort) != 0;
}

__device__ void raise_error(const Ctl& c, uint32_t code, int layer, int stage, int tok) {
  if (atomicCAS(&c.ws->error[0], 0u, code) == 0u) {
    c.ws->error[1] = static_cast<uint32_t>(c.cta);
    c.ws->error[2] = static_cast<uint32_t>(layer);
    c.ws->error[3] = static_cast<uint32_t>(stage);
    c.ws->error[4] = static_cast<uint32_t>(tok);
  }
  *reinterpret_cast<volatile int*>(&c.sm->abort) = 1;
}

// Bounded spin until *ctr >= target (wrap-safe). Single thread.
__device__ void spin_geq(const Ctl& c, const uint32_t* ctr, uint32_t target, uint32_t code, int layer,
                         int stage, int tok) {
  if (aborted(c)) return;
  if (static_cast<int>(ld_acquire(ctr) - target) >= 0) return;
  const uint64_t t0 = global_ns();
  uint32_t it = 0;
  while (true) {
    if (static_cast<int>(ld_acquire(ctr) - target) >= 0) return;
    if ((++it & 15u) == 0u) {
      if (ld_relaxed(&c.ws->error[0]) != 0u) {
        *reinterpret_cast<volatile int*>(&c.sm->abort) = 1;
        return;
      }
      if (global_ns() - t0 > c.timeout) {
        raise_error(c, code, layer, stage, tok);
        return;
      }
    }
  }
}

// Consumer-side transition: thread 0 waits, then all consumers proceed.
__device__ __forceinline__ void transition_wait(const Ctl& c, Tracer& tr, const uint32_t* ctr, uint32_t target,
                                                int layer, int stage, int tok) {
  tr.mark(kTrWaitBegin, stage, layer, tok);
  if (threadIdx.x == 0) spin_geq(c, ctr, target, kErrTimeoutTransition, layer, stage, tok);
  consumer_sync(kConsumerThreads);
  tr.mark(kTrWaitEnd, stage, layer, tok);
}

// Consumer-side publish: every consumer's writes are ordered before the add.
__device__ __forceinline__ void transition_publish(Tracer& tr, uint32_t* ctr, int layer, int stage, int tok) {
  consumer_sync(kConsumerThreads);
  if (threadIdx.x == 0) release_add(ctr, 1u);
  tr.mark(kTrPublish, stage, layer, tok);
}

// ---- ring (consumer side) ----------------------------------------------------
__device__ __forceinline__ uint32_t ring_wait(const Ctl& c, uint32_t n, int layer, int stage, int tok,
                                              Tracer* tr = nullptr) {
  const int s = static_cast<int>(n % kSlots);
  const uint32_t ph = (n / kSlots) & 1u;
  if (!mbar_test(&c.sm->full[s], ph)) {
    if (tr) tr->mark(kTrWaitBegin, kStRing, layer, tok);
    const uint64_t t0 = global_ns();
    while (!mbar_wait(&c.sm->full[s], ph, kSuspendNs)) {
      if (aborted(c)) break;
      if (global_ns() - t0 > c.timeout) {
        raise_error(c, kErrTimeoutRing, layer, stage, tok);
        break;
      }
    }
    if (tr) tr->mark(kTrWaitEnd, kStRing, layer, tok);
  }
  return smem_addr(c.sm->ring[s]);
}
__device__ __forceinline__ void ring_done(const Ctl& c, uint32_t& n) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(&c.sm->empty[n % kSlots]);
  ++n;
}

// ---- math helpers ------------------------------------------------------------
// RMSNorm of a 1024-vector held in shared memory; each lane receives the 32
// normalised elements lane*8 + g*256 + e (g < 4, e < 8) it needs for its part of
// every 2 KB weight row. Same formula as megakernel.cu:704-739.
// The 4 x 16 B of a 1024-element BF16 norm weight this lane needs (loaded ahead
// of the grid transition that gates the norm, so the load latency overlaps it).
__device__ __forceinline__ void load_norm_w(const __nv_bfloat16* w, uint4 wv[4]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int g = 0; g < 4; ++g)
    wv[g] = w ? __ldg(reinterpret_cast<const uint4*>(w + lane * 8 + g * 256))
              : make_uint4(0x3f803f80u, 0x3f803f80u, 0x3f803f80u, 0x3f803f80u);  // bf16 1.0 pairs
}

__device__ __forceinline__ float dot8(const uint4 w, const float* x) {
  float s = bf_lo(w.x) * x[0];
  s = fmaf(bf_hi(w.x), x[1], s);
  s = fmaf(bf_lo(w.y), x[2], s);
  s = fmaf(bf_hi(w.y), x[3], s);
  s = fmaf(bf_lo(w.z), x[4], s);
  s = fmaf(bf_hi(w.z), x[5], s);
  s = fmaf(bf_lo(w.w), x[6], s);
  s = fmaf(bf_hi(w.w), x[7], s);
  return s;
}

// This lane's share of a 2 KB (1024-element) BF16 row in shared memory.
__device__ __forceinline__ float dot_row1024(uint32_t row, const float xr[32], int lane) {
  const uint4 w0 = lds128(row + lane * 16 + 0 * 512);
  const uint4 w1 = lds128(row + lane * 16 + 1 * 512);
  const uint4 w2 = lds128(row + lane * 16 + 2 * 512);
  const uint4 w3 = lds128(row + lane * 16 + 3 * 512);
  return (dot8(w0, xr) + dot8(w1, xr + 8)) + (dot8(w2, xr + 16) + dot8(w3, xr + 24));
}

__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
  const bool vn = v != v, bn = bv != bv;
  if (vn || bn) return vn && (!bn || i < bi);  // torch.argmax: NaN is the maximum
  return v > bv || (v == bv && i < bi);
}

__device__ __forceinline__ float rope_at(const void* table, int fp32, size_t idx) {
  return fp32 ? __ldg(static_cast<const float*>(table) + idx)
              : __bfloat162float(static_cast<const __nv_bfloat16*>(table)[idx]);
}

// Field indices of the shared-memory layer table (LayerWeights order + down_t).
enum LayerField : int {
  kWNorm = 0, kWQ, kWK, kWV, kWQNorm, kWKNorm, kWO, kWPost, kWGate, kWUp, kWDown, kWDownT
};
__device__ __forceinline__ const __nv_bfloat16* lwt(const Ctl& c, int l, int f) { return c.sm->lwp[l][f]; }

// Pointer field of a device-resident table, read through the read-only path.
template <typename T>
__device__ __forceinline__ const T* ldg_ptr(const T* const* field) {
  return reinterpret_cast<const T*>(__ldg(reinterpret_cast<const unsigned long long*>(field)));
}

// ---- producer ----------------------------------------------------------------
struct Producer {
  const Ctl& c;
  uint32_t n;
  bool stop;
  uint64_t pol_w, pol_kv;
  int lane;
  Tracer tr;  // row grid + cta of the trace buffer

  __device__ Producer(const Ctl& ctl) : c(ctl), n(0), stop(false) {
    lane = threadIdx.x & 31;
    pol_w = policy_evict_first();
    pol_kv = policy_evict_last();
    // ctl.trace is this CTA's consumer row (base + cta * cap); its producer row
    // is base + (grid + cta) * cap.
    tr = Tracer{ctl.trace ? ctl.trace + (size_t)gridDim.x * ctl.trace_cap : nullptr, ctl.trace_cap, 0,
                kConsumerThreads};
  }

  // Reserve the next slot for `bytes`; returns its index or -1 once stopped.
  __device__ int begin(uint32_t bytes) {
    if (stop) return -1;
    const int s = static_cast<int>(n % kSlots);
    const uint32_t ph = ((n / kSlots) & 1u) ^ 1u;
    int ok = 1;
    if (lane == 0) {
      if (!mbar_test(&c.sm->empty[s], ph)) {
        tr.mark(kTrWaitBegin, kStSlot, static_cast<int>(n & 31u), 0);
        const uint64_t t0 = global_ns();
        while (!mbar_wait(&c.sm->empty[s], ph, kSuspendNs)) {
          if (aborted(c)) { ok = 0; break; }
          if (global_ns() - t0 > c.timeout) {
            raise_error(c, kErrTimeoutRing, -1, -1, -1);
            ok = 0;
            break;
          }
        }
        tr.mark(kTrWaitEnd, kStSlot, static_cast<int>(n & 31u), 0);
      }
      if (ok && aborted(c)) ok = 0;
      if (ok) mbar_arrive_expect_tx(&c.sm->full[s], bytes);
      tr.mark(kTrMark, kStIssue, static_cast<int>(n & 31u), 0);
    }
    ok = __shfl_sync(0xffffffffu, ok, 0);
    if (!ok) { stop = true; return -1; }
    return s;
  }
  __device__ void end() { __syncwarp(); ++n; }

  // One bulk copy into slot s at byte offset off. Misaligned operands are a
  // caller error: record it and stop instead of issuing the copy.
  __device__ void copy(int s, uint32_t off, const void* src, uint32_t bytes, uint64_t pol) {
    if (bytes == 0) return;
    if (((reinterpret_cast<uintptr_t>(src) | bytes) & 15u) != 0u) {
      raise_error(c, kErrBadArgs, -1, -2, -1);
      return;
    }
    bulk_g2s(c.sm->ring[s] + off, src, bytes, &c.sm->full[s], pol);
  }

  // L2 prefetch (16-byte aligned operands only; others are simply skipped).
  __device__ void prefetch(const void* src, uint32_t bytes) {
    if (bytes == 0 || ((reinterpret_cast<uintptr_t>(src) | bytes) & 15u) != 0u) return;
    bulk_prefetch_l2(src, bytes, pol_kv);
  }

  // Wait for every copy still in flight before the CTA exits.
  __device__ void drain() {
    if (lane != 0) return;
    for (int s = 0; s < kSlots; ++s) {
      if (n <= static_cast<uint32_t>(s)) continue;
      const uint32_t last = n - 1u - ((n - 1u - s) % kSlots);
      const uint32_t ph = (last / kSlots) & 1u;
      const uint64_t t0 = global_ns();
      while (!mbar_wait(&c.sm->full[s], ph, kSuspendNs)) {
        if (global_ns() - t0 > c.timeout) break;
      }
    }
  }
};

// Pull this CTA's bytes of layer `l` (cache length `cl`) into L2 ahead of the
// ring, so HBM keeps streaming while the consumers wait at grid transitions and
// the ring refills from L2.
__device__ void prefetch_layer(Producer& pr, const DecodeParams& p, const Plan& pl, int l, int cl, int splits) {
  if (pr.lane == 0) {
    for (int r = pl.qa; r < pl.qb;) {
      int e = r < kQSize ? kQSize : (r < kQSize + kKVSize ? kQSize + kKVSize : kQKVRows);
      if (e > pl.qb) e = pl.qb;
      const __nv_bfloat16* src = r < kQSize ? lwt(pr.c, l, kWQ) + (size_t)r * kHidden
                                 : r < kQSize + kKVSize
                                     ? lwt(pr.c, l, kWK) + (size_t)(r - kQSize) * kHidden
                                     : lwt(pr.c, l, kWV) + (size_t)(r - kQSize - kKVSize) * kHidden;
      pr.prefetch(src, static_cast<uint32_t>(e - r) * kHidden * 2u);
      r = e;
    }
    if (pl.in_bc) {
      int ka, kb;
      key_range(cl, splits, pl.c, &ka, &kb);
      const size_t head_off = ((size_t)l * kNKV + pl.h) * (size_t)p.max_seq * kHeadDim;
      pr.prefetch(p.k_cache + head_off + (size_t)ka * kHeadDim, static_cast<uint32_t>(kb - ka) * kHeadDim * 2u);
      pr.prefetch(p.v_cache + head_off + (size_t)ka * kHeadDim, static_cast<uint32_t>(kb - ka) * kHeadDim * 2u);
    }
    const uint32_t gu = static_cast<uint32_t>(pl.jb - pl.ja) * kHidden * 2u;
    pr.prefetch(lwt(pr.c, l, kWGate) + (size_t)pl.ja * kHidden, gu);
    pr.prefetch(lwt(pr.c, l, kWUp) + (size_t)pl.ja * kHidden, gu);
    if (p.down_t != nullptr) {
      pr.prefetch(lwt(pr.c, l, kWDownT) + (size_t)pl.ja * kHidden, gu);
    } else {
      pr.prefetch(lwt(pr.c, l, kWDown) + (size_t)pl.da * kInter,
                  static_cast<uint32_t>(pl.db - pl.da) * kInter * 2u);
    }
  }
  if (pl.in_bc) {
    const __nv_bfloat16* wo = lwt(pr.c, l, kWO);
    for (int row = pl.oa + pr.lane; row < pl.ob; row += 32)
      pr.prefetch(wo + (size_t)row * kQSize + pl.h * 2 * kHeadDim, 512u);
  }
  __syncwarp();
}

// Percentage of each CTA's LM-head rows pulled into L2 during the last layers.
constexpr int kLmPreloadPct = 15;
constexpr int kLmPreloadLayers = 4;

__device__ void producer_run(const DecodeParams& p, const Plan& pl, const Ctl& c, int pos0, int cl0,
                             int splits) {
  Producer pr(c);
  const bool fused = p.down_t != nullptr;
  const int nbc = kNKV * p.group_size;
  for (int t = 0; t < p.n_tokens && !pr.stop; ++t) {
    const int pos = pos0 + t;
    const int cl = cl0 + t;
    for (int l = p.layer_begin; l < p.layer_end && !pr.stop; ++l) {
      // L2 prefetch one layer ahead (the next token's first layer after the last)
      if (l == p.layer_begin && t == 0) prefetch_layer(pr, p, pl, l, cl, splits);
      if (l + 1 < p.layer_end) prefetch_layer(pr, p, pl, l + 1, cl, splits);
      else if (t + 1 < p.n_tokens) prefetch_layer(pr, p, pl, p.layer_begin, cl + 1, splits);
      if ((p.flags & kFlagLmHead) && l >= p.layer_end - kLmPreloadLayers && pr.lane == 0) {
        const int npre = (pl.vb - pl.va) * kLmPreloadPct / 100;
        const int part_i = l - (p.layer_end - kLmPreloadLayers);
        const int r0 = pl.va + part(npre, kLmPreloadLayers, part_i);
        const int r1 = pl.va + part(npre, kLmPreloadLayers, part_i + 1);
        pr.prefetch(p.lm_head + (size_t)r0 * kHidden, static_cast<uint32_t>(r1 - r0) * kHidden * 2u);
      }
      // A: QKV rows, one bulk copy per row into a padded row slot
      for (int r = pl.qa; r < pl.qb;) {
        const int e = qkv_chunk_end(r, pl.qb);
        const __nv_bfloat16* src = r < kQSize ? lwt(pr.c, l, kWQ) + (size_t)r * kHidden
                                   : r < kQSize + kKVSize
                                       ? lwt(pr.c, l, kWK) + (size_t)(r - kQSize) * kHidden
                                       : lwt(pr.c, l, kWV) + (size_t)(r - kQSize - kKVSize) * kHidden;
        const int s = pr.begin(static_cast<uint32_t>(e - r) * kHidden * 2u);
        if (s < 0) break;
        if (pr.lane < e - r)
          pr.copy(s, static_cast<uint32_t>(pr.lane) * kRowStride, src + (size_t)pr.lane * kHidden, kHidden * 2u,
                  pr.pol_w);
        pr.end();
        r = e;
      }
      // BC: KV rows of this KV head (old positions only), then the o_proj slice
      if (pl.in_bc) {
        int ka, kb;
        key_range(cl, splits, pl.c, &ka, &kb);
        if (t > 0 && kb > ka && pr.lane == 0) {
          // The previous token of this launch appended K/V at pos-1; make it
          // visible to the bulk-copy engine before re-reading those rows.
          spin_geq(c, &p.ws->sync[l][1][0], static_cast<uint32_t>(nbc * t), kErrTimeoutTransition, l, 10, t);
          fence_proxy_async_global();
        }
        const size_t head_off = ((size_t)l * kNKV + pl.h) * (size_t)p.max_seq * kHeadDim;
        const __nv_bfloat16* kbase = p.k_cache + head_off;
        const __nv_bfloat16* vbase = p.v_cache + head_off;
        for (int k0 = ka; k0 < kb; k0 += kKeysPerChunk) {
          const int k1 = min(kb, k0 + kKeysPerChunk);
          const bool has_pos = pos >= k0 && pos < k1;
          const uint32_t bytes = 2u * kHeadDim * 2u * static_cast<uint32_t>(k1 - k0 - (has_pos ? 1 : 0));
          const int s = pr.begin(bytes);
          if (s < 0) break;
          if (pr.lane == 0) {
            const uint32_t row = kHeadDim * 2u;
            if (!has_pos) {
              pr.copy(s, 0, kbase + (size_t)k0 * kHeadDim, row * (k1 - k0), pr.pol_kv);
              pr.copy(s, kSlotBytes / 2, vbase + (size_t)k0 * kHeadDim, row * (k1 - k0), pr.pol_kv);
            } else {
              pr.copy(s, 0, kbase + (size_t)k0 * kHeadDim, row * (pos - k0), pr.pol_kv);
              pr.copy(s, kSlotBytes / 2, vbase + (size_t)k0 * kHeadDim, row * (pos - k0), pr.pol_kv);
              pr.copy(s, row * (pos + 1 - k0), kbase + (size_t)(pos + 1) * kHeadDim, row * (k1 - pos - 1), pr.pol_kv);
              pr.copy(s, kSlotBytes / 2 + row * (pos + 1 - k0), vbase + (size_t)(pos + 1) * kHeadDim,
                      row * (k1 - pos - 1), pr.pol_kv);
            }
          }
          pr.end();
        }
        const __nv_bfloat16* wo = lwt(pr.c, l, kWO);
        for (int o0 = pl.oa; o0 < pl.ob; o0 += kORowsPerChunk) {
          const int o1 = min(pl.ob, o0 + kORowsPerChunk);
          const int s = pr.begin(static_cast<uint32_t>(o1 - o0) * 512u);
          if (s < 0) break;
          for (int row = o0 + pr.lane; row < o1; row += 32)
            pr.copy(s, static_cast<uint32_t>(row - o0) * kORowStride, wo + (size_t)row * kQSize + pl.h * 2 * kHeadDim,
                    512u, pr.pol_w);
          pr.end();
        }
      }
      // DE / D: gate and up rows
      const __nv_bfloat16* wg = lwt(pr.c, l, kWGate);
      const __nv_bfloat16* wu = lwt(pr.c, l, kWUp);
      for (int j0 = pl.ja; j0 < pl.jb; j0 += kGUPerChunk) {
        const int j1 = min(pl.jb, j0 + kGUPerChunk);
        // gate rows to padded slots in the first half, up rows in the second
        const int s = pr.begin(2u * static_cast<uint32_t>(j1 - j0) * kHidden * 2u);
        if (s < 0) break;
        if (pr.lane < 2 * (j1 - j0)) {
          const int i = pr.lane % (j1 - j0);
          const bool up = pr.lane >= (j1 - j0);
          pr.copy(s, (up ? kSlotBytes / 2 : 0) + static_cast<uint32_t>(i) * kRowStride,
                  (up ? wu : wg) + (size_t)(j0 + i) * kHidden, kHidden * 2u, pr.pol_w);
        }
        pr.end();
      }
      if (fused) {
        const __nv_bfloat16* wdt = lwt(pr.c, l, kWDownT);
        for (int j0 = pl.ja; j0 < pl.jb; j0 += kRowsPerChunk1024) {
          const int j1 = min(pl.jb, j0 + kRowsPerChunk1024);
          const uint32_t bytes = static_cast<uint32_t>(j1 - j0) * kHidden * 2u;
          const int s = pr.begin(bytes);
          if (s < 0) break;
          if (pr.lane == 0) pr.copy(s, 0, wdt + (size_t)j0 * kHidden, bytes, pr.pol_w);
          pr.end();
        }
      } else {
        const __nv_bfloat16* wd = lwt(pr.c, l, kWDown);
        for (int d0 = pl.da; d0 < pl.db; d0 += kDownRowsPerChunk) {
          const int d1 = min(pl.db, d0 + kDownRowsPerChunk);
          const uint32_t bytes = static_cast<uint32_t>(d1 - d0) * kInter * 2u;
          const int s = pr.begin(bytes);
          if (s < 0) break;
          if (pr.lane == 0) pr.copy(s, 0, wd + (size_t)d0 * kInter, bytes, pr.pol_w);
          pr.end();
        }
      }
    }
    if (p.flags & kFlagLmHead) {
      for (int v0 = pl.va; v0 < pl.vb; v0 += kRowsPerChunk1024) {
        const int v1 = min(pl.vb, v0 + kRowsPerChunk1024);
        const uint32_t bytes = static_cast<uint32_t>(v1 - v0) * kHidden * 2u;
        const int s = pr.begin(bytes);
        if (s < 0) break;
        if (pr.lane == 0) pr.copy(s, 0, p.lm_head + (size_t)v0 * kHidden, bytes, pr.pol_w);
        pr.end();
      }
    }
  }
  pr.drain();
}

// ---- consumers -----------------------------------------------------------------

// ---- tensor-core GEMV over padded rows in a ring slot -------------------------
// Warp w owns the reduction range k in [64w, 64w+64) of a 1024-wide row (four
// 16-wide MMA k-steps); the 16 warps' partial sums are added through shared
// memory. The activation x enters as B columns 0 (bf16 hi part) and 1 (bf16
// remainder x - hi), so D[:,0] + D[:,1] carries ~16 mantissa bits of x.
//
// Norm weights for this lane's B-fragment entries (lanes 0-7 only), loaded ahead
// of the transition that gates the norm.
__device__ __forceinline__ void load_norm_k(const __nv_bfloat16* w, uint32_t nw2[4][2]) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int st = 0; st < 4; ++st) {
    const int k = 64 * warp + 16 * st + 2 * (lane & 3);
    if (lane < 8 && w != nullptr) {
      nw2[st][0] = __ldg(reinterpret_cast<const unsigned int*>(w + k));
      nw2[st][1] = __ldg(reinterpret_cast<const unsigned int*>(w + k + 8));
    } else {
      nw2[st][0] = 0x3f803f80u;  // bf16 1.0 pair
      nw2[st][1] = 0x3f803f80u;
    }
  }
}
// B fragments of x = v * rstd * w for this warp's k range (v in shared memory).
__device__ __forceinline__ void build_bfrag(const float* v, float rstd, const uint32_t nw2[4][2], uint32_t bfr[4][2]) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int st = 0; st < 4; ++st) {
    bfr[st][0] = 0u;
    bfr[st][1] = 0u;
    if (lane < 8) {
      const int k = 64 * warp + 16 * st + 2 * (lane & 3);
      const float x0 = v[k] * rstd * bf_lo(nw2[st][0]);
      const float x1 = v[k + 1] * rstd * bf_hi(nw2[st][0]);
      const float x8 = v[k + 8] * rstd * bf_lo(nw2[st][1]);
      const float x9 = v[k + 9] * rstd * bf_hi(nw2[st][1]);
      const uint32_t h0 = pack_bf2(x0, x1), h1 = pack_bf2(x8, x9);
      if (lane < 4) {
        bfr[st][0] = h0;
        bfr[st][1] = h1;
      } else {
        bfr[st][0] = pack_bf2(x0 - bf_lo(h0), x1 - bf_hi(h0));
        bfr[st][1] = pack_bf2(x8 - bf_lo(h1), x9 - bf_hi(h1));
      }
    }
  }
}
// One 16-row tile of padded 1024-wide rows at `base` (rows >= nrows read row 0).
__device__ __forceinline__ void mma_tile_1024(uint32_t base, int nrows, const uint32_t bfr[4][2], float* d) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int tr = lane & 15;
  const uint32_t row = base + (tr < nrows ? tr : 0) * kRowStride + (lane >> 4) * 16 + warp * 128;
#pragma unroll
  for (int st = 0; st < 4; ++st) {
    uint32_t a0, a1, a2, a3;
    ldsm_x4(row + st * 32, a0, a1, a2, a3);
    mma_bf16(d, a0, a1, a2, a3, bfr[st][0], bfr[st][1]);
  }
}
// Gate/up tile: tile rows 0-6 are gate rows, 8-14 up rows (second slot half).
__device__ __forceinline__ void mma_tile_gu(uint32_t base, int nrows, const uint32_t bfr[4][2], float* d) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int tr = lane & 15, i = tr & 7;
  const uint32_t row = base + (tr >= 8 ? kSlotBytes / 2 : 0) + (i < nrows ? i : 0) * kRowStride + (lane >> 4) * 16 +
                       warp * 128;
#pragma unroll
  for (int st = 0; st < 4; ++st) {
    uint32_t a0, a1, a2, a3;
    ldsm_x4(row + st * 32, a0, a1, a2, a3);
    mma_bf16(d, a0, a1, a2, a3, bfr[st][0], bfr[st][1]);
  }
}
// Lanes holding D column pairs write this warp's row partials of tile t.
__device__ __forceinline__ void stash_tile(float (*xred)[64], int t, const float* d) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if ((lane & 3) == 0) {
    xred[warp][t * 16 + (lane >> 2)] = d[0] + d[1];
    xred[warp][t * 16 + (lane >> 2) + 8] = d[2] + d[3];
  }
}
__device__ __forceinline__ float sum_warps(float (*xred)[64], int idx) {
  float v = 0.f;
#pragma unroll
  for (int w = 0; w < kConsumerWarps; ++w) v += xred[w][idx];
  return v;
}

// Wait for `cnt` consecutive chunks from ring position n (all already issued by
// the producer); their slot addresses go to sa[].
__device__ __forceinline__ void ring_wait_all(const Ctl& c, uint32_t n, int cnt, uint32_t* sa, int layer, int stage,
                                              int tok, Tracer* tr) {
#pragma unroll
  for (int i = 0; i < 3; ++i)
    if (i < cnt) sa[i] = ring_wait(c, n + i, layer, stage, tok, tr);
}
__device__ __forceinline__ void ring_done_all(const Ctl& c, uint32_t& n, int cnt) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0)
    for (int i = 0; i < cnt; ++i) mbar_arrive(&c.sm->empty[(n + i) % kSlots]);
  n += cnt;
}

// Block-wide sum of a*a + b*b over the consumer threads (one named barrier;
// s_red alternates between two halves so no trailing barrier is needed).
__device__ __forceinline__ float block_sumsq(float a, float b, float* s_red, int& flip) {
  const float ss = warp_sum(a * a + b * b);
  float* buf = s_red + (flip ? kConsumerWarps : 0);
  flip ^= 1;
  if ((threadIdx.x & 31) == 0) buf[threadIdx.x >> 5] = ss;
  consumer_sync(kConsumerThreads);
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < kConsumerWarps; ++i) tot += buf[i];
  return tot;
}

// The 32 normalised activations this lane multiplies into every 2 KB row:
// elements lane*8 + g*256 + e of v * rstd * w (RMSNorm, megakernel.cu:704-739).
__device__ __forceinline__ void xr_from(const float* v, float rstd, const uint4 wv[4], float xr[32]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const int idx = lane * 8 + g * 256;
    const float4 v0 = *reinterpret_cast<const float4*>(v + idx);
    const float4 v1 = *reinterpret_cast<const float4*>(v + idx + 4);
    xr[g * 8 + 0] = v0.x * rstd * bf_lo(wv[g].x);
    xr[g * 8 + 1] = v0.y * rstd * bf_hi(wv[g].x);
    xr[g * 8 + 2] = v0.z * rstd * bf_lo(wv[g].y);
    xr[g * 8 + 3] = v0.w * rstd * bf_hi(wv[g].y);
    xr[g * 8 + 4] = v1.x * rstd * bf_lo(wv[g].z);
    xr[g * 8 + 5] = v1.y * rstd * bf_hi(wv[g].z);
    xr[g * 8 + 6] = v1.z * rstd * bf_lo(wv[g].w);
    xr[g * 8 + 7] = v1.w * rstd * bf_hi(wv[g].w);
  }
}

// Butterfly sums of three per-lane partials at once (independent shuffle chains).
__device__ __forceinline__ void warp_sum3(float& a, float& b, float& d) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    a += __shfl_xor_sync(0xffffffffu, a, o);
    b += __shfl_xor_sync(0xffffffffu, b, o);
    d += __shfl_xor_sync(0xffffffffu, d, o);
  }
}

// Bounded poll of two tagged words (16 bytes) until both carry `tag`.
__device__ __forceinline__ void poll_tagged2(const Ctl& c, const uint64_t* p, uint32_t tag, float& v0, float& v1,
                                             int layer, int tok) {
  uint64_t a, b;
  ld_tagged2(p, a, b);
  if (static_cast<uint32_t>(a >> 32) != tag || static_cast<uint32_t>(b >> 32) != tag) {
    const uint64_t t0 = global_ns();
    uint32_t it = 0;
    while (true) {
      ld_tagged2(p, a, b);
      if (static_cast<uint32_t>(a >> 32) == tag && static_cast<uint32_t>(b >> 32) == tag) break;
      if ((++it & 15u) == 0u) {
        if (aborted(c) || ld_relaxed(&c.ws->error[0]) != 0u) {
          *reinterpret_cast<volatile int*>(&c.sm->abort) = 1;
          break;
        }
        if (global_ns() - t0 > c.timeout) {
          raise_error(c, kErrTimeoutTransition, layer, kStBC, tok);
          break;
        }
      }
    }
  }
  v0 = __uint_as_float(static_cast<uint32_t>(a));
  v1 = __uint_as_float(static_cast<uint32_t>(b));
}

__device__ void consumer_run(const DecodeParams& p, const Plan& pl, const Ctl& c, int token0, int pos0, int cl0,
                             int splits, uint32_t tag0) {
  Smem& sm = *c.sm;
  Workspace* ws = p.ws;
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const bool fused = p.down_t != nullptr;
  const int G = p.grid;
  const int nbc = kNKV * p.group_size;
  const int lb = p.layer_begin, le = p.layer_end;
  const int zero_cta = G - 1;
  uint32_t n = 0;
  int flip = 0;
  float xr[32];
  Tracer tr{c.trace, c.trace_cap, 0, 0};

  int token = token0;
  for (int t = 0; t < p.n_tokens; ++t) {
    const int pos = pos0 + t;
    const int cl = cl0 + t;
    const uint32_t tgtG = static_cast<uint32_t>(G * (t + 1));
    const uint32_t tgtBC = static_cast<uint32_t>(nbc * (t + 1));
    const uint32_t tag = tag0 + static_cast<uint32_t>(t) + 1u;
    tr.mark(kTrMark, kStToken, 0, t);

    // ---- token input: embedding gather (megakernel.cu:783-795) ----
    if (t > 0) {
      if (tid == 0) spin_geq(c, &ws->tok_flag[0], static_cast<uint32_t>(t), kErrTimeoutToken, -1, 9, t);
      consumer_sync(kConsumerThreads);
      if (tid == 0) sm.token = static_cast<int>(__ldcg(reinterpret_cast<const int*>(&ws->tok_flag[1])));
      consumer_sync(kConsumerThreads);
      token = sm.token;
    }
    token = min(max(token, 0), kVocab - 1);
    float r0 = p.input_residual ? __ldcg(p.input_residual + tid)
                                : __bfloat162float(p.embed[(size_t)token * kHidden + tid]);
    float r1 = p.input_residual ? __ldcg(p.input_residual + tid + kConsumerThreads)
                                : __bfloat162float(p.embed[(size_t)token * kHidden + tid + kConsumerThreads]);

    uint32_t nwA[4][2], nwD[4][2];
    if (le > lb) load_norm_k(lwt(c, lb, kWNorm), nwA);
    for (int l = lb; l < le; ++l) {
      // ================= A: RMSNorm + QKV rows (megakernel.cu:704-739, 633-701) ===
      uint32_t bfr[4][2];
      float(*xred)[64] = reinterpret_cast<float(*)[64]>(&sm.u.att[0][0][0]);
      if (l > lb) {
        transition_wait(c, tr, &ws->sync[l - 1][fused ? 2 : 3][0], tgtG, l, kStA, t);
        if (fused) {
          r0 = sm.rmid[tid] + __ldcg(&ws->acc_down[l - 1][tid]);
          r1 = sm.rmid[tid + kConsumerThreads] + __ldcg(&ws->acc_down[l - 1][tid + kConsumerThreads]);
        } else {
          r0 = __ldcg(&ws->resid[tid]);
          r1 = __ldcg(&ws->resid[tid + kConsumerThreads]);
        }
        // Every CTA has finished layer l-1 (and so read the accumulators of
        // layer l-2): clear those for the next token.
        if (c.cta == zero_cta && l >= lb + 2) {
          ws->acc_mid[l - 2][tid] = 0.f;
          ws->acc_mid[l - 2][tid + kConsumerThreads] = 0.f;
          ws->acc_down[l - 2][tid] = 0.f;
          ws->acc_down[l - 2][tid + kConsumerThreads] = 0.f;
        }
      }
      sm.r[tid] = r0;
      sm.r[tid + kConsumerThreads] = r1;
      {
        const float tot = block_sumsq(r0, r1, sm.red, flip);
        tr.mark(kTrMark, kSubAInput, l, t);
        build_bfrag(sm.r, rsqrtf(tot * (1.0f / kHidden) + kEps), nwA, bfr);
      }
      tr.mark(kTrMark, kSubANorm, l, t);
      // QKV rows: up to three padded chunks (one 16-row MMA tile each) per pass
      for (int r = pl.qa; r < pl.qb;) {
        const int ra0 = r, ea0 = qkv_chunk_end(ra0, pl.qb);
        const int ra1 = ea0, ea1 = ra1 < pl.qb ? qkv_chunk_end(ra1, pl.qb) : ra1;
        const int ra2 = ea1, ea2 = ra2 < pl.qb ? qkv_chunk_end(ra2, pl.qb) : ra2;
        const int na = 1 + (ea1 > ra1) + (ea2 > ra2);
        r = ea2;
        uint32_t sa[3];
        ring_wait_all(c, n, na, sa, l, 0, t, &tr);
        float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f}, d2[4] = {0.f, 0.f, 0.f, 0.f};
        mma_tile_1024(sa[0], ea0 - ra0, bfr, d0);
        if (na > 1) mma_tile_1024(sa[1], ea1 - ra1, bfr, d1);
        if (na > 2) mma_tile_1024(sa[2], ea2 - ra2, bfr, d2);
        ring_done_all(c, n, na);
        stash_tile(xred, 0, d0);
        stash_tile(xred, 1, d1);
        stash_tile(xred, 2, d2);
        consumer_sync(kConsumerThreads);
        if (tid < 48 && !(t == 0 && l == lb && c.cta == p.withhold_cta)) {
          const int i = tid >> 4;
          const int row = (i == 0 ? ra0 : (i == 1 ? ra1 : ra2)) + (tid & 15);
          const int end = i == 0 ? ea0 : (i == 1 ? ea1 : ea2);
          if ((tid & 15) < 15 && row < end) {
            const float val = sum_warps(xred, tid);
            st_tagged(&ws->qkv_tagged[l][row], val, tag);
            float* dst = row < kQSize ? p.q_out + row
                         : row < kQSize + kKVSize ? p.k_out + (row - kQSize)
                                                  : p.v_out + (row - kQSize - kKVSize);
            *dst = val;
          }
        }
        consumer_sync(kConsumerThreads);
      }
      tr.mark(kTrPublish, kStA, l, t);
      load_norm_k(lwt(c, l, kWPost), nwD);  // post-attention norm, one stage ahead

      // ================= BC: head norm + RoPE + KV append, attention, o_proj =====
      if (pl.in_bc) {
        const int h = pl.h;
        // Per-head norm weights and this position's RoPE row do not depend on
        // QKV: load them before polling. Lane owns dims 2l, 2l+1, 64+2l, 65+2l.
        float w0 = 0.f, w1 = 0.f, w2 = 0.f, w3 = 0.f, cs0 = 0.f, sn0 = 0.f, cs1 = 0.f, sn1 = 0.f;
        const int d0 = 2 * lane;
        if (warp < 3) {
          const __nv_bfloat16* nw = lwt(c, l, warp < 2 ? kWQNorm : kWKNorm);
          w0 = __bfloat162float(nw[d0]);
          w1 = __bfloat162float(nw[d0 + 1]);
          w2 = __bfloat162float(nw[d0 + 64]);
          w3 = __bfloat162float(nw[d0 + 65]);
          const size_t rb = (size_t)pos * kHeadDim;
          cs0 = rope_at(p.cos_table, p.rope_fp32, rb + d0);
          sn0 = rope_at(p.sin_table, p.rope_fp32, rb + d0);
          cs1 = rope_at(p.cos_table, p.rope_fp32, rb + d0 + 1);
          sn1 = rope_at(p.sin_table, p.rope_fp32, rb + d0 + 1);
        }
        tr.mark(kTrWaitBegin, kStBC, l, t);
        if (warp < 4) {
          const int base = warp < 2 ? (2 * h + warp) * kHeadDim
                                    : (warp == 2 ? kQSize + h * kHeadDim : kQSize + kKVSize + h * kHeadDim);
          float x0, x1, x2, x3;  // dims d0, d0+1, d0+64, d0+65
          poll_tagged2(c, &ws->qkv_tagged[l][base + d0], tag, x0, x1, l, t);
          poll_tagged2(c, &ws->qkv_tagged[l][base + d0 + 64], tag, x2, x3, l, t);
          if (warp < 3) {
            // q_norm / k_norm + rotate-half RoPE (megakernel.cu:490-630)
            const float ss = warp_sum(x0 * x0 + x1 * x1 + x2 * x2 + x3 * x3);
            const float rstd = rsqrtf(ss * (1.0f / kHeadDim) + kEps);
            const float y0 = x0 * rstd * w0, y1 = x1 * rstd * w1;
            const float y2 = x2 * rstd * w2, y3 = x3 * rstd * w3;
            const float o0 = y0 * cs0 - y2 * sn0, o2 = y2 * cs0 + y0 * sn0;   // pair (d0, d0+64)
            const float o1 = y1 * cs1 - y3 * sn1, o3 = y3 * cs1 + y1 * sn1;   // pair (d0+1, d0+65)
            if (warp < 2) {
              const float sc = 0.08838834764831845f * 1.4426950408889634f;  // 1/sqrt(128) * log2(e)
              sm.q[warp][d0] = o0 * sc;
              sm.q[warp][d0 + 1] = o1 * sc;
              sm.q[warp][d0 + 64] = o2 * sc;
              sm.q[warp][d0 + 65] = o3 * sc;
            } else {
              const __nv_bfloat162 b01 = __floats2bfloat162_rn(o0, o1);
              const __nv_bfloat162 b23 = __floats2bfloat162_rn(o2, o3);
              sm.knew[d0] = __low2float(b01);
              sm.knew[d0 + 1] = __high2float(b01);
              sm.knew[d0 + 64] = __low2float(b23);
              sm.knew[d0 + 65] = __high2float(b23);
              if (pl.c == 0) {
                __nv_bfloat16* dst = p.k_cache + (((size_t)l * kNKV + h) * p.max_seq + pos) * kHeadDim;
                *reinterpret_cast<__nv_bfloat162*>(dst + d0) = b01;
                *reinterpret_cast<__nv_bfloat162*>(dst + d0 + 64) = b23;
              }
            }
          } else {
            const __nv_bfloat162 b01 = __floats2bfloat162_rn(x0, x1);
            const __nv_bfloat162 b23 = __floats2bfloat162_rn(x2, x3);
            sm.vnew[d0] = __low2float(b01);
            sm.vnew[d0 + 1] = __high2float(b01);
            sm.vnew[d0 + 64] = __low2float(b23);
            sm.vnew[d0 + 65] = __high2float(b23);
            if (pl.c == 0) {
              __nv_bfloat16* dst = p.v_cache + (((size_t)l * kNKV + h) * p.max_seq + pos) * kHeadDim;
              *reinterpret_cast<__nv_bfloat162*>(dst + d0) = b01;
              *reinterpret_cast<__nv_bfloat162*>(dst + d0 + 64) = b23;
            }
          }
        }
        consumer_sync(kConsumerThreads);
        tr.mark(kTrWaitEnd, kStBC, l, t);
        tr.mark(kTrMark, kSubBCPrep, l, t);
        // GQA decode attention over keys [ka, kb) (megakernel.cu:228-370),
        // per-warp online softmax in the exp2 domain, then a 16-warp combine.
        int ka, kb;
        key_range(cl, splits, pl.c, &ka, &kb);
        if (kb > ka) {
          float q0[4], q1[4];
#pragma unroll
          for (int d = 0; d < 4; ++d) {
            q0[d] = sm.q[0][lane * 4 + d];
            q1[d] = sm.q[1][lane * 4 + d];
          }
          float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
          float a0[4] = {0.f, 0.f, 0.f, 0.f}, a1[4] = {0.f, 0.f, 0.f, 0.f};
          for (int k0 = ka; k0 < kb; k0 += kKeysPerChunk) {
            const int k1 = min(kb, k0 + kKeysPerChunk);
            const uint32_t sa = ring_wait(c, n, l, 1, t, &tr);
            float s0[4], s1[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int kk = k0 + warp * 4 + i;
              float kx0 = 0.f, kx1 = 0.f, kx2 = 0.f, kx3 = 0.f;
              if (kk < k1) {
                if (kk == pos) {
                  kx0 = sm.knew[lane * 4 + 0];
                  kx1 = sm.knew[lane * 4 + 1];
                  kx2 = sm.knew[lane * 4 + 2];
                  kx3 = sm.knew[lane * 4 + 3];
                } else {
                  const uint2 u = lds64(sa + (kk - k0) * (kHeadDim * 2) + lane * 8);
                  kx0 = bf_lo(u.x);
                  kx1 = bf_hi(u.x);
                  kx2 = bf_lo(u.y);
                  kx3 = bf_hi(u.y);
                }
              }
              s0[i] = fmaf(q0[3], kx3, fmaf(q0[2], kx2, fmaf(q0[1], kx1, q0[0] * kx0)));
              s1[i] = fmaf(q1[3], kx3, fmaf(q1[2], kx2, fmaf(q1[1], kx1, q1[0] * kx0)));
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                s0[i] += __shfl_xor_sync(0xffffffffu, s0[i], o);
                s1[i] += __shfl_xor_sync(0xffffffffu, s1[i], o);
              }
            }
            float mx0 = m0, mx1 = m1;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              if (k0 + warp * 4 + i >= k1) {
                s0[i] = -INFINITY;
                s1[i] = -INFINITY;
              }
              mx0 = fmaxf(mx0, s0[i]);
              mx1 = fmaxf(mx1, s1[i]);
            }
            float p0[4] = {0.f, 0.f, 0.f, 0.f}, p1[4] = {0.f, 0.f, 0.f, 0.f};
            if (mx0 > -INFINITY) {
              const float sc = exp2f(m0 - mx0);
              float ps = 0.f;
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                p0[i] = exp2f(s0[i] - mx0);
                ps += p0[i];
              }
              l0 = l0 * sc + ps;
#pragma unroll
              for (int d = 0; d < 4; ++d) a0[d] *= sc;
              m0 = mx0;
            }
            if (mx1 > -INFINITY) {
              const float sc = exp2f(m1 - mx1);
              float ps = 0.f;
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                p1[i] = exp2f(s1[i] - mx1);
                ps += p1[i];
              }
              l1 = l1 * sc + ps;
#pragma unroll
              for (int d = 0; d < 4; ++d) a1[d] *= sc;
              m1 = mx1;
            }
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int kk = k0 + warp * 4 + i;
              if (kk < k1) {
                float vx[4];
                if (kk == pos) {
#pragma unroll
                  for (int d = 0; d < 4; ++d) vx[d] = sm.vnew[lane * 4 + d];
                } else {
                  const uint2 u = lds64(sa + kSlotBytes / 2 + (kk - k0) * (kHeadDim * 2) + lane * 8);
                  vx[0] = bf_lo(u.x);
                  vx[1] = bf_hi(u.x);
                  vx[2] = bf_lo(u.y);
                  vx[3] = bf_hi(u.y);
                }
#pragma unroll
                for (int d = 0; d < 4; ++d) {
                  a0[d] = fmaf(p0[i], vx[d], a0[d]);
                  a1[d] = fmaf(p1[i], vx[d], a1[d]);
                }
              }
            }
            ring_done(c, n);
          }
          tr.mark(kTrMark, kSubBCAttn, l, t);
#pragma unroll
          for (int d = 0; d < 4; ++d) {
            sm.u.att[warp][0][lane * 4 + d] = a0[d];
            sm.u.att[warp][1][lane * 4 + d] = a1[d];
          }
          if (lane == 0) {
            sm.u.att[warp][0][kHeadDim] = m0;
            sm.u.att[warp][0][kHeadDim + 1] = l0;
            sm.u.att[warp][1][kHeadDim] = m1;
            sm.u.att[warp][1][kHeadDim + 1] = l1;
          }
          consumer_sync(kConsumerThreads);
          if (tid < 2 * kHeadDim) {
            const int hh = tid >> 7, d = tid & (kHeadDim - 1);
            float M = -INFINITY;
#pragma unroll
            for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, sm.u.att[w][hh][kHeadDim]);
            float L = 0.f, O = 0.f;
#pragma unroll
            for (int w = 0; w < kConsumerWarps; ++w) {
              const float mw = sm.u.att[w][hh][kHeadDim];
              const float f = mw > -INFINITY ? exp2f(mw - M) : 0.f;
              L = fmaf(sm.u.att[w][hh][kHeadDim + 1], f, L);
              O = fmaf(sm.u.att[w][hh][d], f, O);
            }
            if (splits <= 1) {
              sm.attn[tid] = O / L;
            } else {
              float* dst = ws->att_part[h][pl.c][hh];
              dst[d] = O;
              if (d == 0) {
                dst[kHeadDim] = M;
                dst[kHeadDim + 1] = L;
              }
            }
          }
          consumer_sync(kConsumerThreads);
          if (splits > 1 && tid == 0) release_add(&ws->att_sync[l][h][0], 1u);
        }
        if (splits > 1) {
          transition_wait(c, tr, &ws->att_sync[l][h][0], static_cast<uint32_t>(splits * (t + 1)), l, kStSplit, t);
          if (tid < 2 * kHeadDim) {
            const int hh = tid >> 7, d = tid & (kHeadDim - 1);
            float M = -INFINITY;
            for (int s = 0; s < splits; ++s) M = fmaxf(M, __ldcg(&ws->att_part[h][s][hh][kHeadDim]));
            float L = 0.f, O = 0.f;
            for (int s = 0; s < splits; ++s) {
              const float ms = __ldcg(&ws->att_part[h][s][hh][kHeadDim]);
              const float f = ms > -INFINITY ? exp2f(ms - M) : 0.f;
              L = fmaf(__ldcg(&ws->att_part[h][s][hh][kHeadDim + 1]), f, L);
              O = fmaf(__ldcg(&ws->att_part[h][s][hh][d]), f, O);
            }
            sm.attn[tid] = O / L;
          }
          consumer_sync(kConsumerThreads);
        }

        // o_proj partial of this KV head's two Q heads (megakernel.cu:191-225)
        tr.mark(kTrMark, kSubBCComb, l, t);
        {
          // K = 256 (two heads x 128): warp w owns the MMA k-step [16w, 16w+16);
          // rows in padded 528-byte slots, four 16-row tiles per chunk.
          uint32_t ob0 = 0u, ob1 = 0u;
          if (lane < 8) {
            const int k = 16 * warp + 2 * (lane & 3);
            const float x0 = sm.attn[k], x1 = sm.attn[k + 1], x8 = sm.attn[k + 8], x9 = sm.attn[k + 9];
            const uint32_t h0 = pack_bf2(x0, x1), h1 = pack_bf2(x8, x9);
            ob0 = lane < 4 ? h0 : pack_bf2(x0 - bf_lo(h0), x1 - bf_hi(h0));
            ob1 = lane < 4 ? h1 : pack_bf2(x8 - bf_lo(h1), x9 - bf_hi(h1));
          }
          for (int o0 = pl.oa; o0 < pl.ob; o0 += kORowsPerChunk) {
            const int nrows = min(pl.ob, o0 + kORowsPerChunk) - o0;
            const uint32_t sa = ring_wait(c, n, l, 3, t, &tr);
            float d[4][4] = {};
            const int tr16 = lane & 15;
#pragma unroll
            for (int tt = 0; tt < 4; ++tt) {
              const int rr = tt * 16 + tr16;
              const uint32_t row = sa + (rr < nrows ? rr : 0) * kORowStride + (lane >> 4) * 16 + warp * 32;
              uint32_t a0, a1, a2, a3;
              ldsm_x4(row, a0, a1, a2, a3);
              mma_bf16(d[tt], a0, a1, a2, a3, ob0, ob1);
            }
            ring_done(c, n);
#pragma unroll
            for (int tt = 0; tt < 4; ++tt) stash_tile(xred, tt, d[tt]);
            consumer_sync(kConsumerThreads);
            if (tid < nrows) red_add_f32(&ws->acc_mid[l][o0 + tid], sum_warps(xred, tid));
            consumer_sync(kConsumerThreads);
          }
        }
        transition_publish(tr, &ws->sync[l][1][0], l, kStBC, t);
      }

      // ================= DE: post norm, SwiGLU rows, down partial ===============
      // the next layer's input-norm weights, one stage ahead of their use
      if (l + 1 < le) load_norm_k(lwt(c, l + 1, kWNorm), nwA);
      transition_wait(c, tr, &ws->sync[l][1][0], tgtBC, l, kStDE, t);
      {
        const float m0 = sm.r[tid] + __ldcg(&ws->acc_mid[l][tid]);
        const float m1 = sm.r[tid + kConsumerThreads] + __ldcg(&ws->acc_mid[l][tid + kConsumerThreads]);
        sm.rmid[tid] = m0;
        sm.rmid[tid + kConsumerThreads] = m1;
        const float tot = block_sumsq(m0, m1, sm.red, flip);
        build_bfrag(sm.rmid, rsqrtf(tot * (1.0f / kHidden) + kEps), nwD, bfr);
      }
      tr.mark(kTrMark, kSubDENorm, l, t);
      const int nj = pl.jb - pl.ja;
      // gate and up rows (megakernel.cu:100-142): each padded chunk holds 7 of
      // each and is one 16-row MMA tile; up to three chunks per pass
      for (int jb0 = 0; jb0 < nj; jb0 += 3 * kGUPerChunk) {
        const int ng = min(3, (nj - jb0 + kGUPerChunk - 1) / kGUPerChunk);
        uint32_t sa[3];
        ring_wait_all(c, n, ng, sa, l, 4, t, &tr);
        float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f}, d2[4] = {0.f, 0.f, 0.f, 0.f};
        mma_tile_gu(sa[0], min(kGUPerChunk, nj - jb0), bfr, d0);
        if (ng > 1) mma_tile_gu(sa[1], min(kGUPerChunk, nj - jb0 - kGUPerChunk), bfr, d1);
        if (ng > 2) mma_tile_gu(sa[2], min(kGUPerChunk, nj - jb0 - 2 * kGUPerChunk), bfr, d2);
        ring_done_all(c, n, ng);
        stash_tile(xred, 0, d0);
        stash_tile(xred, 1, d1);
        stash_tile(xred, 2, d2);
        consumer_sync(kConsumerThreads);
        if (tid < 16 * ng) {
          const int i = (tid & 15) & 7;
          const int j = jb0 + (tid >> 4) * kGUPerChunk + i;
          if (i < kGUPerChunk && j < nj) sm.gu[(tid & 15) >> 3][j] = sum_warps(xred, tid);
        }
        consumer_sync(kConsumerThreads);
      }
      tr.mark(kTrMark, kSubDEGU, l, t);
      if (tid < nj) {
        const float g = sm.gu[0][tid], u = sm.gu[1][tid];
        sm.m[tid] = g / (1.0f + expf(-g)) * u;  // silu (config.cuh:177-179) * up
      }
      consumer_sync(kConsumerThreads);
      if (fused) {
        // down-proj partial over this CTA's intermediate rows: warp w owns
        // outputs [64w, 64w+64), two per lane (megakernel.cu:53-90, split by K)
        const int col = warp * 64 + lane * 2;
        float pa = 0.f, pb = 0.f;
        for (int jb0 = 0; jb0 < nj; jb0 += 3 * kRowsPerChunk1024) {
          const int nd = min(3, (nj - jb0 + kRowsPerChunk1024 - 1) / kRowsPerChunk1024);
          uint32_t sa[3];
          ring_wait_all(c, n, nd, sa, l, 5, t, &tr);
          for (int i = 0; i < nd; ++i) {
            const int js = jb0 + i * kRowsPerChunk1024;
            const int j1 = min(nj, js + kRowsPerChunk1024);
            for (int jj = js; jj < j1; ++jj) {
              const uint32_t w = lds32(sa[i] + (jj - js) * 2048 + col * 2);
              const float mj = sm.m[jj];
              pa = fmaf(bf_lo(w), mj, pa);
              pb = fmaf(bf_hi(w), mj, pb);
            }
          }
          ring_done_all(c, n, nd);
        }
        tr.mark(kTrMark, kSubDEDown, l, t);
        red_add_v2_f32(&ws->acc_down[l][col], pa, pb);
        transition_publish(tr, &ws->sync[l][2][0], l, kStDE, t);
      } else {
        // reference layout: publish the SwiGLU vector, then whole down rows
        for (int j = tid; j < nj; j += kConsumerThreads) p.mlp_out[pl.ja + j] = sm.m[j];
        transition_publish(tr, &ws->sync[l][2][0], l, kStDE, t);
        transition_wait(c, tr, &ws->sync[l][2][0], tgtG, l, kStE, t);
        for (int i = tid; i < kInter; i += kConsumerThreads) sm.u.x[i] = __ldcg(p.mlp_out + i);
        consumer_sync(kConsumerThreads);
        for (int d0 = pl.da; d0 < pl.db; d0 += kDownRowsPerChunk) {
          const int d1 = min(pl.db, d0 + kDownRowsPerChunk);
          const uint32_t sa = ring_wait(c, n, l, 6, t, &tr);
          const int row = warp / 3, third = warp % 3;
          if (warp < 15 && d0 + row < d1) {
            float acc = 0.f;
#pragma unroll
            for (int g = 0; g < 4; ++g) {
              const int e = third * kHidden + lane * 8 + g * 256;
              const uint4 w = lds128(sa + row * (kInter * 2) + e * 2);
              acc += dot8(w, sm.u.x + e);
            }
            acc = warp_sum(acc);
            if (lane == 0) sm.dpart[row][third] = acc;
          }
          ring_done(c, n);
          consumer_sync(kConsumerThreads);
          if (tid < d1 - d0) {
            const int d = d0 + tid;
            ws->resid[d] = sm.rmid[d] + (sm.dpart[tid][0] + sm.dpart[tid][1] + sm.dpart[tid][2]);
          }
          consumer_sync(kConsumerThreads);
        }
        transition_publish(tr, &ws->sync[l][3][0], l, kStE, t);
      }
    }

    // ================= final residual, LM head + argmax (megakernel.cu:870-886) ==
    uint4 fwv[4];
    load_norm_w((p.flags & kFlagSkipFinalNorm) ? nullptr : p.final_norm, fwv);
    if (le > lb) {
      transition_wait(c, tr, &ws->sync[le - 1][fused ? 2 : 3][0], tgtG, le - 1, kStLM, t);
      if (fused) {
        r0 = sm.rmid[tid] + __ldcg(&ws->acc_down[le - 1][tid]);
        r1 = sm.rmid[tid + kConsumerThreads] + __ldcg(&ws->acc_down[le - 1][tid + kConsumerThreads]);
      } else {
        r0 = __ldcg(&ws->resid[tid]);
        r1 = __ldcg(&ws->resid[tid + kConsumerThreads]);
      }
    }
    sm.r[tid] = r0;
    sm.r[tid + kConsumerThreads] = r1;
    if (c.cta == 0 && p.residual_out != nullptr && t == p.n_tokens - 1) {
      p.residual_out[tid] = r0;
      p.residual_out[tid + kConsumerThreads] = r1;
    }
    float bv = -INFINITY;
    int bi = INT_MAX;
    if (p.flags & kFlagLmHead) {
      const float tot = block_sumsq(r0, r1, sm.red, flip);
      const float rstd = (p.flags & kFlagSkipFinalNorm) ? 1.0f : rsqrtf(tot * (1.0f / kHidden) + kEps);
      xr_from(sm.r, rstd, fwv, xr);
      for (int v0 = pl.va; v0 < pl.vb; v0 += kRowsPerChunk1024) {
        const int v1 = min(pl.vb, v0 + kRowsPerChunk1024);
        const uint32_t sa = ring_wait(c, n, -1, 8, t, &tr);
        const int row = v0 + warp;
        if (row < v1) {
          const float v = warp_sum(dot_row1024(sa + warp * 2048, xr, lane));
          if (lane == 0 && p.logits != nullptr) p.logits[row] = v;
          if (better(v, row, bv, bi)) {
            bv = v;
            bi = row;
          }
        }
        ring_done(c, n);
      }
      if (lane == 0) {
        sm.best_v[warp] = bv;
        sm.best_i[warp] = bi;
      }
      consumer_sync(kConsumerThreads);
      if (tid == 0) {
        for (int w = 0; w < kConsumerWarps; ++w)
          if (better(sm.best_v[w], sm.best_i[w], bv, bi)) {
            bv = sm.best_v[w];
            bi = sm.best_i[w];
          }
        ws->cand_val[c.cta] = bv;
        ws->cand_idx[c.cta] = bi;
      }
    }
    // ---- end of token: the last CTA to arrive reduces the argmax and resets ---
    tr.mark(kTrMark, kStLM, 0, t);
    consumer_sync(kConsumerThreads);
    if (tid == 0) {
      // One thread decides for the whole CTA, so every consumer takes the same path.
      if (aborted(c)) {
        sm.is_last = -1;
      } else {
        uint32_t old;
        asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(old) : "l"(&ws->arrive[0]) : "memory");
        sm.is_last = (old == tgtG - 1u) ? 1 : 0;
      }
    }
    consumer_sync(kConsumerThreads);
    const int last_state = sm.is_last;
    consumer_sync(kConsumerThreads);
    tr.mark(kTrMark, kStEnd, 0, t);
    if (last_state < 0) return;
    if (last_state) {
      int best = -1;
      if (p.flags & kFlagLmHead) {
        float v = -INFINITY;
        int i = INT_MAX;
        if (tid < G) {
          v = __ldcg(&ws->cand_val[tid]);
          i = __ldcg(&ws->cand_idx[tid]);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          const float ov = __shfl_xor_sync(0xffffffffu, v, o);
          const int oi = __shfl_xor_sync(0xffffffffu, i, o);
          if (better(ov, oi, v, i)) {
            v = ov;
            i = oi;
          }
        }
        if (lane == 0) {
          sm.best_v[warp] = v;
          sm.best_i[warp] = i;
        }
        consumer_sync(kConsumerThreads);
        if (tid == 0) {
          v = sm.best_v[0];
          i = sm.best_i[0];
          for (int w = 1; w < kConsumerWarps; ++w)
            if (better(sm.best_v[w], sm.best_i[w], v, i)) {
              v = sm.best_v[w];
              i = sm.best_i[w];
            }
          best = i;
        }
      }
      // the last two layers' accumulators (earlier ones were cleared on the way)
      for (int i = tid; i < kHidden; i += kConsumerThreads) {
        for (int l = max(lb, le - 2); l < le; ++l) {
          ws->acc_mid[l][i] = 0.f;
          ws->acc_down[l][i] = 0.f;
        }
      }
      const bool last_tok = t == p.n_tokens - 1;
      if (last_tok) {
        for (int i = tid; i < kMaxLayers * 4; i += kConsumerThreads) ws->sync[i >> 2][i & 3][0] = 0u;
        for (int i = tid; i < kMaxLayers * kNKV; i += kConsumerThreads) ws->att_sync[i / kNKV][i % kNKV][0] = 0u;
      }
      consumer_sync(kConsumerThreads);
      if (tid == 0) {
        if (p.flags & kFlagLmHead) {
          if (p.out_tokens != nullptr) p.out_tokens[t] = best;
          if (p.step != nullptr && (p.flags & kFlagAdvanceStep)) {
            p.step[0] = best;
            p.step[1] = pos + 1;
            p.step[3] += 1;
          }
        }
        if (last_tok) {
          ws->arrive[0] = 0u;
          ws->tok_flag[0] = 0u;
          ws->tag_base[0] = tag0 + static_cast<uint32_t>(p.n_tokens);
        } else {
          ws->tok_flag[1] = static_cast<uint32_t>(best);
          __threadfence();
          st_release(&ws->tok_flag[0], static_cast<uint32_t>(t + 1));
        }
      }
    }
  }
}


__global__ void __launch_bounds__(kThreads, 1) decode_kernel(const DecodeParams p) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  Smem* sm = reinterpret_cast<Smem*>(smem_raw);
  Ctl c{sm, p.ws, p.timeout_ns, static_cast<int>(blockIdx.x),
        p.trace ? p.trace + (size_t)blockIdx.x * p.trace_cap : nullptr, p.trace_cap};

  int token = p.token, pos = p.position, cl = p.cache_len;
  const uint32_t tag0 = __ldcg(&p.ws->tag_base[0]);
  if (p.step != nullptr) {
    token = __ldcg(p.step + 0);
    pos = __ldcg(p.step + 1);
    cl = pos + 1;
  }

  for (int i = threadIdx.x; i < kMaxLayers * 12; i += blockDim.x) {
    const int l = i / 12, f = i % 12;
    const __nv_bfloat16* v = nullptr;
    if (l >= p.layer_begin && l < p.layer_end) {
      if (f < 11) v = reinterpret_cast<const __nv_bfloat16* const*>(p.layers + l)[f];
      else if (p.down_t != nullptr) v = p.down_t[l];
    }
    sm->lwp[l][f] = v;
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < kSlots; ++s) {
      mbar_init(&sm->full[s], 1);
      mbar_init(&sm->empty[s], kConsumerWarps);
    }
    sm->abort = 0;
    sm->is_last = 0;
    fence_mbar_init();
  }
  __syncthreads();

  // Attention splits: fixed for the launch, from its longest cache (the step
  // state may supply the position, so this is decided on the device).
  const int last_cl = cl + p.n_tokens - 1;
  const int splits = p.splits > 0 ? p.splits : choose_splits(last_cl, p.group_size);
  // Argument guard (uniform over the grid, before any wait).
  if (token < 0 || token >= kVocab || pos < 0 || pos + p.n_tokens > p.max_seq || cl < 1 ||
      last_cl > p.max_seq || p.grid != static_cast<int>(gridDim.x) || p.grid > kMaxGrid ||
      p.group_size * kNKV > p.grid || splits < 1 || splits > kMaxSplits ||
      (splits > 1 && splits > p.group_size)) {
    if (threadIdx.x == 0 && blockIdx.x == 0) raise_error(c, kErrBadArgs, -1, -1, -1);
    return;
  }

  const Plan pl = make_plan(blockIdx.x, p.grid, p.group_size, kVocab);
  if (threadIdx.x >= kConsumerThreads) {
    producer_run(p, pl, c, pos, cl, splits);
  } else {
    consumer_run(p, pl, c, token, pos, cl, splits, tag0);
  }
}

// ---- host-side launch ----------------------------------------------------------
cudaError_t launch_decode(const DecodeParams& p, cudaStream_t stream) {
  static int configured[64] = {0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 64 && !configured[dev]) {
    e = cudaFuncSetAttribute(decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kSmemBytes));
    if (e != cudaSuccess) return e;
    configured[dev] = 1;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, decode_kernel, p);
}

size_t decode_smem_bytes() { return kSmemBytes; }

}  // namespace mkb
