// Persistent single-launch batch-one Qwen3-0.6B decode kernel for sm_100a.
//
// Structure (one CTA per SM, clusters of 2 CTAs, 9 warps):
//   * warp 8 (producer) walks this CTA's fixed chunk schedule for the whole
//     launch and streams every weight byte (and the KV rows that do not depend
//     on the current token) into a 6 x 32 KB shared-memory ring with 1-D bulk
//     async copies (cp.async.bulk, completion on mbarriers). It never waits on
//     a grid transition (except a one-off acquire before re-reading KV rows in a
//     multi-token launch), so HBM keeps streaming while the consumers wait.
//   * warps 0-7 (consumers) run the stages of each layer and hand off between
//     CTAs through the workspace without grid barriers or fences:
//        A  : input RMSNorm + QKV GEMV rows -> tagged words (value | tag)
//        BC : q/k RMSNorm + RoPE + KV append, GQA decode attention,
//             o_proj partial of this KV head -> counted fixed-point
//             red.add into acc_mid (complete when 8 heads have added)
//        DE : post RMSNorm + gate/up SwiGLU rows, SwiGLU values swapped with
//             the cluster partner (st.async), down partial of this CTA's 512
//             output columns over both CTAs' rows of the transposed down
//             weight (mma.sync, ldmatrix.trans) -> counted red.add into
//             acc_down (complete at G/2 adds)
//        (reference-layout down weight: D writes the SwiGLU vector and
//         publishes a counter, E computes whole down rows and writes the
//         residual, then publishes the next counter)
//     then final RMSNorm + tied LM head + block/grid argmax.
// Every wait is bounded by DecodeParams::timeout_ns; on expiry the kernel
// records an error in Workspace::error, stops issuing copies, drains the ones in
// flight and returns, so the host gets a status instead of a hang.
//
// Reference: megakernel.cu:744-893 (decode_kernel) and the stage functions it
// calls (megakernel.cu:9-739); see the per-stage comments below.

#include <cfloat>
#include <cstddef>
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
  // One phase per layer: this CTA's own arrival (with the expected byte count)
  // plus the cluster partner's SwiGLU values, each landing with complete_tx.
  uint64_t rxbar;
  // The same for the attention partials of the partner's half of the keys.
  uint64_t atbar;
  alignas(16) float r[kHidden];      // residual entering the current layer
  alignas(16) float rmid[kHidden];   // residual after attention + o_proj
  alignas(16) union {
    float att[kConsumerWarps][2][kHeadDim + 4];  // per-warp attention partials
    float xred[kConsumerWarps][64];              // per-warp GEMV row partials
    float x[kInter];                             // SwiGLU vector (reference-layout down)
  } u;
  // Normalised activation of the current GEMV stage as BF16 high part and
  // remainder (MMA B operand columns 0 and 1).
  alignas(16) __nv_bfloat16 xh[kHidden];
  alignas(16) __nv_bfloat16 xl[kHidden];
  alignas(16) float q[2][kHeadDim];  // rotated, pre-scaled queries of this KV head's two Q heads
  alignas(16) float knew[kHeadDim];  // rotated new key (BF16-rounded)
  alignas(16) float vnew[kHeadDim];  // new value (BF16-rounded)
  alignas(16) float attn[2 * kHeadDim];
  alignas(16) float m[32];
  alignas(16) float mrx[32];  // the cluster partner's SwiGLU values (down projection)
  alignas(16) float apeer[2][kHeadDim + 4];  // the partner's attention partial: o[128], m, l per head
  alignas(16) float pbuf[kConsumerWarps][16];  // attention weights exchanged within a warp
  alignas(16) float2 split_ml[2][kMaxSplits];   // m and l of every attention split (per Q head)
  float red[2 * kConsumerWarps];
  float best_v[kConsumerWarps];
  int best_i[kConsumerWarps];
  // Copy of the device LayerWeights table (+ the transposed down pointer) in
  // shared memory: grid-transition acquires invalidate L1, and these pointers
  // are needed on the critical path of every stage.
  const __nv_bfloat16* lwp[kMaxLayers][12];
  unsigned long long tbuf[kTraceSmem];  // trace staging (traced instantiation only)
  int token;
  int is_last;
  int abort;
  int peer_gone;  // set by the cluster partner when it leaves the token loop early
};

constexpr size_t kSmemBytes = sizeof(Smem);
static_assert(offsetof(Smem, r) % 16 == 0 && offsetof(Smem, rmid) % 16 == 0 && offsetof(Smem, u) % 16 == 0 &&
                  offsetof(Smem, xh) % 16 == 0 && offsetof(Smem, q) % 16 == 0 && offsetof(Smem, pbuf) % 16 == 0,
              "vector-accessed shared arrays must be 16-byte aligned");
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
  uint32_t* err_flag;         // copy of the error code for the host (or null)
};

// Stage time stamps of consumer thread 0, compiled in only for the traced
// instantiation. Stamps go to a shared-memory buffer (a global store per stamp
// would queue behind the bulk copies and slow the stage being measured) and are
// written to the CTA's trace row at the end of each token. Stamps are kept for
// layers [kTraceLayerLo, kTraceLayerLo + kTraceLayers) and the token-level marks.
template <bool kOn>
struct Tracer {
  unsigned long long* row;   // global trace row of this CTA (or null)
  unsigned long long* sbuf;  // shared-memory staging buffer
  int cap;                   // entries of `row`
  int n;                     // entries staged in sbuf
  int base;                  // entries already written to `row`
  __device__ __forceinline__ void mark(uint32_t kind, uint32_t stage, int layer, int tok) {
    if (kOn && row != nullptr && threadIdx.x == 0 && n < kTraceSmem &&
        ((layer >= kTraceLayerLo && layer < kTraceLayerLo + kTraceLayers) || stage == kStLM ||
         stage == kStToken || stage == kStEnd)) {
      const uint64_t code = kind | ((stage & 31u) << 2) | ((static_cast<uint32_t>(layer) & 31u) << 7) |
                            ((static_cast<uint32_t>(tok) & 15u) << 12);
      sbuf[n++] = (code << 48) | (global_ns() & 0xffffffffffffull);
    }
  }
  __device__ __forceinline__ void flush() {
    if (kOn && row != nullptr && threadIdx.x == 0) {
      for (int i = 0; i < n && base + i < cap; ++i) row[base + i] = sbuf[i];
      base += n;
      n = 0;
    }
  }
};

__device__ __forceinline__ bool aborted(const Ctl& c) {
  return *reinterpret_cast<volatile int*>(&c.sm->abort) != 0;
}

__device__ __noinline__ void raise_error(const Ctl c, uint32_t code, int layer, int stage, int tok) {
  if (atomicCAS(&c.ws->error[0], 0u, code) == 0u) {
    c.ws->error[1] = static_cast<uint32_t>(c.cta);
    c.ws->error[2] = static_cast<uint32_t>(layer);
    c.ws->error[3] = static_cast<uint32_t>(stage);
    c.ws->error[4] = static_cast<uint32_t>(tok);
    // the first error also goes to the caller's flag (pinned host memory for the
    // launchers), which the host reads without a copy
    if (c.err_flag != nullptr) *reinterpret_cast<volatile uint32_t*>(c.err_flag) = code;
  }
  *reinterpret_cast<volatile int*>(&c.sm->abort) = 1;
}

// Bounded spin until *ctr >= target (wrap-safe). Single thread.
__device__ __noinline__ void spin_geq(const Ctl c, const uint32_t* ctr, uint32_t target, uint32_t code,
                                      int layer, int stage, int tok) {
  if (aborted(c)) return;
  if (static_cast<int>(ld_acquire(ctr) - target) >= 0) return;
  const uint64_t t0 = global_ns();
  uint32_t it = 0;
  while (true) {
    if (static_cast<int>(ld_acquire(ctr) - target) >= 0) return;
    if ((++it & 15u) == 0u) {
      if (aborted(c)) return;  // also set when the launch stops on a stop token
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

// Bounded wait for token t's broadcast (sequence >= target in the low half of
// the packed word); returns the token id it carries (-1 when the wait gave up).
__device__ __noinline__ int spin_token(const Ctl c, const uint64_t* w, uint32_t target, int tok) {
  const uint64_t t0 = global_ns();
  uint32_t it = 0;
  while (true) {
    const uint64_t v = ld_acquire_u64(w);
    if (static_cast<int>(static_cast<uint32_t>(v) - target) >= 0) return static_cast<int>(v >> 32);
    if ((++it & 15u) == 0u) {
      if (aborted(c)) return -1;
      if (ld_relaxed(&c.ws->error[0]) != 0u) {
        *reinterpret_cast<volatile int*>(&c.sm->abort) = 1;
        return -1;
      }
      if (global_ns() - t0 > c.timeout) {
        raise_error(c, kErrTimeoutToken, -1, 9, tok);
        return -1;
      }
    }
  }
}
__device__ __forceinline__ uint64_t tok_word(int t, int token) {
  return (static_cast<uint64_t>(static_cast<uint32_t>(token)) << 32) | static_cast<uint32_t>(t + 1);
}

// The tag base the next launch starts from (one thread, at the end of a launch,
// when no CTA reads tagged words any more). The split-attention tags carry the
// layer in their low 5 bits ((tag << 5) | layer), so they would repeat after
// 2^27 tokens; long before that every tagged word is cleared and the tags
// restart, so a stale word can never carry a current tag (once per 2^26 tokens,
// a few hundred microseconds).
constexpr uint32_t kTagRestart = 1u << 26;
__device__ __noinline__ uint32_t next_tag_base(Workspace* ws, uint32_t next) {
  if (next < kTagRestart) return next;
  ulonglong2* a = reinterpret_cast<ulonglong2*>(&ws->qkv_tagged[0][0]);
  for (size_t i = 0; i < sizeof(ws->qkv_tagged) / sizeof(ulonglong2); ++i) a[i] = make_ulonglong2(0ull, 0ull);
  ulonglong2* b = reinterpret_cast<ulonglong2*>(&ws->att_part[0][0][0][0]);
  for (size_t i = 0; i < sizeof(ws->att_part) / sizeof(ulonglong2); ++i) b[i] = make_ulonglong2(0ull, 0ull);
  return 0u;
}

// spin_geq on a counter that other GPUs add into (tensor parallel).
__device__ __noinline__ void spin_geq_sys(const Ctl c, const uint32_t* ctr, uint32_t target, uint32_t code,
                                          int layer, int stage, int tok) {
  if (aborted(c)) return;
  const uint64_t t0 = global_ns();
  uint32_t it = 0;
  while (static_cast<int>(ld_acquire_sys(ctr) - target) < 0) {
    if ((++it & 15u) == 0u) {
      if (aborted(c)) return;
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

// Serve mode: bounded wait (the launch's timeout) for the host's request of
// token t in mapped pinned memory: {seq, token} with seq == t + 1, read as one
// 8-byte word (the host writes it as one), so a poll that sees the sequence
// number also has the token: one PCIe round trip. One thread.
__device__ __noinline__ int host_token(const Ctl c, volatile int* mailbox, int t) {
  const uint64_t t0 = global_ns();
  uint32_t it = 0;
  while (true) {
    uint64_t w;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(mailbox) : "memory");
    if (static_cast<int>(static_cast<uint32_t>(w)) == t + 1) return static_cast<int>(static_cast<uint32_t>(w >> 32));
    if ((++it & 15u) == 0u) {
      if (aborted(c)) return -1;
      if (ld_relaxed(&c.ws->error[0]) != 0u) {
        *reinterpret_cast<volatile int*>(&c.sm->abort) = 1;
        return -1;
      }
      if (global_ns() - t0 > c.timeout) {
        raise_error(c, kErrTimeoutToken, -1, kStToken, t);
        return -1;
      }
    }
  }
}

// Consumer-side transition: thread 0 waits, then all consumers proceed.
template <class TR>
__device__ __forceinline__ void transition_wait(const Ctl& c, TR& tr, const uint32_t* ctr, uint32_t target,
                                                int layer, int stage, int tok) {
  tr.mark(kTrWaitBegin, stage, layer, tok);
  if (threadIdx.x == 0) spin_geq(c, ctr, target, kErrTimeoutTransition, layer, stage, tok);
  consumer_sync(kConsumerThreads);
  tr.mark(kTrWaitEnd, stage, layer, tok);
}

// Consumer-side publish: every consumer's writes are ordered before the add.
template <class TR>
__device__ __forceinline__ void transition_publish(TR& tr, uint32_t* ctr, int layer, int stage, int tok) {
  consumer_sync(kConsumerThreads);
  if (threadIdx.x == 0) release_add(ctr, 1u);
  tr.mark(kTrPublish, stage, layer, tok);
}

// ---- ring (consumer side) ----------------------------------------------------
// Bounded hardware-suspended wait on an mbarrier phase (out of line: the
// fast path is a single test at each call site).
__device__ __noinline__ void mbar_wait_bounded(const Ctl c, uint64_t* bar, uint32_t ph, int layer, int stage,
                                               int tok) {
  const uint64_t t0 = global_ns();
  while (!mbar_wait(bar, ph, kSuspendNs)) {
    if (aborted(c)) break;
    if (global_ns() - t0 > c.timeout) {
      raise_error(c, kErrTimeoutRing, layer, stage, tok);
      break;
    }
  }
}

template <class TR = Tracer<false>>
__device__ __forceinline__ uint32_t ring_wait(const Ctl& c, uint32_t n, int layer, int stage, int tok,
                                              TR* tr = nullptr) {
  const int s = static_cast<int>(n % kSlots);
  const uint32_t ph = (n / kSlots) & 1u;
  if (!mbar_test(&c.sm->full[s], ph)) {
    if (tr) tr->mark(kTrWaitBegin, kStRing, layer, tok);
    mbar_wait_bounded(c, &c.sm->full[s], ph, layer, stage, tok);
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

// One 64-bit key per argmax candidate whose unsigned order is better()'s order:
// order-preserving bits of the value (every NaN as one value above +inf, -0 as
// +0) over the complement of the index (first index on ties).
__device__ __forceinline__ unsigned long long argmax_key(float v, int i) {
  uint32_t u = v != v ? 0x7fc00000u : (v == 0.f ? 0u : __float_as_uint(v));
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return (static_cast<unsigned long long>(u) << 32) | (0xffffffffu - static_cast<uint32_t>(i));
}
__device__ __forceinline__ int argmax_key_index(unsigned long long k) {
  return static_cast<int>(0xffffffffu - static_cast<uint32_t>(k & 0xffffffffull));
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

  __device__ Producer(const Ctl& ctl) : c(ctl), n(0), stop(false) {
    lane = threadIdx.x & 31;
    pol_w = policy_evict_first();
    pol_kv = policy_evict_last();
  }

  // Reserve the next slot for `bytes`; returns its index or -1 once stopped.
  __device__ int begin(uint32_t bytes) {
    if (stop) return -1;
    const int s = static_cast<int>(n % kSlots);
    const uint32_t ph = ((n / kSlots) & 1u) ^ 1u;
    int ok = 1;
    if (lane == 0) {
      if (!mbar_test(&c.sm->empty[s], ph)) {
        const uint64_t t0 = global_ns();
        while (!mbar_wait(&c.sm->empty[s], ph, kSuspendNs)) {
          if (aborted(c)) { ok = 0; break; }
          if (global_ns() - t0 > c.timeout) {
            raise_error(c, kErrTimeoutRing, -1, -1, -1);
            ok = 0;
            break;
          }
        }
      }
      if (ok && aborted(c)) ok = 0;
      if (ok) mbar_arrive_expect_tx(&c.sm->full[s], bytes);
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

template <bool kFused, bool kTraced, bool kTP>
__device__ void producer_run(const DecodeParams& p, const Plan& pl, const Ctl& c, int pos0, int cl0,
                             int splits0) {
  Producer pr(c);
  const TpShape tp = tp_shape(kTP ? p.tp_rank : 0, kTP ? p.tp_size : 1, kVocab);
  const bool pair_attn = pair_shares_head(static_cast<int>(blockIdx.x), p.grid, p.group_size, tp);
  for (int t = 0; t < p.n_tokens && !pr.stop; ++t) {
    const int pos = pos0 + t;
    const int cl = cl0 + t;
    const int splits = splits0 > 0 ? splits0 : choose_splits(cl, p.group_size);
    for (int l = p.layer_begin; l < p.layer_end && !pr.stop; ++l) {
      // A: QKV rows, one bulk copy per row into a padded row slot
      for (int r = pl.qa; r < pl.qb;) {
        const int e = qkv_chunk_end(r, pl.qb, tp);
        const int g = qkv_global_row(tp, r);  // rows of a chunk are contiguous in [Wq; Wk; Wv]
        const __nv_bfloat16* src = g < kQSize ? lwt(pr.c, l, kWQ) + (size_t)g * kHidden
                                   : g < kQSize + kKVSize
                                       ? lwt(pr.c, l, kWK) + (size_t)(g - kQSize) * kHidden
                                       : lwt(pr.c, l, kWV) + (size_t)(g - kQSize - kKVSize) * kHidden;
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
        attn_keys(cl, splits, pl.c, pair_attn, static_cast<int>(cluster_ctarank()), &ka, &kb);
        if (t > 0 && kb > ka && pr.lane == 0) {
          // The previous token of this launch appended K/V at pos-1; make it
          // visible to the bulk-copy engine before re-reading those rows.
          spin_geq(c, &p.ws->kv_ready[l][pl.h][0], 2u * static_cast<uint32_t>(t), kErrTimeoutTransition, l, 10, t);
          fence_proxy_async_global();
        }
        // this GPU's cache shard holds its tp.hl heads
        const size_t head_off = ((size_t)l * tp.hl + pl.hl) * (size_t)p.max_seq * kHeadDim;
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
      if constexpr (kFused) {
        // this CTA's column block of the transposed down weight: its own rows,
        // then its cluster partner's rows (one slot each)
        const uint32_t rank = cluster_ctarank();
        const __nv_bfloat16* wdt = lwt(pr.c, l, kWDownT) + (size_t)rank * kInter * kSlice;
        const Plan pp = make_plan(static_cast<int>(blockIdx.x ^ 1u), p.grid, p.group_size, tp);
        const int rows[2][2] = {{pl.ja, pl.jb}, {pp.ja, pp.jb}};
        for (int q = 0; q < 2; ++q) {
          const int nr = rows[q][1] - rows[q][0];
          const int s = pr.begin(static_cast<uint32_t>(nr) * kSlice * 2u);
          if (s < 0) break;
          // one copy per row into kDRowStride-padded rows (ldmatrix.trans reads)
          if (pr.lane < nr)
            pr.copy(s, static_cast<uint32_t>(pr.lane) * kDRowStride, wdt + (size_t)(rows[q][0] + pr.lane) * kSlice,
                    kSlice * 2u, pr.pol_w);
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
    // LM-head rows (prefill: for the last prompt token only)
    if ((p.flags & kFlagLmHead) && (p.prompt == nullptr || t == p.n_tokens - 1)) {
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
//
// Vector ownership: consumer thread i owns elements [kE*i, kE*i + kE) of every
// 1024-vector (residual, accumulators, norm weights).

// ---- tensor-core GEMV over padded rows in a ring slot -------------------------
// Warp w owns the reduction range k in [kKPerWarp*w, kKPerWarp*(w+1)) of a
// 1024-wide row (kKSteps 16-wide MMA k-steps); the warps' partial sums are added
// through shared memory. The activation enters as B columns 0 (BF16 high part)
// and 1 (BF16 remainder x - high), so D[:,0] + D[:,1] carries ~16 mantissa bits
// of x. Both parts are written once per stage into sm.xh / sm.xl.
constexpr int kE = kHidden / kConsumerThreads;       // elements per consumer thread
constexpr int kKPerWarp = kHidden / kConsumerWarps;  // GEMV k range per warp
constexpr int kKSteps = kKPerWarp / 16;
constexpr int kKeysPerWarp = kKeysPerChunk / kConsumerWarps;  // attention keys per warp and chunk
constexpr int kOSteps = 2 * kHeadDim / 16 / kConsumerWarps;   // o_proj k-steps per warp
static_assert(kE == 4, "the vector helpers below move 4 elements per thread");
static_assert(kKeysPerWarp == 8, "the attention butterfly reduces 2 x 8 scores per warp");
static_assert(kOSteps >= 1 && kKSteps >= 1, "warp count");

// This thread's 4 norm-weight elements (8 bytes, read-only path); issued a stage
// ahead of use.
__device__ __forceinline__ uint2 load_w4(const __nv_bfloat16* w) {
  if (w == nullptr) return make_uint2(0x3f803f80u, 0x3f803f80u);  // bf16 1.0 pairs
  return __ldg(reinterpret_cast<const uint2*>(w) + threadIdx.x);
}
// x = v * rstd * w for this thread's 4 elements, written as BF16 high part and
// remainder into sm.xh / sm.xl (8 bytes each).
__device__ __forceinline__ void store_x(Smem& sm, const float v[4], float rstd, uint2 w) {
  const float x0 = v[0] * rstd * bf_lo(w.x), x1 = v[1] * rstd * bf_hi(w.x);
  const float x2 = v[2] * rstd * bf_lo(w.y), x3 = v[3] * rstd * bf_hi(w.y);
  const uint32_t h01 = pack_bf2(x0, x1), h23 = pack_bf2(x2, x3);
  const uint32_t l01 = pack_bf2(x0 - bf_lo(h01), x1 - bf_hi(h01));
  const uint32_t l23 = pack_bf2(x2 - bf_lo(h23), x3 - bf_hi(h23));
  const int e = threadIdx.x * kE;
  *reinterpret_cast<uint2*>(&sm.xh[e]) = make_uint2(h01, h23);
  *reinterpret_cast<uint2*>(&sm.xl[e]) = make_uint2(l01, l23);
}
// B fragments of this warp's k-steps (lanes 0-3: high part, 4-7: remainder).
__device__ __forceinline__ void load_bfrag(const Smem& sm, uint32_t bfr[kKSteps][2]) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t base = smem_addr(lane < 4 ? sm.xh : sm.xl) + (kKPerWarp * warp + 2 * (lane & 3)) * 2;
#pragma unroll
  for (int st = 0; st < kKSteps; ++st) {
    bfr[st][0] = lane < 8 ? lds32(base + st * 32) : 0u;
    bfr[st][1] = lane < 8 ? lds32(base + st * 32 + 16) : 0u;
  }
}
// One 16-row tile of padded 1024-wide rows at `base`. A row past nrows reads row
// (tr & 7) instead, which sits in the same shared-memory banks as the row it
// stands for: padded rows r and r + 8 share banks, so aliasing row 15 to row 0
// (the earlier choice) put a 2-way bank conflict into every ldmatrix of the
// tile (≈240 cycles of a 2-tile pass, measured).
__device__ __forceinline__ void mma_tile_1024(uint32_t base, int nrows, const uint32_t bfr[kKSteps][2], float* d) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int tr = lane & 15;
  const uint32_t row = base + (tr < nrows ? tr : (tr & 7)) * kRowStride + (lane >> 4) * 16 + warp * (kKPerWarp * 2);
  float e[4] = {0.f, 0.f, 0.f, 0.f};  // second accumulator: two independent MMA chains
#pragma unroll
  for (int st = 0; st < kKSteps; ++st) {
    uint32_t a0, a1, a2, a3;
    ldsm_x4(row + st * 32, a0, a1, a2, a3);
    mma_bf16((st & 1) ? e : d, a0, a1, a2, a3, bfr[st][0], bfr[st][1]);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) d[i] += e[i];
}
// Gate/up tile: tile rows 0-6 are gate rows, 8-14 up rows (second slot half).
__device__ __forceinline__ void mma_tile_gu(uint32_t base, int nrows, const uint32_t bfr[kKSteps][2], float* d) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int tr = lane & 15, i = tr & 7;
  const uint32_t row = base + (tr >= 8 ? kSlotBytes / 2 : 0) + (i < nrows ? i : 0) * kRowStride + (lane >> 4) * 16 +
                       warp * (kKPerWarp * 2);
  float e[4] = {0.f, 0.f, 0.f, 0.f};  // second accumulator: two independent MMA chains
#pragma unroll
  for (int st = 0; st < kKSteps; ++st) {
    uint32_t a0, a1, a2, a3;
    ldsm_x4(row + st * 32, a0, a1, a2, a3);
    mma_bf16((st & 1) ? e : d, a0, a1, a2, a3, bfr[st][0], bfr[st][1]);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) d[i] += e[i];
}
// Down projection on the tensor cores: this warp's 64 output columns
// [64 w, 64 w + 64) of the CTA's kSlice block are four 16-column tiles (MMA M),
// the SwiGLU rows of one slot the reduction (MMA K: kDownKSteps steps of 16,
// rows >= nj masked because their slot bytes may be stale), m[] the B operand as
// BF16 high part (column 0) and remainder (column 1). The slot holds transposed
// down rows at kDRowStride bytes; ldmatrix.trans turns them into A fragments.
// Results accumulate into d (D columns 0 and 1 of each tile).
__device__ __forceinline__ void down_mma(uint32_t slot, const float* m, int nj, float (*d)[4]) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, tq = lane & 3, q = lane >> 3;
#pragma unroll
  for (int ks = 0; ks < kDownKSteps; ++ks) {
    const int k0 = 16 * ks;
    // this lane's ldmatrix row: matrices 0/1 rows k0.., 2/3 rows k0+8.., matrices
    // 1/3 eight columns on; rows past kMaxJ (always masked) read a row of the
    // same bank group inside the slot instead
    int kr = k0 + (lane & 7) + 8 * (q >> 1);
    if (kr >= kMaxJ) kr -= 8;
    const uint32_t arow = slot + static_cast<uint32_t>(kr * kDRowStride + (64 * warp + 8 * (q & 1)) * 2);
    uint32_t b0 = 0u, b1 = 0u;
    if (g < 2) {
      const float2 x01 = *reinterpret_cast<const float2*>(m + k0 + 2 * tq);
      const float2 x89 = *reinterpret_cast<const float2*>(m + k0 + 2 * tq + 8);
      const uint32_t h0 = pack_bf2(x01.x, x01.y), h8 = pack_bf2(x89.x, x89.y);
      b0 = g == 0 ? h0 : pack_bf2(x01.x - bf_lo(h0), x01.y - bf_hi(h0));
      b1 = g == 0 ? h8 : pack_bf2(x89.x - bf_lo(h8), x89.y - bf_hi(h8));
    }
    const int ka = k0 + 2 * tq;
    const uint32_t m01 = (ka < nj ? 0x0000ffffu : 0u) | (ka + 1 < nj ? 0xffff0000u : 0u);
    const uint32_t m89 = (ka + 8 < nj ? 0x0000ffffu : 0u) | (ka + 9 < nj ? 0xffff0000u : 0u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint32_t a0, a1, a2, a3;
      ldsm_x4_trans(arow + 32 * i, a0, a1, a2, a3);
      mma_bf16(d[i], a0 & m01, a1 & m01, a2 & m89, a3 & m89, b0, b1);
    }
  }
}
static_assert(kMaxJ > 8 * (kDownKSteps * 2 - 1) - 8 && kMaxJ <= 16 * kDownKSteps && kMaxJ <= 32 &&
                  kMaxJ * kDRowStride <= kSlotBytes && kSlice == 64 * kConsumerWarps,
              "down_mma: row redirect, m[] reads below 32, slot capacity, 64 columns per warp");

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
template <class TR>
__device__ __forceinline__ void ring_wait_all(const Ctl& c, uint32_t n, int cnt, uint32_t* sa, int layer, int stage,
                                              int tok, TR* tr) {
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

// Block-wide sum over the consumer threads of `v` (one named barrier; s_red
// alternates between two halves so no trailing barrier is needed).
__device__ __forceinline__ float block_sum(float v, float* s_red, int& flip) {
  const float ss = warp_sum(v);
  float* buf = s_red + (flip ? kConsumerWarps : 0);
  flip ^= 1;
  if ((threadIdx.x & 31) == 0) buf[threadIdx.x >> 5] = ss;
  consumer_sync(kConsumerThreads);
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < kConsumerWarps; ++i) tot += buf[i];
  return tot;
}

// RMSNorm feeding a GEMV stage with one barrier: x = v * w (without 1/rms)
// goes to sm.xh / sm.xl alongside this warp's sum of squares; after the barrier
// every thread adds the 8 warp sums and gets 1/rms, which scales the GEMV row
// sums instead of x (the GEMV is linear in x; the BF16 high/remainder split of x
// is scale-free). Same formula as megakernel.cu:704-739.
__device__ __forceinline__ float norm_to_x(Smem& sm, const float v[4], uint2 w, int& flip) {
  const float ss = warp_sum(v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3]);
  float* buf = sm.red + (flip ? kConsumerWarps : 0);
  flip ^= 1;
  if ((threadIdx.x & 31) == 0) buf[threadIdx.x >> 5] = ss;
  store_x(sm, v, 1.0f, w);
  consumer_sync(kConsumerThreads);
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < kConsumerWarps; ++i) tot += buf[i];
  return rsqrtf(tot * (1.0f / kHidden) + kEps);
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

// Bounded poll of two tagged words (16 bytes) until both carry `tag`.
__device__ __noinline__ ulonglong2 poll_tagged2_slow(const Ctl c, const uint64_t* p, uint32_t tag, int layer,
                                                    int tok) {
  uint64_t a = 0, b = 0;
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
  return make_ulonglong2(a, b);
}
__device__ __forceinline__ void poll_tagged2(const Ctl& c, const uint64_t* p, uint32_t tag, float& v0, float& v1,
                                             int layer, int tok) {
  uint64_t a, b;
  ld_tagged2(p, a, b);
  if (static_cast<uint32_t>(a >> 32) != tag || static_cast<uint32_t>(b >> 32) != tag) {
    const ulonglong2 w = poll_tagged2_slow(c, p, tag, layer, tok);
    a = w.x;
    b = w.y;
  }
  v0 = __uint_as_float(static_cast<uint32_t>(a));
  v1 = __uint_as_float(static_cast<uint32_t>(b));
}

// ---- counted fixed-point accumulators (layout in mkb_config.cuh) ---------------
// One contribution x: kAccOne + round(x * 2^28) + kAccBias. |x| >= 2^19 (or
// NaN) is clamped and flags `bad`.
__device__ __forceinline__ uint64_t acc_term(float x, bool& bad) {
  float s = x * 268435456.0f;
  constexpr float kLim = 140737488355000.0f;  // just below 2^47
  if (!(fabsf(s) < kLim)) {
    bad = true;
    s = s > 0.f ? kLim : -kLim;  // NaN clamps to the negative limit
  }
  return kAccOne + static_cast<uint64_t>(__float2ll_rn(s) + static_cast<long long>(kAccBias));
}
__device__ __forceinline__ float acc_decode(uint64_t low, uint64_t cnt) {
  const long long fixed = static_cast<long long>(low) - static_cast<long long>(cnt * kAccBias);
  return __ll2float_rn(fixed) * (1.0f / 268435456.0f);
}
// Sum carried by `copies` words at stride kHidden; `count` receives the number
// of contributions.
// `sys`: the words also receive other GPUs' contributions (tensor parallel).
__device__ __forceinline__ float acc_value(const uint64_t* w, int copies, uint32_t& count, bool sys = false) {
  uint64_t low = 0, cnt = 0;
  for (int q = 0; q < copies; ++q) {
    const uint64_t v = sys ? ld_relaxed_u64_sys(w + q * kHidden) : ld_relaxed_u64(w + q * kHidden);
    cnt += v >> 56;
    low += v & kAccLowMask;
  }
  count = static_cast<uint32_t>(cnt);
  return acc_decode(low, cnt);
}
// Bounded poll by one thread until elements e0 and e1 of an accumulator row
// (e1 < 0: e0 only) both hold `expect` contributions; both are loaded in every
// round, so the second costs no extra round trip.
__device__ __noinline__ void acc_wait_pair(const Ctl c, const uint64_t* row, int copies, uint32_t expect, int e0,
                                           int e1, int layer, int stage, int tok, bool sys) {
  const uint64_t t0 = global_ns();
  uint32_t it = 0;
  while (true) {
    uint32_t n0 = 0, n1 = expect;
    acc_value(row + e0, copies, n0, sys);
    if (e1 >= 0) acc_value(row + e1, copies, n1, sys);
    if (n0 == expect && n1 == expect) break;
    if ((++it & 15u) == 0u) {
      if (aborted(c) || ld_relaxed(&c.ws->error[0]) != 0u) {
        *reinterpret_cast<volatile int*>(&c.sm->abort) = 1;
        break;
      }
      if (global_ns() - t0 > c.timeout) {
        raise_error(c, kErrTimeoutTransition, layer, stage, tok);
        break;
      }
    }
  }
}
// This thread's 4 elements of a [copies][kHidden] accumulator row, each
// complete with `expect` contributions in total. One thread of the CTA polls a
// sentinel element of copy 0 (complete at `expect0` contributions), a thread of
// another warp the same element of copy 1 when there is one, and the others
// wait at a barrier: every poll competes with the atomics landing on the same
// L2 lines, so the fewer poll loads the faster the exchange (measured).
// Elements still incomplete after the barrier are polled by their owners, all
// four together (one round trip per poll, not one per element).
__device__ __noinline__ void acc_wait4_slow(const Ctl c, const uint64_t* w, int copies, uint32_t expect, float* v,
                                            int layer, int stage, int tok, bool sys) {
  const uint64_t t0 = global_ns();
  uint32_t it = 0;
  while (true) {
    uint64_t low[4] = {0, 0, 0, 0}, cn[4] = {0, 0, 0, 0};
    for (int q = 0; q < copies; ++q) {
      uint64_t a, b, x, y;
      if (sys) {
        ld_relaxed2_sys(w + q * kHidden, a, b);
        ld_relaxed2_sys(w + q * kHidden + 2, x, y);
      } else {
        ld_tagged2(w + q * kHidden, a, b);
        ld_tagged2(w + q * kHidden + 2, x, y);
      }
      cn[0] += a >> 56; low[0] += a & kAccLowMask;
      cn[1] += b >> 56; low[1] += b & kAccLowMask;
      cn[2] += x >> 56; low[2] += x & kAccLowMask;
      cn[3] += y >> 56; low[3] += y & kAccLowMask;
    }
    bool done = true;
    for (int i = 0; i < 4; ++i) {
      v[i] = acc_decode(low[i], cn[i]);
      done = done && cn[i] == expect;
    }
    if (done) return;
    if ((++it & 15u) == 0u) {
      if (aborted(c) || ld_relaxed(&c.ws->error[0]) != 0u) {
        *reinterpret_cast<volatile int*>(&c.sm->abort) = 1;
        return;
      }
      if (global_ns() - t0 > c.timeout) {
        raise_error(c, kErrTimeoutTransition, layer, stage, tok);
        return;
      }
    }
  }
}
__device__ __forceinline__ void acc_wait4(const Ctl& c, const uint64_t* row, int copies, uint32_t expect,
                                          uint32_t expect0, int s0, float v[4], int layer, int stage, int tok,
                                          bool sys = false) {
  const uint64_t* w = row + threadIdx.x * kE;
  if (threadIdx.x == 0) acc_wait_pair(c, row, 1, expect0, s0, -1, layer, stage, tok, sys);
  if (threadIdx.x == 32 && copies > 1)
    acc_wait_pair(c, row + kHidden, 1, expect - expect0, s0, -1, layer, stage, tok, sys);
  consumer_sync(kConsumerThreads);
  uint64_t low[4] = {0, 0, 0, 0}, cn[4] = {0, 0, 0, 0};
  for (int q = 0; q < copies; ++q) {
    uint64_t a, b, x, y;
    if (sys) {
      ld_relaxed2_sys(w + q * kHidden, a, b);
      ld_relaxed2_sys(w + q * kHidden + 2, x, y);
    } else {
      ld_tagged2(w + q * kHidden, a, b);
      ld_tagged2(w + q * kHidden + 2, x, y);
    }
    cn[0] += a >> 56; low[0] += a & kAccLowMask;
    cn[1] += b >> 56; low[1] += b & kAccLowMask;
    cn[2] += x >> 56; low[2] += x & kAccLowMask;
    cn[3] += y >> 56; low[3] += y & kAccLowMask;
  }
  if (cn[0] == expect && cn[1] == expect && cn[2] == expect && cn[3] == expect) {
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = acc_decode(low[i], cn[i]);
  } else {
    float u[4];
    acc_wait4_slow(c, w, copies, expect, u, layer, stage, tok, sys);
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = u[i];
  }
}
// Clear this thread's 4 elements of an accumulator row.
__device__ __forceinline__ void acc_clear4(uint64_t* row) {
  uint64_t* w = row + threadIdx.x * kE;
  *reinterpret_cast<ulonglong2*>(w) = make_ulonglong2(0ull, 0ull);
  *reinterpret_cast<ulonglong2*>(w + 2) = make_ulonglong2(0ull, 0ull);
}

// The same field of rank g's workspace (tensor parallel), as this GPU addresses it.
template <typename T>
__device__ __forceinline__ T* peer_field(const DecodeParams& p, int g, T* local) {
  const size_t off = reinterpret_cast<const char*>(local) - reinterpret_cast<const char*>(p.ws);
  return reinterpret_cast<T*>(reinterpret_cast<char*>(p.peer_ws[g]) + off);
}
// One counted contribution to an accumulator word: the local word on a single
// GPU; with tensor parallelism the same word on every GPU (each one sums all
// GPUs' contributions). The loop over ranks is unrolled so that the peer table
// is indexed statically.
// `tps`: the launch's tensor-parallel size (the constant 1 in the single-GPU
// kernel, which then carries none of the peer code).
__device__ __forceinline__ void acc_add(const DecodeParams& p, int tps, uint64_t* local, uint64_t term) {
  if (tps <= 1) {
    red_add_u64(local, term);
    return;
  }
#pragma unroll
  for (int g = 0; g < kMaxTP; ++g)
    if (g < tps) red_add_u64_sys(peer_field(p, g, local), term);
}

static_assert(kCluster == 2 && kSlice == 64 * kConsumerWarps, "down projection: 64 output columns per warp");
// bytes of one pair attention exchange: o[128], m and l for each of the two heads
constexpr uint32_t kPairAttnBytes = 2u * (kHeadDim + 2) * 4u;
static_assert(2 * kHeadDim == kConsumerThreads, "one consumer thread per (head, dim) in the combine");


// Bounded wait for the cluster partner's SwiGLU values of this layer; true once
// they have landed. Unlike the other waits it does not give up on an abort:
// an aborted partner still sends every layer until it leaves the token loop
// (and then says so through peer_gone), and each value must have landed before
// this CTA re-arms rxbar or exits.
// The same wait serves the attention partials (atbar).
__device__ __noinline__ bool cluster_rx_wait_slow(const Ctl c, uint64_t* bar, uint32_t ph, int layer, int stage,
                                                  int tok) {
  const uint64_t t0 = global_ns();
  while (!mbar_wait_cluster(bar, ph, kSuspendNs)) {
    if (*reinterpret_cast<volatile int*>(&c.sm->peer_gone) != 0) return false;
    if (global_ns() - t0 > c.timeout) {
      raise_error(c, kErrTimeoutTransition, layer, stage, tok);
      return false;
    }
  }
  return true;
}
__device__ __forceinline__ bool cluster_rx_wait(const Ctl& c, uint64_t* bar, uint32_t ph, int layer, int stage,
                                                int tok) {
  return mbar_wait_cluster(bar, ph, 0u) || cluster_rx_wait_slow(c, bar, ph, layer, stage, tok);
}

// Outputs of a launch that stopped on an error: NaN over the logits rows
// [va, vb) and -1 for output tokens [t0, n_tokens) (none of those completed, so
// no CTA writes a valid id there). Called by every consumer thread of a CTA.
__device__ __forceinline__ void poison_outputs(const DecodeParams& p, int va, int vb, int t0) {
  if (p.logits != nullptr)
    for (int i = va + static_cast<int>(threadIdx.x); i < vb; i += kConsumerThreads) p.logits[i] = __int_as_float(0x7fc00000);
  if (p.out_tokens != nullptr && threadIdx.x == 0)
    for (int i = max(t0, 0); i < p.n_tokens; ++i) p.out_tokens[i] = -1;
}

// The complete down-projection sums of layer l, this thread's 4 elements. One
// GPU: the local counted accumulator (G / 2 cluster pairs). Tensor parallel:
// the last CTA of every GPU waits for its GPU's sums and forwards them, one
// contribution per GPU, into every GPU's acc_x; every CTA then reads acc_x
// (tp_size contributions). Forwarding keeps the cross-GPU traffic at one word
// per element and GPU instead of one per cluster pair.
__device__ __forceinline__ void down_sums(const DecodeParams& p, int tps, const Ctl& c, int l, int down_copy0,
                                          float d[4], int stage, int tok) {
  const int G = p.grid;
  if (tps <= 1) {
    acc_wait4(c, &p.ws->acc_down[l][0][0], kDownCopies, static_cast<uint32_t>(G / kCluster),
              static_cast<uint32_t>(down_copy0), 0, d, l, stage, tok);
    return;
  }
  if (c.cta == G - 1) {
    float v[4];
    acc_wait4(c, &p.ws->acc_down[l][0][0], kDownCopies, static_cast<uint32_t>(G / kCluster),
              static_cast<uint32_t>(down_copy0), 0, v, l, stage, tok);
    bool bad = false;
#pragma unroll
    for (int i = 0; i < kE; ++i) acc_add(p, tps, &p.ws->acc_x[l][threadIdx.x * kE + i], acc_term(v[i], bad));
    if (bad) raise_error(c, kErrRange, l, stage, tok);
  }
  acc_wait4(c, &p.ws->acc_x[l][0], 1, static_cast<uint32_t>(tps), static_cast<uint32_t>(tps), 0, d, l,
            stage, tok, true);
}

template <bool kFused, bool kTraced, bool kTP>
__device__ void consumer_run(const DecodeParams& p, const Plan& pl, const Ctl& c, int token0, int pos0, int cl0,
                             int splits0, uint32_t tag0) {
  Smem& sm = *c.sm;
  Workspace* ws = p.ws;
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int e0 = tid * kE;  // first element owned by this thread
  constexpr bool fused = kFused;
  const int G = p.grid;
  const int tps = kTP ? p.tp_size : 1;
  const TpShape tp = tp_shape(kTP ? p.tp_rank : 0, tps, kVocab);
  const bool tpx = tp.size > 1;
  const int lb = p.layer_begin, le = p.layer_end;
  const int zero_cta = G - 1;
  const bool serve = p.mailbox != nullptr && p.result != nullptr;
  // With 1 + kDownCopies CTAs outside the head groups (148 SMs: 4), those CTAs,
  // idle during attention, clear the layer l-2 accumulators there; otherwise
  // the last CTA clears them before its QKV rows (which then publish late).
  const bool spare_clear = !(tp.size > 1) && G - tp.hl * p.group_size >= 1 + kDownCopies;
  // contributions that land in copy 0 of a down row: clusters k with k % kDownCopies == 0
  const int down_copy0 = (G / kCluster + kDownCopies - 1) / kDownCopies;
  uint32_t n = 0;
  uint32_t xph = 0;     // phase of sm.rxbar for the next cluster exchange
  bool rx_live = true;  // every earlier phase of sm.rxbar was seen to complete
  // Cluster-pair constants of the down projection, fixed for the launch (each
  // costs a dependent chain of long-latency instructions if formed per layer):
  // this CTA's rank, the partner's SwiGLU row count, the partner's mrx slot and
  // rxbar for this thread's value, and this pair's copy of the down accumulators.
  const uint32_t crank = cluster_ctarank();
  const Plan pplan = make_plan(c.cta ^ 1, G, p.group_size, tp);
  const int nj2 = pplan.jb - pplan.ja;
  const uint32_t rx_bar_peer = mapa_shared(smem_addr(&sm.rxbar), crank ^ 1u);
  const uint32_t rx_m_peer = mapa_shared(smem_addr(&sm.mrx[tid & 31]), crank ^ 1u);
  const int down_copy = (c.cta / kCluster) % kDownCopies;
  // Attention split between the two CTAs of the pair (same KV head): partner's
  // apeer buffer and atbar, this CTA's phase of atbar, and liveness as for rxbar.
  const bool pair_attn = pair_shares_head(c.cta, G, p.group_size, tp);
  const uint32_t apeer_remote = mapa_shared(smem_addr(&sm.apeer[0][0]), crank ^ 1u);
  const uint32_t atbar_remote = mapa_shared(smem_addr(&sm.atbar), crank ^ 1u);
  uint32_t aph = 0;
  bool at_live = true;
  int flip = 0;
  float xr[32];
  Tracer<kTraced> tr{c.trace, sm.tbuf, c.trace_cap, 0, 0};
  float(*xred)[64] = sm.u.xred;

  int token = token0;
  for (int t = 0; t < p.n_tokens; ++t) {
    const int pos = pos0 + t;
    const int cl = cl0 + t;
    const uint32_t tgtG = static_cast<uint32_t>(G * (t + 1));
    const uint32_t tag = tag0 + static_cast<uint32_t>(t) + 1u;
    tr.mark(kTrMark, kStToken, 0, t);
    // Prefill (p.prompt): the inputs are given, and the LM head (and the wait
    // for the last layer's sums that feeds it) runs for the last token only.
    const bool last_tok = t == p.n_tokens - 1;
    const bool lm_now = (p.flags & kFlagLmHead) && (p.prompt == nullptr || last_tok);

    // ---- token input: embedding gather (megakernel.cu:783-795) ----
    if (serve) {
      // serve mode: CTA 0 takes the host's token t (mailbox seq == t + 1) and
      // broadcasts it; a negative token ends the launch
      // (every CTA polling the host word itself measured 2.4x slower per token:
      // 148 pollers over PCIe)
      if (c.cta == 0 && tid == 0) {
        const int v = host_token(c, p.mailbox, t);
        if (!aborted(c)) st_release_u64(&ws->tok_flag[0], tok_word(t, v));
      }
      if (tid == 0) sm.token = spin_token(c, &ws->tok_flag[0], static_cast<uint32_t>(t + 1), t);
      consumer_sync(kConsumerThreads);
      token = sm.token;
      if (token < 0 && !aborted(c)) {
        // every CTA leaves here; the last one to see the end restores the
        // workspace for the next launch (every earlier token left its
        // accumulators cleared)
        if (tid == 0) {
          *reinterpret_cast<volatile int*>(&sm.abort) = 1;
          uint32_t old;
          asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(old) : "l"(&ws->stop_seen[0]) : "memory");
          if (old == static_cast<uint32_t>(G - 1)) {
            for (int i = 0; i < kMaxLayers * 4; ++i) ws->sync[i >> 2][i & 3][0] = 0u;
            for (int i = 0; i < kMaxLayers * kNKV; ++i) ws->kv_ready[i / kNKV][i % kNKV][0] = 0u;
            ws->arrive[0] = 0u;
            ws->arrive_x[0] = 0u;
            ws->tag_base[0] = next_tag_base(ws, tag0 + static_cast<uint32_t>(t));
            ws->stop_seen[0] = 0u;
            ws->tok_flag[0] = 0ull;
          }
        }
        return;
      }
    } else if (t > 0) {
      // the previous token is complete (and its last CTA has reset the shared
      // state); the broadcast word carries its argmax
      if (tid == 0) sm.token = spin_token(c, &ws->tok_flag[0], static_cast<uint32_t>(t), t);
      consumer_sync(kConsumerThreads);
      if (p.prompt == nullptr) {
        token = sm.token;
        if (p.stop_token >= 0 && token == p.stop_token && !aborted(c)) {
          // The previous token was the stop id (model.py:102-105 ends its loop
          // there): every CTA leaves here, uniformly; the producer stops too. The
          // token's last CTA already reset the shared state except tok_flag,
          // which the last CTA to see the stop clears.
          if (tid == 0) {
            *reinterpret_cast<volatile int*>(&sm.abort) = 1;
            uint32_t old;
            asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(old) : "l"(&ws->stop_seen[0]) : "memory");
            if (old == static_cast<uint32_t>(G - 1)) {
              ws->stop_seen[0] = 0u;
              ws->tok_flag[0] = 0ull;
            }
            if (c.cta == 0 && p.out_tokens != nullptr)
              for (int i = t; i < p.n_tokens; ++i) p.out_tokens[i] = -1;
          }
          return;
        }
      }
    }
    if (p.prompt != nullptr) token = __ldg(p.prompt + t);
    token = min(max(token, 0), kVocab - 1);
    float r[4];
    if (p.input_residual) {
      const float4 v = __ldcg(reinterpret_cast<const float4*>(p.input_residual) + tid);
      r[0] = v.x; r[1] = v.y; r[2] = v.z; r[3] = v.w;
    } else {
      const uint2 u = __ldg(reinterpret_cast<const uint2*>(p.embed + (size_t)token * kHidden) + tid);
      r[0] = bf_lo(u.x); r[1] = bf_hi(u.x); r[2] = bf_lo(u.y); r[3] = bf_hi(u.y);
    }

    uint2 wA = make_uint2(0u, 0u), wD = make_uint2(0u, 0u);
    if (le > lb) wA = load_w4(lwt(c, lb, kWNorm));
    for (int l = lb; l < le; ++l) {
      // ================= A: RMSNorm + QKV rows (megakernel.cu:704-739, 633-701) ===
      if (l > lb) {
        if constexpr (fused) {
          tr.mark(kTrWaitBegin, kStA, l, t);
          float d[4];
          down_sums(p, tps, c, l - 1, down_copy0, d, kStA, t);
          tr.mark(kTrWaitEnd, kStA, l, t);
          const float4 rm = *reinterpret_cast<const float4*>(&sm.rmid[e0]);
          r[0] = rm.x + d[0]; r[1] = rm.y + d[1]; r[2] = rm.z + d[2]; r[3] = rm.w + d[3];
        } else {
          transition_wait(c, tr, &ws->sync[l - 1][3][0], tgtG, l, kStA, t);
          const float4 v = __ldcg(reinterpret_cast<const float4*>(ws->resid) + tid);
          r[0] = v.x; r[1] = v.y; r[2] = v.z; r[3] = v.w;
        }
        // Every CTA has finished layer l-1 (and so read the accumulators of
        // layer l-2): clear those for the next token.
        if (!spare_clear && c.cta == zero_cta && l >= lb + 2) {
          acc_clear4(&ws->acc_mid[l - 2][0]);
#pragma unroll
          for (int q = 0; q < kDownCopies; ++q) acc_clear4(&ws->acc_down[l - 2][q][0]);
          if (tpx) acc_clear4(&ws->acc_x[l - 2][0]);
        }
      }
      *reinterpret_cast<float4*>(&sm.r[e0]) = make_float4(r[0], r[1], r[2], r[3]);
      uint32_t bfr[kKSteps][2];
      tr.mark(kTrMark, kSubAInput, l, t);
      const float rstd_a = norm_to_x(sm, r, wA, flip);
      load_bfrag(sm, bfr);
      tr.mark(kTrMark, kSubANorm, l, t);
      // QKV rows: up to three padded chunks (one 16-row MMA tile each) per pass
      for (int rr = pl.qa; rr < pl.qb;) {
        const int ra0 = rr, ea0 = qkv_chunk_end(ra0, pl.qb, tp);
        const int ra1 = ea0, ea1 = ra1 < pl.qb ? qkv_chunk_end(ra1, pl.qb, tp) : ra1;
        const int ra2 = ea1, ea2 = ra2 < pl.qb ? qkv_chunk_end(ra2, pl.qb, tp) : ra2;
        const int na = 1 + (ea1 > ra1) + (ea2 > ra2);
        rr = ea2;
        uint32_t sa[3];
        ring_wait_all(c, n, na, sa, l, 0, t, &tr);
        float d0[4] = {0.f, 0.f, 0.f, 0.f}, d1[4] = {0.f, 0.f, 0.f, 0.f}, d2[4] = {0.f, 0.f, 0.f, 0.f};
        mma_tile_1024(sa[0], ea0 - ra0, bfr, d0);
        if (na > 1) mma_tile_1024(sa[1], ea1 - ra1, bfr, d1);
        if (na > 2) mma_tile_1024(sa[2], ea2 - ra2, bfr, d2);
        tr.mark(kTrMark, kSubAMma, l, t);
        stash_tile(xred, 0, d0);
        stash_tile(xred, 1, d1);
        stash_tile(xred, 2, d2);
        consumer_sync(kConsumerThreads);
        tr.mark(kTrMark, kSubABar, l, t);
        if (tid < 48 && !(t == 0 && l == lb && c.cta == p.withhold_cta)) {
          const int i = tid >> 4;
          const int row = (i == 0 ? ra0 : (i == 1 ? ra1 : ra2)) + (tid & 15);
          const int end = i == 0 ? ea0 : (i == 1 ? ea1 : ea2);
          if ((tid & 15) < 15 && row < end) {
            const float val = sum_warps(xred, tid) * rstd_a;
            const int grow = qkv_global_row(tp, row);
            st_tagged(&ws->qkv_tagged[l][grow], val, tag);
            if (l == le - 1) {  // raw QKV outputs are reported for the last layer only
              float* dst = grow < kQSize ? p.q_out + grow
                           : grow < kQSize + kKVSize ? p.k_out + (grow - kQSize)
                                                     : p.v_out + (grow - kQSize - kKVSize);
              *dst = val;
            }
          }
        }
        // The slots go back to the producer after the publish: its next bulk
        // copies would otherwise be issued ahead of the tagged stores (-2.7 us
        // per token measured).
        ring_done_all(c, n, na);
        // xred is reused by the next pass; after the last one the next writer
        // (attention, o_proj) is past the head-preparation barrier
        if (rr < pl.qb) consumer_sync(kConsumerThreads);
      }
      tr.mark(kTrPublish, kStA, l, t);
      wD = load_w4(lwt(c, l, kWPost));  // post-attention norm, one stage ahead

      // ================= BC: head norm + RoPE + KV append, attention, o_proj =====
      if (pl.in_bc) {
        const int h = pl.h;
        const uint32_t stag = (tag << 5) | static_cast<uint32_t>(l);  // split partials: token and layer
        // attention splits of this token (every split range holds keys; a fixed
        // count from the caller may leave some empty)
        const int splits = splits0 > 0 ? splits0 : choose_splits(cl, p.group_size);
        // Per-head norm weights and this position's RoPE row do not depend on
        // QKV: load them before polling. Lane owns dims 2l, 2l+1, 64+2l, 65+2l.
        float w0 = 0.f, w1 = 0.f, w2 = 0.f, w3 = 0.f, cs0 = 0.f, sn0 = 0.f, cs1 = 0.f, sn1 = 0.f;
        const int d0 = 2 * lane;
        if (warp < 3) {
          const __nv_bfloat16* nw = lwt(c, l, warp < 2 ? kWQNorm : kWKNorm);
          const uint32_t wa = __ldg(reinterpret_cast<const unsigned int*>(nw + d0));
          const uint32_t wb = __ldg(reinterpret_cast<const unsigned int*>(nw + d0 + 64));
          w0 = bf_lo(wa); w1 = bf_hi(wa); w2 = bf_lo(wb); w3 = bf_hi(wb);
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
          // every lane polls its own words: a single poller per warp followed by
          // the lanes' reads cost one more L2 round trip (+8.7 us per token measured)
          // both word pairs are loaded before either is checked (one L2 round
          // trip when they are already there, not two)
          {
            uint64_t a, b, e, f;
            ld_tagged2(&ws->qkv_tagged[l][base + d0], a, b);
            ld_tagged2(&ws->qkv_tagged[l][base + d0 + 64], e, f);
            const bool ok = static_cast<uint32_t>(a >> 32) == tag && static_cast<uint32_t>(b >> 32) == tag &&
                            static_cast<uint32_t>(e >> 32) == tag && static_cast<uint32_t>(f >> 32) == tag;
            if (ok) {
              x0 = __uint_as_float(static_cast<uint32_t>(a));
              x1 = __uint_as_float(static_cast<uint32_t>(b));
              x2 = __uint_as_float(static_cast<uint32_t>(e));
              x3 = __uint_as_float(static_cast<uint32_t>(f));
            } else {
              poll_tagged2(c, &ws->qkv_tagged[l][base + d0], tag, x0, x1, l, t);
              poll_tagged2(c, &ws->qkv_tagged[l][base + d0 + 64], tag, x2, x3, l, t);
            }
          }
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
                __nv_bfloat16* dst = p.k_cache + (((size_t)l * tp.hl + pl.hl) * p.max_seq + pos) * kHeadDim;
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
              __nv_bfloat16* dst = p.v_cache + (((size_t)l * tp.hl + pl.hl) * p.max_seq + pos) * kHeadDim;
              *reinterpret_cast<__nv_bfloat162*>(dst + d0) = b01;
              *reinterpret_cast<__nv_bfloat162*>(dst + d0 + 64) = b23;
            }
          }
        }
        consumer_sync(kConsumerThreads);
        tr.mark(kTrWaitEnd, kStBC, l, t);
        tr.mark(kTrMark, kSubBCPrep, l, t);
        // GQA decode attention over keys [ka, kb) (megakernel.cu:228-370): per
        // 64-key chunk warp w takes keys [8w, 8w+8) for both Q heads; lane holds
        // dims [4 lane, 4 lane + 4). The 16 dot products are summed over the
        // warp by a reduce-scatter butterfly (16 shuffles), after which lane L
        // holds score j = (L >> 1) & 15 (head j >> 3, key j & 7). Online softmax
        // per warp in the exp2 domain, then a combine over the warps.
        int ka, kb;
        attn_keys(cl, splits, pl.c, pair_attn, static_cast<int>(crank), &ka, &kb);
        const bool pair_now = splits <= 1 && pair_attn && cl >= kPairSplitKeys;
        if (kb > ka) {
          float q0[4], q1[4];
          {
            const float4 a = *reinterpret_cast<const float4*>(&sm.q[0][lane * 4]);
            const float4 b = *reinterpret_cast<const float4*>(&sm.q[1][lane * 4]);
            q0[0] = a.x; q0[1] = a.y; q0[2] = a.z; q0[3] = a.w;
            q1[0] = b.x; q1[1] = b.y; q1[2] = b.z; q1[3] = b.w;
          }
          const int jm = (lane >> 1) & 15;   // score held after the butterfly
          const int my_key = jm & 7;
          const bool my_head1 = jm >= 8;
          float m = -INFINITY, lsum = 0.f;   // this lane's head: running max and sum
          float a0[4] = {0.f, 0.f, 0.f, 0.f}, a1[4] = {0.f, 0.f, 0.f, 0.f};
          for (int k0 = ka; k0 < kb; k0 += kKeysPerChunk) {
            const int k1 = min(kb, k0 + kKeysPerChunk);
            const int kw = k0 + warp * kKeysPerWarp;  // this warp's first key
            const uint32_t sa = ring_wait(c, n, l, 1, t, &tr);
            // A warp whose 8 keys all lie past the end of the cache leaves its
            // softmax state unchanged: skip the arithmetic (its SM sub-partition
            // then issues for the other warp alone).
            if (kw < k1) {
              // The producer skips row `pos` (the key appended this step): the warp
              // that owns it writes the rotated K and the V row into the slot, so
              // that every key is read the same way.
              if (pos >= kw && pos < kw + kKeysPerWarp && pos < k1) {
                const float4 kn = *reinterpret_cast<const float4*>(&sm.knew[lane * 4]);
                const float4 vn = *reinterpret_cast<const float4*>(&sm.vnew[lane * 4]);
                const uint32_t row = sa + (pos - k0) * (kHeadDim * 2) + lane * 8;
                asm volatile("st.shared.v2.u32 [%0], {%1, %2};" ::"r"(row), "r"(pack_bf2(kn.x, kn.y)),
                             "r"(pack_bf2(kn.z, kn.w)) : "memory");
                asm volatile("st.shared.v2.u32 [%0], {%1, %2};" ::"r"(row + kSlotBytes / 2), "r"(pack_bf2(vn.x, vn.y)),
                             "r"(pack_bf2(vn.z, vn.w)) : "memory");
                fence_proxy_async_shared();  // before the slot is handed back to the bulk-copy engine
                __syncwarp();
              }
              // all eight key rows of this warp (rows past k1 are in the slot but masked)
              uint2 kr[kKeysPerWarp];
  #pragma unroll
              for (int i = 0; i < kKeysPerWarp; ++i) kr[i] = lds64(sa + (kw + i - k0) * (kHeadDim * 2) + lane * 8);
              float v[16];
  #pragma unroll
              for (int i = 0; i < kKeysPerWarp; ++i) {
                const float kx0 = bf_lo(kr[i].x), kx1 = bf_hi(kr[i].x), kx2 = bf_lo(kr[i].y), kx3 = bf_hi(kr[i].y);
                v[i] = fmaf(q0[3], kx3, fmaf(q0[2], kx2, fmaf(q0[1], kx1, q0[0] * kx0)));
                v[8 + i] = fmaf(q1[3], kx3, fmaf(q1[2], kx2, fmaf(q1[1], kx1, q1[0] * kx0)));
              }
              // value rows, loaded while the scores are reduced
              uint2 vr[kKeysPerWarp];
  #pragma unroll
              for (int i = 0; i < kKeysPerWarp; ++i) {
                // rows past k1 are zeroed here (2 selects a row), so stale slot
                // contents never reach the sums below
                const uint2 x = lds64(sa + kSlotBytes / 2 + (kw + i - k0) * (kHeadDim * 2) + lane * 8);
                vr[i] = kw + i < k1 ? x : make_uint2(0u, 0u);
              }
              // reduce-scatter butterfly: 16 -> 8 -> 4 -> 2 -> 1 values, then the last lane bit
  #pragma unroll
              for (int half = 8, bit = 16; half >= 1; half >>= 1, bit >>= 1) {
                const bool up = (lane & bit) != 0;
  #pragma unroll
                for (int j = 0; j < half; ++j) {
                  const float send = up ? v[j] : v[j + half];
                  const float keep = up ? v[j + half] : v[j];
                  v[j] = keep + __shfl_xor_sync(0xffffffffu, send, bit);
                }
              }
              float s = v[0] + __shfl_xor_sync(0xffffffffu, v[0], 1);
              if (kw + my_key >= k1) s = -INFINITY;
              // online softmax for this lane's head over the warp's 8 keys
              float mx = s;
              mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
              mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
              mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
              const float mnew = fmaxf(m, mx);
              float sc = 1.f, pk = 0.f;
              if (mnew > -INFINITY) {
                sc = ex2_approx(m - mnew);
                pk = s > -INFINITY ? ex2_approx(s - mnew) : 0.f;
              }
              float ps = pk;
              ps += __shfl_xor_sync(0xffffffffu, ps, 2);
              ps += __shfl_xor_sync(0xffffffffu, ps, 4);
              ps += __shfl_xor_sync(0xffffffffu, ps, 8);
              lsum = lsum * sc + ps;
              m = mnew;
              // both heads' rescale factors and the 16 weights for the value rows
              const float sco = __shfl_xor_sync(0xffffffffu, sc, 16);
              const float sc0 = my_head1 ? sco : sc, sc1 = my_head1 ? sc : sco;
              if ((lane & 1) == 0) sm.pbuf[warp][jm] = pk;
              __syncwarp();
              float p0[8], p1[8];
              {
                const float4 x = *reinterpret_cast<const float4*>(&sm.pbuf[warp][0]);
                const float4 y = *reinterpret_cast<const float4*>(&sm.pbuf[warp][4]);
                const float4 z = *reinterpret_cast<const float4*>(&sm.pbuf[warp][8]);
                const float4 w = *reinterpret_cast<const float4*>(&sm.pbuf[warp][12]);
                p0[0] = x.x; p0[1] = x.y; p0[2] = x.z; p0[3] = x.w; p0[4] = y.x; p0[5] = y.y; p0[6] = y.z; p0[7] = y.w;
                p1[0] = z.x; p1[1] = z.y; p1[2] = z.z; p1[3] = z.w; p1[4] = w.x; p1[5] = w.y; p1[6] = w.z; p1[7] = w.w;
              }
              __syncwarp();
  #pragma unroll
              for (int d = 0; d < 4; ++d) {
                a0[d] *= sc0;
                a1[d] *= sc1;
              }
  #pragma unroll
              for (int i = 0; i < kKeysPerWarp; ++i) {
                const float vx0 = bf_lo(vr[i].x), vx1 = bf_hi(vr[i].x);
                const float vx2 = bf_lo(vr[i].y), vx3 = bf_hi(vr[i].y);
                a0[0] = fmaf(p0[i], vx0, a0[0]); a0[1] = fmaf(p0[i], vx1, a0[1]);
                a0[2] = fmaf(p0[i], vx2, a0[2]); a0[3] = fmaf(p0[i], vx3, a0[3]);
                a1[0] = fmaf(p1[i], vx0, a1[0]); a1[1] = fmaf(p1[i], vx1, a1[1]);
                a1[2] = fmaf(p1[i], vx2, a1[2]); a1[3] = fmaf(p1[i], vx3, a1[3]);
              }
            }
            ring_done(c, n);
          }
          tr.mark(kTrMark, kSubBCAttn, l, t);
          *reinterpret_cast<float4*>(&sm.u.att[warp][0][lane * 4]) = make_float4(a0[0], a0[1], a0[2], a0[3]);
          *reinterpret_cast<float4*>(&sm.u.att[warp][1][lane * 4]) = make_float4(a1[0], a1[1], a1[2], a1[3]);
          if (lane == 0 || lane == 16) {
            sm.u.att[warp][lane >> 4][kHeadDim] = m;
            sm.u.att[warp][lane >> 4][kHeadDim + 1] = lsum;
          }
          consumer_sync(kConsumerThreads);
          tr.mark(kTrMark, kSubBCAttW, l, t);
          if (tid < 2 * kHeadDim) {
            const int hh = tid >> 7, d = tid & (kHeadDim - 1);
            float M = -INFINITY;
#pragma unroll
            for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, sm.u.att[w][hh][kHeadDim]);
            float L = 0.f, O = 0.f;
#pragma unroll
            for (int w = 0; w < kConsumerWarps; ++w) {
              const float mw = sm.u.att[w][hh][kHeadDim];
              const float f = mw > -INFINITY ? ex2_approx(mw - M) : 0.f;
              L = fmaf(sm.u.att[w][hh][kHeadDim + 1], f, L);
              O = fmaf(sm.u.att[w][hh][d], f, O);
            }
            if (pair_now) {
              // this CTA's half of the keys: partial to the partner, then the
              // partner's partial back, combined in rank order (both CTAs of the
              // pair get identical outputs)
              if (*reinterpret_cast<volatile int*>(&sm.peer_gone) == 0) {
                const uint32_t dst = apeer_remote + static_cast<uint32_t>(hh * (kHeadDim + 4)) * 4u;
                st_async_f32(dst + d * 4u, O, atbar_remote);
                if (d == 0) {
                  st_async_f32(dst + kHeadDim * 4u, M, atbar_remote);
                  st_async_f32(dst + (kHeadDim + 1) * 4u, L, atbar_remote);
                }
              }
              if (at_live) at_live = cluster_rx_wait(c, &sm.atbar, aph, l, kStBC, t);
              const float Mp = sm.apeer[hh][kHeadDim], Lp = sm.apeer[hh][kHeadDim + 1], Op = sm.apeer[hh][d];
              const float Ma = crank == 0 ? M : Mp, La = crank == 0 ? L : Lp, Oa = crank == 0 ? O : Op;
              const float Mb = crank == 0 ? Mp : M, Lb = crank == 0 ? Lp : L, Ob = crank == 0 ? Op : O;
              const float Mx = fmaxf(Ma, Mb);
              const float fa = Ma > -INFINITY ? ex2_approx(Ma - Mx) : 0.f;
              const float fb = Mb > -INFINITY ? ex2_approx(Mb - Mx) : 0.f;
              sm.attn[tid] = fmaf(Oa, fa, Ob * fb) / fmaf(La, fa, Lb * fb);
            } else if (splits <= 1) {
              sm.attn[tid] = O / L;
            } else {
              // this split's partial as tagged words: no counter and no release,
              // the readers poll the words themselves
              uint64_t* dst = ws->att_part[h][pl.c][hh];
              st_tagged(dst + d, O, stag);
              if (d == 0) st_tagged2(dst + kHeadDim, M, L, stag);
            }
          }
          consumer_sync(kConsumerThreads);
          if (pair_now) {
            aph ^= 1u;
            // every thread has read apeer: arm the next phase (one arrival with the
            // expected bytes; the partner's next partial may land before or after)
            if (at_live && tid == 0) mbar_arrive_expect_tx(&sm.atbar, kPairAttnBytes);
          }
        } else if (splits > 1 && pl.c < splits) {
          // The launch's split count comes from its longest cache: an earlier
          // token of the launch (a prefill, a generate that starts short) can
          // leave this split without keys. Publish an empty partial (m = -inf,
          // l = 0, o = 0), which the combine weighs by zero.
          if (tid < 2 * kHeadDim) {
            const int hh = tid >> 7, d = tid & (kHeadDim - 1);
            uint64_t* dst = ws->att_part[h][pl.c][hh];
            st_tagged(dst + d, 0.f, stag);
            if (d == 0) st_tagged2(dst + kHeadDim, -INFINITY, 0.f, stag);
          }
        }
        if (splits > 1) {
          // every split's m and l: lane s of warp hh polls split s (one 16-byte
          // word pair), shared through shared memory
          tr.mark(kTrWaitBegin, kStSplit, l, t);
          if (warp < 2 && lane < splits) {
            float ms, ls;
            poll_tagged2(c, &ws->att_part[h][lane][warp][kHeadDim], stag, ms, ls, l, t);
            sm.split_ml[warp][lane] = make_float2(ms, ls);
          }
          consumer_sync(kConsumerThreads);
          tr.mark(kTrWaitEnd, kStSplit, l, t);
          if (tid < 2 * kHeadDim) {
            const int hh = tid >> 7, d = tid & (kHeadDim - 1);
            float M = -INFINITY;
            for (int s = 0; s < splits; ++s) M = fmaxf(M, sm.split_ml[hh][s].x);
            // o of every split, loaded in batches without a branch per word; a
            // word not yet carrying the tag sends the thread to the polling loop
            float L = 0.f, O = 0.f;
            bool all = true;
#pragma unroll 8
            for (int s = 0; s < splits; ++s) {
              const float2 ml = sm.split_ml[hh][s];
              const float f = ml.x > -INFINITY ? ex2_approx(ml.x - M) : 0.f;
              const uint64_t w = ld_tagged(&ws->att_part[h][s][hh][d]);
              all = all && static_cast<uint32_t>(w >> 32) == stag;
              L = fmaf(ml.y, f, L);
              O = fmaf(__uint_as_float(static_cast<uint32_t>(w)), f, O);
            }
            if (!all) {
              O = 0.f;
              for (int s = 0; s < splits; ++s) {
                const float2 ml = sm.split_ml[hh][s];
                const float f = ml.x > -INFINITY ? ex2_approx(ml.x - M) : 0.f;
                float o, unused;
                poll_tagged2(c, &ws->att_part[h][s][hh][d & ~1], stag, o, unused, l, t);
                if (d & 1) o = unused;
                O = fmaf(o, f, O);
              }
            }
            sm.attn[tid] = O / L;
          }
          consumer_sync(kConsumerThreads);
        }

        // o_proj partial of this KV head's two Q heads (megakernel.cu:191-225)
        tr.mark(kTrMark, kSubBCComb, l, t);
        {
          // K = 256 (two heads x 128): warp w owns kOSteps MMA k-steps from
          // 16*kOSteps*w; rows in padded 528-byte slots, four 16-row tiles per chunk.
          uint32_t ob[kOSteps][2];
#pragma unroll
          for (int st = 0; st < kOSteps; ++st) {
            ob[st][0] = 0u;
            ob[st][1] = 0u;
            if (lane < 8) {
              const int k = 16 * (kOSteps * warp + st) + 2 * (lane & 3);
              const float x0 = sm.attn[k], x1 = sm.attn[k + 1], x8 = sm.attn[k + 8], x9 = sm.attn[k + 9];
              const uint32_t h0 = pack_bf2(x0, x1), h1 = pack_bf2(x8, x9);
              ob[st][0] = lane < 4 ? h0 : pack_bf2(x0 - bf_lo(h0), x1 - bf_hi(h0));
              ob[st][1] = lane < 4 ? h1 : pack_bf2(x8 - bf_lo(h1), x9 - bf_hi(h1));
            }
          }
          for (int o0 = pl.oa; o0 < pl.ob; o0 += kORowsPerChunk) {
            const int nrows = min(pl.ob, o0 + kORowsPerChunk) - o0;
            const uint32_t sa = ring_wait(c, n, l, 3, t, &tr);
            float d[4][4] = {};
            const int tr16 = lane & 15;
#pragma unroll
            for (int tt = 0; tt < 4; ++tt) {
              const int rr = tt * 16 + tr16;
              // rows past nrows alias a row of the same bank group (see mma_tile_1024)
              const uint32_t row = sa + (rr < nrows ? rr : (rr & 7)) * kORowStride + (lane >> 4) * 16 +
                                   warp * (kOSteps * 32);
#pragma unroll
              for (int st = 0; st < kOSteps; ++st) {
                uint32_t a0, a1, a2, a3;
                ldsm_x4(row + st * 32, a0, a1, a2, a3);
                mma_bf16(d[tt], a0, a1, a2, a3, ob[st][0], ob[st][1]);
              }
            }
            tr.mark(kTrMark, kSubBCOMma, l, t);
#pragma unroll
            for (int tt = 0; tt < 4; ++tt) stash_tile(xred, tt, d[tt]);
            consumer_sync(kConsumerThreads);
            tr.mark(kTrMark, kSubBCOBar, l, t);
            if (tid < nrows) {
              bool bad = false;
              acc_add(p, tps, &ws->acc_mid[l][o0 + tid], acc_term(sum_warps(xred, tid), bad));
              if (bad) raise_error(c, kErrRange, l, kStBC, t);
            }
            ring_done(c, n);  // after the publish, as for QKV
            // after the last chunk the next xred writer (gate/up) is past the
            // post-attention norm's barrier
            if (o0 + kORowsPerChunk < pl.ob) consumer_sync(kConsumerThreads);
          }
        }
        tr.mark(kTrPublish, kStBC, l, t);
        // A later token of this launch re-reads this head's K/V rows through the
        // bulk-copy engine: publish the append (K writer and V writer). Moving
        // this gpu-scope release off the consumer warps (to the end of the
        // layer, to the producer once per token, to a tenth warp, or having
        // every attention CTA append and wait locally) measured slower.
        if (p.n_tokens > 1 && pl.c == 0 && (warp == 2 || warp == 3)) {
          __syncwarp();
          if (lane == 0) release_add(&ws->kv_ready[l][h][0], 1u);
        }
      }
      if (!pl.in_bc && spare_clear && l >= lb + 2) {
        // every CTA has read the layer l-2 sums (it has passed layer l-1's first
        // exchange, which this CTA waited for): each spare CTA clears one row
        const int sp = c.cta - tp.hl * p.group_size;
        if (sp == 0) acc_clear4(&ws->acc_mid[l - 2][0]);
        if (sp >= 1 && sp <= kDownCopies) acc_clear4(&ws->acc_down[l - 2][sp - 1][0]);
      }

      // ================= DE: post norm, SwiGLU rows, down partial ===============
      // the next layer's input-norm weights, one stage ahead of their use
      if (l + 1 < le) wA = load_w4(lwt(c, l + 1, kWNorm));
      tr.mark(kTrWaitBegin, kStDE, l, t);
      float rstd_d;
      {
        float a[4];
        acc_wait4(c, &ws->acc_mid[l][0], 1, static_cast<uint32_t>(kNKV), static_cast<uint32_t>(kNKV), 0, a, l, kStDE,
                  t, tpx);
        tr.mark(kTrWaitEnd, kStDE, l, t);
        const float4 rv = *reinterpret_cast<const float4*>(&sm.r[e0]);
        float mres[4] = {rv.x + a[0], rv.y + a[1], rv.z + a[2], rv.w + a[3]};
        *reinterpret_cast<float4*>(&sm.rmid[e0]) = make_float4(mres[0], mres[1], mres[2], mres[3]);
        rstd_d = norm_to_x(sm, mres, wD, flip);
        load_bfrag(sm, bfr);
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
        tr.mark(kTrMark, kSubDEMma, l, t);
        stash_tile(xred, 0, d0);
        stash_tile(xred, 1, d1);
        stash_tile(xred, 2, d2);
        consumer_sync(kConsumerThreads);
        tr.mark(kTrMark, kSubDEBar, l, t);
        // thread j of the pass sums gate row j and up row j over the warps (tile
        // j / 7, rows j % 7 and 8 + j % 7) and forms silu(gate) * up at once
        // (megakernel.cu:100-142, config.cuh:177-179)
        const int jl = tid - jb0;
        if (tid >= jb0 && jl < 3 * kGUPerChunk && tid < nj) {
          const int xi = (jl / kGUPerChunk) * 16 + jl % kGUPerChunk;
          const float g = sum_warps(xred, xi) * rstd_d, u = sum_warps(xred, xi + 8) * rstd_d;
          const float mv = g / (1.0f + expf(-g)) * u;
          sm.m[tid] = mv;
          // The cluster partner reduces the other column block over these rows too:
          // each value lands in its shared memory with 4 bytes of complete_tx on its
          // rxbar, so no thread here waits on a release.
          if constexpr (fused) {
            if (*reinterpret_cast<volatile int*>(&sm.peer_gone) == 0) st_async_f32(rx_m_peer, mv, rx_bar_peer);
          }
        }
        consumer_sync(kConsumerThreads);
      }
      tr.mark(kTrMark, kSubDEGU, l, t);
      tr.mark(kTrMark, kSubDESilu, l, t);
      if constexpr (fused) {
        // Down projection split by output columns within the cluster pair: rank r
        // reduces columns [kSlice r, kSlice (r + 1)) over both CTAs' intermediate
        // rows (megakernel.cu:53-90, split by K across pairs), on the tensor
        // cores. Own rows first, then the partner's once its SwiGLU values land.
        float dd[4][4] = {};
        {
          const uint32_t sa = ring_wait(c, n, l, 5, t, &tr);
          down_mma(sa, sm.m, nj, dd);
          ring_done(c, n);
        }
        tr.mark(kTrMark, kSubDEOwn, l, t);
        if (rx_live) rx_live = cluster_rx_wait(c, &sm.rxbar, xph, l, kStDE, t);
        xph ^= 1u;
        tr.mark(kTrMark, kSubDERx, l, t);
        down_mma(ring_wait(c, n, l, 5, t, &tr), sm.mrx, nj2, dd);
        tr.mark(kTrMark, kSubDEDown, l, t);
        if ((lane & 3) == 0) {
          // D columns 0 and 1 (high part and remainder) of rows g and g + 8
          bool bad = false;
          uint64_t* dst = &ws->acc_down[l][down_copy][crank * kSlice + 64 * warp + (lane >> 2)];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            red_add_u64(dst + 16 * i, acc_term(dd[i][0] + dd[i][1], bad));
            red_add_u64(dst + 16 * i + 8, acc_term(dd[i][2] + dd[i][3], bad));
          }
          if (bad) raise_error(c, kErrRange, l, kStDE, t);
        }
        ring_done_all(c, n, 1);  // the partner rows' slot, after the publish
        tr.mark(kTrPublish, kStDE, l, t);
        // Arm the next phase of rxbar, now that this one is seen complete (one
        // arrival per phase; the partner's bytes may land before or after it).
        if (rx_live && tid == kConsumerThreads - 32) mbar_arrive_expect_tx(&sm.rxbar, static_cast<uint32_t>(nj2) * 4u);
      } else {
        // reference layout: publish the SwiGLU vector, then whole down rows
        if (tid < nj) p.mlp_out[pl.ja + tid] = sm.m[tid];
        transition_publish(tr, &ws->sync[l][2][0], l, kStDE, t);
        transition_wait(c, tr, &ws->sync[l][2][0], tgtG, l, kStE, t);
        for (int i = tid; i < kInter; i += kConsumerThreads) sm.u.x[i] = __ldcg(p.mlp_out + i);
        consumer_sync(kConsumerThreads);
        for (int d0 = pl.da; d0 < pl.db; d0 += kDownRowsPerChunk) {
          const int d1 = min(pl.db, d0 + kDownRowsPerChunk);
          const uint32_t sa = ring_wait(c, n, l, 6, t, &tr);
          for (int row = warp; row < d1 - d0; row += kConsumerWarps) {
            float acc = 0.f;
#pragma unroll 4
            for (int g = 0; g < kInter / 256; ++g) {
              const int e = lane * 8 + g * 256;
              const uint4 w = lds128(sa + row * (kInter * 2) + e * 2);
              acc += dot8(w, sm.u.x + e);
            }
            acc = warp_sum(acc);
            if (lane == 0) {
              const int d = d0 + row;
              ws->resid[d] = sm.rmid[d] + acc;
            }
          }
          ring_done(c, n);
        }
        transition_publish(tr, &ws->sync[l][3][0], l, kStE, t);
      }
    }

    // ================= final residual, LM head + argmax (megakernel.cu:870-886) ==
    uint4 fwv[4];
    load_norm_w((p.flags & kFlagSkipFinalNorm) ? nullptr : p.final_norm, fwv);
    if (le > lb && (p.prompt == nullptr || last_tok)) {
      if constexpr (fused) {
        tr.mark(kTrWaitBegin, kStLM, le - 1, t);
        float d[4];
        down_sums(p, tps, c, le - 1, down_copy0, d, kStLM, t);
        tr.mark(kTrWaitEnd, kStLM, le - 1, t);
        const float4 rm = *reinterpret_cast<const float4*>(&sm.rmid[e0]);
        r[0] = rm.x + d[0]; r[1] = rm.y + d[1]; r[2] = rm.z + d[2]; r[3] = rm.w + d[3];
      } else {
        transition_wait(c, tr, &ws->sync[le - 1][3][0], tgtG, le - 1, kStLM, t);
        const float4 v = __ldcg(reinterpret_cast<const float4*>(ws->resid) + tid);
        r[0] = v.x; r[1] = v.y; r[2] = v.z; r[3] = v.w;
      }
    }
    *reinterpret_cast<float4*>(&sm.r[e0]) = make_float4(r[0], r[1], r[2], r[3]);
    if (c.cta == 0 && p.residual_out != nullptr && t == p.n_tokens - 1)
      *reinterpret_cast<float4*>(p.residual_out + e0) = make_float4(r[0], r[1], r[2], r[3]);
    float bv = -INFINITY;
    int bi = INT_MAX;
    if (lm_now) {
      const float tot = block_sum(r[0] * r[0] + r[1] * r[1] + r[2] * r[2] + r[3] * r[3], sm.red, flip);
      const float rstd = (p.flags & kFlagSkipFinalNorm) ? 1.0f : rsqrtf(tot * (1.0f / kHidden) + kEps);
      xr_from(sm.r, rstd, fwv, xr);
      for (int v0 = pl.va; v0 < pl.vb; v0 += kRowsPerChunk1024) {
        const int v1 = min(pl.vb, v0 + kRowsPerChunk1024);
        const uint32_t sa = ring_wait(c, n, -1, 8, t, &tr);
#pragma unroll
        for (int i = 0; i < kRowsPerChunk1024 / kConsumerWarps; ++i) {
          const int row = v0 + warp + i * kConsumerWarps;
          if (row < v1) {
            const float v = warp_sum(dot_row1024(sa + (warp + i * kConsumerWarps) * 2048, xr, lane));
            if (lane == 0 && p.logits != nullptr) p.logits[row] = v;
            if (better(v, row, bv, bi)) {
              bv = v;
              bi = row;
            }
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
        // ordered before the arrival below by its release
        if (!tpx) {
          asm volatile("red.relaxed.gpu.global.max.u64 [%0], %1;" ::"l"(&ws->tok_best[0]), "l"(argmax_key(bv, bi))
                       : "memory");
        } else {
#pragma unroll
          for (int g = 0; g < kMaxTP; ++g)
            if (g < tp.size) red_max_u64_sys(peer_field(p, g, &ws->tok_best[0]), argmax_key(bv, bi));
        }
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
        if (tpx) {
          // this CTA's arrival on the other GPUs, ordered after its argmax candidate
#pragma unroll
          for (int g = 0; g < kMaxTP; ++g)
            if (g < tp.size && g != tp.rank) red_release_add_sys(peer_field(p, g, &ws->arrive_x[0]), 1u);
        }
        uint32_t old;
        asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(old) : "l"(&ws->arrive[0]) : "memory");
        sm.is_last = (old == tgtG - 1u) ? 1 : 0;
      }
    }
    consumer_sync(kConsumerThreads);
    const int last_state = sm.is_last;
    consumer_sync(kConsumerThreads);
    tr.mark(kTrMark, kStEnd, 0, t);
    tr.flush();
    if (last_state < 0) {
      // leaving early: the cluster partner must not wait for (or send) more
      // SwiGLU values; this store is ordered before the final cluster barrier
      if (tid == 0) st_cluster_u32(mapa_shared(smem_addr(&sm.peer_gone), cluster_ctarank() ^ 1u), 1u);
      // make the failure visible in the outputs: NaN over this CTA's logits rows,
      // -1 for every token of the launch that has not completed
      poison_outputs(p, pl.va, pl.vb, t);
      return;
    }
    if (last_state) {
      int best = -1;
      if (tpx && tid == 0) {
        // every CTA of the other GPUs has arrived too (their candidates are in)
        spin_geq_sys(c, &ws->arrive_x[0], static_cast<uint32_t>(G * (tp.size - 1) * (t + 1)), kErrTimeoutToken, -1,
                     kStEnd, t);
      }
      if (lm_now && tid == 0) {
        best = argmax_key_index(__ldcg(&ws->tok_best[0]));
        ws->tok_best[0] = 0ull;  // for the next token (ordered by the release below)
        sm.token = best;
      }
      consumer_sync(kConsumerThreads);
      // the launch ends after this token: the last one, or a generated stop id
      const bool stop_now = !last_tok && lm_now && p.prompt == nullptr && p.stop_token >= 0 &&
                            sm.token == p.stop_token;
      const bool final_tok = last_tok || stop_now;
      // the last two layers' accumulators (earlier ones were cleared on the way)
      for (int l = max(lb, le - 2); l < le; ++l) {
        acc_clear4(&ws->acc_mid[l][0]);
        for (int q = 0; q < kDownCopies; ++q) acc_clear4(&ws->acc_down[l][q][0]);
        if (tpx) acc_clear4(&ws->acc_x[l][0]);
      }
      if (final_tok) {
        for (int i = tid; i < kMaxLayers * 4; i += kConsumerThreads) ws->sync[i >> 2][i & 3][0] = 0u;
        for (int i = tid; i < kMaxLayers * kNKV; i += kConsumerThreads) ws->kv_ready[i / kNKV][i % kNKV][0] = 0u;
      }
      consumer_sync(kConsumerThreads);
      if (tid == 0) {
        if (lm_now) {
          if (serve) {
            // {seq, argmax} as one 8-byte release store into pinned host memory
            const uint64_t w = (static_cast<uint64_t>(static_cast<uint32_t>(best)) << 32) | static_cast<uint32_t>(t + 1);
            asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p.result), "l"(w) : "memory");
          }
          if (p.out_tokens != nullptr) p.out_tokens[t] = best;
          if (p.step != nullptr && (p.flags & kFlagAdvanceStep)) {
            p.step[0] = best;
            p.step[1] = pos + 1;
            p.step[3] += 1;
          }
        }
        if (last_tok) {
          ws->arrive[0] = 0u;
          ws->arrive_x[0] = 0u;
          ws->tok_flag[0] = 0ull;
          ws->tag_base[0] = next_tag_base(ws, tag0 + static_cast<uint32_t>(p.n_tokens));
        } else if (serve) {
          // the host decides the next token (the mailbox), not the argmax
        } else if (stop_now) {
          // every CTA has arrived for this token and none adds again; tok_flag
          // still carries the stop id to the others (cleared by the last to see it)
          ws->arrive[0] = 0u;
          ws->arrive_x[0] = 0u;
          ws->tag_base[0] = next_tag_base(ws, tag0 + static_cast<uint32_t>(t) + 1u);
          st_release_u64(&ws->tok_flag[0], tok_word(t, best));
        } else {
          st_release_u64(&ws->tok_flag[0], tok_word(t, best));  // covers the CTA's writes above
        }
      }
    }
  }
}


// kTP: the tensor-parallel instantiation (peer accumulators, cross-GPU argmax);
// the single-GPU kernels carry none of that code.
template <bool kFused, bool kTraced, bool kTP>
__global__ void __launch_bounds__(kThreads, 1) decode_kernel(const DecodeParams p) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  Smem* sm = reinterpret_cast<Smem*>(smem_raw);
  Ctl c{sm, p.ws, p.timeout_ns, static_cast<int>(blockIdx.x),
        p.trace ? p.trace + (size_t)blockIdx.x * p.trace_cap : nullptr, p.trace_cap, p.err_flag};

  int token = p.token, pos = p.position, cl = p.cache_len;
  const uint32_t tag0 = __ldcg(&p.ws->tag_base[0]);
  // A workspace that still holds an earlier launch's error has stale counters
  // and sums: refuse to run on it (outputs poisoned) until it is reset.
  const uint32_t stale_err = __ldcg(&p.ws->error[0]);
  if (p.step != nullptr) {
    token = __ldcg(p.step + 0);
    pos = __ldcg(p.step + 1);
    cl = pos + 1;
  }

  // tensor parallel shape: 1, 2, 4 or 8 ranks, every peer workspace present,
  // the fused (transposed-down) schedule
  bool tp_ok = kTP ? (p.tp_size == 2 || p.tp_size == 4 || p.tp_size == 8) && kFused : p.tp_size == 1;
  tp_ok = tp_ok && p.tp_rank >= 0 && p.tp_rank < p.tp_size;
  for (int g = 0; g < kMaxTP; ++g)
    if (g < p.tp_size && p.tp_size > 1) tp_ok = tp_ok && p.peer_ws[g] != nullptr;
  int misaligned = 0;
  for (int i = threadIdx.x; i < kMaxLayers * 12; i += blockDim.x) {
    const int l = i / 12, f = i % 12;
    const __nv_bfloat16* v = nullptr;
    if (l >= p.layer_begin && l < p.layer_end) {
      if (f < 11) v = reinterpret_cast<const __nv_bfloat16* const*>(p.layers + l)[f];
      else if (p.down_t != nullptr) v = p.down_t[l];
    }
    misaligned |= (reinterpret_cast<uintptr_t>(v) & 15u) != 0u;
    sm->lwp[l][f] = v;
  }
  // every weight and vector is read with vector loads or bulk copies: 16-byte alignment
  misaligned |= ((reinterpret_cast<uintptr_t>(p.final_norm) | reinterpret_cast<uintptr_t>(p.input_residual) |
                  reinterpret_cast<uintptr_t>(p.residual_out)) & 15u) != 0u;
  misaligned = __syncthreads_or(misaligned);
  if (threadIdx.x == 0) {
    for (int s = 0; s < kSlots; ++s) {
      mbar_init(&sm->full[s], 1);
      mbar_init(&sm->empty[s], kConsumerWarps);
    }
    mbar_init(&sm->rxbar, 1);
    mbar_init(&sm->atbar, 1);
    mbar_arrive_expect_tx(&sm->atbar, kPairAttnBytes);  // the first pair exchange
    if (kFused) {  // the first layer's phase: one arrival plus the partner's SwiGLU bytes
      const Plan pp = make_plan(static_cast<int>(blockIdx.x) ^ 1, p.grid, p.group_size,
                                tp_shape(p.tp_rank, p.tp_size, kVocab));
      mbar_arrive_expect_tx(&sm->rxbar, static_cast<uint32_t>(pp.jb - pp.ja) * 4u);
    }
    sm->abort = 0;
    sm->peer_gone = 0;
    // SwiGLU values past this CTA's (or its partner's) row count stay zero: the
    // down projection reads kMaxJ of them
    for (int j = 0; j < 32; ++j) sm->m[j] = sm->mrx[j] = 0.f;
    sm->is_last = 0;
    fence_mbar_init();
  }
  __syncthreads();

  // Attention splits: a fixed count from the caller, or chosen per token from
  // its cache length (0 here).
  const int last_cl = cl + p.n_tokens - 1;
  const int splits = p.splits > 0 ? p.splits : 0;
  // Argument guard (uniform over the grid, before any wait).
  if (token < 0 || token >= kVocab || pos < 0 || pos + p.n_tokens > p.max_seq || cl < 1 ||
      last_cl > p.max_seq || p.grid != static_cast<int>(gridDim.x) || p.grid > kMaxGrid || p.grid < kMinGrid ||
      p.group_size * (kNKV / max(p.tp_size, 1)) > p.grid || p.grid % kCluster != 0 || splits < 0 ||
      splits > kMaxSplits || (splits > 1 && splits > p.group_size) || misaligned || !tp_ok) {
    if (threadIdx.x == 0 && blockIdx.x == 0) raise_error(c, kErrBadArgs, -1, -1, -1);
    // nothing was read or appended; the outputs say so
    if (threadIdx.x < kConsumerThreads)
      poison_outputs(p, part(kVocab, gridDim.x, blockIdx.x), part(kVocab, gridDim.x, blockIdx.x + 1), 0);
    return;
  }

  // Every CTA of the cluster has initialised its barriers before any remote
  // arrival, and none exits while a peer may still write into its shared memory.
  cluster_sync_all();
  const Plan pl = make_plan(blockIdx.x, p.grid, p.group_size, tp_shape(p.tp_rank, p.tp_size, kVocab));
  if (stale_err != 0u) {
    // Not uniform over the grid when this launch raised an error of its own
    // before a late CTA started: such a CTA skips its work, so its partner is
    // told (peer_gone) and every wait on it stays bounded.
    if (threadIdx.x == 0 && blockIdx.x == 0 && p.err_flag != nullptr)
      *reinterpret_cast<volatile uint32_t*>(p.err_flag) = stale_err;
    if (threadIdx.x == 0) st_cluster_u32(mapa_shared(smem_addr(&sm->peer_gone), cluster_ctarank() ^ 1u), 1u);
    if (threadIdx.x < kConsumerThreads) poison_outputs(p, pl.va, pl.vb, 0);
  } else if (threadIdx.x >= kConsumerThreads) {
    producer_run<kFused, kTraced, kTP>(p, pl, c, pos, cl, splits);
  } else {
    consumer_run<kFused, kTraced, kTP>(p, pl, c, token, pos, cl, splits, tag0);
  }
  cluster_sync_all();
}

// ---- host-side launch ----------------------------------------------------------
// The instantiations: transposed-down (fused) or reference-layout schedule,
// with or without trace stamps, and the fused tensor-parallel kernel.
template <bool kFused, bool kTraced, bool kTP>
cudaError_t set_smem_attr() {
  return cudaFuncSetAttribute(decode_kernel<kFused, kTraced, kTP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              static_cast<int>(kSmemBytes));
}

// Largest grid of kCluster-CTA clusters that can be resident at once (each CTA
// holds a whole SM's shared memory).
template <bool kFused, bool kTraced, bool kTP>
cudaError_t resident_ctas(int grid, int* out) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmemBytes;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kCluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int clusters = 0;
  const cudaError_t e = cudaOccupancyMaxActiveClusters(&clusters, decode_kernel<kFused, kTraced, kTP>, &cfg);
  *out = clusters * kCluster;
  return e;
}

// The CTAs wait on one another, so the whole grid must be resident: checked
// once per device against the cluster occupancy (the launch is refused with
// cudaErrorCooperativeLaunchTooLarge otherwise, as a cooperative launch would be).
cudaError_t launch_decode(const DecodeParams& p, cudaStream_t stream) {
  static int configured[64] = {0};
  static int resident[64] = {0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    if ((e = set_smem_attr<true, false, false>()) != cudaSuccess) return e;
    if ((e = set_smem_attr<false, false, false>()) != cudaSuccess) return e;
    if ((e = set_smem_attr<true, true, false>()) != cudaSuccess) return e;
    if ((e = set_smem_attr<false, true, false>()) != cudaSuccess) return e;
    if ((e = set_smem_attr<true, false, true>()) != cudaSuccess) return e;
    if ((e = set_smem_attr<true, true, true>()) != cudaSuccess) return e;
    int r[6];
    if ((e = resident_ctas<true, false, false>(p.grid, &r[0])) != cudaSuccess) return e;
    if ((e = resident_ctas<false, false, false>(p.grid, &r[1])) != cudaSuccess) return e;
    if ((e = resident_ctas<true, true, false>(p.grid, &r[2])) != cudaSuccess) return e;
    if ((e = resident_ctas<false, true, false>(p.grid, &r[3])) != cudaSuccess) return e;
    if ((e = resident_ctas<true, false, true>(p.grid, &r[4])) != cudaSuccess) return e;
    if ((e = resident_ctas<true, true, true>(p.grid, &r[5])) != cudaSuccess) return e;
    int m = r[0];
    for (int i = 1; i < 6; ++i) m = min(m, r[i]);
    resident[dev] = m;
    configured[dev] = 1;
  }
  if (p.grid > resident[dev]) return cudaErrorCooperativeLaunchTooLarge;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kCluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const bool fused = p.down_t != nullptr, traced = p.trace != nullptr;
  if (fused && p.tp_size > 1) {
    return traced ? cudaLaunchKernelEx(&cfg, decode_kernel<true, true, true>, p)
                  : cudaLaunchKernelEx(&cfg, decode_kernel<true, false, true>, p);
  }
  if (fused) {
    return traced ? cudaLaunchKernelEx(&cfg, decode_kernel<true, true, false>, p)
                  : cudaLaunchKernelEx(&cfg, decode_kernel<true, false, false>, p);
  }
  return traced ? cudaLaunchKernelEx(&cfg, decode_kernel<false, true, false>, p)
                : cudaLaunchKernelEx(&cfg, decode_kernel<false, false, false>, p);
}

size_t decode_smem_bytes() { return kSmemBytes; }

}  // namespace mkb
