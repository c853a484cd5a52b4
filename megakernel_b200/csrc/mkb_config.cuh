// Model constants, device data layouts and the static work split of the
// B200 decode kernel. Shared by the kernel (device), the launchers (host) and
// the host-side schedule query used by the CPU tests.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_bf16.h>

namespace mkb {

// Qwen3-0.6B dimensions (reference config.cuh:9-18).
constexpr int kHidden = 1024;
constexpr int kInter = 3072;
constexpr int kNQ = 16;
constexpr int kNKV = 8;
constexpr int kHeadDim = 128;
constexpr int kQSize = kNQ * kHeadDim;         // 2048
constexpr int kKVSize = kNKV * kHeadDim;       // 1024
constexpr int kQKVRows = kQSize + 2 * kKVSize; // 4096
constexpr int kVocab = 151936;
constexpr int kMaxLayers = 28;
static_assert(kMaxLayers <= 32, "split-attention tags carry the layer in 5 bits");
constexpr float kEps = 1e-6f;

// Execution shape: one CTA per SM, 8 consumer warps + 1 producer warp (at most
// 3 warps per scheduler, so up to 168 registers per thread).
constexpr int kConsumerWarps = 8;
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr int kThreads = kConsumerThreads + 32;
// Shared-memory weight ring: kSlots slots of kSlotBytes, filled by cp.async.bulk.
constexpr int kSlotBytes = 32768;
constexpr int kSlots = 6;
constexpr int kMaxGrid = 256;
constexpr int kMinGrid = 128;
// SwiGLU rows per CTA are at most kMaxJ (kInter split over at least kMinGrid CTAs).
constexpr int kMaxJ = (kInter + kMinGrid - 1) / kMinGrid;
constexpr int kMaxSplits = 32;
// Caches of at least this many keys are split between the two CTAs of a cluster
// pair that attend over the same KV head (partials swapped in shared memory).
constexpr int kPairSplitKeys = 65;

// Chunk geometry (rows per ring slot) for each streamed matrix. Rows read by
// the tensor-core GEMVs (ldmatrix) are stored at a padded stride so that the 8
// rows of an 8x8 matrix fall in different shared-memory banks.
constexpr int kRowStride = kHidden * 2 + 16;                     // 2064 B per padded 2 KB row
constexpr int kORowStride = 2 * kHeadDim * 2 + 16;              // 528 B per padded o_proj row slice
constexpr int kRowsPerChunk1024 = kSlotBytes / (kHidden * 2);   // 16 contiguous 2 KB rows (LM head, WdT)
constexpr int kQKVRowsPerChunk = kSlotBytes / kRowStride;       // 15 padded QKV rows
constexpr int kKeysPerChunk = kSlotBytes / 2 / (kHeadDim * 2);  // 64 keys: K half + V half
constexpr int kORowsPerChunk = kSlotBytes / kORowStride;        // 62 padded o_proj rows (2 heads)
constexpr int kGUPerChunk = (kSlotBytes / 2) / kRowStride;      // 7 gate rows + 7 up rows (padded)
constexpr int kDownRowsPerChunk = kSlotBytes / (kInter * 2);    // 5 rows of 6 KB (HF layout)

// Error codes written to Workspace::error[0].
enum ErrorCode : uint32_t {
  kErrNone = 0,
  kErrTimeoutTransition = 1,   // a grid transition counter never reached its target
  kErrTimeoutRing = 2,         // a shared-memory ring slot never filled / emptied
  kErrTimeoutToken = 3,        // the greedy token broadcast never arrived
  kErrBadArgs = 4,             // position / cache_len / token out of range
  kErrRange = 5,               // a partial sum outside the counted fixed-point range
};

// Counted fixed-point accumulators. A grid-wide sum of per-CTA partials is kept
// in one 64-bit word per element: bits 56-63 count the contributions, bits
// 0-55 hold sum(round(x * 2^28) + 2^47). Every contribution is one
// red.add.u64, so a reader that sees the expected count also sees the complete
// sum -- no counter, no fence -- and integer addition makes the sum independent
// of arrival order. |x| < 2^19 per contribution; up to 255 contributions (the
// biased field of 255 terms stays below 2^56).
constexpr int kAccShift = 28;
constexpr uint64_t kAccBias = 1ull << 47;
constexpr uint64_t kAccOne = 1ull << 56;
constexpr uint64_t kAccLowMask = kAccOne - 1ull;
// The down projection is split by output columns within a cluster pair: rank r
// reduces columns [kSlice r, kSlice (r + 1)) over both CTAs' intermediate rows
// (the partner's SwiGLU values arrive through distributed shared memory) and adds
// them into acc_down,
// spread over kDownCopies copies (cluster k adds into copy k % kDownCopies) to
// cut same-address atomic contention; readers add the copies.
constexpr int kCluster = 2;  // 74 co-resident pairs use all 148 SMs
constexpr int kSlice = 1024 / kCluster;  // output columns of the down projection per cluster rank
// Transposed-down rows in a ring slot, padded so that the 8 rows of an
// ldmatrix.trans 8x8 matrix fall in 8 different bank groups.
constexpr int kDRowStride = kSlice * 2 + 16;
constexpr int kDownKSteps = (kMaxJ + 15) / 16;  // MMA k-steps over a slot's rows
#ifndef MKB_DOWN_COPIES
#define MKB_DOWN_COPIES 2
#endif
constexpr int kDownCopies = MKB_DOWN_COPIES;
// Tensor parallelism: at most kMaxTP GPUs, each taking kNKV / tp_size KV heads,
// a contiguous block of SwiGLU rows and of vocabulary rows.
constexpr int kMaxTP = 8;

// Flags in DecodeParams::flags.
enum : int {
  kFlagLmHead = 1,          // run final norm + LM head + argmax
  kFlagSkipFinalNorm = 2,   // LM head consumes the residual as-is (isolated LM-head checks)
  kFlagAdvanceStep = 4,     // write the argmax and position+1 back into the step state
};

}  // namespace mkb

// Reference-compatible per-layer weight table: same 11 pointers in the same
// order as the reference's LayerWeights (config.cuh:77-89), so a device table
// built for the reference launcher can be handed to this one unchanged.
struct LayerWeights {
  const __nv_bfloat16* norm_weight;
  const __nv_bfloat16* q_weight;
  const __nv_bfloat16* k_weight;
  const __nv_bfloat16* v_weight;
  const __nv_bfloat16* q_norm_weight;
  const __nv_bfloat16* k_norm_weight;
  const __nv_bfloat16* o_proj_weight;
  const __nv_bfloat16* post_attn_norm_weight;
  const __nv_bfloat16* gate_proj_weight;
  const __nv_bfloat16* up_proj_weight;
  const __nv_bfloat16* down_proj_weight;
};

namespace mkb {

// Persistent device workspace. Zeroed once at allocation; a successful launch
// leaves every counter and accumulator at zero again, so launches (and CUDA
// graph replays) need no reset. After a launch that reported an error the
// owner must zero it before the next launch.
struct alignas(128) Workspace {
  // Grid transition counters, one per 128-byte line. Index [layer][k]:
  // k=0 QKV done, 1 attention+o_proj done, 2 gate/up(+down) done, 3 down done
  // (separate-down schedule only).
  uint32_t sync[kMaxLayers][4][32];
  uint32_t arrive[32];                       // end-of-token arrivals (last one reduces)
  // Token broadcast (multi-token launches): word 0 = sequence (t + 1) in the low
  // 32 bits, the token id in the high 32 bits, published by one release store.
  uint64_t tok_flag[16];
  uint32_t error[32];                        // [0] code, [1] cta, [2] layer, [3] stage, [4] token
  uint32_t tag_base[32];                     // [0]: tag of the last token decoded (tagged words)
  uint32_t stop_seen[32];                    // CTAs that saw a stop token (the last one resets tok_flag)
  uint32_t arrive_x[32];                     // end-of-token arrivals of the other GPUs' CTAs (tensor parallel)
  // Per-layer sums as counted fixed-point words (see kAccShift): o_proj
  // partials (one per KV head) and down-proj partials (one per CTA).
  uint64_t acc_mid[kMaxLayers][kHidden];
  uint64_t acc_down[kMaxLayers][kDownCopies][kHidden];
  // Tensor parallel: each GPU's complete down-projection sum, forwarded by one
  // CTA of every GPU into every GPU's copy (tp_size contributions per element).
  uint64_t acc_x[kMaxLayers][kHidden];
  // K/V append of (layer, KV head) published for a later token of the same
  // launch (two adds per token: the K and the V writer).
  uint32_t kv_ready[kMaxLayers][kNKV][32];
  // split attention partials as tagged words (value | tag << 32, the tag naming
  // token and layer): o[128], then m and l, per (KV head, split, Q head)
  uint64_t att_part[kNKV][kMaxSplits][2][kHeadDim + 2];
  float qkv[kQKVRows];
  // Raw QKV outputs of every layer as tagged words (value | tag << 32); the tag
  // of token t of a launch is tag_base + t + 1, so no reset is ever needed.
  uint64_t qkv_tagged[kMaxLayers][kQKVRows];
  float mlp[kInter];
  float resid[kHidden];
  // Greedy-token candidate of the current token: the largest argmax key over
  // the CTAs (red.max), read and reset by the last CTA to arrive.
  unsigned long long tok_best[16];
};

// Fields read or cleared with 16-byte vector accesses.
static_assert(offsetof(Workspace, acc_mid) % 16 == 0 && offsetof(Workspace, acc_down) % 16 == 0 &&
                  offsetof(Workspace, acc_x) % 16 == 0 &&
                  offsetof(Workspace, resid) % 16 == 0 && offsetof(Workspace, qkv_tagged) % 16 == 0 &&
                  offsetof(Workspace, att_part) % 16 == 0 && ((kHeadDim + 2) * 8) % 16 == 0,
              "workspace vector fields must be 16-byte aligned");

// Scratch of the batched prefill (mkb_prefill.cu), owned by the engine; cap rows.
struct PrefillScratch {
  float* h;                  // [cap, 1024] residual
  __nv_bfloat16* ah;         // [cap, 2048] GEMM A operand (normed activation, attention output), high part
  __nv_bfloat16* al;         //              remainder
  __nv_bfloat16* mh;         // [cap, 3072] SwiGLU output (the down GEMM's A operand), high part
  __nv_bfloat16* ml;         //              remainder
  float* qkv;                // [cap, 4096]
  float* q;                  // [cap, 2048] rotated, scaled queries
  __nv_bfloat16* vt;         // [8, 128, vt_cols] one layer's V cache transposed (key-contiguous)
  int vt_cols;               // max_seq rounded up to 128 keys
  uint32_t* err;             // device error word (a GEMM wait that expired)
  int cap;
};

// Launch parameters (passed by value; all pointers are device pointers).
struct DecodeParams {
  const __nv_bfloat16* embed;        // [V, H] token embedding (gather)
  const __nv_bfloat16* lm_head;      // [V, H] LM head rows (tied: == embed)
  const __nv_bfloat16* final_norm;   // [H]
  const LayerWeights* layers;        // device table, indexed by absolute layer
  const __nv_bfloat16* const* down_t;  // device array of transposed down weights
                                       // [I, H] per layer; null = reference layout
  const void* cos_table;             // [max_seq, 128]
  const void* sin_table;
  int rope_fp32;                     // 1: tables are FP32, 0: BF16
  __nv_bfloat16* k_cache;            // [L, 8, max_seq, 128]
  __nv_bfloat16* v_cache;
  int max_seq;
  int layer_begin, layer_end;        // layers [begin, end) run this launch
  int token, position, cache_len;    // used when step == nullptr
  int* step;                         // device {token, position, cache_len, count} or null
  int n_tokens;                      // greedy tokens decoded by this launch (>= 1)
  int flags;
  const float* input_residual;       // replaces the embedding gather when non-null
  float* logits;                     // [V] FP32 (last token of the launch) or null
  int* out_tokens;                   // [n_tokens] argmax ids or null
  float* residual_out;               // [H] final residual or null
  float* q_out;                      // raw QKV GEMV outputs (FP32)
  float* k_out;
  float* v_out;
  float* mlp_out;                    // SwiGLU output [I] (reference-layout schedule)
  Workspace* ws;
  int grid;                          // CTAs (== gridDim.x)
  int group_size;                    // CTAs per KV head in the attention stage
  int splits;                        // sequence splits of the attention (>= 1)
  unsigned long long timeout_ns;     // bound on every wait
  int withhold_cta;                  // test hook: this CTA never publishes its first
                                     // QKV arrival (-1 = off); the others time out
  unsigned long long* trace;         // optional [2*grid][trace_cap] stage time stamps
  int trace_cap;
  const int* prompt;                 // prefill: forced input tokens [n_tokens], LM head on the last only
  uint32_t* err_flag;                // optional (host-mapped) word that receives the error code
  int stop_token;                    // end the launch after generating this id (-1: none)
  int tp_rank, tp_size;              // tensor parallel position (size 1: single GPU)
  Workspace* peer_ws[kMaxTP];        // every rank's workspace as this GPU addresses it
                                     // (peer_ws[tp_rank] == ws)
  // Serve mode (both non-null): each token's input comes from the host --
  // mailbox {seq, token} in mapped pinned memory, token t taken once seq == t+1,
  // a negative token ends the launch -- and its argmax goes back to result
  // {seq, token} (token first, then seq = t+1).
  volatile int* mailbox;
  volatile int* result;
};

// Trace record: (code << 48) | (globaltimer ns & 0xffffffffffff). Row cta is
// written by consumer thread 0 of that CTA (rows grid..2*grid-1 are reserved).
// code = kind | stage << 2 | layer << 7 | token << 12.
enum TraceKind : uint32_t { kTrWaitBegin = 0, kTrWaitEnd = 1, kTrPublish = 2, kTrMark = 3 };
// Trace window: consumer stamps staged in shared memory for these layers.
constexpr int kTraceLayerLo = 8;
constexpr int kTraceLayers = 4;
constexpr int kTraceSmem = 192;

enum TraceStage : uint32_t {
  kStA = 0, kStBC = 1, kStDE = 2, kStE = 3, kStLM = 4, kStSplit = 5, kStToken = 6, kStEnd = 7,
  // sub-stage marks (kind kTrMark)
  kSubAInput = 8, kSubANorm = 9, kSubBCPrep = 10, kSubBCAttn = 11, kSubBCComb = 12,
  kSubDENorm = 13, kSubDEGU = 14, kSubDEDown = 15,
  kStRing = 16,   // consumer waited for a ring slot to fill
  kStSlot = 17,   // producer waited for a ring slot to empty (layer field = chunk index & 31)
  kStIssue = 18,  // producer issued a chunk
  // finer sub-stage marks of the consumer chain
  kSubAMma = 19,       // QKV: MMA tiles of a pass done
  kSubABar = 20,       // QKV: warp partials stashed, barrier passed
  kSubBCAttW = 21,     // attention: per-warp partials written, barrier passed
  kSubBCOMma = 22,     // o_proj: MMA tiles of a chunk done
  kSubBCOBar = 23,     // o_proj: barrier passed (sums follow)
  kSubDEMma = 24,      // gate/up: MMA tiles of a pass done
  kSubDEBar = 25,      // gate/up: barrier passed (sums follow)
  kSubDESilu = 26,     // SwiGLU values formed and sent, barrier passed
  kSubDEOwn = 27,      // down: own rows reduced
  kSubDERx = 28        // down: partner's SwiGLU values arrived
};

// ---------------------------------------------------------------------------
// Static work split (identical on host and device).
// ---------------------------------------------------------------------------
__host__ __device__ inline int part(int n, int parts, int i) {
  return (int)(((long long)n * i) / parts);
}

// This GPU's share of a tensor-parallel launch (size 1: everything).
struct TpShape {
  int rank, size;
  int hl, h0;     // local KV heads and the first global one
  int i0, i1;     // SwiGLU rows [i0, i1)
  int v0, v1;     // vocabulary rows [v0, v1)
};

__host__ __device__ inline TpShape tp_shape(int rank, int size, int vocab) {
  TpShape s;
  s.rank = rank;
  s.size = size;
  s.hl = kNKV / size;
  s.h0 = rank * s.hl;
  s.i0 = part(kInter, size, rank);
  s.i1 = part(kInter, size, rank + 1);
  s.v0 = part(vocab, size, rank);
  s.v1 = part(vocab, size, rank + 1);
  return s;
}

// This GPU's QKV rows in a local row space: its heads' q rows, then k rows,
// then v rows (2 * 128 * hl, 128 * hl, 128 * hl). A local row maps to the
// concatenated [Wq; Wk; Wv] row space; rows stay contiguous inside a segment.
__host__ __device__ inline int qkv_local_rows(const TpShape& s) { return 4 * kHeadDim * s.hl; }
__host__ __device__ inline int qkv_global_row(const TpShape& s, int r) {
  const int nq = 2 * kHeadDim * s.hl, nk = kHeadDim * s.hl;
  if (r < nq) return s.h0 * 2 * kHeadDim + r;
  if (r < nq + nk) return kQSize + s.h0 * kHeadDim + (r - nq);
  return kQSize + kKVSize + s.h0 * kHeadDim + (r - nq - nk);
}

struct Plan {
  int qa, qb;     // QKV rows [qa, qb) of this GPU's local row space (qkv_global_row)
  int in_bc;      // takes part in attention + o_proj
  int h, c;       // KV head (global) and index inside its group
  int hl;         // KV head index on this GPU (its KV-cache shard)
  int oa, ob;     // o_proj rows
  int ja, jb;     // gate/up rows (and rows of the transposed down weight)
  int da, db;     // down rows (reference layout)
  int va, vb;     // LM-head rows
};

__host__ __device__ inline Plan make_plan(int cta, int grid, int group_size, const TpShape& s) {
  Plan p;
  const int nq = qkv_local_rows(s);
  p.qa = part(nq, grid, cta);
  p.qb = part(nq, grid, cta + 1);
  const int nbc = s.hl * group_size;
  p.in_bc = cta < nbc;
  p.hl = p.in_bc ? cta / group_size : 0;
  p.h = s.h0 + p.hl;
  p.c = p.in_bc ? cta % group_size : 0;
  p.oa = p.in_bc ? part(kHidden, group_size, p.c) : 0;
  p.ob = p.in_bc ? part(kHidden, group_size, p.c + 1) : 0;
  p.ja = s.i0 + part(s.i1 - s.i0, grid, cta);
  p.jb = s.i0 + part(s.i1 - s.i0, grid, cta + 1);
  p.da = part(kHidden, grid, cta);
  p.db = part(kHidden, grid, cta + 1);
  p.va = s.v0 + part(s.v1 - s.v0, grid, cta);
  p.vb = s.v0 + part(s.v1 - s.v0, grid, cta + 1);
  return p;
}

// End of the QKV chunk that starts at local row r: at most kQKVRowsPerChunk
// rows, never crossing the q/k/v segment boundaries of the local row space.
__host__ __device__ inline int qkv_chunk_end(int r, int qb, const TpShape& s) {
  int e = r + kQKVRowsPerChunk;
  const int nq = 2 * kHeadDim * s.hl, nk = kHeadDim * s.hl;
  const int bound = r < nq ? nq : (r < nq + nk ? nq + nk : qkv_local_rows(s));
  if (e > bound) e = bound;
  if (e > qb) e = qb;
  return e;
}

// Keys [ka, kb) that CTA c of a group attends over.
__host__ __device__ inline void key_range(int cache_len, int splits, int c, int* ka, int* kb) {
  if (splits <= 1) { *ka = 0; *kb = cache_len; return; }
  if (c >= splits) { *ka = 0; *kb = 0; return; }
  *ka = part(cache_len, splits, c);
  *kb = part(cache_len, splits, c + 1);
}

// Both CTAs of cluster pair `cta / 2` attend over the same KV head (true for
// every pair when the head group size is even, as on 148 SMs).
__host__ __device__ inline bool pair_shares_head(int cta, int grid, int group_size, const TpShape& s) {
  const Plan a = make_plan(cta & ~1, grid, group_size, s), b = make_plan(cta | 1, grid, group_size, s);
  return a.in_bc && b.in_bc && a.h == b.h;
}

// Keys [ka, kb) this CTA attends over: its part of a split across the head
// group's CTAs (long caches), else its half when the cluster pair shares the
// head and the cache has at least kPairSplitKeys keys, else all keys.
__host__ __device__ inline void attn_keys(int cache_len, int splits, int c, bool pair, int rank, int* ka, int* kb) {
  if (splits > 1) {
    key_range(cache_len, splits, c, ka, kb);
  } else if (pair && cache_len >= kPairSplitKeys) {
    *ka = part(cache_len, 2, rank);
    *kb = part(cache_len, 2, rank + 1);
  } else {
    *ka = 0;
    *kb = cache_len;
  }
}

// Attention sequence splits at a cache length: up to kSplitMinKeys - 1 keys
// one range (halved between the CTAs of a cluster pair from kPairSplitKeys
// on), beyond that ranges of at most one 64-key chunk over the head group's
// CTAs (at most group_size of them), combined through tagged partials.
// Measured per token against the pair split below 385 keys (split from 129 or
// 257 keys on: +50 and +38 us/token at 200 and 300 keys) and against 256-key
// ranges above (-74, -68 and -17 us/token at 450, 1,000 and 3,800 keys).
constexpr int kSplitMinKeys = 385;
__host__ __device__ inline int choose_splits(int cache_len, int group_size) {
  if (cache_len < kSplitMinKeys) return 1;
  int s = (cache_len + kKeysPerChunk - 1) / kKeysPerChunk;
  if (s > group_size) s = group_size;
  if (s > kMaxSplits) s = kMaxSplits;
  return s;
}

}  // namespace mkb
