// Batched prompt prefill: every prompt token of a layer at once, on the
// Blackwell tensor cores (no counterpart in the reference, which prefills with
// Hugging Face, model.py:72-87, and copies the cache, model.py:79-87).
//
// Per layer, for the n prompt tokens (M = n rows):
//   RMSNorm (FP32 residual -> activation split into a BF16 high part and the BF16
//   remainder) -> one QKV GEMM whose epilogue applies the q/k RMSNorm + RoPE and
//   writes q, the K/V cache rows and V^T -> causal attention -> o_proj GEMM added
//   into the residual -> RMSNorm -> gate/up GEMM with the SwiGLU in its epilogue
//   -> down GEMM added into the residual. The last token's residual then goes
//   through the decode kernel's final norm + LM head + argmax.
//
// GEMMs (gemm_kernel): C[M, N] = (A_hi + A_lo)[M, K] * B[N, K]^T with tcgen05.mma
// (kind::f16, BF16 x BF16 -> FP32 in TMEM), persistent CTAs over 128 x 256 output
// tiles, K in steps of 64, operands brought in by TMA tiled loads with 128-byte
// swizzle through a 3-stage shared-memory ring; one warp issues the loads, one
// thread the MMAs into two TMEM accumulators, four warps read the finished one
// back (tcgen05.ld) for the epilogue while the next tile accumulates. Splitting
// the FP32 activation into two BF16 parts keeps the products to about 2^-16
// relative, the accuracy of the decode path's GEMVs.
//
// Attention (attn_tc_kernel): causal flash attention on tcgen05.mma, S and O in
// TMEM, q as BF16 high part + remainder, the probabilities as one BF16 operand,
// online softmax in the exp2 domain. attn_kernel (mma.sync m16n8k16) is the
// earlier kernel, kept behind MKB_PF_ATTN_TC=0 with the unfused QKV path.

#include <cstdint>
#include <cstdio>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "../../include/mkb200.h"
#include "mkb_config.cuh"
#include "mkb_ptx.cuh"
#include "mkb_tc.cuh"

namespace mkb {
namespace pf {

// Prefill attention: tcgen05 kernel (1) or the mma.sync kernel (0).
#ifndef MKB_PF_ATTN_TC
#define MKB_PF_ATTN_TC 1
#endif

constexpr int BM = 128, BK = 64;
constexpr int kTile = BM * BK * 2;  // 16 KB: one 128 x 64 BF16 A-operand tile
constexpr int kGemmThreads = 192;   // warp 0 TMA, warp 1 MMA (+ TMEM), warps 2-5 epilogue

// Output tiles of BM x kBN: kBN = 256 (N a multiple of 256, 3 stages of 64 KB)
// reads 1.5x fewer operand bytes per FLOP than kBN = 128 (4 stages of 48 KB).
template <int kBN>
struct GemmCfg {
  static constexpr int kStages = kBN == 256 ? 3 : 4;
  static constexpr int kTileB = kBN * BK * 2;
};
template <int kBN>
struct GemmSmem {
  uint8_t a_hi[GemmCfg<kBN>::kStages][kTile];
  uint8_t a_lo[GemmCfg<kBN>::kStages][kTile];
  uint8_t b[GemmCfg<kBN>::kStages][GemmCfg<kBN>::kTileB];
  uint64_t full[GemmCfg<kBN>::kStages];
  uint64_t empty[GemmCfg<kBN>::kStages];
  uint64_t acc_full[2];   // accumulator b holds a finished tile
  uint64_t acc_empty[2];  // the epilogue has read accumulator b
  uint32_t tmem_base;
  int err;
};
template <int kBN>
constexpr size_t gemm_smem() { return sizeof(GemmSmem<kBN>) + 1024; }  // + slack for the 1024-byte swizzle atoms
static_assert(gemm_smem<256>() <= 232448 && gemm_smem<128>() <= 232448, "GEMM shared memory");

enum EpiMode : int { kEpiStore = 0, kEpiAdd = 1, kEpiSwiGLU = 2, kEpiQKV = 3 };

__device__ __forceinline__ float rope_val(const void* table, int fp32, size_t idx) {
  return fp32 ? __ldg(static_cast<const float*>(table) + idx)
              : __bfloat162float(static_cast<const __nv_bfloat16*>(table)[idx]);
}
// entries idx .. idx + 3 (idx a multiple of 4) of an FP32 or BF16 table
__device__ __forceinline__ float4 table4(const void* table, int fp32, size_t idx) {
  if (fp32) return __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(table) + idx));
  const uint2 u = __ldg(reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(table) + idx));
  return make_float4(bf_lo(u.x), bf_hi(u.x), bf_lo(u.y), bf_hi(u.y));
}

struct GemmArgs {
  int M, N, K;                 // C [M, N]; K a multiple of 64
  float* c;                    // kEpiStore: C; kEpiAdd: residual += C (row stride ldc)
  int ldc;
  __nv_bfloat16* m_hi;         // kEpiSwiGLU: silu(gate) * up as high part / remainder
  __nv_bfloat16* m_lo;
  int ldm;
  // kEpiQKV (N = 4096: q, k, v columns of token rows at positions pos0 + row):
  // q/k RMSNorm + rotate-half RoPE, q scaled by log2(e) / sqrt(128) into q_hi /
  // q_lo [M, 2048], K and V rows into this layer's cache [8, max_seq, 128], V
  // also transposed into vt [8, 128, vt_cols]
  const __nv_bfloat16* qn;
  const __nv_bfloat16* kn;
  const void* cos_t;
  const void* sin_t;
  int rope_fp32, pos0, max_seq, vt_cols;
  __nv_bfloat16* kc_layer;
  __nv_bfloat16* vc_layer;
  __nv_bfloat16* q_hi;
  __nv_bfloat16* q_lo;
  __nv_bfloat16* vt;
  unsigned long long timeout_ns;
  uint32_t* err;
};

__device__ __forceinline__ bool wait_bounded(uint64_t* bar, uint32_t ph, unsigned long long timeout, int* err) {
  if (mbar_test(bar, ph)) return true;
  const uint64_t t0 = global_ns();
  while (!mbar_wait(bar, ph, 20000)) {
    if (*reinterpret_cast<volatile int*>(err) != 0) return false;
    if (global_ns() - t0 > timeout) {
      *reinterpret_cast<volatile int*>(err) = 1;
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ void split_store(__nv_bfloat16* hi, __nv_bfloat16* lo, const float* v, int n8) {
  // n8 groups of 8 values -> 16-byte stores of each part
  for (int g = 0; g < n8; ++g) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float a = v[8 * g + 2 * i], b = v[8 * g + 2 * i + 1];
      h[i] = pack_bf2(a, b);
      l[i] = pack_bf2(a - bf_lo(h[i]), b - bf_hi(h[i]));
    }
    reinterpret_cast<uint4*>(hi)[g] = make_uint4(h[0], h[1], h[2], h[3]);
    reinterpret_cast<uint4*>(lo)[g] = make_uint4(l[0], l[1], l[2], l[3]);
  }
}

// Persistent: CTA c computes output tiles c, c + gridDim.x, ... (row-block
// major). The TMA ring runs across tile boundaries, and TMEM holds two
// accumulators (2 x kBN columns), so the epilogue of one tile overlaps the MMAs
// of the next.
template <int kMode, int kBN>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap ta_hi, const __grid_constant__ CUtensorMap ta_lo,
                const __grid_constant__ CUtensorMap tb, const __grid_constant__ CUtensorMap tb2,
                const __grid_constant__ CUtensorMap tb3, const GemmArgs g) {
  constexpr int STAGES = GemmCfg<kBN>::kStages, kTileB = GemmCfg<kBN>::kTileB, BN = kBN;
  extern __shared__ uint8_t smem_raw[];
  GemmSmem<kBN>& sm =
      *reinterpret_cast<GemmSmem<kBN>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KT = g.K / BK;
  const int n_tiles_n = g.N / BN, n_tiles = n_tiles_n * ((g.M + BM - 1) / BM);
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sm.acc_full[b], 1);
      mbar_init(&sm.acc_empty[b], 4);  // one arrival per epilogue warp
    }
    sm.err = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(&sm.tmem_base, 2 * BN);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tbase = sm.tmem_base;

  if (warp == 0 && lane == 0) {
    tc::prefetch_tensormap(&ta_hi);
    tc::prefetch_tensormap(&ta_lo);
    tc::prefetch_tensormap(&tb);
    if (kMode == kEpiSwiGLU || kMode == kEpiQKV) tc::prefetch_tensormap(&tb2);
    if (kMode == kEpiQKV) tc::prefetch_tensormap(&tb3);
    int it = 0;  // k-steps issued, over all of this CTA's tiles
    for (int t = blockIdx.x; t < n_tiles && !sm.err; t += gridDim.x) {
      const int m0 = (t / n_tiles_n) * BM;
      const int n0 = (t % n_tiles_n) * BN;  // kEpiSwiGLU: SwiGLU columns [n0 / 2, n0 / 2 + BN / 2)
      for (int kt = 0; kt < KT; ++kt, ++it) {
        const int s = it % STAGES;
        if (it >= STAGES && !wait_bounded(&sm.empty[s], ((it / STAGES) - 1) & 1, g.timeout_ns, &sm.err)) break;
        mbar_arrive_expect_tx(&sm.full[s], 2 * kTile + kTileB);
        tc::tma_load_2d(sm.a_hi[s], &ta_hi, kt * BK, m0, &sm.full[s]);
        tc::tma_load_2d(sm.a_lo[s], &ta_lo, kt * BK, m0, &sm.full[s]);
        if (kMode == kEpiSwiGLU) {
          tc::tma_load_2d(sm.b[s], &tb, kt * BK, n0 / 2, &sm.full[s]);                // BN/2 gate rows
          tc::tma_load_2d(sm.b[s] + kTileB / 2, &tb2, kt * BK, n0 / 2, &sm.full[s]);  // BN/2 up rows
        } else if (kMode == kEpiQKV) {  // q, k or v weight rows (tiles never straddle two)
          const CUtensorMap* m = n0 < kQSize ? &tb : n0 < kQSize + kKVSize ? &tb2 : &tb3;
          const int r0 = n0 < kQSize ? n0 : n0 < kQSize + kKVSize ? n0 - kQSize : n0 - kQSize - kKVSize;
          tc::tma_load_2d(sm.b[s], m, kt * BK, r0, &sm.full[s]);
        } else {
          tc::tma_load_2d(sm.b[s], &tb, kt * BK, n0, &sm.full[s]);
        }
      }
    }
    // after a stop, wait (bounded) for the copies still in flight before leaving
    for (int k = it - 1; k >= 0 && k >= it - STAGES && sm.err; --k) {
      const uint64_t t0 = global_ns();
      while (!mbar_wait(&sm.full[k % STAGES], (k / STAGES) & 1, 20000))
        if (global_ns() - t0 > g.timeout_ns) break;
    }
  } else if (warp == 1 && lane == 0) {
    constexpr uint32_t idesc = tc::idesc_bf16_f32(BM, BN);
    const uint64_t dah0 = tc::desc_sw128(smem_addr(sm.a_hi[0])), dal0 = tc::desc_sw128(smem_addr(sm.a_lo[0])),
                   db0 = tc::desc_sw128(smem_addr(sm.b[0]));
    int it = 0, lt = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < n_tiles && ok; t += gridDim.x, ++lt) {
      const int b = lt & 1;
      if (lt >= 2 && !wait_bounded(&sm.acc_empty[b], ((lt >> 1) - 1) & 1, g.timeout_ns, &sm.err)) break;
      tc::fence_after_sync();
      const uint32_t acc = tbase + b * BN;
      for (int kt = 0; kt < KT; ++kt, ++it) {
        const int s = it % STAGES;
        if (!wait_bounded(&sm.full[s], (it / STAGES) & 1, g.timeout_ns, &sm.err)) {
          ok = false;
          break;
        }
        tc::fence_after_sync();
        const uint64_t dah = tc::desc_advance(dah0, s * kTile), dal = tc::desc_advance(dal0, s * kTile),
                       dbb = tc::desc_advance(db0, s * kTileB);
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
          const uint64_t db = tc::desc_advance(dbb, kk * 32);
          tc::mma_bf16_ss(acc, tc::desc_advance(dah, kk * 32), db, idesc, (kt | kk) != 0);
          tc::mma_bf16_ss(acc, tc::desc_advance(dal, kk * 32), db, idesc, 1u);
        }
        tc::commit(&sm.empty[s]);  // the stage is free once these MMAs have read it
      }
      if (ok) tc::commit(&sm.acc_full[b]);  // the tile's MMAs have all completed
    }
  } else if (warp >= 2) {
    const int q = warp & 3;  // TMEM lanes 32q .. 32q + 31 = tile rows
    const uint32_t lane_off = static_cast<uint32_t>(32 * q) << 16;
    int lt = 0;
    for (int t = blockIdx.x; t < n_tiles; t += gridDim.x, ++lt) {
      const int b = lt & 1;
      // tcgen05.ld is warp-wide: one decision per warp
      if (!__all_sync(0xffffffffu, wait_bounded(&sm.acc_full[b], (lt >> 1) & 1, g.timeout_ns, &sm.err))) break;
      tc::fence_after_sync();
      const int m0 = (t / n_tiles_n) * BM;
      const int n0 = (t % n_tiles_n) * BN;
      const int row = m0 + 32 * q + lane;
      const uint32_t lane_addr = tbase + b * BN + lane_off;
      if (kMode == kEpiQKV) {
        const int pos = g.pos0 + row;
#pragma unroll 1
        for (int hh = 0; hh < BN / kHeadDim; ++hh) {
          const int head = n0 / kHeadDim + hh;  // 0-15 q, 16-23 k, 24-31 v
          float x[kHeadDim];
#pragma unroll
          for (int c = 0; c < kHeadDim / 32; ++c) tc::tmem_ld32(lane_addr + kHeadDim * hh + 32 * c, x + 32 * c);
          if (row >= g.M) continue;
          if (head < kNQ + kNKV) {
            // the same arithmetic, in the same order, as qk_rope_kernel (whose
            // warp_sum adds the lanes' partials in a butterfly)
            const __nv_bfloat16* nw = head < kNQ ? g.qn : g.kn;
            float p[32];
#pragma unroll
            for (int t = 0; t < 32; ++t) {
              const float x0 = x[2 * t], x1 = x[2 * t + 1], x2 = x[2 * t + 64], x3 = x[2 * t + 65];
              p[t] = x0 * x0 + x1 * x1 + x2 * x2 + x3 * x3;
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1)
#pragma unroll
              for (int t = 0; t < o; ++t) p[t] = p[t] + p[t + o];
            const float rstd = rsqrtf(p[0] * (1.0f / kHeadDim) + kEps);
#pragma unroll
            for (int d = 0; d < kHeadDim; d += 4) {
              const uint2 w = __ldg(reinterpret_cast<const uint2*>(nw + d));
              x[d] = x[d] * rstd * bf_lo(w.x);
              x[d + 1] = x[d + 1] * rstd * bf_hi(w.x);
              x[d + 2] = x[d + 2] * rstd * bf_lo(w.y);
              x[d + 3] = x[d + 3] * rstd * bf_hi(w.y);
            }
            const size_t rb = (size_t)pos * kHeadDim;
#pragma unroll
            for (int d = 0; d < kHeadDim / 2; d += 4) {  // rotate-half: (d, d + 64) pairs
              const float4 c4 = table4(g.cos_t, g.rope_fp32, rb + d), s4 = table4(g.sin_t, g.rope_fp32, rb + d);
              const float cs[4] = {c4.x, c4.y, c4.z, c4.w}, sn[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float a = x[d + e], bv = x[d + e + 64];
                x[d + e] = a * cs[e] - bv * sn[e];
                x[d + e + 64] = bv * cs[e] + a * sn[e];
              }
            }
          }
          if (head < kNQ) {
            const float sc = 0.08838834764831845f * 1.4426950408889634f;  // 1/sqrt(128) * log2(e)
            const size_t o = (size_t)row * kQSize + head * kHeadDim;
#pragma unroll
            for (int d = 0; d < kHeadDim; d += 8) {
              uint32_t h[4], lo[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float a = x[d + 2 * e], bv = x[d + 2 * e + 1];
                h[e] = pack_bf2(a * sc, bv * sc);
                lo[e] = pack_bf2(a * sc - bf_lo(h[e]), bv * sc - bf_hi(h[e]));
              }
              *reinterpret_cast<uint4*>(g.q_hi + o + d) = make_uint4(h[0], h[1], h[2], h[3]);
              *reinterpret_cast<uint4*>(g.q_lo + o + d) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
            }
          } else {
            const int h = (head - kNQ) % kNKV;
            __nv_bfloat16* dst =
                (head < kNQ + kNKV ? g.kc_layer : g.vc_layer) + ((size_t)h * g.max_seq + pos) * kHeadDim;
#pragma unroll
            for (int d = 0; d < kHeadDim; d += 8)
              *reinterpret_cast<uint4*>(dst + d) = make_uint4(pack_bf2(x[d], x[d + 1]), pack_bf2(x[d + 2], x[d + 3]),
                                                              pack_bf2(x[d + 4], x[d + 5]), pack_bf2(x[d + 6], x[d + 7]));
            if (head >= kNQ + kNKV && g.vt != nullptr) {  // V^T: lanes hold consecutive keys
              __nv_bfloat16* col = g.vt + (size_t)h * kHeadDim * g.vt_cols + pos;
#pragma unroll
              for (int d = 0; d < kHeadDim; ++d) col[(size_t)d * g.vt_cols] = __float2bfloat16_rn(x[d]);
            }
          }
        }
      } else if (kMode == kEpiSwiGLU) {
#pragma unroll 1
        for (int half = 0; half < BN / 64; ++half) {
          float gv[32], uv[32];
          tc::tmem_ld32(lane_addr + 32 * half, gv);           // gate columns
          tc::tmem_ld32(lane_addr + BN / 2 + 32 * half, uv);  // up columns
          if (row < g.M) {
            float mv[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) mv[i] = gv[i] / (1.0f + expf(-gv[i])) * uv[i];  // silu(g) * u
            const size_t o = (size_t)row * g.ldm + n0 / 2 + 32 * half;
            split_store(g.m_hi + o, g.m_lo + o, mv, 4);
          }
        }
      } else {
#pragma unroll 1
        for (int cb = 0; cb < BN / 32; ++cb) {
          float v[32];
          tc::tmem_ld32(lane_addr + 32 * cb, v);
          if (row < g.M) {
            float4* dst = reinterpret_cast<float4*>(g.c + (size_t)row * g.ldc + n0 + 32 * cb);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              float4 x = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
              if (kMode == kEpiAdd) {
                const float4 r = dst[i];
                x.x += r.x; x.y += r.y; x.z += r.z; x.w += r.w;
              }
              dst[i] = x;
            }
          }
        }
      }
      // the accumulator has been read (tcgen05.ld waited): the MMAs may reuse it
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.acc_empty[b]);
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (threadIdx.x == 0 && sm.err && g.err) atomicCAS(g.err, 0u, static_cast<uint32_t>(kErrTimeoutRing));
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tbase, 2 * BN);
  }
}

// ---- the other prefill kernels --------------------------------------------------

// h[i] = E[ids[i]] (FP32), ids clamped to the vocabulary.
__global__ void embed_kernel(const int* __restrict__ ids, const __nv_bfloat16* __restrict__ embed, float* h) {
  const int i = blockIdx.x;
  const int tok = min(max(ids[i], 0), kVocab - 1);
  const uint2 u = __ldg(reinterpret_cast<const uint2*>(embed + (size_t)tok * kHidden) + threadIdx.x);
  reinterpret_cast<float4*>(h + (size_t)i * kHidden)[threadIdx.x] = make_float4(bf_lo(u.x), bf_hi(u.x), bf_lo(u.y), bf_hi(u.y));
}

// RMSNorm of residual row i (megakernel.cu:704-739 formula), written as the
// BF16 high part and the BF16 remainder (the two GEMM A operands). 256 threads.
__global__ void rmsnorm_split_kernel(const float* __restrict__ h, const __nv_bfloat16* __restrict__ w,
                                     __nv_bfloat16* xh, __nv_bfloat16* xl) {
  __shared__ float red[8];
  const int i = blockIdx.x, t = threadIdx.x;
  const float4 v = reinterpret_cast<const float4*>(h + (size_t)i * kHidden)[t];
  const float ss = warp_sum(v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w);
  if ((t & 31) == 0) red[t >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int k = 0; k < 8; ++k) tot += red[k];
  const float rstd = rsqrtf(tot * (1.0f / kHidden) + kEps);
  const uint2 wv = __ldg(reinterpret_cast<const uint2*>(w) + t);
  const float x[4] = {v.x * rstd * bf_lo(wv.x), v.y * rstd * bf_hi(wv.x), v.z * rstd * bf_lo(wv.y),
                      v.w * rstd * bf_hi(wv.y)};
  const uint32_t h01 = pack_bf2(x[0], x[1]), h23 = pack_bf2(x[2], x[3]);
  reinterpret_cast<uint2*>(xh + (size_t)i * kHidden)[t] = make_uint2(h01, h23);
  reinterpret_cast<uint2*>(xl + (size_t)i * kHidden)[t] =
      make_uint2(pack_bf2(x[0] - bf_lo(h01), x[1] - bf_hi(h01)), pack_bf2(x[2] - bf_lo(h23), x[3] - bf_hi(h23)));
}


// Per token (blockIdx.x) and head row (one warp per head: 16 q, 8 k, 8 v):
// q/k RMSNorm over 128 dims + rotate-half RoPE at the token's position
// (megakernel.cu:490-630), K/V rows into the BF16 cache, q pre-scaled by
// log2(e) / sqrt(128) for the exp2-domain softmax, written either as FP32
// (q_out) or as a BF16 high part and remainder (q_hi / q_lo, when not null).
// blockDim 256 = 8 heads; blockIdx.y picks the group of 8.
__global__ void qk_rope_kernel(const float* __restrict__ qkv, const __nv_bfloat16* __restrict__ qn,
                               const __nv_bfloat16* __restrict__ kn, const void* cos_t, const void* sin_t, int fp32,
                               int pos0, int layer, __nv_bfloat16* kc, __nv_bfloat16* vc, int max_seq, float* q_out,
                               __nv_bfloat16* q_hi, __nv_bfloat16* q_lo) {
  const int i = blockIdx.x;
  const int head = blockIdx.y * 8 + (threadIdx.x >> 5);  // 0-15 q, 16-23 k, 24-31 v
  const int lane = threadIdx.x & 31;
  const int pos = pos0 + i;
  const float* src = qkv + (size_t)i * kQKVRows + head * kHeadDim;  // q 0..2047, k 2048.., v 3072..
  const int d0 = 2 * lane;
  float x0 = src[d0], x1 = src[d0 + 1], x2 = src[d0 + 64], x3 = src[d0 + 65];
  if (head < 24) {
    const __nv_bfloat16* nw = head < 16 ? qn : kn;
    const float ss = warp_sum(x0 * x0 + x1 * x1 + x2 * x2 + x3 * x3);
    const float rstd = rsqrtf(ss * (1.0f / kHeadDim) + kEps);
    const float y0 = x0 * rstd * __bfloat162float(nw[d0]), y1 = x1 * rstd * __bfloat162float(nw[d0 + 1]);
    const float y2 = x2 * rstd * __bfloat162float(nw[d0 + 64]), y3 = x3 * rstd * __bfloat162float(nw[d0 + 65]);
    const size_t rb = (size_t)pos * kHeadDim;
    const float c0 = rope_val(cos_t, fp32, rb + d0), s0 = rope_val(sin_t, fp32, rb + d0);
    const float c1 = rope_val(cos_t, fp32, rb + d0 + 1), s1 = rope_val(sin_t, fp32, rb + d0 + 1);
    x0 = y0 * c0 - y2 * s0;
    x2 = y2 * c0 + y0 * s0;
    x1 = y1 * c1 - y3 * s1;
    x3 = y3 * c1 + y1 * s1;
  }
  if (head < 16) {
    const float sc = 0.08838834764831845f * 1.4426950408889634f;  // 1/sqrt(128) * log2(e)
    const size_t o = (size_t)i * kQSize + head * kHeadDim + d0;
    if (q_hi != nullptr) {
      const uint32_t h01 = pack_bf2(x0 * sc, x1 * sc), h23 = pack_bf2(x2 * sc, x3 * sc);
      *reinterpret_cast<uint32_t*>(q_hi + o) = h01;
      *reinterpret_cast<uint32_t*>(q_hi + o + 64) = h23;
      *reinterpret_cast<uint32_t*>(q_lo + o) = pack_bf2(x0 * sc - bf_lo(h01), x1 * sc - bf_hi(h01));
      *reinterpret_cast<uint32_t*>(q_lo + o + 64) = pack_bf2(x2 * sc - bf_lo(h23), x3 * sc - bf_hi(h23));
    } else {
      float* q = q_out + o;
      q[0] = x0 * sc;
      q[1] = x1 * sc;
      q[64] = x2 * sc;
      q[65] = x3 * sc;
    }
  } else {
    const int h = (head - 16) & 7;
    __nv_bfloat16* dst = (head < 24 ? kc : vc) + (((size_t)layer * kNKV + h) * max_seq + pos) * kHeadDim;
    *reinterpret_cast<__nv_bfloat162*>(dst + d0) = __floats2bfloat162_rn(x0, x1);
    *reinterpret_cast<__nv_bfloat162*>(dst + d0 + 64) = __floats2bfloat162_rn(x2, x3);
  }
}

// Causal attention over the cache for query tokens [64 blockIdx.x, +64) of Q
// head blockIdx.y; 4 warps x 16 query rows. Query token i sits at position
// pos0 + i and attends to keys [0, pos0 + i]. S = Q K^T and O = P V on
// mma.sync m16n8k16 (BF16 in, FP32 out) with Q split into high part +
// remainder and P as one BF16 part; K/V tiles of 64 keys in padded shared rows
// (conflict-free ldmatrix).
constexpr int kAttRow = kHeadDim + 8;  // 136 BF16 = 272 bytes per shared K/V row
// K/V tiles double-buffered: the next 64 keys are copied (cp.async, 16 bytes a
// thread at a time) while the tensor cores work on the current ones.
constexpr int kAttStages = 2;
[[maybe_unused]] constexpr size_t kAttSmem = size_t(kAttStages) * 2 * 64 * kAttRow * 2;  // 69,632 B
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__global__ void __launch_bounds__(128) attn_kernel(const float* __restrict__ q, const __nv_bfloat16* __restrict__ kc,
                                                   const __nv_bfloat16* __restrict__ vc, int n, int pos0, int layer,
                                                   int max_seq, __nv_bfloat16* oh, __nv_bfloat16* ol) {
  extern __shared__ __align__(16) uint8_t att_smem[];
  auto ks = reinterpret_cast<__nv_bfloat16(*)[64][kAttRow]>(att_smem);
  auto vs = reinterpret_cast<__nv_bfloat16(*)[64][kAttRow]>(att_smem + size_t(kAttStages) * 64 * kAttRow * 2);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hq = blockIdx.y, hk = hq >> 1;
  // causal work grows with the query block: the longest blocks go first, so
  // the short ones fill the tail of the grid
  const int i0 = (gridDim.x - 1 - blockIdx.x) * 64;
  const int g = lane >> 2, tq = lane & 3;
  const int r0 = i0 + warp * 16 + g, r1 = r0 + 8;  // this thread's two query rows (tokens)
  // Q fragments (A operand), high part and remainder, for the 8 k-steps of 16 dims
  uint32_t qa_h[8][4], qa_l[8][4];
  {
    const float* qr0 = q + (size_t)min(r0, n - 1) * kQSize + hq * kHeadDim;
    const float* qr1 = q + (size_t)min(r1, n - 1) * kQSize + hq * kHeadDim;
#pragma unroll
    for (int s = 0; s < 8; ++s) {
      const int c = 16 * s + 2 * tq;
      const float a[8] = {qr0[c], qr0[c + 1], qr1[c], qr1[c + 1], qr0[c + 8], qr0[c + 9], qr1[c + 8], qr1[c + 9]};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const uint32_t h = pack_bf2(a[2 * k], a[2 * k + 1]);
        qa_h[s][k] = h;
        qa_l[s][k] = pack_bf2(a[2 * k] - bf_lo(h), a[2 * k + 1] - bf_hi(h));
      }
    }
  }
  float o[16][4];
#pragma unroll
  for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m0r = -INFINITY, m1r = -INFINITY, l0 = 0.f, l1 = 0.f;
  const int last_key = pos0 + min(i0 + 63, n - 1);  // the block's last query attends up to here
  const size_t head_base = ((size_t)layer * kNKV + hk) * max_seq;
  // K and V rows k0 .. k0 + 63 into stage st (rows past the last key are
  // copied from the cache as they are and masked below)
  auto load_tile = [&](int k0, int st) {
    for (int e = threadIdx.x; e < 64 * 16; e += 128) {
      const int r = e >> 4, cidx = (e & 15) * 8;
      const int key = min(k0 + r, max_seq - 1);
      cp_async16(&ks[st][r][cidx], kc + (head_base + key) * kHeadDim + cidx);
      cp_async16(&vs[st][r][cidx], vc + (head_base + key) * kHeadDim + cidx);
    }
    cp_async_commit();
  };
  const int ntiles = last_key / 64 + 1;
  load_tile(0, 0);
  for (int it = 0; it < ntiles; ++it) {
    const int k0 = it * 64, st = it & 1;
    if (it + 1 < ntiles) {
      load_tile(k0 + 64, st ^ 1);
      cp_async_wait<1>();  // this tile's group has landed; the next one stays in flight
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    // S = Q K^T for 8 n-tiles of 8 keys
    float sacc[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      sacc[j][0] = sacc[j][1] = sacc[j][2] = sacc[j][3] = 0.f;
#pragma unroll
      for (int s2 = 0; s2 < 4; ++s2) {  // two k-steps per ldmatrix.x4
        uint32_t b0, b1, b2, b3;
        const int key = 8 * j + (lane & 7), dim = 32 * s2 + 8 * (lane >> 3);
        ldsm_x4(smem_addr(&ks[st][key][dim]), b0, b1, b2, b3);
        mma_bf16(sacc[j], qa_h[2 * s2][0], qa_h[2 * s2][1], qa_h[2 * s2][2], qa_h[2 * s2][3], b0, b1);
        mma_bf16(sacc[j], qa_l[2 * s2][0], qa_l[2 * s2][1], qa_l[2 * s2][2], qa_l[2 * s2][3], b0, b1);
        mma_bf16(sacc[j], qa_h[2 * s2 + 1][0], qa_h[2 * s2 + 1][1], qa_h[2 * s2 + 1][2], qa_h[2 * s2 + 1][3], b2, b3);
        mma_bf16(sacc[j], qa_l[2 * s2 + 1][0], qa_l[2 * s2 + 1][1], qa_l[2 * s2 + 1][2], qa_l[2 * s2 + 1][3], b2, b3);
      }
    }
    // causal mask and online softmax (rows r0, r1)
    const int lim0 = pos0 + r0, lim1 = pos0 + r1;
    float mx0 = m0r, mx1 = m1r;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int kk = k0 + 8 * j + 2 * tq;
      if (kk > lim0) sacc[j][0] = -INFINITY;
      if (kk + 1 > lim0) sacc[j][1] = -INFINITY;
      if (kk > lim1) sacc[j][2] = -INFINITY;
      if (kk + 1 > lim1) sacc[j][3] = -INFINITY;
      mx0 = fmaxf(mx0, fmaxf(sacc[j][0], sacc[j][1]));
      mx1 = fmaxf(mx1, fmaxf(sacc[j][2], sacc[j][3]));
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float sc0 = mx0 > -INFINITY ? ex2_approx(m0r - mx0) : 1.f;
    const float sc1 = mx1 > -INFINITY ? ex2_approx(m1r - mx1) : 1.f;
    m0r = mx0;
    m1r = mx1;
    float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      sacc[j][0] = sacc[j][0] > -INFINITY ? ex2_approx(sacc[j][0] - mx0) : 0.f;
      sacc[j][1] = sacc[j][1] > -INFINITY ? ex2_approx(sacc[j][1] - mx0) : 0.f;
      sacc[j][2] = sacc[j][2] > -INFINITY ? ex2_approx(sacc[j][2] - mx1) : 0.f;
      sacc[j][3] = sacc[j][3] > -INFINITY ? ex2_approx(sacc[j][3] - mx1) : 0.f;
      ps0 += sacc[j][0] + sacc[j][1];
      ps1 += sacc[j][2] + sacc[j][3];
    }
    ps0 += __shfl_xor_sync(0xffffffffu, ps0, 1);
    ps0 += __shfl_xor_sync(0xffffffffu, ps0, 2);
    ps1 += __shfl_xor_sync(0xffffffffu, ps1, 1);
    ps1 += __shfl_xor_sync(0xffffffffu, ps1, 2);
    l0 = l0 * sc0 + ps0;
    l1 = l1 * sc1 + ps1;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      o[j][0] *= sc0; o[j][1] *= sc0;
      o[j][2] *= sc1; o[j][3] *= sc1;
    }
    // O += P V: the S accumulators of n-tiles 2s, 2s+1 are the A fragment of
    // k-step s (16 keys); V^T fragments by ldmatrix.trans from the key rows
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      const float* pa = sacc[2 * s];
      const float* pb = sacc[2 * s + 1];
      const float pv[8] = {pa[0], pa[1], pa[2], pa[3], pb[0], pb[1], pb[2], pb[3]};
      uint32_t ah[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) ah[k] = pack_bf2(pv[2 * k], pv[2 * k + 1]);
#pragma unroll
      for (int j2 = 0; j2 < 8; ++j2) {  // two n-tiles of 8 dims per ldmatrix.x4.trans
        uint32_t b0, b1, b2, b3;
        const int key = 16 * s + (lane & 7) + 8 * ((lane >> 3) & 1), dim = 16 * j2 + 8 * (lane >> 4);
        ldsm_x4_trans(smem_addr(&vs[st][key][dim]), b0, b1, b2, b3);
        mma_bf16(o[2 * j2], ah[0], ah[1], ah[2], ah[3], b0, b1);
        mma_bf16(o[2 * j2 + 1], ah[0], ah[1], ah[2], ah[3], b2, b3);
      }
    }
    __syncthreads();  // every warp is done with stage st before it is refilled
  }
  // O / l -> high part and remainder of the o_proj A operand
  const float inv0 = 1.f / l0, inv1 = 1.f / l1;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int c = hq * kHeadDim + 8 * j + 2 * tq;
    if (r0 < n) {
      const float a = o[j][0] * inv0, b = o[j][1] * inv0;
      const uint32_t h = pack_bf2(a, b);
      *reinterpret_cast<uint32_t*>(oh + (size_t)r0 * kQSize + c) = h;
      *reinterpret_cast<uint32_t*>(ol + (size_t)r0 * kQSize + c) = pack_bf2(a - bf_lo(h), b - bf_hi(h));
    }
    if (r1 < n) {
      const float a = o[j][2] * inv1, b = o[j][3] * inv1;
      const uint32_t h = pack_bf2(a, b);
      *reinterpret_cast<uint32_t*>(oh + (size_t)r1 * kQSize + c) = h;
      *reinterpret_cast<uint32_t*>(ol + (size_t)r1 * kQSize + c) = pack_bf2(a - bf_lo(h), b - bf_hi(h));
    }
  }
}

// ---- causal attention on tcgen05 ---------------------------------------------------
//
// attn_tc_kernel: one CTA per (Q head, 128 query tokens). S = Q K^T and O = P V run
// on tcgen05.mma (M = 128 query rows, N = 128 keys or dims, accumulators in TMEM);
// q enters as a BF16 high part and remainder (two MMAs per k-step, as in the
// GEMMs), P as one BF16 operand. Keys come in tiles of 128: K rows straight from
// the cache (K-major for S), V from a per-layer transposed copy (v_transpose_kernel)
// so that V^T is K-major for O. Warp 0 issues the TMA loads (2-stage K and V^T
// rings), one thread of warp 1 the MMAs, warps 2-9 the softmax: each query row
// has two threads (warps w and w + 4 share TMEM lanes 32 (w % 4)..), each over
// 64 keys of a tile, exchanging their row maxima through shared memory. They
// read S from TMEM, keep the online softmax (exp2 domain; the reference max only
// moves when a row's maximum grows by more than 8, so O is rescaled in TMEM
// rarely and P stays within [0, 256]), and write P into shared memory in the
// MMA's 128-byte-swizzled layout. Two S buffers in TMEM let the tensor cores
// compute the next tile's scores while the softmax works on this one.
constexpr int kTcThreads = 320;
constexpr int kAtom = 128 * 128;  // 16 KB: 128 rows x 64 BF16, 128-byte swizzle
struct AttnTcSmem {
  uint8_t qh[2][kAtom];     // [dim half]: query rows
  uint8_t ql[2][kAtom];
  uint8_t k[2][2][kAtom];   // [stage][dim half]: key rows
  uint8_t vt[2][2][kAtom];  // [stage][key half]: dim rows
  uint8_t p[2][kAtom];      // [key half]: query rows
  float red[2][2][128];     // [tile parity][key half][row]: partial row maxima, then the row sums
  uint64_t q_full, k_full[2], k_empty[2], v_full[2], v_empty[2], s_full[2], p_full, o_done;
  uint64_t xbar[4];         // per row quarter: both softmax threads of its rows have posted
  uint32_t tmem_base;
  int err;
};
// No alignment slack fits beside the 224 KB of tiles: the kernel checks that the
// dynamic shared memory starts on a 1024-byte boundary (the swizzle atom) and
// reports an error otherwise.
constexpr size_t kAttTcSmem = sizeof(AttnTcSmem);
static_assert(kAttTcSmem <= 232448, "attention shared memory");
constexpr uint32_t kAttTmemCols = 512;  // S buffers at columns 0 and 128, O at 256

// Every lane of a warp waits; the warp goes on only if all of them saw the phase.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t ph, unsigned long long timeout, int* err) {
  return __all_sync(0xffffffffu, wait_bounded(bar, ph, timeout, err));
}

__global__ void __launch_bounds__(kTcThreads, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tq_hi, const __grid_constant__ CUtensorMap tq_lo,
                   const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tvt, int n, int pos0,
                   int max_seq, __nv_bfloat16* oh, __nv_bfloat16* ol, unsigned long long timeout_ns, uint32_t* err) {
  extern __shared__ uint8_t smem_raw[];
  if (smem_addr(smem_raw) & 1023u) {
    if (threadIdx.x == 0 && err) atomicCAS(err, 0u, static_cast<uint32_t>(kErrTimeoutRing));
    return;
  }
  AttnTcSmem& sm = *reinterpret_cast<AttnTcSmem*>(smem_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hq = blockIdx.x, hk = hq >> 1;
  // causal work grows with the query block: the longest blocks (of every head) go first
  const int i0 = (gridDim.y - 1 - blockIdx.y) * 128;
  const int nt = (pos0 + min(i0 + 127, n - 1)) / 128 + 1;  // key tiles up to the block's last query
  if (threadIdx.x == 0) {
    mbar_init(&sm.q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&sm.k_full[s], 1);
      mbar_init(&sm.k_empty[s], 1);
      mbar_init(&sm.v_full[s], 1);
      mbar_init(&sm.v_empty[s], 1);
      mbar_init(&sm.s_full[s], 1);
    }
    mbar_init(&sm.p_full, 8);  // one arrival per softmax warp
    mbar_init(&sm.o_done, 1);
    for (int q = 0; q < 4; ++q) mbar_init(&sm.xbar[q], 64);
    sm.err = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tc::tmem_alloc(&sm.tmem_base, kAttTmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tbase = sm.tmem_base, t_o = tbase + 256;

  if (warp == 0 && lane == 0) {
    tc::prefetch_tensormap(&tq_hi);
    tc::prefetch_tensormap(&tq_lo);
    tc::prefetch_tensormap(&tk);
    tc::prefetch_tensormap(&tvt);
    mbar_arrive_expect_tx(&sm.q_full, 4 * kAtom);
    for (int h = 0; h < 2; ++h) {
      tc::tma_load_2d(sm.qh[h], &tq_hi, hq * kHeadDim + 64 * h, i0, &sm.q_full);
      tc::tma_load_2d(sm.ql[h], &tq_lo, hq * kHeadDim + 64 * h, i0, &sm.q_full);
    }
    const int krow = hk * max_seq;  // this KV head's first cache row in the layer's map
    int k_issued = 0, v_issued = 0;
    // K(j) once S(j - 2) has read its stage, V(j) once PV(j - 2) has; issued in
    // the order the MMAs consume them (S(j + 1) runs before PV(j)), so a K tile
    // never queues behind the release of a V stage
    auto load_k = [&](int j) -> bool {
      const int st = j & 1;
      if (j >= 2 && !wait_bounded(&sm.k_empty[st], ((j >> 1) - 1) & 1, timeout_ns, &sm.err)) return false;
      mbar_arrive_expect_tx(&sm.k_full[st], 2 * kAtom);
      tc::tma_load_2d(sm.k[st][0], &tk, 0, krow + 128 * j, &sm.k_full[st]);
      tc::tma_load_2d(sm.k[st][1], &tk, 64, krow + 128 * j, &sm.k_full[st]);
      ++k_issued;
      return true;
    };
    if (load_k(0)) {
      for (int j = 0; j < nt; ++j) {
        if (j + 1 < nt && !load_k(j + 1)) break;
        const int st = j & 1;
        if (j >= 2 && !wait_bounded(&sm.v_empty[st], ((j >> 1) - 1) & 1, timeout_ns, &sm.err)) break;
        mbar_arrive_expect_tx(&sm.v_full[st], 2 * kAtom);
        tc::tma_load_2d(sm.vt[st][0], &tvt, 128 * j, hk * kHeadDim, &sm.v_full[st]);
        tc::tma_load_2d(sm.vt[st][1], &tvt, 128 * j + 64, hk * kHeadDim, &sm.v_full[st]);
        ++v_issued;
      }
    }
    // after a stop, wait (bounded) for the copies still in flight before leaving
    if (sm.err) {
      const uint64_t t0 = global_ns();
      while (!mbar_wait(&sm.q_full, 0, 20000) && global_ns() - t0 < timeout_ns) {
      }
      for (int j = max(k_issued - 2, 0); j < k_issued; ++j)
        while (!mbar_wait(&sm.k_full[j & 1], (j >> 1) & 1, 20000) && global_ns() - t0 < timeout_ns) {
        }
      for (int j = max(v_issued - 2, 0); j < v_issued; ++j)
        while (!mbar_wait(&sm.v_full[j & 1], (j >> 1) & 1, 20000) && global_ns() - t0 < timeout_ns) {
        }
    }
  } else if (warp == 1 && lane == 0) {
    constexpr uint32_t idesc = tc::idesc_bf16_f32(128, 128);
    const uint32_t qh = smem_addr(sm.qh[0]), ql = smem_addr(sm.ql[0]), pa = smem_addr(sm.p[0]);
    // S(j) = (Q_hi + Q_lo) K(j)^T into S buffer j & 1
    // descriptors formed once and advanced by compile-time offsets
    const uint64_t dqh = tc::desc_sw128(qh), dql = tc::desc_sw128(ql), dp = tc::desc_sw128(pa);
    const uint64_t dk0 = tc::desc_sw128(smem_addr(sm.k[0][0])), dv0 = tc::desc_sw128(smem_addr(sm.vt[0][0]));
    auto issue_s = [&](int j) -> bool {
      const int st = j & 1;
      if (!wait_bounded(&sm.k_full[st], (j >> 1) & 1, timeout_ns, &sm.err)) return false;
      tc::fence_after_sync();
      const uint64_t dk = tc::desc_advance(dk0, st * 2 * kAtom);
#pragma unroll
      for (int kk = 0; kk < kHeadDim / 16; ++kk) {
        const uint32_t off = (kk >> 2) * kAtom + (kk & 3) * 32;
        const uint64_t db = tc::desc_advance(dk, off);
        tc::mma_bf16_ss(tbase + 128 * st, tc::desc_advance(dqh, off), db, idesc, kk != 0);
        tc::mma_bf16_ss(tbase + 128 * st, tc::desc_advance(dql, off), db, idesc, 1u);
      }
      tc::commit(&sm.k_empty[st]);
      tc::commit(&sm.s_full[st]);
      return true;
    };
    if (wait_bounded(&sm.q_full, 0, timeout_ns, &sm.err) && issue_s(0)) {
      for (int j = 0; j < nt; ++j) {
        if (j + 1 < nt && !issue_s(j + 1)) break;
        // O (+)= P(j) V(j) once the softmax has written P(j) (and rescaled O)
        if (!wait_bounded(&sm.p_full, j & 1, timeout_ns, &sm.err)) break;
        if (!wait_bounded(&sm.v_full[j & 1], (j >> 1) & 1, timeout_ns, &sm.err)) break;
        tc::fence_after_sync();
        const uint64_t dv = tc::desc_advance(dv0, (j & 1) * 2 * kAtom);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = (kk >> 2) * kAtom + (kk & 3) * 32;
          tc::mma_bf16_ss(t_o, tc::desc_advance(dp, off), tc::desc_advance(dv, off), idesc, (j | kk) != 0);
        }
        tc::commit(&sm.v_empty[j & 1]);
        tc::commit(&sm.o_done);
      }
    }
  } else if (warp >= 2) {
    const int q4 = warp & 3;        // TMEM lanes 32 q4 .. + 31 = query rows
    const int g = (warp - 2) >> 2;  // keys 64 g .. + 63 of each tile, O columns 64 g .. + 63
    const int row = 32 * q4 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(32 * q4) << 16;
    const int lim = pos0 + i0 + row;  // this query's last key
    float m = 0.f, l = 0.f;           // reference max (exp2 domain) and this half's row sum
    // post v for the partner thread of this row, return the partner's value
    auto exchange = [&](int j, float v, float* out) -> bool {
      sm.red[j & 1][g][row] = v;
      mbar_arrive(&sm.xbar[q4]);  // release: the partner's wait sees the value
      if (!wait_bounded(&sm.xbar[q4], j & 1, timeout_ns, &sm.err)) return false;
      *out = sm.red[j & 1][g ^ 1][row];
      return true;
    };
    bool go = true;
    for (int j = 0; j < nt && go; ++j) {
      const int st = j & 1;
      go = warp_wait(&sm.s_full[st], (j >> 1) & 1, timeout_ns, &sm.err);
      if (!go) break;
      tc::fence_after_sync();
      uint32_t sr[2][32];
      tc::tmem_ld32_nowait(tbase + lane_off + 128 * st + 64 * g, sr[0]);
      tc::tmem_ld32_nowait(tbase + lane_off + 128 * st + 64 * g + 32, sr[1]);
      tc::tmem_wait_ld<true>(sr[0]);
      tc::tmem_wait_ld<false>(sr[1]);
      float s[64];
#pragma unroll
      for (int i = 0; i < 64; ++i) s[i] = __uint_as_float(sr[i >> 5][i & 31]);
      const int k0 = 128 * j + 64 * g;
      if (k0 + 63 > lim) {
#pragma unroll
        for (int i = 0; i < 64; ++i)
          if (k0 + i > lim) s[i] = -INFINITY;
      }
      float mx8[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) mx8[i] = s[i];
#pragma unroll
      for (int i = 8; i < 64; ++i) mx8[i & 7] = fmaxf(mx8[i & 7], s[i]);
      float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                       fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
      float mo;
      go = __all_sync(0xffffffffu, exchange(j, mx, &mo));
      if (!go) break;
      mx = fmaxf(mx, mo);  // the row's tile max, identical in both threads (key 0 <= lim: finite in tile 0)
      // the reference max moves (and O is rescaled) only when some row of the
      // warp grew by more than 8; the decision is warp-uniform (tcgen05.ld/st)
      // and the same in both warps of the rows
      float sc = 1.f;
      const bool rescale = j > 0 && __any_sync(0xffffffffu, mx > m + 8.f);
      if (j == 0) {
        m = mx;
      } else if (rescale) {
        sc = mx > m ? ex2_approx(m - mx) : 1.f;
        m = fmaxf(m, mx);
      }
      // P = 2^(S - m) in BF16 (ex2.approx gives 0 at -inf) while PV(j - 1) runs
      float rs[4] = {0.f, 0.f, 0.f, 0.f};
      uint32_t pw[32];
#pragma unroll
      for (int t = 0; t < 32; ++t) {
        const float pa = ex2_approx(s[2 * t] - m), pb = ex2_approx(s[2 * t + 1] - m);
        rs[t & 3] += pa + pb;
        pw[t] = pack_bf2(pa, pb);
      }
      if (j > 0) {
        // PV(j - 1) has completed: the P buffer is free and O may be rescaled
        go = warp_wait(&sm.o_done, (j - 1) & 1, timeout_ns, &sm.err);
        if (!go) break;
        tc::fence_after_sync();
        if (rescale) {
          l *= sc;
#pragma unroll 1
          for (int c = 0; c < 2; ++c) {
            float o[32];
            tc::tmem_ld32(t_o + lane_off + 64 * g + 32 * c, o);
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= sc;
            tc::tmem_st32(t_o + lane_off + 64 * g + 32 * c, o);
          }
        }
      }
      // row r of the 64-key atom at r * 128 bytes, 16-byte chunks swizzled by
      // r & 7 (the layout a 128-byte-swizzle TMA writes)
#pragma unroll
      for (int c = 0; c < 8; ++c)
        *reinterpret_cast<uint4*>(sm.p[g] + row * 128 + ((c ^ (row & 7)) << 4)) =
            make_uint4(pw[4 * c], pw[4 * c + 1], pw[4 * c + 2], pw[4 * c + 3]);
      l += (rs[0] + rs[1]) + (rs[2] + rs[3]);
      fence_proxy_async_shared();  // P is read by the tensor cores (async proxy)
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.p_full);
    }
    float lo = 0.f;
    if (go) go = __all_sync(0xffffffffu, exchange(nt, l, &lo));  // the row sum of both halves
    if (go) go = warp_wait(&sm.o_done, (nt - 1) & 1, timeout_ns, &sm.err);
    if (go) {
      tc::fence_after_sync();
      const int qi = i0 + row;
      const float inv = 1.f / (g == 0 ? l + lo : lo + l);
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        float o[32];
        tc::tmem_ld32(t_o + lane_off + 64 * g + 32 * c, o);
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] *= inv;
        if (qi < n) {
          const size_t off = (size_t)qi * kQSize + hq * kHeadDim + 64 * g + 32 * c;
          split_store(oh + off, ol + off, o, 4);
        }
      }
    }
  }
  tc::fence_before_sync();
  __syncthreads();
  if (threadIdx.x == 0 && sm.err && err) atomicCAS(err, 0u, static_cast<uint32_t>(kErrTimeoutRing));
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tbase, kAttTmemCols);
  }
}

// V^T of one layer: vt[hk][d][key] = v_cache[hk][key][d] for keys
// [64 blockIdx.x, +64) of KV head blockIdx.y, zeros at keys >= kv_len (the
// attention reads whole 128-key tiles; P is 0 there and so must V be).
__global__ void __launch_bounds__(256) v_transpose_kernel(const __nv_bfloat16* __restrict__ vc, int max_seq,
                                                           int kv_len, int vt_cols, __nv_bfloat16* __restrict__ vt) {
  __shared__ __align__(16) __nv_bfloat16 t[64][kHeadDim + 8];
  const int hk = blockIdx.y, k0 = blockIdx.x * 64;
  for (int e = threadIdx.x; e < 64 * 16; e += 256) {
    const int r = e >> 4, c = (e & 15) * 8;
    const int key = k0 + r;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (key < kv_len) v = *reinterpret_cast<const uint4*>(vc + ((size_t)hk * max_seq + key) * kHeadDim + c);
    *reinterpret_cast<uint4*>(&t[r][c]) = v;
  }
  __syncthreads();
  const unsigned short* tu = reinterpret_cast<const unsigned short*>(&t[0][0]);
  for (int e = threadIdx.x; e < kHeadDim * 8; e += 256) {
    const int d = e >> 3, kc = (e & 7) * 8;
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
      w[i] = uint32_t(tu[(kc + 2 * i) * (kHeadDim + 8) + d]) | (uint32_t(tu[(kc + 2 * i + 1) * (kHeadDim + 8) + d]) << 16);
    *reinterpret_cast<uint4*>(vt + ((size_t)hk * kHeadDim + d) * vt_cols + k0 + kc) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// ---- host side ---------------------------------------------------------------------
using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encoder() {
  static EncodeTiled fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiled>(p);
  }
  return fn;
}

// Row-major BF16 [rows, cols] as a 2-D tensor map with 64 x box_rows boxes and
// 128-byte swizzle (the K-major operand layout of the GEMM). Rows past the end
// read as zeros.
cudaError_t map_2d(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
  EncodeTiled enc = encoder();
  if (!enc) return cudaErrorNotSupported;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) || (cols * 2) % 16 || cols % BK) return cudaErrorMisalignedAddress;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * 2};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(BK), box_rows};
  const cuuint32_t es[2] = {1, 1};
  const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

template <int kMode, int kBN>
cudaError_t gemm_launch(const CUtensorMap& ah, const CUtensorMap& al, const CUtensorMap& b, const CUtensorMap& b2,
                        const CUtensorMap& b3, const GemmArgs& g, cudaStream_t stream) {
  static int configured[64] = {0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    e = cudaFuncSetAttribute(gemm_kernel<kMode, kBN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)gemm_smem<kBN>());
    if (e != cudaSuccess) return e;
    configured[dev] = 1;
  }
  if (g.K % BK || g.N % kBN || g.M < 1) return cudaErrorInvalidValue;
  static int sms[64] = {0};
  if (!sms[dev] && (e = cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess)
    return e;
  const int tiles = (g.N / kBN) * ((g.M + BM - 1) / BM);
  gemm_kernel<kMode, kBN><<<tiles < sms[dev] ? tiles : sms[dev], kGemmThreads, gemm_smem<kBN>(), stream>>>(ah, al, b, b2,
                                                                                                         b3, g);
  return cudaGetLastError();
}
constexpr int kPfBN = 256;  // the prefill's GEMMs (every N a multiple of 256)

}  // namespace pf

// Prefill of n prompt tokens at positions pos0 .. pos0 + n - 1 for layers
// [0, n_layers): called by the engine (mkb_host.cu) with its scratch buffers.
cudaError_t prefill_layers(const LayerWeights* host_layers, int n_layers, const __nv_bfloat16* embed,
                           const void* cos_t, const void* sin_t, int rope_fp32, __nv_bfloat16* kc, __nv_bfloat16* vc,
                           int max_seq, const int* ids, int n, int pos0, const PrefillScratch& s, cudaStream_t stream) {
  using namespace pf;
  if (n < 1 || n > s.cap || pos0 < 0 || pos0 + n > max_seq) return cudaErrorInvalidValue;
#if MKB_PF_ATTN_TC
  if (s.vt_cols < pos0 + n || s.vt_cols % 128) return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kAttTcSmem);
  // queries as BF16 high part / remainder in the SwiGLU buffers (free until the gate/up GEMM)
  CUtensorMap tqh, tql, tvt;
  if (e == cudaSuccess) e = map_2d(&tqh, s.mh, n, kQSize, 128);
  if (e == cudaSuccess) e = map_2d(&tql, s.ml, n, kQSize, 128);
  if (e == cudaSuccess) e = map_2d(&tvt, s.vt, kNKV * kHeadDim, s.vt_cols, 128);
#else
  cudaError_t e = cudaFuncSetAttribute(attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kAttSmem);
#endif
  if (e != cudaSuccess) return e;
  embed_kernel<<<n, kHidden / 4, 0, stream>>>(ids, embed, s.h);
  if ((e = cudaGetLastError()) != cudaSuccess) return e;
  // activation operand maps over the scratch (K = 1024, 2048 or 3072 columns)
  CUtensorMap a1h, a1l, a2h, a2l, a3h, a3l;
  if ((e = map_2d(&a1h, s.ah, n, kHidden, BM)) != cudaSuccess) return e;
  if ((e = map_2d(&a1l, s.al, n, kHidden, BM)) != cudaSuccess) return e;
  if ((e = map_2d(&a2h, s.ah, n, kQSize, BM)) != cudaSuccess) return e;
  if ((e = map_2d(&a2l, s.al, n, kQSize, BM)) != cudaSuccess) return e;
  if ((e = map_2d(&a3h, s.mh, n, kInter, BM)) != cudaSuccess) return e;
  if ((e = map_2d(&a3l, s.ml, n, kInter, BM)) != cudaSuccess) return e;
  GemmArgs g = {};
  g.M = n;
  g.timeout_ns = 1000000000ull;
  g.err = s.err;
  for (int l = 0; l < n_layers; ++l) {
    const LayerWeights& w = host_layers[l];
    CUtensorMap bq, bk, bv, bo, bg, bu, bd;
    if ((e = map_2d(&bq, w.q_weight, kQSize, kHidden, kPfBN)) != cudaSuccess) return e;
    if ((e = map_2d(&bk, w.k_weight, kKVSize, kHidden, kPfBN)) != cudaSuccess) return e;
    if ((e = map_2d(&bv, w.v_weight, kKVSize, kHidden, kPfBN)) != cudaSuccess) return e;
    if ((e = map_2d(&bo, w.o_proj_weight, kHidden, kQSize, kPfBN)) != cudaSuccess) return e;
    if ((e = map_2d(&bg, w.gate_proj_weight, kInter, kHidden, kPfBN / 2)) != cudaSuccess) return e;
    if ((e = map_2d(&bu, w.up_proj_weight, kInter, kHidden, kPfBN / 2)) != cudaSuccess) return e;
    if ((e = map_2d(&bd, w.down_proj_weight, kHidden, kInter, kPfBN)) != cudaSuccess) return e;
    // input RMSNorm
    rmsnorm_split_kernel<<<n, kHidden / 4, 0, stream>>>(s.h, w.norm_weight, s.ah, s.al);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    g.K = kHidden;
#if MKB_PF_ATTN_TC
    // one GEMM over the q, k and v weights; its epilogue applies the q/k RMSNorm
    // and RoPE, writes q (BF16 high part / remainder, into the SwiGLU buffers,
    // free until the gate/up GEMM), the K/V cache rows and V^T of the new keys
    const size_t layer_rows = (size_t)l * kNKV * max_seq;  // this layer's first cache row
    g.N = kQKVRows;
    g.qn = w.q_norm_weight;
    g.kn = w.k_norm_weight;
    g.cos_t = cos_t;
    g.sin_t = sin_t;
    g.rope_fp32 = rope_fp32;
    g.pos0 = pos0;
    g.max_seq = max_seq;
    g.kc_layer = kc + layer_rows * kHeadDim;
    g.vc_layer = vc + layer_rows * kHeadDim;
    g.q_hi = s.mh;
    g.q_lo = s.ml;
    g.vt = s.vt;
    g.vt_cols = s.vt_cols;
    if ((e = gemm_launch<kEpiQKV, kPfBN>(a1h, a1l, bq, bk, bv, g, stream)) != cudaSuccess) return e;
    if (pos0 > 0) {  // V^T of the keys cached before this prefill (rows of V^T past them: zeros or old finite values)
      v_transpose_kernel<<<dim3((pos0 + 63) / 64, kNKV), 256, 0, stream>>>(g.vc_layer, max_seq, pos0 + n, s.vt_cols,
                                                                          s.vt);
      if ((e = cudaGetLastError()) != cudaSuccess) return e;
    }
    CUtensorMap tk;
    if ((e = map_2d(&tk, kc + layer_rows * kHeadDim, (uint64_t)kNKV * max_seq, kHeadDim, 128)) != cudaSuccess) return e;
    attn_tc_kernel<<<dim3(kNQ, (n + 127) / 128), kTcThreads, kAttTcSmem, stream>>>(
        tqh, tql, tk, tvt, n, pos0, max_seq, s.ah, s.al, g.timeout_ns, s.err);
#else
    // three GEMMs into the [n, 4096] buffer, then q/k norm + RoPE with the K/V rows into the cache
    g.ldc = kQKVRows;
    g.N = kQSize;
    g.c = s.qkv;
    if ((e = gemm_launch<kEpiStore, kPfBN>(a1h, a1l, bq, bq, bq, g, stream)) != cudaSuccess) return e;
    g.N = kKVSize;
    g.c = s.qkv + kQSize;
    if ((e = gemm_launch<kEpiStore, kPfBN>(a1h, a1l, bk, bk, bk, g, stream)) != cudaSuccess) return e;
    g.c = s.qkv + kQSize + kKVSize;
    if ((e = gemm_launch<kEpiStore, kPfBN>(a1h, a1l, bv, bv, bv, g, stream)) != cudaSuccess) return e;
    qk_rope_kernel<<<dim3(n, 4), 256, 0, stream>>>(s.qkv, w.q_norm_weight, w.k_norm_weight, cos_t, sin_t, rope_fp32,
                                                   pos0, l, kc, vc, max_seq, s.q, nullptr, nullptr);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    attn_kernel<<<dim3((n + 63) / 64, kNQ), 128, kAttSmem, stream>>>(s.q, kc, vc, n, pos0, l, max_seq, s.ah, s.al);
#endif
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    // o_proj added into the residual
    g.K = kQSize;
    g.N = kHidden;
    g.ldc = kHidden;
    g.c = s.h;
    if ((e = gemm_launch<kEpiAdd, kPfBN>(a2h, a2l, bo, bo, bo, g, stream)) != cudaSuccess) return e;
    // post-attention RMSNorm -> gate/up with SwiGLU -> down added into the residual
    rmsnorm_split_kernel<<<n, kHidden / 4, 0, stream>>>(s.h, w.post_attn_norm_weight, s.ah, s.al);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    g.K = kHidden;
    g.N = 2 * kInter;  // 128-column tiles = 64 gate + 64 up columns
    g.m_hi = s.mh;  // a separate buffer: the GEMM still reads s.ah / s.al
    g.m_lo = s.ml;
    g.ldm = kInter;
    if ((e = gemm_launch<kEpiSwiGLU, kPfBN>(a1h, a1l, bg, bu, bu, g, stream)) != cudaSuccess) return e;
    g.K = kInter;
    g.N = kHidden;
    g.c = s.h;
    g.ldc = kHidden;
    if ((e = gemm_launch<kEpiAdd, kPfBN>(a3h, a3l, bd, bd, bd, g, stream)) != cudaSuccess) return e;
  }
  return cudaSuccess;
}

// C[M, N] = (A_hi + A_lo) B^T through the prefill GEMM (test entry point).
cudaError_t gemm_split(const __nv_bfloat16* a_hi, const __nv_bfloat16* a_lo, const __nv_bfloat16* b, float* c, int M,
                       int N, int K, uint32_t* err, cudaStream_t stream) {
  using namespace pf;
  CUtensorMap ah, al, bm;
  cudaError_t e;
  if ((e = map_2d(&ah, a_hi, M, K, BM)) != cudaSuccess) return e;
  if ((e = map_2d(&al, a_lo, M, K, BM)) != cudaSuccess) return e;
  const bool wide = N % 256 == 0;  // 256-column tiles where N allows, else 128
  if ((e = map_2d(&bm, b, N, K, wide ? 256 : 128)) != cudaSuccess) return e;
  GemmArgs g = {};
  g.M = M;
  g.N = N;
  g.K = K;
  g.c = c;
  g.ldc = N;
  g.timeout_ns = 1000000000ull;
  g.err = err;
  return wide ? gemm_launch<kEpiStore, 256>(ah, al, bm, bm, bm, g, stream)
              : gemm_launch<kEpiStore, 128>(ah, al, bm, bm, bm, g, stream);
}

}  // namespace mkb
