// Host side of libmkb200.so: the C ABI declared in include/mkb200.h.
//
//  * launch_decode_kernel -- drop-in for the reference launcher
//    (megakernel.cu:898-994): same arguments, reference weight layout.
//  * mkb_decode            -- explicit-argument launch of the same kernel.
//  * mkb_engine_*          -- resident engine: device LayerWeights table,
//    transposed down weights, workspace, step state and a CUDA graph of the
//    per-token launch stay alive across tokens (the reference rebuilt and freed
//    its table on every call, pytorch_binding.cu:84-126).

#include <atomic>
#include <chrono>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <vector>

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "../../include/mkb200.h"
#include "mkb_config.cuh"

namespace mkb {
cudaError_t launch_decode(const DecodeParams& p, cudaStream_t stream);
size_t decode_smem_bytes();
cudaError_t prefill_layers(const LayerWeights* host_layers, int n_layers, const __nv_bfloat16* embed,
                           const void* cos_t, const void* sin_t, int rope_fp32, __nv_bfloat16* kc, __nv_bfloat16* vc,
                           int max_seq, const int* ids, int n, int pos0, const PrefillScratch& s, cudaStream_t stream);
cudaError_t gemm_split(const __nv_bfloat16* a_hi, const __nv_bfloat16* a_lo, const __nv_bfloat16* b, float* c, int M,
                       int N, int K, uint32_t* err, cudaStream_t stream);
}  // namespace mkb

using namespace mkb;

namespace {

constexpr unsigned long long kDefaultTimeoutNs = 1000000000ull;  // 1 s per wait

struct DeviceInfo {
  int sms = 0;
  void* ws = nullptr;
  // Pinned, mapped word that receives the first in-kernel error of a launch on
  // `ws` (host view / device view); checked before the next launch on `ws`.
  uint32_t* h_err = nullptr;
  uint32_t* d_err = nullptr;
};
std::mutex g_mu;
DeviceInfo g_dev[64];

cudaError_t device_info(int dev, DeviceInfo** out) {
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lk(g_mu);
  DeviceInfo& d = g_dev[dev];
  if (d.sms == 0) {
    cudaError_t e = cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
  }
  *out = &d;
  return cudaSuccess;
}

cudaError_t default_ws(int dev, void** out) {
  DeviceInfo* d = nullptr;
  cudaError_t e = device_info(dev, &d);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lk(g_mu);
  if (d->ws == nullptr) {
    void* p = nullptr;
    uint32_t* h = nullptr;
    uint32_t* dv = nullptr;
    e = cudaHostAlloc(reinterpret_cast<void**>(&h), 32, cudaHostAllocMapped);
    if (e != cudaSuccess) return e;
    *reinterpret_cast<volatile uint32_t*>(h) = 0u;
    e = cudaHostGetDevicePointer(reinterpret_cast<void**>(&dv), h, 0);
    if (e != cudaSuccess) { cudaFreeHost(h); return e; }
    e = cudaMalloc(&p, sizeof(Workspace));
    if (e != cudaSuccess) { cudaFreeHost(h); return e; }
    e = cudaMemset(p, 0, sizeof(Workspace));
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) { cudaFree(p); cudaFreeHost(h); return e; }
    d->ws = p;
    d->h_err = h;
    d->d_err = dv;
  }
  *out = d->ws;
  return cudaSuccess;
}

int grid_for(int sms) { return sms > kMaxGrid ? kMaxGrid : sms; }

// Fill DecodeParams from the C argument block; resolves every default.
cudaError_t to_params(const mkb_decode_args* a, DecodeParams* p, DeviceInfo** dflt = nullptr) {
  if (a == nullptr) return cudaErrorInvalidValue;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  DeviceInfo* d = nullptr;
  e = device_info(dev, &d);
  if (e != cudaSuccess) return e;
  void* ws = a->workspace;
  if (dflt) *dflt = nullptr;
  if (ws == nullptr) {
    e = default_ws(dev, &ws);
    if (e != cudaSuccess) return e;
    if (dflt) *dflt = d;
  }
  std::memset(p, 0, sizeof(*p));
  p->embed = static_cast<const __nv_bfloat16*>(a->embed);
  p->lm_head = static_cast<const __nv_bfloat16*>(a->lm_head ? a->lm_head : a->embed);
  p->final_norm = static_cast<const __nv_bfloat16*>(a->final_norm);
  p->layers = static_cast<const LayerWeights*>(a->layers);
  p->down_t = static_cast<const __nv_bfloat16* const*>(a->down_t);
  p->cos_table = a->cos_table;
  p->sin_table = a->sin_table;
  p->rope_fp32 = a->rope_fp32;
  p->k_cache = static_cast<__nv_bfloat16*>(a->k_cache);
  p->v_cache = static_cast<__nv_bfloat16*>(a->v_cache);
  p->max_seq = a->max_seq;
  p->layer_begin = a->layer_begin;
  p->layer_end = a->layer_end;
  p->token = a->token;
  p->position = a->position;
  p->cache_len = a->cache_len;
  p->step = a->step;
  p->n_tokens = a->n_tokens < 1 ? 1 : a->n_tokens;
  p->flags = a->flags;
  p->input_residual = a->input_residual;
  p->logits = a->logits;
  p->out_tokens = a->out_tokens;
  p->residual_out = a->residual_out;
  Workspace* w = static_cast<Workspace*>(ws);
  p->q_out = a->q_out ? a->q_out : w->qkv;
  p->k_out = a->k_out ? a->k_out : w->qkv + kQSize;
  p->v_out = a->v_out ? a->v_out : w->qkv + kQSize + kKVSize;
  p->mlp_out = a->mlp_out ? a->mlp_out : w->mlp;
  p->ws = w;
  p->grid = a->grid > 0 ? a->grid : grid_for(d->sms);
  if (p->grid > d->sms || p->grid > kMaxGrid || p->grid < kMinGrid || p->grid % kCluster != 0)
    return cudaErrorInvalidConfiguration;
  p->tp_rank = a->tp_size > 1 ? a->tp_rank : 0;
  p->tp_size = a->tp_size > 1 ? a->tp_size : 1;
  if (p->tp_size != 1 && p->tp_size != 2 && p->tp_size != 4 && p->tp_size != 8) return cudaErrorInvalidValue;
  if (p->tp_rank < 0 || p->tp_rank >= p->tp_size) return cudaErrorInvalidValue;
  for (int g = 0; g < kMaxTP; ++g) p->peer_ws[g] = nullptr;
  if (p->tp_size > 1) {
    if (!a->down_t) return cudaErrorInvalidValue;  // tensor parallel runs the transposed-down schedule
    for (int g = 0; g < p->tp_size; ++g) {
      if (!a->peer_workspaces[g]) return cudaErrorInvalidValue;
      p->peer_ws[g] = static_cast<Workspace*>(a->peer_workspaces[g]);
    }
    if (p->peer_ws[p->tp_rank] != w) return cudaErrorInvalidValue;
  } else {
    p->peer_ws[0] = w;
  }
  p->group_size = p->grid / (kNKV / p->tp_size);
  p->splits = a->splits > 0 ? a->splits : 0;  // 0: chosen on the device per token
  if (p->splits > kMaxSplits || p->splits > p->group_size) return cudaErrorInvalidValue;
  p->timeout_ns = a->timeout_ns ? a->timeout_ns : kDefaultTimeoutNs;
  p->withhold_cta = a->withhold_cta;
  p->trace = a->trace;
  p->trace_cap = a->trace ? a->trace_cap : 0;
  p->prompt = a->prompt_tokens;
  p->err_flag = a->err_flag ? a->err_flag : (a->workspace == nullptr ? d->d_err : nullptr);
  p->stop_token = a->stop_token;
  p->mailbox = a->mailbox;
  p->result = a->result;
  if ((a->mailbox == nullptr) != (a->result == nullptr)) return cudaErrorInvalidValue;
  if (p->stop_token >= kVocab) return cudaErrorInvalidValue;
  // Host-side validation of what the host can see (the kernel re-checks the rest).
  if (!p->embed || !p->layers || !p->k_cache || !p->v_cache || !p->cos_table || !p->sin_table)
    return cudaErrorInvalidValue;
  if (p->layer_begin < 0 || p->layer_end < p->layer_begin || p->layer_end > kMaxLayers) return cudaErrorInvalidValue;
  if ((p->flags & kFlagLmHead) && !(p->flags & kFlagSkipFinalNorm) && !p->final_norm) return cudaErrorInvalidValue;
  if (p->max_seq < 1) return cudaErrorInvalidValue;
  if (!a->step) {
    if (a->token < 0 || a->token >= kVocab) return cudaErrorInvalidValue;
    if (a->position < 0 || a->position + p->n_tokens > a->max_seq) return cudaErrorInvalidValue;
    if (a->cache_len < 1 || a->cache_len + p->n_tokens - 1 > a->max_seq) return cudaErrorInvalidValue;
  }
  auto misaligned = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) != 0u; };
  if (misaligned(p->embed) || misaligned(p->lm_head) || misaligned(p->k_cache) || misaligned(p->v_cache))
    return cudaErrorMisalignedAddress;
  return cudaSuccess;
}

// down [1024, 3072] -> down_t [kCluster][3072][1024 / kCluster] BF16: the
// transpose with its 1024 output columns split into kCluster contiguous column
// blocks (block r = the columns cluster rank r reduces), through 32x32 tiles.
__global__ void transpose_down_kernel(const __nv_bfloat16* __restrict__ src, __nv_bfloat16* __restrict__ dst) {
  __shared__ __nv_bfloat16 tile[32][33];
  const int bx = blockIdx.x * 32, by = blockIdx.y * 32;  // bx over 3072 (j), by over 1024 (output column)
  for (int i = threadIdx.y; i < 32; i += blockDim.y)
    tile[i][threadIdx.x] = src[(size_t)(by + i) * kInter + bx + threadIdx.x];
  __syncthreads();
  constexpr int kHalf = kHidden / kCluster;
  const int col = by + threadIdx.x;
  for (int i = threadIdx.y; i < 32; i += blockDim.y)
    dst[((size_t)(col / kHalf) * kInter + bx + i) * kHalf + col % kHalf] = tile[threadIdx.x][i];
}

}  // namespace

extern "C" {

int mkb_version(void) { return 1; }
size_t mkb_workspace_bytes(void) { return sizeof(Workspace); }
size_t mkb_smem_bytes(void) { return decode_smem_bytes(); }

void mkb_decode_args_init(mkb_decode_args* a) {
  std::memset(a, 0, sizeof(*a));
  a->n_tokens = 1;
  a->withhold_cta = -1;
  a->stop_token = -1;
  a->layer_end = kMaxLayers;
  a->flags = MKB_FLAG_LM_HEAD;
}

cudaError_t mkb_decode(const mkb_decode_args* a, cudaStream_t stream) {
  DecodeParams p;
  DeviceInfo* dflt = nullptr;
  cudaError_t e = to_params(a, &p, &dflt);
  if (e != cudaSuccess) return e;
  if (dflt != nullptr && a->err_flag == nullptr) {
    volatile uint32_t* flag = dflt->h_err;
    if (*flag != 0u) {
      // An earlier asynchronous launch on the device's workspace failed in the
      // kernel: report it here (as CUDA reports asynchronous errors), reset the
      // workspace, and do not launch on its stale state.
      fprintf(stderr, "mkb200: an earlier launch on device workspace failed in the kernel: %s\n",
              mkb_error_name(*flag));
      e = cudaMemsetAsync(dflt->ws, 0, sizeof(Workspace), stream);
      if (e != cudaSuccess) return e;
      *flag = 0u;
      return cudaErrorLaunchFailure;
    }
  }
  return launch_decode(p, stream);
}

cudaError_t launch_decode_kernel(int token_id, const void* embed_weight, const void* lm_head_weight,
                                 const void* final_norm_weight, const void* layer_weights,
                                 const void* cos_table, const void* sin_table, void* k_cache, void* v_cache,
                                 void* hidden_buffer, void* g_residual, void* g_activations,
                                 void* g_attn_output, void* g_normalized, void* g_mlp_intermediate,
                                 void* g_logits, void* g_q, void* g_k, void* g_v, int position, int cache_len,
                                 int max_seq_len, cudaStream_t stream) {
  (void)hidden_buffer;
  (void)g_activations;
  (void)g_attn_output;
  (void)g_normalized;
  mkb_decode_args a;
  mkb_decode_args_init(&a);
  a.embed = embed_weight;
  a.lm_head = lm_head_weight;
  a.final_norm = final_norm_weight;
  a.layers = layer_weights;
  a.cos_table = cos_table;
  a.sin_table = sin_table;
  a.rope_fp32 = 0;
  a.k_cache = k_cache;
  a.v_cache = v_cache;
  a.max_seq = max_seq_len;
  a.layer_begin = 0;
  a.layer_end = kMaxLayers;
  a.token = token_id;
  a.position = position;
  a.cache_len = cache_len;
  a.flags = MKB_FLAG_LM_HEAD;
  a.logits = static_cast<float*>(g_logits);
  a.residual_out = static_cast<float*>(g_residual);
  a.q_out = static_cast<float*>(g_q);
  a.k_out = static_cast<float*>(g_k);
  a.v_out = static_cast<float*>(g_v);
  a.mlp_out = static_cast<float*>(g_mlp_intermediate);
  return mkb_decode(&a, stream);
}

cudaError_t mkb_default_workspace(int device, void** out) { return default_ws(device, out); }

cudaError_t mkb_workspace_reset(void* workspace, cudaStream_t stream) {
  {
    // resetting a device's own workspace also clears its pending error word
    std::lock_guard<std::mutex> lk(g_mu);
    for (DeviceInfo& d : g_dev)
      if (d.ws != nullptr && d.ws == workspace) *reinterpret_cast<volatile uint32_t*>(d.h_err) = 0u;
  }
  return cudaMemsetAsync(workspace, 0, sizeof(Workspace), stream);
}

cudaError_t mkb_workspace_status(const void* workspace, uint32_t out[8]) {
  const Workspace* w = static_cast<const Workspace*>(workspace);
  return cudaMemcpy(out, w->error, 8 * sizeof(uint32_t), cudaMemcpyDeviceToHost);
}

cudaError_t mkb_workspace_tag_base(void* workspace, const uint32_t* set, uint32_t* get) {
  if (workspace == nullptr) return cudaErrorInvalidValue;
  Workspace* w = static_cast<Workspace*>(workspace);
  cudaError_t e = cudaSuccess;
  if (set != nullptr) e = cudaMemcpy(w->tag_base, set, sizeof(uint32_t), cudaMemcpyHostToDevice);
  if (e == cudaSuccess && get != nullptr) e = cudaMemcpy(get, w->tag_base, sizeof(uint32_t), cudaMemcpyDeviceToHost);
  return e;
}

const char* mkb_error_name(uint32_t code) {
  switch (code) {
    case kErrNone: return "ok";
    case kErrTimeoutTransition: return "timeout waiting for a grid transition";
    case kErrTimeoutRing: return "timeout waiting for a shared-memory ring slot";
    case kErrTimeoutToken: return "timeout waiting for the greedy token broadcast";
    case kErrBadArgs: return "bad arguments (range or alignment) seen on the device";
    case kErrRange: return "a partial sum outside the counted fixed-point range (|x| >= 2^19 or NaN)";
    default: return "unknown";
  }
}

cudaError_t mkb_transpose_down(const void* down, void* down_t, cudaStream_t stream) {
  dim3 grid(kInter / 32, kHidden / 32), block(32, 8);
  transpose_down_kernel<<<grid, block, 0, stream>>>(static_cast<const __nv_bfloat16*>(down),
                                                    static_cast<__nv_bfloat16*>(down_t));
  return cudaGetLastError();
}

int mkb_plan_query(int grid, int cta, int32_t out[16]) {
  if (grid < kNKV || cta < 0 || cta >= grid) return -1;
  const int gs = grid / kNKV;
  const Plan p = make_plan(cta, grid, gs, tp_shape(0, 1, kVocab));
  const int32_t v[14] = {p.qa, p.qb, p.in_bc, p.h, p.c, p.oa, p.ob, p.ja, p.jb, p.da, p.db, p.va, p.vb, gs};
  for (int i = 0; i < 14; ++i) out[i] = v[i];
  return 0;
}
int mkb_choose_splits(int cache_len, int group_size) { return choose_splits(cache_len, group_size); }
void mkb_key_range(int cache_len, int splits, int c, int32_t out[2]) {
  int a, b;
  key_range(cache_len, splits, c, &a, &b);
  out[0] = a;
  out[1] = b;
}
int mkb_qkv_chunk_end(int r, int qb) { return qkv_chunk_end(r, qb, tp_shape(0, 1, kVocab)); }
int mkb_plan_query_tp(int grid, int cta, int tp_rank, int tp_size, int32_t out[16]) {
  if (tp_size < 1 || tp_size > kMaxTP || kNKV % tp_size || tp_rank < 0 || tp_rank >= tp_size) return -1;
  const TpShape s = tp_shape(tp_rank, tp_size, kVocab);
  if (grid < s.hl || cta < 0 || cta >= grid) return -1;
  const int gs = grid / s.hl;
  const Plan p = make_plan(cta, grid, gs, s);
  const int32_t v[15] = {p.qa, p.qb, p.in_bc, p.h, p.c, p.oa, p.ob, p.ja, p.jb, p.da, p.db, p.va, p.vb, gs, p.hl};
  for (int i = 0; i < 15; ++i) out[i] = v[i];
  return 0;
}
int mkb_qkv_global_row(int tp_rank, int tp_size, int local_row) {
  return qkv_global_row(tp_shape(tp_rank, tp_size, kVocab), local_row);
}
int mkb_attn_keys(int cache_len, int splits, int grid, int cta, int32_t out[2]) {
  const int gs = grid / kNKV;
  const TpShape s = tp_shape(0, 1, kVocab);
  const Plan p = make_plan(cta, grid, gs, s);
  const bool pair = pair_shares_head(cta, grid, gs, s);
  int a, b;
  attn_keys(cache_len, splits, p.c, pair, cta & 1, &a, &b);
  out[0] = a;
  out[1] = b;
  return pair ? 1 : 0;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Resident engine
// ---------------------------------------------------------------------------
struct mkb_engine {
  int device = 0;
  int n_layers = 0;
  int max_seq = 0;
  int grid = 0;
  int tp_size = 1;                            // > 1: tensor-parallel rank
  bool tp_ready = true;                       // false until mkb_engine_tp_attach
  LayerWeights* d_layers = nullptr;
  __nv_bfloat16* d_down_t_buf = nullptr;      // n_layers * [3072, 1024]
  __nv_bfloat16** d_down_t = nullptr;         // n_layers pointers
  void* ws = nullptr;
  int* d_step = nullptr;                      // {token, position, -, count}
  int* d_pf = nullptr;                        // [max_seq] prefill launch ids (last one used)
  float* d_logits = nullptr;
  bool own_logits = false;
  // Pinned, mapped host words: [0..1] (token, position) copied in each step,
  // [4] the argmax, stored there by the kernel's last CTA (no copy back),
  // [5] the first in-kernel error code of a launch (checked by the next call).
  int* h_io = nullptr;
  int* d_io = nullptr;                        // device address of h_io
  cudaGraphExec_t graph = nullptr;
  cudaStream_t cap_stream = nullptr;
  mkb_decode_args step_args;
  std::vector<LayerWeights> host_layers;      // the layer table as the host sees it (prefill tensor maps)
  // serve session: mailbox = h_io[2..3] {seq, token}, result = h_io[6..7] {seq, argmax}
  bool serving = false;
  int serve_seq = 0;
  int serve_max = 0;
  unsigned long long serve_timeout = 0;
  cudaStream_t serve_stream = nullptr;
  PrefillScratch pf = {};                     // batched prefill scratch, allocated on first use
  void* pf_block = nullptr;
};

namespace {
void engine_free(mkb_engine* e) {
  if (!e) return;
  if (e->graph) cudaGraphExecDestroy(e->graph);
  if (e->cap_stream) cudaStreamDestroy(e->cap_stream);
  cudaFree(e->d_layers);
  cudaFree(e->d_down_t_buf);
  cudaFree(e->d_down_t);
  cudaFree(e->ws);
  cudaFree(e->d_step);
  cudaFree(e->d_pf);
  if (e->own_logits) cudaFree(e->d_logits);
  if (e->h_io) cudaFreeHost(e->h_io);
  cudaFree(e->pf_block);
  delete e;
}

cudaError_t engine_check_status(mkb_engine* e) {
  uint32_t st[8];
  cudaError_t err = mkb_workspace_status(e->ws, st);
  if (err != cudaSuccess) return err;
  reinterpret_cast<volatile int*>(e->h_io)[5] = 0;
  if (st[0] != 0) {
    fprintf(stderr, "mkb200: in-kernel error %u (%s) cta=%u layer=%d stage=%d token=%d\n", st[0],
            mkb_error_name(st[0]), st[1], static_cast<int>(st[2]), static_cast<int>(st[3]),
            static_cast<int>(st[4]));
    cudaMemset(e->ws, 0, sizeof(Workspace));
    cudaDeviceSynchronize();
    return cudaErrorLaunchFailure;
  }
  return cudaSuccess;
}
// An earlier asynchronous engine launch (generate, prefill) that failed in the
// kernel is reported by the next engine call: workspace status printed and
// reset, cudaErrorLaunchFailure returned, nothing launched.
cudaError_t engine_report_earlier(mkb_engine* e, cudaStream_t stream) {
  if (!e->tp_ready) return cudaErrorInvalidValue;  // a tensor-parallel rank before mkb_engine_tp_attach
  if (e->serving) return cudaErrorInvalidValue;    // a serve session holds the engine
  if (reinterpret_cast<volatile int*>(e->h_io)[5] == 0) return cudaSuccess;
  cudaError_t err = cudaStreamSynchronize(stream);
  if (err != cudaSuccess) return err;
  err = engine_check_status(e);
  return err != cudaSuccess ? err : cudaErrorLaunchFailure;
}
}  // namespace

extern "C" {

cudaError_t mkb_engine_create(const mkb_model* m, mkb_engine** out) {
  if (!m || !out || !m->layer_weights || m->n_layers < 1 || m->n_layers > kMaxLayers || m->max_seq < 1)
    return cudaErrorInvalidValue;
  *out = nullptr;
  mkb_engine* e = new mkb_engine();
  cudaError_t err = cudaGetDevice(&e->device);
#define MKB_TRY(x)        \
  do {                    \
    err = (x);            \
    if (err != cudaSuccess) { engine_free(e); return err; } \
  } while (0)
  if (err != cudaSuccess) { engine_free(e); return err; }
  DeviceInfo* d = nullptr;
  MKB_TRY(device_info(e->device, &d));
  e->grid = grid_for(d->sms);
  e->tp_size = m->tp_size > 1 ? m->tp_size : 1;
  if (e->tp_size != 1 && e->tp_size != 2 && e->tp_size != 4 && e->tp_size != 8) { engine_free(e); return cudaErrorInvalidValue; }
  if (e->tp_size > 1 && !m->fused_down) { engine_free(e); return cudaErrorInvalidValue; }
  e->tp_ready = e->tp_size == 1;
  e->n_layers = m->n_layers;
  e->max_seq = m->max_seq;

  std::vector<LayerWeights> host(m->n_layers);
  for (int l = 0; l < m->n_layers; ++l) {
    const void* const* w = m->layer_weights + (size_t)l * 11;
    for (int i = 0; i < 11; ++i)
      if (w[i] == nullptr || (reinterpret_cast<uintptr_t>(w[i]) & 15u)) { engine_free(e); return cudaErrorInvalidValue; }
    host[l] = LayerWeights{static_cast<const __nv_bfloat16*>(w[0]), static_cast<const __nv_bfloat16*>(w[1]),
                           static_cast<const __nv_bfloat16*>(w[2]), static_cast<const __nv_bfloat16*>(w[3]),
                           static_cast<const __nv_bfloat16*>(w[4]), static_cast<const __nv_bfloat16*>(w[5]),
                           static_cast<const __nv_bfloat16*>(w[6]), static_cast<const __nv_bfloat16*>(w[7]),
                           static_cast<const __nv_bfloat16*>(w[8]), static_cast<const __nv_bfloat16*>(w[9]),
                           static_cast<const __nv_bfloat16*>(w[10])};
  }
  e->host_layers = host;
  MKB_TRY(cudaMalloc(&e->d_layers, sizeof(LayerWeights) * m->n_layers));
  MKB_TRY(cudaMemcpy(e->d_layers, host.data(), sizeof(LayerWeights) * m->n_layers, cudaMemcpyHostToDevice));
  if (m->fused_down) {
    const size_t per = (size_t)kInter * kHidden;
    MKB_TRY(cudaMalloc(&e->d_down_t_buf, per * sizeof(__nv_bfloat16) * m->n_layers));
    std::vector<__nv_bfloat16*> ptrs(m->n_layers);
    for (int l = 0; l < m->n_layers; ++l) {
      ptrs[l] = e->d_down_t_buf + per * l;
      MKB_TRY(mkb_transpose_down(host[l].down_proj_weight, ptrs[l], 0));
    }
    MKB_TRY(cudaMalloc(&e->d_down_t, sizeof(void*) * m->n_layers));
    MKB_TRY(cudaMemcpy(e->d_down_t, ptrs.data(), sizeof(void*) * m->n_layers, cudaMemcpyHostToDevice));
  }
  MKB_TRY(cudaMalloc(&e->ws, sizeof(Workspace)));
  MKB_TRY(cudaMemset(e->ws, 0, sizeof(Workspace)));
  MKB_TRY(cudaMalloc(&e->d_step, 4 * sizeof(int)));
  MKB_TRY(cudaMemset(e->d_step, 0, 4 * sizeof(int)));
  MKB_TRY(cudaMalloc(&e->d_pf, sizeof(int) * m->max_seq));
  if (m->logits) {
    e->d_logits = m->logits;
  } else {
    MKB_TRY(cudaMalloc(&e->d_logits, sizeof(float) * kVocab));
    e->own_logits = true;
  }
  MKB_TRY(cudaHostAlloc(&e->h_io, 8 * sizeof(int), cudaHostAllocMapped));
  for (int i = 0; i < 8; ++i) e->h_io[i] = 0;
  MKB_TRY(cudaHostGetDevicePointer(reinterpret_cast<void**>(&e->d_io), e->h_io, 0));
  MKB_TRY(cudaDeviceSynchronize());

  mkb_decode_args& a = e->step_args;
  mkb_decode_args_init(&a);
  a.embed = m->embed;
  a.lm_head = m->lm_head ? m->lm_head : m->embed;
  a.final_norm = m->final_norm;
  a.layers = e->d_layers;
  a.down_t = e->d_down_t;
  a.cos_table = m->cos_table;
  a.sin_table = m->sin_table;
  a.rope_fp32 = m->rope_fp32;
  a.k_cache = m->k_cache;
  a.v_cache = m->v_cache;
  a.max_seq = m->max_seq;
  a.layer_begin = 0;
  a.layer_end = m->n_layers;
  a.step = e->d_step;
  a.n_tokens = 1;
  a.flags = MKB_FLAG_LM_HEAD;
  a.logits = e->d_logits;
  a.out_tokens = e->d_io + 4;  // the last CTA writes the argmax straight into host memory
  a.err_flag = reinterpret_cast<uint32_t*>(e->d_io + 5);
  a.workspace = e->ws;
  a.grid = e->grid;

  if (m->use_graph) {
    MKB_TRY(cudaStreamCreateWithFlags(&e->cap_stream, cudaStreamNonBlocking));
  }
  if (m->use_graph && e->tp_ready) {  // a tensor-parallel rank captures at attach time
    cudaGraph_t g = nullptr;
    MKB_TRY(cudaStreamBeginCapture(e->cap_stream, cudaStreamCaptureModeThreadLocal));
    cudaError_t le = mkb_decode(&a, e->cap_stream);
    cudaError_t ce = cudaStreamEndCapture(e->cap_stream, &g);
    if (le != cudaSuccess || ce != cudaSuccess) {
      if (g) cudaGraphDestroy(g);
      cudaGetLastError();
      engine_free(e);
      return le != cudaSuccess ? le : ce;
    }
    err = cudaGraphInstantiate(&e->graph, g, 0);
    cudaGraphDestroy(g);
    if (err != cudaSuccess) { engine_free(e); return err; }
  }
#undef MKB_TRY
  *out = e;
  return cudaSuccess;
}

cudaError_t mkb_engine_step(mkb_engine* e, int token, int position, int* next_token, cudaStream_t stream) {
  if (!e) return cudaErrorInvalidValue;
  if (token < 0 || token >= kVocab || position < 0 || position >= e->max_seq) return cudaErrorInvalidValue;
  cudaError_t err = engine_report_earlier(e, stream);
  if (err != cudaSuccess) return err;
  volatile int* io = e->h_io;
  io[0] = token;
  io[1] = position;
  io[4] = -1;  // stays -1 unless the token completes (no CTA stopped on an error)
  err = cudaMemcpyAsync(e->d_step, e->h_io, 2 * sizeof(int), cudaMemcpyHostToDevice, stream);
  if (err != cudaSuccess) return err;
  err = e->graph ? cudaGraphLaunch(e->graph, stream) : mkb_decode(&e->step_args, stream);
  if (err != cudaSuccess) return err;
  err = cudaStreamSynchronize(stream);
  if (err != cudaSuccess) return err;
  if (io[4] < 0) {
    const cudaError_t st = engine_check_status(e);
    return st != cudaSuccess ? st : cudaErrorLaunchFailure;
  }
  if (next_token) *next_token = io[4];
  return cudaSuccess;
}

cudaError_t mkb_engine_generate(mkb_engine* e, int token, int position, int n, int* out_tokens,
                                cudaStream_t stream) {
  return mkb_engine_generate_until(e, token, position, n, -1, out_tokens, stream);
}

cudaError_t mkb_engine_generate_until(mkb_engine* e, int token, int position, int n, int stop_token,
                                      int* out_tokens, cudaStream_t stream) {
  if (!e || n < 1 || !out_tokens || stop_token >= kVocab) return cudaErrorInvalidValue;
  cudaError_t err = engine_report_earlier(e, stream);
  if (err != cudaSuccess) return err;
  if (token < 0 || token >= kVocab || position < 0 || position + n > e->max_seq) return cudaErrorInvalidValue;
  mkb_decode_args a = e->step_args;
  a.step = nullptr;
  a.token = token;
  a.position = position;
  a.cache_len = position + 1;
  a.n_tokens = n;
  a.out_tokens = out_tokens;
  a.stop_token = stop_token < 0 ? -1 : stop_token;
  return mkb_decode(&a, stream);
}

cudaError_t mkb_engine_prefill(mkb_engine* e, const int* prompt_tokens, int n, int position, int* next_token,
                               cudaStream_t stream) {
  if (!e || !prompt_tokens || n < 1) return cudaErrorInvalidValue;
  if (position < 0 || position + n > e->max_seq) return cudaErrorInvalidValue;
  cudaError_t err = engine_report_earlier(e, stream);
  if (err != cudaSuccess) return err;
  mkb_decode_args a = e->step_args;
  a.step = nullptr;
  a.token = 0;  // the inputs come from prompt_tokens (ids are clamped on the device)
  a.position = position;
  a.cache_len = position + 1;
  a.n_tokens = n;
  a.prompt_tokens = prompt_tokens;
  a.out_tokens = e->d_pf;  // only entry n-1 (the last prompt token) is written
  err = mkb_decode(&a, stream);
  if (err != cudaSuccess || !next_token) return err;
  return cudaMemcpyAsync(next_token, e->d_pf + (n - 1), sizeof(int), cudaMemcpyDeviceToDevice, stream);
}

cudaError_t mkb_engine_tp_attach(mkb_engine* e, int tp_rank, int tp_size, void* const* peer_workspaces) {
  if (!e || !peer_workspaces) return cudaErrorInvalidValue;
  if ((tp_size != 2 && tp_size != 4 && tp_size != 8) || tp_rank < 0 || tp_rank >= tp_size) return cudaErrorInvalidValue;
  if (tp_size != e->tp_size || !e->d_down_t || peer_workspaces[tp_rank] != e->ws) return cudaErrorInvalidValue;
  mkb_decode_args a = e->step_args;
  a.tp_rank = tp_rank;
  a.tp_size = tp_size;
  for (int g = 0; g < 8; ++g) a.peer_workspaces[g] = g < tp_size ? peer_workspaces[g] : nullptr;
  DecodeParams check;
  cudaError_t err = to_params(&a, &check);
  if (err != cudaSuccess) return err;
  e->step_args = a;
  e->tp_ready = true;
  if (e->cap_stream) {
    // the step graph carries the launch parameters: capture it (again)
    if (e->graph) cudaGraphExecDestroy(e->graph);
    e->graph = nullptr;
    cudaGraph_t g = nullptr;
    err = cudaStreamBeginCapture(e->cap_stream, cudaStreamCaptureModeThreadLocal);
    if (err != cudaSuccess) return err;
    const cudaError_t le = mkb_decode(&e->step_args, e->cap_stream);
    const cudaError_t ce = cudaStreamEndCapture(e->cap_stream, &g);
    if (le != cudaSuccess || ce != cudaSuccess) {
      if (g) cudaGraphDestroy(g);
      return le != cudaSuccess ? le : ce;
    }
    err = cudaGraphInstantiate(&e->graph, g, 0);
    cudaGraphDestroy(g);
    if (err != cudaSuccess) return err;
  }
  return cudaSuccess;
}

cudaError_t mkb_ipc_export(const void* device_ptr, unsigned char handle[64]) {
  if (!device_ptr || !handle) return cudaErrorInvalidValue;
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(device_ptr));
  if (e != cudaSuccess) return e;
  static_assert(sizeof(h) == 64, "CUDA IPC handles are 64 bytes");
  std::memcpy(handle, &h, sizeof(h));
  return cudaSuccess;
}

cudaError_t mkb_ipc_open(const unsigned char handle[64], void** device_ptr) {
  if (!handle || !device_ptr) return cudaErrorInvalidValue;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  return cudaIpcOpenMemHandle(device_ptr, h, cudaIpcMemLazyEnablePeerAccess);
}

cudaError_t mkb_ipc_close(void* device_ptr) { return cudaIpcCloseMemHandle(device_ptr); }

cudaError_t mkb_engine_prefill_batched(mkb_engine* e, const int* prompt_tokens, int n, int position, int* next_token,
                                      cudaStream_t stream) {
  if (!e || !prompt_tokens || n < 1) return cudaErrorInvalidValue;
  if (position < 0 || position + n > e->max_seq) return cudaErrorInvalidValue;
  if (e->tp_size > 1) return cudaErrorNotSupported;
  cudaError_t err = engine_report_earlier(e, stream);
  if (err != cudaSuccess) return err;
  const mkb_decode_args& sa = e->step_args;
  if (e->pf_block == nullptr) {
    // one block: residual, GEMM operands, SwiGLU output, QKV, rotated q, V^T
    const size_t cap = static_cast<size_t>(e->max_seq);
    const int vt_cols = (e->max_seq + 127) / 128 * 128;
    const size_t b_h = cap * kHidden * 4, b_a = cap * kQSize * 2, b_m = cap * kInter * 2, b_qkv = cap * kQKVRows * 4,
                 b_q = cap * kQSize * 4, b_vt = static_cast<size_t>(kNKV) * kHeadDim * vt_cols * 2;
    const size_t total = b_h + 2 * b_a + 2 * b_m + b_qkv + b_q + b_vt + 256;
    err = cudaMalloc(&e->pf_block, total);
    if (err != cudaSuccess) return err;
    char* p = static_cast<char*>(e->pf_block);
    e->pf.h = reinterpret_cast<float*>(p);
    p += b_h;
    e->pf.ah = reinterpret_cast<__nv_bfloat16*>(p);
    p += b_a;
    e->pf.al = reinterpret_cast<__nv_bfloat16*>(p);
    p += b_a;
    e->pf.mh = reinterpret_cast<__nv_bfloat16*>(p);
    p += b_m;
    e->pf.ml = reinterpret_cast<__nv_bfloat16*>(p);
    p += b_m;
    e->pf.qkv = reinterpret_cast<float*>(p);
    p += b_qkv;
    e->pf.q = reinterpret_cast<float*>(p);
    p += b_q;
    e->pf.vt = reinterpret_cast<__nv_bfloat16*>(p);
    e->pf.vt_cols = vt_cols;
    p += b_vt;
    // V^T past the keys a prefill writes is read as whole 128-key tiles (with
    // zero weights): it must hold finite values, zeros to begin with
    err = cudaMemsetAsync(e->pf.vt, 0, b_vt, stream);
    if (err != cudaSuccess) return err;
    e->pf.cap = e->max_seq;
  }
  // a GEMM wait that expires is recorded in the workspace's status word (the
  // final LM-head launch then refuses the stale workspace and poisons its outputs)
  e->pf.err = static_cast<Workspace*>(e->ws)->error;
  err = prefill_layers(e->host_layers.data(), e->n_layers, static_cast<const __nv_bfloat16*>(sa.embed), sa.cos_table,
                       sa.sin_table, sa.rope_fp32, static_cast<__nv_bfloat16*>(sa.k_cache),
                       static_cast<__nv_bfloat16*>(sa.v_cache), e->max_seq, prompt_tokens, n, position, e->pf, stream);
  if (err != cudaSuccess) return err;
  // final norm + LM head + argmax of the last prompt token (the decode kernel, no layers)
  mkb_decode_args a = sa;
  a.step = nullptr;
  a.layer_begin = 0;
  a.layer_end = 0;
  a.token = 0;
  a.position = position + n - 1;
  a.cache_len = position + n;
  a.n_tokens = 1;
  a.input_residual = e->pf.h + static_cast<size_t>(n - 1) * kHidden;
  a.out_tokens = e->d_pf + (n - 1);
  err = mkb_decode(&a, stream);
  if (err != cudaSuccess || !next_token) return err;
  return cudaMemcpyAsync(next_token, e->d_pf + (n - 1), sizeof(int), cudaMemcpyDeviceToDevice, stream);
}

cudaError_t mkb_gemm_bf16_split(const void* a_hi, const void* a_lo, const void* b, float* c, int m, int n, int k,
                                cudaStream_t stream) {
  if (!a_hi || !a_lo || !b || !c || m < 1 || n < 128 || n % 128 || k < 64 || k % 64) return cudaErrorInvalidValue;
  return gemm_split(static_cast<const __nv_bfloat16*>(a_hi), static_cast<const __nv_bfloat16*>(a_lo),
                    static_cast<const __nv_bfloat16*>(b), c, m, n, k, nullptr, stream);
}

// Serve mailbox and result words: {seq, value} written and read as one 8-byte
// word of pinned, mapped memory (the device reads and writes them the same way).
static inline void put_pair(volatile int* p, int seq, int value) {
  *reinterpret_cast<volatile uint64_t*>(p) =
      (static_cast<uint64_t>(static_cast<uint32_t>(value)) << 32) | static_cast<uint32_t>(seq);
}
static inline uint64_t get_pair(volatile int* p) { return *reinterpret_cast<volatile uint64_t*>(p); }

cudaError_t mkb_engine_serve_open(mkb_engine* e, int position, int max_tokens, unsigned long long timeout_ns,
                                  cudaStream_t stream) {
  if (!e || e->serving || max_tokens < 1 || position < 0 || position + max_tokens > e->max_seq)
    return cudaErrorInvalidValue;
  if (e->tp_size > 1) return cudaErrorNotSupported;
  cudaError_t err = engine_report_earlier(e, stream);
  if (err != cudaSuccess) return err;
  volatile int* io = e->h_io;
  put_pair(io + 2, 0, 0);
  put_pair(io + 6, 0, -1);
  mkb_decode_args a = e->step_args;
  a.step = nullptr;
  a.token = 0;  // every input comes from the mailbox
  a.position = position;
  a.cache_len = position + 1;
  a.n_tokens = max_tokens;
  a.out_tokens = nullptr;
  a.mailbox = e->d_io + 2;
  a.result = e->d_io + 6;
  a.timeout_ns = timeout_ns ? timeout_ns : 1000000000ull;
  err = mkb_decode(&a, stream);
  if (err != cudaSuccess) return err;
  e->serving = true;
  e->serve_seq = 0;
  e->serve_max = max_tokens;
  e->serve_timeout = a.timeout_ns;
  e->serve_stream = stream;
  return cudaSuccess;
}

namespace {
// Ends a session: stops the launch if it is still waiting for tokens, waits for
// it, and reports an in-kernel failure (workspace reset) as cudaErrorLaunchFailure.
cudaError_t serve_finish(mkb_engine* e) {
  volatile int* io = e->h_io;
  if (e->serve_seq < e->serve_max) put_pair(io + 2, e->serve_seq + 1, -1);  // ends the launch
  e->serving = false;
  cudaError_t err = cudaStreamSynchronize(e->serve_stream);
  if (err != cudaSuccess) return err;
  if (io[5] != 0) {
    const cudaError_t st = engine_check_status(e);
    return st != cudaSuccess ? st : cudaErrorLaunchFailure;
  }
  return cudaSuccess;
}
}  // namespace

cudaError_t mkb_engine_serve_step(mkb_engine* e, int token, int* next_token) {
  if (!e || !e->serving || e->serve_seq >= e->serve_max) return cudaErrorInvalidValue;
  if (token < 0 || token >= kVocab) return cudaErrorInvalidValue;
  volatile int* io = e->h_io;
  const int seq = ++e->serve_seq;
  put_pair(io + 2, seq, token);  // {seq, token} in one 8-byte store
  // the launch answers within a token's time; give up after the session timeout
  const auto t0 = std::chrono::steady_clock::now();
  uint64_t r;
  while (static_cast<int>(static_cast<uint32_t>(r = get_pair(io + 6))) != seq) {
    if (io[5] != 0 ||
        std::chrono::steady_clock::now() - t0 > std::chrono::nanoseconds(2 * e->serve_timeout)) {
      const cudaError_t st = serve_finish(e);
      return st != cudaSuccess ? st : cudaErrorLaunchFailure;
    }
  }
  if (next_token) *next_token = static_cast<int>(static_cast<uint32_t>(r >> 32));
  if (seq == e->serve_max) return serve_finish(e);  // the launch ends after its last token
  return cudaSuccess;
}

cudaError_t mkb_engine_serve_close(mkb_engine* e) {
  if (!e) return cudaErrorInvalidValue;
  if (!e->serving) return cudaSuccess;
  return serve_finish(e);
}

float* mkb_engine_logits(mkb_engine* e) { return e ? e->d_logits : nullptr; }
void* mkb_engine_workspace(mkb_engine* e) { return e ? e->ws : nullptr; }
int mkb_engine_grid(mkb_engine* e) { return e ? e->grid : 0; }
void mkb_engine_destroy(mkb_engine* e) {
  if (e && e->serving) serve_finish(e);
  engine_free(e);
}

}  // extern "C"
