// launch_decode_kernel_noalloc: the drop-in launcher with its synchronisation
// workspace in a file-scope device array instead of a lazily cudaMalloc'd
// buffer, for callers that must not allocate device memory at any call.
//
//  * capacity: kNoAllocScratchBytes (4 MiB) per device; a build whose
//    Workspace is larger is rejected at the call (cudaErrorInvalidValue and
//    one line on stderr naming both sizes);
//  * set-up, once per device on the first call: cudaGetSymbolAddress of the
//    array (return code checked), cached per device;
//  * every call clears the Workspace bytes with cudaMemsetAsync on the call's
//    stream before the launch (counters, accumulators, tagged QKV words and
//    the status word must start at zero; the tag base restarts with them), so
//    a call that timed out in the kernel leaves nothing stale for the next;
//  * the device's one array is shared by every call on that device: calls
//    that overlap in time (other streams, other host threads) race on it;
//  * an in-kernel failure leaves NaN logits and its status in the array, read
//    with mkb_noalloc_status (a synchronous copy, no allocation) after the
//    stream is synchronised and before the next call clears it.

#include <cstdio>
#include <mutex>

#include <cuda_runtime.h>

#include "../../include/mkb200.h"
#include "mkb_config.cuh"

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(4) << 20;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mu;
void* g_noalloc_ptr[64];

cudaError_t noalloc_scratch(int dev, void** out) {
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return e;
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return cudaSuccess;
}

}  // namespace

extern "C" cudaError_t launch_decode_kernel_noalloc(
    int token_id, const void* embed_weight, const void* lm_head_weight, const void* final_norm_weight,
    const void* layer_weights, const void* cos_table, const void* sin_table, void* k_cache, void* v_cache,
    void* hidden_buffer, void* g_residual, void* g_activations, void* g_attn_output, void* g_normalized,
    void* g_mlp_intermediate, void* g_logits, void* g_q, void* g_k, void* g_v, int position, int cache_len,
    int max_seq_len, cudaStream_t stream) {
  (void)hidden_buffer;
  (void)g_activations;
  (void)g_attn_output;
  (void)g_normalized;
  const size_t need = sizeof(mkb::Workspace);
  if (need > kNoAllocScratchBytes) {
    std::fprintf(stderr, "launch_decode_kernel_noalloc: workspace needs %zu bytes, static scratch holds %zu\n",
                 need, kNoAllocScratchBytes);
    return cudaErrorInvalidValue;
  }
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  void* ws = nullptr;
  e = noalloc_scratch(dev, &ws);
  if (e != cudaSuccess) return e;
  e = cudaMemsetAsync(ws, 0, need, stream);
  if (e != cudaSuccess) return e;

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
  a.layer_end = mkb::kMaxLayers;
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
  a.workspace = ws;
  return mkb_decode(&a, stream);
}

extern "C" cudaError_t mkb_noalloc_status(int device, uint32_t out[8]) {
  if (out == nullptr) return cudaErrorInvalidValue;
  int cur = 0;
  cudaError_t e = cudaGetDevice(&cur);
  if (e != cudaSuccess) return e;
  if (device != cur && (e = cudaSetDevice(device)) != cudaSuccess) return e;
  void* ws = nullptr;
  e = noalloc_scratch(device, &ws);
  if (e == cudaSuccess)
    e = cudaMemcpy(out, static_cast<const mkb::Workspace*>(ws)->error, 8 * sizeof(uint32_t), cudaMemcpyDeviceToHost);
  if (device != cur) {
    const cudaError_t r = cudaSetDevice(cur);
    if (e == cudaSuccess) e = r;
  }
  return e;
}
