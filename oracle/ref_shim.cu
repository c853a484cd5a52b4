// Test-infrastructure shim around the reference kernel (built into oracle/_ref
// together with the reference's own megakernel.cu; never part of the product).
//
// ref_decode_call() repeats, without PyTorch, what the reference binding does on
// every decode call (pytorch_binding.cu:62-126): upload a host LayerWeights
// table into a freshly cudaMalloc'd device buffer, launch the kernel, cudaFree
// the buffer. Scratch vectors are passed in by the caller.
#include <cuda_runtime.h>

extern "C" cudaError_t launch_decode_kernel(int, const void*, const void*, const void*, const void*, const void*,
                                            const void*, void*, void*, void*, void*, void*, void*, void*, void*,
                                            void*, void*, void*, void*, int, int, int, cudaStream_t);

extern "C" cudaError_t ref_decode_call(int token_id, const void* embed, const void* lm_head, const void* final_norm,
                                       const void* host_table /* 28*11 device pointers */, const void* cos_table,
                                       const void* sin_table, void* k_cache, void* v_cache, void* scratch[10],
                                       int position, int max_seq_len, cudaStream_t stream) {
  void* device_layers = nullptr;
  const size_t bytes = 28 * 11 * sizeof(void*);
  cudaError_t e = cudaMalloc(&device_layers, bytes);
  if (e != cudaSuccess) return e;
  e = cudaMemcpyAsync(device_layers, host_table, bytes, cudaMemcpyHostToDevice, stream);
  if (e == cudaSuccess)
    e = launch_decode_kernel(token_id, embed, lm_head, final_norm, device_layers, cos_table, sin_table, k_cache,
                             v_cache, scratch[0], scratch[1], scratch[2], scratch[3], scratch[4], scratch[5],
                             scratch[6], scratch[7], scratch[8], scratch[9], position, position + 1, max_seq_len,
                             stream);
  cudaError_t f = cudaFree(device_layers);
  return e != cudaSuccess ? e : f;
}
