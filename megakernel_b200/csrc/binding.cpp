// PyTorch extension `megakernel_extension`: the reference's Python surface
// (pytorch_binding.cu:36-48,132-134) over the C ABI of libmkb200.so.
//
// decode(token_id, embed_weight, lm_head_weight, final_norm_weight,
//        layer_weights[28*11], cos_table, sin_table, k_cache, v_cache,
//        position, max_seq_len) -> FP32 logits [151936]
//
// Same arguments, same result, same in-place K/V append at `position` with
// cache_len = position + 1 (pytorch_binding.cu:98). Differences: arguments are
// validated (dtype, device, shape, contiguity, 16-byte alignment, ranges) and
// raise ValueError/RuntimeError; the device LayerWeights table and the scratch
// vectors are kept resident per device instead of being allocated and freed on
// every call (pytorch_binding.cu:49-60,84-126), so a call performs no
// cudaMalloc/cudaFree. Like the reference's call (whose per-call cudaFree
// synchronises), it returns after the kernel has finished: it synchronises the
// stream and raises RuntimeError, after resetting the workspace, when the kernel
// reported a failure (a bounded wait that expired, bad arguments seen on the
// device), instead of returning the poisoned logits.

#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAException.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>
#include <vector>

#include "mkb200.h"

namespace {

constexpr int64_t kHidden = 1024, kInter = 3072, kVocab = 151936, kLayers = 28, kHeadDim = 128;
const int64_t kShapes[11][2] = {{kHidden, 0}, {2048, kHidden}, {1024, kHidden}, {1024, kHidden},
                                {kHeadDim, 0}, {kHeadDim, 0},   {kHidden, 2048}, {kHidden, 0},
                                {kInter, kHidden}, {kInter, kHidden}, {kHidden, kInter}};

struct DeviceState {
  std::vector<uint64_t> host_table;   // 28*11 pointers last uploaded
  void* table = nullptr;              // device LayerWeights[28]
  torch::Tensor residual, q, k, v, mlp;
};
std::mutex g_mu;
DeviceState g_state[64];

void check_bf16(const torch::Tensor& t, const char* name, c10::Device dev) {
  TORCH_CHECK_VALUE(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK_VALUE(t.device() == dev, name, " must be on ", dev);
  TORCH_CHECK_VALUE(t.scalar_type() == torch::kBFloat16, name, " must be bfloat16");
  TORCH_CHECK_VALUE(t.is_contiguous(), name, " must be contiguous");
  TORCH_CHECK_VALUE(reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, name, " must be 16-byte aligned");
}

void check_shape(const torch::Tensor& t, const char* name, std::vector<int64_t> shape) {
  TORCH_CHECK_VALUE(t.sizes().vec() == shape, name, " has shape ", t.sizes(), ", expected ", shape);
}

}  // namespace

torch::Tensor decode(int64_t token_id, torch::Tensor embed_weight, torch::Tensor lm_head_weight,
                     torch::Tensor final_norm_weight, std::vector<torch::Tensor> layer_weights,
                     torch::Tensor cos_table, torch::Tensor sin_table, torch::Tensor k_cache,
                     torch::Tensor v_cache, int64_t position, int64_t max_seq_len) {
  const c10::Device dev = embed_weight.device();
  check_bf16(embed_weight, "embed_weight", dev);
  check_shape(embed_weight, "embed_weight", {kVocab, kHidden});
  check_bf16(lm_head_weight, "lm_head_weight", dev);
  check_shape(lm_head_weight, "lm_head_weight", {kVocab, kHidden});
  check_bf16(final_norm_weight, "final_norm_weight", dev);
  check_shape(final_norm_weight, "final_norm_weight", {kHidden});
  TORCH_CHECK_VALUE(static_cast<int64_t>(layer_weights.size()) == kLayers * 11,
                    "layer_weights must hold 28*11 tensors in LayerWeights order, got ", layer_weights.size());
  for (size_t i = 0; i < layer_weights.size(); ++i) {
    const auto& t = layer_weights[i];
    check_bf16(t, "layer_weights[i]", dev);
    const auto* s = kShapes[i % 11];
    if (s[1] == 0) check_shape(t, "layer_weights[i]", {s[0]});
    else check_shape(t, "layer_weights[i]", {s[0], s[1]});
  }
  TORCH_CHECK_VALUE(max_seq_len >= 1, "max_seq_len must be positive");
  check_bf16(k_cache, "k_cache", dev);
  check_shape(k_cache, "k_cache", {kLayers, 8, max_seq_len, kHeadDim});
  check_bf16(v_cache, "v_cache", dev);
  check_shape(v_cache, "v_cache", {kLayers, 8, max_seq_len, kHeadDim});
  check_bf16(cos_table, "cos_table", dev);
  check_bf16(sin_table, "sin_table", dev);
  TORCH_CHECK_VALUE(cos_table.dim() == 2 && cos_table.size(1) == kHeadDim && cos_table.size(0) >= max_seq_len,
                    "cos_table must be [>=max_seq_len, 128]");
  TORCH_CHECK_VALUE(sin_table.sizes() == cos_table.sizes(), "sin_table must match cos_table");
  TORCH_CHECK_VALUE(token_id >= 0 && token_id < kVocab, "token_id out of range");
  TORCH_CHECK_VALUE(position >= 0 && position < max_seq_len, "position out of range");

  c10::cuda::CUDAGuard guard(dev);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream().stream();
  const int d = dev.index();
  TORCH_CHECK(d >= 0 && d < 64, "unsupported device index");

  std::lock_guard<std::mutex> lk(g_mu);
  DeviceState& st = g_state[d];
  std::vector<uint64_t> table(kLayers * 11);
  for (size_t i = 0; i < table.size(); ++i) table[i] = reinterpret_cast<uint64_t>(layer_weights[i].data_ptr());
  if (st.table == nullptr) {
    C10_CUDA_CHECK(cudaMalloc(&st.table, table.size() * sizeof(uint64_t)));
    auto f32 = embed_weight.options().dtype(torch::kFloat32);
    st.residual = torch::empty({kHidden}, f32);
    st.q = torch::empty({2048}, f32);
    st.k = torch::empty({1024}, f32);
    st.v = torch::empty({1024}, f32);
    st.mlp = torch::empty({kInter}, f32);
  }
  if (st.host_table != table) {
    // A launch still in flight may read the old table: wait before replacing it.
    C10_CUDA_CHECK(cudaStreamSynchronize(stream));
    C10_CUDA_CHECK(cudaMemcpy(st.table, table.data(), table.size() * sizeof(uint64_t), cudaMemcpyHostToDevice));
    st.host_table = table;
  }
  auto logits = torch::empty({kVocab}, embed_weight.options().dtype(torch::kFloat32));
  const int cache_len = static_cast<int>(position) + 1;
  C10_CUDA_CHECK(launch_decode_kernel(
      static_cast<int>(token_id), embed_weight.data_ptr(), lm_head_weight.data_ptr(), final_norm_weight.data_ptr(),
      st.table, cos_table.data_ptr(), sin_table.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), nullptr,
      st.residual.data_ptr(), nullptr, nullptr, nullptr, st.mlp.data_ptr(), logits.data_ptr(), st.q.data_ptr(),
      st.k.data_ptr(), st.v.data_ptr(), static_cast<int>(position), cache_len, static_cast<int>(max_seq_len),
      stream));
  C10_CUDA_CHECK(cudaStreamSynchronize(stream));
  void* ws = nullptr;
  C10_CUDA_CHECK(mkb_default_workspace(d, &ws));
  uint32_t out[8];
  C10_CUDA_CHECK(mkb_workspace_status(ws, out));
  if (out[0] != 0) {
    C10_CUDA_CHECK(mkb_workspace_reset(ws, stream));
    C10_CUDA_CHECK(cudaStreamSynchronize(stream));
    TORCH_CHECK(false, "decode: in-kernel error ", out[0], " (", mkb_error_name(out[0]), ") at cta ", out[1],
                ", layer ", static_cast<int>(out[2]), ", stage ", static_cast<int>(out[3]),
                "; the workspace was reset and the logits are invalid");
  }
  return logits;
}

// In-kernel status of the launcher's workspace on `device` (0 = ok); resets it
// after an error so the next call starts clean.
std::vector<int64_t> status(int64_t device) {
  void* ws = nullptr;
  C10_CUDA_CHECK(mkb_default_workspace(static_cast<int>(device), &ws));
  uint32_t out[8];
  C10_CUDA_CHECK(mkb_workspace_status(ws, out));
  if (out[0] != 0) {
    C10_CUDA_CHECK(mkb_workspace_reset(ws, nullptr));
    C10_CUDA_CHECK(cudaDeviceSynchronize());
  }
  return std::vector<int64_t>(out, out + 8);
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, module) {
  module.def("decode", &decode, "Qwen3 single-token decode (B200 engine)");
  module.def("status", &status, "in-kernel status of the decode workspace on a device");
}
