// torch_binding.cpp -- the PyTorch C++ extension of this library.
//
// Replaces the reference's pybind module (csrc/binding.cpp:3-8), whose
// `forward(q, k, v)` is attention_decode_cuda (csrc/decode.cu:223-258): the
// same name, argument meaning, checks and error messages (TORCH_CHECK ->
// RuntimeError), the output a fresh tensor like q, every launch on the
// current CUDA stream with no host synchronisation.  The kernels are not
// compiled here: this module calls the C ABI of libattention_decode_b200.so
// (include/attention_decode_b200.h), which it links against and finds next
// to itself.
//
// Additions, all compatible with the 3-argument call: an optional int32
// `seqlens` [B] on forward, forward_partial (unnormalised (acc, m, l) states
// for sequence sharding) and combine (merge of R such states).
#include <torch/extension.h>

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_runtime_api.h>

#include <map>
#include <mutex>
#include <utility>

#include "attention_decode_b200.h"

namespace {

void check_status(int status) {
  TORCH_CHECK(status == ADB_OK, "attention_decode: ", adb_last_error());
}

// The reference's input contract (csrc/decode.cu:225-241 and
// attention_decode/__init__.py:35-38), with the INT_MAX element limit
// dropped (64-bit indexing) and a GQA group of 8 accepted.
void check_inputs(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                  const c10::optional<at::Tensor>& seqlens) {
  TORCH_CHECK(q.is_cuda() && k.is_cuda() && v.is_cuda(), "Q, K, and V must be CUDA tensors");
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && k.scalar_type() == at::kBFloat16 &&
                  v.scalar_type() == at::kBFloat16,
              "Q/K/V dtype must be BF16 (bfloat16)");
  TORCH_CHECK(q.dim() == 4 && k.dim() == 4 && v.dim() == 4, "Q/K/V must have rank four");
  TORCH_CHECK(q.is_contiguous() && k.is_contiguous() && v.is_contiguous(), "Q/K/V must be contiguous");
  TORCH_CHECK(!q.requires_grad() && !k.requires_grad() && !v.requires_grad(),
              "attention_decode is forward inference only; no backward/grad support");
  TORCH_CHECK(q.numel() > 0 && k.numel() > 0 && v.numel() > 0, "empty tensors are unsupported");
  TORCH_CHECK(q.device() == k.device() && q.device() == v.device(), "Q/K/V device must match");
  TORCH_CHECK(k.sizes() == v.sizes(), "K/V shape must match");
  TORCH_CHECK(q.size(2) == 1, "query length must be 1");
  TORCH_CHECK(q.size(0) == k.size(0) && q.size(3) == k.size(3), "Q/K/V batch and head dimension must match");
  TORCH_CHECK(q.size(1) % k.size(1) == 0, "query heads must be divisible by KV heads");
  const int64_t group = q.size(1) / k.size(1);
  TORCH_CHECK(group == 1 || group == 4 || group == 8, "supported GQA group sizes are 1, 4 and 8");
  TORCH_CHECK(q.size(3) == 64 || q.size(3) == 128, "head dimension must be 64 or 128");
  if (seqlens.has_value()) {
    const at::Tensor& s = *seqlens;
    TORCH_CHECK(s.device() == q.device(), "seqlens must be on the same CUDA device as Q/K/V");
    TORCH_CHECK(s.scalar_type() == at::kInt, "seqlens dtype must be int32");
    TORCH_CHECK(s.dim() == 1 && s.size(0) == q.size(0) && s.is_contiguous(),
                "seqlens must be a contiguous [batch] tensor");
  }
}

// One workspace per (device, stream), as the Python layer keeps: calls on one
// stream are ordered and every completed call leaves its scheduler header
// zero, so the header is cleared only when a larger problem's header reaches
// past the prefix known to be zero.  A call being captured into a CUDA graph
// gets its own buffer (from the graph's pool) with the header memset captured.
struct StreamWorkspace {
  at::Tensor buffer;
  size_t clean = 0;  // leading bytes known to be zero
};
std::mutex g_mutex;
std::map<std::pair<int, cudaStream_t>, StreamWorkspace> g_workspaces;
constexpr size_t kMaxWorkspaces = 64;

struct Workspace {
  at::Tensor buffer;
  unsigned flags;
};

Workspace workspace_for(const at::Tensor& q, int device, cudaStream_t stream, size_t bytes,
                        size_t header) {
  bytes = bytes < 256 ? 256 : bytes;
  cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
  TORCH_CHECK(cudaStreamIsCapturing(stream, &capture) == cudaSuccess, "cudaStreamIsCapturing failed");
  if (capture != cudaStreamCaptureStatusNone)
    return {at::empty({static_cast<int64_t>(bytes)}, q.options().dtype(at::kByte)), 0u};
  std::lock_guard<std::mutex> lock(g_mutex);
  const auto key = std::make_pair(device, stream);
  auto it = g_workspaces.find(key);
  if (it == g_workspaces.end() || static_cast<size_t>(it->second.buffer.numel()) < bytes) {
    if (it == g_workspaces.end() && g_workspaces.size() >= kMaxWorkspaces)
      g_workspaces.erase(g_workspaces.begin());  // freed stream-ordered by the caching allocator
    StreamWorkspace ws;
    ws.buffer = at::zeros({static_cast<int64_t>(bytes)}, q.options().dtype(at::kByte));
    ws.clean = bytes;
    it = g_workspaces.insert_or_assign(key, std::move(ws)).first;
  }
  const unsigned flags = header <= it->second.clean ? ADB_FLAG_HEADER_ZEROED : 0u;
  it->second.clean = header;  // after the call only its own header is known to be zero
  return {it->second.buffer, flags};
}

struct Call {
  int device;
  cudaStream_t stream;
  Workspace ws;
};

Call prepare(const at::Tensor& q, const at::Tensor& k, const c10::optional<at::Tensor>& seqlens) {
  const int device = q.get_device();
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(device).stream();
  size_t total = 0, header = 0;
  check_status(adb_decode_workspace_size(q.size(0), q.size(1), k.size(1), k.size(2), q.size(3),
                                         seqlens.has_value() ? 1 : 0, device, &total, &header));
  return {device, stream, workspace_for(q, device, stream, total, header)};
}

// forward(q, k, v, seqlens=None) -> O [B, Hq, 1, D] BF16.
at::Tensor forward(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                   const c10::optional<at::Tensor>& seqlens) {
  check_inputs(q, k, v, seqlens);
  const c10::cuda::CUDAGuard guard(q.device());
  Call call = prepare(q, k, seqlens);
  at::Tensor out = at::empty_like(q);
  check_status(adb_decode(q.data_ptr(), k.data_ptr(), v.data_ptr(),
                          seqlens.has_value() ? seqlens->data_ptr<int32_t>() : nullptr, out.data_ptr(),
                          q.size(0), q.size(1), k.size(1), k.size(2), q.size(3), call.ws.buffer.data_ptr(),
                          static_cast<size_t>(call.ws.buffer.numel()), call.ws.flags, call.device, call.stream));
  return out;
}

// forward_partial(q, k, v, seqlens=None) -> (acc FP32 [B, Hq, D], ml FP32 [B, Hq, 2]).
std::tuple<at::Tensor, at::Tensor> forward_partial(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                                                   const c10::optional<at::Tensor>& seqlens) {
  check_inputs(q, k, v, seqlens);
  const c10::cuda::CUDAGuard guard(q.device());
  Call call = prepare(q, k, seqlens);
  auto f32 = q.options().dtype(at::kFloat);
  at::Tensor acc = at::empty({q.size(0), q.size(1), q.size(3)}, f32);
  at::Tensor ml = at::empty({q.size(0), q.size(1), 2}, f32);
  check_status(adb_decode_partial(q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                  seqlens.has_value() ? seqlens->data_ptr<int32_t>() : nullptr,
                                  acc.data_ptr<float>(), ml.data_ptr<float>(), q.size(0), q.size(1), k.size(1),
                                  k.size(2), q.size(3), call.ws.buffer.data_ptr(),
                                  static_cast<size_t>(call.ws.buffer.numel()), call.ws.flags, call.device,
                                  call.stream));
  return {acc, ml};
}

// combine(acc FP32 [R, B, Hq, D], ml FP32 [R, B, Hq, 2]) -> O BF16 [B, Hq, 1, D].
at::Tensor combine(const at::Tensor& acc, const at::Tensor& ml) {
  TORCH_CHECK(acc.is_cuda() && ml.is_cuda(), "partial states must be CUDA tensors");
  TORCH_CHECK(acc.scalar_type() == at::kFloat && ml.scalar_type() == at::kFloat, "partial states must be float32");
  TORCH_CHECK(acc.dim() == 4 && ml.dim() == 4, "acc must be [R, B, Hq, D] and ml [R, B, Hq, 2]");
  TORCH_CHECK(acc.is_contiguous() && ml.is_contiguous(), "partial states must be contiguous");
  TORCH_CHECK(ml.size(0) == acc.size(0) && ml.size(1) == acc.size(1) && ml.size(2) == acc.size(2) && ml.size(3) == 2,
              "ml must have shape [R, B, Hq, 2]");
  const c10::cuda::CUDAGuard guard(acc.device());
  const int device = acc.get_device();
  const int64_t parts = acc.size(0), rows = acc.size(1) * acc.size(2), dim = acc.size(3);
  at::Tensor out = at::empty({acc.size(1), acc.size(2), 1, dim}, acc.options().dtype(at::kBFloat16));
  check_status(adb_combine(acc.data_ptr<float>(), rows * dim, ml.data_ptr<float>(), rows * 2, parts, rows, dim,
                           out.data_ptr(), device, at::cuda::getCurrentCUDAStream(device).stream()));
  return out;
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "BF16 split-K attention decode for B200 (sm_100a): the reference extension's forward(q, k, v)";
  m.def("forward", &forward, "O = softmax(Q K^T / sqrt(D)) V for one query token per sequence",
        pybind11::arg("q"), pybind11::arg("k"), pybind11::arg("v"), pybind11::arg("seqlens") = pybind11::none());
  m.def("forward_partial", &forward_partial, "unnormalised (acc, (m, l)) states of this call's KV",
        pybind11::arg("q"), pybind11::arg("k"), pybind11::arg("v"), pybind11::arg("seqlens") = pybind11::none());
  m.def("combine", &combine, "merge R partial states into the BF16 output", pybind11::arg("acc"),
        pybind11::arg("ml"));
}
