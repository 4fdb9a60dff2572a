// Host fast path of the per-layer calls a GPUCache makes (append, attend, append +
// attend): the same argument checks and the same C-ABI entry points as the ctypes
// binding in src/gpu_kernels.py, made from C++ so that one eager call costs a few
// microseconds of host time instead of ~25 (ctypes marshals ~35 arguments, and every
// stride and pointer query is a Python call). The reference launches its Triton
// kernels from Python once per layer (src/gpu_cache.py:90-92, 99-103), so this host
// cost is paid on every layer of every frame.
#include <torch/extension.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#include <map>
#include <mutex>
#include <stdexcept>
#include <utility>
#include <vector>

#include "dkv.h"

namespace {

// Pointers of one cache: p4, m4, p8, m8, p16, rows, codes, status.
using Ptrs = std::vector<int64_t>;
using Caps = std::vector<int64_t>;

void* vp(int64_t p) { return reinterpret_cast<void*>(static_cast<uintptr_t>(p)); }

void check(int rc) {
  if (rc == DKV_OK) return;
  const char* m = dkv_last_error();
  if (rc == DKV_ECUDA) throw std::runtime_error(m);
  throw pybind11::value_error(m);
}

// bf16 [1, heads, n, 64] operand whose rows the kernels load 16 bytes at a time
// (else a contiguous copy), as gpu_kernels._rows_ready.
at::Tensor rows_ready(const at::Tensor& x) {
  if (!x.is_cuda()) throw pybind11::value_error("GPU cache requires CUDA, batch one and the configured head dimension");
  if (x.scalar_type() != at::kBFloat16) throw pybind11::value_error("GPU kernels take bfloat16 queries, keys and values");
  if (x.dim() != 4) throw pybind11::value_error("GPU kernels take [1, heads, n, dim] queries, keys and values");
  const bool ok = x.stride(3) == 1 && x.stride(1) % 8 == 0 && x.stride(2) % 8 == 0 &&
                  (reinterpret_cast<uintptr_t>(x.data_ptr()) & 15u) == 0;
  return ok ? x : x.contiguous();
}

void same_device(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v) {
  if (k.device() != q.device() || v.device() != q.device())
    throw pybind11::value_error("queries, keys and values must be on one CUDA device");
}

void check_ptrs(const Ptrs& p, const Caps& c) {
  if (p.size() != 8 || c.size() != 3) throw pybind11::value_error("cache pointers (8) and capacities (3) expected");
}

// Attention workspaces, one per (device, stream): the library leaves the merge
// counters at the head of a workspace zero after every call, so a workspace is
// zero-filled once and reused; calls on one stream never overlap, calls on other
// streams get other workspaces. Outgrown ones stay referenced, so CUDA graphs
// captured with them keep valid addresses.
std::mutex g_ws_mu;
std::map<std::pair<int, cudaStream_t>, at::Tensor> g_ws;
std::vector<at::Tensor> g_retired;

at::Tensor workspace_for(const at::Device& device, cudaStream_t stream, int64_t size) {
  std::lock_guard<std::mutex> lock(g_ws_mu);
  auto& ws = g_ws[{device.index(), stream}];
  if (!ws.defined() || ws.numel() < size) {
    if (ws.defined()) g_retired.push_back(ws);
    ws = at::zeros({size}, at::TensorOptions().dtype(at::kByte).device(device));
  }
  return ws;
}

cudaStream_t current_stream(const at::Tensor& x) {
  return c10::cuda::getCurrentCUDAStream(x.device().index()).stream();
}

}  // namespace

// The workspace of (x's device, current stream) with at least `size` bytes (size > 0).
at::Tensor workspace(const at::Tensor& like, int64_t size) {
  return workspace_for(like.device(), current_stream(like), size);
}

// GPUCache.attend: dkv_packed_attention of q [1, heads*group, n, 64] over the
// cache's packed history plus k / v [1, heads, n, 64]; returns [1, n, heads*group, 64].
at::Tensor attend(const at::Tensor& q_in, const at::Tensor& k_in, const at::Tensor& v_in, const Ptrs& p,
                  int64_t layer, int64_t past, const Caps& caps, int64_t heads, int64_t block_m, int64_t block_n,
                  int64_t layers) {
  check_ptrs(p, caps);
  const at::Tensor q = rows_ready(q_in), k = rows_ready(k_in), v = rows_ready(v_in);
  same_device(q, k, v);
  const c10::cuda::CUDAGuard guard(q.device());  // the library launches on the current device
  const int64_t nq = q.size(2), hq = q.size(1);
  if (heads <= 0 || hq % heads) throw pybind11::value_error("query heads must be a positive multiple of KV heads");
  const int64_t group = hq / heads;
  at::Tensor out = at::empty({1, nq, hq, q.size(3)}, q.options());
  const cudaStream_t stream = current_stream(q);
  const size_t size = dkv_packed_attention_workspace(past, nq, heads, group, q.size(3));
  void* ws = size ? workspace_for(q.device(), stream, size).data_ptr() : nullptr;
  check(dkv_packed_attention(q.data_ptr(), k.data_ptr(), v.data_ptr(), vp(p[0]), vp(p[1]), vp(p[2]), vp(p[3]),
                             vp(p[4]), static_cast<const int32_t*>(vp(p[5])), static_cast<const uint8_t*>(vp(p[6])),
                             out.data_ptr(), q.stride(1), q.stride(2), k.stride(1), k.stride(2), v.stride(1),
                             v.stride(2), layer, past, nq, caps[0], caps[1], caps[2], heads, group, q.size(3),
                             block_m, block_n, layers, ws, size, static_cast<int32_t*>(vp(p[7])), stream));
  return out;
}

// GPUCache.append's launch: dkv_pack_rows of k / v [1, heads, n, 64] at rows
// [row_start, row_start + n) of the `bits` pool.
void pack(const at::Tensor& k_in, const at::Tensor& v_in, const Ptrs& p, int64_t layer, int64_t row_start,
          const Caps& caps, int64_t heads, int64_t bits, int64_t layers) {
  check_ptrs(p, caps);
  const at::Tensor k = rows_ready(k_in), v = rows_ready(v_in);
  same_device(k, k, v);
  const c10::cuda::CUDAGuard guard(k.device());
  check(dkv_pack_rows(k.data_ptr(), v.data_ptr(), vp(p[0]), vp(p[1]), vp(p[2]), vp(p[3]), vp(p[4]), k.stride(1),
                      k.stride(2), v.stride(1), v.stride(2), layer, row_start, k.size(2), caps[0], caps[1], caps[2],
                      heads, k.size(3), bits, layers, static_cast<int32_t*>(vp(p[7])), current_stream(k)));
}

// GPUCache.append_attend: dkv_append_attention (pack + attention of one frame in
// one launch); returns [1, n, heads*group, 64].
at::Tensor append_attend(const at::Tensor& q_in, const at::Tensor& k_in, const at::Tensor& v_in, const Ptrs& p,
                         int64_t layer, int64_t past, int64_t row_start, int64_t bits, bool fill_map,
                         int64_t map_capacity, const Caps& caps, int64_t heads, int64_t block_m, int64_t block_n,
                         int64_t layers) {
  check_ptrs(p, caps);
  const at::Tensor q = rows_ready(q_in), k = rows_ready(k_in), v = rows_ready(v_in);
  same_device(q, k, v);
  const c10::cuda::CUDAGuard guard(q.device());  // the library launches on the current device
  const int64_t nq = q.size(2), hq = q.size(1);
  if (heads <= 0 || hq % heads) throw pybind11::value_error("query heads must be a positive multiple of KV heads");
  const int64_t group = hq / heads;
  at::Tensor out = at::empty({1, nq, hq, q.size(3)}, q.options());
  const cudaStream_t stream = current_stream(q);
  const size_t size = dkv_packed_attention_workspace(past, nq, heads, group, q.size(3));
  void* ws = size ? workspace_for(q.device(), stream, size).data_ptr() : nullptr;
  check(dkv_append_attention(q.data_ptr(), k.data_ptr(), v.data_ptr(), vp(p[0]), vp(p[1]), vp(p[2]), vp(p[3]),
                             vp(p[4]), static_cast<int32_t*>(vp(p[5])), static_cast<uint8_t*>(vp(p[6])),
                             out.data_ptr(), q.stride(1), q.stride(2), k.stride(1), k.stride(2), v.stride(1),
                             v.stride(2), layer, past, nq, row_start, bits, fill_map ? 1 : 0, map_capacity, caps[0],
                             caps[1], caps[2], heads, group, q.size(3), block_m, block_n, layers, ws, size,
                             static_cast<int32_t*>(vp(p[7])), stream));
  return out;
}

// The decoder layer's x + y followed by RMSNorm and its weight (dkv_add_rms_norm)
// over the rows of x / y [..., width]: returns (x + y, norm) — (x, norm) without y.
std::vector<at::Tensor> add_rms_norm(const at::Tensor& x_in, const c10::optional<at::Tensor>& y_in,
                                     const at::Tensor& weight_in, double eps) {
  if (!x_in.is_cuda() || x_in.scalar_type() != at::kBFloat16 || weight_in.scalar_type() != at::kBFloat16)
    throw pybind11::value_error("add_rms_norm takes CUDA bfloat16 tensors");
  const int64_t width = x_in.size(-1);
  const at::Tensor x = x_in.contiguous(), w = weight_in.contiguous();
  if (w.numel() != width || w.device() != x.device()) throw pybind11::value_error("add_rms_norm: weight must be [width]");
  const c10::cuda::CUDAGuard guard(x.device());
  at::Tensor h = at::empty_like(x);
  at::Tensor x_out = x;
  const void* yp = nullptr;
  at::Tensor y;
  if (y_in.has_value()) {
    y = y_in->contiguous();
    if (y.sizes() != x.sizes() || y.scalar_type() != at::kBFloat16 || y.device() != x.device())
      throw pybind11::value_error("add_rms_norm: y must match x");
    yp = y.data_ptr();
    x_out = at::empty_like(x);
  }
  const int64_t rows = width ? x.numel() / width : 0;
  check(dkv_add_rms_norm(x.data_ptr(), yp, yp ? x_out.data_ptr() : nullptr, h.data_ptr(), w.data_ptr(), rows,
                         static_cast<int32_t>(width), width, width, width, width, static_cast<float>(eps),
                         current_stream(x)));
  return {x_out, h};
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "C++ host path of GPUCache's per-layer calls into libdkv.so";
  m.def("workspace", &workspace);
  m.def("attend", &attend);
  m.def("pack", &pack);
  m.def("append_attend", &append_attend);
  m.def("add_rms_norm", &add_rms_norm);
}
