// dkv_packed_attention_noalloc: the packed attention for callers that cannot
// allocate device memory.
//
// Some callers of this path run where no allocator is available: code driven
// from inside a CUDA graph that is being captured elsewhere, embedders with a
// fixed device-memory budget handed out up front, or host runtimes (a serving
// process's custom allocator, a non-PyTorch binding) that forbid cudaMalloc on
// the hot path. The regular entry point needs a caller-provided workspace for
// the split-history partial results; this one takes its scratch from a
// fixed-size array that lives in the library itself, so the caller passes only
// inputs and outputs.
//
// The array is a file-scope __device__ object: every GPU that loads the library
// holds these bytes until the process exits, and every call on that GPU shares
// them. Its head holds the split-merge counters, which must be zero when a call
// starts: static storage starts zeroed and every call leaves them zero again.
// The partials behind them need no clearing: each call writes every partial it
// later reads. Two calls whose kernels overlap on the same GPU (for
// example on two streams) would race on the array; issue them one after the
// other, as the regular entry point's one-stream rule already asks.
#include <atomic>
#include <cstdio>

#include "attention.cuh"

namespace dkv {
int set_last_error(int code, const char* message);  // api.cu: the dkv_last_error() text
}  // namespace dkv

namespace {

// Upper bound of dkv_packed_attention_workspace() over all shapes: the merge
// counters plus at most 148 split CTAs (fewer splits -> no workspace), each with
// at most 256 rows x (64 fp32 outputs + (max, sum)) = 67,584 bytes, plus one
// padding (max, sum) column per row of each of at most 74 groups.
constexpr size_t kScratchBytes = DKV_NOALLOC_SCRATCH_BYTES;
static_assert(dkv::kSyncBytes + static_cast<size_t>(dkv::kTargetCtas) * dkv::kTcCtaRows * (dkv::kDim * 4 + 8) +
                      static_cast<size_t>(dkv::kTargetCtas / 2) * dkv::kTcCtaRows * 8 <=
                  kScratchBytes,
              "static scratch smaller than the planner's largest workspace");

static __device__ __align__(256) unsigned char g_scratch[kScratchBytes];

// Device address of g_scratch per device (host code must not use the symbol's
// name as an address: on the host it is only a stand-in for the device object).
std::atomic<void*> g_scratch_ptr[64];

}  // namespace

extern "C" int dkv_packed_attention_noalloc(
    const void* q, const void* knew, const void* vnew, const void* p4, const void* m4, const void* p8,
    const void* m8, const void* p16, const int32_t* rows, const uint8_t* codes, void* out, int64_t qh, int64_t qt,
    int64_t kh, int64_t kt, int64_t vh, int64_t vt, int32_t layer, int32_t past, int32_t nq, int64_t cap4,
    int64_t cap8, int64_t cap16, int32_t heads, int32_t group, int32_t dim, int32_t block_m, int32_t block_n,
    int32_t layers, int32_t* status, void* stream) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  char msg[256];
  if (e != cudaSuccess || dev < 0 || dev >= 64) {
    snprintf(msg, sizeof(msg), "no-alloc attention: cannot query the current device (%s)", cudaGetErrorString(e));
    return dkv::set_last_error(DKV_ECUDA, msg);
  }
  void* scratch = g_scratch_ptr[dev].load(std::memory_order_acquire);
  if (scratch == nullptr) {  // first call on this device: look the array up once
    e = cudaGetSymbolAddress(&scratch, g_scratch);
    if (e != cudaSuccess || scratch == nullptr) {
      snprintf(msg, sizeof(msg), "no-alloc attention: cudaGetSymbolAddress failed (%s)", cudaGetErrorString(e));
      return dkv::set_last_error(DKV_ECUDA, msg);
    }
    g_scratch_ptr[dev].store(scratch, std::memory_order_release);
  }
  const size_t need = dkv_packed_attention_workspace(past, nq, heads, group, dim);
  if (need > kScratchBytes) {
    snprintf(msg, sizeof(msg),
             "no-alloc attention: this shape needs %zu scratch bytes, more than the library's fixed %zu", need,
             kScratchBytes);
    return dkv::set_last_error(DKV_EWORKSPACE, msg);
  }
  return dkv_packed_attention(q, knew, vnew, p4, m4, p8, m8, p16, rows, codes, out, qh, qt, kh, kt, vh, vt, layer,
                              past, nq, cap4, cap8, cap16, heads, group, dim, block_m, block_n, layers, scratch,
                              kScratchBytes, status, stream);
}
