// Pack, reconstruct and token-map kernels (sm_100a).
//
// pack_rows_kernel  <- reference Triton pack_rows   (src/gpu_kernels.py:11-46)
// reconstruct_kernel<- reference Triton reconstruct (src/gpu_kernels.py:107-119)
// map_fill_kernel   <- reference tensor writes      (src/gpu_cache.py:79-80)
//
// Both K/V kernels give one 64-wide row (a (layer, K|V, head, token) vector) to
// eight consecutive threads; thread `part` owns dims 8*part..8*part+7 and moves
// them with one 128-bit (bf16), 64-bit (int8) or 32-bit (int4) access, so a warp
// touches four whole rows with fully coalesced traffic.
#include "pack_row.cuh"

namespace dkv {

constexpr int kPackThreads = 256;
constexpr int kMaxPackRequests = DKV_MAX_REQUESTS;

template <int BITS>
__global__ void __launch_bounds__(kPackThreads)
pack_rows_kernel(const uint16_t* __restrict__ k, const uint16_t* __restrict__ v,
                 uint8_t* __restrict__ p4, float2* __restrict__ m4, uint8_t* __restrict__ p8,
                 float2* __restrict__ m8, uint16_t* __restrict__ p16, int64_t kh, int64_t kt,
                 int64_t vh, int64_t vt, int layer, int64_t row_start, int n, int blocks,
                 int heads, int32_t* status) {
  // Launched as a programmatic dependent; k / v are the previous kernels' output.
  // The dependents are released only after this grid's own wait: once any kernel
  // of this library has released its dependent, every kernel launched before it
  // has completed, so a dependent may read their results before its own wait.
  asm volatile("griddepcontrol.wait;\n" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
  const int gtid = blockIdx.x * blockDim.x + threadIdx.x;
  const int row = gtid >> 3;
  const int part = gtid & 7;
  const int per_kv = heads * n;
  if (row >= 2 * per_kv) return;  // whole 8-lane groups leave together
  const int kv = row / per_kv;
  const int rem = row - kv * per_kv;
  const int head = rem / n;
  const int token = rem - head * n;
  const uint16_t* src = kv == 0 ? k + head * kh + token * kt : v + head * vh + token * vt;
  const uint4 raw = __ldg(reinterpret_cast<const uint4*>(src) + part);
  const int64_t block = (static_cast<int64_t>(layer) * 2 + kv) * heads + head;
  pack_row_part<BITS>(raw, part, p4, m4, p8, m8, p16, pool_row(block, row_start + token, blocks), status, row);
}

// Per-request destinations of pack_rows_many_kernel: by value in the kernel
// parameters (PackTable), or in device memory (DevicePackTargets: a CUDA graph
// replays with new destinations written there between replays).
struct PackTable {
  dkv_pack_target t[kMaxPackRequests];
  __device__ const dkv_pack_target& operator[](int r) const { return t[r]; }
};
struct DevicePackTargets {
  const dkv_pack_target* t;
  __device__ const dkv_pack_target& operator[](int r) const { return t[r]; }
};

static_assert(sizeof(PackTable) + 128 <= 4096, "pack_rows_many_kernel parameters");

// Frames of several requests in one launch: blockIdx.y = request, each with its
// own precision (uniform over a block, so the branch below does not diverge),
// pools and optional token-map update. Destinations are checked here as well as
// on the host (device-resident ones are not seen by the host): a bad one is
// reported to its status word and skipped.
template <class Targets>
__global__ void __launch_bounds__(kPackThreads)
pack_rows_many_kernel(const uint16_t* __restrict__ k, const uint16_t* __restrict__ v,
                      const __grid_constant__ Targets tab, int64_t kh, int64_t kt, int64_t vh, int64_t vt,
                      int64_t kc, int64_t vc, int layer, int n, int heads, int blocks) {
  asm volatile("griddepcontrol.wait;\n" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
  const dkv_pack_target& d = tab[blockIdx.y];
  if (!pack_target_ok(d, n)) {
    if (blockIdx.x == 0 && threadIdx.x == 0) report_bad_target(d, n, blockIdx.y);
    return;
  }
  const int gtid = blockIdx.x * blockDim.x + threadIdx.x;
  const int row = gtid >> 3;
  if (row >= 2 * heads * n) return;  // whole 8-lane groups leave together
  pack_target_row(d, k + blockIdx.y * kc, v + blockIdx.y * vc, kh, kt, vh, vt, layer, n, heads, blocks, row,
                  gtid & 7);
}

__global__ void __launch_bounds__(kPackThreads)
reconstruct_kernel(Pools P, const int32_t* __restrict__ rows, const uint8_t* __restrict__ codes,
                   uint16_t* __restrict__ out, int layer, int n, int32_t* status) {
  const int gtid = blockIdx.x * blockDim.x + threadIdx.x;
  const int row = gtid >> 3;
  const int part = gtid & 7;
  const int per_kv = P.heads * n;
  if (row >= 2 * per_kv) return;
  const int kv = row / per_kv;
  const int rem = row - kv * per_kv;
  const int head = rem / n;
  const int t = rem - head * n;
  RowPart r = load_history_part(P, rows, codes, layer, kv, head, t, part, status);
  // out[kv, head, t, :] — row index equals `row` in (kv, head, token) order.
  reinterpret_cast<uint4*>(out + static_cast<int64_t>(row) * kDim)[part] = dequant_part(r);
}

__global__ void map_fill_kernel(int32_t* __restrict__ rows, uint8_t* __restrict__ codes,
                                int64_t start, int n, int64_t row, int bits) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) {
    rows[start + i] = static_cast<int32_t>(row + i);
    codes[start + i] = static_cast<uint8_t>(bits);
  }
}

// ---- host launchers (argument checks live in api.cu) ----

cudaError_t launch_pack(const void* k, const void* v, void* p4, void* m4, void* p8, void* m8,
                        void* p16, int64_t kh, int64_t kt, int64_t vh, int64_t vt, int layer,
                        int64_t row_start, int n, int blocks, int heads, int bits,
                        int32_t* status, cudaStream_t stream) {
  const int threads = 2 * heads * n * 8;
  const int grid = (threads + kPackThreads - 1) / kPackThreads;
  const uint16_t* kk = static_cast<const uint16_t*>(k);
  const uint16_t* vv = static_cast<const uint16_t*>(v);
  uint8_t* q4 = static_cast<uint8_t*>(p4);
  uint8_t* q8 = static_cast<uint8_t*>(p8);
  float2* s4 = static_cast<float2*>(m4);
  float2* s8 = static_cast<float2*>(m8);
  uint16_t* h = static_cast<uint16_t*>(p16);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kPackThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  auto kernel = bits == 4 ? pack_rows_kernel<4> : (bits == 8 ? pack_rows_kernel<8> : pack_rows_kernel<16>);
  return cudaLaunchKernelEx(&cfg, kernel, kk, vv, q4, s4, q8, s8, h, kh, kt, vh, vt, layer, row_start, n, blocks,
                            heads, status);
}

template <class Targets>
cudaError_t launch_pack_many_with(const void* k, const void* v, const Targets& tab, int count, int64_t kh,
                                  int64_t kt, int64_t vh, int64_t vt, int64_t kc, int64_t vc, int layer, int n,
                                  int heads, int blocks, cudaStream_t stream) {
  const int threads = 2 * heads * n * 8;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((threads + kPackThreads - 1) / kPackThreads, count);
  cfg.blockDim = dim3(kPackThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, pack_rows_many_kernel<Targets>, static_cast<const uint16_t*>(k),
                            static_cast<const uint16_t*>(v), tab, kh, kt, vh, vt, kc, vc, layer, n, heads, blocks);
}

// targets: host array (copied into the launch) or, with on_device, device memory.
cudaError_t launch_pack_many(const void* k, const void* v, const dkv_pack_target* targets, bool on_device, int count,
                             int64_t kh, int64_t kt, int64_t vh, int64_t vt, int64_t kc, int64_t vc, int layer, int n,
                             int heads, int blocks, cudaStream_t stream) {
  if (on_device)
    return launch_pack_many_with(k, v, DevicePackTargets{targets}, count, kh, kt, vh, vt, kc, vc, layer, n, heads,
                                 blocks, stream);
  PackTable tab{};
  for (int r = 0; r < count; ++r) tab.t[r] = targets[r];
  return launch_pack_many_with(k, v, tab, count, kh, kt, vh, vt, kc, vc, layer, n, heads, blocks, stream);
}

cudaError_t launch_reconstruct(const Pools& P, const int32_t* rows, const uint8_t* codes, void* out,
                               int layer, int n, int32_t* status, cudaStream_t stream) {
  const int threads = 2 * P.heads * n * 8;
  const int blocks = (threads + kPackThreads - 1) / kPackThreads;
  reconstruct_kernel<<<blocks, kPackThreads, 0, stream>>>(P, rows, codes, static_cast<uint16_t*>(out),
                                                         layer, n, status);
  return cudaGetLastError();
}

cudaError_t launch_map_fill(int32_t* rows, uint8_t* codes, int64_t start, int n, int64_t row, int bits,
                            cudaStream_t stream) {
  const int threads = 128;
  map_fill_kernel<<<(n + threads - 1) / threads, threads, 0, stream>>>(rows, codes, start, n, row, bits);
  return cudaGetLastError();
}

}  // namespace dkv
