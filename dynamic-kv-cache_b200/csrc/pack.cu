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
#include "dkv_common.cuh"

namespace dkv {

constexpr int kPackThreads = 256;
constexpr int kMaxPackRequests = DKV_MAX_REQUESTS;

// Quantises part `part` (dims 8*part .. 8*part+7) of one 64-wide row held in
// `raw` (8 bf16) and stores it at row `out_row` of pool block `block` (the
// (layer, K|V, head) slab of `cap` rows). The eight lanes of a row must call it
// together (row min/max by shuffles within the 8-lane group).
template <int BITS>
__device__ __forceinline__ void pack_row_part(uint4 raw, int part, uint8_t* p4, float2* m4, uint8_t* p8,
                                              float2* m8, uint16_t* p16, int64_t block, int64_t cap,
                                              int64_t out_row, int32_t* status, int report_row) {
  float x[8];
  x[0] = bf16_lo(raw.x); x[1] = bf16_hi(raw.x);
  x[2] = bf16_lo(raw.y); x[3] = bf16_hi(raw.y);
  x[4] = bf16_lo(raw.z); x[5] = bf16_hi(raw.z);
  x[6] = bf16_lo(raw.w); x[7] = bf16_hi(raw.w);
  bool finite = true;
#pragma unroll
  for (int i = 0; i < 8; ++i) finite &= isfinite(x[i]);
  if (!finite) report(status, DKV_ENONFINITE, report_row);

  if (BITS == 16) {
    reinterpret_cast<uint4*>(p16 + (block * cap + out_row) * kDim)[part] = raw;
    return;
  }

  // Row min/max over the 8 lanes of this row's group.
  const unsigned lane = threadIdx.x & 31;
  const unsigned mask = 0xffu << (lane & 24);
  float mn = x[0], mx = x[0];
#pragma unroll
  for (int i = 1; i < 8; ++i) { mn = fminf(mn, x[i]); mx = fmaxf(mx, x[i]); }
#pragma unroll
  for (int off = 1; off < 8; off <<= 1) {
    mn = fminf(mn, __shfl_xor_sync(mask, mn, off, 8));
    mx = fmaxf(mx, __shfl_xor_sync(mask, mx, off, 8));
  }
  // Operation order of src/kv_quantization.py:63-66, every step IEEE fp32
  // round-to-nearest (explicit intrinsics: no contraction into FMA).
  constexpr float kLevels = static_cast<float>((1 << BITS) - 1);
  const float offset = mn;
  const float span = __fsub_rn(mx, offset);
  const float scale = span > 0.f ? __fdiv_rn(span, kLevels) : 1.f;
  uint32_t q[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float t = rintf(__fdiv_rn(__fsub_rn(x[i], offset), scale));  // round half to even
    t = fminf(fmaxf(t, 0.f), kLevels);
    q[i] = static_cast<uint32_t>(t);
  }
  if (BITS == 8) {
    uint2 w;
    w.x = q[0] | (q[1] << 8) | (q[2] << 16) | (q[3] << 24);
    w.y = q[4] | (q[5] << 8) | (q[6] << 16) | (q[7] << 24);
    reinterpret_cast<uint2*>(p8 + (block * cap + out_row) * kRowBytes8)[part] = w;
    if (part == 0) m8[block * cap + out_row] = make_float2(offset, scale);
  } else {
    uint32_t w = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) w |= (q[2 * j] | (q[2 * j + 1] << 4)) << (8 * j);
    reinterpret_cast<uint32_t*>(p4 + (block * cap + out_row) * kRowBytes4)[part] = w;
    if (part == 0) m4[block * cap + out_row] = make_float2(offset, scale);
  }
}

template <int BITS>
__global__ void __launch_bounds__(kPackThreads)
pack_rows_kernel(const uint16_t* __restrict__ k, const uint16_t* __restrict__ v,
                 uint8_t* __restrict__ p4, float2* __restrict__ m4, uint8_t* __restrict__ p8,
                 float2* __restrict__ m8, uint16_t* __restrict__ p16, int64_t kh, int64_t kt,
                 int64_t vh, int64_t vt, int layer, int64_t row_start, int n, int64_t cap,
                 int heads, int32_t* status) {
  // Launched as a programmatic dependent: the next kernel (the frame's attention,
  // which reads the new K/V natively and only history rows of the pools) may start
  // streaming history at once; k / v are the previous kernels' output.
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
  asm volatile("griddepcontrol.wait;\n" ::: "memory");
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
  pack_row_part<BITS>(raw, part, p4, m4, p8, m8, p16, block, cap, row_start + token, status, row);
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
                      int64_t kc, int64_t vc, int layer, int n, int heads) {
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
  asm volatile("griddepcontrol.wait;\n" ::: "memory");
  const dkv_pack_target& d = tab[blockIdx.y];
  const int bits = d.bits;
  const int64_t cap = bits == 4 ? d.cap4 : (bits == 8 ? d.cap8 : d.cap16);
  const int64_t row_start = d.row_start;
  const bool pool_ok = bits == 4 ? (d.p4 != nullptr && d.m4 != nullptr)
                                 : (bits == 8 ? (d.p8 != nullptr && d.m8 != nullptr) : d.p16 != nullptr);
  if ((bits != 4 && bits != 8 && bits != 16) || !pool_ok) {
    if (blockIdx.x == 0 && threadIdx.x == 0) report(d.status, DKV_EINVAL, blockIdx.y);
    return;
  }
  if (row_start < 0 || row_start + n > cap) {
    if (blockIdx.x == 0 && threadIdx.x == 0) report(d.status, DKV_ECAPACITY, blockIdx.y);
    return;
  }
  const int gtid = blockIdx.x * blockDim.x + threadIdx.x;
  const int row = gtid >> 3;
  const int part = gtid & 7;
  const int per_kv = heads * n;
  if (row >= 2 * per_kv) return;
  const int kv = row / per_kv;
  const int rem = row - kv * per_kv;
  const int head = rem / n;
  const int token = rem - head * n;
  const uint16_t* src = kv == 0 ? k + blockIdx.y * kc + head * kh + token * kt
                                : v + blockIdx.y * vc + head * vh + token * vt;
  const uint4 raw = __ldg(reinterpret_cast<const uint4*>(src) + part);
  const int64_t block = (static_cast<int64_t>(layer) * 2 + kv) * heads + head;
  const int64_t out_row = row_start + token;
  uint8_t* p4 = static_cast<uint8_t*>(d.p4);
  uint8_t* p8 = static_cast<uint8_t*>(d.p8);
  float2* m4 = static_cast<float2*>(d.m4);
  float2* m8 = static_cast<float2*>(d.m8);
  uint16_t* p16 = static_cast<uint16_t*>(d.p16);
  if (bits == 4) {
    pack_row_part<4>(raw, part, p4, m4, p8, m8, p16, block, cap, out_row, d.status, row);
  } else if (bits == 8) {
    pack_row_part<8>(raw, part, p4, m4, p8, m8, p16, block, cap, out_row, d.status, row);
  } else {
    pack_row_part<16>(raw, part, p4, m4, p8, m8, p16, block, cap, out_row, d.status, row);
  }
  if (d.map_rows != nullptr && kv == 0 && head == 0 && part == 0) {
    const int64_t at = d.map_start + token;
    if (d.map_codes == nullptr || d.map_start < 0 || d.map_start + n > d.map_capacity) {
      report(d.status, DKV_ECAPACITY, blockIdx.y);
    } else {
      d.map_rows[at] = static_cast<int32_t>(out_row);
      d.map_codes[at] = static_cast<uint8_t>(bits);
    }
  }
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
                        int64_t row_start, int n, int64_t cap, int heads, int bits,
                        int32_t* status, cudaStream_t stream) {
  const int threads = 2 * heads * n * 8;
  const int blocks = (threads + kPackThreads - 1) / kPackThreads;
  const uint16_t* kk = static_cast<const uint16_t*>(k);
  const uint16_t* vv = static_cast<const uint16_t*>(v);
  uint8_t* q4 = static_cast<uint8_t*>(p4);
  uint8_t* q8 = static_cast<uint8_t*>(p8);
  float2* s4 = static_cast<float2*>(m4);
  float2* s8 = static_cast<float2*>(m8);
  uint16_t* h = static_cast<uint16_t*>(p16);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(blocks);
  cfg.blockDim = dim3(kPackThreads);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  auto kernel = bits == 4 ? pack_rows_kernel<4> : (bits == 8 ? pack_rows_kernel<8> : pack_rows_kernel<16>);
  return cudaLaunchKernelEx(&cfg, kernel, kk, vv, q4, s4, q8, s8, h, kh, kt, vh, vt, layer, row_start, n, cap,
                            heads, status);
}

template <class Targets>
cudaError_t launch_pack_many_with(const void* k, const void* v, const Targets& tab, int count, int64_t kh,
                                  int64_t kt, int64_t vh, int64_t vt, int64_t kc, int64_t vc, int layer, int n,
                                  int heads, cudaStream_t stream) {
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
                            static_cast<const uint16_t*>(v), tab, kh, kt, vh, vt, kc, vc, layer, n, heads);
}

// targets: host array (copied into the launch) or, with on_device, device memory.
cudaError_t launch_pack_many(const void* k, const void* v, const dkv_pack_target* targets, bool on_device, int count,
                             int64_t kh, int64_t kt, int64_t vh, int64_t vt, int64_t kc, int64_t vc, int layer, int n,
                             int heads, cudaStream_t stream) {
  if (on_device)
    return launch_pack_many_with(k, v, DevicePackTargets{targets}, count, kh, kt, vh, vt, kc, vc, layer, n, heads,
                                 stream);
  PackTable tab{};
  for (int r = 0; r < count; ++r) tab.t[r] = targets[r];
  return launch_pack_many_with(k, v, tab, count, kh, kt, vh, vt, kc, vc, layer, n, heads, stream);
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
