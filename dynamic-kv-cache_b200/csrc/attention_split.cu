// Split-KV causal GQA attention over packed mixed-precision history (sm_100a).
//
// Semantics follow the reference Triton kernel packed_attention
// (src/gpu_kernels.py:71-105): history tokens t < past are dequantised from the
// 4/8/16-bit pools and rounded to bf16 (:93-94), the nq current tokens use the
// native K/V, scores are q.k * D^-0.5 (:95) with the bottom-right causal mask
// t <= past + m (:96), softmax is online with exp (:98-103) and p is rounded to
// bf16 before the P.V product (:102), accumulation in fp32.
//
// B200 decomposition (differs from the reference's one program per query head):
//  - one CTA per (KV head, row block, history split): the G query heads that share
//    a KV head are stacked as rows (row r = query r/G, head r%G), so each history
//    tile is read and dequantised ONCE for all of them instead of G times;
//  - the history is split across CTAs to fill the 148 SMs, partial (max, sum,
//    unnormalised output) go to a workspace and a second kernel merges them in a
//    fixed split order (deterministic, no atomics);
//  - each warp owns 16 rows; tiles of 64 keys are dequantised cooperatively into
//    XOR-swizzled shared memory while the next tile's packed bytes are already in
//    flight (register double buffering), then consumed by ldmatrix + mma.sync.
#include "attention.cuh"
#include "tc_ptx.cuh"

namespace dkv {
namespace {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Byte offset of 16-byte chunk `chunk` of 128-byte row `row` in a swizzled tile.
__device__ __forceinline__ int swz(int row, int chunk) {
  return row * 128 + ((chunk ^ (row & 7)) << 4);
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void mma_bf16(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

constexpr int kTileTasks = 2 * kBN * 8;  // (K|V) x 64 keys x 8 parts of 8 dims

template <int NW, class Hist>
__global__ void __launch_bounds__(NW * 32)
attention_split_kernel(const __grid_constant__ AttnArgs a, const __grid_constant__ Hist hist) {
  constexpr int kThreads = NW * 32;
  constexpr int kTPT = (kTileTasks + kThreads - 1) / kThreads;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* sQ = smem;
  uint8_t* sK = smem + a.cta_rows * 128;
  uint8_t* sV = sK + 2 * kBN * 128;

  const int split = blockIdx.x;
  const int mb = blockIdx.y;
  const int zc = blockIdx.z;  // chunk * heads + KV head
  const int chunk = zc / a.heads;
  const int g = zc - chunk * a.heads;
  const History& H = history_of(a, hist, chunk);
  const int past = checked_past(H, chunk);
  const Pools P{static_cast<const uint8_t*>(H.p4), static_cast<const float2*>(H.m4),
                static_cast<const uint8_t*>(H.p8), static_cast<const float2*>(H.m8),
                static_cast<const uint16_t*>(H.p16), H.cap4, H.cap8, H.cap16, a.heads};
  const int32_t* const map_rows = H.rows;
  const uint8_t* const map_codes = H.codes;
  int32_t* const status = H.status;
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;

  const int row0 = mb * a.cta_rows;
  const int rows_here = min(a.cta_rows, a.mrows - row0);
  const int m_max = (row0 + rows_here - 1) / a.G;
  const int keys = request_chunk(a, past);
  const int kb = split * keys;
  int ke = min(kb + keys, past + a.nq);
  ke = min(ke, past + m_max + 1);  // no row of this block sees further
  const int ntiles = ke > kb ? (ke - kb + kBN - 1) / kBN : 0;

  // ---- Q block -> shared (zero rows past the end) ----
  for (int i = tid; i < a.cta_rows * 8; i += kThreads) {
    const int r = i >> 3, c = i & 7;
    uint4 val = make_uint4(0, 0, 0, 0);
    if (r < rows_here) {
      const int fr = row0 + r;
      const int m = fr / a.G;
      const int h = g * a.G + (fr - m * a.G);
      val = __ldg(reinterpret_cast<const uint4*>(a.q + chunk * a.qc + h * a.qh + m * a.qt) + c);
    }
    *reinterpret_cast<uint4*>(sQ + swz(r, c)) = val;
  }

  // ---- packed tile prefetch (registers) and dequantising store (shared) ----
  RowPart pre[kTPT];
  auto load_tile = [&](int tile) {
    const int t0 = kb + tile * kBN;
#pragma unroll
    for (int i = 0; i < kTPT; ++i) {
      const int task = tid + i * kThreads;
      pre[i].bits = 0;
      if (task < kTileTasks) {
        const int kv = task >> 9;
        const int j = (task >> 3) & (kBN - 1);
        const int part = task & 7;
        const int t = t0 + j;
        if (t < ke) {
          if (t < past) {
            pre[i] = load_history_part(P, map_rows, map_codes, a.layer, kv, g, t, part, status);
          } else {
            const int tn = t - past;
            const uint16_t* src = kv == 0 ? a.knew + chunk * a.kc + g * a.kh + tn * a.kt
                                          : a.vnew + chunk * a.vc + g * a.vh + tn * a.vt;
            pre[i].raw = __ldg(reinterpret_cast<const uint4*>(src) + part);
            pre[i].bits = 16;
          }
        }
      }
    }
  };
  auto store_tile = [&](int buf) {
#pragma unroll
    for (int i = 0; i < kTPT; ++i) {
      const int task = tid + i * kThreads;
      if (task < kTileTasks) {
        const int kv = task >> 9;
        const int j = (task >> 3) & (kBN - 1);
        const int part = task & 7;
        uint8_t* dst = (kv == 0 ? sK : sV) + buf * (kBN * 128) + swz(j, part);
        *reinterpret_cast<uint4*>(dst) = dequant_part(pre[i]);
      }
    }
  };

  const int cw = a.cta_rows >> 4;  // compute warps
  const bool computes = warp < cw;
  // Rows of this thread inside the block: ra (fragment rows 0-7) and ra + 8.
  const int ra = warp * 16 + (lane >> 2);
  const int rb = ra + 8;
  const int lim_a = past + min(row0 + ra, a.mrows - 1) / a.G;  // last visible key
  const int lim_b = past + min(row0 + rb, a.mrows - 1) / a.G;

  float o[8][4];
#pragma unroll
  for (int j = 0; j < 8; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[j][e] = 0.f;
  float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;
  uint32_t qf[4][4];

  if (ntiles > 0) {
    load_tile(0);
    store_tile(0);
  }
  __syncthreads();
  if (computes) {
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const int r = warp * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);
      ldsm_x4(qf[kk], smem_u32(sQ + swz(r, 2 * kk + (lane >> 4))));
    }
  }

  for (int it = 0; it < ntiles; ++it) {
    const int buf = it & 1;
    if (it + 1 < ntiles) load_tile(it + 1);
    if (computes) {
      const int t0 = kb + it * kBN;
      const uint8_t* tK = sK + buf * (kBN * 128);
      const uint8_t* tV = sV + buf * (kBN * 128);
      float s[8][4];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
#pragma unroll
        for (int e = 0; e < 4; ++e) s[j][e] = 0.f;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          uint32_t b[4];
          ldsm_x4(b, smem_u32(tK + swz(8 * j + (lane & 7), 4 * h + (lane >> 3))));
          mma_bf16(s[j], qf[2 * h], b[0], b[1]);
          mma_bf16(s[j], qf[2 * h + 1], b[2], b[3]);
        }
      }
      // mask + scale, row maxima
      float mx_a = m_a, mx_b = m_b;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int t = t0 + 8 * j + 2 * (lane & 3) + (e & 1);
          const int lim = e < 2 ? lim_a : lim_b;
          const bool ok = t < ke && t <= lim;
          s[j][e] = ok ? s[j][e] * kScaleLog2 : -INFINITY;
        }
        mx_a = fmaxf(mx_a, fmaxf(s[j][0], s[j][1]));
        mx_b = fmaxf(mx_b, fmaxf(s[j][2], s[j][3]));
      }
#pragma unroll
      for (int off = 1; off < 4; off <<= 1) {
        mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, off));
        mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, off));
      }
      const float use_a = mx_a == -INFINITY ? 0.f : mx_a;
      const float use_b = mx_b == -INFINITY ? 0.f : mx_b;
      const float al_a = exp2f(m_a - use_a);
      const float al_b = exp2f(m_b - use_b);
      m_a = mx_a;
      m_b = mx_b;
      float sum_a = 0.f, sum_b = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        s[j][0] = exp2f(s[j][0] - use_a);
        s[j][1] = exp2f(s[j][1] - use_a);
        s[j][2] = exp2f(s[j][2] - use_b);
        s[j][3] = exp2f(s[j][3] - use_b);
        sum_a += s[j][0] + s[j][1];
        sum_b += s[j][2] + s[j][3];
      }
      l_a = l_a * al_a + sum_a;
      l_b = l_b * al_b + sum_b;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        o[j][0] *= al_a;
        o[j][1] *= al_a;
        o[j][2] *= al_b;
        o[j][3] *= al_b;
      }
      // O += P V  (P rounded to bf16 as in the reference)
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        uint32_t pa[4];
        pa[0] = pack_bf16x2(s[2 * kk][0], s[2 * kk][1]);
        pa[1] = pack_bf16x2(s[2 * kk][2], s[2 * kk][3]);
        pa[2] = pack_bf16x2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
        pa[3] = pack_bf16x2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
        for (int jd = 0; jd < 8; jd += 2) {
          uint32_t b[4];
          const int r = 16 * kk + (lane & 7) + 8 * ((lane >> 3) & 1);
          ldsm_x4_t(b, smem_u32(tV + swz(r, jd + (lane >> 4))));
          mma_bf16(o[jd], pa, b[0], b[1]);
          mma_bf16(o[jd + 1], pa, b[2], b[3]);
        }
      }
    }
    if (it + 1 < ntiles) store_tile(buf ^ 1);
    __syncthreads();
  }

  if (!computes) return;
#pragma unroll
  for (int off = 1; off < 4; off <<= 1) {
    l_a += __shfl_xor_sync(0xffffffffu, l_a, off);
    l_b += __shfl_xor_sync(0xffffffffu, l_b, off);
  }
  const int c2 = 2 * (lane & 3);
  if (a.splits == 1) {
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int r = half ? rb : ra;
      const int fr = row0 + r;
      if (r >= rows_here) continue;
      const float inv = 1.f / (half ? l_b : l_a);
      const int m = fr / a.G;
      const int h = g * a.G + (fr - m * a.G);
      uint16_t* dst = a.out + chunk * a.oc + (static_cast<int64_t>(m) * a.HQ + h) * kDim;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float x0 = o[j][2 * half] * inv, x1 = o[j][2 * half + 1] * inv;
        *reinterpret_cast<uint32_t*>(dst + 8 * j + c2) = pack_bf16x2(x0, x1);
      }
    }
    return;
  }
  // partial layout of part_o / part_ml, shared with the tensor-core kernel
  const int grp = zc * a.mblocks + mb;
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int r = half ? rb : ra;
    float* base = a.ws_o + part_o(grp, r, a.cta_rows, a.splits, split);
#pragma unroll
    for (int j = 0; j < 8; ++j)
      *reinterpret_cast<float2*>(base + 8 * j + c2) = make_float2(o[j][2 * half], o[j][2 * half + 1]);
    if ((lane & 3) == 0)
      a.ws_ml[part_ml(grp, r, a.cta_rows, a.splits, split)] = half ? make_float2(m_b, l_b) : make_float2(m_a, l_a);
  }
}

// Merges the split partials of 4 (KV head, row) pairs per block when the
// attention kernel did not merge them itself, with the in-kernel merge's
// arithmetic (merge_row_weights, then the fused multiply-add chain in split
// order): the same bits either way. A warp per row finds the weights; then one
// thread per (row, dim) sums its column, 16 partial loads in flight at a time,
// and stores its bf16 output (a warp writes 64 contiguous bytes).
__global__ void __launch_bounds__(256) attention_combine_kernel(const __grid_constant__ AttnArgs a) {
  __shared__ float s_w[4 * kTargetCtas], s_den[4];
  ptx::pdl_wait();  // partials of the attention grid
  ptx::pdl_trigger();
  const int zc = blockIdx.z;  // chunk * heads + KV head
  const int chunk = zc / a.heads;
  const int g = zc - chunk * a.heads;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int fr0 = blockIdx.x * 4;
  if (warp < 4 && fr0 + warp < a.mrows) {
    const int fr = fr0 + warp;
    const int mb = fr / a.cta_rows;
    const float2* ml = a.ws_ml + part_ml(zc * a.mblocks + mb, fr - mb * a.cta_rows, a.cta_rows, a.splits, 0);
    const float den = merge_row_weights([&](int sp) { return ml[sp]; }, a.splits, s_w + warp * kTargetCtas, lane);
    if (lane == 0) s_den[warp] = den;
  }
  __syncthreads();
  const int rl = threadIdx.x >> 6, d = threadIdx.x & 63;
  const int fr = fr0 + rl;
  if (fr >= a.mrows) return;
  const int mb = fr / a.cta_rows;
  const float* src = a.ws_o + part_o(zc * a.mblocks + mb, fr - mb * a.cta_rows, a.cta_rows, a.splits, 0) + d;
  const int64_t sstride = kDim;
  float acc = 0.f;
  int sp = 0;
  for (; sp + 16 <= a.splits; sp += 16) {  // whole batches: 16 loads in flight
    float x[16];
#pragma unroll
    for (int u = 0; u < 16; ++u) x[u] = __ldcg(src + (sp + u) * sstride);
#pragma unroll
    for (int u = 0; u < 16; ++u) acc = __fmaf_rn(s_w[rl * kTargetCtas + sp + u], x[u], acc);
  }
  {
    float x[16];
    const int rem = a.splits - sp;
#pragma unroll
    for (int u = 0; u < 16; ++u) x[u] = u < rem ? __ldcg(src + (sp + u) * sstride) : 0.f;
#pragma unroll
    for (int u = 0; u < 16; ++u)
      if (u < rem) acc = __fmaf_rn(s_w[rl * kTargetCtas + sp + u], x[u], acc);
  }
  const float val = __fdiv_rn(acc, s_den[rl]);
  const int m = fr / a.G;
  const int h = g * a.G + (fr - m * a.G);
  a.out[chunk * a.oc + (static_cast<int64_t>(m) * a.HQ + h) * kDim + d] =
      static_cast<uint16_t>(pack_bf16x2(val, 0.f) & 0xffffu);
}

template <int NW, class Hist>
cudaError_t launch_nw(const AttnArgs& a, const Hist& hist, int heads, size_t smem, cudaStream_t stream) {
  static bool configured[64] = {};  // the attribute is set once per device
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    e = cudaFuncSetAttribute(attention_split_kernel<NW, Hist>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             96 * 1024);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  dim3 grid(a.splits, a.mblocks, heads);
  attention_split_kernel<NW, Hist><<<grid, NW * 32, smem, stream>>>(a, hist);
  return cudaGetLastError();
}

template <class Hist>
cudaError_t launch_split(const AttnArgs& a, const Hist& hist, int heads, cudaStream_t stream) {
  const int cw = a.cta_rows / 16;
  const size_t smem = static_cast<size_t>(a.cta_rows) * 128 + 4 * kBN * 128;
  if (cw <= 4) return launch_nw<4>(a, hist, heads, smem, stream);
  if (cw <= 8) return launch_nw<8>(a, hist, heads, smem, stream);
  return launch_nw<12>(a, hist, heads, smem, stream);
}

}  // namespace

cudaError_t launch_attention_split(const AttnArgs& a, int heads, cudaStream_t stream, const HistoryTable* table,
                                   const History* device_table) {
  if (table != nullptr) return launch_split(a, *table, heads, stream);
  if (device_table != nullptr) return launch_split(a, DeviceHistories{device_table}, heads, stream);
  return launch_split(a, SharedHistory{}, heads, stream);
}

cudaError_t launch_attention_combine(const AttnArgs& a, int heads, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((a.mrows + 3) / 4, 1, heads);
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, attention_combine_kernel, a);
}

}  // namespace dkv
