// Tensor-core (tcgen05 + TMEM) causal GQA attention over packed mixed-precision
// history, sm_100a. Used when the stacked query rows (group * nq) form a real
// dense contraction (frame appends, candidate scoring).
//
// Semantics are those of the reference kernel packed_attention
// (src/gpu_kernels.py:71-105): dequantised history rounded to bf16 (:93-94), the
// current chunk's native K/V, q.k * D^-0.5 (:95), bottom-right causal mask (:96),
// online softmax (:98-103), p rounded to bf16 before P.V (:102), fp32 accumulation.
//
// One CTA per (KV head, block of up to 256 stacked rows, history split), 13 warps
// in three roles connected by mbarriers:
//   warps 9-12  producers: gather the split's packed history tile by tile (token
//               maps -> pool rows), dequantise in registers and write bf16 K and V
//               tiles (64 keys) into a 3-stage ring in the 128B-swizzled K-major
//               layout the tensor core reads;
//   warp 8      MMA issuer (one thread): S = Q K^T into TMEM (double-buffered), then
//               O += P V into TMEM, both tcgen05.mma kind::f16 with M = 128;
//   warps 0-7   softmax: one TMEM lane = one stacked row each; read S, mask, online
//               max / exp2 / sum in fp32, write P (bf16) to shared memory for the
//               P V product, and rescale O in TMEM when the running max moves.
// The running max is only moved when a tile's max exceeds it by more than 2^8
// (p <= 256, exact after the final O / l division); everything else is the
// reference's arithmetic. Partial (max, sum, O) per split go to the workspace and
// are merged by the deterministic combine kernel. Every mbarrier wait is bounded:
// a stalled pipeline reports DKV_ETIMEOUT in the status word and the CTA exits
// after its MMAs drain and TMEM is freed.
#include "attention.cuh"
#include "tc_ptx.cuh"

namespace dkv {
namespace {

using namespace ptx;

constexpr int kStages = 3;
constexpr int kSoftmaxWarps = 8;
constexpr int kMmaWarp = 8;
constexpr int kProdWarp0 = 9;
constexpr int kProdWarps = 4;
constexpr int kThreadsTc = (kSoftmaxWarps + 1 + kProdWarps) * 32;  // 416
constexpr int kProdThreads = kProdWarps * 32;
constexpr int kTasksPerProd = (2 * kBN * 8) / kProdThreads;  // 8 (row, 8-dim part) tasks
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0;    // S[buf][mt] at columns (buf * 2 + mt) * 64
constexpr uint32_t kColO = 256;  // O[mt] at columns 256 + mt * 64

constexpr int kTile = kBN * 128;  // one 64-key bf16 tile, 8 KB
constexpr int kOffQ = 0;          // 2 M-tiles x 128 rows x 128 B
constexpr int kOffP = kOffQ + 2 * 128 * 128;
constexpr int kOffK = kOffP + 2 * 128 * 128;
constexpr int kOffV = kOffK + kStages * kTile;
constexpr int kOffBar = kOffV + kStages * kTile;
enum {
  B_FULL = 0,
  B_EMPTY = B_FULL + kStages,
  B_SFULL = B_EMPTY + kStages,
  B_SFREE = B_SFULL + 2,
  B_PFULL = B_SFREE + 2,
  B_ODONE = B_PFULL + 1,
  B_FIN = B_ODONE + 1,
  B_COUNT = B_FIN + 1
};
constexpr int kOffTmem = kOffBar + B_COUNT * 8;
constexpr int kOffAbort = kOffTmem + 4;
constexpr int kSmemTc = kOffAbort + 4 + 1024;  // + slack to align the base to 1024 B
constexpr long long kWaitCycles = 400000000LL; // ~0.2 s: a healthy wait is microseconds

constexpr uint32_t kIdescS = idesc_bf16(128, kBN, 0);   // S = Q K^T: B = K tile, K-major
constexpr uint32_t kIdescPV = idesc_bf16(128, kDim, 1); // O = P V:  B = V tile, MN-major

__device__ __forceinline__ int swz(int row, int chunk) { return row * 128 + ((chunk ^ (row & 7)) << 4); }

__global__ void __launch_bounds__(kThreadsTc, 1) attention_tc_kernel(const AttnArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_addr(smem);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kOffAbort);

  const int split = blockIdx.x;
  const int mb = blockIdx.y;
  const int g = blockIdx.z;
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;

  const int row0 = mb * kTcCtaRows;
  const int rows_here = min(kTcCtaRows, a.mrows - row0);
  const int mt_count = (rows_here + 127) >> 7;
  const int m_max = (row0 + rows_here - 1) / a.G;
  const int kb = split * a.chunk;
  int ke = min(kb + a.chunk, a.past + a.nq);
  ke = min(ke, a.past + m_max + 1);  // no row of this block sees further
  const int ntiles = ke > kb ? (ke - kb + kBN - 1) / kBN : 0;
  const int soft_threads = ((rows_here + 31) >> 5) << 5;  // threads of softmax warps with real rows

  auto bar = [&](int i) { return sbase + kOffBar + 8 * i; };

  // ---- set-up: barriers, TMEM, Q (zero padding rows), P zeroed ----
  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar(B_FULL + s), kProdThreads);
      mbar_init(bar(B_EMPTY + s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar(B_SFULL + b), 1);
      mbar_init(bar(B_SFREE + b), soft_threads);
    }
    mbar_init(bar(B_PFULL), soft_threads);
    mbar_init(bar(B_ODONE), 1);
    mbar_init(bar(B_FIN), 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  if (warp == kMmaWarp) {
    tmem_alloc(sbase + kOffTmem, kTmemCols);
    tmem_relinquish();
  }
  for (int i = tid; i < 2 * 128 * 8; i += kThreadsTc) {
    const int r = i >> 3, c = i & 7;
    uint4 val = make_uint4(0, 0, 0, 0);
    if (r < rows_here) {
      const int fr = row0 + r;
      const int m = fr / a.G;
      const int h = g * a.G + (fr - m * a.G);
      val = __ldg(reinterpret_cast<const uint4*>(a.q + h * a.qh + m * a.qt) + c);
    }
    *reinterpret_cast<uint4*>(smem + kOffQ + (r >> 7) * 16384 + swz(r & 127, c)) = val;
    *reinterpret_cast<uint4*>(smem + kOffP + (r >> 7) * 16384 + swz(r & 127, c)) = make_uint4(0, 0, 0, 0);
  }
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(smem + kOffTmem);

  if (warp == kMmaWarp) {
    // ================= MMA issuer =================
    if (lane == 0 && ntiles > 0) {
      bool ok = true;
      auto issue_s = [&](int i) {
        const int s = i % kStages, b = i & 1;
        ok = ok && mbar_wait(bar(B_FULL + s), (i / kStages) & 1, kWaitCycles);
        if (i >= 2) ok = ok && mbar_wait(bar(B_SFREE + b), ((i >> 1) + 1) & 1, kWaitCycles);
        if (!ok) return;
        tc_fence_after();
        for (int mt = 0; mt < mt_count; ++mt) {
          const uint32_t d = tmem + kColS + (b * 2 + mt) * 64;
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint64_t ad = sw128_desc(sbase + kOffQ + mt * 16384 + k * 32, 16, 1024);
            const uint64_t bd = sw128_desc(sbase + kOffK + s * kTile + k * 32, 16, 1024);
            umma_f16(d, ad, bd, kIdescS, k > 0);
          }
        }
        umma_commit(bar(B_SFULL + b));
      };
      issue_s(0);
      for (int i = 0; i < ntiles && ok; ++i) {
        if (i + 1 < ntiles) issue_s(i + 1);
        if (!ok) break;
        ok = mbar_wait(bar(B_PFULL), i & 1, kWaitCycles);
        if (!ok) break;
        tc_fence_after();
        const int s = i % kStages;
        for (int mt = 0; mt < mt_count; ++mt) {
          const uint32_t d = tmem + kColO + mt * 64;
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint64_t ad = sw128_desc(sbase + kOffP + mt * 16384 + k * 32, 16, 1024);
            const uint64_t bd = sw128_desc(sbase + kOffV + s * kTile + k * 2048, kTile, 1024);
            umma_f16(d, ad, bd, kIdescPV, (i > 0 || k > 0) ? 1u : 0u);
          }
        }
        umma_commit(bar(B_ODONE));
        umma_commit(bar(B_EMPTY + s));
      }
      if (!ok) {
        *abort_flag = 1;
        report(a.status, DKV_ETIMEOUT, 1);
      }
      umma_commit(bar(B_FIN));  // drain every MMA before TMEM is released
      mbar_wait(bar(B_FIN), 0, kWaitCycles);
    }
    __syncwarp();
  } else if (warp < kSoftmaxWarps) {
    // ================= softmax (one TMEM lane / stacked row per thread) =================
    const int mt = warp >> 2, quad = warp & 3;
    const int rl = mt * 128 + quad * 32 + lane;  // row inside the block
    if (mt * 128 + quad * 32 < rows_here) {
      const int fr = row0 + min(rl, rows_here - 1);
      const int lim = a.past + fr / a.G;  // last key this row may see
      const uint32_t lane_base = tmem + (static_cast<uint32_t>(quad * 32) << 16);
      float m_ref = -INFINITY, l = 0.f;
      bool ok = true;
      uint8_t* prow = smem + kOffP + mt * 16384;
      const int pr = quad * 32 + lane;
      for (int i = 0; i < ntiles; ++i) {
        const int b = i & 1;
        if (__any_sync(0xffffffffu, *abort_flag != 0)) { ok = false; break; }
        ok = __all_sync(0xffffffffu, mbar_wait(bar(B_SFULL + b), (i >> 1) & 1, kWaitCycles));
        if (!ok) break;
        tc_fence_after();
        float s[64];
        {
          uint32_t r0[32], r1[32];
          tmem_ld32(lane_base + kColS + (b * 2 + mt) * 64, r0);
          tmem_ld32(lane_base + kColS + (b * 2 + mt) * 64 + 32, r1);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            s[j] = __uint_as_float(r0[j]);
            s[32 + j] = __uint_as_float(r1[j]);
          }
        }
        tc_fence_before();
        mbar_arrive(bar(B_SFREE + b));
        const int t0 = kb + i * kBN;
        if (t0 + kBN <= ke && t0 + kBN - 1 <= a.past) {
#pragma unroll
          for (int j = 0; j < 64; ++j) s[j] *= kScaleLog2;
        } else {
#pragma unroll
          for (int j = 0; j < 64; ++j) {
            const int t = t0 + j;
            s[j] = (t < ke && t <= lim) ? s[j] * kScaleLog2 : -INFINITY;
          }
        }
        float mx = s[0];
#pragma unroll
        for (int j = 1; j < 64; ++j) mx = fmaxf(mx, s[j]);
        float alpha = 1.f;
        bool rescale = false;
        if (mx > m_ref + 8.f) {  // also true for the first visible tile (m_ref = -inf)
          alpha = ex2(m_ref - mx);
          rescale = m_ref != -INFINITY;
          m_ref = mx;
        }
        const float mu = m_ref == -INFINITY ? 0.f : m_ref;
        uint32_t pk[32];
        float sum = 0.f;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float p0 = ex2(s[2 * j] - mu);
          const float p1 = ex2(s[2 * j + 1] - mu);
          sum += p0 + p1;
          pk[j] = pack_bf16x2(p0, p1);
        }
        l = l * alpha + sum;
        if (i > 0) {  // P(i-1) consumed and O stable
          ok = __all_sync(0xffffffffu, mbar_wait(bar(B_ODONE), (i - 1) & 1, kWaitCycles));
          if (!ok) break;
        }
        tc_fence_after();
        if (__any_sync(0xffffffffu, rescale)) {
          const float f = rescale ? alpha : 1.f;
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            uint32_t o[32];
            const uint32_t ta = lane_base + kColO + mt * 64 + half * 32;
            tmem_ld32(ta, o);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 32; ++j) o[j] = __float_as_uint(__uint_as_float(o[j]) * f);
            tmem_st32(ta, o);
          }
          tmem_wait_st();
        }
#pragma unroll
        for (int c = 0; c < 8; ++c)
          *reinterpret_cast<uint4*>(prow + swz(pr, c)) =
              make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(bar(B_PFULL));
      }
      // ---- epilogue: O row from TMEM ----
      float o[64];
#pragma unroll
      for (int j = 0; j < 64; ++j) o[j] = 0.f;
      if (ok && ntiles > 0) {
        ok = __all_sync(0xffffffffu, mbar_wait(bar(B_ODONE), (ntiles - 1) & 1, kWaitCycles));
        tc_fence_after();
        if (ok) {
          uint32_t r0[32], r1[32];
          tmem_ld32(lane_base + kColO + mt * 64, r0);
          tmem_ld32(lane_base + kColO + mt * 64 + 32, r1);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            o[j] = __uint_as_float(r0[j]);
            o[32 + j] = __uint_as_float(r1[j]);
          }
        }
      }
      if (!ok) {
        *abort_flag = 1;
        report(a.status, DKV_ETIMEOUT, 2);
      } else if (rl < rows_here) {
        const int frow = row0 + rl;
        if (a.splits == 1) {
          const int m = frow / a.G;
          const int h = g * a.G + (frow - m * a.G);
          uint16_t* dst = a.out + (static_cast<int64_t>(m) * a.HQ + h) * kDim;
          const float inv = 1.f / l;
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            uint4 w;
            w.x = pack_bf16x2(o[8 * c + 0] * inv, o[8 * c + 1] * inv);
            w.y = pack_bf16x2(o[8 * c + 2] * inv, o[8 * c + 3] * inv);
            w.z = pack_bf16x2(o[8 * c + 4] * inv, o[8 * c + 5] * inv);
            w.w = pack_bf16x2(o[8 * c + 6] * inv, o[8 * c + 7] * inv);
            reinterpret_cast<uint4*>(dst)[c] = w;
          }
        } else {
          const int64_t cta = (static_cast<int64_t>(g) * a.mblocks + mb) * a.splits + split;
          float4* dst = reinterpret_cast<float4*>(a.ws_o + (cta * kTcCtaRows + rl) * kDim);
#pragma unroll
          for (int c = 0; c < 16; ++c) dst[c] = make_float4(o[4 * c], o[4 * c + 1], o[4 * c + 2], o[4 * c + 3]);
          a.ws_ml[cta * kTcCtaRows + rl] = make_float2(m_ref, l);
        }
      }
    }
  } else {
    // ================= producers: gather, dequantise, stage K/V tiles =================
    const int ptid = tid - kProdWarp0 * 32;
    RowPart pre[kTasksPerProd];
    auto load = [&](int tile) {
      const int t0 = kb + tile * kBN;
#pragma unroll
      for (int i = 0; i < kTasksPerProd; ++i) {
        const int task = ptid + i * kProdThreads;
        const int kv = task >> 9;
        const int j = (task >> 3) & (kBN - 1);
        const int part = task & 7;
        const int t = t0 + j;
        pre[i].bits = 0;
        if (t < ke) {
          if (t < a.past) {
            pre[i] = load_history_part(a.P, a.rows, a.codes, a.layer, kv, g, t, part, a.status);
          } else {
            const int tn = t - a.past;
            const uint16_t* src = kv == 0 ? a.knew + g * a.kh + tn * a.kt : a.vnew + g * a.vh + tn * a.vt;
            pre[i].raw = __ldg(reinterpret_cast<const uint4*>(src) + part);
            pre[i].bits = 16;
          }
        }
      }
    };
    bool ok = true;
    if (ntiles > 0) load(0);
    for (int i = 0; i < ntiles; ++i) {
      const int s = i % kStages;
      if (*abort_flag) { ok = false; break; }
      if (i >= kStages) {
        ok = mbar_wait(bar(B_EMPTY + s), ((i / kStages) + 1) & 1, kWaitCycles);
        if (!ok) break;
      }
#pragma unroll
      for (int k = 0; k < kTasksPerProd; ++k) {
        const int task = ptid + k * kProdThreads;
        const int kv = task >> 9;
        const int j = (task >> 3) & (kBN - 1);
        const int part = task & 7;
        uint8_t* dst = smem + (kv == 0 ? kOffK : kOffV) + s * kTile + swz(j, part);
        *reinterpret_cast<uint4*>(dst) = dequant_part(pre[k]);
      }
      fence_proxy_async_smem();
      mbar_arrive(bar(B_FULL + s));
      if (i + 1 < ntiles) load(i + 1);
    }
    if (!ok) {
      *abort_flag = 1;
      report(a.status, DKV_ETIMEOUT, 3);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace

cudaError_t launch_attention_tc(const AttnArgs& a, int heads, cudaStream_t stream) {
  static bool configured[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!configured[dev]) {
    e = cudaFuncSetAttribute(attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemTc);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  dim3 grid(a.splits, a.mblocks, heads);
  attention_tc_kernel<<<grid, kThreadsTc, kSmemTc, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace dkv
