// Pointwise decoder ops on either side of the packed-KV path (sm_100a), each one
// launch where the PyTorch formulation takes several:
//
// rotary_kernel   <- the rotate-half rotary embedding the reference's patched
//                    attention forward applies to q and k before append/attend
//                    (src/gpu_cache.py:170, HF apply_rotary_pos_emb), in the fp32
//                    form of the streaming decoder (src/decoder.py apply_rope):
//                    seven PyTorch launches (upcast, negate, concatenate, two
//                    products, sum, downcast) become one.
// silu_mul_kernel <- activation_product, silu(gate) * up (src/gpu_ops.py:14-17):
//                    two launches become one.
// add_rms_norm_kernel <- the decoder layer's residual add followed by the next
//                    RMSNorm and its weight (cuda_rms, src/gpu_ops.py:9-12): three
//                    launches become one. Its rounding points are PyTorch's (the sum
//                    rounded to bf16, the normalised row rounded to bf16 before the
//                    weight product), but its fp32 sum of squares has its own order,
//                    so the normalised output can differ from torch's rms_norm in the
//                    last bf16 bit; it serves the streaming decoder, not cuda_rms.
//
// The first two keep PyTorch's rounding points exactly, so their outputs are
// bit-identical to the PyTorch ops they replace: every product and sum is one IEEE fp32 operation
// rounded to nearest (no contraction into FMA), and each value PyTorch stores as
// bf16 is rounded to bf16 (nearest-even) at the same point.
#include "dkv_common.cuh"

namespace dkv {

constexpr int kOpThreads = 256;

__device__ __forceinline__ void load8(const uint16_t* p, float* x) {
  const uint4 w = *reinterpret_cast<const uint4*>(p);
  x[0] = bf16_lo(w.x); x[1] = bf16_hi(w.x);
  x[2] = bf16_lo(w.y); x[3] = bf16_hi(w.y);
  x[4] = bf16_lo(w.z); x[5] = bf16_hi(w.z);
  x[6] = bf16_lo(w.w); x[7] = bf16_hi(w.w);
}

__device__ __forceinline__ void load8f(const float* p, float* x) {
  const float4 a = reinterpret_cast<const float4*>(p)[0];
  const float4 b = reinterpret_cast<const float4*>(p)[1];
  x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
  x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
}

__device__ __forceinline__ void store8(uint16_t* p, const float* y) {
  uint4 w;
  w.x = pack_bf16x2(y[0], y[1]);
  w.y = pack_bf16x2(y[2], y[3]);
  w.z = pack_bf16x2(y[4], y[5]);
  w.w = pack_bf16x2(y[6], y[7]);
  *reinterpret_cast<uint4*>(p) = w;
}

// One (token, head) row of 64 dims per 4 threads; thread `part` owns dims
// 8*part..8*part+7 of the lower half and the same dims + 32 of the upper half:
//   out[i]      = x[i] * cos[i]           + (-x[i + 32]) * sin[i]
//   out[i + 32] = x[i + 32] * cos[i + 32] + x[i] * sin[i + 32]
// x: bf16 [b, n, >= heads, 64] with token strides (xb, xt); cos / sin: fp32
// [b or 1, n, 64] with strides (cb, 64) (cb = 0 broadcasts one table over b);
// out: bf16 [b, n, heads, 64], contiguous.
__global__ void __launch_bounds__(kOpThreads)
rotary_kernel(const uint16_t* __restrict__ x, const float* __restrict__ cos_t, const float* __restrict__ sin_t,
              uint16_t* __restrict__ out, int64_t xb, int64_t xt, int64_t cb, int n, int heads, int64_t total) {
  asm volatile("griddepcontrol.wait;\n" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
  const int64_t gtid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (gtid >= total) return;
  const int part = static_cast<int>(gtid & 3);
  const int64_t row = gtid >> 2;  // (b, t, head)
  const int head = static_cast<int>(row % heads);
  const int64_t token = row / heads;
  const int64_t b = token / n;
  const int64_t t = token - b * n;
  const uint16_t* src = x + b * xb + t * xt + head * kDim + part * 8;
  const int64_t table = b * cb + t * kDim + part * 8;
  float lo[8], hi[8], cl[8], ch[8], sl[8], sh[8], ylo[8], yhi[8];
  load8(src, lo);
  load8(src + kDim / 2, hi);
  load8f(cos_t + table, cl);
  load8f(cos_t + table + kDim / 2, ch);
  load8f(sin_t + table, sl);
  load8f(sin_t + table + kDim / 2, sh);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    ylo[j] = __fadd_rn(__fmul_rn(lo[j], cl[j]), __fmul_rn(-hi[j], sl[j]));
    yhi[j] = __fadd_rn(__fmul_rn(hi[j], ch[j]), __fmul_rn(lo[j], sh[j]));
  }
  uint16_t* dst = out + row * kDim + part * 8;
  store8(dst, ylo);
  store8(dst + kDim / 2, yhi);
}

// silu(gate) * up over rows of `width` elements, 8 per thread: silu as
// gate / (1 + exp(-gate)) in fp32 rounded to bf16, then the bf16 product computed
// in fp32 and rounded to bf16. gate / up: bf16 with row strides gs / us; out:
// bf16 [rows, width], contiguous.
__global__ void __launch_bounds__(kOpThreads)
silu_mul_kernel(const uint16_t* __restrict__ gate, const uint16_t* __restrict__ up, uint16_t* __restrict__ out,
                int64_t gs, int64_t us, int width, int64_t total) {
  asm volatile("griddepcontrol.wait;\n" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
  const int64_t gtid = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (gtid >= total) return;
  const int chunks = width / 8;
  const int64_t row = gtid / chunks;
  const int col = static_cast<int>(gtid - row * chunks) * 8;
  float g[8], u[8], y[8];
  load8(gate + row * gs + col, g);
  load8(up + row * us + col, u);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float s = __bfloat162float(__float2bfloat16_rn(g[j] / (1.0f + expf(-g[j]))));
    y[j] = __fmul_rn(s, u[j]);
  }
  store8(out + row * width + col, y);
}

// One warp per row of `width` (<= kNormMaxWidth) elements: with `y`, x_out = bf16(x +
// y) (fp32 sum rounded, PyTorch's bf16 add) and the norm is taken of x_out; without
// it, of x. Sum of squares in fp32 (each lane its chunks in order, then a fixed xor
// butterfly), rstd = rsqrt(sum / width + eps), h = bf16(bf16(v * rstd) * weight).
// Rows of x / y / x_out / h_out start xs / ys / os / hs elements apart.
constexpr int kNormMaxWidth = 2048;  // 8 chunks of 8 per lane
constexpr int kNormThreads = 128;  // 4 rows per block: a 512-row step spreads over 128 SMs
template <bool ADD>
__global__ void __launch_bounds__(kNormThreads)
add_rms_norm_kernel(const uint16_t* __restrict__ x, const uint16_t* __restrict__ y, uint16_t* __restrict__ x_out,
                    uint16_t* __restrict__ h_out, const uint16_t* __restrict__ weight, int64_t rows, int width,
                    int64_t xs, int64_t ys, int64_t os, int64_t hs, float eps) {
  asm volatile("griddepcontrol.wait;\n" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
  const int64_t row = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;  // whole warps leave together
  const int chunks = width / 8;
  float v[kNormMaxWidth / 256][8];
  uint4 wv[kNormMaxWidth / 256];  // the weights, loaded with the row (no second round trip)
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kNormMaxWidth / 256; ++i) {
    const int c = lane + 32 * i;
    if (c < chunks) {
      wv[i] = __ldg(reinterpret_cast<const uint4*>(weight + c * 8));
      load8(x + row * xs + c * 8, v[i]);
      if (ADD) {
        float b[8];
        load8(y + row * ys + c * 8, b);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] = __bfloat162float(__float2bfloat16_rn(__fadd_rn(v[i][j], b[j])));
        store8(x_out + row * os + c * 8, v[i]);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) ss = __fmaf_rn(v[i][j], v[i][j], ss);
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  const float rstd = rsqrtf(__fdiv_rn(ss, static_cast<float>(width)) + eps);
#pragma unroll
  for (int i = 0; i < kNormMaxWidth / 256; ++i) {
    const int c = lane + 32 * i;
    if (c < chunks) {
      float w[8], h[8];
      w[0] = bf16_lo(wv[i].x); w[1] = bf16_hi(wv[i].x);
      w[2] = bf16_lo(wv[i].y); w[3] = bf16_hi(wv[i].y);
      w[4] = bf16_lo(wv[i].z); w[5] = bf16_hi(wv[i].z);
      w[6] = bf16_lo(wv[i].w); w[7] = bf16_hi(wv[i].w);
#pragma unroll
      for (int j = 0; j < 8; ++j) h[j] = __fmul_rn(__bfloat162float(__float2bfloat16_rn(__fmul_rn(v[i][j], rstd))), w[j]);
      store8(h_out + row * hs + c * 8, h);
    }
  }
}

namespace {

// Launched as a programmatic dependent, like the pack kernel: each kernel waits
// (griddepcontrol.wait) before its first read and only then lets its own
// dependent (the attention kernel after the rotary) start its set-up, so the
// dependent knows every kernel before this one has completed.
template <class Kernel, class... Args>
cudaError_t launch_pdl_block(int block, int64_t threads, cudaStream_t stream, Kernel kernel, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>((threads + block - 1) / block));
  cfg.blockDim = dim3(block);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

template <class Kernel, class... Args>
cudaError_t launch_pdl(int64_t threads, cudaStream_t stream, Kernel kernel, Args... args) {
  return launch_pdl_block(kOpThreads, threads, stream, kernel, args...);
}

}  // namespace

cudaError_t launch_rotary(const void* x, const float* cos_t, const float* sin_t, void* out, int64_t xb, int64_t xt,
                          int64_t cb, int b, int n, int heads, cudaStream_t stream) {
  const int64_t total = static_cast<int64_t>(b) * n * heads * 4;
  return launch_pdl(total, stream, rotary_kernel, static_cast<const uint16_t*>(x), cos_t, sin_t,
                    static_cast<uint16_t*>(out), xb, xt, cb, n, heads, total);
}

cudaError_t launch_silu_mul(const void* gate, const void* up, void* out, int64_t gs, int64_t us, int64_t rows,
                            int width, cudaStream_t stream) {
  const int64_t total = rows * (width / 8);
  return launch_pdl(total, stream, silu_mul_kernel, static_cast<const uint16_t*>(gate),
                    static_cast<const uint16_t*>(up), static_cast<uint16_t*>(out), gs, us, width, total);
}

cudaError_t launch_add_rms_norm(const void* x, const void* y, void* x_out, void* h_out, const void* weight,
                                int64_t rows, int width, int64_t xs, int64_t ys, int64_t os, int64_t hs, float eps,
                                cudaStream_t stream) {
  const auto* xx = static_cast<const uint16_t*>(x);
  const auto* yy = static_cast<const uint16_t*>(y);
  auto* xo = static_cast<uint16_t*>(x_out);
  auto* ho = static_cast<uint16_t*>(h_out);
  const auto* w = static_cast<const uint16_t*>(weight);
  if (y != nullptr)
    return launch_pdl_block(kNormThreads, rows * 32, stream, add_rms_norm_kernel<true>, xx, yy, xo, ho, w, rows, width,
                            xs, ys, os, hs, eps);
  return launch_pdl_block(kNormThreads, rows * 32, stream, add_rms_norm_kernel<false>, xx, yy, xo, ho, w, rows, width,
                          xs, ys, os, hs, eps);
}

}  // namespace dkv
