// Split merge as a kernel of its own (sm_100a): the merge of single-request
// attend-only calls (an eager cooperative launch costs more than this second
// launch), of calls whose attention grid cannot be resident all at once, and of
// every call with DKV_ATTENTION_MERGE=combine. The tensor-core attention kernel
// then only writes the per-split partials of (max, sum, unnormalised output), and
// this kernel merges them in a fixed split order (deterministic, no atomics), with
// the same arithmetic as the in-kernel merge, so the output has the same bits
// either way.
#include "attention.cuh"
#include "tc_ptx.cuh"

namespace dkv {
namespace {

// Merges the split partials of 4 (KV head, row) pairs per block when the
// attention kernel did not merge them itself, with the in-kernel merge's
// arithmetic (merge_row_weights, then the fused multiply-add chain in split
// order): the same bits either way. One thread per (row, dim) loads its column of
// the first kBatch splits at once, so those loads are in flight while a warp per
// row finds the weights (one L2 round trip for both at up to kBatch splits);
// further splits follow 16 loads at a time. Each thread stores its bf16 output
// (a warp writes 64 contiguous bytes).
constexpr int kBatch = 32;

__global__ void __launch_bounds__(256) attention_combine_kernel(const __grid_constant__ AttnArgs a) {
  __shared__ float s_w[4 * kTargetCtas], s_den[4];
  ptx::pdl_wait();  // partials of the attention grid
  ptx::pdl_trigger();
  const int zc = blockIdx.z;  // chunk * heads + KV head
  const int chunk = zc / a.heads;
  const int g = zc - chunk * a.heads;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int fr0 = blockIdx.x * 4;
  const int rl = threadIdx.x >> 6, d = threadIdx.x & 63;
  const int fr = fr0 + rl;
  const bool live = fr < a.mrows;
  const float* src = nullptr;
  float x[kBatch];
  if (live) {
    const int mb = fr / a.cta_rows;
    src = a.ws_o + part_o(zc * a.mblocks + mb, fr - mb * a.cta_rows, a.cta_rows, a.splits, 0) + d;
#pragma unroll
    for (int u = 0; u < kBatch; ++u) x[u] = u < a.splits ? __ldcg(src + u * kDim) : 0.f;
  }
  if (warp < 4 && fr0 + warp < a.mrows) {
    const int wr = fr0 + warp;
    const int mb = wr / a.cta_rows;
    const float2* ml = a.ws_ml + part_ml(zc * a.mblocks + mb, wr - mb * a.cta_rows, a.cta_rows, a.splits, 0);
    const float den = merge_row_weights([&](int sp) { return ml[sp]; }, a.splits, s_w + warp * kTargetCtas, lane);
    if (lane == 0) s_den[warp] = den;
  }
  __syncthreads();
  if (!live) return;
  const float* w = s_w + rl * kTargetCtas;
  float acc = 0.f;
#pragma unroll
  for (int u = 0; u < kBatch; ++u)
    if (u < a.splits) acc = __fmaf_rn(w[u], x[u], acc);
  for (int sp = kBatch; sp < a.splits; sp += 16) {  // 16 loads in flight at a time
    float y[16];
    const int rem = a.splits - sp;
#pragma unroll
    for (int u = 0; u < 16; ++u) y[u] = u < rem ? __ldcg(src + (sp + u) * kDim) : 0.f;
#pragma unroll
    for (int u = 0; u < 16; ++u)
      if (u < rem) acc = __fmaf_rn(w[sp + u], y[u], acc);
  }
  const float val = __fdiv_rn(acc, s_den[rl]);
  const int m = fr / a.G;
  const int h = g * a.G + (fr - m * a.G);
  a.out[chunk * a.oc + (static_cast<int64_t>(m) * a.HQ + h) * kDim + d] =
      static_cast<uint16_t>(pack_bf16x2(val, 0.f) & 0xffffu);
}

}  // namespace

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
