// Shared declarations of the packed-history attention kernels.
#pragma once

#include "dkv_common.cuh"

namespace dkv {

constexpr int kBN = 64;                 // keys per history tile
constexpr int kMaxCtaRows = 192;        // flattened (query, head) rows per CTA, CUDA-core path
constexpr int kTcCtaRows = 256;         // rows per CTA on the tensor-core path (2 x M=128)
constexpr int kTcMinRows = 49;          // group*nq from which the tensor-core path is used
constexpr int kTargetCtas = 148;        // one wave on a B200 (148 SMs)
// D^-0.5 * log2(e): the reference scales scores by D^-0.5 (src/gpu_kernels.py:95)
// and uses exp; the kernels work in the exp2 domain with the factor folded in.
constexpr float kScaleLog2 = 0.125f * 1.4426950408889634f;

// Work decomposition of one attention call. Deterministic in (past, nq, heads,
// group): no dependence on the device, so results are bit-identical across GPUs.
struct AttnPlan {
  int tc;        // 1: tcgen05 tensor-core kernel, 0: mma.sync split kernel
  int mrows;     // group * nq flattened rows per KV head (row r = query r/G, head r%G)
  int mblocks;   // row blocks per KV head
  int cta_rows;  // rows per block (multiple of 16; 256 on the tensor-core path)
  int splits;    // history splits per (head, row block)
  int chunk;     // keys per split, multiple of kBN
  size_t ws_o_bytes, ws_ml_bytes;
};

inline AttnPlan make_plan(int past, int nq, int heads, int group) {
  AttnPlan p{};
  p.mrows = group * nq;
  p.tc = p.mrows >= kTcMinRows;
  if (p.tc) {
    p.cta_rows = kTcCtaRows;
    p.mblocks = (p.mrows + kTcCtaRows - 1) / kTcCtaRows;
  } else {
    p.mblocks = (p.mrows + kMaxCtaRows - 1) / kMaxCtaRows;
    const int per_block = (p.mrows + p.mblocks - 1) / p.mblocks;
    p.cta_rows = ((per_block + 15) / 16) * 16;
  }
  const int total = past + nq;
  const int tiles = (total + kBN - 1) / kBN;
  int target = kTargetCtas / (heads * p.mblocks);
  if (target < 1) target = 1;
  const int per_split = (tiles + target - 1) / target;  // tiles per split
  p.chunk = per_split * kBN;
  p.splits = (tiles + per_split - 1) / per_split;
  if (p.splits > 1) {
    const size_t ctas = static_cast<size_t>(heads) * p.mblocks * p.splits;
    p.ws_o_bytes = ctas * p.cta_rows * kDim * sizeof(float);
    p.ws_ml_bytes = ctas * p.cta_rows * sizeof(float2);
  }
  return p;
}

struct AttnArgs {
  const uint16_t* q;
  const uint16_t* knew;
  const uint16_t* vnew;
  Pools P;
  const int32_t* rows;
  const uint8_t* codes;
  uint16_t* out;
  int64_t qh, qt, kh, kt, vh, vt;
  int layer, past, nq, G, HQ;
  int mrows, cta_rows, mblocks, splits, chunk;
  float* ws_o;    // [heads][mblocks][splits][cta_rows][64] unnormalised partial outputs
  float2* ws_ml;  // [heads][mblocks][splits][cta_rows] (running max in log2 units, sum)
  int32_t* status;
};

cudaError_t launch_attention_split(const AttnArgs& a, int heads, cudaStream_t stream);
cudaError_t launch_attention_tc(const AttnArgs& a, int heads, cudaStream_t stream);
cudaError_t launch_attention_combine(const AttnArgs& a, int heads, cudaStream_t stream);

}  // namespace dkv
