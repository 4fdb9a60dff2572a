// Shared declarations of the packed-history attention kernels.
#pragma once

#include "dkv_common.cuh"

namespace dkv {

constexpr int kBN = 64;                 // keys per history tile
constexpr int kTcCtaRows = 256;         // stacked (query, head) rows per CTA (2 x M=128)
constexpr int kTargetCtas = 148;        // one wave on a B200 (148 SMs)
// D^-0.5 * log2(e): the reference scales scores by D^-0.5 (src/gpu_kernels.py:95)
// and uses exp; the kernels work in the exp2 domain with the factor folded in.
constexpr float kScaleLog2 = 0.125f * 1.4426950408889634f;
// Head of the workspace: per (KV head, row block) group an arrival and a departure
// counter for the in-kernel split merge. Zero before a workspace's first use; every
// call returns them to zero. A split plan never has more than 74 groups (>= 2 splits
// per group out of 148 CTAs), so 128 slots of each suffice.
constexpr int kSyncGroups = 128;
constexpr size_t kSyncBytes = 2 * kSyncGroups * sizeof(uint32_t);

// Work decomposition of one attention call. Deterministic in (past, nq, heads,
// group): no dependence on the device, so results are bit-identical across GPUs.
struct AttnPlan {
  int mrows;     // group * nq flattened rows per KV head (row r = query r/G, head r%G)
  int mblocks;   // row blocks per KV head
  int cta_rows;  // rows per block (kTcCtaRows)
  int splits;    // history splits per (head, row block)
  int chunk;     // keys per split, multiple of kBN
  size_t ws_o_bytes, ws_ml_bytes;
  size_t workspace_bytes() const { return splits > 1 ? kSyncBytes + ws_o_bytes + ws_ml_bytes : 0; }
};

// `chunks` independent query chunks share the history (batched calls): they act as
// chunks x heads groups of the same shape.
inline void size_workspace(AttnPlan& p, int heads) {
  p.ws_o_bytes = p.ws_ml_bytes = 0;
  if (p.splits > 1) {
    const size_t ctas = static_cast<size_t>(heads) * p.mblocks * p.splits;
    p.ws_o_bytes = ctas * p.cta_rows * kDim * sizeof(float);
    p.ws_ml_bytes = ctas * p.cta_rows * sizeof(float2) + sizeof(float2) * p.cta_rows * heads * p.mblocks;  // even split count
  }
}

inline AttnPlan make_plan(int past, int nq, int heads, int group, int chunks = 1) {
  heads *= chunks;
  AttnPlan p{};
  p.mrows = group * nq;
  p.cta_rows = kTcCtaRows;
  p.mblocks = (p.mrows + kTcCtaRows - 1) / kTcCtaRows;
  const int total = past + nq;
  const int tiles = (total + kBN - 1) / kBN;
  int target = kTargetCtas / (heads * p.mblocks);
  if (target < 1) target = 1;
  const int per_split = (tiles + target - 1) / target;  // tiles per split
  p.chunk = per_split * kBN;
  p.splits = (tiles + per_split - 1) / per_split;
  size_workspace(p, heads);
  return p;
}

// Short query chunks (at most kSplitRows stacked rows per KV head: decode steps,
// small candidate chunks) run on the split-K kernel: one CTA of four warps per
// (chunk, KV head, split), up to 16 splits per group forming one cluster, each
// split a multiple of 32 keys and at least one 32-key tile per warp, no more CTAs
// than two per SM. No workspace: the splits merge inside their cluster.
constexpr int kSplitRows = 16;
constexpr int kSplitKeys = 32;
inline AttnPlan make_plan_split(int past, int nq, int heads, int group, int chunks = 1) {
  AttnPlan p{};
  p.mrows = group * nq;
  p.cta_rows = kSplitRows;
  p.mblocks = 1;
  const int groups = heads * chunks;
  const int tiles = (past + nq + kSplitKeys - 1) / kSplitKeys;
  int s = (tiles + 3) / 4;
  if (s > 16) s = 16;
  const int cap = 2 * kTargetCtas / groups;
  if (s > cap) s = cap;
  if (s < 1) s = 1;
  const int per = (tiles + s - 1) / s;
  p.chunk = per * kSplitKeys;
  p.splits = (tiles + per - 1) / per;
  return p;  // no workspace
}

// Plan of a call over `count` independent requests whose histories are at most
// max_past tokens: as many splits as fill one wave (never more than the longest
// history has tiles), and each request divides its own history evenly among them
// (chunk = 0), so short and long histories of one batch finish together.
inline AttnPlan make_plan_many(int max_past, int nq, int heads, int group, int count) {
  AttnPlan p = make_plan(max_past, nq, heads, group, count);
  const int groups = heads * count * p.mblocks;
  const int tiles = (max_past + nq + kBN - 1) / kBN;
  int splits = kTargetCtas / groups;
  if (splits > tiles) splits = tiles;
  p.splits = splits < 1 ? 1 : splits;
  p.chunk = 0;
  size_workspace(p, heads * count);
  return p;
}

// One request's packed history (the C ABI's dkv_history): pools, (offset, scale)
// metadata, token maps rows / codes (pool row and precision of each logical
// token), history length, map length and device status word.
using History = dkv_history;

// Where query chunk c finds its history:
//  SharedHistory   every chunk reads AttnArgs::hist (one request; batched chunks)
//  HistoryTable    chunk c reads h[c], passed by value as a kernel parameter
//                  (3 KB: the launch itself carries the descriptors)
//  DeviceHistories chunk c reads h[c] from device memory, so a CUDA graph can be
//                  replayed with new histories written there between replays
constexpr int kMaxRequests = DKV_MAX_REQUESTS;
struct SharedHistory {};
struct HistoryTable {
  History h[kMaxRequests];
};
struct DeviceHistories {
  const History* h;
};

struct AttnArgs {
  const uint16_t* q;
  const uint16_t* knew;
  const uint16_t* vnew;
  History hist;   // the history of every chunk, unless a table is given
  uint16_t* out;
  int64_t qh, qt, kh, kt, vh, vt;
  int layer, nq, heads, G, HQ;  // heads: KV heads of one chunk
  int blocks;                   // layers * 2 * heads: the pools' blocks (page arithmetic, pool_row)
  int mrows, cta_rows, mblocks, splits;
  int chunk;  // keys per split; 0: each request splits its own history evenly (request_chunk)
  // Batched calls: blockIdx.z = chunk * heads + KV head; chunk c's q / knew / vnew /
  // out start qc / kc / vc / oc elements after chunk 0's (0 for a single chunk).
  int64_t qc, kc, vc, oc;
  float* ws_o;    // [heads * mblocks][cta_rows][splits][64] unnormalised partial outputs
  float2* ws_ml;  // [heads * mblocks][cta_rows][even(splits)] (running max in log2 units, sum)
  uint32_t* sync;  // [2][kSyncGroups] arrival / departure counters of the in-kernel merge
  int fused;       // 1: the attention kernel merges the splits itself (no combine launch)
  // 1: the launch just before this one on the stream may have written history rows
  // of this layer or the token maps, so the history is read only after
  // griddepcontrol.wait; 0: it is streamed while the previous kernel finishes.
  int hist_wait;
  // Fused pack of the call's new K/V rows into the pools (append + attend in one
  // launch; tensor-core kernel only): 0 none, 1 every chunk's frame into `pack`,
  // 2 chunk c's frame into pack_table[c] (device memory).
  int pack_mode;
  dkv_pack_target pack;
  const dkv_pack_target* pack_table;
};

__device__ __forceinline__ const dkv_pack_target* pack_of(const AttnArgs& a, int chunk) {
  return a.pack_mode == 1 ? &a.pack : (a.pack_mode == 2 ? a.pack_table + chunk : nullptr);
}

// The history query chunk c attends over.
__device__ __forceinline__ const History& history_of(const AttnArgs& a, const SharedHistory&, int) {
  return a.hist;
}
__device__ __forceinline__ const History& history_of(const AttnArgs&, const HistoryTable& t, int c) {
  return t.h[c];
}
__device__ __forceinline__ const History& history_of(const AttnArgs&, const DeviceHistories& t, int c) {
  return t.h[c];
}

// History length of a chunk, checked against its token map and pools (descriptors
// in device memory are not seen by the host): a bad one is reported and read as an
// empty history.
__device__ __forceinline__ int checked_past(const History& H, int chunk) {
  const int past = H.past;
  const bool pools = H.p4 != nullptr && H.m4 != nullptr && H.p8 != nullptr && H.m8 != nullptr && H.p16 != nullptr;
  if (past < 0 || past > H.capacity || (past > 0 && (H.rows == nullptr || H.codes == nullptr || !pools))) {
    report(H.status, DKV_EINVAL, chunk);
    return 0;
  }
  return past;
}

// Keys per split: the plan's, or (chunk == 0) this request's own history split
// evenly over the plan's splits.
__device__ __forceinline__ int request_chunk(const AttnArgs& a, int past) {
  if (a.chunk > 0) return a.chunk;
  const int tiles = (past + a.nq + kBN - 1) / kBN;
  return ((tiles + a.splits - 1) / a.splits) * kBN;
}

// Partials of group grp (= KV head * mblocks + row block): for each row, every
// split's 64 outputs side by side, so the splits of a run of rows are one
// contiguous block; the (max, sum) pairs likewise, with the split count rounded
// up to even so that a run of rows starts on a 16-byte boundary.
__host__ __device__ __forceinline__ int even_splits(int splits) { return splits + (splits & 1); }
__host__ __device__ __forceinline__ int64_t part_o(int grp, int row, int cta_rows, int splits, int sp) {
  return ((static_cast<int64_t>(grp) * cta_rows + row) * splits + sp) * kDim;
}
__host__ __device__ __forceinline__ int64_t part_ml(int grp, int row, int cta_rows, int splits, int sp) {
  return (static_cast<int64_t>(grp) * cta_rows + row) * even_splits(splits) + sp;
}

// Split merge of one (row, dim), shared by the in-kernel merge and the combine
// kernel so both give bit-identical results: M = max of the split maxima, weights
// w_s = 2^(m_s - M) (0 for an empty split), out = (sum_s w_s o_s) / (sum_s w_s l_s),
// both sums as fused multiply-adds in split order.
__device__ __forceinline__ float merge_weight(float m, float M) { return m == -INFINITY ? 0.f : exp2f(m - M); }

// One warp: the merge weights of one row. load(sp) returns split sp's (max, sum)
// of the row (called by lane sp % 32). Writes w_s to w[s] (shared memory) and
// returns, in every lane, the denominator sum_s w_s l_s: each lane sums its splits
// (lane, lane + 32, ...) with fused multiply-adds in split order, then the lanes'
// sums are added in a fixed butterfly (xor 16, 8, 4, 2, 1) -- the same order in
// every kernel that merges, so the results are bit-identical.
template <class Load>
__device__ __forceinline__ float merge_row_weights(Load load, int splits, float* w, int lane) {
  const float2 first = lane < splits ? load(lane) : make_float2(-INFINITY, 0.f);
  float M = first.x;
  for (int sp = lane + 32; sp < splits; sp += 32) M = fmaxf(M, load(sp).x);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
  float den = 0.f;
  for (int sp = lane; sp < splits; sp += 32) {
    const float2 v = sp == lane ? first : load(sp);
    const float wv = merge_weight(v.x, M);
    w[sp] = wv;
    den = __fmaf_rn(wv, v.y, den);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) den = __fadd_rn(den, __shfl_xor_sync(0xffffffffu, den, off));
  return den;
}

// `table` (may be null): per-chunk histories of a call over several requests.
// Per-chunk histories of a call over several requests: `table` (by value) or
// `device_table` (device memory); both null: every chunk reads a.hist.
// Sets a.fused when every CTA of the grid can be resident at once (one CTA per SM):
// the split merge then runs inside the kernel and no combine launch follows.
cudaError_t launch_attention_tc(AttnArgs& a, int heads, cudaStream_t stream, const HistoryTable* table = nullptr,
                                const History* device_table = nullptr);
// Whether a call with this plan merges its splits inside the tensor-core kernel
// on the current device (one launch) or needs the combine kernel (two);
// attend_only: one request, no fused pack, no history table.
cudaError_t attention_tc_merges_in_kernel(const AttnPlan& p, int heads, bool attend_only, bool* fused);
cudaError_t launch_attention_combine(const AttnArgs& a, int heads, cudaStream_t stream);
// The split-K kernel for plans of make_plan_split (a.hist holds the history).
cudaError_t launch_attention_split(const AttnArgs& a, int heads, cudaStream_t stream);

}  // namespace dkv
