// Tensor-core (tcgen05 + TMEM) causal GQA attention over packed mixed-precision
// history, sm_100a: every attention call, from a one-token decode step (3 stacked
// rows, padded into the M=128 tile) to frames and candidate chunks of two row
// blocks per KV head.
//
// Semantics are those of the reference kernel packed_attention
// (src/gpu_kernels.py:71-105): dequantised history rounded to bf16 (:93-94), the
// current chunk's native K/V, q.k * D^-0.5 (:95), bottom-right causal mask (:96),
// online softmax (:98-103), p rounded to bf16 before P.V (:102), fp32 accumulation.
//
// One CTA per (KV head, block of up to 256 stacked rows, history split), 16 warps
// in five roles, connected only by mbarriers (warp w runs on sub-partition w % 4):
//   warps 12-13 loaders (even / odd tiles): token maps of tile i+6 arrive by TMA
//               bulk copy; for tile i+4 the warp splits the 64 tokens into runs of
//               consecutive pool rows of one precision and streams each run (codes,
//               and the offset/scale pairs) into a 4-deep raw ring with one TMA bulk
//               copy per run;
//   warps 10, 11, 14, 15 converters: dequantise a raw tile in registers into bf16
//               K and V tiles (64 keys) of a 3-stage ring, 128B-swizzled for the
//               tensor core;
//   warp 8      S issuer (one thread): S = Q K^T into TMEM, double-buffered, with Q
//               held in TMEM; an S buffer is reused as soon as the softmax has read it;
//   warp 9      PV issuer (one thread): O += P V into TMEM with P read from TMEM;
//   warps 0-7   softmax: one TMEM lane = one stacked row each; read S, mask, online
//               max and exp2 in fp32, the row sum of p in fp32 registers, write P
//               (bf16 pairs) into TMEM once the previous P V product has landed, and
//               rescale O in TMEM when the running max moves.
// Both products read their A operand from tensor memory: shared memory carries
// only the K and V tiles (2 KB per MMA), so the tensor core is not held up by the
// converters' and TMA's shared-memory traffic.
// The running max is only moved when a tile's max exceeds it by more than 2^8
// (p <= 256, exact after the final O / l division). Partial (max, sum, O) per
// split go to the workspace. Every mbarrier wait is bounded: a stalled pipeline
// reports DKV_ETIMEOUT in the status word and the CTA exits after its MMAs drain
// and TMEM is freed.
//
// Fused append + attend and batched calls whose whole grid is resident at once
// (one CTA per SM, at most 148 CTAs) merge the splits in the same launch: each CTA
// publishes its partial, counts itself in on its group's arrival counter and, once
// all splits of the group are in, merges an equal slice of the group's rows from
// every split's partial. The wait is bounded; the last CTA to leave resets the
// counters for the next call. Single-request attend-only calls (where an eager
// cooperative launch costs more than a second launch), grids that do not fit, and
// every call under DKV_ATTENTION_MERGE=combine leave the merge to the combine
// kernel, which does the same arithmetic.
// A call that appends (append + attend in one launch) also packs the new rows:
// the CTAs of a (chunk, KV head) share them, each packing its share while it
// waits for its group.
// A query chunk's history comes from the call itself, from a by-value table of
// requests in the kernel parameters, or from a table in device memory (graph
// replay): three instantiations of the same kernel.
#include <cstdlib>
#include <cstring>

#include "attention.cuh"
#include "pack_row.cuh"
#include "tc_ptx.cuh"

namespace dkv {
namespace {

using namespace ptx;

constexpr int kStages = 3;     // bf16 operand ring (K and V tiles)
constexpr int kRawStages = 4;  // packed-bytes ring filled by TMA
constexpr int kMapStages = 6;  // token-map ring filled by TMA
constexpr int kSoftmaxWarps = 8;
constexpr int kSWarp = 8;
constexpr int kPVWarp = 9;
// Warp w runs on SM sub-partition w % 4, and the softmax warp of TMEM lanes
// 32q..32q+31 must sit on sub-partition q. At the usual 192 stacked rows (3 query
// heads x 64 queries) both row tiles have rows on sub-partitions 0 and 1 but only
// the first on 2 and 3, so the four converter warps (the heaviest other role) sit
// on 2 and 3 (warps 10, 11, 14, 15) and the two loader warps on 0 and 1 (12, 13).
constexpr int kLoadWarps = 2;   // even / odd tiles
constexpr int kConvWarps = 4;
constexpr int kThreadsTc = 16 * 32;  // 512
constexpr int kConvThreads = kConvWarps * 32;
__device__ __forceinline__ bool is_load_warp(int w) { return w == 12 || w == 13; }
__device__ __forceinline__ int load_index(int w) { return w - 12; }
__device__ __forceinline__ bool is_conv_warp(int w) { return w == 10 || w == 11 || w == 14 || w == 15; }
__device__ __forceinline__ int conv_index(int w) { return w - 10 - (w >= 14 ? 2 : 0); }
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0;    // S[buf][mt] at columns (buf * 2 + mt) * 64
constexpr uint32_t kColO = 256;  // O[mt] (64 fp32) at columns 256 + mt * 64
constexpr uint32_t kColP = 384;  // P[mt] (64 bf16 = 32 columns) at 384 + mt * 32
constexpr uint32_t kColQ = 448;  // Q[mt] (64 bf16 = 32 columns) at 448 + mt * 32

constexpr int kTile = kBN * 128;  // one 64-key bf16 tile, 8 KB
// Raw stage: K rows, V rows (a run starting at token j0 is packed densely from
// byte j0 * 128), K/V (offset, scale) pairs (a run's pairs from byte j0 * 16,
// shifted by one pair when its first pair sits at an odd pool index), and one
// 64-bit entry per token: {code | raw offset << 8, K meta offset | V meta offset << 16}.
constexpr int kRawK = 0;
constexpr int kRawV = kTile;
constexpr int kRawMetaK = 2 * kTile;
constexpr int kRawMetaV = kRawMetaK + kBN * 16;
constexpr int kRawTab = kRawMetaV + kBN * 16;
// Header word: the tile's code when all 64 tokens form one pool run (else 0),
// bit 8 / bit 9 = K / V pairs shifted by one (odd first pair index).
constexpr int kRawHdr = kRawTab + kBN * 8;
constexpr int kRawStage = kRawHdr + 16;
// Map stage: codes (64 B) then rows (256 B) of one tile.
constexpr int kMapStage = kBN + kBN * 4;

constexpr int kOffQ = 0;  // 2 M-tiles x 128 rows x 128 B
constexpr int kOffP = kOffQ + 2 * 128 * 128;
constexpr int kOffK = kOffP + 2 * 128 * 128;
constexpr int kOffV = kOffK + kStages * kTile;
constexpr int kOffRaw = kOffV + kStages * kTile;
constexpr int kOffMap = kOffRaw + kRawStages * kRawStage;
constexpr int kOffBar = ((kOffMap + kMapStages * kMapStage + 15) / 16) * 16;
enum {
  B_FULL = 0,                           // operand stage ready    (converters, 128)
  B_EMPTY = B_FULL + kStages,           // operand stage free     (PV commit)
  B_RAWFULL = B_EMPTY + kStages,        // raw stage landed       (loader + TMA bytes)
  B_RAWEMPTY = B_RAWFULL + kRawStages,  // raw stage consumed     (converters, 128)
  B_MAPFULL = B_RAWEMPTY + kRawStages,  // map stage landed       (loader + TMA bytes)
  // Per M-tile barriers: the two row tiles run their S -> softmax -> P V chains
  // independently, so one tile's softmax hides the other's barrier and MMA latency.
  B_SFULL = B_MAPFULL + kMapStages,    // S[b][mt] computed        (S commit),  index b * 2 + mt
  B_SFREE = B_SFULL + 4,                // S[b][mt] read            (mt's softmax threads)
  B_PFULL = B_SFREE + 4,                // P[mt] written            (mt's softmax threads)
  B_ODONE = B_PFULL + 2,                // O[mt] updated, P[mt] read (PV commit)
  B_QREADY = B_ODONE + 2,
  B_FINS = B_QREADY + 1,
  B_FINPV = B_FINS + 1,
  B_MERGE = B_FINPV + 1,                // split partials landed   (merge, TMA bytes)
  B_COUNT = B_MERGE + 1
};
constexpr int kOffTmem = kOffBar + B_COUNT * 8;
constexpr int kOffAbort = kOffTmem + 4;
constexpr int kSmemTc = kOffAbort + 4 + 1024;  // + slack to align the base to 1024 B
static_assert(kSmemTc <= 227 * 1024, "shared memory budget");
constexpr long long kWaitCycles = 400000000LL;  // ~0.2 s: a healthy wait is microseconds

constexpr int kMergePairs = kTcCtaRows + kTargetCtas;  // (split, row) pairs one CTA merges, at most
static_assert(kMergePairs * kDim * 4 <= kOffBar - kOffK, "merge staging fits the operand and raw rings");
// (row, split) pairs staged: at most kMergePairs + kTcCtaRows with the split count rounded up to even
static_assert((kMergePairs + kTcCtaRows) * 8 + 2 * kMergePairs * 4 + kTcCtaRows * 4 <= 2 * 128 * 128,
              "merge (max, sum) pairs, weights and denominators fit the Q region");

constexpr uint32_t kIdescS = idesc_bf16(128, kBN, 0);    // S = Q K^T: B = K tile, K-major
constexpr uint32_t kIdescPV = idesc_bf16(128, kDim, 1);  // O += P V: B (the V tile) MN-major

constexpr int kCodeNew = 17;  // token of the current chunk: native row of knew / vnew

__device__ __forceinline__ int swz(int row, int chunk) { return row * 128 + ((chunk ^ (row & 7)) << 4); }

__device__ __forceinline__ int row_bytes(int code) { return code == 4 ? 32 : (code == 8 ? 64 : 128); }

// 32-bit x -> 64-bit with bit i moved to bit 2i.
__device__ __forceinline__ uint64_t spread_bits(uint32_t x) {
  uint64_t v = x;
  v = (v | (v << 16)) & 0x0000FFFF0000FFFFull;
  v = (v | (v << 8)) & 0x00FF00FF00FF00FFull;
  v = (v | (v << 4)) & 0x0F0F0F0F0F0F0F0Full;
  v = (v | (v << 2)) & 0x3333333333333333ull;
  v = (v | (v << 1)) & 0x5555555555555555ull;
  return v;
}

// 8 codes (bytes b0 = elements 0..3 and b1 = 4..7 for 8-bit; nibbles of w for
// 4-bit) -> 8 bf16 of code * scale + offset, one packed FMA per pair. Codes become
// exact floats as 2^23 + code minus 2^23.
template <int BITS>
__device__ __forceinline__ uint4 dequant_fast(uint32_t w0, uint32_t w1, float offset, float scale) {
  uint32_t b0, b1;
  if (BITS == 8) {
    b0 = w0;
    b1 = w1;
  } else {
    b0 = w0 & 0x0F0F0F0Fu;         // byte j = element 2j
    b1 = (w0 >> 4) & 0x0F0F0F0Fu;  // byte j = element 2j + 1
  }
  const float2 sc = make_float2(scale, scale);
  const float2 of = make_float2(offset, offset);
  const float2 mag = make_float2(-8388608.f, -8388608.f);
  uint32_t out[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    uint32_t lo, hi;
    if (BITS == 8) {
      const uint32_t w = e < 2 ? b0 : b1;
      lo = __byte_perm(w, 0x4B000000u, 0x7540 | (2 * (e & 1)));
      hi = __byte_perm(w, 0x4B000000u, 0x7540 | (2 * (e & 1) + 1));
    } else {
      lo = __byte_perm(b0, 0x4B000000u, 0x7540 | e);
      hi = __byte_perm(b1, 0x4B000000u, 0x7540 | e);
    }
    const float2 qf = add2(make_float2(__uint_as_float(lo), __uint_as_float(hi)), mag);
    const float2 x = fma2(qf, sc, of);
    out[e] = pack_bf16x2(x.x, x.y);
  }
  return make_uint4(out[0], out[1], out[2], out[3]);
}

// Whole tile of one precision, rows packed densely from token 0: every load of
// this thread's 8 parts is issued before any conversion, no per-token branches.
template <int BITS>
__device__ __forceinline__ void convert_uniform(const uint8_t* st, uint8_t* dstK, uint8_t* dstV, int jb, int c,
                                                uint32_t hdr) {
  constexpr int rb = BITS == 4 ? 32 : (BITS == 8 ? 64 : 128);
  const int park = (hdr >> 8) & 1, parv = (hdr >> 9) & 1;
  uint4 raw[8];
  float2 mt[8];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int j = jb + 16 * k;
#pragma unroll
    for (int kv = 0; kv < 2; ++kv) {
      const uint8_t* rrow = st + (kv ? kRawV : kRawK) + j * rb;
      const int q = 2 * k + kv;
      if (BITS == 16) {
        raw[q] = *reinterpret_cast<const uint4*>(rrow + c * 16);
      } else {
        if (BITS == 8) {
          const uint2 w = *reinterpret_cast<const uint2*>(rrow + c * 8);
          raw[q] = make_uint4(w.x, w.y, 0, 0);
        } else {
          raw[q] = make_uint4(*reinterpret_cast<const uint32_t*>(rrow + c * 4), 0, 0, 0);
        }
        mt[q] = *reinterpret_cast<const float2*>(st + (kv ? kRawMetaV : kRawMetaK) + ((kv ? parv : park) + j) * 8);
      }
    }
  }
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int j = jb + 16 * k;
#pragma unroll
    for (int kv = 0; kv < 2; ++kv) {
      const int q = 2 * k + kv;
      const uint4 v = BITS == 16 ? raw[q] : dequant_fast<BITS>(raw[q].x, raw[q].y, mt[q].x, mt[q].y);
      *reinterpret_cast<uint4*>((kv ? dstV : dstK) + swz(j, c)) = v;
    }
  }
}

// Few rows per CTA (one (row, dim) per thread, as with many splits): each thread
// loads its column of every split's partial straight into registers before the
// weights are computed, so the partials' and the (max, sum) pairs' trips to L2
// overlap; same arithmetic in the same order as merge_rows.
constexpr int kMergeRegs = 32;
__device__ __forceinline__ void merge_rows_direct(const AttnArgs& a, int g, int grp, int row0, int r_begin, int nr,
                                                  uint16_t* out, uint8_t* smem, int tid) {
  const int S = a.splits;
  float* s_w = reinterpret_cast<float*>(smem + kOffQ) + 2 * (kMergePairs + kTcCtaRows);  // [nr][S]
  float* s_den = s_w + kMergePairs;                                                       // [nr]
  const int warp = tid >> 5, lane = tid & 31;
  const bool mine = tid < nr * kDim;
  const int r = tid >> 6, d = tid & (kDim - 1);
  float ov[kMergeRegs];
  if (mine) {  // partials published by the other splits: plain loads after the acquire
    const float* col = a.ws_o + part_o(grp, r_begin + r, kTcCtaRows, S, 0) + d;
#pragma unroll
    for (int u = 0; u < kMergeRegs; ++u) ov[u] = u < S ? col[u * kDim] : 0.f;
  }
  for (int rr = warp; rr < nr; rr += kThreadsTc / 32) {
    const float2* ml = a.ws_ml + part_ml(grp, r_begin + rr, kTcCtaRows, S, 0);
    const float den = merge_row_weights([&](int sp) { return ml[sp]; }, S, s_w + rr * S, lane);
    if (lane == 0) s_den[rr] = den;
  }
  __syncthreads();
  if (mine) {
    const float* w = s_w + r * S;
    float acc = 0.f;
#pragma unroll
    for (int u = 0; u < kMergeRegs; ++u)
      if (u < S) acc = __fmaf_rn(w[u], ov[u], acc);
    const float val = __fdiv_rn(acc, s_den[r]);
    const int frow = row0 + r_begin + r;
    const int m = frow / a.G;
    const int h = g * a.G + (frow - m * a.G);
    out[(static_cast<int64_t>(m) * a.HQ + h) * kDim + d] = static_cast<uint16_t>(pack_bf16x2(val, 0.f) & 0xffffu);
  }
}

// Rows [r_begin, r_end) of group grp (rows counted from row0), merged from all
// splits' partials and written to `out` (merge_row_weights, then the fused
// multiply-add chain in split order: bit-identical to the combine kernel). The
// rows' partials of every split and their (max, sum) pairs are two contiguous
// blocks (part_o / part_ml layout): two TMA bulk copies bring them into the idle
// operand rings; then a warp per row finds the weights and one thread per
// (row, dim) sums its column from shared memory.
__device__ __forceinline__ void merge_rows(const AttnArgs& a, int g, int grp, int row0, int r_begin, int r_end,
                                           uint16_t* out, uint8_t* smem, int tid, int32_t* status) {
  const int nr = r_end - r_begin;
  if (nr <= 0) return;
  if (nr * kDim <= kThreadsTc && a.splits <= kMergeRegs) {
    merge_rows_direct(a, g, grp, row0, r_begin, nr, out, smem, tid);
    return;
  }
  const uint32_t sbase = smem_addr(smem);
  const uint32_t mbar = sbase + kOffBar + 8 * B_MERGE;
  const int S = a.splits, Se = even_splits(S);
  const uint32_t o_bytes = static_cast<uint32_t>(nr * S) * kDim * 4;
  const uint32_t ml_bytes = static_cast<uint32_t>(nr * Se) * 8;
  const float* s_o = reinterpret_cast<const float*>(smem + kOffK);                // [nr][S][64]
  const float2* s_ml = reinterpret_cast<const float2*>(smem + kOffQ);             // [nr][Se]
  float* s_w = reinterpret_cast<float*>(smem + kOffQ) + 2 * (kMergePairs + kTcCtaRows);  // [nr][S]
  float* s_den = s_w + kMergePairs;                                                       // [nr]
  const int warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    fence_proxy_async_global();  // partials stored through the generic proxy, read by TMA
    fence_proxy_async_smem();    // the rings were last read by generic loads
    mbar_expect_tx(mbar, o_bytes + ml_bytes);
    bulk_g2s(sbase + kOffK, a.ws_o + part_o(grp, r_begin, kTcCtaRows, S, 0), o_bytes, mbar);
    bulk_g2s(sbase + kOffQ, a.ws_ml + part_ml(grp, r_begin, kTcCtaRows, S, 0), ml_bytes, mbar);
    mbar_arrive(mbar);
  }
  if (!mbar_wait(mbar, 0, kWaitCycles)) {
    report(status, DKV_ETIMEOUT, 7);
    mbar_wait(mbar, 0, kWaitCycles);  // the copies still target this CTA's shared memory
    return;
  }
  for (int r = warp; r < nr; r += kThreadsTc / 32) {
    const float2* ml = s_ml + r * Se;
    const float den = merge_row_weights([&](int sp) { return ml[sp]; }, S, s_w + r * S, lane);
    if (lane == 0) s_den[r] = den;
  }
  __syncthreads();
  for (int i = tid; i < nr * kDim; i += kThreadsTc) {
    const int r = i >> 6, d = i & (kDim - 1);
    const float* col = s_o + r * S * kDim + d;
    const float* w = s_w + r * S;
    float acc = 0.f;
    int sp = 0;
    for (; sp + 8 <= S; sp += 8) {  // whole batches: every load issued before the chain
      float wv[8], ov[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        wv[u] = w[sp + u];
        ov[u] = col[(sp + u) * kDim];
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) acc = __fmaf_rn(wv[u], ov[u], acc);
    }
    for (; sp < S; ++sp) acc = __fmaf_rn(w[sp], col[sp * kDim], acc);
    const float val = __fdiv_rn(acc, s_den[r]);
    const int frow = row0 + r_begin + r;
    const int m = frow / a.G;
    const int h = g * a.G + (frow - m * a.G);
    out[(static_cast<int64_t>(m) * a.HQ + h) * kDim + d] = static_cast<uint16_t>(pack_bf16x2(val, 0.f) & 0xffffu);
  }
}

// Hist: SharedHistory (every chunk reads a.hist), HistoryTable (chunk c reads its
// own request's history from the kernel parameters) or DeviceHistories (from
// device memory).
template <class Hist>
__global__ void __launch_bounds__(kThreadsTc, 1)
attention_tc_kernel(const __grid_constant__ AttnArgs a, const __grid_constant__ Hist hist) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_addr(smem);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kOffAbort);

  const int split = blockIdx.x;
  const int mb = blockIdx.y;
  const int zc = blockIdx.z;                  // chunk * heads + KV head
  const int chunk = zc / a.heads;
  const int g = zc - chunk * a.heads;
  const History& H = history_of(a, hist, chunk);
  const int past = checked_past(H, chunk);
  int32_t* const status = H.status;
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;

  const int row0 = mb * kTcCtaRows;
  const int rows_here = min(kTcCtaRows, a.mrows - row0);
  const int mt_count = (rows_here + 127) >> 7;
  const int m_max = (row0 + rows_here - 1) / a.G;
  const int keys = request_chunk(a, past);
  const int kb = split * keys;
  int ke = min(kb + keys, past + a.nq);
  ke = min(ke, past + m_max + 1);  // no row of this block sees further
  const int ntiles = ke > kb ? (ke - kb + kBN - 1) / kBN : 0;
  const int soft_threads = ((rows_here + 31) >> 5) << 5;  // threads of softmax warps with real rows

  auto bar = [&](int i) { return sbase + kOffBar + 8 * i; };

  // ---- set-up: barriers and TMEM, then every role starts at once ----
  if (warp == 0) {  // each lane initialises a share of the barriers
    const int tile_threads[2] = {min(soft_threads, 128), max(soft_threads - 128, 32)};  // (unused tile: any count)
    for (int idx = lane; idx < B_COUNT; idx += 32) {
      uint32_t cnt = 1;  // single-arrival barriers: MMA commits, TMA completions, loader arrivals
      if ((idx >= B_FULL && idx < B_FULL + kStages) || (idx >= B_RAWEMPTY && idx < B_RAWEMPTY + kRawStages)) {
        cnt = kConvThreads;
      } else if (idx >= B_SFREE && idx < B_SFREE + 4) {
        cnt = tile_threads[(idx - B_SFREE) & 1];
      } else if (idx >= B_PFULL && idx < B_PFULL + 2) {
        cnt = tile_threads[idx - B_PFULL];
      } else if (idx == B_QREADY) {
        cnt = kSoftmaxWarps * 32;
      }
      mbar_init(bar(idx), cnt);
    }
    if (lane == 0) *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  if (warp == kSWarp) {
    tmem_alloc(sbase + kOffTmem, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(smem + kOffTmem);

  if (warp == kSWarp) {
    // ================= S = Q K^T issuer =================
    if (lane == 0 && ntiles > 0) {
      bool ok = mbar_wait(bar(B_QREADY), 0, kWaitCycles);
      for (int i = 0; i < ntiles && ok; ++i) {
        const int s = i % kStages, b = i & 1;
        ok = mbar_wait(bar(B_FULL + s), (i / kStages) & 1, kWaitCycles);
        for (int mt = 0; mt < mt_count && ok; ++mt) {
          if (i >= 2) ok = mbar_wait(bar(B_SFREE + b * 2 + mt), ((i >> 1) + 1) & 1, kWaitCycles);
          if (!ok) break;
          tc_fence_after();
          const uint32_t d = tmem + kColS + (b * 2 + mt) * 64;
#pragma unroll
          for (int k = 0; k < 4; ++k) {  // 16 dims per step = 8 TMEM columns of Q
            const uint64_t bd = sw128_desc(sbase + kOffK + s * kTile + k * 32, 16, 1024);
            umma_f16_ts(d, tmem + kColQ + mt * 32 + k * 8, bd, kIdescS, k > 0);
          }
          umma_commit(bar(B_SFULL + b * 2 + mt));
        }
      }
      if (!ok) {
        *abort_flag = 1;
        report(status, DKV_ETIMEOUT, 1);
      }
      umma_commit(bar(B_FINS));  // drain this thread's MMAs before TMEM is released
      mbar_wait(bar(B_FINS), 0, kWaitCycles);
    }
    __syncwarp();
  } else if (warp == kPVWarp) {
    // ================= O += P V issuer =================
    if (lane == 0 && ntiles > 0) {
      bool ok = true;
      for (int i = 0; i < ntiles && ok; ++i) {
        const int s = i % kStages;
        for (int mt = 0; mt < mt_count && ok; ++mt) {
          ok = mbar_wait(bar(B_PFULL + mt), i & 1, kWaitCycles);
          if (!ok) break;
          tc_fence_after();
          const uint32_t d = tmem + kColO + mt * 64;
#pragma unroll
          for (int k = 0; k < 4; ++k) {  // 16 keys per step = 8 TMEM columns of P
            const uint64_t bd = sw128_desc(sbase + kOffV + s * kTile + k * 2048, kTile, 1024);
            umma_f16_ts(d, tmem + kColP + mt * 32 + k * 8, bd, kIdescPV, (i > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit(bar(B_ODONE + mt));
        }
        if (ok) umma_commit(bar(B_EMPTY + s));  // both tiles' products have read V (and S read K)
      }
      if (!ok) {
        *abort_flag = 1;
        report(status, DKV_ETIMEOUT, 2);
      }
      umma_commit(bar(B_FINPV));
      mbar_wait(bar(B_FINPV), 0, kWaitCycles);
    }
    __syncwarp();
  } else if (is_load_warp(warp)) {
    // ================= loader: token maps and packed runs by TMA =================
    // The pools are paged (pool_row): the rows of a page of one block are
    // contiguous, so a run of consecutive rows that stays inside one 64-row page
    // is one copy; runs are cut at page boundaries below.
    const int64_t blk_k = (static_cast<int64_t>(a.layer) * 2) * a.heads + g;  // (layer, K, head)
    const int64_t blk_v = blk_k + a.heads;                                    // (layer, V, head)
    const int64_t nblk = a.blocks;
    const int cap4 = static_cast<int>(H.cap4), cap8 = static_cast<int>(H.cap8);
    const int cap16 = static_cast<int>(H.cap16);
    const uint8_t* const p4 = static_cast<const uint8_t*>(H.p4);
    const uint8_t* const p8 = static_cast<const uint8_t*>(H.p8);
    const uint8_t* const p16 = static_cast<const uint8_t*>(H.p16);
    const float2* const m4 = static_cast<const float2*>(H.m4);
    const float2* const m8 = static_cast<const float2*>(H.m8);
    const int32_t* const map_rows = H.rows;
    const uint8_t* const map_codes = H.codes;
    // pool row index of row r of this head's K (kv = 0) or V block
    auto row_at = [&](int kv, int r) -> int64_t { return pool_row(kv ? blk_v : blk_k, r, nblk); };
    // selectors (no dynamic array indexing: keeps everything in registers)
    auto pool_of = [&](int code) -> const uint8_t* { return code == 4 ? p4 : (code == 8 ? p8 : p16); };
    auto meta_of = [&](int code) -> const float2* { return code == 4 ? m4 : m8; };
    const uint16_t* const knew_g = a.knew + chunk * a.kc + g * a.kh;
    const uint16_t* const vnew_g = a.vnew + chunk * a.vc + g * a.vh;

    auto map_tile = [&](int tile) {  // lane 0: start the map copy of a full history tile
      const int t0 = kb + tile * kBN;
      const int slot = tile % kMapStages;
      if (t0 + kBN <= past) {
        mbar_expect_tx(bar(B_MAPFULL + slot), kMapStage);
        bulk_g2s(sbase + kOffMap + slot * kMapStage, map_codes + t0, kBN, bar(B_MAPFULL + slot));
        bulk_g2s(sbase + kOffMap + slot * kMapStage + kBN, map_rows + t0, kBN * 4, bar(B_MAPFULL + slot));
      }
      mbar_arrive(bar(B_MAPFULL + slot));
    };
    // (offset, scale) pairs of a run of `cnt` rows from block-relative row r0 for
    // K (kv = 0) or V, the run inside one page: one 16-byte aligned bulk copy of
    // the even-aligned span around it (a page starts at an even pair index and
    // holds an even number of rows, so the span stays inside the page) when the
    // run holds >= 2 rows; returns the pair shift (0/1), or -1 for "caller stores
    // the pairs with plain loads".
    auto meta_run = [&](int code, int kv, int r0, int cnt, uint32_t dst, uint32_t rbar) -> int {
      if (cnt < 2) return -1;
      const int par = r0 & 1;
      const int end = r0 + cnt;
      const int hi = end + (end & 1);
      const uint32_t bytes = static_cast<uint32_t>(hi - (r0 - par)) * 8u;
      mbar_expect_tx(rbar, bytes);
      bulk_g2s(dst, meta_of(code) + row_at(kv, r0 - par), bytes, rbar);
      return par;
    };

    const int lw = load_index(warp);  // this warp's tiles: lw, lw + 2, ...
    if (a.hist_wait) pdl_wait();      // the previous launch may have written history rows or maps
    if (lane == 0) {
      for (int t = lw; t < kMapStages && t < ntiles; t += kLoadWarps) map_tile(t);
    }
    __syncwarp();
    bool ok = true;
    for (int i = lw; i < ntiles; i += kLoadWarps) {
      const int rs = i % kRawStages;
      const int slot = i % kMapStages;
      if (i >= kRawStages) ok = mbar_wait(bar(B_RAWEMPTY + rs), ((i / kRawStages) + 1) & 1, kWaitCycles);
      ok = ok && mbar_wait(bar(B_MAPFULL + slot), (i / kMapStages) & 1, kWaitCycles);
      if (!__all_sync(0xffffffffu, ok) || __any_sync(0xffffffffu, *abort_flag != 0)) {
        ok = false;
        break;
      }
      fence_proxy_async_smem();  // converters' reads of this raw stage precede the TMA writes
      const int t0 = kb + i * kBN;
      if (t0 + kBN > past) pdl_wait();  // current-chunk K/V come from the previous kernels
      const uint8_t* mcodes = smem + kOffMap + slot * kMapStage;
      const int32_t* mrows = reinterpret_cast<const int32_t*>(mcodes + kBN);
      const bool full_map = t0 + kBN <= past;
      // --- classify this lane's two tokens j = 2 lane + e ---
      int code[2], row[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int j = 2 * lane + e;
        const int t = t0 + j;
        if (t >= ke) {
          code[e] = 0;
          row[e] = 0;
        } else if (t >= past) {
          code[e] = kCodeNew;
          row[e] = t - past;
        } else {
          if (full_map) {
            code[e] = mcodes[j];
            row[e] = mrows[j];
          } else {  // the tile holding `past`: its map was not prefetched
            code[e] = __ldg(map_codes + t);
            row[e] = __ldg(map_rows + t);
          }
          const int cap = code[e] == 4 ? cap4 : (code[e] == 8 ? cap8 : cap16);
          if (code[e] != 4 && code[e] != 8 && code[e] != 16) {
            report(status, DKV_EPLAN, t);
            code[e] = 0;
          } else if (row[e] < 0 || row[e] >= cap) {
            report(status, DKV_ECAPACITY, t);
            code[e] = 0;
          }
        }
      }
      // --- runs: a token starts one unless it continues the previous token's pool
      // run inside the same page (the first row of a page always starts a run) ---
      const int pcode = __shfl_up_sync(0xffffffffu, code[1], 1);
      const int prow = __shfl_up_sync(0xffffffffu, row[1], 1);
      const bool pooled0 = code[0] == 4 || code[0] == 8 || code[0] == 16;
      const bool pooled1 = code[1] == 4 || code[1] == 8 || code[1] == 16;
      const bool start0 =
          lane == 0 || !pooled0 || pcode != code[0] || prow + 1 != row[0] || (row[0] & (kPageRows - 1)) == 0;
      const bool start1 =
          !pooled1 || code[0] != code[1] || row[0] + 1 != row[1] || (row[1] & (kPageRows - 1)) == 0;
      const uint32_t even_starts = __ballot_sync(0xffffffffu, start0);
      const uint32_t odd_starts = __ballot_sync(0xffffffffu, start1);
      const int code0 = __shfl_sync(0xffffffffu, code[0], 0);
      uint8_t* st = smem + kOffRaw + rs * kRawStage;
      const uint32_t sst = sbase + kOffRaw + rs * kRawStage;
      const uint32_t rbar = bar(B_RAWFULL + rs);
      if (even_starts == 1u && odd_starts == 0u && (code0 == 4 || code0 == 8 || code0 == 16)) {
        // ---- uniform tile: one run of 64 rows (one whole page), copies from lane 0,
        // no per-token table ----
        const int rb = row_bytes(code0);
        const int r0 = __shfl_sync(0xffffffffu, row[0], 0);
        int park = 0, parv = 0;
        if (lane == 0) {
          mbar_expect_tx(rbar, 2 * kBN * rb);
          bulk_g2s(sst + kRawK, pool_of(code0) + row_at(0, r0) * rb, kBN * rb, rbar);
          bulk_g2s(sst + kRawV, pool_of(code0) + row_at(1, r0) * rb, kBN * rb, rbar);
          if (code0 != 16) {
            park = meta_run(code0, 0, r0, kBN, sst + kRawMetaK, rbar);
            parv = meta_run(code0, 1, r0, kBN, sst + kRawMetaV, rbar);
          }
        }
        park = __shfl_sync(0xffffffffu, park, 0);
        parv = __shfl_sync(0xffffffffu, parv, 0);
        if (code0 != 16 && (park < 0 || parv < 0)) {  // no bulk copy of the pairs: plain loads
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int j = 2 * lane + e;
            if (park < 0) *reinterpret_cast<float2*>(st + kRawMetaK + j * 8) = __ldg(meta_of(code0) + row_at(0, r0 + j));
            if (parv < 0) *reinterpret_cast<float2*>(st + kRawMetaV + j * 8) = __ldg(meta_of(code0) + row_at(1, r0 + j));
          }
          park = max(park, 0);
          parv = max(parv, 0);
        }
        if (lane == 0) *reinterpret_cast<uint32_t*>(st + kRawHdr) = code0 | (park << 8) | (parv << 9);
      } else {
        // ---- general tile: per-token table, one copy per run ----
        const uint64_t starts = spread_bits(even_starts) | (spread_bits(odd_starts) << 1);
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int j = 2 * lane + e;
          const int cd = code[e];
          uint32_t raw_off = 0, moff[2] = {0, 0};
          if (cd == kCodeNew) {  // native current-chunk row, raw slot j
            raw_off = j * 128;
            // The tile's new tokens are one run (past .. ke): rows stored 64 elements
            // apart are one contiguous block, fetched by a single copy from the run's
            // first lane; other layouts take one 128-byte copy per row.
            const int jn = max(past - t0, 0);                 // first new token of the tile
            const int nn = min(ke - t0, kBN) - jn;              // new tokens in the tile
            const bool first = j == jn;
            if (a.kt == kDim) {
              if (first) {
                mbar_expect_tx(rbar, nn * 128);
                bulk_g2s(sst + kRawK + raw_off, knew_g + static_cast<int64_t>(row[e]) * kDim, nn * 128, rbar);
              }
            } else {
              mbar_expect_tx(rbar, 128);
              bulk_g2s(sst + kRawK + raw_off, knew_g + static_cast<int64_t>(row[e]) * a.kt, 128, rbar);
            }
            if (a.vt == kDim) {
              if (first) {
                mbar_expect_tx(rbar, nn * 128);
                bulk_g2s(sst + kRawV + raw_off, vnew_g + static_cast<int64_t>(row[e]) * kDim, nn * 128, rbar);
              }
            } else {
              mbar_expect_tx(rbar, 128);
              bulk_g2s(sst + kRawV + raw_off, vnew_g + static_cast<int64_t>(row[e]) * a.vt, 128, rbar);
            }
          } else if (cd != 0) {
            const int j0 = 63 - __clzll(starts & ((2ull << j) - 1));  // first token of j's run
            const uint64_t after = starts & ~((2ull << j0) - 1);
            const int cnt = (after ? __ffsll(static_cast<long long>(after)) - 1 : kBN) - j0;
            const int rb = row_bytes(cd);
            const int r0 = row[e] - (j - j0);  // pool row of the run's first token
            raw_off = j0 * 128 + (j - j0) * rb;
            if (j == j0) {
              mbar_expect_tx(rbar, 2 * cnt * rb);
              bulk_g2s(sst + kRawK + j0 * 128, pool_of(cd) + row_at(0, r0) * rb, cnt * rb, rbar);
              bulk_g2s(sst + kRawV + j0 * 128, pool_of(cd) + row_at(1, r0) * rb, cnt * rb, rbar);
            }
            if (cd != 16) {
#pragma unroll
              for (int kv = 0; kv < 2; ++kv) {
                const bool bulk = cnt >= 2;  // the run's pairs by meta_run's one copy
                const int par = bulk ? (r0 & 1) : 0;
                moff[kv] = j0 * 16 + (par + (j - j0)) * 8;
                if (bulk && j == j0) {
                  meta_run(cd, kv, r0, cnt, sst + (kv ? kRawMetaV : kRawMetaK) + j0 * 16, rbar);
                } else if (!bulk) {  // a one-row run: this token's pair by a plain load
                  *reinterpret_cast<float2*>(st + (kv ? kRawMetaV : kRawMetaK) + moff[kv]) =
                      __ldg(meta_of(cd) + row_at(kv, row[e]));
                }
              }
            }
          }
          reinterpret_cast<uint2*>(st + kRawTab)[j] = make_uint2(cd | (raw_off << 8), moff[0] | (moff[1] << 16));
        }
        if (lane == 0) *reinterpret_cast<uint32_t*>(st + kRawHdr) = 0u;
      }
      __threadfence_block();  // table entries / fallback pairs stored by every lane ...
      __syncwarp();           // ... are ordered before lane 0's release-arrive
      if (lane == 0) mbar_arrive(rbar);
      // the map slot is free again: start the copy of tile i + kMapStages into it
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0 && i + kMapStages < ntiles) map_tile(i + kMapStages);
    }
    if (!ok && lane == 0) {
      *abort_flag = 1;
      report(status, DKV_ETIMEOUT, 3);
    }
  } else if (is_conv_warp(warp)) {
    // ================= converters: raw runs -> swizzled bf16 K / V tiles =================
    const int ctid = conv_index(warp) * 32 + lane;
    const int c = ctid & 7;    // 8-dim part
    const int jb = ctid >> 3;  // tokens jb + 16 k
    bool ok = true;
    for (int i = 0; i < ntiles; ++i) {
      const int rs = i % kRawStages;
      const int s = i % kStages;
      ok = mbar_wait(bar(B_RAWFULL + rs), (i / kRawStages) & 1, kWaitCycles);
      if (ok && i >= kStages) ok = mbar_wait(bar(B_EMPTY + s), ((i / kStages) + 1) & 1, kWaitCycles);
      if (!ok || *abort_flag) break;
      const uint8_t* st = smem + kOffRaw + rs * kRawStage;
      uint8_t* dstK = smem + kOffK + s * kTile;
      uint8_t* dstV = smem + kOffV + s * kTile;
      const uint32_t hdr = *reinterpret_cast<const uint32_t*>(st + kRawHdr);
      const int ucode = hdr & 0xff;
      if (ucode == 16) {
        convert_uniform<16>(st, dstK, dstV, jb, c, hdr);
      } else if (ucode == 8) {
        convert_uniform<8>(st, dstK, dstV, jb, c, hdr);
      } else if (ucode == 4) {
        convert_uniform<4>(st, dstK, dstV, jb, c, hdr);
      } else {
      // general tile: gather every operand of this thread's 8 (token, K|V) parts first, then convert
      uint2 ent[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) ent[k] = reinterpret_cast<const uint2*>(st + kRawTab)[jb + 16 * k];
      uint4 raw[8];
      float2 mt[8];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int code = ent[k].x & 0xff;
        const int raw_off = ent[k].x >> 8;
#pragma unroll
        for (int kv = 0; kv < 2; ++kv) {
          const uint8_t* rrow = st + (kv ? kRawV : kRawK) + raw_off;
          const int q = 2 * k + kv;
          raw[q] = make_uint4(0, 0, 0, 0);
          mt[q] = make_float2(0.f, 0.f);
          if (code == 16 || code == kCodeNew) {
            raw[q] = *reinterpret_cast<const uint4*>(rrow + c * 16);
          } else if (code == 8) {
            const uint2 w = *reinterpret_cast<const uint2*>(rrow + c * 8);
            raw[q].x = w.x;
            raw[q].y = w.y;
          } else if (code == 4) {
            raw[q].x = *reinterpret_cast<const uint32_t*>(rrow + c * 4);
          }
          if (code == 4 || code == 8) {
            const int meta_off = kv ? (ent[k].y >> 16) : (ent[k].y & 0xffff);
            mt[q] = *reinterpret_cast<const float2*>(st + (kv ? kRawMetaV : kRawMetaK) + meta_off);
          }
        }
      }
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int code = ent[k].x & 0xff;
        const int j = jb + 16 * k;
#pragma unroll
        for (int kv = 0; kv < 2; ++kv) {
          const int q = 2 * k + kv;
          uint4 v = raw[q];
          if (code == 8 || code == 4) {
            // codes -> exact floats via 2^23 + code, then code * scale + offset as one
            // packed FMA per pair (the single rounding of a fused multiply-add)
            uint32_t b0, b1;  // byte j of b0 / b1 = element 2j / 2j+1 (int4) or j / j+4 (int8)
            if (code == 8) {
              b0 = raw[q].x;
              b1 = raw[q].y;
            } else {
              b0 = raw[q].x & 0x0F0F0F0Fu;
              b1 = (raw[q].x >> 4) & 0x0F0F0F0Fu;
            }
            const float2 sc = make_float2(mt[q].y, mt[q].y);
            const float2 of = make_float2(mt[q].x, mt[q].x);
            const float2 mag = make_float2(-8388608.f, -8388608.f);
            uint32_t out[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              uint32_t lo, hi;  // elements (2e, 2e+1) in dim order
              if (code == 8) {
                const uint32_t w = e < 2 ? b0 : b1;
                lo = __byte_perm(w, 0x4B000000u, 0x7540 | (2 * (e & 1)));
                hi = __byte_perm(w, 0x4B000000u, 0x7540 | (2 * (e & 1) + 1));
              } else {
                lo = __byte_perm(b0, 0x4B000000u, 0x7540 | e);
                hi = __byte_perm(b1, 0x4B000000u, 0x7540 | e);
              }
              const float2 qf = add2(make_float2(__uint_as_float(lo), __uint_as_float(hi)), mag);
              const float2 x = fma2(qf, sc, of);
              out[e] = pack_bf16x2(x.x, x.y);
            }
            v = make_uint4(out[0], out[1], out[2], out[3]);
          } else if (code != 16 && code != kCodeNew) {
            v = make_uint4(0, 0, 0, 0);
          }
          *reinterpret_cast<uint4*>(smem + (kv ? kOffV : kOffK) + s * kTile + swz(j, c)) = v;
        }
      }
      }
      fence_proxy_async_smem();
      mbar_arrive(bar(B_FULL + s));
      mbar_arrive(bar(B_RAWEMPTY + rs));
    }
    if (!ok) {
      *abort_flag = 1;
      report(status, DKV_ETIMEOUT, 4);
    }
  } else {
    // ---- Q rows -> this thread's TMEM lane (zeros past the last row) ----
    pdl_wait();  // Q is the previous kernels' output; our output / workspace writes follow too
    {
      const int qmt = warp >> 2, qquad = warp & 3;
      const int qrl = qmt * 128 + qquad * 32 + lane;
      if (qmt < mt_count) {
        uint32_t qr[32];
        if (qrl < rows_here) {
          const int fr = row0 + qrl;
          const int m = fr / a.G;
          const int h = g * a.G + (fr - m * a.G);
          const uint4* src = reinterpret_cast<const uint4*>(a.q + chunk * a.qc + h * a.qh + m * a.qt);
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const uint4 v = src[c];
            qr[4 * c] = v.x;
            qr[4 * c + 1] = v.y;
            qr[4 * c + 2] = v.z;
            qr[4 * c + 3] = v.w;
          }
        } else {
#pragma unroll
          for (int c = 0; c < 32; ++c) qr[c] = 0u;
        }
        tmem_st32(tmem + (static_cast<uint32_t>(qquad * 32) << 16) + kColQ + qmt * 32, qr);
        tmem_wait_st();
      }
    }
    tc_fence_before();
    mbar_arrive(bar(B_QREADY));

    // ================= softmax (one TMEM lane / stacked row per thread) =================
    // Scores stay in raw units; p = 2^(s*c - m*c) with c = D^-0.5 log2(e) folded
    // into one FMA. The row sum of p is accumulated in fp32 (before p is rounded to
    // bf16 for the product), as the reference kernel does.
    const int mt = warp >> 2, quad = warp & 3;
    const int rl = mt * 128 + quad * 32 + lane;  // row inside the block
    if (mt * 128 + quad * 32 < rows_here) {
      const int fr = row0 + min(rl, rows_here - 1);
      const int lim = past + fr / a.G;  // last key this row may see
      const uint32_t lane_base = tmem + (static_cast<uint32_t>(quad * 32) << 16);
      const uint32_t col_o = kColO + mt * 64;
      float l_run = 0.f;  // sum of p of this row, scaled like O
      constexpr float kStale = 8.f / kScaleLog2;  // 2^8 headroom, in raw score units
      float m_raw = -INFINITY;
      bool ok = true;
      for (int i = 0; i < ntiles; ++i) {
        const int b = i & 1;
        if (__any_sync(0xffffffffu, *abort_flag != 0)) { ok = false; break; }
        ok = __all_sync(0xffffffffu, mbar_wait(bar(B_SFULL + b * 2 + mt), (i >> 1) & 1, kWaitCycles));
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
        mbar_arrive(bar(B_SFREE + b * 2 + mt));  // S[b][mt] may be overwritten by S(i + 2)
        const int t0 = kb + i * kBN;
        if (!(t0 + kBN <= ke && t0 + kBN - 1 <= past)) {  // boundary tile: mask
#pragma unroll
          for (int j = 0; j < 64; ++j) {
            const int t = t0 + j;
            s[j] = (t < ke && t <= lim) ? s[j] : -INFINITY;
          }
        }
        float mx;
        {  // 3-input max tree: depth 4 instead of a 63-long chain
          float t[22], u[8];
#pragma unroll
          for (int j = 0; j < 21; ++j) t[j] = max3f(s[3 * j], s[3 * j + 1], s[3 * j + 2]);
          t[21] = s[63];
#pragma unroll
          for (int j = 0; j < 7; ++j) u[j] = max3f(t[3 * j], t[3 * j + 1], t[3 * j + 2]);
          u[7] = t[21];
          mx = max3f(max3f(u[0], u[1], u[2]), max3f(u[3], u[4], u[5]), fmaxf(u[6], u[7]));
        }
        float alpha = 1.f;
        bool rescale = false;
        if (mx > m_raw + kStale) {  // also true for the first visible tile (m_raw = -inf)
          alpha = ex2((m_raw - mx) * kScaleLog2);
          rescale = m_raw != -INFINITY;
          m_raw = mx;
        }
        const float mc = m_raw == -INFINITY ? 0.f : m_raw * kScaleLog2;
        uint32_t pk[32];
        const float2 c2 = make_float2(kScaleLog2, kScaleLog2);
        const float2 nm2 = make_float2(-mc, -mc);
        float2 ls[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float2 x = fma2(make_float2(s[2 * j], s[2 * j + 1]), c2, nm2);
          // one pair in four on the FMA / integer pipes: MUFU ex2 is the softmax's bottleneck
          const float2 e = (j & 3) == 3 ? ex2_poly2(x) : make_float2(ex2(x.x), ex2(x.y));
          ls[j & 3] = add2(ls[j & 3], e);
          pk[j] = pack_bf16x2(e.x, e.y);
        }
        {
          const float2 t = add2(add2(ls[0], ls[1]), add2(ls[2], ls[3]));
          l_run = fmaf(l_run, alpha, t.x + t.y);
        }
        // P(i-1) V has landed before this warp touches TMEM again: O is stable for a
        // rescale and P(i-1) is consumed (a P store overlapping an in-flight P V
        // product corrupted the rows of warps that ran ahead, even into other columns)
        if (i > 0) {
          ok = __all_sync(0xffffffffu, mbar_wait(bar(B_ODONE + mt), (i - 1) & 1, kWaitCycles));
          if (!ok) break;
          tc_fence_after();
        }
        if (__any_sync(0xffffffffu, rescale)) {  // scale O
          const float f = rescale ? alpha : 1.f;
#pragma unroll
          for (int part = 0; part < 2; ++part) {
            uint32_t o[32];
            const uint32_t ta = lane_base + col_o + part * 32;
            tmem_ld32(ta, o);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 32; ++j) o[j] = __float_as_uint(__uint_as_float(o[j]) * f);
            tmem_st32(ta, o);
          }
          tmem_wait_st();
        }
        // P (bf16 pairs, 32 columns): the A operand of P V
        tmem_st32(lane_base + kColP + mt * 32, pk);
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(bar(B_PFULL + mt));
      }
      // ---- epilogue: O row from TMEM, its sum of p from registers ----
      float o[64];
      float l = 0.f;
#pragma unroll
      for (int j = 0; j < 64; ++j) o[j] = 0.f;
      if (ok && ntiles > 0) {
        ok = __all_sync(0xffffffffu, mbar_wait(bar(B_ODONE + mt), (ntiles - 1) & 1, kWaitCycles));
        tc_fence_after();
        if (ok) {
          uint32_t r0[32], r1[32];
          tmem_ld32(lane_base + col_o, r0);
          tmem_ld32(lane_base + col_o + 32, r1);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            o[j] = __uint_as_float(r0[j]);
            o[32 + j] = __uint_as_float(r1[j]);
          }
          l = l_run;
        }
      }
      if (!ok) {
        *abort_flag = 1;
        report(status, DKV_ETIMEOUT, 5);
      } else if (rl < rows_here) {
        const int frow = row0 + rl;
        if (a.splits == 1) {
          const int m = frow / a.G;
          const int h = g * a.G + (frow - m * a.G);
          uint16_t* dst = a.out + chunk * a.oc + (static_cast<int64_t>(m) * a.HQ + h) * kDim;
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
          // partial layout of part_o / part_ml: this split's 64 outputs of the row are 256
          // contiguous bytes, stored as eight whole 32-byte sectors
          const int grp = zc * a.mblocks + mb;
          float* dst = a.ws_o + part_o(grp, rl, kTcCtaRows, a.splits, split);
#pragma unroll
          for (int c = 0; c < kDim / 8; ++c) st_global_v8(dst + 8 * c, o + 8 * c);
          a.ws_ml[part_ml(grp, rl, kTcCtaRows, a.splits, split)] =
              make_float2(m_raw == -INFINITY ? -INFINITY : m_raw * kScaleLog2, l);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  // Every thread is now ordered after the softmax warps' griddepcontrol.wait: only
  // now may the dependent grid be scheduled, so that when it starts, every kernel
  // before this one has completed.
  pdl_trigger();
  if (warp == kSWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }

  // The fused pack (append + attend in one launch): the CTAs of this (chunk, KV
  // head) share the head's 2 x nq new rows; a CTA packs its share while the other
  // splits of its group finish (after publishing its partial), or after its
  // epilogue when there is no in-kernel merge. The rows written (>= past) are not
  // read by this call, which takes the new K/V natively.
  auto fused_pack = [&]() {
    const int pchunk = blockIdx.z / a.heads, pg = blockIdx.z - pchunk * a.heads;
    const dkv_pack_target* d = pack_of(a, pchunk);
    if (d == nullptr) return;
    pdl_wait();  // the new K/V are the previous kernel's output
    if (!pack_target_ok(*d, a.nq)) {
      if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) report_bad_target(*d, a.nq, pchunk);
      return;
    }
    const int ctas = gridDim.x * gridDim.y, j = blockIdx.x + gridDim.x * blockIdx.y;
    const int rows = 2 * a.nq, per = (rows + ctas - 1) / ctas;
    const int r_end = min((j + 1) * per, rows);
    const uint16_t* k = a.knew + pchunk * a.kc;
    const uint16_t* v = a.vnew + pchunk * a.vc;
    for (int r = j * per + (threadIdx.x >> 3); r < r_end; r += kThreadsTc / 8) {  // r: kv * nq + token
      const int kv = r >= a.nq;
      pack_frame_row(*d, k, v, a.kh, a.kt, a.vh, a.vt, a.layer, a.nq, a.heads, a.blocks, kv, pg, r - kv * a.nq,
                     threadIdx.x & 7, r);
    }
  };

  // ================= in-kernel split merge =================
  if (!a.fused) fused_pack();
  if (a.fused) {
    // block coordinates re-read here so nothing stays live across the roles above
    const int msplit = blockIdx.x, mrow0 = blockIdx.y * kTcCtaRows, mz = blockIdx.z;
    const int mchunk = mz / a.heads, mg = mz - mchunk * a.heads;
    const int mrows_here = min(kTcCtaRows, a.mrows - mrow0);
    const int grp = mz * a.mblocks + blockIdx.y;
    uint32_t* arrive = a.sync + grp;
    uint32_t* depart = a.sync + kSyncGroups + grp;
    // shared-memory base recomputed here: nothing from the roles above stays live
    uint8_t* msmem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    volatile int* go = reinterpret_cast<volatile int*>(msmem + kOffP);  // P region: idle now
    if (tid == 0) {
      // release at GPU scope, cumulative over the partials every thread of this CTA
      // stored before the barrier above: whoever acquires this arrival sees them
      red_add_release(arrive, 1u);
    }
    fused_pack();
    if (tid == 0) {
      const long long start = clock64();
      int ready = 1;
      while (ld_acquire(arrive) < static_cast<uint32_t>(a.splits)) {
        if (clock64() - start > kWaitCycles) {
          ready = 0;
          break;
        }
        __nanosleep(64);
      }
      if (!ready) report(status, DKV_ETIMEOUT, 6);
      *go = ready;
    }
    __syncthreads();
    if (*go) {
      const int r_begin = msplit * mrows_here / a.splits;
      const int r_end = (msplit + 1) * mrows_here / a.splits;
      merge_rows(a, mg, grp, mrow0, r_begin, r_end, a.out + mchunk * a.oc, msmem, threadIdx.x, status);
    }
    __syncthreads();
    // every CTA departs exactly once (also after a timeout): the last one out
    // returns both counters to zero for the next call on this workspace
    if (tid == 0 && atomicAdd(depart, 1u) == static_cast<uint32_t>(a.splits - 1)) {
      atomicExch(arrive, 0u);
      atomicExch(depart, 0u);
    }
  }
}

}  // namespace

namespace {
bool g_configured[64] = {};
int g_resident[64] = {};  // CTAs of this kernel the device holds at once

cudaError_t configure(int& dev) {
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!g_configured[dev]) {
    e = cudaFuncSetAttribute(attention_tc_kernel<SharedHistory>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kSmemTc);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(attention_tc_kernel<HistoryTable>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kSmemTc);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(attention_tc_kernel<DeviceHistories>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             kSmemTc);
    if (e != cudaSuccess) return e;
    int per_sm = 0, per_sm_table = 0, per_sm_device = 0, sms = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, attention_tc_kernel<SharedHistory>, kThreadsTc,
                                                      kSmemTc);
    if (e != cudaSuccess) return e;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm_table, attention_tc_kernel<HistoryTable>, kThreadsTc,
                                                      kSmemTc);
    if (e != cudaSuccess) return e;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm_device, attention_tc_kernel<DeviceHistories>,
                                                      kThreadsTc, kSmemTc);
    if (e != cudaSuccess) return e;
    per_sm = per_sm < per_sm_table ? per_sm : per_sm_table;
    per_sm = per_sm < per_sm_device ? per_sm : per_sm_device;
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    g_resident[dev] = per_sm * sms;
    g_configured[dev] = true;
  }
  return cudaSuccess;
}

// Where the splits of a call are merged. DKV_ATTENTION_MERGE=combine: always in the
// separate combine kernel (for GPUs shared under MPS, where a grid may not be
// resident at once); =kernel: inside the attention kernel whenever the grid fits.
// Unset: the measured default, which is the combine kernel for single-request
// attend-only calls (an eager cooperative launch costs more than the extra
// launch there) and the in-kernel merge for everything else (fused pack,
// batched requests), where one launch is faster.
enum class MergeMode { kDefault, kCombine, kKernel };

MergeMode merge_mode() {
  static const MergeMode mode = [] {
    const char* v = getenv("DKV_ATTENTION_MERGE");
    if (v && strcmp(v, "combine") == 0) return MergeMode::kCombine;
    if (v && strcmp(v, "kernel") == 0) return MergeMode::kKernel;
    return MergeMode::kDefault;
  }();
  return mode;
}
}  // namespace

bool attention_tc_fused(const AttnPlan& p, int heads, int dev, bool attend_only) {
  const MergeMode mode = merge_mode();
  if (mode == MergeMode::kCombine || (mode == MergeMode::kDefault && attend_only)) return false;
  // in-kernel merge only when no CTA of a group can wait for one that is not yet resident
  const long long grid = static_cast<long long>(p.splits) * p.mblocks * heads;
  return p.splits > 1 && heads * p.mblocks <= kSyncGroups && grid <= g_resident[dev];
}

cudaError_t attention_tc_merges_in_kernel(const AttnPlan& p, int heads, bool attend_only, bool* fused) {
  int dev = 0;
  const cudaError_t e = configure(dev);
  *fused = e == cudaSuccess && attention_tc_fused(p, heads, dev, attend_only);
  return e;
}

cudaError_t launch_attention_tc(AttnArgs& a, int heads, cudaStream_t stream, const HistoryTable* table,
                                const History* device_table) {
  int dev = 0;
  cudaError_t e = configure(dev);
  if (e != cudaSuccess) return e;
  AttnPlan p{};
  p.splits = a.splits;
  p.mblocks = a.mblocks;
  // one request (grid z = its KV heads), no fused pack, no history table
  const bool attend_only = a.pack_mode == 0 && table == nullptr && device_table == nullptr && heads == a.heads;
  a.fused = a.sync != nullptr && attention_tc_fused(p, heads, dev, attend_only);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.splits, a.mblocks, heads);
  cfg.blockDim = dim3(kThreadsTc);
  cfg.dynamicSmemBytes = kSmemTc;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // overlap our set-up and
  attr[0].val.programmaticStreamSerializationAllowed = 1;          // history streaming with the
  cfg.attrs = attr;                                                 // previous kernel's tail
  cfg.numAttrs = 1;
  if (a.fused) {  // the in-kernel merge waits for every block of its group: have them co-scheduled
    attr[1].id = cudaLaunchAttributeCooperative;
    attr[1].val.cooperative = 1;
    cfg.numAttrs = 2;
  }
  if (table != nullptr) return cudaLaunchKernelEx(&cfg, attention_tc_kernel<HistoryTable>, a, *table);
  if (device_table != nullptr)
    return cudaLaunchKernelEx(&cfg, attention_tc_kernel<DeviceHistories>, a, DeviceHistories{device_table});
  return cudaLaunchKernelEx(&cfg, attention_tc_kernel<SharedHistory>, a, SharedHistory{});
}

}  // namespace dkv
