// Split-K attention for short query chunks over packed mixed-precision history
// (sm_100a): decode steps and small candidate chunks, at most 16 stacked
// (query, head) rows per KV head, where the tensor-core kernel would pad its
// 128-row tiles with zeros and its fixed costs would dominate.
//
// Semantics are those of the reference kernel packed_attention
// (src/gpu_kernels.py:71-105): dequantised history rounded to bf16 (:93-94), the
// current chunk's native K/V, q.k * D^-0.5 (:95), bottom-right causal mask (:96),
// online softmax (:98-103), p rounded to bf16 before P.V (:102), fp32 accumulation.
//
// The work is memory-bound: every history byte is read once and the products are
// small. One CTA of eight warps per (chunk, KV head, history split); the splits of
// a group form one thread-block cluster. Each warp streams 32-key tiles of its
// split: the token maps (plain loads, two tiles ahead), the packed rows and their
// (offset, scale) pairs (cp.async, two tiles in flight), dequantisation into a
// bf16 K and V tile in its own shared memory, then S = Q K^T and O += P V on the
// mma.sync units (m16n8k16, one 16-row tile holds every row of the group) with an
// online softmax in registers. With at most 16 splits of the at most 5-10 groups of
// a decode step, most SMs are free, so a call's CTAs start and stream their
// history (two tiles per warp in flight, all of a 512-key split) while the
// previous kernel is still running. The eight warps' partials are merged in shared
// memory; each split then pushes its partial of every row (at most 16 rows x 264
// bytes) into the shared memory of the cluster CTA that finishes the row, and after
// one cluster barrier those rows are merged locally and stored.
#include "attention.cuh"
#include "pack_row.cuh"
#include "tc_ptx.cuh"

namespace dkv {
namespace {

using namespace ptx;

constexpr int kSpWarps = 8;
constexpr int kSpThreads = kSpWarps * 32;
constexpr int kSpKeys = 32;  // keys per warp tile
// Per warp: two raw stages (packed K rows, V rows: 128 B per token slot whatever
// the precision, 16-byte chunks XOR-swizzled by row like the tiles; K and V
// (offset, scale) pairs) and one bf16 K | V tile.
constexpr int kSpRawK = 0;
constexpr int kSpRawV = kSpKeys * 128;
constexpr int kSpRawMK = 2 * kSpKeys * 128;
constexpr int kSpRawMV = kSpRawMK + kSpKeys * 8;
constexpr int kSpRawStage = kSpRawMV + kSpKeys * 8;  // 8704
constexpr int kSpTileV = kSpKeys * 128;              // V tile after the K tile
constexpr int kSpTile = 2 * kSpKeys * 128;           // 8192
constexpr int kSpWarpBytes = 2 * kSpRawStage + kSpTile;
constexpr int kSpCodeNew = 17;  // token of the current chunk: native row of knew / vnew
constexpr int kSpMaxSplits = 16;  // a group's splits form one cluster
// Cluster merge: the partials of the rows this CTA finishes (row r is finished by
// cluster rank r % splits, in slot split * per + r / splits, per = ceil(rows /
// splits)), pushed there by every split; a region of its own, since a split may
// push while this CTA still streams its tiles.
constexpr int kSpRecvSlots = 16 + kSpMaxSplits;  // splits * per <= rows + splits
constexpr int kSpOffRecv = kSpWarps * kSpWarpBytes;
constexpr int kSpOffRecvMl = kSpOffRecv + kSpRecvSlots * kDim * 4;
constexpr int kSpSmem = kSpOffRecvMl + kSpRecvSlots * 8;  // 213,248 bytes: one CTA per SM
// After the tiles, the same memory holds the merge: each warp's partial O [16][64]
// and (max, sum) [16], then the CTA's partial O [16][64] and (max, sum) [16].
constexpr int kSpRows = 16;
constexpr int kSpWarpPart = kSpRows * kDim * 4 + kSpRows * 8;
constexpr int kSpOffCta = kSpWarps * kSpWarpPart;
constexpr int kSpOffCtaMl = kSpOffCta + kSpRows * kDim * 4;
static_assert(kSpOffCtaMl + kSpRows * 8 <= kSpOffRecv, "merge area fits the tiles");
static_assert(kSpSmem <= 227 * 1024, "shared memory budget");

__device__ __forceinline__ int sp_swz(int row, int chunk) { return row * 128 + ((chunk ^ (row & 7)) << 4); }

__device__ __forceinline__ void cp_async16_cg(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(src) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// D (16x8 fp32) += A (16x16 bf16, row) * B (16x8 bf16, col).
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// 8 codes -> 8 bf16 of code * scale + offset (one fused multiply-add per value,
// codes made exact floats as 2^23 + code minus 2^23): the tensor-core kernel's
// dequantisation. w0 (and w1 for 8-bit) hold the codes of 8 consecutive dims.
template <int BITS>
__device__ __forceinline__ uint4 sp_dequant(uint32_t w0, uint32_t w1, float offset, float scale) {
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

// The K (kv = 0) or V row of one token (this lane's key) from a raw stage into the
// bf16 tile: code 4 / 8 / 16 (pool rows), kSpCodeNew (native bf16 row), anything
// else zeros.
__device__ __forceinline__ void sp_convert_row(const uint8_t* raw, uint8_t* tile, int j, int code, int kv) {
  {
    const uint8_t* src = raw + (kv ? kSpRawV : kSpRawK);  // chunk c of row j at sp_swz(j, c)
    uint8_t* dst = tile + (kv ? kSpTileV : 0);
    const float2 m = *reinterpret_cast<const float2*>(raw + (kv ? kSpRawMV : kSpRawMK) + j * 8);
    if (code == 4) {
      const uint4 w0 = *reinterpret_cast<const uint4*>(src + sp_swz(j, 0));
      const uint4 w1 = *reinterpret_cast<const uint4*>(src + sp_swz(j, 1));
      const uint32_t w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
      for (int c = 0; c < 8; ++c) *reinterpret_cast<uint4*>(dst + sp_swz(j, c)) = sp_dequant<4>(w[c], 0u, m.x, m.y);
    } else if (code == 8) {
#pragma unroll
      for (int c = 0; c < 8; c += 2) {
        const uint4 w = *reinterpret_cast<const uint4*>(src + sp_swz(j, c / 2));
        *reinterpret_cast<uint4*>(dst + sp_swz(j, c)) = sp_dequant<8>(w.x, w.y, m.x, m.y);
        *reinterpret_cast<uint4*>(dst + sp_swz(j, c + 1)) = sp_dequant<8>(w.z, w.w, m.x, m.y);
      }
    } else if (code == 16 || code == kSpCodeNew) {
#pragma unroll
      for (int c = 0; c < 8; ++c)
        *reinterpret_cast<uint4*>(dst + sp_swz(j, c)) = *reinterpret_cast<const uint4*>(src + sp_swz(j, c));
    } else {
#pragma unroll
      for (int c = 0; c < 8; ++c) *reinterpret_cast<uint4*>(dst + sp_swz(j, c)) = make_uint4(0, 0, 0, 0);
    }
  }
}

// Merge weight of a partial with running max m against the common max M (0 for a
// partial that saw no key): MUFU ex2, as the softmax itself. The split kernel has
// its own merge (one plan, one order), so it need not match the other kernels' bits.
__device__ __forceinline__ float sp_weight(float m, float M) { return m == -INFINITY ? 0.f : ex2(m - M); }

// out[c] = bf16(acc[c] / den), by one reciprocal (the normalisation of a row)
__device__ __forceinline__ uint4 sp_normalise(const float (&acc)[8], float den) {
  const float inv = __frcp_rn(den);
  uint4 w;
  w.x = pack_bf16x2(acc[0] * inv, acc[1] * inv);
  w.y = pack_bf16x2(acc[2] * inv, acc[3] * inv);
  w.z = pack_bf16x2(acc[4] * inv, acc[5] * inv);
  w.w = pack_bf16x2(acc[6] * inv, acc[7] * inv);
  return w;
}

template <class Hist>
__global__ void __launch_bounds__(kSpThreads, 1)
attention_split_kernel(const __grid_constant__ AttnArgs a, const __grid_constant__ Hist hist) {
  extern __shared__ __align__(128) uint8_t sp_smem[];
  const int split = blockIdx.x;
  const int zc = blockIdx.z;  // chunk * heads + KV head
  const int chunk = zc / a.heads;
  const int g = zc - chunk * a.heads;
  const History& H = history_of(a, hist, chunk);
  const int past = checked_past(H, chunk);
  int32_t* const status = H.status;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int R = a.mrows;  // stacked rows of the group (<= 16)
  const int keys = request_chunk(a, past);
  const int kb = split * keys;
  int ke = min(kb + keys, past + a.nq);
  ke = min(ke, past + (R - 1) / a.G + 1);  // no row sees further
  const int ntiles = ke > kb ? (ke - kb + kSpKeys - 1) / kSpKeys : 0;
  const int mine = ntiles > warp ? (ntiles - warp + kSpWarps - 1) / kSpWarps : 0;  // tiles w, w + 8, ...
  // every CTA of the cluster announces it has started; the wait comes right before
  // the first store into another CTA's shared memory
  if (a.splits > 1) cluster_arrive_relaxed();
  // Q rows head for L2 now (no value is read before the wait below; L2 is coherent,
  // so the loads after it still see the producer's writes)
  if (threadIdx.x < R) {
    const int m = threadIdx.x / a.G;
    const int hq = g * a.G + (threadIdx.x - m * a.G);
    asm volatile("prefetch.global.L2 [%0];\n" ::"l"(a.q + chunk * a.qc + hq * a.qh + m * a.qt));
  }

  uint8_t* const wsm = sp_smem + warp * kSpWarpBytes;
  const uint32_t wsm_a = smem_addr(wsm);
  uint8_t* const tile = wsm + 2 * kSpRawStage;
  const uint32_t tile_a = wsm_a + 2 * kSpRawStage;

  // ---- pools of this (layer, head) ----
  const int64_t blk_k = (static_cast<int64_t>(a.layer) * 2) * a.heads + g;
  const int64_t blk_v = blk_k + a.heads;
  const uint8_t* const p4 = static_cast<const uint8_t*>(H.p4);
  const uint8_t* const p8 = static_cast<const uint8_t*>(H.p8);
  const uint8_t* const p16 = static_cast<const uint8_t*>(H.p16);
  const float2* const m4 = static_cast<const float2*>(H.m4);
  const float2* const m8 = static_cast<const float2*>(H.m8);
  const uint16_t* const knew_g = a.knew + chunk * a.kc + g * a.kh;
  const uint16_t* const vnew_g = a.vnew + chunk * a.vc + g * a.vh;

  // Token of this lane in the warp's jj-th tile, its precision code and pool row.
  auto tile_t0 = [&](int jj) { return kb + (warp + jj * kSpWarps) * kSpKeys; };
  auto load_map = [&](int jj, int& code, int& row) {
    code = 0;
    row = 0;
    if (jj >= mine) return;
    const int t = tile_t0(jj) + lane;
    if (t >= ke) return;
    if (t >= past) {
      code = kSpCodeNew;
      row = t - past;
      return;
    }
    code = __ldg(H.codes + t);
    row = __ldg(H.rows + t);
    const int64_t cap = code == 4 ? H.cap4 : (code == 8 ? H.cap8 : H.cap16);
    if (code != 4 && code != 8 && code != 16) {
      report(status, DKV_EPLAN, t);
      code = 0;
    } else if (row < 0 || row >= cap) {
      report(status, DKV_ECAPACITY, t);
      code = 0;
    }
  };
  // Starts the copies of the warp's tile into raw stage st, every lane giving its
  // token's (code, row) from load_map. Runs of consecutive pool rows (one
  // precision, one page: contiguous bytes) are copied by the whole warp in
  // consecutive 16-byte chunks, so a request covers whole cache lines (a 32-row
  // bf16 run: 8 requests of 512 contiguous bytes per K and V) and every sector is
  // fetched once; a token of the current chunk brings its native row itself
  // (issue_new; with news = false the caller does that later).
  auto issue_new = [&](int st, int code, int row) {
    const uint32_t base = wsm_a + st * kSpRawStage;
    if (code == kSpCodeNew) {
      const uint16_t* kr = knew_g + static_cast<int64_t>(row) * a.kt;
      const uint16_t* vr = vnew_g + static_cast<int64_t>(row) * a.vt;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        cp_async16_cg(base + kSpRawK + sp_swz(lane, c), kr + c * 8);
        cp_async16_cg(base + kSpRawV + sp_swz(lane, c), vr + c * 8);
      }
    }
  };
  auto issue_tile = [&](int st, int code, int row, bool news) {
    const uint32_t base = wsm_a + st * kSpRawStage;
    if (news) issue_new(st, code, row);
    const bool pooled = code == 4 || code == 8 || code == 16;
    const int pcode = __shfl_up_sync(0xffffffffu, code, 1);
    const int prow = __shfl_up_sync(0xffffffffu, row, 1);
    const bool start = pooled && (lane == 0 || pcode != code || prow + 1 != row || (row & (kPageRows - 1)) == 0);
    uint32_t starts = __ballot_sync(0xffffffffu, start);
    const uint32_t breaks = __ballot_sync(0xffffffffu, !pooled);  // a run ends before these
    while (starts != 0u) {
      const int j0 = __ffs(starts) - 1;
      starts &= starts - 1u;
      const uint32_t after = (starts | breaks) & ~((2u << j0) - 1u);  // lanes above j0
      const int cnt = (after != 0u ? __ffs(after) - 1 : 32) - j0;
      const int rc = __shfl_sync(0xffffffffu, code, j0);
      const int r0 = __shfl_sync(0xffffffffu, row, j0);
      const int lg = rc == 4 ? 1 : (rc == 8 ? 2 : 3);  // log2 of 16-byte chunks per row
      const int rb = 16 << lg;
      const uint8_t* pool = rc == 4 ? p4 : (rc == 8 ? p8 : p16);
      const uint8_t* ks = pool + pool_row(blk_k, r0, a.blocks) * rb;
      const uint8_t* vs = pool + pool_row(blk_v, r0, a.blocks) * rb;
      for (int q = lane; q < (cnt << lg); q += 32) {
        const uint32_t at = sp_swz(j0 + (q >> lg), q & ((1 << lg) - 1));
        cp_async16_cg(base + kSpRawK + at, ks + q * 16);
        cp_async16_cg(base + kSpRawV + at, vs + q * 16);
      }
      if (rc != 16 && lane < cnt) {
        const float2* meta = rc == 8 ? m8 : m4;
        cp_async8(base + kSpRawMK + (j0 + lane) * 8, meta + pool_row(blk_k, r0, a.blocks) + lane);
        cp_async8(base + kSpRawMV + (j0 + lane) * 8, meta + pool_row(blk_v, r0, a.blocks) + lane);
      }
    }
  };

  // ---- prologue: maps of tiles 0..2 and the history rows of tiles 0 and 1 (before
  // the wait unless the previous launch may have written this history); the rows
  // of the call's own new tokens, Q and every write after the wait ----
  if (a.hist_wait) pdl_wait();
  int code_c[3], row_c[3];  // maps of tiles jj, jj + 1, jj + 2 (rotating)
  load_map(0, code_c[0], row_c[0]);
  load_map(1, code_c[1], row_c[1]);
  load_map(2, code_c[2], row_c[2]);
  issue_tile(0, code_c[0], row_c[0], false);
  cp_async_commit();
  issue_tile(1, code_c[1], row_c[1], false);
  cp_async_commit();
  if (!a.hist_wait) pdl_wait();  // new K/V and Q are the previous kernels' output
  pdl_trigger();                 // the next kernel may start streaming its own history
  // new-token rows of tiles 0 and 1 as a third group (empty for most warps), so
  // tile 0 waits for it and every later tile keeps waiting for all but one group
  const bool late = __any_sync(0xffffffffu, code_c[0] == kSpCodeNew || code_c[1] == kSpCodeNew);
  issue_new(0, code_c[0], row_c[0]);
  issue_new(1, code_c[1], row_c[1]);
  cp_async_commit();

  // ---- Q fragments (rows g0 = lane / 4 and g0 + 8; zeros past the last row) ----
  const int g0 = lane >> 2, q4 = lane & 3;
  uint32_t qa[4][4];  // [k-step][a0..a3]
  {
    const uint16_t* qr[2] = {nullptr, nullptr};
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int r = g0 + 8 * h;
      if (r < R) {
        const int m = r / a.G;
        const int hq = g * a.G + (r - m * a.G);
        qr[h] = a.q + chunk * a.qc + hq * a.qh + m * a.qt;
      }
    }
#pragma unroll
    for (int kt = 0; kt < 4; ++kt) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int d = 16 * kt + 2 * q4;
        qa[kt][h] = qr[h] ? *reinterpret_cast<const uint32_t*>(qr[h] + d) : 0u;
        qa[kt][h + 2] = qr[h] ? *reinterpret_cast<const uint32_t*>(qr[h] + d + 8) : 0u;
      }
    }
  }
  const int lim0 = past + min(g0, R - 1) / a.G;       // last key row g0 may see
  const int lim1 = past + min(g0 + 8, R - 1) / a.G;   // ... row g0 + 8

  // ---- the warp's tiles ----
  constexpr float kStale = 8.f / kScaleLog2;  // running max moves only by > 2^8 (exact after O / l)
  float m_raw[2] = {-INFINITY, -INFINITY};
  float l_run[2] = {0.f, 0.f};  // this lane's keys' sum of p, scaled like O
  float o[8][4];
#pragma unroll
  for (int dt = 0; dt < 8; ++dt) o[dt][0] = o[dt][1] = o[dt][2] = o[dt][3] = 0.f;
  for (int jj = 0; jj < mine; ++jj) {
    const int st = jj & 1;
    if (jj == 0 && late) {
      cp_async_wait<0>();  // tile 0's copies and the new-token rows of tiles 0 and 1
    } else {
      cp_async_wait<1>();  // tile jj's copies (this lane's) have landed
    }
    __syncwarp();
    sp_convert_row(wsm + st * kSpRawStage, tile, lane, code_c[0], 0);  // K first: S needs only K
    __syncwarp();  // the tile's K rows are in shared memory

    // S = Q K^T: 4 n-tiles of 8 keys, 4 k-steps of 16 dims
    float s[4][4];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
      s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int key = 8 * nt + (lane & 7);
        const int ch = 4 * h + (lane >> 3);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(tile_a + sp_swz(key, ch), b0, b1, b2, b3);
        mma16816(s[nt], qa[2 * h][0], qa[2 * h][1], qa[2 * h][2], qa[2 * h][3], b0, b1);
        mma16816(s[nt], qa[2 * h + 1][0], qa[2 * h + 1][1], qa[2 * h + 1][2], qa[2 * h + 1][3], b2, b3);
      }
    }
    // V rows while the products are in flight
    sp_convert_row(wsm + st * kSpRawStage, tile, lane, code_c[0], 1);
    __syncwarp();  // the whole tile is in shared memory; raw stage st is free
    // rotate the maps and start tile jj + 2 into the freed stage
    code_c[0] = code_c[1];
    row_c[0] = row_c[1];
    code_c[1] = code_c[2];
    row_c[1] = row_c[2];
    issue_tile(st, code_c[1], row_c[1], true);
    cp_async_commit();
    load_map(jj + 3, code_c[2], row_c[2]);
    // mask, online max, p = 2^(s c - m c), row sums
    const int t0 = tile_t0(jj);
    if (!(t0 + kSpKeys <= ke && t0 + kSpKeys - 1 <= past)) {
#pragma unroll
      for (int nt = 0; nt < 4; ++nt) {
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int t = t0 + 8 * nt + 2 * q4 + e;
          if (!(t < ke && t <= lim0)) s[nt][e] = -INFINITY;
          if (!(t < ke && t <= lim1)) s[nt][2 + e] = -INFINITY;
        }
      }
    }
    float alpha[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float mx = max3f(fmaxf(s[0][2 * h], s[0][2 * h + 1]), fmaxf(s[1][2 * h], s[1][2 * h + 1]),
                       fmaxf(s[2][2 * h], s[2][2 * h + 1]));
      mx = fmaxf(mx, fmaxf(s[3][2 * h], s[3][2 * h + 1]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      alpha[h] = 1.f;
      if (mx > m_raw[h] + kStale) {  // also the first visible tile (m_raw = -inf)
        alpha[h] = m_raw[h] == -INFINITY ? 1.f : ex2((m_raw[h] - mx) * kScaleLog2);
        m_raw[h] = mx;
      }
    }
    uint32_t pa[2][4];  // P as the A operand of the two 16-key k-steps
    float ls[2] = {0.f, 0.f};
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float mc = m_raw[h] == -INFINITY ? 0.f : m_raw[h] * kScaleLog2;
        const float e0 = ex2(fmaf(s[nt][2 * h], kScaleLog2, -mc));
        const float e1 = ex2(fmaf(s[nt][2 * h + 1], kScaleLog2, -mc));
        ls[h] += e0 + e1;
        pa[nt >> 1][(nt & 1) * 2 + h] = pack_bf16x2(e0, e1);
      }
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) l_run[h] = fmaf(l_run[h], alpha[h], ls[h]);
    if (alpha[0] != 1.f || alpha[1] != 1.f) {
#pragma unroll
      for (int dt = 0; dt < 8; ++dt) {
        o[dt][0] *= alpha[0];
        o[dt][1] *= alpha[0];
        o[dt][2] *= alpha[1];
        o[dt][3] *= alpha[1];
      }
    }
    // O += P V: 2 k-steps of 16 keys, 8 n-tiles of 8 dims
#pragma unroll
    for (int ks = 0; ks < 2; ++ks) {
#pragma unroll
      for (int dp = 0; dp < 4; ++dp) {
        const int key = 16 * ks + 8 * ((lane >> 3) & 1) + (lane & 7);
        const int ch = 2 * dp + (lane >> 4);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(tile_a + kSpTileV + sp_swz(key, ch), b0, b1, b2, b3);
        mma16816(o[2 * dp], pa[ks][0], pa[ks][1], pa[ks][2], pa[ks][3], b0, b1);
        mma16816(o[2 * dp + 1], pa[ks][0], pa[ks][1], pa[ks][2], pa[ks][3], b2, b3);
      }
    }
    __syncwarp();  // the tile is free for the next conversion
  }
  cp_async_wait<0>();

  // ---- fused pack (append + attend in one launch): the CTAs of this (chunk, KV
  // head) share the head's 2 x nq new rows, 8 threads per row. The rows written
  // (>= past) are not read by this call, which takes the new K/V natively. ----
  if (const dkv_pack_target* d = pack_of(a, chunk)) {
    if (!pack_target_ok(*d, a.nq)) {
      if (split == 0 && threadIdx.x == 0) report_bad_target(*d, a.nq, chunk);
    } else {
      const int rows = 2 * a.nq, per = (rows + a.splits - 1) / a.splits;
      const int r_end = min((split + 1) * per, rows);
      const uint16_t* k = a.knew + chunk * a.kc;
      const uint16_t* v = a.vnew + chunk * a.vc;
      for (int r = split * per + (threadIdx.x >> 3); r < r_end; r += kSpThreads / 8) {  // r: kv * nq + token
        const int kv = r >= a.nq;
        pack_frame_row(*d, k, v, a.kh, a.kt, a.vh, a.vt, a.layer, a.nq, a.heads, a.blocks, kv, g, r - kv * a.nq,
                       threadIdx.x & 7, r);
      }
    }
  }

  // ---- merge the warps' partials in shared memory (the tiles are done) ----
  __syncthreads();
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    l_run[h] += __shfl_xor_sync(0xffffffffu, l_run[h], 1);
    l_run[h] += __shfl_xor_sync(0xffffffffu, l_run[h], 2);
  }
  {
    float* wo = reinterpret_cast<float*>(sp_smem + warp * kSpWarpPart);
    float2* wml = reinterpret_cast<float2*>(sp_smem + warp * kSpWarpPart + kSpRows * kDim * 4);
#pragma unroll
    for (int dt = 0; dt < 8; ++dt) {
      *reinterpret_cast<float2*>(wo + g0 * kDim + 8 * dt + 2 * q4) = make_float2(o[dt][0], o[dt][1]);
      *reinterpret_cast<float2*>(wo + (g0 + 8) * kDim + 8 * dt + 2 * q4) = make_float2(o[dt][2], o[dt][3]);
    }
    if (q4 == 0) {
#pragma unroll
      for (int h = 0; h < 2; ++h)
        wml[g0 + 8 * h] = make_float2(m_raw[h] == -INFINITY ? -INFINITY : m_raw[h] * kScaleLog2, l_run[h]);
    }
  }
  __syncthreads();
  if (a.splits > 1) cluster_wait_acquire();  // every CTA of the cluster has started
  // the CTA's partial: one thread per (row, 8 dims)
  for (int i = threadIdx.x; i < R * 8; i += kSpThreads) {
    const int r = i >> 3, d0 = (i & 7) * 8;
    float M = -INFINITY;
    float2 ml[kSpWarps];
#pragma unroll
    for (int w = 0; w < kSpWarps; ++w) {
      ml[w] = reinterpret_cast<const float2*>(sp_smem + w * kSpWarpPart + kSpRows * kDim * 4)[r];
      M = fmaxf(M, ml[w].x);
    }
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    float den = 0.f;
#pragma unroll
    for (int w = 0; w < kSpWarps; ++w) {
      const float wt = sp_weight(ml[w].x, M);
      den = __fmaf_rn(wt, ml[w].y, den);
      const float* wo = reinterpret_cast<const float*>(sp_smem + w * kSpWarpPart) + r * kDim + d0;
#pragma unroll
      for (int c = 0; c < 8; ++c) acc[c] = __fmaf_rn(wt, wo[c], acc[c]);
    }
    if (a.splits == 1) {  // no other split: normalise and store
      const int m = r / a.G;
      const int hq = g * a.G + (r - m * a.G);
      uint16_t* dst = a.out + chunk * a.oc + (static_cast<int64_t>(m) * a.HQ + hq) * kDim + d0;
      *reinterpret_cast<uint4*>(dst) = sp_normalise(acc, den);
    } else {
      // push this split's partial of row r into the receive buffer of the CTA that
      // finishes the row (fire-and-forget remote stores, released by the barrier)
      const int S = a.splits, per = (R + S - 1) / S;
      const uint32_t owner = static_cast<uint32_t>(r % S);
      const int slot = split * per + r / S;
      const uint32_t dst = dsmem_addr(smem_addr(sp_smem) + kSpOffRecv + (slot * kDim + d0) * 4, owner);
      st_dsmem_f4(dst, make_float4(acc[0], acc[1], acc[2], acc[3]));
      st_dsmem_f4(dst + 16, make_float4(acc[4], acc[5], acc[6], acc[7]));
      if (d0 == 0) st_dsmem_f2(dsmem_addr(smem_addr(sp_smem) + kSpOffRecvMl + slot * 8, owner), make_float2(M, den));
    }
  }
  if (a.splits == 1) return;

  // ---- finish the rows this CTA owns from every split's pushed partial ----
  cluster_arrive_release();  // this CTA's pushes are done
  cluster_wait_acquire();    // ... and every other split's
  const int S = a.splits, per = (R + S - 1) / S;
  for (int i = threadIdx.x; i < R * 8; i += kSpThreads) {
    const int r = i >> 3, d0 = (i & 7) * 8;
    if (r % S != split) continue;
    const int sl = r / S;
    float2 ml[kSpMaxSplits];
    float M = -INFINITY;
#pragma unroll
    for (int sp = 0; sp < kSpMaxSplits; ++sp) {
      ml[sp] = sp < S ? reinterpret_cast<const float2*>(sp_smem + kSpOffRecvMl)[sp * per + sl]
                      : make_float2(-INFINITY, 0.f);
      M = fmaxf(M, ml[sp].x);
    }
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    float den = 0.f;
#pragma unroll
    for (int sp = 0; sp < kSpMaxSplits; ++sp) {
      if (sp < S) {
        const float wt = sp_weight(ml[sp].x, M);
        den = __fmaf_rn(wt, ml[sp].y, den);
        const float* src = reinterpret_cast<const float*>(sp_smem + kSpOffRecv) + (sp * per + sl) * kDim + d0;
#pragma unroll
        for (int c = 0; c < 8; ++c) acc[c] = __fmaf_rn(wt, src[c], acc[c]);
      }
    }
    const int m = r / a.G;
    const int hq = g * a.G + (r - m * a.G);
    uint16_t* dst = a.out + chunk * a.oc + (static_cast<int64_t>(m) * a.HQ + hq) * kDim + d0;
    *reinterpret_cast<uint4*>(dst) = sp_normalise(acc, den);
  }
  // nothing reads another CTA's shared memory after the barrier: no CTA waits to leave
}

bool g_split_configured[64] = {};

cudaError_t configure_split(int dev) {
  if (g_split_configured[dev]) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(attention_split_kernel<SharedHistory>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, kSpSmem);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(attention_split_kernel<SharedHistory>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  if (e != cudaSuccess) return e;
  g_split_configured[dev] = true;
  return cudaSuccess;
}

}  // namespace

cudaError_t launch_attention_split(const AttnArgs& a, int heads, cudaStream_t stream) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  e = configure_split(dev);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.splits, 1, heads);
  cfg.blockDim = dim3(kSpThreads);
  cfg.dynamicSmemBytes = kSpSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (a.splits > 1) {  // the splits of each (chunk, KV head) form one cluster
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = a.splits;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.numAttrs = 2;
  }
  return cudaLaunchKernelEx(&cfg, attention_split_kernel<SharedHistory>, a, SharedHistory{});
}

}  // namespace dkv
