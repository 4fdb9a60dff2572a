// Shared device helpers for libdkv (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "dkv.h"

namespace dkv {

constexpr int kDim = 64;        // head_dim supported by every kernel
constexpr int kRowBytes4 = 32;  // packed 4-bit row
constexpr int kRowBytes8 = 64;  // 8-bit row
constexpr int kRowBytes16 = 128;

// Pools are paged (dkv.h): row r of block b ((layer, K|V, head): b = (layer * 2 +
// kv) * heads + head, of `blocks` = layers * 2 * heads) sits in page r / 64, and
// page p of every block is stored side by side, so growing a pool appends pages
// and moves no row. Returns the row's index in units of pool rows.
constexpr int kPageRows = DKV_PAGE_ROWS;
static_assert(kPageRows == 64, "page arithmetic below assumes 64-row pages");
__host__ __device__ __forceinline__ int64_t pool_row(int64_t block, int64_t row, int64_t blocks) {
  return ((row >> 6) * blocks + block) * kPageRows + (row & 63);
}

// Records the first device-side error. Kernels never trap: they skip the bad
// access and leave the code for the host to read after a synchronisation.
__device__ __forceinline__ void report(int32_t* status, int code, int detail) {
  if (status != nullptr) {
    if (atomicCAS(status, 0, code) == 0) status[1] = detail;
  }
}

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// Round-to-nearest-even float -> bf16 pair packed in one 32-bit word (lo first).
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Dequantise one code exactly as the reference CPU unpack does
// (src/kv_quantization.py:91): fp32 multiply, then fp32 add, each rounded.
__device__ __forceinline__ float dequant(uint32_t code, float offset, float scale) {
  return __fadd_rn(__fmul_rn(static_cast<float>(code), scale), offset);
}

// Dequantises 8 consecutive dims of one row into 4 bf16x2 words.
//   bits 16: raw.{x,y,z,w} already hold 8 bf16
//   bits 8 : raw.x, raw.y hold 8 codes (byte i = dim i)
//   bits 4 : raw.x holds 8 nibbles (byte j = dim 2j | dim 2j+1 << 4)
__device__ __forceinline__ uint4 dequant8(int bits, uint4 raw, float offset, float scale) {
  if (bits == 16) return raw;
  uint32_t c[8];
  if (bits == 8) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      c[i] = (raw.x >> (8 * i)) & 0xffu;
      c[4 + i] = (raw.y >> (8 * i)) & 0xffu;
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) c[i] = (raw.x >> (4 * i)) & 0xfu;
  }
  uint4 o;
  o.x = pack_bf16x2(dequant(c[0], offset, scale), dequant(c[1], offset, scale));
  o.y = pack_bf16x2(dequant(c[2], offset, scale), dequant(c[3], offset, scale));
  o.z = pack_bf16x2(dequant(c[4], offset, scale), dequant(c[5], offset, scale));
  o.w = pack_bf16x2(dequant(c[6], offset, scale), dequant(c[7], offset, scale));
  return o;
}

// Pool geometry of one call, shared by the history readers.
struct Pools {
  const uint8_t* p4;
  const float2* m4;
  const uint8_t* p8;
  const float2* m8;
  const uint16_t* p16;
  int64_t cap4, cap8, cap16;
  int heads;
  int blocks;  // layers * 2 * heads: pages of the blocks side by side
};

// Raw bytes + metadata of 8 dims (one eighth) of a history row.
struct RowPart {
  uint4 raw;
  float offset, scale;
  int bits;  // 0 = nothing valid (zero-filled)
};

// Loads part `part` (dims 8*part .. 8*part+7) of logical history token t for
// (layer, kv, head). Bounds-checks the map entries; a bad entry is reported and
// read as zeros.
__device__ __forceinline__ RowPart load_history_part(const Pools& P, const int32_t* rows,
                                                     const uint8_t* codes, int layer, int kv,
                                                     int head, int t, int part, int32_t* status) {
  RowPart r;
  r.raw = make_uint4(0, 0, 0, 0);
  r.offset = 0.f;
  r.scale = 0.f;
  r.bits = 0;
  const int code = codes[t];
  const int64_t row = rows[t];
  const int64_t base = (static_cast<int64_t>(layer) * 2 + kv) * P.heads + head;
  const int64_t at = row >= 0 ? pool_row(base, row, P.blocks) : 0;  // used only once row is checked
  if (code == 16) {
    if (row < 0 || row >= P.cap16) { report(status, DKV_ECAPACITY, t); return r; }
    const uint4* src = reinterpret_cast<const uint4*>(P.p16 + at * kDim) + part;
    r.raw = __ldg(src);
    r.bits = 16;
  } else if (code == 8) {
    if (row < 0 || row >= P.cap8) { report(status, DKV_ECAPACITY, t); return r; }
    const uint2* src = reinterpret_cast<const uint2*>(P.p8 + at * kRowBytes8) + part;
    uint2 w = __ldg(src);
    r.raw.x = w.x;
    r.raw.y = w.y;
    float2 m = __ldg(P.m8 + at);
    r.offset = m.x;
    r.scale = m.y;
    r.bits = 8;
  } else if (code == 4) {
    if (row < 0 || row >= P.cap4) { report(status, DKV_ECAPACITY, t); return r; }
    const uint32_t* src = reinterpret_cast<const uint32_t*>(P.p4 + at * kRowBytes4) + part;
    r.raw.x = __ldg(src);
    float2 m = __ldg(P.m4 + at);
    r.offset = m.x;
    r.scale = m.y;
    r.bits = 4;
  } else {
    report(status, DKV_EPLAN, t);
  }
  return r;
}

__device__ __forceinline__ uint4 dequant_part(const RowPart& r) {
  if (r.bits == 0) return make_uint4(0, 0, 0, 0);
  return dequant8(r.bits, r.raw, r.offset, r.scale);
}

}  // namespace dkv
