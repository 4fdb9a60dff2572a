// One row of the pack: the quantiser shared by the pack kernels and the
// attention kernel's fused pack (sm_100a).
#pragma once

#include "dkv_common.cuh"

namespace dkv {

// Quantises part `part` (dims 8*part .. 8*part+7) of one 64-wide row held in
// `raw` (8 bf16) and stores it at pool row index `at` (pool_row of its block and
// row). The eight lanes of a row must call it together (row min/max by shuffles
// within the 8-lane group).
template <int BITS>
__device__ __forceinline__ void pack_row_part(uint4 raw, int part, uint8_t* p4, float2* m4, uint8_t* p8,
                                              float2* m8, uint16_t* p16, int64_t at, int32_t* status,
                                              int report_row) {
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
    reinterpret_cast<uint4*>(p16 + at * kDim)[part] = raw;
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
    reinterpret_cast<uint2*>(p8 + at * kRowBytes8)[part] = w;
    if (part == 0) m8[at] = make_float2(offset, scale);
  } else {
    uint32_t w = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) w |= (q[2 * j] | (q[2 * j + 1] << 4)) << (8 * j);
    reinterpret_cast<uint32_t*>(p4 + at * kRowBytes4)[part] = w;
    if (part == 0) m4[at] = make_float2(offset, scale);
  }
}

// Whether a pack destination can take an n-token frame: a precision of 4, 8 or
// 16 with that pool present and rows [row_start, row_start + n) inside it.
__device__ __forceinline__ bool pack_target_ok(const dkv_pack_target& d, int n) {
  const int bits = d.bits;
  if (bits != 4 && bits != 8 && bits != 16) return false;
  const bool pool = bits == 4 ? (d.p4 != nullptr && d.m4 != nullptr)
                              : (bits == 8 ? (d.p8 != nullptr && d.m8 != nullptr) : d.p16 != nullptr);
  const int64_t cap = bits == 4 ? d.cap4 : (bits == 8 ? d.cap8 : d.cap16);
  return pool && d.row_start >= 0 && d.row_start + n <= cap;
}

__device__ __forceinline__ void report_bad_target(const dkv_pack_target& d, int n, int index) {
  const bool bits_ok = d.bits == 4 || d.bits == 8 || d.bits == 16;
  report(d.status, bits_ok && d.row_start >= 0 ? DKV_ECAPACITY : DKV_EINVAL, index);
}

// Packs part `part` of row (kv, head, token) of an n-token frame k / v (bf16
// [heads, n, 64], strides (kh, kt) and (vh, vt)) into destination d, which
// pack_target_ok accepted, whose pools hold `blocks` = layers * 2 * heads blocks;
// with a token map in d, the K row of head 0 also writes the map entry of its
// token. The eight lanes of a row call it together.
__device__ __forceinline__ void pack_frame_row(const dkv_pack_target& d, const uint16_t* k, const uint16_t* v,
                                               int64_t kh, int64_t kt, int64_t vh, int64_t vt, int layer, int n,
                                               int heads, int blocks, int kv, int head, int token, int part,
                                               int report_row) {
  const uint16_t* src = kv == 0 ? k + head * kh + token * kt : v + head * vh + token * vt;
  const uint4 raw = __ldg(reinterpret_cast<const uint4*>(src) + part);
  const int64_t block = (static_cast<int64_t>(layer) * 2 + kv) * heads + head;
  const int64_t out_row = d.row_start + token;
  const int64_t at = pool_row(block, out_row, blocks);
  uint8_t* p4 = static_cast<uint8_t*>(d.p4);
  uint8_t* p8 = static_cast<uint8_t*>(d.p8);
  float2* m4 = static_cast<float2*>(d.m4);
  float2* m8 = static_cast<float2*>(d.m8);
  uint16_t* p16 = static_cast<uint16_t*>(d.p16);
  if (d.bits == 4) {
    pack_row_part<4>(raw, part, p4, m4, p8, m8, p16, at, d.status, report_row);
  } else if (d.bits == 8) {
    pack_row_part<8>(raw, part, p4, m4, p8, m8, p16, at, d.status, report_row);
  } else {
    pack_row_part<16>(raw, part, p4, m4, p8, m8, p16, at, d.status, report_row);
  }
  if (d.map_rows != nullptr && kv == 0 && head == 0 && part == 0) {
    if (d.map_codes == nullptr || d.map_start < 0 || d.map_start + n > d.map_capacity) {
      report(d.status, DKV_ECAPACITY, token);
    } else {
      d.map_rows[d.map_start + token] = static_cast<int32_t>(out_row);
      d.map_codes[d.map_start + token] = static_cast<uint8_t>(d.bits);
    }
  }
}

// Row `row` of the frame in pack-kernel order: K rows of every head, then V rows,
// token fastest.
__device__ __forceinline__ void pack_target_row(const dkv_pack_target& d, const uint16_t* k, const uint16_t* v,
                                                int64_t kh, int64_t kt, int64_t vh, int64_t vt, int layer, int n,
                                                int heads, int blocks, int row, int part) {
  const int per_kv = heads * n;
  const int kv = row / per_kv;
  const int rem = row - kv * per_kv;
  const int head = rem / n;
  pack_frame_row(d, k, v, kh, kt, vh, vt, layer, n, heads, blocks, kv, head, rem - head * n, part, row);
}

}  // namespace dkv
