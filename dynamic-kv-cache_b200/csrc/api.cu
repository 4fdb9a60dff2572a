// extern "C" entry points of libdkv.so (declared in include/dkv.h).
// Host-side argument validation mirrors the reference's ValueError conditions;
// nothing here allocates, synchronises or retains pointers.
#include <cstdarg>
#include <cstddef>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <utility>

#include "attention.cuh"

namespace dkv {
cudaError_t launch_pack(const void* k, const void* v, void* p4, void* m4, void* p8, void* m8,
                        void* p16, int64_t kh, int64_t kt, int64_t vh, int64_t vt, int layer,
                        int64_t row_start, int n, int blocks, int heads, int bits,
                        int32_t* status, cudaStream_t stream);
cudaError_t launch_reconstruct(const Pools& P, const int32_t* rows, const uint8_t* codes, void* out,
                               int layer, int n, int32_t* status, cudaStream_t stream);
cudaError_t launch_map_fill(int32_t* rows, uint8_t* codes, int64_t start, int n, int64_t row, int bits,
                            cudaStream_t stream);
cudaError_t launch_rotary(const void* x, const float* cos_t, const float* sin_t, void* out, int64_t xb, int64_t xt,
                          int64_t cb, int b, int n, int heads, cudaStream_t stream);
cudaError_t launch_silu_mul(const void* gate, const void* up, void* out, int64_t gs, int64_t us, int64_t rows,
                            int width, cudaStream_t stream);
cudaError_t launch_add_rms_norm(const void* x, const void* y, void* x_out, void* h_out, const void* weight,
                                int64_t rows, int width, int64_t xs, int64_t ys, int64_t os, int64_t hs, float eps,
                                cudaStream_t stream);
cudaError_t launch_pack_many(const void* k, const void* v, const dkv_pack_target* targets, bool on_device, int count,
                             int64_t kh, int64_t kt, int64_t vh, int64_t vt, int64_t kc, int64_t vc, int layer, int n,
                             int heads, int blocks, cudaStream_t stream);
}  // namespace dkv

// The request descriptors cross the C ABI by layout: keep it fixed (the Python
// binding declares the same fields in the same order).
static_assert(sizeof(dkv_history) == 96 && offsetof(dkv_history, past) == 80 &&
                  offsetof(dkv_history, capacity) == 84 && offsetof(dkv_history, status) == 88,
              "dkv_history layout");
static_assert(sizeof(dkv_pack_target) == 120 && offsetof(dkv_pack_target, bits) == 72 &&
                  offsetof(dkv_pack_target, map_rows) == 80 && offsetof(dkv_pack_target, status) == 112,
              "dkv_pack_target layout");
static_assert(sizeof(dkv::HistoryTable) + sizeof(dkv::AttnArgs) <= 4096, "attention kernel parameters");

namespace {

thread_local char g_error[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_error, sizeof(g_error), fmt, ap);
  va_end(ap);
  return code;
}

int ok() {
  g_error[0] = '\0';
  return DKV_OK;
}

int cuda_status(cudaError_t e, const char* what) {
  if (e != cudaSuccess) return fail(DKV_ECUDA, "%s: %s", what, cudaGetErrorString(e));
  return ok();
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// bf16 [1, heads, n, 64] operand with 16-byte aligned rows.
bool rows_aligned(const void* p, int64_t hs, int64_t ts) {
  return p != nullptr && aligned16(p) && (hs % 8) == 0 && (ts % 8) == 0;
}

int check_geometry(int32_t heads, int32_t dim, int32_t layers, int32_t layer) {
  if (dim != dkv::kDim) return fail(DKV_EINVAL, "GPU kernel currently supports head_dim=64");
  if (heads <= 0 || layers <= 0) return fail(DKV_EINVAL, "heads and layers must be positive");
  if (static_cast<int64_t>(layers) * 2 * heads > (1 << 24)) return fail(DKV_EINVAL, "too many layers x heads");
  if (layer < 0 || layer >= layers) return fail(DKV_EINVAL, "layer %d outside [0, %d)", layer, layers);
  return DKV_OK;
}

int check_pools(const void* p4, const void* m4, const void* p8, const void* m8, const void* p16,
                int64_t cap4, int64_t cap8, int64_t cap16) {
  if (!p4 || !m4 || !p8 || !m8 || !p16) return fail(DKV_EINVAL, "null pool pointer");
  if (!aligned16(p4) || !aligned16(p8) || !aligned16(p16) || !aligned16(m4) || !aligned16(m8))
    return fail(DKV_EINVAL, "pools must be 16-byte aligned");
  if (cap4 <= 0 || cap8 <= 0 || cap16 <= 0) return fail(DKV_EINVAL, "pool capacities must be positive");
  if (cap4 > INT32_MAX || cap8 > INT32_MAX || cap16 > INT32_MAX)
    return fail(DKV_EINVAL, "pool capacity exceeds int32 row index");
  return DKV_OK;
}

}  // namespace

namespace dkv {
int set_last_error(int code, const char* message) { return fail(code, "%s", message); }
int api_fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_error, sizeof(g_error), fmt, ap);
  va_end(ap);
  return code;
}
int api_ok() { return ok(); }
}  // namespace dkv

namespace {

// What the last launch of this library on each (device, stream) wrote that an
// attention call may read as history: nothing, one layer's pool rows, or token
// maps (read by every layer). Every kernel here releases its programmatic
// dependents only after its own griddepcontrol.wait, so when a kernel starts,
// every kernel launched two or more before it on its stream has completed: only
// the immediately preceding one may still be writing. An attention call streams
// its history before its own wait unless that preceding launch wrote this layer's
// rows or the maps (then it waits first). Kernels of other libraries launched in
// between only make this conservative: they are either ordinary launches (which
// start after everything before them completed) or, if programmatic, must not
// release their dependents before their own wait either.
constexpr int kWroteNothing = -1;
constexpr int kWroteMaps = -2;
std::mutex g_write_mu;
std::map<std::pair<int, const void*>, int> g_last_write;

std::pair<int, const void*> stream_key(void* stream) {
  int dev = -1;
  cudaGetDevice(&dev);
  return {dev, stream};
}

int last_write(void* stream) {
  const auto key = stream_key(stream);
  std::lock_guard<std::mutex> lock(g_write_mu);
  const auto it = g_last_write.find(key);
  return it == g_last_write.end() ? kWroteNothing : it->second;
}

// Records what a launch that succeeded on `stream` wrote; passes `rc` through.
int note_write(void* stream, int wrote, int rc) {
  if (rc == DKV_OK) {
    const auto key = stream_key(stream);
    std::lock_guard<std::mutex> lock(g_write_mu);
    g_last_write[key] = wrote;
  }
  return rc;
}

bool history_may_be_fresh(void* stream, int layer) {
  const int w = last_write(stream);
  return w == kWroteMaps || w == layer;
}

}  // namespace

extern "C" {

int32_t dkv_version(void) { return DKV_VERSION; }

const char* dkv_last_error(void) { return g_error; }

int dkv_pack_rows(const void* k, const void* v, void* p4, void* m4, void* p8, void* m8, void* p16,
                  int64_t kh, int64_t kt, int64_t vh, int64_t vt, int32_t layer, int64_t row_start,
                  int32_t n, int64_t cap4, int64_t cap8, int64_t cap16, int32_t heads, int32_t dim,
                  int32_t bits, int32_t layers, int32_t* status, void* stream) {
  int rc = check_geometry(heads, dim, layers, layer);
  if (rc) return rc;
  if ((rc = check_pools(p4, m4, p8, m8, p16, cap4, cap8, cap16))) return rc;
  if (bits != 4 && bits != 8 && bits != 16) return fail(DKV_EINVAL, "Supported bit widths: 4, 8, 16");
  if (n < 0) return fail(DKV_EINVAL, "negative token count");
  if (n == 0) return ok();
  if (!rows_aligned(k, kh, kt) || !rows_aligned(v, vh, vt))
    return fail(DKV_EINVAL, "k/v rows must be 16-byte aligned (head/token strides multiples of 8)");
  const int64_t cap = bits == 4 ? cap4 : (bits == 8 ? cap8 : cap16);
  if (row_start < 0 || row_start + n > cap)
    return fail(DKV_ECAPACITY, "rows [%lld, %lld) exceed the %d-bit pool capacity %lld",
                (long long)row_start, (long long)(row_start + n), bits, (long long)cap);
  if (2LL * heads * n * 8 > INT32_MAX) return fail(DKV_EINVAL, "frame too large");
  return note_write(stream, layer,
                    cuda_status(dkv::launch_pack(k, v, p4, m4, p8, m8, p16, kh, kt, vh, vt, layer, row_start, n,
                                                 layers * 2 * heads, heads, bits, status,
                                                 static_cast<cudaStream_t>(stream)),
                                "pack_rows launch"));
}

size_t dkv_packed_attention_workspace(int32_t past, int32_t nq, int32_t heads, int32_t group, int32_t dim) {
  return dkv_packed_attention_batched_workspace(past, nq, heads, group, dim, 1);
}

size_t dkv_packed_attention_batched_workspace(int32_t past, int32_t nq, int32_t heads, int32_t group, int32_t dim,
                                              int32_t chunks) {
  if (past < 0 || nq <= 0 || heads <= 0 || group <= 0 || dim != dkv::kDim || chunks <= 0) return 0;
  if (static_cast<int64_t>(group) * nq <= dkv::kSplitRows) return 0;  // split-K kernel: merges in its clusters
  return dkv::make_plan(past, nq, heads, group, chunks).workspace_bytes();
}

int32_t dkv_packed_attention_launches(int32_t past, int32_t nq, int32_t heads, int32_t group, int32_t dim) {
  if (past < 0 || nq <= 0 || heads <= 0 || group <= 0 || dim != dkv::kDim) return 0;
  if (static_cast<int64_t>(group) * nq <= dkv::kSplitRows) return 1;  // split-K kernel
  const dkv::AttnPlan p = dkv::make_plan(past, nq, heads, group);
  if (p.splits == 1) return 1;
  bool fused = false;
  if (dkv::attention_tc_merges_in_kernel(p, heads, true, &fused) != cudaSuccess) return -1;
  return fused ? 1 : 2;
}

}  // extern "C"

namespace {

// Fills the call-wide fields of `a` (its history is set by the caller) and
// launches the planned kernels: attention, then the combine when the splits are
// not merged in the attention kernel.
int launch_planned(dkv::AttnArgs& a, const dkv::AttnPlan& p, const void* q, const void* knew, const void* vnew,
                   void* out, int64_t qh, int64_t qt, int64_t kh, int64_t kt, int64_t vh, int64_t vt, int32_t chunks,
                   int64_t qc, int64_t kc, int64_t vc, int64_t oc, int32_t layer, int32_t nq, int32_t heads,
                   int32_t group, int32_t layers, void* workspace, void* stream, const dkv::HistoryTable* table,
                   const dkv_history* device_table = nullptr, const dkv_pack_target* pack = nullptr,
                   bool pack_on_device = false, bool split = false) {
  a.q = static_cast<const uint16_t*>(q);
  a.knew = static_cast<const uint16_t*>(knew);
  a.vnew = static_cast<const uint16_t*>(vnew);
  a.out = static_cast<uint16_t*>(out);
  a.qh = qh; a.qt = qt; a.kh = kh; a.kt = kt; a.vh = vh; a.vt = vt;
  a.qc = qc; a.kc = kc; a.vc = vc; a.oc = oc;
  a.layer = layer;
  a.nq = nq;
  a.heads = heads;
  a.G = group;
  a.HQ = heads * group;
  a.blocks = layers * 2 * heads;
  a.mrows = p.mrows;
  a.cta_rows = p.cta_rows;
  a.mblocks = p.mblocks;
  a.splits = p.splits;
  a.chunk = p.chunk;
  if (!split && p.workspace_bytes() > 0) {  // [merge counters][partial outputs][partial (max, sum)]
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    a.sync = reinterpret_cast<uint32_t*>(ws);
    a.ws_o = reinterpret_cast<float*>(ws + dkv::kSyncBytes);
    a.ws_ml = reinterpret_cast<float2*>(ws + dkv::kSyncBytes + p.ws_o_bytes);
  }
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int zdim = heads * chunks;  // grid z: chunk * heads + KV head
  if (pack != nullptr) {  // append + attend: the attention kernel packs the frame too
    if (pack_on_device) {
      a.pack_mode = 2;
      a.pack_table = pack;
    } else if (chunks == 1) {
      a.pack_mode = 1;
      a.pack = *pack;
    } else {
      return fail(DKV_EINVAL, "a pack destination by value serves one request");
    }
  }
  a.hist_wait = history_may_be_fresh(stream, layer) ? 1 : 0;
  cudaError_t e = split ? dkv::launch_attention_split(a, zdim, st) : dkv::launch_attention_tc(a, zdim, st, table, device_table);
  const bool combine = !split && p.splits > 1 && !a.fused;
  if (e == cudaSuccess && combine) e = dkv::launch_attention_combine(a, zdim, st);
  // A fused pack runs after the attention kernel has released its dependents; a
  // combine launch after it completes it first.
  int wrote = kWroteNothing;
  if (pack != nullptr && !combine) wrote = (pack_on_device || pack->map_rows != nullptr) ? kWroteMaps : layer;
  return note_write(stream, wrote, cuda_status(e, "packed_attention launch"));
}

int attention_impl(const void* q, const void* knew, const void* vnew, const void* p4, const void* m4,
                   const void* p8, const void* m8, const void* p16, const int32_t* rows, const uint8_t* codes,
                   void* out, int64_t qh, int64_t qt, int64_t kh, int64_t kt, int64_t vh, int64_t vt, int32_t chunks,
                   int64_t qc, int64_t kc, int64_t vc, int64_t oc, int32_t layer, int32_t past, int32_t nq,
                   int64_t cap4, int64_t cap8, int64_t cap16, int32_t heads, int32_t group, int32_t dim,
                   int32_t block_m, int32_t block_n, int32_t layers, void* workspace, size_t workspace_bytes,
                   int32_t* status, void* stream, const dkv_pack_target* pack = nullptr) {
  int rc = check_geometry(heads, dim, layers, layer);
  if (rc) return rc;
  if ((rc = check_pools(p4, m4, p8, m8, p16, cap4, cap8, cap16))) return rc;
  if (group <= 0) return fail(DKV_EINVAL, "query heads must be a positive multiple of KV heads");
  auto pow2 = [](int x) { return x >= 16 && x <= 256 && (x & (x - 1)) == 0; };
  if (!pow2(block_m) || !pow2(block_n)) return fail(DKV_EINVAL, "block_m/block_n must be powers of two in [16, 256]");
  if (past < 0 || nq < 0) return fail(DKV_EINVAL, "negative past or query length");
  if (chunks <= 0 || static_cast<int64_t>(chunks) * heads > 65535) return fail(DKV_EINVAL, "chunk count out of range");
  if (chunks > 1 && ((qc % 8) || (kc % 8) || (vc % 8) || (oc % 8)))
    return fail(DKV_EINVAL, "chunk strides must keep rows 16-byte aligned (multiples of 8 elements)");
  if (nq == 0) return ok();
  if (past > 0 && (rows == nullptr || codes == nullptr)) return fail(DKV_EINVAL, "null token map");
  if (past > 0 && (!aligned16(rows) || !aligned16(codes)))
    return fail(DKV_EINVAL, "token maps must be 16-byte aligned");
  if (!rows_aligned(q, qh, qt) || !rows_aligned(knew, kh, kt) || !rows_aligned(vnew, vh, vt))
    return fail(DKV_EINVAL, "q/k/v rows must be 16-byte aligned (head/token strides multiples of 8)");
  if (out == nullptr || !aligned16(out)) return fail(DKV_EINVAL, "out must be 16-byte aligned");
  // short chunks (decode steps, small candidate chunks) take the split-K kernel
  const bool split = static_cast<int64_t>(group) * nq <= dkv::kSplitRows;
  const dkv::AttnPlan p = split ? dkv::make_plan_split(past, nq, heads, group, chunks)
                                : dkv::make_plan(past, nq, heads, group, chunks);
  const size_t need = split ? 0 : p.workspace_bytes();
  if (need > 0 && (workspace == nullptr || workspace_bytes < need))
    return fail(DKV_EWORKSPACE, "attention workspace needs %zu bytes, got %zu", need, workspace_bytes);
  if (need > 0 && (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return fail(DKV_EWORKSPACE, "attention workspace must be 256-byte aligned");
  dkv::AttnArgs a{};
  a.hist = dkv_history{p4, m4, p8, m8, p16, rows, codes, cap4, cap8, cap16, past, past, status};
  return launch_planned(a, p, q, knew, vnew, out, qh, qt, kh, kt, vh, vt, chunks, qc, kc, vc, oc, layer, nq, heads,
                        group, layers, workspace, stream, nullptr, nullptr, pack, false, split);
}

}  // namespace

extern "C" {

int dkv_packed_attention(const void* q, const void* knew, const void* vnew, const void* p4, const void* m4,
                         const void* p8, const void* m8, const void* p16, const int32_t* rows,
                         const uint8_t* codes, void* out, int64_t qh, int64_t qt, int64_t kh, int64_t kt,
                         int64_t vh, int64_t vt, int32_t layer, int32_t past, int32_t nq, int64_t cap4,
                         int64_t cap8, int64_t cap16, int32_t heads, int32_t group, int32_t dim,
                         int32_t block_m, int32_t block_n, int32_t layers, void* workspace,
                         size_t workspace_bytes, int32_t* status, void* stream) {
  return attention_impl(q, knew, vnew, p4, m4, p8, m8, p16, rows, codes, out, qh, qt, kh, kt, vh, vt, 1, 0, 0, 0, 0,
                        layer, past, nq, cap4, cap8, cap16, heads, group, dim, block_m, block_n, layers, workspace,
                        workspace_bytes, status, stream);
}

int dkv_packed_attention_batched(const void* q, const void* knew, const void* vnew, const void* p4, const void* m4,
                                 const void* p8, const void* m8, const void* p16, const int32_t* rows,
                                 const uint8_t* codes, void* out, int64_t qh, int64_t qt, int64_t kh, int64_t kt,
                                 int64_t vh, int64_t vt, int32_t chunks, int64_t qc, int64_t kc, int64_t vc,
                                 int64_t oc, int32_t layer, int32_t past, int32_t nq, int64_t cap4, int64_t cap8,
                                 int64_t cap16, int32_t heads, int32_t group, int32_t dim, int32_t block_m,
                                 int32_t block_n, int32_t layers, void* workspace, size_t workspace_bytes,
                                 int32_t* status, void* stream) {
  return attention_impl(q, knew, vnew, p4, m4, p8, m8, p16, rows, codes, out, qh, qt, kh, kt, vh, vt, chunks, qc, kc,
                        vc, oc, layer, past, nq, cap4, cap8, cap16, heads, group, dim, block_m, block_n, layers,
                        workspace, workspace_bytes, status, stream);
}

int dkv_pack_rows_many(const void* k, const void* v, const dkv_pack_target* targets, int32_t count, int64_t kh,
                       int64_t kt, int64_t vh, int64_t vt, int64_t kc, int64_t vc, int32_t layer, int32_t n,
                       int32_t heads, int32_t dim, int32_t layers, void* stream) {
  int rc = check_geometry(heads, dim, layers, layer);
  if (rc) return rc;
  if (count <= 0 || count > DKV_MAX_REQUESTS)
    return fail(DKV_EINVAL, "request count %d outside [1, %d]", count, DKV_MAX_REQUESTS);
  if (targets == nullptr) return fail(DKV_EINVAL, "null request table");
  if (n < 0) return fail(DKV_EINVAL, "negative token count");
  if (!rows_aligned(k, kh, kt) || !rows_aligned(v, vh, vt) || (kc % 8) || (vc % 8))
    return fail(DKV_EINVAL, "k/v rows must be 16-byte aligned (strides multiples of 8)");
  if (2LL * heads * n * 8 > INT32_MAX) return fail(DKV_EINVAL, "frame too large");
  for (int r = 0; r < count; ++r) {
    const dkv_pack_target& t = targets[r];
    if ((rc = check_pools(t.p4, t.m4, t.p8, t.m8, t.p16, t.cap4, t.cap8, t.cap16))) return rc;
    if (t.bits != 4 && t.bits != 8 && t.bits != 16) return fail(DKV_EINVAL, "Supported bit widths: 4, 8, 16");
    const int64_t cap = t.bits == 4 ? t.cap4 : (t.bits == 8 ? t.cap8 : t.cap16);
    if (t.row_start < 0 || t.row_start + n > cap)
      return fail(DKV_ECAPACITY, "request %d: rows [%lld, %lld) exceed the %d-bit pool capacity %lld", r,
                  (long long)t.row_start, (long long)(t.row_start + n), t.bits, (long long)cap);
    if (t.row_start + n > INT32_MAX) return fail(DKV_ECAPACITY, "pool row exceeds int32");
    if ((t.map_rows == nullptr) != (t.map_codes == nullptr)) return fail(DKV_EINVAL, "half a token map");
    if (t.map_rows != nullptr && (t.map_start < 0 || t.map_start + n > t.map_capacity))
      return fail(DKV_ECAPACITY, "GPU context limit exceeded");
  }
  if (n == 0) return ok();
  bool maps = false;
  for (int r = 0; r < count; ++r) maps = maps || targets[r].map_rows != nullptr;
  return note_write(stream, maps ? kWroteMaps : layer,
                    cuda_status(dkv::launch_pack_many(k, v, targets, false, count, kh, kt, vh, vt, kc, vc, layer, n,
                                                      heads, layers * 2 * heads, static_cast<cudaStream_t>(stream)),
                                "pack_rows_many launch"));
}

int dkv_pack_rows_many_device(const void* k, const void* v, const dkv_pack_target* targets, int32_t count,
                              int64_t kh, int64_t kt, int64_t vh, int64_t vt, int64_t kc, int64_t vc, int32_t layer,
                              int32_t n, int32_t heads, int32_t dim, int32_t layers, void* stream) {
  int rc = check_geometry(heads, dim, layers, layer);
  if (rc) return rc;
  if (count <= 0 || count > 65535) return fail(DKV_EINVAL, "request count %d outside [1, 65535]", count);
  if (targets == nullptr || !aligned16(targets)) return fail(DKV_EINVAL, "device request table must be 16-byte aligned");
  if (n < 0) return fail(DKV_EINVAL, "negative token count");
  if (!rows_aligned(k, kh, kt) || !rows_aligned(v, vh, vt) || (kc % 8) || (vc % 8))
    return fail(DKV_EINVAL, "k/v rows must be 16-byte aligned (strides multiples of 8)");
  if (2LL * heads * n * 8 > INT32_MAX) return fail(DKV_EINVAL, "frame too large");
  if (n == 0) return ok();
  return note_write(stream, kWroteMaps,  // device targets may update the maps
                    cuda_status(dkv::launch_pack_many(k, v, targets, true, count, kh, kt, vh, vt, kc, vc, layer, n,
                                                      heads, layers * 2 * heads, static_cast<cudaStream_t>(stream)),
                                "pack_rows_many_device launch"));
}

size_t dkv_packed_attention_many_workspace(int32_t max_past, int32_t nq, int32_t heads, int32_t group, int32_t dim,
                                           int32_t count) {
  if (count <= 0 || count > 65535 || max_past < 0 || nq <= 0 || heads <= 0 || group <= 0 || dim != dkv::kDim)
    return 0;
  return dkv::make_plan_many(max_past, nq, heads, group, count).workspace_bytes();
}

// Shared checks and launch of the two many-request attention entry points.
static int attention_many_launch(const void* q, const void* knew, const void* vnew, const dkv::HistoryTable* table,
                          const dkv_history* device_table, int32_t count, int32_t max_past, void* out, int64_t qh,
                          int64_t qt, int64_t kh, int64_t kt, int64_t vh, int64_t vt, int64_t qc, int64_t kc,
                          int64_t vc, int64_t oc, int32_t layer, int32_t nq, int32_t heads, int32_t group,
                          int32_t layers, void* workspace, size_t workspace_bytes, void* stream,
                          const dkv_pack_target* device_pack = nullptr) {
  if (nq == 0) return ok();
  if (!rows_aligned(q, qh, qt) || !rows_aligned(knew, kh, kt) || !rows_aligned(vnew, vh, vt))
    return fail(DKV_EINVAL, "q/k/v rows must be 16-byte aligned (head/token strides multiples of 8)");
  if (out == nullptr || !aligned16(out)) return fail(DKV_EINVAL, "out must be 16-byte aligned");
  if (static_cast<int64_t>(count) * heads > 65535) return fail(DKV_EINVAL, "chunk count out of range");
  const dkv::AttnPlan p = dkv::make_plan_many(max_past, nq, heads, group, count);
  const size_t need = p.workspace_bytes();
  if (need > 0 && (workspace == nullptr || workspace_bytes < need))
    return fail(DKV_EWORKSPACE, "attention workspace needs %zu bytes, got %zu", need, workspace_bytes);
  if (need > 0 && (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0)
    return fail(DKV_EWORKSPACE, "attention workspace must be 256-byte aligned");
  if (2LL * heads * nq * 8 > INT32_MAX) return fail(DKV_EINVAL, "frame too large");
  dkv::AttnArgs a{};
  return launch_planned(a, p, q, knew, vnew, out, qh, qt, kh, kt, vh, vt, count, qc, kc, vc, oc, layer, nq, heads,
                        group, layers, workspace, stream, table, device_table, device_pack, device_pack != nullptr);
}

int dkv_packed_attention_many(const void* q, const void* knew, const void* vnew, const dkv_history* requests,
                              int32_t count, void* out, int64_t qh, int64_t qt, int64_t kh, int64_t kt, int64_t vh,
                              int64_t vt, int64_t qc, int64_t kc, int64_t vc, int64_t oc, int32_t layer, int32_t nq,
                              int32_t heads, int32_t group, int32_t dim, int32_t layers, void* workspace,
                              size_t workspace_bytes, void* stream) {
  int rc = check_geometry(heads, dim, layers, layer);
  if (rc) return rc;
  if (count <= 0 || count > DKV_MAX_REQUESTS)
    return fail(DKV_EINVAL, "request count %d outside [1, %d]", count, DKV_MAX_REQUESTS);
  if (requests == nullptr) return fail(DKV_EINVAL, "null request table");
  if (group <= 0) return fail(DKV_EINVAL, "query heads must be a positive multiple of KV heads");
  if (nq < 0) return fail(DKV_EINVAL, "negative past or query length");
  if ((qc % 8) || (kc % 8) || (vc % 8) || (oc % 8))
    return fail(DKV_EINVAL, "chunk strides must keep rows 16-byte aligned (multiples of 8 elements)");
  dkv::HistoryTable table{};
  int max_past = 0;
  for (int r = 0; r < count; ++r) {
    const dkv_history& h = requests[r];
    if ((rc = check_pools(h.p4, h.m4, h.p8, h.m8, h.p16, h.cap4, h.cap8, h.cap16))) return rc;
    if (h.past < 0) return fail(DKV_EINVAL, "negative past or query length");
    if (h.past > h.capacity) return fail(DKV_EINVAL, "request %d: past %d exceeds its token map (%d)", r, h.past,
                                         h.capacity);
    if (h.past > 0 && (h.rows == nullptr || h.codes == nullptr)) return fail(DKV_EINVAL, "null token map");
    if (h.past > 0 && (!aligned16(h.rows) || !aligned16(h.codes)))
      return fail(DKV_EINVAL, "token maps must be 16-byte aligned");
    table.h[r] = h;
    max_past = h.past > max_past ? h.past : max_past;
  }
  return attention_many_launch(q, knew, vnew, &table, nullptr, count, max_past, out, qh, qt, kh, kt, vh, vt, qc, kc,
                               vc, oc, layer, nq, heads, group, layers, workspace, workspace_bytes, stream);
}

int dkv_packed_attention_many_device(const void* q, const void* knew, const void* vnew, const dkv_history* requests,
                                     int32_t count, int32_t max_past, void* out, int64_t qh, int64_t qt, int64_t kh,
                                     int64_t kt, int64_t vh, int64_t vt, int64_t qc, int64_t kc, int64_t vc,
                                     int64_t oc, int32_t layer, int32_t nq, int32_t heads, int32_t group,
                                     int32_t dim, int32_t layers, void* workspace, size_t workspace_bytes,
                                     void* stream) {
  int rc = check_geometry(heads, dim, layers, layer);
  if (rc) return rc;
  if (count <= 0 || count > 65535) return fail(DKV_EINVAL, "request count %d outside [1, 65535]", count);
  if (requests == nullptr || !aligned16(requests))
    return fail(DKV_EINVAL, "device request table must be 16-byte aligned");
  if (group <= 0) return fail(DKV_EINVAL, "query heads must be a positive multiple of KV heads");
  if (nq < 0 || max_past < 0) return fail(DKV_EINVAL, "negative past or query length");
  if ((qc % 8) || (kc % 8) || (vc % 8) || (oc % 8))
    return fail(DKV_EINVAL, "chunk strides must keep rows 16-byte aligned (multiples of 8 elements)");
  return attention_many_launch(q, knew, vnew, nullptr, requests, count, max_past, out, qh, qt, kh, kt, vh, vt, qc, kc,
                               vc, oc, layer, nq, heads, group, layers, workspace, workspace_bytes, stream);
}

int dkv_append_attention(const void* q, const void* knew, const void* vnew, void* p4, void* m4, void* p8, void* m8,
                         void* p16, int32_t* rows, uint8_t* codes, void* out, int64_t qh, int64_t qt, int64_t kh,
                         int64_t kt, int64_t vh, int64_t vt, int32_t layer, int32_t past, int32_t nq,
                         int64_t row_start, int32_t bits, int32_t fill_map, int64_t map_capacity, int64_t cap4,
                         int64_t cap8, int64_t cap16, int32_t heads, int32_t group, int32_t dim, int32_t block_m,
                         int32_t block_n, int32_t layers, void* workspace, size_t workspace_bytes, int32_t* status,
                         void* stream) {
  int rc = check_geometry(heads, dim, layers, layer);
  if (rc) return rc;
  if ((rc = check_pools(p4, m4, p8, m8, p16, cap4, cap8, cap16))) return rc;
  if (bits != 4 && bits != 8 && bits != 16) return fail(DKV_EINVAL, "Supported bit widths: 4, 8, 16");
  if (nq < 0 || past < 0) return fail(DKV_EINVAL, "negative past or query length");
  const int64_t cap = bits == 4 ? cap4 : (bits == 8 ? cap8 : cap16);
  if (row_start < 0 || row_start + nq > cap)
    return fail(DKV_ECAPACITY, "rows [%lld, %lld) exceed the %d-bit pool capacity %lld", (long long)row_start,
                (long long)(row_start + nq), bits, (long long)cap);
  if (row_start + nq > INT32_MAX) return fail(DKV_ECAPACITY, "pool row exceeds int32");
  if (fill_map && (rows == nullptr || codes == nullptr)) return fail(DKV_EINVAL, "null token map");
  if (fill_map && past + static_cast<int64_t>(nq) > map_capacity)
    return fail(DKV_ECAPACITY, "GPU context limit exceeded");
  if (2LL * heads * nq * 8 > INT32_MAX) return fail(DKV_EINVAL, "frame too large");
  const dkv_pack_target t{p4, m4, p8, m8, p16, cap4, cap8, cap16, row_start, bits, 0,
                          fill_map ? rows : nullptr, fill_map ? codes : nullptr, past, map_capacity, status};
  return attention_impl(q, knew, vnew, p4, m4, p8, m8, p16, rows, codes, out, qh, qt, kh, kt, vh, vt, 1, 0, 0, 0, 0,
                        layer, past, nq, cap4, cap8, cap16, heads, group, dim, block_m, block_n, layers, workspace,
                        workspace_bytes, status, stream, &t);
}

int dkv_append_attention_many_device(const void* q, const void* knew, const void* vnew,
                                     const dkv_pack_target* targets, const dkv_history* requests, int32_t count,
                                     int32_t max_past, void* out, int64_t qh, int64_t qt, int64_t kh, int64_t kt,
                                     int64_t vh, int64_t vt, int64_t qc, int64_t kc, int64_t vc, int64_t oc,
                                     int32_t layer, int32_t nq, int32_t heads, int32_t group, int32_t dim,
                                     int32_t layers, void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_geometry(heads, dim, layers, layer);
  if (rc) return rc;
  if (count <= 0 || count > 65535) return fail(DKV_EINVAL, "request count %d outside [1, 65535]", count);
  if (requests == nullptr || !aligned16(requests) || targets == nullptr || !aligned16(targets))
    return fail(DKV_EINVAL, "device request tables must be 16-byte aligned");
  if (group <= 0) return fail(DKV_EINVAL, "query heads must be a positive multiple of KV heads");
  if (nq < 0 || max_past < 0) return fail(DKV_EINVAL, "negative past or query length");
  if ((qc % 8) || (kc % 8) || (vc % 8) || (oc % 8))
    return fail(DKV_EINVAL, "chunk strides must keep rows 16-byte aligned (multiples of 8 elements)");
  return attention_many_launch(q, knew, vnew, nullptr, requests, count, max_past, out, qh, qt, kh, kt, vh, vt, qc, kc,
                               vc, oc, layer, nq, heads, group, layers, workspace, workspace_bytes, stream, targets);
}

int dkv_reconstruct(const void* p4, const void* m4, const void* p8, const void* m8, const void* p16,
                    const int32_t* rows, const uint8_t* codes, void* out, int32_t layer, int32_t n,
                    int64_t cap4, int64_t cap8, int64_t cap16, int32_t heads, int32_t dim, int32_t layers,
                    int32_t* status, void* stream) {
  int rc = check_geometry(heads, dim, layers, layer);
  if (rc) return rc;
  if ((rc = check_pools(p4, m4, p8, m8, p16, cap4, cap8, cap16))) return rc;
  if (n < 0) return fail(DKV_EINVAL, "negative token count");
  if (n == 0) return ok();
  if (rows == nullptr || codes == nullptr) return fail(DKV_EINVAL, "null token map");
  if (out == nullptr || !aligned16(out)) return fail(DKV_EINVAL, "out must be 16-byte aligned");
  if (2LL * heads * n * 8 > INT32_MAX) return fail(DKV_EINVAL, "history too large");
  dkv::Pools P{static_cast<const uint8_t*>(p4), static_cast<const float2*>(m4),
               static_cast<const uint8_t*>(p8), static_cast<const float2*>(m8),
               static_cast<const uint16_t*>(p16), cap4, cap8, cap16, heads, layers * 2 * heads};
  return note_write(stream, kWroteNothing,
                    cuda_status(dkv::launch_reconstruct(P, rows, codes, out, layer, n, status,
                                                        static_cast<cudaStream_t>(stream)),
                                "reconstruct launch"));
}

int dkv_map_fill(int32_t* rows, uint8_t* codes, int64_t start, int32_t n, int64_t row, int32_t bits,
                 int64_t capacity, void* stream) {
  if (rows == nullptr || codes == nullptr) return fail(DKV_EINVAL, "null token map");
  if (bits != 4 && bits != 8 && bits != 16) return fail(DKV_EINVAL, "Supported bit widths: 4, 8, 16");
  if (n < 0 || start < 0 || row < 0) return fail(DKV_EINVAL, "negative map range");
  if (start + n > capacity) return fail(DKV_ECAPACITY, "GPU context limit exceeded");
  if (row + n > INT32_MAX) return fail(DKV_ECAPACITY, "pool row exceeds int32");
  if (n == 0) return ok();
  return note_write(stream, kWroteMaps,
                    cuda_status(dkv::launch_map_fill(rows, codes, start, n, row, bits,
                                                     static_cast<cudaStream_t>(stream)),
                                "map_fill launch"));
}

int dkv_rotary(const void* x, const float* cos_t, const float* sin_t, void* out, int64_t xb, int64_t xt,
               int64_t cb, int32_t b, int32_t n, int32_t heads, int32_t dim, void* stream) {
  if (dim != dkv::kDim) return fail(DKV_EINVAL, "GPU kernel currently supports head_dim=64");
  if (b < 0 || n < 0 || heads <= 0) return fail(DKV_EINVAL, "rotary: negative sizes or no heads");
  if (static_cast<int64_t>(b) * n == 0) return ok();
  if (!x || !cos_t || !sin_t || !out) return fail(DKV_EINVAL, "rotary: null pointer");
  if (!aligned16(x) || !aligned16(out) || !aligned16(cos_t) || !aligned16(sin_t))
    return fail(DKV_EINVAL, "rotary: tensors must be 16-byte aligned");
  if (xb < 0 || xt < static_cast<int64_t>(heads) * dim || xb % 8 || xt % 8)
    return fail(DKV_EINVAL, "rotary: token strides must hold the heads and be multiples of 8 elements");
  if (cb < 0 || cb % 4) return fail(DKV_EINVAL, "rotary: table batch stride must be a multiple of 4");
  return note_write(stream, kWroteNothing,
                    cuda_status(dkv::launch_rotary(x, cos_t, sin_t, out, xb, xt, cb, b, n, heads,
                                                   static_cast<cudaStream_t>(stream)),
                                "rotary launch"));
}

int dkv_silu_mul(const void* gate, const void* up, void* out, int64_t gs, int64_t us, int64_t rows, int32_t width,
                 void* stream) {
  if (rows < 0 || width <= 0 || width % 8) return fail(DKV_EINVAL, "silu_mul: width must be a positive multiple of 8");
  if (rows == 0) return ok();
  if (!gate || !up || !out) return fail(DKV_EINVAL, "silu_mul: null pointer");
  if (!aligned16(gate) || !aligned16(up) || !aligned16(out))
    return fail(DKV_EINVAL, "silu_mul: tensors must be 16-byte aligned");
  if (gs < width || us < width || gs % 8 || us % 8)
    return fail(DKV_EINVAL, "silu_mul: row strides must hold a row and be multiples of 8 elements");
  return note_write(stream, kWroteNothing,
                    cuda_status(dkv::launch_silu_mul(gate, up, out, gs, us, rows, width,
                                                     static_cast<cudaStream_t>(stream)),
                                "silu_mul launch"));
}

int dkv_add_rms_norm(const void* x, const void* y, void* x_out, void* h_out, const void* weight, int64_t rows,
                     int32_t width, int64_t xs, int64_t ys, int64_t os, int64_t hs, float eps, void* stream) {
  if (rows < 0 || width <= 0 || width % 8 || width > 2048)
    return fail(DKV_EINVAL, "add_rms_norm: width must be a multiple of 8 in [8, 2048]");
  if (rows == 0) return ok();
  if (!x || !h_out || !weight || (y != nullptr && x_out == nullptr)) return fail(DKV_EINVAL, "add_rms_norm: null pointer");
  if (!aligned16(x) || !aligned16(h_out) || !aligned16(weight) || (y && (!aligned16(y) || !aligned16(x_out))))
    return fail(DKV_EINVAL, "add_rms_norm: tensors must be 16-byte aligned");
  if (xs < width || hs < width || xs % 8 || hs % 8 || (y && (ys < width || os < width || ys % 8 || os % 8)))
    return fail(DKV_EINVAL, "add_rms_norm: row strides must hold a row and be multiples of 8 elements");
  if (!(eps >= 0.f)) return fail(DKV_EINVAL, "add_rms_norm: eps must be non-negative");
  if (rows > INT32_MAX / 32) return fail(DKV_EINVAL, "add_rms_norm: too many rows");
  return note_write(stream, kWroteNothing,
                    cuda_status(dkv::launch_add_rms_norm(x, y, x_out, h_out, weight, rows, width, xs, ys, os, hs, eps,
                                                         static_cast<cudaStream_t>(stream)),
                                "add_rms_norm launch"));
}

}  // extern "C"
