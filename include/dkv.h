/*
 * dkv.h — C-ABI of the B200 (sm_100a) packed mixed-precision KV-cache library
 * (libdkv.so).
 *
 * The entry points replace the three Triton kernels of the reference's packed-KV
 * hot path (zoaibs/Dynamic-KV-Cache, src/gpu_kernels.py) plus the two device-side
 * bookkeeping writes of its cache object (src/gpu_cache.py:79-80). Argument lists
 * follow the Triton launch signatures, in the same order, with three additions:
 * the layer count (for bounds checks), a device status word and the CUDA stream.
 *
 * Conventions
 *  - Every pointer is a device pointer unless stated; nothing is freed or retained.
 *  - Strides are in ELEMENTS (bf16), exactly as torch's Tensor.stride() reports
 *    them; the innermost (head_dim) stride must be 1.
 *  - bf16 tensors are passed as void*. Pools are paged: the rows of every
 *    (layer, K|V, head) block come in pages of DKV_PAGE_ROWS = 64, and page p of
 *    every block is stored side by side, so a pool of more rows is the same pool
 *    with more pages at the end (growth maps pages, see dkv_pool_*, and copies
 *    nothing). With P = ceil(cap / 64) pages:
 *      p4  uint8 [P4, layers, 2, heads, 64, dim/2]  two 4-bit codes per byte, lo = even
 *      m4  f32   [P4, layers, 2, heads, 64, 2]      (offset, scale) per row
 *      p8  uint8 [P8, layers, 2, heads, 64, dim]
 *      m8  f32   [P8, layers, 2, heads, 64, 2]
 *      p16 bf16  [P16, layers, 2, heads, 64, dim]
 *    (index 2 selects K = 0 or V = 1; row r of a block is at page r / 64, slot
 *    r % 64). cap4 / cap8 / cap16 are the rows in use per block (the reference's
 *    pool capacities, src/gpu_cache.py:36-41), a row r is valid when r < cap; the
 *    reference lays the same rows out as [layers, 2, heads, cap, ...], and the
 *    token maps
 *      rows  int32 [capacity]  pool row of logical token t
 *      codes uint8 [capacity]  storage bits of logical token t (4, 8 or 16)
 *  - `stream` is a cudaStream_t (NULL = legacy default stream). All work is
 *    asynchronous on it; no entry point synchronises.
 *  - Return value: DKV_OK or a DKV_E* code; dkv_last_error() gives the message
 *    (per host thread). Host-side argument errors launch nothing.
 *  - `status` (may be NULL) is an int32[4] device word: the first device-detected
 *    error stores its DKV_E* code in status[0] and a detail index in status[1]
 *    (kernels never trap; the offending access is skipped). The caller reads it
 *    after a synchronisation and clears it.
 *  - head_dim must be 64 (the reference raises the same restriction,
 *    src/gpu_cache.py:14).
 */
#ifndef DKV_H
#define DKV_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DKV_VERSION 2
#define DKV_PAGE_ROWS 64

enum dkv_status {
  DKV_OK = 0,
  DKV_EINVAL = 1,     /* bad argument (shape, stride, alignment, bits)            */
  DKV_ECAPACITY = 2,  /* row or token outside a pool / map capacity               */
  DKV_EPLAN = 3,      /* token map holds a code other than 4, 8 or 16             */
  DKV_ECUDA = 4,      /* a CUDA runtime call or launch failed                     */
  DKV_ENONFINITE = 5, /* pack input held NaN or Inf                               */
  DKV_EWORKSPACE = 6, /* workspace smaller than dkv_packed_attention_workspace() */
  DKV_ETIMEOUT = 7    /* a kernel pipeline wait gave up (bounded waits, no hang)  */
};

/* Library version (DKV_VERSION). */
int32_t dkv_version(void);

/* Message of the last error returned on this host thread ("" if none). */
const char* dkv_last_error(void);

/*
 * Pack one frame of K and V for one layer into the pools at rows
 * [row_start, row_start + n) of the `bits` pool (4, 8 or 16).
 * Replaces Triton `pack_rows` (src/gpu_kernels.py:11-46), launched by
 * GPUCache.append (src/gpu_cache.py:90-92). k, v: bf16 [1, heads, n, dim] with
 * head/token strides (kh, kt) and (vh, vt). 4/8-bit rows use per-row min/max
 * affine quantisation with IEEE fp32 arithmetic, bit-identical to the reference
 * CPU quantiser src/kv_quantization.py:57-71 (group = one 64-wide row).
 */
int dkv_pack_rows(const void* k, const void* v,
                  void* p4, void* m4, void* p8, void* m8, void* p16,
                  int64_t kh, int64_t kt, int64_t vh, int64_t vt,
                  int32_t layer, int64_t row_start, int32_t n,
                  int64_t cap4, int64_t cap8, int64_t cap16,
                  int32_t heads, int32_t dim, int32_t bits,
                  int32_t layers, int32_t* status, void* stream);

/*
 * Causal GQA attention of nq new queries over `past` packed history tokens plus
 * the nq native new K/V rows. Replaces Triton `packed_attention`
 * (src/gpu_kernels.py:71-105), launched by GPUCache.attend
 * (src/gpu_cache.py:96-104). q: bf16 [1, heads*group, nq, dim] with strides
 * (qh, qt); knew/vnew: bf16 [1, heads, nq, dim]; out: bf16 [1, nq, heads*group,
 * dim] contiguous. Query m sees keys t <= past + m. block_m / block_n are the
 * reference's tile knobs: validated (powers of two, 16..256) but the kernel picks
 * its own B200 tiling. `workspace` must hold dkv_packed_attention_workspace()
 * bytes, 256-byte aligned (it may be NULL when that size is 0). Its first 1024 bytes are the
 * split-merge arrival counters: they must be zero before the first call that
 * uses the workspace, and every call leaves them zero again (also when a
 * pipeline wait times out), so a workspace is zero-filled once and then reused.
 * A workspace belongs to one call at a time: calls that may overlap (different
 * streams) need different workspaces.
 *
 * Calls whose history is split are merged by a second (combine) kernel: two
 * launches per call. The fused and batched entry points (dkv_append_attention*,
 * dkv_packed_attention_batched with more than one chunk, the *_many calls)
 * instead merge inside the attention kernel when every block of the launch fits
 * on the GPU at once (one block per SM, at most 148 blocks): one launch, made as
 * a cooperative launch so
 * that all its blocks are co-scheduled (each waits for the others of its group;
 * work on other streams only delays the launch). The environment variable
 * DKV_ATTENTION_MERGE=kernel merges this call in the kernel too where the grid
 * fits; =combine uses the combine kernel everywhere (e.g. under MPS, where a
 * grid may not be resident at once). Both merges do the same arithmetic in the
 * same order: the output is bit-identical either way.
 */
int dkv_packed_attention(const void* q, const void* knew, const void* vnew,
                         const void* p4, const void* m4, const void* p8,
                         const void* m8, const void* p16,
                         const int32_t* rows, const uint8_t* codes, void* out,
                         int64_t qh, int64_t qt, int64_t kh, int64_t kt,
                         int64_t vh, int64_t vt,
                         int32_t layer, int32_t past, int32_t nq,
                         int64_t cap4, int64_t cap8, int64_t cap16,
                         int32_t heads, int32_t group, int32_t dim,
                         int32_t block_m, int32_t block_n,
                         int32_t layers, void* workspace, size_t workspace_bytes,
                         int32_t* status, void* stream);

/* Workspace bytes dkv_packed_attention needs for this shape (0 = none). */
size_t dkv_packed_attention_workspace(int32_t past, int32_t nq, int32_t heads,
                                      int32_t group, int32_t dim);

/*
 * dkv_packed_attention over `chunks` independent query chunks that share one
 * packed history (no reference counterpart: it serves batched candidate scoring,
 * where every candidate attends to the same prefix + question and to its own
 * tokens only). Chunk c's q / knew / vnew / out begin qc / kc / vc / oc elements
 * after chunk 0's (multiples of 8); each chunk has nq queries with the same
 * causal rule as dkv_packed_attention and reads its own nq new K/V rows natively
 * (they are not appended to the pools). Same workspace contract, sized by
 * dkv_packed_attention_batched_workspace(); chunks = 1 is dkv_packed_attention.
 */
int dkv_packed_attention_batched(const void* q, const void* knew, const void* vnew,
                                 const void* p4, const void* m4, const void* p8,
                                 const void* m8, const void* p16,
                                 const int32_t* rows, const uint8_t* codes, void* out,
                                 int64_t qh, int64_t qt, int64_t kh, int64_t kt,
                                 int64_t vh, int64_t vt, int32_t chunks,
                                 int64_t qc, int64_t kc, int64_t vc, int64_t oc,
                                 int32_t layer, int32_t past, int32_t nq,
                                 int64_t cap4, int64_t cap8, int64_t cap16,
                                 int32_t heads, int32_t group, int32_t dim,
                                 int32_t block_m, int32_t block_n,
                                 int32_t layers, void* workspace, size_t workspace_bytes,
                                 int32_t* status, void* stream);

/* Workspace bytes dkv_packed_attention_batched needs (0 = none). */
size_t dkv_packed_attention_batched_workspace(int32_t past, int32_t nq, int32_t heads,
                                              int32_t group, int32_t dim, int32_t chunks);

/* Kernel launches one dkv_packed_attention call of this shape makes on the
 * current device (1 or 2; 0 for invalid shapes, -1 on a CUDA error). No
 * reference counterpart: it lets callers and benchmarks count launches. */
int32_t dkv_packed_attention_launches(int32_t past, int32_t nq, int32_t heads,
                                      int32_t group, int32_t dim);

/* Size of the fixed scratch array inside libdkv.so used by
 * dkv_packed_attention_noalloc (10 MiB: the largest workspace the attention
 * planner can ask for, at most 148 split blocks of 256 rows). */
#define DKV_NOALLOC_SCRATCH_BYTES (10u * 1024u * 1024u)

/*
 * dkv_packed_attention for callers that cannot allocate device memory. It has no
 * counterpart in the reference (whose Triton kernel needs no scratch): it exists
 * for callers such as embedders with a device-memory budget fixed up front, host
 * runtimes whose own allocator forbids cudaMalloc on the hot path, or bindings
 * without a device allocator at all. Same arguments and results as
 * dkv_packed_attention without the workspace pair; the partial results of the
 * history splits go to a DKV_NOALLOC_SCRATCH_BYTES array that lives in the
 * library, so the call allocates nothing. Every GPU that loads the library holds
 * that array until exit and all calls on a GPU share it: calls whose kernels
 * overlap on one GPU (e.g. on two streams) race and must be serialised. Nothing
 * in it needs clearing between calls. The first call on each device looks the
 * array's device address up (cudaGetSymbolAddress); make that first call before
 * any stream capture. The address is kept for the life of the process, so calls
 * must not span a cudaDeviceReset (which unloads the library's device image and
 * may move the array). Shapes needing more scratch than the array holds return
 * DKV_EWORKSPACE (the planner never asks for more).
 */
int dkv_packed_attention_noalloc(const void* q, const void* knew, const void* vnew,
                                 const void* p4, const void* m4, const void* p8,
                                 const void* m8, const void* p16,
                                 const int32_t* rows, const uint8_t* codes, void* out,
                                 int64_t qh, int64_t qt, int64_t kh, int64_t kt,
                                 int64_t vh, int64_t vt,
                                 int32_t layer, int32_t past, int32_t nq,
                                 int64_t cap4, int64_t cap8, int64_t cap16,
                                 int32_t heads, int32_t group, int32_t dim,
                                 int32_t block_m, int32_t block_n,
                                 int32_t layers, int32_t* status, void* stream);

/*
 * ---- Growable device pools (no reference counterpart) ----
 * The reference grows a precision pool by allocating a larger tensor and copying
 * every old row into it (GPUCache.reserve, src/gpu_cache.py:44-59). A dkv_pool
 * reserves the largest size a pool can reach as device address space once and
 * maps physical memory onto the front of that range as the pool grows (CUDA
 * virtual memory management, in multiples of dkv_pool_granularity() bytes). With
 * the paged layout above, growing cap only appends pages, so the base address
 * never moves and no row is copied; descriptors captured in a CUDA graph stay
 * valid across a growth. Pages are uninitialised, as the reference's torch.empty.
 */
typedef struct dkv_pool dkv_pool;

/* Mapping granularity of `device` in bytes (0 if the driver offers none). */
uint64_t dkv_pool_granularity(int32_t device);

/* Reserves reserve_bytes (rounded up to the granularity) of address space on
   `device` with nothing mapped; *pool receives the handle. */
int dkv_pool_create(int32_t device, uint64_t reserve_bytes, dkv_pool** pool);

/* Maps physical memory so that [base, base + bytes) is usable (rounded up to the
   granularity; never shrinks). DKV_ECAPACITY beyond the reservation, DKV_ECUDA
   when the device is out of memory. Host-side only: enqueues nothing. */
int dkv_pool_map(dkv_pool* pool, uint64_t bytes);

/* First byte of the reservation (fixed for the pool's lifetime). */
void* dkv_pool_base(const dkv_pool* pool);
uint64_t dkv_pool_mapped_bytes(const dkv_pool* pool);
uint64_t dkv_pool_reserved_bytes(const dkv_pool* pool);

/* Synchronises the pool's device (work still queued may read the pages), then
   unmaps and releases everything. The handle is invalid afterwards. */
int dkv_pool_destroy(dkv_pool* pool);

/*
 * ---- Request batching (no reference counterpart) ----
 * The reference serves one request per cache and launches pack and attention
 * once per request and layer. The entry points below take B independent
 * requests, each with its own pools, token maps and history length, and do the
 * work of all of them in one launch per layer: the frame appends of B streams
 * then share every weight read and every launch of the model around the cache.
 * At most DKV_MAX_REQUESTS requests per call (larger batches are split by the
 * caller); the descriptors are passed to the kernels by value, so the arrays
 * below are read on the host during the call and may be reused right after.
 */
#define DKV_MAX_REQUESTS 32

/* One request's packed history, as read by dkv_packed_attention_many. */
typedef struct dkv_history {
  const void* p4;  /* pools and (offset, scale) metadata of this request, */
  const void* m4;  /* laid out as for dkv_packed_attention                */
  const void* p8;
  const void* m8;
  const void* p16;
  const int32_t* rows;   /* token map: pool row of logical token t */
  const uint8_t* codes;  /* token map: precision (4 / 8 / 16) of token t */
  int64_t cap4, cap8, cap16;
  int32_t past;          /* packed history tokens before this call's queries */
  int32_t capacity;      /* length of rows / codes (past must not exceed it) */
  int32_t* status;       /* this request's device status word (may be NULL) */
} dkv_history;

/* One request's destination, as written by dkv_pack_rows_many. */
typedef struct dkv_pack_target {
  void* p4;
  void* m4;
  void* p8;
  void* m8;
  void* p16;
  int64_t cap4, cap8, cap16;
  int64_t row_start;     /* first row of the `bits` pool that the frame fills */
  int32_t bits;          /* 4, 8 or 16 for this request's frame */
  int32_t reserved;
  int32_t* map_rows;     /* when not NULL: also writes the token map entries */
  uint8_t* map_codes;    /* map_rows[map_start + i] = row_start + i and */
  int64_t map_start;     /* map_codes[map_start + i] = bits, i in [0, n) */
  int64_t map_capacity;  /* length of map_rows / map_codes */
  int32_t* status;       /* this request's device status word (may be NULL) */
} dkv_pack_target;

/*
 * dkv_pack_rows for `count` requests in one launch: request r's frame is
 * k + r*kc, v + r*vc (bf16 [heads, n, dim] with strides (kh, kt), (vh, vt); kc and
 * vc multiples of 8), packed at targets[r].bits into targets[r]'s pools. Every
 * row is quantised exactly as dkv_pack_rows does it (bit-identical pools). With
 * map pointers set it also performs dkv_map_fill's update (done once, at layer
 * 0, by GPUCache-style callers).
 */
int dkv_pack_rows_many(const void* k, const void* v, const dkv_pack_target* targets, int32_t count,
                       int64_t kh, int64_t kt, int64_t vh, int64_t vt, int64_t kc, int64_t vc,
                       int32_t layer, int32_t n, int32_t heads, int32_t dim, int32_t layers,
                       void* stream);

/*
 * dkv_packed_attention for `count` requests in one launch: request r's nq queries
 * (q + r*qc, bf16 [heads*group, nq, dim], strides (qh, qt)) attend causally over
 * requests[r]'s packed history (requests[r].past tokens; pasts may differ) plus
 * their own nq new K/V rows (knew + r*kc, vnew + r*vc) read natively; the output
 * goes to out + r*oc as bf16 [nq, heads*group, dim]. Chunk strides are multiples
 * of 8 elements. Same workspace contract as dkv_packed_attention, sized by
 * dkv_packed_attention_many_workspace() for the largest past of the batch.
 */
int dkv_packed_attention_many(const void* q, const void* knew, const void* vnew,
                              const dkv_history* requests, int32_t count, void* out,
                              int64_t qh, int64_t qt, int64_t kh, int64_t kt, int64_t vh, int64_t vt,
                              int64_t qc, int64_t kc, int64_t vc, int64_t oc,
                              int32_t layer, int32_t nq, int32_t heads, int32_t group, int32_t dim,
                              int32_t layers, void* workspace, size_t workspace_bytes, void* stream);

/* Workspace bytes dkv_packed_attention_many needs (0 = none); max_past = the
 * largest requests[r].past of the call. The history is divided into as many
 * splits as fill one wave of the GPU (no more than the longest history has
 * 64-key tiles); each request splits its own history evenly among them. */
size_t dkv_packed_attention_many_workspace(int32_t max_past, int32_t nq, int32_t heads, int32_t group,
                                           int32_t dim, int32_t count);

/*
 * Device-resident descriptors, for CUDA-graph replay: the same two operations
 * with `targets` / `requests` in device memory (16-byte aligned arrays of
 * `count` structs, count <= 65535). A captured graph keeps reading the same
 * arrays, so a caller replays it step after step after writing that step's
 * descriptors there (rows claimed, history lengths, pools after growth) with a
 * stream-ordered copy. The host cannot check device-resident descriptors: the
 * kernels do (precision, pool and map ranges, history length against the map
 * capacity) and report a bad one to its status word instead of using it.
 * dkv_packed_attention_many_device plans for histories of at most max_past
 * tokens (the workspace, from dkv_packed_attention_many_workspace(max_past, ...),
 * and the split count are fixed by it); a longer history is still attended
 * completely, in longer splits. With the same max_past and count as a
 * dkv_packed_attention_many call over the same histories, the output is
 * bit-identical to it.
 */
int dkv_pack_rows_many_device(const void* k, const void* v, const dkv_pack_target* targets, int32_t count,
                              int64_t kh, int64_t kt, int64_t vh, int64_t vt, int64_t kc, int64_t vc,
                              int32_t layer, int32_t n, int32_t heads, int32_t dim, int32_t layers,
                              void* stream);

int dkv_packed_attention_many_device(const void* q, const void* knew, const void* vnew,
                                     const dkv_history* requests, int32_t count, int32_t max_past, void* out,
                                     int64_t qh, int64_t qt, int64_t kh, int64_t kt, int64_t vh, int64_t vt,
                                     int64_t qc, int64_t kc, int64_t vc, int64_t oc,
                                     int32_t layer, int32_t nq, int32_t heads, int32_t group, int32_t dim,
                                     int32_t layers, void* workspace, size_t workspace_bytes, void* stream);

/*
 * Append + attend in one launch (no reference counterpart as one call: the
 * reference's attention forward runs pack_rows then packed_attention back to
 * back, src/gpu_cache.py:172-173). Packs the nq new rows knew / vnew into rows
 * [row_start, row_start + nq) of the `bits` pool exactly as dkv_pack_rows does
 * (with fill_map, also the token-map update of dkv_map_fill at [past, past + nq)),
 * and computes dkv_packed_attention over the `past` history tokens plus the new
 * rows read natively. One kernel does both: its blocks pack their share of the
 * new rows while they wait for the other history splits.
 * Results are bit-identical to dkv_pack_rows (+ dkv_map_fill) followed by
 * dkv_packed_attention; same workspace contract as dkv_packed_attention.
 */
int dkv_append_attention(const void* q, const void* knew, const void* vnew,
                         void* p4, void* m4, void* p8, void* m8, void* p16,
                         int32_t* rows, uint8_t* codes, void* out,
                         int64_t qh, int64_t qt, int64_t kh, int64_t kt, int64_t vh, int64_t vt,
                         int32_t layer, int32_t past, int32_t nq,
                         int64_t row_start, int32_t bits, int32_t fill_map, int64_t map_capacity,
                         int64_t cap4, int64_t cap8, int64_t cap16,
                         int32_t heads, int32_t group, int32_t dim,
                         int32_t block_m, int32_t block_n, int32_t layers,
                         void* workspace, size_t workspace_bytes, int32_t* status, void* stream);

/*
 * dkv_append_attention for `count` requests with device-resident descriptors
 * (CUDA-graph replay of frame steps): request r's frame is packed into
 * targets[r] and its queries attend over requests[r] plus its new rows. Same as
 * dkv_pack_rows_many_device followed by dkv_packed_attention_many_device.
 */
int dkv_append_attention_many_device(const void* q, const void* knew, const void* vnew,
                                     const dkv_pack_target* targets, const dkv_history* requests,
                                     int32_t count, int32_t max_past, void* out,
                                     int64_t qh, int64_t qt, int64_t kh, int64_t kt, int64_t vh, int64_t vt,
                                     int64_t qc, int64_t kc, int64_t vc, int64_t oc,
                                     int32_t layer, int32_t nq, int32_t heads, int32_t group, int32_t dim,
                                     int32_t layers, void* workspace, size_t workspace_bytes, void* stream);

/*
 * Dequantised bf16 history of one layer: out[2, heads, n, dim] (K then V) for
 * logical tokens [0, n). Replaces Triton `reconstruct` (src/gpu_kernels.py:
 * 107-119), launched by GPUCache.materialize (src/gpu_cache.py:106-112).
 * x = bf16(fp32(code * scale) + offset), the operation order of the reference
 * CPU unpack (src/kv_quantization.py:91).
 */
int dkv_reconstruct(const void* p4, const void* m4, const void* p8,
                    const void* m8, const void* p16,
                    const int32_t* rows, const uint8_t* codes, void* out,
                    int32_t layer, int32_t n,
                    int64_t cap4, int64_t cap8, int64_t cap16,
                    int32_t heads, int32_t dim, int32_t layers,
                    int32_t* status, void* stream);

/*
 * Device-resident token-map update for one appended segment:
 * rows[start + i] = row + i and codes[start + i] = bits for i in [0, n).
 * Replaces the two tensor writes at src/gpu_cache.py:79-80 with one launch.
 */
int dkv_map_fill(int32_t* rows, uint8_t* codes, int64_t start, int32_t n,
                 int64_t row, int32_t bits, int64_t capacity, void* stream);

/*
 * Rotate-half rotary embedding of the first `heads` heads of each token, one
 * launch (the reference applies HF apply_rotary_pos_emb to q and k before
 * append / attend, src/gpu_cache.py:170; this is its fp32 form, as in the
 * streaming decoder). x: bf16 [b, n, >= heads, dim], token strides (xb, xt)
 * in elements, heads contiguous; cos / sin: fp32 [b or 1, n, dim] with batch
 * stride cb (0 broadcasts one table over b) and token stride dim; out: bf16
 * [b, n, heads, dim], contiguous. For i < dim/2, with h = dim/2:
 *   out[i]     = bf16(x[i] cos[i]         - x[i + h] sin[i])
 *   out[i + h] = bf16(x[i + h] cos[i + h] + x[i] sin[i + h])
 * each product and the sum one fp32 operation rounded to nearest.
 */
int dkv_rotary(const void* x, const float* cos_t, const float* sin_t, void* out,
               int64_t xb, int64_t xt, int64_t cb, int32_t b, int32_t n,
               int32_t heads, int32_t dim, void* stream);

/*
 * silu(gate) * up over `rows` rows of `width` elements (activation_product,
 * src/gpu_ops.py:14-17), one launch: silu = gate / (1 + exp(-gate)) in fp32
 * rounded to bf16, then the product in fp32 rounded to bf16. gate / up: bf16
 * with row strides gs / us (elements); out: bf16 [rows, width], contiguous.
 */
int dkv_silu_mul(const void* gate, const void* up, void* out, int64_t gs, int64_t us,
                 int64_t rows, int32_t width, void* stream);

/*
 * Residual add + RMSNorm + weight over `rows` rows of `width` (8..2048, a multiple
 * of 8) elements, one launch (the decoder layer's x = x + y, then cuda_rms,
 * src/gpu_ops.py:9-12, of the new x): x_out = bf16(x + y); h_out =
 * bf16(bf16(x_out * rsqrt(mean(x_out^2) + eps)) * weight). With y == NULL there
 * is no add and the norm is of x (x_out unused). The rounding points are
 * PyTorch's; the fp32 sum of squares has this kernel's own order, so h_out may
 * differ from torch.nn.functional.rms_norm in the last bf16 bit. bf16 tensors,
 * row strides xs / ys / os / hs in elements, weight [width] contiguous.
 */
int dkv_add_rms_norm(const void* x, const void* y, void* x_out, void* h_out, const void* weight, int64_t rows,
                     int32_t width, int64_t xs, int64_t ys, int64_t os, int64_t hs, float eps, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* DKV_H */
