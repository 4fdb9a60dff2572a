"""Packed mixed-precision KV cache on the B200 kernels.

Drop-in for the reference's src/gpu_cache.py: same class name, constructor
keywords, methods, attributes and error messages (GPUCache, src/gpu_cache.py:
10-149; install_packed_attention, :151-183). The pools keep the reference's
growth policy and row numbering, so `caps`, `host_counts`, `plan`, the token
maps `rows`/`codes` and `accounting()` read exactly as the reference's do. The
Triton launches are replaced by the sm_100a kernels of libdkv.so (gpu_kernels),
and the per-token map update is one device launch (map_fill).

Pools are paged (include/dkv.h): the rows of every (layer, K|V, head) block come
in pages of 64 and page p of every block is stored side by side, so
`p4` is [pages, layers, 2, heads, 64, 32] where the reference has
[layers, 2, heads, cap4, 32]; `pool_rows` reads rows in the reference's
terms. On CUDA each pool lives in a device region that reserves the address
space of the largest capacity the cache can reach and maps memory as it grows:
growth appends pages and copies no row (the reference allocates a larger tensor
and copies, src/gpu_cache.py:44-59), and the pool pointers never move.
"""
import ctypes
import types

import torch
import torch.nn.functional as F
from transformers.cache_utils import DynamicCache

from . import gpu_kernels as K

BITS = (4, 8, 16)
PAGE_ROWS = 64
# pool attribute -> (dtype, row width in elements, precision)
POOLS = {'p4': (torch.uint8, 32, 4), 'm4': (torch.float32, 2, 4), 'p8': (torch.uint8, 64, 8),
         'm8': (torch.float32, 2, 8), 'p16': (torch.bfloat16, 64, 16)}


def _pages(rows):
    return max(1, (rows + PAGE_ROWS - 1) // PAGE_ROWS)


def _growth(old, needed):
    """The reference's new capacity for a pool of `old` rows that must hold `needed`
    (src/gpu_cache.py:47)."""
    return max(needed, ((int(old * 1.5) + 63) // 64) * 64)


class GPUCache(DynamicCache):
    def __init__(self, plan=None, layers=30, heads=3, dim=64, device='cuda', dtype=torch.bfloat16,
                 backend='fused', block_m=16, block_n=64, max_tokens=8192):
        super().__init__()
        if dim != 64:
            raise ValueError('GPU kernel currently supports head_dim=64')
        if dtype != torch.bfloat16:
            raise ValueError('GPU kernel stores 16-bit rows as bfloat16')
        self.layers, self.heads, self.dim = layers, heads, dim
        self.dtype, self.device = dtype, torch.device(device)
        self.backend, self.block_m, self.block_n = backend, block_m, block_n
        self.seen = [0] * layers
        self.cursors = [0] * layers
        self.pending_bits = 16
        self.frame_id = -1
        self.online = plan is None
        rows, codes, counts = [], [], {4: 0, 8: 0, 16: 0}
        self.plan = []
        # Offline plan: segments (start, end, bits, first pool row), src/gpu_cache.py:23-29.
        for bits, n in (plan or []):
            if bits not in counts or n < 0:
                raise ValueError('Invalid GPU cache plan')
            self.plan.append((len(rows), len(rows) + n, bits, counts[bits]))
            rows.extend(range(counts[bits], counts[bits] + n))
            codes.extend([bits] * n)
            counts[bits] += n
        self.capacity = max_tokens if self.online else len(rows)
        self.caps = {b: 64 if self.online else max(1, n) for b, n in counts.items()}
        if self.online:
            self.rows = torch.zeros(self.capacity, dtype=torch.int32, device=self.device)
            self.codes = torch.zeros(self.capacity, dtype=torch.uint8, device=self.device)
        else:
            self.rows = torch.tensor(rows, dtype=torch.int32, device=self.device)
            self.codes = torch.tensor(codes, dtype=torch.uint8, device=self.device)
        # An online pool never holds more rows than the cache has tokens, so the
        # reference's growth stops at _growth(capacity - 1, capacity); an offline
        # plan fixes the capacities up front.
        limit = _growth(self.capacity - 1, self.capacity) if self.online else 0
        self._leases = {}
        for name, (_, _, bits) in POOLS.items():
            self._allocate(name, self.caps[bits], max(limit, self.caps[bits]))
        self.host_counts = counts
        # Device status word written by the kernels (first error code, detail index).
        self.status = torch.zeros(4, dtype=torch.int32, device=self.device)
        self._refresh_ptrs()

    def _refresh_ptrs(self):
        """Device addresses the per-layer calls pass (pools, maps, status word): one
        list, renewed whenever a pool tensor changes."""
        self._ptrs = [t.data_ptr() for t in (self.p4, self.m4, self.p8, self.m8, self.p16, self.rows, self.codes,
                                             self.status)]

    # -- capacity ---------------------------------------------------------------
    def _page_shape(self, name, pages):
        return (pages, self.layers, 2, self.heads, PAGE_ROWS, POOLS[name][1])

    def _page_bytes(self, name):
        dtype, width, _ = POOLS[name]
        return self.layers * 2 * self.heads * PAGE_ROWS * width * dtype.itemsize

    def _allocate(self, name, rows, limit_rows):
        """Pool `name` with room for `rows` rows per block; on CUDA in a region
        reserved for `limit_rows`."""
        dtype = POOLS[name][0]
        pages = _pages(rows)
        if self.device.type != 'cuda':  # host-side bookkeeping (tests): a plain tensor
            setattr(self, name, torch.empty(self._page_shape(name, pages), dtype=dtype, device=self.device))
            return
        lease = K.lease_region(self.device, _pages(limit_rows) * self._page_bytes(name))
        lease.region.map(pages * self._page_bytes(name))
        self._leases[name] = lease
        setattr(self, name, K.region_tensor(lease, self._page_shape(name, pages), dtype))

    def _grow(self, name, rows):
        """Pool `name` to `rows` rows per block, its old rows left where they are."""
        dtype = POOLS[name][0]
        old = getattr(self, name)
        pages = _pages(rows)
        if pages <= old.shape[0]:
            return
        lease = self._leases.get(name)
        if lease is not None and pages * self._page_bytes(name) <= lease.region.reserved:
            lease.region.map(pages * self._page_bytes(name))  # new pages behind the old ones
            setattr(self, name, K.region_tensor(lease, self._page_shape(name, pages), dtype))
            return
        # beyond the reservation (an explicit reserve() past the cache's token
        # capacity) or a host tensor: a larger pool and one copy of the old pages
        self._leases = dict(self._leases)  # a fork's pools stay with the base
        self._allocate(name, rows, 2 * rows)
        getattr(self, name)[:old.shape[0]].copy_(old)

    def reserve(self, bits, needed):
        """Grows pool `bits` to at least `needed` rows: max(needed, 1.5x rounded up
        to 64), as src/gpu_cache.py:44-59. On CUDA the new pages are mapped behind
        the old ones; no row moves."""
        old = self.caps[bits]
        if needed <= old:
            return
        cap = _growth(old, needed)
        for name, (_, _, b) in POOLS.items():
            if b == bits:
                self._grow(name, cap)
        self.caps[bits] = cap
        self._refresh_ptrs()

    def pool_rows(self, name, layer, kv, start, n):
        """Rows [start, start + n) of pool `name` ('p4', 'm4', 'p8', 'm8', 'p16')
        for (layer, K = 0 | V = 1) as [heads, n, width]: the reference's
        `<pool>[layer, kv, :, start:start + n]` (a gathered copy)."""
        self._check_rows(name, layer, kv, start, n)
        r = torch.arange(start, start + n, device=self.device)
        return getattr(self, name)[r // PAGE_ROWS, layer, kv, :, r % PAGE_ROWS].transpose(0, 1)

    def write_pool_rows(self, name, layer, kv, start, rows):
        """Stores `rows` ([heads, n, width]) at rows [start, start + n) of pool
        `name` for (layer, kv)."""
        self._check_rows(name, layer, kv, start, rows.shape[1])
        r = torch.arange(start, start + rows.shape[1], device=self.device)
        getattr(self, name)[r // PAGE_ROWS, layer, kv, :, r % PAGE_ROWS] = rows.transpose(0, 1).to(self.device)

    def _check_rows(self, name, layer, kv, start, n):
        """Host-side bounds of a pool_rows / write_pool_rows range (a device-side
        index error would end the CUDA context)."""
        if name not in POOLS or not 0 <= layer < self.layers or kv not in (0, 1) or start < 0 or n < 0 \
                or start + n > self.caps[POOLS[name][2]]:
            raise ValueError(f'rows [{start}, {start + n}) of {name} outside the pool')

    def select(self, bits, frame_id=-1):
        self.pending_bits, self.frame_id = bits, frame_id

    def get_seq_length(self, layer_idx=0):
        return self.seen[layer_idx]

    def get_max_cache_shape(self, layer_idx=0):
        return None

    def __len__(self):
        return self.layers

    # transformers 5.x asks every cache for these (the reference targets 4.51, whose
    # DynamicCache had no per-layer objects); here every layer is full attention
    @property
    def is_sliding(self):
        return [False] * self.layers

    @property
    def is_compileable(self):
        return False

    def get_mask_sizes(self, query, layer_idx=0):
        """(kv_length, kv_offset) of the causal mask for `query` new tokens (a count
        or their cache positions)."""
        q = query if isinstance(query, int) else query.shape[0]
        return q + self.seen[layer_idx], 0

    # -- hot path -----------------------------------------------------------------
    def _pools(self):
        return (self.p4, self.m4, self.p8, self.m8, self.p16)

    def append(self, k, v, layer):
        """Packs one frame's K/V for `layer`; returns the history length before it
        (src/gpu_cache.py:68-94)."""
        if k.shape[0] != 1 or k.shape[-1] != self.dim or k.device.type != 'cuda':
            raise ValueError('GPU cache requires CUDA, batch one and the configured head dimension')
        past, n, row = self._claim(layer, k.shape[-2])
        K.FAST.pack(k, v, self._ptrs, layer, row, (self.caps[4], self.caps[8], self.caps[16]), self.heads,
                    self.pending_bits, self.layers)
        self.seen[layer] = past + n
        return past

    def append_attend(self, q, k, v, layer):
        """append() then attend() of one frame in one call (one kernel launch):
        returns [1, n, query_heads, dim], bit-identical to the
        two calls. The reference's attention forward makes the two calls back to
        back (src/gpu_cache.py:172-173)."""
        if k.shape[0] != 1 or k.shape[-1] != self.dim or k.device.type != 'cuda':
            raise ValueError('GPU cache requires CUDA, batch one and the configured head dimension')
        n = q.shape[-2]
        new_segment = self.online and layer == 0
        past, n, row = self._claim(layer, k.shape[-2], fill_map=False)
        out = K.FAST.append_attend(q, k, v, self._ptrs, layer, past, row, self.pending_bits, new_segment,
                                   self.capacity, (self.caps[4], self.caps[8], self.caps[16]), self.heads,
                                   self.block_m, self.block_n, self.layers)
        self.seen[layer] = past + n
        return out

    def _claim(self, layer, n, fill_map=True):
        """Plan bookkeeping of an n-token append to `layer` at the selected precision
        (src/gpu_cache.py:72-90): returns (past, n, first pool row); the caller
        writes the rows and advances seen[layer]. With fill_map=False the token
        map update of a new online segment is left to the caller's pack launch."""
        past = self.seen[layer]
        if past + n > self.capacity:
            raise ValueError('GPU context limit exceeded')
        if self.online:
            if layer == 0:
                row = self.host_counts[self.pending_bits]
                self.reserve(self.pending_bits, row + n)
                self.plan.append((past, past + n, self.pending_bits, row))
                self.host_counts[self.pending_bits] += n
                if fill_map:
                    K.map_fill(self.rows, self.codes, past, n, row, self.pending_bits, self.capacity)
            segment = self.plan[-1]
        else:
            cursor = self.cursors[layer]
            while cursor < len(self.plan) and past >= self.plan[cursor][1]:
                cursor += 1
            self.cursors[layer] = cursor
            segment = self.plan[cursor] if cursor < len(self.plan) else None
        if segment is None or past + n > segment[1] or segment[2] != self.pending_bits:
            raise ValueError(f'Cache append does not match plan at token {past}, length {n}, '
                             f'bits {self.pending_bits}')
        return past, n, segment[3] + past - segment[0]

    def _claim_frame(self, n):
        """The claims of one n-token append on every layer at once (the bookkeeping
        append() does layer by layer, for a frame whose rows are written by a
        device-descriptor launch). Every layer must hold the same history.
        Returns (past, first pool row) and advances every layer."""
        past = self.seen[0]
        if any(s != past for s in self.seen):
            raise ValueError('GPU cache layers disagree about the history length')
        row = None
        for layer in range(self.layers) if not self.online else (0,):
            _, _, r = self._claim(layer, n, fill_map=False)
            if row is not None and r != row:
                raise ValueError('GPU cache plan rows differ between layers')
            row = r
        self.seen = [past + n] * self.layers
        return past, row

    def attend(self, q, k, v, layer, past):
        """Causal GQA attention of the n new queries over the packed history plus
        the native new K/V; returns [1, n, query_heads, dim] (src/gpu_cache.py:96-104)."""
        return K.FAST.attend(q, k, v, self._ptrs, layer, past, (self.caps[4], self.caps[8], self.caps[16]),
                             self.heads, self.block_m, self.block_n, self.layers)

    def attend_batched(self, q, k, v, layer, past):
        """B independent query chunks over the same packed history (batched candidate
        scoring): q [B, query_heads, n, dim], k / v [B, heads, n, dim] are each
        chunk's own new K/V, attended natively and not appended. Returns
        [B, n, query_heads, dim]. Not in the reference."""
        b, _, n, _ = q.shape
        out = torch.empty((b, n, q.shape[1], self.dim), dtype=q.dtype, device=q.device)
        K.packed_attention_batched(q, k, v, *self._pools(), self.rows, self.codes, out, layer, past, n,
                                   self.caps[4], self.caps[8], self.caps[16], self.heads, q.shape[1] // self.heads,
                                   self.dim, self.block_m, self.block_n, self.layers, self.status)
        return out

    def materialize(self, layer):
        """Dequantised bf16 history (k, v), each [1, heads, seen, dim] (src/gpu_cache.py:106-112)."""
        n = self.seen[layer]
        out = torch.empty((2, self.heads, n, self.dim), dtype=self.dtype, device=self.device)
        K.reconstruct(*self._pools(), self.rows, self.codes, out, layer, n, self.caps[4], self.caps[8],
                      self.caps[16], self.heads, self.dim, self.layers, self.status)
        return out[0:1], out[1:2]

    def update(self, key_states, value_states, layer_idx, cache_kwargs=None):
        """HF Cache.update contract used by the sdpa backend (src/gpu_cache.py:114-119)."""
        self.append(key_states, value_states, layer_idx)
        k, v = self.materialize(layer_idx)
        k[:, :, -key_states.shape[-2]:].copy_(key_states)
        v[:, :, -value_states.shape[-2]:].copy_(value_states)
        return k, v

    def fork(self):
        """QA branch sharing the pools and maps; host bookkeeping is copied, so a
        branch's appends and growth never move the base (src/gpu_cache.py:121-132).
        Branches overwrite the same reserved rows and must run one after another
        on one stream. A branch's growth maps pages behind the base's rows in the
        shared regions; the base's capacities and rows stay as they were."""
        other = object.__new__(GPUCache)
        other.__dict__ = self.__dict__.copy()
        other.seen = self.seen.copy()
        other.cursors = self.cursors.copy()
        other.plan = self.plan.copy()
        other.host_counts = self.host_counts.copy()
        other.caps = self.caps.copy()
        other.pending_bits = 16
        return other

    def check(self):
        """Synchronises and raises ValueError if a kernel flagged an error (a
        non-finite pack input or a corrupt token map). Not in the reference,
        whose kernels have no device-side checks."""
        K.raise_for_status(self.status)

    def accounting(self):
        """Used/allocated bytes with the reference's formulas (src/gpu_cache.py:134-149)."""
        # the reference's allocation, [layers, 2, heads, cap, width] per pool
        blocks = self.layers * 2 * self.heads
        allocated = sum(blocks * self.caps[b] * w * dtype.itemsize for dtype, w, b in POOLS.values())
        allocated += self.rows.numel() * self.rows.element_size() + self.codes.numel() * self.codes.element_size()
        used = {4: 0, 8: 0, 16: 0}
        n = self.seen[0]
        for start, end, bits, row in self.plan:
            used[bits] += max(0, min(n, end) - start)
        payload = self.layers * 2 * self.heads * self.dim * sum(used[b] * b / 8 for b in used)
        scales = self.layers * 2 * self.heads * 8 * (used[4] + used[8])
        mapping = n * 5
        return dict(gpu_cache_used_bytes=int(payload + scales + mapping),
                    gpu_cache_allocated_bytes=allocated, cpu_cache_payload_bytes=0,
                    payload_bytes=int(payload), quantization_metadata_bytes=int(scales),
                    token_mapping_bytes=mapping, logical_index_capacity=self.capacity,
                    precision_pool_capacities=self.caps,
                    used_tokens=n, precision_token_counts=used)


def install_packed_attention(model):
    """Routes GPUCache through the fused kernels in every LlamaAttention of `model`;
    other caches keep the upstream forward (src/gpu_cache.py:151-183)."""
    def forward(module, hidden_states, position_embeddings, attention_mask=None,
                past_key_value=None, cache_position=None, **kwargs):
        cache = past_key_value if past_key_value is not None else kwargs.get('past_key_values')
        fused = isinstance(cache, GPUCache) and cache.backend == 'fused'
        fast_gqa = getattr(cache, 'fast_gqa', False)
        if not fused and not fast_gqa:
            if past_key_value is not None:
                kwargs['past_key_value'] = past_key_value
            return module._original_forward(hidden_states=hidden_states,
                                            position_embeddings=position_embeddings,
                                            attention_mask=attention_mask,
                                            cache_position=cache_position, **kwargs)
        if kwargs.get('output_attentions', False):
            raise ValueError('Fused packed attention does not expose attention matrices')
        from transformers.models.llama.modeling_llama import apply_rotary_pos_emb
        shape = hidden_states.shape[:-1]
        if fused and hasattr(module, '_qkv_weight'):
            q, k, v = F.linear(hidden_states, module._qkv_weight).split(module._qkv_sizes, dim=-1)
        else:
            q, k, v = module.q_proj(hidden_states), module.k_proj(hidden_states), module.v_proj(hidden_states)
        q = q.view(*shape, -1, module.head_dim).transpose(1, 2)
        k = k.view(*shape, -1, module.head_dim).transpose(1, 2)
        v = v.view(*shape, -1, module.head_dim).transpose(1, 2)
        q, k = apply_rotary_pos_emb(q, k, *position_embeddings)
        if fused:  # the reference's append + attend (:172-173), here one call and one launch
            output = cache.append_attend(q, k, v, module.layer_idx)
        else:
            k, v = cache.update(k, v, module.layer_idx, {'cache_position': cache_position})
            mask = None if attention_mask is None else attention_mask[:, :, :, :k.shape[-2]]
            output = F.scaled_dot_product_attention(
                q, k, v, attn_mask=mask, dropout_p=0, is_causal=mask is None and q.shape[-2] > 1,
                scale=module.scaling, enable_gqa=True).transpose(1, 2)
        return module.o_proj(output.reshape(*shape, -1).contiguous()), None

    for module in model.modules():
        if module.__class__.__name__ == 'LlamaAttention' and not hasattr(module, '_original_forward'):
            module._original_forward = module.forward
            module.forward = types.MethodType(forward, module)


# -- request batching (not in the reference) -------------------------------------
# The reference serves one request per GPUCache and launches pack and attention
# once per request and layer. These functions step B independent caches together:
# one pack launch and one attention launch per layer for all of them (in launches
# of at most K.MAX_REQUESTS requests), so the model around the cache runs its
# projections and MLP on B frames at once.

def _history(c, past):
    return K.History(c.p4.data_ptr(), c.m4.data_ptr(), c.p8.data_ptr(), c.m8.data_ptr(), c.p16.data_ptr(),
                     c.rows.data_ptr(), c.codes.data_ptr(), c.caps[4], c.caps[8], c.caps[16], past, c.capacity,
                     c.status.data_ptr())


def _pack_target(c, past, row, new_segment):
    return K.PackTarget(c.p4.data_ptr(), c.m4.data_ptr(), c.p8.data_ptr(), c.m8.data_ptr(), c.p16.data_ptr(),
                        c.caps[4], c.caps[8], c.caps[16], row, c.pending_bits, 0,
                        c.rows.data_ptr() if new_segment else None, c.codes.data_ptr() if new_segment else None,
                        past, c.capacity, c.status.data_ptr())


def _check_room(caches, layer, n):
    """Every cache can take n more tokens on `layer` (checked for all before any is
    claimed, so a batch that cannot proceed leaves every cache unchanged)."""
    for c in caches:
        if c.seen[layer] + n > c.capacity:
            raise ValueError('GPU context limit exceeded')


def _claim_all(caches, claim):
    """claim(c) for every cache, all or nothing: if one raises (a frame that does not
    match an offline plan, layers out of step), the caches claimed before it get their
    host bookkeeping back, so the batch leaves every cache as it was. Pools grown on
    the way stay grown (their rows are unchanged)."""
    saved, out = [], []
    try:
        for c in caches:
            saved.append((c, c.seen.copy(), c.cursors.copy(), c.plan.copy(), c.host_counts.copy()))
            out.append(claim(c))
    except Exception:
        for c, seen, cursors, plan, counts in saved:
            c.seen, c.cursors, c.plan, c.host_counts = seen, cursors, plan, counts
        raise
    return out


def _same_geometry(caches):
    if not caches:
        raise ValueError('no caches')
    first = caches[0]
    for c in caches:
        if (c.layers, c.heads, c.dim, c.device) != (first.layers, first.heads, first.dim, first.device):
            raise ValueError('batched caches must share layers, heads, head_dim and device')
    return first


def append_many(caches, k, v, layer):
    """Packs one frame per cache for `layer`: k / v [B, heads, n, dim], request r into
    caches[r] at that cache's selected precision (each one as GPUCache.append would:
    bit-identical pools and maps). Returns the history lengths before the frame."""
    first = _same_geometry(caches)
    b, n = len(caches), k.shape[-2]
    if k.shape[0] != b or v.shape[0] != b or k.shape[1] != first.heads or k.shape[-1] != first.dim \
            or k.device.type != 'cuda':
        raise ValueError('GPU cache requires CUDA, one frame per cache and the configured head dimension')
    if len({c.p16.data_ptr() for c in caches}) != b:
        # a cache listed twice, or forks of one cache (they write the same reserved rows)
        raise ValueError('batched appends need caches with their own pools')
    _check_room(caches, layer, n)
    claimed = _claim_all(caches, lambda c: c._claim(layer, n, fill_map=False))
    claims = [past for past, _, _ in claimed]
    targets = [_pack_target(c, past, row, c.online and layer == 0) for c, (past, _, row) in zip(caches, claimed)]
    for s in range(0, b, K.MAX_REQUESTS):
        e = min(s + K.MAX_REQUESTS, b)
        K.pack_rows_many(k[s:e], v[s:e], targets[s:e], layer, n, first.heads, first.dim, first.layers)
    for c, past in zip(caches, claims):
        c.seen[layer] = past + n
    return claims


def attend_many(caches, q, k, v, layer, pasts):
    """Causal GQA attention of each cache's n new queries over its own packed history
    (pasts[r] tokens) plus its own new K/V: q [B, query_heads, n, dim], k / v
    [B, heads, n, dim]; returns [B, n, query_heads, dim]."""
    first = _same_geometry(caches)
    b, hq, n, _ = q.shape
    if len(pasts) != b or hq % first.heads:
        raise ValueError('one past per cache; query heads must be a multiple of KV heads')
    out = torch.empty((b, n, hq, first.dim), dtype=q.dtype, device=q.device)
    hist = [_history(c, past) for c, past in zip(caches, pasts)]
    for s in range(0, b, K.MAX_REQUESTS):
        e = min(s + K.MAX_REQUESTS, b)
        K.packed_attention_many(q[s:e], k[s:e], v[s:e], hist[s:e], out[s:e], layer, n, first.heads,
                                hq // first.heads, first.dim, first.layers)
    return out


class RequestBatch:
    """Device-resident descriptors of B caches that append n-token frames together,
    for CUDA-graph replay of whole frame steps (not in the reference). The pack
    destinations (dkv_pack_target), histories (dkv_history) and rotary positions
    of the next step live in one device buffer that the *_many_device kernels
    read; `prepare()` does every cache's host bookkeeping for the step (the claims
    GPUCache.append makes on each layer, pool growth included) and refreshes the
    buffer with one stream-ordered copy from pinned memory. A graph captured over
    the kernels therefore replays correctly step after step. The histories are
    planned for at most `max_past` tokens (default: the caches' capacity). With
    append=False the steps attend without appending (query chunks side by side over
    their caches' histories, e.g. candidates over one fork): no claims, and one
    cache may appear several times."""

    def __init__(self, caches, n, max_past=None, append=True):
        first = _same_geometry(caches)
        if append and len({c.p16.data_ptr() for c in caches}) != len(caches):
            raise ValueError('batched appends need caches with their own pools')
        self.append = append
        self.caches, self.n, self.count = list(caches), n, len(caches)
        self.layers, self.heads, self.dim, self.device = first.layers, first.heads, first.dim, first.device
        self.max_past = max(c.capacity for c in caches) if max_past is None else max_past
        b = self.count
        self._hist_off = (b * ctypes.sizeof(K.PackTarget) + 255) // 256 * 256
        self._pos_off = (self._hist_off + b * ctypes.sizeof(K.History) + 255) // 256 * 256
        total = self._pos_off + b * n * 8
        self.host = torch.empty(total, dtype=torch.uint8).pin_memory()
        self.dev = torch.empty(total, dtype=torch.uint8, device=self.device)
        base = self.host.data_ptr()
        self._targets = (K.PackTarget * b).from_address(base)
        self._hists = (K.History * b).from_address(base + self._hist_off)
        self._positions = self.host[self._pos_off:].view(torch.int64).view(b, n)
        self.targets_ptr = self.dev.data_ptr()
        self.histories_ptr = self.dev.data_ptr() + self._hist_off
        self.positions = self.dev[self._pos_off:].view(torch.int64).view(b, n)  # [B, n] on the device
        self._copied = None
        self._ramp = torch.arange(n, dtype=torch.int64)

    def release(self):
        """Drops the references to the caches (the device buffer stays for the next
        rebind), so a kept batch does not hold finished requests' pools."""
        self.caches = []

    def rebind(self, caches):
        """Points the batch at another set of caches of the same count and geometry
        (a captured graph reads only the device buffer, so it serves them too)."""
        first = _same_geometry(caches)
        if len(caches) != self.count or (first.layers, first.heads, first.dim, first.device) != \
                (self.layers, self.heads, self.dim, self.device):
            raise ValueError('rebinding needs as many caches of the same geometry')
        if self.append and len({c.p16.data_ptr() for c in caches}) != len(caches):
            raise ValueError('batched appends need caches with their own pools')
        self.caches = list(caches)

    def prepare(self):
        """Claims the next n-token frame of every cache at its selected precision on
        all layers (append=False: takes each cache's history as it is) and writes the
        step's descriptors to the device (ordered on the current stream before
        whatever is launched next). Returns the pasts."""
        if len(self.caches) != self.count:
            raise ValueError('request batch has no caches bound (rebind before stepping)')
        if self.append:
            _check_room(self.caches, 0, self.n)
        if self._copied is not None:
            self._copied.synchronize()  # the previous step's copy has left the pinned buffer
        if self.append:
            claimed = _claim_all(self.caches, lambda c: c._claim_frame(self.n))
        else:
            claimed = [(c.seen[0], None) for c in self.caches]
            if any(x != c.seen[0] for c in self.caches for x in c.seen):
                raise ValueError('GPU cache layers disagree about the history length')
        pasts = []
        for r, (c, (past, row)) in enumerate(zip(self.caches, claimed)):
            if self.append:
                self._targets[r] = _pack_target(c, past, row, c.online)
            self._hists[r] = _history(c, past)
            self._positions[r] = self._ramp + past
            pasts.append(past)
        self.dev.copy_(self.host, non_blocking=True)
        self._copied = torch.cuda.Event()
        self._copied.record()
        return pasts
