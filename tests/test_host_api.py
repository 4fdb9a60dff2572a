"""CPU tests of the GPUCache host logic (plan, growth, fork, accounting), which
mirrors src/gpu_cache.py of the reference. Pools live on the CPU here; every
path that would launch a kernel is rejected before reaching the library."""
import pytest
import torch

from src.gpu_cache import GPUCache


def test_constructor_validation_messages():
    with pytest.raises(ValueError, match='head_dim=64'):
        GPUCache(dim=128, device='cpu')
    with pytest.raises(ValueError, match='Invalid GPU cache plan'):
        GPUCache([(5, 10)], device='cpu')
    with pytest.raises(ValueError, match='Invalid GPU cache plan'):
        GPUCache([(4, -1)], device='cpu')


def test_offline_plan_rows_codes_and_caps():
    c = GPUCache([(4, 20), (16, 10), (4, 5), (8, 3)], layers=2, device='cpu')
    assert c.plan == [(0, 20, 4, 0), (20, 30, 16, 0), (30, 35, 4, 20), (35, 38, 8, 0)]
    assert c.rows.tolist() == list(range(20)) + list(range(10)) + list(range(20, 25)) + list(range(3))
    assert c.codes.tolist() == [4] * 20 + [16] * 10 + [4] * 5 + [8] * 3
    assert c.caps == {4: 25, 8: 3, 16: 10} and c.capacity == 38
    # paged pools: [pages, layers, 2, heads, 64, width], ceil(cap / 64) pages
    assert c.p4.shape == (1, 2, 2, 3, 64, 32) and c.m8.shape == (1, 2, 2, 3, 64, 2)
    assert c.p16.dtype == torch.bfloat16 and len(c) == 2 and c.get_seq_length() == 0


def test_online_growth_policy_matches_reference():
    c = GPUCache(None, layers=1, device='cpu', max_tokens=512)
    assert c.caps == {4: 64, 8: 64, 16: 64} and c.capacity == 512
    sentinel = torch.arange(c.p4.numel(), dtype=torch.int64).remainder(251).to(torch.uint8).view(c.p4.shape)
    c.p4.copy_(sentinel)
    c.reserve(4, 79)           # max(79, ceil64(96)) = 128
    assert c.caps[4] == 128 and c.p4.shape[0] == 2 and c.m4.shape[0] == 2  # pages of 64 rows
    assert torch.equal(c.p4[:1], sentinel)  # old rows kept: growth appends pages
    c.reserve(4, 167)          # max(167, ceil64(192)) = 192
    assert c.caps[4] == 192 and c.p4.shape[0] == 3
    c.reserve(4, 100)          # no shrink / no-op
    assert c.caps[4] == 192
    c.reserve(16, 400)         # needed beats 1.5x
    assert c.caps[16] == 400 and c.p16.shape[0] == 7


def test_pool_rows_read_and_write_in_reference_terms():
    c = GPUCache(None, layers=2, heads=3, device='cpu', max_tokens=512)
    c.reserve(8, 200)
    rows = torch.arange(3 * 150 * 64, dtype=torch.int64).remainder(253).to(torch.uint8).view(3, 150, 64)
    c.write_pool_rows('p8', 1, 1, 30, rows)  # rows 30..179: across pages 0, 1, 2
    assert torch.equal(c.pool_rows('p8', 1, 1, 30, 150), rows)
    assert torch.equal(c.p8[1, 1, 1, :, 0], rows[:, 34])  # row 64 = page 1, slot 0
    assert torch.equal(c.p8[2, 1, 1, :, 51], rows[:, 149])  # row 179 = page 2, slot 51


def test_append_requires_cuda_and_batch_one():
    c = GPUCache(None, layers=1, device='cpu')
    x = torch.zeros(1, 3, 4, 64, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match='requires CUDA'):
        c.append(x, x, 0)
    with pytest.raises(ValueError, match='requires CUDA'):
        c.append(torch.zeros(2, 3, 4, 64), torch.zeros(2, 3, 4, 64), 0)


def test_fork_copies_host_state_and_shares_pools():
    c = GPUCache([(4, 20), (16, 10)], layers=1, device='cpu')
    c.seen[0] = 20
    c.select(4, 3)
    b = c.fork()
    assert b.pending_bits == 16 and c.pending_bits == 4 and c.frame_id == 3
    b.seen[0] = 25
    b.caps[16] = 999
    b.plan.append((99, 100, 16, 0))
    b.host_counts[16] += 5
    assert c.seen[0] == 20 and c.caps[16] == 10 and len(c.plan) == 2 and c.host_counts[16] == 10
    assert b.p4 is c.p4 and b.rows is c.rows  # pools and maps are shared, as in the reference


def test_accounting_matches_reference_audit_formulas():
    # scripts/gpu_validate.py:61-70 formulas, L=32, H=5
    c = GPUCache(None, layers=32, heads=5, device='cpu')
    plan = [(16, 11), (4, 64), (8, 64), (16, 64), (4, 64)]
    for bits, n in plan:
        row = c.host_counts[bits]
        c.reserve(bits, row + n)
        c.plan.append((c.seen[0], c.seen[0] + n, bits, row))
        c.host_counts[bits] += n
        c.seen = [s + n for s in c.seen]
    a = c.accounting()
    tokens = {4: 128, 8: 64, 16: 75}
    used = sum(tokens.values())
    assert a['precision_token_counts'] == tokens and a['used_tokens'] == used
    assert a['payload_bytes'] == 32 * 2 * 5 * 64 * sum(tokens[b] * b / 8 for b in tokens)
    assert a['quantization_metadata_bytes'] == 32 * 2 * 5 * 8 * (tokens[4] + tokens[8])
    assert a['token_mapping_bytes'] == used * 5
    assert a['gpu_cache_used_bytes'] == a['payload_bytes'] + a['quantization_metadata_bytes'] + used * 5
    caps = a['precision_pool_capacities']
    assert a['gpu_cache_allocated_bytes'] == 32 * 2 * 5 * (40 * caps[4] + 72 * caps[8] + 128 * caps[16]) + 8192 * 5
    assert a['cpu_cache_payload_bytes'] == 0


def test_non_bf16_pool_dtype_is_rejected():
    with pytest.raises(ValueError, match='bfloat16'):
        GPUCache(device='cpu', dtype=torch.float16)


def _layer_by_layer(c, n):
    rows = [c._claim(layer, n, fill_map=False)[2] for layer in range(c.layers)]
    past = c.seen[0]
    c.seen = [past + n] * c.layers
    return past, rows


def test_claim_frame_equals_the_claims_of_every_layer_offline():
    plan = [(4, 64), (16, 64), (8, 30), (8, 34), (4, 64)]
    a = GPUCache(plan, layers=3, device='cpu')
    b = GPUCache(plan, layers=3, device='cpu')
    for bits, n in [(4, 64), (16, 64), (8, 30), (8, 34), (4, 64)]:
        a.select(bits), b.select(bits)
        past, row = a._claim_frame(n)
        past_b, rows = _layer_by_layer(b, n)
        assert past == past_b and rows == [row] * 3
        assert a.seen == b.seen and a.cursors == b.cursors
    with pytest.raises(ValueError, match='context limit'):
        a._claim_frame(1)


def test_claim_frame_online_grows_and_records_the_segment_once():
    a = GPUCache(None, layers=4, device='cpu', max_tokens=512)
    for i, bits in enumerate([4, 8, 4, 16, 4]):
        a.select(bits, i)
        past, row = a._claim_frame(64)
        assert past == 64 * i and a.seen == [64 * (i + 1)] * 4
        assert a.plan[-1] == (past, past + 64, bits, row)
    assert a.host_counts == {4: 192, 8: 64, 16: 64}
    assert a.caps[4] >= 192 and a.p4.shape[0] == (a.caps[4] + 63) // 64
    with pytest.raises(ValueError, match='Cache append does not match plan|context limit'):
        a._claim_frame(512)


def test_claim_frame_rejects_layers_out_of_step():
    a = GPUCache(None, layers=2, device='cpu', max_tokens=512)
    a.seen = [64, 0]
    with pytest.raises(ValueError, match='disagree'):
        a._claim_frame(64)


def _tiny_llama():
    from transformers import LlamaConfig, LlamaForCausalLM
    cfg = LlamaConfig(hidden_size=384, num_attention_heads=6, num_key_value_heads=2, intermediate_size=512,
                      vocab_size=1000, num_hidden_layers=2, head_dim=64)
    torch.manual_seed(0)
    return LlamaForCausalLM(cfg).to(torch.bfloat16)


def test_hf_llama_forward_reaches_the_packed_attention():
    """install_packed_attention on the installed transformers: the model's mask
    and cache bookkeeping accept a GPUCache up to the kernel call (which needs CUDA)."""
    from src.gpu_cache import install_packed_attention
    model = _tiny_llama()
    install_packed_attention(model)
    cache = GPUCache(None, layers=2, heads=2, device='cpu')
    with pytest.raises(ValueError, match='requires CUDA'):
        model(torch.randint(0, 1000, (1, 64)), past_key_values=cache, use_cache=True)
    assert cache.get_mask_sizes(64, 0) == (64, 0) and cache.is_sliding == [False, False]


def test_a_batch_over_the_context_limit_leaves_every_cache_unchanged():
    from src.gpu_cache import _check_room
    a = GPUCache(None, layers=2, device='cpu', max_tokens=256)
    b = GPUCache(None, layers=2, device='cpu', max_tokens=128)
    for c in (a, b):
        c.select(4, 0)
        c._claim_frame(64)
    with pytest.raises(ValueError, match='context limit'):
        _check_room([a, b], 0, 65)
    assert a.seen == [64, 64] and b.seen == [64, 64] and len(a.plan) == len(b.plan) == 1
    _check_room([a, b], 0, 64)


def test_install_fused_ops_joins_weights_and_keeps_the_forward():
    """install_fused_ops (src/gpu_ops.py:19-48): the QKV and gate/up weights become
    views of one joined tensor each (same values, no second copy), and the fused
    RMSNorm / MLP forwards give the original forwards' results (CPU, fp32: the
    reference's PyTorch form of the ops)."""
    from src.gpu_ops import install_fused_ops
    model = _tiny_llama().float()
    ids = torch.randint(0, 1000, (1, 17))
    with torch.no_grad():
        expected = model(ids).logits
    before = {n: p.detach().clone() for n, p in model.named_parameters()}
    state = {'enabled': True}
    install_fused_ops(model.model, state)
    for name, p in model.named_parameters():
        assert torch.equal(p, before[name]), name
    attn, mlp = model.model.layers[0].self_attn, model.model.layers[0].mlp
    assert attn.q_proj.weight.data_ptr() == attn._qkv_weight.data_ptr()
    assert attn.v_proj.weight.data_ptr() == attn._qkv_weight[-attn.v_proj.out_features:].data_ptr()
    assert mlp.up_proj.weight.data_ptr() == mlp._gate_up_weight[mlp.gate_proj.out_features:].data_ptr()
    with torch.no_grad():
        fused = model(ids).logits
        state['enabled'] = False
        original = model(ids).logits
    assert torch.allclose(fused, expected, atol=1e-4, rtol=1e-4)
    assert torch.equal(original, expected)


def test_a_batch_claim_that_fails_leaves_every_cache_unchanged():
    """Batched appends claim all caches or none: a cache whose offline plan does
    not match the frame undoes the claims already made for the others."""
    from src.gpu_cache import _claim_all
    a = GPUCache(None, layers=2, device='cpu', max_tokens=512)
    b = GPUCache(None, layers=2, device='cpu', max_tokens=512)
    bad = GPUCache([(16, 64)], layers=2, device='cpu')
    for c in (a, b, bad):
        c.select(4, 0)
    with pytest.raises(ValueError, match='does not match plan'):
        _claim_all([a, b, bad], lambda c: c._claim_frame(64))
    for c in (a, b):
        assert c.seen == [0, 0] and c.plan == [] and c.host_counts == {4: 0, 8: 0, 16: 0}
    assert bad.seen == [0, 0] and bad.cursors == [0, 0]
    bad.select(16, 0)
    claimed = _claim_all([a, b, bad], lambda c: c._claim_frame(64))
    assert claimed == [(0, 0), (0, 0), (0, 0)]
    assert a.seen == b.seen == bad.seen == [64, 64] and a.plan == [(0, 64, 4, 0)] and a.host_counts[4] == 64


def test_request_descriptors_carry_the_cache_state():
    """The per-request descriptors the batched kernels read (dkv_history,
    dkv_pack_target) hold the cache's own pools, maps, capacities and lengths."""
    from src.gpu_cache import _history, _pack_target
    c = GPUCache(None, layers=2, device='cpu', max_tokens=512)
    c.select(8, 0)
    past, row = c._claim_frame(64)
    h = _history(c, past)
    assert (h.p4, h.m4, h.p8, h.m8, h.p16) == tuple(t.data_ptr() for t in c._pools())
    assert (h.rows, h.codes) == (c.rows.data_ptr(), c.codes.data_ptr())
    assert (h.cap4, h.cap8, h.cap16, h.past, h.capacity) == (c.caps[4], c.caps[8], c.caps[16], 0, 512)
    assert h.status == c.status.data_ptr()
    t = _pack_target(c, past, row, True)
    assert (t.bits, t.row_start, t.map_start, t.map_capacity) == (8, 0, 0, 512)
    assert (t.map_rows, t.map_codes) == (c.rows.data_ptr(), c.codes.data_ptr())
    t = _pack_target(c, past, row, False)
    assert t.map_rows is None and t.map_codes is None
