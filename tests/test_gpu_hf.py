"""The reference's model integration (install_packed_attention, src/gpu_cache.py:
151-183) on a random-init HF Llama of the installed transformers: logits with a
16-bit GPUCache follow the stock cache (bf16 history + SDPA), and quantised frames
stay close; the per-layer append + attend is one fused call."""
import pytest
import torch

from src.gpu_cache import GPUCache, install_packed_attention
from test_host_api import _tiny_llama

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize('bits,tol', [(16, 0.05), (8, 0.15)])
def test_hf_llama_with_gpu_cache_matches_stock_cache(cuda, bits, tol):
    model = _tiny_llama().cuda()
    ids = torch.randint(0, 1000, (1, 128), generator=torch.Generator().manual_seed(3)).cuda()
    with torch.inference_mode():
        stock = model(ids[:, :64], use_cache=True)
        want = model(ids[:, 64:], past_key_values=stock.past_key_values, use_cache=True).logits.float()
        install_packed_attention(model)
        cache = GPUCache(None, layers=2, heads=2, device='cuda')
        cache.select(bits, 0)
        model(ids[:, :64], past_key_values=cache, use_cache=True)
        cache.select(16, 1)
        got = model(ids[:, 64:], past_key_values=cache, use_cache=True).logits.float()
    cache.check()
    assert cache.seen == [128, 128] and [seg[2] for seg in cache.plan] == [bits, 16]
    assert torch.isfinite(got).all()
    assert float((got - want).abs().max()) < tol * float(want.abs().max()), float((got - want).abs().max())
