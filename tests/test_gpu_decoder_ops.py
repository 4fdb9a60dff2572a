"""GPU checks of the decoder's pointwise kernels (dkv_rotary, dkv_silu_mul): each is
bit-identical to the PyTorch ops it replaces, on the layouts the decoder hands them
(strided head views of the joined projection, broadcast rotary tables, the two halves
of the joined gate/up projection) and on extreme values."""
import pytest
import torch

from src import gpu_kernels as K
from src.decoder import SMOLLM2_360M, apply_rope, rope_tables

pytestmark = pytest.mark.gpu


def _tables(b, n, shared, gen):
    cfg = SMOLLM2_360M
    rows = 1 if shared else b
    positions = torch.randint(0, 8192, (rows * n,), generator=gen).cuda()
    cos, sin = rope_tables(cfg, positions, 'cuda')
    return cos.view(rows, n, 1, -1), sin.view(rows, n, 1, -1)


@pytest.mark.parametrize('b,n,shared', [(1, 1, False), (1, 64, False), (8, 64, False), (4, 7, True),
                                        (3, 33, False)])
def test_rotary_is_bit_identical_to_the_fp32_torch_form(cuda, b, n, shared):
    gen = torch.Generator().manual_seed(100 * b + n)
    heads, extra = 20, 5  # q and k heads of the joined projection, v heads left untouched
    h = (torch.randn(b, n, heads + extra, 64, generator=gen) * 3).bfloat16().cuda()
    cos, sin = _tables(b, n, shared, gen)
    expected = apply_rope(h[:, :, :heads], cos, sin)
    actual = K.rotary(h, cos, sin, heads)
    assert actual.shape == (b, n, heads, 64) and actual.is_contiguous()
    assert torch.equal(actual.view(torch.int16), expected.contiguous().view(torch.int16))


def test_rotary_rejects_bad_tables(cuda):
    h = torch.randn(2, 4, 8, 64, device='cuda').bfloat16()
    cos = torch.ones(3, 4, 1, 64, device='cuda')
    with pytest.raises(ValueError):
        K.rotary(h, cos, cos, 8)
    with pytest.raises(ValueError):
        K.rotary(h, cos.half(), cos.half(), 8)


@pytest.mark.parametrize('shape', [(1, 23, 2560), (8, 64, 2560), (1, 1, 64), (3, 5, 8)])
def test_silu_mul_is_bit_identical_to_torch(cuda, shape):
    gen = torch.Generator().manual_seed(sum(shape))
    joined = (torch.randn(*shape[:-1], 2 * shape[-1], generator=gen) * 4).bfloat16().cuda()
    gate, up = joined.chunk(2, -1)
    expected = torch.nn.functional.silu(gate) * up
    actual = K.silu_mul(gate, up)
    assert actual.shape == gate.shape and actual.is_contiguous()
    assert torch.equal(actual.view(torch.int16), expected.view(torch.int16))
    # separate contiguous operands, as HF's MLP may hand them over
    gate, up = gate.contiguous(), up.contiguous()
    assert torch.equal(K.silu_mul(gate, up).view(torch.int16), expected.view(torch.int16))


def test_silu_mul_extreme_values(cuda):
    vals = [0.0, -0.0, 1e-30, -1e-30, 20.0, -20.0, 88.0, -88.0, 90.0, -90.0, 1e4, -1e4, 3e38, -3e38, 0.5, -0.5]
    gate = torch.tensor(vals * 8, device='cuda').bfloat16().view(1, -1)
    up = torch.linspace(-3, 3, gate.numel(), device='cuda').bfloat16().view(1, -1)
    expected = torch.nn.functional.silu(gate) * up
    assert torch.equal(K.silu_mul(gate, up).view(torch.int16), expected.view(torch.int16))


def test_activation_product_routes_cuda_bf16_to_the_kernel(cuda):
    from src.gpu_ops import activation_product
    joined = torch.randn(2, 9, 1024, device='cuda').bfloat16()
    gate, up = joined.chunk(2, -1)
    assert torch.equal(activation_product(gate, up).view(torch.int16),
                       (torch.nn.functional.silu(gate) * up).view(torch.int16))
    g32, u32 = gate.float(), up.float()  # other dtypes keep the reference's PyTorch form
    assert torch.equal(activation_product(g32, u32), torch.nn.functional.silu(g32) * u32)


@pytest.mark.parametrize('shape', [(8, 64, 960), (1, 25, 960), (1, 1, 64), (3, 7, 2048)])
def test_add_rms_norm_against_torch(cuda, shape):
    """x + y is PyTorch's bf16 add bit for bit; the norm keeps PyTorch's rounding points
    and, its fp32 sum of squares running in another order, differs from
    rms_norm(x + y) * w by at most one bf16 unit after the norm and one more after the
    weight product (2 units in the last place), on every element."""
    from src.gpu_ops import add_rms
    gen = torch.Generator().manual_seed(sum(shape))
    x = (torch.randn(*shape, generator=gen) * 3).bfloat16().cuda()
    y = (torch.randn(*shape, generator=gen) * 3).bfloat16().cuda()
    w = (1 + 0.1 * torch.randn(shape[-1], generator=gen)).bfloat16().cuda()
    s, h = add_rms(x, y, w, 1e-5)
    ref_s = x + y
    ref_h = torch.nn.functional.rms_norm(ref_s, (shape[-1],), None, 1e-5) * w
    assert torch.equal(s.view(torch.int16), ref_s.view(torch.int16))
    ulps = (h.view(torch.int16).int() - ref_h.view(torch.int16).int()).abs()
    assert int(ulps.max()) <= 2, int(ulps.max())
    s2, h2 = add_rms(x, None, w, 1e-5)  # no add: the norm of x itself
    assert s2 is x
    ref2 = torch.nn.functional.rms_norm(x, (shape[-1],), None, 1e-5) * w
    assert int((h2.view(torch.int16).int() - ref2.view(torch.int16).int()).abs().max()) <= 2


def test_add_rms_norm_rejects_bad_widths(cuda):
    from src import gpu_kernels as K
    x = torch.zeros(2, 4100, device='cuda').bfloat16()
    with pytest.raises(ValueError, match='width'):
        K.FAST.add_rms_norm(x, None, torch.ones(4100, device='cuda').bfloat16(), 1e-5)
