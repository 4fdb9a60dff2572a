"""Decoder-side engine ops kept from the reference's src/gpu_ops.py.

The reference joins the QKV and gate/up projection weights into single GEMMs
and runs RMSNorm / SiLU*up as prebuilt PyTorch CUDA ops (src/gpu_ops.py:9-48).
The GEMMs and the RMSNorm stay on PyTorch here; SiLU*up on CUDA bf16 tensors is
one libdkv launch (dkv_silu_mul, bit-identical to the two PyTorch ops it
replaces), and other dtypes / devices keep the reference's PyTorch form. The API
and the weight-joining invariants (bit-identical parameter views over one joined
tensor) are the same.
"""
import types

import torch

from . import gpu_kernels as K


def cuda_rms(x, weight, eps):
    """RMSNorm with the bf16 rounding before the weight multiply (src/gpu_ops.py:9-12)."""
    return torch.nn.functional.rms_norm(x, (x.shape[-1],), None, eps) * weight


def add_rms(x, y, weight, eps):
    """(x + y, RMSNorm(x + y) * weight), or (x, RMSNorm(x) * weight) when y is None:
    the decoder layer's residual add and the next norm. On CUDA bf16 one
    dkv_add_rms_norm launch (PyTorch's rounding points, its own fp32 reduction
    order: the norm can differ from cuda_rms in the last bf16 bit); elsewhere the
    PyTorch ops. Not in the reference, whose decoder makes the add and cuda_rms
    separate calls."""
    if x.is_cuda and x.dtype == torch.bfloat16 and weight.dtype == torch.bfloat16 and x.shape[-1] <= 2048 \
            and x.shape[-1] % 8 == 0:
        out = K.FAST.add_rms_norm(x, y, weight, eps)
        return out[0], out[1]
    if y is not None:
        x = x + y
    return x, cuda_rms(x, weight, eps)


def activation_product(gate, up):
    """silu(gate) * up (src/gpu_ops.py:14-17): one dkv_silu_mul launch for CUDA bf16
    tensors, the reference's PyTorch form otherwise."""
    if gate.is_cuda and gate.dtype == torch.bfloat16 and up.dtype == torch.bfloat16 and gate.shape == up.shape:
        return K.silu_mul(gate, up)
    return torch.nn.functional.silu(gate) * up


def join_weights(modules):
    """Concatenates the weights of `modules` along dim 0 and re-points each module's
    weight at its slice of the joined tensor, so no second copy is kept and every
    projection stays bit-identical (src/gpu_ops.py:26-37)."""
    with torch.no_grad():
        joined = torch.cat([m.weight for m in modules], dim=0)
        offset = 0
        for m in modules:
            n = m.weight.shape[0]
            view = joined[offset:offset + n]
            if not torch.equal(view, m.weight):
                raise AssertionError('Projection values changed during packing')
            m.weight = torch.nn.Parameter(view, requires_grad=False)
            offset += n
    return joined


def install_fused_ops(text, state):
    """Patches LlamaRMSNorm / LlamaMLP forwards and joins projection weights of an
    HF Llama text model; `state['enabled']` switches the fused forms on
    (src/gpu_ops.py:19-48)."""
    def rms_forward(module, x):
        return cuda_rms(x, module.weight, module.variance_epsilon) if state['enabled'] else module._original_rms(x)

    def mlp_forward(module, x):
        if not state['enabled']:
            return module._original_mlp(x)
        gate, up = torch.nn.functional.linear(x, module._gate_up_weight).chunk(2, dim=-1)
        return module.down_proj(activation_product(gate, up))

    for module in text.modules():
        name = module.__class__.__name__
        if name == 'LlamaAttention' and all(m.bias is None for m in [module.q_proj, module.k_proj, module.v_proj]):
            module._qkv_weight = join_weights([module.q_proj, module.k_proj, module.v_proj])
            module._qkv_sizes = [module.q_proj.out_features, module.k_proj.out_features,
                                 module.v_proj.out_features]
        elif name == 'LlamaRMSNorm':
            module._original_rms = module.forward
            module.forward = types.MethodType(rms_forward, module)
        elif name == 'LlamaMLP' and text.config.hidden_act == 'silu':
            module._gate_up_weight = join_weights([module.gate_proj, module.up_proj])
            module._original_mlp = module.forward
            module.forward = types.MethodType(mlp_forward, module)
