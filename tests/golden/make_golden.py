"""Generates the golden fixtures in this directory FROM THE REFERENCE ITSELF.

    python tests/golden/make_golden.py --reference <checkout of zoaibs/Dynamic-KV-Cache>

Two sources, both the reference's own code, imported from the checkout:
  * src/kv_quantization.py `pack` (the CPU quantiser, src/kv_quantization.py:41-77)
    on seeded inputs -> pack_golden.npz (payload, scales, offsets, header per case);
  * src/gpu_kernels.py `packed_attention` and `reconstruct` (the reference's
    Triton kernels, src/gpu_kernels.py:71-119) executed by the Triton CPU
    interpreter (TRITON_INTERPRET=1) over pools filled with the reference
    quantiser's output -> attn_<case>.npz. The interpreter needs fp32 q/k/v, so
    the inputs are drawn in bf16 and widened exactly: the GPU path sees the same
    values in bf16.
The reference checkout is needed only to regenerate; the fixtures are committed.
"""
import argparse
import importlib.util
import os
import sys
from pathlib import Path

os.environ['TRITON_INTERPRET'] = '1'  # must precede the first triton import

import numpy as np
import torch

OUT = Path(__file__).resolve().parent
ROW_BYTES = {4: 32, 8: 64, 16: 128}


def load_module(path, name):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def outlier_kv(gen, heads, n, outliers):
    """K ~ N(0,1) with the 4 seeded outlier channels scaled 8x, V ~ N(0,1), in bf16."""
    k = torch.randn(1, heads, n, 64, generator=gen)
    k[..., outliers] *= 8
    v = torch.randn(1, heads, n, 64, generator=gen)
    return k.bfloat16(), v.bfloat16()


def bits_of(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def pack_cases():
    gen = torch.Generator().manual_seed(20261201)
    outliers = torch.randperm(64, generator=gen)[:4]
    k, v = outlier_kv(gen, 5, 64, outliers)
    cases = {'c2_k': k, 'c2_v': v}
    g71 = torch.Generator().manual_seed(71)
    cases['ref19'] = torch.randn((1, 3, 19, 64), generator=g71).bfloat16()
    g10 = torch.Generator().manual_seed(10)
    cases['odd65_f32'] = torch.randn(1, 3, 7, 65, generator=g10)
    cases['const_f32'] = torch.full((1, 1, 3, 17), -2.5)
    # Exact half-step ties: span 15 (scale 1 for 4 bits) and values k + 0.5.
    ties = torch.zeros(1, 2, 2, 64)
    ties[0, 0, 0] = torch.arange(64) % 14 + 0.5  # 0.5, 1.5, 2.5, ... 13.5
    ties[0, 0, 0, 0], ties[0, 0, 0, 1] = 0.0, 15.0
    ties[0, 0, 1] = (torch.arange(64) * 4 + 0.5).clamp(max=255.0)  # ties for the 8-bit path
    ties[0, 0, 1, 0] = 0.0
    ties[0, 1, 0] = 7.0                           # constant row (zero span)
    ties[0, 1, 1] = torch.linspace(-1e38, 1e38, 64)  # huge but finite span
    cases['ties'] = ties.bfloat16()
    tiny = torch.randn(1, 2, 3, 64, generator=gen) * 1e-38  # subnormal fp32 magnitudes
    cases['tiny'] = tiny.bfloat16()
    return cases


def make_pack_golden(kvq):
    arrays = {}
    for name, x in pack_cases().items():
        dtype = 'bfloat16' if x.dtype == torch.bfloat16 else 'float32'
        arrays[f'{name}__x'] = bits_of(x) if dtype == 'bfloat16' else x.numpy()
        arrays[f'{name}__dtype'] = np.array(dtype)
        for bits in (4, 8, 16):
            p = kvq.pack(x, bits, 64)
            arrays[f'{name}__{bits}__payload'] = p.payload.numpy()
            arrays[f'{name}__{bits}__scales'] = p.scales.numpy()
            arrays[f'{name}__{bits}__offsets'] = p.offsets.numpy()
            arrays[f'{name}__{bits}__header'] = p.header.numpy()
    np.savez_compressed(OUT / 'pack_golden.npz', **arrays)
    print('pack_golden.npz', len(arrays), 'arrays')


ATTN_CASES = {
    # name: (kv heads, group, [(bits, tokens) per stored frame], query length, seed)
    'mixed94': (5, 3, [(4, 40), (8, 24), (16, 30)], 16, 101),
    'aligned256': (5, 3, [(8, 64), (4, 64), (16, 64), (4, 64)], 64, 102),
    'plan9q': (3, 3, [(4, 15), (8, 67)], 23, 103),
    'decode256': (5, 3, [(4, 131), (8, 125)], 1, 104),
    'empty': (5, 3, [], 19, 105),
}
LAYERS, LAYER = 2, 1  # data lives in layer 1 of a 2-layer cache (exercises layer offsets)


def make_attention_golden(kvq, kernels, name, spec):
    heads, group, frames, nq, seed = spec
    gen = torch.Generator().manual_seed(seed)
    outliers = torch.randperm(64, generator=gen)[:4]
    counts = {4: 0, 8: 0, 16: 0}
    rows, codes, hk, hv, plan = [], [], [], [], []
    for bits, n in frames:
        k, v = outlier_kv(gen, heads, n, outliers)
        hk.append(k)
        hv.append(v)
        plan.append((bits, n, counts[bits]))
        rows.extend(range(counts[bits], counts[bits] + n))
        codes.extend([bits] * n)
        counts[bits] += n
    caps = {b: max(1, c) for b, c in counts.items()}
    common = (LAYERS, 2, heads)
    p4 = torch.zeros(*common, caps[4], 32, dtype=torch.uint8)
    m4 = torch.zeros(*common, caps[4], 2)
    p8 = torch.zeros(*common, caps[8], 64, dtype=torch.uint8)
    m8 = torch.zeros(*common, caps[8], 2)
    p16 = torch.zeros(*common, caps[16], 64, dtype=torch.bfloat16)
    for (bits, n, row0), k, v in zip(plan, hk, hv):
        for kv, x in enumerate((k, v)):
            p = kvq.pack(x, bits, 64)
            if bits == 16:
                p16[LAYER, kv, :, row0:row0 + n] = p.payload.view(torch.bfloat16).reshape(heads, n, 64)
                continue
            payload = p.payload.reshape(heads, n, ROW_BYTES[bits])
            meta = torch.stack((p.offsets, p.scales), -1).reshape(heads, n, 2)
            (p4 if bits == 4 else p8)[LAYER, kv, :, row0:row0 + n] = payload
            (m4 if bits == 4 else m8)[LAYER, kv, :, row0:row0 + n] = meta
    past = len(rows)
    rows_t = torch.tensor(rows or [0], dtype=torch.int32)
    codes_t = torch.tensor(codes or [16], dtype=torch.uint8)
    q = torch.randn(1, heads * group, nq, 64, generator=gen).bfloat16()
    kn, vn = outlier_kv(gen, heads, nq, outliers)
    qf, kf, vf = q.float(), kn.float(), vn.float()
    out = torch.empty(1, nq, heads * group, 64)
    bm, bn = 16, 64
    kernels.packed_attention[(heads * group, (nq + bm - 1) // bm)](
        qf, kf, vf, p4, m4, p8, m8, p16, rows_t, codes_t, out,
        qf.stride(1), qf.stride(2), kf.stride(1), kf.stride(2), vf.stride(1), vf.stride(2),
        LAYER, past, nq, caps[4], caps[8], caps[16], heads, group, 64, bm, bn)
    arrays = dict(heads=np.array(heads), group=np.array(group), nq=np.array(nq), layers=np.array(LAYERS),
                  layer=np.array(LAYER), frame_bits=np.array([b for b, _ in frames], np.int32),
                  frame_tokens=np.array([n for _, n in frames], np.int32),
                  q=bits_of(q), knew=bits_of(kn), vnew=bits_of(vn), out=out.numpy())
    if past:
        arrays['hist_k'] = bits_of(torch.cat(hk, 2))
        arrays['hist_v'] = bits_of(torch.cat(hv, 2))
    if 0 < past <= 128:  # reconstruct goldens only for the small cases (fixture size)
        recon = torch.empty(2, heads, past, 64)
        kernels.reconstruct[(heads, 2, (past + 31) // 32)](
            p4, m4, p8, m8, p16, rows_t, codes_t, recon, LAYER, past,
            caps[4], caps[8], caps[16], heads, 64, 32)
        arrays['recon'] = recon.numpy()
    np.savez_compressed(OUT / f'attn_{name}.npz', **arrays)
    print(f'attn_{name}.npz past={past} nq={nq}')


def main():
    parser = argparse.ArgumentParser()
    parser.add_argument('--reference', required=True, help='checkout of zoaibs/Dynamic-KV-Cache')
    args = parser.parse_args()
    src = Path(args.reference) / 'src'
    kvq = load_module(src / 'kv_quantization.py', 'reference_kv_quantization')
    kernels = load_module(src / 'gpu_kernels.py', 'reference_gpu_kernels')
    make_pack_golden(kvq)
    for name, spec in ATTN_CASES.items():
        make_attention_golden(kvq, kernels, name, spec)


if __name__ == '__main__':
    sys.exit(main())
