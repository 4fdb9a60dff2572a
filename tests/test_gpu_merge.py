"""The split merge: in the combine kernel for attend-only calls by default (or
everywhere with DKV_ATTENTION_MERGE=combine), inside the tensor-core kernel for
fused append + attend calls, and for every call with DKV_ATTENTION_MERGE=kernel,
when the grid is resident at once. All must give the same bits, and the
workspace's arrival counters must be back at zero after every call."""
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

from dkv_merge_cases import CASES, run_case

pytestmark = pytest.mark.gpu


def test_in_kernel_merge_is_bit_identical_to_combine_kernel(cuda, tmp_path):
    path = tmp_path / 'kernel.npz'
    env = dict(os.environ, DKV_ATTENTION_MERGE='kernel')
    script = os.path.join(os.path.dirname(__file__), 'dkv_merge_cases.py')
    subprocess.run([sys.executable, script, str(path)], env=env, check=True, timeout=600)
    ref = np.load(path)
    for i, case in enumerate(CASES):
        out, launches = run_case(*case)
        assert launches == 2, case  # default: attend-only calls merge in the combine kernel
        assert int(ref[f'launches{i}']) == 1, case  # 148-SM B200: every planned grid is resident at once
        assert np.array_equal(out.view(torch.int16).cpu().numpy(), ref[f'out{i}']), case
        fused, _ = run_case(*case, fused=True)  # in-kernel merge in this process too
        assert torch.equal(fused, out), case


def test_merge_counters_return_to_zero(cuda):
    from src import gpu_kernels as K
    for case in CASES[:3]:  # fused calls: merged inside the attention kernel
        run_case(*case, fused=True)
        run_case(*case, seed=1, fused=True)
    torch.cuda.synchronize()
    ws = K._workspace(torch.device('cuda', torch.cuda.current_device()), None, 1)  # this stream's workspace
    assert int(ws[:1024].count_nonzero()) == 0
