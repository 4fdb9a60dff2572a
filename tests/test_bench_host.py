"""CPU checks of bench.py's reference arm: the JSON line the driver reads (same
metric, unit and direction as the GPU arm, a cpu_baseline block and a host-only
e2e block), and the other ranks of a torchrun launch leaving without output."""
import json
import os
import subprocess
import sys

from conftest import ROOT


def _run(env_extra):
    env = dict(os.environ, **env_extra)
    cmd = [sys.executable, str(ROOT / 'bench.py'), '--impl', 'reference', '--steps', '2', '--warmup', '1',
           '--cpu-seconds', '1']
    return subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)


def test_reference_arm_prints_one_contract_line():
    res = _run({})
    assert res.returncode == 0, res.stderr[-2000:]
    lines = [ln for ln in res.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1
    line = json.loads(lines[0])
    for key in ('metric', 'value', 'unit', 'n_gpus', 'steps', 'warmup', 'higher_is_better', 'scaling', 'vs_baseline',
                'dtype', 'data', 'config', 'cpu_baseline', 'e2e'):
        assert key in line, key
    assert line['impl'] == 'reference' and line['unit'] == 'GB/s' and line['higher_is_better'] is True
    assert line['steps'] == 2 and line['warmup'] == 1 and line['value'] > 0
    base = line['cpu_baseline']
    assert base['kind'] == 'port' and base['cores'] >= 1 and base['value'] == line['value'] and base['sample']
    assert line['e2e'] == {'value': line['value'], 'unit': 'GB/s', 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0}
    assert 'workload' in line['config']


def test_reference_arm_other_ranks_exit_quietly():
    res = _run({'RANK': '1', 'WORLD_SIZE': '2', 'LOCAL_RANK': '1'})
    assert res.returncode == 0, res.stderr[-2000:]
    assert res.stdout.strip() == ''
