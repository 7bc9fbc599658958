"""CPU tests of bench.py's reference arm (the reference's own CPU kernels,
engine/native_quant.cpp built into oracle/_ref, or the oracle port): one JSON
line with the contract's keys on rank 0, nothing and exit 0 on other ranks."""
import json
import os
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def run(env_extra, *args):
    env = dict(os.environ, **env_extra)
    return subprocess.run([sys.executable, str(ROOT / 'bench.py'), '--impl', 'reference', *args], env=env,
                          capture_output=True, text=True, timeout=600, cwd=str(ROOT))


def test_reference_arm_json_line():
    p = run({'RANK': '0'}, '--steps', '1', '--warmup', '3', '--cpu-tokens', '32')
    assert p.returncode == 0, p.stderr[-2000:]
    lines = [l for l in p.stdout.splitlines() if l.strip().startswith('{')]
    assert len(lines) == 1
    d = json.loads(lines[0])
    for key in ('impl', 'metric', 'value', 'unit', 'n_gpus', 'steps', 'warmup', 'ms_per_step', 'higher_is_better',
                'scaling', 'vs_baseline', 'dtype', 'data', 'config', 'cpu_baseline', 'e2e'):
        assert key in d, key
    assert d['impl'] == 'reference' and d['unit'] == 'tokens/s' and d['higher_is_better'] is True
    assert d['steps'] == 1 and d['warmup'] == 3 and d['value'] > 0
    assert d['config']['workload'].startswith('moe_q4k_d4096_e64_f1408_top8')
    cb = d['cpu_baseline']
    assert cb['kind'] in ('reference', 'port') and cb['cores'] >= 1 and cb['value'] == d['value'] and cb['sample']
    e2e = d['e2e']
    assert e2e['value'] == d['value'] and e2e['unit'] == d['unit']
    assert e2e['h2d_bytes_per_step'] == 0 and e2e['d2h_bytes_per_step'] == 0


def test_reference_arm_other_ranks_do_nothing():
    p = run({'RANK': '1', 'WORLD_SIZE': '2'}, '--gpus', '2', '--steps', '1', '--warmup', '3', '--cpu-tokens', '32')
    assert p.returncode == 0, p.stderr[-2000:]
    assert not [l for l in p.stdout.splitlines() if l.strip().startswith('{')]
