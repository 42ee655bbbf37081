"""CPU: bench.py's reference arm (the unpatched e3nn-path model on the host cores) prints one JSON line with the keys
the benchmark contract asks for, on the same metric, unit and workload as the GPU arm."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_the_contract_line():
    r = subprocess.run([sys.executable, os.path.join(ROOT, 'bench.py'), '--impl', 'reference', '--steps', '1',
                        '--warmup', '1'], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith('{')]
    assert len(lines) == 1, r.stdout[-2000:]
    o = json.loads(lines[0])
    for k in ('metric', 'value', 'unit', 'n_gpus', 'steps', 'warmup', 'ms_per_step', 'higher_is_better', 'scaling',
              'vs_baseline', 'dtype', 'data', 'config', 'cpu_baseline', 'e2e', 'impl'):
        assert k in o, k
    assert o['impl'] == 'reference' and o['metric'] == 'E+F atom-steps/s' and o['unit'] == 'atom-steps/s'
    assert o['higher_is_better'] is True and o['value'] > 0 and o['warmup'] >= 3
    assert 'workload' in o['config'] and 'configs[1]' in o['config']['workload']
    assert o['cpu_baseline']['kind'] == 'port' and o['cpu_baseline']['cores'] >= 1
    assert o['e2e']['value'] == o['value'] and o['e2e']['h2d_bytes_per_step'] == 0
