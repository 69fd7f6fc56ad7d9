"""The benchmark's command line and the JSON line of its reference arm (which
times the reference's CPU implementation and runs on any host)."""
import json
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
import bench  # noqa: E402

WORKLOADS = ['config1', 'config2', 'config4_leaf', 'config5_g32', 'config5_g4', 'config4_block', 'config3', 'atlas',
             'model_layers']


@pytest.mark.parametrize('workload', WORKLOADS)
def test_every_workload_parses(workload):
    args = bench.parse_args(['--workload', workload, '--steps', '5', '--warmup', '3'])
    assert args.workload == workload and args.impl == 'ours' and args.gpus == 1


def test_defaults_and_warmup_floor():
    args = bench.parse_args([])
    assert args.workload == 'config2' and args.gpus == 1 and args.warmup >= 3
    with pytest.raises(SystemExit):
        bench.parse_args(['--warmup', '2'])


def test_reference_arm_prints_one_json_line_with_the_contract_keys():
    run = subprocess.run([sys.executable, str(ROOT / 'bench.py'), '--impl', 'reference', '--steps', '3',
                          '--warmup', '3'], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert run.returncode == 0, run.stderr[-2000:]
    lines = [l for l in run.stdout.splitlines() if l.strip()]
    assert len(lines) == 1, run.stdout
    line = json.loads(lines[0])
    if 'unavailable' in line:
        pytest.skip(line['unavailable'])
    assert line['impl'] == 'reference'
    for key in ('metric', 'value', 'unit', 'n_gpus', 'steps', 'warmup', 'ms_per_step', 'higher_is_better',
                'scaling', 'dtype', 'config', 'cpu_baseline', 'e2e'):
        assert key in line, key
    assert line['value'] > 0 and line['steps'] == 3 and line['warmup'] == 3 and line['n_gpus'] == 1
    assert line['config']['workload'] == 'config2'
    cpu = line['cpu_baseline']
    assert cpu['kind'] in ('reference', 'port') and cpu['cores'] >= 1 and cpu['sample'] and cpu['value'] == line['value']
    assert line['e2e']['h2d_bytes_per_step'] == 0 and line['e2e']['d2h_bytes_per_step'] == 0
    assert line['e2e']['value'] == line['value'] and line['e2e']['unit'] == line['unit']
