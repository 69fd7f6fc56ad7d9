"""The benchmark's command line, the JSON line of its reference arm (which
times the reference's CPU implementation and runs on any host), and the
host logic of its strong-scaling path: the pieces each rank convolves and the
correctness gate on them, with the oracle standing in for the device."""
import json
import math
import os
import socket
import subprocess
import sys
from pathlib import Path

import numpy as np
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
    assert args.workload == 'config5_g32' and args.scaling == 'strong' and args.gpus == 1 and args.warmup >= 3
    assert args.block_list == ['config5_g4', 'config2']
    assert bench.parse_args(['--workload', 'config2']).block_list == []
    assert bench.parse_args(['--blocks', '']).block_list == []
    assert bench.parse_args(['--workload', 'config2']).scaling == 'weak'
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
    assert line['config']['workload'] == 'config5_g32'
    from groupconv_atlas_b200 import workloads
    # the same config object as the GPU arm prints for this workload
    assert line['config'] == json.loads(json.dumps(bench.workload_config('config5_g32',
                                                                         workloads.config5(32, with_x=False).shape)))
    cpu = line['cpu_baseline']
    assert cpu['kind'] in ('reference', 'port') and cpu['cores'] >= 1 and cpu['sample'] and cpu['value'] == line['value']
    assert line['e2e']['h2d_bytes_per_step'] == 0 and line['e2e']['d2h_bytes_per_step'] == 0
    assert line['e2e']['value'] == line['value'] and line['e2e']['unit'] == line['unit']


@pytest.mark.parametrize('n,groups,world', [(1024, 32, 8), (1024, 4, 3), (3, 32, 8), (1, 8, 8), (2, 4, 8)])
def test_rank_pieces_cover_the_output_once(n, groups, world):
    """Strong scaling: the pieces of all ranks (and their 8-way end-to-end
    chunks) cover every output element exactly once, and every piece lies
    inside the rank-local buffers."""
    from groupconv_atlas_b200.api import Shape
    full = Shape(n=n, cin=256, cout=256, h=4, w=4, groups=groups)
    for chunks in (1, 8):
        seen = np.zeros((n, 256), np.int32)
        job_bytes = 0
        for rank in range(world):
            first, count, units = bench.rank_work(full, 'strong', world, rank)
            local = Shape(**{**full.__dict__, 'n': max(1, count)})
            for p in bench.pieces_of(units, local, chunks):
                assert p.x_off + p.x_len <= math.prod(local.input)
                assert p.y_off + p.y_len <= math.prod(local.output)
                assert p.w_off + p.w_len <= math.prod(local.weight)
                n0 = p.y_off // (256 * 16)
                c0 = (p.y_off - n0 * 256 * 16) // 16
                seen[first + n0:first + n0 + p.shape.n, c0:c0 + p.shape.cout] += 1
                job_bytes += 4 * (p.x_len + p.y_len)
        assert (seen == 1).all()
        assert job_bytes == 4 * (math.prod(full.input) + math.prod(full.output))


def _free_port():
    with socket.socket() as sock:
        sock.bind(('127.0.0.1', 0))
        return sock.getsockname()[1]


def _gate_rank(rank, world, port, shape_dict, result_path):
    """One rank of the strong-scaling gate: its pieces are computed by the
    oracle (standing in for the device) into a NaN-filled local output; the
    gate must pass, and must fail once a computed element is corrupted."""
    import torch.distributed as dist
    from groupconv_atlas_b200.api import Shape
    from groupconv_atlas_b200 import workloads
    from oracle import oracle as orc
    os.environ.update(MASTER_ADDR='127.0.0.1', MASTER_PORT=str(port))
    dist.init_process_group('gloo', rank=rank, world_size=world)
    try:
        full = Shape(**shape_dict)
        first, count, units = bench.rank_work(full, 'strong', world, rank)
        local = Shape(**{**shape_dict, 'n': max(1, count)})
        x = workloads.images(full, 5, 'uniform', first, local.n)
        w = np.random.default_rng(1).uniform(-1, 1, full.weight).astype(np.float32)
        y = np.full(local.output, np.nan, np.float32)
        pieces = bench.pieces_of(units, local)
        for p in pieces:
            xv = x.reshape(-1)[p.x_off:p.x_off + p.x_len].reshape(p.shape.input)
            wv = w.reshape(-1)[p.w_off:p.w_off + p.w_len].reshape(p.shape.weight)
            y.reshape(-1)[p.y_off:p.y_off + p.y_len] = orc.conv_f32_serial(p.shape, xv, wv).reshape(-1)
        ok = bench.gate(pieces, x, w, y) == []
        if pieces:
            y.reshape(-1)[pieces[0].y_off] += 1.0  # the first point of the selection: (0, 0, 0, 0)
        caught = bench.gate(pieces, x, w, y) != [] if pieces else True
        flags = [None] * world
        dist.all_gather_object(flags, (ok, caught, len(pieces)))
        if rank == 0:
            Path(result_path).write_text(json.dumps(flags))
        dist.barrier()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize('shape_dict', [
    dict(n=1, cin=32, cout=32, h=7, w=9, groups=8),   # one image, group blocks across the ranks
    dict(n=3, cin=16, cout=16, h=6, w=5, groups=4),   # batch ranges
])
def test_gloo_two_ranks_gate_on_units(tmp_path, shape_dict):
    import torch.multiprocessing as mp
    out = tmp_path / 'flags.json'
    mp.start_processes(_gate_rank, args=(2, _free_port(), shape_dict, str(out)), nprocs=2, start_method='spawn',
                       join=True)
    flags = json.loads(out.read_text())
    assert all(ok and caught and n >= 1 for ok, caught, n in flags), flags
