"""The benchmark's reference arm on the CPU: `bench.py --impl reference` prints exactly one JSON line with the keys the
benchmark contract names (the reference's host featurization timed on a bounded ray sample), at one process and under
torchrun with two ranks, where rank 0 alone measures and prints and the other rank exits 0 without work."""
from __future__ import annotations

import json
import os
import socket
import subprocess
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parent.parent
TINY = ['--impl', 'reference', '--steps', '1', '--warmup', '3', '--reference-rays', '64', '--reference-repeats', '1']
KEYS = {'impl', 'metric', 'value', 'unit', 'n_gpus', 'steps', 'warmup', 'higher_is_better', 'scaling', 'vs_baseline', 'dtype', 'data',
        'config', 'cpu_baseline', 'e2e'}


def json_lines(stdout: str) -> list[dict]:
    return [json.loads(line) for line in stdout.splitlines() if line.startswith('{')]


def check_line(line: dict, n_gpus: int) -> None:
    assert KEYS <= set(line), KEYS - set(line)
    assert line['impl'] == 'reference' and line['n_gpus'] == n_gpus and line['steps'] == 1 and line['warmup'] == 3
    assert line['higher_is_better'] is True and line['value'] > 0 and 'workload' in line['config']
    cpu, e2e = line['cpu_baseline'], line['e2e']
    assert cpu['value'] == line['value'] and cpu['unit'] == line['unit'] and cpu['kind'] in ('reference', 'port') and cpu['cores'] >= 1
    assert '64 rays' in cpu['sample']
    assert e2e == {'value': line['value'], 'unit': line['unit'], 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0}


def free_port() -> int:
    with socket.socket() as s:
        s.bind(('127.0.0.1', 0))
        return s.getsockname()[1]


def test_reference_arm_prints_one_contract_line():
    run = subprocess.run([sys.executable, 'bench.py', *TINY], cwd=REPO, capture_output=True, text=True, timeout=600)
    assert run.returncode == 0, run.stderr[-2000:]
    lines = json_lines(run.stdout)
    assert len(lines) == 1, run.stdout
    check_line(lines[0], 1)


def test_reference_arm_under_torchrun_measures_on_rank_zero_only():
    env = {k: v for k, v in os.environ.items() if k not in ('RANK', 'WORLD_SIZE', 'LOCAL_RANK', 'MASTER_ADDR', 'MASTER_PORT')}
    run = subprocess.run([sys.executable, '-m', 'torch.distributed.run', '--nnodes=1', '--nproc-per-node', '2', '--master-addr', '127.0.0.1',
                          '--master-port', str(free_port()), 'bench.py', '--gpus', '2', *TINY],
                         cwd=REPO, capture_output=True, text=True, timeout=600, env=env)
    assert run.returncode == 0, run.stderr[-2000:]
    lines = json_lines(run.stdout)
    assert len(lines) == 1, run.stdout
    check_line(lines[0], 2)


def test_algorithmic_bytes_follow_the_roofline_accounting():
    """Per-interval algorithmic bytes of config 2 (48 unmerged corner rows per level plus the interval's own inputs and
    outputs): proposal 2,008 B forward and backward, NeRF 7,860 B forward and 5,096 B backward (3 fp32 and 7 fp16
    gradient levels); 33.33 GB forward + 27.53 GB backward = 60.86 GB per 65,536-ray step."""
    import importlib.util
    spec = importlib.util.spec_from_file_location('bench_module', REPO / 'bench.py')
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    ab = bench.algorithmic_bytes
    assert ab('forward_proposal', 10, 1, 20) == 2008 and ab('backward_proposal', 10, 1, 20) == 2008
    assert ab('forward_nerf', 10, 4, 50) == 7860 and ab('backward_nerf', 10, 4, 50, 3) == 5096
    rays = 65536
    forward = rays * (2 * 64 * ab('forward_proposal', 10, 1, 20) + 32 * ab('forward_nerf', 10, 4, 50))
    backward = rays * (2 * 64 * ab('backward_proposal', 10, 1, 20) + 32 * ab('backward_nerf', 10, 4, 50, 3))
    assert round(forward / 1e9, 2) == 33.33 and round(backward / 1e9, 2) == 27.53 and round((forward + backward) / 1e9, 2) == 60.86
