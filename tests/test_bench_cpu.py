"""bench.py's reference arm on the CPU: one JSON line with the contract's keys, exactly the requested steps, and
silence on ranks other than 0 (under torchrun only rank 0 times the CPU path)."""

import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def run_bench(*args, env_extra=None):
    env = dict(os.environ, **(env_extra or {}))
    return subprocess.run([sys.executable, os.path.join(ROOT, 'bench.py'), *args], cwd=ROOT, env=env,
                          capture_output=True, text=True, timeout=300)


def test_reference_arm_prints_one_contract_line():
    p = run_bench('--impl', 'reference', '--config', 'c2', '--steps', '2', '--warmup', '3')
    assert p.returncode == 0, p.stderr[-2000:]
    lines = [ln for ln in p.stdout.splitlines() if ln.startswith('{')]
    assert len(lines) == 1
    line = json.loads(lines[0])
    assert line['impl'] == 'reference'
    assert line['steps'] == 2 and line['warmup'] == 3
    assert line['unit'] == 'us' and line['higher_is_better'] is False and line['value'] > 0
    assert line['cpu_baseline']['kind'] == 'port' and line['cpu_baseline']['cores'] >= 1
    assert line['cpu_baseline']['value'] == line['value']
    assert line['e2e'] == {'value': line['value'], 'unit': 'us', 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0}


def test_reference_arm_is_silent_on_other_ranks():
    p = run_bench('--impl', 'reference', '--config', 'c2', '--steps', '2', '--warmup', '3',
                  env_extra={'RANK': '1', 'WORLD_SIZE': '2', 'LOCAL_RANK': '1'})
    assert p.returncode == 0, p.stderr[-2000:]
    assert not [ln for ln in p.stdout.splitlines() if ln.startswith('{')]


def test_reference_arm_config_names_the_gpu_arms_workload():
    """The CPU arm's config is the GPU arm's: per-GPU batch, and 'auto' resolved with the B200 table."""
    p = run_bench('--impl', 'reference', '--steps', '1', '--warmup', '3')
    assert p.returncode == 0, p.stderr[-2000:]
    line = json.loads([ln for ln in p.stdout.splitlines() if ln.startswith('{')][0])
    assert 'per GPU' in line['config']['workload'] and line['config']['mode'] == 'project'


def test_reference_cuda_without_an_installed_upstream_says_unavailable():
    p = run_bench('--impl', 'reference-cuda', '--ref-path', os.path.join(ROOT, 'no_such_checkout'))
    assert p.returncode == 0, p.stderr[-2000:]
    lines = [json.loads(ln) for ln in p.stdout.splitlines() if ln.startswith('{')]
    assert lines == [{'impl': 'reference-cuda', 'unavailable': lines[0]['unavailable']}]
    assert 'no installed marearts_tinydeform' in lines[0]['unavailable']
