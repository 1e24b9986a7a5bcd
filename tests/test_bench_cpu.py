"""The benchmark's contract, on the CPU: the reference arm's one JSON line,
the metric names per config, and the traffic figures read from the ncu
summaries in profiles/ (the GPU arm runs on a B200 only)."""

import json
import os
import subprocess
import sys

import pytest

import bench
from tests import reference_swap

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_defaults_are_the_headline_config_on_one_gpu():
    a = bench.parse_args([])
    assert (a.gpus, a.config, a.impl, a.scaling) == (1, 2, 'vectra',
                                                     'strong')
    assert a.warmup >= 3


@pytest.mark.parametrize('world', [1, 2, 8])
def test_strong_scaling_splits_one_batch(world):
    p = bench.plan(2, 'strong', world)
    assert p['global_batch'] == 1024 and p['per_gpu'] == 1024 // world
    w = bench.plan(2, 'weak', world)
    assert w['global_batch'] == 1024 * world and w['per_gpu'] == 1024
    # The rotating input sets read more than L2 holds (or 32 sets).
    assert (p['n_sets'] * p['set_bytes'] > 3 * bench.L2_BYTES or
            p['n_sets'] == 32)


def test_reference_arm_prints_one_json_line(capfd, monkeypatch):
    monkeypatch.delenv('RANK', raising=False)
    assert bench.main(['--impl', 'reference', '--config', '1', '--steps',
                       '2', '--warmup', '1']) == 0
    out = capfd.readouterr().out.strip().splitlines()
    assert len(out) == 1, out
    line = json.loads(out[0])
    assert line['impl'] == 'reference'
    metric, unit = bench.metric_for(1)
    assert (line['metric'], line['unit']) == (metric, unit)
    assert line['value'] > 0 and line['higher_is_better'] is True
    cpu = line['cpu_baseline']
    assert cpu['value'] == line['value'] and cpu['cores'] >= 1
    assert cpu['kind'] == 'port' and cpu['cpu_model']
    assert line['e2e'] == {'value': line['value'], 'unit': unit,
                           'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0}
    # The same config as the GPU arm's line, key for key.
    assert line['config'] == bench.line_config(bench.parse_args(
        ['--config', '1']), 1)


def test_reference_arm_never_loads_this_library(tmp_path):
    # In a fresh process: the arm's line is printed, no vectra_b200 module
    # is imported and none of this library's shared objects is mapped.
    probe = tmp_path / 'probe.py'
    probe.write_text(
        'import sys\n'
        f'sys.path.insert(0, {ROOT!r})\n'
        'import bench\n'
        "bench.main(['--impl', 'reference', '--config', '2', '--steps', '1',"
        " '--warmup', '0'])\n"
        "mods = [m for m in sys.modules if m.startswith('vectra_b200')]\n"
        "maps = open('/proc/self/maps').read()\n"
        "print('MODS', mods)\n"
        "print('MAPPED', 'libvectra_rbf' in maps or "
        "'_vectra_rbf_torch' in maps)\n")
    env = dict(os.environ)
    env.pop('RANK', None)
    out = subprocess.run([sys.executable, str(probe)], capture_output=True,
                         text=True, check=True, env=env, timeout=600).stdout
    lines = out.strip().splitlines()
    assert json.loads(lines[0])['impl'] == 'reference'
    assert 'MODS []' in out and 'MAPPED False' in out, out


@pytest.mark.parametrize('config', [1, 2, 3, 4, 5])
def test_metric_units(config):
    metric, unit = bench.metric_for(config)
    assert metric and unit == {4: 'TFLOP/s', 5: 'targets/s'}.get(
        config, 'queries/s')


@pytest.mark.parametrize('config,kernel', [(2, 'rbf_decode'),
                                           (3, 'rbf_decode'),
                                           (4, 'rbf_tc'), (5, 'rbf_small')])
def test_traffic_figures_come_from_the_committed_profiles(config, kernel):
    assert os.path.exists(
        os.path.join(ROOT, 'profiles', f'{kernel}_config{config}.txt'))
    traffic = bench.ncu_traffic(config)
    assert traffic is not None and traffic > 1e8


def test_pinned_kernel_traffic_comes_from_its_own_profile():
    assert bench.parse_args([]).kernel == 'auto'
    a = bench.parse_args(['--config', '5', '--kernel', 'small_tc'])
    assert a.kernel == 'small_tc'
    small = bench.ncu_traffic(5)
    pinned = bench.ncu_traffic(5, kernel='small_tc')
    assert small is not None and pinned is not None and pinned > 1e8
    assert pinned != small  # profiles/rbf_small_tc_config5.txt
    assert bench.ncu_traffic(5, kernel='auto') == small


def test_shard_of_options():
    assert bench.parse_args([]).shard_of == 1
    assert bench.parse_args(['--shard-of', '8']).shard_of == 8
    for bad in (['--shard-of', '0'], ['--shard-of', '4', '--scan', 'l2'],
                ['--config', '5', '--model', '--kernel', 'small'],
                ['--kernel', 'nonesuch']):
        with pytest.raises(SystemExit):
            bench.parse_args(bad)
    # One GPU playing rank 0 of 8 times the shard an 8-GPU run gives a rank.
    assert bench.plan(2, 'strong', 8)['per_gpu'] == 128


def test_model_mode_needs_config_5():
    with pytest.raises(SystemExit):
        bench.parse_args(['--model'])
    assert bench.parse_args(['--model', '--config', '5']).model
    assert bench.metric_for(5, model=True)[1] == 'predictions/s'


@pytest.mark.skipif(not reference_swap.installed(),
                    reason='the reference is not installed in baseline/_ref')
def test_model_reference_arm_prints_one_json_line(capfd, monkeypatch):
    monkeypatch.delenv('RANK', raising=False)
    assert bench.main(['--impl', 'reference', '--config', '5', '--model',
                       '--steps', '1', '--warmup', '0']) == 0
    out = capfd.readouterr().out.strip().splitlines()
    assert len(out) == 1, out
    line = json.loads(out[0])
    assert line['impl'] == 'reference' and line['unit'] == 'predictions/s'
    assert line['value'] > 0 and line['cpu_baseline']['cores'] >= 1
    assert line['cpu_baseline']['kind'] == 'reference'
    assert line['e2e']['h2d_bytes_per_step'] == 0
    assert line['config'] == bench.model_config_line(
        bench.parse_args(['--config', '5', '--model']), 1)


@pytest.mark.parametrize('kind', ['l2', 'pq'])
def test_scan_reference_arm_prints_one_json_line(capfd, monkeypatch, kind):
    monkeypatch.delenv('RANK', raising=False)
    # A small shard and short timing windows: the arm's contract, not its
    # number.
    monkeypatch.setattr(bench, 'SCAN_L2', dict(rows=1 << 14, dim=32))
    monkeypatch.setattr(bench, 'SCAN_PQ', dict(rows=1 << 15, subspaces=8))
    timed = bench.time_scan_cpu
    monkeypatch.setattr(
        bench, 'time_scan_cpu',
        lambda k, d, q, seconds, threads: timed(k, d, q, 0.05, threads))
    assert bench.main(['--impl', 'reference', '--scan', kind, '--steps', '1',
                       '--warmup', '0']) == 0
    out = capfd.readouterr().out.strip().splitlines()
    assert len(out) == 1, out
    line = json.loads(out[0])
    assert line['impl'] == 'reference'
    assert (line['metric'], line['unit']) == bench.scan_metric(kind)
    assert line['value'] > 0 and line['cpu_baseline']['cores'] >= 1
    assert line['cpu_baseline']['kind'] in ('reference', 'port')
    assert line['e2e']['h2d_bytes_per_step'] == 0


def test_scan_traffic_comes_from_the_committed_profile():
    traffic = bench.ncu_traffic(None, 'scan_levels',
                                'dram_bytes_full_level_l2')
    rows = bench.SCAN_L2['rows'] * bench.SCAN_L2['dim'] * 4
    assert traffic is not None and rows <= traffic < 1.1 * rows
