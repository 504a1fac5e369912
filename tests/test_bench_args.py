"""CPU checks of bench.py's command line (the driver calls it as `bench.py --gpus N --steps K --warmup W`)."""
import importlib.util
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _bench():
    spec = importlib.util.spec_from_file_location('bench_under_test', ROOT / 'bench.py')
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _parse(argv, monkeypatch):
    bench = _bench()
    monkeypatch.setattr(sys, 'argv', ['bench.py'] + argv)
    return bench.parse()


def test_default_workloads(monkeypatch):
    a = _parse([], monkeypatch)
    assert (a.gpus, a.workload, a.impl) == (1, 'qwen3_1.7b', 'ours') and a.warmup >= 3
    assert _parse(['--gpus', '2', '--steps', '8', '--warmup', '3'], monkeypatch).workload == 'qwen3_8b'
    assert _parse(['--gpus', '8', '--replicas'], monkeypatch).workload == 'qwen3_1.7b'
    assert _parse(['--workload', 'nanogpt'], monkeypatch).workload == 'nanogpt'
    assert _parse(['--impl', 'reference', '--gpus', '4'], monkeypatch).impl == 'reference'


def test_warmup_floor(monkeypatch):
    with pytest.raises(SystemExit):
        _parse(['--warmup', '2'], monkeypatch)
