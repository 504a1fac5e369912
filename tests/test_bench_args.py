"""CPU checks of bench.py's command line and timed-window logic (the driver calls it as
`bench.py --gpus N --steps K --warmup W`)."""
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


def test_same_workload_at_every_gpu_count(monkeypatch):
    a = _parse([], monkeypatch)
    assert (a.gpus, a.workload, a.impl) == (1, 'qwen3_1.7b', 'ours') and a.warmup >= 3
    for n in ('2', '4', '8'):
        assert _parse(['--gpus', n, '--steps', '8', '--warmup', '3'], monkeypatch).workload == 'qwen3_1.7b'
    assert _parse(['--workload', 'nanogpt'], monkeypatch).workload == 'nanogpt'
    assert _parse(['--impl', 'reference', '--gpus', '4'], monkeypatch).impl == 'reference'


def test_warmup_floor(monkeypatch):
    with pytest.raises(SystemExit):
        _parse(['--warmup', '2'], monkeypatch)


def test_timed_positions_cover_the_window():
    b = _bench()
    # fewer steps than the window: spread over 32..287, mean context near the config's mean
    p = b.window_positions(20)
    assert len(p) == 20 and p[0] == 32 and p[-1] <= 287 and p == sorted(set(p))
    assert abs(sum(x + 1 for x in p) / 20 - 160.5) < 7
    # whole windows in order
    p = b.window_positions(512)
    assert p[:256] == list(range(32, 288)) and p[256:] == list(range(32, 288))
    assert all(32 <= x <= 287 for x in b.window_positions(300))


def test_reference_arm_does_not_import_the_product():
    """The reference arm's code path names no module of the product package."""
    import ast
    tree = ast.parse((ROOT / 'bench.py').read_text())
    fn = next(n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name == 'run_reference')
    mods = [n.module for n in ast.walk(fn) if isinstance(n, ast.ImportFrom)]
    mods += [a.name for n in ast.walk(fn) if isinstance(n, ast.Import) for a in n.names]
    assert mods and not any(m.startswith('efficientgpt_b200') for m in mods)
    names = {n.id for n in ast.walk(fn) if isinstance(n, ast.Name)}
    assert not names & {'build', 'run_config2', 'run_tp', 'dist_setup'}
