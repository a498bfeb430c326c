"""Host logic of bench.py that needs no GPU: the chained-graph replays cover
exactly the requested number of steps; the CPU baseline's per-token
extrapolation over the model's kinds of layer."""
import importlib.util
import os

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bench():
    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


@pytest.mark.parametrize("count", [0, 1, 3, 4, 5, 8, 199, 200, 301])
@pytest.mark.parametrize("n_layers", [1, 3, 4])
def test_chain_lengths_cover_exactly(count, n_layers):
    lens = _bench().chain_lengths(count, n_layers)
    assert sum(lens) == count
    assert all(1 <= n <= n_layers for n in lens)
    # only the last replay may be a shorter chain
    assert all(n == n_layers for n in lens[:-1])


def test_cpu_reference_decode_extrapolates_per_kind(monkeypatch):
    """The CPU baseline's per-token time is the model's layers' kind times
    (compress ratio 0 / 4 / 128 in the config-5 pattern) plus the head and
    the embedding, for the all-thread line and the one-thread line alike;
    each kind is timed once on its own checkpoint."""
    bench = _bench()
    layer = {0: 0.010, 4: 0.020, 128: 0.015}
    layer1 = {0: 0.100, 4: 0.200, 128: 0.150}
    calls = []

    def fake_one(threads=None, warm=8, timed=8, ratio=0, one_thread=None):
        calls.append((ratio, one_thread))
        one = (layer1[ratio], 0.5) if one_thread else None
        return layer[ratio], 0.05, 16, one

    monkeypatch.setattr(bench, "cpu_reference_decode_one", fake_one)
    tps, cores, sample, one = bench.cpu_reference_decode(43, one_thread=(2, 4))
    ratios = bench.c5_ratios(43)
    want = sum(layer[r] for r in ratios) + 0.05
    want1 = sum(layer1[r] for r in ratios) + 0.5
    assert sorted(r for r, _ in calls) == sorted(set(ratios))
    assert all(o == (2, 4) for _, o in calls)
    assert cores == 16 and tps == pytest.approx(1.0 / want)
    assert one["cores"] == 1 and one["value"] == pytest.approx(1.0 / want1)
    assert "ratio 4" in sample and "ratio 128" in one["sample"]
    # without the one-thread request: no one-thread line
    calls.clear()
    assert bench.cpu_reference_decode(43)[3] is None
    assert all(o is None for _, o in calls)
