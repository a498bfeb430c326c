"""Host logic of bench.py that needs no GPU: the chained-graph replays cover
exactly the requested number of steps."""
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
