"""Host logic of the tree/chain verify step (dsv4cuda_tree_attn_indices):
each node sees window_topk's window for its position
(src/dsv4/dsv4_model.c:5073-5089) with the uncommitted positions replaced by
its own ancestors' scratch rows. No GPU needed."""
import numpy as np
import pytest

dsv4cuda = pytest.importorskip("dsv4cuda")


def expected(parents, committed, window, ring_base, scratch):
    depth = []
    for j, p in enumerate(parents):
        depth.append(0 if p < 0 else depth[p] + 1)
    rows = []
    for j in range(len(parents)):
        pos = committed + depth[j]
        first = max(0, pos - window + 1)
        r = [ring_base + q % window for q in range(first, committed)]
        chain = []
        a = j
        while a >= 0:
            chain.append(a)
            a = parents[a]
        r += [scratch + a for a in reversed(chain) if committed + depth[a] >= first]
        rows.append(r)
    return rows


@pytest.mark.parametrize("parents", [[-1, 0, 1, 2, 3, 4],            # chain k = 5
                                     [-1, 0, 0, 1, 1, 2, 2],          # 2-ary tree, 7 nodes
                                     [-1], [-1, 0, 0, 0, 1, 4, 5, 5]])
@pytest.mark.parametrize("committed,window", [(0, 128), (50, 128), (300, 128), (130, 4)])
def test_tree_indices(parents, committed, window):
    row_len = window + len(parents) + 2
    got = dsv4cuda.tree_attn_indices(parents, committed, window, 10, 1000, row_len)
    want = expected(parents, committed, window, 10, 1000)
    for j, w in enumerate(want):
        assert list(got[j, :len(w)]) == w
        assert np.all(got[j, len(w):] == -1)


def test_tree_indices_rejects_bad_parents():
    with pytest.raises(dsv4cuda.Dsv4CudaError):
        dsv4cuda.tree_attn_indices([-1, 2, 0], 5, 128, 0, 200, 140)
