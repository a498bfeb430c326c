"""The ordered top-k selection network of comp_list_kernel (csrc/decode.cu),
simulated on the host stage by stage: one key per thread, the thread's
partner tid ^ stride, and the rule the kernel applies to keep its own key or
take the partner's. The reference's order (dsv4_indexer_select_topk,
src/dsv4/dsv4_model.c:5636-5679) is score descending, lower index first, so
the network must produce exactly Python's sort by (-score, index), with
padding keys (index -1) after every real key - on ties, on negative and zero
scores and at every list length up to the CTA width. This checks the
network's design; the device kernel itself is checked against the reference
engine in test_gpu_decoder_comp.py.
"""
import numpy as np
import pytest

CTA = 1024


def before(sa, ia, sb, ib):
    """The kernel's topk_before, elementwise: real before padding (-1), higher
    score first, lower index first."""
    return np.where(ib < 0, ia >= 0,
                    np.where(ia < 0, False,
                             np.where(sa > sb, True, np.where(sa < sb, False, ia < ib))))


def network(scores):
    n = len(scores)
    m2 = 32
    while m2 < n:
        m2 <<= 1
    assert m2 <= CTA
    tid = np.arange(CTA)
    sv = np.where(tid < n, np.pad(scores, (0, CTA - n)), 0.0).astype(np.float32)
    iv = np.where(tid < n, tid, -1)
    size = 2
    while size <= m2:
        stride = size >> 1
        while stride > 0:
            so, io = sv[tid ^ stride], iv[tid ^ stride]
            up = (tid & size) == 0
            lower = (tid & stride) == 0
            mine_first = before(sv, iv, so, io)
            take = np.where(lower == up, ~mine_first, mine_first) & (tid < m2)
            sv, iv = np.where(take, so, sv), np.where(take, io, iv)
            stride >>= 1
        size <<= 1
    return iv[:n]


def want(scores):
    return [i for _, i in sorted((-float(s), i) for i, s in enumerate(scores))]


@pytest.mark.parametrize("n", [1, 2, 5, 31, 32, 33, 100, 255, 512, 513, 777, 1024])
def test_network_sorts_random_scores(n):
    s = np.random.default_rng(n).normal(size=n).astype(np.float32)
    assert list(network(s)) == want(s)


@pytest.mark.parametrize("n", [7, 64, 300, 1000])
def test_network_ties_keep_index_order(n):
    rng = np.random.default_rng(100 + n)
    # few distinct values: long runs of equal scores, zeros (ReLU'd dots) and
    # negative values among them
    s = rng.choice(np.array([0.0, 1.5, -2.0, 3.25], np.float32), size=n)
    assert list(network(s)) == want(s)


def test_network_all_equal():
    s = np.zeros(512, np.float32)
    assert list(network(s)) == list(range(512))
