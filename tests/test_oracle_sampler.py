"""The acceptance/sampling restatement in the oracle (orc_rng_next,
orc_argmax_logits, orc_sample_top_p; src/cli/dsv4_run.c:248-355) against
the reference CLI's own static functions compiled from its sources, and the
verify-step acceptance chain (:951-1043) against a loop over the
reference's primitives."""
import os

import numpy as np
import pytest

from oracle import REFCLI_SO, OracleSampler, RefSampler


@pytest.fixture(scope="module")
def pair():
    if not os.path.exists(REFCLI_SO):
        pytest.skip("reference CLI harness not built here")
    return OracleSampler(), RefSampler()


def test_rng_stream_matches(pair):
    o, r = pair
    so = sr = 0x9E3779B97F4A7C15
    for _ in range(1000):
        a, so = o.rng_next(so)
        b, sr = r.rng_next(sr)
        assert a == b and so == sr


def test_argmax_ties_nan_inf(pair):
    o, r = pair
    rng = np.random.default_rng(0)
    cases = [rng.normal(size=1000).astype(np.float32) for _ in range(20)]
    x = np.zeros(50, np.float32); x[[7, 9, 30]] = 3.0; cases.append(x)          # ties: first
    x = rng.normal(size=50).astype(np.float32); x[0] = np.nan; cases.append(x)  # NaN at 0 wins
    x = rng.normal(size=50).astype(np.float32); x[5] = np.nan; cases.append(x)
    x = np.full(10, -np.inf, np.float32); cases.append(x)
    x = rng.normal(size=50).astype(np.float32); x[11] = np.inf; cases.append(x)
    for c in cases:
        assert o.argmax_logits(c) == r.argmax_logits(c)


@pytest.mark.parametrize("T,p", [(1.0, 1.0), (0.7, 1.0), (1.0, 0.9), (0.3, 0.5), (1e-6, 1.0),
                                 (2.0, 0.999)])
def test_sample_top_p_matches(pair, T, p):
    o, r = pair
    rng = np.random.default_rng(int(T * 100 + p * 10))
    so = sr = 12345
    for _ in range(30):
        logits = (rng.normal(size=2000) * 3).astype(np.float32)
        a, so = o.sample_top_p(logits, T, p, so)
        b, sr = r.sample_top_p(logits, T, p, sr)
        assert a == b and so == sr


def _chain_with_reference(r, proposal, logits, T, p, state, eos):
    """The reference's acceptance loop (src/cli/dsv4_run.c:951-1043) written
    over the reference's own argmax/sample primitives."""
    accepted, correction, samples = 0, -1, 0
    P = len(proposal)
    while accepted < P:
        if T == 0.0:
            t = r.argmax_logits(logits[accepted])
        else:
            t, state = r.sample_top_p(logits[accepted], T, p, state)
            samples += 1
        if proposal[accepted] != t:
            correction = t
            break
        accepted += 1
        if t == eos:
            break
    eos_at = next((i for i in range(accepted) if proposal[i] == eos), -1)
    if eos_at >= 0:
        return list(proposal[:eos_at + 1]), eos_at + 1, accepted, samples, state
    if accepted < P:
        return list(proposal[:accepted]) + [correction], accepted + 1, accepted, samples, state
    if T == 0.0:
        bonus = r.argmax_logits(logits[P])
    else:
        bonus, state = r.sample_top_p(logits[P], T, p, state)
        samples += 1
    return list(proposal) + [bonus], P + 1, accepted, samples, state


@pytest.mark.parametrize("T", [0.0, 1.0])
def test_accept_chain_matches(pair, T):
    o, r = pair
    rng = np.random.default_rng(3)
    V = 64
    for trial in range(200):
        P = int(rng.integers(1, 8))
        logits = (rng.normal(size=(P + 1, V)) * 2).astype(np.float32)
        greedy = logits.argmax(axis=1)
        prop = greedy[:P].copy()
        cut = int(rng.integers(0, P + 1))      # drafts agree up to `cut`
        if cut < P:
            prop[cut] = (prop[cut] + 1 + int(rng.integers(0, V - 1))) % V
        if trial % 17 == 0:
            prop[int(rng.integers(0, P))] = 1  # an EOS draft
        state = int(rng.integers(1, 2**63))
        want = _chain_with_reference(r, prop, logits, T, 1.0, state, 1)
        got = o.accept_chain(prop, logits, T, 1.0, state, 1)
        assert list(got["tokens"]) == want[0]
        assert (got["n_commit"], got["n_accepted"], got["n_samples"], got["state"]) == want[1:]


def test_library_host_sampler_matches_reference(pair):
    """The product's host forms (dsv4cuda_sample_top_p / _accept_chain), no GPU."""
    import dsv4cuda
    _, r = pair
    rng = np.random.default_rng(8)
    s1 = s2 = 777
    for T, p in ((1.0, 1.0), (0.8, 0.95), (0.0, 1.0)):
        for _ in range(10):
            logits = (rng.normal(size=3000) * 2).astype(np.float32)
            if T == 0.0:
                assert dsv4cuda.argmax_logits(logits) == r.argmax_logits(logits)
                continue
            a, s1 = dsv4cuda.sample_top_p(logits, T, p, s1)
            b, s2 = r.sample_top_p(logits, T, p, s2)
            assert a == b and s1 == s2
    o = OracleSampler()
    for trial in range(50):
        P = int(rng.integers(1, 6))
        logits = (rng.normal(size=(P + 1, 40)) * 2).astype(np.float32)
        prop = logits.argmax(axis=1)[:P].copy()
        if trial % 3 == 0:
            prop[-1] = (prop[-1] + 5) % 40
        for T in (0.0, 1.0):
            a = dsv4cuda.accept_chain(prop, logits, T, 1.0, 99 + trial)
            b = o.accept_chain(prop, logits, T, 1.0, 99 + trial)
            assert list(a["tokens"]) == list(b["tokens"])
            assert all(a[k] == b[k] for k in ("n_commit", "n_accepted", "n_samples", "state"))
