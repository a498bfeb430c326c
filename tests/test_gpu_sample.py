"""GPU acceptance kernels (dsv4cuda_argmax_rows / _sample_rows /
_accept_device) against the reference CLI's own argmax_logits and
sample_top_p (src/cli/dsv4_run.c:308-355, compiled from its sources) and the
oracle's restatement of the verify-step acceptance (:951-1043).

Bar: greedy targets and the greedy chain bit-exact; temperature sampling
(top_p = 1) picks the reference's token for every row tested - the device
sums the softmax weights in a different order, which can only matter when
the uniform target lands within a few ulps of a running sum."""
import os

import numpy as np
import pytest
import torch

from oracle import REFCLI_SO, OracleSampler, RefSampler

pytestmark = pytest.mark.gpu
V = 129280  # DSV4 vocabulary


@pytest.fixture(scope="module")
def refs():
    if not os.path.exists(REFCLI_SO):
        pytest.skip("reference CLI harness not built")
    return OracleSampler(), RefSampler()


def test_argmax_rows_exact(cuda, refs):
    _, r = refs
    rng = np.random.default_rng(0)
    rows = (rng.normal(size=(9, V)) * 3).astype(np.float32)
    rows[1, [5, 77, 100000]] = 50.0            # tie -> first
    rows[2, 0] = np.nan                        # NaN at 0 is never displaced
    rows[3, 123] = np.nan
    rows[4, :] = -np.inf
    rows[5, 999] = np.inf
    rows[6, :] = 0.0
    out = torch.empty(9, dtype=torch.int32, device="cuda")
    cuda.argmax_rows(torch.from_numpy(rows).cuda(), out)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    for i in range(rows.shape[0]):
        assert got[i] == r.argmax_logits(rows[i]), i


@pytest.mark.parametrize("T", [1.0, 0.6, 1.7])
def test_sample_rows_match_reference(cuda, refs, T):
    _, r = refs
    rng = np.random.default_rng(int(T * 10))
    R = 48
    rows = (rng.normal(size=(R, V)) * 2.5).astype(np.float32)
    state = 0x1234567
    u, _ = cuda.uniforms(state, R)
    out = torch.empty(R, dtype=torch.int32, device="cuda")
    cuda.sample_rows(torch.from_numpy(rows).cuda(), T, torch.from_numpy(u).cuda(), out)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    st = state
    for i in range(R):
        want, st = r.sample_top_p(rows[i], T, 1.0, st)
        assert got[i] == want, (i, got[i], want)


@pytest.mark.parametrize("T", [0.0, 1.0])
def test_accept_device_matches_chain(cuda, refs, T):
    o, _ = refs
    rng = np.random.default_rng(5)
    Vs = 32000
    for trial in range(12):
        P = int(rng.integers(1, 8))
        logits = (rng.normal(size=(P + 1, Vs)) * 3).astype(np.float32)
        prop = logits.argmax(axis=1)[:P].astype(np.int32)
        cut = int(rng.integers(0, P + 1))
        if cut < P:
            prop[cut] = (prop[cut] + 3) % Vs
        if trial == 5:
            prop[0] = 1
            logits[0, 1] = 100.0                   # an accepted EOS draft
        state = 4242 + trial
        want = o.accept_chain(prop, logits, T, 1.0, state, eos_id=1)
        u, _ = cuda.uniforms(state, P + 1)
        res = torch.zeros(2 * P + 6, dtype=torch.int32, device="cuda")
        cuda.accept_device(torch.from_numpy(prop).cuda(), torch.from_numpy(logits).cuda(), T,
                           None if T == 0.0 else torch.from_numpy(u).cuda(), res, eos_id=1)
        torch.cuda.synchronize()
        got = res.cpu().numpy()
        n = got[0]
        assert list(got[4:4 + n]) == list(want["tokens"])
        assert (got[1], got[2], got[3]) == (want["n_commit"], want["n_accepted"],
                                            want["n_samples"])
