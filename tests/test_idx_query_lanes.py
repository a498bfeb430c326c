"""The lane mapping of idx_query_warp (csrc/decode.cu), simulated on the
host: lane l holds values l * V .. l * V + V - 1 of a 32 V-long head; the
Hadamard butterflies run inside a lane while the stride is below V and
across lanes (partner lane ^ stride / V, the upper lane taking partner -
own) above it. In float32 with the same operations, every stage must equal
the reference's sequential butterfly loop (dsv4_hadamard_inplace,
src/dsv4/dsv4_model.c:1454) bit for bit, for each V the kernel instantiates
(1, 2, 4, 8: index dims 32-256). The GPU parity tests pin V = 1 and V = 4
against the reference engine itself.
"""
import numpy as np
import pytest


def hadamard_sequential(x):
    x = x.copy()
    n = len(x)
    ln = 1
    while ln < n:
        for k in range(n // 2):
            i = (k // ln) * 2 * ln + (k % ln)
            a, b = x[i], x[i + ln]
            x[i] = np.float32(a + b)
            x[i + ln] = np.float32(a - b)
        ln <<= 1
    return x


def hadamard_lanes(x, v):
    lanes = x.reshape(32, v).copy()  # lanes[l][r] = x[l * v + r]
    ln = 1
    while ln < v:  # inside a lane
        for r in range(v):
            if r & ln == 0:
                a, b = lanes[:, r].copy(), lanes[:, r + ln].copy()
                lanes[:, r] = a + b
                lanes[:, r + ln] = a - b
        ln <<= 1
    lm = 1
    lane = np.arange(32)
    while lm < 32:  # across lanes, stride lm = len / v
        other = lanes[lane ^ lm]
        upper = (lane & lm) != 0
        lanes = np.where(upper[:, None], other - lanes, lanes + other).astype(np.float32)
        lm <<= 1
    return lanes.reshape(-1)


@pytest.mark.parametrize("v", [1, 2, 4, 8])
def test_lane_butterflies_match_sequential(v):
    rng = np.random.default_rng(v)
    for _ in range(4):
        x = rng.normal(size=32 * v).astype(np.float32)
        want = hadamard_sequential(x)
        got = hadamard_lanes(x, v)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
