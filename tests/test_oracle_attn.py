"""CPU checks of the attention pieces of the oracle against the reference
library built from its own sources (no GPU)."""
import numpy as np
import pytest


def test_rope_inv_matches_reference(orc, ref):
    rng = np.random.default_rng(7)
    for heads, d, n in ((1, 512, 32), (4, 32, 8), (128, 512, 32)):
        x = rng.normal(size=(heads, d)).astype(np.float32)
        ang = rng.uniform(0, 6.3, size=n).astype(np.float32)
        c, s = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
        a = orc.rope_inv(x, c, s)
        b = ref.rope_inv(x, c, s)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


@pytest.mark.parametrize("n,H,d", [(0, 2, 32), (1, 4, 32), (37, 4, 32), (300, 8, 512)])
def test_sparse_attn_matches_reference(orc, ref, n, H, d):
    rng = np.random.default_rng(n + H)
    rows = max(n, 1) + 3
    q = rng.normal(size=(H, d)).astype(np.float32)
    kv = rng.normal(size=(rows, d)).astype(np.float32)
    sink = rng.normal(size=H).astype(np.float32)
    idx = rng.integers(0, rows, size=n).astype(np.int32)
    if n > 4:
        idx[::5] = -1
    a = orc.sparse_attn(q, kv, sink, idx, d ** -0.5)
    b = ref.sparse_attn(q, kv, sink, idx, d ** -0.5)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_kv_quant_matches_reference(orc, ref):
    """The FP8 latent-cache values are dsv4_act_quant_inplace(group 64, mode 0)."""
    rng = np.random.default_rng(3)
    x = rng.normal(size=(16, 448)).astype(np.float32)
    x[1] = 0.0
    x[2] *= 1e-6
    x[3] *= 1e4
    for r in range(x.shape[0]):
        a = orc.act_quant_inplace(x[r], 64, 0)
        b = ref.act_quant_inplace(x[r], 64, 0)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
