"""GPU parity of the device-resident MoE layer (dsv4cuda_moe_*) against the
CPU oracle of moe_forward (src/dsv4/dsv4_model.c:6599).

Bar: routed expert ids bit-exact; outputs within a relative tolerance of
1e-2 of the output RMS (transcendentals - expf in SiLU, expf/log1pf in the
router score - may differ from glibc in the last ulp); in practice almost all
elements are bit-identical, which the tests also report and bound."""
import numpy as np
import pytest
import torch

from oracle import make_moe_layer

pytestmark = pytest.mark.gpu
TOL = 1e-2


def bf16_vals(rng, shape):
    x = rng.normal(size=shape).astype(np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    return (((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16).astype(np.uint32).view(np.float32)


def check_close(got, want, min_exact=0.9):
    rms = float(np.sqrt(np.mean(want.astype(np.float64) ** 2))) + 1e-30
    err = float(np.max(np.abs(got.astype(np.float64) - want))) / rms
    exact = float(np.mean(got.view(np.uint32) == want.view(np.uint32)))
    assert err <= TOL, (err, exact)
    assert exact >= min_exact, (err, exact)
    return err, exact


@pytest.mark.parametrize("cfg", [
    dict(hid=256, mi=128, E=16, k=2, shared="fp8", hv=0),     # benchmark config-1 MoE shape
    dict(hid=256, mi=128, E=16, k=2, shared="fp4", hv=0),
    dict(hid=256, mi=128, E=16, k=2, shared="fp8", hv=40),    # hash layer
    dict(hid=1024, mi=512, E=64, k=6, shared=None, hv=0),
])
def test_moe_small(cuda, orc, cfg):
    L = make_moe_layer(cfg["hid"], cfg["mi"], cfg["E"], cfg["k"], seed=cfg["E"] + cfg["hv"],
                       shared=cfg["shared"], hash_vocab=cfg["hv"])
    layer = cuda.MoeLayer(L, max_tokens=8)
    rng = np.random.default_rng(1)
    M = 8
    x = bf16_vals(rng, (M, cfg["hid"]))
    tok = np.arange(M, dtype=np.int32) * 3 % max(cfg["hv"], 1)
    got = layer.forward_host(x, tok if cfg["hv"] else None)
    idx, wt, _ = layer.last_routes(M)
    for t in range(M):
        want, widx, wwt = orc.moe_forward(L, x[t], token_id=int(tok[t]))
        assert np.array_equal(idx[t], widx), (t, idx[t], widx)
        np.testing.assert_allclose(wt[t], wwt, rtol=1e-5)
        check_close(got[t], want)
    layer.close()


def test_moe_batch_equals_single(cuda):
    """moe_forward_batch semantics: a token's result does not depend on its
    batch (src/dsv4/dsv4_model.c:6809-6811)."""
    L = make_moe_layer(512, 256, 32, 4, seed=5)
    layer = cuda.MoeLayer(L, max_tokens=8)
    x = bf16_vals(np.random.default_rng(2), (8, 512))
    batched = layer.forward_host(x)
    for t in range(8):
        single = layer.forward_host(x[t:t + 1])
        assert np.array_equal(single[0].view(np.uint32), batched[t].view(np.uint32))
    layer.close()


def test_moe_config2_shapes(cuda, orc):
    """Config-2 expert shapes (hidden 7168, inter 2048, top-8, FP8 shared)
    with 32 experts so the oracle stays fast."""
    L = make_moe_layer(7168, 2048, 32, 8, seed=11, shared="fp8")
    layer = cuda.MoeLayer(L, max_tokens=4)
    x = bf16_vals(np.random.default_rng(3), (2, 7168))
    got = layer.forward_host(x)
    idx, wt, _ = layer.last_routes(2)
    for t in range(2):
        want, widx, wwt = orc.moe_forward(L, x[t])
        assert np.array_equal(idx[t], widx)
        check_close(got[t], want)
    layer.close()


def test_moe_device_api_matches_host_api(cuda):
    L = make_moe_layer(256, 128, 16, 2, seed=9)
    layer = cuda.MoeLayer(L, max_tokens=4)
    x = bf16_vals(np.random.default_rng(4), (4, 256))
    host = layer.forward_host(x)
    xd = torch.from_numpy(x).cuda()
    out = torch.empty_like(xd)
    layer.forward(xd, out)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy().view(np.uint32), host.view(np.uint32))
    layer.close()


def test_router_exact_tie_takes_lower_id(cuda, orc):
    """Two experts with identical gate rows tie exactly at the top-k boundary:
    the reference keeps the lower id (strict > scan). The device router's
    margin check must detect the tie and replay the exact fp32 logits."""
    L = make_moe_layer(256, 128, 16, 2, seed=21, bias=False)
    x = bf16_vals(np.random.default_rng(5), (1, 256))[0]
    z = (L["gate_w"].astype(np.uint32) << 16).view(np.float32) @ x
    order = np.argsort(-z)
    e2 = int(order[1])                                  # second place
    j = min(e for e in range(16) if e not in (int(order[0]), e2))
    L["gate_w"][j] = L["gate_w"][e2]                    # exact tie for second place
    lo, hi = min(j, e2), max(j, e2)
    want, widx, _ = orc.moe_forward(L, x)
    layer = cuda.MoeLayer(L, max_tokens=1)
    got = layer.forward_host(x[None])
    idx, _, fallbacks = layer.last_routes(1)
    assert np.array_equal(idx[0], widx), (idx[0], widx)
    assert lo in widx and hi not in widx and int(order[0]) in widx
    assert fallbacks >= 1
    check_close(got[0], want)
    layer.close()


def test_router_public_dropin(cuda, orc):
    L = make_moe_layer(512, 128, 64, 6, seed=4, hash_vocab=10)
    rng = np.random.default_rng(8)
    for t in range(4):
        x = rng.normal(size=512).astype(np.float32)
        a = cuda.router_public(x, L["gate_w"], L["bias"], 6, 1.5)
        b = orc.router_public(x, L["gate_w"], L["bias"], 6, 1.5)
        assert np.array_equal(a[0], b[0])
        np.testing.assert_allclose(a[1], b[1], rtol=1e-5)
        a = cuda.router_public(x, L["gate_w"], L["bias"], 6, 1.5, L["tid2eid"], t)
        b = orc.router_public(x, L["gate_w"], L["bias"], 6, 1.5, L["tid2eid"], t)
        assert np.array_equal(a[0], b[0])
        np.testing.assert_allclose(a[1], b[1], rtol=1e-5)
