"""The C restatement against the reference itself (oracle/_ref, compiled from
the reference's sources): bit-identical on seeded random inputs, edge cases
included (NaN block scales, ragged tails, hash layers, padding)."""
import numpy as np
import pytest

from oracle import make_moe_layer


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def e8m0(rng, shape, nan_frac=0.0):
    s = (127 + np.round(np.log2(rng.lognormal(0.0, 0.5, size=shape)))).astype(np.uint8)
    if nan_frac:
        s[rng.random(shape) < nan_frac] = 255
    return s


@pytest.mark.parametrize("n", [1, 100, 128, 7168, 333])
def test_quant(orc, ref, n):
    rng = np.random.default_rng(n)
    x = (rng.normal(size=n) * rng.choice([1e-6, 1.0, 300.0])).astype(np.float32)
    a, b = orc.quant_fp8_codes(x), ref.quant_fp8_codes(x)
    assert np.array_equal(bits(a[0]), bits(b[0])) and np.array_equal(bits(a[1]), bits(b[1]))


def test_round_e4m3_sweep(orc, ref):
    rng = np.random.default_rng(0)
    vals = np.concatenate([rng.uniform(-460, 460, 3000), rng.uniform(-0.02, 0.02, 3000),
                           np.arange(-4096, 4097) / 512.0]).astype(np.float32)
    for v in vals[::7]:
        assert orc.round_e4m3(float(v)) == ref.round_e4m3(float(v))


@pytest.mark.parametrize("inn,rows", [(256, 24), (512, 33), (2048, 16), (96, 8), (7168, 8)])
def test_fp4_family(orc, ref, inn, rows):
    rng = np.random.default_rng(inn + rows)
    W0 = rng.integers(0, 256, size=(rows, (inn + 1) // 2), dtype=np.uint8)
    W1 = rng.integers(0, 256, size=(rows, (inn + 1) // 2), dtype=np.uint8)
    S0 = e8m0(rng, (rows, (inn + 31) // 32), 0.02)
    S1 = e8m0(rng, (rows, (inn + 31) // 32))
    qxs, qss = zip(*[orc.quant_fp8_codes(rng.normal(size=inn).astype(np.float32)) for _ in range(3)])
    assert np.array_equal(bits(orc.gemv_fp4_q(qxs[0], qss[0], W0, S0, inn)),
                          bits(ref.gemv_fp4_q(qxs[0], qss[0], W0, S0, inn)))
    assert np.array_equal(bits(orc.gemv_fp4_batch_q(qxs, qss, W0, S0, inn)),
                          bits(ref.gemv_fp4_batch_q(qxs, qss, W0, S0, inn)))
    a = orc.gemv_fp4_pair_q(qxs[1], qss[1], W0, S0, W1, S1, inn)
    b = ref.gemv_fp4_pair_q(qxs[1], qss[1], W0, S0, W1, S1, inn)
    assert np.array_equal(bits(a[0]), bits(b[0])) and np.array_equal(bits(a[1]), bits(b[1]))


@pytest.mark.parametrize("inn,rows", [(384, 130), (1024, 64), (200, 17)])
def test_fp8_family(orc, ref, inn, rows):
    rng = np.random.default_rng(inn * 3 + rows)
    W = rng.integers(0, 254, size=(rows, inn)).astype(np.uint8)
    W[(W & 0x7F) == 0x7F] -= 1
    W1 = rng.integers(0, 126, size=(rows, inn)).astype(np.uint8)
    S = e8m0(rng, ((rows + 127) // 128, (inn + 127) // 128), 0.1)
    qxs, qss = zip(*[orc.quant_fp8_codes(rng.normal(size=inn).astype(np.float32)) for _ in range(2)])
    for ro in (0, 1):
        assert np.array_equal(bits(orc.gemv_fp8_q(qxs[0], qss[0], W, S, ro)),
                              bits(ref.gemv_fp8_q(qxs[0], qss[0], W, S, ro)))
        assert np.array_equal(bits(orc.gemv_fp8_batch_q(qxs, qss, W, S, ro)),
                              bits(ref.gemv_fp8_batch_q(qxs, qss, W, S, ro)))
    a = orc.gemv_fp8_pair_q(qxs[0], qss[0], W, S, W1, S)
    b = ref.gemv_fp8_pair_q(qxs[0], qss[0], W, S, W1, S)
    assert np.array_equal(bits(a[0]), bits(b[0])) and np.array_equal(bits(a[1]), bits(b[1]))


def test_bf16_family(orc, ref):
    rng = np.random.default_rng(5)
    W = rng.integers(0, 65536, size=(72, 520), dtype=np.uint16) & 0xBFFF  # finite values
    xs = [rng.normal(size=520).astype(np.float32) for _ in range(3)]
    for ro in (0, 1):
        assert np.array_equal(bits(orc.gemv_bf16(xs[0], W, ro)), bits(ref.gemv_bf16(xs[0], W, ro)))
        assert np.array_equal(bits(orc.gemv_bf16_batch(xs, W, ro)),
                              bits(ref.gemv_bf16_batch(xs, W, ro)))


@pytest.mark.parametrize("weight", [1.0, 0.37, 1e-3])
def test_swiglu_quant(orc, ref, weight):
    rng = np.random.default_rng(9)
    g = (rng.normal(size=2048) * 6).astype(np.float32)
    u = (rng.normal(size=2048) * 6).astype(np.float32)
    a, b = orc.swiglu_quant(g, u, 10, weight), ref.swiglu_quant(g, u, 10, weight)
    for x, y in zip(a, b):
        assert np.array_equal(bits(x), bits(y))


def test_sqrt_softplus(orc, ref):
    for z in np.linspace(-30, 30, 601, dtype=np.float32):
        assert orc.sqrt_softplus(float(z)) == ref.sqrt_softplus(float(z))


@pytest.mark.parametrize("hash_vocab", [0, 50])
def test_router_public(orc, ref, hash_vocab):
    L = make_moe_layer(256, 128, 32, 4, seed=3, hash_vocab=hash_vocab)
    rng = np.random.default_rng(11)
    for t in range(5):
        x = rng.normal(size=256).astype(np.float32)
        a = orc.router_public(x, L["gate_w"], L["bias"], 4, 1.5, L["tid2eid"], t)
        b = ref.router_public(x, L["gate_w"], L["bias"], 4, 1.5, L["tid2eid"], t)
        assert np.array_equal(a[0], b[0]) and np.array_equal(bits(a[1]), bits(b[1]))


@pytest.mark.parametrize("cfg", [dict(hid=256, mi=128, E=16, k=2, hv=0),
                                 dict(hid=512, mi=256, E=64, k=6, hv=0),
                                 dict(hid=256, mi=128, E=16, k=2, hv=20)])
def test_moe_forward(orc, ref, cfg):
    L = make_moe_layer(cfg["hid"], cfg["mi"], cfg["E"], cfg["k"], seed=cfg["E"],
                       hash_vocab=cfg["hv"])
    slots = ref.pack_slots(L)
    rng = np.random.default_rng(cfg["E"] + 1)
    for t in range(4):
        x = rng.normal(size=cfg["hid"]).astype(np.float32)
        a = orc.moe_forward(L, x, token_id=t)
        b = ref.moe_forward(L, x, token_id=t, slots=slots)
        assert np.array_equal(a[1], b[1])
        assert np.array_equal(bits(a[2]), bits(b[2]))
        assert np.array_equal(bits(a[0]), bits(b[0]))


@pytest.mark.parametrize("H,d,n", [(4, 64, 40), (8, 512, 130), (2, 32, 5)])
def test_sparse_attn(orc, ref, H, d, n):
    rng = np.random.default_rng(H * d + n)
    q = rng.normal(size=(H, d)).astype(np.float32)
    kv = rng.normal(size=(n + 3, d)).astype(np.float32)
    sink = rng.normal(size=H).astype(np.float32)
    idx = rng.permutation(n + 3)[:n].astype(np.int32)
    idx[::9] = -1
    a = orc.sparse_attn(q, kv, sink, idx, d ** -0.5)
    b = ref.sparse_attn(q, kv, sink, idx, d ** -0.5)
    assert np.array_equal(bits(a), bits(b))
