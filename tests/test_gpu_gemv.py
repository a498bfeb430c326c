"""GPU parity of the drop-in kernel ABI (libdsv4_cuda.so through ctypes)
against the CPU oracle: bit-exact on every shape, including the reference
benchmark's golden checksums and the MoE config's expert shapes."""
import numpy as np
import pytest

import bench_inputs as B

pytestmark = pytest.mark.gpu


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def e8m0(rng, shape, nan_frac=0.0):
    s = (127 + np.round(np.log2(rng.lognormal(0.0, 0.5, size=shape)))).astype(np.uint8)
    if nan_frac:
        s[rng.random(shape) < nan_frac] = 255
    return s


@pytest.fixture(scope="module")
def bench(orc):
    return B.make(orc)


def test_bench_golden_checksums(cuda, orc, bench):
    d = bench
    qx, qs = cuda.quant_fp8_codes(d["x2048"])
    oq = orc.quant_fp8_codes(d["x2048"])
    assert np.array_equal(bits(qx), bits(oq[0])) and np.array_equal(bits(qs), bits(oq[1]))
    assert B.checksum(cuda.gemv_fp4_q(qx, qs, d["w2048"], d["s2048"], B.C1)) == B.GOLDEN["fp4_2048x4096"]
    a, b = cuda.gemv_fp4_pair_q(qx, qs, d["w2048"], d["s2048"], d["w2048p"], d["s2048"], B.C1)
    assert (B.checksum(a), B.checksum(b)) == B.GOLDEN["fp4_pair"]
    ys = cuda.gemv_fp4_batch_q([qx] * 6, [qs] * 6, d["w2048"], d["s2048"], B.C1)
    assert all(B.checksum(y) == B.GOLDEN["fp4_batch6"] for y in ys)
    qx4, qs4 = cuda.quant_fp8_codes(d["x4096"])
    assert B.checksum(cuda.gemv_fp4_q(qx4[:B.C2], qs4, d["w4096d"], d["s4096d"], B.C2)) == B.GOLDEN["fp4_4096x2048"]
    assert B.checksum(cuda.gemv_fp8_q(qx4, qs4, d["w4096f"], d["s4096f"], 1)) == B.GOLDEN["fp8_4096x4096"]
    assert B.checksum(cuda.gemv_bf16(d["x4096"], d["w1024b"], 1)) == B.GOLDEN["bf16_1024x4096"]


@pytest.mark.parametrize("inn,rows", [(7168, 2048), (2048, 7168), (4096, 2048), (256, 128),
                                      (128, 256), (96, 40), (512, 33)])
def test_fp4_exact(cuda, orc, inn, rows):
    rng = np.random.default_rng(inn * 7 + rows)
    W0 = rng.integers(0, 256, size=(rows, (inn + 1) // 2), dtype=np.uint8)
    W1 = rng.integers(0, 256, size=(rows, (inn + 1) // 2), dtype=np.uint8)
    S0 = e8m0(rng, (rows, (inn + 31) // 32), 0.01)
    S1 = e8m0(rng, (rows, (inn + 31) // 32))
    qx, qs = orc.quant_fp8_codes(rng.normal(size=inn).astype(np.float32))
    assert np.array_equal(bits(cuda.gemv_fp4_q(qx, qs, W0, S0, inn)),
                          bits(orc.gemv_fp4_q(qx, qs, W0, S0, inn)))
    a = cuda.gemv_fp4_pair_q(qx, qs, W0, S0, W1, S1, inn)
    b = orc.gemv_fp4_pair_q(qx, qs, W0, S0, W1, S1, inn)
    assert np.array_equal(bits(a[0]), bits(b[0])) and np.array_equal(bits(a[1]), bits(b[1]))


@pytest.mark.parametrize("batch", [1, 2, 3, 5, 8, 9, 17, 33])
def test_fp4_batch_exact(cuda, orc, batch):
    rng = np.random.default_rng(batch)
    inn, rows = 2048, 96
    W = rng.integers(0, 256, size=(rows, inn // 2), dtype=np.uint8)
    S = e8m0(rng, (rows, inn // 32))
    qxs, qss = zip(*[orc.quant_fp8_codes(rng.normal(size=inn).astype(np.float32)) for _ in range(batch)])
    assert np.array_equal(bits(cuda.gemv_fp4_batch_q(qxs, qss, W, S, inn)),
                          bits(orc.gemv_fp4_batch_q(qxs, qss, W, S, inn)))


def test_fp4_non_grid_activation(cuda, orc):
    """qx values that are not E4M3/f16-exact take the fp32 activation path."""
    rng = np.random.default_rng(3)
    inn, rows = 256, 64
    W = rng.integers(0, 256, size=(rows, inn // 2), dtype=np.uint8)
    S = e8m0(rng, (rows, inn // 32))
    qx = rng.normal(size=inn).astype(np.float32)
    qs = np.array([0.5, 0.25], np.float32)
    assert np.array_equal(bits(cuda.gemv_fp4_q(qx, qs, W, S, inn)),
                          bits(orc.gemv_fp4_q(qx, qs, W, S, inn)))


@pytest.mark.parametrize("inn,rows", [(7168, 2048), (2048, 7168), (1024, 4096), (384, 130),
                                      (200, 17)])
def test_fp8_exact(cuda, orc, inn, rows):
    rng = np.random.default_rng(inn + 3 * rows)
    W = rng.integers(0, 254, size=(rows, inn)).astype(np.uint8)
    W[(W & 0x7F) == 0x7F] -= 1
    W1 = rng.integers(0, 126, size=(rows, inn)).astype(np.uint8)
    S = e8m0(rng, ((rows + 127) // 128, (inn + 127) // 128), 0.05)
    qx, qs = orc.quant_fp8_codes(rng.normal(size=inn).astype(np.float32))
    for ro in (0, 1):
        assert np.array_equal(bits(cuda.gemv_fp8_q(qx, qs, W, S, ro)),
                              bits(orc.gemv_fp8_q(qx, qs, W, S, ro)))
    a = cuda.gemv_fp8_pair_q(qx, qs, W, S, W1, S)
    b = orc.gemv_fp8_pair_q(qx, qs, W, S, W1, S)
    assert np.array_equal(bits(a[0]), bits(b[0])) and np.array_equal(bits(a[1]), bits(b[1]))
    qxs, qss = zip(*[orc.quant_fp8_codes(rng.normal(size=inn).astype(np.float32)) for _ in range(5)])
    assert np.array_equal(bits(cuda.gemv_fp8_batch_q(qxs, qss, W, S, 1)),
                          bits(orc.gemv_fp8_batch_q(qxs, qss, W, S, 1)))


@pytest.mark.parametrize("inn,rows,batch", [(4096, 256, 1), (520, 72, 3), (7168, 256, 2),
                                            (100, 9, 1)])
def test_bf16_exact(cuda, orc, inn, rows, batch):
    rng = np.random.default_rng(inn + rows)
    Wf = rng.normal(0, 0.05, size=(rows, inn)).astype(np.float32)
    u = Wf.view(np.uint32).astype(np.uint64)
    W = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    xs = [rng.normal(size=inn).astype(np.float32) for _ in range(batch)]
    for ro in (0, 1):
        assert np.array_equal(bits(cuda.gemv_bf16_batch(xs, W, ro)),
                              bits(orc.gemv_bf16_batch(xs, W, ro)))


@pytest.mark.parametrize("n", [1, 127, 128, 7168, 1000])
def test_quant_exact(cuda, orc, n):
    rng = np.random.default_rng(n)
    for scale in (1e-7, 1.0, 5e3):
        x = (rng.normal(size=n) * scale).astype(np.float32)
        a, b = cuda.quant_fp8_codes(x), orc.quant_fp8_codes(x)
        assert np.array_equal(bits(a[0]), bits(b[0])) and np.array_equal(bits(a[1]), bits(b[1]))


def test_quant_e4m3_boundaries(cuda, orc):
    # values that land on the E4M3 subnormal/normal midpoint and on ties
    x = np.array([15.0 / 1024.0, np.nextafter(np.float32(15.0 / 1024.0), np.float32(0)),
                  448.0, 464.0, 0.0, -0.0] + [i / 512.0 for i in range(122)], np.float32)
    a, b = cuda.quant_fp8_codes(x), orc.quant_fp8_codes(x)
    assert np.array_equal(bits(a[0]), bits(b[0])) and np.array_equal(bits(a[1]), bits(b[1]))
