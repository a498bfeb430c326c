"""Pins the CPU oracle (oracle/dsv4_oracle.c) to the reference's own known
answers: the KATs of tests/unit/test_dsv4_ops.c, the golden checksums its
kernel benchmark prints (benchmarks/bench_dsv4_kernels.c) and the fixture
vectors in tests/golden/ generated from the reference library."""
import math
import os

import numpy as np
import pytest

import bench_inputs as B

GOLDEN_NPZ = os.path.join(os.path.dirname(__file__), "golden", "golden_small.npz")


def test_bf16_rne(orc):
    # tests/unit/test_dsv4_ops.c:24-30
    assert orc.f32_to_bf16(1.0) == 0x3F80
    assert orc.f32_to_bf16(1.0 + 2.0 ** -8) == 0x3F80   # tie rounds to even
    assert orc.f32_to_bf16(1.0 + 2.0 ** -7) == 0x3F81


def test_e4m3_decode(orc):
    # tests/unit/test_dsv4_ops.c:33-42
    assert orc.e4m3(0x00) == 0.0
    assert orc.e4m3(0x7E) == 448.0
    assert orc.e4m3(0xFE) == -448.0
    assert orc.e4m3(0x3F) == 1.875
    assert orc.e4m3(0x38) == 1.0
    assert orc.e4m3(0x01) == 2.0 ** -9
    assert math.isnan(orc.e4m3(0x7F))


def test_e4m3_subnormal_boundary(orc):
    # tests/unit/test_dsv4_ops.c:43-54
    mid = np.float32(15.0 / 1024.0)
    below = np.nextafter(mid, np.float32(0.0))
    above = np.nextafter(mid, np.float32(1.0))
    assert orc.round_e4m3(float(below)) == 7.0 / 512.0
    assert orc.round_e4m3(float(mid)) == 8.0 / 512.0
    assert orc.round_e4m3(float(above)) == 8.0 / 512.0
    assert orc.round_e4m3(float(-mid)) == -8.0 / 512.0


def test_e8m0(orc):
    # tests/unit/test_dsv4_ops.c:57-60
    assert orc.e8m0(127) == 1.0 and orc.e8m0(126) == 0.5 and orc.e8m0(128) == 2.0
    assert math.isnan(orc.e8m0(255))


def test_act_quant_pow2_and_clamp(orc):
    # tests/unit/test_dsv4_ops.c:63-79
    x = np.array([-1.0 if i % 2 == 0 else 1.0 for i in range(128)], np.float32)
    q, s = orc.quant_fp8_codes(x)
    assert s[0] == 2.0 ** -8 and q[0] == -256.0 and q[1] == 256.0
    big = np.zeros(128, np.float32)
    big[0] = 448.0 * 1024.0
    q, s = orc.quant_fp8_codes(big)
    assert s[0] == 2.0 ** 10 and q[0] == 448.0


@pytest.fixture(scope="module")
def bench(orc):
    return B.make(orc)


def test_bench_checksums_fp4(orc, bench):
    d = bench
    qx, qs = orc.quant_fp8_codes(d["x2048"])
    assert B.checksum(orc.gemv_fp4_q(qx, qs, d["w2048"], d["s2048"], B.C1)) == B.GOLDEN["fp4_2048x4096"]
    a, b = orc.gemv_fp4_pair_q(qx, qs, d["w2048"], d["s2048"], d["w2048p"], d["s2048"], B.C1)
    assert (B.checksum(a), B.checksum(b)) == B.GOLDEN["fp4_pair"]
    ys = orc.gemv_fp4_batch_q([qx] * 6, [qs] * 6, d["w2048"], d["s2048"], B.C1)
    assert B.checksum(ys[0]) == B.GOLDEN["fp4_batch6"]
    qx4, qs4 = orc.quant_fp8_codes(d["x4096"])
    y = orc.gemv_fp4_q(qx4[:B.C2], qs4, d["w4096d"], d["s4096d"], B.C2)
    assert B.checksum(y) == B.GOLDEN["fp4_4096x2048"]


def test_bench_checksums_fp8_bf16(orc, bench):
    d = bench
    qx4, qs4 = orc.quant_fp8_codes(d["x4096"])
    assert B.checksum(orc.gemv_fp8_q(qx4, qs4, d["w4096f"], d["s4096f"], 1)) == B.GOLDEN["fp8_4096x4096"]
    assert B.checksum(orc.gemv_bf16(d["x4096"], d["w1024b"], 1)) == B.GOLDEN["bf16_1024x4096"]


def test_golden_fixtures(orc):
    """Vectors produced by the reference library (tests/golden/make_golden.py)."""
    g = np.load(GOLDEN_NPZ)
    qx, qs = orc.quant_fp8_codes(g["quant_x"])
    assert np.array_equal(qx.view(np.uint32), g["quant_qx"].view(np.uint32))
    assert np.array_equal(qs, g["quant_qs"])
    y = orc.gemv_fp4_q(g["fp4_qx"], g["fp4_qs"], g["fp4_W"], g["fp4_S"], g["fp4_qx"].size)
    assert np.array_equal(y.view(np.uint32), g["fp4_y"].view(np.uint32))
    y = orc.gemv_fp8_q(g["fp8_qx"], g["fp8_qs"], g["fp8_W"], g["fp8_S"], 1)
    assert np.array_equal(y.view(np.uint32), g["fp8_y"].view(np.uint32))
    y = orc.gemv_bf16(g["bf16_x"], g["bf16_W"], 0)
    assert np.array_equal(y.view(np.uint32), g["bf16_y"].view(np.uint32))
    o = orc.sparse_attn(g["attn_q"], g["attn_kv"], g["attn_sink"], g["attn_idx"],
                        float(g["attn_scale"]))
    assert np.array_equal(o.view(np.uint32), g["attn_o"].view(np.uint32))
    from oracle import make_moe_layer
    L = make_moe_layer(256, 128, 16, 2, seed=int(g["moe_seed"]))
    for t in range(g["moe_x"].shape[0]):
        out, idx, wt = orc.moe_forward(L, g["moe_x"][t])
        assert np.array_equal(idx, g["moe_idx"][t])
        assert np.array_equal(wt.view(np.uint32), g["moe_wt"][t].view(np.uint32))
        assert np.array_equal(out.view(np.uint32), g["moe_out"][t].view(np.uint32))
