"""Re-creates the deterministic inputs of the reference's kernel benchmark
(benchmarks/bench_dsv4_kernels.c:25-120): one xorshift64 stream (13, 7, 17)
seeded 0x9E3779B97F4A7C15 fills, in order, x2048[4096], x4096[4096] (floats
(x % 2001 - 1000) / 1000), three packed FP4 matrices (low bytes), one FP8
matrix (x % 127) and one BF16 matrix; every E8M0 scale is 127. The checksum
is sqrt(sum v^2) in double, printed as a float with %.6f.

Test infrastructure: used by tests/test_oracle_golden.py and the GPU parity
tests to pin results against the golden checksums the reference prints.
"""
import numpy as np

SEED = 0x9E3779B97F4A7C15
R1, C1 = 2048, 4096
R2, C2 = 4096, 2048
R3, C3 = 4096, 4096
R4, C4 = 1024, 4096

# Printed by the reference's bench (verified by building and running it).
GOLDEN = {
    "fp4_2048x4096": "4785.732910",
    "fp4_pair": ("4785.732910", "5041.146484"),
    "fp4_batch6": "4785.732910",
    "fp4_4096x2048": "4841.937500",
    "fp8_4096x4096": "215265.046875",
    "bf16_1024x4096": "663.993408",
}


def _unit(v):
    return (((v % np.uint64(2001)).astype(np.int64) - 1000).astype(np.float32)
            / np.float32(1000.0))


def _bf16(f):
    u = f.view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return u.astype(np.uint16)


def make(orc):
    """Returns the benchmark's inputs using the oracle's xorshift helpers."""
    st = SEED
    raw, st = orc.xs_next_many(C1, st)
    x2048 = _unit(raw)
    raw, st = orc.xs_next_many(C3, st)
    x4096 = _unit(raw)
    w2048, st = orc.xs_fill_u8(R1 * (C1 // 2), st)
    w2048p, st = orc.xs_fill_u8(R1 * (C1 // 2), st)
    w4096d, st = orc.xs_fill_u8(R2 * (C2 // 2), st)
    w4096f, st = orc.xs_fill_u8(R3 * C3, st, 127)
    raw, st = orc.xs_next_many(R4 * C4, st)
    w1024b = _bf16(_unit(raw))
    return dict(
        x2048=x2048, x4096=x4096,
        w2048=w2048.reshape(R1, C1 // 2), w2048p=w2048p.reshape(R1, C1 // 2),
        w4096d=w4096d.reshape(R2, C2 // 2), w4096f=w4096f.reshape(R3, C3),
        w1024b=w1024b.reshape(R4, C4),
        s2048=np.full((R1, C1 // 32), 127, np.uint8),
        s4096d=np.full((R2, C2 // 32), 127, np.uint8),
        s4096f=np.full((R3 // 128, C3 // 128), 127, np.uint8),
    )


def checksum(y):
    return "%.6f" % float(np.float32(np.sqrt(np.sum(np.asarray(y, np.float64) ** 2))))
