"""Generates tests/golden/golden_small.npz from the REFERENCE library
(oracle/_ref/libdsv4_ref.so, built from the reference's own sources by
oracle/Makefile). Run here, where the reference sources exist:

    make -C oracle && python tests/golden/make_golden.py

The fixture lets the oracle be checked against reference outputs on hosts
without the reference (the GPU box)."""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "..", "oracle"))
from oracle import Ref, make_moe_layer  # noqa: E402


def e8m0(rng, shape):
    return (127 + np.round(np.log2(rng.lognormal(0.0, 0.5, size=shape)))).astype(np.uint8)


def main():
    r = Ref()
    rng = np.random.default_rng(1234)
    g = {}
    g["quant_x"] = rng.normal(size=640).astype(np.float32) * np.float32(3.0)
    g["quant_qx"], g["quant_qs"] = r.quant_fp8_codes(g["quant_x"])
    qx, qs = r.quant_fp8_codes(rng.normal(size=512).astype(np.float32))
    g["fp4_qx"], g["fp4_qs"] = qx, qs
    g["fp4_W"] = rng.integers(0, 256, size=(96, 256), dtype=np.uint8)
    S = e8m0(rng, (96, 16))
    S[3, 5] = 255  # a NaN scale skips its group
    g["fp4_S"] = S
    g["fp4_y"] = r.gemv_fp4_q(qx, qs, g["fp4_W"], S, 512)
    qx, qs = r.quant_fp8_codes(rng.normal(size=384).astype(np.float32))
    g["fp8_qx"], g["fp8_qs"] = qx, qs
    W = rng.integers(0, 254, size=(160, 384)).astype(np.uint8)
    W[(W & 0x7F) == 0x7F] -= 1
    g["fp8_W"] = W
    g["fp8_S"] = e8m0(rng, (2, 3))
    g["fp8_y"] = r.gemv_fp8_q(qx, qs, W, g["fp8_S"], 1)
    x = rng.normal(size=300).astype(np.float32)
    g["bf16_x"] = x
    Wf = rng.normal(0, 0.05, size=(40, 300)).astype(np.float32)
    u = Wf.view(np.uint32).astype(np.uint64)
    g["bf16_W"] = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    g["bf16_y"] = r.gemv_bf16(x, g["bf16_W"], 0)
    H, d, n = 4, 64, 40
    g["attn_q"] = rng.normal(size=(H, d)).astype(np.float32)
    g["attn_kv"] = rng.normal(size=(48, d)).astype(np.float32)
    g["attn_sink"] = rng.normal(size=H).astype(np.float32)
    idx = rng.permutation(48)[:n].astype(np.int32)
    idx[7] = -1
    g["attn_idx"] = idx
    g["attn_scale"] = np.float32(d ** -0.5)
    g["attn_o"] = r.sparse_attn(g["attn_q"], g["attn_kv"], g["attn_sink"], idx, float(g["attn_scale"]))
    g["moe_seed"] = np.int64(7)
    L = make_moe_layer(256, 128, 16, 2, seed=7)
    xs = rng.normal(size=(4, 256)).astype(np.float32)
    xs = ((xs.view(np.uint32).astype(np.uint64) + 0x7FFF + ((xs.view(np.uint32).astype(np.uint64) >> 16) & 1)) >> 16 << 16).astype(np.uint32).view(np.float32)
    g["moe_x"] = xs
    outs, idxs, wts = [], [], []
    for t in range(xs.shape[0]):
        o, i, w = r.moe_forward(L, xs[t])
        outs.append(o); idxs.append(i); wts.append(w)
    g["moe_out"], g["moe_idx"], g["moe_wt"] = np.stack(outs), np.stack(idxs), np.stack(wts)
    np.savez_compressed(os.path.join(HERE, "golden_small.npz"), **g)
    print("wrote", os.path.join(HERE, "golden_small.npz"))


if __name__ == "__main__":
    main()
