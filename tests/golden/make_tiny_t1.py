"""Writes T1, a BASELINE-config-1-shaped random-init DeepSeek-V4-Flash
checkpoint, in the reference engine's checkpoint format.

    python tests/golden/make_tiny_t1.py <outdir> [seed]

Shape (benchmark config 1, mapped onto the reference's tensor set): vocab
1024, hidden 256, 2 layers; 4 attention heads over one shared latent of
head_dim 64 with 16 RoPE dims, q_lora 64, o_groups 2 x o_lora 64; 16 routed
FP4 experts top-2 plus one FP8 shared expert, moe_inter 128; hyper-connections
hc_mult 4; layer 1 is a ratio-4 compressed layer with an indexer (4 heads x
32, top-8) and the sliding window is 16, so a 48-token run wraps the ring and
uses the compressed path.

Tensor names, dtypes, shapes and the block layouts follow the contract of
the reference's tiny-fixture writer (tools/make_tiny_dsv4.py:218-282 in the
reference project): BF16 matrices, FP8 E4M3 weights with [128x128] E8M0
block scales, FP4 E2M1 experts (two codes per byte, low nibble first) with
per-32 E8M0 scales, F32 hyper-connection parameters. The values are this
script's own: every weight is N(0, 0.02) quantised to its format (the
smallest power-of-two scale that fits the block's largest magnitude, codes
rounded to the nearest representable value); RMSNorm weights are
1 + N(0, 0.02) and hyper-connection scales 1, so the residual stream keeps
its magnitude through the layers. numpy default_rng(seed), seed 0 by default.
"""
import json
import os
import struct
import sys

import numpy as np

CFG = dict(hidden=256, layers=2, vocab=1024, heads=4, head_dim=64, rope=16, q_lora=64,
           o_groups=2, o_lora=64, window=16, experts=16, topk=2, inter=128, hc=4,
           index_heads=4, index_dim=32, index_topk=8, ratios=[0, 4])

E2M1 = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], np.float64)


def config_json(c):
    return {
        "architectures": ["DeepseekV4ForCausalLM"], "model_type": "deepseek_v4",
        "hidden_size": c["hidden"], "num_hidden_layers": c["layers"],
        "vocab_size": c["vocab"], "max_position_embeddings": 4096,
        "num_attention_heads": c["heads"], "num_key_value_heads": 1,
        "head_dim": c["head_dim"], "qk_rope_head_dim": c["rope"], "q_lora_rank": c["q_lora"],
        "o_groups": c["o_groups"], "o_lora_rank": c["o_lora"], "sliding_window": c["window"],
        "n_routed_experts": c["experts"], "n_shared_experts": 1,
        "num_experts_per_tok": c["topk"], "num_hash_layers": 0,
        "moe_intermediate_size": c["inter"], "routed_scaling_factor": 1.5,
        "scoring_func": "sqrtsoftplus", "swiglu_limit": 10.0, "rms_norm_eps": 1e-6,
        "hc_mult": c["hc"], "hc_sinkhorn_iters": 20, "hc_eps": 1e-6,
        "rope_theta": 10000.0, "compress_rope_theta": 160000.0,
        "rope_scaling": {"factor": 16.0, "beta_fast": 32.0, "beta_slow": 1.0,
                         "original_max_position_embeddings": 256, "type": "yarn"},
        "index_n_heads": c["index_heads"], "index_head_dim": c["index_dim"],
        "index_topk": c["index_topk"], "compress_ratios": c["ratios"],
    }


def bf16_bits(x):
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def e4m3_codes(v):
    """Nearest E4M3 (e4m3fn) code of each value (|v| <= 448), ties to even."""
    v = np.asarray(v, np.float64)
    mags = np.array([(m / 512.0) if m < 8 else (1 + (m & 7) / 8.0) * 2.0 ** ((m >> 3) - 7)
                     for m in range(127)], np.float64)
    a = np.minimum(np.abs(v), 448.0)
    i = np.clip(np.searchsorted(mags, a), 1, 126)
    lo, hi = mags[i - 1], mags[i]
    pick_hi = (a - lo > hi - a) | ((a - lo == hi - a) & (i % 2 == 0))
    m = np.where(pick_hi, i, i - 1)
    return (m | np.where(v < 0, 0x80, 0)).astype(np.uint8)


def e8m0_for(amax, top):
    """Smallest power of two s with amax / s <= top, as an E8M0 code."""
    e = np.ceil(np.log2(np.maximum(amax, 1e-30) / top))
    return np.clip(e + 127, 1, 254).astype(np.uint8), 2.0 ** e


def fp8_matrix(w):
    rows, cols = w.shape
    rb, cb = (rows + 127) // 128, (cols + 127) // 128
    sc = np.empty((rb, cb), np.uint8)
    codes = np.empty(w.shape, np.uint8)
    for i in range(rb):
        for j in range(cb):
            blk = w[i * 128:(i + 1) * 128, j * 128:(j + 1) * 128]
            code, s = e8m0_for(np.abs(blk).max(), 448.0)
            sc[i, j] = code
            codes[i * 128:(i + 1) * 128, j * 128:(j + 1) * 128] = e4m3_codes(blk / s)
    return codes, sc


def fp4_matrix(w):
    rows, cols = w.shape
    g = w.reshape(rows, cols // 32, 32)
    code, s = e8m0_for(np.abs(g).max(axis=2), 6.0)
    q = g / s[:, :, None]
    mag = np.abs(q)
    idx = np.argmin(np.abs(mag[..., None] - E2M1), axis=-1)
    nib = (idx | np.where(q < 0, 8, 0)).astype(np.uint8).reshape(rows, cols)
    packed = (nib[:, 0::2] | (nib[:, 1::2] << 4)).astype(np.uint8)
    return packed, code.astype(np.uint8)


def build(seed=0, c=CFG):
    rng = np.random.default_rng(seed)
    H, V, nh, hd, ql = c["hidden"], c["vocab"], c["heads"], c["head_dim"], c["q_lora"]
    G, ol, ne, mi, mult = c["o_groups"], c["o_lora"], c["experts"], c["inter"], c["hc"]
    mix = (2 + mult) * mult
    t = []  # (name, dtype, shape, bytes)

    def n(*shape):
        return rng.normal(0.0, 0.02, size=shape)

    def bf16(name, x):
        t.append((name, "BF16", list(x.shape), bf16_bits(x).tobytes()))

    def f32(name, x):
        t.append((name, "F32", list(np.shape(x)), np.asarray(x, np.float32).tobytes()))

    def fp8(name, rows, cols):
        codes, sc = fp8_matrix(n(rows, cols))
        t.append((name + ".weight", "F8_E4M3", [rows, cols], codes.tobytes()))
        t.append((name + ".scale", "F8_E8M0", list(sc.shape), sc.tobytes()))

    def norm(name, k):
        bf16(name, 1.0 + n(k))

    bf16("embed.weight", n(V, H))
    bf16("head.weight", n(V, H))
    norm("norm.weight", H)
    f32("hc_head_fn", n(mult, mult * H))
    f32("hc_head_base", n(mult))
    f32("hc_head_scale", [1.0])
    for L in range(c["layers"]):
        p = f"layers.{L}."
        norm(p + "attn_norm.weight", H)
        norm(p + "ffn_norm.weight", H)
        f32(p + "hc_attn_fn", n(mix, mult * H))
        f32(p + "hc_ffn_fn", n(mix, mult * H))
        f32(p + "hc_attn_scale", [1.0, 1.0, 1.0])
        f32(p + "hc_ffn_scale", [1.0, 1.0, 1.0])
        f32(p + "hc_attn_base", n(mix))
        f32(p + "hc_ffn_base", n(mix))
        f32(p + "attn.attn_sink", n(nh))
        fp8(p + "attn.wq_a", ql, H)
        norm(p + "attn.q_norm.weight", ql)
        fp8(p + "attn.wq_b", nh * hd, ql)
        fp8(p + "attn.wkv", hd, H)
        norm(p + "attn.kv_norm.weight", hd)
        fp8(p + "attn.wo_a", G * ol, nh * hd // G)
        fp8(p + "attn.wo_b", H, G * ol)
        ratio = c["ratios"][L]
        if ratio:
            coff = 2 if ratio == 4 else 1
            f32(p + "attn.compressor.ape", n(ratio, coff * hd))
            bf16(p + "attn.compressor.wkv.weight", n(coff * hd, H))
            bf16(p + "attn.compressor.wgate.weight", n(coff * hd, H))
            norm(p + "attn.compressor.norm.weight", hd)
            if ratio == 4:
                ih, idim = c["index_heads"], c["index_dim"]
                fp8(p + "attn.indexer.wq_b", ih * idim, ql)
                bf16(p + "attn.indexer.weights_proj.weight", n(ih, H))
                f32(p + "attn.indexer.compressor.ape", n(ratio, coff * idim))
                bf16(p + "attn.indexer.compressor.wkv.weight", n(coff * idim, H))
                bf16(p + "attn.indexer.compressor.wgate.weight", n(coff * idim, H))
                norm(p + "attn.indexer.compressor.norm.weight", idim)
        bf16(p + "ffn.gate.weight", n(ne, H))
        f32(p + "ffn.gate.bias", n(ne))
        fp8(p + "ffn.shared_experts.w1", mi, H)
        fp8(p + "ffn.shared_experts.w3", mi, H)
        fp8(p + "ffn.shared_experts.w2", H, mi)
        for e in range(ne):
            q = f"{p}ffn.experts.{e}."
            w1, s1 = fp4_matrix(n(mi, H))
            w2, s2 = fp4_matrix(n(H, mi))
            w3, s3 = fp4_matrix(n(mi, H))
            # scale run (w1, w2, w3) then weight run, as the expert slots expect
            t.append((q + "w1.scale", "F8_E8M0", list(s1.shape), s1.tobytes()))
            t.append((q + "w2.scale", "F8_E8M0", list(s2.shape), s2.tobytes()))
            t.append((q + "w3.scale", "F8_E8M0", list(s3.shape), s3.tobytes()))
            t.append((q + "w1.weight", "I8", list(w1.shape), w1.tobytes()))
            t.append((q + "w2.weight", "I8", list(w2.shape), w2.tobytes()))
            t.append((q + "w3.weight", "I8", list(w3.shape), w3.tobytes()))
    return t


def write(outdir, seed=0, c=CFG):
    os.makedirs(outdir, exist_ok=True)
    tensors = build(seed, c)
    header, off = {}, 0
    for name, dt, shape, data in tensors:
        header[name] = {"dtype": dt, "shape": shape, "data_offsets": [off, off + len(data)]}
        off += len(data)
    hdr = json.dumps(header, separators=(",", ":")).encode()
    hdr += b" " * (-(len(hdr) + 8) % 8)  # tensor data 8-byte aligned in the file
    with open(os.path.join(outdir, "model-00001-of-00001.safetensors"), "wb") as f:
        f.write(struct.pack("<Q", len(hdr)))
        f.write(hdr)
        for _, _, _, data in tensors:
            f.write(data)
    with open(os.path.join(outdir, "config.json"), "w") as f:
        json.dump(config_json(c), f, indent=2)
    return outdir


def prompt_ids(seed=0, n=32, vocab=CFG["vocab"]):
    """The benchmark's prompt: n uniform-random token ids."""
    return np.random.default_rng(seed + 1).integers(0, vocab, size=n).tolist()


if __name__ == "__main__":
    out = write(sys.argv[1], int(sys.argv[2]) if len(sys.argv) > 2 else 0)
    print(out)
