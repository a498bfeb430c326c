"""Random-init checkpoints in the reference engine's format, at any
DeepSeek-V4-Flash shape, for timing the reference's own decode on the host
(the CPU baseline of bench.py --workload decode).

TEST/BENCH INFRASTRUCTURE ONLY. The tensor names, dtypes, shapes and block
layouts follow the reference's checkpoint contract (the tensor set its tiny
fixture writer emits, tools/make_tiny_dsv4.py:218-282 in the reference
project). Values are drawn directly in their storage formats so that a
multi-GB checkpoint is written in seconds: FP4 / FP8 codes uniform over the
finite codes, E8M0 scales 127 + round(N(0, 0.5 / ln 2)) (lognormal(0, 0.5)
rounded to a power of two), BF16 N(0, 0.02), RMSNorm gains 1 + N(0, 0.02),
hyper-connection parameters N(0, 0.02) with unit scales, compressor APE
N(0, 0.02). Layer L has compress ratio c["ratios"][L] (default 0,
sliding-window attention); ratio-4 / ratio-128 layers carry the compressor
and, for ratio 4, the indexer tensors of the same contract.
"""
import json
import os
import struct

import numpy as np

CONFIG5 = dict(hidden=4096, vocab=129280, heads=64, head_dim=512, rope=64, q_lora=1024,
               o_groups=8, o_lora=1024, window=128, experts=256, topk=6, inter=2048, hc=4)


def config_json(c, n_layers):
    return {
        "architectures": ["DeepseekV4ForCausalLM"], "model_type": "deepseek_v4",
        "hidden_size": c["hidden"], "num_hidden_layers": n_layers, "vocab_size": c["vocab"],
        "max_position_embeddings": 65536, "num_attention_heads": c["heads"],
        "num_key_value_heads": 1, "head_dim": c["head_dim"], "qk_rope_head_dim": c["rope"],
        "q_lora_rank": c["q_lora"], "o_groups": c["o_groups"], "o_lora_rank": c["o_lora"],
        "sliding_window": c["window"], "n_routed_experts": c["experts"], "n_shared_experts": 1,
        "num_experts_per_tok": c["topk"], "num_hash_layers": 0,
        "moe_intermediate_size": c["inter"], "routed_scaling_factor": 1.5,
        "scoring_func": "sqrtsoftplus", "swiglu_limit": 10.0, "rms_norm_eps": 1e-6,
        "hc_mult": c["hc"], "hc_sinkhorn_iters": 20, "hc_eps": 1e-6, "rope_theta": 10000.0,
        "compress_rope_theta": 160000.0,
        "rope_scaling": {"factor": 16.0, "beta_fast": 32.0, "beta_slow": 1.0,
                         "original_max_position_embeddings": 65536, "type": "yarn"},
        "index_n_heads": c.get("index_heads", 64), "index_head_dim": c.get("index_dim", 128),
        "index_topk": c.get("index_topk", 512),
        "compress_ratios": ratios(c, n_layers),
    }


def ratios(c, n_layers):
    r = list(c.get("ratios", []))[:n_layers]
    return r + [0] * (n_layers - len(r))


def tensor_specs(c, n_layers):
    """(name, dtype, shape, kind) of every tensor, in file order."""
    H, V, nh, hd, ql = c["hidden"], c["vocab"], c["heads"], c["head_dim"], c["q_lora"]
    G, ol, E, I, m = c["o_groups"], c["o_lora"], c["experts"], c["inter"], c["hc"]
    mix = (2 + m) * m
    sp = [("embed.weight", "BF16", [V, H], "w"), ("head.weight", "BF16", [V, H], "w"),
          ("norm.weight", "BF16", [H], "norm"), ("hc_head_fn", "F32", [m, m * H], "w"),
          ("hc_head_base", "F32", [m], "w"), ("hc_head_scale", "F32", [1], "one")]

    def fp8(name, r, k):
        sp.append((name + ".weight", "F8_E4M3", [r, k], "fp8"))
        sp.append((name + ".scale", "F8_E8M0", [(r + 127) // 128, (k + 127) // 128], "e8m0"))

    for L in range(n_layers):
        p = f"layers.{L}."
        sp += [(p + "attn_norm.weight", "BF16", [H], "norm"),
               (p + "ffn_norm.weight", "BF16", [H], "norm"),
               (p + "hc_attn_fn", "F32", [mix, m * H], "w"),
               (p + "hc_ffn_fn", "F32", [mix, m * H], "w"),
               (p + "hc_attn_scale", "F32", [3], "one"), (p + "hc_ffn_scale", "F32", [3], "one"),
               (p + "hc_attn_base", "F32", [mix], "w"), (p + "hc_ffn_base", "F32", [mix], "w"),
               (p + "attn.attn_sink", "F32", [nh], "w")]
        fp8(p + "attn.wq_a", ql, H)
        sp.append((p + "attn.q_norm.weight", "BF16", [ql], "norm"))
        fp8(p + "attn.wq_b", nh * hd, ql)
        fp8(p + "attn.wkv", hd, H)
        sp.append((p + "attn.kv_norm.weight", "BF16", [hd], "norm"))
        fp8(p + "attn.wo_a", G * ol, nh * hd // G)
        fp8(p + "attn.wo_b", H, G * ol)
        ratio = ratios(c, n_layers)[L]
        if ratio:
            coff = 2 if ratio == 4 else 1
            cp = p + "attn.compressor."
            sp += [(cp + "ape", "F32", [ratio, coff * hd], "w"),
                   (cp + "wkv.weight", "BF16", [coff * hd, H], "w"),
                   (cp + "wgate.weight", "BF16", [coff * hd, H], "w"),
                   (cp + "norm.weight", "BF16", [hd], "norm")]
            if ratio == 4:
                ih, idim = c.get("index_heads", 64), c.get("index_dim", 128)
                ip = p + "attn.indexer."
                fp8(ip + "wq_b", ih * idim, ql)
                sp += [(ip + "weights_proj.weight", "BF16", [ih, H], "w"),
                       (ip + "compressor.ape", "F32", [ratio, coff * idim], "w"),
                       (ip + "compressor.wkv.weight", "BF16", [coff * idim, H], "w"),
                       (ip + "compressor.wgate.weight", "BF16", [coff * idim, H], "w"),
                       (ip + "compressor.norm.weight", "BF16", [idim], "norm")]
        sp += [(p + "ffn.gate.weight", "BF16", [E, H], "w"), (p + "ffn.gate.bias", "F32", [E], "w")]
        fp8(p + "ffn.shared_experts.w1", I, H)
        fp8(p + "ffn.shared_experts.w3", I, H)
        fp8(p + "ffn.shared_experts.w2", H, I)
        for e in range(E):
            q = f"{p}ffn.experts.{e}."
            sp += [(q + "w1.scale", "F8_E8M0", [I, H // 32], "e8m0"),
                   (q + "w2.scale", "F8_E8M0", [H, I // 32], "e8m0"),
                   (q + "w3.scale", "F8_E8M0", [I, H // 32], "e8m0"),
                   (q + "w1.weight", "I8", [I, H // 2], "u8"),
                   (q + "w2.weight", "I8", [H, I // 2], "u8"),
                   (q + "w3.weight", "I8", [I, H // 2], "u8")]
    return sp


SIZE = {"F32": 4, "BF16": 2, "F8_E4M3": 1, "F8_E8M0": 1, "I8": 1}


def _values(rng, dt, shape, kind):
    n = int(np.prod(shape))
    if kind == "one":
        return np.ones(n, np.float32).tobytes()
    if kind == "u8":
        return rng.integers(0, 256, size=n, dtype=np.uint8).tobytes()
    if kind == "fp8":
        c = rng.integers(0, 254, size=n, dtype=np.uint8)
        return np.where((c & 0x7F) == 0x7F, c - 1, c).astype(np.uint8).tobytes()
    if kind == "e8m0":
        z = rng.standard_normal(n, dtype=np.float32) * np.float32(0.5 / np.log(2.0))
        return np.clip(127 + np.rint(z), 0, 254).astype(np.uint8).tobytes()
    v = rng.standard_normal(n, dtype=np.float32) * np.float32(0.02)
    if kind == "norm":
        v += np.float32(1.0)
    if dt == "F32":
        return v.tobytes()
    u = v.view(np.uint32)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16).tobytes()


def write(outdir, n_layers, c=CONFIG5, seed=0):
    """Writes config.json + model-00001-of-00001.safetensors; returns outdir."""
    os.makedirs(outdir, exist_ok=True)
    specs = tensor_specs(c, n_layers)
    header, off = {}, 0
    for name, dt, shape, _ in specs:
        nb = int(np.prod(shape)) * SIZE[dt]
        header[name] = {"dtype": dt, "shape": shape, "data_offsets": [off, off + nb]}
        off += nb
    hdr = json.dumps(header, separators=(",", ":")).encode()
    hdr += b" " * (-(len(hdr) + 8) % 8)
    rng = np.random.default_rng(seed)
    with open(os.path.join(outdir, "model-00001-of-00001.safetensors"), "wb") as f:
        f.write(struct.pack("<Q", len(hdr)))
        f.write(hdr)
        for name, dt, shape, kind in specs:
            f.write(_values(rng, dt, shape, kind))
    with open(os.path.join(outdir, "config.json"), "w") as f:
        json.dump(config_json(c, n_layers), f, indent=2)
    return outdir
