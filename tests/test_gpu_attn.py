"""GPU parity of the latent KV cache and the decode attention
(dsv4cuda_kv_write / dsv4cuda_sparse_attn) against the CPU oracle of
sparse_attn (src/dsv4/dsv4_model.c:5767-5822), dsv4_act_quant_inplace
(:1386) and dsv4_rope_apply_buf_inv (:1569).

Bar: the cache is bit-exact (it stores exactly the values the reference
keeps in its fp32 kv_cache). Attention outputs agree with the reference to a
relative tolerance TOL = 1e-2 of each element's accumulation magnitude
A_i = sum_t p_t |v_t,i| (p = the exact softmax including the sink), i.e.
|got_i - want_i| <= TOL * max(|want_i|, A_i), and the relative L2 error of
every (query, head) row is <= TOL. The reference rounds each weight
bf16(exp(s_t - m)) against the global max m, the GPU against the running max
of its key split, so the two results carry independent half-ulp BF16 weight
roundings (2^-9 relative each); their difference is bounded by about
2^-8 * A_i, which exceeds 1e-2 * |want_i| only where the value sum cancels."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
TOL = 1e-2
D, NOPE, ROPE = 512, 448, 64


def bf16_vals(rng, shape, scale=1.0):
    x = (rng.normal(size=shape) * scale).astype(np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    return (((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16).astype(np.uint32).view(np.float32)


def qat_rows(orc, raw):
    """Reference cache rows: act_quant(group 64, mode 0) on the non-RoPE dims."""
    out = raw.copy()
    for r in range(raw.shape[0]):
        out[r, :NOPE] = orc.act_quant_inplace(raw[r, :NOPE], 64, 0)
    return out


def attn_magnitude(q, kv, sink, idx, scale):
    """A [H][d] = sum_t p_t |kv_t| with p the exact (fp64) softmax incl. the sink."""
    idx = np.asarray(idx)
    valid = idx >= 0
    k = kv[idx[valid]].astype(np.float64)
    s = (q.astype(np.float64) @ k.T) * scale
    m = np.maximum(s.max(axis=1) if k.shape[0] else -np.inf, sink.astype(np.float64))
    e = np.exp(s - m[:, None])
    den = e.sum(axis=1) + np.exp(sink - m)
    return (e / den[:, None]) @ np.abs(k)


def rope_magnitude(A, cos, sin):
    """Magnitude of the inverse-RoPE output pairs (|c| A0 + |s| A1, |s| A0 + |c| A1)."""
    A = A.copy()
    n = cos.size
    a0, a1 = A[:, -2 * n::2].copy(), A[:, -2 * n + 1::2].copy()
    c, s = np.abs(cos.astype(np.float64)), np.abs(sin.astype(np.float64))
    A[:, -2 * n::2] = c * a0 + s * a1
    A[:, -2 * n + 1::2] = s * a0 + c * a1
    return A


def rowwise_check(got, want, mag=None, tol=TOL):
    """|got - want| <= tol * max(|want|, mag) elementwise and relative L2 error
    <= tol per (query, head) row; returns (worst element ratio, exact fraction)."""
    d = want.shape[-1]
    got = got.reshape(-1, d).astype(np.float64)
    want = want.reshape(-1, d).astype(np.float64)
    mag = np.abs(want) if mag is None else np.maximum(np.abs(want), mag.reshape(-1, d))
    diff = np.abs(got - want)
    zero = mag == 0.0
    assert np.all(diff[zero] == 0.0)
    ratio = float(np.max(diff[~zero] / mag[~zero])) if np.any(~zero) else 0.0
    norms = np.linalg.norm(want, axis=1)
    l2 = np.linalg.norm(got - want, axis=1)
    rel = float(np.max(l2[norms > 0] / norms[norms > 0])) if np.any(norms > 0) else 0.0
    exact = float(np.mean(got == want))
    assert ratio <= tol and rel <= tol, (ratio, rel, exact)
    assert np.all(l2[norms == 0] == 0.0)
    return ratio, exact


def dev(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t if dtype is None else t.to(dtype)


def test_kv_cache_exact(cuda, orc):
    rng = np.random.default_rng(0)
    n = 64
    raw = bf16_vals(rng, (n, D))
    raw[1] = 0.0
    raw[2, :64] *= 1e-7          # below the 1e-4 amax floor
    raw[3, 64:128] *= 1e5
    raw[4, :NOPE:7] = 0.0
    cache = cuda.LatentCache(rows=100)
    rows = np.arange(n, dtype=np.int64) * 3 % 100
    cache.write(dev(raw), dev(rows))
    back = torch.empty((n, D), dtype=torch.float32, device="cuda")
    cache.read(dev(rows), back)
    torch.cuda.synchronize()
    want = qat_rows(orc, raw)
    assert np.array_equal(back.cpu().numpy().view(np.uint32), want.view(np.uint32))


def run_attn(cuda, q, sink, idx, scale, kv=None, cache=None, kv_rows=0, stride=0, cos=None,
             sin=None, H=None):
    B, H, d = q.shape
    n = idx.shape[1]
    shape = cuda.attn_shape(B, H, d, n, scale, ROPE if d == D else 16, stride, kv_rows)
    out = torch.empty((B, H, d), dtype=torch.float32, device="cuda")
    cuda.sparse_attn(out, dev(q), dev(sink), dev(idx.astype(np.int32)), shape,
                     kv=None if kv is None else dev(kv), cache=cache,
                     rope_cos=None if cos is None else dev(cos),
                     rope_sin=None if sin is None else dev(sin))
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("H,n,scale", [
    (128, 1, D ** -0.5), (128, 32, D ** -0.5), (128, 33, D ** -0.5), (128, 257, D ** -0.5),
    (64, 200, D ** -0.5), (128, 300, 0.25), (7, 70, D ** -0.5)])
def test_attn_tensor_core_fp32_rows(cuda, orc, H, n, scale):
    rng = np.random.default_rng(H * 1000 + n)
    rows = n + 5
    kv = qat_rows(orc, bf16_vals(rng, (rows, D)))
    q = bf16_vals(rng, (1, H, D))
    sink = rng.normal(size=H).astype(np.float32)
    idx = rng.permutation(rows)[:n].astype(np.int32)[None, :]
    if n > 8:
        idx[0, 3::7] = -1
    got = run_attn(cuda, q, sink, idx, scale, kv=kv, kv_rows=rows)
    want = orc.sparse_attn(q[0], kv, sink, idx[0], scale)
    rowwise_check(got[0], want, attn_magnitude(q[0], kv, sink, idx[0], scale))


def test_attn_tensor_core_fp8_cache_batched_rope(cuda, orc):
    """Batch of 3 queries, each with its own cache region, FP8 cache source,
    inverse RoPE fused."""
    rng = np.random.default_rng(11)
    B, H, n, per = 3, 128, 150, 160
    raw = bf16_vals(rng, (B * per, D))
    cache = cuda.LatentCache(rows=B * per)
    rows = np.arange(B * per, dtype=np.int64)
    cache.write(dev(raw), dev(rows))
    kv = qat_rows(orc, raw)
    q = bf16_vals(rng, (B, H, D))
    sink = rng.normal(size=H).astype(np.float32)
    idx = np.stack([rng.permutation(per)[:n] for _ in range(B)]).astype(np.int32)
    idx[1, ::4] = -1
    ang = rng.uniform(0, 6.3, size=(B, ROPE // 2)).astype(np.float32)
    cos, sin = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    got = run_attn(cuda, q, sink, idx, D ** -0.5, cache=cache, kv_rows=per, stride=per,
                   cos=cos, sin=sin)
    for b in range(B):
        kb = kv[b * per:(b + 1) * per]
        o = orc.sparse_attn(q[b], kb, sink, idx[b], D ** -0.5)
        want = orc.rope_inv(o, cos[b], sin[b])
        mag = rope_magnitude(attn_magnitude(q[b], kb, sink, idx[b], D ** -0.5), cos[b], sin[b])
        rowwise_check(got[b], want, mag)


def test_attn_fp8_cache_subnormal_codes(cuda, orc):
    """Groups whose small members quantise to E4M3 subnormal codes (one large
    value per group of 64 sets the scale): the tile conversion must keep
    them exactly. Few keys, so a lost subnormal changes an output element by
    its whole value."""
    rng = np.random.default_rng(21)
    H, n = 128, 3
    raw = bf16_vals(rng, (n, D), scale=0.004)
    raw[:, :NOPE:64] = 400.0                         # scale 2^0: |x| < 2^-6 -> subnormal
    raw[1, 1:NOPE:64] = -2.0 ** -9                   # the smallest subnormal
    raw = (raw.view(np.uint32) & 0xFFFF0000).view(np.float32)
    cache = cuda.LatentCache(rows=n)
    cache.write(dev(raw), dev(np.arange(n, dtype=np.int64)))
    kv = qat_rows(orc, raw)
    tiny = np.abs(kv[:, :NOPE]) < 2.0 ** -6
    assert np.count_nonzero(tiny & (kv[:, :NOPE] != 0)) > 100
    q = bf16_vals(rng, (1, H, D), scale=0.01)
    sink = np.full(H, -3.0, np.float32)
    idx = np.arange(n, dtype=np.int32)[None, :]
    got = run_attn(cuda, q, sink, idx, D ** -0.5, cache=cache, kv_rows=n)
    want = orc.sparse_attn(q[0], kv, sink, idx[0], D ** -0.5)
    rowwise_check(got[0], want, attn_magnitude(q[0], kv, sink, idx[0], D ** -0.5))


def test_attn_rescale_path(cuda, orc):
    """Key norms grow along the index order so the running max rises on
    almost every tile (exercises the O rescale in TMEM)."""
    rng = np.random.default_rng(5)
    H, n = 128, 512
    raw = bf16_vals(rng, (n, D)) * np.linspace(0.5, 3.0, n, dtype=np.float32)[:, None]
    raw = (raw.view(np.uint32) & 0xFFFF0000).view(np.float32)  # back on the BF16 grid
    kv = qat_rows(orc, raw)
    q = bf16_vals(rng, (1, H, D))
    sink = np.full(H, -5.0, np.float32)
    idx = np.arange(n, dtype=np.int32)[None, :]
    got = run_attn(cuda, q, sink, idx, 0.15, kv=kv, kv_rows=n)
    want = orc.sparse_attn(q[0], kv, sink, idx[0], 0.15)
    rowwise_check(got[0], want, attn_magnitude(q[0], kv, sink, idx[0], 0.15))


def test_attn_edges(cuda, orc):
    rng = np.random.default_rng(9)
    H = 128
    kv = qat_rows(orc, bf16_vals(rng, (40, D)))
    q = bf16_vals(rng, (2, H, D))
    sink = rng.normal(size=H).astype(np.float32)
    # no keys at all
    got = run_attn(cuda, q[:1], sink, np.zeros((1, 0), np.int32), D ** -0.5, kv=kv, kv_rows=40)
    assert np.all(got == 0.0)
    # every index is padding
    idx = -np.ones((2, 45), np.int32)
    got = run_attn(cuda, q, sink, idx, D ** -0.5, kv=kv, kv_rows=40)
    want = orc.sparse_attn(q[0], kv, sink, idx[0], D ** -0.5)
    assert np.all(got == 0.0) and np.all(want == 0.0)


def test_attn_index_out_of_range_is_reported(cuda, orc):
    rng = np.random.default_rng(10)
    H = 128
    kv = qat_rows(orc, bf16_vals(rng, (40, D)))
    q = bf16_vals(rng, (1, H, D))
    sink = rng.normal(size=H).astype(np.float32)
    idx = np.arange(40, dtype=np.int32)[None, :].copy()
    idx[0, 5] = 1000  # beyond kv_rows: skipped and flagged
    got = run_attn(cuda, q, sink, idx, D ** -0.5, kv=kv, kv_rows=40)
    flags = cuda.device_error(clear=True)
    assert flags & 4
    idx2 = idx.copy()
    idx2[0, 5] = -1
    want = orc.sparse_attn(q[0], kv, sink, idx2[0], D ** -0.5)
    rowwise_check(got[0], want, attn_magnitude(q[0], kv, sink, idx2[0], D ** -0.5))


@pytest.mark.parametrize("H,d,n", [(4, 32, 48), (4, 32, 1), (16, 128, 300)])
def test_attn_simt_general_shapes(cuda, orc, H, d, n):
    """Shapes outside the tensor-core tile (the tiny model: 4 heads x 32)."""
    rng = np.random.default_rng(d + n)
    rows = n + 2
    kv = bf16_vals(rng, (rows, d))
    q = bf16_vals(rng, (1, H, d))
    sink = rng.normal(size=H).astype(np.float32)
    idx = rng.integers(-1, rows, size=(1, n)).astype(np.int32)
    ang = rng.uniform(0, 6.3, size=(1, 8)).astype(np.float32)
    cos, sin = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    got = run_attn(cuda, q, sink, idx, d ** -0.5, kv=kv, kv_rows=rows, cos=cos, sin=sin)
    want = orc.rope_inv(orc.sparse_attn(q[0], kv, sink, idx[0], d ** -0.5), cos[0], sin[0])
    mag = rope_magnitude(attn_magnitude(q[0], kv, sink, idx[0], d ** -0.5), cos[0], sin[0])
    rowwise_check(got[0], want, mag)


def test_attn_host_dropin_matches_reference(cuda, ref, orc):
    """dsv4cuda_sparse_attn_host takes the reference sparse_attn arguments."""
    rng = np.random.default_rng(12)
    H, n, rows = 128, 96, 128
    kv = qat_rows(orc, bf16_vals(rng, (rows, D)))
    q = bf16_vals(rng, (H, D))
    sink = rng.normal(size=H).astype(np.float32)
    idx = rng.permutation(rows)[:n].astype(np.int32)
    got = cuda.sparse_attn_host(q, kv, sink, idx, D ** -0.5)
    want = ref.sparse_attn(q, kv, sink, idx, D ** -0.5)
    rowwise_check(got, want, attn_magnitude(q, kv, sink, idx, D ** -0.5))


@pytest.mark.parametrize("B,ctx", [(1, 4096), (2, 32768)])
def test_attn_config3_shapes(cuda, orc, B, ctx):
    """Benchmark config 3 shapes through the FP8 cache: 128 heads x 512,
    positions 0..ctx-1; checked against the oracle on a subset of heads."""
    rng = np.random.default_rng(ctx + B)
    H = 128
    raw = bf16_vals(rng, (B * ctx, D))
    cache = cuda.LatentCache(rows=B * ctx)
    cache.write(dev(raw), torch.arange(B * ctx, dtype=torch.int64, device="cuda"))
    q = bf16_vals(rng, (B, H, D))
    sink = rng.normal(size=H).astype(np.float32)
    idx = np.tile(np.arange(ctx, dtype=np.int32), (B, 1))
    got = run_attn(cuda, q, sink, idx, D ** -0.5, cache=cache, kv_rows=ctx, stride=ctx)
    back = torch.empty((B * ctx, D), dtype=torch.float32, device="cuda")
    cache.read(torch.arange(B * ctx, dtype=torch.int64, device="cuda"), back)
    kv = back.cpu().numpy()
    heads = [0, 37, 127] if ctx > 4096 else list(range(0, H, 9))
    for b in range(B):
        kb = kv[b * ctx:(b + 1) * ctx]
        want = orc.sparse_attn(q[b, heads], kb, sink[heads], idx[b], D ** -0.5)
        rowwise_check(got[b, heads], want,
                      attn_magnitude(q[b, heads], kb, sink[heads], idx[b], D ** -0.5))
