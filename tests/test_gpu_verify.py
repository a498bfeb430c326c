"""Batched speculative verify on the GPU (tree and chain), composed from the
library's pieces: verify-row latents in scratch rows of the FP8 cache,
dsv4cuda_tree_attn_indices + dsv4cuda_sparse_attn for all rows at once,
dsv4cuda_accept_device on the rows' logits, and dsv4cuda_kv_copy_rows to
commit the accepted path into the ring.

Checked against (a) the oracle's sparse_attn on each node's visible keys and
(b) sequential decoding of the same positions (write the row into its ring
slot, attend with window_topk's indices, src/dsv4/dsv4_model.c:5073): the
attention outputs agree within the attention tolerance, and after the
commit the ring holds exactly what sequential decoding of the accepted
tokens leaves there."""
import numpy as np
import pytest
import torch

from test_gpu_attn import attn_magnitude, bf16_vals, qat_rows, rowwise_check

pytestmark = pytest.mark.gpu
D, H, WIN = 512, 128, 128


def window_topk(pos, win):
    if pos >= win - 1:
        s = pos % win
        return [(s + 1 + i) % win for i in range(win)]
    return list(range(pos + 1))


def attend(cuda, cache, q, idx, rows_total):
    B = q.shape[0]
    shape = cuda.attn_shape(B, H, D, idx.shape[1], D ** -0.5, 64, 0, rows_total)
    out = torch.empty((B, H, D), dtype=torch.float32, device="cuda")
    sink = torch.linspace(-1, 1, H, device="cuda")
    cuda.sparse_attn(out, torch.from_numpy(q).cuda(), sink,
                     torch.from_numpy(np.ascontiguousarray(idx, np.int32)).cuda(), shape,
                     cache=cache)
    torch.cuda.synchronize()
    return out.cpu().numpy(), sink.cpu().numpy()


def cache_rows(cuda, cache, rows):
    out = torch.empty((len(rows), D), dtype=torch.float32, device="cuda")
    cache.read(torch.tensor(rows, dtype=torch.int64, device="cuda"), out)
    torch.cuda.synchronize()
    return out.cpu().numpy()


def test_tree_verify_attention_matches_oracle(cuda, orc):
    rng = np.random.default_rng(1)
    parents = [-1, 0, 0, 1, 1, 2, 2]          # 2-ary tree, 7 nodes
    committed, scratch = 300, WIN
    rows_total = WIN + len(parents)
    cache = cuda.LatentCache(rows_total)
    cache.write(torch.from_numpy(bf16_vals(rng, (rows_total, D))).cuda(),
                torch.arange(rows_total, dtype=torch.int64, device="cuda"))
    idx = cuda.tree_attn_indices(parents, committed, WIN, 0, scratch, WIN + 8)
    q = bf16_vals(rng, (len(parents), H, D))
    got, sink = attend(cuda, cache, q, idx, rows_total)
    kv = cache_rows(cuda, cache, list(range(rows_total)))
    for j in range(len(parents)):
        want = orc.sparse_attn(q[j], kv, sink, idx[j], D ** -0.5)
        rowwise_check(got[j], want, attn_magnitude(q[j], kv, sink, idx[j], D ** -0.5))


@pytest.mark.parametrize("committed,n_match", [(140, 3), (60, 5), (200, 0)])
def test_chain_verify_step_equals_sequential_decode(cuda, orc, committed, n_match):
    rng = np.random.default_rng(committed)
    P = 5                                      # drafts; rows = pending + drafts
    R = P + 1
    rows_total = WIN + R
    V = 4096
    lat = qat_rows(orc, bf16_vals(rng, (R, D)))  # the verify rows' latents (exact cache values)
    q = bf16_vals(rng, (R, H, D))
    history = bf16_vals(rng, (WIN, D))
    ring0 = torch.from_numpy(history).cuda()

    # ---- batched verify: latents in scratch rows, one attention launch
    cache = cuda.LatentCache(rows_total)
    cache.write(ring0, torch.arange(WIN, dtype=torch.int64, device="cuda"))
    cache.write(torch.from_numpy(lat).cuda(),
                torch.arange(WIN, WIN + R, dtype=torch.int64, device="cuda"))
    parents = [-1] + list(range(P))
    idx = cuda.tree_attn_indices(parents, committed, WIN, 0, WIN, WIN + R + 1)
    got, sink = attend(cuda, cache, q, idx, rows_total)

    # ---- sequential decode of the same positions
    seq = cuda.LatentCache(rows_total)
    seq.write(ring0, torch.arange(WIN, dtype=torch.int64, device="cuda"))
    for t in range(R):
        pos = committed + t
        seq.write(torch.from_numpy(lat[t:t + 1]).cuda(),
                  torch.tensor([pos % WIN], dtype=torch.int64, device="cuda"))
        want, _ = attend(cuda, seq, q[t:t + 1], np.array([window_topk(pos, WIN)]), rows_total)
        kv = cache_rows(cuda, seq, list(range(WIN)))
        rowwise_check(got[t], want[0],
                      attn_magnitude(q[t], kv, sink, np.array(window_topk(pos, WIN)), D ** -0.5))

    # ---- acceptance on the device: drafts agree with the greedy target for n_match rows
    logits = rng.normal(size=(R, V)).astype(np.float32)
    prop = logits.argmax(axis=1)[:P].astype(np.int32)
    if n_match < P:
        prop[n_match] = (prop[n_match] + 1) % V
    res = torch.zeros(2 * P + 6, dtype=torch.int32, device="cuda")
    cuda.accept_device(torch.from_numpy(prop).cuda(), torch.from_numpy(logits).cuda(), 0.0, None,
                       res, eos_id=-7)
    torch.cuda.synchronize()
    r = res.cpu().numpy()
    n_commit = int(r[1])
    assert n_commit == min(n_match, P) + 1
    # commit: the accepted rows move from scratch into their ring slots
    cuda.kv_copy_rows(cache, [WIN + t for t in range(n_commit)],
                      [(committed + t) % WIN for t in range(n_commit)])
    # sequential decode keeps only the committed positions: rebuild its ring
    ref = cuda.LatentCache(rows_total)
    ref.write(ring0, torch.arange(WIN, dtype=torch.int64, device="cuda"))
    ref.write(torch.from_numpy(lat[:n_commit]).cuda(),
              torch.tensor([(committed + t) % WIN for t in range(n_commit)], dtype=torch.int64,
                           device="cuda"))
    torch.cuda.synchronize()
    for a, b in ((cache.codes, ref.codes), (cache.scales, ref.scales), (cache.rope, ref.rope)):
        assert torch.equal(a[:WIN], b[:WIN])
