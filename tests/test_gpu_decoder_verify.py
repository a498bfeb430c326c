"""The batched speculative verify on the device decoder (dsv4cuda_decoder_
verify*) against the reference engine's dsv4_prefill_capture with all_logits
(src/dsv4/dsv4_model.c:8434-8529) on the same checkpoint.

The reference side is oracle/_ref/tiny_verify: it prefills the prompt with
dsv4_prefill, then runs the verify rows through one dsv4_prefill_capture
call (layer-major, every row's logits). The device prefills token by token
(dsv4cuda_decoder_forward_token), then runs the same rows through one
dsv4cuda_decoder_verify call: every GEMV over all rows at once, each row's
latent in a scratch row beside the ring, each row attending to the window
of its own position.

Exact mode (hc_exact = 1): every row's logits bit-identical to the
reference's. Fast mode (the benchmark's): within 2e-2 relative L2 per row,
as the single-token decoder (its HC mixes are summed in double).
The commit and the device acceptance are checked against plain token-by-
token decoding of the accepted tokens: ring bytes and continuation logits
bit-identical.
"""
import os
import subprocess
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REFDIR = os.path.join(ROOT, "oracle", "_ref")
sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))

pytestmark = pytest.mark.gpu
FAST_REL_L2 = 2e-2


def t1_window_checkpoint(tmp_path, seed):
    import make_tiny_t1
    cfg = dict(make_tiny_t1.CFG, ratios=[0, 0], head_dim=80)
    return cfg, make_tiny_t1.write(str(tmp_path / f"t1v{seed}"), seed=seed, c=cfg)


def reference_verify(ckpt, ids, start, n_rows):
    exe = os.path.join(REFDIR, "tiny_verify")
    if not os.path.exists(exe):
        pytest.skip("oracle/_ref/tiny_verify not built here (needs the reference sources)")
    env = dict(os.environ)
    env.pop("LD_PRELOAD", None)
    env["TINY_DECODE_THREADS"] = str(max(2, min(16, os.cpu_count() or 2)))
    r = subprocess.run([exe, ckpt, str(start), str(n_rows), *map(str, ids[:start + n_rows])],
                       cwd=REFDIR, env=env, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stderr[-2000:]
    rows = [np.array([float.fromhex(v) for v in ln.split()[5:]], np.float32)
            for ln in r.stdout.splitlines() if ln.startswith("ROW")]
    assert len(rows) == n_rows
    return np.stack(rows)


def first_argmax(v):
    return int(np.argmax(v))  # numpy returns the first maximum, as argmax_logits does


def check_rows(got, am, want, exact):
    worst = 0.0
    for r in range(len(want)):
        err = float(np.linalg.norm(got[r].astype(np.float64) - want[r]) /
                    (np.linalg.norm(want[r].astype(np.float64)) + 1e-30))
        worst = max(worst, err)
        if exact:
            assert np.array_equal(got[r].view(np.uint32), want[r].view(np.uint32)), (r, err)
        else:
            assert err <= FAST_REL_L2, (r, err)
        assert am[r] == first_argmax(got[r]), r
    return worst


@pytest.mark.parametrize("exact", [True, False], ids=["exact", "fast"])
def test_verify_t1_vs_prefill_capture(cuda, tmp_path, exact):
    """T1 (window 16): a 40-token prompt, so the ring has wrapped, then a
    chain of 6 rows and, at the same start, the maximum of 8 rows (a verify
    leaves the ring untouched, so the second call sees the same context)."""
    cfg, ckpt = t1_window_checkpoint(tmp_path, 0)
    import make_tiny_t1
    ids = make_tiny_t1.prompt_ids(seed=0, n=48)
    start = 40
    dec = cuda.decoder_from_checkpoint(ckpt, max_context=64, hc_exact=exact)
    try:
        for p in range(start):
            dec.forward_token(ids[p], p)
        for n_rows in (6, cuda.Decoder.VERIFY_MAX_ROWS):
            want = reference_verify(ckpt, ids, start, n_rows)
            got, am = dec.verify(ids[start:start + n_rows], start)
            worst = check_rows(got, am, want, exact)
            print(f"verify T1 {n_rows} rows ({'exact' if exact else 'fast'}): "
                  f"worst rel L2 {worst:.2e}")
    finally:
        dec.close()


def test_verify_c5_layer_vs_prefill_capture(cuda, tmp_path):
    """One layer at the benchmark's DeepSeek-V4-Flash shapes (hidden 4096,
    64 heads x 512, q_lora 1024, 8 x 1024 wo_a groups, window 128; 16
    experts and a 2048-token vocabulary for a quick host reference) after a
    136-token prompt: the multi-token FP8 streaming GEMVs, the multi-row
    grouped wo_a and the MoE layer at 6 tokens. Exact mode, bit-identical."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import random_checkpoint
    c = dict(random_checkpoint.CONFIG5, vocab=2048, experts=16)
    ckpt = random_checkpoint.write(str(tmp_path / "c5v"), 1, c=c, seed=4)
    ids = [int(v) for v in np.random.default_rng(4).integers(0, c["vocab"], 142)]
    start, n_rows = 136, 6
    want = reference_verify(ckpt, ids, start, n_rows)
    dec = cuda.decoder_from_checkpoint(ckpt, max_context=len(ids) + 8, hc_exact=True)
    try:
        for p in range(start):
            dec.forward_token(ids[p], p)
        got, am = dec.verify(ids[start:start + n_rows], start)
        check_rows(got, am, want, exact=True)
    finally:
        dec.close()


def ring_bytes(cuda, dec, n_layers, window, head_dim):
    import torch
    rows = torch.arange(window, dtype=torch.int64, device="cuda")
    out = []
    for li in range(n_layers):
        r = torch.empty((window, head_dim), device="cuda")
        cuda.lib.dsv4cuda_kv_read(cuda.C.byref(dec.cache(li)), rows.data_ptr(), window,
                                  r.data_ptr(), 0)
        torch.cuda.synchronize()
        out.append(r.view(torch.int32).cpu().numpy())
    return out


def test_verify_commit_prefix_equals_plain_decode(cuda, tmp_path):
    """A verify of six rows whose first two are the true continuation, at
    positions that cross the ring's wrap, then commit(2): the ring must equal,
    byte for byte, a decoder that only ever saw the accepted tokens, and the
    continuation logits must be bit-identical (the reference's commit-prefix
    gate, tests/unit/test_dsv4_model.c:342-388, on the verify path)."""
    cfg, ckpt = t1_window_checkpoint(tmp_path, 2)
    import make_tiny_t1
    ids = make_tiny_t1.prompt_ids(seed=2, n=40)
    P, W = 30, cfg["window"]
    rows = [ids[P], ids[P + 1]] + [(t * 7 + 3) % cfg["vocab"] for t in ids[P + 2:P + 6]]
    a = cuda.decoder_from_checkpoint(ckpt, max_context=64)
    b = cuda.decoder_from_checkpoint(ckpt, max_context=64)
    try:
        for p in range(P):
            a.forward_token(ids[p], p)
            b.forward_token(ids[p], p)
        b.verify(rows, P)
        b.commit(2)
        for p in (P, P + 1):
            a.forward_token(ids[p], p)
        ra = ring_bytes(cuda, a, cfg["layers"], W, cfg["head_dim"])
        rb = ring_bytes(cuda, b, cfg["layers"], W, cfg["head_dim"])
        for li in range(cfg["layers"]):
            assert np.array_equal(ra[li], rb[li]), li
        for p in range(P + 2, P + 6):
            la, na = a.forward_token(ids[p], p)
            lb, nb = b.forward_token(ids[p], p)
            assert np.array_equal(la.view(np.uint32), lb.view(np.uint32)), p
            assert na == nb
    finally:
        a.close()
        b.close()


def test_accept_greedy_device_chain(cuda, tmp_path):
    """The device speculative loop (verify -> accept_greedy, which commits
    and sets up the next step on the device): drafts that are the true
    greedy continuation are all accepted (6 tokens from one step); then
    random drafts (draft_random) are rejected and each step yields its
    bonus token. The pending token and start the loop leaves must follow
    plain greedy decoding, and the ring must equal the plain decoder's,
    byte for byte."""
    cfg, ckpt = t1_window_checkpoint(tmp_path, 3)
    import make_tiny_t1
    ids = make_tiny_t1.prompt_ids(seed=3, n=24)
    P, n_rows, W = 24, 6, cfg["window"]
    a = cuda.decoder_from_checkpoint(ckpt, max_context=96)
    b = cuda.decoder_from_checkpoint(ckpt, max_context=96)
    try:
        for p in range(P):
            a.forward_token(ids[p], p)
            _, pend = b.forward_token(ids[p], p)
        greedy = [pend]  # greedy[i] is the token at position P + i
        _, nxt = a.read()
        assert nxt == pend
        for i in range(24):
            _, nxt = a.forward_token(greedy[-1], P + i)
            greedy.append(nxt)
        b.verify(greedy[:n_rows], P)  # host form: also fills the device slots
        b.accept_greedy(n_rows)
        assert b.verify_stats() == (n_rows, n_rows - 1, 1)
        assert b.verify_pending() == (greedy[n_rows], P + n_rows)
        for _ in range(3):
            b.draft_random(n_rows)
            b.verify_device(n_rows)
            b.accept_greedy(n_rows)
        tokens, accepted, steps = b.verify_stats()
        assert steps == 4 and tokens == n_rows + 3 + (accepted - (n_rows - 1))
        assert b.verify_pending() == (greedy[tokens], P + tokens)
        a2 = cuda.decoder_from_checkpoint(ckpt, max_context=96)
        try:
            for p in range(P):
                a2.forward_token(ids[p], p)
            for i in range(tokens):
                a2.forward_token(greedy[i], P + i)
            ra = ring_bytes(cuda, a2, cfg["layers"], W, cfg["head_dim"])
            rb = ring_bytes(cuda, b, cfg["layers"], W, cfg["head_dim"])
            for li in range(cfg["layers"]):
                assert np.array_equal(ra[li], rb[li]), li
        finally:
            a2.close()
    finally:
        a.close()
        b.close()
