"""The speculative transaction on the latent KV ring (dsv4cuda_snapshot_*)
against a restatement of the reference's semantics
(dsv4_context_snapshot_take / _commit_prefix / _restore,
src/dsv4/dsv4_model.c:2842-3056): commit restores every saved slot and then
re-applies the first k verified positions' rows; restore puts every saved
slot back. Byte-exact on the cache and the state buffers."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
D = 512


def bf16_rows(rng, n):
    x = rng.normal(size=(n, D)).astype(np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    return (((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16).astype(np.uint32).view(np.float32)


def cache_bytes(cache):
    torch.cuda.synchronize()
    return (cache.codes.cpu().numpy().copy(), cache.scales.cpu().numpy().copy(),
            cache.rope.cpu().numpy().copy())


def reference_commit(before, after, slots, k):
    """Reference semantics on numpy copies of the ring: undo all saved
    slots, then redo positions < k with their post-verify rows."""
    out = tuple(a.copy() for a in after)
    for arr_b, arr_o in zip(before, out):
        for sl in slots:
            arr_o[sl] = arr_b[sl]
    for p in range(k):
        for arr_a, arr_o in zip(after, out):
            arr_o[slots[p]] = arr_a[slots[p]]
    return out


@pytest.mark.parametrize("start,n,k", [(5, 6, 3), (125, 6, 2), (126, 5, 5), (0, 1, 1),
                                       (120, 16, 9)])
def test_commit_prefix_and_restore(cuda, start, n, k):
    rng = np.random.default_rng(start + n)
    win, base = 128, 40
    rows = base + win + 8
    cache = cuda.LatentCache(rows)
    all_rows = torch.arange(rows, dtype=torch.int64, device="cuda")
    cache.write(torch.from_numpy(bf16_rows(rng, rows)).cuda(), all_rows)
    state = torch.from_numpy(rng.normal(size=300).astype(np.float32)).cuda()
    snap = cuda.Snapshot([cache], [win], ring_base=[base], states=[state], max_positions=16)
    slots = [base + (start + p) % win for p in range(n)]
    for mode in ("commit", "restore"):
        before = cache_bytes(cache)
        s0 = state.cpu().numpy().copy()
        snap.take(start, n)
        posts = []
        for p in range(n):  # the verify step writes its rows and updates the state
            cache.write(torch.from_numpy(bf16_rows(rng, 1)).cuda(),
                        torch.tensor([slots[p]], dtype=torch.int64, device="cuda"))
            state.add_(1.0 + p)
            snap.capture_state(p)
            posts.append(state.cpu().numpy().copy())
        after = cache_bytes(cache)
        if mode == "commit":
            snap.commit_prefix(k)
            want = reference_commit(before, after, slots, k)
            want_state = posts[k - 1]
        else:
            snap.restore()
            want = before
            want_state = s0
        got = cache_bytes(cache)
        for g, w in zip(got, want):
            assert np.array_equal(g, w)
        assert np.array_equal(state.cpu().numpy(), want_state)
    snap.close()


def test_commit_needs_captured_state(cuda):
    cache = cuda.LatentCache(200)
    state = torch.zeros(10, device="cuda")
    snap = cuda.Snapshot([cache], [128], states=[state], max_positions=8)
    snap.take(0, 4)
    with pytest.raises(cuda.Dsv4CudaError):
        snap.commit_prefix(2)
    snap.restore()
    snap.close()
