"""Expert-parallel MoE layer on the GPU (dsv4cuda_moe_create_device_ep /
_forward_local / _routed_slots / _combine).

On one GPU the G devices are emulated by G layers with disjoint expert
ranges; their routed slots are summed (every slot has one non-zero
contributor) and combined, and the output must be bit-identical to the
single layer holding every expert. With two or more GPUs the same runs as
one process per GPU with an NCCL all-reduce."""
import datetime
import os
import socket

import numpy as np
import pytest
import torch

from oracle import make_moe_layer

pytestmark = pytest.mark.gpu
HID, MI, NE, TOPK = 1024, 512, 32, 6


def bf16_vals(rng, shape):
    x = rng.normal(size=shape).astype(np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    return (((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16).astype(np.uint32).view(np.float32)


def device_layer(L, lo=0, hi=None, dev="cuda"):
    hi = L["n_experts"] if hi is None else hi
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)  # noqa: E731
    d = {k: v for k, v in L.items() if not isinstance(v, (np.ndarray, dict))}
    d["gate_w"] = t(L["gate_w"])
    d["bias"] = None if L.get("bias") is None else t(L["bias"])
    d["tid2eid"] = None if L.get("tid2eid") is None else t(L["tid2eid"])
    for n in ("w1", "s1", "w3", "s3", "w2", "s2"):
        d[n] = t(L[n][lo:hi])
    sh = L.get("shared")
    d["shared"] = None if sh is None else {k: (t(v) if isinstance(v, np.ndarray) else v)
                                           for k, v in sh.items()}
    return d


@pytest.mark.parametrize("G,M,shared", [(2, 1, "fp8"), (4, 5, "fp8"), (8, 3, None),
                                        (3, 2, "fp4")])
def test_ep_emulated_matches_single_layer(cuda, G, M, shared):
    L = make_moe_layer(HID, MI, NE, TOPK, seed=G * 10 + M, shared=shared)
    full = cuda.MoeLayer(device_layer(L), max_tokens=8, device=True)
    x = torch.from_numpy(bf16_vals(np.random.default_rng(G), (M, HID))).cuda()
    want = torch.empty((M, HID), dtype=torch.float32, device="cuda")
    full.forward(x, want)
    parts, keep = [], []
    for g in range(G):
        lo, hi = g * NE // G, (g + 1) * NE // G
        d = device_layer(L, lo, hi)
        keep.append(d)
        parts.append(cuda.MoeLayer(d, max_tokens=8, device=True, expert_range=(lo, hi)))
    for p in parts:
        p.forward_local(x)
    total = torch.stack([p.routed_slots(M).clone() for p in parts]).sum(0)
    nonzero = torch.stack([(p.routed_slots(M) != 0).any(-1) for p in parts]).sum(0)
    assert int(nonzero.max()) <= 1  # each (token, k) slot is owned by one device
    parts[0].routed_slots(M).copy_(total)
    got = torch.empty_like(want)
    parts[0].combine(M, got)
    torch.cuda.synchronize()
    assert torch.equal(got.view(torch.int32), want.view(torch.int32))
    for p in parts + [full]:
        p.close()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_rank(rank, world, port, out_dir):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for sub in ("oracle", "deepseek-v4-flash-0731-in-c_b200"):
        sys.path.insert(0, os.path.join(root, sub))
    import torch.distributed as dist
    import dsv4cuda
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    dsv4cuda.set_abort_on_error(False)
    L = make_moe_layer(HID, MI, NE, TOPK, seed=77, shared="fp8")
    lo, hi = rank * NE // world, (rank + 1) * NE // world
    d = device_layer(L, lo, hi, dev=f"cuda:{rank}")
    layer = dsv4cuda.MoeLayer(d, max_tokens=8, device=True, expert_range=(lo, hi))
    M = 4
    x = torch.from_numpy(bf16_vals(np.random.default_rng(5), (M, HID))).cuda()
    out = torch.empty((M, HID), dtype=torch.float32, device="cuda")
    layer.forward_local(x)
    dist.all_reduce(layer.routed_slots(M), op=dist.ReduceOp.SUM)
    layer.combine(M, out)
    torch.cuda.synchronize()
    np.save(os.path.join(out_dir, f"nccl_rank{rank}.npy"), out.cpu().numpy())
    layer.close()
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_ep_nccl_two_gpus_matches_single_layer(cuda, tmp_path):
    import torch.multiprocessing as mp
    world = 2
    mp.spawn(_nccl_rank, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    L = make_moe_layer(HID, MI, NE, TOPK, seed=77, shared="fp8")
    full = cuda.MoeLayer(device_layer(L), max_tokens=8, device=True)
    x = torch.from_numpy(bf16_vals(np.random.default_rng(5), (4, HID))).cuda()
    want = torch.empty((4, HID), dtype=torch.float32, device="cuda")
    full.forward(x, want)
    torch.cuda.synchronize()
    w = want.cpu().numpy()
    for r in range(world):
        got = np.load(tmp_path / f"nccl_rank{r}.npy")
        assert np.array_equal(got.view(np.uint32), w.view(np.uint32))
    full.close()


@pytest.mark.parametrize("G,M", [(2, 1), (4, 5), (8, 3)])
def test_ep_p2p_exchange_emulated_matches_single_layer(cuda, G, M):
    """The peer-memory slot exchange (dsv4cuda_moe_ep_attach / _push /
    _combine) with G ranks emulated on one GPU: every rank's pushes are
    issued before any rank's combine waits, in stream order. Three steps
    exercise both halves of the exchange buffer and the step epochs."""
    L = make_moe_layer(HID, MI, NE, TOPK, seed=G * 7 + M, shared="fp8")
    full = cuda.MoeLayer(device_layer(L), max_tokens=8, device=True)
    parts, keep = [], []
    for g in range(G):
        lo, hi = g * NE // G, (g + 1) * NE // G
        d = device_layer(L, lo, hi)
        keep.append(d)
        parts.append(cuda.MoeLayer(d, max_tokens=8, device=True, expert_range=(lo, hi)))
    nbytes = parts[0].ep_buffer_bytes()
    bufs = [torch.empty(nbytes, dtype=torch.uint8, device="cuda") for _ in range(G)]
    for g, p in enumerate(parts):
        p.ep_attach(g, G, [b.data_ptr() for b in bufs])
    rng = np.random.default_rng(G + 100 * M)
    cuda.device_error(clear=True)
    for step in range(3):
        x = torch.from_numpy(bf16_vals(rng, (M, HID))).cuda()
        want = torch.empty((M, HID), dtype=torch.float32, device="cuda")
        full.forward(x, want)
        outs = [torch.full((M, HID), float("nan"), device="cuda") for _ in range(G)]
        for p in parts:
            p.forward_local(x)
            p.ep_push(M)
        for p, o in zip(parts, outs):
            p.ep_combine(M, o)
        torch.cuda.synchronize()
        assert cuda.device_error() == 0
        for o in outs:
            assert torch.equal(o.view(torch.int32), want.view(torch.int32)), step
    for p in parts + [full]:
        p.close()


def _p2p_rank(rank, world, port, out_dir):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for sub in ("oracle", "deepseek-v4-flash-0731-in-c_b200"):
        sys.path.insert(0, os.path.join(root, sub))
    import torch.distributed as dist
    import dsv4cuda
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    dsv4cuda.set_abort_on_error(False)
    L = make_moe_layer(HID, MI, NE, TOPK, seed=78, shared="fp8")
    lo, hi = rank * NE // world, (rank + 1) * NE // world
    d = device_layer(L, lo, hi, dev=f"cuda:{rank}")
    layer = dsv4cuda.MoeLayer(d, max_tokens=8, device=True, expert_range=(lo, hi))
    own, handle = dsv4cuda.ipc_alloc(layer.ep_buffer_bytes())
    handles = [None] * world
    dist.all_gather_object(handles, handle)
    addrs = [own if r == rank else dsv4cuda.ipc_open(handles[r]) for r in range(world)]
    layer.ep_attach(rank, world, addrs)
    dist.barrier()
    M = 3
    rng = np.random.default_rng(6)
    outs = []
    for step in range(3):
        x = torch.from_numpy(bf16_vals(rng, (M, HID))).cuda()
        out = torch.empty((M, HID), dtype=torch.float32, device="cuda")
        layer.forward_ep(x, out)
        torch.cuda.synchronize()
        outs.append(out.cpu().numpy())
    err = dsv4cuda.device_error()
    np.save(os.path.join(out_dir, f"p2p_rank{rank}.npy"), np.stack(outs))
    dist.barrier()
    for r in range(world):
        if r != rank:
            dsv4cuda.ipc_close(addrs[r])
    dist.barrier()
    dsv4cuda.ipc_free(own)
    layer.close()
    dist.destroy_process_group()
    assert err == 0


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_ep_p2p_two_gpus_matches_single_layer(cuda, tmp_path):
    import torch.multiprocessing as mp
    world = 2
    mp.spawn(_p2p_rank, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    L = make_moe_layer(HID, MI, NE, TOPK, seed=78, shared="fp8")
    full = cuda.MoeLayer(device_layer(L), max_tokens=8, device=True)
    rng = np.random.default_rng(6)
    wants = []
    for step in range(3):
        x = torch.from_numpy(bf16_vals(rng, (3, HID))).cuda()
        want = torch.empty((3, HID), dtype=torch.float32, device="cuda")
        full.forward(x, want)
        torch.cuda.synchronize()
        wants.append(want.cpu().numpy())
    w = np.stack(wants)
    for r in range(world):
        got = np.load(tmp_path / f"p2p_rank{r}.npy")
        assert np.array_equal(got.view(np.uint32), w.view(np.uint32))
    full.close()


@pytest.mark.parametrize("G,n_local", [(2, 1), (4, 2), (8, 1)])
def test_ep_tokens_emulated_matches_single_layer(cuda, G, n_local):
    """Token-parallel expert parallelism (dsv4cuda_moe_ep_tokens_*): each of
    G ranks, emulated on one GPU, brings its own n_local tokens; the outputs
    of rank g must equal rows [g * n_local, +n_local) of the single layer run
    on all tokens. All gathers are issued before any wait, then all computes
    before any combine (stream order). Three steps."""
    L = make_moe_layer(HID, MI, NE, TOPK, seed=G * 3 + n_local, shared="fp8")
    M = G * n_local
    full = cuda.MoeLayer(device_layer(L), max_tokens=M, device=True)
    parts, keep = [], []
    for g in range(G):
        lo, hi = g * NE // G, (g + 1) * NE // G
        d = device_layer(L, lo, hi)
        keep.append(d)
        parts.append(cuda.MoeLayer(d, max_tokens=M, device=True, expert_range=(lo, hi)))
    nbytes = parts[0].ep_buffer_bytes()
    bufs = [torch.empty(nbytes, dtype=torch.uint8, device="cuda") for _ in range(G)]
    for g, p in enumerate(parts):
        p.ep_attach(g, G, [b.data_ptr() for b in bufs])
    rng = np.random.default_rng(G * 31 + n_local)
    cuda.device_error(clear=True)
    for step in range(3):
        x = torch.from_numpy(bf16_vals(rng, (M, HID))).cuda()
        want = torch.empty((M, HID), dtype=torch.float32, device="cuda")
        full.forward(x, want)
        xs = [x[g * n_local:(g + 1) * n_local].contiguous() for g in range(G)]
        outs = [torch.full((n_local, HID), float("nan"), device="cuda") for _ in range(G)]
        for p, xg in zip(parts, xs):
            p.ep_tokens_gather(xg)
        for p in parts:
            p.ep_tokens_compute(n_local)
        for p, o in zip(parts, outs):
            p.ep_tokens_combine(n_local, o)
        torch.cuda.synchronize()
        assert cuda.device_error() == 0
        for g, o in enumerate(outs):
            w = want[g * n_local:(g + 1) * n_local]
            assert torch.equal(o.view(torch.int32), w.view(torch.int32)), (step, g)
    for p in parts + [full]:
        p.close()


def _tok_rank(rank, world, port, out_dir):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for sub in ("oracle", "deepseek-v4-flash-0731-in-c_b200"):
        sys.path.insert(0, os.path.join(root, sub))
    import torch.distributed as dist
    import dsv4cuda
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    dsv4cuda.set_abort_on_error(False)
    L = make_moe_layer(HID, MI, NE, TOPK, seed=79, shared="fp8")
    lo, hi = rank * NE // world, (rank + 1) * NE // world
    d = device_layer(L, lo, hi, dev=f"cuda:{rank}")
    n_local = 2
    layer = dsv4cuda.MoeLayer(d, max_tokens=world * n_local, device=True, expert_range=(lo, hi))
    own, handle = dsv4cuda.ipc_alloc(layer.ep_buffer_bytes())
    handles = [None] * world
    dist.all_gather_object(handles, handle)
    addrs = [own if r == rank else dsv4cuda.ipc_open(handles[r]) for r in range(world)]
    layer.ep_attach(rank, world, addrs)
    dist.barrier()
    rng = np.random.default_rng(8)
    outs = []
    for step in range(3):
        x = torch.from_numpy(bf16_vals(rng, (world * n_local, HID))).cuda()
        xl = x[rank * n_local:(rank + 1) * n_local].contiguous()
        out = torch.empty((n_local, HID), dtype=torch.float32, device="cuda")
        layer.forward_ep_tokens(xl, out)
        torch.cuda.synchronize()
        outs.append(out.cpu().numpy())
    err = dsv4cuda.device_error()
    np.save(os.path.join(out_dir, f"tok_rank{rank}.npy"), np.stack(outs))
    dist.barrier()
    for r in range(world):
        if r != rank:
            dsv4cuda.ipc_close(addrs[r])
    dist.barrier()
    dsv4cuda.ipc_free(own)
    layer.close()
    dist.destroy_process_group()
    assert err == 0


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_ep_tokens_two_gpus_matches_single_layer(cuda, tmp_path):
    import torch.multiprocessing as mp
    world, n_local = 2, 2
    mp.spawn(_tok_rank, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    L = make_moe_layer(HID, MI, NE, TOPK, seed=79, shared="fp8")
    full = cuda.MoeLayer(device_layer(L), max_tokens=world * n_local, device=True)
    rng = np.random.default_rng(8)
    wants = []
    for step in range(3):
        x = torch.from_numpy(bf16_vals(rng, (world * n_local, HID))).cuda()
        want = torch.empty((world * n_local, HID), dtype=torch.float32, device="cuda")
        full.forward(x, want)
        torch.cuda.synchronize()
        wants.append(want.cpu().numpy())
    w = np.stack(wants)
    for r in range(world):
        got = np.load(tmp_path / f"tok_rank{r}.npy")
        assert np.array_equal(got.view(np.uint32),
                              w[:, r * n_local:(r + 1) * n_local].view(np.uint32))
    full.close()
