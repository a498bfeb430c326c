"""Expert parallelism on CPU with real collectives (torch.distributed gloo,
world size 2): each rank computes only its experts' (token, k) slots with the
oracle, the zero-padded fp32 slots are summed with all_reduce, and the
ascending-id ordered combine (accumulator from +0, as in
src/dsv4/dsv4_model.c:6795-6805) must reproduce the single-process MoE layer
bit for bit. This is the exchange the GPU expert-parallel path performs with
NCCL (dsv4cuda_moe_forward_local / routed slots / dsv4cuda_moe_combine)."""
import datetime
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

HID, MI, NE, TOPK = 256, 128, 16, 4


def _bf16(x):
    u = x.astype(np.float32).view(np.uint32).astype(np.uint64)
    return (((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16).astype(np.uint32).view(np.float32)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, shared, out_dir):
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "oracle"))
    from oracle import Oracle, make_moe_layer
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    orc = Oracle()
    L = make_moe_layer(HID, MI, NE, TOPK, seed=21, shared=shared)
    lo, hi = rank * NE // world, (rank + 1) * NE // world
    rng = np.random.default_rng(4)
    xs = _bf16(rng.normal(size=(6, HID)))
    outs = []
    for x in xs:
        idx, wt, _ = orc.router_moe(x, L["gate_w"], L.get("bias"), TOPK, L["route_scale"])
        qx, qs = orc.quant_fp8_codes(x)
        slots = np.zeros((TOPK, HID), np.float32)
        for k, e in enumerate(idx):
            if lo <= e < hi:
                slots[k] = orc.expert_forward_fp4(qx, qs, L, int(e), float(wt[k]))
        t = torch.from_numpy(slots)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        summed = t.numpy()
        acc = np.zeros(HID, np.float32)
        for k in range(TOPK):
            acc = acc + summed[k]
        if L.get("shared") is not None:
            acc = acc + orc.shared_forward(qx, qs, L)
        outs.append(_bf16(acc))
    np.save(os.path.join(out_dir, f"ep_rank{rank}.npy"), np.stack(outs))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("shared", ["fp8", None])
def test_expert_parallel_sum_is_exact(tmp_path, orc, shared):
    from oracle import make_moe_layer
    world = 2
    mp.spawn(_rank_main, args=(world, _free_port(), shared, str(tmp_path)), nprocs=world,
             join=True)
    L = make_moe_layer(HID, MI, NE, TOPK, seed=21, shared=shared)
    rng = np.random.default_rng(4)
    xs = _bf16(rng.normal(size=(6, HID)))
    want = np.stack([orc.moe_forward(L, x)[0] for x in xs])
    for r in range(world):
        got = np.load(tmp_path / f"ep_rank{r}.npy")
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
