"""bench.py - greedy decode throughput of DeepSeek-V4-Flash on B200 through
libdsv4_cuda.so (BASELINE config 5 shapes: 43 layers, hidden 4096, 64 heads
x 512, 256 + 1 experts top-6, FP4 experts / FP8 projections, vocabulary
129,280).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

A step is one greedy token: the embedding, every layer (hyper-connection
boundaries, sliding-window attention with FP8 projections and the latent
ring, the MoE layer with its router, six routed FP4 experts and the FP8
shared expert), the HC head, the BF16 vocabulary head and the argmax, all
on the device and replayed as one CUDA graph per token (the argmax feeds
the next step's embedding on the device). Weights are random-init in the
checkpoint's formats; the 43 layers cycle through --decode-sets distinct
weight sets (~3.6 GB each), so no layer's weights are in L2 when it runs.
`e2e` is the same decode through the public host call
(dsv4cuda_decoder_forward_token: token in, logits and next token out).

--impl reference times the reference engine's own dsv4_forward_token on the
host cores (oracle/_ref/ref_decode_bench, built from the reference sources)
on a one-layer checkpoint of the same shapes, extrapolated to 43 layers.
Under torchrun (N > 1) each rank decodes its own sequence and the MoE
layers are expert-parallel (rank r holds experts [r E/N, (r+1) E/N)); the
tokens are gathered and the routed slots returned over peer memory.

--workload moe times the config 2 MoE layer alone (router, 8 routed FP4
experts, FP8 shared expert, combine; four layer weight sets cycled) and
--workload attn the config 3 latent attention (tensor-core kernel).
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "deepseek-v4-flash-0731-in-c_b200")
sys.path.insert(0, PKG)
sys.path.insert(0, os.path.join(ROOT, "oracle"))

H, I, E, TOPK = 7168, 2048, 256, 8
ROUTE_SCALE, LIMIT = 1.5, 10
EXPERT_BYTES = 2 * (I * H // 2 + I * H // 32) + (H * I // 2 + H * I // 32)  # 23,396,352
SHARED_FP8_BYTES = 2 * (I * H + (I // 128) * (H // 128)) + (H * I + (H // 128) * (I // 128))
ROUTER_BYTES = E * H * 2
METRIC = "decode tok/s through one MoE layer (config 2: H7168, I2048, 256+1 experts, top-8)"
# DRAM bytes of one step's two routed GEMV launches (8 experts), from ncu:
# gate/up 125.3 MB read + 4.2 MB written, down 62.5 MB + 0.8 MB
FP4_TRAFFIC_PER_STEP = (125.28 + 4.16 + 62.47 + 0.80) * 1e6


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--ep-mode", default="tokens", choices=["tokens", "replicated"],
                    help="N > 1: each rank brings its own --tokens tokens (weak scaling, "
                         "tokens gathered and slots returned over peer memory) or every rank "
                         "runs the same tokens (strong scaling)")
    ap.add_argument("--ep-exchange", default="p2p", choices=["p2p", "nccl"],
                    help="replicated mode's slot exchange: peer-memory kernels or NCCL all-reduce")
    ap.add_argument("--tokens", type=int, default=1, help="tokens per step (M)")
    ap.add_argument("--layers", type=int, default=4, help="independent layer weight sets")
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--experts", type=int, default=E,
                    help="routed experts per layer (smaller only for profiling captures)")
    ap.add_argument("--inter", type=int, default=I,
                    help="expert intermediate size (smaller only for profiling captures)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-e2e", action="store_true", help="skip the end-to-end leg")
    ap.add_argument("--workload", default="decode", choices=["moe", "attn", "decode"],
                    help="decode (default): config 5 batch-1 greedy decode through every "
                         "layer on the device; moe: config 2 MoE layer; attn: config 3 latent "
                         "decode attention at --attn-batch/--attn-ctx")
    ap.add_argument("--no-moe-sub", action="store_true",
                    help="decode: skip the config 2 expert-GEMV measurement attached to the line")
    ap.add_argument("--decode-sets", type=int, default=4,
                    help="decode: distinct random-init layer weight sets the 43 layers cycle "
                         "through (each ~3.6 GB; L2 never holds a layer between uses)")
    ap.add_argument("--decode-layers", type=int, default=43)
    ap.add_argument("--decode-prompt", type=int, default=2048,
                    help="decode: context positions decoded before timing (2048: the "
                         "benchmark's; fewer only for profiling captures)")
    ap.add_argument("--decode-ratios", default="dsv4", choices=["dsv4", "window"],
                    help="decode: DeepSeek-V4-Flash's compress ratios (two window layers, then "
                         "ratio 4 / 128 alternating) or every layer a sliding-window layer")
    ap.add_argument("--attn-batch", type=int, default=32)
    ap.add_argument("--attn-ctx", type=int, default=32768)
    ap.add_argument("--no-spec", action="store_true",
                    help="decode: skip the speculation-on measurement (verify steps of a "
                         "k = 5 draft chain)")
    ap.add_argument("--no-batch1", action="store_true",
                    help="decode, N > 1: skip the batch-1 (replicated-token) measurement")
    ap.add_argument("--spec-rows", type=int, default=6,
                    help="decode: rows per verify step (the pending token + k drafts)")
    ap.add_argument("--no-attn-sweep", action="store_true",
                    help="skip the config 3 attention sweep attached to the MoE line")
    return ap.parse_args()


def chain_lengths(count, n_layers):
    """Layers per graph replay covering exactly `count` steps: full chains of
    n_layers, then one shorter chain for the remainder."""
    out = []
    while count > 0:
        out.append(min(n_layers, count))
        count -= out[-1]
    return out


# ---------------------------------------------------------------- weights --
EXPERT_BLOCK = 32  # routed experts drawn per generator seed


def expert_blocks(n_experts, world):
    """Experts per generator block: a divisor of every rank's share, so any
    rank can regenerate any expert's weights bit for bit."""
    blk = min(EXPERT_BLOCK, n_experts)
    while blk > 1 and (n_experts % blk or (n_experts // max(world, 1)) % blk):
        blk //= 2
    return max(blk, 1)


def make_device_layer(torch, seed, dev, E=E, I=I, expert_range=None, block=None):
    """Random-init config-2 layer in the reference layouts, on the GPU.
    expert_range=(lo, hi): routed weights of those experts only (expert
    parallelism); the router and shared expert are the same on every rank.
    Routed experts are drawn in blocks of `block` experts, each block from
    its own seed, so a rank's share equals the same experts of the full
    layer bit for bit."""
    lo, hi = expert_range if expert_range else (0, E)
    blk = block or expert_blocks(E, 1)
    assert lo % blk == 0 and hi % blk == 0, (lo, hi, blk)
    g = torch.Generator(device=dev)
    g.manual_seed(seed)

    def u8(*shape, gen):
        return torch.randint(0, 256, shape, dtype=torch.uint8, device=dev, generator=gen)

    def e8m0(*shape, gen):
        # lognormal(0, 0.5) scale rounded to a power of two: 127 + round(log2 s)
        z = torch.randn(shape, device=dev, generator=gen) * (0.5 / np.log(2.0))
        return (127 + torch.round(z)).clamp(0, 254).to(torch.uint8)

    def fp8(*shape):
        c = torch.randint(0, 254, shape, dtype=torch.int32, device=dev, generator=g)
        c = torch.where((c & 0x7F) == 0x7F, c - 1, c)
        return c.to(torch.uint8)

    gate = (torch.randn(E, H, device=dev, generator=g) * 0.02).to(torch.bfloat16).view(torch.uint16)
    shared = dict(fp8=True, w1=fp8(I, H), s1=e8m0(I // 128, H // 128, gen=g),
                  w3=fp8(I, H), s3=e8m0(I // 128, H // 128, gen=g),
                  w2=fp8(H, I), s2=e8m0(H // 128, I // 128, gen=g))
    n = hi - lo
    shapes = dict(w1=(I, H // 2), s1=(I, H // 32), w3=(I, H // 2), s3=(I, H // 32),
                  w2=(H, I // 2), s2=(H, I // 32))
    routed = {k: torch.empty((n, *sh), dtype=torch.uint8, device=dev) for k, sh in shapes.items()}
    for b in range(lo // blk, hi // blk):
        gb = torch.Generator(device=dev)
        gb.manual_seed(seed * 1000 + b + 1)
        r0 = b * blk - lo
        for k, sh in shapes.items():
            draw = u8 if k[0] == "w" else e8m0
            routed[k][r0:r0 + blk].copy_(draw(blk, *sh, gen=gb))
    return dict(hidden=H, moe_inter=I, n_experts=E, topk=TOPK, route_scale=ROUTE_SCALE,
                swiglu_limit=LIMIT, gate_w=gate, bias=None, tid2eid=None, shared=shared,
                **routed)


def bf16_tokens(rng, n, m):
    x = rng.normal(size=(n, m, H)).astype(np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    return (((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16).astype(np.uint32).view(np.float32)


# ------------------------------------------------------------- clocks ----
class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            p = [v.strip() for v in ln.split(",")]
            if len(p) < 9:
                continue
            try:
                sm.append(float(p[1]))
                mx = float(p[2])
            except ValueError:
                continue
            for n, v in zip(names, p[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------ CPU side ----
def host_layer_for_reference(rng):
    """Config-2 layer in host memory, routed experts already in the
    reference's cache-slot layout (scale run then weight run per expert)."""
    s13, s2 = I * (H // 32), H * (I // 32)
    w13, w2 = I * (H // 2), H * (I // 2)

    def e8m0(n):
        return (127 + np.round(rng.normal(0, 0.5 / np.log(2.0), size=n))).clip(0, 254).astype(np.uint8)

    def fp8(shape):
        c = rng.integers(0, 254, size=shape, dtype=np.int32)
        return np.where((c & 0x7F) == 0x7F, c - 1, c).astype(np.uint8)

    gate = (rng.normal(0, 0.02, size=(E, H)).astype(np.float32))
    u = gate.view(np.uint32).astype(np.uint64)
    gate = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    scales = e8m0(E * (2 * s13 + s2)).reshape(E, -1)
    weights = rng.integers(0, 256, size=(E, 2 * w13 + w2), dtype=np.uint8)
    shared = dict(fp8=True, w1=fp8((I, H)), s1=e8m0((I // 128) * (H // 128)).reshape(I // 128, -1),
                  w3=fp8((I, H)), s3=e8m0((I // 128) * (H // 128)).reshape(I // 128, -1),
                  w2=fp8((H, I)), s2=e8m0((H // 128) * (I // 128)).reshape(H // 128, -1))
    return dict(hidden=H, moe_inter=I, n_experts=E, topk=TOPK, route_scale=ROUTE_SCALE,
                swiglu_limit=LIMIT, gate_w=gate, bias=None, tid2eid=None, shared=shared), \
        (scales, weights)


def host_threads():
    try:
        return len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


def cpu_reference_run(seconds, steps_cap=None, warmup=1, threads=None):
    """Times the reference's own MoE-layer step on the host cores with
    `threads` OpenMP threads (default: every core this process may use; set
    explicitly because launchers such as torchrun pre-set OMP_NUM_THREADS=1).
    Returns (tok/s, cores, kind, sample description)."""
    from oracle import REF_SO
    ncpu = os.cpu_count() or 1
    threads = threads or host_threads()
    rng = np.random.default_rng(99)
    layer, slots = host_layer_for_reference(rng)
    toks = bf16_tokens(rng, 64, 1)[:, 0]
    if os.path.exists(REF_SO):
        from oracle import Ref
        r = Ref()
        kind = "reference"
        cores = r.lib.ref_omp_set_threads(threads)
        run = lambda x: r.moe_forward(layer, x, slots=slots)  # noqa: E731
    else:
        from oracle import Oracle
        o = Oracle()
        kind = "port"
        cores = 1
        s13, w13 = I * (H // 32), I * (H // 2)
        lay = dict(layer)
        sc, wt = slots
        lay["w1"], lay["w2"], lay["w3"] = (wt[:, :w13].reshape(E, I, H // 2),
                                           wt[:, w13:w13 + H * I // 2].reshape(E, H, I // 2),
                                           wt[:, w13 + H * I // 2:].reshape(E, I, H // 2))
        lay["s1"], lay["s2"], lay["s3"] = (sc[:, :s13].reshape(E, I, H // 32),
                                           sc[:, s13:s13 + H * I // 32].reshape(E, H, I // 32),
                                           sc[:, s13 + H * I // 32:].reshape(E, I, H // 32))
        lay = {k: (np.ascontiguousarray(v) if isinstance(v, np.ndarray) else v) for k, v in lay.items()}
        run = lambda x: o.moe_forward(lay, x)  # noqa: E731
    for i in range(warmup):
        run(toks[i % len(toks)])
    n, t0 = 0, time.perf_counter()
    while True:
        run(toks[n % len(toks)])
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds or (steps_cap and n >= steps_cap):
            break
    return n / el, cores, kind, f"{n} decode steps (M=1) through one config-2 MoE layer, " \
        f"256 experts resident in host RAM, {el:.1f} s on {cores} thread(s) of {ncpu} cores"


def moe_config(args, world):
    """The `config` of the MoE line, the same in both arms."""
    M = args.tokens
    ep = world > 1
    tok_mode = ep and args.ep_mode == "tokens"
    return {"workload": "config 2 MoE layer op, decode M=%d" % M, "hidden": H,
            "moe_inter": args.inter, "experts": args.experts, "topk": TOPK, "shared": "fp8",
            "tokens_per_step": M * world if tok_mode else M, "tokens_per_gpu": M,
            "layers_cycled": args.layers,
            "graph": "one CUDA graph replay chains the %d layers (a step = one "
                     "layer pass of one token)" % args.layers,
            "l2": "inputs larger than L2: each step reads a different layer's "
                  "~235 MB of weights", "parallelism": f"ep{world}",
            "ep_mode": (args.ep_mode if ep else None),
            "ep_exchange": (("p2p" if (tok_mode or args.ep_exchange == "p2p") else "nccl")
                            if ep else None)}


def run_reference_arm(args, rank, world):
    if rank != 0:
        return
    if args.workload == "decode":
        res = cpu_reference_decode(args.decode_layers, kinds_mode=args.decode_ratios)
        if res is None:
            print(json.dumps({"impl": "reference", "unavailable":
                              "oracle/_ref/ref_decode_bench was not built (reference sources absent)"}))
            return
        tps, cores, sample, _ = res
        print(json.dumps({
            "impl": "reference", "metric": DECODE_METRIC, "value": tps, "unit": "tok/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1e3 / tps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "fp4e2m1/fp8e4m3 weights, bf16 activations, f32 accumulate",
            "data": "synthetic (random-init weights with the checkpoint's formats)",
            "config": decode_config(args, world),
            "cpu_baseline": {"value": tps, "unit": "tok/s", "cores": cores, "kind": "reference",
                             "sample": sample, "extrapolated": True},
            "e2e": {"value": tps, "unit": "tok/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}), flush=True)
        return
    per_step_cap = max(args.steps, 1)
    # warm-up, then K timed steps, each step one decode token (bounded run)
    tps, cores, kind, sample = cpu_reference_run(seconds=max(args.cpu_seconds * 5, 60.0),
                                                 steps_cap=per_step_cap, warmup=args.warmup)
    line = {
        "impl": "reference", "metric": METRIC, "value": tps, "unit": "tok/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 / tps, "higher_is_better": True,
        "scaling": "strong" if args.ep_mode == "replicated" else "weak",
        "vs_baseline": None, "dtype": "fp4e2m1*e4m3->f32", "data": "synthetic",
        "config": moe_config(args, world),
        "cpu_baseline": {"value": tps, "unit": "tok/s", "cores": cores, "kind": kind,
                         "sample": sample},
        "e2e": {"value": tps, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# -------------------------------------------------------------- GPU side --
def main():
    args = parse()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference_arm(args, rank, world)
        return
    if args.workload == "attn":
        main_attn(args, rank, world, local)
        return
    if args.workload == "decode":
        main_decode(args, rank, world, local)
        return

    import torch
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=dev)
    import dsv4cuda
    dsv4cuda.set_abort_on_error(False)
    dsv4cuda.init(local)

    M = args.tokens
    ep = world > 1
    tok_mode = ep and args.ep_mode == "tokens"
    M_all = M * world if tok_mode else M  # tokens each rank's layer routes per step
    erange = (rank * args.experts // world, (rank + 1) * args.experts // world) if ep else None
    layers = []
    block = expert_blocks(args.experts, world)
    for li in range(args.layers):
        lay = make_device_layer(torch, 1000 + li, dev, args.experts, args.inter, erange, block)
        layers.append((lay, dsv4cuda.MoeLayer(lay, max_tokens=M_all, device=True,
                                              expert_range=erange)))
    torch.cuda.synchronize()
    p2p = ep and (tok_mode or args.ep_exchange == "p2p")
    ipc_own, ipc_peers = [], []
    if p2p:
        # one exchange buffer per layer and rank, mapped into every rank
        handles = []
        for _, L in layers:
            addr, h = dsv4cuda.ipc_alloc(L.ep_buffer_bytes())
            ipc_own.append(addr)
            handles.append(h)
        all_h = [None] * world
        dist.all_gather_object(all_h, handles)
        for li, (_, L) in enumerate(layers):
            addrs = []
            for r in range(world):
                if r == rank:
                    addrs.append(ipc_own[li])
                else:
                    a = dsv4cuda.ipc_open(all_h[r][li])
                    ipc_peers.append(a)
                    addrs.append(a)
            L.ep_attach(rank, world, addrs)
        dist.barrier()

    def layer_forward(L, xin, out, s):
        """One MoE layer; expert parallel: local experts, then the routed
        slots reach every rank either through the peer-memory exchange
        kernels or as an NCCL sum of the zero-padded slots, then the ordered
        combine (bit-identical to 1 GPU either way)."""
        if not ep:
            L.forward(xin, out, stream=s)
            return
        if tok_mode:
            L.forward_ep_tokens(xin, out, stream=s)
            return
        if p2p:
            L.forward_ep(xin, out, stream=s)
            return
        L.forward_local(xin, stream=s)
        dist.all_reduce(L.routed_slots(M), op=dist.ReduceOp.SUM)
        L.combine(M, out, stream=s)
    rng = np.random.default_rng(7 + (1000 * rank if tok_mode else 0))  # own tokens per rank
    pool = 8 * len(layers)
    x_host = bf16_tokens(rng, pool, M)
    x_dev = torch.from_numpy(x_host).to(dev)
    out_dev = torch.empty((M, H), dtype=torch.float32, device=dev)

    # one CUDA graph per layer (launch overhead amortised; same kernels)
    stream = torch.cuda.Stream(device=dev)
    graphs = []
    xin = torch.empty((M, H), dtype=torch.float32, device=dev)
    with torch.cuda.stream(stream):
        for _, L in layers:  # warm the kernels (and the communicator) outside capture
            xin.copy_(x_dev[0])
            layer_forward(L, xin, out_dev, stream.cuda_stream)
    stream.synchronize()
    for _, L in layers:
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            layer_forward(L, xin, out_dev, torch.cuda.current_stream().cuda_stream)
        graphs.append(g)

    # The timed loop replays graphs that chain the layers back to back: one
    # decode token through len(layers) consecutive MoE layers, each layer on
    # its own token rows, as a model's decode step runs its layers; chains of
    # 1..len(layers) layers let a run cover exactly the requested steps.
    n_lay = len(layers)
    xch = torch.empty((n_lay, M, H), dtype=torch.float32, device=dev)
    och = torch.empty((n_lay, M, H), dtype=torch.float32, device=dev)
    chains = []
    for n in range(1, n_lay + 1):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            cs = torch.cuda.current_stream().cuda_stream
            for li in range(n):
                layer_forward(layers[li][1], xch[li], och[li], cs)
        chains.append(g)
    replays = [0]

    def run_steps(count, host=None):
        """`count` steps: new token rows for each chained layer, one replay
        per chain. host=(pinned inputs, pinned outputs): the rows come from
        and the outputs go back to host memory, synchronised per replay."""
        for n in chain_lengths(count, n_lay):
            s0 = (replays[0] * n_lay) % pool
            if host is None:
                xch[:n].copy_(x_dev[s0:s0 + n], non_blocking=True)
            else:
                xch[:n].copy_(host[0][s0:s0 + n], non_blocking=True)
            chains[n - 1].replay()
            if host is not None:
                host[1][:n].copy_(och[:n], non_blocking=True)
                stream.synchronize()
            replays[0] += 1

    with torch.cuda.stream(stream):
        run_steps(args.warmup)
    torch.cuda.synchronize()

    def timed_window():
        """K steps between two events on the forward stream, max over ranks.
        Under expert parallelism one untimed step runs first: its peer-memory
        waits line the ranks up, so the window holds no start skew."""
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        ev0 = torch.cuda.Event(enable_timing=True)
        ev1 = torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            if ep:
                run_steps(1)
            ev0.record(stream)
            run_steps(args.steps)
            ev1.record(stream)
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        t = ev0.elapsed_time(ev1)
        if dist:
            tt = torch.tensor([t], device=dev)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            t = float(tt.item())
        return t

    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    windows = [timed_window() for _ in range(5)]
    clk = clocks.stop()
    ms = windows[0]
    ms_per_step = ms / args.steps
    tok_per_step = M * world if tok_mode else M
    value = tok_per_step * args.steps / (ms / 1e3)
    win_vals = [tok_per_step * args.steps / (w / 1e3) for w in windows]

    # ---- expert-GEMV roofline: each layer's forward captured once more into
    # a graph whose event nodes bracket the routed gate/up and down launches
    # (and the router); replayed like the timed steps, read after each replay
    U_total, n_fw, fallbacks = 0, 0, 0
    lib = dsv4cuda.lib
    import ctypes as C
    tgraphs = []
    for _, L in layers:
        lib.dsv4cuda_moe_timing_begin(L.handle)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            layer_forward(L, xin, out_dev, torch.cuda.current_stream().cuda_stream)
        tgraphs.append(g)
    gu_ms = dn_ms = lg_ms = sl_ms = 0.0
    n_timed = 0
    a_, b_, c_, d_ = C.c_float(), C.c_float(), C.c_float(), C.c_float()
    with torch.cuda.stream(stream):
        for i in range(max(8, args.steps // 4)):
            li = i % len(layers)
            _, L = layers[li]
            xin.copy_(x_dev[i % pool])
            tgraphs[li].replay()
            stream.synchronize()
            if lib.dsv4cuda_moe_timing_read(L.handle, 0, C.byref(a_), C.byref(b_), C.byref(c_),
                                            C.byref(d_)) != 0:
                raise RuntimeError(dsv4cuda.last_error())
            gu_ms += a_.value
            dn_ms += b_.value
            lg_ms += c_.value
            sl_ms += d_.value
            n_timed += 1
            idx, _, fb = L.last_routes(M_all)
            U_total += len(np.unique(idx))
            fallbacks = fb
            n_fw += 1
    torch.cuda.synchronize()
    for gr in tgraphs:
        gr.reset()
    tgraphs = []
    g = None
    n = C.c_int()
    for _, L in layers:
        lib.dsv4cuda_moe_timing_end2(L.handle, C.byref(n), None, None, None, None)
    # our kernels per step: activation quant, router (2), shared expert (3),
    # routed gate/up, SwiGLU, down, combine; a second gate/up and down for
    # multi-route items when a step routes two or more tokens; the
    # peer-memory exchange kernels
    launches_per_step = 10 + (2 if M_all >= 2 else 0)
    if tok_mode:
        launches_per_step += 3  # gather, gather wait, owner push (+ owner combine for combine)
    elif p2p:
        launches_per_step += 1  # slot push (+ exchange combine for combine)
    U_avg = U_total / max(n_fw, 1)
    if ep:  # this rank's share of the unique experts (uniform routing)
        U_avg = U_avg * (erange[1] - erange[0]) / args.experts
    alg_bytes = U_avg * EXPERT_BYTES
    kern_ms = (gu_ms + dn_ms) / max(n_timed, 1)
    achieved = alg_bytes / (kern_ms * 1e-3) / 1e9
    peaks_path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    peak, peak_src = 6650.0, "fallback"
    if os.path.exists(peaks_path):
        peak = float(json.load(open(peaks_path))["hbm_gbs"])
        peak_src = "measured"

    # ---- end to end through the public C API with host buffers
    e2e_val = None
    if not args.no_e2e:
        if ep:
            pin_x = torch.from_numpy(x_host).pin_memory()
            pin_out = torch.empty((n_lay, M, H), dtype=torch.float32).pin_memory()
            e2e_steps = max(20, args.steps // 2)
            with torch.cuda.stream(stream):
                run_steps(n_lay, host=(pin_x, pin_out))  # untimed: aligns the ranks
            dist.barrier()
            t0 = time.perf_counter()
            with torch.cuda.stream(stream):
                run_steps(e2e_steps, host=(pin_x, pin_out))
            el = torch.tensor([time.perf_counter() - t0], device=dev)
            dist.all_reduce(el, op=dist.ReduceOp.MAX)
            e2e_val = tok_per_step * e2e_steps / float(el.item())
        else:
            e2e_val = run_e2e(args, layers, x_host, M, pool, lib, dsv4cuda)

    # ---- expert parallelism: this rank's outputs of one step against the
    # full layer (every expert, same weights) run on this GPU alone
    ep_check = None
    if ep:
        full = make_device_layer(torch, 1000, dev, args.experts, args.inter, None, block)
        Lfull = dsv4cuda.MoeLayer(full, max_tokens=M_all, device=True)
        xin.copy_(x_dev[0])
        got = torch.empty((M, H), dtype=torch.float32, device=dev)
        want = torch.empty((M, H), dtype=torch.float32, device=dev)
        with torch.cuda.stream(stream):
            layer_forward(layers[0][1], xin, got, stream.cuda_stream)
            Lfull.forward(xin, want, stream=stream.cuda_stream)
        torch.cuda.synchronize()
        same = torch.tensor([1 if torch.equal(got.view(torch.int32), want.view(torch.int32))
                             else 0], device=dev)
        dist.all_reduce(same, op=dist.ReduceOp.MIN)
        ep_check = {"bit_identical_to_1gpu": bool(same.item()),
                    "tokens_checked": M * world if tok_mode else M,
                    "how": "one step of layer 0 on every rank vs the same layer with all "
                           "experts on one GPU, output bits compared, min over ranks"}
        Lfull.close()
        del full, Lfull
        torch.cuda.empty_cache()

    # ---- config 3 attention sweep (replicated part of the decode layer)
    attn = None
    if world == 1 and not args.no_attn_sweep:
        attn = run_attn_sweep(torch, dsv4cuda, dev)

    line = None
    if rank == 0:
        cpu = cpu1 = None
        if world == 1 and not args.no_cpu:
            try:
                tps, cores, kind, sample = cpu_reference_run(args.cpu_seconds)
                cpu = {"value": tps, "unit": "tok/s", "cores": cores, "kind": kind,
                       "sample": sample}
                tps, cores, kind, sample = cpu_reference_run(min(args.cpu_seconds, 8.0),
                                                             threads=1)
                cpu1 = {"value": tps, "unit": "tok/s", "cores": cores, "kind": kind,
                        "sample": sample}
            except Exception as exc:  # report, do not hide
                cpu = {"value": None, "unit": "tok/s", "cores": 0, "kind": "reference",
                       "sample": f"failed: {exc}"}
        line = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
            "higher_is_better": True,
            "scaling": "strong" if (ep and not tok_mode) else "weak", "vs_baseline": None,
            "dtype": "fp4e2m1*e4m3->f32", "data": "synthetic",
            "config": moe_config(args, world),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": FP4_TRAFFIC_PER_STEP,
                         "traffic_source": "ncu dram__bytes_read+write of the gate/up and down "
                                           "launches for 8 experts "
                                           "(profiles/fp4_stream_kernel_experts8.md)",
                         "kernel": "fp4_stream_kernel (routed gate/up pair + down)",
                         "alg_bytes_per_step": alg_bytes, "peak_source": peak_src,
                         "kernel_ms_per_step": kern_ms,
                         "phase_ms_per_step": {
                             "router_logits": lg_ms / max(n_timed, 1),
                             "router_select": sl_ms / max(n_timed, 1),
                             "expert_gateup": gu_ms / max(n_timed, 1),
                             "expert_down": dn_ms / max(n_timed, 1)}},
            "cpu_baseline": cpu,
            "cpu_baseline_1thread": cpu1,
            "repeat_windows": {"n": len(win_vals), "steps_each": args.steps,
                               "values": win_vals, "min": min(win_vals), "max": max(win_vals),
                               "spread_pct": 100.0 * (max(win_vals) - min(win_vals)) /
                               max(win_vals)},
            "ep_check": ep_check,
            "e2e": {"value": e2e_val, "unit": "tok/s", "h2d_bytes_per_step": M * H * 4,
                    "d2h_bytes_per_step": M * H * 4},
            "gpu_launches": launches_per_step * args.steps,
            "router_tie_fallbacks": fallbacks,
            "clocks": clk,
            "attn_config3": attn,
        }
        print(json.dumps(line), flush=True)
    # graphs holding NCCL calls must be released before the process group
    torch.cuda.synchronize()
    for gr in graphs + chains:
        gr.reset()
    graphs.clear()
    chains.clear()
    g = gr = None  # noqa: F841  (the capture loop's last graph)
    if p2p:
        # every rank stops touching peer memory before any buffer is unmapped
        dist.barrier()
        for a in ipc_peers:
            dsv4cuda.ipc_close(a)
        dist.barrier()
        for a in ipc_own:
            dsv4cuda.ipc_free(a)
    for _, L in layers:
        L.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


def run_e2e(args, layers, x_host, M, pool, lib, dsv4cuda):
    import ctypes as C
    import torch
    pin_x = torch.from_numpy(x_host).pin_memory()
    pin_out = torch.empty((M, H), dtype=torch.float32).pin_memory()
    xs = pin_x.numpy()
    outs = pin_out.numpy()
    for _, Li in layers:  # the first calls per layer capture its forward graph
        for i in range(3):
            Li.forward_host(xs[i % pool])
    ptr_out = outs.ctypes.data_as(C.POINTER(C.c_float))
    t0 = time.perf_counter()
    e2e_steps = max(20, args.steps // 2)
    for i in range(e2e_steps):
        _, Li = layers[i % len(layers)]
        xi = xs[i % pool]
        rc = lib.dsv4cuda_moe_forward_host(Li.handle, xi.ctypes.data_as(C.POINTER(C.c_float)),
                                           None, M, ptr_out)
        if rc != 0:
            raise RuntimeError(dsv4cuda.last_error())
    e2e_s = time.perf_counter() - t0
    e2e_val = M * e2e_steps / e2e_s
    return e2e_val


# ------------------------------------------------- config 3: attention ----
ATTN_H, ATTN_D = 128, 512
ATTN_SWEEP = [(1, 4096), (8, 4096), (32, 4096), (1, 32768), (8, 32768), (32, 32768)]
ATTN_METRIC = "latent decode attention queries/s (config 3: 128 heads x 512, FP8 latent cache)"


def attn_flops(B, ctx):
    return B * 2 * 2 * ATTN_H * ATTN_D * ctx  # Q K^T and P V


def attn_bytes(B, ctx):
    # FP8 cache (584 B per position) + q in + o out (fp32 at the C ABI)
    return B * (ctx * 584 + 2 * ATTN_H * ATTN_D * 4)


class AttnCase:
    """Config 3 inputs on the device: latent rows N(0,1) (BF16) quantised into
    the FP8 cache by the reference's KV QAT rule, q and sink N(0,1), positions
    0..ctx-1 for every query of the batch."""

    def __init__(self, torch, dsv4cuda, dev, B, ctx, seed=0):
        g = torch.Generator(device=dev)
        g.manual_seed(seed)
        rows = B * ctx
        self.cache = dsv4cuda.LatentCache(rows, device=dev)
        chunk = 1 << 16
        for r0 in range(0, rows, chunk):
            n = min(chunk, rows - r0)
            kv = torch.randn((n, ATTN_D), generator=g, device=dev).to(torch.bfloat16).float()
            self.cache.write(kv, torch.arange(r0, r0 + n, device=dev, dtype=torch.int64))
        self.q = torch.randn((B, ATTN_H, ATTN_D), generator=g, device=dev).to(
            torch.bfloat16).float()
        self.sink = torch.randn(ATTN_H, generator=g, device=dev)
        self.idx = torch.arange(ctx, device=dev, dtype=torch.int32).repeat(B, 1).contiguous()
        self.out = torch.empty_like(self.q)
        self.shape = dsv4cuda.attn_shape(B, ATTN_H, ATTN_D, ctx, ATTN_D ** -0.5, 64, ctx, ctx)
        self.ws = torch.empty(dsv4cuda.attn_workspace_bytes(self.shape, True), dtype=torch.uint8,
                              device=dev)
        self.B, self.ctx = B, ctx

    def run(self, dsv4cuda, stream):
        dsv4cuda.sparse_attn(self.out, self.q, self.sink, self.idx, self.shape, cache=self.cache,
                             workspace=self.ws, stream=stream)


def attn_measure(torch, dsv4cuda, case, stream, iters, warmup, flush):
    """Mean device time of one call (all kernels) and of its main tensor-core
    kernel, with L2 flushed before every timed call."""
    with torch.cuda.stream(stream):
        for _ in range(warmup):
            case.run(dsv4cuda, stream.cuda_stream)
    torch.cuda.synchronize()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(iters)]
    dsv4cuda.attn_timing_begin()
    with torch.cuda.stream(stream):
        for a, b in evs:
            flush.zero_()
            a.record(stream)
            case.run(dsv4cuda, stream.cuda_stream)
            b.record(stream)
    torch.cuda.synchronize()
    n, main_ms = dsv4cuda.attn_timing_end()
    call_ms = sum(a.elapsed_time(b) for a, b in evs) / iters
    return call_ms, main_ms / max(n, 1)


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        p = json.load(open(path))
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def attn_point(torch, dsv4cuda, dev, stream, B, ctx, iters, warmup, flush):
    case = AttnCase(torch, dsv4cuda, dev, B, ctx, seed=B * 7 + ctx)
    call_ms, main_ms = attn_measure(torch, dsv4cuda, case, stream, iters, warmup, flush)
    hbm, tfl, src = peaks()
    fl, by = attn_flops(B, ctx), attn_bytes(B, ctx)
    bound_ms = max(fl / (tfl * 1e12), by / (hbm * 1e9)) * 1e3
    res = {"batch": B, "ctx": ctx, "us_per_call": call_ms * 1e3, "main_kernel_us": main_ms * 1e3,
           "tflops": fl / (call_ms * 1e-3) / 1e12, "gbs": by / (call_ms * 1e-3) / 1e9,
           "frac_tensor": fl / (call_ms * 1e-3) / 1e12 / tfl,
           "frac_hbm": by / (call_ms * 1e-3) / 1e9 / hbm,
           "roofline_frac": bound_ms / call_ms}
    del case
    torch.cuda.empty_cache()
    return res


def run_attn_sweep(torch, dsv4cuda, dev, iters=10, warmup=3):
    stream = torch.cuda.Stream(device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    out = [attn_point(torch, dsv4cuda, dev, stream, B, ctx, iters, warmup, flush)
           for B, ctx in ATTN_SWEEP]
    del flush
    return out


def cpu_attn_reference(seconds, B, ctx):
    """Reference sparse_attn (oracle/_ref, OpenMP over heads) on the host:
    queries/s on a bounded sample of the config (one query at a time)."""
    from oracle import REF_SO, Oracle
    rng = np.random.default_rng(5)
    kv = rng.normal(size=(ctx, ATTN_D)).astype(np.float32)
    o = Oracle()
    for r in range(ctx):  # the reference's cache values (KV QAT, group 64)
        kv[r, :448] = o.act_quant_inplace(kv[r, :448], 64, 0)
    q = rng.normal(size=(ATTN_H, ATTN_D)).astype(np.float32)
    sink = rng.normal(size=ATTN_H).astype(np.float32)
    idx = np.arange(ctx, dtype=np.int32)
    if os.path.exists(REF_SO):
        from oracle import Ref
        r = Ref()
        kind, cores = "reference", r.lib.ref_omp_max_threads()
        run = lambda: r.sparse_attn(q, kv, sink, idx, ATTN_D ** -0.5)  # noqa: E731
    else:
        kind, cores = "port", 1
        run = lambda: o.sparse_attn(q, kv, sink, idx, ATTN_D ** -0.5)  # noqa: E731
    run()
    n, t0 = 0, time.perf_counter()
    while True:
        run()
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    return n / el, cores, kind, (f"{n} single-query sparse_attn calls (128 heads x 512, "
                                 f"ctx {ctx}), {el:.1f} s on {cores} thread(s)")


def main_attn(args, rank, world, local):
    """--workload attn: config 3 at --attn-batch x --attn-ctx. Attention is
    replicated (every rank holds every query), so N GPUs run N replicas."""
    import torch
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    import dsv4cuda
    dsv4cuda.set_abort_on_error(False)
    dsv4cuda.init(local)
    B, ctx = args.attn_batch, args.attn_ctx
    case = AttnCase(torch, dsv4cuda, dev, B, ctx, seed=3)
    stream = torch.cuda.Stream(device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            case.run(dsv4cuda, stream.cuda_stream)
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    total = 0.0
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
           for _ in range(args.steps)]
    dsv4cuda.attn_timing_begin()
    with torch.cuda.stream(stream):
        for a, b in evs:
            flush.zero_()
            a.record(stream)
            case.run(dsv4cuda, stream.cuda_stream)
            b.record(stream)
    torch.cuda.synchronize()
    n_main, main_ms = dsv4cuda.attn_timing_end()
    total = sum(a.elapsed_time(b) for a, b in evs)
    if dist:
        dist.barrier()
        t = torch.tensor([total], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total = float(t.item())
    clk = clocks.stop()
    ms = total / args.steps
    main_ms = main_ms / max(n_main, 1)
    hbm, tfl, src = peaks()
    fl, by = attn_flops(B, ctx), attn_bytes(B, ctx)
    # e2e: q from pinned host memory in, o back to pinned host memory, cache resident
    qh = case.q.cpu().pin_memory()
    oh = torch.empty_like(qh).pin_memory()
    e2e_steps = max(5, args.steps // 2)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    with torch.cuda.stream(stream):
        for _ in range(e2e_steps):
            case.q.copy_(qh, non_blocking=True)
            case.run(dsv4cuda, stream.cuda_stream)
            oh.copy_(case.out, non_blocking=True)
            stream.synchronize()
    e2e = B * e2e_steps / (time.perf_counter() - t0)
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu:
            v, cores, kind, sample = cpu_attn_reference(args.cpu_seconds, B, ctx)
            cpu = {"value": v, "unit": "queries/s", "cores": cores, "kind": kind,
                   "sample": sample}
        line = {
            "metric": ATTN_METRIC, "value": B * world / (ms * 1e-3), "unit": "queries/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16*bf16->f32 (FP8 e4m3 cache)", "data": "synthetic",
            "config": {"workload": f"config 3 latent decode attention, batch {B}, ctx {ctx}",
                       "heads": ATTN_H, "head_dim": ATTN_D, "rope": 64, "batch": B, "ctx": ctx,
                       "l2": "flushed (256 MB write) before every timed call",
                       "parallelism": f"replicas{world}"},
            "roofline": {"bound": "tensor" if fl / tfl > by / hbm * 1e3 else "hbm",
                         "achieved": fl / (main_ms * 1e-3) / 1e12, "peak": tfl,
                         "unit": "TFLOP/s", "frac": fl / (main_ms * 1e-3) / 1e12 / tfl,
                         "traffic": None, "kernel": "attn_tc_kernel",
                         "alg_flops_per_call": fl, "alg_bytes_per_call": by,
                         "hbm_gbs": by / (main_ms * 1e-3) / 1e9, "hbm_peak": hbm,
                         "peak_source": src, "main_kernel_ms": main_ms},
            "cpu_baseline": cpu,
            "e2e": {"value": e2e, "unit": "queries/s", "h2d_bytes_per_step": B * ATTN_H * ATTN_D * 4,
                    "d2h_bytes_per_step": B * ATTN_H * ATTN_D * 4},
            "gpu_launches": 2 * args.steps,
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    if dist:
        dist.barrier()
        dist.destroy_process_group()


# ------------------------------------------ config 5: whole-model decode ----
C5 = dict(hidden=4096, vocab=129280, n_heads=64, head_dim=512, rope_dim=64, q_lora=1024,
          o_groups=8, o_lora=1024, window=128, hc_mult=4, hc_iters=20, rms_eps=1e-6,
          hc_eps=1e-6, rope_theta=10000.0, experts=256, topk=6, inter=2048,
          index_heads=64, index_dim=128, index_topk=512, compress_rope_theta=160000.0,
          rope_factor=16.0, beta_fast=32.0, beta_slow=1.0, original_position=65536)


def c5_ratios(n_layers):
    """DeepSeek-V4-Flash's compress ratios: two sliding-window layers, then
    ratio 4 and ratio 128 alternating (21 and 20 of the 43 layers)."""
    return [0 if i < 2 else (4 if (i - 2) % 2 == 0 else 128) for i in range(n_layers)]
DECODE_METRIC = ("decode tok/s, batch 1, speculation off (config 5: DSV4-Flash shapes, "
                 "43 layers, 256+1 experts top-6, FP4 experts / FP8 attention)")


def decode_config(args, world):
    """The `config` of the decode line, the same in both arms."""
    c, n_layers = C5, args.decode_layers
    return {"workload": "config 5 batch-1 greedy decode, speculation off",
            "layers": n_layers, "hidden": c["hidden"], "vocab": c["vocab"],
            "heads": c["n_heads"], "head_dim": c["head_dim"],
            "experts": c["experts"], "topk": c["topk"], "moe_inter": c["inter"],
            "attention": ("DeepSeek-V4-Flash compress ratios: layers 0-1 sliding window "
                          "of 128, then ratio 4 (compressor + indexer, 64 heads x 128, "
                          "top-512 of the compressed rows) and ratio 128 alternating"
                          if args.decode_ratios == "dsv4" else
                          "sliding window of 128 on every layer (compress ratio 0)"),
            "prompt_positions": args.decode_prompt,
            "context": f"a {args.decode_prompt}-token greedy prompt decoded through the same "
                       "graph before timing (rings, compressor state and compressed rows in "
                       "place)",
            "weight_sets": f"{n_layers} layers cycle distinct random-init layer weight sets "
                           "of ~3.6 GB (two per kind of layer); every token reads a whole "
                           "model's bytes, none of it L2-resident",
            "graph": "one CUDA graph per token (argmax fed back on the device)",
            "parallelism": (f"ep{world} (token-parallel: one sequence per GPU, "
                            "experts split, slots exchanged over peer memory)"
                            if world > 1 else "ep1")}


def decode_bytes_per_token(c, n_layers, context=2048):
    """Algorithmic HBM bytes one greedy token reads: every layer's dense
    weights (FP8 projections with their [128x128] scales, BF16 wo_a, the HC
    mixes, the BF16 router), the shared expert, topk routed FP4 experts
    (codes + per-32 scales), the latent ring; a compressed layer's
    compressor projections (and for ratio 4 the indexer's query, weights and
    compressor projections, its compressed keys at `context` and the
    selected latent rows; for ratio 128 every compressed row); then the HC
    head and the BF16 vocab head."""
    H, I, hd, nh = c["hidden"], c["inter"], c["head_dim"], c["n_heads"]
    fp8 = lambda r, k: r * k + ((r + 127) // 128) * ((k + 127) // 128)  # noqa: E731
    mult = c["hc_mult"]
    dense = (fp8(c["q_lora"], H) + fp8(nh * hd, c["q_lora"]) + fp8(hd, H) +
             c["o_groups"] * c["o_lora"] * (nh * hd // c["o_groups"]) * 2 +
             fp8(H, c["o_groups"] * c["o_lora"]) +
             2 * (2 + mult) * mult * mult * H * 4 + c["experts"] * H * 2 +
             3 * fp8(I, H) + c["window"] * 584)
    expert = 3 * (I * H // 2 + I * H // 32)
    per_layer = dense + c["topk"] * expert
    ih, idim = c["index_heads"], c["index_dim"]
    comp = {0: 0,
            4: 2 * (2 * hd) * H * 2 + fp8(ih * idim, c["q_lora"]) + ih * H * 2 +
            2 * (2 * idim) * H * 2 + (context // 4) * idim * 4 +
            min(c["index_topk"], context // 4) * 584,
            128: 2 * hd * H * 2 + (context // 128) * 584}
    extra = sum(comp[r] for r in c5_ratios(n_layers))
    return n_layers * per_layer + extra + c["vocab"] * H * 2 + mult * mult * H * 4 + H * 2


def make_decode_set(torch, seed, dev, c, expert_range=None, ratio=0):
    """One random-init layer weight set at config-5 shapes (distributions as
    config 2: FP4 codes uniform, E8M0 lognormal(0, 0.5) rounded to powers of
    two, FP8 codes uniform over the finite values, BF16 N(0, 0.02), RMSNorm
    gains 1 + N(0, 0.02), HC parameters N(0, 0.02) with unit scales)."""
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    H, I, E, hd, nh = c["hidden"], c["inter"], c["experts"], c["head_dim"], c["n_heads"]
    mult = c["hc_mult"]
    mix = (2 + mult) * mult

    def u8(*shape):
        return torch.randint(0, 256, shape, dtype=torch.uint8, device=dev, generator=g)

    def e8m0(*shape):
        z = torch.randn(shape, device=dev, generator=g) * (0.5 / np.log(2.0))
        return (127 + torch.round(z)).clamp(0, 254).to(torch.uint8)

    def fp8(r, k):
        cd = torch.randint(0, 254, (r, k), dtype=torch.int32, device=dev, generator=g)
        cd = torch.where((cd & 0x7F) == 0x7F, cd - 1, cd).to(torch.uint8)
        return cd, e8m0((r + 127) // 128, (k + 127) // 128)

    def bf16(*shape, mean=0.0):
        return (mean + torch.randn(shape, device=dev, generator=g) * 0.02).to(
            torch.bfloat16).view(torch.uint16)

    def f32(*shape):
        return torch.randn(shape, device=dev, generator=g) * 0.02

    wq_a, wq_a_s = fp8(c["q_lora"], H)
    wq_b, wq_b_s = fp8(nh * hd, c["q_lora"])
    wkv, wkv_s = fp8(hd, H)
    wo_b, wo_b_s = fp8(H, c["o_groups"] * c["o_lora"])
    sh = {}
    for k, (r, cc) in (("1", (I, H)), ("3", (I, H)), ("2", (H, I))):
        sh["w" + k], sh["s" + k] = fp8(r, cc)
    n = (expert_range[1] - expert_range[0]) if expert_range else E  # experts held here
    moe = dict(hidden=H, moe_inter=I, n_experts=E, topk=c["topk"], route_scale=1.5,
               swiglu_limit=10, gate_w=bf16(E, H), bias=f32(E), tid2eid=None,
               w1=u8(n, I, H // 2), s1=e8m0(n, I, H // 32), w3=u8(n, I, H // 2),
               s3=e8m0(n, I, H // 32), w2=u8(n, H, I // 2), s2=e8m0(n, H, I // 32),
               shared=dict(fp8=True, **sh))
    ones3 = torch.ones(3, device=dev)
    comp = {"compress_ratio": ratio}
    if ratio:
        coff = 2 if ratio == 4 else 1
        comp.update(comp_wkv=bf16(coff * hd, H), comp_wgate=bf16(coff * hd, H),
                    comp_ape=f32(ratio, coff * hd), comp_norm=bf16(hd, mean=1.0))
        if ratio == 4:
            ih, idim = c["index_heads"], c["index_dim"]
            iw, iws = fp8(ih * idim, c["q_lora"])
            comp.update(idx_wq_b=iw, idx_wq_b_s=iws, idx_weights_proj=bf16(ih, H),
                        idx_comp_wkv=bf16(2 * idim, H), idx_comp_wgate=bf16(2 * idim, H),
                        idx_ape=f32(4, 2 * idim), idx_comp_norm=bf16(idim, mean=1.0))
    return dict(**comp, attn_norm=bf16(H, mean=1.0), ffn_norm=bf16(H, mean=1.0),
                hc_attn_fn=f32(mix, mult * H), hc_attn_scale=ones3, hc_attn_base=f32(mix),
                hc_ffn_fn=f32(mix, mult * H), hc_ffn_scale=ones3.clone(), hc_ffn_base=f32(mix),
                attn_sink=f32(nh), wq_a=wq_a, wq_a_s=wq_a_s, q_norm=bf16(c["q_lora"], mean=1.0),
                wq_b=wq_b, wq_b_s=wq_b_s, wkv=wkv, wkv_s=wkv_s, kv_norm=bf16(hd, mean=1.0),
                wo_a=bf16(c["o_groups"] * c["o_lora"], nh * hd // c["o_groups"]),
                wo_b=wo_b, wo_b_s=wo_b_s, moe=moe)


def cpu_reference_decode(n_layers=43, threads=None, warm=8, timed=8, kinds_mode="dsv4",
                         one_thread=None):
    """Per kind of layer in the model (compress ratio 0 / 4 / 128), the
    reference's decode of a one-layer checkpoint of that kind
    (cpu_reference_decode_one); per token = sum over the model's layers of
    their kind's layer time + the vocab head and the embedding. Returns
    (tok/s, threads, sample description, one-thread line or None) or None.
    one_thread = (warm, timed) also times every kind on one thread."""
    ratios = c5_ratios(n_layers) if kinds_mode == "dsv4" else [0] * n_layers
    per_kind, head_emb, samples, cores = {}, None, [], None
    per_kind1, head_emb1, samples1 = {}, None, []
    for r in sorted(set(ratios)):
        res = cpu_reference_decode_one(threads, warm, timed, ratio=r, one_thread=one_thread)
        if res is None:
            return None
        layer, he, cores, one = res
        per_kind[r] = layer
        head_emb = he
        samples.append(f"ratio {r}: {layer * 1e3:.1f} ms per layer")
        if one:
            per_kind1[r], head_emb1 = one
            samples1.append(f"ratio {r}: {one[0] * 1e3:.1f} ms per layer")
    per_token = sum(per_kind[r] for r in ratios) + head_emb
    line1 = None
    if one_thread:
        pt1 = sum(per_kind1[r] for r in ratios) + head_emb1
        line1 = {"value": 1.0 / pt1, "unit": "tok/s", "cores": 1,
                 "sample": (f"the same checkpoints, {one_thread[1]} timed tokens after "
                            f"{one_thread[0]} warm-up, 1 thread: {'; '.join(samples1)}; "
                            f"{head_emb1 * 1e3:.1f} ms head + embedding; per token "
                            f"extrapolated ({pt1:.2f} s)")}
    return 1.0 / per_token, cores, (
        f"dsv4_forward_token on one-layer config-5 random checkpoints in RAM (one per kind of "
        f"layer), {timed} timed tokens after {warm} warm-up from position 0, {cores} thread(s): "
        f"{'; '.join(samples)}; {head_emb * 1e3:.1f} ms head + embedding; per token extrapolated "
        f"to the {n_layers}-layer pattern ({per_token:.2f} s)"), line1


def cpu_reference_decode_one(threads=None, warm=8, timed=8, ratio=0, one_thread=None):
    """The reference engine's own decode step on the host cores
    (oracle/_ref/ref_decode_bench: dsv4_forward_token over a config-5-shaped
    random checkpoint of ONE layer of compress ratio `ratio`, written to
    RAM; a 43-layer checkpoint, ~156 GB, does not fit the host). Returns
    (seconds per layer, seconds of head + embedding per token, threads,
    one) - the head and the embedding split off with the engine's own
    profile counters; one = the same pair on one thread when one_thread =
    (warm, timed) is given, on the same checkpoint, else None - or None when
    the reference was not built here."""
    import shutil
    import tempfile
    exe = os.path.join(ROOT, "oracle", "_ref", "ref_decode_bench")
    if not os.path.exists(exe):
        return None
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import random_checkpoint
    threads = threads or host_threads()
    base = "/dev/shm" if os.path.isdir("/dev/shm") else None
    d = tempfile.mkdtemp(prefix="dsv4_c5_", dir=base)
    try:
        random_checkpoint.write(d, 1, c=dict(random_checkpoint.CONFIG5, ratios=[ratio]))

        def run(w, t, th):
            r = subprocess.run([exe, d, str(w), str(t), str(th)], capture_output=True,
                               text=True, timeout=1800)
            line = [ln for ln in r.stdout.splitlines() if ln.startswith("RESULT")]
            if r.returncode != 0 or not line:
                raise RuntimeError(r.stderr[-500:])
            f = line[-1].split()
            tok, total, head, emb = int(f[4]), float(f[6]), float(f[8]), float(f[10])
            return (total - head - emb) / tok, (head + emb) / tok

        layer, he = run(warm, timed, threads)
        one = run(one_thread[0], one_thread[1], 1) if one_thread else None
        return layer, he, threads, one
    finally:
        shutil.rmtree(d, ignore_errors=True)


def main_decode(args, rank, world, local):
    """--workload decode: config 5 batch-1 greedy decode. Under torchrun the
    MoE blocks are expert-parallel (rank r holds experts [r E/N, (r+1) E/N)
    of every layer) and token-parallel: each rank decodes its own sequence,
    attention and the dense weights replicated, and every layer's tokens are
    routed together and their expert slots exchanged over peer memory; N GPUs
    decode N sequences (weak scaling)."""
    import torch
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    import ctypes as C
    import dsv4cuda
    dsv4cuda.set_abort_on_error(False)
    dsv4cuda.init(local)
    c = dict(C5)
    n_layers = args.decode_layers
    ep = world > 1
    erange = (rank * c["experts"] // world, (rank + 1) * c["experts"] // world) if ep else None
    # distinct random-init layer weight sets per kind of layer, cycled so that
    # consecutive layers never share weights
    ratios = c5_ratios(n_layers) if args.decode_ratios == "dsv4" else [0] * n_layers
    kinds = sorted(set(ratios))
    per_kind = max(2, args.decode_sets // max(1, len(kinds)))
    sets_by = {r: [make_decode_set(torch, 500 + 10 * r + i, dev, c, erange, ratio=r)
                   for i in range(per_kind)] for r in kinds}
    sets = [st_ for r in kinds for st_ in sets_by[r]]
    seen = {r: 0 for r in kinds}
    layers, set_of = [], []  # layer i runs weight set sets[set_of[i]]
    for r in ratios:
        st_ = sets_by[r][seen[r] % per_kind]
        layers.append(st_)
        set_of.append(next(k for k, x in enumerate(sets) if x is st_))
        seen[r] += 1
    g = torch.Generator(device=dev)
    g.manual_seed(7)
    model = dict(embed=(torch.randn(c["vocab"], c["hidden"], device=dev, generator=g) * 0.02)
                 .to(torch.bfloat16).view(torch.uint16),
                 head=(torch.randn(c["vocab"], c["hidden"], device=dev, generator=g) * 0.02)
                 .to(torch.bfloat16).view(torch.uint16),
                 norm=(1.0 + torch.randn(c["hidden"], device=dev, generator=g) * 0.02)
                 .to(torch.bfloat16).view(torch.uint16),
                 hc_head_fn=torch.randn(c["hc_mult"], c["hc_mult"] * c["hidden"], device=dev,
                                        generator=g) * 0.02,
                 hc_head_base=torch.randn(c["hc_mult"], device=dev, generator=g) * 0.02,
                 hc_head_scale=torch.ones(1, device=dev))
    prompt, gen = args.decode_prompt, args.steps
    n_e2e = max(32, args.steps // 2)  # host-call tokens after the timed graph replays
    spec_steps = 0 if (args.no_spec or world > 1) else max(10, args.steps // 4)
    spec_warm = 3
    cfg = dict(hidden=c["hidden"], n_layers=n_layers, vocab=c["vocab"], n_heads=c["n_heads"],
               head_dim=c["head_dim"], rope_dim=c["rope_dim"], q_lora=c["q_lora"],
               o_groups=c["o_groups"], o_lora=c["o_lora"], window=c["window"],
               hc_mult=c["hc_mult"], hc_iters=c["hc_iters"], rms_eps=c["rms_eps"],
               hc_eps=c["hc_eps"], rope_theta=c["rope_theta"],
               max_context=prompt + 4 * (gen + args.warmup) + n_e2e + 32 +
               (spec_steps + spec_warm + 1) * args.spec_rows,
               index_heads=c["index_heads"], index_dim=c["index_dim"],
               index_topk=c["index_topk"], compress_rope_theta=c["compress_rope_theta"],
               rope_factor=c["rope_factor"], beta_fast=c["beta_fast"], beta_slow=c["beta_slow"],
               original_position=c["original_position"],
               moe=dict(hidden=c["hidden"], moe_inter=c["inter"], n_experts=c["experts"],
                        topk=c["topk"], swiglu_limit=10, route_scale=1.5,
                        shared_kind=dsv4cuda.SHARED_FP8, hash_vocab=0))
    dec = dsv4cuda.Decoder(cfg, model, layers)
    ipc_own, ipc_peers, moe_ep = [], [], []
    if ep:
        # one EP-attached MoE layer per weight set, its exchange buffer mapped
        # into every rank
        moe_ep = [dsv4cuda.MoeLayer(st_["moe"], max_tokens=world, device=True,
                                    expert_range=erange) for st_ in sets]
        handles = []
        for L in moe_ep:
            addr, hnd = dsv4cuda.ipc_alloc(L.ep_buffer_bytes())
            ipc_own.append(addr)
            handles.append(hnd)
        all_h = [None] * world
        dist.all_gather_object(all_h, handles)
        for li, L in enumerate(moe_ep):
            addrs = []
            for r in range(world):
                if r == rank:
                    addrs.append(ipc_own[li])
                else:
                    a_ = dsv4cuda.ipc_open(all_h[r][li])
                    ipc_peers.append(a_)
                    addrs.append(a_)
            L.ep_attach(rank, world, addrs)
        dist.barrier()
        dec.set_moe_layers([moe_ep[set_of[i]] for i in range(n_layers)])
    lib = dsv4cuda.lib
    h = dec.handle
    _, _, _, am_slot = dec.slots()
    pos = torch.full((1,), 0, dtype=torch.int32, device=dev)
    tok = torch.full((1,), 1, dtype=torch.int32, device=dev)
    stream = torch.cuda.Stream(device=dev)
    with torch.cuda.stream(stream):  # one eager step: its argmax seeds the greedy chain
        dec.step_device(tok, pos, stream.cuda_stream)
        pos.add_(1)
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        cs = torch.cuda.current_stream()
        if lib.dsv4cuda_decoder_step_device(h, C.c_void_p(am_slot), C.c_void_p(pos.data_ptr()),
                                            C.c_void_p(cs.cuda_stream)) != 0:
            raise RuntimeError(lib.dsv4cuda_decoder_last_error().decode())
        pos.add_(1)
    # the context: a greedy prompt through the same graph up to position
    # prompt - warmup (every ring, compressor state, compressed row and
    # indexer key of a 2048-token context is in place), then the warm-up
    with torch.cuda.stream(stream):
        for _ in range(prompt - 1):
            graph.replay()
    torch.cuda.synchronize()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    def decode_window():
        """K greedy steps between a barrier + synchronize on both sides; the
        device time, max over ranks."""
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        ev0 = torch.cuda.Event(enable_timing=True)
        ev1 = torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            ev0.record(stream)
            for _ in range(args.steps):
                graph.replay()
            ev1.record(stream)
        torch.cuda.synchronize()
        if dist:
            dist.barrier()
        w = ev0.elapsed_time(ev1)
        if dist:
            t = torch.tensor([w], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            w = float(t.item())
        return w

    # the reported window is the first; two more give the spread
    windows = [decode_window() for _ in range(3)]
    clk = clocks.stop()
    ms = windows[0]
    ms_tok = ms / args.steps
    value = world * 1e3 / ms_tok
    # e2e: the public host-argument call, greedy on the host, logits to host
    e2e = None
    if not args.no_e2e:
        logits = np.empty(c["vocab"], np.float32)
        nxt = C.c_int()
        p0 = int(pos.item())
        t0v = 1
        for i in range(2):  # eager step, then the call that captures its graph
            lib.dsv4cuda_decoder_forward_token(h, t0v, p0 + i, logits.ctypes.data, C.byref(nxt))
            t0v = nxt.value
        t0 = time.perf_counter()
        for i in range(n_e2e):
            if lib.dsv4cuda_decoder_forward_token(h, t0v, p0 + 2 + i, logits.ctypes.data,
                                                  C.byref(nxt)) != 0:
                raise RuntimeError(lib.dsv4cuda_decoder_last_error().decode())
            t0v = nxt.value
        el = time.perf_counter() - t0
        if dist:
            tt = torch.tensor([el], device=dev)
            dist.all_reduce(tt, op=dist.ReduceOp.MAX)
            el = float(tt.item())
        e2e = world * n_e2e / el
    # batch 1 at N GPUs (strong scaling): every rank decodes the same
    # sequence from cleared rings; each rank routes the token, runs its own
    # experts and the slots are exchanged (a second set of EP layers with
    # their own exchange buffers)
    batch1 = None
    p_next = (p0 + 2 + n_e2e) if e2e is not None else int(pos.item())
    rep_own, rep_peers, moe_rep = [], [], []
    if ep and not args.no_batch1:
        moe_rep = [dsv4cuda.MoeLayer(st_["moe"], max_tokens=world, device=True,
                                     expert_range=erange) for st_ in sets]
        handles = []
        for L in moe_rep:
            addr, hnd = dsv4cuda.ipc_alloc(L.ep_buffer_bytes())
            rep_own.append(addr)
            handles.append(hnd)
        all_h = [None] * world
        dist.all_gather_object(all_h, handles)
        for li, L in enumerate(moe_rep):
            addrs = []
            for r in range(world):
                if r == rank:
                    addrs.append(rep_own[li])
                else:
                    a_ = dsv4cuda.ipc_open(all_h[r][li])
                    rep_peers.append(a_)
                    addrs.append(a_)
            L.ep_attach(rank, world, addrs)
        dist.barrier()
        dec.set_moe_layers([moe_rep[set_of[i]] for i in range(n_layers)])
        dec.set_ep_replicated(True)
        # every rank already holds the same context (same weights, the same
        # greedy tokens); continue after the positions used so far
        pos.fill_(p_next)
        tok.fill_(1)
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            dec.step_device(tok, pos, stream.cuda_stream)
            pos.add_(1)
        stream.synchronize()
        rgraph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(rgraph, stream=stream):
            cs = torch.cuda.current_stream()
            if lib.dsv4cuda_decoder_step_device(h, C.c_void_p(am_slot), C.c_void_p(pos.data_ptr()),
                                                C.c_void_p(cs.cuda_stream)) != 0:
                raise RuntimeError(lib.dsv4cuda_decoder_last_error().decode())
            pos.add_(1)
        with torch.cuda.stream(stream):
            for _ in range(args.warmup):
                rgraph.replay()
        torch.cuda.synchronize()
        dist.barrier()
        torch.cuda.synchronize()
        r0 = torch.cuda.Event(enable_timing=True)
        r1 = torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            r0.record(stream)
            for _ in range(args.steps):
                rgraph.replay()
            r1.record(stream)
        torch.cuda.synchronize()
        dist.barrier()
        t = torch.tensor([r0.elapsed_time(r1)], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        rms = float(t.item()) / args.steps
        last = torch.tensor([int(dec.read()[1])], device=dev)
        lo, hi = last.clone(), last.clone()
        dist.all_reduce(lo, op=dist.ReduceOp.MIN)
        dist.all_reduce(hi, op=dist.ReduceOp.MAX)
        batch1 = {"metric": "decode tok/s, batch 1, speculation off (one sequence on all "
                            f"{world} GPUs: experts split, attention and dense layers "
                            "replicated, slots exchanged over peer memory)",
                  "value": 1e3 / rms, "unit": "tok/s", "ms_per_step": rms,
                  "scaling": "strong", "steps": args.steps,
                  "ranks_agree_on_last_token": bool(int(lo.item()) == int(hi.item()))}
        torch.cuda.synchronize()
        rgraph.reset()
    # speculation on: verify steps of a draft chain (config 4's form: the
    # pending token plus k uniform random drafts), each one CUDA graph of
    # draft_random -> verify (all rows layer-major) -> greedy acceptance +
    # commit, the next step's pending token and position left on the device
    spec = None
    if spec_steps:
        n_rows = args.spec_rows
        # the batched verify runs sliding-window layers; with compressed
        # layers in the model it is measured on a decoder of the same shapes
        # whose layers are all window layers (the window weight sets), and
        # compared with that decoder's own one-token step
        window_only = not any(ratios)
        sdec, ms_ref = dec, ms_tok
        if not window_only:
            wsets = sets_by.get(0) or [make_decode_set(torch, 900, dev, c, erange)]
            sdec = dsv4cuda.Decoder(cfg, model, [wsets[i % len(wsets)] for i in range(n_layers)])
            p_now, pend = prompt, 1
            wtok = torch.full((1,), 1, dtype=torch.int32, device=dev)
            wpos = torch.full((1,), prompt, dtype=torch.int32, device=dev)
            with torch.cuda.stream(stream):
                sdec.step_device(wtok, wpos, stream.cuda_stream)
            stream.synchronize()
            wgraph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(wgraph, stream=stream):
                sdec.step_device(wtok, wpos, torch.cuda.current_stream().cuda_stream)
            with torch.cuda.stream(stream):
                for _ in range(args.warmup):
                    wgraph.replay()
            torch.cuda.synchronize()
            w0 = torch.cuda.Event(enable_timing=True)
            w1 = torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(stream):
                w0.record(stream)
                for _ in range(spec_steps):
                    wgraph.replay()
                w1.record(stream)
            torch.cuda.synchronize()
            ms_ref = w0.elapsed_time(w1) / spec_steps
            wgraph.reset()
        else:
            p_now = p_next + (2 * args.steps + args.warmup + 2 if batch1 is not None else 0)
            _, pend = dec.read()  # the last step's greedy token is the pending row
        first = [pend] + [1] * (n_rows - 1)
        sdec.verify(first, p_now)  # eager: fills the verify slots, one-time set-up
        sdec.accept_greedy(n_rows, stream.cuda_stream)
        stream.synchronize()
        sgraph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(sgraph, stream=stream):
            cs = torch.cuda.current_stream().cuda_stream
            sdec.draft_random(n_rows, cs)
            sdec.verify_device(n_rows, cs)
            sdec.accept_greedy(n_rows, cs)
        with torch.cuda.stream(stream):
            for _ in range(spec_warm):
                sgraph.replay()
        torch.cuda.synchronize()
        st0 = sdec.verify_stats()
        clocks_s = ClockSampler(local)
        clocks_s.start()
        time.sleep(0.2)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(spec_steps):
                sgraph.replay()
            e1.record(stream)
        torch.cuda.synchronize()
        sms = e0.elapsed_time(e1)
        clk_s = clocks_s.stop()
        st1 = sdec.verify_stats()
        emitted, accepted, vsteps = (st1[i] - st0[i] for i in range(3))
        sgraph.reset()
        if sdec is not dec:
            sdec.close()
        spec = {"metric": "decode tok/s, batch 1, speculation on (config 4 form: pending token "
                          f"+ {n_rows - 1} uniform random drafts per verify step, greedy "
                          "acceptance, config 5 model)",
                "value": emitted / (sms * 1e-3), "unit": "tok/s",
                "ms_per_verify_step": sms / vsteps, "verify_steps": vsteps,
                "rows_per_step": n_rows, "tokens_per_step": emitted / vsteps,
                "drafts_accepted_per_step": accepted / vsteps,
                "verified_rows_per_s": n_rows * vsteps / (sms * 1e-3),
                "tok_s_if_every_draft_accepted": n_rows * vsteps / (sms * 1e-3),
                "decode_step_ms_same_layers": ms_ref,
                "verify_vs_decode_step_cost": (sms / vsteps) / ms_ref,
                "break_even_accepted_drafts": (sms / vsteps) / ms_ref - 1.0,
                "layers": ("the benchmark's layers" if window_only else
                           "every layer a sliding-window layer (the batched verify covers "
                           "compress-ratio-0 layers); the costs compare with that decoder's "
                           "own one-token step (decode_step_ms_same_layers)"),
                "clocks": clk_s,
                "note": "uniform random drafts are almost never accepted, so this is the "
                        "floor; a drafter's gain is tokens_per_step x this step rate"}
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        try:
            res = cpu_reference_decode(n_layers, kinds_mode=args.decode_ratios,
                                       one_thread=(2, 4))
            if res:
                cpu = {"value": res[0], "unit": "tok/s", "cores": res[1], "kind": "reference",
                       "sample": res[2], "extrapolated": True, "one_thread": res[3]}
        except Exception as exc:  # report, do not hide
            cpu = {"value": None, "unit": "tok/s", "cores": 0, "kind": "reference",
                   "sample": f"failed: {exc}"}
    hbm, _, src = peaks()
    alg = decode_bytes_per_token(c, n_layers)
    achieved = alg / (ms_tok * 1e-3) / 1e9
    kernels = lib.dsv4cuda_decoder_step_kernels(h)
    # the expert-GEMV half of the metric: the config 2 MoE layer workload in a
    # child process (its routed FP4 GEMV against the HBM roofline)
    moe_sub = None
    if rank == 0 and world == 1 and not args.no_moe_sub:
        r = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--workload", "moe",
                            "--steps", "200", "--warmup", "20", "--no-cpu", "--no-attn-sweep"],
                           capture_output=True, text=True, timeout=900)
        ln = [x for x in r.stdout.splitlines() if x.startswith("{")]
        if r.returncode == 0 and ln:
            m = json.loads(ln[-1])
            moe_sub = {"metric": m["metric"], "value": m["value"], "unit": m["unit"],
                       "ms_per_step": m["ms_per_step"], "roofline": m["roofline"],
                       "e2e": m["e2e"], "clocks": m["clocks"]}
        else:
            moe_sub = {"failed": r.stderr[-500:]}
    if rank == 0:
        line = {
            "metric": DECODE_METRIC, "value": value, "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_tok,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "fp4e2m1/fp8e4m3 weights, bf16 activations, f32 accumulate",
            "data": "synthetic (random-init weights with the checkpoint's formats)",
            "config": decode_config(args, world),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                         "frac": achieved / hbm, "traffic": None,
                         "alg_bytes_per_token": alg, "peak_source": src,
                         "note": "whole-step bytes / whole-step time (every kernel of the "
                                 "token, launch gaps included)"},
            "cpu_baseline": cpu,
            "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": 8,
                    "d2h_bytes_per_step": c["vocab"] * 4 + 4},
            "gpu_launches": kernels * args.steps, "clocks": clk,
            "repeat_windows": {"n": len(windows), "steps_each": args.steps,
                               "tok_s": [world * 1e3 * args.steps / w for w in windows],
                               "spread_pct": 100.0 * (max(windows) - min(windows)) / min(windows)},
            "spec_on": spec,
            "batch1_strong_scaling": batch1,
            "expert_gemv_config2": moe_sub,
        }
        print(json.dumps(line), flush=True)
    torch.cuda.synchronize()
    graph.reset()
    dec.close()
    if ep:
        # every rank stops touching peer memory before any buffer is unmapped
        dist.barrier()
        for a_ in ipc_peers + rep_peers:
            dsv4cuda.ipc_close(a_)
        dist.barrier()
        for a_ in ipc_own + rep_own:
            dsv4cuda.ipc_free(a_)
        for L in moe_ep + moe_rep:
            L.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
