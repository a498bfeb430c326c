"""Benchmark config 1 (the tiny models) through the drop-in boundary: the
reference engine's own host code, compiled from its sources into
oracle/_ref, with libdsv4_cuda.so preloaded so that every kernel call the
engine makes to its exported GEMV / quantiser symbols runs on the GPU.

The engine is built as a shared library with -fPIC, so its calls to its own
exported kernels go through the PLT and resolve to the first definition in
the process: the preloaded library's. DSV4CUDA_DROPIN_REPORT=1 makes the
library print how many calls it served, which proves the swap happened.

T0 is the reference's own gate: its unmodified tests/unit/test_dsv4_model.c
over its checked-in tiny fixture, 130 positions across the ratio-4 and
ratio-128 compressed-attention boundaries, exact equality with the
independent Python oracle's logits (test_dsv4_model.c:132-151). T1 is a
BASELINE-config-1-shaped random checkpoint (tests/golden/make_tiny_t1.py):
a 32-token prompt prefilled layer-major, then 16 greedy tokens; the run on
the GPU kernels must produce the same tokens and the same logits, bit for
bit, as the plain reference.
"""
import os
import re
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REFDIR = os.path.join(ROOT, "oracle", "_ref")
LIB = os.path.join(ROOT, "deepseek-v4-flash-0731-in-c_b200", "lib", "libdsv4_cuda.so")
sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))


def _need(path):
    if not os.path.exists(path):
        pytest.skip(f"{os.path.relpath(path, ROOT)} not built here (needs the reference sources)")


def run(cmd, gpu, timeout=600):
    env = dict(os.environ)
    env.pop("LD_PRELOAD", None)
    if gpu:
        env["LD_PRELOAD"] = LIB
        env["DSV4CUDA_DROPIN_REPORT"] = "1"
    return subprocess.run(cmd, cwd=REFDIR, env=env, capture_output=True, text=True,
                          timeout=timeout)


def served(stderr):
    m = re.search(r"drop-in calls: fp4=(\d+) fp8=(\d+) bf16=(\d+) quant=(\d+)", stderr)
    assert m, stderr[-2000:]
    return dict(zip(("fp4", "fp8", "bf16", "quant"), (int(v) for v in m.groups())))


def t1_checkpoint(tmp_path):
    import make_tiny_t1
    d = str(tmp_path / "t1")
    make_tiny_t1.write(d, seed=0)
    return d, [str(i) for i in make_tiny_t1.prompt_ids(seed=0, n=32)]


def test_t0_reference_gate_plain():
    """The reference's own tiny-model test passes on the plain engine here
    (the gate the GPU run below must also pass)."""
    exe = os.path.join(REFDIR, "test_dsv4_model")
    _need(exe)
    r = run([exe, "tiny_dsv4"], gpu=False)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    assert "maxdiff=0.000000" in r.stdout


def test_t1_reference_decode_plain(tmp_path):
    exe = os.path.join(REFDIR, "tiny_decode")
    _need(exe)
    d, ids = t1_checkpoint(tmp_path)
    r = run([exe, d, "16", *ids], gpu=False)
    assert r.returncode == 0, r.stderr[-2000:]
    assert len([ln for ln in r.stdout.splitlines() if ln.startswith("POS")]) == 16


@pytest.mark.gpu
def test_t0_reference_gate_on_gpu_kernels():
    exe = os.path.join(REFDIR, "test_dsv4_model")
    _need(exe)
    r = run([exe, "tiny_dsv4"], gpu=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "maxdiff=0.000000" in r.stdout and "PASS" in r.stdout
    n = served(r.stderr)
    assert n["fp4"] > 0 and n["fp8"] > 0 and n["quant"] > 0, n
    print("T0 on the GPU kernels:", n)


@pytest.mark.gpu
def test_t1_greedy_tokens_and_logits_bit_exact(tmp_path):
    exe = os.path.join(REFDIR, "tiny_decode")
    _need(exe)
    d, ids = t1_checkpoint(tmp_path)
    plain = run([exe, d, "16", *ids], gpu=False)
    assert plain.returncode == 0, plain.stderr[-2000:]
    gpu = run([exe, d, "16", *ids], gpu=True)
    assert gpu.returncode == 0, gpu.stderr[-3000:]
    n = served(gpu.stderr)
    assert n["fp4"] > 0 and n["fp8"] > 0, n
    want = [ln for ln in plain.stdout.splitlines() if ln.startswith("POS")]
    got = [ln for ln in gpu.stdout.splitlines() if ln.startswith("POS")]
    assert len(want) == 16 and len(got) == 16
    tw = [ln.split()[3] for ln in want]
    tg = [ln.split()[3] for ln in got]
    assert tg == tw, (tg, tw)          # greedy tokens bit-exact
    assert got == want                 # every logit bit-identical
    print("T1 greedy tokens:", " ".join(tg), "| GPU calls:", n)
