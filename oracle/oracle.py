"""ctypes bindings for the CPU checker libraries (test infrastructure only).

``Oracle`` wraps ``_build/libdsv4_oracle.so`` (the C restatement in
dsv4_oracle.c) and ``Ref`` wraps ``_ref/libdsv4_ref.so`` (the reference
engine compiled from its own sources by oracle/Makefile). Both expose the
same numpy-level methods, so a test can run one input through both and
compare bytes. Only tests/, __graft_entry__.smoke() and bench.py's CPU
baseline import this module; the product library never does.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "libdsv4_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libdsv4_ref.so")
REFCLI_SO = os.path.join(HERE, "_ref", "libdsv4_refcli.so")

f32p = C.POINTER(C.c_float)
u8p = C.POINTER(C.c_uint8)
u16p = C.POINTER(C.c_uint16)
i32p = C.POINTER(C.c_int)
i64p = C.POINTER(C.c_int64)


def _p(a, t):
    if a is None:
        return None
    return a.ctypes.data_as(t)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def build_oracle():
    """Compile the C restatement (and the reference, where its sources are)."""
    subprocess.run(["make", "-s", "-C", HERE], check=True)


def _ptr_array(arrs, t):
    arr_t = t * len(arrs)
    return arr_t(*[a.ctypes.data_as(t) for a in arrs])


class _Lib:
    """Shared numpy-level wrappers over a GEMV/quant symbol family."""

    def __init__(self, path, prefix):
        self.lib = C.CDLL(path)
        self.prefix = prefix

    def _fn(self, name):
        return getattr(self.lib, self.prefix + name)

    # ---- quant
    def quant_fp8_codes(self, x):
        x = _f32(x)
        n = x.size
        qx = np.empty(n, np.float32)
        qs = np.empty((n + 127) // 128, np.float32)
        self._fn("quant_fp8_codes")(_p(qx, f32p), _p(qs, f32p), _p(x, f32p), n)
        return qx, qs

    # ---- GEMVs
    def gemv_bf16(self, x, W, round_out=1):
        x = _f32(x)
        out, inn = W.shape
        y = np.empty(out, np.float32)
        self._fn("gemv_bf16")(_p(y, f32p), _p(x, f32p), _p(W, u16p), inn, out, round_out)
        return y

    def gemv_bf16_batch(self, xs, W, round_out=1):
        out, inn = W.shape
        xs = [_f32(x) for x in xs]
        ys = [np.empty(out, np.float32) for _ in xs]
        self._fn("gemv_bf16_batch")(_ptr_array(ys, f32p), _ptr_array(xs, f32p), len(xs),
                                    _p(W, u16p), inn, out, round_out)
        return np.stack(ys)

    def gemv_fp8_q(self, qx, qs, W, S, round_out=1):
        out, inn = W.shape
        y = np.empty(out, np.float32)
        self._fn("gemv_fp8_q")(_p(y, f32p), _p(_f32(qx), f32p), _p(_f32(qs), f32p),
                               _p(W, u8p), _p(S, u8p), inn, out, round_out)
        return y

    def gemv_fp8_batch_q(self, qxs, qss, W, S, round_out=1):
        out, inn = W.shape
        qxs = [_f32(a) for a in qxs]
        qss = [_f32(a) for a in qss]
        ys = [np.empty(out, np.float32) for _ in qxs]
        self._fn("gemv_fp8_batch_q")(_ptr_array(ys, f32p), _ptr_array(qxs, f32p),
                                     _ptr_array(qss, f32p), len(qxs), _p(W, u8p), _p(S, u8p),
                                     inn, out, round_out)
        return np.stack(ys)

    def gemv_fp8_pair_q(self, qx, qs, W0, S0, W1, S1):
        out, inn = W0.shape
        y0 = np.empty(out, np.float32)
        y1 = np.empty(out, np.float32)
        self._fn("gemv_fp8_pair_q")(_p(y0, f32p), _p(y1, f32p), _p(_f32(qx), f32p),
                                    _p(_f32(qs), f32p), _p(W0, u8p), _p(S0, u8p),
                                    _p(W1, u8p), _p(S1, u8p), inn, out)
        return y0, y1

    def gemv_fp4_q(self, qx, qs, W, S, inn):
        rows = W.shape[0]
        y = np.empty(rows, np.float32)
        self._fn("gemv_fp4_q")(_p(y, f32p), _p(_f32(qx), f32p), _p(_f32(qs), f32p),
                               _p(W, u8p), _p(S, u8p), inn, rows)
        return y

    def gemv_fp4_batch_q(self, qxs, qss, W, S, inn):
        rows = W.shape[0]
        qxs = [_f32(a) for a in qxs]
        qss = [_f32(a) for a in qss]
        ys = [np.empty(rows, np.float32) for _ in qxs]
        self._fn("gemv_fp4_batch_q")(_ptr_array(ys, f32p), _ptr_array(qxs, f32p),
                                     _ptr_array(qss, f32p), len(qxs), _p(W, u8p), _p(S, u8p),
                                     inn, rows)
        return np.stack(ys)

    def gemv_fp4_pair_q(self, qx, qs, W0, S0, W1, S1, inn):
        rows = W0.shape[0]
        y0 = np.empty(rows, np.float32)
        y1 = np.empty(rows, np.float32)
        self._fn("gemv_fp4_pair_q")(_p(y0, f32p), _p(y1, f32p), _p(_f32(qx), f32p),
                                    _p(_f32(qs), f32p), _p(W0, u8p), _p(S0, u8p),
                                    _p(W1, u8p), _p(S1, u8p), inn, rows)
        return y0, y1


class Oracle(_Lib):
    """The C restatement (always buildable with gcc)."""

    def __init__(self):
        if not os.path.exists(ORACLE_SO):
            build_oracle()
        super().__init__(ORACLE_SO, "orc_")
        L = self.lib
        L.orc_f32_to_bf16.restype = C.c_uint16
        L.orc_f32_to_bf16.argtypes = [C.c_float]
        for n in ("orc_bf16r", "orc_round_e4m3", "orc_sqrt_softplus"):
            getattr(L, n).restype = C.c_float
            getattr(L, n).argtypes = [C.c_float]
        for n in ("orc_e4m3", "orc_e8m0"):
            getattr(L, n).restype = C.c_float
            getattr(L, n).argtypes = [C.c_uint8]
        L.orc_xorshift_fill_u8.restype = C.c_uint64
        L.orc_xorshift_fill_u8.argtypes = [u8p, C.c_int64, C.c_uint64, C.c_int]
        L.orc_xorshift_next_many.restype = C.c_uint64
        L.orc_xorshift_next_many.argtypes = [C.POINTER(C.c_uint64), C.c_int64, C.c_uint64]

    def f32_to_bf16(self, f):
        return self.lib.orc_f32_to_bf16(f)

    def bf16r(self, f):
        return self.lib.orc_bf16r(f)

    def e4m3(self, c):
        return self.lib.orc_e4m3(c)

    def e8m0(self, c):
        return self.lib.orc_e8m0(c)

    def round_e4m3(self, v):
        return self.lib.orc_round_e4m3(v)

    def sqrt_softplus(self, z):
        return self.lib.orc_sqrt_softplus(z)

    def act_quant_inplace(self, x, group, mode):
        x = _f32(x).copy()
        self.lib.orc_act_quant_inplace(_p(x, f32p), x.size, group, mode)
        return x

    def xs_fill_u8(self, n, state, mod=0):
        out = np.empty(n, np.uint8)
        state = self.lib.orc_xorshift_fill_u8(_p(out, u8p), n, state, mod)
        return out, state

    def xs_next_many(self, n, state):
        out = np.empty(n, np.uint64)
        state = self.lib.orc_xorshift_next_many(out.ctypes.data_as(C.POINTER(C.c_uint64)), n, state)
        return out, state

    def router_moe(self, x, gate, bias, topk, route_scale, tid2eid=None, token_id=0):
        ne, hid = gate.shape
        idx = np.empty(topk, np.int32)
        wt = np.empty(topk, np.float32)
        score = np.empty(ne, np.float32)
        self.lib.orc_router_moe(_p(idx, i32p), _p(wt, f32p), _p(score, f32p), _p(_f32(x), f32p),
                                _p(gate, u16p), _p(bias, f32p), _p(tid2eid, i64p),
                                C.c_int(token_id), hid, ne, topk, C.c_float(route_scale))
        return idx, wt, score

    def router_public(self, x, gate, bias, topk, route_scale, tid2eid=None, token_id=0):
        ne, hid = gate.shape
        idx = np.empty(topk, np.int32)
        wt = np.empty(topk, np.float32)
        self.lib.orc_router_public(_p(idx, i32p), _p(wt, f32p), _p(_f32(x), f32p),
                                   _p(gate, u16p), _p(bias, f32p), _p(tid2eid, i64p),
                                   C.c_int(token_id), hid, ne, topk,
                                   C.c_int(1 if tid2eid is not None else 0), C.c_float(route_scale))
        return idx, wt

    def swiglu_quant(self, gate, up, limit, weight):
        n = gate.size
        y = np.empty(n, np.float32)
        qy = np.empty(n, np.float32)
        qs = np.empty((n + 127) // 128, np.float32)
        self.lib.orc_swiglu_quant(_p(y, f32p), _p(qy, f32p), _p(qs, f32p),
                                  _p(_f32(gate), f32p), _p(_f32(up), f32p), n,
                                  C.c_int(limit), C.c_float(weight))
        return y, qy, qs

    def rope_inv(self, x, cosv, sinv):
        """x [heads][d] (copied), cos/sin [n]: inverse RoPE on the last 2n dims."""
        x = np.array(x, dtype=np.float32, copy=True)
        c, s = _f32(cosv), _f32(sinv)
        self.lib.orc_rope_inv(_p(x, f32p), x.shape[0], x.shape[1], _p(c, f32p), _p(s, f32p),
                              c.size)
        return x

    def sparse_attn(self, q, kv, sink, idx, scale):
        H, d = q.shape
        o = np.empty((H, d), np.float32)
        idx = np.ascontiguousarray(idx, dtype=np.int32)
        self.lib.orc_sparse_attn(_p(o, f32p), _p(_f32(q), f32p), _p(_f32(kv), f32p),
                                 _p(_f32(sink), f32p), _p(idx, i32p), idx.size, H, d,
                                 C.c_float(scale))
        return o

    def expert_forward_fp4(self, qx, qs, layer, e, weight):
        """Routed expert e of `layer` for one token (expert_forward_l1/l2)."""
        hid, mi = layer["hidden"], layer["moe_inter"]
        ex = _OrcFp4Expert(*[_p(np.ascontiguousarray(layer[n][e]), u8p)
                             for n in ("w1", "s1", "w3", "s3", "w2", "s2")])
        out = np.empty(hid, np.float32)
        self.lib.orc_expert_forward_fp4(_p(out, f32p), _p(_f32(qx), f32p), _p(_f32(qs), f32p),
                                        C.byref(ex), hid, mi, layer["swiglu_limit"],
                                        C.c_float(weight))
        return out

    def shared_forward(self, qx, qs, layer):
        """The layer's shared expert for one token (zeros when it has none)."""
        hid, mi = layer["hidden"], layer["moe_inter"]
        out = np.zeros(hid, np.float32)
        sh = layer.get("shared")
        if sh is None:
            return out
        ex_t = _OrcFp8Expert if sh["fp8"] else _OrcFp4Expert
        ex = ex_t(*[_p(np.ascontiguousarray(sh[n]), u8p)
                    for n in ("w1", "s1", "w3", "s3", "w2", "s2")])
        if sh["fp8"]:
            self.lib.orc_shared_forward_fp8(_p(out, f32p), _p(_f32(qx), f32p), _p(_f32(qs), f32p),
                                            C.byref(ex), hid, mi, layer["swiglu_limit"])
        else:
            self.lib.orc_expert_forward_fp4(_p(out, f32p), _p(_f32(qx), f32p), _p(_f32(qs), f32p),
                                            C.byref(ex), hid, mi, layer["swiglu_limit"],
                                            C.c_float(1.0))
        return out

    def moe_forward(self, layer, x, token_id=0):
        """layer: dict from make_moe_layer (numpy weights)."""
        out = np.empty(layer["hidden"], np.float32)
        topk = layer["topk"]
        idx = np.empty(topk, np.int32)
        wt = np.empty(topk, np.float32)
        L = _OrcMoeLayer.from_dict(layer)
        self.lib.orc_moe_forward(_p(out, f32p), _p(idx, i32p), _p(wt, f32p), C.byref(L),
                                 _p(_f32(x), f32p), C.c_int(token_id))
        return out, idx, wt


class _OrcFp8Expert(C.Structure):
    _fields_ = [(n, u8p) for n in ("w1", "s1", "w3", "s3", "w2", "s2")]


class _OrcFp4Expert(C.Structure):
    _fields_ = [(n, u8p) for n in ("w1", "s1", "w3", "s3", "w2", "s2")]


class _OrcMoeLayer(C.Structure):
    _fields_ = [("hidden", C.c_int), ("moe_inter", C.c_int), ("n_experts", C.c_int),
                ("topk", C.c_int), ("swiglu_limit", C.c_int), ("route_scale", C.c_float),
                ("gate_w", u16p), ("bias", f32p), ("tid2eid", i64p),
                ("w1", u8p), ("s1", u8p), ("w3", u8p), ("s3", u8p), ("w2", u8p), ("s2", u8p),
                ("has_shared", C.c_int), ("shared_fp8", C.c_int),
                ("shared8", _OrcFp8Expert), ("shared4", _OrcFp4Expert)]

    @classmethod
    def from_dict(cls, d):
        L = cls()
        L.hidden, L.moe_inter, L.n_experts, L.topk = d["hidden"], d["moe_inter"], d["n_experts"], d["topk"]
        L.swiglu_limit = d["swiglu_limit"]
        L.route_scale = d["route_scale"]
        L.gate_w = _p(d["gate_w"], u16p)
        L.bias = _p(d.get("bias"), f32p)
        L.tid2eid = _p(d.get("tid2eid"), i64p)
        for n in ("w1", "s1", "w3", "s3", "w2", "s2"):
            setattr(L, n, _p(d[n], u8p))
        sh = d.get("shared")
        L.has_shared = 1 if sh is not None else 0
        if sh is not None:
            L.shared_fp8 = 1 if sh["fp8"] else 0
            tgt = L.shared8 if sh["fp8"] else L.shared4
            for n in ("w1", "s1", "w3", "s3", "w2", "s2"):
                setattr(tgt, n, _p(sh[n], u8p))
        return L


class Ref(_Lib):
    """The reference engine itself, compiled from its sources into _ref/."""

    def __init__(self):
        if not os.path.exists(REF_SO):
            raise FileNotFoundError(REF_SO)
        super().__init__(REF_SO, "dsv4_")
        L = self.lib
        L.dsv4_f32_to_bf16.restype = C.c_uint16
        L.dsv4_f32_to_bf16.argtypes = [C.c_float]
        for n in ("dsv4_fp8_e4m3", "dsv4_e8m0"):
            getattr(L, n).restype = C.c_float
            getattr(L, n).argtypes = [C.c_uint8]
        L.dsv4_round_e4m3.restype = C.c_float
        L.dsv4_round_e4m3.argtypes = [C.c_float]
        L.ref_sqrt_softplus.restype = C.c_float
        L.ref_sqrt_softplus.argtypes = [C.c_float]
        L.ref_omp_max_threads.restype = C.c_int
        L.ref_omp_set_threads.restype = C.c_int
        L.ref_omp_set_threads.argtypes = [C.c_int]

    def f32_to_bf16(self, f):
        return self.lib.dsv4_f32_to_bf16(f)

    def e4m3(self, c):
        return self.lib.dsv4_fp8_e4m3(c)

    def e8m0(self, c):
        return self.lib.dsv4_e8m0(c)

    def round_e4m3(self, v):
        return self.lib.dsv4_round_e4m3(v)

    def sqrt_softplus(self, z):
        return self.lib.ref_sqrt_softplus(z)

    def sqrt_softplus_many(self, z):
        z = _f32(z)
        s = np.empty_like(z)
        self.lib.ref_sqrt_softplus_many(_p(z, f32p), _p(s, f32p), z.size)
        return s

    def act_quant_inplace(self, x, group, mode):
        x = _f32(x).copy()
        self.lib.dsv4_act_quant_inplace(_p(x, f32p), x.size, group, mode)
        return x

    def router_public(self, x, gate, bias, topk, route_scale, tid2eid=None, token_id=0):
        ne, hid = gate.shape
        idx = np.empty(topk, np.int32)
        wt = np.empty(topk, np.float32)
        # dsv4_router declares `const float *gate` but reads BF16 words
        # (src/dsv4/dsv4_ops.c:494, :502): pass the uint16 buffer as-is.
        self.lib.dsv4_router(_p(idx, i32p), _p(wt, f32p), _p(_f32(x), f32p),
                             gate.ctypes.data_as(f32p), _p(bias, f32p), _p(tid2eid, i64p),
                             C.c_int(token_id), hid, ne, topk,
                             C.c_int(1 if tid2eid is not None else 0),
                             C.c_float(route_scale), C.c_float(1e-6))
        return idx, wt

    def swiglu_quant(self, gate, up, limit, weight):
        n = gate.size
        y = np.empty(n, np.float32)
        qy = np.empty(n, np.float32)
        qs = np.empty((n + 127) // 128, np.float32)
        self.lib.ref_routed_swiglu_quant(_p(y, f32p), _p(qy, f32p), _p(qs, f32p),
                                         _p(_f32(gate), f32p), _p(_f32(up), f32p), n,
                                         C.c_int(limit), C.c_float(weight))
        return y, qy, qs

    def rope_inv(self, x, cosv, sinv):
        x = np.array(x, dtype=np.float32, copy=True)
        c, s = _f32(cosv).copy(), _f32(sinv).copy()
        self.lib.ref_rope_inv(_p(x, f32p), x.shape[0], x.shape[1], _p(c, f32p), _p(s, f32p),
                              c.size)
        return x

    def sparse_attn(self, q, kv, sink, idx, scale):
        H, d = q.shape
        o = np.empty((H, d), np.float32)
        idx = np.ascontiguousarray(idx, dtype=np.int32)
        self.lib.ref_sparse_attn(_p(o, f32p), _p(_f32(q), f32p), _p(_f32(kv), f32p),
                                 _p(_f32(sink), f32p), _p(idx, i32p), idx.size, H, d,
                                 C.c_float(scale))
        return o

    def pack_slots(self, layer):
        """Pack every routed expert into the reference's cache-slot layout."""
        hid, mi, ne = layer["hidden"], layer["moe_inter"], layer["n_experts"]
        w13 = mi * ((hid + 1) // 2)
        w2 = hid * ((mi + 1) // 2)
        s13 = mi * ((hid + 31) // 32)
        s2 = hid * ((mi + 31) // 32)
        scales = np.empty((ne, 2 * s13 + s2), np.uint8)
        weights = np.empty((ne, 2 * w13 + w2), np.uint8)
        for e in range(ne):
            self.lib.ref_expert_slot_pack(
                _p(scales[e], u8p), _p(weights[e], u8p),
                _p(np.ascontiguousarray(layer["w1"][e]), u8p), _p(np.ascontiguousarray(layer["s1"][e]), u8p),
                _p(np.ascontiguousarray(layer["w2"][e]), u8p), _p(np.ascontiguousarray(layer["s2"][e]), u8p),
                _p(np.ascontiguousarray(layer["w3"][e]), u8p), _p(np.ascontiguousarray(layer["s3"][e]), u8p),
                hid, mi)
        return scales, weights

    def moe_forward(self, layer, x, token_id=0, slots=None):
        hid, mi, ne, topk = layer["hidden"], layer["moe_inter"], layer["n_experts"], layer["topk"]
        if slots is None:
            slots = self.pack_slots(layer)
        scales, weights = slots
        sp = (u8p * ne)(*[_p(scales[e], u8p) for e in range(ne)])
        wp = (u8p * ne)(*[_p(weights[e], u8p) for e in range(ne)])
        sh = layer.get("shared")
        if sh is not None and not sh["fp8"]:
            raise ValueError("the reference has an FP8 shared expert only")
        g = (lambda n: _p(sh[n], u8p)) if sh is not None else (lambda n: None)
        out = np.empty(hid, np.float32)
        idx = np.empty(topk, np.int32)
        wt = np.empty(topk, np.float32)
        self.lib.ref_moe_forward(_p(out, f32p), _p(idx, i32p), _p(wt, f32p), _p(_f32(x), f32p),
                                 C.c_int(token_id), _p(layer["gate_w"], u16p),
                                 _p(layer.get("bias"), f32p), _p(layer.get("tid2eid"), i64p),
                                 sp, wp, g("w1"), g("s1"), g("w3"), g("s3"), g("w2"), g("s2"),
                                 hid, mi, ne, topk, C.c_int(layer["swiglu_limit"]),
                                 C.c_float(layer["route_scale"]))
        return out, idx, wt


def make_moe_layer(hidden, moe_inter, n_experts, topk, seed=0, shared="fp8",
                   route_scale=1.5, swiglu_limit=10, bias=True, hash_vocab=0):
    """Seeded synthetic MoE layer in the reference's tensor layouts.

    Router weights are N(0, 0.02) rounded to BF16; FP4 codes are uniform over
    the 16 nibbles; E8M0 scales are lognormal(0, 0.5) rounded to the nearest
    power of two (code 127 + round(log2 s)); FP8 shared weights are uniform
    over the finite E4M3 codes with block scales drawn the same way.
    """
    rng = np.random.default_rng(seed)
    H, I, E = hidden, moe_inter, n_experts

    def e8m0(shape):
        s = rng.lognormal(0.0, 0.5, size=shape)
        return (127 + np.round(np.log2(s))).astype(np.uint8)

    def fp8_codes(shape):
        c = rng.integers(0, 254, size=shape, dtype=np.int32)
        c = np.where((c & 0x7F) == 0x7F, c - 1, c)   # skip the two NaN codes
        return c.astype(np.uint8)

    g = rng.normal(0.0, 0.02, size=(E, H)).astype(np.float32)
    gate_w = (((g.view(np.uint32) + 0x7FFF + ((g.view(np.uint32) >> 16) & 1)) >> 16)
              .astype(np.uint16))
    layer = dict(hidden=H, moe_inter=I, n_experts=E, topk=topk, route_scale=route_scale,
                 swiglu_limit=swiglu_limit, gate_w=gate_w)
    layer["bias"] = (rng.normal(0.0, 0.01, size=E).astype(np.float32) if bias else None)
    layer["tid2eid"] = None
    if hash_vocab:
        t = np.stack([rng.choice(E, size=topk, replace=False) for _ in range(hash_vocab)])
        layer["tid2eid"] = t.astype(np.int64)
    layer["w1"] = rng.integers(0, 256, size=(E, I, H // 2), dtype=np.uint8)
    layer["w3"] = rng.integers(0, 256, size=(E, I, H // 2), dtype=np.uint8)
    layer["w2"] = rng.integers(0, 256, size=(E, H, I // 2), dtype=np.uint8)
    layer["s1"] = e8m0((E, I, H // 32))
    layer["s3"] = e8m0((E, I, H // 32))
    layer["s2"] = e8m0((E, H, I // 32))
    if shared == "fp8":
        layer["shared"] = dict(
            fp8=True,
            w1=fp8_codes((I, H)), s1=e8m0(((I + 127) // 128, (H + 127) // 128)),
            w3=fp8_codes((I, H)), s3=e8m0(((I + 127) // 128, (H + 127) // 128)),
            w2=fp8_codes((H, I)), s2=e8m0(((H + 127) // 128, (I + 127) // 128)))
    elif shared == "fp4":
        layer["shared"] = dict(
            fp8=False,
            w1=rng.integers(0, 256, size=(I, H // 2), dtype=np.uint8), s1=e8m0((I, H // 32)),
            w3=rng.integers(0, 256, size=(I, H // 2), dtype=np.uint8), s3=e8m0((I, H // 32)),
            w2=rng.integers(0, 256, size=(H, I // 2), dtype=np.uint8), s2=e8m0((H, I // 32)))
    else:
        layer["shared"] = None
    return layer


# ------------------------------------------------- speculative acceptance --
u64p = C.POINTER(C.c_uint64)


class _Sampler:
    """rng_next / argmax_logits / sample_top_p with caller-held rng state;
    `prefix` selects the library's symbol names."""

    def _setup_sampler(self, lib, prefix):
        self._s = lib
        self._pre = prefix
        getattr(lib, prefix + "rng_next").restype = C.c_uint64
        getattr(lib, prefix + "rng_next").argtypes = [u64p]
        getattr(lib, prefix + "argmax_logits").restype = C.c_int
        getattr(lib, prefix + "argmax_logits").argtypes = [f32p, C.c_int]
        getattr(lib, prefix + "sample_top_p").restype = C.c_int
        getattr(lib, prefix + "sample_top_p").argtypes = [f32p, C.c_int, C.c_double, C.c_double,
                                                          u64p]

    def rng_next(self, state):
        """Returns (value, new_state)."""
        st = C.c_uint64(state)
        v = getattr(self._s, self._pre + "rng_next")(C.byref(st))
        return v, st.value

    def argmax_logits(self, logits):
        logits = _f32(logits)
        return getattr(self._s, self._pre + "argmax_logits")(_p(logits, f32p), logits.size)

    def sample_top_p(self, logits, temperature, top_p, state):
        """Returns (token, new_state)."""
        logits = _f32(logits)
        st = C.c_uint64(state)
        tok = getattr(self._s, self._pre + "sample_top_p")(_p(logits, f32p), logits.size,
                                                           temperature, top_p, C.byref(st))
        return tok, st.value


class OracleSampler(_Sampler):
    """The C restatement (dsv4_oracle.c), plus the acceptance chain."""

    def __init__(self):
        self.lib = C.CDLL(ORACLE_SO)
        self._setup_sampler(self.lib, "orc_")
        self.lib.orc_accept_chain.restype = C.c_int

    def accept_chain(self, proposal, logits, temperature, top_p, state, eos_id=1):
        """logits [(proposed+1)][V]. Returns dict(tokens, n_commit, n_accepted,
        n_samples, state)."""
        proposal = np.ascontiguousarray(proposal, dtype=np.int32)
        logits = _f32(logits)
        P = proposal.size
        toks = np.empty(P + 1, np.int32)
        st = C.c_uint64(state)
        nc, na, ns = C.c_int(), C.c_int(), C.c_int()
        n = self.lib.orc_accept_chain(_p(proposal, i32p), P, _p(logits, f32p), logits.shape[-1],
                                      C.c_double(temperature), C.c_double(top_p), C.byref(st),
                                      eos_id, _p(toks, i32p), C.byref(nc), C.byref(na),
                                      C.byref(ns))
        return dict(tokens=toks[:n].copy(), n_commit=nc.value, n_accepted=na.value,
                    n_samples=ns.value, state=st.value)


class RefSampler(_Sampler):
    """The reference CLI's own static helpers (src/cli/dsv4_run.c), compiled
    by oracle/Makefile into _ref/libdsv4_refcli.so."""

    def __init__(self):
        self.lib = C.CDLL(REFCLI_SO)
        self._setup_sampler(self.lib, "ref_")
        self.lib.ref_ngram_draft.restype = C.c_int

    def ngram_draft(self, history, cap=16, min_match=2, allow_overlap=0, periodic_extend=0):
        history = np.ascontiguousarray(history, dtype=np.int32)
        out = np.empty(64, np.int32)
        n = self.lib.ref_ngram_draft(_p(history, i32p), history.size, cap, min_match,
                                     allow_overlap, periodic_extend, _p(out, i32p))
        return out[:n].copy()
