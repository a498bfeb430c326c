"""Python binding of libdsv4_cuda.so (ctypes over the C ABI in
include/dsv4_cuda.h).

The drop-in kernels mirror the reference's kernel API (same names, argument
meaning and error behaviour); numpy arrays stand in for the host pointers.
The device-resident MoE layer takes torch CUDA tensors (data pointers and the
current stream) - torch here only provides device memory and streams.

There is no CPU fallback: if the library is missing, importing this module
raises.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "lib", "libdsv4_cuda.so")

if not os.path.exists(LIB_PATH):
    raise ImportError(f"{LIB_PATH} is missing: run deepseek-v4-flash-0731-in-c_b200/build.py")

lib = C.CDLL(LIB_PATH)

f32p = C.POINTER(C.c_float)
u8p = C.POINTER(C.c_uint8)
u16p = C.POINTER(C.c_uint16)
i32p = C.POINTER(C.c_int)
i64p = C.POINTER(C.c_int64)
vp = C.c_void_p

# Every symbol the header declares (checked by tests/test_capi_symbols.py).
DROPIN = ["dsv4_gemv_bf16", "dsv4_gemv_bf16_batch", "dsv4_gemv_fp8_q", "dsv4_gemv_fp8_batch_q",
          "dsv4_gemv_fp8_pair_q", "dsv4_gemv_fp4_q", "dsv4_gemv_fp4_batch_q",
          "dsv4_gemv_fp4_pair_q", "dsv4_quant_fp8_codes", "dsv4_quant_fp8_act", "dsv4_router"]

lib.dsv4cuda_last_error.restype = C.c_char_p
lib.dsv4cuda_set_abort_on_error.restype = C.c_int
lib.dsv4cuda_set_abort_on_error.argtypes = [C.c_int]
lib.dsv4cuda_init.restype = C.c_int
lib.dsv4cuda_init.argtypes = [C.c_int]
lib.dsv4_router.argtypes = [i32p, f32p, f32p, vp, f32p, i64p, C.c_int, C.c_int, C.c_int,
                            C.c_int, C.c_int, C.c_float, C.c_float]
lib.dsv4cuda_moe_create.restype = C.c_int
lib.dsv4cuda_moe_create_device.restype = C.c_int
lib.dsv4cuda_moe_forward.restype = C.c_int
lib.dsv4cuda_moe_forward.argtypes = [vp, vp, vp, C.c_int, vp, vp]
lib.dsv4cuda_moe_forward_host.restype = C.c_int
lib.dsv4cuda_moe_forward_host.argtypes = [vp, f32p, i32p, C.c_int, f32p]
lib.dsv4cuda_moe_last_routes.restype = C.c_int
lib.dsv4cuda_moe_last_routes.argtypes = [vp, C.c_int, i32p, f32p]
lib.dsv4cuda_moe_route.restype = C.c_int
lib.dsv4cuda_moe_route.argtypes = [vp, vp, vp, C.c_int, C.c_int, i32p, f32p]
lib.dsv4cuda_moe_destroy.argtypes = [vp]
lib.dsv4cuda_router_scores.restype = C.c_int
lib.dsv4cuda_router_scores.argtypes = [vp, vp, C.c_int, vp]
lib.dsv4cuda_routed_swiglu_quant.restype = None
lib.dsv4cuda_routed_swiglu_quant.argtypes = [vp, vp, vp, vp, vp, C.c_int, C.c_int, C.c_float]
lib.dsv4cuda_moe_forward_noalloc.restype = C.c_int
lib.dsv4cuda_moe_forward_noalloc.argtypes = [vp, vp, vp, vp, C.c_int, vp, vp]
lib.dsv4cuda_moe_device_bytes.restype = C.c_size_t
lib.dsv4cuda_moe_device_bytes.argtypes = [vp]
lib.dsv4cuda_moe_create_device_ep.restype = C.c_int
lib.dsv4cuda_moe_create_device_ep.argtypes = [vp, vp, vp, C.c_int, C.c_int, C.c_int]
lib.dsv4cuda_moe_forward_local.restype = C.c_int
lib.dsv4cuda_moe_forward_local.argtypes = [vp, vp, vp, C.c_int, vp]
lib.dsv4cuda_moe_routed_slots.restype = C.c_void_p
lib.dsv4cuda_moe_routed_slots.argtypes = [vp]
lib.dsv4cuda_moe_combine.restype = C.c_int
lib.dsv4cuda_moe_combine.argtypes = [vp, C.c_int, vp, vp]
lib.dsv4cuda_moe_ep_buffer_bytes.restype = C.c_size_t
lib.dsv4cuda_moe_ep_buffer_bytes.argtypes = [vp]
lib.dsv4cuda_moe_ep_attach.restype = C.c_int
lib.dsv4cuda_moe_ep_attach.argtypes = [vp, C.c_int, C.c_int, C.POINTER(vp)]
lib.dsv4cuda_moe_forward_ep.restype = C.c_int
lib.dsv4cuda_moe_forward_ep.argtypes = [vp, vp, vp, C.c_int, vp, vp]
lib.dsv4cuda_moe_forward_ep_tokens.restype = C.c_int
lib.dsv4cuda_moe_forward_ep_tokens.argtypes = [vp, vp, C.c_int, vp, vp]
lib.dsv4cuda_moe_ep_tokens_gather.restype = C.c_int
lib.dsv4cuda_moe_ep_tokens_gather.argtypes = [vp, vp, C.c_int, vp]
lib.dsv4cuda_moe_ep_tokens_compute.restype = C.c_int
lib.dsv4cuda_moe_ep_tokens_compute.argtypes = [vp, C.c_int, vp]
lib.dsv4cuda_moe_ep_tokens_combine.restype = C.c_int
lib.dsv4cuda_moe_ep_tokens_combine.argtypes = [vp, C.c_int, vp, vp]
lib.dsv4cuda_moe_ep_push.restype = C.c_int
lib.dsv4cuda_moe_ep_push.argtypes = [vp, C.c_int, vp]
lib.dsv4cuda_moe_ep_combine.restype = C.c_int
lib.dsv4cuda_moe_ep_combine.argtypes = [vp, C.c_int, vp, vp]
lib.dsv4cuda_ipc_alloc.restype = C.c_int
lib.dsv4cuda_ipc_alloc.argtypes = [C.c_size_t, C.POINTER(vp), C.c_char_p]
lib.dsv4cuda_ipc_open.restype = C.c_int
lib.dsv4cuda_ipc_open.argtypes = [C.c_char_p, C.POINTER(vp)]
lib.dsv4cuda_ipc_close.restype = C.c_int
lib.dsv4cuda_ipc_close.argtypes = [vp]
lib.dsv4cuda_ipc_free.restype = C.c_int
lib.dsv4cuda_ipc_free.argtypes = [vp]


class Dsv4CudaError(RuntimeError):
    pass


def last_error() -> str:
    return lib.dsv4cuda_last_error().decode()


def _check(rc):
    if rc < 0:
        raise Dsv4CudaError(last_error())
    return rc


def _p(a, t):
    return None if a is None else a.ctypes.data_as(t)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def _stream(stream):
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    return stream


def _ptrs(arrs, t):
    return (t * len(arrs))(*[a.ctypes.data_as(t) for a in arrs])


def device_error(clear: bool = False) -> int:
    v = C.c_uint()
    _check(lib.dsv4cuda_device_error(C.byref(v), 1 if clear else 0))
    return v.value


def set_abort_on_error(flag: bool) -> int:
    return lib.dsv4cuda_set_abort_on_error(1 if flag else 0)


def init(device: int = 0):
    _check(lib.dsv4cuda_init(device))


# ------------------------------------------------------ drop-in kernels --
def quant_fp8_codes(x):
    x = _f32(x)
    n = x.size
    qx = np.empty(n, np.float32)
    qs = np.empty((n + 127) // 128, np.float32)
    lib.dsv4_quant_fp8_codes(_p(qx, f32p), _p(qs, f32p), _p(x, f32p), n)
    return qx, qs


def gemv_bf16(x, W, round_out=1):
    out, inn = W.shape
    y = np.empty(out, np.float32)
    lib.dsv4_gemv_bf16(_p(y, f32p), _p(_f32(x), f32p), _p(W, u16p), inn, out, round_out)
    return y


def gemv_bf16_batch(xs, W, round_out=1):
    out, inn = W.shape
    xs = [_f32(x) for x in xs]
    ys = [np.empty(out, np.float32) for _ in xs]
    lib.dsv4_gemv_bf16_batch(_ptrs(ys, f32p), _ptrs(xs, f32p), len(xs), _p(W, u16p), inn, out,
                             round_out)
    return np.stack(ys)


def gemv_fp8_q(qx, qs, W, S, round_out=1):
    out, inn = W.shape
    y = np.empty(out, np.float32)
    lib.dsv4_gemv_fp8_q(_p(y, f32p), _p(_f32(qx), f32p), _p(_f32(qs), f32p), _p(W, u8p),
                        _p(S, u8p), inn, out, round_out)
    return y


def gemv_fp8_batch_q(qxs, qss, W, S, round_out=1):
    out, inn = W.shape
    qxs = [_f32(a) for a in qxs]
    qss = [_f32(a) for a in qss]
    ys = [np.empty(out, np.float32) for _ in qxs]
    lib.dsv4_gemv_fp8_batch_q(_ptrs(ys, f32p), _ptrs(qxs, f32p), _ptrs(qss, f32p), len(qxs),
                              _p(W, u8p), _p(S, u8p), inn, out, round_out)
    return np.stack(ys)


def gemv_fp8_pair_q(qx, qs, W0, S0, W1, S1):
    out, inn = W0.shape
    y0 = np.empty(out, np.float32)
    y1 = np.empty(out, np.float32)
    lib.dsv4_gemv_fp8_pair_q(_p(y0, f32p), _p(y1, f32p), _p(_f32(qx), f32p), _p(_f32(qs), f32p),
                             _p(W0, u8p), _p(S0, u8p), _p(W1, u8p), _p(S1, u8p), inn, out)
    return y0, y1


def gemv_fp4_q(qx, qs, W, S, inn):
    rows = W.shape[0]
    y = np.empty(rows, np.float32)
    lib.dsv4_gemv_fp4_q(_p(y, f32p), _p(_f32(qx), f32p), _p(_f32(qs), f32p), _p(W, u8p),
                        _p(S, u8p), inn, rows)
    return y


def gemv_fp4_batch_q(qxs, qss, W, S, inn):
    rows = W.shape[0]
    qxs = [_f32(a) for a in qxs]
    qss = [_f32(a) for a in qss]
    ys = [np.empty(rows, np.float32) for _ in qxs]
    lib.dsv4_gemv_fp4_batch_q(_ptrs(ys, f32p), _ptrs(qxs, f32p), _ptrs(qss, f32p), len(qxs),
                              _p(W, u8p), _p(S, u8p), inn, rows)
    return np.stack(ys)


def gemv_fp4_pair_q(qx, qs, W0, S0, W1, S1, inn):
    rows = W0.shape[0]
    y0 = np.empty(rows, np.float32)
    y1 = np.empty(rows, np.float32)
    lib.dsv4_gemv_fp4_pair_q(_p(y0, f32p), _p(y1, f32p), _p(_f32(qx), f32p), _p(_f32(qs), f32p),
                             _p(W0, u8p), _p(S0, u8p), _p(W1, u8p), _p(S1, u8p), inn, rows)
    return y0, y1


def routed_swiglu_quant(gate, up, limit, weight):
    """routed_swiglu_quant on the device (host arrays): (y, qy, qscale)."""
    g, u = _f32(gate), _f32(up)
    n = g.size
    y = np.empty(n, np.float32)
    qy = np.empty(n, np.float32)
    qs = np.empty((n + 127) // 128, np.float32)
    lib.dsv4cuda_routed_swiglu_quant(y.ctypes.data, qy.ctypes.data, qs.ctypes.data, g.ctypes.data,
                                     u.ctypes.data, n, int(limit), float(weight))
    return y, qy, qs


def router_scores(z, out, stream=None):
    """Device sqrt(softplus) of the router, z/out torch CUDA float32."""
    _check(lib.dsv4cuda_router_scores(z.data_ptr(), out.data_ptr(), z.numel(), _stream(stream)))


def router_public(x, gate, bias, topk, route_scale, tid2eid=None, token_id=0):
    ne, hid = gate.shape
    idx = np.empty(topk, np.int32)
    wt = np.empty(topk, np.float32)
    lib.dsv4_router(_p(idx, i32p), _p(wt, f32p), _p(_f32(x), f32p), gate.ctypes.data,
                    _p(bias, f32p), _p(tid2eid, i64p), token_id, hid, ne, topk,
                    1 if tid2eid is not None else 0, route_scale, 1e-6)
    return idx, wt


# ------------------------------------------------------------ MoE layer --
class MoeConfig(C.Structure):
    _fields_ = [("hidden", C.c_int), ("moe_inter", C.c_int), ("n_experts", C.c_int),
                ("topk", C.c_int), ("swiglu_limit", C.c_int), ("route_scale", C.c_float),
                ("shared_kind", C.c_int), ("hash_vocab", C.c_int)]


class MoeWeights(C.Structure):
    _fields_ = [("gate_w", vp), ("bias", vp), ("tid2eid", vp)] + \
        [(n, vp) for n in ("w1", "s1", "w3", "s3", "w2", "s2",
                           "sh1", "sh1s", "sh3", "sh3s", "sh2", "sh2s")]


SHARED_NONE, SHARED_FP8, SHARED_FP4 = 0, 1, 2


def _addr(a):
    if a is None:
        return None
    if hasattr(a, "data_ptr"):
        return a.data_ptr()
    return a.ctypes.data


def _moe_structs(layer: dict):
    sh = layer.get("shared")
    kind = SHARED_NONE if sh is None else (SHARED_FP8 if sh["fp8"] else SHARED_FP4)
    tid = layer.get("tid2eid")
    cfg = MoeConfig(layer["hidden"], layer["moe_inter"], layer["n_experts"], layer["topk"],
                    layer["swiglu_limit"], layer["route_scale"], kind,
                    0 if tid is None else int(tid.shape[0]))
    w = MoeWeights()
    w.gate_w = _addr(layer["gate_w"])
    w.bias = _addr(layer.get("bias"))
    w.tid2eid = _addr(tid)
    for n in ("w1", "s1", "w3", "s3", "w2", "s2"):
        setattr(w, n, _addr(layer[n]))
    if sh is not None:
        for n, m in (("sh1", "w1"), ("sh1s", "s1"), ("sh3", "w3"), ("sh3s", "s3"),
                     ("sh2", "w2"), ("sh2s", "s2")):
            setattr(w, n, _addr(sh[m]))
    return cfg, w


def moe_forward_noalloc(layer: dict, x, out, token_ids=None, stream=None):
    """Allocation-free MoE forward (dsv4cuda_moe_forward_noalloc): `layer`
    holds torch CUDA tensors, x/out torch CUDA float32 [n][H]. Raises on the
    library's error (e.g. too many tokens for its fixed working memory)."""
    if stream is None:
        import torch
        stream = torch.cuda.current_stream().cuda_stream
    cfg, w = _moe_structs(layer)
    _check(lib.dsv4cuda_moe_forward_noalloc(C.byref(cfg), C.byref(w), x.data_ptr(),
                                            None if token_ids is None else token_ids.data_ptr(),
                                            x.shape[0], out.data_ptr(), stream))


def ipc_alloc(nbytes):
    """Device buffer exportable to other processes: (address, 64-byte handle)."""
    ptr = C.c_void_p()
    h = C.create_string_buffer(64)
    _check(lib.dsv4cuda_ipc_alloc(nbytes, C.byref(ptr), h))
    return int(ptr.value), bytes(h.raw)


def ipc_open(handle):
    """Maps another process's buffer (ipc_alloc handle) here; returns its address."""
    ptr = C.c_void_p()
    _check(lib.dsv4cuda_ipc_open(C.create_string_buffer(bytes(handle), 64), C.byref(ptr)))
    return int(ptr.value)


def ipc_close(addr):
    _check(lib.dsv4cuda_ipc_close(C.c_void_p(addr)))


def ipc_free(addr):
    _check(lib.dsv4cuda_ipc_free(C.c_void_p(addr)))


class MoeLayer:
    """One MoE layer resident in HBM (dsv4cuda_moe_*).

    `layer` is the dict produced by oracle.make_moe_layer or any dict with the
    same keys holding numpy arrays (copied in) or torch CUDA tensors
    (adopted, device=True).
    """

    def __init__(self, layer: dict, max_tokens: int = 8, device: bool = False,
                 expert_range=None):
        """expert_range=(lo, hi): expert-parallel layer (device weights of
        experts lo..hi-1 only; layer["w1"] etc. hold hi-lo experts)."""
        sh = layer.get("shared")
        kind = SHARED_NONE if sh is None else (SHARED_FP8 if sh["fp8"] else SHARED_FP4)
        tid = layer.get("tid2eid")
        self.cfg = MoeConfig(layer["hidden"], layer["moe_inter"], layer["n_experts"],
                             layer["topk"], layer["swiglu_limit"], layer["route_scale"], kind,
                             0 if tid is None else int(tid.shape[0]))
        w = MoeWeights()
        w.gate_w = _addr(layer["gate_w"])
        w.bias = _addr(layer.get("bias"))
        w.tid2eid = _addr(tid)
        for n in ("w1", "s1", "w3", "s3", "w2", "s2"):
            setattr(w, n, _addr(layer[n]))
        if sh is not None:
            for n, m in (("sh1", "w1"), ("sh1s", "s1"), ("sh3", "w3"), ("sh3s", "s3"),
                         ("sh2", "w2"), ("sh2s", "s2")):
                setattr(w, n, _addr(sh[m]))
        self._keep = layer
        self.max_tokens = max_tokens
        self.handle = C.c_void_p()
        if expert_range is not None:
            if not device:
                raise ValueError("expert-parallel layers take device weights")
            _check(lib.dsv4cuda_moe_create_device_ep(C.byref(self.handle), C.byref(self.cfg),
                                                     C.byref(w), max_tokens,
                                                     int(expert_range[0]), int(expert_range[1])))
        else:
            fn = lib.dsv4cuda_moe_create_device if device else lib.dsv4cuda_moe_create
            _check(fn(C.byref(self.handle), C.byref(self.cfg), C.byref(w), max_tokens))
        self.hidden = layer["hidden"]
        self.topk = layer["topk"]

    def forward_local(self, x, token_ids=None, stream=None):
        """Router, this device's experts and the shared expert (EP step 1)."""
        _check(lib.dsv4cuda_moe_forward_local(self.handle, x.data_ptr(),
                                              None if token_ids is None else token_ids.data_ptr(),
                                              x.shape[0], _stream(stream)))

    def routed_slots(self, n_tokens):
        """torch CUDA float32 view [n][topk][H] of the layer's routed slots."""
        import torch
        ptr = lib.dsv4cuda_moe_routed_slots(self.handle)

        class _Iface:
            __cuda_array_interface__ = {"shape": (n_tokens, self.topk, self.hidden),
                                        "typestr": "<f4", "data": (ptr, False), "version": 3,
                                        "strides": None}
        return torch.as_tensor(_Iface(), device="cuda")

    def combine(self, n_tokens, out, stream=None):
        """Ordered combine of the (summed) routed slots and the shared expert."""
        _check(lib.dsv4cuda_moe_combine(self.handle, n_tokens, out.data_ptr(), _stream(stream)))

    def ep_buffer_bytes(self):
        """Bytes of this layer's exchange buffer for the P2P expert parallelism."""
        return int(lib.dsv4cuda_moe_ep_buffer_bytes(self.handle))

    def ep_attach(self, rank, world, bufs):
        """bufs[r]: device address (int) of rank r's exchange buffer here."""
        arr = (vp * world)(*[C.c_void_p(int(b)) for b in bufs])
        _check(lib.dsv4cuda_moe_ep_attach(self.handle, rank, world, arr))

    def forward_ep(self, x, out, token_ids=None, stream=None):
        """Router, local experts, shared expert, P2P slot exchange, combine."""
        _check(lib.dsv4cuda_moe_forward_ep(self.handle, x.data_ptr(),
                                           None if token_ids is None else token_ids.data_ptr(),
                                           x.shape[0], out.data_ptr(), _stream(stream)))

    def forward_ep_tokens(self, x_local, out_local, stream=None):
        """Token-parallel EP step: this rank's tokens in, their outputs out."""
        _check(lib.dsv4cuda_moe_forward_ep_tokens(self.handle, x_local.data_ptr(),
                                                  x_local.shape[0], out_local.data_ptr(),
                                                  _stream(stream)))

    def ep_tokens_gather(self, x_local, stream=None):
        _check(lib.dsv4cuda_moe_ep_tokens_gather(self.handle, x_local.data_ptr(),
                                                 x_local.shape[0], _stream(stream)))

    def ep_tokens_compute(self, n_local, stream=None):
        _check(lib.dsv4cuda_moe_ep_tokens_compute(self.handle, n_local, _stream(stream)))

    def ep_tokens_combine(self, n_local, out_local, stream=None):
        _check(lib.dsv4cuda_moe_ep_tokens_combine(self.handle, n_local, out_local.data_ptr(),
                                                  _stream(stream)))

    def ep_push(self, n_tokens, stream=None):
        _check(lib.dsv4cuda_moe_ep_push(self.handle, n_tokens, _stream(stream)))

    def ep_combine(self, n_tokens, out, stream=None):
        _check(lib.dsv4cuda_moe_ep_combine(self.handle, n_tokens, out.data_ptr(),
                                           _stream(stream)))

    def close(self):
        if self.handle:
            lib.dsv4cuda_moe_destroy(self.handle)
            self.handle = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def device_bytes(self) -> int:
        return lib.dsv4cuda_moe_device_bytes(self.handle)

    def forward_host(self, x, token_ids=None):
        x = _f32(np.atleast_2d(x))
        n = x.shape[0]
        out = np.empty_like(x)
        tok = None if token_ids is None else np.ascontiguousarray(token_ids, dtype=np.int32)
        _check(lib.dsv4cuda_moe_forward_host(self.handle, _p(x, f32p), _p(tok, i32p), n,
                                             _p(out, f32p)))
        return out

    def forward(self, x, out, token_ids=None, stream=None):
        """x/out: torch CUDA float32 [n][H]; token_ids: torch CUDA int32 [n]."""
        if stream is None:
            import torch
            stream = torch.cuda.current_stream().cuda_stream
        _check(lib.dsv4cuda_moe_forward(self.handle, x.data_ptr(),
                                        None if token_ids is None else token_ids.data_ptr(),
                                        x.shape[0], out.data_ptr(), stream))

    def last_routes(self, n_tokens):
        idx = np.empty((n_tokens, self.topk), np.int32)
        wt = np.empty((n_tokens, self.topk), np.float32)
        fallbacks = _check(lib.dsv4cuda_moe_last_routes(self.handle, n_tokens, _p(idx, i32p),
                                                        _p(wt, f32p)))
        return idx, wt, fallbacks

    def route(self, x, token_ids=None, public_router=False):
        """x: torch CUDA float32 [n][H]."""
        n = x.shape[0]
        idx = np.empty((n, self.topk), np.int32)
        wt = np.empty((n, self.topk), np.float32)
        fallbacks = _check(lib.dsv4cuda_moe_route(
            self.handle, x.data_ptr(), None if token_ids is None else token_ids.data_ptr(), n,
            1 if public_router else 0, _p(idx, i32p), _p(wt, f32p)))
        return idx, wt, fallbacks


# ------------------------------------------------------------ attention --

class KvCache(C.Structure):
    _fields_ = [("codes", vp), ("scales", vp), ("rope", vp), ("nope", C.c_int),
                ("rope_dim", C.c_int), ("rows", C.c_longlong)]


class AttnShape(C.Structure):
    _fields_ = [("batch", C.c_int), ("heads", C.c_int), ("head_dim", C.c_int),
                ("n_keys", C.c_int), ("scale", C.c_float), ("rope_dim", C.c_int),
                ("kv_batch_stride", C.c_longlong), ("kv_rows", C.c_longlong)]


lib.dsv4cuda_kv_write.restype = C.c_int
lib.dsv4cuda_kv_write.argtypes = [vp, vp, vp, C.c_int, vp]
lib.dsv4cuda_kv_read.restype = C.c_int
lib.dsv4cuda_kv_read.argtypes = [vp, vp, C.c_int, vp, vp]
lib.dsv4cuda_attn_workspace_bytes.restype = C.c_size_t
lib.dsv4cuda_attn_workspace_bytes.argtypes = [vp, C.c_int]
lib.dsv4cuda_sparse_attn.restype = C.c_int
lib.dsv4cuda_sparse_attn.argtypes = [vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, C.c_size_t, vp]
lib.dsv4cuda_sparse_attn_host.restype = None
lib.dsv4cuda_sparse_attn_host.argtypes = [f32p, f32p, f32p, f32p, i32p, C.c_int, C.c_int,
                                          C.c_int, C.c_float]
lib.dsv4cuda_attn_timing_begin.restype = C.c_int
lib.dsv4cuda_attn_timing_end.restype = C.c_int
lib.dsv4cuda_attn_timing_end.argtypes = [i32p, f32p]


class LatentCache:
    """FP8 latent cache in HBM (dsv4cuda_kv_cache): torch uint8/int16 tensors
    for codes [rows][nope], scales [rows][8], rope [rows][rope_dim]."""

    def __init__(self, rows: int, nope: int = 448, rope_dim: int = 64, device="cuda"):
        import torch
        self.codes = torch.zeros((rows, nope), dtype=torch.uint8, device=device)
        self.scales = torch.zeros((rows, 8), dtype=torch.uint8, device=device)
        self.rope = torch.zeros((rows, rope_dim), dtype=torch.int16, device=device)
        self.nope, self.rope_dim, self.rows = nope, rope_dim, rows
        self.struct = KvCache(self.codes.data_ptr(), self.scales.data_ptr(),
                              self.rope.data_ptr(), nope, rope_dim, rows)

    @property
    def bytes_per_row(self) -> int:
        return self.nope + 8 + 2 * self.rope_dim

    def write(self, kv, rows, stream=None):
        """kv: torch CUDA float32 [n][nope+rope]; rows: torch CUDA int64 [n]."""
        _check(lib.dsv4cuda_kv_write(C.byref(self.struct), kv.data_ptr(), rows.data_ptr(),
                                     kv.shape[0], _stream(stream)))

    def read(self, rows, out, stream=None):
        _check(lib.dsv4cuda_kv_read(C.byref(self.struct), rows.data_ptr(), rows.shape[0],
                                    out.data_ptr(), _stream(stream)))


def attn_shape(batch, heads, head_dim, n_keys, scale, rope_dim=64, kv_batch_stride=0,
               kv_rows=0):
    return AttnShape(batch, heads, head_dim, n_keys, scale, rope_dim, kv_batch_stride, kv_rows)


def attn_workspace_bytes(shape: AttnShape, use_cache: bool) -> int:
    return lib.dsv4cuda_attn_workspace_bytes(C.byref(shape), 1 if use_cache else 0)


def sparse_attn(out, q, sink, idx, shape: AttnShape, kv=None, cache: LatentCache = None,
                rope_cos=None, rope_sin=None, workspace=None, stream=None):
    """dsv4cuda_sparse_attn on torch CUDA tensors (fp32 q/kv/sink/out, int32
    idx). Either kv (fp32 rows) or cache."""
    ws = None if workspace is None else workspace.data_ptr()
    wsb = 0 if workspace is None else workspace.numel() * workspace.element_size()
    _check(lib.dsv4cuda_sparse_attn(
        out.data_ptr(), q.data_ptr(), None if kv is None else kv.data_ptr(),
        None if cache is None else C.byref(cache.struct), sink.data_ptr(),
        idx.data_ptr(), None if rope_cos is None else rope_cos.data_ptr(),
        None if rope_sin is None else rope_sin.data_ptr(), C.byref(shape), ws, wsb,
        _stream(stream)))


def sparse_attn_host(q, kv, sink, idx, scale):
    """Reference-shaped host form: q [H][d], kv [rows][d], sink [H], idx [n]."""
    q = _f32(q)
    kv = _f32(kv)
    sink = _f32(sink)
    idx = np.ascontiguousarray(idx, dtype=np.int32)
    H, d = q.shape
    o = np.empty_like(q)
    lib.dsv4cuda_sparse_attn_host(_p(o, f32p), _p(q, f32p), _p(kv, f32p), _p(sink, f32p),
                                  _p(idx, i32p), idx.size, H, d, scale)
    return o


def attn_timing_begin():
    _check(lib.dsv4cuda_attn_timing_begin())


def attn_timing_end():
    n = C.c_int(0)
    ms = C.c_float(0)
    _check(lib.dsv4cuda_attn_timing_end(C.byref(n), C.byref(ms)))
    return n.value, ms.value


# ------------------------------------------------- speculative acceptance --
u64p = C.POINTER(C.c_uint64)
lib.dsv4cuda_rng_next.restype = C.c_uint64
lib.dsv4cuda_rng_next.argtypes = [u64p]
lib.dsv4cuda_argmax_logits.restype = C.c_int
lib.dsv4cuda_argmax_logits.argtypes = [f32p, C.c_int]
lib.dsv4cuda_sample_top_p.restype = C.c_int
lib.dsv4cuda_sample_top_p.argtypes = [f32p, C.c_int, C.c_double, C.c_double, u64p]
lib.dsv4cuda_accept_chain.restype = C.c_int
lib.dsv4cuda_accept_chain.argtypes = [i32p, C.c_int, f32p, C.c_int, C.c_double, C.c_double,
                                      u64p, C.c_int, i32p, i32p, i32p, i32p]
lib.dsv4cuda_argmax_rows.restype = C.c_int
lib.dsv4cuda_argmax_rows.argtypes = [vp, C.c_int, C.c_int, vp, vp]
lib.dsv4cuda_sample_rows.restype = C.c_int
lib.dsv4cuda_sample_rows.argtypes = [vp, C.c_int, C.c_int, C.c_double, vp, vp, vp]
lib.dsv4cuda_accept_device.restype = C.c_int
lib.dsv4cuda_accept_device.argtypes = [vp, C.c_int, vp, C.c_int, C.c_double, vp, C.c_int, vp, vp]


def rng_next(state):
    st = C.c_uint64(state)
    v = lib.dsv4cuda_rng_next(C.byref(st))
    return v, st.value


def uniforms(state, n):
    """n 53-bit uniforms in the reference's draw order; returns (array, state)."""
    out = np.empty(n, np.float64)
    for i in range(n):
        v, state = rng_next(state)
        out[i] = (v >> 11) * (1.0 / 9007199254740992.0)
    return out, state


def argmax_logits(logits):
    logits = _f32(logits)
    return lib.dsv4cuda_argmax_logits(_p(logits, f32p), logits.size)


def sample_top_p(logits, temperature, top_p, state):
    logits = _f32(logits)
    st = C.c_uint64(state)
    tok = lib.dsv4cuda_sample_top_p(_p(logits, f32p), logits.size, temperature, top_p,
                                    C.byref(st))
    return tok, st.value


def accept_chain(proposal, logits, temperature, top_p, state, eos_id=1):
    proposal = np.ascontiguousarray(proposal, dtype=np.int32)
    logits = _f32(logits)
    toks = np.empty(proposal.size + 1, np.int32)
    st = C.c_uint64(state)
    nc, na, ns = C.c_int(), C.c_int(), C.c_int()
    n = _check(lib.dsv4cuda_accept_chain(_p(proposal, i32p), proposal.size, _p(logits, f32p),
                                         logits.shape[-1], temperature, top_p, C.byref(st),
                                         eos_id, _p(toks, i32p), C.byref(nc), C.byref(na),
                                         C.byref(ns)))
    return dict(tokens=toks[:n].copy(), n_commit=nc.value, n_accepted=na.value,
                n_samples=ns.value, state=st.value)


def argmax_rows(logits, out, stream=None):
    """logits: torch CUDA float32 [rows][V]; out: torch CUDA int32 [rows]."""
    _check(lib.dsv4cuda_argmax_rows(logits.data_ptr(), logits.shape[0], logits.shape[1],
                                    out.data_ptr(), _stream(stream)))


def sample_rows(logits, temperature, uniforms_dev, out, stream=None):
    _check(lib.dsv4cuda_sample_rows(logits.data_ptr(), logits.shape[0], logits.shape[1],
                                    temperature, uniforms_dev.data_ptr(), out.data_ptr(),
                                    _stream(stream)))


def accept_device(proposal_dev, logits, temperature, uniforms_dev, result, eos_id=1,
                  stream=None):
    """proposal_dev int32 [P]; logits [(P+1)][V]; result int32 [2P + 6]."""
    _check(lib.dsv4cuda_accept_device(
        proposal_dev.data_ptr(), proposal_dev.numel(), logits.data_ptr(), logits.shape[1],
        temperature, None if uniforms_dev is None else uniforms_dev.data_ptr(), eos_id,
        result.data_ptr(), _stream(stream)))


# ---------------------------------------------------- KV-ring snapshot --
lib.dsv4cuda_snapshot_create.restype = C.c_int
lib.dsv4cuda_snapshot_create.argtypes = [vp, C.c_int, C.c_int, vp, vp, vp, C.c_int, vp, vp]
for _n in ("take",):
    getattr(lib, "dsv4cuda_snapshot_" + _n).restype = C.c_int
lib.dsv4cuda_snapshot_take.argtypes = [vp, C.c_int, C.c_int, vp]
lib.dsv4cuda_snapshot_capture_state.restype = C.c_int
lib.dsv4cuda_snapshot_capture_state.argtypes = [vp, C.c_int, vp]
lib.dsv4cuda_snapshot_commit_prefix.restype = C.c_int
lib.dsv4cuda_snapshot_commit_prefix.argtypes = [vp, C.c_int, vp]
lib.dsv4cuda_snapshot_restore.restype = C.c_int
lib.dsv4cuda_snapshot_restore.argtypes = [vp, vp]
lib.dsv4cuda_snapshot_destroy.argtypes = [vp]


class Snapshot:
    """Speculative transaction over LatentCache rings and float32 CUDA state
    tensors (dsv4cuda_snapshot_*)."""

    def __init__(self, caches, windows, ring_base=None, states=(), max_positions=16):
        nc = len(caches)
        arr = (KvCache * max(nc, 1))(*[c.struct for c in caches])
        win = (C.c_int * max(nc, 1))(*windows)
        base = None if ring_base is None else (C.c_longlong * max(nc, 1))(*ring_base)
        ns = len(states)
        sp = (C.c_void_p * max(ns, 1))(*[t.data_ptr() for t in states])
        se = (C.c_size_t * max(ns, 1))(*[t.numel() for t in states])
        self._keep = (caches, states)
        self.handle = C.c_void_p()
        _check(lib.dsv4cuda_snapshot_create(C.byref(self.handle), max_positions, nc, arr, base,
                                            win, ns, sp, se))

    def take(self, start, n, stream=None):
        _check(lib.dsv4cuda_snapshot_take(self.handle, start, n, _stream(stream)))

    def capture_state(self, step, stream=None):
        _check(lib.dsv4cuda_snapshot_capture_state(self.handle, step, _stream(stream)))

    def commit_prefix(self, k, stream=None):
        _check(lib.dsv4cuda_snapshot_commit_prefix(self.handle, k, _stream(stream)))

    def restore(self, stream=None):
        _check(lib.dsv4cuda_snapshot_restore(self.handle, _stream(stream)))

    def close(self):
        if self.handle:
            lib.dsv4cuda_snapshot_destroy(self.handle)
            self.handle = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


# ------------------------------------------------------------ tree verify --
lib.dsv4cuda_tree_attn_indices.restype = C.c_int
lib.dsv4cuda_tree_attn_indices.argtypes = [i32p, C.c_int, C.c_int, C.c_int, C.c_longlong,
                                           C.c_longlong, i32p, C.c_int]
lib.dsv4cuda_kv_copy_rows.restype = C.c_int
lib.dsv4cuda_kv_copy_rows.argtypes = [vp, vp, vp, C.c_int, vp]


def tree_attn_indices(parents, committed, window, ring_base, scratch_row, row_len):
    """idx [n_nodes][row_len] (-1 padded) for a verify over a draft tree."""
    parents = np.ascontiguousarray(parents, dtype=np.int32)
    idx = np.empty((parents.size, row_len), np.int32)
    _check(lib.dsv4cuda_tree_attn_indices(_p(parents, i32p), parents.size, committed, window,
                                          ring_base, scratch_row, _p(idx, i32p), row_len))
    return idx


def kv_copy_rows(cache, src_rows, dst_rows, stream=None):
    s = np.ascontiguousarray(src_rows, dtype=np.int64)
    d = np.ascontiguousarray(dst_rows, dtype=np.int64)
    _check(lib.dsv4cuda_kv_copy_rows(C.byref(cache.struct), s.ctypes.data, d.ctypes.data, s.size,
                                     _stream(stream)))


# ------------------------------------------------------- whole-model decode --
class DecoderConfig(C.Structure):
    _fields_ = [(n, C.c_int) for n in ("hidden", "n_layers", "vocab", "n_heads", "head_dim",
                                       "rope_dim", "q_lora", "o_groups", "o_lora", "window",
                                       "hc_mult", "hc_iters")] + \
        [("rms_eps", C.c_float), ("hc_eps", C.c_float), ("rope_theta", C.c_float),
         ("max_context", C.c_int), ("moe", MoeConfig), ("hc_exact", C.c_int),
         ("index_heads", C.c_int), ("index_dim", C.c_int), ("index_topk", C.c_int),
         ("compress_rope_theta", C.c_float), ("rope_factor", C.c_float),
         ("beta_fast", C.c_float), ("beta_slow", C.c_float), ("original_position", C.c_int)]


class ModelWeights(C.Structure):
    _fields_ = [(n, vp) for n in ("embed", "head", "norm", "hc_head_fn", "hc_head_base",
                                  "hc_head_scale")]


class LayerWeights(C.Structure):
    _fields_ = [(n, vp) for n in (
        "attn_norm", "ffn_norm", "hc_attn_fn", "hc_attn_scale", "hc_attn_base",
        "hc_ffn_fn", "hc_ffn_scale", "hc_ffn_base", "attn_sink", "wq_a", "wq_a_s", "q_norm",
        "wq_b", "wq_b_s", "wkv", "wkv_s", "kv_norm", "wo_a", "wo_a_fp8", "wo_a_fp8_s",
        "wo_b", "wo_b_s")] + [("moe", MoeWeights), ("compress_ratio", C.c_int)] + \
        [(n, vp) for n in ("comp_wkv", "comp_wgate", "comp_ape", "comp_norm", "idx_wq_b",
                           "idx_wq_b_s", "idx_weights_proj", "idx_comp_wkv", "idx_comp_wgate",
                           "idx_ape", "idx_comp_norm")]


for _n, _r, _a in (("dsv4cuda_decoder_create", C.c_int, [vp, vp, vp, vp]),
                   ("dsv4cuda_decoder_destroy", None, [vp]),
                   ("dsv4cuda_decoder_last_error", C.c_char_p, []),
                   ("dsv4cuda_decoder_reset", C.c_int, [vp, vp]),
                   ("dsv4cuda_decoder_forward_token", C.c_int, [vp, C.c_int, C.c_int, vp, vp]),
                   ("dsv4cuda_decoder_step", C.c_int, [vp, vp]),
                   ("dsv4cuda_decoder_step_device", C.c_int, [vp, vp, vp, vp]),
                   ("dsv4cuda_decoder_token_slot", C.c_void_p, [vp]),
                   ("dsv4cuda_decoder_position_slot", C.c_void_p, [vp]),
                   ("dsv4cuda_decoder_logits", C.c_void_p, [vp]),
                   ("dsv4cuda_decoder_argmax", C.c_void_p, [vp]),
                   ("dsv4cuda_decoder_read", C.c_int, [vp, vp, vp]),
                   ("dsv4cuda_decoder_cache", C.c_int, [vp, C.c_int, vp]),
                   ("dsv4cuda_decoder_step_kernels", C.c_int, [vp]),
                   ("dsv4cuda_decoder_set_moe_layers", C.c_int, [vp, vp, C.c_int]),
                   ("dsv4cuda_decoder_set_ep_replicated", C.c_int, [vp, C.c_int]),
                   ("dsv4cuda_decoder_verify", C.c_int, [vp, vp, C.c_int, C.c_int, vp, vp]),
                   ("dsv4cuda_decoder_verify_device", C.c_int, [vp, C.c_int, vp]),
                   ("dsv4cuda_decoder_commit", C.c_int, [vp, C.c_int, vp]),
                   ("dsv4cuda_decoder_accept_greedy", C.c_int, [vp, C.c_int, vp]),
                   ("dsv4cuda_decoder_draft_random", C.c_int, [vp, C.c_int, vp]),
                   ("dsv4cuda_decoder_verify_stats", C.c_int, [vp, vp]),
                   ("dsv4cuda_decoder_verify_pending", C.c_int, [vp, vp, vp]),
                   ("dsv4cuda_decoder_verify_tokens", C.c_void_p, [vp]),
                   ("dsv4cuda_decoder_verify_start", C.c_void_p, [vp]),
                   ("dsv4cuda_decoder_verify_logits", C.c_void_p, [vp]),
                   ("dsv4cuda_decoder_verify_argmax", C.c_void_p, [vp])):
    getattr(lib, _n).restype = _r
    getattr(lib, _n).argtypes = _a


class Decoder:
    """dsv4_forward_token on the device (dsv4cuda_decoder_*). `cfg` is a
    dict of the DecoderConfig fields (moe: a dict of MoeConfig fields);
    `model` and `layers` hold torch CUDA tensors named like the C structs'
    fields (layers[i]["moe"] like a MoE layer dict). The tensors must stay
    alive as long as the decoder."""

    def __init__(self, cfg: dict, model: dict, layers: list):
        c = DecoderConfig()
        for k, v in cfg.items():
            if k != "moe":
                setattr(c, k, v)
        for k, v in cfg["moe"].items():
            setattr(c.moe, k, v)
        self.vocab = cfg["vocab"]
        self._keep = (model, layers)
        mw = ModelWeights(*[_addr(model.get(f[0])) for f in ModelWeights._fields_])
        lws = (LayerWeights * len(layers))()
        for i, L in enumerate(layers):
            for name, _ in LayerWeights._fields_:
                if name == "moe":
                    _, w = _moe_structs(L["moe"])
                    lws[i].moe = w
                elif name == "compress_ratio":
                    lws[i].compress_ratio = int(L.get("compress_ratio", 0))
                else:
                    setattr(lws[i], name, _addr(L.get(name)))
        h = vp()
        if lib.dsv4cuda_decoder_create(C.byref(h), C.byref(c), C.byref(mw), lws) != 0:
            raise Dsv4CudaError(lib.dsv4cuda_decoder_last_error().decode())
        self.handle = h

    def forward_token(self, token, position):
        """(logits [vocab] float32, greedy next token)."""
        logits = np.empty(self.vocab, np.float32)
        nxt = C.c_int()
        if lib.dsv4cuda_decoder_forward_token(self.handle, int(token), int(position),
                                              logits.ctypes.data, C.byref(nxt)) != 0:
            raise Dsv4CudaError(lib.dsv4cuda_decoder_last_error().decode())
        return logits, nxt.value

    def step_device(self, token, position, stream=None):
        """Step with token / position from device int32 tensors (capturable)."""
        if lib.dsv4cuda_decoder_step_device(self.handle, token.data_ptr(), position.data_ptr(),
                                            _stream(stream)) != 0:
            raise Dsv4CudaError(lib.dsv4cuda_decoder_last_error().decode())

    VERIFY_MAX_ROWS = 8

    def verify(self, tokens, start_position):
        """dsv4_prefill_capture with all_logits: (logits [n][vocab] float32,
        argmax [n] int32) of the rows `tokens` at positions start_position..;
        the ring is untouched until commit()."""
        t = np.ascontiguousarray(tokens, np.int32)
        n = len(t)
        logits = np.empty((n, self.vocab), np.float32)
        am = np.empty(n, np.int32)
        if lib.dsv4cuda_decoder_verify(self.handle, t.ctypes.data, n, int(start_position),
                                       logits.ctypes.data, am.ctypes.data) != 0:
            raise Dsv4CudaError(lib.dsv4cuda_decoder_last_error().decode())
        return logits, am

    def commit(self, n_keep, stream=None):
        """Keeps the last verify's rows 0 .. n_keep - 1 (into the ring)."""
        if lib.dsv4cuda_decoder_commit(self.handle, int(n_keep), _stream(stream)) != 0:
            raise Dsv4CudaError(lib.dsv4cuda_decoder_last_error().decode())

    def verify_device(self, n_rows, stream=None):
        if lib.dsv4cuda_decoder_verify_device(self.handle, int(n_rows), _stream(stream)) != 0:
            raise Dsv4CudaError(lib.dsv4cuda_decoder_last_error().decode())

    def accept_greedy(self, n_rows, stream=None):
        if lib.dsv4cuda_decoder_accept_greedy(self.handle, int(n_rows), _stream(stream)) != 0:
            raise Dsv4CudaError(lib.dsv4cuda_decoder_last_error().decode())

    def draft_random(self, n_rows, stream=None):
        if lib.dsv4cuda_decoder_draft_random(self.handle, int(n_rows), _stream(stream)) != 0:
            raise Dsv4CudaError(lib.dsv4cuda_decoder_last_error().decode())

    def verify_stats(self):
        """(tokens emitted, drafts accepted, verify steps) of accept_greedy."""
        st = np.zeros(3, np.int64)
        if lib.dsv4cuda_decoder_verify_stats(self.handle, st.ctypes.data) != 0:
            raise Dsv4CudaError(lib.dsv4cuda_decoder_last_error().decode())
        return tuple(int(x) for x in st)

    def verify_pending(self):
        """(pending token, its position) that accept_greedy left for the next step."""
        t, p = C.c_int(), C.c_int()
        if lib.dsv4cuda_decoder_verify_pending(self.handle, C.byref(t), C.byref(p)) != 0:
            raise Dsv4CudaError(lib.dsv4cuda_decoder_last_error().decode())
        return t.value, p.value

    def verify_slots(self):
        """Device addresses: (row tokens [8], start position, logits [8][vocab], argmax [8])."""
        return (lib.dsv4cuda_decoder_verify_tokens(self.handle),
                lib.dsv4cuda_decoder_verify_start(self.handle),
                lib.dsv4cuda_decoder_verify_logits(self.handle),
                lib.dsv4cuda_decoder_verify_argmax(self.handle))

    def set_moe_layers(self, moe_layers):
        """Expert parallelism: one EP-attached MoeLayer per decoder layer."""
        arr = (vp * max(len(moe_layers), 1))(*[m.handle for m in moe_layers])
        self._ep = list(moe_layers)
        if lib.dsv4cuda_decoder_set_moe_layers(self.handle, arr, len(moe_layers)) != 0:
            raise Dsv4CudaError(lib.dsv4cuda_decoder_last_error().decode())

    def set_ep_replicated(self, on):
        """Batch-1 expert parallelism: every rank decodes the same token."""
        if lib.dsv4cuda_decoder_set_ep_replicated(self.handle, 1 if on else 0) != 0:
            raise Dsv4CudaError(lib.dsv4cuda_decoder_last_error().decode())

    def read(self):
        """The last step's (logits, argmax), copied to the host."""
        logits = np.empty(self.vocab, np.float32)
        nxt = C.c_int()
        if lib.dsv4cuda_decoder_read(self.handle, logits.ctypes.data, C.byref(nxt)) != 0:
            raise Dsv4CudaError(lib.dsv4cuda_decoder_last_error().decode())
        return logits, nxt.value

    def step(self, stream=None):
        if lib.dsv4cuda_decoder_step(self.handle, _stream(stream)) != 0:
            raise Dsv4CudaError(lib.dsv4cuda_decoder_last_error().decode())

    def slots(self):
        """Device addresses: (token slot, position slot, logits, argmax)."""
        return (lib.dsv4cuda_decoder_token_slot(self.handle),
                lib.dsv4cuda_decoder_position_slot(self.handle),
                lib.dsv4cuda_decoder_logits(self.handle), lib.dsv4cuda_decoder_argmax(self.handle))

    def cache(self, layer):
        """Layer `layer`'s latent ring as a KvCache structure (device pointers)."""
        kc = KvCache()
        if lib.dsv4cuda_decoder_cache(self.handle, layer, C.byref(kc)) != 0:
            raise Dsv4CudaError(lib.dsv4cuda_decoder_last_error().decode())
        return kc

    def reset(self, stream=None):
        if lib.dsv4cuda_decoder_reset(self.handle, _stream(stream)) != 0:
            raise Dsv4CudaError(lib.dsv4cuda_decoder_last_error().decode())

    def close(self):
        if getattr(self, "handle", None):
            lib.dsv4cuda_decoder_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def read_safetensors(path):
    """{name: numpy array} of a single-file safetensors checkpoint (F32, BF16
    as uint16, F8_E4M3 / F8_E8M0 / I8 as uint8, I64)."""
    import json
    import struct
    dt = {"F32": np.float32, "BF16": np.uint16, "F8_E4M3": np.uint8, "F8_E8M0": np.uint8,
          "I8": np.uint8, "I64": np.int64}
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        hdr = json.loads(f.read(n))
        data = f.read()
    out = {}
    for name, t in hdr.items():
        if name == "__metadata__":
            continue
        a, b = t["data_offsets"]
        out[name] = np.frombuffer(data[a:b], dtype=dt[t["dtype"]]).reshape(t["shape"])
    return out


def decoder_from_checkpoint(ckpt_dir, max_context, device="cuda", hc_exact=False):
    """Weight ingest for the device decoder: reads a checkpoint directory in
    the reference's format (config.json + one safetensors file), stacks the
    routed experts expert-major and uploads everything to `device`.
    Returns a Decoder. Layers of compress ratio 4 / 128 bring their
    compressor (and for ratio 4 indexer) tensors."""
    import json
    import torch
    with open(os.path.join(ckpt_dir, "config.json")) as f:
        cj = json.load(f)
    files = [fn for fn in os.listdir(ckpt_dir) if fn.endswith(".safetensors")]
    t = {}
    for fn in files:
        t.update(read_safetensors(os.path.join(ckpt_dir, fn)))
    ratios = list(cj["compress_ratios"][:cj["num_hidden_layers"]])
    ys = cj.get("rope_scaling") or {}

    def dev(a):
        return torch.from_numpy(np.ascontiguousarray(a)).to(device)

    E = cj["n_routed_experts"]
    cfg = dict(hidden=cj["hidden_size"], n_layers=cj["num_hidden_layers"],
               vocab=cj["vocab_size"], n_heads=cj["num_attention_heads"],
               head_dim=cj["head_dim"], rope_dim=cj["qk_rope_head_dim"],
               q_lora=cj["q_lora_rank"], o_groups=cj["o_groups"], o_lora=cj["o_lora_rank"],
               window=cj["sliding_window"], hc_mult=cj["hc_mult"],
               hc_iters=cj["hc_sinkhorn_iters"], rms_eps=cj["rms_norm_eps"],
               hc_eps=cj["hc_eps"], rope_theta=cj["rope_theta"], max_context=max_context,
               hc_exact=1 if hc_exact else 0,
               index_heads=cj.get("index_n_heads", 0), index_dim=cj.get("index_head_dim", 0),
               index_topk=cj.get("index_topk", 0),
               compress_rope_theta=cj.get("compress_rope_theta", cj["rope_theta"]),
               rope_factor=ys.get("factor", 1.0), beta_fast=ys.get("beta_fast", 32.0),
               beta_slow=ys.get("beta_slow", 1.0),
               original_position=ys.get("original_max_position_embeddings", 4096),
               moe=dict(hidden=cj["hidden_size"], moe_inter=cj["moe_intermediate_size"],
                        n_experts=E, topk=cj["num_experts_per_tok"],
                        swiglu_limit=int(cj["swiglu_limit"]),
                        route_scale=cj["routed_scaling_factor"], shared_kind=SHARED_FP8,
                        hash_vocab=0))
    model = dict(embed=dev(t["embed.weight"]), head=dev(t["head.weight"]),
                 norm=dev(t["norm.weight"]), hc_head_fn=dev(t["hc_head_fn"]),
                 hc_head_base=dev(t["hc_head_base"]), hc_head_scale=dev(t["hc_head_scale"]))
    layers = []
    for L in range(cfg["n_layers"]):
        p = f"layers.{L}."
        a = p + "attn."
        ex = lambda e, n: t[f"{p}ffn.experts.{e}.{n}"]  # noqa: E731
        moe = dict(hidden=cfg["hidden"], moe_inter=cfg["moe"]["moe_inter"], n_experts=E,
                   topk=cfg["moe"]["topk"], route_scale=cfg["moe"]["route_scale"],
                   swiglu_limit=cfg["moe"]["swiglu_limit"],
                   gate_w=dev(t[p + "ffn.gate.weight"]), bias=dev(t[p + "ffn.gate.bias"]),
                   tid2eid=None,
                   shared=dict(fp8=True,
                               w1=dev(t[p + "ffn.shared_experts.w1.weight"]),
                               s1=dev(t[p + "ffn.shared_experts.w1.scale"]),
                               w3=dev(t[p + "ffn.shared_experts.w3.weight"]),
                               s3=dev(t[p + "ffn.shared_experts.w3.scale"]),
                               w2=dev(t[p + "ffn.shared_experts.w2.weight"]),
                               s2=dev(t[p + "ffn.shared_experts.w2.scale"])))
        for w in ("w1", "w2", "w3"):
            moe[w] = dev(np.stack([ex(e, w + ".weight") for e in range(E)]))
            moe["s" + w[1]] = dev(np.stack([ex(e, w + ".scale") for e in range(E)]))
        layers.append(dict(
            attn_norm=dev(t[p + "attn_norm.weight"]), ffn_norm=dev(t[p + "ffn_norm.weight"]),
            hc_attn_fn=dev(t[p + "hc_attn_fn"]), hc_attn_scale=dev(t[p + "hc_attn_scale"]),
            hc_attn_base=dev(t[p + "hc_attn_base"]), hc_ffn_fn=dev(t[p + "hc_ffn_fn"]),
            hc_ffn_scale=dev(t[p + "hc_ffn_scale"]), hc_ffn_base=dev(t[p + "hc_ffn_base"]),
            attn_sink=dev(t[a + "attn_sink"]),
            wq_a=dev(t[a + "wq_a.weight"]), wq_a_s=dev(t[a + "wq_a.scale"]),
            q_norm=dev(t[a + "q_norm.weight"]),
            wq_b=dev(t[a + "wq_b.weight"]), wq_b_s=dev(t[a + "wq_b.scale"]),
            wkv=dev(t[a + "wkv.weight"]), wkv_s=dev(t[a + "wkv.scale"]),
            kv_norm=dev(t[a + "kv_norm.weight"]),
            wo_a_fp8=dev(t[a + "wo_a.weight"]), wo_a_fp8_s=dev(t[a + "wo_a.scale"]),
            wo_b=dev(t[a + "wo_b.weight"]), wo_b_s=dev(t[a + "wo_b.scale"]), moe=moe,
            compress_ratio=ratios[L]))
        if ratios[L]:
            cp, ip = a + "compressor.", a + "indexer."
            layers[-1].update(comp_wkv=dev(t[cp + "wkv.weight"]),
                              comp_wgate=dev(t[cp + "wgate.weight"]),
                              comp_ape=dev(t[cp + "ape"]), comp_norm=dev(t[cp + "norm.weight"]))
            if ratios[L] == 4:
                layers[-1].update(idx_wq_b=dev(t[ip + "wq_b.weight"]),
                                  idx_wq_b_s=dev(t[ip + "wq_b.scale"]),
                                  idx_weights_proj=dev(t[ip + "weights_proj.weight"]),
                                  idx_comp_wkv=dev(t[ip + "compressor.wkv.weight"]),
                                  idx_comp_wgate=dev(t[ip + "compressor.wgate.weight"]),
                                  idx_ape=dev(t[ip + "compressor.ape"]),
                                  idx_comp_norm=dev(t[ip + "compressor.norm.weight"]))
    return Decoder(cfg, model, layers)
