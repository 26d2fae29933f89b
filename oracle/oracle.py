"""ctypes bindings for the parity checkers (test infrastructure only).

``Oracle`` wraps ``liboracle.so`` (the CPU restatement in att1_oracle.c) and
``Reference`` wraps ``_ref/libatt1ref.so`` (the ATT-1 sources compiled by
oracle/Makefile plus ref_harness.c). Only tests, ``__graft_entry__.smoke`` and
the CPU-baseline leg of ``bench.py`` import this module.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libatt1ref.so")

Q4, Q8 = 4, 8
T_ATTN_NORM, T_WQ, T_WK, T_WV, T_WO, T_FFN_NORM, T_GATE, T_UP, T_DOWN = range(9)
T_OUTPUT_KIND = 9
T_PER_LAYER = 16
T_EMBED = 0x7F000000
T_OUTPUT_NORM = 0x7F000001
T_OUTPUT = 0x7F000002


class Config(C.Structure):
    """Mirror of or_config (att1_oracle.h)."""

    _fields_ = [
        ("vocab", C.c_uint32), ("n_layers", C.c_uint32), ("n_heads", C.c_uint32),
        ("n_kv_heads", C.c_uint32), ("d_model", C.c_uint32), ("d_ff", C.c_uint32),
        ("max_seq", C.c_uint32), ("group", C.c_uint32), ("dtype", C.c_uint32),
        ("eps", C.c_float), ("final_eps", C.c_float), ("theta", C.c_float),
    ]

    @classmethod
    def make(cls, vocab, n_layers, n_heads, n_kv_heads, d_model, d_ff, max_seq,
             dtype=Q4, group=32, eps=1e-5, final_eps=None, theta=10000.0):
        return cls(vocab, n_layers, n_heads, n_kv_heads, d_model, d_ff, max_seq,
                   group, dtype, eps, eps if final_eps is None else final_eps, theta)

    def as_dict(self):
        return {k: getattr(self, k) for k, _ in self._fields_}


def build(ref: bool = True) -> None:
    """Build liboracle.so (and _ref when the reference sources exist)."""
    targets = ["oracle"] + (["ref"] if ref else [])
    subprocess.run(["make", "-s", "-C", HERE] + targets, check=True)


def _fp(a):
    return a.ctypes.data_as(C.POINTER(C.c_float))


def _u8(a):
    return a.ctypes.data_as(C.POINTER(C.c_uint8))


def _i8(a):
    return a.ctypes.data_as(C.POINTER(C.c_int8))


_F = C.POINTER(C.c_float)
_U8 = C.POINTER(C.c_uint8)
_I8 = C.POINTER(C.c_int8)
_SZ = C.c_size_t


class _Lib:
    prefix = ""

    def _sig(self, name, res, *args):
        f = getattr(self.lib, name)
        f.restype = res
        f.argtypes = list(args)
        return f


class Oracle(_Lib):
    """The CPU restatement (att1_oracle.c)."""

    def __init__(self, path: str = ORACLE_SO):
        if not os.path.exists(path):
            build(ref=False)
        self.lib = C.CDLL(path)
        s = self._sig
        s("or_q4_quantize", C.c_int, _F, _SZ, _SZ, C.c_uint32, _U8, _F)
        s("or_q8_quantize", C.c_int, _F, _SZ, _SZ, _I8, _F)
        s("or_matmul_q4", C.c_int, _F, _F, _SZ, _SZ, _U8, _F, _SZ, C.c_uint32, C.c_int)
        s("or_matmul_q8", C.c_int, _F, _F, _SZ, _SZ, _I8, _F, _SZ, C.c_int)
        s("or_rmsnorm", C.c_int, _F, _F, _F, _SZ, C.c_float)
        s("or_softmax", C.c_int, _F, _SZ)
        s("or_rope", C.c_int, _F, _SZ, _SZ, C.c_float)
        s("or_swiglu", C.c_int, _F, _F, _F, _SZ)
        s("or_argmax", C.c_int, _F, _SZ, C.POINTER(C.c_uint32))
        s("or_synth_normal", None, C.c_uint64, C.c_uint64, C.c_uint64, _SZ, C.c_float, _F)
        s("or_synth_token", C.c_uint32, C.c_uint64, C.c_uint64, C.c_uint32)
        s("or_model_synth", C.c_void_p, C.POINTER(Config), C.c_uint64, C.c_int)
        s("or_model_free", None, C.c_void_p)
        s("or_model_q4_view", C.c_int, C.c_void_p, C.c_uint32, C.c_uint32,
          C.POINTER(_U8), C.POINTER(_F), C.POINTER(_SZ), C.POINTER(_SZ))
        s("or_model_q8_view", C.c_int, C.c_void_p, C.c_uint32, C.c_uint32,
          C.POINTER(_I8), C.POINTER(_F), C.POINTER(_SZ), C.POINTER(_SZ))
        s("or_state_create", C.c_void_p, C.c_void_p)
        s("or_state_free", None, C.c_void_p)
        s("or_state_position", _SZ, C.c_void_p)
        s("or_state_keys", _F, C.c_void_p, C.c_uint32)
        s("or_state_values", _F, C.c_void_p, C.c_uint32)
        s("or_decode", C.c_int, C.c_void_p, C.c_void_p, C.c_uint32, _F,
          C.POINTER(C.c_uint32), C.c_int)
        s("or_state_import_kv", C.c_int, C.c_void_p, C.c_void_p, C.c_uint32, _SZ, _F, _F)
        s("or_state_seek", C.c_int, C.c_void_p, C.c_void_p, _SZ)

    # ---- element functions ----
    def synth_normal(self, seed, tensor_id, count, std=0.02, first=0):
        out = np.empty(count, np.float32)
        self.lib.or_synth_normal(seed, tensor_id, first, count, std, _fp(out))
        return out

    def synth_tokens(self, seed, count, vocab, first=0):
        return np.array([self.lib.or_synth_token(seed, first + i, vocab)
                         for i in range(count)], np.uint32)

    def q4_quantize(self, w, group=32):
        w = np.ascontiguousarray(w, np.float32)
        rows, cols = w.shape
        packed = np.zeros(rows * cols // 2, np.uint8)
        scales = np.zeros(rows * (cols // group), np.float32)
        rc = self.lib.or_q4_quantize(_fp(w), rows, cols, group, _u8(packed), _fp(scales))
        if rc != 0:
            raise ValueError("q4 quantise rejected its input")
        return packed, scales

    def q8_quantize(self, w):
        w = np.ascontiguousarray(w, np.float32)
        rows, cols = w.shape
        values = np.zeros(rows * cols, np.int8)
        scales = np.zeros(rows, np.float32)
        rc = self.lib.or_q8_quantize(_fp(w), rows, cols, _i8(values), _fp(scales))
        if rc != 0:
            raise ValueError("q8 quantise rejected its input")
        return values, scales

    def matmul_q4(self, x, packed, scales, rows, cols, group=32, threads=1):
        x = np.ascontiguousarray(x, np.float32).reshape(-1, cols)
        out = np.zeros((x.shape[0], rows), np.float32)
        rc = self.lib.or_matmul_q4(_fp(out), _fp(x), x.shape[0], cols, _u8(packed),
                                   _fp(scales), rows, group, threads)
        if rc != 0:
            raise ValueError("matmul_q4 failed")
        return out

    def matmul_q8(self, x, values, scales, rows, cols, threads=1):
        x = np.ascontiguousarray(x, np.float32).reshape(-1, cols)
        out = np.zeros((x.shape[0], rows), np.float32)
        rc = self.lib.or_matmul_q8(_fp(out), _fp(x), x.shape[0], cols, _i8(values),
                                   _fp(scales), rows, threads)
        if rc != 0:
            raise ValueError("matmul_q8 failed")
        return out

    def rmsnorm(self, x, w, eps):
        x = np.ascontiguousarray(x, np.float32)
        w = np.ascontiguousarray(w, np.float32)
        out = np.empty_like(x)
        assert self.lib.or_rmsnorm(_fp(out), _fp(x), _fp(w), x.size, eps) == 0
        return out

    def rope(self, v, pos, theta):
        v = np.array(v, np.float32)
        assert self.lib.or_rope(_fp(v), v.size, pos, theta) == 0
        return v

    def softmax(self, v):
        v = np.array(v, np.float32)
        assert self.lib.or_softmax(_fp(v), v.size) == 0
        return v

    def swiglu(self, g, u):
        g = np.ascontiguousarray(g, np.float32)
        u = np.ascontiguousarray(u, np.float32)
        out = np.empty_like(g)
        assert self.lib.or_swiglu(_fp(out), _fp(g), _fp(u), g.size) == 0
        return out

    def argmax(self, v):
        v = np.ascontiguousarray(v, np.float32)
        o = C.c_uint32(0)
        rc = self.lib.or_argmax(_fp(v), v.size, C.byref(o))
        return None if rc != 0 else int(o.value)

    # ---- model ----
    def model(self, cfg: Config, seed: int, threads: int = 1) -> "OracleModel":
        return OracleModel(self, cfg, seed, threads)


class OracleModel:
    def __init__(self, orc: Oracle, cfg: Config, seed: int, threads: int = 1):
        self.o = orc
        self.cfg = cfg
        self.seed = seed
        self.threads = threads
        self.ptr = orc.lib.or_model_synth(C.byref(cfg), seed, threads)
        if not self.ptr:
            raise MemoryError("or_model_synth failed")
        self.state = orc.lib.or_state_create(self.ptr)
        if not self.state:
            raise MemoryError("or_state_create failed")

    def close(self):
        if self.state:
            self.o.lib.or_state_free(self.state)
            self.state = None
        if self.ptr and getattr(self, "owner", True):
            self.o.lib.or_model_free(self.ptr)
        self.ptr = None

    def spawn(self) -> "OracleModel":
        """Another decode state (sequence) over the same weights; close it before
        the model it was spawned from."""
        other = OracleModel.__new__(OracleModel)
        other.o, other.cfg, other.seed, other.threads = self.o, self.cfg, self.seed, self.threads
        other.ptr, other.owner = self.ptr, False
        other.state = self.o.lib.or_state_create(self.ptr)
        if not other.state:
            raise MemoryError("or_state_create failed")
        return other

    __del__ = close

    def reset(self):
        self.o.lib.or_state_free(self.state)
        self.state = self.o.lib.or_state_create(self.ptr)

    @property
    def position(self):
        return self.o.lib.or_state_position(self.state)

    def decode(self, token):
        logits = np.zeros(self.cfg.vocab, np.float32)
        nxt = C.c_uint32(0)
        rc = self.o.lib.or_decode(self.ptr, self.state, int(token), _fp(logits),
                                  C.byref(nxt), self.threads)
        if rc != 0:
            raise RuntimeError("or_decode failed")
        return logits, int(nxt.value)

    def q4(self, layer, kind):
        p, s, r, c = _U8(), _F(), _SZ(), _SZ()
        if self.o.lib.or_model_q4_view(self.ptr, layer, kind, C.byref(p), C.byref(s),
                                       C.byref(r), C.byref(c)) != 0:
            raise KeyError((layer, kind))
        rows, cols = r.value, c.value
        packed = np.ctypeslib.as_array(p, (rows * cols // 2,)).copy()
        scales = np.ctypeslib.as_array(s, (rows * (cols // self.cfg.group),)).copy()
        return packed, scales, rows, cols

    def q8(self, layer, kind):
        p, s, r, c = _I8(), _F(), _SZ(), _SZ()
        if self.o.lib.or_model_q8_view(self.ptr, layer, kind, C.byref(p), C.byref(s),
                                       C.byref(r), C.byref(c)) != 0:
            raise KeyError((layer, kind))
        rows, cols = r.value, c.value
        values = np.ctypeslib.as_array(p, (rows * cols,)).copy()
        scales = np.ctypeslib.as_array(s, (rows,)).copy()
        return values, scales, rows, cols

    def import_kv(self, layer, keys, values):
        """K/V rows [0, count) of one layer, each [count][n_kv_heads][head_dim]."""
        keys = np.ascontiguousarray(keys, np.float32)
        values = np.ascontiguousarray(values, np.float32)
        hd = self.cfg.d_model // self.cfg.n_heads
        count = keys.size // (self.cfg.n_kv_heads * hd)
        assert keys.size == values.size == count * self.cfg.n_kv_heads * hd
        if self.o.lib.or_state_import_kv(self.ptr, self.state, layer, count, _fp(keys), _fp(values)) != 0:
            raise ValueError("or_state_import_kv rejected its arguments")

    def seek(self, position):
        if self.o.lib.or_state_seek(self.ptr, self.state, position) != 0:
            raise ValueError("or_state_seek rejected the position")

    def keys(self, layer):
        hd = self.cfg.d_model // self.cfg.n_heads
        n = self.cfg.max_seq * self.cfg.n_kv_heads * hd
        return np.ctypeslib.as_array(self.o.lib.or_state_keys(self.state, layer), (n,)).copy()

    def values(self, layer):
        hd = self.cfg.d_model // self.cfg.n_heads
        n = self.cfg.max_seq * self.cfg.n_kv_heads * hd
        return np.ctypeslib.as_array(self.o.lib.or_state_values(self.state, layer), (n,)).copy()


class Reference(_Lib):
    """The reference sources compiled into _ref/libatt1ref.so + ref_harness.c."""

    def __init__(self, path: str = REF_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        self.lib = C.CDLL(path)
        s = self._sig
        s("rh_model_synth", C.c_void_p, C.POINTER(Config), C.c_uint64, C.c_int)
        s("rh_model_free", None, C.c_void_p)
        s("rh_model_set_threads", None, C.c_void_p, C.c_int)
        s("rh_model_q4_view", C.c_int, C.c_void_p, C.c_uint32, C.c_uint32,
          C.POINTER(_U8), C.POINTER(_F), C.POINTER(_SZ), C.POINTER(_SZ))
        s("rh_state_create", C.c_void_p, C.c_void_p)
        s("rh_state_free", None, C.c_void_p, C.c_void_p)
        s("rh_state_fill", C.c_int, C.c_void_p, C.c_void_p, _SZ, C.c_uint64)
        s("rh_decode", C.c_int, C.c_void_p, C.c_void_p, C.c_uint32, _F,
          C.POINTER(C.c_uint32))
        s("rh_quantize_q4", C.c_int, _F, _SZ, _SZ, C.c_uint32, _U8, _F)
        s("rh_quantize_q8", C.c_int, _F, _SZ, _SZ, _I8, _F)
        s("rh_matmul_q4", C.c_int, _F, _F, _SZ, _SZ, _U8, _F, _SZ, C.c_uint32)
        s("rh_matmul_q8", C.c_int, _F, _F, _SZ, _SZ, _I8, _F, _SZ)
        s("rh_pack_group", C.c_int, _I8, C.c_uint32, _U8)
        s("rh_unpack_group", C.c_int, _U8, C.c_uint32, _I8)
        s("rh_quantize_group", C.c_int, _F, C.c_uint32, _U8, _F)
        s("rh_rmsnorm", C.c_int, _F, _F, _F, _SZ, C.c_float)
        s("rh_softmax", C.c_int, _F, _SZ)
        s("rh_rope", C.c_int, _F, _SZ, _SZ, C.c_float)
        s("rh_swiglu", C.c_int, _F, _F, _F, _SZ)
        s("rh_argmax", C.c_int, _F, _SZ, C.POINTER(C.c_uint32))

    def q4_quantize(self, w, group=32):
        w = np.ascontiguousarray(w, np.float32)
        rows, cols = w.shape
        packed = np.zeros(rows * cols // 2, np.uint8)
        scales = np.zeros(rows * (cols // group), np.float32)
        if self.lib.rh_quantize_q4(_fp(w), rows, cols, group, _u8(packed), _fp(scales)) != 0:
            raise ValueError("reference q4 quantise rejected its input")
        return packed, scales

    def q8_quantize(self, w):
        w = np.ascontiguousarray(w, np.float32)
        rows, cols = w.shape
        values = np.zeros(rows * cols, np.int8)
        scales = np.zeros(rows, np.float32)
        if self.lib.rh_quantize_q8(_fp(w), rows, cols, _i8(values), _fp(scales)) != 0:
            raise ValueError("reference q8 quantise rejected its input")
        return values, scales

    def matmul_q4(self, x, packed, scales, rows, cols, group=32):
        x = np.ascontiguousarray(x, np.float32).reshape(-1, cols)
        out = np.zeros((x.shape[0], rows), np.float32)
        assert self.lib.rh_matmul_q4(_fp(out), _fp(x), x.shape[0], cols, _u8(packed),
                                     _fp(scales), rows, group) == 0
        return out

    def matmul_q8(self, x, values, scales, rows, cols):
        x = np.ascontiguousarray(x, np.float32).reshape(-1, cols)
        out = np.zeros((x.shape[0], rows), np.float32)
        assert self.lib.rh_matmul_q8(_fp(out), _fp(x), x.shape[0], cols, _i8(values),
                                     _fp(scales), rows) == 0
        return out

    def model(self, cfg: Config, seed: int, threads: int = 1) -> "ReferenceModel":
        return ReferenceModel(self, cfg, seed, threads)


class ReferenceModel:
    def __init__(self, ref: Reference, cfg: Config, seed: int, threads: int = 1):
        self.r = ref
        self.cfg = cfg
        self.ptr = ref.lib.rh_model_synth(C.byref(cfg), seed, threads)
        if not self.ptr:
            raise MemoryError("rh_model_synth failed")
        self.state = ref.lib.rh_state_create(self.ptr)
        if not self.state:
            raise MemoryError("rh_state_create failed")

    def close(self):
        if self.state:
            self.r.lib.rh_state_free(self.ptr, self.state)
            self.state = None
        if self.ptr:
            self.r.lib.rh_model_free(self.ptr)
            self.ptr = None

    __del__ = close

    def set_threads(self, n):
        self.r.lib.rh_model_set_threads(self.ptr, n)

    def fill(self, length, seed=1):
        assert self.r.lib.rh_state_fill(self.ptr, self.state, length, seed) == 0

    def decode(self, token):
        logits = np.zeros(self.cfg.vocab, np.float32)
        nxt = C.c_uint32(0)
        if self.r.lib.rh_decode(self.ptr, self.state, int(token), _fp(logits),
                                C.byref(nxt)) != 0:
            raise RuntimeError("rh_decode failed")
        return logits, int(nxt.value)

    def q4(self, layer, kind):
        p, s, r, c = _U8(), _F(), _SZ(), _SZ()
        if self.r.lib.rh_model_q4_view(self.ptr, layer, kind, C.byref(p), C.byref(s),
                                       C.byref(r), C.byref(c)) != 0:
            raise KeyError((layer, kind))
        rows, cols = r.value, c.value
        packed = np.ctypeslib.as_array(p, (rows * cols // 2,)).copy()
        scales = np.ctypeslib.as_array(s, (rows * (cols // self.cfg.group),)).copy()
        return packed, scales, rows, cols
