"""ctypes bindings of libatt1_b200.so (the C ABI in include/*.h).

This is a thin host-side mirror of the ATT-1 C API for Python callers (the
tests and bench.py): the same function names, argument meaning and status
codes. All compute happens in the library's sm_100a kernels; there is no
Python or CPU fallback - loading fails loudly when the library is missing.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libatt1_b200.so")

ATT1_OK = 0
STATUS = {0: "OK", -1: "INVALID_ARG", -2: "OOM", -3: "IO", -4: "BAD_FORMAT", -5: "NOT_FOUND",
          -6: "SHAPE", -7: "QUEUE_FULL", -8: "STATE", -9: "UNSUPPORTED", -10: "QUEUE_EMPTY",
          -11: "TIMEOUT", -12: "ALREADY_STARTED"}
WQ, WK, WV, WO, GATE, UP, DOWN, OUTPUT = 1, 2, 3, 4, 6, 7, 8, 9
EPI_STORE, EPI_RESID, EPI_QKV, EPI_SWIGLU, EPI_LOGITS = range(5)
ROWS_PLAIN, ROWS_GATEUP = 0, 1


class Att1Error(RuntimeError):
    def __init__(self, fn, rc):
        super().__init__(f"{fn} failed: {STATUS.get(rc, rc)}")
        self.rc = rc


class Config(C.Structure):
    """att1_b200_config (include/att1_b200.h)."""

    _fields_ = [
        ("vocab", C.c_uint32), ("n_layers", C.c_uint32), ("n_heads", C.c_uint32),
        ("n_kv_heads", C.c_uint32), ("d_model", C.c_uint32), ("d_ff", C.c_uint32),
        ("max_seq", C.c_uint32), ("group", C.c_uint32), ("dtype", C.c_uint32),
        ("eps", C.c_float), ("final_eps", C.c_float), ("theta", C.c_float),
    ]

    @classmethod
    def make(cls, vocab, n_layers, n_heads, n_kv_heads, d_model, d_ff, max_seq,
             dtype=4, group=32, eps=1e-5, final_eps=None, theta=10000.0):
        return cls(vocab, n_layers, n_heads, n_kv_heads, d_model, d_ff, max_seq, group, dtype,
                   eps, eps if final_eps is None else final_eps, theta)


class QWeight(C.Structure):
    _fields_ = [("data", C.c_void_p), ("row_scale", C.c_void_p), ("format", C.c_uint32),
                ("rows", C.c_uint32), ("cols", C.c_uint32), ("tiles", C.c_uint32),
                ("kunits", C.c_uint32)]


class KVLayout(C.Structure):
    _fields_ = [("k_pool", C.c_void_p), ("v_pool", C.c_void_p), ("page_table", C.c_void_p),
                ("page_tokens", C.c_uint32), ("pages_per_seq", C.c_uint32),
                ("n_kv_heads", C.c_uint32), ("head_dim", C.c_uint32)]


class TpArgs(C.Structure):
    """b2_tp (include/b2_kernels.h): tensor-parallel exchange of one kernel."""
    _fields_ = [("rank", C.c_uint32), ("world", C.c_uint32), ("peer", C.c_void_p * 8), ("points", C.c_uint32),
                ("slot_floats", C.c_uint32), ("logit_floats", C.c_uint32), ("epoch", C.c_void_p),
                ("done", C.c_void_p), ("out_point", C.c_uint32), ("in_point", C.c_uint32),
                ("in_resid", C.c_void_p), ("in_out", C.c_void_p), ("row_offset", C.c_uint32),
                ("wait_polls", C.c_uint32)]


class GemvArgs(C.Structure):
    _fields_ = [("w", QWeight), ("batch", C.c_uint32), ("x", C.c_void_p), ("x_stride", C.c_uint32),
                ("norm_w", C.c_void_p), ("eps", C.c_float), ("epilogue", C.c_int),
                ("out", C.c_void_p), ("out_stride", C.c_uint32), ("resid", C.c_void_p),
                ("q_rows", C.c_uint32), ("kv_rows", C.c_uint32), ("rope_freq", C.c_void_p),
                ("positions", C.c_void_p), ("kv", KVLayout), ("argmax", C.c_void_p),
                ("scratch", C.c_void_p), ("scratch_bytes", C.c_size_t), ("counters", C.c_void_p),
                ("counters_len", C.c_uint32), ("err", C.c_void_p), ("pdl", C.c_int), ("grid", C.c_int),
                ("tp", TpArgs)]


class GemmArgs(C.Structure):
    """b2_gemm_args (include/b2_kernels.h): dequant GEMM on the tensor cores."""
    _fields_ = [("w", QWeight), ("xs", C.c_void_p), ("m", C.c_uint32), ("epilogue", C.c_uint32),
                ("out", C.c_void_p), ("out_stride", C.c_uint32), ("resid", C.c_void_p),
                ("scratch", C.c_void_p), ("scratch_bytes", C.c_size_t), ("splits", C.c_uint32),
                ("err", C.c_void_p), ("pdl", C.c_int)]


class AttnArgs(C.Structure):
    _fields_ = [("batch", C.c_uint32), ("n_heads", C.c_uint32), ("n_kv_heads", C.c_uint32),
                ("head_dim", C.c_uint32), ("q", C.c_void_p), ("kv", KVLayout),
                ("positions", C.c_void_p), ("max_ctx", C.c_uint32), ("ctx", C.c_void_p),
                ("scratch", C.c_void_p), ("scratch_bytes", C.c_size_t), ("counters", C.c_void_p),
                ("counters_len", C.c_uint32), ("err", C.c_void_p), ("pdl", C.c_int)]


class ModelTensor(C.Structure):
    _fields_ = [("name", C.c_char * 64), ("dtype", C.c_uint32), ("ndims", C.c_uint32),
                ("shape", C.c_uint64 * 4), ("offset", C.c_uint64), ("nbytes", C.c_uint64),
                ("shard_id", C.c_uint32), ("flags", C.c_uint32), ("data", C.c_void_p)]


class ModelConfig(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in ("vocab_size", "n_layers", "n_heads", "d_model", "d_ff",
                                          "max_seq_len", "rope_dim", "n_tiles", "shard_count")]


class Model(C.Structure):
    _fields_ = [("config", ModelConfig), ("tensor_count", C.c_uint64),
                ("tensors", C.POINTER(ModelTensor)), ("file_data", C.c_void_p),
                ("file_size", C.c_size_t)]


class TraceCounters(C.Structure):
    _fields_ = [(n, C.c_uint64) for n in (
        "tokens_decoded", "token_time_us_total", "token_time_us_max", "layer_time_us_total",
        "activation_bytes_sent", "logits_bytes_produced", "fabric_packets_sent",
        "fabric_packets_received", "fabric_payload_bytes_sent", "fabric_payload_bytes_received",
        "kv_appends", "kv_key_reads", "kv_value_reads", "tile_layer_executions")]


class SamplerConfig(C.Structure):
    """att1_sampler_config (include/att1_sampler.h)."""
    _fields_ = [("top_k", C.c_uint32), ("temperature", C.c_float)]


class KvMmuConfig(C.Structure):
    """att1_kv_mmu_config (include/att1_kv_mmu.h)."""
    _fields_ = [(n, C.c_size_t) for n in ("max_sessions", "max_pages", "num_layers", "num_heads", "head_dim",
                                          "page_tokens", "max_positions")]


class KvMmuCounters(C.Structure):
    _fields_ = [(n, C.c_uint64) for n in ("page_hits", "page_misses", "page_allocations", "append_ops",
                                          "read_ops", "range_copy_ops", "errors")]


class KvMmuPageRef(C.Structure):
    _fields_ = [("physical_page", C.c_uint64), ("session_id", C.c_uint64), ("layer_id", C.c_size_t),
                ("logical_page", C.c_size_t), ("page_tokens", C.c_size_t)]


class TileCounters(C.Structure):
    """att1_cluster_tile_counters (include/att1_cluster_infer.h)."""
    _fields_ = [("activations_received", C.c_uint64), ("activations_sent", C.c_uint64),
                ("layers_run", C.c_uint64), ("logits_sent", C.c_uint64), ("layer_start", C.c_uint32),
                ("layer_end", C.c_uint32)]


class ClusterConfig(C.Structure):
    _fields_ = [("tile_count", C.c_size_t), ("fabric_queue_capacity", C.c_size_t),
                ("fabric_max_payload_bytes", C.c_size_t), ("shard_plan_mode", C.c_int)]


_P = C.c_void_p
_U32 = C.c_uint32
_SZ = C.c_size_t
_F = C.c_float

_SIGS = {
    # model / infer API (att1_model.h, att1_infer.h)
    "att1_model_load": (C.c_int, [C.c_char_p, C.POINTER(Model)]),
    "att1_model_free": (None, [C.POINTER(Model)]),
    "att1_model_find_tensor": (C.POINTER(ModelTensor), [C.POINTER(Model), C.c_char_p]),
    "att1_infer_create": (C.c_int, [C.POINTER(Model), C.POINTER(_P)]),
    "att1_infer_create_q4": (C.c_int, [C.POINTER(Model), C.POINTER(_P)]),
    "att1_infer_destroy": (None, [_P]),
    "att1_infer_decode_token": (C.c_int, [_P, _U32, C.POINTER(_U32)]),
    "att1_infer_generate": (C.c_int, [_P, C.c_char_p, _SZ, _SZ, C.POINTER(_U32), _SZ, C.POINTER(_SZ)]),
    "att1_infer_logits": (C.POINTER(_F), [_P, C.POINTER(_SZ)]),
    "att1_infer_position": (C.c_int, [_P, C.POINTER(_SZ)]),
    "att1_infer_layer_kv_length": (C.c_int, [_P, _U32, C.POINTER(_SZ)]),
    "att1_infer_set_trace": (C.c_int, [_P, _P]),
    "att1_infer_set_backend": (C.c_int, [_P, _P]),
    # additions (att1_b200.h)
    "att1_b200_infer_create_synth": (C.c_int, [C.POINTER(Config), C.c_uint64, _U32, C.POINTER(_P)]),
    "att1_b200_infer_create_synth_tp": (C.c_int, [C.POINTER(Config), C.c_uint64, _U32, _U32, _U32, C.POINTER(_P)]),
    "att1_b200_infer_tp_handle": (C.c_int, [_P, _P]),
    "att1_b200_infer_tp_connect": (C.c_int, [_P, _P]),
    "att1_b200_infer_tp_connect_local": (C.c_int, [C.POINTER(_P), _U32]),
    "att1_b200_nccl_unique_id": (C.c_int, [_P]),
    "att1_b200_infer_tp_connect_nccl": (C.c_int, [_P, _P]),
    "att1_b200_infer_tp_set_wait": (C.c_int, [_P, _U32]),
    "att1_b200_infer_tp_reset": (C.c_int, [_P]),
    "att1_b200_infer_tp_disconnect": (C.c_int, [_P]),
    "att1_b200_infer_step_async": (C.c_int, [_P, C.POINTER(_U32)]),
    "att1_b200_infer_step_wait": (C.c_int, [_P, C.POINTER(_U32)]),
    "att1_b200_set_device": (C.c_int, [C.c_int]),
    "att1_b200_infer_create_model": (C.c_int, [C.POINTER(Model), _U32, _F, _F, _F, C.POINTER(_P)]),
    "att1_b200_infer_batch": (_U32, [_P]),
    "att1_b200_infer_decode_batch": (C.c_int, [_P, C.POINTER(_U32), C.POINTER(_U32)]),
    "att1_b200_infer_prefill": (C.c_int, [_P, C.POINTER(_U32), _SZ, C.POINTER(_U32)]),
    "att1_b200_infer_logits_batch": (C.POINTER(_F), [_P, C.POINTER(_SZ)]),
    "att1_b200_infer_set_options": (C.c_int, [_P, C.c_int, C.c_int]),
    "att1_b200_infer_set_persistent": (C.c_int, [_P, C.c_int]),
    "att1_b200_infer_run_steps": (C.c_int, [_P, _U32]),
    "att1_b200_infer_sync": (C.c_int, [_P]),
    "att1_b200_infer_stream": (_P, [_P]),
    "att1_b200_infer_export_q4": (C.c_int, [_P, _U32, _U32, _P, _P]),
    "att1_b200_infer_export_q8": (C.c_int, [_P, _U32, _U32, _P, _P]),
    "att1_b200_infer_export_kv": (C.c_int, [_P, _U32, _U32, _SZ, _P, _P]),
    "att1_b200_infer_import_kv": (C.c_int, [_P, _U32, _U32, _SZ, _P, _P]),
    "att1_b200_infer_seek": (C.c_int, [_P, _SZ]),
    "att1_b200_infer_device_bytes": (_SZ, [_P]),
    "att1_b200_infer_step_launches": (_SZ, [_P]),
    # backend vtable (att1_backend.h)
    "att1_backend_cuda_available": (C.c_int, []),
    "att1_backend_cuda_create": (C.c_int, [C.POINTER(_P)]),
    "att1_backend_cuda_q8_create": (C.c_int, [C.POINTER(_P)]),
    "att1_backend_cuda_q4_create": (C.c_int, [C.POINTER(_P)]),
    "att1_backend_default_create": (C.c_int, [C.POINTER(_P)]),
    "att1_backend_destroy": (None, [_P]),
    # trace
    "att1_trace_create": (C.c_int, [_SZ, _SZ, C.POINTER(_P)]),
    "att1_trace_destroy": (None, [_P]),
    "att1_trace_snapshot": (C.c_int, [_P, C.POINTER(TraceCounters)]),
    # cluster
    "att1_cluster_infer_create_q4": (C.c_int, [C.POINTER(Model), C.POINTER(ClusterConfig), C.POINTER(_P)]),
    "att1_cluster_infer_create": (C.c_int, [C.POINTER(Model), C.POINTER(ClusterConfig), C.POINTER(_P)]),
    "att1_cluster_infer_destroy": (None, [_P]),
    "att1_cluster_infer_decode_token": (C.c_int, [_P, _U32, C.POINTER(_U32)]),
    "att1_cluster_infer_logits": (C.POINTER(_F), [_P, C.POINTER(_SZ)]),
    "att1_cluster_infer_get_tile_counters": (C.c_int, [_P, _U32, C.POINTER(TileCounters)]),
    "att1_cluster_infer_position": (C.c_int, [_P, C.POINTER(_SZ)]),
    "att1_b200_infer_create_model_tp": (C.c_int, [C.POINTER(Model), _U32, _F, _F, _F, _U32, _U32, C.POINTER(_P)]),
    # KV-MMU (att1_kv_mmu.h)
    "att1_kv_mmu_create": (C.c_int, [C.POINTER(KvMmuConfig), C.POINTER(_P)]),
    "att1_kv_mmu_destroy": (None, [_P]),
    "att1_kv_mmu_create_session": (C.c_int, [_P, C.c_uint64]),
    "att1_kv_mmu_destroy_session": (C.c_int, [_P, C.c_uint64]),
    "att1_kv_mmu_append": (C.c_int, [_P, C.c_uint64, _SZ, _SZ, _P, _P]),
    "att1_kv_mmu_read": (C.c_int, [_P, C.c_uint64, _SZ, _SZ, _SZ, _P, _P]),
    "att1_kv_mmu_copy_range": (C.c_int, [_P, C.c_uint64, _SZ, _SZ, _SZ, _SZ, _P, _P]),
    "att1_kv_mmu_lookup_page": (C.c_int, [_P, C.c_uint64, _SZ, _SZ, C.POINTER(KvMmuPageRef)]),
    "att1_kv_mmu_get_counters": (None, [_P, C.POINTER(KvMmuCounters)]),
    "att1_kv_mmu_reset_counters": (None, [_P]),
    "att1_b200_kv_mmu_layout": (C.c_int, [_P, C.c_uint64, _SZ, C.POINTER(KVLayout)]),
    "att1_b200_infer_use_kv_mmu": (C.c_int, [_P, _P, C.POINTER(C.c_uint64)]),
    "att1_b200_infer_set_sampler": (C.c_int, [_P, C.POINTER(SamplerConfig), C.c_uint64]),
    "att1_sampler_greedy_f32": (C.c_int, [_P, _SZ, C.POINTER(C.c_uint32)]),
    "b2_sample_topk": (C.c_int, [_P, _U32, _U32, _U32, _U32, C.c_float, C.c_uint64, _P, _P, C.c_int, _P]),
    "b2_sample_topk_sharded": (C.c_int, [_P, _U32, _U32, _U32, _SZ, _U32, _U32, C.c_float, C.c_uint64, _P, _P,
                                         C.c_int, _P]),
    # kernel ABI (b2_kernels.h)
    "b2_q4_bytes": (_SZ, [_U32, _U32]),
    "b2_q8_bytes": (_SZ, [_U32, _U32]),
    "b2_q4_pack": (C.c_int, [_P, _U32, _U32, _U32, _P, _P, _P, _P, _U32, C.c_int, _P]),
    "b2_q4_unpack": (C.c_int, [_P, _P, _P, _U32, _U32, _U32, C.c_int, C.c_int, _P]),
    "b2_q4_synth": (C.c_int, [_P, _U32, _U32, _U32, C.c_uint64, C.c_uint64, C.c_uint64, _F, C.c_int, _P]),
    "b2_q8_pack": (C.c_int, [_P, _P, _U32, _U32, _U32, _P, _P, _P, _P, C.c_int, _P]),
    "b2_q8_unpack": (C.c_int, [_P, _P, _P, _P, _U32, _U32, _U32, C.c_int, C.c_int, _P]),
    "b2_q8_synth": (C.c_int, [_P, _P, _U32, _U32, _U32, C.c_uint64, C.c_uint64, C.c_uint64, _F, C.c_int, _P]),
    "b2_q8_quantize_f32": (C.c_int, [_P, _P, _U32, _U32, _U32, _P, _P, C.c_int, C.c_int, _P]),
    "b2_synth_f32": (C.c_int, [_P, _SZ, C.c_uint64, C.c_uint64, _F, _P]),
    "b2_gemv_scratch_bytes": (_SZ, [C.POINTER(GemvArgs)]),
    "b2_gemv_counters_len": (_U32, [C.POINTER(GemvArgs)]),
    "b2_attn_counters_len": (_U32, [C.POINTER(AttnArgs)]),
    "b2_gemv": (C.c_int, [C.POINTER(GemvArgs), _P]),
    "b2_attn_noalloc": (C.c_int, [C.POINTER(AttnArgs), _P]),
    "b2_gemm_xs_bytes": (_SZ, [_U32, _U32]),
    "b2_gemm_prep": (C.c_int, [_P, _U32, _U32, _U32, _P, _F, _P, _P, _P]),
    "b2_gemm_scratch_bytes": (_SZ, [C.POINTER(GemmArgs)]),
    "b2_gemm": (C.c_int, [C.POINTER(GemmArgs), _P]),
    "b2_attn_scratch_bytes": (_SZ, [C.POINTER(AttnArgs)]),
    "b2_attn": (C.c_int, [C.POINTER(AttnArgs), _P]),
    "b2_rmsnorm": (C.c_int, [_P, _P, _P, _U32, _F, _P]),
    "b2_softmax": (C.c_int, [_P, _U32, _P]),
    "b2_rope": (C.c_int, [_P, _U32, _U32, _F, _P]),
    "b2_swiglu": (C.c_int, [_P, _P, _P, _U32, _P]),
    "b2_argmax": (C.c_int, [_P, _U32, _P, _P]),
    "b2_sm_count": (C.c_int, []),
}

_lib = None


def lib() -> C.CDLL:
    """Load libatt1_b200.so (built by att-1_b200/build.py); raise if missing."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise FileNotFoundError(
                f"{LIB_PATH} is missing: build it with `python att-1_b200/build.py`")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


TP_HANDLE_BYTES = 64
NCCL_ID_BYTES = 128


def check(fn: str, rc: int) -> None:
    if rc != ATT1_OK:
        raise Att1Error(fn, rc)


def _ptr(a) -> int:
    """Device or host address of a torch tensor / numpy array."""
    if a is None:
        return None
    if hasattr(a, "data_ptr"):
        return a.data_ptr()
    return a.ctypes.data


class Infer:
    """Owner of an att1_infer_t (single device)."""

    def __init__(self, handle: int, vocab: int, batch: int):
        self.h = C.c_void_p(handle)
        self.vocab = vocab
        self.batch = batch

    @classmethod
    def synth(cls, cfg: Config, seed: int, batch: int = 1) -> "Infer":
        h = C.c_void_p()
        check("att1_b200_infer_create_synth",
              lib().att1_b200_infer_create_synth(C.byref(cfg), seed, batch, C.byref(h)))
        return cls(h.value, cfg.vocab, batch)

    # ---- tensor parallelism (one context per GPU and rank) ----
    @classmethod
    def synth_tp(cls, cfg: Config, seed: int, rank: int, world: int, batch: int = 1, device: int = None) -> "Infer":
        """This rank's shard of the synthetic model, on `device` (default: rank)."""
        check("att1_b200_set_device", lib().att1_b200_set_device(rank if device is None else device))
        h = C.c_void_p()
        check("att1_b200_infer_create_synth_tp",
              lib().att1_b200_infer_create_synth_tp(C.byref(cfg), seed, batch, rank, world, C.byref(h)))
        return cls(h.value, cfg.vocab, batch)

    def tp_handle(self) -> bytes:
        buf = C.create_string_buffer(TP_HANDLE_BYTES)
        check("att1_b200_infer_tp_handle", lib().att1_b200_infer_tp_handle(self.h, buf))
        return buf.raw

    def tp_connect(self, handles) -> None:
        """handles: every rank's tp_handle() in rank order."""
        blob = b"".join(handles)
        check("att1_b200_infer_tp_connect", lib().att1_b200_infer_tp_connect(self.h, C.c_char_p(blob)))

    @staticmethod
    def nccl_unique_id() -> bytes:
        buf = C.create_string_buffer(NCCL_ID_BYTES)
        check("att1_b200_nccl_unique_id", lib().att1_b200_nccl_unique_id(buf))
        return buf.raw

    def tp_connect_nccl(self, nccl_id: bytes) -> None:
        """The NCCL comparison arm: every rank calls this with rank 0's id, together."""
        check("att1_b200_infer_tp_connect_nccl",
              lib().att1_b200_infer_tp_connect_nccl(self.h, C.c_char_p(bytes(nccl_id))))

    def tp_set_wait(self, polls: int) -> None:
        check("att1_b200_infer_tp_set_wait", lib().att1_b200_infer_tp_set_wait(self.h, polls))

    def tp_reset(self) -> None:
        check("att1_b200_infer_tp_reset", lib().att1_b200_infer_tp_reset(self.h))

    def tp_disconnect(self) -> None:
        check("att1_b200_infer_tp_disconnect", lib().att1_b200_infer_tp_disconnect(self.h))

    @staticmethod
    def tp_connect_local(ranks) -> None:
        arr = (_P * len(ranks))(*[r.h.value for r in ranks])
        check("att1_b200_infer_tp_connect_local", lib().att1_b200_infer_tp_connect_local(arr, len(ranks)))

    def step_async(self, tokens) -> None:
        t = (C.c_uint32 * self.batch)(*[int(x) for x in tokens])
        check("att1_b200_infer_step_async", lib().att1_b200_infer_step_async(self.h, t))

    def step_wait(self) -> np.ndarray:
        o = (C.c_uint32 * self.batch)()
        check("att1_b200_infer_step_wait", lib().att1_b200_infer_step_wait(self.h, o))
        return np.array(o[:], np.uint32)

    def close(self):
        if self.h and self.h.value:
            lib().att1_infer_destroy(self.h)
            self.h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def decode(self, token: int) -> int:
        out = C.c_uint32(0)
        check("att1_infer_decode_token", lib().att1_infer_decode_token(self.h, int(token), C.byref(out)))
        return int(out.value)

    def generate(self, prompt: bytes, count: int) -> np.ndarray:
        """att1_infer_generate: greedy continuation of a byte prompt."""
        out = (C.c_uint32 * max(count, 1))()
        n = C.c_size_t(0)
        check("att1_infer_generate", lib().att1_infer_generate(self.h, bytes(prompt), len(prompt), count, out,
                                                                 count, C.byref(n)))
        return np.array(out[:n.value], np.uint32)

    def prefill(self, tokens) -> int:
        """att1_b200_infer_prefill: the prompt in one pass; returns the greedy next token."""
        ids = np.ascontiguousarray(np.asarray(tokens, np.uint32))
        out = C.c_uint32(0)
        check("att1_b200_infer_prefill", lib().att1_b200_infer_prefill(
            self.h, ids.ctypes.data_as(C.POINTER(C.c_uint32)), ids.size, C.byref(out)))
        return int(out.value)

    def decode_batch(self, tokens) -> np.ndarray:
        t = (C.c_uint32 * self.batch)(*[int(x) for x in tokens])
        o = (C.c_uint32 * self.batch)()
        check("att1_b200_infer_decode_batch", lib().att1_b200_infer_decode_batch(self.h, t, o))
        return np.array(o[:], np.uint32)

    def set_sampler(self, top_k: int = 0, temperature: float = 1.0, seed: int = 0) -> None:
        """att1_b200_infer_set_sampler: top_k <= 1 is greedy."""
        cfg = SamplerConfig(int(top_k), float(temperature))
        check("att1_b200_infer_set_sampler", lib().att1_b200_infer_set_sampler(self.h, C.byref(cfg), int(seed)))

    def logits(self) -> np.ndarray:
        n = C.c_size_t(0)
        p = lib().att1_b200_infer_logits_batch(self.h, C.byref(n))
        if not p:
            raise Att1Error("att1_b200_infer_logits_batch", -8)
        return np.ctypeslib.as_array(p, (n.value,)).reshape(self.batch, self.vocab).copy()

    def position(self) -> int:
        n = C.c_size_t(0)
        check("att1_infer_position", lib().att1_infer_position(self.h, C.byref(n)))
        return n.value

    def set_options(self, graph=True, pdl=True, persistent=None):
        """graph / pdl apply to the per-operation kernel sequence; persistent
        selects the single-launch step (True) or that sequence (False)."""
        check("att1_b200_infer_set_options", lib().att1_b200_infer_set_options(self.h, int(graph), int(pdl)))
        if persistent is not None:
            check("att1_b200_infer_set_persistent", lib().att1_b200_infer_set_persistent(self.h, int(persistent)))

    def run_steps(self, n: int):
        check("att1_b200_infer_run_steps", lib().att1_b200_infer_run_steps(self.h, n))

    def sync(self):
        check("att1_b200_infer_sync", lib().att1_b200_infer_sync(self.h))

    def stream(self) -> int:
        return lib().att1_b200_infer_stream(self.h)

    def export_q4(self, layer: int, kind: int, rows: int, cols: int):
        packed = np.zeros(rows * cols // 2, np.uint8)
        scales = np.zeros(rows * (cols // 32), np.float32)
        check("att1_b200_infer_export_q4",
              lib().att1_b200_infer_export_q4(self.h, layer, kind, packed.ctypes.data, scales.ctypes.data))
        return packed, scales

    def export_q8(self, layer: int, kind: int, rows: int, cols: int):
        values = np.zeros(rows * cols, np.int8)
        scales = np.zeros(rows, np.float32)
        check("att1_b200_infer_export_q8",
              lib().att1_b200_infer_export_q8(self.h, layer, kind, values.ctypes.data, scales.ctypes.data))
        return values, scales

    def export_kv(self, item: int, layer: int, count: int, row: int):
        k = np.zeros(count * row, np.float32)
        v = np.zeros(count * row, np.float32)
        check("att1_b200_infer_export_kv",
              lib().att1_b200_infer_export_kv(self.h, item, layer, count, k.ctypes.data, v.ctypes.data))
        return k, v

    def import_kv(self, item: int, layer: int, keys, values, row: int):
        """K/V rows [0, count) of one sequence and layer, each [count][n_kv_heads][head_dim];
        row = n_kv_heads * head_dim of this context (its shard under tensor parallelism)."""
        k = np.ascontiguousarray(keys, np.float32).reshape(-1)
        v = np.ascontiguousarray(values, np.float32).reshape(-1)
        assert k.size == v.size and k.size % row == 0
        check("att1_b200_infer_import_kv",
              lib().att1_b200_infer_import_kv(self.h, item, layer, k.size // row, k.ctypes.data, v.ctypes.data))

    def seek(self, position: int):
        check("att1_b200_infer_seek", lib().att1_b200_infer_seek(self.h, position))

    def device_bytes(self) -> int:
        return lib().att1_b200_infer_device_bytes(self.h)

    def step_launches(self) -> int:
        """Operations in one step of the captured CUDA graph (0 before a graph step)."""
        return lib().att1_b200_infer_step_launches(self.h)
