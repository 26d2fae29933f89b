"""The C-ABI library without a GPU: it loads, exports every function that
include/*.h declares, parses .att1 files with the reference loader's
validation rules, and refuses device work cleanly when no B200 is present."""
import ctypes as C
import glob
import os
import re
import struct

import numpy as np
import pytest

import att1file

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        text = re.sub(r"typedef[^;]*;", "", text, flags=re.S)
        for m in re.finditer(r"\b([a-z][a-z0-9_]*)\s*\(", text):
            name = m.group(1)
            if name.startswith(("att1_", "b2_")):
                names.add(name)
    return sorted(names)


def test_library_exports_every_declared_function(b2):
    L = b2.lib()
    names = declared_functions()
    assert len(names) > 60
    missing = [n for n in names if not hasattr(L, n)]
    assert not missing, missing


def test_python_signatures_cover_exports(b2):
    for name in b2._SIGS:
        assert name in declared_functions(), name


def test_model_loader_round_trip(b2, orc, tmp_path):
    path = str(tmp_path / "m.att1")
    att1file.synth_model_file(path, orc, 64, 1, 2, 32, 64, 8, "q4", 1)
    L = b2.lib()
    m = b2.Model()
    assert L.att1_model_load(path.encode(), C.byref(m)) == 0
    assert (m.config.vocab_size, m.config.n_layers, m.config.n_heads, m.config.d_model, m.config.d_ff,
            m.config.max_seq_len) == (64, 1, 2, 32, 64, 8)
    names = [m.tensors[i].name.decode() for i in range(m.tensor_count)]
    assert "tok_embeddings.weight" in names and "output.weight" in names
    t = L.att1_model_find_tensor(C.byref(m), b"output.weight").contents
    assert t.nbytes == 64 * 32 // 2 + 64 * (32 // 32) * 4
    emb = L.att1_model_find_tensor(C.byref(m), b"tok_embeddings.weight").contents
    vals = np.ctypeslib.as_array(C.cast(emb.data, C.POINTER(C.c_float)), (64 * 32,))
    assert (vals == orc.synth_normal(1, 0x7F000000, 64 * 32)).all()
    assert not L.att1_model_find_tensor(C.byref(m), b"nope")
    L.att1_model_free(C.byref(m))


def _corrupt(path, offset, data):
    with open(path, "r+b") as f:
        f.seek(offset)
        f.write(data)


def test_model_loader_rejects_bad_files(b2, orc, tmp_path):
    L = b2.lib()
    m = b2.Model()
    assert L.att1_model_load(str(tmp_path / "missing.att1").encode(), C.byref(m)) == -3
    path = str(tmp_path / "m.att1")
    att1file.synth_model_file(path, orc, 64, 1, 2, 32, 64, 8, "q4", 1)
    raw = open(path, "rb").read()
    # bad magic
    _corrupt(path, 0, b"XXXX")
    assert L.att1_model_load(path.encode(), C.byref(m)) == -4
    open(path, "wb").write(raw)
    # unsupported version
    _corrupt(path, 8, struct.pack("<I", 7))
    assert L.att1_model_load(path.encode(), C.byref(m)) == -9
    open(path, "wb").write(raw)
    # first descriptor's nbytes off by one -> shape error
    desc_off = struct.unpack_from("<Q", raw, 32)[0]
    nb = struct.unpack_from("<Q", raw, desc_off + 112)[0]
    _corrupt(path, desc_off + 112, struct.pack("<Q", nb + 1))
    assert L.att1_model_load(path.encode(), C.byref(m)) == -6
    open(path, "wb").write(raw)
    # q4 group flag not a power of two -> shape error
    for i in range(struct.unpack_from("<Q", raw, 40)[0]):
        off = desc_off + 128 * i
        if struct.unpack_from("<I", raw, off + 64)[0] == 3:
            _corrupt(path, off + 124, struct.pack("<I", 48))
            break
    assert L.att1_model_load(path.encode(), C.byref(m)) == -6
    open(path, "wb").write(raw)
    # truncated file
    open(path, "wb").write(raw[: len(raw) // 2])
    assert L.att1_model_load(path.encode(), C.byref(m)) == -4


def test_null_arguments(b2):
    L = b2.lib()
    o = C.c_uint32()
    assert L.att1_infer_decode_token(None, 1, C.byref(o)) == -1
    assert L.att1_infer_create_q4(None, C.byref(C.c_void_p())) == -1
    n = C.c_size_t(7)
    assert not L.att1_infer_logits(None, C.byref(n)) and n.value == 0
    assert L.att1_model_load(None, None) == -1


def test_trace_counters(b2):
    L = b2.lib()
    t = C.c_void_p()
    assert L.att1_trace_create(4, 1, C.byref(t)) == 0
    c = b2.TraceCounters()
    assert L.att1_trace_snapshot(t, C.byref(c)) == 0 and c.tokens_decoded == 0
    L.att1_trace_destroy(t)


def test_no_device_is_reported_cleanly(b2):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    L = b2.lib()
    assert L.att1_backend_cuda_available() == 0
    be = C.c_void_p()
    assert L.att1_backend_cuda_q4_create(C.byref(be)) == -9
    cfg = b2.Config.make(100, 1, 2, 2, 64, 64, 8)
    h = C.c_void_p()
    assert L.att1_b200_infer_create_synth(C.byref(cfg), 1, 1, C.byref(h)) != 0
    assert not h.value


def test_cluster_rejects_bad_tile_counts(b2, orc, tmp_path):
    """tile_count 0 is an argument error; more tiles than GPUs (or than the
    eight of one box) is unsupported: checked before any device work."""
    path = str(tmp_path / "m.att1")
    att1file.synth_model_file(path, orc, 64, 1, 2, 32, 64, 8, "q4", 1)
    L = b2.lib()
    m = b2.Model()
    assert L.att1_model_load(path.encode(), C.byref(m)) == 0
    h = C.c_void_p()
    assert L.att1_cluster_infer_create_q4(C.byref(m), C.byref(b2.ClusterConfig(0, 0, 0, 0)), C.byref(h)) == -1
    assert L.att1_cluster_infer_create_q4(C.byref(m), C.byref(b2.ClusterConfig(16, 0, 0, 0)), C.byref(h)) == -9
    assert L.att1_cluster_infer_create_q4(C.byref(m), C.byref(b2.ClusterConfig(1, 0, 0, 1)), C.byref(h)) == -9
    assert not h.value
    L.att1_model_free(C.byref(m))
