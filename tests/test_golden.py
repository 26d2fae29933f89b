"""Golden fixtures made by running the reference itself (tests/golden/make_golden.py).

CPU: the oracle reproduces them bit for bit; the library's .att1 loader reads
the same file the reference decoded. GPU: the library's file-model path
(att1_model_load + att1_infer_create_q4 / att1_infer_create) reproduces the
reference's logits within the 1e-3 relative tolerance.
"""
import ctypes as C
import os

import numpy as np
import pytest

import att1file
import oracle as O

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    return dict(np.load(os.path.join(GOLDEN, name)))


def test_q4_quantiser_golden(orc):
    g = load("q4_quant.npz")
    w = orc.synth_normal(int(g["seed"]), int(g["tensor_id"]), int(g["rows"]) * int(g["cols"]))
    p, s = orc.q4_quantize(w.reshape(int(g["rows"]), int(g["cols"])))
    assert (p == g["packed"]).all()
    assert (s.view(np.uint32) == g["scales"].view(np.uint32)).all()


@pytest.mark.parametrize("name,dtype", [("file_q4.npz", O.Q4), ("file_q8.npz", O.Q8)])
def test_oracle_reproduces_reference_file_decode(orc, name, dtype):
    g = load(name)
    cfg = O.Config.make(vocab=int(g["vocab"]), n_layers=int(g["n_layers"]), n_heads=int(g["n_heads"]),
                        n_kv_heads=int(g["n_heads"]), d_model=int(g["d_model"]), d_ff=int(g["d_ff"]),
                        max_seq=int(g["max_seq"]), dtype=dtype, eps=1e-6, theta=10000.0)
    om = orc.model(cfg, int(g["seed"]))
    for s, t in enumerate(g["stream"]):
        lg, tok = om.decode(int(t))
        assert (lg.view(np.uint32) == g["logits"][s].view(np.uint32)).all(), s
        assert tok == g["tokens"][s]


def write_file(tmp_path, orc, g, dtype):
    p = str(tmp_path / f"m_{dtype}.att1")
    att1file.synth_model_file(p, orc, int(g["vocab"]), int(g["n_layers"]), int(g["n_heads"]),
                              int(g["d_model"]), int(g["d_ff"]), int(g["max_seq"]), dtype, int(g["seed"]))
    return p


def test_library_loader_reads_golden_file(b2, orc, tmp_path):
    g = load("file_q4.npz")
    path = write_file(tmp_path, orc, g, "q4")
    L = b2.lib()
    m = b2.Model()
    assert L.att1_model_load(path.encode(), C.byref(m)) == 0
    assert m.config.vocab_size == int(g["vocab"]) and m.config.n_layers == int(g["n_layers"])
    assert m.tensor_count == 3 + 9 * int(g["n_layers"])
    t = L.att1_model_find_tensor(C.byref(m), b"layers.1.ffn.w_down.weight")
    assert t and t.contents.dtype == 3 and t.contents.flags == 32
    assert tuple(t.contents.shape[:2]) == (int(g["d_model"]), int(g["d_ff"]))
    L.att1_model_free(C.byref(m))


@pytest.mark.gpu
@pytest.mark.parametrize("name,dtype", [("file_q4.npz", "q4"), ("file_q8.npz", "f32")])
def test_library_file_decode_matches_reference(b2, orc, tmp_path, name, dtype):
    g = load(name)
    path = write_file(tmp_path, orc, g, dtype)
    L = b2.lib()
    m = b2.Model()
    assert L.att1_model_load(path.encode(), C.byref(m)) == 0
    h = C.c_void_p()
    create = L.att1_infer_create_q4 if dtype == "q4" else L.att1_infer_create
    assert create(C.byref(m), C.byref(h)) == 0
    try:
        for s, t in enumerate(g["stream"]):
            o = C.c_uint32()
            assert L.att1_infer_decode_token(h, int(t), C.byref(o)) == 0
            n = C.c_size_t()
            p = L.att1_infer_logits(h, C.byref(n))
            lg = np.ctypeslib.as_array(p, (n.value,))
            ref = g["logits"][s]
            err = float(np.abs(lg - ref).max() / np.abs(ref).max())
            assert err <= 1e-3, (s, err)
            top2 = np.sort(ref)[-2:]
            if (top2[1] - top2[0]) / np.abs(ref).max() > 2e-3:
                assert o.value == g["tokens"][s]
    finally:
        L.att1_infer_destroy(h)
        L.att1_model_free(C.byref(m))


@pytest.mark.gpu
def test_file_q8_weights_match_reference_quantiser(b2, orc, tmp_path):
    """f32 .att1 model -> att1_infer_create: the device q8 weights equal the
    reference rule applied to the transposed f32 tensors (src/infer.c:196-233)."""
    g = load("file_q8.npz")
    path = write_file(tmp_path, orc, g, "f32")
    L = b2.lib()
    m = b2.Model()
    assert L.att1_model_load(path.encode(), C.byref(m)) == 0
    h = C.c_void_p()
    assert L.att1_infer_create(C.byref(m), C.byref(h)) == 0
    inf = b2.Infer(h.value, int(g["vocab"]), 1)
    d, f, V, seed = int(g["d_model"]), int(g["d_ff"]), int(g["vocab"]), int(g["seed"])
    shapes = {b2.WQ: (d, d), b2.WK: (d, d), b2.WV: (d, d), b2.WO: (d, d), b2.GATE: (f, d), b2.UP: (f, d),
              b2.DOWN: (d, f), b2.OUTPUT: (V, d)}
    try:
        for layer in range(int(g["n_layers"])):
            for kind, (rows, cols) in shapes.items():
                tid = O.T_OUTPUT if kind == b2.OUTPUT else layer * O.T_PER_LAYER + kind
                v, s = orc.q8_quantize(orc.synth_normal(seed, tid, rows * cols).reshape(rows, cols))
                gv, gs = inf.export_q8(layer, kind, rows, cols)
                assert (gv == v).all(), (layer, kind)
                assert (gs == s).all(), (layer, kind)
    finally:
        inf.close()
        L.att1_model_free(C.byref(m))
