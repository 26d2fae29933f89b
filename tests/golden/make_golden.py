"""Generate the golden fixtures in tests/golden/ from the REFERENCE itself.

Runs the ATT-1 reference compiled from its own sources (oracle/_ref, built by
`make -C oracle ref` from the read-only reference tree) through its public
API, on inputs produced by the seeded synthetic generator:

  q4_quant.npz      att1_quantize_q4_per_group of a 64x256 seeded matrix
  file_q4.npz       att1_model_load + att1_infer_create_q4 +
                    att1_infer_decode_token on a q4 .att1 file (logits per
                    step, greedy tokens)
  file_q8.npz       att1_infer_create + att1_backend_cpu_q8_create +
                    att1_infer_set_backend (f32 model quantised to q8 at
                    run time), same stream

The .att1 files are written by tests/att1file.py, deterministically, so the
tests can rebuild the identical file wherever they run.

Usage: python tests/golden/make_golden.py
"""
import ctypes as C
import os
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "tests"))

import att1file  # noqa: E402
import oracle as O  # noqa: E402

# the file-model workload: MHA (the .att1 format has no KV-head count)
FILE_MODEL = dict(vocab=512, n_layers=2, n_heads=4, d_model=128, d_ff=192, max_seq=32, seed=2024)
FILE_TOKENS = [1, 511, 42, 7, 7, 300, 128, 9, 0, 64]


def file_model_path(tmpdir, dtype):
    p = os.path.join(tmpdir, f"model_{dtype}.att1")
    m = FILE_MODEL
    att1file.synth_model_file(p, O.Oracle(), m["vocab"], m["n_layers"], m["n_heads"], m["d_model"],
                              m["d_ff"], m["max_seq"], dtype, m["seed"])
    return p


def reference_file_decode(ref_lib, path, q8):
    L = ref_lib
    L.att1_model_load.argtypes = [C.c_char_p, C.c_void_p]
    L.att1_infer_create_q4.argtypes = [C.c_void_p, C.POINTER(C.c_void_p)]
    L.att1_infer_create.argtypes = [C.c_void_p, C.POINTER(C.c_void_p)]
    L.att1_infer_decode_token.argtypes = [C.c_void_p, C.c_uint32, C.POINTER(C.c_uint32)]
    L.att1_infer_logits.argtypes = [C.c_void_p, C.POINTER(C.c_size_t)]
    L.att1_infer_logits.restype = C.POINTER(C.c_float)
    L.att1_backend_cpu_q8_create.argtypes = [C.POINTER(C.c_void_p)]
    L.att1_infer_set_backend.argtypes = [C.c_void_p, C.c_void_p]
    L.att1_infer_destroy.argtypes = [C.c_void_p]
    L.att1_model_free.argtypes = [C.c_void_p]
    model = C.create_string_buffer(1 << 16)  # opaque att1_model of the reference
    assert L.att1_model_load(path.encode(), model) == 0
    inf = C.c_void_p()
    if q8:
        assert L.att1_infer_create(model, C.byref(inf)) == 0
        be = C.c_void_p()
        assert L.att1_backend_cpu_q8_create(C.byref(be)) == 0
        assert L.att1_infer_set_backend(inf, be) == 0
    else:
        assert L.att1_infer_create_q4(model, C.byref(inf)) == 0
    logits, toks = [], []
    for t in FILE_TOKENS:
        o = C.c_uint32()
        assert L.att1_infer_decode_token(inf, t, C.byref(o)) == 0
        n = C.c_size_t()
        p = L.att1_infer_logits(inf, C.byref(n))
        logits.append(np.ctypeslib.as_array(p, (n.value,)).copy())
        toks.append(o.value)
    L.att1_infer_destroy(inf)
    L.att1_model_free(model)
    return np.stack(logits), np.array(toks, np.uint32)


def main():
    ref = O.Reference()
    orc = O.Oracle()
    w = orc.synth_normal(99, 1, 64 * 256).reshape(64, 256)
    p, s = ref.q4_quantize(w)
    np.savez_compressed(os.path.join(HERE, "q4_quant.npz"), packed=p, scales=s, seed=99, tensor_id=1,
                        rows=64, cols=256)
    with tempfile.TemporaryDirectory() as td:
        for dtype, name in (("q4", "file_q4.npz"), ("f32", "file_q8.npz")):
            path = file_model_path(td, dtype)
            logits, toks = reference_file_decode(ref.lib, path, q8=(dtype == "f32"))
            np.savez_compressed(os.path.join(HERE, name), logits=logits, tokens=toks,
                                stream=np.array(FILE_TOKENS, np.uint32), **{k: v for k, v in FILE_MODEL.items()})
            print(name, logits.shape, toks)


if __name__ == "__main__":
    main()
