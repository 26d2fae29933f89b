"""The att1_backend vtable (include/att1_backend.h) served by the B200 device.

The reference's CUDA backend tests (tests/test_cuda_matmul_q4.c,
test_cuda_norm.c, test_cuda_rope.c, test_cuda_ffn.c,
test_cuda_transformer_block.c, test_cuda_infer_q4.c) drive every op through
`backend->ops->...` with host buffers and compare with the CPU functions. The
same checks run here through this library's "cuda", "cuda-q8" and "cuda-q4"
backends, against the oracle (the CPU restatement, bit-identical to the
reference):

  * the reference tests' own cases (hand-checkable 2x16 q4 matrix with group
    16, deterministic medium matrices, zero weights, a larger batch, invalid
    dimensions and metadata, backend identity) with their tolerance (1e-4 for
    q4 against the CPU q4 product; 1e-3 for norm / RoPE / FFN);
  * decode shapes (4096 x 4096 group 32, 14336-column down projections,
    batches above what one GEMV holds) within 2e-5 of the largest output;
  * the reference's own transformer block (src/transformer_block.c, compiled
    in oracle/_ref) running on this library's "cuda" backend against the
    reference's cpu-f32 backend;
  * the reference's own inference loop (src/infer.c) routed by name to this
    library's "cuda-q4" / "cuda-q8" backends, against the reference's cpu-q4 /
    cpu-q8 logits;
  * this library's att1_infer_set_backend: precision switches the file can and
    cannot serve, with the reference's return codes.

Shapes the device's unit layout holds (q4 groups of 32..128, columns a
multiple of 32) run the decode GEMV; the others run kernels that keep the
reference's operation order, so their results equal the reference's bit for
bit (asserted).
"""
import ctypes as C

import numpy as np
import pytest

import att1file
from test_gpu_decode import tokens_agree

pytestmark = pytest.mark.gpu

Q4_CUDA_TOL = 1e-4     # tests/test_cuda_matmul_q4.c: CUDA q4 vs CPU q4
OP_TOL = 1e-3          # tests/test_cuda_norm.c, test_cuda_rope.c, test_cuda_ffn.c
GEMV_RTOL = 2e-5       # decode GEMV vs the oracle, relative to the largest output

_P = C.c_void_p
_F = C.POINTER(C.c_float)
_SZ = C.c_size_t


class Ops(C.Structure):
    _fields_ = [("name", C.c_char_p),
                ("alloc", C.CFUNCTYPE(_P, _P, _SZ)),
                ("free", C.CFUNCTYPE(None, _P, _P)),
                ("sync", C.CFUNCTYPE(C.c_int, _P)),
                ("matmul_f32", C.CFUNCTYPE(C.c_int, _P, _F, _F, _F, _SZ, _SZ, _SZ)),
                ("matmul_q8xf32", C.CFUNCTYPE(C.c_int, _P, _F, _F, _SZ, _SZ, _P)),
                ("matmul_q4xf32", C.CFUNCTYPE(C.c_int, _P, _F, _F, _SZ, _SZ, _P)),
                ("rmsnorm_f32", C.CFUNCTYPE(C.c_int, _P, _F, _F, _F, _SZ, C.c_float)),
                ("softmax_f32", C.CFUNCTYPE(C.c_int, _P, _F, _SZ)),
                ("rope_f32", C.CFUNCTYPE(C.c_int, _P, _F, _SZ, _SZ, C.c_float)),
                ("ffn_swiglu_f32", C.CFUNCTYPE(C.c_int, _P, _F, _F, _F, _SZ))]


class Backend(C.Structure):
    _fields_ = [("ops", C.POINTER(Ops)), ("user_data", _P)]


class Q4Matrix(C.Structure):
    _fields_ = [("rows", _SZ), ("cols", _SZ), ("group_size", C.c_uint32), ("packed", _P), ("scales", _P)]


class Q8Matrix(C.Structure):
    _fields_ = [("rows", _SZ), ("cols", _SZ), ("values", _P), ("scales", _P)]


def fp(a):
    return a.ctypes.data_as(_F)


class Be:
    """One backend of this library, its ops table read through the struct."""

    def __init__(self, b2, kind):
        self.L = b2.lib()
        h = C.c_void_p()
        create = {"cuda": self.L.att1_backend_cuda_create, "cuda-q8": self.L.att1_backend_cuda_q8_create,
                  "cuda-q4": self.L.att1_backend_cuda_q4_create}[kind]
        assert create(C.byref(h)) == 0
        self.h = h
        self.b = C.cast(h, C.POINTER(Backend)).contents
        self.ops = self.b.ops.contents

    def close(self):
        if self.h:
            self.L.att1_backend_destroy(self.h)
            self.h = None

    def q4(self, x, packed, scales, rows, cols, group, m=None):
        x = np.ascontiguousarray(x, np.float32).reshape(-1, cols)
        out = np.full((x.shape[0], rows), np.nan, np.float32)
        w = Q4Matrix(rows, cols, group, packed.ctypes.data, scales.ctypes.data)
        rc = self.ops.matmul_q4xf32(self.h, fp(out), fp(x), x.shape[0], cols, C.cast(C.pointer(w), _P))
        return rc, out

    def q8(self, x, values, scales, rows, cols):
        x = np.ascontiguousarray(x, np.float32).reshape(-1, cols)
        out = np.full((x.shape[0], rows), np.nan, np.float32)
        w = Q8Matrix(rows, cols, values.ctypes.data, scales.ctypes.data)
        rc = self.ops.matmul_q8xf32(self.h, fp(out), fp(x), x.shape[0], cols, C.cast(C.pointer(w), _P))
        return rc, out


@pytest.fixture
def q4be(b2):
    be = Be(b2, "cuda-q4")
    yield be
    be.close()


@pytest.fixture
def q8be(b2):
    be = Be(b2, "cuda-q8")
    yield be
    be.close()


@pytest.fixture
def f32be(b2):
    be = Be(b2, "cuda")
    yield be
    be.close()


def rel(a, b):
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


# ---- matmul_q4xf32 (tests/test_cuda_matmul_q4.c) ------------------------------------------------

def test_q4_reference_cases(q4be, orc):
    """The reference test's matrices, all with q4 group 16: the 2x16 hand case
    (8 and 0), the deterministic 4x32 case with 2 input rows, a zero matrix,
    and the 8x64 case with 4 input rows. Bit-identical to the CPU q4 product."""
    cases = []
    w = np.array([[0.5] * 16, [1.0, -1.0] * 8], np.float32)
    cases.append((w, np.ones((1, 16), np.float32)))
    i = np.arange(4 * 32)
    w = (((i * 3 + 1) % 11) - 5).astype(np.float32).reshape(4, 32) * np.float32(0.1875)
    x = ((np.arange(2 * 32) % 9) - 4).astype(np.float32).reshape(2, 32) * np.float32(0.25)
    cases.append((w, x))
    cases.append((np.zeros((3, 32), np.float32), (np.arange(64, dtype=np.float32) + 1).reshape(2, 32) * 0.5))
    i = np.arange(8 * 64)
    w = (((i * 7 + 3) % 13) - 6).astype(np.float32).reshape(8, 64) * np.float32(0.125)
    x = ((np.arange(4 * 64) % 5) - 2).astype(np.float32).reshape(4, 64) * np.float32(0.5)
    cases.append((w, x))
    for n, (w, x) in enumerate(cases):
        rows, cols = w.shape
        p, s = orc.q4_quantize(w, 16)
        want = orc.matmul_q4(x, p, s, rows, cols, group=16)
        rc, got = q4be.q4(x, p, s, rows, cols, 16)
        assert rc == 0, n
        assert np.abs(got - want).max() <= Q4_CUDA_TOL, n
        assert (got.view(np.uint32) == want.view(np.uint32)).all(), n
    assert np.abs(q4be.q4(cases[0][1], *orc.q4_quantize(cases[0][0], 16), 2, 16, 16)[1] - [8.0, 0.0]).max() <= 0.35


@pytest.mark.parametrize("rows,cols,batch,group", [(4096, 4096, 1, 32), (4096, 4096, 3, 32), (1024, 4096, 20, 32),
                                                   (512, 14336, 16, 32), (256, 4096, 2, 64), (256, 4096, 2, 128),
                                                   (96, 48, 3, 16)])
def test_q4_decode_shapes(q4be, orc, rows, cols, batch, group):
    """Decode shapes through the vtable: the GEMV (and several GEMV passes
    when the batch is larger than one holds), and the ordered kernel for a
    16-column group."""
    w = orc.synth_normal(31, rows, rows * cols).reshape(rows, cols)
    p, s = orc.q4_quantize(w, group)
    x = orc.synth_normal(32, cols, batch * cols, std=1.0).reshape(batch, cols)
    want = orc.matmul_q4(x, p, s, rows, cols, group=group, threads=8)
    rc, got = q4be.q4(x, p, s, rows, cols, group)
    assert rc == 0
    assert rel(got, want) <= GEMV_RTOL
    rc, again = q4be.q4(x, p, s, rows, cols, group)           # weights now from the device cache
    assert rc == 0 and (again == got).all()


def test_q4_invalid_arguments(q4be, orc):
    """The reference test's invalid calls fail with -1 (null dst / lhs /
    weights, zero rows or columns, mismatched columns, a zeroed matrix), and
    so do group sizes the reference rejects."""
    p, s = orc.q4_quantize(np.zeros((2, 16), np.float32), 16)
    w = Q4Matrix(2, 16, 16, p.ctypes.data, s.ctypes.data)
    wp = C.cast(C.pointer(w), _P)
    dst = np.zeros(4, np.float32)
    lhs = np.zeros(32, np.float32)
    ops, h = q4be.ops, q4be.h
    assert ops.matmul_q4xf32(h, None, fp(lhs), 1, 16, wp) != 0
    assert ops.matmul_q4xf32(h, fp(dst), None, 1, 16, wp) != 0
    assert ops.matmul_q4xf32(h, fp(dst), fp(lhs), 1, 16, None) != 0
    assert ops.matmul_q4xf32(h, fp(dst), fp(lhs), 0, 16, wp) != 0
    assert ops.matmul_q4xf32(h, fp(dst), fp(lhs), 1, 0, wp) != 0
    assert ops.matmul_q4xf32(h, fp(dst), fp(lhs), 1, 32, wp) != 0
    zero = Q4Matrix()
    assert ops.matmul_q4xf32(h, fp(dst), fp(lhs), 1, 16, C.cast(C.pointer(zero), _P)) != 0
    for g in (8, 24, 256):
        bad = Q4Matrix(2, 16 if g != 256 else 256, g, p.ctypes.data, s.ctypes.data)
        assert ops.matmul_q4xf32(h, fp(dst), fp(lhs), 1, bad.cols, C.cast(C.pointer(bad), _P)) != 0


def test_backend_identity(b2):
    """Names route the reference's inference code (src/infer.c:143-159); the
    q4 and q8 backends carry every inference op, the f32 one no quantised
    product (the reference then falls back to its CPU product)."""
    for kind, q8, q4 in (("cuda", False, False), ("cuda-q8", True, False), ("cuda-q4", False, True)):
        be = Be(b2, kind)
        try:
            o = be.ops
            assert o.name.decode() == kind
            assert all(bool(getattr(o, f)) for f in ("alloc", "free", "sync", "matmul_f32", "rmsnorm_f32",
                                                      "softmax_f32", "rope_f32", "ffn_swiglu_f32"))
            assert bool(o.matmul_q8xf32) == q8 and bool(o.matmul_q4xf32) == q4
        finally:
            be.close()


# ---- matmul_q8xf32 -----------------------------------------------------------------------------

@pytest.mark.parametrize("rows,cols,batch", [(300, 288, 1), (2048, 4096, 5), (64, 100, 3), (7, 13, 2)])
def test_q8_op(q8be, orc, rows, cols, batch):
    """q8 products: the GEMV for columns in multiples of 32, the ordered
    kernel (bit-identical to the CPU product) otherwise."""
    w = orc.synth_normal(41, rows, rows * cols).reshape(rows, cols)
    v, s = orc.q8_quantize(w)
    x = orc.synth_normal(42, cols, batch * cols, std=1.0).reshape(batch, cols)
    want = orc.matmul_q8(x, v, s, rows, cols)
    rc, got = q8be.q8(x, v, s, rows, cols)
    assert rc == 0
    assert rel(got, want) <= GEMV_RTOL
    if cols % 32:
        assert (got.view(np.uint32) == want.view(np.uint32)).all()
    dst = np.zeros(rows, np.float32)
    wq = Q8Matrix(rows, cols, v.ctypes.data, s.ctypes.data)
    assert q8be.ops.matmul_q8xf32(q8be.h, fp(dst), fp(x), 1, cols + 1, C.cast(C.pointer(wq), _P)) != 0


# ---- f32 ops (tests/test_cuda_norm.c, test_cuda_rope.c, test_cuda_ffn.c) -------------------------

def test_rmsnorm_op(f32be, orc):
    ops, h = f32be.ops, f32be.h
    src = np.array([1.0, -2.0, 3.0, -4.0], np.float32)
    wt = np.array([1.0, 0.5, 1.5, 2.0], np.float32)
    out = np.zeros(4, np.float32)
    assert ops.rmsnorm_f32(h, fp(out), fp(src), fp(wt), 4, 1e-6) == 0
    assert np.abs(out - orc.rmsnorm(src, wt, 1e-6)).max() < OP_TOL
    for n in (4096, 14336, 5):
        src = orc.synth_normal(51, n, n, std=2.0)
        wt = orc.synth_normal(52, n, n, std=1.0)
        out = np.zeros(n, np.float32)
        assert ops.rmsnorm_f32(h, fp(out), fp(src), fp(wt), n, 1e-5) == 0
        assert rel(out, orc.rmsnorm(src, wt, 1e-5)) <= 1e-6
    assert ops.rmsnorm_f32(h, None, fp(src), fp(wt), 5, 1e-5) != 0
    assert ops.rmsnorm_f32(h, fp(out), fp(src), fp(wt), 0, 1e-5) != 0


def test_softmax_op(f32be, orc):
    ops, h = f32be.ops, f32be.h
    for n in (1, 7, 4096, 100000):
        v = orc.synth_normal(53, n, n, std=3.0)
        got = v.copy()
        assert ops.softmax_f32(h, fp(got), n) == 0
        # relative to the largest probability; the CPU sums the n exponentials
        # one after another, whose rounding grows up to n * 2^-24 (the device
        # adds them in a tree)
        assert rel(got, orc.softmax(v)) <= 1e-6 + n * 6e-8
        assert abs(float(got.astype(np.float64).sum()) - 1.0) <= 1e-4
    assert ops.softmax_f32(h, None, 3) != 0


def test_rope_op(f32be, orc):
    """Position 0 leaves the vector unchanged; interleaved pairs rotate as
    the CPU RoPE does at many positions and both thetas; odd lengths fail."""
    ops, h = f32be.ops, f32be.h
    v0 = np.array([1.0, 0.5, -2.0, 3.0, 4.0, -1.0], np.float32)
    got = v0.copy()
    assert ops.rope_f32(h, fp(got), 6, 0, 10000.0) == 0
    assert np.abs(got - v0).max() < OP_TOL
    for n, pos, theta in ((128, 1, 10000.0), (128, 4095, 500000.0), (64, 2047, 10000.0), (48, 300, 10000.0)):
        v = orc.synth_normal(54, n + pos, n, std=1.0)
        got = v.copy()
        assert ops.rope_f32(h, fp(got), n, pos, theta) == 0
        assert np.abs(got - orc.rope(v, pos, theta)).max() <= 2e-6 * max(1.0, np.abs(v).max())
    odd = np.ones(5, np.float32)
    assert ops.rope_f32(h, fp(odd), 5, 3, 10000.0) != 0


def test_ffn_composed_from_ops(f32be, orc):
    """The reference FFN test's composition: gate and up f32 products,
    SwiGLU, down product, all through the vtable, against the CPU ops."""
    ops, h = f32be.ops, f32be.h
    d, f = 64, 160
    x = orc.synth_normal(55, 1, d, std=1.0).reshape(1, d)
    wg, wu = orc.synth_normal(56, 1, d * f, 0.2).reshape(d, f), orc.synth_normal(57, 1, d * f, 0.2).reshape(d, f)
    wd = orc.synth_normal(58, 1, f * d, 0.2).reshape(f, d)
    g, u = np.zeros((1, f), np.float32), np.zeros((1, f), np.float32)
    hs, out = np.zeros(f, np.float32), np.zeros((1, d), np.float32)
    assert ops.matmul_f32(h, fp(g), fp(x), fp(wg), 1, f, d) == 0
    assert ops.matmul_f32(h, fp(u), fp(x), fp(wu), 1, f, d) == 0
    assert ops.ffn_swiglu_f32(h, fp(hs), fp(g), fp(u), f) == 0
    assert ops.matmul_f32(h, fp(out), fp(hs), fp(wd), 1, d, f) == 0
    g64 = x.astype(np.float64) @ wg
    u64 = x.astype(np.float64) @ wu
    assert np.abs(g - g64).max() < OP_TOL and np.abs(u - u64).max() < OP_TOL
    assert np.abs(hs - orc.swiglu(g[0], u[0])).max() <= 1e-6
    want = orc.swiglu(g[0], u[0]).astype(np.float64) @ wd
    assert np.abs(out[0] - want).max() < OP_TOL
    assert ops.ffn_swiglu_f32(h, fp(hs), None, fp(u), f) != 0
    assert ops.matmul_f32(h, fp(out), fp(x), fp(wd), 1, d, 0) != 0


# ---- the reference's own code on this library's backends --------------------------------------

class BlockConfig(C.Structure):
    _fields_ = [("model_dim", _SZ), ("num_heads", _SZ), ("head_dim", _SZ), ("ffn_dim", _SZ),
                ("rms_epsilon", C.c_float), ("rope_theta", C.c_float)]


class BlockWeights(C.Structure):
    _fields_ = [(n, _P) for n in ("attention_norm", "ffn_norm", "wq", "wk", "wv", "wo", "w_gate", "w_up", "w_down")]


def test_reference_block_on_this_backend(b2, ref, orc):
    """src/transformer_block.c (att1_transformer_block_forward_backend,
    compiled from the reference) runs eight positions of one block on this
    library's "cuda" backend and on the reference's cpu-f32 backend, each with
    its own reference KV cache: outputs within the reference test's 1e-3."""
    R = ref.lib
    R.att1_transformer_block_forward_backend.argtypes = [_P, _P, _P, _P, _P, _SZ, _P]
    R.att1_kv_cache_init.argtypes = [_P, _SZ, _SZ, _SZ]
    R.att1_kv_cache_free.argtypes = [_P]
    R.att1_backend_cpu_f32_create.argtypes = [C.POINTER(_P)]
    R.att1_backend_destroy.argtypes = [_P]
    d, H, f, npos = 64, 4, 128, 8
    mats = {}
    tensors = {"wq": (d, d), "wk": (d, d), "wv": (d, d), "wo": (d, d), "w_gate": (d, f), "w_up": (d, f),
               "w_down": (f, d)}
    for i, (n, shp) in enumerate(tensors.items()):
        mats[n] = orc.synth_normal(60 + i, 1, shp[0] * shp[1], std=0.15)
    ones = np.ones(d, np.float32)
    wts = BlockWeights(ones.ctypes.data, ones.ctypes.data, *[mats[n].ctypes.data for n in
                                                             ("wq", "wk", "wv", "wo", "w_gate", "w_up", "w_down")])
    cfg = BlockConfig(d, H, d // H, f, 1e-5, 10000.0)
    ours = Be(b2, "cuda")
    cpu = C.c_void_p()
    assert R.att1_backend_cpu_f32_create(C.byref(cpu)) == 0
    caches = [C.create_string_buffer(256), C.create_string_buffer(256)]
    for c in caches:
        assert R.att1_kv_cache_init(c, 16, H, d // H) == 0
    try:
        worst = 0.0
        for pos in range(npos):
            x = orc.synth_normal(70, pos, d, std=1.0)
            outs = []
            for c, be in zip(caches, (ours.h, cpu)):
                out = np.zeros(d, np.float32)
                assert R.att1_transformer_block_forward_backend(out.ctypes.data, c, x.ctypes.data, C.byref(wts),
                                                                C.byref(cfg), pos, be) == 0
                outs.append(out)
            worst = max(worst, float(np.abs(outs[0] - outs[1]).max()))
        assert worst < OP_TOL, worst
    finally:
        for c in caches:
            R.att1_kv_cache_free(c)
        R.att1_backend_destroy(cpu)
        ours.close()


def ref_infer(R, path, q8, tokens, backend=None):
    """The reference's att1_infer_* on a .att1 file: q4 (create_q4) or q8
    (create + a q8 backend); `backend` replaces the reference's own backend
    through att1_infer_set_backend. Returns logits per step and the tokens."""
    R.att1_model_load.argtypes = [C.c_char_p, _P]
    R.att1_model_free.argtypes = [_P]
    R.att1_infer_create_q4.argtypes = [_P, C.POINTER(_P)]
    R.att1_infer_create.argtypes = [_P, C.POINTER(_P)]
    R.att1_infer_set_backend.argtypes = [_P, _P]
    R.att1_infer_decode_token.argtypes = [_P, C.c_uint32, C.POINTER(C.c_uint32)]
    R.att1_infer_logits.argtypes = [_P, C.POINTER(_SZ)]
    R.att1_infer_logits.restype = _F
    R.att1_infer_destroy.argtypes = [_P]
    R.att1_backend_cpu_q8_create.argtypes = [C.POINTER(_P)]
    model = C.create_string_buffer(1 << 16)       # the reference's att1_model, opaque here
    assert R.att1_model_load(path.encode(), model) == 0
    inf = C.c_void_p()
    try:
        if q8:
            assert R.att1_infer_create(model, C.byref(inf)) == 0
            be = C.c_void_p(backend) if backend is not None else C.c_void_p()
            if backend is None:
                assert R.att1_backend_cpu_q8_create(C.byref(be)) == 0
            assert R.att1_infer_set_backend(inf, be) == 0
        else:
            assert R.att1_infer_create_q4(model, C.byref(inf)) == 0
            if backend is not None:
                assert R.att1_infer_set_backend(inf, C.c_void_p(backend)) == 0
        logits, toks = [], []
        for t in tokens:
            o = C.c_uint32()
            assert R.att1_infer_decode_token(inf, int(t), C.byref(o)) == 0
            n = C.c_size_t()
            p = R.att1_infer_logits(inf, C.byref(n))
            logits.append(np.ctypeslib.as_array(p, (n.value,)).copy())
            toks.append(o.value)
        return np.stack(logits), toks
    finally:
        if inf:
            R.att1_infer_destroy(inf)
        R.att1_model_free(model)


FILE = dict(vocab=512, n_layers=2, n_heads=4, d_model=128, d_ff=192, max_seq=32, seed=2024)
STREAM = [1, 511, 42, 7, 7, 300, 128, 9]


def model_file(tmp_path, orc, dtype):
    p = str(tmp_path / f"vt_{dtype}.att1")
    att1file.synth_model_file(p, orc, FILE["vocab"], FILE["n_layers"], FILE["n_heads"], FILE["d_model"],
                              FILE["d_ff"], FILE["max_seq"], dtype, FILE["seed"])
    return p


@pytest.mark.parametrize("dtype", ["q4", "f32"])
def test_reference_infer_routes_to_this_backend(b2, ref, orc, tmp_path, dtype):
    """src/infer.c routes by backend name: given this library's "cuda-q4"
    (q4 file) or "cuda-q8" (f32 file, quantised to q8 by the reference), the
    reference's own decode loop calls this library's ops for every product
    and element op. Its logits stay within the GEMV tolerance of the
    reference's cpu-q4 / cpu-q8 run, and the tokens agree."""
    path = model_file(tmp_path, orc, dtype)
    want, wtok = ref_infer(ref.lib, path, dtype == "f32", STREAM)
    be = Be(b2, "cuda-q4" if dtype == "q4" else "cuda-q8")
    h = be.h.value
    be.h = None            # the reference context owns it now (and frees it with its own destroy)
    got, gtok = ref_infer(ref.lib, path, dtype == "f32", STREAM, backend=h)
    assert rel(got, want) <= 1e-4
    for i in range(len(STREAM)):
        assert gtok[i] == wtok[i] or tokens_agree(gtok[i], want[i]), i


def test_set_backend_precision_switch(b2, ref, orc, tmp_path):
    """This library's att1_infer_set_backend on file models (reference
    tests/test_cuda_infer_q4.c): a q4 context takes "cuda-q4" and keeps
    decoding; a switch to "cuda-q8" that the q4 file cannot serve returns the
    reference's code for the same switch and leaves the context decoding q4;
    an f32 file's context takes "cuda-q8" (q8 decode, the reference's
    create + set_backend(cpu-q8)) and refuses "cuda-q4" the same way. Every
    step's logits within 1e-3 of the reference's."""
    import att1_b200 as B
    L = b2.lib()
    R = ref.lib
    for dtype in ("q4", "f32"):
        path = model_file(tmp_path, orc, dtype)
        want, wtok = ref_infer(R, path, dtype == "f32", STREAM)
        # the reference's code for the switch the file cannot serve
        model_r = C.create_string_buffer(1 << 16)
        R.att1_model_load.argtypes = [C.c_char_p, _P]
        assert R.att1_model_load(path.encode(), model_r) == 0
        inf_r = C.c_void_p()
        R.att1_backend_cpu_q8_create.argtypes = [C.POINTER(_P)]
        R.att1_backend_cpu_q4_create.argtypes = [C.POINTER(_P)]
        if dtype == "q4":
            assert R.att1_infer_create_q4(model_r, C.byref(inf_r)) == 0
            other = C.c_void_p()
            assert R.att1_backend_cpu_q8_create(C.byref(other)) == 0
        else:
            assert R.att1_infer_create(model_r, C.byref(inf_r)) == 0
            other = C.c_void_p()
            assert R.att1_backend_cpu_q4_create(C.byref(other)) == 0
        ref_code = R.att1_infer_set_backend(inf_r, other)
        assert ref_code != 0
        R.att1_backend_destroy.argtypes = [_P]
        R.att1_infer_destroy.argtypes = [_P]
        R.att1_model_free.argtypes = [_P]
        R.att1_backend_destroy(other)
        R.att1_infer_destroy(inf_r)
        R.att1_model_free(model_r)

        m = B.Model()
        assert L.att1_model_load(path.encode(), C.byref(m)) == 0
        h = C.c_void_p()
        create = L.att1_infer_create_q4 if dtype == "q4" else L.att1_infer_create
        assert create(C.byref(m), C.byref(h)) == 0
        try:
            same = Be(b2, "cuda-q4" if dtype == "q4" else "cuda-q8")
            assert L.att1_infer_set_backend(h, same.h) == 0
            same.h = None                                   # owned by the context now
            steps = []
            for i, t in enumerate(STREAM):
                if i == 3:
                    other = Be(b2, "cuda-q8" if dtype == "q4" else "cuda-q4")
                    assert L.att1_infer_set_backend(h, other.h) == ref_code
                    other.close()
                o = C.c_uint32()
                assert L.att1_infer_decode_token(h, t, C.byref(o)) == 0
                n = C.c_size_t()
                p = L.att1_infer_logits(h, C.byref(n))
                steps.append(np.ctypeslib.as_array(C.cast(p, _F), (n.value,)).copy())
                assert tokens_agree(o.value, want[i]), i
            got = np.stack(steps)
            assert rel(got, want) <= 1e-3
        finally:
            L.att1_infer_destroy(h)
            L.att1_model_free(C.byref(m))
