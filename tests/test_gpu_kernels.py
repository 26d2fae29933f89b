"""Kernel-level parity on the GPU, through the C ABI (b2_kernels.h).

Packed weights must match the reference quantiser bit for bit; GEMV results
are compared with the oracle's f32 matmul (same rounding as the reference's
att1_matmul_q4xf32 / att1_matmul_q8xf32) at max|gpu - cpu| / max|cpu| <= 2e-5
(the kernels compute products exactly and round only in f32 accumulation and
the 2^-22 quantisation of the input vector).
"""
import ctypes as C

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu
GEMV_RTOL = 2e-5


def rel_err(a, b):
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


@pytest.fixture(scope="module")
def torch():
    import torch
    torch.cuda.init()
    return torch


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def q4_device(b2, torch, packed, scales, rows, cols, group=32):
    L = b2.lib()
    buf = torch.zeros(L.b2_q4_bytes(rows, cols), dtype=torch.uint8, device="cuda")
    p, s = dev(torch, packed), dev(torch, scales)
    rc = L.b2_q4_pack(buf.data_ptr(), 0, rows, cols, p.data_ptr(), s.data_ptr(), None, None, group, 0, None)
    assert rc == 0
    torch.cuda.synchronize()
    return buf


def q8_device(b2, torch, values, scales, rows, cols):
    L = b2.lib()
    buf = torch.zeros(L.b2_q8_bytes(rows, cols), dtype=torch.uint8, device="cuda")
    rs = torch.zeros(((rows + 15) // 16) * 16, dtype=torch.float32, device="cuda")
    v, s = dev(torch, values), dev(torch, scales)
    assert L.b2_q8_pack(buf.data_ptr(), rs.data_ptr(), 0, rows, cols, v.data_ptr(), s.data_ptr(),
                        None, None, 0, None) == 0
    torch.cuda.synchronize()
    return buf, rs


def run_gemv(b2, torch, fmt, buf, rs, rows, cols, x, epilogue=0, norm_w=None, eps=1e-5, resid=None,
             out_stride=None, grid=0):
    L = b2.lib()
    batch = x.shape[0]
    xd = dev(torch, x.astype(np.float32))
    out_stride = out_stride or rows
    out = torch.zeros(batch * out_stride, dtype=torch.float32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    a = b2.GemvArgs()
    a.w = b2.QWeight(buf.data_ptr(), rs.data_ptr() if rs is not None else None, fmt, rows, cols,
                     (rows + 15) // 16, (cols + 63) // 64 if fmt == 4 else (cols + 31) // 32)
    a.batch = batch
    a.x = xd.data_ptr()
    a.x_stride = cols
    nw = dev(torch, norm_w) if norm_w is not None else None
    a.norm_w = nw.data_ptr() if nw is not None else None
    a.eps = eps
    a.epilogue = epilogue
    a.out = out.data_ptr()
    a.out_stride = out_stride
    rd = dev(torch, resid) if resid is not None else None
    a.resid = rd.data_ptr() if rd is not None else None
    a.err = err.data_ptr()
    a.grid = grid
    need = L.b2_gemv_scratch_bytes(C.byref(a))
    scratch = torch.full((need,), 0x7F, dtype=torch.uint8, device="cuda")  # contents must not matter
    counters = torch.zeros(L.b2_gemv_counters_len(C.byref(a)), dtype=torch.int32, device="cuda")
    a.scratch = scratch.data_ptr()
    a.scratch_bytes = need
    a.counters = counters.data_ptr()
    a.counters_len = counters.numel()
    assert L.b2_gemv(C.byref(a), None) == 0
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    # counters must be back to zero after the launch
    return out.cpu().numpy().reshape(batch, out_stride), counters.cpu().numpy()


def test_library_loads_sm100(b2):
    assert b2.lib().att1_backend_cuda_available() == 1
    assert b2.lib().b2_sm_count() > 0


@pytest.mark.parametrize("rows,cols", [(16, 64), (40, 96), (300, 288), (1024, 4096)])
def test_q4_pack_unpack_round_trip(b2, torch, orc, rows, cols):
    w = orc.synth_normal(4, 9, rows * cols).reshape(rows, cols)
    p, s = orc.q4_quantize(w)
    buf = q4_device(b2, torch, p, s, rows, cols)
    pd = torch.zeros(rows * cols // 2, dtype=torch.uint8, device="cuda")
    sd = torch.zeros(rows * cols // 32, dtype=torch.float32, device="cuda")
    assert b2.lib().b2_q4_unpack(pd.data_ptr(), sd.data_ptr(), buf.data_ptr(), 0, rows, cols, 0, 0, None) == 0
    torch.cuda.synchronize()
    assert (pd.cpu().numpy() == p).all()
    assert (sd.cpu().numpy().view(np.uint32) == s.view(np.uint32)).all()


@pytest.mark.parametrize("rows,cols", [(16, 32), (48, 160), (512, 4096)])
def test_q4_device_quantiser_bit_exact(b2, torch, orc, rows, cols):
    """Device generator + quantiser == oracle generator + reference-rule quantiser."""
    L = b2.lib()
    buf = torch.zeros(L.b2_q4_bytes(rows, cols), dtype=torch.uint8, device="cuda")
    assert L.b2_q4_synth(buf.data_ptr(), 0, rows, cols, 77, 5, 0, 0.02, 0, None) == 0
    pd = torch.zeros(rows * cols // 2, dtype=torch.uint8, device="cuda")
    sd = torch.zeros(rows * cols // 32, dtype=torch.float32, device="cuda")
    assert L.b2_q4_unpack(pd.data_ptr(), sd.data_ptr(), buf.data_ptr(), 0, rows, cols, 0, 0, None) == 0
    torch.cuda.synchronize()
    p, s = orc.q4_quantize(orc.synth_normal(77, 5, rows * cols).reshape(rows, cols))
    assert (pd.cpu().numpy() == p).all()
    assert (sd.cpu().numpy().view(np.uint32) == s.view(np.uint32)).all()


def test_q4_gateup_interleave_round_trip(b2, torch, orc):
    L = b2.lib()
    F, d = 40, 64
    buf = torch.zeros(L.b2_q4_bytes(2 * F, d), dtype=torch.uint8, device="cuda")
    assert L.b2_q4_synth(buf.data_ptr(), 0, 2 * F, d, 5, 6, 7, 0.02, 1, None) == 0
    for which, tid in ((0, 6), (1, 7)):
        pd = torch.zeros(F * d // 2, dtype=torch.uint8, device="cuda")
        sd = torch.zeros(F * d // 32, dtype=torch.float32, device="cuda")
        assert L.b2_q4_unpack(pd.data_ptr(), sd.data_ptr(), buf.data_ptr(), 0, F, d, 1, which, None) == 0
        torch.cuda.synchronize()
        p, s = orc.q4_quantize(orc.synth_normal(5, tid, F * d).reshape(F, d))
        assert (pd.cpu().numpy() == p).all() and (sd.cpu().numpy() == s).all()


@pytest.mark.parametrize("rows,cols", [(16, 32), (33, 288), (256, 768)])
def test_q8_device_quantiser_bit_exact(b2, torch, orc, rows, cols):
    L = b2.lib()
    buf = torch.zeros(L.b2_q8_bytes(rows, cols), dtype=torch.uint8, device="cuda")
    rs = torch.zeros(((rows + 15) // 16) * 16, dtype=torch.float32, device="cuda")
    assert L.b2_q8_synth(buf.data_ptr(), rs.data_ptr(), 0, rows, cols, 8, 3, 0, 0.02, 0, None) == 0
    vd = torch.zeros(rows * cols, dtype=torch.int8, device="cuda")
    sd = torch.zeros(rows, dtype=torch.float32, device="cuda")
    assert L.b2_q8_unpack(vd.data_ptr(), sd.data_ptr(), buf.data_ptr(), rs.data_ptr(), 0, rows, cols, 0, 0,
                          None) == 0
    torch.cuda.synchronize()
    v, s = orc.q8_quantize(orc.synth_normal(8, 3, rows * cols).reshape(rows, cols))
    assert (vd.cpu().numpy() == v).all()
    assert (sd.cpu().numpy().view(np.uint32) == s.view(np.uint32)).all()


def test_q8_quantize_f32_transposed(b2, torch, orc):
    L = b2.lib()
    rows, cols = 48, 96
    w = orc.synth_normal(2, 2, rows * cols).reshape(rows, cols)
    wt = dev(torch, np.ascontiguousarray(w.T))
    buf = torch.zeros(L.b2_q8_bytes(rows, cols), dtype=torch.uint8, device="cuda")
    rs = torch.zeros(rows, dtype=torch.float32, device="cuda")
    assert L.b2_q8_quantize_f32(buf.data_ptr(), rs.data_ptr(), 0, rows, cols, wt.data_ptr(), None, 1, 0, None) == 0
    vd = torch.zeros(rows * cols, dtype=torch.int8, device="cuda")
    sd = torch.zeros(rows, dtype=torch.float32, device="cuda")
    assert L.b2_q8_unpack(vd.data_ptr(), sd.data_ptr(), buf.data_ptr(), rs.data_ptr(), 0, rows, cols, 0, 0,
                          None) == 0
    torch.cuda.synchronize()
    v, s = orc.q8_quantize(w)
    assert (vd.cpu().numpy() == v).all() and (sd.cpu().numpy() == s).all()


@pytest.mark.parametrize("rows,cols,batch", [
    (16, 64, 1), (40, 96, 1), (300, 288, 2), (4096, 4096, 1), (4096, 4096, 8),
    (14336, 4096, 1), (4096, 14336, 1), (1000, 4096, 3), (7, 32, 5)])
def test_gemv_q4(b2, torch, orc, rows, cols, batch):
    w = orc.synth_normal(31, rows, rows * cols).reshape(rows, cols)
    p, s = orc.q4_quantize(w)
    x = orc.synth_normal(32, cols, batch * cols, std=1.0).reshape(batch, cols)
    buf = q4_device(b2, torch, p, s, rows, cols)
    y, cnt = run_gemv(b2, torch, 4, buf, None, rows, cols, x)
    ref = orc.matmul_q4(x, p, s, rows, cols, threads=8)
    assert rel_err(y, ref) <= GEMV_RTOL
    assert (cnt == 0).all()


@pytest.mark.parametrize("rows,cols,batch", [(16, 32, 1), (300, 288, 1), (768, 288, 2), (32000, 288, 1),
                                             (2048, 4096, 4)])
def test_gemv_q8(b2, torch, orc, rows, cols, batch):
    w = orc.synth_normal(41, rows, rows * cols).reshape(rows, cols)
    v, s = orc.q8_quantize(w)
    x = orc.synth_normal(42, cols, batch * cols, std=1.0).reshape(batch, cols)
    buf, rs = q8_device(b2, torch, v, s, rows, cols)
    y, _ = run_gemv(b2, torch, 8, buf, rs, rows, cols, x)
    ref = orc.matmul_q8(x, v, s, rows, cols, threads=8)
    assert rel_err(y, ref) <= GEMV_RTOL


def test_gemv_wide_dynamic_range(b2, torch, orc):
    """Inputs spanning many binades: the fixed-point digits follow max|x|."""
    rows, cols = 64, 512
    w = orc.synth_normal(1, 1, rows * cols).reshape(rows, cols)
    p, s = orc.q4_quantize(w)
    x = orc.synth_normal(2, 2, cols, std=1.0).reshape(1, cols)
    x = x * np.float32(2.0) ** np.linspace(-30, 30, cols, dtype=np.float32)
    buf = q4_device(b2, torch, p, s, rows, cols)
    y, _ = run_gemv(b2, torch, 4, buf, None, rows, cols, x.astype(np.float32))
    ref = orc.matmul_q4(x.astype(np.float32), p, s, rows, cols)
    assert rel_err(y, ref) <= GEMV_RTOL


def test_gemv_zero_input(b2, torch, orc):
    rows, cols = 32, 64
    p, s = orc.q4_quantize(orc.synth_normal(1, 1, rows * cols).reshape(rows, cols))
    buf = q4_device(b2, torch, p, s, rows, cols)
    y, _ = run_gemv(b2, torch, 4, buf, None, rows, cols, np.zeros((1, cols), np.float32))
    assert (y == 0).all()


def test_gemv_rmsnorm_prologue_resid_epilogue(b2, torch, orc):
    rows, cols = 256, 1024
    w = orc.synth_normal(3, 3, rows * cols).reshape(rows, cols)
    p, s = orc.q4_quantize(w)
    x = orc.synth_normal(4, 4, cols, std=1.0)
    g = orc.synth_normal(5, 5, cols, std=1.0)
    r = orc.synth_normal(6, 6, rows, std=1.0)
    buf = q4_device(b2, torch, p, s, rows, cols)
    y, _ = run_gemv(b2, torch, 4, buf, None, rows, cols, x.reshape(1, cols), epilogue=1, norm_w=g,
                    eps=1e-5, resid=r.reshape(1, rows))
    xn = orc.rmsnorm(x, g, 1e-5)
    ref = r + orc.matmul_q4(xn, p, s, rows, cols)[0]
    assert rel_err(y[0], ref) <= GEMV_RTOL


def test_gemv_swiglu_epilogue(b2, torch, orc):
    L = b2.lib()
    F, d = 96, 256
    buf = torch.zeros(L.b2_q4_bytes(2 * F, d), dtype=torch.uint8, device="cuda")
    assert L.b2_q4_synth(buf.data_ptr(), 0, 2 * F, d, 9, 6, 7, 0.02, 1, None) == 0
    x = orc.synth_normal(10, 10, d, std=1.0)
    y, _ = run_gemv(b2, torch, 4, buf, None, 2 * F, d, x.reshape(1, d), epilogue=3, out_stride=F)
    pg, sg = orc.q4_quantize(orc.synth_normal(9, 6, F * d).reshape(F, d))
    pu, su = orc.q4_quantize(orc.synth_normal(9, 7, F * d).reshape(F, d))
    ref = orc.swiglu(orc.matmul_q4(x, pg, sg, F, d)[0], orc.matmul_q4(x, pu, su, F, d)[0])
    assert rel_err(y[0], ref) <= 1e-4


def test_gemv_grid_sizes_agree(b2, torch, orc):
    """Stream-K split points move with the grid; results stay within f32 reassociation."""
    rows, cols = 512, 2048
    p, s = orc.q4_quantize(orc.synth_normal(7, 7, rows * cols).reshape(rows, cols))
    x = orc.synth_normal(8, 8, cols, std=1.0).reshape(1, cols)
    buf = q4_device(b2, torch, p, s, rows, cols)
    ref = orc.matmul_q4(x, p, s, rows, cols)
    outs = [run_gemv(b2, torch, 4, buf, None, rows, cols, x, grid=g)[0] for g in (1, 3, 37, 148)]
    for y in outs:
        assert rel_err(y, ref) <= GEMV_RTOL
    # deterministic for a fixed grid
    again, _ = run_gemv(b2, torch, 4, buf, None, rows, cols, x, grid=37)
    assert (again == outs[2]).all()


def test_gemv_rejects_bad_args(b2, torch):
    L = b2.lib()
    a = b2.GemvArgs()
    assert L.b2_gemv(C.byref(a), None) == -1
    a.w = b2.QWeight(1, None, 4, 16, 33, 1, 1)  # cols not a multiple of 32
    a.batch = 1
    a.x = 16
    a.out = 16
    assert L.b2_gemv(C.byref(a), None) == -1


def test_element_ops(b2, torch, orc):
    L = b2.lib()
    n = 288
    x = orc.synth_normal(1, 1, n, std=1.0)
    w = orc.synth_normal(1, 2, n, std=1.0)
    xd, wd, od = dev(torch, x), dev(torch, w), torch.zeros(n, device="cuda")
    assert L.b2_rmsnorm(od.data_ptr(), xd.data_ptr(), wd.data_ptr(), n, 1e-5, None) == 0
    torch.cuda.synchronize()
    assert rel_err(od.cpu().numpy(), orc.rmsnorm(x, w, 1e-5)) < 1e-6
    vd = dev(torch, x)
    assert L.b2_softmax(vd.data_ptr(), n, None) == 0
    torch.cuda.synchronize()
    assert rel_err(vd.cpu().numpy(), orc.softmax(x)) < 1e-5
    vd = dev(torch, x)
    assert L.b2_rope(vd.data_ptr(), 48, 1234, 500000.0, None) == 0
    torch.cuda.synchronize()
    assert rel_err(vd.cpu().numpy()[:48], orc.rope(x[:48], 1234, 500000.0)) < 1e-5
    assert L.b2_swiglu(od.data_ptr(), xd.data_ptr(), wd.data_ptr(), n, None) == 0
    torch.cuda.synchronize()
    assert rel_err(od.cpu().numpy(), orc.swiglu(x, w)) < 1e-6
    key = torch.zeros(1, dtype=torch.int64, device="cuda")
    assert L.b2_argmax(xd.data_ptr(), n, key.data_ptr(), None) == 0
    torch.cuda.synchronize()
    k = int(key.item()) & 0xFFFFFFFF
    assert 0xFFFFFFFF - k == orc.argmax(x)
