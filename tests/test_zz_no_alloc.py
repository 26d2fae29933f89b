"""b2_gemv_noalloc: the GEMV entry point that takes its scratch from a fixed
device array instead of the caller (b2_kernels.h). Kept in its own file, run
last, so it is checked both in a fresh process and after every other test has
used the device.

Each case runs the allocating entry point (b2_gemv, caller-owned scratch and
counters) once and the allocation-free one twice in a row on the same inputs;
all three must agree within the GEMV tolerance of the kernel tests.
"""
import ctypes as C

import numpy as np
import pytest

from test_gpu_kernels import GEMV_RTOL, q4_device, q8_device, rel_err

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    import torch
    torch.cuda.init()
    return torch


def make_args(b2, torch, fmt, buf, rs, rows, cols, x, epilogue=0):
    batch = x.shape[0]
    keep = {}
    keep["x"] = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).cuda()
    keep["err"] = torch.zeros(1, dtype=torch.int32, device="cuda")
    out_rows = rows // 2 if epilogue == 3 else rows
    keep["out"] = torch.zeros(batch * out_rows, dtype=torch.float32, device="cuda")
    a = b2.GemvArgs()
    a.w = b2.QWeight(buf.data_ptr(), rs.data_ptr() if rs is not None else None, fmt, rows, cols,
                     (rows + 15) // 16, (cols + 63) // 64 if fmt == 4 else (cols + 31) // 32)
    a.batch = batch
    a.x = keep["x"].data_ptr()
    a.x_stride = cols
    a.eps = 1e-5
    a.epilogue = epilogue
    a.out = keep["out"].data_ptr()
    a.out_stride = out_rows
    a.err = keep["err"].data_ptr()
    return a, keep


def read_out(torch, keep, batch):
    torch.cuda.synchronize()
    assert int(keep["err"].item()) == 0
    return keep["out"].cpu().numpy().reshape(batch, -1).copy()


def run_with_scratch(b2, torch, a, keep, batch):
    L = b2.lib()
    need = L.b2_gemv_scratch_bytes(C.byref(a))
    scratch = torch.zeros(need, dtype=torch.uint8, device="cuda")
    counters = torch.zeros(L.b2_gemv_counters_len(C.byref(a)), dtype=torch.int32, device="cuda")
    a.scratch, a.scratch_bytes = scratch.data_ptr(), need
    a.counters, a.counters_len = counters.data_ptr(), counters.numel()
    assert L.b2_gemv(C.byref(a), None) == 0
    return read_out(torch, keep, batch)


def run_noalloc(b2, torch, a, keep, batch):
    a.scratch, a.scratch_bytes, a.counters, a.counters_len = None, 0, None, 0
    keep["out"].zero_()
    assert b2.lib().b2_gemv_noalloc(C.byref(a), None) == 0
    return read_out(torch, keep, batch)


def check_agree(b2, torch, fmt, buf, rs, rows, cols, x, epilogue=0):
    a, keep = make_args(b2, torch, fmt, buf, rs, rows, cols, x, epilogue)
    batch = x.shape[0]
    want = run_with_scratch(b2, torch, a, keep, batch)
    first = run_noalloc(b2, torch, a, keep, batch)
    second = run_noalloc(b2, torch, a, keep, batch)
    assert np.isfinite(want).all()
    assert rel_err(first, want) <= GEMV_RTOL
    assert rel_err(second, want) <= GEMV_RTOL
    return want


@pytest.mark.parametrize("rows,cols,batch", [(4096, 4096, 1), (1000, 4096, 3), (128256, 4096, 1)])
def test_noalloc_q4_matches_b2_gemv(b2, torch, orc, rows, cols, batch):
    L = b2.lib()
    buf = torch.zeros(L.b2_q4_bytes(rows, cols), dtype=torch.uint8, device="cuda")
    assert L.b2_q4_synth(buf.data_ptr(), 0, rows, cols, 91, rows, 0, 0.02, 0, None) == 0
    x = orc.synth_normal(92, cols, batch * cols, std=1.0).reshape(batch, cols)
    check_agree(b2, torch, 4, buf, None, rows, cols, x)


def test_noalloc_q4_swiglu_epilogue(b2, torch, orc):
    L = b2.lib()
    F, d = 14336, 4096
    buf = torch.zeros(L.b2_q4_bytes(2 * F, d), dtype=torch.uint8, device="cuda")
    assert L.b2_q4_synth(buf.data_ptr(), 0, 2 * F, d, 93, 6, 7, 0.02, 1, None) == 0
    x = orc.synth_normal(94, d, 2 * d, std=1.0).reshape(2, d)
    check_agree(b2, torch, 4, buf, None, 2 * F, d, x, epilogue=3)


@pytest.mark.parametrize("rows,cols,batch", [(2048, 4096, 4), (300, 288, 1)])
def test_noalloc_q8_matches_b2_gemv(b2, torch, orc, rows, cols, batch):
    w = orc.synth_normal(95, rows, rows * cols).reshape(rows, cols)
    v, s = orc.q8_quantize(w)
    buf, rs = q8_device(b2, torch, v, s, rows, cols)
    x = orc.synth_normal(96, cols, batch * cols, std=1.0).reshape(batch, cols)
    want = check_agree(b2, torch, 8, buf, rs, rows, cols, x)
    assert rel_err(want, orc.matmul_q8(x, v, s, rows, cols, threads=8)) <= GEMV_RTOL


def test_noalloc_rejects_tiling_it_cannot_hold(b2, torch, orc):
    """A GEMV whose digit planes do not fit on chip is refused before any launch,
    by the allocation-free entry point exactly as by b2_gemv."""
    L = b2.lib()
    rows, cols, batch = 64, 14336, 16
    w = orc.synth_normal(97, rows, rows * cols).reshape(rows, cols)
    p, s = orc.q4_quantize(w)
    buf = q4_device(b2, torch, p, s, rows, cols)
    a, keep = make_args(b2, torch, 4, buf, None, rows, cols, np.ones((batch, cols), dtype=np.float32))
    assert L.b2_gemv_scratch_bytes(C.byref(a)) == 0
    assert L.b2_gemv_noalloc(C.byref(a), None) == -9
    torch.cuda.synchronize()
    assert int(keep["err"].item()) == 0
    assert L.b2_gemv_noalloc(None, None) == -1
    # an invalid call (no input vector) is rejected before the shared array is touched
    bad, bkeep = make_args(b2, torch, 4, buf, None, rows, cols, np.ones((1, cols), dtype=np.float32))
    bad.x = None
    assert L.b2_gemv_noalloc(C.byref(bad), None) == -1
    bad.x = bkeep["x"].data_ptr()
    bad.out = None
    assert L.b2_gemv_noalloc(C.byref(bad), None) == -1
