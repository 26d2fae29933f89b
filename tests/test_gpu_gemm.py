"""Dequant GEMM on the tensor cores (b2_gemm, tcgen05) against the oracle.

out[n][o] = sum_k x[n][k] * W[o][k] for many rows of x at once (prefill and
large decode batches), through the C ABI. The kernel splits every f32 operand
into bf16 hi + lo and accumulates in f32 in tensor memory; the dropped terms
are below 2^-16 relative, so results must match the oracle's f32 matmul
(att1_matmul_q4xf32 / _q8xf32 rounding) at max|gpu - cpu| / max|cpu| <= 2e-5,
the GEMV's tolerance. Shapes cover ragged row tiles, several token tiles, k
splits with their reduction, the residual epilogue and the RMSNorm prologue.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
GEMM_RTOL = 2e-5


def rel_err(a, b):
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


@pytest.fixture(scope="module")
def torch():
    import torch
    torch.cuda.init()
    return torch


def dev(torch, a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def weights(b2, torch, orc, fmt, rows, cols, seed):
    L = b2.lib()
    w = orc.synth_normal(seed, 1, rows * cols).reshape(rows, cols)
    if fmt == 4:
        packed, scales = orc.q4_quantize(w)
        buf = torch.zeros(L.b2_q4_bytes(rows, cols), dtype=torch.uint8, device="cuda")
        p, s = dev(torch, packed), dev(torch, scales)
        assert L.b2_q4_pack(buf.data_ptr(), 0, rows, cols, p.data_ptr(), s.data_ptr(), None, None, 32, 0, None) == 0
        torch.cuda.synchronize()
        return buf, None, lambda x: orc.matmul_q4(x, packed, scales, rows, cols, threads=16)
    values, scales = orc.q8_quantize(w)
    buf = torch.zeros(L.b2_q8_bytes(rows, cols), dtype=torch.uint8, device="cuda")
    rs = torch.zeros(((rows + 15) // 16) * 16, dtype=torch.float32, device="cuda")
    v, s = dev(torch, values), dev(torch, scales)
    assert L.b2_q8_pack(buf.data_ptr(), rs.data_ptr(), 0, rows, cols, v.data_ptr(), s.data_ptr(),
                        None, None, 0, None) == 0
    torch.cuda.synchronize()
    return buf, rs, lambda x: orc.matmul_q8(x, values, scales, rows, cols, threads=16)


def run_gemm(b2, torch, fmt, buf, rs, rows, cols, x, norm_w=None, eps=1e-5, resid=None, splits=0):
    L = b2.lib()
    m = x.shape[0]
    xd = dev(torch, x.astype(np.float32))
    xs = torch.full((L.b2_gemm_xs_bytes(m, cols),), 0x55, dtype=torch.uint8, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    nw = dev(torch, norm_w) if norm_w is not None else None
    assert L.b2_gemm_prep(xd.data_ptr(), cols, m, cols, nw.data_ptr() if nw is not None else None, eps,
                          xs.data_ptr(), err.data_ptr(), None) == 0
    out = torch.full((m * rows,), float("nan"), dtype=torch.float32, device="cuda")
    a = b2.GemmArgs()
    a.w = b2.QWeight(buf.data_ptr(), rs.data_ptr() if rs is not None else None, fmt, rows, cols,
                     (rows + 15) // 16, (cols + 63) // 64 if fmt == 4 else (cols + 31) // 32)
    a.xs = xs.data_ptr()
    a.m = m
    a.epilogue = 0 if resid is None else 1
    a.out = out.data_ptr()
    a.out_stride = rows
    rd = dev(torch, resid.astype(np.float32)) if resid is not None else None
    a.resid = rd.data_ptr() if rd is not None else None
    a.splits = splits
    a.err = err.data_ptr()
    need = L.b2_gemm_scratch_bytes(C.byref(a))
    assert need > 0
    scratch = torch.full((need,), 0x7F, dtype=torch.uint8, device="cuda")
    a.scratch = scratch.data_ptr()
    a.scratch_bytes = need
    assert L.b2_gemm(C.byref(a), None) == 0
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return out.cpu().numpy().reshape(m, rows)


@pytest.mark.parametrize("fmt", [4, 8])
@pytest.mark.parametrize("rows,cols,m", [(40, 192, 5), (128, 64, 16), (100, 288, 33)])
def test_gemm_small_shapes(b2, torch, orc, fmt, rows, cols, m):
    buf, rs, ref = weights(b2, torch, orc, fmt, rows, cols, 3)
    x = np.random.default_rng(1).normal(0, 1, (m, cols)).astype(np.float32)
    got = run_gemm(b2, torch, fmt, buf, rs, rows, cols, x)
    assert rel_err(got, ref(x)) <= GEMM_RTOL


@pytest.mark.parametrize("fmt", [4, 8])
def test_gemm_token_tiles_and_k_splits(b2, torch, orc, fmt):
    """300 rows of x: two token tiles of 160; 4096 columns over 2 row blocks:
    the k range is split over CTAs and the partials reduced in split order."""
    rows, cols, m = 256, 4096, 300
    buf, rs, ref = weights(b2, torch, orc, fmt, rows, cols, 5)
    x = np.random.default_rng(2).normal(0, 1, (m, cols)).astype(np.float32)
    want = ref(x)
    auto = run_gemm(b2, torch, fmt, buf, rs, rows, cols, x)
    one = run_gemm(b2, torch, fmt, buf, rs, rows, cols, x, splits=1)
    assert rel_err(auto, want) <= GEMM_RTOL
    assert rel_err(one, want) <= GEMM_RTOL


def test_gemm_residual_and_norm(b2, torch, orc):
    rows, cols, m = 192, 512, 24
    buf, rs, ref = weights(b2, torch, orc, 4, rows, cols, 7)
    rng = np.random.default_rng(3)
    x = rng.normal(0, 1, (m, cols)).astype(np.float32)
    nw = rng.uniform(0.5, 1.5, cols).astype(np.float32)
    resid = rng.normal(0, 1, (m, rows)).astype(np.float32)
    xn = np.stack([orc.rmsnorm(x[i], nw, 1e-5) for i in range(m)])
    got = run_gemm(b2, torch, 4, buf, rs, rows, cols, x, norm_w=nw, resid=resid)
    want = resid + ref(xn)
    assert rel_err(got, want) <= GEMM_RTOL


def test_gemm_8b_down_projection_batch32(b2, torch, orc):
    """Llama-3-8B FFN down projection (4096 x 14336) for a 32-sequence decode batch."""
    rows, cols, m = 4096, 14336, 32
    buf, rs, ref = weights(b2, torch, orc, 4, rows, cols, 9)
    x = np.random.default_rng(4).normal(0, 1, (m, cols)).astype(np.float32)
    got = run_gemm(b2, torch, 4, buf, rs, rows, cols, x)
    assert rel_err(got, ref(x)) <= GEMM_RTOL
