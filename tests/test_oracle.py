"""The oracle (CPU restatement) pinned against the reference compiled from its
own sources (oracle/_ref) and against the reference tests' known answers.

Known answers restated from the reference test files (by value, not code):
tests/test_quant_q4_pack.c:41-94 (nibble order), :98-131 (round trip of all
values), :135-171 (saturation), :175-200 (all-zero group -> scale 1.0);
tests/test_matmul_q4.c:124-160 (hand-checkable 2x16 case).
"""
import ctypes as C

import numpy as np
import pytest

import oracle as O


def _q4_group_from_values(orc, q, scale=1.0, group=16):
    """Input whose quantisation is exactly the int4 values q (|q| <= 7): x = q
    with max |x| = 7 gives scale 1 (ensured by appending a 7 when needed)."""
    x = np.zeros(group, np.float32)
    x[: len(q)] = q
    return x


def test_nibble_order_reference(ref):
    src = (C.c_int8 * 16)(-3, 5)
    dst = (C.c_uint8 * 8)()
    assert ref.lib.rh_pack_group(src, 16, dst) == 0
    assert dst[0] == 0x5D
    back = (C.c_int8 * 16)()
    assert ref.lib.rh_unpack_group(dst, 16, back) == 0
    assert (back[0], back[1]) == (-3, 5)


def test_nibble_order_oracle(orc):
    # row [-3, 5, 0.., 7]: max 7 -> scale 1 -> q = x exactly
    w = np.zeros((1, 32), np.float32)
    w[0, 0], w[0, 1], w[0, 31] = -3, 5, 7
    packed, scales = orc.q4_quantize(w)
    assert packed[0] == 0x5D
    assert scales[0] == 1.0


def test_all_values_round_trip(orc, ref):
    vals = np.array([0, -1, 1, -2, 2, -3, 3, -4, 4, -5, 5, -6, 6, -7, 7, 0], np.float32)
    w = np.concatenate([vals, vals]).reshape(1, 32)
    p1, s1 = orc.q4_quantize(w)
    p2, s2 = ref.q4_quantize(w)
    assert (p1 == p2).all() and (s1 == s2).all() and s1[0] == 1.0
    lo = (p1 & 0xF).astype(np.int8)
    hi = (p1 >> 4).astype(np.int8)
    lo = np.where(lo > 7, lo - 16, lo)
    hi = np.where(hi > 7, hi - 16, hi)
    got = np.empty(32, np.int8)
    got[0::2], got[1::2] = lo, hi
    assert (got == w[0].astype(np.int8)).all()


def test_saturation_reference(ref):
    src = (C.c_int8 * 16)(127, -127)
    dst = (C.c_uint8 * 8)()
    assert ref.lib.rh_pack_group(src, 16, dst) == 0
    back = (C.c_int8 * 16)()
    ref.lib.rh_unpack_group(dst, 16, back)
    assert (back[0], back[1]) == (7, -7) and all(v == 0 for v in back[2:])


def test_zero_group_scale_one(orc, ref):
    w = np.zeros((3, 64), np.float32)
    for q in (orc, ref):
        p, s = q.q4_quantize(w)
        assert (p == 0).all() and (s == 1.0).all()
    v, s = orc.q8_quantize(w)
    assert (v == 0).all() and (s == 1.0).all()


def test_nonfinite_rejected(orc, ref):
    w = np.zeros((1, 32), np.float32)
    w[0, 3] = np.inf
    for q in (orc, ref):
        with pytest.raises(ValueError):
            q.q4_quantize(w)
    w[0, 3] = np.nan
    with pytest.raises(ValueError):
        orc.q8_quantize(w)


def test_halfway_rounding(orc, ref):
    # x / scale lands on k + 0.5: lroundf rounds half away from zero
    w = np.array([[7.0, 0.5, -0.5, 1.5, -1.5, 2.5, -2.5, 6.5] * 4], np.float32)
    p1, s1 = orc.q4_quantize(w)
    p2, s2 = ref.q4_quantize(w)
    assert (p1 == p2).all() and (s1 == s2).all()
    assert p1[0] == (0x7 | (0x1 << 4))  # 7 and round(0.5) = 1


@pytest.mark.parametrize("shape", [(16, 32), (37, 96), (128, 288), (64, 1024)])
def test_q4_quantiser_bit_exact(orc, ref, shape):
    w = orc.synth_normal(11, 3, shape[0] * shape[1]).reshape(shape)
    p1, s1 = orc.q4_quantize(w)
    p2, s2 = ref.q4_quantize(w)
    assert (p1 == p2).all()
    assert (s1.view(np.uint32) == s2.view(np.uint32)).all()


@pytest.mark.parametrize("shape", [(16, 32), (33, 288), (128, 768)])
def test_q8_quantiser_bit_exact(orc, ref, shape):
    w = orc.synth_normal(12, 4, shape[0] * shape[1]).reshape(shape)
    v1, s1 = orc.q8_quantize(w)
    v2, s2 = ref.q8_quantize(w)
    assert (v1 == v2).all()
    assert (s1.view(np.uint32) == s2.view(np.uint32)).all()


@pytest.mark.parametrize("batch", [1, 3])
def test_matmuls_bit_exact(orc, ref, batch):
    rows, cols = 48, 256
    w = orc.synth_normal(5, 6, rows * cols).reshape(rows, cols)
    x = orc.synth_normal(5, 7, batch * cols, std=1.0).reshape(batch, cols)
    p, s = orc.q4_quantize(w)
    a = orc.matmul_q4(x, p, s, rows, cols, threads=3)
    b = ref.matmul_q4(x, p, s, rows, cols)
    assert (a.view(np.uint32) == b.view(np.uint32)).all()
    v, s8 = orc.q8_quantize(w)
    a = orc.matmul_q8(x, v, s8, rows, cols, threads=2)
    b = ref.matmul_q8(x, v, s8, rows, cols)
    assert (a.view(np.uint32) == b.view(np.uint32)).all()


def test_hand_case_matmul(orc):
    # tests/test_matmul_q4.c:115-160: row 0 all 0.5, row 1 alternating +1/-1,
    # lhs all ones -> [8, 0]
    w = np.zeros((2, 16), np.float32)
    w[0] = 0.5
    w[1] = [1.0 if i % 2 == 0 else -1.0 for i in range(16)]
    w32 = np.concatenate([w, np.zeros((2, 16), np.float32)], axis=1)
    p, s = orc.q4_quantize(w32)
    y = orc.matmul_q4(np.ones(32, np.float32), p, s, 2, 32)[0]
    assert abs(y[0] - 8.0) < 1e-5 and abs(y[1]) < 1e-5


def test_element_ops_bit_exact(orc, ref):
    x = orc.synth_normal(9, 1, 96, std=1.0)
    w = orc.synth_normal(9, 2, 96, std=1.0)
    out = np.empty_like(x)
    assert ref.lib.rh_rmsnorm(O._fp(out), O._fp(x), O._fp(w), 96, 1e-5) == 0
    assert (orc.rmsnorm(x, w, 1e-5) == out).all()
    r = x.copy()
    assert ref.lib.rh_rope(O._fp(r), 96, 37, 500000.0) == 0
    assert (orc.rope(x, 37, 500000.0) == r).all()
    sm = x.copy()
    assert ref.lib.rh_softmax(O._fp(sm), 96) == 0
    assert (orc.softmax(x) == sm).all()
    sw = np.empty_like(x)
    assert ref.lib.rh_swiglu(O._fp(sw), O._fp(x), O._fp(w), 96) == 0
    assert (orc.swiglu(x, w) == sw).all()


def test_argmax_ties_and_nan(orc, ref):
    v = np.array([1.0, 3.0, 3.0, -1.0], np.float32)
    assert orc.argmax(v) == 1
    o = C.c_uint32()
    assert ref.lib.rh_argmax(O._fp(v), 4, C.byref(o)) == 0 and o.value == 1
    v[2] = np.nan
    assert orc.argmax(v) is None
    assert ref.lib.rh_argmax(O._fp(v), 4, C.byref(o)) != 0


@pytest.mark.parametrize("dtype,heads,kv", [(O.Q4, 4, 2), (O.Q4, 4, 4), (O.Q8, 4, 1)])
def test_decode_bit_exact(orc, ref, dtype, heads, kv):
    cfg = O.Config.make(vocab=300, n_layers=2, n_heads=heads, n_kv_heads=kv, d_model=64, d_ff=96,
                        max_seq=16, dtype=dtype, eps=1e-5, theta=10000.0)
    om, rm = orc.model(cfg, 21), ref.model(cfg, 21)
    for t in [1, 299, 17, 5, 5, 200]:
        lo, no = om.decode(t)
        lr, nr = rm.decode(t)
        assert no == nr
        assert (lo.view(np.uint32) == lr.view(np.uint32)).all()


def test_decode_thread_count_invariant(orc):
    cfg = O.Config.make(vocab=500, n_layers=1, n_heads=2, n_kv_heads=1, d_model=64, d_ff=64,
                        max_seq=8, dtype=O.Q4)
    a, b = orc.model(cfg, 3, threads=1), orc.model(cfg, 3, threads=5)
    for t in [3, 4, 9]:
        la, _ = a.decode(t)
        lb, _ = b.decode(t)
        assert (la.view(np.uint32) == lb.view(np.uint32)).all()


def test_synth_generator_statistics(orc):
    v = orc.synth_normal(1, 2, 200000)
    assert abs(float(v.mean())) < 2e-4
    assert abs(float(v.std()) - 0.02) < 2e-4
    assert (orc.synth_normal(1, 2, 10, first=5) == v[5:15]).all()
    toks = orc.synth_tokens(7, 1000, 32000)
    assert toks.min() >= 0 and toks.max() < 32000 and len(set(toks.tolist())) > 900
