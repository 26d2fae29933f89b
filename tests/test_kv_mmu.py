"""KV-MMU API (include/att1_kv_mmu.h) against the compiled reference (src/kv_mmu.c).

CPU part: configurations are rejected before any device work with the
reference's status codes, and calls on a NULL handle fail cleanly. GPU part:
one sequence of operations (the reference test's isolation / page-boundary
scenario, then a seeded random mix of appends, reads, range copies, lookups,
session churn and invalid calls) replayed on both implementations: every
return code, every output byte and the counters after every call must be
identical. Then the attention kernel reads a session's pages directly
(att1_b200_kv_mmu_layout + b2_attn) and must match a float64 attention.
"""
import ctypes as C

import numpy as np
import pytest


SIGS = {
    "att1_kv_mmu_create": (C.c_int, [C.c_void_p, C.c_void_p]),
    "att1_kv_mmu_destroy": (None, [C.c_void_p]),
    "att1_kv_mmu_create_session": (C.c_int, [C.c_void_p, C.c_uint64]),
    "att1_kv_mmu_destroy_session": (C.c_int, [C.c_void_p, C.c_uint64]),
    "att1_kv_mmu_append": (C.c_int, [C.c_void_p, C.c_uint64, C.c_size_t, C.c_size_t, C.c_void_p, C.c_void_p]),
    "att1_kv_mmu_read": (C.c_int, [C.c_void_p, C.c_uint64, C.c_size_t, C.c_size_t, C.c_size_t, C.c_void_p,
                                   C.c_void_p]),
    "att1_kv_mmu_copy_range": (C.c_int, [C.c_void_p, C.c_uint64, C.c_size_t, C.c_size_t, C.c_size_t, C.c_size_t,
                                         C.c_void_p, C.c_void_p]),
    "att1_kv_mmu_lookup_page": (C.c_int, [C.c_void_p, C.c_uint64, C.c_size_t, C.c_size_t, C.c_void_p]),
    "att1_kv_mmu_get_counters": (None, [C.c_void_p, C.c_void_p]),
    "att1_kv_mmu_reset_counters": (None, [C.c_void_p]),
}


def bind(lib):
    for n, (res, args) in SIGS.items():
        f = getattr(lib, n)
        f.restype = res
        f.argtypes = args
    return lib


@pytest.fixture(scope="module")
def both(b2, ref):
    return bind(b2.lib()), bind(ref.lib)


def cfg(b2, sessions, pages, layers, heads, hd, page_tokens, positions):
    return b2.KvMmuConfig(sessions, pages, layers, heads, hd, page_tokens, positions)


def counters(b2, lib, h):
    k = b2.KvMmuCounters()
    lib.att1_kv_mmu_get_counters(h, C.byref(k))
    return tuple(getattr(k, n) for n, _ in k._fields_)


BAD = [
    (0, 4, 1, 1, 2, 2, 4),                  # no sessions
    (1, 0, 1, 1, 2, 2, 4),                  # no pages
    (1, 4, 0, 1, 2, 2, 4),                  # no layers
    (1, 4, 1, 0, 2, 2, 4),                  # no heads
    (1, 4, 1, 1, 0, 2, 4),                  # no head_dim
    (1, 4, 1, 1, 2, 0, 4),                  # no page_tokens
    (1, 4, 1, 1, 2, 2, 0),                  # no positions
    (1, 4, 1, 1, 2, 2, 9),                  # more positions than pages * page_tokens
    (1, 4, 1, 1 << 62, 1 << 62, 2, 4),      # heads * head_dim overflows
]


@pytest.mark.parametrize("bad", BAD)
def test_invalid_configs_match_reference(b2, both, bad):
    ours, theirs = both
    c = cfg(b2, *bad)
    h1, h2 = C.c_void_p(7), C.c_void_p(7)
    assert ours.att1_kv_mmu_create(C.byref(c), C.byref(h1)) == theirs.att1_kv_mmu_create(C.byref(c), C.byref(h2)) == -1
    assert not h1.value and not h2.value


def test_null_handle(b2, both):
    ours, _ = both
    buf = (C.c_float * 4)()
    assert ours.att1_kv_mmu_create(None, None) == -1
    assert ours.att1_kv_mmu_create_session(None, 1) == -1
    assert ours.att1_kv_mmu_destroy_session(None, 1) == -1
    assert ours.att1_kv_mmu_append(None, 1, 0, 0, buf, buf) == -1
    assert ours.att1_kv_mmu_read(None, 1, 0, 0, 0, buf, buf) == -1
    assert ours.att1_kv_mmu_copy_range(None, 1, 0, 0, 0, 1, buf, buf) == -1
    ours.att1_kv_mmu_get_counters(None, None)
    ours.att1_kv_mmu_reset_counters(None)
    ours.att1_kv_mmu_destroy(None)


class Pair:
    """The same KV-MMU on the device (ours) and on the host (reference)."""

    def __init__(self, b2, both, c):
        self.b2, (self.o, self.r) = b2, both
        self.c = c
        self.ho, self.hr = C.c_void_p(), C.c_void_p()
        assert self.o.att1_kv_mmu_create(C.byref(c), C.byref(self.ho)) == 0
        assert self.r.att1_kv_mmu_create(C.byref(c), C.byref(self.hr)) == 0
        self.hv = c.num_heads * c.head_dim

    def close(self):
        self.o.att1_kv_mmu_destroy(self.ho)
        self.r.att1_kv_mmu_destroy(self.hr)

    def check(self, what):
        a, b = counters(self.b2, self.o, self.ho), counters(self.b2, self.r, self.hr)
        assert a == b, f"{what}: counters {a} != reference {b}"

    def call(self, name, *args, outs=()):
        """Run `name` on both; `outs` are sizes of float output buffers
        (None for a NULL pointer) appended to the arguments."""
        res = []
        for lib, h in ((self.o, self.ho), (self.r, self.hr)):
            bufs = [None if n is None else (C.c_float * max(n, 1))(*([-7.0] * max(n, 1))) for n in outs]
            rc = getattr(lib, name)(h, *args, *bufs)
            res.append((rc, [None if b is None else np.frombuffer(b, np.float32).copy() for b in bufs]))
        (rc1, o1), (rc2, o2) = res
        assert rc1 == rc2, f"{name}{args}: rc {rc1} != reference {rc2}"
        for x, y in zip(o1, o2):
            if x is not None:
                assert x.tobytes() == y.tobytes(), f"{name}{args}: outputs differ"
        self.check(f"{name}{args}")
        return rc1, o1

    def append(self, sid, layer, pos, key, val):
        k = None if key is None else (C.c_float * len(key))(*key)
        v = None if val is None else (C.c_float * len(val))(*val)
        rcs = [lib.att1_kv_mmu_append(h, sid, layer, pos, k, v) for lib, h in ((self.o, self.ho), (self.r, self.hr))]
        assert rcs[0] == rcs[1], f"append({sid},{layer},{pos}): rc {rcs[0]} != reference {rcs[1]}"
        self.check(f"append({sid},{layer},{pos})")
        return rcs[0]

    def lookup(self, sid, layer, pos):
        out = []
        for lib, h in ((self.o, self.ho), (self.r, self.hr)):
            p = self.b2.KvMmuPageRef()
            rc = lib.att1_kv_mmu_lookup_page(h, sid, layer, pos, C.byref(p))
            out.append((rc, tuple(getattr(p, n) for n, _ in p._fields_)))
        assert out[0] == out[1], f"lookup({sid},{layer},{pos}): {out[0]} != reference {out[1]}"
        self.check(f"lookup({sid},{layer},{pos})")
        return out[0]


@pytest.mark.gpu
def test_isolation_and_page_boundaries_match_reference(b2, both):
    """The reference test's scenario: three sessions, two layers, 2-token pages."""
    P = Pair(b2, both, cfg(b2, 4, 16, 3, 2, 2, 2, 6))
    try:
        for sid in (100, 200, 300):
            assert P.call("att1_kv_mmu_create_session", sid)[0] == 0
        assert P.call("att1_kv_mmu_create_session", 200)[0] == -8      # duplicate session (ATT1_ERR_STATE)
        vec = lambda base: [float(base + i) for i in range(4)]
        assert P.append(100, 0, 0, vec(1), vec(101)) == 0
        assert P.append(200, 0, 0, vec(21), vec(201)) == 0
        assert P.append(100, 1, 0, vec(31), vec(301)) == 0
        for sid, layer, head in ((100, 0, 0), (100, 0, 1), (200, 0, 0), (100, 1, 0)):
            assert P.call("att1_kv_mmu_read", sid, layer, head, 0, outs=(2, 2))[0] == 0
        for pos, base in ((1, 5), (2, 9), (3, 13)):
            assert P.append(100, 0, pos, vec(base), vec(100 + base)) == 0
        for pos in range(4):
            assert P.lookup(100, 0, pos)[0] == 0
        assert P.lookup(100, 0, 4)[0] == -5                           # not allocated yet (NOT_FOUND)
        assert P.call("att1_kv_mmu_copy_range", 100, 0, 1, 1, 3, outs=(6, 6))[0] == 0
        assert P.append(100, 0, 5, vec(0), vec(0)) == -8               # gap
        assert P.append(100, 0, 3, vec(0), vec(0)) == -8               # repeat
        assert P.append(100, 0, 6, vec(0), vec(0)) == -1               # beyond max_positions
        assert P.append(100, 3, 0, vec(0), vec(0)) == -1               # bad layer
        assert P.append(999, 0, 0, vec(0), vec(0)) == -5               # unknown session
        assert P.append(100, 0, 4, None, vec(0)) == -1                 # missing key
        assert P.call("att1_kv_mmu_read", 100, 0, 2, 0, outs=(2, 2))[0] == -1   # bad head
        assert P.call("att1_kv_mmu_read", 100, 0, 0, 4, outs=(2, 2))[0] == -5   # not appended
        assert P.call("att1_kv_mmu_read", 100, 0, 0, 0, outs=(None, None))[0] == -1
        assert P.call("att1_kv_mmu_copy_range", 100, 0, 0, 2, 3, outs=(6, 6))[0] == -5  # runs past the end
        assert P.call("att1_kv_mmu_copy_range", 100, 0, 0, 0, 0, outs=(2, 2))[0] == -1
        assert P.call("att1_kv_mmu_destroy_session", 200)[0] == 0
        assert P.call("att1_kv_mmu_destroy_session", 200)[0] == -5
        assert P.call("att1_kv_mmu_read", 200, 0, 0, 0, outs=(2, 2))[0] == -5
        assert P.call("att1_kv_mmu_create_session", 400)[0] == 0
        assert P.append(400, 0, 0, vec(41), vec(401)) == 0             # reuses the freed page
        assert P.lookup(400, 0, 0)[0] == 0
        for b2_, h in ((P.o, P.ho), (P.r, P.hr)):
            b2_.att1_kv_mmu_reset_counters(h)
        P.check("reset")
    finally:
        P.close()


@pytest.mark.gpu
@pytest.mark.parametrize("seed", [1, 2])
def test_random_operations_match_reference(b2, both, seed):
    """Seeded random mix: appends (in and out of order), reads, range copies,
    lookups, session churn until the page pool runs out; codes, bytes and
    counters compared after every call."""
    rng = np.random.default_rng(seed)
    c = cfg(b2, 3, 10, 2, 3, 8, 4, 24)
    P = Pair(b2, both, c)
    try:
        ids = [11, 22, 33, 44]
        length = {}
        for step in range(400):
            op = rng.integers(0, 10)
            sid = int(rng.choice(ids))
            layer = int(rng.integers(0, 3))      # 2 is out of range
            if op == 0:
                P.call("att1_kv_mmu_create_session", sid)
            elif op == 1 and rng.random() < 0.3:
                P.call("att1_kv_mmu_destroy_session", sid)
                for l in range(2):
                    length.pop((sid, l), None)
            elif op <= 5:
                n = length.get((sid, layer), 0)
                pos = n if rng.random() < 0.85 else int(rng.integers(0, 26))
                vals = rng.standard_normal(2 * P.hv).astype(np.float32)
                if P.append(sid, layer, pos, vals[:P.hv].tolist(), vals[P.hv:].tolist()) == 0:
                    length[(sid, layer)] = n + 1
            elif op == 6:
                P.call("att1_kv_mmu_read", sid, layer, int(rng.integers(0, 4)), int(rng.integers(0, 25)),
                       outs=(8, None if rng.random() < 0.3 else 8))
            elif op == 7:
                start, cnt = int(rng.integers(0, 24)), int(rng.integers(0, 8))
                P.call("att1_kv_mmu_copy_range", sid, layer, int(rng.integers(0, 3)), start, cnt,
                       outs=(8 * max(cnt, 1), 8 * max(cnt, 1)))
            else:
                P.lookup(sid, layer, int(rng.integers(0, 25)))
    finally:
        P.close()


@pytest.mark.gpu
@pytest.mark.parametrize("hd", [64, 128])
def test_attention_reads_kv_mmu_pages(b2, both, hd):
    """b2_attn over a session's pages (att1_b200_kv_mmu_layout): grouped-query
    attention of 8 query heads on 2 KV heads at 200 positions (13 pages of 16),
    written through att1_kv_mmu_append, against a float64 attention."""
    import torch
    ours, _ = both
    L = b2.lib()
    Hkv, G, T, n = 2, 4, 16, 200
    c = cfg(b2, 2, 32, 1, Hkv, hd, T, 256)
    h = C.c_void_p()
    assert ours.att1_kv_mmu_create(C.byref(c), C.byref(h)) == 0
    try:
        assert ours.att1_kv_mmu_create_session(h, 5) == 0
        assert ours.att1_kv_mmu_create_session(h, 9) == 0
        rng = np.random.default_rng(3)
        K = rng.standard_normal((n, Hkv, hd)).astype(np.float32)
        V = rng.standard_normal((n, Hkv, hd)).astype(np.float32)
        for p in range(n):
            # another session fills a whole page each time session 9 opens one,
            # so session 9's physical pages alternate with session 5's
            if p % T == 0:
                z = np.zeros(Hkv * hd, np.float32)
                for j in range(T):
                    assert ours.att1_kv_mmu_append(h, 5, 0, p + j, z.ctypes.data, z.ctypes.data) == 0
            assert ours.att1_kv_mmu_append(h, 9, 0, p, K[p].ctypes.data, V[p].ctypes.data) == 0
        lay = b2.KVLayout()
        assert L.att1_b200_kv_mmu_layout(h, 9, 0, C.byref(lay)) == 0
        q = rng.standard_normal((Hkv * G, hd)).astype(np.float32)
        qd = torch.from_numpy(q.reshape(-1)).cuda()
        pos = torch.tensor([n - 1], dtype=torch.int32, device="cuda")
        ctx = torch.zeros(Hkv * G * hd, dtype=torch.float32, device="cuda")
        err = torch.zeros(1, dtype=torch.int32, device="cuda")
        a = b2.AttnArgs()
        a.batch, a.n_heads, a.n_kv_heads, a.head_dim = 1, Hkv * G, Hkv, hd
        a.q, a.kv, a.positions, a.max_ctx, a.ctx, a.err = qd.data_ptr(), lay, pos.data_ptr(), 256, ctx.data_ptr(), \
            err.data_ptr()
        sb = L.b2_attn_scratch_bytes(C.byref(a))
        scratch = torch.zeros(sb, dtype=torch.uint8, device="cuda")
        cnt = torch.zeros(L.b2_attn_counters_len(C.byref(a)), dtype=torch.int32, device="cuda")
        a.scratch, a.scratch_bytes, a.counters, a.counters_len = scratch.data_ptr(), sb, cnt.data_ptr(), cnt.numel()
        assert L.b2_attn(C.byref(a), None) == 0
        torch.cuda.synchronize()
        got = ctx.cpu().numpy().reshape(Hkv * G, hd)
        assert int(err.item()) == 0, f"error word {int(err.item())}, nan {np.isnan(got).sum()}"
        want = np.zeros_like(got, dtype=np.float64)
        for hq in range(Hkv * G):
            kv = hq // G
            s = K[:, kv, :].astype(np.float64) @ q[hq].astype(np.float64) / np.sqrt(hd)
            p = np.exp(s - s.max())
            want[hq] = (p / p.sum()) @ V[:, kv, :].astype(np.float64)
        e = np.abs(got - want).max() / np.abs(want).max()
        assert e <= 1e-5, f"rel err {e:.3e}; worst head/dim {np.unravel_index(np.abs(got - want).argmax(), got.shape)}"
    finally:
        ours.att1_kv_mmu_destroy(h)


@pytest.mark.gpu
def test_decode_on_kv_mmu_sessions_matches_own_pools(b2, both):
    """A two-sequence decode context whose KV lives in KV-MMU sessions
    (att1_b200_infer_use_kv_mmu; another session's appends interleave so the
    pages are scattered) gives bit-identical logits and tokens to the same
    context on its own page pools; the sessions then read back, through the
    KV-MMU API, exactly the K/V that context exports, and the counters show one
    page allocation per (session, layer, 8 positions)."""
    ours, _ = both
    L = b2.lib()
    cfg = b2.Config.make(1000, 2, 4, 2, 128, 256, 64, dtype=4)
    Hkv, hd, layers = 2, 32, 2
    mc = b2.KvMmuConfig(4, 48, layers, Hkv, hd, 8, 64)
    h = C.c_void_p()
    assert ours.att1_kv_mmu_create(C.byref(mc), C.byref(h)) == 0
    a = ref = None
    try:
        for sid in (7, 8, 99):
            assert ours.att1_kv_mmu_create_session(h, sid) == 0
        a = b2.Infer.synth(cfg, 5, batch=2)
        ref = b2.Infer.synth(cfg, 5, batch=2)
        bad = (C.c_uint64 * 2)(8, 7)
        assert L.att1_b200_infer_use_kv_mmu(a.h, h, bad) == -9          # slots out of batch order
        sids = (C.c_uint64 * 2)(7, 8)
        assert L.att1_b200_infer_use_kv_mmu(a.h, h, sids) == 0
        rng = np.random.default_rng(5)
        noise = np.zeros(Hkv * hd, np.float32)
        npos = 0
        for step in range(20):
            if step % 3 == 0:  # the other session takes pages between the context's
                for l in range(layers):
                    assert ours.att1_kv_mmu_append(h, 99, l, npos, noise.ctypes.data, noise.ctypes.data) == 0
                npos += 1
            toks = [int(t) for t in rng.integers(0, 1000, 2)]
            assert list(a.decode_batch(toks)) == list(ref.decode_batch(toks))
            assert np.array_equal(a.logits(), ref.logits())
        a.run_steps(5)
        ref.run_steps(5)
        toks = [3, 4]
        assert list(a.decode_batch(toks)) == list(ref.decode_batch(toks))
        assert np.array_equal(a.logits(), ref.logits())
        n = 26
        assert L.att1_b200_infer_use_kv_mmu(a.h, None, None) == -8    # only at position 0
        with pytest.raises(b2.Att1Error):
            a.prefill([1, 2])                                           # prefill takes one sequence
        k = b2.KvMmuCounters()
        ours.att1_kv_mmu_get_counters(h, C.byref(k))
        assert k.page_allocations == 2 * layers * ((n + 7) // 8) + layers * ((npos + 7) // 8)
        assert k.append_ops == 2 * layers * n + layers * npos
        for item, sid in enumerate((7, 8)):
            for l in range(layers):
                ek = np.zeros((n, Hkv, hd), np.float32)
                ev = np.zeros((n, Hkv, hd), np.float32)
                assert L.att1_b200_infer_export_kv(ref.h, item, l, n, ek.ctypes.data, ev.ctypes.data) == 0
                for hh in range(Hkv):
                    gk = np.zeros((n, hd), np.float32)
                    gv = np.zeros((n, hd), np.float32)
                    assert ours.att1_kv_mmu_copy_range(h, sid, l, hh, 0, n, gk.ctypes.data, gv.ctypes.data) == 0
                    assert np.array_equal(gk, ek[:, hh]) and np.array_equal(gv, ev[:, hh])
    finally:
        for x in (a, ref):
            if x is not None:
                x.close()
        ours.att1_kv_mmu_destroy(h)


@pytest.mark.gpu
def test_prefill_on_kv_mmu_session_matches_own_pools(b2, both):
    """Prompt prefill into a KV-MMU session (pages for the whole prompt mapped
    first, then the tensor-core pass appends there), decode steps with another
    session taking pages in between, and a second prefill further on: tokens
    and logits bit-identical to the same calls on the context's own pools, and
    the session reads back the K/V that context exports."""
    ours, _ = both
    L = b2.lib()
    cfg = b2.Config.make(1000, 2, 4, 2, 128, 256, 64, dtype=4)
    Hkv, hd, layers = 2, 32, 2
    mc = b2.KvMmuConfig(2, 48, layers, Hkv, hd, 8, 64)
    h = C.c_void_p()
    assert ours.att1_kv_mmu_create(C.byref(mc), C.byref(h)) == 0
    a = ref = None
    try:
        for sid in (5, 99):
            assert ours.att1_kv_mmu_create_session(h, sid) == 0
        a = b2.Infer.synth(cfg, 11, batch=1)
        ref = b2.Infer.synth(cfg, 11, batch=1)
        assert L.att1_b200_infer_use_kv_mmu(a.h, h, (C.c_uint64 * 1)(5)) == 0
        rng = np.random.default_rng(8)
        noise = np.zeros(Hkv * hd, np.float32)
        npos = 0
        p1 = [int(t) for t in rng.integers(0, 1000, 19)]
        assert a.prefill(p1) == ref.prefill(p1)
        assert np.array_equal(a.logits(), ref.logits())
        for _ in range(3):
            for l in range(layers):
                assert ours.att1_kv_mmu_append(h, 99, l, npos, noise.ctypes.data, noise.ctypes.data) == 0
            npos += 1
            t = int(rng.integers(0, 1000))
            assert a.decode(t) == ref.decode(t)
            assert np.array_equal(a.logits(), ref.logits())
        p2 = [int(t) for t in rng.integers(0, 1000, 11)]
        assert a.prefill(p2) == ref.prefill(p2)
        assert np.array_equal(a.logits(), ref.logits())
        n = 19 + 3 + 11
        assert a.position() == ref.position() == n
        k = b2.KvMmuCounters()
        ours.att1_kv_mmu_get_counters(h, C.byref(k))
        assert k.page_allocations == layers * ((n + 7) // 8) + layers * ((npos + 7) // 8)
        assert k.append_ops == layers * n + layers * npos
        with pytest.raises(b2.Att1Error):
            a.prefill([1] * (64 - n + 1))                               # past max_positions
        for l in range(layers):
            ek = np.zeros((n, Hkv, hd), np.float32)
            ev = np.zeros((n, Hkv, hd), np.float32)
            assert L.att1_b200_infer_export_kv(ref.h, 0, l, n, ek.ctypes.data, ev.ctypes.data) == 0
            for hh in range(Hkv):
                gk = np.zeros((n, hd), np.float32)
                gv = np.zeros((n, hd), np.float32)
                assert ours.att1_kv_mmu_copy_range(h, 5, l, hh, 0, n, gk.ctypes.data, gv.ctypes.data) == 0
                assert np.array_equal(gk, ek[:, hh]) and np.array_equal(gv, ev[:, hh])
    finally:
        for x in (a, ref):
            if x is not None:
                x.close()
        ours.att1_kv_mmu_destroy(h)
