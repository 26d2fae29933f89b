"""Sampling: the greedy host sampler against the compiled reference (CPU), and
the device top-k / temperature sampler against a numpy restatement (GPU).

att1_sampler_greedy_f32 (include/att1_sampler.h) must return what the
reference's src/sampler.c:5-34 returns on the same buffer: first maximum, -1
on NaN / empty / NULL. b2_sample_topk and att1_b200_infer_set_sampler have no
reference counterpart (the reference declares att1_sampler_config only); their
rule is restated below in numpy: the top_k logits by (value desc, id asc),
weights exp((l - l_max) / T) in float32 summed in that order, u = 24 bits of
splitmix64(splitmix64(seed) ^ (item << 32 | position)), the first rank whose
running sum exceeds u * sum. The device expf may differ from numpy's float32
exp in the last bit, so a different token is accepted only where u * sum lies
within 1e-5 (relative) of a running-sum boundary.
"""
import ctypes as C

import numpy as np
import pytest

M64 = (1 << 64) - 1
BOUNDARY = 1e-5


def splitmix64(x):
    z = (x + 0x9E3779B97F4A7C15) & M64
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M64
    return z ^ (z >> 31)


def sample_ref(row, k, temperature, seed, item, position):
    """(token, distance of u*sum to the nearest running-sum boundary / sum)."""
    row = np.asarray(row, np.float32)
    order = np.lexsort((np.arange(row.size), -row))[:k]
    v = row[order]
    if v[0] == -np.inf:
        return int(order[0]), np.inf
    if v[0] == np.inf:                      # the +inf entries share all the weight
        w = (v == np.inf).astype(np.float32)
    else:
        w = np.exp((v - v[0]) / np.float32(temperature)).astype(np.float32)
    s = np.float32(0)
    for x in w:
        s = np.float32(s + x)
    r = splitmix64(splitmix64(seed) ^ ((item << 32) | position))
    u = np.float32(r >> 40) * np.float32(2.0 ** -24)
    target = np.float32(u * s)
    acc, sel, margin = np.float32(0), k - 1, np.inf
    for j in range(k - 1):
        acc = np.float32(acc + w[j])
        margin = min(margin, abs(float(acc) - float(target)) / float(s))
        if acc > target:
            sel = j
            break
    return int(order[sel]), margin


def agree(got, row, k, temperature, seed, item, position):
    want, margin = sample_ref(row, k, temperature, seed, item, position)
    return int(got) == want or margin <= BOUNDARY


def test_greedy_host_sampler_matches_reference(b2, ref):
    rf = ref.lib.att1_sampler_greedy_f32
    rf.restype = C.c_int
    rf.argtypes = [C.c_void_p, C.c_size_t, C.POINTER(C.c_uint32)]
    ours = b2.lib().att1_sampler_greedy_f32
    rng = np.random.default_rng(4)
    rows = [rng.normal(0, 1, 1000).astype(np.float32),
            np.full(37, 2.5, np.float32),                          # all tied: id 0
            np.array([-np.inf, -1.0, 3.0, 3.0, 2.0], np.float32),  # tie: first of the two
            np.array([1.0, np.nan, 5.0], np.float32),              # NaN rejected
            np.array([-np.inf, -np.inf], np.float32)]
    for row in rows:
        a, b = C.c_uint32(77), C.c_uint32(77)
        ra = ours(row.ctypes.data, row.size, C.byref(a))
        rb = rf(row.ctypes.data, row.size, C.byref(b))
        assert (ra, a.value) == (rb, b.value)
    t = C.c_uint32(0)
    assert ours(rows[0].ctypes.data, 0, C.byref(t)) == -1
    assert ours(None, 3, C.byref(t)) == -1


def test_sampler_restatement_edges():
    inf_row = np.array([0.0, np.inf, 3.0, np.inf], np.float32)
    assert {sample_ref(inf_row, 3, 1.0, 5, 0, p)[0] for p in range(64)} == {1, 3}
    assert sample_ref(np.full(4, -np.inf, np.float32), 3, 1.0, 5, 0, 1)[0] == 0
    row = np.array([0.0, 5.0, 5.0, 1.0], np.float32)
    # top 1 and a huge-weight gap reduce to greedy (ties: lowest id)
    assert sample_ref(row, 1, 1.0, 9, 0, 3)[0] == 1
    assert sample_ref(np.array([0.0, 100.0, -100.0], np.float32), 3, 0.5, 1, 2, 8)[0] == 1


def test_sampler_rule_draws_the_topk_softmax():
    """The stated rule samples softmax(l / T) restricted to the top k: over
    20000 positions the frequencies of a 6-logit row with k = 4 match the
    probabilities within 4 standard errors, and the two excluded ids never
    appear."""
    row = np.array([1.0, 3.0, 2.5, -1.0, 2.0, 0.5], np.float32)
    k, T, n = 4, 1.5, 20000
    top = [1, 2, 4, 0]
    e = np.exp((row[top] - row[top].max()) / T)
    p = e / e.sum()
    counts = np.zeros(row.size)
    for pos in range(n):
        counts[sample_ref(row, k, T, 42, 0, pos)[0]] += 1
    assert counts[3] == 0 and counts[5] == 0
    f = counts[top] / n
    se = np.sqrt(p * (1 - p) / n)
    assert (np.abs(f - p) <= 4 * se).all(), (f, p)


@pytest.fixture(scope="module")
def torch():
    import torch
    torch.cuda.init()
    return torch


@pytest.mark.gpu
@pytest.mark.parametrize("k,temperature", [(2, 1.0), (50, 0.7), (256, 2.5)])
def test_sample_topk_kernel_matches_restatement(b2, torch, k, temperature):
    """Llama-3 vocabulary rows: plain normal logits, logits rounded to halves
    (ties straddle the k-th value), and a row with -inf entries."""
    V, stride = 128256, 128260
    rng = np.random.default_rng(k)
    rows = np.zeros((4, stride), np.float32)
    rows[0, :V] = rng.normal(0, 3, V)
    rows[1, :V] = np.round(rng.normal(0, 2, V) * 2) / 2
    rows[2, :V] = rng.normal(0, 1, V)
    rows[2, rng.integers(0, V, 5000)] = -np.inf
    rows[3, :V] = rng.normal(0, 1, V)
    rows[3, [7, 90000, 128255]] = np.inf                   # +inf: only these three can be drawn
    positions = np.array([5, 17, 4095, 33], np.int32)
    lg = torch.from_numpy(rows.reshape(-1)).cuda()
    pos = torch.from_numpy(positions).cuda()
    L = b2.lib()
    inf_draws = set()
    for seed in (1, 2, 3, 4, 5, 6):
        tok = torch.full((4,), -1, dtype=torch.int32, device="cuda")
        assert L.b2_sample_topk(lg.data_ptr(), 4, V, stride, k, temperature, seed, pos.data_ptr(),
                                tok.data_ptr(), 0, None) == 0
        torch.cuda.synchronize()
        got = tok.cpu().numpy().view(np.uint32)
        for b in range(4):
            assert agree(got[b], rows[b, :V], k, temperature, seed, b, int(positions[b])), (b, got[b])
        assert int(got[3]) in (7, 90000, 128255)
        inf_draws.add(int(got[3]))
    assert len(inf_draws) >= 2 or k == 2       # the +inf entries share the draw (k = 2 holds two of them)
    tok = torch.zeros(3, dtype=torch.int32, device="cuda")
    assert L.b2_sample_topk(lg.data_ptr(), 3, V, stride, 257, 1.0, 1, pos.data_ptr(), tok.data_ptr(), 0, None) == -1
    assert L.b2_sample_topk(lg.data_ptr(), 3, V, stride, 8, 0.0, 1, pos.data_ptr(), tok.data_ptr(), 0, None) == -1


@pytest.mark.gpu
def test_sample_topk_sharded_layout(b2, torch):
    """Four vocabulary shards laid out [shard][item][rows] (the tensor-parallel
    all-gather) draw the same tokens as the same logits in one [item][vocab]
    buffer."""
    V, S, B = 128256, 4, 3
    R = V // S
    rng = np.random.default_rng(12)
    rows = rng.normal(0, 2, (B, V)).astype(np.float32)
    sharded = np.ascontiguousarray(rows.reshape(B, S, R).transpose(1, 0, 2))
    positions = np.array([9, 10, 11], np.int32)
    pos = torch.from_numpy(positions).cuda()
    flat, shd = torch.from_numpy(rows.reshape(-1)).cuda(), torch.from_numpy(sharded.reshape(-1)).cuda()
    L = b2.lib()
    a = torch.full((B,), -1, dtype=torch.int32, device="cuda")
    c = torch.full((B,), -1, dtype=torch.int32, device="cuda")
    assert L.b2_sample_topk(flat.data_ptr(), B, V, V, 40, 0.8, 6, pos.data_ptr(), a.data_ptr(), 0, None) == 0
    assert L.b2_sample_topk_sharded(shd.data_ptr(), B, V, R, B * R, R, 40, 0.8, 6, pos.data_ptr(), c.data_ptr(),
                                    0, None) == 0
    torch.cuda.synchronize()
    assert (a.cpu().numpy() == c.cpu().numpy()).all()
    for b in range(B):
        assert agree(int(a[b]), rows[b], 40, 0.8, 6, b, int(positions[b]))
    assert L.b2_sample_topk_sharded(shd.data_ptr(), B, V, R + 1, B * R, R + 1, 40, 0.8, 6, pos.data_ptr(),
                                    c.data_ptr(), 0, None) == -1                     # shards must tile the vocabulary


@pytest.mark.gpu
def test_context_sampler_decode_and_prefill(b2):
    """A 4-sequence context with top-k sampling: every step's tokens follow
    from that step's logits by the restated rule, a second context with the
    same seed repeats the run, top_k 1 is greedy again, and the token after a
    prefill is drawn the same way."""
    cfg = b2.Config.make(1000, 2, 4, 2, 128, 256, 64, dtype=4)
    k, T, seed = 20, 0.9, 3
    runs = []
    for _ in range(2):
        inf = b2.Infer.synth(cfg, 21, batch=4)
        inf.set_sampler(k, T, seed)
        toks = [1, 2, 3, 4]
        seq = []
        for _ in range(6):
            toks = inf.decode_batch(toks)
            logits = inf.logits()
            pos = inf.position()
            for b in range(4):
                assert agree(toks[b], logits[b], k, T, seed, b, pos)
            seq.append(list(toks))
        inf.set_sampler(0)
        out = inf.decode_batch(toks)
        assert list(out) == [int(np.argmax(r)) for r in inf.logits()]
        inf.close()
        runs.append(seq)
    assert runs[0] == runs[1]
    one = b2.Infer.synth(cfg, 21, batch=1)
    with pytest.raises(b2.Att1Error):
        one.set_sampler(300, 1.0, 0)                                    # top_k above 256
    with pytest.raises(b2.Att1Error):
        one.set_sampler(4, -1.0, 0)                                     # temperature not positive
    one.set_sampler(k, T, seed)
    t = one.prefill([5, 6, 7, 8, 9])
    assert agree(t, one.logits()[0], k, T, seed, 0, one.position())
    one.close()
