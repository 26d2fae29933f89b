"""Decode parity at the benchmarked shapes, deep in the context.

The bench decodes the Llama-3-8B shape (dim 4096, 32 layers, 32/8 heads of
128, SwiGLU 14336, vocabulary 128256, theta 5e5) at context ~4096, where every
one of the attention's position splits is live, and the small GQA decoder
(dim 576, 30 layers, 9/3 heads of 64, vocabulary 49152) to context 2048 with 1
and 16 sequences. Decoding thousands of prefix tokens on the CPU oracle is too
slow for a test, so both sides start from the same K/V: seeded random rows
written into the oracle's cache (or_state_import_kv) and into the device pages
(att1_b200_infer_import_kv), then both continue at the same position
(or_state_seek / att1_b200_infer_seek) and decode teacher-forced. Every step's
logits must satisfy max|gpu - cpu| / max|cpu| <= 1e-3 over the whole
vocabulary, and greedy tokens must agree wherever the oracle's top two logits
are further apart than that (src/infer.c:656-880, src/attention.c:511-541).

The imported keys have a standard deviation of 1.5 and the values of 1.0, so
the attention scores spread over several units and the attention output
outweighs the embedding in the residual stream: an error in the attention over
thousands of positions shows in the logits.
"""
import os

import numpy as np
import pytest

import oracle as O
from test_gpu_decode import LOGITS_RTOL, rel_err, tokens_agree

pytestmark = pytest.mark.gpu
THREADS = max(1, min(32, os.cpu_count() or 1))


def b2_config(b2, ocfg):
    return b2.Config.make(ocfg.vocab, ocfg.n_layers, ocfg.n_heads, ocfg.n_kv_heads, ocfg.d_model, ocfg.d_ff,
                          ocfg.max_seq, dtype=ocfg.dtype, eps=ocfg.eps, final_eps=ocfg.final_eps,
                          theta=ocfg.theta)


def random_kv(rng, count, hkv, hd):
    k = rng.standard_normal((count, hkv, hd), dtype=np.float32) * np.float32(1.5)
    v = rng.standard_normal((count, hkv, hd), dtype=np.float32)
    return k, v


def fill_deep(b2, inf, oms, ocfg, count, seed):
    """The same random K/V rows [0, count) of every layer in the device context
    (item b) and in oracle state b; both then continue at position `count`."""
    hd = ocfg.d_model // ocfg.n_heads
    row = ocfg.n_kv_heads * hd
    rng = np.random.default_rng(seed)
    for b, om in enumerate(oms):
        for layer in range(ocfg.n_layers):
            k, v = random_kv(rng, count, ocfg.n_kv_heads, hd)
            om.import_kv(layer, k, v)
            inf.import_kv(b, layer, k, v, row)
        om.seek(count)
    inf.seek(count)


def decode_compare(inf, oms, tokens):
    """Teacher-forced steps; tokens [steps][batch]. Returns the worst error."""
    worst = 0.0
    batch = len(oms)
    for s, step_toks in enumerate(tokens):
        gtok = inf.decode_batch(list(step_toks)) if batch > 1 else [inf.decode(int(step_toks[0]))]
        glog = inf.logits()
        for b in range(batch):
            clog, _ = oms[b].decode(int(step_toks[b]))
            e = rel_err(glog[b], clog)
            worst = max(worst, e)
            assert e <= LOGITS_RTOL, f"step {s} item {b}: rel err {e:.3e}"
            assert tokens_agree(gtok[b], clog), f"step {s} item {b}: token {gtok[b]} vs {int(np.argmax(clog))}"
    return worst


def test_8b_full_vocab_deep_context(b2, orc):
    """8B widths at 2 layers with the full 128256-row lm_head: positions
    4090..4095 (the last positions of a 4096 context, all attention splits
    live), then positions 2100..2102 of the same cache."""
    ocfg = O.Config.make(vocab=128256, n_layers=2, n_heads=32, n_kv_heads=8, d_model=4096, d_ff=14336,
                         max_seq=4096, dtype=O.Q4, eps=1e-5, theta=500000.0)
    inf = b2.Infer.synth(b2_config(b2, ocfg), 4242)
    om = orc.model(ocfg, 4242, threads=THREADS)
    try:
        fill_deep(b2, inf, [om], ocfg, 4090, seed=1)
        toks = orc.synth_tokens(99, 9, ocfg.vocab)
        decode_compare(inf, [om], [[t] for t in toks[:6]])
        assert inf.position() == 4096
        # back to the middle of the same cache: positions [0, 2100) still hold the imported rows
        inf.seek(2100)
        om.seek(2100)
        decode_compare(inf, [om], [[t] for t in toks[6:]])
    finally:
        inf.close()
        om.close()


def test_8b_full_depth_deep_context(b2, orc):
    """The whole benchmarked model: 32 layers, vocabulary 128256, two tokens at
    positions 4000 and 4001 of a 4096 context."""
    ocfg = O.Config.make(vocab=128256, n_layers=32, n_heads=32, n_kv_heads=8, d_model=4096, d_ff=14336,
                         max_seq=4096, dtype=O.Q4, eps=1e-5, theta=500000.0)
    inf = b2.Infer.synth(b2_config(b2, ocfg), 808)
    om = orc.model(ocfg, 808, threads=THREADS)
    try:
        fill_deep(b2, inf, [om], ocfg, 4000, seed=2)
        toks = orc.synth_tokens(7, 2, ocfg.vocab)
        decode_compare(inf, [om], [[t] for t in toks])
    finally:
        inf.close()
        om.close()


@pytest.mark.parametrize("batch", [1, 16])
def test_small_gqa_to_context_2048(b2, orc, batch):
    """The small GQA decoder (30 layers, 9 query / 3 KV heads of 64, vocabulary
    49152, theta 1e4) decoding positions 2040..2047, the end of its 2048
    context, with 1 and with 16 sequences (each its own K/V and tokens)."""
    ocfg = O.Config.make(vocab=49152, n_layers=30, n_heads=9, n_kv_heads=3, d_model=576, d_ff=1536,
                         max_seq=2048, dtype=O.Q4, eps=1e-5, theta=10000.0)
    inf = b2.Infer.synth(b2_config(b2, ocfg), 5150, batch=batch)
    base = orc.model(ocfg, 5150, threads=THREADS)
    oms = [base] + [base.spawn() for _ in range(batch - 1)]
    try:
        fill_deep(b2, inf, oms, ocfg, 2040, seed=3 + batch)
        toks = np.stack([orc.synth_tokens(600 + b, 8, ocfg.vocab) for b in range(batch)], axis=1)
        decode_compare(inf, oms, toks)
        assert inf.position() == 2048
    finally:
        inf.close()
        for om in oms[1:]:
            om.close()
        base.close()


def test_import_kv_round_trip_and_limits(b2):
    """import_kv writes exactly what export_kv reads back (pages of 64 tokens,
    a partial last page), and both reject out-of-range arguments."""
    cfg = b2.Config.make(1000, 2, 8, 2, 256, 256, 200, dtype=4)
    inf = b2.Infer.synth(cfg, 1, batch=2)
    try:
        row = 2 * 32
        rng = np.random.default_rng(5)
        k, v = random_kv(rng, 150, 2, 32)
        inf.import_kv(1, 1, k, v, row)
        gk, gv = inf.export_kv(1, 1, 150, row)
        assert (gk == k.reshape(-1)).all() and (gv == v.reshape(-1)).all()
        z, _ = inf.export_kv(0, 1, 150, row)
        assert (z == 0).all()                                   # item 0 untouched
        with pytest.raises(b2.Att1Error):
            inf.import_kv(2, 0, k, v, row)                       # item out of range
        with pytest.raises(b2.Att1Error):
            inf.import_kv(0, 2, k, v, row)                       # layer out of range
        with pytest.raises(b2.Att1Error):
            inf.seek(200)                                        # position == max_seq
        inf.seek(150)
        assert inf.position() == 150
    finally:
        inf.close()


@pytest.mark.parametrize("H", [32, 64])
def test_attention_8b_heads_context_4096(b2, H):
    """b2_attn alone at the 8B attention shape (32 query heads on 8 KV heads of
    128) and the 70B one (64 on 8: eight query heads per KV head), two
    sequences at positions 4095 and 2047 of a 4096-position capacity (so the
    grid has all its position splits), pages of 64 tokens in a shuffled order,
    against a float64 attention: max error <= 1e-5 of the largest output."""
    import ctypes as C

    import torch
    L = b2.lib()
    Hkv, hd, T, cap, B = 8, 128, 64, 4096, 2
    pps = cap // T
    rng = np.random.default_rng(17)
    pages = rng.permutation(B * pps).astype(np.int32)
    Kp = np.zeros((B * pps, Hkv, T, hd), np.float32)
    Vp = np.zeros_like(Kp)
    K = rng.standard_normal((B, cap, Hkv, hd), dtype=np.float32) * np.float32(1.5)
    V = rng.standard_normal((B, cap, Hkv, hd), dtype=np.float32)
    for b in range(B):
        for p in range(pps):
            Kp[pages[b * pps + p]] = K[b, p * T:(p + 1) * T].transpose(1, 0, 2)
            Vp[pages[b * pps + p]] = V[b, p * T:(p + 1) * T].transpose(1, 0, 2)
    q = rng.standard_normal((B, H, hd), dtype=np.float32)
    positions = np.array([4095, 2047], np.int32)
    kd, vd = torch.from_numpy(Kp.reshape(-1)).cuda(), torch.from_numpy(Vp.reshape(-1)).cuda()
    pt = torch.from_numpy(pages).cuda()
    qd = torch.from_numpy(q.reshape(-1)).cuda()
    pos = torch.from_numpy(positions).cuda()
    ctx = torch.zeros(B * H * hd, dtype=torch.float32, device="cuda")
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    lay = b2.KVLayout()
    lay.k_pool, lay.v_pool, lay.page_table = kd.data_ptr(), vd.data_ptr(), pt.data_ptr()
    lay.page_tokens, lay.pages_per_seq, lay.n_kv_heads, lay.head_dim = T, pps, Hkv, hd
    a = b2.AttnArgs()
    a.batch, a.n_heads, a.n_kv_heads, a.head_dim = B, H, Hkv, hd
    a.q, a.kv, a.positions, a.max_ctx, a.ctx, a.err = qd.data_ptr(), lay, pos.data_ptr(), cap, ctx.data_ptr(), \
        err.data_ptr()
    sb = L.b2_attn_scratch_bytes(C.byref(a))
    scratch = torch.zeros(max(sb, 256), dtype=torch.uint8, device="cuda")
    cnt = torch.zeros(max(L.b2_attn_counters_len(C.byref(a)), 1), dtype=torch.int32, device="cuda")
    a.scratch, a.scratch_bytes, a.counters, a.counters_len = scratch.data_ptr(), sb, cnt.data_ptr(), cnt.numel()
    for _ in range(2):                                          # the counters are left zero for the next call
        ctx.zero_()
        assert L.b2_attn(C.byref(a), None) == 0
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        got = ctx.cpu().numpy().reshape(B, H, hd)
        for b in range(B):
            n = int(positions[b]) + 1
            want = np.zeros((H, hd))
            for h in range(H):
                kv = h // (H // Hkv)
                s = K[b, :n, kv].astype(np.float64) @ q[b, h].astype(np.float64) / np.sqrt(hd)
                p = np.exp(s - s.max())
                want[h] = (p / p.sum()) @ V[b, :n, kv].astype(np.float64)
            e = np.abs(got[b] - want).max() / np.abs(want).max()
            assert e <= 1e-5, f"item {b}: rel err {e:.3e}"
        assert (cnt.cpu().numpy() == 0).all()


def test_kv_rows_land_in_their_pages(b2):
    """The K/V row a step appends lands in its own page at the full model size.
    Creating the 8B shape queues gigabytes of zero fills on the context's
    stream; the page table and RoPE frequencies are written after them on the
    same stream, so no fill can land on the table afterwards (with the table
    zeroed every position would map to page 0: the row at position 130 would
    land in page 0 at row 2 and position 130's own slot would stay zero)."""
    cfg = b2.Config.make(128256, 32, 32, 8, 4096, 14336, 4096, dtype=4, eps=1e-5, theta=500000.0)
    inf = b2.Infer.synth(cfg, 77)
    try:
        inf.seek(130)
        inf.decode(5)
        row = 8 * 128
        for layer in (0, 31):
            k, v = inf.export_kv(0, layer, 131, row)
            assert np.abs(k[130 * row:]).max() > 0 and np.abs(v[130 * row:]).max() > 0, layer
            assert not k[:130 * row].any() and not v[:130 * row].any(), layer
    finally:
        inf.close()
