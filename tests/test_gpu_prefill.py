"""Prompt prefill and large decode batches through the tensor-core GEMM.

att1_b200_infer_prefill computes a whole prompt (up to 512 tokens per pass
over the weights) with b2_gemm; the reference feeds the prompt through the
decode step token by token (src/infer.c:905-912). Teacher-forced parity: the
logits after the last prompt token, and of every decode step after it, must
match the oracle's token-by-token decode within max|gpu - cpu| / max|cpu| <=
1e-3. Decode batches larger than the fused GEMVs hold (32 sequences at 8B
widths) take the same GEMM route and are checked the same way per sequence.
"""
import numpy as np
import pytest

import oracle as O
from test_gpu_decode import LOGITS_RTOL, rel_err, tokens_agree

pytestmark = pytest.mark.gpu


def make(b2, ocfg):
    return b2.Config.make(ocfg.vocab, ocfg.n_layers, ocfg.n_heads, ocfg.n_kv_heads, ocfg.d_model, ocfg.d_ff,
                          ocfg.max_seq, dtype=ocfg.dtype, eps=ocfg.eps, final_eps=ocfg.final_eps, theta=ocfg.theta)


def prefill_parity(b2, orc, ocfg, prompt_len, decode_steps, seed=1234, before=0, threads=8):
    inf = b2.Infer.synth(make(b2, ocfg), seed)
    om = orc.model(ocfg, seed, threads=threads)
    toks = [int(t) for t in orc.synth_tokens(seed, before + prompt_len + decode_steps, ocfg.vocab)]
    worst = 0.0
    for t in toks[:before]:
        inf.decode(t)
        om.decode(t)
    nxt = inf.prefill(toks[before:before + prompt_len])
    for t in toks[before:before + prompt_len]:
        clog, _ = om.decode(t)
    e = rel_err(inf.logits()[0], clog)
    assert e <= LOGITS_RTOL, f"after prefill: rel err {e:.3e}"
    assert tokens_agree(nxt, clog)
    worst = max(worst, e)
    for s, t in enumerate(toks[before + prompt_len:]):
        g = inf.decode(t)
        clog, _ = om.decode(t)
        e = rel_err(inf.logits()[0], clog)
        assert e <= LOGITS_RTOL, f"decode step {s} after prefill: rel err {e:.3e}"
        assert tokens_agree(g, clog)
        worst = max(worst, e)
    inf.close()
    return worst


def test_prefill_small_gqa(b2, orc):
    ocfg = O.Config.make(vocab=49152, n_layers=30, n_heads=9, n_kv_heads=3, d_model=576, d_ff=1536,
                         max_seq=2048, dtype=O.Q4, eps=1e-5, theta=10000.0)
    assert prefill_parity(b2, orc, ocfg, prompt_len=64, decode_steps=4) <= LOGITS_RTOL


def test_prefill_8b_widths(b2, orc):
    """Llama-3-8B widths at 2 layers, 4096-entry vocabulary, a 100-token prompt."""
    ocfg = O.Config.make(vocab=4096, n_layers=2, n_heads=32, n_kv_heads=8, d_model=4096, d_ff=14336,
                         max_seq=256, dtype=O.Q4, eps=1e-5, theta=500000.0)
    assert prefill_parity(b2, orc, ocfg, prompt_len=100, decode_steps=3) <= LOGITS_RTOL


def test_prefill_two_chunks_q8(b2, orc):
    """A 600-token prompt: two passes (512 + 88 tokens), the second attending
    to the KV pages the first wrote; q8 weights."""
    ocfg = O.Config.make(vocab=32000, n_layers=6, n_heads=6, n_kv_heads=6, d_model=288, d_ff=768,
                         max_seq=1024, dtype=O.Q8, eps=1e-5, theta=10000.0)
    assert prefill_parity(b2, orc, ocfg, prompt_len=600, decode_steps=4) <= LOGITS_RTOL


def test_prefill_after_decode_steps(b2, orc):
    ocfg = O.Config.make(vocab=1000, n_layers=2, n_heads=4, n_kv_heads=2, d_model=128, d_ff=256,
                         max_seq=128, dtype=O.Q4, eps=1e-5, theta=10000.0)
    assert prefill_parity(b2, orc, ocfg, prompt_len=40, decode_steps=5, before=7) <= LOGITS_RTOL


def test_prefill_rejects_bad_input(b2):
    cfg = b2.Config.make(1000, 1, 4, 2, 128, 256, 32, dtype=4)
    inf = b2.Infer.synth(cfg, 3)
    with pytest.raises(b2.Att1Error):
        inf.prefill([1, 2, 1000])        # token id outside the vocabulary
    with pytest.raises(b2.Att1Error):
        inf.prefill(list(range(33)))     # beyond max_seq
    assert inf.prefill([5, 6, 7]) >= 0   # the context is still usable
    inf.close()


def test_generate_uses_prefill_same_tokens(b2):
    """att1_infer_generate (prompt through prefill) gives the tokens of the
    token-by-token decode loop."""
    cfg = b2.Config.make(256, 2, 4, 2, 128, 256, 64, dtype=4)
    prompt = bytes(range(30, 60))
    a = b2.Infer.synth(cfg, 9)
    got = a.generate(prompt, 6)
    a.close()
    b = b2.Infer.synth(cfg, 9)
    tok = 0
    for ch in prompt:
        tok = b.decode(ch)
    want = [tok]
    for _ in range(5):
        want.append(b.decode(want[-1]))
    b.close()
    assert list(got) == want


def batch_parity_replay(b2, orc, ocfg, steps, batch, seed=1234, threads=16):
    """All sequences decode together on the GPU; one oracle model then replays
    each sequence alone (reset between sequences) against the stored logits."""
    inf = b2.Infer.synth(make(b2, ocfg), seed, batch=batch)
    toks = [[int(t) for t in orc.synth_tokens(seed + b, steps, ocfg.vocab)] for b in range(batch)]
    glog, gtok = [], []
    for s in range(steps):
        gtok.append(inf.decode_batch([toks[b][s] for b in range(batch)]))
        glog.append(inf.logits())
    inf.close()
    om = orc.model(ocfg, seed, threads=threads)
    worst = 0.0
    for b in range(batch):
        om.reset()
        for s in range(steps):
            clog, _ = om.decode(toks[b][s])
            e = rel_err(glog[s][b], clog)
            assert e <= LOGITS_RTOL, f"step {s} item {b}: rel err {e:.3e}"
            assert tokens_agree(gtok[s][b], clog)
            worst = max(worst, e)
    return worst


def test_decode_batch32_8b_widths(b2, orc):
    """32 sequences at Llama-3-8B widths (2 layers): the GEMVs cannot hold the
    batch, so every projection goes through the tensor-core GEMM."""
    ocfg = O.Config.make(vocab=4096, n_layers=2, n_heads=32, n_kv_heads=8, d_model=4096, d_ff=14336,
                         max_seq=64, dtype=O.Q4, eps=1e-5, theta=500000.0)
    assert batch_parity_replay(b2, orc, ocfg, steps=3, batch=32) <= LOGITS_RTOL


def test_decode_batch20_small(b2, orc):
    ocfg = O.Config.make(vocab=1000, n_layers=2, n_heads=4, n_kv_heads=2, d_model=128, d_ff=256,
                         max_seq=64, dtype=O.Q8, eps=1e-5, theta=10000.0)
    assert batch_parity_replay(b2, orc, ocfg, steps=8, batch=20) <= LOGITS_RTOL
