"""Tensor-parallel decode on two GPUs against the single-model oracle.

Two ranks (one GPU each) hold the shards of a synthetic model and exchange
partial results through each other's device memory inside the step kernels
(B2_EPI_PUSH epilogues, summing prologues, logits all-gather). Teacher-forced
logits of the rank-0 context (all vocabulary rows) must match the oracle's
full model at the parity tolerance, and both ranks must produce the same
tokens. Once with both ranks in this process (peer access), once as two
processes connected by CUDA IPC handles exchanged over gloo.
"""
import os
import socket

import numpy as np
import pytest

import oracle as O

pytestmark = pytest.mark.gpu
LOGITS_RTOL = 1e-3
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _gpus():
    try:
        import torch
        return torch.cuda.device_count()
    except Exception:
        return 0


need2 = pytest.mark.skipif(_gpus() < 2, reason="needs two GPUs")

OCFG = dict(vocab=2048, n_layers=2, n_heads=8, n_kv_heads=2, d_model=256, d_ff=512, max_seq=64,
            dtype=O.Q4, eps=1e-5, theta=10000.0)


def rel_err(a, b):
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def make_cfg(b2, ocfg):
    return b2.Config.make(ocfg.vocab, ocfg.n_layers, ocfg.n_heads, ocfg.n_kv_heads, ocfg.d_model, ocfg.d_ff,
                          ocfg.max_seq, dtype=ocfg.dtype, eps=ocfg.eps, final_eps=ocfg.final_eps, theta=ocfg.theta)


@need2
def test_tp2_in_process_matches_oracle(b2, orc):
    ocfg = O.Config.make(**OCFG)
    cfg = make_cfg(b2, ocfg)
    ranks = [b2.Infer.synth_tp(cfg, 77, r, 2) for r in range(2)]
    b2.Infer.tp_connect_local(ranks)
    om = orc.model(ocfg, 77, threads=8)
    toks = orc.synth_tokens(5, 24, ocfg.vocab)
    for s, t in enumerate(toks):
        for r in ranks:
            r.step_async([int(t)])
        outs = [r.step_wait() for r in ranks]
        assert outs[0][0] == outs[1][0]
        clog, ctok = om.decode(int(t))
        for r in ranks:
            e = rel_err(r.logits()[0], clog)
            assert e <= LOGITS_RTOL, f"step {s}: rel err {e:.3e}"
    # both ranks keep going on the device loop
    for r in ranks:
        r.run_steps(4)
    for r in ranks:
        r.sync()
    for r in ranks:
        r.close()


@need2
def test_tp2_dense_batch_matches_oracle(b2, orc):
    """20 sequences per step: above the GEMVs' batch, so every projection runs
    on the tensor-core GEMM and the exchange runs as kernels of its own (push,
    rank-ordered sum, logits all-gather). Each sequence is replayed alone on
    the oracle's full model."""
    ocfg = O.Config.make(**OCFG)
    cfg = make_cfg(b2, ocfg)
    batch, steps, seed = 20, 6, 91
    ranks = [b2.Infer.synth_tp(cfg, seed, r, 2, batch=batch) for r in range(2)]
    b2.Infer.tp_connect_local(ranks)
    toks = [[int(t) for t in orc.synth_tokens(seed + b, steps, ocfg.vocab)] for b in range(batch)]
    glog, gtok = [], []
    for s in range(steps):
        for r in ranks:
            r.step_async([toks[b][s] for b in range(batch)])
        outs = [r.step_wait() for r in ranks]
        assert (outs[0] == outs[1]).all()
        gtok.append(outs[0])
        logs = [r.logits() for r in ranks]
        assert (logs[0] == logs[1]).all()
        glog.append(logs[0])
    for r in ranks:
        r.close()
    om = orc.model(ocfg, seed, threads=8)
    for b in range(batch):
        om.reset()
        for s in range(steps):
            clog, _ = om.decode(toks[b][s])
            e = rel_err(glog[s][b], clog)
            assert e <= LOGITS_RTOL, f"step {s} item {b}: rel err {e:.3e}"
            top2 = np.sort(clog)[-2:]
            gap = (top2[1] - top2[0]) / max(np.abs(clog).max(), 1e-30)
            assert gap <= 2 * LOGITS_RTOL or int(gtok[s][b]) == int(np.argmax(clog))


@need2
def test_tp2_sampler_same_tokens_on_both_ranks(b2):
    """Top-k / temperature sampling under tensor parallelism: each rank draws
    from its all-gathered logits, so both ranks return the same tokens, and
    each token follows from the full-vocabulary logits by the restated rule."""
    from test_sampler import agree
    ocfg = O.Config.make(**OCFG)
    cfg = make_cfg(b2, ocfg)
    k, T, seed, batch = 16, 0.8, 5, 3
    ranks = [b2.Infer.synth_tp(cfg, 77, r, 2, batch=batch) for r in range(2)]
    b2.Infer.tp_connect_local(ranks)
    for r in ranks:
        r.set_sampler(k, T, seed)
    toks = [1, 2, 3]
    for _ in range(5):
        for r in ranks:
            r.step_async(toks)
        outs = [r.step_wait() for r in ranks]
        assert (outs[0] == outs[1]).all()
        logits, pos = ranks[0].logits(), ranks[0].position()
        for b in range(batch):
            assert agree(outs[0][b], logits[b], k, T, seed, b, pos)
        toks = [int(t) for t in outs[0]]
    for r in ranks:
        r.close()


def _ipc_rank(rank, port, out_dir):
    import sys
    sys.path.insert(0, os.path.join(ROOT, "att-1_b200"))
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import torch.distributed as dist
    import att1_b200 as b2
    import oracle as O2

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=2)
    ocfg = O2.Config.make(**OCFG)
    inf = b2.Infer.synth_tp(make_cfg(b2, ocfg), 77, rank, 2)
    handles = [None, None]
    dist.all_gather_object(handles, inf.tp_handle())
    inf.tp_connect(handles)
    orc = O2.Oracle()
    toks = orc.synth_tokens(5, 12, ocfg.vocab)
    logits, out = [], []
    for t in toks:
        out.append(int(inf.decode(int(t))))
        logits.append(inf.logits()[0].copy())
    np.save(os.path.join(out_dir, f"tp_rank{rank}.npy"), {"logits": np.stack(logits), "tokens": out},
            allow_pickle=True)
    inf.tp_disconnect()
    dist.barrier()
    inf.close()
    dist.destroy_process_group()


@need2
def test_tp2_two_processes_ipc_matches_oracle(orc, tmp_path):
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.spawn(_ipc_rank, args=(port, str(tmp_path)), nprocs=2, join=True)
    ocfg = O.Config.make(**OCFG)
    om = orc.model(ocfg, 77, threads=8)
    toks = orc.synth_tokens(5, 12, ocfg.vocab)
    res = [np.load(tmp_path / f"tp_rank{r}.npy", allow_pickle=True).item() for r in range(2)]
    assert res[0]["tokens"] == res[1]["tokens"]
    for s, t in enumerate(toks):
        clog, _ = om.decode(int(t))
        for r in range(2):
            assert rel_err(res[r]["logits"][s], clog) <= LOGITS_RTOL


def _cluster_vs_single(b2, orc, tmp_path, dtype):
    """att1_cluster_infer_* with tile_count 2 on a .att1 file against the
    single-device context of the same file: same tokens, logits within the
    parity tolerance, per-tile counters advanced."""
    import ctypes as C
    import att1file
    path = str(tmp_path / f"m_{dtype}.att1")
    att1file.synth_model_file(path, orc, 512, 2, 4, 128, 256, 64, dtype, 21)
    L = b2.lib()
    m = b2.Model()
    assert L.att1_model_load(path.encode(), C.byref(m)) == 0
    single, cl = C.c_void_p(), C.c_void_p()
    create = L.att1_infer_create_q4 if dtype == "q4" else L.att1_infer_create
    ccreate = L.att1_cluster_infer_create_q4 if dtype == "q4" else L.att1_cluster_infer_create
    assert create(C.byref(m), C.byref(single)) == 0
    cfg = b2.ClusterConfig(2, 0, 0, 0)
    assert ccreate(C.byref(m), C.byref(cfg), C.byref(cl)) == 0
    try:
        toks = orc.synth_tokens(9, 12, 512)
        for t in toks:
            a, b = C.c_uint32(), C.c_uint32()
            assert L.att1_infer_decode_token(single, int(t), C.byref(a)) == 0
            assert L.att1_cluster_infer_decode_token(cl, int(t), C.byref(b)) == 0
            n1, n2 = C.c_size_t(), C.c_size_t()
            l1 = np.ctypeslib.as_array(L.att1_infer_logits(single, C.byref(n1)), (512,)).copy()
            l2 = np.ctypeslib.as_array(L.att1_cluster_infer_logits(cl, C.byref(n2)), (512,)).copy()
            assert n1.value == n2.value == 512
            assert rel_err(l2, l1) <= LOGITS_RTOL
            top2 = np.sort(l1)[-2:]
            if (top2[1] - top2[0]) / np.abs(l1).max() > 2 * LOGITS_RTOL:
                assert a.value == b.value
        pos = C.c_size_t()
        assert L.att1_cluster_infer_position(cl, C.byref(pos)) == 0 and pos.value == 12
        for tile in range(2):
            k = b2.TileCounters()
            assert L.att1_cluster_infer_get_tile_counters(cl, tile, C.byref(k)) == 0
            assert k.layers_run == 12 * 2 and k.activations_sent == 12 * 2 * 2
            assert (k.layer_start, k.layer_end) == (0, 2)
    finally:
        L.att1_cluster_infer_destroy(cl)
        L.att1_infer_destroy(single)
        L.att1_model_free(C.byref(m))


@need2
def test_cluster_two_tiles_q4_file(b2, orc, tmp_path):
    _cluster_vs_single(b2, orc, tmp_path, "q4")


@need2
def test_cluster_two_tiles_f32_file_q8(b2, orc, tmp_path):
    """f32 file through att1_cluster_infer_create: q8 weights quantised per
    whole output row before the row-parallel split."""
    _cluster_vs_single(b2, orc, tmp_path, "f32")
