"""Tensor-parallel decode on 2, 4 and 8 GPUs against the single-model oracle.

N ranks (one GPU each) hold the shards of a synthetic model and exchange
partial results through each other's device memory inside the step kernels
(B2_EPI_PUSH epilogues, summing prologues, logits all-gather). Teacher-forced
logits of every rank's context (all vocabulary rows) must match the oracle's
full model at the parity tolerance, and all ranks must produce the same
tokens. With all ranks in this process (peer access), and as N processes
connected by CUDA IPC handles exchanged over gloo. The reference's cluster
API (att1_cluster_infer_*, tile_count N) on .att1 files is checked against
the oracle too (reference src/cluster_infer.c:865-1163; its own test
tests/test_cluster_infer.c:27-75 checks cluster == single tile). Each test
runs for every world size the machine has GPUs for.
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
WORLDS = [pytest.param(w, marks=pytest.mark.skipif(_gpus() < w, reason=f"needs {w} GPUs")) for w in (2, 4, 8)]

# divisible by every world size: 16 query / 8 KV heads of 32, SwiGLU rows and
# vocabulary rows split evenly, 32-aligned WO / down input columns per rank
OCFG = dict(vocab=2048, n_layers=2, n_heads=16, n_kv_heads=8, d_model=512, d_ff=1024, max_seq=64,
            dtype=O.Q4, eps=1e-5, theta=10000.0)


def rel_err(a, b):
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def make_cfg(b2, ocfg):
    return b2.Config.make(ocfg.vocab, ocfg.n_layers, ocfg.n_heads, ocfg.n_kv_heads, ocfg.d_model, ocfg.d_ff,
                          ocfg.max_seq, dtype=ocfg.dtype, eps=ocfg.eps, final_eps=ocfg.final_eps, theta=ocfg.theta)


@pytest.mark.parametrize("world", WORLDS)
def test_tp_in_process_matches_oracle(b2, orc, world):
    ocfg = O.Config.make(**OCFG)
    cfg = make_cfg(b2, ocfg)
    ranks = [b2.Infer.synth_tp(cfg, 77, r, world) for r in range(world)]
    b2.Infer.tp_connect_local(ranks)
    om = orc.model(ocfg, 77, threads=8)
    toks = orc.synth_tokens(5, 24, ocfg.vocab)
    for s, t in enumerate(toks):
        for r in ranks:
            r.step_async([int(t)])
        outs = [r.step_wait() for r in ranks]
        assert all(o[0] == outs[0][0] for o in outs)
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


@pytest.mark.parametrize("world", WORLDS)
def test_tp_dense_batch_matches_oracle(b2, orc, world):
    """20 sequences per step: above the GEMVs' batch, so every projection runs
    on the tensor-core GEMM and the exchange runs as kernels of its own (push,
    rank-ordered sum, logits all-gather). Each sequence is replayed alone on
    the oracle's full model."""
    ocfg = O.Config.make(**OCFG)
    cfg = make_cfg(b2, ocfg)
    batch, steps, seed = 20, 6, 91
    ranks = [b2.Infer.synth_tp(cfg, seed, r, world, batch=batch) for r in range(world)]
    b2.Infer.tp_connect_local(ranks)
    toks = [[int(t) for t in orc.synth_tokens(seed + b, steps, ocfg.vocab)] for b in range(batch)]
    glog, gtok = [], []
    for s in range(steps):
        for r in ranks:
            r.step_async([toks[b][s] for b in range(batch)])
        outs = [r.step_wait() for r in ranks]
        assert all((o == outs[0]).all() for o in outs)
        gtok.append(outs[0])
        logs = [r.logits() for r in ranks]
        assert all((lg == logs[0]).all() for lg in logs)
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


@pytest.mark.parametrize("world", WORLDS)
def test_tp_sampler_same_tokens_on_every_rank(b2, world):
    """Top-k / temperature sampling under tensor parallelism: each rank draws
    from its all-gathered logits, so every rank returns the same tokens, and
    each token follows from the full-vocabulary logits by the restated rule."""
    from test_sampler import agree
    ocfg = O.Config.make(**OCFG)
    cfg = make_cfg(b2, ocfg)
    k, T, seed, batch = 16, 0.8, 5, 3
    ranks = [b2.Infer.synth_tp(cfg, 77, r, world, batch=batch) for r in range(world)]
    b2.Infer.tp_connect_local(ranks)
    for r in ranks:
        r.set_sampler(k, T, seed)
    toks = [1, 2, 3]
    for _ in range(5):
        for r in ranks:
            r.step_async(toks)
        outs = [r.step_wait() for r in ranks]
        assert all((o == outs[0]).all() for o in outs)
        logits, pos = ranks[0].logits(), ranks[0].position()
        for b in range(batch):
            assert agree(outs[0][b], logits[b], k, T, seed, b, pos)
        toks = [int(t) for t in outs[0]]
    for r in ranks:
        r.close()


def _nccl_rank(rank, world, port, out_dir):
    """One rank of the NCCL comparison arm: rank 0's NCCL id shared over gloo,
    every rank connects with it, then the same teacher-forced stream."""
    import sys
    sys.path.insert(0, os.path.join(ROOT, "att-1_b200"))
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import torch
    import torch.distributed as dist
    import att1_b200 as b2
    import oracle as O2

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    torch.cuda.set_device(rank)
    ocfg = O2.Config.make(**OCFG)
    inf = b2.Infer.synth_tp(make_cfg(b2, ocfg), 77, rank, world)
    ids = [b2.Infer.nccl_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(ids, src=0)
    inf.tp_connect_nccl(ids[0])
    orc = O2.Oracle()
    toks = orc.synth_tokens(5, 12, ocfg.vocab)
    logits, out = [], []
    for t in toks:
        out.append(int(inf.decode(int(t))))
        logits.append(inf.logits()[0].copy())
    np.save(os.path.join(out_dir, f"nccl_rank{rank}.npy"), {"logits": np.stack(logits), "tokens": out},
            allow_pickle=True)
    dist.barrier()
    inf.close()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", WORLDS)
def test_tp_nccl_arm_matches_oracle(orc, tmp_path, world):
    """The comparison arm: the same step with the two per-layer all-reduces
    and the logits all-gather as NCCL collectives (att1_b200_infer_tp_connect_nccl)
    gives the oracle's logits and the same tokens on every rank."""
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.spawn(_nccl_rank, args=(world, port, str(tmp_path)), nprocs=world, join=True)
    ocfg = O.Config.make(**OCFG)
    om = orc.model(ocfg, 77, threads=8)
    toks = orc.synth_tokens(5, 12, ocfg.vocab)
    res = [np.load(tmp_path / f"nccl_rank{r}.npy", allow_pickle=True).item() for r in range(world)]
    assert all(r["tokens"] == res[0]["tokens"] for r in res)
    for s, t in enumerate(toks):
        clog, _ = om.decode(int(t))
        for r in range(world):
            assert rel_err(res[r]["logits"][s], clog) <= LOGITS_RTOL


def _ipc_rank(rank, world, port, out_dir):
    import sys
    sys.path.insert(0, os.path.join(ROOT, "att-1_b200"))
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import torch.distributed as dist
    import att1_b200 as b2
    import oracle as O2

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    ocfg = O2.Config.make(**OCFG)
    inf = b2.Infer.synth_tp(make_cfg(b2, ocfg), 77, rank, world)
    handles = [None] * world
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


@pytest.mark.parametrize("world", WORLDS)
def test_tp_processes_ipc_matches_oracle(orc, tmp_path, world):
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.spawn(_ipc_rank, args=(world, port, str(tmp_path)), nprocs=world, join=True)
    ocfg = O.Config.make(**OCFG)
    om = orc.model(ocfg, 77, threads=8)
    toks = orc.synth_tokens(5, 12, ocfg.vocab)
    res = [np.load(tmp_path / f"tp_rank{r}.npy", allow_pickle=True).item() for r in range(world)]
    assert all(r["tokens"] == res[0]["tokens"] for r in res)
    for s, t in enumerate(toks):
        clog, _ = om.decode(int(t))
        for r in range(world):
            assert rel_err(res[r]["logits"][s], clog) <= LOGITS_RTOL


def _cluster_vs_oracle(b2, orc, tmp_path, dtype, world):
    """att1_cluster_infer_* with tile_count = world on a .att1 file against the
    oracle's model of the same file (eps 1e-6, theta 1e4, the reference's
    file-model settings; q8 for an f32 file) and against the single-device
    context: logits within the parity tolerance, the same tokens where the
    oracle's top two are apart, per-tile counters advanced."""
    import ctypes as C
    import att1file
    V, NL, H, D, F = 512, 2, 8, 256, 512
    path = str(tmp_path / f"m_{dtype}.att1")
    att1file.synth_model_file(path, orc, V, NL, H, D, F, 64, dtype, 21)
    ocfg = O.Config.make(vocab=V, n_layers=NL, n_heads=H, n_kv_heads=H, d_model=D, d_ff=F, max_seq=64,
                         dtype=O.Q4 if dtype == "q4" else O.Q8, eps=1e-6, theta=10000.0)
    om = orc.model(ocfg, 21, threads=8)
    L = b2.lib()
    m = b2.Model()
    assert L.att1_model_load(path.encode(), C.byref(m)) == 0
    single, cl = C.c_void_p(), C.c_void_p()
    create = L.att1_infer_create_q4 if dtype == "q4" else L.att1_infer_create
    ccreate = L.att1_cluster_infer_create_q4 if dtype == "q4" else L.att1_cluster_infer_create
    assert create(C.byref(m), C.byref(single)) == 0
    cfg = b2.ClusterConfig(world, 0, 0, 0)
    assert ccreate(C.byref(m), C.byref(cfg), C.byref(cl)) == 0
    try:
        toks = orc.synth_tokens(9, 12, V)
        for t in toks:
            a, b = C.c_uint32(), C.c_uint32()
            assert L.att1_infer_decode_token(single, int(t), C.byref(a)) == 0
            assert L.att1_cluster_infer_decode_token(cl, int(t), C.byref(b)) == 0
            n1, n2 = C.c_size_t(), C.c_size_t()
            l1 = np.ctypeslib.as_array(L.att1_infer_logits(single, C.byref(n1)), (V,)).copy()
            l2 = np.ctypeslib.as_array(L.att1_cluster_infer_logits(cl, C.byref(n2)), (V,)).copy()
            assert n1.value == n2.value == V
            want, _ = om.decode(int(t))
            assert rel_err(l2, want) <= LOGITS_RTOL
            assert rel_err(l1, want) <= LOGITS_RTOL
            top2 = np.sort(want)[-2:]
            if (top2[1] - top2[0]) / np.abs(want).max() > 2 * LOGITS_RTOL:
                assert a.value == b.value == int(np.argmax(want))
        pos = C.c_size_t()
        assert L.att1_cluster_infer_position(cl, C.byref(pos)) == 0 and pos.value == 12
        for tile in range(world):
            k = b2.TileCounters()
            assert L.att1_cluster_infer_get_tile_counters(cl, tile, C.byref(k)) == 0
            assert k.layers_run == 12 * NL and k.activations_sent == 12 * NL * 2
            assert (k.layer_start, k.layer_end) == (0, NL)
    finally:
        L.att1_cluster_infer_destroy(cl)
        L.att1_infer_destroy(single)
        L.att1_model_free(C.byref(m))


@pytest.mark.parametrize("world", WORLDS)
def test_cluster_tiles_q4_file(b2, orc, tmp_path, world):
    _cluster_vs_oracle(b2, orc, tmp_path, "q4", world)


@pytest.mark.parametrize("world", WORLDS)
def test_cluster_tiles_f32_file_q8(b2, orc, tmp_path, world):
    """f32 file through att1_cluster_infer_create: q8 weights quantised per
    whole output row before the row-parallel split."""
    _cluster_vs_oracle(b2, orc, tmp_path, "f32", world)


@need2
def test_tp_wait_runs_out_and_ranks_recover(b2, orc):
    """A rank that never takes its step: the other rank's bounded waits for
    its exchange flags run out (a flag nothing sets), the step ends with
    ATT1_ERR_TIMEOUT instead of a hang or a fault, the position stays where it
    was, and after att1_b200_infer_tp_reset on both ranks the next joint steps
    (repeating the failed one) match the oracle."""
    ocfg = O.Config.make(**OCFG)
    cfg = make_cfg(b2, ocfg)
    ranks = [b2.Infer.synth_tp(cfg, 77, r, 2) for r in range(2)]
    b2.Infer.tp_connect_local(ranks)
    om = orc.model(ocfg, 77, threads=8)
    toks = [int(t) for t in orc.synth_tokens(5, 4, ocfg.vocab)]
    try:
        for r in ranks:
            r.step_async([toks[0]])
        for r in ranks:
            r.step_wait()
        om.decode(toks[0])
        for r in ranks:
            r.tp_set_wait(1 << 12)                     # about half a millisecond per wait
        ranks[0].step_async([toks[1]])                 # rank 1 does not take this step
        with pytest.raises(b2.Att1Error) as e:
            ranks[0].step_wait()
        assert e.value.rc == -11                       # ATT1_ERR_TIMEOUT
        assert ranks[0].position() == 1 and ranks[1].position() == 1
        for r in ranks:
            r.tp_reset()
            r.tp_set_wait(0)
        for t in toks[1:]:
            for r in ranks:
                r.step_async([t])
            outs = [r.step_wait() for r in ranks]
            assert outs[0][0] == outs[1][0]
            clog, _ = om.decode(t)
            for r in ranks:
                assert rel_err(r.logits()[0], clog) <= LOGITS_RTOL
    finally:
        for r in ranks:
            r.close()
