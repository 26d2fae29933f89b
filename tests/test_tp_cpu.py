"""Tensor-parallel split of the decode path, checked on CPU with two gloo ranks.

The device ranks (att1_b200_infer_create_synth_tp) hold, per rank r of N:
query/KV head rows r*H/N.. of wq/wk/wv, FFN rows r*F/N.. of gate and up,
input columns r*H*hd/N.. of wo and r*F/N.. of down (partial outputs summed
over ranks), vocabulary rows r*V/N.. of the lm_head (all-gathered). This test
runs that split with the oracle's q4 arithmetic on two processes and checks:
  * quantising a 32-aligned column slice gives the same bytes as slicing the
    quantised matrix (so per-rank synthesis equals sharding the full model);
  * row-parallel products summed over ranks match the full product;
  * row splits and the vocabulary all-gather reproduce the full outputs
    bit for bit, and the greedy token is the same;
  * rank-ordered exchange of opaque handles (what bench.py does with the
    CUDA IPC handles).
"""
import os
import socket

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
WORLD = 2
D, F, H, HKV, HD, V = 128, 256, 4, 2, 32, 512


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, port, out_dir):
    import sys
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import torch
    import torch.distributed as dist
    import oracle as O

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    orc = O.Oracle()
    res = {}
    x = orc.synth_normal(7, 1, D, std=1.0).reshape(1, D)

    def full(tid, rows, cols):
        return orc.synth_normal(3, tid, rows * cols).reshape(rows, cols)

    # row-parallel wo: input columns of this rank, partial outputs summed
    qr = H * HD // WORLD
    wo = full(4, D, H * HD)
    p_full, s_full = orc.q4_quantize(wo)
    p_r, s_r = orc.q4_quantize(wo[:, rank * qr:(rank + 1) * qr])
    pf = p_full.reshape(D, H * HD // 2)[:, rank * qr // 2:(rank + 1) * qr // 2]
    sf = s_full.reshape(D, H * HD // 32)[:, rank * qr // 32:(rank + 1) * qr // 32]
    res["slice_bytes_equal"] = bool((p_r.reshape(D, -1) == pf).all() and (s_r.reshape(D, -1) == sf).all())
    ctx = orc.synth_normal(8, 1, H * HD, std=1.0).reshape(1, H * HD)
    part = orc.matmul_q4(ctx[:, rank * qr:(rank + 1) * qr], p_r, s_r, D, qr)
    t = torch.from_numpy(part.copy())
    dist.all_reduce(t)
    want = orc.matmul_q4(ctx, p_full, s_full, D, H * HD)
    res["wo_rel"] = float(np.abs(t.numpy() - want).max() / np.abs(want).max())

    # column-parallel gate rows and the vocabulary split: all-gather
    fl = F // WORLD
    gate = full(6, F, D)
    pg, sg = orc.q4_quantize(gate[rank * fl:(rank + 1) * fl])
    loc = torch.from_numpy(orc.matmul_q4(x, pg, sg, fl, D).copy())
    parts = [torch.zeros_like(loc) for _ in range(WORLD)]
    dist.all_gather(parts, loc)
    pgf, sgf = orc.q4_quantize(gate)
    res["gate_equal"] = bool((torch.cat(parts, 1).numpy() == orc.matmul_q4(x, pgf, sgf, F, D)).all())

    vl = V // WORLD
    out = full(9, V, D)
    po, so = orc.q4_quantize(out[rank * vl:(rank + 1) * vl])
    lg = torch.from_numpy(orc.matmul_q4(x, po, so, vl, D).copy())
    parts = [torch.zeros_like(lg) for _ in range(WORLD)]
    dist.all_gather(parts, lg)
    full_lg = orc.matmul_q4(x, *orc.q4_quantize(out), V, D)
    res["logits_equal"] = bool((torch.cat(parts, 1).numpy() == full_lg).all())
    # greedy over ranks: each rank's best (value, lowest global id), then the best of those
    loc_best = int(np.argmax(lg.numpy()[0])) + rank * vl
    bests = [None] * WORLD
    dist.all_gather_object(bests, (float(lg.numpy()[0].max()), -loc_best))
    res["token"] = -max(bests)[1]
    res["token_full"] = int(np.argmax(full_lg[0]))

    # rank-ordered opaque handles
    handles = [None] * WORLD
    dist.all_gather_object(handles, bytes([rank]) * 64)
    res["handles_ordered"] = handles == [bytes([r]) * 64 for r in range(WORLD)]
    np.save(os.path.join(out_dir, f"rank{rank}.npy"), res, allow_pickle=True)
    dist.destroy_process_group()


def test_tensor_parallel_split_two_gloo_ranks(tmp_path):
    import torch.multiprocessing as mp
    mp.spawn(_rank_main, args=(_free_port(), str(tmp_path)), nprocs=WORLD, join=True)
    for r in range(WORLD):
        res = np.load(tmp_path / f"rank{r}.npy", allow_pickle=True).item()
        assert res["slice_bytes_equal"]
        assert res["wo_rel"] <= 1e-5
        assert res["gate_equal"]
        assert res["logits_equal"]
        assert res["token"] == res["token_full"]
        assert res["handles_ordered"]
