"""b2_attn_noalloc: the attention entry point for callers that cannot allocate
device memory where they run it (code inside a memory pool or arena it does
not own, code that must not synchronise the device with cudaMalloc/cudaFree,
hosts whose allocator is closed to plugins). It takes the split partials and
counters from one fixed device array instead of the caller (b2_kernels.h).

Kept in its own file, collected last, so it is checked both in a fresh
process and after every other test has used the device. Each case runs the
allocating entry point (b2_attn, caller-owned scratch and counters) once and
the allocation-free one twice in a row on the same inputs; all three must
agree within the attention tolerance of the kernel tests (1e-5 of the largest
output), and the allocation-free results must match a float64 attention.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
ATTN_RTOL = 1e-5


@pytest.fixture(scope="module")
def torch():
    import torch
    torch.cuda.init()
    return torch


def make_case(b2, torch, B, H, Hkv, hd, cap, positions, seed, T=64):
    """Shuffled pages [page][Hkv][T][hd] and the b2_attn_args over them."""
    rng = np.random.default_rng(seed)
    pps = cap // T
    pages = rng.permutation(B * pps).astype(np.int32)
    K = rng.standard_normal((B, cap, Hkv, hd), dtype=np.float32)
    V = rng.standard_normal((B, cap, Hkv, hd), dtype=np.float32)
    Kp = np.zeros((B * pps, Hkv, T, hd), np.float32)
    Vp = np.zeros_like(Kp)
    for b in range(B):
        for p in range(pps):
            Kp[pages[b * pps + p]] = K[b, p * T:(p + 1) * T].transpose(1, 0, 2)
            Vp[pages[b * pps + p]] = V[b, p * T:(p + 1) * T].transpose(1, 0, 2)
    q = rng.standard_normal((B, H, hd), dtype=np.float32)
    keep = {"k": torch.from_numpy(Kp.reshape(-1)).cuda(), "v": torch.from_numpy(Vp.reshape(-1)).cuda(),
            "pt": torch.from_numpy(pages).cuda(), "q": torch.from_numpy(q.reshape(-1)).cuda(),
            "pos": torch.from_numpy(np.asarray(positions, np.int32)).cuda(),
            "ctx": torch.zeros(B * H * hd, dtype=torch.float32, device="cuda"),
            "err": torch.zeros(1, dtype=torch.int32, device="cuda")}
    lay = b2.KVLayout()
    lay.k_pool, lay.v_pool, lay.page_table = keep["k"].data_ptr(), keep["v"].data_ptr(), keep["pt"].data_ptr()
    lay.page_tokens, lay.pages_per_seq, lay.n_kv_heads, lay.head_dim = T, pps, Hkv, hd
    a = b2.AttnArgs()
    a.batch, a.n_heads, a.n_kv_heads, a.head_dim = B, H, Hkv, hd
    a.q, a.kv, a.positions, a.max_ctx = keep["q"].data_ptr(), lay, keep["pos"].data_ptr(), cap
    a.ctx, a.err = keep["ctx"].data_ptr(), keep["err"].data_ptr()
    return a, keep, (K, V, q)


def reference(K, V, q, positions, H, Hkv, hd):
    B = q.shape[0]
    want = np.zeros((B, H, hd))
    for b in range(B):
        n = int(positions[b]) + 1
        for h in range(H):
            kv = h // (H // Hkv)
            s = K[b, :n, kv].astype(np.float64) @ q[b, h].astype(np.float64) / np.sqrt(hd)
            p = np.exp(s - s.max())
            want[b, h] = (p / p.sum()) @ V[b, :n, kv].astype(np.float64)
    return want


def read(torch, keep, shape):
    torch.cuda.synchronize()
    assert int(keep["err"].item()) == 0
    return keep["ctx"].cpu().numpy().reshape(shape).copy()


@pytest.mark.parametrize("B,H,Hkv,hd,cap,positions", [
    (1, 32, 8, 128, 4096, [4095]),              # 8B attention at context 4096
    (2, 9, 3, 64, 2048, [2047, 100]),           # small GQA decoder, two sequences
    (3, 6, 6, 48, 256, [255, 0, 17]),           # tiny decoder, no GQA
])
def test_noalloc_matches_b2_attn(b2, torch, B, H, Hkv, hd, cap, positions):
    L = b2.lib()
    a, keep, (K, V, q) = make_case(b2, torch, B, H, Hkv, hd, cap, positions, seed=cap + B)
    shape = (B, H, hd)
    need = L.b2_attn_scratch_bytes(C.byref(a))
    scratch = torch.zeros(max(need, 256), dtype=torch.uint8, device="cuda")
    counters = torch.zeros(max(L.b2_attn_counters_len(C.byref(a)), 1), dtype=torch.int32, device="cuda")
    a.scratch, a.scratch_bytes = scratch.data_ptr(), need
    a.counters, a.counters_len = counters.data_ptr(), counters.numel()
    assert L.b2_attn(C.byref(a), None) == 0
    want = read(torch, keep, shape)
    outs = []
    for _ in range(2):                                  # two calls in a row on the shared array
        keep["ctx"].zero_()
        a.scratch, a.scratch_bytes, a.counters, a.counters_len = None, 0, None, 0
        assert L.b2_attn_noalloc(C.byref(a), None) == 0
        outs.append(read(torch, keep, shape))
    ref = reference(K, V, q, positions, H, Hkv, hd)
    for got in outs:
        assert np.abs(got - want).max() <= ATTN_RTOL * np.abs(want).max()
        assert np.abs(got - ref).max() <= ATTN_RTOL * np.abs(ref).max()


def test_noalloc_rejects_before_touching_the_array(b2, torch):
    """Calls that b2_attn would reject, and plans larger than the array, are
    refused before anything is launched or cleared."""
    L = b2.lib()
    assert L.b2_attn_noalloc(None, None) == -1
    a, keep, _ = make_case(b2, torch, 1, 8, 2, 64, 128, [127], seed=3)
    q = a.q
    a.q = None
    assert L.b2_attn_noalloc(C.byref(a), None) == -1
    a.q = q
    a.n_heads = 7                                      # not a multiple of the KV heads
    assert L.b2_attn_noalloc(C.byref(a), None) == -1
    a.n_heads = 8
    # 64 sequences of 8 query heads per KV head at head_dim 128 on 64 KV heads:
    # one split each, 64 * 64 * 8 * 130 floats of partials, more than the array
    big = b2.AttnArgs()
    big.batch, big.n_heads, big.n_kv_heads, big.head_dim = 64, 512, 64, 128
    big.q, big.positions, big.max_ctx, big.ctx, big.err = a.q, a.positions, 64, a.ctx, a.err
    lay = b2.KVLayout()
    lay.k_pool, lay.v_pool, lay.page_table = a.kv.k_pool, a.kv.v_pool, a.kv.page_table
    lay.page_tokens, lay.pages_per_seq, lay.n_kv_heads, lay.head_dim = 64, 1, 64, 128
    big.kv = lay
    assert L.b2_attn_scratch_bytes(C.byref(big)) > (4 << 20)
    assert L.b2_attn_noalloc(C.byref(big), None) == -9
    torch.cuda.synchronize()
    assert int(keep["err"].item()) == 0
