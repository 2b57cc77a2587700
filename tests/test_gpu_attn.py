"""GPU parity of the fused decompress-KQ/V decode attention against the
CPU oracle (double-accumulated softmax attention over decompressed rows).
Tolerance: relative L2 error <= 1e-3 per output tensor (the path's stated
floating-point tolerance); the fp16 output rounding alone is ~3e-4."""
import numpy as np
import pytest

import oracle as O
import spb200
from spb200 import synth

pytestmark = pytest.mark.gpu
KB, VB = [5, 5, 4, 3], [3]
RTOL_L2 = 1e-3


def _rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _build(torch, n_layers, H, T, n, seed, kb=KB, vb=VB, mobius=True, max_seq=None):
    cache = spb200.Cache(n, n_layers, H, max_seq or T, kb, vb, mobius)
    for layer in range(n_layers):
        ks, vs = [], []
        for h in range(H):
            k, v = synth.kv_slot_np(seed, layer, h, T, n)
            ks.append(k)
            vs.append(v)
        cache.write_kv_tokens(layer, 0, torch.from_numpy(np.stack(ks, 1)).cuda(),
                              torch.from_numpy(np.stack(vs, 1)).cuda())
    torch.cuda.synchronize()
    return cache


def _oracle(cache, layer, q, kv_len, n, kb, vb, mobius, scale):
    H = cache.n_heads_kv
    ks = cache.slab(0).cpu().numpy()[layer * H:(layer + 1) * H]
    vs = cache.slab(1).cpu().numpy()[layer * H:(layer + 1) * H]
    return O.attn_decode(ks, vs, n, kb, vb, mobius, q, kv_len, scale)


@pytest.mark.parametrize("impl", [1, 2, 3, 0])
@pytest.mark.parametrize("kv_len", [1, 15, 16, 100, 1000, 4096])
def test_decode_matches_oracle(cuda, impl, kv_len):
    import torch
    n, H, G, L = 128, 8, 4, 2
    cache = _build(torch, L, H, 4096, n, seed=1)
    q = synth.q_np(1, L, H * G, n, 1.0 / np.sqrt(128))
    out = torch.empty(L, H * G, n, dtype=torch.float16, device="cuda")
    spb200.lib().sp_cuda_attn_force_impl(impl)
    try:
        cache.attn_decode(0, L, torch.from_numpy(q).cuda(), kv_len, out)
        torch.cuda.synchronize()
    finally:
        spb200.lib().sp_cuda_attn_force_impl(0)
    got = out.float().cpu().numpy()
    for layer in range(L):
        ref = _oracle(cache, layer, q[layer], kv_len, n, KB, VB, True, 1.0)
        err = _rel_l2(got[layer], ref)
        assert err <= RTOL_L2, (layer, err)


@pytest.mark.parametrize("impl", [1, 2, 3, 0])
def test_decode_layer_offset_scale_and_partial_bands(cuda, impl):
    import torch
    n, H, G = 128, 2, 4
    # 384 slots: whole 128-position tiles, so the tcgen05 kernel takes it
    cache = _build(torch, 3, H, 300, n, seed=3, max_seq=384)
    q = synth.q_np(3, 1, H * G, n, 1.0)
    out = torch.empty(1, H * G, n, dtype=torch.float16, device="cuda")
    spb200.lib().sp_cuda_attn_force_impl(impl)
    try:
        cache.attn_decode(2, 1, torch.from_numpy(q).cuda(), 300, out, logit_scale=0.125)
        torch.cuda.synchronize()
        ref = _oracle(cache, 2, q[0], 300, n, KB, VB, True, 0.125)
        assert _rel_l2(out.float().cpu().numpy()[0], ref) <= RTOL_L2
        # max_bands=2: bands 2,3 of K and nothing past V's single band dropped
        cache.attn_decode(2, 1, torch.from_numpy(q).cuda(), 300, out, logit_scale=0.125, max_bands=2)
        torch.cuda.synchronize()
    finally:
        spb200.lib().sp_cuda_attn_force_impl(0)
    ks = cache.slab(0).cpu().numpy()[2 * H:3 * H, :300]
    vs = cache.slab(1).cpu().numpy()[2 * H:3 * H, :300]
    kh = O.ship_read(ks.reshape(-1, ks.shape[-1]), n, KB, True, max_bands=2).reshape(H, 300, n)
    vh = O.ship_read(vs.reshape(-1, vs.shape[-1]), n, VB, False).reshape(H, 300, n)
    got = out.float().cpu().numpy()[0]
    for g in range(H * G):
        s = 0.125 * (kh[g // G].astype(np.float64) @ q[0, g].astype(np.float64))
        p = np.exp(s - s.max())
        p /= p.sum()
        assert _rel_l2(got[g], p @ vh[g // G]) <= RTOL_L2


@pytest.mark.parametrize("n,kb,vb,G,mobius", [
    (64, [5, 4, 4], [5], 2, True),
    (256, [5, 5, 4, 3], [3], 1, True),
    (128, [4, 4], [4], 8, False),
])
def test_generic_layouts(cuda, n, kb, vb, G, mobius):
    import torch
    H, T = 2, 257
    cache = _build(torch, 1, H, T, n, seed=5, kb=kb, vb=vb, mobius=mobius)
    q = synth.q_np(5, 1, H * G, n, 0.2)
    out = torch.empty(1, H * G, n, dtype=torch.float16, device="cuda")
    cache.attn_decode(0, 1, torch.from_numpy(q).cuda(), T, out)
    torch.cuda.synchronize()
    ref = _oracle(cache, 0, q[0], T, n, kb, vb, mobius, 1.0)
    assert _rel_l2(out.float().cpu().numpy()[0], ref) <= RTOL_L2


def test_kv_len_zero_and_errors(cuda):
    import torch
    cache = _build(torch, 1, 2, 32, 128, seed=6)
    q = torch.ones(1, 8, 128, dtype=torch.float16, device="cuda")
    out = torch.full((1, 8, 128), 7.0, dtype=torch.float16, device="cuda")
    cache.attn_decode(0, 1, q, 0, out)
    torch.cuda.synchronize()
    assert not out.float().abs().sum().item()
    L = spb200.lib()
    import ctypes as C
    rc = L.sp_cuda_attn_decode(C.byref(cache.cc), 0, 1, q.data_ptr(), 7, 10, 1.0,
                               out.data_ptr(), -1, None)
    assert rc == spb200.SP_ERR_ARG                       # 7 q heads over 2 kv heads
    rc = L.sp_cuda_attn_decode(C.byref(cache.cc), 0, 1, q.data_ptr(), 8, 10_000, 1.0,
                               out.data_ptr(), -1, None)
    assert rc == spb200.SP_ERR_ARG                       # kv_len beyond the cache


@pytest.mark.parametrize("impl", [2, 3])
@pytest.mark.parametrize("G,kv_len", [(8, 2000), (8, 17), (3, 700), (1, 999)])
def test_ship_decode_group_sizes(cuda, G, kv_len, impl):
    """The tensor-core kernel serves 1..8 query heads per KV head (8: two
    MMA column tiles, as config 3's 32 Q / 4 KV heads)."""
    import torch
    n, H, L = 128, 2, 2
    cache = _build(torch, L, H, 2048, n, seed=12)
    q = synth.q_np(12, L, H * G, n, 1.0 / np.sqrt(128))
    out = torch.empty(L, H * G, n, dtype=torch.float16, device="cuda")
    spb200.lib().sp_cuda_attn_force_impl(impl)       # the tensor-core kernel must take it
    try:
        cache.attn_decode(0, L, torch.from_numpy(q).cuda(), kv_len, out, logit_scale=0.7)
        torch.cuda.synchronize()
    finally:
        spb200.lib().sp_cuda_attn_force_impl(0)
    got = out.float().cpu().numpy()
    for layer in range(L):
        ref = _oracle(cache, layer, q[layer], kv_len, n, KB, VB, True, 0.7)
        assert _rel_l2(got[layer], ref) <= RTOL_L2, (layer, G)
