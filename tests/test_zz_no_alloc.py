"""The allocation-free fused decode (sp_cuda_attn_decode_noalloc).

It exists for callers that cannot call cudaMalloc — engines that own every
device buffer through their own allocator (llama.cpp's ggml backend
buffers) or plugin hosts that forbid a library from growing its device
footprint — and so keeps its split partials in a fixed device array inside
the library.  These tests call it through the C-ABI on a cache whose
buffers the caller owns and check its output against sp_cuda_attn_decode
(the workspace-backed entry point) within the same 1e-3 relative-L2
tolerance as the other decode tests, on two calls in a row: the shared
array keeps the previous call's contents, which must not leak into the next.

This file is named to be collected last, so a stop-at-first-failure run has
already run every other test before it.
"""
import ctypes as C

import numpy as np
import pytest

import oracle as O
import spb200
from spb200 import synth

pytestmark = pytest.mark.gpu
RTOL_L2 = 1e-3


def _rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _filled_cache(torch, n_layers, H, T, seed, mobius=True):
    cache = spb200.Cache(128, n_layers, H, T, mobius=mobius)
    for layer in range(n_layers):
        k = np.stack([synth.kv_slot_np(seed, layer, h, T, 128)[0] for h in range(H)], 1)
        v = np.stack([synth.kv_slot_np(seed, layer, h, T, 128)[1] for h in range(H)], 1)
        cache.write_kv_tokens(layer, 0, torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda())
    torch.cuda.synchronize()
    return cache


def _noalloc(cache, layer0, n_layers, q, kv_len, out, scale=1.0, max_bands=-1, slabs=None):
    """slabs: optional (k_ptr, v_ptr, max_seq_len) of caller-owned copies."""
    cc = cache.cc
    kp, vp, ms = slabs if slabs else (cc.d_k_cache, cc.d_v_cache, cc.max_seq_len)
    return spb200.lib().sp_cuda_attn_decode_noalloc(
        kp, vp, ms, C.byref(cc.k_bands), C.byref(cc.v_bands),
        cc.d_mobius_order if cache.cfg.use_mobius_mask else None, cc.config.n_heads_kv, layer0,
        n_layers, q.data_ptr(), q.shape[1], kv_len, scale, out.data_ptr(), max_bands, None)


def _status_clear():
    """Read and clear the no-alloc entry point's shared status word."""
    st = C.c_uint(0xFFFFFFFF)
    assert spb200.lib().sp_cuda_attn_decode_noalloc_status(C.byref(st), 1, None) == 0
    return st.value


@pytest.mark.parametrize("impl", [0, 1])
def test_noalloc_matches_workspace_entry_point_twice(cuda, impl):
    import torch
    H, G, T = 8, 4, 3000
    cache = _filled_cache(torch, 3, H, T, seed=21)
    L = spb200.lib()
    L.sp_cuda_attn_force_impl(impl)
    try:
        _status_clear()
        calls = [(0, 1, T, 1.0, 1), (1, 2, 1234, 0.5, 2)]   # different shapes back to back
        for layer0, nl, kv_len, scale, qseed in calls:
            q = torch.from_numpy(synth.q_np(qseed, nl, H * G, 128, 1 / np.sqrt(128))).cuda()
            ref = torch.empty(nl, H * G, 128, dtype=torch.float16, device="cuda")
            got = torch.full_like(ref, 9.0)
            cache.attn_decode(layer0, nl, q, kv_len, ref, logit_scale=scale)
            rc = _noalloc(cache, layer0, nl, q, kv_len, got, scale)
            assert rc == 0, spb200.last_error()
            torch.cuda.synchronize()
            err = _rel_l2(got.float().cpu().numpy(), ref.float().cpu().numpy())
            assert err <= RTOL_L2, (layer0, nl, kv_len, err)
        assert _status_clear() == 0
    finally:
        L.sp_cuda_attn_force_impl(0)


def _oracle_decode(cache, layer, q_layer, kv_len, scale, mobius):
    H = cache.n_heads_kv
    kp = cache.slab(0).cpu().numpy()[layer * H:(layer + 1) * H]
    vp = cache.slab(1).cpu().numpy()[layer * H:(layer + 1) * H]
    return O.attn_decode(kp, vp, 128, [5, 5, 4, 3], [3], mobius, q_layer, kv_len, scale)


@pytest.mark.parametrize("mobius", [True, False])
def test_noalloc_against_oracle(cuda, mobius):
    """Against the CPU oracle directly, with the Möbius order and with
    d_mobius_order = NULL (a cache written without the reorder)."""
    import torch
    H, G, T = 4, 4, 777
    cache = _filled_cache(torch, 2, H, T, seed=23, mobius=mobius)
    q_np = synth.q_np(5, 2, H * G, 128, 1 / np.sqrt(128))
    q = torch.from_numpy(q_np).cuda()
    got = torch.full((2, H * G, 128), 9.0, dtype=torch.float16, device="cuda")
    assert _noalloc(cache, 0, 2, q, T, got, 0.9) == 0, spb200.last_error()
    torch.cuda.synchronize()
    for layer in range(2):
        ref = _oracle_decode(cache, layer, q_np[layer], T, 0.9, mobius)
        err = _rel_l2(got[layer].float().cpu().numpy(), ref)
        assert err <= RTOL_L2, (mobius, layer, err)
    assert _status_clear() == 0


def test_noalloc_generic_fallback_on_unaligned_slabs(cuda):
    """Caller-owned slabs whose slot stride breaks the tensor-core kernel's
    16-byte tile alignment (max_seq_len 1001) take the generic kernel; the
    result still matches sp_cuda_attn_decode and the oracle, twice."""
    import torch
    H, G, T, MS = 8, 4, 1000, 1001
    cache = _filled_cache(torch, 1, H, T, seed=24)
    kb, vb = cache.k_bytes, cache.v_bytes
    ks = torch.zeros(H, MS, kb, dtype=torch.uint8, device="cuda")
    vs = torch.zeros(H, MS, vb, dtype=torch.uint8, device="cuda")
    ks[:, :T] = cache.slab(0)[:, :T]
    vs[:, :T] = cache.slab(1)[:, :T]
    for qseed in (6, 7):
        q_np = synth.q_np(qseed, 1, H * G, 128, 1 / np.sqrt(128))
        q = torch.from_numpy(q_np).cuda()
        ref = torch.empty(1, H * G, 128, dtype=torch.float16, device="cuda")
        cache.attn_decode(0, 1, q, T, ref)
        got = torch.full_like(ref, 9.0)
        assert _noalloc(cache, 0, 1, q, T, got, slabs=(ks.data_ptr(), vs.data_ptr(), MS)) == 0
        torch.cuda.synchronize()
        g = got[0].float().cpu().numpy()
        assert _rel_l2(g, ref[0].float().cpu().numpy()) <= RTOL_L2
        assert _rel_l2(g, _oracle_decode(cache, 0, q_np[0], T, 1.0, True)) <= RTOL_L2
    assert _status_clear() == 0


def test_noalloc_rejects_requests_beyond_its_scratch(cuda):
    import torch
    cache = _filled_cache(torch, 1, 8, 64, seed=22)
    q = torch.zeros(16, 32, 128, dtype=torch.float16, device="cuda")
    out = torch.zeros_like(q)
    cc = cache.cc
    # 16 layers x 32 q heads exceeds the 16 MiB scratch at head_dim 128
    rc = spb200.lib().sp_cuda_attn_decode_noalloc(
        cc.d_k_cache, cc.d_v_cache, cc.max_seq_len, C.byref(cc.k_bands), C.byref(cc.v_bands),
        cc.d_mobius_order, 8, 0, 16, q.data_ptr(), 32, 64, 1.0, out.data_ptr(), -1, None)
    assert rc == spb200.SP_ERR_ARG
    assert "scratch" in spb200.last_error()[1]
