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

import spb200
from spb200 import synth

pytestmark = pytest.mark.gpu
RTOL_L2 = 1e-3


def _rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _filled_cache(torch, n_layers, H, T, seed):
    cache = spb200.Cache(128, n_layers, H, T)
    for layer in range(n_layers):
        k = np.stack([synth.kv_slot_np(seed, layer, h, T, 128)[0] for h in range(H)], 1)
        v = np.stack([synth.kv_slot_np(seed, layer, h, T, 128)[1] for h in range(H)], 1)
        cache.write_kv_tokens(layer, 0, torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda())
    torch.cuda.synchronize()
    return cache


def _noalloc(cache, layer0, n_layers, q, kv_len, out, scale=1.0, max_bands=-1):
    cc = cache.cc
    return spb200.lib().sp_cuda_attn_decode_noalloc(
        cc.d_k_cache, cc.d_v_cache, cc.max_seq_len, C.byref(cc.k_bands), C.byref(cc.v_bands),
        cc.d_mobius_order, cc.config.n_heads_kv, layer0, n_layers, q.data_ptr(), q.shape[1],
        kv_len, scale, out.data_ptr(), max_bands, None)


@pytest.mark.parametrize("impl", [0, 1])
def test_noalloc_matches_workspace_entry_point_twice(cuda, impl):
    import torch
    H, G, T = 8, 4, 3000
    cache = _filled_cache(torch, 3, H, T, seed=21)
    L = spb200.lib()
    L.sp_cuda_attn_force_impl(impl)
    try:
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
    finally:
        L.sp_cuda_attn_force_impl(0)


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
