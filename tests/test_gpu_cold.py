"""GPU tests of the cold-storage tier (sp_cuda_cold_*): byte-exact mirror of
a layer slab through incremental writebacks and a restore, ring wrap-around
bookkeeping, and the refusals the engine relies on (kv_cache.cpp:1385-1530
drives these calls)."""
import ctypes as C

import numpy as np
import pytest

import spb200
from spb200 import synth
from spb200.cache import Cache

pytestmark = pytest.mark.gpu


def _filled_cache(T=96, L=2, H=4, hd=128):
    import torch
    cache = Cache(hd, L, H, T)
    for layer in range(L):
        k = np.stack([synth.kv_slot_np(3, layer, h, T, hd)[0] for h in range(H)], 1)
        v = np.stack([synth.kv_slot_np(3, layer, h, T, hd)[1] for h in range(H)], 1)
        cache.write_kv_tokens(layer, 0, torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda())
    torch.cuda.synchronize()
    return cache


def test_cold_writeback_restore_round_trip(cuda):
    import torch
    L_ = spb200.lib()
    cache = _filled_cache()
    H, S, kb = cache.n_heads_kv, cache.max_seq_len, cache.k_bytes
    layer = 1
    slab = cache.slab(0)[layer * H:(layer + 1) * H]          # this layer's K slab
    before = slab.clone()
    base = cache.cc.d_k_cache + layer * H * S * kb
    cl = spb200.SpColdLayer()
    assert L_.sp_cuda_cold_layer_init(C.byref(cl), H * S * kb, kb, H) == 0
    try:
        assert cl.initialized and not cl.ring_mode and cl.oldest_pos == -1
        # incremental writebacks, as KvCache::cold_writeback issues them
        assert L_.sp_cuda_cold_writeback(C.byref(cl), base, 0, 40, None) == 0
        assert L_.sp_cuda_cold_writeback(C.byref(cl), base, 40, 25, None) == 0
        torch.cuda.synchronize()
        assert (cl.oldest_pos, cl.newest_pos, cl.write_head) == (0, 64, 65 * H * kb)
        n = 65 * H * kb
        host = np.ctypeslib.as_array((C.c_uint8 * n).from_address(cl.h_pinned))
        np.testing.assert_array_equal(host, before.flatten()[:n].cpu().numpy())
        slab.zero_()
        assert L_.sp_cuda_cold_restore(C.byref(cl), base, 65, None) == 0
        torch.cuda.synchronize()
        np.testing.assert_array_equal(slab.flatten()[:n].cpu().numpy(), before.flatten()[:n].cpu().numpy())
        assert int(slab.flatten()[n:].abs().sum()) == 0        # nothing past the restored range
    finally:
        L_.sp_cuda_cold_layer_free(C.byref(cl))
    assert not cl.initialized and not cl.h_pinned


def test_cold_ring_wrap_and_refusals(cuda):
    import torch
    L_ = spb200.lib()
    cache = _filled_cache()
    H, kb = cache.n_heads_kv, cache.k_bytes
    base = cache.cc.d_k_cache
    per_pos = H * kb
    cl = spb200.SpColdLayer()
    assert L_.sp_cuda_cold_layer_init(C.byref(cl), 50 * per_pos, kb, H) == 0
    try:
        assert L_.sp_cuda_cold_writeback(C.byref(cl), base, 0, 30, None) == 0
        assert not cl.ring_mode
        assert L_.sp_cuda_cold_writeback(C.byref(cl), base, 30, 30, None) == 0   # wraps
        torch.cuda.synchronize()
        assert cl.ring_mode and cl.write_head == 30 * per_pos
        assert (cl.newest_pos, cl.oldest_pos) == (59, 10)       # 50 positions held
        assert L_.sp_cuda_cold_restore(C.byref(cl), base, 10, None) == -1      # ring mode
        assert L_.sp_cuda_cold_writeback(C.byref(cl), base, 0, 51, None) == -1  # larger than the buffer
        assert L_.sp_cuda_cold_writeback(C.byref(cl), None, 0, 1, None) == -1
        assert L_.sp_cuda_cold_writeback(C.byref(cl), base, 0, 0, None) == -1
    finally:
        L_.sp_cuda_cold_layer_free(C.byref(cl))
    assert L_.sp_cuda_cold_layer_init(C.byref(cl), 0, kb, H) == -1
    assert L_.sp_cuda_cold_restore(C.byref(cl), base, 1, None) == -1           # not initialised


def test_d2h_h2d_async_wrappers(cuda):
    import torch
    L_ = spb200.lib()
    src = torch.arange(4096, dtype=torch.int32, device="cuda")
    host = torch.zeros(4096, dtype=torch.int32).pin_memory()
    L_.sp_cuda_d2h_async(host.data_ptr(), src.data_ptr(), 4 * 4096, None)
    torch.cuda.synchronize()
    assert torch.equal(host, src.cpu())
    dst = torch.zeros_like(src)
    L_.sp_cuda_h2d_async(dst.data_ptr(), host.data_ptr(), 4 * 4096, None)
    torch.cuda.synchronize()
    assert torch.equal(dst, src)
