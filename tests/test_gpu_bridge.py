"""The sp_llama_* bridge on the GPU, called with HOST buffers as llama.cpp
does: codes and reconstructions equal the oracle's; memory accounting,
clear_range, validate_k and the host-buffer fused decode."""
import ctypes as C

import numpy as np
import pytest

import oracle as O
import spb200
from spb200 import synth

pytestmark = pytest.mark.gpu
KB, VB = [5, 5, 4, 3], [3]


@pytest.fixture
def bridge(cuda, monkeypatch):
    monkeypatch.setenv("SHANNON_PRIME_ENABLED", "1")
    for k in ("SHANNON_PRIME_K_BITS", "SHANNON_PRIME_V_BITS", "SHANNON_PRIME_MOBIUS"):
        monkeypatch.delenv(k, raising=False)
    L = spb200.lib()
    p = spb200.SpLlamaParams(128, 2, 2, 600, 1, None, None)
    ctx = L.sp_llama_init(C.byref(p))
    assert ctx
    yield L, ctx
    L.sp_llama_free(ctx)


def _f(a):
    return np.ascontiguousarray(a, np.float32).ctypes.data


def test_bridge_round_trip(bridge):
    L, ctx = bridge
    k, v = synth.kv_slot_np(0, 1, 1, 500, 128)
    k = np.ascontiguousarray(k)
    v = np.ascontiguousarray(v)
    L.sp_llama_write_k_batch(ctx, 1, 1, 0, 500, k.ctypes.data)
    L.sp_llama_write_v_batch(ctx, 1, 1, 0, 500, v.ctypes.data)
    ko = np.zeros_like(k)
    vo = np.zeros_like(v)
    L.sp_llama_read_k_batch(ctx, 1, 1, 0, 500, ko.ctypes.data)
    L.sp_llama_read_v_batch(ctx, 1, 1, 0, 500, vo.ctypes.data)
    np.testing.assert_array_equal(ko, O.ship_read(O.ship_write(k, KB, True), 128, KB, True))
    np.testing.assert_array_equal(vo, O.ship_read(O.ship_write(v, VB, False), 128, VB, False))
    one = np.zeros(128, np.float32)
    L.sp_llama_read_k_partial(ctx, 1, 1, 7, one.ctypes.data, 1)
    ref = O.ship_read(O.ship_write(k[7:8], KB, True), 128, KB, True, max_bands=1)[0]
    np.testing.assert_array_equal(one, ref)
    m = L.sp_llama_memory(ctx)
    assert m.n_positions == 500
    assert m.compressed_bytes == 2 * 2 * 500 * (76 + 50)
    assert abs(m.compression_ratio - 512 / 126) < 1e-4
    L.sp_llama_clear_range(ctx, 0, 250)
    L.sp_llama_read_k_batch(ctx, 1, 1, 0, 500, ko.ctypes.data)
    assert not ko[:250].any() and ko[250:].any()
    assert L.sp_llama_validate_k(ctx, k[3].ctypes.data, 128) > 0.97
    assert not L.sp_llama_get_freq_factors(ctx) and L.sp_llama_get_n_freqs(ctx) == 0


def test_bridge_env_bits(cuda, monkeypatch):
    monkeypatch.setenv("SHANNON_PRIME_ENABLED", "1")
    monkeypatch.setenv("SHANNON_PRIME_DRAFT_K_BITS", "4,3")
    monkeypatch.setenv("SHANNON_PRIME_V_BITS", "2")
    L = spb200.lib()
    p = spb200.SpLlamaParams(128, 1, 1, 64, 1, None, None)
    draft = L.sp_llama_init_with_role(C.byref(p), 2)
    target = L.sp_llama_init_with_role(C.byref(p), 1)
    try:
        x = np.ascontiguousarray(synth.kv_slot_np(2, 0, 0, 4, 128)[0])
        for ctx, kb in ((draft, [4, 3]), (target, KB)):
            L.sp_llama_write_k_batch(ctx, 0, 0, 0, 4, x.ctypes.data)
            y = np.zeros_like(x)
            L.sp_llama_read_k_batch(ctx, 0, 0, 0, 4, y.ctypes.data)
            np.testing.assert_array_equal(y, O.ship_read(O.ship_write(x, kb, True), 128, kb, True))
        m = L.sp_llama_memory(draft)
        # K 4,3 over two bands of 64: (2+32)+(2+24); V 2-bit: 2+32
        assert m.compressed_bytes == 4 * ((2 + 32) + (2 + 24) + (2 + 32))
    finally:
        L.sp_llama_free(draft)
        L.sp_llama_free(target)


def test_bridge_fused_decode_host_buffers(bridge):
    L, ctx = bridge
    T, H, G, n = 512, 2, 4, 128
    ks = np.stack([synth.kv_slot_np(9, 0, h, T, n)[0] for h in range(H)], 1)
    vs = np.stack([synth.kv_slot_np(9, 0, h, T, n)[1] for h in range(H)], 1)
    rc = L.sp_llama_write_kv_tokens(ctx, 0, 0, T, np.ascontiguousarray(ks).ctypes.data,
                                    np.ascontiguousarray(vs).ctypes.data)
    assert rc == 0
    q = synth.q_np(9, 1, H * G, n, 0.1)
    out = np.zeros((1, H * G, n), np.float16)
    rc = L.sp_llama_attn_decode(ctx, 0, 1, q.ctypes.data, H * G, T, 1.0, out.ctypes.data, -1)
    assert rc == 0
    kp = np.stack([O.ship_write(ks[:, h], KB, True) for h in range(H)])
    vp = np.stack([O.ship_write(vs[:, h], VB, False) for h in range(H)])
    ref = O.attn_decode(kp, vp, n, KB, VB, True, q[0], T, 1.0)
    err = np.linalg.norm(out[0].astype(np.float64) - ref) / np.linalg.norm(ref)
    assert err <= 1e-3
    # page-locked (mapped) caller buffers are read and written in place by
    # the decode kernels: same result
    import torch
    qp = torch.from_numpy(q).pin_memory()
    op = torch.zeros(out.shape, dtype=torch.float16).pin_memory()
    rc = L.sp_llama_attn_decode(ctx, 0, 1, qp.data_ptr(), H * G, T, 1.0, op.data_ptr(), -1)
    assert rc == 0
    np.testing.assert_array_equal(op.numpy(), out)
    # pinned q with a pageable output: same bytes
    out2 = np.zeros_like(out)
    rc = L.sp_llama_attn_decode(ctx, 0, 1, qp.data_ptr(), H * G, T, 1.0, out2.ctypes.data, -1)
    assert rc == 0
    np.testing.assert_array_equal(out2, out)
    # pageable q with a page-locked output: same bytes
    op2 = torch.zeros(out.shape, dtype=torch.float16).pin_memory()
    rc = L.sp_llama_attn_decode(ctx, 0, 1, q.ctypes.data, H * G, T, 1.0, op2.data_ptr(), -1)
    assert rc == 0
    np.testing.assert_array_equal(op2.numpy(), out)
