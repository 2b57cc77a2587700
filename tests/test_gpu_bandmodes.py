"""Band modes and the dual-cache merge (the f4 row):

- ternary noise-tail bands (sp_config_t::{k,v}_ternary_mask, set by the
  bridge from SHANNON_PRIME_{K,V}_TERNARY_BANDS as the reference's
  parse_role_ternary_mask does, shannon_prime_llama.c:142-166): the masked
  band is stored at 2 bits per code ({-1, 0, +1}); codes bit-exact with the
  oracle's quantiser at those bits, and the fused decode within 1e-3;
- SHANNON_PRIME_FP8=1 is advisory at the bridge, as in the reference
  (shannon_prime_llama.c:287-326): the context comes up with integer bands;
- the System 1 <-> 2 merged read (sp_cuda_dual_merge) against a host select.
"""
import ctypes as C

import numpy as np
import pytest

import oracle as O
import spb200
from spb200 import synth

pytestmark = pytest.mark.gpu


def test_ternary_band_codes_and_decode(cuda):
    import torch
    H, G, T = 4, 4, 500
    cfg = spb200.make_config(128, 1, H)
    cfg.k_ternary_mask = 1 << 3
    cfg.v_ternary_mask = 1 << 0
    cc = spb200.SpCudaCache()
    L = spb200.lib()
    assert L.sp_cuda_cache_init(C.byref(cc), C.byref(cfg), T, None) == 0
    kb, vb = [5, 5, 4, 2], [2]
    assert list(cc.k_bands.band_bits)[:4] == kb and cc.k_bands.total_bytes == 72
    assert cc.v_bands.band_bits[0] == 2 and cc.v_bands.total_bytes == 34
    k = np.stack([synth.kv_slot_np(41, 0, h, T, 128)[0] for h in range(H)], 1)
    v = np.stack([synth.kv_slot_np(41, 0, h, T, 128)[1] for h in range(H)], 1)
    kd, vd = torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda()
    rc = L.sp_cuda_write_kv_tokens(C.byref(cc), 0, 0, T, kd.data_ptr(), vd.data_ptr(), 0)
    assert rc == 0
    torch.cuda.synchronize()
    from spb200.cache import _wrap_device
    ks = _wrap_device(cc.d_k_cache, H * cc.max_seq_len * 72, torch.uint8).view(H, cc.max_seq_len, 72)
    vs = _wrap_device(cc.d_v_cache, H * cc.max_seq_len * 34, torch.uint8).view(H, cc.max_seq_len, 34)
    ks, vs = ks.cpu().numpy(), vs.cpu().numpy()
    for h in range(H):
        assert np.array_equal(ks[h, :T], O.ship_write(k[:, h], kb, True))
        assert np.array_equal(vs[h, :T], O.ship_write(v[:, h], vb, False))
    q = synth.q_np(41, 1, H * G, 128, 1 / np.sqrt(128))
    out = torch.empty(1, H * G, 128, dtype=torch.float16, device="cuda")
    qd = torch.from_numpy(q).cuda()
    assert L.sp_cuda_attn_decode(C.byref(cc), 0, 1, qd.data_ptr(), H * G, T, 1.0, out.data_ptr(), -1, None) == 0
    torch.cuda.synchronize()
    ref = O.attn_decode(ks, vs, 128, kb, vb, True, q[0], T, 1.0)
    got = out[0].float().cpu().numpy()
    assert np.linalg.norm(got - ref) / np.linalg.norm(ref) <= 1e-3
    L.sp_cuda_cache_free(C.byref(cc))


def test_bridge_ternary_env_and_fp8_advisory(cuda, monkeypatch):
    L = spb200.lib()
    monkeypatch.setenv("SHANNON_PRIME_ENABLED", "1")
    monkeypatch.setenv("SHANNON_PRIME_K_TERNARY_BANDS", " 3, x,40")
    monkeypatch.setenv("SHANNON_PRIME_FP8", "1")
    p = spb200.SpLlamaParams(128, 2, 2, 64, 1, None, None)
    ctx = L.sp_llama_init(C.byref(p))
    assert ctx
    cc = C.cast(L.sp_llama_get_cuda_cache(ctx), C.POINTER(spb200.SpCudaCache)).contents
    assert list(cc.k_bands.band_bits)[:4] == [5, 5, 4, 2]
    assert cc.config.k_ternary_mask == 1 << 3 and cc.config.use_fp8 == 0
    assert cc.v_bands.band_bits[0] == 3
    L.sp_llama_free(ctx)


@pytest.mark.parametrize("in_place", [False, True])
def test_dual_merge(cuda, in_place):
    import torch
    rng = np.random.default_rng(3)
    n, row = 1000, 128
    a = torch.from_numpy(rng.standard_normal((n, row)).astype(np.float32)).cuda()
    b = torch.from_numpy(rng.standard_normal((n, row)).astype(np.float32)).cuda()
    route = rng.random(n) < 0.2
    words = np.zeros((n + 31) // 32, np.uint32)
    for p in np.nonzero(route)[0]:
        words[p >> 5] |= np.uint32(1 << (p & 31))
    rb = torch.from_numpy(words.view(np.int32)).cuda()
    expect = np.where(route[:, None], b.cpu().numpy(), a.cpu().numpy())
    out = a if in_place else torch.empty_like(a)
    assert spb200.lib().sp_cuda_dual_merge(a.data_ptr(), b.data_ptr(), rb.data_ptr(), n, row,
                                           out.data_ptr(), None) == 0
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), expect)
