"""Disk tier (sp_cuda_cache_save / _load / _load_partial): the properties of
the reference's disk round-trip test (CHANGELOG.md:127-131, tests/
test_disk_cache_roundtrip.cpp of its engine) — round-trip exactness, strict
model-hash rejection and the SP_DISK_HASH_STRICT=0 escape — for both body
layouts, plus the band-major partial load, which must read back exactly as a
partial-band read of the original cache (shannon_prime_llama.h:240-255)."""
import ctypes as C

import numpy as np
import pytest

import oracle as O
import spb200
from spb200 import synth

KB, VB = [5, 5, 4, 3], [3]


def test_fnv1a64_known_answers(built_lib):
    L = spb200.lib()
    assert L.sp_fnv1a64(b"", 0) == 0xCBF29CE484222325
    assert L.sp_fnv1a64(b"a", 1) == 0xAF63DC4C8601EC8C
    assert L.sp_fnv1a64(b"foobar", 6) == 0x85944171F73967E8


def _filled(torch, L, H, T, n_pos, seed):
    cache = spb200.Cache(128, L, H, T)
    for layer in range(L):
        k = np.stack([synth.kv_slot_np(seed, layer, h, n_pos, 128)[0] for h in range(H)], 1)
        v = np.stack([synth.kv_slot_np(seed, layer, h, n_pos, 128)[1] for h in range(H)], 1)
        cache.write_kv_tokens(layer, 0, torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda())
    torch.cuda.synchronize()
    return cache


@pytest.mark.gpu
@pytest.mark.parametrize("version", [2, 3])
def test_roundtrip_hash_guard_and_partial(cuda, tmp_path, monkeypatch, version):
    import torch
    L, H, T, n_pos = 3, 4, 1024, 777
    Lb = spb200.lib()
    src = _filled(torch, L, H, T, n_pos, seed=31)
    prefix = str(tmp_path / f"cache_v{version}").encode()
    h = Lb.sp_fnv1a64(b"/models/a.gguf", 14)
    assert Lb.sp_cuda_cache_save(C.byref(src.cc), prefix, n_pos, h, version) == 0
    ks, vs = src.slab(0).cpu().numpy(), src.slab(1).cpu().numpy()

    dst = spb200.Cache(128, L, H, T)
    assert Lb.sp_cuda_cache_load(C.byref(dst.cc), prefix, h) == n_pos
    torch.cuda.synchronize()
    np.testing.assert_array_equal(dst.slab(0).cpu().numpy()[:, :n_pos], ks[:, :n_pos])
    np.testing.assert_array_equal(dst.slab(1).cpu().numpy()[:, :n_pos], vs[:, :n_pos])

    # strict hash guard, and the escape hatch
    other = Lb.sp_fnv1a64(b"/models/b.gguf", 14)
    bad = spb200.Cache(128, L, H, T)
    assert Lb.sp_cuda_cache_load(C.byref(bad.cc), prefix, other) == spb200.SP_ERR_ARG
    assert "hash" in spb200.last_error()[1]
    monkeypatch.setenv("SP_DISK_HASH_STRICT", "0")
    assert Lb.sp_cuda_cache_load(C.byref(bad.cc), prefix, other) == n_pos
    monkeypatch.delenv("SP_DISK_HASH_STRICT")
    # a cache of another layout is refused
    wrong = spb200.Cache(128, L, H, T, k_bits=[5, 4, 4])
    assert Lb.sp_cuda_cache_load(C.byref(wrong.cc), prefix, h) == spb200.SP_ERR_ARG

    # partial loads: every band at or past max_bands reads as zero, exactly
    # like a partial read of the original rows
    for mb in (0, 1, 2, 3):
        part = spb200.Cache(128, L, H, T)
        assert Lb.sp_cuda_cache_load_partial(C.byref(part.cc), prefix, h, mb) == n_pos
        for which, bits, mob, slab in ((0, KB, True, ks), (1, VB, False, vs)):
            out = torch.empty(n_pos, 128, device="cuda")
            part.read_batch(which, 1, 2, 0, out)
            torch.cuda.synchronize()
            ref = O.ship_read(slab[1 * H + 2, :n_pos], 128, bits, mob, max_bands=mb)
            np.testing.assert_array_equal(out.cpu().numpy(), ref)
