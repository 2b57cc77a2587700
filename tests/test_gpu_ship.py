"""GPU parity of the ship-path codec against the CPU oracle (through the
C-ABI): packed codes bit-exact, reconstructions bit-exact / within 1e-6."""
import ctypes as C

import numpy as np
import pytest

import oracle as O
import spb200
from spb200 import synth

pytestmark = pytest.mark.gpu
KB, VB = [5, 5, 4, 3], [3]


def _torch():
    import torch
    return torch


def _layer_inputs(seed, H, T, n, sigma=0.5):
    ks, vs = [], []
    for h in range(H):
        k, v = synth.kv_slot_np(seed, 0, h, T, n, sigma)
        ks.append(k)
        vs.append(v)
    return np.stack(ks, 1), np.stack(vs, 1)          # [T][H][n]


def test_config0_codes_bit_exact(cuda):
    """Config 0: 1 layer, 8 KV heads, hd 128, 4096 positions, seed 0."""
    torch = _torch()
    H, T, n = 8, 4096, 128
    k, v = _layer_inputs(0, H, T, n)
    cache = spb200.Cache(n, 1, H, T)
    cache.write_kv_tokens(0, 0, torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda())
    torch.cuda.synchronize()
    kg = cache.slab(0).cpu().numpy()[:, :T]
    vg = cache.slab(1).cpu().numpy()[:, :T]
    for h in range(H):
        ko = O.ship_write(k[:, h], KB, True)
        vo = O.ship_write(v[:, h], VB, False)
        assert np.array_equal(kg[h], ko), f"K codes differ in head {h}"
        assert np.array_equal(vg[h], vo), f"V codes differ in head {h}"
    # reconstruction through the read path
    out = torch.empty(T, n, device="cuda")
    for h in (0, 7):
        cache.read_batch(0, 0, h, 0, out)
        ref = O.ship_read(kg[h], n, KB, True)
        np.testing.assert_array_equal(out.cpu().numpy(), ref)
        cache.read_batch(1, 0, h, 0, out)
        ref = O.ship_read(vg[h], n, VB, False)
        np.testing.assert_array_equal(out.cpu().numpy(), ref)


@pytest.mark.parametrize("n,kb,vb,mobius", [
    (64, [5, 4, 4], [5], True),
    (256, [5, 5, 4, 3], [3], True),
    (128, [8, 6, 4, 2, 1], [4, 2], False),
    (512, [5, 5, 4, 3, 3, 2, 2], [3], True),
    (32, [4], [2], True),
])
def test_other_layouts_bit_exact(cuda, n, kb, vb, mobius):
    torch = _torch()
    H, T = 3, 77
    k, v = _layer_inputs(11, H, T, n, sigma=1.0)
    cache = spb200.Cache(n, 2, H, 100, kb, vb, mobius)
    cache.write_kv_tokens(1, 5, torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda())
    torch.cuda.synchronize()
    kg = cache.slab(0).cpu().numpy()
    vg = cache.slab(1).cpu().numpy()
    for h in range(H):
        assert np.array_equal(kg[H + h, 5:5 + T], O.ship_write(k[:, h], kb, mobius))
        assert np.array_equal(vg[H + h, 5:5 + T], O.ship_write(v[:, h], vb, False))
        out = torch.empty(T, n, device="cuda")
        for mb in (-1, 0, 1, 2):
            cache.read_batch(0, 1, h, 5, out, max_bands=mb)
            ref = O.ship_read(kg[H + h, 5:5 + T], n, kb, mobius, max_bands=mb)
            np.testing.assert_array_equal(out.cpu().numpy(), ref)


@pytest.mark.parametrize("dt", ["float16", "bfloat16"])
def test_half_inputs(cuda, dt):
    torch = _torch()
    H, T, n = 2, 40, 128
    k, v = _layer_inputs(4, H, T, n, sigma=1.0)
    tk = torch.from_numpy(k).to(getattr(torch, dt)).cuda()
    tv = torch.from_numpy(v).to(getattr(torch, dt)).cuda()
    cache = spb200.Cache(n, 1, H, T)
    cache.write_kv_tokens(0, 0, tk, tv)
    torch.cuda.synchronize()
    k32 = tk.float().cpu().numpy()
    v32 = tv.float().cpu().numpy()
    for h in range(H):
        assert np.array_equal(cache.slab(0).cpu().numpy()[h, :T], O.ship_write(k32[:, h], KB, True))
        assert np.array_equal(cache.slab(1).cpu().numpy()[h, :T], O.ship_write(v32[:, h], VB, False))


def test_reference_api_single_and_batch(cuda):
    """sp_cuda_write_k/_v, _batch and read_k/_v (reference names)."""
    torch = _torch()
    L = spb200.lib()
    n, H = 128, 4
    cache = spb200.Cache(n, 2, H, 64)
    k, v = _layer_inputs(5, 1, 20, n)
    tk = torch.from_numpy(np.ascontiguousarray(k[:, 0])).cuda()
    tv = torch.from_numpy(np.ascontiguousarray(v[:, 0])).cuda()
    cc = C.byref(cache.cc)
    L.sp_cuda_write_k_batch(cc, 1, 2, 3, 10, tk.data_ptr())
    L.sp_cuda_write_v_batch(cc, 1, 2, 3, 10, tv.data_ptr())
    for i in range(10, 20):
        L.sp_cuda_write_k(cc, 1, 2, 3 + i, tk[i].data_ptr())
        L.sp_cuda_write_v(cc, 1, 2, 3 + i, tv[i].data_ptr())
    torch.cuda.synchronize()
    assert L.sp_cuda_last_error() == 0
    slot = 1 * H + 2
    assert np.array_equal(cache.slab(0).cpu().numpy()[slot, 3:23], O.ship_write(k[:, 0], KB, True))
    assert np.array_equal(cache.slab(1).cpu().numpy()[slot, 3:23], O.ship_write(v[:, 0], VB, False))
    out = torch.empty(n, device="cuda")
    L.sp_cuda_read_k(cc, 1, 2, 7, out.data_ptr())
    torch.cuda.synchronize()
    ref = O.ship_read(cache.slab(0).cpu().numpy()[slot, 7:8], n, KB, True)[0]
    np.testing.assert_array_equal(out.cpu().numpy(), ref)
    outb = torch.empty(20, n, device="cuda")
    L.sp_cuda_read_v_batch(cc, 1, 2, 3, 20, outb.data_ptr())
    torch.cuda.synchronize()
    ref = O.ship_read(cache.slab(1).cpu().numpy()[slot, 3:23], n, VB, False)
    np.testing.assert_array_equal(outb.cpu().numpy(), ref)


def test_kernel_launchers(cuda):
    """sp_cuda_vht2_forward / mobius (un)reorder / band (de)quantize."""
    torch = _torch()
    L = spb200.lib()
    rng = np.random.default_rng(9)
    x = rng.standard_normal((33, 128)).astype(np.float32)
    t = torch.from_numpy(x).cuda()
    L.sp_cuda_vht2_forward(t.data_ptr(), 128, 33, None)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(t.cpu().numpy(), O.vht2(x))
    order = torch.from_numpy(O.mobius_order(128)).cuda()
    t2 = torch.from_numpy(x).cuda()
    L.sp_cuda_mobius_reorder(t2.data_ptr(), order.data_ptr(), 128, 33, None)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(t2.cpu().numpy(), x[:, O.mobius_order(128)])
    L.sp_cuda_mobius_unreorder(t2.data_ptr(), order.data_ptr(), 128, 33, None)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(t2.cpu().numpy(), x)
    bc = spb200.SpBandConfig()
    bits = (C.c_int * 4)(5, 5, 4, 3)
    assert L.sp_band_config_init(C.byref(bc), 128, 4, bits) == 0
    packed = torch.zeros(33, bc.total_bytes, dtype=torch.uint8, device="cuda")
    L.sp_cuda_band_quantize(t.data_ptr(), packed.data_ptr(), C.byref(bc), 33, None)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(packed.cpu().numpy(), O.band_quantize(O.vht2(x), KB))
    deq = torch.empty(33, 128, device="cuda")
    L.sp_cuda_band_dequantize(packed.data_ptr(), deq.data_ptr(), C.byref(bc), 33, None)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(deq.cpu().numpy(), O.band_dequantize(packed.cpu().numpy(), 128, KB))


def test_edge_values(cuda):
    """Zero vectors, huge values (fp16 scale overflow -> inf scale), NaN."""
    torch = _torch()
    n = 128
    x = np.zeros((6, 1, n), np.float32)
    x[1, 0] = 1e6
    x[2, 0, 3] = 7e6
    x[3, 0] = np.linspace(-1e-7, 1e-7, n)
    x[4, 0, 10] = np.nan
    x[5, 0] = np.random.default_rng(1).standard_normal(n) * 1e-3
    cache = spb200.Cache(n, 1, 1, 16)
    t = torch.from_numpy(x).cuda()
    cache.write_kv_tokens(0, 0, t, t)
    torch.cuda.synchronize()
    got_k = cache.slab(0).cpu().numpy()[0, :6]
    got_v = cache.slab(1).cpu().numpy()[0, :6]
    assert np.array_equal(got_k, O.ship_write(x[:, 0], KB, True))
    assert np.array_equal(got_v, O.ship_write(x[:, 0], VB, False))


def test_argument_errors(cuda):
    torch = _torch()
    L = spb200.lib()
    cache = spb200.Cache(128, 2, 2, 32)
    t = torch.zeros(4, 2, 128, device="cuda")
    rc = L.sp_cuda_write_kv_tokens(C.byref(cache.cc), 2, 0, 4, t.data_ptr(), 0, 0)
    assert rc == spb200.SP_ERR_ARG
    rc = L.sp_cuda_write_kv_tokens(C.byref(cache.cc), 0, 30, 4, t.data_ptr(), 0, 0)
    assert rc == spb200.SP_ERR_ARG
    L.sp_cuda_read_k_batch(C.byref(cache.cc), 0, 5, 0, 1, t.data_ptr())
    assert L.sp_cuda_last_error() == spb200.SP_ERR_ARG
    cfg = spb200.make_config(96, 1, 1)
    bad = spb200.SpCudaCache()
    assert L.sp_cuda_cache_init(C.byref(bad), C.byref(cfg), 16, None) == spb200.SP_ERR_UNSUPPORTED


@pytest.mark.parametrize("start,T,dt", [(3, 77, "float32"), (8, 64, "float32"), (0, 33, "bfloat16"),
                                        (5, 100, "float16")])
def test_ship_lane_encoder_ragged(cuda, monkeypatch, start, T, dt):
    """The lane-per-vector ship encoder (head_dim 128) at unaligned start
    positions and partial 32-position batches: codes bit-exact with the
    oracle and with the lane-group encoder (SHANNON_PRIME_ENCODE_LANEGROUP)."""
    torch = _torch()
    H, n = 3, 128
    k, v = _layer_inputs(21, H, T, n, sigma=1.0)
    tk = torch.from_numpy(k).to(getattr(torch, dt)).cuda()
    tv = torch.from_numpy(v).to(getattr(torch, dt)).cuda()
    slabs = []
    for lanegroup in (False, True):
        if lanegroup:
            monkeypatch.setenv("SHANNON_PRIME_ENCODE_LANEGROUP", "1")
        cache = spb200.Cache(n, 2, H, 112)
        cache.write_kv_tokens(1, start, tk, tv)
        torch.cuda.synchronize()
        slabs.append((cache.slab(0).cpu().numpy(), cache.slab(1).cpu().numpy()))
        monkeypatch.delenv("SHANNON_PRIME_ENCODE_LANEGROUP", raising=False)
    (kl, vl), (kg, vg) = slabs
    assert np.array_equal(kl, kg) and np.array_equal(vl, vg)
    k32, v32 = tk.float().cpu().numpy(), tv.float().cpu().numpy()
    for h in range(H):
        assert np.array_equal(kl[H + h, start:start + T], O.ship_write(k32[:, h], KB, True))
        assert np.array_equal(vl[H + h, start:start + T], O.ship_write(v32[:, h], VB, False))
        assert not kl[H + h, :start].any() and not kl[H + h, start + T:].any()
        assert not vl[H + h, :start].any() and not vl[H + h, start + T:].any()


@pytest.mark.parametrize("start,T", [(0, 4096), (3, 77), (5, 1)])
def test_ship_lane_read_matches_warp_read_and_oracle(cuda, monkeypatch, start, T):
    """The lane-per-vector ship read (head_dim 128) returns the rows of the
    warp-per-position read (SHANNON_PRIME_DECODE_WARP) and of the oracle,
    bit for bit, for full and partial band reads and ragged ranges."""
    torch = _torch()
    H, n = 2, 128
    k, v = _layer_inputs(31, H, T, n, sigma=1.0)
    cache = spb200.Cache(n, 1, H, 4112)
    cache.write_kv_tokens(0, start, torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda())
    torch.cuda.synchronize()
    kp = cache.slab(0).cpu().numpy()[:, start:start + T]
    vp = cache.slab(1).cpu().numpy()[:, start:start + T]
    for which, packed, bands, mob in ((0, kp, KB, True), (1, vp, VB, False)):
        for mb in (-1, 0, 1, 3):
            outs = []
            for warp_path in (False, True):
                if warp_path:
                    monkeypatch.setenv("SHANNON_PRIME_DECODE_WARP", "1")
                out = torch.full((T, n), 5.0, device="cuda")
                cache.read_batch(which, 0, 1, start, out, max_bands=mb)
                torch.cuda.synchronize()
                outs.append(out.cpu().numpy())
                monkeypatch.delenv("SHANNON_PRIME_DECODE_WARP", raising=False)
            np.testing.assert_array_equal(outs[0], outs[1])
            np.testing.assert_array_equal(outs[0], O.ship_read(packed[1], n, bands, mob, max_bands=mb))


@pytest.mark.parametrize("layer0,nl,start,T", [(0, 3, 0, 4096), (1, 2, 7, 333), (2, 1, 100, 1)])
def test_read_kv_tokens_matches_per_slot_reads(cuda, layer0, nl, start, T):
    """The token-major all-heads read (one launch over a layer range) puts
    every slot's rows at [layer][token][head], bit-identical with the per-slot
    reference read, for full and partial band reads."""
    torch = _torch()
    H, n, L = 3, 128, 3
    cache = spb200.Cache(n, L, H, 4112)
    for layer in range(L):
        k, v = _layer_inputs(40 + layer, H, 4096, n, sigma=1.0)
        cache.write_kv_tokens(layer, 0, torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda())
    torch.cuda.synchronize()
    lib = spb200.lib()
    for which in (0, 1):
        for mb in (-1, 1):
            got = torch.full((nl, T, H, n), 5.0, device="cuda")
            rc = lib.sp_cuda_read_kv_tokens(C.byref(cache.cc), which, layer0, nl, start, T, got.data_ptr(), mb)
            assert rc == 0, spb200.last_error()
            ref = torch.full((nl, T, H, n), 6.0, device="cuda")
            for l in range(nl):
                for h in range(H):
                    one = torch.empty(T, n, device="cuda")
                    cache.read_batch(which, layer0 + l, h, start, one, max_bands=mb)
                    ref[l, :, h] = one
            torch.cuda.synchronize()
            assert torch.equal(got, ref), (which, mb)
    bad = torch.empty(1, 4, H, n, device="cuda")
    assert lib.sp_cuda_read_kv_tokens(C.byref(cache.cc), 0, 2, 2, 0, 4, bad.data_ptr(), -1) == spb200.SP_ERR_ARG
