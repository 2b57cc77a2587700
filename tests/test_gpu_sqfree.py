"""GPU parity of the sqfree+spinor and hierarchical-Vilenkin caches against
the CPU oracle, through the C-ABI: packed slots (skeleton codes, magnitude,
residual levels, sheet bits) bit-exact, reconstructions exact, and the
sqfree fused decode attention within 1e-3 relative L2."""
import ctypes as C

import numpy as np
import pytest

import oracle as O
import spb200
from spb200 import synth
from spb200.sqfree import HierCache, SqfreeCache

pytestmark = pytest.mark.gpu
RTOL_L2 = 1e-3


def _rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _inputs(seed, n_layers, H, T, hd, sigma=0.5):
    k = np.zeros((n_layers, T, H, hd), np.float32)
    v = np.zeros_like(k)
    for layer in range(n_layers):
        for h in range(H):
            k[layer, :, h], v[layer, :, h] = synth.kv_slot_np(seed, layer, h, T, hd, sigma)
    return k, v


@pytest.mark.parametrize("hd,sk_frac,spinor,rb", [
    (128, 0.75, True, 3),      # config 2
    (128, None, True, 3),      # reference CUDA default skeleton pad_dim / 2
    (128, 0.75, False, 2),
    (64, 0.75, True, 4),
    (256, 0.5, True, 3),
])
def test_sqfree_codes_and_reads_match_oracle(cuda, hd, sk_frac, spinor, rb):
    import torch
    L, H, T = 2, 3, 80
    cache = SqfreeCache(hd, L, H, T, residual_bits=rb, use_spinor=spinor, sk_frac=sk_frac)
    OL = O.sqfree_layout(hd, sk_k=cache.cc.sk_k, residual_bits=rb, use_spinor=spinor)
    assert OL.bytes_per_pos == cache.cc.bytes_per_pos_k
    k, v = _inputs(2, L, H, T, hd)
    cache.write_kv_tokens(0, 0, torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda())
    torch.cuda.synchronize()
    ks, vs = cache.slab(0).cpu().numpy(), cache.slab(1).cpu().numpy()
    for layer in range(L):
        for h in range(H):
            s = layer * H + h
            assert np.array_equal(ks[s, :T], O.sqfree_write(k[layer, :, h], OL)), (layer, h, "K")
            assert np.array_equal(vs[s, :T], O.sqfree_write(v[layer, :, h], OL)), (layer, h, "V")
    out = torch.empty(T, hd, device="cuda")
    cache.read_batch(0, 1, 2, 0, out)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), O.sqfree_read(ks[1 * H + 2, :T], OL))
    cache.read_batch(1, 0, 1, 0, out)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), O.sqfree_read(vs[1, :T], OL))


def test_sqfree_single_vector_api(cuda):
    import torch
    cache = SqfreeCache(128, 2, 2, 16)
    OL = O.sqfree_layout(128, sk_k=cache.cc.sk_k)
    k, _ = synth.kv_slot_np(9, 0, 0, 4, 128)
    L = spb200.lib()
    dk = torch.from_numpy(k).cuda()
    for pos in range(4):
        L.sp_cuda_sqfree_write_k(C.byref(cache.cc), 1, 1, 5 + pos, dk[pos].data_ptr())
        spb200.check(None, "write_k")
    out = torch.empty(128, device="cuda")
    L.sp_cuda_sqfree_read_k(C.byref(cache.cc), 1, 1, 7, out.data_ptr())
    torch.cuda.synchronize()
    packed = cache.slab(0).cpu().numpy()[3, 5:9]
    assert np.array_equal(packed, O.sqfree_write(k, OL))
    assert np.array_equal(out.cpu().numpy(), O.sqfree_read(packed[2:3], OL)[0])


@pytest.mark.parametrize("T,G,hd,sk_frac", [
    (1, 4, 128, 0.75), (77, 4, 128, 0.75), (1000, 4, 128, 0.75), (333, 2, 128, 0.75),
    (300, 8, 128, 0.75), (300, 4, 128, None), (300, 4, 256, 0.75), (200, 4, 32, 0.75),
])
def test_sqfree_fused_decode_matches_oracle(cuda, T, G, hd, sk_frac):
    """Register-resident kernel for the common slot shapes; the shared-memory
    kernel for the others (hd 32: one skeleton and one residual slot per lane)."""
    import torch
    H, L = 2, 2
    cache = SqfreeCache(hd, L, H, 1024, sk_frac=sk_frac)
    OL = O.sqfree_layout(hd, sk_k=cache.cc.sk_k)
    k, v = _inputs(5, L, H, T, hd)
    cache.write_kv_tokens(0, 0, torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda())
    q = synth.q_np(5, L, H * G, hd, 1.0 / np.sqrt(hd))
    out = torch.empty(L, H * G, hd, dtype=torch.float16, device="cuda")
    cache.attn_decode(0, L, torch.from_numpy(q).cuda(), T, out, logit_scale=0.9)
    torch.cuda.synchronize()
    ks, vs = cache.slab(0).cpu().numpy(), cache.slab(1).cpu().numpy()
    got = out.float().cpu().numpy()
    for layer in range(L):
        ref = O.sqfree_attn_decode(ks[layer * H:(layer + 1) * H], vs[layer * H:(layer + 1) * H], OL, OL,
                                   q[layer], T, 0.9)
        assert _rel_l2(got[layer], ref) <= RTOL_L2


@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
def test_hier_codes_and_reads_match_oracle(cuda, dtype, monkeypatch):
    """Slots bit-exact; batched reads within 1e-3 relative L2 on the
    tensor-core path (fp16 operands) and exact on the SIMT path."""
    import torch
    hd, L, H, T = 256, 2, 2, 96
    OL = O.hier_layout(hd)
    cache = HierCache(hd, L, H, T, OL.pd, OL.n_skel)
    k, v = _inputs(4, L, H, T, hd, sigma=1.0)
    tdt = getattr(torch, dtype)
    kt, vt = torch.from_numpy(k).to(tdt), torch.from_numpy(v).to(tdt)
    k32, v32 = kt.float().numpy(), vt.float().numpy()      # what the kernel sees
    Ws = np.stack([O.hier_fit_W(k32[layer, :, h], OL) for layer in range(L) for h in range(H)])
    cache.upload_W(Ws)
    cache.write_kv_tokens(0, 0, kt.cuda(), vt.cuda())
    torch.cuda.synchronize()
    ks, vs = cache.slab(0).cpu().numpy(), cache.slab(1).cpu().numpy()
    for layer in range(L):
        for h in range(H):
            s = layer * H + h
            assert np.array_equal(ks[s, :T], O.hier_write(k32[layer, :, h], OL, Ws[s])), (s, "K")
            assert np.array_equal(vs[s, :T], O.hier_write(v32[layer, :, h], OL, Ws[s])), (s, "V")
    assert cache.hc.d_recon, "tensor-core read expected for the hd-256 hier layout"
    for simt in (False, True):
        if simt:
            monkeypatch.setenv("SHANNON_PRIME_HIER_READ_SIMT", "1")
        ko = torch.empty(L, T, H, hd, device="cuda")
        vo = torch.empty_like(ko)
        cache.read_kv_tokens(0, 0, ko, vo)
        torch.cuda.synchronize()
        ko, vo = ko.cpu().numpy(), vo.cpu().numpy()
        for layer in range(L):
            for h in range(H):
                s = layer * H + h
                for got, slab in ((ko[layer, :, h], ks), (vo[layer, :, h], vs)):
                    ref = O.hier_read(slab[s, :T], OL, Ws[s])
                    if simt:
                        assert np.array_equal(got, ref)
                    else:
                        assert _rel_l2(got, ref) <= RTOL_L2, (s, _rel_l2(got, ref))


def test_hier_single_vector_api(cuda):
    import torch
    hd = 256
    OL = O.hier_layout(hd)
    cache = HierCache(hd, 1, 2, 8, OL.pd, OL.n_skel)
    k, _ = synth.kv_slot_np(8, 0, 1, 64, hd, 1.0)
    W = O.hier_fit_W(k, OL)
    cache.upload_W(np.stack([W, W]))
    L = spb200.lib()
    dk = torch.from_numpy(k[:3]).cuda()
    for pos in range(3):
        L.sp_cuda_hier_write_k(C.byref(cache.hc), 0, 1, pos, dk[pos].data_ptr())
    out = torch.empty(hd, device="cuda")
    L.sp_cuda_hier_read_k(C.byref(cache.hc), 0, 1, 2, out.data_ptr())
    torch.cuda.synchronize()
    packed = cache.slab(0).cpu().numpy()[1, :3]
    assert np.array_equal(packed, O.hier_write(k[:3], OL, W))
    assert np.array_equal(out.cpu().numpy(), O.hier_read(packed[2:3], OL, W)[0])

@pytest.mark.parametrize("T", [5, 64, 1001])
def test_sqfree_blocked_and_register_decodes_agree(cuda, T, monkeypatch):
    """The lane decode (one thread per slot, tensor-core contractions), the
    blocked decode (4-position bulk-copied blocks, balanced residual lanes)
    and the register kernel give the same attention, and the decodes leave
    their status word clear."""
    import torch
    H, L, G, hd = 2, 2, 4, 128
    cache = SqfreeCache(hd, L, H, 2048, sk_frac=0.75)
    assert 0 < cache.cc.lane_max_terms <= 8
    k, v = _inputs(9, L, H, T, hd)
    cache.write_kv_tokens(0, 0, torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda())
    q = torch.from_numpy(synth.q_np(9, L, H * G, hd, 1.0 / np.sqrt(hd))).cuda()
    outs = []
    for env in (None, "SHANNON_PRIME_SQFREE_DECODE_BLOCKED", "SHANNON_PRIME_SQFREE_DECODE_REG"):
        if env:
            monkeypatch.setenv(env, "1")
        out = torch.empty(L, H * G, hd, dtype=torch.float16, device="cuda")
        cache.attn_decode(0, L, q, T, out, logit_scale=0.7)
        torch.cuda.synchronize()
        outs.append(out.float().cpu().numpy())
    assert _rel_l2(outs[0], outs[2]) <= 1e-3
    assert _rel_l2(outs[1], outs[2]) <= 1e-3
    # status word: 4 bytes after the partials in the decode workspace
    cudart = C.CDLL("libcudart.so.12") if _has_lib("libcudart.so.12") else None
    if cudart is not None:
        word = C.c_uint32(7)
        src = C.c_void_p(cache.cc.d_attn_ws + cache.cc.attn_ws_bytes)
        assert cudart.cudaMemcpy(C.byref(word), src, C.c_size_t(4), 2) == 0   # device -> host
        assert word.value == 0


def _has_lib(name):
    try:
        C.CDLL(name)
        return True
    except OSError:
        return False


@pytest.mark.parametrize("start,T,dt", [(0, 64, "float32"), (3, 77, "float32"), (5, 40, "bfloat16"),
                                        (8, 33, "float16")])
def test_sqfree_lane_encoder_matches_warp_encoder(cuda, monkeypatch, start, T, dt):
    """The lane-per-vector sqfree encoder (config 2 layout) writes the same
    slots as the warp-per-vector encoder (SHANNON_PRIME_SQFREE_ENCODE_WARP)
    and as the oracle, at unaligned start positions, partial 32-position
    batches, half-precision inputs and edge values."""
    import torch
    L, H, hd = 2, 3, 128
    k, v = _inputs(7, L, H, T, hd, sigma=1.0)
    k[0, 0, 0] = 0.0                       # zero vector
    k[1, 1, 2] = 3e4                       # fp16 scale overflow
    v[0, 2, 1, :7] = 1e-30                 # tiny values
    tk = torch.from_numpy(k).to(getattr(torch, dt)).cuda()
    tv = torch.from_numpy(v).to(getattr(torch, dt)).cuda()
    slabs = []
    for warp_path in (False, True):
        if warp_path:
            monkeypatch.setenv("SHANNON_PRIME_SQFREE_ENCODE_WARP", "1")
        cache = SqfreeCache(hd, L, H, 128, sk_frac=0.75)
        cache.write_kv_tokens(0, start, tk, tv)
        torch.cuda.synchronize()
        slabs.append((cache.slab(0).cpu().numpy(), cache.slab(1).cpu().numpy()))
        monkeypatch.delenv("SHANNON_PRIME_SQFREE_ENCODE_WARP", raising=False)
    (kl, vl), (kw, vw) = slabs
    assert np.array_equal(kl, kw) and np.array_equal(vl, vw)
    OL = O.sqfree_layout(hd, sk_k=cache.cc.sk_k, residual_bits=3, use_spinor=True)
    k32, v32 = tk.float().cpu().numpy(), tv.float().cpu().numpy()
    for layer in range(L):
        for h in range(H):
            s = layer * H + h
            assert np.array_equal(kl[s, start:start + T], O.sqfree_write(k32[layer, :, h], OL))
            assert np.array_equal(vl[s, start:start + T], O.sqfree_write(v32[layer, :, h], OL))


@pytest.mark.parametrize("start,T", [(0, 96), (3, 77), (6, 1)])
def test_sqfree_lane_read_matches_warp_read(cuda, monkeypatch, start, T):
    """The lane-per-vector sqfree read (config 2 layout) returns the rows of
    the warp-per-vector read (SHANNON_PRIME_SQFREE_DECODE_WARP) and of the
    oracle, bit for bit."""
    import torch
    L, H, hd = 1, 2, 128
    k, v = _inputs(9, L, H, T, hd, sigma=1.0)
    cache = SqfreeCache(hd, L, H, 128, sk_frac=0.75)
    cache.write_kv_tokens(0, start, torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda())
    torch.cuda.synchronize()
    OL = O.sqfree_layout(hd, sk_k=cache.cc.sk_k, residual_bits=3, use_spinor=True)
    for which in (0, 1):
        outs = []
        for warp_path in (False, True):
            if warp_path:
                monkeypatch.setenv("SHANNON_PRIME_SQFREE_DECODE_WARP", "1")
            out = torch.full((T, hd), 5.0, device="cuda")
            cache.read_batch(which, 0, 1, start, out)
            torch.cuda.synchronize()
            outs.append(out.cpu().numpy())
            monkeypatch.delenv("SHANNON_PRIME_SQFREE_DECODE_WARP", raising=False)
        np.testing.assert_array_equal(outs[0], outs[1])
        slab = cache.slab(which).cpu().numpy()[1, start:start + T]
        np.testing.assert_array_equal(outs[0], O.sqfree_read(slab, OL))


@pytest.mark.parametrize("layer0,nl,start,T", [(0, 2, 0, 300), (1, 1, 5, 77)])
def test_sqfree_read_kv_tokens_matches_per_slot_reads(cuda, layer0, nl, start, T):
    """The token-major all-heads sqfree read (one launch over a layer range)
    puts every slot's rows at [layer][token][head], bit-identical with the
    per-slot batch read."""
    import torch
    L, H, hd = 2, 3, 128
    k, v = _inputs(11, L, H, 320, hd, sigma=1.0)
    cache = SqfreeCache(hd, L, H, 320, sk_frac=0.75)
    cache.write_kv_tokens(0, 0, torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda())
    torch.cuda.synchronize()
    for which in (0, 1):
        got = torch.full((nl, T, H, hd), 5.0, device="cuda")
        cache.read_kv_tokens(which, layer0, nl, start, got)
        ref = torch.full((nl, T, H, hd), 6.0, device="cuda")
        for l in range(nl):
            for h in range(H):
                one = torch.empty(T, hd, device="cuda")
                cache.read_batch(which, layer0 + l, h, start, one)
                ref[l, :, h] = one
        torch.cuda.synchronize()
        assert torch.equal(got, ref), which


@pytest.mark.parametrize("dtype", ["float32", "float16", "bfloat16"])
@pytest.mark.parametrize("start,T", [(0, 300), (5, 77), (13, 1)])
def test_hier_lane_and_warp_encoders_agree(cuda, dtype, start, T, monkeypatch):
    """The lane-per-vector hier writer (hd 256 layout) and the warp encoder
    write identical slots, also for ragged tiles at unaligned positions, and
    both equal the oracle."""
    import torch
    hd, L, H = 256, 2, 3
    OL = O.hier_layout(hd)
    k, _ = _inputs(6, L, H, T, hd, sigma=1.0)
    tdt = getattr(torch, dtype)
    kt = torch.from_numpy(k).to(tdt)
    k32 = kt.float().numpy()
    Ws = np.stack([O.hier_fit_W(np.concatenate([k32[layer, :, h]] * 4)[:max(64, T)], OL)
                   for layer in range(L) for h in range(H)])
    slabs = []
    for warp_enc in (False, True):
        if warp_enc:
            monkeypatch.setenv("SHANNON_PRIME_HIER_ENCODE_WARP", "1")
        cache = HierCache(hd, L, H, 512, OL.pd, OL.n_skel)
        cache.upload_W(Ws)
        cache.write_kv_tokens(0, start, kt.cuda(), None)
        torch.cuda.synchronize()
        slabs.append(cache.slab(0).cpu().numpy())
    assert np.array_equal(slabs[0], slabs[1])
    for layer in range(L):
        for h in range(H):
            s = layer * H + h
            assert np.array_equal(slabs[0][s, start:start + T], O.hier_write(k32[layer, :, h], OL, Ws[s]))
            assert not slabs[0][s, :start].any() and not slabs[0][s, start + T:].any()
