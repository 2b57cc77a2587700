"""GPU parity at the benchmark configurations' full sizes, through
size-independent properties (the CPU oracle only sees sampled slots):

- config 1 (32 layers x 8 KV heads x 32768 positions, 1.06 GB cache): the
  tensor-core decode against the independent SIMT decode, the oracle's
  attention on sampled heads over all 32768 positions, sampled slots' packed
  codes bit-exact with the oracle's writer, and a repeated decode bit-identical;
- config 3 shape, one layer (4 KV heads x 131072 positions, 8 query heads per
  KV head): tensor-core against SIMT decode and one oracle head;
- config 2 (sqfree, 16384 positions): blocked against register decode, a
  sampled slot's bytes bit-exact with the oracle's writer and a sampled
  head's decode against the oracle's attention over all 16384 positions;
- config 4 (hier, 8192 positions x 16 heads): tensor-core batched read against
  the exact SIMT read, a sampled slot's bytes bit-exact with the oracle's
  writer and its tensor-core read against the oracle's read.

Tolerance: relative L2 <= 1e-3 per output, as in the small-size tests."""
import numpy as np
import pytest

import oracle as O
import spb200
from spb200 import synth

pytestmark = pytest.mark.gpu
KB, VB = [5, 5, 4, 3], [3]
RTOL = 1e-3


def _rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _decode(torch, cache, q, kv_len, impl, scale=1.0):
    out = torch.empty(q.shape, dtype=torch.float16, device="cuda")
    spb200.lib().sp_cuda_attn_force_impl(impl)
    try:
        cache.attn_decode(0, q.shape[0], q, kv_len, out, logit_scale=scale)
        torch.cuda.synchronize()
    finally:
        spb200.lib().sp_cuda_attn_force_impl(0)
    return out


def test_config1_full_size(cuda):
    import torch
    L, H, G, T, n = 32, 8, 4, 32768, 128
    cache = spb200.Cache(n, L, H, T, KB, VB, True)
    gen = torch.Generator(device="cuda")
    sample_k = {}
    for layer in range(L):
        gen.manual_seed(1 * 1000003 + layer)
        k, v = synth.kv_layer_torch(gen, T, H, n)
        cache.write_kv_tokens(layer, 0, k, v)
        if layer in (0, 31):
            sample_k[layer] = (k[:, 5].cpu().numpy(), v[:, 5].cpu().numpy())
    torch.cuda.synchronize()
    gq = torch.Generator(device="cuda")
    gq.manual_seed(1)
    q = (torch.randn(L, H * G, n, device="cuda", generator=gq) / n ** 0.5).half()
    mma = _decode(torch, cache, q, T, 2)
    simt = _decode(torch, cache, q, T, 1)
    again = _decode(torch, cache, q, T, 2)
    assert torch.equal(mma, again)                      # deterministic
    tc = _decode(torch, cache, q, T, 3)
    assert torch.equal(tc, _decode(torch, cache, q, T, 3))
    a, b, c = mma.float().cpu().numpy(), simt.float().cpu().numpy(), tc.float().cpu().numpy()
    for layer in range(L):
        assert _rel(a[layer], b[layer]) <= RTOL, layer
        assert _rel(c[layer], b[layer]) <= RTOL, layer
    ks, vs = cache.slab(0), cache.slab(1)
    qn = q.cpu().numpy()
    for layer, h in ((0, 5), (31, 5), (17, 2)):
        slot = layer * H + h
        ref = O.attn_decode(ks[slot:slot + 1].cpu().numpy(), vs[slot:slot + 1].cpu().numpy(), n, KB, VB, True,
                            qn[layer, h * G:(h + 1) * G], T, 1.0)
        assert _rel(a[layer, h * G:(h + 1) * G], ref) <= RTOL, (layer, h)
        assert _rel(c[layer, h * G:(h + 1) * G], ref) <= RTOL, (layer, h)
    for layer, (kx, vx) in sample_k.items():
        slot = layer * H + 5
        assert np.array_equal(ks[slot].cpu().numpy(), O.ship_write(kx, KB, True))
        assert np.array_equal(vs[slot].cpu().numpy(), O.ship_write(vx, VB, False))


def test_config3_shape_one_layer(cuda):
    import torch
    H, G, T, n = 4, 8, 131072, 128
    cache = spb200.Cache(n, 1, H, T, KB, VB, True)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(3 * 1000003)
    k, v = synth.kv_layer_torch(gen, T, H, n)
    cache.write_kv_tokens(0, 0, k, v)
    del k, v
    gq = torch.Generator(device="cuda")
    gq.manual_seed(3)
    q = torch.randn(1, H * G, n, device="cuda", generator=gq).half()
    scale = 1.0 / n ** 0.5
    a = _decode(torch, cache, q, T, 2, scale).float().cpu().numpy()
    b = _decode(torch, cache, q, T, 1, scale).float().cpu().numpy()
    c = _decode(torch, cache, q, T, 3, scale).float().cpu().numpy()
    assert _rel(a, b) <= RTOL
    assert _rel(c, b) <= RTOL
    h = 3
    ref = O.attn_decode(cache.slab(0)[h:h + 1].cpu().numpy(), cache.slab(1)[h:h + 1].cpu().numpy(), n, KB, VB,
                        True, q.cpu().numpy()[0, h * G:(h + 1) * G], T, scale)
    assert _rel(a[0, h * G:(h + 1) * G], ref) <= RTOL
    assert _rel(c[0, h * G:(h + 1) * G], ref) <= RTOL


def test_config2_sqfree_full_length(cuda, monkeypatch):
    import torch
    from spb200.sqfree import SqfreeCache
    L, H, G, T, n = 2, 8, 4, 16384, 128
    cache = SqfreeCache(n, L, H, T, sk_frac=0.75)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(2)
    kept = None
    for layer in range(L):
        k, v = synth.kv_layer_torch(gen, T, H, n)
        cache.write_kv_tokens(layer, 0, k.unsqueeze(0), v.unsqueeze(0))
        if layer == 1:
            kept = (k[:, 3].cpu().numpy(), v[:, 3].cpu().numpy())
    q = torch.from_numpy(synth.q_np(2, L, H * G, n, 1.0 / np.sqrt(n))).cuda()
    outs = []
    for reg in (False, True):
        if reg:
            monkeypatch.setenv("SHANNON_PRIME_SQFREE_DECODE_REG", "1")
        out = torch.empty(L, H * G, n, dtype=torch.float16, device="cuda")
        cache.attn_decode(0, L, q, T, out)
        torch.cuda.synchronize()
        outs.append(out.float().cpu().numpy())
    for layer in range(L):
        assert _rel(outs[0][layer], outs[1][layer]) <= RTOL
    OL = O.sqfree_layout(n, sk_k=cache.cc.sk_k)
    ks, vs = cache.slab(0).cpu().numpy(), cache.slab(1).cpu().numpy()
    slot = 1 * H + 3
    assert np.array_equal(ks[slot, :T], O.sqfree_write(kept[0], OL))
    assert np.array_equal(vs[slot, :T], O.sqfree_write(kept[1], OL))
    h = 3
    ref = O.sqfree_attn_decode(ks[slot:slot + 1], vs[slot:slot + 1], OL, OL,
                               q.cpu().numpy()[1, h * G:(h + 1) * G], T, 1.0)
    assert _rel(outs[0][1, h * G:(h + 1) * G], ref) <= RTOL


def test_config4_hier_full_length(cuda, monkeypatch):
    import torch
    from spb200.sqfree import HierCache
    hd, H, T = 256, 16, 8192
    OL = O.hier_layout(hd)
    cache = HierCache(hd, 1, H, T, OL.pd, OL.n_skel)
    assert cache.hc.d_recon
    rng = np.random.default_rng(4)
    W = (rng.standard_normal((H, OL.pd - OL.n_skel, OL.n_skel)) * 0.05).astype(np.float16)
    cache.upload_W(W)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(4)
    k, v = synth.kv_layer_torch(gen, T, H, hd, sigma=1.0, dtype=torch.bfloat16)
    cache.write_kv_tokens(0, 0, k.unsqueeze(0), v.unsqueeze(0))
    outs = []
    # tcgen05 read (default), mma.sync read, exact SIMT read
    for env in (None, "SHANNON_PRIME_HIER_READ_MMA_SYNC", "SHANNON_PRIME_HIER_READ_SIMT"):
        if env:
            monkeypatch.setenv(env, "1")
        ko = torch.empty(1, T, H, hd, device="cuda")
        cache.read_kv_tokens(0, 0, ko, None)
        torch.cuda.synchronize()
        outs.append(ko.cpu().numpy())
    for h in range(H):
        assert _rel(outs[0][0, :, h], outs[2][0, :, h]) <= RTOL, h
        assert _rel(outs[1][0, :, h], outs[2][0, :, h]) <= RTOL, h
    outs.pop(1)
    h = 7
    kh = k[:, h].float().cpu().numpy()
    packed = cache.slab(0).cpu().numpy()[h, :T]
    assert np.array_equal(packed, O.hier_write(kh, OL, W[h]))
    ref = O.hier_read(packed, OL, W[h])
    assert _rel(outs[0][0, :, h], ref) <= RTOL
