"""CPU tests of the oracle: fp16 rounding, band layout, VHT2, Möbius order,
quantiser, and the reference's surviving known answers (byte counts,
correlation thresholds, compression ratio)."""
import math

import numpy as np
import pytest

import oracle as O
from spb200 import synth


def test_f16_rounding_matches_numpy():
    rng = np.random.default_rng(0)
    vals = np.concatenate([
        rng.standard_normal(20000).astype(np.float32) * 10.0 ** rng.integers(-9, 6, 20000),
        np.array([0.0, -0.0, 65504.0, 65519.0, 65520.0, 1e9, -1e9, 6e-8, 5.96e-8, 2.98e-8,
                  2.99e-8, 6.1e-5, 6.104e-5, np.inf, -np.inf], dtype=np.float32),
    ]).astype(np.float32)
    ours = np.array([O.f32_to_f16(float(v)) for v in vals], dtype=np.uint16)
    ref = vals.astype(np.float16).view(np.uint16)
    assert np.array_equal(ours, ref)
    L = O.lib()
    for h in range(0, 65536, 7):
        f = np.array([h], dtype=np.uint16).view(np.float16).astype(np.float32)[0]
        g = L.or_f16_to_f32(h)
        assert (math.isnan(f) and math.isnan(g)) or f == g


@pytest.mark.parametrize("n,kbits,vbits,kb,vb", [
    (128, [5, 5, 4, 3], [3], 76, 50),     # shannon_prime_vulkan.c:99-105; test_adreno_phone.log:10
    (64, [5, 4, 4], [3], 42, 26),         # shannon_prime_llama.h:336-338
])
def test_packed_byte_counts(n, kbits, vbits, kb, vb):
    assert O.bands(n, kbits).total_bytes == kb
    assert O.bands(n, vbits).total_bytes == vb


def test_band_spans_last_band_takes_remainder():
    b = O.bands(128, [5, 5, 4, 3, 3, 3, 2, 2, 2, 2])
    assert list(b.off)[:10] == [12 * i for i in range(10)]
    assert list(b.size)[:10] == [12] * 9 + [20]


def _vht2_numpy(x):
    """The same butterfly in numpy float32 (independent restatement)."""
    x = x.astype(np.float32).copy()
    n = x.shape[-1]
    length = 1
    while length < n:
        y = x.reshape(*x.shape[:-1], n // (2 * length), 2, length)
        u, v = y[..., 0, :].copy(), y[..., 1, :].copy()
        y[..., 0, :] = u + v
        y[..., 1, :] = u - v
        x = y.reshape(*x.shape)
        length *= 2
    return (x * np.float32(1.0 / np.sqrt(np.float32(n), dtype=np.float32))).astype(np.float32)


@pytest.mark.parametrize("n", [32, 64, 128, 256])
def test_vht2_bit_exact_and_self_inverse(n):
    rng = np.random.default_rng(n)
    x = rng.standard_normal((50, n)).astype(np.float32)
    y = O.vht2(x)
    assert np.array_equal(y.view(np.uint32), _vht2_numpy(x).view(np.uint32))
    # orthonormal Hadamard (Sylvester order)
    H = np.array([[1.0]])
    while H.shape[0] < n:
        H = np.block([[H, H], [H, -H]])
    np.testing.assert_allclose(y, x @ H.T / math.sqrt(n), rtol=1e-4, atol=1e-5)
    np.testing.assert_allclose(O.vht2(y), x, rtol=1e-4, atol=1e-5)


def test_mobius_order_squarefree_first():
    o = O.mobius_order(128)
    assert sorted(o.tolist()) == list(range(128))

    def sqf(m):
        return all(m % (p * p) for p in range(2, int(m ** 0.5) + 1))
    n_sqf = sum(sqf(i + 1) for i in range(128))
    assert all(sqf(i + 1) for i in o[:n_sqf]) and not any(sqf(i + 1) for i in o[n_sqf:])
    assert list(o[:n_sqf]) == sorted(o[:n_sqf]) and list(o[n_sqf:]) == sorted(o[n_sqf:])


def _quantize_py(x, bits_list, n):
    """Pure-Python restatement of kernel_band_quantize_simple
    (shannon_prime_cuda.cu:131-204) for small cases."""
    out = []
    bs = n // len(bits_list)
    for b, bits in enumerate(bits_list):
        off = b * bs
        sz = n - off if b == len(bits_list) - 1 else bs
        band = x[off:off + sz]
        mv = (1 << (bits - 1)) - 1
        amax = np.float32(0)
        for v in band:
            a = np.float32(abs(v))
            if a > amax:
                amax = a
        scale = np.float32(amax / np.float32(mv)) if amax > 0 else np.float32(0)
        h = np.float16(scale)
        out += list(h.view(np.uint16).tobytes())
        stored = np.float32(h)
        inv = np.float32(np.float32(1) / stored) if stored > 0 else np.float32(0)
        acc, nb = 0, 0
        for v in band:
            q = int(np.rint(np.float32(v * inv)))
            q = max(-mv, min(mv, q))
            acc |= (q + mv) << nb
            nb += bits
            while nb >= 8:
                out.append(acc & 0xFF)
                acc >>= 8
                nb -= 8
        if nb:
            out.append(acc & 0xFF)
    return np.array(out, dtype=np.uint8)


@pytest.mark.parametrize("bits", [[5, 5, 4, 3], [3], [5, 4, 4], [8, 6, 2, 1, 7]])
def test_quantizer_matches_python_restatement(bits):
    rng = np.random.default_rng(len(bits))
    n = 64
    x = (rng.standard_normal((20, n)) * rng.lognormal(0, 1, (20, 1))).astype(np.float32)
    x[3, :] = 0.0                                  # all-zero vector
    x[4, 5] = 3.0 * np.float32(0.5)                # exact ties exercise RNE
    got = O.band_quantize(x, bits)
    for i in range(x.shape[0]):
        assert np.array_equal(got[i], _quantize_py(x[i], bits, n)), i


def test_dequantize_error_bound_and_partial():
    rng = np.random.default_rng(3)
    bits = [5, 5, 4, 3]
    x = rng.standard_normal((100, 128)).astype(np.float32)
    p = O.band_quantize(x, bits)
    y = O.band_dequantize(p, 128, bits)
    for b in range(4):
        sl = slice(32 * b, 32 * b + 32)
        mv = (1 << (bits[b] - 1)) - 1
        scale = np.abs(x[:, sl]).max(1, keepdims=True) / mv
        assert np.all(np.abs(y[:, sl] - x[:, sl]) <= scale * 0.5 * 1.01 + 1e-6)
    y2 = O.band_dequantize(p, 128, bits, max_bands=2)
    assert np.array_equal(y2[:, :64], y[:, :64]) and not y2[:, 64:].any()
    assert not O.band_dequantize(p, 128, bits, max_bands=0).any()


def test_nonfinite_scale_reads_as_zero():
    bits = [5, 5, 4, 3]
    p = O.band_quantize(np.ones((1, 128), np.float32), bits)
    p[0, 0:2] = np.frombuffer(np.float16(np.inf).tobytes(), np.uint8)
    y = O.band_dequantize(p, 128, bits)
    assert not y[0, :32].any() and np.all(y[0, 32:] != 0)


def test_ship_round_trip_known_answer_correlations():
    """Reference thresholds at hd 128: K > 0.985 (observed 0.9897), V > 0.950
    (observed 0.9702) (android_build/test_adreno_phone.log:50-51)."""
    ks, vs = [], []
    for h in range(8):
        k, v = synth.kv_slot_np(0, 0, h, 512, 128)
        ks.append(k)
        vs.append(v)
    k = np.concatenate(ks)
    v = np.concatenate(vs)
    kr = O.ship_read(O.ship_write(k, [5, 5, 4, 3], True), 128, [5, 5, 4, 3], True)
    vr = O.ship_read(O.ship_write(v, [3], False), 128, [3], False)
    ck = O.mean_vector_correlation(k, kr)
    cv = O.mean_vector_correlation(v, vr)
    assert ck > 0.985, ck
    assert cv > 0.950, cv


def test_compression_ratio_formula():
    """sp_llama_memory (shannon_prime_llama.c:901-905): fp16 K+V over packed."""
    kb, vb = O.bands(128, [5, 5, 4, 3]).total_bytes, O.bands(128, [3]).total_bytes
    assert abs(128 * 2 * 2 / (kb + vb) - 4.063) < 1e-3


def test_attention_oracle_matches_numpy():
    rng = np.random.default_rng(7)
    H, G, T, n = 2, 4, 200, 128
    kb, vb = [5, 5, 4, 3], [3]
    k = rng.standard_normal((H, T, n)).astype(np.float32)
    v = rng.standard_normal((H, T, n)).astype(np.float32)
    kp = O.ship_write(k.reshape(-1, n), kb, True).reshape(H, T, -1)
    vp = O.ship_write(v.reshape(-1, n), vb, False).reshape(H, T, -1)
    q = (rng.standard_normal((H * G, n)) * 0.1).astype(np.float16)
    out = O.attn_decode(kp, vp, n, kb, vb, True, q, T, 0.5)
    kh = O.ship_read(kp.reshape(-1, kp.shape[-1]), n, kb, True).reshape(H, T, n).astype(np.float64)
    vh = O.ship_read(vp.reshape(-1, vp.shape[-1]), n, vb, False).reshape(H, T, n).astype(np.float64)
    for g in range(H * G):
        h = g // G
        s = 0.5 * (kh[h] @ q[g].astype(np.float64))
        p = np.exp(s - s.max())
        p /= p.sum()
        np.testing.assert_allclose(out[g], p @ vh[h], rtol=1e-5, atol=1e-6)
