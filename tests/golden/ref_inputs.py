"""Seeded inputs of the reference-run fixtures (tests/golden/ref_*.npz).

Shared by tests/golden/make_ref_fixtures.py, which ran them through the
reference's own CUDA code (oracle/_ref) on a B200, and by the tests that
recompute the oracle's and this repo's outputs on the same inputs.  Every
input is rebuilt from seeds, so the fixtures hold only the reference's
outputs.
"""
from __future__ import annotations

import numpy as np

import oracle as O
from spb200 import synth

KB = [5, 5, 4, 3]
VB = [3]
SQ_BITS = [5, 4, 4, 4, 5]
SQ_RES_BITS = 3
HIER_BITS = [5, 5]
HIER_RES_BITS = 2


def ship_cfg0(n_pos: int = 4096, heads: int = 8):
    """Config 0: layer 0, KV heads 0..7, 4096 positions, seed 0 -> K, V
    [heads][n_pos][128] float32."""
    ks, vs = zip(*(synth.kv_slot_np(0, 0, h, n_pos, 128) for h in range(heads)))
    return np.stack(ks), np.stack(vs)


def ship_coeffs(x: np.ndarray, mobius: bool) -> np.ndarray:
    """The oracle's VHT2 (then Möbius order when mobius) of rows [...][n]."""
    c = O.vht2(x)
    return c[..., O.mobius_order(x.shape[-1])] if mobius else c


def edge_coeffs() -> np.ndarray:
    """[64][128] coefficient rows that exercise the quantiser's edges: zero
    rows, fp16-overflowing bands (inf scale -> zero codes), subnormal fp16
    scales, NaN, -0.0, exact half-step ties, values that clamp, one large
    coefficient per band, and alternating signs."""
    rng = np.random.default_rng(11)
    e = np.zeros((64, 128), np.float32)
    e[1] = 7.0e4                               # amax/m overflows fp16
    e[2, 5] = 1.0e6
    e[3] = np.linspace(-1e-6, 1e-6, 128)       # subnormal scales
    e[4] = np.linspace(-3e-8, 3e-8, 128)
    e[5, 40] = np.nan
    e[6] = -0.0
    e[7, ::2] = 1.0
    e[7, 1::2] = -1.0
    for r in range(8, 24):                     # ties: band amax = m*s, x = (k+1/2)*s
        s = np.float32(2.0 ** rng.integers(-6, 3))
        for b, bits in enumerate(KB):
            m = 2 ** (bits - 1) - 1
            seg = slice(32 * b, 32 * b + 32)
            k = rng.integers(-m, m, 32).astype(np.float32)
            e[r, seg] = (k + np.float32(0.5)) * s
            e[r, 32 * b] = m * s
    for r in range(24, 32):                    # one large coefficient per band
        e[r] = rng.standard_normal(128).astype(np.float32) * 1e-3
        e[r, ::32] = rng.standard_normal(4).astype(np.float32) * 50
    e[32:] = rng.standard_normal((32, 128)).astype(np.float32) * \
        np.float32(10.0) ** rng.integers(-5, 5, (32, 1)).astype(np.float32)
    return e


def _pad_rows(x: np.ndarray, pd: int) -> np.ndarray:
    hd = x.shape[1]
    out = np.empty((x.shape[0], pd), np.float32)
    out[:, :hd] = x
    for i, row in enumerate(np.ascontiguousarray(x, np.float32)):
        out[i, hd:] = O.lib().or_lane_tree_sum(row.ctypes.data, hd) / np.float32(hd)
    return out


def sqfree_stages(n: int = 2048):
    """Config 2 layout (hd 128 -> pad 154, sk_frac 0.75 -> 115 skeleton,
    39 residuals, spinor on): skeleton, actual residual coefficients and the
    oracle's prediction for n K vectors of seed 2 (layer 0, head 0)."""
    L = O.sqfree_layout(128, bits=SQ_BITS, residual_bits=SQ_RES_BITS, use_spinor=True,
                        sk_frac=0.75)
    k, _ = synth.kv_slot_np(2, 0, 0, n, 128)
    c = O.vilenkin(_pad_rows(k, L.pd))
    sk = c[:, list(L.skel_idx)[:L.sk_k]]
    act = c[:, list(L.res_idx)[:L.n_res]]
    csr = (np.array(L.csr_off[:L.n_res + 1], np.int32),
           np.array(L.csr_slot[:L.n_terms], np.int32),
           np.array(L.csr_sign[:L.n_terms], np.int32))
    return L, sk, act, csr


def hier_stages(n: int = 2048, n_calib: int = 512):
    """Config 4 layout (hd 256 -> pad 330, skeleton 30, 300 targets, 2-bit
    residuals): W fitted on n_calib K vectors, then the skeleton and target
    coefficients of n further K vectors of seed 4 (layer 0, head 0)."""
    L = O.hier_layout(256, bits=HIER_BITS, residual_bits=HIER_RES_BITS)
    k, _ = synth.kv_slot_np(4, 0, 0, n_calib + n, 256, sigma=1.0)
    W = O.hier_fit_W(k[:n_calib], L)
    c = O.vilenkin(_pad_rows(k[n_calib:], L.pd))
    return L, W, c[:, :L.n_skel], c[:, L.n_skel:]


def residual_ties(n_res: int, bits: int, form: str, n: int = 64):
    """Deviation rows on a half-level grid (k + 1/2 steps of a power-of-two
    step), which puts many scaled values on or next to rounding boundaries,
    plus rows with one outlier that saturates the clamp."""
    rng = np.random.default_rng(5)
    Lv = 1 << bits
    d = np.zeros((n, n_res), np.float32)
    for r in range(n):
        step = np.float32(2.0 ** rng.integers(-4, 2))
        k = rng.integers(0, Lv - 1, n_res).astype(np.float32)
        d[r] = (k + np.float32(0.5) - np.float32(0.5 * (Lv - 1))) * step
        if r % 4 == 3:
            d[r, 0] = step * 40
    return d


def cuda_form_vht2(x: np.ndarray) -> np.ndarray:
    """The reference CUDA backend's VHT2 (kernel_vht2_p2,
    shannon_prime_cuda.cu:37-75) restated in float32 numpy: ascending
    butterfly lengths, each stage (u+v)*c and (u-v)*c with c the float32
    nearest 1/sqrt(2).  The oracle and this repo follow the CPU core's form
    (unnormalised butterfly, then one multiply by 1/sqrt(n)); the two forms
    differ in the last bits of some coefficients."""
    y = np.array(x, np.float32, copy=True)
    n = y.shape[-1]
    c = np.float32(0.70710678118654752440)
    ln = 1
    while ln < n:
        y = y.reshape(*y.shape[:-1], n // (2 * ln), 2, ln)
        u = y[..., 0, :].copy()
        v = y[..., 1, :].copy()
        y[..., 0, :] = (u + v) * c
        y[..., 1, :] = (u - v) * c
        y = y.reshape(*y.shape[:-3], n)
        ln *= 2
    return y
