"""CPU tests of the sqfree+spinor and hierarchical-Vilenkin restatement in
the oracle: pad dimensions, the staged transform against an independent
float64 Kronecker-product Hartley matrix, the Knight mask and Möbius CSR
against a direct restatement, slot sizes, the lane-tree reduction order, and
round-trip quality."""
import math
import sys
from pathlib import Path

import numpy as np
import pytest

import oracle as O
from spb200 import synth


def _squarefree(m):
    return all(m % (p * p) for p in range(2, int(math.isqrt(m)) + 1))


def _mu(m):
    k = 0
    p = 2
    while p * p <= m:
        if m % p == 0:
            m //= p
            if m % p == 0:
                return 0
            k += 1
        p += 1
    if m > 1:
        k += 1
    return -1 if k % 2 else 1


@pytest.mark.parametrize("hd,pd", [(32, 33), (64, 66), (128, 154), (256, 330)])
def test_pad_dim_is_smallest_squarefree_11_smooth(hd, pd):
    assert O.lib().or_sqfree_pad_dim(hd) == pd          # 66/154/330: patches/README.md:105
    for m in range(hd, pd):
        r = m
        for p in (2, 3, 5, 7, 11):
            while r % p == 0:
                r //= p
        assert not (_squarefree(m) and r == 1)


@pytest.mark.parametrize("pd", [33, 66, 154, 330])
def test_vilenkin_matches_kronecker_hartley_and_is_self_inverse(pd):
    fac = []
    r = pd
    for p in (2, 3, 5, 7, 11):
        while r % p == 0:
            fac.append(p)
            r //= p
    # x index = d0 + p0*(d1 + p1*(...)): stage k acts on digit k
    M = np.array([[1.0]])
    for p in fac:
        k = np.arange(p)
        Hp = (np.cos(2 * np.pi * np.outer(k, k) / p) + np.sin(2 * np.pi * np.outer(k, k) / p)) / np.sqrt(p)
        M = np.kron(Hp, M)
    rng = np.random.default_rng(pd)
    x = rng.standard_normal((6, pd)).astype(np.float32)
    y = O.vilenkin(x)
    ref = x.astype(np.float64) @ M.T
    assert np.abs(y - ref).max() < 2e-5
    assert np.abs(O.vilenkin(y) - x).max() < 2e-5


def test_knight_mask_and_csr_restated_directly():
    L = O.sqfree_layout(128, sk_frac=0.75)
    pd, sk = L.pd, L.sk_k
    assert (pd, sk, L.n_res) == (154, 115, 39)
    rank = [i for i in range(pd) if _squarefree(i + 1)] + [i for i in range(pd) if not _squarefree(i + 1)]
    skel = list(L.skel_idx)[:sk]
    res = list(L.res_idx)[:L.n_res]
    assert skel == rank[:sk]
    assert res == sorted(set(range(pd)) - set(skel))
    slot = {i: s for s, i in enumerate(skel)}
    t = 0
    for r, i in enumerate(res):
        n = i + 1
        want = [(slot[d - 1], _mu(n // d)) for d in range(1, n) if n % d == 0 and _mu(n // d) and (d - 1) in slot]
        got = [(L.csr_slot[k], L.csr_sign[k]) for k in range(L.csr_off[r], L.csr_off[r + 1])]
        assert got == want
        t += len(want)
    assert t == L.n_terms


def test_slot_sizes():
    # sqfree+spinor at hd 128, sk_frac 0.75, bands 5,4,4,4,5, 3 residual bits:
    # 76 B skeleton + 4 B magnitude + 15 B levels + 5 B sheet = 100 B
    L = O.sqfree_layout(128, sk_frac=0.75)
    assert (L.bands.total_bytes, L.res_bytes, L.sheet_bytes, L.bytes_per_pos) == (76, 15, 5, 100)
    # reference CUDA default: skeleton pad_dim / 2 (shannon_prime_sqfree.cu:606)
    assert O.sqfree_layout(128).sk_k == 77
    # hier at hd 256: pad 330, skeleton 330/11 = 30 (bands 5,5), 300 targets at 2 bits
    H = O.hier_layout(256)
    assert (H.pd, H.n_skel, H.n_target, H.bytes_per_pos) == (330, 30, 300, 103)


def test_lane_tree_sum_order():
    rng = np.random.default_rng(3)
    for n in (1, 31, 39, 128, 300):
        v = (rng.standard_normal(n) * 10.0 ** rng.integers(-3, 4, n)).astype(np.float32)
        s = np.zeros(32, np.float32)
        for lane in range(32):
            acc = np.float32(0)
            for i in range(lane, n, 32):
                acc = np.float32(acc + v[i])
            s[lane] = acc
        for off in (16, 8, 4, 2, 1):
            s = np.array([np.float32(s[l] + s[l ^ off]) for l in range(32)], np.float32)
        assert np.float32(O.lib().or_lane_tree_sum(v.ctypes.data, n)) == s[0]


def test_sqfree_round_trip_quality_and_spinor():
    k, v = synth.kv_slot_np(2, 0, 0, 1024, 128)
    for use_spinor in (True, False):
        L = O.sqfree_layout(128, sk_frac=0.75, use_spinor=use_spinor)
        kr = O.sqfree_read(O.sqfree_write(k, L), L)
        vr = O.sqfree_read(O.sqfree_write(v, L), L)
        floor = 0.98 if use_spinor else 0.97
        assert O.mean_vector_correlation(k, kr) > floor
        assert O.mean_vector_correlation(v, vr) > floor
    # the sheet bit picks the smaller deviation, so the stored magnitudes
    # with the spinor are never larger than without it
    Ls, Ln = O.sqfree_layout(128, sk_frac=0.75), O.sqfree_layout(128, sk_frac=0.75, use_spinor=False)
    ms = O.sqfree_write(k[:64], Ls)[:, 76:80].copy().view(np.float32)
    mn = O.sqfree_write(k[:64], Ln)[:, 76:80].copy().view(np.float32)
    assert np.all(ms <= mn)


def test_hier_round_trip_with_fitted_predictor():
    k, _ = synth.kv_slot_np(4, 0, 0, 3072, 256, sigma=1.0)
    H = O.hier_layout(256)
    W = O.hier_fit_W(k[:2048], H)
    kr = O.hier_read(O.hier_write(k[2048:], H, W), H, W)
    assert O.mean_vector_correlation(k[2048:], kr) > 0.9


def test_hier_prediction_order_changes_slot_bytes():
    """Why the hier encoder keeps the W . skeleton product as the oracle's
    sequential fp32 fma chain instead of a tensor-core product: a prediction
    summed in another order, even an exactly rounded one from split fp16
    operands (what two tensor-core passes would at best give), leaves the
    residual levels alone on these inputs but changes the stored fp32
    magnitude (mean |deviation|, 4 bytes of the slot) of a large share of
    vectors, so the slots would no longer be byte-identical."""
    sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
    import ref_inputs as RI
    L, W, sk, tgt = RI.hier_stages(n=1024)
    p_seq = O.hier_predict(L, W, sk)
    hi = sk.astype(np.float16).astype(np.float64)
    lo = (sk.astype(np.float64) - hi).astype(np.float16).astype(np.float64)
    p_tc = ((hi + lo) @ W.astype(np.float64).T).astype(np.float32)
    d0, d1 = tgt - p_seq, tgt - p_tc
    m0, m1 = O.residual_mag(d0), O.residual_mag(d1)
    l0 = O.residual_levels(d0, 2, m0, "hier")
    l1 = O.residual_levels(d1, 2, m1, "hier")
    assert np.mean(p_seq != p_tc) > 0.5
    assert np.count_nonzero(l0 != l1) <= 1e-5 * l0.size
    assert np.mean(m0 != m1) > 0.05
