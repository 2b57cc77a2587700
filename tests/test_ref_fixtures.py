"""The oracle against outputs that the reference's own CUDA code computed.

tests/golden/ref_*.npz were written by tests/golden/make_ref_fixtures.py,
which ran the reference sources src/backends/cuda/shannon_prime_{cuda,sqfree,
hier}.cu, compiled unmodified (oracle/ref/Makefile), on a B200.  Each check
rebuilds the reference's full output from the oracle's plus the stored rows
where the two differ, and verifies it against the stored SHA-256, so the
whole output is pinned, not only the stored rows.
"""
import hashlib
import json
import sys
from pathlib import Path

import numpy as np
import pytest

GOLD = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(GOLD))

import oracle as O  # noqa: E402
import ref_inputs as RI  # noqa: E402


def _load(name):
    return np.load(GOLD / name)


def _rebuild(f, name, ours):
    """The reference's output: ours with the reference's differing rows
    substituted; checked against the stored hash."""
    r = np.ascontiguousarray(ours).reshape(-1, ours.shape[-1]).copy()
    idx = f[f"{name}_diff_idx"]
    r[idx] = f[f"{name}_diff_rows"]
    assert hashlib.sha256(r.tobytes()).hexdigest() == str(f[f"{name}_sha"]), name
    np.testing.assert_array_equal(r[:len(f[f"{name}_head"])], f[f"{name}_head"])
    return r, idx


@pytest.fixture(scope="module")
def cfg0():
    return RI.ship_cfg0()


def test_band_quantizer_bit_exact_with_reference_run(cfg0):
    """sp_cuda_band_quantize (shannon_prime_cuda.cu:131-204, 352-379) on the
    oracle's config-0 coefficients (8 heads x 4096 positions, K and V) and on
    edge rows (zeros, fp16 overflow, subnormal scales, NaN, -0, ties):
    byte-for-byte equal to the oracle's quantiser."""
    K, V = cfg0
    f = _load("ref_ship_cfg0.npz")
    for name, c, bits in (("qk", RI.ship_coeffs(K, True), RI.KB),
                          ("qv", RI.ship_coeffs(V, False), RI.VB),
                          ("qedge", RI.edge_coeffs(), RI.KB),
                          ("qedgev", RI.edge_coeffs(), RI.VB)):
        c = c.reshape(-1, 128)
        _, idx = _rebuild(f, name, O.band_quantize(c, bits))
        assert idx.size == 0, (name, idx[:10])
    # the reference's dequantiser of its own edge rows (non-finite scale -> 0)
    q = O.band_quantize(RI.edge_coeffs(), RI.KB)
    np.testing.assert_array_equal(f["qedge_deq"], O.band_dequantize(q, 128, RI.KB))


def test_reference_write_explained_by_its_vht2_form(cfg0):
    """The reference's whole CUDA write (sp_cuda_write_{k,v}_batch) equals
    the oracle's quantiser applied to the CUDA-form VHT2 (per-stage 1/sqrt 2)
    bit for bit.  The oracle's own write (the CPU core's single 1/sqrt(n)
    scale) differs from it only in bands whose max|x|/m lies within a few
    float32 ulps of an fp16 rounding midpoint (the stored scale rounds to
    the neighbouring fp16 value and the band re-quantises), and at single
    codes whose scaled value x/scale lies within 1e-5 of a half-integer."""
    K, V = cfg0
    f = _load("ref_ship_cfg0.npz")
    order = O.mobius_order(128)
    summary = json.loads((GOLD / "ref_summary.json").read_text())
    for name, X, bits, mob in (("wk", K, RI.KB, True), ("wv", V, RI.VB, False)):
        X = X.reshape(-1, 128)
        ours = O.ship_write(X, bits, mob)
        ref, idx = _rebuild(f, name, ours)
        c_cuda = RI.cuda_form_vht2(X)
        c_cuda = c_cuda[:, order] if mob else c_cuda
        np.testing.assert_array_equal(O.band_quantize(c_cuda, bits), ref)
        c_core = O.vht2(X)
        c_core = c_core[:, order] if mob else c_core
        bc = O.bands(128, bits)
        n_bands_diff = n_code_bands = 0
        for bi in range(bc.n_bands):
            o, lo, sz = bc.byte_off[bi], bc.off[bi], bc.size[bi]
            nb = 2 + (sz * bits[bi] + 7) // 8
            band_diff = np.any(ours[idx, o:o + nb] != ref[idx, o:o + nb], axis=1)
            scale_diff = np.any(ours[idx, o:o + 2] != ref[idx, o:o + 2], axis=1)
            code_rows = idx[band_diff & ~scale_diff]
            if code_rows.size:
                a = O.band_dequantize(ours[code_rows], 128, bits)[:, lo:lo + sz]
                b = O.band_dequantize(ref[code_rows], 128, bits)[:, lo:lo + sz]
                sc = ours[code_rows, o:o + 2].copy().view(np.float16).astype(np.float64)
                x = c_core[code_rows, lo:lo + sz].astype(np.float64) / sc
                fl = a != b
                assert fl.any()
                frac = np.abs(np.abs(x[fl] - np.trunc(x[fl])) - 0.5)
                assert frac.max() < 1e-5, frac.max()
                n_code_bands += code_rows.size
            rows = idx[scale_diff]
            n_bands_diff += rows.size
            m = (1 << (bits[bi] - 1)) - 1
            s = np.max(np.abs(c_core[rows, lo:lo + sz]), axis=1).astype(np.float32) / np.float32(m)
            h1 = ours[rows, o:o + 2].copy().view(np.float16)[:, 0].astype(np.float64)
            h2 = ref[rows, o:o + 2].copy().view(np.float16)[:, 0].astype(np.float64)
            mid = (h1 + h2) / 2
            assert np.all(np.abs(s - mid) / s < 4e-7), np.abs(s - mid) / s
        assert n_bands_diff == summary[name]["scale_flips"]
        assert (n_bands_diff + n_code_bands) / (X.shape[0] * bc.n_bands) < 2e-4


def test_reference_vht2_and_read(cfg0):
    """kernel_vht2_p2 equals its float32 restatement bit for bit and the CPU
    form within 1e-6 relative; the reference's batch read of its own rows
    equals dequantise -> unreorder -> CUDA-form VHT2, and the oracle's read
    of the same rows within 1e-6 relative L2."""
    K, _ = cfg0
    f = _load("ref_ship_cfg0.npz")
    np.testing.assert_array_equal(f["vht2"], RI.cuda_form_vht2(K[0, :64]))
    core = O.vht2(K[0, :64])
    assert np.linalg.norm(core - f["vht2"]) / np.linalg.norm(core) < 1e-6
    wk, _ = _rebuild(f, "wk", O.ship_write(K.reshape(-1, 128), RI.KB, True))
    wk = wk.reshape(8, 4096, -1)
    order = O.mobius_order(128)
    for h in range(2):
        rows = wk[h, :64]
        c = O.band_dequantize(rows, 128, RI.KB)
        un = np.empty_like(c)
        un[:, order] = c
        np.testing.assert_array_equal(f["rk"][h], RI.cuda_form_vht2(un))
        mine = O.ship_read(rows, 128, RI.KB, True)
        assert np.linalg.norm(mine - f["rk"][h]) / np.linalg.norm(mine) < 1e-6


def test_sqfree_residual_stages_bit_exact_with_reference_run():
    """shannon_prime_sqfree.cu: Möbius CSR prediction, spinor sheet choice,
    mean |dev|, residual levels, LSB-first packing and dequantisation on
    config-2 vectors: identical to the oracle's stages."""
    f = _load("ref_sqfree_stages.npz")
    L, sk, act, _ = RI.sqfree_stages()
    pred = O.sq_predict(L, sk)
    _rebuild(f, "pred", pred)
    dev, sheet = O.sq_spinor(act, pred)
    for name, ours in (("dev", dev), ("sheet", sheet)):
        assert _rebuild(f, name, ours)[1].size == 0, name
    np.testing.assert_array_equal(f["mag"], O.residual_mag(dev))
    lv = O.residual_levels(dev, RI.SQ_RES_BITS, f["mag"], "sqfree")
    for name, ours in (("pred", pred), ("levels", lv),
                       ("packed", O.pack_levels(lv, RI.SQ_RES_BITS)),
                       ("deq", O.residual_unlevels(lv, RI.SQ_RES_BITS, f["mag"], "sqfree"))):
        assert _rebuild(f, name, ours)[1].size == 0, name
    ties = RI.residual_ties(L.n_res, RI.SQ_RES_BITS, "sqfree")
    np.testing.assert_array_equal(f["tie_mag"], O.residual_mag(ties))
    tl = O.residual_levels(ties, RI.SQ_RES_BITS, f["tie_mag"], "sqfree")
    np.testing.assert_array_equal(f["tie_levels"], tl)
    np.testing.assert_array_equal(f["tie_packed"], O.pack_levels(tl, RI.SQ_RES_BITS))


def test_hier_residual_stages_against_reference_run():
    """shannon_prime_hier.cu: W·skeleton (fp16 W, fma chain), levels and
    dequantisation bit-exact; the magnitude's sum order differs (the
    reference's 256-thread tree vs the lane tree of the B200 kernels) by at
    most 2 ulp, and no level changes with either magnitude."""
    f = _load("ref_hier_stages.npz")
    H, W, sk, tgt = RI.hier_stages()
    pred = O.hier_predict(H, W, sk)
    assert _rebuild(f, "pred", pred)[1].size == 0
    dev = tgt - pred
    mine = O.residual_mag(dev)
    ulp = np.abs(mine.view(np.int32) - f["mag"].view(np.int32))
    assert ulp.max() <= 2
    lv = O.residual_levels(dev, RI.HIER_RES_BITS, f["mag"], "hier")
    assert _rebuild(f, "levels", lv)[1].size == 0
    np.testing.assert_array_equal(lv, O.residual_levels(dev, RI.HIER_RES_BITS, mine, "hier"))
    deq = O.residual_unlevels(lv, RI.HIER_RES_BITS, f["mag"], "hier")
    assert _rebuild(f, "deq", deq)[1].size == 0
    ties = RI.residual_ties(H.n_target, RI.HIER_RES_BITS, "hier")
    tmag = O.residual_mag(ties)
    assert np.abs(tmag.view(np.int32) - f["tie_mag"].view(np.int32)).max() <= 2
    np.testing.assert_array_equal(
        f["tie_levels"], O.residual_levels(ties, RI.HIER_RES_BITS, f["tie_mag"], "hier"))


def test_reference_vilenkin_within_table_precision():
    """kernel_vilenkin_inplace builds its cas values with __cosf/__sinf; the
    oracle's tables are computed in double.  The transforms agree to the
    precision of the reference's fast-math tables."""
    f = _load("ref_sqfree_stages.npz")
    x = np.random.default_rng(3).standard_normal((32, 154)).astype(np.float32)
    mine = O.vilenkin(x)
    assert np.max(np.abs(mine - f["vilenkin"])) < 5e-5
    assert np.linalg.norm(mine - f["vilenkin"]) / np.linalg.norm(mine) < 1e-5
