"""Generate the reference-run fixtures tests/golden/ref_*.npz.

Runs the reference's own CUDA code (oracle/_ref/libsp_ref_cuda.so, built
unmodified from src/backends/cuda/shannon_prime_{cuda,sqfree,hier}.cu by
oracle/ref/Makefile) on the seeded inputs of tests/golden/ref_inputs.py and
stores what it computed.  Needs a GPU; the fixtures it writes are then
checked on CPU against the oracle (tests/test_ref_fixtures.py) and on the GPU
against this repo's kernels (tests/test_gpu_refpin.py).

Outputs that are expected to equal the oracle's bit for bit are stored
compactly: the SHA-256 of the reference's whole output, the first rows, and
every row where the reference differs from the oracle (with the reference's
bytes for those rows), so a test can rebuild the reference's full output from
the oracle's and check the hash.

    python tests/golden/make_ref_fixtures.py [OUT_DIR]
"""
from __future__ import annotations

import hashlib
import json
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
for p in (ROOT / "oracle", ROOT / "shannon-prime-llama_b200", HERE):
    sys.path.insert(0, str(p))

import numpy as np  # noqa: E402

import oracle as O  # noqa: E402
import ref_inputs as RI  # noqa: E402
import refrun as R  # noqa: E402


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def compact(name: str, ref: np.ndarray, ours: np.ndarray, head: int = 16) -> dict:
    """ref/ours [N][B] -> fixture fields: hash, first rows, differing rows."""
    ref2 = ref.reshape(-1, ref.shape[-1])
    ours2 = ours.reshape(-1, ours.shape[-1])
    diff = np.nonzero(np.any(ref2 != ours2, axis=1))[0].astype(np.int64)
    return {f"{name}_sha": np.array(sha(ref2)), f"{name}_head": ref2[:head].copy(),
            f"{name}_diff_idx": diff, f"{name}_diff_rows": ref2[diff].copy()}


def code_flips(ref: np.ndarray, ours: np.ndarray, n: int, bits) -> tuple[int, int, int]:
    """(differing codes, differing scales, total codes) between packed rows."""
    a = O.band_dequantize(ref, n, bits)
    b = O.band_dequantize(ours, n, bits)
    bc = O.bands(n, bits)
    scales = 0
    for bi in range(bc.n_bands):
        o = bc.byte_off[bi]
        scales += int(np.count_nonzero(np.any(ref[:, o:o + 2] != ours[:, o:o + 2], axis=1)))
    codes = int(np.count_nonzero(a != b))
    return codes, scales, a.size


def opt_build_divergence(ck: np.ndarray) -> dict:
    """The default-optimised build of shannon_prime_cuda.cu (oracle/_ref/opt,
    `make -C oracle/ref opt`) on the same coefficients: which bytes differ
    from the unoptimised build's (i.e. the source's) output."""
    path = R.LIB_PATH.parent / "opt" / R.LIB_PATH.name
    if not path.exists():
        return {"available": False}
    good = R.band_quantize(ck, RI.KB)
    saved, R._lib = R._lib, None
    R.LIB_PATH, keep = path, R.LIB_PATH
    try:
        bad = R.band_quantize(ck, RI.KB)
    finally:
        R.LIB_PATH, R._lib = keep, saved
    bc = O.bands(128, RI.KB)
    lo = [bc.byte_off[b] for b in range(bc.n_bands)]
    hi = [o + 1 for o in lo]
    rest = np.ones(good.shape[1], bool)
    rest[lo + hi] = False
    return {"available": True, "rows": int(good.shape[0]),
            "rows_differing": int(np.count_nonzero(np.any(good != bad, axis=1))),
            "code_bytes_differing": int(np.count_nonzero(good[:, rest] != bad[:, rest])),
            "scale_high_bytes_differing": int(np.count_nonzero(good[:, hi] != bad[:, hi])),
            "scale_low_bytes_differing": int(np.count_nonzero(good[:, lo] != bad[:, lo])),
            "low_byte_values_seen": sorted(int(x) for x in np.unique(bad[:, lo]))}


def main(out_dir: Path) -> dict:
    out_dir.mkdir(parents=True, exist_ok=True)
    summary: dict = {}

    # ---- ship path, config 0 ------------------------------------------------
    K, V = RI.ship_cfg0()
    ck = RI.ship_coeffs(K, True).reshape(-1, 128)
    cv = RI.ship_coeffs(V, False).reshape(-1, 128)
    edge = RI.edge_coeffs()
    f = {}
    # band quantiser on identical coefficients
    for nm, c, bits in (("qk", ck, RI.KB), ("qv", cv, RI.VB), ("qedge", edge, RI.KB),
                        ("qedgev", edge, RI.VB)):
        ref = R.band_quantize(c, bits)
        f.update(compact(nm, ref, O.band_quantize(c, bits)))
        summary[nm] = {"rows": int(ref.shape[0]), "rows_differing": int(f[f"{nm}_diff_idx"].size)}
        if nm == "qedge":
            deq = R.band_dequantize(ref, 128, bits)
            f["qedge_deq"] = deq
    # the reference's whole write (its VHT2 scales each stage by 1/sqrt 2)
    wk = np.stack([R.ship_write(K[h], False, RI.KB, RI.VB, True) for h in range(K.shape[0])])
    wv = np.stack([R.ship_write(V[h], True, RI.KB, RI.VB, True) for h in range(V.shape[0])])
    ok = O.ship_write(K.reshape(-1, 128), RI.KB, True).reshape(wk.shape)
    ov = O.ship_write(V.reshape(-1, 128), RI.VB, False).reshape(wv.shape)
    f.update(compact("wk", wk, ok))
    f.update(compact("wv", wv, ov))
    for nm, r, o, bits in (("wk", wk, ok, RI.KB), ("wv", wv, ov, RI.VB)):
        codes, scales, total = code_flips(r.reshape(-1, r.shape[-1]), o.reshape(-1, o.shape[-1]),
                                          128, bits)
        summary[nm] = {"code_flips": codes, "scale_flips": scales, "codes": total,
                       "flip_rate": codes / total}
    # the reference's read of its own rows (first 64 positions of heads 0 and 1)
    f["rk"] = np.stack([R.ship_read(wk[h, :64], 128, False, RI.KB, RI.VB, True) for h in range(2)])
    f["rv"] = np.stack([R.ship_read(wv[h, :64], 128, True, RI.KB, RI.VB, True) for h in range(2)])
    # transform alone
    f["vht2"] = R.vht2(K[0, :64])
    np.savez_compressed(out_dir / "ref_ship_cfg0.npz", **f)
    summary["opt_build"] = opt_build_divergence(ck)

    # ---- sqfree residual stages (config 2 layout) --------------------------
    L, sk, act, (off, slot, sign) = RI.sqfree_stages()
    g = {}
    opred = O.sq_predict(L, sk)
    g.update(compact("pred", R.sq_predict(sk, off, slot, sign, L.n_res), opred))
    rdev, rsheet = R.sq_spinor(act, opred)
    odev, osheet = O.sq_spinor(act, opred)
    g.update(compact("dev", rdev, odev))
    g.update(compact("sheet", rsheet, osheet))
    rmag, rlv, rpk = R.sq_residual(odev, RI.SQ_RES_BITS)
    g["mag"] = rmag
    g.update(compact("levels", rlv, O.residual_levels(odev, RI.SQ_RES_BITS, rmag, "sqfree")))
    g.update(compact("packed", rpk, O.pack_levels(rlv, RI.SQ_RES_BITS)))
    g.update(compact("deq", R.sq_dequant(rlv, rmag, RI.SQ_RES_BITS),
                     O.residual_unlevels(rlv, RI.SQ_RES_BITS, rmag, "sqfree")))
    ties = RI.residual_ties(L.n_res, RI.SQ_RES_BITS, "sqfree")
    g["tie_mag"], g["tie_levels"], g["tie_packed"] = R.sq_residual(ties, RI.SQ_RES_BITS)
    pd_rows = np.random.default_rng(3).standard_normal((32, L.pd)).astype(np.float32)
    g["vilenkin"] = R.vilenkin(pd_rows)
    np.savez_compressed(out_dir / "ref_sqfree_stages.npz", **g)
    omag = O.residual_mag(odev)
    summary["sqfree"] = {
        "vectors": int(sk.shape[0]),
        **{k: int(g[f"{k}_diff_idx"].size) for k in ("pred", "dev", "sheet", "levels", "packed", "deq")},
        "mag_differing": int(np.count_nonzero(rmag != omag)),
        "level_flips_own_mag": int(np.count_nonzero(
            rlv != O.residual_levels(odev, RI.SQ_RES_BITS, omag, "sqfree"))),
        "vilenkin_max_abs_diff": float(np.max(np.abs(g["vilenkin"] - O.vilenkin(pd_rows)))),
    }

    # ---- hier residual stages (config 4 layout) ----------------------------
    H, W, hsk, htgt = RI.hier_stages()
    h = {}
    opred = O.hier_predict(H, W, hsk)
    h.update(compact("pred", R.hier_predict(W, hsk), opred))
    hdev = htgt - opred
    rmag, rlv = R.hier_residual(hdev, RI.HIER_RES_BITS)
    h["mag"] = rmag
    h.update(compact("levels", rlv, O.residual_levels(hdev, RI.HIER_RES_BITS, rmag, "hier")))
    h.update(compact("deq", R.hier_dequant(rlv, rmag, RI.HIER_RES_BITS),
                     O.residual_unlevels(rlv, RI.HIER_RES_BITS, rmag, "hier")))
    ties = RI.residual_ties(H.n_target, RI.HIER_RES_BITS, "hier")
    h["tie_mag"], h["tie_levels"] = R.hier_residual(ties, RI.HIER_RES_BITS)
    np.savez_compressed(out_dir / "ref_hier_stages.npz", **h)
    omag = O.residual_mag(hdev)
    summary["hier"] = {
        "vectors": int(hsk.shape[0]),
        **{k: int(h[f"{k}_diff_idx"].size) for k in ("pred", "levels", "deq")},
        "mag_differing": int(np.count_nonzero(rmag != omag)),
        "level_flips_own_mag": int(np.count_nonzero(
            rlv != O.residual_levels(hdev, RI.HIER_RES_BITS, omag, "hier"))),
    }
    (out_dir / "ref_summary.json").write_text(json.dumps(summary, indent=1) + "\n")
    return summary


if __name__ == "__main__":
    out = Path(sys.argv[1]) if len(sys.argv) > 1 else HERE
    print(json.dumps(main(out), indent=1))
