"""ctypes binding of the CPU oracle (oracle/sp_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline legs, never by the shipped library.  See
oracle/sp_oracle.h for what pins the restatement (the reference's own CUDA
code, run on a B200: tests/golden/ref_*.npz).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "lib" / "libsp_oracle.so"
MAX_BANDS = 16


class Bands(C.Structure):
    _fields_ = [
        ("n", C.c_int), ("n_bands", C.c_int),
        ("bits", C.c_int * MAX_BANDS), ("off", C.c_int * MAX_BANDS),
        ("size", C.c_int * MAX_BANDS), ("byte_off", C.c_int * MAX_BANDS),
        ("total_bytes", C.c_int),
    ]


OR_SQ_MAX_PD = 512
OR_SQ_MAX_TERMS = 16384


class Sqfree(C.Structure):
    _fields_ = [
        ("hd", C.c_int), ("pd", C.c_int), ("sk_k", C.c_int), ("n_res", C.c_int),
        ("n_terms", C.c_int), ("res_bits", C.c_int), ("use_spinor", C.c_int),
        ("skel_idx", C.c_int * OR_SQ_MAX_PD), ("res_idx", C.c_int * OR_SQ_MAX_PD),
        ("csr_off", C.c_int * (OR_SQ_MAX_PD + 1)), ("csr_slot", C.c_int * OR_SQ_MAX_TERMS),
        ("csr_sign", C.c_int * OR_SQ_MAX_TERMS), ("bands", Bands),
        ("res_bytes", C.c_int), ("sheet_bytes", C.c_int), ("bytes_per_pos", C.c_int),
    ]


class Hier(C.Structure):
    _fields_ = [
        ("hd", C.c_int), ("pd", C.c_int), ("n_skel", C.c_int), ("n_target", C.c_int),
        ("res_bits", C.c_int), ("bands", Bands), ("res_bytes", C.c_int),
        ("bytes_per_pos", C.c_int),
    ]


_lib = None
_P = C.c_void_p


def build() -> Path:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)
    return LIB_PATH


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            build()
        L = C.CDLL(str(LIB_PATH))
        L.or_f32_to_f16.restype = C.c_uint16
        L.or_f32_to_f16.argtypes = [C.c_float]
        L.or_f16_to_f32.restype = C.c_float
        L.or_f16_to_f32.argtypes = [C.c_uint16]
        L.or_band_config.restype = C.c_int
        L.or_band_config.argtypes = [C.POINTER(Bands), C.c_int, C.c_int, C.POINTER(C.c_int)]
        L.or_vht2.argtypes = [_P, C.c_int]
        L.or_mobius_order.argtypes = [C.c_int, _P]
        L.or_band_quantize.argtypes = [_P, _P, C.POINTER(Bands)]
        L.or_band_dequantize.argtypes = [_P, _P, C.POINTER(Bands), C.c_int]
        L.or_ship_write_batch.argtypes = [C.c_int, _P, C.c_size_t, _P, C.POINTER(Bands), _P, C.c_int]
        L.or_ship_read_batch.argtypes = [C.c_int, _P, _P, C.POINTER(Bands), _P, C.c_int, C.c_int]
        L.or_attn_decode.argtypes = [_P, C.c_size_t, _P, C.c_size_t, C.POINTER(Bands),
                                     C.POINTER(Bands), _P, C.c_int, C.c_int, C.c_int, _P,
                                     C.c_float, _P, C.c_int]
        L.or_lane_tree_sum.restype = C.c_float
        L.or_lane_tree_sum.argtypes = [_P, C.c_int]
        L.or_sqfree_pad_dim.restype = C.c_int
        L.or_sqfree_pad_dim.argtypes = [C.c_int]
        L.or_vilenkin.argtypes = [_P, C.c_int]
        L.or_cas_table.argtypes = [C.c_int, _P, _P]
        L.or_sqfree_layout.restype = C.c_int
        L.or_sqfree_layout.argtypes = [C.POINTER(Sqfree), C.c_int, C.c_int, C.c_int, _P, C.c_int, C.c_int]
        L.or_sqfree_write_batch.argtypes = [C.c_int, _P, _P, C.POINTER(Sqfree), C.c_int]
        L.or_sqfree_read_batch.argtypes = [C.c_int, _P, _P, C.POINTER(Sqfree), C.c_int]
        L.or_sqfree_coeffs.argtypes = [_P, _P, C.POINTER(Sqfree)]
        L.or_sqfree_attn_decode.argtypes = [_P, C.c_size_t, _P, C.c_size_t, C.POINTER(Sqfree),
                                            C.POINTER(Sqfree), C.c_int, C.c_int, C.c_int, _P,
                                            C.c_float, _P, C.c_int]
        L.or_hier_layout.restype = C.c_int
        L.or_hier_layout.argtypes = [C.POINTER(Hier), C.c_int, C.c_int, _P, C.c_int]
        L.or_hier_write_batch.argtypes = [C.c_int, _P, _P, C.POINTER(Hier), _P, C.c_int]
        L.or_hier_read_batch.argtypes = [C.c_int, _P, _P, C.POINTER(Hier), _P, C.c_int]
        L.or_correlation.restype = C.c_double
        L.or_correlation.argtypes = [_P, _P, C.c_int]
        _lib = L
    return _lib


def _p(a: np.ndarray | None) -> int | None:
    return None if a is None else a.ctypes.data


def bands(n: int, bits) -> Bands:
    b = Bands()
    arr = (C.c_int * len(bits))(*bits)
    if lib().or_band_config(C.byref(b), n, len(bits), arr) != 0:
        raise ValueError(f"bad band config n={n} bits={bits}")
    return b


def threads() -> int:
    return int(os.environ.get("SP_ORACLE_THREADS", os.cpu_count() or 1))


def f32_to_f16(x: float) -> int:
    return lib().or_f32_to_f16(x)


def vht2(x: np.ndarray) -> np.ndarray:
    y = np.ascontiguousarray(x, dtype=np.float32).copy()
    flat = y.reshape(-1, y.shape[-1])
    for row in flat:
        lib().or_vht2(row.ctypes.data, row.shape[0])
    return y


def mobius_order(n: int) -> np.ndarray:
    o = np.zeros(n, dtype=np.int32)
    lib().or_mobius_order(n, o.ctypes.data)
    return o


def ship_write(vecs: np.ndarray, bits, mobius: bool, n_threads: int | None = None) -> np.ndarray:
    """vecs [N][n] float32 -> packed uint8 [N][total_bytes]."""
    v = np.ascontiguousarray(vecs, dtype=np.float32).reshape(-1, vecs.shape[-1])
    n = v.shape[1]
    bc = bands(n, bits)
    out = np.zeros((v.shape[0], bc.total_bytes), dtype=np.uint8)
    order = mobius_order(n) if mobius else None
    lib().or_ship_write_batch(v.shape[0], v.ctypes.data, n, out.ctypes.data, C.byref(bc),
                              _p(order), n_threads or threads())
    return out


def ship_read(packed: np.ndarray, n: int, bits, mobius: bool, max_bands: int = -1,
              n_threads: int | None = None) -> np.ndarray:
    p = np.ascontiguousarray(packed, dtype=np.uint8)
    bc = bands(n, bits)
    assert p.shape[-1] == bc.total_bytes
    p2 = p.reshape(-1, bc.total_bytes)
    out = np.zeros((p2.shape[0], n), dtype=np.float32)
    order = mobius_order(n) if mobius else None
    lib().or_ship_read_batch(p2.shape[0], p2.ctypes.data, out.ctypes.data, C.byref(bc),
                             _p(order), max_bands, n_threads or threads())
    return out


def band_quantize(coeffs: np.ndarray, bits) -> np.ndarray:
    c = np.ascontiguousarray(coeffs, dtype=np.float32).reshape(-1, coeffs.shape[-1])
    bc = bands(c.shape[1], bits)
    out = np.zeros((c.shape[0], bc.total_bytes), dtype=np.uint8)
    for i in range(c.shape[0]):
        lib().or_band_quantize(c[i].ctypes.data, out[i].ctypes.data, C.byref(bc))
    return out


def band_dequantize(packed: np.ndarray, n: int, bits, max_bands: int = -1) -> np.ndarray:
    p = np.ascontiguousarray(packed, dtype=np.uint8)
    bc = bands(n, bits)
    p2 = p.reshape(-1, bc.total_bytes)
    out = np.zeros((p2.shape[0], n), dtype=np.float32)
    for i in range(p2.shape[0]):
        lib().or_band_dequantize(p2[i].ctypes.data, out[i].ctypes.data, C.byref(bc), max_bands)
    return out


def attn_decode(k_slots: np.ndarray, v_slots: np.ndarray, n: int, k_bits, v_bits, mobius: bool,
                q_f16: np.ndarray, kv_len: int, logit_scale: float = 1.0,
                n_threads: int | None = None) -> np.ndarray:
    """k_slots [H][>=kv_len][kb] uint8, v_slots likewise, q_f16 [n_q][n] float16
    -> out [n_q][n] float32 (double-accumulated reference attention)."""
    kb, vb = bands(n, k_bits), bands(n, v_bits)
    ks = np.ascontiguousarray(k_slots, dtype=np.uint8)
    vs = np.ascontiguousarray(v_slots, dtype=np.uint8)
    H = ks.shape[0]
    q = np.ascontiguousarray(q_f16, dtype=np.float16).view(np.uint16)
    nq = q.shape[0]
    out = np.zeros((nq, n), dtype=np.float32)
    order = mobius_order(n) if mobius else None
    lib().or_attn_decode(ks.ctypes.data, ks.shape[1] * ks.shape[2], vs.ctypes.data,
                         vs.shape[1] * vs.shape[2], C.byref(kb), C.byref(vb), _p(order), H,
                         nq, kv_len, q.ctypes.data, logit_scale, out.ctypes.data,
                         n_threads or threads())
    return out


def correlation(a: np.ndarray, b: np.ndarray) -> float:
    a = np.ascontiguousarray(a, dtype=np.float32).ravel()
    b = np.ascontiguousarray(b, dtype=np.float32).ravel()
    return lib().or_correlation(a.ctypes.data, b.ctypes.data, a.shape[0])


def mean_vector_correlation(a: np.ndarray, b: np.ndarray) -> float:
    """Pearson correlation per vector, averaged (the reference's per-vector
    validation measure, sp_llama_validate_k)."""
    a2 = a.reshape(-1, a.shape[-1])
    b2 = b.reshape(-1, b.shape[-1])
    return float(np.mean([correlation(x, y) for x, y in zip(a2, b2)]))


# ------------------------------------------------------------ sqfree / hier --

def sqfree_layout(hd: int, sk_k: int | None = None, bits=(5, 4, 4, 4, 5), residual_bits: int = 3,
                  use_spinor: bool = True, sk_frac: float | None = None) -> Sqfree:
    """Sqfree+spinor slot layout; sk_k defaults to floor(sk_frac * pad_dim)
    (sk_frac 0.75) or pad_dim // 2 when sk_frac is None and sk_k is None."""
    pd = lib().or_sqfree_pad_dim(hd)
    if sk_k is None:
        sk_k = int(sk_frac * pd) if sk_frac is not None else pd // 2
    L = Sqfree()
    arr = (C.c_int * len(bits))(*bits)
    if lib().or_sqfree_layout(C.byref(L), hd, sk_k, len(bits), arr, residual_bits,
                              1 if use_spinor else 0) != 0:
        raise ValueError("bad sqfree layout")
    return L


def sqfree_write(vecs: np.ndarray, L: Sqfree, n_threads: int | None = None) -> np.ndarray:
    v = np.ascontiguousarray(vecs, dtype=np.float32).reshape(-1, L.hd)
    out = np.zeros((v.shape[0], L.bytes_per_pos), np.uint8)
    lib().or_sqfree_write_batch(v.shape[0], v.ctypes.data, out.ctypes.data, C.byref(L),
                                n_threads or threads())
    return out


def sqfree_read(packed: np.ndarray, L: Sqfree, n_threads: int | None = None) -> np.ndarray:
    p = np.ascontiguousarray(packed, dtype=np.uint8).reshape(-1, L.bytes_per_pos)
    out = np.zeros((p.shape[0], L.hd), np.float32)
    lib().or_sqfree_read_batch(p.shape[0], p.ctypes.data, out.ctypes.data, C.byref(L),
                               n_threads or threads())
    return out


def sqfree_attn_decode(k_slots, v_slots, LK: Sqfree, LV: Sqfree, q_f16, kv_len: int,
                       logit_scale: float = 1.0, n_threads: int | None = None) -> np.ndarray:
    ks = np.ascontiguousarray(k_slots, dtype=np.uint8)
    vs = np.ascontiguousarray(v_slots, dtype=np.uint8)
    q = np.ascontiguousarray(q_f16, dtype=np.float16).view(np.uint16)
    H, nq = ks.shape[0], q.shape[0]
    out = np.zeros((nq, LK.hd), np.float32)
    lib().or_sqfree_attn_decode(ks.ctypes.data, ks[0].nbytes, vs.ctypes.data, vs[0].nbytes,
                                C.byref(LK), C.byref(LV), H, nq, kv_len, q.ctypes.data,
                                logit_scale, out.ctypes.data, n_threads or threads())
    return out


def vilenkin(x: np.ndarray) -> np.ndarray:
    y = np.ascontiguousarray(x, dtype=np.float32).copy()
    flat = y.reshape(-1, y.shape[-1])
    for row in flat:
        lib().or_vilenkin(row.ctypes.data, row.shape[0])
    return y


def hier_layout(hd: int, bits=(5, 5), residual_bits: int = 2) -> Hier:
    L = Hier()
    arr = (C.c_int * len(bits))(*bits)
    if lib().or_hier_layout(C.byref(L), hd, len(bits), arr, residual_bits) != 0:
        raise ValueError("bad hier layout")
    return L


def hier_write(vecs: np.ndarray, L: Hier, W: np.ndarray, n_threads: int | None = None) -> np.ndarray:
    v = np.ascontiguousarray(vecs, dtype=np.float32).reshape(-1, L.hd)
    w = np.ascontiguousarray(W, dtype=np.float16).view(np.uint16)
    assert w.shape == (L.n_target, L.n_skel)
    out = np.zeros((v.shape[0], L.bytes_per_pos), np.uint8)
    lib().or_hier_write_batch(v.shape[0], v.ctypes.data, out.ctypes.data, C.byref(L),
                              w.ctypes.data, n_threads or threads())
    return out


def hier_read(packed: np.ndarray, L: Hier, W: np.ndarray, n_threads: int | None = None) -> np.ndarray:
    p = np.ascontiguousarray(packed, dtype=np.uint8).reshape(-1, L.bytes_per_pos)
    w = np.ascontiguousarray(W, dtype=np.float16).view(np.uint16)
    out = np.zeros((p.shape[0], L.hd), np.float32)
    lib().or_hier_read_batch(p.shape[0], p.ctypes.data, out.ctypes.data, C.byref(L),
                             w.ctypes.data, n_threads or threads())
    return out


def hier_fit_W(calib: np.ndarray, L: Hier, ridge: float = 1e-6) -> np.ndarray:
    """Predictor W [n_target][n_skel] (fp16) fitted by ridge least squares in
    double on a calibration set of vectors: padded, transformed, skeleton
    coefficients -> target coefficients.  Calibration is host-side work (the
    reference fits W on the CPU and uploads it, kv_cache.cpp:519-808)."""
    v = np.ascontiguousarray(calib, dtype=np.float32).reshape(-1, L.hd)
    pad = np.empty((v.shape[0], L.pd), np.float32)
    for i, row in enumerate(v):
        pad[i, :L.hd] = row
        pad[i, L.hd:] = lib().or_lane_tree_sum(row.ctypes.data, L.hd) / np.float32(L.hd)
    c = vilenkin(pad).astype(np.float64)
    S, T = c[:, :L.n_skel], c[:, L.n_skel:]
    A = S.T @ S + ridge * np.eye(L.n_skel)
    W = np.linalg.solve(A, S.T @ T).T
    return W.astype(np.float16)


# ------------------------------------------------- residual stages (pinning) --

def _stage_lib():
    L = lib()
    if not getattr(L, "_stages_bound", False):
        L.or_sq_predict.argtypes = [C.POINTER(Sqfree), _P, _P]
        L.or_hier_predict.argtypes = [C.POINTER(Hier), _P, _P, _P]
        L.or_sq_spinor.argtypes = [_P, _P, C.c_int, _P, _P]
        L.or_residual_mag.restype = C.c_float
        L.or_residual_mag.argtypes = [_P, C.c_int]
        for f in ("or_sq_levels", "or_hier_levels"):
            getattr(L, f).argtypes = [_P, C.c_int, C.c_int, C.c_float, _P]
        for f in ("or_sq_unlevels", "or_hier_unlevels"):
            getattr(L, f).argtypes = [_P, C.c_int, C.c_int, C.c_float, _P]
        L._stages_bound = True
    return L


def sq_predict(L: Sqfree, skel: np.ndarray) -> np.ndarray:
    s = np.ascontiguousarray(skel, np.float32).reshape(-1, L.sk_k)
    out = np.zeros((s.shape[0], L.n_res), np.float32)
    for i in range(s.shape[0]):
        _stage_lib().or_sq_predict(C.byref(L), s[i].ctypes.data, out[i].ctypes.data)
    return out


def hier_predict(L: Hier, W: np.ndarray, skel: np.ndarray) -> np.ndarray:
    w = np.ascontiguousarray(W, np.float16).view(np.uint16)
    s = np.ascontiguousarray(skel, np.float32).reshape(-1, L.n_skel)
    out = np.zeros((s.shape[0], L.n_target), np.float32)
    for i in range(s.shape[0]):
        _stage_lib().or_hier_predict(C.byref(L), w.ctypes.data, s[i].ctypes.data,
                                     out[i].ctypes.data)
    return out


def sq_spinor(actual: np.ndarray, pred: np.ndarray):
    a = np.ascontiguousarray(actual, np.float32)
    p = np.ascontiguousarray(pred, np.float32)
    n = a.shape[-1]
    dev = np.zeros_like(a)
    sheet = np.zeros((a.shape[0], (n + 7) // 8), np.uint8)
    for i in range(a.shape[0]):
        _stage_lib().or_sq_spinor(a[i].ctypes.data, p[i].ctypes.data, n, dev[i].ctypes.data,
                                  sheet[i].ctypes.data)
    return dev, sheet


def residual_mag(dev: np.ndarray) -> np.ndarray:
    d = np.ascontiguousarray(dev, np.float32)
    return np.array([_stage_lib().or_residual_mag(r.ctypes.data, d.shape[-1]) for r in d],
                    np.float32)


def residual_levels(dev: np.ndarray, bits: int, mag: np.ndarray, form: str) -> np.ndarray:
    """form 'sqfree' (round-half-up of fma + 0.5, sat = mag*bits) or 'hier'
    (rint of the fma, step from mag)."""
    d = np.ascontiguousarray(dev, np.float32)
    out = np.zeros(d.shape, np.uint8)
    f = _stage_lib().or_sq_levels if form == "sqfree" else _stage_lib().or_hier_levels
    for i in range(d.shape[0]):
        f(d[i].ctypes.data, d.shape[-1], bits, float(mag[i]), out[i].ctypes.data)
    return out


def residual_unlevels(lv: np.ndarray, bits: int, mag: np.ndarray, form: str) -> np.ndarray:
    v = np.ascontiguousarray(lv, np.uint8)
    out = np.zeros(v.shape, np.float32)
    f = _stage_lib().or_sq_unlevels if form == "sqfree" else _stage_lib().or_hier_unlevels
    for i in range(v.shape[0]):
        f(v[i].ctypes.data, v.shape[-1], bits, float(mag[i]), out[i].ctypes.data)
    return out


def pack_levels(lv: np.ndarray, bits: int) -> np.ndarray:
    """LSB-first level packing, ceil(n*bits/8) bytes per row."""
    v = np.ascontiguousarray(lv, np.uint8)
    n = v.shape[-1]
    nb = (n * bits + 7) // 8
    out = np.zeros((v.shape[0], nb), np.uint8)
    for i in range(n):
        b = i * bits
        out[:, b >> 3] |= (v[:, i].astype(np.uint16) << (b & 7)).astype(np.uint8)
        if (b & 7) + bits > 8 and (b >> 3) + 1 < nb:
            out[:, (b >> 3) + 1] |= (v[:, i] >> (8 - (b & 7))).astype(np.uint8)
    return out
