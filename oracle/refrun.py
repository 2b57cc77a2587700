"""ctypes binding of oracle/_ref/libsp_ref_cuda.so: the reference's own CUDA
code (src/backends/cuda/shannon_prime_{cuda,sqfree,hier}.cu, compiled
unmodified by oracle/ref/Makefile) behind host-buffer entry points
(oracle/ref/ref_glue.cu).

TEST INFRASTRUCTURE ONLY: used by tests/golden/make_ref_fixtures.py (which
writes the reference-run fixtures under tests/golden/) and by the GPU tests
that re-run the reference live when the library is present.  Needs a GPU.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "_ref" / "libsp_ref_cuda.so"
_P = C.c_void_p
_lib = None


def available() -> bool:
    return LIB_PATH.exists()


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        _lib = C.CDLL(str(LIB_PATH))
    return _lib


def _ck(rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"reference {what} failed: {rc}")


def _ints(v):
    return (C.c_int * len(v))(*v)


def vht2(x: np.ndarray) -> np.ndarray:
    y = np.ascontiguousarray(x, np.float32).copy()
    _ck(lib().refg_vht2(_P(y.ctypes.data), y.shape[-1], y.size // y.shape[-1]), "vht2")
    return y


def mobius(x: np.ndarray, order: np.ndarray, inverse: bool = False) -> np.ndarray:
    y = np.ascontiguousarray(x, np.float32).copy()
    o = np.ascontiguousarray(order, np.int32)
    _ck(lib().refg_mobius(_P(y.ctypes.data), _P(o.ctypes.data), y.shape[-1],
                          y.size // y.shape[-1], int(inverse)), "mobius")
    return y


def _total_bytes(n: int, bits) -> int:
    nb = len(bits)
    bs = n // nb
    return sum(2 + (((n - b * bs) if b == nb - 1 else bs) * bits[b] + 7) // 8 for b in range(nb))


def band_quantize(coeffs: np.ndarray, bits) -> np.ndarray:
    c = np.ascontiguousarray(coeffs, np.float32).reshape(-1, coeffs.shape[-1])
    out = np.zeros((c.shape[0], _total_bytes(c.shape[1], bits)), np.uint8)
    _ck(lib().refg_band_quantize(_P(c.ctypes.data), c.shape[1], c.shape[0], len(bits),
                                 _ints(bits), _P(out.ctypes.data)), "band_quantize")
    return out


def band_dequantize(packed: np.ndarray, n: int, bits) -> np.ndarray:
    p = np.ascontiguousarray(packed, np.uint8).reshape(-1, packed.shape[-1])
    out = np.zeros((p.shape[0], n), np.float32)
    _ck(lib().refg_band_dequantize(_P(p.ctypes.data), n, p.shape[0], len(bits), _ints(bits),
                                   _P(out.ctypes.data)), "band_dequantize")
    return out


def ship_write(vecs: np.ndarray, is_v: bool, k_bits, v_bits, mobius_on: bool) -> np.ndarray:
    """One slot through sp_cuda_cache_init + sp_cuda_write_{k,v}_batch."""
    v = np.ascontiguousarray(vecs, np.float32).reshape(-1, vecs.shape[-1])
    n = v.shape[1]
    out = np.zeros((v.shape[0], _total_bytes(n, v_bits if is_v else k_bits)), np.uint8)
    _ck(lib().refg_ship_write(int(is_v), _P(v.ctypes.data), n, v.shape[0], len(k_bits),
                              _ints(k_bits), len(v_bits), _ints(v_bits), int(mobius_on),
                              _P(out.ctypes.data)), "ship_write")
    return out


def ship_read(packed: np.ndarray, n: int, is_v: bool, k_bits, v_bits, mobius_on: bool) -> np.ndarray:
    p = np.ascontiguousarray(packed, np.uint8)
    out = np.zeros((p.shape[0], n), np.float32)
    _ck(lib().refg_ship_read(int(is_v), _P(p.ctypes.data), n, p.shape[0], len(k_bits),
                             _ints(k_bits), len(v_bits), _ints(v_bits), int(mobius_on),
                             _P(out.ctypes.data)), "ship_read")
    return out


def vilenkin(x: np.ndarray) -> np.ndarray:
    y = np.ascontiguousarray(x, np.float32).copy()
    _ck(lib().refg_vilenkin(_P(y.ctypes.data), y.shape[-1], y.size // y.shape[-1]), "vilenkin")
    return y


def sq_predict(skel: np.ndarray, off, slot, sign, n_res: int) -> np.ndarray:
    s = np.ascontiguousarray(skel, np.float32)
    o, sl, sg = (np.ascontiguousarray(a, np.int32) for a in (off, slot, sign))
    out = np.zeros((s.shape[0], n_res), np.float32)
    _ck(lib().refg_sq_predict(_P(s.ctypes.data), s.shape[0], s.shape[1], n_res,
                              _P(o.ctypes.data), _P(sl.ctypes.data), _P(sg.ctypes.data),
                              _P(out.ctypes.data)), "sq_predict")
    return out


def sq_spinor(actual: np.ndarray, pred: np.ndarray):
    a = np.ascontiguousarray(actual, np.float32)
    p = np.ascontiguousarray(pred, np.float32)
    n = a.shape[1]
    dev = np.zeros_like(a)
    sheet = np.zeros((a.shape[0], (n + 7) // 8), np.uint8)
    _ck(lib().refg_sq_spinor(_P(a.ctypes.data), _P(p.ctypes.data), a.shape[0], n,
                             _P(dev.ctypes.data), _P(sheet.ctypes.data)), "sq_spinor")
    return dev, sheet


def sq_residual(dev: np.ndarray, bits: int):
    """-> (mag [N], levels [N][n], packed [N][ceil(n*bits/8)])."""
    d = np.ascontiguousarray(dev, np.float32)
    N, n = d.shape
    mag = np.zeros(N, np.float32)
    lv = np.zeros((N, n), np.uint8)
    pk = np.zeros((N, (n * bits + 7) // 8), np.uint8)
    _ck(lib().refg_sq_residual(_P(d.ctypes.data), N, n, bits, _P(mag.ctypes.data),
                               _P(lv.ctypes.data), _P(pk.ctypes.data)), "sq_residual")
    return mag, lv, pk


def sq_dequant(levels: np.ndarray, mag: np.ndarray, bits: int) -> np.ndarray:
    lv = np.ascontiguousarray(levels, np.uint8)
    m = np.ascontiguousarray(mag, np.float32)
    out = np.zeros(lv.shape, np.float32)
    _ck(lib().refg_sq_dequant(_P(lv.ctypes.data), _P(m.ctypes.data), lv.shape[0], lv.shape[1],
                              bits, _P(out.ctypes.data)), "sq_dequant")
    return out


def hier_predict(W_f16: np.ndarray, skel: np.ndarray) -> np.ndarray:
    w = np.ascontiguousarray(W_f16, np.float16).view(np.uint16)
    s = np.ascontiguousarray(skel, np.float32)
    out = np.zeros((s.shape[0], w.shape[0]), np.float32)
    _ck(lib().refg_hier_predict(_P(w.ctypes.data), _P(s.ctypes.data), s.shape[0], w.shape[0],
                                w.shape[1], _P(out.ctypes.data)), "hier_predict")
    return out


def hier_residual(dev: np.ndarray, bits: int):
    d = np.ascontiguousarray(dev, np.float32)
    N, n = d.shape
    mag = np.zeros(N, np.float32)
    lv = np.zeros((N, n), np.uint8)
    _ck(lib().refg_hier_residual(_P(d.ctypes.data), N, n, bits, _P(mag.ctypes.data),
                                 _P(lv.ctypes.data)), "hier_residual")
    return mag, lv


def hier_dequant(levels: np.ndarray, mag: np.ndarray, bits: int) -> np.ndarray:
    lv = np.ascontiguousarray(levels, np.uint8)
    m = np.ascontiguousarray(mag, np.float32)
    out = np.zeros(lv.shape, np.float32)
    _ck(lib().refg_hier_dequant(_P(lv.ctypes.data), _P(m.ctypes.data), lv.shape[0], lv.shape[1],
                                bits, _P(out.ctypes.data)), "hier_dequant")
    return out
