"""This repo's CUDA kernels against outputs that the reference's own CUDA
code computed (tests/golden/ref_*.npz, written by
tests/golden/make_ref_fixtures.py) and, when oracle/_ref holds the compiled
reference, against the reference run live on the same device."""
import ctypes as C
import hashlib
import sys
from pathlib import Path

import numpy as np
import pytest

GOLD = Path(__file__).resolve().parent / "golden"
sys.path.insert(0, str(GOLD))

import oracle as O  # noqa: E402
import ref_inputs as RI  # noqa: E402
import refrun  # noqa: E402
import spb200  # noqa: E402

pytestmark = pytest.mark.gpu


def _bc(bits):
    bc = spb200.SpBandConfig()
    assert spb200.lib().sp_band_config_init(C.byref(bc), 128, len(bits),
                                            (C.c_int * len(bits))(*bits)) == 0
    return bc


def _quantize_gpu(coeffs, bits):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(coeffs, np.float32)).cuda()
    bc = _bc(bits)
    out = torch.zeros(t.shape[0], bc.total_bytes, dtype=torch.uint8, device="cuda")
    spb200.lib().sp_cuda_band_quantize(t.data_ptr(), out.data_ptr(), C.byref(bc), t.shape[0], None)
    torch.cuda.synchronize()
    return out.cpu().numpy()


def test_band_quantize_matches_reference_run(cuda):
    """sp_cuda_band_quantize on config-0 coefficients and edge rows: the
    SHA-256 of the output equals that of the reference kernel's output."""
    K, V = RI.ship_cfg0()
    f = np.load(GOLD / "ref_ship_cfg0.npz")
    for name, c, bits in (("qk", RI.ship_coeffs(K, True), RI.KB),
                          ("qv", RI.ship_coeffs(V, False), RI.VB),
                          ("qedge", RI.edge_coeffs(), RI.KB),
                          ("qedgev", RI.edge_coeffs(), RI.VB)):
        got = _quantize_gpu(c.reshape(-1, 128), bits)
        assert hashlib.sha256(got.tobytes()).hexdigest() == str(f[f"{name}_sha"]), name


def test_ship_write_against_reference_run(cuda):
    """The fused writer (sp_cuda_write_kv_tokens, all 8 heads of config 0 in
    one launch) against the reference's per-slot batch write: the rows that
    differ are exactly the rows where the CPU oracle differs from it (bands
    decided by fp16-midpoint scales or half-integer ties, see
    test_ref_fixtures.py), and everywhere else the bytes are equal."""
    import torch
    K, V = RI.ship_cfg0()
    f = np.load(GOLD / "ref_ship_cfg0.npz")
    cache = spb200.Cache(128, 1, 8, 4096)
    cache.write_kv_tokens(0, 0, torch.from_numpy(np.ascontiguousarray(K.transpose(1, 0, 2))).cuda(),
                          torch.from_numpy(np.ascontiguousarray(V.transpose(1, 0, 2))).cuda())
    torch.cuda.synchronize()
    for which, name, X, bits, mob in ((0, "wk", K, RI.KB, True), (1, "wv", V, RI.VB, False)):
        got = cache.slab(which).cpu().numpy()[:, :4096].reshape(-1, cache.k_bytes if which == 0
                                                                 else cache.v_bytes)
        ref = got.copy()
        ref[f[f"{name}_diff_idx"]] = f[f"{name}_diff_rows"]
        assert hashlib.sha256(ref.tobytes()).hexdigest() == str(f[f"{name}_sha"]), name
        diff = np.nonzero(np.any(got != ref, axis=1))[0]
        np.testing.assert_array_equal(diff, f[f"{name}_diff_idx"])
    cache.free()


@pytest.mark.skipif(not refrun.available(), reason="oracle/_ref (compiled reference) not present")
def test_live_reference_quantize_and_read(cuda):
    """The compiled reference on this device, on fresh seeded coefficients
    (mixed magnitudes, K and V layouts), against sp_cuda_band_quantize and
    against this repo's batch read of the reference's own packed rows."""
    import torch
    rng = np.random.default_rng(2024)
    c = (rng.standard_normal((4096, 128)) *
         10.0 ** rng.integers(-6, 6, (4096, 1))).astype(np.float32)
    c = np.concatenate([c, RI.edge_coeffs()])
    for bits in (RI.KB, RI.VB, [5, 4, 4], [8], [2, 2, 2, 2]):
        np.testing.assert_array_equal(_quantize_gpu(c, bits), refrun.band_quantize(c, bits))
    x = rng.standard_normal((1024, 128)).astype(np.float32)
    packed = refrun.ship_write(x, False, RI.KB, RI.VB, True)
    ref_read = refrun.ship_read(packed, 128, False, RI.KB, RI.VB, True)
    cache = spb200.Cache(128, 1, 1, 1024)
    cache.slab(0)[0, :1024].copy_(torch.from_numpy(packed).cuda())
    out = torch.empty(1024, 128, device="cuda")
    cache.read_batch(0, 0, 0, 0, out)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    assert np.linalg.norm(got - ref_read) / np.linalg.norm(ref_read) < 1e-6
    cache.free()
