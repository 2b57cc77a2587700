"""CPU tests of the C-ABI library: it loads, exports every function the
public headers declare, its struct sizes match the bindings, and the bridge
answers NULL where the reference bridge does (no GPU needed)."""
import ctypes as C
import os
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


def _declared_functions():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        for m in re.finditer(r"^[A-Za-z_][\w \*]*?\b(sp_\w+)\s*\(", text, flags=re.M):
            names.add(m.group(1))
    return sorted(names)


def test_headers_declare_the_reference_surface():
    names = set(_declared_functions())
    for ref_name in ["sp_cuda_cache_init", "sp_cuda_cache_free", "sp_cuda_write_k",
                     "sp_cuda_write_v", "sp_cuda_read_k", "sp_cuda_read_v",
                     "sp_cuda_write_k_batch", "sp_cuda_write_v_batch",
                     "sp_cuda_read_k_batch", "sp_cuda_read_v_batch", "sp_cuda_vht2_forward",
                     "sp_cuda_mobius_reorder", "sp_cuda_mobius_unreorder",
                     "sp_cuda_band_quantize", "sp_cuda_band_dequantize",
                     "sp_cuda_print_memory", "sp_llama_init", "sp_llama_init_with_role",
                     "sp_llama_init_config", "sp_llama_free", "sp_llama_write_kv",
                     "sp_llama_write_k", "sp_llama_write_v", "sp_llama_write_k_batch",
                     "sp_llama_write_v_batch", "sp_llama_read_k", "sp_llama_read_v",
                     "sp_llama_read_k_partial", "sp_llama_read_v_partial",
                     "sp_llama_read_k_batch", "sp_llama_read_v_batch", "sp_llama_clear_range",
                     "sp_llama_memory", "sp_llama_validate_k", "sp_llama_print_config",
                     "sp_llama_get_freq_factors", "sp_llama_get_n_freqs",
                     "sp_llama_get_hexagon_k_buf", "sp_llama_get_hexagon_k_total_bytes"]:
        assert ref_name in names, ref_name


def test_library_exports_every_declared_symbol(built_lib):
    L = C.CDLL(str(built_lib))
    missing = [n for n in _declared_functions() if not hasattr(L, n)]
    assert not missing, missing


def test_binding_struct_mirrors(built_lib):
    import spb200
    spb200.lib()   # raises if a mirror is wrong
    assert set(spb200.SIGNATURES) >= set(_declared_functions())


def test_bridge_disabled_returns_null(built_lib, monkeypatch):
    import spb200
    monkeypatch.delenv("SHANNON_PRIME_ENABLED", raising=False)
    p = spb200.SpLlamaParams(128, 2, 2, 64, 1, None, None)
    assert not spb200.lib().sp_llama_init(C.byref(p))


def test_bridge_without_device_returns_null(built_lib, monkeypatch):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a CUDA device is present")
    import spb200
    monkeypatch.setenv("SHANNON_PRIME_ENABLED", "1")
    p = spb200.SpLlamaParams(128, 2, 2, 64, 1, None, None)
    assert not spb200.lib().sp_llama_init(C.byref(p))


def test_host_config_utilities(built_lib):
    import spb200
    L = spb200.lib()
    cfg = spb200.make_config(128, 32, 8)
    assert list(cfg.k_band_bits)[:4] == [5, 5, 4, 3] and cfg.k_n_bands == 4
    assert cfg.v_n_bands == 1 and cfg.v_band_bits[0] == 3 and cfg.use_mobius_mask == 1
    cfg64 = spb200.make_config(64, 1, 1)
    assert list(cfg64.k_band_bits)[:3] == [5, 4, 4] and cfg64.v_band_bits[0] == 5
    bc = spb200.SpBandConfig()
    assert L.sp_band_config_init(C.byref(bc), 128, 4, (C.c_int * 4)(5, 5, 4, 3)) == 0
    assert bc.total_bytes == 76 and bc.band_size == 32
    assert L.sp_band_config_init(C.byref(bc), 128, 1, (C.c_int * 1)(9)) != 0
