"""ctypes binding of the B200 Shannon-Prime C-ABI (include/shannon_prime_cuda.h,
include/shannon_prime_llama.h).

The library is the in-tree lib/libshannon_prime_b200.so built by
shannon-prime-llama_b200/build.py.  There is no fallback: if the library is
missing, importing the binding raises.  Device buffers are passed as torch
CUDA tensors (their data_ptr); torch is used only for device memory and
streams.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

PKG = Path(__file__).resolve().parent.parent
# SPB200_LIB selects another build of the same library (e.g. one compiled
# with different tuning flags); the default is the in-tree build.
LIB_PATH = Path(os.environ["SPB200_LIB"]) if os.environ.get("SPB200_LIB") else PKG / "lib" / "libshannon_prime_b200.so"

SP_MAX_BANDS = 16
SP_OK, SP_ERR_ARG, SP_ERR_CUDA, SP_ERR_UNSUPPORTED, SP_ERR_TIMEOUT = 0, -1, -2, -3, -4
SP_DTYPE_F32, SP_DTYPE_F16, SP_DTYPE_BF16 = 0, 1, 2


class SpConfig(C.Structure):
    _fields_ = [
        ("head_dim", C.c_int), ("n_layers", C.c_int), ("n_heads_kv", C.c_int),
        ("k_n_bands", C.c_int), ("k_band_bits", C.c_int * SP_MAX_BANDS),
        ("v_n_bands", C.c_int), ("v_band_bits", C.c_int * SP_MAX_BANDS),
        ("use_mobius_mask", C.c_int),
        ("k_ternary_mask", C.c_uint32), ("v_ternary_mask", C.c_uint32),
        ("use_fp8", C.c_int),
    ]


class SpBandConfig(C.Structure):
    _fields_ = [
        ("head_dim", C.c_int), ("n_bands", C.c_int),
        ("band_bits", C.c_int * SP_MAX_BANDS),
        ("band_size", C.c_int), ("total_bytes", C.c_int),
    ]


class SpCudaCache(C.Structure):
    _fields_ = [
        ("config", SpConfig), ("k_bands", SpBandConfig), ("v_bands", SpBandConfig),
        ("d_k_cache", C.c_void_p), ("d_v_cache", C.c_void_p), ("max_seq_len", C.c_int),
        ("d_mobius_order", C.c_void_p), ("d_mobius_inv", C.c_void_p),
        ("d_scratch", C.c_void_p), ("stream", C.c_void_p),
        ("n_slots", C.c_int), ("device", C.c_int),
        ("d_attn_ws", C.c_void_p), ("attn_ws_bytes", C.c_size_t),
        ("attn_max_q_heads", C.c_int), ("attn_ws_layers", C.c_int),
        ("d_status", C.c_void_p),
    ]


class SpSqfreeCache(C.Structure):
    _fields_ = [
        ("config", SpConfig), ("pad_dim", C.c_int), ("sk_k", C.c_int), ("n_res", C.c_int),
        ("n_terms", C.c_int), ("residual_bits", C.c_int), ("use_spinor", C.c_int),
        ("use_skel_mobius", C.c_int), ("k_bands", SpBandConfig), ("v_bands", SpBandConfig),
        ("d_skeleton_idx", C.c_void_p), ("d_residual_idx", C.c_void_p),
        ("d_csr_offsets", C.c_void_p), ("d_csr_skel_slot", C.c_void_p),
        ("d_csr_mu_sign", C.c_void_p), ("d_vilenkin_factors", C.c_void_p),
        ("n_factors", C.c_int), ("d_k_cache", C.c_void_p), ("d_v_cache", C.c_void_p),
        ("bytes_per_pos_k", C.c_int), ("bytes_per_pos_v", C.c_int), ("max_seq_len", C.c_int),
        ("n_slots", C.c_int),
        ("d_pad_scratch", C.c_void_p), ("d_coeff_scratch", C.c_void_p),
        ("d_skel_scratch", C.c_void_p), ("d_pred_scratch", C.c_void_p),
        ("d_dev_scratch", C.c_void_p), ("d_levels_scratch", C.c_void_p),
        ("d_mag_scratch", C.c_void_p), ("d_actual_scratch", C.c_void_p),
        ("d_sheet_scratch", C.c_void_p), ("stream", C.c_void_p),
        ("device", C.c_int), ("d_tables", C.c_void_p), ("d_attn_ws", C.c_void_p),
        ("attn_ws_bytes", C.c_size_t), ("csr_max_terms", C.c_int),
        ("lane_max_terms", C.c_int),
    ]


class SpHierCache(C.Structure):
    _fields_ = [
        ("config", SpConfig), ("pad_dim", C.c_int), ("n_skeleton", C.c_int),
        ("n_target", C.c_int), ("target_res_bits", C.c_int), ("n_slots", C.c_int),
        ("max_seq_len", C.c_int), ("d_W", C.c_void_p), ("d_skeleton_idx", C.c_void_p),
        ("d_target_idx", C.c_void_p), ("d_vilenkin_factors", C.c_void_p), ("n_factors", C.c_int),
        ("skel_bands", SpBandConfig), ("d_skel_band_bits", C.c_void_p),
        ("d_k_cache", C.c_void_p), ("d_v_cache", C.c_void_p),
        ("bytes_per_pos_k", C.c_int), ("bytes_per_pos_v", C.c_int),
        ("d_pad_scratch", C.c_void_p), ("d_coeff_scratch", C.c_void_p),
        ("d_skel_scratch", C.c_void_p), ("d_pred_scratch", C.c_void_p),
        ("d_dev_scratch", C.c_void_p), ("d_mag_scratch", C.c_void_p),
        ("d_levels_scratch", C.c_void_p), ("stream", C.c_void_p),
        ("device", C.c_int), ("d_tables", C.c_void_p), ("d_vrows", C.c_void_p), ("d_recon", C.c_void_p),
        ("d_status", C.c_void_p),
    ]


class SpColdLayer(C.Structure):
    """sp_cuda_cold_layer_t: pinned host mirror of one layer slab."""
    _fields_ = [
        ("h_pinned", C.c_void_p), ("capacity", C.c_int64), ("packed_stride", C.c_int),
        ("n_heads", C.c_int), ("write_head", C.c_int64), ("oldest_pos", C.c_int64),
        ("newest_pos", C.c_int64), ("ring_mode", C.c_bool), ("initialized", C.c_bool),
    ]


class SpLlamaParams(C.Structure):
    _fields_ = [
        ("head_dim", C.c_int), ("n_layers", C.c_int), ("n_heads_kv", C.c_int),
        ("max_seq_len", C.c_int), ("backend", C.c_int), ("gpu_context", C.c_void_p),
        ("arch_name", C.c_char_p),
    ]


class SpLlamaMemory(C.Structure):
    _fields_ = [
        ("compressed_bytes", C.c_size_t), ("baseline_bytes", C.c_size_t),
        ("compression_ratio", C.c_float), ("n_positions", C.c_int),
    ]


# (name, restype, argtypes) of every symbol the headers declare.
_V, _I, _P, _F = None, C.c_int, C.c_void_p, C.c_float
_CC = C.POINTER(SpCudaCache)
SIGNATURES = {
    # shannon_prime.h (host utilities)
    "sp_config_init": (_V, [C.POINTER(SpConfig), _I, _I, _I]),
    "sp_band_config_init": (_I, [C.POINTER(SpBandConfig), _I, _I, C.POINTER(C.c_int)]),
    "sp_band_span": (_V, [C.POINTER(SpBandConfig), _I, C.POINTER(C.c_int), C.POINTER(C.c_int)]),
    "sp_mobius_mask_init": (_I, [_P, _I]),
    "sp_mobius_mask_free": (_V, [_P]),
    "sp_correlation_f32": (_F, [_P, _P, _I]),
    "sp_config_print": (_V, [C.POINTER(SpConfig)]),
    # shannon_prime_cuda.h
    "sp_cuda_cache_init": (_I, [_CC, C.POINTER(SpConfig), _I, _P]),
    "sp_cuda_cache_free": (_V, [_CC]),
    "sp_cuda_write_k": (_V, [_CC, _I, _I, _I, _P]),
    "sp_cuda_write_v": (_V, [_CC, _I, _I, _I, _P]),
    "sp_cuda_write_k_batch": (_V, [_CC, _I, _I, _I, _I, _P]),
    "sp_cuda_write_v_batch": (_V, [_CC, _I, _I, _I, _I, _P]),
    "sp_cuda_write_kv_tokens": (_I, [_CC, _I, _I, _I, _P, _P, _I]),
    "sp_cuda_read_k": (_V, [_CC, _I, _I, _I, _P]),
    "sp_cuda_read_v": (_V, [_CC, _I, _I, _I, _P]),
    "sp_cuda_read_k_batch": (_V, [_CC, _I, _I, _I, _I, _P]),
    "sp_cuda_read_v_batch": (_V, [_CC, _I, _I, _I, _I, _P]),
    "sp_cuda_read_batch_partial": (_I, [_CC, _I, _I, _I, _I, _I, _P, _I]),
    "sp_cuda_read_kv_tokens": (_I, [_CC, _I, _I, _I, _I, _I, _P, _I]),
    "sp_cuda_attn_decode": (_I, [_CC, _I, _I, _P, _I, _I, _F, _P, _I, _P]),
    "sp_cuda_attn_decode_allgather": (_I, [_CC, _I, _I, _P, _I, _I, _F, _I, _P, _P, _P, _P, _I, C.c_longlong,
                                           C.c_longlong, _I, _I, C.c_uint, _P]),
    "sp_cuda_kq_scores": (_I, [_P, _I, _I, _I, _I, _P, _I, C.c_longlong, _I, _P, C.c_longlong, _P]),
    "sp_cuda_kq_scores_strided": (_I, [_P, C.c_longlong, _I, _I, _I, _I, _I, _P, _I, C.c_longlong, C.c_longlong, _I,
                                       _P, C.c_longlong, C.c_longlong, _P]),
    "sp_cuda_attn_decode_noalloc": (_I, [_P, _P, _I, C.POINTER(SpBandConfig),
                                         C.POINTER(SpBandConfig), _P, _I, _I, _I, _P, _I, _I,
                                         _F, _P, _I, _P]),
    "sp_cuda_attn_decode_noalloc_status": (_I, [C.POINTER(C.c_uint), _I, _P]),
    "sp_fnv1a64": (C.c_uint64, [C.c_char_p, C.c_size_t]),
    "sp_cuda_dual_merge": (_I, [_P, _P, _P, _I, _I, _P, _P]),
    "sp_ggml_attn_decode": (_I, [_CC, _I, _P, _I, _P, _P, _P, _I, _P, _P, _F, _I, _I, _P]),
    "sp_cuda_cache_save": (_I, [_CC, C.c_char_p, _I, C.c_uint64, _I]),
    "sp_cuda_cache_load": (_I, [_CC, C.c_char_p, C.c_uint64]),
    "sp_cuda_cache_load_partial": (_I, [_CC, C.c_char_p, C.c_uint64, _I]),
    "sp_cuda_sqfree_cache_init": (_I, [C.POINTER(SpSqfreeCache), C.POINTER(SpConfig), _I, _I, _I, _P]),
    "sp_cuda_sqfree_cache_init_ex": (_I, [C.POINTER(SpSqfreeCache), C.POINTER(SpConfig), _I, _I, _I,
                                          _F, _P]),
    "sp_cuda_sqfree_cache_free": (_V, [C.POINTER(SpSqfreeCache)]),
    "sp_cuda_sqfree_write_k": (_V, [C.POINTER(SpSqfreeCache), _I, _I, _I, _P]),
    "sp_cuda_sqfree_write_v": (_V, [C.POINTER(SpSqfreeCache), _I, _I, _I, _P]),
    "sp_cuda_sqfree_read_k": (_V, [C.POINTER(SpSqfreeCache), _I, _I, _I, _P]),
    "sp_cuda_sqfree_read_v": (_V, [C.POINTER(SpSqfreeCache), _I, _I, _I, _P]),
    "sp_cuda_sqfree_read_k_batch": (_V, [C.POINTER(SpSqfreeCache), _I, _I, _I, _I, _P]),
    "sp_cuda_sqfree_read_kv_tokens": (_I, [C.POINTER(SpSqfreeCache), _I, _I, _I, _I, _I, _P]),
    "sp_cuda_sqfree_read_v_batch": (_V, [C.POINTER(SpSqfreeCache), _I, _I, _I, _I, _P]),
    "sp_cuda_sqfree_write_kv_tokens": (_I, [C.POINTER(SpSqfreeCache), _I, _I, _I, _I, _P, _P, _I]),
    "sp_cuda_sqfree_attn_decode": (_I, [C.POINTER(SpSqfreeCache), _I, _I, _P, _I, _I, _F, _P, _P]),
    "sp_cuda_hier_cache_init": (_I, [C.POINTER(SpHierCache), C.POINTER(SpConfig), _I, _I, _I, _I,
                                     _P, _P, C.POINTER(SpBandConfig), _I, _I, _P]),
    "sp_cuda_hier_cache_free": (_V, [C.POINTER(SpHierCache)]),
    "sp_cuda_hier_cache_upload_W": (_I, [C.POINTER(SpHierCache), _P]),
    "sp_cuda_hier_write_k": (_V, [C.POINTER(SpHierCache), _I, _I, _I, _P]),
    "sp_cuda_hier_write_v": (_V, [C.POINTER(SpHierCache), _I, _I, _I, _P]),
    "sp_cuda_hier_read_k": (_V, [C.POINTER(SpHierCache), _I, _I, _I, _P]),
    "sp_cuda_hier_read_v": (_V, [C.POINTER(SpHierCache), _I, _I, _I, _P]),
    "sp_cuda_hier_write_kv_tokens": (_I, [C.POINTER(SpHierCache), _I, _I, _I, _I, _P, _P, _I]),
    "sp_cuda_hier_read_kv_tokens": (_I, [C.POINTER(SpHierCache), _I, _I, _I, _I, _P, _P]),
    "sp_cuda_vht2_forward": (_V, [_P, _I, _I, _P]),
    "sp_cuda_mobius_reorder": (_V, [_P, _P, _I, _I, _P]),
    "sp_cuda_mobius_unreorder": (_V, [_P, _P, _I, _I, _P]),
    "sp_cuda_band_quantize": (_V, [_P, _P, C.POINTER(SpBandConfig), _I, _P]),
    "sp_cuda_band_dequantize": (_V, [_P, _P, C.POINTER(SpBandConfig), _I, _P]),
    "sp_cuda_print_memory": (_V, [_CC]),
    "sp_cuda_last_error": (_I, []),
    "sp_cuda_last_error_string": (C.c_char_p, []),
    "sp_cuda_abi_struct_size": (_I, [_I]),
    "sp_cuda_cold_layer_init": (_I, [C.POINTER(SpColdLayer), C.c_int64, _I, _I]),
    "sp_cuda_cold_layer_free": (_V, [C.POINTER(SpColdLayer)]),
    "sp_cuda_cold_writeback": (_I, [C.POINTER(SpColdLayer), _P, _I, _I, _P]),
    "sp_cuda_cold_restore": (_I, [C.POINTER(SpColdLayer), _P, _I, _P]),
    "sp_cuda_d2h_async": (_V, [_P, _P, C.c_int64, _P]),
    "sp_cuda_h2d_async": (_V, [_P, _P, C.c_int64, _P]),
    "sp_cuda_attn_force_impl": (_V, [_I]),
    "sp_cuda_attn_profile": (_V, [_I]),
    "sp_cuda_attn_last_kernel_ms": (_F, []),
    "sp_cuda_attn_last_splits": (_I, []),
    # shannon_prime_llama.h
    "sp_llama_init": (_P, [C.POINTER(SpLlamaParams)]),
    "sp_llama_init_with_role": (_P, [C.POINTER(SpLlamaParams), _I]),
    "sp_llama_init_config": (_P, [C.POINTER(SpLlamaParams), C.POINTER(SpConfig)]),
    "sp_llama_free": (_V, [_P]),
    "sp_llama_write_kv": (_V, [_P, _I, _I, _I, _P, _P]),
    "sp_llama_write_k": (_V, [_P, _I, _I, _I, _P]),
    "sp_llama_write_v": (_V, [_P, _I, _I, _I, _P]),
    "sp_llama_write_k_batch": (_V, [_P, _I, _I, _I, _I, _P]),
    "sp_llama_write_v_batch": (_V, [_P, _I, _I, _I, _I, _P]),
    "sp_llama_read_k": (_V, [_P, _I, _I, _I, _P]),
    "sp_llama_read_v": (_V, [_P, _I, _I, _I, _P]),
    "sp_llama_read_k_partial": (_V, [_P, _I, _I, _I, _P, _I]),
    "sp_llama_read_v_partial": (_V, [_P, _I, _I, _I, _P, _I]),
    "sp_llama_read_k_batch": (_V, [_P, _I, _I, _I, _I, _P]),
    "sp_llama_read_v_batch": (_V, [_P, _I, _I, _I, _I, _P]),
    "sp_llama_clear_range": (_V, [_P, _I, _I]),
    "sp_llama_memory": (SpLlamaMemory, [_P]),
    "sp_llama_validate_k": (_F, [_P, _P, _I]),
    "sp_llama_print_config": (_V, [_P]),
    "sp_llama_get_freq_factors": (_P, [_P]),
    "sp_llama_get_n_freqs": (_I, [_P]),
    "sp_llama_get_hexagon_k_buf": (_P, [_P, _I, _I]),
    "sp_llama_get_hexagon_k_total_bytes": (_I, [_P]),
    "sp_llama_get_cuda_cache": (_P, [_P]),
    "sp_llama_attn_decode": (_I, [_P, _I, _I, _P, _I, _I, _F, _P, _I]),
    "sp_llama_write_kv_tokens": (_I, [_P, _I, _I, _I, _P, _P]),
}

_lib = None


def lib() -> C.CDLL:
    """Load the in-tree library (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing: run shannon-prime-llama_b200/build.py")
        L = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            if os.environ.get("SPB200_LIB") and not hasattr(L, name):
                continue        # another build may predate some entry points
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        for which, st in enumerate((SpConfig, SpBandConfig, SpCudaCache, SpSqfreeCache, SpHierCache,
                                     SpColdLayer)):
            if L.sp_cuda_abi_struct_size(which) != C.sizeof(st):
                raise RuntimeError(f"struct mirror {st.__name__} does not match the C ABI")
        _lib = L
    return _lib


def last_error() -> tuple[int, str]:
    L = lib()
    return L.sp_cuda_last_error(), L.sp_cuda_last_error_string().decode()


def check(rc: int | None = None, what: str = "") -> None:
    """Raise on a non-zero status (rc, or the thread's last status)."""
    code, msg = last_error()
    if rc is not None and rc != 0:
        raise RuntimeError(f"{what}: status {rc}: {msg}")
    if rc is None and code != 0:
        raise RuntimeError(f"{what}: status {code}: {msg}")


def make_config(head_dim: int, n_layers: int, n_heads_kv: int, k_bits=None, v_bits=None,
                mobius: bool = True) -> SpConfig:
    cfg = SpConfig()
    lib().sp_config_init(C.byref(cfg), head_dim, n_layers, n_heads_kv)
    if k_bits is not None:
        cfg.k_n_bands = len(k_bits)
        for i, b in enumerate(k_bits):
            cfg.k_band_bits[i] = b
    if v_bits is not None:
        cfg.v_n_bands = len(v_bits)
        for i, b in enumerate(v_bits):
            cfg.v_band_bits[i] = b
    cfg.use_mobius_mask = 1 if mobius else 0
    return cfg


def _ptr(t) -> int:
    return 0 if t is None else t.data_ptr()


def _stream_ptr(stream) -> int:
    return 0 if stream is None else stream.cuda_stream


from .cache import Cache  # noqa: E402,F401
