"""Python mirrors of the sqfree+spinor and hierarchical-Vilenkin caches
(sp_cuda_sqfree_* / sp_cuda_hier_* in shannon_prime_cuda.h).  Every method
calls straight into the C-ABI."""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import (SpBandConfig, SpHierCache, SpSqfreeCache, _ptr, _stream_ptr, check, lib,
               make_config)
from .cache import _dtype_code, _wrap_device


class SqfreeCache:
    def __init__(self, head_dim: int, n_layers: int, n_heads_kv: int, max_seq_len: int,
                 bits=(5, 4, 4, 4, 5), residual_bits: int = 3, use_spinor: bool = True,
                 sk_frac: float | None = 0.75, stream=None):
        self.cfg = make_config(head_dim, n_layers, n_heads_kv, list(bits), list(bits), False)
        self.cc = SpSqfreeCache()
        if sk_frac is None:
            rc = lib().sp_cuda_sqfree_cache_init(C.byref(self.cc), C.byref(self.cfg), max_seq_len,
                                                 residual_bits, int(use_spinor), _stream_ptr(stream))
        else:
            rc = lib().sp_cuda_sqfree_cache_init_ex(C.byref(self.cc), C.byref(self.cfg), max_seq_len,
                                                    residual_bits, int(use_spinor), sk_frac,
                                                    _stream_ptr(stream))
        check(rc, "sp_cuda_sqfree_cache_init")
        self.head_dim, self.n_layers, self.n_heads_kv = head_dim, n_layers, n_heads_kv
        self.max_seq_len = max_seq_len

    def free(self):
        if self.cc.d_k_cache:
            lib().sp_cuda_sqfree_cache_free(C.byref(self.cc))

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass

    def slab(self, which: int):
        import torch
        b = self.cc.bytes_per_pos_k if which == 0 else self.cc.bytes_per_pos_v
        n = self.cc.n_slots * self.max_seq_len * b
        ptr = self.cc.d_k_cache if which == 0 else self.cc.d_v_cache
        return _wrap_device(ptr, n, torch.uint8).view(self.cc.n_slots, self.max_seq_len, b)

    def write_kv_tokens(self, layer0: int, start_pos: int, k, v) -> None:
        """k, v: [n_layers][n_tokens][H][hd] (or [n_tokens][H][hd] for one layer)."""
        t = k if k is not None else v
        if t.dim() == 3:
            k = None if k is None else k.unsqueeze(0)
            v = None if v is None else v.unsqueeze(0)
            t = k if k is not None else v
        rc = lib().sp_cuda_sqfree_write_kv_tokens(C.byref(self.cc), layer0, t.shape[0], start_pos,
                                                  t.shape[1], _ptr(k), _ptr(v), _dtype_code(t))
        check(rc, "sp_cuda_sqfree_write_kv_tokens")

    def read_batch(self, which: int, layer: int, head: int, start_pos: int, out) -> None:
        f = lib().sp_cuda_sqfree_read_k_batch if which == 0 else lib().sp_cuda_sqfree_read_v_batch
        f(C.byref(self.cc), layer, head, start_pos, out.shape[0], out.data_ptr())
        check(None, "sp_cuda_sqfree_read_batch")

    def read_kv_tokens(self, which: int, layer0: int, n_layers: int, start_pos: int, out) -> None:
        """out: fp32 CUDA tensor [n_layers][n_tok][n_heads_kv][head_dim]."""
        rc = lib().sp_cuda_sqfree_read_kv_tokens(C.byref(self.cc), which, layer0, n_layers, start_pos,
                                                 out.shape[1], out.data_ptr())
        check(rc, "sp_cuda_sqfree_read_kv_tokens")

    def attn_decode(self, layer0: int, n_layers: int, q, kv_len: int, out,
                    logit_scale: float = 1.0, stream=None) -> None:
        rc = lib().sp_cuda_sqfree_attn_decode(C.byref(self.cc), layer0, n_layers, q.data_ptr(),
                                              q.shape[1], kv_len, logit_scale, out.data_ptr(),
                                              _stream_ptr(stream))
        check(rc, "sp_cuda_sqfree_attn_decode")


class HierCache:
    """Hierarchical cache with the default index sets: skeleton = the first
    pad_dim / p_last coefficients, targets = the rest (ascending)."""

    def __init__(self, head_dim: int, n_layers: int, n_heads_kv: int, max_seq_len: int,
                 pad_dim: int, n_skeleton: int, bits=(5, 5), residual_bits: int = 2, stream=None):
        self.cfg = make_config(head_dim, n_layers, n_heads_kv, None, None, False)
        self.hc = SpHierCache()
        bc = SpBandConfig()
        arr = (C.c_int * len(bits))(*bits)
        check(lib().sp_band_config_init(C.byref(bc), n_skeleton, len(bits), arr), "band config")
        n_target = pad_dim - n_skeleton
        skel = np.arange(n_skeleton, dtype=np.int32)
        targ = np.arange(n_skeleton, pad_dim, dtype=np.int32)
        rc = lib().sp_cuda_hier_cache_init(C.byref(self.hc), C.byref(self.cfg), pad_dim, n_skeleton,
                                           n_target, residual_bits, skel.ctypes.data, targ.ctypes.data,
                                           C.byref(bc), max_seq_len, n_layers * n_heads_kv,
                                           _stream_ptr(stream))
        check(rc, "sp_cuda_hier_cache_init")
        self.head_dim, self.n_layers, self.n_heads_kv = head_dim, n_layers, n_heads_kv
        self.max_seq_len = max_seq_len

    def free(self):
        if self.hc.d_k_cache:
            lib().sp_cuda_hier_cache_free(C.byref(self.hc))

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass

    def upload_W(self, W_all: np.ndarray) -> None:
        w = np.ascontiguousarray(W_all, dtype=np.float16).view(np.uint16)
        check(lib().sp_cuda_hier_cache_upload_W(C.byref(self.hc), w.ctypes.data), "upload_W")

    def slab(self, which: int):
        import torch
        b = self.hc.bytes_per_pos_k
        n = self.hc.n_slots * self.max_seq_len * b
        ptr = self.hc.d_k_cache if which == 0 else self.hc.d_v_cache
        return _wrap_device(ptr, n, torch.uint8).view(self.hc.n_slots, self.max_seq_len, b)

    def write_kv_tokens(self, layer0: int, start_pos: int, k, v) -> None:
        t = k if k is not None else v
        rc = lib().sp_cuda_hier_write_kv_tokens(C.byref(self.hc), layer0, t.shape[0], start_pos,
                                                t.shape[1], _ptr(k), _ptr(v), _dtype_code(t))
        check(rc, "sp_cuda_hier_write_kv_tokens")

    def read_kv_tokens(self, layer0: int, start_pos: int, k_out, v_out) -> None:
        t = k_out if k_out is not None else v_out
        rc = lib().sp_cuda_hier_read_kv_tokens(C.byref(self.hc), layer0, t.shape[0], start_pos,
                                               t.shape[1], _ptr(k_out), _ptr(v_out))
        check(rc, "sp_cuda_hier_read_kv_tokens")
