"""Python mirror of the sp_cuda_* cache interface (shannon_prime_cuda.h), for
tests and the benchmark.  Every method calls straight into the C-ABI."""
from __future__ import annotations

import ctypes as C

from . import (SP_DTYPE_BF16, SP_DTYPE_F16, SP_DTYPE_F32, SpCudaCache, _ptr, _stream_ptr,
               check, lib, make_config)


def _dtype_code(t) -> int:
    import torch
    return {torch.float32: SP_DTYPE_F32, torch.float16: SP_DTYPE_F16,
            torch.bfloat16: SP_DTYPE_BF16}[t.dtype]


class Cache:
    """A GPU-resident ship-path cache (sp_cuda_cache_t) on the current device."""

    def __init__(self, head_dim: int, n_layers: int, n_heads_kv: int, max_seq_len: int,
                 k_bits=None, v_bits=None, mobius: bool = True, stream=None):
        self.cfg = make_config(head_dim, n_layers, n_heads_kv, k_bits, v_bits, mobius)
        self.cc = SpCudaCache()
        self.stream = stream
        rc = lib().sp_cuda_cache_init(C.byref(self.cc), C.byref(self.cfg), max_seq_len,
                                      _stream_ptr(stream))
        check(rc, "sp_cuda_cache_init")
        self.head_dim, self.n_layers, self.n_heads_kv = head_dim, n_layers, n_heads_kv
        self.max_seq_len = self.cc.max_seq_len

    # -- sizes ---------------------------------------------------------------
    @property
    def k_bytes(self) -> int:
        return self.cc.k_bands.total_bytes

    @property
    def v_bytes(self) -> int:
        return self.cc.v_bands.total_bytes

    def free(self) -> None:
        if self.cc.d_k_cache:
            lib().sp_cuda_cache_free(C.byref(self.cc))

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass

    # -- raw slabs -----------------------------------------------------------
    def slab(self, which: int):
        """The packed K (0) or V (1) slab as a uint8 CUDA tensor view
        [n_slots][max_seq_len][bytes] (shares memory with the cache)."""
        import torch
        nbytes = self.k_bytes if which == 0 else self.v_bytes
        n = self.cc.n_slots * self.max_seq_len * nbytes
        ptr = self.cc.d_k_cache if which == 0 else self.cc.d_v_cache
        return _wrap_device(ptr, n, torch.uint8).view(self.cc.n_slots, self.max_seq_len, nbytes)

    # -- write / read ----------------------------------------------------------
    def write_kv_tokens(self, layer: int, start_pos: int, k, v) -> None:
        """k, v: CUDA tensors [n_tokens][n_heads_kv][head_dim] (f32/f16/bf16)."""
        t = k if k is not None else v
        rc = lib().sp_cuda_write_kv_tokens(C.byref(self.cc), layer, start_pos, t.shape[0],
                                           _ptr(k), _ptr(v), _dtype_code(t))
        check(rc, "sp_cuda_write_kv_tokens")

    def write_batch(self, which: int, layer: int, head: int, start_pos: int, vecs) -> None:
        f = lib().sp_cuda_write_k_batch if which == 0 else lib().sp_cuda_write_v_batch
        f(C.byref(self.cc), layer, head, start_pos, vecs.shape[0], vecs.data_ptr())
        check(None, "sp_cuda_write_batch")

    def read_batch(self, which: int, layer: int, head: int, start_pos: int, out,
                   max_bands: int = -1) -> None:
        rc = lib().sp_cuda_read_batch_partial(C.byref(self.cc), which, layer, head, start_pos,
                                              out.shape[0], out.data_ptr(), max_bands)
        check(rc, "sp_cuda_read_batch_partial")

    def attn_decode(self, layer0: int, n_layers: int, q, kv_len: int, out,
                    logit_scale: float = 1.0, max_bands: int = -1, stream=None) -> None:
        """q, out: fp16 CUDA tensors [n_layers][n_q_heads][head_dim]."""
        rc = lib().sp_cuda_attn_decode(C.byref(self.cc), layer0, n_layers, q.data_ptr(),
                                       q.shape[1], kv_len, logit_scale, out.data_ptr(),
                                       max_bands, _stream_ptr(stream))
        check(rc, "sp_cuda_attn_decode")


def _wrap_device(ptr: int, nbytes: int, dtype):
    """A torch CUDA tensor aliasing nbytes of device memory at ptr."""
    import torch

    class _Holder:
        def __init__(self, p, n):
            self.__cuda_array_interface__ = {
                "shape": (n,), "typestr": "|u1", "data": (p, False), "version": 3}

    return torch.as_tensor(_Holder(ptr, nbytes), device="cuda").view(dtype)
