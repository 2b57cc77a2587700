"""Peer-memory gather buffers for the fused decode + all-gather
(sp_cuda_attn_decode_allgather): one symmetric-memory buffer per rank holding
two copies of the gathered fp16 outputs [n_rows][n_q_total][head_dim] (odd
and even epochs) followed by a [32] uint32 flag array, mapped into every rank
of the group.  With two copies a rank may start the next call while a slower
rank still reads the current one, as long as each rank's reads are
stream-ordered before its own next call.

The caller allocates it once per (shape, group), then passes `peers_dev`
(device array of every rank's buffer address), the buffer's own address,
`flags_offset` and the next epoch to each call.  torch.distributed must be
initialised (one process per GPU, NCCL)."""
from __future__ import annotations

import ctypes as C

from . import check, lib

MAX_WORLD = 32


class PeerGather:
    """Symmetric gather buffer of n_rows x n_q_total x head_dim fp16."""

    def __init__(self, n_rows: int, n_q_total: int, head_dim: int, device, group=None):
        import torch
        import torch.distributed as dist
        import torch.distributed._symmetric_memory as symm

        self.group = group if group is not None else dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        if self.world > MAX_WORLD:
            raise ValueError(f"world {self.world} > {MAX_WORLD}")
        self.shape = (n_rows, n_q_total, head_dim)
        out_bytes = n_rows * n_q_total * head_dim * 2
        self.epoch_stride = (out_bytes + 255) // 256 * 256
        self.flags_offset = 2 * self.epoch_stride
        self.buf = symm.empty(self.flags_offset + 4 * MAX_WORLD, dtype=torch.uint8, device=device)
        self.buf.zero_()
        torch.cuda.synchronize(device)
        self.hdl = symm.rendezvous(self.buf, self.group)
        dist.barrier(group=self.group)          # every rank's flags are zero before any call
        torch.cuda.synchronize(device)
        self.peers_dev = int(self.hdl.buffer_ptrs_dev)
        self._copies = [self.buf[c * self.epoch_stride:c * self.epoch_stride + out_bytes]
                        .view(torch.float16).view(*self.shape) for c in range(2)]
        self.epoch = 0

    @property
    def out(self):
        """The gathered rows of the latest call (epoch)."""
        return self._copies[self.epoch & 1]

    def decode(self, cc, layer0: int, n_layers: int, q, n_q_heads: int, kv_len: int, dst_layer, dst_qhead,
               logit_scale: float = 1.0, max_bands: int = -1, stream=None) -> None:
        """One fused decode + all-gather on the sp_cuda_cache_t `cc` (a
        ctypes pointer or byref).  dst_layer / dst_qhead: int32 CUDA tensors
        (destination row of each local layer and query head)."""
        self.epoch += 1
        s = 0 if stream is None else (stream if isinstance(stream, int) else stream.cuda_stream)
        rc = lib().sp_cuda_attn_decode_allgather(
            cc, layer0, n_layers, q.data_ptr(), n_q_heads, kv_len, logit_scale, max_bands,
            self.buf.data_ptr(), self.peers_dev, dst_layer.data_ptr(), dst_qhead.data_ptr(),
            self.shape[1], self.flags_offset, self.epoch_stride, self.rank, self.world,
            C.c_uint(self.epoch & 0xffffffff), s)
        check(rc, "sp_cuda_attn_decode_allgather")
