"""Partition of the compressed cache across the GPUs of one box.

The cache is sharded by (layer, KV head): attention for a KV head needs only
that head's slots and its GQA query heads, so no cache byte ever crosses
NVLink; each decode step ends with one all-gather of the per-head fp16
outputs.  The reference has no multi-GPU code on this path; its only notion
is a layer -> GPU map, layer L on GPU floor(L * n_gpus / n_layer)
(src/engine/engine.h:55-68), which this generalises to heads as well.

    world <= H and H % world == 0 : rank r owns KV heads h with h % world == r,
                                    every layer;
    world >  H and world % H == 0 : rank r owns KV head r % H and the
                                    (r // H)-th of world // H contiguous layer
                                    ranges (config 3: 4 heads x 2 halves on 8).
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class Shard:
    rank: int
    layer0: int
    n_layers: int
    heads: tuple          # KV heads owned (ascending)

    def q_heads(self, group: int) -> list:
        """Query heads served, in output order."""
        return [h * group + g for h in self.heads for g in range(group)]


def partition(n_layers: int, n_kv_heads: int, world: int) -> list:
    if world < 1:
        raise ValueError("world must be >= 1")
    if world <= n_kv_heads and n_kv_heads % world == 0:
        return [Shard(r, 0, n_layers, tuple(h for h in range(n_kv_heads) if h % world == r))
                for r in range(world)]
    if world > n_kv_heads and world % n_kv_heads == 0:
        parts = world // n_kv_heads
        if n_layers < parts:
            raise ValueError(f"{n_layers} layers cannot be split {parts} ways")
        bounds = [n_layers * i // parts for i in range(parts + 1)]
        out = []
        for r in range(world):
            p = r // n_kv_heads
            out.append(Shard(r, bounds[p], bounds[p + 1] - bounds[p], (r % n_kv_heads,)))
        return out
    raise ValueError(f"cannot shard {n_kv_heads} KV heads over {world} GPUs")


def max_shard_shape(shards: list, group: int) -> tuple:
    """(layers, q heads) of the largest shard: the padded all-gather block."""
    return (max(s.n_layers for s in shards), max(len(s.heads) for s in shards) * group)


def assemble(blocks, shards: list, n_layers: int, n_q_heads: int, group: int, out):
    """Scatter gathered per-rank output blocks [Lmax][Qmax][hd] into the full
    output out[n_layers][n_q_heads][hd] (numpy arrays or torch tensors)."""
    for s, blk in zip(shards, blocks):
        qh = s.q_heads(group)
        for i, q in enumerate(qh):
            out[s.layer0:s.layer0 + s.n_layers, q] = blk[:s.n_layers, i]
    return out
