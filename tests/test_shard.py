"""Multi-GPU sharding logic on CPU ranks (gloo, world size 2 and 4): each
rank attends over its own (layer, KV head) shard of a compressed cache with
the oracle, the per-head outputs are all-gathered, and the assembled result
must equal the single-process attention over the whole cache bit for bit."""
import os
import socket

import numpy as np
import pytest

import oracle as O
from spb200 import shard, synth

KB, VB = [5, 5, 4, 3], [3]
N, T = 128, 96


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _cache(n_layers, H, seed):
    kp = np.zeros((n_layers, H, T, 76), np.uint8)
    vp = np.zeros((n_layers, H, T, 50), np.uint8)
    for layer in range(n_layers):
        for h in range(H):
            k, v = synth.kv_slot_np(seed, layer, h, T, N)
            kp[layer, h] = O.ship_write(k, KB, True, 1)
            vp[layer, h] = O.ship_write(v, VB, False, 1)
    return kp, vp


def _attend(kp, vp, q, layers, heads, group):
    """Oracle attention of the given layers / KV heads -> [len(layers)][heads*group][N]."""
    out = np.zeros((len(layers), len(heads) * group, N), np.float32)
    for i, layer in enumerate(layers):
        qs = np.stack([q[layer, h * group + g] for h in heads for g in range(group)])
        out[i] = O.attn_decode(kp[layer][list(heads)], vp[layer][list(heads)], N, KB, VB, True,
                               qs, T, 1.0, 1)
    return out


def _rank(rank, world, port, n_layers, H, group, result):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        kp, vp = _cache(n_layers, H, seed=11)
        q = synth.q_np(11, n_layers, H * group, N, 1 / np.sqrt(128)).astype(np.float16)
        shards = shard.partition(n_layers, H, world)
        me = shards[rank]
        Lm, Qm = shard.max_shard_shape(shards, group)
        blk = np.zeros((Lm, Qm, N), np.float32)
        mine = _attend(kp, vp, q, range(me.layer0, me.layer0 + me.n_layers), me.heads, group)
        blk[:me.n_layers, :len(me.heads) * group] = mine
        gathered = [torch.zeros(Lm, Qm, N) for _ in range(world)]
        dist.all_gather(gathered, torch.from_numpy(blk))
        if rank == 0:
            full = np.zeros((n_layers, H * group, N), np.float32)
            shard.assemble([g.numpy() for g in gathered], shards, n_layers, H * group, group, full)
            ref = _attend(kp, vp, q, range(n_layers), range(H), group)
            result.put(bool(np.array_equal(full, ref)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,n_layers,H,group", [(2, 3, 4, 4), (4, 4, 2, 2)])
def test_sharded_decode_matches_single_process(world, n_layers, H, group):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    result = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, n_layers, H, group, result))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert result.get(timeout=5) is True


def test_partition_rules():
    s = shard.partition(32, 8, 4)
    assert [x.heads for x in s] == [(0, 4), (1, 5), (2, 6), (3, 7)]
    assert all(x.layer0 == 0 and x.n_layers == 32 for x in s)
    s = shard.partition(48, 4, 8)                  # config 3 on 8 GPUs
    assert [(x.heads, x.layer0, x.n_layers) for x in s[:5]] == [
        ((0,), 0, 24), ((1,), 0, 24), ((2,), 0, 24), ((3,), 0, 24), ((0,), 24, 24)]
    covered = sorted((layer, h) for x in s for h in x.heads
                     for layer in range(x.layer0, x.layer0 + x.n_layers))
    assert covered == [(layer, h) for layer in range(48) for h in range(4)]
    with pytest.raises(ValueError):
        shard.partition(32, 8, 3)
