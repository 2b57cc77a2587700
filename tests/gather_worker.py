"""Worker of tests/test_gpu_gather.py (one process per GPU, run by
torch.distributed.run): the fused decode + all-gather over peer memory
against each rank's own single-GPU decode of the same shard.

Cache: 3 layers x 8 KV heads x hd 128, 700 positions (a partial last tile),
4 query heads per KV head; rank r owns KV heads h % world == r.  Every rank
checks, for three consecutive calls (epochs 1..3) with a barrier between
them, that every row of its gathered buffer equals (bit for bit) the owning
rank's local decode; then for eight calls issued back to back with no
barrier or host synchronisation between them, each with different queries,
and with one rank delayed by a spin on its stream, that every call's rows
(copied out on the stream right after the call) are right; and that the
cache's status word stays clear."""
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)), "..", "shannon-prime-llama_b200"))
import spb200  # noqa: E402
from spb200 import synth  # noqa: E402
from spb200.cache import Cache  # noqa: E402
from spb200.gather import PeerGather  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", device_id=dev)
    L, H, G, HD, T = 3, 8, 4, 128, 700
    heads = [h for h in range(H) if h % world == rank]
    cache = Cache(HD, L, len(heads), T)
    for layer in range(L):
        k = np.stack([synth.kv_slot_np(21, layer, h, T, HD)[0] for h in heads], 1)
        v = np.stack([synth.kv_slot_np(21, layer, h, T, HD)[1] for h in heads], 1)
        cache.write_kv_tokens(layer, 0, torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda())
    q_all = torch.from_numpy(synth.q_np(21, L, H * G, HD, 1.0 / np.sqrt(HD))).cuda()
    qcols = [h * G + g for h in heads for g in range(G)]
    q = q_all[:, qcols].contiguous()
    local = torch.empty(L, len(qcols), HD, dtype=torch.float16, device=dev)
    cache.attn_decode(0, L, q, T, local, logit_scale=0.8)
    # every rank's local rows, for the check
    rows = [torch.empty_like(local) for _ in range(world)]
    dist.all_gather(rows, local)
    expect = torch.empty(L, H * G, HD, dtype=torch.float16, device=dev)
    for r in range(world):
        cols = [h * G + g for h in range(H) if h % world == r for g in range(G)]
        expect[:, cols] = rows[r]
    pg = PeerGather(L, H * G, HD, dev)
    dst_layer = torch.arange(L, dtype=torch.int32, device=dev)
    dst_qhead = torch.tensor(qcols, dtype=torch.int32, device=dev)
    for _ in range(3):
        pg.out.fill_(float("nan"))          # every row must be rewritten by this call
        torch.cuda.synchronize()
        dist.barrier()
        pg.decode(C_byref(cache), 0, L, q, len(qcols), T, dst_layer, dst_qhead, logit_scale=0.8)
        torch.cuda.synchronize()
        if not torch.equal(pg.out, expect):
            bad = (pg.out != expect).nonzero()[:5].tolist()
            print(f"rank {rank} epoch {pg.epoch}: mismatch at {bad}", flush=True)
            sys.exit(1)
        dist.barrier()
    # back to back: queries differ per call, so a late overwrite would show
    n_bb = 8
    qs = [(q.float() * (1.0 + 0.07 * e)).half() for e in range(n_bb)]
    expects = []
    for e in range(n_bb):
        loc = torch.empty_like(local)
        cache.attn_decode(0, L, qs[e], T, loc, logit_scale=0.8)
        rows = [torch.empty_like(loc) for _ in range(world)]
        dist.all_gather(rows, loc)
        ex = torch.empty(L, H * G, HD, dtype=torch.float16, device=dev)
        for r in range(world):
            cols = [h * G + g for h in range(H) if h % world == r for g in range(G)]
            ex[:, cols] = rows[r]
        expects.append(ex)
    torch.cuda.synchronize()
    dist.barrier()
    got = []
    for e in range(n_bb):
        if rank == 1 and e % 3 == 1:
            torch.cuda._sleep(2_000_000)        # this rank lags behind on its stream
        pg.decode(C_byref(cache), 0, L, qs[e], len(qcols), T, dst_layer, dst_qhead, logit_scale=0.8)
        got.append(pg.out.clone())
    torch.cuda.synchronize()
    for e in range(n_bb):
        if not torch.equal(got[e], expects[e]):
            bad = (got[e] != expects[e]).nonzero()[:5].tolist()
            print(f"rank {rank} back-to-back call {e}: mismatch at {bad}", flush=True)
            sys.exit(1)
    dist.barrier()
    status = torch.zeros(4, dtype=torch.int32)
    spb200.lib().sp_cuda_d2h_async(status.data_ptr(), cache.cc.d_status, 16, None)
    torch.cuda.synchronize()
    if int(status[0]) != 0:
        print(f"rank {rank}: status word {int(status[0])}", flush=True)
        sys.exit(1)
    dist.barrier()
    if rank == 0:
        print("GATHER_OK", flush=True)
    dist.destroy_process_group()


def C_byref(cache):
    import ctypes
    return ctypes.byref(cache.cc)


if __name__ == "__main__":
    main()
