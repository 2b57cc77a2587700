"""Benchmark of the B200 Shannon-Prime KV-cache hot path.

Headline workload: fused decompress-KQ/V decode attention
in Llama-3-8B shape — 32 layers, 32 query heads / 8 KV heads (GQA 4),
head_dim 128, batch 1, 32768 cached positions compressed on the ship path
(K bands 5,5,4,3; V 3-bit).  One step = one decode token: attention of every
layer's 32 queries over the whole compressed cache (one sp_cuda_attn_decode
call over all 32 layers).  The compressed cache (1.06 GB) is larger than L2
(126 MB), so no flush is needed between steps.  Also measured: ship-path
compression throughput on one full layer (32768 positions x 8 KV heads, fp32
in, 268 MB > L2).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 (torchrun, one rank per GPU): KV heads are partitioned across ranks
(rank r owns heads h with h % N == r, all layers), each rank attends over its
own shard, then one NCCL all-gather of the per-head fp16 outputs
(torch.distributed) completes the step; the time is the max over ranks.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
PKG = ROOT / "shannon-prime-llama_b200"
for _p in (ROOT, PKG, ROOT / "oracle"):
    if str(_p) not in sys.path:
        sys.path.insert(0, str(_p))

# Workload (config 1).
N_LAYERS, N_Q, N_KV, HD, CTX = 32, 32, 8, 128, 32768
KB, VB = [5, 5, 4, 3], [3]
K_ROW, V_ROW = 76, 50
SEED = 1
METRIC = ("fused decompress-KQ/V decode latency per token @32K ctx "
          "(Llama-3-8B shape: 32 layers, 32 Q / 8 KV heads, hd 128, ship K 5/5/4/3 + V 3-bit)")
UNIT = "us/token"
# The workload both arms (this one and --impl reference) report in config.
WORKLOAD = ("config 1: fused decode, %d layers x 32 Q / 8 KV heads x hd 128, ctx 32768, batch 1, "
            "ship K 5/5/4/3 + V 3-bit")
# DRAM bytes (read + write) of one fused-decode launch per cached layer, from
# an ncu capture of the 8-layer case of this workload
# (dram__bytes_read.sum + dram__bytes_write.sum = 264.49 MB + 4.23 MB over 8
# layers, 48-position stages); traffic grows in proportion to the layers
# processed.
NCU_TRAFFIC_PER_LAYER = 268.72e6 / 8


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs, burst copy)"
    return 6650.0, "fallback 6.65 TB/s"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.p = None

    def __enter__(self):
        try:
            self.p = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=self.f, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except OSError:
            self.p = None
        return self

    def __exit__(self, *exc):
        if self.p:
            time.sleep(0.2)
            self.p.terminate()
            self.p.wait()

    def summary(self):
        self.f.flush()
        rows = []
        for line in Path(self.f.name).read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.f.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(rows)}


# ----------------------------------------------------------------- helpers --

def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


def local_heads(rank: int, world: int):
    """KV heads owned by a rank (spb200.shard: h % world == rank for world | 8;
    every rank keeps all layers of config 1)."""
    from spb200 import shard
    sh = shard.partition(N_LAYERS, N_KV, world)[rank]
    assert sh.layer0 == 0 and sh.n_layers == N_LAYERS
    return list(sh.heads)


def cpu_decode_sample(n_threads: int, layers: int = 1):
    """The oracle's decode attention (the reference's fused decompress-KQ
    algorithm plus softmax and V) on `layers` layers of the workload, cache
    built by the oracle itself.  Returns (seconds per layer, threads used)."""
    import numpy as np
    import oracle as O
    from spb200 import synth
    kp = np.zeros((N_KV, CTX, K_ROW), np.uint8)
    vp = np.zeros((N_KV, CTX, V_ROW), np.uint8)
    for h in range(N_KV):
        k, v = synth.kv_slot_np(SEED, 0, h, CTX, HD)
        kp[h] = O.ship_write(k, KB, True, n_threads)
        vp[h] = O.ship_write(v, VB, False, n_threads)
    q = synth.q_np(SEED, 1, N_Q, HD, 1.0 / 128 ** 0.5)[0]
    O.attn_decode(kp, vp, HD, KB, VB, True, q, CTX, 1.0, n_threads)      # warm-up pass
    times = []
    for _ in range(layers):
        t0 = time.perf_counter()
        O.attn_decode(kp, vp, HD, KB, VB, True, q, CTX, 1.0, n_threads)
        times.append(time.perf_counter() - t0)
    return times, n_threads


def cpu_compress_sample(n_threads: int, n_pos: int = 8192):
    """Oracle ship-path compression of n_pos positions x 8 heads (K and V)."""
    import numpy as np
    import oracle as O
    from spb200 import synth
    ks, vs = [], []
    for h in range(N_KV):
        k, v = synth.kv_slot_np(0, 0, h, n_pos, HD)
        ks.append(k)
        vs.append(v)
    k = np.concatenate(ks)
    v = np.concatenate(vs)
    t0 = time.perf_counter()
    O.ship_write(k, KB, True, n_threads)
    O.ship_write(v, VB, False, n_threads)
    dt = time.perf_counter() - t0
    return k.shape[0] / dt, n_threads


# ------------------------------------------------- configs 2 and 4 (extras) --

def _hartley_matrix(pd: int, torch, dev):
    """The staged prime-Hartley (Vilenkin) transform of size pd as a dense
    float64 matrix (Kronecker product of 1/sqrt(p) cas matrices, the first
    prime acting on the fastest index digit)."""
    import math
    M = torch.ones(1, 1, dtype=torch.float64, device=dev)
    r = pd
    for p in (2, 3, 5, 7, 11):
        while r % p == 0:
            k = torch.arange(p, dtype=torch.float64, device=dev)
            ang = 2 * math.pi * torch.outer(k, k) / p
            M = torch.kron((torch.cos(ang) + torch.sin(ang)) / math.sqrt(p), M)
            r //= p
    return M


def measure_sqfree(torch, dev, stream, steps: int, warmup: int, peak: float, scale: int = 1):
    """Config 2: sqfree+spinor, hd 128 (pad 154), skeleton 0.75 (115), bands
    5,4,4,4,5, 3 residual bits, 8 KV heads x 16384 positions x 32 layers,
    seeded as config 0 (seed 2).  Compression throughput over all layers and
    the fused decode step (32 query heads, GQA 4, fp16 queries)."""
    from spb200.sqfree import SqfreeCache
    from spb200 import synth
    L_, H_, T_, hd = max(1, 32 // scale), 8, 16384, 128
    cache = SqfreeCache(hd, L_, H_, T_, residual_bits=3, use_spinor=True, sk_frac=0.75,
                        stream=stream)
    gen = torch.Generator(device=dev)
    inputs = []
    for layer in range(4):
        gen.manual_seed(2 * 1000003 + layer)
        inputs.append(synth.kv_layer_torch(gen, T_, H_, hd, device=dev))
    def compress_all():
        for layer in range(L_):
            k, v = inputs[layer % 4]
            cache.write_kv_tokens(layer, 0, k, v)
    compress_all()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    compress_all()
    e1.record(stream)
    torch.cuda.synchronize()
    c_ms = e0.elapsed_time(e1)
    pairs = L_ * H_ * T_
    bpp = cache.cc.bytes_per_pos_k + cache.cc.bytes_per_pos_v
    q = (torch.randn(L_, 32, hd, device=dev, generator=gen) / hd ** 0.5).half()
    out = torch.empty(L_, 32, hd, dtype=torch.float16, device=dev)
    for _ in range(warmup):
        cache.attn_decode(0, L_, q, T_, out, stream=stream)
    torch.cuda.synchronize()
    e0.record(stream)
    for _ in range(steps):
        cache.attn_decode(0, L_, q, T_, out, stream=stream)
    e1.record(stream)
    torch.cuda.synchronize()
    d_ms = e0.elapsed_time(e1) / steps
    step_bytes = pairs * bpp + 2 * 2 * L_ * 32 * hd
    res = {
        "workload": "config 2: sqfree+spinor hd 128 (pad 154, skeleton 115, bands 5,4,4,4,5, "
                    "residual 3 bits), %d layers x 8 KV heads x 16384 positions" % L_,
        "bytes_per_pos_k": cache.cc.bytes_per_pos_k, "bytes_per_pos_v": cache.cc.bytes_per_pos_v,
        "compression_ratio": 2 * 2 * hd / bpp,
        "compress": {"value": pairs / (c_ms * 1e-3) / 1e6, "unit": "Mpairs/s", "ms": c_ms,
                     "achieved_gbs": pairs * (2 * hd * 4 + bpp) / (c_ms * 1e-3) / 1e9},
        "decode": {"value": d_ms * 1e3, "unit": "us/token", "algorithmic_bytes": step_bytes,
                   "achieved_gbs": step_bytes / (d_ms * 1e-3) / 1e9},
    }
    res["compress"]["frac"] = res["compress"]["achieved_gbs"] / peak
    res["decode"]["frac"] = res["decode"]["achieved_gbs"] / peak
    # the read of layer 0, K and V, fp32 rows out: every KV head token-major in
    # one sp_cuda_sqfree_read_kv_tokens launch per half; the reference-named
    # per-slot batch read timed beside it
    rd_all = torch.empty(1, T_, H_, hd, dtype=torch.float32, device=dev)
    rd = torch.empty(T_, hd, dtype=torch.float32, device=dev)

    def read_all():
        for which in (0, 1):
            cache.read_kv_tokens(which, 0, 1, 0, rd_all)

    def read_per_slot():
        for which in (0, 1):
            for h in range(H_):
                cache.read_batch(which, 0, h, 0, rd)

    def time_read(fn):
        fn()
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(3):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / (3 * 2 * H_)
    r_ms = time_read(read_all)
    r_ms_one = time_read(read_per_slot)
    r_bytes = T_ * (cache.cc.bytes_per_pos_k + hd * 4)
    res["read"] = {"value": r_bytes / (r_ms * 1e-3) / 1e9, "unit": "GB/s", "ms_per_slot": r_ms,
                   "frac": r_bytes / (r_ms * 1e-3) / 1e9 / peak,
                   "per_slot_call_gbs": r_bytes / (r_ms_one * 1e-3) / 1e9,
                   "workload": "layer 0, %d KV heads x K and V, %d positions, all heads per "
                               "sp_cuda_sqfree_read_kv_tokens launch, fp32 [pos][head][128] out" % (H_, T_)}
    cache.free()
    return res


def measure_hier(torch, dev, stream, peak: float, scale: int = 1):
    """Config 4: hierarchical Vilenkin, hd 256 (pad 330, skeleton 30, bands
    5,5, 2 residual bits), 16 KV heads, 64 sequences x 8192 positions
    compressed in one call from bf16 K (log-normal sigma 1.0 channel scales,
    RoPE) and N(0,1) V (seed 4).  The predictor W is fitted per head by
    ridge least squares (float64) on a 4096-vector calibration sample of the
    first sequence and shared by the sequences."""
    from spb200.sqfree import HierCache
    from spb200 import synth
    S_, H_, T_, hd, pd, nsk = max(1, 64 // scale), 16, 8192, 256, 330, 30
    cache = HierCache(hd, S_, H_, T_, pd, nsk, stream=stream)
    gen = torch.Generator(device=dev)
    gen.manual_seed(4)
    k = torch.empty(S_, T_, H_, hd, dtype=torch.bfloat16, device=dev)
    v = torch.empty_like(k)
    for sq in range(S_):
        kk, vv = synth.kv_layer_torch(gen, T_, H_, hd, sigma=1.0, device=dev, dtype=torch.bfloat16)
        k[sq], v[sq] = kk, vv
    M = _hartley_matrix(pd, torch, dev)
    Ws = []
    for h in range(H_):
        x = k[0, :4096, h].double()
        pad = torch.cat([x, x.mean(1, keepdim=True).expand(-1, pd - hd)], 1)
        c = pad @ M.T
        Sk, Tg = c[:, :nsk], c[:, nsk:]
        A = Sk.T @ Sk + 1e-6 * torch.eye(nsk, dtype=torch.float64, device=dev)
        Ws.append(torch.linalg.solve(A, Sk.T @ Tg).T.half())
    W = torch.stack(Ws)                                   # [H][300][30]
    cache.upload_W(W.unsqueeze(0).expand(S_, -1, -1, -1).reshape(S_ * H_, pd - nsk, nsk).cpu().numpy())
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    cache.write_kv_tokens(0, 0, k, v)
    torch.cuda.synchronize()
    e0.record(stream)
    cache.write_kv_tokens(0, 0, k, v)
    e1.record(stream)
    torch.cuda.synchronize()
    c_ms = e0.elapsed_time(e1)
    del v
    ko = torch.empty(S_, T_, H_, hd, dtype=torch.float32, device=dev)
    cache.read_kv_tokens(0, 0, ko, None)
    torch.cuda.synchronize()
    e0.record(stream)
    cache.read_kv_tokens(0, 0, ko, None)
    e1.record(stream)
    torch.cuda.synchronize()
    r_ms = e0.elapsed_time(e1)
    pairs = S_ * H_ * T_
    bpp = cache.hc.bytes_per_pos_k
    corr = torch.nn.functional.cosine_similarity(ko[0, :2048].flatten(0, 1),
                                                 k[0, :2048].float().flatten(0, 1), dim=1).mean().item()
    res = {
        "workload": "config 4: hier hd 256 (pad 330, skeleton 30, bands 5,5, residual 2 bits), "
                    "16 KV heads x %d sequences x 8192 positions, bf16 in, one call" % S_,
        "bytes_per_pos": bpp, "compression_ratio": 2 * hd / bpp,
        "compress": {"value": pairs / (c_ms * 1e-3) / 1e6, "unit": "Mpairs/s", "ms": c_ms,
                     "achieved_gbs": pairs * (2 * 2 * hd + 2 * bpp) / (c_ms * 1e-3) / 1e9},
        "decompress_k": {"value": pairs * (bpp + 4 * hd) / (r_ms * 1e-3) / 1e9, "unit": "GB/s",
                         "ms": r_ms, "out": "fp32 [%d][8192][16][256]" % S_},
        "k_cosine_first_2048": corr,
    }
    res["compress"]["frac"] = res["compress"]["achieved_gbs"] / peak
    res["decompress_k"]["frac"] = res["decompress_k"]["value"] / peak
    cache.free()
    return res


def peer_gather(torch, n_rows: int, n_q_total: int, dev):
    """(PeerGather, description) for the fused decode + all-gather, or
    (None, why) when symmetric memory cannot be set up (NCCL is used then)."""
    try:
        from spb200.gather import PeerGather
        return (PeerGather(n_rows, n_q_total, HD, dev),
                "fused: the combine kernel stores each output row into every rank's symmetric-memory "
                "buffer over NVLink, then a bounded flag wait")
    except Exception as e:  # noqa: BLE001 - reported in the JSON line
        return None, ("nccl all_gather (peer memory unavailable: %s: %s)" % (type(e).__name__, e))[:240]


def measure_config3(torch, dist, dev, stream, ws: int, rank: int, steps: int, warmup: int, peak: float,
                    max_over_ranks, barrier, scale: int = 1):
    """Config 3: MoE-scale long context, 48 layers, 32 Q / 4 KV heads (8 query
    heads per KV head), head_dim 128, ctx 131072, batch 4 (four independent
    caches), ship K 5/5/4/3 + V 3-bit, seeded as config 0 (seed 3).  The
    (layer, KV head) slots are partitioned over the ranks (spb200.shard:
    heads first, then layer halves at 8 GPUs); the four sequences of a rank
    are its cache layers seq * L_local + l, attended in one call, and one
    all-gather of the per-head fp16 outputs completes the step.  scale > 1
    (profiling only) keeps 48 / scale layers (at least 2)."""
    import ctypes as C

    import spb200
    from spb200 import shard, synth
    L3, Q3, KV3, CTX3, B3 = max(2, 48 // max(1, scale)), 32, 4, 131072, 4
    sh = shard.partition(L3, KV3, ws)[rank]
    Hl, Ll, G = len(sh.heads), sh.n_layers, Q3 // KV3
    cache = spb200.Cache(HD, B3 * Ll, Hl, CTX3, KB, VB, True, stream)
    gen = torch.Generator(device=dev)
    for b in range(B3):
        for l in range(Ll):
            gen.manual_seed(3 * 1000003 + b * 1009 + sh.layer0 + l)
            k, v = synth.kv_layer_torch(gen, CTX3, KV3, HD, device=dev)
            idx = list(sh.heads)
            cache.write_kv_tokens(b * Ll + l, 0, k[:, idx].contiguous(), v[:, idx].contiguous())
    torch.cuda.synchronize()
    gq = torch.Generator(device=dev)
    gq.manual_seed(3)
    q_all = torch.randn(B3, L3, Q3, HD, device=dev, generator=gq).half()
    qidx = torch.tensor(sh.q_heads(G), device=dev)
    q = q_all[:, sh.layer0:sh.layer0 + Ll][:, :, qidx].reshape(B3 * Ll, Hl * G, HD).contiguous()
    out = torch.empty_like(q)
    shards = shard.partition(L3, KV3, ws)
    Lm, Qm = shard.max_shard_shape(shards, G)
    blk = torch.zeros(B3 * Lm, Qm, HD, dtype=torch.float16, device=dev)
    gathered = [torch.empty_like(blk) for _ in range(ws)] if ws > 1 else None
    gather, collective = None, "none (single GPU)"
    if ws > 1:
        # destination rows: sequence b, global layer; global query heads
        gather, collective = peer_gather(torch, B3 * L3, Q3, dev)
        dst_layer = torch.tensor([b * L3 + sh.layer0 + l for b in range(B3) for l in range(Ll)],
                                 dtype=torch.int32, device=dev)
        dst_qhead = qidx.to(torch.int32)

    def step():
        if gather is not None:
            gather.decode(C.byref(cache.cc), 0, B3 * Ll, q, Hl * G, CTX3, dst_layer, dst_qhead,
                          1.0 / HD ** 0.5, -1, stream)
            return
        cache.attn_decode(0, B3 * Ll, q, CTX3, out, logit_scale=1.0 / HD ** 0.5, stream=stream)
        if ws > 1:
            blk.view(B3, Lm, Qm, HD)[:, :Ll, :Hl * G] = out.view(B3, Ll, Hl * G, HD)
            dist.all_gather(gathered, blk)

    for _ in range(warmup):
        step()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        step()
    e1.record(stream)
    barrier()
    ms = max_over_ranks(e0.elapsed_time(e1) / steps)
    bytes_all = B3 * L3 * KV3 * CTX3 * (K_ROW + V_ROW)
    res = {
        "workload": "config 3: %d layers x 32 Q / 4 KV heads x hd 128, ctx 131072, batch 4, ship 5/5/4/3 + V3, "
                    "(layer, KV head) slots sharded over %d GPU(s)" % (L3, ws),
        "value": ms * 1e3, "unit": "us/step (batch 4)", "tokens_per_s": B3 / (ms * 1e-3),
        "cache_bytes_total": bytes_all,
        "achieved_gbs_total": bytes_all / (ms * 1e-3) / 1e9,
        "frac_of_n_gpu_peak": bytes_all / (ms * 1e-3) / 1e9 / (peak * ws),
        "scaling": "strong",
        "collective": collective,
    }
    cache.free()
    return res


def run_reference(args):
    """--impl reference: the oracle port of the reference CPU path (the
    reference's own CPU core is an empty submodule and cannot be built),
    timed on this box's host cores.  Each step = one layer of the decode
    step, scaled x32 to a full token."""
    ws, rank, _ = dist_env()
    if rank != 0:
        return
    n_threads = os.cpu_count() or 1
    import numpy as np
    import oracle as O
    from spb200 import synth
    kp = np.zeros((N_KV, CTX, K_ROW), np.uint8)
    vp = np.zeros((N_KV, CTX, V_ROW), np.uint8)
    for h in range(N_KV):
        k, v = synth.kv_slot_np(SEED, 0, h, CTX, HD)
        kp[h] = O.ship_write(k, KB, True, n_threads)
        vp[h] = O.ship_write(v, VB, False, n_threads)
    q = synth.q_np(SEED, 1, N_Q, HD, 1.0 / 128 ** 0.5)[0]
    for _ in range(args.warmup):
        O.attn_decode(kp, vp, HD, KB, VB, True, q, CTX, 1.0, n_threads)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        O.attn_decode(kp, vp, HD, KB, VB, True, q, CTX, 1.0, n_threads)
        times.append(time.perf_counter() - t0)
    per_layer = statistics.median(times)
    us_tok = per_layer * N_LAYERS * 1e6
    cores = n_threads
    line = {
        "impl": "reference", "metric": METRIC, "value": us_tok, "unit": UNIT,
        "n_gpus": ws, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": us_tok / 1e3, "higher_is_better": False, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded, config-1 distributions)",
        "config": {"workload": WORKLOAD % N_LAYERS, "sample": "1 of 32 layers per step, scaled x32"},
        "cpu_baseline": {"value": us_tok, "unit": UNIT, "cores": cores, "kind": "port",
                         "min": min(times) * N_LAYERS * 1e6, "passes": len(times),
                         "sample": "one layer (8 KV heads x 32768 positions) per step, median over the "
                                   "timed steps (min also given), x32"},
        "e2e": {"value": us_tok, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "reference CPU core (lib/shannon-prime) is absent from the reference checkout; "
                "this is the CPU restatement of its algorithm (oracle/sp_oracle.c), OpenMP over (KV head, token chunk) tasks on every host thread",
    }
    print(json.dumps(line), flush=True)


def run_ours(args):
    import ctypes as C

    import torch
    import torch.distributed as dist

    import spb200
    from spb200 import synth

    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        dist.init_process_group("nccl", device_id=dev)
    L = spb200.lib()
    # A dedicated stream: the legacy default stream's handle is NULL, which the
    # bridge would read as "make a private stream".
    stream = torch.cuda.Stream(device=dev)
    torch.cuda.set_stream(stream)
    heads = local_heads(rank, ws)
    H = len(heads)
    G = N_Q // N_KV
    nq_local = H * G

    # The bridge context (the reference-facing API) owns the cache; the device
    # entry points run on its sp_cuda_cache_t.
    os.environ["SHANNON_PRIME_ENABLED"] = "1"
    params = spb200.SpLlamaParams(HD, N_LAYERS, H, CTX, 1, stream.cuda_stream, None)
    ctx = L.sp_llama_init(C.byref(params))
    if not ctx:
        raise RuntimeError("sp_llama_init failed")
    cc = C.cast(L.sp_llama_get_cuda_cache(ctx), C.POINTER(spb200.SpCudaCache))

    # Fill the cache: per layer, synthetic K/V for this rank's heads.
    gen = torch.Generator(device=dev)
    kept = []                  # inputs of 4 layers (1.07 GB fp32) for the compress timing
    t_fill = time.perf_counter()
    for layer in range(N_LAYERS):
        gen.manual_seed(SEED * 1000003 + layer)
        k, v = synth.kv_layer_torch(gen, CTX, N_KV, HD, device=dev)
        k = k[:, heads].contiguous()
        v = v[:, heads].contiguous()
        rc = L.sp_cuda_write_kv_tokens(cc, layer, 0, CTX, k.data_ptr(), v.data_ptr(), 0)
        spb200.check(rc, "write_kv_tokens")
        if layer < 4:
            kept.append((layer, k, v))
    torch.cuda.synchronize()
    t_fill = time.perf_counter() - t_fill

    gq = torch.Generator(device=dev)
    gq.manual_seed(SEED)
    q_all = (torch.randn(N_LAYERS, N_Q, HD, device=dev, generator=gq) / HD ** 0.5).half()
    qidx = torch.tensor([h * G + g for h in heads for g in range(G)], device=dev)
    q = q_all[:, qidx].contiguous()
    out = torch.empty(N_LAYERS, nq_local, HD, dtype=torch.float16, device=dev)
    gathered = [torch.empty_like(out) for _ in range(ws)] if ws > 1 else None
    # Multi-GPU: the combine kernel stores every output row straight into each
    # rank's symmetric-memory gather buffer (sp_cuda_attn_decode_allgather);
    # NCCL all_gather only if peer memory cannot be set up.
    gather, collective = None, "none (single GPU)"
    if ws > 1:
        gather, collective = peer_gather(torch, N_LAYERS, N_Q, dev)
        dst_layer = torch.arange(N_LAYERS, dtype=torch.int32, device=dev)
        dst_qhead = qidx.to(torch.int32)

    def step():
        if gather is not None:
            gather.decode(cc, 0, N_LAYERS, q, nq_local, CTX, dst_layer, dst_qhead, 1.0, -1, stream)
            return
        rc = L.sp_cuda_attn_decode(cc, 0, N_LAYERS, q.data_ptr(), nq_local, CTX, 1.0,
                                   out.data_ptr(), -1, stream.cuda_stream)
        if rc:
            spb200.check(rc, "attn_decode")
        if ws > 1:
            dist.all_gather(gathered, out)

    def barrier():
        if ws > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x: float) -> float:
        if ws == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        step()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        barrier()
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        barrier()
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)
    clocks = clk.summary()

    # Main-kernel duration (roofline), measured with events inside the call.
    L.sp_cuda_attn_profile(1)
    kms = []
    for _ in range(max(3, min(args.steps, 20))):
        L.sp_cuda_attn_decode(cc, 0, N_LAYERS, q.data_ptr(), nq_local, CTX, 1.0,
                              out.data_ptr(), -1, stream.cuda_stream)
        kms.append(L.sp_cuda_attn_last_kernel_ms())
    L.sp_cuda_attn_profile(0)
    splits = L.sp_cuda_attn_last_splits()
    kernel_ms = max_over_ranks(statistics.mean(kms))
    cache_bytes = N_LAYERS * H * CTX * (K_ROW + V_ROW)
    q_bytes = N_LAYERS * nq_local * HD * 2
    alg_bytes = cache_bytes + q_bytes
    peak, peak_src = peaks()
    achieved = alg_bytes / (kernel_ms * 1e-3) / 1e9

    # End to end through the bridge with host buffers.
    hq = q.cpu().pin_memory()
    hout = torch.empty(out.shape, dtype=torch.float16).pin_memory()
    hgat = [torch.empty(out.shape, dtype=torch.float16) for _ in range(ws)]

    dq = torch.empty_like(q)
    hfull = torch.empty(N_LAYERS, N_Q, HD, dtype=torch.float16).pin_memory() if gather is not None else None

    def e2e_step():
        if gather is not None:
            # host q in (pinned) -> fused decode + gather -> whole output back
            with torch.cuda.stream(stream):
                dq.copy_(hq, non_blocking=True)
                gather.decode(cc, 0, N_LAYERS, dq, nq_local, CTX, dst_layer, dst_qhead, 1.0, -1, stream)
                hfull.copy_(gather.out, non_blocking=True)
            stream.synchronize()
            return
        rc = L.sp_llama_attn_decode(ctx, 0, N_LAYERS, hq.data_ptr(), nq_local, CTX, 1.0,
                                    hout.data_ptr(), -1)
        if rc:
            raise RuntimeError(f"sp_llama_attn_decode {rc}")
        if ws > 1:
            d = hout.to(dev, non_blocking=True)
            dist.all_gather(gathered, d)
            for i in range(ws):
                hgat[i].copy_(gathered[i])
    for _ in range(args.warmup):
        e2e_step()
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        e2e_step()
    barrier()
    e2e_ms = max_over_ranks((time.perf_counter() - t0) / args.steps * 1e3)
    if gather is not None:
        h2d, d2h = hq.numel() * 2, hfull.numel() * 2
    else:
        h2d = hq.numel() * 2 + (out.numel() * 2 if ws > 1 else 0)
        d2h = hout.numel() * 2 * (ws if ws > 1 else 1)

    # Multi-GPU correctness, once after timing: the gathered rows of every
    # rank against each rank's own local decode of its shard (bit-exact).
    gather_check = None
    if ws > 1:
        L.sp_cuda_attn_decode(cc, 0, N_LAYERS, q.data_ptr(), nq_local, CTX, 1.0,
                              out.data_ptr(), -1, stream.cuda_stream)
        stream.synchronize()
        locs = [torch.empty_like(out) for _ in range(ws)]
        dist.all_gather(locs, out)
        if gather is not None:
            gather.decode(cc, 0, N_LAYERS, q, nq_local, CTX, dst_layer, dst_qhead, 1.0, -1, stream)
            stream.synchronize()
            got = gather.out
        else:
            step()
            torch.cuda.synchronize()
            got = torch.empty(N_LAYERS, N_Q, HD, dtype=torch.float16, device=dev)
            for r in range(ws):
                got[:, [h * G + g for h in range(N_KV) if h % ws == r for g in range(G)]] = gathered[r]
        expect = torch.empty(N_LAYERS, N_Q, HD, dtype=torch.float16, device=dev)
        for r in range(ws):
            expect[:, [h * G + g for h in range(N_KV) if h % ws == r for g in range(G)]] = locs[r]
        bad = torch.tensor([float((got != expect).any(dim=-1).sum())], device=dev)
        dist.all_reduce(bad, op=dist.ReduceOp.SUM)
        gather_check = {"rows": N_LAYERS * N_Q * ws, "mismatches": int(bad.item()),
                        "what": "gathered rows on every rank vs the owning rank's local decode, bit-exact"}

    # Ship-path compression throughput: re-compress 4 full layers (K and V,
    # fp32 in, 1.07 GB of inputs > L2) through the token-major entry point.
    def compress_pass():
        for layer, kk, vv in kept:
            L.sp_cuda_write_kv_tokens(cc, layer, 0, CTX, kk.data_ptr(), vv.data_ptr(), 0)
    for _ in range(2):
        compress_pass()
    barrier()
    c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 5
    c0.record(stream)
    for _ in range(reps):
        compress_pass()
    c1.record(stream)
    barrier()
    cms = max_over_ranks(c0.elapsed_time(c1) / (reps * len(kept)))
    pairs = CTX * H
    comp_mpairs = pairs * ws / (cms * 1e-3) / 1e6
    comp_gbs = pairs * (2 * HD * 4 + K_ROW + V_ROW) / (cms * 1e-3) / 1e9

    # The scores-only op (sp_cuda_kq_scores, the GPU body of the reference's
    # ggml fused-KQ op): every (layer, KV head) slot of 4 layers against its
    # G query rows, fp32 scores [G][CTX] per slot.
    kslot = int(cc.contents.max_seq_len) * K_ROW
    kbase = int(cc.contents.d_k_cache or 0)

    kq_layers = min(4, N_LAYERS)

    # One strided launch over all slots of the layers (sp_cuda_kq_scores_strided);
    # the reference-shaped per-slot call is timed beside it.
    kq_dst = torch.empty(kq_layers * H, G, CTX, dtype=torch.float32, device=dev)

    def kq_pass():
        rc = L.sp_cuda_kq_scores_strided(kbase, kslot, kq_layers * H, K_ROW, 0, HD, CTX, q.data_ptr(), 1, HD * 2,
                                         G * HD * 2, G, kq_dst.data_ptr(), CTX * 4, G * CTX * 4,
                                         stream.cuda_stream)
        assert rc == 0

    def kq_pass_per_slot():
        for layer in range(kq_layers):
            for h in range(H):
                L.sp_cuda_kq_scores(kbase + (layer * H + h) * kslot, K_ROW, 0, HD, CTX,
                                    q[layer, h * G].data_ptr(), 1, HD * 2, G, kq_dst[layer * H + h].data_ptr(),
                                    CTX * 4, stream.cuda_stream)
    kq_pass()
    barrier()
    c0.record(stream)
    for _ in range(reps):
        kq_pass()
    c1.record(stream)
    barrier()
    kq_ms = max_over_ranks(c0.elapsed_time(c1) / (reps * kq_layers * H))     # per slot
    kq_pass_per_slot()
    barrier()
    c0.record(stream)
    for _ in range(reps):
        kq_pass_per_slot()
    c1.record(stream)
    barrier()
    kq_ms_one = max_over_ranks(c0.elapsed_time(c1) / (reps * kq_layers * H))
    kq_bytes = CTX * K_ROW + G * CTX * 4 + G * HD * 2
    kq_gbs = kq_bytes / (kq_ms * 1e-3) / 1e9

    # Ship read (decompress to fp32 rows): every slot of layer 0, K and V,
    # token-major over all KV heads in one sp_cuda_read_kv_tokens launch per
    # half; the reference-named per-slot call (sp_cuda_read_batch_partial)
    # is timed beside it.
    rd_all = torch.empty(CTX, H, HD, dtype=torch.float32, device=dev)
    rd_out = torch.empty(CTX, HD, dtype=torch.float32, device=dev)

    def read_pass():
        for which in (0, 1):
            assert L.sp_cuda_read_kv_tokens(cc, which, 0, 1, 0, CTX, rd_all.data_ptr(), -1) == 0

    def read_pass_per_slot():
        for which in (0, 1):
            for h in range(H):
                L.sp_cuda_read_batch_partial(cc, which, 0, h, 0, CTX, rd_out.data_ptr(), -1)

    def time_read(fn):
        fn()
        barrier()
        c0.record(stream)
        for _ in range(reps):
            fn()
        c1.record(stream)
        barrier()
        return max_over_ranks(c0.elapsed_time(c1) / (reps * 2 * H))      # per (slot, half)
    rd_ms = time_read(read_pass)
    rd_ms_one = time_read(read_pass_per_slot)
    rd_bytes = CTX * ((K_ROW + V_ROW) / 2 + HD * 4)
    rd_gbs = rd_bytes / (rd_ms * 1e-3) / 1e9

    # CPU baseline (rank 0, N = 1): the oracle on a bounded sample.
    cpu = None
    if ws == 1 and not args.no_cpu:
        n_threads = os.cpu_count() or 1
        times, cores = cpu_decode_sample(n_threads, layers=5)
        cpu = {"value": statistics.median(times) * N_LAYERS * 1e6, "unit": UNIT, "cores": cores, "kind": "port",
               "min": min(times) * N_LAYERS * 1e6, "passes": len(times),
               "sample": "one layer (8 KV heads x 32768 positions) per pass, 1 warm-up + 5 timed passes, "
                         "median (min also given), scaled x32 layers; OpenMP on every host thread",
               "compress_mpairs_s": None}
        mp, _ = cpu_compress_sample(n_threads)
        cpu["compress_mpairs_s"] = mp / 1e6
        cpu["compress_cores"] = n_threads

    launches_per_step = 2        # fused decode kernel + split combine kernel
    if gather is not None:
        launches_per_step = 3    # + the bounded wait for the peers' flags
    line = {
        "metric": METRIC, "value": ms * 1e3, "unit": UNIT, "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
        "higher_is_better": False, "scaling": "strong", "vs_baseline": None,
        "dtype": "u8 codes -> f32 accumulate (fp16 q/out)",
        "data": "synthetic (seeded; K = RoPE(N(0,1) x LogNormal(0,0.5) per dim), V = N(0,1), q = N(0,1/sqrt(128)) fp16)",
        "config": {"workload": WORKLOAD % N_LAYERS,
                   "l2": "inputs larger than L2 (compressed cache %.2f GB per GPU)" % (cache_bytes / 1e9),
                   "parallelism": f"kv-head shards x{ws}" if ws > 1 else "single GPU",
                   "collective": collective,
                   "kv_heads_per_gpu": H, "splits": splits},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak,
                     "traffic": NCU_TRAFFIC_PER_LAYER * N_LAYERS * H / N_KV,
                     "traffic_source": "ncu dram bytes of the 8-layer capture, scaled by layers x kv heads",
                     "peak_source": peak_src,
                     "kernel": "fused decode main kernel", "kernel_ms": kernel_ms,
                     "algorithmic_bytes": alg_bytes},
        "e2e": {"value": e2e_ms * 1e3, "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h,
                "path": ("sp_cuda_attn_decode_allgather (pinned host q in, gathered output of all ranks back)"
                         if gather is not None else "sp_llama_attn_decode (pinned host q in, host out back: the decode kernels read q and write the output rows over the host link in place)")},
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clocks,
        "compress": {"metric": "ship-path compress throughput (K+V pairs)", "value": comp_mpairs,
                     "unit": "Mpairs/s", "model_tokens_per_s_M": comp_mpairs / (N_KV * 1.0),
                     "achieved_gbs": comp_gbs, "frac": comp_gbs / peak,
                     "workload": "4 layers x 32768 positions x %d KV heads, fp32 in, 5 passes; ms is per layer" % H,
                     "ms": cms},
        "kq_op": {"metric": "fused decompress-KQ scores op, per (layer, KV head) slot, all slots of the layers in "
                            "one sp_cuda_kq_scores_strided launch",
                  "value": kq_ms * 1e3, "unit": "us/slot", "achieved_gbs": kq_gbs, "frac": kq_gbs / peak,
                  "per_slot_call_us": kq_ms_one * 1e3,
                  "workload": "4 layers x %d KV heads, %d query rows per slot, ctx %d, fp32 scores out" % (H, G, CTX),
                  "bytes_per_slot": kq_bytes},
        "read": {"metric": "ship read (decompress to fp32 rows), all KV heads of a layer per sp_cuda_read_kv_tokens "
                           "launch",
                 "value": rd_gbs, "unit": "GB/s", "ms_per_slot": rd_ms, "frac": rd_gbs / peak,
                 "per_slot_call_gbs": rd_bytes / (rd_ms_one * 1e-3) / 1e9,
                 "workload": "layer 0, %d KV heads x K and V, %d positions, fp32 [pos][128] out" % (H, CTX)},
        "cache_fill_s": t_fill,
    }
    if gather_check is not None:
        line["gather_check"] = gather_check
    # Everything of a step after the main kernel: the segment combine with its
    # inverse VHT2 and, at N > 1, the NVLink peer stores of the gathered rows
    # and the flag wait (step time minus the main kernel's event-timed
    # duration, max over ranks for both).
    tail_us = max(0.0, ms - kernel_ms) * 1e3
    line["gather_latency"] = {"per_step_us": tail_us, "per_layer_us": tail_us / N_LAYERS,
                              "what": ("combine + peer-store all-gather + flag wait" if ws > 1 else
                                       "combine (no gather at N = 1)") +
                                      ": step time minus the main kernel's event-timed duration"}
    if cpu is not None:
        line["cpu_baseline"] = cpu
    if not args.no_extra:
        del kept
        torch.cuda.empty_cache()
        line["config3"] = measure_config3(torch, dist, dev, stream, ws, rank, max(3, args.steps // 2),
                                          args.warmup, peak, max_over_ranks, barrier, args.extras_scale)
    if ws == 1 and not args.no_extra:
        torch.cuda.empty_cache()
        line["sqfree"] = measure_sqfree(torch, dev, stream, max(3, args.steps // 2), args.warmup, peak,
                                        args.extras_scale)
        torch.cuda.empty_cache()
        line["hier"] = measure_hier(torch, dev, stream, peak, args.extras_scale)
    if rank == 0:
        print(json.dumps(line), flush=True)
    L.sp_llama_free(ctx)
    if ws > 1:
        dist.destroy_process_group()


def main():
    global N_LAYERS
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--extras-scale", type=int, default=1,
                    help="divide config 2 layers and config 4 sequences by this (profiling aid)")
    ap.add_argument("--no-extra", action="store_true",
                    help="skip the config 2 (sqfree) and config 4 (hier) measurements")
    ap.add_argument("--layers", type=int, default=N_LAYERS,
                    help="layers in the cache (profiling aid: a smaller case for ncu; "
                         "the headline number is the default, all 32)")
    ap.add_argument("--attn-impl", type=int, default=0, choices=[0, 1, 2, 3],
                    help="fused-decode kernel family (profiling aid: 0 automatic = 2, 1 generic SIMT, "
                         "2 mma.sync, 3 tcgen05); the headline number is the default")
    args = ap.parse_args()
    N_LAYERS = args.layers
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    else:
        if args.attn_impl:
            import spb200
            spb200.lib().sp_cuda_attn_force_impl(args.attn_impl)
        run_ours(args)


if __name__ == "__main__":
    main()
