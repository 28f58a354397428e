"""Benchmark of the vllm-jax B200 hot path (one JSON line on rank 0).

Default workload (the first half of the headline metric):
Qwen3-8B continuous batching through Engine.generate -- 512 requests, prompt
and output lengths uniform in [100, 1024] (seed 0), random token ids, greedy,
max_num_batched_tokens 16384, random-init N(0, 0.02) bf16 weights. Metric:
output tokens/s of the whole job. One "step" = one generate() over the whole
request set; --steps K times K of them (CUDA events, max over ranks) after
--warmup W untimed ones.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload e2e|decode|prefill|kvstore|c5] [--tp T]

N > 1 (torchrun, one process per GPU): tensor parallel by KV head -- rank r
holds KV heads [r*8/N, (r+1)*8/N), its q heads, 1/N of the MLP and its pool
slice; o_proj and down_proj are summed over ranks by the fused NVLink
all-reduce + residual add + RMSNorm kernel. Total work is fixed ("strong").

--workload decode: C3 paged decode attention (HBM GB/s). --workload prefill:
C2 paged prefill attention (TFLOP/s). --workload kvstore: K3 (q/k norm + RoPE
+ KV scatter) on the C2 batch (GB/s). --workload c4step: one Qwen3-8B decode
step as a CUDA graph (ms) with per-kernel shares on stderr. --workload c5: C5, Qwen3-32B with
chunked prefill mixed with decode (output tok/s; --batch R runs the first R
of the 1024 requests, and says so). For the kernel workloads N > 1 splits the
KV heads with no collective on the data path.

--impl reference times the reference algorithm on the host CPU cores: the
reference (JAX/Pallas) cannot be installed in this image, so its NumPy
restatement in oracle/ runs instead (cpu_baseline.kind = "port").
"""
from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "vllm-jax_b200"))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402

# C3
C3 = dict(batch=256, num_q_heads=32, num_kv_heads=8, head_dim=128, block_size=16,
          ctx_min=512, ctx_max=32768, pool_blocks=200_000, table_width=2048, seed=0)
# C2
C2 = dict(num_seqs=64, num_q_heads=32, num_kv_heads=8, head_dim=128, block_size=16,
          new_min=128, new_max=4096, prefix_min=0, prefix_max=2048, pool_blocks=200_000,
          seed=0)


def c3_lengths(cfg=C3) -> np.ndarray:
    rng = np.random.default_rng(cfg["seed"])
    u = rng.uniform(math.log(cfg["ctx_min"]), math.log(cfg["ctx_max"]), 256)
    return np.round(np.exp(u)).astype(np.int32)[:cfg["batch"]]


def c3_block_tables(lens: np.ndarray, cfg=C3) -> np.ndarray:
    rng = np.random.default_rng(cfg["seed"] + 1)
    perm = rng.permutation(cfg["pool_blocks"]).astype(np.int32)
    bt = np.full((len(lens), cfg["table_width"]), -1, np.int32)
    used = 0
    for b, L in enumerate(lens):
        n = (int(L) + cfg["block_size"] - 1) // cfg["block_size"]
        bt[b, :n] = perm[used:used + n]
        used += n
    return bt


def c2_batch(cfg=C2):
    """C2: per-sequence new-token counts, cached prefixes and block tables."""
    rng = np.random.default_rng(cfg["seed"])
    S = cfg["num_seqs"]
    new = rng.integers(cfg["new_min"], cfg["new_max"] + 1, S).astype(np.int32)
    pre = rng.integers(cfg["prefix_min"], cfg["prefix_max"] + 1, S).astype(np.int32)
    # profiling cases: every sequence the same length (--new-tokens / --prefix-tokens)
    if cfg.get("new_fixed"):
        new[:] = cfg["new_fixed"]
    if cfg.get("prefix_fixed") is not None:
        pre[:] = cfg["prefix_fixed"]
    ctx = new + pre
    bs = cfg["block_size"]
    perm = rng.permutation(cfg["pool_blocks"]).astype(np.int32)
    width = int(((ctx + bs - 1) // bs).max())
    bt = np.full((S, width), -1, np.int32)
    used = 0
    for s_, c in enumerate(ctx):
        k = (int(c) + bs - 1) // bs
        bt[s_, :k] = perm[used:used + k]
        used += k
    return new, pre, bt


def prefill_flops(new: np.ndarray, pre: np.ndarray, hq: int, d: int = 128) -> float:
    """Causal-pair FLOPs: 4*Hq*D*(n*p + n(n+1)/2) per sequence (QK^T and PV)."""
    n = new.astype(np.float64)
    p = pre.astype(np.float64)
    return float((4.0 * hq * d * (n * p + n * (n + 1) / 2)).sum())


def decode_bytes(lens: np.ndarray, hkv: int, hq: int, d: int = 128, bs: int = 16) -> int:
    """Algorithmic HBM bytes of one decode call: K+V rows of every context token,
    q in + out, the used block-table entries and the lengths."""
    lens = lens.astype(np.int64)
    kv = int(lens.sum()) * hkv * d * 2 * 2
    qo = len(lens) * hq * d * 2 * 2
    bt = int(((lens + bs - 1) // bs).sum()) * 4 + len(lens) * 4
    return kv + qo + bt


def load_peaks() -> tuple[dict, str]:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f), "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


# ---------------------------------------------------------------------------
# clocks sampled during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.out = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.out, _ = self.proc.communicate()

    def summary(self) -> dict:
        if not self.out:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"]}
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# CPU baseline (oracle port), bounded sample
# ---------------------------------------------------------------------------
def _cpu_decode_seq(args):
    L, hkv, g, seed = args
    from oracle import attention as oatt
    rng = np.random.default_rng(seed)
    bs, d = 16, 128
    npg = (L + bs - 1) // bs
    kc = rng.standard_normal((npg, bs, hkv, d), dtype=np.float32)
    vc = rng.standard_normal((npg, bs, hkv, d), dtype=np.float32)
    q = rng.standard_normal((1, hkv * g, d), dtype=np.float32)
    bt = np.arange(npg, dtype=np.int32)[None]
    t0 = time.perf_counter()
    oatt.decode_attention(q, kc, vc, bt, np.array([L], np.int32), 1 / math.sqrt(d))
    return time.perf_counter() - t0


def cpu_decode_baseline(lens: np.ndarray, hkv: int, hq: int, budget_s: float, pool) -> dict:
    """Time the oracle on a seeded subsample of sequences with all host cores."""
    rng = np.random.default_rng(123)
    order = rng.permutation(len(lens))
    cores = pool._processes if pool is not None else 1
    done, sample, t_cpu = 0, [], 0.0
    batch = max(1, cores)
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < budget_s and done < len(order):
        idx = order[done:done + batch]
        done += len(idx)
        args = [(int(lens[i]), hkv, hq // hkv, int(i)) for i in idx]
        times = (pool.map(_cpu_decode_seq, args) if pool is not None
                 else [_cpu_decode_seq(a) for a in args])
        t_cpu += float(sum(times))
        sample.extend(int(i) for i in idx)
    t_eff = t_cpu / cores  # compute seconds spread over the worker processes
    sb = decode_bytes(lens[sample], hkv, hq)
    return {"value": sb / t_eff / 1e9, "unit": "GB/s", "cores": cores, "kind": "port",
            "sample": f"{len(sample)} of {len(lens)} C3 sequences "
                      f"({int(lens[sample].sum())} ctx tokens) through the numpy oracle "
                      f"(oracle/attention.py:decode_attention), one sequence per process; "
                      f"{t_cpu:.1f} s of compute over {cores} processes"}


def _one_blas_thread():
    """Pool initializer: one BLAS thread per worker process, so that N
    processes use N cores instead of oversubscribing them N x N."""
    try:
        from threadpoolctl import threadpool_limits
        threadpool_limits(1)
    except ImportError:
        pass


def make_pool(n: int | None = None):
    import multiprocessing as mp
    n = n or len(os.sched_getaffinity(0))
    return mp.get_context("spawn").Pool(n, initializer=_one_blas_thread)


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    from vllm_b200.kernels.decode_paged_attention import paged_decode

    cfg = C3
    pool = make_pool() if (rank == 0 and not args.no_cpu_baseline) else None
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    hkv_all, hq_all = cfg["num_kv_heads"], cfg["num_q_heads"]
    if hkv_all % world:
        raise SystemExit(f"--gpus {world} must divide {hkv_all} KV heads")
    hkv = hkv_all // world
    hq = hq_all // world
    lens = c3_lengths()
    bt = c3_block_tables(lens)
    B, nb, bs, D = cfg["batch"], cfg["pool_blocks"], cfg["block_size"], cfg["head_dim"]

    gen = torch.Generator(device=dev)
    gen.manual_seed(1000 + rank)
    kv_cache = torch.empty((2, nb, bs, hkv, D), dtype=torch.bfloat16, device=dev)
    for i in range(2):
        for c in range(0, nb, 20000):
            kv_cache[i, c:c + 20000].normal_(generator=gen)
    q = torch.randn((B, hq, D), generator=gen, device=dev).to(torch.bfloat16)
    d_bt = torch.from_numpy(bt).to(dev)
    d_len = torch.from_numpy(lens).to(dev)
    out = torch.empty_like(q)
    scale = 1.0 / math.sqrt(D)

    def step():
        paged_decode(q, kv_cache, d_bt, d_len, scale, out=out)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(dev)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clk:
        t_start.record(stream)
        for i in range(args.steps):
            ev[i][0].record(stream)
            step()
            ev[i][1].record(stream)
        t_end.record(stream)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    total_ms = t_start.elapsed_time(t_end)
    per_launch_ms = float(np.mean([a.elapsed_time(b) for a, b in ev]))

    # e2e through the public API with host buffers: H2D of q, block tables and
    # lengths from pinned memory, the call, D2H of the output, every step.
    h_q = q.cpu().pin_memory()
    h_bt = torch.from_numpy(bt).pin_memory()
    h_len = torch.from_numpy(lens).pin_memory()
    h_out = torch.empty(q.shape, dtype=q.dtype).pin_memory()
    e_q, e_bt, e_len = torch.empty_like(q), torch.empty_like(d_bt), torch.empty_like(d_len)

    def e2e_step():
        e_q.copy_(h_q, non_blocking=True)
        e_bt.copy_(h_bt, non_blocking=True)
        e_len.copy_(h_len, non_blocking=True)
        paged_decode(e_q, kv_cache, e_bt, e_len, scale, out=out)
        h_out.copy_(out, non_blocking=True)

    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)

    t = torch.tensor([total_ms, per_launch_ms, e2e_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms, per_launch_ms, e2e_ms = t.tolist()
    if rank != 0:
        return
    step_bytes = decode_bytes(lens, hkv_all, hq_all)      # all ranks together
    rank_bytes = decode_bytes(lens, hkv, hq)               # one launch on one GPU
    value = step_bytes * args.steps / (total_ms / 1e3) / 1e9
    e2e_val = step_bytes * args.steps / (e2e_ms / 1e3) / 1e9
    peaks, peak_src = load_peaks()
    achieved = rank_bytes / (per_launch_ms / 1e3) / 1e9
    cpu = (cpu_decode_baseline(lens, hkv_all, hq_all, args.cpu_budget, pool)
           if pool is not None and world == 1 else None)
    h2d = h_q.numel() * 2 + h_bt.numel() * 4 + h_len.numel() * 4
    line = {
        "metric": "paged-decode HBM GB/s (C3: Qwen3-8B heads, B=256, ctx log-U[512,32768])",
        "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": round(total_ms / args.steps, 4),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded C3 lengths/tables; K,V,q ~ N(0,1) bf16)",
        "config": {"workload": "C3 paged decode attention", "batch": B,
                   "num_q_heads": hq_all, "num_kv_heads": hkv_all, "head_dim": D,
                   "block_size": bs, "pool_blocks": nb, "table_width": C3["table_width"],
                   "ctx_tokens": int(lens.sum()),
                   "parallelism": f"tp{world} by KV head" if world > 1 else "single GPU",
                   "l2": f"inputs larger than L2 ({step_bytes / 1e9:.2f} GB read per step)"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1),
                     "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / peaks["hbm_gbs"], 4),
                     "peak_source": f"{peak_src} hbm_gbs",
                     "kernel": "vj_paged_decode (plan + chunk + combine launches)",
                     "traffic": decode_traffic(int(lens.sum())) if world == 1 else None,
                     "traffic_source": "ncu dram bytes of a 48-sequence C3 capture, scaled "
                                       "by context tokens"},
        "e2e": {"value": round(e2e_val, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": h_out.numel() * 2},
        "gpu_launches": 3 * args.steps,
        "clocks": clk.summary(),
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    print(json.dumps(line), flush=True)
    if pool is not None:
        pool.terminate()


def _cpu_kvstore_chunk(args):
    T, hq, hkv, seed = args
    from oracle import kv_store as okv
    from oracle.bf16 import bf16
    rng = np.random.default_rng(seed)
    d = 128
    q = bf16(rng.standard_normal((T, hq, d)))
    k = bf16(rng.standard_normal((T, hkv, d)))
    v = bf16(rng.standard_normal((T, hkv, d)))
    ones = np.ones(d, np.float32)
    kc = np.zeros(((T + 15) // 16, 16, hkv, d), np.float32)
    vc = np.zeros_like(kc)
    pos = rng.integers(0, 6000, T).astype(np.int32)
    t0 = time.perf_counter()
    okv.kv_store_qknorm_rope(q, k, v, ones, ones, pos, np.arange(T, dtype=np.int32), kc, vc)
    return time.perf_counter() - t0


def kvstore_bytes(T: int, hq: int, hkv: int, d: int = 128) -> int:
    """Algorithmic HBM bytes of one K3 call: q, k, v rows read; q_out and the
    K/V slots written; positions and slots read (norm weights and the RoPE
    frequencies are a few hundred bytes)."""
    return T * ((hq + 2 * hkv) * d * 2 + (hq + 2 * hkv) * d * 2 + 8)


def run_kvstore(args, rank, world, local_rank):
    """K3 on the C2 prefill batch: q/k RMSNorm + RoPE + KV-slot scatter of all
    new tokens of the 64 C2 sequences (positions prefix + i, slots from the C2
    block tables), Qwen3-8B heads. HBM-bound: one read and one write of every
    row. N > 1: TP by KV head (each rank its heads of every token)."""
    import torch
    import torch.distributed as dist
    from vllm_b200.kernels.kv_store import kv_store_qknorm_rope, rope_table

    cfg = C2
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    hq_all, hkv_all, D, bs = cfg["num_q_heads"], cfg["num_kv_heads"], cfg["head_dim"], 16
    if hkv_all % world:
        raise SystemExit(f"--gpus {world} must divide {hkv_all} KV heads")
    hq, hkv = hq_all // world, hkv_all // world
    new, pre, bt = c2_batch()
    pos_l, slot_l = [], []
    for s_, (n, p) in enumerate(zip(new, pre)):
        t = np.arange(p, p + n)
        pos_l.append(t)
        slot_l.append(bt[s_, t // bs] * bs + t % bs)
    positions = np.concatenate(pos_l).astype(np.int32)
    slots = np.concatenate(slot_l).astype(np.int32)
    T = len(slots)
    nb = cfg["pool_blocks"]
    gen = torch.Generator(device=dev)
    gen.manual_seed(2000 + rank)
    kv_cache = torch.zeros((2, nb, bs, hkv, D), dtype=torch.bfloat16, device=dev)
    q = torch.randn((T, hq, D), generator=gen, device=dev).to(torch.bfloat16)
    k = torch.randn((T, hkv, D), generator=gen, device=dev).to(torch.bfloat16)
    v = torch.randn((T, hkv, D), generator=gen, device=dev).to(torch.bfloat16)
    qw = torch.ones(D, dtype=torch.bfloat16, device=dev)
    kw = torch.ones(D, dtype=torch.bfloat16, device=dev)
    d_pos = torch.from_numpy(positions).to(dev)
    d_slot = torch.from_numpy(slots).to(dev)
    q_out = torch.empty_like(q)
    table = rope_table(dev, 1e6, int(positions.max()) + 1)

    def step():
        kv_store_qknorm_rope(q, k, v, kv_cache, d_slot, d_pos, qw, kw, q_out=q_out, table=table)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    stream = torch.cuda.current_stream(dev)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clk:
        t_start.record(stream)
        for i in range(args.steps):
            ev[i][0].record(stream)
            step()
            ev[i][1].record(stream)
        t_end.record(stream)
        torch.cuda.synchronize()
    total_ms = t_start.elapsed_time(t_end)
    per_launch_ms = float(np.mean([a.elapsed_time(b) for a, b in ev]))
    # e2e: the projected rows come from pinned host memory, q_out goes back
    h_q, h_k, h_v = q.cpu().pin_memory(), k.cpu().pin_memory(), v.cpu().pin_memory()
    h_pos, h_slot = d_pos.cpu().pin_memory(), d_slot.cpu().pin_memory()
    h_out = torch.empty(q.shape, dtype=q.dtype).pin_memory()
    e_q, e_k, e_v = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    e_pos, e_slot = torch.empty_like(d_pos), torch.empty_like(d_slot)

    def e2e_step():
        for dst, src in ((e_q, h_q), (e_k, h_k), (e_v, h_v), (e_pos, h_pos), (e_slot, h_slot)):
            dst.copy_(src, non_blocking=True)
        kv_store_qknorm_rope(e_q, e_k, e_v, kv_cache, e_slot, e_pos, qw, kw, q_out=q_out,
                             table=table)
        h_out.copy_(q_out, non_blocking=True)

    e2e_step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    t = torch.tensor([total_ms, per_launch_ms, e2e_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms, per_launch_ms, e2e_ms = t.tolist()
    if rank != 0:
        return
    step_bytes = kvstore_bytes(T, hq_all, hkv_all)
    rank_bytes = kvstore_bytes(T, hq, hkv)
    peaks, peak_src = load_peaks()
    achieved = rank_bytes / (per_launch_ms / 1e3) / 1e9
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        cores = max(1, min(16, len(os.sched_getaffinity(0))))
        chunk, n_chunks = 4096, 8 * cores          # ~0.5 s per chunk: a few seconds per core
        with make_pool(cores) as pool:
            pool.map(_cpu_kvstore_chunk, [(256, hq_all, hkv_all, i) for i in range(cores)])
            t0 = time.perf_counter()
            pool.map(_cpu_kvstore_chunk, [(chunk, hq_all, hkv_all, i) for i in range(n_chunks)])
            wall = time.perf_counter() - t0
        cpu = {"value": round(kvstore_bytes(chunk * n_chunks, hq_all, hkv_all) / wall / 1e9, 3),
               "unit": "GB/s", "cores": cores, "kind": "port",
               "sample": f"{n_chunks} chunks of {chunk} tokens over {cores} processes "
                         "(oracle.kv_store)"}
    h2d = (h_q.numel() + h_k.numel() + h_v.numel()) * 2 + (h_pos.numel() + h_slot.numel()) * 4
    line = {
        "metric": "KV-scatter + q/k RMSNorm + RoPE HBM GB/s (K3 on the C2 batch, Qwen3-8B heads)",
        "value": round(step_bytes * args.steps / (total_ms / 1e3) / 1e9, 2), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": max(args.warmup, 3),
        "ms_per_step": round(total_ms / args.steps, 4), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (C2 positions/slots; q,k,v ~ N(0,1) bf16)",
        "config": {"workload": "K3 kv_store_qknorm_rope on the C2 batch", "tokens": T,
                   "num_q_heads": hq_all, "num_kv_heads": hkv_all, "head_dim": D,
                   "parallelism": f"tp{world} by KV head" if world > 1 else "single GPU",
                   "l2": f"inputs larger than L2 ({step_bytes / 1e9:.2f} GB per step)"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"],
                     "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4),
                     "peak_source": f"{peak_src} hbm_gbs", "kernel": "kv_store_tma_kernel",
                     "traffic": (int(KVSTORE_PROFILE["dram_bytes"] * T / KVSTORE_PROFILE["tokens"])
                                 if world == 1 else None),
                     "traffic_source": "ncu dram bytes of a 16-sequence C2 capture, scaled by "
                                       "tokens"},
        "e2e": {"value": round(step_bytes * args.steps / (e2e_ms / 1e3) / 1e9, 2), "unit": "GB/s",
                "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": h_out.numel() * 2},
        "gpu_launches": args.steps,
        "clocks": clk.summary(),
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    print(json.dumps(line), flush=True)


def _cpu_prefill_seq(args):
    n, p, hkv, g, seed = args
    from oracle import attention as oatt
    rng = np.random.default_rng(seed)
    bs, d = 16, 128
    L = n + p
    npg = (L + bs - 1) // bs
    kc = rng.standard_normal((npg, bs, hkv, d), dtype=np.float32)
    vc = rng.standard_normal((npg, bs, hkv, d), dtype=np.float32)
    q = rng.standard_normal((n, hkv * g, d), dtype=np.float32)
    bt = np.arange(npg, dtype=np.int32)[None]
    t0 = time.perf_counter()
    oatt.prefill_attention(q, kc, vc, bt, np.array([0, n], np.int32), np.array([L], np.int32),
                           1 / math.sqrt(d))
    return time.perf_counter() - t0


def cpu_prefill_baseline(new, pre, hkv, hq, budget_s, pool) -> dict:
    """Oracle prefill on a seeded subsample of C2 sequences (shortest first so the
    bounded sample covers several sequences), all host cores."""
    order = np.argsort(new + pre)
    cores = pool._processes if pool is not None else 1
    done, sample, t_cpu = 0, [], 0.0
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < budget_s and done < len(order):
        idx = order[done:done + cores]
        done += len(idx)
        args = [(int(new[i]), int(pre[i]), hkv, hq // hkv, int(i)) for i in idx]
        times = (pool.map(_cpu_prefill_seq, args) if pool is not None
                 else [_cpu_prefill_seq(a) for a in args])
        t_cpu += float(sum(times))
        sample.extend(int(i) for i in idx)
    fl = prefill_flops(new[sample], pre[sample], hq)
    return {"value": fl / (t_cpu / cores) / 1e12, "unit": "TFLOP/s", "cores": cores,
            "kind": "port",
            "sample": f"{len(sample)} of {len(new)} C2 sequences ({int(new[sample].sum())} new "
                      f"tokens) through the numpy oracle (oracle/attention.py:prefill_attention),"
                      f" one sequence per process; {t_cpu:.1f} s of compute over {cores} "
                      f"processes"}


def run_prefill(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    from vllm_b200.kernels.prefill_paged_attention import paged_prefill, pipeline_error

    cfg = C2
    pool = make_pool() if (rank == 0 and not args.no_cpu_baseline) else None
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    hkv_all, hq_all, D = cfg["num_kv_heads"], cfg["num_q_heads"], cfg["head_dim"]
    if hkv_all % world:
        raise SystemExit(f"--gpus {world} must divide {hkv_all} KV heads")
    hkv, hq = hkv_all // world, hq_all // world
    if args.batch is not None:
        cfg["num_seqs"] = args.batch
    if args.pool_blocks is not None:
        cfg["pool_blocks"] = args.pool_blocks
    new, pre, bt = c2_batch(cfg)
    nb, bs = cfg["pool_blocks"], cfg["block_size"]
    T = int(new.sum())
    gen = torch.Generator(device=dev)
    gen.manual_seed(2000 + rank)
    kv_cache = torch.empty((2, nb, bs, hkv, D), dtype=torch.bfloat16, device=dev)
    for i in range(2):
        for c in range(0, nb, 20000):
            kv_cache[i, c:c + 20000].normal_(generator=gen)
    q = torch.randn((T, hq, D), generator=gen, device=dev).to(torch.bfloat16)
    cu = np.concatenate([[0], np.cumsum(new)]).astype(np.int32)
    ctx = (new + pre).astype(np.int32)
    d_bt, d_cu, d_ctx = (torch.from_numpy(x).to(dev) for x in (bt, cu, ctx))
    out = torch.empty_like(q)
    maxq = int(new.max())

    def step():
        paged_prefill(q, kv_cache, d_bt, d_cu, d_ctx, max_seqlen_q=maxq, out=out)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    if pipeline_error(dev):
        raise SystemExit("prefill pipeline wait timed out")
    if world > 1:
        dist.barrier()
    stream = torch.cuda.current_stream(dev)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    t0e, t1e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clk:
        t0e.record(stream)
        for i in range(args.steps):
            ev[i][0].record(stream)
            step()
            ev[i][1].record(stream)
        t1e.record(stream)
        torch.cuda.synchronize()
    total_ms = t0e.elapsed_time(t1e)
    per_launch_ms = float(np.mean([a.elapsed_time(b) for a, b in ev]))

    h_q = q.cpu().pin_memory()
    h_bt, h_cu, h_ctx = (torch.from_numpy(x).pin_memory() for x in (bt, cu, ctx))
    h_out = torch.empty(q.shape, dtype=q.dtype).pin_memory()
    e_q, e_bt, e_cu, e_ctx = (torch.empty_like(x) for x in (q, d_bt, d_cu, d_ctx))

    def e2e_step():
        e_q.copy_(h_q, non_blocking=True)
        e_bt.copy_(h_bt, non_blocking=True)
        e_cu.copy_(h_cu, non_blocking=True)
        e_ctx.copy_(h_ctx, non_blocking=True)
        paged_prefill(e_q, kv_cache, e_bt, e_cu, e_ctx, max_seqlen_q=maxq, out=out)
        h_out.copy_(out, non_blocking=True)

    for _ in range(3):
        e2e_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1)
    t = torch.tensor([total_ms, per_launch_ms, e2e_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms, per_launch_ms, e2e_ms = t.tolist()
    if rank != 0:
        return
    fl_all = prefill_flops(new, pre, hq_all)
    fl_rank = prefill_flops(new, pre, hq)
    value = fl_all * args.steps / (total_ms / 1e3) / 1e12
    peaks, src = load_peaks()
    achieved = fl_rank / (per_launch_ms / 1e3) / 1e12
    cpu = (cpu_prefill_baseline(new, pre, hkv_all, hq_all, args.cpu_budget, pool)
           if pool is not None and world == 1 else None)
    line = {
        "metric": "paged-prefill TFLOP/s (C2: Qwen3-8B heads, 64 seqs, new U[128,4096], "
                  "prefix U[0,2048], causal)",
        "value": round(value, 2), "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": round(total_ms / args.steps, 4),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded C2 lengths/prefixes/tables; q,K,V ~ N(0,1) bf16)",
        "config": {"workload": "C2 paged prefill attention", "num_seqs": len(new),
                   "new_tokens": T, "prefix_tokens": int(pre.sum()), "num_q_heads": hq_all,
                   "num_kv_heads": hkv_all, "head_dim": D, "block_size": bs, "pool_blocks": nb,
                   "parallelism": f"tp{world} by KV head" if world > 1 else "single GPU",
                   "l2": f"inputs larger than L2 (q {T * hq_all * D * 2 / 1e9:.2f} GB)"},
        "roofline": {"bound": "tensor", "achieved": round(achieved, 1),
                     "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": round(achieved / peaks["bf16_tflops"], 4),
                     "peak_source": f"{src} bf16_tflops (burst)",
                     "kernel": "vj_paged_prefill (prefill_kernel + zero-tail)",
                     "traffic": None},
        "e2e": {"value": round(fl_all * args.steps / (e2e_ms / 1e3) / 1e12, 2), "unit": "TFLOP/s",
                "h2d_bytes_per_step": h_q.numel() * 2 + (h_bt.numel() + h_cu.numel() +
                                                         h_ctx.numel()) * 4,
                "d2h_bytes_per_step": h_out.numel() * 2},
        "gpu_launches": 2 * args.steps,
        "clocks": clk.summary(),
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    print(json.dumps(line), flush=True)
    if pool is not None:
        pool.terminate()


# ncu capture of decode_chunk_kernel on the first 48 C3 sequences (402,759
# context tokens): dram read + write bytes.
# DRAM traffic grows with the context tokens streamed, so a full C3 launch is
# scaled by its context-token count.
DECODE_PROFILE = {"ctx_tokens": 402_759, "dram_bytes": 1_651_833_000 + 23_638_016}
# K3 (kv_store_tma_kernel) on the first 16 C2 sequences, 34,069 tokens
KVSTORE_PROFILE = {"tokens": 34_069, "dram_bytes": 424_025_344 + 367_532_544}


def decode_traffic(ctx_tokens: int) -> int:
    return int(DECODE_PROFILE["dram_bytes"] * ctx_tokens / DECODE_PROFILE["ctx_tokens"])


# ---------------------------------------------------------------------------
# reference arm: the reference's algorithm on host CPU cores (oracle port)
# ---------------------------------------------------------------------------
def run_reference_e2e(args, rank, world):
    """C4 output tok/s of the reference's algorithm on the host CPU cores: the
    oracle restatement of the Qwen3-8B forward, one bounded sample per step
    (CpuQwen3Sample), scaled to the whole 512-request job."""
    if rank != 0:
        return
    from vllm_b200.model.qwen3 import get_config
    mcfg = get_config(C4["model"])
    prompts, outs = c4_requests(C4, mcfg.vocab_size)
    sample = CpuQwen3Sample(mcfg, prompts, outs)
    ptoks, otoks = sum(len(p) for p in prompts), sum(outs)
    for _ in range(args.warmup):
        sample.measure()
    vals = []
    t0 = time.perf_counter()
    for _ in range(args.steps):
        vals.append(sample.tok_per_s(sample.measure(), ptoks, otoks))
    wall = time.perf_counter() - t0
    v = float(np.mean(vals))
    cores = len(os.sched_getaffinity(0))
    line = {
        "impl": "reference", "metric": C4_METRIC, "value": round(v, 4), "unit": "tok/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(wall / args.steps * 1e3, 1), "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded random token ids and lengths; random-init N(0,0.02) weights)",
        "config": {"workload": "C4 end-to-end continuous batching", "model": C4["model"],
                   "num_requests": C4["num_requests"], "output_tokens": otoks,
                   "prompt_tokens": ptoks, "parallelism": "host CPU cores"},
        "cpu_baseline": {"value": round(v, 4), "unit": "tok/s", "cores": cores, "kind": "port",
                         "sample": sample.describe(cores)},
        "e2e": {"value": round(v, 4), "unit": "tok/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "note": "jax/flax are not installable in this image (no network); the reference's "
                "forward runs as its NumPy restatement (oracle/), fp32 GEMMs with per-op "
                "bf16 rounding, on every host core through numpy BLAS.",
    }
    print(json.dumps(line), flush=True)


def run_reference(args, rank, world):
    if args.workload == "e2e":
        return run_reference_e2e(args, rank, world)
    if rank != 0:
        return
    pool = make_pool()
    lens = c3_lengths()
    hkv, hq = C3["num_kv_heads"], C3["num_q_heads"]
    # each step: a bounded sample of the C3 batch (budget split over the steps)
    budget = max(1.0, args.ref_budget / max(args.steps + args.warmup, 1))
    for _ in range(args.warmup):
        cpu_decode_baseline(lens, hkv, hq, budget, pool)
    vals, samples = [], []
    t0 = time.perf_counter()
    for _ in range(args.steps):
        r = cpu_decode_baseline(lens, hkv, hq, budget, pool)
        vals.append(r["value"])
        samples.append(r)
    wall = time.perf_counter() - t0
    v = float(np.mean(vals))
    line = {
        "impl": "reference",
        "metric": "paged-decode HBM GB/s (C3: Qwen3-8B heads, B=256, ctx log-U[512,32768])",
        "value": round(v, 4), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(wall / args.steps * 1e3, 1),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded C3 lengths)",
        "config": {"workload": "C3 paged decode attention", "batch": C3["batch"],
                   "num_q_heads": hq, "num_kv_heads": hkv, "head_dim": 128, "block_size": 16},
        "cpu_baseline": {"value": round(v, 4), "unit": "GB/s", "cores": samples[-1]["cores"],
                         "kind": "port", "sample": samples[-1]["sample"]},
        "e2e": {"value": round(v, 4), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "note": "jax/flax are not installable in this image (no network); the reference's "
                "paged-attention algorithm runs as its NumPy restatement (oracle/).",
    }
    print(json.dumps(line), flush=True)
    pool.terminate()


C4_METRIC = ("output tok/s Qwen3-8B continuous batching (C4: 512 requests, prompts "
             "U[100,1024], outputs U[100,1024])")

# C4: Qwen3-8B continuous batching
C4 = dict(model="Qwen3-8B", num_requests=512, prompt_min=100, prompt_max=1024, out_min=100,
          out_max=1024, max_num_batched_tokens=16384, max_num_seqs=512, seed=0)


# C5: Qwen3-32B, chunked prefill mixed with decode.
# Prompt lengths clip(lognormal(ln 1024, sigma), 32, 16384) with sigma = 1.0;
# the token budget per step is not named by the config: 8192 is used.
C5 = dict(model="Qwen3-32B", num_requests=1024, prompt_median=1024, sigma=1.0, prompt_min=32,
          prompt_max=16384, out_min=64, out_max=2048, max_num_batched_tokens=8192,
          max_num_seqs=512, seed=0)


def c5_requests(cfg=C5, vocab=151936):
    rng = np.random.default_rng(cfg["seed"])
    n = cfg["num_requests"]
    plen = np.clip(np.rint(rng.lognormal(math.log(cfg["prompt_median"]), cfg["sigma"], n)),
                   cfg["prompt_min"], cfg["prompt_max"]).astype(np.int64)
    olen = rng.integers(cfg["out_min"], cfg["out_max"] + 1, n)
    prompts = [rng.integers(0, vocab, int(L)).tolist() for L in plen]
    return prompts, [int(x) for x in olen]


def c4_requests(cfg=C4, vocab=151936):
    rng = np.random.default_rng(cfg["seed"])
    n = cfg["num_requests"]
    plen = rng.integers(cfg["prompt_min"], cfg["prompt_max"] + 1, n)
    olen = rng.integers(cfg["out_min"], cfg["out_max"] + 1, n)
    prompts = [rng.integers(0, vocab, int(L)).tolist() for L in plen]
    return prompts, [int(x) for x in olen]


class CpuQwen3Sample:
    """A bounded CPU sample of one engine's work at a Qwen3 architecture,
    run through the oracle's restatement of the reference forward
    (oracle/qwen3.py: same layer dataflow, bf16 rounding per op, fp32 GEMM
    accumulation through numpy BLAS on every host core):
      * one decoder layer of a decode step at `batch` rows whose contexts are
        drawn from the workload's mid-generation lengths (prompt + U[0, out]),
      * 1/16 of the lm_head GEMM of those rows,
      * one decoder layer of a prefill of a median-length prompt.
    tok_per_s() scales these to the whole job: every output token costs
    (layers x decode layer + lm_head) / batch and every prompt token layers x
    prefill layer / prompt length (the reference computes no logits in
    prefill, model_runner.py:41-59)."""

    def __init__(self, mcfg, prompts, outs, batch=32, seed=0):
        from types import SimpleNamespace

        from oracle.bf16 import bf16
        from oracle.qwen3 import OracleQwen3
        rng = np.random.default_rng(seed)
        H, I, D = mcfg.hidden_size, mcfg.intermediate_size, mcfg.head_dim
        Hq, Hkv = mcfg.num_attention_heads, mcfg.num_key_value_heads
        self.mcfg, self.batch = mcfg, batch

        def w(*shape):
            return bf16(rng.standard_normal(shape, dtype=np.float32) * np.float32(0.02))
        one_h, one_d = np.ones(H, np.float32), np.ones(D, np.float32)
        layer = {"w_qkv": w((Hq + 2 * Hkv) * D, H), "w_o": w(H, Hq * D),
                 "w_gate_up": w(2 * I, H), "w_down": w(H, I), "ln1": one_h, "ln2": one_h,
                 "q_norm": one_d, "k_norm": one_d}
        self.vocab_frac = 16
        self.lm = w(mcfg.vocab_size // self.vocab_frac, H)
        pick = rng.choice(len(prompts), size=batch, replace=False)
        self.ctx = [int(len(prompts[i]) + rng.integers(0, outs[i] + 1)) for i in pick]
        self.prompt_len = int(np.median([len(p) for p in prompts]))
        bs = 16
        nblk = sum((L + bs - 1) // bs for L in self.ctx) + (self.prompt_len + bs - 1) // bs
        cfg1 = SimpleNamespace(**{**mcfg.__dict__, "num_hidden_layers": 1})
        self.model = OracleQwen3(cfg1, {"layers": [layer]}, nblk, bs)
        self.model.kc[0][:] = bf16(rng.standard_normal(self.model.kc[0].shape, dtype=np.float32))
        self.model.vc[0][:] = bf16(rng.standard_normal(self.model.vc[0].shape, dtype=np.float32))
        self.tables = np.zeros((batch, max((L + bs - 1) // bs for L in self.ctx)), np.int64)
        o = 0
        for i, L in enumerate(self.ctx):
            n = (L + bs - 1) // bs
            self.tables[i, :n] = np.arange(o, o + n)
            o += n
        self.pre_blocks = np.arange(o, o + (self.prompt_len + bs - 1) // bs)
        self.x_dec = bf16(rng.standard_normal((batch, H), dtype=np.float32))
        self.x_pre = bf16(rng.standard_normal((self.prompt_len, H), dtype=np.float32))

    def measure(self):
        """(decode layer s, full lm_head s, prefill layer s) of one sample."""
        bs = 16
        pos = [L - 1 for L in self.ctx]
        slots = [int(self.tables[i, (L - 1) // bs]) * bs + (L - 1) % bs
                 for i, L in enumerate(self.ctx)]
        t0 = time.perf_counter()
        h = self.model.decode_layers(self.x_dec, pos, slots, self.tables, self.ctx)
        t1 = time.perf_counter()
        np.matmul(h, self.lm.T)
        t2 = time.perf_counter()
        P = self.prompt_len
        pslots = [int(self.pre_blocks[t // bs]) * bs + t % bs for t in range(P)]
        self.model.prefill_layers(self.x_pre, list(range(P)), pslots, [0, P], 1)
        t3 = time.perf_counter()
        return t1 - t0, (t2 - t1) * self.vocab_frac, t3 - t2

    def tok_per_s(self, m, prompt_tokens: int, output_tokens: int) -> float:
        t_dec, t_lm, t_pre = m
        L = self.mcfg.num_hidden_layers
        per_out = (L * t_dec + t_lm) / self.batch
        per_prompt = L * t_pre / self.prompt_len
        return output_tokens / (output_tokens * per_out + prompt_tokens * per_prompt)

    def describe(self, cores: int) -> str:
        return (f"oracle.qwen3 restatement of the reference forward on {cores} host cores "
                f"(numpy BLAS): 1 of {self.mcfg.num_hidden_layers} decoder layers at "
                f"{self.batch} decode rows (contexts prompt + U[0, out] of sampled requests), "
                f"1/{self.vocab_frac} of lm_head, 1 layer of a {self.prompt_len}-token prefill; "
                "scaled to the whole job by layers, rows and tokens")


def run_e2e(args, rank, world, local_rank):
    """C4 end to end: output tokens/s of Engine.generate over 512 requests
    (random prompts and output lengths, greedy, ignore_eos), tensor parallel
    over `world` GPUs (KV heads and MLP split, NCCL all-reduce after o_proj and
    down_proj). The timed region is the whole generate() call: host scheduling,
    metadata uploads, prefill and CUDA-graph decode steps, token D2H."""
    import torch
    import torch.distributed as dist
    from vllm_b200 import Config, SamplingParams, _native
    from vllm_b200.model.qwen3 import get_config
    from vllm_b200.src.engine import Engine

    c5 = args.workload == "c5"
    cfg = dict(C5 if c5 else C4)
    if args.model:
        cfg["model"] = args.model
    if args.batch is not None:
        cfg["num_requests"] = args.batch
    if args.max_num_seqs:
        cfg["max_num_seqs"] = args.max_num_seqs
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    mcfg = get_config(cfg["model"])
    all_prompts, all_outs = (c5_requests if c5 else c4_requests)(cfg, mcfg.vocab_size)
    max_len = max(len(p) + o for p, o in zip(all_prompts, all_outs))
    # world = dp x tp: dp engine replicas, each tensor parallel over tp GPUs,
    # request i served by replica i % dp
    tp = args.tp or world
    if world % tp:
        raise SystemExit("--tp must divide the number of GPUs")
    dp = world // tp
    replica = rank // tp
    pg = None
    if world > 1:
        groups = [dist.new_group(list(range(d * tp, (d + 1) * tp))) for d in range(dp)]
        pg = groups[replica] if tp > 1 else None
    prompts, outs = all_prompts[replica::dp], all_outs[replica::dp]
    econf = Config(model=cfg["model"], max_num_batched_tokens=cfg["max_num_batched_tokens"],
                   max_num_seqs=cfg["max_num_seqs"], num_blocks=0, block_size=16,
                   tensor_parallel_size=tp, gpu_memory_utilization=0.9,
                   max_model_len=((max_len + 15) // 16) * 16, compat=False,
                   enable_chunked_prefill=c5, fused_gemm_max_rows=args.fused_gemm)

    def progress(msg):
        print(f"[rank {rank}] {msg}", file=sys.stderr, flush=True)

    eng = Engine(econf, dev, seed=0, process_group=pg, max_slots=cfg["num_requests"] + 8)
    progress(f"engine ready ({eng.config.num_blocks} blocks)")
    eng.runner.capture_all(cfg["max_num_seqs"])
    progress("decode graphs captured" if eng.runner.use_cuda_graphs else "eager decode (TP)")
    params = [SamplingParams(temperature=0, max_new_tokens=o, ignore_eos=True) for o in outs]
    stream = torch.cuda.current_stream(dev)

    def one_pass():
        """One step: generate() over the whole request set. Prompts go host ->
        device and every step's tokens device -> host inside it."""
        for k in eng.stats:
            eng.stats[k] = 0 if isinstance(eng.stats[k], int) else 0.0
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        res = eng.generate(prompts, params)
        e1.record(stream)
        torch.cuda.synchronize()
        assert [len(r) for r in res] == outs
        return e0.elapsed_time(e1) / 1e3

    for i in range(args.warmup):
        progress(f"warm-up generate {i + 1}/{args.warmup}: {one_pass():.2f} s")
    eng.runner.decode_events = []
    launches0 = _native.launch_count
    times, stats = [], []
    with ClockSampler(local_rank) as clk:
        for i in range(args.steps):
            times.append(one_pass())
            stats.append(dict(eng.stats))
            progress(f"timed generate {i + 1}/{args.steps}: {times[-1]:.2f} s")
    launches = _native.launch_count - launches0
    dec_s = sum(a.elapsed_time(b) for a, b in eng.runner.decode_events) / 1e3
    eng.runner.decode_events = None
    t = torch.tensor([sum(times)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_s = float(t.item())
    eng.close()       # every rank: graphs and the NVLink communicator
    if rank != 0:
        return
    out_tokens = sum(all_outs)
    value = out_tokens * args.steps / total_s
    peaks, src = load_peaks()
    # decode-step roofline: weights of one rank + K/V of every context token
    # per decode step, over the CUDA-event time of the decode forwards
    wbytes = sum(p.numel() * 2 for lw in eng.weights.layers for p in
                 (lw.w_qkv, lw.w_o, lw.w_gate_up, lw.w_down)) + eng.weights.lm_head.numel() * 2
    kvb = mcfg.num_hidden_layers * 2 * (mcfg.num_key_value_heads // tp) * mcfg.head_dim * 2
    dec_steps = sum(st["decode_steps"] for st in stats)
    dec_ctx = sum(st["decode_ctx_tokens"] for st in stats)
    achieved = (dec_steps * wbytes + dec_ctx * kvb) / max(dec_s, 1e-9) / 1e9
    st = stats[-1]
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        sample = CpuQwen3Sample(mcfg, all_prompts, all_outs)
        sample.measure()                                   # warm the BLAS pools
        m = [sample.measure() for _ in range(2)]
        med = tuple(float(np.median([x[j] for x in m])) for j in range(3))
        cores = len(os.sched_getaffinity(0))
        cpu = {"value": round(sample.tok_per_s(med, sum(len(p) for p in all_prompts),
                                               out_tokens), 3),
               "unit": "tok/s", "cores": cores, "kind": "port",
               "sample": sample.describe(cores)}
    if c5:
        metric = (f"output tok/s {cfg['model']} continuous batching with chunked prefill (C5: "
                  f"{cfg['num_requests']} requests, prompts clip(lognormal(ln 1024, "
                  f"{cfg['sigma']}), 32, 16384), outputs U[64,2048])")
        workload = "C5 end-to-end, chunked prefill mixed with decode"
    else:
        metric = C4_METRIC
        workload = "C4 end-to-end continuous batching"
    line = {
        "metric": metric,
        "value": round(value, 1), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(total_s / args.steps * 1e3, 1),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded random token ids and lengths; random-init N(0,0.02) weights)",
        "config": {"workload": workload, "model": cfg["model"],
                   "fused_gemm_max_rows": args.fused_gemm,
                   "step": "one Engine.generate() over the whole request set",
                   "num_requests": cfg["num_requests"], "output_tokens": out_tokens,
                   "prompt_tokens": sum(len(p) for p in all_prompts),
                   "chunked_prefill": c5,
                   "max_num_batched_tokens": cfg["max_num_batched_tokens"],
                   "max_num_seqs": cfg["max_num_seqs"], "num_blocks": eng.config.num_blocks,
                   "parallelism": (f"dp{dp}x" if dp > 1 else "") + f"tp{tp}" if world > 1
                   else "single GPU",
                   "engine_steps": st["steps"], "decode_steps": st["decode_steps"],
                   "decode_s_per_pass": round(dec_s / args.steps, 3),
                   "timing": "CUDA events around each generate(), max over ranks",
                   "l2": "decode steps stream all weights + KV (> L2)"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"],
                     "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4),
                     "peak_source": f"{src} hbm_gbs",
                     "kernel": "decode forward (weights of one rank + KV of every context "
                               "token per step / CUDA-event time of the decode forwards)",
                     "traffic": None},
        "e2e": {"value": round(value, 1), "unit": "tok/s",
                "h2d_bytes_per_step": st["h2d_bytes"], "d2h_bytes_per_step": st["d2h_bytes"],
                "note": "the step is the public generate() call itself: prompts are copied "
                        "host->device and tokens device->host inside every pass"},
        "gpu_launches": launches,
        "clocks": clk.summary(),
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    print(json.dumps(line), flush=True)


def run_c4step(args, rank, world, local_rank):
    """One Qwen3-8B decode step (the C4 engine's decode forward: 36 layers,
    K3, paged decode, cuBLAS GEMMs, norms, lm_head) replayed as a CUDA graph
    at batch --batch (default 512) and context --context (default 840, C4's
    mean context during generation), device-timed with CUDA events; the
    per-kernel shares of three replays (torch profiler) go to stderr. Its
    roofline: weights + KV of every context token per step."""
    import collections

    import torch
    from torch.profiler import ProfilerActivity, profile
    from vllm_b200 import _native
    from vllm_b200.kernels.decode_paged_attention import decode_workspace_bytes
    from vllm_b200.kernels.kv_store import rope_table
    from vllm_b200.kernels.metadata import DecodeMeta
    from vllm_b200.model.qwen3 import Qwen3Model, Qwen3Weights, get_config
    if world > 1:
        raise SystemExit("--workload c4step runs on one GPU")
    B, L = args.batch or 512, args.context
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    cfg = get_config("Qwen3-8B")
    w = Qwen3Weights(cfg, dev, seed=0)
    m = Qwen3Model(w)
    if args.fused_gemm:
        m.enable_fused_gemm(args.fused_gemm)
    bs, D, Hkv = 16, cfg.head_dim, cfg.num_key_value_heads
    pages = (L + bs - 1) // bs
    nb = B * pages + 8
    gen = torch.Generator(device=dev)
    gen.manual_seed(5)
    kv = [torch.randn((2, nb, bs, Hkv, D), generator=gen, device=dev).to(torch.bfloat16)
          for _ in range(cfg.num_hidden_layers)]
    m.decode_workspace = torch.empty(decode_workspace_bytes(B, cfg.num_attention_heads, D),
                                     dtype=torch.uint8, device=dev)
    m.rope_table = rope_table(dev, cfg.rope_theta, L + 1)
    perm = torch.randperm(B * pages, generator=gen, device=dev).to(torch.int32)
    bt = perm.view(B, pages)
    ctx = torch.full((B,), L, device=dev, dtype=torch.int32)
    ids = torch.randint(0, cfg.vocab_size, (B,), generator=gen, device=dev).to(torch.int32)
    slots = (bt[:, -1] * bs + (L - 1) % bs).to(torch.int32)
    meta = DecodeMeta(ids, ctx - 1, slots, bt, ctx, B)
    for _ in range(max(args.warmup, 3)):
        m.forward_decode(meta, kv)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    before = _native.launch_count
    with torch.cuda.graph(graph):
        m.forward_decode(meta, kv)
    per_step = _native.launch_count - before
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clk:
        e0.record(stream)
        for _ in range(args.steps):
            graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    wbytes = sum(p.numel() * 2 for lw in w.layers for p in
                 (lw.w_qkv, lw.w_o, lw.w_gate_up, lw.w_down)) + w.lm_head.numel() * 2
    kvbytes = B * L * cfg.num_hidden_layers * 2 * Hkv * D * 2
    peaks, src = load_peaks()
    achieved = (wbytes + kvbytes) / (ms / 1e3) / 1e9
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
    agg = collections.defaultdict(lambda: [0, 0.0])
    for e in prof.key_averages():
        if e.device_time_total > 0:
            agg[e.key][0] += e.count
            agg[e.key][1] += e.device_time_total
    tot = sum(v[1] for v in agg.values()) or 1.0
    print("per-kernel device time of one decode step (3 graph replays, torch profiler):",
          file=sys.stderr)
    for k, (c, t) in sorted(agg.items(), key=lambda kv: -kv[1][1])[:20]:
        print(f"  {t / 3 / 1000:8.3f} ms/step {100 * t / tot:5.1f}%  launches/step "
              f"{c / 3:6.1f}  {k[:100]}", file=sys.stderr)
    line = {
        "metric": f"Qwen3-8B decode step ms (batch {B}, context {L})",
        "value": round(ms, 4), "unit": "ms", "n_gpus": 1, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": round(ms, 4),
        "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (random-init N(0,0.02) weights, N(0,1) KV, random tables)",
        "config": {"workload": "C4 decode step (CUDA graph)", "batch": B, "context": L,
                   "fused_gemm_max_rows": args.fused_gemm,
                   "l2": "weights + KV per step > L2"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"],
                     "unit": "GB/s", "frac": round(achieved / peaks["hbm_gbs"], 4),
                     "peak_source": f"{src} hbm_gbs",
                     "kernel": "decode step (weights + KV bytes / step time)", "traffic": None},
        "gpu_launches": per_step * args.steps,
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)


def run_mixedstep(args, rank, world, local_rank):
    """One chunked-prefill step of Qwen3-8B (the engine's forward_mixed):
    --batch decode rows (default 128) at context --context, packed first,
    then 2 prompt chunks of 2048 new tokens after cached prefixes of 1024 and
    3072 tokens. Each layer's attention over both kinds is one
    vj_paged_attention_mixed launch. CUDA events around --steps eager
    forwards; per-kernel device time and launches of one step (torch
    profiler) on stderr. The line's value: ms per step."""
    import collections

    import torch
    from torch.profiler import ProfilerActivity, profile
    from vllm_b200 import _native
    from vllm_b200.kernels.kv_store import rope_table
    from vllm_b200.kernels.metadata import RangesMeta
    from vllm_b200.model.qwen3 import Qwen3Model, Qwen3Weights, get_config
    if world > 1:
        raise SystemExit("--workload mixedstep runs on one GPU")
    nd, L = args.batch or 128, args.context
    chunks = [(1024, 2048), (3072, 2048)]            # (cached prefix, new tokens)
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    cfg = get_config("Qwen3-8B")
    m = Qwen3Model(Qwen3Weights(cfg, dev, seed=0))
    bs, D, Hkv, Hq = 16, cfg.head_dim, cfg.num_key_value_heads, cfg.num_attention_heads
    ctx = [L] * nd + [p + n for p, n in chunks]
    S = len(ctx)
    pages = [(c + bs - 1) // bs for c in ctx]
    width = max(pages)
    gen = torch.Generator(device=dev)
    gen.manual_seed(7)
    perm = torch.randperm(sum(pages), generator=gen, device=dev).to(torch.int32)
    bt = torch.full((S, width), -1, dtype=torch.int32, device=dev)
    o = 0
    for s, p in enumerate(pages):
        bt[s, :p] = perm[o:o + p]
        o += p
    nb = sum(pages) + 8
    kv = [torch.randn((2, nb, bs, Hkv, D), generator=gen, device=dev).to(torch.bfloat16)
          for _ in range(cfg.num_hidden_layers)]
    pos, cu = [], [0]
    for s in range(S):
        start, n = (ctx[s] - 1, 1) if s < nd else chunks[s - nd]
        pos += list(range(start, start + n))
        cu.append(cu[-1] + n)
    T = cu[-1]
    pos_t = torch.tensor(pos, dtype=torch.int32, device=dev)
    seq_of = torch.repeat_interleave(torch.arange(S, device=dev),
                                     torch.tensor([cu[i + 1] - cu[i] for i in range(S)],
                                                  device=dev))
    slots = (bt[seq_of, (pos_t // bs).long()] * bs + pos_t % bs).to(torch.int32)
    rows = torch.tensor(cu[1:], dtype=torch.int64, device=dev) - 1
    meta = RangesMeta(torch.randint(0, cfg.vocab_size, (T,), generator=gen, device=dev)
                      .to(torch.int32), pos_t, slots, bt,
                      torch.tensor(cu, dtype=torch.int32, device=dev),
                      torch.tensor(ctx, dtype=torch.int32, device=dev), S, T,
                      max(n for _, n in chunks), rows, rows, rows)
    m.decode_workspace = torch.empty(
        max(_native.load().vj_paged_attention_mixed_workspace_size(nd, Hq, D, 0), 16),
        dtype=torch.uint8, device=dev)
    m.rope_table = rope_table(dev, cfg.rope_theta, max(ctx) + 1)

    def step():
        return m.forward_mixed(meta, kv, nd, rows)

    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream(dev)
    before = _native.launch_count
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clk:
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
    launches = _native.launch_count - before
    ms = e0.elapsed_time(e1) / args.steps
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        step()
        torch.cuda.synchronize()
    agg = collections.defaultdict(lambda: [0, 0.0])
    for e in prof.key_averages():
        if e.device_time_total > 0:
            agg[e.key][0] += e.count
            agg[e.key][1] += e.device_time_total
    tot = sum(v[1] for v in agg.values()) or 1.0
    print(f"per-kernel device time of one mixed step ({nd} decode rows at context {L}, "
          f"chunks {chunks}; torch profiler):", file=sys.stderr)
    for k, (c, t) in sorted(agg.items(), key=lambda kv: -kv[1][1])[:16]:
        print(f"  {t / 1000:8.3f} ms {100 * t / tot:5.1f}%  launches {c:5d}  {k[:100]}",
              file=sys.stderr)
    line = {
        "metric": f"Qwen3-8B chunked-prefill step ms ({nd} decode rows + 2 x 2048-token chunks)",
        "value": round(ms, 4), "unit": "ms", "n_gpus": 1, "steps": args.steps,
        "warmup": max(args.warmup, 3), "ms_per_step": round(ms, 4),
        "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (random-init N(0,0.02) weights, N(0,1) KV, random tables)",
        "config": {"workload": "mixed chunked step (forward_mixed, eager)", "decode_rows": nd,
                   "context": L, "chunks": chunks, "tokens": T,
                   "library_launches_per_step": launches // args.steps},
        "gpu_launches": launches,
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)


def run_gemm(args, rank, world, local_rank):
    """The four projections of one Qwen3-8B decoder layer at decode batch
    sizes, cuBLAS (+ the separate K3 / SiLU-mul launches) against this
    library's tcgen05 GEMMs with fused epilogues (vj_qkv_gemm_kv_store,
    vj_decode_gemm PLAIN / SWIGLU). Four weight sets are cycled so that every
    call streams its weights from HBM (4 x 50-200 MB > L2). Rows: --batch, or
    a sweep of 1..512. Each op is timed as replays of a CUDA graph of --steps
    calls (the engine's decode path), CUDA events on the launching stream;
    one JSON line for the largest row count, the per-op table on stderr."""
    import torch
    import torch.nn.functional as F
    from vllm_b200.kernels.fused import silu_mul
    from vllm_b200.kernels.gemm import decode_gemm, gemm_workspace_bytes, qkv_gemm_kv_store
    from vllm_b200.kernels.kv_store import kv_store_qknorm_rope, rope_table
    from vllm_b200.model.qwen3 import get_config
    if world > 1:
        raise SystemExit("--workload gemm runs on one GPU")
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    cfg = get_config("Qwen3-8B")
    H, I, D = cfg.hidden_size, cfg.intermediate_size, cfg.head_dim
    Hq, Hkv = cfg.num_attention_heads, cfg.num_key_value_heads
    NQKV = (Hq + 2 * Hkv) * D
    gen = torch.Generator(device=dev)
    gen.manual_seed(11)
    rnd = lambda *s, std=0.02: (torch.randn(s, generator=gen, device=dev) * std).to(torch.bfloat16)
    from vllm_b200.kernels.gemm import TiledWeight
    sets = [dict(qkv=rnd(NQKV, H), o=rnd(H, Hq * D), gu=rnd(2 * I, H), down=rnd(H, I))
            for _ in range(4)]
    for st in sets:   # the engine's decode path reads packed weight tiles
        st.update(qkv_t=TiledWeight(st["qkv"]), o_t=TiledWeight(st["o"]),
                  gu_t=TiledWeight(st["gu"], "swiglu"), down_t=TiledWeight(st["down"]))
    qn, kn = rnd(D, std=0.1) + 1, rnd(D, std=0.1) + 1
    nb, bs = 4096, 16
    cache = rnd(2, nb, bs, Hkv, D, std=1.0)
    table = rope_table(dev, cfg.rope_theta, 4096)
    rows_list = [args.batch] if args.batch else [1, 8, 16, 32, 64, 128, 256, 512]
    maxr = max(rows_list)
    ws = torch.zeros(max(gemm_workspace_bytes(r, n, k, m) for r in rows_list for n, k, m in
                         ((NQKV, H, "plain"), (H, Hq * D, "plain"), (2 * I, H, "swiglu"),
                          (H, I, "plain"))), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    reps = max(args.steps, 8)

    def timed(fn):
        """Device time of one call: `reps` calls captured in a CUDA graph (as
        the engine runs decode steps), replayed 3 times after a warm-up."""
        for i in range(max(args.warmup, 3)):
            fn(sets[i % 4])
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for i in range(reps):
                fn(sets[i % 4])
        graph.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(3):
            graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        del graph
        return e0.elapsed_time(e1) / (3 * reps) * 1e3   # us

    results = {}
    with ClockSampler(local_rank) as clk:
        for R in rows_list:
            x = rnd(R, H, std=1.0)
            xo = rnd(R, Hq * D, std=1.0)
            xi = rnd(R, I, std=1.0)
            slots = torch.randperm(nb * bs, generator=gen, device=dev)[:R].to(torch.int32)
            pos = torch.randint(0, 4000, (R,), generator=gen, device=dev).to(torch.int32)

            def cub_qkv(s):
                qkv = F.linear(x, s["qkv"])
                q, k, v = torch.split(qkv, [Hq * D, Hkv * D, Hkv * D], -1)
                kv_store_qknorm_rope(q.view(R, Hq, D), k.view(R, Hkv, D), v.view(R, Hkv, D),
                                     cache, slots, pos, qn, kn, table=table)

            def our_qkv(s):
                qkv_gemm_kv_store(x, s["qkv_t"], cache, slots, pos, qn, kn, Hq, table=table,
                                  ws=ws)

            ops = {
                "qkv+K3": (cub_qkv, our_qkv, NQKV * H * 2),
                "o_proj": (lambda s: F.linear(xo, s["o"]),
                           lambda s: decode_gemm(xo, s["o_t"], ws=ws), H * Hq * D * 2),
                "gate_up+SiLU": (lambda s: silu_mul(F.linear(x, s["gu"])),
                                 lambda s: decode_gemm(x, s["gu_t"], "swiglu", ws=ws),
                                 2 * I * H * 2),
                "down": (lambda s: F.linear(xi, s["down"]),
                         lambda s: decode_gemm(xi, s["down_t"], ws=ws), H * I * 2),
            }
            if args.gemm_op != "all":
                ops = {k: v for k, v in ops.items() if k.startswith(args.gemm_op)}
            for name, (cub, ours, wb) in ops.items():
                tc, to = timed(cub), timed(ours)
                results[(R, name)] = (tc, to, wb)
                print(f"rows {R:4d} {name:13s} cuBLAS {tc:8.2f} us ({wb / tc / 1e3:6.0f} GB/s)"
                      f"   vj {to:8.2f} us ({wb / to / 1e3:6.0f} GB/s)  x{tc / to:5.2f}",
                      file=sys.stderr)
    peaks, src = load_peaks()
    tot_c = sum(results[(maxr, n)][0] for n in ops)
    tot_o = sum(results[(maxr, n)][1] for n in ops)
    wbytes = sum(results[(maxr, n)][2] for n in ops)
    line = {
        "metric": f"Qwen3-8B decoder-layer projections us at {maxr} decode rows "
                  "(qkv+K3, o_proj, gate_up+SiLU, down)",
        "value": round(tot_o, 2), "unit": "us", "n_gpus": 1, "steps": reps,
        "warmup": max(args.warmup, 3), "ms_per_step": round(tot_o / 1e3, 5),
        "higher_is_better": False, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (random N(0,0.02) weights, N(0,1) activations)",
        "config": {"workload": "decode-step GEMMs with fused epilogues", "rows": maxr,
                   "cublas_plus_separate_kernels_us": round(tot_c, 2),
                   "per_op_us": {n: [round(results[(maxr, n)][0], 2),
                                     round(results[(maxr, n)][1], 2)] for n in ops},
                   "l2": "4 weight sets cycled (> L2)"},
        "roofline": {"bound": "hbm", "achieved": round(wbytes / tot_o / 1e3, 1),
                     "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(wbytes / tot_o / 1e3 / peaks["hbm_gbs"], 4),
                     "peak_source": f"{src} hbm_gbs", "kernel": "weights / time", "traffic": None},
        "gpu_launches": 4 * reps * len(rows_list),
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["e2e", "decode", "prefill", "kvstore", "c5", "c4step",
                                           "gemm", "mixedstep"],
                    default="e2e",
                    help="e2e (default): C4 Qwen3-8B output tok/s, tensor parallel over "
                         "--gpus; decode: C3 paged decode GB/s; prefill: C2 TFLOP/s; "
                         "kvstore: K3 GB/s; c5: Qwen3-32B chunked prefill tok/s; c4step: "
                         "one decode step; gemm: decode-step projections vs cuBLAS; "
                         "mixedstep: one chunked-prefill step")
    ap.add_argument("--model", default=None, help="e2e: model preset (default Qwen3-8B)")
    ap.add_argument("--max-num-seqs", type=int, default=None, help="e2e: scheduler seats")
    ap.add_argument("--tp", type=int, default=None,
                    help="e2e/c5: tensor-parallel degree (default all GPUs); the rest is "
                         "data parallel (engine replicas, requests split round-robin)")
    ap.add_argument("--cpu-budget", type=float, default=15.0)
    ap.add_argument("--ref-budget", type=float, default=60.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch", type=int, default=None,
                    help="profiling only: B sequences of the C3 / C2 batch (e2e: requests)")
    ap.add_argument("--pool-blocks", type=int, default=None,
                    help="profiling only: KV pool size in blocks (C3 / C2)")
    ap.add_argument("--context", type=int, default=840,
                    help="c4step: context length of every decode row")
    ap.add_argument("--fused-gemm", type=int, default=0,
                    help="e2e/c5/c4step: forwards of at most this many rows run their "
                         "projections on the fused tcgen05 GEMMs (0: cuBLAS)")
    ap.add_argument("--gemm-op", default="all", choices=["all", "qkv", "o_proj", "gate_up", "down"],
                    help="gemm: time one projection only (profiling)")
    ap.add_argument("--new-tokens", type=int, default=None,
                    help="profiling only (prefill): every sequence this many new tokens")
    ap.add_argument("--prefix-tokens", type=int, default=None,
                    help="profiling only (prefill): every sequence this cached prefix")
    args = ap.parse_args()
    if args.batch is not None:
        C3["batch"] = args.batch
        C2["num_seqs"] = args.batch
    if args.pool_blocks is not None:
        C3["pool_blocks"] = args.pool_blocks
        C2["pool_blocks"] = args.pool_blocks
    if args.new_tokens is not None:
        C2["new_fixed"] = args.new_tokens
    if args.prefix_tokens is not None:
        C2["prefix_fixed"] = args.prefix_tokens
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        if args.workload == "prefill":
            run_prefill(args, rank, world, local_rank)
        elif args.workload == "kvstore":
            run_kvstore(args, rank, world, local_rank)
        elif args.workload in ("e2e", "c5"):
            run_e2e(args, rank, world, local_rank)
        elif args.workload == "c4step":
            run_c4step(args, rank, world, local_rank)
        elif args.workload == "gemm":
            run_gemm(args, rank, world, local_rank)
        elif args.workload == "mixedstep":
            run_mixedstep(args, rank, world, local_rank)
        else:
            run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
