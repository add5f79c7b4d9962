#!/usr/bin/env python3
"""Benchmark of the NVFP4 paged KV-cache read path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W]
                    [--workload sparse|dense8k|dense128k|long|prefill|append|dedup]
                    [--impl ours|reference]

Default workload = configuration 3, the sparse (indexer) decode the metric is quoted on at
1/2/4/8 GPUs: batch 16 sequences of 128K tokens on shuffled pages of the 288-byte NVFP4 pool,
64 query heads, qk 576 / v 512, each sequence's top-2048 rows drawn without replacement
(synthetic, seeded).  One step = one fused gather + dequant + MLA decode call (Q preparation,
attention, split combine) over the batch for one layer; steps rotate over 32 layers' top-k
sets, whose rows (32 x 9.4 MB) exceed the 126 MB L2, so timed steps read the KV rows from HBM.
dense8k is configuration 2 (batch 16 x 8192 tokens, page tables from randperm).

value  = KV bytes read (288 B per attended token row per query group) per second, whole job
         (all ranks), device-timed with CUDA events over exactly K steps replayed from CUDA
         graphs.
e2e    = the same metric through the public API (glm53_nvfp4_runtime.mla_decode), with the
         per-step q / table / seq_lens host->device copies and the output device->host copy
         (pinned buffers) inside the timed region.  As an engine runs decode: one CUDA graph
         per step, captured once, holds step k+1's input copies, the mla_decode call of step
         k and step k-1's output copy as parallel branches (each replay re-runs the copies);
         the graphs replay in order on one stream, so decodes run one after another.  Beside it: e2e.eager_value (eager
         calls, copies on two copy streams with double buffers) and e2e.serial_value (one
         stream, eager).
gpu_reference = the reference's own read path on the same GPU (its Triton gather into 656 B
         rows, then a stock consumer of those rows), N = 1.
Multi-GPU (torchrun): each rank owns its own 16 sequences and their pages (weak scaling);
NCCL is used after the timed loop only: the max time, and one all-gather of the outputs that
rank 0 checks against its own decode of every other rank's layer.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "KV-read GB/s (% of 8 TB/s) + decode-attn tokens/s at 1/2/4/8 B200"
NV_BYTES = 288
L2_BYTES = 126 * 1024 * 1024

WORKLOADS = {
    "dense8k": dict(desc="config 2: dense NVFP4 MLA decode, batch 16 x 8192 tokens, 64 heads, "
                         "qk 576 / v 512, page 64, randperm page table",
                    B=16, H=64, QL=1, ctx=8192, topk=0),
    "dense128k": dict(desc="config 2 at 128K context: batch 16 x 131072 tokens, 64 heads",
                      B=16, H=64, QL=1, ctx=131072, topk=0),
    "sparse": dict(desc="config 3: sparse top-2048 decode, batch 16, 64 heads, 128K-token "
                        "sequences on shuffled pages, indices drawn without replacement",
                   B=16, H=64, QL=1, ctx=131072, topk=2048),
    # config 4 per layer: 5 x 460,000 + 3 x 900,000 tokens, MTP q_len 3, split over the ranks
    # by the token-balanced sequence partition (strong scaling: the job is fixed)
    # config 5's append half: 16 x 2048-token chunks per step into a ~2.7M-token pool at random
    # free pages, latent ~N(0,1) with 1 % of the values at 20x (outliers)
    "append": dict(desc="config 5 append: 16 seqs x 2048-token chunks per step quantised into a "
                        "2,713,846-token pool (42,404 pages of 64) at random free pages, 1 % outliers x20",
                   B=16, H=0, QL=0, ctx=2048, topk=0, pool_tokens=2713846),
    # config 5's prefill scratch: build_scratch's large-step branch (torch.unique in
    # the reference) on the device: one step's block tables deduplicated and gathered to 656 B rows
    "dedup": dict(desc="config 5 prefill step, build_scratch without a host sync: 2048 tokens x top-2048 "
                       "entries from a 300,000-token context of a 2,713,846-token pool (10 % -1 padding), "
                       "deduplicated on the device and gathered into 656 B rows",
                  B=2048, H=0, QL=0, ctx=300000, topk=2048, pool_tokens=2713846, dedup=True),
    # config 3's full sparse read path: the DSA indexer's top-2048 selection over NVFP4 indexer
    # keys (the indexer K-pool), then the fused sparse decode on the rows it picked
    "dsa": dict(desc="config 3 with its indexer: batch 16, 64 heads, 128K-token sequences on shuffled pages; "
                     "top-2048 rows chosen by the DSA indexer rule over NVFP4 indexer keys (64 heads x 128), "
                     "then the fused sparse decode",
                B=16, H=64, QL=1, ctx=131072, topk=2048, dsa=True),
    # config 5's attention half, as the reference's large-step read path runs it: every new token
    # attends the top-2048 rows its indexer picks from its causal window (the prior 300,000
    # tokens of its sequence and the chunk up to itself); one step = one layer for all 32,768
    "prefill": dict(desc="config 5 attention: 16 seqs x 2048-token chunks, each token attending its top-2048 "
                         "rows of a causal window over 300,000 prior tokens (stratified random picks through a "
                         "shuffled page table of a 2,713,846-token pool), 64 heads",
                    B=16, H=64, QL=1, ctx=2048, topk=2048, prior=300000, pool_tokens=2713846, prefill=True),
    "long": dict(desc="config 4 (one layer): 5 x 460,000 + 3 x 900,000-token sequences, 64 heads, "
                      "MTP q_len 3, token-balanced sequence / page-range partition over the ranks",
                 B=8, H=64, QL=3, ctx=0, topk=0, lens=[460000] * 5 + [900000] * 3),
}


def load_measured(key: str, fallback: float) -> float:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        return float(json.load(open(p)).get(key, fallback))
    return fallback


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def profile_traffic(workload: str):
    """DRAM bytes per launch of the workload's dominant kernel from profiles/traffic.json (one
    ncu capture each, with the command that made it), or None when none was captured."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if not os.path.exists(p):
        return None
    ent = json.load(open(p)).get("workloads", {}).get(workload)
    return float(ent["bytes_per_launch"]) if ent else None


def cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


class ClockSampler:
    """Samples SM clock and clock-event reasons through NVML while the GPU is busy."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
        0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
        0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
    }

    def __init__(self, index: int):
        self.samples = []
        self.ok = False
        self._stop = threading.Event()
        try:
            import pynvml

            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:  # noqa: BLE001 - NVML missing: report clocks as unavailable
            self.max_mhz = None

    def _run(self):
        while not self._stop.is_set():
            try:
                mhz = self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM)
                rs = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                self.samples.append((time.perf_counter(), mhz, rs))
            except Exception:  # noqa: BLE001
                pass
            time.sleep(0.005)

    def start(self):
        if self.ok:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()

    def stop(self):
        if self.ok:
            self._stop.set()
            self.t.join()

    def summary(self, t0=None, t1=None):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["nvml unavailable"]}
        inside = [s for s in self.samples if t0 is not None and t0 <= s[0] <= t1]
        use = inside if len(inside) >= 3 else self.samples
        busy = [s for s in use if not (s[2] & 0x1)] or use
        reasons = set()
        for _, _, rs in busy:
            for bit, name in self.REASONS.items():
                if rs & bit and bit != 0x1:
                    reasons.add(name)
        return {"sm_mhz": statistics.median(s[1] for s in busy), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(reasons), "samples": len(busy),
                "window": "timed" if use is inside else "soak+timed"}


# ---------------------------------------------------------------------------- setup
def make_layers(rt, torch, wl, layers, dev, seed):
    """Per layer: a pool written by the append kernel, page tables / top-k rows, q."""
    B, H, QL, ctx, topk = wl["B"], wl["H"], wl["QL"], wl["ctx"], wl["topk"]
    pages = B * ctx // 64
    g = torch.Generator(device="cpu").manual_seed(seed)
    out = []
    shared_pool = None
    for layer in range(layers):
        if topk == 0 or shared_pool is None:
            pool = torch.empty(pages, 64, NV_BYTES, dtype=torch.uint8, device=dev)
            torch.manual_seed(seed * 1000 + layer)
            for c in range(0, pages * 64, 1 << 20):
                n = min(1 << 20, pages * 64 - c)
                x = torch.randn(n, 512, device=dev).to(torch.bfloat16)
                rt.write_nvfp4(x, pool, torch.arange(c, c + n, device=dev))
            if topk:
                shared_pool = pool
        else:
            pool = shared_pool                      # sparse layers: one pool, fresh top-k sets
        page_table = torch.randperm(pages, generator=g).view(B, ctx // 64)
        if topk:
            logical = torch.stack([torch.randperm(ctx, generator=g)[:topk] for _ in range(B)])
            tables = (page_table.gather(1, logical // 64) * 64 + logical % 64).to(torch.int32)
            tables = tables.view(B, 1, topk)
            seq = torch.full((B,), topk, dtype=torch.int32)
        else:
            tables = page_table.to(torch.int32)
            seq = torch.full((B,), ctx, dtype=torch.int32)
        q = torch.randn(B, QL, H, 576, generator=g).to(torch.bfloat16)
        out.append(dict(pool=pool, tables=tables.to(dev), seq=seq.to(dev), q=q.to(dev),
                        out=torch.empty(B, QL, H, 512, dtype=torch.bfloat16, device=dev),
                        tables_h=tables.pin_memory(), seq_h=seq.pin_memory(), q_h=q.pin_memory()))
    return out


APPEND_BYTES_PER_TOKEN = 1024 + 288 + 8   # bf16 latent read, 288 B row written, int64 slot read


DEDUP_ENTRY_BYTES = 4 + 4          # entry read, table written
DEDUP_ROW_BYTES = NV_BYTES + 656    # distinct row read, 656 B row written


INDEX_ROW_BYTES = 72


def kv_bytes_per_step(wl) -> int:
    if wl.get("dsa"):   # every visible indexer key once, then the selected latent rows
        return wl["B"] * wl["ctx"] * INDEX_ROW_BYTES + wl["B"] * wl["topk"] * NV_BYTES
    if wl.get("prefill"):
        return wl["B"] * wl["ctx"] * wl["topk"] * NV_BYTES
    if wl.get("dedup"):
        raise ValueError("the dedup workload's bytes depend on its distinct entries (dedup_bytes)")
    if "pool_tokens" in wl:
        return wl["B"] * wl["ctx"] * APPEND_BYTES_PER_TOKEN
    if "lens" in wl:
        return sum(wl["lens"]) * NV_BYTES
    rows = wl["B"] * (wl["topk"] if wl["topk"] else wl["ctx"])
    return rows * NV_BYTES


# pieces per rank of the long workload: one call's split plan is uniform over its units, so
# the rank's tokens are cut into this many equal ranges.  Each call decodes one CTA per
# (piece, query group); 48 pieces x 3 groups keep every call at <= 144 CTAs on 1-8 ranks
# (partition.plan adds a unit where a cut crosses a sequence end), one wave on 148 SMs
LONG_PIECES_PER_RANK = 48


def long_rank_pool(rt, torch, wl, dev, rank, world, seed):
    """Rank ``rank``'s share of the config-4 job: (plan, its units, its pool [pages, 64, 288]
    written by the append kernel, each unit's page list in token order).  Deterministic in
    (seed, rank, world), so any rank can rebuild any other rank's pool."""
    from glm53_flash_dual_dgx_spark_b200 import partition as P

    plan = P.plan(wl["lens"], world * LONG_PIECES_PER_RANK, 64, q_len=wl["QL"])
    units = [u for part in plan[rank * LONG_PIECES_PER_RANK:(rank + 1) * LONG_PIECES_PER_RANK] for u in part]
    pages = [(u.tokens + 63) // 64 for u in units]
    pool = torch.empty(sum(pages), 64, NV_BYTES, dtype=torch.uint8, device=dev)
    gd = torch.Generator(device=dev).manual_seed(seed * 1000 + rank)
    for c in range(0, pool.shape[0] * 64, 1 << 20):
        n = min(1 << 20, pool.shape[0] * 64 - c)
        x = torch.randn(n, 512, device=dev, generator=gd).to(torch.bfloat16)
        rt.write_nvfp4(x, pool, torch.arange(c, c + n, device=dev))
    g = torch.Generator().manual_seed(seed * 1000 + rank)
    perm = torch.randperm(pool.shape[0], generator=g).to(torch.int32)
    tables, k = [], 0
    for m in pages:
        tables.append(perm[k:k + m])
        k += m
    return plan, units, pool, tables


def long_query(torch, wl, seed):
    """The batch's q [B, QL, H, 576] bf16, identical on every rank (the pieces of one sequence
    on different ranks attend the same query)."""
    g = torch.Generator().manual_seed(seed + 7)
    return torch.randn(len(wl["lens"]), wl["QL"], wl["H"], 576, generator=g).to(torch.bfloat16)


def long_check(rt, torch, wl, dev, world, merged, seed, sm):
    """Rank 0, after timing: rebuild every rank's pool, lay each sequence's pages end to end in
    one pool, decode the whole batch unpartitioned in one call and compare it with the
    partitioned result merged across the ranks (``merged``, [B, QL, H, 512]).  The pieces and
    the whole sequences accumulate in different orders, so the gate is the attention tolerance
    (2e-2 rel / 1e-2 abs elementwise), with the largest difference and the relative L2 reported."""
    pools, seq_pages, base = [], [[] for _ in wl["lens"]], 0
    for r in range(world):
        _, units, pool, tables = long_rank_pool(rt, torch, wl, dev, r, world, seed)
        for u, t in zip(units, tables):
            seq_pages[u.seq].append((u.start, t.to(torch.int64) + base))
        pools.append(pool)
        base += pool.shape[0]
    full = torch.cat(pools)
    del pools
    width = max(sum(t.numel() for _, t in sp) for sp in seq_pages)
    tb = torch.full((len(wl["lens"]), width), -1, dtype=torch.int32)
    for s, sp in enumerate(seq_pages):
        t = torch.cat([t for _, t in sorted(sp, key=lambda x: x[0])])
        tb[s, :t.numel()] = t.to(torch.int32)
    sl = torch.tensor(wl["lens"], dtype=torch.int32, device=dev)
    q = long_query(torch, wl, seed).to(dev)
    ref = rt.mla_decode(q, full, None, 128, 512, 64, tb.to(dev), sl, max(wl["lens"]), bmm1_scale=sm)
    torch.cuda.synchronize()
    got, want = merged.float(), ref.float()
    diff = (got - want).abs()
    within = bool((diff <= 1e-2 + 2e-2 * want.abs()).all())
    rel = float(torch.linalg.vector_norm(got - want) / torch.linalg.vector_norm(want))
    del full
    torch.cuda.empty_cache()
    return {"merged_vs_unpartitioned": {"max_abs_diff": round(float(diff.max()), 6), "rel_l2": round(rel, 7),
                                        "within_tol": within, "ranks": world}, "passed": within and rel < 1e-2}


def make_long_step(rt, torch, wl, dev, rank, world, seed):
    """The partitioned long-context step on this rank: its pieces' pages written by the append
    kernel into a rank-local pool, two decode calls (pieces before a sequence's causal tail
    with q_len folded into the heads; tails with the causal limit) and the exact log-sum-exp
    merge of the pieces into per-sequence partial results.  Returns (step_fn, state)."""
    from glm53_flash_dual_dgx_spark_b200 import partition as P

    lens, QL, H = wl["lens"], wl["QL"], wl["H"]
    plan, units, pool, tables = long_rank_pool(rt, torch, wl, dev, rank, world, seed)
    q = long_query(torch, wl, seed).to(dev)
    calls = []
    for last in (False, True):
        idx = [i for i, u in enumerate(units) if u.last == last]
        if not idx:
            continue
        width = max(tables[i].numel() for i in idx)
        tb = torch.full((len(idx), width), -1, dtype=torch.int32)
        for row, i in enumerate(idx):
            tb[row, :tables[i].numel()] = tables[i]
        sl = torch.tensor([units[i].tokens for i in idx], dtype=torch.int32)
        seqs = torch.tensor([units[i].seq for i in idx], dtype=torch.long, device=dev)
        n = len(idx)
        fold = not last and QL > 1
        calls.append(dict(idx=torch.tensor(idx, dtype=torch.long, device=dev), seqs=seqs, tables=tb.to(dev),
                          seq=sl.to(dev), max_len=int(sl.max()), fold=fold, n=n,
                          qbuf=torch.empty(n, QL, H, 576, dtype=torch.bfloat16, device=dev),
                          out=torch.empty(n, QL, H, 512, dtype=torch.bfloat16, device=dev)))
    U = len(units)
    out_u = torch.empty(U, QL, H, 512, dtype=torch.bfloat16, device=dev)
    lse_u = torch.empty(U, QL, H, dtype=torch.float32, device=dev)
    seq_of = torch.tensor([u.seq for u in units], dtype=torch.long, device=dev)
    sm = 1.0 / math.sqrt(576)
    state = dict(units=units, plan=plan, pool=pool, q=q, out=None, lse=None, out_u=out_u, lse_u=lse_u,
                 calls=calls)

    def step():
        for c in calls:
            torch.index_select(q, 0, c["seqs"], out=c["qbuf"])
            qq = c["qbuf"].view(c["n"], 1, QL * H, 576) if c["fold"] else c["qbuf"]
            oo = c["out"].view(c["n"], 1, QL * H, 512) if c["fold"] else c["out"]
            o, l = rt.mla_decode_lse(qq, pool, None, 128, 512, 64, c["tables"], c["seq"], c["max_len"],
                                     out=oo, bmm1_scale=sm, bmm2_scale=1.0)
            out_u[c["idx"]] = c["out"]
            lse_u[c["idx"]] = l.view(c["n"], QL, H)
        state["out"], state["lse"] = P.merge(out_u, lse_u, seq_of, len(lens))

    return step, state, sum(u.tokens for u in units) * NV_BYTES


def cpu_append_sample(seconds: float):
    """The oracle's append (C restatement of the reference's _quant_kernel) on 4096 tokens,
    repeated for ~`seconds`; returns (GB/s of algorithmic bytes, seconds per run, tokens)."""
    import numpy as np
    import torch

    from oracle import oracle as O

    T = 4096
    x = torch.randn(T, 512, generator=torch.Generator().manual_seed(0)).to(torch.bfloat16)
    pool = np.zeros((T, NV_BYTES), np.uint8)
    slots = np.arange(T, dtype=np.int64)
    runs, t0 = 0, time.perf_counter()
    while True:
        O.quant(x, slots, pool)
        runs += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    return runs * T * APPEND_BYTES_PER_TOKEN / el / 1e9, el / runs, T


def dedup_tables(wl, seed):
    """block_tables [T, 1, K] int32 of the dedup workload: entries uniform over a context window
    of the pool, 10 % -1 padding."""
    import torch

    g = torch.Generator().manual_seed(seed)
    rows = wl["pool_tokens"] // 64 * 64
    base = int(torch.randint(0, rows - wl["ctx"], (1,), generator=g))
    bt = base + torch.randint(0, wl["ctx"], (wl["B"], 1, wl["topk"]), generator=g)
    bt[torch.rand(bt.shape, generator=g) < 0.1] = -1
    return bt.to(torch.int32)


_CPU_SAMPLE: dict = {}


def dedup_bytes(n_entries: int, n_unique: int) -> int:
    return n_entries * DEDUP_ENTRY_BYTES + n_unique * DEDUP_ROW_BYTES


def cpu_dedup_sample(wl, seconds: float):
    """The oracle's large-step build_scratch (numpy unique + the C restatement of _gather_kernel)
    on 64 of the workload's 2048 tokens, repeated for ~`seconds`; returns (GB/s, s per run, desc)."""
    import numpy as np

    from oracle import oracle as O

    if "dedup" not in _CPU_SAMPLE:                   # inputs built once per process
        bt = dedup_tables(wl, 0)[:64].numpy()
        pool = np.zeros((wl["pool_tokens"] // 64 * 64, NV_BYTES), np.uint8)
        pool[:, 256:] = 0x38
        _CPU_SAMPLE["dedup"] = (bt, pool, len(np.unique(bt)))
    bt, pool, n_unique = _CPU_SAMPLE["dedup"]
    runs, t0 = 0, time.perf_counter()
    while True:
        O.build_scratch(pool, bt, sync_free_t=0)
        runs += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    per = el / runs
    return dedup_bytes(bt.size, n_unique) / per / 1e9, per, f"64 tokens x {wl['topk']} entries, {n_unique} distinct"


def run_dedup(args, wl, rt, torch, dist, dev, rank, world, local):
    """--workload dedup: build_scratch_sync_free on a config-5 prefill step (weak scaling)."""
    rows = wl["pool_tokens"] // 64 * 64
    pool = torch.zeros(rows // 64, 64, NV_BYTES, dtype=torch.uint8, device=dev)
    pool[..., 256:] = 0x38                           # scale 1.0 in every block
    tabs = [dedup_tables(wl, 1 + rank * 7 + k) for k in range(2)]
    tabs_d = [t.to(dev) for t in tabs]
    n_entries = tabs[0].numel()
    cap = wl["ctx"] + 1                              # distinct entries: the context window and -1
    outs = []
    for t in tabs_d:                                 # eager warm-up (allocates the workspace)
        outs.append(rt.build_scratch_sync_free(pool, t, capacity_rows=cap))
    torch.cuda.synchronize()
    n_unique = [int(o[2].item()) for o in outs]
    step_bytes = sum(dedup_bytes(n_entries, u) for u in n_unique) / len(n_unique)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    graphs = []
    with torch.cuda.stream(s):
        for t in tabs_d:
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=s):
                rt.build_scratch_sync_free(pool, t, capacity_rows=cap)
            graphs.append(gr)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    sampler.start()
    soak_end = time.perf_counter() + 1.0
    k = 0
    while time.perf_counter() < soak_end or k < args.warmup:
        graphs[k % 2].replay()
        k += 1
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for k in range(args.steps):
        graphs[k % 2].replay()
    ev1.record()
    ev1.synchronize()
    t1 = time.perf_counter()
    if world > 1:
        dist.barrier()
    sampler.stop()
    t_max = torch.tensor([ev0.elapsed_time(ev1)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t_max, op=dist.ReduceOp.MAX)
    per_ms = float(t_max.item()) / args.steps
    value = step_bytes * world / (per_ms / 1e3) / 1e9

    # end to end through the public API: the block tables host->device, the inverse tables
    # device->host, serial on one stream
    e_steps = max(10, min(args.e2e_steps, 50))
    bt_h = [t.pin_memory() for t in tabs]
    tb_h = torch.empty(n_entries, dtype=torch.int32).pin_memory()
    btd = torch.empty_like(tabs_d[0])
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for k in range(e_steps):
        btd.copy_(bt_h[k % 2], non_blocking=True)
        _, tables, _ = rt.build_scratch_sync_free(pool, btd, capacity_rows=cap)
        tb_h.copy_(tables.view(-1), non_blocking=True)
    e1.record()
    e1.synchronize()
    e_ms = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(e_ms, op=dist.ReduceOp.MAX)
    e2e_value = step_bytes * world * e_steps / (float(e_ms.item()) / 1e3) / 1e9
    errors = rt.device_errors(dev)
    if rank == 0:
        peak, peak_kind = load_peaks()
        achieved = step_bytes / (per_ms / 1e3) / 1e9
        line = {
            "metric": "sync-free dedup + 656 B gather GB/s (8 B per table entry, 944 B per distinct row)",
            "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(per_ms, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "u8",
            "data": "synthetic (seeded uniform top-k entries over a context window, 10 % -1)",
            "config": {"workload": wl["desc"], "entries_per_step": n_entries,
                       "distinct_per_step": n_unique, "pool_rows": rows,
                       "l2": f"inputs larger than L2: {step_bytes / 2**20:.0f} MiB moved per step",
                       "parallelism": f"a pool per rank x{world} (weak scaling)"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                         "traffic": profile_traffic("dedup"),
                         "per_launch_bytes": int(step_bytes), "kernel_ms": round(per_ms, 5),
                         "kernel": "dedup_* (mark, block sums, scan, positions, tables, gather): the whole call",
                         "step_frac_in_kernel": 1.0},
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": n_entries * 4,
                    "d2h_bytes_per_step": n_entries * 4, "steps": e_steps},
            "gpu_launches": args.steps * 6,
            "clocks": sampler.summary(t0, t1),
            "device_errors": errors,
        }
        if world == 1:
            line["gpu_reference"] = gpu_reference_dedup(torch, pool, tabs_d, per_ms * 1e3)
            gbs, per, desc = cpu_dedup_sample(wl, args.cpu_seconds)
            line["cpu_baseline"] = {
                "value": round(gbs, 4), "unit": "GB/s", "cores": 1, "kind": "port",
                "sample": f"oracle build_scratch large-step branch (numpy unique + C gather) on {desc}, "
                          f"repeated for ~{args.cpu_seconds:.0f} s ({per * 1e3:.1f} ms each; {cpu_model()})"}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_append(args, wl, rt, torch, dist, dev, rank, world, local):
    """--workload append: quantise-on-append of prefill chunks (weak scaling: a pool per rank)."""
    T = wl["B"] * wl["ctx"]
    pages = (wl["pool_tokens"] + 63) // 64
    pool = torch.zeros(pages, 64, NV_BYTES, dtype=torch.uint8, device=dev)
    g = torch.Generator().manual_seed(1 + rank)
    step_bytes = T * APPEND_BYTES_PER_TOKEN
    n_in = max(2, math.ceil(2 * L2_BYTES / step_bytes))          # inputs read per rotation > 2 x L2
    inputs = []
    for k in range(n_in):
        x = torch.randn(T, 512, generator=g)
        out_mask = torch.rand(T, 512, generator=g) < 0.01
        x = torch.where(out_mask, x * 20.0, x).to(torch.bfloat16)
        # each sequence's 32 new pages go to random free pages of the pool
        free = torch.randperm(pages, generator=g)[:T // 64]
        slots = (free.view(-1, 1) * 64 + torch.arange(64).view(1, -1)).reshape(-1).to(torch.int64)
        inputs.append(dict(x=x.to(dev), slots=slots.to(dev), x_h=x.pin_memory(), slots_h=slots.pin_memory()))
    for inp in inputs:
        rt.write_nvfp4(inp["x"], pool, inp["slots"])
    torch.cuda.synchronize()
    # one graph holds a whole rotation (n_in appends back to back): a single append is a few
    # microseconds, shorter than the host's graph-launch interval
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    rot = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(rot, stream=s):
            for inp in inputs:
                rt.write_nvfp4(inp["x"], pool, inp["slots"])
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    args.steps = math.ceil(args.steps / n_in) * n_in
    sampler = ClockSampler(local)
    sampler.start()
    soak_end = time.perf_counter() + 1.0
    k = 0
    while time.perf_counter() < soak_end or k * n_in < args.warmup:
        rot.replay()
        k += 1
        if k % 64 == 0:
            torch.cuda.synchronize()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for k in range(args.steps // n_in):
        rot.replay()
    ev1.record()
    ev1.synchronize()
    t1 = time.perf_counter()
    if world > 1:
        dist.barrier()
    sampler.stop()
    t_max = torch.tensor([ev0.elapsed_time(ev1)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t_max, op=dist.ReduceOp.MAX)
    ms_max = float(t_max.item())
    per_ms = ms_max / args.steps
    value = step_bytes * world / (per_ms / 1e3) / 1e9

    # end to end through the public API: the chunk and its slots host->device, the written
    # rows device->host.  Pipelined like the decode's (the next chunk's copy-in and the previous
    # chunk's read-back overlap this chunk's append on two copy streams, double buffers); the
    # one-stream serial figure is reported beside it.
    e_steps = max(10, min(args.e2e_steps, 100))
    flat = pool.view(-1, NV_BYTES)

    def append_e2e(pipelined: bool) -> float:
        nb = 2 if pipelined else 1
        xs = [torch.empty_like(inputs[0]["x"]) for _ in range(nb)]
        ss = [torch.empty_like(inputs[0]["slots"]) for _ in range(nb)]
        rows_d = [torch.empty(T, NV_BYTES, dtype=torch.uint8, device=dev) for _ in range(nb)]
        rows_h = [torch.empty(T, NV_BYTES, dtype=torch.uint8).pin_memory() for _ in range(nb)]
        main = torch.cuda.current_stream()
        cin = torch.cuda.Stream() if pipelined else main
        cout = torch.cuda.Stream() if pipelined else main
        in_ready = [torch.cuda.Event() for _ in range(e_steps)]
        done = [torch.cuda.Event() for _ in range(e_steps)]
        out_done = [torch.cuda.Event() for _ in range(e_steps)]

        def copy_in(k):
            with torch.cuda.stream(cin):
                if k >= nb:
                    cin.wait_event(done[k - nb])
                xs[k % nb].copy_(inputs[k % n_in]["x_h"], non_blocking=True)
                ss[k % nb].copy_(inputs[k % n_in]["slots_h"], non_blocking=True)
                in_ready[k].record(cin)

        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(cin)
        copy_in(0)
        for k in range(e_steps):
            if pipelined and k + 1 < e_steps:
                copy_in(k + 1)
            elif not pipelined and k > 0:
                copy_in(k)
            b = k % nb
            main.wait_event(in_ready[k])
            if k >= nb:
                main.wait_event(out_done[k - nb])
            rt.write_nvfp4(xs[b], pool, ss[b])
            torch.index_select(flat, 0, ss[b], out=rows_d[b])
            done[k].record(main)
            with torch.cuda.stream(cout):
                cout.wait_event(done[k])
                rows_h[b].copy_(rows_d[b], non_blocking=True)
                out_done[k].record(cout)
        e1.record(cout)
        e1.synchronize()
        torch.cuda.synchronize()
        e_ms = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(e_ms, op=dist.ReduceOp.MAX)
        return step_bytes * world * e_steps / (float(e_ms.item()) / 1e3) / 1e9

    e2e_serial = append_e2e(False)
    e2e_value = append_e2e(True)
    errors = rt.device_errors(dev)
    if rank == 0:
        peak, peak_kind = load_peaks()
        achieved = step_bytes / (per_ms / 1e3) / 1e9
        line = {
            "metric": "NVFP4 append GB/s (1320 B per token: bf16 latent read, 288 B row and slot)",
            "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(per_ms, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16->e2m1/e4m3",
            "data": "synthetic (seeded N(0,1) latent, 1 % of values x20)",
            "config": {"workload": wl["desc"], "tokens_per_step": T, "pool_pages": pages,
                       "inputs_rotated": n_in, "steps_per_graph": n_in,
                       "l2": f"inputs larger than L2: {n_in} chunks x {step_bytes / 2**20:.1f} MiB per rotation",
                       "parallelism": f"one pool per rank x{world} (weak scaling)"},
            "tokens_per_s": round(T * world / (per_ms / 1e3), 1),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                         "traffic": profile_traffic("append"),
                         "per_launch_bytes": step_bytes, "kernel_ms": round(per_ms, 5),
                         "kernel": "append_kernel", "step_frac_in_kernel": 1.0},
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s",
                    "h2d_bytes_per_step": T * 1024 + T * 8, "d2h_bytes_per_step": T * NV_BYTES,
                    "steps": e_steps,
                    "pipeline": "copies of step k+1 / k-1 overlap the append of step k (3 streams)",
                    "serial_value": round(e2e_serial, 2)},
            "gpu_launches": args.steps,
            "clocks": sampler.summary(t0, t1),
            "device_errors": errors,
        }
        if world == 1:
            line["gpu_reference"] = gpu_reference_append(torch, inputs, pages * 64, dev, per_ms * 1e3)
            gbs, per, n = cpu_append_sample(args.cpu_seconds)
            line["cpu_baseline"] = {
                "value": round(gbs, 4), "unit": "GB/s", "cores": 1, "kind": "port",
                "sample": f"oracle append (C restatement of _quant_kernel, one thread) of {n} tokens "
                          f"repeated for ~{args.cpu_seconds:.0f} s ({per * 1e3:.1f} ms each; {cpu_model()})"}
        print(json.dumps(line), flush=True)
    del rot
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


PREFILL_FLOPS_PER_ROW = 64 * 2 * (512 + 512)   # per query token and attended row: QK^T and PV, 64 heads


def make_prefill(rt, torch, wl, dev, seed):
    """Config 5's attention step: a 2.7M-token pool written by the append kernel (N(0,1) latent,
    1 % of values x20), and for each of the 16 x 2048 new tokens its top-2048 pool rows: one pick
    per 1/2048 stratum of its causal window (positions below 300,000 + its index + 1), mapped
    through its sequence's shuffled page table, so the picks are distinct and spread over the
    window as an indexer's are.  Returns the layer dict decode calls take."""
    B, T, K, H, prior = wl["B"], wl["ctx"], wl["topk"], wl["H"], wl["prior"]
    pages_total = wl["pool_tokens"] // 64
    pool = torch.empty(pages_total, 64, NV_BYTES, dtype=torch.uint8, device=dev)
    torch.manual_seed(seed)
    for c in range(0, pages_total * 64, 1 << 20):
        n = min(1 << 20, pages_total * 64 - c)
        x = torch.randn(n, 512, device=dev)
        x = torch.where(torch.rand(n, 512, device=dev) < 0.01, x * 20.0, x)
        rt.write_nvfp4(x.to(torch.bfloat16), pool, torch.arange(c, c + n, device=dev))
    g = torch.Generator(device=dev).manual_seed(seed)
    npages = (prior + T + 63) // 64
    tables = torch.empty(B * T, 1, K, dtype=torch.int32, device=dev)
    ar = torch.arange(K, device=dev, dtype=torch.float64)
    for s_ in range(B):
        pt = torch.randperm(pages_total, generator=g, device=dev)[:npages]
        vis = (prior + 1 + torch.arange(T, device=dev)).to(torch.float64)
        u = torch.rand(T, K, generator=g, device=dev, dtype=torch.float64)
        pos = torch.minimum(((ar + u) * vis[:, None] / K).long(), vis[:, None].long() - 1)
        tables[s_ * T:(s_ + 1) * T, 0] = (pt[pos // 64] * 64 + pos % 64).to(torch.int32)
    q = torch.randn(B * T, 1, H, 576, generator=g, device=dev).to(torch.bfloat16)
    return dict(pool=pool, tables=tables, q=q, seq=torch.full((B * T,), K, dtype=torch.int32, device=dev),
                out=torch.empty(B * T, 1, H, 512, dtype=torch.bfloat16, device=dev))


def prefill_check(torch, rt, ly, tokens, sm):
    """Decode outputs of the given query tokens against the exact dequantised attention (fp32)."""
    worst, ok = 0.0, True
    for j in tokens:
        kv = rt.dequant(ly["pool"], ly["tables"][j, 0]).float()
        qf = ly["q"][j, 0, :, :512].float()
        tru = torch.softmax(qf @ kv.t() * sm, dim=-1) @ kv
        o = ly["out"][j, 0].float()
        worst = max(worst, float((o - tru).norm() / tru.norm()))
        ok = ok and bool(((o - tru).abs() <= 1e-2 + 2e-2 * tru.abs()).all())
    return {"fp32_rel_l2_max": round(worst, 5), "fp32_within_tol": ok, "tokens_checked": len(tokens), "passed": ok}


def run_prefill(args, wl, rt, torch, dist, dev, rank, world, local):
    """--workload prefill: config 5's attention step, the fused sparse kernel with one query
    group per new token (weak scaling: a pool and 16 sequences per rank)."""
    ly = make_prefill(rt, torch, wl, dev, seed=1 + rank)
    n_q = ly["q"].shape[0]
    K = wl["topk"]
    sm = 1.0 / math.sqrt(576)
    kvb = kv_bytes_per_step(wl)
    flops = n_q * K * PREFILL_FLOPS_PER_ROW

    def call(out=None, q=None, tables=None):
        return rt.mla_decode(ly["q"] if q is None else q, ly["pool"], None, 128, 512, 64,
                             ly["tables"] if tables is None else tables, ly["seq"], K, sparse_mla_top_k=K,
                             out=ly["out"] if out is None else out, bmm1_scale=sm, bmm2_scale=1.0)

    call()
    torch.cuda.synchronize()
    s_ = torch.cuda.Stream()
    s_.wait_stream(torch.cuda.current_stream())
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s_):
        with torch.cuda.graph(gr, stream=s_):
            call()
    torch.cuda.current_stream().wait_stream(s_)
    torch.cuda.synchronize()
    steps = args.steps if args.steps_given else 20
    sampler = ClockSampler(local)
    sampler.start()
    soak_end = time.perf_counter() + 1.0
    k = 0
    while time.perf_counter() < soak_end or k < args.warmup:
        gr.replay()
        k += 1
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(steps):
        gr.replay()
    ev1.record()
    ev1.synchronize()
    t1 = time.perf_counter()
    if world > 1:
        dist.barrier()
    sampler.stop()
    t_max = torch.tensor([ev0.elapsed_time(ev1)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t_max, op=dist.ReduceOp.MAX)
    per_ms = float(t_max.item()) / steps
    value = kvb * world / (per_ms / 1e3) / 1e9

    # the attention kernel alone (events the library records around it)
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(3)]
    for a, b in kev:
        rt.set_kernel_events(a, b)
        call()
    torch.cuda.synchronize()
    kernel_ms = sum(a.elapsed_time(b) for a, b in kev) / len(kev)

    # end to end through the public API: q and the top-k tables host->device, the output back,
    # serial on one stream (each step's copies are several times its decode)
    q_h = ly["q"].cpu().pin_memory()
    t_h = ly["tables"].cpu().pin_memory()
    o_h = torch.empty(ly["out"].shape, dtype=torch.bfloat16).pin_memory()
    qd, td = torch.empty_like(ly["q"]), torch.empty_like(ly["tables"])
    e_steps = 3
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(e_steps):
        qd.copy_(q_h, non_blocking=True)
        td.copy_(t_h, non_blocking=True)
        call(q=qd, tables=td)
        o_h.copy_(ly["out"], non_blocking=True)
    e1.record()
    e1.synchronize()
    e_ms = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(e_ms, op=dist.ReduceOp.MAX)
    e2e_value = kvb * world * e_steps / (float(e_ms.item()) / 1e3) / 1e9
    check = prefill_check(torch, rt, ly, [0, wl["ctx"] - 1, n_q - 1], sm)
    errors = rt.device_errors(dev)
    if rank == 0:
        peak = load_measured("bf16_tflops_sustained", 1400.0)
        achieved = flops / (kernel_ms / 1e3) / 1e12
        line = {
            "metric": METRIC + " (prefill attention step)", "value": round(value, 2), "unit": "GB/s",
            "n_gpus": world, "steps": steps, "warmup": args.warmup, "ms_per_step": round(per_ms, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic (seeded N(0,1) latent with 1 % x20 quantised by the append kernel; N(0,1) q)",
            "config": {"workload": wl["desc"], "query_tokens": n_q, "topk": K, "heads": wl["H"],
                       "pool_rows": wl["pool_tokens"] // 64 * 64,
                       "l2": f"inputs larger than L2: {kvb / 2**30:.1f} GiB of row reads per step from a "
                             f"{wl['pool_tokens'] * NV_BYTES / 2**20:.0f} MiB pool",
                       "parallelism": f"a pool and 16 sequences per rank x{world} (weak scaling)"},
            "query_tokens_per_s": round(n_q * world / (per_ms / 1e3), 1),
            "roofline": {"bound": "tensor", "achieved": round(achieved, 2), "peak": peak, "unit": "TFLOP/s",
                         "frac": round(achieved / peak, 4), "peak_kind": "measured bf16 sustained",
                         "flops_per_launch": flops, "kernel_ms": round(kernel_ms, 4),
                         "kernel": "decode_fp4_kernel<sparse>", "traffic": profile_traffic("prefill"),
                         "step_frac_in_kernel": round(kernel_ms / per_ms, 3)},
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s",
                    "h2d_bytes_per_step": q_h.numel() * 2 + t_h.numel() * 4, "d2h_bytes_per_step": o_h.numel() * 2,
                    "steps": e_steps},
            "gpu_launches": steps * 2,
            "clocks": sampler.summary(t0, t1),
            "result_check": check,
            "device_errors": errors,
        }
        print(json.dumps(line), flush=True)
    del gr
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if not check["passed"]:
        sys.exit("result check failed: a prefill output is outside 2e-2 rel / 1e-2 abs")


def run_dsa(args, wl, rt, torch, dist, dev, rank, world, local):
    """--workload dsa: the indexer's top-k over NVFP4 indexer keys, then the sparse decode, per
    layer (weak scaling: 16 sequences and their pools per rank)."""
    B, H, ctx, K = wl["B"], wl["H"], wl["ctx"], wl["topk"]
    pages = B * ctx // 64
    sm = 1.0 / math.sqrt(576)
    layers = []
    g = torch.Generator().manual_seed(1 + rank)
    for li in range(2):                                 # 2 x (604 + 151) MB: well past the L2
        pool = torch.empty(pages, 64, NV_BYTES, dtype=torch.uint8, device=dev)
        index = torch.empty(pages, 64, INDEX_ROW_BYTES, dtype=torch.uint8, device=dev)
        torch.manual_seed(1000 * (1 + rank) + li)
        for c in range(0, pages * 64, 1 << 20):
            n = min(1 << 20, pages * 64 - c)
            slots = torch.arange(c, c + n, device=dev)
            rt.write_nvfp4(torch.randn(n, 512, device=dev).to(torch.bfloat16), pool, slots)
            rt.index_append(torch.randn(n, 128, device=dev).to(torch.bfloat16), index, slots)
        tables = torch.randperm(pages, generator=g).view(B, ctx // 64).to(torch.int32).to(dev)
        layers.append(dict(pool=pool, index=index, tables=tables,
                           iq=torch.randn(B, 64, 128, generator=g).to(torch.bfloat16).to(dev),
                           iw=(torch.rand(B, 64, generator=g) / 64).to(dev),
                           q=torch.randn(B, 1, H, 576, generator=g).to(torch.bfloat16).to(dev),
                           seq=torch.full((B,), ctx, dtype=torch.int32, device=dev),
                           rows=torch.empty(B, K, dtype=torch.int32, device=dev),
                           count=torch.empty(B, dtype=torch.int32, device=dev),
                           out=torch.empty(B, 1, H, 512, dtype=torch.bfloat16, device=dev)))

    def select(ly):
        rt.index_topk(ly["iq"], ly["iw"], ly["index"], ly["tables"], ly["seq"], ctx, K,
                      out_rows=ly["rows"], out_count=ly["count"])

    def decode(ly):
        rt.mla_decode(ly["q"], ly["pool"], None, 128, 512, 64, ly["rows"].view(B, 1, K), ly["count"], K,
                      sparse_mla_top_k=K, out=ly["out"], bmm1_scale=sm)

    for ly in layers:
        select(ly)
        decode(ly)
    torch.cuda.synchronize()
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    graphs = []
    with torch.cuda.stream(st):
        for ly in layers:
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=st):
                select(ly)
                decode(ly)
            graphs.append(gr)
    torch.cuda.current_stream().wait_stream(st)
    torch.cuda.synchronize()
    steps = args.steps if args.steps_given else 500
    sampler = ClockSampler(local)
    sampler.start()
    soak_end = time.perf_counter() + 1.0
    k = 0
    while time.perf_counter() < soak_end or k < args.warmup:
        graphs[k % 2].replay()
        k += 1
        if k % 32 == 0:
            torch.cuda.synchronize()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for k in range(steps):
        graphs[k % 2].replay()
    ev1.record()
    ev1.synchronize()
    t1 = time.perf_counter()
    if world > 1:
        dist.barrier()
    sampler.stop()
    t_max = torch.tensor([ev0.elapsed_time(ev1)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t_max, op=dist.ReduceOp.MAX)
    per_ms = float(t_max.item()) / steps
    kvb = kv_bytes_per_step(wl)
    value = kvb * world / (per_ms / 1e3) / 1e9
    # the two halves alone (eager, events around each)
    sel_ms, dec_ms = [], []
    for k in range(20):
        ly = layers[k % 2]
        a, b_, c = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        a.record()
        select(ly)
        b_.record()
        decode(ly)
        c.record()
        c.synchronize()
        sel_ms.append(a.elapsed_time(b_))
        dec_ms.append(b_.elapsed_time(c))
    sel_us = statistics.median(sel_ms) * 1e3
    dec_us = statistics.median(dec_ms) * 1e3
    # the decode of layer 0 against the exact attention over the rows the indexer picked
    ly = layers[0]
    check = prefill_check(torch, rt, dict(pool=ly["pool"], tables=ly["rows"].view(B, 1, K), q=ly["q"],
                                          out=ly["out"]), [0, B - 1], sm)
    errors = rt.device_errors(dev)
    if rank == 0:
        peak, peak_kind = load_peaks()
        index_bytes = B * ctx * INDEX_ROW_BYTES
        line = {
            "metric": METRIC + " (indexer + sparse decode)", "value": round(value, 2), "unit": "GB/s",
            "n_gpus": world, "steps": steps, "warmup": args.warmup, "ms_per_step": round(per_ms, 5),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16/f16",
            "data": "synthetic (seeded N(0,1) latent and indexer keys quantised by the append kernels; N(0,1) q)",
            "config": {"workload": wl["desc"], "global_batch": B * world, "seq_len": ctx, "topk": K,
                       "index_heads": 64, "index_dim": 128,
                       "l2": f"inputs larger than L2: 2 layers x {kvb / 2**20:.0f} MiB read per step",
                       "parallelism": f"sequence-partitioned x{world} (weak scaling)"},
            "bytes_per_step": {"index_keys": index_bytes, "latent_rows": B * K * NV_BYTES},
            "decode_tokens_per_s": round(B * world / (per_ms / 1e3), 1),
            "roofline": {"bound": "hbm", "achieved": round(index_bytes / (sel_us / 1e6) / 1e9, 2), "peak": peak,
                         "unit": "GB/s", "frac": round(index_bytes / (sel_us / 1e6) / 1e9 / peak, 4),
                         "peak_kind": peak_kind, "kernel": "index_score_kernel + index_topk_kernel",
                         "per_launch_bytes": index_bytes, "kernel_ms": round(sel_us / 1e3, 5),
                         "traffic": profile_traffic("dsa"), "decode_us": round(dec_us, 2),
                         "step_frac_in_kernel": round(sel_us / 1e3 / per_ms, 3)},
            "gpu_launches": steps * 5,
            "clocks": sampler.summary(t0, t1),
            "result_check": check,
            "device_errors": errors,
        }
        print(json.dumps(line), flush=True)
    del graphs
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if not check["passed"]:
        sys.exit("result check failed: a decode output is outside 2e-2 rel / 1e-2 abs")


def run_long(args, wl, rt, torch, dist, dev, rank, world, local):
    """--workload long: the partitioned config-4 layer (strong scaling)."""
    from glm53_flash_dual_dgx_spark_b200 import partition as P

    step, st, rank_bytes = make_long_step(rt, torch, wl, dev, rank, world, seed=1)
    job_bytes = kv_bytes_per_step(wl)
    for _ in range(3):
        step()
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(gr, stream=s):
            step()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    launches = 0
    for c in st["calls"]:
        qlen, heads = (1, wl["QL"] * wl["H"]) if c["fold"] else (wl["QL"], wl["H"])
        launches += rt.mla_decode_plan(c["n"], qlen, heads, c["max_len"], 0, dev)[1]
    sampler = ClockSampler(local)
    sampler.start()
    soak_end = time.perf_counter() + 1.0
    k = 0
    while time.perf_counter() < soak_end or k < args.warmup:
        gr.replay()
        k += 1
        if k % 16 == 0:
            torch.cuda.synchronize()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(args.steps):
        gr.replay()
    ev1.record()
    ev1.synchronize()
    t1 = time.perf_counter()
    if world > 1:
        dist.barrier()
    sampler.stop()
    t_max = torch.tensor([ev0.elapsed_time(ev1)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t_max, op=dist.ReduceOp.MAX)
    ms_max = float(t_max.item())
    value = job_bytes * args.steps / (ms_max / 1e3) / 1e9

    # end to end through the public API: q host->device, the rank's decode + merge, the rank's
    # merged partial outputs device->host (eager)
    q_h = st["q"].cpu().pin_memory()
    out_h = torch.empty(wl["B"], wl["QL"], wl["H"], 512, dtype=torch.bfloat16).pin_memory()
    e_steps = max(10, min(args.e2e_steps, 50))
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(e_steps):
        st["q"].copy_(q_h, non_blocking=True)
        step()
        out_h.copy_(st["out"], non_blocking=True)
    e1.record()
    e1.synchronize()
    e_ms = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(e_ms, op=dist.ReduceOp.MAX)
    e2e_value = job_bytes * e_steps / (float(e_ms.item()) / 1e3) / 1e9

    # the dominant attention kernel alone (the pieces before each causal tail), events
    # recorded by the library around it
    big = max(st["calls"], key=lambda c: c["n"])
    big_bytes = int(big["seq"].sum().item()) * NV_BYTES
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(10)]
    sm = 1.0 / math.sqrt(576)
    for a, b in kev:
        qq = big["qbuf"].view(big["n"], 1, wl["QL"] * wl["H"], 576) if big["fold"] else big["qbuf"]
        oo = big["out"].view(big["n"], 1, wl["QL"] * wl["H"], 512) if big["fold"] else big["out"]
        rt.set_kernel_events(a, b)
        rt.mla_decode_lse(qq, st["pool"], None, 128, 512, 64, big["tables"], big["seq"], big["max_len"],
                          out=oo, bmm1_scale=sm)
    torch.cuda.synchronize()
    kernel_ms = sum(a.elapsed_time(b) for a, b in kev) / len(kev)
    k_ms = torch.tensor([kernel_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(k_ms, op=dist.ReduceOp.MAX)
    kernel_ms = float(k_ms.item())

    # after timing: the cross-rank merge (the only data collective), then rank 0 checks the
    # merged result against the unpartitioned decode of the same sequences
    step()
    torch.cuda.synchronize()
    if world > 1:
        out_u, lse_u = st["out_u"], st["lse_u"]
        merged, _ = P.gather_merge(out_u, lse_u, [[u for part in st["plan"][r * LONG_PIECES_PER_RANK:(r + 1) * LONG_PIECES_PER_RANK]
                                                  for u in part] for r in range(world)], rank, wl["B"])
        torch.cuda.synchronize()
    else:
        merged = st["out"]
    check = long_check(rt, torch, wl, dev, world, merged, 1, sm) if rank == 0 else {"passed": True}
    flag = torch.tensor([1 if check["passed"] else 0], dtype=torch.int32, device=dev)
    if world > 1:
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    passed = bool(flag.item())
    errors = rt.device_errors(dev)
    if rank == 0:
        peak, peak_kind = load_peaks()
        achieved = big_bytes / (kernel_ms / 1e3) / 1e9
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 5),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic (seeded N(0,1) latent quantised by the append kernel; N(0,1) q)",
            "config": {"workload": wl["desc"], "global_batch": wl["B"], "seq_len": max(wl["lens"]),
                       "tokens": sum(wl["lens"]), "heads": wl["H"], "q_len": wl["QL"],
                       "pieces_per_rank": LONG_PIECES_PER_RANK, "units_on_rank0": len(st["units"]),
                       "l2": f"inputs larger than L2: {rank_bytes / 2**20:.0f} MiB read per step on rank 0",
                       "parallelism": f"sequence / page-range partition x{world} (strong scaling)"},
            "decode_tokens_per_s": round(wl["B"] * wl["QL"] * args.steps / (ms_max / 1e3), 1),
            "kv_rows_per_s": round(job_bytes * args.steps / (ms_max / 1e3) / NV_BYTES, 1),
            "hbm_frac_of_8tbs": round(value / world / 8000.0, 4),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_kind": peak_kind, "traffic": None,
                         "per_launch_bytes": big_bytes, "kernel_ms": round(kernel_ms, 5),
                         "kernel": "decode_fp4_kernel<dense>",
                         "step_frac_in_kernel": round(kernel_ms / (ms_max / args.steps), 3)},
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": q_h.numel() * 2,
                    "d2h_bytes_per_step": out_h.numel() * 2, "steps": e_steps},
            "gpu_launches": args.steps * launches,
            "clocks": sampler.summary(t0, t1),
            "result_check": check,
            "device_errors": errors,
        }
        if world == 1:
            gbs, per, ctx = cpu_decode_sample(wl, args.cpu_seconds)
            line["cpu_baseline"] = {
                "value": round(gbs, 4), "unit": "GB/s", "cores": os.cpu_count(), "kind": "port",
                "sample": f"oracle decode of one {ctx}-token piece x {wl['QL']} x {wl['H']} query rows "
                          f"repeated for ~{args.cpu_seconds:.0f} s ({per * 1e3:.1f} ms each; {cpu_model()})"}
        print(json.dumps(line), flush=True)
    del gr
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if not passed:
        sys.exit("long: the merged partitioned result differs from the unpartitioned decode")


# ---------------------------------------------------------------------------- CPU side
def cpu_decode_sample(wl, seconds: float):
    """The oracle (CPU restatement of the reference path) on a bounded sample: whole
    sequences of the workload (dequantise + fp32 attention), repeated for ~`seconds`."""
    import numpy as np
    import torch

    from oracle import oracle as O

    ctx = wl["topk"] if wl["topk"] else min(wl["ctx"] or 8192, 8192)
    g = torch.Generator().manual_seed(11)
    x = torch.randn(ctx, 512, generator=g).to(torch.bfloat16)
    pool = O.quant_new(x)
    q = torch.randn(1, wl["QL"], wl["H"], 576, generator=g).float().numpy()
    if wl["topk"]:
        tables, seq, sparse = np.arange(ctx, dtype=np.int32).reshape(1, 1, ctx), np.array([ctx]), True
    else:
        pool = np.concatenate([pool, np.zeros(((-ctx) % 64, NV_BYTES), np.uint8)])
        tables, seq, sparse = np.arange(pool.shape[0] // 64, dtype=np.int32)[None], np.array([ctx]), False
    sm = 1.0 / math.sqrt(576)
    runs, t0 = 0, time.perf_counter()
    while True:
        O.mla_decode(q, pool, tables, seq, sparse=sparse, bmm1_scale=sm, dtype=np.float32)
        runs += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    gbs = runs * ctx * NV_BYTES / el / 1e9
    return gbs, el / runs, ctx


def reference_arm(args, wl):
    """--impl reference: the CPU restatement of the reference path (the reference's own code
    is Python + Triton and is not available on the GPU host), rank 0 only."""
    if int(os.environ.get("RANK", "0")) != 0:
        return
    import numpy as np  # noqa: F401

    cores = os.cpu_count()
    if wl.get("dedup"):
        cpu_dedup_sample(wl, 0.0)
        times = []
        for i in range(args.warmup + args.steps):
            gbs, per, desc = cpu_dedup_sample(wl, 0.0)
            if i >= args.warmup:
                times.append((gbs, per))
        gbs = sum(g for g, _ in times) / len(times)
        per = sum(p for _, p in times) / len(times)
        line = {"impl": "reference",
                "metric": "sync-free dedup + 656 B gather GB/s (8 B per table entry, 944 B per distinct row)",
                "value": round(gbs, 4), "unit": "GB/s", "n_gpus": args.gpus, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(per * 1e3, 3), "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "u8",
                "data": "synthetic (seeded uniform top-k entries over a context window, 10 % -1)",
                "config": {"workload": wl["desc"], "parallelism": f"a pool per rank x{args.gpus}"},
                "cpu_baseline": {"value": round(gbs, 4), "unit": "GB/s", "cores": 1, "kind": "port",
                                 "sample": f"oracle build_scratch large-step branch on {desc} ({cpu_model()})"},
                "e2e": {"value": round(gbs, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
        print(json.dumps(line), flush=True)
        return
    append = "pool_tokens" in wl
    sample_fn = (lambda: cpu_append_sample(0.0)) if append else (lambda: cpu_decode_sample(wl, 0.0))
    sample_fn()                                    # warm: build oracle, fault pages in
    times = []
    for i in range(args.warmup + args.steps):
        gbs, per, ctx = sample_fn()
        if i >= args.warmup:
            times.append(per)
    per = sum(times) / len(times)
    if append:
        value = ctx * APPEND_BYTES_PER_TOKEN / per / 1e9
        cores = 1
        sample = (f"{ctx} tokens per step: oracle append (C restatement of _quant_kernel) on one "
                  f"host thread ({cpu_model()})")
    else:
        value = ctx * NV_BYTES / per / 1e9
        sample = (f"one sequence of the workload per step ({ctx} tokens x {wl['H']} heads): oracle "
                  f"dequantise (C) + numpy fp32 attention on {cores} host threads ({cpu_model()})")
    metric = ("NVFP4 append GB/s (1320 B per token: bf16 latent read, 288 B row and slot)" if append
              else METRIC)
    line = {"impl": "reference", "metric": metric, "value": round(value, 4), "unit": "GB/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(per * 1e3, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0,1) latent and q)",
            "config": {"workload": wl["desc"], "global_batch": wl["B"] * args.gpus,
                       "seq_len": wl["topk"] or wl["ctx"] or max(wl.get("lens", [0])),
                       "parallelism": f"sequence-partitioned x{args.gpus}"},
            "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": cores, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------- the reference on the GPU
REF_RUNTIME = os.environ.get("GLM53_REFERENCE_RUNTIME",
                             os.path.join(ROOT, "baseline", "_ref", "nvfp4-kv", "glm53_nvfp4_runtime.py"))


def load_reference_runtime():
    """The reference's own runtime module (unmodified, from its install under baseline/_ref), or
    (None, reason)."""
    import importlib.util

    if not os.path.exists(REF_RUNTIME):
        return None, f"reference runtime not installed at {REF_RUNTIME}"
    try:
        spec = importlib.util.spec_from_file_location("glm53_reference_runtime", REF_RUNTIME)
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        return mod, None
    except Exception as e:  # noqa: BLE001
        return None, f"reference runtime failed to import: {e!r}"[:300]


def graph_time_us(torch, fns, steps, warm=3):
    """Mean device time of fns[k % len(fns)]() replayed from CUDA graphs (one per fn), CUDA events
    on the replay stream; eager if a capture fails."""
    for f in fns:
        for _ in range(warm):
            f()
    torch.cuda.synchronize()
    graphs, mode = [], "cuda graphs"
    try:
        st = torch.cuda.Stream()
        st.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(st):
            for f in fns:
                gr = torch.cuda.CUDAGraph()
                with torch.cuda.graph(gr, stream=st):
                    f()
                graphs.append(gr)
        torch.cuda.current_stream().wait_stream(st)
        torch.cuda.synchronize()
        run = [g.replay for g in graphs]
    except Exception:  # noqa: BLE001
        graphs, run, mode = [], fns, "eager"
        torch.cuda.synchronize()
    for k in range(2 * len(run)):
        run[k % len(run)]()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for k in range(steps):
        run[k % len(run)]()
    b.record()
    b.synchronize()
    del graphs
    return a.elapsed_time(b) / steps * 1e3, mode


def gpu_reference_decode(torch, wl, L, dev, ours_us):
    """The reference's read path on this GPU for the same layers: its build_scratch (Triton
    _gather_kernel into 656 B fp8_ds_mla rows, runtime:143-176) followed by a stock B200 consumer
    of those rows, vLLM's FlashMLA sparse fp8 decode (the fork's FlashInfer consumer of the
    656 B rows is not in this image; FlashInfer 0.6.11's trtllm-gen MLA takes only 576 B rows)."""
    ref, why = load_reference_runtime()
    if ref is None:
        return {"unavailable": why}
    B, ctx, topk = wl["B"], wl["ctx"], wl["topk"]
    K = topk or ctx
    sm = 1.0 / math.sqrt(576)
    rec = {"path": "reference build_scratch (Triton _gather_kernel, 656 B rows) -> FlashMLA sparse fp8 decode "
                   "(vLLM 0.22) on those rows", "config": f"batch {B}, {K} rows per sequence"}
    rows = []
    for ly in L:
        if topk:
            rows.append(ly["tables"].view(B, 1, topk))
        else:
            pos = torch.arange(ctx, device=dev)
            pt = ly["tables"].long()
            rows.append((pt[:, pos // 64] * 64 + pos % 64).to(torch.int32).view(B, 1, ctx))
    ref._bufs.clear()
    try:
        g_us, mode = graph_time_us(torch, [lambda i=i: ref.build_scratch(L[i]["pool"], rows[i]) for i in range(len(L))],
                                   50 if K > 8192 else 400)
        rec["gather_us"], rec["timing"] = round(g_us, 2), mode
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"reference gather failed: {e!r}"[:300]}
    rec["gather_bytes_per_step"] = B * K * (NV_BYTES + 656)
    if K > 8192:
        rec["consumer"] = ("not run: FlashMLA's sparse decode at top-k %d is outside its design point; the "
                           "reference gather alone bounds the path from below" % K)
        rec["step_us_lower_bound"] = rec["gather_us"]
        rec["ours_step_us"] = round(ours_us, 2)
        rec["speedup_at_least"] = round(rec["gather_us"] / ours_us, 2)
        return rec
    try:
        from vllm.third_party.flashmla.flash_mla_interface import flash_mla_with_kvcache, get_mla_metadata

        metas = [get_mla_metadata()[0] for _ in L]

        def consume(i, scratch, tables):
            return flash_mla_with_kvcache(q=L[i]["q"], k_cache=scratch.view(-1, 64, 1, 656), block_table=None,
                                          cache_seqlens=None, head_dim_v=512, tile_scheduler_metadata=metas[i],
                                          is_fp8_kvcache=True, indices=tables.view(B, 1, K), softmax_scale=sm)[0]

        def full(i):
            scratch, tables = ref.build_scratch(L[i]["pool"], rows[i])
            return consume(i, scratch, tables)

        f_us, mode = graph_time_us(torch, [lambda i=i: full(i) for i in range(len(L))], 400)
        rec["step_us"] = round(f_us, 2)
        rec["consumer_us"] = round(max(f_us - rec["gather_us"], 0.0), 2)
        rec["ours_step_us"] = round(ours_us, 2)
        rec["speedup"] = round(f_us / ours_us, 2)
        rec["timing"] = mode
        # the consumer's accuracy on these rows, against the exact dequantised attention
        o = full(0).float().view(B, wl["H"], 512)
        kv = _exact_rows(torch, L[0], rows[0][0, 0])
        qf = L[0]["q"][0, 0, :, :512].float()
        tru = torch.softmax(qf @ kv.t() * sm, dim=-1) @ kv
        rec["consumer_rel_err_seq0"] = round(float((o[0] - tru).norm() / tru.norm()), 4)
        rec["note"] = ("FlashMLA's output on these rows does not match the fp8_ds_mla format "
                       "(consumer_rel_err_seq0; also on rows written by vLLM's own concat_and_cache_mla), so its "
                       "time stands in for the fork's consumer, not its numbers")
    except Exception as e:  # noqa: BLE001
        rec["consumer"] = f"unavailable: {e!r}"[:300]
        rec["step_us_lower_bound"] = rec["gather_us"]
        rec["speedup_at_least"] = round(rec["gather_us"] / ours_us, 2)
    return rec


def _exact_rows(torch, ly, rows):
    from glm53_flash_dual_dgx_spark_b200 import glm53_nvfp4_runtime as rt

    return rt.dequant(ly["pool"], rows.to(torch.int32)).float()


def gpu_reference_append(torch, inputs, pool_rows, dev, ours_us):
    """The reference's write_nvfp4 (its Triton _quant_kernel, runtime:37-76) on the same chunks."""
    ref, why = load_reference_runtime()
    if ref is None:
        return {"unavailable": why}
    pool = torch.zeros(pool_rows, NV_BYTES, dtype=torch.uint8, device=dev)
    try:
        us, mode = graph_time_us(torch, [lambda inp=inp: ref.write_nvfp4(inp["x"], pool, inp["slots"])
                                         for inp in inputs], 200)
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"reference append failed: {e!r}"[:300]}
    return {"path": "reference write_nvfp4 (Triton _quant_kernel)", "step_us": round(us, 3), "timing": mode,
            "ours_step_us": round(ours_us, 3), "speedup": round(us / ours_us, 2)}


def gpu_reference_dedup(torch, pool, tabs_d, ours_us):
    """The reference's large-step build_scratch (torch.unique + its Triton gather, runtime:177-182),
    eager: torch.unique synchronises with the host to size its output."""
    ref, why = load_reference_runtime()
    if ref is None:
        return {"unavailable": why}
    try:
        for t in tabs_d:
            ref.build_scratch(pool, t)
        torch.cuda.synchronize()
        n = 20
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0 = time.perf_counter()
        a.record()
        for k in range(n):
            ref.build_scratch(pool, tabs_d[k % len(tabs_d)])
        b.record()
        b.synchronize()
        wall = (time.perf_counter() - t0) / n * 1e6
        us = a.elapsed_time(b) / n * 1e3
    except Exception as e:  # noqa: BLE001
        return {"unavailable": f"reference build_scratch failed: {e!r}"[:300]}
    return {"path": "reference build_scratch large-step branch (torch.unique + Triton gather, host sync)",
            "step_us": round(us, 2), "wall_us": round(wall, 2), "timing": "eager (the branch synchronises)",
            "ours_step_us": round(ours_us, 2), "speedup": round(us / ours_us, 2)}


def host_link_gbs(torch, dev, h2d_step: int, d2h_step: int) -> dict:
    """The box's pinned host<->device copy rates: one 64 MiB copy each way, and one copy of a
    step's input / output size, CUDA events on one stream (what bounds the e2e figure)."""
    res = {}
    for name, n in (("h2d_64MiB", 64 << 20), ("h2d_step", h2d_step), ("d2h_64MiB", 64 << 20), ("d2h_step", d2h_step)):
        h = torch.empty(n, dtype=torch.uint8).pin_memory()
        d = torch.empty(n, dtype=torch.uint8, device=dev)
        src, dst = (h, d) if name.startswith("h2d") else (d, h)
        for _ in range(3):
            dst.copy_(src, non_blocking=True)
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(10):
            dst.copy_(src, non_blocking=True)
        b.record()
        b.synchronize()
        us = a.elapsed_time(b) / 10 * 1e3
        res[name] = {"bytes": n, "us": round(us, 2), "GBs": round(n / us / 1e3, 1)}
    # a step's input and output copies at the same time, on two streams (what an engine's
    # pipelined step does): whether the link carries both directions at once
    hi = torch.empty(h2d_step, dtype=torch.uint8).pin_memory()
    di = torch.empty(h2d_step, dtype=torch.uint8, device=dev)
    do = torch.empty(d2h_step, dtype=torch.uint8, device=dev)
    ho = torch.empty(d2h_step, dtype=torch.uint8).pin_memory()
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    s1.wait_stream(torch.cuda.current_stream())
    s2.wait_stream(torch.cuda.current_stream())
    for _ in range(10):
        with torch.cuda.stream(s1):
            di.copy_(hi, non_blocking=True)
        with torch.cuda.stream(s2):
            ho.copy_(do, non_blocking=True)
    torch.cuda.current_stream().wait_stream(s1)
    torch.cuda.current_stream().wait_stream(s2)
    b.record()
    b.synchronize()
    us = a.elapsed_time(b) / 10 * 1e3
    res["both_step"] = {"bytes": h2d_step + d2h_step, "us": round(us, 2),
                        "GBs": round((h2d_step + d2h_step) / us / 1e3, 1)}
    return res


# ---------------------------------------------------------------------------- checks of the results
def fp32_check(torch, rt, wl, ly, seqs, sm):
    """Layer `ly`'s decode output for sequences `seqs` against the exact dequantised attention in
    fp32: (max over them of rel L2, whether every element is within 2e-2 rel / 1e-2 abs)."""
    B, H, ctx, topk = wl["B"], wl["H"], wl["ctx"], wl["topk"]
    worst, ok = 0.0, True
    for b in seqs:
        if topk:
            rows = ly["tables"].view(B, topk)[b]
        else:
            pos = torch.arange(ctx, device=ly["q"].device)
            rows = ly["tables"][b].long()[pos // 64] * 64 + pos % 64
        kv = rt.dequant(ly["pool"], rows.to(torch.int32)).float()
        qf = ly["q"][b, 0, :, :512].float()
        tru = torch.softmax(qf @ kv.t() * sm, dim=-1) @ kv
        o = ly["out"][b, 0].float()
        worst = max(worst, float((o - tru).norm() / tru.norm()))
        ok = ok and bool(((o - tru).abs() <= 1e-2 + 2e-2 * tru.abs()).all())
    return worst, ok


def check_ranks(torch, rt, dist, wl, L, dev, rank, world, call, sm):
    """After timing: every rank's layer-0 output is all-gathered over NCCL, and rank 0 rebuilds each
    other rank's layer 0 from its seed, decodes it itself and compares (same kernels and inputs:
    expected bit-identical; the gate is 2e-2 rel / 1e-2 abs).  Every rank also checks two of its
    own sequences against the exact fp32 attention.  Returns the record (rank 0) and whether every
    check passed (all ranks agree on it)."""
    rel, ok_fp32 = fp32_check(torch, rt, wl, L[0], [0, wl["B"] - 1], sm)
    rec = {"fp32_rel_l2_max": round(rel, 5), "fp32_within_tol": ok_fp32}
    ok = ok_fp32
    if world > 1:
        gathered = [torch.empty_like(L[0]["out"]) for _ in range(world)]
        dist.all_gather(gathered, L[0]["out"])
        torch.cuda.synchronize()
        if rank == 0:
            max_diff, identical, within = 0.0, True, True
            for r in range(1, world):
                lr = make_layers(rt, torch, wl, 1, dev, seed=1 + r)[0]
                call(lr)
                torch.cuda.synchronize()
                got, mine = gathered[r].float(), lr["out"].float()
                max_diff = max(max_diff, float((got - mine).abs().max()))
                identical = identical and bool(torch.equal(gathered[r], lr["out"]))
                within = within and bool(((got - mine).abs() <= 1e-2 + 2e-2 * mine.abs()).all())
                del lr
                torch.cuda.empty_cache()
            rec.update({"ranks_rechecked_on_rank0": world - 1, "max_abs_diff": max_diff,
                        "bit_identical": identical, "within_tol": within})
            ok = ok and within
        flag = torch.tensor([1 if ok else 0], dtype=torch.int32, device=dev)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        ok = bool(flag.item())
    rec["passed"] = ok
    return rec, ok


# ---------------------------------------------------------------------------- GPU side
def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--workload", default="sparse", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=200)
    ap.add_argument("--cpu-seconds", type=float, default=8.0)
    args = ap.parse_args()
    args.steps_given = args.steps is not None
    if args.steps is None:
        args.steps = 2000
    wl = WORKLOADS[args.workload]
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        reference_arm(args, wl)
        return

    import torch
    import torch.distributed as dist

    from glm53_flash_dual_dgx_spark_b200 import glm53_nvfp4_runtime as rt

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)
    if "lens" in wl:
        run_long(args, wl, rt, torch, dist, dev, rank, world, local)
        return
    if wl.get("prefill"):
        run_prefill(args, wl, rt, torch, dist, dev, rank, world, local)
        return
    if wl.get("dsa"):
        run_dsa(args, wl, rt, torch, dist, dev, rank, world, local)
        return
    if wl.get("dedup"):
        run_dedup(args, wl, rt, torch, dist, dev, rank, world, local)
        return
    if "pool_tokens" in wl:
        run_append(args, wl, rt, torch, dist, dev, rank, world, local)
        return

    kvb = kv_bytes_per_step(wl)
    # layers so that one rotation reads more than L2 (sparse: distinct top-k sets)
    touched = kvb
    layers = max(1, math.ceil(2 * L2_BYTES / touched)) if wl["topk"] == 0 else 32
    layers = min(layers, 32)
    L = make_layers(rt, torch, wl, layers, dev, seed=1 + rank)
    sm = 1.0 / math.sqrt(576)

    def call(ly, out=None):
        return rt.mla_decode(ly["q"], ly["pool"], None, 128, 512, 64, ly["tables"], ly["seq"],
                             wl["topk"] or wl["ctx"], sparse_mla_top_k=wl["topk"],
                             out=ly["out"] if out is None else out, bmm1_scale=sm, bmm2_scale=1.0)

    for ly in L:                                   # eager warm-up (allocates the workspace once)
        call(ly)
    torch.cuda.synchronize()
    graphs = []
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for ly in L:
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=s):
                call(ly)
            graphs.append(gr)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    splits, launches_per_step = rt.mla_decode_plan(wl["B"], wl["QL"], wl["H"], wl["topk"] or wl["ctx"],
                                                    wl["topk"], dev)

    sampler = ClockSampler(local)
    sampler.start()
    soak_end = time.perf_counter() + 1.0           # clocks settle under load first
    k = 0
    while time.perf_counter() < soak_end or k < args.warmup:
        graphs[k % layers].replay()
        k += 1
        if k % 64 == 0:
            torch.cuda.synchronize()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for k in range(args.steps):
        graphs[k % layers].replay()
    ev1.record()
    ev1.synchronize()
    torch.cuda.synchronize()
    t1 = time.perf_counter()
    if world > 1:
        dist.barrier()
    sampler.stop()
    ms = ev0.elapsed_time(ev1)
    t_max = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t_max, op=dist.ReduceOp.MAX)
    ms_max = float(t_max.item())
    sec = ms_max / 1e3
    value = kvb * args.steps * world / sec / 1e9
    tokens_s = wl["B"] * wl["QL"] * args.steps * world / sec

    # ---- end to end through the public API (eager, host buffers, copies in the region).
    # Pipelined as a serving loop runs it: step k+1's q / tables / seq_lens go host->device on
    # a copy stream while step k decodes, and step k's output comes back on a third stream;
    # two buffer sets, with events ordering every reuse.  Every step's copies are inside the
    # timed region.  The serial variant (one stream: copies, decode, read-back) is reported
    # beside it.
    e2e_steps = max(args.e2e_steps, 10)
    h2d = L[0]["q_h"].numel() * 2 + L[0]["tables_h"].numel() * 4 + L[0]["seq_h"].numel() * 4
    d2h = L[0]["out"].numel() * 2

    def e2e_run(pipelined: bool) -> float:
        nb = 2 if pipelined else 1
        ins = [(torch.empty_like(L[0]["q"]), torch.empty_like(L[0]["tables"]), torch.empty_like(L[0]["seq"]))
               for _ in range(nb)]
        outs = [torch.empty_like(L[0]["out"]) for _ in range(nb)]
        outs_h = [torch.empty(L[0]["out"].shape, dtype=torch.bfloat16).pin_memory() for _ in range(nb)]
        main = torch.cuda.current_stream()
        cin = torch.cuda.Stream() if pipelined else main
        cout = torch.cuda.Stream() if pipelined else main
        ev = lambda: torch.cuda.Event()   # noqa: E731
        in_ready = [ev() for _ in range(e2e_steps)]
        dec_done = [ev() for _ in range(e2e_steps)]
        out_done = [ev() for _ in range(e2e_steps)]

        def h2d_copy(k):
            ly, bset = L[k % layers], ins[k % nb]
            with torch.cuda.stream(cin):
                if k >= nb:
                    cin.wait_event(dec_done[k - nb])          # decode k - nb has read this set
                bset[0].copy_(ly["q_h"], non_blocking=True)
                bset[1].copy_(ly["tables_h"], non_blocking=True)
                bset[2].copy_(ly["seq_h"], non_blocking=True)
                in_ready[k].record(cin)

        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(cin)
        h2d_copy(0)
        for k in range(e2e_steps):
            if pipelined and k + 1 < e2e_steps:
                h2d_copy(k + 1)
            elif not pipelined and k > 0:
                h2d_copy(k)
            b = k % nb
            main.wait_event(in_ready[k])
            if k >= nb:
                main.wait_event(out_done[k - nb])             # the output set was read back
            qd, td, sd = ins[b]
            rt.mla_decode(qd, L[k % layers]["pool"], None, 128, 512, 64, td, sd, wl["topk"] or wl["ctx"],
                          sparse_mla_top_k=wl["topk"], out=outs[b], bmm1_scale=sm, bmm2_scale=1.0)
            dec_done[k].record(main)
            with torch.cuda.stream(cout):
                cout.wait_event(dec_done[k])
                outs_h[b].copy_(outs[b], non_blocking=True)
                out_done[k].record(cout)
        e1.record(cout)
        e1.synchronize()
        torch.cuda.synchronize()
        e_ms = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(e_ms, op=dist.ReduceOp.MAX)
        return kvb * e2e_steps * world / (float(e_ms.item()) / 1e3) / 1e9

    def e2e_graph_run() -> tuple:
        """The serving loop as an engine runs decode, with each step's host work captured once:
        one CUDA graph per step of the rotation, three branches joined at its end - step k+1's
        input copies from pinned host memory, the public mla_decode call of step k, and step
        k-1's output copy to pinned host memory.  Graphs replay one after another on one
        stream, so decodes run in order (as layers do) while the copies of the neighbouring
        steps overlap them; every replay re-runs its copies.  Two buffer sets, step k on set
        k % 2: a step writes the inputs and reads the output of the other set; the graphs cover
        a period of lcm(layers, 2) steps.  Returns (GB/s, steps, whether the last read-back
        matches its device output)."""
        nb = 2
        period = layers if layers % nb == 0 else nb * layers
        ins = [(torch.empty_like(L[0]["q"]), torch.empty_like(L[0]["tables"]), torch.empty_like(L[0]["seq"]))
               for _ in range(nb)]
        outs = [torch.empty_like(L[0]["out"]) for _ in range(nb)]
        outs_h = [torch.empty(L[0]["out"].shape, dtype=torch.bfloat16).pin_memory() for _ in range(nb)]
        main, cin, cout = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()
        for st in (main, cin, cout):
            st.wait_stream(torch.cuda.current_stream())

        def copy_in(j, b):
            qd, td, sd = ins[b]
            qd.copy_(L[j]["q_h"], non_blocking=True)
            td.copy_(L[j]["tables_h"], non_blocking=True)
            sd.copy_(L[j]["seq_h"], non_blocking=True)

        graphs = []
        for pk in range(period):
            j, b, nxt = pk % layers, pk % nb, (pk + 1) % nb
            qd, td, sd = ins[b]
            g = torch.cuda.CUDAGraph()
            with torch.cuda.stream(main), torch.cuda.graph(g, stream=main):
                cin.wait_stream(main)
                cout.wait_stream(main)
                with torch.cuda.stream(cin):
                    copy_in((j + 1) % layers, nxt)
                with torch.cuda.stream(cout):
                    outs_h[nxt].copy_(outs[nxt], non_blocking=True)
                rt.mla_decode(qd, L[j]["pool"], None, 128, 512, 64, td, sd, wl["topk"] or wl["ctx"],
                              sparse_mla_top_k=wl["topk"], out=outs[b], bmm1_scale=sm, bmm2_scale=1.0)
                main.wait_stream(cin)
                main.wait_stream(cout)
            graphs.append(g)
        torch.cuda.synchronize()
        n = max(e2e_steps, 2 * period)
        n += (-n) % period
        for rep in range(2):                       # an untimed pass, then the timed one
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(main)
            with torch.cuda.stream(main):
                copy_in(0, 0)                      # step 0's inputs
                for k in range(n):
                    graphs[k % period].replay()
                last = (n - 1) % nb
                outs_h[last].copy_(outs[last], non_blocking=True)   # step n-1's output
            e1.record(main)
            e1.synchronize()
        # the last read-back equals the device-side decode of that layer (same inputs,
        # deterministic kernels)
        ok = bool(torch.equal(outs_h[(n - 1) % nb], L[(n - 1) % layers]["out"].cpu()))
        e_ms = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(e_ms, op=dist.ReduceOp.MAX)
        del graphs
        return kvb * n * world / (float(e_ms.item()) / 1e3) / 1e9, n, ok

    for k in range(3):                             # warm the eager path
        ly = L[k % layers]
        call(ly)
    e2e_serial = e2e_run(False)
    e2e_eager = e2e_run(True)
    e2e_value, e2e_graph_steps, e2e_graph_same = e2e_graph_run()
    link = host_link_gbs(torch, dev, h2d, d2h)

    # ---- the attention kernel alone: CUDA events recorded by the library immediately around
    # it (on its stream), over a separate run of the same steps
    k_steps = min(args.steps, 200)
    kev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(k_steps)]
    for k in range(k_steps):
        ly = L[k % layers]
        rt.set_kernel_events(*kev[k])
        call(ly)
    torch.cuda.synchronize()
    kernel_ms = sum(a.elapsed_time(b) for a, b in kev) / k_steps
    k_ms = torch.tensor([kernel_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(k_ms, op=dist.ReduceOp.MAX)
    kernel_ms = float(k_ms.item())

    # ---- outputs of every rank gathered once, after timing (the only data collective), and
    # checked: rank 0 decodes every other rank's layer 0 itself and compares
    check, passed = check_ranks(torch, rt, dist, wl, L, dev, rank, world, call, sm)

    errors = rt.device_errors(dev)
    if rank == 0:
        peak, peak_kind = load_peaks()
        achieved = kvb / (kernel_ms / 1e3) / 1e9   # KV bytes per launch / attention-kernel time
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 5),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16",
            "data": "synthetic (seeded N(0,1) latent quantised by the append kernel; N(0,1) q)",
            "config": {"workload": wl["desc"], "global_batch": wl["B"] * world,
                       "seq_len": wl["ctx"], "topk": wl["topk"], "heads": wl["H"], "q_len": wl["QL"],
                       "layers_rotated": layers,
                       "l2": f"inputs larger than L2: {layers} layer(s) x {kvb / 2**20:.1f} MiB read per rotation",
                       "parallelism": f"sequence-partitioned x{world} (weak scaling)"},
            "decode_tokens_per_s": round(tokens_s, 1),
            "kv_rows_per_s": round(kvb * args.steps * world / sec / NV_BYTES, 1),
            "hbm_frac_of_8tbs": round(value / world / 8000.0, 4),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                         "traffic": profile_traffic(args.workload),
                         "per_launch_bytes": kvb, "kernel_ms": round(kernel_ms, 5),
                         "kernel": "decode_fp4_kernel<sparse>" if wl["topk"] else "decode_fp4_kernel<dense>",
                         "step_frac_in_kernel": round(kernel_ms / (ms_max / args.steps), 3),
                         "splits": splits},
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "steps": e2e_graph_steps,
                    "pipeline": "one CUDA graph per step, captured once: step k+1's pinned-host input copies, "
                                "the public mla_decode call of step k and step k-1's output copy to pinned host "
                                "memory as three parallel branches (every replay re-runs the copies); graphs replay "
                                "in order on one stream, so decodes run one after another",
                    "read_back_matches_device_output": e2e_graph_same,
                    "eager_value": round(e2e_eager, 2),
                    "eager_pipeline": "eager mla_decode calls; copies of step k+1 / k-1 overlap the decode of "
                                      "step k (3 streams)",
                    "serial_value": round(e2e_serial, 2), "host_link": link},
            "gpu_launches": args.steps * launches_per_step,
            "clocks": sampler.summary(t0, t1),
            "device_errors": errors,
        }
        line["result_check"] = check
        if world == 1:
            line["gpu_reference"] = gpu_reference_decode(torch, wl, L, dev, ms_max / args.steps * 1e3)
            gbs, per, ctx = cpu_decode_sample(wl, args.cpu_seconds)
            line["cpu_baseline"] = {
                "value": round(gbs, 4), "unit": "GB/s", "cores": os.cpu_count(), "kind": "port",
                "sample": f"oracle decode of one {ctx}-token sequence x {wl['H']} heads repeated for "
                          f"~{args.cpu_seconds:.0f} s ({per * 1e3:.1f} ms each; C dequantise + numpy "
                          f"fp32 attention; {cpu_model()})"}
        print(json.dumps(line), flush=True)
    del graphs
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if not passed:
        sys.exit("result check failed: a rank's output is outside 2e-2 rel / 1e-2 abs")


if __name__ == "__main__":
    main()
