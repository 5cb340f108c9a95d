#!/usr/bin/env python
"""Benchmark of the CSA 4-bit-KV decode hot path.

One *step* = one fused decode pass (indexer -> exact top-256 -> sparse sink
attention over the selected compressed blocks + 128-token window) for a batch
of 64 sequences whose contexts are drawn uniformly from 16K-32K tokens
(4096-8192 compressed blocks), 12 heads x 128, 4-bit TurboQuant paged cache.
A *query* is one sequence x one step x one layer.

  value      queries/s over all ranks, inputs resident in HBM; steps replayed
             from a CUDA graph; every step reads a different cache set, and
             the sets together are > 4x L2 so every step reads cold HBM
  e2e        queries/s through the public host-buffer API (``CsaDecodeHostPlan``)
             with the step's inputs copied from pinned host memory and the
             outputs copied back inside the timed region
  roofline   algorithmic bytes per launch / CUDA-event launch time, against
             the measured HBM copy bandwidth (MEASURED_PEAKS.json)
  cpu_baseline  the CPU restatement of the reference's fp32 torch path
             (dequant, indexer, topk, gather, sparse attention) timed on the
             host cores on a bounded sample of the same workload

Multi-GPU: one process per GPU (torchrun); every rank runs its own batch of
64 sequences (request partitioning, no collective on the data path);
`value` = all ranks' queries / the slowest rank's time.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "deepseek-v4-codebase_b200"))

METRIC = "CSA 4-bit-KV decode queries/s at 16K-32K ctx (batch 64/GPU)"
UNIT = "queries/s"
CFG = dict(batch=64, ctx_lo=16384, ctx_hi=32768, bits=4, compression=4, heads=12, window=128, top_k=256)
FALLBACK_HBM_GBS = 6650.0
NCU_SUMMARY = ROOT / "profiles" / "csa_decode_4bit_b64_ncu.md"


def algorithmic_bytes(nblocks, window_len, bits, heads=12, top_k=256):
    """Bytes one decode step must move: index pages (codes + scales), the
    selected main entries, the bf16 window, q in / out, index query, head
    weights, sink and the page-table entries."""
    total = 0
    for nb, wl in zip(nblocks, window_len):
        k = min(top_k, nb)
        total += nb * (64 * bits // 8 + 4)
        total += k * (128 * bits // 8 + 4)
        total += wl * 128 * 2
        total += heads * 128 * 2 * 2
        total += 4 * 64 * 4 + 4 * 4 + heads * 4
        total += 4 * ((nb + 63) // 64)
    return total


def read_peak():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback"


def read_traffic(summary=None):
    """Per-launch DRAM bytes of a kernel from its committed ncu summary (line
    'traffic_bytes_per_launch: N'; default: the CSA decode one), or None."""
    summary = NCU_SUMMARY if summary is None else summary
    if not summary.exists():
        return None
    for line in summary.read_text().splitlines():
        if line.strip().startswith("traffic_bytes_per_launch:"):
            try:
                return int(line.split(":", 1)[1].strip())
            except ValueError:
                return None
    return None


def init_nccl(dist, dev):
    """init_process_group over NCCL with the communicator created eagerly; fd
    1 points at stderr meanwhile, so a banner NCCL prints at init (NCCL_DEBUG)
    stays out of rank 0's stdout, which carries only the JSON line."""
    sys.stdout.flush()
    saved = os.dup(1)
    os.dup2(2, 1)
    try:
        dist.init_process_group("nccl", device_id=dev)
    finally:
        sys.stdout.flush()
        os.dup2(saved, 1)
        os.close(saved)


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""

    FIELDS = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.thread.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) != 6:
                continue
            try:
                sm.append(float(parts[0]))
                mx = float(parts[1])
            except ValueError:
                continue
            for nm, v in zip(names, parts[2:]):
                if v.lower() == "active":
                    reasons.add(nm)
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def max_ws_bytes(batch):
    from aether_kernels.paged import csa_workspace_bytes

    return csa_workspace_bytes(batch, CFG["ctx_hi"] // CFG["compression"])


def build_sets(nsets, device, rank):
    from aether_kernels.paged import PAGE, TurboQuantPagedCache
    from aether_kernels.synthetic import make_decode_batch

    B, bits = CFG["batch"], CFG["bits"]
    max_pages = CFG["ctx_hi"] // CFG["compression"] // PAGE
    cache = TurboQuantPagedCache(nsets * B * max_pages, bits, device)
    sets = []
    for s in range(nsets):
        sets.append(make_decode_batch("csa", B, CFG["ctx_lo"], CFG["ctx_hi"], bits, CFG["compression"],
                                      heads=CFG["heads"], window=CFG["window"], top_k=CFG["top_k"],
                                      seed=1000 * rank + s, device=device, cache=cache, gen_device=str(device)))
    return cache, sets


# ------------------------------------------------------------ CPU baseline
def make_cpu_batch():
    """The config-1 batch built with the CPU oracle encoder (no GPU needed)."""
    from oracle import turboquant as otq
    from aether_kernels.rope import RopeConfig, apply_rope, rope_attention_scale

    g = torch.Generator().manual_seed(4242)
    B, bits = CFG["batch"], CFG["bits"]
    toks = (CFG["ctx_lo"] + torch.randint(0, CFG["ctx_hi"] - CFG["ctx_lo"] + 1, (B,), generator=g)).tolist()
    nbs = [t // 4 for t in toks]
    max_pages = max((n + 63) // 64 for n in nbs)
    total_pages = sum((n + 63) // 64 for n in nbs)
    perm = torch.randperm(total_pages, generator=g)
    table = torch.zeros(B, max_pages, dtype=torch.int32)
    pools = {
        "idx_codes": torch.zeros(total_pages, 64, 64 * bits // 8, dtype=torch.uint8),
        "idx_scale": torch.zeros(total_pages, 64),
        "kv_codes": torch.zeros(total_pages, 64, 128 * bits // 8, dtype=torch.uint8),
        "kv_scale": torch.zeros(total_pages, 64),
    }
    off = 0
    rope = RopeConfig()
    for b, n in enumerate(nbs):
        npg = (n + 63) // 64
        pages = perm[off: off + npg]
        off += npg
        table[b, :npg] = pages.to(torch.int32)
        kv = torch.zeros(npg * 64, 128)
        kv[:n] = apply_rope(torch.randn(n, 128, generator=g), torch.arange(n) * 4 + 3, rope)
        ik = torch.zeros(npg * 64, 64)
        ik[:n] = torch.randn(n, 64, generator=g)
        c, s = otq.encode(kv.view(npg, 64, 128), bits)
        pools["kv_codes"][pages], pools["kv_scale"][pages] = c, s.squeeze(-1)
        c, s = otq.encode(ik.view(npg, 64, 64), bits)
        pools["idx_codes"][pages], pools["idx_scale"][pages] = c, s.squeeze(-1)
    return dict(pools=pools, q=torch.randn(B, CFG["heads"], 128, generator=g).to(torch.bfloat16),
                index_q=torch.randn(B, 4, 64, generator=g), index_weight=torch.randn(B, 4, generator=g),
                sink=torch.randn(CFG["heads"], generator=g),
                window=torch.randn(B, CFG["window"], 128, generator=g).to(torch.bfloat16),
                window_len=torch.full((B,), CFG["window"], dtype=torch.int32), page_table=table,
                nblocks=torch.tensor(nbs, dtype=torch.int32),
                softmax_scale=128 ** -0.5 * rope_attention_scale(rope))


def cpu_decode(bt, rows):
    from oracle import decode as odec

    r = torch.tensor(rows)
    p = bt["pools"]
    return odec.decode_step("csa", bt["q"][r], bt["index_q"][r], bt["index_weight"][r], bt["sink"], bt["window"][r],
                            bt["window_len"][r], p["idx_codes"], p["idx_scale"], p["kv_codes"], p["kv_scale"],
                            bt["page_table"][r], bt["nblocks"][r], CFG["bits"], CFG["top_k"], bt["softmax_scale"],
                            classify_ties=False)


def cpu_predecode(bt, rows):
    """The reference's memoised dequant (aether_2b/serving.py:368-375): each
    sequence's index keys and main entries decoded once, outside the timing."""
    from oracle import decode as odec
    from oracle import turboquant as otq

    p = bt["pools"]
    cache = {}
    for b in rows:
        nb, table = int(bt["nblocks"][b]), bt["page_table"][b]
        keys = otq.decode(odec.gather_pages(p["idx_codes"], table, nb),
                          odec.gather_pages(p["idx_scale"], table, nb).unsqueeze(-1), CFG["bits"], 42)
        main = otq.decode(odec.gather_pages(p["kv_codes"], table, nb),
                          odec.gather_pages(p["kv_scale"], table, nb).unsqueeze(-1), CFG["bits"], 42)
        cache[b] = (keys, main)
    return cache


def cpu_decode_memo(bt, rows, cache):
    """One step of the reference path on already-decoded caches: indexer,
    top-k, gather, sparse sink attention (oracle.decode.decode_step minus the
    dequant)."""
    from oracle import decode as odec

    outs = []
    for b in rows:
        keys, main = cache[b]
        k = min(CFG["top_k"], keys.shape[0])
        s32 = odec.index_scores(bt["index_q"][b].float(), bt["index_weight"][b].float(), keys)
        sel = torch.sort(odec.topk_stable(s32, k)).values
        src = torch.cat([main[sel], bt["window"][b, : int(bt["window_len"][b])].float()], dim=0)
        outs.append(odec.sink_attention(bt["q"][b].float(), src, bt["sink"].float(), bt["softmax_scale"]))
    return torch.stack(outs)


def cpu_baseline(steps: int, warmup: int, budget_s: float, full_line: bool = False, n_gpus: int = 1):
    """The reference's fp32 CPU path on the host cores, two ways: with the
    dequant of every visible block in every step, and with the dequant
    memoised (the reference re-decodes a sequence's cache only when an
    emitted block changes its shape: every 4 tokens for CSA).  ``value`` is
    the steady state of the reference's decode loop: the memoised step plus
    a quarter of the dequant."""
    sys.path.insert(0, str(ROOT))
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    bt = make_cpu_batch()
    B, per_step = CFG["batch"], 4

    def rows_of(i):
        return [(i * per_step + j) % B for j in range(per_step)]

    for i in range(max(warmup, 0)):
        cpu_decode(bt, rows_of(i))
    half = budget_s / 2
    t0 = time.perf_counter()
    n = 0
    while n < max(steps, 1):
        cpu_decode(bt, rows_of(n))
        n += 1
        if time.perf_counter() - t0 > half:
            break
    dt_full = (time.perf_counter() - t0) / n
    # memoised: decode the sample's sequences first (untimed), then the steps
    n_memo_rows = sorted({r for i in range(max(n, 1)) for r in rows_of(i)})
    memo = cpu_predecode(bt, n_memo_rows)
    cpu_decode_memo(bt, rows_of(0), memo)
    t0 = time.perf_counter()
    m = 0
    while m < max(steps, 1):
        cpu_decode_memo(bt, rows_of(m % max(n, 1)), memo)
        m += 1
        if time.perf_counter() - t0 > half:
            break
    dt_memo = (time.perf_counter() - t0) / m
    dt_steady = dt_memo + (dt_full - dt_memo) / 4
    qps = per_step / dt_steady
    base = {"value": round(qps, 2), "unit": UNIT, "cores": threads, "kind": "port",
            "value_dequant_every_step": round(per_step / dt_full, 2),
            "value_memoised_dequant": round(per_step / dt_memo, 2),
            "sample": f"{n * per_step} + {m * per_step} queries ({n} steps with dequant, {m} with memoised dequant, "
                      f"{per_step} sequences of the 64-sequence, 16K-32K-token, 4-bit batch per step); fp32 torch CPU "
                      "restatement of the reference path; value = memoised step + 1/4 of the dequant (re-decode per "
                      "emitted CSA block, every 4 tokens)"}
    if not full_line:
        return base
    # each of the K requested steps is timed twice (with and without the
    # dequant) unless the time budget ends the sample first
    return {"metric": METRIC, "value": round(qps, 2), "unit": UNIT, "n_gpus": n_gpus, "steps": steps,
            "steps_timed": {"dequant_every_step": n, "memoised_dequant": m}, "warmup": warmup,
            "ms_per_step": round(dt_steady * 1e3, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
            "config": {"workload": "csa_decode_4bit_b64_ctx16k-32k", **CFG},
            "cpu_baseline": base,
            "e2e": {"value": round(qps, 2), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


# ------------------------------------------------------------------- main
ATTEND_PHASES = ["keys_rescale_histogram", "select", "compaction", "gather_expand", "qk", "softmax",
                 "pv_merge", "final"]
SCORE_PHASES = ["page_table_tma_issue", "wait_and_index_query_limbs", "page_wait", "scoring"]


def phase_stamps(n, step, err, dev):
    """Median per-CTA phase durations (us) of the two decode kernels over n
    eager steps (no PDL), from the library's SM-clock phase stamps."""
    import ctypes

    import numpy as np
    from aether_kernels import _lib

    lib = _lib.load()
    buf = torch.zeros(65536 + 8 * 8192, dtype=torch.int64, device=dev)
    for i in range(3):
        step(i, False)
    torch.cuda.synchronize()
    khz = getattr(torch.cuda.get_device_properties(dev), "clock_rate", 0)
    if khz:
        mhz = float(khz) / 1000.0
    else:  # max SM clock from nvidia-smi (the stamps count SM cycles)
        out = subprocess.run(["nvidia-smi", "-i", str(dev.index or 0), "--query-gpu=clocks.max.sm",
                              "--format=csv,noheader,nounits"], capture_output=True, text=True).stdout
        mhz = float(out.strip().splitlines()[0])
    att, sco = [], []
    lib.aether_csa_decode_set_debug_timer(ctypes.c_void_p(buf.data_ptr()))
    try:
        for i in range(n):
            buf.zero_()
            torch.cuda.synchronize()
            step(i, False)
            torch.cuda.synchronize()
            a = buf[:65536].view(-1, 16).cpu().numpy().astype(np.float64)
            a = a[(a[:, 2] > 0) & (a[:, 10] > 0)]
            att.append(np.median(np.diff(a[:, 2:11], axis=1), axis=0))
            sc = buf[65536:].view(-1, 8).cpu().numpy().astype(np.float64)
            sc = sc[(sc[:, 0] > 0) & (sc[:, 4] > 0)]
            sco.append(np.median(np.diff(sc[:, :5], axis=1), axis=0))
    finally:
        lib.aether_csa_decode_set_debug_timer(ctypes.c_void_p(0))
    assert int(err.item()) == 0
    ma, ms = np.median(np.array(att), axis=0) / mhz, np.median(np.array(sco), axis=0) / mhz
    return {"phase_stamps_us": {"attend": dict(zip(ATTEND_PHASES, np.round(ma, 3).tolist())),
                                "attend_chain_total": round(float(ma.sum()), 3),
                                "score": dict(zip(SCORE_PHASES, np.round(ms, 3).tolist()))},
            "clock_mhz": mhz, "steps": n, "mode": "eager launches, no PDL"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=102400)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--sets", type=int, default=16)
    ap.add_argument("--e2e-steps", type=int, default=200)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-pdl", dest="pdl", action="store_false",
                    help="launch without programmatic dependent launch (no prefetch overlap across steps)")
    ap.add_argument("--microbatches", type=int, default=1,
                    help="split each step's batch into this many independent micro-batches on separate streams")
    ap.add_argument("--profile-launches", type=int, default=0,
                    help="profiling mode: build the sets, run this many plain launches, print timings, exit")
    ap.add_argument("--phase-stamps", type=int, default=0,
                    help="decode: run N eager steps with the per-CTA SM-clock phase stamps on and print the "
                         "median phase durations (profiling aid; prints no bench line)")
    ap.add_argument("--workload", default="decode", choices=["decode", "prefill", "hca", "long"],
                    help="decode: BASELINE config 1 (the headline); prefill: config 4 chunked prefill; "
                         "hca: config 2 HCA decode; long: config 3 single 262K-token sequence, block range "
                         "split over the ranks (context parallel, NCCL)")
    ap.add_argument("--prefill-requests", type=int, default=8)
    ap.add_argument("--prefill-queries", type=int, default=4096)
    ap.add_argument("--prefill-cached", type=int, default=65536)
    ap.add_argument("--cp-exchange", default="peer", choices=["peer", "nccl"],
                    help="long workload on several GPUs: peer-memory stores or NCCL all-gathers")
    ap.add_argument("--indexer", default="exact", choices=["exact", "fp8"],
                    help="prefill indexer: exact fp16 limbs, or the e4m3 low-precision indexer")
    args = ap.parse_args()
    if args.workload == "prefill":
        run_prefill(args)
        return
    if args.workload == "hca":
        run_hca(args)
        return
    if args.workload == "long":
        run_long(args)
        return

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        if rank == 0:
            print(json.dumps(cpu_baseline(args.steps, args.warmup, budget_s=60.0, full_line=True, n_gpus=world)), flush=True)
        return
    assert args.warmup >= 3, "at least 3 warm-up steps"
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import torch.distributed as dist

        init_nccl(dist, dev)
    from aether_kernels.paged import csa_decode_paged

    cache, sets = build_sets(args.sets, dev, rank)
    B = CFG["batch"]
    outs = [torch.empty(B, CFG["heads"], 128, dtype=torch.bfloat16, device=dev) for _ in sets]
    sels = [torch.empty(B, CFG["top_k"], dtype=torch.int32, device=dev) for _ in sets]
    err = torch.zeros(1, dtype=torch.int32, device=dev)

    mb = args.microbatches
    assert B % mb == 0
    mbs = B // mb
    side = [torch.cuda.Stream(dev) for _ in range(mb)]
    ws = [torch.zeros(max_ws_bytes(mbs), dtype=torch.uint8, device=dev) for _ in range(mb)]

    def launch(i, lo, hi, pdl, w):
        s = sets[i % len(sets)]
        csa_decode_paged(s.q[lo:hi], s.index_q[lo:hi], s.index_weight[lo:hi], s.sink, s.window[lo:hi],
                         s.window_len[lo:hi], cache, s.page_table[lo:hi], s.nblocks[lo:hi], s.softmax_scale,
                         top_k=s.top_k, out=outs[i % len(sets)][lo:hi], indices=sels[i % len(sets)][lo:hi],
                         err=err, overlap_prefetch=pdl, workspace=w)

    def step(i, pdl=args.pdl):
        if mb == 1:
            launch(i, 0, B, pdl, ws[0])
            return
        # independent micro-batches on their own streams (fork / join)
        cur = torch.cuda.current_stream(dev)
        for k in range(mb):
            side[k].wait_stream(cur)
            with torch.cuda.stream(side[k]):
                launch(i, k * mbs, (k + 1) * mbs, pdl, ws[k])
        for k in range(mb):
            cur.wait_stream(side[k])

    if args.phase_stamps:
        print(json.dumps(phase_stamps(args.phase_stamps, step, err, dev)), flush=True)
        return

    if args.profile_launches:
        evs = [torch.cuda.Event(enable_timing=True) for _ in range(args.profile_launches + 1)]
        for i in range(args.warmup):
            step(i, False)
        torch.cuda.synchronize()
        for i in range(args.profile_launches):
            evs[i].record()
            step(i, False)
        evs[-1].record()
        torch.cuda.synchronize()
        print("per-launch ms (plain launches):",
              [round(evs[i].elapsed_time(evs[i + 1]), 4) for i in range(args.profile_launches)], flush=True)
        assert int(err.item()) == 0
        return

    stream = torch.cuda.Stream(dev)
    # exactly args.steps timed steps: whole graphs of per_graph steps, then a
    # graph with the remainder; consecutive steps read different cache sets
    steps = max(1, args.steps)
    per_graph = min(16 * len(sets), steps)
    replays, rem = divmod(steps, per_graph)
    with torch.cuda.stream(stream):
        for i in range(args.warmup):
            step(i)
        stream.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for i in range(per_graph):
                step(i)
        g.replay()
        g_rem = None
        if rem:
            g_rem = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g_rem, stream=stream):
                for i in range(rem):
                    step(i)
            g_rem.replay()
        stream.synchronize()
    assert int(err.item()) == 0, f"kernel error flag {int(err.item())}"

    sampler = ClockSampler(local)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize(dev)
    sampler.start()
    time.sleep(0.2)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        ev0.record(stream)
        for _ in range(replays):
            g.replay()
        if g_rem is not None:
            g_rem.replay()
        ev1.record(stream)
    ev1.synchronize()
    clocks = sampler.stop()
    torch.cuda.synchronize(dev)
    ms = ev0.elapsed_time(ev1)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
        torch.distributed.barrier()
    ms_step = ms / steps
    value = world * B * steps / (ms / 1e3)

    per_set = [algorithmic_bytes(s.nblocks.tolist(), s.window_len.tolist(), CFG["bits"]) for s in sets]
    bytes_launch = sum(per_set) / len(per_set)
    achieved = bytes_launch / (ms_step / 1e3) / 1e9
    peak, peak_src = read_peak()

    # ---- e2e through the public C-ABI with host buffers: every step is one
    # aether_csa_decode_host_plan_step call (CsaDecodeHostPlan.step), which
    # enqueues the copy of that step's packed inputs (q, index q, head
    # weights, window lengths, block counts of the step's cache set) from
    # pinned host memory, the decode, and the copy of the packed output and
    # selected indices back to pinned host memory.
    from aether_kernels.paged import CsaDecodeHostPlan

    # a prepared plan: two staging slots on copy streams, so a step's copies
    # overlap its neighbours' kernels, and one short C call per step
    plan = CsaDecodeHostPlan(cache, B, max(st.page_table.shape[1] for st in sets), CFG["heads"], CFG["top_k"],
                             window=sets[0].window.shape[1], err=err, overlap_prefetch=args.pdl, device=dev)
    host_ins = [plan.pack_inputs(st.q, st.index_q, st.index_weight, st.window_len, st.nblocks) for st in sets]
    host_outs = [plan.new_host_output() for _ in range(2)]
    h2d, d2h = plan.in_bytes, plan.out_bytes

    def e2e_step(i):
        st = sets[i % len(sets)]
        plan.step(host_ins[i % len(sets)], host_outs[i & 1], st.page_table, st.sink, st.window, st.softmax_scale)

    with torch.cuda.stream(stream):
        for i in range(4):
            e2e_step(i)
        plan.fence(wait_for_copies=True)
        stream.synchronize()
        # the host copy of a result matches the device-resident path
        ref_o, ref_s = csa_decode_paged(sets[3].q, sets[3].index_q, sets[3].index_weight, sets[3].sink,
                                        sets[3].window, sets[3].window_len, cache, sets[3].page_table,
                                        sets[3].nblocks, sets[3].softmax_scale, top_k=sets[3].top_k)
        torch.cuda.synchronize(dev)
        ho, hs = plan.unpack_outputs(host_outs[1])
        assert torch.equal(hs, ref_s.cpu()) and torch.equal(ho, ref_o.cpu()), "host-buffer decode differs"
        if world > 1:
            torch.distributed.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        plan.fence(wait_for_copies=False)  # the first input copy starts inside the timed region
        for i in range(args.e2e_steps):
            e2e_step(i)
        plan.fence(wait_for_copies=True)
        e1.record(stream)
    e1.synchronize()
    assert int(err.item()) == 0, f"kernel error flag {int(err.item())}"
    e2e_ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_value = world * B * args.e2e_steps / (e2e_ms / 1e3)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(steps=1000, warmup=1, budget_s=15.0)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world, "steps": steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 6), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "s8+f16", "data": "synthetic",
            "config": {"workload": "csa_decode_4bit_b64_ctx16k-32k", **CFG, "cache_sets": len(sets),
                       "cache_bytes_cycled": int(sum(t.numel() * t.element_size() for t in cache.tensors())),
                       "l2_policy": "inputs larger than L2: each step reads a different cache set, sets > 4x L2",
                       "parallelism": f"request-sharded x{world}", "pdl": bool(args.pdl),
                       "microbatches": args.microbatches,
                       "timing": "CUDA graph replay, CUDA events"},
            "gpu_launches": steps * 2,
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_source": peak_src, "traffic": read_traffic(),
                         "algorithmic_bytes_per_launch": int(bytes_launch)},
            "e2e": {"value": round(e2e_value, 1), "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "clocks": clocks,
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


LONG_METRIC = "CSA 8-bit-KV decode queries/s, one 262K-token sequence (65536 blocks) split over the GPUs"


def run_long(args):
    """batch 1, 262144-token context (65536 compressed
    blocks), 8-bit, YaRN factor 8.  On N ranks each holds a contiguous 1/N of
    the blocks (the window on the last rank): local candidates, NCCL
    all-gather, exact global top-256, attention over the owned winners,
    all-gather of the partials, LSE merge (aether_kernels.dist).  One rank:
    the single-device path (per-chunk top-256, then the top-256 of the chunk
    winners).  Cache sets cycle so every step reads cold HBM.  On N ranks the
    two exchanges are stores into the peers' memory (aether_peer_push /
    aether_peer_wait, PeerContextParallel) and a CUDA graph of the steps is
    replayed; --cp-exchange nccl runs the NCCL all-gather path eagerly."""
    import torch.distributed as dist

    from aether_kernels.dist import PeerContextParallel, csa_decode_context_parallel
    from aether_kernels.paged import PAGE, TurboQuantPagedCache, csa_decode_paged, csa_workspace_bytes
    from aether_kernels.rope import RopeConfig
    from aether_kernels.synthetic import make_decode_batch

    local = int(os.environ.get("LOCAL_RANK", "0"))
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        init_nccl(dist, dev)
    NB, bits = 65536, 8
    assert NB % (world * PAGE) == 0
    per = NB // world
    nsets = 40
    cache = TurboQuantPagedCache(nsets * (NB // PAGE), bits, dev)
    sets, slices = [], []
    for i in range(nsets):
        # identical query and cache contents on every rank (seeded by set)
        st = make_decode_batch("csa", 1, 4 * NB, 4 * NB, bits, 4, seed=500 + i, device=dev,
                               rope=RopeConfig.yarn(8.0), cache=cache, gen_device=str(dev))
        lo = rank * per
        table = st.page_table[:, lo // PAGE: (lo + per) // PAGE].contiguous()
        wl = st.window_len if rank == world - 1 else torch.zeros_like(st.window_len)
        slices.append((table, torch.full_like(st.nblocks, per), wl))
        sets.append(st)
    out = torch.empty(1, 12, 128, dtype=torch.bfloat16, device=dev)
    ws = torch.zeros(csa_workspace_bytes(1, NB), dtype=torch.uint8, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    peer = world > 1 and args.cp_exchange == "peer"
    plan = PeerContextParallel(1, 12, per, 256, device=dev) if peer else None

    def step(i):
        st = sets[i % nsets]
        table, nb, wl = slices[i % nsets]
        if world == 1:
            csa_decode_paged(st.q, st.index_q, st.index_weight, st.sink, st.window, st.window_len, cache, table, nb,
                             st.softmax_scale, out=out, workspace=ws, err=err)
        elif peer:
            plan.step(st.q, st.index_q, st.index_weight, st.sink, st.window, wl, cache, table, nb, rank * per,
                      st.softmax_scale, err=err)
        else:
            csa_decode_context_parallel(st.q, st.index_q, st.index_weight, st.sink, st.window, wl, cache, table, nb,
                                        rank * per, st.softmax_scale, err=err)

    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        for i in range(max(args.warmup, 3)):
            step(i)
    torch.cuda.synchronize(dev)
    assert int(err.item()) == 0, f"kernel error flag {int(err.item())}"
    # one GPU, or the peer exchange: a CUDA graph of nsets steps replayed.
    # The NCCL path runs eagerly (a captured graph holding NCCL collectives
    # left the ranks hanging in process-group teardown)
    graph = None
    if world == 1 or peer:
        if peer:
            dist.barrier()
        try:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                for i in range(nsets):
                    step(i)
            g.replay()
            torch.cuda.synchronize(dev)
            graph = g
        except Exception as exc:  # noqa: BLE001
            print(f"graph capture unavailable ({exc}); eager launches", file=sys.stderr)
    replays = max(1, min(args.steps, 2000) // nsets)
    steps = replays * nsets
    sampler = ClockSampler(local)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    sampler.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for r in range(replays):
            if graph is not None:
                graph.replay()
            else:
                for i in range(nsets):
                    step(i)
        e1.record(stream)
    e1.synchronize()
    clocks = sampler.stop()
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_step = ms / steps
    per_q = algorithmic_bytes([NB], [128], bits)
    achieved = per_q / (ms_step / 1e3) / 1e9
    peak, src = read_peak()
    if rank == 0:
        print(json.dumps({
            "metric": LONG_METRIC, "value": round(steps / (ms / 1e3), 1), "unit": "queries/s", "n_gpus": world,
            "steps": steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 6), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "s8+f16", "data": "synthetic",
            "config": {"workload": "csa_decode_8bit_b1_ctx262k", "nblocks": NB, "blocks_per_gpu": per, "bits": bits,
                       "rope": "yarn x8", "cache_sets": nsets, "parallelism": f"context-parallel x{world}",
                       "l2_policy": "inputs larger than L2: each step reads a different cache set",
                       "exchange": None if world == 1 else args.cp_exchange,
                       "timing": ("CUDA graph replay; CUDA events" if graph is not None
                                  else "eager launches with NCCL; CUDA events")},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": round(peak * world, 1),
                         "unit": "GB/s", "frac": round(achieved / (peak * world), 4), "peak_source": src,
                         "traffic": None, "algorithmic_bytes_per_launch": per_q},
            "clocks": clocks,
        }), flush=True)
    if plan is not None:
        del graph
        plan.close()
    if world > 1:
        dist.destroy_process_group()


HCA_METRIC = "HCA 4-bit-KV decode queries/s at 131K ctx (batch 32/GPU, 1024 blocks)"


def run_hca(args):
    """HCA decode, batch 32, 131072-token contexts (1024
    compressed blocks at compression 128), 4-bit, YaRN factor 4, all visible
    blocks plus the 128-token window.  Steps cycle through cache sets whose
    total exceeds 4x L2; CUDA-graph replay, CUDA events."""
    from aether_kernels.paged import PAGE, TurboQuantPagedCache, hca_decode_paged
    from aether_kernels.rope import RopeConfig
    from aether_kernels.synthetic import make_decode_batch

    local = int(os.environ.get("LOCAL_RANK", "0"))
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import torch.distributed as dist

        init_nccl(dist, dev)
    B, bits, nsets = 32, 4, 240
    pages_per_set = B * (1024 // PAGE)
    cache = TurboQuantPagedCache(nsets * pages_per_set, bits, dev, with_index=False)
    sets = [make_decode_batch("hca", B, 131072, 131072, bits, 128, seed=1000 * rank + i, device=dev,
                              rope=RopeConfig.yarn(4.0), cache=cache, gen_device=str(dev)) for i in range(nsets)]
    outs = [torch.empty(B, 12, 128, dtype=torch.bfloat16, device=dev) for _ in range(nsets)]
    err = torch.zeros(1, dtype=torch.int32, device=dev)

    def step(i):
        s = sets[i % nsets]
        hca_decode_paged(s.q, s.sink, s.window, s.window_len, cache, s.page_table, s.nblocks, s.softmax_scale,
                         out=outs[i % nsets], err=err, overlap_prefetch=args.pdl)

    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        for i in range(max(args.warmup, 3)):
            step(i)
        stream.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for i in range(nsets):
                step(i)
        g.replay()
        stream.synchronize()
    assert int(err.item()) == 0, f"kernel error flag {int(err.item())}"
    replays = max(1, min(args.steps, 20480) // nsets)
    sampler = ClockSampler(local)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize(dev)
    sampler.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for _ in range(replays):
            g.replay()
        e1.record(stream)
    e1.synchronize()
    clocks = sampler.stop()
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    steps = replays * nsets
    ms_step = ms / steps
    per_q = 1024 * (128 * bits // 8 + 4) + 128 * 256 + 12 * 128 * 2 * 2 + 12 * 4 + 4 * (1024 // PAGE)
    achieved = B * per_q / (ms_step / 1e3) / 1e9
    peak, src = read_peak()
    if rank == 0:
        print(json.dumps({
            "metric": HCA_METRIC, "value": round(world * B * steps / (ms / 1e3), 1), "unit": "queries/s",
            "n_gpus": world, "steps": steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 6),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "s8+f16", "data": "synthetic",
            "config": {"workload": "hca_decode_4bit_b32_ctx131k", "batch": B, "nblocks": 1024, "bits": bits,
                       "window": 128, "rope": "yarn x4", "cache_sets": nsets,
                       "cache_bytes_cycled": int(cache.kv_pages.numel()),
                       "l2_policy": "inputs larger than L2: each step reads a different cache set",
                       "timing": "CUDA graph replay, CUDA events"},
            "gpu_launches": steps,
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_source": src,
                         "traffic": read_traffic(NCU_SUMMARY.parent / "hca_decode_4bit_b32_ncu.md"),
                         "algorithmic_bytes_per_launch": B * per_q},
            "clocks": clocks,
        }), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


PREFILL_METRIC = "CSA 4-bit chunked-prefill query tokens/s (8 x 4096-token chunks vs 64K cached)"


def run_prefill(args):
    """R requests, each a chunk of new query tokens against
    cached 4-bit compressed context.  One step = indexer top-256 (tcgen05)
    plus attention for every query token.  Synthetic caches (random codes and
    positive scales), pages in random order; inputs resident in HBM.  The
    roofline is the indexer's algorithmic FLOPs (4 heads x 64 x 2 per visible
    block per query) against the measured bf16 tensor peak."""
    from aether_kernels.paged import TurboQuantPagedCache
    from aether_kernels.prefill import PrefillRequest, _plan, csa_prefill_attend, csa_prefill_topk, query_rows

    local = int(os.environ.get("LOCAL_RANK", "0"))
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import torch.distributed as dist

        init_nccl(dist, dev)
    R, NQ, CACHED, H, bits = args.prefill_requests, args.prefill_queries, args.prefill_cached, 12, 4
    nblk = (CACHED + NQ) // 4
    pages = (nblk + 63) // 64
    g = torch.Generator(device=dev)
    g.manual_seed(1234 + rank)
    cache = TurboQuantPagedCache(R * pages + 8, bits, dev)
    for pool, sc in ((cache.idx_pages, cache.idx_scale), (cache.kv_pages, cache.kv_scale)):
        pool.copy_(torch.randint(0, 256, pool.shape, device=dev, dtype=torch.uint8, generator=g))
        sc.copy_(torch.rand(sc.shape, device=dev, generator=g) * 0.1 + 0.01)
    table = torch.randperm(R * pages + 8, device=dev, generator=g)[: R * pages].to(torch.int32).view(R, pages)
    reqs = [PrefillRequest(r * NQ, NQ, CACHED, nblk) for r in range(R)]
    iq = torch.randn(R * NQ, 4, 64, device=dev, generator=g)
    iw = torch.randn(R * NQ, 4, device=dev, generator=g)
    q = torch.randn(R * NQ, H, 128, device=dev, generator=g).to(torch.bfloat16)
    sink = torch.randn(H, device=dev, generator=g)
    window = torch.randn(R * (NQ + 127), 128, device=dev, generator=g).to(torch.bfloat16)
    first = [r * (NQ + 127) for r in range(R)]
    q_row, vis, wrow, wlen = query_rows(reqs, 4, 128, first, dev)
    plan = _plan(reqs, dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    mid = torch.cuda.Event(enable_timing=True)

    def step():
        keys, ids = csa_prefill_topk(iq, iw, cache, table, reqs, err=err, plan=plan, indexer=args.indexer)
        mid.record()
        return csa_prefill_attend(q, sink, window, wrow, wlen, cache, table, q_row, vis, keys, ids, 128 ** -0.5,
                                  err=err)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    assert int(err.item()) == 0, f"kernel error flag {int(err.item())}"
    steps = max(1, min(args.steps, 20))
    sampler = ClockSampler(local)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize(dev)
    sampler.start()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_idx = t_all = 0.0
    for _ in range(steps):
        e0.record()
        step()
        e1.record()
        e1.synchronize()
        t_all += e0.elapsed_time(e1)
        t_idx += e0.elapsed_time(mid)
    clocks = sampler.stop()
    ms = t_all / steps
    if world > 1:
        t = torch.tensor([ms], device=dev)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        ms = float(t.item())
    vis_sum = sum(min(nblk, (CACHED + i) // 4) for i in range(NQ)) * R
    flops = vis_sum * 4 * 64 * 2
    idx_ms = t_idx / steps
    peak = 1621.8
    pp = ROOT / "MEASURED_PEAKS.json"
    src = "fallback"
    if pp.exists():
        try:
            peak, src = float(json.loads(pp.read_text())["bf16_tflops"]), "measured"
        except Exception:
            pass
    achieved = flops / (idx_ms / 1e3) / 1e12
    if rank == 0:
        print(json.dumps({
            "metric": PREFILL_METRIC, "value": round(world * R * NQ / (ms / 1e3), 1), "unit": "query tokens/s",
            "n_gpus": world, "steps": steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16 limbs / u8 codes" if args.indexer == "exact" else "e4m3 (indexer) / f16",
            "data": "synthetic",
            "config": {"workload": "csa_prefill_4bit", "indexer": args.indexer, "requests": R, "queries_per_request": NQ,
                       "cached_tokens": CACHED, "visible_blocks_max": nblk, "top_k": 256, "heads": H,
                       "timing": "CUDA events per step", "l2_policy": "index caches L2-resident (5 MB)"},
            "gpu_launches": steps * 2,
            "indexer_ms": round(idx_ms, 4), "attention_ms": round(ms - idx_ms, 4),
            "roofline": {"bound": "tensor", "achieved": round(achieved, 2), "peak": peak, "unit": "TFLOP/s",
                         "frac": round(achieved / peak, 4), "peak_source": src, "traffic": None,
                         "algorithmic_flops_per_launch": flops},
            "clocks": clocks,
        }), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
