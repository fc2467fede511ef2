"""Benchmark of the B200 small-q paged attention path (one JSON line on rank 0).

Workload (one "step" = one operator call over one batch): BASELINE config 2,
B=4 sequences x q_len=4 draft tokens x kv_len=8192, fp16, 32 query / 8 KV
heads, head_dim 128, page 16, random pages from a pool of 1.5x the needed
pages.  With N GPUs every rank runs its own batch of 4 (batch sharding,
weak scaling: global batch 4N, no collective on the hot path).

Reported:
* ``value``      effective HBM TB/s of the whole job = algorithmic bytes of all
                 ranks' calls / max-over-ranks device time of K steps, inputs
                 resident in HBM, the K calls replayed from one CUDA graph, each
                 step on the next of 4 input replicas (805 MB > the 126 MB L2,
                 so K/V always come from HBM);
* ``e2e``        the same metric through the public Python API with the step's
                 query, page table and lengths copied from pinned host memory
                 and the output copied back every step (the KV cache is the
                 serving state and stays resident);
* ``roofline``   the split-KV kernel alone: algorithmic bytes / its mean
                 CUDA-event duration, against the measured HBM copy bandwidth;
* ``cpu_baseline`` the CPU oracle (numpy restatement of the upstream reference)
                 on the host cores, on a bounded sample of the same workload.

``--impl reference`` times the upstream algorithm on the CPU (the oracle port:
the upstream reference is a Python/torch CPU function that does not travel to
the GPU box) on the same workload; rank 0 only.

``--matrix PATH`` instead writes one JSONL row per case of the 36-case matrix
and the five named configurations (µs/call p50, TB/s, fraction of peak).
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
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "us/call and HBM TB/s (% of peak) over the 36-case matrix; 1/2/4/8 B200"
FALLBACK_HBM_GBS = 6650.0
WORKLOAD = "cfg2"
REPLICAS = 4


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


KERNEL_NAMES = {1: "sqa_split_kv_kernel", 2: "sqa_split_kv_tc_kernel"}
DTYPES = {}  # filled lazily (torch is imported inside the run functions)


def _as_dtype(c, name):
    """A workload dict with its Q/K/V cast to ``name`` ("f16" leaves it as generated)."""
    if name == "f16":
        return c
    import torch

    if name == "fp8":  # fp16 queries, fp8 e4m3 caches
        f8 = torch.float8_e4m3fn
        return dict(c, key_cache=c["key_cache"].to(f8), value_cache=c["value_cache"].to(f8))
    t = {"bf16": torch.bfloat16}[name]
    return dict(c, query=c["query"].to(t), key_cache=c["key_cache"].to(t), value_cache=c["value_cache"].to(t))


def _traffic(workload: str, kernel_id: int):
    """DRAM bytes per split-KV launch of this kernel from the committed ncu summary, if any."""
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None
    return json.loads(p.read_text()).get(f"{workload}/{KERNEL_NAMES[kernel_id]}")


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """Samples SM clock and throttle reasons through NVML in a background thread."""

    REASONS = {
        "gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4, "hw_slowdown": 0x8,
        "sync_boost": 0x10, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40,
        "hw_power_brake_slowdown": 0x80, "display_clock_setting": 0x100,
    }

    def __init__(self, device_index: int, period_s: float = 0.002):
        self.samples, self.reasons = [], 0
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        self.period = period_s
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nv = pynvml
            uuid = None
            try:
                import torch

                uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            except Exception:
                pass
            handle = None
            if uuid:
                for i in range(pynvml.nvmlDeviceGetCount()):
                    h = pynvml.nvmlDeviceGetHandleByIndex(i)
                    u = pynvml.nvmlDeviceGetUUID(h)
                    u = u.decode() if isinstance(u, bytes) else u
                    if u.replace("GPU-", "") == uuid.replace("GPU-", ""):
                        handle = h
                        break
            self._h = handle or pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._nv = None

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                self.reasons |= nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self._nv is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread:
            self._thread.join()

    def summary(self):
        names = sorted(k for k, v in self.REASONS.items() if self.reasons & v)
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "reasons": names, "samples": len(self.samples),
                "source": "nvml" if self._nv else "unavailable"}


# ------------------------------------------------------------------ helpers
def _dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def _init_pg(world, backend):
    import datetime

    import torch.distributed as dist

    if world > 1 and not dist.is_initialized():
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120))
    return dist if world > 1 else None


def _max_over_ranks(x: float, dist, device) -> float:
    if dist is None:
        return x
    import torch

    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _case_bytes(c):
    from small_q_attention_b200.workloads import algorithmic_bytes

    q = c["query"]
    return algorithmic_bytes(q.shape[0], q.shape[1], c["lens"], q.shape[2], c["num_kv_heads"],
                             c["key_cache"].element_size())


def _cpu_cores():
    try:
        from threadpoolctl import threadpool_info

        return max((i.get("num_threads") or 1) for i in threadpool_info()) if threadpool_info() else os.cpu_count()
    except Exception:
        return os.cpu_count()


def _cpu_model():
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except Exception:
        pass
    return "unknown"


def time_oracle(c, budget_s: float, max_calls: int = 50):
    """Time whole oracle calls on the host until ~budget_s has passed."""
    from oracle import paged_mtp_attention_reference

    host = {k: (v.cpu() if hasattr(v, "cpu") else v) for k, v in c.items()}
    args = (host["query"], host["key_cache"], host["value_cache"], host["block_tables"], host["seq_lens"],
            host["page_size"], host["num_kv_heads"])
    paged_mtp_attention_reference(*args)  # warm the BLAS pool
    times = []
    t_end = time.perf_counter() + budget_s
    while len(times) < max_calls and (not times or time.perf_counter() < t_end):
        t0 = time.perf_counter()
        paged_mtp_attention_reference(*args)
        times.append(time.perf_counter() - t0)
    return times


# ------------------------------------------------------------------ arms
WORKLOADS = {
    "cfg2": "cfg2 batch-sharded, weak: B=4 per GPU, q_len=4, kv_len=8192, random pages, pool 1.5x",
    "cfg3": "cfg3 KV-head-sharded, strong: B=16, q_len=8, kv_len=32768, 8/N KV heads per GPU",
    "cfg4": "cfg4 batch-sharded (LPT by tokens), strong: B=64, q_len=4, kv_len U[512,32768], K x4 on 1%",
    "cfg5": "cfg5 long-context, strong: B=1, q_len=16, kv_len=262144 split over N GPUs, (O, LSE) all-gather + merge",
}


def _rank_cases(name, world, rank, device, n_rep):
    """This rank's input replicas for a workload, with its algorithmic bytes per
    step and the whole job's bytes per step."""
    import torch

    from small_q_attention_b200.sharding import kv_head_range, lpt_batch_shards, page_split, shard_lengths
    from small_q_attention_b200.workloads import CONFIGS, algorithmic_bytes, config_lens, make_case, make_config

    if name == "cfg2":
        reps = [make_config("cfg2", seed=1000 * rank + r, device=device) for r in range(n_rep)]
        mine = _case_bytes(reps[0])
        return reps, mine, mine * world
    if name == "cfg3":
        lo, hi = kv_head_range(8, world, rank)
        lens = [32768] * 16
        reps = [make_case(16, 8, lens, hkv=hi - lo, pool_factor=1.0, seed=1000 * rank + r, device=device)
                for r in range(n_rep)]
        return reps, _case_bytes(reps[0]), algorithmic_bytes(16, 8, lens)
    if name == "cfg4":
        lens = config_lens("cfg4")
        mine_idx = lpt_batch_shards(lens, world)[rank]
        my_lens = [lens[i] for i in mine_idx]
        reps = [make_case(len(my_lens), 4, my_lens, pool_factor=1.25, k_outlier_frac=0.01,
                          seed=1000 * rank + r, device=device) for r in range(n_rep)]
        return reps, _case_bytes(reps[0]), algorithmic_bytes(64, 4, lens)
    if name == "cfg5":
        total = CONFIGS["cfg5"]["kv_len"]
        lo, hi = page_split(total // 16, world, rank)
        held, mlen = shard_lengths(total, lo, hi)
        g = torch.Generator(device=device).manual_seed(5)  # the same query on every rank
        q = torch.randn(1, 16, 32, 128, generator=g, device=device, dtype=torch.float16)
        reps = []
        for r in range(n_rep):
            c = make_case(1, 16, [held], pool_factor=1.0, seed=1000 * rank + r, device=device)
            c["query"] = q
            c["mask_lens"] = torch.tensor([mlen], dtype=torch.int32, device=device)
            reps.append(c)
        mine = algorithmic_bytes(1, 16, [held]) - 2 * 16 * 32 * 128 * 2  # K/V + table; Q/O counted once below
        return reps, mine, algorithmic_bytes(1, 16, [total])
    raise ValueError(name)


def run_ours(args):
    import ctypes

    import torch

    import small_q_attention_b200 as sqa
    from small_q_attention_b200 import _native
    from small_q_attention_b200.attention import _fill_args
    from small_q_attention_b200.sharding import gather_partials, long_context_attention

    world, rank, local = _dist()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist = _init_pg(world, "nccl")
    lib = _native.library()
    peak_gbs, peak_src = _peaks()
    name = args.workload
    longctx = name == "cfg5"

    reps, bytes_rank, bytes_job = _rank_cases(name, world, rank, device, REPLICAS)
    max_len = max(max(r["lens"]) for r in reps)
    ws_bytes = 0
    cargs, outs, lses = [], [], []
    for r in reps:
        a = _fill_args(r["query"], r["key_cache"], r["value_cache"], r["block_tables"], r["seq_lens"],
                       r.get("mask_lens"), max_len, 0, 0, args.kernel)
        if longctx:
            o = torch.empty(r["query"].shape, dtype=torch.float32, device=device)
            l = torch.empty(r["query"].shape[:3], dtype=torch.float32, device=device)
            a.out_partial, a.out_lse = o.data_ptr(), l.data_ptr()
            lses.append(l)
        else:
            o = torch.empty_like(r["query"])
            a.out = o.data_ptr()
        outs.append(o)
        cargs.append(a)
        st = ctypes.c_int(0)
        ws_bytes = max(ws_bytes, lib.sqa_workspace_bytes(ctypes.byref(a), local, ctypes.byref(st)))
        _native.check(st.value, "sqa_workspace_bytes")
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=device)
    merged = torch.empty(reps[0]["query"].shape, dtype=torch.float16, device=device)
    kernel_id = lib.sqa_selected_kernel(ctypes.byref(cargs[0]), local)  # what kernel=args.kernel resolves to
    if kernel_id < 0:
        _native.check(-kernel_id, "sqa_selected_kernel")

    def call(i, stream, ev0=None, ev1=None):
        a = cargs[i % REPLICAS]
        if ev0 is None:
            code = lib.sqa_forward(ctypes.byref(a), ctypes.c_void_p(ws.data_ptr()), ctypes.c_size_t(ws_bytes),
                                   ctypes.c_void_p(stream))
        else:
            code = lib.sqa_forward_timed(ctypes.byref(a), ctypes.c_void_p(ws.data_ptr()),
                                         ctypes.c_size_t(ws_bytes), ctypes.c_void_p(stream),
                                         ctypes.c_void_p(ev0), ctypes.c_void_p(ev1))
        _native.check(code, "sqa_forward")
        if longctx:  # the exchange step: gather every rank's (O, LSE), merge on every rank
            j = i % REPLICAS
            if dist is not None:
                parts_o, parts_lse = gather_partials(outs[j], lses[j])
            else:
                parts_o, parts_lse = outs[j][None], lses[j][None]
            sqa.merge_partials(parts_o, parts_lse, out=merged)

    stream = torch.cuda.Stream(device)
    sh = stream.cuda_stream
    K, W = args.steps, args.warmup

    # --- warm-up (eager), then capture exactly K steps in one graph
    with torch.cuda.stream(stream):
        for i in range(W):
            call(i, sh)
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for i in range(K):
            call(i, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    graph.replay()  # warm the graph itself
    torch.cuda.synchronize()

    # --- timed region: K steps, barrier + synchronize on both sides
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()
        start.record(stream)
        with torch.cuda.stream(stream):
            graph.replay()
        end.record(stream)
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
    t_ms = _max_over_ranks(start.elapsed_time(end), dist, device)
    value_tbs = K * bytes_job / (t_ms * 1e-3) / 1e12
    del graph  # holds NCCL work in the long-context mode: release before the group

    # --- roofline: the split-KV kernel alone, one event pair per launch (this rank)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    for e0, e1 in evs:  # create the underlying CUDA events
        e0.record(stream)
        e1.record(stream)
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        for i, (e0, e1) in enumerate(evs):
            call(i, sh, e0.cuda_event, e1.cuda_event)
    torch.cuda.synchronize()
    kern_ms = statistics.mean(e0.elapsed_time(e1) for e0, e1 in evs)
    kern_bytes = bytes_rank + (2 * 16 * 32 * 128 * 2 if longctx else 0)
    achieved_gbs = kern_bytes / (kern_ms * 1e-3) / 1e9

    # --- e2e through the public API with host buffers: the step's small inputs
    # (Q, page table, lengths) go up in one pinned copy, the output comes back
    small = ("query", "block_tables", "seq_lens") + (("mask_lens",) if longctx else ())

    def _packed(r, pin):
        """One uint8 buffer holding the step's small inputs back to back (256-B aligned) + typed views."""
        sizes = [r[k].numel() * r[k].element_size() for k in small]
        offs, total = [], 0
        for n in sizes:
            offs.append(total)
            total += (n + 255) // 256 * 256
        buf = torch.empty(total, dtype=torch.uint8, pin_memory=pin, device="cpu" if pin else device)
        views = {k: buf[o:o + n].view(r[k].dtype).view(r[k].shape) for k, o, n in zip(small, offs, sizes)}
        return buf, views

    host_in, dev_in = [], []
    for r in reps:
        hb, hv = _packed(r, True)
        for k in small:
            hv[k].copy_(r[k].cpu())
        db, dv = _packed(r, False)
        host_in.append(hb)
        dev_in.append((db, dv))
    host_out = torch.empty(reps[0]["query"].shape, dtype=torch.float16, pin_memory=True)
    h2d = host_in[0].numel()
    d2h = host_out.numel() * host_out.element_size()
    e2e_out = [torch.empty_like(r["query"]) for r in reps]

    # A serving loop's pipeline: each step's H2D copy runs on a copy stream and may
    # overlap the previous step's kernel; the step's D2H read runs on a second copy
    # stream after its kernel.  Every step's copies are inside the timed region.
    s_in, s_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
    ev_in = [torch.cuda.Event() for _ in range(REPLICAS)]
    ev_done = [torch.cuda.Event() for _ in range(REPLICAS)]
    ev_out = [torch.cuda.Event() for _ in range(REPLICAS)]

    def e2e_step(i):
        j = i % REPLICAS
        s_in.wait_event(ev_done[j])  # the kernel that last read dev_in[j] has finished
        with torch.cuda.stream(s_in):
            dev_in[j][0].copy_(host_in[j], non_blocking=True)
            ev_in[j].record(s_in)
        stream.wait_event(ev_in[j])
        stream.wait_event(ev_out[j])  # the D2H that last read e2e_out[j] has finished
        d = dev_in[j][1]
        # `stream` is the current stream for the whole loop (set once below)
        if longctx:
            o = long_context_attention(d["query"], reps[j]["key_cache"], reps[j]["value_cache"],
                                       d["block_tables"], d["seq_lens"], d["mask_lens"], 16, out=e2e_out[j],
                                       workspace=ws)
        else:
            o = sqa.small_q_attention(d["query"], reps[j]["key_cache"], reps[j]["value_cache"],
                                      d["block_tables"], d["seq_lens"], 16, max_len, out=e2e_out[j],
                                      workspace=ws, kernel=args.kernel)
        ev_done[j].record(stream)
        s_out.wait_event(ev_done[j])
        with torch.cuda.stream(s_out):
            host_out.copy_(o, non_blocking=True)
            ev_out[j].record(s_out)

    with torch.cuda.stream(stream):
        for i in range(W):
            e2e_step(i)
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        s_in.wait_stream(stream)
        for i in range(K):
            e2e_step(i)
        for ev in ev_out:
            stream.wait_event(ev)
        e1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = _max_over_ranks(e0.elapsed_time(e1), dist, device)
    e2e_tbs = K * bytes_job / (e2e_ms * 1e-3) / 1e12

    # --- CPU baseline: the oracle on a bounded sample (rank 0, N=1, the cfg2 line only)
    cpu = None
    if rank == 0 and world == 1 and name == "cfg2" and not args.no_cpu_baseline:
        times = time_oracle(reps[0], args.cpu_seconds)
        t = statistics.median(times)
        cpu = {"value": bytes_rank / t / 1e12, "unit": "TB/s", "cores": _cpu_cores(), "kind": "port",
               "sample": f"{len(times)} whole cfg2 calls (B=4,q=4,kv=8192) of the numpy oracle, "
                         f"median {t * 1e3:.1f} ms/call, {_cpu_model()}"}

    if dist is not None:
        dist.barrier()
    if rank == 0:
        q = reps[0]["query"]
        line = {
            "metric": METRIC, "value": round(value_tbs, 4), "unit": "TB/s", "n_gpus": world, "steps": K,
            "warmup": W, "ms_per_step": round(t_ms / K, 6), "higher_is_better": True,
            "scaling": "weak" if name == "cfg2" else "strong",
            "vs_baseline": None, "dtype": "f16 in, f32 accumulate", "data": "synthetic (seeded N(0,1) fp16)",
            "config": {"workload": WORKLOADS[name],
                       "global_batch": (q.shape[0] * world if name == "cfg2" else
                                        {"cfg3": 16, "cfg4": 64, "cfg5": 1}[name]),
                       "seq_len": max_len if name != "cfg5" else 262144, "q_len": int(q.shape[1]),
                       "parallelism": {"cfg2": f"batch-shard x{world}", "cfg3": f"kv-head-shard x{world}",
                                       "cfg4": f"batch-shard (LPT) x{world}",
                                       "cfg5": f"kv-range split x{world} + NCCL all-gather"}[name],
                       "l2": f"inputs rotated over {REPLICAS} replicas per GPU "
                             f"({REPLICAS * reps[0]['key_cache'].numel() * 4 / 1e6:.0f} MB > 126 MB L2)",
                       "us_per_call": round(t_ms / K * 1e3, 3),
                       "algorithmic_bytes_per_call": bytes_job},
            "roofline": {"bound": "hbm", "achieved": round(achieved_gbs, 1), "peak": peak_gbs, "unit": "GB/s",
                         "frac": round(achieved_gbs / peak_gbs, 4), "peak_source": f"{peak_src} hbm_gbs (burst)",
                         "traffic": _traffic(name, kernel_id) if world == 1 else None,
                         "kernel": KERNEL_NAMES[kernel_id],
                         "kernel_us": round(kern_ms * 1e3, 3), "rank": 0},
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_tbs, 4), "unit": "TB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "us_per_step": round(e2e_ms / K * 1e3, 3)},
            "clocks": clocks.summary(),
            "gpu_launches": (3 if longctx else 2) * K,
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def _oracle_sample(c, level):
    """The workload restricted to a bounded sample: level 0 = the whole batch,
    1 = one sequence (all 8 KV heads), 2 = one sequence and one KV head."""
    if level == 0:
        return c
    d = dict(c)
    d["query"], d["block_tables"], d["seq_lens"] = c["query"][:1], c["block_tables"][:1], c["seq_lens"][:1]
    d["lens"] = c["lens"][:1]
    if level == 2:
        d["query"] = d["query"][:, :, :4].contiguous()
        d["key_cache"] = c["key_cache"][:, :, :1]
        d["value_cache"] = c["value_cache"][:, :, :1]
        d["num_kv_heads"] = 1
    return d


def run_reference(args):
    world, rank, _ = _dist()
    if rank != 0:
        return
    import torch

    from oracle import paged_mtp_attention_reference
    from small_q_attention_b200.workloads import CONFIGS, algorithmic_bytes, make_config

    c = make_config(WORKLOAD, seed=0, device="cpu", gen_device="cpu")
    cfg = CONFIGS[WORKLOAD]

    def one(d):
        paged_mtp_attention_reference(d["query"], d["key_cache"], d["value_cache"], d["block_tables"],
                                      d["seq_lens"], 16, d["num_kv_heads"])

    # pick the largest sample whose K + W steps fit the time budget
    level, d = 0, c
    for level in range(3):
        d = _oracle_sample(c, level)
        one(d)
        t0 = time.perf_counter()
        one(d)
        est = (time.perf_counter() - t0) * (args.steps + args.warmup)
        if est <= args.reference_budget_s:
            break
    q = d["query"]
    nbytes = algorithmic_bytes(q.shape[0], q.shape[1], d["lens"], q.shape[2], d["num_kv_heads"])
    for _ in range(args.warmup):
        one(d)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        one(d)
    dt = time.perf_counter() - t0
    v = args.steps * nbytes / dt / 1e12
    cores = _cpu_cores()
    sample = ["whole call (B=4, 8 KV heads)", "one sequence of the batch (8 KV heads)",
              "one sequence, one KV head"][level]
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "TB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32 (CPU oracle)",
        "data": "synthetic (seeded N(0,1) fp16, upcast to fp32)",
        "config": {"workload": f"{WORKLOAD}: B={cfg['batch']}, q_len={cfg['q_len']}, kv_len={cfg['kv_len']}",
                   "global_batch": cfg["batch"], "seq_len": cfg["kv_len"], "parallelism": "cpu, rank 0 only"},
        "cpu_baseline": {"value": v, "unit": "TB/s", "cores": cores, "kind": "port",
                         "sample": f"each step = {sample} of {WORKLOAD}, numpy restatement of "
                                   f"reference.py:10-74 ({_cpu_model()}, torch {torch.__version__})"},
        "e2e": {"value": v, "unit": "TB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_matrix(args):
    """Per-case p50 µs/call and TB/s over the 36-case matrix and the named configs."""
    import torch

    import small_q_attention_b200 as sqa
    from small_q_attention_b200.workloads import CONFIGS, make_case, make_config, matrix_cases

    torch.cuda.set_device(0)
    DTYPES.update({"f16": torch.float16, "bf16": torch.bfloat16})
    peak_gbs, peak_src = _peaks()
    rows = []
    # one explicit workspace, large enough for every case (16 KV-head segments x 64 rows worst case)
    ws = torch.zeros(64 << 20, dtype=torch.uint8, device="cuda")
    cases = [("matrix", c) for c in matrix_cases()] + [(n, None) for n in CONFIGS]
    if args.only:  # config names, "q<N>" for a q_len, or case labels like q16_kv8192_b16
        def label_of(n, c):
            return n if c is None else f"q{c['q_len']}_kv{c['kv_len']}_b{c['batch']}"
        cases = [(n, c) for n, c in cases
                 if label_of(n, c) in args.only or (c and f"q{c['q_len']}" in args.only)]
    for name, c in cases:
        if c is None:
            first = _as_dtype(make_config(name, seed=0), args.dtype)
            label = name
        else:
            first = _as_dtype(make_case(c["batch"], c["q_len"], [c["kv_len"]] * c["batch"], pool_factor=1.0,
                                        page_mode=args.page_mode, seed=0), args.dtype)
            label = f"q{c['q_len']}_kv{c['kv_len']}_b{c['batch']}"
        nb = _case_bytes(first)
        # distinct input copies so that consecutive calls never find K/V in L2:
        # at least 2 and enough for >= 400 MB of caches in rotation (at most 64)
        cache_bytes = first["key_cache"].numel() * first["key_cache"].element_size() * 2
        n_rep = max(2, min(64, math.ceil(400e6 / max(1, cache_bytes))))
        inst = [first]
        for s_ in range(1, n_rep):
            if c is None:
                inst.append(_as_dtype(make_config(name, seed=s_), args.dtype))
            else:
                inst.append(_as_dtype(make_case(c["batch"], c["q_len"], [c["kv_len"]] * c["batch"], pool_factor=1.0,
                                                page_mode=args.page_mode, seed=s_), args.dtype))
        outs = [torch.empty_like(x["query"]) for x in inst]
        fn = lambda i: sqa.small_q_attention(  # noqa: E731
            inst[i]["query"], inst[i]["key_cache"], inst[i]["value_cache"], inst[i]["block_tables"],
            inst[i]["seq_lens"], 16, max(inst[i]["lens"]), out=outs[i], workspace=ws, kernel=args.kernel)
        for i in range(5):
            fn(i % len(inst))
        torch.cuda.synchronize()
        s = torch.cuda.Stream()
        g = torch.cuda.CUDAGraph()
        reps = max(20, n_rep)  # every replica once per replay
        with torch.cuda.graph(g, stream=s):
            for i in range(reps):
                fn(i % len(inst))
        g.replay()
        torch.cuda.synchronize()
        # A burst of heavy cases leaves the SM clock low for up to ~2 s afterwards
        # (measured: ~1.1 GHz with no throttle reason reported); let it recover so
        # every case is timed at the same clock, and record the clock per case.
        time.sleep(args.settle)
        g.replay()
        torch.cuda.synchronize()
        samples = []
        with ClockSampler(torch.cuda.current_device()) as clocks:
            for _ in range(5):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                g.replay()
                e1.record()
                torch.cuda.synchronize()
                samples.append(e0.elapsed_time(e1) * 1e3 / reps)
        us = statistics.median(samples)
        bits = sqa.read_device_status(ws.data_ptr(), clear=True)
        if bits:
            detail = int(ws[4:8].view(torch.int32).item())
            raise RuntimeError(f"{label}: device status bits {bits:#x}, detail {detail:#010x}")
        row = {"case": label, "q_len": inst[0]["query"].shape[1], "batch": inst[0]["query"].shape[0],
               "kv_len_max": max(inst[0]["lens"]), "page_mode": args.page_mode if c else "random",
               "p50_us": round(us, 3), "min_us": round(min(samples), 3), "alg_bytes": nb,
               "tb_s": round(nb / (us * 1e-6) / 1e12, 4),
               "roofline_frac": round(nb / (us * 1e-6) / 1e9 / peak_gbs, 4), "peak_gbs": peak_gbs,
               "peak_source": peak_src, "n_gpus": 1, "replicas": n_rep, "kernel": args.kernel,
               "sm_mhz": clocks.summary()["sm_mhz"], "clock_reasons": clocks.summary()["reasons"],
               "dtype": args.dtype,
               "timing": f"CUDA graph of {reps} back-to-back calls over rotating replicas, median of 5"}
        rows.append(row)
        print(json.dumps(row), flush=True)
        del g, inst, outs
        torch.cuda.empty_cache()
    if args.matrix:
        Path(args.matrix).parent.mkdir(parents=True, exist_ok=True)
        Path(args.matrix).write_text("".join(json.dumps(r) + "\n" for r in rows))


def main():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", choices=tuple(WORKLOADS), default="cfg2",
                    help="cfg2 (default, the driver's line) or a sharded configuration")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--reference-budget-s", type=float, default=150.0)
    ap.add_argument("--matrix", type=str, default=None, help="write the per-case matrix JSONL here")
    ap.add_argument("--matrix-only", action="store_true", help="run only the matrix sweep")
    ap.add_argument("--only", nargs="*", default=None)
    ap.add_argument("--page-mode", default="random", choices=("random", "unique", "shared"))
    ap.add_argument("--dtype", default="f16", choices=("f16", "bf16", "fp8"),
                    help="matrix: element type of Q/K/V (fp8: fp16 Q, fp8 e4m3 K/V; the driver line is always f16)")
    ap.add_argument("--settle", type=float, default=1.0,
                    help="matrix: seconds of idle before timing each case (clock recovery)")
    ap.add_argument("--kernel", type=int, default=0, choices=(0, 1, 2),
                    help="0 auto, 1 warp-level mma.sync kernel, 2 tcgen05 kernel")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.impl == "reference":
        run_reference(args)
    elif args.matrix_only or args.matrix:
        run_matrix(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
