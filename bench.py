"""Benchmark of the B200 small-q paged attention path (one JSON line on rank 0).

Workload (one "step" = one operator call over one batch): BASELINE config 2,
B=4 sequences x q_len=4 draft tokens x kv_len=8192, fp16, 32 query / 8 KV
heads, head_dim 128, page 16, random pages from a pool of 1.5x the needed
pages.  With N GPUs every rank runs its own batch of 4 (batch sharding,
weak scaling: global batch 4N, no collective on the hot path).

Reported:
* ``value``      effective HBM TB/s of the whole job = algorithmic bytes of all
                 ranks' calls / max-over-ranks device time of K steps, inputs
                 resident in HBM, the K calls replayed from one CUDA graph whose
                 first and last nodes are the timing events (the device time of
                 the K steps, not the host's graph launch), each step on the next
                 of 4 input replicas (805 MB > the 126 MB L2, so K/V always come
                 from HBM);
* ``e2e``        the same metric through the public Python API with the step's
                 query, page table and lengths copied from pinned host memory
                 and the output copied back every step (the KV cache is the
                 serving state and stays resident);
* ``roofline``   the split-KV kernel: algorithmic bytes / its mean duration in a
                 replay of the same K calls, between CUDA events that are graph
                 nodes on side branches (the launches keep their overlap: from the
                 end of the previous call's merge to the end of the split kernel),
                 and beside it with eager launches (an event pair around each, no
                 overlap), against the measured HBM copy bandwidth; ``frac_step``
                 is the whole step (split + merge) against the same peak;
* ``cpu_baseline`` the CPU oracle (numpy restatement of the upstream reference)
                 on the host cores, on a bounded sample of the same workload;
* ``sharded``    cfg3 (KV-head shards), cfg4 (LPT batch shards) and cfg5
                 (long-context split + merge) at this N, strong scaling, device leg;
* ``matrix``     (N=1) the 36-case matrix and the five named configs: graph p50
                 and the upstream's eager per-call p50, TB/s, fraction of peak,
                 the kernel chosen.

``--impl reference`` times the upstream algorithm on the CPU (the oracle port:
the upstream reference is a Python/torch CPU function that does not travel to
the GPU box) on the same workload; rank 0 only.

``--matrix PATH`` instead writes one JSONL row per case of the 36-case matrix
and the five named configurations (slower, 1 s of clock settle per case).
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


class _KernelNames(dict):
    """Kernel id (sqa_selected_kernel) -> name; 2 + 100 * C is the tcgen05 kernel in clusters of C,
    2 + 10000 * k the tcgen05 kernel with every segment split evenly over k CTAs."""

    def __missing__(self, k):
        if k >= 10000:
            return f"sqa_split_kv_tc_kernel (segments split over {(k - 2) // 10000} CTAs each)"
        return f"sqa_split_kv_tc_kernel (clusters of {(k - 2) // 100})" if k > 100 else f"kernel {k}"


def _cluster_mode(kernel_id: int) -> bool:
    """The launch reduces every segment inside its clusters: no merge kernel."""
    return kernel_id > 100 and (kernel_id // 100) % 100 > 0


KERNEL_NAMES = _KernelNames({1: "sqa_split_kv_kernel", 2: "sqa_split_kv_tc_kernel"})
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
    return json.loads(p.read_text()).get(f"{workload}/{KERNEL_NAMES[kernel_id]}")  # measured per build


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
    "cfg5": "cfg5 long-context, strong: B=1, q_len=16, kv_len=262144 split over N GPUs, (O, LSE) to rank 0 by "
            "NVLink peer stores + merge",
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


class DeviceArm:
    """One rank's inputs for a workload and the operator call on them (the C ABI,
    arguments packed once per replica, as a serving loop holds them)."""

    def __init__(self, name, args, world, rank, device, dist, lib):
        import ctypes

        import torch

        from small_q_attention_b200 import _native
        from small_q_attention_b200.attention import _fill_args

        self.name, self.world, self.rank, self.dist, self.lib = name, world, rank, dist, lib
        self.longctx = name == "cfg5"
        self.reps, self.bytes_rank, self.bytes_job = _rank_cases(name, world, rank, device, REPLICAS)
        self.max_len = max(max(r["lens"]) for r in self.reps)
        self.min_len = 0 if args.no_length_hints else min(min(r["lens"]) for r in self.reps)
        self.cargs, self.outs, self.lses = [], [], []
        ws_bytes = 0
        for r in self.reps:
            a = _fill_args(r["query"], r["key_cache"], r["value_cache"], r["block_tables"], r["seq_lens"],
                           r.get("mask_lens"), self.max_len, 0, 0, args.kernel)
            # the serving loop knows its lengths: both bounds steer the launch (cluster mode
            # for near-uniform batches), as a planned step would
            a.min_seq_len = min(r["lens"]) if not args.no_length_hints else 0
            if self.longctx:
                o = torch.empty(r["query"].shape, dtype=torch.float32, device=device)
                l = torch.empty(r["query"].shape[:3], dtype=torch.float32, device=device)
                a.out_partial, a.out_lse = o.data_ptr(), l.data_ptr()
                self.lses.append(l)
            else:
                o = torch.empty_like(r["query"])
                a.out = o.data_ptr()
            self.outs.append(o)
            self.cargs.append(a)
            st = ctypes.c_int(0)
            ws_bytes = max(ws_bytes, lib.sqa_workspace_bytes(ctypes.byref(a), device.index, ctypes.byref(st)))
            _native.check(st.value, "sqa_workspace_bytes")
        self.ws_bytes = ws_bytes
        self.ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=device)
        self.merged = torch.empty(self.reps[0]["query"].shape, dtype=torch.float16, device=device)
        # long-context exchange across ranks: peer stores into rank 0 + its merge (NVLink)
        self.lc = None
        if self.longctx and dist is not None:
            from small_q_attention_b200.sharding import LongContextGroup

            q0 = self.reps[0]["query"]
            self.lc = LongContextGroup(rows=q0.shape[0] * q0.shape[1] * q0.shape[2], device=device)
        self.kernel_id = lib.sqa_selected_kernel(ctypes.byref(self.cargs[0]), device.index)
        if self.kernel_id < 0:
            _native.check(-self.kernel_id, "sqa_selected_kernel")
        # our kernels per step on rank 0: split-KV + per-call merge (none in cluster mode), in
        # long-context mode also the cross-rank merge (one GPU) or the exchange's send + merge
        self.launches_per_step = (1 if _cluster_mode(self.kernel_id) else 2) + (
            (2 if self.lc is not None else 1) if self.longctx else 0)

    def close(self):
        if self.lc is not None:
            self.lc.close()
            self.lc = None

    def call(self, i, stream, ev0=None, ev1=None):
        import ctypes

        import small_q_attention_b200 as sqa
        from small_q_attention_b200 import _native
        lib, a = self.lib, self.cargs[i % REPLICAS]
        if ev0 is None:
            code = lib.sqa_forward(ctypes.byref(a), ctypes.c_void_p(self.ws.data_ptr()),
                                   ctypes.c_size_t(self.ws_bytes), ctypes.c_void_p(stream))
        else:
            code = lib.sqa_forward_timed(ctypes.byref(a), ctypes.c_void_p(self.ws.data_ptr()),
                                         ctypes.c_size_t(self.ws_bytes), ctypes.c_void_p(stream),
                                         ctypes.c_void_p(ev0), ctypes.c_void_p(ev1))
        _native.check(code, "sqa_forward")
        if self.longctx:  # the exchange step: every rank's (O, LSE) merged on rank 0
            j = i % REPLICAS
            if self.lc is not None:
                self.lc.exchange(self.outs[j], self.lses[j], out=self.merged)
            else:
                sqa.merge_partials(self.outs[j][None], self.lses[j][None], out=self.merged)


def measure_device(arm, args, device, with_clocks=True):
    """Device throughput of K steps replayed from one CUDA graph (inputs resident),
    the max over ranks; then the split-KV kernel's own duration, inside a replay
    of the same K calls (events as side-branch graph nodes) and eagerly (an event
    pair per launch)."""
    import torch

    K, W, dist = args.steps, args.warmup, arm.dist
    stream = torch.cuda.Stream(device)
    sh = stream.cuda_stream
    with torch.cuda.stream(stream):
        for i in range(W):
            arm.call(i, sh)
    stream.synchronize()
    # the timing events are nodes of the graph, first and last: the timed region is the K
    # steps on the device, not the host's graph launch before them
    start, end = torch.cuda.Event(enable_timing=True, external=True), torch.cuda.Event(enable_timing=True,
                                                                                        external=True)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        start.record()
        for i in range(K):
            arm.call(i, torch.cuda.current_stream().cuda_stream)
        end.record()
    torch.cuda.synchronize()
    clocks = ClockSampler(device.index) if with_clocks else None
    if clocks:  # sampling from before the warm replays: the sampler's start-up stays out of the timed replay
        clocks.__enter__()
    # warm replays (untimed) so that the timed replay starts at the clock of a busy GPU; the
    # count is the same on every rank (a replay holds cross-rank exchanges)
    t_warm = time.perf_counter()
    graph.replay()
    torch.cuda.synchronize()
    t_first = time.perf_counter() - t_warm
    if arm.lc is not None:  # a cross-rank exchange that timed out anywhere: stop, do not replay it again
        bits = arm.lc.device_status()
        if _max_over_ranks(float(bits), dist, device) != 0:
            raise RuntimeError(f"long-context exchange reported device status bits {bits:#x}")
    n_warm = int(_max_over_ranks(float(math.ceil(0.05 / max(t_first, 1e-4))), dist, device))
    for _ in range(min(n_warm, 50)):
        graph.replay()
    torch.cuda.synchronize()

    try:
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            graph.replay()
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
    finally:
        if clocks:
            clocks.__exit__()
    t_ms = _max_over_ranks(start.elapsed_time(end), dist, device)
    del graph  # holds NCCL work in the long-context mode: release it before the group

    # the split-KV kernel inside a replay of the same K calls: sqa_forward_timed adds its
    # two event-record nodes on side branches of the graph (nothing captured later waits
    # for them), so the launches keep the overlap they have in the timed graph; call k's
    # "before" event fires when call k-1's merge ends (when the split kernel's dependency
    # wait returns), its "after" event when the split kernel ends.  Call 0's "before"
    # event fires at the replay's start, so the mean is over calls 1..K-1.
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    for e0, e1 in evs:  # create the underlying CUDA events
        e0.record(stream)
        e1.record(stream)
    torch.cuda.synchronize()
    kern_graph_ms = step_same_ms = None
    try:
        s2, t2 = torch.cuda.Event(enable_timing=True, external=True), torch.cuda.Event(enable_timing=True,
                                                                                      external=True)
        g2 = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g2, stream=stream):
            s2.record()
            for i, (e0, e1) in enumerate(evs):
                arm.call(i, torch.cuda.current_stream().cuda_stream, e0.cuda_event, e1.cuda_event)
            t2.record()
        torch.cuda.synchronize()
        for _ in range(3):
            g2.replay()
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            g2.replay()
        torch.cuda.synchronize()
        kern_graph_ms = statistics.mean(e0.elapsed_time(e1) for e0, e1 in evs[1:] or evs)
        step_same_ms = s2.elapsed_time(t2) / K
        del g2
    except Exception as e:  # event nodes not capturable here: the eager figure stands alone
        print(f"bench: in-graph kernel timing unavailable ({e})", file=sys.stderr)
    # the same kernel launched eagerly, one event pair per launch
    with torch.cuda.stream(stream):
        for i, (e0, e1) in enumerate(evs):
            arm.call(i, sh, e0.cuda_event, e1.cuda_event)
    torch.cuda.synchronize()
    kern_eager_ms = statistics.mean(e0.elapsed_time(e1) for e0, e1 in evs)
    return {"t_ms": t_ms, "kern_graph_ms": kern_graph_ms, "kern_eager_ms": kern_eager_ms,
            "step_same_ms": step_same_ms, "clocks": clocks.summary() if clocks else None}


def measure_e2e(arm, args, device):
    """The metric end to end through the public Python API with host buffers: each
    step's query, page table and lengths go up from pinned host memory in one
    packed copy and the output comes back (the KV cache is serving state and
    stays resident).  pipelined: the H2D copy runs on a copy stream and may
    overlap the previous step's kernel, the D2H read on a second copy stream after
    the step's kernel (a serving loop's pipeline); serial: all on one stream."""
    import torch

    import small_q_attention_b200 as sqa
    from small_q_attention_b200.sharding import long_context_attention

    K, W, dist = args.steps, args.warmup, arm.dist
    reps, longctx = arm.reps, arm.longctx
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
    stream = torch.cuda.Stream(device)
    s_in, s_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
    ev_in = [torch.cuda.Event() for _ in range(REPLICAS)]
    ev_done = [torch.cuda.Event() for _ in range(REPLICAS)]
    ev_out = [torch.cuda.Event() for _ in range(REPLICAS)]
    pipelined = args.e2e_mode == "pipelined"
    set_stream = torch.cuda.set_stream

    def attend(j):
        d = dev_in[j][1]
        if longctx:
            o = long_context_attention(d["query"], reps[j]["key_cache"], reps[j]["value_cache"],
                                       d["block_tables"], d["seq_lens"], d["mask_lens"], 16, out=e2e_out[j],
                                       workspace=arm.ws, exchange=arm.lc)
            return e2e_out[j] if o is None else o  # ranks > 0 hold no merged output: read back their buffer
        return sqa.small_q_attention(d["query"], reps[j]["key_cache"], reps[j]["value_cache"], d["block_tables"],
                                     d["seq_lens"], 16, arm.max_len, out=e2e_out[j], workspace=arm.ws,
                                     kernel=args.kernel, min_seq_len=arm.min_len)

    def step(i):
        j = i % REPLICAS
        if not pipelined:  # `stream` is current
            dev_in[j][0].copy_(host_in[j], non_blocking=True)
            host_out.copy_(attend(j), non_blocking=True)
            return
        s_in.wait_event(ev_done[j])  # the kernel that last read dev_in[j] has finished
        set_stream(s_in)
        dev_in[j][0].copy_(host_in[j], non_blocking=True)
        ev_in[j].record(s_in)
        set_stream(stream)
        stream.wait_event(ev_in[j])
        stream.wait_event(ev_out[j])  # the D2H that last read e2e_out[j] has finished
        o = attend(j)
        ev_done[j].record(stream)
        s_out.wait_event(ev_done[j])
        set_stream(s_out)
        host_out.copy_(o, non_blocking=True)
        ev_out[j].record(s_out)
        set_stream(stream)

    prev = torch.cuda.current_stream(device)
    set_stream(stream)
    try:
        for i in range(W):
            step(i)
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        s_in.wait_stream(stream)
        for i in range(K):
            step(i)
        for ev in ev_out:
            stream.wait_event(ev)
        e1.record(stream)
        torch.cuda.synchronize()
    finally:
        set_stream(prev)
    e2e_ms = _max_over_ranks(e0.elapsed_time(e1), dist, device)
    return {"e2e_ms": e2e_ms, "h2d": h2d, "d2h": d2h}


def _sharded_line(arm, res, args, peak_gbs):
    K = args.steps
    return {"workload": WORKLOADS[arm.name], "value": round(K * arm.bytes_job / (res["t_ms"] * 1e-3) / 1e12, 4),
            "unit": "TB/s", "us_per_call": round(res["t_ms"] / K * 1e3, 3),
            "algorithmic_bytes_per_call": arm.bytes_job,
            "scaling": "strong", "kernel": KERNEL_NAMES[arm.kernel_id],
            "per_gpu_frac": round(K * arm.bytes_job / (res["t_ms"] * 1e-3) / 1e9 / arm.world / peak_gbs, 4)}


def run_ours(args):
    import torch

    from small_q_attention_b200 import _native

    world, rank, local = _dist()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist = _init_pg(world, "nccl")
    lib = _native.library()
    peak_gbs, peak_src = _peaks()
    name = args.workload
    K, W = args.steps, args.warmup

    arm = DeviceArm(name, args, world, rank, device, dist, lib)
    res = measure_device(arm, args, device)
    t_ms = res["t_ms"]
    value_tbs = K * arm.bytes_job / (t_ms * 1e-3) / 1e12
    kern_bytes = arm.bytes_rank + (2 * 16 * 32 * 128 * 2 if arm.longctx else 0)
    kern_ms = res["kern_graph_ms"] if res["kern_graph_ms"] is not None else res["kern_eager_ms"]
    achieved_gbs = kern_bytes / (kern_ms * 1e-3) / 1e9
    eager_gbs = kern_bytes / (res["kern_eager_ms"] * 1e-3) / 1e9
    e2e = measure_e2e(arm, args, device)
    e2e_tbs = K * arm.bytes_job / (e2e["e2e_ms"] * 1e-3) / 1e12
    arm.close()
    launches = arm.launches_per_step * K
    main_desc = dict(kernel_id=arm.kernel_id, max_len=arm.max_len, q=arm.reps[0]["query"],
                     cache_mb=REPLICAS * arm.reps[0]["key_cache"].numel() * 4 / 1e6, bytes_job=arm.bytes_job)
    del arm
    torch.cuda.empty_cache()

    # the sharded configurations at this N (strong scaling), the device leg only
    sharded = {}
    if not args.no_sharded:
        for sub in ("cfg3", "cfg4", "cfg5"):
            if sub == name:
                continue
            sarm = None
            try:  # a failed sub-measurement is reported in its entry; the line above stands
                sarm = DeviceArm(sub, args, world, rank, device, dist, lib)
                sres = measure_device(sarm, args, device, with_clocks=False)
                sharded[sub] = _sharded_line(sarm, sres, args, peak_gbs)
            except Exception as e:  # noqa: BLE001
                print(f"bench: {sub} failed: {e}", file=sys.stderr)
                sharded[sub] = {"workload": WORKLOADS[sub], "error": f"{type(e).__name__}: {e}"[:300]}
            finally:
                if sarm is not None:
                    try:
                        sarm.close()
                    except Exception as e:  # noqa: BLE001
                        print(f"bench: {sub} close failed: {e}", file=sys.stderr)
                del sarm
                torch.cuda.empty_cache()

    # --- the 36-case matrix and the named configs (N=1 only: it would hold every GPU)
    matrix = None
    if world == 1 and not args.no_matrix:
        matrix = matrix_rows(args, settle=args.settle_line, replica_mb=args.matrix_replica_mb, verbose=False)

    # --- CPU baseline: the oracle on a bounded sample (rank 0, N=1, the cfg2 line only)
    cpu = None
    if rank == 0 and world == 1 and name == "cfg2" and not args.no_cpu_baseline:
        from small_q_attention_b200.workloads import make_config

        c0 = make_config("cfg2", seed=0, device=device)
        times = time_oracle(c0, args.cpu_seconds)
        t = statistics.median(times)
        cpu = {"value": _case_bytes(c0) / t / 1e12, "unit": "TB/s", "cores": _cpu_cores(), "kind": "port",
               "sample": f"{len(times)} whole cfg2 calls (B=4,q=4,kv=8192) of the numpy oracle, "
                         f"median {t * 1e3:.1f} ms/call, {_cpu_model()}"}

    if dist is not None:
        dist.barrier()
    if rank == 0:
        q = main_desc["q"]
        line = {
            "metric": METRIC, "value": round(value_tbs, 4), "unit": "TB/s", "n_gpus": world, "steps": K,
            "warmup": W, "ms_per_step": round(t_ms / K, 6), "higher_is_better": True,
            "scaling": "weak" if name == "cfg2" else "strong",
            "vs_baseline": None, "dtype": "f16 in, f32 accumulate", "data": "synthetic (seeded N(0,1) fp16)",
            "config": {"workload": WORKLOADS[name],
                       "global_batch": (q.shape[0] * world if name == "cfg2" else
                                        {"cfg3": 16, "cfg4": 64, "cfg5": 1}[name]),
                       "seq_len": main_desc["max_len"] if name != "cfg5" else 262144, "q_len": int(q.shape[1]),
                       "parallelism": {"cfg2": f"batch-shard x{world}", "cfg3": f"kv-head-shard x{world}",
                                       "cfg4": f"batch-shard (LPT) x{world}",
                                       "cfg5": f"kv-range split x{world} + NVLink exchange to rank 0"}[name],
                       "l2": f"inputs rotated over {REPLICAS} replicas per GPU "
                             f"({main_desc['cache_mb']:.0f} MB > 126 MB L2)",
                       "us_per_call": round(t_ms / K * 1e3, 3),
                       "algorithmic_bytes_per_call": main_desc["bytes_job"]},
            "roofline": {"bound": "hbm", "achieved": round(achieved_gbs, 1), "peak": peak_gbs, "unit": "GB/s",
                         "frac": round(achieved_gbs / peak_gbs, 4), "peak_source": f"{peak_src} hbm_gbs (burst)",
                         "traffic": _traffic(name, main_desc["kernel_id"]) if world == 1 else None,
                         "kernel": KERNEL_NAMES[main_desc["kernel_id"]],
                         "kernel_us": round(kern_ms * 1e3, 3),
                         "kernel_timing": ("mean over calls 2..K of one replay of the K calls: CUDA events as "
                                           "graph nodes on side branches (launch overlap kept), from the end of "
                                           "the previous call's merge to the end of the split-KV kernel (rank 0)"
                                           if res["kern_graph_ms"] is not None else
                                           "eager launches, one CUDA event pair per launch (rank 0)"),
                         "step_us_same_replay": (round(res["step_same_ms"] * 1e3, 3)
                                                 if res["step_same_ms"] is not None else None),
                         "kernel_us_eager": round(res["kern_eager_ms"] * 1e3, 3),
                         "kernel_eager_def": "eager launches with an event pair on the stream around each "
                                             "(no launch overlap: start-up not hidden behind the previous call)",
                         "frac_eager": round(eager_gbs / peak_gbs, 4),
                         "frac_step": round(value_tbs * 1e3 / world / peak_gbs, 4),
                         "frac_step_def": "algorithmic bytes per GPU / ms_per_step (split-KV + merge kernels, "
                                          "back to back in the timed graph) / peak",
                         "rank": 0},
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_tbs, 4), "unit": "TB/s", "h2d_bytes_per_step": e2e["h2d"],
                    "d2h_bytes_per_step": e2e["d2h"], "us_per_step": round(e2e["e2e_ms"] / K * 1e3, 3),
                    "mode": args.e2e_mode,
                    "api": "small_q_attention_b200.small_q_attention (torch extension over the C ABI)"},
            "clocks": dict(res["clocks"], window="NVML every 2 ms from the warm replays through the timed replay")
            if res["clocks"] else None,
            "gpu_launches": launches,
        }
        if sharded:
            line["sharded"] = sharded
        if matrix is not None:
            line["matrix"] = matrix
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
    ref_gpu = None
    if not args.no_ref_gpu:
        ref_gpu = time_reference_gpu(args, [WORKLOAD])
    if ref_gpu:
        line["reference_gpu_kernel"] = ref_gpu[0]
    print(json.dumps(line), flush=True)
    if args.ref_gpu_matrix:
        rows = time_reference_gpu(args, [n for n, _ in _matrix_cases(args.only)])
        Path(args.ref_gpu_matrix).parent.mkdir(parents=True, exist_ok=True)
        Path(args.ref_gpu_matrix).write_text("".join(json.dumps(r) + "\n" for r in rows))


def time_reference_gpu(args, labels):
    """The upstream's own GPU path on this box: ``forward_v3`` of its CUDA extension
    (``csrc/small_q_attention_ext.cu:1132-1210``, built unmodified for sm_100a by
    ``oracle/build_ref_gpu.py``), chunk_keys 512 and max_seq_len given, as its
    matrix runs it (``scripts/run_gpu_matrix.py:116``), timed with its own protocol
    (``scripts/run_gpu_matrix.py:63-81``: 5 warm-up calls, 15 calls on the same
    inputs, a CUDA event pair and a synchronise around each, median).  A same-box
    comparator reported beside the CPU reference; None when the extension is not
    built or there is no GPU.  q_len 16 is outside its contract (``cuda.py:206-207``)."""
    try:
        import torch

        from oracle import build_ref_gpu

        if not torch.cuda.is_available() or build_ref_gpu.built_module_path() is None:
            return None
        mod = build_ref_gpu.load_module()
    except Exception as e:  # the comparator is optional: report why it is missing
        print(f"bench: upstream GPU extension unavailable ({e})", file=sys.stderr)
        return None
    from small_q_attention_b200.workloads import CONFIGS, make_case, make_config

    torch.cuda.set_device(0)
    rows = []
    for label in labels:
        if label in CONFIGS:
            c = make_config(label, seed=0)
        else:
            q, kv, b = (int(x) for x in label.replace("q", "").replace("kv", "").replace("b", "").split("_"))
            c = make_case(b, q, [kv] * b, pool_factor=1.0, seed=0)
        q_len = c["query"].shape[1]
        if q_len not in (2, 4, 8):
            rows.append({"case": label, "unsupported": "q_len outside the upstream contract (2, 4, 8)"})
            continue
        args_ = (c["query"], c["key_cache"], c["value_cache"], c["block_tables"], c["seq_lens"], 16, 512,
                 max(c["lens"]))
        for _ in range(5):
            mod.forward_v3(*args_)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        samples = []
        for _ in range(15):
            e0.record()
            mod.forward_v3(*args_)
            e1.record()
            e1.synchronize()
            samples.append(e0.elapsed_time(e1) * 1e3)
        us = statistics.median(samples)
        nb = _case_bytes(c)
        rows.append({"case": label, "impl": "upstream forward_v3 (ext.cu:1132-1210), sm_100a build, chunk_keys 512",
                     "p50_us": round(us, 3), "tb_s": round(nb / (us * 1e-6) / 1e12, 4), "alg_bytes": nb,
                     "protocol": "scripts/run_gpu_matrix.py:63-81 (same inputs, event pair + sync per call, "
                                 "median of 15)"})
        del c
        torch.cuda.empty_cache()
    return rows


def _matrix_cases(only=None):
    from small_q_attention_b200.workloads import CONFIGS, matrix_cases

    cases = [(f"q{c['q_len']}_kv{c['kv_len']}_b{c['batch']}", c) for c in matrix_cases()]
    cases += [(n, None) for n in CONFIGS]
    if only:  # config names, "q<N>" for a q_len, or case labels like q16_kv8192_b16
        cases = [(n, c) for n, c in cases if n in only or (c and f"q{c['q_len']}" in only)]
    return cases


def matrix_rows(args, settle: float = 1.0, replica_mb: float = 400.0, verbose: bool = True):
    """Per case of the 36-cell matrix and the five named configs, through the public API:

    * ``p50_us``: CUDA graph of >= 20 back-to-back calls rotating over enough distinct
      input replicas (>= ``replica_mb`` of K/V) that no call finds its pages in L2;
      median over 5 replays; ``tb_s`` / ``roofline_frac`` from it;
    * ``eager_p50_us``: the upstream's protocol (``scripts/run_gpu_matrix.py:63-81``):
      5 warm-up calls, then 15 calls on the same inputs, a CUDA event pair around each
      call and a synchronise after it, median -- comparable cell for cell with the
      upstream's published per-call latencies (the same inputs every call, so small
      cases may be served from L2, as the upstream's were).
    """
    import torch

    import small_q_attention_b200 as sqa
    from small_q_attention_b200.workloads import make_case, make_config

    torch.cuda.set_device(0)
    peak_gbs, peak_src = _peaks()
    rows = []
    ws = torch.zeros(64 << 20, dtype=torch.uint8, device="cuda")  # one workspace for every case

    def make(name, c, seed):
        if c is None:
            return _as_dtype(make_config(name, seed=seed), args.dtype)
        return _as_dtype(make_case(c["batch"], c["q_len"], [c["kv_len"]] * c["batch"], pool_factor=1.0,
                                   page_mode=args.page_mode, seed=seed), args.dtype)

    for label, c in _matrix_cases(args.only):
        first = make(label, c, 0)
        nb = _case_bytes(first)
        cache_bytes = first["key_cache"].numel() * first["key_cache"].element_size() * 2
        n_rep = max(2, min(64, math.ceil(replica_mb * 1e6 / max(1, cache_bytes))))
        inst = [first] + [make(label, c, s_) for s_ in range(1, n_rep)]
        outs = [torch.empty_like(x["query"]) for x in inst]
        min_len = 0 if args.no_length_hints else min(inst[0]["lens"])
        fn = lambda i: sqa.small_q_attention(  # noqa: E731
            inst[i]["query"], inst[i]["key_cache"], inst[i]["value_cache"], inst[i]["block_tables"],
            inst[i]["seq_lens"], 16, max(inst[i]["lens"]), out=outs[i], workspace=ws, kernel=args.kernel,
            min_seq_len=min_len)
        kernel_id = sqa.selected_kernel(inst[0]["query"], inst[0]["key_cache"], inst[0]["value_cache"],
                                        inst[0]["block_tables"], inst[0]["seq_lens"], 16, max(inst[0]["lens"]),
                                        kernel=args.kernel, min_seq_len=min_len)
        for i in range(5):
            fn(i % len(inst))
        torch.cuda.synchronize()
        s = torch.cuda.Stream()
        g = torch.cuda.CUDAGraph()
        reps = max(20, n_rep)  # every replica once per replay
        e0, e1 = torch.cuda.Event(enable_timing=True, external=True), torch.cuda.Event(enable_timing=True,
                                                                                      external=True)
        with torch.cuda.graph(g, stream=s):  # the timing events are the graph's first and last nodes
            e0.record()
            for i in range(reps):
                fn(i % len(inst))
            e1.record()
        g.replay()
        torch.cuda.synchronize()
        # A burst of heavy cases leaves the SM clock low for up to ~2 s afterwards
        # (measured: ~1.1 GHz with no throttle reason reported); let it recover so
        # every case is timed at the same clock, and record the clock per case.
        time.sleep(settle)
        g.replay()
        torch.cuda.synchronize()
        samples = []
        with ClockSampler(torch.cuda.current_device()) as clocks:
            for _ in range(5):
                g.replay()
                torch.cuda.synchronize()
                samples.append(e0.elapsed_time(e1) * 1e3 / reps)
            # the upstream's per-call protocol on replica 0
            for _ in range(5):
                fn(0)
            torch.cuda.synchronize()
            eager = []
            f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            for _ in range(15):
                f0.record()
                fn(0)
                f1.record()
                f1.synchronize()
                eager.append(f0.elapsed_time(f1) * 1e3)
        us = statistics.median(samples)
        eager_us = statistics.median(eager)
        bits = sqa.read_device_status(ws.data_ptr(), clear=True)
        if bits:
            detail = int(ws[4:8].view(torch.int32).item())
            raise RuntimeError(f"{label}: device status bits {bits:#x}, detail {detail:#010x}")
        cs = clocks.summary()
        row = {"case": label, "q_len": inst[0]["query"].shape[1], "batch": inst[0]["query"].shape[0],
               "kv_len_max": max(inst[0]["lens"]), "page_mode": args.page_mode if c else "random",
               "kernel": KERNEL_NAMES[kernel_id], "p50_us": round(us, 3), "min_us": round(min(samples), 3),
               "alg_bytes": nb, "tb_s": round(nb / (us * 1e-6) / 1e12, 4),
               "roofline_frac": round(nb / (us * 1e-6) / 1e9 / peak_gbs, 4),
               "eager_p50_us": round(eager_us, 3), "eager_tb_s": round(nb / (eager_us * 1e-6) / 1e12, 4),
               "peak_gbs": peak_gbs, "peak_source": peak_src, "replicas": n_rep, "sm_mhz": cs["sm_mhz"],
               "clock_reasons": cs["reasons"], "dtype": args.dtype}
        if verbose:
            row["timing"] = (f"p50: CUDA graph of {reps} back-to-back calls over rotating replicas, timed by "
                             "events that are the graph's first and last nodes, median of 5 replays; "
                             "eager: upstream per-call protocol, median of 15")
            print(json.dumps(row), flush=True)
        rows.append(row)
        del g, inst, outs
        torch.cuda.empty_cache()
    return rows


def run_matrix(args):
    rows = matrix_rows(args, settle=args.settle, replica_mb=args.matrix_replica_mb)
    if args.matrix:
        Path(args.matrix).parent.mkdir(parents=True, exist_ok=True)
        Path(args.matrix).write_text("".join(json.dumps(r) + "\n" for r in rows))


def run_kernel_case(args):
    """A few launches of one kernel of the path on a small case (for profiling with ncu
    -k / -c: the same command runs without the profiler first)."""
    import torch

    import small_q_attention_b200 as sqa
    from small_q_attention_b200.workloads import make_case, make_config

    torch.cuda.set_device(0)
    name = args.kernel_case
    if name == "append":  # 64 sequences of 2048 tokens, q_len 4: 2 MB of new K/V per call, 0.5 GB pool
        from small_q_attention_b200.cache import cache_append

        c = make_case(64, 4, [2048] * 64, pool_factor=1.0, seed=0)
        newk = torch.randn(64, 4, 8, 128, dtype=torch.float16, device="cuda")
        newv = torch.randn_like(newk)
        for _ in range(5):
            cache_append(newk, newv, c["key_cache"], c["value_cache"], c["block_tables"], c["seq_lens"])
    elif name == "merge":  # 8 per-GPU partials of cfg5's rows (q16 x 32 heads)
        parts_o = torch.randn(8, 1, 16, 32, 128, device="cuda")
        parts_lse = torch.randn(8, 1, 16, 32, device="cuda")
        out = torch.empty(1, 16, 32, 128, dtype=torch.float16, device="cuda")
        for _ in range(5):
            sqa.merge_partials(parts_o, parts_lse, out=out)
    elif name == "exchange":  # the NVLink exchange's kernels at world 1 (own slot, own merge)
        from small_q_attention_b200.sharding import LongContextGroup

        grp = LongContextGroup(rows=16 * 32)
        o = torch.randn(1, 16, 32, 128, device="cuda")
        lse = torch.randn(1, 16, 32, device="cuda")
        for _ in range(5):
            grp.exchange(o, lse)
        torch.cuda.synchronize()
        if grp.device_status():
            raise RuntimeError("exchange reported a device error")
        grp.close()
    else:  # a split-KV case: cfg2 or a matrix label, through the public API
        if name.startswith("cfg"):
            c = make_config(name, seed=0)
        else:
            q, kv, b = (int(x) for x in name.replace("q", "").replace("kv", "").replace("b", "").split("_"))
            c = make_case(b, q, [kv] * b, pool_factor=1.0, seed=0)
        hint = 0 if args.no_length_hints else min(c["lens"])  # both bounds, as the bench line passes them
        for _ in range(5):
            sqa.small_q_attention(c["query"], c["key_cache"], c["value_cache"], c["block_tables"], c["seq_lens"],
                                  16, max(c["lens"]), kernel=args.kernel, min_seq_len=hint)
    torch.cuda.synchronize()
    print(json.dumps({"kernel_case": name, "ok": True}), flush=True)


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
    ap.add_argument("--e2e-mode", default="pipelined", choices=("pipelined", "serial"),
                    help="e2e: copies on their own streams overlapping the kernels, or all on one stream")
    ap.add_argument("--no-matrix", action="store_true", help="leave the matrix out of the N=1 line")
    ap.add_argument("--no-sharded", action="store_true", help="leave the cfg3/cfg4/cfg5 sub-results out")
    ap.add_argument("--settle-line", type=float, default=0.2,
                    help="matrix inside the driver line: seconds of idle before each case")
    ap.add_argument("--no-ref-gpu", action="store_true",
                    help="--impl reference: leave out the upstream GPU kernel beside the CPU reference")
    ap.add_argument("--ref-gpu-matrix", type=str, default=None,
                    help="--impl reference: also time the upstream GPU kernel on every matrix case, JSONL here")
    ap.add_argument("--no-length-hints", action="store_true",
                    help="do not pass min_seq_len (no cluster mode or segment-aligned split): the cost-balanced "
                         "schedule for every call")
    ap.add_argument("--kernel-case", type=str, default=None,
                    help="run one kernel a few times on a small case (append, merge, exchange, cfg2, q4_kv8192_b4, "
                         "...) for an ncu capture")
    ap.add_argument("--matrix-replica-mb", type=float, default=400.0,
                    help="matrix: MB of distinct K/V replicas rotated per case (>= 126 MB L2)")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.kernel_case:
        run_kernel_case(args)
    elif args.impl == "reference":
        run_reference(args)
    elif args.matrix_only or args.matrix:
        run_matrix(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
