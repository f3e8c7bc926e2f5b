"""Decode-attention + KV-append throughput of the paged KV engine.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload scaleout|batched16|churn|headsplit|backbone]

One process per GPU (torchrun for N > 1).  A step is one decode step of every
slot on the rank: for each of the 36 layers, the RoPE + K/V append of one row
per slot and the GQA decode attention over each slot's whole context, issued
as hkv_decode_step (one kernel launch per layer), then the length advance.

Workloads (synthetic N(0,1) data, random physical page order):
  scaleout   (default) the per-GPU share of the 8xB200 scale-out config:
             32 slots per GPU, contexts uniform in [2048, 16384] (seeded per
             rank), so N GPUs run 32N slots (weak scaling, no collective).
  batched16  16 slots, contexts uniform in [256, 4096], one GPU.
  churn      64 slots in 8 groups sharing a 768-token prefix (copy-on-write);
             slots finish with p=0.01 per step and are replaced at once.
  headsplit  one request near the 32768-position context, split by KV head
             over the N GPUs with an NCCL all-gather per layer.
  backbone   the whole 36-layer Q4_K backbone decode step (the projections,
             norms and output head around the KV path) at batch 1, or with
             --batch B for B requests per step (hkv_backbone_decode with
             max_batch B: the projections run on the tensor cores): a
             1024-token prompt, then greedy steps.

Reported: `value` = tokens/s over all ranks (slots advanced one position
through all 36 layers per second), device-timed with CUDA events, max over
ranks, inputs resident in HBM (the KV read per step, tens of GB, is far
larger than the 126 MB L2, so no flush is needed); `e2e` = the same metric
through the C ABI with q/k/v copied in from pinned host memory and the
attention outputs copied back (one copy each way per 9 layers) every step;
`roofline` of the attention kernel (live per-launch CUDA events); `cpu_baseline` = the reference's F32 GGML
decode graph restated in C (oracle/hkv_oracle_graph.c) on a bounded sample.
The default one-GPU run adds short legs to its line: `headsplit` (one
request near 32768 positions), and `batched16`, `backbone_batch1` and
`backbone_batch16` (those workloads run as child processes on the same GPU,
each reported with its own roofline, e2e and clocks).
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO / "higgs-audio.cpp_b200"))

H, G, D = 32, 8, 128
N_LAYERS = 36  # --layers overrides it for small profiler captures (same per-launch sizes)
METRIC = "decode-attn+KV-append tokens/s (all slots), % of HBM peak, at 1/2/4/8 B200"
HBM_FALLBACK_GBS = 6650.0


def measured_peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return HBM_FALLBACK_GBS, "fallback"


SCALEOUT_REQUESTS, SCALEOUT_GPUS = 256, 8


def scaleout_population():
    """The scale-out config's 256 requests: contexts uniform in [2048, 16384]
    (seed 1000), placed on 8 GPUs in balanced shards of 32 (equal request
    counts, nearly equal total context)."""
    import synth
    from hkv_dist import balanced_shards
    pop = [int(x) for x in synth.uniform_int(1000, SCALEOUT_REQUESTS, 2048, 16384)]
    return pop, balanced_shards(pop, SCALEOUT_GPUS)


def workload(name: str, rank: int, prefix: int = 768):
    import synth
    if name == "scaleout":
        if rank >= SCALEOUT_GPUS:
            raise SystemExit(f"the scale-out workload has {SCALEOUT_GPUS} shards")
        pop, shards = scaleout_population()
        lens = [pop[i] for i in shards[rank]]
        desc = ("scale-out shard: 32 slots per GPU (shard %d of the 256-request population, "
                "contexts U[2048,16384], balanced placement), 36 layers, F16 KV in 16-token "
                "pages (permuted), GQA 32/8, head_dim 128" % rank)
    elif name == "headsplit":
        n = 1
        lens = [32768 - 16]
        desc = ("one request near the 32768-position context, split by KV head, 36 layers, "
                "F16 KV in 16-token pages")
    elif name == "churn":
        n = 64
        lens = synth.uniform_int(3000 + rank, n, prefix + 1, 8192)
        desc = (f"slot churn with prefix sharing: 64 slots in 8 groups sharing a {prefix}-token "
                "prefix (copy-on-write pages), contexts U[prefix+1, 8192], each slot finishes "
                "with p=0.01 per step and is replaced at once, 36 layers, F16 KV")
    elif name == "batched16":
        n = 16
        lens = synth.uniform_int(2000 + rank, n, 256, 4096)
        desc = ("batched paged decode: 16 slots, contexts U[256,4096], 36 layers, F16 KV in "
                "16-token pages (permuted), GQA 32/8, head_dim 128")
    else:
        raise SystemExit(f"unknown workload {name}")
    return [int(x) for x in lens], desc


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """SM clock and clock-event (throttle) reasons sampled during the timed
    region: NVML read-only queries from a thread every ~5 ms (the timed region
    can be well under a second).  Nothing here changes a GPU setting."""

    REASONS = {"hw_slowdown": "HwSlowdown", "hw_thermal_slowdown": "HwThermalSlowdown",
               "sw_thermal_slowdown": "SwThermalSlowdown", "sw_power_cap": "SwPowerCap"}

    def __init__(self, device: int):
        self.device = device
        self.samples = []
        self.thread = None
        self.stop_flag = False
        self.handle = None
        self.max_mhz = None

    def _nvml_handle(self):
        import pynvml
        import torch
        pynvml.nvmlInit()
        uuid = str(torch.cuda.get_device_properties(self.device).uuid)
        for cand in (uuid, "GPU-" + uuid):
            try:
                return pynvml.nvmlDeviceGetHandleByUUID(cand)
            except Exception:
                pass
        return pynvml.nvmlDeviceGetHandleByIndex(self.device)

    def start(self):
        import threading
        try:
            import pynvml
            self.handle = self._nvml_handle()
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.handle = None
            return
        masks = {}
        for key, name in self.REASONS.items():
            masks[key] = getattr(pynvml, "nvmlClocksEventReason" + name,
                                 getattr(pynvml, "nvmlClocksThrottleReason" + name, 0))

        def loop():
            import time as _t
            while not self.stop_flag:
                try:
                    mhz = pynvml.nvmlDeviceGetClockInfo(self.handle, pynvml.NVML_CLOCK_SM)
                    try:
                        bits = pynvml.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
                    except Exception:
                        bits = pynvml.nvmlDeviceGetCurrentClocksThrottleReasons(self.handle)
                    self.samples.append((mhz, [k for k, m in masks.items() if bits & m]))
                except Exception:
                    break
                _t.sleep(0.005)

        self.thread = threading.Thread(target=loop, daemon=True)
        self.thread.start()

    def stop(self):
        if self.thread is None:
            return None
        self.stop_flag = True
        self.thread.join(timeout=5)
        if not self.samples:
            return None
        mhz = [m for m, _ in self.samples]
        reasons = sorted({r for _, rs in self.samples for r in rs})
        return {"sm_mhz": float(np.median(mhz)), "sm_max_mhz": float(self.max_mhz),
                "reasons": reasons, "samples": len(self.samples), "source": "nvml"}


# ----------------------------------------------------------- CPU baseline
def cpu_complete_steps(groups, budget_s: float, max_steps: int):
    """Complete decode steps of a whole workload on the host cores: the
    reference's F32 decode graph restated in C (oracle/hkv_oracle_graph.c:
    F32 cache, materialised GQA repeat, QK, scale, softmax, permuted V, PV),
    one graph per slot and layer as the reference runs requests, every slot
    at its real context, all N_LAYERS layers per step, contexts growing by
    one per step.  `groups` holds the slots' contexts in groups of at most 32
    (one per GPU shard); the groups run one after another through one
    group-sized F32 cache of one layer, which the layers and groups share
    (host memory holds one group's contexts for one layer).  Every pass reads
    it from DRAM -- gigabytes, far beyond any CPU cache -- so the traffic is
    that of distinct caches.  Times at least one complete step and stops
    before the next one would end past budget_s or max_steps."""
    sys.path.insert(0, str(REPO / "oracle"))
    import cpu_oracle
    cpu_oracle.build()
    cores = cpu_oracle.max_threads()
    width = max(len(g) for g in groups)
    cap = max(max(g) for g in groups) + max_steps + 2
    base = cpu_oracle.GraphBaseline(width, cap, fill_seed=7)
    rng = np.random.default_rng(0)
    q = rng.standard_normal((N_LAYERS, width, H, D), dtype=np.float32)
    k = rng.standard_normal((N_LAYERS, width, G, D), dtype=np.float32)
    v = rng.standard_normal((N_LAYERS, width, G, D), dtype=np.float32)
    past = [np.array(g, np.int32) for g in groups]
    m0 = len(groups[0])
    base.decode_layer(q[0, :m0], k[0, :m0], v[0, :m0], past[0])  # first touch of the scratch
    t0 = time.perf_counter()
    per_step = []
    while len(per_step) < max_steps:
        ts = time.perf_counter()
        for p in past:
            m = len(p)
            for layer in range(N_LAYERS):
                base.decode_layer(q[layer, :m], k[layer, :m], v[layer, :m], p)
            p += 1
        per_step.append(time.perf_counter() - ts)
        if time.perf_counter() - t0 + per_step[-1] > budget_s:
            break
    total = float(sum(per_step))
    n_slots = sum(len(g) for g in groups)
    steps = len(per_step)
    return {
        "value": steps * n_slots / total, "unit": "tokens/s", "cores": cores, "kind": "port",
        "steps_timed": steps, "step_s": total / steps,
        "sample": (f"{steps} complete step(s) of the whole workload: {n_slots} slots at their "
                   f"real contexts x {N_LAYERS} layers per step, {total:.1f} s on {cores} "
                   f"threads (F32 cache, materialised GQA repeat, one graph per slot and layer)"),
    }


def run_config(name: str, world: int, lens_all, lens_rank0, desc: str, extra=None) -> dict:
    """The `config` of a run's JSON line; both arms print the same one."""
    gb = N_LAYERS * sum(4096 * L + 45056 for L in lens_rank0) / 1e9
    cfg = {
        "workload": desc,
        "slots_per_gpu": len(lens_rank0),
        "global_batch": len(lens_all),
        "layers": N_LAYERS,
        "mean_context": float(np.mean(lens_all)),
        "seq_len": "per-slot contexts, see workload",
        "parallelism": f"slot-sharded x{world} (no collective)",
        "l2": "inputs larger than L2: %.1f GB of KV read per step per GPU" % gb,
    }
    if extra:
        cfg.update(extra)
    return cfg


def workload_all(name: str, world: int, prefix: int = 768):
    """Every rank's contexts (rank order) and rank 0's description."""
    groups = [[int(x) for x in workload(name, r, prefix)[0]] for r in range(world)]
    return groups, workload(name, 0, prefix)[1]


# ------------------------------------------------------------------ ours
def prefill(eng, slots, lens, stream, gen, dev):
    import torch
    sh = stream.cuda_stream
    chunk = 4096
    with torch.cuda.stream(stream):
        for s, L in zip(slots, lens):
            done = 0
            while done < L:
                t = min(chunk, L - done)
                for layer in range(N_LAYERS):
                    k = torch.randn((t, G, D), generator=gen, device=dev)
                    v = torch.randn((t, G, D), generator=gen, device=dev)
                    eng.rope_append_range(layer, s, t, k, v, sh)
                eng.advance([s], t)
                done += t
    eng.sync_check(sh)


def bench_ours(args):
    import torch
    import hkv

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as tdist
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                 device_id=torch.device("cuda", local))
        dist = tdist

    def barrier():
        if dist is not None:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if dist is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=f"cuda:{local}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def sum_over_ranks(x: float) -> float:
        if dist is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=f"cuda:{local}")
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return float(t.item())

    total_steps = args.warmup + args.steps + args.e2e_steps + 4
    dev = f"cuda:{local}"
    stream = torch.cuda.Stream(device=local)
    sh = stream.cuda_stream
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234 + rank)
    churn = None
    if args.workload == "churn":
        # 64 slots in 8 groups; each group shares a published reference-prompt
        # prefix (copy-on-write pages); slots finish with probability 0.01 per
        # step and are replaced by fresh prefix-only slots of the same group.
        n, group, prefix = 64, 8, args.prefix
        lens, desc = workload("churn", rank, prefix)
        lens = [int(x) for x in lens]
        prefix_pages = (prefix + 15) // 16
        n_pages = (sum((L - prefix + total_steps + 15) // 16 + 2 for L in lens)
                   + (n // group) * prefix_pages + n * ((total_steps + 15) // 16 + 2) + 64)
        eng = hkv.Engine(n_layers=N_LAYERS, n_pages=n_pages, max_slots=n + 1, device=local,
                         shuffle_seed=0x5EED + rank)
        for g in range(n // group):
            owner = eng.acquire(prefix)
            prefill(eng, [owner], [prefix], stream, gen, dev)
            eng.publish(g + 1, prefix, owner)
            eng.release(owner)  # the published prefix keeps its pages
        slots = []
        for i, L in enumerate(lens):
            s_ = eng.acquire(L + total_steps, share=(i // group + 1, prefix))
            prefill(eng, [s_], [L - prefix], stream, gen, dev)
            slots.append(s_)
        cur_len = list(lens)
        rng = np.random.default_rng(4242 + rank)
        churn_stats = {"replaced": 0}

        def churn():
            for i in range(n):
                if rng.random() < 0.01:
                    eng.release(slots[i])
                    slots[i] = eng.acquire(prefix + total_steps, share=(i // group + 1, prefix))
                    cur_len[i] = prefix
                    churn_stats["replaced"] += 1
    else:
        lens, desc = workload(args.workload, rank)
        n = len(lens)
        n_pages = sum((L + total_steps + 15) // 16 + 1 for L in lens) + 16
        eng = hkv.Engine(n_layers=N_LAYERS, n_pages=n_pages, max_slots=n, device=local,
                         shuffle_seed=0x5EED + rank)
        slots = [eng.acquire(L + total_steps) for L in lens]
        prefill(eng, slots, lens, stream, gen, dev)
        cur_len = list(lens)

    # Step inputs, resident in HBM: q [36][n][32][128], k/v [36][n][8][128] F32.
    q = torch.randn((N_LAYERS, n, H, D), generator=gen, device=dev)
    k = torch.randn((N_LAYERS, n, G, D), generator=gen, device=dev)
    v = torch.randn((N_LAYERS, n, G, D), generator=gen, device=dev)
    out = torch.empty((N_LAYERS, n, H * D), device=dev)

    rows_seen = [0]  # rows attended, summed over decode steps (algorithmic bytes)

    def step():
        rows_seen[0] += sum(L + 1 for L in cur_len)
        for layer in range(N_LAYERS):
            eng.decode_step(layer, slots, q[layer], k[layer], v[layer], out[layer], sh)
        eng.advance(slots, 1)
        for i in range(n):
            cur_len[i] += 1
        if churn is not None:
            churn()

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step()
    torch.cuda.synchronize()
    eng.sync_check(sh)

    # ---------------- device-timed region (inputs resident)
    stats_before = eng.stats()
    rows_seen[0] = 0
    clocks = ClockSampler(local)
    barrier()
    torch.cuda.synchronize()
    clocks.start()
    # No per-launch profiler events in the timed region: they would sit between
    # the 36 launches of a step and stop each launch from overlapping the tail
    # of the previous one.
    torch.cuda.nvtx.range_push("timed")
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    with torch.cuda.stream(stream):
        for _ in range(args.steps):
            step()
    ev1.record(stream)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    barrier()
    clk = clocks.stop()
    ms_local = ev0.elapsed_time(ev1)
    rows = rows_seen[0]
    stats_after = eng.stats()
    eng.sync_check(sh)
    # Kernel-only time from the engine's event profiler on two extra steps.
    eng.profile_reset()
    eng.profile_enable(True)
    with torch.cuda.stream(stream):
        for _ in range(2):
            step()
    torch.cuda.synchronize()
    eng.profile_enable(False)
    prof_launches, prof_ms = eng.profile_read(hkv.KERNEL_STEP)
    eng.sync_check(sh)
    ms = max_over_ranks(ms_local)

    # Algorithmic bytes per (slot, layer, step) with L rows attended:
    # 4096 L (K+V F16 read) + 4096 (new row write) + 8192 (k, v in) + 16384
    # (q in) + 16384 (out) = 4096 L + 45056, all of it moved by the one fused
    # kernel launch of the layer.
    step_bytes_local = N_LAYERS * (4096 * rows + 45056 * n * args.steps) / args.steps
    launch_bytes = step_bytes_local / N_LAYERS
    tokens_total = sum_over_ranks(n * args.steps)
    step_bytes_all = sum_over_ranks(step_bytes_local)
    value = tokens_total / (ms / 1e3)
    peak, peak_kind = measured_peaks()
    # Each layer of a step is one launch of the decode kernel; its duration is
    # taken from the timed region itself: step time / 36 launches (this still
    # counts the small gaps between launches, so it understates the kernel).
    step_avg_ms = ms_local / (N_LAYERS * args.steps)
    kernel_gbs = launch_bytes / (step_avg_ms / 1e3) / 1e9
    kernel_only_ms = prof_ms / max(prof_launches, 1)
    step_gbs_per_gpu = step_bytes_all / world / (ms / args.steps / 1e3) / 1e9

    # ---------------- end to end through the C ABI from pinned host buffers
    e2e = None
    if args.e2e_steps > 0:
        # Host inputs q | k | v per layer in one pinned buffer; device inputs
        # and outputs double-buffered by step parity.  The layers run in
        # chunks of 9: the inputs of step s+1's chunk c stream in while step
        # s computes, and the outputs of chunk c stream out while the next
        # chunk computes, so the stream sees event waits only at chunk
        # boundaries and the launches inside a chunk still overlap.
        qkv_floats = n * (H + 2 * G) * D
        chunk = args.e2e_chunk
        chunks = [(c, min(c + chunk, N_LAYERS)) for c in range(0, N_LAYERS, chunk)]
        hin = torch.randn((N_LAYERS, qkv_floats)).pin_memory()
        hout = torch.empty((2, N_LAYERS, n, H * D)).pin_memory()
        din = torch.empty((2, N_LAYERS, qkv_floats), device=dev)
        dout = torch.empty((2, N_LAYERS, n, H * D), device=dev)
        h2d = torch.cuda.Stream(device=local)
        d2h = torch.cuda.Stream(device=local)
        # Per-call arguments prepared once, as a caller of the C ABI keeps
        # them: device pointers of q, k, v and out per (buffer, layer), the
        # slot array per step (rebuilt only when the batch changes).
        fsz = 4
        ptrs = [[(din[p_, layer].data_ptr(), din[p_, layer].data_ptr() + n * H * D * fsz,
                  din[p_, layer].data_ptr() + n * (H + G) * D * fsz, dout[p_, layer].data_ptr())
                 for layer in range(N_LAYERS)] for p_ in range(2)]
        slot_arg = [eng.slots_array(slots)]
        ev_in = [[torch.cuda.Event() for _ in chunks] for _ in range(2)]
        ev_done = [[torch.cuda.Event() for _ in chunks] for _ in range(2)]
        ev_back = [[torch.cuda.Event() for _ in chunks] for _ in range(2)]
        used = [[False] * len(chunks) for _ in range(2)]
        host_s = [0.0]

        def upload(p, c):
            lo, hi = chunks[c]
            with torch.cuda.stream(h2d):
                if used[p][c]:
                    h2d.wait_event(ev_done[p][c])  # the step two back has read din[p]
                din[p, lo:hi].copy_(hin[lo:hi], non_blocking=True)
                ev_in[p][c].record(h2d)

        def e2e_step(s, first, last):
            t0 = time.perf_counter()
            p = s % 2
            if first:
                for c in range(len(chunks)):
                    upload(p, c)
            for c, (lo, hi) in enumerate(chunks):
                if not last:
                    upload(1 - p, c)
                stream.wait_event(ev_in[p][c])
                if used[p][c]:
                    stream.wait_event(ev_back[p][c])  # dout[p] chunk is on the host
                n_, arr = slot_arg[0]
                for layer in range(lo, hi):
                    qp, kp, vp, op = ptrs[p][layer]
                    eng.decode_step_ptrs(layer, n_, arr, qp, kp, vp, op, sh)
                ev_done[p][c].record(stream)
                used[p][c] = True
                with torch.cuda.stream(d2h):
                    d2h.wait_event(ev_done[p][c])
                    hout[p, lo:hi].copy_(dout[p, lo:hi], non_blocking=True)
                    ev_back[p][c].record(d2h)
            eng.advance(slots, 1)
            for i in range(n):
                cur_len[i] += 1
            if churn is not None:
                churn()
                slot_arg[0] = eng.slots_array(slots)
            host_s[0] += time.perf_counter() - t0

        e2e_step(0, True, True)
        stream.wait_stream(d2h)
        torch.cuda.synchronize()
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        h2d.wait_stream(stream)
        d2h.wait_stream(stream)
        host_s[0] = 0.0
        eng.host_stats(reset=True)
        for i in range(args.e2e_steps):
            e2e_step(i, i == 0, i == args.e2e_steps - 1)
        stream.wait_stream(d2h)  # the last outputs are on the host
        e1.record(stream)
        eng_calls, eng_us, eng_launch_us = eng.host_stats(reset=True)
        torch.cuda.synchronize()
        e2e_ms = max_over_ranks(e0.elapsed_time(e1))
        e2e_tokens = sum_over_ranks(n * args.e2e_steps)
        h2d_bytes = N_LAYERS * qkv_floats * 4
        d2h_bytes = N_LAYERS * n * H * D * 4
        e2e = {"value": e2e_tokens / (e2e_ms / 1e3), "unit": "tokens/s",
               "h2d_bytes_per_step": h2d_bytes, "d2h_bytes_per_step": d2h_bytes,
               "steps": args.e2e_steps, "ms_per_step": e2e_ms / args.e2e_steps,
               "host_enqueue_ms_per_step": 1e3 * host_s[0] / args.e2e_steps,
               "engine_cpu_us_per_call": (eng_us - eng_launch_us) / max(eng_calls, 1),
               "engine_blocking_us_per_call": eng_launch_us / max(eng_calls, 1),
               "engine_blocking_note": "inside the CUDA launch calls and waits to reuse a plan "
                                       "upload buffer: blocks when the host is ahead of the GPU",
               "chunk_layers": chunk,
               "path": "pinned host q|k|v -> hkv_decode_step -> pinned host out "
                       f"(one copy each way per {chunk} layers)"}
        eng.sync_check(sh)
        if churn is None:
            # The host outputs of the last timed step, checked bit for bit
            # against the same step run again from device-resident inputs:
            # lengths rolled back by one, the same 36 decode launches (the
            # same rows appended, the same plan), no copies or events between.
            p_last = (args.e2e_steps - 1) % 2
            for s_ in slots:
                eng.set_length(s_, eng.length(s_) - 1)
            redo = torch.empty((N_LAYERS, n, H * D), device=dev)
            with torch.cuda.stream(stream):
                for layer in range(N_LAYERS):
                    x = din[p_last, layer]
                    eng.decode_step(layer, slots, x[:n * H * D], x[n * H * D:n * (H + G) * D],
                                    x[n * (H + G) * D:], redo[layer], sh)
            eng.advance(slots, 1)
            torch.cuda.synchronize()
            eng.sync_check(sh)
            same = bool(torch.equal(redo.cpu(), hout[p_last]))
            e2e["check"] = {"bitwise_equal": same, "layers": N_LAYERS,
                            "what": "last timed step's host outputs vs the same step from "
                                    "device-resident inputs"}
            if not same:
                raise SystemExit("e2e outputs differ from the device-resident recompute")
    eng.sync_check(sh)
    eng.close()

    split = headsplit_run(args, dist, rank, world, local, steps=max(3, args.steps // 2),
                          warmup=3) if not args.no_headsplit else None

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        groups_cpu, _ = workload_all(args.workload, 1, args.prefix)
        cpu = cpu_complete_steps(groups_cpu, budget_s=30.0, max_steps=1)
        if churn is not None:
            cpu["sample"] += "; slots do not churn in this sample"

    legs = {}
    if rank == 0 and world == 1 and args.workload == "scaleout" and not args.no_extra_legs:
        torch.cuda.empty_cache()
        for name, argv in EXTRA_LEGS.items():
            legs[name] = child_leg(argv + ["--no-cpu-baseline", "--no-headsplit", "--no-extra-legs"])

    if rank == 0:
        groups_all, desc_all = workload_all(args.workload, world, args.prefix)
        traffic = None
        tfile = REPO / "profiles" / "attention_traffic.json"
        if tfile.exists():
            t = json.loads(tfile.read_text())
            traffic = t.get("dram_bytes_per_launch", {}).get(args.workload)
        line = {
            "metric": METRIC,
            "value": value,
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms / args.steps,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "f16 KV, f32 accumulate",
            "data": "synthetic N(0,1) (torch generator on device), random physical page order",
            "config": run_config(args.workload, world, [x for g in groups_all for x in g],
                                 groups_all[0], desc_all),
            "hbm": {"step_gbs_per_gpu": step_gbs_per_gpu, "peak_gbs": peak,
                    "frac": step_gbs_per_gpu / peak, "peak_kind": peak_kind},
            "roofline": {
                "kernel": "attention_kernel<append> (fused RoPE append + split-K decode "
                          "attention + merge, one launch per layer)",
                "bound": "hbm", "achieved": kernel_gbs, "peak": peak, "unit": "GB/s",
                "frac": kernel_gbs / peak, "traffic": traffic,
                "algorithmic_bytes_per_launch": launch_bytes,
                "avg_launch_ms": step_avg_ms, "peak_kind": peak_kind,
                "launch_ms_from": "timed region: step time / launches (includes launch gaps)",
                "kernel_only_ms_profiled": kernel_only_ms,
            },
            "gpu_launches": stats_after["kernel_launches"] - stats_before["kernel_launches"],
            "pool": {"cow_copies_timed": stats_after["cow_copies"] - stats_before["cow_copies"],
                     "shared_pages": stats_after["shared_pages"],
                     "replaced_slots": (churn_stats["replaced"] if churn is not None else 0)},
            "e2e": e2e,
            "cpu_baseline": cpu,
            "clocks": clk,
            "headsplit": split,
            **legs,
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def child_leg(argv: list, timeout_s: int = 600) -> dict:
    """One more workload as a child process on this GPU (`python bench.py
    <argv>`), with the same timing rules as the main run; returns the figures
    of its JSON line (or why it failed)."""
    import subprocess

    cmd = [sys.executable, str(REPO / "bench.py")] + argv
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=timeout_s)
    lines = [x for x in r.stdout.splitlines() if x.startswith("{")]
    if r.returncode != 0 or not lines:
        return {"failed": f"exit {r.returncode}: {r.stderr.strip().splitlines()[-1:]}"}
    d = json.loads(lines[-1])
    return {"value": d["value"], "unit": d["unit"], "steps": d["steps"], "warmup": d["warmup"],
            "ms_per_step": d["ms_per_step"], "config": d["config"], "dtype": d["dtype"],
            "roofline_frac": d["roofline"]["frac"], "roofline_achieved": d["roofline"]["achieved"],
            "e2e_value": (d["e2e"] or {}).get("value"), "clocks": d["clocks"],
            "gpu_launches": d["gpu_launches"], "command": "python bench.py " + " ".join(argv)}


# Legs the default one-GPU run adds to its line: the small-batch attention
# workload and the whole backbone decode step at batch 1 and 16.
EXTRA_LEGS = {
    "batched16": ["--workload", "batched16", "--steps", "20", "--warmup", "3", "--e2e-steps", "10"],
    "backbone_batch1": ["--workload", "backbone", "--steps", "60", "--warmup", "5", "--e2e-steps", "10"],
    "backbone_batch16": ["--workload", "backbone", "--batch", "16", "--steps", "60", "--warmup", "5",
                         "--e2e-steps", "10"],
}


def headsplit_run(args, dist, rank: int, world: int, local: int, steps: int, warmup: int):
    """One request near the 32768-position context split by KV head across
    the ranks (HeadSplit): rank g holds KV heads [8g/N, 8(g+1)/N) of every
    layer and attends its 32/N query heads.  The head-major output of each
    layer reaches every rank either inside the decode kernel (--xchg p2p:
    peer stores over NVLink + a bounded arrival wait, hkv_split_step /
    hkv_split_wait) or by an NCCL all-gather after it (--xchg nccl).

    Timed twice with CUDA events, max over ranks: the split decode alone
    (each rank's hkv_decode_step, no exchange) and with the exchange; their
    difference per layer is the exchange's cost.  Then the last step's output
    of the last layer, as assembled on rank 0, is checked against the oracle
    over the caches every rank holds (gathered with hkv_gather).  Returns a
    dict on rank 0 (None elsewhere)."""
    import torch
    import hkv
    from hkv_dist import HeadSplit

    # --split-shape N on one GPU: rank 0's engine shape of an N-way split, no
    # exchange (tunes the per-rank launch without N GPUs)
    shape_world = args.split_shape if (dist is None and args.split_shape > 1) else world
    split = HeadSplit(world=shape_world, rank=rank)
    Gl, Hl = split.local_kv_heads, split.local_q_heads
    total_steps = 2 * (warmup + steps) + 2
    L0 = 32768 - total_steps - 1  # the last step's new row sits at position <= 32766
    dev = f"cuda:{local}"
    eng = hkv.Engine(n_layers=N_LAYERS, n_pages=(L0 + total_steps) // 16 + 2, max_slots=1,
                     device=local, shuffle_seed=0xBEEF + rank, **split.engine_shape())
    stream = torch.cuda.Stream(device=local)
    sh = stream.cuda_stream
    slot = eng.acquire(L0 + total_steps)
    gen = torch.Generator(device=dev)
    gen.manual_seed(77 + rank)
    with torch.cuda.stream(stream):
        done = 0
        while done < L0:
            t = min(4096, L0 - done)
            for layer in range(N_LAYERS):
                k = torch.randn((t, Gl, D), generator=gen, device=dev)
                v = torch.randn((t, Gl, D), generator=gen, device=dev)
                eng.rope_append_range(layer, slot, t, k, v, sh)
            eng.advance([slot], t)
            done += t
        q = torch.randn((N_LAYERS, 1, Hl, D), generator=gen, device=dev)
        k = torch.randn((N_LAYERS, 1, Gl, D), generator=gen, device=dev)
        v = torch.randn((N_LAYERS, 1, Gl, D), generator=gen, device=dev)
        out_local = torch.empty((N_LAYERS, 1, Hl * D), device=dev)
        out_full = torch.empty((N_LAYERS, world, Hl * D), device=dev)
    eng.sync_check(sh)

    p2p = dist is not None and args.xchg == "p2p"
    if p2p:
        handles = [None] * world
        dist.all_gather_object(handles, eng.split_export(world, rank))
        eng.split_connect(handles)
        dist.barrier()

    def step(exchange: bool):
        for layer in range(N_LAYERS):
            if exchange and p2p:
                eng.split_step(layer, [slot], q[layer], k[layer], v[layer], sh)
                eng.split_wait(layer, sh)
            else:
                eng.decode_step(layer, [slot], q[layer], k[layer], v[layer], out_local[layer], sh)
                if exchange and dist is not None:
                    dist.all_gather_into_tensor(out_full[layer], out_local[layer])
        eng.advance([slot], 1)

    def timed(exchange: bool):
        with torch.cuda.stream(stream):
            for _ in range(warmup):
                step(exchange)
        torch.cuda.synchronize()
        if dist is not None:
            dist.barrier()
        ctx0 = eng.length(slot) + 1
        ev0 = torch.cuda.Event(enable_timing=True)
        ev1 = torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            ev0.record(stream)
            for _ in range(steps):
                step(exchange)
            ev1.record(stream)
        torch.cuda.synchronize()
        ms = ev0.elapsed_time(ev1)
        if dist is not None:
            t = torch.tensor([ms], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        eng.sync_check(sh)
        return ms, ctx0

    ms_alone, _ = timed(False)
    launches0 = eng.stats()["kernel_launches"]
    ms, ctx0 = timed(True)
    launches_per_step = (eng.stats()["kernel_launches"] - launches0) / (warmup + steps)

    # ---- parity of the assembled output (last step, last layer) on rank 0
    layer = N_LAYERS - 1
    rows = eng.length(slot)
    kb = torch.empty((rows, Gl, D), dtype=torch.int16, device=dev)
    vb = torch.empty_like(kb)
    eng.gather(slot, layer, 0, rows, kb, vb, sh)
    torch.cuda.synchronize()
    if p2p:
        ptr, width = eng.split_output(layer)
        full = torch.as_tensor(hkv.DeviceArray(ptr, (1, width)), device=dev).clone()
    elif dist is not None:
        full = out_full[layer].reshape(1, -1).clone()
    else:
        full = out_local[layer].reshape(1, -1).clone()
    if dist is not None:
        parts = {}
        for name, t in (("k", kb), ("v", vb), ("q", q[layer].reshape(Hl, D))):
            lst = [torch.empty_like(t) for _ in range(world)]
            src = t.view(torch.float16) if t.dtype == torch.int16 else t
            lst16 = [x.view(torch.float16) if x.dtype == torch.int16 else x for x in lst]
            dist.all_gather(lst16, src.contiguous())
            parts[name] = lst
        k_all = torch.cat(parts["k"], dim=1)
        v_all = torch.cat(parts["v"], dim=1)
        q_all = torch.cat(parts["q"], dim=0)
    else:
        k_all, v_all, q_all = kb, vb, q[layer].reshape(Hl, D)
        full = full[:, :Hl * D]
    out = None
    if rank == 0:
        sys.path.insert(0, str(REPO / "oracle"))
        import cpu_oracle
        cpu_oracle.build()
        cos, sin = cpu_oracle.rope_table()
        pos = rows - 1
        qr = cpu_oracle.rope_neox(q_all.cpu().numpy(), cos[pos], sin[pos])[None]
        kh = k_all.cpu().numpy().view(np.uint16)
        vh = v_all.cpu().numpy().view(np.uint16)
        got = full.cpu().numpy().astype(np.float64).reshape(-1, D)
        errs = []
        for mode in (cpu_oracle.EXACT, cpu_oracle.GGML_F16):
            ref = cpu_oracle.decode_attn(qr, [kh], [vh], mode).astype(np.float64).reshape(-1, D)
            errs.append(float(np.max(np.abs(got - ref).max(1) / np.abs(ref).max(1))))
        rows_attended = sum(ctx0 + s_ for s_ in range(steps))
        bytes_per_rank = N_LAYERS * 512 * Gl * (rows_attended + 11 * steps)
        peak, peak_kind = measured_peaks()
        gbs = bytes_per_rank / (ms / 1e3) / 1e9
        out = {
            "tokens_s": steps / (ms / 1e3), "ms_per_step": ms / steps,
            "decode_alone_tokens_s": steps / (ms_alone / 1e3),
            "exchange_us_per_layer": 1e3 * (ms - ms_alone) / steps / N_LAYERS,
            "max_rel_err": max(errs), "max_rel_err_modes": {"exact": errs[0], "ggml_f16": errs[1]},
            "parity_case": f"layer {layer} of the last timed step, 32 query heads over {rows} "
                           "positions, assembled output on rank 0 vs the oracle",
            "context": ctx0, "steps": steps, "warmup": warmup, "gpus": world,
            "launches_per_step": launches_per_step,
            "shape_of_split": shape_world,
            "kv_heads_per_gpu": Gl,
            "exchange": ("in-kernel peer stores over NVLink + bounded arrival wait" if p2p else
                         ("NCCL all-gather" if dist is not None else "none (one GPU)")),
            "hbm_frac_per_gpu": gbs / peak, "peak_kind": peak_kind,
            "scaling": "strong (one request, total work fixed)",
        }
        if max(errs) > 2e-3:
            raise SystemExit(f"KV-head split output differs from the oracle: {max(errs):.3e}")
    if p2p:
        dist.barrier()
        eng.split_disconnect()
    if dist is not None:
        dist.barrier()
    eng.close()
    if dist is not None:
        dist.barrier()
    return out


def bench_headsplit(args):
    """The KV-head split of one long request alone (see headsplit_run)."""
    import datetime

    import torch

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as tdist
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                 device_id=torch.device("cuda", local))
        dist = tdist
    res = headsplit_run(args, dist, rank, world, local, args.steps, args.warmup)
    if rank == 0:
        peak, peak_kind = measured_peaks()
        print(json.dumps({
            "metric": METRIC, "value": res["tokens_s"], "unit": "tokens/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": res["ms_per_step"], "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f16 KV, f32 accumulate",
            "data": "synthetic N(0,1) (torch generator on device)",
            "config": {"workload": (f"one {res['context']}-position request split by KV head "
                                    f"over {world} GPU(s), {res['kv_heads_per_gpu']} KV heads "
                                    f"each, 36 layers; per-head outputs assembled every layer "
                                    f"by {res['exchange']}"),
                       "global_batch": 1, "layers": N_LAYERS,
                       "parallelism": f"KV-head split x{world}"},
            "hbm": {"frac_per_gpu": res["hbm_frac_per_gpu"], "peak_kind": peak_kind},
            "headsplit": res, "gpu_launches": res["launches_per_step"] * args.steps, "e2e": None,
        }), flush=True)
    if dist is not None:
        dist.destroy_process_group()


def make_backbone_weights(hkv, n_layers: int, text_vocab: int, dev: str, seed: int = 1234):
    """Random-init N(0, 0.02) weights of the Qwen3-4B-shaped backbone quantised
    to Q4_K on the device by the repo's encoder; norms N(1, 0.1) in F32.
    Returns (name -> device tensor, Q4_K bytes per decode step)."""
    import torch
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed)
    w = {}
    step_bytes = [0]

    def mat(name, rows, cols, read_per_step=True):
        out = torch.empty((rows, cols // 256 * 144), dtype=torch.uint8, device=dev)
        for r0 in range(0, rows, 16384):  # bounded F32 staging
            r1 = min(rows, r0 + 16384)
            f = torch.randn((r1 - r0, cols), generator=gen, device=dev) * 0.02
            hkv.q4k_quantize(f, r1 - r0, cols, out[r0:r1])
            del f
        w[name] = out
        if read_per_step:
            step_bytes[0] += out.numel()

    def norm(name, size):
        w[name] = torch.randn((size,), generator=gen, device=dev) * 0.1 + 1.0
        step_bytes[0] += 4 * size

    for l in range(n_layers):
        p = f"blk.{l}."
        mat(p + "attn_q", 4096, 2560)
        mat(p + "attn_k", 1024, 2560)
        mat(p + "attn_v", 1024, 2560)
        mat(p + "attn_output", 2560, 4096)
        mat(p + "ffn_gate", 9728, 2560)
        mat(p + "ffn_up", 9728, 2560)
        mat(p + "ffn_down", 2560, 9728)
        for k, size in (("attn_norm", 2560), ("ffn_norm", 2560), ("attn_q_norm", 128),
                        ("attn_k_norm", 128)):
            norm(p + k, size)
    mat("token_embd", text_vocab, 2560, read_per_step=False)
    mat("a.token_embd", 8 * 1026, 2560, read_per_step=False)
    step_bytes[0] += 8 * 10 * 144  # the 8 embedding rows of a step
    mat("a.output", 8 * 1026, 2560)
    norm("output_norm", 2560)
    torch.cuda.synchronize()
    return w, step_bytes[0]


def bench_backbone(args):
    """The whole 36-layer Q4_K backbone decode step (Qwen3-4B shape: hidden
    2560, FFN 9728, GQA 32/8) for args.batch requests: a 1024-token prompt of
    uniform random text ids per request, fed one token per request per decode
    call, then greedy steps (the first maximum of each of the 8 codebooks'
    logits, whose embedding rows are summed into the next input).  A step =
    embedding + 36 x (q/k/v with per-head norms, RoPE + append + attention,
    o_proj + residual, SwiGLU FFN, down + residual) + output head + greedy
    codes, for every request at once.  Batch 1 uses the one-vector (dp4a)
    projections; a backbone created for batches runs them on the tensor
    cores.  Under torchrun each rank runs its own replica."""
    import datetime

    import torch
    import hkv

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import torch.distributed as tdist
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                 device_id=torch.device("cuda", local))
        dist = tdist
    dev = f"cuda:{local}"
    text_vocab, prompt_len = 151936, args.prompt_len
    B = args.batch
    weights, weight_bytes = make_backbone_weights(hkv, N_LAYERS, text_vocab, dev, 1234 + rank)
    total = prompt_len + args.warmup + args.steps + args.e2e_steps + 4
    eng = hkv.Engine(n_layers=N_LAYERS, n_pages=B * (total // 16 + 4), max_slots=B, device=local,
                     shuffle_seed=99 + rank)
    bb = hkv.Backbone(eng, weights, text_vocab=text_vocab, rms_eps=1e-6, max_batch=B)
    stream = torch.cuda.Stream(device=local)
    sh = stream.cuda_stream
    slots = [eng.acquire(total) for _ in range(B)]
    ids = np.random.default_rng(5 + rank).integers(0, text_vocab, (prompt_len, B))
    with torch.cuda.stream(stream):
        for t in range(prompt_len):
            bb.embed_text([int(i) for i in ids[t]], sh)
            bb.decode(slots, want_logits=(t == prompt_len - 1), stream=sh)
    bb.sync_check(sh)

    def step():
        bb.embed_codes(B, None, sh)
        bb.decode(slots, want_logits=True, stream=sh)

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    ctx0 = eng.length(slots[0])
    launches0 = eng.stats()["kernel_launches"]
    bb_launches0 = bb.kernel_launches
    clocks = ClockSampler(local)
    clocks.start()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("timed")
    ev0.record(stream)
    h0 = time.perf_counter()
    with torch.cuda.stream(stream):
        for _ in range(args.steps):
            step()
    host_ms = (time.perf_counter() - h0) * 1e3
    ev1.record(stream)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    clk = clocks.stop()
    ms_local = ev0.elapsed_time(ev1)
    bb.sync_check(sh)
    # the engine counts its own launches (append + attention, and a combine
    # launch where the plan merges split partials after the grid); the
    # backbone counts its embedding, projection and argmax launches
    engine_launches = eng.stats()["kernel_launches"] - launches0
    backbone_launches = bb.kernel_launches - bb_launches0

    def max_ranks(x):
        if dist is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    ms = max_ranks(ms_local)
    # Algorithmic bytes per step: every Q4_K matrix of the step once (a
    # tensor-core launch takes up to 8 requests), the norms, 8 embedding
    # rows per request, and per layer and request the KV path's
    # 4096 L + 45056.
    kv_bytes = B * sum(N_LAYERS * (4096 * (ctx0 + s + 1) + 45056) for s in range(args.steps))
    step_bytes = weight_bytes + kv_bytes / args.steps
    peak, peak_kind = measured_peaks()
    gbs = step_bytes / (ms / args.steps / 1e3) / 1e9

    # End to end through the public API: each step's codes are read back to
    # the host (what a caller streaming them to the audio decoder does) and
    # handed back as the next step's input.
    e2e = None
    if args.e2e_steps > 0:
        hcodes = torch.empty((B, 8), dtype=torch.int32).pin_memory()
        dcodes = torch.empty((B, 8), dtype=torch.int32, device=dev)
        codes_view = torch.as_tensor(hkv.DeviceArray(bb.codes_ptr, (B, 8), "<i4"), device=dev)

        def e2e_step():
            with torch.cuda.stream(stream):
                hcodes.copy_(codes_view, non_blocking=True)
            stream.synchronize()
            with torch.cuda.stream(stream):
                dcodes.copy_(hcodes, non_blocking=True)
            bb.embed_codes(B, dcodes, sh)
            bb.decode(slots, want_logits=True, stream=sh)

        e2e_step()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.e2e_steps):
            e2e_step()
        with torch.cuda.stream(stream):
            hcodes.copy_(codes_view, non_blocking=True)
        e1.record(stream)
        torch.cuda.synchronize()
        e_ms = max_ranks(e0.elapsed_time(e1))
        e2e = {"value": world * B * args.e2e_steps / (e_ms / 1e3), "unit": "tokens/s",
               "h2d_bytes_per_step": 32 * B, "d2h_bytes_per_step": 32 * B, "steps": args.e2e_steps,
               "ms_per_step": e_ms / args.e2e_steps,
               "path": "codes read back to pinned host memory and fed back through "
                       "hkv_backbone_embed_codes + hkv_backbone_decode each step"}
    bb.sync_check(sh)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_backbone(weights, ctx0)
        if B > 1:
            cpu["sample"] += ("; the reference decodes one request at a time, so B requests "
                              "take B of these steps: the same tokens/s")
    if rank == 0:
        print(json.dumps({
            "metric": "backbone decode tokens/s (36-layer Q4_K step incl. KV append + attention)",
            "value": world * B * args.steps / (ms / 1e3), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": ("q4_k weights x q8_k activations (int dp4a), f32 accumulate, f16 KV" if B == 1 else
                      "q4_k weights x q8_k activations (int8 mma m16n8k32 on the tensor cores), "
                      "f32 accumulate, f16 KV"),
            "data": "synthetic: N(0,0.02) weights quantised to Q4_K on the device, uniform "
                    "random prompt ids",
            "config": {"workload": f"backbone decode, batch {B}: 36 layers, hidden 2560, FFN 9728, "
                                   f"GQA 32/8, {prompt_len}-token prompt then greedy steps "
                                   f"(contexts {ctx0 + 1}..{ctx0 + args.steps})",
                       "global_batch": world * B, "batch_per_gpu": B, "layers": N_LAYERS,
                       "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
                       "l2": "inputs larger than L2: 2.2 GB of weights read per step"},
            "roofline": {"kernel": f"whole decode step ({backbone_launches // args.steps} "
                                   "embedding/projection/argmax launches + the engine's)", "bound": "hbm",
                         "achieved": gbs, "peak": peak, "unit": "GB/s", "frac": gbs / peak,
                         "traffic": None, "algorithmic_bytes_per_step": step_bytes,
                         "peak_kind": peak_kind},
            "cpu_baseline": cpu, "clocks": clk, "e2e": e2e,
            "gpu_launches": backbone_launches + engine_launches,
            "host_enqueue_ms_per_step": host_ms / args.steps,
        }), flush=True)
    bb.close()
    eng.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def cpu_baseline_backbone(weights, ctx: int, budget_s: float = 12.0):
    """The oracle's restatement of the reference's CPU graph (Q4_K x Q8_K
    projections, F16 KV attention) on the host cores: decode steps of a
    2-layer slice of the same weights at the same context (prefilled with
    random rows), scaled to 36 layers + the output head."""
    sys.path.insert(0, str(REPO / "oracle"))
    import cpu_oracle
    cpu_oracle.build()
    cores = cpu_oracle.max_threads()
    L = 2
    host = {}
    for k, t in weights.items():
        if k.startswith("blk.") and int(k.split(".")[1]) >= L:
            continue
        if k == "token_embd":
            continue
        host[k] = t.cpu().numpy()
    ref = cpu_oracle.BackboneOracle(host, L)
    rng = np.random.default_rng(0)
    for l in range(L):
        kc = rng.integers(0x3000, 0x3800, (ctx, 8, 128)).astype(np.uint16)
        ref.caches[(0, l)] = (kc, kc.copy())
    h = ref.embed_codes(np.zeros((1, 8), np.int32))
    ref.decode(h, [0], [ctx], want_logits=False)  # warm-up
    t0 = time.perf_counter()
    steps = 0
    pos = ctx
    while time.perf_counter() - t0 < budget_s or steps < 2:
        ref.decode(h, [0], [pos], want_logits=False)
        steps += 1
    per_layer_s = (time.perf_counter() - t0) / steps / L
    t1 = time.perf_counter()
    ref.decode(h, [0], [pos], want_logits=True)
    head_s = max(0.0, time.perf_counter() - t1 - per_layer_s * L)
    step_s = per_layer_s * N_LAYERS + head_s
    return {"value": 1.0 / step_s, "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"{steps} decode steps of 2 of the 36 layers at context {ctx} "
                      f"({budget_s:.0f} s), scaled to 36 layers + the output head"}


def random_q4k_host(rng, rows, cols):
    """Random well-formed Q4_K blocks (test data: random quants and 6-bit
    scales, positive f16 super-scales of N(0, 0.02)-like magnitude)."""
    b = rng.integers(0, 256, size=(rows, cols // 256, 144), dtype=np.uint8)
    d = rng.uniform(2e-4, 1e-3, (rows, cols // 256)).astype(np.float16)
    b[:, :, 0:2] = d.view(np.uint8).reshape(rows, cols // 256, 2)
    b[:, :, 2:4] = d.view(np.uint8).reshape(rows, cols // 256, 2)
    return b.reshape(rows, -1)


def reference_backbone(args):
    """The reference arm of the backbone workload: the oracle's restatement of
    the GGML CPU graph (Q4_K x Q8_K projections, F16 KV attention) on the host
    cores, 2 of the 36 layers timed and scaled, at the same context."""
    sys.path.insert(0, str(REPO / "oracle"))
    import cpu_oracle
    cpu_oracle.build()
    rng = np.random.default_rng(0)
    L, ctx = 2, 1024 + args.warmup + args.steps // 2
    host = {}
    for l in range(L):
        p = f"blk.{l}."
        for name, rows, cols in (("attn_q", 4096, 2560), ("attn_k", 1024, 2560), ("attn_v", 1024, 2560),
                                 ("attn_output", 2560, 4096), ("ffn_gate", 9728, 2560),
                                 ("ffn_up", 9728, 2560), ("ffn_down", 2560, 9728)):
            host[p + name] = random_q4k_host(rng, rows, cols)
        for name, size in (("attn_norm", 2560), ("ffn_norm", 2560), ("attn_q_norm", 128),
                           ("attn_k_norm", 128)):
            host[p + name] = (1.0 + 0.1 * rng.standard_normal(size)).astype(np.float32)
    host["a.token_embd"] = random_q4k_host(rng, 8 * 1026, 2560)
    host["a.output"] = random_q4k_host(rng, 8 * 1026, 2560)
    host["output_norm"] = np.ones(2560, np.float32)
    ref = cpu_oracle.BackboneOracle(host, L)
    for l in range(L):
        kc = rng.integers(0x3000, 0x3800, (ctx, 8, 128)).astype(np.uint16)
        ref.caches[(0, l)] = (kc, kc.copy())
    h = ref.embed_codes(np.zeros((1, 8), np.int32))
    ref.decode(h, [0], [ctx], want_logits=False)
    budget = max(3.0, 1.0 * (args.steps + args.warmup))
    t0 = time.perf_counter()
    steps = 0
    while time.perf_counter() - t0 < budget or steps < 2:
        ref.decode(h, [0], [ctx], want_logits=False)
        steps += 1
    per_layer = (time.perf_counter() - t0) / steps / L
    t1 = time.perf_counter()
    ref.decode(h, [0], [ctx], want_logits=True)
    head = max(0.0, time.perf_counter() - t1 - per_layer * L)
    step_s = per_layer * 36 + head
    value = 1.0 / step_s
    cores = cpu_oracle.max_threads()
    print(json.dumps({
        "metric": "backbone decode tokens/s (36-layer Q4_K step incl. KV append + attention)",
        "value": value, "unit": "tokens/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": step_s * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "q4_k weights x q8_k activations, f32",
        "data": "synthetic random Q4_K blocks", "impl": "reference",
        "config": {"workload": f"backbone decode, batch {args.batch}, context {ctx}",
                   "global_batch": args.batch, "layers": 36, "parallelism": "host cores"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": f"{steps} decode steps of 2 of the 36 layers, scaled"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": ("the reference's GGML CPU graph cannot be built here (ggml submodule absent); "
                 "this times its restatement in oracle/ on the host cores; the reference decodes "
                 "one request at a time, so its tokens/s does not depend on the batch"),
    }), flush=True)


def bench_reference(args):
    """The reference arm: the reference's CPU decode graph (its GGML CPU path
    restated in oracle/hkv_oracle_graph.c; ggml itself is absent) on the host
    cores, on this run's exact workload -- every slot of every rank at its
    real context, 36 layers -- timed over COMPLETE steps.  One step of the
    full workload takes tens of seconds per 32 slots on the host, so the arm
    times as many complete steps as fit a fixed budget (at least one) and
    prints that count in `steps`; `steps_requested` keeps the driver's.
    Under torchrun only rank 0 works."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    if args.workload == "backbone":
        reference_backbone(args)
        return
    if args.workload == "headsplit":
        print(json.dumps({"impl": "reference", "unavailable":
                          "the reference has no multi-GPU path; see the scaleout workload"}))
        return
    groups, desc = workload_all(args.workload, world, args.prefix)
    t0 = time.perf_counter()
    cpu = cpu_complete_steps(groups, budget_s=100.0, max_steps=max(1, args.steps))
    wall = time.perf_counter() - t0
    flat = [x for g in groups for x in g]
    line = {
        "metric": METRIC,
        "value": cpu["value"],
        "unit": "tokens/s",
        "n_gpus": world,
        "steps": cpu["steps_timed"],
        "warmup": 0,
        "ms_per_step": cpu["step_s"] * 1e3,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32 (the reference's F32 cache and graph)",
        "data": "synthetic N(0,1)",
        "impl": "reference",
        "config": run_config(args.workload, world, flat, groups[0], desc),
        "cpu_baseline": {k: cpu[k] for k in ("value", "unit", "cores", "kind", "sample")},
        "e2e": {"value": cpu["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "steps_requested": args.steps,
        "warmup_requested": args.warmup,
        "note": ("the reference's GGML CPU graph cannot be built here (its ggml submodule is "
                 "absent); this times its restatement in oracle/hkv_oracle_graph.c on "
                 f"{cpu['cores']} host threads over {cpu['steps_timed']} complete step(s) of the "
                 f"whole workload ({len(flat)} slots x {N_LAYERS} layers, {cpu['step_s']:.1f} s "
                 f"per step; {args.steps} requested steps would take "
                 f"{args.steps * cpu['step_s']:.0f} s); warm-up: one single-layer graph, not a "
                 f"step; wall {wall:.1f} s"
                 + ("; slots do not churn in this arm" if args.workload == "churn" else "")),
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default="scaleout")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--e2e-chunk", type=int, default=9,
                    help="e2e: layers per host<->device copy (and per event wait)")
    ap.add_argument("--no-headsplit", action="store_true",
                    help="skip the KV-head split leg that follows the slot-sharded measurement")
    ap.add_argument("--no-extra-legs", action="store_true",
                    help="skip the batched16 and backbone legs that the default one-GPU run adds")
    ap.add_argument("--prefix", type=int, default=768,
                    help="churn: shared prefix length (770 puts the first append of every "
                         "replacement slot into a shared partial page: copy-on-write)")
    ap.add_argument("--split-shape", type=int, default=1,
                    help="headsplit on one GPU: run rank 0's shape of an N-way KV-head split "
                         "(8/N KV heads) without the exchange")
    ap.add_argument("--xchg", choices=["p2p", "nccl"], default="p2p",
                    help="headsplit: how the per-head outputs reach every rank")
    ap.add_argument("--batch", type=int, default=1,
                    help="backbone: requests per decode step (1: the reference's one request at a "
                         "time; more: a backbone created for batches, tensor-core projections)")
    ap.add_argument("--prompt-len", type=int, default=1024,
                    help="backbone: prompt tokens before the greedy steps (1024 for every "
                         "reported number; fewer only for profiler captures)")
    ap.add_argument("--layers", type=int, default=36,
                    help="layers per step (36 for every reported number; fewer only for "
                         "profiler captures of the same per-launch sizes)")
    args = ap.parse_args()
    global N_LAYERS
    N_LAYERS = args.layers
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    if args.impl == "reference":
        bench_reference(args)
    elif args.workload == "headsplit":
        bench_headsplit(args)
    elif args.workload == "backbone":
        bench_backbone(args)
    else:
        bench_ours(args)


if __name__ == "__main__":
    main()
