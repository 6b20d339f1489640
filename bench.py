"""Bench of the Qwen3-ASR text-decoder KV-cache path on B200.

Workload (the metric's "KV append + GQA attn" step):
per GPU 256 independent streams, context lengths log-uniform in [64, 4096]
(seeded per GPU), 28 layers of bf16 paged cache, 16-token pages handed out in
a seeded random order.  One step = for every stream and every layer: append
one token (K1: QK-RMSNorm + RoPE + page store of q/k/v ~ N(0,1)) and decode
attention over the whole context (K2).  value = decoded tokens/s over all GPUs
(one token per stream per step).  Streams are partitioned across GPUs with no
collective on the data path ("weak" scaling); torch.distributed is used only
for the barrier and the max-over-ranks timing.

    python bench.py [--gpus N --steps K --warmup W] [--impl ours|reference]
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

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

N_LAYERS, HQ, HKV, D = 28, 16, 8, 128
QKV = (HQ + 2 * HKV) * D
STREAMS_PER_GPU = 256
CTX_LO, CTX_HI = 64, 4096
WORKLOAD_SEED = 1004          # 1000 + config index
METRIC = "decode tokens/s (KV append+GQA attn) & KV-read HBM GB/s vs 8 TB/s, 1-8 B200"
# DRAM bytes (read + write) of one K2 launch on this workload (with the
# append-ahead of the next layer), from an ncu capture of the same 256
# streams and contexts (2 layers of cache held; a launch reads one).
K2_NCU_TRAFFIC_BYTES = 1_022_283_000 + 4_984_576


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d.get("bf16_tflops", 1590.0)),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def stream_lengths(rank: int) -> np.ndarray:
    """The seeded contexts of GPU `rank`'s 256 streams (log-uniform [64, 4096])."""
    rng = np.random.default_rng(WORKLOAD_SEED * 1_000_003 + rank * 65_536)
    return np.exp(rng.uniform(np.log(CTX_LO), np.log(CTX_HI), size=STREAMS_PER_GPU)).astype(np.int64).clip(CTX_LO, CTX_HI)


def box_lengths(rank: int, world: int) -> np.ndarray:
    """Whole-box workload: one seeded set of world x 256 streams (the union of
    every GPU's seeded contexts), partitioned over the ranks by greedy LPT on
    each stream's per-step KV read (its context length), 256 streams per rank
    (shard.lpt_partition).  world = 1 gives stream_lengths(0) unchanged."""
    if world == 1:
        return stream_lengths(0)
    import __graft_entry__ as ge
    ge.load_package()
    from qwenasr_cpp_b200 import shard
    pool = np.concatenate([stream_lengths(g) for g in range(world)])
    parts = shard.lpt_partition(pool, world, cap=STREAMS_PER_GPU)
    return pool[np.asarray(parts[rank], dtype=np.int64)]


def bind_numa(gpu: int) -> str | None:
    """Pin this process to the host cores of its GPU's NUMA node (before any
    pinned host buffer is allocated, so those pages land on that node).
    Best effort: returns the node, or None where the topology is not exposed."""
    try:
        import torch
        pr = torch.cuda.get_device_properties(gpu)
        bus = f"{pr.pci_domain_id:04x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
        node = int(Path(f"/sys/bus/pci/devices/{bus}/numa_node").read_text().strip())
        if node < 0:
            return None
        cpus = set()
        for part in Path(f"/sys/devices/system/node/node{node}/cpulist").read_text().strip().split(","):
            a, _, b = part.partition("-")
            cpus.update(range(int(a), int(b or a) + 1))
        os.sched_setaffinity(0, cpus)
        return f"node{node}"
    except Exception:
        return None


def qk_norm_weights(seed: int = 0):
    rng = np.random.default_rng(seed)
    qn = (1.0 + 0.02 * rng.standard_normal((N_LAYERS, D))).astype(np.float32)
    kn = (1.0 + 0.02 * rng.standard_normal((N_LAYERS, D))).astype(np.float32)
    return qn, kn


class ClockSampler:
    """SM clocks and clock-event (throttle) reasons sampled during the timed
    region: through NVML every 5 ms (read-only queries), else nvidia-smi
    every 0.2 s."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.rows = []
        self._stop = threading.Event()
        self._t = None
        # NVML set up here, before the timed region, so sampling starts with it
        self._nv, self._h = self._nvml_handle()
        self.source = "nvml 5 ms" if self._h is not None else "nvidia-smi 0.2 s"

    def _nvml_handle(self):
        try:
            import pynvml
            import torch
            pynvml.nvmlInit()
            pr = torch.cuda.get_device_properties(self.gpu)
            bus = f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
            return pynvml, pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            return None, None

    def _nvml_sample(self):
        nv, h = self._nv, self._h
        bits = (nv.nvmlClocksEventReasonHwSlowdown, nv.nvmlClocksEventReasonHwThermalSlowdown,
                nv.nvmlClocksEventReasonSwThermalSlowdown, nv.nvmlClocksEventReasonSwPowerCap)
        try:
            if not hasattr(self, "_mx"):
                self._mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
            sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
            rs = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
            self.rows.append([str(self.gpu), str(sm), str(self._mx), "", hex(rs)] +
                             ["Active" if rs & b else "Not Active" for b in bits])
        except Exception:
            pass

    def _run(self):
        if self._h is not None:
            while not self._stop.is_set():
                self._nvml_sample()
                self._stop.wait(0.005)
            return
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                      "--format=csv,noheader,nounits"], capture_output=True, text=True, timeout=5)
                if out.returncode == 0 and out.stdout.strip():
                    self.rows.append([c.strip() for c in out.stdout.strip().split(",")])
            except Exception:
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        if self._h is not None:
            self._nvml_sample()   # one sample as the timed region starts
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        self._t.join(timeout=10)
        if self._h is not None:
            self._nvml_sample()   # and one as it ends

    def summary(self) -> dict:
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if len(r) > 5 + i and "Active" in r[5 + i]
                          and "Not" not in r[5 + i]})
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows), "sampler": getattr(self, "source", None)}


def dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
        return rank, local, world, dist
    return 0, 0, 1, None


def barrier(dist):
    if dist is not None:
        dist.barrier()


def max_over_ranks(dist, v: float) -> float:
    import __graft_entry__ as ge
    ge.load_package()
    from qwenasr_cpp_b200 import shard
    return shard.reduce_max(dist, v, device="cuda" if dist is not None else None)


def sum_over_ranks(dist, v: float) -> float:
    import __graft_entry__ as ge
    ge.load_package()
    from qwenasr_cpp_b200 import shard
    return shard.reduce_sum(dist, v, device="cuda" if dist is not None else None)


# ------------------------------------------------------------------ CPU legs

def config4(kv_dtype: str, world: int, mean_ctx: float) -> dict:
    """The config of the default workload's line, shared by both arms."""
    return {"workload": "config4: KV append + GQA decode attention, 28 layers, 256 streams/GPU, "
                        "ctx log-uniform [64,4096], 16-token pages, permuted page table",
            "streams_per_gpu": STREAMS_PER_GPU, "mean_ctx": round(mean_ctx, 1),
            "kv_cache": f"{kv_dtype} paged",
            "parallelism": (f"streams sharded x{world}, no collectives" if world == 1 else
                            f"one seeded set of {world}x{STREAMS_PER_GPU} streams, LPT-partitioned on per-step KV "
                            f"read ({STREAMS_PER_GPU} per GPU), no collectives"),
            "l2": "inputs larger than L2 (per-layer KV read ~1 GB >> 126 MB)"}


def cpu_sample(lens: np.ndarray, n_streams: int) -> np.ndarray:
    """Context lengths of a CPU sample of n_streams streams that follows the
    whole workload's length distribution: the middle stream of each of
    n_streams equal rank bins of the sorted lengths (for config 4: mean 964.1
    against 957.5 for all 256 streams)."""
    s = np.sort(lens)
    bin_w = len(s) // n_streams
    return s[bin_w // 2::bin_w][:n_streams]


def cpu_kv_sample(lens: np.ndarray, n_streams: int, steps: int, threads: int, warmup: int = 1):
    """Time the reference arithmetic (oracle port, bit-exact with the reference's
    scalar path) on n_streams streams of this GPU's workload chosen by
    cpu_sample, after `warmup` untimed steps.  Returns (tokens/s, seconds,
    the sample's mean context before the first step)."""
    from oracle import oracle as checker

    sel = cpu_sample(lens, n_streams)
    rng = np.random.default_rng(7)
    # Cache contents: a random block tiled over the context (values do not change
    # the arithmetic's cost; filling GBs with fresh random numbers would dominate).
    appends = warmup + steps                      # every step, warm-up included, appends one token per stream
    block = rng.standard_normal((2, CTX_HI + appends + 2, HKV * D), dtype=np.float32)
    kcs, vcs = [], []
    for L in sel:
        cap = int(L) + appends + 2
        k = np.empty((N_LAYERS, cap, HKV * D), np.float32)
        v = np.empty((N_LAYERS, cap, HKV * D), np.float32)
        k[:] = block[0, :cap]
        v[:] = block[1, :cap]
        kcs.append(k)
        vcs.append(v)
    qn, kn = qk_norm_weights()
    cur = sel.astype(np.int32).copy()
    qkv = rng.standard_normal((N_LAYERS, len(sel), QKV), dtype=np.float32)
    for _ in range(warmup):   # untimed (the first pages the cache in)
        checker.kv_step_batch(qkv, qn, kn, kcs, vcs, cur, threads=threads)
    t0 = time.perf_counter()
    for _ in range(steps):
        checker.kv_step_batch(qkv, qn, kn, kcs, vcs, cur, threads=threads)
    dt = time.perf_counter() - t0
    return len(sel) * steps / dt, dt, float(sel.mean())


def run_reference(args) -> int:
    """--impl reference: the reference's CPU arithmetic for this path on the host
    cores (all threads), same workload definition, bounded sample per step."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    threads = os.cpu_count() or 1
    lens = stream_lengths(0)
    n = min(STREAMS_PER_GPU, 16)
    value, dt, sample_ctx = cpu_kv_sample(lens, n, max(args.steps, 1), threads, warmup=max(args.warmup, 1))
    per_step_ms = dt / max(args.steps, 1) * 1e3
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "tokens/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(per_step_ms, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config4(args.kv_dtype, args.gpus, float(lens.mean())),
        "cpu_baseline": {"value": round(value, 3), "unit": "tokens/s", "cores": threads, "kind": "port",
                         "cache": "f32 contiguous (the reference's layout)",
                         "sample_mean_ctx": round(sample_ctx, 1),
                         "sample": f"{n} of the {STREAMS_PER_GPU} streams of GPU 0 (the middle stream of each "
                                   f"of {n} equal rank bins of the sorted lengths) x {args.steps} steps "
                                   f"(after {max(args.warmup, 1)} untimed), in the reference's layout and arithmetic "
                                   f"(f32 contiguous cache; oracle/qkv_oracle.c, bit-exact with the reference scalar "
                                   f"path), OpenMP over streams"},
        "e2e": {"value": round(value, 3), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------ GPU leg

def run_ours(args) -> int:
    import torch

    global N_LAYERS
    N_LAYERS = args.layers
    import __graft_entry__ as ge
    pkg = ge.load_package()
    rank, local, world, dist = dist_setup(args.gpus)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    numa = bind_numa(local) if world > 1 else None

    lens = box_lengths(rank, world)
    total_steps = args.warmup + args.steps + 2 + 14   # + kernel-timing pass + e2e pass (1 + 10 steps)
    max_ctx = int(lens.max()) + total_steps + 16
    pages = int(sum((int(L) + total_steps + 15) // 16 for L in lens)) + 64
    qn, kn = qk_norm_weights()
    cfg = dict(n_layers=N_LAYERS, hidden=1024, n_heads=HQ, n_kv_heads=HKV, head_dim=D, intermediate=3072,
               vocab=151936, rope_theta=1.0e6, rms_norm_eps=1.0e-6)
    kvd = {"bf16": pkg.BF16, "fp8": pkg.FP8, "e4i8": pkg.E4I8, "f32": pkg.F32}[args.kv_dtype]
    elem = {"bf16": 2, "fp8": 1, "e4i8": 1, "f32": 4}[args.kv_dtype]
    rt = pkg.runtime_config(device=local, weight_dtype=pkg.F32, kv_dtype=kvd, max_streams=STREAMS_PER_GPU,
                            max_context=max_ctx, max_pages=pages, page_order_seed=WORKLOAD_SEED + rank)
    dec = pkg.Decoder.kv_only(cfg, rt, qn, kn)
    streams = [dec.open() for _ in range(STREAMS_PER_GPU)]
    for s, L in zip(streams, lens):
        dec.extend(s, int(L))
    dec.fill_random(WORKLOAD_SEED + rank)

    g = torch.Generator(device=dev).manual_seed(WORKLOAD_SEED + rank)
    qkv = torch.randn((N_LAYERS, STREAMS_PER_GPU, QKV), device=dev, generator=g)
    out = torch.empty((N_LAYERS, STREAMS_PER_GPU, HQ * D), device=dev)
    st = torch.cuda.current_stream(dev)
    sp = st.cuda_stream

    def step():
        dec.kv_step(streams, qkv.data_ptr(), out.data_ptr(), sp)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    dec.sync()

    launches0 = dec.launches()
    sampler = ClockSampler(local)
    barrier(dist)
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with sampler:
        e0.record(st)
        for _ in range(args.steps):
            step()
        e1.record(st)
        torch.cuda.synchronize(dev)
    barrier(dist)
    ms = e0.elapsed_time(e1)
    launches = dec.launches() - launches0
    dec.sync()
    ms_max = max_over_ranks(dist, ms)
    tokens = sum_over_ranks(dist, float(STREAMS_PER_GPU * args.steps))
    value = tokens / (ms_max / 1e3)

    # K2 alone: the dominant kernel, timed per launch on the same stream, every layer.
    n_rep = 2
    cur_lens = torch.tensor([dec.length(s) for s in streams], dtype=torch.int32, device=dev)
    slots = torch.tensor(streams, dtype=torch.int32, device=dev)
    q_in = torch.randn((STREAMS_PER_GPU, HQ * D), device=dev, generator=g)
    o_buf = torch.empty_like(q_in)
    torch.cuda.synchronize(dev)
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a0.record(st)
    for _ in range(n_rep):
        for layer in range(N_LAYERS):
            dec.kv_attend(layer, STREAMS_PER_GPU, slots.data_ptr(), cur_lens.data_ptr(), q_in.data_ptr(),
                          o_buf.data_ptr(), sp)
    a1.record(st)
    torch.cuda.synchronize(dev)
    dec.sync()
    attn_ms = a0.elapsed_time(a1) / (n_rep * N_LAYERS)
    ctx_tokens = int(cur_lens.sum().item())
    kv_bytes_per_launch = ctx_tokens * HKV * D * 2 * elem       # K and V, one layer
    if elem == 1:
        kv_bytes_per_launch += sum((dec.length(s) + 15) // 16 for s in streams) * 2 * HKV * 16 * 4   # 8-bit scales: one per (token, head) of K and V
    achieved_gbs = kv_bytes_per_launch / (attn_ms / 1e3) / 1e9
    probe = read_probe(pkg, dec, streams, elem, st, attn_ms)

    # e2e: the same step through the C ABI with pinned host buffers (copies in the timed region).
    e2e_steps = 10
    h_qkv = torch.randn((N_LAYERS, STREAMS_PER_GPU, QKV), generator=torch.Generator().manual_seed(3)).pin_memory()
    h_out = torch.empty((N_LAYERS, STREAMS_PER_GPU, HQ * D)).pin_memory()
    dec.kv_step_host(streams, h_qkv.data_ptr(), h_out.data_ptr())    # warm
    barrier(dist)
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        dec.kv_step_host(streams, h_qkv.data_ptr(), h_out.data_ptr())
    box_mean = sum_over_ranks(dist, float(lens.sum())) / (world * STREAMS_PER_GPU)
    e2e_rank_s = time.perf_counter() - t0
    e2e_s = max_over_ranks(dist, e2e_rank_s)
    e2e_value = sum_over_ranks(dist, float(STREAMS_PER_GPU * e2e_steps)) / e2e_s
    per_rank = [STREAMS_PER_GPU * e2e_steps / e2e_rank_s]
    k2_frac_ranks = [achieved_gbs / peaks()["hbm_gbs"]]
    if dist is not None:
        gathered = [None] * world
        dist.all_gather_object(gathered, (per_rank[0], k2_frac_ranks[0], numa))
        per_rank = [g[0] for g in gathered]
        k2_frac_ranks = [g[1] for g in gathered]
        numa_ranks = [g[2] for g in gathered]

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        threads = os.cpu_count() or 1
        n_cpu = min(STREAMS_PER_GPU, 16)
        cpu_val, _, sample_ctx = cpu_kv_sample(lens, n_cpu, 1, threads)
        cpu = {"value": round(cpu_val, 3), "unit": "tokens/s", "cores": threads, "kind": "port",
               "sample_mean_ctx": round(sample_ctx, 1),
               "sample": f"{n_cpu} streams (the middle stream of each of {n_cpu} equal rank bins of the "
                         f"sorted lengths) x 1 step of this workload on the host cores "
                         f"(oracle/qkv_oracle.c, bit-exact with the reference scalar path)"}

    pk = peaks()
    if rank == 0:
        mean_ctx = box_mean   # the configured contexts, before any step (as the reference arm)
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": args.kv_dtype,
            "data": "synthetic",
            "config": config4(args.kv_dtype, world, mean_ctx),
            "kv_read_gbs_step": round(kv_bytes_per_launch * N_LAYERS / (ms_max / args.steps / 1e3) / 1e9, 1),
            "roofline": {"bound": "hbm", "achieved": round(achieved_gbs, 1), "peak": pk["hbm_gbs"], "unit": "GB/s",
                         "frac": round(achieved_gbs / pk["hbm_gbs"], 4), "frac_of_8tbs": round(achieved_gbs / 8000, 4),
                         "traffic": {"bf16": K2_NCU_TRAFFIC_BYTES}.get(args.kv_dtype),
                         "kernel": "decode_attn_kernel (K2)",
                         "launch_ms": round(attn_ms, 4), "bytes_per_launch": kv_bytes_per_launch,
                         "peak_source": pk["source"], "read_probe": probe,
                         "frac_per_rank": [round(v, 4) for v in k2_frac_ranks]},
            "e2e": {"value": round(e2e_value, 2), "unit": "tokens/s",
                    "h2d_bytes_per_step": int(qkv.numel() * 4), "d2h_bytes_per_step": int(out.numel() * 4),
                    "per_rank": [round(v, 1) for v in per_rank]},
            "gpu_launches": int(launches),
            "clocks": sampler.summary(),
        }
        if world > 1:
            line["numa_per_rank"] = numa_ranks
        if cpu is not None:
            line["cpu_baseline"] = cpu
    dec.close()
    if not args.no_model:
        # The full model step the ASR user runs (config 2: 0.6B, 32 streams per
        # GPU, greedy decode), measured after the KV step on the same ranks.
        margs = argparse.Namespace(**vars(args))
        margs.steps, margs.warmup, margs.weights = 50, 3, "bf16"
        m = run_model(margs, ctx=(rank, local, world, dist), big=False)
        if rank == 0 and m is not None:
            line["model_decode_config2"] = {"value": m["value"], "unit": "tokens/s", "ms_per_step": m["ms_per_step"],
                                            "steps": 50, "n_gpus": world, "metric": m["metric"]}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()
    return 0


def read_probe(pkg, dec, streams, elem: int, st, attn_ms: float | None, reps: int = 2) -> dict | None:
    """The read ceiling of K2's access pattern on this workload: the same
    pages of every stream (K2's order), the same persistent grid and page
    split, one bulk copy per page into shared memory, nothing computed
    (qkv_page_read_probe), one launch per layer, timed with CUDA events on
    the launching stream.  k2_time_frac = probe time / K2 time over the same
    pages (1.0 = K2 streams as fast as a pure read of its pages)."""
    import torch
    if elem > 2:
        return None
    plist = np.concatenate([dec.pages(s) for s in streams]).astype(np.int32)
    d_pages = torch.tensor(plist, device=torch.device("cuda", torch.cuda.current_device()))
    page_bytes = 2 * HKV * 16 * D * elem
    sp = st.cuda_stream
    for layer in range(N_LAYERS):   # warm (one pass)
        rc = pkg.lib.qkv_page_read_probe(dec.h, layer, len(plist), d_pages.data_ptr(), sp)
        if rc != 0:
            raise RuntimeError(f"qkv_page_read_probe failed: {rc}")
    torch.cuda.synchronize()
    b0, b1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    b0.record(st)
    for _ in range(reps):
        for layer in range(N_LAYERS):
            pkg.lib.qkv_page_read_probe(dec.h, layer, len(plist), d_pages.data_ptr(), sp)
    b1.record(st)
    torch.cuda.synchronize()
    dec.sync()
    ms = b0.elapsed_time(b1) / (reps * N_LAYERS)
    gbs = len(plist) * page_bytes / (ms / 1e3) / 1e9
    out = {"gbs": round(gbs, 1), "launch_ms": round(ms, 4), "pages": int(len(plist)), "page_bytes": page_bytes,
           "frac_of_copy_peak": round(gbs / peaks()["hbm_gbs"], 4)}
    if attn_ms:
        out["k2_time_frac"] = round(ms / attn_ms, 4)
    return out


def run_readprobe(args) -> int:
    """--workload readprobe: the read ceiling of K2's page stream on the
    config-4 cache (same streams, contexts, page permutation and dtype as the
    default line; nothing is appended).  value = page bytes read per second,
    whole job (sum over ranks of bytes, max over ranks of time)."""
    import torch

    global N_LAYERS
    N_LAYERS = args.layers
    import __graft_entry__ as ge
    pkg = ge.load_package()
    rank, local, world, dist = dist_setup(args.gpus)
    torch.cuda.set_device(local)
    lens = stream_lengths(rank)
    qn, kn = qk_norm_weights()
    cfg = dict(n_layers=N_LAYERS, hidden=1024, n_heads=HQ, n_kv_heads=HKV, head_dim=D, intermediate=3072,
               vocab=151936, rope_theta=1.0e6, rms_norm_eps=1.0e-6)
    kvd = {"bf16": pkg.BF16, "fp8": pkg.FP8, "e4i8": pkg.E4I8}[args.kv_dtype]
    elem = 2 if args.kv_dtype == "bf16" else 1
    rt = pkg.runtime_config(device=local, weight_dtype=pkg.F32, kv_dtype=kvd, max_streams=STREAMS_PER_GPU,
                            max_context=int(lens.max()) + 16, max_pages=int(sum((int(L) + 15) // 16 for L in lens)) + 64,
                            page_order_seed=WORKLOAD_SEED + rank)
    with pkg.Decoder.kv_only(cfg, rt, qn, kn) as dec:
        streams = [dec.open() for _ in range(STREAMS_PER_GPU)]
        for s, L in zip(streams, lens):
            dec.extend(s, int(L))
        dec.fill_random(WORKLOAD_SEED + rank)
        st = torch.cuda.current_stream()
        sampler = ClockSampler(local)
        barrier(dist)
        with sampler:
            probe = read_probe(pkg, dec, streams, elem, st, None, reps=max(args.steps, 1))
        barrier(dist)
    ms = max_over_ranks(dist, probe["launch_ms"])
    total = sum_over_ranks(dist, float(probe["pages"] * probe["page_bytes"]))
    if rank == 0:
        gbs = total / (ms / 1e3) / 1e9
        print(json.dumps({
            "metric": "KV page-stream read GB/s (read probe of the decode-attention access pattern)",
            "value": round(gbs, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": 1,
            "ms_per_step": round(ms, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": args.kv_dtype, "data": "synthetic", "config": config4(args.kv_dtype, world, float(lens.mean())),
            "roofline": {"bound": "hbm", "achieved": round(gbs / world, 1), "peak": peaks()["hbm_gbs"], "unit": "GB/s",
                         "frac": round(gbs / world / peaks()["hbm_gbs"], 4), "traffic": None,
                         "kernel": "page_read_probe_kernel", "peak_source": peaks()["source"]},
            "clocks": sampler.summary()}), flush=True)
    if dist is not None:
        dist.destroy_process_group()
    return 0


def run_model(args, ctx=None, big=None):
    """Config 2: 0.6B, bf16 weights + bf16 paged cache, 32 streams/GPU, prompts
    U[100, 400] with 90% audio rows, greedy decode; value = decode tokens/s
    (config 3 with --workload model3).  With ctx = (rank, local, world, dist)
    from a caller that already set up the ranks, returns rank 0's line as a
    dict (None elsewhere) instead of printing it, and leaves the process
    group to the caller."""
    import tempfile

    import torch

    import __graft_entry__ as ge
    pkg = ge.load_package()
    synth = ge.load_synth()
    rank, local, world, dist = ctx if ctx is not None else dist_setup(args.gpus)
    torch.cuda.set_device(local)
    if big is None:
        big = args.workload == "model3"
    cfg = dict(synth.QWEN3_ASR_1_7B if big else synth.QWEN3_ASR_0_6B)
    n_streams = 64 if big else 32
    steps = args.steps
    tmpdir = Path(os.environ.get("QWENASR_BENCH_TMP", "/dev/shm" if Path("/dev/shm").is_dir() else tempfile.gettempdir()))
    audio_hidden = 896 if big else 0   # config 3 also runs the audio projector (encoder width 896)
    path = tmpdir / f"qwen3asr_{'1p7b' if big else '0p6b'}_bf16_seed0{'_ap' if big else ''}_r{rank}.gguf"
    t0 = time.perf_counter()
    if not path.exists():
        synth.write_gguf(path, cfg, seed=0, weights="bf16", norm_init="normal", tokenizer=False,
                         audio_hidden=audio_hidden)
    gen_s = time.perf_counter() - t0
    embd = synth.read_gguf(path)["text.token_embd.weight"]
    prompt_ids = []
    if big:   # config 3: 390 audio rows + 20 text tokens per stream
        prompts = []
        for sidx in range(n_streams):
            rng = np.random.default_rng(1003 * 1_000_003 + rank * 65_536 + sidx)
            x, ids = synth.prompt_rows(embd, 410, rng, audio_rows=390, audio_start=9)
            prompts.append(x)
            prompt_ids.append(ids)
    else:
        prompts = synth.config2_prompts(embd, n_streams, seed=1002, gpu=rank)
    max_ctx = max(p.shape[0] for p in prompts) + args.warmup + steps + 8
    wdt = {"bf16": pkg.BF16, "fp8": pkg.FP8}[args.weights]
    rt = pkg.runtime_config(device=local, weight_dtype=wdt, kv_dtype=pkg.BF16, max_streams=n_streams,
                            max_context=max_ctx, max_batch_tokens=sum(p.shape[0] for p in prompts),
                            page_order_seed=1002 + rank)
    dec = pkg.Decoder.from_gguf(path, rt, cfg)
    streams = [dec.open() for _ in prompts]
    torch.cuda.synchronize()
    t1 = time.perf_counter()
    dec.prefill(streams, prompts)
    prefill_s = time.perf_counter() - t1
    for _ in range(args.warmup):
        dec.decode_step(streams)
    launches0 = dec.launches()
    sampler = ClockSampler(local)
    barrier(dist)
    with sampler:
        t2 = time.perf_counter()
        for _ in range(steps):
            dec.decode_step(streams)
        dt = time.perf_counter() - t2
    launches = dec.launches() - launches0
    dt_max = max_over_ranks(dist, dt)
    tokens = sum_over_ranks(dist, float(n_streams * steps))
    prefill_cmp = {}
    if big:
        # Warm prefill of the same prompts on fresh streams, two ways: rows
        # uploaded from the host (qkv_prefill_rows), and ids with the audio rows
        # already on the device, as an audio encoder on the GPU leaves them
        # (qkv_prefill_ids: the embedding gather and splice run on the device).
        aid = synth.TOKEN_IDS["audio"]
        ids_l, audio_l = [], []
        for x, ids in zip(prompts, prompt_ids):
            ids = ids.copy()
            ids[ids == aid] = 0
            ids[9:399] = aid
            ids_l.append(ids)
            audio_l.append(torch.tensor(x[9:399], device=torch.device("cuda", local)))
        for s_ in streams:
            dec.close_stream(s_)

        def timed(fn) -> float:
            ss = [dec.open() for _ in prompts]
            torch.cuda.synchronize()
            t = time.perf_counter()
            fn(ss)
            torch.cuda.synchronize()
            d = time.perf_counter() - t
            for s_ in ss:
                dec.close_stream(s_)
            return d

        rows_s = min(timed(lambda ss: dec.prefill(ss, prompts)) for _ in range(2))
        ids_s = min(timed(lambda ss: dec.prefill_ids(ss, ids_l, audio_l, aid)) for _ in range(2))
        # From audio-encoder rows on the device: projector, then the same prefill.
        # All streams' encoder rows in one block, projected by one call.
        gdev = torch.Generator(device=torch.device("cuda", local)).manual_seed(1003 + rank)
        n_enc = 390 * len(prompts)
        enc = torch.randn((n_enc, audio_hidden), device=torch.device("cuda", local), generator=gdev)
        proj = torch.empty((n_enc, cfg["hidden"]), device=torch.device("cuda", local))
        proj_l = [proj[390 * k:390 * (k + 1)] for k in range(len(prompts))]

        def project():
            dec.audio_project(n_enc, enc.data_ptr(), proj.data_ptr())

        project()
        torch.cuda.synchronize()
        pe0, pe1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        pe0.record()
        project()
        pe1.record()
        torch.cuda.synchronize()
        proj_ms = pe0.elapsed_time(pe1)
        enc_s = min(timed(lambda ss: (project(), dec.prefill_ids(ss, ids_l, proj_l, aid))) for _ in range(2))
        T = int(sum(p.shape[0] for p in prompts))
        prefill_cmp = {"prefill_warm_rows_s": round(rows_s, 4), "prefill_warm_ids_device_audio_s": round(ids_s, 4),
                       "prefill_warm_from_encoder_rows_s": round(enc_s, 4),
                       "audio_projector_ms": round(proj_ms, 3),
                       "audio_projector_tflops": round(n_enc * 2.0 * audio_hidden *
                                       (audio_hidden + cfg["hidden"]) / (proj_ms / 1e3) / 1e12, 1),
                       "prefill_h2d_bytes_rows": T * cfg["hidden"] * 4, "prefill_h2d_bytes_ids": T * 4}
        streams = []
    if rank == 0:
        line = {
            "metric": f"greedy decode tokens/s (full {'1.7B' if big else '0.6B'} step: KV path + projections + LM head)",
            "value": round(tokens / dt_max, 2), "unit": "tokens/s", "n_gpus": world, "steps": steps,
            "warmup": args.warmup, "ms_per_step": round(dt_max / steps * 1e3, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16" if args.weights == "bf16" else "fp8 projections (e4m3), bf16 elsewhere",
            "data": "synthetic",
            "config": {"weights": args.weights,
                       "workload": ("config3: Qwen3-ASR-1.7B bf16 weights + bf16 paged KV, 64 streams/GPU, "
                                    "390 audio rows + 20 text tokens, greedy decode") if big else
                                   ("config2: Qwen3-ASR-0.6B bf16 weights + bf16 paged KV, 32 streams/GPU, "
                                    "prompts U[100,400] (90% audio rows), greedy decode"),
                       "prompt_tokens": int(sum(p.shape[0] for p in prompts)), "prefill_s": round(prefill_s, 3),
                       "gguf_write_s": round(gen_s, 1), **prefill_cmp},
            "e2e": {"value": round(tokens / dt_max, 2), "unit": "tokens/s", "h2d_bytes_per_step": n_streams * 4 * 4,
                    "d2h_bytes_per_step": n_streams * 4, "note": "qkv_decode_step with host id buffers"},
            "gpu_launches": int(launches), "clocks": sampler.summary()}
        if ctx is None:
            print(json.dumps(line), flush=True)
    dec.close()
    if ctx is not None:
        return line if rank == 0 else None
    if dist is not None:
        dist.destroy_process_group()
    return 0


def gguf_path(synth, cfg, name: str, rank: int) -> tuple[Path, float]:
    import tempfile
    tmpdir = Path(os.environ.get("QWENASR_BENCH_TMP", "/dev/shm" if Path("/dev/shm").is_dir() else tempfile.gettempdir()))
    path = tmpdir / f"qwen3asr_{name}_bf16_seed0_r{rank}.gguf"
    t0 = time.perf_counter()
    if not path.exists():
        synth.write_gguf(path, cfg, seed=0, weights="bf16", norm_init="normal", tokenizer=False)
    return path, time.perf_counter() - t0


def run_serve(args) -> int:
    """Config 5: 1.7B, FP8-e4m3 paged cache (per-page-per-head scales), continuous
    batching.  512 requests are admitted at start; each timed step first admits
    Poisson(lambda) new requests (chunked prefill), then decodes one token for
    every active stream, closes streams that reached their output length (pages
    freed) and compacts the pool every 64 steps.  lambda = concurrency / mean
    output length keeps ~512 streams in flight.  value = decoded tokens / wall
    time of the timed steps (arrival prefills, closes and compaction included)."""
    import torch

    import __graft_entry__ as ge
    pkg = ge.load_package()
    synth = ge.load_synth()
    rank, local, world, dist = dist_setup(args.gpus)
    torch.cuda.set_device(local)
    cfg = dict(synth.QWEN3_ASR_1_7B)
    path, gen_s = gguf_path(synth, cfg, "1p7b", rank)
    embd = synth.read_gguf(path)["text.token_embd.weight"]
    conc = args.concurrency
    rng = np.random.default_rng(1005 * 1_000_003 + rank * 65_536)
    text_tokens, out_lo, out_hi = 20, 32, 512
    lam = conc / ((out_lo + out_hi) / 2.0)
    max_ctx = 780 + text_tokens + out_hi + 8
    slots_cap = conc + 128
    serve_kv = {"e4i8": pkg.E4I8, "fp8": pkg.FP8}[args.serve_kv]
    rt = pkg.runtime_config(device=local, weight_dtype={"bf16": pkg.BF16, "fp8": pkg.FP8}[args.weights],
                            kv_dtype=serve_kv, max_streams=slots_cap,
                            max_context=max_ctx, max_pages=slots_cap * ((max_ctx + 15) // 16),
                            max_batch_tokens=32768, page_order_seed=1005 + rank)
    dec = pkg.Decoder.from_gguf(path, rt, cfg)
    active: dict[int, int] = {}

    def make_request():
        audio = int(rng.integers(65, 781))
        x, _ = synth.prompt_rows(embd, audio + text_tokens, rng, audio_rows=audio, audio_start=9)
        return x, int(rng.integers(out_lo, out_hi + 1))

    # Requests are synthesised before any timing: per step a Poisson count of arrivals.
    arrivals = [[make_request() for _ in range(int(rng.poisson(lam)))] for _ in range(args.warmup + args.steps)]
    phase = {"prefill_s": 0.0, "decode_s": 0.0, "close_s": 0.0, "compact_s": 0.0}

    def admit(pending) -> int:
        reqs = []
        for r in pending:
            if len(active) + len(reqs) >= slots_cap:
                break
            reqs.append(r)
        tokens = 0
        i = 0
        while i < len(reqs):   # chunked by the handle's prompt-token budget
            chunk, budget = [], 0
            while i < len(reqs) and budget + reqs[i][0].shape[0] <= 32768:
                chunk.append(reqs[i])
                budget += reqs[i][0].shape[0]
                i += 1
            streams = [dec.open() for _ in chunk]
            dec.prefill(streams, [c[0] for c in chunk])
            for s, (_, n_out) in zip(streams, chunk):
                active[s] = n_out - 1      # the prefill produced the first token
            tokens += budget
        return tokens

    t0 = time.perf_counter()
    admit([make_request() for _ in range(conc)])
    fill_s = time.perf_counter() - t0
    decoded = prefill_tokens = closed = moved = 0
    conc_seen = []
    sampler = ClockSampler(local)

    def step(k: int, timed: bool):
        nonlocal decoded, prefill_tokens, closed, moved
        ta = time.perf_counter()
        pt = admit(arrivals[k])
        tb = time.perf_counter()
        streams = list(active.keys())
        dec.decode_step(streams)
        tc = time.perf_counter()
        for s in streams:
            active[s] -= 1
            if active[s] <= 0:
                dec.close_stream(s)
                del active[s]
                closed += timed
        td = time.perf_counter()
        if timed:
            decoded += len(streams)
            prefill_tokens += pt
            conc_seen.append(len(streams))
            phase["prefill_s"] += tb - ta
            phase["decode_s"] += tc - tb
            phase["close_s"] += td - tc

    for k in range(args.warmup):
        step(k, False)
    barrier(dist)
    with sampler:
        t1 = time.perf_counter()
        for k in range(args.steps):
            step(args.warmup + k, True)
            if (k + 1) % 64 == 0:
                tc0 = time.perf_counter()
                moved += dec.compact()
                phase["compact_s"] += time.perf_counter() - tc0
        torch.cuda.synchronize()
        dt = time.perf_counter() - t1
    dt_max = max_over_ranks(dist, dt)
    total = sum_over_ranks(dist, float(decoded))
    free_pages, total_pages = dec.pool_stats()
    dec.close()

    # Deviation of the 8-bit caches vs the bf16 cache: 8 config-5 prompts, the
    # bf16-cache path's greedy ids teacher-force the 8-bit-cache paths.
    dev_line = None
    if rank == 0:
        drng = np.random.default_rng(4242)
        prompts = []
        for _ in range(8):
            audio = int(drng.integers(65, 781))
            x, _ = synth.prompt_rows(embd, audio + text_tokens, drng, audio_rows=audio, audio_start=9)
            prompts.append(x)
        n_steps = 32
        outs = {}
        for kvd in (pkg.BF16, pkg.E4I8, pkg.FP8):
            rt2 = pkg.runtime_config(device=local, weight_dtype=pkg.BF16, kv_dtype=kvd, max_streams=8,
                                     max_context=max_ctx, max_batch_tokens=8 * 800)
            with pkg.Decoder.from_gguf(path, rt2, cfg) as d2:
                ss = [d2.open() for _ in prompts]
                ids, lg = d2.prefill(ss, prompts, want_logits=True)
                steps_ids, steps_lg = [ids], [lg]
                for t in range(n_steps - 1):
                    feed = outs[pkg.BF16][0][t] if kvd != pkg.BF16 else steps_ids[-1]
                    ids, lg = d2.decode_step(ss, in_ids=feed, want_logits=True)
                    steps_ids.append(ids)
                    steps_lg.append(lg)
                outs[kvd] = (steps_ids, steps_lg)
        dev_line = {"streams": 8, "steps": n_steps}
        for name, kvd in (("e4i8", pkg.E4I8), ("fp8", pkg.FP8)):
            agree = np.mean([np.mean(a == b) for a, b in zip(outs[pkg.BF16][0], outs[kvd][0])])
            rel = max(float(np.max(np.abs(a - b)) / np.max(np.abs(b))) for a, b in zip(outs[kvd][1], outs[pkg.BF16][1]))
            dev_line[name] = {"greedy_agreement_vs_bf16": round(float(agree), 4),
                              "max_rel_logit_dev_vs_bf16": float(f"{rel:.3e}")}
    if rank == 0:
        line = {
            "metric": "serving decode tokens/s (1.7B, 8-bit KV cache, continuous batching)",
            "value": round(total / dt_max, 2), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(dt_max / args.steps * 1e3, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16 weights, " + ("e4m3 K + int8 V" if args.serve_kv == "e4i8" else "e4m3 K and V") + " KV",
            "data": "synthetic",
            "config": {"workload": "config5: Qwen3-ASR-1.7B, 8-bit paged KV (f32 scale per stored token and head), Poisson arrivals, "
                                   "audio 65-780 rows + 20 text tokens, outputs 32-512 tokens",
                       "kv_cache": args.serve_kv,
                       "target_concurrency": conc, "mean_concurrency": round(float(np.mean(conc_seen)), 1),
                       "arrival_rate_per_step": round(lam, 3), "initial_fill_s": round(fill_s, 2),
                       "prefill_tokens_timed": int(prefill_tokens), "streams_closed": int(closed),
                       "pages_moved_by_compaction": int(moved), "free_pages_end": int(free_pages),
                       "pool_pages": int(total_pages), "gguf_write_s": round(gen_s, 1),
                       "phase_s": {k: round(v, 3) for k, v in phase.items()}},
            "deviation_vs_bf16_cache": dev_line,
            "clocks": sampler.summary()}
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()
    return 0



# ------------------------------------------------------------------ operator legs

PREFILL_STREAMS, PREFILL_TOKENS = 64, 410      # config 3's prompts: 390 audio rows + 20 text tokens


def run_prefill_attn(args) -> int:
    """K3 on its own: causal prefill attention over 28 layers of a paged cache
    holding config-3 prompts (64 streams x 410 tokens per GPU), through
    qkv_prefill_attend_q16 (queries in the kernel's operand form, as the fused
    append writes them in a prefill).  A step = one launch per layer (every layer's cache is
    a different 107 MB block (bf16), so 28 of them exceed L2 between reuses).
    value = useful attention TFLOP/s (QK^T and PV of the causal triangle, 16 q
    heads, D = 128); roofline against the measured dense bf16 peak."""
    global N_LAYERS
    N_LAYERS = args.layers
    import torch

    import __graft_entry__ as ge
    pkg = ge.load_package()
    rank, local, world, dist = dist_setup(args.gpus)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    n, P = PREFILL_STREAMS, PREFILL_TOKENS
    qn, kn = qk_norm_weights()
    cfg = dict(n_layers=N_LAYERS, hidden=1024, n_heads=HQ, n_kv_heads=HKV, head_dim=D, intermediate=3072,
               vocab=151936, rope_theta=1.0e6, rms_norm_eps=1.0e-6)
    kvd = {"bf16": pkg.BF16, "fp8": pkg.FP8, "e4i8": pkg.E4I8, "f32": pkg.F32}[args.kv_dtype]
    rt = pkg.runtime_config(device=local, weight_dtype=pkg.F32, kv_dtype=kvd, max_streams=n, max_context=P + 16,
                            max_batch_tokens=n * P, page_order_seed=WORKLOAD_SEED + rank)
    dec = pkg.Decoder.kv_only(cfg, rt, qn, kn)
    streams = [dec.open() for _ in range(n)]
    for s_ in streams:
        dec.extend(s_, P)
    dec.fill_random(WORKLOAD_SEED + rank)
    g = torch.Generator(device=dev).manual_seed(WORKLOAD_SEED + rank)
    q = torch.randn((n * P, HQ * D), device=dev, generator=g)
    out = torch.empty_like(q)
    st = torch.cuda.current_stream(dev)
    lens = [P] * n
    q_scale = float(np.float32(1.4426950408889634 / np.sqrt(float(D))))
    q16 = (q * q_scale).to(torch.float16 if args.kv_dtype in ("fp8", "e4i8") else torch.bfloat16)
    tc = args.kv_dtype != "f32"

    def step():
        for layer in range(N_LAYERS):
            if tc:
                dec.prefill_attend_q16(layer, streams, lens, q16.data_ptr(), out.data_ptr(), st.cuda_stream)
            else:
                dec.prefill_attend(layer, streams, lens, q.data_ptr(), out.data_ptr(), st.cuda_stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    dec.sync()
    barrier(dist)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as sampler:
        torch.cuda.synchronize(dev)
        e0.record(st)
        for _ in range(args.steps):
            step()
        e1.record(st)
        torch.cuda.synchronize(dev)
    dec.sync()
    ms = max_over_ranks(dist, e0.elapsed_time(e1))
    flops_launch = n * HQ * D * 4 * (P * (P + 1) / 2)
    tflops = flops_launch * N_LAYERS * args.steps * world / (ms / 1e3) / 1e12
    per_gpu = flops_launch * N_LAYERS * args.steps / (ms / 1e3) / 1e12
    pk = peaks()
    if rank == 0:
        line = {
            "metric": "prefill attention TFLOP/s (K3, causal, paged cache)", "value": round(tflops, 2),
            "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": args.kv_dtype + " cache", "data": "synthetic",
            "config": {"workload": f"K3 over config-3 prompts: {n} streams x {P} tokens per GPU, 28 layers of "
                                   f"{args.kv_dtype} paged cache, permuted pages, one launch per layer",
                       "flops_per_launch": flops_launch},
            "roofline": {"bound": "tensor", "achieved": round(per_gpu, 1), "peak": pk["bf16_tflops"],
                         "unit": "TFLOP/s", "frac": round(per_gpu / pk["bf16_tflops"], 4), "traffic": None,
                         "kernel": "prefill_attn_tc_kernel (K3)" if args.kv_dtype != "f32" else "prefill_attn_kernel",
                         "launch_ms": round(ms / args.steps / N_LAYERS, 4), "peak_source": pk["source"]},
            "gpu_launches": int(dec.launches()),
            "clocks": sampler.summary(),
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()
    return 0


GEMM_SHAPES = {   # name: (N, K) of the decoder projections (W [N][K])
    "qkv_0.6B": (4096, 1024), "o_0.6B": (1024, 2048), "gate_up_0.6B": (6144, 1024), "down_0.6B": (1024, 3072),
    "qkv_1.7B": (4096, 2048), "o_1.7B": (2048, 2048), "gate_up_1.7B": (12288, 2048), "down_1.7B": (2048, 6144),
}


def run_gemm(args) -> int:
    """The tcgen05 projection GEMM (qkv_gemm_bf16) on every decoder projection
    shape at a decode batch (M = 32, 64) and a prefill batch (M = 1024); each
    shape is launched 20 times inside one CUDA graph over 4 weight copies.
    value = FLOP-weighted TFLOP/s over all shapes."""
    import torch

    import __graft_entry__ as ge
    pkg = ge.load_package()
    rank, local, world, dist = dist_setup(args.gpus)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    rows, tot_flop, tot_ms = [], 0.0, 0.0
    reps = 20
    f8 = args.weights == "fp8"
    for M in (32, 64, 1024):
        for name, (N, K) in GEMM_SHAPES.items():
            if f8:   # e4m3 codes + one scale per row (the scales' values do not change the timing)
                ws = [torch.randint(0, 120, (N, K), device=dev, dtype=torch.uint8) for _ in range(4)]
                x = torch.randint(0, 120, (M, K), device=dev, dtype=torch.uint8)
                w_s, x_s = torch.ones(N, device=dev), torch.ones(M, device=dev)
            else:
                ws = [torch.randn(N, K, device=dev).to(torch.bfloat16) for _ in range(4)]
                x = torch.randn(M, K, device=dev).to(torch.bfloat16)
            c = torch.empty(M, N, device=dev)

            def call(i, st):
                if f8:
                    rc = pkg.lib.qkv_gemm_fp8(x.data_ptr(), x_s.data_ptr(), ws[i % 4].data_ptr(), w_s.data_ptr(),
                                              c.data_ptr(), M, N, K, 0, st)
                else:
                    rc = pkg.lib.qkv_gemm_bf16(x.data_ptr(), ws[i % 4].data_ptr(), c.data_ptr(), M, N, K, 0, st)
                if rc != 0:
                    raise RuntimeError(f"projection GEMM failed: {rc}")

            for i in range(args.warmup):
                call(i, torch.cuda.current_stream(dev).cuda_stream)
            torch.cuda.synchronize(dev)
            graph, side = torch.cuda.CUDAGraph(), torch.cuda.Stream(dev)
            with torch.cuda.stream(side):
                with torch.cuda.graph(graph, stream=side):
                    for i in range(reps):
                        call(i, side.cuda_stream)
            graph.replay()
            torch.cuda.synchronize(dev)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(args.steps):
                graph.replay()
            e1.record()
            torch.cuda.synchronize(dev)
            ms = e0.elapsed_time(e1) / (args.steps * reps)
            fl = 2.0 * M * N * K
            tot_flop += fl
            tot_ms += ms
            rows.append({"M": M, "shape": name, "N": N, "K": K, "us": round(ms * 1e3, 2),
                         "tflops": round(fl / (ms / 1e3) / 1e12, 1),
                         "weight_gbs": round(N * K * (1 if f8 else 2) / (ms / 1e3) / 1e9, 1)})
            del graph
    pk = peaks()
    value = tot_flop / (tot_ms / 1e3) / 1e12
    if rank == 0:
        line = {
            "metric": "projection GEMM TFLOP/s (tcgen05, " + ("e4m3 x e4m3" if f8 else "bf16 x bf16") + " -> f32)",
            "value": round(value, 2),
            "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(tot_ms, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "e4m3" if f8 else "bf16", "data": "synthetic",
            "config": {"workload": "decoder projections of 0.6B and 1.7B at M = 32, 64, 1024 tokens; "
                                   "20 launches per CUDA graph, 4 weight copies", "shapes": rows},
            "roofline": {"bound": "tensor", "achieved": round(value, 1),
                         "peak": pk["bf16_tflops"] * (2 if f8 else 1), "unit": "TFLOP/s",
                         "frac": round(value / (pk["bf16_tflops"] * (2 if f8 else 1)), 4), "traffic": None,
                         "kernel": "gemm_tc_kernel",
                         "peak_source": pk["source"] + (" bf16 x 2 (the nominal fp8/bf16 ratio)" if f8 else "")},
        }
        print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()
    return 0

def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    # Each step appends a token to every stream, so a long config-4 run drifts
    # the workload away from its definition (contexts log-uniform in [64, 4096],
    # mean ~970): 20 steps move it by ~2 %, 100 steps by ~10 %.  Serving
    # compacts the pool every 64 steps, so it times at least that many.
    ap.add_argument("--steps", type=int, default=None,
                    help="timed steps (default: 20 for the config-4 KV step, 64 for serve, 100 otherwise)")
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--workload", choices=("kv", "model", "model3", "serve", "prefill", "gemm", "readprobe"),
                    default="kv",
                    help="kv: config 4 KV step (default); readprobe: the read ceiling of K2's page stream on "
                         "the config-4 cache; model: config 2 full greedy decode (0.6B bf16, 32 "
                         "streams); model3: config 3 (1.7B bf16, 64 streams, 390 audio + 20 text tokens); "
                         "serve: config 5 (1.7B, 8-bit cache, 512 concurrent streams, Poisson arrivals); "
                         "prefill: K3 prefill attention over config-3 prompts (--kv-dtype bf16/fp8/f32); "
                         "gemm: the tcgen05 projection GEMM on every decoder projection shape")
    ap.add_argument("--concurrency", type=int, default=512, help="serve: target concurrent streams per GPU")
    ap.add_argument("--serve-kv", choices=("e4i8", "fp8"), default="e4i8",
                    help="serve: 8-bit cache (e4i8 = e4m3 K + int8 V, fp8 = e4m3 K and V)")
    ap.add_argument("--kv-dtype", choices=("bf16", "fp8", "e4i8", "f32"), default="bf16",
                    help="kv workload: cache dtype (bf16 is the config-4 workload)")
    ap.add_argument("--weights", choices=("bf16", "fp8"), default="bf16",
                    help="model / model3 / serve: projection weights (fp8 = e4m3 weights and token rows, "
                         "one scale per row, tcgen05 kind::f8f6f4)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--no-model", action="store_true",
                    help="kv workload: skip the config-2 full-model decode figure added to the line")
    ap.add_argument("--layers", type=int, default=N_LAYERS,
                    help="layers of cache (28 = the workload; fewer only for small profiling captures)")
    args = ap.parse_args()
    if args.steps is None:
        args.steps = {"kv": 20, "serve": 64}.get(args.workload, 100)
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    if args.workload in ("model", "model3"):
        return run_model(args)
    if args.workload == "serve":
        return run_serve(args)
    if args.workload == "prefill":
        return run_prefill_attn(args)
    if args.workload == "gemm":
        return run_gemm(args)
    if args.workload == "readprobe":
        return run_readprobe(args)
    return run_ours(args)


if __name__ == "__main__":
    raise SystemExit(main())
