"""Benchmark of the paged-KV hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload llama70b-shard|llama70b-shard-tokens|llama8b|mla-layer-shard[-fp8]|
                                decode-mix|adapter|host-tier|clock-stress]

One step = one pass of the hot path over one batch: gather every block of a
GPU's paged KV cache, for every layer and K/V, through a seeded random block
table into contiguous 256-token chunks (LMCache KV_2LTD order: K/V x layer x
tokens x row), then scatter the chunks back through the same table.  Both
moves are single launches of the row-mover kernel.

Default workload (the per-GPU shard of the Llama-3-70B-shaped cache split by
KV head): 80 layers x K/V, 1 KV head per GPU, head_dim 128, block 16 tokens,
bf16, 16 sequences x 32k tokens = 32,768 blocks per GPU, 21.47 GB of cache
per GPU.  With N GPUs each rank owns its own head shard and block table
(weak scaling, no collective in the data path; NCCL only aggregates timings).
llama70b-shard-tokens moves the same cache token by token (256-byte rows)
through the slot mapping of the same block table.

Also reported: the device-resident clock stream on the clock-stress workload
(1,048,576 slots, usage U{0..3}, 5% pinned, 200k allocations, one Zipf(1.1)
re-access per allocation) in evictions/s.

--impl reference times the reference's CPU implementation of the same moves
(torch index_select / index_copy_ per plane, the oracle restatement) on a
bounded sample of the workload with all host cores, on rank 0 only.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import pathlib
import statistics
import sys
import threading
import time

REPO = pathlib.Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

import torch  # noqa: E402

WORKLOADS = {
    "llama70b-shard": dict(layers=80, kv=2, heads=1, head_dim=128, block_size=16, dtype=torch.bfloat16,
                           seqs=16, seq_tokens=32768, chunk_tokens=256,
                           label="Llama-3-70B KV-head shard: 80 layers x K/V, 1 KV head/GPU, head_dim 128, "
                                 "block 16, bf16, 16 x 32k-token sequences (32,768 blocks/GPU), 256-token chunks"),
    "llama8b": dict(layers=32, kv=2, heads=8, head_dim=128, block_size=16, dtype=torch.float16,
                    seqs=64, seq_tokens=256, chunk_tokens=256,
                    label="Llama-3-8B cache: 32 layers x K/V, 8 KV heads, head_dim 128, block 16, fp16, "
                          "1024 blocks/layer, 64 requests x 256 tokens"),
    "llama70b-shard-tokens": dict(layers=80, kv=2, heads=1, head_dim=128, block_size=16, dtype=torch.bfloat16,
                                  seqs=16, seq_tokens=32768, chunk_tokens=256, tokens=True,
                                  label="Llama-3-70B KV-head shard, token-granular: 80 layers x K/V, 1 KV head/GPU, "
                                        "head_dim 128, block 16, bf16, 16 x 32k-token sequences (524,288 tokens/GPU), "
                                        "slot_mapping = block table x 16 + offset, 256-byte token rows, "
                                        "256-token chunks"),
    "mla-layer-shard": dict(layers=8, kv=1, heads=1, head_dim=576, block_size=64, dtype=torch.bfloat16,
                            seqs=1, seq_tokens=131072, chunk_tokens=256,
                            label="MLA latent cache, one GPU's layer range (8 of 61 layers): one 576-wide "
                                  "row (512 + 64 rope) per token, block 64, bf16, 128k-token context "
                                  "(2,048 blocks), 256-token chunks"),
    "mla-layer-shard-fp8": dict(layers=8, kv=1, heads=1, head_dim=576, block_size=64,
                                dtype=torch.float8_e4m3fn, seqs=1, seq_tokens=131072, chunk_tokens=256,
                                label="MLA latent cache, fp8-e4m3 byte view: one GPU's layer range (8 of 61 "
                                      "layers), 576 bytes per token, block 64, 128k-token context, "
                                      "256-token chunks"),
}

CPU_SAMPLE_BLOCKS = 2048  # blocks per plane in the bounded CPU sample


def _peaks() -> tuple[float, str]:
    path = REPO / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(path.read_text())["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def _traffic_per_launch(workload: str) -> float | None:
    """DRAM bytes per mover launch from the committed ncu summary, if any."""
    path = REPO / "profiles" / "mover_traffic.json"
    try:
        rec = json.loads(path.read_text())[workload]
        return float(rec["dram_bytes_per_launch"])
    except Exception:
        return None



class ClockSampler:
    """NVML sampling of SM clock and throttle reasons during a timed region."""

    def __init__(self, device_index: int, period_s: float = 0.05):
        self.samples: list[tuple[int, int]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nvml = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._nvml = None
        self.period_s = period_s

    def _run(self) -> None:
        while not self._stop.is_set():
            try:
                mhz = self._nvml.nvmlDeviceGetClockInfo(self._h, self._nvml.NVML_CLOCK_SM)
                reasons = self._nvml.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                self.samples.append((mhz, reasons))
            except Exception:
                pass
            self._stop.wait(self.period_s)

    def __enter__(self):
        if self._nvml is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join()

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unavailable"]}
        n = self._nvml
        names = {
            "gpu_idle": getattr(n, "nvmlClocksEventReasonGpuIdle", 0x1),
            "applications_clocks_setting": getattr(n, "nvmlClocksEventReasonApplicationsClocksSetting", 0x2),
            "sw_power_cap": getattr(n, "nvmlClocksEventReasonSwPowerCap", 0x4),
            "hw_slowdown": getattr(n, "nvmlClocksEventReasonHwSlowdown", 0x8),
            "sync_boost": getattr(n, "nvmlClocksEventReasonSyncBoost", 0x10),
            "sw_thermal_slowdown": getattr(n, "nvmlClocksEventReasonSwThermalSlowdown", 0x20),
            "hw_thermal_slowdown": getattr(n, "nvmlClocksEventReasonHwThermalSlowdown", 0x40),
            "hw_power_brake_slowdown": getattr(n, "nvmlClocksEventReasonHwPowerBrakeSlowdown", 0x80),
        }
        seen = 0
        for _, r in self.samples:
            seen |= r
        reasons = [k for k, bit in names.items() if seen & bit and k != "gpu_idle"]
        return {"sm_mhz": statistics.median(m for m, _ in self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": reasons, "samples": len(self.samples)}


def _dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def _max_over_ranks(x: float, world: int, device) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t[0])


def _barrier(world: int) -> None:
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def _min_over_ranks(x: float, world: int, device) -> float:
    return -_max_over_ranks(-x, world, device)


def _same_on_all_ranks(digest: str, world: int) -> bool:
    """True when every rank computed the same digest (replicated slot tables
    must pick identical victims on every KV-head shard)."""
    if world == 1:
        return True
    import torch.distributed as dist

    digests: list[str | None] = [None] * world
    dist.all_gather_object(digests, digest)
    return all(d == digest for d in digests)


# ---------------------------------------------------------------------------
# workload construction
# ---------------------------------------------------------------------------


def build_cache(w: dict, device, seed: int, num_blocks: int | None = None):
    """Planes ordered K of every layer, then V of every layer (KV_2LTD chunks),
    as views of one (layers, 2, num_blocks, block, heads, head_dim) tensor."""
    nb = num_blocks or (w["seqs"] * w["seq_tokens"] // w["block_size"])
    shape = (w["layers"], w["kv"], nb, w["block_size"], w["heads"], w["head_dim"])
    gen = torch.Generator(device=device).manual_seed(seed) if device.type == "cuda" else \
        torch.Generator().manual_seed(seed)
    if w["dtype"] == torch.float8_e4m3fn:  # moved as raw bytes
        kv = torch.empty(shape, dtype=torch.uint8, device=device)
        kv.random_(0, 256, generator=gen)
        kv = kv.view(torch.float8_e4m3fn)
    else:
        kv = torch.empty(shape, dtype=w["dtype"], device=device)
        kv.normal_(generator=gen)
    planes = [kv[l, h] for h in range(w["kv"]) for l in range(w["layers"])]
    table = torch.randperm(nb, generator=torch.Generator().manual_seed(seed))
    return kv, planes, table, nb


def _dtype_name(dt) -> str:
    return {torch.bfloat16: "bf16", torch.float16: "fp16", torch.float8_e4m3fn: "fp8-e4m3 (bytes)"}.get(dt, str(dt))


def slot_mapping_of(table: torch.Tensor, block_size: int) -> torch.Tensor:
    """Token slots of the blocks of ``table`` in order: block * block_size +
    offset (the slot_mapping of a request whose block table is ``table``)."""
    offsets = torch.arange(block_size, dtype=torch.int64, device=table.device)
    return (table.view(-1, 1) * block_size + offsets.view(1, -1)).reshape(-1)


def full_byte_check(chunks: torch.Tensor, planes, index: torch.Tensor, tokens: bool) -> int:
    """Every byte of ``chunks`` against the cache rows that ``index`` names,
    plane by plane, with torch ``index_select`` on the device (the reference's
    own gather op, adapter.py:543) as the checker.  Returns the bytes compared;
    raises on the first differing plane."""
    n = index.numel()
    for p, plane in enumerate(planes):
        rows = plane.shape[0] * plane.shape[1] if tokens else plane.shape[0]
        src = plane.reshape(rows, -1)
        src = src.view(torch.uint8) if src.element_size() == 1 else src.view(torch.int16)
        got = chunks[:, p].reshape(n, -1)
        got = got.view(torch.uint8) if got.element_size() == 1 else got.view(torch.int16)
        if not torch.equal(got, src.index_select(0, index)):
            raise RuntimeError(f"bench data check failed: plane {p} of the chunks differs from the cache")
    return chunks.numel() * chunks.element_size()


def block_bytes(w: dict) -> int:
    return w["block_size"] * w["heads"] * w["head_dim"] * torch.empty(0, dtype=w["dtype"]).element_size()


# ---------------------------------------------------------------------------
# CPU leg (the reference's torch CPU indexing, restated in oracle/moves.py)
# ---------------------------------------------------------------------------


def cpu_moves(w: dict, steps: int, warmup: int) -> dict:
    from oracle import moves

    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    cb = w["chunk_tokens"] // w["block_size"]
    nb = min(CPU_SAMPLE_BLOCKS, w["seqs"] * w["seq_tokens"] // w["block_size"])
    _, planes, table, nb = build_cache(w, torch.device("cpu"), 1234, num_blocks=nb)
    planes = [p.view(torch.uint8) if p.dtype == torch.float8_e4m3fn else p for p in planes]
    payload = len(planes) * nb * block_bytes(w)
    tokens = bool(w.get("tokens"))
    if tokens:
        mapping = slot_mapping_of(table, w["block_size"])
    times = []
    for i in range(warmup + steps):
        t0 = time.perf_counter()
        if tokens:
            chunks = moves.gather_tokens(planes, mapping, tokens_per_chunk=w["chunk_tokens"])
            moves.scatter_tokens(planes, mapping, chunks, tokens_per_chunk=w["chunk_tokens"])
        else:
            chunks = moves.gather_layers(planes, table, blocks_per_chunk=cb)
            moves.scatter_layers(planes, table, chunks, blocks_per_chunk=cb)
        t1 = time.perf_counter()
        if i >= warmup:
            times.append(t1 - t0)
    gbs = 4 * payload * len(times) / sum(times) / 1e9
    return {"value": round(gbs, 3), "unit": "GB/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"{len(planes)} planes x {nb} blocks ({payload / 1e9:.2f} GB of the cache) per step, "
                      f"{len(times)} steps: per-plane "
                      + ("token-row indexing through the slot mapping" if tokens else "index_select + index_copy_")
                      + " on CPU tensors"}


CLOCK_VARIANTS = {
    # the clock stress as specified: 25% of the slots start at usage 0, so no pop ages
    "stress": dict(slots=1 << 20, usage_hi=3, no_zero=False,
                   label="1,048,576 slots, usage U{0..3}, 5% pinned"),
    # no usage-0 slot at the start and a pool the size of the decode mix's:
    # the first pop ages, and aging recurs whenever the zeros it made run out
    "aging": dict(slots=1 << 16, usage_hi=15, no_zero=True,
                  label="65,536 slots, usage U{1..15} (no usage-0 slot at the start), 5% pinned"),
}


def clock_inputs(k: int, variant: str = "stress"):
    """Parameters, initial slot_meta (CPU) and re-access ids (CPU) of a clock
    stream: 200k allocations in steps of k, one Zipf(1.1) re-access each."""
    from kv_cache_adapter_b200 import adapter as adapter_mod
    from kv_cache_adapter_b200 import workloads

    v = CLOCK_VARIANTS[variant]
    steps = 200_000 // k
    p = workloads.clock_params(v["slots"], steps, k, k, seed=1234, usage_hi=v["usage_hi"])
    meta = workloads.clock_initial_meta(p, adapter_mod._pack_slot_meta)
    if v["no_zero"]:
        usage = (meta >> 4).to(torch.int64)
        meta = adapter_mod._pack_slot_meta((meta & 15).to(torch.int64), torch.clamp(usage, min=1))
    return p, meta, workloads.zipf_reaccess(p)


def clock_algorithmic_bytes(victims: torch.Tensor, thresholds: torch.Tensor, n: int, k: int) -> int:
    """Algorithmic bytes of a clock stream from the oracle's trace: per pop,
    the slot words scanned from search_start to its last victim when it does
    not age, else a read and a write of every word; the 8-byte victim ids;
    the refill (read + write of each victim's word); the 8-byte re-access ids
    and the usage bump (read + write of each re-accessed word)."""
    import numpy as np

    steps = thresholds.numel()
    last = victims.view(steps, k)[:, -1].numpy()
    ss = np.concatenate([[0], (last[:-1] + 1) % n])
    scanned = np.where(thresholds.numpy() > 0, 2 * n, (last - ss) % n + 1)
    return int(scanned.sum()) + steps * k * (8 + 2) + steps * k * (8 + 2)


def cpu_clock(k: int, variant: str = "stress") -> dict:
    """The sequential C restatement of the stream on one host core, and the
    stream's algorithmic bytes and aging steps from its trace."""
    import oracle

    p, meta, reacc = clock_inputs(k, variant)
    steps = p["num_steps"]
    ss = torch.zeros(1, dtype=torch.int64)
    t0 = time.perf_counter()
    victims, done, rc, thresholds = oracle.clock_stream(meta, ss, steps, k, reacc, k, trace=True)
    dt = time.perf_counter() - t0
    assert rc == 0 and done == steps
    return {"value": round(done * k / dt, 1), "unit": "evictions/s", "cores": 1, "kind": "port",
            "sample": f"the full {variant} stream ({done * k} allocations), sequential C restatement",
            "alloc_per_step": k, "variant": variant,
            "algorithmic_bytes": clock_algorithmic_bytes(victims, thresholds, p["num_slots"], k),
            "aging_steps": int((thresholds > 0).sum())}


def clock_roofline(run: dict, trace: dict, peak: float) -> dict:
    achieved = trace["algorithmic_bytes"] / (run["ms"] / 1e3) / 1e9
    return {"bound": "latency", "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
            "frac": round(achieved / peak, 5), "traffic": None,
            "algorithmic_bytes": trace["algorithmic_bytes"], "aging_steps": trace["aging_steps"],
            "note": "a chain of dependent pops over a few MB of slot words: dependent phases and grid "
                    "barriers bound it, not HBM"}


# ---------------------------------------------------------------------------
# GPU legs
# ---------------------------------------------------------------------------


def gpu_clock(device, k: int, reps: int = 3, method: str = "batched", variant: str = "stress") -> dict:
    from kv_cache_adapter_b200 import kv_cache_adapter_cuda as ops
    from kv_cache_adapter_b200 import workloads

    p, meta0, reacc = clock_inputs(k, variant)
    steps = p["num_steps"]
    meta0, reacc = meta0.to(device), reacc.to(device)
    meta = meta0.clone()
    ss = torch.zeros(1, dtype=torch.int64, device=device)
    victims = torch.empty(steps * k, dtype=torch.int64, device=device)
    ms = []
    for r in range(reps + 1):
        meta.copy_(meta0)
        ss.zero_()
        torch.cuda.synchronize(device)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        ops.clock_stream(meta, ss, steps, k, reacc, k, victims=victims, method=method, check=False)
        e1.record()
        torch.cuda.synchronize(device)
        if r:
            ms.append(e0.elapsed_time(e1))
    ops.check_status(device)
    best = min(ms)
    return {"variant": variant, "alloc_per_step": k, "method": method, "steps": steps, "ms": round(best, 3),
            "evictions_per_s": round(steps * k / (best / 1e3), 1), "launches": 1,
            "victims_sha256": workloads.sha256_of(victims), "slot_meta_sha256": workloads.sha256_of(meta)}


# ---------------------------------------------------------------------------
# Per-call pop at 1,048,576 slots (the clock-stress table)
# ---------------------------------------------------------------------------

POP_SLOTS = 1 << 20
POP_CASES = ((1, 0), (256, 0), (1, 64), (256, 64))  # (count, blocked ids)


def pop_inputs() -> tuple[dict, torch.Tensor]:
    """The clock-stress table (usage U{0..3}, 5% pinned, seed 1234) and its
    aging variant (every usage + 1: no free slot has usage 0, so each pop must
    age the whole table), plus 64 seeded blocked ids."""
    import numpy as np

    from kv_cache_adapter_b200 import adapter as adapter_mod
    from kv_cache_adapter_b200 import workloads

    p = workloads.clock_params(POP_SLOTS, 1, 1, 1, seed=1234)
    meta = workloads.clock_initial_meta(p, adapter_mod._pack_slot_meta)
    pins, usage = meta & 15, meta >> 4
    aging = adapter_mod._pack_slot_meta(pins.to(torch.int64), usage.to(torch.int64) + 1)
    blocked = torch.from_numpy(np.random.default_rng(99).integers(0, POP_SLOTS, 64).astype(np.int64))
    return {"no-aging": meta, "aging": aging}, blocked


def _pop_bytes(table: str, ss_before: int, last: int, count: int) -> int:
    """Algorithmic bytes of one pop: the slot words scanned up to the last
    victim when nothing ages, else a read and a write of every word; plus the
    8-byte victim ids."""
    scanned = (last - ss_before) % POP_SLOTS + 1 if table == "no-aging" else 2 * POP_SLOTS
    return scanned + 8 * count


def _graph_pop_ms(ops, meta, base, ss, blocked, count: int, order: str, restore: bool, k: int = 50) -> float:
    """Device time of one pop launch: k pops captured in a CUDA graph and
    replayed back to back (each after a restore of the table when it ages),
    less the same graph's restores alone."""
    device = meta.device
    s = torch.cuda.Stream(device)
    s.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(s):  # the op's per-stream scratch exists before the capture
        ops.pop_reusable_slots(meta, ss, blocked, count, order=order, check=False)
    torch.cuda.synchronize(device)

    def graph_of(with_pop: bool) -> torch.cuda.CUDAGraph:
        g = torch.cuda.CUDAGraph()
        s.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(s), torch.cuda.graph(g, stream=s):
            for _ in range(k):
                if restore:
                    meta.copy_(base)
                if with_pop:
                    ops.pop_reusable_slots(meta, ss, blocked, count, order=order, check=False)
        torch.cuda.current_stream(device).wait_stream(s)
        return g

    def replay_ms(g) -> float:
        g.replay()
        torch.cuda.synchronize(device)
        best = float("inf")
        for _ in range(5):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            g.replay()
            e1.record()
            torch.cuda.synchronize(device)
            best = min(best, e0.elapsed_time(e1))
        return best

    pops = graph_of(True)
    ms = replay_ms(pops)
    if restore:
        ms -= replay_ms(graph_of(False))
    ops.check_status(device)
    return ms / k


def gpu_pop(device, calls: int = 200, tables: str | None = None) -> dict:
    """kv_cache_adapter_cuda.pop_reusable_slots per call: wall time of a call
    that returns with the victims ready and the status read (as the reference's
    op synchronises at nonzero), and the device time of its launch."""
    from kv_cache_adapter_b200 import kv_cache_adapter_cuda as ops

    chosen = tables
    tables, blocked_h = pop_inputs()
    peak, _ = _peaks()
    runs = []
    for name, base_h in tables.items():
        if chosen and name != chosen:
            continue
        base = base_h.to(device)
        restore = name == "aging"
        for count, nb in POP_CASES:
            blocked = blocked_h[:nb].to(device)
            for order in ("prefix", "grouped"):
                meta = base.clone()
                ss = torch.zeros(1, dtype=torch.int64, device=device)
                for _ in range(5):
                    if restore:
                        meta.copy_(base)
                    ops.pop_reusable_slots(meta, ss, blocked, count, order=order)
                wall, nbytes = [], []
                for _ in range(calls):
                    if restore:
                        meta.copy_(base)
                    torch.cuda.synchronize(device)
                    ss0 = int(ss[0])
                    t0 = time.perf_counter()
                    out = ops.pop_reusable_slots(meta, ss, blocked, count, order=order)
                    wall.append(time.perf_counter() - t0)
                    nbytes.append(_pop_bytes(name, ss0, int(out[-1]), count))
                dev = _graph_pop_ms(ops, meta, base, ss, blocked, count, order, restore)
                us = statistics.median(wall) * 1e6
                alg = statistics.median(nbytes)
                runs.append({"table": name, "count": count, "blocked": nb, "order": order,
                             "us_per_call": round(us, 2), "evictions_per_s": round(count / (us / 1e6), 1),
                             "kernel_us": round(dev * 1e3, 2), "algorithmic_bytes": int(alg),
                             "kernel_gbs": round(alg / (dev / 1e3) / 1e9, 1),
                             "hbm_frac": round(alg / (dev / 1e3) / 1e9 / peak, 4)})
    return {"metric": "per-call pop", "slots": POP_SLOTS, "calls_per_case": calls,
            "api": "kv_cache_adapter_cuda.pop_reusable_slots (check=True: one status read per call)",
            "kernel_us": "device time per pop launch: 50 pops in a CUDA graph replayed back to back (less the "
                         "table restores of the aging case), no status read",
            "roofline": "no-aging pops scan a few words (latency-bound); aging pops read and write every "
                        "slot word (HBM-bound; hbm_frac against MEASURED_PEAKS.json hbm_gbs)",
            "runs": runs}


def reference_gpu_pop(device, calls: int = 50) -> dict:
    """The reference's own CUDA pop (csrc/kv_adapter_cuda.cu:64-237, host
    :406-450, compiled unchanged into oracle/_ref), per call on the same
    inputs: unpacked usage (uint8) and reusable mask (pin == 0) as the
    reference adapter passes them (adapter.py:485-491)."""
    from oracle import build_ref

    if not build_ref.available():
        return {"unavailable": "reference CUDA extension not built (python -m oracle.build_ref)"}
    ref = build_ref.load()
    tables, blocked_h = pop_inputs()
    runs = []
    for name, base_h in tables.items():
        usage0 = (base_h >> 4).to(torch.uint8).to(device)
        reusable = ((base_h & 15) == 0).to(device)
        restore = name == "aging"
        for count, nb in POP_CASES:
            blocked = blocked_h[:nb].to(device)
            usage = usage0.clone()
            ss = torch.zeros(1, dtype=torch.int64, device=device)
            for _ in range(3):
                if restore:
                    usage.copy_(usage0)
                ref.pop_reusable_slots(usage, reusable, ss, blocked, count)
            torch.cuda.synchronize(device)
            wall, dev_ms = [], []
            for _ in range(calls):
                if restore:
                    usage.copy_(usage0)
                torch.cuda.synchronize(device)
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                t0 = time.perf_counter()
                e0.record()
                ref.pop_reusable_slots(usage, reusable, ss, blocked, count)
                e1.record()
                torch.cuda.synchronize(device)  # the kernel runs after the op returns
                wall.append(time.perf_counter() - t0)
                dev_ms.append(e0.elapsed_time(e1))
            us = statistics.median(wall) * 1e6
            runs.append({"table": name, "count": count, "blocked": nb, "order": "prefix (the reference kernel)",
                         "us_per_call": round(us, 2), "evictions_per_s": round(count / (us / 1e6), 1),
                         "device_us_per_call": round(statistics.median(dev_ms) * 1e3, 2)})
    return {"metric": "per-call pop", "slots": POP_SLOTS, "calls_per_case": calls,
            "api": "reference torch extension pop_reusable_slots (host nonzero sync, then one 1-CTA kernel)",
            "device_us_per_call": "GPU time from before the op's first kernel to after its pop kernel, "
                                  "including the gap while the host waits for nonzero",
            "runs": runs}


def cpu_strict_pop(calls: int = 20) -> dict:
    """The reference's strict-path pop (adapter.py:472-525) as torch CPU ops
    (oracle/strict_pop.py), per call on the same inputs, grouped order."""
    from oracle import strict_pop

    cores = len(os.sched_getaffinity(0))
    torch.set_num_threads(cores)
    tables, blocked_h = pop_inputs()
    runs = []
    for name, base in tables.items():
        for count, nb in POP_CASES:
            blocked = blocked_h[:nb]
            meta = base.clone()
            ss = torch.zeros(1, dtype=torch.int64)
            times = []
            for i in range(calls + 2):
                if name == "aging":
                    meta.copy_(base)
                t0 = time.perf_counter()
                strict_pop.pop_reusable_slots(meta, ss, blocked, count)
                if i >= 2:
                    times.append(time.perf_counter() - t0)
            us = statistics.median(times) * 1e6
            runs.append({"table": name, "count": count, "blocked": nb, "order": "grouped",
                         "us_per_call": round(us, 1), "evictions_per_s": round(count / (us / 1e6), 1)})
    return {"kind": "port", "cores": torch.get_num_threads(), "slots": POP_SLOTS,
            "sample": f"{calls} calls per case of the strict path's torch CPU ops (oracle/strict_pop.py)",
            "runs": runs}


def run_pop(args, world: int, rank: int, device) -> None:
    """Per-call pop alone (the default bench line carries the same record)."""
    pop = gpu_pop(device, calls=max(args.steps, 20), tables=args.pop_table)
    for r in pop["runs"]:
        r["us_per_call"] = _max_over_ranks(r["us_per_call"], world, device)
    if rank != 0:
        return
    first = pop["runs"][0]
    line = {"metric": "per-call pop evictions/s", "value": round(world * first["evictions_per_s"], 1),
            "unit": "evictions/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8",
            "data": "synthetic (the clock-stress table, seed 1234)",
            "config": {"workload": f"per-call pop, {POP_SLOTS:,} slots: counts 1 / 256, 0 / 64 blocked ids, "
                                   "a table that needs no aging and one that ages on every pop"},
            "pop": pop}
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_strict_pop()
    print(json.dumps(line), flush=True)


TOKEN_ROW_WIDTHS = (64, 128, 256, 576, 1152, 2048)


def run_token_rows(args, world: int, rank: int, device) -> None:
    """Random token rows through a slot mapping: per row width, gather half
    of the token slots of every plane (chosen at random) into 256-token
    chunks and scatter them back, about --move-mib MiB per move.  Rows of
    64 B take the small-row mover, 128 B to 1.5 KiB the stream mover, 2 KiB
    the SIMT mover."""
    from kv_cache_adapter_b200 import kv_cache_adapter_cuda as ops

    widths = [args.row_bytes] if args.row_bytes else list(TOKEN_ROW_WIDTHS)
    peak, _ = _peaks()
    runs = []
    for rb in widths:
        planes_n = 8 if rb in (576, 1152) else 64
        rows = max(256, (args.move_mib << 20) // (planes_n * rb) // 256 * 256)
        bs = 16
        nb = -(-2 * rows // bs)
        gen = torch.Generator(device=device).manual_seed(1234 + rb)
        cache = torch.empty((planes_n, nb, bs, rb), dtype=torch.uint8, device=device)
        cache.random_(0, 256, generator=gen)
        planes = [cache[p] for p in range(planes_n)]
        ptab = ops.PlaneTable(planes, 2)
        mapping = torch.randperm(nb * bs, generator=torch.Generator().manual_seed(rb))[:rows].to(device)
        chunks = torch.empty((rows // 256, planes_n, 256, rb), dtype=torch.uint8, device=device)
        ops.gather_tokens(ptab, mapping, chunks, tokens_per_chunk=256, check=True)
        flat = cache.view(planes_n, nb * bs, rb)
        for p in range(planes_n):
            if not torch.equal(chunks[:, p].reshape(rows, rb), flat[p].index_select(0, mapping)):
                raise RuntimeError(f"token-rows check failed: {rb}-byte rows, plane {p}")
        for _ in range(args.warmup):
            ops.gather_tokens(ptab, mapping, chunks, tokens_per_chunk=256, check=False)
            ops.scatter_tokens(ptab, mapping, chunks, tokens_per_chunk=256, check=False)
        ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
        _barrier(world)
        torch.cuda.synchronize(device)
        for e0, e1, e2 in ev:
            e0.record()
            ops.gather_tokens(ptab, mapping, chunks, tokens_per_chunk=256, check=False)
            e1.record()
            ops.scatter_tokens(ptab, mapping, chunks, tokens_per_chunk=256, check=False)
            e2.record()
        torch.cuda.synchronize(device)
        ops.check_status(device)
        moved = 2 * planes_n * rows * rb
        g_ms = _max_over_ranks(statistics.median(a.elapsed_time(b) for a, b, _ in ev), world, device)
        s_ms = _max_over_ranks(statistics.median(b.elapsed_time(c) for _, b, c in ev), world, device)
        ceil_g, ceil_s = _row_ceiling(ops, device, rb, planes_n * rows, args.steps, world)
        g_gbs, s_gbs = moved / (g_ms / 1e3) / 1e9, moved / (s_ms / 1e3) / 1e9
        runs.append({"row_bytes": rb, "planes": planes_n, "rows_per_plane": rows, "bytes_per_move": moved,
                     "gather_gbs": round(g_gbs, 1), "scatter_gbs": round(s_gbs, 1),
                     "gather_frac": round(g_gbs / peak, 4), "scatter_frac": round(s_gbs / peak, 4),
                     "gather_ms": round(g_ms, 4), "scatter_ms": round(s_ms, 4),
                     "random_row_ceiling_gbs": {"gather": round(ceil_g, 1), "scatter": round(ceil_s, 1)},
                     "frac_of_random_row_ceiling": {"gather": round(g_gbs / ceil_g, 4),
                                                    "scatter": round(s_gbs / ceil_s, 4)}})
        del cache, chunks, planes, ptab
        torch.cuda.empty_cache()
    if rank != 0:
        return
    worst = min(min(r["gather_frac"], r["scatter_frac"]) for r in runs)
    line = {"metric": "random token-row gather / scatter GB/s", "value": runs[0]["gather_gbs"], "unit": "GB/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "u8 (rows moved as bytes)",
            "data": "synthetic (seeded random bytes, seeded random half of the token slots)",
            "config": {"workload": "token rows through a random slot mapping, 256-token chunks, row widths "
                                   + ", ".join(str(r["row_bytes"]) for r in runs) + " B",
                       "l2": "each move reads and writes about 2 x move_mib MiB, above L2"},
            "roofline": {"bound": "hbm", "peak": peak, "unit": "GB/s", "worst_frac": worst,
                         "peak_source": "measured (MEASURED_PEAKS.json hbm_gbs)",
                         "random_row_ceiling": "kvca_row_ceiling on the same box and the same bytes: one dense "
                                               "plane, rows through a uint32 permutation, no slot or chunk "
                                               "arithmetic (the DRAM limit of random rows of that width)"},
            "runs": runs, "gpu_launches": 4 * args.steps * len(runs)}
    print(json.dumps(line), flush=True)


def _row_ceiling(ops, device, row_bytes: int, rows: int, steps: int, world: int) -> tuple[float, float]:
    """GB/s of kvca_row_ceiling gathering and scattering `rows` rows of
    row_bytes between two dense buffers through a random permutation (median
    of `steps` launches each, 8 CTAs of 256 threads per SM)."""
    src = torch.empty(rows * row_bytes, dtype=torch.uint8, device=device)
    src.random_(0, 256)
    dst = torch.empty_like(src)
    perm = torch.randperm(rows, generator=torch.Generator().manual_seed(row_bytes)).to(torch.int32).to(device)
    lib = ops._lib_handle
    ctas = 8 * torch.cuda.get_device_properties(device).multi_processor_count
    out = []
    for scatter in (0, 1):
        def launch():
            rc = lib.kvca_row_ceiling(ctypes.c_void_p(src.data_ptr()), ctypes.c_void_p(dst.data_ptr()),
                                      ctypes.c_void_p(perm.data_ptr()), rows, row_bytes, scatter, ctas,
                                      ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream))
            if rc != 0:
                raise RuntimeError(f"kvca_row_ceiling failed ({rc})")
        for _ in range(3):
            launch()
        ts = []
        for _ in range(max(steps, 3)):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            launch()
            b.record()
            torch.cuda.synchronize(device)
            ts.append(a.elapsed_time(b))
        out.append(2 * rows * row_bytes / (_max_over_ranks(statistics.median(ts), world, device) / 1e3) / 1e9)
    if not torch.equal(dst.view(rows, row_bytes)[perm.long()], src.view(rows, row_bytes)):
        raise RuntimeError(f"row ceiling check failed: {row_bytes}-byte rows")
    del src, dst, perm
    torch.cuda.empty_cache()
    return out[0], out[1]


def run_ours(args, w: dict, world: int, rank: int, device) -> None:
    from kv_cache_adapter_b200 import kv_cache_adapter_cuda as ops

    seed = 1234 + rank
    kv, planes, table_h, nb = build_cache(w, device, seed)
    cb = w["chunk_tokens"] // w["block_size"]
    P = len(planes)
    bbytes = block_bytes(w)
    payload = P * nb * bbytes  # bytes of cache moved by one gather (and by one scatter)
    tokens = bool(w.get("tokens"))
    if tokens:  # token-granular: one row per token and plane (256 bytes here), through a slot mapping
        tpc = w["chunk_tokens"]
        index_h = slot_mapping_of(table_h, w["block_size"])
        chunks = torch.empty((nb * w["block_size"] // tpc, P, tpc, w["heads"], w["head_dim"]), dtype=w["dtype"],
                             device=device)
        ptab = ops.PlaneTable(planes, 2)

        def gather(idx):
            ops.gather_tokens(ptab, idx, chunks, tokens_per_chunk=tpc, check=False)

        def scatter(idx):
            ops.scatter_tokens(ptab, idx, chunks, tokens_per_chunk=tpc, check=False)
    else:
        index_h = table_h
        chunks = torch.empty((nb // cb, P, cb, w["block_size"], w["heads"], w["head_dim"]), dtype=w["dtype"],
                             device=device)
        ptab = ops.PlaneTable(planes, 1)

        def gather(idx):
            ops.gather_layers(ptab, idx, chunks, blocks_per_chunk=cb, check=False)

        def scatter(idx):
            ops.scatter_layers(ptab, idx, chunks, blocks_per_chunk=cb, check=False)
    index = index_h.to(device)

    def step():
        gather(index)
        scatter(index)

    # full-size byte check, outside the timed region: a gather through the
    # bench's table, then a scatter through a second permutation (the cache
    # becomes a permutation of itself), each compared on every plane
    table2_h = torch.randperm(nb, generator=torch.Generator().manual_seed(seed + 1000))
    index2 = (slot_mapping_of(table2_h, w["block_size"]) if tokens else table2_h).to(device)
    gather(index)
    torch.cuda.synchronize(device)
    ops.check_status(device)
    verified = full_byte_check(chunks, planes, index, tokens)
    scatter(index2)
    torch.cuda.synchronize(device)
    ops.check_status(device)
    verified += full_byte_check(chunks, planes, index2, tokens)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(device)
    ops.check_status(device)

    # ---- device-timed region ------------------------------------------------
    events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True),
               torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    _barrier(world)
    torch.cuda.synchronize(device)
    with ClockSampler(device.index) as clocks:
        start.record()
        for g0, g1, s1 in events:
            g0.record()
            gather(index)
            g1.record()
            scatter(index)
            s1.record()
        end.record()
        torch.cuda.synchronize(device)
    _barrier(world)
    ops.check_status(device)
    verified += full_byte_check(chunks, planes, index, tokens)  # the timed steps' last gather
    total_ms = _max_over_ranks(start.elapsed_time(end), world, device)
    launch_ms = [g0.elapsed_time(g1) for g0, g1, _ in events] + [g1.elapsed_time(s1) for _, g1, s1 in events]
    avg_launch_ms = _max_over_ranks(sum(launch_ms) / len(launch_ms), world, device)

    # ---- end-to-end through the public API with host buffers ------------------
    index_pinned = index_h.clone().pin_memory()
    index_dev = torch.empty_like(index)
    _barrier(world)
    torch.cuda.synchronize(device)
    # every step copies its inputs host -> device and its status word device ->
    # pinned host memory; the host reads step i's word while step i + 1 runs
    status_host = torch.zeros((2, 2), dtype=torch.int64, pin_memory=True)
    done = [torch.cuda.Event(), torch.cuda.Event()]
    word = ops.status_word(device)
    t0 = time.perf_counter()
    for i in range(args.steps):
        index_dev.copy_(index_pinned, non_blocking=True)
        gather(index_dev)
        scatter(index_dev)
        status_host[i % 2].copy_(word, non_blocking=True)
        done[i % 2].record()
        if i > 0:
            done[(i - 1) % 2].synchronize()
            ops.raise_status(*status_host[(i - 1) % 2].tolist(), "bench step")
    done[(args.steps - 1) % 2].synchronize()
    ops.raise_status(*status_host[(args.steps - 1) % 2].tolist(), "bench step")
    e2e_s = _max_over_ranks(time.perf_counter() - t0, world, device)
    _barrier(world)

    # ---- clock stream (replicated pool per GPU) -------------------------------
    clock = None if args.no_clock else [
        gpu_clock(device, 1), gpu_clock(device, 256), gpu_clock(device, 1, reps=1, method="steps"),
        gpu_clock(device, 1, variant="aging"), gpu_clock(device, 256, variant="aging"),
        gpu_clock(device, 1, reps=1, method="steps", variant="aging")]
    if clock is not None:
        for c in clock:
            c["evictions_per_s"] = _min_over_ranks(c["evictions_per_s"], world, device)  # slowest rank
            c["identical_on_all_ranks"] = _same_on_all_ranks(c["victims_sha256"] + c["slot_meta_sha256"], world)
    pop = None if args.no_clock else gpu_pop(device)
    if pop is not None:
        for r in pop["runs"]:
            r["us_per_call"] = _max_over_ranks(r["us_per_call"], world, device)  # slowest rank

    if rank != 0:
        return
    algo_per_step = 4 * payload  # gather r+w + scatter r+w
    value = world * algo_per_step * args.steps / (total_ms / 1e3) / 1e9
    peak, peak_kind = _peaks()
    achieved = 2 * payload / (avg_launch_ms / 1e3) / 1e9
    traffic = _traffic_per_launch(args.workload)
    line = {
        "metric": "paged-KV gather+scatter GB/s",
        "value": round(value, 2),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(total_ms / args.steps, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": _dtype_name(w["dtype"]),
        "data": "synthetic (seeded N(0,1) cache, seeded random block tables)",
        "config": {
            "workload": w["label"],
            "planes": P,
            "blocks_per_gpu": nb,
            "block_bytes_per_plane": bbytes,
            "cache_bytes_per_gpu": payload,
            "chunk_layout": "KV_2LTD per 256-token chunk",
            "granularity": "token rows through a slot mapping" if tokens else "blocks through a block table",
            "l2": "inputs larger than L2 (cache and chunks are each > 126 MB)",
            "parallelism": f"kv-head shard x{world}, no data-path collective",
        },
        "verified_bytes": verified,
        "verification": "outside the timed region, every byte of the chunks against torch index_select on the "
                        "device, plane by plane: after a gather, after a scatter through a second permutation, "
                        "and after the last timed step",
        "per_gpu_gbs": round(value / world, 2),
        "hbm_frac_per_gpu": round(value / world / peak, 4),
        "roofline": {
            "bound": "hbm",
            "achieved": round(achieved, 1),
            "peak": peak,
            "unit": "GB/s",
            "frac": round(achieved / peak, 4),
            "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else "fallback",
            "traffic": traffic,
            "kernel": ("move_rows_stream_kernel (gather and scatter launches; warp-cooperative: 18 rows of 256 bytes per "
                       "warp and batch, 9 vectors per lane, plane-major)" if tokens else
                       "move_rows_bulk_kernel (gather and scatter launches; TMA bulk copies)"),
            "algorithmic_bytes_per_launch": 2 * payload,
            "avg_launch_ms": round(avg_launch_ms, 4),
        },
        "e2e": {
            "value": round(world * algo_per_step * args.steps / e2e_s / 1e9, 2),
            "unit": "GB/s",
            "h2d_bytes_per_step": index_h.numel() * 8,
            "d2h_bytes_per_step": 16,
            "api": ("kv_cache_adapter_cuda.gather_tokens / scatter_tokens" if tokens else
                    "kv_cache_adapter_cuda.gather_layers / scatter_layers") + " (ctypes -> C ABI)",
            "pipelining": "each step's status word is copied to pinned host memory and read by the host "
                          "while the next step runs (one step of lag); the last one after the loop",
        },
        "gpu_launches": 2 * args.steps,
        "clocks": clocks.summary(),
    }
    if clock is not None:
        line["clock_eviction"] = {
            "metric": "clock evictions/s",
            "workload": "200k allocations, 1 Zipf(1.1) re-access per allocation, device-resident stream "
                        "(1 launch); variants: " + "; ".join(f"{k}: {v['label']}" for k, v in CLOCK_VARIANTS.items())
                        + "; method batched = runs of steps without aging resolved at once (exact), "
                          "steps = one step after another",
            "runs": clock,
            "aggregate_evictions_per_s": {str(c["alloc_per_step"]): round(world * c["evictions_per_s"], 1)
                                          for c in clock if c["method"] == "batched" and c["variant"] == "stress"},
        }
    if pop is not None:
        line["pop"] = pop
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_moves(w, steps=2, warmup=1)
        if clock is not None:
            traces = {(c["variant"], c["alloc_per_step"]): c for c in
                      (cpu_clock(k, v) for v in CLOCK_VARIANTS for k in (1, 256))}
            for c in clock:
                c["roofline"] = clock_roofline(c, traces[(c["variant"], c["alloc_per_step"])], peak)
            line["cpu_baseline_clock"] = list(traces.values())
        if pop is not None:
            line["cpu_baseline_pop"] = cpu_strict_pop()
    print(json.dumps(line), flush=True)


def run_clock_stress(args, world: int, rank: int, device) -> None:
    """The clock stress alone: 1,048,576 slots, 200k allocations with one
    Zipf(1.1) re-access each, batches k = 1 and k = 256, one launch each."""
    reps = max(args.steps, 1)
    runs = [gpu_clock(device, k, reps=reps, variant=v) for v in CLOCK_VARIANTS for k in (1, 256)]
    runs += [gpu_clock(device, 1, reps=1, method="steps", variant=v) for v in CLOCK_VARIANTS]
    if rank != 0:
        return
    k1 = runs[0]
    peak, _ = _peaks()
    line = {
        "metric": "clock evictions/s",
        "value": round(world * k1["evictions_per_s"], 1),
        "unit": "evictions/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": k1["ms"],
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "u8",
        "data": "synthetic (seeded usage, pins and Zipf re-access stream)",
        "config": {"workload": "clock stress: 1,048,576 slots, usage U{0..3}, 5% pinned, 200k allocations, "
                               "1 Zipf(1.1) re-access per allocation, batch k = 1 (value) and 256, "
                               "device-resident stream, one cooperative launch per run; also the aging "
                               "variant (" + CLOCK_VARIANTS["aging"]["label"] + ")",
                   "timing": "CUDA events around each launch, best of the timed runs"},
        "runs": runs,
        "gpu_launches": 4 * (reps + 1) + 2 * 2,
    }
    if world == 1 and not args.no_cpu_baseline:
        traces = {(c["variant"], c["alloc_per_step"]): c for c in
                  (cpu_clock(k, v) for v in CLOCK_VARIANTS for k in (1, 256))}
        for c in runs:
            c["roofline"] = clock_roofline(c, traces[(c["variant"], c["alloc_per_step"])], peak)
        line["roofline"] = runs[0]["roofline"]
        line["cpu_baseline"] = traces[("stress", 1)]
        line["cpu_baseline_all"] = list(traces.values())
    print(json.dumps(line), flush=True)


DECODE_STEPS_PER_BENCH_STEP = 50


def run_decode_mix(args, world: int, rank: int, device) -> None:
    """Decode append + gather mix: 256 sequences append one token per decode
    step into a full 65,536-block pool (reshape-and-cache through a per-token
    slot_mapping); sequences whose block fills up get a new one from the clock
    sweep, whose victims are gathered to a spill chunk first.  One bench step
    = 50 decode steps, so the default 20 timed bench steps are 1,000 decode
    steps."""
    from kv_cache_adapter_b200 import kv_cache_adapter_cuda as ops
    from kv_cache_adapter_b200.workloads import DecodeMix

    per = DECODE_STEPS_PER_BENCH_STEP
    heads = args.heads or 1
    cycles = -(-args.steps * per // 16)  # timed decode steps, rounded up to whole 16-step cycles
    pool = args.pool_blocks or 65536
    mix = DecodeMix(ops, device, layers=32, heads=heads, head_dim=128, block_size=16, num_blocks=pool,
                    seqs=256, dtype=torch.float16, seed=1234 + rank,
                    max_steps=(args.warmup * per + 17) + 5 * (cycles + 8) * 16 + 256)  # warm-up + 5 timed runs
    rows = torch.randn((1, mix.num_planes, mix.seqs, *mix.row_shape), dtype=torch.float16, device=device)
    # the whole-cycle runs take a new token row per sequence, plane and step
    # (16 steps' rows, 512 MiB with 8 KV heads), so no step re-reads the last
    # one's rows from L2
    cycle_rows = torch.randn((16, mix.num_planes, mix.seqs, *mix.row_shape), dtype=torch.float16, device=device)
    # warm-up: eager steps (at least one full cycle), aligned to the start of a cycle
    warm = max(args.warmup * per, 17)
    warm += (1 - warm) % 16
    for _ in range(warm):
        mix.step(rows)
    torch.cuda.synchronize(device)
    ops.check_status(device)

    def timed(run) -> float:
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        _barrier(world)
        torch.cuda.synchronize(device)
        start.record()
        run()
        end.record()
        torch.cuda.synchronize(device)
        _barrier(world)
        ops.check_status(device)
        return _max_over_ranks(start.elapsed_time(end), world, device)

    # host-issued: one Python call per op
    tok0, blk0 = mix.tokens, mix.gathered_blocks
    eager_ms = timed(lambda: [mix.step(rows) for _ in range(cycles * 16)])
    eager_tokens, eager_blocks = mix.tokens - tok0, mix.gathered_blocks - blk0
    # graph-captured: one replay per 16-step cycle, first with every step's
    # launches in order on one stream, then pipelined (each step's bookkeeping
    # on a second stream, overlapping the previous step's moves)
    graph, per_cycle = mix.capture_cycle(rows)
    graph.replay()  # uploads the graph; untimed warm-up
    serial_ms = timed(lambda: [graph.replay() for _ in range(cycles)])
    del graph
    mix.pipelined = True
    graph, per_cycle_p = mix.capture_cycle(rows)
    assert per_cycle_p == per_cycle
    graph.replay()  # untimed warm-up
    step_ms = timed(lambda: [graph.replay() for _ in range(cycles)])
    tokens, blocks = cycles * 16 * mix.seqs, cycles * per_cycle
    assert (tokens, blocks) == (eager_tokens, eager_blocks)
    row_bytes = heads * 128 * 2
    moved = 2 * mix.num_planes * (tokens * row_bytes + blocks * row_bytes * mix.block_size)
    del graph
    # whole-cycle booking: one append_steps launch books the 16 steps of a
    # later cycle while the current cycle's moves run; a replay =
    # DecodeMix.CYCLE_BUFFERS cycles.  First each step's scatter paired with
    # the next step's gather (one launch per decode step), then each cycle's
    # moves as one move_cycle launch.
    mix.pipelined = False
    cpr = mix.CYCLE_BUFFERS
    replays = -(-cycles // cpr)
    cyc_steps = cpr * replays * 16
    results = {}
    for one_launch in (False, True):
        mix.start_cycles(one_launch=one_launch)
        mix.run_cycle(cycle_rows)
        graph, per_replay = mix.capture_cycles(cycle_rows)
        assert per_replay == cpr * per_cycle
        graph.replay()  # uploads the graph; untimed warm-up
        with ClockSampler(device.index) as clk:
            results[one_launch] = (timed(lambda: [graph.replay() for _ in range(replays)]), clk)
        del graph
        mix.stop_cycles(cycle_rows)
        torch.cuda.synchronize(device)
        ops.check_status(device)
    ms, clocks = results[False]
    one_ms = results[True][0]
    # launches per cycle: the booking, then one per step (the token scatter
    # with the next step's spill gather)
    cycle_launches = 1 + 16
    cyc_moved = 2 * mix.num_planes * (cyc_steps * mix.seqs * row_bytes + replays * per_replay * row_bytes * mix.block_size)
    if rank != 0:
        return
    decode_steps = cycles * 16
    peak, peak_kind = _peaks()
    line = {
        "metric": "paged-KV decode append + eviction gather GB/s",
        "value": round(world * cyc_moved / (ms / 1e3) / 1e9, 2),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms / cyc_steps * per, 4),
        "ms_per_decode_step": round(ms / cyc_steps, 5),
        "decode_steps_timed": cyc_steps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "fp16",
        "data": "synthetic (seeded N(0,1) cache and token rows, seeded pool state)",
        "config": {
            "workload": f"decode append + gather mix: 32 layers x K/V, {heads} KV head(s)/GPU, head_dim 128, "
                        f"block 16, fp16, {'full 65,536' if pool == 65536 else f'reduced {pool:,}'}-block pool, "
                        f"256 sequences x 1 token per decode step, "
                        f"{per} decode steps per bench step (timed in whole 16-step cycles), clock eviction + "
                        f"spill gather when a block fills",
            "parallelism": f"kv-head shard x{world}, no data-path collective",
        },
        "gpu_launches": replays * cpr * cycle_launches,
        "tokens_per_s": round(world * cyc_steps * mix.seqs / (ms / 1e3), 1),
        "evictions_per_s": round(world * replays * per_replay / (ms / 1e3), 1),
        "gpu_launches_per_decode_step": "one scatter_tokens_gather_layers launch (this step's token scatter with the "
                                        "next step's spill gather) plus 1/16 of an append_steps launch (pop, commit, "
                                        "release, slot_mapping of 16 steps)",
        "issue": f"CUDA graph, one replay per {cpr} 16-step cycles; the bookkeeping of each later cycle (one "
                 "append_steps launch) on a second stream, overlapping the current cycle's moves and up to two "
                 f"cycles ahead of them (victims and slot_mappings in {cpr} buffers by cycle); each step's moves "
                 "are one launch, issued as the step comes",
        "token_rows": "a new row per sequence, plane and step (16 steps' rows in HBM)",
        "roofline": {
            "bound": "hbm",
            "achieved": round(cyc_moved / (ms / 1e3) / 1e9, 1),
            "peak": peak,
            "unit": "GB/s",
            "frac": round(cyc_moved / (ms / 1e3) / 1e9 / peak, 4),
            "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured" else "fallback",
            "traffic": _traffic_per_launch("decode-mix-8heads") if heads == 8 else None,
            "kernel": f"{'move_pair_all_kernel' if heads == 8 else 'move_pair_kernel'} (one launch per decode step; "
                      "the cycle's booking runs beside the cycle's launches on another stream), timed over whole "
                      "graph replays",
            "algorithmic_bytes_per_decode_step": 2 * mix.num_planes * (mix.seqs * row_bytes +
                                                                       per_cycle // 16 * row_bytes * mix.block_size),
        },
        "one_launch_cycles_graph": {"value": round(world * cyc_moved / (one_ms / 1e3) / 1e9, 2), "unit": "GB/s",
                                    "ms_per_decode_step": round(one_ms / cyc_steps, 5),
                                    "gpu_launches_per_decode_step": 2 / 16,
                                    "issue": "same booking; each cycle's 16 spill gathers and 16 token scatters in "
                                             "one move_cycle launch (needs every step's token rows when the launch "
                                             "starts)"},
        "per_step_pipelined_graph": {"value": round(world * moved / (step_ms / 1e3) / 1e9, 2), "unit": "GB/s",
                                     "ms_per_decode_step": round(step_ms / decode_steps, 5),
                                     "issue": "CUDA graph per 16-step cycle, each step's append_step on a second "
                                              "stream, one step ahead of the moves"},
        "serial_graph": {"value": round(world * moved / (serial_ms / 1e3) / 1e9, 2), "unit": "GB/s",
                         "ms_per_decode_step": round(serial_ms / decode_steps, 5),
                         "issue": "CUDA graph, every step's launches in order on one stream"},
        "host_issued": {"value": round(world * moved / (eager_ms / 1e3) / 1e9, 2), "unit": "GB/s",
                        "ms_per_decode_step": round(eager_ms / decode_steps, 5),
                        "issue": "one Python call per op, one stream"},
        "clocks": clocks.summary(),
    }
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_decode_mix(heads, rows.cpu())
    print(json.dumps(line), flush=True)


def cpu_decode_mix(heads: int, rows: torch.Tensor, steps: int = 32) -> dict:
    """The decode mix's steps through the same driver on CPU tensors with the
    oracle op set (the reference's strict pop / commit / release restated,
    torch CPU indexing for the moves), on a smaller pool (the per-step moves
    are the same; the pool only sets how far the sweep scans)."""
    sys.path.insert(0, str(REPO / "tests"))
    from oracle_ops import OracleOps
    from kv_cache_adapter_b200.workloads import DecodeMix

    torch.set_num_threads(len(os.sched_getaffinity(0)))
    pool = 8192 if heads == 1 else 1024
    mix = DecodeMix(OracleOps(), torch.device("cpu"), layers=32, heads=heads, head_dim=128, block_size=16,
                    num_blocks=pool, seqs=256, dtype=torch.float16, seed=1234, max_steps=17 + steps + 16)
    for _ in range(17):
        mix.step(rows)
    tok0, blk0 = mix.tokens, mix.gathered_blocks
    t0 = time.perf_counter()
    for _ in range(steps):
        mix.step(rows)
    dt = time.perf_counter() - t0
    row_bytes = heads * 128 * 2
    moved = 2 * mix.num_planes * ((mix.tokens - tok0) * row_bytes + (mix.gathered_blocks - blk0) * row_bytes * 16)
    return {"value": round(moved / dt / 1e9, 3), "unit": "GB/s", "cores": torch.get_num_threads(), "kind": "port",
            "ms_per_decode_step": round(dt / steps * 1e3, 3),
            "sample": f"{steps} decode steps of the same shapes (256 sequences, 32 layers x K/V, {heads} KV head(s)) "
                      f"on a {pool:,}-block pool, CPU tensors, oracle op set (strict-path restatement) and torch "
                      f"CPU indexing"}


ADAPTER_CONFIG = dict(num_actual=256, num_logical=1024, batch=32, block=128, hit_rates=(0.0, 0.5, 1.0))


def _adapter_case(device, ops=None, backend_ops=None):
    from kv_cache_adapter_b200 import InMemoryBlockStoreBackend, KVCacheAdapter

    c = ADAPTER_CONFIG
    payloads = torch.arange(c["num_logical"] * c["block"], dtype=torch.float32, device=device)
    backend = InMemoryBlockStoreBackend(payloads.reshape(c["num_logical"], c["block"]), ops=backend_ops)
    actual = torch.zeros((c["num_actual"], c["block"]), dtype=torch.float32, device=device)
    return KVCacheAdapter(c["num_actual"], c["num_logical"], actual, backend, native_ext=ops)


def _sample_ids(ad, rng: "np.random.Generator", hit_rate: float) -> torch.Tensor:
    """Seeded batch: `hit_rate` of it resident unpinned logical ids, the rest
    non-resident ones, in random order (reads the adapter state on the host)."""
    import numpy as np

    c = ADAPTER_CONFIG
    p2l = ad._physical_to_logical.cpu().numpy()
    pins = (ad._slot_meta.cpu().numpy().astype(np.int64) & 15)
    resident = p2l[(p2l >= 0) & (pins == 0)]
    cold = np.setdiff1d(np.arange(c["num_logical"]), p2l[p2l >= 0])
    hits = int(round(c["batch"] * hit_rate))
    ids = np.concatenate([rng.permutation(resident)[:hits], rng.permutation(cold)[: c["batch"] - hits]])
    return torch.tensor(rng.permutation(ids), dtype=torch.int64, device=ad.actual_blocks.device)


def _time_adapter(ad, device, steps: int, warmup: int, complete_on_return: bool = False) -> list[dict]:
    """Host clock around each call.  complete_on_return: the call returns
    with its device work done (a device-store call through its session waits
    for the kernel's completion word), so the synchronisation that follows
    it is outside the timed region; otherwise it is inside."""
    import numpy as np

    def sync():
        if device.type == "cuda":
            torch.cuda.synchronize(device)

    c = ADAPTER_CONFIG
    rng = np.random.default_rng(1234)
    initial = torch.arange(c["num_actual"], dtype=torch.int64, device=device)
    ad.load(initial)
    ad.release(initial)
    out = []
    for hr in c["hit_rates"]:
        load_s = save_s = 0.0
        for i in range(warmup + steps):
            ids = _sample_ids(ad, rng, hr)
            sync()
            t0 = time.perf_counter()
            ad.load(ids)
            if not complete_on_return:
                sync()
            t1 = time.perf_counter()
            sync()
            ad.release(ids)
            ids = _sample_ids(ad, rng, hr)
            data = torch.tensor(rng.standard_normal((c["batch"], c["block"])), dtype=torch.float32, device=device)
            sync()
            t2 = time.perf_counter()
            ad.save(ids, data)
            if not complete_on_return:
                sync()
            t3 = time.perf_counter()
            sync()
            if i >= warmup:
                load_s += t1 - t0
                save_s += t3 - t2
        out.append({"hit_rate": hr, "load_ms": round(load_s * 1e3 / steps, 4), "save_ms": round(save_s * 1e3 / steps, 4)})
    return out


def run_adapter(args, world: int, rank: int, device) -> None:
    """KVCacheAdapter.load / save per call on the configuration of the
    reference's runtime-path benchmark (256 physical / 1,024 logical blocks,
    batch 32, 128-float blocks, in-memory backend on the device)."""
    steps = max(args.steps, 100)  # calls per hit rate and path: enough to average out single slow calls
    cuda_ad = _adapter_case(device)
    cuda_ad.load(torch.arange(ADAPTER_CONFIG["num_actual"], dtype=torch.int64, device=device))  # opens the session
    assert cuda_ad._session is not None
    cuda_ad.release(torch.arange(ADAPTER_CONFIG["num_actual"], dtype=torch.int64, device=device))
    cuda = _time_adapter(cuda_ad, device, steps, args.warmup, complete_on_return=True)
    planned_ad = _adapter_case(device)
    planned_ad._device_store = lambda: None  # one-launch plan, then the backend's own calls
    planned = _time_adapter(planned_ad, device, steps, args.warmup)
    stepwise_ad = _adapter_case(device)
    stepwise_ad._planned = False  # inspect, pop, commit as separate launches
    stepwise = _time_adapter(stepwise_ad, device, steps, args.warmup)
    if rank != 0:
        return
    calls = sum(2 for _ in cuda) * steps
    total_ms = sum((r["load_ms"] + r["save_ms"]) * steps for r in cuda)
    line = {
        "metric": "KVCacheAdapter load+save calls/s",
        "value": round(world * calls / (total_ms / 1e3), 1),
        "unit": "calls/s",
        "n_gpus": world,
        "steps": steps,
        "warmup": args.warmup,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "fp32",
        "data": "synthetic (seeded batches at fixed hit rates)",
        "config": {"workload": "adapter load/save: 256 physical / 1,024 logical blocks, batch 32, "
                               "128 x fp32 blocks, in-memory backend on the device, hit rates 0 / 0.5 / 1",
                   "timing": "host clock around each call, synchronised before; the device-store calls return "
                             "with their work done (the session waits for the kernel's completion word in pinned "
                             "host memory), the other paths are synchronised inside the timed region"},
        "per_hit_rate": cuda,
        "path": "device store through a session: one C call per load / save (plan, spill, fill, commit in one "
                "launch whose last action writes the counts and a completion word to pinned host memory)",
        "per_hit_rate_planned": planned,
        "per_hit_rate_stepwise": stepwise,
    }
    if world == 1 and not args.no_cpu_baseline:
        sys.path.insert(0, str(REPO / "tests"))
        from oracle_ops import OracleOps

        ops = OracleOps()
        cpu = _time_adapter(_adapter_case(torch.device("cpu"), ops, ops), torch.device("cpu"), steps, args.warmup)
        line["cpu_baseline"] = {"kind": "port", "cores": torch.get_num_threads(), "per_hit_rate": cpu,
                                "sample": "the same calls through the same adapter code on CPU tensors with "
                                          "the oracle op set (restatement of the reference's strict path)"}
    print(json.dumps(line), flush=True)


HOST_TIER_CONFIG = dict(num_actual=4096, num_logical=16384, moved=1024, block=(2, 16, 8, 128), dtype=torch.float16)


def run_host_tier(args, world: int, rank: int, device) -> None:
    """A load's traffic with a pinned host tier: per step, 1,024 random victim
    slots of 64 KiB merged K/V blocks (Llama-3-8B layer, bs 16, fp16) spill
    their old bytes to random rows of a 1 GiB pinned arena and are filled
    from 1,024 other rows.  Measured: the exchange kernel (both directions in
    one launch), the two directions as separate copy kernels, the reference's
    CUDA host path (one cudaMemcpyAsync per block and direction,
    adapter.py:960-966, :1035-1037), and contiguous copy-engine transfers of
    the same bytes, one direction at a time and both at once (the host link's
    duplex rate: the roofline)."""
    from kv_cache_adapter_b200 import kv_cache_adapter_cuda as ext

    c = HOST_TIER_CONFIG
    g = torch.Generator().manual_seed(1234)
    actual = torch.randn((c["num_actual"], *c["block"]), generator=g).to(c["dtype"]).to(device)
    arena = torch.zeros((c["num_logical"], *c["block"]), dtype=c["dtype"], pin_memory=True)
    block_bytes = actual[0].numel() * actual.element_size()
    k = c["moved"]
    plans = []
    for _ in range(args.warmup + args.steps):
        slots = torch.randperm(c["num_actual"], generator=g)[:k]
        rows = torch.randperm(c["num_logical"], generator=g)[: 2 * k]
        plans.append((slots.to(device), rows[:k].to(device), rows[k:].to(device)))
    stream = torch.cuda.current_stream(device)

    def timed(fn) -> float:
        for i in range(args.warmup):
            fn(i)
        torch.cuda.synchronize(device)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(args.warmup, args.warmup + args.steps):
            fn(i)
        e1.record(stream)
        torch.cuda.synchronize(device)
        return e0.elapsed_time(e1) / 1e3 / args.steps

    def exchange(i):
        slots, spill, fill = plans[i]
        ext.exchange_blocks(actual, slots, arena, spill, fill, check=False)

    def two_copies(i):
        slots, spill, fill = plans[i]
        ext.copy_blocks(actual, slots, arena, spill, check=False)
        ext.copy_blocks(arena, fill, actual, slots, check=False)

    host_plans = [tuple(t.cpu().tolist() for t in p) for p in plans]

    def per_block(i):
        slots, spill, fill = host_plans[i]
        for s_, r_ in zip(slots, spill):
            arena[r_].copy_(actual[s_], non_blocking=True)
        for s_, r_ in zip(slots, fill):
            actual[s_].copy_(arena[r_], non_blocking=True)

    staging_d = torch.empty((k, *c["block"]), dtype=c["dtype"], device=device)
    staging_d2 = torch.empty_like(staging_d)
    staging_h = torch.empty((k, *c["block"]), dtype=c["dtype"], pin_memory=True)
    staging_h2 = torch.empty_like(staging_h, pin_memory=True)
    side = torch.cuda.Stream(device)

    def ce_one_way(i):
        staging_h.copy_(staging_d, non_blocking=True)
        staging_d2.copy_(staging_h2, non_blocking=True)

    def ce_duplex(i):
        side.wait_stream(stream)
        staging_h.copy_(staging_d, non_blocking=True)
        with torch.cuda.stream(side):
            staging_d2.copy_(staging_h2, non_blocking=True)
        stream.wait_stream(side)

    t_x = timed(exchange)
    t_two = timed(two_copies)
    t_ref = timed(per_block)
    t_ce1 = timed(ce_one_way)
    t_ce2 = timed(ce_duplex)
    ext.check_status(device)
    moved = 2 * k * block_bytes  # bytes crossing the host link per step (half each way)
    # parity of the timed kernel on a fresh step: old bytes out, new bytes in
    slots, spill, fill = plans[-1]
    before = actual.index_select(0, slots).cpu()
    incoming = arena.index_select(0, fill.cpu()).clone()
    ext.exchange_blocks(actual, slots, arena, spill, fill)
    torch.cuda.synchronize(device)
    assert torch.equal(arena.index_select(0, spill.cpu()), before)
    assert torch.equal(actual.index_select(0, slots).cpu(), incoming)
    if rank != 0:
        return
    gbs = lambda t: round(moved / t / 1e9, 2)  # noqa: E731
    line = {
        "metric": "host-tier spill+fill GB/s",
        "value": round(world * moved / t_x / 1e9, 2),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(t_x * 1e3, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "fp16",
        "data": "synthetic (seeded N(0,1) blocks, seeded random slots and rows)",
        "config": {"workload": "host tier: 1,024 victim slots of 64 KiB blocks per step spill to and fill from "
                               "random rows of a 1 GiB pinned arena (exchange kernel)",
                   "bytes_per_step": moved},
        "roofline": {"bound": "host-link duplex", "achieved": gbs(t_x), "peak": gbs(t_ce2), "unit": "GB/s",
                     "frac": round(t_ce2 / t_x, 4), "traffic": None,
                     "peak_source": "contiguous cudaMemcpyAsync of the same bytes, both directions at once, this run"},
        "two_copy_kernels": {"value": gbs(t_two), "unit": "GB/s"},
        "per_block_memcpy": {"value": gbs(t_ref), "unit": "GB/s", "ms_per_step": round(t_ref * 1e3, 4),
                             "what": "one cudaMemcpyAsync per block and direction (reference CUDA host path)"},
        "copy_engine_one_way_at_a_time": {"value": gbs(t_ce1), "unit": "GB/s"},
        "gpu_launches": args.steps,
    }
    print(json.dumps(line), flush=True)


def run_reference(args, w: dict, world: int, rank: int) -> None:
    if rank != 0:
        return
    cpu = cpu_moves(w, steps=args.steps, warmup=args.warmup)
    line = {
        "impl": "reference",
        "metric": "paged-KV gather+scatter GB/s",
        "value": cpu["value"],
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": _dtype_name(w["dtype"]),
        "data": "synthetic (seeded N(0,1) cache, seeded random block tables)",
        "config": {"workload": w["label"], "sample": cpu["sample"]},
        "cpu_baseline": cpu,
        "e2e": {"value": cpu["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if not args.no_clock:
        # the reference's own CUDA pop kernel per call on the GPU, beside its strict CPU path
        line["pop"] = (reference_gpu_pop(torch.device("cuda", 0)) if torch.cuda.is_available()
                       else {"unavailable": "no CUDA device"})
        line["cpu_baseline_pop"] = cpu_strict_pop()
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS) + ["decode-mix", "adapter", "host-tier", "clock-stress",
                                                             "pop", "token-rows"],
                    default="llama70b-shard")
    ap.add_argument("--heads", type=int, default=None, help="KV heads per GPU for the decode mix (default 1)")
    ap.add_argument("--pool-blocks", type=int, default=None,
                    help="blocks of the decode mix's pool (default 65,536; smaller only for profiler captures)")
    ap.add_argument("--seqs", type=int, default=None,
                    help="override the number of sequences (smaller cases for profiling)")
    ap.add_argument("--row-bytes", type=int, default=None, help="token-rows: one row width instead of all")
    ap.add_argument("--pop-table", choices=["no-aging", "aging"], default=None, help="pop: one table instead of both")
    ap.add_argument("--move-mib", type=int, default=1024, help="token-rows: MiB per move (smaller for profiling)")
    ap.add_argument("--no-clock", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be at least 3")
    w = dict(WORKLOADS.get(args.workload, WORKLOADS["llama8b"]))
    if args.seqs is not None:
        w["seqs"] = args.seqs
        w["label"] += f" [reduced to {args.seqs} sequences]"
    world, rank, local = _dist()

    if args.impl == "reference":
        if args.workload == "pop":
            if rank == 0:
                print(json.dumps({"impl": "reference", "metric": "per-call pop evictions/s",
                                  "pop": reference_gpu_pop(torch.device("cuda", 0)),
                                  "cpu_baseline": cpu_strict_pop()}), flush=True)
            return
        run_reference(args, w, world, rank)
        return

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=device)
    try:
        if args.workload == "decode-mix":
            run_decode_mix(args, world, rank, device)
        elif args.workload == "adapter":
            run_adapter(args, world, rank, device)
        elif args.workload == "host-tier":
            run_host_tier(args, world, rank, device)
        elif args.workload == "clock-stress":
            run_clock_stress(args, world, rank, device)
        elif args.workload == "pop":
            run_pop(args, world, rank, device)
        elif args.workload == "token-rows":
            run_token_rows(args, world, rank, device)
        else:
            run_ours(args, w, world, rank, device)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
