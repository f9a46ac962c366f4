"""Benchmark of the grammar-masked selection hot path on B200.

Default workload (the headline metric): masked argmax over bf16 logits [64, 128256] with
per-row uint32 token bitmasks [64, 4008] (density U[0.5%, 20%]). A step is one kernel
launch over one 64-row batch. Distinct input sets totalling more than twice the L2 (17
sets, 297 MB, for the headline) are rotated so every step streams its batch from HBM; the K
timed steps are replayed from CUDA graphs behind a GPU-side delay.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload batched|spec_verify|table_gather|scaling|vocab_parallel|
                                dfa_masks|sample|grammar_row]

One process per GPU (torchrun for N > 1). Batches shard over ranks with no communication
("weak" scaling) except ``vocab_parallel``, which splits the vocabulary and exchanges 8-byte
row keys by NVLink peer stores (``--exchange nccl``: one all-gather). Rank 0 prints one JSON
line.

``--impl reference`` times the reference's own selection semantics on the host cores: the
CPU oracle (a C restatement of the reference's mask + first-max selection, OpenMP over
rows, every core the process may use), on the same workload and metric, rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "masked-argmax rows/s and HBM GB/s (vs ~8 TB/s), B=64 V=128256 bf16"
UNIT = "rows/s"

FALLBACK_HBM_GBS = 6650.0

# GPU-side delay (SM clock cycles, about 5 ms) enqueued just before the start event of a
# timed region: the host enqueues the timed graph replays while the GPU spins, so the
# region holds the steps back to back and none of the host's launch latency.
DELAY_CYCLES = 10_000_000

# dram__bytes_read.sum + dram__bytes_write.sum of one launch of each workload's dominant
# kernel on one B200, from a single-launch ncu capture of that kernel in this program
# (`--workload <name> --steps 3 --warmup 3`, the fifth launch). The vocabulary-sharded entry
# is the whole vocabulary on one rank (a rank of N reads 1/N of it); the batch-sharded entry
# is a launch of 128 rows (traffic grows with the rows).
NCU_TRAFFIC_PER_LAUNCH: dict[str, float] = {
    "batched": 17_459_712,
    "table_gather": 70_165_760,
    "spec_verify": 52_285_184,
    "scaling": 69_837_312,
    "vocab_parallel": 560_186_368,
    "grammar_row": 147_968,
    "dfa_masks": 1_756_928,
    "sample": 17_542_912,
}


# ---------------------------------------------------------------------------------------
# workload definitions (bytes follow the algorithmic count: every logit once, every mask
# word once, the outputs)
# ---------------------------------------------------------------------------------------
WORKLOADS = {
    "batched": dict(rows=64, vocab=128256, desc="masked argmax bf16 [64,128256], mask u32 [64,4008]"),
    "table_gather": dict(rows=256, vocab=128256,
                         desc="DFA table gather + masked argmax: table u32 [4096,4008], bf16 [256,128256]"),
    "spec_verify": dict(rows=32, vocab=151936, gamma=4,
                        desc="spec verify bf16 [32,5,151936], masks u32 [32,5,4748], drafts i32 [32,4]"),
    "scaling": dict(rows=1024, vocab=256000,
                    desc="batch-sharded masked argmax bf16 [1024,256000] at 5% density, rows split "
                         "over N GPUs ([1024/N,256000] each)"),
    "vocab_parallel": dict(rows=1024, vocab=256000,
                           desc="vocabulary-sharded masked argmax bf16 [1024,256000/N], row keys "
                                "exchanged between ranks"),
    "grammar_row": dict(rows=1, vocab=32000,
                        desc="one fp32 row [1,32000] under the grammar [0-9]{1,8} at its initial "
                             "state: the valid-token mask built on the GPU from the DFA state, "
                             "then the masked argmax"),
    "sample": dict(rows=64, vocab=128256, temperature=0.8, top_p=0.9,
                   desc="masked temperature / top-p sampling bf16 [64,128256], mask u32 [64,4008], "
                        "T=0.8, top_p=0.9"),
    "dfa_masks": dict(rows=64, vocab=128256,
                      desc="mask producer: valid-token masks of every state of a 64-state DFA "
                           "over 128,256 tokens, u32 [64,4008]"),
}


def bytes_per_row(name: str, world: int = 1) -> float:
    w = WORKLOADS[name]
    v = w["vocab"]
    words = (v + 31) // 32
    if name == "spec_verify":
        g1 = w["gamma"] + 1
        return g1 * (v * 2 + words * 4) + w["gamma"] * 4 + 12
    if name == "table_gather":
        return words * 4 + 4 + v * 2 + 8
    if name == "vocab_parallel":
        return (v * 2 + words * 4) / world + 8 + 8
    if name == "grammar_row":  # one f32 row, its mask words, the output
        return v * 4 + words * 4 + 4
    if name == "dfa_masks":  # per state row: its mask words written, plus its share of the
        # vocabulary read once per step (offsets 8 B/token, about 5 token bytes/token)
        return words * 4 + 4 + (v * 8 + v * 5) / w["rows"]
    return v * 2 + words * 4 + 8


L2_POLICY = {
    "dfa_masks": "inputs (the vocabulary and the DFA table) stay in L2 by design: the walk is "
                 "latency-bound and the masks are written once per step",
    "grammar_row": "logits rows rotate through distinct buffers totalling more than 2 x L2; "
                   "the vocabulary and the DFA table stay resident by design",
}


def rows_per_gpu(name: str, world: int) -> int:
    """Rows one GPU selects per step: the batch-sharded job of 1,024 rows splits over the
    ranks (strong scaling); every other workload is per GPU."""
    rows = WORKLOADS[name]["rows"]
    return rows // world if name == "scaling" else rows


def traffic_per_launch(name: str, world: int) -> float | None:
    """The captured DRAM traffic, scaled to one launch of this run's shard."""
    t = NCU_TRAFFIC_PER_LAUNCH.get(name)
    if t is None:
        return None
    if name == "vocab_parallel":
        return t / world
    if name == "scaling":
        return t * rows_per_gpu(name, world) / 128
    return t


def workload_config(name: str, world: int, exchange: str) -> dict:
    """The ``config`` object of a JSON line; both arms print the same one."""
    spec = WORKLOADS[name]
    if name == "vocab_parallel":
        par = f"vocab-sharded x{world}, keys exchanged by " + (
            "NVLink peer stores" if exchange == "peer" else "NCCL all-gather")
    elif name in ("dfa_masks", "grammar_row"):
        par = f"replicas x{world}"
    else:
        par = f"batch-sharded x{world}"
    return {
        "workload": name,
        "desc": spec["desc"],
        "rows_per_step_per_gpu": rows_per_gpu(name, world),
        "parallelism": par,
        "l2_policy": L2_POLICY.get(
            name, "input sets rotate through distinct device buffers totalling more than 2 x L2"),
    }


# ---------------------------------------------------------------------------------------
def _peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        data = json.loads(p.read_text())
        return float(data["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def gpu_delay(stream) -> None:
    """Keep the GPU busy on ``stream`` for about DELAY_CYCLES SM cycles (a spin kernel), so
    that work the host enqueues next starts back to back once the delay ends."""
    import torch

    with torch.cuda.stream(stream):
        torch.cuda._sleep(DELAY_CYCLES)


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while the timed region runs (from
    the GPU-side delay before its start event to its end)."""

    def __init__(self, device_index: int, period_s: float = 0.001) -> None:
        self.samples: list[tuple[int, int]] = []
        self.period = period_s
        self._stop = threading.Event()
        self._thread = None
        self.max_mhz = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nvml = pynvml
            uuid = None
            try:
                import torch

                uuid = str(torch.cuda.get_device_properties(device_index).uuid)
            except Exception:
                pass
            self._h = None
            if uuid:
                try:
                    self._h = pynvml.nvmlDeviceGetHandleByUUID(("GPU-" + uuid).encode())
                except Exception:
                    self._h = None
            if self._h is None:
                self._h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._nvml = None

    def _run(self) -> None:
        nv = self._nvml
        while not self._stop.is_set():
            try:
                sm = nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM)
                reasons = nv.nvmlDeviceGetCurrentClocksEventReasons(self._h)
                self.samples.append((sm, reasons))
            except Exception:
                pass
            time.sleep(self.period)

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
        if self._nvml is None or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        nv = self._nvml
        names = {
            "gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4,
            "hw_slowdown": 0x8, "sync_boost": 0x10, "sw_thermal_slowdown": 0x20,
            "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80,
            "display_clock_setting": 0x100,
        }
        seen = 0
        for _, r in self.samples:
            seen |= r
        mhz = sorted(s for s, _ in self.samples)
        del nv
        return {
            "sm_mhz": mhz[len(mhz) // 2],
            "sm_max_mhz": self.max_mhz,
            "reasons": [k for k, bit in names.items() if seen & bit],
            "samples": len(self.samples),
        }


# ---------------------------------------------------------------------------------------
# CPU reference arm / CPU baseline
# ---------------------------------------------------------------------------------------
def _cpu_inputs(name: str):
    from onyx_b200 import workloads

    if name in ("batched", "sample"):
        w = workloads.batched()
        return w
    if name == "table_gather":
        return workloads.table_gather()
    if name == "scaling":
        return workloads.scaling(rows=128)
    if name == "vocab_parallel":
        return workloads.scaling(rows=128)
    if name == "dfa_masks":
        rng = workloads.np.random.default_rng(workloads.SEEDS[4])
        return {"dfa": workloads.synthetic_dfa(rng, WORKLOADS[name]["rows"]),
                "vocabulary": workloads.synthetic_vocabulary(rng, WORKLOADS[name]["vocab"])}
    raise ValueError(name)


def cpu_measure(name: str, budget_s: float, steps: int | None = None, warmup: int = 0,
                min_seconds: float = 1.0):
    """Time the oracle (C, OpenMP over rows, all usable cores) on this workload.

    With ``steps``: whole blocks of ``steps`` calls until at least ``min_seconds`` have
    passed (or ``budget_s``). Without: calls until ``budget_s``.
    Returns (rows/s, threads, sample description, seconds, rows processed)."""
    import oracle

    threads = oracle.default_threads()
    oracle.load()
    if name == "spec_verify":
        from onyx_b200 import workloads

        w = workloads.spec_verify(lambda x, m: oracle.masked_argmax(x, m, dtype="bf16", threads=threads)[0])

        def run_once():
            oracle.spec_verify(w["logits_bf16"], w["masks"], w["drafts"], dtype="bf16", threads=threads)

        rows_per_call = w["logits_bf16"].shape[0]
        what = "spec verify of 32 entries x 5 rows x 151936 bf16"
    elif name == "grammar_row":
        from types import SimpleNamespace

        from onyx_b200 import workloads

        w = workloads.single_row()
        d = workloads.digits_dfa(8)
        dfa = SimpleNamespace(trans=d["trans"], dead=d["dead"])
        threads = 1  # one row: the scan and the selection run on one thread

        packed = oracle.pack_vocabulary(w["vocabulary"])  # once, as the reference holds its vocabulary

        def run_once():
            words = oracle.dfa_scan_bitmask(dfa, d["start"], w["vocabulary"], packed=packed)
            oracle.masked_argmax(w["logits"], words[None], dtype="f32", threads=1)

        rows_per_call = 1
        what = ("valid-token scan of 32000 tokens + masked argmax of one f32 row "
                "(the C oracle, one thread)")
    elif name == "sample":
        from oracle import sampling as osamp
        from onyx_b200 import workloads

        w = _cpu_inputs(name)
        spec = WORKLOADS[name]
        xs = workloads.bf16_bits_to_f32(w["logits_bf16"][:2]).astype(np.float64)
        ms_ = w["masks"][:2]
        threads = 1  # the float64 oracle is plain Python

        def run_once():
            osamp.masked_sample(xs, ms_, spec["temperature"], spec["top_p"], 1234, 0)

        rows_per_call = 2
        what = "masked sampling of 2 rows x 128256 bf16 (the float64 oracle, one thread)"
    elif name == "dfa_masks":
        w = _cpu_inputs(name)

        class _Dfa:  # the oracle's scan reads the table and the dead state
            trans = w["dfa"]["trans"]
            dead = w["dfa"]["dead"]

        def run_once():
            oracle.dfa_table(_Dfa, w["vocabulary"], threads=threads)

        rows_per_call = _Dfa.trans.shape[0]
        what = f"valid-token table of {rows_per_call} DFA states x {len(w['vocabulary'])} tokens"
    else:
        w = _cpu_inputs(name)
        if name == "table_gather":
            def run_once():
                oracle.gather_masked_argmax(w["logits_bf16"], w["table"], w["state_ids"],
                                            dtype="bf16", threads=threads)
            rows_per_call = w["logits_bf16"].shape[0]
            what = "table gather + masked argmax of 256 rows x 128256 bf16"
        else:
            def run_once():
                oracle.masked_argmax(w["logits_bf16"], w["masks"], dtype="bf16", threads=threads)
            rows_per_call = w["logits_bf16"].shape[0]
            what = f"masked argmax of {rows_per_call} rows x {w['logits_bf16'].shape[1]} bf16"
    for _ in range(warmup):
        run_once()
    t0 = time.perf_counter()
    n = 0
    while True:
        run_once()
        n += 1
        el = time.perf_counter() - t0
        if steps is not None:
            # whole blocks of `steps` calls, until at least min_seconds of work (or the budget)
            if (n % steps == 0 and el >= min_seconds) or el > budget_s:
                break
        elif el > budget_s and n >= 2:
            break
    el = time.perf_counter() - t0
    rows = n * rows_per_call
    return rows / el, threads, f"{n} calls of {what} ({rows} rows, {el:.1f} s)", el, rows


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    # bounded: each step is one call over the workload's batch; whole blocks of --steps
    # calls run until at least 1 s of CPU work is timed, and the run stops early once about
    # 60 s of CPU work is done, so any --steps finishes within minutes
    value, threads, sample, el, rows = cpu_measure(args.workload, budget_s=60.0,
                                                   steps=args.steps, warmup=min(args.warmup, 3),
                                                   min_seconds=1.0)
    line = {
        "impl": "reference",
        "metric": METRIC if args.workload == "batched" else f"{args.workload} rows/s",
        "value": value,
        "unit": UNIT,
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "higher_is_better": True,
        "scaling": "strong" if args.workload in ("vocab_parallel", "scaling") else "weak",
        "vs_baseline": None,
        "dtype": {"dfa_masks": "u32", "grammar_row": "f32"}.get(args.workload, "bf16"),
        "data": "synthetic (seeded, shapes and distributions of the workload)",
        "config": workload_config(args.workload, args.gpus, args.exchange),
        "timing": "wall clock (perf_counter) around whole blocks of --steps calls on the host "
                  "cores, at least 1 s",
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------------------
def run_ours(args) -> None:
    import torch
    import torch.distributed as dist

    from onyx_b200 import masked_selection as ms
    from onyx_b200 import sampling, vocab_parallel, workloads

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus and world > 1:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    distributed = world > 1
    if distributed:
        from datetime import timedelta

        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))

    name = args.workload
    spec = WORKLOADS[name]
    if name == "vocab_parallel" and not distributed:
        # one rank still selects through the exchange path: a single-member group
        dist.init_process_group("nccl", store=dist.HashStore(), rank=0, world_size=1,
                                device_id=dev)
    props = torch.cuda.get_device_properties(dev)
    l2 = int(getattr(props, "L2_cache_size", 126 * 2**20))

    def bf16(a):
        return torch.from_numpy(np.ascontiguousarray(a).view(np.int16)).to(dev).view(torch.bfloat16)

    def words(a):
        return torch.from_numpy(np.ascontiguousarray(a, dtype=np.uint32).view(np.int32)).to(dev)

    # ---- inputs, one seeded set copied into R rotating device buffers -------------------
    seed_shift = 17 * rank
    exchange = None  # vocab_parallel over NVLink peer memory (collective set-up)
    if name in ("batched", "sample"):
        w = workloads.batched(seed=workloads.SEEDS[2] + seed_shift)
        host_in = {"x": w["logits_bf16"], "m": w["masks"]}
    elif name == "table_gather":
        w = workloads.table_gather(seed=workloads.SEEDS[4] + seed_shift)
        host_in = {"x": w["logits_bf16"], "ids": w["state_ids"]}
        table = words(w["table"])
    elif name == "spec_verify":
        def gpu_argmax(x, m):
            r = ms.masked_argmax(bf16(x), words(m))
            return r.token_ids.cpu().numpy()
        w = workloads.spec_verify(gpu_argmax, seed=workloads.SEEDS[3] + seed_shift)
        host_in = {"x": w["logits_bf16"], "m": w["masks"], "d": w["drafts"]}
    elif name == "scaling":
        w = workloads.scaling(seed=workloads.SEEDS[5] + seed_shift, rows=rows_per_gpu(name, world))
        host_in = {"x": w["logits_bf16"], "m": w["masks"]}
    elif name == "vocab_parallel":
        if args.exchange == "peer":
            exchange = vocab_parallel.PeerExchange(rows_cap=spec["rows"], device=dev)
        w = workloads.scaling(seed=workloads.SEEDS[5], rows=spec["rows"])
        lo, hi = vocab_parallel.vocab_shard_bounds(spec["vocab"], rank, world)
        host_in = {"x": np.ascontiguousarray(w["logits_bf16"][:, lo:hi]),
                   "m": np.ascontiguousarray(w["masks"][:, lo // 32 : (hi + 31) // 32])}
        col_offset = lo
    else:
        raise SystemExit(f"unknown workload {name}")
    set_bytes = sum(v.nbytes for v in host_in.values())
    R = max(2, math.ceil(2 * l2 / set_bytes) + 1)
    bufs = []
    for _ in range(R):
        b = {}
        for k, v in host_in.items():
            if k == "x":
                b[k] = bf16(v)
            elif k in ("m",):
                b[k] = words(v)
            else:
                b[k] = torch.from_numpy(np.ascontiguousarray(v)).to(dev)
        bufs.append(b)
    rows_per_step = rows_per_gpu(name, world)

    def step(k: int):
        b = bufs[k % R]
        if name in ("batched", "scaling"):
            return ms.masked_argmax(b["x"], b["m"])
        if name == "table_gather":
            return ms.gather_masked_argmax(b["x"], table, b["ids"])
        if name == "sample":
            return sampling.masked_sample(b["x"], b["m"], temperature=spec["temperature"],
                                          top_p=spec["top_p"], seed=1234 + rank, call=k)
        if name == "spec_verify":
            return ms.spec_verify(b["x"], b["m"], b["d"])
        if name == "vocab_parallel":
            return vocab_parallel.vocab_parallel_masked_argmax(b["x"], b["m"], col_offset,
                                                               exchange=exchange)
        raise AssertionError

    launches_per_step = 1 if name != "vocab_parallel" else 2

    # ---- graphs of steps (the collective path is replayed eagerly) ----------------------
    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        for k in range(R):
            step(k)  # warm the workspace for this stream and load the library
    stream.synchronize()
    # the peer exchange counts its calls on the device, so its steps replay from graphs too;
    # the NCCL path is replayed eagerly
    use_graphs = name != "vocab_parallel" or exchange is not None
    chunk = min(args.steps, 1024)

    def make_graph(n: int):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for k in range(n):
                step(k)
        return g

    if use_graphs:
        g_main = make_graph(chunk)
        rem = args.steps % chunk
        g_rem = make_graph(rem) if rem else None
        reps = args.steps // chunk

    def run_steps(n_steps: int):
        # untimed: whole graph replays covering at least n_steps steps
        if use_graphs:
            with torch.cuda.stream(stream):
                for _ in range(max(1, math.ceil(n_steps / chunk))):
                    g_main.replay()
        else:
            with torch.cuda.stream(stream):
                for k in range(n_steps):
                    step(k)

    # ---- pre-heat (clocks up) + warm-up ------------------------------------------------
    t_end = time.perf_counter() + args.preheat_seconds
    while time.perf_counter() < t_end:
        run_steps(chunk if use_graphs else 16)
        stream.synchronize()
    run_steps(args.warmup)
    stream.synchronize()

    # ---- timed region -------------------------------------------------------------------
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    # NVML starts before the barrier: its start-up takes long enough on a busy box to skew
    # the ranks' timed regions by more than the peer exchange's wait limit
    clocks = ClockSampler(local)
    if distributed:
        dist.barrier()
    torch.cuda.synchronize(dev)
    with clocks:
        gpu_delay(stream)
        start.record(stream)
        if use_graphs:
            with torch.cuda.stream(stream):
                for _ in range(reps):
                    g_main.replay()
                if g_rem is not None:
                    g_rem.replay()
        else:
            run_steps(args.steps)
        end.record(stream)
        end.synchronize()
    torch.cuda.synchronize(dev)
    if distributed:
        dist.barrier()
    ms_total = start.elapsed_time(end)
    t = torch.tensor([ms_total], dtype=torch.float64, device=dev)
    per_rank = [t.clone() for _ in range(world)] if distributed else [t]
    if distributed:
        dist.all_gather(per_rank, t)
    per_rank_ms = [float(x.item()) for x in per_rank]
    ms_total = max(per_rank_ms)
    ms_per_step = ms_total / args.steps
    total_rows = rows_per_step * args.steps * (world if name != "vocab_parallel" else 1)
    value = total_rows / (ms_total / 1e3)

    # ---- roofline of the dominant kernel ------------------------------------------------
    per_launch_bytes = bytes_per_row(name, world) * rows_per_step
    achieved = per_launch_bytes / (ms_per_step / 1e3) / 1e9
    peak, peak_kind = _peaks()
    roofline = {
        "bound": "hbm",
        "achieved": achieved,
        "peak": peak,
        "unit": "GB/s",
        "frac": achieved / peak,
        "traffic": traffic_per_launch(name, world),
        "peak_source": f"MEASURED_PEAKS.json hbm_gbs (of {peak_kind})",
        "algorithmic_bytes_per_launch": per_launch_bytes,
    }

    # ---- end to end through the public API with host buffers ---------------------------
    # at least 200 steps (the copy pipeline's first step is not overlapped), bounded by about
    # 35 GB of host-to-device copies
    e2e_steps = max(args.steps, 200) if name != "vocab_parallel" else 50
    e2e_steps = min(e2e_steps, max(20, int(2000 * 17.5e6 / max(set_bytes, 1))))
    def _host_view(k, v):
        v = np.ascontiguousarray(v)
        if k == "x":
            return v.view(np.int16)
        return v.view(np.int32) if v.dtype == np.uint32 else v

    pinned = {k: torch.from_numpy(_host_view(k, v)).pin_memory() for k, v in host_in.items()}
    # two device input sets and two pinned result buffers: step k+1's inputs are copied on
    # their own stream while step k's kernel and read-back run
    out_host = [torch.empty((2, rows_per_step), dtype=torch.int32).pin_memory() for _ in range(2)]
    dev_in = [{k: torch.empty(v.shape, dtype=v.dtype, device=dev) for k, v in pinned.items()}
              for _ in range(2)]
    h2d = sum(v.numel() * v.element_size() for v in pinned.values())
    d2h = out_host[0].numel() * 4
    copy_stream = torch.cuda.Stream(dev)
    copied = [torch.cuda.Event() for _ in range(2)]
    consumed = [torch.cuda.Event() for _ in range(2)]

    def e2e_step(k: int):
        j = k & 1
        with torch.cuda.stream(copy_stream):
            if k >= 2:  # the kernel of step k-2 has finished reading this input set
                copy_stream.wait_event(consumed[j])
            for key, v in pinned.items():
                dev_in[j][key].copy_(v, non_blocking=True)
            copied[j].record(copy_stream)
        stream.wait_event(copied[j])
        with torch.cuda.stream(stream):
            d = dev_in[j]
            xin = d["x"].view(torch.bfloat16)
            if name in ("batched", "scaling"):
                r = ms.masked_argmax(xin, d["m"])
                out = (r.token_ids, r.status)
            elif name == "table_gather":
                r = ms.gather_masked_argmax(xin, table, d["ids"])
                out = (r.token_ids, r.status)
            elif name == "sample":
                r = sampling.masked_sample(xin, d["m"], temperature=spec["temperature"],
                                           top_p=spec["top_p"], seed=1234 + rank, call=0)
                out = (r.token_ids, r.status)
            elif name == "spec_verify":
                r = ms.spec_verify(xin, d["m"], d["d"])
                out = (r.accept_len, r.correction)
            else:
                r = vocab_parallel.vocab_parallel_masked_argmax(xin, d["m"], col_offset,
                                                                exchange=exchange)
                out = (r.token_ids, r.status)
            consumed[j].record(stream)
            out_host[j][0].copy_(out[0], non_blocking=True)
            out_host[j][1].copy_(out[1], non_blocking=True)

    # untimed warm-up of about 10 GB of copies (~0.2 s at the link's rate; the same count on
    # every rank): a host-to-device link that was idle runs below its rate for the first
    # tens of milliseconds of traffic
    for k in range(min(1000, max(3, math.ceil(1e10 / max(h2d, 1))))):
        e2e_step(k)
    torch.cuda.synchronize(dev)
    if distributed:
        dist.barrier()
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record(copy_stream)
    stream.wait_stream(copy_stream)
    for k in range(e2e_steps):
        e2e_step(k)
    e_end.record(stream)
    e_end.synchronize()
    et = torch.tensor([e_start.elapsed_time(e_end)], dtype=torch.float64, device=dev)
    if distributed:
        dist.all_reduce(et, op=dist.ReduceOp.MAX)
    e2e_rows = rows_per_step * e2e_steps * (world if name != "vocab_parallel" else 1)
    e2e_value = e2e_rows / (float(et.item()) / 1e3)
    # a timed-out exchange wait is sticky: the last step's statuses show whether any wait of
    # the timed or end-to-end steps gave up (those numbers would not be selections)
    if name != "spec_verify":
        last = out_host[(e2e_steps - 1) & 1][1]
        if bool(((last & ms.STATUS_WAIT_TIMEOUT) != 0).any()):
            raise RuntimeError(f"rank {rank}: a selection reported a wait timeout; no "
                               "measurement is printed")

    # ---- CPU baseline (rank 0, N=1 only) -----------------------------------------------
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, threads, sample, _, _ = cpu_measure(name, budget_s=args.cpu_seconds)
        cpu = {"value": v, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample}

    if exchange is not None:
        exchange.close()
    if dist.is_initialized():
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    clock = clocks.summary()
    line = {
        "metric": METRIC if name == "batched" else f"{name} rows/s",
        "value": value,
        "unit": UNIT,
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_per_step,
        "higher_is_better": True,
        "scaling": "strong" if name in ("vocab_parallel", "scaling") else "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,3) bf16 logits, Bernoulli token bitmasks)",
        "config": workload_config(name, world, args.exchange),
        "l2_rotation": f"{R} input sets ({R * set_bytes / 1e6:.0f} MB > 2 x L2 {l2 / 1e6:.0f} MB)",
        "timing": "CUDA events on the launching stream around K graph-replayed steps enqueued "
                  "behind a GPU-side delay, max over ranks",
        "per_rank_ms_per_step": [round(x / args.steps, 6) for x in per_rank_ms],
        "gbs": achieved,
        "roofline": roofline,
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h, "steps": e2e_steps},
        "cpu_baseline": cpu,
        "gpu_launches": args.steps * launches_per_step,
        "clocks": clock,
    }
    print(json.dumps(line), flush=True)


def run_dfa_masks(args) -> None:
    """Mask producer leg: each step builds the valid-token masks of every state of a
    synthetic DFA over the vocabulary (one launch). One GPU; N > 1 replicas (weak)."""
    import torch
    import torch.distributed as dist

    from onyx_b200 import dfa_masks, workloads

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
    spec = WORKLOADS["dfa_masks"]
    w = _cpu_inputs("dfa_masks")
    dfa, vocab = w["dfa"], w["vocabulary"]
    builder = dfa_masks.DfaMaskBuilder(dfa["trans"], dfa["dead"], vocab, device=dev)
    R = spec["rows"]
    states = torch.arange(R, dtype=torch.int32, device=dev)
    out_words = builder.words
    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        for _ in range(max(3, args.warmup)):
            builder.masks(states)
    stream.synchronize()
    chunk = min(args.steps, 1024)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for _ in range(chunk):
            builder.masks(states)
    graph.replay()
    stream.synchronize()
    clocks = ClockSampler(local)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with clocks:
        gpu_delay(stream)
        start.record(stream)
        done = 0
        with torch.cuda.stream(stream):
            while done < args.steps:
                graph.replay()
                done += chunk
        end.record(stream)
        end.synchronize()
    ms_total = start.elapsed_time(end)
    t = torch.tensor([ms_total / done], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_per_step = float(t.item())
    value = R * world / (ms_per_step / 1e3)
    peak, peak_kind = _peaks()
    per_launch = bytes_per_row("dfa_masks") * R
    achieved = per_launch / (ms_per_step / 1e3) / 1e9

    # end to end: the state ids up, the masks down, every step
    pinned_states = torch.arange(R, dtype=torch.int32).pin_memory()
    host_out = torch.empty((R, out_words), dtype=torch.int32).pin_memory()
    dev_states = torch.empty(R, dtype=torch.int32, device=dev)
    e2e_steps = min(max(args.steps, 200), 500)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        a.record(stream)
        for _ in range(e2e_steps):
            dev_states.copy_(pinned_states, non_blocking=True)
            host_out.copy_(builder.masks(dev_states), non_blocking=True)
        b.record(stream)
    b.synchronize()
    e2e_value = R * e2e_steps / (a.elapsed_time(b) / 1e3)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, threads, sample, _, _ = cpu_measure("dfa_masks", budget_s=args.cpu_seconds)
        cpu = {"value": v, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample}
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": "dfa_masks rows/s", "value": value, "unit": UNIT, "n_gpus": world,
        "steps": done, "warmup": args.warmup, "ms_per_step": ms_per_step,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u32",
        "data": "synthetic (seeded 64-state DFA, 20% live transitions; synthetic vocabulary)",
        "config": workload_config("dfa_masks", world, args.exchange),
        "timing": "CUDA events on the launching stream around graph-replayed steps enqueued "
                  "behind a GPU-side delay",
        "gbs": achieved,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": NCU_TRAFFIC_PER_LAUNCH.get("dfa_masks"),
                     "peak_source": f"MEASURED_PEAKS.json hbm_gbs (of {peak_kind})",
                     "algorithmic_bytes_per_launch": per_launch},
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": R * 4,
                "d2h_bytes_per_step": R * out_words * 4, "steps": e2e_steps},
        "cpu_baseline": cpu,
        "gpu_launches": done,
        "clocks": clocks.summary(),
    }
    print(json.dumps(line), flush=True)


def run_grammar_row(args) -> None:
    """One-row grammar leg: each step builds the row's valid-token mask on the GPU from the
    DFA state (the reference's per-step scan) and selects the masked argmax of one fp32 row:
    two launches. Logits rows rotate through more than twice the L2; the vocabulary and the
    DFA table stay resident by design. One GPU; N > 1 replicas (weak)."""
    import torch
    import torch.distributed as dist

    from onyx_b200 import dfa_masks
    from onyx_b200 import masked_selection as ms
    from onyx_b200 import workloads

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
    spec = WORKLOADS["grammar_row"]
    w = workloads.single_row()
    d = workloads.digits_dfa(8)
    builder = dfa_masks.DfaMaskBuilder(d["trans"], d["dead"], w["vocabulary"], device=dev)
    V = spec["vocab"]
    props = torch.cuda.get_device_properties(dev)
    l2 = int(getattr(props, "L2_cache_size", 126 * 2**20))
    R = math.ceil(2 * l2 / (V * 4)) + 1
    gen = torch.Generator(device=dev)
    gen.manual_seed(workloads.SEEDS[1] + 17 * rank)
    X = torch.randn((R, V), generator=gen, device=dev, dtype=torch.float32) * 3.0
    X[0].copy_(torch.from_numpy(w["logits"][0]).to(dev))
    states = torch.full((1,), d["start"], dtype=torch.int32, device=dev)

    def step(k: int):
        m = builder.masks(states)
        return ms.masked_argmax(X[k % R : k % R + 1], m)

    stream = torch.cuda.Stream(dev)
    with torch.cuda.stream(stream):
        for k in range(max(3, args.warmup)):
            step(k)
    stream.synchronize()
    chunk = min(args.steps, 1024)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for k in range(chunk):
            step(k)
    with torch.cuda.stream(stream):
        graph.replay()
    stream.synchronize()
    clocks = ClockSampler(local)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with clocks:
        gpu_delay(stream)
        start.record(stream)
        done = 0
        with torch.cuda.stream(stream):
            while done < args.steps:
                graph.replay()
                done += chunk
        end.record(stream)
        end.synchronize()
    t = torch.tensor([start.elapsed_time(end) / done], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_per_step = float(t.item())
    value = world / (ms_per_step / 1e3)
    peak, peak_kind = _peaks()
    per_launch = bytes_per_row("grammar_row")
    achieved = per_launch / (ms_per_step / 1e3) / 1e9

    # the table path, for context: every state's mask built once, then one gather launch per
    # step (the state id selects the row's mask from the table)
    table = builder.table()
    g_graph = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        for k in range(3):
            ms.gather_masked_argmax(X[k % R : k % R + 1], table, states)
    stream.synchronize()
    with torch.cuda.graph(g_graph, stream=stream):
        for k in range(chunk):
            ms.gather_masked_argmax(X[k % R : k % R + 1], table, states)
    with torch.cuda.stream(stream):
        g_graph.replay()
    stream.synchronize()
    ta, tb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    gpu_delay(stream)
    ta.record(stream)
    g_done = 0
    with torch.cuda.stream(stream):
        while g_done < args.steps:
            g_graph.replay()
            g_done += chunk
    tb.record(stream)
    tb.synchronize()
    table_us = ta.elapsed_time(tb) / g_done * 1e3

    # end to end: the row and the state id up, the token id and status down, every step
    pinned_x = torch.from_numpy(w["logits"]).pin_memory()
    pinned_s = torch.full((1,), d["start"], dtype=torch.int32).pin_memory()
    host_out = torch.empty((2, 1), dtype=torch.int32).pin_memory()
    dev_x = torch.empty((1, V), dtype=torch.float32, device=dev)
    dev_s = torch.empty(1, dtype=torch.int32, device=dev)

    def e2e_step():
        dev_x.copy_(pinned_x, non_blocking=True)
        dev_s.copy_(pinned_s, non_blocking=True)
        r = ms.masked_argmax(dev_x, builder.masks(dev_s))
        host_out[0].copy_(r.token_ids, non_blocking=True)
        host_out[1].copy_(r.status, non_blocking=True)

    e2e_steps = min(max(args.steps, 200), 2000)
    with torch.cuda.stream(stream):
        for _ in range(3):
            e2e_step()
    stream.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        a.record(stream)
        for _ in range(e2e_steps):
            e2e_step()
        b.record(stream)
    b.synchronize()
    e2e_value = e2e_steps * world / (a.elapsed_time(b) / 1e3)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        v, threads, sample, _, _ = cpu_measure("grammar_row", budget_s=args.cpu_seconds)
        cpu = {"value": v, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample}
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    line = {
        "metric": "grammar_row rows/s", "value": value, "unit": UNIT, "n_gpus": world,
        "steps": done, "warmup": args.warmup, "ms_per_step": ms_per_step,
        "us_per_row": ms_per_step * 1e3,
        "table_path_us_per_row": table_us,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,3) f32 logits; synthetic 32,000-token vocabulary; "
                "the grammar [0-9]{1,8})",
        "config": workload_config("grammar_row", world, args.exchange),
        "l2_rotation": f"{R} logits rows ({R * V * 4 / 1e6:.0f} MB > 2 x L2)",
        "timing": "CUDA events on the launching stream around graph-replayed steps enqueued "
                  "behind a GPU-side delay; 2 launches per step (mask producer, masked argmax)",
        "gbs": achieved,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak,
                     "traffic": NCU_TRAFFIC_PER_LAUNCH.get("grammar_row"),  # the argmax launch
                     "peak_source": f"MEASURED_PEAKS.json hbm_gbs (of {peak_kind})",
                     "algorithmic_bytes_per_launch": per_launch},
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": V * 4 + 4,
                "d2h_bytes_per_step": 8, "steps": e2e_steps},
        "cpu_baseline": cpu,
        "gpu_launches": done * 2,
        "clocks": clocks.summary(),
    }
    print(json.dumps(line), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=4000)
    ap.add_argument("--warmup", type=int, default=200)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="batched")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--exchange", choices=["peer", "nccl"], default="peer",
                    help="vocab_parallel: keys over NVLink peer memory, or an NCCL all-gather")
    ap.add_argument("--preheat-seconds", type=float, default=0.5,
                    help="untimed replays before the warm-up, to bring the SM clock up")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "dfa_masks":
        run_dfa_masks(args)
    elif args.workload == "grammar_row":
        run_grammar_row(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
