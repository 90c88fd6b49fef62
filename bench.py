"""Benchmark: NanoRTS env-steps/s on B200 (BASELINE.json metric).

Headline workload (configs[1] of BASELINE.json): basesWorkers16x16,
VERSION_ORIGINAL, CANCEL_RANDOM, 70 slots per player, symbolic uint8[16,16,6]
observations, 16384 games per GPU, both players draw uniform random legal
actions per factor from the masks, auto-reset.  One step = one nrts_step
launch: decode, core step, auto-reset, the next step's masks and both
observations, and the fused uniform draw of the next actions from those masks
(``--separate-sampler`` draws them with nrts_sample_actions instead).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--config C] [--impl reference]

After the headline, the line's ``configs`` key holds the other BASELINE.json
configurations measured the same way (fewer steps): 1 (basesWorkers8x8,
1024 games per GPU), 3 (fine-tuned table, CANCEL_ALTERNATING, partial
observability, 65536 games split over the GPUs), 4 (WorkerRush against
LightRush, 32768 games per GPU, one nrts_duel_step per step) and 5
(GardenOfWar64x64, 4096 games per GPU).  ``--config N`` makes N the headline;
``--only`` skips the others.

Under torchrun each rank steps its own games (no collective on the step
path); one NCCL all-reduce of episode statistics runs after the timed region,
over a stretch long enough for every game to end at least once.  Rank 0
prints one JSON line.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
METRIC = "env steps/sec (both players, incl. masks+obs)"
DUEL_METRIC = "env steps/sec (bot vs bot: both bots' commands + core step + auto-reset)"
MAP, UTT = "basesWorkers16x16", "VERSION_ORIGINAL"
DUEL_STRATEGY = "CANCEL_BOTH"
DUEL_LANES = 32768
# BASELINE.json configs with uniform random legal actions (config 4 is the duel):
# map, unit table, conflict strategy, partial observability, capacity profile,
# games (per GPU, or in all for strong scaling), scaling.
CONFIGS = {
    1: ("basesWorkers8x8", "VERSION_ORIGINAL", "CANCEL_BOTH", False, True, 1024, "weak"),
    2: ("basesWorkers16x16", "VERSION_ORIGINAL", "CANCEL_RANDOM", False, True, 16384, "weak"),
    3: ("basesWorkers16x16", "VERSION_ORIGINAL_FINETUNED", "CANCEL_ALTERNATING", True, True, 65536, "strong"),
    5: ("GardenOfWar64x64", "VERSION_ORIGINAL", "CANCEL_RANDOM", False, False, 4096, "weak"),
}
# family.py strategy numbers and trained types of WorkerRush (player 0) and LightRush (player 1).
DUEL_BOTS = ((0, -1), (1, 4))
MAX_CYCLES = 5000
# Untimed steps from the reset before each timed region: the midpoint of the
# run BASELINE.json configures (1000 / 2000 / 2000 / 3000 steps for configs 1,
# 2, 3, 5; config 4's games end after 400-1000 steps), so the timed steps see
# mid-game states rather than the first steps after a reset.
MIDPOINT = {1: 500, 2: 1000, 3: 1000, 4: 300, 5: 1500}

# The kernel each configuration's step launches on a B200 (148 SMs) and the
# committed ncu summary holding its DRAM bytes per env-step.
KERNELS = {
    1: ("nrts::step_kernel_wide<8> (2-warp CTAs, the whole batch resident)", None),
    2: ("nrts::step_kernel_big<16>", "step_kernel_16x16_traffic.txt"),
    3: ("nrts::step_kernel_big<16>", "step_kernel_16x16_partial_traffic.txt"),
    4: ("nrts::duel_kernel_big<16>", "duel_kernel_16x16_traffic.txt"),
    5: ("nrts::step_kernel_wide<64>", "step_kernel_64x64_traffic.txt"),
}


def scenario(config: int):
    from nanorts_b200 import map_name_to_scenario

    if config == 4:
        return map_name_to_scenario(MAP, utt=UTT, conflict_strategy=DUEL_STRATEGY, max_cycles=MAX_CYCLES)
    name, utt, strategy, _, profile, _, _ = CONFIGS[config]
    return map_name_to_scenario(name, utt=utt, conflict_strategy=strategy, max_cycles=MAX_CYCLES,
                                capacity_profile=profile)


def workload_name(config: int) -> str:
    if config == 4:
        return (f"configs[3]: {MAP} {UTT} {DUEL_STRATEGY}, player_0 WorkerRush vs player_1 LightRush, every game "
                f"from its reset, auto-reset, max_cycles {MAX_CYCLES}")
    name, utt, strategy, partial, profile, _, _ = CONFIGS[config]
    obs = ", partial observability" if partial else ""
    cap = "" if profile else ", capacity_profile=False"
    return f"configs[{config - 1}]: {name} {utt} {strategy}{obs}{cap}, uniform random legal actions per factor, auto-reset"


def default_lanes(config: int) -> int:
    return DUEL_LANES if config == 4 else CONFIGS[config][5]


def scaling_of(config: int) -> str:
    return "weak" if config == 4 else CONFIGS[config][6]


def state_bytes(game) -> int:
    """One game's State in the reference layout plus the 12 lifecycle bytes."""
    b = game.bucket
    return 35 * b.entity_capacity + 2 * b.cell_count + 37 + 12


def algorithmic_bytes(game, fused: bool) -> dict[str, int]:
    """Bytes one env-step must move: the State read and written in place, both
    players' action rows, legality rows, feature maps and scalars, the step
    outputs; with the fused draw also the next step's action rows."""
    b = game.bucket
    C = b.per_player_capacity
    parts = {
        "state_read": state_bytes(game),
        "state_write": state_bytes(game),
        "actions": 2 * C * 7 * 4,
        "masks": 2 * C * b.mask_width,
        "observations": 2 * (b.cell_count * 6 + 16),
        "outputs": 8 + 1 + 1 + 1 + 4 + 8,
    }
    if fused:
        parts["sampled_actions"] = 2 * C * 7 * 4
    parts["total"] = sum(parts.values())
    parts["total_without_draw"] = parts["total"] - parts.get("sampled_actions", 0)
    return parts


def duel_algorithmic_bytes(game) -> dict[str, int]:
    """Bytes one bot-against-bot env-step must move: the State read and written
    in place, both players' carries (nine int32 fields, trained, next_order per
    slot block) read and written, and the step outputs."""
    C = game.bucket.per_player_capacity
    carry = 37 * C + 4
    parts = {
        "state_read": state_bytes(game),
        "state_write": state_bytes(game),
        "carries_read": 2 * carry,
        "carries_write": 2 * carry,
        "outputs": 8 + 1 + 1 + 1 + 4 + 8,
    }
    parts["total"] = sum(parts.values())
    return parts


def load_peaks() -> tuple[float, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        return float(json.loads(path.read_text())["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def load_traffic(config: int) -> float | None:
    """DRAM bytes per env-step of the measured kernel from the committed ncu summary."""
    name = KERNELS[config][1]
    if name is None:
        return None
    path = ROOT / "profiles" / name
    if not path.exists():
        return None
    for line in path.read_text().splitlines():
        if line.startswith("dram_bytes_per_env_step:"):
            return float(line.split(":", 1)[1])
    return None


# Environment states (each on its own stream) the end-to-end loop splits a
# GPU's games into.
E2E_SHARDS = 8


class ClockSampler:
    """Samples SM clocks and throttle reasons through NVML every 5 ms while running."""

    REASONS = {
        "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40, "sw_power_cap": 0x4,
        "hw_power_brake_slowdown": 0x80,
    }

    def __init__(self, device_index: int) -> None:
        self.samples: list[tuple[int, int]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nvml = pynvml
            self._handle = nvml_handle(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._handle, pynvml.NVML_CLOCK_SM)
        except Exception:  # noqa: BLE001 - clocks are reported as unknown
            self._nvml = None
        self._thread = threading.Thread(target=self._run, daemon=True)

    def _run(self) -> None:
        while not self._stop.is_set():
            try:
                mhz = self._nvml.nvmlDeviceGetClockInfo(self._handle, self._nvml.NVML_CLOCK_SM)
                reasons = self._nvml.nvmlDeviceGetCurrentClocksEventReasons(self._handle)
                self.samples.append((mhz, reasons))
            except Exception:  # noqa: BLE001
                pass
            time.sleep(0.005)

    def __enter__(self):
        if self._nvml is not None:
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._nvml is not None:
            self._thread.join()

    def summary(self, window: str) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0, "window": window}
        seen = 0
        for _, r in self.samples:
            seen |= r
        return {
            "sm_mhz": statistics.median(m for m, _ in self.samples),
            "sm_max_mhz": self.max_mhz,
            "reasons": sorted(name for name, bit in self.REASONS.items() if seen & bit),
            "samples": len(self.samples),
            "window": window,
        }


def nvml_handle(device_index: int):
    """The NVML handle of CUDA device `device_index` (matched by PCI address)."""
    import pynvml
    import torch

    p = torch.cuda.get_device_properties(device_index)
    return pynvml.nvmlDeviceGetHandleByPciBusId(f"{p.pci_domain_id:08X}:{p.pci_bus_id:02X}:{p.pci_device_id:02X}.0")


def gpu_local_cpus(device_index: int) -> list[int] | None:
    """Host CPUs on the GPU's NUMA node (NVML's CPU affinity of the device), or None."""
    try:
        import pynvml

        pynvml.nvmlInit()
        words = pynvml.nvmlDeviceGetCpuAffinity(nvml_handle(device_index), ((os.cpu_count() or 64) + 63) // 64)
        cpus = {64 * i + bit for i, w in enumerate(words) for bit in range(64) if (int(w) >> bit) & 1}
        allowed = cpus & os.sched_getaffinity(0)
        return sorted(allowed) or None
    except Exception:  # noqa: BLE001 - placement is then the default
        return None


class NodeLocal:
    """Runs the body with this process on the GPU's local CPUs, so pinned host
    buffers allocated (and first touched) inside land on the GPU's NUMA node;
    the process's CPU set is restored afterwards."""

    def __init__(self, device_index: int) -> None:
        self.cpus = gpu_local_cpus(device_index)
        self.before = os.sched_getaffinity(0)

    def __enter__(self):
        if self.cpus:
            os.sched_setaffinity(0, self.cpus)
        return self

    def __exit__(self, *exc):
        os.sched_setaffinity(0, self.before)


def pinned_copy_bandwidth(device, megabytes: int = 128, reps: int = 5) -> dict:
    """Pinned host<->device copy bandwidth of this rank, both directions at once
    on two streams (the e2e loop overlaps them), best of `reps`, GB/s."""
    import torch

    n = megabytes << 20
    with NodeLocal(device.index):
        host_in = torch.empty(n, dtype=torch.uint8).pin_memory()
        host_out = torch.empty(n, dtype=torch.uint8).pin_memory()
    dev_in = torch.empty(n, dtype=torch.uint8, device=device)
    dev_out = torch.empty(n, dtype=torch.uint8, device=device)
    up, down = torch.cuda.Stream(device), torch.cuda.Stream(device)
    best = {"h2d": 0.0, "d2h": 0.0, "both": 0.0}
    for _ in range(reps):
        for kind in ("h2d", "d2h", "both"):
            torch.cuda.synchronize(device)
            t0 = time.perf_counter()
            if kind in ("h2d", "both"):
                with torch.cuda.stream(up):
                    dev_in.copy_(host_in, non_blocking=True)
            if kind in ("d2h", "both"):
                with torch.cuda.stream(down):
                    host_out.copy_(dev_out, non_blocking=True)
            torch.cuda.synchronize(device)
            moved = n * (2 if kind == "both" else 1)
            best[kind] = max(best[kind], moved / (time.perf_counter() - t0) / 1e9)
    return best


def cpu_baseline(game, seconds: float = 12.0, lanes: int = 512, threads: int | None = None, partial: bool = False,
                 label: str = "") -> dict:
    """The CPU oracle (C++ restatement of the reference's JAX program path,
    OpenMP over games) on a bounded sample of the same workload."""
    from oracle.oracle import Oracle, sample_uniform_legal

    threads = threads or os.cpu_count() or 1
    orc = Oracle(game, lanes, threads=threads, partial_observability=partial)
    rng = np.random.default_rng(0)
    orc.reset(rng.integers(0, 2**32, size=(lanes, 2), dtype=np.uint64).astype(np.uint32))
    widths = (6, 4, 4, 4, 4, game.bucket.unit_type_capacity, game.bucket.attack_offset_capacity)
    for _ in range(3):  # warm-up
        orc.step(sample_uniform_legal(orc.legal_masks(), widths, rng))
    steps, step_time = 0, 0.0
    start = time.perf_counter()
    while time.perf_counter() - start < seconds:
        actions = sample_uniform_legal(orc.legal_masks(), widths, rng)
        t0 = time.perf_counter()
        orc.step(actions)
        orc.legal_masks()  # masks of the next step are part of the metric
        step_time += time.perf_counter() - t0
        steps += 1
    return {
        "value": lanes * steps / step_time,
        "unit": "env-steps/s",
        "cores": threads,
        "kind": "port",
        "sample": f"{lanes} games x {steps} steps of {label}, C++ oracle step + masks + observations "
                  f"(sampling excluded), {threads} OpenMP threads",
    }


def duel_cpu_baseline(game, seconds: float = 12.0, lanes: int = 256, threads: int | None = None) -> dict:
    """The CPU oracle's bot-against-bot step (C++ restatement of the reference's
    JAX program path for WorkerRush/LightRush and core.step, OpenMP over games)
    on a bounded sample: `lanes` games from their reset, stepped for `seconds`."""
    from oracle.oracle import Oracle, empty_carry

    threads = threads or os.cpu_count() or 1
    orc = Oracle(game, lanes, threads=threads)
    orc.reset(np.zeros((lanes, 2), np.uint32))
    C = game.bucket.per_player_capacity
    carries = (empty_carry(lanes, C), empty_carry(lanes, C))
    strategies, trained = tuple(b[0] for b in DUEL_BOTS), tuple(b[1] for b in DUEL_BOTS)
    for _ in range(3):
        orc.duel_step(strategies, trained, carries)
    steps, start = 0, time.perf_counter()
    while time.perf_counter() - start < seconds:
        orc.duel_step(strategies, trained, carries)
        steps += 1
    elapsed = time.perf_counter() - start
    return {
        "value": lanes * steps / elapsed,
        "unit": "env-steps/s",
        "cores": threads,
        "kind": "port",
        "sample": f"{lanes} games x {steps} steps of {MAP}/{DUEL_STRATEGY} WorkerRush vs LightRush from the reset, "
                  f"C++ oracle bots + core step + auto-reset, {threads} OpenMP threads",
    }


# ---------------------------------------------------------------------------
# The reference arm
# ---------------------------------------------------------------------------
def reference_gpu_kernels(config: int, lanes: int, steps: int, warmup: int, soak: int | None = None) -> dict:
    """The reference's own CUDA kernels (built unchanged for sm_100 by
    oracle/Makefile target `ref`) on this box's GPU, for the same workload:
    per step nanorts_legality_words, nanorts_visible_cells x2 (partial
    observability), nanorts_step and nanorts_reset_packed_where_done, with
    torch in place of the reference's XLA fusions between them (not timed;
    the observation fusion is not computed at all).  Kernel time only."""
    import torch

    from oracle import ref_kernels

    if not ref_kernels.available():
        return {"unavailable": "oracle/_ref/libref_kernels.so not built (make -C oracle ref with a NanoRTS checkout)"}
    if config == 4:
        return reference_duel_kernels(lanes, steps, warmup, soak)
    game = scenario(config)
    path = ref_kernels.ReferencePath(game, lanes, partial=CONFIGS[config][3], seed=0)
    soak = MIDPOINT[config] if soak is None else soak
    for _ in range(warmup + soak):  # mid-game states, as the timed steps of this implementation
        path.step(timed=False)
    torch.cuda.synchronize()
    path.kernel_ms.clear()
    for _ in range(steps):
        path.step(timed=True)
    ms = statistics.mean(path.kernel_ms)
    kernels = ["nanorts_legality_words", "nanorts_step", "nanorts_reset_packed_where_done"]
    if CONFIGS[config][3]:
        kernels.insert(1, "nanorts_visible_cells x2")
    return {
        "value": lanes / (ms * 1e-3),
        "unit": "env-steps/s",
        "kernel_ms_per_step": ms,
        "games": lanes,
        "steps": steps,
        "untimed_steps_before": warmup + soak,
        "kernels": kernels,
        "build": "reference sources unchanged, nvcc -O3 -gencode arch=compute_100,code=sm_100 (the image its own "
                 "build makes for a B200)",
        "excluded": "the reference's XLA fusions (action decode, observations, mask assembly, lifecycle select) "
                    "stand in as untimed torch ops; observations are not computed",
    }


def reference_duel_kernels(lanes: int, steps: int, warmup: int, soak: int | None = None) -> dict:
    """Config 4 on the reference's own kernels (sm_100, same B200): per step
    nanorts_abstraction_act for each player's bot, nanorts_step and
    nanorts_reset_packed_where_done, with torch for the seat merge, the
    counter select and the carry reset (untimed).  Kernel time only."""
    import torch

    from oracle import ref_kernels

    path = ref_kernels.ReferenceDuelPath(scenario(4), lanes, DUEL_BOTS)
    soak = MIDPOINT[4] if soak is None else soak
    for _ in range(warmup + soak):
        path.step(timed=False)
    torch.cuda.synchronize()
    path.kernel_ms.clear()
    for _ in range(steps):
        path.step(timed=True)
    ms = statistics.mean(path.kernel_ms)
    return {
        "value": lanes / (ms * 1e-3),
        "unit": "env-steps/s",
        "kernel_ms_per_step": ms,
        "games": lanes,
        "steps": steps,
        "untimed_steps_before": warmup + soak,
        "kernels": ["nanorts_abstraction_act x2", "nanorts_step", "nanorts_reset_packed_where_done"],
        "build": "reference sources unchanged, nvcc -O3 -gencode arch=compute_100,code=sm_100 (the image its own "
                 "build makes for a B200)",
        "excluded": "the seat merge of the two bots' Commands, the lifecycle select and the carry reset stand in as "
                    "untimed torch ops",
    }


def run_reference(args) -> None:
    """--impl reference: the reference's CPU path for this workload.  The
    reference's JAX program cannot run here (jax absent, the install fails),
    so its C++ restatement (the oracle) runs on all host cores, each step a
    bounded sample of the workload.  Where a GPU and the reference-kernel
    build are present, the line also carries the reference's own sm_100
    kernels timed on the same B200 (``gpu_kernels``)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    config = args.config
    game = scenario(config)
    if config == 4:
        from oracle.oracle import Oracle, empty_carry

        lanes = 256
        orc = Oracle(game, lanes, threads=threads)
        orc.reset(np.zeros((lanes, 2), np.uint32))
        C = game.bucket.per_player_capacity
        carries = (empty_carry(lanes, C), empty_carry(lanes, C))
        strategies, trained = tuple(b[0] for b in DUEL_BOTS), tuple(b[1] for b in DUEL_BOTS)
        for _ in range(args.warmup):
            orc.duel_step(strategies, trained, carries)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            orc.duel_step(strategies, trained, carries)
        elapsed = time.perf_counter() - t0
        metric = DUEL_METRIC
    else:
        from oracle.oracle import Oracle, sample_uniform_legal

        lanes = 256 if config != 5 else 32
        orc = Oracle(game, lanes, threads=threads, partial_observability=CONFIGS[config][3])
        rng = np.random.default_rng(0)
        orc.reset(rng.integers(0, 2**32, size=(lanes, 2), dtype=np.uint64).astype(np.uint32))
        widths = (6, 4, 4, 4, 4, game.bucket.unit_type_capacity, game.bucket.attack_offset_capacity)
        for _ in range(args.warmup):
            orc.step(sample_uniform_legal(orc.legal_masks(), widths, rng))
        elapsed = 0.0
        for _ in range(args.steps):
            actions = sample_uniform_legal(orc.legal_masks(), widths, rng)
            t0 = time.perf_counter()
            orc.step(actions)
            orc.legal_masks()
            elapsed += time.perf_counter() - t0
        metric = METRIC
    value = lanes * args.steps / elapsed
    line = {
        "impl": "reference",
        "metric": metric, "value": value, "unit": "env-steps/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1000 * elapsed / args.steps, "higher_is_better": True,
        "scaling": scaling_of(config), "vs_baseline": None, "dtype": "int32", "data": "synthetic",
        "config": {"workload": workload_name(config), "lanes_per_step_sample": lanes, "full_lanes": args.lanes},
        "cpu_baseline": {"value": value, "unit": "env-steps/s", "cores": threads, "kind": "port",
                         "sample": f"{lanes} games per step on {threads} threads; the reference's JAX CPU path is not "
                                   "runnable here (jax absent, reference install failed), so its C++ restatement runs"},
        "e2e": {"value": value, "unit": "env-steps/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if not args.no_reference_kernels:
        try:
            import torch

            if torch.cuda.is_available():
                line["gpu_kernels"] = reference_gpu_kernels(config, args.lanes, steps=min(args.steps, 50), warmup=3,
                                                            soak=args.soak_steps)
        except Exception as error:  # noqa: BLE001 - the CPU figure stands alone then
            line["gpu_kernels"] = {"unavailable": f"{type(error).__name__}: {error}"}
    print(json.dumps(line))


# ---------------------------------------------------------------------------
# This implementation
# ---------------------------------------------------------------------------
class Run:
    """Per-rank context of a benchmark run."""

    def __init__(self, args, world: int, rank: int, local: int, device) -> None:
        self.args, self.world, self.rank, self.local, self.device = args, world, rank, local, device

    def barrier(self) -> None:
        if self.world > 1:
            import torch.distributed as dist

            dist.barrier()

    def max_over_ranks(self, values: list[float]) -> list[float]:
        import torch

        t = torch.tensor(values, dtype=torch.float64, device=self.device)
        if self.world > 1:
            import torch.distributed as dist

            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.tolist()

    def sum_over_ranks(self, values: list[float]) -> list[float]:
        import torch

        t = torch.tensor(values, dtype=torch.float64, device=self.device)
        if self.world > 1:
            import torch.distributed as dist

            dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return t.tolist()

    def check_device(self, what: str) -> None:
        """Fails the run when a kernel's bounded staging wait gave up: then some
        games were not stepped and no number of this run stands."""
        from nanorts_b200.runtime import check_device

        try:
            check_device(self.local)
        except Exception as error:
            raise SystemExit(f"rank {self.rank}: device status after {what}: {error}") from error


def timed_steps(run: Run, step, steps: int, soak_steps: int):
    """`soak_steps` untimed steps (the games reach mid-game; clocks settle under
    load and are sampled), then `steps` timed steps; CUDA events around each
    step and the whole region on the launching stream.  Returns (region ms,
    mean step ms, clock summary), the times as the max over ranks."""
    import torch

    stream = torch.cuda.current_stream(run.device)
    marks = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(run.local) as clocks:
        for i in range(soak_steps):
            step(-1 - i)
            if i % 64 == 63:
                torch.cuda.synchronize(run.device)
        run.barrier()
        torch.cuda.synchronize(run.device)
        start.record(stream)
        for k in range(steps):
            marks[k][0].record(stream)
            step(k)
            marks[k][1].record(stream)
        end.record(stream)
        torch.cuda.synchronize(run.device)
    region_ms = start.elapsed_time(end)
    step_ms = sum(a.elapsed_time(b) for a, b in marks) / steps
    region_ms, step_ms = run.max_over_ranks([region_ms, step_ms])
    return region_ms, step_ms, clocks.summary(f"{soak_steps} untimed steps right before the timed region, then "
                                              "the timed region")


def roofline(config: int, bytes_per: dict, games: int, step_ms: float, kernel: str) -> dict:
    peak, peak_kind = load_peaks()
    achieved = bytes_per["total"] * games / (step_ms * 1e-3) / 1e9
    traffic = load_traffic(config)
    out = {
        "bound": "hbm",
        "achieved": achieved,
        "peak": peak,
        "unit": "GB/s",
        "frac": achieved / peak,
        "traffic": traffic * games if traffic is not None else None,
        "traffic_unit": f"DRAM bytes per launch (ncu capture, profiles/{KERNELS[config][1]})" if traffic else None,
        "algorithmic_bytes_per_launch": bytes_per["total"] * games,
        "bytes_per_env_step": bytes_per["total"],
        "kernel": kernel,
        "kernel_ms": step_ms,
        "peak_kind": peak_kind,
    }
    if "total_without_draw" in bytes_per and bytes_per["total_without_draw"] != bytes_per["total"]:
        without = bytes_per["total_without_draw"] * games / (step_ms * 1e-3) / 1e9
        out["frac_without_draw"] = without / peak
        out["bytes_per_env_step_without_draw"] = bytes_per["total_without_draw"]
    return out


def measure_random(run: Run, config: int, lanes: int, steps: int, warmup: int, e2e_steps: int, stat_steps: int,
                   fused: bool, soak_steps: int) -> dict:
    """One uniform-random-play configuration (1, 2, 3 or 5) on this rank."""
    import torch

    from nanorts_b200.env import make
    from nanorts_b200.sharding import EpisodeStats, Shard, shard_keys

    game = scenario(config)
    partial, scaling = CONFIGS[config][3], CONFIGS[config][6]
    device, rank, world = run.device, run.rank, run.world
    env = make("NanoRTS", scenario=game, final_observation=False, device=device, partial_observability=partial)
    # Weak scaling: world * lanes games, each rank steps its contiguous block of
    # lanes; strong scaling (config 3): lanes games in all, split over the ranks.
    global_games = lanes if scaling == "strong" else world * lanes
    shard = Shard(rank, world, global_games)
    L = shard.lanes
    rng = np.random.default_rng(1234 + config)
    all_keys = torch.from_numpy(rng.integers(0, 2**32, size=(global_games, 2), dtype=np.uint64).astype(np.uint32).view(np.int32))
    _, state = env.reset(shard_keys(all_keys, shard).to(device).view(torch.uint32))
    current = {"actions": env.sample_actions(state, seed=rank, counter=0)}

    def one_step(counter: int):
        if fused:  # draw the next actions inside the step kernel
            out = env.step(None, state, current["actions"], sample=(rank, counter))
            current["actions"] = out[4]["sampled_actions"]
            return out
        actions = env.sample_actions(state, seed=rank, counter=counter)
        return env.step(None, state, actions)

    for i in range(warmup):
        one_step(i)
    torch.cuda.synchronize(device)
    region_ms, step_ms, clocks = timed_steps(run, lambda k: one_step(warmup + (k if k >= 0 else 10**8 - k)), steps,
                                             soak_steps)
    run.check_device(f"the timed steps of config {config}")

    episodes = None
    if stat_steps > 0:
        # Episode statistics over an untimed stretch in which every game ends at
        # least once (the horizon is MAX_CYCLES), reduced once over NCCL.
        stats = EpisodeStats(device)
        for i in range(stat_steps):
            _, _, rewards, dones, infos = one_step(10**9 + i)
            stats.add_step(dones["__all__"], infos["winner"], infos["telemetry"].spawn_overflow)
        episodes = stats.reduce()
        run.check_device(f"the episode stretch of config {config}")

    # End to end through the public API with host buffers: each step copies the
    # actions from pinned host memory, steps (drawing the next actions on the
    # device as the timed steps do) and writes the next actions, rewards and
    # dones back to pinned host memory, where the next step's actions are read
    # from.  The round trip is stream-ordered: no host synchronisation per step
    # (the host reads the rewards and dones of every step, from a ring of
    # per-step buffers, after the loop).  The rank's games run as E2E_SHARDS
    # environment states, each on its own stream, so that one shard's
    # host->device copy overlaps another's device->host copy and kernels (PCIe
    # moves both ways at once).  Pinned buffers sit on the GPU's NUMA node.
    C = game.bucket.per_player_capacity
    # Small batches (under 32 MB of actions per step) stay one state: there the
    # per-launch latency outweighs the copy overlap.
    K = run.args.e2e_shards if L % run.args.e2e_shards == 0 and L * C * 7 * 4 * 2 >= 32 << 20 else 1
    per = L // K
    e2e_keys = shard_keys(all_keys, shard).to(device).view(torch.uint32)
    streams = [torch.cuda.Stream(device) for _ in range(K)]
    shards = []
    with NodeLocal(run.local) as placement:
        for k in range(K):
            with torch.cuda.stream(streams[k]):
                _, st = env.reset(e2e_keys[k * per:(k + 1) * per].contiguous())
                first = env.sample_actions(st, seed=rank, counter=1)
                sh = {
                    "state": st,
                    "host": torch.empty((2, per, C, 7), dtype=torch.int32).pin_memory(),
                    "dev": torch.empty((2, per, C, 7), dtype=torch.int32, device=device),
                    "rewards": torch.empty((e2e_steps + 3, per, 2), dtype=torch.float32).pin_memory(),
                    "dones": torch.empty((e2e_steps + 3, per), dtype=torch.bool).pin_memory(),
                }
                sh["host"][0].copy_(first["player_0"])
                sh["host"][1].copy_(first["player_1"])
            shards.append(sh)
    torch.cuda.synchronize(device)

    def e2e_step(i: int) -> None:
        for k, sh in enumerate(shards):
            with torch.cuda.stream(streams[k]):
                sh["dev"].copy_(sh["host"], non_blocking=True)
                acts = {"player_0": sh["dev"][0], "player_1": sh["dev"][1]}
                if fused:
                    _, _, rewards, dones, infos = env.step(None, sh["state"], acts, sample=(rank, 2 * 10**9 + i))
                    nxt = infos["sampled_actions"]
                else:
                    _, _, rewards, dones, _ = env.step(None, sh["state"], acts)
                    nxt = env.sample_actions(sh["state"], seed=rank, counter=2 * 10**9 + i)
                sh["host"][0].copy_(nxt["player_0"], non_blocking=True)
                sh["host"][1].copy_(nxt["player_1"], non_blocking=True)
                sh["rewards"][i].copy_(torch.stack([rewards["player_0"], rewards["player_1"]], 1), non_blocking=True)
                sh["dones"][i].copy_(dones["__all__"], non_blocking=True)

    stream = torch.cuda.current_stream(device)
    e2e_steps_total = e2e_steps + 3
    for i in range(3):
        e2e_step(i)
    for s_k in streams:
        s_k.synchronize()
    run.barrier()
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for s_k in streams:
        s_k.wait_event(e0)
    for i in range(e2e_steps):
        e2e_step(3 + i)
    for s_k in streams:
        stream.wait_stream(s_k)
    e1.record(stream)
    torch.cuda.synchronize(device)
    (e2e_ms,) = run.max_over_ranks([e0.elapsed_time(e1)])
    run.check_device(f"the end-to-end steps of config {config}")
    ended_e2e = sum(int(sh["dones"][:e2e_steps_total].sum()) for sh in shards)  # the host reads every step's results

    bytes_per = algorithmic_bytes(game, fused)
    h2d = global_games * C * 7 * 4 * 2
    d2h = global_games * C * 7 * 4 * 2 + global_games * (2 * 4 + 1)
    e2e_value = global_games * e2e_steps / (e2e_ms * 1e-3)
    result = {
        "metric": METRIC,
        "value": global_games * steps / (region_ms * 1e-3),
        "unit": "env-steps/s",
        "ms_per_step": region_ms / steps,
        "steps": steps,
        "scaling": scaling,
        "config": {
            "workload": workload_name(config),
            "games_per_gpu": L,
            "global_games": global_games,
            "parallelism": f"dp{world} (independent games per GPU)",
            "step": "nrts_sample_actions + nrts_step" if not fused else
                    "nrts_step with the fused uniform draw of the next actions",
            "l2": "inputs larger than L2 (per-GPU working set "
                  f"{(bytes_per['total'] + 2 * C * 7 * 4) * L / 1e6:.0f} MB)" if L * bytes_per["total"] > 126e6 else
                  f"working set {bytes_per['total'] * L / 1e6:.0f} MB fits in L2: the step is one game's latency",
        },
        "roofline": roofline(config, bytes_per, L, step_ms, KERNELS[config][0]),
        "clocks": clocks,
        "e2e": {
            "value": e2e_value,
            "unit": "env-steps/s",
            "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h,
            "shards_per_gpu": K,
            "host_copy_gbs": (h2d + d2h) * e2e_steps / (e2e_ms * 1e-3) / 1e9,
            "loop": "stream-ordered host round trip of actions and results, no host synchronisation per step",
            "games_ended": ended_e2e,
            "pinned_buffers": "on the GPU's NUMA node" if placement.cpus else "default placement (NVML affinity unknown)",
        },
        "gpu_launches": (1 if fused else 2) * steps,
    }
    if L * bytes_per["total"] < 126e6:
        result["roofline"]["note"] = ("the working set fits in the 126 MB L2 and every game is resident at once: the "
                                      "launch lasts about one game's latency, so the HBM fraction is not its bound")
        result["roofline"]["game_latency_us"] = step_ms * 1e3
    if episodes is not None:
        result["episodes"] = episodes
        result["episode_steps"] = stat_steps
    return result


def measure_duel(run: Run, lanes: int, steps: int, warmup: int, e2e_steps: int, stat_steps: int, soak_steps: int) -> dict:
    """WorkerRush (player 0) against LightRush (player 1), one
    nrts_duel_step launch per step, every game from its reset and restarting
    when it ends.  The bots read no host input, so the end-to-end number times
    the same launches plus the per-step read-back of rewards, dones and winners."""
    import torch

    from nanorts_b200.bots import Bot, Duel
    from nanorts_b200.env import make
    from nanorts_b200.sharding import EpisodeStats, Shard, shard_keys

    device, rank, world = run.device, run.rank, run.world
    game = scenario(4)
    env = make("NanoRTS", scenario=game, final_observation=False, device=device)
    duel = Duel(env, tuple(Bot(f"player_{p}", s, t) for p, (s, t) in enumerate(DUEL_BOTS)))
    L = lanes
    shard = Shard(rank, world, world * L)
    rng = np.random.default_rng(1234)
    all_keys = torch.from_numpy(rng.integers(0, 2**32, size=(world * L, 2), dtype=np.uint64).astype(np.uint32).view(np.int32))
    ds = duel.reset(shard_keys(all_keys, shard).to(device).view(torch.uint32))
    stream = torch.cuda.current_stream(device)
    for _ in range(warmup):
        duel.step(ds)
    torch.cuda.synchronize(device)
    region_ms, kernel_ms, clocks = timed_steps(run, lambda k: duel.step(ds), steps, soak_steps)
    run.check_device("the timed duel steps")

    episodes = None
    if stat_steps > 0:
        stats = EpisodeStats(device)
        for _ in range(stat_steps):
            _, _, dones, infos = duel.step(ds)
            stats.add_step(dones["__all__"], infos["winner"], infos["telemetry"].spawn_overflow)
        episodes = stats.reduce()

    # End to end through the public API: each step launches the duel and reads
    # the rewards, dones and winners back into pinned host memory.
    with NodeLocal(run.local):
        host_rewards = torch.empty((L, 2), dtype=torch.float32).pin_memory()
        host_dones = torch.empty((L,), dtype=torch.bool).pin_memory()
        host_winner = torch.empty((L,), dtype=torch.int32).pin_memory()

    def e2e_step() -> None:
        _, rewards, dones, infos = duel.step(ds)
        host_rewards.copy_(torch.stack([rewards["player_0"], rewards["player_1"]], 1), non_blocking=True)
        host_dones.copy_(dones["__all__"], non_blocking=True)
        host_winner.copy_(infos["winner"], non_blocking=True)
        stream.synchronize()

    for _ in range(3):
        e2e_step()
    run.barrier()
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(e2e_steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize(device)
    (e2e_ms,) = run.max_over_ranks([e0.elapsed_time(e1)])
    run.check_device("the end-to-end duel steps")

    bytes_per = duel_algorithmic_bytes(game)
    line = roofline(4, bytes_per, L, kernel_ms, KERNELS[4][0])
    line["note"] = "latency-bound (serial A* walks, low occupancy); the HBM fraction is reported, not a target"
    result = {
        "metric": DUEL_METRIC,
        "value": world * L * steps / (region_ms * 1e-3),
        "unit": "env-steps/s",
        "ms_per_step": region_ms / steps,
        "steps": steps,
        "scaling": "weak",
        "config": {
            "workload": workload_name(4),
            "games_per_gpu": L,
            "global_games": world * L,
            "parallelism": f"dp{world} (independent games per GPU)",
            "step": "nrts_duel_step (both bots, core step, auto-reset of State and carries)",
            "l2": f"inputs larger than L2 (per-GPU working set {bytes_per['total'] * L / 2e6:.0f} MB read + written)",
        },
        "roofline": line,
        "clocks": clocks,
        "e2e": {
            "value": world * L * e2e_steps / (e2e_ms * 1e-3),
            "unit": "env-steps/s",
            "h2d_bytes_per_step": 0,
            "d2h_bytes_per_step": world * L * (2 * 4 + 1 + 4),
        },
        "gpu_launches": steps,
    }
    if episodes is not None:
        result["episodes"] = episodes
        result["episode_steps"] = stat_steps
    return result


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=2000)
    parser.add_argument("--warmup", type=int, default=20)
    parser.add_argument("--config", type=int, default=2, choices=(1, 2, 3, 4, 5),
                        help="BASELINE.json config number (1-based) of the headline; 4 is the bot duel")
    parser.add_argument("--workload", default=None, choices=("random", "duel"),
                        help="duel is --config 4 (kept for older command lines)")
    parser.add_argument("--lanes", type=int, default=None, help="games per GPU (config 3: in all)")
    parser.add_argument("--only", action="store_true", help="measure the headline configuration alone")
    parser.add_argument("--extra-steps", type=int, default=300, help="timed steps of each further configuration")
    parser.add_argument("--e2e-shards", type=int, default=E2E_SHARDS,
                        help="environment states (one stream each) the e2e loop splits a GPU's games into")
    parser.add_argument("--impl", default="nanorts_b200", choices=("nanorts_b200", "reference"))
    parser.add_argument("--e2e-steps", type=int, default=50)
    parser.add_argument("--stat-steps", type=int, default=None,
                        help=f"untimed steps whose episode statistics are reduced (default {MAX_CYCLES}: every game ends)")
    parser.add_argument("--soak-steps", type=int, default=None,
                        help="untimed steps before each timed region (default: the midpoint of the configured run)")
    parser.add_argument("--separate-sampler", action="store_true",
                        help="draw actions with nrts_sample_actions instead of inside nrts_step")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--no-reference-kernels", action="store_true",
                        help="reference arm: skip timing the reference's own kernels on the GPU")
    args = parser.parse_args()
    if args.warmup < 3:
        parser.error("--warmup must be at least 3")
    if args.workload == "duel":
        args.config = 4
    if args.lanes is None:
        args.lanes = default_lanes(args.config)
    if args.stat_steps is None:
        args.stat_steps = MAX_CYCLES
    if args.impl == "reference":
        run_reference(args)
        return

    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    run = Run(args, world, rank, local, device)
    fused = not args.separate_sampler

    def measure(config: int, lanes: int, steps: int, stat_steps: int, e2e_steps: int) -> dict:
        soak = MIDPOINT[config] if args.soak_steps is None else args.soak_steps
        if config == 4:
            return measure_duel(run, lanes, steps, args.warmup, e2e_steps, stat_steps, soak)
        return measure_random(run, config, lanes, steps, args.warmup, e2e_steps, stat_steps, fused, soak)

    head = measure(args.config, args.lanes, args.steps, args.stat_steps, args.e2e_steps)
    # Pinned copy bandwidth of every rank at once (the ceiling of the e2e loop).
    run.barrier()
    copy = pinned_copy_bandwidth(device)
    both, h2d, d2h = run.sum_over_ranks([copy["both"], copy["h2d"], copy["d2h"]])
    head["e2e"]["pinned_copy_gbs"] = {"both_directions": both, "h2d": h2d, "d2h": d2h,
                                      "how": "128 MB pinned buffers on the GPU's NUMA node, every rank at once, "
                                             "summed over ranks"}
    if "host_copy_gbs" in head["e2e"]:  # bytes all ranks copied per second in the e2e loop
        head["e2e"]["copy_frac"] = head["e2e"]["host_copy_gbs"] / both if both > 0 else None
        head["e2e"]["limiter"] = ("host copies (PCIe / host memory): the loop moves its action rows both ways "
                                  "every step")
    extras = {}
    if not args.only:
        for config in (1, 2, 3, 4, 5):
            if config == args.config:
                continue
            extras[f"config{config}"] = measure(config, default_lanes(config), args.extra_steps, 0,
                                                min(args.e2e_steps, 20))
    if rank == 0:
        line = {
            "metric": head["metric"],
            "value": head["value"],
            "unit": "env-steps/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": head["ms_per_step"],
            "higher_is_better": True,
            "scaling": head["scaling"],
            "vs_baseline": None,
            "dtype": "int32",
            "data": "synthetic",
            "config": head["config"],
            "roofline": head["roofline"],
            "clocks": head["clocks"],
            "e2e": head["e2e"],
            "gpu_launches": head["gpu_launches"],
        }
        if "episodes" in head:
            line["episodes"] = head["episodes"]
            line["episode_steps"] = head["episode_steps"]
        if not args.no_cpu_baseline and world == 1:
            if args.config == 4:
                line["cpu_baseline"] = duel_cpu_baseline(scenario(4))
            else:
                name, _, strategy = CONFIGS[args.config][:3]
                line["cpu_baseline"] = cpu_baseline(scenario(args.config), lanes=512 if args.config != 5 else 48,
                                                    partial=CONFIGS[args.config][3], label=f"{name}/{strategy}")
        if extras:
            line["configs"] = extras
        print(json.dumps(line))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
