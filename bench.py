"""Benchmark: NanoRTS env-steps/s on B200 (BASELINE.json metric).

Workload (configs[1] of BASELINE.json): basesWorkers16x16, VERSION_ORIGINAL,
CANCEL_RANDOM, 70 slots per player, symbolic uint8[16,16,6] observations,
16384 games per GPU, both players draw uniform random legal actions per
factor from the masks, auto-reset.  One step = sample actions from the
current masks (nrts_sample_actions) + one environment step of every game
(nrts_step: decode, core step, auto-reset, next masks, both observations).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--lanes L] [--impl reference]

``--workload duel`` measures BASELINE.json's configs[3] instead: bot against
bot on basesWorkers16x16 (VERSION_ORIGINAL, CANCEL_BOTH), player 0 WorkerRush,
player 1 LightRush, 32768 games per GPU from their reset, auto-reset at the end
of each game, no masks or observations.  One step = one nrts_duel_step launch
(both bots' Commands, the core step, the auto-reset of State and carries).

Under torchrun each rank steps its own L games (weak scaling, no collective
on the step path); one NCCL all-reduce of episode statistics runs after the
timed region.  Rank 0 prints one JSON line.
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
MAP, UTT, STRATEGY = "basesWorkers16x16", "VERSION_ORIGINAL", "CANCEL_RANDOM"
DUEL_STRATEGY = "CANCEL_BOTH"
DEFAULT_LANES = {"random": 16384, "duel": 32768}
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


def scenario(workload: str = "random", config: int = 2):
    from nanorts_b200 import map_name_to_scenario

    if workload == "duel":
        return map_name_to_scenario(MAP, utt=UTT, conflict_strategy=DUEL_STRATEGY, max_cycles=5000)
    name, utt, strategy, _, profile, _, _ = CONFIGS[config]
    return map_name_to_scenario(name, utt=utt, conflict_strategy=strategy, max_cycles=5000, capacity_profile=profile)


def workload_name(config: int) -> str:
    name, utt, strategy, partial, profile, _, _ = CONFIGS[config]
    obs = ", partial observability" if partial else ""
    cap = "" if profile else ", capacity_profile=False"
    return f"configs[{config - 1}]: {name} {utt} {strategy}{obs}{cap}, uniform random legal actions per factor, auto-reset"


def duel_algorithmic_bytes(game) -> dict[str, int]:
    """Bytes one bot-against-bot env-step must move: the State read and written
    in place, both players' carries (nine int32 fields, trained, next_order per
    slot block) read and written, and the step outputs."""
    b = game.bucket
    E, HW, C = b.entity_capacity, b.cell_count, b.per_player_capacity
    state = 35 * E + 2 * HW + 37 + 12
    carry = 37 * C + 4
    parts = {
        "state_read": state,
        "state_write": state,
        "carries_read": 2 * carry,
        "carries_write": 2 * carry,
        "outputs": 8 + 1 + 1 + 1 + 4 + 8,
    }
    parts["total"] = sum(parts.values())
    return parts


def algorithmic_bytes(game) -> dict[str, int]:
    """Bytes one env-step must move: the State read and written in place
    (reference layout, with the 12 lifecycle bytes), both players' action
    rows, legality rows, feature maps and scalars, and the step outputs."""
    b = game.bucket
    E, HW, C = b.entity_capacity, b.cell_count, b.per_player_capacity
    state = 35 * E + 2 * HW + 37 + 12
    parts = {
        "state_read": state,
        "state_write": state,
        "actions": 2 * C * 7 * 4,
        "masks": 2 * C * b.mask_width,
        "observations": 2 * (HW * 6 + 16),
        "outputs": 8 + 1 + 1 + 1 + 4 + 8,
    }
    parts["total"] = sum(parts.values())
    return parts


def load_peaks() -> tuple[float, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        return float(json.loads(path.read_text())["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# Environment states (each on its own stream) the end-to-end loop splits a
# GPU's games into.
E2E_SHARDS = 8

# The kernel each configuration's step launches on a B200 (148 SMs) and the
# committed ncu summary holding its DRAM bytes per env-step.
KERNELS = {
    1: ("nrts::step_kernel_wide<8> (2-warp CTAs)", None),
    2: ("nrts::step_kernel_big<16>", "step_kernel_16x16_traffic.txt"),
    3: ("nrts::step_kernel_big<16>", "step_kernel_16x16_partial_traffic.txt"),
    5: ("nrts::step_kernel_wide<64>", "step_kernel_64x64_traffic.txt"),
}


def load_traffic(workload: str = "random", config: int = 2) -> float | None:
    """DRAM bytes per env-step of the measured kernel from the committed ncu summary."""
    name = "duel_kernel_16x16_traffic.txt" if workload == "duel" else KERNELS[config][1]
    if name is None:
        return None
    path = ROOT / "profiles" / name
    if not path.exists():
        return None
    for line in path.read_text().splitlines():
        if line.startswith("dram_bytes_per_env_step:"):
            return float(line.split(":", 1)[1])
    return None


class ClockSampler:
    """Samples SM clocks and throttle reasons through NVML while running."""

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
            self._handle = pynvml.nvmlDeviceGetHandleByIndex(device_index)
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
            time.sleep(0.02)

    def __enter__(self):
        if self._nvml is not None:
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._nvml is not None:
            self._thread.join()

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        seen = 0
        for _, r in self.samples:
            seen |= r
        return {
            "sm_mhz": statistics.median(m for m, _ in self.samples),
            "sm_max_mhz": self.max_mhz,
            "reasons": sorted(name for name, bit in self.REASONS.items() if seen & bit),
            "samples": len(self.samples),
        }


def cpu_baseline(game, seconds: float = 12.0, lanes: int = 512, threads: int | None = None, partial: bool = False,
                 label: str = f"{MAP}/{STRATEGY}") -> dict:
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


def run_reference(args) -> None:
    """--impl reference: the reference's CPU path for this workload.  The reference
    (JAX) cannot be installed here, so this times the C++ oracle port of its JAX
    program on the host cores; each step is a bounded sample of the workload."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    if args.workload == "duel":
        game = scenario("duel")
        from oracle.oracle import Oracle, empty_carry

        threads = os.cpu_count() or 1
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
        value = lanes * args.steps / elapsed
        print(json.dumps({
            "impl": "reference",
            "metric": DUEL_METRIC, "value": value, "unit": "env-steps/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1000 * elapsed / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int32", "data": "synthetic",
            "config": {"workload": f"{MAP} {UTT} {DUEL_STRATEGY}, WorkerRush vs LightRush, auto-reset",
                       "lanes_per_step_sample": lanes, "full_lanes": args.lanes},
            "cpu_baseline": {"value": value, "unit": "env-steps/s", "cores": threads, "kind": "port",
                             "sample": f"{lanes} games per step on {threads} threads; the reference's JAX CPU path is "
                                       "not runnable here (jax absent, reference install failed), so its C++ "
                                       "restatement runs"},
            "e2e": {"value": value, "unit": "env-steps/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }))
        return
    game = scenario(config=args.config)
    partial = CONFIGS[args.config][3]
    from oracle.oracle import Oracle, sample_uniform_legal

    threads = os.cpu_count() or 1
    lanes = 256 if args.config != 5 else 32
    orc = Oracle(game, lanes, threads=threads, partial_observability=partial)
    rng = np.random.default_rng(0)
    orc.reset(rng.integers(0, 2**32, size=(lanes, 2), dtype=np.uint64).astype(np.uint32))
    widths = (6, 4, 4, 4, 4, game.bucket.unit_type_capacity, game.bucket.attack_offset_capacity)
    for _ in range(args.warmup):
        orc.step(sample_uniform_legal(orc.legal_masks(), widths, rng))
    elapsed = 0.0
    for _ in range(args.steps):
        masks = orc.legal_masks()
        actions = sample_uniform_legal(masks, widths, rng)
        t0 = time.perf_counter()
        orc.step(actions)
        orc.legal_masks()
        elapsed += time.perf_counter() - t0
    value = lanes * args.steps / elapsed
    line = {
        "impl": "reference",
        "metric": METRIC, "value": value, "unit": "env-steps/s", "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1000 * elapsed / args.steps, "higher_is_better": True,
        "scaling": CONFIGS[args.config][6],
        "vs_baseline": None, "dtype": "int32", "data": "synthetic",
        "config": {"workload": workload_name(args.config), "lanes_per_step_sample": lanes, "full_lanes": args.lanes},
        "cpu_baseline": {"value": value, "unit": "env-steps/s", "cores": threads, "kind": "port",
                         "sample": f"{lanes} games per step on {threads} threads; the reference's JAX CPU path is not "
                                   "runnable here (jax absent, reference install failed), so its C++ restatement runs"},
        "e2e": {"value": value, "unit": "env-steps/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=2000)
    parser.add_argument("--warmup", type=int, default=20)
    parser.add_argument("--workload", default="random", choices=("random", "duel"),
                        help="random: uniform legal actions (configs 1, 2, 3, 5); duel: configs[3] (WorkerRush vs LightRush)")
    parser.add_argument("--config", type=int, default=2, choices=(1, 2, 3, 4, 5),
                        help="BASELINE.json config number (1-based); 2 is the headline, 4 selects the duel")
    parser.add_argument("--lanes", type=int, default=None, help="games per GPU")
    parser.add_argument("--e2e-shards", type=int, default=E2E_SHARDS,
                        help="environment states (one stream each) the e2e loop splits a GPU's games into")
    parser.add_argument("--impl", default="nanorts_b200", choices=("nanorts_b200", "reference"))
    parser.add_argument("--e2e-steps", type=int, default=50)
    parser.add_argument("--stat-steps", type=int, default=None,
                        help="untimed steps whose episode statistics are reduced (default 200; duel 600, about one game)")
    parser.add_argument("--separate-sampler", action="store_true",
                        help="draw actions with nrts_sample_actions instead of inside nrts_step")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    args = parser.parse_args()
    if args.warmup < 3:
        parser.error("--warmup must be at least 3")
    if args.config == 4:
        args.workload = "duel"
    if args.lanes is None:
        args.lanes = DEFAULT_LANES["duel"] if args.workload == "duel" else CONFIGS[args.config][5]
    if args.stat_steps is None:
        args.stat_steps = 600 if args.workload == "duel" else 200
    if args.impl == "reference":
        run_reference(args)
        return

    import torch
    import torch.distributed as dist

    from nanorts_b200.env import make

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)

    from nanorts_b200.sharding import EpisodeStats, Shard, shard_keys

    if args.workload == "duel":
        run_duel(args, world, rank, local, device)
        return
    game = scenario(config=args.config)
    partial, scaling = CONFIGS[args.config][3], CONFIGS[args.config][6]
    env = make("NanoRTS", scenario=game, final_observation=False, device=device, partial_observability=partial)
    # Weak scaling: world * lanes games, each rank steps its contiguous block of
    # lanes; strong scaling (config 3): lanes games in all, split over the ranks.
    global_games = args.lanes if scaling == "strong" else world * args.lanes
    shard = Shard(rank, world, global_games)
    L = shard.lanes
    rng = np.random.default_rng(1234)
    all_keys = torch.from_numpy(rng.integers(0, 2**32, size=(global_games, 2), dtype=np.uint64).astype(np.uint32).view(np.int32))
    _, state = env.reset(shard_keys(all_keys, shard).to(device).view(torch.uint32))
    stream = torch.cuda.current_stream(device)

    fused = not args.separate_sampler
    current = {"actions": env.sample_actions(state, seed=rank, counter=0)}

    def one_step(counter: int):
        if fused:  # draw the next actions inside the step kernel
            out = env.step(None, state, current["actions"], sample=(rank, counter))
            current["actions"] = out[4]["sampled_actions"]
            return out
        actions = env.sample_actions(state, seed=rank, counter=counter)
        return env.step(None, state, actions)

    for i in range(args.warmup):
        one_step(i)
    torch.cuda.synchronize(device)

    # Timed region: K steps, events around every step kernel for the roofline.
    step_events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(device)
    with ClockSampler(local) as clocks:
        start.record(stream)
        for i in range(args.steps):
            if fused:
                step_events[i][0].record(stream)
                out = env.step(None, state, current["actions"], sample=(rank, args.warmup + i))
                current["actions"] = out[4]["sampled_actions"]
                step_events[i][1].record(stream)
            else:
                actions = env.sample_actions(state, seed=rank, counter=args.warmup + i)
                step_events[i][0].record(stream)
                env.step(None, state, actions)
                step_events[i][1].record(stream)
        end.record(stream)
        torch.cuda.synchronize(device)
    elapsed_ms = start.elapsed_time(end)
    step_kernel_ms = sum(a.elapsed_time(b) for a, b in step_events) / args.steps

    # Episode statistics over a further untimed stretch, reduced once over NCCL.
    stats = EpisodeStats(device)
    for i in range(args.stat_steps):
        _, _, rewards, dones, infos = one_step(10**9 + i)
        stats.add_step(dones["__all__"], infos["winner"], infos["telemetry"].spawn_overflow)
    episode_stats = stats.reduce()
    timing = torch.tensor([elapsed_ms, step_kernel_ms], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(timing, op=dist.ReduceOp.MAX)
    elapsed_ms, step_kernel_ms = timing.tolist()

    # End to end through the public API with host buffers: each step copies the
    # actions from pinned host memory, steps (drawing the next actions on the
    # device as the timed steps do) and reads the next actions, rewards and
    # dones back to the host.  The rank's games run as E2E_SHARDS environment
    # states, each on its own stream, so that one shard's host->device copy
    # overlaps another's device->host copy (PCIe moves both ways at once).
    C = game.bucket.per_player_capacity
    # Small batches (under 32 MB of actions per step) stay one state: there the
    # per-launch latency outweighs the copy overlap.
    K = args.e2e_shards if L % args.e2e_shards == 0 and L * C * 7 * 4 * 2 >= 32 << 20 else 1
    per = L // K
    e2e_keys = shard_keys(all_keys, shard).to(device).view(torch.uint32)
    streams = [torch.cuda.Stream(device) for _ in range(K)]
    shards = []
    for k in range(K):
        with torch.cuda.stream(streams[k]):
            _, st = env.reset(e2e_keys[k * per:(k + 1) * per].contiguous())
            first = env.sample_actions(st, seed=rank, counter=1)
            sh = {
                "state": st,
                "host": torch.empty((2, per, C, 7), dtype=torch.int32).pin_memory(),
                "dev": torch.empty((2, per, C, 7), dtype=torch.int32, device=device),
                "rewards": torch.empty((per, 2), dtype=torch.float32).pin_memory(),
                "dones": torch.empty((per,), dtype=torch.bool).pin_memory(),
            }
            sh["host"][0].copy_(first["player_0"])
            sh["host"][1].copy_(first["player_1"])
        shards.append(sh)
    torch.cuda.synchronize(device)
    e2e_steps = args.e2e_steps

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
                sh["rewards"].copy_(torch.stack([rewards["player_0"], rewards["player_1"]], 1), non_blocking=True)
                sh["dones"].copy_(dones["__all__"], non_blocking=True)
        for s_k in streams:
            s_k.synchronize()

    for i in range(3):
        e2e_step(i)
    if world > 1:
        dist.barrier()
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
    e2e_ms = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
    e2e_ms = float(e2e_ms.item())

    bytes_per = algorithmic_bytes(game)
    if fused:  # the step kernel also writes the drawn actions of the next step
        bytes_per["sampled_actions"] = 2 * C * 7 * 4
        bytes_per["total"] += bytes_per["sampled_actions"]
    peak, peak_kind = load_peaks()
    achieved = bytes_per["total"] * L / (step_kernel_ms * 1e-3) / 1e9
    traffic = load_traffic("random", args.config)
    if traffic is not None:  # ncu DRAM bytes per env-step -> per launch of L games
        traffic *= L
    line = None
    if rank == 0:
        value = global_games * args.steps / (elapsed_ms * 1e-3)
        line = {
            "metric": METRIC,
            "value": value,
            "unit": "env-steps/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": elapsed_ms / args.steps,
            "higher_is_better": True,
            "scaling": scaling,
            "vs_baseline": None,
            "dtype": "int32",
            "data": "synthetic",
            "config": {
                "workload": workload_name(args.config),
                "games_per_gpu": L,
                "global_games": global_games,
                "parallelism": f"dp{world} (independent games per GPU)",
                "step": "nrts_sample_actions + nrts_step" if not fused else
                        "nrts_step with the fused uniform draw of the next actions",
                "l2": "inputs larger than L2 (per-GPU working set "
                      f"{(bytes_per['total'] + 2 * C * 7 * 4) * L / 1e6:.0f} MB)",
            },
            "roofline": {
                "bound": "hbm",
                "achieved": achieved,
                "peak": peak,
                "unit": "GB/s",
                "frac": achieved / peak,
                "traffic": traffic,
                "traffic_unit": f"DRAM bytes per launch (ncu capture, profiles/{KERNELS[args.config][1]})",
                "algorithmic_bytes_per_launch": bytes_per["total"] * L,
                "kernel": KERNELS[args.config][0],
                "kernel_ms": step_kernel_ms,
                "bytes_per_env_step": bytes_per["total"],
                "peak_kind": peak_kind,
            },
            "clocks": clocks.summary(),
            "e2e": {
                "value": global_games * e2e_steps / (e2e_ms * 1e-3),
                "unit": "env-steps/s",
                "h2d_bytes_per_step": global_games * C * 7 * 4 * 2,
                "d2h_bytes_per_step": global_games * C * 7 * 4 * 2 + global_games * (2 * 4 + 1),
                "shards_per_gpu": K,
            },
            "gpu_launches": (1 if fused else 2) * args.steps,
            "episodes": episode_stats,
        }
        if not args.no_cpu_baseline and world == 1:
            name, _, strategy = CONFIGS[args.config][:3]
            line["cpu_baseline"] = cpu_baseline(game, lanes=512 if args.config != 5 else 48, partial=partial,
                                                label=f"{name}/{strategy}")
        print(json.dumps(line))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_duel(args, world: int, rank: int, local: int, device) -> None:
    """WorkerRush (player 0) against LightRush (player 1), one
    nrts_duel_step launch per step, every game from its reset and restarting
    when it ends.  The bots read no host input, so the end-to-end number times
    the same launches plus the per-step read-back of rewards, dones and winners."""
    import torch
    import torch.distributed as dist

    from nanorts_b200.bots import Bot, Duel
    from nanorts_b200.env import make
    from nanorts_b200.sharding import EpisodeStats, Shard, shard_keys

    game = scenario("duel")
    env = make("NanoRTS", scenario=game, final_observation=False, device=device)
    duel = Duel(env, tuple(Bot(f"player_{p}", s, t) for p, (s, t) in enumerate(DUEL_BOTS)))
    L = args.lanes
    shard = Shard(rank, world, world * L)
    rng = np.random.default_rng(1234)
    all_keys = torch.from_numpy(rng.integers(0, 2**32, size=(world * L, 2), dtype=np.uint64).astype(np.uint32).view(np.int32))
    ds = duel.reset(shard_keys(all_keys, shard).to(device).view(torch.uint32))
    stream = torch.cuda.current_stream(device)
    for _ in range(args.warmup):
        duel.step(ds)
    torch.cuda.synchronize(device)
    step_events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(device)
    with ClockSampler(local) as clocks:
        start.record(stream)
        for i in range(args.steps):
            step_events[i][0].record(stream)
            duel.step(ds)
            step_events[i][1].record(stream)
        end.record(stream)
        torch.cuda.synchronize(device)
    elapsed_ms = start.elapsed_time(end)
    kernel_ms = sum(a.elapsed_time(b) for a, b in step_events) / args.steps

    stats = EpisodeStats(device)
    for _ in range(args.stat_steps):
        _, _, dones, infos = duel.step(ds)
        stats.add_step(dones["__all__"], infos["winner"], infos["telemetry"].spawn_overflow)
    episode_stats = stats.reduce()
    timing = torch.tensor([elapsed_ms, kernel_ms], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(timing, op=dist.ReduceOp.MAX)
    elapsed_ms, kernel_ms = timing.tolist()

    # End to end through the public API: each step launches the duel and reads
    # the rewards, dones and winners back into pinned host memory.
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
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.e2e_steps):
        e2e_step()
    e1.record(stream)
    torch.cuda.synchronize(device)
    e2e_ms = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(e2e_ms, op=dist.ReduceOp.MAX)
    e2e_ms = max(float(e2e_ms.item()), 1e-9)

    bytes_per = duel_algorithmic_bytes(game)
    peak, peak_kind = load_peaks()
    achieved = bytes_per["total"] * L / (kernel_ms * 1e-3) / 1e9
    traffic = load_traffic("duel")
    if traffic is not None:
        traffic *= L
    if rank == 0:
        line = {
            "metric": DUEL_METRIC,
            "value": world * L * args.steps / (elapsed_ms * 1e-3),
            "unit": "env-steps/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": elapsed_ms / args.steps,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "int32",
            "data": "synthetic",
            "config": {
                "workload": f"{MAP} {UTT} {DUEL_STRATEGY}, player_0 WorkerRush vs player_1 LightRush, "
                            "every game from its reset, auto-reset, max_cycles 5000",
                "games_per_gpu": L,
                "global_games": world * L,
                "parallelism": f"dp{world} (independent games per GPU)",
                "step": "nrts_duel_step (both bots, core step, auto-reset of State and carries)",
                "l2": f"inputs larger than L2 (per-GPU working set {bytes_per['total'] * L / 2e6:.0f} MB read + written)",
            },
            "roofline": {
                "bound": "hbm",
                "achieved": achieved,
                "peak": peak,
                "unit": "GB/s",
                "frac": achieved / peak,
                "traffic": traffic,
                "traffic_unit": "DRAM bytes per launch (ncu capture, profiles/duel_kernel_16x16.md)",
                "algorithmic_bytes_per_launch": bytes_per["total"] * L,
                "kernel": "nrts::duel_kernel",
                "kernel_ms": kernel_ms,
                "bytes_per_env_step": bytes_per["total"],
                "peak_kind": peak_kind,
                "note": "latency-bound (serial A* walks, low occupancy); the HBM fraction is reported, not a target",
            },
            "clocks": clocks.summary(),
            "e2e": {
                "value": world * L * args.e2e_steps / (e2e_ms * 1e-3),
                "unit": "env-steps/s",
                "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": world * L * (2 * 4 + 1 + 4),
            },
            "gpu_launches": args.steps,
            "episodes": episode_stats,
        }
        if not args.no_cpu_baseline and world == 1:
            line["cpu_baseline"] = duel_cpu_baseline(game)
        print(json.dumps(line))
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
