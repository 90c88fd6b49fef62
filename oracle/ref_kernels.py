"""The reference's own CUDA kernels, called through oracle/ref_kernels.cu (TEST INFRASTRUCTURE ONLY).

``make -C oracle ref`` (run by ``oracle.build()`` where a NanoRTS checkout is
found) compiles NanoRTS's ``nanorts_step``, ``nanorts_legality``,
``nanorts_legality_words``, ``nanorts_visible_cells``,
``nanorts_reset_packed_where_done`` and ``nanorts_abstraction_act`` handlers
unchanged into
``oracle/_ref/libref_kernels.so``.  This module hands them torch CUDA tensors
laid out as the reference's lane-major operands (``kernels/batching.py:64-88``:
``[L, ...]`` per leaf, a leading 1 for a row every lane shares), so the tests
can compare the product and the oracle with the reference itself.  Only tests/
and bench.py's reference arm use it.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np
import torch

from nanorts_b200.model import STRATEGY_CODES, UNIT_COLUMNS, GameConfig

HERE = Path(__file__).resolve().parent
LIBRARY = HERE / "_ref" / "libref_kernels.so"

# Element type codes of the stand-in DataType (ffi_standin/xla/ffi/api/ffi.h).
_CODES = {torch.bool: 1, torch.int8: 2, torch.int16: 3, torch.int32: 4, torch.uint8: 6}
U32 = 8

# State leaves in the reference's Leaf order (core/cuda/step.cu:61-85).
LEAVES = (
    "birth", "unit_type", "owner", "cell", "hit_points", "carried_resources", "pending_kind", "pending_direction",
    "pending_none_duration", "pending_target_cell", "pending_produced_type", "pending_issued_at",
    "pending_completes_at", "pending_order", "entity_at", "time", "player_resources", "next_birth",
    "next_pending_order", "alternating_conflict_count", "game_over", "winner", "spawn_overflow",
)
ROWS = LEAVES[:15]  # per-slot leaves and entity_at: aliased in place by nanorts_step and the reset
COUNTERS = LEAVES[15:]

# core/unit_tables.py:9-27: the reference kernels' table and timing columns.
TABLE_COLUMNS = ("can_move", "can_harvest", "is_resource", "is_stockpile", "can_attack", "attack_range", "cost")
TIMING_COLUMNS = ("move_time", "harvest_time", "attack_time", "produce_time", "hit_points", "attack_damage",
                  "harvest_amount")
# bots/whole_act.py:22-42: the State leaves and unit-table columns the bots read.
BOT_LEAVES = ("birth", "unit_type", "owner", "cell", "carried_resources", "pending_kind", "pending_direction",
              "pending_produced_type", "entity_at", "player_resources")
BOT_TABLE_COLUMNS = ("can_harvest", "is_resource", "is_stockpile", "can_attack", "attack_range", "cost")
# bots/abstraction.py:71-82: the carry's int32 rows, then trained and next_order.
CARRY_FIELDS = ("kind", "unit_birth", "order", "target", "target_birth", "base", "base_birth", "cell", "unit_type")
# core/cycle.py:59-77: event record columns.
INT32_COLUMNS, INDEX_COLUMNS, INT8_COLUMNS = 6, 4, 6
TARGET_OWNERS = 3


class RefBuffer(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("dtype", ctypes.c_int32), ("rank", ctypes.c_int32),
                ("dims", ctypes.c_int64 * 6)]


def available() -> bool:
    return LIBRARY.exists()


_LIB: ctypes.CDLL | None = None


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        if not LIBRARY.exists():
            raise FileNotFoundError(f"{LIBRARY} is not built (make -C oracle ref with NANORTS_REFERENCE set)")
        ref = ctypes.CDLL(str(LIBRARY))
        p, i64 = ctypes.c_void_p, ctypes.c_int64
        ref.ref_step.argtypes = [p, p, i64, p, i64, i64]
        ref.ref_legality_words.argtypes = [p, p, p, i64]
        ref.ref_legality_rows.argtypes = [p, p, p]
        ref.ref_visible_cells.argtypes = [p, p, p, i64, i64, i64, i64]
        ref.ref_reset_packed_where_done.argtypes = [p, p, p, p, p, i64]
        ref.ref_abstraction_act.argtypes = [p, p, i64, p, i64, i64, i64]
        for name in ("ref_step", "ref_legality_words", "ref_legality_rows", "ref_visible_cells",
                     "ref_reset_packed_where_done", "ref_abstraction_act"):
            getattr(ref, name).restype = ctypes.c_int
        ref.ref_last_error.restype = ctypes.c_char_p
        _LIB = ref
    return _LIB


def describe(t: torch.Tensor, code: int | None = None) -> RefBuffer:
    assert t.is_contiguous() and t.dim() <= 6
    b = RefBuffer(data=t.data_ptr(), dtype=_CODES[t.dtype] if code is None else code, rank=t.dim())
    for k, n in enumerate(t.shape):
        b.dims[k] = n
    return b


def _array(buffers: list[RefBuffer]):
    return (RefBuffer * len(buffers))(*buffers)


def _check(rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"{what}: {lib().ref_last_error().decode()}")


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


class ReferenceKernels:
    """The reference's kernels for one scenario on the current CUDA device."""

    def __init__(self, game: GameConfig, device: str | torch.device = "cuda") -> None:
        self.game, b = game, game.bucket
        self.bucket, self.device = b, torch.device(device)
        table = game.table
        col = {name: UNIT_COLUMNS.index(name) for name in UNIT_COLUMNS}
        T = b.unit_type_capacity
        ref_table = np.concatenate([table[:, [col[c] for c in TABLE_COLUMNS]], table[:, len(UNIT_COLUMNS):]], axis=1)
        timings = table[:, [col[c] for c in TIMING_COLUMNS]]
        dev = self.device
        self.terrain = torch.from_numpy(np.ascontiguousarray(game.terrain, bool)).reshape(1, b.height, b.width).to(dev)
        self.table = torch.from_numpy(np.ascontiguousarray(ref_table, np.int32)).reshape(1, T, 7 + T).to(dev)
        self.timings = torch.from_numpy(np.ascontiguousarray(timings, np.int32)).reshape(1, T, 7).to(dev)
        self.radius = torch.from_numpy(np.ascontiguousarray(table[:, col["sight_radius"]], np.int32)).reshape(1, T).to(dev)
        bot_table = table[:, [col[c] for c in BOT_TABLE_COLUMNS]]
        self.bot_table = torch.from_numpy(np.ascontiguousarray(bot_table, np.int32)).reshape(1, T, 6).to(dev)
        self.strategy = STRATEGY_CODES[b.conflict_strategy]

    # -- nanorts_step ---------------------------------------------------------------------------------------
    def event_buffers(self, lanes: int) -> list[torch.Tensor]:
        """The step's 8 event results (core/cycle.py:260-270)."""
        b, dev = self.bucket, self.device
        E, T = b.entity_capacity, b.unit_type_capacity
        i32 = dict(dtype=torch.int32, device=dev)
        return [
            torch.empty((lanes, 2), **i32), torch.empty((lanes, 2), **i32), torch.empty((lanes, 2, T), **i32),
            torch.empty((lanes, 2, TARGET_OWNERS), **i32), torch.empty((lanes, E), dtype=torch.bool, device=dev),
            torch.empty((lanes, E, INT32_COLUMNS), **i32), torch.empty((lanes, E, INDEX_COLUMNS), dtype=torch.int16, device=dev),
            torch.empty((lanes, E, INT8_COLUMNS), dtype=torch.int8, device=dev),
        ]

    def step(self, leaves: dict[str, torch.Tensor], counters_out: dict[str, torch.Tensor], commands: list[torch.Tensor],
             keys: torch.Tensor, events: list[torch.Tensor]) -> None:
        """``nanorts_step`` on L games.

        ``leaves``: the 23 State leaves (the row leaves are updated in place);
        ``counters_out``: result tensors for the 8 counter leaves (time ...
        spawn_overflow); ``commands``: the six Commands rows, int32 [L, 2, C]
        each; ``keys``: int32 view of the uint32 [L, 2] random roots.
        """
        operands = [describe(keys, U32), *(describe(c) for c in commands), describe(self.terrain), describe(self.table),
                    describe(self.timings), *(describe(leaves[name]) for name in LEAVES)]
        results = [*(describe(leaves[name]) for name in ROWS), *(describe(counters_out[name]) for name in COUNTERS),
                   *(describe(e) for e in events)]
        _check(lib().ref_step(_stream(), _array(operands), len(operands), _array(results), len(results), self.strategy),
               "nanorts_step")

    # -- legality -------------------------------------------------------------------------------------------
    def _legality_operands(self, leaves: dict[str, torch.Tensor]):
        names = ("birth", "unit_type", "owner", "carried_resources", "cell", "entity_at", "player_resources")
        return _array([*(describe(leaves[n]) for n in names), describe(self.terrain), describe(self.table)])

    def legality_words(self, leaves: dict[str, torch.Tensor], words: torch.Tensor) -> None:
        """``nanorts_legality_words``: uint32 [L, 2, C, 3] (given as int32)."""
        _check(lib().ref_legality_words(_stream(), self._legality_operands(leaves), ctypes.byref(describe(words, U32)),
                                        self.bucket.attack_offset_capacity), "nanorts_legality_words")

    def legality_rows(self, leaves: dict[str, torch.Tensor], rows: torch.Tensor) -> None:
        """``nanorts_legality``: bool [L, 2, C, 22 + T + O]."""
        _check(lib().ref_legality_rows(_stream(), self._legality_operands(leaves), ctypes.byref(describe(rows))),
               "nanorts_legality")

    def avail_rows(self, leaves: dict[str, torch.Tensor]) -> torch.Tensor:
        """``legal_actions`` (adapters/jaxmarl/actions.py:28-41) from the words
        kernel, as the reference's CUDA path assembles it: unpack the words
        (core/legality.py:148-151), AND ``available`` (legality.py:169-170),
        rows not available keep only the KIND_NONE bit.  bool [L, 2, C, 78]."""
        b = self.bucket
        L, C, N = leaves["birth"].shape[0], b.per_player_capacity, b.neutral_capacity
        words = torch.empty((L, 2, C, 3), dtype=torch.int32, device=self.device)
        self.legality_words(leaves, words)
        shifts = torch.arange(32, device=self.device, dtype=torch.int64)
        bits = ((words.to(torch.int64) & 0xFFFFFFFF)[..., None] >> shifts) & 1
        rows = bits.reshape(L, 2, C, 96)[..., : b.mask_width] != 0
        owned_birth = leaves["birth"][:, N:].reshape(L, 2, C)
        owned_pending = leaves["pending_kind"][:, N:].reshape(L, 2, C)
        avail = (owned_birth != -1) & (owned_pending == -1)
        idle = torch.zeros(b.mask_width, dtype=torch.bool, device=self.device)
        idle[0] = True
        return (rows & avail[..., None]) | (~avail[..., None] & idle)

    # -- visibility -----------------------------------------------------------------------------------------
    def visible_cells(self, leaves: dict[str, torch.Tensor], player: int, out: torch.Tensor) -> None:
        """``nanorts_visible_cells`` for ``player``'s slot block: bool [L, H, W]."""
        b = self.bucket
        operands = _array([describe(leaves["birth"]), describe(leaves["unit_type"]), describe(leaves["cell"]),
                           describe(self.radius)])
        first = b.neutral_capacity + player * b.per_player_capacity
        _check(lib().ref_visible_cells(_stream(), operands, ctypes.byref(describe(out)), first, b.per_player_capacity,
                                       b.width, b.height), "nanorts_visible_cells")

    # -- auto-reset -----------------------------------------------------------------------------------------
    def packed_reset_rows(self, reset: dict[str, np.ndarray]) -> torch.Tensor:
        """One shared uint8 row of the reset State's row leaves, each at the
        next 16-byte offset (adapters/lifecycle.py:126-137)."""
        parts = []
        for name in ROWS:
            data = np.ascontiguousarray(reset[name]).reshape(-1).view(np.uint8)
            parts.append(np.pad(data, (0, -data.size % 16)))
        return torch.from_numpy(np.concatenate(parts)).reshape(1, -1).to(self.device)

    def reset_where_done(self, done: torch.Tensor, packed: torch.Tensor, leaves: dict[str, torch.Tensor]) -> None:
        """``nanorts_reset_packed_where_done`` in place on the row leaves."""
        rows = _array([describe(leaves[name]) for name in ROWS])
        _check(lib().ref_reset_packed_where_done(_stream(), ctypes.byref(describe(done)), ctypes.byref(describe(packed)),
                                                 rows, rows, len(ROWS)), "nanorts_reset_packed_where_done")

    # -- rush bots ------------------------------------------------------------------------------------------
    def bot_act(self, leaves: dict[str, torch.Tensor], player: int, strategy: int, trained: int,
                carry: dict[str, torch.Tensor]) -> torch.Tensor:
        """``nanorts_abstraction_act`` for one player's rush bot: updates the
        carry (CARRY_FIELDS int32 [L, C], ``trained`` 0/1 uint8 [L, C],
        ``next_order`` int32 [L]) in place, returns Commands int32 [L, 6, 2, C]."""
        b = self.bucket
        L = leaves["birth"].shape[0]
        who = torch.tensor([player], dtype=torch.int32, device=self.device)
        carried = [*(describe(carry[n]) for n in CARRY_FIELDS), describe(carry["trained"], _CODES[torch.bool]),
                   describe(carry["next_order"])]
        operands = [*(describe(leaves[n]) for n in BOT_LEAVES), describe(self.terrain), describe(self.bot_table),
                    describe(who), *carried]
        commands = torch.empty((L, 6, 2, b.per_player_capacity), dtype=torch.int32, device=self.device)
        results = [*carried, describe(commands)]
        _check(lib().ref_abstraction_act(_stream(), _array(operands), len(operands), _array(results), len(results),
                                         strategy, trained), "nanorts_abstraction_act")
        return commands


def sample_uniform(rows: torch.Tensor, widths: tuple[int, ...], generator: torch.Generator | None = None) -> torch.Tensor:
    """One legal value per factor, uniform over the factor's set bits (0 when
    none): bool [..., 78] rows -> int32 [..., 7].  The torch form of the
    oracle's ``sample_uniform_legal``: the stand-in for the reference
    benchmark's per-factor ``jax.random.categorical`` over masked logits."""
    out = []
    start = 0
    for width in widths:
        group = rows[..., start:start + width]
        count = group.sum(-1)
        u = torch.rand(count.shape, device=rows.device, generator=generator)
        pick = torch.floor(u * count.clamp(min=1)).to(torch.int64)
        chosen = torch.argmax((group.cumsum(-1) > pick[..., None]).to(torch.int8), -1)
        out.append(torch.where(count > 0, chosen, torch.zeros_like(chosen)))
        start += width
    return torch.stack(out, -1).to(torch.int32)


def decode_actions(leaves: dict[str, torch.Tensor], actions: torch.Tensor, bucket) -> list[torch.Tensor]:
    """``decode_actions`` (adapters/jaxmarl/actions.py:61-84, factors.py:117-151)
    in torch: int32 [L, 2, C, 7] rows -> the six Commands rows int32 [L, 2, C]
    (kind, direction, none_duration, target_cell, produced_type, request_order).
    This is the XLA fusion the reference runs before ``nanorts_step``."""
    L = actions.shape[0]
    N, C, W, H = bucket.neutral_capacity, bucket.per_player_capacity, bucket.width, bucket.height
    side = int(round(bucket.attack_offset_capacity ** 0.5))
    radius = (side - 1) // 2
    birth = leaves["birth"][:, N:].reshape(L, 2, C)
    pending = leaves["pending_kind"][:, N:].reshape(L, 2, C)
    cell = leaves["cell"][:, N:].reshape(L, 2, C).to(torch.int32)
    available = (birth != -1) & (pending == -1)
    a = actions.to(torch.int32)
    kind = torch.where(available, a[..., 0], -1)
    by_kind = torch.gather(a[..., :5], -1, kind.clamp(0, 4).to(torch.int64)[..., None])[..., 0]
    direction = torch.where((kind >= 1) & (kind <= 4), by_kind, -1)
    produced = torch.where(kind == 4, a[..., 5], -1)
    offset = a[..., 6]
    tx = torch.remainder(cell, W) + (torch.remainder(offset, side) - radius)
    ty = torch.div(cell, W, rounding_mode="floor") + (torch.div(offset, side, rounding_mode="floor") - radius)
    on_board = (tx >= 0) & (tx < W) & (ty >= 0) & (ty < H)
    target = torch.where((kind == 5) & on_board, ty * W + tx, -1)
    none_duration = torch.where(kind == 0, 1, 0).to(torch.int32)
    order = torch.full_like(kind, -1)
    return [t.to(torch.int32).contiguous() for t in (kind, direction, none_duration, target, produced, order)]


class ReferencePath:
    """The reference's CUDA path for ``NanoRTS.step`` + ``get_avail_actions``
    on L games: its kernels ``nanorts_step``, ``nanorts_reset_packed_where_done``,
    ``nanorts_legality_words`` and (partial observability) two
    ``nanorts_visible_cells`` per step, with torch standing in for the XLA
    fusions between them (action sampling, ``decode_actions``, the lifecycle's
    select of the counter leaves, mask assembly).  Only the reference kernels
    are timed; the feature maps (an XLA fusion in the reference) are not
    computed, which favours the reference."""

    def __init__(self, game: GameConfig, lanes: int, *, partial: bool = False, seed: int = 0,
                 device: str | torch.device = "cuda") -> None:
        from nanorts_b200.content import decide

        self.ref = ReferenceKernels(game, device)
        self.game, self.lanes, self.partial, self.device = game, lanes, partial, torch.device(device)
        b = game.bucket
        reset = decide(game.initial_state, b)
        self.packed = self.ref.packed_reset_rows(reset)
        self.reset_rows = {n: torch.from_numpy(np.ascontiguousarray(reset[n])).to(self.device) for n in LEAVES}
        self.leaves = {n: v.expand(lanes, *v.shape).contiguous() for n, v in self.reset_rows.items()}
        self.counters = {n: torch.empty_like(self.leaves[n]) for n in COUNTERS}
        self.events = self.ref.event_buffers(lanes)
        self.generator = torch.Generator(device=self.device)
        self.generator.manual_seed(seed)
        self.keys = torch.randint(-2**31, 2**31 - 1, (lanes, 2), dtype=torch.int32, device=self.device,
                                  generator=self.generator)
        self.widths = (6, 4, 4, 4, 4, b.unit_type_capacity, b.attack_offset_capacity)
        self.words = torch.empty((lanes, 2, b.per_player_capacity, 3), dtype=torch.int32, device=self.device)
        self.seen = torch.empty((lanes, b.height, b.width), dtype=torch.bool, device=self.device)
        self.kernel_ms: list[float] = []

    def _rows(self) -> torch.Tensor:
        b = self.game.bucket
        L, C, N = self.lanes, b.per_player_capacity, b.neutral_capacity
        shifts = torch.arange(32, device=self.device, dtype=torch.int64)
        bits = ((self.words.to(torch.int64) & 0xFFFFFFFF)[..., None] >> shifts) & 1
        rows = bits.reshape(L, 2, C, 96)[..., : b.mask_width] != 0
        avail = (self.leaves["birth"][:, N:].reshape(L, 2, C) != -1) & (self.leaves["pending_kind"][:, N:].reshape(L, 2, C) == -1)
        rows = rows & avail[..., None]
        rows[..., 0] |= ~avail
        return rows

    def step(self, timed: bool = True, actions: torch.Tensor | None = None) -> torch.Tensor:
        """One env step of every game; appends the summed reference-kernel
        time (CUDA events on the current stream) to ``kernel_ms``.  Draws the
        actions from the step's masks unless ``actions`` (int32 [L, 2, C, 7])
        are given; returns the masks (bool [L, 2, C, 78]) the step drew from."""
        stream = torch.cuda.current_stream(self.device)
        marks = []

        def run(call):
            if timed:
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                call()
                b.record(stream)
                marks.append((a, b))
            else:
                call()

        run(lambda: self.ref.legality_words(self.leaves, self.words))  # the masks of this step's state
        if self.partial:
            for p in range(2):
                run(lambda p=p: self.ref.visible_cells(self.leaves, p, self.seen))
        rows = self._rows()
        if actions is None:
            actions = sample_uniform(rows, self.widths, self.generator)
        commands = decode_actions(self.leaves, actions, self.game.bucket)
        run(lambda: self.ref.step(self.leaves, self.counters, commands, self.keys, self.events))
        done = self.counters["game_over"] | (self.counters["time"] >= self.game.max_cycles)
        run(lambda: self.ref.reset_where_done(done, self.packed, self.leaves))
        for n in COUNTERS:  # lifecycle.py:116-124: the counters take the reset State's values by select
            shape = (-1,) + (1,) * (self.counters[n].dim() - 1)
            self.leaves[n].copy_(torch.where(done.view(shape), self.reset_rows[n], self.counters[n]))
        if timed:
            torch.cuda.synchronize(self.device)
            self.kernel_ms.append(sum(a.elapsed_time(b) for a, b in marks))
        return rows


class ReferenceDuelPath:
    """The reference's CUDA path for config 4's bot-against-bot step on L
    games: ``nanorts_abstraction_act`` for each player's rush bot (WorkerRush,
    LightRush), ``nanorts_step`` on the two bots' Commands, and
    ``nanorts_reset_packed_where_done``, with torch standing in for the JAX
    between them (``seat_commands``' merge of each player's own rows,
    bots/seat.py:152-157; the lifecycle's select of the counter leaves; the
    empty carries of ended games, seat.py:127).  Only the reference kernels
    are timed."""

    def __init__(self, game: GameConfig, lanes: int, bots: tuple[tuple[int, int], tuple[int, int]],
                 device: str | torch.device = "cuda") -> None:
        from nanorts_b200.content import decide

        self.ref = ReferenceKernels(game, device)
        self.game, self.lanes, self.bots, self.device = game, lanes, bots, torch.device(device)
        reset = decide(game.initial_state, game.bucket)
        self.packed = self.ref.packed_reset_rows(reset)
        self.reset_rows = {n: torch.from_numpy(np.ascontiguousarray(reset[n])).to(self.device) for n in LEAVES}
        self.leaves = {n: v.expand(lanes, *v.shape).contiguous() for n, v in self.reset_rows.items()}
        self.counters = {n: torch.empty_like(self.leaves[n]) for n in COUNTERS}
        self.events = self.ref.event_buffers(lanes)
        self.keys = torch.zeros((lanes, 2), dtype=torch.int32, device=self.device)  # CANCEL_BOTH draws nothing
        C = game.bucket.per_player_capacity
        self.carries = [self._empty_carry(lanes, C) for _ in range(2)]
        self.kernel_ms: list[float] = []

    def _empty_carry(self, lanes: int, capacity: int) -> dict[str, torch.Tensor]:
        carry = {n: torch.full((lanes, capacity), -1, dtype=torch.int32, device=self.device) for n in CARRY_FIELDS}
        carry["trained"] = torch.zeros((lanes, capacity), dtype=torch.uint8, device=self.device)
        carry["next_order"] = torch.zeros((lanes,), dtype=torch.int32, device=self.device)
        return carry

    def step(self, timed: bool = True) -> torch.Tensor:
        """One bot-against-bot step of every game; returns done bool [L]."""
        stream = torch.cuda.current_stream(self.device)
        marks = []

        def run(call):
            if timed:
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                out = call()
                b.record(stream)
                marks.append((a, b))
                return out
            return call()

        issued = [run(lambda p=p: self.ref.bot_act(self.leaves, p, self.bots[p][0], self.bots[p][1], self.carries[p]))
                  for p in range(2)]
        commands = [torch.cat([issued[0][:, f, :1], issued[1][:, f, 1:]], dim=1).contiguous() for f in range(6)]
        run(lambda: self.ref.step(self.leaves, self.counters, commands, self.keys, self.events))
        done = self.counters["game_over"] | (self.counters["time"] >= self.game.max_cycles)
        run(lambda: self.ref.reset_where_done(done, self.packed, self.leaves))
        for n in COUNTERS:
            shape = (-1,) + (1,) * (self.counters[n].dim() - 1)
            self.leaves[n].copy_(torch.where(done.view(shape), self.reset_rows[n], self.counters[n]))
        for carry in self.carries:  # a finished game's carries start over from empty_actions
            for n, v in carry.items():
                fill = -1 if n in CARRY_FIELDS else 0
                shape = (-1,) + (1,) * (v.dim() - 1)
                v.copy_(torch.where(done.view(shape), torch.full_like(v, fill), v))
        if timed:
            torch.cuda.synchronize(self.device)
            self.kernel_ms.append(sum(a.elapsed_time(b) for a, b in marks))
        return done.reshape(-1)
