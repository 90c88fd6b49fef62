"""The jax.ffi handlers on a B200, bit for bit against the facade.

The handlers (nanorts_b200/ffi/nanorts_b200_ffi.cc) are built against the
XLA FFI interface stand-in with the test harness (tests/test_jax_ffi.py
build_shim) and handed device buffers laid out as XLA would: the State
leaves aliased in place, the reset State as shared-row operands, the
scenario as attributes.  Reset, steps with auto-reset, legality rows,
observations and a rush bot's act through the handlers equal the same calls
through the facade (env.reset / env.step / get_avail_actions / get_obs /
Bot.act) on the same inputs.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from tests.parity import CONFIGS, random_keys
from tests.test_jax_ffi import build_shim

pytestmark = pytest.mark.gpu

CODES = {torch.bool: 1, torch.int8: 2, torch.int16: 3, torch.int32: 4, torch.uint8: 6, torch.uint32: 8, torch.float32: 10}


class Buf(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("dtype", ctypes.c_int32), ("rank", ctypes.c_int32),
                ("dims", ctypes.c_int64 * 6)]


def describe(t: torch.Tensor) -> Buf:
    assert t.is_contiguous()
    b = Buf(data=t.data_ptr(), dtype=CODES[t.dtype], rank=t.dim())
    for k, n in enumerate(t.shape):
        b.dims[k] = n
    return b


@pytest.fixture(scope="module")
def shim(tmp_path_factory):
    lib = ctypes.CDLL(str(build_shim(tmp_path_factory.mktemp("shim"))))
    p, i64 = ctypes.c_void_p, ctypes.c_int64
    lib.shim_call.argtypes = [ctypes.c_int32, p, p, i64, p, i64, p, p, i64, p, i64]
    lib.shim_call.restype = ctypes.c_int
    lib.shim_last_error.restype = ctypes.c_char_p
    return lib


class Handlers:
    """The five handlers for one scenario through the harness."""

    def __init__(self, lib, game, partial=False):
        from nanorts_b200 import jax_binding

        self.lib = lib
        attrs = jax_binding.scenario_attributes(game, partial)
        self.ints = np.array([int(attrs[k]) for k in ("height", "width", "neutral", "capacity", "types", "offsets",
                                                      "strategy", "max_cycles", "partial_observability")] + [0, 0, 0],
                             np.int64)
        self.terrain, self.table = attrs["terrain"], attrs["table"]
        self.reset_rows = [torch.from_numpy(r).cuda() for r in jax_binding.reset_operands(game)]

    def call(self, target, args, rets, bot=(0, 0, 0)):
        self.ints[9:] = bot
        a = (Buf * len(args))(*[describe(t) for t in args])
        r = (Buf * len(rets))(*[describe(t) for t in rets])
        rc = self.lib.shim_call(target, torch.cuda.current_stream().cuda_stream, a, len(args), r, len(rets),
                                self.ints.ctypes.data, self.terrain.ctypes.data, self.terrain.size,
                                self.table.ctypes.data, self.table.size)
        assert rc == 0, self.lib.shim_last_error().decode()

    @staticmethod
    def state(es):
        return [*es.core_state.leaves(), es.environment_root, es.episode_index]


def _same(got: torch.Tensor, want: torch.Tensor, where: str) -> None:
    g, w = got.cpu(), want.cpu()
    if g.dtype == torch.uint32:
        g, w = g.view(torch.int32), w.view(torch.int32)
    assert torch.equal(g.view(w.shape) if g.numel() == w.numel() else g, w), where


@pytest.mark.parametrize("config_name", ["c2_16x16_random", "c3_16x16_alternating_partial", "c5_64x64_random"])
def test_handlers_match_the_facade(shim, config_name):
    from nanorts_b200.env import make

    cfg = CONFIGS[config_name]
    game = cfg.game(60)
    b = game.bucket
    L = 24 if not config_name.startswith("c5") else 6
    C, H, W = b.per_player_capacity, b.height, b.width
    env = make("NanoRTS", scenario=game, partial_observability=cfg.partial, final_observation=False)
    h = Handlers(shim, game, cfg.partial)
    keys = torch.from_numpy(random_keys(np.random.default_rng(3), L).view(np.int32)).cuda().view(torch.uint32)
    obs, state = env.reset(keys)
    mine = env._empty_state(L)
    dev = dict(device="cuda")
    masks = [torch.empty((L, C, b.mask_width), dtype=torch.bool, **dev) for _ in range(2)]
    maps = [torch.empty((L, H, W, 6), dtype=torch.uint8, **dev) for _ in range(2)]
    scalars = [torch.empty((L, 4), dtype=torch.int32, **dev) for _ in range(2)]
    h.call(1, [*h.state(mine), *h.reset_rows, keys.contiguous()], [*h.state(mine), *masks, *maps, *scalars])
    for k, (x, y) in enumerate(zip(h.state(mine), h.state(state))):
        _same(x, y, f"reset leaf {k}")
    reward = torch.empty((L, 2), dtype=torch.float32, **dev)
    done, term, trunc = (torch.empty((L,), dtype=torch.bool, **dev) for _ in range(3))
    winner = torch.empty((L,), dtype=torch.int32, **dev)
    overflow = torch.empty((L, 2), dtype=torch.int32, **dev)
    ended = 0
    for t in range(90):
        acts = {a: v.clone() for a, v in env.sample_actions(state, seed=5, counter=t).items()}
        obs, state, rewards, dones, infos = env.step(None, state, acts)
        h.call(0, [*h.state(mine), *h.reset_rows, acts["player_0"], acts["player_1"]],
               [*h.state(mine), *masks, *maps, *scalars, reward, done, term, trunc, winner, overflow])
        where = f"{config_name} step {t}"
        for k, (x, y) in enumerate(zip(h.state(mine), h.state(state))):
            _same(x, y, f"{where}: leaf {k}")
        got = env.get_avail_actions(state)
        for p, agent in enumerate(("player_0", "player_1")):
            _same(masks[p], got[agent], f"{where}: masks {agent}")
            _same(maps[p], obs[agent].feature_maps, f"{where}: feature maps {agent}")
            _same(scalars[p], obs[agent].scalars, f"{where}: scalars {agent}")
            _same(reward[:, p].contiguous(), rewards[agent], f"{where}: reward {agent}")
        _same(done, dones["__all__"], f"{where}: done")
        _same(term, infos["terminated"], f"{where}: terminated")
        _same(trunc, infos["truncated"], f"{where}: truncated")
        _same(winner, infos["winner"], f"{where}: winner")
        _same(overflow, infos["telemetry"].spawn_overflow, f"{where}: spawn_overflow")
        ended += int(done.sum())
    assert ended > 0
    # Stand-alone legality rows and observations of the same state.
    env.invalidate(state)
    h.call(2, [*h.state(mine), *h.reset_rows], masks)
    h.call(3, [*h.state(mine), *h.reset_rows], [*maps, *scalars])
    want_masks, want_obs = env.get_avail_actions(state), env.get_obs(state)
    for p, agent in enumerate(("player_0", "player_1")):
        _same(masks[p], want_masks[agent], f"legal_masks {agent}")
        _same(maps[p], want_obs[agent].feature_maps, f"observe {agent}")
        _same(scalars[p], want_obs[agent].scalars, f"observe scalars {agent}")


def test_bot_act_handler_matches_the_facade(shim):
    from nanorts_b200.bots import CARRY_FIELDS, lightRushAI, workerRushAI
    from nanorts_b200.env import make
    from nanorts_b200.model import ConflictStrategy, UnitTypeTableVersion
    from tests.parity import Config

    game = Config("c4", "basesWorkers16x16", UnitTypeTableVersion.ORIGINAL, ConflictStrategy.CANCEL_BOTH).game(5000)
    L = 16
    env = make("NanoRTS", scenario=game, final_observation=False)
    h = Handlers(shim, game)
    _, state = env.reset(torch.zeros((L, 2), dtype=torch.int32, device="cuda").view(torch.uint32))
    carries = [workerRushAI.init(env, L), lightRushAI.init(env, L)]
    mine = [bot.init(env, L) for bot in (workerRushAI, lightRushAI)]
    rng = np.random.default_rng(0)
    for t in range(120):
        for p, bot in enumerate((workerRushAI, lightRushAI)):
            want = bot.act(None, carries[p], state, env, p)
            carry = [*(getattr(mine[p], f) for f in CARRY_FIELDS), mine[p].trained, mine[p].next_order]
            commands = torch.empty((L, 6, 2, game.bucket.per_player_capacity), dtype=torch.int32, device="cuda")
            trained = mine[p].trained
            carry_view = [*carry[:-2], trained.view(torch.bool) if trained.dtype == torch.uint8 else trained, carry[-1]]
            h.call(4, [*Handlers.state(state), *h.reset_rows, *carry_view], [*carry_view, commands],
                   bot=(p, bot.strategy, bot.trained))
            _same(commands, want, f"step {t} player {p}: commands")
            for f in CARRY_FIELDS:
                _same(getattr(mine[p], f), getattr(carries[p], f), f"step {t} player {p}: carry {f}")
        acts = {a: v.clone() for a, v in env.sample_actions(state, seed=int(rng.integers(1 << 30)), counter=t).items()}
        env.step(None, state, acts)
