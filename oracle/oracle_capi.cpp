// C ABI of the CPU oracle (test infrastructure only; see oracle.hpp).
//
// Buffers are lane-major like the product's: leaf k of lane l starts at
// leaf[k] + l * row_bytes(k).  Leaves follow the reference State declaration
// order (state.py:35-80, telemetry.spawn_overflow last), the same order as the
// reference step kernel's Leaf enum (core/cuda/step.cu:61-85).
#include <omp.h>

#include <cstdint>
#include <cstring>
#include <vector>

#include "bots.hpp"
#include "oracle.hpp"

using namespace oracle;

namespace {

enum LeafIndex : int {
    kBirth, kUnitType, kOwner, kCell, kHitPoints, kCarried, kPendingKind, kPendingDirection, kPendingNoneDuration,
    kPendingTargetCell, kPendingProducedType, kPendingIssuedAt, kPendingCompletesAt, kPendingOrder, kEntityAt, kTime,
    kPlayerResources, kNextBirth, kNextPendingOrder, kAlternating, kGameOver, kWinner, kSpawnOverflow, kLeaves
};

}  // namespace

extern "C" {

struct OracleConfig {
    int32_t height, width, neutral, capacity, types, offsets, strategy, max_cycles;
    int32_t partial_observability;
    int32_t final_observation;
    const uint8_t* terrain;
    const int32_t* table;
    const void* reset[kLeaves];  // one game's reset State (decide(initial_state))
};

struct OracleStates {
    void* leaf[kLeaves];
    uint32_t* environment_root;  // [L, 2]
    uint32_t* episode_index;     // [L]
};

// One player's bot carry, AbstractActions (bots/abstraction.py:71-82),
// lane-major: nine int32 [L, C] fields in declaration order, trained
// uint8 [L, C], next_order int32 [L].
struct OracleCarry {
    int32_t* field[9];
    uint8_t* trained;
    int32_t* next_order;
};

}  // extern "C"

namespace {

int64_t row_bytes(const Extents& x, int leaf) {
    const int64_t E = x.entities();
    switch (leaf) {
        case kBirth: case kCarried: case kPendingNoneDuration: case kPendingIssuedAt: case kPendingCompletesAt: case kPendingOrder:
            return 4 * E;
        case kUnitType: case kOwner: case kPendingKind: case kPendingDirection: case kPendingProducedType:
            return E;
        case kCell: case kHitPoints: case kPendingTargetCell:
            return 2 * E;
        case kEntityAt:
            return 2 * static_cast<int64_t>(x.cells());
        case kPlayerResources: case kSpawnOverflow:
            return 8;
        case kGameOver:
            return 1;
        default:
            return 4;
    }
}

Extents extents_of(const OracleConfig* c) {
    return Extents{c->height, c->width, c->neutral, c->capacity, c->types, c->offsets, c->strategy, c->max_cycles};
}

Game game_at(void* const leaf[kLeaves], const Extents& x, int64_t lane) {
    auto at = [&](int k) { return static_cast<char*>(leaf[k]) + lane * row_bytes(x, k); };
    Game g;
    g.birth = reinterpret_cast<int32_t*>(at(kBirth));
    g.unit_type = reinterpret_cast<int8_t*>(at(kUnitType));
    g.owner = reinterpret_cast<int8_t*>(at(kOwner));
    g.cell = reinterpret_cast<int16_t*>(at(kCell));
    g.hit_points = reinterpret_cast<int16_t*>(at(kHitPoints));
    g.carried = reinterpret_cast<int32_t*>(at(kCarried));
    g.pending_kind = reinterpret_cast<int8_t*>(at(kPendingKind));
    g.pending_direction = reinterpret_cast<int8_t*>(at(kPendingDirection));
    g.pending_none_duration = reinterpret_cast<int32_t*>(at(kPendingNoneDuration));
    g.pending_target_cell = reinterpret_cast<int16_t*>(at(kPendingTargetCell));
    g.pending_produced_type = reinterpret_cast<int8_t*>(at(kPendingProducedType));
    g.pending_issued_at = reinterpret_cast<int32_t*>(at(kPendingIssuedAt));
    g.pending_completes_at = reinterpret_cast<int32_t*>(at(kPendingCompletesAt));
    g.pending_order = reinterpret_cast<int32_t*>(at(kPendingOrder));
    g.entity_at = reinterpret_cast<int16_t*>(at(kEntityAt));
    g.time = reinterpret_cast<int32_t*>(at(kTime));
    g.player_resources = reinterpret_cast<int32_t*>(at(kPlayerResources));
    g.next_birth = reinterpret_cast<int32_t*>(at(kNextBirth));
    g.next_pending_order = reinterpret_cast<int32_t*>(at(kNextPendingOrder));
    g.alternating_conflict_count = reinterpret_cast<int32_t*>(at(kAlternating));
    g.game_over = reinterpret_cast<uint8_t*>(at(kGameOver));
    g.winner = reinterpret_cast<int32_t*>(at(kWinner));
    g.spawn_overflow = reinterpret_cast<int32_t*>(at(kSpawnOverflow));
    return g;
}

void copy_reset(const OracleConfig* c, void* const leaf[kLeaves], const Extents& x, int64_t lane) {
    for (int k = 0; k < kLeaves; ++k) {
        const int64_t bytes = row_bytes(x, k);
        std::memcpy(static_cast<char*>(leaf[k]) + lane * bytes, c->reset[k], bytes);
    }
}

void set_threads(int threads) {
    if (threads > 0) omp_set_num_threads(threads);
}

int check(const OracleConfig* c) {
    if (c->height * c->width > 32767 || c->neutral + 2 * c->capacity > 32767) return 1;  // int16 indices only
    if (4 * 4 + 6 + c->types + c->offsets > 96) return 2;
    return 0;
}

}  // namespace

extern "C" {

// lifecycle.py:34-37 episode_root = fold_in(environment_root, episode_index).
static Key episode_root(const OracleStates* s, int64_t lane) {
    return fold_in(Key{s->environment_root[2 * lane], s->environment_root[2 * lane + 1]}, s->episode_index[lane]);
}

// The JaxMARL step (adapters/jaxmarl/env.py:72-75 step = transition + respond):
// decode -> core.step -> lifecycle.advance (auto-reset) -> observe the carried state.
// `final_*` (may be null) receive observe(next_state) before the reset (env.py:161-170);
// `components` (may be null) receives the reward components [L, 2, 6] (env.py:173-174).
int oracle_env_step(const OracleConfig* c, OracleStates* s, int64_t lanes, const int32_t* actions0, const int32_t* actions1,
                    uint8_t* fm0, uint8_t* fm1, int32_t* sc0, int32_t* sc1, float* reward, uint8_t* done, uint8_t* terminated,
                    uint8_t* truncated, int32_t* winner, int32_t* spawn_overflow, uint8_t* final_fm0, uint8_t* final_fm1,
                    int32_t* final_sc0, int32_t* final_sc1, float* components, int threads) {
    if (int e = check(c)) return e;
    set_threads(threads);
    const Extents x = extents_of(c);
    const Content content{c->terrain, c->table, c->types};
    const int64_t C = x.capacity, cells = x.cells();
#pragma omp parallel for schedule(dynamic, 4)
    for (int64_t lane = 0; lane < lanes; ++lane) {
        Game g = game_at(s->leaf, x, lane);
        const int32_t* actions[kPlayers] = {actions0 + lane * C * 7, actions1 + lane * C * 7};
        const Commands cmd = decode_actions(g, x, actions);
        const Key key = episode_root(s, lane);
        const StepOutcome out = core_step(g, content, x, cmd, key);
        const bool finished = out.terminated || out.truncated;
        reward[2 * lane] = out.reward[0];
        reward[2 * lane + 1] = out.reward[1];
        done[lane] = finished;
        terminated[lane] = out.terminated;
        truncated[lane] = out.truncated;
        winner[lane] = *g.winner;
        spawn_overflow[2 * lane] = g.spawn_overflow[0];
        spawn_overflow[2 * lane + 1] = g.spawn_overflow[1];
        if (components != nullptr) std::memcpy(components + lane * 12, out.components, sizeof(out.components));
        if (final_fm0 != nullptr) {
            uint8_t* maps[kPlayers] = {final_fm0 + lane * cells * 6, final_fm1 + lane * cells * 6};
            int32_t* scalars[kPlayers] = {final_sc0 + lane * 4, final_sc1 + lane * 4};
            observe(g, content, x, c->partial_observability != 0, maps, scalars);
        }
        if (finished) {
            s->episode_index[lane] += 1u;
            copy_reset(c, s->leaf, x, lane);
        }
        uint8_t* maps[kPlayers] = {fm0 + lane * cells * 6, fm1 + lane * cells * 6};
        int32_t* scalars[kPlayers] = {sc0 + lane * 4, sc1 + lane * 4};
        observe(g, content, x, c->partial_observability != 0, maps, scalars);
    }
    return 0;
}

// core.step with explicit Commands (core/__init__.py:46-60); commands are
// [L, 6, 2, C] int32 in the field order of Commands (commands.py:22-35).
int oracle_core_step(const OracleConfig* c, OracleStates* s, int64_t lanes, const int32_t* commands, const uint32_t* keys,
                     uint8_t* terminated, uint8_t* truncated, float* reward, int threads) {
    if (int e = check(c)) return e;
    set_threads(threads);
    const Extents x = extents_of(c);
    const Content content{c->terrain, c->table, c->types};
    const int64_t owned = x.owned();
#pragma omp parallel for schedule(dynamic, 4)
    for (int64_t lane = 0; lane < lanes; ++lane) {
        Game g = game_at(s->leaf, x, lane);
        Commands cmd(static_cast<int>(owned));
        const int32_t* row = commands + lane * 6 * owned;
        for (int64_t k = 0; k < owned; ++k) {
            cmd.kind[k] = row[k];
            cmd.direction[k] = row[owned + k];
            cmd.none_duration[k] = row[2 * owned + k];
            cmd.target_cell[k] = row[3 * owned + k];
            cmd.produced_type[k] = row[4 * owned + k];
            cmd.request_order[k] = row[5 * owned + k];
        }
        const StepOutcome out = core_step(g, content, x, cmd, Key{keys[2 * lane], keys[2 * lane + 1]});
        terminated[lane] = out.terminated;
        truncated[lane] = out.truncated;
        reward[2 * lane] = out.reward[0];
        reward[2 * lane + 1] = out.reward[1];
    }
    return 0;
}

// adapters/jaxmarl/actions.py:61-84 decode_actions alone: the Commands
// int32 [L, 6, 2, C] (kind, direction, none_duration, target_cell,
// produced_type, request_order) the JaxMARL step hands core.step.
int oracle_decode_actions(const OracleConfig* c, OracleStates* s, int64_t lanes, const int32_t* actions0,
                          const int32_t* actions1, int32_t* commands, int threads) {
    if (int e = check(c)) return e;
    set_threads(threads);
    const Extents x = extents_of(c);
    const int64_t owned = x.owned();
    const int64_t span = static_cast<int64_t>(x.capacity) * 7;
#pragma omp parallel for schedule(dynamic, 8)
    for (int64_t lane = 0; lane < lanes; ++lane) {
        const Game g = game_at(s->leaf, x, lane);
        const int32_t* const actions[kPlayers] = {actions0 + lane * span, actions1 + lane * span};
        const Commands cmd = decode_actions(g, x, actions);
        int32_t* row = commands + lane * 6 * owned;
        for (int64_t k = 0; k < owned; ++k) {
            row[k] = cmd.kind[k];
            row[owned + k] = cmd.direction[k];
            row[2 * owned + k] = cmd.none_duration[k];
            row[3 * owned + k] = cmd.target_cell[k];
            row[4 * owned + k] = cmd.produced_type[k];
            row[5 * owned + k] = cmd.request_order[k];
        }
    }
    return 0;
}

// observations/visibility.py:70-77: uint8 [L, H*W] cells `player` sees (0/1).
int oracle_visible_cells(const OracleConfig* c, OracleStates* s, int64_t lanes, int32_t player, uint8_t* out, int threads) {
    if (int e = check(c)) return e;
    set_threads(threads);
    const Extents x = extents_of(c);
    const Content content{c->terrain, c->table, c->types};
#pragma omp parallel for schedule(dynamic, 8)
    for (int64_t lane = 0; lane < lanes; ++lane) {
        const Game g = game_at(s->leaf, x, lane);
        std::vector<uint8_t> seen;
        visible_cells(g, content, x, player, seen);
        std::memcpy(out + lane * x.cells(), seen.data(), seen.size());
    }
    return 0;
}

int oracle_legal_masks(const OracleConfig* c, OracleStates* s, int64_t lanes, uint8_t* masks0, uint8_t* masks1, int threads) {
    if (int e = check(c)) return e;
    set_threads(threads);
    const Extents x = extents_of(c);
    const Content content{c->terrain, c->table, c->types};
    const int64_t span = static_cast<int64_t>(x.capacity) * x.mask_width();
#pragma omp parallel for schedule(dynamic, 8)
    for (int64_t lane = 0; lane < lanes; ++lane) {
        Game g = game_at(s->leaf, x, lane);
        uint8_t* masks[kPlayers] = {masks0 + lane * span, masks1 + lane * span};
        legal_rows(g, content, x, masks);
    }
    return 0;
}

int oracle_observe(const OracleConfig* c, OracleStates* s, int64_t lanes, uint8_t* fm0, uint8_t* fm1, int32_t* sc0, int32_t* sc1, int threads) {
    if (int e = check(c)) return e;
    set_threads(threads);
    const Extents x = extents_of(c);
    const Content content{c->terrain, c->table, c->types};
    const int64_t cells = x.cells();
#pragma omp parallel for schedule(dynamic, 8)
    for (int64_t lane = 0; lane < lanes; ++lane) {
        Game g = game_at(s->leaf, x, lane);
        uint8_t* maps[kPlayers] = {fm0 + lane * cells * 6, fm1 + lane * cells * 6};
        int32_t* scalars[kPlayers] = {sc0 + lane * 4, sc1 + lane * 4};
        observe(g, content, x, c->partial_observability != 0, maps, scalars);
    }
    return 0;
}

// reset (lifecycle.py:44-50): every lane to the reset State, episode 0.
int oracle_reset(const OracleConfig* c, OracleStates* s, int64_t lanes) {
    const Extents x = extents_of(c);
    for (int64_t lane = 0; lane < lanes; ++lane) {
        copy_reset(c, s->leaf, x, lane);
        s->episode_index[lane] = 0u;
    }
    return 0;
}

static bots::Actions load_carry(const OracleCarry* k, int64_t lane, int32_t C) {
    bots::Actions a(C);
    std::vector<int32_t>* fields[9] = {&a.kind, &a.unit_birth, &a.order, &a.target, &a.target_birth,
                                       &a.base, &a.base_birth, &a.cell, &a.unit_type};
    for (int f = 0; f < 9; ++f) std::memcpy(fields[f]->data(), k->field[f] + lane * C, 4 * C);
    std::memcpy(a.trained.data(), k->trained + lane * C, C);
    a.next_order = k->next_order[lane];
    return a;
}

static void store_carry(OracleCarry* k, int64_t lane, int32_t C, const bots::Actions& a) {
    const std::vector<int32_t>* fields[9] = {&a.kind, &a.unit_birth, &a.order, &a.target, &a.target_birth,
                                             &a.base, &a.base_birth, &a.cell, &a.unit_type};
    for (int f = 0; f < 9; ++f) std::memcpy(k->field[f] + lane * C, fields[f]->data(), 4 * C);
    std::memcpy(k->trained + lane * C, a.trained.data(), C);
    k->next_order[lane] = a.next_order;
}

// family.act (bots/family.py:34-81, program branch) for one player's rush
// bot: the carry is updated in place and `commands` [L, 6, 2, C] receives
// the Commands fields (kind, direction, none_duration, target_cell,
// produced_type, request_order); the other player's row is unissued.
int oracle_bot_act(const OracleConfig* c, OracleStates* s, int64_t lanes, int32_t player, int32_t strategy,
                   int32_t trained_type, OracleCarry* carry, int32_t* commands, int threads) {
    if (int e = check(c)) return e;
    if (player < 0 || player > 1 || strategy < 0 || strategy > 1) return 3;
    set_threads(threads);
    const Extents x = extents_of(c);
    const Content content{c->terrain, c->table, c->types};
    const int32_t C = x.capacity;
#pragma omp parallel for schedule(dynamic, 4)
    for (int64_t lane = 0; lane < lanes; ++lane) {
        Game g = game_at(s->leaf, x, lane);
        bots::Actions a = load_carry(carry, lane, C);
        int32_t* base = commands + lane * 6 * 2 * C;
        static const int32_t empty[6] = {kAbsent, kAbsent, 0, kAbsent, kAbsent, kAbsent};
        for (int f = 0; f < 6; ++f) std::fill(base + (f * 2 + (1 - player)) * C, base + (f * 2 + (1 - player) + 1) * C, empty[f]);
        int32_t* rows[6];
        for (int f = 0; f < 6; ++f) rows[f] = base + (f * 2 + player) * C;
        const bots::Bot bot{x, content, g, player};
        bot.act(strategy, trained_type, a, rows);
        store_carry(carry, lane, C, a);
    }
    return 0;
}

// Bot against bot: each player's commands come from its own rush bot acting
// on the step's starting state (bots/seat.py:152-157 for one seat, applied to
// both), then core.step, then the lifecycle's auto-reset
// (adapters/lifecycle.py:53-75); a finished game's carries go back to
// empty_actions (bots/seat.py:127).
int oracle_duel_step(const OracleConfig* c, OracleStates* s, int64_t lanes, const int32_t* strategies, const int32_t* trained,
                     OracleCarry* carry0, OracleCarry* carry1, float* reward, uint8_t* done, uint8_t* terminated,
                     uint8_t* truncated, int32_t* winner, int32_t* spawn_overflow, int threads) {
    if (int e = check(c)) return e;
    for (int p = 0; p < kPlayers; ++p)
        if (strategies[p] < 0 || strategies[p] > 1) return 3;
    set_threads(threads);
    const Extents x = extents_of(c);
    const Content content{c->terrain, c->table, c->types};
    const int32_t C = x.capacity;
    OracleCarry* carries[kPlayers] = {carry0, carry1};
#pragma omp parallel for schedule(dynamic, 4)
    for (int64_t lane = 0; lane < lanes; ++lane) {
        Game g = game_at(s->leaf, x, lane);
        Commands cmd(x.owned());
        bots::Actions acts[kPlayers] = {load_carry(carry0, lane, C), load_carry(carry1, lane, C)};
        for (int p = 0; p < kPlayers; ++p) {
            int32_t* rows[6] = {cmd.kind.data() + p * C, cmd.direction.data() + p * C, cmd.none_duration.data() + p * C,
                                cmd.target_cell.data() + p * C, cmd.produced_type.data() + p * C,
                                cmd.request_order.data() + p * C};
            const bots::Bot bot{x, content, g, p};
            bot.act(strategies[p], trained[p], acts[p], rows);
        }
        const StepOutcome out = core_step(g, content, x, cmd, episode_root(s, lane));
        const bool finished = out.terminated || out.truncated;
        reward[2 * lane] = out.reward[0];
        reward[2 * lane + 1] = out.reward[1];
        done[lane] = finished;
        terminated[lane] = out.terminated;
        truncated[lane] = out.truncated;
        winner[lane] = *g.winner;
        spawn_overflow[2 * lane] = g.spawn_overflow[0];
        spawn_overflow[2 * lane + 1] = g.spawn_overflow[1];
        if (finished) {
            s->episode_index[lane] += 1u;
            copy_reset(c, s->leaf, x, lane);
            acts[0] = bots::Actions(C);
            acts[1] = bots::Actions(C);
        }
        for (int p = 0; p < kPlayers; ++p) store_carry(carries[p], lane, C, acts[p]);
    }
    return 0;
}

// pathfinding.search (program branch): out = {found, step, distance, pops}.
void oracle_astar(const uint8_t* free, int32_t height, int32_t width, int32_t start, int32_t target, int32_t range, int32_t* out) {
    const bots::Mask open(free, free + height * width);
    const bots::Path p = bots::Bot::search(open, start, target, range, height, width);
    out[0] = p.found;
    out[1] = p.step;
    out[2] = p.distance;
    out[3] = p.pops;
}

void oracle_threefry2x32(uint32_t k0, uint32_t k1, uint32_t* x0, uint32_t* x1) { threefry2x32(k0, k1, *x0, *x1); }

void oracle_fold_in(uint32_t k0, uint32_t k1, uint32_t data, uint32_t* out) {
    const Key k = fold_in(Key{k0, k1}, data);
    out[0] = k.k0;
    out[1] = k.k1;
}

int32_t oracle_conflict_draw(uint32_t k0, uint32_t k1, int32_t time, int32_t birth, int32_t ordinal) {
    return randint01(fold_in(conflict_event_key(Key{k0, k1}, time, birth), static_cast<uint32_t>(ordinal)));
}

}  // extern "C"
