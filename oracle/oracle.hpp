// CPU oracle: a C++17 restatement of NanoRTS's JAX program path.
//
// TEST INFRASTRUCTURE ONLY.  Nothing in the product (nanorts_b200/) may call,
// link or load this code; only tests/, __graft_entry__.smoke() and the
// cpu_baseline / --impl reference leg of bench.py use it, as the checker and as
// the timed CPU baseline.
//
// It follows the reference's JAX program (the CPU branch of
// kernels.dispatch), not its CUDA kernels, and keeps the program's data-parallel
// formulation where the kernels take shortcuts: full-length sorts, full-length
// prefix scans over every slot in pending order, masked writes.  Each function
// cites the reference file:line it restates (paths under src/nanorts/).
//
// Parity pin: the reference ships no tests and no golden vectors, and its JAX
// program cannot run here (no jax/jaxlib).  The threefry composition is pinned
// against the reference's own core/cuda/conflict_draw.cuh compiled from its
// source (oracle/ref_draws.cpp) and against the Random123 known-answer vectors;
// the game rules are pinned by hand-derived known-answer scenarios in tests/.
#pragma once

#include <algorithm>
#include <climits>
#include <cstdint>
#include <cstring>
#include <numeric>
#include <vector>

namespace oracle {

constexpr int kAbsent = -1;
constexpr int kPlayers = 2;
constexpr int kKindNone = 0, kKindMove = 1, kKindHarvest = 2, kKindReturn = 3, kKindProduce = 4, kKindAttack = 5;
constexpr int kKinds = 6;
constexpr int kDirections = 4;
constexpr int32_t kNoCap = INT32_MAX;
constexpr int kStrategyBoth = 0, kStrategyRandom = 1, kStrategyAlternating = 2;

// Unit table columns (nanorts_b200/model.py UNIT_COLUMNS), then `produces`.
enum Column : int {
    kCost, kHitPoints, kProduceTime, kMoveTime, kAttackTime, kHarvestTime, kAttackRange, kAttackDamage,
    kHarvestAmount, kSightRadius, kIsResource, kIsStockpile, kCanHarvest, kCanMove, kCanAttack, kColumns
};

// ---------------------------------------------------------------------------
// threefry2x32 (Salmon et al., SC'11, "Parallel random numbers: as easy as
// 1, 2, 3"): 20 rounds, key schedule with the Skein parity constant, the
// rotation set R_{2x32} and a key injection after every fourth round.
// ---------------------------------------------------------------------------
inline uint32_t rotl(uint32_t v, int r) { return (v << r) | (v >> (32 - r)); }

inline void threefry2x32(uint32_t k0, uint32_t k1, uint32_t& x0, uint32_t& x1) {
    static const int kRot[8] = {13, 15, 26, 6, 17, 29, 16, 24};
    const uint32_t ks[3] = {k0, k1, k0 ^ k1 ^ 0x1BD11BDAu};
    x0 += ks[0];
    x1 += ks[1];
    for (int round = 0; round < 20; ++round) {
        x0 += x1;
        x1 = rotl(x1, kRot[round % 8]);
        x1 ^= x0;
        if (round % 4 == 3) {
            const int s = round / 4 + 1;
            x0 += ks[s % 3];
            x1 += ks[(s + 1) % 3] + static_cast<uint32_t>(s);
        }
    }
}

struct Key {
    uint32_t k0, k1;
};

// jax.random.fold_in under threefry: threefry(key, threefry_seed(data)) with
// threefry_seed(d) = (d >> 32, d & 0xffffffff) = (0, d) for 32-bit data.
inline Key fold_in(Key key, uint32_t data) {
    uint32_t x0 = 0u, x1 = data;
    threefry2x32(key.k0, key.k1, x0, x1);
    return Key{x0, x1};
}

// jax.random.randint(key, (), 0, 2) with jax_threefry_partitionable: split
// the key foldlike into (threefry(key,(0,0)), threefry(key,(0,1))); the second
// key's 32 random bits (b0 ^ b1 of threefry(k2,(0,0))) taken mod 2 (the span-2
// multiplier term of randint vanishes).  reservations.py:303-306.
inline int32_t randint01(Key key) {
    uint32_t s0 = 0u, s1 = 1u;
    threefry2x32(key.k0, key.k1, s0, s1);
    uint32_t b0 = 0u, b1 = 0u;
    threefry2x32(s0, s1, b0, b1);
    return static_cast<int32_t>((b0 ^ b1) & 1u);
}

// reservations.py:297-300: fold_in(fold_in(fold_in(key, time), birth), 0).
inline Key conflict_event_key(Key key, int32_t time, int32_t birth) {
    return fold_in(fold_in(fold_in(key, static_cast<uint32_t>(time)), static_cast<uint32_t>(birth)), 0u);
}

// ---------------------------------------------------------------------------
// Extents and views.
// ---------------------------------------------------------------------------
struct Extents {
    int32_t height, width, neutral, capacity, types, offsets, strategy, max_cycles;
    int32_t cells() const { return height * width; }
    int32_t entities() const { return neutral + kPlayers * capacity; }
    int32_t owned() const { return kPlayers * capacity; }
    int32_t side() const { int s = 1; while (s * s < offsets) ++s; return s; }
    int32_t radius() const { return (side() - 1) / 2; }
    int32_t mask_width() const { return kKinds + 4 * kDirections + types + offsets; }
};

struct Content {
    const uint8_t* terrain;  // [cells]
    const int32_t* table;    // [types, kColumns + types]
    int32_t types;
    int32_t at(int32_t type, int column) const { return table[type * (kColumns + types) + column]; }
    bool produces(int32_t producer, int32_t produced) const { return table[producer * (kColumns + types) + kColumns + produced] != 0; }
};

// One game's State, as pointers into lane-major leaves (state.py:35-80).
struct Game {
    int32_t* birth;
    int8_t* unit_type;
    int8_t* owner;
    int16_t* cell;
    int16_t* hit_points;
    int32_t* carried;
    int8_t* pending_kind;
    int8_t* pending_direction;
    int32_t* pending_none_duration;
    int16_t* pending_target_cell;
    int8_t* pending_produced_type;
    int32_t* pending_issued_at;
    int32_t* pending_completes_at;
    int32_t* pending_order;
    int16_t* entity_at;
    int32_t* time;
    int32_t* player_resources;
    int32_t* next_birth;
    int32_t* next_pending_order;
    int32_t* alternating_conflict_count;
    uint8_t* game_over;
    int32_t* winner;
    int32_t* spawn_overflow;

    bool active(int32_t slot) const { return birth[slot] != kAbsent; }
};

// Commands of one game (commands.py:22-35), player-major [2, C].
struct Commands {
    std::vector<int32_t> kind, direction, none_duration, target_cell, produced_type, request_order;
    explicit Commands(int owned)
        : kind(owned, kAbsent), direction(owned, kAbsent), none_duration(owned, 0), target_cell(owned, kAbsent),
          produced_type(owned, kAbsent), request_order(owned, kAbsent) {}
};

inline int32_t clip(int32_t v, int32_t lo, int32_t hi) { return v < lo ? lo : (v > hi ? hi : v); }
inline int32_t floor_div(int32_t a, int32_t b) { int32_t q = a / b; return (a % b != 0 && ((a < 0) != (b < 0))) ? q - 1 : q; }
inline int32_t floor_mod(int32_t a, int32_t b) { return a - floor_div(a, b) * b; }
// JAX gathers clamp out-of-range indices (after wrapping negatives once).
inline int32_t gather(int32_t index, int32_t size) { if (index < 0) index += size; return clip(index, 0, size - 1); }

constexpr int kDx[4] = {0, 1, 0, -1};
constexpr int kDy[4] = {-1, 0, 1, 0};

// board.py:64-77 reserved_position: cell + (dx + dy * W) of the clipped direction.
inline int32_t reserved_position(int32_t cell, int32_t direction, const Extents& x) {
    const int d = clip(direction, 0, kDirections - 1);
    return cell + kDx[d] + kDy[d] * x.width;
}

struct Neighbour {
    bool free, occupied;
    int32_t slot, unit_type, owner;
};

// board.py:23-61.
inline Neighbour neighbour(const Game& g, const Content& c, const Extents& x, int32_t cell, int32_t direction) {
    const int32_t px = floor_mod(cell, x.width), py = floor_div(cell, x.width);
    const int d = clip(direction, 0, kDirections - 1);
    const int32_t nx = px + kDx[d], ny = py + kDy[d];
    const bool is_direction = direction >= 0 && direction < kDirections;
    const bool on_board = is_direction && nx >= 0 && nx < x.width && ny >= 0 && ny < x.height;
    const int32_t ncell = on_board ? ny * x.width + nx : 0;
    const int32_t occupant = g.entity_at[ncell];
    Neighbour n;
    n.occupied = on_board && occupant != kAbsent;
    n.slot = n.occupied ? occupant : 0;
    n.free = on_board && occupant == kAbsent && !c.terrain[ncell];
    n.unit_type = clip(g.unit_type[n.slot], 0, x.types - 1);
    n.owner = g.owner[n.slot];
    return n;
}

// admission.py:443-452 with kinds/*.py `_duration`.
inline int32_t action_duration(const Content& c, const Extents& x, int32_t actor_type, int32_t kind, int32_t none_duration, int32_t produced_type) {
    const int32_t actor = clip(actor_type, 0, x.types - 1);
    switch (kind) {
        case kKindNone: return none_duration;
        case kKindMove: return c.at(actor, kMoveTime);
        case kKindHarvest: return c.at(actor, kHarvestTime);
        case kKindReturn: return c.at(actor, kMoveTime);
        case kKindProduce: return c.at(clip(produced_type, 0, x.types - 1), kProduceTime);
        case kKindAttack: return c.at(actor, kAttackTime);
        default: return 0;
    }
}

// kinds/*.py `_is_valid` for one slot (admission.py:455-462).
inline bool can_execute(const Game& g, const Content& c, const Extents& x, int32_t slot, int32_t kind, int32_t direction, int32_t target_cell, int32_t produced_type) {
    const int32_t actor = clip(g.unit_type[slot], 0, x.types - 1);
    const int32_t owner = g.owner[slot];
    const int32_t carried = g.carried[slot];
    const int32_t cell = g.cell[slot];
    switch (kind) {
        case kKindNone: return true;
        case kKindMove: {  // move.py:15-16
            const Neighbour n = neighbour(g, c, x, cell, direction);
            return c.at(actor, kCanMove) && n.free;
        }
        case kKindHarvest: {  // harvest.py:14-21
            const Neighbour n = neighbour(g, c, x, cell, direction);
            return c.at(actor, kCanHarvest) && carried == 0 && n.occupied && c.at(n.unit_type, kIsResource);
        }
        case kKindReturn: {  // return_.py:15-23
            const Neighbour n = neighbour(g, c, x, cell, direction);
            return c.at(actor, kCanHarvest) && carried > 0 && n.occupied && c.at(n.unit_type, kIsStockpile) && n.owner == owner;
        }
        case kKindProduce: {  // produce.py:25-35
            const Neighbour n = neighbour(g, c, x, cell, direction);
            const int32_t balance = g.player_resources[clip(owner, 0, kPlayers - 1)];
            const int32_t known = clip(produced_type, 0, x.types - 1);
            return produced_type >= 0 && produced_type < x.types && c.produces(actor, known) && balance >= c.at(known, kCost) && n.free;
        }
        case kKindAttack: {  // attack.py:34-55
            const bool on_board = target_cell >= 0 && target_cell < x.cells();
            const int32_t target_slot = g.entity_at[on_board ? target_cell : 0];
            const bool holds_unit = on_board && target_slot != kAbsent;
            const int32_t target_owner = holds_unit ? g.owner[target_slot] : kAbsent;
            const int32_t range = c.at(actor, kAttackRange);
            const int32_t dx = floor_mod(target_cell, x.width) - floor_mod(cell, x.width);
            const int32_t dy = floor_div(target_cell, x.width) - floor_div(cell, x.width);
            return c.at(actor, kCanAttack) && target_owner >= 0 && target_owner != owner && dx * dx + dy * dy <= range * range;
        }
        default: return false;
    }
}

struct Reservation {
    bool claims_position;
    int32_t position, cost, player;
};

// admission.py:465-479.
inline Reservation reservation(const Content& c, const Extents& x, int32_t cell, int32_t owner, int32_t kind, int32_t direction, int32_t produced_type, bool has_action) {
    Reservation r;
    r.cost = (has_action && kind == kKindProduce) ? c.at(clip(produced_type, 0, x.types - 1), kCost) : 0;
    r.claims_position = has_action && (kind == kKindMove || kind == kKindProduce);
    r.position = reserved_position(cell, direction, x);
    r.player = clip(owner, 0, kPlayers - 1);
    return r;
}

// reservations.py:122-135.
inline bool reservations_conflict(const Reservation& existing, const Reservation& requested, const int32_t* balance) {
    const bool shared = existing.claims_position && requested.claims_position && existing.position == requested.position;
    const int32_t same = existing.player == requested.player ? existing.cost : 0;
    const int32_t claimed = same + requested.cost;
    const bool over = requested.cost != 0 && claimed > 0 && claimed > balance[requested.player];
    return shared || over;
}

// Masked single-slot write, like residue.masked_set (residue.py:24-26).
template <typename T, typename V>
inline void masked_set(T* field, int32_t size, int32_t index, bool when, V value) {
    if (when && index >= 0 && index < size) field[index] = static_cast<T>(value);
}

inline void clear_pending(Game& g, int32_t s) {  // pending.py:70-76 canonical empties
    g.pending_kind[s] = kAbsent;
    g.pending_direction[s] = kAbsent;
    g.pending_none_duration[s] = 0;
    g.pending_target_cell[s] = kAbsent;
    g.pending_produced_type[s] = kAbsent;
    g.pending_issued_at[s] = 0;
    g.pending_completes_at[s] = 0;
    g.pending_order[s] = kAbsent;
}

inline void remove_unit(Game& g, int32_t s) {  // units.py:22-31: every PER_SLOT leaf to its empty
    g.birth[s] = kAbsent;
    g.unit_type[s] = kAbsent;
    g.owner[s] = kAbsent;
    g.cell[s] = kAbsent;
    g.hit_points[s] = 0;
    g.carried[s] = 0;
    clear_pending(g, s);
}

// ---------------------------------------------------------------------------
// Admission (admission.py:48-156) with reservations.resolve (reservations.py:69-306).
// ---------------------------------------------------------------------------
struct Step {
    const Extents& x;
    const Content& c;
    Game& g;
    const Commands& cmd;
    Key key;

    std::vector<int32_t> ranking;  // pending.ranking: slot at each pending rank

    // StepEvents admission counts (model/step.py:24-33, admission.py:273-296):
    // requests per player whose kind after the legality and blocking checks is
    // HARVEST, RETURN, PRODUCE (by clipped produced type) or ATTACK (by the
    // owner + 1 of the target cell's occupant, -1 for none).
    int32_t admitted_harvest[kPlayers] = {0, 0};
    int32_t admitted_return[kPlayers] = {0, 0};
    int32_t admitted_attack[kPlayers][kPlayers + 1] = {{0, 0, 0}, {0, 0, 0}};
    std::vector<int32_t> admitted_produce = std::vector<int32_t>(kPlayers * 8, 0);

    // admission.py:67-101 _ordered_requests.
    void ordered_requests(std::vector<int32_t>& order, std::vector<uint8_t>& issued_sorted, int32_t& issued_count) {
        const int32_t owned = x.owned();
        std::vector<int32_t> key_(owned), unit_order(owned);
        std::vector<uint8_t> issued(owned);
        int rank_bits = 1;
        {
            int v = x.capacity - 1, bits = 0;
            while (v > 0) { ++bits; v >>= 1; }
            rank_bits = std::max(1, bits);
        }
        issued_count = 0;
        for (int32_t p = 0; p < owned; ++p) {
            const bool active = g.active(x.neutral + p);
            issued[p] = active && cmd.kind[p] != kAbsent;
            issued_count += issued[p];
            unit_order[p] = active ? g.birth[x.neutral + p] : INT32_MAX;
            const int32_t ro = cmd.request_order[p];
            const int32_t rank = clip(ro == kAbsent ? 0 : ro, 0, (1 << rank_bits) - 1);
            key_[p] = ((issued[p] ? 0 : 1) << (rank_bits + 1)) | ((p / x.capacity) << rank_bits) | rank;
        }
        order.resize(owned);
        std::iota(order.begin(), order.end(), 0);
        std::sort(order.begin(), order.end(), [&](int32_t a, int32_t b) {
            if (key_[a] != key_[b]) return key_[a] < key_[b];
            if (unit_order[a] != unit_order[b]) return unit_order[a] < unit_order[b];
            return a < b;
        });
        issued_sorted.resize(owned);
        for (int32_t k = 0; k < owned; ++k) issued_sorted[k] = issued[order[k]];
    }

    // pending.py:17-44 ranking.
    void pending_ranking(const std::vector<int32_t>& order, const std::vector<uint8_t>& issued_sorted) {
        const int32_t owned = x.owned();
        std::vector<int32_t> keys(owned);
        for (int32_t i = 0; i < owned; ++i) {
            const int32_t held = g.pending_order[x.neutral + i];
            keys[i] = held == kAbsent ? INT32_MAX : held;
        }
        int32_t appended_before = 0;
        std::vector<int32_t> new_keys = keys;
        for (int32_t k = 0; k < owned; ++k) {
            const int32_t local = order[k];
            const bool appends = issued_sorted[k] && g.pending_order[x.neutral + local] == kAbsent;
            const int32_t appended_order = *g.next_pending_order + appended_before;
            appended_before += appends;
            new_keys[local] = appends ? appended_order : keys[local];
        }
        std::vector<int32_t> pos(owned);
        std::iota(pos.begin(), pos.end(), 0);
        std::sort(pos.begin(), pos.end(), [&](int32_t a, int32_t b) {
            if (new_keys[a] != new_keys[b]) return new_keys[a] < new_keys[b];
            return a < b;
        });
        ranking.resize(x.entities());
        for (int32_t s = 0; s < x.neutral; ++s) ranking[s] = s;
        for (int32_t i = 0; i < owned; ++i) ranking[x.neutral + i] = x.neutral + pos[i];
    }

    // reservations.py:69-111 resolve; returns (kind, none_duration) of the request.
    void resolve(int32_t slot, const Reservation& request, int32_t request_duration, int32_t& kind, int32_t& none_duration) {
        const int32_t E = x.entities();
        const int32_t time = *g.time;
        // Entries in pending order (_in_pending_order).
        std::vector<int32_t> same(E), cross(E), duration(E);
        for (int32_t i = 0; i < E; ++i) {
            const int32_t s = ranking[i];
            const bool has = g.pending_kind[s] != kAbsent;
            const Reservation existing = reservation(c, x, g.cell[s], g.owner[s], g.pending_kind[s], g.pending_direction[s], g.pending_produced_type[s], has);
            const bool conflicts = has && reservations_conflict(existing, request, g.player_resources);
            const bool cross_cycle = g.pending_issued_at[s] != time;
            same[i] = conflicts && !cross_cycle;
            cross[i] = conflicts && cross_cycle;
            duration[i] = action_duration(c, x, g.unit_type[s], g.pending_kind[s], g.pending_none_duration[s], g.pending_produced_type[s]);
        }
        // _running_conflict_counts: inclusive prefix sums.
        std::vector<int32_t> same_before(E), cross_before(E);
        int32_t same_run = 0, cross_run = 0;
        for (int32_t i = 0; i < E; ++i) {
            same_before[i] = same_run;
            cross_before[i] = cross_run > 0;
            same_run += same[i];
            cross_run += cross[i];
        }
        const int32_t same_total = same_run;
        const bool any_cross = cross_run > 0;
        // _consumed_draws (CANCEL_RANDOM only).
        std::vector<int32_t> draws;
        if (x.strategy == kStrategyRandom) {
            const Key event = conflict_event_key(key, time, g.birth[slot]);
            draws.resize(std::max(same_total, 1));
            for (int32_t j = 0; j < same_total; ++j) draws[j] = randint01(fold_in(event, static_cast<uint32_t>(j)));
        }
        // _cancelled_sides.
        std::vector<uint8_t> cancels_request(E), cancels_pending(E);
        for (int32_t i = 0; i < E; ++i) {
            bool req = true, pend = true;
            if (x.strategy == kStrategyAlternating) {
                req = ((*g.alternating_conflict_count + same_before[i]) % 2) == 0;
                pend = !req;
            } else if (x.strategy == kStrategyRandom) {
                const int32_t ordinal = same_before[i];
                req = (ordinal < static_cast<int32_t>(draws.size()) ? draws[ordinal] : 0) == 0;
                pend = !req;
            }
            cancels_request[i] = req;
            cancels_pending[i] = pend;
        }
        // _settle_durations.
        std::vector<int32_t> caps(E), pending_duration(E);
        int32_t running = kNoCap;
        for (int32_t i = 0; i < E; ++i) {
            const bool cancels_request_at = same[i] && cancels_request[i];
            running = std::min(running, cancels_request_at ? duration[i] : kNoCap);
            caps[i] = running;
        }
        for (int32_t i = 0; i < E; ++i) {
            const int32_t before = cross_before[i] ? -1 : (i == 0 ? request_duration : std::min(request_duration, caps[i - 1]));
            pending_duration[i] = std::min(duration[i], before);
        }
        const bool request_cancelled = any_cross || caps[E - 1] != kNoCap;
        const int32_t final_duration = any_cross ? -1 : std::min(request_duration, caps[E - 1]);
        // _back_in_slot_order + _cancel_pending.
        for (int32_t i = 0; i < E; ++i) {
            if (!(same[i] && cancels_pending[i])) continue;
            const int32_t s = ranking[i];
            g.pending_kind[s] = kKindNone;
            g.pending_direction[s] = kAbsent;
            g.pending_none_duration[s] = pending_duration[i];
            g.pending_target_cell[s] = kAbsent;
            g.pending_produced_type[s] = kAbsent;
            g.pending_completes_at[s] = g.pending_issued_at[s] + pending_duration[i];
        }
        if (x.strategy == kStrategyAlternating) *g.alternating_conflict_count += same_total;
        if (request_cancelled) {
            kind = kKindNone;
            none_duration = final_duration;
        }
    }

    // admission.py:109-156 _admit_one.
    void admit_one(int32_t player, int32_t local, int32_t slot) {
        const int32_t p = player * x.capacity + local;
        const int32_t ckind = cmd.kind[p], cdir = cmd.direction[p], cnone = cmd.none_duration[p];
        const int32_t ctarget = cmd.target_cell[p], cptype = cmd.produced_type[p];
        const bool issued = g.active(slot) && ckind != kAbsent;
        const int32_t requested = action_duration(c, x, g.unit_type[slot], ckind, cnone, cptype);
        // _none_if_illegal
        const bool legal = can_execute(g, c, x, slot, ckind, cdir, ctarget, cptype);
        int32_t kind = legal ? ckind : kKindNone;
        int32_t none_duration = legal ? cnone : requested;
        // _none_if_blocked
        const bool claims = kind == kKindMove || kind == kKindProduce;
        const int32_t reserved = reserved_position(g.cell[slot], cdir, x);
        const bool blocked = claims && (c.terrain[gather(reserved, x.cells())] || g.entity_at[gather(reserved, x.cells())] != kAbsent);
        if (blocked) {
            kind = kKindNone;
            none_duration = requested;
        }
        if (issued) {  // _count_admitted (admission.py:273-307)
            if (kind == kKindHarvest) ++admitted_harvest[player];
            if (kind == kKindReturn) ++admitted_return[player];
            if (kind == kKindProduce) ++admitted_produce[player * 8 + clip(cptype, 0, x.types - 1)];
            if (kind == kKindAttack) {
                const int32_t occupant = g.entity_at[clip(ctarget, 0, x.cells() - 1)];
                const int32_t owner = occupant == kAbsent ? kAbsent : g.owner[clip(occupant, 0, x.entities() - 1)];
                if (owner >= -1 && owner <= 1) ++admitted_attack[player][owner + 1];
            }
        }
        const Reservation request = reservation(c, x, g.cell[slot], g.owner[slot], kind, cdir, cptype, issued);
        resolve(slot, request, requested, kind, none_duration);
        const int32_t duration = kind == kKindNone ? none_duration : requested;
        // _assign_pending_action (admission.py:241-270)
        if (issued) {
            const int32_t held = g.pending_order[slot];
            const bool appends = held == kAbsent;
            const int32_t order = appends ? *g.next_pending_order : held;
            const bool keeps_direction = kind == kKindMove || kind == kKindHarvest || kind == kKindReturn || kind == kKindProduce;
            g.pending_kind[slot] = static_cast<int8_t>(kind);
            g.pending_direction[slot] = static_cast<int8_t>(keeps_direction ? cdir : kAbsent);
            g.pending_none_duration[slot] = kind == kKindNone ? none_duration : 0;
            g.pending_target_cell[slot] = static_cast<int16_t>(kind == kKindAttack ? ctarget : kAbsent);
            g.pending_produced_type[slot] = static_cast<int8_t>(kind == kKindProduce ? cptype : kAbsent);
            g.pending_issued_at[slot] = *g.time;
            g.pending_completes_at[slot] = *g.time + duration;
            g.pending_order[slot] = order;
            *g.next_pending_order += appends ? 1 : 0;
        }
    }

    void admit() {
        std::vector<int32_t> order;
        std::vector<uint8_t> issued_sorted;
        int32_t issued_count = 0;
        ordered_requests(order, issued_sorted, issued_count);
        pending_ranking(order, issued_sorted);
        for (int32_t k = 0; k < issued_count; ++k) {
            const int32_t position = order[k];
            admit_one(position / x.capacity, position % x.capacity, x.neutral + position);
        }
    }

    // -----------------------------------------------------------------------
    // Completion (completion.py:30-79) with kinds/*.py `_complete`.
    // -----------------------------------------------------------------------
    struct Retained {
        int32_t kind, direction, target_cell, produced_type, birth, owner, unit_type, cell, carried;
    };

    void complete() {
        const int32_t E = x.entities();
        const int32_t time = *g.time;  // already advanced by pending.select
        std::vector<uint8_t> completed(E);
        std::vector<Retained> retained(E);
        for (int32_t s = 0; s < E; ++s) {
            completed[s] = g.pending_kind[s] != kAbsent && g.pending_completes_at[s] <= time;
            retained[s] = Retained{g.pending_kind[s], g.pending_direction[s], g.pending_target_cell[s], g.pending_produced_type[s],
                                   g.birth[s], g.owner[s], g.unit_type[s], g.cell[s], g.carried[s]};
        }
        // pending.batch_order (pending.py:55-60): acting owned slots by pending_order.
        std::vector<int32_t> members;
        for (int32_t s = x.neutral; s < E; ++s) {
            if (completed[s] && g.pending_kind[s] != kKindNone) members.push_back(s);
        }
        std::stable_sort(members.begin(), members.end(), [&](int32_t a, int32_t b) { return g.pending_order[a] < g.pending_order[b]; });
        for (int32_t s = 0; s < E; ++s) {
            if (completed[s]) clear_pending(g, s);
        }
        for (int32_t slot : members) take_turn(slot, retained[slot], completed[slot]);
    }

    // completion.py:58-79.
    void take_turn(int32_t slot, const Retained& r, bool in_batch) {
        const int32_t cells = x.cells();
        const int32_t E = x.entities();
        const int32_t actor = clip(r.unit_type, 0, x.types - 1);
        const int32_t player = clip(r.owner, 0, kPlayers - 1);
        const bool alive = g.active(slot) && g.birth[slot] == r.birth;
        const int32_t destination = reserved_position(r.cell, r.direction, x);
        const Neighbour nb = neighbour(g, c, x, r.cell, r.direction);
        auto performs = [&](int k) { return in_batch && r.kind == k; };

        bool removes = false;
        int32_t removed_slot = 0;

        if (performs(kKindMove)) {  // move.py:24-32
            const bool moving = alive;
            masked_set(g.entity_at, cells, destination, moving, slot);
            masked_set(g.entity_at, cells, r.cell, moving, kAbsent);
            masked_set(g.cell, E, slot, moving, destination);
        } else if (performs(kKindHarvest)) {  // harvest.py:30-58
            const bool harvesting = nb.occupied && c.at(nb.unit_type, kIsResource);
            const int32_t amount = c.at(actor, kHarvestAmount);
            const int32_t left = g.carried[nb.slot] - amount;
            const bool depleted = harvesting && left <= 0;
            masked_set(g.carried, E, nb.slot, harvesting, left);
            masked_set(g.carried, E, slot, harvesting && alive, amount);
            if (depleted) { removes = true; removed_slot = nb.slot; }
        } else if (performs(kKindReturn)) {  // return_.py:31-59
            const bool returning = nb.occupied && c.at(nb.unit_type, kIsStockpile) && r.carried > 0;
            const int32_t credit = returning ? r.carried : 0;
            const int32_t balance = g.player_resources[player] + credit;
            masked_set(g.carried, E, slot, returning && alive, 0);
            masked_set(g.player_resources, kPlayers, player, returning, balance);
        } else if (performs(kKindProduce)) {  // produce.py:49-89
            const int32_t newborn_type = clip(r.produced_type, 0, x.types - 1);
            const int32_t balance = g.player_resources[player] - c.at(newborn_type, kCost);
            const bool affordable = balance >= 0;
            // units.py:12-19 lowest_free_slot
            const int32_t start = x.neutral + player * x.capacity;
            int32_t newborn = 0;
            bool has_free = false;
            for (int32_t s = 0; s < E; ++s) {
                if (s >= start && s < start + x.capacity && !g.active(s)) { newborn = s; has_free = true; break; }
            }
            const bool spawns = affordable && has_free;
            const bool overflows = affordable && !has_free;
            masked_set(g.player_resources, kPlayers, player, spawns, balance);
            masked_set(g.entity_at, cells, destination, spawns, newborn);
            if (spawns) {
                g.birth[newborn] = *g.next_birth;
                g.unit_type[newborn] = static_cast<int8_t>(newborn_type);
                g.owner[newborn] = static_cast<int8_t>(player);
                g.cell[newborn] = static_cast<int16_t>(destination);
                g.hit_points[newborn] = static_cast<int16_t>(c.at(newborn_type, kHitPoints));
                *g.next_birth += 1;
            }
            if (overflows) g.spawn_overflow[player] += 1;
        } else if (performs(kKindAttack)) {  // attack.py:78-102
            const int32_t occupant = g.entity_at[clip(r.target_cell, 0, cells - 1)];
            const bool hit = occupant != kAbsent;
            const int32_t victim = hit ? occupant : 0;
            const int32_t left = static_cast<int32_t>(g.hit_points[victim]) - c.at(actor, kAttackDamage);
            masked_set(g.hit_points, E, victim, hit, left);
            if (hit && left <= 0) { removes = true; removed_slot = victim; }
        }
        if (removes) {
            // completion.py:67 then units.remove.
            masked_set(g.entity_at, cells, static_cast<int32_t>(g.cell[removed_slot]), true, kAbsent);
            remove_unit(g, removed_slot);
        }
    }
};

// outcome.py:11-19.
inline void decide(Game& g, const Extents& x) {
    bool surviving[kPlayers];
    int count = 0;
    for (int p = 0; p < kPlayers; ++p) {
        surviving[p] = false;
        for (int32_t i = 0; i < x.capacity; ++i) surviving[p] |= g.active(x.neutral + p * x.capacity + i);
        count += surviving[p];
    }
    *g.game_over = count <= 1;
    int first = 0;
    while (first < kPlayers - 1 && !surviving[first]) ++first;
    *g.winner = count == 1 ? first : kAbsent;
}

struct StepOutcome {
    bool terminated, truncated;
    float reward[kPlayers];
    float components[kPlayers][6];  // encode_components (adapters/rewards.py:47-72)
};

constexpr int kTypeBaseIdx = 1, kTypeBarracksIdx = 2, kTypeWorkerIdx = 3, kTypeLightIdx = 4, kTypeHeavyIdx = 5,
              kTypeRangedIdx = 6;

// core/__init__.py:99-110 _t1_step.
inline StepOutcome core_step(Game& g, const Content& c, const Extents& x, const Commands& cmd, Key key) {
    Step step{x, c, g, cmd, key, {}};
    step.admit();
    *g.time = static_cast<int32_t>(static_cast<uint32_t>(*g.time) + 1u);  // pending.select
    step.complete();
    decide(g, x);
    StepOutcome out;
    out.terminated = *g.game_over != 0;
    out.truncated = !*g.game_over && *g.time >= x.max_cycles;  // outcome.py:28-29
    const bool ended = out.terminated || out.truncated;
    for (int p = 0; p < kPlayers; ++p) out.reward[p] = ended ? (p == *g.winner ? 1.0f : -1.0f) : 0.0f;
    // adapters/rewards.py:47-72 (order: win_loss, resource_gather, produce_worker,
    // produce_building, attack, produce_combat_unit).
    for (int p = 0; p < kPlayers; ++p) {
        const int opponent = (p + 1) % kPlayers;
        const int32_t* produced = &step.admitted_produce[p * 8];
        out.components[p][0] = *g.game_over ? (*g.winner == p ? 1.0f : -1.0f) : 0.0f;
        out.components[p][1] = static_cast<float>(step.admitted_harvest[p] + step.admitted_return[p]);
        out.components[p][2] = static_cast<float>(produced[kTypeWorkerIdx]);
        out.components[p][3] = static_cast<float>(produced[kTypeBaseIdx] + produced[kTypeBarracksIdx]);
        out.components[p][4] = static_cast<float>(step.admitted_attack[p][opponent + 1] - step.admitted_attack[p][p + 1]);
        out.components[p][5] = static_cast<float>(produced[kTypeLightIdx] + produced[kTypeHeavyIdx] + produced[kTypeRangedIdx]);
    }
    return out;
}

// adapters/jaxmarl/actions.py:61-84 decode_actions (+ adapters/factors.py:117-151).
inline Commands decode_actions(const Game& g, const Extents& x, const int32_t* const actions[kPlayers]) {
    Commands cmd(x.owned());
    const int side = x.side(), radius = x.radius();
    for (int p = 0; p < kPlayers; ++p) {
        for (int32_t i = 0; i < x.capacity; ++i) {
            const int32_t slot = x.neutral + p * x.capacity + i;
            const int32_t* row = actions[p] + static_cast<int64_t>(i) * 7;
            const bool available = g.active(slot) && g.pending_kind[slot] == kAbsent;
            if (!available) continue;
            const int32_t kind = row[0];
            const int32_t k = p * x.capacity + i;
            cmd.kind[k] = kind;
            cmd.direction[k] = kind == kKindMove ? row[1] : kind == kKindHarvest ? row[2] : kind == kKindReturn ? row[3] : kind == kKindProduce ? row[4] : kAbsent;
            cmd.produced_type[k] = kind == kKindProduce ? row[5] : kAbsent;
            const int32_t cell = g.cell[slot];
            const int32_t tx = floor_mod(cell, x.width) + (floor_mod(row[6], side) - radius);
            const int32_t ty = floor_div(cell, x.width) + (floor_div(row[6], side) - radius);
            const bool on_board = tx >= 0 && tx < x.width && ty >= 0 && ty < x.height;
            cmd.target_cell[k] = (kind == kKindAttack && on_board) ? ty * x.width + tx : kAbsent;
            cmd.none_duration[k] = kind == kKindNone ? 1 : 0;
        }
    }
    return cmd;
}

// core/legality.py:32-64 derive + kinds/*.py `_legality`, concatenated by
// factors.concatenated and masked by availability (actions.py:28-41).
inline void legal_rows(const Game& g, const Content& c, const Extents& x, uint8_t* const masks[kPlayers]) {
    const int32_t width = x.mask_width();
    const int side = x.side(), radius = x.radius();
    for (int p = 0; p < kPlayers; ++p) {
        for (int32_t i = 0; i < x.capacity; ++i) {
            const int32_t slot = x.neutral + p * x.capacity + i;
            uint8_t* row = masks[p] + static_cast<int64_t>(i) * width;
            std::memset(row, 0, width);
            const bool active = g.active(slot);
            const bool available = active && g.pending_kind[slot] == kAbsent;
            if (!available) {
                row[0] = 1;  // only KIND_NONE
                continue;
            }
            const int32_t actor = clip(g.unit_type[slot], 0, x.types - 1);
            const int32_t owner = g.owner[slot];
            const int32_t carried = g.carried[slot];
            const int32_t cell = g.cell[slot];
            const int32_t balance = g.player_resources[clip(owner, 0, kPlayers - 1)];
            uint8_t* kind = row;
            uint8_t* move = row + kKinds;
            uint8_t* harvest = move + kDirections;
            uint8_t* ret = harvest + kDirections;
            uint8_t* pdir = ret + kDirections;
            uint8_t* ptype = pdir + kDirections;
            uint8_t* attack = ptype + x.types;
            for (int d = 0; d < kDirections; ++d) {
                const Neighbour n = neighbour(g, c, x, cell, d);
                move[d] = c.at(actor, kCanMove) && n.free;
                harvest[d] = c.at(actor, kCanHarvest) && carried == 0 && n.occupied && c.at(n.unit_type, kIsResource);
                ret[d] = c.at(actor, kCanHarvest) && carried > 0 && n.occupied && c.at(n.unit_type, kIsStockpile) && n.owner == owner;
                for (int t = 0; t < x.types; ++t) {
                    const bool valid = c.produces(actor, t) && balance >= c.at(t, kCost) && n.free;
                    pdir[d] |= valid;
                    ptype[t] |= valid;
                }
            }
            // attack.py:57-75: owner of each window cell (off-board and empty cells are neutral).
            const int32_t range = c.at(actor, kAttackRange);
            const int32_t ax = floor_mod(cell, x.width), ay = floor_div(cell, x.width);
            bool any_attack = false;
            for (int o = 0; o < x.offsets; ++o) {
                const int32_t dx = o % side - radius, dy = o / side - radius;
                const int32_t tx = ax + dx, ty = ay + dy;
                int32_t target_owner = kAbsent;
                if (tx >= 0 && tx < x.width && ty >= 0 && ty < x.height) {
                    const int32_t occupant = g.entity_at[ty * x.width + tx];
                    if (occupant != kAbsent) target_owner = g.owner[occupant];
                }
                attack[o] = c.at(actor, kCanAttack) && target_owner >= 0 && target_owner != owner && dx * dx + dy * dy <= range * range;
                any_attack |= attack[o];
            }
            bool any_move = false, any_harvest = false, any_return = false, any_produce = false;
            for (int d = 0; d < kDirections; ++d) {
                any_move |= move[d];
                any_harvest |= harvest[d];
                any_return |= ret[d];
                any_produce |= pdir[d];
            }
            kind[kKindNone] = 1;
            kind[kKindMove] = any_move;
            kind[kKindHarvest] = any_harvest;
            kind[kKindReturn] = any_return;
            kind[kKindProduce] = any_produce;
            kind[kKindAttack] = any_attack;
        }
    }
}

// observations/visibility.py:70-77 _cells_by_test for one observer.
inline void visible_cells(const Game& g, const Content& c, const Extents& x, int player, std::vector<uint8_t>& seen) {
    seen.assign(x.cells(), 0);
    const int32_t start = x.neutral + player * x.capacity;
    for (int32_t s = start; s < start + x.capacity; ++s) {
        if (!g.active(s)) continue;
        const int32_t cell = g.cell[s];
        const int32_t r = c.at(clip(g.unit_type[s], 0, x.types - 1), kSightRadius);
        const int32_t ux = floor_mod(cell, x.width), uy = floor_div(cell, x.width);
        for (int32_t y = 0; y < x.height; ++y) {
            for (int32_t xx = 0; xx < x.width; ++xx) {
                const int32_t dx = xx - ux, dy = y - uy;
                if (dx * dx + dy * dy <= r * r) seen[y * x.width + xx] = 1;
            }
        }
    }
}

// observations/symbolic.py:130-180 _byte_feature_maps + scalar_vector.
inline void observe(const Game& g, const Content& c, const Extents& x, bool partial, uint8_t* const maps[kPlayers], int32_t* const scalars[kPlayers]) {
    const int32_t cells = x.cells();
    std::vector<uint32_t> word(cells);
    for (int32_t cell = 0; cell < cells; ++cell) {
        const int32_t s = g.entity_at[cell];
        if (s == kAbsent) { word[cell] = 0; continue; }
        const uint32_t hp = static_cast<uint32_t>(static_cast<int32_t>(g.hit_points[s])) & 0xFFu;
        const uint32_t carried = static_cast<uint32_t>(g.carried[s]) & 0xFFu;
        const uint32_t type = static_cast<uint32_t>(g.unit_type[s] + 1) & 0xFFu;
        const uint32_t pending = static_cast<uint32_t>(std::max<int32_t>(g.pending_kind[s], kKindNone)) & 0xFu;
        const uint32_t owner = static_cast<uint32_t>(g.owner[s] + 1) & 0x3u;
        word[cell] = hp | (carried << 8) | (type << 16) | (pending << 24) | (owner << 28);
    }
    std::vector<uint8_t> seen;
    for (int p = 0; p < kPlayers; ++p) {
        if (partial) visible_cells(g, c, x, p, seen);
        for (int32_t cell = 0; cell < cells; ++cell) {
            uint32_t w = word[cell];
            const uint32_t owner = (w >> 28) & 0x3u;
            if (partial && !(owner == static_cast<uint32_t>(p + 1) || seen[cell])) w = 0;
            const uint32_t o = (w >> 28) & 0x3u;
            uint8_t* out = maps[p] + static_cast<int64_t>(cell) * 6;
            out[0] = static_cast<uint8_t>(w & 0xFFu);
            out[1] = static_cast<uint8_t>((w >> 8) & 0xFFu);
            out[2] = static_cast<uint8_t>(o > 0 ? ((o - 1 + p) % kPlayers) + 1 : 0);
            out[3] = static_cast<uint8_t>((w >> 16) & 0xFFu);
            out[4] = static_cast<uint8_t>((w >> 24) & 0xFu);
            out[5] = c.terrain[cell] ? 1 : 0;
        }
        scalars[p][0] = g.player_resources[p];
        scalars[p][1] = g.player_resources[(p + 1) % kPlayers];
        scalars[p][2] = *g.time;
        scalars[p][3] = *g.alternating_conflict_count;
    }
}

}  // namespace oracle
