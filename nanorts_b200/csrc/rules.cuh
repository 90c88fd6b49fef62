// The game rules on a warp's slab: decode, admission with conflict
// resolution, completion and outcome.  Paths below are under src/nanorts/ of
// NanoRTS, whose JAX program these functions follow.
#pragma once

#include <cstdint>

#include "device.cuh"
#include "game.cuh"

namespace nrts {

// DIRECTION_OFFSETS (model/vocabulary.py): up, right, down, left.
__device__ __forceinline__ int dir_dx(int d) { return (d == 1) - (d == 3); }
__device__ __forceinline__ int dir_dy(int d) { return (d == 2) - (d == 0); }

// board.py:64-77: cell + (dx + dy * W) of the clipped direction.
template <int kW>
__device__ __forceinline__ int32_t reserved_position(const Geo<kW>& G, int32_t cell, int32_t direction) {
    const int d = clampi(direction, 0, kDirections - 1);
    return cell + dir_dx(d) + dir_dy(d) * G.width();
}

__device__ __forceinline__ bool claims_kind(int32_t kind) { return kind == kKindMove || kind == kKindProduce; }

__device__ __forceinline__ int8_t narrow8(int32_t v) { return static_cast<int8_t>(v); }

struct Neighbour {
    bool free, occupied;
    int32_t slot, unit_type, owner;
};

// board.py:23-61 for a cell index >= 0.
template <int kW>
__device__ __forceinline__ Neighbour neighbour(const Params& P, const Header& H, const Geo<kW>& G, const Game& g, int32_t cell,
                                               int32_t direction) {
    const int d = clampi(direction, 0, kDirections - 1);
    const int32_t nx = G.x(cell) + dir_dx(d), ny = G.y(cell) + dir_dy(d);
    const bool on_board = static_cast<uint32_t>(direction) < kDirections && nx >= 0 && nx < G.width() && ny >= 0 && ny < G.h;
    const int32_t ncell = on_board ? ny * G.width() + nx : 0;
    const int32_t occupant = g.entity_at[ncell];
    Neighbour n;
    n.occupied = on_board && occupant != kAbsent;
    n.slot = n.occupied ? occupant : 0;
    n.free = on_board && occupant == kAbsent && !((H.terrain_rows[on_board ? ny : 0] >> (on_board ? nx : 0)) & 1ull);
    n.unit_type = clampi(g.unit_type[n.slot], 0, P.types - 1);
    n.owner = g.owner[n.slot];
    return n;
}

// admission.py:443-452 with each kind's `_duration`.
__device__ __forceinline__ int32_t action_duration(const Params& P, const Header& H, int32_t unit_type, int32_t kind,
                                                   int32_t none_duration, int32_t produced_type) {
    const int32_t actor = clampi(unit_type, 0, P.types - 1);
    switch (kind) {
        case kKindNone: return none_duration;
        case kKindMove: return H.at(actor, kMoveTime);
        case kKindHarvest: return H.at(actor, kHarvestTime);
        case kKindReturn: return H.at(actor, kMoveTime);
        case kKindProduce: return H.at(clampi(produced_type, 0, P.types - 1), kProduceTime);
        case kKindAttack: return H.at(actor, kAttackTime);
        default: return 0;
    }
}

__device__ __forceinline__ int32_t kind_cost(const Params& P, const Header& H, int32_t kind, int32_t produced_type) {
    return kind == kKindProduce ? H.at(clampi(produced_type, 0, P.types - 1), kCost) : 0;
}

// Each kind's `_is_valid` (kinds/*.py) for an active slot.
template <int kW>
__device__ bool can_execute(const Params& P, const Header& H, const Geo<kW>& G, const Game& g, int32_t slot, int32_t kind,
                            int32_t direction, int32_t target_cell, int32_t produced_type) {
    const int32_t actor = clampi(g.unit_type[slot], 0, P.types - 1);
    const int32_t owner = g.owner[slot];
    const int32_t cell = g.cell[slot];
    switch (kind) {
        case kKindNone: return true;
        case kKindMove: return H.at(actor, kCanMove) && neighbour(P, H, G, g, cell, direction).free;
        case kKindHarvest: {
            const Neighbour n = neighbour(P, H, G, g, cell, direction);
            return H.at(actor, kCanHarvest) && g.carried[slot] == 0 && n.occupied && H.at(n.unit_type, kIsResource);
        }
        case kKindReturn: {
            const Neighbour n = neighbour(P, H, G, g, cell, direction);
            return H.at(actor, kCanHarvest) && g.carried[slot] > 0 && n.occupied && H.at(n.unit_type, kIsStockpile) &&
                   n.owner == owner;
        }
        case kKindProduce: {
            const int32_t balance = g.s[kSRes0 + clampi(owner, 0, kPlayers - 1)];
            const int32_t known = clampi(produced_type, 0, P.types - 1);
            return produced_type >= 0 && produced_type < P.types && H.produces(actor, known) && balance >= H.at(known, kCost) &&
                   neighbour(P, H, G, g, cell, direction).free;
        }
        case kKindAttack: {
            if (target_cell < 0 || target_cell >= G.cells) return false;
            const int32_t target_slot = g.entity_at[target_cell];
            if (target_slot == kAbsent) return false;
            const int32_t target_owner = g.owner[target_slot];
            const int32_t range = H.at(actor, kAttackRange);
            const int32_t dx = G.x(target_cell) - G.x(cell), dy = G.y(target_cell) - G.y(cell);
            return H.at(actor, kCanAttack) && target_owner >= 0 && target_owner != owner && dx * dx + dy * dy <= range * range;
        }
        default: return false;
    }
}

// One admission request, decided before the ordered loop: legality, blocking,
// durations and the claimed cell read only fields admission never changes.
// `duration` is the requested duration (admission.py:247-253) of a kind other
// than NONE, and the none duration of a request whose kind, after the
// legality and blocking rules, is NONE: only one of the two is ever read.
struct ReqInfo {
    int32_t duration;
    int16_t target;     // attack target cell or -1
    int16_t pos;        // reserved position (claimed cell when kind claims)
    int8_t kind;        // kind after the legality and blocking rules
    int8_t dir;         // canonical direction
    int8_t ptype;       // canonical produced type
    uint8_t serial;     // needs the ordered conflict loop
};
static_assert(sizeof(ReqInfo) == 12, "request info");

struct Retained {
    int32_t birth;
    int32_t carried;
    int16_t cell;
    int16_t target;
    int8_t kind, direction, produced_type, owner;
    int8_t unit_type;
    int8_t pad[3];
};
static_assert(sizeof(Retained) == 20, "packed retained actor");

// Claims per cell: a byte counter per cell, or (kTwoBit, for slabs short of
// room) a 2-bit saturating counter, 16 cells per word, whose bit 0 the first
// claim of a cell sets and bit 1 any later one.  Byte counters take one
// atomic per claim and measured faster where the room is there.
__host__ __device__ __forceinline__ int32_t claim_words(int32_t cells, bool two_bit) {
    return two_bit ? (cells + 15) >> 4 : (cells + 3) >> 2;
}

template <bool kTwoBit>
__device__ __forceinline__ void add_claim(uint32_t* counts, int32_t cells, int32_t pos) {
    if (pos < 0 || pos >= cells) return;
    if constexpr (kTwoBit) {
        const uint32_t shift = 2u * static_cast<uint32_t>(pos & 15);
        const uint32_t before = atomicOr(&counts[pos >> 4], 1u << shift);
        if ((before >> shift) & 1u) atomicOr(&counts[pos >> 4], 2u << shift);
    } else {
        atomicAdd(&counts[pos >> 2], 1u << (8 * (pos & 3)));
    }
}

// Whether more than one claim names cell `pos`.
template <bool kTwoBit>
__device__ __forceinline__ bool claimed_twice(const uint32_t* counts, int32_t cells, int32_t pos) {
    if (pos < 0 || pos >= cells) return false;
    if constexpr (kTwoBit) return (counts[pos >> 4] >> (2u * static_cast<uint32_t>(pos & 15) + 1u)) & 1u;
    else return ((counts[pos >> 2] >> (8 * (pos & 3))) & 0xffu) > 1u;
}

// Assigns a decided request's pending action (admission.py:241-270).
__device__ __forceinline__ void assign_pending(Game& g, int32_t slot, int32_t kind, int32_t none_duration, int32_t requested,
                                               int32_t dir, int32_t target, int32_t ptype, int32_t time, int32_t order) {
    const int32_t duration = kind == kKindNone ? none_duration : requested;
    const bool keeps_direction = kind == kKindMove || kind == kKindHarvest || kind == kKindReturn || kind == kKindProduce;
    g.pending_kind[slot] = narrow8(kind);
    g.pending_direction[slot] = narrow8(keeps_direction ? dir : kAbsent);
    g.pending_none_duration[slot] = kind == kKindNone ? none_duration : 0;
    g.pending_target_cell[slot] = static_cast<int16_t>(kind == kKindAttack ? target : kAbsent);
    g.pending_produced_type[slot] = narrow8(kind == kKindProduce ? ptype : kAbsent);
    g.pending_issued_at[slot] = time;
    g.pending_completes_at[slot] = static_cast<int32_t>(static_cast<uint32_t>(time) + static_cast<uint32_t>(duration));
    g.pending_order[slot] = order;
}

constexpr int kEventCounts = 5;

// One admitted request's share of the reward components: kind is the kind
// after the legality and blocking checks (admission.py:273-296).
__device__ __forceinline__ void count_event(const Params& P, const Game& g, int32_t* ev, int32_t player, int32_t kind,
                                            int32_t ptype, int32_t target) {
    if (kind == kKindHarvest || kind == kKindReturn) {
        atomicAdd(&ev[0], 1);
    } else if (kind == kKindProduce) {
        const int32_t t = clampi(ptype, 0, P.types - 1);
        if (t == 3) atomicAdd(&ev[1], 1);                      // TYPE_WORKER
        if (t == 1 || t == 2) atomicAdd(&ev[2], 1);            // TYPE_BASE, TYPE_BARRACKS
        if (t == 4 || t == 5 || t == 6) atomicAdd(&ev[4], 1);  // TYPE_LIGHT, TYPE_HEAVY, TYPE_RANGED
    } else if (kind == kKindAttack) {
        const int32_t occupant = g.entity_at[clampi(target, 0, P.cells - 1)];
        const int32_t owner = occupant == kAbsent ? kAbsent : g.owner[clampi(occupant, 0, P.entities - 1)];
        if (owner == 1 - player) atomicAdd(&ev[3], 1);
        else if (owner == player) atomicAdd(&ev[3], -1);
    }
}

// ---------------------------------------------------------------------------
// Admission (admission.py:48-156, reservations.py:69-306).
// ---------------------------------------------------------------------------
// The contested requests in Java order: conflict resolution against the claim
// holders (reservations.py:69-306), then the pending assignment.  `holders`
// claim holders are listed in `scan`; assigned claimers are appended.
template <int kW>
__device__ __forceinline__ void admit_contested(const Params& P, const Header& H, const Geo<kW>& G, Game& g, char* slab, int lane,
                                             int32_t S, int32_t holders) {
    const Layout& L = P.layout;
    const int32_t N = P.neutral, E = P.entities;
    const int32_t time = g.s[kSTime];
    const int16_t* list = reinterpret_cast<const int16_t*>(slab + L.list_off);
    const int16_t* order = reinterpret_cast<const int16_t*>(slab + L.order_off);
    const int16_t* serial = reinterpret_cast<const int16_t*>(slab + L.serial_off);
    int16_t* scan = reinterpret_cast<int16_t*>(slab + L.scan_off);
    int16_t* conf = reinterpret_cast<int16_t*>(slab + L.conf_off);
    const uint32_t* keys = reinterpret_cast<const uint32_t*>(slab + L.key_off);
    const ReqInfo* info = reinterpret_cast<const ReqInfo*>(slab + L.info_off);
    const int16_t* rank_of = reinterpret_cast<const int16_t*>(slab + L.rank_off);
    uint32_t k0 = 0, k1 = 0;
    if (P.strategy == 1) {  // episode_root = fold_in(environment_root, episode_index)
        k0 = static_cast<uint32_t>(g.s[kSRoot0]);
        k1 = static_cast<uint32_t>(g.s[kSRoot1]);
        fold_in(k0, k1, static_cast<uint32_t>(g.s[kSEpisode]));
    }
    for (int32_t c = 0; c < S; ++c) {
        const int32_t r = serial[c];
        const int32_t i = order[r];
        const int32_t slot = N + list[i];
        const ReqInfo q = info[i];
        const int32_t ord = static_cast<int32_t>(keys[i]);
        // Only a claiming or paying kind (never NONE) meets conflicts below,
        // so q.duration is its requested duration wherever `before` reads it.
        int32_t kind = q.kind, none = q.duration;
        const bool rclaims = claims_kind(kind);
        const int32_t rcost = kind_cost(P, H, kind, q.ptype);
        const int32_t rplayer = clampi(g.owner[slot], 0, kPlayers - 1);
        const int32_t balance = g.s[kSRes0 + rplayer];
        const bool every_holder = rcost > 0 && rcost > balance;
        auto conflicts = [&](int32_t s) {
            const int32_t pk = g.pending_kind[s];
            if (pk == kAbsent) return false;
            if (every_holder && s >= N && rank_of[s - N] > r) return false;  // decided later in Java order
            const bool shared = claims_kind(pk) && rclaims && reserved_position(G, g.cell[s], g.pending_direction[s]) == q.pos;
            const int32_t hcost = clampi(g.owner[s], 0, kPlayers - 1) == rplayer ? kind_cost(P, H, pk, g.pending_produced_type[s]) : 0;
            const int32_t claimed = hcost + rcost;
            return shared || (rcost != 0 && claimed > 0 && claimed > balance);
        };
        int32_t n = 0;
        if (every_holder) {
            n = warp_compact(E, lane, conf, conflicts);
        } else {
            for (int32_t base = 0; base < holders; base += 32) {
                const int32_t j = base + lane;
                const int32_t s = j < holders ? scan[j] : 0;
                const bool keep = j < holders && conflicts(s);
                const unsigned m = __ballot_sync(kFull, keep);
                if (keep) conf[n + __popc(m & lanes_below(lane))] = static_cast<int16_t>(s);
                n += __popc(m);
            }
            __syncwarp();
        }
        if (lane == 0) {
            if (n > 0) {
                // Pending order (pending.py:17-44): ascending pending_order.
                for (int32_t a = 1; a < n; ++a) {
                    const int16_t v = conf[a];
                    const int32_t key = g.pending_order[v];
                    int32_t b = a - 1;
                    while (b >= 0 && g.pending_order[conf[b]] > key) {
                        conf[b + 1] = conf[b];
                        --b;
                    }
                    conf[b + 1] = v;
                }
                uint32_t e0 = 0, e1 = 0;
                if (P.strategy == 1) {  // reservations.py:297-300
                    e0 = k0;
                    e1 = k1;
                    fold_in(e0, e1, static_cast<uint32_t>(time));
                    fold_in(e0, e1, static_cast<uint32_t>(g.birth[slot]));
                    fold_in(e0, e1, 0u);
                }
                int32_t same_before = 0;
                bool cross_seen = false;
                int32_t cap = kNoCap;
                const int32_t alt = g.s[kSAlt];
                for (int32_t a = 0; a < n; ++a) {
                    const int32_t e = conf[a];
                    if (g.pending_issued_at[e] != time) {  // cross-cycle conflict
                        cross_seen = true;
                        continue;
                    }
                    const int32_t dur = action_duration(P, H, g.unit_type[e], g.pending_kind[e], g.pending_none_duration[e],
                                                        g.pending_produced_type[e]);
                    bool cancels_request = true, cancels_pending = true;  // CANCEL_BOTH
                    if (P.strategy == 2) {  // CANCEL_ALTERNATING
                        cancels_request = ((alt + same_before) % 2) == 0;
                        cancels_pending = !cancels_request;
                    } else if (P.strategy == 1) {  // CANCEL_RANDOM
                        uint32_t d0 = e0, d1 = e1;
                        fold_in(d0, d1, static_cast<uint32_t>(same_before));
                        cancels_request = randint01(d0, d1) == 0;
                        cancels_pending = !cancels_request;
                    }
                    if (cancels_pending) {  // _settle_durations, _cancel_pending
                        const int32_t before = cross_seen ? -1 : min(q.duration, cap);
                        const int32_t settled = min(dur, before);
                        g.pending_kind[e] = kKindNone;
                        g.pending_direction[e] = kAbsent;
                        g.pending_none_duration[e] = settled;
                        g.pending_target_cell[e] = kAbsent;
                        g.pending_produced_type[e] = kAbsent;
                        g.pending_completes_at[e] = g.pending_issued_at[e] + settled;
                    }
                    if (cancels_request) cap = min(cap, dur);
                    ++same_before;
                }
                if (P.strategy == 2) g.s[kSAlt] = alt + same_before;
                if (cross_seen || cap != kNoCap) {
                    kind = kKindNone;
                    none = cross_seen ? -1 : min(q.duration, cap);
                }
            }
            assign_pending(g, slot, kind, none, q.duration, q.dir, q.target, q.ptype, time, ord);
            if (claims_kind(kind)) scan[holders] = static_cast<int16_t>(slot);
        }
        __syncwarp();
        if (claims_kind(g.pending_kind[slot])) ++holders;
        __syncwarp();
    }
}

// ---------------------------------------------------------------------------
// Admission (admission.py:48-156, reservations.py:69-306).
//
// Requests whose outcome cannot depend on another request are decided and
// assigned by the lanes in parallel: a request meets a conflict only through a
// pending holder that claims the same cell (MOVE and PRODUCE claim) or, for a
// PRODUCE, a same-player PRODUCE holder whose cost with its own exceeds the
// balance.  Requests claiming a cell that some other holder or request also
// claims, and PRODUCE requests of a player with several PRODUCE claims, run
// in Java order through the conflict resolution; the holders they can meet
// are the claim holders of the step's start and the contested requests already
// admitted.  A request whose own cost exceeds the balance conflicts with every
// holder (reservations.py:122-135) and scans every slot.
// ---------------------------------------------------------------------------
//
// kCmd: the requests are the slab's command rows a scripted bot wrote (kind,
// direction, none_duration, target cell, produced type and an explicit rank
// per owned slot) instead of action rows.  Admission orders requests by
// player, rank, birth (admission.py:67-115); Commands hold, per player, either
// no ranks or a permutation of ranks (model/commands.py:37-66), so the key
// (player, rank) or (player, birth) orders them alike.  Bots issue commands
// only to available units, the slots this pass scans.  kTwoBit: the
// layout's claim counters are 2-bit (the compact layout of wide boards).
// kHbmRows: the rules-only rows stay in HBM, so the holders' directions are
// read after the pass, one load per holder at once, instead of inside it.
template <int kW, bool kCmd = false, bool kTwoBit = false, bool kHbmRows = false>
__device__ void admit(const Params& P, const Header& H, const Geo<kW>& G, Game& g, char* slab, int64_t game, int lane) {
    const Layout& L = P.layout;
    const int32_t N = P.neutral, C = P.capacity, E = P.entities;
    const int32_t time = g.s[kSTime];
    int16_t* list = reinterpret_cast<int16_t*>(slab + L.list_off);
    int16_t* order = reinterpret_cast<int16_t*>(slab + L.order_off);
    int16_t* scan = reinterpret_cast<int16_t*>(slab + L.scan_off);
    uint32_t* keys = reinterpret_cast<uint32_t*>(slab + L.key_off);
    ReqInfo* info = reinterpret_cast<ReqInfo*>(slab + L.info_off);
    int16_t* rank_of = reinterpret_cast<int16_t*>(slab + L.rank_off);
    uint32_t* counts = reinterpret_cast<uint32_t*>(slab + L.count_off);
    const int32_t count_words = claim_words(G.cells, kTwoBit);
    uint32_t* produce_claims = counts + count_words;

    // Reward-component counts (admission.py:273-296 as adapters/rewards.py:47-72
    // combines them), per player: gathered, workers, buildings, attacks on the
    // opponent minus attacks on own units, combat units.
    int32_t* events = reinterpret_cast<int32_t*>(produce_claims + 2);
    const bool counting = P.out.reward_components != nullptr;
    for (int32_t i = lane; 4 * i < count_words + 2 + 2 * kEventCounts; i += 32)  // the region is 16-byte aligned and padded
        reinterpret_cast<uint4*>(counts)[i] = make_uint4(0u, 0u, 0u, 0u);
    __syncwarp();
    // One pass over the slots: available owned slots (actions.py:65-75,
    // legality.py:169-170) and the claim holders at the step's start.
    int32_t A = 0, holders = 0;
    for (int32_t base = 0; base < E; base += 32) {
        const int32_t s = base + lane;
        const bool in = s < E;
        const int32_t pk = in ? g.pending_kind[s] : kAbsent;
        const bool available = in && s >= N && pk == kAbsent && g.birth[s] != kAbsent;
        const bool holds = in && claims_kind(pk);
        const unsigned ma = __ballot_sync(kFull, available);
        const unsigned mh = __ballot_sync(kFull, holds);
        if (available) list[A + __popc(ma & lanes_below(lane))] = static_cast<int16_t>(s - N);
        if (holds) {
            scan[holders + __popc(mh & lanes_below(lane))] = static_cast<int16_t>(s);
            if constexpr (!kHbmRows) add_claim<kTwoBit>(counts, G.cells, reserved_position(G, g.cell[s], g.pending_direction[s]));
            if (pk == kKindProduce) atomicAdd(&produce_claims[clampi(g.owner[s], 0, kPlayers - 1)], 1u);
        }
        if (in && s >= N) rank_of[s - N] = -1;
        A += __popc(ma);
        holders += __popc(mh);
    }
    __syncwarp();
    if constexpr (kHbmRows) {  // the holders' claimed cells, from the list
        for (int32_t j = lane; j < holders; j += 32) {
            const int32_t s = scan[j];
            add_claim<kTwoBit>(counts, G.cells, reserved_position(G, g.cell[s], g.pending_direction[s]));
        }
        __syncwarp();
    }
    // Decode every available slot's row (actions.py:61-84) and decide the issued
    // ones in parallel; a row whose kind is absent issues nothing.
    int32_t R = 0;
    for (int32_t base = 0; base < A; base += 32) {
        const int32_t i = base + lane;
        bool issued = false;
        if (i < A) {
            const int32_t p = list[i];
            const int32_t slot = N + p;
            const int32_t player = p >= C, local = p - player * C;
            // Canonical forms decide exactly like the raw values: kinds outside
            // [-1, 5] are unknown (duration 0, never legal), directions outside
            // [0, 3] are off the board, produced types are only clipped or range-checked.
            auto decide_request = [&](int32_t raw, int32_t raw_dir, int32_t raw_type, int32_t target, int32_t cnone, int32_t cell) {
                const int32_t ckind = (raw >= kAbsent && raw <= kKindAttack) ? raw : kKinds;
                const int32_t cdir = (raw_dir >= 0 && raw_dir < kDirections) ? raw_dir : kDirections;
                const int32_t cptype = clampi(raw_type, kAbsent, P.types);
                const int32_t requested = action_duration(P, H, g.unit_type[slot], ckind, cnone, cptype);
                const bool legal = can_execute(P, H, G, g, slot, ckind, cdir, target, cptype);
                int32_t kind = legal ? ckind : kKindNone;
                int32_t none = legal ? cnone : requested;
                const int32_t pos = reserved_position(G, cell, cdir);
                if (claims_kind(kind)) {
                    const int32_t at = clampi(pos < 0 ? pos + G.cells : pos, 0, G.cells - 1);
                    if (wall(H, G, at) || g.entity_at[at] != kAbsent) {  // admission.py:185-192
                        kind = kKindNone;
                        none = requested;
                    }
                }
                if (claims_kind(kind)) add_claim<kTwoBit>(counts, G.cells, pos);
                if (kind == kKindProduce) atomicAdd(&produce_claims[player], 1u);
                if (counting) count_event(P, g, events + player * kEventCounts, player, kind, cptype, target);
                ReqInfo r;
                r.duration = kind == kKindNone ? none : requested;
                r.target = static_cast<int16_t>(target);
                r.pos = static_cast<int16_t>(pos);
                r.kind = narrow8(kind);
                r.dir = narrow8(cdir);
                r.ptype = narrow8(cptype);
                r.serial = 0;
                info[i] = r;
            };
            if constexpr (kCmd) {
                const Cmds m = cmd_view(P, slab);
                const int32_t raw = m.kind[p];
                issued = raw != kAbsent;
                if (issued) {
                    decide_request(raw, m.dir[p], m.ptype[p], m.target[p], m.none[p], g.cell[slot]);
                    const int32_t rank = m.order[p];
                    const uint32_t minor = rank == kAbsent ? static_cast<uint32_t>(g.birth[slot])
                                                           : static_cast<uint32_t>(clampi(rank, 0, (1 << P.rank_bits) - 1));
                    keys[i] = (static_cast<uint32_t>(player) << 31) | minor;
                } else {
                    keys[i] = 0xffffffffu;
                }
            } else {
                const int32_t* row = P.actions[player] + (game * C + local) * kActionColumns;
                // Read once per step: evict-first loads (ld.global.cs).
                const int32_t raw = __ldcs(row), r1 = __ldcs(row + 1), r2 = __ldcs(row + 2), r3 = __ldcs(row + 3),
                              r4 = __ldcs(row + 4), r5 = __ldcs(row + 5), r6 = __ldcs(row + 6);
                issued = raw != kAbsent;
                if (issued) {
                    const int32_t raw_dir = raw == kKindMove ? r1 : raw == kKindHarvest ? r2 : raw == kKindReturn ? r3
                                            : raw == kKindProduce ? r4 : kAbsent;
                    const int32_t raw_type = raw == kKindProduce ? r5 : kAbsent;
                    const int32_t cell = g.cell[slot];
                    int32_t target = kAbsent;
                    if (raw == kKindAttack) {
                        const int32_t tx = G.x(cell) + (floor_mod(r6, P.side) - P.radius);
                        const int32_t ty = G.y(cell) + (floor_div(r6, P.side) - P.radius);
                        if (tx >= 0 && tx < G.width() && ty >= 0 && ty < G.h) target = ty * G.width() + tx;
                    }
                    const int32_t ckind = (raw >= kAbsent && raw <= kKindAttack) ? raw : kKinds;
                    decide_request(raw, raw_dir, raw_type, target, ckind == kKindNone ? 1 : 0, cell);
                    keys[i] = (static_cast<uint32_t>(player) << 31) | static_cast<uint32_t>(g.birth[slot]);
                } else {
                    keys[i] = 0xffffffffu;  // sorts after every issued request
                }
            }
        }
        R += __popc(__ballot_sync(kFull, issued));
    }
    __syncwarp();
    if (counting && lane < 2 * kEventCounts) {
        const int32_t player = lane / kEventCounts, c = lane % kEventCounts;
        P.out.reward_components[(game * kPlayers + player) * 6 + 1 + c] = static_cast<float>(events[lane]);
    }
    // Java order (admission.py:67-101): player, then rank or birth.
    {
        for (int32_t i = lane; i < A; i += 32) {
            const uint32_t k = keys[i];
            if (k == 0xffffffffu) continue;
            int32_t rank = 0;
            for (int32_t j = 0; j < A; ++j) {
                const uint32_t kj = keys[j];
                rank += kj < k || (kj == k && j < i);
            }
            order[rank] = static_cast<int16_t>(i);
        }
    }
    __syncwarp();
    // Pending orders by prefix count of appends in admission order; the
    // requests nothing can contest are assigned here.
    const int32_t next_order = g.s[kSNextOrder];
    int32_t appended = 0;
    for (int32_t base = 0; base < R; base += 32) {
        const int32_t r = base + lane;
        int32_t i = 0, slot = 0;
        bool appends = false;
        if (r < R) {
            i = order[r];
            slot = N + list[i];
            appends = g.pending_order[slot] == kAbsent;
        }
        const unsigned m = __ballot_sync(kFull, appends);
        if (r < R) {
            const int32_t held = g.pending_order[slot];
            const int32_t ord = appends ? next_order + appended + __popc(m & lanes_below(lane)) : held;
            rank_of[slot - N] = static_cast<int16_t>(r);
            ReqInfo q = info[i];
            const int32_t player = (slot - N) >= C;
            const int32_t rcost = kind_cost(P, H, q.kind, q.ptype);
            const bool contested = claims_kind(q.kind) && (claimed_twice<kTwoBit>(counts, G.cells, q.pos) ||
                                                           (q.kind == kKindProduce && produce_claims[player] > 1));
            const bool serial = contested || (rcost > 0 && rcost > g.s[kSRes0 + player]);
            keys[i] = static_cast<uint32_t>(ord);
            if (serial) {
                info[i].serial = 1;
            } else {
                assign_pending(g, slot, q.kind, q.duration, q.duration, q.dir, q.target, q.ptype, time, ord);
            }
        }
        appended += __popc(m);
    }
    __syncwarp();
    if (lane == 0) g.s[kSNextOrder] = next_order + appended;
    // `serial` lies over the claim counts: the loop above read them last.
    int16_t* serial = reinterpret_cast<int16_t*>(slab + L.serial_off);
    const int32_t S = warp_compact(R, lane, serial, [&](int32_t r) { return info[order[r]].serial != 0; });
    if (S > 0) admit_contested(P, H, G, g, slab, lane, S, holders);
}

// ---------------------------------------------------------------------------
// Completion (pending.py:47-67, completion.py:30-79, kinds/*.py `_complete`).
// The turns run in pending order on lane 0; lowest free slots come from a
// per-player bitmap of inactive slots kept current by spawns and removals.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void free_set(uint32_t* free_words, const Params& P, int32_t slot, bool is_free) {
    const int32_t p = slot - P.neutral;
    if (p < 0 || p >= P.owned) return;
    const int32_t player = p >= P.capacity, local = p - player * P.capacity;
    uint32_t* w = free_words + player * P.free_words + (local >> 5);
    const uint32_t bit = 1u << (local & 31);
    *w = is_free ? (*w | bit) : (*w & ~bit);
}

// kHbmRows: the rules-only rows stay in HBM; the pass reads them for the
// pending slots only, listed first.
template <int kW, bool kHbmRows = false>
__device__ void complete(const Params& P, const Header& H, const Geo<kW>& G, Game& g, char* slab, int lane) {
    const Layout& L = P.layout;
    const int32_t N = P.neutral, E = P.entities, C = P.capacity;
    int16_t* list = reinterpret_cast<int16_t*>(slab + L.list_off);
    int16_t* order = reinterpret_cast<int16_t*>(slab + L.order_off);
    uint32_t* keys = reinterpret_cast<uint32_t*>(slab + L.member_key_off);
    Retained* ret = reinterpret_cast<Retained*>(slab + L.ret_off);
    uint32_t* free_words = reinterpret_cast<uint32_t*>(slab + L.free_off);
    const int32_t time = static_cast<int32_t>(static_cast<uint32_t>(g.s[kSTime]) + 1u);  // pending.select
    __syncwarp();
    if (lane == 0) g.s[kSTime] = time;
    // The acting owned members (completed, kind != NONE) listed with their
    // retained facts, and every completed slot's pending action cleared
    // (pending.clear): one pass over the slots, or with kHbmRows the neutral
    // slots first and then the pending owned slots, listed in slot order from
    // pending_kind alone (`order` is free until the ranking below), so that
    // the rows in HBM are read for those slots only, with their loads at once.
    int32_t Q = E;
    if constexpr (kHbmRows) {
        for (int32_t s = lane; s < N; s += 32) {
            if (g.pending_kind[s] != kAbsent && g.pending_completes_at[s] <= time) g.clear_pending(s);
        }
        Q = warp_compact(P.owned, lane, order, [&](int32_t p) { return g.pending_kind[N + p] != kAbsent; });
    }
    int32_t M = 0;
    for (int32_t base = 0; base < Q; base += 32) {
        int32_t s = base + lane;
        if constexpr (kHbmRows) s = s < Q ? N + order[s] : 0;
        const int32_t pk = base + lane < Q ? g.pending_kind[s] : kAbsent;
        const bool completed = pk != kAbsent && g.pending_completes_at[s] <= time;
        const bool acting = completed && pk != kKindNone && s >= N;
        const unsigned m = __ballot_sync(kFull, acting);
        if (acting) {
            const int32_t i = M + __popc(m & lanes_below(lane));
            list[i] = static_cast<int16_t>(s);
            keys[i] = static_cast<uint32_t>(g.pending_order[s]) ^ 0x80000000u;
            Retained r;
            r.birth = g.birth[s];
            r.carried = g.carried[s];
            r.cell = g.cell[s];
            r.target = g.pending_target_cell[s];
            r.kind = static_cast<int8_t>(pk);
            r.direction = g.pending_direction[s];
            r.produced_type = g.pending_produced_type[s];
            r.owner = g.owner[s];
            r.unit_type = g.unit_type[s];
            ret[i] = r;
        }
        if (completed) g.clear_pending(s);
        M += __popc(m);
    }
    // Free-slot bitmaps of both blocks (inactive slots).
    for (int32_t player = 0; player < kPlayers; ++player) {
        for (int32_t base = 0; base < C; base += 32) {
            const int32_t i = base + lane;
            const unsigned m = __ballot_sync(kFull, i < C && !g.active(N + player * C + i));
            if (lane == 0) free_words[player * P.free_words + (base >> 5)] = m;
        }
    }
    __syncwarp();
    // Pending order (pending.py:55-60): ascending pending_order.
    for (int32_t i = lane; i < M; i += 32) {
        const uint32_t k = keys[i];
        int32_t rank = 0;
        for (int32_t j = 0; j < M; ++j) {
            const uint32_t kj = keys[j];
            rank += kj < k || (kj == k && j < i);
        }
        order[rank] = static_cast<int16_t>(i);
    }
    __syncwarp();
    if (lane == 0) {
        const int32_t cells = G.cells;
        for (int32_t m = 0; m < M; ++m) {
            const int32_t i = order[m];
            const int32_t slot = list[i];
            const Retained r = ret[i];
            const int32_t kind = r.kind;
            const int32_t actor = clampi(r.unit_type, 0, P.types - 1);
            const int32_t player = clampi(r.owner, 0, kPlayers - 1);
            const bool alive = g.birth[slot] == r.birth && r.birth != kAbsent;
            bool removes = false;
            int32_t removed = 0;
            if (kind == kKindMove) {  // move.py:24-32
                if (alive) {
                    const int32_t destination = reserved_position(G, r.cell, r.direction);
                    if (destination >= 0 && destination < cells) g.entity_at[destination] = static_cast<int16_t>(slot);
                    if (r.cell >= 0 && r.cell < cells) g.entity_at[r.cell] = kAbsent;
                    g.cell[slot] = static_cast<int16_t>(destination);
                }
            } else if (kind == kKindHarvest) {  // harvest.py:30-58
                const Neighbour nb = neighbour(P, H, G, g, r.cell, r.direction);
                if (nb.occupied && H.at(nb.unit_type, kIsResource)) {
                    const int32_t amount = H.at(actor, kHarvestAmount);
                    const int32_t left = g.carried[nb.slot] - amount;
                    g.carried[nb.slot] = left;
                    if (alive) g.carried[slot] = amount;
                    if (left <= 0) {
                        removes = true;
                        removed = nb.slot;
                    }
                }
            } else if (kind == kKindReturn) {  // return_.py:31-59
                const Neighbour nb = neighbour(P, H, G, g, r.cell, r.direction);
                if (nb.occupied && H.at(nb.unit_type, kIsStockpile) && r.carried > 0) {
                    if (alive) g.carried[slot] = 0;
                    g.s[kSRes0 + player] += r.carried;
                }
            } else if (kind == kKindProduce) {  // produce.py:49-89, units.py:12-19
                const int32_t newborn_type = clampi(r.produced_type, 0, P.types - 1);
                const int32_t balance = g.s[kSRes0 + player] - H.at(newborn_type, kCost);
                if (balance >= 0) {
                    int32_t newborn = -1;
                    const uint32_t* words = free_words + player * P.free_words;
                    for (int32_t w = 0; w < P.free_words && newborn < 0; ++w) {
                        const int32_t valid = min(32, C - 32 * w);
                        const uint32_t bits = words[w] & (valid == 32 ? ~0u : ((1u << valid) - 1u));
                        if (bits) newborn = N + player * C + 32 * w + __ffs(bits) - 1;
                    }
                    if (newborn >= 0) {
                        const int32_t destination = reserved_position(G, r.cell, r.direction);
                        g.s[kSRes0 + player] = balance;
                        if (destination >= 0 && destination < cells) g.entity_at[destination] = static_cast<int16_t>(newborn);
                        g.birth[newborn] = g.s[kSNextBirth];
                        g.unit_type[newborn] = narrow8(newborn_type);
                        g.owner[newborn] = narrow8(player);
                        g.cell[newborn] = static_cast<int16_t>(destination);
                        g.hit_points[newborn] = static_cast<int16_t>(H.at(newborn_type, kHitPoints));
                        g.s[kSNextBirth] += 1;
                        free_set(free_words, P, newborn, false);
                    } else {
                        g.s[kSOverflow0 + player] += 1;
                    }
                }
            } else if (kind == kKindAttack) {  // attack.py:78-102
                const int32_t occupant = g.entity_at[clampi(r.target, 0, cells - 1)];
                if (occupant != kAbsent) {
                    const int32_t left = static_cast<int32_t>(g.hit_points[occupant]) - H.at(actor, kAttackDamage);
                    g.hit_points[occupant] = static_cast<int16_t>(left);
                    if (left <= 0) {
                        removes = true;
                        removed = occupant;
                    }
                }
            }
            if (removes) {  // completion.py:67, units.remove
                const int32_t at = g.cell[removed];
                if (at >= 0 && at < cells) g.entity_at[at] = kAbsent;
                g.remove(removed);
                free_set(free_words, P, removed, true);
            }
        }
    }
    __syncwarp();
}

// outcome.py:11-37 from the free-slot bitmaps.
__device__ void decide(const Params& P, Game& g, char* slab, int lane, bool& terminated, bool& truncated) {
    const uint32_t* free_words = reinterpret_cast<const uint32_t*>(slab + P.layout.free_off);
    bool surviving[kPlayers];
    for (int p = 0; p < kPlayers; ++p) {
        bool any = false;
        for (int32_t w = 0; w < P.free_words; ++w) {
            const int32_t valid = min(32, P.capacity - 32 * w);
            const uint32_t mask = valid == 32 ? ~0u : ((1u << valid) - 1u);
            any |= (~free_words[p * P.free_words + w] & mask) != 0;
        }
        surviving[p] = any;
    }
    const int count = surviving[0] + surviving[1];
    const bool over = count <= 1;
    const int32_t winner = count == 1 ? (surviving[0] ? 0 : 1) : kAbsent;
    __syncwarp();
    if (lane == 0) {
        g.s[kSGameOver] = over;
        g.s[kSWinner] = winner;
    }
    terminated = over;
    truncated = !over && g.s[kSTime] >= P.max_cycles;
    __syncwarp();
}

}  // namespace nrts
