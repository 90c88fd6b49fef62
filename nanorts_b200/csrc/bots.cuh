// Rush-family scripted bots (WorkerRush, LightRush) on a warp's game slab.
//
// One warp runs a player's bot for one game whose State is already staged in
// the warp's shared-memory slab.  The script (bots/rush.py:24-246) writes
// abstract actions into the player's carry, which lives in the slab beside
// the State; the abstraction layer (bots/abstraction.py:268-1119) turns the
// executing entries into Commands, written to the slab's command rows where
// admission reads them.  Paths under src/nanorts/ of NanoRTS.
//
// Parallel over the player's units: unit lists, birth ranks, nearest-unit
// queries, each `put` of the script, standing/plan/fallback of every entry,
// fillers and the settled carry.  Serial (lane 0): the walk over the executing
// entries in carry order, one A* search each, because every search sees the
// cells claimed by the entries before it (abstraction.py:945-966).
//
// The A* search keeps the reference's pop order exactly.  The reference pops
// the open cell of least key f * (cells + 1) + (cells - sequence), i.e. least
// f, then the latest inserted (pathfinding.py:166-228).  With unit steps and
// the Manhattan heuristic a neighbour's f is its parent's f or f + 2, so the
// open cells always hold just two f values; two stacks (one per value, newest
// on top) give the same pops as the argmin over every cell.
#pragma once

#include <cstdint>

#include "device.cuh"
#include "game.cuh"

namespace nrts {

constexpr int32_t kLast = INT32_MAX;
// Abstract kinds (abstraction.py:34-44) held by the rush bots (rush.py:19-21).
constexpr int32_t kAbsAttack = 1, kAbsHarvest = 2, kAbsTrain = 3, kAbsBuild = 4, kAbsTrainDirection = 6;
constexpr int32_t kFillerDuration = 10;  // abstraction.py:63
constexpr int32_t kWorkerRush = 0, kBarracksRush = 1;
constexpr int32_t kTypeBase = 1, kTypeBarracks = 2, kTypeWorker = 3;  // unit_types.py:122-128
// The carry's int16 order field holds every stamp of a cycle (below 9C + 7).
constexpr int32_t kMaxBotCapacity = 3600;

// AbstractActions fields (abstraction.py:70-81) in carry order.
enum CarryField : int { kCKind, kCUnitBirth, kCOrder, kCTarget, kCTargetBirth, kCBase, kCBaseBirth, kCCell, kCUnitType, kCarryFields };

// One player's carry in the slab, each field at its narrowest exact width:
// births int32; order, target/base slots and the site cell int16 (stamps
// stay below 9C + 7 within a cycle, settled orders below C); kind, unit type
// and trained int8.  HBM keeps the reference's int32 leaves.
struct Carry {
    int32_t *unit_birth, *target_birth, *base_birth;
    int16_t *order, *target, *base, *cell;
    int8_t *kind, *unit_type;
    uint8_t* trained;
    int32_t* next_order;
};

__host__ __device__ inline int32_t carry_bytes(int32_t C) {
    return 3 * round16i(4 * C) + 4 * round16i(2 * C) + 3 * round16i(C) + 16;
}

// Bot scratch (aliases the admission/completion scratch, which it precedes).
struct BotLayout {
    int32_t claimed, free;                                // uint32 [CW]
    int32_t lists;                                        // int16 [2E]: the five unit lists back to back
    int32_t counts;                                       // int32 [16]: list sizes, list offsets, reserved costs
    int32_t own, brank, enemy, queue, temp;               // int16 [C]
    int32_t standing;                                     // uint8 [C]
    int32_t rows;                                         // PlanRow [C]
    int32_t seen, used, kept;                             // uint32 [CW]
    int32_t first;                                        // uint8 [cells]
    int32_t stack;                                        // int16 [cells]
    int32_t bytes;
};

struct PlanRow {
    int16_t start, goal, target, claimed;
    int8_t kind, dir, ptype, radius;  // attack ranges fit int8 (the attack window is at most 7 wide)
    int32_t cost;
};
static_assert(sizeof(PlanRow) == 16, "PlanRow layout");

__host__ __device__ inline BotLayout bot_layout(int32_t C, int32_t E, int32_t cells, int32_t base) {
    BotLayout b;
    const int32_t CW = (cells + 31) / 32;
    int32_t off = base;
    b.claimed = off;  off += round16i(CW * 4);
    b.free = off;  off += round16i(CW * 4);
    b.lists = off;  off += round16i(2 * E * 2);
    b.counts = off;  off += 64;
    b.own = off;  off += round16i(C * 2);
    b.brank = off;  off += round16i(C * 2);
    b.enemy = off;  off += round16i(C * 2);
    b.queue = off;  off += round16i(C * 2);
    b.temp = off;  off += round16i(C * 2);
    b.standing = off;  off += round16i(C);
    b.rows = off;  off += round16i(C * static_cast<int32_t>(sizeof(PlanRow)));
    b.seen = off;  off += round16i(CW * 4);
    b.used = off;  off += round16i(CW * 4);
    b.kept = off;  off += round16i(CW * 4);
    b.first = off;  off += round16i(cells);
    b.stack = off;  off += round16i(cells * 2);
    b.bytes = off - base;
    return b;
}

// counts[]: sizes of the five lists, their offsets in the packed array, the
// players' reserved PRODUCE costs and the walk's kept count.
enum BotCount : int { kNResources, kNEnemies0, kNEnemies1, kNStock0, kNStock1, kOffsets, kNReserved0 = 10, kNReserved1, kNKept };

__device__ __forceinline__ Carry carry_view(const Params& P, char* slab, int player) {
    const int32_t C = P.capacity;
    char* at = slab + P.layout.carry_off + player * carry_bytes(C);
    Carry k;
    k.unit_birth = reinterpret_cast<int32_t*>(at);  at += round16i(4 * C);
    k.target_birth = reinterpret_cast<int32_t*>(at);  at += round16i(4 * C);
    k.base_birth = reinterpret_cast<int32_t*>(at);  at += round16i(4 * C);
    k.order = reinterpret_cast<int16_t*>(at);  at += round16i(2 * C);
    k.target = reinterpret_cast<int16_t*>(at);  at += round16i(2 * C);
    k.base = reinterpret_cast<int16_t*>(at);  at += round16i(2 * C);
    k.cell = reinterpret_cast<int16_t*>(at);  at += round16i(2 * C);
    k.kind = reinterpret_cast<int8_t*>(at);  at += round16i(C);
    k.unit_type = reinterpret_cast<int8_t*>(at);  at += round16i(C);
    k.trained = reinterpret_cast<uint8_t*>(at);  at += round16i(C);
    k.next_order = reinterpret_cast<int32_t*>(at);
    return k;
}

// HBM carries of the acting players -> slab.  Every lane issues all its
// independent loads of a slot chunk before converting and storing them.
__device__ void load_carries(const Params& P, char* slab, int64_t game, int lane) {
    const int32_t C = P.capacity;
    for (int p = 0; p < kPlayers; ++p) {
        if (P.mode != kModeDuel && p != P.bot_player) continue;
        const NrtsBotCarry& src = P.bot[p].carry;
        const Carry k = carry_view(P, slab, p);
        for (int32_t i = lane; i < C; i += 32) {
            const int64_t at = game * C + i;
            int32_t v[kCarryFields];
#pragma unroll
            for (int f = 0; f < kCarryFields; ++f) v[f] = __ldg(src.field[f] + at);
            const uint8_t t = __ldg(src.trained + at);
            k.kind[i] = static_cast<int8_t>(v[kCKind]);
            k.unit_birth[i] = v[kCUnitBirth];
            k.order[i] = static_cast<int16_t>(v[kCOrder]);
            k.target[i] = static_cast<int16_t>(v[kCTarget]);
            k.target_birth[i] = v[kCTargetBirth];
            k.base[i] = static_cast<int16_t>(v[kCBase]);
            k.base_birth[i] = v[kCBaseBirth];
            k.cell[i] = static_cast<int16_t>(v[kCCell]);
            k.unit_type[i] = static_cast<int8_t>(v[kCUnitType]);
            k.trained[i] = t;
        }
        if (lane == 0) *k.next_order = __ldg(src.next_order + game);
    }
}

// Slab carries of the acting players -> HBM (plain stores).
__device__ void store_carries(const Params& P, char* slab, int64_t game, int lane) {
    const int32_t C = P.capacity;
    for (int p = 0; p < kPlayers; ++p) {
        if (P.mode != kModeDuel && p != P.bot_player) continue;
        const NrtsBotCarry& dst = P.bot[p].carry;
        const Carry k = carry_view(P, slab, p);
        for (int32_t i = lane; i < C; i += 32) {
            const int64_t at = game * C + i;
            dst.field[kCKind][at] = k.kind[i];
            dst.field[kCUnitBirth][at] = k.unit_birth[i];
            dst.field[kCOrder][at] = k.order[i];
            dst.field[kCTarget][at] = k.target[i];
            dst.field[kCTargetBirth][at] = k.target_birth[i];
            dst.field[kCBase][at] = k.base[i];
            dst.field[kCBaseBirth][at] = k.base_birth[i];
            dst.field[kCCell][at] = k.cell[i];
            dst.field[kCUnitType][at] = k.unit_type[i];
            dst.trained[at] = k.trained[i];
        }
        if (lane == 0) dst.next_order[game] = *k.next_order;
    }
}

// Bot launches keep the rules-only rows in HBM (kRulesRows): their slab
// shrinks from 15.5 KB to 12.6 KB per 16x16 game, 16 games fit per SM instead
// of 14, and a bot-against-bot step measured 7 % faster.
constexpr uint32_t kBotHbmRows = kRulesRows;

// The State rows a bot launch moves between HBM and the slab (bot-act reads
// the State and never writes it back).
struct RowRef {
    char* global;
    char* smem;
    uint32_t bytes;
};

__device__ __forceinline__ bool bot_row(const Params& P, char* slab, int64_t game, int r, bool leaves, RowRef& out) {
    const Layout& L = P.layout;
    if (!staged_row<kBotHbmRows>(r) || !leaves) return false;
    out.global = global_row(P, r, game);
    out.smem = slab_row(slab, L, r, out.global);
    out.bytes = static_cast<uint32_t>(L.row_bytes[r]);
    return true;
}

constexpr int kBotRows = kSlabLeaves;

// State leaves -> slab in one mbarrier phase, carries while it is in flight.
// Lane r owns row r: it issues the TMA bulk copy of the row's 16-byte-aligned
// body and copies the unaligned head and tail bytes itself.
__device__ bool stage_bots(const Params& P, char* slab, int64_t game, uint64_t* bar, uint32_t parity, int lane) {
    RowRef a;
    const bool has_a = bot_row(P, slab, game, lane, true, a);
    const Span sa = has_a ? split_row(a.global, a.bytes) : Span{0, 0, 0};
    const uint32_t total = __reduce_add_sync(kFull, sa.body);
    if (lane == 0) mbar_arrive_expect_tx(bar, total);
    __syncwarp();
    if (sa.body) bulk_load(a.smem + sa.head, a.global + sa.head, sa.body, bar);
    if (has_a) {
        copy_edge_in(a.smem, a.global, sa.head);
        copy_edge_in(a.smem + sa.head + sa.body, a.global + sa.head + sa.body, sa.tail);
    }
    load_scalars_at_once(P, slab, game, lane);
    load_carries(P, slab, game, lane);
    const bool ok = wait_phase(bar, parity);
    __syncwarp();
    return ok;
}

// Slab -> HBM for what a bot launch writes: the State rows (duel), lane r
// owning row r (TMA bulk store of the body, plain stores of head and tail),
// and the carries; every lane commits a bulk group and waits for it in
// finish_bot_stores.
__device__ void store_bots(const Params& P, char* slab, int64_t game, int lane) {
    const bool leaves = P.mode == kModeDuel;
    fence_proxy_async_smem();
    __syncwarp();
    for (int r = lane; r < kBotRows; r += 32) {
        RowRef ref;
        if (!bot_row(P, slab, game, r, leaves, ref)) continue;
        const Span sp = split_row(ref.global, ref.bytes);
        if (sp.body) bulk_store(ref.global + sp.head, ref.smem + sp.head, sp.body);
        copy_edge_out(ref.global, ref.smem, sp.head);
        copy_edge_out(ref.global + sp.head + sp.body, ref.smem + sp.head + sp.body, sp.tail);
    }
    bulk_commit();
    if (leaves) store_scalars(P, slab, game, lane);
    store_carries(P, slab, game, lane);
}

__device__ __forceinline__ void finish_bot_stores() { bulk_wait_read_all(); }

__device__ __forceinline__ void clear_entry(const Carry& k, int32_t i) {
    k.unit_birth[i] = k.target_birth[i] = k.base_birth[i] = kAbsent;
    k.order[i] = k.target[i] = k.base[i] = k.cell[i] = kAbsent;
    k.kind[i] = k.unit_type[i] = kAbsent;
    k.trained[i] = 0;
}

// empty_actions (abstraction.py:120-135).
__device__ void empty_carry(const Params& P, const Carry& k, int lane) {
    const int32_t C = P.capacity;
    for (int32_t i = lane; i < C; i += 32) clear_entry(k, i);
    if (lane == 0) *k.next_order = 0;
    __syncwarp();
}

__device__ __forceinline__ bool bit_at(const uint32_t* words, int32_t c) { return (words[c >> 5] >> (c & 31)) & 1u; }

__device__ __forceinline__ int32_t iabs(int32_t v) { return v < 0 ? -v : v; }

// ---------------------------------------------------------------------------
// Per-game inputs both players' bots share: cells claimed by pending MOVE and
// PRODUCE actions and each player's reserved PRODUCE cost (_pending_usage,
// abstraction.py:334-361), free cells (:364-367) and the unit lists the
// nearest-unit queries scan (enemies :161-163; harvest_sites, rush.py:151-167).
// ---------------------------------------------------------------------------
template <int kW>
__device__ void bot_prepare(const Params& P, const Header& H, const Geo<kW>& G, const Game& g, char* slab, int lane) {
    const BotLayout B = bot_layout(P.capacity, P.entities, P.cells, P.layout.bot_off);
    uint32_t* claimed = reinterpret_cast<uint32_t*>(slab + B.claimed);
    uint32_t* free_w = reinterpret_cast<uint32_t*>(slab + B.free);
    int32_t* counts = reinterpret_cast<int32_t*>(slab + B.counts);
    const int32_t N = P.neutral, C = P.capacity, E = P.entities, cells = G.cells;
    const int32_t CW = (cells + 31) >> 5;
    for (int32_t w = lane; w < CW; w += 32) claimed[w] = 0u;
    __syncwarp();
    int32_t reserved[kPlayers] = {0, 0};
    int16_t* lists = reinterpret_cast<int16_t*>(slab + B.lists);
    // Two passes over the slots: list sizes, then members at their offsets.
    // Resources and the two players' units are disjoint, as are the two
    // players' stockpiles, so the five lists fit in 2E entries.
    auto members = [&](int32_t s, bool* member) {
        const int32_t type = clampi(g.unit_type[s], 0, P.types - 1);
        const int32_t owner = g.owner[s];
        member[0] = (H.resource_types >> type) & 1u;
        member[1] = owner != kAbsent && owner != 0;
        member[2] = owner != kAbsent && owner != 1;
        const bool stock = (H.stockpile_types >> type) & 1u;
        member[3] = stock && owner == 0;
        member[4] = stock && owner == 1;
    };
    int32_t n[5] = {0, 0, 0, 0, 0};
    for (int32_t base = 0; base < E; base += 32) {
        const int32_t s = base + lane;
        bool member[5] = {false, false, false, false, false};
        if (s < E && g.birth[s] != kAbsent) members(s, member);
#pragma unroll
        for (int l = 0; l < 5; ++l) n[l] += __popc(__ballot_sync(kFull, member[l]));
    }
    int32_t at[5];
    at[0] = 0;
#pragma unroll
    for (int l = 1; l < 5; ++l) at[l] = at[l - 1] + n[l - 1];
    const int32_t room = 2 * E;
    for (int32_t base = 0; base < E; base += 32) {
        const int32_t s = base + lane;
        bool member[5] = {false, false, false, false, false};
        if (s < E && g.birth[s] != kAbsent) {
            const int32_t pk = g.pending_kind[s];
            if (pk == kKindMove || pk == kKindProduce) {
                const int32_t d = clampi(g.pending_direction[s], 0, kDirections - 1);
                int32_t t = g.cell[s] + (d == 1 ? 1 : d == 3 ? -1 : 0) + (d == 0 ? -G.width() : d == 2 ? G.width() : 0);
                if (t < 0) t += cells;  // scatter indices wrap once; the rest drop
                if (t >= 0 && t < cells) atomicOr(&claimed[t >> 5], 1u << (t & 31));
            }
            if (pk == kKindProduce && s >= N) {
                reserved[(s - N) >= C] += H.at(clampi(g.pending_produced_type[s], 0, P.types - 1), kCost);
            }
            members(s, member);
        }
#pragma unroll
        for (int l = 0; l < 5; ++l) {
            const unsigned m = __ballot_sync(kFull, member[l]);
            const int32_t to = at[l] + __popc(m & lanes_below(lane));
            if (member[l] && to < room) lists[to] = static_cast<int16_t>(s);
            at[l] += __popc(m);
        }
    }
    reserved[0] = __reduce_add_sync(kFull, reserved[0]);
    reserved[1] = __reduce_add_sync(kFull, reserved[1]);
    __syncwarp();
    for (int32_t base = 0; base < cells; base += 32) {
        const int32_t c = base + lane;
        const bool open = c < cells && !wall(H, G, c) && g.entity_at[c] == kAbsent && !bit_at(claimed, c);
        const unsigned m = __ballot_sync(kFull, open);
        if (lane == 0) free_w[base >> 5] = m;
    }
    // Sizes clipped to the packed array (they never exceed it for valid States).
    int32_t start = 0;
#pragma unroll
    for (int l = 0; l < 5; ++l) {
        const int32_t size = start + n[l] <= room ? n[l] : (start < room ? room - start : 0);
        if (lane == l) counts[l] = size;
        if (lane == 5 + l) counts[kOffsets + l] = start;
        start += n[l];
    }
    if (lane == 10) counts[kNReserved0] = reserved[0];
    if (lane == 11) counts[kNReserved1] = reserved[1];
    __syncwarp();
}

// _closest (rush.py:31-46): least Manhattan distance, then least birth, then
// least slot; -1 when the list is empty.
template <int kW>
__device__ __forceinline__ int32_t closest(const Geo<kW>& G, const Game& g, const int16_t* list, int32_t n, int32_t origin) {
    const int32_t ox = G.x(origin), oy = G.y(origin);
    int32_t best = -1, best_d = kLast, best_b = kLast;
    for (int32_t j = 0; j < n; ++j) {
        const int32_t s = list[j];
        const int32_t c = g.cell[s];
        const int32_t d = iabs(ox - floor_mod(c, G.width())) + iabs(oy - floor_div(c, G.width()));
        const int32_t b = g.birth[s];
        if (d < best_d || (d == best_d && b < best_b)) {
            best = s;
            best_d = d;
            best_b = b;
        }
    }
    return best;
}

// first_in_unit_order (rush.py:55-57): the member of least birth; -1 if none.
template <typename Pred>
__device__ __forceinline__ int32_t first_by_birth(const int16_t* own, int32_t n, const Game& g, int32_t base_slot, int lane, Pred pred) {
    uint32_t best = 0xffffffffu;
    int32_t who = -1;
    for (int32_t e0 = 0; e0 < n; e0 += 32) {
        const int32_t e = e0 + lane;
        uint32_t b = 0xffffffffu;
        int32_t i = -1;
        if (e < n) {
            i = own[e];
            if (pred(i)) b = static_cast<uint32_t>(g.birth[base_slot + i]);
        }
        const uint32_t m = __reduce_min_sync(kFull, b);
        if (m < best) {
            const int src = __ffs(__ballot_sync(kFull, b == m)) - 1;
            who = __shfl_sync(kFull, i, src);
            best = m;
        }
    }
    return who;
}

// _building_site (abstraction.py:221-253): the first open cell around
// `desired` in ring order (each ring from its top edge, then right, bottom,
// left); -1 if none.  Warp-wide.
template <int kW>
__device__ int32_t building_site(const Params& P, const Header& H, const Geo<kW>& G, const Game& g, int32_t desired,
                                 int32_t reserved, int lane) {
    const int32_t longest = P.height > P.width ? P.height : P.width;
    const int32_t dxd = G.x(desired), dyd = G.y(desired);
    uint32_t best = 0xffffffffu;
    for (int32_t c = lane; c < G.cells; c += 32) {
        const int32_t dx = G.x(c) - dxd, dy = G.y(c) - dyd;
        const int32_t ring = iabs(dx) > iabs(dy) ? iabs(dx) : iabs(dy);
        if (ring == 0 || wall(H, G, c) || g.entity_at[c] != kAbsent || c == reserved) continue;
        const int32_t side = dy == -ring ? 0 : dx == ring ? 1 : dy == ring ? 2 : 3;
        const int32_t along = ((side & 1) == 0 ? dx : dy) + ring;
        const uint32_t visit = static_cast<uint32_t>((ring * 4 + side) * (2 * longest + 1) + along);
        const uint32_t key = visit * static_cast<uint32_t>(G.cells) + static_cast<uint32_t>(c);
        best = key < best ? key : best;
    }
    best = __reduce_min_sync(kFull, best);
    return best == 0xffffffffu ? kAbsent : static_cast<int32_t>(best % static_cast<uint32_t>(G.cells));
}

// The slab view of one player's bot for one game.
struct BotView {
    const Game& g;
    Carry k;
    int32_t* counts;
    int16_t *own, *brank, *enemy, *queue, *temp;
    uint8_t* standing;
    PlanRow* rows;
    uint32_t *claimed, *free_w, *seen, *used, *kept;
    uint8_t* first;
    int16_t* stack;
    const int16_t *resources, *enemies, *stock;
    int32_t n_resources, n_enemies, n_stock;
    int32_t player, base_slot;
};

__device__ __forceinline__ BotView bot_view(const Params& P, const Game& g, char* slab, int player) {
    const BotLayout B = bot_layout(P.capacity, P.entities, P.cells, P.layout.bot_off);
    int32_t* counts = reinterpret_cast<int32_t*>(slab + B.counts);
    BotView v{g, carry_view(P, slab, player), counts,
              reinterpret_cast<int16_t*>(slab + B.own), reinterpret_cast<int16_t*>(slab + B.brank),
              reinterpret_cast<int16_t*>(slab + B.enemy), reinterpret_cast<int16_t*>(slab + B.queue),
              reinterpret_cast<int16_t*>(slab + B.temp), reinterpret_cast<uint8_t*>(slab + B.standing),
              reinterpret_cast<PlanRow*>(slab + B.rows), reinterpret_cast<uint32_t*>(slab + B.claimed),
              reinterpret_cast<uint32_t*>(slab + B.free), reinterpret_cast<uint32_t*>(slab + B.seen),
              reinterpret_cast<uint32_t*>(slab + B.used), reinterpret_cast<uint32_t*>(slab + B.kept),
              reinterpret_cast<uint8_t*>(slab + B.first), reinterpret_cast<int16_t*>(slab + B.stack),
              reinterpret_cast<const int16_t*>(slab + B.lists) + counts[kOffsets + kNResources],
              reinterpret_cast<const int16_t*>(slab + B.lists) + counts[kOffsets + (player == 0 ? kNEnemies0 : kNEnemies1)],
              reinterpret_cast<const int16_t*>(slab + B.lists) + counts[kOffsets + (player == 0 ? kNStock0 : kNStock1)],
              counts[kNResources], counts[player == 0 ? kNEnemies0 : kNEnemies1], counts[player == 0 ? kNStock0 : kNStock1],
              player, P.neutral + player * P.capacity};
    return v;
}

// put / _written (abstraction.py:170-219) of one chosen entry; `stamp` is the
// order a fresh entry takes.
__device__ __forceinline__ void write_entry(const Carry& k, int32_t i, int32_t birth, int32_t kind, int32_t stamp, int32_t target,
                                            int32_t target_birth, int32_t base, int32_t base_birth, int32_t cell, int32_t unit_type) {
    const bool known = k.kind[i] != kAbsent && k.unit_birth[i] == birth;
    if (!known) k.order[i] = static_cast<int16_t>(stamp);
    k.kind[i] = static_cast<int8_t>(kind);
    k.unit_birth[i] = birth;
    k.target[i] = static_cast<int16_t>(target);
    k.target_birth[i] = target_birth;
    k.base[i] = static_cast<int16_t>(base);
    k.base_birth[i] = base_birth;
    k.cell[i] = static_cast<int16_t>(cell);
    k.unit_type[i] = static_cast<int8_t>(unit_type);
    k.trained[i] = 0;
}

__device__ __forceinline__ int32_t birth_of(const Game& g, int32_t slot) { return slot == kAbsent ? kAbsent : g.birth[slot]; }

// ---------------------------------------------------------------------------
// The script: worker_rush (rush.py:225-231) or barracks_rush (rush.py:240-246).
// ---------------------------------------------------------------------------
template <int kW>
__device__ void bot_script(const Params& P, const Header& H, const Geo<kW>& G, BotView& v, int strategy, int32_t trained_type, int lane) {
    const Game& g = v.g;
    const Carry& k = v.k;
    const int32_t C = P.capacity, T = P.types, bs = v.base_slot;
    // own_units (abstraction.py:138-158): present units, birth ranks.
    const int32_t n = warp_compact(C, lane, v.own, [&](int32_t i) { return g.birth[bs + i] != kAbsent; });
    for (int32_t e = lane; e < n; e += 32) {
        const int32_t i = v.own[e];
        const int32_t b = g.birth[bs + i];
        int32_t r = 0;
        for (int32_t j = 0; j < n; ++j) r += g.birth[bs + v.own[j]] < b;
        v.brank[i] = static_cast<int16_t>(r);
        v.enemy[i] = static_cast<int16_t>(closest(G, g, v.enemies, v.n_enemies, g.cell[bs + i]));  // nearest_enemy, rush.py:49-52
    }
    __syncwarp();
    auto type_of = [&](int32_t i) { return clampi(g.unit_type[bs + i], 0, T - 1); };
    auto available = [&](int32_t i) { return g.pending_kind[bs + i] == kAbsent; };  // present by construction
    auto can_harvest = [&](int32_t i) { return H.at(type_of(i), kCanHarvest) != 0; };
    const int32_t resources = g.s[kSRes0 + v.player];
    const bool enemy_found = v.n_enemies > 0;
    int32_t next_order = *k.next_order;

    // put of every own unit `chosen` picks; `chosen` fills the fields (target, target_birth, base, base_birth, cell, unit_type).
    auto put = [&](int32_t kind, auto chosen, auto last) {
        for (int32_t e = lane; e < n; e += 32) {
            const int32_t i = v.own[e];
            int32_t f[6];
            if (chosen(i, f)) {
                write_entry(k, i, g.birth[bs + i], kind, next_order + (last(i) ? C : v.brank[i]), f[0], f[1], f[2], f[3], f[4], f[5]);
            }
        }
        next_order += C + 1;
        __syncwarp();
    };
    auto never = [](int32_t) { return false; };
    auto set6 = [](int32_t* f, int32_t a, int32_t b, int32_t c, int32_t d, int32_t e, int32_t t) {
        f[0] = a; f[1] = b; f[2] = c; f[3] = d; f[4] = e; f[5] = t;
    };
    // build_if_not_already_building (abstraction.py:256-265) for one builder
    // (or none); returns the site it reserves (-1 if none).
    auto build_if = [&](int32_t builder, int32_t unit_type, int32_t reserved) {
        bool builds = false;
        if (builder >= 0) {
            const bool building = k.kind[builder] == kAbsBuild && k.unit_birth[builder] == g.birth[bs + builder] &&
                                  k.unit_type[builder] == unit_type;
            builds = !building;
        }
        const int32_t site = builds ? building_site(P, H, G, g, g.cell[bs + builder], reserved, lane) : kAbsent;
        put(kAbsBuild,
            [&](int32_t i, int32_t* f) { set6(f, kAbsent, kAbsent, kAbsent, kAbsent, site, unit_type); return builds && i == builder; },
            never);
        return builds ? site : reserved;
    };
    // _harvest (rush.py:170-193) for the units `harvesters` picks.
    auto harvest = [&](auto harvesters) {
        const bool res_found = v.n_resources > 0, stock_found = v.n_stock > 0;
        put(kAbsHarvest,
            [&](int32_t i, int32_t* f) {
                if (!harvesters(i)) return false;
                const int32_t cell = g.cell[bs + i];
                const int32_t rs = closest(G, g, v.resources, v.n_resources, cell);
                const int32_t ss = closest(G, g, v.stock, v.n_stock, cell);
                const int32_t rb = birth_of(g, rs), sb = birth_of(g, ss);
                const bool carrying = g.carried[bs + i] > 0;
                const bool harvesting = k.kind[i] == kAbsHarvest && k.unit_birth[i] == g.birth[bs + i];
                const bool same_base = k.base[i] == ss && k.base_birth[i] == sb;
                const bool same_target = k.target[i] == rs && k.target_birth[i] == rb;
                const bool occupied = carrying ? stock_found : (stock_found && res_found);
                const bool unchanged = harvesting && same_base && (carrying || same_target);
                set6(f, carrying ? kAbsent : rs, carrying ? kAbsent : rb, ss, sb, kAbsent, kAbsent);
                return occupied && !unchanged;
            },
            never);
    };
    auto idle_after_harvest = [&](int32_t i) {
        const bool carrying = g.carried[bs + i] > 0;
        const bool occupied = carrying ? v.n_stock > 0 : (v.n_stock > 0 && v.n_resources > 0);
        return !occupied;
    };
    auto attack = [&](auto attackers, auto last) {  // _attack_nearest, rush.py:60-69
        put(kAbsAttack,
            [&](int32_t i, int32_t* f) {
                const int32_t es = v.enemy[i];
                set6(f, es, birth_of(g, es), kAbsent, kAbsent, kAbsent, kAbsent);
                return attackers(i) && enemy_found;
            },
            last);
    };
    auto melee = [&](int32_t i) {  // available_melee, rush.py:72-78
        const int32_t t = type_of(i);
        return H.at(t, kCanAttack) != 0 && H.at(t, kCanHarvest) == 0 && available(i);
    };
    auto any_of_type = [&](int32_t type) {
        bool any = false;
        for (int32_t e = lane; e < n; e += 32) any |= type_of(v.own[e]) == type;
        return __any_sync(kFull, any) != 0;
    };
    const int32_t cost_worker = H.at(clampi(kTypeWorker, 0, T - 1), kCost);
    const int32_t cost_base = H.at(clampi(kTypeBase, 0, T - 1), kCost);
    const int32_t cost_barracks = H.at(clampi(kTypeBarracks, 0, T - 1), kCost);

    if (strategy == kWorkerRush) {
        // train_workers (rush.py:86-95).
        put(kAbsTrain,
            [&](int32_t i, int32_t* f) {
                set6(f, kAbsent, kAbsent, kAbsent, kAbsent, kAbsent, kTypeWorker);
                return type_of(i) == kTypeBase && available(i) && resources >= cost_worker;
            },
            never);
        attack(melee, never);
        // _rushing_workers (rush.py:216-222) with build_base (rush.py:98-113).
        const bool builds = !any_of_type(kTypeBase) && resources >= cost_base;
        const int32_t builder = builds ? first_by_birth(v.own, n, g, bs, lane, can_harvest) : -1;
        build_if(builder, kTypeBase, kAbsent);
        const int32_t harvester = first_by_birth(v.own, n, g, bs, lane, [&](int32_t i) { return can_harvest(i) && i != builder; });
        harvest([&](int32_t i) { return i == harvester; });
        const bool idle = harvester >= 0 && idle_after_harvest(harvester);
        attack([&](int32_t i) { return (can_harvest(i) && i != builder && i != harvester) || (idle && i == harvester); },
               [&](int32_t i) { return idle && i == harvester; });
    } else {
        // train_at_base_and_barracks (rush.py:116-148).
        int32_t held = 0;
        for (int32_t e = lane; e < n; e += 32) held += type_of(v.own[e]) == kTypeWorker;
        held = __reduce_add_sync(kFull, held);
        put(kAbsTrain,
            [&](int32_t i, int32_t* f) {
                set6(f, kAbsent, kAbsent, kAbsent, kAbsent, kAbsent, kTypeWorker);
                return type_of(i) == kTypeBase && available(i) && held < 1 && resources >= cost_worker;
            },
            never);
        const int32_t cost_trained = H.at(clampi(trained_type, 0, T - 1), kCost);
        put(kAbsTrain,
            [&](int32_t i, int32_t* f) {
                set6(f, kAbsent, kAbsent, kAbsent, kAbsent, kAbsent, trained_type);
                return type_of(i) == kTypeBarracks && available(i) && resources >= cost_trained;
            },
            never);
        attack(melee, never);
        // build_base_and_barracks (rush.py:196-213).
        const bool any_barracks = any_of_type(kTypeBarracks);
        const bool builds_base = !any_of_type(kTypeBase) && resources >= cost_base;
        const int32_t base_builder = builds_base ? first_by_birth(v.own, n, g, bs, lane, can_harvest) : -1;
        const int32_t reserved = build_if(base_builder, kTypeBase, kAbsent);
        const int32_t used = base_builder >= 0 ? cost_base : 0;
        const bool builds_barracks = !any_barracks && resources >= cost_barracks + used;
        const int32_t barracks_builder =
            builds_barracks ? first_by_birth(v.own, n, g, bs, lane, [&](int32_t i) { return can_harvest(i) && i != base_builder; }) : -1;
        build_if(barracks_builder, kTypeBarracks, reserved);
        auto free_worker = [&](int32_t i) { return can_harvest(i) && i != base_builder && i != barracks_builder; };
        // _workers_behavior (rush.py:234-237).
        harvest(free_worker);
        attack([&](int32_t i) { return free_worker(i) && idle_after_harvest(i); }, never);
    }
    if (lane == 0) *k.next_order = next_order;
    __syncwarp();
}

// ---------------------------------------------------------------------------
// A* (pathfinding.py:125-252) from `start` to any cell within `radius` of
// `target` over the cells open in `seen` (consumed).  Returns the first step's
// direction, or -1 when the start is already within range or nothing is.
// Single thread.
// ---------------------------------------------------------------------------
template <int kW>
__device__ int32_t astar(const Geo<kW>& G, int32_t height, uint32_t* seen, uint8_t* first, int16_t* stack, int32_t start,
                         int32_t target, int32_t radius) {
    const int32_t cells = G.cells, width = G.width();
    const int32_t tx = G.x(target), ty = G.y(target);
    const int32_t r2 = radius * radius;
    int32_t f = iabs(G.x(start) - tx) + iabs(G.y(start) - ty);
    seen[start >> 5] &= ~(1u << (start & 31));
    int32_t na = 1, nb = 0;  // stack A grows up from 0, stack B down from cells - 1
    bool cur_a = true;       // the stack holding the current (least) f
    stack[0] = static_cast<int16_t>(start);
    for (int32_t pops = 0; pops < cells; ++pops) {
        if ((cur_a ? na : nb) == 0) {
            if ((cur_a ? nb : na) == 0) return kAbsent;  // open list exhausted
            cur_a = !cur_a;
            f += 2;
        }
        const int32_t cell = cur_a ? stack[--na] : stack[cells - 1 - (--nb)];
        const int32_t cx = G.x(cell), cy = G.y(cell);
        const int32_t dx = cx - tx, dy = cy - ty;
        if (dx * dx + dy * dy <= r2) return cell == start ? kAbsent : first[cell];
        const int32_t g_cost = f - (iabs(dx) + iabs(dy));
        const int32_t inherited = cell == start ? -1 : first[cell];
#pragma unroll
        for (int dir = 0; dir < kDirections; ++dir) {
            const int32_t nx = cx + (dir == 1 ? 1 : dir == 3 ? -1 : 0);
            const int32_t ny = cy + (dir == 0 ? -1 : dir == 2 ? 1 : 0);
            if (nx < 0 || nx >= width || ny < 0 || ny >= height) continue;
            const int32_t nc = ny * width + nx;
            const uint32_t bit = 1u << (nc & 31);
            if (!(seen[nc >> 5] & bit)) continue;
            seen[nc >> 5] &= ~bit;
            first[nc] = static_cast<uint8_t>(inherited < 0 ? dir : inherited);
            const int32_t fn = g_cost + 1 + iabs(nx - tx) + iabs(ny - ty);
            if ((fn == f) == cur_a) stack[na++] = static_cast<int16_t>(nc);
            else stack[cells - 1 - nb++] = static_cast<int16_t>(nc);
        }
    }
    return kAbsent;
}

// ---------------------------------------------------------------------------
// translate (abstraction.py:268-294, rush kinds, no draws): standing entries,
// the walk in carry order, the player's Commands rows and the settled carry.
// ---------------------------------------------------------------------------
template <int kW>
__device__ __forceinline__ int32_t adjacent_direction(const Geo<kW>& G, int32_t origin, int32_t goal) {  // abstraction.py:426-433
    if (goal == kAbsent) return kAbsent;
    const int32_t dx = floor_mod(goal, G.width()) - G.x(origin);
    const int32_t dy = floor_div(goal, G.width()) - G.y(origin);
    return (dx == 0 && dy == -1) ? 0 : (dx == 1 && dy == 0) ? 1 : (dx == 0 && dy == 1) ? 2 : (dx == -1 && dy == 0) ? 3 : kAbsent;
}

template <int kW>
__device__ void bot_translate(const Params& P, const Header& H, const Geo<kW>& G, BotView& v, const Cmds& cmd, int lane) {
    const Game& g = v.g;
    const Carry& k = v.k;
    const int32_t C = P.capacity, E = P.entities, T = P.types, cells = G.cells, bs = v.base_slot, p = v.player;
    const int32_t CW = (cells + 31) >> 5;
    const int32_t reserved = v.counts[kNReserved0 + p];
    const int32_t balance = g.s[kSRes0 + p];
    const int32_t other_reserved = v.counts[kNReserved0 + 1 - p];
    const int32_t other_balance = g.s[kSRes0 + 1 - p];
    const bool within_own = reserved == 0 || reserved <= balance;  // _within_balance, abstraction.py:370-371
    const bool within_other = other_reserved == 0 || other_reserved <= other_balance;
    const bool moves_allowed = within_own && within_other;
    auto exists = [&](int32_t slot, int32_t birth) { return slot != kAbsent && g.birth[clampi(slot, 0, E - 1)] == birth; };
    auto cell_of = [&](int32_t slot) { return slot != kAbsent ? static_cast<int32_t>(g.cell[clampi(slot, 0, E - 1)]) : kAbsent; };

    // _standing (abstraction.py:395-423) and executes; this player's rows unissued.
    for (int32_t i = lane; i < C; i += 32) {
        const int32_t kind = k.kind[i];
        const int32_t b = g.birth[bs + i];
        const bool alive = kind != kAbsent && k.unit_birth[i] == b;
        const bool carrying = g.carried[bs + i] > 0;
        const bool target_gone = !exists(k.target[i], k.target_birth[i]);
        bool completed = false;
        if (kind == kAbsAttack) completed = target_gone;
        else if (kind == kAbsHarvest) completed = carrying ? !exists(k.base[i], k.base_birth[i]) : target_gone;
        else if (kind == kAbsTrain) completed = k.trained[i] != 0;
        else if (kind == kAbsBuild) completed = k.cell[i] != kAbsent && g.entity_at[clampi(k.cell[i], 0, cells - 1)] != kAbsent;
        const bool st = alive && !completed;
        const bool ex = st && b != kAbsent && g.pending_kind[bs + i] == kAbsent;
        v.standing[i] = static_cast<uint8_t>(st ? (ex ? 3 : 1) : 0);
        const int32_t o = p * C + i;
        cmd.kind[o] = kAbsent;
        cmd.dir[o] = kAbsent;
        cmd.ptype[o] = kAbsent;
        cmd.target[o] = kAbsent;
        cmd.order[o] = kAbsent;
        cmd.none[o] = 0;
    }
    __syncwarp();
    // _queue (abstraction.py:800-801): executing entries by (order, slot).
    const int32_t q = warp_compact(C, lane, v.temp, [&](int32_t i) { return v.standing[i] == 3; });
    for (int32_t e = lane; e < q; e += 32) {
        const int32_t i = v.temp[e];
        const int32_t o = k.order[i];
        int32_t r = 0;
        for (int32_t j = 0; j < q; ++j) {
            const int32_t oj = k.order[v.temp[j]];
            r += oj < o || (oj == o && j < e);
        }
        v.queue[r] = static_cast<int16_t>(i);
    }
    __syncwarp();
    // _plan (abstraction.py:667-727) with _reach (:576-591) and _fallback (:594-664).
    for (int32_t e = lane; e < q; e += 32) {
        const int32_t i = v.queue[e];
        const int32_t slot = bs + i;
        const int32_t kind = k.kind[i];
        const int32_t ucell = g.cell[slot];
        const int32_t utype = clampi(g.unit_type[slot], 0, T - 1);
        const int32_t target_cell = cell_of(k.target[i]);
        const int32_t range = H.at(utype, kAttackRange);
        const int32_t tdx = G.x(ucell) - floor_mod(target_cell, G.width()), tdy = G.y(ucell) - floor_div(target_cell, G.width());
        const bool in_range = tdx * tdx + tdy * tdy <= range * range;
        const bool carrying = g.carried[slot] > 0;
        const int32_t harvest_goal = carrying ? cell_of(k.base[i]) : target_cell;
        const int32_t goal = kind == kAbsAttack ? target_cell : kind == kAbsHarvest ? harvest_goal : kind == kAbsBuild ? k.cell[i] : kAbsent;
        const int32_t radius = kind == kAbsAttack ? range : (kind == kAbsHarvest || kind == kAbsBuild) ? 1 : 0;
        const bool searches = goal != kAbsent && !(kind == kAbsAttack && in_range);
        PlanRow row;
        row.start = static_cast<int16_t>(ucell);
        row.goal = static_cast<int16_t>(searches ? goal : ucell);
        row.radius = static_cast<int8_t>(searches ? clampi(radius, 0, 127) : 0);
        row.target = kAbsent;
        row.claimed = kAbsent;
        row.kind = kAbsent;
        row.dir = kAbsent;
        row.ptype = kAbsent;
        row.cost = 0;
        if (kind == kAbsAttack) {  // strike
            if (in_range && target_cell != kAbsent) {
                row.kind = kKindAttack;
                row.target = static_cast<int16_t>(target_cell);
            }
        } else if (kind == kAbsHarvest) {  // harvest
            const int32_t dir = adjacent_direction(G, ucell, harvest_goal);
            if (dir != kAbsent) {
                row.kind = carrying ? kKindReturn : kKindHarvest;
                row.dir = static_cast<int8_t>(dir);
            }
        } else if (kind == kAbsTrain || kind == kAbsBuild) {  // train / adjacent production (_production, :465-484)
            int32_t dir = kAbsent;
            const int32_t produced = k.unit_type[i];
            if (kind == kAbsBuild) {
                dir = adjacent_direction(G, ucell, k.cell[i]);
            } else {  // _training_direction (abstraction.py:487-511)
                const bool harvests = H.at(clampi(produced, 0, T - 1), kCanHarvest) != 0;
                const int16_t* near = harvests ? v.resources : v.enemies;
                const int32_t n_near = harvests ? v.n_resources : v.n_enemies;
                int32_t best_score = INT32_MIN;
                for (int d = 0; d < kDirections; ++d) {
                    const int32_t nx = G.x(ucell) + (d == 1 ? 1 : d == 3 ? -1 : 0);
                    const int32_t ny = G.y(ucell) + (d == 0 ? -1 : d == 2 ? 1 : 0);
                    if (nx < 0 || nx >= G.width() || ny < 0 || ny >= P.height || !bit_at(v.free_w, ny * G.width() + nx)) continue;
                    int32_t nearest = kLast;
                    for (int32_t j = 0; j < n_near; ++j) {
                        const int32_t c = g.cell[near[j]];
                        const int32_t dd = iabs(nx - floor_mod(c, G.width())) + iabs(ny - floor_div(c, G.width()));
                        nearest = dd < nearest ? dd : nearest;
                    }
                    const int32_t score = n_near > 0 ? -nearest : 0;
                    if (score > best_score) {
                        best_score = score;
                        dir = d;
                    }
                }
            }
            if (dir != kAbsent) {
                const int32_t claimed = ucell + (dir == 1 ? 1 : dir == 3 ? -1 : 0) + (dir == 0 ? -G.width() : dir == 2 ? G.width() : 0);
                const int32_t cost = H.at(clampi(produced, 0, T - 1), kCost);
                const bool allowed = !bit_at(v.claimed, clampi(claimed, 0, cells - 1)) &&
                                     (reserved == 0 || cost + reserved <= balance) && within_other;  // _produce_allowed, :374-382
                if (allowed) {
                    row.kind = kKindProduce;
                    row.dir = static_cast<int8_t>(dir);
                    row.ptype = static_cast<int8_t>(clampi(produced, kAbsent, T));
                    row.claimed = static_cast<int16_t>(claimed);
                    row.cost = cost;
                }
            }
        }
        v.rows[e] = row;
    }
    for (int32_t w = lane; w < CW; w += 32) {
        v.used[w] = 0u;
        v.kept[w] = 0u;
    }
    __syncwarp();
    // The walk (_in_order / _walk_step, abstraction.py:873-966): lane 0.
    if (lane == 0) {
        int32_t kept_cost = 0, kept_count = 0;
        for (int32_t e = 0; e < q; ++e) {
            const PlanRow row = v.rows[e];
            const int32_t sdx = G.x(row.start) - G.x(row.goal), sdy = G.y(row.start) - G.y(row.goal);
            int32_t step = kAbsent;
            if (sdx * sdx + sdy * sdy > row.radius * row.radius) {
                for (int32_t w = 0; w < CW; ++w) v.seen[w] = v.free_w[w] & ~v.used[w];
                step = astar(G, P.height, v.seen, v.first, v.stack, row.start, row.goal, row.radius);
            }
            int32_t kind, dir, target, ptype, claimed, cost;
            if (step != kAbsent) {  // _answer (abstraction.py:771-786)
                kind = moves_allowed ? kKindMove : kAbsent;
                dir = moves_allowed ? step : kAbsent;
                claimed = moves_allowed ? row.start + (step == 1 ? 1 : step == 3 ? -1 : 0) + (step == 0 ? -G.width() : step == 2 ? G.width() : 0)
                                        : kAbsent;
                target = kAbsent;
                ptype = kAbsent;
                cost = 0;
            } else {
                kind = row.kind;
                dir = row.dir;
                target = row.target;
                ptype = row.ptype;
                claimed = row.claimed;
                cost = row.cost;
            }
            // _kept (abstraction.py:789-797).
            const bool claims = claimed >= 0 && claimed < cells;
            const bool conflicting = claims && (bit_at(v.claimed, claimed) || bit_at(v.kept, claimed));
            const bool overdrawn = cost > 0 && reserved + kept_cost + cost > balance;
            const bool kept = kind != kAbsent && !conflicting && !overdrawn;
            if (claims) v.used[claimed >> 5] |= 1u << (claimed & 31);
            if (kept) {
                if (claims) v.kept[claimed >> 5] |= 1u << (claimed & 31);
                kept_cost += cost;
                const int32_t o = p * C + v.queue[e];
                cmd.kind[o] = static_cast<int8_t>(kind);
                cmd.dir[o] = static_cast<int8_t>(dir);
                cmd.ptype[o] = static_cast<int8_t>(ptype);
                cmd.target[o] = static_cast<int16_t>(target);
                cmd.order[o] = static_cast<int16_t>(kept_count++);
            }
        }
        v.counts[kNKept] = kept_count;
    }
    __syncwarp();
    const int32_t kept_count = v.counts[kNKept];
    // _commands (abstraction.py:1068-1096): available units without a kept desire wait.
    const int32_t nf = warp_compact(C, lane, v.temp, [&](int32_t i) {
        return g.birth[bs + i] != kAbsent && g.pending_kind[bs + i] == kAbsent && cmd.kind[p * C + i] == kAbsent;
    });
    for (int32_t e = lane; e < nf; e += 32) {
        const int32_t i = v.temp[e];
        const int32_t b = g.birth[bs + i];
        int32_t r = 0;
        for (int32_t j = 0; j < nf; ++j) r += g.birth[bs + v.temp[j]] < b;
        const int32_t o = p * C + i;
        cmd.kind[o] = kKindNone;
        cmd.none[o] = kFillerDuration;
        cmd.order[o] = static_cast<int16_t>(kept_count + r);
    }
    __syncwarp();
    // _settled (abstraction.py:1099-1119).
    const int32_t ns = warp_compact(C, lane, v.temp, [&](int32_t i) { return v.standing[i] != 0; });
    for (int32_t i = lane; i < C; i += 32) {
        int32_t r = kAbsent;
        if (v.standing[i] != 0) {
            const int32_t o = k.order[i];
            r = 0;
            for (int32_t j = 0; j < ns; ++j) r += k.order[v.temp[j]] < o;
        }
        v.brank[i] = static_cast<int16_t>(r);
    }
    __syncwarp();
    for (int32_t i = lane; i < C; i += 32) {
        const uint8_t st = v.standing[i];
        if (st != 0) {
            const int32_t kind = k.kind[i];
            const bool trains = kind == kAbsTrain || kind == kAbsTrainDirection;
            k.trained[i] = static_cast<uint8_t>(k.trained[i] != 0 || (st == 3 && trains));
            k.order[i] = v.brank[i];
        } else {
            clear_entry(k, i);
        }
    }
    if (lane == 0) *k.next_order = ns;
    __syncwarp();
}

}  // namespace nrts
