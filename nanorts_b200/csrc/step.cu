// Fused NanoRTS environment step for sm_100a, and its C ABI.
//
// One warp owns one game for the whole step.  A CTA holds G games.  The
// game's State rows are staged into the warp's shared-memory slab with 1D TMA
// bulk copies (cp.async.bulk, completion on an mbarrier), stepped there, and
// written back in place with TMA bulk stores while the same warp computes the
// next step's legality rows and both players' observations and streams them
// to HBM with 16-byte stores.
//
// Semantics follow NanoRTS's JAX program (paths under src/nanorts/):
//   decode            adapters/jaxmarl/actions.py:61-84, adapters/factors.py:117-151
//   admission         core/admission.py:48-156 (Java order, legality, blocking,
//                     pending assignment)
//   conflicts         core/reservations.py:69-306 (CANCEL_BOTH / RANDOM / ALTERNATING,
//                     duration caps, cross-cycle -1 durations)
//   completion        core/pending.py:47-67, core/completion.py:30-79, core/kinds/*.py
//   outcome           core/outcome.py:11-37
//   auto-reset        adapters/lifecycle.py:53-75, adapters/jaxmarl/env.py:109-170
//   legality rows     core/legality.py:32-64, kinds/*.py `_legality`, actions.py:28-41
//   observations      observations/symbolic.py:130-180, observations/visibility.py:70-77
//
// Conflict resolution scans only the holders that can conflict: a request
// conflicts with a pending holder through a shared claimed cell (MOVE and
// PRODUCE claim) or a same-player cost over the balance (PRODUCE costs), so
// the entries in pending order that reservations.resolve scans reduce to the
// conflicting holders sorted by pending order; every other entry adds nothing
// to the prefix counts and the duration caps.  A request whose own cost
// exceeds the balance would conflict with every holder; that branch scans all
// slots.
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>

#include "../../include/nanorts_b200.h"
#include "device.cuh"

namespace nrts {

constexpr int kAbsent = -1;
constexpr int kPlayers = 2;
constexpr int kKindNone = 0, kKindMove = 1, kKindHarvest = 2, kKindReturn = 3, kKindProduce = 4, kKindAttack = 5;
constexpr int kKinds = 6;
constexpr int kDirections = 4;
constexpr int kActionColumns = 7;
constexpr int kFeatures = 6;
constexpr int kScalars = 4;
constexpr int kMaxTypes = 8;
constexpr int kMaxWidth = 64;
constexpr int kMaxHeight = 64;
constexpr int kMaxMaskBits = 96;
constexpr int kSlabLeaves = 15;  // 14 per-slot leaves + entity_at
constexpr int32_t kNoCap = INT32_MAX;
constexpr uint64_t kWaitNanoseconds = 2000000000ull;  // 2 s bound on any wait

enum Column : int {
    kCost, kHitPoints, kProduceTime, kMoveTime, kAttackTime, kHarvestTime, kAttackRange, kAttackDamage,
    kHarvestAmount, kSightRadius, kIsResource, kIsStockpile, kCanHarvest, kCanMove, kCanAttack, kColumns
};

enum Mode : int { kModeStep = 0, kModeReset = 1, kModeOutputs = 2 };

// Scalar slots of a game's slab.
enum Scalar : int {
    kSTime, kSRes0, kSRes1, kSNextBirth, kSNextOrder, kSAlt, kSGameOver, kSWinner, kSOverflow0, kSOverflow1,
    kSEpisode, kSRoot0, kSRoot1, kSCount
};

__device__ int32_t g_status;  // nonzero after a bounded wait gave up

struct Layout {
    int32_t leaf_off[kSlabLeaves];
    int32_t row_bytes[kSlabLeaves];
    int32_t scal_off, req_off, ord_off, cmd_off, ch_off, conf_off, ret_off, words_off, bits_off, bar_off;
    int32_t slab_bytes;
    int32_t header_bytes;  // CTA-wide: terrain rows, unit table, attack windows
};

struct Params {
    int32_t height, width, neutral, capacity, types, offsets, strategy, max_cycles, partial;
    int32_t entities, cells, owned, side, radius, mask_width;
    int32_t mode;
    int64_t lanes;
    void* leaf[NRTS_LEAVES];
    uint32_t* root;
    uint32_t* episode;
    const uint32_t* keys;  // reset mode
    const void* reset[NRTS_LEAVES];
    const uint8_t* terrain;
    const int32_t* table;
    const int32_t* actions[kPlayers];
    NrtsOutputs out;
    Layout layout;
};

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

// Per-CTA constants in shared memory.
struct Header {
    uint64_t* terrain_rows;  // [H] bit x of row y: wall
    int32_t* table;          // [T, kColumns + T]
    uint64_t* attack_window; // [T] window bits within the type's attack range (0 if it cannot attack)
    int32_t stride;          // kColumns + T
    __device__ int32_t at(int32_t type, int column) const { return table[type * stride + column]; }
    __device__ bool produces(int32_t producer, int32_t produced) const { return table[producer * stride + kColumns + produced] != 0; }
    __device__ bool wall(int32_t cell, int32_t width) const { return (terrain_rows[cell / width] >> (cell % width)) & 1ull; }
};

// One game's state in the warp's slab.
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
    int32_t* s;  // scalars
    __device__ bool active(int32_t slot) const { return birth[slot] != kAbsent; }
};

__device__ __forceinline__ int64_t leaf_row_bytes(const Params& P, int leaf) {
    const int64_t E = P.entities;
    switch (leaf) {
        case NRTS_BIRTH: case NRTS_CARRIED_RESOURCES: case NRTS_PENDING_NONE_DURATION: case NRTS_PENDING_ISSUED_AT:
        case NRTS_PENDING_COMPLETES_AT: case NRTS_PENDING_ORDER:
            return 4 * E;
        case NRTS_UNIT_TYPE: case NRTS_OWNER: case NRTS_PENDING_KIND: case NRTS_PENDING_DIRECTION:
        case NRTS_PENDING_PRODUCED_TYPE:
            return E;
        case NRTS_CELL: case NRTS_HIT_POINTS: case NRTS_PENDING_TARGET_CELL:
            return 2 * E;
        case NRTS_ENTITY_AT:
            return 2 * static_cast<int64_t>(P.cells);
        default:
            return 0;
    }
}

// The slab address of a leaf row whose global copy starts at `global`: the
// region start shifted by the global address's offset within 16 bytes, so the
// 16-byte-aligned body of the row maps onto 16-byte-aligned shared memory.
__device__ __forceinline__ char* slab_row(char* slab, const Layout& L, int leaf, const void* global) {
    return slab + L.leaf_off[leaf] + (reinterpret_cast<uintptr_t>(global) & 15u);
}

__device__ __forceinline__ const char* global_row(const Params& P, int leaf, int64_t game) {
    return static_cast<const char*>(P.leaf[leaf]) + game * leaf_row_bytes(P, leaf);
}

__device__ Game game_view(const Params& P, char* slab, int64_t game) {
    const Layout& L = P.layout;
    auto row = [&](int leaf) { return slab_row(slab, L, leaf, global_row(P, leaf, game)); };
    Game g;
    g.birth = reinterpret_cast<int32_t*>(row(NRTS_BIRTH));
    g.unit_type = reinterpret_cast<int8_t*>(row(NRTS_UNIT_TYPE));
    g.owner = reinterpret_cast<int8_t*>(row(NRTS_OWNER));
    g.cell = reinterpret_cast<int16_t*>(row(NRTS_CELL));
    g.hit_points = reinterpret_cast<int16_t*>(row(NRTS_HIT_POINTS));
    g.carried = reinterpret_cast<int32_t*>(row(NRTS_CARRIED_RESOURCES));
    g.pending_kind = reinterpret_cast<int8_t*>(row(NRTS_PENDING_KIND));
    g.pending_direction = reinterpret_cast<int8_t*>(row(NRTS_PENDING_DIRECTION));
    g.pending_none_duration = reinterpret_cast<int32_t*>(row(NRTS_PENDING_NONE_DURATION));
    g.pending_target_cell = reinterpret_cast<int16_t*>(row(NRTS_PENDING_TARGET_CELL));
    g.pending_produced_type = reinterpret_cast<int8_t*>(row(NRTS_PENDING_PRODUCED_TYPE));
    g.pending_issued_at = reinterpret_cast<int32_t*>(row(NRTS_PENDING_ISSUED_AT));
    g.pending_completes_at = reinterpret_cast<int32_t*>(row(NRTS_PENDING_COMPLETES_AT));
    g.pending_order = reinterpret_cast<int32_t*>(row(NRTS_PENDING_ORDER));
    g.entity_at = reinterpret_cast<int16_t*>(row(NRTS_ENTITY_AT));
    g.s = reinterpret_cast<int32_t*>(slab + L.scal_off);
    return g;
}

// Splits a row copy into a plain-copied head, a TMA body and a plain tail.
struct Span {
    uint32_t head, body, tail;
};

__device__ __forceinline__ Span split_row(const void* global, int64_t bytes) {
    const uint32_t mis = reinterpret_cast<uintptr_t>(global) & 15u;
    const int64_t room = static_cast<int64_t>((16u - mis) & 15u);
    const uint32_t head = static_cast<uint32_t>(bytes < room ? bytes : room);
    const uint32_t body = static_cast<uint32_t>((bytes - head) & ~int64_t{15});
    return Span{head, body, static_cast<uint32_t>(bytes - head - body)};
}

// Waits for the warp's mbarrier phase with a bounded spin; on timeout records
// the status code and waits once more (bounded) for copies still in flight.
__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ bool wait_phase(uint64_t* bar, uint32_t parity) {
    const uint64_t start = global_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (global_ns() - start > kWaitNanoseconds) {
            atomicExch(&g_status, 1);
            const uint64_t again = global_ns();
            while (!mbar_try_wait(bar, parity) && global_ns() - again < kWaitNanoseconds) {
            }
            return false;
        }
    }
    return true;
}

// ---------------------------------------------------------------------------
// Staging: global rows -> slab.
// ---------------------------------------------------------------------------
__device__ bool stage_state(const Params& P, char* slab, int64_t game, uint64_t* bar, int lane) {
    const Layout& L = P.layout;
    if (lane == 0) {
        uint32_t total = 0;
        for (int k = 0; k < kSlabLeaves; ++k) total += split_row(global_row(P, k, game), L.row_bytes[k]).body;
        mbar_arrive_expect_tx(bar, total);
        for (int k = 0; k < kSlabLeaves; ++k) {
            const char* src = global_row(P, k, game);
            const Span sp = split_row(src, L.row_bytes[k]);
            if (sp.body) bulk_load(slab_row(slab, L, k, src) + sp.head, src + sp.head, sp.body, bar);
        }
    }
    // Unaligned heads and tails byte by byte.
    for (int k = 0; k < kSlabLeaves; ++k) {
        const char* src = global_row(P, k, game);
        const Span sp = split_row(src, L.row_bytes[k]);
        char* dst = slab_row(slab, L, k, src);
        for (uint32_t i = lane; i < sp.head; i += 32) dst[i] = src[i];
        for (uint32_t i = lane; i < sp.tail; i += 32) dst[sp.head + sp.body + i] = src[sp.head + sp.body + i];
    }
    int32_t* s = reinterpret_cast<int32_t*>(slab + L.scal_off);
    const int32_t* time = static_cast<const int32_t*>(P.leaf[NRTS_TIME]);
    const int32_t* res = static_cast<const int32_t*>(P.leaf[NRTS_PLAYER_RESOURCES]);
    const int32_t* ov = static_cast<const int32_t*>(P.leaf[NRTS_SPAWN_OVERFLOW]);
    switch (lane) {
        case kSTime: s[kSTime] = time[game]; break;
        case kSRes0: s[kSRes0] = res[2 * game]; break;
        case kSRes1: s[kSRes1] = res[2 * game + 1]; break;
        case kSNextBirth: s[kSNextBirth] = static_cast<const int32_t*>(P.leaf[NRTS_NEXT_BIRTH])[game]; break;
        case kSNextOrder: s[kSNextOrder] = static_cast<const int32_t*>(P.leaf[NRTS_NEXT_PENDING_ORDER])[game]; break;
        case kSAlt: s[kSAlt] = static_cast<const int32_t*>(P.leaf[NRTS_ALTERNATING_CONFLICT_COUNT])[game]; break;
        case kSGameOver: s[kSGameOver] = static_cast<const uint8_t*>(P.leaf[NRTS_GAME_OVER])[game]; break;
        case kSWinner: s[kSWinner] = static_cast<const int32_t*>(P.leaf[NRTS_WINNER])[game]; break;
        case kSOverflow0: s[kSOverflow0] = ov[2 * game]; break;
        case kSOverflow1: s[kSOverflow1] = ov[2 * game + 1]; break;
        case kSEpisode: s[kSEpisode] = static_cast<int32_t>(P.episode[game]); break;
        case kSRoot0: s[kSRoot0] = static_cast<int32_t>(P.root[2 * game]); break;
        case kSRoot1: s[kSRoot1] = static_cast<int32_t>(P.root[2 * game + 1]); break;
        default: break;
    }
    const bool ok = wait_phase(bar, 0);
    __syncwarp();
    return ok;
}

// Reset rows (one game's decided initial State) -> slab.
__device__ void load_reset(const Params& P, char* slab, int64_t game, int lane) {
    const Layout& L = P.layout;
    for (int k = 0; k < kSlabLeaves; ++k) {
        char* dst = slab_row(slab, L, k, global_row(P, k, game));
        const char* src = static_cast<const char*>(P.reset[k]);
        for (int32_t i = lane; i < L.row_bytes[k]; i += 32) dst[i] = src[i];
    }
    int32_t* s = reinterpret_cast<int32_t*>(slab + L.scal_off);
    auto i32 = [&](int leaf, int k) { return static_cast<const int32_t*>(P.reset[leaf])[k]; };
    switch (lane) {
        case kSTime: s[kSTime] = i32(NRTS_TIME, 0); break;
        case kSRes0: s[kSRes0] = i32(NRTS_PLAYER_RESOURCES, 0); break;
        case kSRes1: s[kSRes1] = i32(NRTS_PLAYER_RESOURCES, 1); break;
        case kSNextBirth: s[kSNextBirth] = i32(NRTS_NEXT_BIRTH, 0); break;
        case kSNextOrder: s[kSNextOrder] = i32(NRTS_NEXT_PENDING_ORDER, 0); break;
        case kSAlt: s[kSAlt] = i32(NRTS_ALTERNATING_CONFLICT_COUNT, 0); break;
        case kSGameOver: s[kSGameOver] = static_cast<const uint8_t*>(P.reset[NRTS_GAME_OVER])[0]; break;
        case kSWinner: s[kSWinner] = i32(NRTS_WINNER, 0); break;
        case kSOverflow0: s[kSOverflow0] = i32(NRTS_SPAWN_OVERFLOW, 0); break;
        case kSOverflow1: s[kSOverflow1] = i32(NRTS_SPAWN_OVERFLOW, 1); break;
        default: break;
    }
    __syncwarp();
}

// Slab -> global rows (TMA bulk stores for bodies), and the scalar leaves.
__device__ void store_state(const Params& P, char* slab, int64_t game, int lane) {
    const Layout& L = P.layout;
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
        for (int k = 0; k < kSlabLeaves; ++k) {
            char* dst = static_cast<char*>(P.leaf[k]) + game * L.row_bytes[k];
            const Span sp = split_row(dst, L.row_bytes[k]);
            if (sp.body) bulk_store(dst + sp.head, slab_row(slab, L, k, dst) + sp.head, sp.body);
        }
        bulk_commit();
    }
    for (int k = 0; k < kSlabLeaves; ++k) {
        char* dst = static_cast<char*>(P.leaf[k]) + game * L.row_bytes[k];
        const Span sp = split_row(dst, L.row_bytes[k]);
        const char* src = slab_row(slab, L, k, dst);
        for (uint32_t i = lane; i < sp.head; i += 32) dst[i] = src[i];
        for (uint32_t i = lane; i < sp.tail; i += 32) dst[sp.head + sp.body + i] = src[sp.head + sp.body + i];
    }
    const int32_t* s = reinterpret_cast<const int32_t*>(slab + L.scal_off);
    int32_t* res = static_cast<int32_t*>(P.leaf[NRTS_PLAYER_RESOURCES]);
    int32_t* ov = static_cast<int32_t*>(P.leaf[NRTS_SPAWN_OVERFLOW]);
    switch (lane) {
        case kSTime: static_cast<int32_t*>(P.leaf[NRTS_TIME])[game] = s[kSTime]; break;
        case kSRes0: res[2 * game] = s[kSRes0]; break;
        case kSRes1: res[2 * game + 1] = s[kSRes1]; break;
        case kSNextBirth: static_cast<int32_t*>(P.leaf[NRTS_NEXT_BIRTH])[game] = s[kSNextBirth]; break;
        case kSNextOrder: static_cast<int32_t*>(P.leaf[NRTS_NEXT_PENDING_ORDER])[game] = s[kSNextOrder]; break;
        case kSAlt: static_cast<int32_t*>(P.leaf[NRTS_ALTERNATING_CONFLICT_COUNT])[game] = s[kSAlt]; break;
        case kSGameOver: static_cast<uint8_t*>(P.leaf[NRTS_GAME_OVER])[game] = static_cast<uint8_t>(s[kSGameOver]); break;
        case kSWinner: static_cast<int32_t*>(P.leaf[NRTS_WINNER])[game] = s[kSWinner]; break;
        case kSOverflow0: ov[2 * game] = s[kSOverflow0]; break;
        case kSOverflow1: ov[2 * game + 1] = s[kSOverflow1]; break;
        case kSEpisode: P.episode[game] = static_cast<uint32_t>(s[kSEpisode]); break;
        case kSRoot0: P.root[2 * game] = static_cast<uint32_t>(s[kSRoot0]); break;
        case kSRoot1: P.root[2 * game + 1] = static_cast<uint32_t>(s[kSRoot1]); break;
        default: break;
    }
}

// ---------------------------------------------------------------------------
// Rules.
// ---------------------------------------------------------------------------
// DIRECTION_OFFSETS (model/vocabulary.py): up, right, down, left.
__device__ __forceinline__ int dir_dx(int d) { return (d == 1) - (d == 3); }
__device__ __forceinline__ int dir_dy(int d) { return (d == 2) - (d == 0); }

__device__ __forceinline__ int32_t reserved_position(int32_t cell, int32_t direction, int32_t width) {
    const int d = clampi(direction, 0, kDirections - 1);
    return cell + dir_dx(d) + dir_dy(d) * width;
}

struct Neighbour {
    bool free, occupied;
    int32_t slot, unit_type, owner;
};

// core/board.py:23-61.
__device__ __forceinline__ Neighbour neighbour(const Params& P, const Header& H, const Game& g, int32_t cell, int32_t direction) {
    const int32_t px = floor_mod(cell, P.width), py = floor_div(cell, P.width);
    const int d = clampi(direction, 0, kDirections - 1);
    const int32_t nx = px + dir_dx(d), ny = py + dir_dy(d);
    const bool on_board = direction >= 0 && direction < kDirections && nx >= 0 && nx < P.width && ny >= 0 && ny < P.height;
    const int32_t ncell = on_board ? ny * P.width + nx : 0;
    const int32_t occupant = g.entity_at[ncell];
    Neighbour n;
    n.occupied = on_board && occupant != kAbsent;
    n.slot = n.occupied ? occupant : 0;
    n.free = on_board && occupant == kAbsent && !H.wall(ncell, P.width);
    n.unit_type = clampi(g.unit_type[n.slot], 0, P.types - 1);
    n.owner = g.owner[n.slot];
    return n;
}

// core/admission.py:443-452.
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

// kinds/*.py `_is_valid`.
__device__ bool can_execute(const Params& P, const Header& H, const Game& g, int32_t slot, int32_t kind, int32_t direction,
                            int32_t target_cell, int32_t produced_type) {
    const int32_t actor = clampi(g.unit_type[slot], 0, P.types - 1);
    const int32_t owner = g.owner[slot];
    const int32_t cell = g.cell[slot];
    switch (kind) {
        case kKindNone: return true;
        case kKindMove: return H.at(actor, kCanMove) && neighbour(P, H, g, cell, direction).free;
        case kKindHarvest: {
            const Neighbour n = neighbour(P, H, g, cell, direction);
            return H.at(actor, kCanHarvest) && g.carried[slot] == 0 && n.occupied && H.at(n.unit_type, kIsResource);
        }
        case kKindReturn: {
            const Neighbour n = neighbour(P, H, g, cell, direction);
            return H.at(actor, kCanHarvest) && g.carried[slot] > 0 && n.occupied && H.at(n.unit_type, kIsStockpile) && n.owner == owner;
        }
        case kKindProduce: {
            const int32_t balance = g.s[kSRes0 + clampi(owner, 0, kPlayers - 1)];
            const int32_t known = clampi(produced_type, 0, P.types - 1);
            return produced_type >= 0 && produced_type < P.types && H.produces(actor, known) && balance >= H.at(known, kCost) &&
                   neighbour(P, H, g, cell, direction).free;
        }
        case kKindAttack: {
            const bool on_board = target_cell >= 0 && target_cell < P.cells;
            const int32_t target_slot = g.entity_at[on_board ? target_cell : 0];
            const bool holds = on_board && target_slot != kAbsent;
            const int32_t target_owner = holds ? g.owner[target_slot] : kAbsent;
            const int32_t range = H.at(actor, kAttackRange);
            const int32_t dx = floor_mod(target_cell, P.width) - floor_mod(cell, P.width);
            const int32_t dy = floor_div(target_cell, P.width) - floor_div(cell, P.width);
            return H.at(actor, kCanAttack) && target_owner >= 0 && target_owner != owner && dx * dx + dy * dy <= range * range;
        }
        default: return false;
    }
}

__device__ __forceinline__ bool claims_kind(int32_t kind) { return kind == kKindMove || kind == kKindProduce; }

__device__ __forceinline__ int32_t kind_cost(const Params& P, const Header& H, int32_t kind, int32_t produced_type) {
    return kind == kKindProduce ? H.at(clampi(produced_type, 0, P.types - 1), kCost) : 0;
}

// Order-preserving warp compaction of indices [0, n) satisfying `pred` into `out`.
template <typename Pred>
__device__ __forceinline__ int32_t warp_compact(int32_t n, int lane, int16_t* out, Pred pred) {
    int32_t count = 0;
    for (int32_t base = 0; base < n; base += 32) {
        const int32_t i = base + lane;
        const bool keep = i < n && pred(i);
        const unsigned m = __ballot_sync(kFull, keep);
        if (keep) out[count + __popc(m & lanes_below(lane))] = static_cast<int16_t>(i);
        count += __popc(m);
    }
    __syncwarp();
    return count;
}

// Packed command of one request: kind | direction << 8 | produced_type << 16, target.
struct Cmd {
    int32_t packed;
    int32_t target;
    __device__ int32_t kind() const { return static_cast<int8_t>(packed & 0xff); }
    __device__ int32_t direction() const { return static_cast<int8_t>((packed >> 8) & 0xff); }
    __device__ int32_t produced_type() const { return static_cast<int8_t>((packed >> 16) & 0xff); }
};

__device__ __forceinline__ int8_t narrow8(int32_t v) { return static_cast<int8_t>(v); }

struct Scratch {
    int16_t* req;    // request slots, then members
    int16_t* ord;    // sorted request / member order
    Cmd* cmd;        // per request
    int16_t* ch;     // claim holders
    int16_t* conf;   // conflicting holders
    Retained* ret;   // per member
    uint32_t* words; // mask words per owned slot (epilogue)
    uint64_t* bits;  // occupancy [2][H], visibility [2][H] (epilogue)
};

__device__ Scratch scratch_view(const Layout& L, char* slab) {
    Scratch s;
    s.req = reinterpret_cast<int16_t*>(slab + L.req_off);
    s.ord = reinterpret_cast<int16_t*>(slab + L.ord_off);
    s.cmd = reinterpret_cast<Cmd*>(slab + L.cmd_off);
    s.ch = reinterpret_cast<int16_t*>(slab + L.ch_off);
    s.conf = reinterpret_cast<int16_t*>(slab + L.conf_off);
    s.ret = reinterpret_cast<Retained*>(slab + L.ret_off);
    s.words = reinterpret_cast<uint32_t*>(slab + L.words_off);
    s.bits = reinterpret_cast<uint64_t*>(slab + L.bits_off);
    return s;
}

// ---------------------------------------------------------------------------
// Admission: decode, Java order, then each request in turn.
// ---------------------------------------------------------------------------
__device__ void admit(const Params& P, const Header& H, Game& g, const Scratch& X, int64_t game, int lane) {
    const int32_t N = P.neutral, C = P.capacity;
    const int32_t time = g.s[kSTime];

    // Decode the rows of available slots (actions.py:61-84) into compact requests.
    const int32_t R = warp_compact(P.owned, lane, X.req, [&](int32_t p) {
        const int32_t slot = N + p;
        if (!(g.active(slot) && g.pending_kind[slot] == kAbsent)) return false;
        const int32_t player = p / C, local = p % C;
        const int32_t* row = P.actions[player] + (game * C + local) * kActionColumns;
        return row[0] != kAbsent;
    });
    for (int32_t i = lane; i < R; i += 32) {
        const int32_t p = X.req[i];
        const int32_t slot = N + p;
        const int32_t player = p / C, local = p % C;
        const int32_t* row = P.actions[player] + (game * C + local) * kActionColumns;
        const int32_t kind = row[0];
        const int32_t direction = kind == kKindMove      ? row[1]
                                  : kind == kKindHarvest ? row[2]
                                  : kind == kKindReturn  ? row[3]
                                  : kind == kKindProduce ? row[4]
                                                         : kAbsent;
        const int32_t produced = kind == kKindProduce ? row[5] : kAbsent;
        const int32_t cell = g.cell[slot];
        const int32_t offset = row[6];
        const int32_t tx = floor_mod(cell, P.width) + (floor_mod(offset, P.side) - P.radius);
        const int32_t ty = floor_div(cell, P.width) + (floor_div(offset, P.side) - P.radius);
        const bool on_board = tx >= 0 && tx < P.width && ty >= 0 && ty < P.height;
        // Canonical forms that decide exactly like the raw values: every kind
        // outside [-1, 5] is unknown (duration 0, never legal), every
        // direction outside [0, 3] is off the board, and a produced type is
        // only ever clipped to [0, T-1] or range-checked.
        const int32_t ckind = (kind >= kAbsent && kind <= kKindAttack) ? kind : kKinds;
        const int32_t cdir = (direction >= 0 && direction < kDirections) ? direction : kDirections;
        const int32_t cptype = clampi(produced, kAbsent, P.types);
        Cmd c;
        c.packed = (ckind & 0xff) | ((cdir & 0xff) << 8) | ((cptype & 0xff) << 16);
        c.target = (kind == kKindAttack && on_board) ? ty * P.width + tx : kAbsent;
        X.cmd[i] = c;
    }
    __syncwarp();
    // Java order (admission.py:67-101): player, then birth, then position.
    for (int32_t i = lane; i < R; i += 32) {
        const int32_t pi = X.req[i];
        const int32_t player_i = pi / C;
        const int32_t birth_i = g.birth[N + pi];
        int32_t rank = 0;
        for (int32_t j = 0; j < R; ++j) {
            const int32_t pj = X.req[j];
            const int32_t player_j = pj / C;
            const int32_t birth_j = g.birth[N + pj];
            rank += (player_j < player_i) || (player_j == player_i && (birth_j < birth_i || (birth_j == birth_i && pj < pi)));
        }
        X.ord[rank] = static_cast<int16_t>(i);
    }
    // Claim holders: pending MOVE / PRODUCE.
    int32_t holders = warp_compact(P.entities, lane, X.ch, [&](int32_t s) { return claims_kind(g.pending_kind[s]); });

    uint32_t k0 = 0, k1 = 0;
    if (P.strategy == 1) {  // episode_root = fold_in(environment_root, episode_index)
        k0 = static_cast<uint32_t>(g.s[kSRoot0]);
        k1 = static_cast<uint32_t>(g.s[kSRoot1]);
        fold_in(k0, k1, static_cast<uint32_t>(g.s[kSEpisode]));
    }

    for (int32_t k = 0; k < R; ++k) {
        const int32_t i = X.ord[k];
        const int32_t slot = N + X.req[i];
        const Cmd c = X.cmd[i];
        const int32_t ckind = c.kind(), cdir = c.direction(), cptype = c.produced_type(), ctarget = c.target;
        const int32_t cnone = ckind == kKindNone ? 1 : 0;
        const int32_t requested = action_duration(P, H, g.unit_type[slot], ckind, cnone, cptype);
        const bool legal = can_execute(P, H, g, slot, ckind, cdir, ctarget, cptype);
        int32_t kind = legal ? ckind : kKindNone;
        int32_t none_duration = legal ? cnone : requested;
        const int32_t cell = g.cell[slot];
        const int32_t reserved = reserved_position(cell, cdir, P.width);
        if (claims_kind(kind)) {
            const int32_t at = clampi(reserved < 0 ? reserved + P.cells : reserved, 0, P.cells - 1);
            if (H.wall(at, P.width) || g.entity_at[at] != kAbsent) {
                kind = kKindNone;
                none_duration = requested;
            }
        }
        const bool rclaims = claims_kind(kind);
        const int32_t rcost = kind_cost(P, H, kind, cptype);
        const int32_t rplayer = clampi(g.owner[slot], 0, kPlayers - 1);
        const int32_t balance = g.s[kSRes0 + rplayer];
        if (rclaims || rcost != 0) {
            // Conflicting holders (reservations.py:122-135).
            const bool every_holder = rcost > 0 && rcost > balance;
            auto conflicts = [&](int32_t s) {
                const int32_t pk = g.pending_kind[s];
                if (pk == kAbsent) return false;
                const bool hclaims = claims_kind(pk);
                const bool shared = hclaims && rclaims && reserved_position(g.cell[s], g.pending_direction[s], P.width) == reserved;
                const int32_t hcost = (clampi(g.owner[s], 0, kPlayers - 1) == rplayer) ? kind_cost(P, H, pk, g.pending_produced_type[s]) : 0;
                const int32_t claimed = hcost + rcost;
                const bool over = rcost != 0 && claimed > 0 && claimed > balance;
                return shared || over;
            };
            int32_t n;
            if (every_holder) {
                n = warp_compact(P.entities, lane, X.conf, conflicts);
            } else {
                int32_t count = 0;
                for (int32_t base = 0; base < holders; base += 32) {
                    const int32_t j = base + lane;
                    const int32_t s = j < holders ? X.ch[j] : 0;
                    const bool keep = j < holders && conflicts(s);
                    const unsigned m = __ballot_sync(kFull, keep);
                    if (keep) X.conf[count + __popc(m & lanes_below(lane))] = static_cast<int16_t>(s);
                    count += __popc(m);
                }
                __syncwarp();
                n = count;
            }
            if (n > 0) {
                if (lane == 0) {
                    // Pending order (pending.py:17-44): ascending pending_order.
                    for (int32_t a = 1; a < n; ++a) {
                        const int16_t v = X.conf[a];
                        const int32_t key = g.pending_order[v];
                        int32_t b = a - 1;
                        while (b >= 0 && g.pending_order[X.conf[b]] > key) {
                            X.conf[b + 1] = X.conf[b];
                            --b;
                        }
                        X.conf[b + 1] = v;
                    }
                    uint32_t e0 = 0, e1 = 0;
                    if (P.strategy == 1) {
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
                        const int32_t e = X.conf[a];
                        if (g.pending_issued_at[e] != time) {
                            cross_seen = true;
                            continue;
                        }
                        const int32_t dur = action_duration(P, H, g.unit_type[e], g.pending_kind[e], g.pending_none_duration[e],
                                                            g.pending_produced_type[e]);
                        bool cancels_request = true, cancels_pending = true;
                        if (P.strategy == 2) {
                            cancels_request = ((alt + same_before) % 2) == 0;
                            cancels_pending = !cancels_request;
                        } else if (P.strategy == 1) {
                            uint32_t d0 = e0, d1 = e1;
                            fold_in(d0, d1, static_cast<uint32_t>(same_before));
                            cancels_request = randint01(d0, d1) == 0;
                            cancels_pending = !cancels_request;
                        }
                        if (cancels_pending) {
                            const int32_t before = cross_seen ? -1 : min(requested, cap);
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
                        none_duration = cross_seen ? -1 : min(requested, cap);
                    }
                    X.conf[0] = static_cast<int16_t>(kind);
                    reinterpret_cast<int32_t*>(X.conf)[1] = none_duration;
                }
                __syncwarp();
                kind = X.conf[0];
                none_duration = reinterpret_cast<int32_t*>(X.conf)[1];
                __syncwarp();
            }
        }
        // _assign_pending_action (admission.py:241-270); every listed request is issued.
        if (lane == 0) {
            const int32_t duration = kind == kKindNone ? none_duration : requested;
            const int32_t held = g.pending_order[slot];
            const bool appends = held == kAbsent;
            const bool keeps_direction = kind == kKindMove || kind == kKindHarvest || kind == kKindReturn || kind == kKindProduce;
            g.pending_kind[slot] = narrow8(kind);
            g.pending_direction[slot] = narrow8(keeps_direction ? cdir : kAbsent);
            g.pending_none_duration[slot] = kind == kKindNone ? none_duration : 0;
            g.pending_target_cell[slot] = static_cast<int16_t>(kind == kKindAttack ? ctarget : kAbsent);
            g.pending_produced_type[slot] = narrow8(kind == kKindProduce ? cptype : kAbsent);
            g.pending_issued_at[slot] = time;
            g.pending_completes_at[slot] = time + duration;
            g.pending_order[slot] = appends ? g.s[kSNextOrder] : held;
            if (appends) g.s[kSNextOrder] += 1;
            if (claims_kind(kind)) X.ch[holders] = static_cast<int16_t>(slot);
        }
        if (claims_kind(kind)) ++holders;
        __syncwarp();
    }
}

// ---------------------------------------------------------------------------
// Completion (completion.py:30-79).
// ---------------------------------------------------------------------------
__device__ void complete(const Params& P, const Header& H, Game& g, const Scratch& X, int lane) {
    const int32_t N = P.neutral, E = P.entities, C = P.capacity;
    const int32_t time = static_cast<int32_t>(static_cast<uint32_t>(g.s[kSTime]) + 1u);  // pending.select, wrapping
    __syncwarp();
    if (lane == 0) g.s[kSTime] = time;
    // Acting owned members (completed, kind != NONE), in pending order.
    const int32_t M = warp_compact(P.owned, lane, X.req, [&](int32_t p) {
        const int32_t s = N + p;
        const int32_t pk = g.pending_kind[s];
        return pk != kAbsent && pk != kKindNone && g.pending_completes_at[s] <= time;
    });
    for (int32_t i = lane; i < M; i += 32) {
        const int32_t si = N + X.req[i];
        const int32_t oi = g.pending_order[si];
        int32_t rank = 0;
        for (int32_t j = 0; j < M; ++j) {
            const int32_t sj = N + X.req[j];
            const int32_t oj = g.pending_order[sj];
            rank += oj < oi || (oj == oi && sj < si);
        }
        X.ord[rank] = static_cast<int16_t>(si);
        Retained r;
        r.birth = g.birth[si];
        r.carried = g.carried[si];
        r.cell = g.cell[si];
        r.target = g.pending_target_cell[si];
        r.kind = g.pending_kind[si];
        r.direction = g.pending_direction[si];
        r.produced_type = g.pending_produced_type[si];
        r.owner = g.owner[si];
        r.unit_type = g.unit_type[si];
        X.ret[rank] = r;
    }
    __syncwarp();
    // pending.clear of every completed slot.
    for (int32_t s = lane; s < E; s += 32) {
        if (g.pending_kind[s] != kAbsent && g.pending_completes_at[s] <= time) {
            g.pending_kind[s] = kAbsent;
            g.pending_direction[s] = kAbsent;
            g.pending_none_duration[s] = 0;
            g.pending_target_cell[s] = kAbsent;
            g.pending_produced_type[s] = kAbsent;
            g.pending_issued_at[s] = 0;
            g.pending_completes_at[s] = 0;
            g.pending_order[s] = kAbsent;
        }
    }
    __syncwarp();
    for (int32_t m = 0; m < M; ++m) {
        const int32_t slot = X.ord[m];
        const Retained r = X.ret[m];
        const int32_t kind = r.kind;
        const int32_t player = clampi(r.owner, 0, kPlayers - 1);
        // units.lowest_free_slot over the player's block, by ballot.
        int32_t newborn = -1;
        if (kind == kKindProduce) {
            const int32_t start = N + player * C;
            for (int32_t base = 0; base < C && newborn < 0; base += 32) {
                const int32_t i = base + lane;
                const unsigned m2 = __ballot_sync(kFull, i < C && !g.active(start + i));
                if (m2) newborn = start + base + __ffs(m2) - 1;
            }
        }
        if (lane == 0) {
            const int32_t cells = P.cells;
            const int32_t actor = clampi(r.unit_type, 0, P.types - 1);
            const bool alive = g.active(slot) && g.birth[slot] == r.birth;
            const int32_t destination = reserved_position(r.cell, r.direction, P.width);
            bool removes = false;
            int32_t removed = 0;
            if (kind == kKindMove) {  // move.py:24-32
                if (alive) {
                    if (destination >= 0 && destination < cells) g.entity_at[destination] = static_cast<int16_t>(slot);
                    if (r.cell >= 0 && r.cell < cells) g.entity_at[r.cell] = kAbsent;
                    g.cell[slot] = static_cast<int16_t>(destination);
                }
            } else if (kind == kKindHarvest) {  // harvest.py:30-58
                const Neighbour nb = neighbour(P, H, g, r.cell, r.direction);
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
                const Neighbour nb = neighbour(P, H, g, r.cell, r.direction);
                if (nb.occupied && H.at(nb.unit_type, kIsStockpile) && r.carried > 0) {
                    if (alive) g.carried[slot] = 0;
                    g.s[kSRes0 + player] += r.carried;
                }
            } else if (kind == kKindProduce) {  // produce.py:49-89
                const int32_t newborn_type = clampi(r.produced_type, 0, P.types - 1);
                const int32_t balance = g.s[kSRes0 + player] - H.at(newborn_type, kCost);
                if (balance >= 0) {
                    if (newborn >= 0) {
                        g.s[kSRes0 + player] = balance;
                        if (destination >= 0 && destination < cells) g.entity_at[destination] = static_cast<int16_t>(newborn);
                        g.birth[newborn] = g.s[kSNextBirth];
                        g.unit_type[newborn] = narrow8(newborn_type);
                        g.owner[newborn] = narrow8(player);
                        g.cell[newborn] = static_cast<int16_t>(destination);
                        g.hit_points[newborn] = static_cast<int16_t>(H.at(newborn_type, kHitPoints));
                        g.s[kSNextBirth] += 1;
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
            if (removes) {  // completion.py:67 and units.remove
                const int32_t at = g.cell[removed];
                if (at >= 0 && at < cells) g.entity_at[at] = kAbsent;
                g.birth[removed] = kAbsent;
                g.unit_type[removed] = kAbsent;
                g.owner[removed] = kAbsent;
                g.cell[removed] = kAbsent;
                g.hit_points[removed] = 0;
                g.carried[removed] = 0;
                g.pending_kind[removed] = kAbsent;
                g.pending_direction[removed] = kAbsent;
                g.pending_none_duration[removed] = 0;
                g.pending_target_cell[removed] = kAbsent;
                g.pending_produced_type[removed] = kAbsent;
                g.pending_issued_at[removed] = 0;
                g.pending_completes_at[removed] = 0;
                g.pending_order[removed] = kAbsent;
            }
        }
        __syncwarp();
    }
}

// outcome.py:11-37 on the slab; returns terminated, truncated through refs.
__device__ void decide(const Params& P, Game& g, int lane, bool& terminated, bool& truncated) {
    bool surviving[kPlayers];
    for (int p = 0; p < kPlayers; ++p) {
        bool any = false;
        const int32_t start = P.neutral + p * P.capacity;
        for (int32_t base = 0; base < P.capacity; base += 32) {
            const int32_t i = base + lane;
            any |= __any_sync(kFull, i < P.capacity && g.active(start + i));
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

// ---------------------------------------------------------------------------
// Epilogue: legality rows and observations.
// ---------------------------------------------------------------------------
// Row bits of the cells whose occupant belongs to each player: the owner
// plane of board_view (model/board_view.py:44-69), read through entity_at.
__device__ void occupancy_rows(const Params& P, const Game& g, uint64_t* occ, int lane) {
    for (int32_t r = lane; r < 2 * P.height; r += 32) occ[r] = 0ull;
    __syncwarp();
    for (int32_t cell = lane; cell < P.cells; cell += 32) {
        const int32_t s = g.entity_at[cell];
        if (s == kAbsent) continue;
        const int32_t owner = g.owner[s];
        if (owner < 0 || owner >= kPlayers) continue;
        atomicOr(reinterpret_cast<unsigned long long*>(&occ[owner * P.height + cell / P.width]), 1ull << (cell % P.width));
    }
    __syncwarp();
}

// Disks of sight (visibility.py:70-77) of each player's units, as row bits.
__device__ void visibility_rows(const Params& P, const Header& H, const Game& g, uint64_t* vis, int lane) {
    for (int32_t r = lane; r < 2 * P.height; r += 32) vis[r] = 0ull;
    __syncwarp();
    for (int32_t p = lane; p < P.owned; p += 32) {
        const int32_t s = P.neutral + p;
        if (!g.active(s)) continue;
        const int32_t player = p / P.capacity;
        const int32_t cell = g.cell[s];
        const int32_t radius = H.at(clampi(g.unit_type[s], 0, P.types - 1), kSightRadius);
        const int32_t ux = floor_mod(cell, P.width), uy = floor_div(cell, P.width);
        for (int32_t dy = -radius; dy <= radius; ++dy) {
            const int32_t y = uy + dy;
            if (y < 0 || y >= P.height) continue;
            int32_t half = 0;
            while ((half + 1) * (half + 1) + dy * dy <= radius * radius) ++half;
            const int32_t lo = max(ux - half, 0), hi = min(ux + half, P.width - 1);
            if (lo > hi) continue;
            const uint64_t bits = (hi - lo == 63) ? ~0ull : (((1ull << (hi - lo + 1)) - 1ull) << lo);
            atomicOr(reinterpret_cast<unsigned long long*>(&vis[player * P.height + y]), bits);
        }
    }
    __syncwarp();
}

// 78-bit legality row of one owned slot (legality.py:32-64, actions.py:28-41).
__device__ void legality_words(const Params& P, const Header& H, const Game& g, const uint64_t* occ, int32_t p, uint32_t* w) {
    const int32_t slot = P.neutral + p;
    const bool available = g.active(slot) && g.pending_kind[slot] == kAbsent;
    if (!available) {
        w[0] = 1u;
        w[1] = 0u;
        w[2] = 0u;
        return;
    }
    const int32_t actor = clampi(g.unit_type[slot], 0, P.types - 1);
    const int32_t owner = g.owner[slot];
    const int32_t carried = g.carried[slot];
    const int32_t cell = g.cell[slot];
    const int32_t balance = g.s[kSRes0 + clampi(owner, 0, kPlayers - 1)];
    uint32_t move = 0, harvest = 0, ret = 0, free = 0;
    const bool can_move = H.at(actor, kCanMove), can_harvest = H.at(actor, kCanHarvest);
#pragma unroll
    for (int d = 0; d < kDirections; ++d) {
        const Neighbour n = neighbour(P, H, g, cell, d);
        free |= static_cast<uint32_t>(n.free) << d;
        move |= static_cast<uint32_t>(can_move && n.free) << d;
        harvest |= static_cast<uint32_t>(can_harvest && carried == 0 && n.occupied && H.at(n.unit_type, kIsResource)) << d;
        ret |= static_cast<uint32_t>(can_harvest && carried > 0 && n.occupied && H.at(n.unit_type, kIsStockpile) && n.owner == owner) << d;
    }
    uint32_t type_ok = 0;
    for (int32_t t = 0; t < P.types; ++t) type_ok |= static_cast<uint32_t>(H.produces(actor, t) && balance >= H.at(t, kCost)) << t;
    const uint32_t pdir = type_ok ? free : 0u;
    const uint32_t ptype = free ? type_ok : 0u;
    // Attack window: opponent-occupied cells within range.
    uint64_t attack = 0;
    const uint64_t in_range = H.attack_window[actor];
    if (in_range != 0 && owner >= 0 && owner < kPlayers) {
        const uint64_t* enemy = occ + (1 - owner) * P.height;
        const int32_t cx = floor_mod(cell, P.width), cy = floor_div(cell, P.width);
        const int32_t R = P.radius, side = P.side;
        const uint64_t row_mask = (1ull << side) - 1ull;
        for (int32_t dy = -R; dy <= R; ++dy) {
            const int32_t y = cy + dy;
            if (y < 0 || y >= P.height) continue;
            const uint64_t bits = enemy[y];
            const int32_t x0 = cx - R;
            const uint64_t window = x0 >= 0 ? (bits >> x0) : (bits << (-x0));
            attack |= (window & row_mask) << ((dy + R) * side);
        }
        attack &= in_range;
    }
    const uint32_t kinds = 1u | (static_cast<uint32_t>(move != 0) << kKindMove) | (static_cast<uint32_t>(harvest != 0) << kKindHarvest) |
                           (static_cast<uint32_t>(ret != 0) << kKindReturn) |
                           (static_cast<uint32_t>(type_ok != 0 && free != 0) << kKindProduce) |
                           (static_cast<uint32_t>(attack != 0) << kKindAttack);
    const int a = kKinds + 4 * kDirections + P.types;  // first attack column
    const uint64_t lo = static_cast<uint64_t>(kinds) | (static_cast<uint64_t>(move) << 6) | (static_cast<uint64_t>(harvest) << 10) |
                        (static_cast<uint64_t>(ret) << 14) | (static_cast<uint64_t>(pdir) << 18) | (static_cast<uint64_t>(ptype) << 22) |
                        (attack << a);
    const uint64_t hi = attack >> (64 - a);
    w[0] = static_cast<uint32_t>(lo);
    w[1] = static_cast<uint32_t>(lo >> 32);
    w[2] = static_cast<uint32_t>(hi);
}

// 32 row bits starting at column c of row r (rows of 3 words, a zero word after).
__device__ __forceinline__ uint32_t row_bits(const uint32_t* words, int32_t r, int32_t c) {
    const uint32_t* w = words + r * 3;
    const int wi = c >> 5, b = c & 31;
    const uint32_t a0 = wi < 3 ? w[wi] : 0u;
    const uint32_t a1 = wi + 1 < 3 ? w[wi + 1] : 0u;
    return __funnelshift_r(a0, a1, b);
}

// Writes one player's legality rows [C, width] of this game as bytes.
__device__ void write_masks(const Params& P, const uint32_t* words, int player, int64_t game, uint8_t* out, int lane) {
    const int32_t width = P.mask_width, C = P.capacity;
    const int64_t span = static_cast<int64_t>(C) * width;
    uint8_t* base = out + game * span;
    const uintptr_t start = reinterpret_cast<uintptr_t>(base);
    const uintptr_t first = start & ~uintptr_t{15};
    const uintptr_t end = start + span;
    const uint32_t* rows = words + player * C * 3;
    for (uintptr_t q = first + 16u * lane; q < end; q += 16u * 32u) {
        const int64_t o = static_cast<int64_t>(q) - static_cast<int64_t>(start);
        if (o >= 0 && q + 16 <= end) {
            const int32_t r0 = static_cast<int32_t>(o / width), c0 = static_cast<int32_t>(o % width);
            const int32_t n0 = min(16, width - c0);
            uint32_t bits = row_bits(rows, r0, c0);
            bits &= (1u << n0) - 1u;
            if (n0 < 16) bits |= row_bits(rows, r0 + 1, 0) << n0;
            uint4 v;
            v.x = spread4(bits & 0xfu);
            v.y = spread4((bits >> 4) & 0xfu);
            v.z = spread4((bits >> 8) & 0xfu);
            v.w = spread4((bits >> 12) & 0xfu);
            *reinterpret_cast<uint4*>(q) = v;
        } else {
            for (int b = 0; b < 16; ++b) {
                const int64_t ob = o + b;
                if (ob < 0 || ob >= span) continue;
                const int32_t r = static_cast<int32_t>(ob / width), c = static_cast<int32_t>(ob % width);
                reinterpret_cast<uint8_t*>(q)[b] = static_cast<uint8_t>((row_bits(rows, r, c) & 1u));
            }
        }
    }
}

// Six feature bytes of one cell for `player` (symbolic.py:130-168), packed little-endian.
__device__ __forceinline__ uint64_t cell_features(const Params& P, const Header& H, const Game& g, const uint64_t* vis, int player,
                                                  int32_t cell) {
    const int32_t s = g.entity_at[cell];
    uint32_t hp = 0, carried = 0, type = 0, pending = 0, owner = 0;
    if (s != kAbsent) {
        hp = static_cast<uint32_t>(static_cast<int32_t>(g.hit_points[s])) & 0xffu;
        carried = static_cast<uint32_t>(g.carried[s]) & 0xffu;
        type = static_cast<uint32_t>(g.unit_type[s] + 1) & 0xffu;
        pending = static_cast<uint32_t>(max(static_cast<int32_t>(g.pending_kind[s]), kKindNone)) & 0xfu;
        owner = static_cast<uint32_t>(g.owner[s] + 1) & 0x3u;
        if (P.partial) {
            const bool seen = (vis[player * P.height + cell / P.width] >> (cell % P.width)) & 1ull;
            if (!(owner == static_cast<uint32_t>(player + 1) || seen)) hp = carried = type = pending = owner = 0;
        }
    }
    const uint32_t rel = owner > 0 ? ((owner - 1 + player) % kPlayers) + 1 : 0u;
    const uint32_t wall = H.wall(cell, P.width) ? 1u : 0u;
    return static_cast<uint64_t>(hp) | (static_cast<uint64_t>(carried) << 8) | (static_cast<uint64_t>(rel) << 16) |
           (static_cast<uint64_t>(type) << 24) | (static_cast<uint64_t>(pending) << 32) | (static_cast<uint64_t>(wall) << 40);
}

__device__ void write_observation(const Params& P, const Header& H, const Game& g, const uint64_t* vis, int player, int64_t game,
                                  uint8_t* maps, int32_t* scalars, int lane) {
    if (maps != nullptr) {
        const int32_t cells = P.cells;
        uint8_t* base = maps + game * static_cast<int64_t>(cells) * kFeatures;
        const bool grouped = (cells % 8 == 0) && ((reinterpret_cast<uintptr_t>(base) & 15u) == 0);
        if (grouped) {
            // 8 cells = 48 bytes = three 16-byte stores.
            for (int32_t c0 = lane * 8; c0 < cells; c0 += 32 * 8) {
                uint32_t w[12];
#pragma unroll
                for (int k = 0; k < 12; ++k) w[k] = 0;
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    const uint64_t f = cell_features(P, H, g, vis, player, c0 + c);
#pragma unroll
                    for (int b = 0; b < kFeatures; ++b) {
                        const int pos = c * kFeatures + b;
                        w[pos >> 2] |= static_cast<uint32_t>((f >> (8 * b)) & 0xffu) << (8 * (pos & 3));
                    }
                }
                uint4* dst = reinterpret_cast<uint4*>(base + c0 * kFeatures);
                dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
                dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
                dst[2] = make_uint4(w[8], w[9], w[10], w[11]);
            }
        } else {
            for (int32_t c = lane; c < cells; c += 32) {
                const uint64_t f = cell_features(P, H, g, vis, player, c);
                for (int b = 0; b < kFeatures; ++b) base[c * kFeatures + b] = static_cast<uint8_t>(f >> (8 * b));
            }
        }
    }
    if (scalars != nullptr && lane == 0) {
        int4 v = make_int4(g.s[kSRes0 + player], g.s[kSRes0 + 1 - player], g.s[kSTime], g.s[kSAlt]);
        *reinterpret_cast<int4*>(scalars + game * kScalars) = v;
    }
}

__device__ void write_outputs(const Params& P, const Header& H, const Game& g, const Scratch& X, int64_t game, uint8_t* const masks[2],
                              uint8_t* const maps[2], int32_t* const scalars[2], int lane) {
    uint64_t* occ = X.bits;
    uint64_t* vis = X.bits + 2 * P.height;
    if (masks[0] != nullptr || masks[1] != nullptr) {
        occupancy_rows(P, g, occ, lane);
        for (int32_t p = lane; p < P.owned; p += 32) legality_words(P, H, g, occ, p, X.words + p * 3);
        __syncwarp();
        for (int player = 0; player < kPlayers; ++player) {
            if (masks[player] != nullptr) write_masks(P, X.words, player, game, masks[player], lane);
        }
    }
    if (maps[0] != nullptr || maps[1] != nullptr || scalars[0] != nullptr || scalars[1] != nullptr) {
        if (P.partial) visibility_rows(P, H, g, vis, lane);
        for (int player = 0; player < kPlayers; ++player) write_observation(P, H, g, vis, player, game, maps[player], scalars[player], lane);
    }
    __syncwarp();
}

// ---------------------------------------------------------------------------
// The kernel.
// ---------------------------------------------------------------------------
__device__ Header setup_header(const Params& P, char* smem) {
    Header H;
    H.terrain_rows = reinterpret_cast<uint64_t*>(smem);
    H.attack_window = H.terrain_rows + P.height;
    H.table = reinterpret_cast<int32_t*>(H.attack_window + kMaxTypes);
    H.stride = kColumns + P.types;
    for (int32_t r = threadIdx.x; r < P.height; r += blockDim.x) {
        uint64_t bits = 0;
        for (int32_t x = 0; x < P.width; ++x) bits |= static_cast<uint64_t>(P.terrain[r * P.width + x] != 0) << x;
        H.terrain_rows[r] = bits;
    }
    for (int32_t i = threadIdx.x; i < P.types * H.stride; i += blockDim.x) H.table[i] = P.table[i];
    for (int32_t t = threadIdx.x; t < P.types; t += blockDim.x) {
        const int32_t range = P.table[t * H.stride + kAttackRange];
        uint64_t window = 0;
        if (P.table[t * H.stride + kCanAttack] != 0) {
            for (int32_t o = 0; o < P.offsets; ++o) {
                const int32_t dx = o % P.side - P.radius, dy = o / P.side - P.radius;
                if (dx * dx + dy * dy <= range * range) window |= 1ull << o;
            }
        }
        H.attack_window[t] = window;
    }
    return H;
}

__global__ void __launch_bounds__(256) step_kernel(const __grid_constant__ Params P) {
    extern __shared__ __align__(128) char smem[];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int warps = blockDim.x >> 5;
    const Layout& L = P.layout;
    Header H = setup_header(P, smem);
    char* slab = smem + L.header_bytes + warp * L.slab_bytes;
    uint64_t* bar = reinterpret_cast<uint64_t*>(slab + L.bar_off);
    if (lane == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    const int64_t game = static_cast<int64_t>(blockIdx.x) * warps + warp;
    if (game >= P.lanes) return;
    Game g = game_view(P, slab, game);
    const Scratch X = scratch_view(L, slab);

    if (P.mode == kModeReset) {
        load_reset(P, slab, game, lane);
        if (lane == 0) {
            g.s[kSEpisode] = 0;
            g.s[kSRoot0] = static_cast<int32_t>(P.keys[2 * game]);
            g.s[kSRoot1] = static_cast<int32_t>(P.keys[2 * game + 1]);
        }
        __syncwarp();
    } else {
        if (!stage_state(P, slab, game, bar, lane)) return;
    }

    if (P.mode == kModeStep) {
        admit(P, H, g, X, game, lane);
        complete(P, H, g, X, lane);
        bool terminated, truncated;
        decide(P, g, lane, terminated, truncated);
        const bool done = terminated || truncated;
        if (lane == 0) {
            const NrtsOutputs& o = P.out;
            const int32_t winner = g.s[kSWinner];
            if (o.reward) {
                float2 r;
                r.x = done ? (winner == 0 ? 1.f : -1.f) : 0.f;
                r.y = done ? (winner == 1 ? 1.f : -1.f) : 0.f;
                reinterpret_cast<float2*>(o.reward)[game] = r;
            }
            if (o.done) o.done[game] = done;
            if (o.terminated) o.terminated[game] = terminated;
            if (o.truncated) o.truncated[game] = truncated;
            if (o.winner) o.winner[game] = winner;
            if (o.spawn_overflow) reinterpret_cast<int2*>(o.spawn_overflow)[game] = make_int2(g.s[kSOverflow0], g.s[kSOverflow1]);
        }
        if (P.out.final_feature_maps[0] != nullptr || P.out.final_feature_maps[1] != nullptr ||
            P.out.final_scalars[0] != nullptr || P.out.final_scalars[1] != nullptr) {
            uint8_t* const no_masks[2] = {nullptr, nullptr};
            write_outputs(P, H, g, X, game, no_masks, P.out.final_feature_maps, P.out.final_scalars, lane);
        }
        if (done) {
            const int32_t episode = g.s[kSEpisode];
            const int32_t r0 = g.s[kSRoot0], r1 = g.s[kSRoot1];
            __syncwarp();
            load_reset(P, slab, game, lane);
            if (lane == 0) {
                g.s[kSEpisode] = static_cast<int32_t>(static_cast<uint32_t>(episode) + 1u);
                g.s[kSRoot0] = r0;
                g.s[kSRoot1] = r1;
            }
            __syncwarp();
        }
    }
    if (P.mode != kModeOutputs) store_state(P, slab, game, lane);
    write_outputs(P, H, g, X, game, P.out.masks, P.out.feature_maps, P.out.scalars, lane);
    if (P.mode != kModeOutputs && lane == 0) bulk_wait_read_all();
}

// Uniform legal draw per factor group (nrts_sample_actions).
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

__global__ void sample_kernel(int64_t rows, int32_t width, int32_t types, int32_t capacity, const uint8_t* masks0, const uint8_t* masks1,
                              int32_t* actions0, int32_t* actions1, uint64_t seed, uint64_t counter) {
    const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= 2 * rows) return;
    const int player = t >= rows;
    const int64_t row = player ? t - rows : t;
    const uint8_t* m = (player ? masks1 : masks0) + row * width;
    int32_t* a = (player ? actions1 : actions0) + row * kActionColumns;
    const int32_t widths[kActionColumns] = {kKinds, kDirections, kDirections, kDirections, kDirections, types, width - 22 - types};
    int32_t offset = 0;
    const uint64_t stream = mix64(seed ^ mix64(counter + 0x9e3779b97f4a7c15ull * static_cast<uint64_t>(t + 1)));
    for (int f = 0; f < kActionColumns; ++f) {
        int32_t count = 0;
        for (int32_t i = 0; i < widths[f]; ++i) count += m[offset + i] != 0;
        int32_t value = 0;
        if (count > 0) {
            const uint64_t h = mix64(stream + 0x632be59bd9b4e019ull * static_cast<uint64_t>(f + 1));
            int32_t pick = static_cast<int32_t>(((h >> 32) * static_cast<uint64_t>(count)) >> 32);
            for (int32_t i = 0; i < widths[f]; ++i) {
                if (m[offset + i] != 0) {
                    if (pick == 0) {
                        value = i;
                        break;
                    }
                    --pick;
                }
            }
        }
        a[f] = value;
        offset += widths[f];
    }
}

__global__ void slot_cells_kernel(int64_t lanes, int32_t entities, int32_t neutral, int32_t owned, const int32_t* birth,
                                  const int16_t* cell, int32_t* out) {
    const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (t >= lanes * owned) return;
    const int64_t game = t / owned;
    const int32_t p = static_cast<int32_t>(t % owned);
    const int64_t s = game * entities + neutral + p;
    out[t] = birth[s] == kAbsent ? -1 : static_cast<int32_t>(cell[s]);
}

__global__ void probe_kernel(int32_t* out) {
    const int lane = threadIdx.x & 31;
    const unsigned ballot = __ballot_sync(kFull, (lane & 1) != 0);
    const int shuffled = __shfl_sync(kFull, lane * 3, (lane + 5) & 31);
    if (lane == 0) out[0] = ballot == 0xaaaaaaaau;
    out[1 + lane] = shuffled == ((lane + 5) & 31) * 3;
}

}  // namespace nrts

// ===========================================================================
// Host side: validation, layout, launches.
// ===========================================================================
namespace {

using namespace nrts;

thread_local std::string g_last_error;

int fail(int code, const std::string& message) {
    g_last_error = message;
    return code;
}

int32_t round16(int64_t v) { return static_cast<int32_t>((v + 15) & ~int64_t{15}); }

int validate(const NrtsExtents* x) {
    if (x == nullptr) return fail(NRTS_E_ARGUMENT, "extents is null");
    if (x->height <= 0 || x->width <= 0 || x->width > kMaxWidth || x->height > kMaxHeight)
        return fail(NRTS_E_ARGUMENT, "the field must be between 1x1 and 64x64");
    if (x->capacity <= 0 || x->neutral < 0) return fail(NRTS_E_ARGUMENT, "slot capacities must be positive");
    if (x->neutral + 2 * x->capacity > 32767 || x->height * x->width > 32767)
        return fail(NRTS_E_ARGUMENT, "cell and slot indices must fit int16");
    if (x->types <= 0 || x->types > kMaxTypes) return fail(NRTS_E_ARGUMENT, "between 1 and 8 unit types are supported");
    int side = 1;
    while (side * side < x->offsets) ++side;
    if (side * side != x->offsets || side % 2 == 0 || side > 7) return fail(NRTS_E_ARGUMENT, "the attack window must be an odd square of side <= 7");
    if (kKinds + 4 * kDirections + x->types + x->offsets > kMaxMaskBits) return fail(NRTS_E_ARGUMENT, "legality rows wider than 96 columns");
    if (x->strategy < 0 || x->strategy > 2) return fail(NRTS_E_ARGUMENT, "unknown conflict strategy");
    return NRTS_OK;
}

int row_bytes_host(const NrtsExtents* x, int leaf) {
    const int E = x->neutral + 2 * x->capacity;
    switch (leaf) {
        case NRTS_BIRTH: case NRTS_CARRIED_RESOURCES: case NRTS_PENDING_NONE_DURATION: case NRTS_PENDING_ISSUED_AT:
        case NRTS_PENDING_COMPLETES_AT: case NRTS_PENDING_ORDER:
            return 4 * E;
        case NRTS_UNIT_TYPE: case NRTS_OWNER: case NRTS_PENDING_KIND: case NRTS_PENDING_DIRECTION:
        case NRTS_PENDING_PRODUCED_TYPE:
            return E;
        case NRTS_CELL: case NRTS_HIT_POINTS: case NRTS_PENDING_TARGET_CELL:
            return 2 * E;
        case NRTS_ENTITY_AT:
            return 2 * x->height * x->width;
        default:
            return 0;
    }
}

Layout make_layout(const NrtsExtents* x) {
    Layout L{};
    const int E = x->neutral + 2 * x->capacity;
    const int owned = 2 * x->capacity;
    int32_t off = 0;
    for (int k = 0; k < kSlabLeaves; ++k) {
        L.row_bytes[k] = row_bytes_host(x, k);
        L.leaf_off[k] = off;
        off += round16(L.row_bytes[k] + 16);
    }
    L.scal_off = off;
    off += round16(kSCount * 4);
    L.req_off = off;
    off += round16(owned * 2);
    L.ord_off = off;
    off += round16(owned * 2);
    L.ch_off = off;
    off += round16(E * 2);
    L.conf_off = off;
    off += round16(std::max(E * 2, 16));
    // Admission/completion scratch and epilogue scratch share one region.
    const int32_t union_start = off;
    L.cmd_off = union_start;
    L.ret_off = union_start + round16(owned * 8);
    const int32_t phase_a = round16(owned * 8) + round16(owned * static_cast<int>(sizeof(Retained)));
    L.words_off = union_start;
    L.bits_off = union_start + round16(owned * 12 + 8);
    const int32_t phase_b = round16(owned * 12 + 8) + round16(4 * x->height * 8);
    off = union_start + std::max(phase_a, phase_b);
    L.bar_off = off;
    off += 16;
    L.slab_bytes = round16(off);
    L.header_bytes = round16(x->height * 8 + kMaxTypes * 8 + x->types * (kColumns + x->types) * 4);
    return L;
}

struct DeviceInfo {
    int smem_optin = 0;
    int sms = 0;
    bool attributes_set = false;
};

DeviceInfo g_devices[64];

int prepare_device(int& device, DeviceInfo*& info) {
    if (cudaGetDevice(&device) != cudaSuccess) return fail(NRTS_E_CUDA, "cudaGetDevice failed");
    if (device < 0 || device >= 64) return fail(NRTS_E_CUDA, "device index out of range");
    info = &g_devices[device];
    if (!info->attributes_set) {
        cudaDeviceGetAttribute(&info->smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
        cudaDeviceGetAttribute(&info->sms, cudaDevAttrMultiProcessorCount, device);
        if (cudaFuncSetAttribute(step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, info->smem_optin) != cudaSuccess)
            return fail(NRTS_E_CUDA, "cudaFuncSetAttribute(step_kernel) failed");
        info->attributes_set = true;
    }
    return NRTS_OK;
}

int fill_params(Params& P, const NrtsExtents* x, const NrtsContent* content, const NrtsState* state, int64_t lanes) {
    if (int rc = validate(x)) return rc;
    if (content == nullptr || content->terrain == nullptr || content->table == nullptr) return fail(NRTS_E_ARGUMENT, "content is null");
    if (state == nullptr) return fail(NRTS_E_ARGUMENT, "state is null");
    if (lanes < 0) return fail(NRTS_E_ARGUMENT, "negative lane count");
    std::memset(&P, 0, sizeof(P));
    P.height = x->height;
    P.width = x->width;
    P.neutral = x->neutral;
    P.capacity = x->capacity;
    P.types = x->types;
    P.offsets = x->offsets;
    P.strategy = x->strategy;
    P.max_cycles = x->max_cycles;
    P.partial = x->partial_observability != 0;
    P.entities = x->neutral + 2 * x->capacity;
    P.cells = x->height * x->width;
    P.owned = 2 * x->capacity;
    int side = 1;
    while (side * side < x->offsets) ++side;
    P.side = side;
    P.radius = (side - 1) / 2;
    P.mask_width = kKinds + 4 * kDirections + x->types + x->offsets;
    P.lanes = lanes;
    for (int k = 0; k < NRTS_LEAVES; ++k) {
        if (state->leaf[k] == nullptr) return fail(NRTS_E_ARGUMENT, "a state leaf is null");
        P.leaf[k] = state->leaf[k];
        if (content->reset[k] == nullptr) return fail(NRTS_E_ARGUMENT, "a reset leaf is null");
        P.reset[k] = content->reset[k];
    }
    for (int k = 0; k < NRTS_LEAVES; ++k) {
        const uintptr_t a = reinterpret_cast<uintptr_t>(state->leaf[k]);
        if (a % 4 != 0) return fail(NRTS_E_ARGUMENT, "state leaves must be 4-byte aligned");
    }
    if (state->environment_root == nullptr || state->episode_index == nullptr) return fail(NRTS_E_ARGUMENT, "lifecycle leaves are null");
    P.root = state->environment_root;
    P.episode = state->episode_index;
    P.terrain = content->terrain;
    P.table = content->table;
    P.layout = make_layout(x);
    return NRTS_OK;
}

int launch_step(Params& P, void* stream) {
    int device;
    DeviceInfo* info;
    if (int rc = prepare_device(device, info)) return rc;
    if (P.lanes == 0) return NRTS_OK;
    const Layout& L = P.layout;
    int warps = 8;
    while (warps > 1 && L.header_bytes + warps * L.slab_bytes > info->smem_optin) warps /= 2;
    if (L.header_bytes + warps * L.slab_bytes > info->smem_optin) return fail(NRTS_E_ARGUMENT, "one game does not fit in shared memory");
    // Prefer smaller CTAs when the whole batch would not fill the device.
    while (warps > 2 && (P.lanes + warps - 1) / warps < 2 * info->sms) warps /= 2;
    const int64_t blocks = (P.lanes + warps - 1) / warps;
    const size_t smem = L.header_bytes + static_cast<size_t>(warps) * L.slab_bytes;
    step_kernel<<<static_cast<unsigned>(blocks), warps * 32, smem, static_cast<cudaStream_t>(stream)>>>(P);
    const cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess) return fail(NRTS_E_CUDA, std::string("step kernel launch: ") + cudaGetErrorString(err));
    return NRTS_OK;
}

}  // namespace

extern "C" {

int nrts_step(const NrtsExtents* extents, const NrtsContent* content, const NrtsState* state, int64_t lanes, const int32_t* actions0,
              const int32_t* actions1, const NrtsOutputs* outputs, void* stream) {
    Params P;
    if (int rc = fill_params(P, extents, content, state, lanes)) return rc;
    if (actions0 == nullptr || actions1 == nullptr) return fail(NRTS_E_ARGUMENT, "actions are null");
    if (outputs == nullptr) return fail(NRTS_E_ARGUMENT, "outputs is null");
    P.mode = kModeStep;
    P.actions[0] = actions0;
    P.actions[1] = actions1;
    P.out = *outputs;
    return launch_step(P, stream);
}

int nrts_reset(const NrtsExtents* extents, const NrtsContent* content, const NrtsState* state, int64_t lanes, const uint32_t* keys,
               const NrtsOutputs* outputs, void* stream) {
    Params P;
    if (int rc = fill_params(P, extents, content, state, lanes)) return rc;
    if (keys == nullptr) return fail(NRTS_E_ARGUMENT, "keys are null");
    P.mode = kModeReset;
    P.keys = keys;
    if (outputs != nullptr) {
        P.out.masks[0] = outputs->masks[0];
        P.out.masks[1] = outputs->masks[1];
        P.out.feature_maps[0] = outputs->feature_maps[0];
        P.out.feature_maps[1] = outputs->feature_maps[1];
        P.out.scalars[0] = outputs->scalars[0];
        P.out.scalars[1] = outputs->scalars[1];
    }
    return launch_step(P, stream);
}

int nrts_legal_masks(const NrtsExtents* extents, const NrtsContent* content, const NrtsState* state, int64_t lanes, uint8_t* masks0,
                     uint8_t* masks1, void* stream) {
    Params P;
    if (int rc = fill_params(P, extents, content, state, lanes)) return rc;
    P.mode = kModeOutputs;
    P.out.masks[0] = masks0;
    P.out.masks[1] = masks1;
    return launch_step(P, stream);
}

int nrts_observe(const NrtsExtents* extents, const NrtsContent* content, const NrtsState* state, int64_t lanes, uint8_t* feature_maps0,
                 uint8_t* feature_maps1, int32_t* scalars0, int32_t* scalars1, void* stream) {
    Params P;
    if (int rc = fill_params(P, extents, content, state, lanes)) return rc;
    P.mode = kModeOutputs;
    P.out.feature_maps[0] = feature_maps0;
    P.out.feature_maps[1] = feature_maps1;
    P.out.scalars[0] = scalars0;
    P.out.scalars[1] = scalars1;
    return launch_step(P, stream);
}

int nrts_slot_cells(const NrtsExtents* extents, const NrtsState* state, int64_t lanes, int32_t* cells, void* stream) {
    if (int rc = validate(extents)) return rc;
    if (state == nullptr || cells == nullptr || state->leaf[NRTS_BIRTH] == nullptr || state->leaf[NRTS_CELL] == nullptr)
        return fail(NRTS_E_ARGUMENT, "null pointer");
    const int32_t owned = 2 * extents->capacity;
    const int64_t n = lanes * owned;
    if (n == 0) return NRTS_OK;
    slot_cells_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        lanes, extents->neutral + owned, extents->neutral, owned, static_cast<const int32_t*>(state->leaf[NRTS_BIRTH]),
        static_cast<const int16_t*>(state->leaf[NRTS_CELL]), cells);
    const cudaError_t err = cudaGetLastError();
    return err == cudaSuccess ? NRTS_OK : fail(NRTS_E_CUDA, cudaGetErrorString(err));
}

int nrts_sample_actions(const NrtsExtents* extents, int64_t lanes, const uint8_t* masks0, const uint8_t* masks1, int32_t* actions0,
                        int32_t* actions1, uint64_t seed, uint64_t counter, void* stream) {
    if (int rc = validate(extents)) return rc;
    if (!masks0 || !masks1 || !actions0 || !actions1) return fail(NRTS_E_ARGUMENT, "null pointer");
    const int64_t rows = lanes * extents->capacity;
    if (rows == 0) return NRTS_OK;
    const int32_t width = kKinds + 4 * kDirections + extents->types + extents->offsets;
    sample_kernel<<<static_cast<unsigned>((2 * rows + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        rows, width, extents->types, extents->capacity, masks0, masks1, actions0, actions1, seed, counter);
    const cudaError_t err = cudaGetLastError();
    return err == cudaSuccess ? NRTS_OK : fail(NRTS_E_CUDA, cudaGetErrorString(err));
}

int nrts_device_status(int device) {
    int previous;
    if (cudaGetDevice(&previous) != cudaSuccess) return fail(NRTS_E_CUDA, "cudaGetDevice failed");
    if (cudaSetDevice(device) != cudaSuccess) return fail(NRTS_E_CUDA, "cudaSetDevice failed");
    int32_t value = 0, zero = 0;
    cudaError_t err = cudaMemcpyFromSymbol(&value, g_status, sizeof(value));
    if (err == cudaSuccess) err = cudaMemcpyToSymbol(g_status, &zero, sizeof(zero));
    cudaSetDevice(previous);
    if (err != cudaSuccess) return fail(NRTS_E_CUDA, cudaGetErrorString(err));
    return value;
}

const char* nrts_build_id(void) { return "nanorts_b200 sm_100a " __DATE__ " " __TIME__; }

int nrts_self_check(const int32_t* devices, int64_t count) {
    int previous;
    if (cudaGetDevice(&previous) != cudaSuccess) return fail(NRTS_E_CUDA, "cudaGetDevice failed");
    for (int64_t i = 0; i < count; ++i) {
        if (cudaSetDevice(devices[i]) != cudaSuccess) return fail(NRTS_E_CUDA, "cudaSetDevice failed");
        cudaFuncAttributes attributes;
        const void* kernels[] = {reinterpret_cast<const void*>(step_kernel), reinterpret_cast<const void*>(sample_kernel),
                                 reinterpret_cast<const void*>(slot_cells_kernel), reinterpret_cast<const void*>(probe_kernel)};
        for (const void* k : kernels) {
            if (cudaFuncGetAttributes(&attributes, k) != cudaSuccess) {
                cudaSetDevice(previous);
                return fail(NRTS_E_CUDA, "a kernel image does not load on this device");
            }
        }
        int32_t* d = nullptr;
        int32_t h[33];
        if (cudaMalloc(&d, sizeof(h)) != cudaSuccess) {
            cudaSetDevice(previous);
            return fail(NRTS_E_CUDA, "cudaMalloc failed in the self check");
        }
        probe_kernel<<<1, 32>>>(d);
        const cudaError_t err = cudaMemcpy(h, d, sizeof(h), cudaMemcpyDeviceToHost);
        cudaFree(d);
        if (err != cudaSuccess) {
            cudaSetDevice(previous);
            return fail(NRTS_E_CUDA, cudaGetErrorString(err));
        }
        for (int k = 0; k < 33; ++k) {
            if (h[k] != 1) {
                cudaSetDevice(previous);
                return fail(NRTS_E_DEVICE, "warp ballot or shuffle returned a wrong value");
            }
        }
    }
    cudaSetDevice(previous);
    return NRTS_OK;
}

const char* nrts_last_error(void) { return g_last_error.c_str(); }

}  // extern "C"
