// Kernel parameters, the per-game shared-memory slab and its staging.
//
// A game's State rows (the per-slot leaves and entity_at, lane-major in HBM)
// are copied into the owning warp's slab with 1D TMA bulk copies that
// complete on the warp's mbarrier, and written back in place with TMA bulk
// stores; on wide boards the rules-only pending rows stay in HBM (kRulesRows).  A row's copy in the slab starts at its region plus the global
// address's offset within 16 bytes, so the row's 16-byte-aligned body maps
// onto 16-byte-aligned shared memory; unaligned heads and tails (rows of
// boards whose slot counts are not multiples of 16) are copied by the lanes.
#pragma once

#include <cstdint>

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
// Rows only the rules touch (pending direction, none duration, target cell,
// produced type, issued at, completes at, order).  On boards whose staged
// game would not fit a small slab (wide boards, one game per CTA) the rules
// read and write them in place in HBM (through L2, where the CTA's prefetch
// put them): the slab shrinks by a quarter and one more game fits per SM
// (64x64: 4 CTAs instead of 3, measured 15 % faster).  On small boards, where
// a warp's serial rules phases dominate, staging them measured faster.
constexpr uint32_t kRulesRows = (1u << NRTS_PENDING_DIRECTION) | (1u << NRTS_PENDING_NONE_DURATION) |
                                (1u << NRTS_PENDING_TARGET_CELL) | (1u << NRTS_PENDING_PRODUCED_TYPE) |
                                (1u << NRTS_PENDING_ISSUED_AT) | (1u << NRTS_PENDING_COMPLETES_AT) |
                                (1u << NRTS_PENDING_ORDER);
constexpr int32_t kNoCap = INT32_MAX;
constexpr uint64_t kWaitNanoseconds = 2000000000ull;  // bound on any wait: 2 s

enum Column : int {
    kCost, kHitPoints, kProduceTime, kMoveTime, kAttackTime, kHarvestTime, kAttackRange, kAttackDamage,
    kHarvestAmount, kSightRadius, kIsResource, kIsStockpile, kCanHarvest, kCanMove, kCanAttack, kColumns
};

enum Mode : int { kModeStep = 0, kModeReset = 1, kModeOutputs = 2, kModeDuel = 3, kModeBotAct = 4 };

// Scalar slots of a game's slab.
enum Scalar : int {
    kSTime, kSRes0, kSRes1, kSNextBirth, kSNextOrder, kSAlt, kSGameOver, kSWinner, kSOverflow0, kSOverflow1,
    kSEpisode, kSRoot0, kSRoot1, kSCount
};

// Byte offsets within a warp's slab (host-computed).
struct Layout {
    int32_t leaf_off[kSlabLeaves];
    int32_t row_bytes[kSlabLeaves];
    int32_t scal_off;
    int32_t list_off;    // int16 [2C]: requests, then members, then the available units
    int32_t order_off;   // int16 [2C]: sorted requests, then sorted members
    // Admission scratch.
    int32_t serial_off;  // int16 [2C] ranks of the contested requests (over `count`, read by then)
    int32_t scan_off;    // int16 [E]:  claim holders scanned by contested requests
    int32_t conf_off;    // int16 [E]:  conflicting holders
    int32_t key_off;     // uint32 [2C] sort keys
    int32_t info_off;    // ReqInfo [2C]
    int32_t rank_off;    // int16 [2C] admission rank of each owned slot's request (-1 none)
    int32_t count_off;   // uint32 [claim_words]: claims per cell (byte or 2-bit counters), 2 x uint32 produce claims, 2 x 5 int32 reward-component counts
    // Completion and outcome scratch (aliases admission scratch).
    int32_t free_off;    // uint32 [2 * ceil(C/32)]: free slots of each player block
    int32_t member_key_off;  // uint32 [2C] pending-order keys of the completing members
    int32_t ret_off;     // Retained [2C]
    // Epilogue scratch (aliases both, and `order` when no bots run).
    int32_t word_off;    // uint32 [cells] occupant words (per slot, [E], in slot-word layouts)
    int32_t rows_off;    // uint64 [4H] occupancy (2) and visibility (2) rows
    int32_t mask_off;    // uint32 [2C * 3 + 6] legality row words, then up to 4 per-warp counts
    // Scripted bots (duel and bot-act launches only; 0 otherwise).
    int32_t carry_off;   // two players' carries (bots.cuh carry_bytes each)
    int32_t cmd_off;     // command rows of both players (CmdLayout)
    int32_t bot_off;     // bot scratch (BotLayout), aliasing the admission scratch
    int32_t bar_off;     // mbarrier
    int32_t aligned;     // every leaf base and row is 16-byte aligned: rows copy whole, one TMA copy per lane
    int32_t total_bytes; // sum of the staged rows' row_bytes
    uint32_t hbm_rows;   // rows the rules use in place in HBM (kRulesRows or 0); the others are staged
    int32_t slab_bytes;
    int32_t header_bytes;  // CTA-wide constants: terrain rows, attack windows, unit table
};

struct Params {
    int32_t height, width, neutral, capacity, types, offsets, strategy, max_cycles, partial;
    int32_t entities, cells, owned, side, radius, mask_width, free_words;
    int32_t mode;
    int64_t lanes;
    void* leaf[NRTS_LEAVES];
    uint32_t* root;
    uint32_t* episode;
    const uint32_t* keys;  // reset mode
    const void* reset[NRTS_LEAVES];
    const int32_t* actions[kPlayers];
    int32_t* sampled[kPlayers];  // fused uniform draw of the next actions (optional)
    uint32_t sample_key;         // sample_key(seed, counter)
    NrtsOutputs out;
    NrtsBot bot[kPlayers];  // duel: both; bot-act: bot[bot_player]
    int32_t bot_player;     // bot-act: the acting player
    int32_t* commands;      // bot-act: Commands int32 [L, 6, 2, C]
    int32_t rank_bits;      // admission rank field width (admission.py:104-115)
    int32_t reverse;        // take the games last to first (NrtsOutputs.reverse_order)
    Layout layout;
    NrtsScenario scenario;  // copied to shared memory by every CTA
};

__host__ __device__ constexpr int32_t round16i(int32_t v) { return (v + 15) & ~15; }

// Command rows in the slab, one entry per owned slot [2C]: what a scripted
// bot issues and admission reads (Commands, model/commands.py:22-35).
struct CmdLayout {
    int32_t target, order, none, kind, dir, ptype, bytes;
};

__host__ __device__ inline CmdLayout cmd_layout(int32_t owned, int32_t base) {
    CmdLayout c;
    int32_t off = base;
    c.target = off;  off += round16i(owned * 2);
    c.order = off;  off += round16i(owned * 2);
    c.none = off;  off += round16i(owned * 2);
    c.kind = off;  off += round16i(owned);
    c.dir = off;  off += round16i(owned);
    c.ptype = off;  off += round16i(owned);
    c.bytes = off - base;
    return c;
}

struct Cmds {
    int16_t *target, *order, *none;
    int8_t *kind, *dir, *ptype;  // ptype clamped to [-1, T]: every out-of-range type decides alike
};

__device__ __forceinline__ Cmds cmd_view(const Params& P, char* slab) {
    const CmdLayout c = cmd_layout(P.owned, P.layout.cmd_off);
    Cmds m;
    m.target = reinterpret_cast<int16_t*>(slab + c.target);
    m.order = reinterpret_cast<int16_t*>(slab + c.order);
    m.none = reinterpret_cast<int16_t*>(slab + c.none);
    m.kind = reinterpret_cast<int8_t*>(slab + c.kind);
    m.dir = reinterpret_cast<int8_t*>(slab + c.dir);
    m.ptype = reinterpret_cast<int8_t*>(slab + c.ptype);
    return m;
}

// Per-CTA constants: the launch's NrtsScenario, copied to shared memory.
struct Header {
    const uint64_t* terrain_rows;   // [H] bit x of row y: wall
    const uint64_t* attack_window;  // [T] window cells within the type's attack range (0 if it cannot attack)
    const uint32_t* producible;     // [T] bit t: the type produces type t
    const int32_t* table;           // [T, kColumns + T]
    int32_t stride;
    uint32_t resource_types;        // bit t: type t is a resource
    uint32_t stockpile_types;       // bit t: type t is a stockpile
    __device__ __forceinline__ int32_t at(int32_t type, int column) const { return table[type * stride + column]; }
    __device__ __forceinline__ bool produces(int32_t producer, int32_t produced) const {
        return table[producer * stride + kColumns + produced] != 0;
    }
};

// Board geometry; kW > 0 fixes a power-of-two width at compile time.
template <int kW>
struct Geo {
    int32_t w, h, cells;
    __device__ __forceinline__ int32_t width() const {
        if constexpr (kW > 0) return kW; else return w;
    }
    // Coordinates of a cell index >= 0.
    __device__ __forceinline__ int32_t x(int32_t c) const {
        if constexpr (kW > 0) return c & (kW - 1); else return c % w;
    }
    __device__ __forceinline__ int32_t y(int32_t c) const {
        if constexpr (kW > 0) return c >> (31 - __clz(kW)); else return c / w;
    }
};

template <int kW>
__device__ __forceinline__ bool wall(const Header& H, const Geo<kW>& G, int32_t cell) {
    return (H.terrain_rows[G.y(cell)] >> G.x(cell)) & 1ull;
}

// One game's State in the warp's slab.
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
    __device__ __forceinline__ bool active(int32_t slot) const { return birth[slot] != kAbsent; }
    __device__ __forceinline__ void clear_pending(int32_t slot) const {
        pending_kind[slot] = kAbsent;
        pending_direction[slot] = kAbsent;
        pending_none_duration[slot] = 0;
        pending_target_cell[slot] = kAbsent;
        pending_produced_type[slot] = kAbsent;
        pending_issued_at[slot] = 0;
        pending_completes_at[slot] = 0;
        pending_order[slot] = kAbsent;
    }
    // units.remove (core/units.py:22-31): every per-slot leaf to its empty.
    __device__ __forceinline__ void remove(int32_t slot) const {
        birth[slot] = kAbsent;
        unit_type[slot] = kAbsent;
        owner[slot] = kAbsent;
        cell[slot] = kAbsent;
        hit_points[slot] = 0;
        carried[slot] = 0;
        clear_pending(slot);
    }
};

__device__ __forceinline__ int64_t leaf_row_bytes(const Params& P, int leaf) { return P.layout.row_bytes[leaf]; }

// Whether State row `leaf` lives in the slab, for a launch whose rows kHbm
// stay in HBM (a kernel template constant: every slab pointer then stays
// known to the compiler as shared memory).
template <uint32_t kHbm>
__host__ __device__ __forceinline__ constexpr bool staged_row(int leaf) {
    return leaf >= 0 && leaf < kSlabLeaves && !((kHbm >> leaf) & 1u);
}

__host__ __forceinline__ bool staged_row(const Layout& L, int leaf) {
    return leaf >= 0 && leaf < kSlabLeaves && !((L.hbm_rows >> leaf) & 1u);
}

__device__ __forceinline__ char* slab_row(char* slab, const Layout& L, int leaf, const void* global) {
    return slab + L.leaf_off[leaf] + (reinterpret_cast<uintptr_t>(global) & 15u);
}

__device__ __forceinline__ char* global_row(const Params& P, int leaf, int64_t game) {
    return static_cast<char*>(P.leaf[leaf]) + game * P.layout.row_bytes[leaf];
}

// A game's view: staged rows in the slab, rules-only rows in place in HBM.
template <uint32_t kHbm = 0>
__device__ __forceinline__ Game game_view(const Params& P, char* slab, int64_t game) {
    const Layout& L = P.layout;
    auto row = [&](int leaf) {
        char* global = global_row(P, leaf, game);
        return staged_row<kHbm>(leaf) ? slab_row(slab, L, leaf, global) : global;
    };
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

__device__ int32_t g_status;  // nonzero after a bounded wait gave up

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Waits for the warp's mbarrier phase, bounded in time; on timeout records the
// status code in `status` (the library's status word unless given) and waits
// once more (bounded) for copies still in flight.
__device__ bool wait_phase(uint64_t* bar, uint32_t parity, uint64_t limit_ns = kWaitNanoseconds, int32_t* status = nullptr) {
    const uint64_t start = global_ns();
    while (!mbar_try_wait(bar, parity)) {
        if (global_ns() - start > limit_ns) {
            atomicExch(status != nullptr ? status : &g_status, 1);
            const uint64_t again = global_ns();
            while (!mbar_try_wait(bar, parity) && global_ns() - again < limit_ns) {
            }
            return false;
        }
    }
    return true;
}

// Copies n < 16 bytes; every load issues before the first store.
__device__ __forceinline__ void copy_edge_in(char* dst, const char* src, uint32_t n) {
    uint8_t b[15];
#pragma unroll
    for (uint32_t i = 0; i < 15; ++i) b[i] = i < n ? __ldg(reinterpret_cast<const unsigned char*>(src) + i) : 0;
#pragma unroll
    for (uint32_t i = 0; i < 15; ++i)
        if (i < n) dst[i] = static_cast<char>(b[i]);
}

__device__ __forceinline__ void copy_edge_out(char* dst, const char* src, uint32_t n) {
    uint8_t b[15];
#pragma unroll
    for (uint32_t i = 0; i < 15; ++i) b[i] = i < n ? static_cast<uint8_t>(src[i]) : 0;
#pragma unroll
    for (uint32_t i = 0; i < 15; ++i)
        if (i < n) dst[i] = static_cast<char>(b[i]);
}

// The game's scalar leaves -> slab scalars, one per lane.  The warp-per-game
// kernels load them one lane after another (each case's load and store run
// before the next case's): measured on 16x16 with 23 games per SM, that
// pacing of the stage gives 101 M env-steps/s against 88 M for loading all 13
// at once, whose launches end on a longer tail of late warps.
__device__ __forceinline__ void load_scalars(const Params& P, char* slab, int64_t game, int lane) {
    const Layout& L = P.layout;
    int32_t* s = reinterpret_cast<int32_t*>(slab + L.scal_off);
    const int32_t* res = static_cast<const int32_t*>(P.leaf[NRTS_PLAYER_RESOURCES]);
    const int32_t* ov = static_cast<const int32_t*>(P.leaf[NRTS_SPAWN_OVERFLOW]);
    switch (lane) {
        case kSTime: s[kSTime] = static_cast<const int32_t*>(P.leaf[NRTS_TIME])[game]; break;
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
}

// The same, every lane loading at once (each lane picks its address first):
// the team and duel kernels' stage is shorter this way (measured: config 5
// +7.5 %, bot duels +3.4 %).
__device__ __forceinline__ void load_scalars_at_once(const Params& P, char* slab, int64_t game, int lane) {
    const Layout& L = P.layout;
    int32_t* s = reinterpret_cast<int32_t*>(slab + L.scal_off);
    const int32_t* res = static_cast<const int32_t*>(P.leaf[NRTS_PLAYER_RESOURCES]);
    const int32_t* ov = static_cast<const int32_t*>(P.leaf[NRTS_SPAWN_OVERFLOW]);
    const void* src = nullptr;
    switch (lane) {
        case kSTime: src = static_cast<const int32_t*>(P.leaf[NRTS_TIME]) + game; break;
        case kSRes0: src = res + 2 * game; break;
        case kSRes1: src = res + 2 * game + 1; break;
        case kSNextBirth: src = static_cast<const int32_t*>(P.leaf[NRTS_NEXT_BIRTH]) + game; break;
        case kSNextOrder: src = static_cast<const int32_t*>(P.leaf[NRTS_NEXT_PENDING_ORDER]) + game; break;
        case kSAlt: src = static_cast<const int32_t*>(P.leaf[NRTS_ALTERNATING_CONFLICT_COUNT]) + game; break;
        case kSGameOver: src = static_cast<const uint8_t*>(P.leaf[NRTS_GAME_OVER]) + game; break;
        case kSWinner: src = static_cast<const int32_t*>(P.leaf[NRTS_WINNER]) + game; break;
        case kSOverflow0: src = ov + 2 * game; break;
        case kSOverflow1: src = ov + 2 * game + 1; break;
        case kSEpisode: src = P.episode + game; break;
        case kSRoot0: src = P.root + 2 * game; break;
        case kSRoot1: src = P.root + 2 * game + 1; break;
        default: break;
    }
    if (src != nullptr) {
        const int32_t v = lane == kSGameOver ? static_cast<int32_t>(__ldg(static_cast<const uint8_t*>(src)))
                                             : __ldg(static_cast<const int32_t*>(src));
        s[lane] = v;
    }
}

// L2 prefetch of a game's State rows and action rows (their 16-byte-aligned
// parts), issued one game ahead by warps that step several games.
__device__ __forceinline__ void prefetch_game(const Params& P, int64_t game, int lane) {
    if (lane < kSlabLeaves) {
        const char* src = global_row(P, lane, game);
        const Span sp = split_row(src, P.layout.row_bytes[lane]);
        if (sp.body) bulk_prefetch_l2(src + sp.head, sp.body);
    } else if (lane == 16 || lane == 17) {
        const int64_t span = static_cast<int64_t>(P.capacity) * kActionColumns * 4;
        const uintptr_t base = reinterpret_cast<uintptr_t>(P.actions[lane - 16]);
        const uintptr_t begin = (base + game * span + 15) & ~uintptr_t{15};
        const uintptr_t end = (base + (game + 1) * span) & ~uintptr_t{15};
        if (end > begin) bulk_prefetch_l2(reinterpret_cast<const void*>(begin), static_cast<uint32_t>(end - begin));
    }
}

// Global rows -> slab; scalar leaves -> slab scalars.
template <uint32_t kHbm = 0>
__device__ bool stage_state(const Params& P, char* slab, int64_t game, uint64_t* bar, uint32_t parity, int lane,
                            bool scalars_at_once = false) {
    const Layout& L = P.layout;
    if (P.mode == kModeStep && (lane == 16 || lane == 17)) {
        // The game's action rows are read during admission: pull their
        // 16-byte-aligned part into L2 now.
        const int64_t span = static_cast<int64_t>(P.capacity) * kActionColumns * 4;
        const uintptr_t base = reinterpret_cast<uintptr_t>(P.actions[lane - 16]);
        const uintptr_t begin = (base + game * span + 15) & ~uintptr_t{15};
        const uintptr_t end = (base + (game + 1) * span) & ~uintptr_t{15};
        if (end > begin) bulk_prefetch_l2(reinterpret_cast<const void*>(begin), static_cast<uint32_t>(end - begin));
    }
    const bool mine = staged_row<kHbm>(lane);
    if (L.aligned) {
        if (lane == 0) mbar_arrive_expect_tx(bar, static_cast<uint32_t>(L.total_bytes));
        __syncwarp();
        if (mine) bulk_load(slab + L.leaf_off[lane], global_row(P, lane, game), L.row_bytes[lane], bar);
    } else {
        // Lane k owns row k: the TMA bulk copy of its 16-byte-aligned body and
        // its own unaligned head and tail bytes.
        const char* src = mine ? global_row(P, lane, game) : nullptr;
        const Span sp = mine ? split_row(src, L.row_bytes[lane]) : Span{0, 0, 0};
        const uint32_t total = __reduce_add_sync(kFull, sp.body);
        if (lane == 0) mbar_arrive_expect_tx(bar, total);
        __syncwarp();
        if (mine) {
            char* dst = slab_row(slab, L, lane, src);
            if (sp.body) bulk_load(dst + sp.head, src + sp.head, sp.body, bar);
            copy_edge_in(dst, src, sp.head);
            copy_edge_in(dst + sp.head + sp.body, src + sp.head + sp.body, sp.tail);
        }
    }
    if (scalars_at_once) load_scalars_at_once(P, slab, game, lane);
    else load_scalars(P, slab, game, lane);
    const bool ok = wait_phase(bar, parity);
    __syncwarp();
    return ok;
}

// The reset State (one game's decided initial State, L2-resident) -> slab,
// and its rules-only rows straight into the game's rows in HBM.
template <uint32_t kHbm = 0>
__device__ void load_reset(const Params& P, char* slab, int64_t game, int lane) {
    const Layout& L = P.layout;
    for (int k = 0; k < kSlabLeaves; ++k) {
        char* global = global_row(P, k, game);
        char* dst = staged_row<kHbm>(k) ? slab_row(slab, L, k, global) : global;
        const char* src = static_cast<const char*>(P.reset[k]);
        const int32_t bytes = L.row_bytes[k];
        if ((reinterpret_cast<uintptr_t>(dst) & 3u) == 0 && (bytes & 3) == 0) {
            for (int32_t i = lane; i < bytes / 4; i += 32)
                reinterpret_cast<int32_t*>(dst)[i] = reinterpret_cast<const int32_t*>(src)[i];
        } else {
            for (int32_t i = lane; i < bytes; i += 32) dst[i] = src[i];
        }
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

// Slab scalars -> the game's scalar leaves, one per lane.
__device__ __forceinline__ void store_scalars(const Params& P, char* slab, int64_t game, int lane) {
    const Layout& L = P.layout;
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

// Slab -> global rows (TMA bulk stores of the bodies), scalars -> leaves.
// Every lane that issued stores must later wait for its bulk group (finish_stores).
template <uint32_t kHbm = 0>
__device__ void store_state(const Params& P, char* slab, int64_t game, int lane) {
    const Layout& L = P.layout;
    fence_proxy_async_smem();
    __syncwarp();
    if (L.aligned) {
        if (staged_row<kHbm>(lane)) {
            bulk_store(global_row(P, lane, game), slab + L.leaf_off[lane], L.row_bytes[lane]);
            bulk_commit();
        }
    } else if (staged_row<kHbm>(lane)) {  // lane k owns row k, as in stage_state
        char* dst = global_row(P, lane, game);
        const Span sp = split_row(dst, L.row_bytes[lane]);
        const char* src = slab_row(slab, L, lane, dst);
        if (sp.body) bulk_store(dst + sp.head, src + sp.head, sp.body);
        bulk_commit();
        copy_edge_out(dst, src, sp.head);
        copy_edge_out(dst + sp.head + sp.body, src + sp.head + sp.body, sp.tail);
    }
    store_scalars(P, slab, game, lane);
}

// Waits until the slab rows read by this lane's bulk stores may be reused.
template <uint32_t kHbm = 0>
__device__ __forceinline__ void finish_stores(const Params& P, int lane) {
    if (staged_row<kHbm>(lane)) bulk_wait_read_all();
}

// The threads that write one game's outputs: its warp (tid = lane), or every
// warp of a CTA that holds a single large game.
struct Team {
    int32_t tid, size;
    __device__ __forceinline__ bool cta() const { return size > 32; }
    __device__ __forceinline__ int32_t lane() const { return tid & 31; }
    __device__ __forceinline__ int32_t warp() const { return tid >> 5; }
    __device__ __forceinline__ void sync() const {
        if (cta()) __syncthreads();
        else __syncwarp();
    }
};

__device__ __forceinline__ Team warp_team(int lane) { return Team{lane, 32}; }

// Order-preserving warp compaction of indices [0, n) satisfying `pred`.
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

}  // namespace nrts
