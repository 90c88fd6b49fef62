// Fused NanoRTS environment step for sm_100a, and its C ABI.
//
// One warp owns one game for the whole step; a CTA holds several games.  The
// game's State rows are staged into the warp's shared-memory slab with 1D TMA
// bulk copies, stepped there (game.cuh, rules.cuh), written back in place with
// TMA bulk stores, and the same warp computes the next step's legality rows and
// both players' observations and streams them to HBM (outputs.cuh).
//
// Semantics follow NanoRTS's JAX program (paths under src/nanorts/):
//   decode            adapters/jaxmarl/actions.py:61-84, adapters/factors.py:117-151
//   admission         core/admission.py:48-156
//   conflicts         core/reservations.py:69-306
//   completion        core/pending.py:47-67, core/completion.py:30-79, core/kinds/*.py
//   outcome           core/outcome.py:11-37
//   auto-reset        adapters/lifecycle.py:53-75, adapters/jaxmarl/env.py:109-170
//   legality rows     core/legality.py:32-64, kinds/*.py `_legality`, actions.py:28-41
//   observations      observations/symbolic.py:130-180, observations/visibility.py:70-77
//   rush bots         bots/rush.py:24-246, bots/abstraction.py:268-1119, bots/pathfinding.py:125-252
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/nanorts_b200.h"
#include "device.cuh"
#include "game.cuh"
#include "outputs.cuh"
#include "rules.cuh"
#include "bots.cuh"

namespace nrts {

// Copies the launch's scenario constants to shared memory (no global loads).
__device__ Header setup_header(const Params& P, char* smem) {
    NrtsScenario* sc = reinterpret_cast<NrtsScenario*>(smem);
    const uint32_t* from = reinterpret_cast<const uint32_t*>(&P.scenario);
    uint32_t* to = reinterpret_cast<uint32_t*>(sc);
    for (int32_t i = threadIdx.x; i < static_cast<int32_t>(sizeof(NrtsScenario) / 4); i += blockDim.x) to[i] = from[i];
    Header H;
    H.terrain_rows = sc->terrain_rows;
    H.attack_window = sc->attack_window;
    H.producible = sc->producible;
    H.table = sc->table;
    H.stride = kColumns + P.types;
    H.resource_types = P.scenario.resource_types;
    H.stockpile_types = P.scenario.stockpile_types;
    return H;
}

// After admission: completion, outcome (outcome.py:11-37) and its outputs,
// the optional observation of the ending state, and the lifecycle's auto-reset
// (lifecycle.py:53-75).  Returns whether the game ended.  kCompact: the
// compact layout (one occupant word per slot, 2-bit claim counters).
template <int kW, uint32_t kHbm = 0, bool kCompact = false>
__device__ __forceinline__ bool finish_core_step(const Params& P, const Header& H, const Geo<kW>& G, Game& g, char* slab,
                                                 int64_t game, int lane) {
    complete<kW, (kHbm != 0u)>(P, H, G, g, slab, lane);
    bool terminated, truncated;
    decide(P, g, slab, lane, terminated, truncated);
    const bool done = terminated || truncated;
    if (lane == 0) {
        const NrtsOutputs& o = P.out;
        const int32_t winner = g.s[kSWinner];
        if (o.reward) {  // outcome.py:32-37
            reinterpret_cast<float2*>(o.reward)[game] =
                make_float2(done ? (winner == 0 ? 1.f : -1.f) : 0.f, done ? (winner == 1 ? 1.f : -1.f) : 0.f);
        }
        if (o.done) o.done[game] = done;
        if (o.terminated) o.terminated[game] = terminated;
        if (o.truncated) o.truncated[game] = truncated;
        if (o.winner) o.winner[game] = winner;
        if (o.spawn_overflow) reinterpret_cast<int2*>(o.spawn_overflow)[game] = make_int2(g.s[kSOverflow0], g.s[kSOverflow1]);
        if (o.reward_components) {  // win_loss (adapters/rewards.py:51-53): decided games only, not truncated ones
            const bool over = g.s[kSGameOver] != 0;
            o.reward_components[game * 12] = over ? (winner == 0 ? 1.f : -1.f) : 0.f;
            o.reward_components[game * 12 + 6] = over ? (winner == 1 ? 1.f : -1.f) : 0.f;
        }
    }
    if (P.out.final_feature_maps[0] || P.out.final_feature_maps[1] || P.out.final_scalars[0] || P.out.final_scalars[1]) {
        uint8_t* const no_masks[2] = {nullptr, nullptr};
        write_outputs<kW, kCompact>(P, H, G, g, slab, game, no_masks, P.out.final_feature_maps, P.out.final_scalars, false,
                                      warp_team(lane));
    }
    if (done) {  // lifecycle.advance: the next episode starts from the reset State
        const int32_t episode = g.s[kSEpisode];
        const int32_t r0 = g.s[kSRoot0], r1 = g.s[kSRoot1];
        __syncwarp();
        load_reset<kHbm>(P, slab, game, lane);
        if (lane == 0) {
            g.s[kSEpisode] = static_cast<int32_t>(static_cast<uint32_t>(episode) + 1u);
            g.s[kSRoot0] = r0;
            g.s[kSRoot1] = r1;
        }
        __syncwarp();
    }
    return done;
}

// A game's State through the launch's mode, up to issuing its stores; false
// when a bounded wait gave up.
template <int kW, uint32_t kHbm = 0, bool kCompact = false>
__device__ __forceinline__ bool game_core(const Params& P, const Header& H, const Geo<kW>& G, char* slab, uint64_t* bar,
                                          uint32_t parity, int64_t game, int lane, bool team = false) {
    Game g = game_view<kHbm>(P, slab, game);
    if (P.mode == kModeReset) {
        load_reset<kHbm>(P, slab, game, lane);
        if (lane == 0) {
            g.s[kSEpisode] = 0;
            g.s[kSRoot0] = static_cast<int32_t>(P.keys[2 * game]);
            g.s[kSRoot1] = static_cast<int32_t>(P.keys[2 * game + 1]);
        }
        __syncwarp();
    } else if (!stage_state<kHbm>(P, slab, game, bar, parity, lane, team)) {
        return false;
    }

    if (P.mode == kModeStep) {
        admit<kW, false, kCompact, (kHbm != 0u)>(P, H, G, g, slab, game, lane);
        finish_core_step<kW, kHbm, kCompact>(P, H, G, g, slab, game, lane);
    }
    if (P.mode != kModeOutputs) store_state<kHbm>(P, slab, game, lane);
    return true;
}

// One game through the launch's mode on its warp; false when a bounded wait
// gave up.  `next` (>= 0) is the warp's next game, whose rows are pulled into
// L2 while this game's outputs are written.
template <int kW>
__device__ __forceinline__ bool run_game(const Params& P, const Header& H, const Geo<kW>& G, char* slab, uint64_t* bar,
                                         uint32_t parity, int64_t game, int lane, int64_t next = -1) {
    if (!game_core(P, H, G, slab, bar, parity, game, lane)) return false;
    if (next >= 0) prefetch_game(P, next, lane);
    const Game g = game_view(P, slab, game);
    write_outputs(P, H, G, g, slab, game, P.out.masks, P.out.feature_maps, P.out.scalars, P.sampled[0] != nullptr, warp_team(lane));
    if (P.mode != kModeOutputs) finish_stores(P, lane);
    __syncwarp();
    return true;
}

// Each warp steps the games block * warps + warp + k * (blocks * warps); the
// launch gives every game its own warp.
template <int kW>
__device__ __forceinline__ void step_block(const Params& P, int64_t block, int64_t blocks) {
    extern __shared__ __align__(128) char smem[];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int warps = blockDim.x >> 5;
    const Layout& L = P.layout;
    const Header H = setup_header(P, smem);
    const Geo<kW> G{P.width, P.height, P.cells};
    char* slab = smem + L.header_bytes + warp * L.slab_bytes;
    uint64_t* bar = reinterpret_cast<uint64_t*>(slab + L.bar_off);
    if (lane == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    const int64_t stride = blocks * warps;
    uint32_t parity = 0;
    for (int64_t g0 = block * warps + warp; g0 < P.lanes; g0 += stride) {
        const int64_t game = P.reverse ? P.lanes - 1 - g0 : g0;
        const int64_t g1 = g0 + stride;
        const int64_t next = P.mode == kModeStep && g1 < P.lanes ? (P.reverse ? P.lanes - 1 - g1 : g1) : -1;
        if (!run_game(P, H, G, slab, bar, parity, game, lane, next)) break;
        if (P.mode != kModeReset) parity ^= 1u;
    }
}

template <int kW>
__global__ void __launch_bounds__(256, 3) step_kernel(const __grid_constant__ Params P) {
    step_block<kW>(P, blockIdx.x, gridDim.x);
}

// One CTA per SM holding as many games (one per warp) as its shared memory
// takes, up to kBigWarps: no per-CTA reserve or header copy is paid more than
// once per SM, which fits more games per SM than CTAs of at most 8 warps.
// The grid is persistent: each warp steps every (SMs * warps)-th game, so the
// whole GPU sweeps the batch in order (consecutive games' rows are adjacent in
// every leaf array), and pulls its next game's rows into L2 while writing the
// current one's outputs.
constexpr int kBigWarps = 28;

template <int kW>
__global__ void __launch_bounds__(32 * kBigWarps, 1) step_kernel_big(const __grid_constant__ Params P) {
    step_block<kW>(P, blockIdx.x, gridDim.x);
}

// Wide boards (a slab too large for more than a few games per SM): one game
// per CTA of kTeamWarps warps.  Warp 0 runs the game's State through the
// launch's mode; then every warp writes its outputs.  With the rules-only
// rows in HBM (kHbm) the slab is also compact (one occupant word per slot
// instead of one per cell, 2-bit claim counters): five games fit per SM on
// 64 x 64 boards.
constexpr int kTeamWarps = 4;
constexpr int32_t kWideSlabBytes = 24 * 1024;  // above this a game gets a CTA of its own

template <int kW, uint32_t kHbm>
__global__ void __launch_bounds__(32 * kTeamWarps, kHbm ? 5 : 4) step_kernel_wide(const __grid_constant__ Params P) {
    constexpr bool kCompact = kHbm != 0u;
    extern __shared__ __align__(128) char smem[];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const Team T{static_cast<int32_t>(threadIdx.x), static_cast<int32_t>(blockDim.x)};
    const Layout& L = P.layout;
    const Header H = setup_header(P, smem);
    const Geo<kW> G{P.width, P.height, P.cells};
    char* slab = smem + L.header_bytes;
    uint64_t* bar = reinterpret_cast<uint64_t*>(slab + L.bar_off);
    volatile int32_t* ok = reinterpret_cast<int32_t*>(slab + L.bar_off + 8);  // beside the mbarrier
    if (threadIdx.x == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    uint32_t parity = 0;
    for (int64_t g0 = blockIdx.x; g0 < P.lanes; g0 += gridDim.x) {
        const int64_t game = P.reverse ? P.lanes - 1 - g0 : g0;
        if (warp == 0) {
            const bool done = game_core<kW, kHbm, kCompact>(P, H, G, slab, bar, parity, game, lane, true);
            if (lane == 0) *ok = done;
            const int64_t g1 = g0 + gridDim.x;
            if (done && P.mode == kModeStep && g1 < P.lanes) prefetch_game(P, P.reverse ? P.lanes - 1 - g1 : g1, lane);
        }
        __syncthreads();
        if (!*ok) break;
        const Game g = game_view<kHbm>(P, slab, game);
        write_outputs<kW, kCompact>(P, H, G, g, slab, game, P.out.masks, P.out.feature_maps, P.out.scalars, P.sampled[0] != nullptr,
                                      T);
        if (warp == 0 && P.mode != kModeOutputs) finish_stores<kHbm>(P, lane);
        __syncthreads();
        if (P.mode != kModeReset) parity ^= 1u;
    }
}

// Several groups of games in one launch: the CTAs of group k are the blocks
// [block_start[k], block_start[k + 1]), each group with its own Params.
constexpr int kMaxGroups = NRTS_MAX_GROUPS;
struct GroupParams {
    int32_t count;
    int32_t block_start[kMaxGroups + 1];
    Params group[kMaxGroups];
};

template <int kW>
__global__ void __launch_bounds__(256, 3) groups_kernel(const __grid_constant__ GroupParams GP) {
    int k = 0;
    while (k + 1 < GP.count && static_cast<int32_t>(blockIdx.x) >= GP.block_start[k + 1]) ++k;
    step_block<kW>(GP.group[k], static_cast<int64_t>(blockIdx.x) - GP.block_start[k], GP.block_start[k + 1] - GP.block_start[k]);
}

// One game of a bot launch.  Bot-act: the bot of P.bot_player chooses that
// player's Commands, written to HBM with the settled carry; the State is only
// read.  Duel: both players' bots choose Commands from the starting State,
// then the core step as run_game, with the carries of a finished game reset
// to empty_actions (bots/seat.py:127).
template <int kW>
__device__ __forceinline__ bool run_bots(const Params& P, const Header& H, const Geo<kW>& G, char* slab, uint64_t* bar,
                                         uint32_t parity, int64_t game, int lane) {
    Game g = game_view<kBotHbmRows>(P, slab, game);
    if (!stage_bots(P, slab, game, bar, parity, lane)) return false;
    const bool duel = P.mode == kModeDuel;
    bot_prepare(P, H, G, g, slab, lane);
    const Cmds cmd = cmd_view(P, slab);
    for (int p = 0; p < kPlayers; ++p) {
        if (!duel && p != P.bot_player) continue;
        BotView v = bot_view(P, g, slab, p);
        bot_script(P, H, G, v, P.bot[p].strategy, P.bot[p].trained, lane);
        bot_translate(P, H, G, v, cmd, lane);
    }
    if (!duel) {
        const int32_t C = P.capacity, owned = P.owned;
        int32_t* out = P.commands + game * 6 * owned;
        for (int32_t o = lane; o < owned; o += 32) {
            const bool mine = (o >= C) == (P.bot_player == 1);
            out[o] = mine ? cmd.kind[o] : kAbsent;
            out[owned + o] = mine ? cmd.dir[o] : kAbsent;
            out[2 * owned + o] = mine ? cmd.none[o] : 0;
            out[3 * owned + o] = mine ? cmd.target[o] : kAbsent;
            out[4 * owned + o] = mine ? cmd.ptype[o] : kAbsent;
            out[5 * owned + o] = mine ? cmd.order[o] : kAbsent;
        }
        store_bots(P, slab, game, lane);
        finish_bot_stores();
        __syncwarp();
        return true;
    }
    admit<kW, true, false, true>(P, H, G, g, slab, game, lane);
    if (finish_core_step<kW, kBotHbmRows>(P, H, G, g, slab, game, lane)) {
        empty_carry(P, carry_view(P, slab, 0), lane);
        empty_carry(P, carry_view(P, slab, 1), lane);
    }
    store_bots(P, slab, game, lane);
    const NrtsOutputs& o = P.out;
    if (o.masks[0] || o.masks[1] || o.packed_masks[0] || o.packed_masks[1] || o.feature_maps[0] || o.feature_maps[1] ||
        o.scalars[0] || o.scalars[1] || P.sampled[0])
        write_outputs(P, H, G, g, slab, game, o.masks, o.feature_maps, o.scalars, P.sampled[0] != nullptr, warp_team(lane));
    finish_bot_stores();
    __syncwarp();
    return true;
}

// Each warp runs the bot launch's games block * warps + warp + k * (blocks * warps).
template <int kW>
__device__ __forceinline__ void duel_block(const Params& P) {
    extern __shared__ __align__(128) char smem[];
    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int warps = blockDim.x >> 5;
    const Layout& L = P.layout;
    const Header H = setup_header(P, smem);
    const Geo<kW> G{P.width, P.height, P.cells};
    char* slab = smem + L.header_bytes + warp * L.slab_bytes;
    uint64_t* bar = reinterpret_cast<uint64_t*>(slab + L.bar_off);
    if (lane == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    const int64_t stride = static_cast<int64_t>(gridDim.x) * warps;
    uint32_t parity = 0;
    for (int64_t g0 = static_cast<int64_t>(blockIdx.x) * warps + warp; g0 < P.lanes; g0 += stride) {
        const int64_t game = P.reverse ? P.lanes - 1 - g0 : g0;
        if (!run_bots(P, H, G, slab, bar, parity, game, lane)) break;
        parity ^= 1u;
    }
}

template <int kW>
__global__ void __launch_bounds__(256) duel_kernel(const __grid_constant__ Params P) {
    duel_block<kW>(P);
}

// Full bot batches: one CTA per SM holding up to kDuelBigWarps games, on a
// persistent grid.  The bound of 20 warps per SM caps registers at 102 per
// thread (the kernel needs 96), where the 8-warp CTAs of duel_kernel take
// 128 and fit 16 games per SM.
constexpr int kDuelBigWarps = 20;

template <int kW>
__global__ void __launch_bounds__(32 * kDuelBigWarps, 1) duel_kernel_big(const __grid_constant__ Params P) {
    duel_block<kW>(P);
}

// Uniform draw per factor group from mask rows in HBM (nrts_sample_actions).
// Standalone draw (nrts_sample_actions): one warp per 32 consecutive mask rows
// of one player.  The warp reads the rows' bytes as coalesced 16-byte loads,
// turns each into 16 flag bits (byte != 0) in a shared bit string, then each
// lane takes its row's width bits from the string and draws as the fused path.
constexpr int kSampleWarps = 8;
constexpr int kSampleMaxWidth = 96;

__global__ void __launch_bounds__(32 * kSampleWarps) sample_kernel(int64_t rows, int32_t width, int32_t types,
                                                                   const uint8_t* masks0, const uint8_t* masks1,
                                                                   int32_t* actions0, int32_t* actions1, uint32_t key) {
    __shared__ uint32_t bits[kSampleWarps][kSampleMaxWidth + 1];  // 32 rows x width bits, one spare word
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int64_t chunks = (rows + 31) / 32;
    const int64_t chunk = static_cast<int64_t>(blockIdx.x) * kSampleWarps + warp;
    if (chunk >= 2 * chunks) return;
    const int player = chunk >= chunks;
    const int64_t r0 = (chunk - player * chunks) * 32;
    const int32_t n_rows = static_cast<int32_t>(rows - r0 < 32 ? rows - r0 : 32);
    const uint8_t* src = (player ? masks1 : masks0) + r0 * width;
    const int32_t n = n_rows * width;  // bytes of this chunk
    uint16_t* bits16 = reinterpret_cast<uint16_t*>(bits[warp]);
    auto flags4 = [](uint32_t x) { return ((__vcmpne4(x, 0u) & 0x01010101u) * 0x00204081u) >> 21 & 0xfu; };
    if ((reinterpret_cast<uintptr_t>(src) & 15u) == 0) {
        for (int32_t j = lane; 16 * j < n; j += 32) {
            uint32_t f = 0;
            if (16 * j + 16 <= n) {
                const uint4 q = __ldg(reinterpret_cast<const uint4*>(src) + j);
                f = flags4(q.x) | flags4(q.y) << 4 | flags4(q.z) << 8 | flags4(q.w) << 12;
            } else {
                for (int32_t b = 0; 16 * j + b < n; ++b) f |= static_cast<uint32_t>(__ldg(src + 16 * j + b) != 0) << b;
            }
            bits16[j] = static_cast<uint16_t>(f);
        }
    } else {
        for (int32_t j = lane; 16 * j < n; j += 32) {
            uint32_t f = 0;
            for (int32_t b = 0; b < 16 && 16 * j + b < n; ++b) f |= static_cast<uint32_t>(__ldg(src + 16 * j + b) != 0) << b;
            bits16[j] = static_cast<uint16_t>(f);
        }
    }
    if (lane == 0) bits[warp][kSampleMaxWidth] = 0u;
    __syncwarp();
    if (lane >= n_rows) return;
    // Row `lane`: bits [lane * width, lane * width + width) of the string.
    auto take = [&](int32_t at) {  // 32 bits from bit `at`
        const int32_t wi = at >> 5, b = at & 31;
        return __funnelshift_r(bits[warp][wi], bits[warp][wi + 1], b);
    };
    const int32_t at = lane * width;
    const uint32_t w0 = take(at);
    const uint32_t w1 = width > 32 ? take(at + 32) : 0u;
    uint32_t w2 = width > 64 ? take(at + 64) : 0u;
    uint32_t w1m = w1;
    if (width < 64) w1m &= width > 32 ? (1u << (width - 32)) - 1u : 0u;
    if (width < 96) w2 &= width > 64 ? (1u << (width - 64)) - 1u : 0u;
    const uint32_t w0m = width < 32 ? w0 & ((1u << width) - 1u) : w0;
    const int64_t row = r0 + lane;
    int32_t a[kActionColumns];
    draw_row(w0m, w1m, w2, types, key, static_cast<uint32_t>(player * rows + row), a);
    int32_t* dst = (player ? actions1 : actions0) + row * kActionColumns;
#pragma unroll
    for (int f = 0; f < kActionColumns; ++f) dst[f] = a[f];
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

// A wait on an mbarrier that no copy or thread ever completes: it must give
// up after `limit_ns`, record the status in out[1] and return.  This runs the
// bounded-wait path of every staging wait without any fault, and leaves the
// library's status word to the step kernels.
__global__ void wait_probe_kernel(int32_t* out, uint64_t limit_ns) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
    }
    __syncwarp();
    const bool completed = wait_phase(&bar, 0, limit_ns, out + 1);
    if (threadIdx.x == 0) out[0] = completed ? 0 : 1;
}

// Reads and clears the status word in one atomic step.
__device__ int32_t g_status_taken;
__global__ void take_status_kernel() { g_status_taken = atomicExch(&g_status, 0); }

// Probe words of nrts_self_check_no_alloc, in place of the buffer that
// nrts_self_check allocates: words 0-32 take probe_kernel's results, words
// 33-34 wait_probe_kernel's.  256 bytes on every device that loads the
// library, held until the process exits; every call reuses them.
constexpr int kNoAllocCheckWords = 64;
constexpr int kNoAllocProbeWords = 33;
constexpr int kNoAllocWaitWords = 2;
static_assert(kNoAllocProbeWords + kNoAllocWaitWords <= kNoAllocCheckWords, "the probes' words fit the static array");
static __device__ __align__(256) int32_t g_no_alloc_check[kNoAllocCheckWords];

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
    if (side * side != x->offsets || side % 2 == 0 || side > 7)
        return fail(NRTS_E_ARGUMENT, "the attack window must be an odd square of side <= 7");
    if (kKinds + 4 * kDirections + x->types + x->offsets > kMaxMaskBits)
        return fail(NRTS_E_ARGUMENT, "legality rows wider than 96 columns");
    if (x->strategy < 0 || x->strategy > 2) return fail(NRTS_E_ARGUMENT, "unknown conflict strategy");
    if (x->max_cycles <= 0) return fail(NRTS_E_ARGUMENT, "max_cycles must be positive");
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

// The slab layout of a launch; `hbm_rows` are rows the rules use in place
// in HBM (no slab room), as the team kernel does on wide boards, where its
// layout is also `compact`: one occupant word per slot instead of one per
// cell, 2-bit claim counters instead of byte counters.
Layout make_layout(const NrtsExtents* x, bool aligned_rows, bool bots, uint32_t hbm_rows = 0u, bool compact = false) {
    Layout L{};
    L.hbm_rows = hbm_rows;
    const int E = x->neutral + 2 * x->capacity;
    const int owned = 2 * x->capacity;
    const int cells = x->height * x->width;
    const int free_words = (x->capacity + 31) / 32;
    int32_t off = 0;
    for (int k = 0; k < kSlabLeaves; ++k) {
        L.row_bytes[k] = row_bytes_host(x, k);
        L.leaf_off[k] = staged_row(L, k) ? off : -1;  // rows in HBM get no slab room
        if (staged_row(L, k)) off += round16(L.row_bytes[k] + (aligned_rows ? 0 : 16));
    }
    L.scal_off = off;
    off += round16(kSCount * 4);
    L.list_off = off;
    off += round16(owned * 2);
    L.order_off = off;
    off += round16(owned * 2);
    if (bots) {
        L.carry_off = off;
        off += 2 * carry_bytes(x->capacity);
        L.cmd_off = off;
        off += cmd_layout(owned, 0).bytes;
    }
    // Scratch shared in turn by the bots, admission, completion (with the
    // outcome that reads its free-slot bitmaps) and the epilogue.  The
    // epilogue keeps only `list` (its available units) and starts at `order`.
    const int32_t U = off;
    L.scan_off = U;
    L.conf_off = L.scan_off + round16(E * 2);
    L.key_off = L.conf_off + round16(E * 2);
    L.info_off = L.key_off + round16(owned * 4);
    L.rank_off = L.info_off + round16(owned * 12);
    L.count_off = L.rank_off + round16(owned * 2);
    // The contested requests' ranks are listed after the last read of the
    // claim counts, into the same bytes.
    L.serial_off = L.count_off;
    const int32_t end_admission = L.count_off + std::max(round16(claim_words(cells, compact) * 4 + 8 + 2 * 5 * 4), round16(owned * 2));
    L.free_off = U;
    L.member_key_off = L.free_off + round16(2 * free_words * 4);
    L.ret_off = L.member_key_off + round16(owned * 4);
    const int32_t end_completion = L.ret_off + round16(owned * 20);
    L.word_off = bots ? U : L.order_off;
    L.rows_off = L.word_off + round16((compact ? E : cells) * 4);
    L.mask_off = L.rows_off + round16(4 * x->height * 8);
    const int32_t end_epilogue = L.mask_off + round16((owned * 3 + 2 + 4) * 4);  // + the team counts
    off = std::max(end_admission, std::max(end_completion, end_epilogue));
    if (bots) {
        L.bot_off = U;
        off = std::max(off, U + bot_layout(x->capacity, E, cells, 0).bytes);
    }
    L.bar_off = off;
    off += 16;
    L.slab_bytes = round16(off);
    L.aligned = aligned_rows ? 1 : 0;
    L.total_bytes = 0;
    for (int k = 0; k < kSlabLeaves; ++k)
        if (staged_row(L, k)) L.total_bytes += L.row_bytes[k];
    L.header_bytes = round16(sizeof(NrtsScenario));
    return L;
}

struct DeviceInfo {
    int smem_optin = 0;
    int sms = 0;
    bool ready = false;
};

DeviceInfo g_devices[64];

template <uint32_t kHbm>
const void* pick_wide_kernel_rows(int width) {
    switch (width) {
        case 8: return reinterpret_cast<const void*>(step_kernel_wide<8, kHbm>);
        case 16: return reinterpret_cast<const void*>(step_kernel_wide<16, kHbm>);
        case 32: return reinterpret_cast<const void*>(step_kernel_wide<32, kHbm>);
        case 64: return reinterpret_cast<const void*>(step_kernel_wide<64, kHbm>);
        default: return reinterpret_cast<const void*>(step_kernel_wide<0, kHbm>);
    }
}

// The team kernel of a board width, for a layout with or without rows in HBM.
const void* pick_wide_kernel(int width, bool hbm = false) {
    return hbm ? pick_wide_kernel_rows<kRulesRows>(width) : pick_wide_kernel_rows<0u>(width);
}

const void* pick_big_kernel(int width) {
    switch (width) {
        case 8: return reinterpret_cast<const void*>(step_kernel_big<8>);
        case 16: return reinterpret_cast<const void*>(step_kernel_big<16>);
        case 32: return reinterpret_cast<const void*>(step_kernel_big<32>);
        case 64: return reinterpret_cast<const void*>(step_kernel_big<64>);
        default: return reinterpret_cast<const void*>(step_kernel_big<0>);
    }
}

const void* pick_duel_big_kernel(int width) {
    switch (width) {
        case 8: return reinterpret_cast<const void*>(duel_kernel_big<8>);
        case 16: return reinterpret_cast<const void*>(duel_kernel_big<16>);
        case 32: return reinterpret_cast<const void*>(duel_kernel_big<32>);
        case 64: return reinterpret_cast<const void*>(duel_kernel_big<64>);
        default: return reinterpret_cast<const void*>(duel_kernel_big<0>);
    }
}

const void* pick_groups_kernel(int width) {
    switch (width) {
        case 8: return reinterpret_cast<const void*>(groups_kernel<8>);
        case 16: return reinterpret_cast<const void*>(groups_kernel<16>);
        case 32: return reinterpret_cast<const void*>(groups_kernel<32>);
        case 64: return reinterpret_cast<const void*>(groups_kernel<64>);
        default: return reinterpret_cast<const void*>(groups_kernel<0>);
    }
}

const void* pick_kernel(int width, bool bots = false) {
    if (bots) {
        switch (width) {
            case 8: return reinterpret_cast<const void*>(duel_kernel<8>);
            case 16: return reinterpret_cast<const void*>(duel_kernel<16>);
            case 32: return reinterpret_cast<const void*>(duel_kernel<32>);
            case 64: return reinterpret_cast<const void*>(duel_kernel<64>);
            default: return reinterpret_cast<const void*>(duel_kernel<0>);
        }
    }
    switch (width) {
        case 8: return reinterpret_cast<const void*>(step_kernel<8>);
        case 16: return reinterpret_cast<const void*>(step_kernel<16>);
        case 32: return reinterpret_cast<const void*>(step_kernel<32>);
        case 64: return reinterpret_cast<const void*>(step_kernel<64>);
        default: return reinterpret_cast<const void*>(step_kernel<0>);
    }
}

int prepare_device(int& device, DeviceInfo*& info) {
    if (cudaGetDevice(&device) != cudaSuccess) return fail(NRTS_E_CUDA, "cudaGetDevice failed");
    if (device < 0 || device >= 64) return fail(NRTS_E_CUDA, "device index out of range");
    info = &g_devices[device];
    if (!info->ready) {
        cudaDeviceGetAttribute(&info->smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
        cudaDeviceGetAttribute(&info->sms, cudaDevAttrMultiProcessorCount, device);
        for (int w : {8, 16, 32, 64, 7}) {
            for (bool bots : {false, true}) {
                if (cudaFuncSetAttribute(pick_kernel(w, bots), cudaFuncAttributeMaxDynamicSharedMemorySize, info->smem_optin) != cudaSuccess)
                    return fail(NRTS_E_CUDA, "cudaFuncSetAttribute(step/duel kernel) failed");
            }
            if (cudaFuncSetAttribute(pick_groups_kernel(w), cudaFuncAttributeMaxDynamicSharedMemorySize, info->smem_optin) != cudaSuccess)
                return fail(NRTS_E_CUDA, "cudaFuncSetAttribute(groups kernel) failed");
            for (bool hbm : {false, true})
                if (cudaFuncSetAttribute(pick_wide_kernel(w, hbm), cudaFuncAttributeMaxDynamicSharedMemorySize, info->smem_optin) != cudaSuccess)
                    return fail(NRTS_E_CUDA, "cudaFuncSetAttribute(wide kernel) failed");
            if (cudaFuncSetAttribute(pick_big_kernel(w), cudaFuncAttributeMaxDynamicSharedMemorySize, info->smem_optin) != cudaSuccess)
                return fail(NRTS_E_CUDA, "cudaFuncSetAttribute(big kernel) failed");
            if (cudaFuncSetAttribute(pick_duel_big_kernel(w), cudaFuncAttributeMaxDynamicSharedMemorySize, info->smem_optin) != cudaSuccess)
                return fail(NRTS_E_CUDA, "cudaFuncSetAttribute(duel big kernel) failed");
        }
        info->ready = true;
    }
    return NRTS_OK;
}

int fill_params(Params& P, const NrtsExtents* x, const NrtsContent* content, const NrtsState* state, int64_t lanes, bool bots = false) {
    if (int rc = validate(x)) return rc;
    if (content == nullptr) return fail(NRTS_E_ARGUMENT, "content is null");
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
    P.free_words = (x->capacity + 31) / 32;
    int side = 1;
    while (side * side < x->offsets) ++side;
    P.side = side;
    P.radius = (side - 1) / 2;
    P.mask_width = kKinds + 4 * kDirections + x->types + x->offsets;
    P.lanes = lanes;
    bool aligned = true;
    for (int k = 0; k < NRTS_LEAVES; ++k) {
        if (state->leaf[k] == nullptr) return fail(NRTS_E_ARGUMENT, "a state leaf is null");
        if (content->reset[k] == nullptr) return fail(NRTS_E_ARGUMENT, "a reset leaf is null");
        if (reinterpret_cast<uintptr_t>(state->leaf[k]) % 4 != 0) return fail(NRTS_E_ARGUMENT, "state leaves must be 4-byte aligned");
        if (reinterpret_cast<uintptr_t>(content->reset[k]) % 4 != 0) return fail(NRTS_E_ARGUMENT, "reset leaves must be 4-byte aligned");
        P.leaf[k] = state->leaf[k];
        P.reset[k] = content->reset[k];
        if (k < kSlabLeaves) aligned &= (reinterpret_cast<uintptr_t>(state->leaf[k]) % 16 == 0) && (row_bytes_host(x, k) % 16 == 0);
    }
    if (state->environment_root == nullptr || state->episode_index == nullptr) return fail(NRTS_E_ARGUMENT, "lifecycle leaves are null");
    P.root = state->environment_root;
    P.episode = state->episode_index;
    P.scenario = content->scenario;
    P.layout = make_layout(x, aligned, bots, bots ? kBotHbmRows : 0u);
    int bits = 0;
    for (int v = x->capacity - 1; v > 0; v >>= 1) ++bits;
    P.rank_bits = bits > 1 ? bits : 1;  // admission.py:104-115
    return NRTS_OK;
}

template <uint32_t kHbm>
void launch_wide(const Params& P, unsigned blocks, int threads, size_t smem, cudaStream_t s) {
    switch (P.width) {
        case 8: step_kernel_wide<8, kHbm><<<blocks, threads, smem, s>>>(P); break;
        case 16: step_kernel_wide<16, kHbm><<<blocks, threads, smem, s>>>(P); break;
        case 32: step_kernel_wide<32, kHbm><<<blocks, threads, smem, s>>>(P); break;
        case 64: step_kernel_wide<64, kHbm><<<blocks, threads, smem, s>>>(P); break;
        default: step_kernel_wide<0, kHbm><<<blocks, threads, smem, s>>>(P); break;
    }
}

template <int kW>
void launch_instance(const Params& P, unsigned blocks, int threads, size_t smem, cudaStream_t stream) {
    if (P.mode == kModeDuel || P.mode == kModeBotAct) duel_kernel<kW><<<blocks, threads, smem, stream>>>(P);
    else step_kernel<kW><<<blocks, threads, smem, stream>>>(P);
}

template <int kW>
void launch_big(const Params& P, unsigned grid, int threads, size_t smem, cudaStream_t stream) {
    if (P.mode == kModeDuel || P.mode == kModeBotAct) duel_kernel_big<kW><<<grid, threads, smem, stream>>>(P);
    else step_kernel_big<kW><<<grid, threads, smem, stream>>>(P);
}

// Games per SM of a one-CTA-per-SM step launch: each warp steps every
// (SMs x warps)-th game, so the launch lasts as many rounds as its busiest
// warp has games, and a round of more resident games takes longer (the SM's
// issue slots are shared).  Of `top` and up to four fewer warps (more than
// `floor`), the count with the fewest rounds x warps; the larger on a tie.
int balanced_warps(int64_t lanes, int sms, int top, int floor) {
    int best = top;
    int64_t best_cost = INT64_MAX;
    for (int w = top; w > floor && w >= top - 4; --w) {
        const int64_t per_round = static_cast<int64_t>(sms) * w;
        const int64_t cost = (lanes + per_round - 1) / per_round * w;
        if (cost < best_cost) {
            best_cost = cost;
            best = w;
        }
    }
    return best;
}

// Warps per CTA with the most games resident per SM (registers and shared
// memory), fewer when the batch would not fill every SM twice.
int choose_warps(const void* kernel, const Layout& L, int64_t lanes, const DeviceInfo* info) {
    int best_warps = 1, best_resident = 0;
    for (int warps = 1; warps <= 8; ++warps) {
        const size_t smem = L.header_bytes + static_cast<size_t>(warps) * L.slab_bytes;
        if (smem > static_cast<size_t>(info->smem_optin)) break;
        int blocks = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, kernel, warps * 32, smem) != cudaSuccess) continue;
        if (blocks * warps >= best_resident) {
            best_resident = blocks * warps;
            best_warps = warps;
        }
    }
    int warps = best_warps;
    while (warps > 1 && (lanes + warps - 1) / warps < 2 * info->sms) --warps;
    return warps;
}

int launch_step(Params& P, void* stream) {
    int device;
    DeviceInfo* info;
    if (int rc = prepare_device(device, info)) return rc;
    if (P.lanes == 0) return NRTS_OK;
    const Layout& L = P.layout;
    if (L.header_bytes + L.slab_bytes > info->smem_optin) return fail(NRTS_E_ARGUMENT, "one game does not fit in shared memory");
    const bool bots = P.mode == kModeDuel || P.mode == kModeBotAct;
    if (!bots) {
        // Team launches: one game per CTA of `team` warps (the warps share the
        // output phase), on a persistent grid (each CTA steps every grid-th
        // game and pulls its next game's rows into L2 while writing the
        // current one's outputs).  Wide boards always take 4-warp teams (few
        // of their games fit per SM anyway); smaller boards take the widest
        // team that keeps the whole batch resident at once, when the batch is
        // that small: their step is then bound by one game's latency.
        // Wide boards keep the rules-only rows in HBM (kRulesRows) and a
        // compact layout: a slab small enough for five games per SM on 64 x 64
        // boards.
        const bool wide = L.slab_bytes > kWideSlabBytes;
        if (wide) {
            NrtsExtents x{};
            x.height = P.height;
            x.width = P.width;
            x.neutral = P.neutral;
            x.capacity = P.capacity;
            x.types = P.types;
            x.offsets = P.offsets;
            x.strategy = P.strategy;
            x.max_cycles = P.max_cycles;
            x.partial_observability = P.partial;
            P.layout = make_layout(&x, P.layout.aligned != 0, false, kRulesRows, true);
        }
        const size_t smem = L.header_bytes + static_cast<size_t>(L.slab_bytes);
        int team = 0, resident = 0;
        for (int warps = kTeamWarps; warps >= 2 && team == 0; warps /= 2) {
            int r = 0;
            if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&r, pick_wide_kernel(P.width, wide), 32 * warps, smem) != cudaSuccess) r = 0;
            if (wide || static_cast<int64_t>(r) * info->sms >= P.lanes) {
                team = warps;
                resident = std::max(r, 1);
            }
            if (wide) break;
        }
        if (team > 0) {
            const unsigned blocks = static_cast<unsigned>(std::min<int64_t>(P.lanes, static_cast<int64_t>(info->sms) * resident));
            const int threads = 32 * team;
            cudaStream_t s = static_cast<cudaStream_t>(stream);
            if (wide) launch_wide<kRulesRows>(P, blocks, threads, smem, s);
            else launch_wide<0u>(P, blocks, threads, smem, s);
            const cudaError_t err = cudaGetLastError();
            if (err != cudaSuccess) return fail(NRTS_E_CUDA, std::string("team kernel launch: ") + cudaGetErrorString(err));
            return NRTS_OK;
        }
    }
    // Warps per CTA with the most games resident per SM (registers and shared memory).
    const void* kernel = pick_kernel(P.width, bots);
    int best_warps = 1, best_resident = 0;
    for (int warps = 1; warps <= 8; ++warps) {
        const size_t smem = L.header_bytes + static_cast<size_t>(warps) * L.slab_bytes;
        if (smem > static_cast<size_t>(info->smem_optin)) break;
        int blocks = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, kernel, warps * 32, smem) != cudaSuccess) continue;
        if (blocks * warps >= best_resident) {
            best_resident = blocks * warps;
            best_warps = warps;
        }
    }
    {
        // One CTA per SM when that holds more games and the batch fills it.
        const int64_t room = (static_cast<int64_t>(info->smem_optin) - L.header_bytes) / L.slab_bytes;
        int big = static_cast<int>(std::min<int64_t>(bots ? kDuelBigWarps : kBigWarps, room));
        if (!bots) big = balanced_warps(P.lanes, info->sms, big, best_resident);
        int blocks = 0;
        const size_t smem = L.header_bytes + static_cast<size_t>(big) * L.slab_bytes;
        const void* kernel_big = bots ? pick_duel_big_kernel(P.width) : pick_big_kernel(P.width);
        if (big > best_resident && P.lanes >= static_cast<int64_t>(info->sms) * big &&
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, kernel_big, big * 32, smem) == cudaSuccess && blocks >= 1) {
            const unsigned grid = static_cast<unsigned>(info->sms);
            cudaStream_t s = static_cast<cudaStream_t>(stream);
            switch (P.width) {
                case 8: launch_big<8>(P, grid, big * 32, smem, s); break;
                case 16: launch_big<16>(P, grid, big * 32, smem, s); break;
                case 32: launch_big<32>(P, grid, big * 32, smem, s); break;
                case 64: launch_big<64>(P, grid, big * 32, smem, s); break;
                default: launch_big<0>(P, grid, big * 32, smem, s); break;
            }
            const cudaError_t err = cudaGetLastError();
            if (err != cudaSuccess) return fail(NRTS_E_CUDA, std::string("big kernel launch: ") + cudaGetErrorString(err));
            return NRTS_OK;
        }
    }
    int warps = best_warps;
    // Smaller CTAs when the batch would not fill every SM twice.
    while (warps > 1 && (P.lanes + warps - 1) / warps < 2 * info->sms) --warps;
    // One game per warp, up to the grid limit; the kernels' stride loops cover
    // a grid smaller than the batch.
    const int64_t blocks = std::min<int64_t>((P.lanes + warps - 1) / warps, INT32_MAX);
    const size_t smem = L.header_bytes + static_cast<size_t>(warps) * L.slab_bytes;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    switch (P.width) {
        case 8: launch_instance<8>(P, static_cast<unsigned>(blocks), warps * 32, smem, s); break;
        case 16: launch_instance<16>(P, static_cast<unsigned>(blocks), warps * 32, smem, s); break;
        case 32: launch_instance<32>(P, static_cast<unsigned>(blocks), warps * 32, smem, s); break;
        case 64: launch_instance<64>(P, static_cast<unsigned>(blocks), warps * 32, smem, s); break;
        default: launch_instance<0>(P, static_cast<unsigned>(blocks), warps * 32, smem, s); break;
    }
    const cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess) return fail(NRTS_E_CUDA, std::string("kernel launch: ") + cudaGetErrorString(err));
    return NRTS_OK;
}

// factors.refuse_mask_form (adapters/factors.py:63-86): the packed words hold
// the non-attack groups in one word and the attack window in two.
int check_packable(const NrtsExtents* x) {
    if (kKinds + 4 * kDirections + x->types > 32) return fail(NRTS_E_ARGUMENT, "packed masks need 6+16+T <= 32 bits in word 0");
    if (x->offsets > 64) return fail(NRTS_E_ARGUMENT, "packed masks need an attack window of at most 64 cells");
    return NRTS_OK;
}

int check_bot(const NrtsExtents* x, const NrtsContent* content, const NrtsBot* bot) {
    if (bot == nullptr) return fail(NRTS_E_ARGUMENT, "bot is null");
    for (int t = 0; t < x->types; ++t) {
        const int32_t range = content->scenario.table[t * (kColumns + x->types) + kAttackRange];
        if (range < 0 || range > 127) return fail(NRTS_E_ARGUMENT, "the rush bots take attack ranges between 0 and 127");
    }
    if (bot->strategy != NRTS_WORKER_RUSH && bot->strategy != NRTS_BARRACKS_RUSH) return fail(NRTS_E_ARGUMENT, "unknown bot strategy");
    if (x->types <= kTypeWorker) return fail(NRTS_E_ARGUMENT, "the rush bots need the base, barracks and worker unit types");
    if (x->capacity > kMaxBotCapacity) return fail(NRTS_E_ARGUMENT, "the rush bots take at most 3600 slots per player");
    if (bot->strategy == NRTS_BARRACKS_RUSH && (bot->trained < 0 || bot->trained >= x->types))
        return fail(NRTS_E_ARGUMENT, "a barracks rush needs a trained unit type of the table");
    for (int f = 0; f < NRTS_CARRY_FIELDS; ++f)
        if (bot->carry.field[f] == nullptr) return fail(NRTS_E_ARGUMENT, "a carry field is null");
    if (bot->carry.trained == nullptr || bot->carry.next_order == nullptr) return fail(NRTS_E_ARGUMENT, "a carry field is null");
    return NRTS_OK;
}

// Device addresses of g_no_alloc_check, one per device.  In host code the
// array's name stands for a host-side shadow, never for device memory, so
// the kernels get the address cudaGetSymbolAddress returns with the device
// current: looked up on the first call that checks the device, kept after.
int32_t* g_no_alloc_check_ptr[64] = {};
std::mutex g_no_alloc_check_mutex;

// The current device's copy of g_no_alloc_check (the caller made `device`
// current).
int no_alloc_check_words(int device, int32_t*& words) {
    std::lock_guard<std::mutex> lock(g_no_alloc_check_mutex);
    if (g_no_alloc_check_ptr[device] == nullptr) {
        void* address = nullptr;
        const cudaError_t err = cudaGetSymbolAddress(&address, g_no_alloc_check);
        if (err != cudaSuccess) return fail(NRTS_E_CUDA, std::string("cudaGetSymbolAddress(probe words): ") + cudaGetErrorString(err));
        g_no_alloc_check_ptr[device] = static_cast<int32_t*>(address);
    }
    words = g_no_alloc_check_ptr[device];
    return NRTS_OK;
}

// Whether every kernel image of the library loads on the current device.
bool kernel_images_load() {
    const void* kernels[] = {pick_kernel(8), pick_kernel(16), pick_kernel(32), pick_kernel(64), pick_kernel(7),
                             pick_kernel(8, true), pick_kernel(16, true), pick_kernel(32, true), pick_kernel(64, true),
                             pick_kernel(7, true), pick_groups_kernel(8), pick_groups_kernel(16), pick_groups_kernel(32),
                             pick_groups_kernel(64), pick_groups_kernel(7), pick_wide_kernel(8), pick_wide_kernel(16),
                             pick_wide_kernel(32), pick_wide_kernel(64), pick_wide_kernel(7), pick_wide_kernel(8, true),
                             pick_wide_kernel(16, true), pick_wide_kernel(32, true), pick_wide_kernel(64, true),
                             pick_wide_kernel(7, true), pick_big_kernel(8), pick_big_kernel(16), pick_big_kernel(32),
                             pick_big_kernel(64), pick_big_kernel(7), pick_duel_big_kernel(8), pick_duel_big_kernel(16),
                             pick_duel_big_kernel(32), pick_duel_big_kernel(64), pick_duel_big_kernel(7),
                             reinterpret_cast<const void*>(sample_kernel),
                             reinterpret_cast<const void*>(slot_cells_kernel), reinterpret_cast<const void*>(probe_kernel),
                             reinterpret_cast<const void*>(wait_probe_kernel), reinterpret_cast<const void*>(take_status_kernel)};
    cudaFuncAttributes attributes;
    for (const void* k : kernels)
        if (cudaFuncGetAttributes(&attributes, k) != cudaSuccess) return false;
    return true;
}

}  // namespace

extern "C" {

int nrts_step(const NrtsExtents* extents, const NrtsContent* content, const NrtsState* state, int64_t lanes, const int32_t* actions0,
              const int32_t* actions1, const NrtsOutputs* outputs, void* stream) {
    Params P;
    if (int rc = fill_params(P, extents, content, state, lanes)) return rc;
    if (actions0 == nullptr || actions1 == nullptr) return fail(NRTS_E_ARGUMENT, "actions are null");
    if (outputs == nullptr) return fail(NRTS_E_ARGUMENT, "outputs is null");
    if ((outputs->sampled_actions[0] == nullptr) != (outputs->sampled_actions[1] == nullptr))
        return fail(NRTS_E_ARGUMENT, "sampled_actions needs both players' buffers or neither");
    if (outputs->reward_components != nullptr && extents->types < 7)
        return fail(NRTS_E_ARGUMENT, "reward components need the seven standard unit types");
    if (outputs->packed_masks[0] != nullptr || outputs->packed_masks[1] != nullptr)
        if (int rc = check_packable(extents)) return rc;
    P.mode = kModeStep;
    P.actions[0] = actions0;
    P.actions[1] = actions1;
    P.out = *outputs;
    P.reverse = outputs->reverse_order != 0;
    P.sampled[0] = outputs->sampled_actions[0];
    P.sampled[1] = outputs->sampled_actions[1];
    P.sample_key = sample_key(outputs->sample_seed, outputs->sample_counter);
    return launch_step(P, stream);
}

int nrts_step_groups(const NrtsGroupStep* groups, int32_t count, void* stream) {
    if (groups == nullptr) return fail(NRTS_E_ARGUMENT, "groups is null");
    if (count < 1 || count > kMaxGroups) return fail(NRTS_E_ARGUMENT, "between 1 and 8 groups per launch");
    static thread_local GroupParams GP;
    std::memset(&GP, 0, sizeof(GP));
    const NrtsExtents* x0 = groups[0].extents;
    if (x0 == nullptr) return fail(NRTS_E_ARGUMENT, "a group's extents is null");
    bool aligned = true;
    int64_t total = 0;
    for (int k = 0; k < count; ++k) {
        const NrtsGroupStep& gs = groups[k];
        const NrtsExtents* x = gs.extents;
        if (x == nullptr) return fail(NRTS_E_ARGUMENT, "a group's extents is null");
        if (x->height != x0->height || x->width != x0->width || x->neutral != x0->neutral || x->capacity != x0->capacity ||
            x->types != x0->types || x->offsets != x0->offsets || x->strategy != x0->strategy ||
            x->partial_observability != x0->partial_observability)
            return fail(NRTS_E_ARGUMENT, "groups of one launch must share their extents (all but max_cycles)");
        Params& P = GP.group[k];
        if (int rc = fill_params(P, x, gs.content, gs.state, gs.lanes)) return rc;
        if (gs.actions[0] == nullptr || gs.actions[1] == nullptr) return fail(NRTS_E_ARGUMENT, "a group's actions are null");
        if (gs.outputs == nullptr) return fail(NRTS_E_ARGUMENT, "a group's outputs is null");
        const NrtsOutputs* o = gs.outputs;
        if ((o->sampled_actions[0] == nullptr) != (o->sampled_actions[1] == nullptr))
            return fail(NRTS_E_ARGUMENT, "sampled_actions needs both players' buffers or neither");
        if (o->reward_components != nullptr && x->types < 7)
            return fail(NRTS_E_ARGUMENT, "reward components need the seven standard unit types");
        P.mode = kModeStep;
        P.actions[0] = gs.actions[0];
        P.actions[1] = gs.actions[1];
        P.out = *o;
        P.reverse = o->reverse_order != 0;
        P.sampled[0] = o->sampled_actions[0];
        P.sampled[1] = o->sampled_actions[1];
        P.sample_key = sample_key(o->sample_seed, o->sample_counter);
        aligned &= P.layout.aligned != 0;
        total += gs.lanes;
    }
    // One slab layout for every CTA of the launch.
    const Layout common = make_layout(x0, aligned, false);
    for (int k = 0; k < count; ++k) GP.group[k].layout = common;
    int device;
    DeviceInfo* info;
    if (int rc = prepare_device(device, info)) return rc;
    if (total == 0) return NRTS_OK;
    if (common.header_bytes + common.slab_bytes > info->smem_optin) return fail(NRTS_E_ARGUMENT, "one game does not fit in shared memory");
    const int warps = choose_warps(pick_groups_kernel(x0->width), common, total, info);
    GP.count = count;
    GP.block_start[0] = 0;
    for (int k = 0; k < count; ++k) {
        const int64_t blocks = (GP.group[k].lanes + warps - 1) / warps;
        if (GP.block_start[k] + blocks > INT32_MAX) return fail(NRTS_E_ARGUMENT, "too many games for one launch");
        GP.block_start[k + 1] = GP.block_start[k] + static_cast<int32_t>(blocks);
    }
    const size_t smem = common.header_bytes + static_cast<size_t>(warps) * common.slab_bytes;
    const unsigned blocks = static_cast<unsigned>(GP.block_start[count]);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    switch (x0->width) {
        case 8: groups_kernel<8><<<blocks, warps * 32, smem, s>>>(GP); break;
        case 16: groups_kernel<16><<<blocks, warps * 32, smem, s>>>(GP); break;
        case 32: groups_kernel<32><<<blocks, warps * 32, smem, s>>>(GP); break;
        case 64: groups_kernel<64><<<blocks, warps * 32, smem, s>>>(GP); break;
        default: groups_kernel<0><<<blocks, warps * 32, smem, s>>>(GP); break;
    }
    const cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess) return fail(NRTS_E_CUDA, std::string("groups kernel launch: ") + cudaGetErrorString(err));
    return NRTS_OK;
}

int nrts_reset(const NrtsExtents* extents, const NrtsContent* content, const NrtsState* state, int64_t lanes, const uint32_t* keys,
               const NrtsOutputs* outputs, void* stream) {
    Params P;
    if (int rc = fill_params(P, extents, content, state, lanes)) return rc;
    if (keys == nullptr) return fail(NRTS_E_ARGUMENT, "keys are null");
    P.mode = kModeReset;
    P.keys = keys;
    if (outputs != nullptr) {
        if ((outputs->sampled_actions[0] == nullptr) != (outputs->sampled_actions[1] == nullptr))
            return fail(NRTS_E_ARGUMENT, "sampled_actions needs both players' buffers or neither");
        if (outputs->packed_masks[0] != nullptr || outputs->packed_masks[1] != nullptr)
            if (int rc = check_packable(extents)) return rc;
        for (int p = 0; p < kPlayers; ++p) {
            P.out.masks[p] = outputs->masks[p];
            P.out.packed_masks[p] = outputs->packed_masks[p];
            P.out.feature_maps[p] = outputs->feature_maps[p];
            P.out.scalars[p] = outputs->scalars[p];
            P.sampled[p] = outputs->sampled_actions[p];
        }
        P.sample_key = sample_key(outputs->sample_seed, outputs->sample_counter);
    }
    return launch_step(P, stream);
}

int nrts_bot_act(const NrtsExtents* extents, const NrtsContent* content, const NrtsState* state, int64_t lanes, int32_t player,
                 const NrtsBot* bot, int32_t* commands, void* stream) {
    Params P;
    if (int rc = fill_params(P, extents, content, state, lanes, true)) return rc;
    if (player != 0 && player != 1) return fail(NRTS_E_ARGUMENT, "player must be 0 or 1");
    if (int rc = check_bot(extents, content, bot)) return rc;
    if (commands == nullptr) return fail(NRTS_E_ARGUMENT, "commands is null");
    P.mode = kModeBotAct;
    P.bot_player = player;
    P.bot[player] = *bot;
    P.commands = commands;
    return launch_step(P, stream);
}

int nrts_duel_step(const NrtsExtents* extents, const NrtsContent* content, const NrtsState* state, int64_t lanes, const NrtsBot* bots,
                   const NrtsOutputs* outputs, void* stream) {
    Params P;
    if (int rc = fill_params(P, extents, content, state, lanes, true)) return rc;
    if (bots == nullptr) return fail(NRTS_E_ARGUMENT, "bots is null");
    for (int p = 0; p < kPlayers; ++p)
        if (int rc = check_bot(extents, content, &bots[p])) return rc;
    if (outputs == nullptr) return fail(NRTS_E_ARGUMENT, "outputs is null");
    if ((outputs->sampled_actions[0] == nullptr) != (outputs->sampled_actions[1] == nullptr))
        return fail(NRTS_E_ARGUMENT, "sampled_actions needs both players' buffers or neither");
    if (outputs->reward_components != nullptr && extents->types < 7)
        return fail(NRTS_E_ARGUMENT, "reward components need the seven standard unit types");
    P.mode = kModeDuel;
    P.bot[0] = bots[0];
    P.bot[1] = bots[1];
    P.out = *outputs;
    P.reverse = outputs->reverse_order != 0;
    P.sampled[0] = outputs->sampled_actions[0];
    P.sampled[1] = outputs->sampled_actions[1];
    P.sample_key = sample_key(outputs->sample_seed, outputs->sample_counter);
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

int nrts_packed_masks(const NrtsExtents* extents, const NrtsContent* content, const NrtsState* state, int64_t lanes, uint32_t* words0,
                      uint32_t* words1, void* stream) {
    Params P;
    if (int rc = fill_params(P, extents, content, state, lanes)) return rc;
    if (int rc = check_packable(extents)) return rc;
    P.mode = kModeOutputs;
    P.out.packed_masks[0] = words0;
    P.out.packed_masks[1] = words1;
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
    if (lanes < 0) return fail(NRTS_E_ARGUMENT, "negative lane count");
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
    if (lanes < 0) return fail(NRTS_E_ARGUMENT, "negative lane count");
    if (!masks0 || !masks1 || !actions0 || !actions1) return fail(NRTS_E_ARGUMENT, "null pointer");
    const int64_t rows = lanes * extents->capacity;
    if (rows == 0) return NRTS_OK;
    const int32_t width = kKinds + 4 * kDirections + extents->types + extents->offsets;
    if (width > kSampleMaxWidth) return fail(NRTS_E_ARGUMENT, "mask rows wider than 96 bits");
    const int64_t chunks = 2 * ((rows + 31) / 32);
    sample_kernel<<<static_cast<unsigned>((chunks + kSampleWarps - 1) / kSampleWarps), 32 * kSampleWarps, 0,
                    static_cast<cudaStream_t>(stream)>>>(rows, width, extents->types, masks0, masks1, actions0, actions1,
                                                         sample_key(seed, counter));
    const cudaError_t err = cudaGetLastError();
    return err == cudaSuccess ? NRTS_OK : fail(NRTS_E_CUDA, cudaGetErrorString(err));
}

int nrts_prepare_scenario(const NrtsExtents* extents, const uint8_t* terrain, const int32_t* table, NrtsScenario* out) {
    if (int rc = validate(extents)) return rc;
    if (terrain == nullptr || table == nullptr || out == nullptr) return fail(NRTS_E_ARGUMENT, "null pointer");
    std::memset(out, 0, sizeof(*out));
    const int T = extents->types, stride = kColumns + T;
    for (int32_t y = 0; y < extents->height; ++y) {
        uint64_t bits = 0;
        for (int32_t x = 0; x < extents->width; ++x) bits |= static_cast<uint64_t>(terrain[y * extents->width + x] != 0) << x;
        out->terrain_rows[y] = bits;
    }
    int side = 1;
    while (side * side < extents->offsets) ++side;
    const int radius = (side - 1) / 2;
    for (int t = 0; t < T; ++t) {
        for (int c = 0; c < stride; ++c) out->table[t * stride + c] = table[t * stride + c];
        const int32_t range = table[t * stride + kAttackRange];
        uint64_t window = 0;
        if (table[t * stride + kCanAttack] != 0) {
            for (int o = 0; o < extents->offsets; ++o) {
                const int dx = o % side - radius, dy = o / side - radius;
                if (dx * dx + dy * dy <= range * range) window |= 1ull << o;
            }
        }
        out->attack_window[t] = window;
        uint32_t produces = 0;
        for (int u = 0; u < T; ++u) produces |= static_cast<uint32_t>(table[t * stride + kColumns + u] != 0) << u;
        out->producible[t] = produces;
        out->resource_types |= static_cast<uint32_t>(table[t * stride + kIsResource] != 0) << t;
        out->stockpile_types |= static_cast<uint32_t>(table[t * stride + kIsStockpile] != 0) << t;
    }
    return NRTS_OK;
}

int nrts_device_status(int device) {
    int previous;
    if (cudaGetDevice(&previous) != cudaSuccess) return fail(NRTS_E_CUDA, "cudaGetDevice failed");
    if (cudaSetDevice(device) != cudaSuccess) return fail(NRTS_E_CUDA, "cudaSetDevice failed");
    int32_t value = 0;
    // One thread swaps the word with 0, so a code recorded meanwhile is either
    // returned now or kept for the next call.
    take_status_kernel<<<1, 1>>>();
    cudaError_t err = cudaGetLastError();
    if (err == cudaSuccess) err = cudaMemcpyFromSymbol(&value, g_status_taken, sizeof(value));
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
        if (!kernel_images_load()) {
            cudaSetDevice(previous);
            return fail(NRTS_E_CUDA, "a kernel image does not load on this device");
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
        // The bounded wait gives up (1 ms) and records its status in a word of
        // its own: the library's status word is not touched.
        int32_t probe[2] = {0, 0};
        if (cudaMalloc(&d, sizeof(probe)) != cudaSuccess) {
            cudaSetDevice(previous);
            return fail(NRTS_E_CUDA, "allocation failed in the self check");
        }
        cudaError_t werr = cudaMemset(d, 0, sizeof(probe));
        if (werr == cudaSuccess) {
            wait_probe_kernel<<<1, 32>>>(d, 1000000ull);
            werr = cudaMemcpy(probe, d, sizeof(probe), cudaMemcpyDeviceToHost);
        }
        cudaFree(d);
        if (werr != cudaSuccess) {
            cudaSetDevice(previous);
            return fail(NRTS_E_CUDA, cudaGetErrorString(werr));
        }
        if (probe[0] != 1 || probe[1] != 1) {
            cudaSetDevice(previous);
            return fail(NRTS_E_DEVICE, "a bounded wait did not give up and record its status");
        }
    }
    cudaSetDevice(previous);
    return NRTS_OK;
}

int nrts_self_check_no_alloc(const int32_t* devices, int64_t count) {
    if (count < 0 || count > 64) return fail(NRTS_E_ARGUMENT, "the no-alloc self check takes between 0 and 64 devices per call");
    if (count > 0 && devices == nullptr) return fail(NRTS_E_ARGUMENT, "devices is null");
    for (int64_t i = 0; i < count; ++i)
        if (devices[i] < 0 || devices[i] >= 64) return fail(NRTS_E_ARGUMENT, "a device index is outside 0..63");
    int previous;
    if (cudaGetDevice(&previous) != cudaSuccess) return fail(NRTS_E_CUDA, "cudaGetDevice failed");
    for (int64_t i = 0; i < count; ++i) {
        const int device = devices[i];
        int rc = NRTS_OK;
        int32_t* words = nullptr;
        cudaError_t err = cudaSetDevice(device);
        if (err == cudaSuccess && !kernel_images_load()) rc = fail(NRTS_E_CUDA, "a kernel image does not load on this device");
        if (err == cudaSuccess && rc == NRTS_OK) rc = no_alloc_check_words(device, words);
        int32_t h[kNoAllocProbeWords + kNoAllocWaitWords] = {};
        if (err == cudaSuccess && rc == NRTS_OK) {
            // The words keep the previous call's results: clear them first,
            // so that only this call's probes can set them.
            err = cudaMemset(words, 0, kNoAllocCheckWords * sizeof(int32_t));
            if (err == cudaSuccess) {
                probe_kernel<<<1, 32>>>(words);
                wait_probe_kernel<<<1, 32>>>(words + kNoAllocProbeWords, 1000000ull);
                err = cudaGetLastError();
            }
            if (err == cudaSuccess) err = cudaMemcpy(h, words, sizeof(h), cudaMemcpyDeviceToHost);
        }
        if (err != cudaSuccess) rc = fail(NRTS_E_CUDA, cudaGetErrorString(err));
        if (rc == NRTS_OK) {
            for (int k = 0; k < kNoAllocProbeWords; ++k)
                if (h[k] != 1) rc = fail(NRTS_E_DEVICE, "warp ballot or shuffle returned a wrong value");
            if (rc == NRTS_OK && (h[kNoAllocProbeWords] != 1 || h[kNoAllocProbeWords + 1] != 1))
                rc = fail(NRTS_E_DEVICE, "a bounded wait did not give up and record its status");
        }
        if (rc != NRTS_OK) {
            cudaSetDevice(previous);
            return rc;
        }
    }
    cudaSetDevice(previous);
    return NRTS_OK;
}

const char* nrts_last_error(void) { return g_last_error.c_str(); }

}  // extern "C"
