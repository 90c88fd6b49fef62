// Per-step outputs of a game from its slab: legality rows, both players'
// feature maps and scalars, and the optional fused draw of the next actions.
//
// The epilogue first packs every cell's occupant into one word (the
// reference's own uint8 encoding, observations/symbolic.py:142-168), builds
// per-player row bitmaps of occupied cells and of visible cells, computes each
// owned slot's legality row as three 32-bit words, then streams rows and maps
// to HBM with 16-byte stores.
#pragma once

#include <cstdint>

#include "device.cuh"
#include "game.cuh"
#include "rules.cuh"

namespace nrts {

// Cell word: the occupant's hp 8 | carried 8 | type+1 8 | max(pending kind, 0) 4 |
// owner+1 2, and the wall bit 30.  Zero exactly when the cell is free.
constexpr uint32_t kWallBit = 1u << 30;
constexpr uint32_t kTypeField = 0x00ff0000u;

__device__ __forceinline__ uint32_t occupant_word(const Game& g, int32_t s) {
    const uint32_t hp = static_cast<uint32_t>(static_cast<int32_t>(g.hit_points[s])) & 0xffu;
    const uint32_t carried = static_cast<uint32_t>(g.carried[s]) & 0xffu;
    const uint32_t type = static_cast<uint32_t>(g.unit_type[s] + 1) & 0xffu;
    const uint32_t pending = static_cast<uint32_t>(max(static_cast<int32_t>(g.pending_kind[s]), kKindNone)) & 0xfu;
    const uint32_t owner = static_cast<uint32_t>(g.owner[s] + 1) & 0x3u;
    return hp | (carried << 8) | (type << 16) | (pending << 24) | (owner << 28);
}

// Cell words kept in the slab, one per cell (built by cell_words).
struct SlabWords {
    const uint32_t* words;
    __device__ __forceinline__ uint32_t at(int32_t c) const { return words[c]; }
    // Cells c0 .. c0 + 7 (c0 a multiple of 8; two 16-byte loads).
    __device__ __forceinline__ void eight(int32_t c0, uint32_t (&cw)[8]) const {
        const uint4 qa = reinterpret_cast<const uint4*>(words + c0)[0];
        const uint4 qb = reinterpret_cast<const uint4*>(words + c0)[1];
        cw[0] = qa.x; cw[1] = qa.y; cw[2] = qa.z; cw[3] = qa.w;
        cw[4] = qb.x; cw[5] = qb.y; cw[6] = qb.z; cw[7] = qb.w;
    }
};

// Cell words gathered through entity_at from one occupant word per slot, as
// the reference builds them (symbolic.py:149-168: word[clip(entity_at)] where
// entity_at is not ABSENT), plus the wall bit: for slabs with no room for a
// word per cell.
template <int kW>
struct SlotWords {
    const Header& H;
    const Geo<kW>& G;
    const int16_t* entity_at;
    const uint32_t* slot;  // occupant_word of every slot
    int32_t entities;
    __device__ __forceinline__ uint32_t occupant(int32_t s) const {
        return s == kAbsent ? 0u : slot[clampi(s, 0, entities - 1)];
    }
    __device__ __forceinline__ uint32_t at(int32_t c) const {
        const uint32_t wall = ((H.terrain_rows[G.y(c)] >> G.x(c)) & 1ull) ? kWallBit : 0u;
        return occupant(entity_at[c]) | wall;
    }
    __device__ __forceinline__ void eight(int32_t c0, uint32_t (&cw)[8]) const {
        int16_t at8[8];
        if ((reinterpret_cast<uintptr_t>(entity_at + c0) & 15u) == 0) {
            const uint4 q = *reinterpret_cast<const uint4*>(entity_at + c0);
            const uint32_t v[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                at8[2 * k] = static_cast<int16_t>(v[k] & 0xffffu);
                at8[2 * k + 1] = static_cast<int16_t>(v[k] >> 16);
            }
        } else {
#pragma unroll
            for (int k = 0; k < 8; ++k) at8[k] = entity_at[c0 + k];
        }
        if constexpr (kW >= 8) {  // eight cells of one row
            const uint32_t walls = static_cast<uint32_t>(H.terrain_rows[G.y(c0)] >> G.x(c0)) & 0xffu;
#pragma unroll
            for (int k = 0; k < 8; ++k) cw[k] = occupant(at8[k]) | (((walls >> k) & 1u) ? kWallBit : 0u);
        } else {
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const int32_t c = c0 + k;
                cw[k] = occupant(at8[k]) | (((H.terrain_rows[G.y(c)] >> G.x(c)) & 1ull) ? kWallBit : 0u);
            }
        }
    }
};

// Disks of sight of each player's units (observations/visibility.py:70-77).
template <int kW>
__device__ void visibility_rows(const Params& P, const Header& H, const Geo<kW>& G, const Game& g, uint64_t* vis, const Team& T) {
    for (int32_t r = T.tid; r < 2 * G.h; r += T.size) vis[r] = 0ull;
    T.sync();
    for (int32_t p = T.tid; p < P.owned; p += T.size) {
        const int32_t s = P.neutral + p;
        if (!g.active(s)) continue;
        const int32_t player = p >= P.capacity;
        const int32_t cell = g.cell[s];
        const int32_t radius = H.at(clampi(g.unit_type[s], 0, P.types - 1), kSightRadius);
        const int32_t ux = G.x(cell), uy = G.y(cell);
        int32_t half = radius;
        for (int32_t dy = 0; dy <= radius; ++dy) {
            while (half > 0 && half * half + dy * dy > radius * radius) --half;
            if (half * half + dy * dy > radius * radius) break;
            const int32_t lo = max(ux - half, 0), hi = min(ux + half, G.width() - 1);
            if (lo > hi) continue;
            const uint64_t bits = (hi - lo == 63) ? ~0ull : (((1ull << (hi - lo + 1)) - 1ull) << lo);
            if (uy - dy >= 0) atomicOr(reinterpret_cast<unsigned long long*>(&vis[player * G.h + uy - dy]), bits);
            if (dy > 0 && uy + dy < G.h) atomicOr(reinterpret_cast<unsigned long long*>(&vis[player * G.h + uy + dy]), bits);
        }
    }
    T.sync();
}

// Neighbour facts from occupant words (board.py:23-61 over board_view).
template <int kW, class Words>
__device__ __forceinline__ void neighbour_word(const Geo<kW>& G, const Words& words, int32_t x, int32_t y, int d, bool& free,
                                               uint32_t& word) {
    const int32_t nx = x + dir_dx(d), ny = y + dir_dy(d);
    const bool on_board = nx >= 0 && nx < G.width() && ny >= 0 && ny < G.h;
    word = on_board ? words.at(ny * G.width() + nx) : kWallBit;
    free = word == 0u;
}

// Legality row of owned slot p as bits (legality.py:32-64, actions.py:28-41):
// kind 6 | move 4 | harvest 4 | return 4 | produce direction 4 | produce type T | attack O.
template <int kW, class Words>
__device__ __forceinline__ void legality_row(const Params& P, const Header& H, const Geo<kW>& G, const Game& g, const Words& words,
                                             const uint64_t* occ, uint32_t afford0, uint32_t afford1, int32_t p, uint32_t& w0, uint32_t& w1,
                                             uint32_t& w2) {
    const int32_t slot = P.neutral + p;
    w0 = 1u;
    w1 = w2 = 0u;
    if (g.birth[slot] == kAbsent || g.pending_kind[slot] != kAbsent) return;  // only KIND_NONE
    const int32_t actor = clampi(g.unit_type[slot], 0, P.types - 1);
    const int32_t owner = g.owner[slot];
    const int32_t carried = g.carried[slot];
    const int32_t cell = g.cell[slot];
    const int32_t cx = G.x(cell), cy = G.y(cell);
    const bool can_move = H.at(actor, kCanMove), can_harvest = H.at(actor, kCanHarvest);
    uint32_t free = 0, resource = 0, stockpile = 0;
#pragma unroll
    for (int d = 0; d < kDirections; ++d) {
        bool f;
        uint32_t w;
        neighbour_word(G, words, cx, cy, d, f, w);
        const bool occupied = (w & kTypeField) != 0u;
        const int32_t t = clampi(static_cast<int32_t>((w >> 16) & 0xffu) - 1, 0, P.types - 1);
        const int32_t nowner = static_cast<int32_t>((w >> 28) & 0x3u) - 1;
        free |= static_cast<uint32_t>(f) << d;
        resource |= static_cast<uint32_t>(occupied && ((H.resource_types >> t) & 1u)) << d;
        stockpile |= static_cast<uint32_t>(occupied && ((H.stockpile_types >> t) & 1u) && nowner == owner) << d;
    }
    const uint32_t move = can_move ? free : 0u;
    const uint32_t harvest = (can_harvest && carried == 0) ? resource : 0u;
    const uint32_t ret = (can_harvest && carried > 0) ? stockpile : 0u;
    const uint32_t type_ok = H.producible[actor] & (owner > 0 ? afford1 : afford0);
    const uint32_t pdir = type_ok ? free : 0u;
    const uint32_t ptype = free ? type_ok : 0u;
    uint64_t attack = 0;
    const uint64_t in_range = H.attack_window[actor];
    if (in_range != 0 && owner >= 0 && owner < kPlayers) {
        const uint64_t* enemy = occ + (1 - owner) * G.h;
        const int32_t R = P.radius, side = P.side;
        const uint64_t row_mask = (1ull << side) - 1ull;
        const int32_t x0 = cx - R;
        for (int32_t dy = -R; dy <= R; ++dy) {
            const int32_t y = cy + dy;
            if (y < 0 || y >= G.h) continue;
            const uint64_t bits = enemy[y];
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
                        (static_cast<uint64_t>(ret) << 14) | (static_cast<uint64_t>(pdir) << 18) |
                        (static_cast<uint64_t>(ptype) << 22) | (attack << a);
    const uint64_t hi = attack >> (64 - a);
    w0 = static_cast<uint32_t>(lo);
    w1 = static_cast<uint32_t>(lo >> 32);
    w2 = static_cast<uint32_t>(hi);
}

// 32 row bits starting at column c of row r (rows of 3 words).
__device__ __forceinline__ uint32_t row_bits(const uint32_t* rows, int32_t r, int32_t c) {
    const uint32_t* w = rows + r * 3;
    const int wi = c >> 5, b = c & 31;
    const uint32_t a0 = w[wi];
    const uint32_t a1 = wi < 2 ? w[wi + 1] : 0u;
    return __funnelshift_r(a0, a1, b);
}

__device__ __forceinline__ uint32_t chunk_bits(const uint32_t* rows, int32_t r, int32_t c, int32_t width) {
    const int32_t n0 = min(16, width - c);
    uint32_t bits = row_bits(rows, r, c) & ((1u << n0) - 1u);
    if (n0 < 16) bits |= row_bits(rows, r + 1, 0) << n0;
    return bits;
}

// One player's legality rows [C, width] of this game, as 0/1 bytes: full
// 16-byte chunks by vector stores (row and column advanced incrementally),
// the bytes before the first and after the last full chunk one by one.
__device__ void write_masks(const Params& P, const uint32_t* rows, int64_t game, uint8_t* out, const Team& T) {
    const int32_t width = P.mask_width;
    const int32_t span = P.capacity * width;
    uint8_t* base = out + game * static_cast<int64_t>(span);
    const int32_t head = min(span, static_cast<int32_t>((16u - (reinterpret_cast<uintptr_t>(base) & 15u)) & 15u));
    const int32_t full = (span - head) >> 4;
    const int32_t tail_start = head + 16 * full;
    const int32_t loose = head + (span - tail_start);
    for (int32_t k = T.tid; k < loose; k += T.size) {
        const int32_t o = k < head ? k : tail_start + (k - head);
        const int32_t r = o / width, c = o - r * width;
        base[o] = static_cast<uint8_t>(row_bits(rows, r, c) & 1u);
    }
    if (full == 0) return;
    const int32_t step = 16 * T.size;
    const int32_t step_rows = step / width, step_cols = step - step_rows * width;
    const int32_t o = head + 16 * T.tid;
    int32_t r = o / width, c = o - r * width;
    for (int32_t k = T.tid; k < full; k += T.size) {
        const uint32_t bits = chunk_bits(rows, r, c, width);
        uint4 v;
        v.x = spread4(bits & 0xfu);
        v.y = spread4((bits >> 4) & 0xfu);
        v.z = spread4((bits >> 8) & 0xfu);
        v.w = spread4((bits >> 12) & 0xfu);
        // Evict-first (st.global.cs): the next launch reads the State and the
        // drawn actions, not the masks, so they should not push those out of L2.
        __stcs(reinterpret_cast<uint4*>(base + head + 16 * k), v);
        r += step_rows;
        c += step_cols;
        if (c >= width) {
            c -= width;
            ++r;
        }
    }
}

// One player's legality rows in the packed form (adapters/factors.py:89-103):
// word 0 = the first 6+16+T bits, words 1-2 = the attack window's bits.
__device__ void write_packed(const Params& P, const uint32_t* rows, int64_t game, uint32_t* out, const Team& T) {
    const int32_t head = P.mask_width - P.offsets;
    const uint32_t head_mask = (1u << head) - 1u;
    const uint32_t hi_mask = P.offsets > 32 ? ((P.offsets >= 64) ? ~0u : ((1u << (P.offsets - 32)) - 1u)) : 0u;
    const uint32_t lo_mask = P.offsets >= 32 ? ~0u : ((1u << P.offsets) - 1u);
    uint32_t* base = out + game * static_cast<int64_t>(P.capacity) * 3;
    for (int32_t r = T.tid; r < P.capacity; r += T.size) {
        const uint32_t w0 = rows[3 * r], w1 = rows[3 * r + 1], w2 = rows[3 * r + 2];
        base[3 * r] = w0 & head_mask;
        base[3 * r + 1] = __funnelshift_r(w0, w1, head) & lo_mask;
        base[3 * r + 2] = __funnelshift_r(w1, w2, head) & hi_mask;
    }
}

// Feature bytes [hp, carried, owner (1 self, 2 opponent), type+1, pending, terrain]
// of a cell word seen by `player`, as the low four bytes and the high two.
__device__ __forceinline__ void features(uint32_t w, int player, bool shown, uint32_t& lo, uint32_t& hi) {
    if (!shown) w &= kWallBit;
    const uint32_t owner = (w >> 28) & 0x3u;
    const uint32_t rel = (player == 0 || owner == 0u) ? owner : 3u - owner;
    lo = (w & 0xffffu) | (rel << 16) | ((w & kTypeField) << 8);
    hi = ((w >> 24) & 0xfu) | (((w >> 30) & 1u) << 8);
}

template <int kW, class Words>
__device__ void write_observation(const Params& P, const Geo<kW>& G, const Game& g, const Words& words, const uint64_t* vis, int player,
                                  int64_t game, uint8_t* maps, int32_t* scalars, const Team& T) {
    if (maps != nullptr) {
        uint8_t* base = maps + game * static_cast<int64_t>(G.cells) * kFeatures;
        auto cell_features = [&](int32_t c, uint32_t w, uint32_t& lo, uint32_t& hi) {
            bool shown = true;
            if (P.partial) {
                const bool seen = (vis[player * G.h + G.y(c)] >> G.x(c)) & 1ull;
                shown = ((w >> 28) & 0x3u) == static_cast<uint32_t>(player + 1) || seen;
            }
            features(w, player, shown, lo, hi);
        };
        if ((G.cells & 7) == 0 && (reinterpret_cast<uintptr_t>(base) & 15u) == 0) {
            // 8 cells = 48 bytes = three 16-byte stores; two cells fill three
            // words.  The 8 cell words come by 16-byte loads (lanes 32 bytes
            // apart: 2-way bank conflicts instead of 8-way for single words).
            for (int32_t c0 = T.tid * 8; c0 < G.cells; c0 += T.size * 8) {
                uint32_t cw[8];
                words.eight(c0, cw);
                // Bit k: cell c0 + k visible to the player (one row load when
                // the 8 cells share a row).
                uint32_t seen = 0xffu;
                if (P.partial) {
                    if constexpr (kW >= 8 && (kW & 7) == 0) {
                        seen = static_cast<uint32_t>(vis[player * G.h + G.y(c0)] >> G.x(c0)) & 0xffu;
                    } else {
                        seen = 0u;
#pragma unroll
                        for (int k = 0; k < 8; ++k)
                            seen |= static_cast<uint32_t>((vis[player * G.h + G.y(c0 + k)] >> G.x(c0 + k)) & 1ull) << k;
                    }
                }
                auto group_features = [&](int k, uint32_t& lo, uint32_t& hi) {
                    const bool shown = !P.partial || ((cw[k] >> 28) & 0x3u) == static_cast<uint32_t>(player + 1) || ((seen >> k) & 1u);
                    features(cw[k], player, shown, lo, hi);
                };
                uint32_t w[12];
#pragma unroll
                for (int pair = 0; pair < 4; ++pair) {
                    uint32_t lo0, hi0, lo1, hi1;
                    group_features(2 * pair, lo0, hi0);
                    group_features(2 * pair + 1, lo1, hi1);
                    w[3 * pair] = lo0;
                    w[3 * pair + 1] = hi0 | (lo1 << 16);
                    w[3 * pair + 2] = (lo1 >> 16) | (hi1 << 16);
                }
                uint4* dst = reinterpret_cast<uint4*>(base + c0 * kFeatures);  // evict-first, as the masks
                __stcs(dst, make_uint4(w[0], w[1], w[2], w[3]));
                __stcs(dst + 1, make_uint4(w[4], w[5], w[6], w[7]));
                __stcs(dst + 2, make_uint4(w[8], w[9], w[10], w[11]));
            }
        } else {
            for (int32_t c = T.tid; c < G.cells; c += T.size) {
                uint32_t lo, hi;
                cell_features(c, words.at(c), lo, hi);
                for (int b = 0; b < 4; ++b) base[c * kFeatures + b] = static_cast<uint8_t>(lo >> (8 * b));
                base[c * kFeatures + 4] = static_cast<uint8_t>(hi);
                base[c * kFeatures + 5] = static_cast<uint8_t>(hi >> 8);
            }
        }
    }
    if (scalars != nullptr && T.tid == 0) {  // symbolic.py:171-180
        *reinterpret_cast<int4*>(scalars + game * kScalars) =
            make_int4(g.s[kSRes0 + player], g.s[kSRes0 + 1 - player], g.s[kSTime], g.s[kSAlt]);
    }
}

// Both players' feature maps (and scalars) from one read of each group of 8
// cells' words and visibility bits, on boards whose rows hold whole groups;
// elsewhere one player at a time (write_observation).  For gathered words
// (SlotWords): reading them once per group for both players measured 5 %
// faster on config 5; with the slab's cell words (two 16-byte loads per group)
// the per-player loops measured faster (config 2: 0.157 against 0.161 ms).
template <int kW, class Words>
__device__ void write_observations(const Params& P, const Geo<kW>& G, const Game& g, const Words& words, const uint64_t* vis,
                                   int64_t game, uint8_t* const maps[2], int32_t* const scalars[2], const Team& T) {
    uint8_t* base[2] = {nullptr, nullptr};
    bool grouped = kW >= 8 && (kW & 7) == 0 && maps[0] != nullptr && maps[1] != nullptr;
    for (int player = 0; player < kPlayers && grouped; ++player) {
        base[player] = maps[player] + game * static_cast<int64_t>(G.cells) * kFeatures;
        grouped = (reinterpret_cast<uintptr_t>(base[player]) & 15u) == 0;
    }
    if (!grouped) {
        for (int player = 0; player < kPlayers; ++player)
            write_observation(P, G, g, words, vis, player, game, maps[player], scalars[player], T);
        return;
    }
    for (int32_t c0 = T.tid * 8; c0 < G.cells; c0 += T.size * 8) {
        uint32_t cw[8];
        words.eight(c0, cw);
        uint32_t seen[2] = {0xffu, 0xffu};  // bit k: cell c0 + k visible to the player
        if (P.partial) {
            seen[0] = static_cast<uint32_t>(vis[G.y(c0)] >> G.x(c0)) & 0xffu;
            seen[1] = static_cast<uint32_t>(vis[G.h + G.y(c0)] >> G.x(c0)) & 0xffu;
        }
#pragma unroll
        for (int player = 0; player < kPlayers; ++player) {
            uint32_t w[12];
#pragma unroll
            for (int pair = 0; pair < 4; ++pair) {
                uint32_t lo[2], hi[2];
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int k = 2 * pair + h;
                    const bool shown = !P.partial || ((cw[k] >> 28) & 0x3u) == static_cast<uint32_t>(player + 1) || ((seen[player] >> k) & 1u);
                    features(cw[k], player, shown, lo[h], hi[h]);
                }
                w[3 * pair] = lo[0];
                w[3 * pair + 1] = hi[0] | (lo[1] << 16);
                w[3 * pair + 2] = (lo[1] >> 16) | (hi[1] << 16);
            }
            uint4* dst = reinterpret_cast<uint4*>(base[player] + c0 * kFeatures);  // evict-first, as the masks
            __stcs(dst, make_uint4(w[0], w[1], w[2], w[3]));
            __stcs(dst + 1, make_uint4(w[4], w[5], w[6], w[7]));
            __stcs(dst + 2, make_uint4(w[8], w[9], w[10], w[11]));
        }
    }
    for (int player = 0; player < kPlayers; ++player) {
        if (scalars[player] != nullptr && T.tid == 0) {  // symbolic.py:171-180
            *reinterpret_cast<int4*>(scalars[player] + game * kScalars) =
                make_int4(g.s[kSRes0 + player], g.s[kSRes0 + 1 - player], g.s[kSTime], g.s[kSAlt]);
        }
    }
}

// Per-launch draw key from the caller's (seed, counter); host and device agree.
__host__ __device__ __forceinline__ uint32_t sample_key(uint64_t seed, uint64_t counter) {
    uint32_t k = mix32(static_cast<uint32_t>(seed) ^ 0x9e3779b9u);
    k = mix32(k ^ static_cast<uint32_t>(seed >> 32));
    k = mix32(k ^ static_cast<uint32_t>(counter));
    return mix32(k ^ static_cast<uint32_t>(counter >> 32));
}

// Uniform draw over the set bits of each factor group of one legality row (0
// when a group has none) for row index t = player * L * C + game * C + slot;
// identical in the step kernel and in sample_kernel.
__device__ __forceinline__ void draw_row(uint32_t w0, uint32_t w1, uint32_t w2, int32_t types, uint32_t key, uint32_t t, int32_t* out) {
    const int a = kKinds + 4 * kDirections + types;
    const uint64_t lo = static_cast<uint64_t>(w0) | (static_cast<uint64_t>(w1) << 32);
    const uint64_t attack = (lo >> a) | (static_cast<uint64_t>(w2) << (64 - a));
    const uint64_t groups[kActionColumns] = {lo & 0x3full, (lo >> 6) & 0xfull, (lo >> 10) & 0xfull, (lo >> 14) & 0xfull,
                                             (lo >> 18) & 0xfull, (lo >> 22) & ((1ull << types) - 1ull), attack};
    const uint32_t stream = mix32(key + t * 0x9e3779b9u);
#pragma unroll
    for (int f = 0; f < kActionColumns; ++f) {
        const uint64_t bits = groups[f];
        const uint32_t low = static_cast<uint32_t>(bits), high = static_cast<uint32_t>(bits >> 32);
        const int low_count = __popc(low), count = low_count + __popc(high);
        int value = 0;
        if (count > 0) {
            const uint32_t h = mix32(stream ^ (static_cast<uint32_t>(f + 1) * 0x85ebca6bu));
            const int pick = static_cast<int>(__umulhi(h, static_cast<uint32_t>(count)));
            value = pick < low_count ? select32(low, pick) : 32 + select32(high, pick - low_count);
        }
        out[f] = value;
    }
}

// Cell words of every cell and, for the legality rows, row bitmaps of the cells
// each player occupies (the owner plane of board_view, model/board_view.py:44-69).
template <int kW>
__device__ __forceinline__ void cell_words(const Header& H, const Geo<kW>& G, const Game& g, uint32_t* words, uint64_t* occ, bool rows,
                                           int32_t entities, const Team& T) {
    auto word_of = [&](int32_t c) {
        const int32_t s = g.entity_at[c];
        const uint32_t wall_bit = ((H.terrain_rows[G.y(c)] >> G.x(c)) & 1ull) ? kWallBit : 0u;
        return (s == kAbsent ? 0u : occupant_word(g, s)) | wall_bit;
    };
    if constexpr (kW > 0) {
        // Boards hold few units per cell: the wall bits of every cell in
        // 16-byte groups (four cells of one row), then the occupant word of
        // each cell entity_at names, found from the active slots (entity_at
        // names exactly the active slots' cells, the State invariant of
        // model/state.py:87-165).
        if (rows)
            for (int32_t r = T.tid; r < 2 * G.h; r += T.size) occ[r] = 0ull;
        for (int32_t q = T.tid; q < (G.cells >> 2); q += T.size) {
            const int32_t c = q << 2;
            const uint32_t bits = static_cast<uint32_t>(H.terrain_rows[c / kW] >> (c % kW)) & 0xfu;
            reinterpret_cast<uint4*>(words)[q] = make_uint4(bits & 1u ? kWallBit : 0u, bits & 2u ? kWallBit : 0u,
                                                            bits & 4u ? kWallBit : 0u, bits & 8u ? kWallBit : 0u);
        }
        T.sync();
        for (int32_t s = T.tid; s < entities; s += T.size) {
            if (g.birth[s] == kAbsent) continue;
            const int32_t c = g.cell[s];
            if (c < 0 || c >= G.cells || g.entity_at[c] != s) continue;
            const uint32_t w = occupant_word(g, s) | words[c];
            words[c] = w;
            const uint32_t code = (w >> 28) & 3u;
            if (rows && (code == 1u || code == 2u))
                atomicOr(reinterpret_cast<unsigned long long*>(&occ[(code - 1) * G.h + c / kW]), 1ull << (c % kW));
        }
    } else {
        if (rows)
            for (int32_t r = T.tid; r < 2 * G.h; r += T.size) occ[r] = 0ull;
        T.sync();
        for (int32_t c = T.tid; c < G.cells; c += T.size) {
            const uint32_t w = word_of(c);
            words[c] = w;
            const uint32_t owner = (w >> 28) & 3u;
            if (rows && owner != 0u) atomicOr(reinterpret_cast<unsigned long long*>(&occ[(owner - 1) * G.h + G.y(c)]), 1ull << G.x(c));
        }
    }
    T.sync();
}

// One occupant word per slot (for SlotWords) and, when the masks need them,
// the row bitmaps of the cells each player's active units occupy.
template <int kW>
__device__ __forceinline__ void slot_words(const Geo<kW>& G, const Game& g, uint32_t* slot, uint64_t* occ, bool rows, int32_t entities,
                                           const Team& T) {
    if (rows)
        for (int32_t r = T.tid; r < 2 * G.h; r += T.size) occ[r] = 0ull;
    T.sync();
    for (int32_t s = T.tid; s < entities; s += T.size) {
        const uint32_t w = occupant_word(g, s);
        slot[s] = w;
        if (!rows || g.birth[s] == kAbsent) continue;
        const int32_t c = g.cell[s];
        if (c < 0 || c >= G.cells || g.entity_at[c] != s) continue;
        const uint32_t code = (w >> 28) & 3u;
        if (code == 1u || code == 2u)
            atomicOr(reinterpret_cast<unsigned long long*>(&occ[(code - 1) * G.h + G.y(c)]), 1ull << G.x(c));
    }
    T.sync();
}

// Zero int32 [count] at dst (4-byte aligned) with 16-byte stores where aligned.
__device__ __forceinline__ void zero_words(int32_t* dst, int32_t count, const Team& T) {
    const int32_t head = min(count, static_cast<int32_t>(((16u - (reinterpret_cast<uintptr_t>(dst) & 15u)) & 15u) >> 2));
    const int32_t quads = (count - head) >> 2;
    const int32_t tail = head + 4 * quads;
    if (T.tid < head) dst[T.tid] = 0;
    uint4* body = reinterpret_cast<uint4*>(dst + head);
    for (int32_t k = T.tid; k < quads; k += T.size) body[k] = make_uint4(0u, 0u, 0u, 0u);
    if (T.tid < count - tail) dst[tail + T.tid] = 0;
}

template <int kW, class Words, bool kGrouped = false>
__device__ void write_outputs_from(const Params& P, const Header& H, const Geo<kW>& G, const Game& g, char* slab, int64_t game,
                                   const Words& words, uint8_t* const masks[2], uint8_t* const maps[2], int32_t* const scalars[2],
                                   bool want_masks, bool want_obs, bool sample, const Team& T) {
    const Layout& L = P.layout;
    const uint64_t* occ = reinterpret_cast<const uint64_t*>(slab + L.rows_off);
    uint64_t* vis = reinterpret_cast<uint64_t*>(slab + L.rows_off) + 2 * G.h;
    uint32_t* rows = reinterpret_cast<uint32_t*>(slab + L.mask_off);
    if (want_masks) {
        // Types each player can afford (the balance rule of produce.py:25-35).
        uint32_t afford0 = 0u, afford1 = 0u;
        for (int32_t t = 0; t < P.types; ++t) {
            const int32_t cost = H.at(t, kCost);
            afford0 |= static_cast<uint32_t>(g.s[kSRes0] >= cost) << t;
            afford1 |= static_cast<uint32_t>(g.s[kSRes1] >= cost) << t;
        }
        if (sample) {  // every row draws 0 unless it holds an available unit (written below)
            for (int player = 0; player < kPlayers; ++player)
                zero_words(P.sampled[player] + game * P.capacity * kActionColumns, P.capacity * kActionColumns, T);
        }
        // Rows of slots without an available unit hold only KIND_NONE; the
        // available ones are listed (by the first warp) and computed densely.
        int16_t* avail = reinterpret_cast<int16_t*>(slab + L.list_off);
        int32_t A = 0;
        const int lane = T.lane();
        if (!T.cta()) {
            for (int32_t base = 0; base < P.owned; base += 32) {
                const int32_t p = base + lane;
                const bool in = p < P.owned;
                const bool available = in && g.birth[P.neutral + p] != kAbsent && g.pending_kind[P.neutral + p] == kAbsent;
                if (in && !available) {
                    rows[3 * p] = 1u;
                    rows[3 * p + 1] = 0u;
                    rows[3 * p + 2] = 0u;
                }
                const unsigned m = __ballot_sync(kFull, available);
                if (available) avail[A + __popc(m & lanes_below(lane))] = static_cast<int16_t>(p);
                A += __popc(m);
            }
        } else {
            // Each warp of the CTA lists the available units of its own run
            // of 32-slot chunks (and writes the others' NONE rows); the
            // per-warp counts place every run in slot order.
            const int32_t teams = T.size >> 5, chunks = (P.owned + 31) >> 5, per = (chunks + teams - 1) / teams;
            const int32_t first = min(chunks, T.warp() * per) * 32, last = min(chunks, (T.warp() + 1) * per) * 32;
            auto available_at = [&](int32_t p) {
                return p < P.owned && g.birth[P.neutral + p] != kAbsent && g.pending_kind[P.neutral + p] == kAbsent;
            };
            uint32_t* team_counts = rows + 3 * P.owned + 2;  // spare words after the rows
            int32_t mine = 0;
            for (int32_t base = first; base < last; base += 32) mine += __popc(__ballot_sync(kFull, available_at(base + lane)));
            if (lane == 0) team_counts[T.warp()] = static_cast<uint32_t>(mine);
            T.sync();
            int32_t at = 0;
            for (int32_t k = 0; k < teams; ++k) {
                const int32_t v = static_cast<int32_t>(team_counts[k]);
                at += k < T.warp() ? v : 0;
                A += v;
            }
            for (int32_t base = first; base < last; base += 32) {
                const int32_t p = base + lane;
                const bool available = available_at(p);
                if (p < P.owned && !available) {
                    rows[3 * p] = 1u;
                    rows[3 * p + 1] = 0u;
                    rows[3 * p + 2] = 0u;
                }
                const unsigned m = __ballot_sync(kFull, available);
                if (available) avail[at + __popc(m & lanes_below(lane))] = static_cast<int16_t>(p);
                at += __popc(m);
            }
        }
        T.sync();
        for (int32_t i = T.tid; i < A; i += T.size) {
            const int32_t p = avail[i];
            uint32_t w0, w1, w2;
            legality_row(P, H, G, g, words, occ, afford0, afford1, p, w0, w1, w2);
            rows[3 * p] = w0;
            rows[3 * p + 1] = w1;
            rows[3 * p + 2] = w2;
            if (sample) {
                const int32_t player = p >= P.capacity, local = p - player * P.capacity;
                const int64_t row = game * P.capacity + local;
                int32_t a[kActionColumns];
                draw_row(w0, w1, w2, P.types, P.sample_key, static_cast<uint32_t>(player * P.lanes * P.capacity + row), a);
                int32_t* dst = P.sampled[player] + row * kActionColumns;
#pragma unroll
                for (int f = 0; f < kActionColumns; ++f) dst[f] = a[f];
            }
        }
        T.sync();
        for (int player = 0; player < kPlayers; ++player) {
            if (masks[player] != nullptr) write_masks(P, rows + player * P.capacity * 3, game, masks[player], T);
            if (P.out.packed_masks[player] != nullptr)
                write_packed(P, rows + player * P.capacity * 3, game, P.out.packed_masks[player], T);
        }
    }
    if (want_obs) {
        if (P.partial) visibility_rows(P, H, G, g, vis, T);
        if constexpr (kGrouped) {
            write_observations(P, G, g, words, vis, game, maps, scalars, T);
        } else {
            for (int player = 0; player < kPlayers; ++player)
                write_observation(P, G, g, words, vis, player, game, maps[player], scalars[player], T);
        }
    }
    T.sync();
}

// A game's outputs from its slab.  kSlotWords: the layout holds one
// occupant word per slot instead of one word per cell.
template <int kW, bool kSlotWords = false>
__device__ void write_outputs(const Params& P, const Header& H, const Geo<kW>& G, const Game& g, char* slab, int64_t game,
                              uint8_t* const masks[2], uint8_t* const maps[2], int32_t* const scalars[2], bool sample, const Team& T) {
    const Layout& L = P.layout;
    uint64_t* occ = reinterpret_cast<uint64_t*>(slab + L.rows_off);
    const bool want_masks = masks[0] != nullptr || masks[1] != nullptr || sample || P.out.packed_masks[0] != nullptr ||
                            P.out.packed_masks[1] != nullptr;
    const bool want_obs = maps[0] != nullptr || maps[1] != nullptr || scalars[0] != nullptr || scalars[1] != nullptr;
    if constexpr (kSlotWords) {
        uint32_t* slot = reinterpret_cast<uint32_t*>(slab + L.word_off);
        slot_words(G, g, slot, occ, want_masks, P.entities, T);
        const SlotWords<kW> words{H, G, g.entity_at, slot, P.entities};
        write_outputs_from<kW, SlotWords<kW>, true>(P, H, G, g, slab, game, words, masks, maps, scalars, want_masks, want_obs, sample,
                                                    T);
    } else {
        uint32_t* words = reinterpret_cast<uint32_t*>(slab + L.word_off);
        cell_words(H, G, g, words, occ, want_masks, P.entities, T);
        write_outputs_from(P, H, G, g, slab, game, SlabWords{words}, masks, maps, scalars, want_masks, want_obs, sample, T);
    }
}

}  // namespace nrts
