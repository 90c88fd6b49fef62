// CPU oracle for the rush-family scripted bots (WorkerRush, LightRush).
//
// TEST INFRASTRUCTURE ONLY, like oracle.hpp.  A C++17 restatement of the
// reference's JAX program path for `family.act` with the rush strategies
// (bots/family.py:34-81): the script (bots/rush.py:24-246) writes abstract
// actions into the bot's carry, and the abstraction layer
// (bots/abstraction.py:268-1119, program branch `_in_order`) turns them into
// Commands with one A* search per executing unit (bots/pathfinding.py:125-252,
// the `_search_by_program` branch).  It keeps the program's formulation:
// full-length argmin/argsort over slots and cells, the A* open list as an
// argmin over every cell's key.
//
// Only the abstract kinds the rush bots hold are restated
// (rush.KINDS = {ATTACK, HARVEST, TRAIN, BUILD}, rush.py:19-21); translate()
// is called with exactly that set (family.py:65-67), so every `_held` branch
// of another kind is absent from the program the reference traces.
//
// Parity pin: none beyond the reference's source (no tests or fixtures ship
// with it); hand-derived known answers for the search and the building-site
// order live in tests/test_oracle_bots.py.
#pragma once

#include <algorithm>
#include <climits>
#include <cstdint>
#include <cstdlib>
#include <vector>

#include "oracle.hpp"

namespace oracle::bots {

constexpr int32_t kLast = INT32_MAX;  // abstraction.py:62 LAST
// Abstract action kinds (abstraction.py:34-44); the rush bots hold these four.
constexpr int32_t kAbsMove = 0, kAbsAttack = 1, kAbsHarvest = 2, kAbsTrain = 3, kAbsBuild = 4;
constexpr int32_t kAbsTrainDirection = 6;
constexpr int32_t kFillerDuration = 10;  // abstraction.py:63 _FILLER_DURATION
// family.py:14-17.
constexpr int kWorkerRush = 0, kBarracksRush = 1;
// unit_types.py:122-128 order.
constexpr int32_t kTypeResource = 0, kTypeBase = 1, kTypeBarracks = 2, kTypeWorker = 3, kTypeLight = 4;
constexpr int kDirUp = 0, kDirRight = 1, kDirDown = 2, kDirLeft = 3;

// AbstractActions (abstraction.py:70-81): one player's bot carry, C entries.
struct Actions {
    std::vector<int32_t> kind, unit_birth, order, target, target_birth, base, base_birth, cell, unit_type;
    std::vector<uint8_t> trained;
    int32_t next_order = 0;

    explicit Actions(int32_t capacity)  // empty_actions, abstraction.py:120-135
        : kind(capacity, kAbsent), unit_birth(capacity, kAbsent), order(capacity, kAbsent), target(capacity, kAbsent),
          target_birth(capacity, kAbsent), base(capacity, kAbsent), base_birth(capacity, kAbsent),
          cell(capacity, kAbsent), unit_type(capacity, kAbsent), trained(capacity, 0) {}
};

// Units (abstraction.py:84-91) of one player.
struct Units {
    std::vector<int32_t> birth, cell, unit_type, carried, birth_rank;
    std::vector<uint8_t> present, available;
};

struct Closest {  // rush.py:24-28
    std::vector<int32_t> slot, birth;
    bool found = false;
};

// _Desire (abstraction.py:100-107).
struct Desire {
    int32_t kind = kAbsent, direction = kAbsent, target_cell = kAbsent, produced_type = kAbsent, claimed = kAbsent,
            cost = 0, none_duration = 0;
};

// _Usage (abstraction.py:94-97).
struct Usage {
    std::vector<uint8_t> claimed;  // [cells]
    int32_t reserved[kPlayers] = {0, 0};
    int32_t balance[kPlayers] = {0, 0};
};

// pathfinding.py:34-38.
struct Path {
    bool found = false;
    int32_t step = kAbsent, distance = kAbsent, pops = 0;
};

using Mask = std::vector<uint8_t>;

struct Bot {
    const Extents& x;
    const Content& c;
    const Game& g;
    int32_t player;

    int32_t C() const { return x.capacity; }
    int32_t W() const { return x.width; }
    int32_t E() const { return x.entities(); }
    int32_t cost_of(int32_t type) const { return c.at(clip(type, 0, x.types - 1), kCost); }
    int32_t column(int32_t type, int col) const { return c.at(clip(type, 0, x.types - 1), col); }

    // abstraction.py:138-158 own_units.
    Units own_units() const {
        const int32_t first = x.neutral + player * C();
        Units u;
        for (int32_t i = 0; i < C(); ++i) {
            const int32_t s = first + i;
            u.birth.push_back(g.birth[s]);
            u.cell.push_back(g.cell[s]);
            u.unit_type.push_back(clip(g.unit_type[s], 0, x.types - 1));
            u.carried.push_back(g.carried[s]);
            u.present.push_back(g.birth[s] != kAbsent);
            u.available.push_back(g.birth[s] != kAbsent && g.pending_kind[s] == kAbsent);
        }
        u.birth_rank = rank(u.present, u.birth);
        return u;
    }

    // abstraction.py:297-299 _rank: how many members have a smaller key.
    static std::vector<int32_t> rank(const Mask& among, const std::vector<int32_t>& key) {
        std::vector<int32_t> r(key.size(), 0);
        for (size_t i = 0; i < key.size(); ++i)
            for (size_t j = 0; j < key.size(); ++j) r[i] += among[j] && key[j] < key[i];
        return r;
    }

    // abstraction.py:161-163 enemies.
    Mask enemies() const {
        Mask m(E());
        for (int32_t s = 0; s < E(); ++s) m[s] = g.active(s) && g.owner[s] != kAbsent && g.owner[s] != player;
        return m;
    }

    // rush.py:31-46 _closest: Manhattan distance, ties by birth.
    Closest closest(const std::vector<int32_t>& origin, const Mask& candidates) const {
        Closest out;
        out.found = std::any_of(candidates.begin(), candidates.end(), [](uint8_t v) { return v != 0; });
        for (int32_t o : origin) {
            std::vector<int32_t> distance(E());
            int32_t nearest = kLast;
            for (int32_t s = 0; s < E(); ++s) {
                const int32_t cs = g.cell[s];
                distance[s] = candidates[s] ? std::abs(floor_mod(o, W()) - floor_mod(cs, W())) +
                                                  std::abs(floor_div(o, W()) - floor_div(cs, W()))
                                            : kLast;
                nearest = std::min(nearest, distance[s]);
            }
            int32_t slot = 0, best = kLast;
            for (int32_t s = 0; s < E(); ++s) {
                const int32_t v = (candidates[s] && distance[s] == nearest) ? g.birth[s] : kLast;
                if (v < best) { best = v; slot = s; }
            }
            out.slot.push_back(out.found ? slot : kAbsent);
            out.birth.push_back(out.found ? g.birth[slot] : kAbsent);
        }
        return out;
    }

    // rush.py:49-52.
    Closest nearest_enemy(const Units& u) const { return closest(u.cell, enemies()); }

    // rush.py:55-57.
    static Mask first_in_unit_order(const Mask& chosen, const Units& u) {
        int32_t first = 0, best = kLast;
        for (size_t i = 0; i < chosen.size(); ++i) {
            const int32_t v = chosen[i] ? u.birth[i] : kLast;
            if (v < best) { best = v; first = static_cast<int32_t>(i); }
        }
        Mask m(chosen.size());
        for (size_t i = 0; i < chosen.size(); ++i) m[i] = chosen[i] && static_cast<int32_t>(i) == first;
        return m;
    }

    struct Fields {
        std::vector<int32_t> target, target_birth, base, base_birth, cell, unit_type;
        explicit Fields(int32_t n)
            : target(n, kAbsent), target_birth(n, kAbsent), base(n, kAbsent), base_birth(n, kAbsent), cell(n, kAbsent),
              unit_type(n, kAbsent) {}
    };

    // abstraction.py:166-167 is_entry.
    static bool is_entry(const Actions& a, const Units& u, int32_t i, int32_t kind) {
        return a.kind[i] == kind && a.unit_birth[i] == u.birth[i];
    }

    // abstraction.py:170-186 put + :198-219 _written.
    void put(Actions& a, const Units& u, const Mask& chosen, const Mask& last, int32_t kind, const Fields& f) const {
        for (int32_t i = 0; i < C(); ++i) {
            if (!chosen[i]) continue;
            const bool known = a.kind[i] != kAbsent && a.unit_birth[i] == u.birth[i];
            if (!known) a.order[i] = a.next_order + (last[i] ? C() : u.birth_rank[i]);
            a.kind[i] = kind;
            a.unit_birth[i] = u.birth[i];
            a.target[i] = f.target[i];
            a.target_birth[i] = f.target_birth[i];
            a.base[i] = f.base[i];
            a.base_birth[i] = f.base_birth[i];
            a.cell[i] = f.cell[i];
            a.unit_type[i] = f.unit_type[i];
            a.trained[i] = 0;
        }
        a.next_order += C() + 1;
    }

    // abstraction.py:221-235 _visits, read at the desired cell's offset.
    int32_t visit(int32_t cell, int32_t desired) const {
        const int32_t longest = std::max(x.height, x.width);
        const int32_t dy = floor_div(cell, W()) - floor_div(desired, W());
        const int32_t dx = floor_mod(cell, W()) - floor_mod(desired, W());
        const int32_t ring = std::max(std::abs(dx), std::abs(dy));
        if (ring == 0) return kLast;
        const int32_t side = dy == -ring ? 0 : dx == ring ? 1 : dy == ring ? 2 : 3;
        const int32_t along = ((side == 0 || side == 2) ? dx : dy) + ring;
        return (ring * 4 + side) * (2 * longest + 1) + along;
    }

    // abstraction.py:238-253 _building_site.
    int32_t building_site(int32_t desired, const Mask& reserved) const {
        int32_t first = 0, best = kLast;
        bool any = false;
        for (int32_t cell = 0; cell < x.cells(); ++cell) {
            const int32_t v = visit(cell, desired);
            const bool open = !c.terrain[cell] && g.entity_at[cell] == kAbsent && !reserved[cell] && v != kLast;
            any |= open;
            if ((open ? v : kLast) < best) { best = v; first = cell; }
        }
        return any ? first : kAbsent;
    }

    // abstraction.py:256-265 build_if_not_already_building.
    void build_if_not_already_building(Actions& a, const Units& u, const Mask& builder, int32_t unit_type, Mask& reserved) const {
        Mask builds(C());
        int32_t desired = 0;
        bool any = false;
        for (int32_t i = 0; i < C(); ++i) {
            const bool building = is_entry(a, u, i, kAbsBuild) && a.unit_type[i] == unit_type;
            builds[i] = builder[i] && !building;
            any |= builds[i] != 0;
            if (builder[i]) desired += u.cell[i];
        }
        const int32_t site = building_site(desired, reserved);
        Fields f(C());
        std::fill(f.cell.begin(), f.cell.end(), site);
        std::fill(f.unit_type.begin(), f.unit_type.end(), unit_type);
        put(a, u, builds, Mask(C(), 0), kAbsBuild, f);
        if (any && site >= 0 && site < x.cells()) reserved[site] = 1;
    }

    // rush.py:60-69 _attack_nearest.
    void attack_nearest(Actions& a, const Units& u, const Mask& attackers, const Mask& last, const Closest& enemy) const {
        Mask chosen(C());
        for (int32_t i = 0; i < C(); ++i) chosen[i] = attackers[i] && enemy.found;
        Fields f(C());
        f.target = enemy.slot;
        f.target_birth = enemy.birth;
        put(a, u, chosen, last, kAbsAttack, f);
    }

    // rush.py:72-83.
    void melee_units_attack(Actions& a, const Units& u, const Closest& enemy) const {
        Mask melee(C());
        for (int32_t i = 0; i < C(); ++i)
            melee[i] = u.present[i] && column(u.unit_type[i], kCanAttack) && !column(u.unit_type[i], kCanHarvest) && u.available[i];
        attack_nearest(a, u, melee, Mask(C(), 0), enemy);
    }

    // rush.py:86-95.
    void train_workers(Actions& a, const Units& u, int32_t resources) const {
        Mask trains(C());
        for (int32_t i = 0; i < C(); ++i)
            trains[i] = u.present[i] && u.unit_type[i] == kTypeBase && u.available[i] && resources >= cost_of(kTypeWorker);
        Fields f(C());
        std::fill(f.unit_type.begin(), f.unit_type.end(), kTypeWorker);
        put(a, u, trains, Mask(C(), 0), kAbsTrain, f);
    }

    // rush.py:98-113 build_base; returns the builder, updates `reserved`.
    Mask build_base(Actions& a, const Units& u, const Mask& workers, Mask& reserved) const {
        bool any_base = false;
        for (int32_t i = 0; i < C(); ++i) any_base |= u.present[i] && u.unit_type[i] == kTypeBase;
        const bool builds = !any_base && g.player_resources[player] >= cost_of(kTypeBase);
        Mask builder = first_in_unit_order(workers, u);
        for (auto& b : builder) b = b && builds;
        reserved.assign(x.cells(), 0);
        build_if_not_already_building(a, u, builder, kTypeBase, reserved);
        return builder;
    }

    // rush.py:116-148.
    void train_at_base_and_barracks(Actions& a, const Units& u, int32_t resources, int32_t trained_type) const {
        int32_t workers_held = 0;
        for (int32_t i = 0; i < C(); ++i) workers_held += u.present[i] && u.unit_type[i] == kTypeWorker;
        Mask trains_worker(C()), barracks_train(C());
        for (int32_t i = 0; i < C(); ++i) {
            trains_worker[i] = u.present[i] && u.unit_type[i] == kTypeBase && u.available[i] && workers_held < 1 &&
                               resources >= cost_of(kTypeWorker);
        }
        Fields fw(C());
        std::fill(fw.unit_type.begin(), fw.unit_type.end(), kTypeWorker);
        put(a, u, trains_worker, Mask(C(), 0), kAbsTrain, fw);
        for (int32_t i = 0; i < C(); ++i) {
            barracks_train[i] = u.present[i] && u.unit_type[i] == kTypeBarracks && u.available[i] && resources >= cost_of(trained_type);
        }
        Fields fb(C());
        std::fill(fb.unit_type.begin(), fb.unit_type.end(), trained_type);
        put(a, u, barracks_train, Mask(C(), 0), kAbsTrain, fb);
    }

    // rush.py:151-167 harvest_sites.
    void harvest_sites(const Units& u, Closest& resource, Closest& stockpile) const {
        Mask res(E()), stock(E());
        for (int32_t s = 0; s < E(); ++s) {
            const int32_t t = clip(g.unit_type[s], 0, x.types - 1);
            res[s] = g.active(s) && c.at(t, kIsResource);
            stock[s] = g.active(s) && c.at(t, kIsStockpile) && g.owner[s] == player;
        }
        resource = closest(u.cell, res);
        stockpile = closest(u.cell, stock);
    }

    // rush.py:170-193 _harvest; returns the harvesters with no site.
    Mask harvest(Actions& a, const Units& u, const Mask& harvesters) const {
        Closest resource, stockpile;
        harvest_sites(u, resource, stockpile);
        Mask chosen(C()), idle(C());
        Fields f(C());
        for (int32_t i = 0; i < C(); ++i) {
            const bool carrying = u.carried[i] > 0;
            const bool harvesting = is_entry(a, u, i, kAbsHarvest);
            const bool same_base = a.base[i] == stockpile.slot[i] && a.base_birth[i] == stockpile.birth[i];
            const bool same_target = a.target[i] == resource.slot[i] && a.target_birth[i] == resource.birth[i];
            const bool occupied = carrying ? stockpile.found : (stockpile.found && resource.found);
            const bool unchanged = harvesting && same_base && (carrying || same_target);
            chosen[i] = harvesters[i] && occupied && !unchanged;
            idle[i] = harvesters[i] && !occupied;
            f.target[i] = carrying ? kAbsent : resource.slot[i];
            f.target_birth[i] = carrying ? kAbsent : resource.birth[i];
            f.base[i] = stockpile.slot[i];
            f.base_birth[i] = stockpile.birth[i];
        }
        put(a, u, chosen, Mask(C(), 0), kAbsHarvest, f);
        return idle;
    }

    Mask workers_of(const Units& u) const {
        Mask w(C());
        for (int32_t i = 0; i < C(); ++i) w[i] = u.present[i] && column(u.unit_type[i], kCanHarvest);
        return w;
    }

    // rush.py:196-213; returns the workers left free.
    Mask build_base_and_barracks(Actions& a, const Units& u) const {
        const int32_t resources = g.player_resources[player];
        const Mask workers = workers_of(u);
        bool any_barracks = false;
        for (int32_t i = 0; i < C(); ++i) any_barracks |= u.present[i] && u.unit_type[i] == kTypeBarracks;
        Mask reserved;
        const Mask base_builder = build_base(a, u, workers, reserved);
        const bool any_builder = std::any_of(base_builder.begin(), base_builder.end(), [](uint8_t v) { return v != 0; });
        const int32_t used = any_builder ? cost_of(kTypeBase) : 0;
        const bool builds_barracks = !any_barracks && resources >= cost_of(kTypeBarracks) + used;
        Mask rest(C());
        for (int32_t i = 0; i < C(); ++i) rest[i] = workers[i] && !base_builder[i];
        Mask barracks_builder = first_in_unit_order(rest, u);
        for (auto& b : barracks_builder) b = b && builds_barracks;
        build_if_not_already_building(a, u, barracks_builder, kTypeBarracks, reserved);
        Mask free(C());
        for (int32_t i = 0; i < C(); ++i) free[i] = workers[i] && !base_builder[i] && !barracks_builder[i];
        return free;
    }

    // rush.py:216-222.
    void rushing_workers(Actions& a, const Units& u, const Closest& enemy) const {
        const Mask workers = workers_of(u);
        Mask reserved;
        const Mask builder = build_base(a, u, workers, reserved);
        Mask rest(C());
        for (int32_t i = 0; i < C(); ++i) rest[i] = workers[i] && !builder[i];
        const Mask harvester = first_in_unit_order(rest, u);
        const Mask idle = harvest(a, u, harvester);
        Mask free(C());
        for (int32_t i = 0; i < C(); ++i) free[i] = (workers[i] && !builder[i] && !harvester[i]) || idle[i];
        attack_nearest(a, u, free, idle, enemy);
    }

    // rush.py:225-231.
    void worker_rush(Actions& a) const {
        const Units u = own_units();
        const int32_t resources = g.player_resources[player];
        const Closest enemy = nearest_enemy(u);
        train_workers(a, u, resources);
        melee_units_attack(a, u, enemy);
        rushing_workers(a, u, enemy);
    }

    // rush.py:240-246 (with _workers_behavior :234-237).
    void barracks_rush(Actions& a, int32_t trained_type) const {
        const Units u = own_units();
        const int32_t resources = g.player_resources[player];
        const Closest enemy = nearest_enemy(u);
        train_at_base_and_barracks(a, u, resources, trained_type);
        melee_units_attack(a, u, enemy);
        const Mask free = build_base_and_barracks(a, u);
        const Mask idle = harvest(a, u, free);
        attack_nearest(a, u, idle, Mask(C(), 0), enemy);
    }

    // ---------------------------------------------------------------------
    // The abstraction layer (abstraction.py:279-294 _translate, rush kinds).
    // ---------------------------------------------------------------------
    int32_t neighbour_cell(int32_t cell, int32_t direction) const {  // abstraction.py:319-325
        const int d = clip(direction, 0, kDirections - 1);
        return cell + kDy[d] * W() + kDx[d];
    }

    int32_t squared_distance(int32_t a, int32_t b) const {  // abstraction.py:328-331
        const int32_t dx = floor_mod(a, W()) - floor_mod(b, W());
        const int32_t dy = floor_div(a, W()) - floor_div(b, W());
        return dx * dx + dy * dy;
    }

    // abstraction.py:334-361 _pending_usage.
    Usage pending_usage() const {
        Usage us;
        us.claimed.assign(x.cells(), 0);
        for (int32_t s = 0; s < E(); ++s) {
            const int32_t kind = g.pending_kind[s];
            const bool claims = g.active(s) && (kind == kKindMove || kind == kKindProduce);
            if (claims) {
                int32_t t = neighbour_cell(g.cell[s], g.pending_direction[s]);
                if (t < 0) t += x.cells();  // scatter indices wrap once, then out-of-range drops
                if (t >= 0 && t < x.cells()) us.claimed[t] = 1;
            }
        }
        for (int p = 0; p < kPlayers; ++p) {
            for (int32_t i = 0; i < C(); ++i) {
                const int32_t s = x.neutral + p * C() + i;
                if (g.active(s) && g.pending_kind[s] == kKindProduce) us.reserved[p] += cost_of(g.pending_produced_type[s]);
            }
            us.balance[p] = g.player_resources[p];
        }
        return us;
    }

    Mask free_cells(const Usage& us) const {  // abstraction.py:364-367
        Mask f(x.cells());
        for (int32_t cell = 0; cell < x.cells(); ++cell) f[cell] = !(c.terrain[cell] || g.entity_at[cell] != kAbsent || us.claimed[cell]);
        return f;
    }

    static bool within_balance(const Usage& us, int p) { return us.reserved[p] == 0 || us.reserved[p] <= us.balance[p]; }

    bool produce_allowed(const Usage& us, int32_t cost, int32_t cell) const {  // abstraction.py:370-382
        const int32_t reserved = us.reserved[player];
        return !us.claimed[clip(cell, 0, x.cells() - 1)] && (reserved == 0 || cost + reserved <= us.balance[player]) &&
               within_balance(us, 1 - player);
    }

    bool exists(int32_t slot, int32_t birth) const {  // abstraction.py:385-387
        return slot != kAbsent && g.birth[clip(slot, 0, E() - 1)] == birth;
    }

    int32_t cell_of(int32_t slot) const {  // abstraction.py:390-392
        return slot != kAbsent ? g.cell[clip(slot, 0, E() - 1)] : kAbsent;
    }

    // abstraction.py:395-423 _standing (rush kinds).
    Mask standing(const Actions& a, const Units& u) const {
        Mask st(C());
        for (int32_t i = 0; i < C(); ++i) {
            const int32_t kind = a.kind[i];
            const bool alive = kind != kAbsent && a.unit_birth[i] == u.birth[i];
            const bool carrying = u.carried[i] > 0;
            const bool built_on = a.cell[i] != kAbsent && g.entity_at[clip(a.cell[i], 0, x.cells() - 1)] != kAbsent;
            const bool target_gone = !exists(a.target[i], a.target_birth[i]);
            bool completed = false;
            if (kind == kAbsAttack) completed = target_gone;
            else if (kind == kAbsHarvest) completed = carrying ? !exists(a.base[i], a.base_birth[i]) : target_gone;
            else if (kind == kAbsTrain) completed = a.trained[i] != 0;
            else if (kind == kAbsBuild) completed = built_on;
            st[i] = alive && !completed;
        }
        return st;
    }

    // abstraction.py:426-433 _adjacent_direction.
    int32_t adjacent_direction(int32_t origin, int32_t goal) const {
        const int32_t dx = floor_mod(goal, W()) - floor_mod(origin, W());
        const int32_t dy = floor_div(goal, W()) - floor_div(origin, W());
        if (goal == kAbsent) return kAbsent;
        for (int k = 0; k < kDirections; ++k)
            if (dx == kDx[k] && dy == kDy[k]) return k;
        return kAbsent;
    }

    // abstraction.py:465-484 _production.
    Desire production(int32_t direction, int32_t produced_type, int32_t cell, const Usage& us) const {
        Desire d;
        const int32_t claimed = direction != kAbsent ? neighbour_cell(cell, direction) : kAbsent;
        const int32_t cost = cost_of(produced_type);
        if (direction != kAbsent && produce_allowed(us, cost, claimed)) {
            d.kind = kKindProduce;
            d.direction = direction;
            d.produced_type = produced_type;
            d.claimed = claimed;
            d.cost = cost;
        }
        return d;
    }

    // abstraction.py:487-511 _training_direction.
    int32_t training_direction(const Actions& a, const Units& u, int32_t i, const Mask& free) const {
        const Mask enemy = enemies();
        const bool harvests = column(a.unit_type[i], kCanHarvest) != 0;
        Mask near(E());
        bool any_near = false;
        for (int32_t s = 0; s < E(); ++s) {
            const bool resource = g.active(s) && c.at(clip(g.unit_type[s], 0, x.types - 1), kIsResource);
            near[s] = harvests ? resource : enemy[s];
            any_near |= near[s] != 0;
        }
        int32_t best = 0, best_score = INT32_MIN;
        bool any_open = false;
        for (int k = 0; k < kDirections; ++k) {
            const int32_t nx = floor_mod(u.cell[i], W()) + kDx[k], ny = floor_div(u.cell[i], W()) + kDy[k];
            const bool on_board = nx >= 0 && nx < W() && ny >= 0 && ny < x.height;
            const int32_t nb = on_board ? ny * W() + nx : 0;
            const bool open = on_board && free[nb];
            any_open |= open;
            int32_t closest_d = kLast;
            for (int32_t s = 0; s < E(); ++s) {
                if (!near[s]) continue;
                const int32_t cs = g.cell[s];
                closest_d = std::min(closest_d, std::abs(nx - floor_mod(cs, W())) + std::abs(ny - floor_div(cs, W())));
            }
            const int32_t score = any_near ? -closest_d : 0;
            const int32_t v = open ? score : -kLast;
            if (v > best_score) { best_score = v; best = k; }
        }
        return any_open ? best : kAbsent;
    }

    // abstraction.py:594-664 _fallback (rush kinds: ATTACK strike, HARVEST
    // harvest, TRAIN train, BUILD adjacent production).
    Desire fallback(const Actions& a, const Units& u, int32_t i, const Usage& us, int32_t target_cell, bool in_range,
                    int32_t harvest_goal, const Mask& free) const {
        Desire d;
        switch (a.kind[i]) {
            case kAbsAttack:
                if (in_range && target_cell != kAbsent) {
                    d.kind = kKindAttack;
                    d.target_cell = target_cell;
                }
                break;
            case kAbsHarvest: {
                const int32_t dir = adjacent_direction(u.cell[i], harvest_goal);
                if (dir != kAbsent) {
                    d.kind = u.carried[i] > 0 ? kKindReturn : kKindHarvest;
                    d.direction = dir;
                }
                break;
            }
            case kAbsTrain:
                d = production(training_direction(a, u, i, free), a.unit_type[i], u.cell[i], us);
                break;
            case kAbsBuild:
                d = production(adjacent_direction(u.cell[i], a.cell[i]), a.unit_type[i], u.cell[i], us);
                break;
            default:
                break;
        }
        return d;
    }

    struct PlanRow {
        int32_t start, goal, radius;
        Desire fallback;
    };

    // abstraction.py:667-727 _plan (drawing off, rush kinds; `blocked` is no desire).
    std::vector<PlanRow> plan(const Actions& a, const Units& u, const Usage& us, const Mask& free) const {
        std::vector<PlanRow> rows(C());
        for (int32_t i = 0; i < C(); ++i) {
            const int32_t kind = a.kind[i];
            const int32_t target_cell = cell_of(a.target[i]);  // _reach, abstraction.py:576-591
            const int32_t attack_range = column(u.unit_type[i], kAttackRange);
            const bool in_range = squared_distance(u.cell[i], target_cell) <= attack_range * attack_range;
            const int32_t harvest_goal = u.carried[i] > 0 ? cell_of(a.base[i]) : target_cell;
            const int32_t goal = kind == kAbsAttack ? target_cell : kind == kAbsHarvest ? harvest_goal
                                 : kind == kAbsBuild ? a.cell[i] : kAbsent;
            const int32_t radius = kind == kAbsAttack ? attack_range : (kind == kAbsHarvest || kind == kAbsBuild) ? 1 : 0;
            const bool searches = goal != kAbsent && !(kind == kAbsAttack && in_range);
            rows[i].start = u.cell[i];
            rows[i].goal = searches ? goal : u.cell[i];
            rows[i].radius = searches ? radius : 0;
            rows[i].fallback = fallback(a, u, i, us, target_cell, in_range, harvest_goal, free);
        }
        return rows;
    }

    // pathfinding.py:125-252 _search_by_program: A* over free cells, the open
    // list an argmin over every cell's key f * (cells + 1) + (cells - sequence).
    static Path search(const Mask& free, int32_t start, int32_t target, int32_t range, int32_t height, int32_t width) {
        const int32_t cells = height * width;
        const int32_t closed = INT32_MAX, blocked = INT32_MAX - 1, unseen = INT32_MAX - 2;
        auto manhattan = [&](int32_t a, int32_t b) {
            return std::abs(floor_mod(a, width) - floor_mod(b, width)) + std::abs(floor_div(a, width) - floor_div(b, width));
        };
        auto open_key = [&](int32_t f, int32_t sequence) { return f * (cells + 1) + (cells - sequence); };
        const int32_t squared_range = range * range;
        std::vector<int32_t> key(cells), after(cells);
        for (int32_t cell = 0; cell < cells; ++cell) {
            key[cell] = cell == start ? open_key(manhattan(start, target), 0) : (free[cell] ? unseen : blocked);
            after[cell] = cell == start ? start : kAbsent;
        }
        int32_t inserted = 1, goal = kAbsent, pops = 0;
        bool searching = true;
        while (searching && pops < cells) {
            int32_t cell = 0;
            for (int32_t k = 1; k < cells; ++k)
                if (key[k] < key[cell]) cell = k;
            const int32_t k_cell = key[cell];
            const bool exhausted = k_cell >= unseen;
            const int32_t dx = floor_mod(cell, width) - floor_mod(target, width);
            const int32_t dy = floor_div(cell, width) - floor_div(target, width);
            const bool reached = !exhausted && dx * dx + dy * dy <= squared_range;
            const bool expands = !exhausted && !reached;
            int32_t nb[kDirections];
            bool inserts[kDirections];
            for (int k = 0; k < kDirections; ++k) {
                const int32_t nx = floor_mod(cell, width) + kDx[k], ny = floor_div(cell, width) + kDy[k];
                const bool on_board = nx >= 0 && nx < width && ny >= 0 && ny < height;
                nb[k] = on_board ? ny * width + nx : 0;
                inserts[k] = expands && on_board && key[nb[k]] == unseen;
            }
            const int32_t g_cost = k_cell / (cells + 1) - manhattan(cell, target);
            if (expands) key[cell] = closed;
            int32_t sequence = inserted;
            for (int k = 0; k < kDirections; ++k) {
                if (!inserts[k]) continue;
                key[nb[k]] = open_key(g_cost + 1 + manhattan(nb[k], target), sequence++);
                after[nb[k]] = cell == start ? nb[k] : after[cell];
            }
            inserted = sequence;
            if (reached) goal = cell;
            searching = expands;
            pops += !exhausted;
        }
        Path p;
        p.pops = pops;
        p.found = goal != kAbsent;
        const int32_t gg = clip(goal, 0, cells - 1);
        const int32_t offset = after[gg] - start;
        const int32_t step = offset == width ? kDirDown : offset == -1 ? kDirLeft : offset == -width ? kDirUp
                             : offset == 1 ? kDirRight : kAbsent;
        p.step = p.found ? step : kAbsent;
        p.distance = p.found ? key[gg] / (cells + 1) - manhattan(gg, target) : kAbsent;
        return p;
    }

    // abstraction.py:279-294 _translate (+ :800-819 _execute_in_order, :873-966
    // _in_order/_walk_step, :1068-1096 _commands, :1099-1119 _settled).  Writes this player's
    // Commands row (C entries of each field) and settles the carry.
    void translate(Actions& a, int32_t* kind_out, int32_t* direction_out, int32_t* none_out, int32_t* target_out,
                   int32_t* ptype_out, int32_t* order_out) const {
        const Units u = own_units();
        const Usage us = pending_usage();
        const Mask st = standing(a, u);
        Mask executes(C());
        for (int32_t i = 0; i < C(); ++i) executes[i] = st[i] && u.available[i];
        const Mask free = free_cells(us);
        const std::vector<PlanRow> rows = plan(a, u, us, free);

        // _execute_in_order: stable argsort of the executing entries by order.
        std::vector<int32_t> queue(C());
        for (int32_t i = 0; i < C(); ++i) queue[i] = i;
        std::stable_sort(queue.begin(), queue.end(), [&](int32_t l, int32_t r) {
            return (executes[l] ? a.order[l] : kLast) < (executes[r] ? a.order[r] : kLast);
        });
        int32_t queued = 0;
        for (auto e : executes) queued += e != 0;
        const bool moves_allowed = within_balance(us, 0) && within_balance(us, 1);
        Mask used(x.cells(), 0), kept_cells(x.cells(), 0);
        int32_t kept_cost = 0, kept_count = 0;
        std::vector<Desire> desires(C());
        std::vector<int32_t> ranks(C(), kAbsent);
        for (int32_t pos = 0; pos < queued; ++pos) {
            const int32_t i = queue[pos];
            const PlanRow& row = rows[i];
            Mask open(x.cells());
            for (int32_t cell = 0; cell < x.cells(); ++cell) open[cell] = free[cell] && !used[cell];
            const Path path = search(open, row.start, row.goal, row.radius, x.height, x.width);
            Desire desire;  // _answer, abstraction.py:771-786 (blocked is no desire)
            if (path.step != kAbsent) {
                if (moves_allowed) {
                    desire.kind = kKindMove;
                    desire.direction = path.step;
                    desire.claimed = neighbour_cell(row.start, path.step);
                }
            } else {
                desire = row.fallback;
            }
            // _kept, abstraction.py:789-797.
            const bool claims = desire.claimed >= 0 && desire.claimed < x.cells();
            const bool conflicting = claims && (us.claimed[desire.claimed] || kept_cells[desire.claimed]);
            const bool overdrawn = desire.cost > 0 && us.reserved[player] + kept_cost + desire.cost > us.balance[player];
            const bool kept = desire.kind != kAbsent && !conflicting && !overdrawn;
            if (claims) used[desire.claimed] = 1;
            if (kept) {
                if (claims) kept_cells[desire.claimed] = 1;
                kept_cost += desire.cost;
                desires[i] = desire;
                ranks[i] = kept_count++;
            }
        }
        // _commands.
        Mask filler(C());
        for (int32_t i = 0; i < C(); ++i) filler[i] = u.available[i] && desires[i].kind == kAbsent;
        const std::vector<int32_t> filler_rank = rank(filler, u.birth);
        for (int32_t i = 0; i < C(); ++i) {
            const Desire& d = desires[i];
            const bool kept = d.kind != kAbsent;
            kind_out[i] = kept ? d.kind : filler[i] ? kKindNone : kAbsent;
            direction_out[i] = kept ? d.direction : kAbsent;
            none_out[i] = (kept && d.kind == kKindNone) ? d.none_duration : filler[i] ? kFillerDuration : 0;
            target_out[i] = kept ? d.target_cell : kAbsent;
            ptype_out[i] = kept ? d.produced_type : kAbsent;
            order_out[i] = kept ? ranks[i] : filler[i] ? kept_count + filler_rank[i] : kAbsent;
        }
        // _settled.
        const std::vector<int32_t> settled_order = rank(st, a.order);
        int32_t standing_count = 0;
        for (int32_t i = 0; i < C(); ++i) {
            const bool s = st[i] != 0;
            standing_count += s;
            const bool trains = a.kind[i] == kAbsTrain || a.kind[i] == kAbsTrainDirection;
            a.trained[i] = s && (a.trained[i] || (executes[i] && trains));
            a.order[i] = s ? settled_order[i] : kAbsent;
            if (!s) {
                a.kind[i] = a.unit_birth[i] = a.target[i] = a.target_birth[i] = kAbsent;
                a.base[i] = a.base_birth[i] = a.cell[i] = a.unit_type[i] = kAbsent;
            }
        }
        a.next_order = standing_count;
    }

    // family.py:72-81 _decided, then translate (family.py:65-67).
    void act(int strategy, int32_t trained_type, Actions& a, int32_t* rows[6]) const {
        if (strategy == kWorkerRush) worker_rush(a);
        else barracks_rush(a, trained_type);
        translate(a, rows[0], rows[1], rows[2], rows[3], rows[4], rows[5]);
    }
};

}  // namespace oracle::bots
