/*
 * nanorts_b200: C ABI of the B200-native NanoRTS batched environment step.
 *
 * Every entry point takes plain device pointers (lane-major buffers, leading
 * extent L = games), sizes and a CUDA stream passed as `void*`; none
 * allocates, synchronises the host or keeps per-call state.  Calls are
 * stream-ordered and asynchronous.  Each returns 0 on success or a negative
 * NRTS_E_* code; nrts_last_error() then names the problem (per host thread).
 *
 * Buffers (per game; all lane-major [L, ...], C = per-player slot capacity,
 * E = neutral + 2*C slots, H x W field):
 *   State leaves (NrtsState.leaf, in the order of NrtsLeaf): the reference's
 *     State pytree leaves (src/nanorts/model/state.py:27-84) with their dtypes;
 *     cell/slot indices are int16.  Updated in place.
 *   actions[p]       int32 [L, C, 7]    one row per player slot (factor order
 *                                       kind, move/harvest/return/produce
 *                                       direction, produce type, attack offset)
 *   masks[p]         uint8 [L, C, 6+16+T+O]  0/1 legality rows
 *   feature_maps[p]  uint8 [L, H, W, 6]
 *   scalars[p]       int32 [L, 4]
 *
 * Reference interfaces replaced (paths under src/nanorts/ of NanoRTS):
 *   nrts_step          XLA FFI targets nanorts_step (core/cuda/step.cu:653-698),
 *                      nanorts_reset_packed_where_done (adapters/cuda/reset.cu:196),
 *                      nanorts_legality_words (core/cuda/legality.cu:547-561) and
 *                      nanorts_visible_cells (observations/cuda/visibility.cu) plus
 *                      the XLA fusions of decode_actions, observe and mask
 *                      assembly, as called by NanoRTS.step (adapters/jaxmarl/facade.py:107-119)
 *   nrts_step_groups   the XLA FFI target nanorts_step_groups that core.step_groups calls
 *                      (core/__init__.py:63-89, core/cuda/step.cu:390-405) for GroupMix
 *                      (bots/mix.py:107-160): one launch over several groups of games
 *   nrts_reset         NanoRTS.reset (adapters/jaxmarl/facade.py:100-105)
 *   nrts_legal_masks   NanoRTS.get_avail_actions (facade.py:172-174 -> core/cuda/legality.cu)
 *   nrts_packed_masks  jaxmarl.legal_actions with mask_form="packed" (adapters/jaxmarl/actions.py:28-41,
 *                      adapters/factors.py:89-103)
 *   nrts_observe       NanoRTS.get_obs (facade.py:166-170 -> observations/cuda/visibility.cu)
 *   nrts_slot_cells    NanoRTS.get_slot_cells (facade.py:176-178)
 *   nrts_bot_act       XLA FFI target nanorts_abstraction_act (bots/cuda/abstraction_act.cu:1099-1322),
 *                      as called by family.act (bots/family.py:34-69 through
 *                      bots/whole_act.py:113-153) for WorkerRush and LightRush
 *   nrts_duel_step     bot against bot: seat_commands for both players
 *                      (bots/seat.py:152-157), core.step (core/__init__.py:46-60) and
 *                      the lifecycle's auto-reset (adapters/lifecycle.py:53-75), one launch
 *   nrts_build_id      nanorts_build_id (kernels/cuda/registry.cu:201-229)
 *   nrts_self_check    nanorts_self_check (kernels/cuda/registry.cu:201-229)
 */
#ifndef NANORTS_B200_H
#define NANORTS_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum NrtsStatus {
    NRTS_OK = 0,
    NRTS_E_ARGUMENT = -1,    /* a null pointer, a bad extent or an unsupported configuration */
    NRTS_E_CUDA = -2,        /* a CUDA runtime error (launch or attribute) */
    NRTS_E_DEVICE = -3,      /* the device reported an error in the status word */
};

/* State leaves, in the reference's declaration order (state.py:35-80); the
 * same order as the reference step kernel's Leaf enum (core/cuda/step.cu:61-85). */
enum NrtsLeaf {
    NRTS_BIRTH, NRTS_UNIT_TYPE, NRTS_OWNER, NRTS_CELL, NRTS_HIT_POINTS, NRTS_CARRIED_RESOURCES,
    NRTS_PENDING_KIND, NRTS_PENDING_DIRECTION, NRTS_PENDING_NONE_DURATION, NRTS_PENDING_TARGET_CELL,
    NRTS_PENDING_PRODUCED_TYPE, NRTS_PENDING_ISSUED_AT, NRTS_PENDING_COMPLETES_AT, NRTS_PENDING_ORDER,
    NRTS_ENTITY_AT, NRTS_TIME, NRTS_PLAYER_RESOURCES, NRTS_NEXT_BIRTH, NRTS_NEXT_PENDING_ORDER,
    NRTS_ALTERNATING_CONFLICT_COUNT, NRTS_GAME_OVER, NRTS_WINNER, NRTS_SPAWN_OVERFLOW,
    NRTS_LEAVES
};

/* Static extents of one scenario (BucketSpec, model/bucket.py:24-105). */
typedef struct NrtsExtents {
    int32_t height, width;        /* field; width <= 64 */
    int32_t neutral;              /* neutral slots */
    int32_t capacity;             /* slots per player (C) */
    int32_t types;                /* unit types (T) */
    int32_t offsets;              /* attack window cells (O = side^2, side <= 7) */
    int32_t strategy;             /* 0 CANCEL_BOTH, 1 CANCEL_RANDOM, 2 CANCEL_ALTERNATING */
    int32_t max_cycles;           /* time limit */
    int32_t partial_observability;/* 0/1 */
} NrtsExtents;

/* Per-scenario constants in the form the kernels read them, filled once by
 * nrts_prepare_scenario from host arrays and passed by value with every launch. */
#define NRTS_MAX_HEIGHT 64
#define NRTS_MAX_TYPES 8
#define NRTS_TABLE_COLUMNS 15 /* followed by one `produces` column per type */
typedef struct NrtsScenario {
    uint64_t terrain_rows[NRTS_MAX_HEIGHT];   /* bit x of row y: wall */
    uint64_t attack_window[NRTS_MAX_TYPES];   /* attack-window cells within each type's range (0: cannot attack) */
    uint32_t producible[NRTS_MAX_TYPES];      /* bit t: the type produces type t */
    uint32_t resource_types;                  /* bit t: type t is a resource */
    uint32_t stockpile_types;                 /* bit t: type t is a stockpile */
    int32_t table[NRTS_MAX_TYPES * (NRTS_TABLE_COLUMNS + NRTS_MAX_TYPES)]; /* [T, 15+T], see nrts_prepare_scenario */
} NrtsScenario;

/* Per-scenario content of a launch. */
typedef struct NrtsContent {
    NrtsScenario scenario;          /* host struct, passed by value to the kernels */
    const void* reset[NRTS_LEAVES]; /* device pointers: one game's reset State, decide(initial_state) */
} NrtsContent;

/* Fills `out` from host arrays: terrain uint8 [H*W] (0/1 walls) and the unit
 * table int32 [T, 15+T] with columns cost, hit_points, produce_time,
 * move_time, attack_time, harvest_time, attack_range, attack_damage,
 * harvest_amount, sight_radius, is_resource, is_stockpile, can_harvest,
 * can_move, can_attack, then produces[T] (model/unit_types.py:47-148). */
int nrts_prepare_scenario(const NrtsExtents* extents, const uint8_t* terrain, const int32_t* table, NrtsScenario* out);

/* A batch of games, device pointers, updated in place. */
typedef struct NrtsState {
    void* leaf[NRTS_LEAVES];
    uint32_t* environment_root;   /* [L, 2] threefry key data of each game's reset key */
    uint32_t* episode_index;      /* [L] */
} NrtsState;

/* Outputs of a step, device pointers.  Null pointers skip that output. */
typedef struct NrtsOutputs {
    uint8_t* masks[2];            /* legality rows of the carried (post-reset) state */
    uint8_t* feature_maps[2];     /* observation of the carried state */
    int32_t* scalars[2];
    float* reward;                /* [L, 2] */
    uint8_t* done;                /* [L] terminated | truncated */
    uint8_t* terminated;          /* [L] */
    uint8_t* truncated;           /* [L] */
    int32_t* winner;              /* [L] of the ending state, before the reset */
    int32_t* spawn_overflow;      /* [L, 2] telemetry of the ending state */
    uint8_t* final_feature_maps[2]; /* observation of the ending state, before the reset */
    int32_t* final_scalars[2];
    /* Optional fused draw of the next actions from the legality rows this
     * call writes: int32 [L, C, 7] per player, the same values
     * nrts_sample_actions gives for (sample_seed, sample_counter). */
    int32_t* sampled_actions[2];
    uint64_t sample_seed;
    uint64_t sample_counter;
    /* Optional reward components float [L, 2, 6] of each step
     * (adapters/rewards.py:20-72): win_loss, resource_gather, produce_worker,
     * produce_building, attack, produce_combat_unit; needs the 7 standard unit types. */
    float* reward_components;
    /* Optional legality rows in the packed form uint32 [L, C, 3] per player
     * (mask_form="packed", adapters/factors.py:89-103): word 0 holds the
     * 6+16+T kind, direction and produce-type bits, words 1 and 2 the attack
     * window's bits 0-31 and 32-63. */
    uint32_t* packed_masks[2];
    /* Scheduling hint: nonzero takes the games last to first.  Alternating it
     * between consecutive steps of one batch lets the games the previous launch
     * wrote last (still in L2) go first; results do not depend on it. */
    uint32_t reverse_order;
} NrtsOutputs;

/* One environment step for every game: decode the action rows, the core step
 * (admission, conflicts, completion, outcome), auto-reset of finished games,
 * then the next step's masks and both players' observations.
 * Replaces NanoRTS.step (adapters/jaxmarl/facade.py:107-119). */
int nrts_step(const NrtsExtents* extents, const NrtsContent* content, const NrtsState* state, int64_t lanes,
              const int32_t* actions0, const int32_t* actions1, const NrtsOutputs* outputs, void* stream);

/* One group of a multi-group step: its own content (map, unit table, reset
 * State), State buffers, lane count, action rows and outputs.  Every group's
 * extents must equal the first group's except max_cycles. */
#define NRTS_MAX_GROUPS 8
typedef struct NrtsGroupStep {
    const NrtsExtents* extents;
    const NrtsContent* content;
    const NrtsState* state;
    int64_t lanes;
    const int32_t* actions[2];
    const NrtsOutputs* outputs;
} NrtsGroupStep;

/* nrts_step for up to NRTS_MAX_GROUPS groups of games in one launch
 * (core.step_groups, core/__init__.py:63-89, as GroupMix steps groups that
 * share a bucket, bots/mix.py:130-160). */
int nrts_step_groups(const NrtsGroupStep* groups, int32_t count, void* stream);

/* Every game to its reset State with episode 0 and the given root keys
 * ([L, 2] uint32, may alias state->environment_root); writes masks and
 * observations of that state.  Replaces NanoRTS.reset (facade.py:100-105). */
int nrts_reset(const NrtsExtents* extents, const NrtsContent* content, const NrtsState* state, int64_t lanes,
               const uint32_t* keys, const NrtsOutputs* outputs, void* stream);

/* Legality rows of the current state (get_avail_actions, facade.py:172-174). */
int nrts_legal_masks(const NrtsExtents* extents, const NrtsContent* content, const NrtsState* state, int64_t lanes,
                     uint8_t* masks0, uint8_t* masks1, void* stream);

/* Legality rows of the current state in the packed form (see
 * NrtsOutputs.packed_masks): jaxmarl.legal_actions with mask_form="packed"
 * (adapters/jaxmarl/actions.py:28-41). */
int nrts_packed_masks(const NrtsExtents* extents, const NrtsContent* content, const NrtsState* state, int64_t lanes,
                      uint32_t* words0, uint32_t* words1, void* stream);

/* Observations of the current state (get_obs, facade.py:166-170). */
int nrts_observe(const NrtsExtents* extents, const NrtsContent* content, const NrtsState* state, int64_t lanes,
                 uint8_t* feature_maps0, uint8_t* feature_maps1, int32_t* scalars0, int32_t* scalars1, void* stream);

/* int32 [L, 2, C] cell of each player slot, -1 when empty (get_slot_cells, facade.py:176-178). */
int nrts_slot_cells(const NrtsExtents* extents, const NrtsState* state, int64_t lanes, int32_t* cells, void* stream);

/* Uniform draw over the set bits of each factor group of every mask row
 * (0 when a group has none), for rollouts and benchmarks: the stand-in for
 * per-factor jax.random.categorical over masked logits (README.md:53-63).
 * Deterministic in (seed, counter, game, player, slot, factor). */
int nrts_sample_actions(const NrtsExtents* extents, int64_t lanes, const uint8_t* masks0, const uint8_t* masks1,
                        int32_t* actions0, int32_t* actions1, uint64_t seed, uint64_t counter, void* stream);

/* One player's rush-bot carry: the reference's AbstractActions pytree
 * (bots/abstraction.py:71-82) as lane-major device buffers.  The nine int32
 * [L, C] fields are, in order, kind, unit_birth, order, target, target_birth,
 * base, base_birth, cell, unit_type; trained is uint8 [L, C] (0/1) and
 * next_order int32 [L].  A new episode starts from empty_actions
 * (abstraction.py:120-135): every int32 field -1, trained 0, next_order 0. */
#define NRTS_CARRY_FIELDS 9
typedef struct NrtsBotCarry {
    int32_t* field[NRTS_CARRY_FIELDS];
    uint8_t* trained;
    int32_t* next_order;
} NrtsBotCarry;

/* Rush-family strategies (bots/family.py:14-15). */
enum NrtsBotStrategy { NRTS_WORKER_RUSH = 0, NRTS_BARRACKS_RUSH = 1 };

/* One scripted player: WorkerRush is {NRTS_WORKER_RUSH, -1}; LightRush is
 * {NRTS_BARRACKS_RUSH, 4} (TYPE_LIGHT, bots/light_rush.py:13-18). */
typedef struct NrtsBot {
    int32_t strategy;   /* NrtsBotStrategy */
    int32_t trained;    /* unit type a BARRACKS_RUSH barracks trains; ignored by WORKER_RUSH */
    NrtsBotCarry carry; /* updated in place */
} NrtsBot;

/* family.act of one player's rush bot on every game: the script
 * (bots/rush.py:225-246) updates the carry, the abstraction layer
 * (bots/abstraction.py:282-314, one A* search per executing unit) turns it
 * into Commands.  `commands` is int32 [L, 6, 2, C]: the Commands fields kind,
 * direction, none_duration, target_cell, produced_type, request_order
 * (model/commands.py:22-35), each [2, C]; the other player's row is unissued
 * (-1, -1, 0, -1, -1, -1).  The state is read only. */
int nrts_bot_act(const NrtsExtents* extents, const NrtsContent* content, const NrtsState* state, int64_t lanes,
                 int32_t player, const NrtsBot* bot, int32_t* commands, void* stream);

/* One bot-against-bot step for every game: bots[p] chooses player p's
 * Commands from the step's starting state, then the core step, outcome and
 * auto-reset as nrts_step; a finished game's carries return to
 * empty_actions (bots/seat.py:127).  Outputs as nrts_step; masks,
 * observations and the fused draw are optional (null skips them). */
int nrts_duel_step(const NrtsExtents* extents, const NrtsContent* content, const NrtsState* state, int64_t lanes,
                   const NrtsBot* bots, const NrtsOutputs* outputs, void* stream);

/* Status word: the device writes a nonzero code here when a kernel's bounded
 * wait gives up (that game and the rest of its warp's games are then left
 * unstepped).  Reads and clears it in one atomic swap on the device (the
 * legacy default stream, synchronously) and returns it. */
int nrts_device_status(int device);

/* Build identity string of this library. */
const char* nrts_build_id(void);

/* Runs probe kernels on each listed device and checks warp ballot and
 * shuffle results, that every kernel image loads, and that a bounded wait on
 * an mbarrier nothing completes gives up after 1 ms and records a status of
 * its own (the status word above is not touched).  Returns 0 when all pass. */
int nrts_self_check(const int32_t* devices, int64_t count);

/* The same checks as nrts_self_check, with no device allocation: no
 * cudaMalloc, cudaFree or allocating library routine.  No counterpart in the
 * reference (its self check, registry.cu:201-229, is nrts_self_check).
 *
 * For callers that cannot allocate device memory themselves.  A JAX process
 * is the usual one: XLA's client takes most or all of each GPU's memory at
 * start-up for its own allocator, so a cudaMalloc outside it can fail even
 * for a few bytes, and a custom call is meant to draw memory only from XLA.
 * nrts_self_check allocates 140 bytes per device for its probe results; this
 * entry point writes them instead into a static device array of the library
 * (64 int32, 256 bytes, present on every GPU that loads the library until the
 * process exits).
 *
 * Limits: at most 64 devices per call, each index in 0..63; more, or a
 * negative count, is refused with NRTS_E_ARGUMENT before any device work.
 * The first call on a device looks up the array's device address with that
 * device current (cudaGetSymbolAddress) and keeps it; make that first call
 * before any stream capture.  Every call on a device reuses the same array
 * (cleared at the start of each call), so calls that overlap on one GPU, from
 * two host threads or processes sharing a context, race on it. */
int nrts_self_check_no_alloc(const int32_t* devices, int64_t count);

/* Message of the last failed call on this host thread. */
const char* nrts_last_error(void);

#ifdef __cplusplus
}
#endif

#endif /* NANORTS_B200_H */
