// XLA FFI handlers over the nanorts_b200 C ABI: the jax.ffi custom calls a
// JAX program (NanoRTS's own core.step / legal_commands / observe / bots)
// registers in place of the reference's targets.
//
// Built by nanorts_b200/build.py (build_ffi) only where jaxlib's
// xla/ffi/api/ffi.h is found, linked with libnanorts_b200.so, and registered
// by nanorts_b200/jax_binding.py:register(), as NanoRTS registers its own
// library (src/nanorts/kernels/library.py:27-69; handler symbols as
// kernels/cuda/nanorts_ffi.cuh:57-59 declares them).
//
// Every handler takes the same operand prefix, all lane-major [L, ...]:
//   0..22   the 23 State leaves (NrtsLeaf order), aliased to results 0..22
//   23      environment_root uint32 [L, 2]     (aliased to result 23)
//   24      episode_index   uint32 [L]         (aliased to result 24)
//   25..47  the reset State, one game's decided initial State per leaf as a
//           shared row [1, ...] (the rows nanorts_reset_packed_where_done
//           copies, reset.cu:196): operands, not attributes, so the
//           executable holds no device pointer and runs on any device
// and the scenario as attributes: height, width, neutral, capacity, types,
// offsets, strategy, max_cycles, partial_observability (int64), terrain
// (int32 [H * W], 0/1 walls) and table (int32 [T * (15 + T)], the unit table
// nrts_prepare_scenario reads).  Handlers launch on the XLA stream and are
// graph-capturable (no host synchronisation, no allocation).
//
//   nanorts_b200_step         + actions0, actions1 int32 [L, C, 7]
//                             results: 25 leaves, masks0/1 (pred or uint8) [L, C, W],
//                             feature maps0/1 uint8 [L, H, W, 6], scalars0/1 int32 [L, 4],
//                             reward f32 [L, 2], done, terminated, truncated pred [L],
//                             winner int32 [L], spawn_overflow int32 [L, 2]
//   nanorts_b200_reset        + keys uint32 [L, 2]; results: 25 leaves, masks0/1,
//                             feature maps0/1, scalars0/1
//   nanorts_b200_legal_masks  results: masks0/1
//   nanorts_b200_observe      results: feature maps0/1, scalars0/1
//   nanorts_b200_bot_act      + the bot's carry (nine int32 [L, C] fields, trained
//                             pred/uint8 [L, C], next_order int32 [L]);
//                             results: the carry (aliased), Commands int32 [L, 6, 2, C];
//                             attributes player, bot_strategy, trained_type
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

#include <cuda_runtime.h>

#include "xla/ffi/api/ffi.h"
#include "nanorts_b200.h"

namespace ffi = xla::ffi;

namespace {

constexpr int64_t kStateOperands = NRTS_LEAVES + 2;           // leaves, root, episode
constexpr int64_t kPrefix = kStateOperands + NRTS_LEAVES;     // + reset rows

ffi::Error failed(const std::string& what) { return ffi::Error::InvalidArgument("nanorts_b200: " + what); }

// The launch's extents and content from attributes and the reset-row operands.
struct Bound {
    NrtsExtents x{};
    NrtsContent content{};
    NrtsState state{};
    int64_t lanes = 0;
};

ffi::Error bind(const ffi::RemainingArgs& args, int64_t height, int64_t width, int64_t neutral, int64_t capacity,
                int64_t types, int64_t offsets, int64_t strategy, int64_t max_cycles, int64_t partial,
                ffi::Span<const int32_t> terrain, ffi::Span<const int32_t> table, Bound& b) {
    if (static_cast<int64_t>(args.size()) < kPrefix) return failed("too few operands");
    b.x = NrtsExtents{static_cast<int32_t>(height), static_cast<int32_t>(width), static_cast<int32_t>(neutral),
                      static_cast<int32_t>(capacity), static_cast<int32_t>(types), static_cast<int32_t>(offsets),
                      static_cast<int32_t>(strategy), static_cast<int32_t>(max_cycles), static_cast<int32_t>(partial)};
    if (static_cast<int64_t>(terrain.size()) != height * width) return failed("terrain holds one value per cell");
    if (static_cast<int64_t>(table.size()) != types * (NRTS_TABLE_COLUMNS + types)) return failed("the table is [T, 15 + T]");
    std::vector<uint8_t> walls(terrain.size());
    for (size_t k = 0; k < terrain.size(); ++k) walls[k] = terrain[k] != 0;
    if (nrts_prepare_scenario(&b.x, walls.data(), table.data(), &b.content.scenario) != NRTS_OK)
        return failed(nrts_last_error());
    for (int k = 0; k < NRTS_LEAVES; ++k) {
        auto leaf = args.get<ffi::AnyBuffer>(k);
        auto reset = args.get<ffi::AnyBuffer>(kStateOperands + k);
        if (!leaf.has_value() || !reset.has_value()) return failed("a State or reset operand is missing");
        const auto dims = leaf->dimensions();
        if (dims.size() == 0) return failed("State leaves are lane-major [L, ...]");
        if (k == 0) b.lanes = dims[0];
        if (dims[0] != b.lanes) return failed("every State leaf has the same lane count");
        if (reset->dimensions().size() == 0 || reset->dimensions()[0] != 1) return failed("reset rows are shared rows [1, ...]");
        if (b.lanes > 0 && reset->size_bytes() * static_cast<size_t>(b.lanes) != leaf->size_bytes())
            return failed("a reset row does not match its State leaf");
        b.state.leaf[k] = leaf->untyped_data();
        b.content.reset[k] = reset->untyped_data();
    }
    auto root = args.get<ffi::AnyBuffer>(NRTS_LEAVES);
    auto episode = args.get<ffi::AnyBuffer>(NRTS_LEAVES + 1);
    if (!root.has_value() || !episode.has_value()) return failed("environment_root or episode_index is missing");
    if (root->size_bytes() != static_cast<size_t>(b.lanes) * 8 || episode->size_bytes() != static_cast<size_t>(b.lanes) * 4)
        return failed("environment_root is uint32 [L, 2] and episode_index uint32 [L]");
    b.state.environment_root = static_cast<uint32_t*>(root->untyped_data());
    b.state.episode_index = static_cast<uint32_t*>(episode->untyped_data());
    return ffi::Error::Success();
}

// Result k's device pointer, checked to hold `bytes` bytes.
template <typename T>
ffi::Error result(const ffi::RemainingRets& rets, size_t k, size_t bytes, T*& out) {
    auto r = rets.get<ffi::AnyBuffer>(k);
    if (!r.has_value()) return failed("a result is missing");
    if ((*r)->size_bytes() != bytes) return failed("result " + std::to_string(k) + " has another size");
    out = static_cast<T*>((*r)->untyped_data());
    return ffi::Error::Success();
}

// The State results must alias their operands (the state is updated in place).
ffi::Error check_aliased(const ffi::RemainingRets& rets, const Bound& b) {
    for (int k = 0; k < NRTS_LEAVES + 2; ++k) {
        auto r = rets.get<ffi::AnyBuffer>(k);
        if (!r.has_value()) return failed("a State result is missing");
        const void* operand = k < NRTS_LEAVES ? b.state.leaf[k]
                              : k == NRTS_LEAVES ? static_cast<const void*>(b.state.environment_root)
                                                 : static_cast<const void*>(b.state.episode_index);
        if ((*r)->untyped_data() != operand) return failed("State results alias their operands (input_output_aliases)");
    }
    return ffi::Error::Success();
}

ffi::Error finish(int rc) { return rc == NRTS_OK ? ffi::Error::Success() : ffi::Error::Internal(nrts_last_error()); }

int64_t mask_width(const NrtsExtents& x) { return 6 + 16 + x.types + x.offsets; }

// masks0/1, feature maps0/1, scalars0/1 results from `first`.
ffi::Error bind_outputs(const ffi::RemainingRets& rets, size_t first, const Bound& b, bool masks, bool maps, NrtsOutputs& out) {
    const size_t L = static_cast<size_t>(b.lanes), C = static_cast<size_t>(b.x.capacity);
    const size_t cells = static_cast<size_t>(b.x.height) * static_cast<size_t>(b.x.width);
    size_t k = first;
    if (masks)
        for (int p = 0; p < 2; ++p)
            if (auto e = result(rets, k++, L * C * static_cast<size_t>(mask_width(b.x)), out.masks[p]); e.failure()) return e;
    if (maps) {
        for (int p = 0; p < 2; ++p)
            if (auto e = result(rets, k++, L * cells * 6, out.feature_maps[p]); e.failure()) return e;
        for (int p = 0; p < 2; ++p)
            if (auto e = result(rets, k++, L * 4 * sizeof(int32_t), out.scalars[p]); e.failure()) return e;
    }
    return ffi::Error::Success();
}

#define NRTS_SCENARIO_PARAMS                                                                                    \
    int64_t height, int64_t width, int64_t neutral, int64_t capacity, int64_t types, int64_t offsets,          \
        int64_t strategy, int64_t max_cycles, int64_t partial_observability, ffi::Span<const int32_t> terrain, \
        ffi::Span<const int32_t> table
#define NRTS_SCENARIO_ARGS \
    height, width, neutral, capacity, types, offsets, strategy, max_cycles, partial_observability, terrain, table

ffi::Error Step(cudaStream_t stream, ffi::RemainingArgs args, ffi::RemainingRets rets, NRTS_SCENARIO_PARAMS) {
    Bound b;
    if (auto e = bind(args, NRTS_SCENARIO_ARGS, b); e.failure()) return e;
    if (static_cast<int64_t>(args.size()) != kPrefix + 2 || rets.size() != static_cast<size_t>(kStateOperands + 12))
        return failed("nanorts_b200_step takes 50 operands and returns 37 results");
    if (auto e = check_aliased(rets, b); e.failure()) return e;
    auto a0 = args.get<ffi::AnyBuffer>(kPrefix), a1 = args.get<ffi::AnyBuffer>(kPrefix + 1);
    const size_t row_bytes = static_cast<size_t>(b.lanes) * static_cast<size_t>(b.x.capacity) * 7 * sizeof(int32_t);
    if (!a0.has_value() || !a1.has_value() || a0->size_bytes() != row_bytes || a1->size_bytes() != row_bytes)
        return failed("actions are int32 [L, C, 7] per player");
    NrtsOutputs out{};
    if (auto e = bind_outputs(rets, kStateOperands, b, true, true, out); e.failure()) return e;
    const size_t L = static_cast<size_t>(b.lanes);
    size_t k = kStateOperands + 6;
    if (auto e = result(rets, k++, L * 2 * sizeof(float), out.reward); e.failure()) return e;
    if (auto e = result(rets, k++, L, out.done); e.failure()) return e;
    if (auto e = result(rets, k++, L, out.terminated); e.failure()) return e;
    if (auto e = result(rets, k++, L, out.truncated); e.failure()) return e;
    if (auto e = result(rets, k++, L * sizeof(int32_t), out.winner); e.failure()) return e;
    if (auto e = result(rets, k++, L * 2 * sizeof(int32_t), out.spawn_overflow); e.failure()) return e;
    return finish(nrts_step(&b.x, &b.content, &b.state, b.lanes, static_cast<const int32_t*>(a0->untyped_data()),
                            static_cast<const int32_t*>(a1->untyped_data()), &out, stream));
}

ffi::Error Reset(cudaStream_t stream, ffi::RemainingArgs args, ffi::RemainingRets rets, NRTS_SCENARIO_PARAMS) {
    Bound b;
    if (auto e = bind(args, NRTS_SCENARIO_ARGS, b); e.failure()) return e;
    if (static_cast<int64_t>(args.size()) != kPrefix + 1 || rets.size() != static_cast<size_t>(kStateOperands + 6))
        return failed("nanorts_b200_reset takes 49 operands and returns 31 results");
    if (auto e = check_aliased(rets, b); e.failure()) return e;
    auto keys = args.get<ffi::AnyBuffer>(kPrefix);
    if (!keys.has_value() || keys->size_bytes() != static_cast<size_t>(b.lanes) * 8) return failed("keys are uint32 [L, 2]");
    NrtsOutputs out{};
    if (auto e = bind_outputs(rets, kStateOperands, b, true, true, out); e.failure()) return e;
    return finish(nrts_reset(&b.x, &b.content, &b.state, b.lanes, static_cast<const uint32_t*>(keys->untyped_data()), &out, stream));
}

ffi::Error LegalMasks(cudaStream_t stream, ffi::RemainingArgs args, ffi::RemainingRets rets, NRTS_SCENARIO_PARAMS) {
    Bound b;
    if (auto e = bind(args, NRTS_SCENARIO_ARGS, b); e.failure()) return e;
    if (static_cast<int64_t>(args.size()) != kPrefix || rets.size() != 2)
        return failed("nanorts_b200_legal_masks takes 48 operands and returns 2 results");
    NrtsOutputs out{};
    if (auto e = bind_outputs(rets, 0, b, true, false, out); e.failure()) return e;
    return finish(nrts_legal_masks(&b.x, &b.content, &b.state, b.lanes, out.masks[0], out.masks[1], stream));
}

ffi::Error Observe(cudaStream_t stream, ffi::RemainingArgs args, ffi::RemainingRets rets, NRTS_SCENARIO_PARAMS) {
    Bound b;
    if (auto e = bind(args, NRTS_SCENARIO_ARGS, b); e.failure()) return e;
    if (static_cast<int64_t>(args.size()) != kPrefix || rets.size() != 4)
        return failed("nanorts_b200_observe takes 48 operands and returns 4 results");
    NrtsOutputs out{};
    if (auto e = bind_outputs(rets, 0, b, false, true, out); e.failure()) return e;
    return finish(nrts_observe(&b.x, &b.content, &b.state, b.lanes, out.feature_maps[0], out.feature_maps[1], out.scalars[0],
                               out.scalars[1], stream));
}

ffi::Error BotAct(cudaStream_t stream, ffi::RemainingArgs args, ffi::RemainingRets rets, NRTS_SCENARIO_PARAMS, int64_t player,
                  int64_t bot_strategy, int64_t trained_type) {
    Bound b;
    if (auto e = bind(args, NRTS_SCENARIO_ARGS, b); e.failure()) return e;
    constexpr int kCarry = NRTS_CARRY_FIELDS + 2;
    if (static_cast<int64_t>(args.size()) != kPrefix + kCarry || rets.size() != static_cast<size_t>(kCarry + 1))
        return failed("nanorts_b200_bot_act takes 59 operands and returns 12 results");
    const size_t L = static_cast<size_t>(b.lanes), C = static_cast<size_t>(b.x.capacity);
    NrtsBot bot{};
    bot.strategy = static_cast<int32_t>(bot_strategy);
    bot.trained = static_cast<int32_t>(trained_type);
    for (int f = 0; f < kCarry; ++f) {
        auto in = args.get<ffi::AnyBuffer>(kPrefix + f);
        auto r = rets.get<ffi::AnyBuffer>(f);
        if (!in.has_value() || !r.has_value() || (*r)->untyped_data() != in->untyped_data())
            return failed("the carry results alias their operands");
        const size_t bytes = f < NRTS_CARRY_FIELDS ? L * C * 4 : f == NRTS_CARRY_FIELDS ? L * C : L * 4;
        if (in->size_bytes() != bytes) return failed("the carry is nine int32 [L, C] fields, trained [L, C], next_order int32 [L]");
        if (f < NRTS_CARRY_FIELDS) bot.carry.field[f] = static_cast<int32_t*>(in->untyped_data());
        else if (f == NRTS_CARRY_FIELDS) bot.carry.trained = static_cast<uint8_t*>(in->untyped_data());
        else bot.carry.next_order = static_cast<int32_t*>(in->untyped_data());
    }
    int32_t* commands = nullptr;
    if (auto e = result(rets, kCarry, L * 6 * 2 * C * sizeof(int32_t), commands); e.failure()) return e;
    return finish(nrts_bot_act(&b.x, &b.content, &b.state, b.lanes, static_cast<int32_t>(player), &bot, commands, stream));
}

}  // namespace

#define NRTS_SCENARIO_ATTRS                                                                                  \
    .Attr<int64_t>("height").Attr<int64_t>("width").Attr<int64_t>("neutral").Attr<int64_t>("capacity")       \
        .Attr<int64_t>("types").Attr<int64_t>("offsets").Attr<int64_t>("strategy").Attr<int64_t>("max_cycles") \
        .Attr<int64_t>("partial_observability").Attr<ffi::Span<const int32_t>>("terrain")                    \
        .Attr<ffi::Span<const int32_t>>("table")

XLA_FFI_DEFINE_HANDLER_SYMBOL(nanorts_b200_step, Step,
                              ffi::Ffi::Bind().Ctx<ffi::PlatformStream<cudaStream_t>>().RemainingArgs().RemainingRets()
                                  NRTS_SCENARIO_ATTRS,
                              {ffi::Traits::kCmdBufferCompatible});
XLA_FFI_DEFINE_HANDLER_SYMBOL(nanorts_b200_reset, Reset,
                              ffi::Ffi::Bind().Ctx<ffi::PlatformStream<cudaStream_t>>().RemainingArgs().RemainingRets()
                                  NRTS_SCENARIO_ATTRS,
                              {ffi::Traits::kCmdBufferCompatible});
XLA_FFI_DEFINE_HANDLER_SYMBOL(nanorts_b200_legal_masks, LegalMasks,
                              ffi::Ffi::Bind().Ctx<ffi::PlatformStream<cudaStream_t>>().RemainingArgs().RemainingRets()
                                  NRTS_SCENARIO_ATTRS,
                              {ffi::Traits::kCmdBufferCompatible});
XLA_FFI_DEFINE_HANDLER_SYMBOL(nanorts_b200_observe, Observe,
                              ffi::Ffi::Bind().Ctx<ffi::PlatformStream<cudaStream_t>>().RemainingArgs().RemainingRets()
                                  NRTS_SCENARIO_ATTRS,
                              {ffi::Traits::kCmdBufferCompatible});
XLA_FFI_DEFINE_HANDLER_SYMBOL(nanorts_b200_bot_act, BotAct,
                              ffi::Ffi::Bind().Ctx<ffi::PlatformStream<cudaStream_t>>().RemainingArgs().RemainingRets()
                                  NRTS_SCENARIO_ATTRS.Attr<int64_t>("player").Attr<int64_t>("bot_strategy")
                                  .Attr<int64_t>("trained_type"),
                              {ffi::Traits::kCmdBufferCompatible});
