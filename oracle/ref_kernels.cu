// Harness around NanoRTS's own CUDA kernels (TEST INFRASTRUCTURE).
//
// The Makefile target `ref` compiles the reference's kernel sources unchanged,
// from where they lie in the reference tree, together with this file:
//   core/cuda/step.cu              nanorts_step            (step.cu:653-698, kernel :379-387)
//   core/cuda/legality.cu          nanorts_legality(_words) (legality.cu:535-561, kernel :344-378)
//   observations/cuda/visibility.cu nanorts_visible_cells  (visibility.cu:86-141, kernel :21-71)
//   adapters/cuda/reset.cu         nanorts_reset_packed_where_done (reset.cu:196-221, kernel :42-80)
//   bots/cuda/abstraction_act.cu   nanorts_abstraction_act (abstraction_act.cu:1232-1322, kernel :1099)
// against the interface stand-in in ffi_standin/ (jaxlib, which ships the real
// XLA FFI header, is absent).  Each handler's XLA_FFI_DEFINE_HANDLER_SYMBOL
// there exports the address of its implementation function; the entry points
// below describe plain device buffers as the handler's buffers and call that
// implementation, so the reference's own validation, launch geometry and
// kernels run as they do under XLA.  The build compiles them for
// `arch=compute_100,code=sm_100`, the image the reference's own build
// (kernels/build.py:84-86,137-143) produces for a B200.
//
// The tests use these entry points to pin the oracle and the product's
// kernels to the reference; nothing in the product links them.
#include <cstdint>
#include <string>
#include <string_view>
#include <vector>

#include <cuda_runtime.h>

#include "xla/ffi/api/ffi.h"
#include "nanorts_ffi.cuh"

namespace ffi = xla::ffi;

// Definitions the reference declares in kernels/cuda/nanorts_ffi.cuh and
// defines in its registry (kernels/cuda/registry.cu), which is not built here:
// one fixed build id (every call passes it back), and no kernel registry.
namespace nanorts {
std::string_view build_id() { return "nanorts-reference-harness"; }
Target::Target(const char*) {}
Kernels::Kernels(const char*, std::vector<const void*>) {}
}  // namespace nanorts

extern "C" {
void* nanorts_step_implementation(void);
void* nanorts_legality_implementation(void);
void* nanorts_legality_words_implementation(void);
void* nanorts_visible_cells_implementation(void);
void* nanorts_reset_packed_where_done_implementation(void);
void* nanorts_abstraction_act_implementation(void);
}

// A device buffer described by the caller: element type code of the
// stand-in's DataType, rank and extents.
struct RefBufferView {
    void* data;
    int32_t dtype;
    int32_t rank;
    int64_t dims[6];
};

namespace {

thread_local std::string g_error;

ffi::AnyBuffer any(const RefBufferView& b) {
    return ffi::AnyBuffer(b.data, static_cast<ffi::DataType>(b.dtype), b.dims, static_cast<size_t>(b.rank));
}

std::vector<ffi::AnyBuffer> all(const RefBufferView* b, int64_t n) {
    std::vector<ffi::AnyBuffer> out;
    for (int64_t k = 0; k < n; ++k) out.push_back(any(b[k]));
    return out;
}

int finish(const ffi::Error& error) {
    if (error.failure()) {
        g_error = error.message();
        return error.code();
    }
    return 0;
}

using StepFn = ffi::Error (*)(cudaStream_t, ffi::RemainingArgs, ffi::RemainingRets, std::string_view, int64_t);
using WordsFn = ffi::Error (*)(cudaStream_t, ffi::AnyBuffer, ffi::AnyBuffer, ffi::AnyBuffer, ffi::AnyBuffer, ffi::AnyBuffer,
                               ffi::AnyBuffer, ffi::AnyBuffer, ffi::AnyBuffer, ffi::AnyBuffer, ffi::Result<ffi::AnyBuffer>,
                               std::string_view, int64_t);
using RowsFn = ffi::Error (*)(cudaStream_t, ffi::AnyBuffer, ffi::AnyBuffer, ffi::AnyBuffer, ffi::AnyBuffer, ffi::AnyBuffer,
                              ffi::AnyBuffer, ffi::AnyBuffer, ffi::AnyBuffer, ffi::AnyBuffer, ffi::Result<ffi::AnyBuffer>,
                              std::string_view);
using VisibleFn = ffi::Error (*)(cudaStream_t, ffi::AnyBuffer, ffi::AnyBuffer, ffi::AnyBuffer, ffi::AnyBuffer,
                                 ffi::Result<ffi::AnyBuffer>, std::string_view, int64_t, int64_t, int64_t, int64_t);
using ActFn = ffi::Error (*)(cudaStream_t, ffi::RemainingArgs, ffi::RemainingRets, std::string_view, int64_t, int64_t);
using ResetFn = ffi::Error (*)(cudaStream_t, ffi::Buffer<ffi::PRED>, ffi::AnyBuffer, ffi::RemainingArgs, ffi::RemainingRets,
                               std::string_view, int64_t);

}  // namespace

extern "C" {

typedef RefBufferView RefBuffer;

const char* ref_last_error(void) { return g_error.c_str(); }

// nanorts_step: 33 operands (key, the six Commands rows, terrain, unit table,
// timings, the 23 State leaves) and 31 results (the 23 leaves, per-slot leaves
// and entity_at aliased with their operands, then the step's event rows), in
// the order of the reference's Operand / Leaf / Result enums (step.cu:48-108).
int ref_step(void* stream, const RefBuffer* operands, int64_t n_operands, const RefBuffer* results, int64_t n_results,
             int64_t strategy) {
    const std::vector<ffi::AnyBuffer> args = all(operands, n_operands), rets = all(results, n_results);
    const StepFn fn = reinterpret_cast<StepFn>(nanorts_step_implementation());
    return finish(fn(static_cast<cudaStream_t>(stream), ffi::RemainingArgs(args.data(), args.size()),
                     ffi::RemainingRets(rets.data(), rets.size()), nanorts::build_id(), strategy));
}

// nanorts_legality_words: operands birth, unit_type, owner, carried_resources,
// cell, entity_at, player_resources, terrain, table; result uint32[L, 2, C, 3].
int ref_legality_words(void* stream, const RefBuffer* operands, const RefBuffer* words, int64_t offsets) {
    const std::vector<ffi::AnyBuffer> a = all(operands, 9);
    const WordsFn fn = reinterpret_cast<WordsFn>(nanorts_legality_words_implementation());
    return finish(fn(static_cast<cudaStream_t>(stream), a[0], a[1], a[2], a[3], a[4], a[5], a[6], a[7], a[8],
                     ffi::Result<ffi::AnyBuffer>(any(*words)), nanorts::build_id(), offsets));
}

// nanorts_legality: the same operands; result bool[L, 2, C, 22 + T + O].
int ref_legality_rows(void* stream, const RefBuffer* operands, const RefBuffer* rows) {
    const std::vector<ffi::AnyBuffer> a = all(operands, 9);
    const RowsFn fn = reinterpret_cast<RowsFn>(nanorts_legality_implementation());
    return finish(fn(static_cast<cudaStream_t>(stream), a[0], a[1], a[2], a[3], a[4], a[5], a[6], a[7], a[8],
                     ffi::Result<ffi::AnyBuffer>(any(*rows)), nanorts::build_id()));
}

// nanorts_visible_cells: operands birth, unit_type, cell, sight radius [1, T];
// result bool[L, H, W] for the slots [first, first + count).
int ref_visible_cells(void* stream, const RefBuffer* operands, const RefBuffer* out, int64_t first, int64_t count, int64_t width,
                      int64_t height) {
    const std::vector<ffi::AnyBuffer> a = all(operands, 4);
    const VisibleFn fn = reinterpret_cast<VisibleFn>(nanorts_visible_cells_implementation());
    return finish(fn(static_cast<cudaStream_t>(stream), a[0], a[1], a[2], a[3], ffi::Result<ffi::AnyBuffer>(any(*out)),
                     nanorts::build_id(), first, count, width, height));
}

// nanorts_reset_packed_where_done: done bool[L], the packed reset rows (one
// shared uint8 row, each leaf's row at the next 16-byte offset), then `count`
// next leaves and `count` results (aliased for an in-place reset).
int ref_reset_packed_where_done(void* stream, const RefBuffer* done, const RefBuffer* packed, const RefBuffer* next,
                                const RefBuffer* results, int64_t count) {
    const std::vector<ffi::AnyBuffer> args = all(next, count), rets = all(results, count);
    const ResetFn fn = reinterpret_cast<ResetFn>(nanorts_reset_packed_where_done_implementation());
    return finish(fn(static_cast<cudaStream_t>(stream), ffi::Buffer<ffi::PRED>(any(*done)), any(*packed),
                     ffi::RemainingArgs(args.data(), args.size()), ffi::RemainingRets(rets.data(), rets.size()),
                     nanorts::build_id(), count));
}

// nanorts_abstraction_act: operands are the ten State leaves the bots read
// (bots/whole_act.py:22-33), terrain, the bot unit table [1, T, 6], the player
// [1], then the carry (nine int32 [L, C] rows, trained, next_order); results
// are the carry (aliased) and the Commands int32 [L, 6, 2, C].
int ref_abstraction_act(void* stream, const RefBuffer* operands, int64_t n_operands, const RefBuffer* results,
                        int64_t n_results, int64_t strategy, int64_t trained) {
    const std::vector<ffi::AnyBuffer> args = all(operands, n_operands), rets = all(results, n_results);
    const ActFn fn = reinterpret_cast<ActFn>(nanorts_abstraction_act_implementation());
    return finish(fn(static_cast<cudaStream_t>(stream), ffi::RemainingArgs(args.data(), args.size()),
                     ffi::RemainingRets(rets.data(), rets.size()), nanorts::build_id(), strategy, trained));
}

}  // extern "C"
