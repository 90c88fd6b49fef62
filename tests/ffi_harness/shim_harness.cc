// Test harness for nanorts_b200/ffi/nanorts_b200_ffi.cc (TEST INFRASTRUCTURE).
//
// Built by tests/test_jax_ffi.py together with the handler file against the
// XLA FFI interface stand-in (oracle/ffi_standin), whose handler macro
// exports each handler's implementation.  These entry points describe plain
// device buffers as the handler's operands and results and call it, so the
// tests drive the jax.ffi handlers exactly as XLA would hand them buffers.
#include <cstdint>
#include <string>
#include <vector>

#include <cuda_runtime.h>

#include "xla/ffi/api/ffi.h"

namespace ffi = xla::ffi;

// Same layout as oracle/ref_kernels.py RefBuffer.
struct ShimBuffer {
    void* data;
    int32_t dtype;
    int32_t rank;
    int64_t dims[6];
};

extern "C" {
void* nanorts_b200_step_implementation(void);
void* nanorts_b200_reset_implementation(void);
void* nanorts_b200_legal_masks_implementation(void);
void* nanorts_b200_observe_implementation(void);
void* nanorts_b200_bot_act_implementation(void);
}

namespace {

thread_local std::string g_error;

std::vector<ffi::AnyBuffer> all(const ShimBuffer* b, int64_t n) {
    std::vector<ffi::AnyBuffer> out;
    for (int64_t k = 0; k < n; ++k)
        out.emplace_back(b[k].data, static_cast<ffi::DataType>(b[k].dtype), b[k].dims, static_cast<size_t>(b[k].rank));
    return out;
}

int finish(const ffi::Error& e) {
    if (e.failure()) {
        g_error = e.message();
        return e.code();
    }
    return 0;
}

using Handler = ffi::Error (*)(cudaStream_t, ffi::RemainingArgs, ffi::RemainingRets, int64_t, int64_t, int64_t, int64_t,
                               int64_t, int64_t, int64_t, int64_t, int64_t, ffi::Span<const int32_t>,
                               ffi::Span<const int32_t>);
using BotHandler = ffi::Error (*)(cudaStream_t, ffi::RemainingArgs, ffi::RemainingRets, int64_t, int64_t, int64_t, int64_t,
                                  int64_t, int64_t, int64_t, int64_t, int64_t, ffi::Span<const int32_t>,
                                  ffi::Span<const int32_t>, int64_t, int64_t, int64_t);

}  // namespace

extern "C" {

const char* shim_last_error(void) { return g_error.c_str(); }

// target: 0 step, 1 reset, 2 legal_masks, 3 observe, 4 bot_act.  ints: the
// nine scenario attributes, then (bot_act) player, bot_strategy, trained_type.
int shim_call(int32_t target, void* stream, const ShimBuffer* args, int64_t n_args, const ShimBuffer* rets, int64_t n_rets,
              const int64_t* ints, const int32_t* terrain, int64_t n_terrain, const int32_t* table, int64_t n_table) {
    const std::vector<ffi::AnyBuffer> a = all(args, n_args), r = all(rets, n_rets);
    const ffi::RemainingArgs ra(a.data(), a.size());
    const ffi::RemainingRets rr(r.data(), r.size());
    const ffi::Span<const int32_t> t(terrain, static_cast<size_t>(n_terrain)), tb(table, static_cast<size_t>(n_table));
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    void* (*const impl[4])(void) = {nanorts_b200_step_implementation, nanorts_b200_reset_implementation,
                                    nanorts_b200_legal_masks_implementation, nanorts_b200_observe_implementation};
    if (target >= 0 && target < 4) {
        const Handler h = reinterpret_cast<Handler>(impl[target]());
        return finish(h(s, ra, rr, ints[0], ints[1], ints[2], ints[3], ints[4], ints[5], ints[6], ints[7], ints[8], t, tb));
    }
    if (target == 4) {
        const BotHandler h = reinterpret_cast<BotHandler>(nanorts_b200_bot_act_implementation());
        return finish(h(s, ra, rr, ints[0], ints[1], ints[2], ints[3], ints[4], ints[5], ints[6], ints[7], ints[8], t, tb, ints[9],
                        ints[10], ints[11]));
    }
    g_error = "unknown target";
    return -1;
}

}  // extern "C"
