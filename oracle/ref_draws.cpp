// Reference build of NanoRTS's conflict-draw composition (TEST INFRASTRUCTURE).
//
// Compiles the reference's own header src/nanorts/core/cuda/conflict_draw.cuh
// (its restatement of jax.random.fold_in / randint under threefry2x32) from
// where it lies in the reference tree, as host code: its functions are
// __host__ __device__, so defining both qualifiers away leaves plain C++.
// The Makefile target `ref` builds this into oracle/_ref/libref_draws.so; the
// oracle's own threefry (oracle.hpp) is checked against it in tests/.
#include <cstdint>

#include "conflict_draw.cuh"

extern "C" {

void ref_threefry2x32(uint32_t k0, uint32_t k1, uint32_t* x0, uint32_t* x1) {
    nanorts::draws::threefry2x32(nanorts::draws::Key{k0, k1}, *x0, *x1);
}

void ref_fold_in(uint32_t k0, uint32_t k1, int32_t data, uint32_t* out) {
    const nanorts::draws::Key k = nanorts::draws::fold_in(nanorts::draws::Key{k0, k1}, data);
    out[0] = k.k0;
    out[1] = k.k1;
}

int32_t ref_conflict_draw(uint32_t k0, uint32_t k1, int32_t time, int32_t birth, int32_t ordinal) {
    const nanorts::draws::Key address = nanorts::draws::conflict_address(nanorts::draws::Key{k0, k1}, time, birth);
    return nanorts::draws::conflict_draw(address, ordinal);
}

}
