// Device helpers for the sm_100a kernels: TMA bulk copies, mbarriers, warp
// primitives, threefry2x32.
#pragma once

#include <cstdint>

namespace nrts {

constexpr unsigned kFull = 0xffffffffu;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// 1D TMA bulk copy global -> shared, completing on an mbarrier.  Both
// addresses 16-byte aligned, size a multiple of 16.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// 1D TMA bulk copy shared -> global in the issuing thread's bulk group.
__device__ __forceinline__ void bulk_store(void* dst, const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(smem_u32(src)), "r"(bytes)
                 : "memory");
}

// L2 prefetch of a 16-byte-aligned span whose size is a multiple of 16.
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }

// Orders this thread's generic-proxy shared-memory writes before later
// async-proxy (TMA) reads of them.
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ unsigned lanes_below(int lane) { return (1u << lane) - 1u; }

__device__ __forceinline__ int32_t clampi(int32_t v, int32_t lo, int32_t hi) { return v < lo ? lo : (v > hi ? hi : v); }

__device__ __forceinline__ int32_t floor_div(int32_t a, int32_t b) {
    const int32_t q = a / b;
    return (a % b != 0 && ((a < 0) != (b < 0))) ? q - 1 : q;
}

__device__ __forceinline__ int32_t floor_mod(int32_t a, int32_t b) { return a - floor_div(a, b) * b; }

// lowbias32 (C. Wellons' published 32-bit integer hash): an avalanching mixer.
__host__ __device__ __forceinline__ uint32_t mix32(uint32_t x) {
    x ^= x >> 16;
    x *= 0x7feb352du;
    x ^= x >> 15;
    x *= 0x846ca68bu;
    x ^= x >> 16;
    return x;
}

// Bit position of the k-th (0-based) set bit of v; k < popc(v).
__device__ __forceinline__ int select32(uint32_t v, int k) {
    int pos = 0, c = __popc(v & 0xffffu);
    if (k >= c) { k -= c; v >>= 16; pos += 16; }
    c = __popc(v & 0xffu);
    if (k >= c) { k -= c; v >>= 8; pos += 8; }
    c = __popc(v & 0xfu);
    if (k >= c) { k -= c; v >>= 4; pos += 4; }
    c = __popc(v & 0x3u);
    if (k >= c) { k -= c; v >>= 2; pos += 2; }
    return pos + (k >= static_cast<int>(v & 1u) ? 1 : 0);
}

// Four bits -> four 0/1 bytes (bit i to byte i).
__device__ __forceinline__ uint32_t spread4(uint32_t v) { return (v * 0x00204081u) & 0x01010101u; }

// threefry2x32, 20 rounds (Salmon et al., SC'11): key schedule with the
// Skein parity constant and a key injection after every fourth round.
__device__ __forceinline__ void threefry2x32(uint32_t k0, uint32_t k1, uint32_t& x0, uint32_t& x1) {
    const uint32_t k2 = k0 ^ k1 ^ 0x1BD11BDAu;
    const uint32_t ks[3] = {k0, k1, k2};
    x0 += k0;
    x1 += k1;
#pragma unroll
    for (int group = 0; group < 5; ++group) {
        const int base = (group & 1) * 4;
        const int rot[8] = {13, 15, 26, 6, 17, 29, 16, 24};
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            x0 += x1;
            x1 = __funnelshift_l(x1, x1, rot[base + r]);
            x1 ^= x0;
        }
        x0 += ks[(group + 1) % 3];
        x1 += ks[(group + 2) % 3] + static_cast<uint32_t>(group + 1);
    }
}

// jax.random.fold_in under threefry: threefry(key, (0, data)).
__device__ __forceinline__ void fold_in(uint32_t& k0, uint32_t& k1, uint32_t data) {
    uint32_t x0 = 0u, x1 = data;
    threefry2x32(k0, k1, x0, x1);
    k0 = x0;
    k1 = x1;
}

// jax.random.randint(key, (), 0, 2) with partitionable threefry: the second
// foldlike split key's 32 random bits, mod 2.
__device__ __forceinline__ int32_t randint01(uint32_t k0, uint32_t k1) {
    uint32_t s0 = 0u, s1 = 1u;
    threefry2x32(k0, k1, s0, s1);
    uint32_t b0 = 0u, b1 = 0u;
    threefry2x32(s0, s1, b0, b1);
    return static_cast<int32_t>((b0 ^ b1) & 1u);
}

}  // namespace nrts
