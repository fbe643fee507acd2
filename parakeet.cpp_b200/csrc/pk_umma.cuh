// pk_umma.cuh -- sm_100a building blocks shared by libparakeet_cuda's tensor-memory
// kernels (pk_encproj.cu: the enc-proj GEMM; pk_bulk.cu: the step loop for large
// live batches): mbarrier waits bounded in time, tcgen05.mma operand descriptors
// for 128-byte-swizzled K-major f16 tiles, the kind::f16 instruction descriptor,
// MMA issue / commit and 2-D TMA tile loads.
#pragma once

#include "pk_internal.h"

#include <cuda.h>

namespace pk {
namespace {

__device__ __forceinline__ unsigned smem_u32(const void * p) { return (unsigned) __cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(unsigned long long * b, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(smem_u32(b)), "r"(count) : "memory");
}

__device__ __forceinline__ bool mbar_test(unsigned long long * b, unsigned parity) {
    unsigned done;
    asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
                 : "=r"(done) : "r"(smem_u32(b)), "r"(parity) : "memory");
    return done != 0;
}

// Bounded wait on one phase of an mbarrier; false (and *err set) on timeout.
__device__ __forceinline__ bool mbar_wait(unsigned long long * b, unsigned parity, long long timeout_ns, int * err) {
    unsigned long long t0 = 0;
    for (unsigned it = 0;; ++it) {
        if (mbar_test(b, parity)) return true;
        if (*reinterpret_cast<volatile int *>(err) != 0) return false;
        if ((it & 255u) == 0u) {
            unsigned long long now;
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
            if (it == 0) t0 = now;
            else if ((long long) (now - t0) > timeout_ns) { atomicExch(err, 1); return false; }
        }
    }
}

__device__ __forceinline__ void mbar_arrive(unsigned long long * b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(smem_u32(b)) : "memory");
}

// K-major operand tile of `rows` x 128 bytes (64 f16 or 128 int8) in the 128-byte swizzle layout:
// 8-row atoms of 1024 bytes, row r at byte r * 128, 16-byte chunk c stored at
// chunk c ^ (r & 7).
__device__ __forceinline__ unsigned long long umma_desc_sw128(unsigned saddr) {
    unsigned long long d = 0;
    d |= (unsigned long long) ((saddr >> 4) & 0x3FFFu);          // start address
    d |= (unsigned long long) 1u << 16;                           // leading byte offset (unused for SW128 K-major)
    d |= (unsigned long long) (1024u >> 4) << 32;                 // stride byte offset: next 8-row atom
    d |= (unsigned long long) 1u << 46;                           // descriptor version (tcgen05)
    d |= (unsigned long long) 2u << 61;                           // layout: 128-byte swizzle
    return d;
}

// kind::f16 instruction descriptor: f32 accumulator, f16 A and B, both K-major.
__host__ __device__ constexpr unsigned umma_idesc_f16(int m, int n) {
    return (1u << 4)                          // D format f32
         | (0u << 7) | (0u << 10)             // A, B format f16
         | ((unsigned) (n >> 3) << 17)        // N / 8
         | ((unsigned) (m >> 4) << 24);       // M / 16
}

__device__ __forceinline__ void umma_f16(unsigned tmem_d, unsigned long long adesc, unsigned long long bdesc,
                                         unsigned idesc, unsigned accumulate) {
    asm volatile("{ .reg .pred p; setp.ne.b32 p, %4, 0;\n"
                 "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }"
                 :: "r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate) : "memory");
}

// kind::i8 instruction descriptor: s32 accumulator, signed 8-bit A and B, both K-major.
__host__ __device__ constexpr unsigned umma_idesc_s8(int m, int n) {
    return (2u << 4)                          // D format s32
         | (1u << 7) | (1u << 10)             // A, B format signed 8-bit
         | ((unsigned) (n >> 3) << 17)        // N / 8
         | ((unsigned) (m >> 4) << 24);       // M / 16
}

// One kind::i8 MMA (K = 32 bytes of each operand row).
__device__ __forceinline__ void umma_i8(unsigned tmem_d, unsigned long long adesc, unsigned long long bdesc,
                                        unsigned idesc, unsigned accumulate) {
    asm volatile("{ .reg .pred p; setp.ne.b32 p, %4, 0;\n"
                 "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p; }"
                 :: "r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate) : "memory");
}

__device__ __forceinline__ void umma_commit(unsigned long long * b) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 :: "r"(smem_u32(b)) : "memory");
}

__device__ __forceinline__ void tma_load_2d(void * dst, const CUtensorMap * map, int x, int y, unsigned long long * bar) {
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
                 :: "r"(smem_u32(dst)), "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar)) : "memory");
}

}  // namespace
}  // namespace pk
