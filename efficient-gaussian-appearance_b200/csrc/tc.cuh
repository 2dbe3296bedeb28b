// Thin wrappers over the sm_100a tensor-core instructions (tcgen05) used by the neural appearance MLP:
// shared-memory matrix descriptors, the kind::f16 MMA with fp32 accumulation in tensor memory (TMEM),
// completion tracking through an mbarrier, TMEM allocation and TMEM -> register loads.
//
// Operand layouts are the no-swizzle canonical layouts of 16-bit elements: a "core matrix" is 8 rows of 16 bytes
// (8 elements) stored contiguously (128 bytes).
//   K-major (rows r, reduction index k):  byte(r, k) = (r / 8) * SBO + (k / 8) * LBO + (r % 8) * 16 + (k % 8) * 2
//   MN-major (index m along M or N, k):   byte(m, k) = (m / 8) * SBO + (k / 8) * LBO + (k % 8) * 16 + (m % 8) * 2
// so one buffer written K-major with LBO = 128 and SBO = 16 * K is also the MN-major view of its transpose with
// SBO' = 128 and LBO' = 16 * K: weights serve the forward (B K-major) and the data gradient (B MN-major), and
// activations serve the forward (A K-major) and the weight gradient (A / B MN-major, reduction over rows).
#pragma once

#include <cstdint>

namespace fgs {
namespace tc {

__device__ inline uint32_t smem_addr(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

// byte offset of element (r, k) in a K-major buffer with K columns (LBO = 128, SBO = 16 * K)
__host__ __device__ constexpr uint32_t kmajor_offset(uint32_t r, uint32_t k, uint32_t K) {
    return (r >> 3) * (16u * K) + (k >> 3) * 128u + (r & 7u) * 16u + (k & 7u) * 2u;
}

// shared-memory matrix descriptor (no swizzle): start address, leading and stride byte offsets, version 1
__device__ inline uint64_t desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    return static_cast<uint64_t>((addr >> 4) & 0x3FFFu) | (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16) |
           (static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}

// instruction descriptor of kind::f16: fp16 A and B, fp32 accumulator, operand majors (0 = K, 1 = MN), M x N
__host__ __device__ constexpr uint32_t idesc(uint32_t M, uint32_t N, uint32_t a_mn, uint32_t b_mn) {
    return (1u << 4) | (a_mn << 15) | (b_mn << 16) | ((N >> 3) << 17) | ((M >> 4) << 24);
}

// D[tmem] (+)= A[desc] * B[desc]; issued by a single thread
__device__ inline void mma(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t id, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(a), "l"(b), "r"(id), "r"(accumulate)
        : "memory");
}

// arrive once on the mbarrier when every MMA this thread issued before has completed
__device__ inline void commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ inline void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ inline bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred P1;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 P1, [%1], %2;\n\t"
        "selp.b32 %0, 1, 0, P1;\n\t}\n"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// bounded wait for the phase with the given parity to complete; false when the bound ran out
__device__ inline bool mbar_wait(uint64_t* bar, uint32_t parity) {
    for (uint32_t it = 0; it < (1u << 20); it++)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}

// bulk copy of `bytes` (a multiple of 16) from shared memory to global memory (both 16-byte aligned), in this thread's
// current bulk group; the wait forms make the group's shared-memory reads, or the whole copies, complete
__device__ inline void bulk_s2g(void* dst, uint32_t src, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(src), "r"(bytes) : "memory");
}
__device__ inline void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ inline void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ inline void bulk_wait() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// one arrival of this thread (release: its earlier shared-memory writes are visible to the threads that observe the
// completed phase)
__device__ inline void mbar_arrive(uint64_t* bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}\n" ::"r"(smem_addr(bar)) : "memory");
}

// true in exactly one lane of the (fully active) warp. Issue code placed under it with operands computed from
// warp-uniform values keeps the MMA operands in uniform registers.
__device__ inline bool elect_one() {
    uint32_t p;
    asm volatile(
        "{\n\t.reg .pred P;\n\t"
        "elect.sync _|P, 0xffffffff;\n\t"
        "selp.b32 %0, 1, 0, P;\n\t}\n"
        : "=r"(p));
    return p != 0;
}
// the warp index as a value the compiler knows to be warp-uniform
__device__ inline int warp_id_uniform() { return __shfl_sync(0xffffffffu, static_cast<int>(threadIdx.x >> 5), 0); }

// named barrier `id` (1..15) over `n` threads (whole warps)
__device__ inline void bar_sync(uint32_t id, uint32_t n) { asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory"); }
// the same barrier, returning whether any of the `n` threads passed true
__device__ inline bool bar_or(uint32_t id, uint32_t n, bool p) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred q, o;\n\t"
        "setp.ne.b32 q, %1, 0;\n\t"
        "bar.red.or.pred o, %2, %3, q;\n\t"
        "selp.b32 %0, 1, 0, o;\n\t}\n"
        : "=r"(r)
        : "r"(p ? 1u : 0u), "r"(id), "r"(n)
        : "memory");
    return r != 0;
}

// TMEM allocation (whole warp): the base address is written to *dst
__device__ inline void tmem_alloc(uint32_t* dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst)), "r"(ncols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ inline void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ inline void fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ inline void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// generic-proxy shared-memory writes become visible to the tensor core's operand reads
__device__ inline void fence_smem_to_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// 16 consecutive 32-bit TMEM columns of this warp's 32 lanes (lane = thread), completed before returning
__device__ inline void ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];\n\t"
        "tcgen05.wait::ld.sync.aligned;\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]),
          "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}

// 8 / 32 consecutive 32-bit TMEM columns of this warp's 32 lanes, completed before returning
__device__ inline void ld8(uint32_t taddr, float (&v)[8]) {
    uint32_t r[8];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];\n\t"
        "tcgen05.wait::ld.sync.aligned;\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 8; i++) v[i] = __uint_as_float(r[i]);
}
__device__ inline void ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, "
        "%21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n\t"
        "tcgen05.wait::ld.sync.aligned;\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]),
          "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]),
          "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
}

// 64 consecutive 32-bit TMEM columns of this warp's 32 lanes, completed before returning
__device__ inline void ld64(uint32_t taddr, float (&v)[64]) {
    uint32_t r[64];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x64.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, %17, %18, %19, %20, "
        "%21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, "
        "%48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63}, [%64];\n\t"
        "tcgen05.wait::ld.sync.aligned;\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]),
          "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]),
          "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
          "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]),
          "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]), "=r"(r[50]),
          "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]),
          "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 64; i++) v[i] = __uint_as_float(r[i]);
}

// a descriptor whose start address is `bytes` further (the start field holds the address / 16 in its low 14 bits)
__device__ inline uint64_t desc_advance(uint64_t d, uint32_t bytes) { return d + (bytes >> 4); }

// TMEM address of (lane, column)
__device__ inline uint32_t taddr(uint32_t base, uint32_t lane, uint32_t col) { return base + (lane << 16) + col; }

}  // namespace tc
}  // namespace fgs
