// Building blocks of the kernels on the 5th-generation tensor cores (sm_100a):
// shared-memory operand descriptors, the instruction descriptor, TMEM loads
// and bounded mbarrier waits.  Used by the prefill GEMM (prefill.cu) and the
// Heavy Medium prompt's window attention (heavy_prefill.cuh).
#pragma once

#include <cstdint>

namespace mr {
namespace tc {

constexpr unsigned long long kWaitNs = 2000000000ull;  // a wait gives up after 2 s and reports it

__device__ __forceinline__ uint64_t now() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ uint32_t saddr(const void *p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }
__device__ __forceinline__ bool try_wait(uint64_t *bar, int parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(saddr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// bounded wait; false (and *err set) when it gives up or another wait already did
__device__ inline bool wait(uint64_t *bar, int parity, int *err) {
    if (try_wait(bar, parity)) return true;
    const uint64_t start = now();
    for (unsigned spin = 0;; ++spin) {
        if (try_wait(bar, parity)) return true;
        if ((spin & 255u) == 255u) {
            if (*reinterpret_cast<volatile int *>(err)) return false;
            if (now() - start > kWaitNs) {
                atomicExch(err, 1);
                return false;
            }
        }
    }
}
// K-major operand tile in shared memory, 128-byte swizzle: rows of 128 bytes,
// 8-row groups 1024 bytes apart (stride byte offset), descriptor version 1
// (sm100); the start address steps 32 bytes per K16 step inside the swizzle atom.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr) {
    return static_cast<uint64_t>((addr >> 4) & 0x3FFFu) | (static_cast<uint64_t>(1) << 16) |
           (static_cast<uint64_t>(1024 >> 4) << 32) | (static_cast<uint64_t>(1) << 46) | (static_cast<uint64_t>(2) << 61);
}
// kind::f16 instruction descriptor: D F32, A and B BF16, both K-major, M x N
__host__ __device__ constexpr uint32_t idesc(int M, int N) {
    return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(N >> 3) << 17) |
           (static_cast<uint32_t>(M >> 4) << 24);
}
// Byte offset of element (row r, k) of a K-major tile of 64-element (128-byte)
// rows in the 128-byte swizzle: 16-byte chunk k / 8 of row r sits at chunk
// (k / 8) ^ (r % 8); 8-row groups are 1024 bytes apart.
__host__ __device__ __forceinline__ uint32_t sw128_offset(int r, int k) {
    return static_cast<uint32_t>((r >> 3) * 1024 + (r & 7) * 128 + ((((k >> 3) ^ (r & 7)) & 7) << 4) + (k & 7) * 2);
}

// 32 consecutive TMEM columns of this thread's lane (32x32b shape), waited for.
__device__ __forceinline__ void tmem_ld32(uint32_t addr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
          "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
          "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
          "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(addr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// D (+)= A B^T for one K16 step, issued by one thread.
__device__ __forceinline__ void mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc_v, bool accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc_v), "r"(accumulate ? 1u : 0u)
        : "memory");
}
// The mbarrier completes once every MMA this thread issued before has finished.
__device__ __forceinline__ void commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(saddr(bar))
                 : "memory");
}

}  // namespace tc
}  // namespace mr
