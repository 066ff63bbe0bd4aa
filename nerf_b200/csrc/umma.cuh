// umma.cuh -- 5th-generation tensor-core (tcgen05) building blocks for sm_100a:
// tensor-memory allocation, shared-memory matrix descriptors, the f16 MMA with
// an fp32 accumulator in tensor memory, completion through an mbarrier with a
// bounded wait, and tensor-memory loads.
//
// Operand layout used throughout: "K-major interleaved" without swizzle.  An
// R x K fp16 matrix (row r, column k; K a multiple of 16) is stored as 8 x 8
// core matrices of 128 contiguous bytes (8 rows of 16 bytes):
//   byte offset(r, k) = (r / 8) * (K * 16) + (k / 8) * 128 + (r % 8) * 16 + (k % 8) * 2.
// As a K-major operand (rows = M or N, columns = K) its descriptor has leading
// byte offset 128 (next 8 columns of K) and stride byte offset K * 16 (next 8
// rows); one MMA consumes 16 columns, so K-step s starts 256 * s bytes in.
// The same bytes read as an MN-major operand (rows = K, columns = M or N) have
// leading byte offset K * 16 (next 8 rows, now along K) and stride byte offset
// 128 (next 8 columns, now along M / N), and K-step s starts 16 rows in:
// s * 2 * (K * 16) bytes.
#pragma once
#include "common.cuh"

namespace nb {
namespace umma {

NB_DEV uint32_t interleaved_offset(uint32_t r, uint32_t k, uint32_t K) {
    return (r >> 3) * (K * 16u) + (k >> 3) * 128u + (r & 7u) * 16u + (k & 7u) * 2u;
}

// Shared-memory matrix descriptor, no swizzle (layout type 0), descriptor
// version 1 (sm_100), base offset 0.
NB_DEV uint64_t smem_desc(uint32_t smem_addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
    return static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu) | (static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16) |
           (static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}
// K-step s of an R x K K-major interleaved matrix at smem_addr.
NB_DEV uint64_t desc_k_major(uint32_t smem_addr, uint32_t K, uint32_t s) {
    return smem_desc(smem_addr + 256u * s, 128u, K * 16u);
}
// K-step s (rows 16s..16s+15) of an R x C interleaved matrix read MN-major:
// the MMA's K runs along the R rows, its M / N along the C columns.
NB_DEV uint64_t desc_mn_major(uint32_t smem_addr, uint32_t C, uint32_t s) {
    return smem_desc(smem_addr + 2u * s * (C * 16u), C * 16u, 128u);
}

// Instruction descriptor of kind::f16: fp16 A and B, fp32 D, M x N tile;
// a_mn / b_mn select MN-major operands.
__host__ __device__ constexpr uint32_t idesc_f16(uint32_t M, uint32_t N, uint32_t a_mn, uint32_t b_mn) {
    return (1u << 4) | (a_mn << 15) | (b_mn << 16) | ((N >> 3) << 17) | ((M >> 4) << 24);
}

// ---- tensor memory ----
// Allocation by one whole warp; the base address is written to *slot.
NB_DEV void tmem_alloc(uint32_t* slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(slot)), "r"(ncols)
                 : "memory");
}
NB_DEV void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory"); }
NB_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(taddr), "r"(ncols) : "memory");
}
NB_DEV void fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
NB_DEV void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }
// Generic-proxy shared-memory writes made visible to the tensor core's async proxy.
NB_DEV void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory"); }

// D (tensor memory) = A x B^T (+ D when accumulate != 0), issued by one thread.
NB_DEV void mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n"
        ".reg .pred p;\n"
        "setp.ne.b32 p, %4, 0;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n"
        "}\n" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// The mbarrier receives one arrival when every MMA issued so far by this
// thread has completed.
NB_DEV void commit(uint64_t* mbar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(smem_u32(mbar))
                 : "memory");
}

// ---- mbarrier ----
NB_DEV void mbar_init(uint64_t* mbar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(mbar)), "r"(count) : "memory");
}
NB_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory"); }
NB_DEV uint64_t globaltimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
    return t;
}
// Waits for the phase with the given parity to complete; gives up after
// limit_ns of wall time and returns false.
NB_DEV bool mbar_wait(uint64_t* mbar, uint32_t parity, uint64_t limit_ns) {
    const uint32_t a = smem_u32(mbar);
    const uint64_t t0 = globaltimer();
    for (;;) {
        uint32_t done;
        asm volatile(
            "{\n"
            ".reg .pred p;\n"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
            "selp.u32 %0, 1, 0, p;\n"
            "}\n"
            : "=r"(done)
            : "r"(a), "r"(parity)
            : "memory");
        if (done) return true;
        if (globaltimer() - t0 > limit_ns) return false;
    }
}

// ---- tensor memory -> registers ----
// 32 consecutive fp32 columns of this thread's lane (warp w reads lanes
// 32 (w % 4) .. +31; taddr carries that lane base).  The wait for the load is
// part of the same statement, so the registers are valid when it returns.
NB_DEV void tmem_ld32(uint32_t taddr, float v[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
        "tcgen05.wait::ld.sync.aligned;\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
// 16 columns, same contract.
NB_DEV void tmem_ld16(uint32_t taddr, float v[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
        "tcgen05.wait::ld.sync.aligned;\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

}  // namespace umma
}  // namespace nb
