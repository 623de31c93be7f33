// 5th-generation tensor-core (tcgen05) building blocks shared by the sm_100a
// kernels: shared-memory matrix descriptors, kind::tf32 MMAs with the A operand in
// shared or tensor memory, commits, tensor-memory loads / stores, and bounded
// mbarrier waits.
#pragma once

#include "common.cuh"

namespace b200 {

// Shared-memory matrix descriptor for a K-major tile written by TMA with the
// 128-byte swizzle: rows of 128 bytes, 8-row groups 1024 bytes apart (stride byte
// offset), leading byte offset unused (1), descriptor version 1, layout SWIZZLE_128B
// (2 at bits 61-63). The tile base is 1024-byte aligned; stepping K by 8 TF32
// elements inside the 128-byte row advances the start address by 32 bytes.
B200_DEVICE uint64_t desc_k_sw128(uint32_t saddr) {
    uint64_t d = static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
    d |= static_cast<uint64_t>(1) << 16;
    d |= static_cast<uint64_t>(1024 >> 4) << 32;
    d |= static_cast<uint64_t>(1) << 46;
    d |= static_cast<uint64_t>(2) << 61;
    return d;
}

// Descriptor for an MN-major tile of 32-bit elements (TF32 B operand): each 128-byte
// row holds 32 consecutive M/N elements of one k, and the 32-byte chunks of a row are
// swizzled by the row index mod 4 (layout type 1, SWIZZLE_128B_BASE32B: the pattern
// TMA writes with CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B). Rows k .. k+3 form a 512-byte
// atom (stride byte offset 512); the next 32 M/N elements start `lbo` bytes further
// (leading byte offset). One MMA (K 8) reads two atoms per 32 M/N elements; stepping
// K by 8 advances the start address by 1024 bytes. The plain 128-byte swizzle
// (layout type 2) is not accepted for MN-major TF32: the product reads as zero.
B200_DEVICE uint64_t desc_mn_sw128_b32(uint32_t saddr, uint32_t lbo) {
    uint64_t d = static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
    d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
    d |= static_cast<uint64_t>(512 >> 4) << 32;
    d |= static_cast<uint64_t>(1) << 46;
    d |= static_cast<uint64_t>(1) << 61;
    return d;
}

// Instruction descriptor of kind::tf32: F32 accumulate (bits 4-5 = 1), A and B TF32
// (bits 7-9, 10-12 = 2), A / B MN-major flags at bits 15 / 16, N >> 3 at bits
// 17-22, M >> 4 at bits 24-28.
constexpr uint32_t idesc_tf32(int M, int N, bool a_mn, bool b_mn) {
    return (1u << 4) | (2u << 7) | (2u << 10) | (static_cast<uint32_t>(a_mn) << 15) |
           (static_cast<uint32_t>(b_mn) << 16) | (static_cast<uint32_t>(N >> 3) << 17) |
           (static_cast<uint32_t>(M >> 4) << 24);
}

B200_DEVICE void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
B200_DEVICE void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D (tensor memory) (+)= A (shared memory) . B (shared memory)
B200_DEVICE void tc_mma_tf32(uint32_t tmem, uint64_t da, uint64_t db, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}" ::"r"(tmem),
        "l"(da), "l"(db), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
        : "memory");
}

// D (tensor memory) (+)= A (tensor memory: lanes = rows, one 32-bit column per k) . B (shared memory)
B200_DEVICE void tc_mma_tf32_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t db, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n}" ::"r"(tmem_d),
        "r"(tmem_a), "l"(db), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
        : "memory");
}

// Arrives on `bar` once every tcgen05.mma this thread issued so far has completed.
B200_DEVICE void tc_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

// 32 lanes x 16 consecutive 32-bit columns of tensor memory (thread t: lane t).
B200_DEVICE void tc_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(r[j]);
}

// 32 lanes x 32 consecutive columns; the caller issues tcgen05.wait::ld (tc_wait_ld)
// before using the registers, so several loads can be in flight.
B200_DEVICE void tc_ld32_nowait(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
B200_DEVICE void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// Orders every later use of r after the preceding tc_wait_ld (the load's outputs
// carry no dependency on the wait; this empty volatile statement per register does).
B200_DEVICE void tc_reg_fence(uint32_t (&r)[32]) {
#pragma unroll
    for (int i = 0; i < 32; ++i) asm volatile("" : "+r"(r[i]));
}

// 32 lanes x 32 consecutive columns from registers; tc_wait_st() before the columns
// are handed to another thread or the tensor cores.
B200_DEVICE void tc_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
        "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]),
        "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
B200_DEVICE void tc_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Bounded mbarrier wait (hardware-suspended polls); false and B200_DEV_TIMEOUT
// after ~2 s, or at once if another CTA already reported an error.
B200_DEVICE bool wait_bounded(uint64_t *bar, uint32_t parity, int32_t *status) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
#pragma unroll 1
    for (uint32_t i = 0; i < B200_SPIN_LIMIT; ++i) {
        if (mbar_try_wait_sleep(bar, parity, 20000u)) return true;
        if ((i & 7) == 7) {
            if (status && *reinterpret_cast<volatile int32_t *>(status)) return false;
            if (global_ns() - t0 > 2000000000ull) break;
        }
    }
    set_status(status, B200_DEV_TIMEOUT);
    return false;
}

// As wait_bounded, with plain try_wait polls and no suspend-time hint: the thread
// resumes as soon as the phase completes (a hinted wait may let a thread sleep ~1 µs
// past the completion, which a per-tile handshake on the critical path cannot afford).
B200_DEVICE bool wait_poll(uint64_t *bar, uint32_t parity, int32_t *status) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
#pragma unroll 1
    for (uint32_t i = 0; i < B200_SPIN_LIMIT; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255) == 255) {
            if (status && *reinterpret_cast<volatile int32_t *>(status)) return false;
            if (global_ns() - t0 > 2000000000ull) break;
        }
    }
    set_status(status, B200_DEV_TIMEOUT);
    return false;
}

}  // namespace b200
