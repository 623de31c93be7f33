// Issue-rate probe of the tcgen05 kind::tf32 MMA (M 128, K 8), used by
// tests/test_gpu_tcgen05_rate.py: one CTA per SM issues `iters` MMAs back to back into
// one TMEM accumulator (operands fixed: A in shared or tensor memory, B K-major in
// shared memory), commits, and reports the cycles until the last one completed.
#include "tcgen05.cuh"
using namespace b200;

__global__ void mma_rate_kernel(long long *cycles, int n, int a_tmem, int iters) {
    extern __shared__ unsigned char sm[];
    __shared__ uint64_t bar;
    __shared__ uint32_t slot;
    const uint32_t base = (smem_addr(sm) + 1023u) & ~1023u;
    unsigned char *p = sm + (base - smem_addr(sm));
    for (int i = threadIdx.x; i < (16384 + 32768) / 4; i += blockDim.x) reinterpret_cast<float *>(p)[i] = 0.001f * (i & 255);
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_barrier_init();
    }
    if (threadIdx.x < 32) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&slot)), "r"(512u)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = slot;
    if (threadIdx.x == 0) {
        const uint32_t idesc = idesc_tf32(128, n, false, false);
        const uint64_t da = desc_k_sw128(base), db = desc_k_sw128(base + 16384);
        const long long t0 = clock64();
        for (int i = 0; i < iters; ++i) {
            const int kk = i & 3;
            if (a_tmem)  // A: TMEM columns 256.. (whatever they hold; only the rate matters)
                tc_mma_tf32_ts(tmem, tmem + 256 + 8 * kk, db + 2 * kk, idesc, 1u);
            else
                tc_mma_tf32(tmem, da + 2 * kk, db + 2 * kk, idesc, 1u);
        }
        tc_commit(smem_addr(&bar));
        wait_poll(&bar, 0, nullptr);
        cycles[blockIdx.x] = clock64() - t0;
    }
    tc_fence_before();
    __syncthreads();
    if (threadIdx.x < 32) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(512u) : "memory");
    }
}

extern "C" int mma_rate(long long *cycles, int n, int a_tmem, int iters, int blocks) {
    const int smem = 16384 + 32768 + 1024;
    if (cudaFuncSetAttribute(mma_rate_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return -1;
    mma_rate_kernel<<<blocks, 128, smem>>>(cycles, n, a_tmem, iters);
    return static_cast<int>(cudaDeviceSynchronize());
}
