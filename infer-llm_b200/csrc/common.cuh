// Shared device helpers for the sm_100a kernels: bulk-copy (TMA engine) staging
// with mbarriers, bounded waits, programmatic dependent launch, warp reductions.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>
#include <set>
#include <tuple>

#include "../../include/b200_infer.h"

#define B200_HOST_DEVICE __host__ __device__ __forceinline__
#define B200_DEVICE __device__ __forceinline__

// Upper bound on mbarrier / flag polling iterations before a wait is declared
// stuck. At ~20 ns per try_wait round trip this is several seconds: no correct
// run gets near it, and a stuck kernel still returns with B200_DEV_TIMEOUT.
#define B200_SPIN_LIMIT (1u << 28)

namespace b200 {

B200_HOST_DEVICE int64_t min64(int64_t a, int64_t b) { return a < b ? a : b; }
B200_HOST_DEVICE int64_t max64(int64_t a, int64_t b) { return a > b ? a : b; }

// ---------------------------------------------------------------------------
// Status word: the first non-zero code wins.
B200_DEVICE void set_status(int32_t *status, int32_t code) {
    if (status) atomicCAS(status, 0, code);
}

// ---------------------------------------------------------------------------
// Device-side step trace: a kernel given a trace slot (8 x u64, preset to
// {0, 0, 0, UINT64_MAX, 0...}) records the global timer at CTA 0's start [0],
// after CTA 0's dependency wait [1], the last CTA end [2], the first CTA start
// [3], CTA 0 after its prologue (inputs staged) [4] and after its main loop [5].
B200_DEVICE uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
struct TraceMark {
    unsigned long long *slot;
    B200_DEVICE explicit TraceMark(unsigned long long *s) : slot(s) {
        if (slot && threadIdx.x == 0) {
            const unsigned long long t = global_ns();
            if (blockIdx.x == 0 && blockIdx.y == 0) slot[0] = t;
            atomicMin(slot + 3, t);
        }
    }
    B200_DEVICE void waited() const {
        if (slot && threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0) slot[1] = global_ns();
    }
    B200_DEVICE void at(int k) const {
        if (slot && threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == 0) slot[k] = global_ns();
    }
    B200_DEVICE void done() const {
        if (slot && threadIdx.x == 0) atomicMax(slot + 2, static_cast<unsigned long long>(global_ns()));
    }
};

// ---------------------------------------------------------------------------
// Programmatic dependent launch (PDL). Every kernel launched with the
// programmatic-serialization attribute calls grid_wait() before it reads data
// produced by the previous kernel in the stream, and grid_launch_dependents()
// as early as possible so the next kernel's CTAs can be scheduled and start
// prefetching their (input-independent) weights.
B200_DEVICE void grid_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
B200_DEVICE void grid_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------------------
// mbarrier + cp.async.bulk (the 1-D form of the TMA engine).
B200_DEVICE uint32_t smem_addr(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// 16-byte shared-memory load at a 32-bit shared address (an explicit ld.shared:
// generic loads of shared data through pointers kept in structs cost a
// generic-to-shared resolution each).
B200_DEVICE float4 lds4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
    return v;
}

B200_DEVICE void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
                 : "memory");
}

// Makes mbarrier initialisation visible to the async proxy (bulk copies).
B200_DEVICE void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

B200_DEVICE void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

B200_DEVICE void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// `count` arrivals at once.
B200_DEVICE void mbar_arrive_n(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

B200_DEVICE bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n"
        " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// As mbar_try_wait, but the thread may sleep up to `sleep_ns` in hardware until the
// phase completes instead of returning at once: a waiting warp takes no issue slots
// from the warps that share its scheduler.
B200_DEVICE bool mbar_try_wait_sleep(uint64_t *bar, uint32_t parity, uint32_t sleep_ns) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n"
        " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
        " selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity), "r"(sleep_ns)
        : "memory");
    return ok != 0;
}

// Bounded wait for the phase with the given parity to complete. Returns false
// (after B200_SPIN_LIMIT polls) if it never does.
B200_DEVICE bool mbar_wait(uint64_t *bar, uint32_t parity) {
    for (uint32_t i = 0; i < B200_SPIN_LIMIT; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    return false;
}

// Global -> shared bulk copy completing on `bar` (bytes: multiple of 16, both
// addresses 16-byte aligned). L2 evict-first: weights are streamed once per step.
B200_DEVICE void bulk_g2s(void *smem_dst, const void *gmem_src, uint32_t bytes, uint64_t *bar,
                          uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1], %2, [%3], %4;" ::"r"(smem_addr(smem_dst)),
        "l"(gmem_src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}

// Nearest TF32 value of x (top 19 bits, ties away from zero). Kernels whose output
// only feeds a TF32 tensor-core product write it rounded: the tensor cores would
// truncate it, a bias toward zero that compounds over the layers.
B200_DEVICE float tf32_rn(float x) { return __uint_as_float((__float_as_uint(x) + 0x1000u) & 0xFFFFE000u); }

B200_DEVICE uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

B200_DEVICE uint64_t policy_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// TMA-engine bulk prefetch of [p, p + bytes) into L2 (p and bytes 16-byte multiples).
B200_DEVICE void prefetch_l2_bulk(const void *p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// This CTA's share of an L2 prefetch of a byte range split evenly over the grid
// (one bulk prefetch per CTA, issued by thread 0).
B200_DEVICE void prefetch_share_l2(const void *base, size_t bytes) {
    if (!base || bytes == 0 || threadIdx.x != 0) return;
    const size_t nblk = static_cast<size_t>(gridDim.x) * gridDim.y;
    const size_t b = static_cast<size_t>(blockIdx.y) * gridDim.x + blockIdx.x;
    const size_t chunk = ((bytes + nblk - 1) / nblk + 15) & ~size_t(15);
    const size_t off = b * chunk;
    if (off >= bytes) return;
    size_t len = bytes - off < chunk ? bytes - off : chunk;
    len &= ~size_t(15);
    const char *p = static_cast<const char *>(base) + off;
    while (len > 0) {  // the bulk-prefetch size operand is 32-bit
        const uint32_t n = len > (1u << 30) ? (1u << 30) : static_cast<uint32_t>(len);
        prefetch_l2_bulk(p, n);
        p += n;
        len -= n;
    }
}

// ---------------------------------------------------------------------------
// Thread-block clusters: hardware cluster barrier and distributed shared memory.
// Every thread of every CTA in the cluster must execute each cluster_sync().
B200_DEVICE void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Address of `p` (this CTA's shared memory) in the shared memory of cluster rank `rank`.
B200_DEVICE uint32_t dsmem_addr(const void *p, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr(p)), "r"(rank));
    return r;
}
B200_DEVICE float ld_dsmem(uint32_t addr) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
    return v;
}

// Named barrier over `threads` threads (a multiple of 32) with id 1..15.
B200_DEVICE void named_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ---------------------------------------------------------------------------
// Ampere-style 16-byte async copies (used where tiles are gathered row by row).
B200_DEVICE void cp_async16(void *smem_dst, const void *gmem_src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(smem_dst)),
                 "l"(gmem_src)
                 : "memory");
}
B200_DEVICE void cp_async16_zfill(void *smem_dst, const void *gmem_src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(smem_dst)),
                 "l"(gmem_src), "r"(valid ? 16 : 0)
                 : "memory");
}
B200_DEVICE void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
B200_DEVICE void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Streaming 128-bit load that does not allocate in L1.
B200_DEVICE float4 ld_stream4(const float4 *p) {
    float4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p));
    return v;
}

// ---------------------------------------------------------------------------
B200_DEVICE float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
B200_DEVICE double warp_sum(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
B200_DEVICE float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// RMSNorm scale with the reference's rounding (cpu_backend.cpp:369-376): squares
// are float products accumulated in double; scale = float(1 / sqrt(mean + eps)).
B200_DEVICE float rms_scale_from_sumsq(double sumsq, int64_t D, float eps) {
    return static_cast<float>(1.0 / sqrt(sumsq / static_cast<double>(D) + static_cast<double>(eps)));
}

}  // namespace b200

namespace b200 {
// Kernel function attributes (cudaFuncSetAttribute) belong to the current device:
// `set()` runs once per (device, kernel, attribute group) and is recorded only when
// it succeeded, so a second GPU driven from the same process configures its own.
template <typename Set>
inline cudaError_t once_per_device(const void *kernel, int what, Set set) {
    static std::mutex mu;
    static std::set<std::tuple<int, const void *, int>> done;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    const auto key = std::make_tuple(dev, kernel, what);
    std::lock_guard<std::mutex> lock(mu);
    if (done.count(key)) return cudaSuccess;
    e = set();
    if (e == cudaSuccess) done.insert(key);
    return e;
}
enum { ATTR_CARVEOUT = 0, ATTR_SMEM = 1 };
}  // namespace b200

// Host-side launch helper: launch with the PDL attribute on `stream`.
// Every kernel asks for the maximum shared-memory carveout, so consecutive kernels
// never need an SM reconfiguration (which would serialise programmatic launches).
template <typename Kernel, typename... Args>
static inline cudaError_t b200_launch(Kernel kernel, dim3 grid, dim3 block, size_t smem,
                                      cudaStream_t stream, bool pdl, Args... args) {
    cudaError_t e = b200::once_per_device(reinterpret_cast<const void *>(kernel), b200::ATTR_CARVEOUT, [&] {
        return cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                    cudaSharedmemCarveoutMaxShared);
    });
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, args...);
}
