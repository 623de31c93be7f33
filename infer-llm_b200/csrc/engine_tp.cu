// Tensor-parallel communication for the Qwen3 engine: NCCL for the plumbing and
// the prefill all-reduces, and -- on the decode path -- an all-reduce kernel of its
// own over NVLink peer memory.
//
// Peer exchange. At init every rank allocates a receive buffer of tagged 64-bit
// words, [2 parities][world][slot] (tag << 32 | float bits), and the ranks swap
// CUDA IPC handles of those buffers over NCCL, so each rank holds device pointers
// into every peer's buffer. One all-reduce call then is one kernel per rank:
//   1. every thread takes its elements of this rank's partial and stores them as
//      tagged words into slot [parity][this rank] of every rank's buffer (plain
//      64-bit stores over NVLink, system scope);
//   2. it polls its own buffer until slot [parity][r] carries this call's tag for
//      every rank r, and sums the world values in rank order 0..world-1 -- the
//      same order on every rank, so every rank gets bit-identical sums and the
//      replicated activations stay identical.
// Calls are numbered from per-rank ticket counters (every CTA of every launch
// takes one; call = ticket / grid), the same on every rank because all ranks
// launch the same sequence. The tag is the call number (mod 2^32 - 1, + 1, never
// 0); two parities suffice because no rank can start call k + 2 before every
// rank has read call k (finishing call k + 1 needs every rank's k + 1 partial,
// written only after that rank finished call k). Every wait gives up after 2 s or
// as soon as the status word is set, and records B200_DEV_TIMEOUT.
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <cstring>
#include <thread>
#include <vector>

#include "common.cuh"
#include "engine_tp.cuh"

struct b200_tp {
    ncclComm_t comm = nullptr;
    int rank = 0, world = 1;
    // peer exchange (null when a peer is not reachable by peer access: NCCL then)
    unsigned long long *rbuf = nullptr;      // this rank's receive words [2][world][slot]
    unsigned long long **peers = nullptr;    // device table: every rank's rbuf (own included)
    unsigned long long *tickets = nullptr;   // [2]: all-reduce, token selection
    std::vector<void *> opened;              // peer buffers opened through IPC
    int64_t slot = 0;                        // words per (parity, rank)
};

namespace {

__global__ void select_kernel(const int32_t *pairs, int world, int32_t *token, int32_t *token_log, int32_t *log_pos,
                              int32_t log_cap, int32_t *n_past, int32_t add) {
    float best = -INFINITY;
    int32_t id = -1;
    bool bad = false;
    for (int r = 0; r < world; ++r) {  // rank r owns vocab rows [r*V/W, (r+1)*V/W)
        const float v = __int_as_float(pairs[2 * r]);
        const int32_t i = pairs[2 * r + 1];
        if (i < 0) bad = true;
        if (v > best) {
            best = v;
            id = i;
        }
    }
    if (bad) id = -1;
    *token = id;
    if (token_log) {
        const int32_t p = *log_pos;
        token_log[p % log_cap] = id;
        *log_pos = p + 1;
    }
    if (n_past) *n_past += add;
}

__global__ void pack_kernel(const float *val, const int32_t *idx, int32_t *out) {
    out[0] = __float_as_int(*val);
    out[1] = *idx;
}

}  // namespace

int tp_unique_id(unsigned char out_id[128]) {
    ncclUniqueId id;
    if (ncclGetUniqueId(&id) != ncclSuccess) return B200_ERR_CUDA;
    std::memcpy(out_id, id.internal, 128);
    return B200_OK;
}

int tp_create(b200_tp **out, const unsigned char id_bytes[128], int rank, int world) {
    ncclUniqueId id;
    std::memcpy(id.internal, id_bytes, 128);
    auto *tp = new b200_tp();
    tp->rank = rank;
    tp->world = world;
    if (ncclCommInitRank(&tp->comm, world, id, rank) != ncclSuccess) {
        delete tp;
        return B200_ERR_CUDA;
    }
    *out = tp;
    return B200_OK;
}

void tp_destroy(b200_tp *tp) {
    if (!tp) return;
    for (void *p : tp->opened) cudaIpcCloseMemHandle(p);
    if (tp->peers) cudaFree(tp->peers);
    if (tp->tickets) cudaFree(tp->tickets);
    if (tp->rbuf) cudaFree(tp->rbuf);
    if (tp->comm) ncclCommDestroy(tp->comm);
    delete tp;
}

int tp_p2p_init(b200_tp *tp, int64_t slot_words, cudaStream_t stream) {
    if (!tp || tp->world < 2 || slot_words <= 0) return B200_ERR_INVALID_ARGUMENT;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return B200_ERR_CUDA;
    const size_t bytes = static_cast<size_t>(2) * tp->world * slot_words * 8;
    cudaError_t e = cudaMalloc(&tp->rbuf, bytes);
    if (e == cudaSuccess) e = cudaMemset(tp->rbuf, 0, bytes);  // tag 0 never matches a call
    if (e == cudaSuccess) e = cudaMalloc(&tp->tickets, 16);
    if (e == cudaSuccess) e = cudaMemset(tp->tickets, 0, 16);
    if (e == cudaSuccess) e = cudaMalloc(&tp->peers, sizeof(void *) * tp->world);
    // every rank's IPC handle and device, gathered over NCCL
    struct Info {
        cudaIpcMemHandle_t h;
        int dev, pad[15];
    };
    static_assert(sizeof(Info) % 8 == 0, "gathered as 8-byte words");
    Info mine{};
    mine.dev = dev;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&mine.h, tp->rbuf);
    Info *d_all = nullptr;
    if (e == cudaSuccess) e = cudaMalloc(&d_all, sizeof(Info) * (tp->world + 1));
    std::vector<Info> all(tp->world);
    if (e == cudaSuccess) e = cudaMemcpyAsync(d_all + tp->world, &mine, sizeof mine, cudaMemcpyHostToDevice, stream);
    if (e == cudaSuccess &&
        ncclAllGather(d_all + tp->world, d_all, sizeof(Info) / 8, ncclUint64, tp->comm, stream) != ncclSuccess)
        e = cudaErrorUnknown;
    if (e == cudaSuccess) e = cudaMemcpyAsync(all.data(), d_all, sizeof(Info) * tp->world, cudaMemcpyDeviceToHost, stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    if (d_all) cudaFree(d_all);
    // peer access to every rank's buffer; any rank it cannot reach -> the NCCL path
    std::vector<unsigned long long *> ptrs(tp->world, nullptr);
    bool ok = e == cudaSuccess;
    for (int r = 0; ok && r < tp->world; ++r) {
        if (r == tp->rank) {
            ptrs[r] = tp->rbuf;
            continue;
        }
        int can = 0;
        if (all[r].dev != dev && (cudaDeviceCanAccessPeer(&can, dev, all[r].dev) != cudaSuccess || !can)) {
            ok = false;
            break;
        }
        void *p = nullptr;
        if (cudaIpcOpenMemHandle(&p, all[r].h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            ok = false;
            break;
        }
        tp->opened.push_back(p);
        ptrs[r] = static_cast<unsigned long long *>(p);
    }
    if (ok) ok = cudaMemcpy(tp->peers, ptrs.data(), sizeof(void *) * tp->world, cudaMemcpyHostToDevice) == cudaSuccess;
    if (!ok) {
        cudaGetLastError();
        for (void *p : tp->opened) cudaIpcCloseMemHandle(p);
        tp->opened.clear();
        if (tp->peers) cudaFree(tp->peers);
        if (tp->tickets) cudaFree(tp->tickets);
        if (tp->rbuf) cudaFree(tp->rbuf);
        tp->peers = nullptr;
        tp->tickets = nullptr;
        tp->rbuf = nullptr;
        return e == cudaSuccess ? B200_ERR_NOT_SUPPORTED : B200_ERR_CUDA;
    }
    tp->slot = slot_words;
    return B200_OK;
}

bool tp_p2p_ready(const b200_tp *tp) { return tp && tp->rbuf; }

int tp_sync(b200_tp *tp, cudaStream_t stream, int64_t timeout_ms) {
    // Bounded host wait for the rank's stream: NCCL's collectives wait for every rank
    // without a limit of their own, so a rank that stopped would hold this one in
    // cudaStreamSynchronize for good. Poll the stream and NCCL's asynchronous error;
    // on an NCCL error or after timeout_ms, abort the communicator (its kernels
    // return) and report the failure. The engine's tensor parallelism is unusable
    // afterwards (create it again).
    if (!tp->comm) return B200_ERR_CUDA;
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        const cudaError_t q = cudaStreamQuery(stream);
        if (q == cudaSuccess) return B200_OK;
        if (q != cudaErrorNotReady) return B200_ERR_CUDA;
        ncclResult_t ae = ncclSuccess;
        const bool nccl_failed = ncclCommGetAsyncError(tp->comm, &ae) != ncclSuccess ||
                                 (ae != ncclSuccess && ae != ncclInProgress);
        const bool late = std::chrono::steady_clock::now() - t0 > std::chrono::milliseconds(timeout_ms);
        if (nccl_failed || late) {
            ncclCommAbort(tp->comm);
            tp->comm = nullptr;
            cudaStreamSynchronize(stream);  // the aborted collectives return
            cudaGetLastError();
            return nccl_failed ? B200_ERR_CUDA : B200_ERR_TIMEOUT;
        }
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

namespace {

constexpr int kArThreads = 256;
constexpr uint64_t kArWaitNs = 2000000000ull;

__device__ __forceinline__ void st_sys(unsigned long long *p, unsigned long long v) {
    asm volatile("st.relaxed.sys.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_sys(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// This launch's call number from the ticket counter (thread 0), shared by the CTA.
__device__ __forceinline__ unsigned long long take_call(unsigned long long *ticket) {
    __shared__ unsigned long long s_call;
    if (threadIdx.x == 0) s_call = atomicAdd(ticket, 1ull) / gridDim.x;
    __syncthreads();
    return s_call;
}

__device__ __forceinline__ uint32_t call_tag(unsigned long long call) {
    return static_cast<uint32_t>(call % 0xFFFFFFFFull) + 1u;
}

// Polls word `w` until it carries `tag`; false (status set) after kArWaitNs or once
// another kernel reported an error.
__device__ bool wait_tag(const unsigned long long *w, uint32_t tag, unsigned long long *out, int32_t *status) {
    unsigned long long v = ld_sys(w);
    if (static_cast<uint32_t>(v >> 32) == tag) {
        *out = v;
        return true;
    }
    const uint64_t t0 = b200::global_ns();
#pragma unroll 1
    for (uint32_t i = 0; i < B200_SPIN_LIMIT; ++i) {
        v = ld_sys(w);
        if (static_cast<uint32_t>(v >> 32) == tag) {
            *out = v;
            return true;
        }
        if ((i & 63) == 63) {
            if (status && *reinterpret_cast<volatile int32_t *>(status)) return false;
            if (b200::global_ns() - t0 > kArWaitNs) break;
        }
    }
    b200::set_status(status, B200_DEV_TIMEOUT);
    return false;
}

// x[0..n) := sum over ranks of every rank's x (see the file comment).
__global__ void __launch_bounds__(kArThreads) ar_kernel(float *x, int64_t n, unsigned long long *const *peers,
                                                        unsigned long long *rbuf, unsigned long long *ticket,
                                                        int64_t slot, int rank, int world, int32_t *status) {
    const unsigned long long call = take_call(ticket);
    b200::grid_launch_dependents();
    b200::grid_wait();  // x is the previous kernel's output
    const uint32_t tag = call_tag(call);
    const int64_t par = static_cast<int64_t>(call & 1);
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    const int64_t i0 = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    for (int64_t i = i0; i < n; i += stride) {
        const unsigned long long w = (static_cast<unsigned long long>(tag) << 32) | __float_as_uint(x[i]);
        for (int r = 0; r < world; ++r) st_sys(peers[r] + (par * world + rank) * slot + i, w);
    }
    for (int64_t i = i0; i < n; i += stride) {
        float acc = 0.f;
        bool ok = true;
        for (int r = 0; r < world && ok; ++r) {
            unsigned long long v = 0;
            ok = wait_tag(rbuf + (par * world + r) * slot + i, tag, &v, status);
            acc = r == 0 ? __uint_as_float(static_cast<uint32_t>(v)) : acc + __uint_as_float(static_cast<uint32_t>(v));
        }
        if (!ok) return;  // status recorded; the step reports it
        x[i] = acc;
    }
}

// The greedy token from every rank's (first maximum, index) pair, exchanged as two
// tagged words per rank; the first maximum in rank order (ranks own increasing
// vocabulary ranges) wins.
__global__ void sel_p2p_kernel(const float *local_val, const int32_t *local_idx, unsigned long long *const *peers,
                               unsigned long long *rbuf, unsigned long long *ticket, int64_t slot, int rank,
                               int world, int32_t *token, int32_t *token_log, int32_t *log_pos, int32_t log_cap,
                               int32_t *n_past, int32_t add, int32_t *status) {
    const unsigned long long call = take_call(ticket);
    b200::grid_wait();
    const uint32_t tag = call_tag(call);
    // the selection words live after the all-reduce region of each parity
    const int64_t base = static_cast<int64_t>(call & 1) * world * slot + slot - 2 * world;
    const int t = threadIdx.x;
    if (t < world) {  // thread t pushes this rank's pair to rank t
        const unsigned long long hi = static_cast<unsigned long long>(tag) << 32;
        st_sys(peers[t] + base + 2 * rank, hi | __float_as_uint(*local_val));
        st_sys(peers[t] + base + 2 * rank + 1, hi | static_cast<uint32_t>(*local_idx));
    }
    __syncthreads();
    if (t != 0) return;
    float best = -INFINITY;
    int32_t id = -1;
    bool bad = false;
    for (int r = 0; r < world; ++r) {
        unsigned long long v = 0, ix = 0;
        if (!wait_tag(rbuf + base + 2 * r, tag, &v, status) || !wait_tag(rbuf + base + 2 * r + 1, tag, &ix, status))
            return;
        const float fv = __uint_as_float(static_cast<uint32_t>(v));
        const int32_t fi = static_cast<int32_t>(static_cast<uint32_t>(ix));
        if (fi < 0) bad = true;
        if (fv > best) {
            best = fv;
            id = fi;
        }
    }
    if (bad) id = -1;
    *token = id;
    if (token_log) {
        const int32_t p = *log_pos;
        token_log[p % log_cap] = id;
        *log_pos = p + 1;
    }
    if (n_past) *n_past += add;
}

}  // namespace

cudaError_t tp_allreduce(b200_tp *tp, float *buf, size_t count, cudaStream_t stream, bool pdl, int32_t *status) {
    if (tp->rbuf && static_cast<int64_t>(count) <= tp->slot - 2 * tp->world) {
        const int grid = static_cast<int>(std::min<int64_t>(64, (static_cast<int64_t>(count) + kArThreads - 1) / kArThreads));
        return b200_launch(ar_kernel, dim3(grid), dim3(kArThreads), 0, stream, pdl, buf, static_cast<int64_t>(count),
                           static_cast<unsigned long long *const *>(tp->peers), tp->rbuf, tp->tickets, tp->slot,
                           tp->rank, tp->world, status);
    }
    if (!tp->comm || ncclAllReduce(buf, buf, count, ncclFloat32, ncclSum, tp->comm, stream) != ncclSuccess)
        return cudaErrorUnknown;
    return cudaSuccess;
}

cudaError_t tp_select_token(b200_tp *tp, const float *local_val, const int32_t *local_idx, float *pairs,
                            int32_t *token, int32_t *token_log, int32_t *log_pos, int32_t log_cap,
                            int32_t *n_past, int32_t n_past_add, cudaStream_t stream, bool pdl, int32_t *status) {
    if (tp->rbuf)
        return b200_launch(sel_p2p_kernel, dim3(1), dim3(32), 0, stream, pdl, local_val, local_idx,
                           static_cast<unsigned long long *const *>(tp->peers), tp->rbuf, tp->tickets + 1, tp->slot,
                           tp->rank, tp->world, token, token_log, log_pos, log_cap, n_past, n_past_add, status);
    int32_t *p = reinterpret_cast<int32_t *>(pairs);
    int32_t *mine = p + 2 * tp->world;
    pack_kernel<<<1, 1, 0, stream>>>(local_val, local_idx, mine);
    if (!tp->comm || ncclAllGather(mine, p, 2, ncclInt32, tp->comm, stream) != ncclSuccess) return cudaErrorUnknown;
    select_kernel<<<1, 1, 0, stream>>>(p, tp->world, token, token_log, log_pos, log_cap, n_past, n_past_add);
    return cudaGetLastError();
}
