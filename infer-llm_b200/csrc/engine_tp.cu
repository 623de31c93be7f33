// NCCL plumbing for the tensor-parallel Qwen3 engine.
#include <nccl.h>

#include <cstring>

#include "common.cuh"
#include "engine_tp.cuh"

struct b200_tp {
    ncclComm_t comm = nullptr;
    int rank = 0, world = 1;
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
    if (tp->comm) ncclCommDestroy(tp->comm);
    delete tp;
}

cudaError_t tp_allreduce(b200_tp *tp, float *buf, size_t count, cudaStream_t stream) {
    if (ncclAllReduce(buf, buf, count, ncclFloat32, ncclSum, tp->comm, stream) != ncclSuccess)
        return cudaErrorUnknown;
    return cudaSuccess;
}

cudaError_t tp_select_token(b200_tp *tp, const float *local_val, const int32_t *local_idx, float *pairs,
                            int32_t *token, int32_t *token_log, int32_t *log_pos, int32_t log_cap,
                            int32_t *n_past, int32_t n_past_add, cudaStream_t stream) {
    int32_t *p = reinterpret_cast<int32_t *>(pairs);
    int32_t *mine = p + 2 * tp->world;
    pack_kernel<<<1, 1, 0, stream>>>(local_val, local_idx, mine);
    if (ncclAllGather(mine, p, 2, ncclInt32, tp->comm, stream) != ncclSuccess) return cudaErrorUnknown;
    select_kernel<<<1, 1, 0, stream>>>(p, tp->world, token, token_log, log_pos, log_cap, n_past, n_past_add);
    return cudaGetLastError();
}
