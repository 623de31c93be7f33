// Tensor-parallel communication for the Qwen3 engine (one process per GPU, NCCL
// over NVLink / NVSwitch). Heads and FFN columns are split across ranks; the
// o_proj and ffn_down partial sums are all-reduced (the residual is added on rank
// 0 only, so the reduced value is residual + sum of partials); the LM head is
// vocab-sharded and the greedy token is chosen from the ranks' (max, index) pairs.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

struct b200_tp;

int tp_unique_id(unsigned char out_id[128]);
int tp_create(b200_tp **out, const unsigned char id[128], int rank, int world);
void tp_destroy(b200_tp *tp);
// Sets up the peer-memory exchange of the decode path: receive buffers of
// slot_words words per (parity, rank) (the largest all-reduce + 2 words per rank
// for the token selection), IPC handles swapped over NCCL. B200_ERR_NOT_SUPPORTED
// if some peer is not reachable by peer access (the NCCL path stays in use).
int tp_p2p_init(b200_tp *tp, int64_t slot_words, cudaStream_t stream);
bool tp_p2p_ready(const b200_tp *tp);
// Waits for `stream` at most timeout_ms, polling NCCL's asynchronous error; on an
// NCCL error or timeout aborts the communicator (B200_ERR_CUDA / B200_ERR_TIMEOUT).
int tp_sync(b200_tp *tp, cudaStream_t stream, int64_t timeout_ms);
// In-place sum over ranks of buf[0..count): the peer-memory kernel when set up and
// count fits its slots (decode), else ncclAllReduce (prefill). Bounded waits record
// B200_DEV_TIMEOUT in *status.
cudaError_t tp_allreduce(b200_tp *tp, float *buf, size_t count, cudaStream_t stream, bool pdl, int32_t *status);
// local_val/local_idx: this rank's first maximum (idx already offset into the full
// vocabulary, -1 for bad logits). Chooses the global first maximum in rank order,
// writes it to `token` (and token_log), advances n_past by n_past_add.
cudaError_t tp_select_token(b200_tp *tp, const float *local_val, const int32_t *local_idx, float *pairs,
                            int32_t *token, int32_t *token_log, int32_t *log_pos, int32_t log_cap,
                            int32_t *n_past, int32_t n_past_add, cudaStream_t stream, bool pdl, int32_t *status);
