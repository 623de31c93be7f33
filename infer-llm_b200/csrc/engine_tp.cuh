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
cudaError_t tp_allreduce(b200_tp *tp, float *buf, size_t count, cudaStream_t stream);
// local_val/local_idx: this rank's first maximum (idx already offset into the full
// vocabulary, -1 for bad logits). Chooses the global first maximum in rank order,
// writes it to `token` (and token_log), advances n_past by n_past_add.
cudaError_t tp_select_token(b200_tp *tp, const float *local_val, const int32_t *local_idx, float *pairs,
                            int32_t *token, int32_t *token_log, int32_t *log_pos, int32_t log_cap,
                            int32_t *n_past, int32_t n_past_add, cudaStream_t stream);
