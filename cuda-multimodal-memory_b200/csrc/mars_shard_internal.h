// mars_shard_internal.h -- what the sharded query (mars_shard_bfs.cu) uses
// of the row-shard communicator (mars_shard.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "mars_b200.h"

namespace mars {

struct ShardCommView {
    int32_t device = 0;
    int32_t rank = 0;
    int32_t world = 1;
    int32_t max_k = 0;
    void** bfs_state = nullptr;   // the sharded query's scratch, owned by the communicator
};

int shard_comm_view(mars_shard_comm* c, ShardCommView* v);

// B queries x K local results (global ids, scores; d_ids == NULL or
// neutral: no entries) -> one all-gather of packed keys -> the merged
// [B][K] lists and counts on every rank.
int shard_gather_merge(const ShardCommView& v, const int32_t* d_ids, const float* d_vals, int32_t B, int32_t K,
                       int32_t* d_ids_out, float* d_vals_out, int32_t* d_counts, bool neutral, cudaStream_t st);

// In-place all-reduce (max) of n floats / ints on st.
int shard_allreduce_max_f32(const ShardCommView& v, float* d, int32_t n, cudaStream_t st);
int shard_allreduce_max_i32(const ShardCommView& v, int32_t* d, int32_t n, cudaStream_t st);

}  // namespace mars

// Frees the sharded query's scratch (mars_shard_bfs.cu).
void shard_bfs_state_free(void* st);
