// tp.cuh — tensor-parallel pieces of the model: the NCCL entry points (loaded
// at run time) and the three small kernels around each collective.
#pragma once

#include <nccl.h>

#include <string>

#include "kernels.cuh"

namespace bitnet {

// The NCCL functions the model uses, resolved from the process's
// libnccl.so.2 (the copy torch already loaded, else the first one on the
// library path) or from the file named by BITNET_NCCL_LIBRARY.
struct NcclApi {
  decltype(&ncclGetUniqueId) get_unique_id;
  decltype(&ncclCommInitRank) comm_init_rank;
  decltype(&ncclCommInitRankConfig) comm_init_rank_config;
  decltype(&ncclCommGetAsyncError) comm_get_async_error;
  decltype(&ncclCommAbort) comm_abort;
  decltype(&ncclCommDestroy) comm_destroy;
  decltype(&ncclAllReduce) all_reduce;
  decltype(&ncclAllGather) all_gather;
  decltype(&ncclGetErrorString) error_string;
};
// nullptr (and *why set) when no NCCL library loads or a symbol is missing.
const NcclApi* nccl_api(std::string* why);

// out[t][j] = sqrelu(gu[t][j]) * gu[t][Fr + j] for t < T, j < Fr: the gate of
// sqrelu_gate (activation.rs) on one rank's gate/up slice, rows [T][2*Fr]
// in, [T][Fr] out. Fr % 4 == 0.
void launch_tp_gate_rows(const float* gu, int T, int Fr, float* out, cudaStream_t st);

// src [G][T][C] (what an all-gather of [T][C] per rank returns) ->
// dst [T][G*C] with dst[t][g*C + c] = src[g][t][c]. C % 4 == 0.
void launch_tp_unchunk(const float* src, int G, int T, int C, float* dst, cudaStream_t st);

// The matmul epilogue on all-reduced int32 accumulators acc [M][N]:
// out[m][n] = acc * ((ws * amax[m]) / 127), stored or added to out (row
// stride ldo), the same f32 operations as the fused epilogue.
void launch_acc_epilogue(const int32_t* acc, int M, int N, float ws, const float* amax, Epi epi, float* out, int ldo,
                         cudaStream_t st);

// Vocabulary-parallel greedy argmax: each row's largest logit of this rank's
// slice [M][V] (row stride ld) as (value bits, offset + index) in pairs[m];
// ties to the larger index, as Iterator::max_by (inference/src/lib.rs:263-271).
void launch_argmax_pairs(const float* logits, int ld, int M, int V, uint32_t offset, uint2* pairs, cudaStream_t st);
// out[m] = index of the best of the G ranks' pairs all[g][m] (larger value,
// ties to the larger index).
void launch_argmax_combine(const uint2* all, int G, int M, uint32_t* out, cudaStream_t st);

}  // namespace bitnet
