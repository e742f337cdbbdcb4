// Host <-> device argument blocks and launchers of the NF4 kernels.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "nf4_table.h"

namespace persona {

// One base linear of a launch: y[M, N] = x[M, K] W^T, W in the tiled NF4
// format.  Its units are (tile of 128 output rows, split of the K chunks).
struct Nf4Problem {
  const uint8_t* w;
  const float* offset;  // device scalar written by the quantiser
  uint16_t* y;
  int64_t ldy;
  const float* addend;  // non-null: y = fp16(x W^T + addend), fp32 [M, ld_addend]
  int64_t ld_addend;
  int N, K;
  int splits;           // K splits per tile
  int chunks_per_split;
  int unit_base;        // first unit of this problem
  int counter_base;     // first tile counter of this problem
};

struct Nf4GemmArgs {
  Nf4Problem prob[kNf4MaxProblems];
  int num_problems;
  int units;
  int M;
  float* partials;   // [units][128][M_pad] fp32 (split problems only)
  int* counters;     // per tile, zero between launches (the finishing unit resets it)
  int32_t* err;
};

struct Nf4Maps {
  CUtensorMap x[kNf4MaxProblems];  // x[M, K] fp16, box {64, M_pad}, 128-byte swizzle
};

cudaError_t launch_nf4_absmax(const uint16_t* w, int64_t ldw, int N, int K, float* absmax, uint32_t* minmax,
                              cudaStream_t st);
cudaError_t launch_nf4_pack(const uint16_t* w, int64_t ldw, int N, int K, const float* absmax,
                            const uint32_t* minmax, uint8_t* packed, float* offset, cudaStream_t st);
cudaError_t launch_nf4_dequant(const uint8_t* packed, const float* offset, int N, int K, uint16_t* w, int64_t ldw,
                               cudaStream_t st);
cudaError_t launch_nf4_gemm(const Nf4Maps& maps, const Nf4GemmArgs& args, int m_pad, cudaStream_t st);
int nf4_sm_count();

}  // namespace persona
