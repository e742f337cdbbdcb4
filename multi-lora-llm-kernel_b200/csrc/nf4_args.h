// Host <-> device argument blocks and launchers of the NF4 kernels.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "nf4_table.h"

namespace persona {
// CTAs of the NF4 GEMM per SM, at most (the partial buffer is sized for it).
constexpr int kNf4MaxCtasPerSm = 2;

// One base linear of a launch: y[M, N] = x[M, K] W^T, W in the tiled NF4
// format.  Its chunks (tile of 128 output rows, 128-wide K chunk) follow
// those of the problems before it in one linear order, tile-major.
struct Nf4Problem {
  const uint8_t* w;
  const float* offset;  // device scalar written by the quantiser
  uint16_t* y;
  int64_t ldy;
  const float* addend;  // non-null: y = fp16(x W^T + addend), fp32 [M, ld_addend]
  int64_t ld_addend;
  int64_t chunk_base;  // first chunk of this problem in the launch's order
  int N, K;
  int counter_base;     // first tile counter of this problem
};

struct Nf4GemmArgs {
  Nf4Problem prob[kNf4MaxProblems];
  int64_t chunks;    // all problems' chunks
  int num_problems;
  int max_ctas;      // grid bound that the partial buffer is sized for
  int M;
  float* partials;   // [CTA][2][128][M_pad] fp32: a CTA's first and last tile pieces
  int* counters;     // per tile, zero between launches (the finishing piece resets it)
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
