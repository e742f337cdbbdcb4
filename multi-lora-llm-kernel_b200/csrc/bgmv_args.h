// Kernel arguments of the clustered BGMV kernel, shared by the host entry
// points (capi.cu) and the kernel (bgmv_cluster.cu).
#pragma once

#include <stdint.h>

#include <cuda.h>
#include <cuda_runtime.h>

namespace persona {

enum BgmvMode : int { kModeShrink = 1, kModeExpand = 2, kModeFused = 3 };

struct BgmvArgs {
  const void* x;       // [T, K] 16-bit, row stride ldx
  int64_t ldx;
  const float* v_in;   // expand: [T, R] fp32
  float* v_out;        // shrink: [T, R] fp32
  void* y;             // [T, N] 16-bit, row stride ldy
  int64_t ldy;
  const int32_t* slots;
  const int32_t* plan;
  int32_t* err;
  int T, K, N, S;
  int units_per_cta;  // split kernels: target work units per CTA (0 = default)
  int k_per_cta;       // K slice of one cluster CTA, multiple of 64
  int n_per_cta;       // N slice of one cluster CTA, multiple of n_box
  int n_box;           // rows of one B tile, multiple of 8, <= 256
};

cudaError_t launch_bgmv_plan(const int32_t* slots, int T, int S, int rows_per_item, int32_t* plan,
                             int32_t* dev_err, cudaStream_t stream);
cudaError_t launch_bgmv_cluster(int mode, int dtype, int R, const CUtensorMap& tmA,
                                const CUtensorMap& tmB, const BgmvArgs& a, int cluster_size,
                                int max_clusters, cudaStream_t st);
cudaError_t launch_shrink_rowwise(int dtype, const void* x, int64_t ldx, const void* a_pool,
                                  int64_t a_slot_stride, int64_t a_row_stride,
                                  const int32_t* slots, float* v, int T, int K, int R, int S,
                                  int32_t* err, cudaStream_t st);
cudaError_t launch_sgmv_plan(const int32_t* indptr, const int32_t* seg_slots, int nseg, int T, int S,
                             int rows_per_item, int32_t* plan, int32_t* row_slots, int32_t* dev_err,
                             cudaStream_t stream);
int bgmv_stage_rows(int R);
// Split kernels (bgmv_split.cu): every item cut into K / N slices claimed by
// all CTAs; workspace = bgmv_ws_bytes(T) (plan_layout.h).
cudaError_t launch_bgmv_split(int mode, int dtype, int R, const CUtensorMap& tmA, const CUtensorMap& tmB,
                              const BgmvArgs& a, int max_ctas, cudaStream_t st);

// Segmented tensor-core kernels (sgmv_tcgen05.cu).
struct SgmvTcArgs {
  const int32_t* plan;  // segment plan, 128-row items, identity perm
  const float* v_in;    // expand only: [T, R]
  float* v_out;         // shrink only: [T, R]
  uint16_t* y;          // [T, N] row stride ldy (plain stores of short items)
  int64_t ldy;
  int32_t* err;
  int T, K, N;
};
cudaError_t launch_sgmv_tc(int mode, int dtype, int R, const CUtensorMap& tx, const CUtensorMap& ta,
                           const CUtensorMap& tb, const CUtensorMap& ty, const SgmvTcArgs& a, int max_items,
                           cudaStream_t st);
cudaError_t launch_gemv_fp16(const void* x, const void* W, void* y, int K, int N, cudaStream_t st);

}  // namespace persona
