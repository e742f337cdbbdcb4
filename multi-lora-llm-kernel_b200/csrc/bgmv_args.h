// Kernel arguments of the BGMV kernels, shared by the host entry points
// (capi.cu) and the kernels.
#pragma once

#include <stdint.h>

#include <cuda.h>
#include <cuda_runtime.h>

#include "plan_layout.h"

namespace persona {

enum BgmvMode : int { kModeShrink = 1, kModeExpand = 2, kModeFused = 3 };


cudaError_t launch_bgmv_plan(const int32_t* slots, int T, int S, int rows_per_item, int32_t* plan,
                             int32_t* dev_err, cudaStream_t stream);
cudaError_t launch_shrink_rowwise(int dtype, const void* x, int64_t ldx, const void* a_pool,
                                  int64_t a_slot_stride, int64_t a_row_stride,
                                  const int32_t* slots, float* v, int T, int K, int R, int S,
                                  int32_t* err, cudaStream_t st);
cudaError_t launch_sgmv_plan(const int32_t* indptr, const int32_t* seg_slots, int nseg, int T, int S,
                             int rows_per_item, int32_t* plan, int32_t* row_slots, int32_t* dev_err,
                             cudaStream_t stream, int32_t* item_state = nullptr, int item_state_stride = 0);
constexpr int kSgmvMaxCtas = 160;  // CTAs of a tensor-core SGMV launch (pieces are sized for it)
// Bytes of the pieces region of the SGMV workspace (two pieces of 128 x R
// fp32 per CTA, R <= 64).
constexpr size_t kSgmvPieceBytes = static_cast<size_t>(2) * kSgmvMaxCtas * 128 * 64 * 4;
int bgmv_stage_rows(int R);  // B rows one ring slot holds at rank R
// Split kernels (bgmv_split.cu): every item of every problem cut into K / N
// slices claimed by all CTAs; workspace = bgmv_ws_bytes(T, problems)
// (plan_layout.h).  Up to kMaxProblems projections that share the batch's
// slots, rank and pool size run in one launch.
struct SplitProblem {
  const void* x;  // [T, K] 16-bit, row stride ldx
  void* y;        // [T, N] 16-bit, row stride ldy
  int64_t ldx, ldy;
  int K, N;
  int n_box;  // rows of one B tile (128 for ranks >= 16)
  int pad;
};
struct SplitArgs {
  SplitProblem prob[kMaxProblems];
  const float* v_in;  // expand only (one problem): [T, R] fp32
  float* v_out;       // shrink only (one problem): [T, R] fp32
  const int32_t* slots;
  int32_t* ws;  // plan + shared state
  int32_t* err;
  int num_problems, T, S, units_per_cta;
};
struct SplitMaps {
  CUtensorMap a[kMaxProblems];  // A pools, box {64, R, 1}
  CUtensorMap b[kMaxProblems];  // B pools, box {R, n_box, 1}
};
cudaError_t launch_bgmv_split(int mode, int dtype, int R, const SplitMaps& maps, const SplitArgs& a,
                              cudaStream_t st);

// Segmented tensor-core kernels (sgmv_tcgen05.cu).
// One projection of a decode-sized fused launch (bgmv_small.cu).
struct SmallProblem {
  const void* x;
  const void* a;
  const void* b;
  void* y;
  int64_t ldx, a_slot_stride, a_row_stride, b_slot_stride, ldy;
  int K, N;
  int slices;   // column slices per row (set by the launcher)
  int x_bytes;  // shared-memory bytes of one x row (set by the launcher)
  float* delta;      // non-null: write B[s] (A[s] x) here (fp32, 0 for rows
  int64_t ld_delta;  // without adapter) instead of adding it into y
};

struct SmallArgs {
  SmallProblem prob[kMaxProblems];
  int unit_base[kMaxProblems];  // first CTA of each problem (set by the launcher)
  const int32_t* slots;
  int32_t* err;
  int num_problems;
  int S;
};

cudaError_t launch_bgmv_small(int dtype, int R, SmallArgs& a, int T, cudaStream_t st);

constexpr int kMaxTpPeers = 7;  // other ranks a tensor-parallel launch writes to
// Width of one tensor-core SGMV fill: the shrink's K chunk and the expand's
// output tile (MMA N); x, y and A move as 64-element boxes side by side.
constexpr int kSgmvTcTileN = 128;
struct SgmvTcArgs {
  const int32_t* plan;  // segment plan, 128-row items, identity perm
  const float* v_in;    // expand only: [T, R]
  float* v_out;         // shrink only: [T, R]
  uint16_t* y;          // [T, N_total] row stride ldy (plain stores of short items)
  int64_t ldy;
  int32_t* err;
  int T, K, N;  // N: output columns this launch computes, from column n0 of y and B
  int n0;
  float* vfin;        // fused: [T, R] the items' v (workspace)
  float* pieces;      // [2 * CTAs][128][R] partial v of items cut between CTAs (workspace)
  int32_t* item_cnt;  // [items] pieces counted (zeroed by the plan kernel)
  int32_t* item_ready;  // [items] 1 once the item's v is complete (zeroed by the plan kernel)
  int num_peers;                   // tensor parallel: other ranks' y (same layout as y)
  uint16_t* peers[kMaxTpPeers];    // that receive every finished tile
};
cudaError_t launch_sgmv_tc(int mode, int dtype, int R, const CUtensorMap& tx, const CUtensorMap& ta,
                           const CUtensorMap& tb, const CUtensorMap& ty, const SgmvTcArgs& a, int max_items,
                           cudaStream_t st);
cudaError_t launch_gemv_fp16(const void* x, const void* W, void* y, int K, int N, cudaStream_t st);

// persona_bgmv_fused (capi.cu); plan_small = false: no plan on the
// decode-sized path, whose kernel reads none.
int fused_impl(const void* x, int64_t ldx, const void* a_pool, int64_t a_slot_stride, int64_t a_row_stride,
               const void* b_pool, int64_t b_slot_stride, const int32_t* slots, void* y, int64_t ldy, int64_t T,
               int64_t K, int64_t N, int64_t R, int64_t S, int dtype, void* workspace, size_t workspace_bytes,
               int flags, int32_t* dev_err, cudaStream_t stream, bool plan_small);

}  // namespace persona
