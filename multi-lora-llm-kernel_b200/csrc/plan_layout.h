// Layout of the BGMV workspace: the row-grouping plan, then the state the
// split kernels share across CTAs.
//
//   word 0..7   header (kHdr* below)
//   word 8..    perm[T_pad]         int32 row indices
//   then        items[T_pad]        int4 {slot, begin, count, 0}, 16-byte aligned
//   then (each region starting on a 256-byte boundary)
//   sync        kSyncWords words (claim counter, CTAs done, epoch, abort), then
//               s_cnt[kMaxProblems][T_pad] (shrink slices done per item) and
//               ready[kMaxProblems][T_pad] (epoch at which v is complete)
//   vfinal      fp32 [problems][T_pad][64]  v per plan position
//   parts       fp32 [kPartSlots][16][64]   partial v per (item, K slice)
// T_pad = T rounded up to a multiple of 4, so the item table is aligned.
// The plan kernels zero the sync region and set the epoch to 1.
#pragma once

#include <stddef.h>
#include <stdint.h>

#include <vector_types.h>

namespace persona {

constexpr int kHdrItems = 0;
constexpr int kHdrValid = 1;
constexpr int kHdrNull = 2;
constexpr int kHdrBad = 3;
constexpr int kHdrT = 4;
constexpr int kHdrS = 5;
constexpr int kHdrRowsPerItem = 6;
constexpr int kHdrMagic = 7;
constexpr int32_t kPlanMagic = 0x4e414c50;  // "PLAN"
constexpr int kRowsPerItem = 16;             // rows of one item (8 row pairs)

__host__ __device__ constexpr int64_t plan_tpad(int64_t T) { return (T + 3) & ~int64_t(3); }

__host__ __device__ constexpr size_t plan_bytes(int64_t T) {
  return static_cast<size_t>(32 + 20 * plan_tpad(T));
}

constexpr int kSyncWords = 16;
constexpr int kSyncQueue = 0;
constexpr int kSyncDone = 1;
constexpr int kSyncEpoch = 2;
constexpr int kSyncAbort = 3;  // a CTA of the launch gave up a wait: the last CTA clears the counters
constexpr int kPartSlots = 1024;
constexpr int kPartFloats = 16 * 64;
constexpr int kMaxProblems = 8;  // projections one split launch can carry

__host__ __device__ constexpr size_t align256(size_t n) { return (n + 255) & ~size_t(255); }

__host__ __device__ constexpr size_t sync_offset(int64_t T) { return align256(plan_bytes(T)); }
__host__ __device__ constexpr size_t vfinal_offset(int64_t T) {
  return align256(sync_offset(T) + 4 * (kSyncWords + 2 * static_cast<size_t>(kMaxProblems * plan_tpad(T))));
}
__host__ __device__ constexpr size_t parts_offset(int64_t T, int problems) {
  return align256(vfinal_offset(T) + static_cast<size_t>(problems) * static_cast<size_t>(plan_tpad(T)) * 64 * 4);
}
// Total BGMV workspace for T rows and `problems` projections per launch.
__host__ __device__ constexpr size_t bgmv_ws_bytes(int64_t T, int problems = 1) {
  return parts_offset(T, problems) + static_cast<size_t>(kPartSlots) * kPartFloats * 4;
}

struct WorkView {
  int32_t* sync;
  int32_t* s_cnt;
  int32_t* ready;
  float* vfinal;
  float* parts;
};

// s_cnt / ready of problem p start at p * T_pad; vfinal of problem p at
// p * T_pad * 64 floats.
__host__ __device__ inline WorkView work_view(int32_t* base, int64_t T, int problems = 1) {
  uint8_t* b = reinterpret_cast<uint8_t*>(base);
  WorkView w;
  w.sync = reinterpret_cast<int32_t*>(b + sync_offset(T));
  w.s_cnt = w.sync + kSyncWords;
  w.ready = w.s_cnt + kMaxProblems * plan_tpad(T);
  w.vfinal = reinterpret_cast<float*>(b + vfinal_offset(T));
  w.parts = reinterpret_cast<float*>(b + parts_offset(T, problems));
  return w;
}

struct PlanView {
  int32_t* hdr;
  int32_t* perm;
  int4* items;
};

__host__ __device__ inline PlanView plan_view(int32_t* base, int64_t T) {
  PlanView v;
  v.hdr = base;
  v.perm = base + 8;
  v.items = reinterpret_cast<int4*>(base + 8 + plan_tpad(T));
  return v;
}

}  // namespace persona
