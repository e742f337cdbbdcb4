// Layout of the BGMV row-grouping plan in the caller's workspace.
//
//   word 0..7   header (kHdr* below)
//   word 8..    perm[T_pad]         int32 row indices
//   then        items[T_pad]        int4 {slot, begin, count, 0}, 16-byte aligned
// T_pad = T rounded up to a multiple of 4, so the item table is aligned.
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

__host__ __device__ inline int64_t plan_tpad(int64_t T) { return (T + 3) & ~int64_t(3); }

__host__ __device__ inline size_t plan_bytes(int64_t T) {
  const int64_t tp = plan_tpad(T);
  return static_cast<size_t>(32 + 4 * tp + 16 * tp);
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
