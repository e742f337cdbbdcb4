// Row-grouping plan for the BGMV kernels (device side, one CTA, no host sync).
//
// The reference reads each row's slot on the host (`slots[t].item()`,
// csrc/bgmv_shrink.cu:106-109 and csrc/bgmv_expand.cu:113-116: 2*T device->
// host syncs per projection) and then lets every row re-read its adapter.
// Here one small kernel sorts the rows by slot instead, so that the main
// kernels stream each used adapter's A and B once for all of its rows, and
// flags out-of-range slots in the device error word.
//
// Output (the "plan", int32 words, see plan_layout.h):
//   header  n_items, n_valid, n_null, n_bad, T, S, rows_per_item, magic
//   perm    row indices; per chunk of kChunk rows: valid rows sorted by slot
//           (ties in row order), then rows with slot -1, then invalid rows
//   items   int4 {slot, begin (index into perm), count <= rows_per_item, 0};
//           per chunk, the full items (count == rows_per_item) in slot order,
//           then the partial ones in slot order
// Items never straddle a chunk; for T <= kChunk there is one chunk and the
// layout is exactly the oracle's `plan_ref`.
#include <cub/block/block_radix_sort.cuh>
#include <cub/block/block_scan.cuh>

#include "bgmv_args.h"
#include "common.cuh"
#include "plan_layout.h"

namespace persona {

template <int THREADS, int IPT>
__global__ void __launch_bounds__(THREADS)
    bgmv_plan_kernel(const int32_t* __restrict__ slots, int T, int S, int rows_per_item,
                     int32_t* __restrict__ plan, int32_t* dev_err) {
  constexpr int CH = THREADS * IPT;
  using Sort = cub::BlockRadixSort<uint32_t, THREADS, IPT, int32_t>;
  using ScanI = cub::BlockScan<int, THREADS>;
  __shared__ union {
    typename Sort::TempStorage sort;
    typename ScanI::TempStorage scan;
  } tmp;
  __shared__ uint32_t skey[CH];
  __shared__ int s_counts[4];  // valid, null, bad, items (running over chunks)

  const int tid = threadIdx.x;
  PlanView pv = plan_view(plan, T);
  if (tid < 4) s_counts[tid] = 0;

  const uint32_t key_null = static_cast<uint32_t>(S);
  const uint32_t key_bad = static_cast<uint32_t>(S) + 1u;
  const uint32_t key_pad = static_cast<uint32_t>(S) + 2u;
  const int end_bit = 32 - __clz(static_cast<int>(key_pad));
  __syncthreads();

  for (int base = 0; base < T; base += CH) {
    const int len = min(CH, T - base);
    uint32_t keys[IPT];
    int32_t vals[IPT];
    int nv = 0, nn = 0, nb = 0;
#pragma unroll
    for (int j = 0; j < IPT; ++j) {
      const int pos = tid * IPT + j;  // blocked arrangement keeps the sort stable in row order
      if (pos < len) {
        const int s = slots[base + pos];
        if (s >= 0 && s < S) {
          keys[j] = static_cast<uint32_t>(s);
          ++nv;
        } else if (s == -1) {
          keys[j] = key_null;
          ++nn;
        } else {
          keys[j] = key_bad;
          ++nb;
        }
        vals[j] = base + pos;
      } else {
        keys[j] = key_pad;
        vals[j] = -1;
      }
    }
    if (nv) atomicAdd(&s_counts[0], nv);
    if (nn) atomicAdd(&s_counts[1], nn);
    if (nb) atomicAdd(&s_counts[2], nb);

    Sort(tmp.sort).Sort(keys, vals, 0, end_bit);
    __syncthreads();
#pragma unroll
    for (int j = 0; j < IPT; ++j) {
      const int pos = tid * IPT + j;
      skey[pos] = keys[j];
      if (pos < len) pv.perm[base + pos] = vals[j];
    }
    __syncthreads();

    // Segment starts, then item starts every rows_per_item rows of a segment.
    int seg_start[IPT];
#pragma unroll
    for (int j = 0; j < IPT; ++j) {
      const int pos = tid * IPT + j;
      const bool start = pos == 0 || skey[pos] != skey[pos - 1];
      seg_start[j] = start ? pos : 0;
    }
    ScanI(tmp.scan).InclusiveScan(seg_start, seg_start, cub::Max());
    __syncthreads();
    // Items heaviest first: full items (rows_per_item rows) of every slot in
    // slot order, then the remainder items in slot order.  The BGMV kernels
    // deal items to clusters in serpentine rounds, so the heavy items are
    // spread over the clusters and start first.
    int full[IPT], part[IPT], cntv[IPT];
#pragma unroll
    for (int j = 0; j < IPT; ++j) {
      const int pos = tid * IPT + j;
      const uint32_t k = skey[pos];
      const bool start = k < static_cast<uint32_t>(S) && ((pos - seg_start[j]) % rows_per_item) == 0;
      int cnt = 0;
      if (start) {
        cnt = 1;
        while (cnt < rows_per_item && pos + cnt < CH && skey[pos + cnt] == k) ++cnt;
      }
      cntv[j] = cnt;
      full[j] = (start && cnt == rows_per_item) ? 1 : 0;
      part[j] = (start && cnt < rows_per_item) ? 1 : 0;
    }
    int idx_full[IPT], idx_part[IPT];
    int n_full = 0, n_part = 0;
    ScanI(tmp.scan).ExclusiveSum(full, idx_full, n_full);
    __syncthreads();
    ScanI(tmp.scan).ExclusiveSum(part, idx_part, n_part);
    const int chunk_items = n_full + n_part;
    const int item_base = s_counts[3];
#pragma unroll
    for (int j = 0; j < IPT; ++j) {
      if (!full[j] && !part[j]) continue;
      const int pos = tid * IPT + j;
      const int at = full[j] ? idx_full[j] : n_full + idx_part[j];
      pv.items[item_base + at] = make_int4(static_cast<int>(skey[pos]), base + pos, cntv[j], 0);
    }
    __syncthreads();
    if (tid == 0) s_counts[3] = item_base + chunk_items;
    __syncthreads();
  }

  if (tid == 0) {
    pv.hdr[kHdrItems] = s_counts[3];
    pv.hdr[kHdrValid] = s_counts[0];
    pv.hdr[kHdrNull] = s_counts[1];
    pv.hdr[kHdrBad] = s_counts[2];
    pv.hdr[kHdrT] = T;
    pv.hdr[kHdrS] = S;
    pv.hdr[kHdrRowsPerItem] = rows_per_item;
    pv.hdr[kHdrMagic] = kPlanMagic;
    if (s_counts[2] > 0) raise_error(dev_err, PERSONA_DEV_ERR_SLOT);
  }
}

cudaError_t launch_bgmv_plan(const int32_t* slots, int T, int S, int rows_per_item,
                             int32_t* plan, int32_t* dev_err, cudaStream_t stream) {
  if (T <= 256) {
    bgmv_plan_kernel<128, 2><<<1, 128, 0, stream>>>(slots, T, S, rows_per_item, plan, dev_err);
  } else if (T <= 512) {
    bgmv_plan_kernel<128, 4><<<1, 128, 0, stream>>>(slots, T, S, rows_per_item, plan, dev_err);
  } else if (T <= 1024) {
    bgmv_plan_kernel<256, 4><<<1, 256, 0, stream>>>(slots, T, S, rows_per_item, plan, dev_err);
  } else {
    bgmv_plan_kernel<256, 8><<<1, 256, 0, stream>>>(slots, T, S, rows_per_item, plan, dev_err);
  }
  return cudaGetLastError();
}

}  // namespace persona
