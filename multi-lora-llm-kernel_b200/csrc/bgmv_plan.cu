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
#include <climits>

#include <cub/block/block_radix_sort.cuh>
#include <cub/block/block_scan.cuh>

#include "bgmv_args.h"
#include "common.cuh"
#include "plan_layout.h"

namespace persona {

// Zero the split kernels' shared state (claim counter, per-item counters and
// ready words) and start the epoch at 1; run by every thread of a plan kernel.
__device__ __forceinline__ void init_work_state(int32_t* ws, int T, int tid, int nthreads) {
  WorkView w = work_view(ws, T);
  const int words = kSyncWords + 2 * kMaxProblems * static_cast<int>(plan_tpad(T));
  for (int i = tid; i < words; i += nthreads) w.sync[i] = (i == kSyncEpoch) ? 1 : 0;
}


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
  // The BGMV kernel after this one is launched as a programmatic dependent:
  // let it become resident and set up now; it reads the plan only after
  // this kernel has completed (griddepcontrol.wait).
  asm volatile("griddepcontrol.launch_dependents;");
  PlanView pv = plan_view(plan, T);
  if (tid < 4) s_counts[tid] = 0;
  init_work_state(plan, T, tid, THREADS);

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
    // slot order, then the remainder items in slot order, so that the split
    // kernel's claim order starts with the items that carry the most rows.
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

namespace persona {

// Plan of a segmented batch (rows grouped contiguously by adapter, as in a
// prefill): segment i covers rows [indptr[i], indptr[i+1]) and uses slot
// seg_slots[i].  No sort is needed: perm is the identity, items are the
// segments cut into chunks of rows_per_item rows (full chunks first, then the
// remainders, each in segment order), and row_slots[t] receives every row's
// slot (-1 outside the segments) for the kernels that zero rows without an
// adapter.  A segment is used only if 0 <= lo <= hi <= T and no earlier
// indptr entry exceeds lo, so the used segments never overlap and the items
// never outnumber the rows; any other segment raises PERSONA_DEV_ERR_SEGMENT
// and is skipped.  A slot outside [-1, S) raises PERSONA_DEV_ERR_SLOT (its
// rows are skipped).
template <int THREADS>
__global__ void __launch_bounds__(THREADS)
    sgmv_plan_kernel(const int32_t* __restrict__ indptr, const int32_t* __restrict__ seg_slots, int nseg,
                     int T, int S, int rows_per_item, int32_t* __restrict__ plan, int32_t* __restrict__ row_slots,
                     int32_t* dev_err, int32_t* __restrict__ item_state, int item_state_stride) {
  // The tensor-core kernel after this one is launched as a programmatic
  // dependent: it may set up while this kernel runs.
  asm volatile("griddepcontrol.launch_dependents;");
  // row_slots == nullptr: items and header only (the tensor-core kernels
  // read nothing else); otherwise also the per-row slots, the identity
  // permutation and the split kernels' shared state.
  const bool rows = row_slots != nullptr;
  using ScanI = cub::BlockScan<int, THREADS>;
  __shared__ typename ScanI::TempStorage scan;
  __shared__ int s_base[2];  // running full / partial item counts
  __shared__ int s_total_full;
  __shared__ int s_err;
  __shared__ int s_carry;    // max indptr entry of the previous chunks
  __shared__ int s_lo[THREADS], s_hi[THREADS], s_slot[THREADS];
  const int tid = threadIdx.x;
  PlanView pv = plan_view(plan, T);
  if (rows) {
    init_work_state(plan, T, tid, THREADS);
    for (int t = tid; t < T; t += THREADS) {
      row_slots[t] = -1;
      pv.perm[t] = t;
    }
  }
  if (tid == 0) {
    s_base[0] = s_base[1] = 0;
    s_total_full = 0;
    s_err = 0;
  }
  __syncthreads();
  // pass 0 counts the full items of all segments; pass 1 writes the items
  // and the row slots
  for (int pass = 0; pass < 2; ++pass) {
    if (tid == 0) s_carry = 0;
    __syncthreads();
    for (int base = 0; base < nseg; base += THREADS) {
      const int i = base + tid;
      int lo = 0, hi = 0, slot = -1;
      if (i < nseg) {
        lo = indptr[i];
        hi = indptr[i + 1];
        slot = seg_slots[i];
      }
      int run_max;
      ScanI(scan).InclusiveScan(i < nseg ? lo : INT_MIN, run_max, cub::Max());
      __syncthreads();
      run_max = max(run_max, s_carry);
      if (i < nseg) {
        if (lo < 0 || hi < lo || hi > T || run_max > lo) {
          if (pass == 0) atomicOr(&s_err, PERSONA_DEV_ERR_SEGMENT);
          lo = hi = 0;
          slot = -1;
        } else if (slot < -1 || slot >= S) {
          if (pass == 0) atomicOr(&s_err, PERSONA_DEV_ERR_SLOT);
          slot = -1;
        }
      }
      const int len = slot >= 0 ? hi - lo : 0;
      const int nfull = len / rows_per_item;
      const int npart = (len % rows_per_item) ? 1 : 0;
      int off_full, off_part, agg_full, agg_part;
      ScanI(scan).ExclusiveSum(nfull, off_full, agg_full);
      __syncthreads();
      ScanI(scan).ExclusiveSum(npart, off_part, agg_part);
      __syncthreads();
      if (pass == 1) {
        for (int f = 0; f < nfull; ++f)
          pv.items[s_base[0] + off_full + f] = make_int4(slot, lo + f * rows_per_item, rows_per_item, 0);
        if (npart)
          pv.items[s_total_full + s_base[1] + off_part] =
              make_int4(slot, lo + nfull * rows_per_item, len - nfull * rows_per_item, 0);
        s_lo[tid] = lo;
        s_hi[tid] = slot >= 0 ? hi : lo;
        s_slot[tid] = slot;
      }
      __syncthreads();
      if (pass == 1 && rows) {  // row slots of this chunk's segments, one warp per segment
        const int n = min(THREADS, nseg - base);
        for (int q = tid >> 5; q < n; q += THREADS / 32)
          for (int t = s_lo[q] + (tid & 31); t < s_hi[q]; t += 32) row_slots[t] = s_slot[q];
      }
      if (tid == THREADS - 1) s_carry = run_max;  // inclusive max up to the chunk's last entry
      if (tid == 0) {
        s_base[0] += agg_full;
        s_base[1] += agg_part;
      }
      __syncthreads();
    }
    if (pass == 0 && tid == 0) {
      s_total_full = s_base[0];
      s_base[0] = s_base[1] = 0;
    }
    __syncthreads();
  }
  // Per-item counter and ready word of the tensor-core kernel (two arrays
  // item_state_stride words apart), zero for every item of this plan.
  if (item_state != nullptr)
    for (int i = tid; i < s_total_full + s_base[1]; i += THREADS) {
      item_state[i] = 0;
      item_state[item_state_stride + i] = 0;
    }
  if (tid == 0) {
    pv.hdr[kHdrItems] = s_total_full + s_base[1];
    pv.hdr[kHdrValid] = 0;
    pv.hdr[kHdrNull] = 0;
    pv.hdr[kHdrBad] = 0;
    pv.hdr[kHdrT] = T;
    pv.hdr[kHdrS] = S;
    pv.hdr[kHdrRowsPerItem] = rows_per_item;
    pv.hdr[kHdrMagic] = kPlanMagic;
    if (s_err) raise_error(dev_err, s_err);
  }
}

cudaError_t launch_sgmv_plan(const int32_t* indptr, const int32_t* seg_slots, int nseg, int T, int S,
                             int rows_per_item, int32_t* plan, int32_t* row_slots, int32_t* dev_err,
                             cudaStream_t stream, int32_t* item_state, int item_state_stride) {
  sgmv_plan_kernel<512><<<1, 512, 0, stream>>>(indptr, seg_slots, nseg, T, S, rows_per_item, plan, row_slots,
                                               dev_err, item_state, item_state_stride);
  return cudaGetLastError();
}

}  // namespace persona
