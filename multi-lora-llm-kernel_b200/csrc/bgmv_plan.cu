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

// The same plan by a stable counting sort, for pools of at most
// kCountMaxKeys - 2 slots (keys: the slot, S for -1, S + 1 for a slot out of
// range).  One CTA of 512 threads; per chunk of CH rows (the chunking of
// bgmv_plan_kernel, so the two give the same plan):
//  * per-key row counts (one shared-memory atomic per distinct key of a
//    warp) and their exclusive scan:
//    the first perm position of every key;
//  * rounds of 512 rows, 32 consecutive rows per warp: a row's rank among
//    the earlier rows of its key is its rank among the equal keys of its warp
//    (__match_any_sync), plus the same key's rows in the earlier warps of the
//    round (a per-warp count table, scanned per key), plus those of the
//    earlier rounds;
//  * items: per key, its full items then its partial one, placed by two
//    scans over the keys (full items of all keys first, in key order).
// About ten block barriers per chunk, instead of the radix sort's passes.
constexpr int kCountThreads = 512;
constexpr int kCountWarps = kCountThreads / 32;
constexpr int kCountMaxKeys = 512;

template <int CH>
__global__ void __launch_bounds__(kCountThreads)
    bgmv_plan_count_kernel(const int32_t* __restrict__ slots, int T, int S, int rows_per_item,
                           int32_t* __restrict__ plan, int32_t* dev_err) {
  static_assert(CH % kCountThreads == 0, "rounds of whole warps");
  using Scan = cub::BlockScan<int, kCountThreads>;
  __shared__ typename Scan::TempStorage scan;
  __shared__ int cnt[kCountMaxKeys];    // rows per key in this chunk
  __shared__ int start[kCountMaxKeys];  // first perm position of the key in this chunk
  __shared__ int run[kCountMaxKeys];    // rows of the key placed by earlier rounds
  __shared__ int whist[kCountWarps][kCountMaxKeys];
  __shared__ int s_counts[4];  // valid, null, bad, items (running over chunks)
  __shared__ int s_full;       // full items of this chunk
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // The BGMV kernel after this one is launched as a programmatic dependent.
  asm volatile("griddepcontrol.launch_dependents;");
  PlanView pv = plan_view(plan, T);
  if (tid < 4) s_counts[tid] = 0;
  init_work_state(plan, T, tid, kCountThreads);
  const int nkeys = S + 2;
  const uint32_t lt_mask = (1u << lane) - 1u;

  for (int base = 0; base < T; base += CH) {
    const int len = min(CH, T - base);
    for (int k = tid; k < nkeys; k += kCountThreads) {
      cnt[k] = 0;
      run[k] = 0;
    }
    __syncthreads();
    int keys[CH / kCountThreads];
#pragma unroll
    for (int r = 0; r < CH / kCountThreads; ++r) {
      const int i = r * kCountThreads + tid;
      int key = -1;
      if (i < len) {
        const int sl = slots[base + i];
        key = sl >= 0 && sl < S ? sl : sl == -1 ? S : S + 1;
      }
      // one atomic per distinct key of the warp: a hot slot (a Zipf batch
      // puts a fifth of its rows on one adapter) would otherwise serialise
      // its rows on one shared-memory word
      const uint32_t act = __ballot_sync(0xffffffffu, key >= 0);
      if (key >= 0) {
        const uint32_t peers = __match_any_sync(act, key);
        if ((peers & lt_mask) == 0) atomicAdd(&cnt[key], __popc(peers));
      }
      keys[r] = key;
    }
    __syncthreads();
    {
      const int c = tid < nkeys ? cnt[tid] : 0;
      int off;
      Scan(scan).ExclusiveSum(c, off);
      if (tid < nkeys) start[tid] = off;
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < CH / kCountThreads; ++r) {
      if (r * kCountThreads >= len) break;
      for (int k = lane; k < nkeys; k += 32) whist[warp][k] = 0;
      __syncwarp();
      const int key = keys[r];
      const uint32_t act = __ballot_sync(0xffffffffu, key >= 0);
      int rank = 0;
      if (key >= 0) {
        const uint32_t peers = __match_any_sync(act, key);
        rank = __popc(peers & lt_mask);
        if (rank == 0) whist[warp][key] = __popc(peers);
      }
      __syncthreads();
      // per key: rows of the earlier warps of this round (exclusive), and the
      // running count over the rounds
      for (int k = tid; k < nkeys; k += kCountThreads) {
        int off = run[k];
#pragma unroll
        for (int w = 0; w < kCountWarps; ++w) {
          const int h = whist[w][k];
          whist[w][k] = off;
          off += h;
        }
        run[k] = off;
      }
      __syncthreads();
      if (key >= 0) pv.perm[base + start[key] + whist[warp][key] + rank] = base + r * kCountThreads + tid;
      __syncthreads();
    }
    // items of the valid keys: full ones first (key order), then partial ones
    int nf = 0, np = 0, c = 0;
    if (tid < S) {
      c = cnt[tid];
      nf = c / rows_per_item;
      np = (c % rows_per_item) != 0 ? 1 : 0;
    }
    int off_f, off_p, tot_f, tot_p;
    Scan(scan).ExclusiveSum(nf, off_f, tot_f);
    __syncthreads();
    Scan(scan).ExclusiveSum(np, off_p, tot_p);
    const int item_base = s_counts[3];
    if (tid < S && c > 0) {
      const int p0 = base + start[tid];
      for (int f = 0; f < nf; ++f)
        pv.items[item_base + off_f + f] = make_int4(tid, p0 + f * rows_per_item, rows_per_item, 0);
      if (np) pv.items[item_base + tot_f + off_p] = make_int4(tid, p0 + nf * rows_per_item, c - nf * rows_per_item, 0);
    }
    if (tid == 0) {
      s_full = tot_f;
      s_counts[0] += start[S];                 // valid rows: every key below S
      s_counts[1] += cnt[S];
      s_counts[2] += cnt[S + 1];
      s_counts[3] = item_base + tot_f + tot_p;
    }
    __syncthreads();
  }
  (void)s_full;
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
  if (S + 2 <= kCountMaxKeys) {
    // chunks as in bgmv_plan_kernel below
    if (T <= 512)
      bgmv_plan_count_kernel<512><<<1, kCountThreads, 0, stream>>>(slots, T, S, rows_per_item, plan, dev_err);
    else if (T <= 1024)
      bgmv_plan_count_kernel<1024><<<1, kCountThreads, 0, stream>>>(slots, T, S, rows_per_item, plan, dev_err);
    else
      bgmv_plan_count_kernel<2048><<<1, kCountThreads, 0, stream>>>(slots, T, S, rows_per_item, plan, dev_err);
    return cudaGetLastError();
  }
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
