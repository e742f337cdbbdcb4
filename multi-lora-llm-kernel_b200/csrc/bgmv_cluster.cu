// Clustered BGMV kernels for B200 (sm_100a): shrink, expand and fused
// shrink->expand over a row-grouping plan.
//
// Math (reference persona/ops.py:12-56, csrc/bgmv_shrink.cu:9-45,
// csrc/bgmv_expand.cu:9-30): for every row t with slot s = slots[t] >= 0
//   shrink  v[t, r] = sum_k A[s, r, k] * x[t, k]                (fp32)
//   expand  y[t, n] = round(y[t, n] + sum_r B[s, n, r] * v[t, r]) (fp32 sum)
// Rows with slot -1 get v = 0 and keep y bit-identical.
//
// Design (nothing here follows the reference's one-warp-per-(row, rank)
// layout):
// * Work unit = one plan item: one adapter slot and up to 16 rows that use
//   it.  The adapter's A and B are streamed from HBM once per item, not once
//   per row.
// * A thread-block cluster of CS (1 or 2) CTAs owns an item.  CTA q shrinks
//   the K-slice q (partial v over its slice) and expands the N-slice q.  The
//   partial v's are exchanged through distributed shared memory: each CTA
//   pushes its partial into the peer's receive buffer with st.async, whose
//   completion lands on the peer's mbarrier (no release fence), and both sum
//   the partials in rank order, so the rank-R intermediate never leaves the
//   chip in the fused kernel.
// * Each CTA is one producer warp and four consumer warps, and two CTAs share
//   an SM, so every SM runs two independent pipelines.  The producer feeds a
//   4-slot ring of 21 KB slots with everything the consumers read: an A
//   stage holds an A tile ({64 k x R rows} TMA boxes, 128-byte swizzle) plus
//   the item's x rows for the same k range; a B stage holds a B tile
//   ({R x n_box rows} TMA boxes) plus the item's y rows for the same columns
//   (1-D bulk copies, one lane per row); the expand-only kernel adds a v
//   stage.  The producer also prefetches the next item's data into L2.  Item
//   descriptors (slot, row count, row indices) reach the consumers through a
//   4-deep item ring.  Consumers never wait on a global load, release a slot
//   as soon as its data is in registers (relaxed arrive) and only then issue
//   their y stores, so no arrive waits on global stores.
// * The item's 16 rows are one warp-MMA tile (m16n8k16, fp32 accumulate):
//   x and v fragments are loaded once and reused over every rank / output
//   column tile of the warp, so the inner products cost neither CUDA-core
//   issue slots nor shared-memory bandwidth (a packed-FMA version was bound by
//   broadcast shared loads).  The expand multiplies B by v split into two
//   16-bit halves (v = hi + lo, power-of-two scaled against overflow), which
//   keeps the fp32 accuracy of v.
#include "bgmv_stages.cuh"

namespace persona {
constexpr int kMaxPeers = 1;                   // clusters of at most 2 CTAs

struct ItemDesc {
  int slot;
  int count;
  int pad[2];
  int rows[kRowsPerItem];
};

constexpr int kRingBytes = kSlots * kSlotBytes;
constexpr int kVBytes = kRowsPerItem * kMaxR * 4;  // fp32 [16][R]
constexpr int kVFloats = kRowsPerItem * kMaxR;
constexpr int kRecvBytes = 2 * kMaxPeers * kVBytes;  // fp32 [2][peers][16][R]
constexpr int kRedBytes = kRowsPerItem * kMaxR * 4;  // fp32 [warp][tiles][16][8] == [16][R] worth
constexpr int kItemBytes = kItemRing * static_cast<int>(sizeof(ItemDesc));
constexpr int kBarCount = 2 * kSlots + 2 * kItemRing + 2;
constexpr int kSmemLayoutBytes = kRingBytes + 2 * kVBytes + kRecvBytes + kRedBytes + kItemBytes + kBarCount * 8;
constexpr int kBgmvSmemBytes = kSmemLayoutBytes + 1024;  // slack to align the base
static_assert(kBgmvSmemBytes * kCtasPerSm <= 228 * 1024 - 2048, "two CTAs per SM");

int bgmv_stage_rows(int R) {
  switch (R) {
    case 8: return RankCfg<8>::kNB;
    case 16: return RankCfg<16>::kNB;
    case 32: return RankCfg<32>::kNB;
    default: return RankCfg<64>::kNB;
  }
}

int bgmv_max_cluster() { return kMaxPeers + 1; }

struct SmemPtrs {
  uint8_t* ring;
  float* pv;    // [16][R] this CTA's partial v of the current item
  float* vf;    // [16][R] full v of the current item
  float* recv;  // [2][peers][16][R] partial v pushed here by the cluster peer
  float* red;   // per-warp MMA tiles / maxima
  ItemDesc* items;
  uint64_t* full;      // [kSlots]
  uint64_t* empty;     // [kSlots]
  uint64_t* ifull;     // [kItemRing]
  uint64_t* iempty;    // [kItemRing]
  uint64_t* recv_bar;  // [2] completes when the peer's partial has landed
};

__device__ __forceinline__ SmemPtrs carve_smem(uint8_t* raw) {
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
  SmemPtrs p;
  p.ring = base;
  uint8_t* q = base + kRingBytes;
  p.pv = reinterpret_cast<float*>(q);
  p.vf = reinterpret_cast<float*>(q + kVBytes);
  p.recv = reinterpret_cast<float*>(q + 2 * kVBytes);
  p.red = reinterpret_cast<float*>(q + 2 * kVBytes + kRecvBytes);
  p.items = reinterpret_cast<ItemDesc*>(q + 2 * kVBytes + kRecvBytes + kRedBytes);
  uint64_t* bars = reinterpret_cast<uint64_t*>(q + 2 * kVBytes + kRecvBytes + kRedBytes + kItemBytes);
  p.full = bars;
  p.empty = bars + kSlots;
  p.ifull = bars + 2 * kSlots;
  p.iempty = bars + 2 * kSlots + kItemRing;
  p.recv_bar = bars + 2 * kSlots + 2 * kItemRing;
  return p;
}

// The j-th item of cluster `cid` out of `ncl`: rounds of ncl items, visited in
// serpentine order so that clusters that take a heavy (early) item in one
// round take a light one in the next.  The plan lists items heaviest first.
__device__ __forceinline__ int item_of(int cid, int ncl, int j) {
  return (j & 1) ? (j + 1) * ncl - 1 - cid : j * ncl + cid;
}

template <typename DT, int R, int MODE>
__global__ void __launch_bounds__(kBgmvThreads, kCtasPerSm)
    bgmv_cluster_kernel(const __grid_constant__ CUtensorMap tmA,
                        const __grid_constant__ CUtensorMap tmB, const BgmvArgs args) {
  using C = RankCfg<R>;
  constexpr bool kDoShrink = (MODE & kModeShrink) != 0;
  constexpr bool kDoExpand = (MODE & kModeExpand) != 0;
  extern __shared__ uint8_t smem_raw[];
  SmemPtrs sm = carve_smem(smem_raw);

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const uint32_t q = cluster_ctarank();
  const uint32_t CS = cluster_nctarank();
  const int cid = static_cast<int>(cluster_id_x());
  const int ncl = static_cast<int>(nclusters_x());

  if (tid == 0) {
    for (int s = 0; s < kSlots; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], kConsumerWarps);
    }
    for (int i = 0; i < kItemRing; ++i) {
      mbar_init(&sm.ifull[i], 1);
      mbar_init(&sm.iempty[i], kConsumerWarps);
    }
    for (int b = 0; b < 2; ++b) mbar_init(&sm.recv_bar[b], 1);
    fence_mbar_init_cluster();
  }
  cluster_sync_all();

  PlanView pv = plan_view(const_cast<int32_t*>(args.plan), args.T);
  const int n_items = pv.hdr[kHdrItems];
  const int kbeg = static_cast<int>(q) * args.k_per_cta;
  const int kend = min(args.K, kbeg + args.k_per_cta);
  const int nbeg = static_cast<int>(q) * args.n_per_cta;
  const int nend = min(args.N, nbeg + args.n_per_cta);
  const int stage_rows = (C::kNB / args.n_box) * args.n_box;

  if (warp == kConsumerWarps) {
    // ------------------------------------------------------- producer --
    const uint16_t* x = static_cast<const uint16_t*>(args.x);
    const uint16_t* yg = static_cast<const uint16_t*>(args.y);
    if (lane == 0) {
      if (kDoShrink) tma_prefetch_desc(&tmA);
      if (kDoExpand) tma_prefetch_desc(&tmB);
    }
    uint32_t g = 0;
    int item = item_of(cid, ncl, 0);
    int4 it = make_int4(0, 0, 0, 0);
    int row = 0;
    if (item < n_items) {
      it = pv.items[item];
      row = lane < it.z ? pv.perm[it.y + lane] : 0;
    }
    // Claim ring slot g % kSlots (waiting for the consumers to free it) and
    // post the byte count its copies will deliver.
    auto claim = [&](uint32_t bytes) -> int {
      const int s = static_cast<int>(g % kSlots);
      if (lane == 0) {
        if (g >= kSlots) mbar_wait(&sm.empty[s], ((g / kSlots) - 1) & 1, args.err);
        mbar_arrive_expect_tx(&sm.full[s], bytes);
      }
      __syncwarp();
      return s;
    };
    for (int j = 0; item < n_items; ++j) {
      const int slot = it.x, c = it.z;
      // publish the item descriptor
      const int iq = j % kItemRing;
      if (lane == 0 && j >= kItemRing) mbar_wait(&sm.iempty[iq], ((j / kItemRing) - 1) & 1, args.err);
      __syncwarp();
      if (lane < kRowsPerItem) sm.items[iq].rows[lane] = row;
      if (lane == 0) {
        sm.items[iq].slot = slot;
        sm.items[iq].count = c;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.ifull[iq]);
      // prefetch the next item's descriptor while this one streams
      const int nitem = item_of(cid, ncl, j + 1);
      int4 nit = make_int4(0, 0, 0, 0);
      if (nitem < n_items) nit = pv.items[nitem];

      if (kDoShrink) {
        for (int k0 = kbeg; k0 < kend; k0 += C::kKC) {
          const int valid = min(C::kKC, kend - k0);
          const int nbox = (valid + 63) / 64;
          const uint32_t xb = static_cast<uint32_t>(valid) * 2u;
          const int s = claim(static_cast<uint32_t>(nbox * C::kABoxBytes) + static_cast<uint32_t>(c) * xb);
          uint8_t* st = sm.ring + s * kSlotBytes;
          if (lane == 0)
            for (int b = 0; b < nbox; ++b) tma_load_3d(st + b * C::kABoxBytes, &tmA, &sm.full[s], k0 + 64 * b, 0, slot);
          if (lane < c)
            bulk_load(st + C::kXOff + lane * C::kXPitch, x + static_cast<int64_t>(row) * args.ldx + k0, xb,
                      &sm.full[s]);
          ++g;
        }
      }
      // The next item's rows (its descriptor has long arrived by now), then an
      // L2 prefetch of everything the next item will stream, so that its TMA
      // and bulk loads hit L2: this keeps far more bytes in flight per SM
      // than the shared-memory ring alone can hold.
      int nrow = 0;
      if (nitem < n_items) {
        nrow = lane < nit.z ? pv.perm[nit.y + lane] : 0;
        if (kDoShrink) {
          for (int k0 = kbeg + 64 * lane; k0 < kend; k0 += 64 * 32) tma_prefetch_3d(&tmA, k0, 0, nit.x);
          if (lane < nit.z && kend > kbeg)
            bulk_prefetch_l2(x + static_cast<int64_t>(nrow) * args.ldx + kbeg,
                             static_cast<uint32_t>(kend - kbeg) * 2u);
        }
        if (kDoExpand) {
          for (int n0 = nbeg + args.n_box * lane; n0 < nend; n0 += args.n_box * 32)
            tma_prefetch_3d(&tmB, 0, n0, nit.x);
          if (lane < nit.z && nend > nbeg)
            bulk_prefetch_l2(yg + static_cast<int64_t>(nrow) * args.ldy + nbeg,
                             static_cast<uint32_t>(nend - nbeg) * 2u);
        }
      }
      if (MODE == kModeExpand) {
        const int s = claim(static_cast<uint32_t>(c * R * 4));
        if (lane < c)
          bulk_load(sm.ring + s * kSlotBytes + lane * R * 4, args.v_in + static_cast<int64_t>(row) * R, R * 4,
                    &sm.full[s]);
        ++g;
      }
      if (kDoExpand) {
        for (int n0 = nbeg; n0 < nend; n0 += stage_rows) {
          const int rows_here = min(stage_rows, nend - n0);
          const int nbox = (rows_here + args.n_box - 1) / args.n_box;
          const uint32_t yb = static_cast<uint32_t>(rows_here) * 2u;
          const int s = claim(static_cast<uint32_t>(nbox * args.n_box * 2 * R) + static_cast<uint32_t>(c) * yb);
          uint8_t* st = sm.ring + s * kSlotBytes;
          if (lane == 0)
            for (int b = 0; b < nbox; ++b)
              tma_load_3d(st + b * args.n_box * 2 * R, &tmB, &sm.full[s], 0, n0 + b * args.n_box, slot);
          if (lane < c)
            bulk_load(st + C::kYOff + lane * C::kYStride, yg + static_cast<int64_t>(row) * args.ldy + n0, yb,
                      &sm.full[s]);
          ++g;
        }
      }
      it = nit;
      row = nrow;
      item = nitem;
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------ consumers --
    uint16_t* y = static_cast<uint16_t*>(args.y);
    if (MODE == kModeShrink) {
      // Rows without a (valid) adapter get v = 0; the items never touch them.
      const int gtid = (blockIdx.x * kConsumers) + tid;
      const int gstride = gridDim.x * kConsumers;
      for (int i = gtid; i < args.T * R; i += gstride) {
        const int s = args.slots[i / R];
        if (s < 0 || s >= args.S) args.v_out[i] = 0.f;
      }
    }
    uint32_t g = 0;
    int j = 0;
    for (int item = item_of(cid, ncl, 0); item < n_items; ++j, item = item_of(cid, ncl, j)) {
      const int iq = j % kItemRing;
      mbar_wait(&sm.ifull[iq], (j / kItemRing) & 1, args.err);
      const ItemDesc* itd = &sm.items[iq];
      const int c = itd->count;
      const int* rows = itd->rows;
      const int b = j & 1;
      const uint32_t recv_parity = (j >> 1) & 1;
      float* pvb = sm.pv;
      float* vfb = sm.vf;
      const int E = c * R;  // live entries of v (rows < c)
      // Bytes the peer will push into recv[b] for this item (its partial v).
      if (kDoShrink && tid == 0)
        mbar_arrive_expect_tx(&sm.recv_bar[b], (CS - 1) * static_cast<uint32_t>(E) * 4u);

      if (kDoShrink) {
        float d[C::kTPW][2][4];
#pragma unroll
        for (int t = 0; t < C::kTPW; ++t)
#pragma unroll
          for (int i = 0; i < 4; ++i) d[t][0][i] = d[t][1][i] = 0.f;
        for (int k0 = kbeg; k0 < kend; k0 += C::kKC, ++g) {
          const int s = static_cast<int>(g % kSlots);
          mbar_wait(&sm.full[s], (g / kSlots) & 1, args.err);
          uint8_t* st = sm.ring + s * kSlotBytes;
          const int valid = min(C::kKC, kend - k0);
          if (valid & 63) {
            // The last A tile reads zeros past K; zero the matching x columns so
            // that stale shared memory cannot inject NaN * 0.
            const int tail = ((valid + 63) & ~63) - valid;
            for (int e = tid; e < c * tail; e += kConsumers) {
              const int rr = e / tail, kk = valid + e % tail;
              reinterpret_cast<uint16_t*>(st + C::kXOff + rr * C::kXPitch)[kk] = 0;
            }
            named_sync(kNamedBarConsumers, kConsumers);
          }
          shrink_stage<DT, R>(st, ((valid + 63) / 64) * 4, warp, lane, d);
          __syncwarp();
          if (lane == 0) mbar_arrive_relaxed(&sm.empty[s]);
        }
        // This CTA's partial v: sum the two accumulators and the warps that
        // split k for each rank tile.
#pragma unroll
        for (int t = 0; t < C::kTPW; ++t) {
          float* rw = sm.red + (warp * C::kTPW + t) * (kRowsPerItem * 8);
          const int gg = lane >> 2, tt = lane & 3;
          rw[gg * 8 + 2 * tt] = d[t][0][0] + d[t][1][0];
          rw[gg * 8 + 2 * tt + 1] = d[t][0][1] + d[t][1][1];
          rw[(gg + 8) * 8 + 2 * tt] = d[t][0][2] + d[t][1][2];
          rw[(gg + 8) * 8 + 2 * tt + 1] = d[t][0][3] + d[t][1][3];
        }
        named_sync(kNamedBarConsumers, kConsumers);
        for (int e = tid; e < E; e += kConsumers) {
          const int rr = e / R, r = e - rr * R;
          const int T = r >> 3, col = r & 7;
          float sum = 0.f;
#pragma unroll
          for (int ks = 0; ks < C::kKS; ++ks)
            sum += sm.red[(((T / C::kTPW) * C::kKS + ks) * C::kTPW + (T % C::kTPW)) * (kRowsPerItem * 8) +
                          rr * 8 + col];
          pvb[e] = sum;
        }
        // Exchange through DSMEM: push this CTA's partial to the peer with
        // st.async (completing on the peer's recv barrier), then sum the
        // partials in rank order, so both CTAs hold the bit-identical full v.
        named_sync(kNamedBarConsumers, kConsumers);
        if (CS > 1) {
          for (int e4 = tid; e4 < (E >> 2); e4 += kConsumers) {
            const float4 val = *reinterpret_cast<const float4*>(pvb + 4 * e4);
            for (uint32_t r = 0; r < CS; ++r) {
              if (r == q) continue;
              const int pslot = q < r ? static_cast<int>(q) : static_cast<int>(q) - 1;  // my slot at peer r
              st_async_v4(sm.recv + (b * kMaxPeers + pslot) * kVFloats + 4 * e4, &sm.recv_bar[b], r, val);
            }
          }
        }
        mbar_wait<true>(&sm.recv_bar[b], recv_parity, args.err);
        const float* rb = sm.recv + b * kMaxPeers * kVFloats;
        const int share = (E + static_cast<int>(CS) - 1) / static_cast<int>(CS);
        for (int e = tid; e < E; e += kConsumers) {
          float sum = 0.f;
          for (uint32_t r = 0; r < CS; ++r) sum += r == q ? pvb[e] : rb[(r < q ? r : r - 1) * kVFloats + e];
          vfb[e] = sum;
          if (MODE == kModeShrink && e / share == static_cast<int>(q)) {
            const int rr = e / R, rk = e - rr * R;  // CTA q writes the entries of share q
            args.v_out[static_cast<int64_t>(rows[rr]) * R + rk] = sum;
          }
        }
        named_sync(kNamedBarConsumers, kConsumers);
      }

      if (kDoExpand) {
        if (MODE == kModeExpand) {
          const int s = static_cast<int>(g % kSlots);
          mbar_wait(&sm.full[s], (g / kSlots) & 1, args.err);
          const float* vs = reinterpret_cast<const float*>(sm.ring + s * kSlotBytes);
          for (int e = tid; e < E; e += kConsumers) vfb[e] = vs[e];
          __syncwarp();
          if (lane == 0) mbar_arrive_relaxed(&sm.empty[s]);
          ++g;
          named_sync(kNamedBarConsumers, kConsumers);
        }
        // Power-of-two scale that keeps the 16-bit v halves finite (f16 only).
        float scale_down = 1.f, scale_up = 1.f;
        if (std::is_same<DT, __half>::value) {
          float m = 0.f;
          for (int e = tid; e < E; e += kConsumers) m = fmaxf(m, fabsf(vfb[e]));
#pragma unroll
          for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
          if (lane == 0) sm.red[warp] = m;  // red[] is free: the shrink reduction is done
          named_sync(kNamedBarConsumers, kConsumers);
          m = sm.red[0];
#pragma unroll
          for (int w = 1; w < kConsumerWarps; ++w) m = fmaxf(m, sm.red[w]);
          const int ex = static_cast<int>((__float_as_uint(m) >> 23) & 0xff) - 127;
          const int e2 = ex > 14 ? ex - 14 : 0;
          if (e2 > 0) {
            scale_down = __uint_as_float(static_cast<uint32_t>(127 - e2) << 23);
            scale_up = __uint_as_float(static_cast<uint32_t>(127 + (e2 < 127 ? e2 : 127)) << 23);
          }
        }
        uint32_t vhi[C::kKSteps][4], vlo[C::kKSteps][4];
        v_fragments<DT, R>(vfb, scale_down, lane, vhi, vlo);
        for (int n0 = nbeg; n0 < nend; n0 += stage_rows, ++g) {
          const int s = static_cast<int>(g % kSlots);
          mbar_wait(&sm.full[s], (g / kSlots) & 1, args.err);
          const int rows_here = min(stage_rows, nend - n0);
          expand_stage<DT, R>(sm.ring + s * kSlotBytes, vhi, vlo, rows_here, args.n_box, n0, c, rows, y, args.ldy,
                              scale_up, warp, lane, &sm.empty[s]);
        }
        // the next item overwrites red[] / vf only after named syncs
        named_sync(kNamedBarConsumers, kConsumers);
      }
      // done with this item's descriptor
      __syncwarp();
      if (lane == 0) mbar_arrive_relaxed(&sm.iempty[iq]);
    }
  }
  // No CTA may leave while a peer can still reach its shared memory.
  __syncwarp();
  cluster_sync_all();
}

// ------------------------------------------------------------------ host --

template <typename DT, int R, int MODE>
static cudaError_t launch_one(const CUtensorMap& tmA, const CUtensorMap& tmB, const BgmvArgs& a,
                              int cluster_size, int max_clusters, cudaStream_t stream) {
  auto kern = bgmv_cluster_kernel<DT, R, MODE>;
  // Function attributes and occupancy are per device; cache both per device
  // and per cluster size (1, 2).
  constexpr int kMaxDev = 64;
  static bool configured[kMaxDev] = {};
  static int occ[kMaxDev][2] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDev) return cudaErrorInvalidDevice;
  if (cluster_size != 1 && cluster_size != 2) return cudaErrorInvalidValue;
  const int ci = cluster_size - 1;
  if (!configured[dev]) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kBgmvSmemBytes);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cluster_size;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(kBgmvThreads, 1, 1);
  cfg.dynamicSmemBytes = kBgmvSmemBytes;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // Persistent clusters: as many as can be resident, at most one per possible item.
  if (occ[dev][ci] == 0) {
    cfg.gridDim = dim3(cluster_size * 64, 1, 1);
    int n = 0;
    e = cudaOccupancyMaxActiveClusters(&n, kern, &cfg);
    if (e != cudaSuccess) return e;
    occ[dev][ci] = n > 0 ? n : 1;
  }
  int ncl = occ[dev][ci] < max_clusters ? occ[dev][ci] : max_clusters;
  if (ncl < 1) ncl = 1;
  cfg.gridDim = dim3(cluster_size * ncl, 1, 1);
  e = cudaLaunchKernelEx(&cfg, kern, tmA, tmB, a);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

template <typename DT, int MODE>
static cudaError_t dispatch_rank(int R, const CUtensorMap& tmA, const CUtensorMap& tmB,
                                 const BgmvArgs& a, int cs, int maxcl, cudaStream_t st) {
  switch (R) {
    case 8: return launch_one<DT, 8, MODE>(tmA, tmB, a, cs, maxcl, st);
    case 16: return launch_one<DT, 16, MODE>(tmA, tmB, a, cs, maxcl, st);
    case 32: return launch_one<DT, 32, MODE>(tmA, tmB, a, cs, maxcl, st);
    case 64: return launch_one<DT, 64, MODE>(tmA, tmB, a, cs, maxcl, st);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_bgmv_cluster(int mode, int dtype, int R, const CUtensorMap& tmA,
                                const CUtensorMap& tmB, const BgmvArgs& a, int cluster_size,
                                int max_clusters, cudaStream_t st) {
  const bool bf = dtype == PERSONA_DTYPE_BF16;
  switch (mode) {
    case kModeShrink:
      return bf ? dispatch_rank<__nv_bfloat16, kModeShrink>(R, tmA, tmB, a, cluster_size, max_clusters, st)
                : dispatch_rank<__half, kModeShrink>(R, tmA, tmB, a, cluster_size, max_clusters, st);
    case kModeExpand:
      return bf ? dispatch_rank<__nv_bfloat16, kModeExpand>(R, tmA, tmB, a, cluster_size, max_clusters, st)
                : dispatch_rank<__half, kModeExpand>(R, tmA, tmB, a, cluster_size, max_clusters, st);
    default:
      return bf ? dispatch_rank<__nv_bfloat16, kModeFused>(R, tmA, tmB, a, cluster_size, max_clusters, st)
                : dispatch_rank<__half, kModeFused>(R, tmA, tmB, a, cluster_size, max_clusters, st);
  }
}

}  // namespace persona
