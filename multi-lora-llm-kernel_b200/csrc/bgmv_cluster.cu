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
// * A thread-block cluster of CS CTAs owns an item.  CTA q shrinks the
//   K-slice q (partial v over its slice) and expands the N-slice q.  The
//   partial v's are reduced through distributed shared memory: each CTA sums
//   one share of the entries over the CS CTAs and broadcasts the sum back,
//   so the rank-R intermediate never leaves the chip in the fused kernel.
// * One producer warp streams A tiles ({64 k x R rows}, 128-byte swizzle)
//   and B tiles ({R x n_box rows}) with TMA into a 4-stage ring of 32 KB
//   stages; eight consumer warps compute with packed fp32x2 FMAs.  The
//   producer runs ahead across item boundaries, so HBM stays busy while the
//   consumers reduce.
// * x rows of an item are gathered by the consumers into a 512-wide fp32
//   window laid out as row pairs; y is read-modified-written once per row.
#include "bgmv_args.h"
#include "common.cuh"
#include "plan_layout.h"

namespace persona {

constexpr int kConsumerWarps = 8;
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kBgmvThreads = kConsumers + 32;  // + one producer warp
constexpr int kStageBytes = 32768;
constexpr int kStages = 4;
constexpr int kXWin = 512;                     // k extent of the staged x window
constexpr int kPairs = kRowsPerItem / 2;       // row pairs per item
constexpr int kMaxR = 64;
constexpr int kNamedBarConsumers = 1;

constexpr int kRingBytes = kStages * kStageBytes;
constexpr int kX2Bytes = kPairs * kXWin * 8;            // float2 [pairs][window]
constexpr int kVBytes = kPairs * kMaxR * 8;             // float2 [pairs][R]
constexpr int kSmemLayoutBytes = kRingBytes + kX2Bytes + 4 * kVBytes + 64 + 16 * 8;
constexpr int kBgmvSmemBytes = kSmemLayoutBytes + 1024;  // slack to align the base

template <int R>
struct RankCfg {
  static_assert(R == 8 || R == 16 || R == 32 || R == 64, "rank");
  static constexpr int kRP = R / 2;  // a thread's rank pair is (rp, rp + R/2)
  static constexpr int kKC = (kStageBytes / (2 * R)) < kXWin ? (kStageBytes / (2 * R)) : kXWin;
  static constexpr int kABoxBytes = 128 * R;  // TMA box {64 k, R rows}
  static constexpr int kAUnits = kKC / 8;     // 16-byte k units per A stage
  static constexpr int kKGroups = kConsumers / kRP;
  static constexpr int kKUPT = kAUnits / kKGroups;
  static_assert(kKUPT >= 1 && kKUPT * kKGroups == kAUnits, "shrink mapping");
  static constexpr int kNB = kStageBytes / (2 * R);  // B rows per stage (capacity)
  static constexpr uint32_t kBSwz = (2 * R == 128) ? 7u : (2 * R == 64) ? 3u : (2 * R == 32) ? 1u : 0u;
  static constexpr int kRU = R / 8;  // 16-byte units per B row
};


struct SmemPtrs {
  uint8_t* ring;
  float2* x2;
  float2* pv;      // [2][pairs][R] local partial of v
  float2* vf;      // [2][pairs][R] full v (row pairs)
  int* rows;       // [16]
  uint64_t* full;  // [kStages]
  uint64_t* empty; // [kStages]
  uint64_t* red;   // [2]
  uint64_t* gat;   // [2]
};

__device__ __forceinline__ SmemPtrs carve_smem(uint8_t* raw) {
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
  SmemPtrs p;
  p.ring = base;
  p.x2 = reinterpret_cast<float2*>(base + kRingBytes);
  p.pv = reinterpret_cast<float2*>(base + kRingBytes + kX2Bytes);
  p.vf = reinterpret_cast<float2*>(base + kRingBytes + kX2Bytes + 2 * kVBytes);
  p.rows = reinterpret_cast<int*>(base + kRingBytes + kX2Bytes + 4 * kVBytes);
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + kRingBytes + kX2Bytes + 4 * kVBytes + 64);
  p.full = bars;
  p.empty = bars + kStages;
  p.red = bars + 2 * kStages;
  p.gat = bars + 2 * kStages + 2;
  return p;
}

__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }

// ---------------------------------------------------------------- shrink --
// acc0/acc1[p] accumulate (v[2p][r], v[2p+1][r]) for r = rp and rp + R/2
// over the k units this thread owns in one A stage.
template <typename DT, int R, int P>
__device__ __forceinline__ void shrink_stage(const uint8_t* stage, const float2* x2, int xoff,
                                             int units_loaded, int tid, float2 (&acc0)[kPairs],
                                             float2 (&acc1)[kPairs]) {
  using C = RankCfg<R>;
  const int rp = tid % C::kRP;
  const int kg = tid / C::kRP;
  const int r0 = rp, r1 = rp + C::kRP;
  const uint32_t sbase = smem_u32(stage);
  const uint32_t xbase = smem_u32(x2);
#pragma unroll
  for (int j = 0; j < C::kKUPT; ++j) {
    const int ku = kg + j * C::kKGroups;
    if (ku >= units_loaded) break;
    const int bx = ku >> 3, u = ku & 7;
    const uint32_t boff = sbase + bx * C::kABoxBytes;
    const uint4 a0 = lds128(boff + r0 * 128 + ((u ^ (r0 & 7)) << 4));
    const uint4 a1 = lds128(boff + r1 * 128 + ((u ^ (r1 & 7)) << 4));
    float fa0[8], fa1[8];
    {
      float2 t;
      t = Cvt<DT>::to2(a0.x); fa0[0] = t.x; fa0[1] = t.y;
      t = Cvt<DT>::to2(a0.y); fa0[2] = t.x; fa0[3] = t.y;
      t = Cvt<DT>::to2(a0.z); fa0[4] = t.x; fa0[5] = t.y;
      t = Cvt<DT>::to2(a0.w); fa0[6] = t.x; fa0[7] = t.y;
      t = Cvt<DT>::to2(a1.x); fa1[0] = t.x; fa1[1] = t.y;
      t = Cvt<DT>::to2(a1.y); fa1[2] = t.x; fa1[3] = t.y;
      t = Cvt<DT>::to2(a1.z); fa1[4] = t.x; fa1[5] = t.y;
      t = Cvt<DT>::to2(a1.w); fa1[6] = t.x; fa1[7] = t.y;
    }
    const int kx = xoff + ku * 8;
#pragma unroll
    for (int p = 0; p < P; ++p) {
      const uint32_t xa = xbase + static_cast<uint32_t>((p * kXWin + kx) * 8);
      const float4 q0 = lds128f(xa), q1 = lds128f(xa + 16), q2 = lds128f(xa + 32), q3 = lds128f(xa + 48);
      acc0[p] = __ffma2_rn(f2(q0.x, q0.y), f2(fa0[0], fa0[0]), acc0[p]);
      acc1[p] = __ffma2_rn(f2(q0.x, q0.y), f2(fa1[0], fa1[0]), acc1[p]);
      acc0[p] = __ffma2_rn(f2(q0.z, q0.w), f2(fa0[1], fa0[1]), acc0[p]);
      acc1[p] = __ffma2_rn(f2(q0.z, q0.w), f2(fa1[1], fa1[1]), acc1[p]);
      acc0[p] = __ffma2_rn(f2(q1.x, q1.y), f2(fa0[2], fa0[2]), acc0[p]);
      acc1[p] = __ffma2_rn(f2(q1.x, q1.y), f2(fa1[2], fa1[2]), acc1[p]);
      acc0[p] = __ffma2_rn(f2(q1.z, q1.w), f2(fa0[3], fa0[3]), acc0[p]);
      acc1[p] = __ffma2_rn(f2(q1.z, q1.w), f2(fa1[3], fa1[3]), acc1[p]);
      acc0[p] = __ffma2_rn(f2(q2.x, q2.y), f2(fa0[4], fa0[4]), acc0[p]);
      acc1[p] = __ffma2_rn(f2(q2.x, q2.y), f2(fa1[4], fa1[4]), acc1[p]);
      acc0[p] = __ffma2_rn(f2(q2.z, q2.w), f2(fa0[5], fa0[5]), acc0[p]);
      acc1[p] = __ffma2_rn(f2(q2.z, q2.w), f2(fa1[5], fa1[5]), acc1[p]);
      acc0[p] = __ffma2_rn(f2(q3.x, q3.y), f2(fa0[6], fa0[6]), acc0[p]);
      acc1[p] = __ffma2_rn(f2(q3.x, q3.y), f2(fa1[6], fa1[6]), acc1[p]);
      acc0[p] = __ffma2_rn(f2(q3.z, q3.w), f2(fa0[7], fa0[7]), acc0[p]);
      acc1[p] = __ffma2_rn(f2(q3.z, q3.w), f2(fa1[7], fa1[7]), acc1[p]);
    }
  }
}

// ---------------------------------------------------------------- expand --
// One stage of B rows: y[rows][n] += sum_r B[n][r] * v[rows][r].
template <typename DT, int R, int P>
__device__ __forceinline__ void expand_stage(const uint8_t* stage, const float2* vf, int nboxes,
                                             int n_box, int n0, int nend, int c, const int* rows,
                                             uint16_t* y, int64_t ldy, int tid) {
  using C = RankCfg<R>;
  const uint32_t sbase = smem_u32(stage);
  const uint32_t vbase = smem_u32(vf);
  for (int bx = 0; bx < nboxes; ++bx) {
    const int nb0 = n0 + bx * n_box;
    const int rows_here = min(n_box, nend - nb0);
    const uint32_t boff = sbase + static_cast<uint32_t>(bx * n_box * 2 * R);
    for (int rib = tid; rib < rows_here; rib += kConsumers) {
      float2 acc[kPairs];
#pragma unroll
      for (int p = 0; p < kPairs; ++p) acc[p] = f2(0.f, 0.f);
#pragma unroll
      for (int u = 0; u < C::kRU; ++u) {
        const uint4 bw = lds128(boff + swz(static_cast<uint32_t>(rib * 2 * R + u * 16), C::kBSwz));
        float fb[8];
        {
          float2 t;
          t = Cvt<DT>::to2(bw.x); fb[0] = t.x; fb[1] = t.y;
          t = Cvt<DT>::to2(bw.y); fb[2] = t.x; fb[3] = t.y;
          t = Cvt<DT>::to2(bw.z); fb[4] = t.x; fb[5] = t.y;
          t = Cvt<DT>::to2(bw.w); fb[6] = t.x; fb[7] = t.y;
        }
#pragma unroll
        for (int p = 0; p < P; ++p) {
          const uint32_t va = vbase + static_cast<uint32_t>((p * R + u * 8) * 8);
          const float4 q0 = lds128f(va), q1 = lds128f(va + 16), q2 = lds128f(va + 32), q3 = lds128f(va + 48);
          acc[p] = __ffma2_rn(f2(q0.x, q0.y), f2(fb[0], fb[0]), acc[p]);
          acc[p] = __ffma2_rn(f2(q0.z, q0.w), f2(fb[1], fb[1]), acc[p]);
          acc[p] = __ffma2_rn(f2(q1.x, q1.y), f2(fb[2], fb[2]), acc[p]);
          acc[p] = __ffma2_rn(f2(q1.z, q1.w), f2(fb[3], fb[3]), acc[p]);
          acc[p] = __ffma2_rn(f2(q2.x, q2.y), f2(fb[4], fb[4]), acc[p]);
          acc[p] = __ffma2_rn(f2(q2.z, q2.w), f2(fb[5], fb[5]), acc[p]);
          acc[p] = __ffma2_rn(f2(q3.x, q3.y), f2(fb[6], fb[6]), acc[p]);
          acc[p] = __ffma2_rn(f2(q3.z, q3.w), f2(fb[7], fb[7]), acc[p]);
        }
      }
      const int n = nb0 + rib;
      uint16_t yo[2 * kPairs];
#pragma unroll
      for (int p = 0; p < P; ++p) {
        if (2 * p < c) yo[2 * p] = y[static_cast<int64_t>(rows[2 * p]) * ldy + n];
        if (2 * p + 1 < c) yo[2 * p + 1] = y[static_cast<int64_t>(rows[2 * p + 1]) * ldy + n];
      }
#pragma unroll
      for (int p = 0; p < P; ++p) {
        if (2 * p < c)
          y[static_cast<int64_t>(rows[2 * p]) * ldy + n] = Cvt<DT>::from1(Cvt<DT>::to1(yo[2 * p]) + acc[p].x);
        if (2 * p + 1 < c)
          y[static_cast<int64_t>(rows[2 * p + 1]) * ldy + n] =
              Cvt<DT>::from1(Cvt<DT>::to1(yo[2 * p + 1]) + acc[p].y);
      }
    }
  }
}

// Gather the item's x rows for k in [w0, w0 + kXWin) into x2 as fp32 row pairs.
// Columns at or past `klim` (the end of this CTA's K slice) read as zero.
template <typename DT>
__device__ __forceinline__ void load_x_window(const uint16_t* x, int64_t ldx, int klim, int w0,
                                              const int* rows, int c, int P, float2* x2, int tid) {
#pragma unroll 4
  for (int idx = tid; idx < P * (kXWin / 2); idx += kConsumers) {
    const int p = idx / (kXWin / 2);
    const int kk = (idx % (kXWin / 2)) * 2;
    const int k = w0 + kk;
    uint32_t w_lo = 0, w_hi = 0;
    if (k < klim) {
      if (2 * p < c) w_lo = *reinterpret_cast<const uint32_t*>(x + static_cast<int64_t>(rows[2 * p]) * ldx + k);
      if (2 * p + 1 < c)
        w_hi = *reinterpret_cast<const uint32_t*>(x + static_cast<int64_t>(rows[2 * p + 1]) * ldx + k);
    }
    const float2 lo = Cvt<DT>::to2(w_lo), hi = Cvt<DT>::to2(w_hi);
    float4* dst = reinterpret_cast<float4*>(x2 + p * kXWin + kk);
    *dst = make_float4(lo.x, hi.x, lo.y, hi.y);
  }
}

template <typename DT, int R, int MODE>
__global__ void __launch_bounds__(kBgmvThreads, 1)
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
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], kConsumerWarps);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sm.red[b], CS);
      mbar_init(&sm.gat[b], CS);
    }
    fence_mbar_init_cluster();
  }
  cluster_sync_all();

  PlanView pv = plan_view(const_cast<int32_t*>(args.plan), args.T);
  const int n_items = pv.hdr[kHdrItems];
  const int kbeg = static_cast<int>(q) * args.k_per_cta;
  const int kend = min(args.K, kbeg + args.k_per_cta);
  const int nbeg = static_cast<int>(q) * args.n_per_cta;
  const int nend = min(args.N, nbeg + args.n_per_cta);
  const int bps = C::kNB / args.n_box;           // B boxes per stage
  const int stage_rows = bps * args.n_box;

  if (warp == kConsumerWarps) {
    // ------------------------------------------------------- producer --
    if (lane == 0) {
      if (kDoShrink) tma_prefetch_desc(&tmA);
      if (kDoExpand) tma_prefetch_desc(&tmB);
      uint32_t g = 0;
      for (int item = cid; item < n_items; item += ncl) {
        const int slot = pv.items[item].x;
        if (kDoShrink) {
          for (int k0 = kbeg; k0 < kend; k0 += C::kKC, ++g) {
            const int s = g % kStages;
            if (g >= kStages) mbar_wait(&sm.empty[s], ((g / kStages) - 1) & 1, args.err);
            const int nbox = (min(C::kKC, kend - k0) + 63) / 64;
            mbar_arrive_expect_tx(&sm.full[s], nbox * C::kABoxBytes);
            for (int b = 0; b < nbox; ++b)
              tma_load_3d(sm.ring + s * kStageBytes + b * C::kABoxBytes, &tmA, &sm.full[s],
                          k0 + 64 * b, 0, slot);
          }
        }
        if (kDoExpand) {
          for (int n0 = nbeg; n0 < nend; n0 += stage_rows, ++g) {
            const int s = g % kStages;
            if (g >= kStages) mbar_wait(&sm.empty[s], ((g / kStages) - 1) & 1, args.err);
            const int nbox = (min(stage_rows, nend - n0) + args.n_box - 1) / args.n_box;
            mbar_arrive_expect_tx(&sm.full[s], nbox * args.n_box * 2 * R);
            for (int b = 0; b < nbox; ++b)
              tma_load_3d(sm.ring + s * kStageBytes + b * args.n_box * 2 * R, &tmB, &sm.full[s], 0,
                          n0 + b * args.n_box, slot);
          }
        }
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------ consumers --
    const uint16_t* x = static_cast<const uint16_t*>(args.x);
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
    for (int item = cid; item < n_items; item += ncl, ++j) {
      const int4 it = pv.items[item];
      const int c = it.z;
      const int P = (c + 1) >> 1;
      const int b = j & 1;
      const uint32_t red_parity = (j >> 1) & 1;
      float2* pvb = sm.pv + b * kPairs * kMaxR;
      float2* vfb = sm.vf + b * kPairs * kMaxR;
      named_sync(kNamedBarConsumers, kConsumers);  // previous item done with rows / x2
      if (tid < kRowsPerItem) sm.rows[tid] = tid < c ? pv.perm[it.y + tid] : 0;
      named_sync(kNamedBarConsumers, kConsumers);

      if (kDoShrink) {
        float2 acc0[kPairs], acc1[kPairs];
#pragma unroll
        for (int p = 0; p < kPairs; ++p) acc0[p] = acc1[p] = f2(0.f, 0.f);
        int w0 = kbeg;
        for (int k0 = kbeg; k0 < kend; k0 += C::kKC, ++g) {
          if (((k0 - kbeg) % kXWin) == 0) {
            w0 = k0;
            if (k0 != kbeg) named_sync(kNamedBarConsumers, kConsumers);
            load_x_window<DT>(x, args.ldx, kend, w0, sm.rows, c, P, sm.x2, tid);
            named_sync(kNamedBarConsumers, kConsumers);
          }
          const int s = g % kStages;
          mbar_wait(&sm.full[s], (g / kStages) & 1, args.err);
          const int units = ((min(C::kKC, kend - k0) + 63) / 64) * 8;
          const uint8_t* st = sm.ring + s * kStageBytes;
          switch (P) {
            case 1: shrink_stage<DT, R, 1>(st, sm.x2, k0 - w0, units, tid, acc0, acc1); break;
            case 2: shrink_stage<DT, R, 2>(st, sm.x2, k0 - w0, units, tid, acc0, acc1); break;
            case 3: case 4: shrink_stage<DT, R, 4>(st, sm.x2, k0 - w0, units, tid, acc0, acc1); break;
            default: shrink_stage<DT, R, 8>(st, sm.x2, k0 - w0, units, tid, acc0, acc1); break;
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&sm.empty[s]);
        }
        // Reduce the k groups of this CTA: lanes sharing a rank pair, then warps.
#pragma unroll
        for (int off = C::kRP; off < 32; off <<= 1) {
#pragma unroll
          for (int p = 0; p < kPairs; ++p) {
            acc0[p].x += __shfl_xor_sync(0xffffffffu, acc0[p].x, off);
            acc0[p].y += __shfl_xor_sync(0xffffffffu, acc0[p].y, off);
            acc1[p].x += __shfl_xor_sync(0xffffffffu, acc1[p].x, off);
            acc1[p].y += __shfl_xor_sync(0xffffffffu, acc1[p].y, off);
          }
        }
        named_sync(kNamedBarConsumers, kConsumers);  // x2 free -> reduction scratch
        float2* red = sm.x2;                         // [warp][pairs][R]
        if (lane < C::kRP) {
          const int rp = lane;
#pragma unroll
          for (int p = 0; p < kPairs; ++p) {
            if (p < P) {
              red[(warp * kPairs + p) * R + rp] = acc0[p];
              red[(warp * kPairs + p) * R + rp + C::kRP] = acc1[p];
            }
          }
        }
        named_sync(kNamedBarConsumers, kConsumers);
        for (int e = tid; e < P * R; e += kConsumers) {
          float2 sum = red[e];
#pragma unroll
          for (int w = 1; w < kConsumerWarps; ++w) {
            const float2 t = red[w * kPairs * R + e];
            sum.x += t.x;
            sum.y += t.y;
          }
          pvb[e] = sum;
        }
        // Cluster reduce-scatter of the partial v's through DSMEM.
        named_sync(kNamedBarConsumers, kConsumers);
        if (tid == 0) {
          fence_acq_rel_cluster();
          for (uint32_t r = 0; r < CS; ++r) mbar_arrive_remote(&sm.red[b], r);
        }
        mbar_wait<true>(&sm.red[b], red_parity, args.err);
        const int E = P * R;
        const int share = (E + CS - 1) / CS;
        const int e_lo = static_cast<int>(q) * share;
        const int e_hi = min(E, e_lo + share);
        for (int e = e_lo + tid; e < e_hi; e += kConsumers) {
          float2 sum = f2(0.f, 0.f);
          for (uint32_t r = 0; r < CS; ++r) {
            const float2 t = ld_dsmem_f2(mapa(pvb + e, r));
            sum.x += t.x;
            sum.y += t.y;
          }
          if (MODE == kModeFused) {
            for (uint32_t r = 0; r < CS; ++r) st_dsmem_f2(mapa(vfb + e, r), sum);
          } else {
            const int p = e / R, rr = e % R;
            if (2 * p < c) args.v_out[static_cast<int64_t>(sm.rows[2 * p]) * R + rr] = sum.x;
            if (2 * p + 1 < c) args.v_out[static_cast<int64_t>(sm.rows[2 * p + 1]) * R + rr] = sum.y;
          }
        }
        if (MODE == kModeFused) {
          named_sync(kNamedBarConsumers, kConsumers);
          if (tid == 0) {
            fence_acq_rel_cluster();
            for (uint32_t r = 0; r < CS; ++r) mbar_arrive_remote(&sm.gat[b], r);
          }
          mbar_wait<true>(&sm.gat[b], red_parity, args.err);
        }
      }

      if (kDoExpand) {
        if (MODE == kModeExpand) {
          for (int e = tid; e < P * R; e += kConsumers) {
            const int p = e / R, rr = e % R;
            float lo = 0.f, hi = 0.f;
            if (2 * p < c) lo = args.v_in[static_cast<int64_t>(sm.rows[2 * p]) * R + rr];
            if (2 * p + 1 < c) hi = args.v_in[static_cast<int64_t>(sm.rows[2 * p + 1]) * R + rr];
            vfb[e] = f2(lo, hi);
          }
          named_sync(kNamedBarConsumers, kConsumers);
        }
        for (int n0 = nbeg; n0 < nend; n0 += stage_rows, ++g) {
          const int s = g % kStages;
          mbar_wait(&sm.full[s], (g / kStages) & 1, args.err);
          const int nbox = (min(stage_rows, nend - n0) + args.n_box - 1) / args.n_box;
          const uint8_t* st = sm.ring + s * kStageBytes;
          switch (P) {
            case 1: expand_stage<DT, R, 1>(st, vfb, nbox, args.n_box, n0, nend, c, sm.rows, y, args.ldy, tid); break;
            case 2: expand_stage<DT, R, 2>(st, vfb, nbox, args.n_box, n0, nend, c, sm.rows, y, args.ldy, tid); break;
            case 3: case 4: expand_stage<DT, R, 4>(st, vfb, nbox, args.n_box, n0, nend, c, sm.rows, y, args.ldy, tid); break;
            default: expand_stage<DT, R, 8>(st, vfb, nbox, args.n_box, n0, nend, c, sm.rows, y, args.ldy, tid); break;
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(&sm.empty[s]);
        }
      }
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
  // and per portable (<= 8) / non-portable (16) cluster size.
  constexpr int kMaxDev = 64;
  static bool configured[kMaxDev][2] = {};
  static int occ[kMaxDev][2] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDev) return cudaErrorInvalidDevice;
  const int ci = cluster_size > 8 ? 1 : 0;
  if (!configured[dev][ci]) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kBgmvSmemBytes);
    if (e != cudaSuccess) return e;
    if (cluster_size > 8) {
      e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
      if (e != cudaSuccess) return e;
    }
    configured[dev][ci] = true;
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
