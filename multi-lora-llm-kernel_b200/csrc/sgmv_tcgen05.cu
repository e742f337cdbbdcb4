// Segmented (SGMV) shrink / expand / fused kernels on the sm_100a tensor
// cores (tcgen05 + TMEM), for prefill batches whose rows come in long runs
// that share an adapter.
//
// Same math as the BGMV ops (reference persona/ops.py:12-56) on the rows the
// segment table assigns to each adapter: v = x A[s]^T, y += v B[s]^T.
//
// Work unit: a 128-row item of one segment (from the segment plan), one MMA
// tile high.  Per CTA (persistent over items), six warps:
//   warp 0  TMA producer: x / A chunks (K = 64) into a 4-stage shrink ring,
//           y / B tiles (128 columns) into a 3-stage expand ring;
//   warp 1  MMA issuer (one thread): shrink D_v[128 x R] += x_chunk A_chunk^T
//           (M = 128, N = R, K = 16 per instruction) into TMEM; expand
//           D_y[128 x 128] = V'[128 x 2R] B_tile^T into one of two TMEM
//           accumulators; completion is signalled with tcgen05.commit;
//   warps 2-5  epilogue, one thread per TMEM lane (= row): read D_v, split v
//           into 16-bit hi + lo halves (per-row power-of-two scale for f16)
//           and write them to shared memory as the expand's A operand V';
//           read D_y, add the y tile, write it back and TMA-store it;
//   warps 6-9  exchange (tensor parallel only): copy each finished y tile
//           from shared memory into the other ranks' y over NVLink, then
//           release the y stage, so the transfer runs beside the math of the
//           next tiles instead of inside the epilogue.
// The expand multiplies B by hi and by lo, so v keeps ~fp32 precision.
// Only full items use the TMA store; a short item (segment tail) writes its
// valid rows with plain stores, so rows of the next segment are never
// touched.
#include <type_traits>

#include "bgmv_args.h"
#include "common.cuh"
#include "plan_layout.h"
#include "tcgen05.cuh"

namespace persona {

constexpr int kTcRows = 128;   // rows per item (MMA M)
constexpr int kTcNT = 128;     // expand output columns per tile (MMA N)
constexpr int kTcKC = 64;      // shrink K chunk (one 128-byte swizzled row)
constexpr int kSStages = 4;
constexpr int kEStages = 3;
constexpr int kTcThreads = 10 * 32;
constexpr int kEpiBar = 1;     // named barrier of the four epilogue warps
constexpr int kXchWarps = 4;   // warps 6-9
constexpr uint32_t kTmemCols = 512;


template <int R>
struct TcCfg {
  static_assert(R == 16 || R == 32, "tensor-core SGMV ranks");
  static constexpr int kXBytes = kTcRows * kTcKC * 2;  // 16 KB
  static constexpr int kABytes = R * kTcKC * 2;
  static constexpr int kSBytes = kXBytes + kABytes;    // multiple of 1024
  static constexpr int kYBox = kTcRows * 64 * 2;       // 16 KB: 64 columns x 128 rows
  static constexpr int kYBytes = 2 * kYBox;
  static constexpr int kBBytes = kTcNT * R * 2;
  static constexpr int kEBytes = kYBytes + kBBytes;
  static constexpr uint32_t kBLayout = R == 16 ? tc::kLayoutSw32 : tc::kLayoutSw64;
  static constexpr uint32_t kBSbo = 8 * 2 * R;  // 8 rows of 2R bytes
  static constexpr int kVBytes = kTcRows * 128;  // V' rows of 128 bytes (hi | lo | 0)
  static constexpr int kSmem = kSStages * kSBytes + kEStages * kEBytes + kVBytes;
  static_assert(kSBytes % 1024 == 0 && kEBytes % 1024 == 0, "stage alignment");
};

struct TcBars {
  uint64_t sfull[kSStages], sempty[kSStages];
  uint64_t efull[kEStages], eempty[kEStages];
  uint64_t xready[kEStages];  // y tile complete in shared memory (exchange warps)
  uint64_t v_ready, v_used, vsm_ready;
  uint64_t acc_full[2], acc_empty[2];
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort;  // set by the first wait that runs out; later waits return at once
};

// Bounded wait that also gives up as soon as another thread of the CTA has
// given up, so a CTA whose pipeline broke ends after one wait budget.
__device__ __forceinline__ bool tc_wait(uint64_t* bar, uint32_t parity, int32_t* err, int* abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*reinterpret_cast<volatile int*>(abort)) return false;
    if (clock64() - t0 > kWaitBudgetCycles) {
      *reinterpret_cast<volatile int*>(abort) = 1;
      raise_error(err, PERSONA_DEV_ERR_TIMEOUT);
      return false;
    }
  }
}

template <typename DT, int R, int MODE>
__global__ void __launch_bounds__(kTcThreads, 1)
    sgmv_tc_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmA,
                   const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmY,
                   const SgmvTcArgs args) {
  using C = TcCfg<R>;
  constexpr bool kDoShrink = (MODE & kModeShrink) != 0;
  constexpr bool kDoExpand = (MODE & kModeExpand) != 0;
  constexpr uint32_t kFmt = std::is_same<DT, __nv_bfloat16>::value ? 1u : 0u;
  constexpr uint32_t kIdescV = tc::idesc_f16(kFmt, kTcRows, R);
  constexpr uint32_t kIdescY = tc::idesc_f16(kFmt, kTcRows, kTcNT);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sring = base;
  uint8_t* ering = base + kSStages * C::kSBytes;
  uint8_t* vsm = ering + kEStages * C::kEBytes;
  __shared__ TcBars bars;

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int i = 0; i < kSStages; ++i) {
      mbar_init(&bars.sfull[i], 1);
      mbar_init(&bars.sempty[i], 1);
    }
    // A y stage is free again once the epilogue's TMA store has read it
    // and, with peers, once every exchange warp has copied it out.
    const int xch = args.num_peers > 0 ? kXchWarps : 0;
    for (int i = 0; i < kEStages; ++i) {
      mbar_init(&bars.efull[i], 1);
      mbar_init(&bars.eempty[i], 1 + xch);
      mbar_init(&bars.xready[i], 1);
    }
    mbar_init(&bars.v_ready, 1);
    mbar_init(&bars.v_used, 4);
    mbar_init(&bars.vsm_ready, 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&bars.acc_full[b], 1);
      mbar_init(&bars.acc_empty[b], 4);
    }
    mbar_init(&bars.mma_done, 1);
    bars.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    tc::tmem_alloc(&bars.tmem_base, kTmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = bars.tmem_base;
  int* abort = &bars.abort;

  PlanView pv = plan_view(const_cast<int32_t*>(args.plan), args.T);
  const int n_items = pv.hdr[kHdrItems];
  const int nk = (args.K + kTcKC - 1) / kTcKC;
  const int nn = args.N / kTcNT;

  if (warp == 0) {
    // ------------------------------------------------------ producer ----
    if (lane == 0) {
      if (kDoShrink) {
        tma_prefetch_desc(&tmX);
        tma_prefetch_desc(&tmA);
      }
      if (kDoExpand) {
        tma_prefetch_desc(&tmY);
        tma_prefetch_desc(&tmB);
      }
      uint32_t gs = 0, ge = 0;
      bool ok = true;
      for (int item = blockIdx.x; ok && item < n_items; item += gridDim.x) {
        const int4 it = pv.items[item];
        const int slot = it.x, row0 = it.y;
        if (kDoShrink) {
          for (int kc = 0; kc < nk; ++kc) {
            const int s = gs % kSStages;
            if (gs >= kSStages && !tc_wait(&bars.sempty[s], ((gs / kSStages) - 1) & 1, args.err, abort)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&bars.sfull[s], C::kSBytes);
            uint8_t* st = sring + s * C::kSBytes;
            tc::tma_load_2d(st, &tmX, &bars.sfull[s], kc * kTcKC, row0);
            tma_load_3d(st + C::kXBytes, &tmA, &bars.sfull[s], kc * kTcKC, 0, slot);
            ++gs;
          }
        }
        if (kDoExpand && ok) {
          for (int t = 0; t < nn; ++t) {
            const int e = ge % kEStages;
            if (ge >= kEStages && !tc_wait(&bars.eempty[e], ((ge / kEStages) - 1) & 1, args.err, abort)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&bars.efull[e], C::kEBytes);
            uint8_t* st = ering + e * C::kEBytes;
            const int col = args.n0 + t * kTcNT;
            tc::tma_load_2d(st, &tmY, &bars.efull[e], col, row0);
            tc::tma_load_2d(st + C::kYBox, &tmY, &bars.efull[e], col + 64, row0);
            tma_load_3d(st + C::kYBytes, &tmB, &bars.efull[e], 0, col, slot);
            ++ge;
          }
        }
      }
      // Every load this thread issued lands before the CTA can exit: wait
      // (bounded, whatever the abort flag says) for the last fill of each
      // stage.  Earlier fills of a stage completed before it was refilled.
      for (int s = 0; s < kSStages; ++s)
        if (gs > static_cast<uint32_t>(s)) {
          const uint32_t last = (gs - 1 - s) / kSStages;  // index of the stage's last fill
          mbar_wait(&bars.sfull[s], last & 1, args.err);
        }
      for (int e = 0; e < kEStages; ++e)
        if (ge > static_cast<uint32_t>(e)) {
          const uint32_t last = (ge - 1 - e) / kEStages;
          mbar_wait(&bars.efull[e], last & 1, args.err);
        }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ----------------------------------------------------------- MMA ----
    if (lane == 0) {
      uint32_t gs = 0, ge = 0, nt = 0, j = 0;
      bool ok = true;
      const uint32_t d_v = tmem;
      for (int item = blockIdx.x; ok && item < n_items; item += gridDim.x, ++j) {
        if (kDoShrink) {
          if (j > 0 && !tc_wait(&bars.v_used, (j - 1) & 1, args.err, abort)) break;  // D_v of the previous item read
          tc::fence_after_sync();
          for (int kc = 0; kc < nk; ++kc, ++gs) {
            const int s = gs % kSStages;
            if (!tc_wait(&bars.sfull[s], (gs / kSStages) & 1, args.err, abort)) {
              ok = false;
              break;
            }
            tc::fence_after_sync();
            const uint32_t sx = smem_u32(sring + s * C::kSBytes);
#pragma unroll
            for (int ks = 0; ks < kTcKC / 16; ++ks) {
              const uint64_t a = tc::smem_desc(sx + ks * 32, 1024, tc::kLayoutSw128);
              const uint64_t b = tc::smem_desc(sx + C::kXBytes + ks * 32, 1024, tc::kLayoutSw128);
              tc::mma_f16(d_v, a, b, kIdescV, (kc > 0 || ks > 0) ? 1u : 0u);
            }
            tc::commit(&bars.sempty[s]);
          }
          if (!ok) break;
          tc::commit(&bars.v_ready);
        }
        if (kDoExpand) {
          if (!tc_wait(&bars.vsm_ready, j & 1, args.err, abort)) break;
          tc::fence_after_sync();
          const uint32_t sv = smem_u32(vsm);
          for (int t = 0; t < nn; ++t, ++ge, ++nt) {
            const int e = ge % kEStages;
            const uint32_t buf = nt & 1;
            if (!tc_wait(&bars.efull[e], (ge / kEStages) & 1, args.err, abort) ||
                (nt >= 2 && !tc_wait(&bars.acc_empty[buf], ((nt / 2) - 1) & 1, args.err, abort))) {
              ok = false;
              break;
            }
            tc::fence_after_sync();
            const uint32_t sb = smem_u32(ering + e * C::kEBytes + C::kYBytes);
            const uint32_t d_y = tmem + 128u * (buf + 1);
#pragma unroll
            for (int ks = 0; ks < R / 16; ++ks) {
              const uint64_t b = tc::smem_desc(sb + ks * 32, C::kBSbo, C::kBLayout);
              tc::mma_f16(d_y, tc::smem_desc(sv + ks * 32, 1024, tc::kLayoutSw128), b, kIdescY, ks > 0 ? 1u : 0u);
              tc::mma_f16(d_y, tc::smem_desc(sv + (R / 16 + ks) * 32, 1024, tc::kLayoutSw128), b, kIdescY, 1u);
            }
            tc::commit(&bars.acc_full[buf]);
          }
        }
      }
      // All MMAs this thread issued complete before TMEM is released.
      tc::commit(&bars.mma_done);
      mbar_wait(&bars.mma_done, 0, args.err);
    }
    __syncwarp();
  } else if (warp < 6) {
    // ------------------------------------------------------ epilogue ----
    // Every epilogue thread runs the same item / tile loop to the end, so
    // the named barriers stay matched; after an abort the waits return at
    // once and nothing more is written to global memory.
    const int quarter = warp & 3;          // TMEM lanes this warp may access
    const int row = quarter * 32 + lane;   // row of the item this thread owns
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    const int ew = warp - 2;
    uint32_t ge = 0, nt = 0, j = 0;
    bool stored = false;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x, ++j) {
      const int4 it = pv.items[item];
      const int row0 = it.y, count = it.z;
      const bool valid = row < count;
      const int64_t grow = static_cast<int64_t>(row0) + row;
      float v[R];
      if (kDoShrink) {
        tc_wait(&bars.v_ready, j & 1, args.err, abort);
        __syncwarp();
        tc::fence_after_sync();
        uint32_t r16[16];
#pragma unroll
        for (int h = 0; h < R / 16; ++h) {
          tc::ld16(tmem + lane_addr + 16 * h, r16);
          tc::wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i) v[16 * h + i] = __uint_as_float(r16[i]);
        }
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars.v_used);
        if (MODE == kModeShrink && valid && !*reinterpret_cast<volatile int*>(abort)) {
#pragma unroll
          for (int i = 0; i < R; i += 4)
            *reinterpret_cast<float4*>(args.v_out + grow * R + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
        }
      } else {
#pragma unroll
        for (int i = 0; i < R; i += 4) {
          const float4 q = valid ? *reinterpret_cast<const float4*>(args.v_in + grow * R + i) : make_float4(0, 0, 0, 0);
          v[i] = q.x;
          v[i + 1] = q.y;
          v[i + 2] = q.z;
          v[i + 3] = q.w;
        }
      }
      if (kDoExpand) {
        // Per-row power-of-two scale keeps the f16 halves finite.
        float scale_up = 1.f, scale_down = 1.f;
        if (kFmt == 0) {
          float m = 0.f;
#pragma unroll
          for (int i = 0; i < R; ++i) m = fmaxf(m, fabsf(v[i]));
          const int ex = static_cast<int>((__float_as_uint(m) >> 23) & 0xff) - 127;
          const int e2 = ex > 14 ? (ex - 14 < 100 ? ex - 14 : 100) : 0;
          scale_down = __uint_as_float(static_cast<uint32_t>(127 - e2) << 23);
          scale_up = __uint_as_float(static_cast<uint32_t>(127 + e2) << 23);
        }
        // V' row: [hi(R) | lo(R) | zeros] as 16-bit, 128-byte swizzled rows.
        uint32_t w[32];
#pragma unroll
        for (int i = 0; i < R; i += 2) {
          const float a = v[i] * scale_down, b = v[i + 1] * scale_down;
          const float ha = Mma<DT>::round_trip(a), hb = Mma<DT>::round_trip(b);
          w[i / 2] = Mma<DT>::pack(ha, hb);
          w[R / 2 + i / 2] = Mma<DT>::pack(a - ha, b - hb);
        }
#pragma unroll
        for (int i = R; i < 32; ++i) w[i] = 0u;
        const uint32_t vrow = smem_u32(vsm) + row * 128;
#pragma unroll
        for (int c = 0; c < 8; ++c)
          asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(vrow + ((c ^ (row & 7)) << 4)),
                       "r"(w[4 * c]), "r"(w[4 * c + 1]), "r"(w[4 * c + 2]), "r"(w[4 * c + 3])
                       : "memory");
        tc::fence_proxy_async();
        named_sync(kEpiBar, 128);
        if (ew == 0 && lane == 0) mbar_arrive(&bars.vsm_ready);

        for (int t = 0; t < nn; ++t, ++ge, ++nt) {
          const int e = ge % kEStages;
          const uint32_t buf = nt & 1;
          tc_wait(&bars.efull[e], (ge / kEStages) & 1, args.err, abort);
          tc_wait(&bars.acc_full[buf], (nt / 2) & 1, args.err, abort);
          __syncwarp();
          tc::fence_after_sync();
          const bool live = !*reinterpret_cast<volatile int*>(abort);
          uint8_t* st = ering + e * C::kEBytes;
          const uint32_t ybase = smem_u32(st);
#pragma unroll
          for (int c32 = 0; c32 < kTcNT / 32; ++c32) {
            uint32_t d0[16], d1[16];
            tc::ld16(tmem + lane_addr + 128u * (buf + 1) + 32 * c32, d0);
            tc::ld16(tmem + lane_addr + 128u * (buf + 1) + 32 * c32 + 16, d1);
            tc::wait_ld();
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) {  // 8-column chunks of this 32-column group
              const int chunk = c32 * 4 + cc;  // 0..15
              const int box = chunk >> 3, cb = chunk & 7;
              const uint32_t addr = ybase + box * C::kYBox + row * 128 + ((cb ^ (row & 7)) << 4);
              const uint4 yo = lds128(addr);
              const uint32_t* dd = cc < 2 ? d0 : d1;
              const int o = (cc & 1) * 8;
              const float2 y0 = Cvt<DT>::to2(yo.x), y1 = Cvt<DT>::to2(yo.y), y2 = Cvt<DT>::to2(yo.z),
                           y3 = Cvt<DT>::to2(yo.w);
              uint4 out;
              out.x = Mma<DT>::pack(y0.x + scale_up * __uint_as_float(dd[o + 0]),
                                    y0.y + scale_up * __uint_as_float(dd[o + 1]));
              out.y = Mma<DT>::pack(y1.x + scale_up * __uint_as_float(dd[o + 2]),
                                    y1.y + scale_up * __uint_as_float(dd[o + 3]));
              out.z = Mma<DT>::pack(y2.x + scale_up * __uint_as_float(dd[o + 4]),
                                    y2.y + scale_up * __uint_as_float(dd[o + 5]));
              out.w = Mma<DT>::pack(y3.x + scale_up * __uint_as_float(dd[o + 6]),
                                    y3.y + scale_up * __uint_as_float(dd[o + 7]));
              if (count == kTcRows) {
                asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(out.x), "r"(out.y),
                             "r"(out.z), "r"(out.w)
                             : "memory");
              } else if (valid && live) {
                const int64_t off = grow * args.ldy + args.n0 + t * kTcNT + chunk * 8;
                *reinterpret_cast<uint4*>(args.y + off) = out;
                for (int q = 0; q < args.num_peers; ++q) *reinterpret_cast<uint4*>(args.peers[q] + off) = out;
              }
            }
          }
          tc::fence_before_sync();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars.acc_empty[buf]);
          if (count == kTcRows) tc::fence_proxy_async();
          named_sync(kEpiBar, 128);
          const bool full_live = count == kTcRows && !*reinterpret_cast<volatile int*>(abort);
          if (ew == 0 && lane == 0 && full_live) {
            tc::tma_store_2d(&tmY, st, args.n0 + t * kTcNT, row0);
            tc::tma_store_2d(&tmY, st + C::kYBox, args.n0 + t * kTcNT + 64, row0);
            tc::bulk_commit();
            stored = true;
          }
          if (ew == 0 && lane == 0) {
            // The tile is complete in shared memory (barrier above): the
            // exchange warps may copy it out while the next tile is computed.
            if (args.num_peers > 0) mbar_arrive(&bars.xready[e]);
            if (full_live) tc::bulk_wait_read0();
            mbar_arrive(&bars.eempty[e]);
          }
        }
      }
    }
    if (stored) tc::bulk_wait0();
    // Plain stores into the peers' y (short items) are ordered before
    // whatever this thread's kernel completion is followed by.
    if (args.num_peers > 0) __threadfence_system();
  } else if (args.num_peers > 0) {
    // ------------------------------------------------------ exchange ----
    // Tensor parallel: every full 128 x 128 tile also goes to every other
    // rank's y over NVLink, 256 contiguous bytes per row, 16 threads per row
    // (rows of a short item were stored by the epilogue itself).  Each warp
    // releases the y stage when its share of the copy is issued; the values
    // are in registers by then, so the stage may be refilled.
    const int xw = warp - 6;
    uint32_t ge = 0;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
      const int4 it = pv.items[item];
      const int row0 = it.y, count = it.z;
      for (int t = 0; t < nn; ++t, ++ge) {
        const int e = ge % kEStages;
        const bool ok = tc_wait(&bars.xready[e], (ge / kEStages) & 1, args.err, abort);
        if (ok && count == kTcRows && !*reinterpret_cast<volatile int*>(abort)) {
          const uint32_t ybase = smem_u32(ering + e * C::kEBytes);
          const int64_t col = args.n0 + t * kTcNT;
#pragma unroll 4
          for (int i = 0; i < (kTcRows * 16) / (kXchWarps * 32); ++i) {
            const int idx = (xw * 32 + lane) + i * (kXchWarps * 32);
            const int r = idx >> 4, c16 = idx & 15, box = c16 >> 3, cb = c16 & 7;
            const uint4 val = lds128(ybase + box * C::kYBox + r * 128 + ((cb ^ (r & 7)) << 4));
            const int64_t off = (static_cast<int64_t>(row0) + r) * args.ldy + col + c16 * 8;
            for (int q = 0; q < args.num_peers; ++q) *reinterpret_cast<uint4*>(args.peers[q] + off) = val;
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars.eempty[e]);
      }
    }
    __threadfence_system();
  }
  tc::fence_before_sync();
  __syncthreads();
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, kTmemCols);
  }
}

// ------------------------------------------------------------------ host --

template <typename DT, int R, int MODE>
static cudaError_t tc_launch(const CUtensorMap& tx, const CUtensorMap& ta, const CUtensorMap& tb,
                             const CUtensorMap& ty, const SgmvTcArgs& a, int max_items, cudaStream_t st) {
  auto kern = sgmv_tc_kernel<DT, R, MODE>;
  constexpr int kMaxDev = 64;
  static bool configured[kMaxDev] = {};
  static int sms[kMaxDev] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDev) return cudaErrorInvalidDevice;
  const int smem = TcCfg<R>::kSmem + 1024;
  if (!configured[dev]) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    e = cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  int grid = sms[dev] < max_items ? sms[dev] : max_items;
  if (grid < 1) grid = 1;
  kern<<<grid, kTcThreads, smem, st>>>(tx, ta, tb, ty, a);
  return cudaGetLastError();
}

template <typename DT, int MODE>
static cudaError_t tc_rank(int R, const CUtensorMap& tx, const CUtensorMap& ta, const CUtensorMap& tb,
                           const CUtensorMap& ty, const SgmvTcArgs& a, int max_items, cudaStream_t st) {
  return R == 16 ? tc_launch<DT, 16, MODE>(tx, ta, tb, ty, a, max_items, st)
                 : tc_launch<DT, 32, MODE>(tx, ta, tb, ty, a, max_items, st);
}

cudaError_t launch_sgmv_tc(int mode, int dtype, int R, const CUtensorMap& tx, const CUtensorMap& ta,
                           const CUtensorMap& tb, const CUtensorMap& ty, const SgmvTcArgs& a, int max_items,
                           cudaStream_t st) {
  const bool bf = dtype == PERSONA_DTYPE_BF16;
  switch (mode) {
    case kModeShrink:
      return bf ? tc_rank<__nv_bfloat16, kModeShrink>(R, tx, ta, tb, ty, a, max_items, st)
                : tc_rank<__half, kModeShrink>(R, tx, ta, tb, ty, a, max_items, st);
    case kModeExpand:
      return bf ? tc_rank<__nv_bfloat16, kModeExpand>(R, tx, ta, tb, ty, a, max_items, st)
                : tc_rank<__half, kModeExpand>(R, tx, ta, tb, ty, a, max_items, st);
    default:
      return bf ? tc_rank<__nv_bfloat16, kModeFused>(R, tx, ta, tb, ty, a, max_items, st)
                : tc_rank<__half, kModeFused>(R, tx, ta, tb, ty, a, max_items, st);
  }
}

}  // namespace persona
