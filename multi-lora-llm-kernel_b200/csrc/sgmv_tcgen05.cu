// Segmented (SGMV) shrink / expand / fused kernels on the sm_100a tensor
// cores (tcgen05 + TMEM), for prefill batches whose rows come in long runs
// that share an adapter.
//
// Same math as the BGMV ops (reference persona/ops.py:12-56) on the rows the
// segment table assigns to each adapter: v = x A[s]^T, y += v B[s]^T.
//
// Work unit: a 128-row item of one segment (from the segment plan), one MMA
// tile high.  Per CTA (persistent over items), ten warps around one ring of
// equal shared-memory slots; per item the ring carries K/128 shrink fills
// (x chunk + A chunk) and then N/128 expand fills (y tile + B tile):
//   warp 0  TMA producer, fills the ring in that order;
//   warp 1  MMA issuer (one thread): shrink D_v[128 x R] += x_chunk A_chunk^T
//           (M = 128, N = R, K = 16 per instruction) into TMEM; expand
//           D_y[128 x 128] = V'[128 x 2R] B_tile^T into one of two TMEM
//           accumulators; completion is signalled with tcgen05.commit;
//   warps 2-5  epilogue, one thread per TMEM lane (= row): read D_v, split v
//           into 16-bit hi + lo halves (per-row power-of-two scale for f16)
//           and write them to shared memory as the expand's A operand V';
//           read D_y, add the y tile, write it back in place and TMA-store it;
//   warps 6-9  exchange (tensor parallel only): copy each finished y tile
//           from shared memory into the other ranks' y over NVLink, then
//           release the slot, so the transfer runs beside the math of the
//           next tiles instead of inside the epilogue.
// The expand multiplies B by hi and by lo, so v keeps ~fp32 precision.
// Only full items use the TMA store; a short item (segment tail) writes its
// valid rows with plain stores, so rows of the next segment are never
// touched.
#include <atomic>
#include <type_traits>

#include "bgmv_args.h"
#include "common.cuh"
#include "plan_layout.h"
#include "tcgen05.cuh"

namespace persona {

constexpr int kTcRows = 128;   // rows per item (MMA M)
constexpr int kBoxCols = 64;   // elements per 128-byte swizzled row: one TMA box is 128 rows x 64
constexpr int kBoxes = kSgmvTcTileN / kBoxCols;  // boxes per fill
constexpr int kTcNT = kSgmvTcTileN;  // expand output columns per tile (MMA N)
constexpr int kTcKC = kSgmvTcTileN;  // shrink K chunk
constexpr int kTcThreads = 10 * 32;
constexpr int kEpiBar = 1;     // named barrier of the four epilogue warps
constexpr int kXchBar = 2;     // named barrier of the four exchange warps
constexpr int kXchWarps = 4;   // warps 6-9
constexpr int kAccBufs = 256 / kTcNT;  // expand accumulators in TMEM, columns [128, 384)
constexpr int kMaxSlots = 12;
constexpr uint32_t kTmemCols = 512;
constexpr int kSmemPerBlock = 227 * 1024;  // opt-in maximum per block on sm_100

// One ring of equal slots serves both phases: a shrink fill is an x chunk
// (128 rows x kTcKC) + the A chunk (R x kTcKC); an expand fill is a y tile
// (128 rows x kTcNT) + the B tile (kTcNT x R).  x, y and A arrive as boxes
// of 64 elements (128-byte swizzled rows), several side by side per fill.
// Sharing the ring keeps ~200 KB of loads in flight in either phase.
template <int R>
struct TcCfg {
  static_assert(R == 16 || R == 32 || R == 64, "tensor-core SGMV ranks");
  static constexpr int kBoxBytes = kTcRows * 128;      // one x / y box: 16 KB
  static constexpr int kTileBytes = kBoxes * kBoxBytes;
  static constexpr int kABox = R * 128;                // one A box
  static constexpr int kABytes = kBoxes * kABox;
  static constexpr int kBBytes = kTcNT * R * 2;
  static constexpr int kSlotBytes = kTileBytes + (kABytes > kBBytes ? kABytes : kBBytes);
  // V': rows of 128 bytes [hi | lo | 0] up to rank 32; at rank 64 one
  // 128-byte-row block of hi, then one of lo.
  static constexpr int kVBytes = kTcRows * 128 * (R <= 32 ? 1 : 2);
  // byte offset of K step ks of the lo half inside V'
  __host__ __device__ static constexpr uint32_t lo_off(int ks) { return R <= 32 ? (R / 16 + ks) * 32 : kTcRows * 128 + ks * 32; }
  static constexpr int kSlots = (kSmemPerBlock - 2048 - kVBytes) / kSlotBytes < kMaxSlots
                                    ? (kSmemPerBlock - 2048 - kVBytes) / kSlotBytes
                                    : kMaxSlots;
  static constexpr int kSmem = kSlots * kSlotBytes + kVBytes;
  static constexpr uint32_t kBLayout = R == 16 ? tc::kLayoutSw32 : R == 32 ? tc::kLayoutSw64 : tc::kLayoutSw128;
  static constexpr uint32_t kBSbo = 8 * 2 * R;  // 8 rows of 2R bytes
  static_assert(kSlotBytes % 1024 == 0, "slot alignment");
  static_assert(kSlots >= 4, "ring depth");
};

struct TcBars {
  uint64_t full[kMaxSlots], empty[kMaxSlots];
  uint64_t xready[kMaxSlots];  // y tile finished in shared memory, for the store warps
  uint64_t v_ready, v_used, vsm_ready;
  uint64_t acc_full[kAccBufs], acc_empty[kAccBufs];
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort;  // set by the first wait that runs out; later waits return at once
  int fin;    // this CTA's piece of an item was the last one counted
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

// Work split (stream-K).  The launch's shrink work is the sequence of
// (item, K chunk) fills, item by item, and its expand work the sequence of
// (item, 128-column tile) fills.  Every CTA takes an equal contiguous range
// of each sequence, first its shrink range, then its expand range, so every
// SM streams the same number of bytes whatever the number and length of the
// items.  An item whose K chunks are cut between CTAs leaves one fp32 piece
// of v (128 rows x R) per CTA (a CTA's first and last item may be pieces);
// the last piece counted sums them in CTA order, so the result does not
// depend on scheduling, writes the item's v to the workspace and sets the
// item's ready word.  The expand range reads the v of each of its items
// (waiting, bounded, for the ready word) and builds V' once per item.
struct Seg {
  int item, lo, hi;  // fills [lo, hi) of the item
};

namespace {

// CTA g of `ctas` owns fills [range_start(g), range_start(g + 1)).
__device__ __forceinline__ int64_t range_start(int64_t total, int ctas, int g) {
  return static_cast<int64_t>(g) * total / ctas;
}
// The CTA whose range holds fill f.
__device__ __forceinline__ int range_cta(int64_t total, int ctas, int64_t f) {
  return static_cast<int>(((f + 1) * ctas - 1) / total);
}

__device__ __forceinline__ void st_release_gpu(int* p, int v) {
  asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Bounded spin until *p == want (acquire); gives up like tc_wait.
__device__ __forceinline__ bool tc_wait_word(const int* p, int want, int32_t* err, int* abort) {
  auto ld = [&]() {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
  };
  if (ld() == want) return true;
  const long long t0 = clock64();
  while (ld() != want) {
    if (*reinterpret_cast<volatile int*>(abort)) return false;
    if (clock64() - t0 > kWaitBudgetCycles) {
      *reinterpret_cast<volatile int*>(abort) = 1;
      raise_error(err, PERSONA_DEV_ERR_TIMEOUT);
      return false;
    }
    __nanosleep(64);
  }
  return true;
}

}  // namespace

template <typename DT, int R, int MODE>
__global__ void __launch_bounds__(kTcThreads, 1)
    sgmv_tc_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmA,
                   const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmY,
                   const SgmvTcArgs args) {
  using C = TcCfg<R>;
  constexpr int kSlots = C::kSlots;
  constexpr bool kDoShrink = (MODE & kModeShrink) != 0;
  constexpr bool kDoExpand = (MODE & kModeExpand) != 0;
  constexpr uint32_t kFmt = std::is_same<DT, __nv_bfloat16>::value ? 1u : 0u;
  constexpr uint32_t kIdescV = tc::idesc_f16(kFmt, kTcRows, R);
  constexpr uint32_t kIdescY = tc::idesc_f16(kFmt, kTcRows, kTcNT);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ring = base;
  uint8_t* vsm = ring + kSlots * C::kSlotBytes;
  __shared__ TcBars bars;

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int i = 0; i < kSlots; ++i) {
      mbar_init(&bars.full[i], 1);
      mbar_init(&bars.empty[i], 1);   // MMA commit (shrink fill), store leader (expand fill)
      mbar_init(&bars.xready[i], 4);  // one arrive per epilogue warp
    }
    mbar_init(&bars.v_ready, 1);
    mbar_init(&bars.v_used, 4);
    mbar_init(&bars.vsm_ready, 1);
    for (int b = 0; b < kAccBufs; ++b) {
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
  // The plan and the workspace's counters are written by the plan kernel
  // just before this one (launched as its programmatic dependent).
  asm volatile("griddepcontrol.wait;" ::: "memory");
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = bars.tmem_base;
  int* abort = &bars.abort;

  PlanView pv = plan_view(const_cast<int32_t*>(args.plan), args.T);
  const int n_items = pv.hdr[kHdrItems];
  const int nk = kDoShrink ? (args.K + kTcKC - 1) / kTcKC : 0;  // shrink fills per item (last may be part)
  const int nn = kDoExpand ? (args.N + kTcNT - 1) / kTcNT : 0;  // expand fills per item (last may be part)
  const int me = static_cast<int>(blockIdx.x);
  const int64_t tot_s = static_cast<int64_t>(n_items) * nk, tot_e = static_cast<int64_t>(n_items) * nn;
  // A phase with fewer fills than CTAs runs on its first tot CTAs only, so
  // that every CTA taking part has a non-empty range (the pieces of an item
  // are counted over the CTAs g0 .. g1 that hold its first and last fill).
  const int G = static_cast<int>(tot_s < static_cast<int64_t>(gridDim.x) ? tot_s : gridDim.x);
  const int Ge = static_cast<int>(tot_e < static_cast<int64_t>(gridDim.x) ? tot_e : gridDim.x);
  const int64_t s0 = me < G ? range_start(tot_s, G, me) : 0, s1 = me < G ? range_start(tot_s, G, me + 1) : 0;
  const int64_t e0 = me < Ge ? range_start(tot_e, Ge, me) : 0, e1 = me < Ge ? range_start(tot_e, Ge, me + 1) : 0;
  // Segment of this CTA's range that starts at fill f: item and fills [lo, hi).
  auto seg_at = [](int64_t f, int64_t f_end, int per) -> Seg {
    Seg s;
    s.item = static_cast<int>(f / per);
    s.lo = static_cast<int>(f - static_cast<int64_t>(s.item) * per);
    s.hi = f_end - f < per - s.lo ? s.lo + static_cast<int>(f_end - f) : per;
    return s;
  };

  if (warp == 0) {
    // ------------------------------------------------------ producer ----
    // Fills in the order every role walks them: this CTA's shrink range
    // (x chunk + A chunk), then its expand range (y tile + B tile).  Fill g
    // uses slot g % kSlots.
    if (lane == 0) {
      if (kDoShrink) {
        tma_prefetch_desc(&tmX);
        tma_prefetch_desc(&tmA);
      }
      if (kDoExpand) {
        tma_prefetch_desc(&tmY);
        tma_prefetch_desc(&tmB);
      }
      uint32_t g = 0;
      bool ok = true;
      auto next_slot = [&]() -> int {
        const int s = g % kSlots;
        if (g >= static_cast<uint32_t>(kSlots) && !tc_wait(&bars.empty[s], ((g / kSlots) - 1) & 1, args.err, abort))
          ok = false;
        return s;
      };
      for (int64_t f = s0; ok && f < s1;) {
        const Seg sg = seg_at(f, s1, nk);
        f += sg.hi - sg.lo;
        const int4 it = pv.items[sg.item];
        for (int kc = sg.lo; kc < sg.hi; ++kc, ++g) {
          const int s = next_slot();
          if (!ok) break;
          uint8_t* st = ring + s * C::kSlotBytes;
          // only boxes that start inside K are loaded (K is a multiple of 64)
          const int nb = min(kBoxes, (args.K - kc * kTcKC) / kBoxCols);
          mbar_arrive_expect_tx(&bars.full[s], nb * (C::kBoxBytes + C::kABox));
          for (int b = 0; b < nb; ++b) {
            tc::tma_load_2d(st + b * C::kBoxBytes, &tmX, &bars.full[s], kc * kTcKC + b * kBoxCols, it.y);
            tma_load_3d(st + C::kTileBytes + b * C::kABox, &tmA, &bars.full[s], kc * kTcKC + b * kBoxCols, 0, it.x);
          }
        }
      }
      for (int64_t f = e0; ok && f < e1;) {
        const Seg sg = seg_at(f, e1, nn);
        f += sg.hi - sg.lo;
        const int4 it = pv.items[sg.item];
        for (int t = sg.lo; t < sg.hi; ++t, ++g) {
          const int s = next_slot();
          if (!ok) break;
          uint8_t* st = ring + s * C::kSlotBytes;
          // only y boxes inside the column block are loaded (its width is a
          // multiple of 64); the B box reads zeros past N
          const int col = args.n0 + t * kTcNT;
          const int nb = min(kBoxes, (args.N - t * kTcNT) / kBoxCols);
          mbar_arrive_expect_tx(&bars.full[s], nb * C::kBoxBytes + C::kBBytes);
          for (int b = 0; b < nb; ++b)
            tc::tma_load_2d(st + b * C::kBoxBytes, &tmY, &bars.full[s], col + b * kBoxCols, it.y);
          tma_load_3d(st + C::kTileBytes, &tmB, &bars.full[s], 0, col, it.x);
        }
      }
      // Every load this thread issued lands before the CTA can exit: wait
      // (bounded, whatever the abort flag says) for the last fill of each
      // slot.  Earlier fills of a slot completed before it was refilled.
      for (int s = 0; s < kSlots; ++s)
        if (g > static_cast<uint32_t>(s)) {
          const uint32_t last = (g - 1 - s) / kSlots;  // use count of the slot's last fill
          mbar_wait(&bars.full[s], last & 1, args.err);
        }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ----------------------------------------------------------- MMA ----
    if (lane == 0) {
      uint32_t g = 0, nt = 0, j = 0, je = 0;
      bool ok = true;
      const uint32_t d_v = tmem;
      const uint32_t sv = smem_u32(vsm);
      for (int64_t f = s0; ok && f < s1; ++j) {
        const Seg sg = seg_at(f, s1, nk);
        f += sg.hi - sg.lo;
        if (j > 0 && !tc_wait(&bars.v_used, (j - 1) & 1, args.err, abort)) break;  // D_v of the previous segment read
        tc::fence_after_sync();
        for (int kc = sg.lo; kc < sg.hi; ++kc, ++g) {
          const int s = g % kSlots;
          if (!tc_wait(&bars.full[s], (g / kSlots) & 1, args.err, abort)) {
            ok = false;
            break;
          }
          tc::fence_after_sync();
          const uint32_t sx = smem_u32(ring + s * C::kSlotBytes);
          const int nks = min(kTcKC, args.K - kc * kTcKC) / 16;  // K steps of the boxes loaded
#pragma unroll
          for (int ks = 0; ks < kTcKC / 16; ++ks) {
            if (ks >= nks) break;
            const uint32_t box = ks / (kBoxCols / 16), in = (ks % (kBoxCols / 16)) * 32;
            const uint64_t a = tc::smem_desc(sx + box * C::kBoxBytes + in, 1024, tc::kLayoutSw128);
            const uint64_t b = tc::smem_desc(sx + C::kTileBytes + box * C::kABox + in, 1024, tc::kLayoutSw128);
            tc::mma_f16(d_v, a, b, kIdescV, (kc > sg.lo || ks > 0) ? 1u : 0u);
          }
          tc::commit(&bars.empty[s]);  // the chunk is consumed once these MMAs complete
        }
        if (!ok) break;
        tc::commit(&bars.v_ready);
      }
      for (int64_t f = e0; ok && f < e1; ++je) {
        const Seg sg = seg_at(f, e1, nn);
        f += sg.hi - sg.lo;
        if (!tc_wait(&bars.vsm_ready, je & 1, args.err, abort)) break;
        tc::fence_after_sync();
        for (int t = sg.lo; t < sg.hi; ++t, ++g, ++nt) {
          const int s = g % kSlots;
          const uint32_t buf = nt % kAccBufs;
          if (!tc_wait(&bars.full[s], (g / kSlots) & 1, args.err, abort) ||
              (nt >= kAccBufs && !tc_wait(&bars.acc_empty[buf], ((nt / kAccBufs) - 1) & 1, args.err, abort))) {
            ok = false;
            break;
          }
          tc::fence_after_sync();
          const uint32_t sb = smem_u32(ring + s * C::kSlotBytes + C::kTileBytes);
          const uint32_t d_y = tmem + 128u + kTcNT * buf;
#pragma unroll
          for (int ks = 0; ks < R / 16; ++ks) {
            const uint64_t b = tc::smem_desc(sb + ks * 32, C::kBSbo, C::kBLayout);
            tc::mma_f16(d_y, tc::smem_desc(sv + ks * 32, 1024, tc::kLayoutSw128), b, kIdescY, ks > 0 ? 1u : 0u);
            tc::mma_f16(d_y, tc::smem_desc(sv + C::lo_off(ks), 1024, tc::kLayoutSw128), b, kIdescY, 1u);
          }
          tc::commit(&bars.acc_full[buf]);  // the epilogue releases the slot (it also holds the y tile)
        }
      }
      // All MMAs this thread issued complete before TMEM is released.
      tc::commit(&bars.mma_done);
      mbar_wait(&bars.mma_done, 0, args.err);
    }
    __syncwarp();
  } else if (warp < 6) {
    // ------------------------------------------------------ epilogue ----
    // Every epilogue thread walks the same segments to the end, so the
    // named barriers stay matched; after an abort the waits return at once
    // and nothing more is written to global memory.
    const int quarter = warp & 3;          // TMEM lanes this warp may access
    const int row = quarter * 32 + lane;   // row of the item this thread owns
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    const int ew = warp - 2;
    uint32_t g = 0, nt = 0, j = 0, je = 0;
    int* const cnt = args.item_cnt;
    int* const ready = args.item_ready;
    for (int64_t f = s0; f < s1; ++j) {
      // ---- shrink segment: D_v -> the item's v, or a piece of it
      const Seg sg = seg_at(f, s1, nk);
      f += sg.hi - sg.lo;
      g += sg.hi - sg.lo;  // the MMA warp releases shrink fills
      const int4 it = pv.items[sg.item];
      const int row0 = it.y, count = it.z;
      const bool valid = row < count;
      const int64_t grow = static_cast<int64_t>(row0) + row;
      tc_wait(&bars.v_ready, j & 1, args.err, abort);
      __syncwarp();
      tc::fence_after_sync();
      float v[R];
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
      const bool live = !*reinterpret_cast<volatile int*>(abort);
      bool final_v = sg.lo == 0 && sg.hi == nk;  // the whole item in this CTA's range
      if (!final_v) {
        // A piece: CTA me holds it as its first (slot 0) or last (slot 1).
        const int64_t t0 = static_cast<int64_t>(sg.item) * nk;
        const int slot = s0 >= t0 ? 0 : 1;
        float* piece = args.pieces + (static_cast<int64_t>(me) * 2 + slot) * (kTcRows * R);
#pragma unroll
        for (int i = 0; i < R; i += 4)
          *reinterpret_cast<float4*>(piece + row * R + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
        named_sync(kEpiBar, 128);
        const int g0 = range_cta(tot_s, G, t0), g1 = range_cta(tot_s, G, t0 + nk - 1);
        if (tid == 64) {  // epilogue thread 0
          __threadfence();
          bars.fin = live && atomicAdd(cnt + sg.item, 1) == g1 - g0;
          if (bars.fin) __threadfence();  // acquire side: the other CTAs' pieces
        }
        named_sync(kEpiBar, 128);
        final_v = *reinterpret_cast<volatile int*>(&bars.fin) != 0;
        if (final_v) {
          // sum the pieces in CTA order, so the result does not depend on
          // which CTA finished last
#pragma unroll
          for (int i = 0; i < R; ++i) v[i] = 0.f;
          for (int q = g0; q <= g1; ++q) {
            const int qs = range_start(tot_s, G, q) >= t0 ? 0 : 1;
            const float* pq = args.pieces + (static_cast<int64_t>(q) * 2 + qs) * (kTcRows * R) + row * R;
#pragma unroll
            for (int i = 0; i < R; i += 4) {
              const float4 w = __ldcg(reinterpret_cast<const float4*>(pq + i));
              v[i] += w.x;
              v[i + 1] += w.y;
              v[i + 2] += w.z;
              v[i + 3] += w.w;
            }
          }
        }
      }
      // final_v is the same in every epilogue thread (bars.fin is read after
      // the barrier), so the barrier below is always matched; `live` (this
      // thread's view of the abort flag) only gates stores
      if (final_v) {
        float* dst = MODE == kModeShrink ? args.v_out : args.vfin;
        if (valid && live) {
#pragma unroll
          for (int i = 0; i < R; i += 4)
            *reinterpret_cast<float4*>(dst + grow * R + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
        }
        if (MODE != kModeShrink) {
          named_sync(kEpiBar, 128);
          if (tid == 64 && live) {
            __threadfence();
            st_release_gpu(ready + sg.item, 1);
          }
        }
      }
    }
    for (int64_t f = e0; f < e1; ++je) {
      // ---- expand segment: V' of the item once, then its tiles
      const Seg sg = seg_at(f, e1, nn);
      f += sg.hi - sg.lo;
      const int4 it = pv.items[sg.item];
      const int row0 = it.y, count = it.z;
      const bool valid = row < count;
      const int64_t grow = static_cast<int64_t>(row0) + row;
      const float* vsrc = args.v_in;
      if (MODE == kModeFused) {
        // the item's v is complete once its ready word is set
        if (tid == 64) tc_wait_word(ready + sg.item, 1, args.err, abort);
        named_sync(kEpiBar, 128);
        vsrc = args.vfin;
      }
      float v[R];
#pragma unroll
      for (int i = 0; i < R; i += 4) {
        const float4 q = valid ? __ldcg(reinterpret_cast<const float4*>(vsrc + grow * R + i)) : make_float4(0, 0, 0, 0);
        v[i] = q.x;
        v[i + 1] = q.y;
        v[i + 2] = q.z;
        v[i + 3] = q.w;
      }
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
      // V' as 16-bit, 128-byte swizzled rows: [hi(R) | lo(R) | zeros] up to
      // rank 32; at rank 64 a block of hi rows, then a block of lo rows.
      auto store_row = [&](uint32_t vrow, const uint32_t* w) {
#pragma unroll
        for (int c = 0; c < 8; ++c)
          asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(vrow + ((c ^ (row & 7)) << 4)),
                       "r"(w[4 * c]), "r"(w[4 * c + 1]), "r"(w[4 * c + 2]), "r"(w[4 * c + 3])
                       : "memory");
      };
      if constexpr (R <= 32) {
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
        store_row(smem_u32(vsm) + row * 128, w);
      } else {
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint32_t w[32];
#pragma unroll
          for (int i = 0; i < R; i += 2) {
            const float a = v[i] * scale_down, b = v[i + 1] * scale_down;
            const float ha = Mma<DT>::round_trip(a), hb = Mma<DT>::round_trip(b);
            w[i / 2] = half == 0 ? Mma<DT>::pack(ha, hb) : Mma<DT>::pack(a - ha, b - hb);
          }
          store_row(smem_u32(vsm) + half * (kTcRows * 128) + row * 128, w);
        }
      }
      tc::fence_proxy_async();
      named_sync(kEpiBar, 128);
      if (ew == 0 && lane == 0) mbar_arrive(&bars.vsm_ready);

      for (int t = sg.lo; t < sg.hi; ++t, ++g, ++nt) {
        const int s = g % kSlots;
        const uint32_t buf = nt % kAccBufs;
        tc_wait(&bars.full[s], (g / kSlots) & 1, args.err, abort);
        tc_wait(&bars.acc_full[buf], (nt / kAccBufs) & 1, args.err, abort);
        __syncwarp();
        tc::fence_after_sync();
        const bool live = !*reinterpret_cast<volatile int*>(abort);
        uint8_t* st = ring + s * C::kSlotBytes;
        const uint32_t ybase = smem_u32(st);
        const int64_t col = args.n0 + t * kTcNT;
        // boxes of this tile inside the column block (N is a multiple of 64)
        const int nbox = min(kBoxes, (args.N - t * kTcNT) / kBoxCols);
#pragma unroll
        for (int c32 = 0; c32 < kTcNT / 32; ++c32) {
          uint32_t d0[16], d1[16];
          tc::ld16(tmem + lane_addr + 128u + kTcNT * buf + 32 * c32, d0);
          tc::ld16(tmem + lane_addr + 128u + kTcNT * buf + 32 * c32 + 16, d1);
          tc::wait_ld();
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) {  // 8-column chunks of this 32-column group
            const int chunk = c32 * 4 + cc;  // 16-byte chunk of the row
            const int box = chunk >> 3, cb = chunk & 7;
            const uint32_t addr = ybase + box * C::kBoxBytes + row * 128 + ((cb ^ (row & 7)) << 4);
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
            if (box >= nbox) {
              // outside the column block: neither written back nor stored
            } else if (count == kTcRows) {
              asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(out.x), "r"(out.y),
                           "r"(out.z), "r"(out.w)
                           : "memory");
            } else if (valid && live) {
              const int64_t off = grow * args.ldy + col + chunk * 8;
              *reinterpret_cast<uint4*>(args.y + off) = out;
              for (int q = 0; q < args.num_peers; ++q) *reinterpret_cast<uint4*>(args.peers[q] + off) = out;
            }
          }
        }
        tc::fence_before_sync();
        if (count == kTcRows) tc::fence_proxy_async();  // this warp's rows, for the TMA store
        __syncwarp();
        // The warps go on to the next tile independently; the store warp
        // takes the tile once all four have arrived.
        if (lane == 0) {
          mbar_arrive(&bars.acc_empty[buf]);
          mbar_arrive(&bars.xready[s]);
        }
      }
      // the next segment rewrites V': every MMA that reads it has completed
      // (each tile's accumulator was waited for above)
      named_sync(kEpiBar, 128);
    }
    // Plain stores into the peers' y (short items) are ordered before
    // whatever this thread's kernel completion is followed by.
    if (args.num_peers > 0) __threadfence_system();
  } else if (args.num_peers > 0 || warp == 6) {
    // ------------------------------------------------ store / exchange ----
    // Warp 6 lane 0 TMA-stores each finished full tile from its slot, waits
    // until the store has read the slot and releases it, so the epilogue
    // never waits on a store.  Tensor parallel: warps 6-9 also copy the tile
    // into every other rank's y over NVLink, 128 contiguous bytes per row
    // and box (rows of a short item were stored by the epilogue itself).
    const int xw = warp - 6;
    const bool tp = args.num_peers > 0;
    const bool leader = xw == 0 && lane == 0;
    bool stored = false;
    uint32_t g = static_cast<uint32_t>(s1 - s0), xphase = 0;  // bit s: parity of the next xready[s] phase
    for (int64_t f = e0; f < e1;) {
      const Seg sg = seg_at(f, e1, nn);
      f += sg.hi - sg.lo;
      const int4 it = pv.items[sg.item];
      const int row0 = it.y, count = it.z;
      for (int t = sg.lo; t < sg.hi; ++t, ++g) {
        const int s = g % kSlots;
        const bool ok = tc_wait(&bars.xready[s], (xphase >> s) & 1u, args.err, abort);
        xphase ^= 1u << s;
        tc::fence_after_sync();
        const bool full_live = ok && count == kTcRows && !*reinterpret_cast<volatile int*>(abort);
        const uint32_t ybase = smem_u32(ring + s * C::kSlotBytes);
        const int64_t col = args.n0 + t * kTcNT;
        const int nbox = min(kBoxes, (args.N - t * kTcNT) / kBoxCols);
        if (leader && full_live) {
          for (int b = 0; b < nbox; ++b)
            tc::tma_store_2d(&tmY, ring + s * C::kSlotBytes + b * C::kBoxBytes, static_cast<int>(col) + b * kBoxCols,
                             row0);
          tc::bulk_commit();
          stored = true;
        }
        if (tp && full_live) {
          for (int b = 0; b < nbox; ++b) {
#pragma unroll
            for (int i = 0; i < (kTcRows * 8) / (kXchWarps * 32); ++i) {
              const int idx = (xw * 32 + lane) + i * (kXchWarps * 32);
              const int r = idx >> 3, c16 = idx & 7;
              const uint4 val = lds128(ybase + b * C::kBoxBytes + r * 128 + ((c16 ^ (r & 7)) << 4));
              const int64_t off = (static_cast<int64_t>(row0) + r) * args.ldy + col + b * kBoxCols + c16 * 8;
              for (int q = 0; q < args.num_peers; ++q) *reinterpret_cast<uint4*>(args.peers[q] + off) = val;
            }
          }
        }
        if (leader && full_live) tc::bulk_wait_read0();
        if (tp)
          named_sync(kXchBar, kXchWarps * 32);
        else
          __syncwarp();
        if (leader) mbar_arrive(&bars.empty[s]);
      }
    }
    if (stored) tc::bulk_wait0();
    if (tp) __threadfence_system();
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
  // per instantiation and device: SM count once the smem attribute is set
  // (racing first calls store the same value)
  static std::atomic<int> sms[kMaxDev];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDev) return cudaErrorInvalidDevice;
  const int smem = TcCfg<R>::kSmem + 1024;
  int n = sms[dev].load(std::memory_order_acquire);
  if (n == 0) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    e = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    sms[dev].store(n, std::memory_order_release);
  }
  (void)max_items;
  // one CTA per SM (at most kSgmvMaxCtas, the pieces region's size), each
  // with an equal share of the launch's fills
  const int grid = n < kSgmvMaxCtas ? n : kSgmvMaxCtas;
  // programmatic dependent of the plan kernel: TMEM and barriers are set up
  // while the plan is built
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kern, tx, ta, tb, ty, a);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

template <typename DT, int MODE>
static cudaError_t tc_rank(int R, const CUtensorMap& tx, const CUtensorMap& ta, const CUtensorMap& tb,
                           const CUtensorMap& ty, const SgmvTcArgs& a, int max_items, cudaStream_t st) {
  return R == 16   ? tc_launch<DT, 16, MODE>(tx, ta, tb, ty, a, max_items, st)
         : R == 32 ? tc_launch<DT, 32, MODE>(tx, ta, tb, ty, a, max_items, st)
                   : tc_launch<DT, 64, MODE>(tx, ta, tb, ty, a, max_items, st);
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
