// Split BGMV kernels for B200 (sm_100a): shrink, expand and fused
// shrink->expand over a row-grouping plan, for one projection or for up to
// kMaxProblems projections that share the batch's slots (one decoder layer's
// q/k/v/o/gate/up/down), with every item's work cut into slices that every
// pipeline of the GPU can take.
//
// Work units.  A plan item is one adapter slot and up to 16 rows that use it.
// For each problem its shrink is cut into nks K-slices and its expand into
// nes N-slices; the unit list is [all shrink slices, problem by problem,
// item by item] then [all expand slices, same order].  Slice counts are
// chosen on the device from the item count so that each pipeline gets 8
// (few items) to 24 (many items: items / 4) units, none shorter than about
// kMinUnitStages (one problem: kMinUnitStagesOne) stages on average: a
// decode batch of 8 adapters spreads over the whole GPU, a batch of ~150
// adapters leaves no pipeline streaming a second whole adapter while others
// idle, and the seven projections of a layer fill each other's tails.
//
// Scheduling.  Persistent pipelines claim units in list order from a
// device-wide counter.  Every shrink unit precedes every expand unit in claim
// order, so a pipeline that waits for an item's v only waits on shrink units
// that running pipelines have already claimed: the kernel always makes
// progress, even when not all CTAs are resident.
//
// Partial v.  A shrink slice writes its partial v (16 rows x R, fp32) to the
// workspace (L2-resident).  The pipeline that completes an item's last slice
// (per-item counter) sums the partials in slice order -- so the result does
// not depend on which pipeline ran what -- writes v, and releases the item by
// storing the launch's epoch into its ready word.  Expand slices wait for
// that word (bounded), read v, and stream B and y.  The epoch (bumped by the
// last CTA of every launch) makes stale ready words from earlier launches
// harmless, and the last CTA also resets the claim counter.
//
// Inside a CTA.  Kernels that allocate tensor memory run one CTA per SM, so
// each CTA carries kGroups independent pipelines of six warps: a producer
// warp (TMA boxes of A / B, 1-D bulk copies of the x / y / v rows) feeding a
// 4-slot ring, four consumer warps that
// run the shrink stages on the 16-row warp-MMA tiles of bgmv_stages.cuh, and
// an MMA warp.  For ranks 16 / 32 / 64 the expand runs on the tensor cores:
// the item's rows are the N = 16 side of a tcgen05 MMA whose M = 128 side is
// a TMA-loaded B tile, so the MMA warp turns a stage into D[128 output
// columns][16 rows] in tensor memory with 2 * R / 16 instructions (v split
// into 16-bit hi and lo halves, both small swizzled shared-memory operands),
// and a consumer thread per output column reads its 16 accumulators, adds y
// and stores.  Rank 8 keeps the warp-MMA expand.
#include <atomic>

#include "bgmv_stages.cuh"
#include "tcgen05.cuh"


namespace persona {

namespace {

constexpr int kUnitRing = 4;
// Units per pipeline: items / kItemsPerUnitStep, between these bounds.
// Measured on 7-projection launches: 128 rows over 8 adapters 65.8 us at 8
// units (67.0 at 12); an 8-GPU rank's 51 items 146.5 us at 12 (150.5 at 8);
// the 1-GPU batch's 139 items best at 24.
constexpr int kUnitsPerCta = 8;       // units per pipeline, few items
constexpr int kUnitsPerCtaMany = 24;  // units per pipeline, many items
constexpr int kItemsPerUnitStep = 4;
// An item's units average at least this many stages (launches of several
// problems / of one problem).  Without a floor a launch with few items per
// pipeline (one projection of a 512-row batch: 139 items for 296 pipelines)
// cut gate's expand into 4-stage units, each paying a unit's start.
// Measured on that batch: the 7-projection launch takes 286.0 us with a
// floor of 16 (288.5 with 8 or none); the seven projections launched one at
// a time take 498.7 us in all with 8, 519.5 with 16, 565.5 with none.  A
// launch of several problems drops the floor when it would leave fewer than
// kMinUnitsPerPipe units per pipeline: the shard of one of 8 GPUs (51 items,
// already sliced coarsely) took 158.8 us with the floor and 150.7 without
// it, while a shard of one of 4 GPUs (70 items) took 173.3 with it and 179.0
// without.
constexpr int kMinUnitStages = 16;
constexpr int kMinUnitStagesOne = 8;
constexpr int kMinUnitsPerPipe = 8;
enum : int { kUnitEnd = 0, kUnitShrink = 1, kUnitExpand = 2 };

constexpr int kGroups = 2;
constexpr int kGroupThreads = kBgmvThreads + 32;  // + one MMA warp
constexpr int kSplitThreads = kGroups * kGroupThreads;
constexpr int kMmaWarp = kConsumerWarps + 1;
constexpr uint32_t kGroupTmemCols = 128;  // one 16-column accumulator per (ring slot, 128-row box)
constexpr uint32_t kTmemCols = kGroups * kGroupTmemCols;

struct UnitDesc {
  int kind;
  int prob;
  int item;
  int slice;
  int slot;
  int count;
  int pos;  // plan position of the item's first row
  int pad;
  int rows[kRowsPerItem];
};

// Slice geometry of one problem; identical in every thread of every CTA.
struct ProbGeom {
  int kst, nst;      // A stages over K, B stages over N
  int ks_st, es_st;  // stages per shrink / expand slice
  int nks, nes;      // slices per item
  int stage_rows;    // output columns per B stage
  int s_base;        // first shrink unit of this problem
  int e_base;        // first expand unit of this problem
  int p_base;        // first partial-v slot of this problem
};

struct SplitShared {
  ProbGeom geom[kMaxProblems];
  int sorder[kMaxProblems], eorder[kMaxProblems];  // problems in claim order (longest units first)
  int units_s, units;
  int first[kGroups];  // each pipeline's first claimed unit
  uint32_t tmem;
  int abort;  // set by the first wait of the CTA that gives up
};

constexpr int kSRingBytes = kSlots * kSlotBytes;
constexpr int kSVopBytes = 2 * kRowsPerItem * kMaxR * 2;  // v hi / lo MMA operands, 16 rows x R each
constexpr int kSVBytes = kRowsPerItem * kMaxR * 4;
constexpr int kSRedBytes = kRowsPerItem * kMaxR * 4;
constexpr int kSUnitBytes = kUnitRing * static_cast<int>(sizeof(UnitDesc));
constexpr int kSBarCount = 3 * kSlots + 2 * kUnitRing + 2 + 4;
constexpr int kGroupSmemRaw =
    kSRingBytes + kSVopBytes + 4 * kSVBytes + kSRedBytes + kSUnitBytes + kSBarCount * 8 + 16;
constexpr int kGroupSmem = (kGroupSmemRaw + 1023) / 1024 * 1024;
constexpr int kSplitSmemBytes = kGroups * kGroupSmem + 1024;
static_assert(kSplitSmemBytes <= 227 * 1024, "one CTA per SM");

struct SplitSmem {
  uint8_t* ring;
  uint8_t* vop;  // [hi | lo] expand operands (1024-aligned)
  float* pv;     // [16][R] this unit's partial / the item's v
  float* vf;     // [16][R] the item's v for the expand (separate expand op)
  float* vbuf;   // [2][16][R] the items' v of the next fused expand units, copied in by the producer
  float* red;    // per-warp MMA tiles / maxima
  UnitDesc* units;
  uint64_t* full;
  uint64_t* empty;
  uint64_t* ufull;
  uint64_t* uempty;
  uint64_t* mma_done;  // [kSlots] expand MMAs of the slot's stage complete
  uint64_t* vready;    // the expand unit's v operands are in shared memory
  uint64_t* mma_fin;   // every MMA of the pipeline complete (before TMEM is freed)
  uint64_t* vfull;     // [2] vbuf[b] has landed
  uint64_t* vempty;    // [2] the consumers are done with vbuf[b]
  int* flag;
};

__device__ __forceinline__ SplitSmem carve(uint8_t* raw, int grp) {
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023)) +
                  grp * kGroupSmem;
  SplitSmem p;
  p.ring = base;
  p.vop = base + kSRingBytes;
  uint8_t* q = base + kSRingBytes + kSVopBytes;
  p.pv = reinterpret_cast<float*>(q);
  p.vf = reinterpret_cast<float*>(q + kSVBytes);
  p.vbuf = reinterpret_cast<float*>(q + 2 * kSVBytes);
  p.red = reinterpret_cast<float*>(q + 4 * kSVBytes);
  p.units = reinterpret_cast<UnitDesc*>(q + 4 * kSVBytes + kSRedBytes);
  uint64_t* bars = reinterpret_cast<uint64_t*>(q + 4 * kSVBytes + kSRedBytes + kSUnitBytes);
  p.full = bars;
  p.empty = bars + kSlots;
  p.ufull = bars + 2 * kSlots;
  p.uempty = bars + 2 * kSlots + kUnitRing;
  p.mma_done = bars + 2 * kSlots + 2 * kUnitRing;
  p.vready = p.mma_done + kSlots;
  p.mma_fin = p.vready + 1;
  p.vfull = p.mma_fin + 1;
  p.vempty = p.vfull + 2;
  p.flag = reinterpret_cast<int*>(bars + kSBarCount);
  return p;
}

// Slice counts for every problem: about units_per_cta units per pipeline in
// total, shared between the problems by their stage counts and, within a
// problem, between shrink and expand by theirs.  Run by one warp, lane p for
// problem p (the divisions of all problems run side by side: done by one
// thread they took 5 us at the start of every launch of seven problems).
__device__ __noinline__ void plan_units(SplitShared& sh, int K, int N, int n_box, int P, int units_per_cta,
                                        int n_items, int kc, int nb_rows, int pipes, bool shrink, bool expand,
                                        int lane) {
  const int items = n_items > 0 ? n_items : 1;
  // Many items (large batches): small units, so the tail stays short.  Few
  // items (decode): fewer, larger units, so the latency chain shrink slice ->
  // finisher -> expand slice has fewer links per item.
  const int upc = units_per_cta > 0 ? units_per_cta
                                    : min(kUnitsPerCtaMany, max(kUnitsPerCta, n_items / kItemsPerUnitStep));
  const bool mine = lane < P;
  int kst = 0, nst = 0, stage_rows = 0;
  if (mine) {
    stage_rows = (nb_rows / n_box) * n_box;
    kst = shrink ? (K + kc - 1) / kc : 0;
    nst = expand ? (N + stage_rows - 1) / stage_rows : 0;
  }
  int work = kst + nst;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) work += __shfl_xor_sync(0xffffffffu, work, off);
  int ks_st = 0, es_st = 0, nks = 0, nes = 0;
  int per_item = 1, per_floor = 1;
  if (mine) {
    const long long budget = static_cast<long long>(upc) * pipes * (kst + nst) / (work > 0 ? work : 1);
    const int min_st = P > 1 ? kMinUnitStages : kMinUnitStagesOne;
    per_item = max(1, static_cast<int>((budget + items - 1) / items));
    per_floor = max(1, min(per_item, (kst + nst) / min_st));
  }
  // units the floor would leave, over all problems
  long long u_floor = mine ? static_cast<long long>(n_items) * per_floor : 0;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) u_floor += __shfl_xor_sync(0xffffffffu, u_floor, off);
  if (P == 1 || u_floor >= static_cast<long long>(kMinUnitsPerPipe) * pipes) per_item = per_floor;
  if (mine) {
    int n1 = 1, n2 = 1;
    if (shrink && expand) {
      n1 = max(1, (per_item * kst + (kst + nst) / 2) / max(1, kst + nst));
      n2 = max(1, per_item - n1);
    } else if (shrink) {
      n1 = per_item;
    } else {
      n2 = per_item;
    }
    n1 = min(min(n1, max(1, kst)), max(1, kPartSlots / (items * P)));
    n2 = min(n2, max(1, nst));
    ks_st = shrink ? (kst + n1 - 1) / n1 : 0;
    nks = shrink ? (kst + ks_st - 1) / ks_st : 0;
    es_st = expand ? (nst + n2 - 1) / n2 : 0;
    nes = expand ? (nst + es_st - 1) / es_st : 0;
  }
  // Claim order inside each phase: problem by problem, the same order in
  // both phases, so an expand unit's item was shrunk long before (ordering
  // the phases by unit length instead made the first expand units wait for
  // the last shrink units: 356 against 306 us per launch).  Unit bases are
  // prefix sums over the lanes.
  const int s_cnt = mine ? n_items * nks : 0, e_cnt = mine ? n_items * nes : 0;
  int s_inc = s_cnt, e_inc = e_cnt;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int ts = __shfl_up_sync(0xffffffffu, s_inc, off), te = __shfl_up_sync(0xffffffffu, e_inc, off);
    if (lane >= off) {
      s_inc += ts;
      e_inc += te;
    }
  }
  const int s_units = __shfl_sync(0xffffffffu, s_inc, 31), e_units = __shfl_sync(0xffffffffu, e_inc, 31);
  if (mine) {
    ProbGeom& g = sh.geom[lane];
    g.kst = kst;
    g.nst = nst;
    g.stage_rows = stage_rows;
    g.ks_st = ks_st;
    g.nks = nks;
    g.es_st = es_st;
    g.nes = nes;
    g.s_base = s_inc - s_cnt;
    g.p_base = g.s_base;  // partial slots follow the shrink units one to one
    g.e_base = s_units + e_inc - e_cnt;
    sh.sorder[lane] = sh.eorder[lane] = lane;
  }
  if (lane == 0) {
    sh.units_s = s_units;
    sh.units = s_units + e_units;
  }
}

__device__ __forceinline__ void sts16(uint32_t addr, uint16_t v) {
  asm volatile("st.shared.u16 [%0], %1;" ::"r"(addr), "h"(v) : "memory");
}
__device__ __forceinline__ void sts32(uint32_t addr, uint32_t v) {
  asm volatile("st.shared.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}

__device__ __forceinline__ int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ int ld_relaxed(const int* p) {
  int v;
  asm volatile("ld.relaxed.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Orders this thread's generic-proxy global accesses with async-proxy (bulk
// copy) accesses of the same memory.
__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }
__device__ __forceinline__ void st_release(int* p, int v) {
  asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Spin (bounded) until *p == want.  False if it never does (timeout bit,
// CTA abort flag and the launch's abort word set) or if the CTA or the
// launch has already given up.
__device__ __forceinline__ bool wait_word(const int* p, int want, int32_t* err, int* abort, int* launch_abort) {
  if (ld_acquire(p) == want) return true;
  volatile int* ab = abort;
  const long long t0 = clock64();
  while (ld_acquire(p) != want) {
    if (*ab || ld_acquire(launch_abort) != 0) {
      *ab = 1;
      return false;
    }
    if (clock64() - t0 > kWaitBudgetCycles) {
      *ab = 1;
      atomicExch(launch_abort, 1);
      raise_error(err, PERSONA_DEV_ERR_TIMEOUT);
      return false;
    }
    __nanosleep(64);
  }
  return true;
}

}  // namespace

// Failure handling.  Every wait is bounded and, through sh.abort, gives up
// at once after any wait of the CTA gave up.  Roles leave their loops at a
// unit boundary (the consumers decide together, so that their named
// barriers stay matched); a stage whose wait failed is still walked through
// but its slot is not released, so the producer never re-arms a slot whose
// loads may still be landing.  The producer waits (bounded) for its own
// loads before the CTA exits, and the MMA warp for its own MMAs before the
// tensor memory is freed.
template <typename DT, int R, int MODE>
__global__ void __launch_bounds__(kSplitThreads, 1)
    bgmv_split_kernel(const __grid_constant__ SplitMaps maps, const SplitArgs args) {
  using C = RankCfg<R>;
  constexpr bool kDoShrink = (MODE & kModeShrink) != 0;
  constexpr bool kDoExpand = (MODE & kModeExpand) != 0;
  constexpr bool kTcE = kDoExpand && R >= 16;  // expand on tcgen05
  // expand MMA operands: K-major rows of 2R bytes, swizzled over 2R bytes
  constexpr uint32_t kOpLayout = R >= 64 ? tc::kLayoutSw128 : R == 32 ? tc::kLayoutSw64 : tc::kLayoutSw32;
  constexpr uint32_t kOpSbo = 8 * 2 * R;
  constexpr uint32_t kIdesc = tc::idesc_f16(std::is_same<DT, __nv_bfloat16>::value ? 1u : 0u, 128, kRowsPerItem);
  extern __shared__ uint8_t smem_raw[];
  __shared__ SplitShared sh;
  const int grp = static_cast<int>(threadIdx.x) / kGroupThreads;  // pipeline of this thread
  const int tid = static_cast<int>(threadIdx.x) - grp * kGroupThreads;
  const int warp = tid >> 5, lane = tid & 31;
  const int bar_cons = kNamedBarConsumers + grp;  // named barrier of this group's consumers
  SplitSmem sm = carve(smem_raw, grp);

  PlanView pv = plan_view(args.ws, args.T);
  const int P = args.num_problems;
  WorkView wv = work_view(args.ws, args.T, P);
  const int64_t tpad = plan_tpad(args.T);

  // Prologue that touches no input: it may overlap the kernel before this
  // one (launched as its programmatic dependent; normally the plan kernel).
  if (tid == 0) {
    for (int s = 0; s < kSlots; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], kConsumerWarps);
      mbar_init(&sm.mma_done[s], 1);
    }
    for (int i = 0; i < kUnitRing; ++i) {
      mbar_init(&sm.ufull[i], 1);
      mbar_init(&sm.uempty[i], kConsumerWarps + 1);  // consumers + the MMA warp
    }
    mbar_init(sm.vready, 1);
    mbar_init(sm.mma_fin, 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sm.vfull[b], 1);
      mbar_init(&sm.vempty[b], 1);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kConsumerWarps && lane < P) {
    if (kDoShrink) tma_prefetch_desc(&maps.a[lane]);
    if (kDoExpand) tma_prefetch_desc(&maps.b[lane]);
  }
  if (kTcE && grp == 0 && warp == kMmaWarp) {  // one allocation for both groups
    tc::tmem_alloc(&sh.tmem, kTmemCols);
    tc::tmem_relinquish();
  }
  // The plan, x, y and the shared counters may be written by the kernel
  // before this one: nothing below reads them before it has completed.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // With PERSONA_REUSE_PLAN the workspace is trusted only if its header is
  // the plan of this T and S; every CTA reads the same header, so they all
  // take the same branch.
  const int n_items = pv.hdr[kHdrItems];
  const bool plan_ok = pv.hdr[kHdrMagic] == kPlanMagic && pv.hdr[kHdrT] == args.T && pv.hdr[kHdrS] == args.S &&
                       pv.hdr[kHdrRowsPerItem] == kRowsPerItem && n_items >= 0 && n_items <= tpad;
  const int epoch = wv.sync[kSyncEpoch];
  // Each producer's first claim goes out now; its round trip overlaps the
  // unit geometry below.
  if (plan_ok && warp == kConsumerWarps && lane == 0) sh.first[grp] = atomicAdd(&wv.sync[kSyncQueue], 1);
  if (threadIdx.x < 32) {
    if (plan_ok) {
      // lane p takes problem p's sizes (constant indices: no local copy of the arguments)
      int pk = 0, pn = 0, pb = 1;
#pragma unroll
      for (int q = 0; q < kMaxProblems; ++q) {
        if (static_cast<int>(threadIdx.x) == q && q < P) {
          pk = args.prob[q].K;
          pn = args.prob[q].N;
          pb = args.prob[q].n_box;
        }
      }
      plan_units(sh, pk, pn, pb, P, args.units_per_cta, n_items, C::kKC, C::kNB,
                 static_cast<int>(gridDim.x) * kGroups, kDoShrink, kDoExpand, static_cast<int>(threadIdx.x));
    } else if (threadIdx.x == 0) {
      sh.units_s = sh.units = 0;
      if (blockIdx.x == 0) raise_error(args.err, PERSONA_DEV_ERR_PLAN);
    }
    if (threadIdx.x == 0) sh.abort = 0;
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = sh.tmem + static_cast<uint32_t>(grp) * kGroupTmemCols;
  const int units_s = sh.units_s, units = sh.units;
  int* const abort = &sh.abort;

  // Unit u -> (kind, problem, item, slice); [lo, hi) is the k range of a
  // shrink slice or the n range of an expand slice.
  struct Dec {
    int kind, prob, item, slice, lo, hi;
  };
  auto decode = [&](int u) -> Dec {
    Dec d;
    d.kind = kUnitEnd;
    d.prob = d.item = d.slice = d.lo = d.hi = 0;
    if (u >= units) return d;
    if (u < units_s) {
      int p = sh.sorder[0];
      for (int q = 1; q < P && sh.geom[sh.sorder[q]].s_base <= u; ++q) p = sh.sorder[q];
      const ProbGeom& gg = sh.geom[p];
      const int v = u - gg.s_base;
      d.kind = kUnitShrink;
      d.prob = p;
      d.item = v / gg.nks;
      d.slice = v - d.item * gg.nks;
      d.lo = d.slice * gg.ks_st * C::kKC;
      d.hi = min(args.prob[p].K, d.lo + gg.ks_st * C::kKC);
    } else {
      int p = sh.eorder[0];
      for (int q = 1; q < P && sh.geom[sh.eorder[q]].e_base <= u; ++q) p = sh.eorder[q];
      const ProbGeom& gg = sh.geom[p];
      const int v = u - gg.e_base;
      d.kind = kUnitExpand;
      d.prob = p;
      d.item = v / gg.nes;
      d.slice = v - d.item * gg.nes;
      d.lo = d.slice * gg.es_st * gg.stage_rows;
      d.hi = min(args.prob[p].N, d.lo + gg.es_st * gg.stage_rows);
    }
    return d;
  };

  if (!plan_ok) {
    // nothing to do; fall through to the teardown (no counter is touched)
  } else if (warp == kConsumerWarps) {
    // ------------------------------------------------------- producer --
    // Claims run two units ahead: the atomic for unit j+2 is issued while
    // unit j streams and its result is first read one unit later, so the
    // round trip to L2 never stalls the loads.  The kernel issues no L2
    // prefetch: with the whole GPU streaming, prefetched lines were evicted
    // before use and prefetching a unit ahead cost up to 25% of the
    // throughput (measured: 3.53 TB/s with whole units two ahead, 4.33 with
    // six stages, 4.75 with none).
    auto claim_issue = [&]() -> int { return lane == 0 ? atomicAdd(&wv.sync[kSyncQueue], 1) : 0; };
    auto claim_read = [&](int pending) -> int { return __shfl_sync(0xffffffffu, pending, 0); };
    uint32_t g = 0;
    // Arms the next ring slot for `bytes`; -1 if its wait gave up (the slot
    // is then left alone).  A slot is only ever released by consumers whose
    // own wait for its loads succeeded, so a completed empty wait means the
    // slot's previous loads have landed and re-arming it is safe.
    auto claim_slot = [&](uint32_t bytes) -> int {
      const int s = static_cast<int>(g % kSlots);
      int ok = 1;
      if (lane == 0) {
        if (g >= kSlots) ok = mbar_wait_abortable(&sm.empty[s], ((g / kSlots) - 1) & 1, args.err, abort) ? 1 : 0;
        if (ok) mbar_arrive_expect_tx(&sm.full[s], bytes);
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      return ok ? s : -1;
    };
    // A plan item is used only if it lies inside the plan: one from the plan
    // kernels always does; a damaged one becomes a no-op unit (no rows)
    // instead of an access out of range.
    auto item_ok = [&](const int4& q) {
      return q.x >= 0 && q.x < args.S && q.z >= 1 && q.z <= kRowsPerItem && q.y >= 0 && q.y <= args.T - q.z;
    };
    int u = sh.first[grp];
    int pending = u < units ? claim_issue() : 0;
    // The item record and rows of the next unit are loaded while the current
    // unit's stages are issued, so no unit waits on them.
    // Fused expand units: the item's v (written by the finisher of its last
    // shrink slice) is copied into vbuf by this warp, so the consumers find
    // it in shared memory; its ready word is read one unit ahead too.
    auto ready_word = [&](const Dec& q) -> const int* { return wv.ready + q.prob * tpad + q.item; };
    Dec d = decode(u);
    int4 it = d.kind != kUnitEnd ? pv.items[d.item] : make_int4(0, 0, 0, 0);
    int row = d.kind != kUnitEnd && item_ok(it) && lane < it.z ? pv.perm[it.y + lane] : 0;
    int rd = MODE == kModeFused && d.kind == kUnitExpand && lane == 0 ? ld_relaxed(ready_word(d)) : 0;
    uint32_t ev = 0;  // fused expand units whose v this warp has copied
    bool dead = false;
    for (int j = 0; !dead; ++j) {
      const int iq = j % kUnitRing;
      int ok = 1;
      if (lane == 0 && j >= kUnitRing)
        ok = mbar_wait_abortable(&sm.uempty[iq], ((j / kUnitRing) - 1) & 1, args.err, abort) ? 1 : 0;
      if (!__shfl_sync(0xffffffffu, ok, 0)) break;  // the other roles find no unit and give up too
      if (d.kind != kUnitEnd) {
        const bool good = __all_sync(0xffffffffu, item_ok(it) && (lane >= it.z || (row >= 0 && row < args.T)));
        if (!good) {
          if (lane == 0 && d.slice == 0) raise_error(args.err, PERSONA_DEV_ERR_PLAN);
          it = make_int4(0, it.y >= 0 && it.y < args.T ? it.y : 0, 0, 0);
          row = 0;
        }
      }
      UnitDesc* ud = &sm.units[iq];
      if (lane < kRowsPerItem) ud->rows[lane] = row;
      if (lane == 0) {
        ud->kind = d.kind;
        ud->prob = d.prob;
        ud->item = d.item;
        ud->slice = d.slice;
        ud->slot = it.x;
        ud->count = it.z;
        ud->pos = it.y;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.ufull[iq]);
      if (d.kind == kUnitEnd) break;

      const int slot = it.x, c = it.z;
      const SplitProblem& pr = args.prob[d.prob];
      // Fused expand unit: acquire the item's v and start its copy before the
      // next unit's loads are issued, so the acquire fence waits for none of
      // them (after them it held the copy, and the first stage's loads behind
      // it, back by about 2 us per unit).
      if (MODE == kModeFused && d.kind == kUnitExpand) {
        int vok = 1;
        if (lane == 0) {
          const int eb = static_cast<int>(ev & 1);
          if (ev >= 2) vok = mbar_wait_abortable(&sm.vempty[eb], ((ev >> 1) - 1) & 1, args.err, abort) ? 1 : 0;
          if (vok) {
            if (rd == epoch)
              asm volatile("fence.acq_rel.gpu;" ::: "memory");  // acquire side of the value read a unit ago
            else
              vok = wait_word(ready_word(d), epoch, args.err, abort, &wv.sync[kSyncAbort]) ? 1 : 0;
          }
          if (vok) {
            fence_proxy_async_global();  // the finisher's stores, read by the bulk copy
            const uint32_t vb = static_cast<uint32_t>(c * R * 4);
            mbar_arrive_expect_tx(&sm.vfull[eb], vb);
            if (vb > 0)
              bulk_load(sm.vbuf + eb * (kRowsPerItem * kMaxR),
                        wv.vfinal + (static_cast<int64_t>(d.prob) * tpad + it.y) * R, vb, &sm.vfull[eb]);
          }
        }
        if (__shfl_sync(0xffffffffu, vok, 0))
          ++ev;
        else
          dead = true;
      }
      // The next unit's claim has returned by now; issue the one after it,
      // and start loading the next unit's item record.
      const int u_next = claim_read(pending);
      pending = u_next < units ? claim_issue() : 0;
      const Dec dn = decode(u_next);
      const int4 itn = dn.kind != kUnitEnd ? pv.items[dn.item] : make_int4(0, 0, 0, 0);
      const int rdn = MODE == kModeFused && dn.kind == kUnitExpand && lane == 0 ? ld_relaxed(ready_word(dn)) : 0;
      int rown = 0;
      bool rows_loaded = false;
      auto load_next_rows = [&]() {  // once itn has arrived: after the first stage is issued
        if (!rows_loaded) {
          rows_loaded = true;
          if (dn.kind != kUnitEnd && item_ok(itn) && lane < itn.z) rown = pv.perm[itn.y + lane];
        }
      };

      if (d.kind == kUnitShrink) {
        const uint16_t* x = static_cast<const uint16_t*>(pr.x);
        for (int k0 = d.lo; !dead && k0 < d.hi; k0 += C::kKC) {
          const int valid = min(C::kKC, d.hi - k0);
          const int nbox = (valid + 63) / 64;
          const uint32_t xb = static_cast<uint32_t>(valid) * 2u;
          const int s = claim_slot(static_cast<uint32_t>(nbox * C::kABoxBytes) + static_cast<uint32_t>(c) * xb);
          if (s < 0) {
            dead = true;
            break;
          }
          uint8_t* st = sm.ring + s * kSlotBytes;
          if (lane == 0)
            for (int b = 0; b < nbox; ++b)
              tma_load_3d(st + b * C::kABoxBytes, &maps.a[d.prob], &sm.full[s], k0 + 64 * b, 0, slot);
          if (lane < c)
            bulk_load(st + C::kXOff + lane * C::kXPitch, x + static_cast<int64_t>(row) * pr.ldx + k0, xb, &sm.full[s]);
          ++g;
          load_next_rows();
        }
      } else {
        const uint16_t* yg = static_cast<const uint16_t*>(pr.y);
        const int stage_rows = sh.geom[d.prob].stage_rows;
        if (MODE == kModeExpand) {
          const int s = claim_slot(static_cast<uint32_t>(c * R * 4));
          if (s < 0) {
            dead = true;
          } else {
            if (lane < c)
              bulk_load(sm.ring + s * kSlotBytes + lane * R * 4, args.v_in + static_cast<int64_t>(row) * R, R * 4,
                        &sm.full[s]);
            ++g;
          }
        }
        for (int n0 = d.lo; !dead && n0 < d.hi; n0 += stage_rows) {
          const int rows_here = min(stage_rows, d.hi - n0);
          const int nbox = (rows_here + pr.n_box - 1) / pr.n_box;
          const uint32_t yb = static_cast<uint32_t>(rows_here) * 2u;
          const int s = claim_slot(static_cast<uint32_t>(nbox * pr.n_box * 2 * R) + static_cast<uint32_t>(c) * yb);
          if (s < 0) {
            dead = true;
            break;
          }
          uint8_t* st = sm.ring + s * kSlotBytes;
          if (lane == 0)
            for (int b = 0; b < nbox; ++b)
              tma_load_3d(st + b * pr.n_box * 2 * R, &maps.b[d.prob], &sm.full[s], 0, n0 + b * pr.n_box, slot);
          if (lane < c)
            bulk_load(st + C::kYOff + lane * C::kYStride, yg + static_cast<int64_t>(row) * pr.ldy + n0, yb,
                      &sm.full[s]);
          ++g;
          load_next_rows();
        }
      }
      load_next_rows();
      u = u_next;
      d = dn;
      it = itn;
      row = rown;
      rd = rdn;
    }
    // Every copy this warp issued lands before the CTA exits (normally the
    // consumers have waited for all of them already).
    if (lane == 0) {
      for (int s = 0; s < kSlots; ++s)
        if (g > static_cast<uint32_t>(s)) mbar_wait(&sm.full[s], ((g - 1 - s) / kSlots) & 1, args.err);
      for (uint32_t b = 0; b < 2; ++b)
        if (ev > b) mbar_wait(&sm.vfull[b], ((ev - 1 - b) >> 1) & 1, args.err);
    }
    __syncwarp();
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA --
    // Follows the unit ring and the stage ring; for every expand stage of a
    // tensor-core kernel it issues D[box] = B_box * (v_hi + v_lo)^T into the
    // slot's accumulators and commits to mma_done[slot]; every other stage
    // gets a plain arrive so that mma_done keeps one phase per slot use.
    // (Releasing a slot from the MMA commit instead, with a separate ring of
    // accumulators, measured slower: 340 against 305 us per launch.)
    if (lane == 0) {
      uint32_t g = 0, ue = 0;
      const uint32_t vop = smem_u32(sm.vop);
      bool dead = false;
      for (int j = 0; !dead; ++j) {
        const int iq = j % kUnitRing;
        if (!mbar_wait_abortable(&sm.ufull[iq], (j / kUnitRing) & 1, args.err, abort)) break;
        const int kind = sm.units[iq].kind, prob = sm.units[iq].prob, slice = sm.units[iq].slice;
        if (kind == kUnitEnd) break;
        const ProbGeom& gg = sh.geom[prob];
        int nst, lo = 0, hi = 0;
        if (kind == kUnitShrink) {
          const int klo = slice * gg.ks_st * C::kKC;
          nst = (min(args.prob[prob].K, klo + gg.ks_st * C::kKC) - klo + C::kKC - 1) / C::kKC;
        } else {
          lo = slice * gg.es_st * gg.stage_rows;
          hi = min(args.prob[prob].N, lo + gg.es_st * gg.stage_rows);
          nst = (hi - lo + gg.stage_rows - 1) / gg.stage_rows;
          if (MODE == kModeExpand) {  // the v stage
            const int s = static_cast<int>(g % kSlots);
            if (!mbar_wait_abortable(&sm.full[s], (g / kSlots) & 1, args.err, abort)) break;
            mbar_arrive(&sm.mma_done[s]);
            ++g;
          }
        }
        const bool tc_unit = kTcE && kind == kUnitExpand;
        if (tc_unit) {
          if (!mbar_wait_abortable(sm.vready, ue & 1, args.err, abort)) break;
          tc::fence_after_sync();
          ++ue;
        }
        for (int i = 0; i < nst; ++i, ++g) {
          const int s = static_cast<int>(g % kSlots);
          if (!mbar_wait_abortable(&sm.full[s], (g / kSlots) & 1, args.err, abort)) {
            dead = true;
            break;
          }
          if (tc_unit) {
            tc::fence_after_sync();
            const int rows_here = min(gg.stage_rows, hi - (lo + i * gg.stage_rows));
            const int nbt = (rows_here + 127) / 128;
            const uint32_t sb = smem_u32(sm.ring + s * kSlotBytes);
            for (int b = 0; b < nbt; ++b) {
              const uint32_t d = tmem + static_cast<uint32_t>((s * 2 + b) * kRowsPerItem);
#pragma unroll
              for (int ks = 0; ks < R / 16; ++ks) {
                const uint64_t a = tc::smem_desc(sb + b * 128 * 2 * R + ks * 32, kOpSbo, kOpLayout);
                tc::mma_f16(d, a, tc::smem_desc(vop + ks * 32, kOpSbo, kOpLayout), kIdesc, ks > 0 ? 1u : 0u);
                tc::mma_f16(d, a, tc::smem_desc(vop + kRowsPerItem * 2 * R + ks * 32, kOpSbo, kOpLayout), kIdesc,
                            1u);
              }
            }
            tc::commit(&sm.mma_done[s]);
          } else {
            mbar_arrive(&sm.mma_done[s]);
          }
        }
        if (!dead) mbar_arrive(&sm.uempty[iq]);
      }
      // Every MMA this thread issued completes before TMEM is released.
      tc::commit(sm.mma_fin);
      mbar_wait(sm.mma_fin, 0, args.err);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------ consumers --
    if (MODE == kModeShrink) {
      // Rows without a (valid) adapter get v = 0; the items never touch them.
      const int gtid = (blockIdx.x * kGroups + grp) * kConsumers + tid;
      const int gstride = gridDim.x * kGroups * kConsumers;
      for (int i = gtid; i < args.T * R; i += gstride) {
        const int s = args.slots[i / R];
        if (s < 0 || s >= args.S) args.v_out[i] = 0.f;
      }
    }
    uint32_t g = 0;   // stage counter, as in the producer and the MMA warp
    uint32_t ev = 0;  // fused expand units, as in the producer
    for (int j = 0;; ++j) {
      const int iq = j % kUnitRing;
      const bool got = mbar_wait_abortable(&sm.ufull[iq], (j / kUnitRing) & 1, args.err, abort);
      // all four consumer warps go on, or none does
      if (!named_all(bar_cons, kConsumers, got && *reinterpret_cast<volatile int*>(abort) == 0)) break;
      const UnitDesc* ud = &sm.units[iq];
      const int kind = ud->kind;
      if (kind == kUnitEnd) break;
      const int prob = ud->prob, c = ud->count, item = ud->item, slice = ud->slice, pos = ud->pos;
      const int* rows = ud->rows;
      const int E = c * R;
      const ProbGeom& gg = sh.geom[prob];
      const SplitProblem& pr = args.prob[prob];

      if (kDoShrink && kind == kUnitShrink) {
        const int klo = slice * gg.ks_st * C::kKC;
        const int khi = min(pr.K, klo + gg.ks_st * C::kKC);
        float d[C::kTPW][2][4];
#pragma unroll
        for (int t = 0; t < C::kTPW; ++t)
#pragma unroll
          for (int i = 0; i < 4; ++i) d[t][0][i] = d[t][1][i] = 0.f;
        for (int k0 = klo; k0 < khi; k0 += C::kKC, ++g) {
          const int s = static_cast<int>(g % kSlots);
          const bool ok = mbar_wait_abortable(&sm.full[s], (g / kSlots) & 1, args.err, abort);
          uint8_t* st = sm.ring + s * kSlotBytes;
          const int valid = min(C::kKC, khi - k0);
          if (valid & 63) {
            // The last A tile reads zeros past K; zero the matching x columns so
            // that stale shared memory cannot inject NaN * 0.
            const int tail = ((valid + 63) & ~63) - valid;
            for (int e = tid; e < c * tail; e += kConsumers) {
              const int rr = e / tail, kk = valid + e % tail;
              reinterpret_cast<uint16_t*>(st + C::kXOff + rr * C::kXPitch)[kk] = 0;
            }
            named_sync(bar_cons, kConsumers);
          }
          shrink_stage<DT, R>(st, ((valid + 63) / 64) * 4, warp, lane, d);
          __syncwarp();
          if (lane == 0 && ok) mbar_arrive_relaxed(&sm.empty[s]);
        }
        // This slice's partial v: sum the two accumulators and the warps that
        // split k for each rank tile.
#pragma unroll
        for (int t = 0; t < C::kTPW; ++t) {
          float* rw = sm.red + (warp * C::kTPW + t) * (kRowsPerItem * 8);
          const int gq = lane >> 2, tq = lane & 3;
          rw[gq * 8 + 2 * tq] = d[t][0][0] + d[t][1][0];
          rw[gq * 8 + 2 * tq + 1] = d[t][0][1] + d[t][1][1];
          rw[(gq + 8) * 8 + 2 * tq] = d[t][0][2] + d[t][1][2];
          rw[(gq + 8) * 8 + 2 * tq + 1] = d[t][0][3] + d[t][1][3];
        }
        named_sync(bar_cons, kConsumers);
        for (int e = tid; e < E; e += kConsumers) {
          const int rr = e / R, r = e - rr * R;
          const int T = r >> 3, col = r & 7;
          float sum = 0.f;
#pragma unroll
          for (int ks = 0; ks < C::kKS; ++ks)
            sum += sm.red[(((T / C::kTPW) * C::kKS + ks) * C::kTPW + (T % C::kTPW)) * (kRowsPerItem * 8) +
                          rr * 8 + col];
          sm.pv[e] = sum;
        }
        named_sync(bar_cons, kConsumers);
        int* s_cnt = wv.s_cnt + prob * tpad + item;
        bool finisher = true;
        if (gg.nks > 1) {
          float* part = wv.parts + static_cast<int64_t>(gg.p_base + item * gg.nks + slice) * kPartFloats;
          for (int e = tid; e < E; e += kConsumers) part[e] = sm.pv[e];
          named_sync(bar_cons, kConsumers);
          // One acquire-release count after the barrier: its release side
          // (cumulative) orders every consumer's partial stores before it, its
          // acquire side the other slices' partials before the finisher's reads.
          if (tid == 0) {
            int old;
            asm volatile("atom.add.acq_rel.gpu.global.s32 %0, [%1], 1;" : "=r"(old) : "l"(s_cnt) : "memory");
            *sm.flag = old == gg.nks - 1;
          }
          named_sync(bar_cons, kConsumers);
          finisher = *sm.flag != 0;
          if (finisher) {
            const float* p0 = wv.parts + static_cast<int64_t>(gg.p_base + item * gg.nks) * kPartFloats;
            for (int e = tid; e < E; e += kConsumers) {
              // eight slices' loads in flight at a time, summed in slice order
              float sum = 0.f;
              int q = 0;
              for (; q + 8 <= gg.nks; q += 8) {
                float pv8[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) pv8[i] = __ldcg(p0 + (q + i) * kPartFloats + e);
#pragma unroll
                for (int i = 0; i < 8; ++i) sum += pv8[i];
              }
              for (; q < gg.nks; ++q) sum += __ldcg(p0 + q * kPartFloats + e);
              sm.pv[e] = sum;
            }
          }
        }
        if (finisher) {
          if (MODE == kModeShrink) {
            for (int e = tid; e < E; e += kConsumers) {
              const int rr = e / R, rk = e - rr * R;
              args.v_out[static_cast<int64_t>(rows[rr]) * R + rk] = sm.pv[e];
            }
          } else {
            float* vfin = wv.vfinal + (static_cast<int64_t>(prob) * tpad + pos) * R;
            for (int e = tid; e < E; e += kConsumers) vfin[e] = sm.pv[e];
            fence_proxy_async_global();  // another SM's producer bulk-copies v
          }
          named_sync(bar_cons, kConsumers);
          if (tid == 0) {
            if (gg.nks > 1) *s_cnt = 0;  // every slice has counted: ready for the next launch
            // the release store orders the CTA's v stores (cumulative over the barrier)
            if (MODE != kModeShrink) st_release(wv.ready + prob * tpad + item, epoch);
          }
        }
        named_sync(bar_cons, kConsumers);
      }

      if (kDoExpand && kind == kUnitExpand) {
        uint16_t* y = static_cast<uint16_t*>(pr.y);
        float* vfb = sm.vf;
        bool okv = true;
        if (MODE == kModeExpand) {
          const int s = static_cast<int>(g % kSlots);
          const bool ok = mbar_wait_abortable(&sm.full[s], (g / kSlots) & 1, args.err, abort);
          const float* vs = reinterpret_cast<const float*>(sm.ring + s * kSlotBytes);
          for (int e = tid; e < E; e += kConsumers) vfb[e] = vs[e];
          __syncwarp();
          if (lane == 0 && ok) mbar_arrive_relaxed(&sm.empty[s]);
          ++g;
        } else {
          // the producer has copied this item's v into vbuf[ev & 1]
          okv = mbar_wait_abortable(&sm.vfull[ev & 1], (ev >> 1) & 1, args.err, abort);
          vfb = sm.vbuf + (ev & 1) * (kRowsPerItem * kMaxR);
        }
        named_sync(bar_cons, kConsumers);
        // Power-of-two scale that keeps the 16-bit v halves finite (f16 only).
        float scale_down = 1.f, scale_up = 1.f;
        if (std::is_same<DT, __half>::value) {
          float m = 0.f;
          for (int e = tid; e < E; e += kConsumers) m = fmaxf(m, fabsf(vfb[e]));
#pragma unroll
          for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
          if (lane == 0) sm.red[warp] = m;
          named_sync(bar_cons, kConsumers);
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
        const int stage_rows = gg.stage_rows;
        const int nlo = slice * gg.es_st * stage_rows;
        const int nhi = min(pr.N, nlo + gg.es_st * stage_rows);
        if constexpr (kTcE) {
          // MMA operands: rows of v_hi and v_lo (2R bytes each, swizzled like
          // the TMA-written B tile); rows >= c are zero.
          const uint32_t vop = smem_u32(sm.vop);
          for (int e = tid; e < kRowsPerItem * R / 2; e += kConsumers) {
            const int t = e / (R / 2), k = (e - t * (R / 2)) * 2;
            float a = 0.f, b = 0.f;
            if (t < c) {
              a = vfb[t * R + k] * scale_down;
              b = vfb[t * R + k + 1] * scale_down;
            }
            const float ha = Mma<DT>::round_trip(a), hb = Mma<DT>::round_trip(b);
            const uint32_t off = swz(static_cast<uint32_t>(t * 2 * R + k * 2), C::kBSwz);
            sts32(vop + off, Mma<DT>::pack(ha, hb));
            sts32(vop + kRowsPerItem * 2 * R + off, Mma<DT>::pack(a - ha, b - hb));
          }
          tc::fence_proxy_async();
          named_sync(bar_cons, kConsumers);
          if (tid == 0) mbar_arrive(sm.vready);
          // tcgen05.ld lets a warp reach the TMEM lanes of its physical warp
          // id mod 4; lane = output column within the 128-row box.
          const int quarter = (static_cast<int>(threadIdx.x) >> 5) & 3;
          const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
          for (int n0 = nlo; n0 < nhi; n0 += stage_rows, ++g) {
            const int s = static_cast<int>(g % kSlots);
            bool ok = mbar_wait_abortable(&sm.full[s], (g / kSlots) & 1, args.err, abort);
            ok = mbar_wait_abortable(&sm.mma_done[s], (g / kSlots) & 1, args.err, abort) && ok;
            __syncwarp();
            tc::fence_after_sync();
            const int rows_here = min(stage_rows, nhi - n0);
            const int nbt = (rows_here + 127) / 128;
            const uint32_t ytile = smem_u32(sm.ring + s * kSlotBytes + C::kYOff);
            uint16_t out[2][kRowsPerItem];
#pragma unroll
            for (int b = 0; b < 2; ++b) {
              if (b < nbt) {
                uint32_t dr[16];
                tc::ld16(tmem + lane_addr + static_cast<uint32_t>((s * 2 + b) * kRowsPerItem), dr);
                tc::wait_ld();
                const int n = b * 128 + quarter * 32 + lane;
#pragma unroll
                for (int t = 0; t < kRowsPerItem; ++t) {
                  if (t < c) {
                    const float yo = Cvt<DT>::to1(lds16(ytile + t * C::kYStride + n * 2));
                    out[b][t] = Cvt<DT>::from1(yo + scale_up * __uint_as_float(dr[t]));
                  }
                }
              }
            }
            tc::fence_before_sync();
            // The new values go back into the staged y tile (this thread's
            // column), then each lane stores 16-byte runs of 8 columns of one
            // row: a warp's 32 columns of c rows take 4c vector stores instead
            // of 32c two-byte ones.
#pragma unroll
            for (int b = 0; b < 2; ++b) {
              if (b < nbt) {
                const int n = b * 128 + quarter * 32 + lane;
#pragma unroll
                for (int t = 0; t < kRowsPerItem; ++t)
                  if (t < c) sts16(ytile + t * C::kYStride + n * 2, out[b][t]);
              }
            }
            __syncwarp();
#pragma unroll
            for (int b = 0; b < 2; ++b) {
              if (b < nbt) {
                for (int q = lane; q < 4 * c; q += 32) {
                  const int t = q >> 2, col = b * 128 + quarter * 32 + (q & 3) * 8;
                  if (n0 + col < nhi) {  // nhi and the column are multiples of 8
                    const uint4 val = lds128(ytile + t * C::kYStride + col * 2);
                    *reinterpret_cast<uint4*>(y + static_cast<int64_t>(rows[t]) * pr.ldy + n0 + col) = val;
                  }
                }
              }
            }
            __syncwarp();
            if (lane == 0 && ok) mbar_arrive_relaxed(&sm.empty[s]);
          }
        } else {
          uint32_t vhi[C::kKSteps][4], vlo[C::kKSteps][4];
          v_fragments<DT, R>(vfb, scale_down, lane, vhi, vlo);
          for (int n0 = nlo; n0 < nhi; n0 += stage_rows, ++g) {
            const int s = static_cast<int>(g % kSlots);
            const bool ok = mbar_wait_abortable(&sm.full[s], (g / kSlots) & 1, args.err, abort);
            const int rows_here = min(stage_rows, nhi - n0);
            expand_stage<DT, R>(sm.ring + s * kSlotBytes, vhi, vlo, rows_here, pr.n_box, n0, c, rows, y, pr.ldy,
                                scale_up, warp, lane, ok ? &sm.empty[s] : nullptr);
          }
        }
        named_sync(bar_cons, kConsumers);
        if (MODE == kModeFused) {
          // vbuf[ev & 1] may take the v of a later unit
          if (tid == 0 && okv) mbar_arrive(&sm.vempty[ev & 1]);
          ++ev;
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive_relaxed(&sm.uempty[iq]);
    }
  }
  // The last CTA to finish resets the claim counter and bumps the epoch for
  // the next launch on this workspace; after a launch in which a CTA gave up
  // it also clears the per-item counters and ready words, so the next launch
  // starts clean.
  tc::fence_before_sync();
  __syncthreads();
  if (kTcE && grp == 0 && warp == kMmaWarp) {
    tc::fence_after_sync();
    tc::tmem_dealloc(sh.tmem, kTmemCols);
  }
  if (threadIdx.x == 0 && plan_ok) {
    if (sh.abort) atomicExch(&wv.sync[kSyncAbort], 1);
    __threadfence();
    if (atomicAdd(&wv.sync[kSyncDone], 1) == static_cast<int>(gridDim.x) - 1) {
      __threadfence();
      if (ld_acquire(&wv.sync[kSyncAbort]) != 0) {
        for (int64_t i = 0; i < 2 * kMaxProblems * tpad; ++i) wv.s_cnt[i] = 0;  // s_cnt, then ready
        wv.sync[kSyncAbort] = 0;
      }
      wv.sync[kSyncQueue] = 0;
      wv.sync[kSyncDone] = 0;
      wv.sync[kSyncEpoch] = epoch + 1 > 0 ? epoch + 1 : 1;
      __threadfence();
    }
  }
}

// ------------------------------------------------------------------ host --

int bgmv_stage_rows(int R) {
  switch (R) {
    case 8: return RankCfg<8>::kNB;
    case 16: return RankCfg<16>::kNB;
    case 32: return RankCfg<32>::kNB;
    default: return RankCfg<64>::kNB;
  }
}

template <typename DT, int R, int MODE>
static cudaError_t split_launch(const SplitMaps& maps, const SplitArgs& a, cudaStream_t stream) {
  auto kern = bgmv_split_kernel<DT, R, MODE>;
  constexpr int kMaxDev = 64;
  // CTAs per device (one per SM); racing first calls compute the same value
  static std::atomic<int> ctas[kMaxDev];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDev) return cudaErrorInvalidDevice;
  int grid = ctas[dev].load(std::memory_order_acquire);
  if (grid == 0) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSplitSmemBytes);
    if (e != cudaSuccess) return e;
    int per_sm = 0, sms = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kSplitThreads, kSplitSmemBytes);
    if (e != cudaSuccess) return e;
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    grid = (per_sm > 0 ? per_sm : 1) * sms;
    ctas[dev].store(grid, std::memory_order_release);
  }
  // Programmatic dependent of the kernel before it (normally the plan
  // kernel, which lets its dependents start at once): the CTAs set up their
  // barriers and tensor memory while it runs, then wait for it to complete.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kSplitThreads);
  cfg.dynamicSmemBytes = kSplitSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kern, maps, a);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

template <typename DT, int MODE>
static cudaError_t split_rank(int R, const SplitMaps& maps, const SplitArgs& a, cudaStream_t st) {
  switch (R) {
    case 8: return split_launch<DT, 8, MODE>(maps, a, st);
    case 16: return split_launch<DT, 16, MODE>(maps, a, st);
    case 32: return split_launch<DT, 32, MODE>(maps, a, st);
    case 64: return split_launch<DT, 64, MODE>(maps, a, st);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t launch_bgmv_split(int mode, int dtype, int R, const SplitMaps& maps, const SplitArgs& a,
                              cudaStream_t st) {
  if (a.num_problems < 1 || a.num_problems > kMaxProblems) return cudaErrorInvalidValue;
  if (mode != kModeFused && a.num_problems != 1) return cudaErrorInvalidValue;
  const bool bf = dtype == PERSONA_DTYPE_BF16;
  switch (mode) {
    case kModeShrink:
      return bf ? split_rank<__nv_bfloat16, kModeShrink>(R, maps, a, st)
                : split_rank<__half, kModeShrink>(R, maps, a, st);
    case kModeExpand:
      return bf ? split_rank<__nv_bfloat16, kModeExpand>(R, maps, a, st)
                : split_rank<__half, kModeExpand>(R, maps, a, st);
    default:
      return bf ? split_rank<__nv_bfloat16, kModeFused>(R, maps, a, st)
                : split_rank<__half, kModeFused>(R, maps, a, st);
  }
}

}  // namespace persona
