// NF4 base linears for B200 (sm_100a): the quantiser, the dequantiser and
// the decode GEMM y[M, N] = x[M, K] W^T with W in the tiled NF4 format
// (nf4_table.h) and M <= 64 rows of x.
//
// The reference runs its base linears through bitsandbytes' Linear4bit
// (reference bench/e2e.py:70-90: nf4, blocksize 64, double-quantised
// scales, fp16 compute) under MultiLoRALinear.base (persona/lora_layer.py).
//
// GEMM design.  At decode sizes the op streams 0.52 bytes per weight from
// HBM and does 2 M flops per weight, so it is bound by HBM and by the
// instructions that turn 4-bit codes into tensor-core operands.  The codes
// are stored in the A-fragment order of mma.sync.m16n8k16, so one 32-bit
// word of codes is exactly one thread's A fragment for one k-step: four
// bytes, each mapped by a 256-entry table to the two fp16 NF4 values it
// holds.  The table sits in shared memory once per lane (entry b of lane l at
// byte 256 b + 4 l), so every lookup is free of bank conflicts and its offset
// is one byte permute of the code word and 4 l.  The fragments
// never go through shared memory, and the per-block scale is applied to the
// fp32 partial sum of each 64-wide block (two per 128-wide chunk), not to
// every weight.  x (M rows, fp16) is the B operand, TMA-loaded per chunk
// with a 128-byte swizzle so that the B-fragment loads are conflict-free.
// Tensor-core work per weight is tiny at M <= 64, well inside what the
// warp-level MMA delivers; staging dequantised tiles in shared memory for
// tcgen05 would instead cost 4 bytes of shared-memory traffic per weight.
//
// Work: the launch's chunks (problem, tile of 128 output rows, 128-wide K
// chunk) in one linear order, cut into equal contiguous ranges, one per CTA
// (two CTAs per SM at 8 rows, one above), so every SM streams the same
// number of bytes.  A producer warp bulk-copies each 8464-byte chunk and
// TMA-loads the x chunk into a ring of 4 (8 rows) or 6 slots; eight compute
// warps each own 16 rows of the tile.  A tile inside one range is written
// straight to y.  A tile cut between ranges leaves one fp32 piece per CTA
// (a CTA's first and last tile may be such pieces); the last piece to finish
// (per-tile counter) sums them in CTA order, so the result does not depend
// on scheduling, writes y and resets the counter.  A first piece followed by
// more of the range is counted by an epilogue warp, so the compute warps do
// not wait for the count.
#include <cuda_fp16.h>

#include <atomic>

#include "common.cuh"
#include "nf4_args.h"
#include "tcgen05.cuh"

namespace persona {
namespace {

constexpr int kNf4Warps = 8;                      // compute warps
constexpr int kNf4ProducerWarp = kNf4Warps;       // bulk copies and TMA loads
constexpr int kNf4EpilogueWarp = kNf4Warps + 1;   // counts a CTA's first tile piece
constexpr int kNf4Threads = (kNf4Warps + 2) * 32;
constexpr int kNf4MaxSlots = 6;

// Dynamic shared memory: the lookup table at offset 0, then the slots' x
// boxes (two per slot, 8 MT rows each, 1 KB aligned for the 128-byte
// swizzle), then the slots' chunks (16-byte aligned, packed).
//
// The table holds entry b of lane l at byte kLutRow b + 4 l.  At MT = 1 a row
// is 256 bytes (the upper 128 unused): one byte permute of the code word and
// the lane's 4 l is then the whole offset of a lookup, which matters because
// there the lookups are most of the instructions.  Above, every lookup feeds
// MT MMAs and the rows are 128 bytes (a permute and a shift-add), which
// leaves more of the SM's shared memory to L1.
//
// At MT = 1 four slots keep two CTAs on an SM, which doubles the warps that
// hide the load and MMA latencies; at MT >= 2 one CTA fits and gets six.
template <int MT>
struct Nf4Cfg {
  static constexpr int kLutRow = MT == 1 ? 256 : 128;
  static constexpr int kLutBytes = 256 * kLutRow;
  static constexpr int kSlots = MT == 1 ? 4 : kNf4MaxSlots;
  static constexpr int kXBytes = 2 * 8 * MT * 128;
  static constexpr int kSmem = kLutBytes + 1024 + kSlots * (kXBytes + kNf4ChunkBytes);
  static_assert(kXBytes % 1024 == 0, "x box alignment");
  static_assert(kSlots <= kNf4MaxSlots, "slot count");
};
constexpr int kNf4EpiBar = 1;
static_assert(kNf4ChunkBytes % 16 == 0, "chunk layout");

__device__ __forceinline__ float h2f(uint32_t bits) { return __half2float(__ushort_as_half(static_cast<uint16_t>(bits))); }

__device__ __forceinline__ int nf4_index(float v, float am) {
  const float r = am > 0.f ? __fdiv_rn(v, am) : 0.f;
  int idx = 0;
#pragma unroll
  for (int i = 0; i < 15; ++i) idx += r > __uint_as_float(kNf4Mid[i]) ? 1 : 0;
  return idx;
}

__device__ __forceinline__ uint32_t nf4_half_bits(int i) {
  uint32_t h = 0;
#pragma unroll
  for (int k = 0; k < 16; ++k) h = i == k ? kNf4Half[k] : h;
  return h;
}

// (row, column) of the first of the two weights in code byte q of a chunk.
__device__ __forceinline__ void nf4_byte_pos(int q, int& row, int& col) {
  const int j = q & 3, ks = (q >> 2) & 3, lane = (q >> 4) & 31, kh = (q >> 9) & 1, wt = q >> 10;
  const int g = lane >> 2, t = lane & 3;
  row = 16 * wt + g + 8 * (j & 1);
  col = 64 * kh + 16 * ks + 2 * t + 8 * (j >> 1);
}

// ------------------------------------------------------------ quantiser ----
__global__ void nf4_minmax_init_kernel(uint32_t* minmax) {
  if (threadIdx.x == 0) {
    minmax[0] = 0x7f800000u;  // +inf: no block seen yet
    minmax[1] = 0u;
  }
}

__global__ void nf4_absmax_kernel(const uint16_t* __restrict__ w, int64_t ldw, int N, int K,
                                  float* __restrict__ absmax, uint32_t* __restrict__ minmax) {
  const int nb = K / kNf4Block;
  const int64_t total = static_cast<int64_t>(N) * nb;
  uint32_t lmin = 0x7f800000u, lmax = 0u;  // absmax >= 0 orders like its bits
  for (int64_t b = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; b < total;
       b += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = b / nb;
    const int kb = static_cast<int>(b - row * nb);
    const uint4* p = reinterpret_cast<const uint4*>(w + row * ldw + kb * kNf4Block);
    float m = 0.f;
#pragma unroll
    for (int i = 0; i < kNf4Block / 8; ++i) {
      const uint4 q = p[i];
      const uint32_t v[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) m = fmaxf(m, fmaxf(fabsf(h2f(v[k] & 0xffffu)), fabsf(h2f(v[k] >> 16))));
    }
    absmax[b] = m;
    lmin = min(lmin, __float_as_uint(m));
    lmax = max(lmax, __float_as_uint(m));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    lmin = min(lmin, __shfl_xor_sync(0xffffffffu, lmin, o));
    lmax = max(lmax, __shfl_xor_sync(0xffffffffu, lmax, o));
  }
  if ((threadIdx.x & 31) == 0) {
    atomicMin(&minmax[0], lmin);
    atomicMax(&minmax[1], lmax);
  }
}

// One CTA of 256 threads per 128 x 128 tile.
__global__ void __launch_bounds__(256) nf4_pack_kernel(const uint16_t* __restrict__ w, int64_t ldw, int N, int K,
                                                       const float* __restrict__ absmax,
                                                       const uint32_t* __restrict__ minmax,
                                                       uint8_t* __restrict__ packed, float* __restrict__ offset_out) {
  const int kc = blockIdx.x, nt = blockIdx.y, kt = K / kNf4Tile;
  uint8_t* chunk = packed + (static_cast<int64_t>(nt) * kt + kc) * kNf4ChunkBytes;
  const float off = __fmul_rn(__fadd_rn(__uint_as_float(minmax[0]), __uint_as_float(minmax[1])), 0.5f);
  const int tid = threadIdx.x;
  if (kc == 0 && nt == 0 && tid == 0) *offset_out = off;
  __shared__ float s_am[2 * kNf4Tile];
  __shared__ float s_red[8];
  {
    const int r = tid >> 1, kh = tid & 1;
    const float a = absmax[static_cast<int64_t>(nt * kNf4Tile + r) * (K / kNf4Block) + kc * 2 + kh];
    s_am[tid] = a;
    const float d = __fsub_rn(a, off);
    float m = fabsf(d);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((tid & 31) == 0) s_red[tid >> 5] = m;
    __syncthreads();
    float scale = s_red[0];
#pragma unroll
    for (int i = 1; i < 8; ++i) scale = fmaxf(scale, s_red[i]);
    const float s127 = __fdiv_rn(scale, 127.f);
    int q = 0;
    if (s127 > 0.f) q = min(127, max(-127, __float2int_rn(__fdiv_rn(d, s127))));
    chunk[kNf4ScaleOff + tid] = static_cast<uint8_t>(static_cast<int8_t>(q));
    if (tid < 4) reinterpret_cast<float*>(chunk + kNf4S127Off)[tid] = tid == 0 ? s127 : 0.f;
  }
  __syncthreads();
  const uint16_t* wt = w + static_cast<int64_t>(nt) * kNf4Tile * ldw + kc * kNf4Tile;
  for (int q = tid; q < kNf4CodeBytes; q += 256) {
    int row, col;
    nf4_byte_pos(q, row, col);
    const float am = s_am[row * 2 + (col >> 6)];
    const uint32_t pair = *reinterpret_cast<const uint32_t*>(wt + static_cast<int64_t>(row) * ldw + col);
    const int hi = nf4_index(h2f(pair & 0xffffu), am), lo = nf4_index(h2f(pair >> 16), am);
    chunk[q] = static_cast<uint8_t>((hi << 4) | lo);
  }
}

// ---------------------------------------------------------- dequantiser ----
// One CTA of 256 threads per tile: fp16(fp32(NF4) * absmax_q) into W.
__global__ void __launch_bounds__(256) nf4_dequant_kernel(const uint8_t* __restrict__ packed,
                                                          const float* __restrict__ offset, int N, int K,
                                                          uint16_t* __restrict__ w, int64_t ldw) {
  const int kc = blockIdx.x, nt = blockIdx.y, kt = K / kNf4Tile;
  const uint8_t* chunk = packed + (static_cast<int64_t>(nt) * kt + kc) * kNf4ChunkBytes;
  constexpr int kPitch = kNf4Tile + 8;  // halves; rows stay 16-byte aligned
  __shared__ __align__(16) uint16_t tile[kNf4Tile * kPitch];
  __shared__ float s_am[2 * kNf4Tile];
  __shared__ float s_val[16];
  const int tid = threadIdx.x;
  if (tid < 16) s_val[tid] = h2f(nf4_half_bits(tid));
  {
    const float s127 = *reinterpret_cast<const float*>(chunk + kNf4S127Off);
    const float code = static_cast<float>(static_cast<int8_t>(chunk[kNf4ScaleOff + tid]));
    s_am[tid] = __fadd_rn(__fmul_rn(code, s127), *offset);
  }
  __syncthreads();
  for (int q = tid; q < kNf4CodeBytes; q += 256) {
    int row, col;
    nf4_byte_pos(q, row, col);
    const uint32_t b = chunk[q];
    const float am = s_am[row * 2 + (col >> 6)];
    const __half h0 = __float2half_rn(__fmul_rn(s_val[b >> 4], am));
    const __half h1 = __float2half_rn(__fmul_rn(s_val[b & 15], am));
    tile[row * kPitch + col] = __half_as_ushort(h0);
    tile[row * kPitch + col + 1] = __half_as_ushort(h1);
  }
  __syncthreads();
  uint16_t* dst = w + static_cast<int64_t>(nt) * kNf4Tile * ldw + kc * kNf4Tile;
  for (int c = tid; c < kNf4Tile * 16; c += 256) {
    const int row = c >> 4, c8 = c & 15;
    *reinterpret_cast<uint4*>(dst + static_cast<int64_t>(row) * ldw + c8 * 8) =
        *reinterpret_cast<const uint4*>(tile + row * kPitch + c8 * 8);
  }
}

// ------------------------------------------------------------------ GEMM ----
// The launch's chunks in one linear order (problem, tile, K chunk); CTA g
// owns [range_start(g), range_start(g + 1)).
__device__ __forceinline__ int64_t range_start(int64_t chunks, int ctas, int g) {
  return static_cast<int64_t>(g) * chunks / ctas;
}

// The CTA whose range holds chunk c.
__device__ __forceinline__ int range_cta(int64_t chunks, int ctas, int64_t c) {
  return static_cast<int>(((c + 1) * ctas - 1) / chunks);
}

// A run of chunks of one tile inside a CTA's range: K chunks [kc0, kc1).
struct Nf4Seg {
  int p, tile, kt, kc0, kc1;
};

__device__ __forceinline__ Nf4Seg seg_at(const Nf4GemmArgs& a, int64_t c, int64_t c_end) {
  int p = 0;
#pragma unroll
  for (int i = 1; i < kNf4MaxProblems; ++i)
    if (i < a.num_problems && c >= a.prob[i].chunk_base) p = i;
  const Nf4Problem& pr = a.prob[p];
  Nf4Seg r;
  r.p = p;
  r.kt = pr.K / kNf4Tile;
  const int64_t lc = c - pr.chunk_base;
  r.tile = static_cast<int>(lc / r.kt);
  r.kc0 = static_cast<int>(lc - static_cast<int64_t>(r.tile) * r.kt);
  const int64_t left = c_end - c;
  r.kc1 = left < r.kt - r.kc0 ? r.kc0 + static_cast<int>(left) : r.kt;
  return r;
}

__device__ __forceinline__ void store_y(const Nf4Problem& pr, int M, int n0, int m0, float v0, float v1, float v2,
                                        float v3) {
  // v0 / v1: rows m0 / m0 + 1 of column n0; v2 / v3: the same of column n0 + 8.
  // With an addend (the LoRA term) it joins before the one rounding.
  uint16_t* y = pr.y;
  const int64_t ldy = pr.ldy;
  if (m0 < M) {
    if (pr.addend) {
      v0 += pr.addend[static_cast<int64_t>(m0) * pr.ld_addend + n0];
      v2 += pr.addend[static_cast<int64_t>(m0) * pr.ld_addend + n0 + 8];
    }
    y[static_cast<int64_t>(m0) * ldy + n0] = __half_as_ushort(__float2half_rn(v0));
    y[static_cast<int64_t>(m0) * ldy + n0 + 8] = __half_as_ushort(__float2half_rn(v2));
  }
  if (m0 + 1 < M) {
    if (pr.addend) {
      v1 += pr.addend[static_cast<int64_t>(m0 + 1) * pr.ld_addend + n0];
      v3 += pr.addend[static_cast<int64_t>(m0 + 1) * pr.ld_addend + n0 + 8];
    }
    y[static_cast<int64_t>(m0 + 1) * ldy + n0] = __half_as_ushort(__float2half_rn(v1));
    y[static_cast<int64_t>(m0 + 1) * ldy + n0 + 8] = __half_as_ushort(__float2half_rn(v3));
  }
}

// Sums the pieces of a tile cut between the ranges of CTAs g0 .. g1 (in
// CTA order) for the 16 rows of the tile that compute warp vw owns, and
// writes them to y.  t0: the tile's first chunk in the launch's order.
template <int MT>
__device__ __forceinline__ void finish_rows(const Nf4GemmArgs& args, const Nf4Problem& pr, int64_t C, int G,
                                            int64_t t0, int g0, int g1, int tile, int vw, int lane) {
  constexpr int MP = 8 * MT;
  const int g8 = lane >> 2, t = lane & 3;
  const int nl = 16 * vw + g8;
  const int n0 = tile * kNf4Tile + nl;
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    // four pieces' loads in flight at a time, summed in CTA order
    for (int q0 = g0; q0 <= g1; q0 += 4) {
      float2 a[4], b[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        if (q0 + q <= g1) {
          const int gq = q0 + q;
          // a range that starts inside the tile holds it as its first
          // piece, one that starts before it as its last
          const int slot = range_start(C, G, gq) >= t0 ? 0 : 1;
          const float* src = args.partials + (static_cast<int64_t>(gq) * 2 + slot) * kNf4Tile * MP;
          a[q] = __ldcg(reinterpret_cast<const float2*>(src + nl * MP + 8 * mt + 2 * t));
          b[q] = __ldcg(reinterpret_cast<const float2*>(src + (nl + 8) * MP + 8 * mt + 2 * t));
        }
      }
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        if (q0 + q <= g1) {
          v[0] += a[q].x;
          v[1] += a[q].y;
          v[2] += b[q].x;
          v[3] += b[q].y;
        }
      }
    }
    store_y(pr, args.M, n0, 8 * mt + 2 * t, v[0], v[1], v[2], v[3]);
  }
}

template <int MT>
__global__ void __launch_bounds__(kNf4Threads, MT == 1 ? 2 : 1)
    nf4_gemm_kernel(const __grid_constant__ Nf4Maps maps, const Nf4GemmArgs args) {
  constexpr int MP = 8 * MT;  // rows of x per TMA box (zero past M)
  constexpr int kSlots = Nf4Cfg<MT>::kSlots;
  constexpr int kXBytes = Nf4Cfg<MT>::kXBytes;
  constexpr int kLutRow = Nf4Cfg<MT>::kLutRow;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  // the table first: its shared address is a constant of the kernel
  uint32_t* lut = reinterpret_cast<uint32_t*>(smem_raw);
  uint8_t* xring = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw + Nf4Cfg<MT>::kLutBytes) + 1023) & ~uintptr_t(1023));
  uint8_t* cring = xring + kSlots * kXBytes;
  __shared__ uint64_t full[kNf4MaxSlots], empty[kNf4MaxSlots];
  __shared__ uint64_t first_piece_bar;  // the compute warps have stored the first piece
  __shared__ uint32_t lut1[256];
  __shared__ int s_fin;
  __shared__ int s_abort;  // set by the first wait of the CTA that gives up; later waits return at once
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t C = args.chunks;
  const int G = static_cast<int>(gridDim.x);
  const int64_t c_begin = range_start(C, G, blockIdx.x), c_end = range_start(C, G, blockIdx.x + 1);
  // the LoRA kernel after this one may start prefetching its weights
  asm volatile("griddepcontrol.launch_dependents;");

  if (tid < 256) lut1[tid] = nf4_half_bits(tid >> 4) | (nf4_half_bits(tid & 15) << 16);
  if (tid == 0) {
    for (int s = 0; s < kSlots; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kNf4Warps);
    }
    mbar_init(&first_piece_bar, kNf4Warps);
    s_abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  // the compute warps spread the table to one copy per lane while the
  // producer already streams the first chunks
  if (warp < kNf4Warps) {
    for (int i = tid; i < 256 * 32; i += kNf4Warps * 32) lut[(i >> 5) * (kLutRow / 4) + (i & 31)] = lut1[i >> 5];
    named_sync(kNf4EpiBar, kNf4Warps * 32);
  }

  if (warp == kNf4EpilogueWarp) {
    // -------------------------------------------------------- epilogue ----
    // The first tile of this CTA's range is a piece (a tile's tail, cut at
    // the range start) and more follows it: the compute warps store it and
    // go on; this warp counts it, and sums the tile if it came last (the
    // other pieces come at the ends of the ranges before, so it rarely does).
    const Nf4Seg sg = seg_at(args, c_begin, c_end);
    const bool piece = !(sg.kc0 == 0 && sg.kc1 == sg.kt);
    if (piece && c_begin + (sg.kc1 - sg.kc0) < c_end) {
      const Nf4Problem& pr = args.prob[sg.p];
      const int64_t t0 = pr.chunk_base + static_cast<int64_t>(sg.tile) * sg.kt;
      const int g0 = range_cta(C, G, t0), g1 = range_cta(C, G, t0 + sg.kt - 1);
      int* cnt = args.counters + pr.counter_base + sg.tile;
      int fin = 0;
      if (lane == 0 && mbar_wait_abortable(&first_piece_bar, 0, args.err, &s_abort)) {
        // the wait acquires the compute warps' piece stores; one cumulative
        // fence orders them before the count
        __threadfence();
        const int old = atomicAdd(cnt, 1);
        fin = old == g1 - g0;
        if (fin) __threadfence();
      }
      fin = __shfl_sync(0xffffffffu, fin, 0);
      if (fin) {
        for (int vw = 0; vw < kNf4Warps; ++vw) finish_rows<MT>(args, pr, C, G, t0, g0, g1, sg.tile, vw, lane);
        __syncwarp();
        if (lane == 0) *cnt = 0;  // every piece has counted: ready for the next launch
      }
    }
  } else if (warp == kNf4ProducerWarp) {
    // -------------------------------------------------------- producer ----
    if (lane == 0) {
      for (int p = 0; p < args.num_problems; ++p) tma_prefetch_desc(&maps.x[p]);
      // Launched as a programmatic dependent of the kernel that writes x:
      // the weight chunks of the first kSlots fills do not depend on it
      // and are requested at once; their x boxes wait for that kernel.
      int pend_kc[kSlots], pend_p[kSlots], n_pend = 0;
      bool waited = false;
      auto flush = [&]() {
        asm volatile("griddepcontrol.wait;" ::: "memory");
        for (int i = 0; i < n_pend; ++i) {
          uint8_t* xs = xring + i * kXBytes;
          tc::tma_load_2d(xs, &maps.x[pend_p[i]], &full[i], pend_kc[i] * kNf4Tile, 0);
          tc::tma_load_2d(xs + MP * 128, &maps.x[pend_p[i]], &full[i], pend_kc[i] * kNf4Tile + 64, 0);
        }
        waited = true;
      };
      uint32_t g = 0;
      bool ok = true;
      for (int64_t c = c_begin; ok && c < c_end;) {
        const Nf4Seg sg = seg_at(args, c, c_end);
        c += sg.kc1 - sg.kc0;
        const Nf4Problem& pr = args.prob[sg.p];
        for (int kc = sg.kc0; kc < sg.kc1; ++kc, ++g) {
          const int s = static_cast<int>(g % kSlots);
          if (g >= static_cast<uint32_t>(kSlots)) {
            if (!waited) flush();
            if (!mbar_wait_abortable(&empty[s], ((g / kSlots) - 1) & 1, args.err, &s_abort)) {
              ok = false;
              break;
            }
          }
          uint8_t* xs = xring + s * kXBytes;
          mbar_arrive_expect_tx(&full[s], kNf4ChunkBytes + 2 * MP * 128);
          bulk_load(cring + s * kNf4ChunkBytes,
                    pr.w + (static_cast<int64_t>(sg.tile) * sg.kt + kc) * kNf4ChunkBytes, kNf4ChunkBytes,
                    &full[s]);
          if (waited) {
            tc::tma_load_2d(xs, &maps.x[sg.p], &full[s], kc * kNf4Tile, 0);
            tc::tma_load_2d(xs + MP * 128, &maps.x[sg.p], &full[s], kc * kNf4Tile + 64, 0);
          } else {
            pend_kc[n_pend] = kc;
            pend_p[n_pend] = sg.p;
            ++n_pend;
          }
        }
      }
      if (!waited) flush();
      // every copy this thread issued lands before the CTA exits
      for (int s = 0; s < kSlots; ++s)
        if (g > static_cast<uint32_t>(s)) mbar_wait(&full[s], ((g - 1 - s) / kSlots) & 1, args.err);
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------- compute ----
    const int g8 = lane >> 2, t = lane & 3;
    const uint32_t lut_base = smem_u32(lut);
    const uint32_t lane4 = static_cast<uint32_t>(lane) * 4;  // bytes (4 lane, 0, 0, 0)
    uint32_t g = 0;
    for (int64_t c = c_begin; c < c_end;) {
      const Nf4Seg sg = seg_at(args, c, c_end);
      const bool first_piece = c == c_begin;
      c += sg.kc1 - sg.kc0;
      const Nf4Problem& pr = args.prob[sg.p];
      const float off = *pr.offset;
      float acc[MT][4];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) acc[mt][0] = acc[mt][1] = acc[mt][2] = acc[mt][3] = 0.f;
      for (int kc = sg.kc0; kc < sg.kc1; ++kc, ++g) {
        const int s = static_cast<int>(g % kSlots);
        // A failed wait (CTA gave up) still walks the chunk, so that the
        // warps' barriers stay matched, but keeps the slot: the producer
        // never re-arms a slot whose copies may still be landing.
        const bool ok = mbar_wait_abortable(&full[s], (g / kSlots) & 1, args.err, &s_abort);
        const uint32_t st = smem_u32(cring + s * kNf4ChunkBytes);
        const uint4 c0 = lds128(st + ((warp * 2 + 0) * 32 + lane) * 16);
        const uint4 c1 = lds128(st + ((warp * 2 + 1) * 32 + lane) * 16);
        const float s127 = __uint_as_float(lds32(st + kNf4S127Off));
        const int r0 = 16 * warp + g8;
        // scale codes of rows r0 and r0 + 8: (kh 0, kh 1) in the low / high byte
        const uint32_t s0 = lds16(st + kNf4ScaleOff + r0 * 2);
        const uint32_t s1 = lds16(st + kNf4ScaleOff + (r0 + 8) * 2);
        float am[2][2];
#pragma unroll
        for (int kh = 0; kh < 2; ++kh) {
          am[kh][0] = __fadd_rn(__fmul_rn(static_cast<float>(static_cast<int8_t>((s0 >> (8 * kh)) & 0xffu)), s127), off);
          am[kh][1] = __fadd_rn(__fmul_rn(static_cast<float>(static_cast<int8_t>((s1 >> (8 * kh)) & 0xffu)), s127), off);
        }
#pragma unroll
        for (int kh = 0; kh < 2; ++kh) {
          const uint4 cw = kh ? c1 : c0;
          const uint32_t words[4] = {cw.x, cw.y, cw.z, cw.w};
          const uint32_t xb = smem_u32(xring + s * kXBytes) + kh * MP * 128;
          float part[MT][4];
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) part[mt][0] = part[mt][1] = part[mt][2] = part[mt][3] = 0.f;
          // B fragments of the four k-steps: ldmatrix.x4 gives two k-steps
          // (four 8 x 8 tiles: 16-byte chunks 4h .. 4h + 3 of rows 8 mt ..)
          uint32_t bf[MT][2][4];
#pragma unroll
          for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int row = 8 * mt + (lane & 7), cc = 4 * h + (lane >> 3);
              ldsm_x4(xb + row * 128 + ((cc ^ (row & 7)) << 4), bf[mt][h]);
            }
#pragma unroll
          for (int ks = 0; ks < 4; ++ks) {
            uint32_t a[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              if constexpr (kLutRow == 256)  // offset (byte j) * 256 + 4 lane in one byte permute
                a[j] = lds32(lut_base + __byte_perm(words[ks], lane4, 0x5504u + (j << 4)));
              else  // byte j alone (one byte permute), then one shift-add
                a[j] = lds32(lut_base + lane4 + (__byte_perm(words[ks], 0u, 0x4440u + j) << 7));
            }
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
              const uint32_t b[2] = {bf[mt][ks >> 1][(ks & 1) * 2], bf[mt][ks >> 1][(ks & 1) * 2 + 1]};
              Mma<__half>::k16(part[mt], a, b);
            }
          }
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) {
            acc[mt][0] = fmaf(am[kh][0], part[mt][0], acc[mt][0]);
            acc[mt][1] = fmaf(am[kh][0], part[mt][1], acc[mt][1]);
            acc[mt][2] = fmaf(am[kh][1], part[mt][2], acc[mt][2]);
            acc[mt][3] = fmaf(am[kh][1], part[mt][3], acc[mt][3]);
          }
        }
        __syncwarp();
        if (lane == 0 && ok) mbar_arrive(&empty[s]);
      }
      // D fragment: rows n0 = tile*128 + 16 warp + g8 (acc 0, 1) and n0 + 8
      // (acc 2, 3); x rows 8 mt + 2t and + 1.
      const int nl = 16 * warp + g8;
      const int n0 = sg.tile * kNf4Tile + nl;
      if (sg.kc0 == 0 && sg.kc1 == sg.kt) {
        // the whole tile in this CTA's range
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
          store_y(pr, args.M, n0, 8 * mt + 2 * t, acc[mt][0], acc[mt][1], acc[mt][2], acc[mt][3]);
      } else {
        // A piece of a tile shared with the neighbouring CTAs: the first
        // piece of this CTA's range goes to its slot 0, the last to slot 1.
        float* part = args.partials + (static_cast<int64_t>(blockIdx.x) * 2 + (first_piece ? 0 : 1)) * kNf4Tile * MP;
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
          *reinterpret_cast<float2*>(part + nl * MP + 8 * mt + 2 * t) = make_float2(acc[mt][0], acc[mt][1]);
          *reinterpret_cast<float2*>(part + (nl + 8) * MP + 8 * mt + 2 * t) = make_float2(acc[mt][2], acc[mt][3]);
        }
        if (first_piece && c < c_end) {
          // the epilogue warp counts this piece; the range goes on
          __syncwarp();
          if (lane == 0) mbar_arrive(&first_piece_bar);
          continue;
        }
        // the tile's pieces come from CTAs g0 .. g1, in that order
        const int64_t t0 = pr.chunk_base + static_cast<int64_t>(sg.tile) * sg.kt;
        const int g0 = range_cta(C, G, t0), g1 = range_cta(C, G, t0 + sg.kt - 1);
        // one cumulative fence after the barrier orders every warp's
        // partial stores before the count
        named_sync(kNf4EpiBar, kNf4Warps * 32);
        int* cnt = args.counters + pr.counter_base + sg.tile;
        if (tid == 0) {
          __threadfence();
          const int old = atomicAdd(cnt, 1);
          s_fin = old == g1 - g0;
          if (s_fin) __threadfence();
        }
        named_sync(kNf4EpiBar, kNf4Warps * 32);
        if (s_fin) {
          finish_rows<MT>(args, pr, C, G, t0, g0, g1, sg.tile, warp, lane);
          named_sync(kNf4EpiBar, kNf4Warps * 32);
          if (tid == 0) *cnt = 0;  // every piece has counted: ready for the next launch
        }
      }
    }
  }
  __syncthreads();
}

}  // namespace

int nf4_sm_count() {
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
  return sms;
}

cudaError_t launch_nf4_absmax(const uint16_t* w, int64_t ldw, int N, int K, float* absmax, uint32_t* minmax,
                              cudaStream_t st) {
  nf4_minmax_init_kernel<<<1, 32, 0, st>>>(minmax);
  const int64_t blocks = static_cast<int64_t>(N) * (K / kNf4Block);
  int grid = static_cast<int>((blocks + 255) / 256);
  const int cap = 8 * (nf4_sm_count() > 0 ? nf4_sm_count() : 148);
  if (grid > cap) grid = cap;
  if (grid < 1) grid = 1;
  nf4_absmax_kernel<<<grid, 256, 0, st>>>(w, ldw, N, K, absmax, minmax);
  return cudaGetLastError();
}

cudaError_t launch_nf4_pack(const uint16_t* w, int64_t ldw, int N, int K, const float* absmax,
                            const uint32_t* minmax, uint8_t* packed, float* offset, cudaStream_t st) {
  nf4_pack_kernel<<<dim3(K / kNf4Tile, N / kNf4Tile), 256, 0, st>>>(w, ldw, N, K, absmax, minmax, packed, offset);
  return cudaGetLastError();
}

cudaError_t launch_nf4_dequant(const uint8_t* packed, const float* offset, int N, int K, uint16_t* w, int64_t ldw,
                               cudaStream_t st) {
  nf4_dequant_kernel<<<dim3(K / kNf4Tile, N / kNf4Tile), 256, 0, st>>>(packed, offset, N, K, w, ldw);
  return cudaGetLastError();
}

template <int MT>
static cudaError_t gemm_launch(const Nf4Maps& maps, const Nf4GemmArgs& args, cudaStream_t st) {
  auto kern = nf4_gemm_kernel<MT>;
  constexpr int smem = Nf4Cfg<MT>::kSmem;
  constexpr int kMaxDev = 64;
  // CTAs per SM, per device; racing first calls compute the same value
  static std::atomic<int> per_sm[kMaxDev];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDev) return cudaErrorInvalidDevice;
  int occ = per_sm[dev].load(std::memory_order_acquire);
  if (occ == 0) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kNf4Threads, smem);
    if (e != cudaSuccess) return e;
    if (occ < 1) occ = 1;
    per_sm[dev].store(occ, std::memory_order_release);
  }
  const int ctas = occ * nf4_sm_count();
  // never more CTAs than chunks, nor than the partial buffer was sized for
  int grid = ctas < args.max_ctas ? ctas : args.max_ctas;
  if (grid < 1) grid = 1;
  // programmatic dependent launch: the weight streaming of this kernel may
  // start while the kernel before it on the stream finishes
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kNf4Threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kern, maps, args);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

cudaError_t launch_nf4_gemm(const Nf4Maps& maps, const Nf4GemmArgs& args, int m_pad, cudaStream_t st) {
  switch (m_pad) {
    case 8: return gemm_launch<1>(maps, args, st);
    case 16: return gemm_launch<2>(maps, args, st);
    case 32: return gemm_launch<4>(maps, args, st);
    case 64: return gemm_launch<8>(maps, args, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace persona
