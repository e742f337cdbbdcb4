// Shared pieces of the BGMV kernels: CTA shape, ring geometry per rank, and
// the per-stage math on the 16-row warp-MMA tiles (shrink and expand).
//
// Math (reference persona/ops.py:12-56, csrc/bgmv_shrink.cu:9-45,
// csrc/bgmv_expand.cu:9-30): for every row t with slot s = slots[t] >= 0
//   shrink  v[t, r] = sum_k A[s, r, k] * x[t, k]                (fp32)
//   expand  y[t, n] = round(y[t, n] + sum_r B[s, n, r] * v[t, r]) (fp32 sum)
#pragma once

#include <type_traits>

#include "bgmv_args.h"
#include "common.cuh"
#include "plan_layout.h"

namespace persona {

constexpr int kConsumerWarps = 4;
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kBgmvThreads = kConsumers + 32;  // + one producer warp
constexpr int kCtasPerSm = 2;
constexpr int kSlotBytes = 21504;              // one ring slot (multiple of 1024)
constexpr int kSlots = 4;
constexpr int kItemRing = 4;
constexpr int kMaxR = 64;
constexpr int kNamedBarConsumers = 1;

template <int R>
struct RankCfg {
  static_assert(R == 8 || R == 16 || R == 32 || R == 64, "rank");
  // A stage: A tile (kKC k x R rows) + x chunk (16 rows x kKC, padded pitch).
  static constexpr int kKC = R >= 32 ? 128 : 256;
  static constexpr int kABoxBytes = 128 * R;  // TMA box {64 k, R rows}
  static constexpr int kXOff = kKC * 2 * R;   // byte offset of the x chunk in an A slot
  static constexpr int kXPitch = kKC * 2 + 16;
  static_assert(kXOff + kRowsPerItem * kXPitch <= kSlotBytes, "A slot");
  static constexpr int kNT = R / 8;                                    // 8-wide rank tiles
  static constexpr int kTPW = kNT >= kConsumerWarps ? kNT / kConsumerWarps : 1;  // rank tiles per warp
  static constexpr int kKS = kNT >= kConsumerWarps ? 1 : kConsumerWarps / kNT;   // warps splitting k per tile
  static constexpr int kMaxSteps = kKC / 16 / kKS;                     // k16 steps per warp per stage
  // B stage: B tile (2R bytes/row) + y tile (16 rows x 2 bytes/col) in one slot.
  static constexpr int kNBraw = (kSlotBytes - 16 * kRowsPerItem) / (2 * R + 2 * kRowsPerItem) / 8 * 8;
  static constexpr int kNB = kNBraw < 256 ? kNBraw : 256;
  static constexpr int kYOff = kNB * 2 * R;     // byte offset of the y tile in a B slot
  static constexpr int kYStride = kNB * 2 + 16;  // bytes per y-tile row (padded: rows land on distinct banks)
  static_assert(kYOff + kRowsPerItem * kYStride <= kSlotBytes, "B slot");
  static constexpr uint32_t kBSwz = (2 * R == 128) ? 7u : (2 * R == 64) ? 3u : (2 * R == 32) ? 1u : 0u;
  static constexpr int kKSteps = R >= 16 ? R / 16 : 1;  // expand: k16 steps over the rank
  static constexpr int kMaxTiles = (kNB / 8 + kConsumerWarps - 1) / kConsumerWarps;  // expand tiles per warp
};

// ---------------------------------------------------------------- shrink --
// One A stage: this warp's rank tiles d[t] (16 rows x 8 ranks) += x * A^T over
// the k16 steps it owns (warps sharing a rank tile split the steps).  All
// fragments are loaded before the MMAs, which alternate between two
// accumulators, so shared-memory and MMA latency overlap.
template <typename DT, int R>
__device__ __forceinline__ void shrink_stage(const uint8_t* stage, int ksteps, int warp, int lane,
                                             float (&d)[RankCfg<R>::kTPW][2][4]) {
  using C = RankCfg<R>;
  const uint32_t abase = smem_u32(stage);
  const uint32_t x16 = abase + C::kXOff + (lane & 15) * C::kXPitch + ((lane >> 4) * 8) * 2;
  const int ksplit = warp % C::kKS;
  const int tile0 = (warp / C::kKS) * C::kTPW;
  const int uofs = (lane >> 3) & 1;
  uint32_t a[C::kMaxSteps][4], b[C::kMaxSteps][C::kTPW][2];
#pragma unroll
  for (int i = 0; i < C::kMaxSteps; ++i) {
    const int ks = ksplit + i * C::kKS;
    if (ks < ksteps) {
      ldsm_x4(x16 + ks * 32, a[i]);
      const int ku = ks * 2 + uofs;
      const int bx = ku >> 3, u = ku & 7;
#pragma unroll
      for (int t = 0; t < C::kTPW; ++t) {
        const int r = (tile0 + t) * 8 + (lane & 7);
        ldsm_x2(abase + bx * C::kABoxBytes + r * 128 + ((u ^ (r & 7)) << 4), b[i][t]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < C::kMaxSteps; ++i) {
    if (ksplit + i * C::kKS < ksteps) {
#pragma unroll
      for (int t = 0; t < C::kTPW; ++t) Mma<DT>::k16(d[t][i & 1], a[i], b[i][t]);
    }
  }
}

// ---------------------------------------------------------------- expand --
// One B stage: for each 8-column tile this warp owns,
// y[row][n] = round(y_tile[row][n] + scale * (v_hi + v_lo)[row] . B[n]).
// The slot is released (relaxed arrive on `empty`) as soon as its data is in
// registers, before the y stores, so that no arrive waits on global stores;
// `empty` is null when the stage's wait gave up (the slot stays held).
template <typename DT, int R>
__device__ __forceinline__ void expand_stage(const uint8_t* stage, const uint32_t (&vhi)[RankCfg<R>::kKSteps][4],
                                             const uint32_t (&vlo)[RankCfg<R>::kKSteps][4], int rows_here,
                                             int n_box, int n0, int c, const int* rows, uint16_t* y, int64_t ldy,
                                             float scale, int warp, int lane, uint64_t* empty) {
  using C = RankCfg<R>;
  constexpr int kMT = C::kMaxTiles;
  constexpr int KS = C::kKSteps;
  const uint32_t sbase = smem_u32(stage);
  const uint32_t ytile = sbase + C::kYOff;
  const int g = lane >> 2, t = lane & 3;
  const int tiles = rows_here >> 3;
  uint32_t bf[kMT][KS][2];
#pragma unroll
  for (int ti = 0; ti < kMT; ++ti) {
    const int tile = warp + ti * kConsumerWarps;
    if (tile < tiles) {
      const int nl = tile * 8;
      const int bx = nl / n_box;
      const int rib = nl - bx * n_box + (lane & 7);
      const uint32_t boff = sbase + static_cast<uint32_t>(bx * n_box * 2 * R);
      if (R >= 16) {
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
          const int u = ks * 2 + ((lane >> 3) & 1);
          ldsm_x2(boff + swz(static_cast<uint32_t>(rib * 2 * R + u * 16), C::kBSwz), bf[ti][ks]);
        }
      } else {
        ldsm_x1(boff + static_cast<uint32_t>(rib * 2 * R), bf[ti][0][0]);
      }
    }
  }
  float dh[kMT][4], dl[kMT][4];
#pragma unroll
  for (int ti = 0; ti < kMT; ++ti) {
#pragma unroll
    for (int i = 0; i < 4; ++i) dh[ti][i] = dl[ti][i] = 0.f;
    if (warp + ti * kConsumerWarps < tiles) {
      if (R >= 16) {
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
          Mma<DT>::k16(dh[ti], vhi[ks], bf[ti][ks]);
          Mma<DT>::k16(dl[ti], vlo[ks], bf[ti][ks]);
        }
      } else {
        const uint32_t ah[2] = {vhi[0][0], vhi[0][1]};
        const uint32_t al[2] = {vlo[0][0], vlo[0][1]};
        Mma<DT>::k8(dh[ti], ah, bf[ti][0][0]);
        Mma<DT>::k8(dl[ti], al, bf[ti][0][0]);
      }
    }
  }
  uint32_t out[kMT][2];
#pragma unroll
  for (int ti = 0; ti < kMT; ++ti) {
    const int tile = warp + ti * kConsumerWarps;
    // dh/dl[0..1]: row g, columns nl+2t, nl+2t+1; [2..3]: row g+8.
    const int col = tile * 8 + 2 * t;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int row = g + 8 * h;
      out[ti][h] = 0u;
      if (tile < tiles && row < c) {
        const uint32_t yw = lds32(ytile + row * C::kYStride + col * 2);
        const float2 yo = Cvt<DT>::to2(yw);
        const float s0 = dh[ti][2 * h] + dl[ti][2 * h], s1 = dh[ti][2 * h + 1] + dl[ti][2 * h + 1];
        out[ti][h] = Mma<DT>::pack(yo.x + scale * s0, yo.y + scale * s1);
      }
    }
  }
  const int row0 = g < c ? static_cast<int>(lds32(smem_u32(rows + g))) : 0;
  const int row1 = g + 8 < c ? static_cast<int>(lds32(smem_u32(rows + g + 8))) : 0;
  __syncwarp();
  if (lane == 0 && empty != nullptr) mbar_arrive_relaxed(empty);
#pragma unroll
  for (int ti = 0; ti < kMT; ++ti) {
    const int tile = warp + ti * kConsumerWarps;
    const int col = tile * 8 + 2 * t;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int row = g + 8 * h;
      if (tile < tiles && row < c)
        *reinterpret_cast<uint32_t*>(y + static_cast<int64_t>(h ? row1 : row0) * ldy + n0 + col) = out[ti][h];
    }
  }
}

// A-operand fragments of v (rows x rank, fp32 in smem, row stride R) for the
// expand MMAs: v * 2^-e split into a 16-bit high part and the 16-bit
// rounding of the remainder.
template <typename DT, int R>
__device__ __forceinline__ void v_fragments(const float* vf, float scale_down, int lane,
                                            uint32_t (&vhi)[RankCfg<R>::kKSteps][4],
                                            uint32_t (&vlo)[RankCfg<R>::kKSteps][4]) {
  using C = RankCfg<R>;
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int ks = 0; ks < C::kKSteps; ++ks) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      // register i: (row g | g+8) x (k 2t,2t+1 | +8) as in the m16n8k16 A layout
      const int row = g + 8 * (i & 1);
      const int k = ks * 16 + 2 * t + 8 * (i >> 1);
      if (R < 16 && i >= 2) {
        vhi[ks][i] = 0u;
        vlo[ks][i] = 0u;
        continue;
      }
      const float2 v = *reinterpret_cast<const float2*>(vf + row * R + k);
      const float a = v.x * scale_down, b = v.y * scale_down;
      const float ha = Mma<DT>::round_trip(a), hb = Mma<DT>::round_trip(b);
      vhi[ks][i] = Mma<DT>::pack(ha, hb);
      vlo[ks][i] = Mma<DT>::pack(a - ha, b - hb);
    }
  }
}

}  // namespace persona
