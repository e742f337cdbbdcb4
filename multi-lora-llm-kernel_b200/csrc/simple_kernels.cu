// Small kernels outside the split hot path:
// * a row-by-row shrink for ranks the split kernel does not specialise
//   (the reference's shrink accepts any R: csrc/bgmv_shrink.cu:56-58),
// * the warm-up fp16 GEMV kept behind torch.ops.persona.gemv_fp16
//   (reference csrc/gemv_fp16.cu:9-31: y[n] = W[n, :] . x, fp32 accumulate).
#include "bgmv_args.h"
#include "common.cuh"

namespace persona {

// One CTA per row; each warp computes whole rank entries with 16-byte loads.
template <typename DT>
__global__ void __launch_bounds__(256)
    shrink_rowwise_kernel(const uint16_t* __restrict__ x, int64_t ldx,
                          const uint16_t* __restrict__ a_pool, int64_t a_slot_stride,
                          int64_t a_row_stride, const int32_t* __restrict__ slots,
                          float* __restrict__ v, int K, int R, int S, int32_t* err) {
  const int t = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int s = slots[t];
  if (s < 0 || s >= S) {
    if (s < -1 || s >= S) {
      if (threadIdx.x == 0) raise_error(err, PERSONA_DEV_ERR_SLOT);
    }
    for (int r = threadIdx.x; r < R; r += blockDim.x) v[static_cast<int64_t>(t) * R + r] = 0.f;
    return;
  }
  const uint16_t* xr = x + static_cast<int64_t>(t) * ldx;
  for (int r = warp; r < R; r += blockDim.x >> 5) {
    const uint16_t* ar = a_pool + static_cast<int64_t>(s) * a_slot_stride + static_cast<int64_t>(r) * a_row_stride;
    float acc = 0.f;
    for (int k = lane * 8; k < K; k += 32 * 8) {
      const uint4 av = *reinterpret_cast<const uint4*>(ar + k);
      const uint4 xv = *reinterpret_cast<const uint4*>(xr + k);
      const uint32_t aw[4] = {av.x, av.y, av.z, av.w};
      const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 af = Cvt<DT>::to2(aw[i]);
        const float2 xf = Cvt<DT>::to2(xw[i]);
        acc = fmaf(af.x, xf.x, acc);
        acc = fmaf(af.y, xf.y, acc);
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (lane == 0) v[static_cast<int64_t>(t) * R + r] = acc;
  }
}

cudaError_t launch_shrink_rowwise(int dtype, const void* x, int64_t ldx, const void* a_pool,
                                  int64_t a_slot_stride, int64_t a_row_stride,
                                  const int32_t* slots, float* v, int T, int K, int R, int S,
                                  int32_t* err, cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  const uint16_t* xp = static_cast<const uint16_t*>(x);
  const uint16_t* ap = static_cast<const uint16_t*>(a_pool);
  if (dtype == PERSONA_DTYPE_BF16)
    shrink_rowwise_kernel<__nv_bfloat16><<<T, 256, 0, st>>>(xp, ldx, ap, a_slot_stride, a_row_stride,
                                                            slots, v, K, R, S, err);
  else
    shrink_rowwise_kernel<__half><<<T, 256, 0, st>>>(xp, ldx, ap, a_slot_stride, a_row_stride, slots,
                                                     v, K, R, S, err);
  return cudaGetLastError();
}

// One warp per output row; 16-byte loads when the row is aligned.
__global__ void __launch_bounds__(128)
    gemv_fp16_kernel(const __half* __restrict__ x, const __half* __restrict__ W,
                     __half* __restrict__ y, int K, int N) {
  const int n = blockIdx.x * 4 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (n >= N) return;
  const __half* w = W + static_cast<int64_t>(n) * K;
  float acc = 0.f;
  const bool vec = (K % 8 == 0) && ((reinterpret_cast<uintptr_t>(W) & 15) == 0) &&
                   ((reinterpret_cast<uintptr_t>(x) & 15) == 0);
  if (vec) {
    for (int k = lane * 8; k < K; k += 256) {
      const uint4 wv = *reinterpret_cast<const uint4*>(w + k);
      const uint4 xv = *reinterpret_cast<const uint4*>(x + k);
      const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
      const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 a = Cvt<__half>::to2(ww[i]);
        const float2 b = Cvt<__half>::to2(xw[i]);
        acc = fmaf(a.x, b.x, acc);
        acc = fmaf(a.y, b.y, acc);
      }
    }
  } else {
    for (int k = lane; k < K; k += 32) acc = fmaf(__half2float(w[k]), __half2float(x[k]), acc);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (lane == 0) y[n] = __float2half_rn(acc);
}

cudaError_t launch_gemv_fp16(const void* x, const void* W, void* y, int K, int N, cudaStream_t st) {
  if (N == 0) return cudaSuccess;
  gemv_fp16_kernel<<<(N + 3) / 4, 128, 0, st>>>(static_cast<const __half*>(x),
                                                static_cast<const __half*>(W),
                                                static_cast<__half*>(y), K, N);
  return cudaGetLastError();
}

}  // namespace persona
