// Small fused kernels of the end-to-end decode loop around the LoRA layers
// (Mistral-7B architecture, fp16): residual add + RMSNorm, rotary embedding
// + KV-cache write, SiLU(gate) * up, and GQA attention of one new token per
// sequence over its cache.  Each replaces several elementwise launches of the
// reference's Hugging Face model (reference persona/engine.py:101-107 runs
// model.generate); the arithmetic follows that model's fp16 conventions:
// RMSNorm in fp32 then weight * fp16(x * rsqrt(mean(x^2) + eps)); RoPE with
// the rotate-half layout; SiLU rounded to fp16 before the product.
#include <cuda_fp16.h>

#include <cstdint>

#include "decode_args.h"

namespace persona {
namespace {

__device__ __forceinline__ float h2f(__half h) { return __half2float(h); }

// h[r] += delta[r] (fp16, when delta is given); out[r] = w * fp16(h / rms).
// One CTA of 256 threads per row, D a multiple of 8.
__global__ void __launch_bounds__(256) add_rmsnorm_kernel(__half* __restrict__ h, const __half* __restrict__ delta,
                                                          const __half* __restrict__ w, __half* __restrict__ out,
                                                          int D, float eps) {
  const int r = blockIdx.x;
  __half* hr = h + static_cast<int64_t>(r) * D;
  const __half* dr = delta ? delta + static_cast<int64_t>(r) * D : nullptr;
  __half* orow = out + static_cast<int64_t>(r) * D;
  __shared__ float s_red[8];
  float ss = 0.f;
  for (int i = threadIdx.x * 8; i < D; i += 256 * 8) {
    uint4 hv = *reinterpret_cast<const uint4*>(hr + i);
    __half* hp = reinterpret_cast<__half*>(&hv);
    if (dr) {
      const uint4 dv = *reinterpret_cast<const uint4*>(dr + i);
      const __half* dp = reinterpret_cast<const __half*>(&dv);
#pragma unroll
      for (int k = 0; k < 8; ++k) hp[k] = __float2half_rn(h2f(hp[k]) + h2f(dp[k]));
      *reinterpret_cast<uint4*>(hr + i) = hv;
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) ss += h2f(hp[k]) * h2f(hp[k]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int k = 0; k < 8; ++k) tot += s_red[k];
  const float inv = rsqrtf(tot / static_cast<float>(D) + eps);
  for (int i = threadIdx.x * 8; i < D; i += 256 * 8) {
    const uint4 hv = *reinterpret_cast<const uint4*>(hr + i);
    const uint4 wv = *reinterpret_cast<const uint4*>(w + i);
    const __half* hp = reinterpret_cast<const __half*>(&hv);
    const __half* wp = reinterpret_cast<const __half*>(&wv);
    uint4 ov;
    __half* op = reinterpret_cast<__half*>(&ov);
#pragma unroll
    for (int k = 0; k < 8; ++k) op[k] = __hmul(wp[k], __float2half_rn(h2f(hp[k]) * inv));
    *reinterpret_cast<uint4*>(orow + i) = ov;
  }
}

// Rows r = b * per_seq + i of q [rows, Hq, 128] and k / v [rows, Hkv, 128]
// sit at position *start + i of sequence b.  q and k are rotated in place
// (rotate-half layout, angle = pos * theta^(-2j/128), computed in fp32);
// k and v are written to the caches [B, Hkv, L, 128].  One CTA per row,
// 64 threads per head pair (j = 0..63 handles dims j and j + 64).
__global__ void rope_cache_kernel(__half* __restrict__ q, __half* __restrict__ k, const __half* __restrict__ v,
                                  __half* __restrict__ kc, __half* __restrict__ vc, const int* __restrict__ start,
                                  int per_seq, int Hq, int Hkv, int L, float log2_theta) {
  constexpr int D = 128;
  const int r = blockIdx.x;
  const int b = r / per_seq, pos = *start + (r - b * per_seq);
  if (pos >= L) return;
  const int j = threadIdx.x & 63;
  // inv_freq = theta^(-2j/D), angle in fp32
  const float inv_freq = exp2f(-log2_theta * static_cast<float>(2 * j) / static_cast<float>(D));
  float sn, cs;
  sincosf(static_cast<float>(pos) * inv_freq, &sn, &cs);
  const __half c = __float2half_rn(cs), s = __float2half_rn(sn);
  for (int hh = threadIdx.x >> 6; hh < Hq + Hkv; hh += blockDim.x >> 6) {
    __half* x = hh < Hq ? q + (static_cast<int64_t>(r) * Hq + hh) * D : k + (static_cast<int64_t>(r) * Hkv + hh - Hq) * D;
    const __half x1 = x[j], x2 = x[j + 64];
    const __half o1 = __hsub(__hmul(x1, c), __hmul(x2, s));
    const __half o2 = __hadd(__hmul(x2, c), __hmul(x1, s));
    x[j] = o1;
    x[j + 64] = o2;
    if (hh >= Hq) {
      const int kh = hh - Hq;
      const int64_t dst = ((static_cast<int64_t>(b) * Hkv + kh) * L + pos) * D;
      const __half* vr = v + (static_cast<int64_t>(r) * Hkv + kh) * D;
      kc[dst + j] = o1;
      kc[dst + j + 64] = o2;
      vc[dst + j] = vr[j];
      vc[dst + j + 64] = vr[j + 64];
    }
  }
}

// out = fp16(fp16(silu(g)) * u), n a multiple of 8.
__global__ void silu_mul_kernel(const __half* __restrict__ g, const __half* __restrict__ u, __half* __restrict__ out,
                                int64_t n) {
  for (int64_t i = (blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x) * 8; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x * 8) {
    const uint4 gv = *reinterpret_cast<const uint4*>(g + i);
    const uint4 uv = *reinterpret_cast<const uint4*>(u + i);
    const __half* gp = reinterpret_cast<const __half*>(&gv);
    const __half* up = reinterpret_cast<const __half*>(&uv);
    uint4 ov;
    __half* op = reinterpret_cast<__half*>(&ov);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float x = h2f(gp[k]);
      const __half sl = __float2half_rn(x / (1.f + __expf(-x)));
      op[k] = __float2half_rn(h2f(sl) * h2f(up[k]));
    }
    *reinterpret_cast<uint4*>(out + i) = ov;
  }
}

// One new token per sequence: out[b, h] = softmax(q[b, h] K[b, h / G]^T *
// scale) V[b, h / G] over positions [0, *len).  One CTA per (sequence, kv
// head), one warp per query head of the group (G = Hq / Hkv <= 8); the
// cache is staged 32 positions at a time, rows padded to 65 words so that a
// lane per position reads without bank conflicts.
constexpr int kAttnChunk = 32;
constexpr int kAttnPitch = 130;  // halves per staged row (65 words)

__global__ void decode_attention_kernel(const __half* __restrict__ q, const __half* __restrict__ kc,
                                        const __half* __restrict__ vc, const int* __restrict__ len_ptr,
                                        __half* __restrict__ out, int Hq, int Hkv, int L, float scale) {
  constexpr int D = 128;
  const int b = blockIdx.x, kh = blockIdx.y;
  const int G = Hq / Hkv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = kh * G + warp;
  const int len = min(*len_ptr, L);
  __shared__ __half ks[kAttnChunk * kAttnPitch];
  __shared__ __half vs[kAttnChunk * kAttnPitch];
  __shared__ float qs[8][D];
  if (warp < G)
    for (int d = lane; d < D; d += 32) qs[warp][d] = h2f(q[(static_cast<int64_t>(b) * Hq + h) * D + d]);
  const __half* kb = kc + (static_cast<int64_t>(b) * Hkv + kh) * L * D;
  const __half* vb = vc + (static_cast<int64_t>(b) * Hkv + kh) * L * D;
  float m = -INFINITY, l = 0.f;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};  // dims 4 lane .. 4 lane + 3
  for (int p0 = 0; p0 < len; p0 += kAttnChunk) {
    const int n = min(kAttnChunk, len - p0);
    __syncthreads();
    for (int e = threadIdx.x; e < kAttnChunk * (D / 2); e += blockDim.x) {
      const int pr = e / (D / 2), c2 = e - pr * (D / 2);
      uint32_t kv = 0, vv = 0;
      if (pr < n) {
        kv = reinterpret_cast<const uint32_t*>(kb + static_cast<int64_t>(p0 + pr) * D)[c2];
        vv = reinterpret_cast<const uint32_t*>(vb + static_cast<int64_t>(p0 + pr) * D)[c2];
      }
      reinterpret_cast<uint32_t*>(ks + pr * kAttnPitch)[c2] = kv;
      reinterpret_cast<uint32_t*>(vs + pr * kAttnPitch)[c2] = vv;
    }
    __syncthreads();
    if (warp < G) {
      float sc = -INFINITY;
      if (lane < n) {
        const __half* kr = ks + lane * kAttnPitch;
        float dot = 0.f;
#pragma unroll 8
        for (int d = 0; d < D; d += 2) {
          const float2 kf = __half22float2(*reinterpret_cast<const __half2*>(kr + d));
          dot = fmaf(qs[warp][d], kf.x, dot);
          dot = fmaf(qs[warp][d + 1], kf.y, dot);
        }
        sc = dot * scale;
      }
      float mx = sc;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float m_new = fmaxf(m, mx);
      const float corr = __expf(m - m_new);
      const float pw = lane < n ? __expf(sc - m_new) : 0.f;
      float ps = pw;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
      l = l * corr + ps;
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[i] *= corr;
      for (int pr = 0; pr < n; ++pr) {
        const float wgt = __shfl_sync(0xffffffffu, pw, pr);
        const __half* vr = vs + pr * kAttnPitch + 4 * lane;
        const float2 v0 = __half22float2(*reinterpret_cast<const __half2*>(vr));
        const float2 v1 = __half22float2(*reinterpret_cast<const __half2*>(vr + 2));
        acc[0] = fmaf(wgt, v0.x, acc[0]);
        acc[1] = fmaf(wgt, v0.y, acc[1]);
        acc[2] = fmaf(wgt, v1.x, acc[2]);
        acc[3] = fmaf(wgt, v1.y, acc[3]);
      }
      m = m_new;
    }
  }
  if (warp < G) {
    const float inv = l > 0.f ? 1.f / l : 0.f;
    __half* o = out + (static_cast<int64_t>(b) * Hq + h) * D + 4 * lane;
#pragma unroll
    for (int i = 0; i < 4; ++i) o[i] = __float2half_rn(acc[i] * inv);
  }
}

}  // namespace

cudaError_t launch_add_rmsnorm(void* h, const void* delta, const void* w, void* out, int rows, int D, float eps,
                               cudaStream_t st) {
  add_rmsnorm_kernel<<<rows, 256, 0, st>>>(static_cast<__half*>(h), static_cast<const __half*>(delta),
                                           static_cast<const __half*>(w), static_cast<__half*>(out), D, eps);
  return cudaGetLastError();
}

cudaError_t launch_rope_cache(void* q, void* k, const void* v, void* kc, void* vc, const int* start, int rows,
                              int per_seq, int Hq, int Hkv, int L, float log2_theta, cudaStream_t st) {
  rope_cache_kernel<<<rows, 256, 0, st>>>(static_cast<__half*>(q), static_cast<__half*>(k),
                                          static_cast<const __half*>(v), static_cast<__half*>(kc),
                                          static_cast<__half*>(vc), start, per_seq, Hq, Hkv, L, log2_theta);
  return cudaGetLastError();
}

cudaError_t launch_silu_mul(const void* g, const void* u, void* out, int64_t n, cudaStream_t st) {
  int64_t blocks = (n / 8 + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  if (blocks < 1) blocks = 1;
  silu_mul_kernel<<<static_cast<int>(blocks), 256, 0, st>>>(static_cast<const __half*>(g),
                                                            static_cast<const __half*>(u), static_cast<__half*>(out), n);
  return cudaGetLastError();
}

cudaError_t launch_decode_attention(const void* q, const void* kc, const void* vc, const int* len, void* out, int B,
                                    int Hq, int Hkv, int L, float scale, cudaStream_t st) {
  decode_attention_kernel<<<dim3(B, Hkv), 32 * (Hq / Hkv), 0, st>>>(
      static_cast<const __half*>(q), static_cast<const __half*>(kc), static_cast<const __half*>(vc), len,
      static_cast<__half*>(out), Hq, Hkv, L, scale);
  return cudaGetLastError();
}

}  // namespace persona
