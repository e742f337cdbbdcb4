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

#include <cooperative_groups.h>

#include "decode_args.h"

namespace persona {
namespace cg = cooperative_groups;
namespace {

__device__ __forceinline__ float h2f(__half h) { return __half2float(h); }

// Every kernel here is launched as a programmatic dependent of the kernel
// before it (the LoRA kernel, the attention or the norm), so that it is
// resident when that kernel ends.  Each one waits here, before its first read
// or write, until the kernel before it has finished and its writes are
// visible (no CTA returns before this point, so the grid never completes
// ahead of that kernel), and only then lets its own dependent launch: a
// dependent launched earlier would hold SMs while two kernels still run.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// cudaLaunchKernelEx with programmatic stream serialization allowed.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

// h[r] += delta[r] (fp16, when delta is given); out[r] = w * fp16(h / rms).
// One CTA of 256 threads per row, D a multiple of 8.
__global__ void __launch_bounds__(256) add_rmsnorm_kernel(__half* __restrict__ h, const __half* __restrict__ delta,
                                                          const __half* __restrict__ w, __half* __restrict__ out,
                                                          int D, float eps) {
  pdl_wait();
  asm volatile("griddepcontrol.launch_dependents;");  // a dependent NF4 GEMM may start streaming weights
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
  pdl_wait();
  asm volatile("griddepcontrol.launch_dependents;");
  const int r = blockIdx.x;
  const int b = r / per_seq, pos = *start + (r - b * per_seq);
  if (pos < 0 || pos >= L) return;
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
  pdl_wait();
  asm volatile("griddepcontrol.launch_dependents;");
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
// scale) V[b, h / G] over positions [0, *len).  One thread-block cluster of
// P CTAs (128 threads each) per (sequence, kv head) computes the G = Hq / Hkv
// <= 8 query heads that share the cache rows, so K and V are read once; the
// positions are cut into P equal ranges, one per CTA, so that B * Hkv * P
// CTAs (not B * Hkv) stream the cache.  Per CTA: scores, a thread per
// position (16-byte loads of its K row, G dot products, q in shared memory);
// the softmax statistics of its range (max m, sum l of exp(s - m)); P V as 8
// position groups x 16 column chunks of 8 dims (16-byte V loads), summed
// over the groups in shared memory.  The CTAs then combine their ranges
// through distributed shared memory: out = sum_r e^(m_r - M) acc_r /
// sum_r e^(m_r - M) l_r with M = max_r m_r, each CTA writing a slice of the
// output.
constexpr int kAttnThreads = 128;
constexpr int kAttnMaxSplit = 8;  // CTAs per cluster (portable maximum)
constexpr int kAttnChunk = 64;    // positions per CTA the split aims at

// With a position (rope.pos != nullptr), rank 0 of the cluster first does
// what rope_cache_kernel does for this (sequence, kv head), with the same
// arithmetic: it rotates the G query heads and the k head of the new token
// in place and writes k and v to the caches at *pos (nothing at all when
// *pos is outside [0, L)); after a cluster barrier every CTA reads them back.
struct RopeIn {
  __half* q;  // [B, Hq, 128], rotated in place (and read below)
  __half* k;  // [B, Hkv, 128], rotated in place
  const __half* v;
  __half* kc;  // the caches, written at *pos
  __half* vc;
  const int* pos;
  float log2_theta;
};

__device__ __forceinline__ void rope_pair(__half* x, int j, __half c, __half s, __half& o1, __half& o2) {
  const __half x1 = x[j], x2 = x[j + 64];
  o1 = __hsub(__hmul(x1, c), __hmul(x2, s));
  o2 = __hadd(__hmul(x2, c), __hmul(x1, s));
  x[j] = o1;
  x[j + 64] = o2;
}

// q, kc and vc are not restrict: with a position they are written above
// their reads, through rope.  cmax: the largest range a CTA can get,
// ceil(L / P), which sizes the score buffer.
__global__ void __launch_bounds__(kAttnThreads) decode_attention_kernel(
    const __half* q, const __half* kc, const __half* vc, const int* __restrict__ len_ptr, __half* __restrict__ out,
    int Hq, int Hkv, int L, int cmax, float scale, const RopeIn rope) {
  constexpr int D = 128;
  cg::cluster_group cluster = cg::this_cluster();
  const int P = static_cast<int>(cluster.num_blocks());
  const int rank = static_cast<int>(cluster.block_rank());
  pdl_wait();
  asm volatile("griddepcontrol.launch_dependents;");
  const int b = blockIdx.x, kh = blockIdx.y, tid = threadIdx.x;
  const int G = Hq / Hkv;
  const int len = min(*len_ptr, L);
  const int chunk = (len + P - 1) / P;
  const int p0 = min(len, rank * chunk), p1 = min(len, p0 + chunk);
  extern __shared__ float attn_smem[];
  float* sc = attn_smem;          // [G][cmax] scores, then exp(s - m)
  float* part = sc + G * cmax;    // [8][G][D] P V per position group
  float* qs = part + 8 * G * D;   // [G][D]
  float* accs = qs + G * D;       // [G][D] this range's unnormalised P V
  __shared__ float s_m[8], s_l[8];
  // With a position: every CTA rotates this kv head's query heads itself
  // (the rotary kernel's half arithmetic), and the CTA whose range holds the
  // position (rank 0 if none does) rotates k and writes the new cache row,
  // which only that CTA reads back.  So no CTA waits for another before
  // scoring; rank 0 writes the rotated q back once every CTA of the cluster
  // has read the original (after the cluster barrier below).
  const int pos = rope.pos != nullptr ? *rope.pos : -1;
  const bool rot = rope.pos != nullptr && pos >= 0 && pos < L;
  const int owner = !rot ? -1 : pos < len ? pos / chunk : 0;
  const __half* qg = q + (static_cast<int64_t>(b) * Hq + kh * G) * D;
  if (rot) {
    for (int i = tid; i < G * 64; i += kAttnThreads) {
      const int h = i >> 6, j = i & 63;
      const float inv_freq = exp2f(-rope.log2_theta * static_cast<float>(2 * j) / static_cast<float>(D));
      float sn, cs;
      sincosf(static_cast<float>(pos) * inv_freq, &sn, &cs);
      const __half c = __float2half_rn(cs), sv = __float2half_rn(sn);
      const __half x1 = qg[h * D + j], x2 = qg[h * D + j + 64];
      qs[h * D + j] = __half2float(__hsub(__hmul(x1, c), __hmul(x2, sv)));
      qs[h * D + j + 64] = __half2float(__hadd(__hmul(x2, c), __hmul(x1, sv)));
    }
    if (rank == owner && tid < 64) {
      const int j = tid;
      const float inv_freq = exp2f(-rope.log2_theta * static_cast<float>(2 * j) / static_cast<float>(D));
      float sn, cs;
      sincosf(static_cast<float>(pos) * inv_freq, &sn, &cs);
      const __half c = __float2half_rn(cs), sv = __float2half_rn(sn);
      __half o1, o2;
      rope_pair(rope.k + (static_cast<int64_t>(b) * Hkv + kh) * D, j, c, sv, o1, o2);
      const int64_t dst = ((static_cast<int64_t>(b) * Hkv + kh) * L + pos) * D;
      const __half* vr = rope.v + (static_cast<int64_t>(b) * Hkv + kh) * D;
      rope.kc[dst + j] = o1;
      rope.kc[dst + j + 64] = o2;
      rope.vc[dst + j] = vr[j];
      rope.vc[dst + j + 64] = vr[j + 64];
    }
  } else {
    for (int i = tid; i < G * D; i += kAttnThreads) qs[i] = __half2float(qg[i]);
  }
  __syncthreads();
  const __half* kb = kc + (static_cast<int64_t>(b) * Hkv + kh) * L * D;
  const __half* vb = vc + (static_cast<int64_t>(b) * Hkv + kh) * L * D;
  // scores
  for (int p = p0 + tid; p < p1; p += kAttnThreads) {
    const uint4* kr = reinterpret_cast<const uint4*>(kb + static_cast<int64_t>(p) * D);
    uint4 kv[D / 8];
#pragma unroll
    for (int i = 0; i < D / 8; ++i) kv[i] = kr[i];
    for (int h = 0; h < G; ++h) {
      const float* qh = qs + h * D;
      float dot = 0.f;
#pragma unroll
      for (int i = 0; i < D / 8; ++i) {
        const __half2* k2 = reinterpret_cast<const __half2*>(&kv[i]);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 kf = __half22float2(k2[j]);
          dot = fmaf(qh[8 * i + 2 * j], kf.x, dot);
          dot = fmaf(qh[8 * i + 2 * j + 1], kf.y, dot);
        }
      }
      sc[h * cmax + (p - p0)] = dot * scale;
    }
  }
  __syncthreads();
  // softmax statistics of this range per head: warp w reduces heads w, w + 4
  const int warp = tid >> 5, lane = tid & 31;
  const int n = p1 - p0;
  for (int h = warp; h < G; h += kAttnThreads / 32) {
    float m = -INFINITY;
    for (int p = lane; p < n; p += 32) m = fmaxf(m, sc[h * cmax + p]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float l = 0.f;
    for (int p = lane; p < n; p += 32) {
      const float e = __expf(sc[h * cmax + p] - m);
      sc[h * cmax + p] = e;
      l += e;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    if (lane == 0) {
      s_m[h] = m;
      s_l[h] = l;
    }
  }
  __syncthreads();
  // P V over this range: position group pg, 8-dim column chunk dc
  const int pg = tid >> 4, dc = tid & 15;
  float acc[8][8];
#pragma unroll
  for (int h = 0; h < 8; ++h)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[h][j] = 0.f;
  for (int q0 = pg; q0 < n; q0 += 8 * 8) {
    uint4 vv[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int p = q0 + 8 * i;
      vv[i] = p < n ? reinterpret_cast<const uint4*>(vb + static_cast<int64_t>(p0 + p) * D)[dc] : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int p = q0 + 8 * i;
      if (p < n) {
        const __half2* v2 = reinterpret_cast<const __half2*>(&vv[i]);
#pragma unroll
        for (int h = 0; h < 8; ++h) {
          if (h < G) {
            const float w = sc[h * cmax + p];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float2 vf = __half22float2(v2[j]);
              acc[h][2 * j] = fmaf(w, vf.x, acc[h][2 * j]);
              acc[h][2 * j + 1] = fmaf(w, vf.y, acc[h][2 * j + 1]);
            }
          }
        }
      }
    }
  }
#pragma unroll
  for (int h = 0; h < 8; ++h)
    if (h < G)
#pragma unroll
      for (int j = 0; j < 8; ++j) part[(pg * G + h) * D + 8 * dc + j] = acc[h][j];
  __syncthreads();
  for (int i = tid; i < G * D; i += kAttnThreads) {
    float sum = 0.f;
#pragma unroll
    for (int g = 0; g < 8; ++g) sum += part[g * G * D + i];
    accs[i] = sum;
  }
  // every range's statistics and P V are in its CTA's shared memory, and
  // every CTA has read the original q
  cluster.sync();
  if (rot && rank == 0)
    for (int i = tid; i < G * D; i += kAttnThreads)
      rope.q[(static_cast<int64_t>(b) * Hq + kh * G) * D + i] = __float2half_rn(qs[i]);
  // combine the ranges, in rank order: this CTA writes outputs
  // [rank * G * D / P, (rank + 1) * G * D / P)
  const int o0 = rank * G * D / P, o1 = (rank + 1) * G * D / P;
  for (int i = o0 + tid; i < o1; i += kAttnThreads) {
    const int h = i / D;
    float M = -INFINITY;
    for (int r = 0; r < P; ++r) M = fmaxf(M, *cluster.map_shared_rank(&s_m[h], r));
    float num = 0.f, den = 0.f;
    if (M != -INFINITY) {
      for (int r = 0; r < P; ++r) {
        const float w = __expf(*cluster.map_shared_rank(&s_m[h], r) - M);
        num = fmaf(w, *cluster.map_shared_rank(accs + i, r), num);
        den = fmaf(w, *cluster.map_shared_rank(&s_l[h], r), den);
      }
    }
    out[(static_cast<int64_t>(b) * Hq + kh * G) * D + i] = __float2half_rn(den > 0.f ? num / den : 0.f);
  }
  // no CTA leaves while another may still read its shared memory
  cluster.sync();
}

}  // namespace

cudaError_t launch_add_rmsnorm(void* h, const void* delta, const void* w, void* out, int rows, int D, float eps,
                               cudaStream_t st) {
  return launch_pdl(add_rmsnorm_kernel, dim3(rows), dim3(256), 0, st, static_cast<__half*>(h),
                    static_cast<const __half*>(delta), static_cast<const __half*>(w), static_cast<__half*>(out), D,
                    eps);
}

cudaError_t launch_rope_cache(void* q, void* k, const void* v, void* kc, void* vc, const int* start, int rows,
                              int per_seq, int Hq, int Hkv, int L, float log2_theta, cudaStream_t st) {
  return launch_pdl(rope_cache_kernel, dim3(rows), dim3(256), 0, st, static_cast<__half*>(q),
                    static_cast<__half*>(k), static_cast<const __half*>(v), static_cast<__half*>(kc),
                    static_cast<__half*>(vc), start, per_seq, Hq, Hkv, L, log2_theta);
}

cudaError_t launch_silu_mul(const void* g, const void* u, void* out, int64_t n, cudaStream_t st) {
  int64_t blocks = (n / 8 + 255) / 256;
  if (blocks > 148 * 8) blocks = 148 * 8;
  if (blocks < 1) blocks = 1;
  return launch_pdl(silu_mul_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, st,
                    static_cast<const __half*>(g), static_cast<const __half*>(u), static_cast<__half*>(out), n);
}

namespace {
cudaError_t attention_launch(const void* q, const void* kc, const void* vc, const int* len, void* out, int B, int Hq,
                             int Hkv, int L, float scale, const RopeIn& rope, cudaStream_t st) {
  const int G = Hq / Hkv;
  int P = (L + kAttnChunk - 1) / kAttnChunk;
  P = P < 1 ? 1 : P > kAttnMaxSplit ? kAttnMaxSplit : P;
  const int cmax = (L + P - 1) / P;
  const size_t smem = (static_cast<size_t>(G) * cmax + 8 * G * 128 + 2 * G * 128) * sizeof(float);
  if (smem > 227 * 1024) return cudaErrorInvalidValue;
  if (smem > 48 * 1024) {
    const cudaError_t e =
        cudaFuncSetAttribute(decode_attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  // one cluster of P CTAs per (sequence, kv head), launched as a
  // programmatic dependent of the kernel before it
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(B, Hkv, P);
  cfg.blockDim = dim3(kAttnThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = P;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, decode_attention_kernel, static_cast<const __half*>(q),
                                           static_cast<const __half*>(kc), static_cast<const __half*>(vc), len,
                                           static_cast<__half*>(out), Hq, Hkv, L, cmax, scale, rope);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_decode_attention(const void* q, const void* kc, const void* vc, const int* len, void* out, int B,
                                    int Hq, int Hkv, int L, float scale, cudaStream_t st) {
  const RopeIn none = {};
  return attention_launch(q, kc, vc, len, out, B, Hq, Hkv, L, scale, none, st);
}

cudaError_t launch_rope_decode_attention(void* q, void* k, const void* v, void* kc, void* vc, const int* pos,
                                         const int* len, void* out, int B, int Hq, int Hkv, int L, float log2_theta,
                                         float scale, cudaStream_t st) {
  RopeIn rope;
  rope.q = static_cast<__half*>(q);
  rope.k = static_cast<__half*>(k);
  rope.v = static_cast<const __half*>(v);
  rope.kc = static_cast<__half*>(kc);
  rope.vc = static_cast<__half*>(vc);
  rope.pos = pos;
  rope.log2_theta = log2_theta;
  return attention_launch(q, kc, vc, len, out, B, Hq, Hkv, L, scale, rope, st);
}

}  // namespace persona
