// Fused BGMV for decode-sized batches (a few rows per launch): y[t] +=
// B[s] (A[s] x[t]) without any step through global memory between CTAs.
//
// Same math as the split kernels (reference persona/ops.py:12-56: fp32
// accumulation, one rounding of y, slot -1 rows untouched).  At a handful
// of rows the split kernel's chain shrink slice -> finisher -> expand slice
// is all latency.  Here one thread-block cluster of kSmallCluster CTAs takes
// one (projection, row): CTA c computes the partial v over its eighth of K
// (one warp per rank row, 16-byte loads, all in flight at once), the cluster
// sums the eight partials in rank order through distributed shared memory,
// and CTA c then writes its eighth of the row's columns.  One launch for up
// to kMaxProblems projections that share the slots.
#include <cooperative_groups.h>

#include <type_traits>

#include "bgmv_args.h"
#include "common.cuh"

namespace cg = cooperative_groups;

namespace persona {
namespace {

constexpr int kSmallThreads = 256;
constexpr int kSmallCluster = 8;

template <typename DT, int R>
__global__ void __launch_bounds__(kSmallThreads) bgmv_small_kernel(const SmallArgs args) {
  // a base GEMM launched after this kernel may start streaming its weights
  asm volatile("griddepcontrol.launch_dependents;");
  extern __shared__ __align__(16) uint8_t small_smem[];
  __shared__ float v_part[R];
  __shared__ float v_all[R];
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = static_cast<int>(cluster.block_rank());
  // cluster -> (problem, row)
  const int u = blockIdx.x / kSmallCluster;
  int p = 0;
#pragma unroll
  for (int i = 1; i < kMaxProblems; ++i)
    if (i < args.num_problems && u >= args.unit_base[i]) p = i;
  const SmallProblem& pr = args.prob[p];
  const int row = u - args.unit_base[p];
  const int K = pr.K, N = pr.N, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // this CTA's K range (eighths rounded to 8 values) and column range
  const int kper = ((K + kSmallCluster * 8 - 1) / (kSmallCluster * 8)) * 8;
  const int k0 = min(K, rank * kper), k1 = min(K, k0 + kper);
  const int nper = (N + kSmallCluster - 1) / kSmallCluster;
  const int n0 = min(N, rank * nper), n1 = min(N, n0 + nper);
  {
    // Launched as a programmatic dependent of the kernel before it (at
    // decode: the base GEMM that writes y): pull this CTA's A and B lines
    // into L2 while that kernel finishes.  Only a prefetch reads the slot
    // here (it may not be final yet), and only for a slot in range.
    const int sp = args.slots[row];
    if (sp >= 0 && sp < args.S) {
      const char* ab = static_cast<const char*>(pr.a) + static_cast<int64_t>(sp) * pr.a_slot_stride * 2;
      const int lines_a = (2 * (k1 - k0) + 127) / 128;
      for (int i = tid; i < R * lines_a; i += kSmallThreads) {
        const char* q = ab + (static_cast<int64_t>(i / lines_a) * pr.a_row_stride + k0) * 2 + (i % lines_a) * 128;
        asm volatile("prefetch.global.L2 [%0];" ::"l"(q));
      }
      const char* bb = static_cast<const char*>(pr.b) + (static_cast<int64_t>(sp) * pr.b_slot_stride +
                                                          static_cast<int64_t>(n0) * R) * 2;
      for (int i = tid; i < ((n1 - n0) * R * 2 + 127) / 128; i += kSmallThreads)
        asm volatile("prefetch.global.L2 [%0];" ::"l"(bb + static_cast<int64_t>(i) * 128));
    }
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int s = args.slots[row];
  // the whole cluster takes the same exit, so the barriers below stay matched;
  // a row without adapter adds nothing (a zero delta)
  if (s < 0 || s >= args.S) {
    if (s >= args.S && threadIdx.x == 0 && rank == 0 && p == 0) raise_error(args.err, PERSONA_DEV_ERR_SLOT);
    if (pr.delta)
      for (int n = n0 + tid; n < n1; n += kSmallThreads) pr.delta[static_cast<int64_t>(row) * pr.ld_delta + n] = 0.f;
    return;
  }
  uint16_t* xs = reinterpret_cast<uint16_t*>(small_smem);
  const uint16_t* xr = static_cast<const uint16_t*>(pr.x) + static_cast<int64_t>(row) * pr.ldx;
  for (int i = k0 + tid * 8; i < k1; i += kSmallThreads * 8)
    *reinterpret_cast<uint4*>(xs + (i - k0)) = *reinterpret_cast<const uint4*>(xr + i);
  __syncthreads();
  // partial shrink over [k0, k1): warp w takes rank rows w, w + 8, ...
  const uint16_t* ab = static_cast<const uint16_t*>(pr.a) + static_cast<int64_t>(s) * pr.a_slot_stride;
  for (int r = warp; r < R; r += kSmallThreads / 32) {
    const uint16_t* ar = ab + static_cast<int64_t>(r) * pr.a_row_stride;
    float acc = 0.f;
#pragma unroll 8
    for (int k = k0 + lane * 8; k < k1; k += 32 * 8) {
      const uint4 av = *reinterpret_cast<const uint4*>(ar + k);
      const uint4 xv = *reinterpret_cast<const uint4*>(xs + (k - k0));
      const uint32_t aw[4] = {av.x, av.y, av.z, av.w}, xw[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 af = Cvt<DT>::to2(aw[j]), xf = Cvt<DT>::to2(xw[j]);
        acc = fmaf(af.x, xf.x, acc);
        acc = fmaf(af.y, xf.y, acc);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) v_part[r] = acc;
  }
  cluster.sync();
  // v = the eight partials summed in rank order (the same in every CTA)
  if (tid < R) {
    float v = 0.f;
#pragma unroll
    for (int c = 0; c < kSmallCluster; ++c) v += cluster.map_shared_rank(v_part, c)[tid];
    v_all[tid] = v;
  }
  // This CTA is done with the other CTAs' partials: it says so now and waits
  // for the others only before it exits (no CTA may leave, dropping its
  // shared memory, while another still reads it), so the expand below runs
  // inside that barrier instead of after it.
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  __syncthreads();  // v_all complete for every thread of the CTA
  float v[R];
#pragma unroll
  for (int r = 0; r < R; ++r) v[r] = v_all[r];
  // expand: this CTA's eighth of the columns, one per thread
  const uint16_t* bb = static_cast<const uint16_t*>(pr.b) + static_cast<int64_t>(s) * pr.b_slot_stride;
  uint16_t* yr = static_cast<uint16_t*>(pr.y) + static_cast<int64_t>(row) * pr.ldy;
#pragma unroll 2
  for (int n = n0 + tid; n < n1; n += kSmallThreads) {
    const uint4* br = reinterpret_cast<const uint4*>(bb + static_cast<int64_t>(n) * R);
    uint4 bv[R / 8];
#pragma unroll
    for (int c = 0; c < R / 8; ++c) bv[c] = br[c];
    const uint16_t yo = pr.delta ? uint16_t(0) : yr[n];
    float acc = 0.f;
#pragma unroll
    for (int c = 0; c < R / 8; ++c) {
      const uint32_t bw[4] = {bv[c].x, bv[c].y, bv[c].z, bv[c].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 bf = Cvt<DT>::to2(bw[j]);
        acc = fmaf(bf.x, v[8 * c + 2 * j], acc);
        acc = fmaf(bf.y, v[8 * c + 2 * j + 1], acc);
      }
    }
    if (pr.delta)
      pr.delta[static_cast<int64_t>(row) * pr.ld_delta + n] = acc;
    else
      yr[n] = Cvt<DT>::from1(Cvt<DT>::to1(yo) + acc);
  }
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

template <typename DT, int R>
cudaError_t small_launch(const SmallArgs& a, int clusters, size_t smem, cudaStream_t st) {
  auto kern = bgmv_small_kernel<DT, R>;
  if (smem > 48 * 1024) {
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(clusters * kSmallCluster);
  cfg.blockDim = dim3(kSmallThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = kSmallCluster;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

template <typename DT>
cudaError_t small_rank(int R, const SmallArgs& a, int clusters, size_t smem, cudaStream_t st) {
  switch (R) {
    case 8: return small_launch<DT, 8>(a, clusters, smem, st);
    case 16: return small_launch<DT, 16>(a, clusters, smem, st);
    case 32: return small_launch<DT, 32>(a, clusters, smem, st);
    case 64: return small_launch<DT, 64>(a, clusters, smem, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

cudaError_t launch_bgmv_small(int dtype, int R, SmallArgs& a, int T, cudaStream_t st) {
  int clusters = 0, kmax = 0;
  for (int i = 0; i < a.num_problems; ++i) {
    SmallProblem& p = a.prob[i];
    p.slices = kSmallCluster;
    a.unit_base[i] = clusters;
    clusters += T;
    kmax = p.K > kmax ? p.K : kmax;
  }
  if (clusters == 0) return cudaSuccess;
  // x slice of one CTA: an eighth of K rounded up to 8 values
  const int kper = ((kmax + kSmallCluster * 8 - 1) / (kSmallCluster * 8)) * 8;
  const int x_bytes = kper * 2;
  for (int i = 0; i < a.num_problems; ++i) a.prob[i].x_bytes = x_bytes;
  const size_t smem = static_cast<size_t>(x_bytes);
  return dtype == PERSONA_DTYPE_BF16 ? small_rank<__nv_bfloat16>(R, a, clusters, smem, st)
                                     : small_rank<__half>(R, a, clusters, smem, st);
}

}  // namespace persona
