// Device helpers shared by the B200 (sm_100a) BGMV / SGMV kernels:
// 16-bit <-> fp32 conversion, mbarriers with bounded waits, TMA tile loads,
// bulk copies, warp-MMA wrappers and the error word.
//
// Every wait in this file is bounded by a clock budget.  A wait that runs out
// sets PERSONA_DEV_ERR_TIMEOUT in the caller's error word and returns, so a
// kernel never spins forever on the shared GPU.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "persona_bgmv.h"

namespace persona {

// ---------------------------------------------------------------- types --

template <typename DT> struct Cvt;
template <> struct Cvt<__half> {
  static __device__ __forceinline__ float2 to2(uint32_t w) {
    __half2 h = *reinterpret_cast<__half2*>(&w);
    return __half22float2(h);
  }
  static __device__ __forceinline__ float to1(uint16_t w) {
    return __half2float(__ushort_as_half(w));
  }
  static __device__ __forceinline__ uint16_t from1(float f) {
    return __half_as_ushort(__float2half_rn(f));
  }
};
template <> struct Cvt<__nv_bfloat16> {
  static __device__ __forceinline__ float2 to2(uint32_t w) {
    // bf16 -> fp32 is a 16-bit left shift of the bit pattern.
    return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
  }
  static __device__ __forceinline__ float to1(uint16_t w) {
    return __uint_as_float(static_cast<uint32_t>(w) << 16);
  }
  static __device__ __forceinline__ uint16_t from1(float f) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(f));
  }
};

// -------------------------------------------------------------- errors ---

// The error word may live in mapped pinned host memory, where device atomics
// are not guaranteed over PCIe: a plain read-or-write keeps it nonzero once
// any error is seen (concurrent writers may drop each other's bits, never
// the fact that an error happened).
__device__ __forceinline__ void raise_error(int32_t* err, int32_t bits) {
  if (err != nullptr) {
    volatile int32_t* p = err;
    *p = *p | bits;
    __threadfence_system();
  }
}

// Clock budget of one bounded wait: about 2 s at the B200's 1.9 GHz boost.
constexpr long long kWaitBudgetCycles = 4000000000LL;

// ------------------------------------------------------------ addresses --

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ------------------------------------------------------------ mbarrier ---

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}


__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
          smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

// Relaxed arrive: no release fence, so it never waits for the thread's earlier
// global stores.  Used where the only ordering that matters is that the
// caller's shared-memory reads are done, which holds because their values
// have already been consumed.
__device__ __forceinline__ void mbar_arrive_relaxed(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.relaxed.cta.shared::cta.b64 st, [%0];\n\t}" ::"r"(
                   smem_u32(bar))
               : "memory");
}



__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}


// Bounded wait for phase `parity` of `bar` to complete.  Returns false (and
// flags the error word) if the budget ran out.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int32_t* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try_wait(bar, parity))
      return true;
    if (clock64() - t0 > kWaitBudgetCycles) {
      raise_error(err, PERSONA_DEV_ERR_TIMEOUT);
      return false;
    }
  }
}

// Bounded wait that also gives up when *abort is set, i.e. when another
// thread of the CTA has already given up; running out of budget sets *abort.
// A CTA whose pipeline broke therefore ends after about one wait budget
// instead of spending a full budget on every later wait.  The flag is read
// only once a wait has lasted kAbortPollCycles, so a wait that completes
// normally costs what the plain bounded wait costs.  A phase that has
// completed is reported as complete after an abort too.
constexpr long long kAbortPollCycles = 1LL << 16;
__device__ __forceinline__ bool mbar_wait_abortable(uint64_t* bar, uint32_t parity, int32_t* err, int* abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long dt = clock64() - t0;
    if (dt > kAbortPollCycles) {
      volatile int* ab = abort;
      if (*ab) return false;
      if (dt > kWaitBudgetCycles) {
        *ab = 1;
        raise_error(err, PERSONA_DEV_ERR_TIMEOUT);
        return false;
      }
    }
  }
}

// True in every thread of named barrier `id` (nthreads threads) iff `v` is
// true in all of them; also a barrier.
__device__ __forceinline__ bool named_all(uint32_t id, uint32_t nthreads, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\tbar.red.and.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(v ? 1u : 0u), "r"(id), "r"(nthreads)
      : "memory");
  return r != 0;
}

// ------------------------------------------------------------------ TMA --

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 3-D tiled TMA load into this CTA's shared memory, completing on `bar`.
// The innermost coordinate c0 times the element size must be a multiple of
// 16 bytes; every caller passes c0 as a multiple of 8 16-bit elements.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// 1-D bulk copy global -> this CTA's shared memory, completing on `bar`.
// Both addresses 16-byte aligned, `bytes` a multiple of 16.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// L2 prefetch of one TMA tile / of a 1-D range (16-byte multiple); no
// completion to wait for, no shared memory used.
__device__ __forceinline__ void tma_prefetch_3d(const CUtensorMap* map, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}

__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(reinterpret_cast<uint64_t>(src)), "r"(bytes)
               : "memory");
}

// Named barrier over `nthreads` threads (a multiple of 32), id != 0.
__device__ __forceinline__ void named_sync(uint32_t id, uint32_t nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ------------------------------------------------------ shared memory ---

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}

__device__ __forceinline__ uint16_t lds16(uint32_t addr) {
  uint16_t v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(addr));
  return v;
}

__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}



// ldmatrix: four (x4) or two (x2) 8x8 16-bit matrices from shared memory.
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2(uint32_t addr, uint32_t (&r)[2]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0, %1}, [%2];" : "=r"(r[0]), "=r"(r[1]) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x1(uint32_t addr, uint32_t& r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x1.shared.b16 {%0}, [%1];" : "=r"(r) : "r"(addr));
}

// Warp MMA D(16x8, fp32) += A(16xK) * B(Kx8) with 16-bit A/B (f16 or bf16).
template <typename DT> struct Mma;
template <> struct Mma<__half> {
  static __device__ __forceinline__ void k16(float (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
  }
  static __device__ __forceinline__ void k8(float (&d)[4], const uint32_t (&a)[2], uint32_t b) {
    asm(
        "mma.sync.aligned.m16n8k8.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5}, {%6}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(b));
  }
  // Two fp32 values -> packed 16-bit pair (round to nearest even).
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  static __device__ __forceinline__ float round_trip(float v) { return __half2float(__float2half_rn(v)); }
};
template <> struct Mma<__nv_bfloat16> {
  static __device__ __forceinline__ void k16(float (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
    asm(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
  }
  static __device__ __forceinline__ void k8(float (&d)[4], const uint32_t (&a)[2], uint32_t b) {
    asm(
        "mma.sync.aligned.m16n8k8.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5}, {%6}, {%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(b));
  }
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  static __device__ __forceinline__ float round_trip(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }
};

// Byte offset inside a TMA box written with swizzle of 2^(mask bits) 16-byte
// units: bits [4, 4+b) are XORed with bits [7, 7+b) (b = 3, 2, 1 for the
// 128-, 64-, 32-byte modes; mask 0 = no swizzle).
__device__ __forceinline__ uint32_t swz(uint32_t off, uint32_t mask) {
  return off ^ (((off >> 7) & mask) << 4);
}

}  // namespace persona
