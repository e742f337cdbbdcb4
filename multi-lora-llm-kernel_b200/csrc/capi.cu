// extern "C" entry points of libpersona_bgmv.so (declared in persona_bgmv.h).
//
// Host side of every op: validate the arguments (the reference's TORCH_CHECKs,
// csrc/bgmv_shrink.cu:85-121 and csrc/bgmv_expand.cu:92-128, as status
// codes), build the TMA tensor maps of the adapter pools, then enqueue the
// plan kernel (unless the caller reuses a plan) and the split kernel.
// Nothing here synchronises with the device or allocates device memory.
#include <cudaTypedefs.h>

#include <cmath>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "bgmv_args.h"
#include "common.cuh"
#include "decode_args.h"
#include "nf4_args.h"
#include "plan_layout.h"

namespace persona {


namespace {

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
bool rank_supported(int64_t R) { return R == 8 || R == 16 || R == 32 || R == 64; }
constexpr int64_t kI32Max = 2147483647;

// A pool [S, R, K] (k fastest) as a 3-D tensor {K, R, S}; box {64 k, R rows, 1 slot}.
int encode_a_map(CUtensorMap* m, const void* a_pool, int dtype, int64_t K, int64_t R, int64_t S,
                 int64_t row_stride, int64_t slot_stride) {
  auto enc = tensor_map_encoder();
  if (!enc) return PERSONA_ERR_CUDA;
  const CUtensorMapDataType dt =
      dtype == PERSONA_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(K), static_cast<cuuint64_t>(R), static_cast<cuuint64_t>(S)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(row_stride * 2), static_cast<cuuint64_t>(slot_stride * 2)};
  cuuint32_t box[3] = {64u, static_cast<cuuint32_t>(R), 1u};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  CUresult r = enc(m, dt, 3, const_cast<void*>(a_pool), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? PERSONA_OK : PERSONA_ERR_CUDA;
}

// B pool [S, N, R] (r fastest) as {R, N, S}; box {R, n_box rows, 1 slot},
// swizzled over the 2R-byte rows.
int encode_b_map(CUtensorMap* m, const void* b_pool, int dtype, int64_t N, int64_t R, int64_t S,
                 int64_t slot_stride, int n_box) {
  auto enc = tensor_map_encoder();
  if (!enc) return PERSONA_ERR_CUDA;
  const CUtensorMapDataType dt =
      dtype == PERSONA_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(R), static_cast<cuuint64_t>(N), static_cast<cuuint64_t>(S)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(R * 2), static_cast<cuuint64_t>(slot_stride * 2)};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(R), static_cast<cuuint32_t>(n_box), 1u};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  CUtensorMapSwizzle sw = R == 64   ? CU_TENSOR_MAP_SWIZZLE_128B
                          : R == 32 ? CU_TENSOR_MAP_SWIZZLE_64B
                          : R == 16 ? CU_TENSOR_MAP_SWIZZLE_32B
                                    : CU_TENSOR_MAP_SWIZZLE_NONE;
  CUresult r = enc(m, dt, 3, const_cast<void*>(b_pool), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? PERSONA_OK : PERSONA_ERR_CUDA;
}

// Row-major [rows, cols] 16-bit matrix as a 2-D tensor {cols, rows}; box
// {box_cols, box_rows}, 128-byte swizzle (box_cols * 2 == 128).
int encode_2d_map(CUtensorMap* m, const void* base, int dtype, int64_t cols, int64_t rows, int64_t row_stride,
                  int box_cols, int box_rows) {
  auto enc = tensor_map_encoder();
  if (!enc) return PERSONA_ERR_CUDA;
  const CUtensorMapDataType dt =
      dtype == PERSONA_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_stride * 2)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = enc(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? PERSONA_OK : PERSONA_ERR_CUDA;
}

int check_common(int64_t T, int64_t S, int dtype, const void* workspace, size_t ws_bytes,
                 const int32_t* slots) {
  if (T < 0 || S <= 0) return PERSONA_ERR_SHAPE;
  if (T > kI32Max / 64) return PERSONA_ERR_SHAPE;
  if (dtype != PERSONA_DTYPE_F16 && dtype != PERSONA_DTYPE_BF16) return PERSONA_ERR_DTYPE;
  if (T > 0 && slots == nullptr) return PERSONA_ERR_INVALID_ARG;
  if (T > 0 && (workspace == nullptr || ws_bytes < bgmv_ws_bytes(T))) return PERSONA_ERR_WORKSPACE;
  if (T > 0 && !aligned16(workspace)) return PERSONA_ERR_ALIGNMENT;
  return PERSONA_OK;
}

int check_a(const void* x, int64_t ldx, const void* a_pool, int64_t a_slot_stride,
            int64_t a_row_stride, int64_t K, int64_t R, int64_t S) {
  if (x == nullptr || a_pool == nullptr) return PERSONA_ERR_INVALID_ARG;
  if (K <= 0 || R <= 0 || K > kI32Max) return PERSONA_ERR_SHAPE;
  if (K % 8 != 0) return PERSONA_ERR_SHAPE;  // csrc/bgmv_shrink.cu:100
  if (ldx < K || a_row_stride < K || a_slot_stride < (R - 1) * a_row_stride + K) return PERSONA_ERR_SHAPE;
  if (!aligned16(x) || !aligned16(a_pool)) return PERSONA_ERR_ALIGNMENT;  // :101-104
  if (ldx % 8 || a_row_stride % 8 || a_slot_stride % 8) return PERSONA_ERR_ALIGNMENT;
  (void)S;
  return PERSONA_OK;
}

int check_b(const void* b_pool, int64_t b_slot_stride, const void* y, int64_t ldy, int64_t N,
            int64_t R) {
  if (b_pool == nullptr || y == nullptr) return PERSONA_ERR_INVALID_ARG;
  if (N <= 0 || N > kI32Max) return PERSONA_ERR_SHAPE;
  if (!rank_supported(R)) return PERSONA_ERR_RANK;       // csrc/bgmv_expand.cu:68-83
  if (N % 8 != 0) return PERSONA_ERR_SHAPE;              // csrc/bgmv_expand.cu:107
  if (ldy < N || b_slot_stride < N * R) return PERSONA_ERR_SHAPE;
  if (!aligned16(b_pool) || !aligned16(y)) return PERSONA_ERR_ALIGNMENT;  // :108-111
  if (ldy % 8 || b_slot_stride % 8) return PERSONA_ERR_ALIGNMENT;
  return PERSONA_OK;
}

// Rows of one B tile: the tcgen05 M side (128) for ranks >= 16, else as
// many rows as a ring slot holds.
int b_box_rows(int64_t N, int64_t R) {
  const int64_t nb = R >= 16 ? 128 : bgmv_stage_rows(static_cast<int>(R));
  const int64_t n8 = (N + 7) / 8 * 8;
  return static_cast<int>(n8 < nb ? n8 : nb);
}

// Work units per pipeline of the split kernel (PERSONA_UNITS_PER_CTA overrides).
int units_per_cta() {
  static const int v = [] {
    const char* e = std::getenv("PERSONA_UNITS_PER_CTA");
    const int n = e != nullptr ? std::atoi(e) : 0;
    return n > 0 && n <= 64 ? n : 0;
  }();
  return v;
}

int run_split(int mode, int dtype, int64_t R, const SplitMaps& maps, SplitArgs& a, cudaStream_t stream) {
  a.units_per_cta = units_per_cta();
  return launch_bgmv_split(mode, dtype, static_cast<int>(R), maps, a, stream) == cudaSuccess ? PERSONA_OK
                                                                                             : PERSONA_ERR_CUDA;
}

// Decode-sized fused launches: the kernel without cross-CTA steps.
bool small_path(int64_t T, int flags, const int64_t* Ks, int n) {
  if (T > PERSONA_SMALL_MAX_ROWS || (flags & PERSONA_SPLIT_ONLY)) return false;
  for (int i = 0; i < n; ++i)
    if (Ks[i] > 32768) return false;
  return true;
}

int run_small(const persona_bgmv_problem* probs, int n, const int32_t* slots, int64_t T, int64_t R, int64_t S,
              int dtype, int32_t* dev_err, cudaStream_t stream) {
  SmallArgs a = {};
  for (int i = 0; i < n; ++i) {
    const persona_bgmv_problem& q = probs[i];
    SmallProblem& p = a.prob[i];
    p.x = q.x;
    p.a = q.a_pool;
    p.b = q.b_pool;
    p.y = q.y;
    p.ldx = q.ldx;
    p.a_slot_stride = q.a_slot_stride;
    p.a_row_stride = q.a_row_stride;
    p.b_slot_stride = q.b_slot_stride;
    p.ldy = q.ldy;
    p.K = static_cast<int>(q.K);
    p.N = static_cast<int>(q.N);
  }
  a.slots = slots;
  a.err = dev_err;
  a.num_problems = n;
  a.S = static_cast<int>(S);
  return launch_bgmv_small(dtype, static_cast<int>(R), a, static_cast<int>(T), stream) == cudaSuccess
             ? PERSONA_OK
             : PERSONA_ERR_CUDA;
}

int plan_if_needed(const int32_t* slots, int64_t T, int64_t S, void* ws, int flags,
                   int32_t* dev_err, cudaStream_t st) {
  if (flags & PERSONA_REUSE_PLAN) return PERSONA_OK;
  return launch_bgmv_plan(slots, static_cast<int>(T), static_cast<int>(S), kRowsPerItem,
                          static_cast<int32_t*>(ws), dev_err, st) == cudaSuccess
             ? PERSONA_OK
             : PERSONA_ERR_CUDA;
}

}  // namespace
}  // namespace persona

using namespace persona;

extern "C" {

const char* persona_status_string(int status) {
  switch (status) {
    case PERSONA_OK: return "ok";
    case PERSONA_ERR_INVALID_ARG: return "invalid argument (null pointer, negative size or bad flag)";
    case PERSONA_ERR_SHAPE: return "inconsistent or unsupported shape";
    case PERSONA_ERR_DTYPE: return "only float16 and bfloat16 supported";
    case PERSONA_ERR_ALIGNMENT: return "pointer or stride not 16-byte aligned";
    case PERSONA_ERR_RANK: return "R must be 8, 16, 32, or 64";
    case PERSONA_ERR_WORKSPACE: return "workspace missing, misaligned or too small";
    case PERSONA_ERR_CUDA: return "CUDA runtime or launch failure";
    case PERSONA_ERR_NOALLOC_ROWS: return "T above PERSONA_NOALLOC_MAX_ROWS, the fixed plan scratch of persona_bgmv_fused_noalloc";
    default: return "unknown status";
  }
}

int persona_abi_version(void) { return PERSONA_ABI_VERSION; }

size_t persona_bgmv_workspace_size(int64_t T) { return T < 0 ? 0 : bgmv_ws_bytes(T); }

int persona_bgmv_plan(const int32_t* slots, int64_t T, int64_t S, void* workspace,
                      size_t workspace_bytes, int32_t* dev_err, cudaStream_t stream) {
  int st = check_common(T, S, PERSONA_DTYPE_F16, workspace, workspace_bytes, slots);
  if (st != PERSONA_OK) return st;
  if (T == 0) return PERSONA_OK;
  return plan_if_needed(slots, T, S, workspace, 0, dev_err, stream);
}

int persona_bgmv_shrink(const void* x, int64_t ldx, const void* a_pool, int64_t a_slot_stride,
                        int64_t a_row_stride, const int32_t* slots, float* v, int64_t T,
                        int64_t K, int64_t R, int64_t S, int dtype, void* workspace,
                        size_t workspace_bytes, int flags, int32_t* dev_err,
                        cudaStream_t stream) {
  if (flags & ~PERSONA_REUSE_PLAN) return PERSONA_ERR_INVALID_ARG;
  // Ranks 8/16/32/64 with K >= 64 run the split kernel over a plan; any
  // other rank runs row by row and needs no workspace.
  const bool planned = rank_supported(R) && K >= 64;
  int st;
  if (planned) {
    st = check_common(T, S, dtype, workspace, workspace_bytes, slots);
  } else {
    st = check_common(T, S, dtype, nullptr, 0, slots);
    if (st == PERSONA_ERR_WORKSPACE || st == PERSONA_ERR_ALIGNMENT) st = PERSONA_OK;
  }
  if (st != PERSONA_OK) return st;
  if (T == 0) return PERSONA_OK;
  if ((st = check_a(x, ldx, a_pool, a_slot_stride, a_row_stride, K, R, S)) != PERSONA_OK) return st;
  if (v == nullptr) return PERSONA_ERR_INVALID_ARG;
  if (!aligned16(v)) return PERSONA_ERR_ALIGNMENT;
  if (R > 4096 || T * R > kI32Max) return PERSONA_ERR_SHAPE;
  if (!planned) {
    return launch_shrink_rowwise(dtype, x, ldx, a_pool, a_slot_stride, a_row_stride, slots, v,
                                 static_cast<int>(T), static_cast<int>(K), static_cast<int>(R),
                                 static_cast<int>(S), dev_err, stream) == cudaSuccess
               ? PERSONA_OK
               : PERSONA_ERR_CUDA;
  }
  SplitMaps maps;
  std::memset(&maps, 0, sizeof(maps));
  if ((st = encode_a_map(&maps.a[0], a_pool, dtype, K, R, S, a_row_stride, a_slot_stride)) != PERSONA_OK) return st;
  if ((st = plan_if_needed(slots, T, S, workspace, flags, dev_err, stream)) != PERSONA_OK) return st;
  SplitArgs a = {};
  a.prob[0].x = x;
  a.prob[0].ldx = ldx;
  a.prob[0].K = static_cast<int>(K);
  a.prob[0].n_box = 8;
  a.num_problems = 1;
  a.v_out = v;
  a.slots = slots;
  a.ws = static_cast<int32_t*>(workspace);
  a.err = dev_err;
  a.T = static_cast<int>(T);
  a.S = static_cast<int>(S);
  return run_split(kModeShrink, dtype, R, maps, a, stream);
}

int persona_bgmv_expand(const float* v, const void* b_pool, int64_t b_slot_stride,
                        const int32_t* slots, void* y, int64_t ldy, int64_t T, int64_t N,
                        int64_t R, int64_t S, int dtype, void* workspace,
                        size_t workspace_bytes, int flags, int32_t* dev_err,
                        cudaStream_t stream) {
  if (flags & ~PERSONA_REUSE_PLAN) return PERSONA_ERR_INVALID_ARG;
  int st = check_common(T, S, dtype, workspace, workspace_bytes, slots);
  if (st != PERSONA_OK) return st;
  if (!rank_supported(R)) return PERSONA_ERR_RANK;
  if (T == 0) return PERSONA_OK;
  if ((st = check_b(b_pool, b_slot_stride, y, ldy, N, R)) != PERSONA_OK) return st;
  if (v == nullptr) return PERSONA_ERR_INVALID_ARG;
  if (!aligned16(v)) return PERSONA_ERR_ALIGNMENT;
  SplitArgs a = {};
  a.prob[0].y = y;
  a.prob[0].ldy = ldy;
  a.prob[0].N = static_cast<int>(N);
  a.prob[0].n_box = b_box_rows(N, R);
  SplitMaps maps;
  std::memset(&maps, 0, sizeof(maps));
  if ((st = encode_b_map(&maps.b[0], b_pool, dtype, N, R, S, b_slot_stride, a.prob[0].n_box)) != PERSONA_OK)
    return st;
  if ((st = plan_if_needed(slots, T, S, workspace, flags, dev_err, stream)) != PERSONA_OK) return st;
  a.num_problems = 1;
  a.v_in = v;
  a.slots = slots;
  a.ws = static_cast<int32_t*>(workspace);
  a.err = dev_err;
  a.T = static_cast<int>(T);
  a.S = static_cast<int>(S);
  return run_split(kModeExpand, dtype, R, maps, a, stream);
}

}  // extern "C"

namespace persona {
// persona_bgmv_fused; plan_small = false skips the plan on the decode-sized
// path (whose kernel reads no plan), for callers that keep no plan around.
int fused_impl(const void* x, int64_t ldx, const void* a_pool, int64_t a_slot_stride, int64_t a_row_stride,
               const void* b_pool, int64_t b_slot_stride, const int32_t* slots, void* y, int64_t ldy, int64_t T,
               int64_t K, int64_t N, int64_t R, int64_t S, int dtype, void* workspace, size_t workspace_bytes,
               int flags, int32_t* dev_err, cudaStream_t stream, bool plan_small) {
  if (flags & ~(PERSONA_REUSE_PLAN | PERSONA_SPLIT_ONLY)) return PERSONA_ERR_INVALID_ARG;
  int st = check_common(T, S, dtype, workspace, workspace_bytes, slots);
  if (st != PERSONA_OK) return st;
  if (!rank_supported(R)) return PERSONA_ERR_RANK;
  if (T == 0) return PERSONA_OK;
  if ((st = check_a(x, ldx, a_pool, a_slot_stride, a_row_stride, K, R, S)) != PERSONA_OK) return st;
  if ((st = check_b(b_pool, b_slot_stride, y, ldy, N, R)) != PERSONA_OK) return st;
  if (K < 64) return PERSONA_ERR_SHAPE;
  if (small_path(T, flags, &K, 1)) {
    if (plan_small && (st = plan_if_needed(slots, T, S, workspace, flags, dev_err, stream)) != PERSONA_OK) return st;
    const persona_bgmv_problem one = {x, ldx, a_pool, a_slot_stride, a_row_stride, b_pool, b_slot_stride,
                                      y, ldy, K, N};
    return run_small(&one, 1, slots, T, R, S, dtype, dev_err, stream);
  }
  SplitArgs a = {};
  SplitMaps maps;
  std::memset(&maps, 0, sizeof(maps));
  a.prob[0].x = x;
  a.prob[0].ldx = ldx;
  a.prob[0].y = y;
  a.prob[0].ldy = ldy;
  a.prob[0].K = static_cast<int>(K);
  a.prob[0].N = static_cast<int>(N);
  a.prob[0].n_box = b_box_rows(N, R);
  if ((st = encode_a_map(&maps.a[0], a_pool, dtype, K, R, S, a_row_stride, a_slot_stride)) != PERSONA_OK) return st;
  if ((st = encode_b_map(&maps.b[0], b_pool, dtype, N, R, S, b_slot_stride, a.prob[0].n_box)) != PERSONA_OK)
    return st;
  if ((st = plan_if_needed(slots, T, S, workspace, flags, dev_err, stream)) != PERSONA_OK) return st;
  a.num_problems = 1;
  a.slots = slots;
  a.ws = static_cast<int32_t*>(workspace);
  a.err = dev_err;
  a.T = static_cast<int>(T);
  a.S = static_cast<int>(S);
  return run_split(kModeFused, dtype, R, maps, a, stream);
}

}  // namespace persona

extern "C" {

int persona_bgmv_fused(const void* x, int64_t ldx, const void* a_pool, int64_t a_slot_stride,
                       int64_t a_row_stride, const void* b_pool, int64_t b_slot_stride,
                       const int32_t* slots, void* y, int64_t ldy, int64_t T, int64_t K,
                       int64_t N, int64_t R, int64_t S, int dtype, void* workspace,
                       size_t workspace_bytes, int flags, int32_t* dev_err,
                       cudaStream_t stream) {
  return persona::fused_impl(x, ldx, a_pool, a_slot_stride, a_row_stride, b_pool, b_slot_stride, slots, y, ldy, T, K,
                             N, R, S, dtype, workspace, workspace_bytes, flags, dev_err, stream, true);
}

size_t persona_bgmv_multi_workspace_size(int64_t T, int num_problems) {
  if (T < 0 || num_problems < 1 || num_problems > PERSONA_MAX_PROBLEMS) return 0;
  return bgmv_ws_bytes(T, num_problems);
}

int persona_bgmv_fused_multi(const persona_bgmv_problem* problems, int num_problems, const int32_t* slots,
                             int64_t T, int64_t R, int64_t S, int dtype, void* workspace, size_t workspace_bytes,
                             int flags, int32_t* dev_err, cudaStream_t stream) {
  if (flags & ~(PERSONA_REUSE_PLAN | PERSONA_SPLIT_ONLY)) return PERSONA_ERR_INVALID_ARG;
  if (problems == nullptr || num_problems < 1 || num_problems > PERSONA_MAX_PROBLEMS) return PERSONA_ERR_INVALID_ARG;
  int st = check_common(T, S, dtype, workspace, workspace_bytes, slots);
  if (st != PERSONA_OK) return st;
  if (T > 0 && workspace_bytes < bgmv_ws_bytes(T, num_problems)) return PERSONA_ERR_WORKSPACE;
  if (!rank_supported(R)) return PERSONA_ERR_RANK;
  SplitArgs a = {};
  SplitMaps maps;
  std::memset(&maps, 0, sizeof(maps));
  for (int p = 0; p < num_problems; ++p) {
    const persona_bgmv_problem& q = problems[p];
    if ((st = check_a(q.x, q.ldx, q.a_pool, q.a_slot_stride, q.a_row_stride, q.K, R, S)) != PERSONA_OK) return st;
    if ((st = check_b(q.b_pool, q.b_slot_stride, q.y, q.ldy, q.N, R)) != PERSONA_OK) return st;
    if (q.K < 64) return PERSONA_ERR_SHAPE;
    a.prob[p].x = q.x;
    a.prob[p].ldx = q.ldx;
    a.prob[p].y = q.y;
    a.prob[p].ldy = q.ldy;
    a.prob[p].K = static_cast<int>(q.K);
    a.prob[p].N = static_cast<int>(q.N);
    a.prob[p].n_box = b_box_rows(q.N, R);
  }
  if (T == 0) return PERSONA_OK;
  int64_t Ks[PERSONA_MAX_PROBLEMS];
  for (int p = 0; p < num_problems; ++p) Ks[p] = problems[p].K;
  if (small_path(T, flags, Ks, num_problems)) {
    if ((st = plan_if_needed(slots, T, S, workspace, flags, dev_err, stream)) != PERSONA_OK) return st;
    return run_small(problems, num_problems, slots, T, R, S, dtype, dev_err, stream);
  }
  for (int p = 0; p < num_problems; ++p) {
    const persona_bgmv_problem& q = problems[p];
    if ((st = encode_a_map(&maps.a[p], q.a_pool, dtype, q.K, R, S, q.a_row_stride, q.a_slot_stride)) != PERSONA_OK)
      return st;
    if ((st = encode_b_map(&maps.b[p], q.b_pool, dtype, q.N, R, S, q.b_slot_stride, a.prob[p].n_box)) !=
        PERSONA_OK)
      return st;
  }
  if ((st = plan_if_needed(slots, T, S, workspace, flags, dev_err, stream)) != PERSONA_OK) return st;
  a.num_problems = num_problems;
  a.slots = slots;
  a.ws = static_cast<int32_t*>(workspace);
  a.err = dev_err;
  a.T = static_cast<int>(T);
  a.S = static_cast<int>(S);
  return run_split(kModeFused, dtype, R, maps, a, stream);
}

int persona_gemv_fp16(const void* x, const void* W, void* y, int64_t K, int64_t N,
                      cudaStream_t stream) {
  if (K < 0 || N < 0 || K > kI32Max || N > kI32Max) return PERSONA_ERR_SHAPE;
  if (N == 0) return PERSONA_OK;
  if (x == nullptr || W == nullptr || y == nullptr) return PERSONA_ERR_INVALID_ARG;
  return launch_gemv_fp16(x, W, y, static_cast<int>(K), static_cast<int>(N), stream) == cudaSuccess
             ? PERSONA_OK
             : PERSONA_ERR_CUDA;
}

}  // extern "C"

// ----------------------------------------------------------------- SGMV ---
namespace {
// Workspace of the segmented ops: the BGMV workspace (plan, counters, v),
// the per-row slots of the split-kernel path, and the tensor-core kernel's
// partial-v pieces.
size_t sgmv_rows_offset(int64_t T) { return persona::bgmv_ws_bytes(T); }
size_t sgmv_pieces_offset(int64_t T) {
  return persona::align256(sgmv_rows_offset(T) + 4 * static_cast<size_t>(persona::plan_tpad(T)));
}
size_t sgmv_ws_bytes(int64_t T) { return sgmv_pieces_offset(T) + persona::kSgmvPieceBytes; }

int sgmv_prepare(const int32_t* seg_indptr, const int32_t* seg_slots, int64_t nseg, int64_t T, int64_t S,
                 void* workspace, size_t workspace_bytes, int32_t* dev_err, cudaStream_t stream,
                 int32_t** row_slots) {
  if (T < 0 || S <= 0 || nseg < 0 || T > (int64_t{1} << 30) || nseg > (int64_t{1} << 30)) return PERSONA_ERR_SHAPE;
  if (T == 0) return PERSONA_OK;
  if (seg_indptr == nullptr || (nseg > 0 && seg_slots == nullptr)) return PERSONA_ERR_INVALID_ARG;
  if (workspace == nullptr || workspace_bytes < sgmv_ws_bytes(T)) return PERSONA_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(workspace) & 15) != 0) return PERSONA_ERR_ALIGNMENT;
  *row_slots = reinterpret_cast<int32_t*>(static_cast<uint8_t*>(workspace) + sgmv_rows_offset(T));
  return persona::launch_sgmv_plan(seg_indptr, seg_slots, static_cast<int>(nseg), static_cast<int>(T),
                                   static_cast<int>(S), persona::kRowsPerItem, static_cast<int32_t*>(workspace),
                                   *row_slots, dev_err, stream) == cudaSuccess
             ? PERSONA_OK
             : PERSONA_ERR_CUDA;
}
}  // namespace

namespace {
// Tensor-core path: ranks 16 / 32 / 64, K and N multiples of 64.
// PERSONA_SGMV_TENSOR_CORES=0 selects the BGMV split path instead.
bool sgmv_tc_eligible(int64_t R, int64_t K, int64_t N, bool need_k, bool need_n) {
  static const bool enabled = [] {
    const char* e = std::getenv("PERSONA_SGMV_TENSOR_CORES");
    return !(e != nullptr && e[0] == '0');
  }();
  if (!enabled || !(R == 16 || R == 32 || R == 64)) return false;
  if (need_k && (K % 64 != 0 || K <= 0)) return false;
  if (need_n && (N % 64 != 0 || N <= 0)) return false;
  return true;
}

int sgmv_tc_run(int mode, const void* x, int64_t ldx, const void* a_pool, int64_t a_slot_stride,
                int64_t a_row_stride, const void* b_pool, int64_t b_slot_stride, const int32_t* seg_indptr,
                const int32_t* seg_slots, int64_t nseg, const float* v_in, float* v_out, void* y, int64_t ldy,
                int64_t T, int64_t K, int64_t N, int64_t R, int64_t S, int dtype, void* workspace,
                size_t workspace_bytes, int32_t* dev_err, cudaStream_t stream, int64_t n0 = 0, int64_t n1 = -1,
                void* const* peers = nullptr, int num_peers = 0) {
  using namespace persona;
  if (T < 0 || S <= 0 || nseg < 0 || T > (int64_t{1} << 30)) return PERSONA_ERR_SHAPE;
  if (n1 < 0) n1 = N;
  if (n0 < 0 || n1 < n0 || n1 > N || n0 % 64 != 0 || (n1 - n0) % 64 != 0) return PERSONA_ERR_SHAPE;
  if (num_peers < 0 || num_peers > kMaxTpPeers || (num_peers > 0 && peers == nullptr)) return PERSONA_ERR_INVALID_ARG;
  for (int q = 0; q < num_peers; ++q)
    if (peers[q] == nullptr || !aligned16(peers[q])) return PERSONA_ERR_ALIGNMENT;
  if (T == 0) return PERSONA_OK;
  if (seg_indptr == nullptr || (nseg > 0 && seg_slots == nullptr)) return PERSONA_ERR_INVALID_ARG;
  if (workspace == nullptr || workspace_bytes < sgmv_ws_bytes(T)) return PERSONA_ERR_WORKSPACE;
  if (!aligned16(workspace)) return PERSONA_ERR_ALIGNMENT;
  int st;
  CUtensorMap tx, ta, tb, ty;
  std::memset(&tx, 0, sizeof(tx));
  std::memset(&ta, 0, sizeof(ta));
  std::memset(&tb, 0, sizeof(tb));
  std::memset(&ty, 0, sizeof(ty));
  if (mode & kModeShrink) {
    if ((st = check_a(x, ldx, a_pool, a_slot_stride, a_row_stride, K, R, S)) != PERSONA_OK) return st;
    if ((st = encode_2d_map(&tx, x, dtype, K, T, ldx, 64, 128)) != PERSONA_OK) return st;
    if ((st = encode_a_map(&ta, a_pool, dtype, K, R, S, a_row_stride, a_slot_stride)) != PERSONA_OK) return st;
  }
  if (mode & kModeExpand) {
    if ((st = check_b(b_pool, b_slot_stride, y, ldy, N, R)) != PERSONA_OK) return st;
    if ((st = encode_2d_map(&ty, y, dtype, N, T, ldy, 64, 128)) != PERSONA_OK) return st;
    if ((st = encode_b_map(&tb, b_pool, dtype, N, R, S, b_slot_stride, kSgmvTcTileN)) != PERSONA_OK) return st;
  }
  if (mode == kModeShrink && (v_out == nullptr || !aligned16(v_out))) return PERSONA_ERR_ALIGNMENT;
  if (mode == kModeExpand && (v_in == nullptr || !aligned16(v_in))) return PERSONA_ERR_ALIGNMENT;
  // The tensor-core kernel reads the header and the items of 128 rows; the
  // plan kernel also zeroes the per-item counters and ready words it uses.
  const WorkView wv = work_view(static_cast<int32_t*>(workspace), T);
  if (launch_sgmv_plan(seg_indptr, seg_slots, static_cast<int>(nseg), static_cast<int>(T), static_cast<int>(S),
                       128, static_cast<int32_t*>(workspace), nullptr, dev_err, stream, wv.s_cnt,
                       static_cast<int>(wv.ready - wv.s_cnt)) != cudaSuccess)
    return PERSONA_ERR_CUDA;
  if (mode == kModeShrink) {
    // rows outside every segment (or with slot -1) get v = 0 first
    if (cudaMemsetAsync(v_out, 0, static_cast<size_t>(T * R) * sizeof(float), stream) != cudaSuccess)
      return PERSONA_ERR_CUDA;
  }
  SgmvTcArgs a = {};
  a.plan = static_cast<const int32_t*>(workspace);
  a.v_in = v_in;
  a.v_out = v_out;
  a.y = static_cast<uint16_t*>(y);
  a.ldy = ldy;
  a.err = dev_err;
  a.T = static_cast<int>(T);
  a.K = static_cast<int>(K);
  a.N = static_cast<int>(n1 - n0);
  a.n0 = static_cast<int>(n0);
  a.vfin = wv.vfinal;
  a.pieces = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + sgmv_pieces_offset(T));
  a.item_cnt = wv.s_cnt;
  a.item_ready = wv.ready;
  a.num_peers = num_peers;
  for (int q = 0; q < num_peers; ++q) a.peers[q] = static_cast<uint16_t*>(peers[q]);
  if (n1 == n0 && (mode & kModeExpand)) return PERSONA_OK;
  const int64_t max_items = (T + 127) / 128 + nseg;
  return launch_sgmv_tc(mode, dtype, static_cast<int>(R), tx, ta, tb, ty, a,
                        static_cast<int>(max_items < (1 << 30) ? max_items : (1 << 30)), stream) == cudaSuccess
             ? PERSONA_OK
             : PERSONA_ERR_CUDA;
}
}  // namespace

extern "C" {

size_t persona_sgmv_workspace_size(int64_t T) { return T < 0 ? 0 : sgmv_ws_bytes(T); }

int persona_sgmv_fused_tp(const void* x, int64_t ldx, const void* a_pool, int64_t a_slot_stride,
                          int64_t a_row_stride, const void* b_pool, int64_t b_slot_stride, const int32_t* seg_indptr,
                          const int32_t* seg_slots, int64_t num_segments, void* y, int64_t ldy, void* const* peer_ys,
                          int num_peers, int64_t n0, int64_t n1, int64_t T, int64_t K, int64_t N, int64_t R,
                          int64_t S, int dtype, void* workspace, size_t workspace_bytes, int32_t* dev_err,
                          cudaStream_t stream) {
  if (dtype != PERSONA_DTYPE_F16 && dtype != PERSONA_DTYPE_BF16) return PERSONA_ERR_DTYPE;
  if (!(R == 16 || R == 32 || R == 64)) return PERSONA_ERR_RANK;
  if (K <= 0 || K % 64 != 0 || N <= 0 || N % 64 != 0) return PERSONA_ERR_SHAPE;
  return sgmv_tc_run(persona::kModeFused, x, ldx, a_pool, a_slot_stride, a_row_stride, b_pool, b_slot_stride,
                     seg_indptr, seg_slots, num_segments, nullptr, nullptr, y, ldy, T, K, N, R, S, dtype, workspace,
                     workspace_bytes, dev_err, stream, n0, n1, peer_ys, num_peers);
}

// Base of the allocation that holds ptr, through the driver entry point (no
// link-time dependency on libcuda).
static int allocation_base(const void* ptr, void** base, size_t* offset) {
  using Fn = CUresult (*)(CUdeviceptr*, size_t*, CUdeviceptr);
  static Fn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<Fn>(p);
  });
  if (fn == nullptr) return PERSONA_ERR_CUDA;
  CUdeviceptr b = 0;
  size_t size = 0;
  if (fn(&b, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) return PERSONA_ERR_CUDA;
  *base = reinterpret_cast<void*>(b);
  *offset = static_cast<size_t>(reinterpret_cast<uintptr_t>(ptr) - static_cast<uintptr_t>(b));
  return PERSONA_OK;
}

int persona_ipc_export(const void* ptr, void* handle, size_t* offset) {
  if (ptr == nullptr || handle == nullptr || offset == nullptr) return PERSONA_ERR_INVALID_ARG;
  void* base = nullptr;
  int st = allocation_base(ptr, &base, offset);
  if (st != PERSONA_OK) return st;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, base) != cudaSuccess) return PERSONA_ERR_CUDA;
  std::memcpy(handle, &h, sizeof(h));
  return PERSONA_OK;
}

int persona_ipc_import(const void* handle, size_t offset, void** ptr, void** base) {
  if (handle == nullptr || ptr == nullptr || base == nullptr) return PERSONA_ERR_INVALID_ARG;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* b = nullptr;
  if (cudaIpcOpenMemHandle(&b, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return PERSONA_ERR_CUDA;
  *base = b;
  *ptr = static_cast<uint8_t*>(b) + offset;
  return PERSONA_OK;
}

int persona_ipc_close(void* base) {
  if (base == nullptr) return PERSONA_ERR_INVALID_ARG;
  return cudaIpcCloseMemHandle(base) == cudaSuccess ? PERSONA_OK : PERSONA_ERR_CUDA;
}

int persona_sgmv_shrink(const void* x, int64_t ldx, const void* a_pool, int64_t a_slot_stride, int64_t a_row_stride,
                        const int32_t* seg_indptr, const int32_t* seg_slots, int64_t num_segments, float* v,
                        int64_t T, int64_t K, int64_t R, int64_t S, int dtype, void* workspace,
                        size_t workspace_bytes, int32_t* dev_err, cudaStream_t stream) {
  if (dtype != PERSONA_DTYPE_F16 && dtype != PERSONA_DTYPE_BF16) return PERSONA_ERR_DTYPE;
  if (sgmv_tc_eligible(R, K, 0, true, false))
    return sgmv_tc_run(persona::kModeShrink, x, ldx, a_pool, a_slot_stride, a_row_stride, nullptr, 0, seg_indptr,
                       seg_slots, num_segments, nullptr, v, nullptr, 0, T, K, 0, R, S, dtype, workspace,
                       workspace_bytes, dev_err, stream);
  int32_t* row_slots = nullptr;
  int st = sgmv_prepare(seg_indptr, seg_slots, num_segments, T, S, workspace, workspace_bytes, dev_err, stream,
                        &row_slots);
  if (st != PERSONA_OK || T == 0) return st;
  return persona_bgmv_shrink(x, ldx, a_pool, a_slot_stride, a_row_stride, row_slots, v, T, K, R, S, dtype,
                             workspace, persona::bgmv_ws_bytes(T), PERSONA_REUSE_PLAN, dev_err, stream);
}

int persona_sgmv_expand(const float* v, const void* b_pool, int64_t b_slot_stride, const int32_t* seg_indptr,
                        const int32_t* seg_slots, int64_t num_segments, void* y, int64_t ldy, int64_t T, int64_t N,
                        int64_t R, int64_t S, int dtype, void* workspace, size_t workspace_bytes,
                        int32_t* dev_err, cudaStream_t stream) {
  if (dtype != PERSONA_DTYPE_F16 && dtype != PERSONA_DTYPE_BF16) return PERSONA_ERR_DTYPE;
  if (!rank_supported(R)) return PERSONA_ERR_RANK;
  if (sgmv_tc_eligible(R, 0, N, false, true))
    return sgmv_tc_run(persona::kModeExpand, nullptr, 0, nullptr, 0, 0, b_pool, b_slot_stride, seg_indptr,
                       seg_slots, num_segments, v, nullptr, y, ldy, T, 0, N, R, S, dtype, workspace,
                       workspace_bytes, dev_err, stream);
  int32_t* row_slots = nullptr;
  int st = sgmv_prepare(seg_indptr, seg_slots, num_segments, T, S, workspace, workspace_bytes, dev_err, stream,
                        &row_slots);
  if (st != PERSONA_OK || T == 0) return st;
  return persona_bgmv_expand(v, b_pool, b_slot_stride, row_slots, y, ldy, T, N, R, S, dtype, workspace,
                             persona::bgmv_ws_bytes(T), PERSONA_REUSE_PLAN, dev_err, stream);
}

int persona_sgmv_fused(const void* x, int64_t ldx, const void* a_pool, int64_t a_slot_stride, int64_t a_row_stride,
                       const void* b_pool, int64_t b_slot_stride, const int32_t* seg_indptr,
                       const int32_t* seg_slots, int64_t num_segments, void* y, int64_t ldy, int64_t T, int64_t K,
                       int64_t N, int64_t R, int64_t S, int dtype, void* workspace, size_t workspace_bytes,
                       int32_t* dev_err, cudaStream_t stream) {
  if (dtype != PERSONA_DTYPE_F16 && dtype != PERSONA_DTYPE_BF16) return PERSONA_ERR_DTYPE;
  if (!rank_supported(R)) return PERSONA_ERR_RANK;
  if (sgmv_tc_eligible(R, K, N, true, true))
    return sgmv_tc_run(persona::kModeFused, x, ldx, a_pool, a_slot_stride, a_row_stride, b_pool, b_slot_stride,
                       seg_indptr, seg_slots, num_segments, nullptr, nullptr, y, ldy, T, K, N, R, S, dtype,
                       workspace, workspace_bytes, dev_err, stream);
  int32_t* row_slots = nullptr;
  int st = sgmv_prepare(seg_indptr, seg_slots, num_segments, T, S, workspace, workspace_bytes, dev_err, stream,
                        &row_slots);
  if (st != PERSONA_OK || T == 0) return st;
  return persona_bgmv_fused(x, ldx, a_pool, a_slot_stride, a_row_stride, b_pool, b_slot_stride, row_slots, y, ldy,
                            T, K, N, R, S, dtype, workspace, persona::bgmv_ws_bytes(T), PERSONA_REUSE_PLAN, dev_err,
                            stream);
}

}  // extern "C"

// ------------------------------------------------------------------ NF4 ---
namespace {
int nf4_linear_impl(const persona_nf4_problem* problems, int num_problems, const float* const* addends,
                    const int64_t* ld_addends, int64_t M, void* workspace, size_t workspace_bytes, int32_t* dev_err,
                    cudaStream_t stream);

struct Nf4Plan {
  persona::Nf4GemmArgs args;
  size_t counter_bytes;
  size_t partial_bytes;
};

// Every CTA of the launch gets an equal contiguous range of the problems'
// chunks (tile-major, problem after problem).  A tile that one CTA covers
// whole is written straight to y; a tile split between CTAs is summed from
// their pieces, so the partial buffer holds two pieces (a CTA's first and
// last tile) per CTA.
int nf4_plan(const persona_nf4_problem* probs, int n, Nf4Plan* out) {
  using namespace persona;
  if (n < 1 || n > kNf4MaxProblems || probs == nullptr) return PERSONA_ERR_INVALID_ARG;
  Nf4GemmArgs& a = out->args;
  std::memset(&a, 0, sizeof(a));
  a.num_problems = n;
  int64_t chunks = 0, tiles = 0;
  for (int i = 0; i < n; ++i) {
    const persona_nf4_problem& p = probs[i];
    if (p.N <= 0 || p.K <= 0 || p.N % kNf4Tile || p.K % kNf4Tile || p.N > (int64_t{1} << 24) ||
        p.K > (int64_t{1} << 24))
      return PERSONA_ERR_SHAPE;
    Nf4Problem& q = a.prob[i];
    q.N = static_cast<int>(p.N);
    q.K = static_cast<int>(p.K);
    q.chunk_base = chunks;
    q.counter_base = static_cast<int>(tiles);
    chunks += (p.N / kNf4Tile) * (p.K / kNf4Tile);
    tiles += p.N / kNf4Tile;
  }
  int sms = nf4_sm_count();
  if (sms <= 0) sms = 148;
  const int64_t cap = static_cast<int64_t>(kNf4MaxCtasPerSm) * sms;
  a.chunks = chunks;
  a.max_ctas = static_cast<int>(chunks < cap ? chunks : cap);
  out->counter_bytes = (static_cast<size_t>(tiles) * 4 + 255) & ~size_t(255);
  out->partial_bytes = static_cast<size_t>(a.max_ctas) * 2 * kNf4Tile * kNf4MaxRows * 4;
  return PERSONA_OK;
}
}  // namespace

extern "C" {

size_t persona_nf4_packed_bytes(int64_t N, int64_t K) {
  if (N <= 0 || K <= 0 || N % 128 || K % 128) return 0;
  return static_cast<size_t>(N / 128) * static_cast<size_t>(K / 128) * persona::kNf4ChunkBytes;
}

size_t persona_nf4_quantize_workspace_size(int64_t N, int64_t K) {
  if (N <= 0 || K <= 0 || N % 128 || K % 128) return 0;
  return 256 + static_cast<size_t>(N) * static_cast<size_t>(K / 64) * 4;
}

int persona_nf4_quantize(const void* w, int64_t ldw, int64_t N, int64_t K, void* packed, float* offset,
                         void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  using namespace persona;
  if (w == nullptr || packed == nullptr || offset == nullptr) return PERSONA_ERR_INVALID_ARG;
  if (N <= 0 || K <= 0 || N % 128 || K % 128 || ldw < K || N > (int64_t{1} << 24) || K > (int64_t{1} << 24))
    return PERSONA_ERR_SHAPE;
  if (!aligned16(w) || ldw % 8 || !aligned16(packed) || (reinterpret_cast<uintptr_t>(offset) & 3))
    return PERSONA_ERR_ALIGNMENT;
  if (workspace == nullptr || workspace_bytes < persona_nf4_quantize_workspace_size(N, K))
    return PERSONA_ERR_WORKSPACE;
  if (!aligned16(workspace)) return PERSONA_ERR_ALIGNMENT;
  uint32_t* minmax = static_cast<uint32_t*>(workspace);
  float* absmax = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + 256);
  if (launch_nf4_absmax(static_cast<const uint16_t*>(w), ldw, static_cast<int>(N), static_cast<int>(K), absmax,
                        minmax, stream) != cudaSuccess)
    return PERSONA_ERR_CUDA;
  if (launch_nf4_pack(static_cast<const uint16_t*>(w), ldw, static_cast<int>(N), static_cast<int>(K), absmax, minmax,
                      static_cast<uint8_t*>(packed), offset, stream) != cudaSuccess)
    return PERSONA_ERR_CUDA;
  return PERSONA_OK;
}

int persona_nf4_dequantize(const void* packed, const float* offset, int64_t N, int64_t K, void* w, int64_t ldw,
                           cudaStream_t stream) {
  using namespace persona;
  if (packed == nullptr || offset == nullptr || w == nullptr) return PERSONA_ERR_INVALID_ARG;
  if (N <= 0 || K <= 0 || N % 128 || K % 128 || ldw < K || N > (int64_t{1} << 24) || K > (int64_t{1} << 24))
    return PERSONA_ERR_SHAPE;
  if (!aligned16(packed) || !aligned16(w) || ldw % 8) return PERSONA_ERR_ALIGNMENT;
  return launch_nf4_dequant(static_cast<const uint8_t*>(packed), offset, static_cast<int>(N), static_cast<int>(K),
                            static_cast<uint16_t*>(w), ldw, stream) == cudaSuccess
             ? PERSONA_OK
             : PERSONA_ERR_CUDA;
}

size_t persona_nf4_linear_workspace_size(const persona_nf4_problem* problems, int num_problems) {
  Nf4Plan plan;
  if (nf4_plan(problems, num_problems, &plan) != PERSONA_OK) return 0;
  return plan.counter_bytes + plan.partial_bytes;
}

int persona_nf4_linear(const persona_nf4_problem* problems, int num_problems, int64_t M, void* workspace,
                       size_t workspace_bytes, int32_t* dev_err, cudaStream_t stream) {
  return nf4_linear_impl(problems, num_problems, nullptr, nullptr, M, workspace, workspace_bytes, dev_err, stream);
}

int persona_nf4_linear_add(const persona_nf4_problem* problems, int num_problems, const float* const* addends,
                           const int64_t* ld_addends, int64_t M, void* workspace, size_t workspace_bytes,
                           int32_t* dev_err, cudaStream_t stream) {
  if (addends == nullptr || ld_addends == nullptr) return PERSONA_ERR_INVALID_ARG;
  return nf4_linear_impl(problems, num_problems, addends, ld_addends, M, workspace, workspace_bytes, dev_err, stream);
}

}  // extern "C"

namespace {
int nf4_linear_impl(const persona_nf4_problem* problems, int num_problems, const float* const* addends,
                    const int64_t* ld_addends, int64_t M, void* workspace, size_t workspace_bytes, int32_t* dev_err,
                    cudaStream_t stream) {
  using namespace persona;
  Nf4Plan plan;
  int st = nf4_plan(problems, num_problems, &plan);
  if (st != PERSONA_OK) return st;
  if (M < 0 || M > (int64_t{1} << 30)) return PERSONA_ERR_SHAPE;
  for (int i = 0; i < num_problems; ++i) {
    const persona_nf4_problem& p = problems[i];
    if (p.packed == nullptr || p.offset == nullptr || p.x == nullptr || p.y == nullptr)
      return PERSONA_ERR_INVALID_ARG;
    if (p.ldx < p.K || p.ldy < p.N) return PERSONA_ERR_SHAPE;
    if (!aligned16(p.packed) || !aligned16(p.x) || p.ldx % 8 || (reinterpret_cast<uintptr_t>(p.y) & 1) ||
        (reinterpret_cast<uintptr_t>(p.offset) & 3))
      return PERSONA_ERR_ALIGNMENT;
    if (addends != nullptr && addends[i] != nullptr) {
      if (ld_addends[i] < p.N) return PERSONA_ERR_SHAPE;
      if (reinterpret_cast<uintptr_t>(addends[i]) & 3) return PERSONA_ERR_ALIGNMENT;
    }
  }
  if (M == 0) return PERSONA_OK;
  if (workspace == nullptr || workspace_bytes < plan.counter_bytes + plan.partial_bytes)
    return PERSONA_ERR_WORKSPACE;
  if (!aligned16(workspace)) return PERSONA_ERR_ALIGNMENT;
  Nf4GemmArgs& a = plan.args;
  a.counters = static_cast<int*>(workspace);
  a.partials = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + plan.counter_bytes);
  a.err = dev_err;
  for (int64_t m0 = 0; m0 < M; m0 += kNf4MaxRows) {
    const int mc = static_cast<int>(M - m0 < kNf4MaxRows ? M - m0 : kNf4MaxRows);
    const int m_pad = mc <= 8 ? 8 : mc <= 16 ? 16 : mc <= 32 ? 32 : 64;
    Nf4Maps maps;
    std::memset(&maps, 0, sizeof(maps));
    for (int i = 0; i < num_problems; ++i) {
      const persona_nf4_problem& p = problems[i];
      const uint16_t* x = static_cast<const uint16_t*>(p.x) + m0 * p.ldx;
      if ((st = encode_2d_map(&maps.x[i], x, PERSONA_DTYPE_F16, p.K, mc, p.ldx, 64, m_pad)) != PERSONA_OK) return st;
      a.prob[i].w = static_cast<const uint8_t*>(p.packed);
      a.prob[i].offset = p.offset;
      a.prob[i].y = static_cast<uint16_t*>(p.y) + m0 * p.ldy;
      a.prob[i].ldy = p.ldy;
      a.prob[i].addend = nullptr;
      if (addends != nullptr && addends[i] != nullptr) {
        a.prob[i].addend = addends[i] + m0 * ld_addends[i];
        a.prob[i].ld_addend = ld_addends[i];
      }
    }
    a.M = mc;
    if (launch_nf4_gemm(maps, a, m_pad, stream) != cudaSuccess) return PERSONA_ERR_CUDA;
  }
  return PERSONA_OK;
}
}  // namespace

// ---------------------------------------------------- decode helpers ----
extern "C" {

int persona_add_rmsnorm(void* h, const void* delta, const void* w, void* out, int64_t rows, int64_t D, float eps,
                        cudaStream_t stream) {
  if (h == nullptr || w == nullptr || out == nullptr) return PERSONA_ERR_INVALID_ARG;
  if (rows < 0 || rows > kI32Max || D <= 0 || D % 8 || D > (1 << 20)) return PERSONA_ERR_SHAPE;
  if (!aligned16(h) || !aligned16(w) || !aligned16(out) || (delta != nullptr && !aligned16(delta)))
    return PERSONA_ERR_ALIGNMENT;
  if (rows == 0) return PERSONA_OK;
  return persona::launch_add_rmsnorm(h, delta, w, out, static_cast<int>(rows), static_cast<int>(D), eps, stream) ==
                 cudaSuccess
             ? PERSONA_OK
             : PERSONA_ERR_CUDA;
}

int persona_rope_cache(void* q, void* k, const void* v, void* k_cache, void* v_cache, const int32_t* start,
                       int64_t rows, int64_t per_seq, int64_t Hq, int64_t Hkv, int64_t L, float theta,
                       cudaStream_t stream) {
  if (q == nullptr || k == nullptr || v == nullptr || k_cache == nullptr || v_cache == nullptr || start == nullptr)
    return PERSONA_ERR_INVALID_ARG;
  if (rows < 0 || rows > kI32Max || per_seq <= 0 || Hq <= 0 || Hkv <= 0 || Hq > 256 || Hkv > 256 || L <= 0 ||
      L > kI32Max || !(theta > 1.f))
    return PERSONA_ERR_SHAPE;
  if (rows == 0) return PERSONA_OK;
  return persona::launch_rope_cache(q, k, v, k_cache, v_cache, start, static_cast<int>(rows),
                                    static_cast<int>(per_seq), static_cast<int>(Hq), static_cast<int>(Hkv),
                                    static_cast<int>(L), std::log2(theta), stream) == cudaSuccess
             ? PERSONA_OK
             : PERSONA_ERR_CUDA;
}

int persona_silu_mul(const void* g, const void* u, void* out, int64_t n, cudaStream_t stream) {
  if (g == nullptr || u == nullptr || out == nullptr) return PERSONA_ERR_INVALID_ARG;
  if (n < 0 || n % 8) return PERSONA_ERR_SHAPE;
  if (!aligned16(g) || !aligned16(u) || !aligned16(out)) return PERSONA_ERR_ALIGNMENT;
  if (n == 0) return PERSONA_OK;
  return persona::launch_silu_mul(g, u, out, n, stream) == cudaSuccess ? PERSONA_OK : PERSONA_ERR_CUDA;
}

int persona_rope_decode_attention(void* q, void* k, const void* v, void* k_cache, void* v_cache, const int32_t* pos,
                                  const int32_t* len, void* out, int64_t B, int64_t Hq, int64_t Hkv, int64_t L,
                                  float theta, float scale, cudaStream_t stream) {
  if (q == nullptr || k == nullptr || v == nullptr || k_cache == nullptr || v_cache == nullptr || pos == nullptr ||
      len == nullptr || out == nullptr)
    return PERSONA_ERR_INVALID_ARG;
  if (B < 0 || B > 65535 || Hkv <= 0 || Hq <= 0 || Hq % Hkv || Hq / Hkv > 8 || Hkv > 65535 || L <= 0 ||
      L > kI32Max || !(theta > 1.f))
    return PERSONA_ERR_SHAPE;
  if (!aligned16(k_cache) || !aligned16(v_cache) || (reinterpret_cast<uintptr_t>(q) & 1) ||
      (reinterpret_cast<uintptr_t>(k) & 1) || (reinterpret_cast<uintptr_t>(v) & 1) ||
      (reinterpret_cast<uintptr_t>(out) & 1))
    return PERSONA_ERR_ALIGNMENT;
  if (B == 0) return PERSONA_OK;
  return persona::launch_rope_decode_attention(q, k, v, k_cache, v_cache, pos, len, out, static_cast<int>(B),
                                               static_cast<int>(Hq), static_cast<int>(Hkv), static_cast<int>(L),
                                               std::log2(theta), scale, stream) == cudaSuccess
             ? PERSONA_OK
             : PERSONA_ERR_CUDA;
}

int persona_decode_attention(const void* q, const void* k_cache, const void* v_cache, const int32_t* len, void* out,
                             int64_t B, int64_t Hq, int64_t Hkv, int64_t L, float scale, cudaStream_t stream) {
  if (q == nullptr || k_cache == nullptr || v_cache == nullptr || len == nullptr || out == nullptr)
    return PERSONA_ERR_INVALID_ARG;
  if (B < 0 || B > 65535 || Hkv <= 0 || Hq <= 0 || Hq % Hkv || Hq / Hkv > 8 || Hkv > 65535 || L <= 0 ||
      L > kI32Max)
    return PERSONA_ERR_SHAPE;
  if (!aligned16(k_cache) || !aligned16(v_cache) || (reinterpret_cast<uintptr_t>(q) & 1) ||
      (reinterpret_cast<uintptr_t>(out) & 1))
    return PERSONA_ERR_ALIGNMENT;
  if (B == 0) return PERSONA_OK;
  return persona::launch_decode_attention(q, k_cache, v_cache, len, out, static_cast<int>(B), static_cast<int>(Hq),
                                          static_cast<int>(Hkv), static_cast<int>(L), scale, stream) == cudaSuccess
             ? PERSONA_OK
             : PERSONA_ERR_CUDA;
}

}  // extern "C"

// ------------------------------------------------- LoRA delta at decode ---
extern "C" int persona_bgmv_lora_delta_multi(const persona_bgmv_problem* problems, int num_problems,
                                             float* const* deltas, const int64_t* ld_deltas, const int32_t* slots,
                                             int64_t T, int64_t R, int64_t S, int dtype, int32_t* dev_err,
                                             cudaStream_t stream) {
  if (problems == nullptr || deltas == nullptr || ld_deltas == nullptr || num_problems < 1 ||
      num_problems > PERSONA_MAX_PROBLEMS)
    return PERSONA_ERR_INVALID_ARG;
  if (dtype != PERSONA_DTYPE_F16 && dtype != PERSONA_DTYPE_BF16) return PERSONA_ERR_DTYPE;
  if (T < 0 || S <= 0 || T > PERSONA_SMALL_MAX_ROWS) return PERSONA_ERR_SHAPE;
  if (!rank_supported(R)) return PERSONA_ERR_RANK;
  if (T > 0 && slots == nullptr) return PERSONA_ERR_INVALID_ARG;
  SmallArgs a = {};
  for (int i = 0; i < num_problems; ++i) {
    const persona_bgmv_problem& q = problems[i];
    int st = check_a(q.x, q.ldx, q.a_pool, q.a_slot_stride, q.a_row_stride, q.K, R, S);
    if (st != PERSONA_OK) return st;
    if ((st = check_b(q.b_pool, q.b_slot_stride, deltas[i], ld_deltas[i], q.N, R)) != PERSONA_OK) return st;
    if (q.K < 64 || q.K > 32768) return PERSONA_ERR_SHAPE;
    SmallProblem& p = a.prob[i];
    p.x = q.x;
    p.a = q.a_pool;
    p.b = q.b_pool;
    p.y = nullptr;
    p.ldx = q.ldx;
    p.a_slot_stride = q.a_slot_stride;
    p.a_row_stride = q.a_row_stride;
    p.b_slot_stride = q.b_slot_stride;
    p.ldy = 0;
    p.K = static_cast<int>(q.K);
    p.N = static_cast<int>(q.N);
    p.delta = deltas[i];
    p.ld_delta = ld_deltas[i];
  }
  if (T == 0) return PERSONA_OK;
  a.slots = slots;
  a.err = dev_err;
  a.num_problems = num_problems;
  a.S = static_cast<int>(S);
  return launch_bgmv_small(dtype, static_cast<int>(R), a, static_cast<int>(T), stream) == cudaSuccess
             ? PERSONA_OK
             : PERSONA_ERR_CUDA;
}
