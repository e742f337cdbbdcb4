// persona_bgmv_fused_noalloc: the fused BGMV op with its row-grouping plan in
// a fixed device array of this library instead of a caller workspace.
//
// The array is a file-scope __device__ variable, one copy per device, loaded
// with the library's device code.  Its device address is looked up once per
// device (cudaGetSymbolAddress with that device current) and then handed to
// persona_bgmv_fused as its workspace: the plan kernel writes the plan there,
// then the split kernels use it for their partial sums and counters (at up to
// PERSONA_SMALL_MAX_ROWS rows the decode-sized kernel runs instead and reads
// nothing from it).  Nothing here calls cudaMalloc / cudaFree or any
// allocating routine.
//
// The plan kernel rewrites every field the fused kernel reads (header, row
// permutation, items) and resets the kernel's shared counters on each call,
// so no part of the array has to start at zero.  All calls on one device share the array: calls whose device work
// overlaps in time (different streams, or threads without ordering) race on
// it and must be serialised, e.g. by issuing them on one stream.
#include <mutex>

#include "persona_bgmv.h"
#include "plan_layout.h"

namespace persona {
namespace {

constexpr int64_t kNoAllocMaxRows = PERSONA_NOALLOC_MAX_ROWS;
constexpr size_t kNoAllocPlanBytes = bgmv_ws_bytes(kNoAllocMaxRows);
static_assert(kNoAllocPlanBytes % 16 == 0, "workspace size");

// Host-side name is a stand-in for the per-device copies; only its device
// address (cudaGetSymbolAddress) is ever used.
static __device__ __align__(256) unsigned char g_noalloc_plan[kNoAllocPlanBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch[kMaxDevices] = {};

// Device address of this device's plan array; looked up on first use.
int scratch_for_current_device(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return PERSONA_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return PERSONA_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_scratch[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_plan) != cudaSuccess || p == nullptr) return PERSONA_ERR_CUDA;
    g_scratch[dev] = p;
  }
  *out = g_scratch[dev];
  return PERSONA_OK;
}

}  // namespace
}  // namespace persona

extern "C" int persona_bgmv_fused_noalloc(const void* x, int64_t ldx, const void* a_pool, int64_t a_slot_stride,
                                          int64_t a_row_stride, const void* b_pool, int64_t b_slot_stride,
                                          const int32_t* slots, void* y, int64_t ldy, int64_t T, int64_t K,
                                          int64_t N, int64_t R, int64_t S, int dtype, int32_t* dev_err,
                                          cudaStream_t stream) {
  using namespace persona;
  if (T > kNoAllocMaxRows) return PERSONA_ERR_NOALLOC_ROWS;
  if (T < 0) return PERSONA_ERR_SHAPE;
  if (T == 0) return PERSONA_OK;
  void* scratch = nullptr;
  const int st = scratch_for_current_device(&scratch);
  if (st != PERSONA_OK) return st;
  return persona_bgmv_fused(x, ldx, a_pool, a_slot_stride, a_row_stride, b_pool, b_slot_stride, slots, y, ldy, T, K,
                            N, R, S, dtype, scratch, kNoAllocPlanBytes, 0, dev_err, stream);
}
