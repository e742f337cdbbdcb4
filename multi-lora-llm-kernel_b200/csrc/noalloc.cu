// persona_bgmv_fused_noalloc: the fused BGMV op with its workspace in a
// fixed device array of this library instead of a buffer from the caller.
//
// The array is a file-scope __device__ variable, one copy per device, loaded
// with the library's device code.  Its device address is looked up once per
// device, by the first call on that device (cudaGetSymbolAddress with that
// device current; make that first call before any stream capture begins),
// and then handed to the fused op as its workspace: above
// PERSONA_SMALL_MAX_ROWS rows the plan kernel writes the row grouping there
// and the split kernel keeps its partial sums and counters there.  At up to PERSONA_SMALL_MAX_ROWS rows
// the decode-sized kernel runs, which needs no plan, so such calls neither
// read nor write the array.  Nothing here calls cudaMalloc / cudaFree or any
// allocating routine.
//
// The plan kernel rewrites every field the split kernel reads (header, row
// permutation, items) and resets its shared counters on each call, so no
// part of the array has to start at zero.  All calls on one device share the
// array: calls whose device work overlaps in time (different streams, or
// threads without ordering) race on it and must be serialised, e.g. by
// issuing them on one stream.
#include <mutex>

#include "bgmv_args.h"
#include "persona_bgmv.h"
#include "plan_layout.h"

namespace persona {
namespace {

constexpr int64_t kNoAllocMaxRows = PERSONA_NOALLOC_MAX_ROWS;
constexpr size_t kNoAllocPlanBytes = bgmv_ws_bytes(kNoAllocMaxRows);
static_assert(kNoAllocPlanBytes % 16 == 0, "workspace size");

// Host-side name is a stand-in for the per-device copies; only its device
// address (cudaGetSymbolAddress) is ever used.
static __device__ __align__(256) unsigned char g_noalloc_ws[kNoAllocPlanBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch[kMaxDevices] = {};

// Device address of this device's workspace array; looked up on first use.
int scratch_for_current_device(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return PERSONA_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return PERSONA_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_scratch[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_ws) != cudaSuccess || p == nullptr) return PERSONA_ERR_CUDA;
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
  return fused_impl(x, ldx, a_pool, a_slot_stride, a_row_stride, b_pool, b_slot_stride, slots, y, ldy, T, K, N, R, S,
                    dtype, scratch, kNoAllocPlanBytes, 0, dev_err, stream, /*plan_small=*/false);
}
