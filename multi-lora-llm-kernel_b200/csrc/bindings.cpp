// torch.ops.persona registration over the C ABI of libpersona_bgmv.so.
//
// The three reference schemas are registered byte-identically on the CUDA
// dispatch key (reference csrc/bindings.cpp:19-29), with the same C++ host
// symbols (bgmv_shrink_cuda, bgmv_expand_cuda, persona::gemv_fp16_cuda) and
// the same TORCH_CHECK messages.  New ops (fused, planned variants, plan)
// are registered beside them.  Python module persona._C keeps `noop`
// (reference csrc/bindings.cpp:31-33) and adds the device error word
// helpers.
//
// Slot validation: the reference syncs with the host once per row
// (csrc/bgmv_shrink.cu:106-109).  Here the device flags an out-of-range
// slot in a per-device error word held in mapped pinned host memory; every
// op first reads that word (no sync) and raises RuntimeError if an earlier
// call flagged it, and PERSONA_STRICT_SLOTS=1 makes each op synchronise and
// raise on its own call instead.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>
#include <torch/library.h>

#include <cstdlib>
#include <mutex>
#include <sstream>

#include "persona_bgmv.h"

namespace {

constexpr int kMaxDevices = 64;

struct ErrorWords {
  std::mutex mu;
  int32_t* host[kMaxDevices] = {};
};
ErrorWords& error_words() {
  static ErrorWords w;
  return w;
}

// Mapped pinned int32 of `device` (allocated on first use), host view.
int32_t* error_word_host(int device) {
  TORCH_CHECK(device >= 0 && device < kMaxDevices, "persona: device index out of range");
  auto& w = error_words();
  std::lock_guard<std::mutex> lock(w.mu);
  if (w.host[device] == nullptr) {
    void* p = nullptr;
    C10_CUDA_CHECK(cudaHostAlloc(&p, sizeof(int32_t), cudaHostAllocMapped | cudaHostAllocPortable));
    *static_cast<volatile int32_t*>(p) = 0;
    w.host[device] = static_cast<int32_t*>(p);
  }
  return w.host[device];
}

int32_t* error_word_device(int device) {
  static int32_t* dev_ptr[kMaxDevices] = {};
  if (dev_ptr[device] == nullptr) {
    int32_t* h = error_word_host(device);
    void* d = nullptr;
    C10_CUDA_CHECK(cudaHostGetDevicePointer(&d, h, 0));
    dev_ptr[device] = static_cast<int32_t*>(d);
  }
  return dev_ptr[device];
}

std::string describe_error(int bits) {
  std::ostringstream os;
  os << "persona: a BGMV/SGMV call on this device flagged an error (bits 0x" << std::hex << bits
     << std::dec << "):";
  if (bits & PERSONA_DEV_ERR_SLOT) os << " slot out of range;";
  if (bits & PERSONA_DEV_ERR_TIMEOUT) os << " device wait timed out;";
  if (bits & PERSONA_DEV_ERR_SEGMENT) os << " invalid segment table;";
  if (bits & PERSONA_DEV_ERR_PLAN) os << " reused plan does not match the call;";
  return os.str();
}

// Raise (and clear) an error flagged by an earlier call on `device`.
void raise_pending(int device, const char* op) {
  volatile int32_t* h = error_word_host(device);
  const int bits = *h;
  if (bits != 0) {
    *h = 0;
    TORCH_CHECK(false, op, ": ", describe_error(bits));
  }
}

bool strict_slots() {
  static const bool strict = [] {
    const char* e = std::getenv("PERSONA_STRICT_SLOTS");
    return e != nullptr && e[0] == '1';
  }();
  return strict;
}

void after_launch(int device, const char* op, cudaStream_t stream) {
  if (!strict_slots()) return;
  C10_CUDA_CHECK(cudaStreamSynchronize(stream));
  volatile int32_t* h = error_word_host(device);
  const int bits = *h;
  if (bits & PERSONA_DEV_ERR_SLOT) {
    *h = 0;
    TORCH_CHECK(false, op, ": slot out of range");
  }
  raise_pending(device, op);
}

void check_status(int st, const char* op) {
  TORCH_CHECK(st == PERSONA_OK, op, ": ", persona_status_string(st));
}

int dtype_code(const at::Tensor& t, const char* op) {
  if (t.scalar_type() == at::kHalf) return PERSONA_DTYPE_F16;
  if (t.scalar_type() == at::kBFloat16) return PERSONA_DTYPE_BF16;
  TORCH_CHECK(false, op, ": only float16 and bfloat16 supported");
  return -1;
}

// Row-major [rows, cols] with unit inner stride (a view of a wider buffer is
// fine); returns the row stride in elements.
int64_t row_stride(const at::Tensor& t) { return t.size(0) <= 1 ? t.size(1) : t.stride(0); }

// Sized for a multi-projection launch, so that any plan serves every op.
at::Tensor workspace_for(int64_t T, const at::Tensor& like) {
  const size_t bytes = persona_bgmv_multi_workspace_size(T, PERSONA_MAX_PROBLEMS);
  return at::empty({static_cast<int64_t>(bytes)}, like.options().dtype(at::kByte));
}

void check_pool_a(const at::Tensor& a_pool, const char* op) {
  TORCH_CHECK(a_pool.dim() == 3, op, ": a_pool must be [S, R, K]");
  TORCH_CHECK(a_pool.stride(2) == 1, op, ": tensors must be contiguous");
}

void check_pool_b(const at::Tensor& b_pool, const char* op) {
  TORCH_CHECK(b_pool.dim() == 3, op, ": b_pool must be [S, N, R]");
  TORCH_CHECK(b_pool.stride(2) == 1 && b_pool.stride(1) == b_pool.size(2), op,
              ": tensors must be contiguous");
}

void shrink_impl(const at::Tensor& x, const at::Tensor& a_pool, const at::Tensor& slots,
                 at::Tensor& v, const c10::optional<at::Tensor>& plan) {
  const char* op = "bgmv_shrink";
  TORCH_CHECK(x.is_cuda() && a_pool.is_cuda() && slots.is_cuda() && v.is_cuda(),
              "bgmv_shrink: all tensors must be CUDA");
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && slots.is_contiguous() && v.is_contiguous(),
              "bgmv_shrink: tensors must be contiguous");
  check_pool_a(a_pool, op);
  TORCH_CHECK(slots.scalar_type() == at::kInt, "bgmv_shrink: slots must be int32");
  TORCH_CHECK(v.scalar_type() == at::kFloat, "bgmv_shrink: v must be float32");
  const int64_t T = x.size(0), K = x.size(1), S = a_pool.size(0), R = a_pool.size(1);
  TORCH_CHECK(a_pool.size(2) == K, "bgmv_shrink: a_pool shape mismatch");
  TORCH_CHECK(slots.dim() == 1 && slots.size(0) == T, "bgmv_shrink: slots length must match T");
  TORCH_CHECK(v.dim() == 2 && v.size(0) == T && v.size(1) == R, "bgmv_shrink: v shape mismatch");
  TORCH_CHECK(K % 8 == 0, "bgmv_shrink: K must be a multiple of 8");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0, "bgmv_shrink: x must be 16-byte aligned");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(a_pool.data_ptr()) % 16 == 0,
              "bgmv_shrink: a_pool must be 16-byte aligned");
  const int dt = dtype_code(x, op);
  TORCH_CHECK(a_pool.scalar_type() == x.scalar_type(), "bgmv_shrink: dtype mismatch");
  const at::cuda::OptionalCUDAGuard guard(x.device());
  const int dev = x.get_device();
  raise_pending(dev, op);
  if (T == 0) return;
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  at::Tensor ws = plan.has_value() ? *plan : workspace_for(T, x);
  const int flags = plan.has_value() ? PERSONA_REUSE_PLAN : 0;
  TORCH_CHECK(static_cast<size_t>(ws.numel()) >= persona_bgmv_workspace_size(T),
              "bgmv_shrink: plan was built for fewer rows");
  const int st = persona_bgmv_shrink(x.data_ptr(), row_stride(x), a_pool.data_ptr(), a_pool.stride(0),
                                     a_pool.stride(1), slots.data_ptr<int32_t>(), v.data_ptr<float>(), T,
                                     K, R, S, dt, ws.data_ptr(), ws.numel(), flags,
                                     error_word_device(dev), stream);
  check_status(st, op);
  after_launch(dev, op, stream);
}

void expand_impl(const at::Tensor& v, const at::Tensor& b_pool, const at::Tensor& slots, at::Tensor& y,
                 const c10::optional<at::Tensor>& plan) {
  const char* op = "bgmv_expand";
  TORCH_CHECK(v.is_cuda() && b_pool.is_cuda() && slots.is_cuda() && y.is_cuda(),
              "bgmv_expand: all tensors must be CUDA");
  TORCH_CHECK(v.is_contiguous() && slots.is_contiguous() && y.dim() == 2 && y.stride(1) == 1,
              "bgmv_expand: tensors must be contiguous");
  check_pool_b(b_pool, op);
  TORCH_CHECK(slots.scalar_type() == at::kInt, "bgmv_expand: slots must be int32");
  TORCH_CHECK(v.scalar_type() == at::kFloat, "bgmv_expand: v must be float32");
  const int64_t T = v.size(0), R = v.size(1), S = b_pool.size(0), N = b_pool.size(1);
  TORCH_CHECK(b_pool.size(2) == R, "bgmv_expand: b_pool rank dim mismatch");
  TORCH_CHECK(slots.dim() == 1 && slots.size(0) == T, "bgmv_expand: slots length must match T");
  TORCH_CHECK(y.size(0) == T && y.size(1) == N, "bgmv_expand: y shape mismatch");
  TORCH_CHECK(N % 8 == 0, "bgmv_expand: N must be a multiple of 8");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(b_pool.data_ptr()) % 16 == 0,
              "bgmv_expand: b_pool must be 16-byte aligned");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(y.data_ptr()) % 16 == 0, "bgmv_expand: y must be 16-byte aligned");
  TORCH_CHECK(R == 8 || R == 16 || R == 32 || R == 64, "bgmv_expand: R must be 8, 16, 32, or 64");
  const int dt = dtype_code(y, op);
  TORCH_CHECK(b_pool.scalar_type() == y.scalar_type(), "bgmv_expand: dtype mismatch");
  const at::cuda::OptionalCUDAGuard guard(v.device());
  const int dev = v.get_device();
  raise_pending(dev, op);
  if (T == 0) return;
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  at::Tensor ws = plan.has_value() ? *plan : workspace_for(T, v);
  const int flags = plan.has_value() ? PERSONA_REUSE_PLAN : 0;
  TORCH_CHECK(static_cast<size_t>(ws.numel()) >= persona_bgmv_workspace_size(T),
              "bgmv_expand: plan was built for fewer rows");
  const int st = persona_bgmv_expand(v.data_ptr<float>(), b_pool.data_ptr(), b_pool.stride(0),
                                     slots.data_ptr<int32_t>(), y.data_ptr(), row_stride(y), T, N, R, S,
                                     dt, ws.data_ptr(), ws.numel(), flags, error_word_device(dev), stream);
  check_status(st, op);
  after_launch(dev, op, stream);
}

void fused_impl(const at::Tensor& x, const at::Tensor& a_pool, const at::Tensor& b_pool,
                const at::Tensor& slots, at::Tensor& y, const c10::optional<at::Tensor>& plan) {
  const char* op = "bgmv_fused";
  TORCH_CHECK(x.is_cuda() && a_pool.is_cuda() && b_pool.is_cuda() && slots.is_cuda() && y.is_cuda(),
              "bgmv_fused: all tensors must be CUDA");
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && slots.is_contiguous() && y.dim() == 2 &&
                  y.stride(1) == 1,
              "bgmv_fused: tensors must be contiguous");
  check_pool_a(a_pool, op);
  check_pool_b(b_pool, op);
  TORCH_CHECK(slots.scalar_type() == at::kInt, "bgmv_fused: slots must be int32");
  const int64_t T = x.size(0), K = x.size(1), S = a_pool.size(0), R = a_pool.size(1), N = b_pool.size(1);
  TORCH_CHECK(a_pool.size(2) == K, "bgmv_fused: a_pool shape mismatch");
  TORCH_CHECK(b_pool.size(0) == S && b_pool.size(2) == R, "bgmv_fused: b_pool shape mismatch");
  TORCH_CHECK(slots.dim() == 1 && slots.size(0) == T, "bgmv_fused: slots length must match T");
  TORCH_CHECK(y.size(0) == T && y.size(1) == N, "bgmv_fused: y shape mismatch");
  const int dt = dtype_code(x, op);
  TORCH_CHECK(a_pool.scalar_type() == x.scalar_type() && b_pool.scalar_type() == x.scalar_type() &&
                  y.scalar_type() == x.scalar_type(),
              "bgmv_fused: dtype mismatch");
  const at::cuda::OptionalCUDAGuard guard(x.device());
  const int dev = x.get_device();
  raise_pending(dev, op);
  if (T == 0) return;
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  at::Tensor ws = plan.has_value() ? *plan : workspace_for(T, x);
  const int flags = plan.has_value() ? PERSONA_REUSE_PLAN : 0;
  TORCH_CHECK(static_cast<size_t>(ws.numel()) >= persona_bgmv_workspace_size(T),
              "bgmv_fused: plan was built for fewer rows");
  const int st = persona_bgmv_fused(x.data_ptr(), row_stride(x), a_pool.data_ptr(), a_pool.stride(0),
                                    a_pool.stride(1), b_pool.data_ptr(), b_pool.stride(0),
                                    slots.data_ptr<int32_t>(), y.data_ptr(), row_stride(y), T, K, N, R,
                                    S, dt, ws.data_ptr(), ws.numel(), flags, error_word_device(dev),
                                    stream);
  check_status(st, op);
  after_launch(dev, op, stream);
}

void fused_multi_impl(at::TensorList xs, at::TensorList a_pools, at::TensorList b_pools, const at::Tensor& slots,
                      at::TensorList ys, const c10::optional<at::Tensor>& plan) {
  const char* op = "bgmv_fused_multi";
  const int P = static_cast<int>(xs.size());
  TORCH_CHECK(P >= 1 && P <= PERSONA_MAX_PROBLEMS, op, ": 1 to ", PERSONA_MAX_PROBLEMS, " projections");
  TORCH_CHECK(a_pools.size() == xs.size() && b_pools.size() == xs.size() && ys.size() == xs.size(), op,
              ": xs, a_pools, b_pools and ys must have the same length");
  TORCH_CHECK(slots.is_cuda() && slots.is_contiguous() && slots.dim() == 1 && slots.scalar_type() == at::kInt, op,
              ": slots must be a contiguous int32 CUDA vector");
  const int64_t T = slots.size(0);
  const int64_t S = a_pools[0].size(0), R = a_pools[0].size(1);
  const int dt = dtype_code(xs[0], op);
  persona_bgmv_problem probs[PERSONA_MAX_PROBLEMS];
  for (int p = 0; p < P; ++p) {
    const at::Tensor &x = xs[p], &a = a_pools[p], &b = b_pools[p], &y = ys[p];
    TORCH_CHECK(x.is_cuda() && a.is_cuda() && b.is_cuda() && y.is_cuda(), op, ": all tensors must be CUDA");
    TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && y.dim() == 2 && y.stride(1) == 1, op,
                ": tensors must be contiguous");
    check_pool_a(a, op);
    check_pool_b(b, op);
    TORCH_CHECK(x.size(0) == T && y.size(0) == T, op, ": x / y rows must match slots");
    TORCH_CHECK(a.size(0) == S && a.size(1) == R && a.size(2) == x.size(1), op, ": a_pool shape mismatch");
    TORCH_CHECK(b.size(0) == S && b.size(2) == R && b.size(1) == y.size(1), op, ": b_pool shape mismatch");
    TORCH_CHECK(x.scalar_type() == xs[0].scalar_type() && a.scalar_type() == x.scalar_type() &&
                    b.scalar_type() == x.scalar_type() && y.scalar_type() == x.scalar_type(),
                op, ": dtype mismatch");
    TORCH_CHECK(x.get_device() == slots.get_device() && y.get_device() == slots.get_device(), op,
                ": tensors on different devices");
    probs[p] = persona_bgmv_problem{x.data_ptr(), row_stride(x), a.data_ptr(), a.stride(0), a.stride(1),
                                    b.data_ptr(), b.stride(0),   y.data_ptr(), row_stride(y), x.size(1),
                                    y.size(1)};
  }
  const at::cuda::OptionalCUDAGuard guard(slots.device());
  const int dev = slots.get_device();
  raise_pending(dev, op);
  if (T == 0) return;
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  at::Tensor ws = plan.has_value() ? *plan : workspace_for(T, slots);
  const int flags = plan.has_value() ? PERSONA_REUSE_PLAN : 0;
  TORCH_CHECK(static_cast<size_t>(ws.numel()) >= persona_bgmv_multi_workspace_size(T, P), op,
              ": plan was built for fewer rows");
  check_status(persona_bgmv_fused_multi(probs, P, slots.data_ptr<int32_t>(), T, R, S, dt, ws.data_ptr(),
                                        ws.numel(), flags, error_word_device(dev), stream),
               op);
  after_launch(dev, op, stream);
}

at::Tensor plan_impl(const at::Tensor& slots, int64_t S) {
  const char* op = "bgmv_plan";
  TORCH_CHECK(slots.is_cuda(), "bgmv_plan: all tensors must be CUDA");
  TORCH_CHECK(slots.is_contiguous() && slots.dim() == 1, "bgmv_plan: tensors must be contiguous");
  TORCH_CHECK(slots.scalar_type() == at::kInt, "bgmv_plan: slots must be int32");
  const at::cuda::OptionalCUDAGuard guard(slots.device());
  const int dev = slots.get_device();
  raise_pending(dev, op);
  const int64_t T = slots.size(0);
  at::Tensor ws = workspace_for(T, slots);
  if (T == 0) return ws;
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  check_status(persona_bgmv_plan(slots.data_ptr<int32_t>(), T, S, ws.data_ptr(), ws.numel(),
                                 error_word_device(dev), stream),
               op);
  after_launch(dev, op, stream);
  return ws;
}

}  // namespace

// Same C++ host symbols as the reference (csrc/bgmv_shrink.cu:81, csrc/bgmv_expand.cu:88).
void bgmv_shrink_cuda(const at::Tensor& x, const at::Tensor& a_pool, const at::Tensor& slots, at::Tensor& v) {
  shrink_impl(x, a_pool, slots, v, c10::nullopt);
}

void bgmv_expand_cuda(const at::Tensor& v, const at::Tensor& b_pool, const at::Tensor& slots, at::Tensor& y) {
  expand_impl(v, b_pool, slots, y, c10::nullopt);
}

namespace persona {
// Reference csrc/gemv_fp16.cu:33-50.
void gemv_fp16_cuda(const at::Tensor& x, const at::Tensor& W, at::Tensor& y) {
  TORCH_CHECK(x.is_cuda() && W.is_cuda() && y.is_cuda(), "gemv_fp16: CUDA only");
  TORCH_CHECK(x.dim() == 1 && W.dim() == 2 && y.dim() == 1, "gemv_fp16: shape");
  const int64_t K = x.size(0), N = W.size(0);
  TORCH_CHECK(W.size(1) == K && y.size(0) == N, "gemv_fp16: mismatch");
  TORCH_CHECK(x.scalar_type() == at::kHalf && W.scalar_type() == at::kHalf && y.scalar_type() == at::kHalf,
              "gemv_fp16: half only in v1 scaffold");
  TORCH_CHECK(x.is_contiguous() && W.is_contiguous() && y.is_contiguous(), "gemv_fp16: contiguous only");
  const at::cuda::OptionalCUDAGuard guard(x.device());
  check_status(persona_gemv_fp16(x.data_ptr(), W.data_ptr(), y.data_ptr(), K, N,
                                 at::cuda::getCurrentCUDAStream()),
               "gemv_fp16");
}
}  // namespace persona

namespace {
void shrink_with_plan(const at::Tensor& x, const at::Tensor& a_pool, const at::Tensor& slots,
                      const at::Tensor& plan, at::Tensor& v) {
  shrink_impl(x, a_pool, slots, v, plan);
}
void expand_with_plan(const at::Tensor& v, const at::Tensor& b_pool, const at::Tensor& slots,
                      const at::Tensor& plan, at::Tensor& y) {
  expand_impl(v, b_pool, slots, y, plan);
}
void fused_noplan(const at::Tensor& x, const at::Tensor& a_pool, const at::Tensor& b_pool,
                  const at::Tensor& slots, at::Tensor& y) {
  fused_impl(x, a_pool, b_pool, slots, y, c10::nullopt);
}
void fused_with_plan(const at::Tensor& x, const at::Tensor& a_pool, const at::Tensor& b_pool,
                     const at::Tensor& slots, const at::Tensor& plan, at::Tensor& y) {
  fused_impl(x, a_pool, b_pool, slots, y, plan);
}
}  // namespace

namespace {
void check_segments(const at::Tensor& indptr, const at::Tensor& seg_slots, const char* op) {
  TORCH_CHECK(indptr.is_cuda() && seg_slots.is_cuda(), op, ": all tensors must be CUDA");
  TORCH_CHECK(indptr.dim() == 1 && seg_slots.dim() == 1 && indptr.size(0) == seg_slots.size(0) + 1, op,
              ": seg_indptr must have one more entry than seg_slots");
  TORCH_CHECK(indptr.is_contiguous() && seg_slots.is_contiguous(), op, ": tensors must be contiguous");
  TORCH_CHECK(indptr.scalar_type() == at::kInt && seg_slots.scalar_type() == at::kInt, op,
              ": seg_indptr and seg_slots must be int32");
}

at::Tensor sgmv_workspace(int64_t T, const at::Tensor& like) {
  return at::empty({static_cast<int64_t>(persona_sgmv_workspace_size(T))}, like.options().dtype(at::kByte));
}

void sgmv_shrink_op(const at::Tensor& x, const at::Tensor& a_pool, const at::Tensor& indptr,
                    const at::Tensor& seg_slots, at::Tensor& v) {
  const char* op = "sgmv_shrink";
  check_segments(indptr, seg_slots, op);
  TORCH_CHECK(x.is_cuda() && a_pool.is_cuda() && v.is_cuda(), "sgmv_shrink: all tensors must be CUDA");
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && v.is_contiguous(), "sgmv_shrink: tensors must be contiguous");
  check_pool_a(a_pool, op);
  TORCH_CHECK(v.scalar_type() == at::kFloat, "sgmv_shrink: v must be float32");
  const int64_t T = x.size(0), K = x.size(1), S = a_pool.size(0), R = a_pool.size(1);
  TORCH_CHECK(a_pool.size(2) == K, "sgmv_shrink: a_pool shape mismatch");
  TORCH_CHECK(v.dim() == 2 && v.size(0) == T && v.size(1) == R, "sgmv_shrink: v shape mismatch");
  const int dt = dtype_code(x, op);
  TORCH_CHECK(a_pool.scalar_type() == x.scalar_type(), "sgmv_shrink: dtype mismatch");
  const at::cuda::OptionalCUDAGuard guard(x.device());
  const int dev = x.get_device();
  raise_pending(dev, op);
  if (T == 0) return;
  at::Tensor ws = sgmv_workspace(T, x);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  check_status(persona_sgmv_shrink(x.data_ptr(), row_stride(x), a_pool.data_ptr(), a_pool.stride(0),
                                   a_pool.stride(1), indptr.data_ptr<int32_t>(), seg_slots.data_ptr<int32_t>(),
                                   seg_slots.size(0), v.data_ptr<float>(), T, K, R, S, dt, ws.data_ptr(),
                                   ws.numel(), error_word_device(dev), stream),
               op);
  after_launch(dev, op, stream);
}

void sgmv_expand_op(const at::Tensor& v, const at::Tensor& b_pool, const at::Tensor& indptr,
                    const at::Tensor& seg_slots, at::Tensor& y) {
  const char* op = "sgmv_expand";
  check_segments(indptr, seg_slots, op);
  TORCH_CHECK(v.is_cuda() && b_pool.is_cuda() && y.is_cuda(), "sgmv_expand: all tensors must be CUDA");
  TORCH_CHECK(v.is_contiguous() && y.dim() == 2 && y.stride(1) == 1, "sgmv_expand: tensors must be contiguous");
  check_pool_b(b_pool, op);
  TORCH_CHECK(v.scalar_type() == at::kFloat, "sgmv_expand: v must be float32");
  const int64_t T = v.size(0), R = v.size(1), S = b_pool.size(0), N = b_pool.size(1);
  TORCH_CHECK(b_pool.size(2) == R, "sgmv_expand: b_pool rank dim mismatch");
  TORCH_CHECK(y.size(0) == T && y.size(1) == N, "sgmv_expand: y shape mismatch");
  const int dt = dtype_code(y, op);
  TORCH_CHECK(b_pool.scalar_type() == y.scalar_type(), "sgmv_expand: dtype mismatch");
  const at::cuda::OptionalCUDAGuard guard(v.device());
  const int dev = v.get_device();
  raise_pending(dev, op);
  if (T == 0) return;
  at::Tensor ws = sgmv_workspace(T, v);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  check_status(persona_sgmv_expand(v.data_ptr<float>(), b_pool.data_ptr(), b_pool.stride(0),
                                   indptr.data_ptr<int32_t>(), seg_slots.data_ptr<int32_t>(), seg_slots.size(0),
                                   y.data_ptr(), row_stride(y), T, N, R, S, dt, ws.data_ptr(), ws.numel(),
                                   error_word_device(dev), stream),
               op);
  after_launch(dev, op, stream);
}

void sgmv_fused_op(const at::Tensor& x, const at::Tensor& a_pool, const at::Tensor& b_pool,
                   const at::Tensor& indptr, const at::Tensor& seg_slots, at::Tensor& y) {
  const char* op = "sgmv_fused";
  check_segments(indptr, seg_slots, op);
  TORCH_CHECK(x.is_cuda() && a_pool.is_cuda() && b_pool.is_cuda() && y.is_cuda(),
              "sgmv_fused: all tensors must be CUDA");
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && y.dim() == 2 && y.stride(1) == 1,
              "sgmv_fused: tensors must be contiguous");
  check_pool_a(a_pool, op);
  check_pool_b(b_pool, op);
  const int64_t T = x.size(0), K = x.size(1), S = a_pool.size(0), R = a_pool.size(1), N = b_pool.size(1);
  TORCH_CHECK(a_pool.size(2) == K && b_pool.size(0) == S && b_pool.size(2) == R, "sgmv_fused: pool shape mismatch");
  TORCH_CHECK(y.size(0) == T && y.size(1) == N, "sgmv_fused: y shape mismatch");
  const int dt = dtype_code(x, op);
  TORCH_CHECK(a_pool.scalar_type() == x.scalar_type() && b_pool.scalar_type() == x.scalar_type() &&
                  y.scalar_type() == x.scalar_type(),
              "sgmv_fused: dtype mismatch");
  const at::cuda::OptionalCUDAGuard guard(x.device());
  const int dev = x.get_device();
  raise_pending(dev, op);
  if (T == 0) return;
  at::Tensor ws = sgmv_workspace(T, x);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  check_status(persona_sgmv_fused(x.data_ptr(), row_stride(x), a_pool.data_ptr(), a_pool.stride(0),
                                  a_pool.stride(1), b_pool.data_ptr(), b_pool.stride(0), indptr.data_ptr<int32_t>(),
                                  seg_slots.data_ptr<int32_t>(), seg_slots.size(0), y.data_ptr(), row_stride(y), T,
                                  K, N, R, S, dt, ws.data_ptr(), ws.numel(), error_word_device(dev), stream),
               op);
  after_launch(dev, op, stream);
}
}  // namespace

namespace {
// ------------------------------------------------------------------ NF4 ---
// Base linears of the end-to-end decode (persona_nf4_* in the C ABI).
std::tuple<at::Tensor, at::Tensor> nf4_quantize_op(const at::Tensor& w) {
  const char* op = "nf4_quantize";
  TORCH_CHECK(w.is_cuda() && w.dim() == 2 && w.stride(1) == 1, op, ": w must be a CUDA [N, K] matrix");
  TORCH_CHECK(w.scalar_type() == at::kHalf, op, ": w must be float16");
  const int64_t N = w.size(0), K = w.size(1);
  TORCH_CHECK(N % 128 == 0 && K % 128 == 0 && N > 0 && K > 0, op, ": N and K must be multiples of 128");
  const at::cuda::OptionalCUDAGuard guard(w.device());
  auto u8 = w.options().dtype(at::kByte);
  at::Tensor packed = at::empty({N / 128, K / 128, PERSONA_NF4_CHUNK_BYTES}, u8);
  at::Tensor offset = at::empty({1}, w.options().dtype(at::kFloat));
  at::Tensor ws = at::empty({static_cast<int64_t>(persona_nf4_quantize_workspace_size(N, K))}, u8);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  check_status(persona_nf4_quantize(w.data_ptr(), row_stride(w), N, K, packed.data_ptr(), offset.data_ptr<float>(),
                                    ws.data_ptr(), ws.numel(), stream),
               op);
  after_launch(w.get_device(), op, stream);
  return {packed, offset};
}

void check_nf4_weight(const at::Tensor& packed, const at::Tensor& offset, int64_t N, int64_t K, const char* op) {
  TORCH_CHECK(packed.is_cuda() && offset.is_cuda(), op, ": tensors must be CUDA");
  TORCH_CHECK(packed.scalar_type() == at::kByte && packed.is_contiguous() && packed.dim() == 3 &&
                  packed.size(0) * 128 == N && packed.size(1) * 128 == K && packed.size(2) == PERSONA_NF4_CHUNK_BYTES,
              op, ": packed must be uint8 [N/128, K/128, ", PERSONA_NF4_CHUNK_BYTES, "]");
  TORCH_CHECK(offset.scalar_type() == at::kFloat && offset.numel() == 1, op, ": offset must be one float32");
}

at::Tensor nf4_dequantize_op(const at::Tensor& packed, const at::Tensor& offset, int64_t N, int64_t K) {
  const char* op = "nf4_dequantize";
  check_nf4_weight(packed, offset, N, K, op);
  const at::cuda::OptionalCUDAGuard guard(packed.device());
  at::Tensor w = at::empty({N, K}, packed.options().dtype(at::kHalf));
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  check_status(persona_nf4_dequantize(packed.data_ptr(), offset.data_ptr<float>(), N, K, w.data_ptr(), K, stream),
               op);
  after_launch(packed.get_device(), op, stream);
  return w;
}

// Per-device workspace of the NF4 linear: zero-filled when made or grown
// (its counters must start at zero; the kernel leaves them at zero).
at::Tensor nf4_workspace(size_t bytes, const at::Tensor& like) {
  static std::mutex mu;
  static std::vector<at::Tensor> cache(64);
  const int dev = like.get_device();
  TORCH_CHECK(dev >= 0 && dev < 64, "nf4_linear: device index out of range");
  std::lock_guard<std::mutex> lock(mu);
  at::Tensor& t = cache[dev];
  if (!t.defined() || static_cast<size_t>(t.numel()) < bytes)
    t = at::zeros({static_cast<int64_t>(bytes)}, like.options().dtype(at::kByte));
  return t;
}

void nf4_linear_op(const at::Tensor& x, at::TensorList packed, at::TensorList offsets, at::TensorList ys) {
  const char* op = "nf4_linear";
  const int n = static_cast<int>(packed.size());
  TORCH_CHECK(n >= 1 && n <= PERSONA_NF4_MAX_PROBLEMS, op, ": 1 to ", PERSONA_NF4_MAX_PROBLEMS, " weights");
  TORCH_CHECK(static_cast<int>(offsets.size()) == n && static_cast<int>(ys.size()) == n, op,
              ": one offset and one y per weight");
  TORCH_CHECK(x.is_cuda() && x.dim() == 2 && x.stride(1) == 1 && x.scalar_type() == at::kHalf, op,
              ": x must be a CUDA float16 [M, K] matrix with unit inner stride");
  const int64_t M = x.size(0), K = x.size(1);
  persona_nf4_problem probs[PERSONA_NF4_MAX_PROBLEMS];
  for (int i = 0; i < n; ++i) {
    const at::Tensor& y = ys[i];
    TORCH_CHECK(y.is_cuda() && y.dim() == 2 && y.stride(1) == 1 && y.scalar_type() == at::kHalf && y.size(0) == M,
                op, ": y must be a CUDA float16 [M, N] matrix with unit inner stride");
    const int64_t N = y.size(1);
    check_nf4_weight(packed[i], offsets[i], N, K, op);
    TORCH_CHECK(packed[i].get_device() == x.get_device() && y.get_device() == x.get_device(), op,
                ": tensors must be on one device");
    probs[i] = persona_nf4_problem{packed[i].data_ptr(), offsets[i].data_ptr<float>(), x.data_ptr(), row_stride(x),
                                   y.data_ptr(), row_stride(y), N, K};
  }
  const at::cuda::OptionalCUDAGuard guard(x.device());
  const int dev = x.get_device();
  raise_pending(dev, op);
  if (M == 0) return;
  at::Tensor ws = nf4_workspace(persona_nf4_linear_workspace_size(probs, n), x);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  check_status(persona_nf4_linear(probs, n, M, ws.data_ptr(), ws.numel(), error_word_device(dev), stream), op);
  after_launch(dev, op, stream);
}
}  // namespace

namespace {
// ---------------------------------------------------- decode helpers ----
void check_half_cuda(const at::Tensor& t, const char* op) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kHalf && t.is_contiguous(), op,
              ": tensors must be contiguous CUDA float16");
}

void add_rmsnorm_op(at::Tensor& h, const c10::optional<at::Tensor>& delta, const at::Tensor& w, at::Tensor& out,
                    double eps) {
  const char* op = "add_rmsnorm";
  check_half_cuda(h, op);
  check_half_cuda(w, op);
  check_half_cuda(out, op);
  const int64_t D = h.size(-1), rows = h.numel() / D;
  TORCH_CHECK(w.numel() == D && out.numel() == h.numel(), op, ": shape mismatch");
  if (delta.has_value()) {
    check_half_cuda(*delta, op);
    TORCH_CHECK(delta->numel() == h.numel(), op, ": delta shape mismatch");
  }
  const at::cuda::OptionalCUDAGuard guard(h.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  check_status(persona_add_rmsnorm(h.data_ptr(), delta.has_value() ? delta->data_ptr() : nullptr, w.data_ptr(),
                                   out.data_ptr(), rows, D, static_cast<float>(eps), stream),
               op);
}

void rope_cache_op(at::Tensor& q, at::Tensor& k, const at::Tensor& v, at::Tensor& k_cache, at::Tensor& v_cache,
                   const at::Tensor& start, int64_t per_seq, double theta) {
  const char* op = "rope_cache";
  for (const at::Tensor* t : std::initializer_list<const at::Tensor*>{&q, &k, &v, &k_cache, &v_cache})
    check_half_cuda(*t, op);
  TORCH_CHECK(q.dim() == 3 && k.dim() == 3 && v.sizes() == k.sizes() && q.size(2) == 128 && k.size(2) == 128 &&
                  q.size(0) == k.size(0),
              op, ": q [rows, Hq, 128], k / v [rows, Hkv, 128]");
  TORCH_CHECK(k_cache.dim() == 4 && v_cache.sizes() == k_cache.sizes() && k_cache.size(1) == k.size(1) &&
                  k_cache.size(3) == 128 && k_cache.size(0) * per_seq == q.size(0),
              op, ": caches [B, Hkv, L, 128] with B * per_seq rows");
  TORCH_CHECK(start.is_cuda() && start.scalar_type() == at::kInt && start.numel() >= 1, op,
              ": start must be a CUDA int32 scalar");
  const at::cuda::OptionalCUDAGuard guard(q.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  check_status(persona_rope_cache(q.data_ptr(), k.data_ptr(), v.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(),
                                  start.data_ptr<int32_t>(), q.size(0), per_seq, q.size(1), k.size(1),
                                  k_cache.size(2), static_cast<float>(theta), stream),
               op);
}

void silu_mul_op(const at::Tensor& g, const at::Tensor& u, at::Tensor& out) {
  const char* op = "silu_mul";
  check_half_cuda(g, op);
  check_half_cuda(u, op);
  check_half_cuda(out, op);
  TORCH_CHECK(g.numel() == u.numel() && out.numel() == g.numel(), op, ": shape mismatch");
  const at::cuda::OptionalCUDAGuard guard(g.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  check_status(persona_silu_mul(g.data_ptr(), u.data_ptr(), out.data_ptr(), g.numel(), stream), op);
}

void rope_decode_attention_op(at::Tensor& q, at::Tensor& k, const at::Tensor& v, at::Tensor& k_cache,
                              at::Tensor& v_cache, const at::Tensor& pos, const at::Tensor& len, at::Tensor& out,
                              double theta, double scale) {
  const char* op = "rope_decode_attention";
  for (const at::Tensor* t : std::initializer_list<const at::Tensor*>{&q, &k, &v, &k_cache, &v_cache, &out})
    check_half_cuda(*t, op);
  TORCH_CHECK(q.dim() == 3 && q.size(2) == 128 && out.sizes() == q.sizes() && k.dim() == 3 && v.sizes() == k.sizes() &&
                  k.size(2) == 128 && k.size(0) == q.size(0),
              op, ": q, out [B, Hq, 128], k / v [B, Hkv, 128]");
  TORCH_CHECK(k_cache.dim() == 4 && v_cache.sizes() == k_cache.sizes() && k_cache.size(0) == q.size(0) &&
                  k_cache.size(1) == k.size(1) && k_cache.size(3) == 128,
              op, ": caches [B, Hkv, L, 128]");
  TORCH_CHECK(pos.is_cuda() && pos.scalar_type() == at::kInt && pos.numel() >= 1 && len.is_cuda() &&
                  len.scalar_type() == at::kInt && len.numel() >= 1,
              op, ": pos and len must be CUDA int32 scalars");
  const at::cuda::OptionalCUDAGuard guard(q.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  check_status(persona_rope_decode_attention(q.data_ptr(), k.data_ptr(), v.data_ptr(), k_cache.data_ptr(),
                                             v_cache.data_ptr(), pos.data_ptr<int32_t>(), len.data_ptr<int32_t>(),
                                             out.data_ptr(), q.size(0), q.size(1), k.size(1), k_cache.size(2),
                                             static_cast<float>(theta), static_cast<float>(scale), stream),
               op);
}

void decode_attention_op(const at::Tensor& q, const at::Tensor& k_cache, const at::Tensor& v_cache,
                         const at::Tensor& len, at::Tensor& out, double scale) {
  const char* op = "decode_attention";
  for (const at::Tensor* t : std::initializer_list<const at::Tensor*>{&q, &k_cache, &v_cache, &out})
    check_half_cuda(*t, op);
  TORCH_CHECK(q.dim() == 3 && q.size(2) == 128 && out.sizes() == q.sizes(), op, ": q, out [B, Hq, 128]");
  TORCH_CHECK(k_cache.dim() == 4 && v_cache.sizes() == k_cache.sizes() && k_cache.size(0) == q.size(0) &&
                  k_cache.size(3) == 128,
              op, ": caches [B, Hkv, L, 128]");
  TORCH_CHECK(len.is_cuda() && len.scalar_type() == at::kInt && len.numel() >= 1, op,
              ": len must be a CUDA int32 scalar");
  const at::cuda::OptionalCUDAGuard guard(q.device());
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  check_status(persona_decode_attention(q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), len.data_ptr<int32_t>(),
                                        out.data_ptr(), q.size(0), q.size(1), k_cache.size(1), k_cache.size(2),
                                        static_cast<float>(scale), stream),
               op);
}
}  // namespace

namespace {
// LoRA term alone at decode sizes (persona_bgmv_lora_delta_multi): deltas[i]
// is fp32 [T, N_i]; the base projection adds it (nf4_linear_add).
void lora_delta_multi_op(at::TensorList xs, at::TensorList a_pools, at::TensorList b_pools, const at::Tensor& slots,
                         at::TensorList deltas) {
  const char* op = "bgmv_lora_delta_multi";
  const int P = static_cast<int>(xs.size());
  TORCH_CHECK(P >= 1 && P <= PERSONA_MAX_PROBLEMS, op, ": 1 to ", PERSONA_MAX_PROBLEMS, " projections");
  TORCH_CHECK(a_pools.size() == xs.size() && b_pools.size() == xs.size() && deltas.size() == xs.size(), op,
              ": xs, a_pools, b_pools and deltas must have the same length");
  TORCH_CHECK(slots.is_cuda() && slots.is_contiguous() && slots.dim() == 1 && slots.scalar_type() == at::kInt, op,
              ": slots must be a contiguous int32 CUDA vector");
  const int64_t T = slots.size(0);
  const int64_t S = a_pools[0].size(0), R = a_pools[0].size(1);
  const int dt = dtype_code(xs[0], op);
  persona_bgmv_problem probs[PERSONA_MAX_PROBLEMS];
  float* dptr[PERSONA_MAX_PROBLEMS];
  int64_t dld[PERSONA_MAX_PROBLEMS];
  for (int p = 0; p < P; ++p) {
    const at::Tensor &x = xs[p], &a = a_pools[p], &b = b_pools[p], &d = deltas[p];
    TORCH_CHECK(x.is_cuda() && a.is_cuda() && b.is_cuda() && d.is_cuda(), op, ": all tensors must be CUDA");
    TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && d.dim() == 2 && d.stride(1) == 1, op,
                ": tensors must be contiguous");
    TORCH_CHECK(d.scalar_type() == at::kFloat, op, ": deltas must be float32");
    check_pool_a(a, op);
    check_pool_b(b, op);
    TORCH_CHECK(x.size(0) == T && d.size(0) == T, op, ": x / delta rows must match slots");
    TORCH_CHECK(a.size(0) == S && a.size(1) == R && a.size(2) == x.size(1), op, ": a_pool shape mismatch");
    TORCH_CHECK(b.size(0) == S && b.size(2) == R && b.size(1) == d.size(1), op, ": b_pool shape mismatch");
    TORCH_CHECK(x.scalar_type() == xs[0].scalar_type() && a.scalar_type() == x.scalar_type() &&
                    b.scalar_type() == x.scalar_type(),
                op, ": dtype mismatch");
    probs[p] = persona_bgmv_problem{x.data_ptr(), row_stride(x), a.data_ptr(), a.stride(0), a.stride(1),
                                    b.data_ptr(), b.stride(0),   nullptr,      0,            x.size(1),
                                    d.size(1)};
    dptr[p] = d.data_ptr<float>();
    dld[p] = row_stride(d);
  }
  const at::cuda::OptionalCUDAGuard guard(slots.device());
  const int dev = slots.get_device();
  raise_pending(dev, op);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  check_status(persona_bgmv_lora_delta_multi(probs, P, dptr, dld, slots.data_ptr<int32_t>(), T, R, S, dt,
                                             error_word_device(dev), stream),
               op);
  after_launch(dev, op, stream);
}

void nf4_linear_add_op(const at::Tensor& x, at::TensorList packed, at::TensorList offsets, at::TensorList addends,
                       at::TensorList ys) {
  const char* op = "nf4_linear_add";
  const int n = static_cast<int>(packed.size());
  TORCH_CHECK(n >= 1 && n <= PERSONA_NF4_MAX_PROBLEMS, op, ": 1 to ", PERSONA_NF4_MAX_PROBLEMS, " weights");
  TORCH_CHECK(static_cast<int>(offsets.size()) == n && static_cast<int>(ys.size()) == n &&
                  static_cast<int>(addends.size()) == n,
              op, ": one offset, one addend and one y per weight");
  TORCH_CHECK(x.is_cuda() && x.dim() == 2 && x.stride(1) == 1 && x.scalar_type() == at::kHalf, op,
              ": x must be a CUDA float16 [M, K] matrix with unit inner stride");
  const int64_t M = x.size(0), K = x.size(1);
  persona_nf4_problem probs[PERSONA_NF4_MAX_PROBLEMS];
  const float* add[PERSONA_NF4_MAX_PROBLEMS];
  int64_t ldadd[PERSONA_NF4_MAX_PROBLEMS];
  for (int i = 0; i < n; ++i) {
    const at::Tensor& y = ys[i];
    const at::Tensor& d = addends[i];
    TORCH_CHECK(y.is_cuda() && y.dim() == 2 && y.stride(1) == 1 && y.scalar_type() == at::kHalf && y.size(0) == M,
                op, ": y must be a CUDA float16 [M, N] matrix with unit inner stride");
    const int64_t N = y.size(1);
    TORCH_CHECK(d.is_cuda() && d.dim() == 2 && d.stride(1) == 1 && d.scalar_type() == at::kFloat &&
                    d.size(0) == M && d.size(1) == N,
                op, ": addend must be a CUDA float32 [M, N] matrix with unit inner stride");
    check_nf4_weight(packed[i], offsets[i], N, K, op);
    probs[i] = persona_nf4_problem{packed[i].data_ptr(), offsets[i].data_ptr<float>(), x.data_ptr(), row_stride(x),
                                   y.data_ptr(), row_stride(y), N, K};
    add[i] = d.data_ptr<float>();
    ldadd[i] = row_stride(d);
  }
  const at::cuda::OptionalCUDAGuard guard(x.device());
  const int dev = x.get_device();
  raise_pending(dev, op);
  if (M == 0) return;
  at::Tensor ws = nf4_workspace(persona_nf4_linear_workspace_size(probs, n), x);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  check_status(persona_nf4_linear_add(probs, n, add, ldadd, M, ws.data_ptr(), ws.numel(), error_word_device(dev),
                                      stream),
               op);
  after_launch(dev, op, stream);
}
}  // namespace

TORCH_LIBRARY(persona, m) {
  // Reference schemas, unchanged (csrc/bindings.cpp:19-23).
  m.def("bgmv_shrink(Tensor x, Tensor a_pool, Tensor slots, Tensor(a!) v) -> ()");
  m.def("bgmv_expand(Tensor v, Tensor b_pool, Tensor slots, Tensor(a!) y) -> ()");
  m.def("gemv_fp16(Tensor x, Tensor W, Tensor(a!) y) -> ()");
  // New in this build.
  m.def("bgmv_plan(Tensor slots, int S) -> Tensor");
  m.def("bgmv_shrink_with_plan(Tensor x, Tensor a_pool, Tensor slots, Tensor plan, Tensor(a!) v) -> ()");
  m.def("bgmv_expand_with_plan(Tensor v, Tensor b_pool, Tensor slots, Tensor plan, Tensor(a!) y) -> ()");
  m.def("bgmv_fused(Tensor x, Tensor a_pool, Tensor b_pool, Tensor slots, Tensor(a!) y) -> ()");
  m.def("bgmv_fused_with_plan(Tensor x, Tensor a_pool, Tensor b_pool, Tensor slots, Tensor plan, "
        "Tensor(a!) y) -> ()");
  m.def("bgmv_fused_multi(Tensor[] xs, Tensor[] a_pools, Tensor[] b_pools, Tensor slots, Tensor(a!)[] ys, "
        "Tensor? plan=None) -> ()");
  m.def("sgmv_shrink(Tensor x, Tensor a_pool, Tensor seg_indptr, Tensor seg_slots, Tensor(a!) v) -> ()");
  m.def("sgmv_expand(Tensor v, Tensor b_pool, Tensor seg_indptr, Tensor seg_slots, Tensor(a!) y) -> ()");
  m.def("sgmv_fused(Tensor x, Tensor a_pool, Tensor b_pool, Tensor seg_indptr, Tensor seg_slots, "
        "Tensor(a!) y) -> ()");
  m.def("nf4_quantize(Tensor w) -> (Tensor, Tensor)");
  m.def("nf4_dequantize(Tensor packed, Tensor offset, int N, int K) -> Tensor");
  m.def("nf4_linear(Tensor x, Tensor[] packed, Tensor[] offsets, Tensor(a!)[] ys) -> ()");
  m.def("nf4_linear_add(Tensor x, Tensor[] packed, Tensor[] offsets, Tensor[] addends, Tensor(a!)[] ys) -> ()");
  m.def("bgmv_lora_delta_multi(Tensor[] xs, Tensor[] a_pools, Tensor[] b_pools, Tensor slots, "
        "Tensor(a!)[] deltas) -> ()");
  m.def("add_rmsnorm(Tensor(a!) h, Tensor? delta, Tensor w, Tensor(b!) out, float eps) -> ()");
  m.def("rope_cache(Tensor(a!) q, Tensor(b!) k, Tensor v, Tensor(c!) k_cache, Tensor(d!) v_cache, Tensor start, "
        "int per_seq, float theta) -> ()");
  m.def("silu_mul(Tensor g, Tensor u, Tensor(a!) out) -> ()");
  m.def("decode_attention(Tensor q, Tensor k_cache, Tensor v_cache, Tensor len, Tensor(a!) out, float scale) -> ()");
  m.def("rope_decode_attention(Tensor(a!) q, Tensor(b!) k, Tensor v, Tensor(c!) k_cache, Tensor(d!) v_cache, "
        "Tensor pos, Tensor len, Tensor(e!) out, float theta, float scale) -> ()");
}

TORCH_LIBRARY_IMPL(persona, CUDA, m) {
  m.impl("nf4_quantize", &nf4_quantize_op);
  m.impl("nf4_dequantize", &nf4_dequantize_op);
  m.impl("nf4_linear", &nf4_linear_op);
  m.impl("nf4_linear_add", &nf4_linear_add_op);
  m.impl("bgmv_lora_delta_multi", &lora_delta_multi_op);
  m.impl("add_rmsnorm", &add_rmsnorm_op);
  m.impl("rope_cache", &rope_cache_op);
  m.impl("silu_mul", &silu_mul_op);
  m.impl("decode_attention", &decode_attention_op);
  m.impl("rope_decode_attention", &rope_decode_attention_op);
  m.impl("bgmv_shrink", &bgmv_shrink_cuda);
  m.impl("bgmv_expand", &bgmv_expand_cuda);
  m.impl("gemv_fp16", &persona::gemv_fp16_cuda);
  m.impl("bgmv_plan", &plan_impl);
  m.impl("bgmv_shrink_with_plan", &shrink_with_plan);
  m.impl("bgmv_expand_with_plan", &expand_with_plan);
  m.impl("bgmv_fused", &fused_noplan);
  m.impl("bgmv_fused_with_plan", &fused_with_plan);
  m.impl("bgmv_fused_multi", &fused_multi_impl);
  m.impl("sgmv_shrink", &sgmv_shrink_op);
  m.impl("sgmv_expand", &sgmv_expand_op);
  m.impl("sgmv_fused", &sgmv_fused_op);
}

namespace {
// Tensor-parallel segmented fused op (persona_sgmv_fused_tp); `peers` are the
// other ranks' y buffers mapped into this process, as integers.
void sgmv_fused_tp_op(const at::Tensor& x, const at::Tensor& a_pool, const at::Tensor& b_pool,
                      const at::Tensor& indptr, const at::Tensor& seg_slots, at::Tensor& y,
                      const std::vector<int64_t>& peers, int64_t n0, int64_t n1) {
  const char* op = "sgmv_fused_tp";
  check_segments(indptr, seg_slots, op);
  TORCH_CHECK(x.is_cuda() && a_pool.is_cuda() && b_pool.is_cuda() && y.is_cuda(), op, ": all tensors must be CUDA");
  TORCH_CHECK(x.dim() == 2 && x.stride(1) == 1 && y.dim() == 2 && y.stride(1) == 1, op,
              ": tensors must be contiguous");
  check_pool_a(a_pool, op);
  check_pool_b(b_pool, op);
  const int64_t T = x.size(0), K = x.size(1), S = a_pool.size(0), R = a_pool.size(1), N = b_pool.size(1);
  TORCH_CHECK(a_pool.size(2) == K && b_pool.size(0) == S && b_pool.size(2) == R, op, ": pool shape mismatch");
  TORCH_CHECK(y.size(0) == T && y.size(1) == N, op, ": y shape mismatch");
  TORCH_CHECK(peers.size() <= PERSONA_MAX_TP_PEERS, op, ": too many peers");
  const int dt = dtype_code(x, op);
  TORCH_CHECK(a_pool.scalar_type() == x.scalar_type() && b_pool.scalar_type() == x.scalar_type() &&
                  y.scalar_type() == x.scalar_type(),
              op, ": dtype mismatch");
  const at::cuda::OptionalCUDAGuard guard(x.device());
  const int dev = x.get_device();
  raise_pending(dev, op);
  if (T == 0) return;
  void* pp[PERSONA_MAX_TP_PEERS];
  for (size_t i = 0; i < peers.size(); ++i) pp[i] = reinterpret_cast<void*>(peers[i]);
  at::Tensor ws = sgmv_workspace(T, x);
  cudaStream_t stream = at::cuda::getCurrentCUDAStream();
  check_status(persona_sgmv_fused_tp(x.data_ptr(), row_stride(x), a_pool.data_ptr(), a_pool.stride(0),
                                     a_pool.stride(1), b_pool.data_ptr(), b_pool.stride(0),
                                     indptr.data_ptr<int32_t>(), seg_slots.data_ptr<int32_t>(), seg_slots.size(0),
                                     y.data_ptr(), row_stride(y), pp, static_cast<int>(peers.size()), n0, n1, T, K,
                                     N, R, S, dt, ws.data_ptr(), ws.numel(), error_word_device(dev), stream),
               op);
  after_launch(dev, op, stream);
}
}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("sgmv_fused_tp", &sgmv_fused_tp_op,
        "Tensor-parallel segmented fused LoRA: columns [n0, n1) of y, every finished tile also stored into the "
        "peers' y (pointers from ipc_import).");
  m.def(
      "ipc_export",
      [](const at::Tensor& t) {
        TORCH_CHECK(t.is_cuda(), "ipc_export: CUDA tensor expected");
        const at::cuda::OptionalCUDAGuard guard(t.device());
        char handle[64];
        size_t offset = 0;
        check_status(persona_ipc_export(t.data_ptr(), handle, &offset), "ipc_export");
        return pybind11::make_tuple(pybind11::bytes(handle, sizeof(handle)), static_cast<int64_t>(offset));
      },
      "64-byte CUDA IPC handle of the allocation holding `t`, and t's offset in it.");
  m.def(
      "ipc_import",
      [](const std::string& handle, int64_t offset, int device) {
        TORCH_CHECK(handle.size() == 64, "ipc_import: 64-byte handle expected");
        const at::cuda::OptionalCUDAGuard guard(at::Device(at::kCUDA, device));
        void* ptr = nullptr;
        void* base = nullptr;
        check_status(persona_ipc_import(handle.data(), static_cast<size_t>(offset), &ptr, &base), "ipc_import");
        return pybind11::make_tuple(reinterpret_cast<int64_t>(ptr), reinterpret_cast<int64_t>(base));
      },
      "Map another process's buffer: returns (pointer, mapping base).");
  m.def(
      "ipc_close", [](int64_t base, int device) {
        const at::cuda::OptionalCUDAGuard guard(at::Device(at::kCUDA, device));
        check_status(persona_ipc_close(reinterpret_cast<void*>(base)), "ipc_close");
      },
      "Unmap a buffer mapped by ipc_import (its mapping base).");
  m.def("noop", []() { return 0; });
  m.def("abi_version", []() { return persona_abi_version(); });
  m.def("workspace_size", [](int64_t T) { return persona_bgmv_workspace_size(T); });
  m.def(
      "take_device_error",
      [](int device) {
        volatile int32_t* h = error_word_host(device);
        const int bits = *h;
        *h = 0;
        return bits;
      },
      "Read and clear the device error word of `device` (no synchronisation).");
}
