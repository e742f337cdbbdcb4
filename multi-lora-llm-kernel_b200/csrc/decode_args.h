// Launchers of the small fused kernels of the end-to-end decode loop.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace persona {

cudaError_t launch_add_rmsnorm(void* h, const void* delta, const void* w, void* out, int rows, int D, float eps,
                               cudaStream_t st);
cudaError_t launch_rope_cache(void* q, void* k, const void* v, void* kc, void* vc, const int* start, int rows,
                              int per_seq, int Hq, int Hkv, int L, float log2_theta, cudaStream_t st);
cudaError_t launch_silu_mul(const void* g, const void* u, void* out, int64_t n, cudaStream_t st);
cudaError_t launch_decode_attention(const void* q, const void* kc, const void* vc, const int* len, void* out, int B,
                                    int Hq, int Hkv, int L, float scale, cudaStream_t st);
cudaError_t launch_rope_decode_attention(void* q, void* k, const void* v, void* kc, void* vc, const int* pos,
                                         const int* len, void* out, int B, int Hq, int Hkv, int L, float log2_theta,
                                         float scale, cudaStream_t st);

}  // namespace persona
