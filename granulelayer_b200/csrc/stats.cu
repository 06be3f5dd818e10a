// Per-group bounds used by the fixed-point backward (bwd.cu): the largest
// |weight| of each group's valid slots, and the largest number of the group's
// valid (slot, k) records that share one input feature.  Neither has a
// counterpart in the reference; they exist because the B200 backward
// accumulates dX in int32 shared memory and must choose an overflow-free scale.
#include "common.cuh"

namespace gl {

constexpr int kStatThreads = 512;

__device__ __forceinline__ float block_max(float m, float* red) {
#pragma unroll
  for (int off = 16; off; off >>= 1) m = fmaxf(m, __shfl_xor_sync(kFullMask, m, off));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int i = 1; i < (int)(blockDim.x >> 5); ++i) m = fmaxf(m, red[i]);
  }
  return m;
}

__global__ void __launch_bounds__(kStatThreads) group_absmax_kernel(const float* __restrict__ w,
                                                                    const int32_t* __restrict__ counts, int64_t NB,
                                                                    int64_t g0, float* __restrict__ out) {
  __shared__ float red[kStatThreads / 32];
  const int64_t g = g0 + blockIdx.x;
  const int64_t slots = NB * 8;
  const int64_t ng = min((int64_t)counts[g], slots);
  const float4* p = reinterpret_cast<const float4*>(w + g * slots * 8);
  float m = 0.f;
  for (int64_t i = threadIdx.x; i < ng * 2; i += kStatThreads) {  // 8 floats per slot = 2 float4
    const float4 v = __ldg(p + i);
    m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
  }
  m = block_max(m, red);
  if (threadIdx.x == 0) out[blockIdx.x] = m;
}

__global__ void __launch_bounds__(kStatThreads) group_index_maxcount_kernel(const int16_t* __restrict__ idx,
                                                                            const int32_t* __restrict__ counts,
                                                                            int D, int64_t NB, int64_t g0,
                                                                            int32_t* __restrict__ out) {
  extern __shared__ int hist[];
  __shared__ float red[kStatThreads / 32];
  for (int d = threadIdx.x; d < D; d += kStatThreads) hist[d] = 0;
  __syncthreads();
  const int64_t g = g0 + blockIdx.x;
  const int64_t slots = NB * 8;
  const int64_t ng = min((int64_t)counts[g], slots);
  const int16_t* p = idx + g * slots * 8;
  for (int64_t i = threadIdx.x; i < ng * 8; i += kStatThreads) {
    const int v = min((int)(uint16_t)__ldg(p + i), D - 1);
    atomicAdd(&hist[v], 1);
  }
  __syncthreads();
  int m = 0;
  for (int d = threadIdx.x; d < D; d += kStatThreads) m = max(m, hist[d]);
  const float mf = block_max((float)m, red);
  if (threadIdx.x == 0) out[blockIdx.x] = (int32_t)mf;
}

}  // namespace gl

using namespace gl;

extern "C" int gl_group_absmax_f32(const float* w, const int32_t* counts, int64_t NB, int64_t g0, int64_t g1,
                                   float* out, void* stream) {
  if (NB < 1 || g0 < 0 || g1 < g0) return GL_ERR_SHAPE;
  if (g1 == g0) return GL_OK;
  if (!w || !counts || !out) return GL_ERR_NULL;
  if ((uintptr_t)w & 15) return GL_ERR_ALIGN;
  if (g1 - g0 > 2147483647LL) return GL_ERR_SHAPE;
  group_absmax_kernel<<<(unsigned)(g1 - g0), kStatThreads, 0, (cudaStream_t)stream>>>(w, counts, NB, g0, out);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e);
  count_launches(1);
  return GL_OK;
}

extern "C" int gl_group_index_maxcount(const int16_t* idx, const int32_t* counts, int64_t D, int64_t NB,
                                       int64_t g0, int64_t g1, int32_t* out, void* stream) {
  if (D < 1 || D > 32767 || NB < 1 || g0 < 0 || g1 < g0) return GL_ERR_SHAPE;
  if (g1 == g0) return GL_OK;
  if (!idx || !counts || !out) return GL_ERR_NULL;
  if (g1 - g0 > 2147483647LL) return GL_ERR_SHAPE;
  const size_t smem = (size_t)D * sizeof(int);
  int rc = ensure_dynamic_smem((const void*)group_index_maxcount_kernel, smem);
  if (rc) return rc;
  group_index_maxcount_kernel<<<(unsigned)(g1 - g0), kStatThreads, smem, (cudaStream_t)stream>>>(
      idx, counts, (int)D, NB, g0, out);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e);
  count_launches(1);
  return GL_OK;
}
