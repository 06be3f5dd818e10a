// Shared device helpers and host launch utilities of the B200 sparse-pooling library.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "granule_b200.h"

namespace gl {

constexpr unsigned kFullMask = 0xffffffffu;

// Per-neuron activation and its derivative (sparse_pooling/config.py:33, the
// reference's Triton _act/_dact, kernels/triton_fused.py:28-47).  GELU is the
// exact erf form, as in the reference.
template <int ACT>
__device__ __forceinline__ float act_f(float z) {
  if constexpr (ACT == GL_ACT_IDENTITY) {
    return z;
  } else if constexpr (ACT == GL_ACT_RELU) {
    return fmaxf(z, 0.f);
  } else {
    return 0.5f * z * (1.f + erff(z * 0.7071067811865476f));
  }
}

template <int ACT>
__device__ __forceinline__ float dact_f(float z) {
  if constexpr (ACT == GL_ACT_IDENTITY) {
    return 1.f;
  } else if constexpr (ACT == GL_ACT_RELU) {
    return z > 0.f ? 1.f : 0.f;
  } else {
    const float cdf = 0.5f * (1.f + erff(z * 0.7071067811865476f));
    const float pdf = 0.3989422804014327f * expf(-0.5f * z * z);
    return cdf + z * pdf;
  }
}

// Eight int16 indices of one neuron record, loaded as one 16-byte vector and
// widened; every index is clamped to [0, dmax] so that a corrupt record can
// never address outside the staged input tile.
struct Rec8 {
  int i[8];
};

__device__ __forceinline__ Rec8 load_rec8(const int16_t* __restrict__ p, int dmax) {
  const int4 r = __ldg(reinterpret_cast<const int4*>(p));
  const unsigned u[4] = {(unsigned)r.x, (unsigned)r.y, (unsigned)r.z, (unsigned)r.w};
  Rec8 o;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    o.i[2 * j] = min((int)(u[j] & 0xffffu), dmax);
    o.i[2 * j + 1] = min((int)(u[j] >> 16), dmax);
  }
  return o;
}

struct W8 {
  float w[8];
};

__device__ __forceinline__ W8 load_w8(const float* __restrict__ p) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(p));
  const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
  W8 o;
  o.w[0] = a.x; o.w[1] = a.y; o.w[2] = a.z; o.w[3] = a.w;
  o.w[4] = b.x; o.w[5] = b.y; o.w[6] = b.z; o.w[7] = b.w;
  return o;
}

// Vector reductions into global memory (sm_90+ PTX vector red).
__device__ __forceinline__ void red_add(float* p, float a) {
  asm volatile("red.global.add.f32 [%0], %1;" ::"l"(p), "f"(a) : "memory");
}
__device__ __forceinline__ void red_add2(float* p, float a, float b) {
  asm volatile("red.global.add.v2.f32 [%0], {%1, %2};" ::"l"(p), "f"(a), "f"(b) : "memory");
}
__device__ __forceinline__ void red_add4(float* p, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}

// Stage x[t0 .. t0+T-1, 0 .. D-1] (token-major, row stride ldx) into the
// feature-major tile xs[d * T + t]; tokens >= B read as 0.  One thread per
// feature: T coalesced 128-byte row loads per warp, then one or two vector
// stores of the feature's T values.
template <int T, int NTHREADS>
__device__ __forceinline__ void stage_tile(float* __restrict__ xs, const float* __restrict__ x, int t0, int B,
                                           int D, int64_t ldx) {
  for (int d = threadIdx.x; d < D; d += NTHREADS) {
    float v[T];
#pragma unroll
    for (int t = 0; t < T; ++t) v[t] = (t0 + t < B) ? __ldg(x + (int64_t)(t0 + t) * ldx + d) : 0.f;
    float* row = xs + (int64_t)d * T;
    if constexpr (T >= 4) {
#pragma unroll
      for (int q = 0; q < T / 4; ++q)
        reinterpret_cast<float4*>(row)[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    } else if constexpr (T == 2) {
      reinterpret_cast<float2*>(row)[0] = make_float2(v[0], v[1]);
    } else {
      row[0] = v[0];
    }
  }
}

// Element offsets of the fragment-packed layout (layout.py:146-179): with NT = C/8,
// Q = NB*NT/4, UB = max(1, 4/NT), fragment f = j*NT + c/8, quad = f/4, fi = f%4, n = c%8:
//   w (g, j, c, k = 2 kh + e) at [g, quad, n*4 + kh, fi, e];  b (g, j, c = 8*(f%NT) + 2 l4 + e) at
//   [g, quad, l4, fi, e];  idx (g, j, k) at [g, j / UB, k, j % UB].
struct MbPacked {
  int64_t Q;
  int NT, UB;
};

__host__ __device__ __forceinline__ MbPacked mb_packed(int C, int64_t NB) {
  MbPacked m;
  m.NT = C >> 3;
  m.Q = NB * m.NT / 4;
  m.UB = m.NT >= 4 ? 1 : 4 / m.NT;
  return m;
}

// Offset of w (g, j, c, k = 2 kh) in the packed layout (the pair k, k+1 is contiguous).
__device__ __forceinline__ int64_t mb_packed_w(const MbPacked& m, int64_t g, int j, int c, int kh) {
  const int f = j * m.NT + (c >> 3);
  return ((((g * m.Q + (f >> 2)) * 32) + (c & 7) * 4 + kh) * 4 + (f & 3)) * 2;
}

// Offset of b (g, j, c) for even c (the pair c, c+1 is contiguous).
__device__ __forceinline__ int64_t mb_packed_b(const MbPacked& m, int64_t g, int j, int c) {
  const int f = j * m.NT + (c >> 3);
  return (((g * m.Q + (f >> 2)) * 4 + ((c & 7) >> 1)) * 4 + (f & 3)) * 2;
}

// Per-group input feature maps (gl_group_feature_map): when given, a block processes one group
// and stages only the group's features, fmap[g][0 .. nfeat[g]-1], reading the records' inputs as
// positions in that list (lidx, same shape as the indices).
struct LocalMap {
  const int16_t* lidx;
  const int16_t* fmap;
  const int32_t* nfeat;
  int fcap;
};

// Stage x[t0 .. t0+T-1, cols[j]] into xs[j * T + t] for j < ncols (tokens >= B read as 0).
template <int T, int NTHREADS>
__device__ __forceinline__ void stage_cols(float* __restrict__ xs, const float* __restrict__ x, int t0, int B,
                                           const int16_t* __restrict__ cols, int ncols, int64_t ldx, int D) {
  for (int j = threadIdx.x; j < ncols; j += NTHREADS) {
    const int d = min((int)(uint16_t)__ldg(cols + j), D - 1);
    float v[T];
#pragma unroll
    for (int t = 0; t < T; ++t) v[t] = (t0 + t < B) ? __ldg(x + (int64_t)(t0 + t) * ldx + d) : 0.f;
    float* row = xs + (int64_t)j * T;
    if constexpr (T >= 4) {
#pragma unroll
      for (int q = 0; q < T / 4; ++q)
        reinterpret_cast<float4*>(row)[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    } else {
#pragma unroll
      for (int t = 0; t < T; ++t) row[t] = v[t];
    }
  }
}

}  // namespace gl

// ---- host-side helpers (defined in abi.cu) ----
namespace gl {
int set_cuda_error(cudaError_t e);                      // records e, returns GL_ERR_LAUNCH
void count_launches(int n);                             // adds n to gl_launch_count()
int device_smem_optin(int* bytes);                      // max dynamic smem per block, current device
int device_sm_count(int* sms);
int ensure_dynamic_smem(const void* func, size_t bytes);  // raises the kernel's opt-in once per device
}  // namespace gl
