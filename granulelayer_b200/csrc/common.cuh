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

// Bound of |act'(z)| (the fixed-point dX scales divide by it).
template <int ACT>
__host__ __device__ constexpr float dact_bound() {
  return ACT == GL_ACT_GELU ? 1.13f : 1.f;  // max |gelu'(z)| = 1.1289 at z ~ 1.41
}

// ---------------------------------------------------------------------------
// Pooling states (the reference's per-(token, group) states, kernels/triton_fused.py:121-225, and
// their merge / finalisation, kernels/ops.py:182-239).  Forward kinds:
//   PK_ADD  mean / sum: s0 = sum a
//   PK_MAX  max: s0 = max a and the winning slot
//   PK_LSE  LogMeanExp / softmax-weighted, base-2 log-sum-exp of u = a * param:
//           s0 = m = max u, s1 = sum 2^(u - m), s2 = sum a 2^(u - m) (softmax only)
//   PK_POW  power mean of a = relu(z) >= 0: s0 = m = max a, s1 = sum (a / m)^p, s2 = 1 / m
//   PK_TOPK top-K mean: per-warp lists of the best keys (below); PK_TOPK64 for k = 64
// A lane folds its values in one at a time and rescales its sums only when a new maximum
// arrives; lanes and warps then merge their states.
enum { PK_ADD = 0, PK_MAX = 1, PK_LSE = 2, PK_POW = 3, PK_TOPK = 4, PK_TOPK64 = 5 };

inline int pool_kind(int pool, int k = 0) {
  return pool == GL_POOL_MAX ? PK_MAX
       : pool == GL_POOL_TOPK ? (k > 32 ? PK_TOPK64 : PK_TOPK)
       : (pool == GL_POOL_LME || pool == GL_POOL_SOFTMAX) ? PK_LSE
       : pool == GL_POOL_POWER ? PK_POW : PK_ADD;
}

// Integer exponent code of a power-mean exponent: p itself for p in {1, 2, 4, 8} (the reference's
// P_INT, kernels/ops.py:68-71), else -1 (the general 2^(p log2 r) form).
__host__ __device__ __forceinline__ int pow_code(float p) {
  return (p == 1.f || p == 2.f || p == 4.f || p == 8.f) ? (int)p : -1;
}

// r^e for r >= 0, by products for the exponents the power mean uses (ie = e in {0, 1, 2, 3, 4, 7, 8},
// in the reference's multiplication order) and 2^(e log2 r) otherwise (0^e = 0 for e > 0).
__device__ __forceinline__ float powr(float r, int ie, float e) {
  switch (ie) {
    case 0: return 1.f;
    case 1: return r;
    case 2: return r * r;
    case 3: return r * r * r;
    case 4: { const float r2 = r * r; return r2 * r2; }
    case 7: { const float r2 = r * r, r4 = r2 * r2; return r4 * r2 * r; }
    case 8: { const float r2 = r * r, r4 = r2 * r2; return r4 * r4; }
    default: return exp2f(e * log2f(r));
  }
}

struct PoolParam {
  float param;  // LME: log2(e) / tau; softmax: log2(e) * beta; power: p
  int ip;       // power: pow_code(p)
  bool want_t;  // softmax: track sum a 2^(u - m)
  int k;        // top-K: slots kept
};

// A valid top-K count: a power of two in [1, 64] (config.py:117-119).
inline bool topk_k_ok(int k) { return k >= 1 && k <= 64 && (k & (k - 1)) == 0; }

__device__ __forceinline__ void lse_push(float& m, float& s, float& t, float u, float a, bool want_t) {
  const float d = u - m;
  const float e = exp2f(-fabsf(d));  // 2^(m - u) for a new maximum, else 2^(u - m)
  const bool up = d > 0.f;
  s = up ? fmaf(s, e, 1.f) : s + e;
  if (want_t) t = up ? fmaf(t, e, a) : fmaf(a, e, t);
  m = up ? u : m;
}

__device__ __forceinline__ void lse_merge(float& m, float& s, float& t, float m2, float s2, float t2) {
  const float M = fmaxf(m, m2);
  const float e1 = M == -INFINITY ? 0.f : exp2f(m - M);
  const float e2 = M == -INFINITY ? 0.f : exp2f(m2 - M);
  s = fmaf(s, e1, s2 * e2);
  t = fmaf(t, e1, t2 * e2);
  m = M;
}

__device__ __forceinline__ void pow_push(float& m, float& s, float& inv, float a, const PoolParam& pp) {
  if (a > m) {
    const float ia = 1.f / a;
    s = fmaf(s, powr(m * ia, pp.ip, pp.param), 1.f);
    m = a;
    inv = ia;
  } else {
    s += powr(a * inv, pp.ip, pp.param);
  }
}

__device__ __forceinline__ void pow_merge(float& m, float& s, float m2, float s2, const PoolParam& pp) {
  const float M = fmaxf(m, m2);
  if (M > 0.f) {
    const float iM = 1.f / M;
    s = fmaf(s, powr(m * iM, pp.ip, pp.param), s2 * powr(m2 * iM, pp.ip, pp.param));
  } else {
    s = 0.f;
  }
  m = M;
}

// pre (and the log2-normaliser L2 of the LSE kinds) of a merged state over n valid slots
// (kernels/ops.py:200-217).
__device__ __forceinline__ float pool_finalize(int pool, float s0, float s1, float s2, int n, float param,
                                               float* l2) {
  if (pool == GL_POOL_LME || pool == GL_POOL_SOFTMAX) {
    const float L2 = s0 + log2f(s1);
    *l2 = L2;
    return pool == GL_POOL_LME ? (L2 - log2f((float)n)) / param : s2 / s1;
  }
  // power mean
  return s0 > 0.f ? s0 * powf(s1 / (float)n, 1.f / param) : 0.f;
}

// dz = c1 * h * act'(z) of the pools with a dense backward (kernels/triton_fused.py:365-399).
template <int ACT>
__device__ __forceinline__ float pool_dz(int pool, float z, float c1, float c2, float c3, float param, int ipm1) {
  if (pool == GL_POOL_MEAN || pool == GL_POOL_SUM) return c1 * dact_f<ACT>(z);
  if (pool == GL_POOL_POWER) {
    const float q = fmaxf(z, 0.f) * c2;
    return z > 0.f ? c1 * powr(q, ipm1, param - 1.f) : 0.f;
  }
  const float a = act_f<ACT>(z);
  const float pw = exp2f(fmaf(a, param, -c2));
  if (pool == GL_POOL_LME) return c1 * pw * dact_f<ACT>(z);
  const float beta = param * 0.6931471805599453f;
  return c1 * pw * fmaf(beta, a - c3, 1.f) * dact_f<ACT>(z);
}

// ---------------------------------------------------------------------------
// Top-K pooling (kernels/triton_fused.py:51-55, 141-173): candidates are ranked by 64-bit keys, the
// order-preserving bits of z above the complemented slot, so a larger key is a larger z and, on
// ties, the smaller slot.  A warp keeps one sorted (descending) list per token: position p at lane
// p % 32 of word p / 32 (KW = 1 word for k <= 32, 2 for k = 64), LLONG_MIN past the entries.
__device__ __forceinline__ long long topk_key(float z, int slot) {
  const int zb = __float_as_int(z);
  const unsigned s = (unsigned)(zb >= 0 ? zb : zb ^ 0x7FFFFFFF);
  return (long long)(((unsigned long long)s << 32) | (unsigned long long)(0xFFFFFFFFu - (unsigned)slot));
}

__device__ __forceinline__ float topk_value(long long key) {
  const int hi = (int)(key >> 32);
  return __int_as_float(hi >= 0 ? hi : hi ^ 0x7FFFFFFF);
}

__device__ __forceinline__ int topk_slot(long long key) {
  return (int)(0xFFFFFFFFu - (unsigned)(key & 0xFFFFFFFFll));
}

// The key at position k - 1 (the entry a candidate must beat).
template <int KW>
__device__ __forceinline__ long long topk_last(const long long (&w)[KW], int k) {
  return KW == 1 ? __shfl_sync(kFullMask, w[0], k - 1) : __shfl_sync(kFullMask, w[KW - 1], 31);
}

// Insert the warp-uniform key c (keys in a list are distinct: their slots differ).
template <int KW>
__device__ __forceinline__ void topk_insert(long long (&w)[KW], long long c, int k, int lane) {
  const unsigned live = k >= 32 ? kFullMask : (1u << k) - 1u;
  int pos = __popc(__ballot_sync(kFullMask, w[0] > c) & live);
  if constexpr (KW == 2) pos += __popc(__ballot_sync(kFullMask, w[1] > c));
  if (pos >= k) return;
  const long long up0 = __shfl_up_sync(kFullMask, w[0], 1);
  if constexpr (KW == 1) {
    w[0] = lane > pos ? up0 : (lane == pos ? c : w[0]);
  } else {
    const long long carry = __shfl_sync(kFullMask, w[0], 31);
    const long long up1 = __shfl_up_sync(kFullMask, w[1], 1);
    if (pos < 32) {
      w[1] = lane == 0 ? carry : up1;
      w[0] = lane > pos ? up0 : (lane == pos ? c : w[0]);
    } else {
      const int p1 = pos - 32;
      w[1] = lane > p1 ? up1 : (lane == p1 ? c : w[1]);
    }
  }
}

// Offer each lane's candidate key (where `has`) to the warp's list; thr tracks topk_last.
template <int KW>
__device__ __forceinline__ void topk_offer(long long (&w)[KW], long long& thr, bool has, long long key, int k,
                                           int lane) {
  unsigned m = __ballot_sync(kFullMask, has && key > thr);
  while (m) {
    const int src = __ffs(m) - 1;
    topk_insert<KW>(w, __shfl_sync(kFullMask, key, src), k, lane);
    thr = topk_last<KW>(w, k);
    m &= ~(1u << src);
    m &= __ballot_sync(kFullMask, has && key > thr);
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

// bf16 storage (the reference's default parameter dtype): a bf16 value is the upper half of the
// fp32 with the same bits, so widening is exact.  `bf` is uniform across the launch.
__device__ __forceinline__ float bf16_lo(unsigned u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf16_hi(unsigned u) { return __uint_as_float(u & 0xFFFF0000u); }

// Weights of neuron f (8 consecutive values) in fp32 or bf16 storage.
__device__ __forceinline__ W8 load_w8_any(const float* __restrict__ w, int64_t f, bool bf) {
  if (!bf) return load_w8(w + f * 8);
  const uint4 u = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(w) + f * 8));
  W8 o;
  o.w[0] = bf16_lo(u.x); o.w[1] = bf16_hi(u.x); o.w[2] = bf16_lo(u.y); o.w[3] = bf16_hi(u.y);
  o.w[4] = bf16_lo(u.z); o.w[5] = bf16_hi(u.z); o.w[6] = bf16_lo(u.w); o.w[7] = bf16_hi(u.w);
  return o;
}

// Element i of an fp32 or bf16 array.
__device__ __forceinline__ float load_any(const float* __restrict__ a, int64_t i, bool bf) {
  return bf ? __uint_as_float((unsigned)__ldg(reinterpret_cast<const unsigned short*>(a) + i) << 16) : __ldg(a + i);
}

// Elements i, i+1 (i even) of an fp32 or bf16 array.
__device__ __forceinline__ float2 load2_any(const float* __restrict__ a, int64_t i, bool bf) {
  if (!bf) return __ldg(reinterpret_cast<const float2*>(a + i));
  const unsigned u = __ldg(reinterpret_cast<const unsigned*>(reinterpret_cast<const uint16_t*>(a) + i));
  return make_float2(bf16_lo(u), bf16_hi(u));
}

// Elements i .. i+3 (i a multiple of 4) of an fp32 or bf16 array.
__device__ __forceinline__ float4 load4_any(const float* __restrict__ a, int64_t i, bool bf) {
  if (!bf) return __ldg(reinterpret_cast<const float4*>(a + i));
  const uint2 u = __ldg(reinterpret_cast<const uint2*>(reinterpret_cast<const uint16_t*>(a) + i));
  return make_float4(bf16_lo(u.x), bf16_hi(u.x), bf16_lo(u.y), bf16_hi(u.y));
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
// argument checks of gl_bwd_shared_det_f32 (defined in modeb_det.cu)
int det_check_args(const GlSharedArgs& a, const float* qscale, const float* qinv, int* T);
}  // namespace gl
