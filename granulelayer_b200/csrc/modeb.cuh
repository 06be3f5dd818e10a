// Mode B (shared index records): parameters and helpers shared by the forward (modeb.cu) and
// backward (modeb_bwd.cu) kernels.
#pragma once
#include "common.cuh"

namespace gl {

constexpr int kMbFwdThreads = 384;
constexpr int kMbBwdThreads = 256;
constexpr int kMbStaticSmem = 8192;  // bound on either kernel's static shared memory (reduction buffers)

struct MbParams {
  const float* x;
  const int16_t* idx;
  const float* w;
  const float* b;
  const int32_t* counts;
  float* pre;
  const float* gpre;
  float* dx;
  float* dw;
  float* db;
  int B, D, C, lgLPR;  // lgLPR = log2(C / 4): lanes per record
  int64_t NB, g0, g1, ldx, ldp, ldg, lddx;
  int pool, gpc;
  int32_t* winners;
  int64_t ldwin;
  float* stat;      // forward, LME / softmax: the log2-normaliser [B, ldstat]
  int64_t ldstat;
  const float* c2;  // backward, smooth pools: coefficients c2, c3 [B, ldg]
  const float* c3;
  PoolParam pp;
  int ipm1;         // integer code of the power mean's p - 1 (-1: general)
  bool wbf;         // w and b stored as bf16 (gradients stay fp32)
};

template <bool PACKED>
__device__ __forceinline__ Rec8 mb_load_rec(const MbParams& p, int64_t g, int j) {
  if constexpr (!PACKED) {
    return load_rec8(p.idx + (g * p.NB + j) * 8, p.D - 1);
  } else {
    const MbPacked m = mb_packed(p.C, p.NB);
    const int16_t* base = p.idx + ((g * (p.NB / m.UB) + j / m.UB) * 8) * m.UB + j % m.UB;
    Rec8 r;
#pragma unroll
    for (int k = 0; k < 8; ++k) r.i[k] = min((int)(uint16_t)__ldg(base + k * m.UB), p.D - 1);
    return r;
  }
}

// Weights and bias of neurons c0 .. c0+3 of block j, from fp32 or bf16 storage (BF).
template <bool PACKED, bool BF>
__device__ __forceinline__ void mb_load_w4_t(const MbParams& p, int64_t g, int j, int c0, float (&w)[4][8],
                                             float (&bb)[4]) {
  if constexpr (!PACKED) {
    const int64_t base = ((g * p.NB + j) * p.C + c0) * 8;
#pragma unroll
    for (int n = 0; n < 4; ++n) {
      const float4 a = load4_any(p.w, base + 8 * n, BF), c = load4_any(p.w, base + 8 * n + 4, BF);
      w[n][0] = a.x; w[n][1] = a.y; w[n][2] = a.z; w[n][3] = a.w;
      w[n][4] = c.x; w[n][5] = c.y; w[n][6] = c.z; w[n][7] = c.w;
    }
    const float4 b4 = load4_any(p.b, (g * p.NB + j) * p.C + c0, BF);
    bb[0] = b4.x; bb[1] = b4.y; bb[2] = b4.z; bb[3] = b4.w;
  } else {
    const MbPacked m = mb_packed(p.C, p.NB);
#pragma unroll
    for (int n = 0; n < 4; ++n)
#pragma unroll
      for (int kh = 0; kh < 4; ++kh) {
        const float2 v = load2_any(p.w, mb_packed_w(m, g, j, c0 + n, kh), BF);
        w[n][2 * kh] = v.x;
        w[n][2 * kh + 1] = v.y;
      }
    const float2 b0 = load2_any(p.b, mb_packed_b(m, g, j, c0), BF);
    const float2 b1 = load2_any(p.b, mb_packed_b(m, g, j, c0 + 2), BF);
    bb[0] = b0.x; bb[1] = b0.y; bb[2] = b1.x; bb[3] = b1.y;
  }
}

// The storage type is uniform over the launch: one branch per record, around all of its loads.
template <bool PACKED>
__device__ __forceinline__ void mb_load_w4(const MbParams& p, int64_t g, int j, int c0, float (&w)[4][8],
                                           float (&bb)[4]) {
  if (p.wbf) mb_load_w4_t<PACKED, true>(p, g, j, c0, w, bb);
  else mb_load_w4_t<PACKED, false>(p, g, j, c0, w, bb);
}

// Row strides of the shared tiles.  Rows of 32 or more bytes start every row on the same banks
// when the stride is a multiple of 32 floats; the x tile pads rows by 4 floats (keeping the
// 16-byte alignment of its vector reads) and the dX tile by 1 float (scalar atomics), so that
// different rows read or add at different banks.
template <int T>
__host__ __device__ constexpr int mb_xld() { return T >= 8 ? T + 4 : T; }
template <int T>
__host__ __device__ constexpr int mb_dld() { return T >= 4 ? T + 1 : T; }

// Stage x[t0 .. t0+T-1, :] into xs[d * LD + t] (tokens >= B read as 0): one thread per feature.
template <int T, int LD, int NTHREADS>
__device__ __forceinline__ void mb_stage(float* __restrict__ xs, const float* __restrict__ x, int t0, int B, int D,
                                         int64_t ldx) {
  for (int d = threadIdx.x; d < D; d += NTHREADS) {
    float v[T];
#pragma unroll
    for (int t = 0; t < T; ++t) v[t] = (t0 + t < B) ? __ldg(x + (int64_t)(t0 + t) * ldx + d) : 0.f;
    float* row = xs + (int64_t)d * LD;
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

// T consecutive floats of an xs row.
template <int T>
__device__ __forceinline__ void mb_row(const float* __restrict__ row, float (&v)[T]) {
  if constexpr (T >= 4) {
#pragma unroll
    for (int q = 0; q < T / 4; ++q) {
      const float4 a = reinterpret_cast<const float4*>(row)[q];
      v[4 * q] = a.x; v[4 * q + 1] = a.y; v[4 * q + 2] = a.z; v[4 * q + 3] = a.w;
    }
  } else if constexpr (T == 2) {
    const float2 a = *reinterpret_cast<const float2*>(row);
    v[0] = a.x; v[1] = a.y;
  } else {
    v[0] = row[0];
  }
}

// v[k] <- v[k ^ km] for the top NBITS bits of k (bit 2 first); km has no other bits set.
template <int NBITS, typename V>
__device__ __forceinline__ void mb_xor_perm8(V (&v)[8], int km) {
#pragma unroll
  for (int s = 0; s < NBITS; ++s) {
    const int bit = 2 - s;
    const bool f = (km >> bit) & 1;
#pragma unroll
    for (int i = 0; i < 8; ++i)
      if (!((i >> bit) & 1)) {
        const V lo = v[i], hi = v[i | (1 << bit)];
        v[i] = f ? hi : lo;
        v[i | (1 << bit)] = f ? lo : hi;
      }
  }
}

// Weights of neurons c0 .. c0+3 of block j with the k index permuted: w[n][k] = W[c0+n][k ^ km].
template <bool PACKED, bool BF>
__device__ __forceinline__ void mb_load_w4_perm_t(const MbParams& p, int64_t g, int j, int c0, int km,
                                                  float (&w)[4][8]) {
  const int khm = km >> 1;
  const bool sw = km & 1;
  const MbPacked m = mb_packed(p.C, p.NB);
#pragma unroll
  for (int n = 0; n < 4; ++n)
#pragma unroll
    for (int khp = 0; khp < 4; ++khp) {
      const int kh = khp ^ khm;
      const int64_t off = PACKED ? mb_packed_w(m, g, j, c0 + n, kh) : ((g * p.NB + j) * p.C + c0 + n) * 8 + 2 * kh;
      const float2 v = load2_any(p.w, off, BF);
      w[n][2 * khp] = sw ? v.y : v.x;
      w[n][2 * khp + 1] = sw ? v.x : v.y;
    }
}

template <bool PACKED>
__device__ __forceinline__ void mb_load_w4_perm(const MbParams& p, int64_t g, int j, int c0, int km,
                                                float (&w)[4][8]) {
  if (p.wbf) mb_load_w4_perm_t<PACKED, true>(p, g, j, c0, km, w);
  else mb_load_w4_perm_t<PACKED, false>(p, g, j, c0, km, w);
}

// Dynamic shared memory: the padded x tile, plus the padded dX tile for the backward.
static inline int64_t mb_smem_bytes(int64_t D, int T, bool bwd) {
  const int xld = T >= 8 ? T + 4 : T, dld = T >= 4 ? T + 1 : T;
  return (((D * xld + 3) & ~3LL) + (bwd ? D * dld : 0)) * 4;
}

// Launches the backward kernel for token tile T (modeb_bwd.cu).
int mb_bwd_launch(const MbParams& p, int T, int act, bool packed, cudaStream_t st);

}  // namespace gl
