// Mode B (shared index records), fan-in 8, fp32: forward and backward.
//
// Replaces the reference's Mode-B CUDA kernels (sparse_pooling/kernels/cuda/sparse_pool_fwd.cuh:311,
// sparse_pool_bwd.cuh:387-876, entries sparse_pool.cu:12-44), which run BF16 mma tiles on the
// fragment-packed layout.  Model (pytorch_reference.py:29-48): block j of group g holds C neurons
// that share one index record idx[g][j][0..7];
//   z[t, g, j, c] = b[g][j][c] + sum_k w[g][j][c][k] * x[t, idx[g][j][k]]
// and slot s = j*C + c is valid iff s < counts[g].  Storage is read in place, canonical
// (idx [G, NB, 8], w [G, NB, C, 8], b [G, NB, C]) or fragment-packed (layout.py:20-33, 146-179;
// the permutations are evaluated per element below).
//
// Because C neurons share each gather, the work per (token, neuron) is 8 FMAs and 8/C
// gathers: the kernels are FMA kernels fed from a shared-memory tile.  Lanes are (record,
// neuron quad): C/4 lanes per record, each holding 4 neurons' weights in registers, so every
// x value a lane loads feeds 4 FMAs.
//
// Forward: a block owns a token tile of T tokens (x staged feature-major, xs[d][t]) and a chunk
// of whole groups; per group the block sums act(z) over the valid slots with shuffles plus one
// shared-memory pass and writes pre[t, g] once (deterministic).
// Backward: the same tiling with a block-private fp32 dX tile [D][T].  Per record a lane
// recomputes z, forms dz = c1 * act'(z), adds its neurons' dW/db partials (summed over the tile's
// tokens) to dw/db with vector global reductions, and forms its quad's dX partial
// sum_n dz[n][t] w[n][k]; a transpose-reduction over the record's C/4 lanes leaves each (k, t)
// sum on one lane, which adds it to the dX tile.  Each (token, record, k) costs one shared
// atomic, 1/C of the per-neuron scatter of Mode A.  The tile is flushed once per block.
#include "common.cuh"

namespace gl {

constexpr int kMbFwdThreads = 384;
constexpr int kMbBwdThreads = 256;

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

// Weights and bias of neurons c0 .. c0+3 of block j.
template <bool PACKED>
__device__ __forceinline__ void mb_load_w4(const MbParams& p, int64_t g, int j, int c0, float (&w)[4][8],
                                           float (&bb)[4]) {
  if constexpr (!PACKED) {
    const float4* wp = reinterpret_cast<const float4*>(p.w + ((g * p.NB + j) * p.C + c0) * 8);
#pragma unroll
    for (int n = 0; n < 4; ++n) {
      const float4 a = __ldg(wp + 2 * n), c = __ldg(wp + 2 * n + 1);
      w[n][0] = a.x; w[n][1] = a.y; w[n][2] = a.z; w[n][3] = a.w;
      w[n][4] = c.x; w[n][5] = c.y; w[n][6] = c.z; w[n][7] = c.w;
    }
    const float4 b4 = __ldg(reinterpret_cast<const float4*>(p.b + (g * p.NB + j) * p.C + c0));
    bb[0] = b4.x; bb[1] = b4.y; bb[2] = b4.z; bb[3] = b4.w;
  } else {
    const MbPacked m = mb_packed(p.C, p.NB);
#pragma unroll
    for (int n = 0; n < 4; ++n)
#pragma unroll
      for (int kh = 0; kh < 4; ++kh) {
        const float2 v = __ldg(reinterpret_cast<const float2*>(p.w + mb_packed_w(m, g, j, c0 + n, kh)));
        w[n][2 * kh] = v.x;
        w[n][2 * kh + 1] = v.y;
      }
    const float2 b0 = __ldg(reinterpret_cast<const float2*>(p.b + mb_packed_b(m, g, j, c0)));
    const float2 b1 = __ldg(reinterpret_cast<const float2*>(p.b + mb_packed_b(m, g, j, c0 + 2)));
    bb[0] = b0.x; bb[1] = b0.y; bb[2] = b1.x; bb[3] = b1.y;
  }
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

// MAXP: max pooling with the winning slot (smallest on ties) written to p.winners.
template <int T, int ACT, bool PACKED, bool MAXP>
__global__ void __launch_bounds__(kMbFwdThreads, 1) mb_fwd_kernel(const MbParams p) {
  constexpr int NW = kMbFwdThreads / 32;
  constexpr int TS = T < 8 ? T : 8;  // tokens per sub-chunk (registers per lane stay fixed as T grows)
  extern __shared__ __align__(16) float xs[];
  __shared__ float red[NW][T];
  __shared__ int redi[MAXP ? NW : 1][T];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int t0 = blockIdx.x * T;
  constexpr int XLD = mb_xld<T>();
  mb_stage<T, XLD, kMbFwdThreads>(xs, p.x, t0, p.B, p.D, p.ldx);
  __syncthreads();
  const int C = p.C, LPR = 1 << p.lgLPR, RPW = 32 >> p.lgLPR;
  const int r = lane >> p.lgLPR, nq = lane & (LPR - 1);
  const int slots = (int)(p.NB * C);
  const int64_t gb = p.g0 + (int64_t)blockIdx.y * p.gpc;
  const int64_t ge = gb + p.gpc < p.g1 ? gb + p.gpc : p.g1;
  for (int64_t g = gb; g < ge; ++g) {
    const int ng = min(p.counts[g], slots);
    const int nbv = (ng + C - 1) / C;
    float acc[T];
    int wid[MAXP ? T : 1];
#pragma unroll
    for (int t = 0; t < T; ++t) {
      acc[t] = MAXP ? -INFINITY : 0.f;
      if constexpr (MAXP) wid[t] = 0x7fffffff;
    }
    for (int base = warp * RPW; base < nbv; base += NW * RPW) {
      const int j = base + r;
      const bool okr = j < nbv;
      const int jj = okr ? j : 0;
      const Rec8 rec = mb_load_rec<PACKED>(p, g, jj);
      float w[4][8], bb[4];
      mb_load_w4<PACKED>(p, g, jj, nq * 4, w, bb);
      const int nv = okr ? min(max(ng - (j * C + nq * 4), 0), 4) : 0;
#pragma unroll
      for (int tc = 0; tc < T; tc += TS) {
        float z[4][TS];
#pragma unroll
        for (int n = 0; n < 4; ++n)
#pragma unroll
          for (int t = 0; t < TS; ++t) z[n][t] = bb[n];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          float v[TS];
          mb_row<TS>(xs + rec.i[k] * XLD + tc, v);
#pragma unroll
          for (int n = 0; n < 4; ++n)
#pragma unroll
            for (int t = 0; t < TS; ++t) z[n][t] = fmaf(w[n][k], v[t], z[n][t]);
        }
#pragma unroll
        for (int n = 0; n < 4; ++n)
          if (n < nv)
#pragma unroll
            for (int t = 0; t < TS; ++t) {
              const float a = act_f<ACT>(z[n][t]);
              if constexpr (MAXP) {
                const int slot = j * C + nq * 4 + n;
                if (a > acc[tc + t] || (a == acc[tc + t] && slot < wid[tc + t])) {
                  acc[tc + t] = a;
                  wid[tc + t] = slot;
                }
              } else {
                acc[tc + t] += a;
              }
            }
      }
    }
#pragma unroll
    for (int off = 16; off; off >>= 1)
#pragma unroll
      for (int t = 0; t < T; ++t) {
        const float ov = __shfl_xor_sync(kFullMask, acc[t], off);
        if constexpr (MAXP) {
          const int ow = __shfl_xor_sync(kFullMask, wid[t], off);
          if (ov > acc[t] || (ov == acc[t] && ow < wid[t])) {
            acc[t] = ov;
            wid[t] = ow;
          }
        } else {
          acc[t] += ov;
        }
      }
    if (lane == 0)
#pragma unroll
      for (int t = 0; t < T; ++t) {
        red[warp][t] = acc[t];
        if constexpr (MAXP) redi[warp][t] = wid[t];
      }
    __syncthreads();
    if (threadIdx.x < T) {
      const int t = t0 + threadIdx.x;
      if constexpr (MAXP) {
        float m = -INFINITY;
        int wi = 0x7fffffff;
#pragma unroll
        for (int i = 0; i < NW; ++i) {
          const float v = red[i][threadIdx.x];
          const int vi = redi[i][threadIdx.x];
          if (v > m || (v == m && vi < wi)) {
            m = v;
            wi = vi;
          }
        }
        if (t < p.B) {
          p.pre[(int64_t)t * p.ldp + (g - p.g0)] = m;
          if (p.winners != nullptr) p.winners[(int64_t)t * p.ldwin + (g - p.g0)] = wi;
        }
      } else {
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < NW; ++i) s += red[i][threadIdx.x];
        if (t < p.B) p.pre[(int64_t)t * p.ldp + (g - p.g0)] = p.pool == GL_POOL_MEAN ? s / (float)ng : s;
      }
    }
    __syncthreads();
  }
}

template <int T, int ACT, bool PACKED>
__global__ void __launch_bounds__(kMbBwdThreads, 1) mb_bwd_kernel(const MbParams p) {
  constexpr int NW = kMbBwdThreads / 32;
  constexpr int TS = T < 4 ? T : 4;  // tokens per sub-chunk
  constexpr int V = 8 * TS;          // dX partials per lane and sub-chunk: (k, t), index k*TS + t
  extern __shared__ __align__(16) float smem[];
  float* xs = smem;
  constexpr int XLD = mb_xld<T>(), DLD = mb_dld<T>();
  float* dxs = smem + (((size_t)p.D * XLD + 3) & ~(size_t)3);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int t0 = blockIdx.x * T;
  mb_stage<T, XLD, kMbBwdThreads>(xs, p.x, t0, p.B, p.D, p.ldx);
  for (int e = threadIdx.x; e < p.D * DLD; e += kMbBwdThreads) dxs[e] = 0.f;
  __syncthreads();
  const int C = p.C, LPR = 1 << p.lgLPR, RPW = 32 >> p.lgLPR;
  const int r = lane >> p.lgLPR, nq = lane & (LPR - 1);
  const int slots = (int)(p.NB * C);
  const int64_t gb = p.g0 + (int64_t)blockIdx.y * p.gpc;
  const int64_t ge = gb + p.gpc < p.g1 ? gb + p.gpc : p.g1;
  for (int64_t g = gb; g < ge; ++g) {
    const int ng = min(p.counts[g], slots);
    const int nbv = (ng + C - 1) / C;
    float c1[T];
#pragma unroll
    for (int t = 0; t < T; ++t) {
      const float v = t0 + t < p.B ? __ldg(p.gpre + (int64_t)(t0 + t) * p.ldg + (g - p.g0)) : 0.f;
      c1[t] = p.pool == GL_POOL_MEAN ? v / (float)ng : v;
    }
    for (int base = warp * RPW; base < nbv; base += NW * RPW) {
      const int j = base + r;
      const bool okr = j < nbv;
      const int jj = okr ? j : 0;
      const Rec8 rec = mb_load_rec<PACKED>(p, g, jj);
      float w[4][8], bb[4];
      mb_load_w4<PACKED>(p, g, jj, nq * 4, w, bb);
      const int nv = okr ? min(max(ng - (j * C + nq * 4), 0), 4) : 0;
      float dwacc[4][8], dbacc[4];
#pragma unroll
      for (int n = 0; n < 4; ++n) {
        dbacc[n] = 0.f;
#pragma unroll
        for (int k = 0; k < 8; ++k) dwacc[n][k] = 0.f;
      }
#pragma unroll
      for (int tc = 0; tc < T; tc += TS) {
        float xv[8][TS];
#pragma unroll
        for (int k = 0; k < 8; ++k) mb_row<TS>(xs + rec.i[k] * XLD + tc, xv[k]);
        float dz[4][TS];
#pragma unroll
        for (int n = 0; n < 4; ++n) {
#pragma unroll
          for (int t = 0; t < TS; ++t) {
            float z = bb[n];
#pragma unroll
            for (int k = 0; k < 8; ++k) z = fmaf(w[n][k], xv[k][t], z);
            dz[n][t] = n < nv ? c1[tc + t] * dact_f<ACT>(z) : 0.f;
            dbacc[n] += dz[n][t];
          }
#pragma unroll
          for (int k = 0; k < 8; ++k)
#pragma unroll
            for (int t = 0; t < TS; ++t) dwacc[n][k] = fmaf(dz[n][t], xv[k][t], dwacc[n][k]);
        }
        // dX partials of the quad, then a transpose-reduction over the record's LPR lanes
        float a[V];
#pragma unroll
        for (int k = 0; k < 8; ++k)
#pragma unroll
          for (int t = 0; t < TS; ++t) {
            float sum = 0.f;
#pragma unroll
            for (int n = 0; n < 4; ++n) sum = fmaf(dz[n][t], w[n][k], sum);
            a[k * TS + t] = sum;
          }
        int vbase = 0;      // first partial index this lane holds
        bool writer = true; // false on the upper lane of a plain (non-transposing) butterfly stage
#pragma unroll
        for (int s = 0; s < 4; ++s) {
          const int width = V >> s;  // a compile-time constant once the loop is unrolled
          if (s < p.lgLPR) {
            const bool hi = (nq >> s) & 1;
            if (width > 1) {
#pragma unroll
              for (int i = 0; i < width / 2; ++i) {
                const float keep = hi ? a[i + width / 2] : a[i];
                const float send = hi ? a[i] : a[i + width / 2];
                a[i] = keep + __shfl_xor_sync(kFullMask, send, 1 << s);
              }
              if (hi) vbase += width / 2;
            } else {
              a[0] += __shfl_xor_sync(kFullMask, a[0], 1 << s);
              if (hi) writer = false;
            }
          }
        }
        const int held = max(V >> p.lgLPR, 1);
        if (okr && writer) {
#pragma unroll
          for (int i = 0; i < V; ++i) {
            if (i < held) {
              const int v = vbase + i, k = v / TS, t = v - k * TS;
              int row = rec.i[0];  // rec.i[k] through selects: a dynamic index would place rec in local memory
#pragma unroll
              for (int q = 1; q < 8; ++q) row = k == q ? rec.i[q] : row;
              atomicAdd(&dxs[row * DLD + tc + t], a[i]);
            }
          }
        }
      }
      if (nv > 0) {
        if constexpr (!PACKED) {
          float* dwp = p.dw + ((g * p.NB + j) * C + nq * 4) * 8;
#pragma unroll
          for (int n = 0; n < 4; ++n) {
            red_add4(dwp + 8 * n, dwacc[n][0], dwacc[n][1], dwacc[n][2], dwacc[n][3]);
            red_add4(dwp + 8 * n + 4, dwacc[n][4], dwacc[n][5], dwacc[n][6], dwacc[n][7]);
          }
          red_add4(p.db + (g * p.NB + j) * C + nq * 4, dbacc[0], dbacc[1], dbacc[2], dbacc[3]);
        } else {
          const MbPacked m = mb_packed(C, p.NB);
#pragma unroll
          for (int n = 0; n < 4; ++n)
#pragma unroll
            for (int kh = 0; kh < 4; ++kh)
              red_add2(p.dw + mb_packed_w(m, g, j, nq * 4 + n, kh), dwacc[n][2 * kh], dwacc[n][2 * kh + 1]);
          red_add2(p.db + mb_packed_b(m, g, j, nq * 4), dbacc[0], dbacc[1]);
          red_add2(p.db + mb_packed_b(m, g, j, nq * 4 + 2), dbacc[2], dbacc[3]);
        }
      }
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < p.D * T; e += kMbBwdThreads) {
    const int tt = e / p.D, d = e - tt * p.D;
    if (t0 + tt < p.B) {
      const float v = dxs[d * DLD + tt];
      if (v != 0.f) red_add(p.dx + (int64_t)(t0 + tt) * p.lddx + d, v);
    }
  }
}

// Dynamic shared memory: the padded x tile, plus the padded dX tile for the backward.
static int64_t mb_smem_bytes(int64_t D, int T, bool bwd) {
  const int xld = T >= 8 ? T + 4 : T, dld = T >= 4 ? T + 1 : T;
  return (((D * xld + 3) & ~3LL) + (bwd ? D * dld : 0)) * 4;
}

template <int T, int ACT, bool PACKED>
static int mb_launch(const MbParams& p, bool bwd, cudaStream_t st) {
  const size_t smem = (size_t)mb_smem_bytes(p.D, T, bwd);
  const bool maxp = !bwd && p.pool == GL_POOL_MAX;
  const void* kern = bwd ? (const void*)mb_bwd_kernel<T, ACT, PACKED>
                         : (maxp ? (const void*)mb_fwd_kernel<T, ACT, PACKED, true>
                                 : (const void*)mb_fwd_kernel<T, ACT, PACKED, false>);
  int rc = ensure_dynamic_smem(kern, smem);
  if (rc) return rc;
  const int64_t tiles = (p.B + T - 1) / T;
  const int64_t chunks = (p.g1 - p.g0 + p.gpc - 1) / p.gpc;
  if (tiles > 2147483647LL || chunks > 65535) return GL_ERR_SHAPE;
  const dim3 grid((unsigned)tiles, (unsigned)chunks);
  if (bwd) mb_bwd_kernel<T, ACT, PACKED><<<grid, kMbBwdThreads, smem, st>>>(p);
  else if (maxp) mb_fwd_kernel<T, ACT, PACKED, true><<<grid, kMbFwdThreads, smem, st>>>(p);
  else mb_fwd_kernel<T, ACT, PACKED, false><<<grid, kMbFwdThreads, smem, st>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e);
  count_launches(1);
  return GL_OK;
}

template <int T, bool PACKED>
static int mb_dispatch_act(const MbParams& p, int act, bool bwd, cudaStream_t st) {
  switch (act) {
    case GL_ACT_IDENTITY: return mb_launch<T, GL_ACT_IDENTITY, PACKED>(p, bwd, st);
    case GL_ACT_RELU: return mb_launch<T, GL_ACT_RELU, PACKED>(p, bwd, st);
    case GL_ACT_GELU: return mb_launch<T, GL_ACT_GELU, PACKED>(p, bwd, st);
    default: return GL_ERR_UNSUPPORTED;
  }
}

template <int T>
static int mb_dispatch(const MbParams& p, int act, bool packed, bool bwd, cudaStream_t st) {
  return packed ? mb_dispatch_act<T, true>(p, act, bwd, st) : mb_dispatch_act<T, false>(p, act, bwd, st);
}

// Largest token tile in {32, 16, 8, 4, 2, 1} whose tiles (1 forward, 2 backward) fit the opt-in shared memory.
static int mb_pick_tokens(int64_t D, bool bwd, int optin) {
  for (int T = 32; T >= 1; T >>= 1)
    if (mb_smem_bytes(D, T, bwd) + 2048 <= optin) return T;
  return GL_ERR_SMEM;
}

static int mb_run(const GlSharedArgs& a, bool bwd, void* stream) {
  if (a.B < 0 || a.D < 1 || a.D > 32767 || a.NB < 1 || a.g0 < 0 || a.g1 < a.g0) return GL_ERR_SHAPE;
  if (a.C != 8 && a.C != 16 && a.C != 32 && a.C != 64) return GL_ERR_SHAPE;
  if (a.packed && (a.NB * (a.C / 8)) % 4) return GL_ERR_SHAPE;
  if (a.packed && (a.C / 8) < 4 && a.NB % (4 / (a.C / 8))) return GL_ERR_SHAPE;
  if (a.B == 0 || a.g1 == a.g0) return GL_OK;
  if (!a.x || !a.idx || !a.w || !a.b || !a.counts) return GL_ERR_NULL;
  if (a.B > 2147483647LL || a.ldx < a.D || a.NB * a.C > 2147483647LL) return GL_ERR_SHAPE;
  if (((uintptr_t)a.idx & 15) || ((uintptr_t)a.w & 15) || ((uintptr_t)a.b & 15)) return GL_ERR_ALIGN;
  if (a.pool != GL_POOL_MEAN && a.pool != GL_POOL_SUM && !(a.pool == GL_POOL_MAX && !bwd)) return GL_ERR_UNSUPPORTED;
  if (a.winners && a.ldwin < a.g1 - a.g0) return GL_ERR_SHAPE;
  if (!bwd) {
    if (!a.pre) return GL_ERR_NULL;
    if (a.ldp < a.g1 - a.g0) return GL_ERR_SHAPE;
  } else {
    if (!a.gpre || !a.dx || !a.dw || !a.db) return GL_ERR_NULL;
    if (a.ldg < a.g1 - a.g0 || a.lddx < a.D) return GL_ERR_SHAPE;
    if (((uintptr_t)a.dw & 15) || ((uintptr_t)a.db & 15)) return GL_ERR_ALIGN;
  }
  int optin = 0, sms = 0;
  int rc = device_smem_optin(&optin);
  if (rc) return rc;
  if ((rc = device_sm_count(&sms))) return rc;
  int T = a.tokens;
  if (T == 0) {
    T = mb_pick_tokens(a.D, bwd, optin);
    if (T < 0) return T;
    if (a.pool == GL_POOL_MAX && T > 16) T = 16;  // max keeps a winner per token in registers
  } else if (T != 1 && T != 2 && T != 4 && T != 8 && T != 16 && T != 32) {
    return GL_ERR_UNSUPPORTED;
  }
  if (mb_smem_bytes(a.D, T, bwd) + 2048 > optin) return GL_ERR_SMEM;
  const int64_t G = a.g1 - a.g0;
  int gpc = a.groups_per_cta;
  if (gpc <= 0) {
    const int64_t units = ((a.B + T - 1) / T) * G;
    const int64_t want = units / ((int64_t)sms * 32);
    gpc = (int)(want < 1 ? 1 : (want > 8 ? 8 : want));
  }
  while ((G + gpc - 1) / gpc > 65535) gpc *= 2;
  MbParams p;
  p.x = a.x; p.idx = a.idx; p.w = a.w; p.b = a.b; p.counts = a.counts; p.pre = a.pre; p.gpre = a.gpre;
  p.dx = a.dx; p.dw = a.dw; p.db = a.db;
  p.B = (int)a.B; p.D = (int)a.D; p.C = (int)a.C;
  p.lgLPR = a.C == 8 ? 1 : a.C == 16 ? 2 : a.C == 32 ? 3 : 4;
  p.NB = a.NB; p.g0 = a.g0; p.g1 = a.g1; p.ldx = a.ldx; p.ldp = a.ldp; p.ldg = a.ldg; p.lddx = a.lddx;
  p.pool = a.pool; p.gpc = gpc; p.winners = a.winners; p.ldwin = a.ldwin;
  cudaStream_t st = (cudaStream_t)stream;
  const bool packed = a.packed != 0;
  switch (T) {
    case 32: return mb_dispatch<32>(p, a.act, packed, bwd, st);
    case 16: return mb_dispatch<16>(p, a.act, packed, bwd, st);
    case 8: return mb_dispatch<8>(p, a.act, packed, bwd, st);
    case 4: return mb_dispatch<4>(p, a.act, packed, bwd, st);
    case 2: return mb_dispatch<2>(p, a.act, packed, bwd, st);
    default: return mb_dispatch<1>(p, a.act, packed, bwd, st);
  }
}

}  // namespace gl

extern "C" int gl_fwd_shared_f32(const GlSharedArgs* args, void* stream) {
  if (!args) return GL_ERR_NULL;
  return gl::mb_run(*args, false, stream);
}

extern "C" int gl_bwd_shared_f32(const GlSharedArgs* args, void* stream) {
  if (!args) return GL_ERR_NULL;
  return gl::mb_run(*args, true, stream);
}

extern "C" int gl_shared_auto_tokens(int64_t D, int32_t backward) {
  int optin = 0;
  const int rc = gl::device_smem_optin(&optin);
  if (rc) return rc;
  return gl::mb_pick_tokens(D, backward != 0, optin);
}
