// Mode B (shared index records), fan-in 8, fp32: backward kernel (instantiated by modeb_bwd.cu for
// the mean / sum pools and by modeb_bwd_smooth.cu for LogMeanExp / power mean / softmax-weighted).
//
// Replaces the reference's Mode-B backward (sparse_pooling/kernels/cuda/sparse_pool_bwd.cuh:387-876),
// which runs BF16 mma tiles on the fragment-packed layout.  Tiling as the forward (modeb.cu): a
// block owns a token tile of T tokens (x staged feature-major, xs[d][t]) plus a block-private fp32
// dX tile [D][T], and a chunk of whole groups; lanes are (record, neuron quad), 2^LG = C/4 lanes
// per record.  Per record a lane recomputes z for its 4 neurons, forms dz = c1 * act'(z),
// accumulates its neurons' dW/db over the tile's tokens in registers (one vector global reduction
// per weight pair when the record is done) and, per sub-chunk of TS tokens, forms the quad's dX
// partials a[k][t] = sum_n dz[n][t] w[n][k].  A transpose-reduction over the record's lanes
// leaves each (k, t) sum on one lane, which adds it to the dX tile with one shared atomic: each
// (token, record, k) costs one atomic, 1/C of the per-neuron scatter of Mode A.  The tile is
// flushed to dx once per block.
//
// Select-free transpose-reduction.  At stage s the lanes whose lane bit s is set keep the upper
// half of their partials and send the lower half.  Each lane instead forms its partials with k
// XOR-permuted by a mask of its own lane bits (kmask): a[k'][t] is the partial of k' ^ kmask,
// computed from a second copy of its weights loaded with permuted columns (the pair index
// permutation is an address change, the bit-0 swap a select).  Every lane then keeps the lower
// half and sends the upper half, and the sum it ends with belongs to row idx[k' ^ kmask].  The x
// reads, z and dW keep the natural order, so the record's lanes read the same x row at the same
// time (one shared-memory broadcast).  The stage over a token bit (C = 64, the fourth stage) uses
// explicit selects.
#pragma once
#include "modeb.cuh"

namespace gl {

template <int T, int ACT, bool PACKED, int LG, bool SMOOTH>
__global__ void __launch_bounds__(kMbBwdThreads, 1) mb_bwd_kernel(const MbParams p) {
  constexpr int NW = kMbBwdThreads / 32;
  constexpr int TS = T < 4 ? T : 4;     // tokens per sub-chunk
  constexpr int V = 8 * TS;             // dX partials per lane and sub-chunk, index k * TS + t
  constexpr int LPR = 1 << LG, RPW = 32 >> LG, C = 4 * LPR;
  constexpr int LGK = LG < 3 ? LG : 3;  // select-free stages (over k bits)
  constexpr int HK = V >> LGK;          // partials a lane holds after them: NK rows x TS tokens
  constexpr int NK = 8 >> LGK;
  constexpr int HELD = LG < 4 ? HK : (HK >= 2 ? HK / 2 : 1);
  constexpr int XLD = mb_xld<T>(), DLD = mb_dld<T>();
  extern __shared__ __align__(16) float smem[];
  __shared__ float c1s[NW][T], c2s[NW][T], c3s[NW][T];  // per-warp copies of the group's coefficients
  float* xs = smem;
  float* dxs = smem + (((size_t)p.D * XLD + 3) & ~(size_t)3);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int t0 = blockIdx.x * T;
  mb_stage<T, XLD, kMbBwdThreads>(xs, p.x, t0, p.B, p.D, p.ldx);
  for (int e = threadIdx.x; e < p.D * DLD; e += kMbBwdThreads) dxs[e] = 0.f;
  __syncthreads();
  const int r = lane >> LG, nq = lane & (LPR - 1);
  int km = 0;
#pragma unroll
  for (int s = 0; s < LGK; ++s) km |= ((nq >> s) & 1) << (2 - s);
  const bool hi3 = LG >= 4 && ((nq >> 3) & 1);  // the token-bit stage: this lane keeps the upper tokens
  constexpr bool smooth = SMOOTH;                // LogMeanExp / power mean / softmax-weighted: pool_dz
  const int slots = (int)(p.NB * C);
  const int64_t gb = p.g0 + (int64_t)blockIdx.y * p.gpc;
  const int64_t ge = gb + p.gpc < p.g1 ? gb + p.gpc : p.g1;
  for (int64_t g = gb; g < ge; ++g) {
    const int ng = min(p.counts[g], slots);
    const int nbv = (ng + C - 1) / C;
    __syncwarp();
    if (lane < T) {
      const bool ok = t0 + lane < p.B;
      const int64_t ci = (int64_t)(t0 + lane) * p.ldg + (g - p.g0);
      const float v = ok ? __ldg(p.gpre + ci) : 0.f;
      c1s[warp][lane] = p.pool == GL_POOL_MEAN ? v / (float)ng : v;
      c2s[warp][lane] = ok && p.c2 != nullptr ? __ldg(p.c2 + ci) : 0.f;
      c3s[warp][lane] = ok && p.c3 != nullptr ? __ldg(p.c3 + ci) : 0.f;
    }
    __syncwarp();
    for (int base = warp * RPW; base < nbv; base += NW * RPW) {
      const int j = base + r;
      const bool okr = j < nbv;
      const int jj = okr ? j : 0;
      const Rec8 rec = mb_load_rec<PACKED>(p, g, jj);
      int ri[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) ri[k] = rec.i[k];
      mb_xor_perm8<LGK>(ri, km);
      int xrow[8], drow[NK];
#pragma unroll
      for (int k = 0; k < 8; ++k) xrow[k] = rec.i[k] * XLD;
#pragma unroll
      for (int k = 0; k < NK; ++k) drow[k] = ri[k] * DLD;
      float w[4][8], bb[4], wp[4][8];
      mb_load_w4<PACKED>(p, g, jj, nq * 4, w, bb);
      mb_load_w4_perm<PACKED>(p, g, jj, nq * 4, km, wp);
      const int nv = okr ? min(max(ng - (j * C + nq * 4), 0), 4) : 0;
      float dwacc[4][8], dbacc[4];
#pragma unroll
      for (int n = 0; n < 4; ++n) {
        dbacc[n] = 0.f;
#pragma unroll
        for (int k = 0; k < 8; ++k) dwacc[n][k] = 0.f;
      }
#pragma unroll 1
      for (int tc = 0; tc < T; tc += TS) {
        float c1[TS];
#pragma unroll
        for (int t = 0; t < TS; ++t) c1[t] = c1s[warp][tc + t];
        float xv[8][TS];
#pragma unroll
        for (int k = 0; k < 8; ++k) mb_row<TS>(xs + xrow[k] + tc, xv[k]);
        float dz[4][TS];
#pragma unroll
        for (int n = 0; n < 4; ++n) {
#pragma unroll
          for (int t = 0; t < TS; ++t) {
            float z = bb[n];
#pragma unroll
            for (int k = 0; k < 8; ++k) z = fmaf(w[n][k], xv[k][t], z);
            float d;
            if (smooth) d = pool_dz<ACT>(p.pool, z, c1[t], c2s[warp][tc + t], c3s[warp][tc + t], p.pp.param, p.ipm1);
            else d = c1[t] * dact_f<ACT>(z);
            dz[n][t] = n < nv ? d : 0.f;
            dbacc[n] += dz[n][t];
          }
#pragma unroll
          for (int k = 0; k < 8; ++k)
#pragma unroll
            for (int t = 0; t < TS; ++t) dwacc[n][k] = fmaf(dz[n][t], xv[k][t], dwacc[n][k]);
        }
        float a[V];
#pragma unroll
        for (int k = 0; k < 8; ++k)
#pragma unroll
          for (int t = 0; t < TS; ++t) {
            float sum = 0.f;
#pragma unroll
            for (int n = 0; n < 4; ++n) sum = fmaf(dz[n][t], wp[n][k], sum);
            a[k * TS + t] = sum;
          }
#pragma unroll
        for (int s = 0; s < LGK; ++s) {
          const int W = V >> s;
#pragma unroll
          for (int i = 0; i < W / 2; ++i) a[i] += __shfl_xor_sync(kFullMask, a[i + W / 2], 1 << s);
        }
        int tb = 0;
        bool writer = true;
        if constexpr (LG >= 4) {
          if constexpr (HK >= 2) {
#pragma unroll
            for (int i = 0; i < HK / 2; ++i) {
              const float keep = hi3 ? a[i + HK / 2] : a[i];
              const float send = hi3 ? a[i] : a[i + HK / 2];
              a[i] = keep + __shfl_xor_sync(kFullMask, send, 8);
            }
            tb = hi3 ? HK / 2 : 0;
          } else {
            a[0] += __shfl_xor_sync(kFullMask, a[0], 8);
            writer = !hi3;
          }
        }
        if (okr && writer) {
#pragma unroll
          for (int i = 0; i < HELD; ++i) {
            const int kk = LG >= 4 ? 0 : i / TS;
            const int t = LG >= 4 ? tb + i : i % TS;
            atomicAdd(&dxs[drow[kk] + tc + t], a[i]);
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

template <int T, int ACT, bool PACKED, int LG, bool SMOOTH>
static int mb_bwd_run(const MbParams& p, cudaStream_t st) {
  const size_t smem = (size_t)mb_smem_bytes(p.D, T, true);
  const void* kern = (const void*)mb_bwd_kernel<T, ACT, PACKED, LG, SMOOTH>;
  int rc = ensure_dynamic_smem(kern, smem);
  if (rc) return rc;
  const int64_t tiles = (p.B + T - 1) / T;
  const int64_t chunks = (p.g1 - p.g0 + p.gpc - 1) / p.gpc;
  if (tiles > 2147483647LL || chunks > 65535) return GL_ERR_SHAPE;
  mb_bwd_kernel<T, ACT, PACKED, LG, SMOOTH><<<dim3((unsigned)tiles, (unsigned)chunks), kMbBwdThreads, smem, st>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e);
  count_launches(1);
  return GL_OK;
}

template <int T, int ACT, bool PACKED, bool SMOOTH>
static int mb_bwd_lg2(const MbParams& p, cudaStream_t st) {
  switch (p.lgLPR) {
    case 1: return mb_bwd_run<T, ACT, PACKED, 1, SMOOTH>(p, st);
    case 2: return mb_bwd_run<T, ACT, PACKED, 2, SMOOTH>(p, st);
    case 3: return mb_bwd_run<T, ACT, PACKED, 3, SMOOTH>(p, st);
    case 4: return mb_bwd_run<T, ACT, PACKED, 4, SMOOTH>(p, st);
    default: return GL_ERR_SHAPE;
  }
}

template <int T, bool PACKED, bool SMOOTH>
static int mb_bwd_act(const MbParams& p, int act, cudaStream_t st) {
  switch (act) {
    case GL_ACT_IDENTITY: return mb_bwd_lg2<T, GL_ACT_IDENTITY, PACKED, SMOOTH>(p, st);
    case GL_ACT_RELU: return mb_bwd_lg2<T, GL_ACT_RELU, PACKED, SMOOTH>(p, st);
    case GL_ACT_GELU: return mb_bwd_lg2<T, GL_ACT_GELU, PACKED, SMOOTH>(p, st);
    default: return GL_ERR_UNSUPPORTED;
  }
}

template <bool SMOOTH>
static int mb_bwd_dispatch(const MbParams& p, int T, int act, bool packed, cudaStream_t st) {
#define GL_MB_BWD_T(TT) \
  case TT: return packed ? mb_bwd_act<TT, true, SMOOTH>(p, act, st) : mb_bwd_act<TT, false, SMOOTH>(p, act, st);
  switch (T) {
    GL_MB_BWD_T(32)
    GL_MB_BWD_T(16)
    GL_MB_BWD_T(8)
    GL_MB_BWD_T(4)
    GL_MB_BWD_T(2)
    GL_MB_BWD_T(1)
    default: return GL_ERR_UNSUPPORTED;
  }
#undef GL_MB_BWD_T
}

// The smooth pools' instantiations (modeb_bwd_smooth.cu).
int mb_bwd_launch_smooth(const MbParams& p, int T, int act, bool packed, cudaStream_t st);

}  // namespace gl
