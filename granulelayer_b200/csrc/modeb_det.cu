// Deterministic Mode-B backward (PhysicalPlan.reduction = "deterministic"), fp32 arithmetic with an
// exact 64-bit integer dX accumulation.
//
// Replaces the reference's deterministic reductions (sparse_pooling/kernels/cuda/sg_det.cu and the
// workspace owners of its grouped kernels; sparse_pooling/README.md "Deterministic execution"):
// every sum has a fixed owner and order, or is exact, so repeated runs are bitwise identical.
//   dW, db  a block owns a run of records of one group and walks the token tiles in order; the lane
//           that holds a record loads its dw/db, adds the tile's sums and stores them back.
//   dX      each (token, record, k) sum, reduced over the record's lanes in a fixed butterfly order,
//           is rounded once to a 64-bit integer at a per-token power-of-two scale qscale[t] = 2^e_t
//           (the caller picks e_t so that sum_d |dx[t, d]| 2^e_t < 2^61) and added with integer
//           atomics to a shared tile, whose entries are then added with integer atomics to the
//           caller's zeroed int64 buffer dxq [B, D].  Integer sums do not depend on their order.
//           A second kernel adds dxq[t, d] * qinv[t] to dx.
// The per-record arithmetic (z, dz, the dX partials and their select-free transpose-reduction) is
// the one of modeb_bwd.cu.
#include "modeb.cuh"

namespace gl {

constexpr int kDetThreads = 256;

template <int T>
__host__ __device__ constexpr int det_qld() { return T + 1; }  // int64 tile row stride: rows start on different banks

static int64_t det_smem_bytes(int64_t D, int T) {
  const int xld = T >= 8 ? T + 4 : T;
  return ((D * xld + 3) & ~3LL) * 4 + D * (T + 1) * 8;
}

template <int T, int ACT, bool PACKED, int LG>
__global__ void __launch_bounds__(kDetThreads, 1)
    mb_det_bwd_kernel(const MbParams p, unsigned long long* __restrict__ dxq, const float* __restrict__ qscale,
                      int cpg, int rpb) {
  constexpr int NW = kDetThreads / 32;
  constexpr int TS = T < 4 ? T : 4;
  constexpr int V = 8 * TS;
  constexpr int LPR = 1 << LG, RPW = 32 >> LG, C = 4 * LPR;
  constexpr int LGK = LG < 3 ? LG : 3;
  constexpr int HK = V >> LGK;
  constexpr int NK = 8 >> LGK;
  constexpr int HELD = LG < 4 ? HK : (HK >= 2 ? HK / 2 : 1);
  constexpr int XLD = mb_xld<T>(), QLD = det_qld<T>();
  extern __shared__ __align__(16) float smem[];
  __shared__ float c1s[NW][T], qs[T];
  float* xs = smem;
  unsigned long long* dq = reinterpret_cast<unsigned long long*>(smem + (((size_t)p.D * XLD + 3) & ~(size_t)3));
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int r = lane >> LG, nq = lane & (LPR - 1);
  int km = 0;
#pragma unroll
  for (int s = 0; s < LGK; ++s) km |= ((nq >> s) & 1) << (2 - s);
  const bool hi3 = LG >= 4 && ((nq >> 3) & 1);
  const int64_t g = p.g0 + blockIdx.x / cpg;
  const int slots = (int)(p.NB * C);
  const int ng = min(p.counts[g], slots);
  const int nbv = (ng + C - 1) / C;
  const int j0 = (int)(blockIdx.x % cpg) * rpb, j1 = min(j0 + rpb, nbv);
  if (j0 >= j1) return;  // uniform over the block, before any barrier
  const MbPacked m = mb_packed(C, p.NB);
  for (int t0 = 0; t0 < p.B; t0 += T) {
    mb_stage<T, XLD, kDetThreads>(xs, p.x, t0, p.B, p.D, p.ldx);
    for (int e = threadIdx.x; e < p.D * QLD; e += kDetThreads) dq[e] = 0ull;
    if (threadIdx.x < T) qs[threadIdx.x] = t0 + (int)threadIdx.x < p.B ? __ldg(qscale + t0 + threadIdx.x) : 0.f;
    if (lane < T) {
      const float v = t0 + lane < p.B ? __ldg(p.gpre + (int64_t)(t0 + lane) * p.ldg + (g - p.g0)) : 0.f;
      c1s[warp][lane] = p.pool == GL_POOL_MEAN ? v / (float)ng : v;
    }
    __syncthreads();
    for (int base = j0 + warp * RPW; base < j1; base += NW * RPW) {
      const int j = base + r;
      const bool okr = j < j1;
      const int jj = okr ? j : j0;
      const Rec8 rec = mb_load_rec<PACKED>(p, g, jj);
      int ri[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) ri[k] = rec.i[k];
      mb_xor_perm8<LGK>(ri, km);
      int xrow[8], drow[NK];
#pragma unroll
      for (int k = 0; k < 8; ++k) xrow[k] = rec.i[k] * XLD;
#pragma unroll
      for (int k = 0; k < NK; ++k) drow[k] = ri[k] * QLD;
      float w[4][8], bb[4], wp[4][8];
      mb_load_w4<PACKED>(p, g, jj, nq * 4, w, bb);
      mb_load_w4_perm<PACKED>(p, g, jj, nq * 4, km, wp);
      const int nv = okr ? min(max(ng - (j * C + nq * 4), 0), 4) : 0;
      // this lane owns these neurons' dW / db: the tile's sums accumulate onto the current values,
      // read here so that the loads overlap the token loop, and are stored back after it
      float dwacc[4][8], dbacc[4];
      if (nv > 0) {
        if constexpr (!PACKED) {
          const float4* dwp = reinterpret_cast<const float4*>(p.dw + ((g * p.NB + j) * C + nq * 4) * 8);
#pragma unroll
          for (int n = 0; n < 4; ++n)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const float4 v = dwp[2 * n + h];
              dwacc[n][4 * h] = v.x; dwacc[n][4 * h + 1] = v.y; dwacc[n][4 * h + 2] = v.z; dwacc[n][4 * h + 3] = v.w;
            }
          const float4 v = *reinterpret_cast<const float4*>(p.db + (g * p.NB + j) * C + nq * 4);
          dbacc[0] = v.x; dbacc[1] = v.y; dbacc[2] = v.z; dbacc[3] = v.w;
        } else {
#pragma unroll
          for (int n = 0; n < 4; ++n)
#pragma unroll
            for (int kh = 0; kh < 4; ++kh) {
              const float2 v = *reinterpret_cast<const float2*>(p.dw + mb_packed_w(m, g, j, nq * 4 + n, kh));
              dwacc[n][2 * kh] = v.x;
              dwacc[n][2 * kh + 1] = v.y;
            }
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const float2 v = *reinterpret_cast<const float2*>(p.db + mb_packed_b(m, g, j, nq * 4 + 2 * h));
            dbacc[2 * h] = v.x;
            dbacc[2 * h + 1] = v.y;
          }
        }
      } else {
#pragma unroll
        for (int n = 0; n < 4; ++n) {
          dbacc[n] = 0.f;
#pragma unroll
          for (int k = 0; k < 8; ++k) dwacc[n][k] = 0.f;
        }
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
            dz[n][t] = n < nv ? c1[t] * dact_f<ACT>(z) : 0.f;
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
            const long long q = __float2ll_rn(a[i] * qs[tc + t]);
            if (q != 0) atomicAdd(&dq[drow[kk] + tc + t], (unsigned long long)q);
          }
        }
      }
      if (nv > 0) {
        if constexpr (!PACKED) {
          float4* dwp = reinterpret_cast<float4*>(p.dw + ((g * p.NB + j) * C + nq * 4) * 8);
#pragma unroll
          for (int n = 0; n < 4; ++n)
#pragma unroll
            for (int h = 0; h < 2; ++h)
              dwp[2 * n + h] = make_float4(dwacc[n][4 * h], dwacc[n][4 * h + 1], dwacc[n][4 * h + 2], dwacc[n][4 * h + 3]);
          *reinterpret_cast<float4*>(p.db + (g * p.NB + j) * C + nq * 4) =
              make_float4(dbacc[0], dbacc[1], dbacc[2], dbacc[3]);
        } else {
#pragma unroll
          for (int n = 0; n < 4; ++n)
#pragma unroll
            for (int kh = 0; kh < 4; ++kh)
              *reinterpret_cast<float2*>(p.dw + mb_packed_w(m, g, j, nq * 4 + n, kh)) =
                  make_float2(dwacc[n][2 * kh], dwacc[n][2 * kh + 1]);
#pragma unroll
          for (int h = 0; h < 2; ++h)
            *reinterpret_cast<float2*>(p.db + mb_packed_b(m, g, j, nq * 4 + 2 * h)) =
                make_float2(dbacc[2 * h], dbacc[2 * h + 1]);
        }
      }
    }
    __syncthreads();
    for (int e = threadIdx.x; e < p.D * T; e += kDetThreads) {
      const int tt = e / p.D, d = e - tt * p.D;
      if (t0 + tt < p.B) {
        const unsigned long long v = dq[d * QLD + tt];
        if (v != 0ull) atomicAdd(dxq + (int64_t)(t0 + tt) * p.D + d, v);
      }
    }
    __syncthreads();
  }
}

// dx[t, d] += dxq[t, d] * qinv[t]  (qinv = 2^-e_t; NaN marks a token whose bound was not finite).
__global__ void det_finalize_kernel(const long long* __restrict__ dxq, const float* __restrict__ qinv,
                                    float* __restrict__ dx, int64_t B, int64_t D, int64_t lddx) {
  const int64_t n = B * D;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = e / D, d = e - t * D;
    const long long q = dxq[e];
    const float inv = __ldg(qinv + t);
    if (q != 0 || inv != inv) dx[t * lddx + d] += (float)((double)q * (double)inv);
  }
}

template <int T, int ACT, bool PACKED, int LG>
static int det_run(const MbParams& p, unsigned long long* dxq, const float* qscale, int cpg, int rpb,
                   cudaStream_t st) {
  const size_t smem = (size_t)det_smem_bytes(p.D, T);
  const void* kern = (const void*)mb_det_bwd_kernel<T, ACT, PACKED, LG>;
  int rc = ensure_dynamic_smem(kern, smem);
  if (rc) return rc;
  const int64_t blocks = (p.g1 - p.g0) * (int64_t)cpg;
  if (blocks > 2147483647LL) return GL_ERR_SHAPE;
  mb_det_bwd_kernel<T, ACT, PACKED, LG><<<(unsigned)blocks, kDetThreads, smem, st>>>(p, dxq, qscale, cpg, rpb);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e);
  count_launches(1);
  return GL_OK;
}

template <int T, int ACT, bool PACKED>
static int det_lg(const MbParams& p, unsigned long long* dxq, const float* qs, int cpg, int rpb, cudaStream_t st) {
  switch (p.lgLPR) {
    case 1: return det_run<T, ACT, PACKED, 1>(p, dxq, qs, cpg, rpb, st);
    case 2: return det_run<T, ACT, PACKED, 2>(p, dxq, qs, cpg, rpb, st);
    case 3: return det_run<T, ACT, PACKED, 3>(p, dxq, qs, cpg, rpb, st);
    case 4: return det_run<T, ACT, PACKED, 4>(p, dxq, qs, cpg, rpb, st);
    default: return GL_ERR_SHAPE;
  }
}

template <int T, bool PACKED>
static int det_act(const MbParams& p, int act, unsigned long long* dxq, const float* qs, int cpg, int rpb,
                   cudaStream_t st) {
  switch (act) {
    case GL_ACT_IDENTITY: return det_lg<T, GL_ACT_IDENTITY, PACKED>(p, dxq, qs, cpg, rpb, st);
    case GL_ACT_RELU: return det_lg<T, GL_ACT_RELU, PACKED>(p, dxq, qs, cpg, rpb, st);
    case GL_ACT_GELU: return det_lg<T, GL_ACT_GELU, PACKED>(p, dxq, qs, cpg, rpb, st);
    default: return GL_ERR_UNSUPPORTED;
  }
}

template <int T>
static int det_t(const MbParams& p, int act, bool packed, unsigned long long* dxq, const float* qs, int cpg, int rpb,
                 cudaStream_t st) {
  return packed ? det_act<T, true>(p, act, dxq, qs, cpg, rpb, st) : det_act<T, false>(p, act, dxq, qs, cpg, rpb, st);
}

}  // namespace gl

using namespace gl;

namespace gl {

// Every argument check of gl_bwd_shared_det_f32 except its scratch pointer, and the token tile the
// shared memory allows (*T).  GL_OK with *T = 0 means there is nothing to do (B = 0 or an empty
// group range).  The allocation-free variant runs it before it touches its shared scratch.
int det_check_args(const GlSharedArgs& a, const float* qscale, const float* qinv, int* T) {
  *T = 0;
  if (a.B < 0 || a.D < 1 || a.D > 32767 || a.NB < 1 || a.g0 < 0 || a.g1 < a.g0) return GL_ERR_SHAPE;
  if (a.C != 8 && a.C != 16 && a.C != 32 && a.C != 64) return GL_ERR_SHAPE;
  if (a.packed && (a.NB * (a.C / 8)) % 4) return GL_ERR_SHAPE;
  if (a.packed && (a.C / 8) < 4 && a.NB % (4 / (a.C / 8))) return GL_ERR_SHAPE;
  if (a.pool != GL_POOL_MEAN && a.pool != GL_POOL_SUM) return GL_ERR_UNSUPPORTED;
  if (a.wdtype != GL_DTYPE_F32 && a.wdtype != GL_DTYPE_BF16) return GL_ERR_UNSUPPORTED;
  if (a.B == 0 || a.g1 == a.g0) return GL_OK;
  if (!a.x || !a.idx || !a.w || !a.b || !a.counts || !a.gpre || !a.dx || !a.dw || !a.db) return GL_ERR_NULL;
  if (!qscale || !qinv) return GL_ERR_NULL;
  if (a.B > 2147483647LL || a.ldx < a.D || a.ldg < a.g1 - a.g0 || a.lddx < a.D) return GL_ERR_SHAPE;
  if (((uintptr_t)a.idx & 15) || ((uintptr_t)a.w & 15) || ((uintptr_t)a.b & 15) || ((uintptr_t)a.dw & 15) ||
      ((uintptr_t)a.db & 15))
    return GL_ERR_ALIGN;
  int optin = 0;
  int rc = device_smem_optin(&optin);
  if (rc) return rc;
  for (int c = 16; c >= 1 && !*T; c >>= 1)
    if (det_smem_bytes(a.D, c) + 2048 <= optin) *T = c;
  return *T ? GL_OK : GL_ERR_SMEM;
}

}  // namespace gl

extern "C" int gl_bwd_shared_det_f32(const GlSharedArgs* args, int64_t* dxq, const float* qscale, const float* qinv,
                                     void* stream) {
  if (!args) return GL_ERR_NULL;
  const GlSharedArgs& a = *args;
  int T = 0;
  int rc = det_check_args(a, qscale, qinv, &T);
  if (rc || !T) return rc;
  if (!dxq) return GL_ERR_NULL;
  if ((uintptr_t)dxq & 7) return GL_ERR_ALIGN;
  int sms = 0;
  if ((rc = device_sm_count(&sms))) return rc;
  const int64_t G = a.g1 - a.g0;
  const int64_t total = G * a.NB;
  int64_t rpb = (total + (int64_t)sms * 2 - 1) / ((int64_t)sms * 2);
  rpb = rpb < 64 ? 64 : rpb;
  rpb = rpb > a.NB ? a.NB : rpb;
  const int cpg = (int)((a.NB + rpb - 1) / rpb);
  MbParams p{};
  p.x = a.x; p.idx = a.idx; p.w = a.w; p.b = a.b; p.counts = a.counts; p.gpre = a.gpre;
  p.dx = a.dx; p.dw = a.dw; p.db = a.db;
  p.B = (int)a.B; p.D = (int)a.D; p.C = (int)a.C;
  p.lgLPR = a.C == 8 ? 1 : a.C == 16 ? 2 : a.C == 32 ? 3 : 4;
  p.NB = a.NB; p.g0 = a.g0; p.g1 = a.g1; p.ldx = a.ldx; p.ldg = a.ldg; p.lddx = a.lddx;
  p.pool = a.pool; p.gpc = 1;
  p.wbf = a.wdtype == GL_DTYPE_BF16;
  cudaStream_t st = (cudaStream_t)stream;
  unsigned long long* q = reinterpret_cast<unsigned long long*>(dxq);
  const bool packed = a.packed != 0;
  switch (T) {
    case 16: rc = det_t<16>(p, a.act, packed, q, qscale, cpg, (int)rpb, st); break;
    case 8: rc = det_t<8>(p, a.act, packed, q, qscale, cpg, (int)rpb, st); break;
    case 4: rc = det_t<4>(p, a.act, packed, q, qscale, cpg, (int)rpb, st); break;
    case 2: rc = det_t<2>(p, a.act, packed, q, qscale, cpg, (int)rpb, st); break;
    default: rc = det_t<1>(p, a.act, packed, q, qscale, cpg, (int)rpb, st); break;
  }
  if (rc) return rc;
  const int64_t n = a.B * a.D;
  const int64_t want = (n + 255) / 256;
  const unsigned blocks = (unsigned)(want < (int64_t)sms * 8 ? want : (int64_t)sms * 8);
  det_finalize_kernel<<<blocks, 256, 0, st>>>(reinterpret_cast<const long long*>(dxq), qinv, a.dx, a.B, a.D, a.lddx);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e);
  count_launches(1);
  return GL_OK;
}
