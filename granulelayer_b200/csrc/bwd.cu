// Backward: recompute z, then dX, dW and db in one pass (Mode A, fan-in 8, fp32).
//
// Replaces the reference's dense recompute backward: coefficients
// (sparse_pooling/kernels/ops.py:242-249, mean: c1 = g_pre / n_g), and the
// Triton bwd_dense_kernel (kernels/triton_fused.py:448-472) with its Mode-A
// tile (triton_fused.py:402-445, dz from _dz_from_z :364-374), which adds every
// (token, neuron, k) contribution to dX with a global FP32 atomic.
//
// B200 structure.  A thread block owns a token tile of T tokens and a chunk of
// whole pooling groups.  Shared memory holds feature-major tiles:
//   xs [D][T]  the staged inputs (read by the recompute and by dW),
//   a block-private dX accumulator [D][T],
// so the B*N*8 dX contributions become shared-memory reductions and global
// memory sees one coalesced flush of the tile per block.  Lanes are
// (neuron, token) pairs: T consecutive lanes hold one neuron's T tokens, so a
// warp step covers 32/T neurons; each lane recomputes its z, forms
// dz = c1[t, g] * act'(z), scatters dz * w_k into the accumulator, and keeps
// dz * x_k for dW.  The T lanes of a neuron then fold their 8 dW partials and
// the db partial with a transpose-reduce (each shuffle step halves the values
// a lane holds) and add them to dw/db with one vector reduction per lane.
//
// The accumulator is the kernel's hot spot: eight scattered shared-memory
// reductions per (token, neuron), on a shared-memory/L1 data path that ncu
// shows saturated.  Two variants:
//   generic  fp32 atomicAdd into an fp32 tile;
//   fixed    int32 atomicAdd into an int32 tile holding dz * w_k * s[t, g] rounded
//            to integers, folded into an fp32 tile after every group.  Integer
//            shared-memory atomics run ~2.4x the fp32 rate on B200.  The scale
//            s[t, g] = K_g / (|c1[t, g]| * max|w|_g * max|act'|) with
//            K_g = min(2^22, 0.9 * 2^31 / m_g), m_g the largest number of the
//            group's (slot, k) records sharing one input feature: every rounded
//            term then has |q| <= 2^22 (exact float->int rounding by the
//            1.5 * 2^23 magic-number add) and no tile word can exceed 0.9 * 2^31
//            within a group.  Rounding error per term is <= 0.5 / s, about 2^-23 of
//            the group's largest possible term, well inside the dX tolerance.
//            Integer sums within a group are also order-independent.
#include "common.cuh"

namespace gl {

constexpr int kBwdThreads = 1024;

// Transpose-reduce of the 8 dW partials and the db partial over the T token
// lanes of a neuron, then one vector reduction per lane into dw/db.
template <int T>
__device__ __forceinline__ void reduce_dw(float (&a)[8], float dz, int t, unsigned active, float* __restrict__ dw,
                                          float* __restrict__ db, int64_t f) {
  int kb = 0;
#pragma unroll
  for (int step = 1, width = 8; step < T; step <<= 1, width >>= 1) {
    const bool hi = (t & step) != 0;
#pragma unroll
    for (int j = 0; j < width / 2; ++j) {
      const float send = hi ? a[j] : a[j + width / 2];
      const float keep = hi ? a[j + width / 2] : a[j];
      a[j] = keep + __shfl_xor_sync(active, send, step);
    }
    if (hi) kb += width / 2;
  }
  float dbs = dz;
#pragma unroll
  for (int step = 1; step < T; step <<= 1) dbs += __shfl_xor_sync(active, dbs, step);
  float* dwp = dw + f * 8 + kb;
  if constexpr (T == 1) {
    red_add4(dwp, a[0], a[1], a[2], a[3]);
    red_add4(dwp + 4, a[4], a[5], a[6], a[7]);
  } else if constexpr (T == 2) {
    red_add4(dwp, a[0], a[1], a[2], a[3]);
  } else if constexpr (T == 4) {
    red_add2(dwp, a[0], a[1]);
  } else {
    red_add(dwp, a[0]);
  }
  if (t == 0) red_add(db + f, dbs);
}

struct BwdParams {
  const float* x;
  const int16_t* idx;
  const float* w;
  const float* bias;
  const int32_t* counts;
  const float* gpre;
  float* dx;
  float* dw;
  float* db;
  const float* wabsmax;
  const int32_t* rowmax;
  const int32_t* order;
  LocalMap lm;
  int B, D;
  int64_t NB, g0, g1, ldx, ldg, lddx;
  int pool, gpc;
  const float* c2;  // smooth pools: coefficients c2, c3 [B, ldg] and the pool's parameter
  const float* c3;
  float param;
  int ipm1;         // integer code of the power mean's p - 1 (-1: general)
};

// FIXED = false: fp32 tile.  FIXED = true: int32 tile + fp32 fold tile.  LOCAL: one group per block,
// tiles over the group's feature map only (rows = its features, records read as positions).
template <int T, int ACT, bool FIXED, bool LOCAL, bool SMOOTH, bool BF>
__global__ void __launch_bounds__(kBwdThreads, 1) bwd_kernel(const BwdParams p) {
  constexpr int NPW = 32 / T;
  constexpr int NW = kBwdThreads / 32;
  extern __shared__ __align__(16) float smem[];
  const size_t tile = ((size_t)(LOCAL ? p.lm.fcap : p.D) * T + 3) & ~(size_t)3;  // tiles start on 16-byte boundaries
  float* xs = smem;
  float* dxf = smem + tile;
  int* dxi = reinterpret_cast<int*>(smem + 2 * tile);
  __shared__ __align__(16) float inv_s[T];
  __shared__ int bad[T];

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int t0 = blockIdx.x * T;
  int D = p.D;  // rows of the tiles: the input features, or the group's feature map
  const int16_t* ridx = p.idx;
  const int16_t* cols = nullptr;
  if constexpr (LOCAL) {
    const int64_t gl = (int64_t)blockIdx.y * p.gpc;
    D = min(max(__ldg(p.lm.nfeat + gl), 1), p.lm.fcap);
    cols = p.lm.fmap + gl * p.lm.fcap;
    ridx = p.lm.lidx;
    stage_cols<T, kBwdThreads>(xs, p.x, t0, p.B, cols, D, p.ldx, p.D);
  } else {
    stage_tile<T, kBwdThreads>(xs, p.x, t0, p.B, D, p.ldx);
  }
  for (int e = threadIdx.x; e < D * T; e += kBwdThreads) {
    dxf[e] = 0.f;
    if constexpr (FIXED) dxi[e] = 0;
  }
  if (threadIdx.x < T) bad[threadIdx.x] = 0;
  __syncthreads();

  const int nsub = lane / T, t = lane % T;
  const bool tok_ok = t0 + t < p.B;
  const int slots = (int)(p.NB * 8);
  const int64_t gb = p.g0 + (int64_t)blockIdx.y * p.gpc;
  const int64_t ge = gb + p.gpc < p.g1 ? gb + p.gpc : p.g1;

  for (int64_t g = gb; g < ge; ++g) {
    const int ng = min(p.counts[g], slots);
    const int64_t fbase = g * (int64_t)slots;
    const int64_t ci = (int64_t)(t0 + t) * p.ldg + (g - p.g0);
    float c1 = tok_ok ? __ldg(p.gpre + ci) : 0.f;
    if (p.pool == GL_POOL_MEAN) c1 = c1 / (float)ng;
    constexpr bool smooth = SMOOTH;  // LogMeanExp / power mean / softmax-weighted: dz through pool_dz
    const float c2 = smooth && tok_ok && p.c2 != nullptr ? __ldg(p.c2 + ci) : 0.f;
    const float c3 = smooth && tok_ok && p.c3 != nullptr ? __ldg(p.c3 + ci) : 0.f;
    float c1s = 0.f;
    if constexpr (FIXED) {
      const float wm = __ldg(p.wabsmax + (g - p.g0));
      const float K = fminf(4194304.f, 0.9f * 2147483648.f / (float)max(__ldg(p.rowmax + (g - p.g0)), 1));
      const float den = fabsf(c1) * wm * dact_bound<ACT>();
      float sc = 0.f;
      if (!isfinite(c1) || !isfinite(wm)) {
        if (warp == 0 && nsub == 0 && tok_ok) bad[t] = 1;
      } else if (den > 1e-30f) {
        sc = K / den;
      }
      if (warp == 0 && nsub == 0) inv_s[t] = sc > 0.f ? 1.f / sc : 0.f;
      c1s = sc > 0.f ? c1 * sc : 0.f;
    }

    for (int s0 = warp * NPW; s0 < ng; s0 += NW * NPW) {
      const int s = s0 + nsub;
      const unsigned active = __ballot_sync(kFullMask, s < ng);
      if (s < ng) {
        const int slot =
            p.order != nullptr ? min(max(__ldg(p.order + (g - p.g0) * (int64_t)slots + s), 0), slots - 1) : s;
        const int64_t f = fbase + slot;
        const Rec8 r = load_rec8(ridx + f * 8, D - 1);
        const W8 wr = load_w8_any(p.w, f, BF);
        float z = load_any(p.bias, f, BF);
        float xv[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          xv[k] = xs[r.i[k] * T + t];
          z = fmaf(wr.w[k], xv[k], z);
        }
        const float da = dact_f<ACT>(z);
        const float dz = smooth ? pool_dz<ACT>(p.pool, z, c1, c2, c3, p.param, p.ipm1) : c1 * da;
        if constexpr (FIXED) {
          const float dzs = c1s * da;
          if (dzs != 0.f) {
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              const int q = __float_as_int(fmaf(dzs, wr.w[k], 12582912.f)) - 0x4B400000;
              atomicAdd(&dxi[r.i[k] * T + t], q);
            }
          }
        } else {
          if (dz != 0.f) {
#pragma unroll
            for (int k = 0; k < 8; ++k) atomicAdd(&dxf[r.i[k] * T + t], dz * wr.w[k]);
          }
        }
        float a[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) a[k] = dz * xv[k];
        reduce_dw<T>(a, dz, t, active, p.dw, p.db, f);
      }
    }
    if constexpr (FIXED) {
      // fold the group's integer tile into the fp32 tile and clear it
      __syncthreads();
      float inv[T];
#pragma unroll
      for (int j = 0; j < T; ++j) inv[j] = inv_s[j];
      for (int e4 = threadIdx.x; e4 < D * T / 4; e4 += kBwdThreads) {
        const int4 q = reinterpret_cast<const int4*>(dxi)[e4];
        float4 v = reinterpret_cast<float4*>(dxf)[e4];
        // tokens of the four elements: (4*e4 + j) % T, i.e. j % T, or 4*(e4 & 1) + j for T = 8
        float s0, s1, s2, s3;
        if constexpr (T == 8) {
          const bool hi = (e4 & 1) != 0;
          s0 = hi ? inv[4] : inv[0];
          s1 = hi ? inv[5] : inv[1];
          s2 = hi ? inv[6] : inv[2];
          s3 = hi ? inv[7] : inv[3];
        } else {
          s0 = inv[0];
          s1 = inv[1 % T];
          s2 = inv[2 % T];
          s3 = inv[3 % T];
        }
        v.x = fmaf((float)q.x, s0, v.x);
        v.y = fmaf((float)q.y, s1, v.y);
        v.z = fmaf((float)q.z, s2, v.z);
        v.w = fmaf((float)q.w, s3, v.w);
        reinterpret_cast<float4*>(dxf)[e4] = v;
        reinterpret_cast<int4*>(dxi)[e4] = make_int4(0, 0, 0, 0);
      }
      if ((D * T) % 4) {  // tail (D*T not a multiple of 4: only when T < 4 and D is odd)
        for (int e = (D * T / 4) * 4 + threadIdx.x; e < D * T; e += kBwdThreads) {
          const float sj = (T == 2 && (e & 1)) ? inv[T - 1] : inv[0];
          dxf[e] = fmaf((float)dxi[e], sj, dxf[e]);
          dxi[e] = 0;
        }
      }
      __syncthreads();
    }
  }
  __syncthreads();
  // flush the block's dX tile: consecutive threads take consecutive features
  const float nan = __int_as_float(0x7fc00000);
  for (int e = threadIdx.x; e < D * T; e += kBwdThreads) {
    const int tt = e / D, d = e - tt * D;
    if (t0 + tt < p.B) {
      const float v = (FIXED && bad[tt]) ? nan : dxf[d * T + tt];
      int col = d;
      if constexpr (LOCAL) col = min((int)(uint16_t)__ldg(cols + d), p.D - 1);
      if (v != 0.f) red_add(p.dx + (int64_t)(t0 + tt) * p.lddx + col, v);
    }
  }
}

// Dynamic shared-memory bytes: 2 tiles (generic) or 3 (fixed point) of D*T floats,
// each rounded up to 16 bytes.
static int64_t bwd_smem(int64_t D, int T, bool fixed) { return ((D * T + 3) & ~3LL) * 4 * (fixed ? 3 : 2); }

template <int T, int ACT, bool FIXED, bool LOCAL, bool SMOOTH, bool BF>
static int launch_bwd(const BwdParams& p, int64_t B, cudaStream_t st) {
  const size_t smem = (size_t)bwd_smem(LOCAL ? p.lm.fcap : p.D, T, FIXED);
  auto kern = bwd_kernel<T, ACT, FIXED, LOCAL, SMOOTH, BF>;
  int rc = ensure_dynamic_smem((const void*)kern, smem);
  if (rc) return rc;
  const int64_t tiles = (B + T - 1) / T;
  const int64_t chunks = (p.g1 - p.g0 + p.gpc - 1) / p.gpc;
  if (tiles > 2147483647LL || chunks > 65535) return GL_ERR_SHAPE;
  dim3 grid((unsigned)tiles, (unsigned)chunks);
  kern<<<grid, kBwdThreads, smem, st>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e);
  count_launches(1);
  return GL_OK;
}

template <int T, bool FIXED, bool LOCAL, bool SMOOTH, bool BF>
static int dispatch_act_bwd(const BwdParams& p, int64_t B, int act, cudaStream_t st) {
  switch (act) {
    case GL_ACT_IDENTITY: return launch_bwd<T, GL_ACT_IDENTITY, FIXED, LOCAL, SMOOTH, BF>(p, B, st);
    case GL_ACT_RELU: return launch_bwd<T, GL_ACT_RELU, FIXED, LOCAL, SMOOTH, BF>(p, B, st);
    case GL_ACT_GELU: return launch_bwd<T, GL_ACT_GELU, FIXED, LOCAL, SMOOTH, BF>(p, B, st);
    default: return GL_ERR_UNSUPPORTED;
  }
}

template <bool FIXED, bool LOCAL, bool SMOOTH, bool BF>
static int dispatch_tokens_bwd(const BwdParams& p, int64_t B, int act, int T, cudaStream_t st) {
  switch (T) {
    case 8: return dispatch_act_bwd<8, FIXED, LOCAL, SMOOTH, BF>(p, B, act, st);
    case 4: return dispatch_act_bwd<4, FIXED, LOCAL, SMOOTH, BF>(p, B, act, st);
    case 2: return dispatch_act_bwd<2, FIXED, LOCAL, SMOOTH, BF>(p, B, act, st);
    default: return dispatch_act_bwd<1, FIXED, LOCAL, SMOOTH, BF>(p, B, act, st);
  }
}


static int pick_bwd_tokens(int64_t D, int smem_optin, bool fixed) {
  for (int T = 8; T >= 1; T >>= 1)
    if (bwd_smem(D, T, fixed) <= smem_optin) return T;
  return GL_ERR_SMEM;
}

}  // namespace gl

using namespace gl;

extern "C" int gl_bwd_auto_tokens(int64_t D) {
  int optin = 0;
  int rc = device_smem_optin(&optin);
  if (rc) return rc;
  return pick_bwd_tokens(D, optin, true);
}

extern "C" int gl_bwd_f32(const GlBwdArgs* args, void* stream) {
  if (!args) return GL_ERR_NULL;
  const GlBwdArgs& a = *args;
  if (a.B < 0 || a.D < 1 || a.D > 32767 || a.NB < 1 || a.g0 < 0 || a.g1 < a.g0) return GL_ERR_SHAPE;
  if (a.B == 0 || a.g1 == a.g0) return GL_OK;
  if (!a.x || !a.idx || !a.w || !a.b || !a.counts || !a.gpre || !a.dx || !a.dw || !a.db) return GL_ERR_NULL;
  if ((a.wabsmax == nullptr) != (a.rowmax == nullptr)) return GL_ERR_NULL;
  if (a.B > 2147483647LL || a.ldx < a.D || a.ldg < a.g1 - a.g0 || a.lddx < a.D) return GL_ERR_SHAPE;
  if (((uintptr_t)a.idx & 15) || ((uintptr_t)a.w & 15) || ((uintptr_t)a.dw & 31)) return GL_ERR_ALIGN;
  if (a.pool != GL_POOL_MEAN && a.pool != GL_POOL_SUM && a.pool != GL_POOL_LME && a.pool != GL_POOL_POWER &&
      a.pool != GL_POOL_SOFTMAX)
    return GL_ERR_UNSUPPORTED;
  const bool smooth = a.pool >= GL_POOL_LME;
  if (smooth && (!a.c2 || (a.pool == GL_POOL_SOFTMAX && !a.c3))) return GL_ERR_NULL;
  if (a.wdtype != GL_DTYPE_F32 && a.wdtype != GL_DTYPE_BF16) return GL_ERR_UNSUPPORTED;
  if ((a.pool == GL_POOL_LME || a.pool == GL_POOL_SOFTMAX) && !(a.param > 0.f)) return GL_ERR_SHAPE;
  if (a.pool == GL_POOL_POWER && !(a.param >= 1.f)) return GL_ERR_SHAPE;
  int optin = 0, sms = 0;
  int rc = device_smem_optin(&optin);
  if (rc) return rc;
  if ((rc = device_sm_count(&sms))) return rc;
  const bool local = a.lidx != nullptr;
  if (local) {
    if (!a.fmap || !a.nfeat) return GL_ERR_NULL;
    if (a.fcap < 1 || a.fcap > a.D) return GL_ERR_SHAPE;
    if ((uintptr_t)a.lidx & 15) return GL_ERR_ALIGN;
    if (a.g1 - a.g0 > 65535) return GL_ERR_SHAPE;  // one group per block
  }
  const int64_t rows = local ? a.fcap : a.D;
  // fixed-point tiles when the caller supplied the two per-group bounds and they fit (mean / sum:
  // their |dz| <= |c1| max|act'| bound the terms)
  bool fixed = a.wabsmax != nullptr && !smooth;
  int T = a.tokens;
  if (T == 0) {
    T = pick_bwd_tokens(rows, optin, fixed);
    if (T < 0 && fixed) {
      fixed = false;
      T = pick_bwd_tokens(rows, optin, false);
    }
    if (T < 0) return T;
  } else if (T != 1 && T != 2 && T != 4 && T != 8) {
    return GL_ERR_UNSUPPORTED;
  }
  if (fixed && bwd_smem(rows, T, true) > optin) fixed = false;
  if (bwd_smem(rows, T, false) > optin) return GL_ERR_SMEM;
  const int64_t G = a.g1 - a.g0;
  int gpc = local ? 1 : a.groups_per_cta;
  if (gpc <= 0) {
    const int64_t tiles = (a.B + T - 1) / T;
    const int64_t units = tiles * G;
    int64_t want = units / ((int64_t)sms * 32);
    gpc = (int)(want < 1 ? 1 : (want > 8 ? 8 : want));
  }
  while ((G + gpc - 1) / gpc > 65535) gpc *= 2;
  BwdParams p{a.x, a.idx, a.w, a.b, a.counts, a.gpre, a.dx, a.dw, a.db, a.wabsmax, a.rowmax, a.order,
              LocalMap{a.lidx, a.fmap, a.nfeat, (int)a.fcap}, (int)a.B, (int)a.D,
              a.NB, a.g0, a.g1, a.ldx, a.ldg, a.lddx, a.pool, gpc, a.c2, a.c3, a.param,
              pow_code(a.param) >= 1 ? pow_code(a.param) - 1 : -1};
  cudaStream_t st = (cudaStream_t)stream;
  if (a.wdtype == GL_DTYPE_BF16) {  // bf16 storage: compiled for the full-row staging
    if (local) return GL_ERR_UNSUPPORTED;
    if (smooth) return dispatch_tokens_bwd<false, false, true, true>(p, a.B, a.act, T, st);
    return fixed ? dispatch_tokens_bwd<true, false, false, true>(p, a.B, a.act, T, st)
                 : dispatch_tokens_bwd<false, false, false, true>(p, a.B, a.act, T, st);
  }
  if (smooth)
    return local ? dispatch_tokens_bwd<false, true, true, false>(p, a.B, a.act, T, st)
                 : dispatch_tokens_bwd<false, false, true, false>(p, a.B, a.act, T, st);
  if (local)
    return fixed ? dispatch_tokens_bwd<true, true, false, false>(p, a.B, a.act, T, st)
                 : dispatch_tokens_bwd<false, true, false, false>(p, a.B, a.act, T, st);
  return fixed ? dispatch_tokens_bwd<true, false, false, false>(p, a.B, a.act, T, st)
               : dispatch_tokens_bwd<false, false, false, false>(p, a.B, a.act, T, st);
}
