// Mode B (shared index records), fan-in 8, fp32: forward (the backward is in modeb_bwd.cu).
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
#include "modeb.cuh"

namespace gl {

// PK (the pooling state, common.cuh): PK_MAX writes the winning slot (smallest on ties) to
// p.winners; PK_LSE / PK_POW hold three-word states (their tiles stay at 8 tokens or fewer);
// PK_TOPK / PK_TOPK64 keep per-warp lists (tiles of 4 tokens or fewer) merged per group.
template <int T, int ACT, bool PACKED, int PK>
__global__ void __launch_bounds__(kMbFwdThreads, 1) mb_fwd_kernel(const MbParams p) {
  constexpr bool MAXP = PK == PK_MAX;
  constexpr bool SM = PK == PK_LSE || PK == PK_POW;
  constexpr bool TK = PK == PK_TOPK || PK == PK_TOPK64;
  constexpr int KW = PK == PK_TOPK64 ? 2 : 1;
  constexpr int NW = kMbFwdThreads / 32;
  constexpr int TS = T < 8 ? T : 8;  // tokens per sub-chunk (registers per lane stay fixed as T grows)
  extern __shared__ __align__(16) float xs[];
  // per-warp partials, double-buffered by group parity: one barrier per group
  __shared__ float red[2][NW][T];
  __shared__ int redi[2][MAXP ? NW : 1][T];
  __shared__ float red1[2][SM ? NW : 1][T], red2[2][SM ? NW : 1][T];
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
  long long* tks = reinterpret_cast<long long*>(xs + (((int64_t)p.D * XLD + 3) & ~3LL));  // top-K lists
  for (int64_t g = gb; g < ge; ++g) {
    const int ng = min(p.counts[g], slots);
    const int nbv = (ng + C - 1) / C;
    const int buf = (int)((g - gb) & 1);
    long long tkw[TK ? T : 1][KW], tthr[TK ? T : 1];
    if constexpr (TK) {
#pragma unroll
      for (int t = 0; t < T; ++t) {
        tthr[t] = LLONG_MIN;
#pragma unroll
        for (int wd = 0; wd < KW; ++wd) tkw[t][wd] = LLONG_MIN;
      }
    }
    float acc[T];
    int wid[MAXP ? T : 1];
    float st1[SM ? T : 1], st2[SM ? T : 1];
#pragma unroll
    for (int t = 0; t < T; ++t) {
      acc[t] = (MAXP || PK == PK_LSE) ? -INFINITY : 0.f;
      if constexpr (MAXP) wid[t] = 0x7fffffff;
      if constexpr (SM) st1[t] = st2[t] = 0.f;
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
        if constexpr (TK) {  // every lane takes part in the warp's insertions
#pragma unroll
          for (int n = 0; n < 4; ++n)
#pragma unroll
            for (int t = 0; t < TS; ++t)
              topk_offer<KW>(tkw[tc + t], tthr[tc + t], n < nv, topk_key(z[n][t], j * C + nq * 4 + n), p.pp.k,
                             lane);
        }
#pragma unroll
        for (int n = 0; n < 4; ++n)
          if (n < nv && !TK)
#pragma unroll
            for (int t = 0; t < TS; ++t) {
              const float a = act_f<ACT>(z[n][t]);
              if constexpr (MAXP) {
                // a lane visits its slots in increasing order, so a strict compare keeps the
                // smallest slot among its ties; ties across lanes are settled in the reduction
                const bool up = a > acc[tc + t];
                acc[tc + t] = up ? a : acc[tc + t];
                wid[tc + t] = up ? j * C + nq * 4 + n : wid[tc + t];
              } else if constexpr (PK == PK_LSE) {
                lse_push(acc[tc + t], st1[tc + t], st2[tc + t], a * p.pp.param, a, p.pp.want_t);
              } else if constexpr (PK == PK_POW) {
                pow_push(acc[tc + t], st1[tc + t], st2[tc + t], a, p.pp);
              } else {
                acc[tc + t] += a;
              }
            }
      }
    }
    if constexpr (TK) {
      // merge the warps' lists: warp t takes token t
#pragma unroll
      for (int t = 0; t < T; ++t)
#pragma unroll
        for (int wd = 0; wd < KW; ++wd) tks[((warp * T + t) * KW + wd) * 32 + lane] = tkw[t][wd];
      __syncthreads();
      if (warp < T) {
        const int t = warp;
        long long wl[KW];
#pragma unroll
        for (int wd = 0; wd < KW; ++wd) wl[wd] = tks[(t * KW + wd) * 32 + lane];
        long long thr = topk_last<KW>(wl, p.pp.k);
        for (int i = 1; i < NW; ++i)
#pragma unroll
          for (int wd = 0; wd < KW; ++wd) {
            const long long c = tks[((i * T + t) * KW + wd) * 32 + lane];
            topk_offer<KW>(wl, thr, c != LLONG_MIN, c, p.pp.k, lane);
          }
        const int kk = min(p.pp.k, ng);
        float sum = 0.f;
#pragma unroll
        for (int wd = 0; wd < KW; ++wd)
          if (wd * 32 + lane < kk) sum += act_f<ACT>(topk_value(wl[wd]));
#pragma unroll
        for (int off = 16; off; off >>= 1) sum += __shfl_xor_sync(kFullMask, sum, off);
        if (t0 + t < p.B) {
          if (lane == 0) p.pre[(int64_t)(t0 + t) * p.ldp + (g - p.g0)] = sum / (float)kk;
          if (p.winners != nullptr)
#pragma unroll
            for (int wd = 0; wd < KW; ++wd) {
              const int pos = wd * 32 + lane;
              if (pos < p.pp.k)
                p.winners[(int64_t)(t0 + t) * p.ldwin + (g - p.g0) * p.pp.k + pos] = pos < kk ? topk_slot(wl[wd]) : -1;
            }
        }
      }
      __syncthreads();
    } else {
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
        } else if constexpr (PK == PK_LSE) {
          const float o1 = __shfl_xor_sync(kFullMask, st1[t], off), o2 = __shfl_xor_sync(kFullMask, st2[t], off);
          lse_merge(acc[t], st1[t], st2[t], ov, o1, o2);
        } else if constexpr (PK == PK_POW) {
          pow_merge(acc[t], st1[t], ov, __shfl_xor_sync(kFullMask, st1[t], off), p.pp);
        } else {
          acc[t] += ov;
        }
      }
    if (lane == 0)
#pragma unroll
      for (int t = 0; t < T; ++t) {
        red[buf][warp][t] = acc[t];
        if constexpr (MAXP) redi[buf][warp][t] = wid[t];
        if constexpr (SM) {
          red1[buf][warp][t] = st1[t];
          red2[buf][warp][t] = st2[t];
        }
      }
    __syncthreads();
    if (threadIdx.x < T) {
      const int t = t0 + threadIdx.x;
      if constexpr (MAXP) {
        float m = -INFINITY;
        int wi = 0x7fffffff;
#pragma unroll
        for (int i = 0; i < NW; ++i) {
          const float v = red[buf][i][threadIdx.x];
          const int vi = redi[buf][i][threadIdx.x];
          if (v > m || (v == m && vi < wi)) {
            m = v;
            wi = vi;
          }
        }
        if (t < p.B) {
          p.pre[(int64_t)t * p.ldp + (g - p.g0)] = m;
          if (p.winners != nullptr) p.winners[(int64_t)t * p.ldwin + (g - p.g0)] = wi;
        }
      } else if constexpr (SM) {
        float m = red[buf][0][threadIdx.x], s1 = red1[buf][0][threadIdx.x], s2 = red2[buf][0][threadIdx.x];
#pragma unroll
        for (int i = 1; i < NW; ++i) {
          if constexpr (PK == PK_LSE)
            lse_merge(m, s1, s2, red[buf][i][threadIdx.x], red1[buf][i][threadIdx.x], red2[buf][i][threadIdx.x]);
          else
            pow_merge(m, s1, red[buf][i][threadIdx.x], red1[buf][i][threadIdx.x], p.pp);
        }
        float l2 = 0.f;
        const float y = pool_finalize(p.pool, m, s1, s2, ng, p.pp.param, &l2);
        if (t < p.B) {
          p.pre[(int64_t)t * p.ldp + (g - p.g0)] = y;
          if (PK == PK_LSE && p.stat != nullptr) p.stat[(int64_t)t * p.ldstat + (g - p.g0)] = l2;
        }
      } else {
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < NW; ++i) s += red[buf][i][threadIdx.x];
        if (t < p.B) p.pre[(int64_t)t * p.ldp + (g - p.g0)] = p.pool == GL_POOL_MEAN ? s / (float)ng : s;
      }
    }
    // no second barrier: the next group writes the other buffer, and a warp can write this one
    // again only after the next group's barrier, which the reducing threads reach after reading it
    }
  }
}

// Dynamic shared memory of the forward: the padded x tile, plus the top-K lists.
static int64_t mb_fwd_smem(int64_t D, int T, int pool, int k) {
  const int64_t tile = mb_smem_bytes(D, T, false);
  if (pool != GL_POOL_TOPK) return tile;
  return ((tile + 15) & ~15LL) + (int64_t)(kMbFwdThreads / 32) * T * (k > 32 ? 64 : 32) * 8;
}

template <int T, int ACT, bool PACKED, int PK>
static int mb_fwd_launch(const MbParams& p, cudaStream_t st) {
  const size_t smem = (size_t)mb_fwd_smem(p.D, T, p.pool, p.pp.k);
  const void* kern = (const void*)mb_fwd_kernel<T, ACT, PACKED, PK>;
  int rc = ensure_dynamic_smem(kern, smem);
  if (rc) return rc;
  const int64_t tiles = (p.B + T - 1) / T;
  const int64_t chunks = (p.g1 - p.g0 + p.gpc - 1) / p.gpc;
  if (tiles > 2147483647LL || chunks > 65535) return GL_ERR_SHAPE;
  mb_fwd_kernel<T, ACT, PACKED, PK><<<dim3((unsigned)tiles, (unsigned)chunks), kMbFwdThreads, smem, st>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e);
  count_launches(1);
  return GL_OK;
}

template <int T, int ACT, bool PACKED>
static int mb_fwd_pk(const MbParams& p, cudaStream_t st) {
  switch (pool_kind(p.pool, p.pp.k)) {
    case PK_MAX: return mb_fwd_launch<T, ACT, PACKED, PK_MAX>(p, st);
    case PK_TOPK:
      if constexpr (T > 4) return GL_ERR_UNSUPPORTED;
      else return mb_fwd_launch<T, ACT, PACKED, PK_TOPK>(p, st);
    case PK_TOPK64:
      if constexpr (T > 4) return GL_ERR_UNSUPPORTED;
      else return mb_fwd_launch<T, ACT, PACKED, PK_TOPK64>(p, st);
    case PK_LSE:
      if constexpr (T > 8) return GL_ERR_UNSUPPORTED;
      else return mb_fwd_launch<T, ACT, PACKED, PK_LSE>(p, st);
    case PK_POW:
      if constexpr (T > 8) return GL_ERR_UNSUPPORTED;
      else return mb_fwd_launch<T, ACT, PACKED, PK_POW>(p, st);
    default: return mb_fwd_launch<T, ACT, PACKED, PK_ADD>(p, st);
  }
}

template <int T, bool PACKED>
static int mb_fwd_act(const MbParams& p, int act, cudaStream_t st) {
  switch (act) {
    case GL_ACT_IDENTITY: return mb_fwd_pk<T, GL_ACT_IDENTITY, PACKED>(p, st);
    case GL_ACT_RELU: return mb_fwd_pk<T, GL_ACT_RELU, PACKED>(p, st);
    case GL_ACT_GELU: return mb_fwd_pk<T, GL_ACT_GELU, PACKED>(p, st);
    default: return GL_ERR_UNSUPPORTED;
  }
}

template <int T>
static int mb_dispatch(const MbParams& p, int act, bool packed, bool bwd, cudaStream_t st) {
  if (bwd) return mb_bwd_launch(p, T, act, packed, st);
  return packed ? mb_fwd_act<T, true>(p, act, st) : mb_fwd_act<T, false>(p, act, st);
}

// Largest token tile in {32, 16, 8, 4, 2, 1} whose tiles (1 forward, 2 backward) fit the opt-in shared memory.
static int mb_pick_tokens(int64_t D, bool bwd, int optin) {
  for (int T = 32; T >= 1; T >>= 1)
    if (mb_smem_bytes(D, T, bwd) + kMbStaticSmem <= optin) return T;
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
  if (a.pool < GL_POOL_MEAN || a.pool > GL_POOL_TOPK || ((a.pool == GL_POOL_MAX || a.pool == GL_POOL_TOPK) && bwd))
    return GL_ERR_UNSUPPORTED;
  if (a.pool == GL_POOL_TOPK && !topk_k_ok(a.k)) return GL_ERR_SHAPE;
  if (a.wdtype != GL_DTYPE_F32 && a.wdtype != GL_DTYPE_BF16) return GL_ERR_UNSUPPORTED;
  const bool smooth = a.pool >= GL_POOL_LME;
  if ((a.pool == GL_POOL_LME || a.pool == GL_POOL_SOFTMAX) && !(a.param > 0.f)) return GL_ERR_SHAPE;
  if (a.pool == GL_POOL_POWER && !(a.param >= 1.f)) return GL_ERR_SHAPE;
  if (bwd && smooth && (!a.c2 || (a.pool == GL_POOL_SOFTMAX && !a.c3))) return GL_ERR_NULL;
  if (a.winners && a.ldwin < (a.g1 - a.g0) * (a.pool == GL_POOL_TOPK ? a.k : 1)) return GL_ERR_SHAPE;
  if (a.stat && a.ldstat < a.g1 - a.g0) return GL_ERR_SHAPE;
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
    if (!bwd && smooth && T > 8) T = 8;  // three-word states per token in registers
    if (!bwd && a.pool == GL_POOL_TOPK && T > 4) T = 4;  // top-K lists per token in registers
  } else if (T != 1 && T != 2 && T != 4 && T != 8 && T != 16 && T != 32) {
    return GL_ERR_UNSUPPORTED;
  }
  if (mb_smem_bytes(a.D, T, bwd) + kMbStaticSmem > optin) return GL_ERR_SMEM;
  if (!bwd && a.pool == GL_POOL_TOPK) {
    while (T > 1 && mb_fwd_smem(a.D, T, a.pool, a.k) + kMbStaticSmem > optin) T >>= 1;
    if (mb_fwd_smem(a.D, T, a.pool, a.k) + kMbStaticSmem > optin) return GL_ERR_SMEM;
  }
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
  p.stat = a.stat; p.ldstat = a.ldstat; p.c2 = a.c2; p.c3 = a.c3;
  p.pp = PoolParam{a.param, pow_code(a.param), a.pool == GL_POOL_SOFTMAX, a.k};
  p.ipm1 = pow_code(a.param) >= 1 ? pow_code(a.param) - 1 : -1;
  p.wbf = a.wdtype == GL_DTYPE_BF16;
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
