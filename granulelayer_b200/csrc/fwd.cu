// Forward: fused sparse projection + activation + group pooling (Mode A, fan-in 8, fp32).
//
// Replaces the reference's Triton fwd_pool_kernel (sparse_pooling/kernels/triton_fused.py:289-358,
// Mode-A tile math at :253-264, mean update at :174-178) and the host merge
// (kernels/ops.py:182-199).  The [B, H] hidden tensor never exists: every
// z[t, n] lives in registers for the few instructions between its gathers and
// its pooled sum.
//
// Work decomposition.  A thread block owns one token tile of T tokens and a
// contiguous chunk of whole pooling groups.  It stages its token tile once in
// shared memory, feature-major (xs[d * T + t], D*T*4 bytes; 128 KiB at
// D = 4096, T = 8), then streams the groups' neuron records (16-byte index
// record, 32-byte weight row, bias) straight from HBM/L2 with 128-bit loads.
// Each warp step covers 32 / (T/4) neurons: a neuron's T tokens are split over
// T/4 lanes holding 4 tokens each, so every gather is one LDS.128 of a
// 4-token slice of the feature's row.  Lanes accumulate act(z) per token;
// the block reduces per group with warp shuffles plus one shared-memory
// pass, and writes pre[t, g] once (no atomics, deterministic).
//
// Consecutive blocks are consecutive token tiles of the same group chunk, so
// the chunk's parameters are fetched from HBM once and re-served from L2 to
// the other token tiles.
#include "common.cuh"

namespace gl {

constexpr int kFwdThreads = 512;

// PK (the pooling state, common.cuh): PK_ADD mean / sum; PK_MAX max (the largest act(z) over the
// valid slots; winner = the smallest slot attaining it, kernels/triton_fused.py:129-140, written to
// `winners`); PK_LSE LogMeanExp / softmax-weighted and PK_POW power mean (their log2-normaliser
// written to `stat`).
template <int T, int ACT, bool LOCAL, int PK, bool BF>
__global__ void __launch_bounds__(kFwdThreads, 1)
    fwd_kernel(const float* __restrict__ x, const int16_t* __restrict__ idx, const float* __restrict__ w,
               const float* __restrict__ bias, const int32_t* __restrict__ counts, float* __restrict__ pre,
               int B, int D, int64_t NB, int64_t g0, int64_t g1, int64_t ldx, int64_t ldp, int pool, int gpc,
               float* __restrict__ wabsmax, const int32_t* __restrict__ order, const LocalMap lm,
               int32_t* __restrict__ winners, int64_t ldwin, float* __restrict__ stat, int64_t ldstat,
               const PoolParam pp) {
  constexpr bool MAXP = PK == PK_MAX;
  constexpr bool SM = PK == PK_LSE || PK == PK_POW;  // three-word states
  constexpr bool TK = PK == PK_TOPK || PK == PK_TOPK64;
  constexpr int KW = PK == PK_TOPK64 ? 2 : 1;        // top-K list words per lane
  constexpr int V = T < 4 ? T : 4;   // tokens per lane
  constexpr int LPN = T / V;         // lanes per neuron
  constexpr int NPW = 32 / LPN;      // neurons per warp step
  constexpr int NW = kFwdThreads / 32;
  constexpr int UNR = 2;             // neurons in flight per lane
  extern __shared__ __align__(16) float xs[];
  __shared__ float red[NW][T];
  __shared__ int redi[MAXP ? NW : 1][T];
  __shared__ float red1[SM ? NW : 1][T], red2[SM ? NW : 1][T];
  __shared__ float redw[NW];

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int t0 = blockIdx.x * T;
  int dmax = D - 1;
  const int16_t* ridx = idx;
  if constexpr (LOCAL) {  // one group per block: stage only its features
    const int64_t gl = (int64_t)blockIdx.y * gpc;
    const int nf = min(max(__ldg(lm.nfeat + gl), 1), lm.fcap);
    stage_cols<T, kFwdThreads>(xs, x, t0, B, lm.fmap + gl * lm.fcap, nf, ldx, D);
    dmax = nf - 1;
    ridx = lm.lidx;
  } else {
    stage_tile<T, kFwdThreads>(xs, x, t0, B, D, ldx);
  }
  __syncthreads();

  const int nsub = lane / LPN, q = lane % LPN;
  const int slots = (int)(NB * 8);
  const int64_t gb = g0 + (int64_t)blockIdx.y * gpc;
  const int64_t ge = gb + gpc < g1 ? gb + gpc : g1;
  const float* xq = xs + q * V;
  // top-K: each warp's lists, then the block's merge ([NW][T][KW * 32] keys after the staged tile)
  long long* tks = reinterpret_cast<long long*>(xs + ((((LOCAL ? lm.fcap : D) * T) + 3) & ~3));

  for (int64_t g = gb; g < ge; ++g) {
    const int ng = min(counts[g], slots);
    const int64_t fbase = g * (int64_t)slots;
    float acc[V], st1[V], st2[V];  // st1, st2: the second and third words of the SM states
    int wid[V];
#pragma unroll
    for (int v = 0; v < V; ++v) {
      acc[v] = (MAXP || PK == PK_LSE) ? -INFINITY : 0.f;
      st1[v] = 0.f;
      st2[v] = 0.f;
      wid[v] = 0x7fffffff;
    }
    float wmx = 0.f;  // max |w| over the valid slots this lane reads (for the backward's fixed-point scale)
    long long tkw[TK ? T : 1][KW], tthr[TK ? T : 1];
    if constexpr (TK) {
#pragma unroll
      for (int t = 0; t < T; ++t) {
        tthr[t] = LLONG_MIN;
#pragma unroll
        for (int wd = 0; wd < KW; ++wd) tkw[t][wd] = LLONG_MIN;
      }
    }

    for (int s0 = warp * NPW * UNR; s0 < ng; s0 += NW * NPW * UNR) {
      Rec8 r[UNR];
      W8 wr[UNR];
      float bb[UNR];
      bool ok[UNR];
      int sl[UNR];
#pragma unroll
      for (int u = 0; u < UNR; ++u) {
        const int s = s0 + u * NPW + nsub;
        ok[u] = s < ng;
        int slot = ok[u] ? s : 0;
        if (order != nullptr && ok[u]) slot = min(max(__ldg(order + (g - g0) * (int64_t)slots + s), 0), slots - 1);
        const int64_t f = fbase + slot;
        sl[u] = slot;
        r[u] = load_rec8(ridx + f * 8, dmax);
        wr[u] = load_w8_any(w, f, BF);
        bb[u] = load_any(bias, f, BF);
      }
#pragma unroll
      for (int u = 0; u < UNR; ++u) {
        float z[V];
#pragma unroll
        for (int v = 0; v < V; ++v) z[v] = bb[u];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float* row = xq + r[u].i[k] * T;
          if constexpr (V == 4) {
            const float4 xv = *reinterpret_cast<const float4*>(row);
            z[0] = fmaf(wr[u].w[k], xv.x, z[0]);
            z[1] = fmaf(wr[u].w[k], xv.y, z[1]);
            z[2] = fmaf(wr[u].w[k], xv.z, z[2]);
            z[3] = fmaf(wr[u].w[k], xv.w, z[3]);
          } else if constexpr (V == 2) {
            const float2 xv = *reinterpret_cast<const float2*>(row);
            z[0] = fmaf(wr[u].w[k], xv.x, z[0]);
            z[1] = fmaf(wr[u].w[k], xv.y, z[1]);
          } else {
            z[0] = fmaf(wr[u].w[k], row[0], z[0]);
          }
        }
        if constexpr (TK) {  // every lane takes part in the warp's insertions
#pragma unroll
          for (int t = 0; t < T; ++t)
            topk_offer<KW>(tkw[t], tthr[t], ok[u] && q == t / V, topk_key(z[t % V], sl[u]), pp.k, lane);
        }
        if (ok[u] && !TK) {
#pragma unroll
          for (int v = 0; v < V; ++v) {
            const float a = act_f<ACT>(z[v]);
            if constexpr (MAXP) {
              if (a > acc[v] || (a == acc[v] && sl[u] < wid[v])) {
                acc[v] = a;
                wid[v] = sl[u];
              }
            } else if constexpr (PK == PK_LSE) {
              lse_push(acc[v], st1[v], st2[v], a * pp.param, a, pp.want_t);
            } else if constexpr (PK == PK_POW) {
              pow_push(acc[v], st1[v], st2[v], a, pp);
            } else {
              acc[v] += a;
            }
          }
#pragma unroll
          for (int k = 0; k < 8; ++k) wmx = fmaxf(wmx, fabsf(wr[u].w[k]));
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
        long long thr = topk_last<KW>(wl, pp.k);
        for (int i = 1; i < NW; ++i)
#pragma unroll
          for (int wd = 0; wd < KW; ++wd) {
            const long long c = tks[((i * T + t) * KW + wd) * 32 + lane];
            topk_offer<KW>(wl, thr, c != LLONG_MIN, c, pp.k, lane);
          }
        const int kk = min(pp.k, ng);
        float sum = 0.f;
#pragma unroll
        for (int wd = 0; wd < KW; ++wd)
          if (wd * 32 + lane < kk) sum += act_f<ACT>(topk_value(wl[wd]));
#pragma unroll
        for (int off = 16; off; off >>= 1) sum += __shfl_xor_sync(kFullMask, sum, off);
        if (t0 + t < B) {
          if (lane == 0) pre[(int64_t)(t0 + t) * ldp + (g - g0)] = sum / (float)kk;
          if (winners != nullptr)
#pragma unroll
            for (int wd = 0; wd < KW; ++wd) {
              const int pos = wd * 32 + lane;
              if (pos < pp.k)
                winners[(int64_t)(t0 + t) * ldwin + (g - g0) * pp.k + pos] = pos < kk ? topk_slot(wl[wd]) : -1;
            }
        }
      }
      __syncthreads();
    } else {
    // reduce over the neurons of the warp (lanes with equal q), then over warps
#pragma unroll
    for (int off = LPN; off < 32; off <<= 1)
#pragma unroll
      for (int v = 0; v < V; ++v) {
        const float ov = __shfl_xor_sync(kFullMask, acc[v], off);
        if constexpr (MAXP) {
          const int ow = __shfl_xor_sync(kFullMask, wid[v], off);
          if (ov > acc[v] || (ov == acc[v] && ow < wid[v])) {
            acc[v] = ov;
            wid[v] = ow;
          }
        } else if constexpr (PK == PK_LSE) {
          const float o1 = __shfl_xor_sync(kFullMask, st1[v], off), o2 = __shfl_xor_sync(kFullMask, st2[v], off);
          lse_merge(acc[v], st1[v], st2[v], ov, o1, o2);
        } else if constexpr (PK == PK_POW) {
          pow_merge(acc[v], st1[v], ov, __shfl_xor_sync(kFullMask, st1[v], off), pp);
        } else {
          acc[v] += ov;
        }
      }
    if (lane < LPN)
#pragma unroll
      for (int v = 0; v < V; ++v) {
        red[warp][lane * V + v] = acc[v];
        if constexpr (MAXP) redi[warp][lane * V + v] = wid[v];
        if constexpr (SM) {
          red1[warp][lane * V + v] = st1[v];
          red2[warp][lane * V + v] = st2[v];
        }
      }
    const bool want_w = wabsmax != nullptr && blockIdx.x == 0;
    if (want_w) {
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) wmx = fmaxf(wmx, __shfl_xor_sync(kFullMask, wmx, off));
      if (lane == 0) redw[warp] = wmx;
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
        if (t < B) {
          pre[(int64_t)t * ldp + (g - g0)] = m;
          if (winners != nullptr) winners[(int64_t)t * ldwin + (g - g0)] = wi;
        }
      } else if constexpr (SM) {
        float m = red[0][threadIdx.x], s1 = red1[0][threadIdx.x], s2 = red2[0][threadIdx.x];
#pragma unroll
        for (int i = 1; i < NW; ++i) {
          if constexpr (PK == PK_LSE) lse_merge(m, s1, s2, red[i][threadIdx.x], red1[i][threadIdx.x], red2[i][threadIdx.x]);
          else pow_merge(m, s1, red[i][threadIdx.x], red1[i][threadIdx.x], pp);
        }
        float l2 = 0.f;
        const float y = pool_finalize(pool, m, s1, s2, ng, pp.param, &l2);
        if (t < B) {
          pre[(int64_t)t * ldp + (g - g0)] = y;
          if (PK == PK_LSE && stat != nullptr) stat[(int64_t)t * ldstat + (g - g0)] = l2;
        }
      } else {
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < NW; ++i) s += red[i][threadIdx.x];
        if (t < B) pre[(int64_t)t * ldp + (g - g0)] = (pool == GL_POOL_MEAN) ? s / (float)ng : s;
      }
    }
    if (want_w && threadIdx.x == 32) {
      float m = 0.f;
#pragma unroll
      for (int i = 0; i < NW; ++i) m = fmaxf(m, redw[i]);
      wabsmax[g - g0] = m;
    }
    __syncthreads();
    }
  }
}

// Dynamic shared memory: the staged tile, plus the top-K lists ([NW][T][KW * 32] keys).
static size_t fwd_smem(int64_t rows, int T, int pool, int k) {
  const size_t tile = (size_t)((rows * T + 3) & ~3LL) * sizeof(float);
  if (pool != GL_POOL_TOPK) return (size_t)rows * T * sizeof(float);
  return tile + (size_t)(kFwdThreads / 32) * T * (k > 32 ? 64 : 32) * sizeof(long long);
}

template <int T, int ACT, bool LOCAL, int PK, bool BF>
static int launch_fwd(const GlFwdArgs& a, int gpc, cudaStream_t st) {
  const size_t smem = fwd_smem(LOCAL ? a.fcap : a.D, T, a.pool, a.k);
  auto kern = fwd_kernel<T, ACT, LOCAL, PK, BF>;
  int rc = ensure_dynamic_smem((const void*)kern, smem);
  if (rc) return rc;
  const int64_t tiles = (a.B + T - 1) / T;
  const int64_t chunks = (a.g1 - a.g0 + gpc - 1) / gpc;
  if (tiles > 2147483647LL || chunks > 65535) return GL_ERR_SHAPE;
  dim3 grid((unsigned)tiles, (unsigned)chunks);
  const LocalMap lm{a.lidx, a.fmap, a.nfeat, (int)a.fcap};
  kern<<<grid, kFwdThreads, smem, st>>>(a.x, a.idx, a.w, a.b, a.counts, a.pre, (int)a.B, (int)a.D, a.NB, a.g0,
                                        a.g1, a.ldx, a.ldp, a.pool, gpc, a.wabsmax, a.order, lm, a.winners, a.ldwin,
                                        a.stat, a.ldstat, PoolParam{a.param, pow_code(a.param),
                                                                    a.pool == GL_POOL_SOFTMAX, a.k});
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e);
  count_launches(1);
  return GL_OK;
}

template <int T, bool LOCAL, int PK, bool BF>
static int dispatch_act_fwd2(const GlFwdArgs& a, int gpc, cudaStream_t st) {
  switch (a.act) {
    case GL_ACT_IDENTITY: return launch_fwd<T, GL_ACT_IDENTITY, LOCAL, PK, BF>(a, gpc, st);
    case GL_ACT_RELU: return launch_fwd<T, GL_ACT_RELU, LOCAL, PK, BF>(a, gpc, st);
    case GL_ACT_GELU: return launch_fwd<T, GL_ACT_GELU, LOCAL, PK, BF>(a, gpc, st);
    default: return GL_ERR_UNSUPPORTED;
  }
}

template <int T, bool LOCAL, bool BF>
static int dispatch_pk_fwd(const GlFwdArgs& a, int gpc, cudaStream_t st) {
  switch (pool_kind(a.pool, a.k)) {
    case PK_MAX: return dispatch_act_fwd2<T, LOCAL, PK_MAX, BF>(a, gpc, st);
    case PK_TOPK:
      if constexpr (LOCAL || T > 4) return GL_ERR_UNSUPPORTED;
      else return dispatch_act_fwd2<T, false, PK_TOPK, BF>(a, gpc, st);
    case PK_TOPK64:
      if constexpr (LOCAL || T > 4) return GL_ERR_UNSUPPORTED;
      else return dispatch_act_fwd2<T, false, PK_TOPK64, BF>(a, gpc, st);
    case PK_LSE:
      if constexpr (LOCAL) return GL_ERR_UNSUPPORTED;
      else return dispatch_act_fwd2<T, false, PK_LSE, BF>(a, gpc, st);
    case PK_POW:
      if constexpr (LOCAL) return GL_ERR_UNSUPPORTED;
      else return dispatch_act_fwd2<T, false, PK_POW, BF>(a, gpc, st);
    default: return dispatch_act_fwd2<T, LOCAL, PK_ADD, BF>(a, gpc, st);
  }
}

// The smooth pools (LSE, POW kinds) and top-K run on the full-row staging only (no locality maps);
// top-K tiles hold at most 4 tokens (its lists live in registers).  bf16 storage is compiled for
// the full-row staging (the storage type is a template parameter: no per-load branch).
template <int T, bool LOCAL>
static int dispatch_act_fwd(const GlFwdArgs& a, int gpc, cudaStream_t st) {
  if (a.wdtype == GL_DTYPE_BF16) {
    if constexpr (LOCAL) return GL_ERR_UNSUPPORTED;
    else return dispatch_pk_fwd<T, false, true>(a, gpc, st);
  }
  return dispatch_pk_fwd<T, LOCAL, false>(a, gpc, st);
}

// Bound on the forward kernel's static shared memory (its reduction buffers).
constexpr int kFwdStaticSmem = 9216;

// Largest token tile in {tmax, ..., 2, 1} whose staged input (D rows) fits the opt-in shared
// memory (leaving room for the static reduction buffers).  tmax is 8 for the full input row and
// 32 for a group's feature map.
static int pick_fwd_tokens(int64_t D, int smem_optin, int tmax = 8) {
  for (int T = tmax; T >= 1; T >>= 1)
    if ((int64_t)D * T * 4 + kFwdStaticSmem <= smem_optin) return T;
  return GL_ERR_SMEM;
}

}  // namespace gl

using namespace gl;

extern "C" int gl_fwd_auto_tokens(int64_t D) {
  int optin = 0;
  int rc = device_smem_optin(&optin);
  if (rc) return rc;
  return pick_fwd_tokens(D, optin);
}

extern "C" int gl_fwd_f32(const GlFwdArgs* args, void* stream) {
  if (!args) return GL_ERR_NULL;
  const GlFwdArgs& a = *args;
  if (a.B < 0 || a.D < 1 || a.D > 32767 || a.NB < 1 || a.g0 < 0 || a.g1 < a.g0) return GL_ERR_SHAPE;
  if (a.B == 0 || a.g1 == a.g0) return GL_OK;
  if (!a.x || !a.idx || !a.w || !a.b || !a.counts || !a.pre) return GL_ERR_NULL;
  if (a.B > 2147483647LL || a.ldx < a.D || a.ldp < a.g1 - a.g0) return GL_ERR_SHAPE;
  if (((uintptr_t)a.idx & 15) || ((uintptr_t)a.w & 15)) return GL_ERR_ALIGN;
  if (a.pool < GL_POOL_MEAN || a.pool > GL_POOL_TOPK) return GL_ERR_UNSUPPORTED;
  if (a.wdtype != GL_DTYPE_F32 && a.wdtype != GL_DTYPE_BF16) return GL_ERR_UNSUPPORTED;
  if (a.pool == GL_POOL_TOPK && !topk_k_ok(a.k)) return GL_ERR_SHAPE;
  if ((a.pool == GL_POOL_LME || a.pool == GL_POOL_SOFTMAX) && !(a.param > 0.f)) return GL_ERR_SHAPE;
  if (a.pool == GL_POOL_POWER && !(a.param >= 1.f)) return GL_ERR_SHAPE;
  if (a.winners && a.ldwin < (a.g1 - a.g0) * (a.pool == GL_POOL_TOPK ? a.k : 1)) return GL_ERR_SHAPE;
  if (a.stat && a.ldstat < a.g1 - a.g0) return GL_ERR_SHAPE;
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
  int T = a.tokens;
  if (T == 0) {
    T = pick_fwd_tokens(rows, optin, local ? 32 : (a.pool == GL_POOL_TOPK ? 4 : 8));
    if (T < 0) return T;
  } else if (T != 1 && T != 2 && T != 4 && T != 8 && T != 16 && T != 32) {
    return GL_ERR_UNSUPPORTED;
  }
  if ((int64_t)fwd_smem(rows, T, a.pool, a.k) + kFwdStaticSmem > optin) {
    if (a.tokens != 0) return GL_ERR_SMEM;
    while (T > 1 && (int64_t)fwd_smem(rows, T, a.pool, a.k) + kFwdStaticSmem > optin) T >>= 1;
    if ((int64_t)fwd_smem(rows, T, a.pool, a.k) + kFwdStaticSmem > optin) return GL_ERR_SMEM;
  }
  const int64_t G = a.g1 - a.g0;
  int gpc = local ? 1 : a.groups_per_cta;
  if (gpc <= 0) {
    const int64_t tiles = (a.B + T - 1) / T;
    const int64_t units = tiles * G;
    int64_t want = units / ((int64_t)sms * 32);
    gpc = (int)(want < 1 ? 1 : (want > 8 ? 8 : want));
  }
  while ((G + gpc - 1) / gpc > 65535) gpc *= 2;
  cudaStream_t st = (cudaStream_t)stream;
  if (local) {
    switch (T) {
      case 32: return dispatch_act_fwd<32, true>(a, gpc, st);
      case 16: return dispatch_act_fwd<16, true>(a, gpc, st);
      case 8: return dispatch_act_fwd<8, true>(a, gpc, st);
      case 4: return dispatch_act_fwd<4, true>(a, gpc, st);
      case 2: return dispatch_act_fwd<2, true>(a, gpc, st);
      default: return dispatch_act_fwd<1, true>(a, gpc, st);
    }
  }
  switch (T) {
    case 32: return dispatch_act_fwd<32, false>(a, gpc, st);
    case 16: return dispatch_act_fwd<16, false>(a, gpc, st);
    case 8: return dispatch_act_fwd<8, false>(a, gpc, st);
    case 4: return dispatch_act_fwd<4, false>(a, gpc, st);
    case 2: return dispatch_act_fwd<2, false>(a, gpc, st);
    default: return dispatch_act_fwd<1, false>(a, gpc, st);
  }
}
