// Mode B with bf16 parameters, forward on the tensor cores (operand path in modeb_tc.cuh).
//
// Replaces the reference's bf16 Mode-B forward (sparse_pooling/kernels/cuda/sparse_pool_fwd.cuh:311,
// entry sparse_pool.cu:12-44) for the mean, sum and max pools on fragment-packed storage:
//   z[t, g, j, c] = b[g][j][c] + sum_k w[g][j][c][k] * bf16(x[t, idx[g][j][k]])
//   pre[t, g] = pool over the valid slots s = j C + c < counts[g] of act(z)
// Max keeps the smallest slot among equal maxima (kernels/triton_fused.py:129-140).
//
// A CTA owns BM tokens (the bf16 slab) and a chunk of whole groups.  A warp takes fragment quads
// (32 consecutive slots) of the current group in turn: one ldmatrix gather per record and 32
// tokens, one mma per n-tile and 16 tokens, then act and the pool on the accumulator fragments.
// The lane's partial of a token row is folded over the lane quad with two shuffles, over the
// warps through shared memory (double-buffered by group: one barrier per group), and pre[t, g]
// is written once (deterministic).
#include <type_traits>

#include "modeb_tc.cuh"

namespace gl {

template <int BM, int NT, int ACT, bool MAXP>
__global__ void __launch_bounds__(kTcFwdThreads, 1) tc_fwd_kernel(const TcParams p) {
  constexpr int NW = kTcFwdThreads / 32;
  constexpr int MT = BM / 16;
  extern __shared__ __align__(128) unsigned char tc_smem[];
  __shared__ float red[2][NW][BM];
  __shared__ int redi[2][MAXP ? NW : 1][BM];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int t0 = blockIdx.x * BM;
  const uint32_t slab = (uint32_t)__cvta_generic_to_shared(tc_smem);
  tc_stage<BM, kTcFwdThreads>(slab, p.x, t0, p.B, p.D, p.ldx);
  __syncthreads();
  const int slots = (int)(p.NB * p.C);
  const int64_t gb = p.g0 + (int64_t)blockIdx.y * p.gpc;
  const int64_t ge = gb + p.gpc < p.g1 ? gb + p.gpc : p.g1;
  const int cq = 2 * (lane & 3);  // the lane's first accumulator column within an n-tile
  for (int64_t g = gb; g < ge; ++g) {
    const int ng = min(p.counts[g], slots);
    const int nq = (ng + 31) >> 5;  // quads holding a valid slot
    const int buf = (int)((g - gb) & 1);
    float acc[MT][2];
    int wid[MAXP ? MT : 1][2];
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        acc[m][h] = MAXP ? -INFINITY : 0.f;
        if constexpr (MAXP) wid[m][h] = 0x7fffffff;
      }
    TcQuad nxt;
    if (warp < nq) nxt = tc_load_quad<NT>(p, g, warp, lane);
    for (int q = warp; q < nq; q += NW) {
      const TcQuad cur = nxt;
      if (q + NW < nq) nxt = tc_load_quad<NT>(p, g, q + NW, lane);
      // all quads but a group's last are full: the sum pools' epilogue is compiled without the slot masks
      auto quad = [&](auto masked) {
        constexpr bool MK = decltype(masked)::value;
        uint32_t a[MT][2];
#pragma unroll
        for (int fi = 0; fi < 4; ++fi) {
          if (NT >= 4 ? fi == 0 : fi % NT == 0)
            tc_gather<BM>(a, slab, tc_row<NT>(cur, NT >= 4 ? 0 : fi / NT, lane), lane);
          const uint32_t bw = tc_word(cur.w, fi), bb = tc_word(cur.b, fi);
          const float b0 = bf16_lo(bb), b1 = bf16_hi(bb);
          const int s0 = 32 * q + 8 * fi + cq;  // slots of the lane's two columns: s0, s0 + 1
          const bool v0 = !MK || s0 < ng, v1 = !MK || s0 + 1 < ng;
#pragma unroll
          for (int m = 0; m < MT; ++m) {
            float d[4];
            const float c[4] = {b0, b1, b0, b1};
            mma_bf16_k8(d, a[m], bw, c);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const float e0 = act_f<ACT>(d[2 * h]), e1 = act_f<ACT>(d[2 * h + 1]);
              if constexpr (MAXP) {
                // a lane meets its slots in increasing order: a strict compare keeps the smallest
                if (v0 && e0 > acc[m][h]) { acc[m][h] = e0; wid[m][h] = s0; }
                if (v1 && e1 > acc[m][h]) { acc[m][h] = e1; wid[m][h] = s0 + 1; }
              } else if constexpr (MK) {
                acc[m][h] += (v0 ? e0 : 0.f) + (v1 ? e1 : 0.f);
              } else {
                acc[m][h] += e0 + e1;
              }
            }
          }
        }
      };
      if constexpr (MAXP) {
        quad(std::true_type{});  // max: one body (measured faster than two at 168 registers)
      } else {
        if (32 * q + 32 <= ng) quad(std::false_type{});
        else quad(std::true_type{});
      }
    }
    // fold the lane quad (the four lanes holding one token row), then the warps
#pragma unroll
    for (int off = 1; off <= 2; off <<= 1)
#pragma unroll
      for (int m = 0; m < MT; ++m)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const float ov = __shfl_xor_sync(kFullMask, acc[m][h], off);
          if constexpr (MAXP) {
            const int ow = __shfl_xor_sync(kFullMask, wid[m][h], off);
            if (ov > acc[m][h] || (ov == acc[m][h] && ow < wid[m][h])) {
              acc[m][h] = ov;
              wid[m][h] = ow;
            }
          } else {
            acc[m][h] += ov;
          }
        }
    if ((lane & 3) == 0)
#pragma unroll
      for (int m = 0; m < MT; ++m)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int t = 16 * m + 8 * h + (lane >> 2);
          red[buf][warp][t] = acc[m][h];
          if constexpr (MAXP) redi[buf][warp][t] = wid[m][h];
        }
    __syncthreads();
    if (threadIdx.x < BM) {
      const int t = t0 + threadIdx.x;
      if constexpr (MAXP) {
        float mv = -INFINITY;
        int wi = 0x7fffffff;
#pragma unroll
        for (int i = 0; i < NW; ++i) {
          const float v = red[buf][i][threadIdx.x];
          const int vi = redi[buf][i][threadIdx.x];
          if (v > mv || (v == mv && vi < wi)) {
            mv = v;
            wi = vi;
          }
        }
        if (t < p.B) {
          p.pre[(int64_t)t * p.ldp + (g - p.g0)] = mv;
          if (p.winners != nullptr) p.winners[(int64_t)t * p.ldwin + (g - p.g0)] = wi;
        }
      } else {
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < NW; ++i) s += red[buf][i][threadIdx.x];
        if (t < p.B) p.pre[(int64_t)t * p.ldp + (g - p.g0)] = p.pool == GL_POOL_MEAN ? s / (float)ng : s;
      }
    }
    // no second barrier: the next group writes the other buffer (as in modeb.cu)
  }
}

static int64_t tc_slab_bytes(int64_t D, int BM) { return D * BM * 2; }

template <int BM, int NT, int ACT, bool MAXP>
static int tc_fwd_launch(const TcParams& p, cudaStream_t st) {
  const size_t smem = (size_t)tc_slab_bytes(p.D, BM);
  const void* kern = (const void*)tc_fwd_kernel<BM, NT, ACT, MAXP>;
  int rc = ensure_dynamic_smem(kern, smem);
  if (rc) return rc;
  const int64_t tiles = (p.B + BM - 1) / BM;
  const int64_t chunks = (p.g1 - p.g0 + p.gpc - 1) / p.gpc;
  if (tiles > 2147483647LL || chunks > 65535) return GL_ERR_SHAPE;
  tc_fwd_kernel<BM, NT, ACT, MAXP><<<dim3((unsigned)tiles, (unsigned)chunks), kTcFwdThreads, smem, st>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e);
  count_launches(1);
  return GL_OK;
}

template <int BM, int NT, bool MAXP>
static int tc_fwd_act(const TcParams& p, int act, cudaStream_t st) {
  switch (act) {
    case GL_ACT_IDENTITY: return tc_fwd_launch<BM, NT, GL_ACT_IDENTITY, MAXP>(p, st);
    case GL_ACT_RELU: return tc_fwd_launch<BM, NT, GL_ACT_RELU, MAXP>(p, st);
    case GL_ACT_GELU: return tc_fwd_launch<BM, NT, GL_ACT_GELU, MAXP>(p, st);
    default: return GL_ERR_UNSUPPORTED;
  }
}

template <int BM>
static int tc_fwd_nt(const TcParams& p, int act, cudaStream_t st) {
  const bool mx = p.pool == GL_POOL_MAX;
  switch (p.C) {
    case 8: return mx ? tc_fwd_act<BM, 1, true>(p, act, st) : tc_fwd_act<BM, 1, false>(p, act, st);
    case 16: return mx ? tc_fwd_act<BM, 2, true>(p, act, st) : tc_fwd_act<BM, 2, false>(p, act, st);
    case 32: return mx ? tc_fwd_act<BM, 4, true>(p, act, st) : tc_fwd_act<BM, 4, false>(p, act, st);
    default: return mx ? tc_fwd_act<BM, 8, true>(p, act, st) : tc_fwd_act<BM, 8, false>(p, act, st);
  }
}

// Largest token tile in {64, 32, 16} whose bf16 slab fits the opt-in shared memory.
int tc_pick_tokens(int64_t D, int optin) {
  for (int BM = 64; BM >= 16; BM >>= 1)
    if (tc_slab_bytes(D, BM) + kTcStaticSmem <= optin) return BM;
  return GL_ERR_SMEM;
}

// Checks shared by the forward and backward entry points; fills p.
int tc_prepare(const GlSharedArgs& a, bool bwd, TcParams& p) {
  if (a.B < 0 || a.D < 1 || a.D > 32767 || a.NB < 1 || a.g0 < 0 || a.g1 < a.g0) return GL_ERR_SHAPE;
  if (a.C != 8 && a.C != 16 && a.C != 32 && a.C != 64) return GL_ERR_SHAPE;
  if (!a.packed || a.wdtype != GL_DTYPE_BF16) return GL_ERR_UNSUPPORTED;
  if ((a.NB * (a.C / 8)) % 4 || ((a.C / 8) < 4 && a.NB % (4 / (a.C / 8)))) return GL_ERR_SHAPE;
  if (a.act < GL_ACT_IDENTITY || a.act > GL_ACT_GELU) return GL_ERR_UNSUPPORTED;
  if (bwd ? (a.pool != GL_POOL_MEAN && a.pool != GL_POOL_SUM)
          : (a.pool != GL_POOL_MEAN && a.pool != GL_POOL_SUM && a.pool != GL_POOL_MAX))
    return GL_ERR_UNSUPPORTED;
  if (a.B == 0 || a.g1 == a.g0) return 1;  // nothing to do
  if (!a.x || !a.idx || !a.w || !a.b || !a.counts) return GL_ERR_NULL;
  if (a.B > 2147483647LL || a.ldx < a.D || a.NB * a.C > 2147483647LL) return GL_ERR_SHAPE;
  if (((uintptr_t)a.idx & 15) || ((uintptr_t)a.w & 15) || ((uintptr_t)a.b & 15)) return GL_ERR_ALIGN;
  if (!bwd) {
    if (!a.pre) return GL_ERR_NULL;
    if (a.ldp < a.g1 - a.g0) return GL_ERR_SHAPE;
    if (a.winners && a.ldwin < a.g1 - a.g0) return GL_ERR_SHAPE;
  } else {
    if (!a.gpre || !a.dx || !a.dw || !a.db) return GL_ERR_NULL;
    if (a.ldg < a.g1 - a.g0 || a.lddx < a.D) return GL_ERR_SHAPE;
    if (((uintptr_t)a.dw & 15) || ((uintptr_t)a.db & 15)) return GL_ERR_ALIGN;
  }
  p = TcParams{};
  p.x = a.x; p.idx = a.idx; p.counts = a.counts; p.pre = a.pre; p.gpre = a.gpre;
  p.w = reinterpret_cast<const uint16_t*>(a.w);
  p.b = reinterpret_cast<const uint16_t*>(a.b);
  p.dx = a.dx; p.dw = a.dw; p.db = a.db; p.winners = a.pool == GL_POOL_MAX ? a.winners : nullptr;
  p.B = (int)a.B; p.D = (int)a.D; p.C = (int)a.C;
  p.NB = a.NB; p.g0 = a.g0; p.g1 = a.g1; p.ldx = a.ldx; p.ldp = a.ldp; p.ldg = a.ldg; p.lddx = a.lddx;
  p.ldwin = a.ldwin; p.pool = a.pool;
  return GL_OK;
}

}  // namespace gl

using namespace gl;

extern "C" int gl_fwd_shared_tc(const GlSharedArgs* args, void* stream) {
  if (!args) return GL_ERR_NULL;
  const GlSharedArgs& a = *args;
  TcParams p;
  int rc = tc_prepare(a, false, p);
  if (rc) return rc > 0 ? GL_OK : rc;
  int optin = 0, sms = 0;
  if ((rc = device_smem_optin(&optin))) return rc;
  if ((rc = device_sm_count(&sms))) return rc;
  int BM = a.tokens;
  if (BM == 0) {
    BM = tc_pick_tokens(a.D, optin);
    if (BM < 0) return BM;
  } else if (BM != 16 && BM != 32 && BM != 64) {
    return GL_ERR_UNSUPPORTED;
  }
  if (tc_slab_bytes(a.D, BM) + kTcStaticSmem > optin) return GL_ERR_SMEM;
  const int64_t G = a.g1 - a.g0;
  int gpc = a.groups_per_cta;
  if (gpc <= 0) {
    const int64_t units = ((a.B + BM - 1) / BM) * G;
    const int64_t want = units / ((int64_t)sms * 32);
    gpc = (int)(want < 1 ? 1 : (want > 8 ? 8 : want));
  }
  while ((G + gpc - 1) / gpc > 65535) gpc *= 2;
  p.gpc = gpc;
  cudaStream_t st = (cudaStream_t)stream;
  switch (BM) {
    case 64: return tc_fwd_nt<64>(p, a.act, st);
    case 32: return tc_fwd_nt<32>(p, a.act, st);
    default: return tc_fwd_nt<16>(p, a.act, st);
  }
}
