// Mode B with bf16 parameters, backward of the mean and sum pools on the tensor cores (operand path in
// modeb_tc.cuh).
//
// Replaces the reference's bf16 Mode-B backward (sparse_pooling/kernels/cuda/sparse_pool_bwd.cuh:387-876)
// with its default "split" gradient precision: dz is carried as the sum of two bf16 values (hi + lo,
// 16 significant bits), so the products dz * w and dz * x are accumulated in fp32 from exact terms.
// With c1[t, g] = gpre[t, g - g0] / counts[g] (mean) or gpre (sum) and x rounded to bf16:
//   dz[t, s] = c1[t, g] * act'(z[t, s])                 (0 for padding slots)
//   dx[t, d] += sum_{s, k: idx_k(s) = d} dz[t, s] * w[s][k]
//   dw[s][k] += sum_t dz[t, s] * x[t, idx_k(s)]       db[s] += sum_t dz[t, s]
// dw and db are the fp32 gradients in the fragment-packed layout (the reference's main_grad).
//
// A CTA owns BM tokens (the bf16 x slab and an fp32 dX tile, both in shared memory) and a chunk of
// whole groups; a warp takes fragment quads (32 slots) in turn.  Per quad and 16-token m-tile:
//   z   = mma(x fragments, w) + bias                  (m16n8k8, as the forward)
//   dz  from the accumulator fragments, split into hi + lo bf16 pairs
//   P   = dz w^T (m16n8k8: the dz accumulator fragments are already A fragments; w^T fragments come
//         from the packed w by movmatrix.trans), added to the dX tile with shared-memory atomics
//   dW += dz^T x (m16n8k16: A = dz^T and B = x^T by movmatrix.trans of fragments held in registers);
//         the result fragment of lane l is exactly the lane's slice of the packed dw layout
//   db += sum over the tile's tokens (lane-quad shuffles)
// and once per quad and tile the lane adds its 8 dw values (and lanes 0-3 their 8 db values) with two
// 16-byte global reductions.  The dX tile is added to dx once per CTA.
#include "modeb_tc_bwd.cuh"

namespace gl {

// FIXED: the dX tile holds int32 fixed-point sums (shared int32 atomics run at 2.4x the rate of fp32
// ones on B200).  Per group and token the partials are scaled by a power of two s with
// m_g * C * |c1[t, g]| * max|w|_g * max|act'| * s <= 2^30 (m_g = the group's largest number of record
// inputs on one feature), so no tile word can overflow within the group; the tile is added to dx
// (times 1 / s) and cleared after every group.  A token with a non-finite bound gets NaN in dx.
template <int BM, int NT, int ACT, bool FIXED>
__global__ void __launch_bounds__(kTcBwdThreads, 1) tc_bwd_kernel(const TcParams p) {
  constexpr int MT = BM / 16;
  constexpr int NW = kTcBwdThreads / 32;
  extern __shared__ __align__(128) unsigned char tc_smem[];
  float* dxs = reinterpret_cast<float*>(tc_smem + (size_t)p.D * BM * 2);
  int* dxi = reinterpret_cast<int*>(dxs);  // the same tile, in fixed point
  __shared__ float qsc[2][FIXED ? BM : 1], qinv[2][FIXED ? BM : 1];  // per-group scales, by group parity
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int t0 = blockIdx.x * BM;
  const uint32_t slab = (uint32_t)__cvta_generic_to_shared(tc_smem);
  tc_stage<BM, kTcBwdThreads>(slab, p.x, t0, p.B, p.D, p.ldx);
  for (int i = threadIdx.x; i < p.D * BM; i += kTcBwdThreads) dxs[i] = 0.f;
  __syncthreads();
  const int slots = (int)(p.NB * p.C);
  const int64_t gb = p.g0 + (int64_t)blockIdx.y * p.gpc;
  const int64_t ge = gb + p.gpc < p.g1 ? gb + p.gpc : p.g1;
  for (int64_t g = gb; g < ge; ++g) {
    const int ng = min(p.counts[g], slots);
    const int nq = (ng + 31) >> 5;
    float sc[MT][2];
    if constexpr (FIXED) {
      const int buf = (int)((g - gb) & 1);
      if (threadIdx.x < BM) {
        const int t = t0 + threadIdx.x;
        const float gv = t < p.B ? __ldg(p.gpre + (int64_t)t * p.ldg + (g - p.g0)) : 0.f;
        const float cv = p.pool == GL_POOL_MEAN ? gv / (float)ng : gv;
        const float bound = fabsf(cv) * (float)p.C * (float)__ldg(p.rowmax + (g - p.g0)) *
                            __ldg(p.wabsmax + (g - p.g0)) * (ACT == GL_ACT_GELU ? 1.13f : 1.f);
        float s_ = 0.f, i_ = 0.f;  // a group without valid slots contributes nothing
        if (ng == 0) {
        } else if (!(bound <= 3.0e38f)) {
          i_ = __int_as_float(0x7fc00000);  // non-finite bound: NaN for the token's dx
        } else if (bound > 0.f) {
          const int e = min(max(30 - ilogbf(bound) - 1, -126), 126);
          s_ = ldexpf(1.f, e);
          i_ = ldexpf(1.f, -e);
        }
        qsc[buf][threadIdx.x] = s_;
        qinv[buf][threadIdx.x] = i_;
      }
      __syncthreads();  // scales visible; the previous group's flush has ended everywhere
#pragma unroll
      for (int m = 0; m < MT; ++m)
#pragma unroll
        for (int h = 0; h < 2; ++h) sc[m][h] = qsc[buf][16 * m + 8 * h + (lane >> 2)];
    }
    // c1 of the lane's token rows: 16 m + 8 h + lane / 4
    float c1[MT][2];
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int t = t0 + 16 * m + 8 * h + (lane >> 2);
        const float gv = t < p.B ? __ldg(p.gpre + (int64_t)t * p.ldg + (g - p.g0)) : 0.f;
        c1[m][h] = p.pool == GL_POOL_MEAN ? gv / (float)ng : gv;
      }
    TcQuad nxt;
    if (warp < nq) nxt = tc_load_quad<NT>(p, g, warp, lane);
    for (int q = warp; q < nq; q += NW) {
      const TcQuad cur = nxt;
      if (q + NW < nq) nxt = tc_load_quad<NT>(p, g, q + NW, lane);
      tc_bwd_quad<BM, NT, ACT, FIXED, false>(p, g, q, ng, cur, c1, sc, slab, dxs, dxi, nullptr, lane);
    }
    if constexpr (FIXED) {
      // dx[t0 + t, d] += q / s[t], and clear the tile for the next group
      const int buf = (int)((g - gb) & 1);
      __syncthreads();
      for (int i = threadIdx.x; i < p.D * BM; i += kTcBwdThreads) {
        const int t = i / p.D, d = i - t * p.D;
        const int o = dxs_off<BM>(d, t);
        const int qv = dxi[o];
        const float inv = qinv[buf][t];
        if (t0 + t < p.B && (qv != 0 || inv != inv)) atomicAdd(p.dx + (int64_t)(t0 + t) * p.lddx + d, (float)qv * inv);
        dxi[o] = 0;
      }
    }
  }
  if constexpr (!FIXED) {
    __syncthreads();
    // dx[t0 + t, d] += tile; consecutive threads take consecutive features of one token row
    for (int i = threadIdx.x; i < p.D * BM; i += kTcBwdThreads) {
      const int t = i / p.D, d = i - t * p.D;
      const float v = dxs[dxs_off<BM>(d, t)];
      if (t0 + t < p.B && v != 0.f) atomicAdd(p.dx + (int64_t)(t0 + t) * p.lddx + d, v);
    }
  }
}

static int64_t tc_bwd_smem(int64_t D, int BM) { return D * BM * 2 + D * BM * 4; }

template <int BM, int NT, int ACT, bool FIXED>
static int tc_bwd_launch(const TcParams& p, cudaStream_t st) {
  const size_t smem = (size_t)tc_bwd_smem(p.D, BM);
  const void* kern = (const void*)tc_bwd_kernel<BM, NT, ACT, FIXED>;
  int rc = ensure_dynamic_smem(kern, smem);
  if (rc) return rc;
  const int64_t tiles = (p.B + BM - 1) / BM;
  const int64_t chunks = (p.g1 - p.g0 + p.gpc - 1) / p.gpc;
  if (tiles > 2147483647LL || chunks > 65535) return GL_ERR_SHAPE;
  tc_bwd_kernel<BM, NT, ACT, FIXED><<<dim3((unsigned)tiles, (unsigned)chunks), kTcBwdThreads, smem, st>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e);
  count_launches(1);
  return GL_OK;
}

template <int BM, int NT, bool FIXED>
static int tc_bwd_act2(const TcParams& p, int act, cudaStream_t st) {
  switch (act) {
    case GL_ACT_IDENTITY: return tc_bwd_launch<BM, NT, GL_ACT_IDENTITY, FIXED>(p, st);
    case GL_ACT_RELU: return tc_bwd_launch<BM, NT, GL_ACT_RELU, FIXED>(p, st);
    case GL_ACT_GELU: return tc_bwd_launch<BM, NT, GL_ACT_GELU, FIXED>(p, st);
    default: return GL_ERR_UNSUPPORTED;
  }
}

template <int BM, int NT>
static int tc_bwd_act(const TcParams& p, int act, cudaStream_t st) {
  return p.wabsmax != nullptr ? tc_bwd_act2<BM, NT, true>(p, act, st) : tc_bwd_act2<BM, NT, false>(p, act, st);
}

template <int BM>
static int tc_bwd_nt(const TcParams& p, int act, cudaStream_t st) {
  switch (p.C) {
    case 8: return tc_bwd_act<BM, 1>(p, act, st);
    case 16: return tc_bwd_act<BM, 2>(p, act, st);
    case 32: return tc_bwd_act<BM, 4>(p, act, st);
    default: return tc_bwd_act<BM, 8>(p, act, st);
  }
}

int tc_prepare(const GlSharedArgs& a, bool bwd, TcParams& p);
int tc_pick_tokens(int64_t D, int optin);

// Largest token tile in {32, 16} whose slab and dX tile fit the opt-in shared memory.
int tc_bwd_pick_tokens(int64_t D, int optin) {
  for (int BM = 32; BM >= 16; BM >>= 1)
    if (tc_bwd_smem(D, BM) + kTcStaticSmem <= optin) return BM;
  return GL_ERR_SMEM;
}

}  // namespace gl

using namespace gl;

extern "C" int gl_bwd_shared_tc(const GlSharedArgs* args, const float* wabsmax, const int32_t* rowmax,
                                void* stream) {
  if (!args) return GL_ERR_NULL;
  const GlSharedArgs& a = *args;
  if ((wabsmax == nullptr) != (rowmax == nullptr)) return GL_ERR_NULL;
  TcParams p;
  int rc = tc_prepare(a, true, p);
  if (rc) return rc > 0 ? GL_OK : rc;
  p.wabsmax = wabsmax;
  p.rowmax = rowmax;
  int optin = 0, sms = 0;
  if ((rc = device_smem_optin(&optin))) return rc;
  if ((rc = device_sm_count(&sms))) return rc;
  int BM = a.tokens;
  if (BM == 0) {
    BM = tc_bwd_pick_tokens(a.D, optin);
    if (BM < 0) return BM;
  } else if (BM != 16 && BM != 32) {
    return GL_ERR_UNSUPPORTED;
  }
  if (tc_bwd_smem(a.D, BM) + kTcStaticSmem > optin) return GL_ERR_SMEM;
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
  return BM == 32 ? tc_bwd_nt<32>(p, a.act, st) : tc_bwd_nt<16>(p, a.act, st);
}

extern "C" int gl_shared_tc_auto_tokens(int64_t D, int32_t backward) {
  int optin = 0;
  const int rc = gl::device_smem_optin(&optin);
  if (rc) return rc;
  if (D < 1 || D > 32767) return GL_ERR_SHAPE;
  return backward ? gl::tc_bwd_pick_tokens(D, optin) : gl::tc_pick_tokens(D, optin);
}
