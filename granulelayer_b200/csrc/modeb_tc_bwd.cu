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
#include "modeb_tc.cuh"

namespace gl {

constexpr int kTcBwdThreads = 384;

__device__ __forceinline__ uint32_t movt(uint32_t a) {
  uint32_t d;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(a));
  return d;
}

// d = a (16x16 bf16, row) * b (16x8 bf16, col) + c, fp32 accumulation.
__device__ __forceinline__ void mma_bf16_k16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1,
                                             const float (&c)[4]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%10, %11, %12, %13};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "f"(c[0]), "f"(c[1]), "f"(c[2]),
        "f"(c[3]));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// dz pair (v0, v1) as hi + lo bf16 pairs: hi = bf16(v), lo = bf16(v - hi).
__device__ __forceinline__ void split2(float v0, float v1, uint32_t& hi, uint32_t& lo) {
  hi = pack_bf16(v0, v1);
  lo = pack_bf16(v0 - bf16_lo(hi), v1 - bf16_hi(hi));
}

__device__ __forceinline__ void red_v4(float* p, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}

// fp32 dX tile [D][BM]: element (d, t) at d * BM + (t ^ (d & (BM - 1))), so that a column read for
// the flush (consecutive d) and the scatter's 8-token runs spread over the banks.
template <int BM>
__device__ __forceinline__ int dxs_off(int d, int t) {
  return d * BM + (t ^ (d & (BM - 1)));
}

// FIXED: the dX tile holds int32 fixed-point sums (shared int32 atomics run at 2.4x the rate of fp32
// ones on B200).  Per group and token the partials are scaled by a power of two s with
// m_g * C * |c1[t, g]| * max|w|_g * max|act'| * s <= 2^30 (m_g = the group's largest number of record
// inputs on one feature), so no tile word can overflow within the group; the tile is added to dx
// (times 1 / s) and cleared after every group.  A token with a non-finite bound gets NaN in dx.
template <int BM, int NT, int ACT, bool FIXED>
__global__ void __launch_bounds__(kTcBwdThreads, 1) tc_bwd_kernel(const TcParams p) {
  constexpr int MT = BM / 16;
  constexpr int NW = kTcBwdThreads / 32;
  constexpr int R = NT < 4 ? 4 / NT : 1;      // records per quad
  constexpr int NPR = NT < 4 ? NT : 4;        // n-tiles per record within a quad
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
  const int64_t Q = p.NB * NT / 4;
  const int64_t gb = p.g0 + (int64_t)blockIdx.y * p.gpc;
  const int64_t ge = gb + p.gpc < p.g1 ? gb + p.gpc : p.g1;
  const int cq = 2 * (lane & 3);
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
      const bool full = 32 * q + 32 <= ng;
      uint32_t wt[4];
#pragma unroll
      for (int fi = 0; fi < 4; ++fi) wt[fi] = movt(tc_word(cur.w, fi));
      float dwa[4][2], dba[4][2];
#pragma unroll
      for (int fi = 0; fi < 4; ++fi) dwa[fi][0] = dwa[fi][1] = dba[fi][0] = dba[fi][1] = 0.f;
#pragma unroll
      for (int u = 0; u < R; ++u) {
        const int row = tc_row<NT>(cur, u, lane);
        const int f0 = __shfl_sync(kFullMask, row, cq), f1 = __shfl_sync(kFullMask, row, cq + 1);
        uint32_t a[MT][2];
        tc_gather<BM>(a, slab, row, lane);
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          float P[4] = {0.f, 0.f, 0.f, 0.f};
          uint32_t dh[NPR][2], dl[NPR][2];
#pragma unroll
          for (int n = 0; n < NPR; ++n) {
            const int fi = u * NPR + n;
            const uint32_t bb = tc_word(cur.b, fi);
            const float b0 = bf16_lo(bb), b1 = bf16_hi(bb);
            float z[4];
            const float c[4] = {b0, b1, b0, b1};
            mma_bf16_k8(z, a[m], tc_word(cur.w, fi), c);
            const int s0 = 32 * q + 8 * fi + cq;
            const bool v0 = full || s0 < ng, v1 = full || s0 + 1 < ng;
            float dz[4];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              dz[2 * h] = v0 ? c1[m][h] * dact_f<ACT>(z[2 * h]) : 0.f;
              dz[2 * h + 1] = v1 ? c1[m][h] * dact_f<ACT>(z[2 * h + 1]) : 0.f;
            }
            dba[fi][0] += dz[0] + dz[2];
            dba[fi][1] += dz[1] + dz[3];
            split2(dz[0], dz[1], dh[n][0], dl[n][0]);
            split2(dz[2], dz[3], dh[n][1], dl[n][1]);
            const uint32_t ah[2] = {dh[n][0], dh[n][1]}, al[2] = {dl[n][0], dl[n][1]};
            mma_bf16_k8(P, ah, wt[fi], P);
            mma_bf16_k8(P, al, wt[fi], P);
          }
          // dW of this m-tile: B = x^T of the record's inputs over the m-tile's 16 tokens
          const uint32_t xb0 = movt(a[m][0]), xb1 = movt(a[m][1]);
          if constexpr (NPR == 1) {
            const int fi = u;
#pragma unroll
            for (int part = 0; part < 2; ++part) {
              const uint32_t(&d)[1][2] = part ? dl : dh;
              const uint32_t A[4] = {movt(d[0][0]), 0u, movt(d[0][1]), 0u};
              float o[4];
              const float c[4] = {dwa[fi][0], dwa[fi][1], 0.f, 0.f};
              mma_bf16_k16(o, A, xb0, xb1, c);
              dwa[fi][0] = o[0];
              dwa[fi][1] = o[1];
            }
          } else {
#pragma unroll
            for (int n = 0; n < NPR; n += 2) {
              const int fa = u * NPR + n, fb = fa + 1;
#pragma unroll
              for (int part = 0; part < 2; ++part) {
                const uint32_t(&d)[NPR][2] = part ? dl : dh;
                const uint32_t A[4] = {movt(d[n][0]), movt(d[n + 1][0]), movt(d[n][1]), movt(d[n + 1][1])};
                float o[4];
                const float c[4] = {dwa[fa][0], dwa[fa][1], dwa[fb][0], dwa[fb][1]};
                mma_bf16_k16(o, A, xb0, xb1, c);
                dwa[fa][0] = o[0];
                dwa[fa][1] = o[1];
                dwa[fb][0] = o[2];
                dwa[fb][1] = o[3];
              }
            }
          }
          // scatter the record's dX partials of this m-tile: P[h][e] = (token 16 m + 8 h + lane / 4, input cq + e)
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int t = 16 * m + 8 * h + (lane >> 2);
            if constexpr (FIXED) {
              atomicAdd(dxi + dxs_off<BM>(f0, t), __float2int_rn(P[2 * h] * sc[m][h]));
              atomicAdd(dxi + dxs_off<BM>(f1, t), __float2int_rn(P[2 * h + 1] * sc[m][h]));
            } else {
              atomicAdd(dxs + dxs_off<BM>(f0, t), P[2 * h]);
              atomicAdd(dxs + dxs_off<BM>(f1, t), P[2 * h + 1]);
            }
          }
        }
      }
      // dw: the lane's packed slice [lane][fi][e]; db: lanes 0-3 after folding the 8 token rows
      float* dwp = p.dw + ((g * Q + q) * 32 + lane) * 8;
      red_v4(dwp, dwa[0][0], dwa[0][1], dwa[1][0], dwa[1][1]);
      red_v4(dwp + 4, dwa[2][0], dwa[2][1], dwa[3][0], dwa[3][1]);
#pragma unroll
      for (int off = 4; off < 32; off <<= 1)
#pragma unroll
        for (int fi = 0; fi < 4; ++fi) {
          dba[fi][0] += __shfl_xor_sync(kFullMask, dba[fi][0], off);
          dba[fi][1] += __shfl_xor_sync(kFullMask, dba[fi][1], off);
        }
      if (lane < 4) {
        float* dbp = p.db + ((g * Q + q) * 4 + lane) * 8;
        red_v4(dbp, dba[0][0], dba[0][1], dba[1][0], dba[1][1]);
        red_v4(dbp + 4, dba[2][0], dba[2][1], dba[3][0], dba[3][1]);
      }
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
