// Mode B with bf16 parameters on the tensor cores: the backward's per-quad work, shared by the
// group-chunk kernel (modeb_tc_bwd.cu) and the input-set kernel (modeb_tc_sets.cu).
#pragma once
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

// One fragment quad q of group g over the CTA's BM tokens: dz, the dX partials into the shared tile
// (rows = slab rows: the feature itself, or its position in the staged set when LOCAL), and the quad's
// dw / db added to the packed fp32 gradients.  c1 / sc are the lane's token rows' coefficients and
// fixed-point scales.
template <int BM, int NT, int ACT, bool FIXED, bool LOCAL>
__device__ __forceinline__ void tc_bwd_quad(const TcParams& p, int64_t g, int q, int ng, const TcQuad& cur,
                                            const float (&c1)[BM / 16][2], const float (&sc)[BM / 16][2],
                                            uint32_t slab, float* dxs, int* dxi, const int16_t* lmap, int lane) {
  constexpr int MT = BM / 16;
  constexpr int R = NT < 4 ? 4 / NT : 1;      // records per quad
  constexpr int NPR = NT < 4 ? NT : 4;        // n-tiles per record within a quad
  const int64_t Q = p.NB * NT / 4;
  const int cq = 2 * (lane & 3);
  const bool full = 32 * q + 32 <= ng;
  uint32_t wt[4];
#pragma unroll
  for (int fi = 0; fi < 4; ++fi) wt[fi] = movt(tc_word(cur.w, fi));
  float dwa[4][2], dba[4][2];
#pragma unroll
  for (int fi = 0; fi < 4; ++fi) dwa[fi][0] = dwa[fi][1] = dba[fi][0] = dba[fi][1] = 0.f;
#pragma unroll
  for (int u = 0; u < R; ++u) {
    const int row = LOCAL ? (int)lmap[tc_row<NT>(cur, u, lane)] : tc_row<NT>(cur, u, lane);
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

}  // namespace gl
