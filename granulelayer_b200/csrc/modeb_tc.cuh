// Mode B with bf16 parameters on the tensor cores: helpers shared by the forward (modeb_tc.cu) and
// the backward (modeb_tc_bwd.cu).
//
// The reference's bf16 layers compute with bf16 operands (x cast to the layer dtype,
// sparse_pooling/autograd.py:349-354) and fp32 accumulation on m16n8k8 BF16 tensor-core tiles over
// its fragment-packed storage (layout.py:20-33, 146-179).  These kernels compute the same
// products: every bf16 x bf16 product is exact in fp32, only the order of the fp32 sums differs.
//
// Operand path (B200, one CTA per SM, up to 227 KB of shared memory):
//   x slab   the CTA's BM tokens of x, staged once as a bf16 feature-major tile xs[d][t]
//            (BM * 2 bytes per feature row, 16-byte chunks XOR-swizzled by the row so that the
//            staging stores of consecutive rows spread over all banks);
//   A        per record and 32 tokens, one ldmatrix.x4.trans whose lanes point at the record's 8
//            feature rows: the gather lands directly in the m16n8k8 A fragments (rows = tokens,
//            k = the record's inputs), no gathered copy is written;
//   B        the fragment-packed weights give each lane its B fragments of 4 n-tiles (32 neurons)
//            in one 128-bit load; the bias comes the same way in the accumulator layout;
//   D        the fp32 accumulators of mma.sync.m16n8k8 stay in registers, where the pooling (or
//            the backward's dz) consumes them element by element.
// Why not tcgen05: each record has K = 8 inputs and its products are consumed per element by the
// pooling, so the work is bounded by the gather and the per-element epilogue, not by MMA rate; a
// TMEM accumulator would add a tcgen05.ld round trip per tile and the A operand would have to be
// written to shared memory in the UMMA layout (a second copy of every gathered row).
#pragma once
#include <cuda_bf16.h>

#include "common.cuh"

namespace gl {

constexpr int kTcFwdThreads = 384;
constexpr int kTcStaticSmem = 16384;  // bound on the kernels' static shared memory

struct TcParams {
  const float* x;
  const int16_t* idx;       // fragment-packed indices [G, NB/UB, 8, UB]
  const uint16_t* w;        // fragment-packed bf16 weights [G, Q, 32, 4, 2]
  const uint16_t* b;        // fragment-packed bf16 bias [G, Q, 4, 4, 2]
  const int32_t* counts;
  float* pre;
  const float* gpre;
  float* dx;
  float* dw;
  float* db;
  int32_t* winners;
  const float* wabsmax;     // backward, fixed-point dX tile: max |w| per group (g - g0), or NULL
  const int32_t* rowmax;    // backward, fixed-point dX tile: max record inputs per feature per group
  int B, D, C;
  int64_t NB, g0, g1, ldx, ldp, ldg, lddx, ldwin;
  int pool, gpc;
};

// Shared-memory address of 16-byte chunk c (tokens 8c .. 8c+7) of feature row f of the slab.
template <int BM>
__device__ __forceinline__ uint32_t tc_chunk(uint32_t base, int f, int c) {
  constexpr int CH = BM / 8;
  return base + (uint32_t)(f * (BM * 2) + ((c ^ (f & (CH - 1))) << 4));
}

// Stage x[t0 .. t0+BM) (fp32, token-major, row stride ldx) as the bf16 slab, rounded to nearest
// even; tokens past B are zero.  One item = one 16-byte chunk (8 tokens of one feature); consecutive
// threads take consecutive features, so every global load instruction reads one token row coalesced.
template <int BM, int NTHR>
__device__ __forceinline__ void tc_stage(uint32_t slab, const float* __restrict__ x, int t0, int B, int D,
                                         int64_t ldx) {
  constexpr int CH = BM / 8;
  for (int i = threadIdx.x; i < D * CH; i += NTHR) {
    const int f = i % D, c = i / D;
    float v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int t = t0 + 8 * c + u;
      v[u] = t < B ? __ldg(x + (int64_t)t * ldx + f) : 0.f;
    }
    uint32_t q[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * u], v[2 * u + 1]);
      q[u] = *reinterpret_cast<const uint32_t*>(&h);
    }
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(tc_chunk<BM>(slab, f, c)), "r"(q[0]), "r"(q[1]),
                 "r"(q[2]), "r"(q[3])
                 : "memory");
  }
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x2_t(uint32_t (&r)[2], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0, %1}, [%2];" : "=r"(r[0]), "=r"(r[1]) : "r"(addr));
}

// d = a (16x8 bf16, row) * b (8x8 bf16, col) + c, fp32 accumulation.
__device__ __forceinline__ void mma_bf16_k8(float (&d)[4], const uint32_t (&a)[2], uint32_t b, const float (&c)[4]) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5}, {%6}, {%7, %8, %9, %10};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(b), "f"(c[0]), "f"(c[1]), "f"(c[2]), "f"(c[3]));
}

// A fragments of one record for the CTA's BM tokens: a[mt] = m-tile mt (tokens 16 mt .. 16 mt + 15).
// `row` is the slab row (feature) this lane points at: the record's input k = lane & 7.
template <int BM>
__device__ __forceinline__ void tc_gather(uint32_t (&a)[BM / 16][2], uint32_t slab, int row, int lane) {
  if constexpr (BM == 16) {
    ldsm_x2_t(a[0], tc_chunk<BM>(slab, row, (lane >> 3) & 1));
  } else {
#pragma unroll
    for (int h = 0; h < BM / 32; ++h) {
      uint32_t r[4];
      ldsm_x4_t(r, tc_chunk<BM>(slab, row, 4 * h + (lane >> 3)));
      a[2 * h][0] = r[0];
      a[2 * h][1] = r[1];
      a[2 * h + 1][0] = r[2];
      a[2 * h + 1][1] = r[3];
    }
  }
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x2(uint32_t (&r)[2], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0, %1}, [%2];" : "=r"(r[0]), "=r"(r[1]) : "r"(addr));
}

// The same rows without the transpose: b[mt][o] is the m16n8k16 B fragment (k = the 8 tokens of octet
// o of m-tile mt, n = the record's input lane / 4), i.e. x^T of the record's inputs.
template <int BM>
__device__ __forceinline__ void tc_gather_nt(uint32_t (&b)[BM / 16][2], uint32_t slab, int row, int lane) {
  if constexpr (BM == 16) {
    ldsm_x2(b[0], tc_chunk<BM>(slab, row, (lane >> 3) & 1));
  } else {
#pragma unroll
    for (int h = 0; h < BM / 32; ++h) {
      uint32_t r[4];
      ldsm_x4(r, tc_chunk<BM>(slab, row, 4 * h + (lane >> 3)));
      b[2 * h][0] = r[0];
      b[2 * h][1] = r[1];
      b[2 * h + 1][0] = r[2];
      b[2 * h + 1][1] = r[3];
    }
  }
}

// Operands of fragment quad q of group g (4 n-tiles of 8 neurons = slots 32q .. 32q+31):
// the lane's B fragments (one per n-tile), its bias pairs (accumulator columns 2 (lane & 3) + {0, 1}),
// and the quad's index words (lane l < 8 R holds input l / R of the quad's record l % R).
struct TcQuad {
  uint4 w, b;
  int idx;
};

template <int NT>
__device__ __forceinline__ TcQuad tc_load_quad(const TcParams& p, int64_t g, int q, int lane) {
  constexpr int R = NT < 4 ? 4 / NT : 1;  // records per quad
  const int64_t Q = p.NB * NT / 4;
  TcQuad o;
  o.w = __ldg(reinterpret_cast<const uint4*>(p.w + ((g * Q + q) * 32 + lane) * 8));
  o.b = __ldg(reinterpret_cast<const uint4*>(p.b + ((g * Q + q) * 4 + (lane & 3)) * 8));
  const int64_t base = g * p.NB * 8 + (NT < 4 ? (int64_t)q * 8 * R : (int64_t)(q * 4 / NT) * 8);
  o.idx = lane < 8 * R ? min((int)(uint16_t)__ldg(p.idx + base + lane), p.D - 1) : 0;
  return o;
}

// Slab row of input (lane & 7) of the quad's record u.
template <int NT>
__device__ __forceinline__ int tc_row(const TcQuad& qd, int u, int lane) {
  constexpr int R = NT < 4 ? 4 / NT : 1;
  return __shfl_sync(kFullMask, qd.idx, (lane & 7) * R + u);
}

__device__ __forceinline__ uint32_t tc_word(const uint4& v, int i) {
  return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

}  // namespace gl
