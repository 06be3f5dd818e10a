// Compact K16/C16 execution of the Cover-TopK/16 layer on the tensor cores: bf16 parameters, and fp32
// ones through three-term bf16 splits (below).
//
// Replaces the reference's kgen K = 16 kernels (sparse_pooling/experimental/kgen/kgen.cuh:142-536,
// launched by experimental/kgen_layer.py:61-143) with their arithmetic: bf16 parameters, x rounded to
// bf16 (the layer's compute dtype), fp32 accumulation, and the backward's "split" gradient precision
// (dz carried as hi + lo bf16).  Model as csrc/k16.cu:
//   z[t, f, n] = b[f, n] + sum_k w[f, n, k] * x[t, feat[q][env[f, k]]]      (record f of set q)
//   pre[t, g] += sum_{valid n of the records of g} act(z) / n_g
//   dz = c1t[g, t] act'(z), dW[f, n, k] += sum_t dz x, db[f, n] += sum_t dz, dx += sum_n dz w.
//
// A record is a 16-input x 16-neuron tile, one K step of mma.m16n8k16: per 16 tokens the forward is
// one ldmatrix.x4.trans (the lanes point at the record's 16 slab rows) and two MMAs (neurons 0-7,
// 8-15).  A CTA owns one input set q and BM tokens: the set's S rows of x are staged once as a bf16
// slab (modeb_tc.cuh layout); the set's records (its buckets, in order) are split into one
// contiguous run per warp, so a warp changes output (bucket) rarely.  The forward folds each warp's
// per-token sums of an output over the lane quad and adds them to pre with one atomic per (token,
// warp, output).  The backward keeps, per record, z again, the split dz, the dX partials
// P = dz w (A = the dz accumulator fragments, B = w^T by movmatrix) added to an [S][BM] tile (int32
// fixed point with the bounds, else fp32) with shared atomics, and dW += dz^T x (A = dz^T, B = x^T, both by movmatrix), whose fragments are reduced
// into the fp32 gradients once per record and token tile.
//
// fp32 parameters (gl_k16_fwd_tc_f32 / gl_k16_bwd_tc_f32, NS = 3) run the same tiles on three-term
// bf16 splits: v = v1 + v2 + v3 with v1 = bf16(v), v2 = bf16(v - v1), v3 = bf16(v - v1 - v2), exact
// for 2^-110 <= |v| below bf16's largest value (each step takes 8 more significant bits; bf16 has fp32's
// exponent range, its smallest subnormal is 2^-133, and smaller v lose only what lies below that).  x is split while it is staged (three slab planes), w when its
// record is used, dz when it is formed.  A product sum a.b is the six MMAs of the term pairs
// i + j <= 2 (the smallest first); the three dropped pairs are below 2^-23 |a||b| together, the
// rounding of an fp32 FMA chain, and every product of bf16 terms is exact in the fp32 accumulator.
// The fp32 SIMT kernels (k16.cu) compute the same sums in the k order; these run them on the tensor
// cores at about three times the MMA work of the bf16 layer.
#include "modeb_tc_bwd.cuh"

namespace gl {

// Threads per CTA: the bf16 kernels hold one bf16 term per operand; the split kernels three, so they
// run 8 warps for up to 255 registers a thread.
template <int NS>
__host__ __device__ constexpr int k16tc_threads() { return NS == 1 ? 384 : 256; }

struct K16TcParams {
  const float* x;
  const uint8_t* env;
  const int16_t* feat;
  const int32_t* buckets;
  const int32_t* q_off;
  const int32_t* rec_off;
  const uint16_t* w;        // bf16 [G*NB16, 16, 16] (NS = 1), fp32 (NS = 3)
  const uint16_t* b;        // bf16 [G*NB16, 16] (NS = 1), fp32 (NS = 3)
  const int32_t* counts;
  float* pre;
  const float* c1t;
  float* dx;
  float* dw;
  float* db;
  const float* wabsmax;     // backward, fixed-point dX tile: [G] max |w| per output, or NULL
  const int32_t* brow;      // backward, fixed-point dX tile: [nb] per bucket, its largest number of record
                            // inputs on one set row
  int B, D, G, NB16, S, nbk;
  int64_t ldx, ldp, ldc, lddx;
};

// The three bf16 terms of two fp32 values, packed as pairs (the module comment).
__device__ __forceinline__ void split3(float v0, float v1, uint32_t& t0, uint32_t& t1, uint32_t& t2) {
  t0 = pack_bf16(v0, v1);
  const float r0 = v0 - bf16_lo(t0), r1 = v1 - bf16_hi(t0);
  t1 = pack_bf16(r0, r1);
  t2 = pack_bf16(r0 - bf16_lo(t1), r1 - bf16_hi(t1));
}

// Stage x[t0 .. t0+BM, feat[q][s]] (fp32) as the bf16 slab rows s = 0 .. S-1 and the set's features;
// NS = 3 writes the three terms of x to three slab planes of S * BM * 2 bytes.
template <int BM, int NS>
__device__ __forceinline__ void k16tc_stage(uint32_t slab, int* fq, const K16TcParams& p, int q, int t0) {
  constexpr int CH = BM / 8, NT = k16tc_threads<NS>();
  const uint32_t plane = (uint32_t)p.S * BM * 2;
  for (int s = threadIdx.x; s < p.S; s += NT) {
    const int d = (int)(uint16_t)__ldg(p.feat + (int64_t)q * p.S + s);
    fq[s] = d < p.D ? d : p.D - 1;
  }
  __syncthreads();
  for (int it = threadIdx.x; it < p.S * CH; it += NT) {
    const int i = it % p.S, k = it / p.S;
    const int f = fq[i];
    float v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int t = t0 + 8 * k + u;
      v[u] = t < p.B ? __ldg(p.x + (int64_t)t * p.ldx + f) : 0.f;
    }
    uint32_t w4[NS][4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if constexpr (NS == 1) w4[0][u] = pack_bf16(v[2 * u], v[2 * u + 1]);
      else split3(v[2 * u], v[2 * u + 1], w4[0][u], w4[1][u], w4[2][u]);
    }
#pragma unroll
    for (int j = 0; j < NS; ++j)
      asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(tc_chunk<BM>(slab + j * plane, i, k)),
                   "r"(w4[j][0]), "r"(w4[j][1]), "r"(w4[j][2]), "r"(w4[j][3])
                   : "memory");
  }
}

// One record's operands for lane l: B fragments (neurons 8 nt + l/4, inputs 8 kh + 2 (l%4) + {0,1}), bias
// pairs (neurons 8 nt + 2 (l%4) + {0,1}), and the record's 16 local positions (4 words).  NS = 1: bf16 pairs
// wf[nt][kh], bb[nt]; NS = 3: the fp32 pairs, split when the record is used (k16tc_operands).
template <int NS>
struct K16TcRec {
  uint32_t wf[2][2], bb[2];
  uint4 env;
};
template <>
struct K16TcRec<3> {
  float2 wv[2][2], bb[2];
  uint4 env;
};

template <int NS>
__device__ __forceinline__ K16TcRec<NS> k16tc_load(const K16TcParams& p, int64_t f, int lane) {
  K16TcRec<NS> r;
  if constexpr (NS == 1) {
    const uint32_t* w32 = reinterpret_cast<const uint32_t*>(p.w + f * 256);
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int kh = 0; kh < 2; ++kh) r.wf[nt][kh] = __ldg(w32 + (8 * nt + (lane >> 2)) * 8 + 4 * kh + (lane & 3));
    const uint32_t* b32 = reinterpret_cast<const uint32_t*>(p.b + f * 16);
    r.bb[0] = __ldg(b32 + (lane & 3));
    r.bb[1] = __ldg(b32 + 4 + (lane & 3));
  } else {
    const float2* w2 = reinterpret_cast<const float2*>(p.w) + f * 128;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int kh = 0; kh < 2; ++kh) r.wv[nt][kh] = __ldg(w2 + (8 * nt + (lane >> 2)) * 8 + 4 * kh + (lane & 3));
    const float2* b2 = reinterpret_cast<const float2*>(p.b) + f * 8;
    r.bb[0] = __ldg(b2 + (lane & 3));
    r.bb[1] = __ldg(b2 + 4 + (lane & 3));
  }
  r.env = __ldg(reinterpret_cast<const uint4*>(p.env + f * 16));
  return r;
}

// A record's B fragments as bf16 terms wf[nt][term][kh] and its fp32 bias pairs bias[nt][e].
template <int NS>
__device__ __forceinline__ void k16tc_operands(const K16TcRec<NS>& r, uint32_t (&wf)[2][NS][2], float (&bias)[2][2]) {
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
    if constexpr (NS == 1) {
      wf[nt][0][0] = r.wf[nt][0];
      wf[nt][0][1] = r.wf[nt][1];
      bias[nt][0] = bf16_lo(r.bb[nt]);
      bias[nt][1] = bf16_hi(r.bb[nt]);
    } else {
#pragma unroll
      for (int kh = 0; kh < 2; ++kh) split3(r.wv[nt][kh].x, r.wv[nt][kh].y, wf[nt][0][kh], wf[nt][1][kh], wf[nt][2][kh]);
      bias[nt][0] = r.bb[nt].x;
      bias[nt][1] = r.bb[nt].y;
    }
  }
}

// z += sum over the term pairs i + j < NS of A_i B_j (B_j = the fragments (b[j][0], b[j][1])), the
// smallest pairs first: one MMA for NS = 1, six for NS = 3.
template <int NS>
__device__ __forceinline__ void k16tc_dot(float (&z)[4], const uint32_t (&a)[NS][4], const uint32_t (&b)[NS][2]) {
#pragma unroll
  for (int s = NS - 1; s >= 0; --s)
#pragma unroll
    for (int i = 0; i <= s; ++i) mma_bf16_k16(z, a[i], b[s - i][0], b[s - i][1], z);
}

// Local position of input k of the record (clamped to the set).
__device__ __forceinline__ int k16tc_pos(const uint4& env, int k, int smax) {
  const uint32_t wd = k < 4 ? env.x : k < 8 ? env.y : k < 12 ? env.z : env.w;
  return min((int)((wd >> (8 * (k & 3))) & 0xffu), smax);
}

// The warp's run of the set's records: [r0, r1) in flat record numbers, and the bucket walk.
struct K16TcWalk {
  int bk, bend;  // current bucket index, end of the set's buckets
  int r, r1;
};

__device__ __forceinline__ K16TcWalk k16tc_walk(const K16TcParams& p, int q, int warp, int nw) {
  K16TcWalk w;
  const int qa = min(max(__ldg(p.q_off + q), 0), p.nbk), qb = min(max(__ldg(p.q_off + q + 1), qa), p.nbk);
  const int ra = __ldg(p.rec_off + qa), rb = __ldg(p.rec_off + qb);
  const int per = (rb - ra + nw - 1) / nw;
  w.r = ra + warp * per;
  w.r1 = min(w.r + per, rb);
  w.bk = qa;
  w.bend = qb;
  while (w.bk < w.bend && __ldg(p.rec_off + w.bk + 1) <= w.r) ++w.bk;
  return w;
}

// Record f and output g of flat record r (the walk advances monotonically); false for a malformed row.
__device__ __forceinline__ bool k16tc_at(const K16TcParams& p, K16TcWalk& w, int r, int& g, int& j16) {
  while (w.bk < w.bend && __ldg(p.rec_off + w.bk + 1) <= r) ++w.bk;
  if (w.bk >= w.bend) return false;
  const int4 bk = __ldg(reinterpret_cast<const int4*>(p.buckets) + w.bk);
  g = bk.y;
  j16 = bk.z + (r - __ldg(p.rec_off + w.bk));
  return g >= 0 && g < p.G && j16 >= 0 && j16 < p.NB16;
}

// The warp's next valid record, with its operands already requested.
template <int NS>
struct K16TcNext {
  int r, g, j16;
  bool have;
  K16TcRec<NS> rec;
  __device__ __forceinline__ K16TcNext(const K16TcParams& p, K16TcWalk& w, int lane) : r(w.r - 1), have(false) {
    advance(p, w, lane);
  }
  __device__ __forceinline__ void advance(const K16TcParams& p, K16TcWalk& w, int lane) {
    have = false;
    while (++r < w.r1)
      if (k16tc_at(p, w, r, g, j16)) {
        have = true;
        rec = k16tc_load<NS>(p, (int64_t)g * p.NB16 + j16, lane);
        return;
      }
  }
};

template <int BM, int ACT, int NS>
__global__ void __launch_bounds__(k16tc_threads<NS>(), 1) k16tc_fwd_kernel(const K16TcParams p) {
  constexpr int MT = BM / 16, NW = k16tc_threads<NS>() / 32;
  extern __shared__ __align__(128) unsigned char tc_smem[];
  __shared__ int fq[256];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int q = blockIdx.y, t0 = blockIdx.x * BM;
  const uint32_t slab = (uint32_t)__cvta_generic_to_shared(tc_smem), plane = (uint32_t)p.S * BM * 2;
  k16tc_stage<BM, NS>(slab, fq, p, q, t0);
  __syncthreads();
  K16TcWalk wk = k16tc_walk(p, q, warp, NW);
  const int cq = 2 * (lane & 3), smax = p.S - 1;
  float acc[MT][2];
  int gcur = -1;
  auto flush = [&]() {
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        acc[m][h] += __shfl_xor_sync(kFullMask, acc[m][h], 1);
        acc[m][h] += __shfl_xor_sync(kFullMask, acc[m][h], 2);
      }
    if ((lane & 3) == 0) {
      const float inv = 1.f / (float)max(__ldg(p.counts + gcur), 1);
#pragma unroll
      for (int m = 0; m < MT; ++m)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int t = t0 + 16 * m + 8 * h + (lane >> 2);
          if (t < p.B) atomicAdd(p.pre + (int64_t)t * p.ldp + gcur, acc[m][h] * inv);
        }
    }
  };
  K16TcNext<NS> nx(p, wk, lane);
  while (nx.have) {
    const int g = nx.g, j16 = nx.j16;
    uint32_t wf[2][NS][2];
    float bias[2][2];
    k16tc_operands<NS>(nx.rec, wf, bias);
    const uint4 env = nx.rec.env;
    nx.advance(p, wk, lane);  // the next record's operands load while this one computes
    if (g != gcur) {
      if (gcur >= 0) flush();
      gcur = g;
#pragma unroll
      for (int m = 0; m < MT; ++m) acc[m][0] = acc[m][1] = 0.f;
    }
    const int nv = __ldg(p.counts + g) - 16 * j16;  // valid neurons of this record (<= 0: none)
    const int row = k16tc_pos(env, (lane & 7) + 8 * (lane >> 4), smax);
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      uint32_t a[NS][4];
#pragma unroll
      for (int j = 0; j < NS; ++j) ldsm_x4_t(a[j], tc_chunk<BM>(slab + j * plane, row, 2 * m + ((lane >> 3) & 1)));
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        float z[4] = {bias[nt][0], bias[nt][1], bias[nt][0], bias[nt][1]};
        k16tc_dot<NS>(z, a, wf[nt]);
        const bool v0 = 8 * nt + cq < nv, v1 = 8 * nt + cq + 1 < nv;
#pragma unroll
        for (int h = 0; h < 2; ++h)
          acc[m][h] += (v0 ? act_f<ACT>(z[2 * h]) : 0.f) + (v1 ? act_f<ACT>(z[2 * h + 1]) : 0.f);
      }
    }
  }
  if (gcur >= 0) flush();
}

// dX tile [S][BM]: element (s, t) at s * BM + (t ^ (s & (BM - 1))), as dxs_off.  FIXED: int32 fixed
// point at one power-of-two scale per token for the CTA's set, with
//   16 * max|act'| * sum over the set's buckets b of m_b * |c1t[g_b, t]| * max|w|_{g_b} * scale <= 2^30
// (m_b = the bucket's largest number of record inputs on one set row), so no word can overflow; shared
// int32 atomics run at 2.4x the rate of fp32 ones.  A token whose bound is not finite gets NaN in dx.
// dz is carried as ND bf16 terms: hi + lo for the bf16 layer (its "split" precision), three for NS = 3.
template <int BM, int ACT, bool FIXED, int NS>
__global__ void __launch_bounds__(k16tc_threads<NS>(), 1) k16tc_bwd_kernel(const K16TcParams p) {
  constexpr int MT = BM / 16, NT = k16tc_threads<NS>(), NW = NT / 32, ND = NS == 1 ? 2 : 3;
  extern __shared__ __align__(128) unsigned char tc_smem[];
  __shared__ int fq[256];
  __shared__ float qsc[FIXED ? BM : 1], qinv[FIXED ? BM : 1];
  float* dxs = reinterpret_cast<float*>(tc_smem + (size_t)NS * p.S * BM * 2);
  int* dxi = reinterpret_cast<int*>(dxs);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int q = blockIdx.y, t0 = blockIdx.x * BM;
  const uint32_t slab = (uint32_t)__cvta_generic_to_shared(tc_smem), plane = (uint32_t)p.S * BM * 2;
  k16tc_stage<BM, NS>(slab, fq, p, q, t0);
  for (int i = threadIdx.x; i < p.S * BM; i += NT) dxs[i] = 0.f;
  if constexpr (FIXED) {
    if (threadIdx.x < BM) {
      const int t = t0 + threadIdx.x;
      const int qa = min(max(__ldg(p.q_off + q), 0), p.nbk), qb = min(max(__ldg(p.q_off + q + 1), qa), p.nbk);
      float bound = 0.f;
      if (t < p.B)
        for (int b = qa; b < qb; ++b) {
          const int g = __ldg(p.buckets + 4 * b + 1);
          if (g < 0 || g >= p.G) continue;
          bound += fabsf(__ldg(p.c1t + (int64_t)g * p.ldc + t)) * (float)__ldg(p.brow + b) * __ldg(p.wabsmax + g);
        }
      bound *= 16.f * (ACT == GL_ACT_GELU ? 1.13f : 1.f);
      float s_ = 0.f, i_ = 0.f;
      if (!(bound <= 3.0e38f)) {
        i_ = __int_as_float(0x7fc00000);
      } else if (bound > 0.f) {
        const int e = min(max(30 - ilogbf(bound) - 1, -126), 126);
        s_ = ldexpf(1.f, e);
        i_ = ldexpf(1.f, -e);
      }
      qsc[threadIdx.x] = s_;
      qinv[threadIdx.x] = i_;
    }
  }
  __syncthreads();
  float sc[MT][2];
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int h = 0; h < 2; ++h) sc[m][h] = FIXED ? qsc[16 * m + 8 * h + (lane >> 2)] : 0.f;
  K16TcWalk wk = k16tc_walk(p, q, warp, NW);
  const int cq = 2 * (lane & 3), smax = p.S - 1;
  float c1[MT][2];
  int gcur = -1;
  K16TcNext<NS> nx(p, wk, lane);
  while (nx.have) {
    const int g = nx.g, j16 = nx.j16;
    uint32_t wf[2][NS][2];
    float bias[2][2];
    k16tc_operands<NS>(nx.rec, wf, bias);
    const uint4 env = nx.rec.env;
    nx.advance(p, wk, lane);
    if (g != gcur) {
      gcur = g;
#pragma unroll
      for (int m = 0; m < MT; ++m)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int t = t0 + 16 * m + 8 * h + (lane >> 2);
          c1[m][h] = t < p.B ? __ldg(p.c1t + (int64_t)g * p.ldc + t) : 0.f;
        }
    }
    const int64_t f = (int64_t)g * p.NB16 + j16;
    const int nv = __ldg(p.counts + g) - 16 * j16;
    const int row = k16tc_pos(env, (lane & 7) + 8 * (lane >> 4), smax);
    int prow[2][2];  // slab rows of the inputs 8 kh + cq + e this lane's dX partials belong to
#pragma unroll
    for (int kh = 0; kh < 2; ++kh)
#pragma unroll
      for (int e = 0; e < 2; ++e) prow[kh][e] = k16tc_pos(env, 8 * kh + cq + e, smax);
    uint32_t wt[2][NS][2];  // [kh][term]: w^T fragments (k = neurons 8 nt + cq + {0,1}, n = input 8 kh + lane / 4)
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int j = 0; j < NS; ++j)
#pragma unroll
        for (int kh = 0; kh < 2; ++kh) wt[kh][j][nt] = movt(wf[nt][j][kh]);
    float dwa[2][4] = {};   // [kh]: (neuron lane/4, inputs 8 kh + cq + {0,1}), (neuron lane/4 + 8, same)
    float dba[2][2] = {};   // [nt][e]: neuron 8 nt + cq + e, this lane's tokens
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      uint32_t a[NS][4];
#pragma unroll
      for (int j = 0; j < NS; ++j) ldsm_x4_t(a[j], tc_chunk<BM>(slab + j * plane, row, 2 * m + ((lane >> 3) & 1)));
      uint32_t dt[ND][2][2];  // [term][nt][rows 0-7 | 8-15]
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        float z[4] = {bias[nt][0], bias[nt][1], bias[nt][0], bias[nt][1]};
        k16tc_dot<NS>(z, a, wf[nt]);
        const bool v0 = 8 * nt + cq < nv, v1 = 8 * nt + cq + 1 < nv;
        float dz[4];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          dz[2 * h] = v0 ? c1[m][h] * dact_f<ACT>(z[2 * h]) : 0.f;
          dz[2 * h + 1] = v1 ? c1[m][h] * dact_f<ACT>(z[2 * h + 1]) : 0.f;
        }
        dba[nt][0] += dz[0] + dz[2];
        dba[nt][1] += dz[1] + dz[3];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          if constexpr (NS == 1) split2(dz[2 * h], dz[2 * h + 1], dt[0][nt][h], dt[1][nt][h]);
          else split3(dz[2 * h], dz[2 * h + 1], dt[0][nt][h], dt[1][nt][h], dt[2][nt][h]);
        }
      }
      // dX partials of the record's 16 inputs: P_kh = dz (tokens x neurons) w^T (neurons x inputs 8 kh ..)
      uint32_t ad[ND][4];
#pragma unroll
      for (int i = 0; i < ND; ++i) {
        ad[i][0] = dt[i][0][0];
        ad[i][1] = dt[i][0][1];
        ad[i][2] = dt[i][1][0];
        ad[i][3] = dt[i][1][1];
      }
#pragma unroll
      for (int kh = 0; kh < 2; ++kh) {
        float P[4] = {0.f, 0.f, 0.f, 0.f};
        if constexpr (NS == 1) {
          mma_bf16_k16(P, ad[0], wt[kh][0][0], wt[kh][0][1], P);
          mma_bf16_k16(P, ad[1], wt[kh][0][0], wt[kh][0][1], P);
        } else {
          k16tc_dot<NS>(P, ad, wt[kh]);
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int t = 16 * m + 8 * h + (lane >> 2);
          if constexpr (FIXED) {
            atomicAdd(dxi + dxs_off<BM>(prow[kh][0], t), __float2int_rn(P[2 * h] * sc[m][h]));
            atomicAdd(dxi + dxs_off<BM>(prow[kh][1], t), __float2int_rn(P[2 * h + 1] * sc[m][h]));
          } else {
            atomicAdd(dxs + dxs_off<BM>(prow[kh][0], t), P[2 * h]);
            atomicAdd(dxs + dxs_off<BM>(prow[kh][1], t), P[2 * h + 1]);
          }
        }
      }
      // dW: A = dz^T (neurons x tokens), B = x^T (tokens x inputs 8 kh ..), both transposed in registers
      uint32_t td[ND][4];
#pragma unroll
      for (int i = 0; i < ND; ++i) {
        td[i][0] = movt(dt[i][0][0]);
        td[i][1] = movt(dt[i][1][0]);
        td[i][2] = movt(dt[i][0][1]);
        td[i][3] = movt(dt[i][1][1]);
      }
#pragma unroll
      for (int kh = 0; kh < 2; ++kh) {
        uint32_t xt[NS][2];
#pragma unroll
        for (int j = 0; j < NS; ++j) {
          xt[j][0] = movt(a[j][2 * kh]);
          xt[j][1] = movt(a[j][2 * kh + 1]);
        }
        if constexpr (NS == 1) {
          mma_bf16_k16(dwa[kh], td[0], xt[0][0], xt[0][1], dwa[kh]);
          mma_bf16_k16(dwa[kh], td[1], xt[0][0], xt[0][1], dwa[kh]);
        } else {
          k16tc_dot<NS>(dwa[kh], td, xt);
        }
      }
    }
    // dw[f][n][k]: lane holds (n = lane/4, k = 8 kh + cq + {0,1}) and (n + 8, same k)
    float* dwp = p.dw + f * 256;
#pragma unroll
    for (int kh = 0; kh < 2; ++kh) {
      const int k = 8 * kh + cq;
      atomicAdd(reinterpret_cast<float2*>(dwp + (lane >> 2) * 16 + k), make_float2(dwa[kh][0], dwa[kh][1]));
      atomicAdd(reinterpret_cast<float2*>(dwp + ((lane >> 2) + 8) * 16 + k), make_float2(dwa[kh][2], dwa[kh][3]));
    }
#pragma unroll
    for (int off = 4; off < 32; off <<= 1)
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        dba[nt][0] += __shfl_xor_sync(kFullMask, dba[nt][0], off);
        dba[nt][1] += __shfl_xor_sync(kFullMask, dba[nt][1], off);
      }
    if (lane < 4) {
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
        atomicAdd(reinterpret_cast<float2*>(p.db + f * 16 + 8 * nt + 2 * lane), make_float2(dba[nt][0], dba[nt][1]));
    }
  }
  __syncthreads();
  // dx[t0 + t, feat[q][s]] += tile; consecutive threads take consecutive set rows of one token
  for (int it = threadIdx.x; it < p.S * BM; it += NT) {
    const int t = it / p.S, s = it - t * p.S;
    float v;
    bool add;
    if constexpr (FIXED) {
      const int qv = dxi[dxs_off<BM>(s, t)];
      v = (float)qv * qinv[t];
      add = qv != 0 || qinv[t] != qinv[t];
    } else {
      v = dxs[dxs_off<BM>(s, t)];
      add = v != 0.f;
    }
    if (t0 + t < p.B && add) atomicAdd(p.dx + (int64_t)(t0 + t) * p.lddx + fq[s], v);
  }
}

static int k16tc_prepare(const GlK16Args& a, bool bwd, K16TcParams& p, const float* wabsmax, const int32_t* brow) {
  if (a.B < 0 || a.D < 1 || a.D > 32767 || a.G < 1 || a.NB16 < 1 || a.Q < 1 || a.S < 16 || a.S > 256 ||
      a.nbuckets < 0)
    return GL_ERR_SHAPE;
  if (a.act != GL_ACT_RELU && a.act != GL_ACT_IDENTITY) return GL_ERR_UNSUPPORTED;
  if (a.B == 0 || a.nbuckets == 0) return 1;
  if (!a.x || !a.env || !a.feat || !a.buckets || !a.q_off || !a.rec_off || !a.w || !a.b || !a.counts)
    return GL_ERR_NULL;
  if (a.B > 2147483647LL || a.ldx < a.D || a.Q > 65535 || a.G * a.NB16 > 2147483647LL) return GL_ERR_SHAPE;
  if (((uintptr_t)a.env & 15) || ((uintptr_t)a.buckets & 15) || ((uintptr_t)a.w & 15) || ((uintptr_t)a.b & 15))
    return GL_ERR_ALIGN;
  if (!bwd) {
    if (!a.pre) return GL_ERR_NULL;
    if (a.ldp < a.G) return GL_ERR_SHAPE;
  } else {
    if (!a.c1t || !a.dx || !a.dw || !a.db) return GL_ERR_NULL;
    if (a.ldc < a.B || a.lddx < a.D) return GL_ERR_SHAPE;
    if (((uintptr_t)a.dw & 7) || ((uintptr_t)a.db & 7)) return GL_ERR_ALIGN;
  }
  p = K16TcParams{a.x, a.env, a.feat, a.buckets, a.q_off, a.rec_off, reinterpret_cast<const uint16_t*>(a.w),
                  reinterpret_cast<const uint16_t*>(a.b), a.counts, a.pre, a.c1t, a.dx, a.dw, a.db, wabsmax, brow,
                  (int)a.B, (int)a.D, (int)a.G, (int)a.NB16, (int)a.S, (int)a.nbuckets,
                  a.ldx, a.ldp, a.ldc, a.lddx};
  return GL_OK;
}

template <int BM, int ACT, bool BWD, bool FIXED, int NS>
static int k16tc_launch(const K16TcParams& p, int64_t Q, cudaStream_t st) {
  constexpr int NT = k16tc_threads<NS>();
  const size_t smem = (size_t)p.S * BM * (2 * NS + (BWD ? 4 : 0));
  const void* kern = BWD ? (const void*)k16tc_bwd_kernel<BM, ACT, FIXED, NS> : (const void*)k16tc_fwd_kernel<BM, ACT, NS>;
  int rc = ensure_dynamic_smem(kern, smem);
  if (rc) return rc;
  const dim3 grid((unsigned)((p.B + BM - 1) / BM), (unsigned)Q);
  if constexpr (BWD) k16tc_bwd_kernel<BM, ACT, FIXED, NS><<<grid, NT, smem, st>>>(p);
  else k16tc_fwd_kernel<BM, ACT, NS><<<grid, NT, smem, st>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e);
  count_launches(1);
  return GL_OK;
}

template <int BM, bool BWD, int NS>
static int k16tc_act(const K16TcParams& p, int64_t Q, bool relu, bool fixed, cudaStream_t st) {
  if (fixed) return relu ? k16tc_launch<BM, GL_ACT_RELU, BWD, true, NS>(p, Q, st)
                         : k16tc_launch<BM, GL_ACT_IDENTITY, BWD, true, NS>(p, Q, st);
  return relu ? k16tc_launch<BM, GL_ACT_RELU, BWD, false, NS>(p, Q, st)
              : k16tc_launch<BM, GL_ACT_IDENTITY, BWD, false, NS>(p, Q, st);
}

template <bool BWD, int NS>
static int k16tc_run(const GlK16Args* args, const float* wabsmax, const int32_t* brow, void* stream) {
  if (!args) return GL_ERR_NULL;
  if ((wabsmax == nullptr) != (brow == nullptr)) return GL_ERR_NULL;
  K16TcParams p;
  int rc = k16tc_prepare(*args, BWD, p, wabsmax, brow);
  if (rc) return rc > 0 ? GL_OK : rc;
  int optin = 0;
  if ((rc = device_smem_optin(&optin))) return rc;
  const int64_t row_bytes = (int64_t)p.S * (2 * NS + (BWD ? 4 : 0));  // shared bytes per token of a tile
  int BM = args->tokens;
  if (BM == 0) {
    // measured at config 4: 128 tokens, the backward's where its tile fits (split kernels 51.8 ms against
    // 58.2 ms at 64; bf16 25.9 against 30.8 ms), else 64
    BM = (!BWD || row_bytes * 128 + 8192 <= optin) ? 128 : 64;
  }
  if (BM != 32 && BM != 64 && BM != 128) return GL_ERR_UNSUPPORTED;
  if (row_bytes * BM + 8192 > optin) return GL_ERR_SMEM;
  cudaStream_t st = (cudaStream_t)stream;
  const bool relu = args->act == GL_ACT_RELU, fixed = BWD && wabsmax != nullptr;
  switch (BM) {
    case 128: return k16tc_act<128, BWD, NS>(p, args->Q, relu, fixed, st);
    case 64: return k16tc_act<64, BWD, NS>(p, args->Q, relu, fixed, st);
    default: return k16tc_act<32, BWD, NS>(p, args->Q, relu, fixed, st);
  }
}

}  // namespace gl

extern "C" int gl_k16_fwd_tc(const GlK16Args* args, void* stream) {
  return gl::k16tc_run<false, 1>(args, nullptr, nullptr, stream);
}

extern "C" int gl_k16_bwd_tc(const GlK16Args* args, const float* wabsmax, const int32_t* rowmax, void* stream) {
  return gl::k16tc_run<true, 1>(args, wabsmax, rowmax, stream);
}

extern "C" int gl_k16_fwd_tc_f32(const GlK16Args* args, void* stream) {
  return gl::k16tc_run<false, 3>(args, nullptr, nullptr, stream);
}

extern "C" int gl_k16_bwd_tc_f32(const GlK16Args* args, const float* wabsmax, const int32_t* rowmax, void* stream) {
  return gl::k16tc_run<true, 3>(args, wabsmax, rowmax, stream);
}
