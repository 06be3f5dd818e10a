// Compact K16/C16 execution of the Cover-TopK/16 layer (fp32).
//
// Replaces the reference's kgen kernels at K = 16 (sparse_pooling/experimental/kgen/kgen.cuh:142-536,
// entries kgen_abi.cu, launched by experimental/kgen_layer.py:61-143), which run BF16 tensor-core
// tiles on sm_80.  Same model (experimental/reference.py:7-27):
//   record f = g*NB16 + j (16 neurons sharing one 16-input record), neuron slot s = 16 j + n of
//   output g is valid iff s < n_g;
//   z[t, f, n]  = b[f, n] + sum_k w[f, n, k] * x[t, feat[q][env[f, k]]]
//   pre[t, g]  += sum_{valid (f, n) of g} act(z) / n_g
// and the backward with c1t[g, t] = dL/dpre[t, g] / n_g:
//   dz = c1t[g, t] * act'(z) (valid slots), dW[f, n, k] += sum_t dz x,  db[f, n] += sum_t dz,
//   dx[t, feat[q][env[f, k]]] += sum_n dz[t, f, n] w[f, n, k].
//
// Both kernels are input-set stationary: a block owns one input set q (every record of the
// set reads only the set's S features feat[q]) and a chunk of TT tokens.  It stages the set's
// S x-columns for those tokens in shared memory (S * TT floats), then walks the set's
// records (the sorted bucket list: one bucket = a run of consecutive records of one output);
// each record's weights are loaded once per token chunk and kept in registers while the
// warp sweeps all TT tokens.  With one chunk (B <= TT) the weights stream from HBM once.
//
// Forward lanes: lane = (neuron pair p = lane >> 2, token quarter = lane & 3); a warp step
// covers one record and 16 tokens, the four quarters read adjacent float4s of the same
// shared-memory row (one wavefront per load).  The 16 neurons' activations are summed with a
// transpose-reduction (4 shuffles per 16 tokens) and added to a per-bucket token row in shared
// memory; rows are flushed to pre with one global reduction per (bucket, token).
//
// Backward lanes: lane = (token half h = lane >> 4, neuron n = lane & 15); a warp step covers one
// record and 8 tokens.  Each lane recomputes z for its neuron, forms dz, accumulates its 16 dW
// and db in registers across the chunk, and publishes dz to a per-warp shared slab; lane n then
// acts as input k = n of the record: dX[k][t] = sum_m dz[m][t] w[m][k] (the column w[:, k] is
// held in registers) is added to the block's dX tile with shared-memory atomics.  The block
// ends with global reductions of dW/db (per record) and of the dX tile into dx.
#include "common.cuh"

namespace gl {

constexpr int kK16FwdThreads = 512;
constexpr int kK16BwdThreads = 256;
constexpr int kK16Pass = 64;       // buckets resolved per pass (rows of the per-bucket token tiles)
constexpr int kK16MaxS = 256;      // env holds uint8 local positions

struct K16Params {
  const float* x;
  const uint8_t* env;
  const int16_t* feat;
  const int32_t* buckets;
  const int32_t* q_off;
  const int32_t* rec_off;
  const float* w;
  const float* b;
  const int32_t* counts;
  float* pre;
  const float* c1t;
  float* dx;
  float* dw;
  float* db;
  int B, D, G, NB16, S, TT, nbk;
  int64_t ldx, ldp, ldc, lddx;
};

// Bucket rows of one pass: record start (relative to the pass), output, first 16-block.
struct K16PassInfo {
  int rstart[kK16Pass + 1];
  int g[kK16Pass];
  int first[kK16Pass];
};

__device__ __forceinline__ void k16_load_pass(K16PassInfo& ps, const K16Params& p, int p0, int np) {
  const int base = __ldg(p.rec_off + p0);
  for (int i = threadIdx.x; i <= np; i += blockDim.x) {
    ps.rstart[i] = __ldg(p.rec_off + p0 + i) - base;
    if (i < np) {
      const int4 bk = __ldg(reinterpret_cast<const int4*>(p.buckets) + p0 + i);
      ps.g[i] = bk.y;
      ps.first[i] = bk.z;
    }
  }
}

// Bucket row of pass-relative record r: the largest i with rstart[i] <= r (empty buckets skipped).
__device__ __forceinline__ int k16_find(const K16PassInfo& ps, int np, int r) {
  int lo = 0, hi = np;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (ps.rstart[mid] <= r) lo = mid; else hi = mid;
  }
  return lo;
}

// Stage x[t0 + t, feat[q][s]] into xs[s * TT + t] (zeros past the batch) and the clamped features.
__device__ __forceinline__ void k16_stage_x(float* __restrict__ xs, int* __restrict__ fq, const K16Params& p,
                                            int q, int t0, int ntok) {
  for (int s = threadIdx.x; s < p.S; s += blockDim.x) {
    const int d = (int)(uint16_t)__ldg(p.feat + (int64_t)q * p.S + s);
    fq[s] = d < p.D ? d : p.D - 1;
  }
  __syncthreads();
  const int n = p.S * p.TT;
  for (int e = threadIdx.x; e < n; e += blockDim.x) {
    const int s = e / p.TT, t = e - s * p.TT;
    xs[e] = t < ntok ? __ldg(p.x + (int64_t)(t0 + t) * p.ldx + fq[s]) : 0.f;
  }
}

// The record's 16 local positions (clamped to the set), each times `mul` (a row stride).
__device__ __forceinline__ void k16_env(const uint8_t* __restrict__ env, int64_t f, int smax, int mul,
                                        int (&off)[16]) {
  const uint4 e4 = __ldg(reinterpret_cast<const uint4*>(env + f * 16));
  const unsigned ev[4] = {e4.x, e4.y, e4.z, e4.w};
#pragma unroll
  for (int j = 0; j < 4; ++j)
#pragma unroll
    for (int c = 0; c < 4; ++c) off[4 * j + c] = min((int)((ev[j] >> (8 * c)) & 0xffu), smax) * mul;
}

template <int ACT>
__global__ void __launch_bounds__(kK16FwdThreads, 1) k16_fwd_kernel(const K16Params p) {
  constexpr int NW = kK16FwdThreads / 32;
  extern __shared__ __align__(16) float sm[];
  const int TT = p.TT;
  float* xs = sm;                          // [S][TT]
  float* ys = sm + (size_t)p.S * TT;       // [kK16Pass][TT] per-bucket token sums
  __shared__ K16PassInfo ps;
  __shared__ int fq[kK16MaxS];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int q = blockIdx.x, t0 = blockIdx.y * TT;
  const int ntok = min(TT, p.B - t0);
  k16_stage_x(xs, fq, p, q, t0, ntok);
  for (int e = threadIdx.x; e < kK16Pass * TT; e += kK16FwdThreads) ys[e] = 0.f;
  const int qtr = lane & 3, n0 = 2 * (lane >> 2);
  const int b_hi = min(max(__ldg(p.q_off + q + 1), 0), p.nbk);
  const int b_lo = min(max(__ldg(p.q_off + q), 0), b_hi);
  for (int p0 = b_lo; p0 < b_hi; p0 += kK16Pass) {
    const int np = min(kK16Pass, b_hi - p0);
    __syncthreads();
    k16_load_pass(ps, p, p0, np);
    __syncthreads();
    const int nrec = ps.rstart[np];
    for (int r = warp; r < nrec; r += NW) {
      const int i = k16_find(ps, np, r);
      const int g = ps.g[i];
      const int j16 = ps.first[i] + (r - ps.rstart[i]);
      if (g < 0 || g >= p.G || j16 < 0 || j16 >= p.NB16) continue;  // warp-uniform: malformed bucket row
      const int64_t f = (int64_t)g * p.NB16 + j16;
      const int ng = __ldg(p.counts + g);
      const bool ok0 = j16 * 16 + n0 < ng, ok1 = j16 * 16 + n0 + 1 < ng;
      float w0[16], w1[16];
      {
        const float4* wp = reinterpret_cast<const float4*>(p.w + (f * 16 + n0) * 16);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const float4 a = __ldg(wp + c), b = __ldg(wp + 4 + c);
          w0[4 * c] = a.x; w0[4 * c + 1] = a.y; w0[4 * c + 2] = a.z; w0[4 * c + 3] = a.w;
          w1[4 * c] = b.x; w1[4 * c + 1] = b.y; w1[4 * c + 2] = b.z; w1[4 * c + 3] = b.w;
        }
      }
      const float b0 = __ldg(p.b + f * 16 + n0), b1 = __ldg(p.b + f * 16 + n0 + 1);
      int off[16];
      k16_env(p.env, f, p.S - 1, TT, off);
      float* yrow = ys + i * TT;
      for (int tq = 0; tq < ntok; tq += 16) {
        const int col = tq + 4 * qtr;
        float z0[4] = {b0, b0, b0, b0}, z1[4] = {b1, b1, b1, b1};
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          const float4 v = *reinterpret_cast<const float4*>(xs + off[k] + col);
          z0[0] = fmaf(w0[k], v.x, z0[0]); z0[1] = fmaf(w0[k], v.y, z0[1]);
          z0[2] = fmaf(w0[k], v.z, z0[2]); z0[3] = fmaf(w0[k], v.w, z0[3]);
          z1[0] = fmaf(w1[k], v.x, z1[0]); z1[1] = fmaf(w1[k], v.y, z1[1]);
          z1[2] = fmaf(w1[k], v.z, z1[2]); z1[3] = fmaf(w1[k], v.w, z1[3]);
        }
        float a[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) a[j] = (ok0 ? act_f<ACT>(z0[j]) : 0.f) + (ok1 ? act_f<ACT>(z1[j]) : 0.f);
        // transpose-reduction over the 8 neuron pairs (lane bits 4, 3, 2); the 4 tokens end up
        // split by lane bits 4 and 3
        const bool hi = lane & 16, mid = lane & 8;
        const float s0 = hi ? a[0] : a[2], s1 = hi ? a[1] : a[3];
        const float k0 = hi ? a[2] : a[0], k1 = hi ? a[3] : a[1];
        const float c0 = k0 + __shfl_xor_sync(kFullMask, s0, 16);
        const float c1 = k1 + __shfl_xor_sync(kFullMask, s1, 16);
        float v = (mid ? c1 : c0) + __shfl_xor_sync(kFullMask, mid ? c0 : c1, 8);
        v += __shfl_xor_sync(kFullMask, v, 4);
        const int t = col + (hi ? 2 : 0) + (mid ? 1 : 0);
        if (!(lane & 4) && t < ntok) atomicAdd(yrow + t, v);
      }
    }
    __syncthreads();
    for (int e = threadIdx.x; e < np * TT; e += kK16FwdThreads) {
      const int i = e / TT, t = e - i * TT;
      const float v = ys[e];
      ys[e] = 0.f;
      const int g = ps.g[i];
      if (t < ntok && g >= 0 && g < p.G)
        red_add(p.pre + (int64_t)(t0 + t) * p.ldp + g, v / (float)__ldg(p.counts + g));
    }
  }
}

template <int ACT>
__device__ __forceinline__ float k16_dz(float c, float z) {
  if constexpr (ACT == GL_ACT_RELU) {
    return z > 0.f ? c : 0.f;  // a select, as a masked gradient: a non-finite c stays out of inactive slots
  } else {
    return c * dact_f<ACT>(z);
  }
}

template <int ACT>
__global__ void __launch_bounds__(kK16BwdThreads, 1) k16_bwd_kernel(const K16Params p) {
  constexpr int NW = kK16BwdThreads / 32;
  extern __shared__ __align__(16) float sm[];
  const int TT = p.TT, TTD = TT + 1;        // dX rows padded by one word: distinct features spread over banks
  float* xs = sm;                            // [S][TT]
  float* c1s = xs + (size_t)p.S * TT;        // [kK16Pass][TT] per-bucket coefficients
  float* dxs = c1s + (size_t)kK16Pass * TT;  // [S][TT + 1] dX tile
  __shared__ K16PassInfo ps;
  __shared__ int fq[kK16MaxS];
  __shared__ __align__(16) float dzs[NW][16][8];  // per warp: 16 neurons x 8 tokens of the current step
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int q = blockIdx.x, t0 = blockIdx.y * TT;
  const int ntok = min(TT, p.B - t0);
  k16_stage_x(xs, fq, p, q, t0, ntok);
  for (int e = threadIdx.x; e < p.S * TTD; e += kK16BwdThreads) dxs[e] = 0.f;
  const int h = lane >> 4, n = lane & 15;
  float* dzw = &dzs[warp][0][0];
  const int b_hi = min(max(__ldg(p.q_off + q + 1), 0), p.nbk);
  const int b_lo = min(max(__ldg(p.q_off + q), 0), b_hi);
  for (int p0 = b_lo; p0 < b_hi; p0 += kK16Pass) {
    const int np = min(kK16Pass, b_hi - p0);
    __syncthreads();
    k16_load_pass(ps, p, p0, np);
    __syncthreads();
    for (int e = threadIdx.x; e < np * TT; e += kK16BwdThreads) {
      const int i = e / TT, t = e - i * TT;
      const int g = ps.g[i];
      c1s[e] = (t < ntok && g >= 0 && g < p.G) ? __ldg(p.c1t + (int64_t)g * p.ldc + t0 + t) : 0.f;
    }
    __syncthreads();
    const int nrec = ps.rstart[np];
    for (int r = warp; r < nrec; r += NW) {
      const int i = k16_find(ps, np, r);
      const int g = ps.g[i];
      const int j16 = ps.first[i] + (r - ps.rstart[i]);
      if (g < 0 || g >= p.G || j16 < 0 || j16 >= p.NB16) continue;  // warp-uniform
      const int64_t f = (int64_t)g * p.NB16 + j16;
      const bool ok = j16 * 16 + n < __ldg(p.counts + g);
      float wr[16], wc[16];
      {
        const float4* wp = reinterpret_cast<const float4*>(p.w + (f * 16 + n) * 16);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const float4 a = __ldg(wp + c);
          wr[4 * c] = a.x; wr[4 * c + 1] = a.y; wr[4 * c + 2] = a.z; wr[4 * c + 3] = a.w;
        }
        const float* wcp = p.w + f * 256 + n;
#pragma unroll
        for (int m = 0; m < 16; ++m) wc[m] = __ldg(wcp + m * 16);
      }
      const float bb = __ldg(p.b + f * 16 + n);
      int off[16];
      k16_env(p.env, f, p.S - 1, TT, off);
      const int dxrow = min((int)__ldg(p.env + f * 16 + n), p.S - 1) * TTD;
      float dwacc[16];
#pragma unroll
      for (int k = 0; k < 16; ++k) dwacc[k] = 0.f;
      float dbacc = 0.f;
      const float* crow = c1s + i * TT;
      for (int tq = 0; tq < ntok; tq += 8) {
        const int col = tq + 4 * h;
        float xv[16][4];
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          const float4 v = *reinterpret_cast<const float4*>(xs + off[k] + col);
          xv[k][0] = v.x; xv[k][1] = v.y; xv[k][2] = v.z; xv[k][3] = v.w;
        }
        const float4 c4 = *reinterpret_cast<const float4*>(crow + col);
        const float cc[4] = {c4.x, c4.y, c4.z, c4.w};
        float z[4] = {bb, bb, bb, bb};
#pragma unroll
        for (int k = 0; k < 16; ++k)
#pragma unroll
          for (int j = 0; j < 4; ++j) z[j] = fmaf(wr[k], xv[k][j], z[j]);
        float dz[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) dz[j] = ok ? k16_dz<ACT>(cc[j], z[j]) : 0.f;
#pragma unroll
        for (int k = 0; k < 16; ++k)
#pragma unroll
          for (int j = 0; j < 4; ++j) dwacc[k] = fmaf(dz[j], xv[k][j], dwacc[k]);
        dbacc += (dz[0] + dz[1]) + (dz[2] + dz[3]);
        *reinterpret_cast<float4*>(dzw + n * 8 + 4 * h) = make_float4(dz[0], dz[1], dz[2], dz[3]);
        __syncwarp();
        float dxk[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int m = 0; m < 16; ++m) {
          const float4 d = *reinterpret_cast<const float4*>(dzw + m * 8 + 4 * h);
          dxk[0] = fmaf(d.x, wc[m], dxk[0]);
          dxk[1] = fmaf(d.y, wc[m], dxk[1]);
          dxk[2] = fmaf(d.z, wc[m], dxk[2]);
          dxk[3] = fmaf(d.w, wc[m], dxk[3]);
        }
        float* dst = dxs + dxrow + col;
#pragma unroll
        for (int j = 0; j < 4; ++j) atomicAdd(dst + j, dxk[j]);
        __syncwarp();
      }
#pragma unroll
      for (int k = 0; k < 16; ++k) dwacc[k] += __shfl_xor_sync(kFullMask, dwacc[k], 16);
      dbacc += __shfl_xor_sync(kFullMask, dbacc, 16);
      if (h == 0 && ok) {
        float* dwp = p.dw + (f * 16 + n) * 16;
#pragma unroll
        for (int c = 0; c < 4; ++c)
          red_add4(dwp + 4 * c, dwacc[4 * c], dwacc[4 * c + 1], dwacc[4 * c + 2], dwacc[4 * c + 3]);
        red_add(p.db + f * 16 + n, dbacc);
      }
    }
  }
  __syncthreads();
  const int n_el = p.S * ntok;
  for (int e = threadIdx.x; e < n_el; e += kK16BwdThreads) {
    const int s = e / ntok, t = e - s * ntok;
    const float v = dxs[s * TTD + t];
    if (v != 0.f) red_add(p.dx + (int64_t)(t0 + t) * p.lddx + fq[s], v);
  }
}

static size_t k16_fwd_smem(int S, int TT) { return ((size_t)S + kK16Pass) * TT * sizeof(float); }
static size_t k16_bwd_smem(int S, int TT) {
  return ((size_t)S * TT + (size_t)kK16Pass * TT + (size_t)S * (TT + 1)) * sizeof(float);
}

// Static shared memory of the kernels (pass info, feature list, dz slabs), with margin.
constexpr int kK16StaticBytes = 8 * 1024;

// Token chunk: a multiple of 16 (the forward step), at most 256, the largest that fits.
static int k16_pick_tt(int64_t B, int S, bool bwd, int optin) {
  int64_t tt = (B + 15) / 16 * 16;
  if (tt > 256) tt = 256;
  for (; tt >= 16; tt -= 16) {
    const size_t need = bwd ? k16_bwd_smem(S, (int)tt) : k16_fwd_smem(S, (int)tt);
    if ((int64_t)need + kK16StaticBytes <= optin) return (int)tt;
  }
  return -1;
}

static int k16_check(const GlK16Args& a, bool bwd) {
  if (a.B < 0 || a.D < 1 || a.D > 32767 || a.G < 1 || a.NB16 < 1 || a.Q < 0 || a.S < 16 || a.S > kK16MaxS)
    return GL_ERR_SHAPE;
  if (a.B > 2147483647LL || a.G * a.NB16 > 2147483647LL / 256 || a.nbuckets < 0 || a.nbuckets > 2147483646LL)
    return GL_ERR_SHAPE;
  if (a.B == 0 || a.Q == 0) return GL_OK;
  if (!a.x || !a.env || !a.feat || !a.buckets || !a.q_off || !a.rec_off || !a.w || !a.b || !a.counts)
    return GL_ERR_NULL;
  if (a.ldx < a.D) return GL_ERR_SHAPE;
  if (((uintptr_t)a.env & 15) || ((uintptr_t)a.w & 15) || ((uintptr_t)a.buckets & 15)) return GL_ERR_ALIGN;
  if (a.act != GL_ACT_RELU && a.act != GL_ACT_IDENTITY) return GL_ERR_UNSUPPORTED;
  if (!bwd) {
    if (!a.pre) return GL_ERR_NULL;
    if (a.ldp < a.G) return GL_ERR_SHAPE;
  } else {
    if (!a.c1t || !a.dx || !a.dw || !a.db) return GL_ERR_NULL;
    if (a.ldc < a.B || a.lddx < a.D) return GL_ERR_SHAPE;
    if (((uintptr_t)a.dw & 15) || ((uintptr_t)a.c1t & 3)) return GL_ERR_ALIGN;
  }
  return GL_OK;
}

static int k16_launch(const GlK16Args& a, void* stream, bool bwd) {
  int rc = k16_check(a, bwd);
  if (rc) return rc;
  if (a.B == 0 || a.Q == 0) return GL_OK;
  int optin = 0;
  if ((rc = device_smem_optin(&optin))) return rc;
  const int TT = a.tokens ? (int)a.tokens : k16_pick_tt(a.B, (int)a.S, bwd, optin);
  if (TT < 0) return GL_ERR_SMEM;
  if (TT < 16 || TT % 16 || TT > 1024) return GL_ERR_UNSUPPORTED;
  const size_t smem = bwd ? k16_bwd_smem((int)a.S, TT) : k16_fwd_smem((int)a.S, TT);
  if ((int64_t)smem + kK16StaticBytes > optin) return GL_ERR_SMEM;
  const int64_t chunks = (a.B + TT - 1) / TT;
  if (a.Q > 2147483647LL || chunks > 65535) return GL_ERR_SHAPE;
  const bool relu = a.act == GL_ACT_RELU;
  const void* kern = bwd ? (relu ? (const void*)k16_bwd_kernel<GL_ACT_RELU> : (const void*)k16_bwd_kernel<GL_ACT_IDENTITY>)
                         : (relu ? (const void*)k16_fwd_kernel<GL_ACT_RELU> : (const void*)k16_fwd_kernel<GL_ACT_IDENTITY>);
  if ((rc = ensure_dynamic_smem(kern, smem))) return rc;
  K16Params p;
  p.x = a.x; p.env = a.env; p.feat = a.feat; p.buckets = a.buckets; p.q_off = a.q_off; p.rec_off = a.rec_off;
  p.w = a.w; p.b = a.b; p.counts = a.counts; p.pre = a.pre; p.c1t = a.c1t; p.dx = a.dx; p.dw = a.dw; p.db = a.db;
  p.B = (int)a.B; p.D = (int)a.D; p.G = (int)a.G; p.NB16 = (int)a.NB16; p.S = (int)a.S; p.TT = TT; p.nbk = (int)a.nbuckets;
  p.ldx = a.ldx; p.ldp = a.ldp; p.ldc = a.ldc; p.lddx = a.lddx;
  const dim3 grid((unsigned)a.Q, (unsigned)chunks);
  cudaStream_t st = (cudaStream_t)stream;
  if (bwd) {
    if (relu) k16_bwd_kernel<GL_ACT_RELU><<<grid, kK16BwdThreads, smem, st>>>(p);
    else k16_bwd_kernel<GL_ACT_IDENTITY><<<grid, kK16BwdThreads, smem, st>>>(p);
  } else {
    if (relu) k16_fwd_kernel<GL_ACT_RELU><<<grid, kK16FwdThreads, smem, st>>>(p);
    else k16_fwd_kernel<GL_ACT_IDENTITY><<<grid, kK16FwdThreads, smem, st>>>(p);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e);
  count_launches(1);
  return GL_OK;
}

}  // namespace gl

extern "C" int gl_k16_fwd_f32(const GlK16Args* args, void* stream) {
  if (!args) return GL_ERR_NULL;
  return gl::k16_launch(*args, stream, false);
}

extern "C" int gl_k16_bwd_f32(const GlK16Args* args, void* stream) {
  if (!args) return GL_ERR_NULL;
  return gl::k16_launch(*args, stream, true);
}

extern "C" int gl_k16_auto_tokens(int64_t B, int64_t S, int32_t backward) {
  if (B < 1 || S < 16 || S > gl::kK16MaxS) return GL_ERR_SHAPE;
  int optin = 0;
  const int rc = gl::device_smem_optin(&optin);
  if (rc) return rc;
  const int tt = gl::k16_pick_tt(B, (int)S, backward != 0, optin);
  return tt < 0 ? GL_ERR_SMEM : tt;
}
