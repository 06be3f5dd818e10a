// Lane-per-neuron forward and backward for octet-arranged Mode-A storage (no counterpart in the
// reference: they compute the sums of gl_fwd_f32 / gl_bwd_f32 for the mean and sum pools with fp32
// parameters, i.e. the reference's Triton fwd_pool_kernel and bwd_dense_kernel on Mode-A layers,
// sparse_pooling/kernels/triton_fused.py:289-358 and :402-472).
//
// Octet storage.  gl_group_octets (octets.cu) permutes each group's neurons so that every 8 consecutive
// records form an "octet", and permutes each record's 8 (index, weight) pairs, such that at every input
// position k the octet's 8 records read features in 8 distinct residue classes d mod 8 (for ~97% of the
// (octet, k) pairs at the benchmarked geometry).  The kernels are correct on any storage order; the
// arrangement only removes shared-memory bank conflicts.
//
// Bank geometry.  A staged 4-token tile holds feature d's row of 4 fp32 values at byte 16 d, i.e. in
// the bank quad d mod 8 of a 128-byte wavefront.  A warp step covers 32 consecutive records, one per
// lane; lane quarter q = lane / 8 holds one octet.
//   gathers  one LDS.128 of the 4-token row per (record, k): each quarter reads 8 rows in 8 distinct
//            bank quads, one conflict-free wavefront per quarter (4 per instruction, the minimum);
//   scatter  (backward) for j = 0..3 the lane adds token j ^ q of its contribution at word 4 d + (j ^ q)
//            of an int32 dX tile: the quarters use disjoint bank offsets and each quarter's rows distinct
//            bank quads, so the 32 lanes of one atomic instruction hit 32 distinct banks.
// One lane per record reads the record once per 4 (backward) or 8 (forward) tokens, keeps the gathered
// inputs in registers and sums dW / db over its tokens without shuffles.  Weights and dW use the octet
// weight layout (oct_woff: per block of 32 records, weights 0-3 then weights 4-7), so the warp's 16-byte
// weight loads and dW reductions cover whole sectors.
//
// Backward dX accumulation: int32 fixed point at one scale per token for the whole thread block (all
// its groups), s[t] = K / (max_g |c1[t, g]| max|w|_g max|act'|), K = min(2^22, 0.9 * 2^31 / sum_g rowmax_g)
// over the block's groups g: every rounded term then has |q| <= K (exact rounding by the 1.5 * 2^23
// magic-number add), no tile word can exceed 0.9 * 2^31, and the rounding error per term is <= 0.5 / s[t].
// The tile is folded once per block into dx with coalesced fp32 reductions.  A token with a non-finite
// coefficient or bound gets a NaN dx row, as fp32 arithmetic would.
#include "common.cuh"

namespace gl {

constexpr int kOctThreads = 512;
constexpr int kOctWarps = kOctThreads / 32;

struct OctRec {
  int4 i;
  float4 w0, w1;
  float b;
};

// Offset (in floats) of record f's weights 0-3 in the octet weight layout: within each block of 32 records
// (f = 32 q + j, blocks aligned since a group's slot count is a multiple of 32) the records' weights 0-3
// come first, 16 bytes each, then their weights 4-7 at +128 floats; a warp's loads and reductions of one
// half then cover 512 contiguous bytes.
__device__ __forceinline__ int64_t oct_woff(int64_t f) { return (f & ~(int64_t)31) * 8 + (f & 31) * 4; }

__device__ __forceinline__ OctRec oct_load(const int16_t* __restrict__ idx, const float* __restrict__ w,
                                           const float* __restrict__ bias, int64_t f) {
  OctRec r;
  r.i = __ldg(reinterpret_cast<const int4*>(idx + f * 8));
  const float* wp = w + oct_woff(f);
  r.w0 = __ldg(reinterpret_cast<const float4*>(wp));
  r.w1 = __ldg(reinterpret_cast<const float4*>(wp + 128));
  r.b = __ldg(bias + f);
  return r;
}

// Index k of a record (k a compile-time constant after unrolling), clamped to [0, dmax].
__device__ __forceinline__ int oct_index(const int4& r, int k, int dmax) {
  const unsigned u = k < 2 ? (unsigned)r.x : k < 4 ? (unsigned)r.y : k < 6 ? (unsigned)r.z : (unsigned)r.w;
  return min((int)((k & 1) ? (u >> 16) : (u & 0xffffu)), dmax);
}

__device__ __forceinline__ float oct_weight(const OctRec& r, int k) {
  const float4& v = k < 4 ? r.w0 : r.w1;
  const int j = k & 3;
  return j == 0 ? v.x : j == 1 ? v.y : j == 2 ? v.z : v.w;
}

// o[j] = v[j ^ q] (q in 0..3).
__device__ __forceinline__ void oct_rot4(const float (&v)[4], int q, float (&o)[4]) {
  const bool b0 = (q & 1) != 0, b1 = (q & 2) != 0;
  const float t0 = b0 ? v[1] : v[0], t1 = b0 ? v[0] : v[1], t2 = b0 ? v[3] : v[2], t3 = b0 ? v[2] : v[3];
  o[0] = b1 ? t2 : t0;
  o[1] = b1 ? t3 : t1;
  o[2] = b1 ? t0 : t2;
  o[3] = b1 ? t1 : t3;
}

// ---------------------------------------------------------------------------------------------------
// Forward: 8 tokens per block, staged as two 4-token half tiles (tokens t0..t0+3 at byte 0, t0+4..t0+7
// at byte hoff), so each gather of a half is one conflict-free LDS.128 per octet.

struct OctFwdParams {
  const float* x;
  const int16_t* idx;
  const float* w;
  const float* bias;
  const int32_t* counts;
  float* pre;
  float* wabsmax;
  int B, D;
  int64_t NB, g0, g1, ldx, ldp;
  int pool, gpc, hoff;
};

template <int ACT, int HOFF>
__global__ void __launch_bounds__(kOctThreads, 1) fwd_octet_kernel(const OctFwdParams p) {
  extern __shared__ __align__(16) float smem[];
  __shared__ float red[kOctWarps][8];
  __shared__ float redw[kOctWarps];
  const int hoff = HOFF ? HOFF : p.hoff;
  const float4* xlo = reinterpret_cast<const float4*>(smem);
  const float4* xhi = reinterpret_cast<const float4*>(reinterpret_cast<const char*>(smem) + hoff);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int t0 = blockIdx.x * 8;
  const int D = p.D, dmax = D - 1;
  stage_tile<4, kOctThreads>(smem, p.x, t0, p.B, D, p.ldx);
  stage_tile<4, kOctThreads>(reinterpret_cast<float*>(reinterpret_cast<char*>(smem) + hoff), p.x, t0 + 4, p.B, D,
                             p.ldx);
  __syncthreads();
  const int slots = (int)(p.NB * 8);
  const int64_t gb = p.g0 + (int64_t)blockIdx.y * p.gpc;
  const int64_t ge = gb + p.gpc < p.g1 ? gb + p.gpc : p.g1;
  const bool want_w = p.wabsmax != nullptr && blockIdx.x == 0;
  for (int64_t g = gb; g < ge; ++g) {
    const int ng = min(__ldg(p.counts + g), slots);
    const int64_t fbase = g * (int64_t)slots;
    float acc[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) acc[t] = 0.f;
    float wmx = 0.f;
    int n = warp * 32 + lane;
    OctRec cur;
    if (n < ng) cur = oct_load(p.idx, p.w, p.bias, fbase + n);
    for (; n < ng; n += kOctThreads) {
      OctRec nxt;
      if (n + kOctThreads < ng) nxt = oct_load(p.idx, p.w, p.bias, fbase + n + kOctThreads);
      float z[8];
#pragma unroll
      for (int t = 0; t < 8; ++t) z[t] = cur.b;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int d = oct_index(cur.i, k, dmax);
        const float wk = oct_weight(cur, k);
        const float4 lo = xlo[d], hi = xhi[d];
        z[0] = fmaf(wk, lo.x, z[0]);
        z[1] = fmaf(wk, lo.y, z[1]);
        z[2] = fmaf(wk, lo.z, z[2]);
        z[3] = fmaf(wk, lo.w, z[3]);
        z[4] = fmaf(wk, hi.x, z[4]);
        z[5] = fmaf(wk, hi.y, z[5]);
        z[6] = fmaf(wk, hi.z, z[6]);
        z[7] = fmaf(wk, hi.w, z[7]);
        wmx = fmaxf(wmx, fabsf(wk));
      }
#pragma unroll
      for (int t = 0; t < 8; ++t) acc[t] += act_f<ACT>(z[t]);
      cur = nxt;
    }
#pragma unroll
    for (int off = 16; off; off >>= 1)
#pragma unroll
      for (int t = 0; t < 8; ++t) acc[t] += __shfl_xor_sync(kFullMask, acc[t], off);
    if (lane == 0)
#pragma unroll
      for (int t = 0; t < 8; ++t) red[warp][t] = acc[t];
    if (want_w) {
#pragma unroll
      for (int off = 16; off; off >>= 1) wmx = fmaxf(wmx, __shfl_xor_sync(kFullMask, wmx, off));
      if (lane == 0) redw[warp] = wmx;
    }
    __syncthreads();
    if (threadIdx.x < 8) {
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < kOctWarps; ++i) s += red[i][threadIdx.x];
      const int t = t0 + threadIdx.x;
      if (t < p.B) p.pre[(int64_t)t * p.ldp + (g - p.g0)] = p.pool == GL_POOL_MEAN ? s / (float)ng : s;
    }
    if (want_w && threadIdx.x == 32) {
      float m = 0.f;
#pragma unroll
      for (int i = 0; i < kOctWarps; ++i) m = fmaxf(m, redw[i]);
      p.wabsmax[g - p.g0] = m;
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------------------------------
// Backward: 4 tokens per block; the x tile at byte 0, the int32 dX tile at byte xoff.

struct OctBwdParams {
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
  const int32_t* fprefix;   // FOLD: [g1-g0+1][D] record inputs per feature over the groups g0 .. g0+i-1
  int B, D;
  int64_t NB, g0, g1, ldx, ldg, lddx;
  int pool, gpc, xoff;
};

// FOLD: the dX tile accumulates the rounding's raw bits, the fixed-point value plus the magic number's bit
// pattern 0x4B400000, and the flush subtracts that pattern once per record input of the word's feature in the
// block's groups (every record input adds to each of the feature's 4 token words once); integer sums modulo
// 2^32, so dX is bit for bit that of the per-term subtraction, one instruction fewer per shared atomic.
constexpr uint32_t kOctMagicBits = 0x4B400000u;

template <int ACT, int XOFF, bool FOLD>
__global__ void __launch_bounds__(kOctThreads, 1) bwd_octet_kernel(const OctBwdParams p) {
  extern __shared__ __align__(16) float smem[];
  __shared__ float s_scale[4], s_inv[4];
  __shared__ int s_bad[4];
  const int xoff = XOFF ? XOFF : p.xoff;
  const float4* xs = reinterpret_cast<const float4*>(smem);
  int* dxi = reinterpret_cast<int*>(reinterpret_cast<char*>(smem) + xoff);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int t0 = blockIdx.x * 4;
  const int D = p.D, dmax = D - 1;
  stage_tile<4, kOctThreads>(smem, p.x, t0, p.B, D, p.ldx);
  for (int e = threadIdx.x; e < D; e += kOctThreads) reinterpret_cast<int4*>(dxi)[e] = make_int4(0, 0, 0, 0);
  const int slots = (int)(p.NB * 8);
  const int64_t gb = p.g0 + (int64_t)blockIdx.y * p.gpc;
  const int64_t ge = gb + p.gpc < p.g1 ? gb + p.gpc : p.g1;
  if (threadIdx.x < 4) {  // the block's fixed-point scale of token t
    const int t = threadIdx.x;
    float m = 0.f;
    int64_t rows = 0;
    int bad = 0;
    if (t0 + t < p.B) {
      for (int64_t g = gb; g < ge; ++g) {
        const int ng = min(__ldg(p.counts + g), slots);
        if (ng <= 0) continue;
        float c = __ldg(p.gpre + (int64_t)(t0 + t) * p.ldg + (g - p.g0));
        if (p.pool == GL_POOL_MEAN) c /= (float)ng;
        const float a = fabsf(c) * __ldg(p.wabsmax + (g - p.g0));
        if (!(a <= 3.0e38f)) bad = 1;  // NaN or infinite
        else m = fmaxf(m, a);
        rows += max(__ldg(p.rowmax + (g - p.g0)), 0);
      }
    }
    const float K = fminf(4194304.f, 0.9f * 2147483648.f / (float)(rows > 1 ? rows : 1));
    const float den = m * dact_bound<ACT>();
    const float sc = (bad || !(den > 1e-30f)) ? 0.f : K / den;
    s_scale[t] = sc;
    s_inv[t] = sc > 0.f ? 1.f / sc : 0.f;
    s_bad[t] = bad;
  }
  __syncthreads();
  const int q = lane >> 3;
  float sc[4];
#pragma unroll
  for (int t = 0; t < 4; ++t) sc[t] = s_scale[t];
  for (int64_t g = gb; g < ge; ++g) {
    const int ng = min(__ldg(p.counts + g), slots);
    if (ng <= 0) continue;
    float c1[4], cq[4], cqr[4];
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      float c = t0 + t < p.B ? __ldg(p.gpre + (int64_t)(t0 + t) * p.ldg + (g - p.g0)) : 0.f;
      if (p.pool == GL_POOL_MEAN) c /= (float)ng;
      c1[t] = c;
      cq[t] = c * sc[t];
    }
    oct_rot4(cq, q, cqr);
    const int64_t fbase = g * (int64_t)slots;
    int n = warp * 32 + lane;
    OctRec cur;
    if (n < ng) cur = oct_load(p.idx, p.w, p.bias, fbase + n);
    for (; n < ng; n += kOctThreads) {
      OctRec nxt;
      if (n + kOctThreads < ng) nxt = oct_load(p.idx, p.w, p.bias, fbase + n + kOctThreads);
      int d[8];
      float4 xv[8];
      float z[4] = {cur.b, cur.b, cur.b, cur.b};
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        d[k] = oct_index(cur.i, k, dmax);
        xv[k] = xs[d[k]];
        const float wk = oct_weight(cur, k);
        z[0] = fmaf(wk, xv[k].x, z[0]);
        z[1] = fmaf(wk, xv[k].y, z[1]);
        z[2] = fmaf(wk, xv[k].z, z[2]);
        z[3] = fmaf(wk, xv[k].w, z[3]);
      }
      float da[4], dz[4], dar[4], dq[4];
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        da[t] = dact_f<ACT>(z[t]);
        dz[t] = c1[t] * da[t];
      }
      oct_rot4(da, q, dar);
#pragma unroll
      for (int j = 0; j < 4; ++j) dq[j] = cqr[j] * dar[j];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const float wk = oct_weight(cur, k);
        int* row = dxi + (d[k] << 2);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int v = FOLD ? __float_as_int(fmaf(dq[j], wk, 12582912.f))
                             : __float_as_int(fmaf(dq[j], wk, 12582912.f)) - (int)kOctMagicBits;
          atomicAdd(row + (j ^ q), v);
        }
      }
      float gw[8];
#pragma unroll
      for (int k = 0; k < 8; ++k)
        gw[k] = fmaf(dz[3], xv[k].w, fmaf(dz[2], xv[k].z, fmaf(dz[1], xv[k].y, dz[0] * xv[k].x)));
      const float gb_ = (dz[0] + dz[1]) + (dz[2] + dz[3]);
      if (dz[0] != 0.f || dz[1] != 0.f || dz[2] != 0.f || dz[3] != 0.f) {
        const int64_t f = fbase + n;
        float* dwp = p.dw + oct_woff(f);
        red_add4(dwp, gw[0], gw[1], gw[2], gw[3]);
        red_add4(dwp + 128, gw[4], gw[5], gw[6], gw[7]);
        red_add(p.db + f, gb_);
      }
      cur = nxt;
    }
  }
  __syncthreads();
  const float nan = __int_as_float(0x7fc00000);
  const int32_t* fp_lo = FOLD ? p.fprefix + (gb - p.g0) * (int64_t)D : nullptr;
  const int32_t* fp_hi = FOLD ? p.fprefix + (ge - p.g0) * (int64_t)D : nullptr;
  for (int e = threadIdx.x; e < D * 4; e += kOctThreads) {
    const int t = e / D, dd = e - t * D;
    if (t0 + t < p.B) {
      int word = dxi[dd * 4 + t];
      if (FOLD) word = (int)((uint32_t)word - (uint32_t)(__ldg(fp_hi + dd) - __ldg(fp_lo + dd)) * kOctMagicBits);
      const float v = s_bad[t] ? nan : (float)word * s_inv[t];
      if (v != 0.f) red_add(p.dx + (int64_t)(t0 + t) * p.lddx + dd, v);
    }
  }
}

// Shared memory of both kernels: two 16-byte-per-feature tiles.
static int64_t oct_smem(int64_t D) { return 32 * D; }

static int oct_groups_per_cta(int64_t tiles, int64_t G, int sms, int requested) {
  int gpc = requested;
  if (gpc <= 0) {
    const int64_t want = tiles * G / ((int64_t)sms * 32);
    gpc = (int)(want < 1 ? 1 : (want > 8 ? 8 : want));
  }
  while ((G + gpc - 1) / gpc > 65535) gpc *= 2;
  return gpc;
}

template <int ACT, int OFF>
static int launch_fwd_octet(const OctFwdParams& p, dim3 grid, size_t smem, cudaStream_t st) {
  auto kern = fwd_octet_kernel<ACT, OFF>;
  int rc = ensure_dynamic_smem((const void*)kern, smem);
  if (rc) return rc;
  kern<<<grid, kOctThreads, smem, st>>>(p);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e);
  count_launches(1);
  return GL_OK;
}

template <int ACT, int OFF>
static int launch_bwd_octet(const OctBwdParams& p, dim3 grid, size_t smem, cudaStream_t st) {
  auto kern = p.fprefix ? bwd_octet_kernel<ACT, OFF, true> : bwd_octet_kernel<ACT, OFF, false>;
  int rc = ensure_dynamic_smem((const void*)kern, smem);
  if (rc) return rc;
  kern<<<grid, kOctThreads, smem, st>>>(p);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e);
  count_launches(1);
  return GL_OK;
}

}  // namespace gl

using namespace gl;

extern "C" int gl_fwd_octet_f32(const GlFwdArgs* args, void* stream) {
  if (!args) return GL_ERR_NULL;
  const GlFwdArgs& a = *args;
  if (a.B < 0 || a.D < 1 || a.D > 32767 || a.NB < 1 || a.g0 < 0 || a.g1 < a.g0) return GL_ERR_SHAPE;
  if (a.pool != GL_POOL_MEAN && a.pool != GL_POOL_SUM) return GL_ERR_UNSUPPORTED;
  if (a.wdtype != GL_DTYPE_F32 || a.order || a.lidx || (a.tokens != 0 && a.tokens != 8)) return GL_ERR_UNSUPPORTED;
  if (a.act != GL_ACT_IDENTITY && a.act != GL_ACT_RELU && a.act != GL_ACT_GELU) return GL_ERR_UNSUPPORTED;
  if (a.B == 0 || a.g1 == a.g0) return GL_OK;
  if (!a.x || !a.idx || !a.w || !a.b || !a.counts || !a.pre) return GL_ERR_NULL;
  if (a.B > 2147483647LL || a.ldx < a.D || a.ldp < a.g1 - a.g0) return GL_ERR_SHAPE;
  if (((uintptr_t)a.idx & 15) || ((uintptr_t)a.w & 15)) return GL_ERR_ALIGN;
  int optin = 0, sms = 0;
  int rc = device_smem_optin(&optin);
  if (rc) return rc;
  if ((rc = device_sm_count(&sms))) return rc;
  const int64_t smem = oct_smem(a.D);
  if (smem + 1024 > optin) return GL_ERR_SMEM;
  const int64_t tiles = (a.B + 7) / 8, G = a.g1 - a.g0;
  const int gpc = oct_groups_per_cta(tiles, G, sms, a.groups_per_cta);
  const int64_t chunks = (G + gpc - 1) / gpc;
  if (tiles > 2147483647LL || chunks > 65535) return GL_ERR_SHAPE;
  OctFwdParams p{a.x, a.idx, a.w, a.b, a.counts, a.pre, a.wabsmax, (int)a.B, (int)a.D, a.NB, a.g0, a.g1, a.ldx,
                 a.ldp, a.pool, gpc, (int)(16 * a.D)};
  const dim3 grid((unsigned)tiles, (unsigned)chunks);
  cudaStream_t st = (cudaStream_t)stream;
  const bool fixed_off = a.D == 4096;
  switch (a.act) {
    case GL_ACT_IDENTITY:
      return fixed_off ? launch_fwd_octet<GL_ACT_IDENTITY, 65536>(p, grid, smem, st)
                       : launch_fwd_octet<GL_ACT_IDENTITY, 0>(p, grid, smem, st);
    case GL_ACT_RELU:
      return fixed_off ? launch_fwd_octet<GL_ACT_RELU, 65536>(p, grid, smem, st)
                       : launch_fwd_octet<GL_ACT_RELU, 0>(p, grid, smem, st);
    default:
      return fixed_off ? launch_fwd_octet<GL_ACT_GELU, 65536>(p, grid, smem, st)
                       : launch_fwd_octet<GL_ACT_GELU, 0>(p, grid, smem, st);
  }
}

static int bwd_octet_run(const GlBwdArgs* args, const int32_t* fprefix, void* stream) {
  if (!args) return GL_ERR_NULL;
  const GlBwdArgs& a = *args;
  if (a.B < 0 || a.D < 1 || a.D > 32767 || a.NB < 1 || a.g0 < 0 || a.g1 < a.g0) return GL_ERR_SHAPE;
  if (a.pool != GL_POOL_MEAN && a.pool != GL_POOL_SUM) return GL_ERR_UNSUPPORTED;
  if (a.wdtype != GL_DTYPE_F32 || a.order || a.lidx || (a.tokens != 0 && a.tokens != 4)) return GL_ERR_UNSUPPORTED;
  if (a.act != GL_ACT_IDENTITY && a.act != GL_ACT_RELU && a.act != GL_ACT_GELU) return GL_ERR_UNSUPPORTED;
  if (a.B == 0 || a.g1 == a.g0) return GL_OK;
  if (!a.x || !a.idx || !a.w || !a.b || !a.counts || !a.gpre || !a.dx || !a.dw || !a.db) return GL_ERR_NULL;
  if (!a.wabsmax || !a.rowmax) return GL_ERR_NULL;  // the fixed-point bounds are required
  if (a.B > 2147483647LL || a.ldx < a.D || a.ldg < a.g1 - a.g0 || a.lddx < a.D) return GL_ERR_SHAPE;
  if (((uintptr_t)a.idx & 15) || ((uintptr_t)a.w & 15) || ((uintptr_t)a.dw & 15)) return GL_ERR_ALIGN;
  int optin = 0, sms = 0;
  int rc = device_smem_optin(&optin);
  if (rc) return rc;
  if ((rc = device_sm_count(&sms))) return rc;
  const int64_t smem = oct_smem(a.D);
  if (smem + 1024 > optin) return GL_ERR_SMEM;
  const int64_t tiles = (a.B + 3) / 4, G = a.g1 - a.g0;
  const int gpc = oct_groups_per_cta(tiles, G, sms, a.groups_per_cta);
  const int64_t chunks = (G + gpc - 1) / gpc;
  if (tiles > 2147483647LL || chunks > 65535) return GL_ERR_SHAPE;
  OctBwdParams p{a.x, a.idx, a.w, a.b, a.counts, a.gpre, a.dx, a.dw, a.db, a.wabsmax, a.rowmax, fprefix, (int)a.B,
                 (int)a.D, a.NB, a.g0, a.g1, a.ldx, a.ldg, a.lddx, a.pool, gpc, (int)(16 * a.D)};
  const dim3 grid((unsigned)tiles, (unsigned)chunks);
  cudaStream_t st = (cudaStream_t)stream;
  const bool fixed_off = a.D == 4096;
  switch (a.act) {
    case GL_ACT_IDENTITY:
      return fixed_off ? launch_bwd_octet<GL_ACT_IDENTITY, 65536>(p, grid, smem, st)
                       : launch_bwd_octet<GL_ACT_IDENTITY, 0>(p, grid, smem, st);
    case GL_ACT_RELU:
      return fixed_off ? launch_bwd_octet<GL_ACT_RELU, 65536>(p, grid, smem, st)
                       : launch_bwd_octet<GL_ACT_RELU, 0>(p, grid, smem, st);
    default:
      return fixed_off ? launch_bwd_octet<GL_ACT_GELU, 65536>(p, grid, smem, st)
                       : launch_bwd_octet<GL_ACT_GELU, 0>(p, grid, smem, st);
  }
}

extern "C" int gl_bwd_octet_f32(const GlBwdArgs* args, void* stream) { return bwd_octet_run(args, nullptr, stream); }

extern "C" int gl_bwd_octet_prefix_f32(const GlBwdArgs* args, const int32_t* feat_prefix, void* stream) {
  if (!feat_prefix) return GL_ERR_NULL;
  if ((uintptr_t)feat_prefix & 3) return GL_ERR_ALIGN;
  return bwd_octet_run(args, feat_prefix, stream);
}

// ---------------------------------------------------------------------------------------------------
// Record inputs per feature, cumulated over groups: out[i][d] = number of (record, input) pairs of groups
// g0 .. g0+i-1 whose index (clamped to D-1, as the kernels clamp) is d, over each group's valid records.

namespace gl {

__global__ void __launch_bounds__(512) group_feature_hist_kernel(const int16_t* __restrict__ idx,
                                                                 const int32_t* __restrict__ counts, int D,
                                                                 int64_t NB, int64_t g0, int32_t* __restrict__ out) {
  extern __shared__ int hist[];
  const int64_t g = g0 + blockIdx.x;
  for (int d = threadIdx.x; d < D; d += blockDim.x) hist[d] = 0;
  __syncthreads();
  const int slots = (int)(NB * 8);
  const int ng = min(__ldg(counts + g), slots);
  const int16_t* rec = idx + g * (int64_t)slots * 8;
  for (int e = threadIdx.x; e < ng * 8; e += blockDim.x) {
    const int d = min((int)(uint16_t)__ldg(rec + e), D - 1);
    atomicAdd(&hist[d], 1);
  }
  __syncthreads();
  int32_t* row = out + (int64_t)(blockIdx.x + 1) * D;
  for (int d = threadIdx.x; d < D; d += blockDim.x) row[d] = hist[d];
}

__global__ void group_feature_scan_kernel(int32_t* __restrict__ out, int D, int64_t G) {
  const int d = blockIdx.x * blockDim.x + threadIdx.x;
  if (d >= D) return;
  int32_t acc = 0;
  out[d] = 0;
  for (int64_t i = 1; i <= G; ++i) {
    acc += out[i * D + d];
    out[i * D + d] = acc;
  }
}

}  // namespace gl

extern "C" int gl_group_feature_prefix(const int16_t* idx, const int32_t* counts, int64_t D, int64_t NB, int64_t g0,
                                       int64_t g1, int32_t* out, void* stream) {
  if (D < 1 || D > 32767 || NB < 1 || g0 < 0 || g1 < g0 || g1 - g0 > 2147483647LL) return GL_ERR_SHAPE;
  if (!out) return GL_ERR_NULL;
  cudaStream_t st = (cudaStream_t)stream;
  const int64_t G = g1 - g0;
  if (G > 0) {
    if (!idx || !counts) return GL_ERR_NULL;
    if ((uintptr_t)idx & 15) return GL_ERR_ALIGN;
    const size_t smem = (size_t)D * 4;
    int rc = ensure_dynamic_smem((const void*)group_feature_hist_kernel, smem);
    if (rc) return rc;
    group_feature_hist_kernel<<<(unsigned)G, 512, smem, st>>>(idx, counts, (int)D, NB, g0, out);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_cuda_error(e);
    count_launches(1);
  }
  group_feature_scan_kernel<<<(unsigned)((D + 255) / 256), 256, 0, st>>>(out, (int)D, G);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e);
  count_launches(1);
  return GL_OK;
}
