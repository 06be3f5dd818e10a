// Mode B with bf16 parameters and input-supergroup connectivity: backward of the mean and sum pools
// on the tensor cores, one CTA per (token tile, chunk of buckets of one input set).
//
// Replaces the reference's grouped supergroup backward (sparse_pooling/kernels/cuda/sparse_pool_sg.cuh,
// sg_dx / sg_dw) for bf16 fragment-packed layers.  Every record of a bucket (q, g, first unit, units)
// reads only features of the set feat[q] (S sorted features, supergroups.py), so a CTA whose work
// all belongs to set q stages only those S rows of x (as the bf16 slab) and keeps a dX tile of S
// rows; with S << D the token tile grows (128 tokens at S = 64 instead of 32 with all D rows), which
// divides the per-tile costs -- the packed weight loads and the dw / db global reductions -- by 4.
// A D-entry shared map translates a record's global features to slab rows.
//
// The per-quad work is the group-chunk kernel's (modeb_tc_bwd.cuh: z, the split-precision dz, the
// dX partials by mma into the shared tile, dW by mma into the packed gradient).  The CTA's quads --
// the units of its buckets, concatenated -- are dealt to the warps in turn.  The dX tile is int32
// fixed point at one power-of-two scale per token for the whole chunk, bounded by
//   C * max|act'| * sum over the chunk's buckets b of m_b * |c1[t, g_b]| * max|w|_{g_b} <= 2^30
// (m_b = the bucket's largest number of record inputs on one feature), or fp32 without the bounds.
// It is added to dx once per CTA.
#include "modeb_tc_bwd.cuh"

namespace gl {

constexpr int kSetMaxChunk = 256;  // buckets per chunk (the CTA keeps their quad offsets in shared memory)

struct SetParams {
  const int16_t* feat;      // [Q, S]
  const int32_t* buckets;   // [n, 4] (q, g, first unit, units)
  const int32_t* chunks;    // [m, 3] (q, first bucket, end bucket)
  const int32_t* rowmax;    // [n] or NULL
  const float* wabsmax;     // [g1 - g0] or NULL
  int S;
};

template <int BM, int NT, int ACT, bool FIXED>
__global__ void __launch_bounds__(kTcBwdThreads, 1) tc_bwd_sets_kernel(const TcParams p, const SetParams sp) {
  constexpr int MT = BM / 16;
  constexpr int NW = kTcBwdThreads / 32;
  constexpr int CH = BM / 8;
  constexpr int QPU = NT >= 4 ? NT / 4 : 1;  // fragment quads per assignment unit
  extern __shared__ __align__(128) unsigned char tc_smem[];
  const int S = sp.S;
  float* dxs = reinterpret_cast<float*>(tc_smem + (size_t)S * BM * 2);
  int* dxi = reinterpret_cast<int*>(dxs);
  int16_t* lmap = reinterpret_cast<int16_t*>(tc_smem + (size_t)S * BM * 6);
  __shared__ int qoff[kSetMaxChunk + 1];  // first flat quad of each bucket of the chunk
  __shared__ float qsc[FIXED ? BM : 1], qinv[FIXED ? BM : 1];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int t0 = blockIdx.x * BM;
  const int c = blockIdx.y;
  const int q = sp.chunks[3 * c], lo = sp.chunks[3 * c + 1];
  const int hi = min(max(sp.chunks[3 * c + 2], lo), lo + kSetMaxChunk);
  const int16_t* fq = sp.feat + (int64_t)q * S;
  const uint32_t slab = (uint32_t)__cvta_generic_to_shared(tc_smem);
  const int slots = (int)(p.NB * p.C);
  // stage the set's rows: item = (row i, 8-token chunk k); consecutive threads take consecutive rows
  for (int it = threadIdx.x; it < S * CH; it += kTcBwdThreads) {
    const int i = it % S, k = it / S;
    const int f = min((int)(uint16_t)__ldg(fq + i), p.D - 1);
    float v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int t = t0 + 8 * k + u;
      v[u] = t < p.B ? __ldg(p.x + (int64_t)t * p.ldx + f) : 0.f;
    }
    uint32_t w4[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) w4[u] = pack_bf16(v[2 * u], v[2 * u + 1]);
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(tc_chunk<BM>(slab, i, k)), "r"(w4[0]), "r"(w4[1]),
                 "r"(w4[2]), "r"(w4[3])
                 : "memory");
  }
  for (int i = threadIdx.x; i < S * BM; i += kTcBwdThreads) dxs[i] = 0.f;
  for (int i = threadIdx.x; i < p.D; i += kTcBwdThreads) lmap[i] = 0;  // rows stay in the slab for any index
  __syncthreads();
  for (int i = threadIdx.x; i < S; i += kTcBwdThreads) lmap[min((int)(uint16_t)__ldg(fq + i), p.D - 1)] = (int16_t)i;
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int b = lo; b < hi; ++b) {
      qoff[b - lo] = acc;
      const int g = sp.buckets[4 * b + 1];
      const int ng = min(p.counts[g], slots);
      const int qa = sp.buckets[4 * b + 2] * QPU, qb = min((sp.buckets[4 * b + 2] + sp.buckets[4 * b + 3]) * QPU,
                                                          (ng + 31) >> 5);
      acc += qb > qa && g >= p.g0 && g < p.g1 ? qb - qa : 0;
    }
    qoff[hi - lo] = acc;
  }
  if constexpr (FIXED) {
    if (threadIdx.x < BM) {
      const int t = t0 + threadIdx.x;
      float bound = 0.f;
      if (t < p.B)
        for (int b = lo; b < hi; ++b) {
          const int g = sp.buckets[4 * b + 1];
          if (g < p.g0 || g >= p.g1) continue;
          const int ng = min(p.counts[g], slots);
          if (ng == 0) continue;
          const float gv = __ldg(p.gpre + (int64_t)t * p.ldg + (g - p.g0));
          const float cv = p.pool == GL_POOL_MEAN ? gv / (float)ng : gv;
          bound += fabsf(cv) * (float)__ldg(sp.rowmax + b) * __ldg(sp.wabsmax + (g - p.g0));
        }
      bound *= (float)p.C * (ACT == GL_ACT_GELU ? 1.13f : 1.f);
      float s_ = 0.f, i_ = 0.f;
      if (!(bound <= 3.0e38f)) {
        i_ = __int_as_float(0x7fc00000);  // non-finite bound: NaN for the token's dx
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
  const int total = qoff[hi - lo];
  int bi = 0, gcur = -1, ng = 0;
  float c1[MT][2];
  // the group and quad of flat quad f (nb: its bucket, advanced monotonically by the caller's order)
  auto locate = [&](int f, int& nb, int& gg, int& qq) {
    while (f >= qoff[nb + 1]) ++nb;
    const int b = lo + nb;
    gg = sp.buckets[4 * b + 1];
    qq = sp.buckets[4 * b + 2] * QPU + (f - qoff[nb]);
  };
  int nbi = 0, ng_next = 0, qn = 0;
  TcQuad nxt;
  if (warp < total) {
    locate(warp, nbi, ng_next, qn);
    nxt = tc_load_quad<NT>(p, ng_next, qn, lane);
  }
  for (int fq_ = warp; fq_ < total; fq_ += NW) {
    const TcQuad cur = nxt;
    const int g = ng_next, qq = qn;
    bi = nbi;
    if (fq_ + NW < total) {  // the next quad's operands load while this one computes
      locate(fq_ + NW, nbi, ng_next, qn);
      nxt = tc_load_quad<NT>(p, ng_next, qn, lane);
    }
    if (g != gcur) {
      gcur = g;
      ng = min(p.counts[g], slots);
#pragma unroll
      for (int m = 0; m < MT; ++m)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int t = t0 + 16 * m + 8 * h + (lane >> 2);
          const float gv = t < p.B ? __ldg(p.gpre + (int64_t)t * p.ldg + (g - p.g0)) : 0.f;
          c1[m][h] = p.pool == GL_POOL_MEAN ? gv / (float)ng : gv;
        }
    }
    tc_bwd_quad<BM, NT, ACT, FIXED, true>(p, g, qq, ng, cur, c1, sc, slab, dxs, dxi, lmap, lane);
  }
  __syncthreads();
  // dx[t0 + t, feat[q][i]] += tile row i; consecutive threads take consecutive rows of one token
  for (int it = threadIdx.x; it < S * BM; it += kTcBwdThreads) {
    const int t = it / S, i = it - t * S;
    const int o = dxs_off<BM>(i, t);
    float v;
    bool add;
    if constexpr (FIXED) {
      const int qv = dxi[o];
      const float inv = qinv[t];
      v = (float)qv * inv;
      add = qv != 0 || inv != inv;
    } else {
      v = dxs[o];
      add = v != 0.f;
    }
    if (t0 + t < p.B && add) atomicAdd(p.dx + (int64_t)(t0 + t) * p.lddx + min((int)(uint16_t)__ldg(fq + i), p.D - 1), v);
  }
}

// Forward (mean, sum) over the same chunks: the set's rows staged as above, the chunk's quads dealt to
// the warps; a warp sums act(z) over the valid slots of its quads per token row and adds the partial of
// each (token, bucket) to pre (one fp32 atomic; the entry point zeroes pre first).
template <int BM, int NT, int ACT>
__global__ void __launch_bounds__(kTcFwdThreads, 1) tc_fwd_sets_kernel(const TcParams p, const SetParams sp) {
  constexpr int MT = BM / 16;
  constexpr int NW = kTcFwdThreads / 32;
  constexpr int CH = BM / 8;
  constexpr int QPU = NT >= 4 ? NT / 4 : 1;
  extern __shared__ __align__(128) unsigned char tc_smem[];
  const int S = sp.S;
  int16_t* lmap = reinterpret_cast<int16_t*>(tc_smem + (size_t)S * BM * 2);
  __shared__ int qoff[kSetMaxChunk + 1];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int t0 = blockIdx.x * BM;
  const int c = blockIdx.y;
  const int q = sp.chunks[3 * c], lo = sp.chunks[3 * c + 1];
  const int hi = min(max(sp.chunks[3 * c + 2], lo), lo + kSetMaxChunk);
  const int16_t* fq = sp.feat + (int64_t)q * S;
  const uint32_t slab = (uint32_t)__cvta_generic_to_shared(tc_smem);
  const int slots = (int)(p.NB * p.C);
  for (int it = threadIdx.x; it < S * CH; it += kTcFwdThreads) {
    const int i = it % S, k = it / S;
    const int f = min((int)(uint16_t)__ldg(fq + i), p.D - 1);
    float v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int t = t0 + 8 * k + u;
      v[u] = t < p.B ? __ldg(p.x + (int64_t)t * p.ldx + f) : 0.f;
    }
    uint32_t w4[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) w4[u] = pack_bf16(v[2 * u], v[2 * u + 1]);
    asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(tc_chunk<BM>(slab, i, k)), "r"(w4[0]), "r"(w4[1]),
                 "r"(w4[2]), "r"(w4[3])
                 : "memory");
  }
  for (int i = threadIdx.x; i < p.D; i += kTcFwdThreads) lmap[i] = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < S; i += kTcFwdThreads) lmap[min((int)(uint16_t)__ldg(fq + i), p.D - 1)] = (int16_t)i;
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int b = lo; b < hi; ++b) {
      qoff[b - lo] = acc;
      const int g = sp.buckets[4 * b + 1];
      const int ng = min(p.counts[g], slots);
      const int qa = sp.buckets[4 * b + 2] * QPU, qb = min((sp.buckets[4 * b + 2] + sp.buckets[4 * b + 3]) * QPU,
                                                          (ng + 31) >> 5);
      acc += qb > qa && g >= p.g0 && g < p.g1 ? qb - qa : 0;
    }
    qoff[hi - lo] = acc;
  }
  __syncthreads();
  const int total = qoff[hi - lo];
  const int cq = 2 * (lane & 3);
  auto locate = [&](int f, int& nb, int& gg, int& qq) {
    while (f >= qoff[nb + 1]) ++nb;
    const int b = lo + nb;
    gg = sp.buckets[4 * b + 1];
    qq = sp.buckets[4 * b + 2] * QPU + (f - qoff[nb]);
  };
  float acc[MT][2];
  int gcur = -1, ng = 0;
  // fold the lane quad and add this warp's partial of (token, bucket group) to pre
  auto flush = [&]() {
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        acc[m][h] += __shfl_xor_sync(kFullMask, acc[m][h], 1);
        acc[m][h] += __shfl_xor_sync(kFullMask, acc[m][h], 2);
      }
    if ((lane & 3) == 0) {
      const float scale = p.pool == GL_POOL_MEAN ? 1.f / (float)ng : 1.f;
#pragma unroll
      for (int m = 0; m < MT; ++m)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int t = t0 + 16 * m + 8 * h + (lane >> 2);
          if (t < p.B) atomicAdd(p.pre + (int64_t)t * p.ldp + (gcur - p.g0), acc[m][h] * scale);
        }
    }
  };
  int nbi = 0, gn = 0, qn = 0;
  TcQuad nxt;
  if (warp < total) {
    locate(warp, nbi, gn, qn);
    nxt = tc_load_quad<NT>(p, gn, qn, lane);
  }
  for (int f_ = warp; f_ < total; f_ += NW) {
    const TcQuad cur = nxt;
    const int g = gn, qq = qn;
    if (f_ + NW < total) {
      locate(f_ + NW, nbi, gn, qn);
      nxt = tc_load_quad<NT>(p, gn, qn, lane);
    }
    if (g != gcur) {  // warp-uniform
      if (gcur >= 0) flush();
      gcur = g;
      ng = min(p.counts[g], slots);
#pragma unroll
      for (int m = 0; m < MT; ++m) acc[m][0] = acc[m][1] = 0.f;
    }
    uint32_t a[MT][2];
#pragma unroll
    for (int fi = 0; fi < 4; ++fi) {
      if (NT >= 4 ? fi == 0 : fi % NT == 0)
        tc_gather<BM>(a, slab, (int)lmap[tc_row<NT>(cur, NT >= 4 ? 0 : fi / NT, lane)], lane);
      const uint32_t bw = tc_word(cur.w, fi), bb = tc_word(cur.b, fi);
      const float b0 = bf16_lo(bb), b1 = bf16_hi(bb);
      const int s0 = 32 * qq + 8 * fi + cq;
      const bool v0 = s0 < ng, v1 = s0 + 1 < ng;
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        float d[4];
        const float cc[4] = {b0, b1, b0, b1};
        mma_bf16_k8(d, a[m], bw, cc);
#pragma unroll
        for (int h = 0; h < 2; ++h)
          acc[m][h] += (v0 ? act_f<ACT>(d[2 * h]) : 0.f) + (v1 ? act_f<ACT>(d[2 * h + 1]) : 0.f);
      }
    }
  }
  if (gcur >= 0) flush();
}

// pre[t, 0 .. g1-g0) = 0 before the set forward's atomics (NaN for the mean of a group without valid slots,
// as the generic forward computes it).
__global__ void tc_zero_pre_kernel(float* pre, const int32_t* counts, int64_t B, int64_t G0, int64_t G, int64_t ldp,
                                   int slots, int mean) {
  const int64_t n = B * G;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = e / G, g = e - t * G;
    pre[t * ldp + g] = mean && min(counts[G0 + g], slots) == 0 ? __int_as_float(0x7fc00000) : 0.f;
  }
}

static int64_t sets_fwd_smem(int64_t S, int64_t D, int BM) { return S * BM * 2 + ((D * 2 + 15) & ~15LL); }

static int64_t sets_smem(int64_t S, int64_t D, int BM) { return S * BM * 6 + ((D * 2 + 15) & ~15LL); }

template <int BM, int NT, int ACT, bool FIXED>
static int sets_launch(const TcParams& p, const SetParams& sp, int64_t nchunks, cudaStream_t st) {
  const size_t smem = (size_t)sets_smem(sp.S, p.D, BM);
  const void* kern = (const void*)tc_bwd_sets_kernel<BM, NT, ACT, FIXED>;
  int rc = ensure_dynamic_smem(kern, smem);
  if (rc) return rc;
  const int64_t tiles = (p.B + BM - 1) / BM;
  if (tiles > 2147483647LL || nchunks > 65535) return GL_ERR_SHAPE;
  tc_bwd_sets_kernel<BM, NT, ACT, FIXED><<<dim3((unsigned)tiles, (unsigned)nchunks), kTcBwdThreads, smem, st>>>(p, sp);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e);
  count_launches(1);
  return GL_OK;
}

template <int BM, int NT, bool FIXED>
static int sets_act(const TcParams& p, const SetParams& sp, int64_t m, int act, cudaStream_t st) {
  switch (act) {
    case GL_ACT_IDENTITY: return sets_launch<BM, NT, GL_ACT_IDENTITY, FIXED>(p, sp, m, st);
    case GL_ACT_RELU: return sets_launch<BM, NT, GL_ACT_RELU, FIXED>(p, sp, m, st);
    case GL_ACT_GELU: return sets_launch<BM, NT, GL_ACT_GELU, FIXED>(p, sp, m, st);
    default: return GL_ERR_UNSUPPORTED;
  }
}

template <int BM>
static int sets_nt(const TcParams& p, const SetParams& sp, int64_t m, int act, cudaStream_t st) {
  const bool fx = sp.rowmax != nullptr;
  switch (p.C) {
    case 8: return fx ? sets_act<BM, 1, true>(p, sp, m, act, st) : sets_act<BM, 1, false>(p, sp, m, act, st);
    case 16: return fx ? sets_act<BM, 2, true>(p, sp, m, act, st) : sets_act<BM, 2, false>(p, sp, m, act, st);
    case 32: return fx ? sets_act<BM, 4, true>(p, sp, m, act, st) : sets_act<BM, 4, false>(p, sp, m, act, st);
    default: return fx ? sets_act<BM, 8, true>(p, sp, m, act, st) : sets_act<BM, 8, false>(p, sp, m, act, st);
  }
}

template <int BM, int NT, int ACT>
static int sets_fwd_launch(const TcParams& p, const SetParams& sp, int64_t nchunks, cudaStream_t st) {
  const size_t smem = (size_t)sets_fwd_smem(sp.S, p.D, BM);
  const void* kern = (const void*)tc_fwd_sets_kernel<BM, NT, ACT>;
  int rc = ensure_dynamic_smem(kern, smem);
  if (rc) return rc;
  const int64_t tiles = (p.B + BM - 1) / BM;
  if (tiles > 2147483647LL || nchunks > 65535) return GL_ERR_SHAPE;
  tc_fwd_sets_kernel<BM, NT, ACT><<<dim3((unsigned)tiles, (unsigned)nchunks), kTcFwdThreads, smem, st>>>(p, sp);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e);
  count_launches(1);
  return GL_OK;
}

template <int BM, int NT>
static int sets_fwd_act(const TcParams& p, const SetParams& sp, int64_t m, int act, cudaStream_t st) {
  switch (act) {
    case GL_ACT_IDENTITY: return sets_fwd_launch<BM, NT, GL_ACT_IDENTITY>(p, sp, m, st);
    case GL_ACT_RELU: return sets_fwd_launch<BM, NT, GL_ACT_RELU>(p, sp, m, st);
    case GL_ACT_GELU: return sets_fwd_launch<BM, NT, GL_ACT_GELU>(p, sp, m, st);
    default: return GL_ERR_UNSUPPORTED;
  }
}

template <int BM>
static int sets_fwd_nt(const TcParams& p, const SetParams& sp, int64_t m, int act, cudaStream_t st) {
  switch (p.C) {
    case 8: return sets_fwd_act<BM, 1>(p, sp, m, act, st);
    case 16: return sets_fwd_act<BM, 2>(p, sp, m, act, st);
    case 32: return sets_fwd_act<BM, 4>(p, sp, m, act, st);
    default: return sets_fwd_act<BM, 8>(p, sp, m, act, st);
  }
}

int tc_prepare(const GlSharedArgs& a, bool bwd, TcParams& p);

// Largest token tile in {128, 64, 32} whose set slab and feature map fit (forward).
static int sets_fwd_pick_tokens(int64_t S, int64_t D, int optin) {
  for (int BM = 128; BM >= 32; BM >>= 1)
    if (sets_fwd_smem(S, D, BM) + kTcStaticSmem + 2048 <= optin) return BM;
  return GL_ERR_SMEM;
}

// Largest token tile in {128, 64, 32} whose set slab, dX tile and feature map fit.
static int sets_pick_tokens(int64_t S, int64_t D, int optin) {
  for (int BM = 128; BM >= 32; BM >>= 1)
    if (sets_smem(S, D, BM) + kTcStaticSmem + 2048 <= optin) return BM;
  return GL_ERR_SMEM;
}

}  // namespace gl

using namespace gl;

extern "C" int gl_bwd_shared_tc_sets(const GlSharedArgs* args, const GlSetArgs* sets, void* stream) {
  if (!args || !sets) return GL_ERR_NULL;
  const GlSharedArgs& a = *args;
  const GlSetArgs& s = *sets;
  if ((s.rowmax == nullptr) != (s.wabsmax == nullptr)) return GL_ERR_NULL;
  TcParams p;
  int rc = tc_prepare(a, true, p);
  if (rc) return rc > 0 ? GL_OK : rc;
  if (s.nchunks == 0) return GL_OK;
  if (!s.feat || !s.buckets || !s.chunks) return GL_ERR_NULL;
  if (s.S < 8 || s.S > a.D || s.S > 32767 || s.nchunks < 0 || s.max_chunk > kSetMaxChunk || s.max_chunk < 1)
    return GL_ERR_SHAPE;
  int optin = 0;
  if ((rc = device_smem_optin(&optin))) return rc;
  int BM = a.tokens;
  if (BM == 0) {
    BM = sets_pick_tokens(s.S, a.D, optin);
    if (BM < 0) return BM;
  } else if (BM != 32 && BM != 64 && BM != 128) {
    return GL_ERR_UNSUPPORTED;
  }
  if (sets_smem(s.S, a.D, BM) + kTcStaticSmem + 2048 > optin) return GL_ERR_SMEM;
  const SetParams sp{s.feat, s.buckets, s.chunks, s.rowmax, s.wabsmax, (int)s.S};
  cudaStream_t st = (cudaStream_t)stream;
  switch (BM) {
    case 128: return sets_nt<128>(p, sp, s.nchunks, a.act, st);
    case 64: return sets_nt<64>(p, sp, s.nchunks, a.act, st);
    default: return sets_nt<32>(p, sp, s.nchunks, a.act, st);
  }
}

extern "C" int gl_fwd_shared_tc_sets(const GlSharedArgs* args, const GlSetArgs* sets, void* stream) {
  if (!args || !sets) return GL_ERR_NULL;
  const GlSharedArgs& a = *args;
  const GlSetArgs& s = *sets;
  if (a.pool != GL_POOL_MEAN && a.pool != GL_POOL_SUM) return GL_ERR_UNSUPPORTED;
  TcParams p;
  int rc = tc_prepare(a, false, p);
  if (rc) return rc > 0 ? GL_OK : rc;
  if (!s.feat || !s.buckets || (!s.chunks && s.nchunks)) return GL_ERR_NULL;
  if (s.S < 8 || s.S > a.D || s.S > 32767 || s.nchunks < 0 || s.max_chunk > kSetMaxChunk || s.max_chunk < 1)
    return GL_ERR_SHAPE;
  int optin = 0, sms = 0;
  if ((rc = device_smem_optin(&optin))) return rc;
  if ((rc = device_sm_count(&sms))) return rc;
  int BM = a.tokens;
  if (BM == 0) {
    BM = sets_fwd_pick_tokens(s.S, a.D, optin);
    if (BM < 0) return BM;
  } else if (BM != 32 && BM != 64 && BM != 128) {
    return GL_ERR_UNSUPPORTED;
  }
  if (sets_fwd_smem(s.S, a.D, BM) + kTcStaticSmem + 2048 > optin) return GL_ERR_SMEM;
  cudaStream_t st = (cudaStream_t)stream;
  const int64_t G = a.g1 - a.g0, n = a.B * G;
  const unsigned zb = (unsigned)((n + 255) / 256 < (int64_t)sms * 8 ? (n + 255) / 256 : (int64_t)sms * 8);
  tc_zero_pre_kernel<<<zb, 256, 0, st>>>(a.pre, a.counts, a.B, a.g0, G, a.ldp, (int)(a.NB * a.C),
                                          a.pool == GL_POOL_MEAN);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e);
  count_launches(1);
  if (s.nchunks == 0) return GL_OK;
  const SetParams sp{s.feat, s.buckets, s.chunks, nullptr, nullptr, (int)s.S};
  switch (BM) {
    case 128: return sets_fwd_nt<128>(p, sp, s.nchunks, a.act, st);
    case 64: return sets_fwd_nt<64>(p, sp, s.nchunks, a.act, st);
    default: return sets_fwd_nt<32>(p, sp, s.nchunks, a.act, st);
  }
}
