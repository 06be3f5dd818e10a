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

int tc_prepare(const GlSharedArgs& a, bool bwd, TcParams& p);

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
