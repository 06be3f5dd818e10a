// Cover-TopK16 forward on the 5th-generation tensor cores (tcgen05, TMEM accumulators), bf16 parameters
// and fp32 ones through three-term bf16 splits.  Same model and arguments as gl_k16_fwd_tc /
// gl_k16_fwd_tc_f32 (k16_tc.cu), i.e. the reference's kgen K = 16 forward
// (sparse_pooling/experimental/kgen/kgen.cuh:142-200, launched by experimental/kgen_layer.py:61-143):
//   pre[t, g] += sum over the valid neurons n of g's records f of act(z[t, f, n]) / n_g,
//   z[t, f, n] = b[f, n] + sum_k w[f, n, k] x[t, feat[q][env[f, k]]].
//
// Formulation.  A CTA owns one input set q (S = 64 features) and 128 tokens.  The set's x rows are staged
// once as the MMA's A operand X [128 tokens x 64 positions] (bf16, 128-byte swizzled, K-major).  The
// set's records are taken 8 at a time: their weights are written, expanded over the set's 64 positions
// (zeros where a record has no input), as the B operand W [8 records x 16 neurons = 128 x 64 positions]
// (K-major), and one 128 x 128 x 64 product X W^T lands in a TMEM accumulator (128 lanes = tokens, 128
// fp32 columns = the batch's neurons).  Each record's inputs are 16 distinct positions of its set (the
// reference's lowering requires sorted distinct positions, kgen_lowered.py:175-176), so the expanded
// weights hold each weight once and every product of the MMA is a product of the model (or zero): the
// MMA does 4x the useful multiply-adds at tcgen05's rate, in exchange for no gathers.  Eight warps then
// read the accumulator (warp w: TMEM lanes 32 (w % 4) .., columns 64 (w / 4) ..), add the bias, apply the
// activation, sum each record's valid neurons per token and keep one partial per token and output,
// added to pre with one atomic when the output changes (records come in the set's bucket order).
//
// fp32 parameters: x and w are each split into three bf16 terms (v = v1 + v2 + v3, as k16_tc.cu), and
// the accumulator receives the six products of term pairs i + j <= 2 (smallest first) per 16-wide K
// step, which agrees with the fp32 SIMT kernels to fp32 rounding.
//
// Pipeline: each thread loads its share of the next batch's weights, positions and bias into registers
// while the current batch's MMAs run and its epilogue reads the accumulator; the expanded weight planes
// are cleared position by position after use (no bulk clearing), and the set's bucket table sits in
// shared memory, so a batch costs two barriers.  One mbarrier, armed by tcgen05.commit after each batch's
// MMAs; all threads wait on it with an iteration limit (on expiry the CTA records a timeout in *status,
// stops issuing work and still frees its TMEM).  Several CTAs share an SM (TMEM 128 columns each, at most
// 4 resident by their shared memory), so one CTA's MMAs overlap another's expansion and epilogue.
#include <cuda_bf16.h>

#include "common.cuh"
#include "tc5.cuh"

namespace gl {

constexpr int kT5Threads = 256;
constexpr int kT5Tokens = 128;
constexpr int kT5Set = 64;              // positions per set (the MMA's K)
constexpr uint32_t kT5Plane = 16384;    // one 128 x 64 bf16 operand plane
constexpr uint32_t kT5WaitLimit = 1u << 20;

struct K16T5Params {
  const float* x;
  const uint8_t* env;
  const int16_t* feat;
  const int32_t* buckets;
  const int32_t* q_off;
  const int32_t* rec_off;
  const void* w;
  const void* b;
  const int32_t* counts;
  float* pre;
  int32_t* status;
  int B, D, G, NB16, nbk;
  int64_t ldx, ldp;
  const float* c1t;   // backward: [G, ldc] coefficients
  float* dx;          // backward: [B, lddx], accumulated
  float* dw;          // backward: fp32, weight-shaped, accumulated
  float* db;          // backward: fp32, bias-shaped, accumulated
  int64_t ldc, lddx;
};

// The three bf16 terms of v (NS = 3), or its bf16 rounding (NS = 1), as raw bits.
template <int NS>
__device__ __forceinline__ void t5_terms(float v, uint16_t (&t)[NS]) {
  float r = v;
#pragma unroll
  for (int j = 0; j < NS; ++j) {
    const __nv_bfloat16 h = __float2bfloat16_rn(r);
    t[j] = __bfloat16_as_ushort(h);
    r -= __bfloat162float(h);
  }
}

constexpr int kT5MaxBuckets = 512;     // buckets of one set cached in shared memory (else global lookups)

// Output g, storage index f and valid neurons nv of flat record r of set (qa .. qb): g = -1 when r is past
// the set's records or its bucket row is malformed.  Bucket rows come from the shared-memory copy when the
// set has at most kT5MaxBuckets of them.
struct T5Rec {
  int g, nv;
  long long f;
};

__device__ __forceinline__ T5Rec t5_record(const K16T5Params& p, int qa, int qb, int rb, int r, bool cached,
                                           const int* bk_rec, const int4* bk_row) {
  T5Rec o{-1, 0, 0};
  if (r >= rb || qb <= qa) return o;
  int lo = qa, hi = qb - 1;  // the bucket b with rec_off[b] <= r < rec_off[b + 1]
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    const int v = cached ? bk_rec[mid - qa] : __ldg(p.rec_off + mid);
    if (v <= r) lo = mid;
    else hi = mid - 1;
  }
  const int4 bk = cached ? bk_row[lo - qa] : __ldg(reinterpret_cast<const int4*>(p.buckets) + lo);
  const int j16 = bk.z + (r - (cached ? bk_rec[lo - qa] : __ldg(p.rec_off + lo)));
  if (bk.y >= 0 && bk.y < p.G && j16 >= 0 && j16 < p.NB16) {
    o.g = bk.y;
    o.f = (long long)bk.y * p.NB16 + j16;
    o.nv = min(max(__ldg(p.counts + bk.y) - 16 * j16, 0), 16);
  }
  return o;
}

// One thread's share of a batch's operands, loaded one batch ahead: the 8 weights of (record warp,
// neuron lane / 2, inputs 8 (lane % 2) ..), their 8 positions, and (threads < 128) one bias value.
struct T5Ops {
  uint2 env;
  float w[8];
  float bias;
};

template <int NS>
__device__ __forceinline__ T5Ops t5_load_ops(const K16T5Params& p, const int* rg, const long long* rf, int tid) {
  T5Ops o;
  const int r = tid >> 5, n = (tid & 31) >> 1, kh = tid & 1;
  o.env = make_uint2(0, 0);
#pragma unroll
  for (int e = 0; e < 8; ++e) o.w[e] = 0.f;
  if (rg[r] >= 0) {
    const long long f = rf[r];
    o.env = __ldg(reinterpret_cast<const uint2*>(p.env + f * 16 + 8 * kh));
    if constexpr (NS == 1) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.w) + f * 256 + n * 16 + 8 * kh));
      const uint32_t uu[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        o.w[2 * e] = bf16_lo(uu[e]);
        o.w[2 * e + 1] = bf16_hi(uu[e]);
      }
    } else {
      const float4* w4 = reinterpret_cast<const float4*>(static_cast<const float*>(p.w) + f * 256 + n * 16 + 8 * kh);
      const float4 a = __ldg(w4), c = __ldg(w4 + 1);
      o.w[0] = a.x; o.w[1] = a.y; o.w[2] = a.z; o.w[3] = a.w;
      o.w[4] = c.x; o.w[5] = c.y; o.w[6] = c.z; o.w[7] = c.w;
    }
  }
  o.bias = 0.f;
  if (tid < 128) {
    const int rr = tid >> 4, nn = tid & 15;
    if (rg[rr] >= 0) {
      const long long bi = rf[rr] * 16 + nn;
      o.bias = NS == 1 ? __uint_as_float((uint32_t)__ldg(static_cast<const uint16_t*>(p.b) + bi) << 16)
                       : __ldg(static_cast<const float*>(p.b) + bi);
    }
  }
  return o;
}

// Position (bytes into a plane) of input e of this thread's share of a row, from the packed positions.
__device__ __forceinline__ uint32_t t5_wpos(const uint2& env, int e, int row) {
  const uint32_t word = e < 4 ? env.x : env.y;
  return t5_sw128_off((uint32_t)row, min((word >> (8 * (e & 3))) & 0xffu, (uint32_t)(kT5Set - 1)));
}

template <int NS, int ACT>
__global__ void __launch_bounds__(kT5Threads) k16t5_fwd_kernel(const K16T5Params p) {
  extern __shared__ unsigned char t5_raw[];
  __shared__ __align__(8) uint64_t mbar[2];
  __shared__ uint32_t tmem_s;
  __shared__ int abort_s;
  __shared__ int fq[kT5Set];
  __shared__ __align__(16) float bias_s[2][8][16];
  __shared__ int rg_s[3][8], rnv_s[3][8];
  __shared__ long long rf_s[3][8];
  __shared__ int bk_rec[kT5MaxBuckets + 1];
  __shared__ int4 bk_row[kT5MaxBuckets];
  unsigned char* smem = reinterpret_cast<unsigned char*>(((uintptr_t)t5_raw + 1023) & ~(uintptr_t)1023);
  unsigned char* xpl = smem;                    // NS planes: X [128 tokens][64 positions]
  unsigned char* wpl = smem + NS * kT5Plane;    // 2 buffers x NS planes: W [128 batch neurons][64 positions]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int q = blockIdx.y, t0 = blockIdx.x * kT5Tokens;
  if (warp == 0) t5_tmem_alloc(t5_smem_u32(&tmem_s), 256);
  if (tid == 0) {
    t5_mbar_init(t5_smem_u32(&mbar[0]), 1);
    t5_mbar_init(t5_smem_u32(&mbar[1]), 1);
    abort_s = 0;
  }
  if (tid < kT5Set) {
    const int d = (int)(uint16_t)__ldg(p.feat + (int64_t)q * kT5Set + tid);
    fq[tid] = d < p.D ? d : p.D - 1;
  }
  const int qa = min(max(__ldg(p.q_off + q), 0), p.nbk), qb = min(max(__ldg(p.q_off + q + 1), qa), p.nbk);
  const int ra = __ldg(p.rec_off + qa), rb = __ldg(p.rec_off + qb);
  const bool cached = qb - qa <= kT5MaxBuckets;
  if (cached) {
    for (int i = tid; i <= qb - qa; i += kT5Threads) bk_rec[i] = __ldg(p.rec_off + qa + i);
    for (int i = tid; i < qb - qa; i += kT5Threads) bk_row[i] = __ldg(reinterpret_cast<const int4*>(p.buckets) + qa + i);
  }
  for (int i = tid; i < 2 * NS * (int)kT5Plane / 16; i += kT5Threads)
    reinterpret_cast<uint4*>(wpl)[i] = make_uint4(0, 0, 0, 0);
  __syncthreads();
  // stage X: 128 rows x 8 chunks of 8 positions per plane
  for (int c = tid; c < kT5Tokens * 8; c += kT5Threads) {
    const int row = c >> 3, ch = c & 7, t = t0 + row;
    uint16_t terms[8][NS];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float v = t < p.B ? __ldg(p.x + (int64_t)t * p.ldx + fq[8 * ch + e]) : 0.f;
      t5_terms<NS>(v, terms[e]);
    }
#pragma unroll
    for (int j = 0; j < NS; ++j) {
      uint4 u;
      u.x = (uint32_t)terms[0][j] | ((uint32_t)terms[1][j] << 16);
      u.y = (uint32_t)terms[2][j] | ((uint32_t)terms[3][j] << 16);
      u.z = (uint32_t)terms[4][j] | ((uint32_t)terms[5][j] << 16);
      u.w = (uint32_t)terms[6][j] | ((uint32_t)terms[7][j] << 16);
      *reinterpret_cast<uint4*>(xpl + j * kT5Plane + t5_sw128_off(row, 8 * ch)) = u;
    }
  }
  const int nbatch = rb > ra ? (rb - ra + 7) / 8 : 0;
  if (tid < 8) {  // batch 0's records
    const T5Rec rc = t5_record(p, qa, qb, rb, ra + tid, cached, bk_rec, bk_row);
    rg_s[0][tid] = rc.g;
    rf_s[0][tid] = rc.f;
    rnv_s[0][tid] = rc.nv;
  }
  t5_fence_smem_to_async();
  t5_fence_before_sync();
  __syncthreads();
  t5_fence_after_sync();
  const uint32_t tmem = tmem_s;
  const uint32_t idesc = t5_idesc_bf16(128, 128, 0, 0);
  const uint32_t xs_u = t5_smem_u32(xpl), ws_u = t5_smem_u32(wpl);
  // epilogue geometry: this thread's token row and its warp's 64 columns (4 records)
  const int erow = 32 * (warp & 3) + lane, et = t0 + erow, ecol = 64 * (warp >> 2);
  const int wrow = 16 * warp + ((tid & 31) >> 1);  // the W row this thread expands
  float acc = 0.f;
  int gcur = -1;
  auto flush = [&]() {
    if (gcur >= 0 && et < p.B)
      atomicAdd(p.pre + (int64_t)et * p.ldp + gcur, acc / (float)max(__ldg(p.counts + gcur), 1));
  };
  T5Ops ops = t5_load_ops<NS>(p, rg_s[0], rf_s[0], tid);
  uint2 env_prev = make_uint2(0, 0);
  // iteration b: expand and multiply batch b (buffer b & 1) while the epilogue reads batch b - 1
  for (int b = 0; b <= nbatch; ++b) {
    const uint2 env_cur = ops.env;
    if (b < nbatch) {
      unsigned char* wb = wpl + (b & 1) * NS * kT5Plane;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        uint16_t terms[NS];
        t5_terms<NS>(ops.w[e], terms);
        const uint32_t off = t5_wpos(env_cur, e, wrow);
#pragma unroll
        for (int j = 0; j < NS; ++j) *reinterpret_cast<uint16_t*>(wb + j * kT5Plane + off) = terms[j];
      }
      if (tid < 128) bias_s[b & 1][tid >> 4][tid & 15] = ops.bias;
      if (tid < 8) {  // the next batch's records
        const T5Rec rc = t5_record(p, qa, qb, rb, ra + 8 * (b + 1) + tid, cached, bk_rec, bk_row);
        rg_s[(b + 1) % 3][tid] = rc.g;
        rf_s[(b + 1) % 3][tid] = rc.f;
        rnv_s[(b + 1) % 3][tid] = rc.nv;
      }
    }
    t5_fence_smem_to_async();
    __syncthreads();
    if (b < nbatch && tid == 0 && !abort_s) {
      t5_fence_after_sync();
      const uint32_t wb_u = ws_u + (b & 1) * NS * kT5Plane, d_t = tmem + (uint32_t)((b & 1) * 128);
      uint32_t first = 1;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
#pragma unroll
        for (int sum = NS - 1; sum >= 0; --sum)
#pragma unroll
          for (int i = 0; i <= sum; ++i) {
            const uint64_t ad = t5_desc_sw128(xs_u + i * kT5Plane + 32 * kk, 16, 1024);
            const uint64_t bd = t5_desc_sw128(wb_u + (sum - i) * kT5Plane + 32 * kk, 16, 1024);
            t5_mma_bf16(d_t, ad, bd, idesc, first ? 0u : 1u);
            first = 0;
          }
      t5_commit(t5_smem_u32(&mbar[b & 1]));
    }
    if (b + 1 < nbatch) ops = t5_load_ops<NS>(p, rg_s[(b + 1) % 3], rf_s[(b + 1) % 3], tid);  // under the MMAs
    if (b >= 1) {  // epilogue of batch b - 1
      const int pb = b - 1, sl = pb & 1, is = pb % 3;
      const bool ok = abort_s == 0 &&
                      t5_mbar_wait(t5_smem_u32(&mbar[sl]), (uint32_t)((pb >> 1) & 1), kT5WaitLimit);
      if (!ok) {
        if (p.status) atomicExch(p.status, 1);
        abort_s = 1;
      }
      t5_fence_after_sync();
      if (__all_sync(kFullMask, ok)) {  // warp-uniform: the TMEM loads below are .sync.aligned
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          float v[32];
          t5_ld32(tmem + ((uint32_t)(32 * (warp & 3)) << 16) + (uint32_t)(sl * 128 + ecol + 32 * c), v);
#pragma unroll
          for (int rr = 0; rr < 2; ++rr) {
            const int r = (ecol >> 4) + 2 * c + rr;
            const int g = rg_s[is][r], nv = rnv_s[is][r];
            if (g < 0) continue;
            const float4* bq = reinterpret_cast<const float4*>(bias_s[sl][r]);
            float sm = 0.f;
#pragma unroll
            for (int n4 = 0; n4 < 4; ++n4) {
              const float4 bb = bq[n4];
              const float a0 = act_f<ACT>(v[16 * rr + 4 * n4] + bb.x), a1 = act_f<ACT>(v[16 * rr + 4 * n4 + 1] + bb.y);
              const float a2 = act_f<ACT>(v[16 * rr + 4 * n4 + 2] + bb.z), a3 = act_f<ACT>(v[16 * rr + 4 * n4 + 3] + bb.w);
              if (nv == 16) {
                sm += (a0 + a1) + (a2 + a3);
              } else {
                sm += (4 * n4 < nv ? a0 : 0.f) + (4 * n4 + 1 < nv ? a1 : 0.f) + (4 * n4 + 2 < nv ? a2 : 0.f) +
                      (4 * n4 + 3 < nv ? a3 : 0.f);
              }
            }
            if (g != gcur) {
              flush();
              gcur = g;
              acc = 0.f;
            }
            acc += sm;
          }
        }
      }
      // clear the positions batch b - 1 wrote (its MMAs have completed)
      unsigned char* wb = wpl + sl * NS * kT5Plane;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const uint32_t off = t5_wpos(env_prev, e, wrow);
#pragma unroll
        for (int j = 0; j < NS; ++j) *reinterpret_cast<uint16_t*>(wb + j * kT5Plane + off) = 0;
      }
    }
    env_prev = env_cur;
    t5_fence_before_sync();
    __syncthreads();
    if (abort_s) break;
  }
  flush();
  t5_fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    t5_fence_after_sync();
    t5_tmem_dealloc(tmem, 256);
  }
}

// Shared memory of the forward: the X planes and two buffers of W planes (1 KiB alignment slack), at least
// 80 KiB so that at most two CTAs (2 x 256 TMEM columns) are resident on an SM.
template <int NS>
static size_t t5_fwd_smem() {
  const size_t need = 3u * NS * kT5Plane + 1024;
  return need < 81920 ? 81920 : need;
}

template <int NS, int ACT>
static int t5_fwd_launch(const K16T5Params& p, int64_t Q, cudaStream_t st) {
  const size_t smem = t5_fwd_smem<NS>();
  auto kern = k16t5_fwd_kernel<NS, ACT>;
  int rc = ensure_dynamic_smem((const void*)kern, smem);
  if (rc) return rc;
  const dim3 grid((unsigned)((p.B + kT5Tokens - 1) / kT5Tokens), (unsigned)Q);
  kern<<<grid, kT5Threads, smem, st>>>(p);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e);
  count_launches(1);
  return GL_OK;
}

template <int NS>
static int t5_fwd_run(const GlK16Args* args, int32_t* status, void* stream) {
  if (!args) return GL_ERR_NULL;
  const GlK16Args& a = *args;
  if (a.B < 0 || a.D < 1 || a.D > 32767 || a.G < 1 || a.NB16 < 1 || a.Q < 1 || a.nbuckets < 0) return GL_ERR_SHAPE;
  if (a.S != kT5Set) return GL_ERR_UNSUPPORTED;
  if (a.act != GL_ACT_RELU && a.act != GL_ACT_IDENTITY) return GL_ERR_UNSUPPORTED;
  if (a.tokens != 0 && a.tokens != kT5Tokens) return GL_ERR_UNSUPPORTED;
  if (a.B == 0 || a.nbuckets == 0) return GL_OK;
  if (!a.x || !a.env || !a.feat || !a.buckets || !a.q_off || !a.rec_off || !a.w || !a.b || !a.counts || !a.pre)
    return GL_ERR_NULL;
  if (a.B > 2147483647LL || a.ldx < a.D || a.Q > 65535 || a.G * a.NB16 > 2147483647LL || a.ldp < a.G)
    return GL_ERR_SHAPE;
  if (((uintptr_t)a.env & 15) || ((uintptr_t)a.buckets & 15) || ((uintptr_t)a.w & 15) || ((uintptr_t)a.b & 15))
    return GL_ERR_ALIGN;
  int optin = 0;
  int rc = device_smem_optin(&optin);
  if (rc) return rc;
  if ((int64_t)t5_fwd_smem<NS>() > optin) return GL_ERR_SMEM;
  const K16T5Params p{a.x, a.env, a.feat, a.buckets, a.q_off, a.rec_off, a.w, a.b, a.counts, a.pre, status,
                      (int)a.B, (int)a.D, (int)a.G, (int)a.NB16, (int)a.nbuckets, a.ldx, a.ldp,
                      nullptr, nullptr, nullptr, nullptr, 0, 0};
  cudaStream_t st = (cudaStream_t)stream;
  return a.act == GL_ACT_RELU ? t5_fwd_launch<NS, GL_ACT_RELU>(p, a.Q, st) : t5_fwd_launch<NS, GL_ACT_IDENTITY>(p, a.Q, st);
}

// ---------------------------------------------------------------------------------------------------
// Backward on tcgen05 (gl_k16_bwd_t5 / gl_k16_bwd_t5_f32): the reference's kgen K = 16 backward
// (experimental/kgen/kgen.cuh:202-342 dX, :356-536 dW) for one input set and 128 tokens per CTA, per batch of
// 8 records (128 neurons), all products on the tensor cores over shared-memory operands:
//   Z   [128 tokens x 128 neurons]  = X W^T             (A = X, B = W; K = the set's 64 positions)
//   dz  = c1t[g, t] act'(Z + b), masked to the valid neurons, written back as bf16 terms
//   dXs [128 tokens x 64 positions] += dz W             (A = dz, B = W read MN-major; K = 128 neurons)
//   dWs [128 neurons x 64 positions] = dz^T X           (A = dz read MN-major, B = X read MN-major; K = tokens)
//   db  [128 neurons]                = dz^T 1           (a 65th column of X's MN-major view, all ones)
// W is the batch's weights expanded over the set's positions (as the forward), so dWs holds each record's
// 16 weight gradients at its positions and zeros elsewhere; the dW epilogue reads those 16 columns and adds
// them to dw.  dXs stays in TMEM for all of the set's records (a fixed summation order within the set) and
// is added to dx once per CTA: no shared-memory atomics and no fixed-point bounds.  The same shared-memory
// tile serves as a K-major operand of one product and an MN-major operand of another (rows of 64 bf16 in
// 128-byte-swizzled 8-row atoms: for K-major operands the rows are M or N, for MN-major ones K).  bf16
// parameters (NS = 1): x and w one bf16 term, dz two (hi + lo, the reference's split precision); fp32
// parameters (NS = 3): three terms each, term pairs i + j <= 2 per product, as the forward.
//
// Warp roles (448 threads), handing work over through mbarriers (every wait has an iteration limit; on
// expiry the CTA records a timeout in *status, every role leaves its loop, and the TMEM is still freed):
//   warps 0-7   dz epilogue: warp w reads TMEM lanes 32 (w % 4) .. (tokens) and computes dz for the 64
//               neurons of records 4 (w / 4) ..; at the end they add dXs to dx;
//   warps 8-11  producer and dW epilogue: warp 8 + q owns records 2q, 2q + 1 of every batch (lane = record
//               half x neuron): it finds the records and loads their operands a batch ahead, expands the
//               weights into W, and after the batch's products reads the 16 dWs columns of each record
//               (one tcgen05.ld per column, one wait) and db;
//   warp 12     allocates TMEM, and its lane 0 issues the Z and dX MMAs;
//   warp 13     its lane 0 issues the dW | db MMAs (narrow products whose issue, not the tensor pipe, bounds a
//               single issuing thread), committing to the same barrier as warp 12.
// bf16 parameters keep three W buffers and two dz buffers, so the next batch's Z product runs ahead of the
// current batch's products while its dz epilogue runs; fp32 ones (three-term planes) fit one buffer of each,
// and then only Z and dWs (in TMEM) are double-buffered.  With bf16 parameters the epilogue also writes the
// two dz terms back over the batch's Z columns in TMEM (a 32-neuron chunk's hi and lo halves in its own 32
// columns), and the dX product reads its A operand from there: the tensor cores then read dz from shared
// memory once per batch (for dW), which bounds these narrow products (N = 64 / 80) more than their math.
// TMEM columns: Z [0, 256) (two buffers), dXs [256, 320), dWs [320, 480) (two buffers of 64 dW columns and
// the db column).
constexpr uint32_t kT5DzPlane = 32768;    // dz [128 tokens][128 neurons]: two 64-neuron halves of 16 KiB
constexpr uint32_t kT5DzHalf = 16384;
constexpr int kB5EpiWarps = 8;                       // dz epilogue: warps 0-7
constexpr int kB5Issuer = kB5EpiWarps + 4;            // producer: warps 8-11; MMA issuers: warps 12 and 13
constexpr int kB5Threads = 32 * (kB5Issuer + 2);
constexpr int kB5EpiArrivals = 32 * kB5EpiWarps, kB5ProdArrivals = 128;   // one arrival per thread
constexpr int kB5Meta = 4;                            // batches whose record data is kept (ring)
constexpr uint32_t kB5TZ = 0, kB5TdX = 256, kB5TdW = 320, kB5DWCols = 80;

template <int NS>
__host__ __device__ constexpr int t5_dz_terms() { return NS == 1 ? 2 : 3; }
// Buffers of W and of dz: three and two for bf16 parameters; one each for the fp32 ones' three-term planes.
template <int NS>
__host__ __device__ constexpr int t5_wbufs() { return NS == 1 ? 3 : 1; }
template <int NS>
__host__ __device__ constexpr int t5_zbufs() { return NS == 1 ? 2 : 1; }

// X planes, the ones block beside X term 0 (its second 64-column block in the MN-major view), W and dz buffers.
template <int NS>
static size_t t5_bwd_smem() {
  return (size_t)kT5Plane * (NS + 1 + NS * t5_wbufs<NS>()) + (size_t)t5_zbufs<NS>() * t5_dz_terms<NS>() * kT5DzPlane +
         1024;
}

// MMAs of a product over term planes a_i (NA terms) and b_j (NB terms), pairs i + j <= max(NA, NB) - 1, the
// smallest first, at K step kk.  `first` clears the accumulator on the first MMA.
template <int NA, int NBT, typename FA, typename FB>
__device__ __forceinline__ void t5_mma_terms(uint32_t d_t, uint32_t idesc, FA adesc, FB bdesc, int kk, uint32_t& first) {
  constexpr int top = (NA > NBT ? NA : NBT) - 1;
#pragma unroll
  for (int sum = top; sum >= 0; --sum)
#pragma unroll
    for (int i = 0; i <= sum; ++i) {
      const int j = sum - i;
      if (i < NA && j < NBT) {
        t5_mma_bf16(d_t, adesc(i, kk), bdesc(j, kk), idesc, first ? 0u : 1u);
        first = 0;
      }
    }
}

// The bf16 terms of (a, b) as packed pairs (a in the low half): ND steps of round-to-nearest and subtract.
template <int ND>
__device__ __forceinline__ void t5_pair_terms(float a, float b, uint32_t (&u)[ND]) {
#pragma unroll
  for (int i = 0; i < ND; ++i) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    u[i] = *reinterpret_cast<const uint32_t*>(&h);
    a -= __uint_as_float(u[i] << 16);
    b -= __uint_as_float(u[i] & 0xffff0000u);
  }
}

constexpr int kB5Buckets = 256;   // buckets of one set cached in shared memory (else read from global)

struct B5Shared {   // 16-byte members first: bias and env are read as 16-byte vectors
  __align__(16) float bias[kB5Meta][8][16];
  uint4 env[kB5Meta][8];
  int4 bk_row[kB5Buckets];
  long long rf[kB5Meta][8];
  uint64_t w_full[3], z_full[2], z_empty[2], dz_full[2], mma2[2], dw_empty[2], fin[2];
  int bk_rec[kB5Buckets + 1];
  int rg[kB5Meta][8], rnv[kB5Meta][8];
  int fq[kT5Set];
  uint32_t tmem;
  int abort;
};
static_assert(offsetof(B5Shared, bias) % 16 == 0 && offsetof(B5Shared, env) % 16 == 0 &&
              offsetof(B5Shared, bk_row) % 16 == 0 && offsetof(B5Shared, w_full) % 8 == 0, "B5Shared alignment");

// Bounded wait of a whole warp on phase `parity` of an mbarrier; false (for every lane) once any lane gave
// up or the CTA is aborting.  Records a timeout in *status and the CTA's abort flag.
__device__ __forceinline__ bool b5_wait(B5Shared& sh, uint64_t& bar, uint32_t parity, int32_t* status) {
  volatile int* ab = &sh.abort;
  bool got = *ab == 0 && t5_mbar_wait(t5_smem_u32(&bar), parity, kT5WaitLimit);
  got = __all_sync(kFullMask, got);
  if (!got) {
    if ((threadIdx.x & 31) == 0) {
      if (*ab == 0 && status) atomicExch(status, 1);
      *ab = 1;
    }
    return false;
  }
  t5_fence_after_sync();
  return true;
}

// Every lane arrives (after its own preceding shared-memory writes or TMEM loads, fenced by the caller).
__device__ __forceinline__ void b5_arrive(uint64_t& bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(t5_smem_u32(&bar)) : "memory");
}

// Record data of flat record r of the CTA's set (buckets qa .. qb), found from bucket cursor *bc (advanced
// monotonically); bucket rows from the shared-memory copy when `cached`.  nv is left to the caller.
__device__ __forceinline__ T5Rec b5_record(const K16T5Params& p, const B5Shared& sh, bool cached, int qa, int qb,
                                           int rb, int r, int* bc) {
  T5Rec o{-1, 0, 0};
  if (r >= rb) return o;
  int b = *bc;
  if (cached) {
    while (b + 1 < qb && sh.bk_rec[b + 1 - qa] <= r) ++b;
  } else {
    while (b + 1 < qb && __ldg(p.rec_off + b + 1) <= r) ++b;
  }
  *bc = b;
  const int4 bk = cached ? sh.bk_row[b - qa] : __ldg(reinterpret_cast<const int4*>(p.buckets) + b);
  const int j16 = bk.z + (r - (cached ? sh.bk_rec[b - qa] : __ldg(p.rec_off + b)));
  if (bk.y >= 0 && bk.y < p.G && j16 >= 0 && j16 < p.NB16) {
    o.g = bk.y;
    o.f = (long long)bk.y * p.NB16 + j16;
  }
  return o;
}

// One producer lane's operands of a batch, loaded a batch ahead of their use.
struct B5Load {
  int g, nv;
  long long f;
  uint4 env;
  float w[16];
  float bias;
};

template <int NS, int ACT>
__global__ void __launch_bounds__(kB5Threads, 1) k16t5_bwd_kernel(const K16T5Params p) {
  constexpr int ND = t5_dz_terms<NS>(), NWB = t5_wbufs<NS>(), NZB = t5_zbufs<NS>();
  extern __shared__ unsigned char t5_raw[];
  __shared__ __align__(16) B5Shared sh;
  unsigned char* smem = reinterpret_cast<unsigned char*>(((uintptr_t)t5_raw + 1023) & ~(uintptr_t)1023);
  unsigned char* xpl = smem;                          // NS planes X [128 tokens][64 positions]
  unsigned char* opl = xpl + NS * kT5Plane;           // [128 tokens][64]: column 0 ones (X term 0's 65th column)
  unsigned char* wpl = opl + kT5Plane;                // NWB buffers x NS planes W [128 neurons][64 positions]
  unsigned char* dpl = wpl + NWB * NS * kT5Plane;     // NZB buffers x ND planes dz [128 tokens][2 x 64 neurons]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int q = blockIdx.y, t0 = blockIdx.x * kT5Tokens;
  volatile int* abort_v = &sh.abort;
  if (warp == kB5Issuer) t5_tmem_alloc(t5_smem_u32(&sh.tmem), 512);
  if (tid == 0) {
    for (int i = 0; i < 3; ++i) t5_mbar_init(t5_smem_u32(&sh.w_full[i]), kB5ProdArrivals);
    for (int i = 0; i < 2; ++i) {
      t5_mbar_init(t5_smem_u32(&sh.z_full[i]), 1);
      t5_mbar_init(t5_smem_u32(&sh.z_empty[i]), kB5EpiArrivals);
      t5_mbar_init(t5_smem_u32(&sh.dz_full[i]), kB5EpiArrivals);
      t5_mbar_init(t5_smem_u32(&sh.mma2[i]), 2);   // the dX and the dW issuer commit
      t5_mbar_init(t5_smem_u32(&sh.dw_empty[i]), kB5ProdArrivals);
    }
    t5_mbar_init(t5_smem_u32(&sh.fin[0]), 1);
    t5_mbar_init(t5_smem_u32(&sh.fin[1]), 1);
    sh.abort = 0;
  }
  if (tid < kT5Set) {
    const int d = (int)(uint16_t)__ldg(p.feat + (int64_t)q * kT5Set + tid);
    sh.fq[tid] = d < p.D ? d : p.D - 1;
  }
  const int qa = min(max(__ldg(p.q_off + q), 0), p.nbk), qb = min(max(__ldg(p.q_off + q + 1), qa), p.nbk);
  const int ra = __ldg(p.rec_off + qa), rb = __ldg(p.rec_off + qb);
  const int nbatch = rb > ra ? (rb - ra + 7) / 8 : 0;
  const bool cached = qb - qa <= kB5Buckets;
  if (cached) {
    for (int i = tid; i <= qb - qa; i += kB5Threads) sh.bk_rec[i] = __ldg(p.rec_off + qa + i);
    for (int i = tid; i < qb - qa; i += kB5Threads) sh.bk_row[i] = __ldg(reinterpret_cast<const int4*>(p.buckets) + qa + i);
  }
  for (int i = tid; i < NWB * NS * (int)kT5Plane / 16; i += kB5Threads) reinterpret_cast<uint4*>(wpl)[i] = make_uint4(0, 0, 0, 0);
  for (int i = tid; i < (int)kT5Plane / 16; i += kB5Threads) {   // element (token, 0) = bf16 one
    const int row = i >> 3, ch = i & 7;
    reinterpret_cast<uint4*>(opl)[i] = ch == (row & 7) ? make_uint4(0x3F80u, 0, 0, 0) : make_uint4(0, 0, 0, 0);
  }
  __syncthreads();
  for (int c = tid; c < kT5Tokens * 8; c += kB5Threads) {   // stage X, as the forward
    const int row = c >> 3, ch = c & 7, t = t0 + row;
    uint16_t terms[8][NS];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float v = t < p.B ? __ldg(p.x + (int64_t)t * p.ldx + sh.fq[8 * ch + e]) : 0.f;
      t5_terms<NS>(v, terms[e]);
    }
#pragma unroll
    for (int j = 0; j < NS; ++j) {
      uint4 u;
      u.x = (uint32_t)terms[0][j] | ((uint32_t)terms[1][j] << 16);
      u.y = (uint32_t)terms[2][j] | ((uint32_t)terms[3][j] << 16);
      u.z = (uint32_t)terms[4][j] | ((uint32_t)terms[5][j] << 16);
      u.w = (uint32_t)terms[6][j] | ((uint32_t)terms[7][j] << 16);
      *reinterpret_cast<uint4*>(xpl + j * kT5Plane + t5_sw128_off(row, 8 * ch)) = u;
    }
  }
  t5_fence_smem_to_async();
  t5_fence_before_sync();
  __syncthreads();
  t5_fence_after_sync();
  const uint32_t tmem = sh.tmem;
  const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;   // this warp's TMEM lanes

  if (warp < kB5EpiWarps) {
    // ---- dz epilogue: token row erow, the 64 neurons of records 4 eh .. 4 eh + 3
    const int erow = 32 * (warp & 3) + lane, et = t0 + erow, eh = warp >> 2;
    float c1n[4];   // the next batch's coefficients of this token and the half's records
    auto load_c1 = [&](int c) -> bool {
      if (!b5_wait(sh, sh.w_full[c % NWB], (uint32_t)((c / NWB) & 1), p.status)) return false;   // record data of c
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int g = sh.rg[c % kB5Meta][4 * eh + r];
        c1n[r] = (g >= 0 && et < p.B) ? __ldg(p.c1t + (int64_t)g * p.ldc + et) : 0.f;
      }
      return true;
    };
    bool live = nbatch > 0 && load_c1(0);
    for (int c = 0; c < nbatch && live; ++c) {
      const int sl = c % kB5Meta, zb = c & 1, dzb = c % NZB;
      if (c >= NZB && !b5_wait(sh, sh.mma2[(c - NZB) & 1], (uint32_t)(((c - NZB) >> 1) & 1), p.status)) break;  // dz free
      if (!b5_wait(sh, sh.z_full[zb], (uint32_t)((c >> 1) & 1), p.status)) break;
      float c1[4];   // first used here, after the waits: the loads had them to complete
#pragma unroll
      for (int r = 0; r < 4; ++r) c1[r] = c1n[r];
      unsigned char* dz = dpl + dzb * ND * kT5DzPlane + eh * kT5DzHalf;
#pragma unroll
      for (int cc = 0; cc < 2; ++cc) {
        float v[32];
        uint32_t tpk[2][16];   // (bf16) the chunk's dz terms as packed pairs, for the TMEM copy
        t5_ld32(tmem + lane_base + kB5TZ + (uint32_t)(128 * zb + 64 * eh + 32 * cc), v);
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
          const int r = 2 * cc + rr, nv = sh.rnv[sl][4 * eh + r];
          const float4* bq = reinterpret_cast<const float4*>(sh.bias[sl][4 * eh + r]);
          float d[16];
#pragma unroll
          for (int n4 = 0; n4 < 4; ++n4) {
            const float4 bb = bq[n4];
            const float bv[4] = {bb.x, bb.y, bb.z, bb.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int n = 4 * n4 + e;
              const float z = v[16 * rr + n] + bv[e];
              d[n] = ACT == GL_ACT_RELU ? (z > 0.f ? c1[r] : 0.f) : c1[r] * dact_f<ACT>(z);
            }
          }
          if (nv < 16) {
#pragma unroll
            for (int n = 0; n < 16; ++n) d[n] = n < nv ? d[n] : 0.f;
          }
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            uint32_t u[4][ND];
#pragma unroll
            for (int e = 0; e < 4; ++e) t5_pair_terms<ND>(d[8 * hh + 2 * e], d[8 * hh + 2 * e + 1], u[e]);
            const uint32_t off = t5_sw128_off(erow, 32 * cc + 16 * rr + 8 * hh);
#pragma unroll
            for (int i = 0; i < ND; ++i) {
              *reinterpret_cast<uint4*>(dz + i * kT5DzPlane + off) = make_uint4(u[0][i], u[1][i], u[2][i], u[3][i]);
              if constexpr (NS == 1)
#pragma unroll
                for (int e = 0; e < 4; ++e) tpk[i][8 * rr + 4 * hh + e] = u[e][i];
            }
          }
        }
        if constexpr (NS == 1) {   // hi and lo halves of this chunk over its own (already read) Z columns
          const uint32_t tc = tmem + lane_base + kB5TZ + (uint32_t)(128 * zb + 64 * eh + 32 * cc);
          t5_st16(tc, tpk[0]);
          t5_st16(tc + 16, tpk[1]);
        }
      }
      if constexpr (NS == 1) t5_wait_st();
      t5_fence_before_sync();
      b5_arrive(sh.z_empty[zb]);
      t5_fence_smem_to_async();
      b5_arrive(sh.dz_full[dzb]);
      if (c + 1 < nbatch && !load_c1(c + 1)) break;
    }
    // dx[t, feat[q][s]] += dXs, once every product has completed
    if (nbatch > 0 && b5_wait(sh, sh.mma2[(nbatch - 1) & 1], (uint32_t)(((nbatch - 1) >> 1) & 1), p.status)) {
      float v[32];
      t5_ld32(tmem + lane_base + kB5TdX + (uint32_t)(32 * eh), v);
      if (et < p.B) {
        float* dxr = p.dx + (int64_t)et * p.lddx;
#pragma unroll
        for (int s = 0; s < 32; ++s)
          if (v[s] != 0.f || v[s] != v[s]) atomicAdd(dxr + sh.fq[32 * eh + s], v[s]);
      }
    }
  } else if (warp < kB5EpiWarps + 4) {
    // ---- producer and dW epilogue: records 2 pq + (lane >> 4), neuron lane & 15 (TMEM lanes 32 pq ..)
    const int pq = warp & 3, rr = lane >> 4, n = lane & 15, r = 2 * pq + rr;
    const int row = 16 * r + n;    // this lane's W row
    int bc = qa;                   // bucket cursor of this lane's record (lanes n == 0 use it)
    uint4 envh[3] = {make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0)};   // per W buffer
    // issue the loads of batch e's operands (consumed by store(), a batch later)
    auto fetch = [&](int e) {
      B5Load o;
      T5Rec rc{-1, 0, 0};
      if (n == 0) rc = b5_record(p, sh, cached, qa, qb, rb, ra + 8 * e + r, &bc);
      o.g = __shfl_sync(kFullMask, rc.g, lane & 16);
      o.f = __shfl_sync(kFullMask, rc.f, lane & 16);
      o.nv = 0;
      o.env = make_uint4(0, 0, 0, 0);
      o.bias = 0.f;
#pragma unroll
      for (int k = 0; k < 16; ++k) o.w[k] = 0.f;
      if (o.g >= 0) {
        const long long f = o.f;
        o.nv = min(max(__ldg(p.counts + o.g) - 16 * (int)(f - (long long)o.g * p.NB16), 0), 16);
        o.env = __ldg(reinterpret_cast<const uint4*>(p.env + f * 16));
        if constexpr (NS == 1) {
          const uint4* wp = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p.w) + f * 256 + n * 16);
          const uint4 a = __ldg(wp), b = __ldg(wp + 1);
          const uint32_t uu[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            o.w[2 * k] = bf16_lo(uu[k]);
            o.w[2 * k + 1] = bf16_hi(uu[k]);
          }
          o.bias = __uint_as_float((uint32_t)__ldg(static_cast<const uint16_t*>(p.b) + f * 16 + n) << 16);
        } else {
          const float4* wp = reinterpret_cast<const float4*>(static_cast<const float*>(p.w) + f * 256 + n * 16);
#pragma unroll
          for (int k4 = 0; k4 < 4; ++k4) {
            const float4 a = __ldg(wp + k4);
            o.w[4 * k4] = a.x; o.w[4 * k4 + 1] = a.y; o.w[4 * k4 + 2] = a.z; o.w[4 * k4 + 3] = a.w;
          }
          o.bias = __ldg(static_cast<const float*>(p.b) + f * 16 + n);
        }
      }
      return o;
    };
    // expand batch e (operands o) into W buffer e % NWB, whose previous products have completed
    auto store = [&](int e, const B5Load& o) {
      const int sl = e % kB5Meta, wb = e % NWB;
      unsigned char* wbuf = wpl + wb * NS * kT5Plane;
      const uint4 eh = wb == 0 ? envh[0] : wb == 1 ? envh[1] : envh[2];
      if (e >= NWB) {   // clear the positions the buffer's previous batch wrote in this row
        const uint32_t ew[4] = {eh.x, eh.y, eh.z, eh.w};
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          const uint32_t off = t5_sw128_off((uint32_t)row, min((ew[k >> 2] >> (8 * (k & 3))) & 0xffu, (uint32_t)(kT5Set - 1)));
#pragma unroll
          for (int j = 0; j < NS; ++j) *reinterpret_cast<uint16_t*>(wbuf + j * kT5Plane + off) = 0;
        }
      }
      const uint32_t ew[4] = {o.env.x, o.env.y, o.env.z, o.env.w};
#pragma unroll
      for (int k = 0; k < 16; ++k) {
        uint16_t terms[NS];
        t5_terms<NS>(o.w[k], terms);
        const uint32_t off = t5_sw128_off((uint32_t)row, min((ew[k >> 2] >> (8 * (k & 3))) & 0xffu, (uint32_t)(kT5Set - 1)));
#pragma unroll
        for (int j = 0; j < NS; ++j) *reinterpret_cast<uint16_t*>(wbuf + j * kT5Plane + off) = terms[j];
      }
      if (wb == 0) envh[0] = o.env;
      else if (wb == 1) envh[1] = o.env;
      else envh[2] = o.env;
      sh.bias[sl][r][n] = o.bias;
      if (n == 0) {
        sh.rg[sl][r] = o.g;
        sh.rf[sl][r] = o.f;
        sh.rnv[sl][r] = o.nv;
        sh.env[sl][r] = o.env;
      }
      t5_fence_smem_to_async();
      b5_arrive(sh.w_full[wb]);
    };
    for (int e = 0; e < NWB && e < nbatch; ++e) store(e, fetch(e));
    B5Load nxt;
    if (NWB < nbatch) nxt = fetch(NWB);
    for (int c = 0; c < nbatch; ++c) {
      const int sl = c % kB5Meta, zb = c & 1;
      if (!b5_wait(sh, sh.mma2[zb], (uint32_t)((c >> 1) & 1), p.status)) break;
      // dW of the lane's neuron at its record's 16 positions (one load per position of each of the warp's
      // two records), and db
      const int g = sh.rg[sl][r], nv = sh.rnv[sl][r];
      const uint32_t tw = tmem + lane_base + kB5TdW + kB5DWCols * (uint32_t)zb;
      float va[16], vb[16];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint4 e4 = sh.env[sl][2 * pq + h];
        const uint32_t ew[4] = {e4.x, e4.y, e4.z, e4.w};
        uint32_t ad[16];
#pragma unroll
        for (int k = 0; k < 16; ++k) ad[k] = tw + min((ew[k >> 2] >> (8 * (k & 3))) & 0xffu, (uint32_t)(kT5Set - 1));
        if (h == 0) t5_ld16_cols(ad, va);
        else t5_ld16_cols(ad, vb);
      }
      const float dbv = t5_ld1(tw + 64);
      t5_fence_before_sync();
      b5_arrive(sh.dw_empty[zb]);
      if (g >= 0 && n < nv) {
        float* dwp = p.dw + sh.rf[sl][r] * 256 + n * 16;
#pragma unroll
        for (int k4 = 0; k4 < 4; ++k4)
          red_add4(dwp + 4 * k4, rr ? vb[4 * k4] : va[4 * k4], rr ? vb[4 * k4 + 1] : va[4 * k4 + 1],
                   rr ? vb[4 * k4 + 2] : va[4 * k4 + 2], rr ? vb[4 * k4 + 3] : va[4 * k4 + 3]);
        red_add(p.db + sh.rf[sl][r] * 16 + n, dbv);
      }
      if (c + NWB < nbatch) {
        store(c + NWB, nxt);
        if (c + NWB + 1 < nbatch) nxt = fetch(c + NWB + 1);
      }
    }
  } else {
    // ---- MMA issuers (lane 0 issues; the warp waits): warp 12 the Z and dX products, warp 13 the dW | db
    // products, each committing to mma2 (two arrivals per batch)
    const bool dw_role = warp == kB5Issuer + 1;
    const uint32_t xs_u = t5_smem_u32(xpl), ws_u = t5_smem_u32(wpl), ds_u = t5_smem_u32(dpl);
    const uint32_t idz = t5_idesc_bf16(128, 128, 0, 0), idx_ = t5_idesc_bf16(128, 64, 0, 1),
                   idw = t5_idesc_bf16(128, 64, 1, 1), idw80 = t5_idesc_bf16(128, 80, 1, 1);
    constexpr int top = (ND > NS ? ND : NS) - 1;
    bool issued = false;
    auto issue_z = [&](int b) -> bool {
      if (!b5_wait(sh, sh.w_full[b % NWB], (uint32_t)((b / NWB) & 1), p.status)) return false;
      if (b >= 2 && !b5_wait(sh, sh.z_empty[b & 1], (uint32_t)(((b >> 1) - 1) & 1), p.status)) return false;
      if (lane == 0) {
        const uint32_t wsb = ws_u + (uint32_t)((b % NWB) * NS) * kT5Plane;
        uint32_t first = 1;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          t5_mma_terms<NS, NS>(tmem + kB5TZ + (uint32_t)(128 * (b & 1)), idz,
                               [&](int i, int k) { return t5_desc_sw128(xs_u + i * kT5Plane + 32 * k, 16, 1024); },
                               [&](int j, int k) { return t5_desc_sw128(wsb + j * kT5Plane + 32 * k, 16, 1024); }, kk, first);
        t5_commit(t5_smem_u32(&sh.z_full[b & 1]));
      }
      __syncwarp();
      issued = true;
      return true;
    };
    // dXs += dz W: term pairs (dz i, w j), i + j <= max(ND, NS) - 1, the smallest first
    auto issue_dx = [&](int c) -> bool {
      if (!b5_wait(sh, sh.dz_full[c % NZB], (uint32_t)((c / NZB) & 1), p.status)) return false;
      if (lane == 0) {
        const uint32_t wsb = ws_u + (uint32_t)((c % NWB) * NS) * kT5Plane;
        const uint32_t dsb = ds_u + (uint32_t)((c % NZB) * ND) * kT5DzPlane;
        uint32_t first = c == 0 ? 1u : 0u;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
#pragma unroll
          for (int sum = top; sum >= 0; --sum)
#pragma unroll
            for (int i = 0; i <= sum; ++i) {
              const int j = sum - i;
              if (i >= ND || j >= NS) continue;
              const uint64_t bd = t5_desc_sw128(wsb + j * kT5Plane + 2048 * kk, 1024, 1024);
              if constexpr (NS == 1) {   // A = the dz terms in TMEM (over the batch's Z columns)
                const uint32_t at = tmem + kB5TZ + (uint32_t)(128 * (c & 1) + 32 * (kk >> 1) + 16 * i + 8 * (kk & 1));
                t5_mma_bf16_ta(tmem + kB5TdX, at, bd, idx_, first ? 0u : 1u);
              } else {
                const uint64_t ad = t5_desc_sw128(dsb + i * kT5DzPlane + (kk >> 2) * kT5DzHalf + 32 * (kk & 3), 16, 1024);
                t5_mma_bf16(tmem + kB5TdX, ad, bd, idx_, first ? 0u : 1u);
              }
              first = 0;
            }
        t5_commit(t5_smem_u32(&sh.mma2[c & 1]));
      }
      __syncwarp();
      return true;
    };
    // dWs | db = dz^T [X | 1]: term pairs (dz i, x j); x term 0 carries the ones column (N = 80).  Within a sum
    // the pair with j = 0 comes first, so the MMA that clears the accumulator also clears db's column (an MMA
    // with accumulate = 0 clears only the N columns it writes).
    auto issue_dw = [&](int c) -> bool {
      if (!b5_wait(sh, sh.dz_full[c % NZB], (uint32_t)((c / NZB) & 1), p.status)) return false;
      if (c >= 2 && !b5_wait(sh, sh.dw_empty[c & 1], (uint32_t)(((c >> 1) - 1) & 1), p.status)) return false;
      if (lane == 0) {
        const uint32_t dsb = ds_u + (uint32_t)((c % NZB) * ND) * kT5DzPlane;
        uint32_t first = 1;
        const uint32_t dwt = tmem + kB5TdW + kB5DWCols * (uint32_t)(c & 1);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
#pragma unroll
          for (int sum = top; sum >= 0; --sum)
#pragma unroll
            for (int i = sum; i >= 0; --i) {
              const int j = sum - i;
              if (i >= ND || j >= NS) continue;
              const uint64_t ad = t5_desc_sw128(dsb + i * kT5DzPlane + 2048 * kk, kT5DzHalf, 1024);
              const uint64_t bd = t5_desc_sw128(xs_u + j * kT5Plane + 2048 * kk, j == 0 ? NS * kT5Plane : 1024, 1024);
              t5_mma_bf16(dwt, ad, bd, j == 0 ? idw80 : idw, first ? 0u : 1u);
              first = 0;
            }
        t5_commit(t5_smem_u32(&sh.mma2[c & 1]));
      }
      __syncwarp();
      issued = true;
      return true;
    };
    if (dw_role) {
      for (int c = 0; c < nbatch; ++c)
        if (!issue_dw(c)) break;
    } else if (NWB >= 2 && NZB >= 2) {   // Z of the next batch ahead of this batch's dX product
      if (nbatch > 0 && issue_z(0)) {
        for (int c = 0; c < nbatch; ++c) {
          if (c + 1 < nbatch && !issue_z(c + 1)) break;
          if (!issue_dx(c)) break;
        }
      }
    } else {
      for (int c = 0; c < nbatch; ++c)
        if (!issue_z(c) || !issue_dx(c)) break;
    }
    if (issued) {   // every MMA this thread issued has completed before the TMEM is freed
      uint64_t& fin = sh.fin[dw_role ? 1 : 0];
      if (lane == 0) t5_commit(t5_smem_u32(&fin));
      __syncwarp();
      const bool done = t5_mbar_wait(t5_smem_u32(&fin), 0, kT5WaitLimit);
      if (!__all_sync(kFullMask, done) && lane == 0) {
        if (p.status) atomicExch(p.status, 1);
        *abort_v = 1;
      }
    }
  }
  t5_fence_before_sync();
  __syncthreads();
  if (warp == kB5Issuer) {
    t5_fence_after_sync();
    t5_tmem_dealloc(tmem, 512);
  }
}

template <int NS, int ACT>
static int t5_bwd_launch(const K16T5Params& p, int64_t Q, cudaStream_t st) {
  const size_t smem = t5_bwd_smem<NS>();
  auto kern = k16t5_bwd_kernel<NS, ACT>;
  int rc = ensure_dynamic_smem((const void*)kern, smem);
  if (rc) return rc;
  const dim3 grid((unsigned)((p.B + kT5Tokens - 1) / kT5Tokens), (unsigned)Q);
  kern<<<grid, kB5Threads, smem, st>>>(p);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e);
  count_launches(1);
  return GL_OK;
}

template <int NS>
static int t5_bwd_run(const GlK16Args* args, int32_t* status, void* stream) {
  if (!args) return GL_ERR_NULL;
  const GlK16Args& a = *args;
  if (a.B < 0 || a.D < 1 || a.D > 32767 || a.G < 1 || a.NB16 < 1 || a.Q < 1 || a.nbuckets < 0) return GL_ERR_SHAPE;
  if (a.S != kT5Set) return GL_ERR_UNSUPPORTED;
  if (a.act != GL_ACT_RELU && a.act != GL_ACT_IDENTITY) return GL_ERR_UNSUPPORTED;
  if (a.tokens != 0 && a.tokens != kT5Tokens) return GL_ERR_UNSUPPORTED;
  if (a.B == 0 || a.nbuckets == 0) return GL_OK;
  if (!a.x || !a.env || !a.feat || !a.buckets || !a.q_off || !a.rec_off || !a.w || !a.b || !a.counts || !a.c1t ||
      !a.dx || !a.dw || !a.db)
    return GL_ERR_NULL;
  if (a.B > 2147483647LL || a.ldx < a.D || a.Q > 65535 || a.G * a.NB16 > 2147483647LL || a.ldc < a.B || a.lddx < a.D)
    return GL_ERR_SHAPE;
  if (((uintptr_t)a.env & 15) || ((uintptr_t)a.buckets & 15) || ((uintptr_t)a.w & 15) || ((uintptr_t)a.b & 15) ||
      ((uintptr_t)a.dw & 15) || ((uintptr_t)a.db & 3))
    return GL_ERR_ALIGN;
  int optin = 0;
  int rc = device_smem_optin(&optin);
  if (rc) return rc;
  if ((int64_t)(t5_bwd_smem<NS>() + sizeof(B5Shared)) > optin) return GL_ERR_SMEM;
  const K16T5Params p{a.x, a.env, a.feat, a.buckets, a.q_off, a.rec_off, a.w, a.b, a.counts, nullptr, status,
                      (int)a.B, (int)a.D, (int)a.G, (int)a.NB16, (int)a.nbuckets, a.ldx, 0,
                      a.c1t, a.dx, a.dw, a.db, a.ldc, a.lddx};
  cudaStream_t st = (cudaStream_t)stream;
  return a.act == GL_ACT_RELU ? t5_bwd_launch<NS, GL_ACT_RELU>(p, a.Q, st) : t5_bwd_launch<NS, GL_ACT_IDENTITY>(p, a.Q, st);
}

}  // namespace gl

extern "C" int gl_k16_fwd_t5(const GlK16Args* args, int32_t* status, void* stream) {
  return gl::t5_fwd_run<1>(args, status, stream);
}

extern "C" int gl_k16_fwd_t5_f32(const GlK16Args* args, int32_t* status, void* stream) {
  return gl::t5_fwd_run<3>(args, status, stream);
}

extern "C" int gl_k16_bwd_t5(const GlK16Args* args, int32_t* status, void* stream) {
  return gl::t5_bwd_run<1>(args, status, stream);
}

extern "C" int gl_k16_bwd_t5_f32(const GlK16Args* args, int32_t* status, void* stream) {
  return gl::t5_bwd_run<3>(args, status, stream);
}
