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
//   dz  = c1t[g, t] act'(Z + b), masked to the valid neurons, written back as bf16 terms (SIMT epilogue)
//   dXs [128 tokens x 64 positions] += dz W             (A = dz, B = W read MN-major; K = 128 neurons)
//   dWs [128 neurons x 64 positions] = dz^T X           (A = dz read MN-major, B = X read MN-major; K = tokens)
//   db  [128 neurons]                = dz^T 1           (B = a tile whose first row is ones)
// W is the batch's weights expanded over the set's positions (as the forward), so dWs holds each record's
// 16 weight gradients at its positions and zeros elsewhere; the epilogue adds those 16 to dw.  dXs stays in
// TMEM for all of the set's records (a fixed summation order within the set) and is added to dx once per
// CTA: no shared-memory atomics and no fixed-point bounds.  The same shared-memory tile serves as a K-major operand of one
// product and an MN-major operand of another (rows of 64 bf16 in 128-byte-swizzled 8-row atoms: for K-major
// operands the rows are M or N, for MN-major ones K).  bf16 parameters (NS = 1): x and w one bf16 term, dz
// two (hi + lo, the reference's split precision); fp32 parameters (NS = 3): three terms each, term pairs
// i + j <= 2 per product, as the forward.  TMEM columns: Z [0, 128) (db reuses [0, 16) once the epilogue
// has read Z), dXs [128, 192), dWs [192, 256).  The CTA's steps run in order (one mbarrier, armed by
// tcgen05.commit after each group of MMAs and waited on with an iteration limit); two CTAs share an SM for
// bf16 parameters, so one's MMAs run under the other's epilogues.
constexpr uint32_t kT5DzPlane = 32768;    // dz [128 tokens][128 neurons]: two 64-neuron halves of 16 KiB
constexpr uint32_t kT5DzHalf = 16384;
constexpr uint32_t kT5OnesBytes = 2048;   // [16 rows][64 tokens] bf16, row 0 ones
constexpr int kT5BwdMaxBuckets = 256;

template <int NS>
__host__ __device__ constexpr int t5_dz_terms() { return NS == 1 ? 2 : 3; }

template <int NS>
static size_t t5_bwd_smem() {
  return (size_t)2 * NS * kT5Plane + (size_t)t5_dz_terms<NS>() * kT5DzPlane + kT5OnesBytes + 1024;
}

// MMAs of a product over term planes a_i (NA terms) and b_j (NB terms), pairs i + j <= max(NA, NB) - 1, the
// smallest first; kk is the 16-wide K step.  `first` clears the accumulator on the first MMA.
template <int NA, int NB, typename FA, typename FB>
__device__ __forceinline__ void t5_mma_terms(uint32_t d_t, uint32_t idesc, FA adesc, FB bdesc, int kk, uint32_t& first) {
  constexpr int top = (NA > NB ? NA : NB) - 1;
#pragma unroll
  for (int sum = top; sum >= 0; --sum)
#pragma unroll
    for (int i = 0; i <= sum; ++i) {
      const int j = sum - i;
      if (i < NA && j < NB) {
        t5_mma_bf16(d_t, adesc(i, kk), bdesc(j, kk), idesc, first ? 0u : 1u);
        first = 0;
      }
    }
}

template <int NS, int ACT>
__global__ void __launch_bounds__(kT5Threads, NS == 1 ? 2 : 1) k16t5_bwd_kernel(const K16T5Params p) {
  constexpr int ND = t5_dz_terms<NS>();
  extern __shared__ unsigned char t5_raw[];
  __shared__ __align__(8) uint64_t mbar;
  __shared__ uint32_t tmem_s;
  __shared__ int abort_s;
  __shared__ int fq[kT5Set];
  __shared__ __align__(16) float bias_s[8][16];
  __shared__ int rg_s[2][8], rnv_s[2][8];
  __shared__ long long rf_s[2][8];
  __shared__ signed char kx_s[8][kT5Set];   // per record of the batch: position -> input index, or -1
  __shared__ int bk_rec[kT5BwdMaxBuckets + 1];
  __shared__ int4 bk_row[kT5BwdMaxBuckets];
  unsigned char* smem = reinterpret_cast<unsigned char*>(((uintptr_t)t5_raw + 1023) & ~(uintptr_t)1023);
  unsigned char* xpl = smem;                          // NS planes X [128 tokens][64 positions]
  unsigned char* wpl = xpl + NS * kT5Plane;           // NS planes W [128 neurons][64 positions]
  unsigned char* dpl = wpl + NS * kT5Plane;           // ND planes dz [128 tokens][2 x 64 neurons]
  unsigned char* opl = dpl + ND * kT5DzPlane;         // ones [16][64]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int q = blockIdx.y, t0 = blockIdx.x * kT5Tokens;
  if (warp == 0) t5_tmem_alloc(t5_smem_u32(&tmem_s), 256);
  if (tid == 0) {
    t5_mbar_init(t5_smem_u32(&mbar), 1);
    abort_s = 0;
  }
  if (tid < kT5Set) {
    const int d = (int)(uint16_t)__ldg(p.feat + (int64_t)q * kT5Set + tid);
    fq[tid] = d < p.D ? d : p.D - 1;
  }
  const int qa = min(max(__ldg(p.q_off + q), 0), p.nbk), qb = min(max(__ldg(p.q_off + q + 1), qa), p.nbk);
  const int ra = __ldg(p.rec_off + qa), rb = __ldg(p.rec_off + qb);
  const bool cached = qb - qa <= kT5BwdMaxBuckets;
  if (cached) {
    for (int i = tid; i <= qb - qa; i += kT5Threads) bk_rec[i] = __ldg(p.rec_off + qa + i);
    for (int i = tid; i < qb - qa; i += kT5Threads) bk_row[i] = __ldg(reinterpret_cast<const int4*>(p.buckets) + qa + i);
  }
  for (int i = tid; i < NS * (int)kT5Plane / 16; i += kT5Threads) reinterpret_cast<uint4*>(wpl)[i] = make_uint4(0, 0, 0, 0);
  for (int i = tid; i < (int)kT5OnesBytes / 16; i += kT5Threads)   // row 0 (the first 128 bytes): bf16 ones
    reinterpret_cast<uint4*>(opl)[i] = i < 8 ? make_uint4(0x3F803F80u, 0x3F803F80u, 0x3F803F80u, 0x3F803F80u)
                                             : make_uint4(0, 0, 0, 0);
  for (int i = tid; i < 8 * kT5Set; i += kT5Threads) (&kx_s[0][0])[i] = -1;
  __syncthreads();
  for (int c = tid; c < kT5Tokens * 8; c += kT5Threads) {   // stage X, as the forward
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
  if (tid < 8) {
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
  const uint32_t xs_u = t5_smem_u32(xpl), ws_u = t5_smem_u32(wpl), ds_u = t5_smem_u32(dpl), os_u = t5_smem_u32(opl);
  const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;   // this warp's TMEM lanes
  const int wrow = 16 * warp + (lane >> 1);                       // the W row this thread expands
  const int erow = 32 * (warp & 3) + lane, et = t0 + erow;        // token row of the dz epilogue
  const int eh = warp >> 2;                                       // its 64 neurons: records 4 eh .. 4 eh + 3
  uint32_t use = 0;
  auto wait_mma = [&]() {
    const bool got = abort_s == 0 && t5_mbar_wait(t5_smem_u32(&mbar), use & 1u, kT5WaitLimit);
    ++use;
    if (!got) {
      if (p.status) atomicExch(p.status, 1);
      abort_s = 1;
    }
    t5_fence_after_sync();
    return __all_sync(kFullMask, got);   // warp-uniform: the TMEM loads after it are .sync.aligned
  };
  auto kx_pos = [](const uint2& env, int e) {
    const uint32_t word = e < 4 ? env.x : env.y;
    return min((word >> (8 * (e & 3))) & 0xffu, (uint32_t)(kT5Set - 1));
  };
  T5Ops ops = t5_load_ops<NS>(p, rg_s[0], rf_s[0], tid);
  uint2 env_prev = make_uint2(0, 0);
  bool kown_prev = false;
  for (int b = 0; b < nbatch; ++b) {   // leaves only through abort_s, read by all threads after a barrier
    const int sl = b & 1;
    const uint2 env_cur = ops.env;
    const bool kown = (lane >> 1) == 0 && rg_s[sl][warp] >= 0;   // lanes 0 / 1 map the record's positions
    // the position map of record `warp`: the previous batch's entries (read by the previous dW epilogue,
    // before the last barrier) are cleared, then this batch's are written
    if (kown_prev)
#pragma unroll
      for (int e = 0; e < 8; ++e) kx_s[warp][kx_pos(env_prev, e)] = -1;
    __syncwarp();
    if (kown)
#pragma unroll
      for (int e = 0; e < 8; ++e) kx_s[warp][kx_pos(env_cur, e)] = (signed char)(8 * (lane & 1) + e);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      uint16_t terms[NS];
      t5_terms<NS>(ops.w[e], terms);
      const uint32_t off = t5_wpos(env_cur, e, wrow);
#pragma unroll
      for (int j = 0; j < NS; ++j) *reinterpret_cast<uint16_t*>(wpl + j * kT5Plane + off) = terms[j];
    }
    if (tid < 128) bias_s[tid >> 4][tid & 15] = ops.bias;
    if (tid < 8) {
      const T5Rec rc = t5_record(p, qa, qb, rb, ra + 8 * (b + 1) + tid, cached, bk_rec, bk_row);
      rg_s[sl ^ 1][tid] = rc.g;
      rf_s[sl ^ 1][tid] = rc.f;
      rnv_s[sl ^ 1][tid] = rc.nv;
    }
    t5_fence_smem_to_async();
    __syncthreads();
    if (tid == 0 && !abort_s) {   // Z = X W^T
      t5_fence_after_sync();
      uint32_t first = 1;
      const uint32_t idz = t5_idesc_bf16(128, 128, 0, 0);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        t5_mma_terms<NS, NS>(tmem, idz,
                             [&](int i, int k) { return t5_desc_sw128(xs_u + i * kT5Plane + 32 * k, 16, 1024); },
                             [&](int j, int k) { return t5_desc_sw128(ws_u + j * kT5Plane + 32 * k, 16, 1024); }, kk, first);
      t5_commit(t5_smem_u32(&mbar));
    }
    if (b + 1 < nbatch) ops = t5_load_ops<NS>(p, rg_s[sl ^ 1], rf_s[sl ^ 1], tid);   // under the MMAs
    if (wait_mma()) {   // dz epilogue: token erow, neurons 64 eh .. 64 eh + 63
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        float v[32];
        t5_ld32(tmem + lane_base + (uint32_t)(64 * eh + 32 * c), v);
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
          const int r = 4 * eh + 2 * c + rr, g = rg_s[sl][r], nv = rnv_s[sl][r];
          const float c1 = (g >= 0 && et < p.B) ? __ldg(p.c1t + (int64_t)g * p.ldc + et) : 0.f;
          uint32_t pk[ND][8];
#pragma unroll
          for (int n2 = 0; n2 < 8; ++n2) {
            float dz2[2];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              const int n = 2 * n2 + u;
              dz2[u] = n < nv ? c1 * dact_f<ACT>(v[16 * rr + n] + bias_s[r][n]) : 0.f;
            }
            uint16_t t0s[ND], t1s[ND];
            t5_terms<ND>(dz2[0], t0s);
            t5_terms<ND>(dz2[1], t1s);
#pragma unroll
            for (int i = 0; i < ND; ++i) pk[i][n2] = (uint32_t)t0s[i] | ((uint32_t)t1s[i] << 16);
          }
#pragma unroll
          for (int i = 0; i < ND; ++i)
#pragma unroll
            for (int hh = 0; hh < 2; ++hh)
              *reinterpret_cast<uint4*>(dpl + i * kT5DzPlane + eh * kT5DzHalf + t5_sw128_off(erow, 32 * c + 16 * rr + 8 * hh)) =
                  make_uint4(pk[i][4 * hh], pk[i][4 * hh + 1], pk[i][4 * hh + 2], pk[i][4 * hh + 3]);
        }
      }
    }
    t5_fence_smem_to_async();
    t5_fence_before_sync();
    __syncthreads();
    if (tid == 0 && !abort_s) {   // dXs += dz W, dWs = dz^T X, db = dz^T 1
      t5_fence_after_sync();
      uint32_t first = b == 0 ? 1u : 0u;
      const uint32_t idx_ = t5_idesc_bf16(128, 64, 0, 1), idw = t5_idesc_bf16(128, 64, 1, 1), idb = t5_idesc_bf16(128, 16, 1, 0);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk)
        t5_mma_terms<ND, NS>(tmem + 128, idx_,
                             [&](int i, int k) { return t5_desc_sw128(ds_u + i * kT5DzPlane + (k >> 2) * kT5DzHalf + 32 * (k & 3), 16, 1024); },
                             [&](int j, int k) { return t5_desc_sw128(ws_u + j * kT5Plane + 2048 * k, 1024, 1024); }, kk, first);
      first = 1;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk)
        t5_mma_terms<ND, NS>(tmem + 192, idw,
                             [&](int i, int k) { return t5_desc_sw128(ds_u + i * kT5DzPlane + 2048 * k, kT5DzHalf, 1024); },
                             [&](int j, int k) { return t5_desc_sw128(xs_u + j * kT5Plane + 2048 * k, 1024, 1024); }, kk, first);
      first = 1;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk)
        t5_mma_terms<ND, 1>(tmem, idb,
                            [&](int i, int k) { return t5_desc_sw128(ds_u + i * kT5DzPlane + 2048 * k, kT5DzHalf, 1024); },
                            [&](int, int k) { return t5_desc_sw128(os_u + 32 * (k & 3), 16, 1024); }, kk, first);
      t5_commit(t5_smem_u32(&mbar));
    }
    if (wait_mma()) {   // dW / db epilogue: neuron 32 (warp % 4) + lane, positions 32 eh ..
      const int n = 32 * (warp & 3) + lane, r = n >> 4, nn = n & 15, g = rg_s[sl][r];
      const bool live = g >= 0 && nn < rnv_s[sl][r];
      float v[32];
      t5_ld32(tmem + lane_base + (uint32_t)(192 + 32 * eh), v);
      const float dbv = t5_ld1(tmem + lane_base);
      if (live) {
        float* dwp = p.dw + rf_s[sl][r] * 256 + nn * 16;
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const int k = kx_s[r][32 * eh + c];
          if (k >= 0) red_add(dwp + k, v[c]);
        }
        if (eh == 0) red_add(p.db + rf_s[sl][r] * 16 + nn, dbv);
      }
    }
    // clear the weight positions this batch wrote (its MMAs have completed; only they read W)
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const uint32_t off = t5_wpos(env_cur, e, wrow);
#pragma unroll
      for (int j = 0; j < NS; ++j) *reinterpret_cast<uint16_t*>(wpl + j * kT5Plane + off) = 0;
    }
    env_prev = env_cur;
    kown_prev = kown;
    t5_fence_before_sync();
    __syncthreads();
    if (abort_s) break;
  }
  if (nbatch > 0 && !abort_s) {   // dx[t, feat[q][s]] += dXs (every MMA has completed: the last wait)
    float v[32];
    t5_ld32(tmem + lane_base + (uint32_t)(128 + 32 * eh), v);
    if (et < p.B) {
      float* dxr = p.dx + (int64_t)et * p.lddx;
#pragma unroll
      for (int c = 0; c < 32; ++c)
        if (v[c] != 0.f || v[c] != v[c]) atomicAdd(dxr + fq[32 * eh + c], v[c]);
    }
  }
  t5_fence_before_sync();
  __syncthreads();
  if (warp == 0) {
    t5_fence_after_sync();
    t5_tmem_dealloc(tmem, 256);
  }
}

template <int NS, int ACT>
static int t5_bwd_launch(const K16T5Params& p, int64_t Q, cudaStream_t st) {
  const size_t smem = t5_bwd_smem<NS>();
  auto kern = k16t5_bwd_kernel<NS, ACT>;
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
      ((uintptr_t)a.dw & 3) || ((uintptr_t)a.db & 3))
    return GL_ERR_ALIGN;
  int optin = 0;
  int rc = device_smem_optin(&optin);
  if (rc) return rc;
  if ((int64_t)t5_bwd_smem<NS>() > optin) return GL_ERR_SMEM;
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
