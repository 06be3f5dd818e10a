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
// Both are FMA kernels fed from shared memory.  A shared-memory load delivers at most 32 floats
// per wavefront whatever the broadcast pattern, against 128 FMAs per clock per SM, so every x
// value a lane loads must feed several FMAs from registers: the forward keeps 8 neurons per lane
// (32 FMAs per 128-bit load), the backward 4 neurons per lane (8 FMAs per loaded value for z
// and dW, plus the dX products from the same registers).  Lane layouts are described at each
// kernel.  The forward adds per-bucket token sums into a shared row and flushes them with one
// global reduction per (bucket, token); the backward keeps dW/db in registers across the token
// chunk, adds dX into a shared [S][TT] tile with conflict-free shared atomics, and ends with
// global reductions of dW/db (per record) and of the tile into dx.
#include "common.cuh"

namespace gl {

constexpr int kK16FwdThreads = 256;
constexpr int kK16BwdThreads = 256;
constexpr int kK16FwdStep = 64;    // tokens per forward warp step (16 token groups x 4)
constexpr int kK16BwdStep = 16;    // tokens per backward warp step (8 token groups x 2)
constexpr int kK16FwdPass = 32;    // buckets per forward pass (rows of the shared token-sum tile)
constexpr int kK16BwdPass = 64;    // buckets per backward pass (rows of the shared coefficient tile)
constexpr int kK16MaxPass = 64;
constexpr int kK16MaxS = 256;      // env holds uint8 local positions
constexpr int kK16MaxTT = 512;

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
  int rstart[kK16MaxPass + 1];
  int g[kK16MaxPass];
  int first[kK16MaxPass];
};

// One record staged in shared memory by its warp (weights [16][16], bias [16], local positions).
struct __align__(16) K16Stage {
  float w[256];
  float b[16];
  uint32_t env[4];
};

struct K16Rec {
  int i, g, j16;
  bool ok;
};

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const unsigned d = (unsigned)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

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

// Bucket row of pass-relative record r: the largest i with rstart[i] <= r (empty buckets skipped),
// and the record it names; `ok` is false for a malformed row (the record is then skipped).
__device__ __forceinline__ K16Rec k16_meta(const K16PassInfo& ps, const K16Params& p, int np, int r) {
  int lo = 0, hi = np;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (ps.rstart[mid] <= r) lo = mid; else hi = mid;
  }
  K16Rec m;
  m.i = lo;
  m.g = ps.g[lo];
  m.j16 = ps.first[lo] + (r - ps.rstart[lo]);
  m.ok = m.g >= 0 && m.g < p.G && m.j16 >= 0 && m.j16 < p.NB16;
  return m;
}

// Warp-cooperative asynchronous copy of a record's weights, bias and local positions into `st`
// (one commit group per call, empty for a skipped record).
__device__ __forceinline__ void k16_prefetch(K16Stage& st, const K16Params& p, const K16Rec& m, int lane) {
  if (m.ok) {
    const int64_t f = (int64_t)m.g * p.NB16 + m.j16;
    const float* wsrc = p.w + f * 256 + lane * 8;
    cp_async16(st.w + lane * 8, wsrc);
    cp_async16(st.w + lane * 8 + 4, wsrc + 4);
    if (lane < 4) cp_async16(st.b + lane * 4, p.b + f * 16 + lane * 4);
    else if (lane == 4) cp_async16(st.env, p.env + f * 16);
  }
  cp_async_commit();
}

// Stage x[t0 + t, feat[q][s]] into xs[s * ld + t] (zeros past the batch, up to TT) and the features.
__device__ __forceinline__ void k16_stage_x(float* __restrict__ xs, int ld, int* __restrict__ fq,
                                            const K16Params& p, int q, int t0, int ntok) {
  for (int s = threadIdx.x; s < p.S; s += blockDim.x) {
    const int d = (int)(uint16_t)__ldg(p.feat + (int64_t)q * p.S + s);
    fq[s] = d < p.D ? d : p.D - 1;
  }
  __syncthreads();
  const int n = p.S * p.TT;
  for (int e = threadIdx.x; e < n; e += blockDim.x) {
    const int s = e / p.TT, t = e - s * p.TT;
    xs[s * ld + t] = t < ntok ? __ldg(p.x + (int64_t)(t0 + t) * p.ldx + fq[s]) : 0.f;
  }
}

// Local position k of a staged record (clamped to the set).
__device__ __forceinline__ int k16_pos(const K16Stage& st, int k, int smax) {
  return min((int)((st.env[k >> 2] >> (8 * (k & 3))) & 0xffu), smax);
}

// Forward.  lane = (token group tg = lane >> 1: 4 tokens, neuron octet no = lane & 1: 8 neurons);
// a warp step covers one record and 64 tokens.  Each lane keeps its 8 neurons' 128 weights in
// registers, so one 128-bit shared load of x feeds 32 FMAs.  The warp's next record is copied
// into shared memory (cp.async) while the current one runs.
template <int ACT>
__global__ void __launch_bounds__(kK16FwdThreads, 1) k16_fwd_kernel(const K16Params p) {
  constexpr int NW = kK16FwdThreads / 32;
  extern __shared__ __align__(16) float sm[];
  const int TT = p.TT;                     // a multiple of kK16FwdStep
  float* xs = sm;                          // [S][TT]
  float* ys = sm + (size_t)p.S * TT;       // [kK16FwdPass][TT] per-bucket token sums
  __shared__ K16PassInfo ps;
  __shared__ int fq[kK16MaxS];
  __shared__ K16Stage stg[NW][2];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int q = blockIdx.x, t0 = blockIdx.y * TT;
  const int ntok = min(TT, p.B - t0);
  k16_stage_x(xs, TT, fq, p, q, t0, ntok);
  for (int e = threadIdx.x; e < kK16FwdPass * TT; e += kK16FwdThreads) ys[e] = 0.f;
  const int no = lane & 1, tg = lane >> 1;
  const int b_hi = min(max(__ldg(p.q_off + q + 1), 0), p.nbk);
  const int b_lo = min(max(__ldg(p.q_off + q), 0), b_hi);
  for (int p0 = b_lo; p0 < b_hi; p0 += kK16FwdPass) {
    const int np = min(kK16FwdPass, b_hi - p0);
    __syncthreads();
    k16_load_pass(ps, p, p0, np);
    __syncthreads();
    const int nrec = ps.rstart[np];
    K16Rec cur;
    cur.ok = false;
    if (warp < nrec) {
      cur = k16_meta(ps, p, np, warp);
      k16_prefetch(stg[warp][0], p, cur, lane);
    }
    int buf = 0;
    for (int r = warp; r < nrec; r += NW) {
      K16Rec nxt;
      nxt.ok = false;
      if (r + NW < nrec) {
        nxt = k16_meta(ps, p, np, r + NW);
        k16_prefetch(stg[warp][buf ^ 1], p, nxt, lane);
        cp_async_wait<1>();
      } else {
        cp_async_wait<0>();
      }
      __syncwarp();
      if (cur.ok) {
        const K16Stage& st = stg[warp][buf];
        const int nv = min(max(__ldg(p.counts + cur.g) - (cur.j16 * 16 + no * 8), 0), 8);  // valid neurons
        float wr[8][16], bb[8];
#pragma unroll
        for (int n = 0; n < 8; ++n)
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const float4 a = reinterpret_cast<const float4*>(st.w + (no * 8 + n) * 16)[c];
            wr[n][4 * c] = a.x; wr[n][4 * c + 1] = a.y; wr[n][4 * c + 2] = a.z; wr[n][4 * c + 3] = a.w;
          }
#pragma unroll
        for (int n = 0; n < 8; ++n) bb[n] = st.b[no * 8 + n];
        int off[16];
#pragma unroll
        for (int k = 0; k < 16; ++k) off[k] = k16_pos(st, k, p.S - 1) * TT;
        float* yrow = ys + cur.i * TT;
        for (int tq = 0; tq < ntok; tq += kK16FwdStep) {
          const int col = tq + 4 * tg;
          float z[8][4];
#pragma unroll
          for (int n = 0; n < 8; ++n) z[n][0] = z[n][1] = z[n][2] = z[n][3] = bb[n];
#pragma unroll
          for (int k = 0; k < 16; ++k) {
            const float4 v = *reinterpret_cast<const float4*>(xs + off[k] + col);
#pragma unroll
            for (int n = 0; n < 8; ++n) {
              z[n][0] = fmaf(wr[n][k], v.x, z[n][0]);
              z[n][1] = fmaf(wr[n][k], v.y, z[n][1]);
              z[n][2] = fmaf(wr[n][k], v.z, z[n][2]);
              z[n][3] = fmaf(wr[n][k], v.w, z[n][3]);
            }
          }
          float a[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int n = 0; n < 8; ++n)
            if (n < nv)
#pragma unroll
              for (int j = 0; j < 4; ++j) a[j] += act_f<ACT>(z[n][j]);
          // sum the two octets (lane bit 0); lane `no` ends with tokens col + 2 no, col + 2 no + 1
          const float s0 = no ? a[0] : a[2], s1 = no ? a[1] : a[3];
          const float k0 = no ? a[2] : a[0], k1 = no ? a[3] : a[1];
          const float v0 = k0 + __shfl_xor_sync(kFullMask, s0, 1);
          const float v1 = k1 + __shfl_xor_sync(kFullMask, s1, 1);
          const int t = col + 2 * no;
          if (t < ntok) atomicAdd(yrow + t, v0);
          if (t + 1 < ntok) atomicAdd(yrow + t + 1, v1);
        }
      }
      __syncwarp();
      cur = nxt;
      buf ^= 1;
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

// Backward.  lane bits: 4 = lo, 3..1 = token group tg (2 tokens), 0 = hi; the lane's neuron quad
// is nq = lo + 2 hi (4 neurons).  A warp step covers one record and 16 tokens.  A lane keeps its
// quad's 64 weights, 64 dW sums and the step's x values (16 inputs x 2 tokens) in registers, so
// each x value feeds 8 FMAs (z and dW).  dX: the lane forms its quad's partial sums
// sum_n dz[n][t] w[n][k]; a transpose-reduction over the 4 quads (lane bit 0 splits the 2 tokens,
// lane bit 4 the 2 inputs of a pair) leaves one (k, t) per lane, and each half-warp adds 16
// consecutive tokens of one row of the dX tile.  Lanes with lo set hold their record's inputs in
// pair-swapped order (k ^ 1), which makes both reduction stages select-free and gives each
// half-warp a single x row per load; the order is undone when dW is written.
template <int ACT>
__global__ void __launch_bounds__(kK16BwdThreads, 1) k16_bwd_kernel(const K16Params p) {
  constexpr int NW = kK16BwdThreads / 32;
  extern __shared__ __align__(16) float sm[];
  const int TT = p.TT;                          // a multiple of 32
  const int LD = TT + 16;                       // row stride of the x and dX tiles
  float* xs = sm;                               // [S][LD]
  float* dxs = xs + (size_t)p.S * LD;           // [S][LD] dX tile
  float* c1s = dxs + (size_t)p.S * LD;          // [kK16BwdPass][TT] per-bucket coefficients
  __shared__ K16PassInfo ps;
  __shared__ int fq[kK16MaxS];
  __shared__ K16Stage stg[NW][2];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int q = blockIdx.x, t0 = blockIdx.y * TT;
  const int ntok = min(TT, p.B - t0);
  k16_stage_x(xs, LD, fq, p, q, t0, ntok);
  for (int e = threadIdx.x; e < p.S * LD; e += kK16BwdThreads) dxs[e] = 0.f;
  const bool lo = lane & 16, hi = lane & 1;
  const int tg = (lane >> 1) & 7;
  const int nq = (lo ? 1 : 0) + (hi ? 2 : 0);
  const int b_hi = min(max(__ldg(p.q_off + q + 1), 0), p.nbk);
  const int b_lo = min(max(__ldg(p.q_off + q), 0), b_hi);
  for (int p0 = b_lo; p0 < b_hi; p0 += kK16BwdPass) {
    const int np = min(kK16BwdPass, b_hi - p0);
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
    K16Rec cur;
    cur.ok = false;
    if (warp < nrec) {
      cur = k16_meta(ps, p, np, warp);
      k16_prefetch(stg[warp][0], p, cur, lane);
    }
    int buf = 0;
    for (int r = warp; r < nrec; r += NW) {
      K16Rec nxt;
      nxt.ok = false;
      if (r + NW < nrec) {
        nxt = k16_meta(ps, p, np, r + NW);
        k16_prefetch(stg[warp][buf ^ 1], p, nxt, lane);
        cp_async_wait<1>();
      } else {
        cp_async_wait<0>();
      }
      __syncwarp();
      if (cur.ok) {
        const K16Stage& st = stg[warp][buf];
        const int64_t f = (int64_t)cur.g * p.NB16 + cur.j16;
        const int nv = min(max(__ldg(p.counts + cur.g) - (cur.j16 * 16 + nq * 4), 0), 4);  // valid neurons
        float wr[4][16], bb[4];
#pragma unroll
        for (int n = 0; n < 4; ++n)
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const float4 a = reinterpret_cast<const float4*>(st.w + (nq * 4 + n) * 16)[c];
            wr[n][4 * c] = lo ? a.y : a.x;
            wr[n][4 * c + 1] = lo ? a.x : a.y;
            wr[n][4 * c + 2] = lo ? a.w : a.z;
            wr[n][4 * c + 3] = lo ? a.z : a.w;
          }
        {
          const float4 b4 = reinterpret_cast<const float4*>(st.b)[nq];
          bb[0] = b4.x; bb[1] = b4.y; bb[2] = b4.z; bb[3] = b4.w;
        }
        int off[16];
#pragma unroll
        for (int k = 0; k < 16; ++k) off[k] = k16_pos(st, lo ? (k ^ 1) : k, p.S - 1) * LD;
        float dwacc[4][16], dbacc[4];
#pragma unroll
        for (int n = 0; n < 4; ++n) {
          dbacc[n] = 0.f;
#pragma unroll
          for (int k = 0; k < 16; ++k) dwacc[n][k] = 0.f;
        }
        const float* crow = c1s + cur.i * TT;
        for (int tq = 0; tq < ntok; tq += kK16BwdStep) {
          const int col = tq + 2 * tg;
          float xv[16][2];
#pragma unroll
          for (int k = 0; k < 16; ++k) {
            const float2 v = *reinterpret_cast<const float2*>(xs + off[k] + col);
            xv[k][0] = v.x; xv[k][1] = v.y;
          }
          const float2 c2 = *reinterpret_cast<const float2*>(crow + col);
          float z0[4], z1[4];
#pragma unroll
          for (int n = 0; n < 4; ++n) z0[n] = z1[n] = bb[n];
#pragma unroll
          for (int k = 0; k < 16; ++k)
#pragma unroll
            for (int n = 0; n < 4; ++n) {
              z0[n] = fmaf(wr[n][k], xv[k][0], z0[n]);
              z1[n] = fmaf(wr[n][k], xv[k][1], z1[n]);
            }
          float d0[4], d1[4];
#pragma unroll
          for (int n = 0; n < 4; ++n) {
            d0[n] = n < nv ? k16_dz<ACT>(c2.x, z0[n]) : 0.f;
            d1[n] = n < nv ? k16_dz<ACT>(c2.y, z1[n]) : 0.f;
            dbacc[n] += d0[n] + d1[n];
          }
#pragma unroll
          for (int k = 0; k < 16; ++k)
#pragma unroll
            for (int n = 0; n < 4; ++n) dwacc[n][k] = fmaf(d1[n], xv[k][1], fmaf(d0[n], xv[k][0], dwacc[n][k]));
          // dX partials of the token this lane keeps (dk) and of the one it sends (ds), per input
          float pk[16], ps_[16];
#pragma unroll
          for (int k = 0; k < 16; ++k) {
            float a = 0.f, b = 0.f;
#pragma unroll
            for (int n = 0; n < 4; ++n) {
              a = fmaf(hi ? d1[n] : d0[n], wr[n][k], a);
              b = fmaf(hi ? d0[n] : d1[n], wr[n][k], b);
            }
            pk[k] = a;
            ps_[k] = b;
          }
#pragma unroll
          for (int k = 0; k < 16; ++k) pk[k] += __shfl_xor_sync(kFullMask, ps_[k], 1);
          float* drow = dxs + col + (hi ? 1 : 0);
#pragma unroll
          for (int m = 0; m < 8; ++m)
            atomicAdd(drow + off[2 * m], pk[2 * m] + __shfl_xor_sync(kFullMask, pk[2 * m + 1], 16));
        }
        // dW: transpose-reduce the 64 sums over the 8 token groups (lane bits 3, 2, 1); the lane ends
        // with positions 2 tg, 2 tg + 1 of its 4 neurons (inputs swapped when lo)
        float r8[4][8], r4[4][4], r2[4][2];
        const bool b3 = lane & 8, b2 = lane & 4, b1 = lane & 2;
#pragma unroll
        for (int n = 0; n < 4; ++n)
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const float keep = b3 ? dwacc[n][kk + 8] : dwacc[n][kk];
            const float send = b3 ? dwacc[n][kk] : dwacc[n][kk + 8];
            r8[n][kk] = keep + __shfl_xor_sync(kFullMask, send, 8);
          }
#pragma unroll
        for (int n = 0; n < 4; ++n)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const float keep = b2 ? r8[n][kk + 4] : r8[n][kk];
            const float send = b2 ? r8[n][kk] : r8[n][kk + 4];
            r4[n][kk] = keep + __shfl_xor_sync(kFullMask, send, 4);
          }
#pragma unroll
        for (int n = 0; n < 4; ++n)
#pragma unroll
          for (int kk = 0; kk < 2; ++kk) {
            const float keep = b1 ? r4[n][kk + 2] : r4[n][kk];
            const float send = b1 ? r4[n][kk] : r4[n][kk + 2];
            r2[n][kk] = keep + __shfl_xor_sync(kFullMask, send, 2);
          }
#pragma unroll
        for (int n = 0; n < 4; ++n)
#pragma unroll
          for (int s = 2; s <= 8; s <<= 1) dbacc[n] += __shfl_xor_sync(kFullMask, dbacc[n], s);
        if (nv > 0) {
          float* dwp = p.dw + (f * 16 + nq * 4) * 16 + 2 * tg;
#pragma unroll
          for (int m = 0; m < 4; ++m) red_add2(dwp + 16 * m, lo ? r2[m][1] : r2[m][0], lo ? r2[m][0] : r2[m][1]);
          if (tg == 0) red_add4(p.db + f * 16 + nq * 4, dbacc[0], dbacc[1], dbacc[2], dbacc[3]);
        }
      }
      __syncwarp();
      cur = nxt;
      buf ^= 1;
    }
  }
  __syncthreads();
  const int n_el = p.S * ntok;
  for (int e = threadIdx.x; e < n_el; e += kK16BwdThreads) {
    const int s = e / ntok, t = e - s * ntok;
    const float v = dxs[s * LD + t];
    if (v != 0.f) red_add(p.dx + (int64_t)(t0 + t) * p.lddx + fq[s], v);
  }
}

static size_t k16_fwd_smem(int S, int TT) { return ((size_t)S + kK16FwdPass) * TT * sizeof(float); }
static size_t k16_bwd_smem(int S, int TT) {
  return ((size_t)2 * S * (TT + 16) + (size_t)kK16BwdPass * TT) * sizeof(float);
}

template <int ACT>
static const void* k16_kernel(bool bwd) {
  return bwd ? (const void*)k16_bwd_kernel<ACT> : (const void*)k16_fwd_kernel<ACT>;
}

// Static shared memory of a kernel (pass info, feature list, record stages).
static int k16_static_smem(bool bwd, size_t* bytes) {
  cudaFuncAttributes fa;
  const cudaError_t e = cudaFuncGetAttributes(&fa, k16_kernel<GL_ACT_RELU>(bwd));
  if (e != cudaSuccess) return set_cuda_error(e);
  *bytes = fa.sharedSizeBytes;
  return GL_OK;
}

// Token chunk: a multiple of 64 (forward) or 32 (backward), at most 512 / 256, the largest that fits.
static int k16_pick_tt(int64_t B, int S, bool bwd, int optin, size_t stat) {
  const int step = bwd ? 32 : kK16FwdStep;
  int64_t tt = (B + step - 1) / step * step;
  const int64_t cap = bwd ? 256 : kK16MaxTT;
  if (tt > cap) tt = cap;
  for (; tt >= step; tt -= step) {
    const size_t need = bwd ? k16_bwd_smem(S, (int)tt) : k16_fwd_smem(S, (int)tt);
    if ((int64_t)(need + stat) <= optin) return (int)tt;
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
  if (((uintptr_t)a.env & 15) || ((uintptr_t)a.w & 15) || ((uintptr_t)a.b & 15) || ((uintptr_t)a.buckets & 15))
    return GL_ERR_ALIGN;
  if (a.act != GL_ACT_RELU && a.act != GL_ACT_IDENTITY) return GL_ERR_UNSUPPORTED;
  if (!bwd) {
    if (!a.pre) return GL_ERR_NULL;
    if (a.ldp < a.G) return GL_ERR_SHAPE;
  } else {
    if (!a.c1t || !a.dx || !a.dw || !a.db) return GL_ERR_NULL;
    if (a.ldc < a.B || a.lddx < a.D) return GL_ERR_SHAPE;
    if (((uintptr_t)a.dw & 15) || ((uintptr_t)a.db & 15) || ((uintptr_t)a.c1t & 3)) return GL_ERR_ALIGN;
  }
  return GL_OK;
}

static int k16_launch(const GlK16Args& a, void* stream, bool bwd) {
  int rc = k16_check(a, bwd);
  if (rc) return rc;
  if (a.B == 0 || a.Q == 0) return GL_OK;
  int optin = 0;
  if ((rc = device_smem_optin(&optin))) return rc;
  size_t stat = 0;
  if ((rc = k16_static_smem(bwd, &stat))) return rc;
  const int TT = a.tokens ? (int)a.tokens : k16_pick_tt(a.B, (int)a.S, bwd, optin, stat);
  if (TT < 0) return GL_ERR_SMEM;
  const int step = bwd ? 32 : kK16FwdStep;
  if (TT < step || TT % step || TT > 1024) return GL_ERR_UNSUPPORTED;
  const size_t smem = bwd ? k16_bwd_smem((int)a.S, TT) : k16_fwd_smem((int)a.S, TT);
  if ((int64_t)(smem + stat) > optin) return GL_ERR_SMEM;
  const int64_t chunks = (a.B + TT - 1) / TT;
  if (a.Q > 2147483647LL || chunks > 65535) return GL_ERR_SHAPE;
  const bool relu = a.act == GL_ACT_RELU;
  const void* kern = relu ? k16_kernel<GL_ACT_RELU>(bwd) : k16_kernel<GL_ACT_IDENTITY>(bwd);
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
  size_t stat = 0;
  const int rs = gl::k16_static_smem(backward != 0, &stat);
  if (rs) return rs;
  const int tt = gl::k16_pick_tt(B, (int)S, backward != 0, optin, stat);
  return tt < 0 ? GL_ERR_SMEM : tt;
}
