// Backward: recompute z, then dX, dW and db in one pass (Mode A, fan-in 8, fp32).
//
// Replaces the reference's dense recompute backward: coefficients
// (sparse_pooling/kernels/ops.py:242-249, mean: c1 = g_pre / n_g), and the
// Triton bwd_dense_kernel (kernels/triton_fused.py:448-472) with its Mode-A
// tile (triton_fused.py:402-445, dz from _dz_from_z :364-374), which adds every
// (token, neuron, k) contribution to dX with a global FP32 atomic.
//
// B200 structure.  A thread block owns a token tile of T tokens and a chunk of
// whole pooling groups.  Shared memory holds two feature-major tiles:
//   xs [D][T]  the staged inputs (read by the recompute and by dW),
//   dxs[D][T]  a block-private dX accumulator,
// so the B*N*8 dX contributions become shared-memory reductions, and global
// memory sees one flush of the tile per block (D*T coalesced reductions).
// Lanes are (neuron, token) pairs: T consecutive lanes hold one neuron's T
// tokens, so a warp step covers 32/T neurons; each lane recomputes its z,
// forms dz = c1[t, g] * act'(z), scatters dz * w_k into dxs, and keeps
// dz * x_k for dW.  The T lanes of a neuron then fold their 8 dW partials and
// the db partial with a transpose-reduce (each shuffle step halves the values
// a lane holds), and add them to dw/db with one vector reduction per lane.
#include "common.cuh"

namespace gl {

constexpr int kBwdThreads = 512;

template <int T, int ACT>
__global__ void __launch_bounds__(kBwdThreads, 1)
    bwd_kernel(const float* __restrict__ x, const int16_t* __restrict__ idx, const float* __restrict__ w,
               const float* __restrict__ bias, const int32_t* __restrict__ counts, const float* __restrict__ gpre,
               float* __restrict__ dx, float* __restrict__ dw, float* __restrict__ db, int B, int D, int64_t NB,
               int64_t g0, int64_t g1, int64_t ldx, int64_t ldg, int64_t lddx, int pool, int gpc) {
  constexpr int NPW = 32 / T;  // neurons per warp step
  constexpr int NW = kBwdThreads / 32;
  extern __shared__ __align__(16) float smem[];
  float* xs = smem;
  float* dxs = smem + (size_t)D * T;

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int t0 = blockIdx.x * T;
  stage_tile<T, kBwdThreads>(xs, x, t0, B, D, ldx);
  for (int e = threadIdx.x; e < D * T; e += kBwdThreads) dxs[e] = 0.f;
  __syncthreads();

  const int nsub = lane / T, t = lane % T;
  const bool tok_ok = t0 + t < B;
  const int slots = (int)(NB * 8);
  const int64_t gb = g0 + (int64_t)blockIdx.y * gpc;
  const int64_t ge = gb + gpc < g1 ? gb + gpc : g1;

  for (int64_t g = gb; g < ge; ++g) {
    const int ng = min(counts[g], slots);
    const int64_t fbase = g * (int64_t)slots;
    float c1 = tok_ok ? __ldg(gpre + (int64_t)(t0 + t) * ldg + (g - g0)) : 0.f;
    if (pool == GL_POOL_MEAN) c1 = c1 / (float)ng;

    for (int s0 = warp * NPW; s0 < ng; s0 += NW * NPW) {
      const int s = s0 + nsub;
      const unsigned active = __ballot_sync(kFullMask, s < ng);
      if (s < ng) {
        const int64_t f = fbase + s;
        const Rec8 r = load_rec8(idx + f * 8, D - 1);
        const W8 wr = load_w8(w + f * 8);
        float z = __ldg(bias + f);
        float xv[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          xv[k] = xs[r.i[k] * T + t];
          z = fmaf(wr.w[k], xv[k], z);
        }
        const float dz = c1 * dact_f<ACT>(z);
#pragma unroll
        for (int k = 0; k < 8; ++k) atomicAdd(&dxs[r.i[k] * T + t], dz * wr.w[k]);

        // dW partials dz * x_k, folded over the neuron's T token lanes.
        float a[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) a[k] = dz * xv[k];
        int kb = 0;
#pragma unroll
        for (int step = 1, width = 8; step < T; step <<= 1, width >>= 1) {
          const bool hi = (t & step) != 0;
#pragma unroll
          for (int j = 0; j < width / 2; ++j) {
            const float send = hi ? a[j] : a[j + width / 2];
            const float keep = hi ? a[j + width / 2] : a[j];
            a[j] = keep + __shfl_xor_sync(active, send, step);
          }
          if (hi) kb += width / 2;
        }
        float dbs = dz;
#pragma unroll
        for (int step = 1; step < T; step <<= 1) dbs += __shfl_xor_sync(active, dbs, step);
        float* dwp = dw + f * 8 + kb;
        if constexpr (T == 1) {
          red_add4(dwp, a[0], a[1], a[2], a[3]);
          red_add4(dwp + 4, a[4], a[5], a[6], a[7]);
        } else if constexpr (T == 2) {
          red_add4(dwp, a[0], a[1], a[2], a[3]);
        } else if constexpr (T == 4) {
          red_add2(dwp, a[0], a[1]);
        } else {
          red_add(dwp, a[0]);
        }
        if (t == 0) red_add(db + f, dbs);
      }
    }
  }
  __syncthreads();
  // flush the block's dX tile: consecutive threads take consecutive features
  for (int e = threadIdx.x; e < D * T; e += kBwdThreads) {
    const int tt = e / D, d = e - tt * D;
    if (t0 + tt < B) {
      const float v = dxs[d * T + tt];
      if (v != 0.f) red_add(dx + (int64_t)(t0 + tt) * lddx + d, v);
    }
  }
}

template <int T, int ACT>
static int launch_bwd(const GlBwdArgs& a, int gpc, cudaStream_t st) {
  const size_t smem = (size_t)a.D * T * sizeof(float) * 2;
  auto kern = bwd_kernel<T, ACT>;
  int rc = ensure_dynamic_smem((const void*)kern, smem);
  if (rc) return rc;
  const int64_t tiles = (a.B + T - 1) / T;
  const int64_t chunks = (a.g1 - a.g0 + gpc - 1) / gpc;
  if (tiles > 2147483647LL || chunks > 65535) return GL_ERR_SHAPE;
  dim3 grid((unsigned)tiles, (unsigned)chunks);
  kern<<<grid, kBwdThreads, smem, st>>>(a.x, a.idx, a.w, a.b, a.counts, a.gpre, a.dx, a.dw, a.db, (int)a.B,
                                        (int)a.D, a.NB, a.g0, a.g1, a.ldx, a.ldg, a.lddx, a.pool, gpc);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e);
  count_launches(1);
  return GL_OK;
}

template <int T>
static int dispatch_act_bwd(const GlBwdArgs& a, int gpc, cudaStream_t st) {
  switch (a.act) {
    case GL_ACT_IDENTITY: return launch_bwd<T, GL_ACT_IDENTITY>(a, gpc, st);
    case GL_ACT_RELU: return launch_bwd<T, GL_ACT_RELU>(a, gpc, st);
    case GL_ACT_GELU: return launch_bwd<T, GL_ACT_GELU>(a, gpc, st);
    default: return GL_ERR_UNSUPPORTED;
  }
}

static int pick_bwd_tokens(int64_t D, int smem_optin) {
  for (int T = 8; T >= 1; T >>= 1)
    if ((int64_t)D * T * 8 <= smem_optin) return T;
  return GL_ERR_SMEM;
}

}  // namespace gl

using namespace gl;

extern "C" int gl_bwd_auto_tokens(int64_t D) {
  int optin = 0;
  int rc = device_smem_optin(&optin);
  if (rc) return rc;
  return pick_bwd_tokens(D, optin);
}

extern "C" int gl_bwd_f32(const GlBwdArgs* args, void* stream) {
  if (!args) return GL_ERR_NULL;
  const GlBwdArgs& a = *args;
  if (a.B < 0 || a.D < 1 || a.D > 32767 || a.NB < 1 || a.g0 < 0 || a.g1 < a.g0) return GL_ERR_SHAPE;
  if (a.B == 0 || a.g1 == a.g0) return GL_OK;
  if (!a.x || !a.idx || !a.w || !a.b || !a.counts || !a.gpre || !a.dx || !a.dw || !a.db) return GL_ERR_NULL;
  if (a.B > 2147483647LL || a.ldx < a.D || a.ldg < a.g1 - a.g0 || a.lddx < a.D) return GL_ERR_SHAPE;
  if (((uintptr_t)a.idx & 15) || ((uintptr_t)a.w & 15) || ((uintptr_t)a.dw & 31)) return GL_ERR_ALIGN;
  if (a.pool != GL_POOL_MEAN && a.pool != GL_POOL_SUM) return GL_ERR_UNSUPPORTED;
  int optin = 0, sms = 0;
  int rc = device_smem_optin(&optin);
  if (rc) return rc;
  if ((rc = device_sm_count(&sms))) return rc;
  int T = a.tokens;
  if (T == 0) {
    T = pick_bwd_tokens(a.D, optin);
    if (T < 0) return T;
  } else if (T != 1 && T != 2 && T != 4 && T != 8) {
    return GL_ERR_UNSUPPORTED;
  }
  if ((int64_t)a.D * T * 8 > optin) return GL_ERR_SMEM;
  const int64_t G = a.g1 - a.g0;
  int gpc = a.groups_per_cta;
  if (gpc <= 0) {
    const int64_t tiles = (a.B + T - 1) / T;
    const int64_t units = tiles * G;
    int64_t want = units / ((int64_t)sms * 32);
    gpc = (int)(want < 1 ? 1 : (want > 8 ? 8 : want));
  }
  while ((G + gpc - 1) / gpc > 65535) gpc *= 2;
  cudaStream_t st = (cudaStream_t)stream;
  switch (T) {
    case 8: return dispatch_act_bwd<8>(a, gpc, st);
    case 4: return dispatch_act_bwd<4>(a, gpc, st);
    case 2: return dispatch_act_bwd<2>(a, gpc, st);
    default: return dispatch_act_bwd<1>(a, gpc, st);
  }
}
