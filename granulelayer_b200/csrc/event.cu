// Winner-event backward of max and top-K pooling (Mode A and Mode B), fp32.
//
// Replaces the reference's sparse winner-event backward (kernels/triton_fused.py:476-520
// bwd_events_kernel, launched by ops.py:281-293): each event (token t, group g, j < kev) names one
// neuron, a slot s the forward chose (the max's winner, or one of the top-K), and the coefficient
// c of (t, g) (dL/dpre[t, g], divided by min(k, n) for top-K); the neuron's z is recomputed
// (8 FMAs, only act'(z) is needed) and
//   dz = c * act'(z),  db[s] += dz,  dw[s][k] += dz * x[t, idx_k],  dx[t, idx_k] += dz * w[s][k].
// One thread per event; events with s < 0 or c == 0 do nothing.  The B*G*kev events touch that
// many neurons (not B*N): the whole backward is a few global reductions per event.
#include "common.cuh"

namespace gl {

constexpr int kEventThreads = 256;

template <int ACT, int MODE>  // MODE 0: Mode A; 1: Mode B canonical; 2: Mode B fragment-packed
__global__ void __launch_bounds__(kEventThreads) event_bwd_kernel(const GlEventArgs a, int64_t n_events) {
  const int64_t e = (int64_t)blockIdx.x * kEventThreads + threadIdx.x;
  if (e >= n_events) return;
  const int64_t kev = a.kev > 0 ? a.kev : 1;
  const int64_t per_t = (a.g1 - a.g0) * kev;
  const int64_t t = e / per_t, re = e - t * per_t, gl = re / kev, g = a.g0 + gl;
  const int slots = (int)(a.NB * (MODE == 0 ? 8 : a.C));
  const int s = __ldg(a.winners + t * a.ldwin + re);
  const float c = __ldg(a.coef + t * a.ldc + gl);
  if (s < 0 || s >= slots || c == 0.f) return;
  const int D = (int)a.D;
  Rec8 r;
  float wv[8], bb;
  int64_t woff[4], boff;  // offsets of the weight pairs (k = 2 kh, 2 kh + 1) and of the bias
  const bool wbf = a.wdtype == GL_DTYPE_BF16;
  if constexpr (MODE == 0) {
    const int64_t f = g * slots + s;
    r = load_rec8(a.idx + f * 8, D - 1);
    const W8 w8 = load_w8_any(a.w, f, wbf);
#pragma unroll
    for (int k = 0; k < 8; ++k) wv[k] = w8.w[k];
#pragma unroll
    for (int kh = 0; kh < 4; ++kh) woff[kh] = f * 8 + 2 * kh;
    boff = f;
  } else {
    const int C = (int)a.C, j = s / C, cc = s - j * C;
    if constexpr (MODE == 1) {
      r = load_rec8(a.idx + (g * a.NB + j) * 8, D - 1);
      const int64_t f = (g * a.NB + j) * C + cc;
#pragma unroll
      for (int kh = 0; kh < 4; ++kh) woff[kh] = f * 8 + 2 * kh;
      boff = f;
    } else {
      const MbPacked m = mb_packed(C, a.NB);
      const int16_t* base = a.idx + ((g * (a.NB / m.UB) + j / m.UB) * 8) * m.UB + j % m.UB;
#pragma unroll
      for (int k = 0; k < 8; ++k) r.i[k] = min((int)(uint16_t)__ldg(base + k * m.UB), D - 1);
#pragma unroll
      for (int kh = 0; kh < 4; ++kh) woff[kh] = mb_packed_w(m, g, j, cc, kh);
      boff = mb_packed_b(m, g, j, cc & ~1) + (cc & 1);
    }
#pragma unroll
    for (int kh = 0; kh < 4; ++kh) {
      const float2 v = load2_any(a.w, woff[kh], wbf);
      wv[2 * kh] = v.x;
      wv[2 * kh + 1] = v.y;
    }
  }
  bb = load_any(a.b, boff, wbf);
  float xv[8];
  float z = bb;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    xv[k] = __ldg(a.x + t * a.ldx + r.i[k]);
    z = fmaf(wv[k], xv[k], z);
  }
  const float dz = c * dact_f<ACT>(z);
  if (dz == 0.f) return;
  red_add(a.db + boff, dz);
#pragma unroll
  for (int kh = 0; kh < 4; ++kh) red_add2(a.dw + woff[kh], dz * xv[2 * kh], dz * xv[2 * kh + 1]);
#pragma unroll
  for (int k = 0; k < 8; ++k) red_add(a.dx + t * a.lddx + r.i[k], dz * wv[k]);
}

template <int ACT>
static int event_launch(const GlEventArgs& a, int mode, int64_t n, cudaStream_t st) {
  const int64_t blocks = (n + kEventThreads - 1) / kEventThreads;
  if (blocks > 2147483647LL) return GL_ERR_SHAPE;
  if (mode == 0) event_bwd_kernel<ACT, 0><<<(unsigned)blocks, kEventThreads, 0, st>>>(a, n);
  else if (mode == 1) event_bwd_kernel<ACT, 1><<<(unsigned)blocks, kEventThreads, 0, st>>>(a, n);
  else event_bwd_kernel<ACT, 2><<<(unsigned)blocks, kEventThreads, 0, st>>>(a, n);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e);
  count_launches(1);
  return GL_OK;
}

}  // namespace gl

using namespace gl;

extern "C" int gl_bwd_events_f32(const GlEventArgs* args, void* stream) {
  if (!args) return GL_ERR_NULL;
  const GlEventArgs& a = *args;
  if (a.B < 0 || a.D < 1 || a.D > 32767 || a.NB < 1 || a.g0 < 0 || a.g1 < a.g0) return GL_ERR_SHAPE;
  if (a.shared && a.C != 8 && a.C != 16 && a.C != 32 && a.C != 64) return GL_ERR_SHAPE;
  if (a.shared && a.packed && ((a.NB * (a.C / 8)) % 4 || ((a.C / 8) < 4 && a.NB % (4 / (a.C / 8)))))
    return GL_ERR_SHAPE;
  if (a.B == 0 || a.g1 == a.g0) return GL_OK;
  if (!a.x || !a.idx || !a.w || !a.b || !a.winners || !a.coef || !a.dx || !a.dw || !a.db) return GL_ERR_NULL;
  const int64_t kev = a.kev > 0 ? a.kev : 1;
  if (kev > 64) return GL_ERR_SHAPE;
  if (a.wdtype != GL_DTYPE_F32 && a.wdtype != GL_DTYPE_BF16) return GL_ERR_UNSUPPORTED;
  if (a.ldx < a.D || a.lddx < a.D || a.ldwin < (a.g1 - a.g0) * kev || a.ldc < a.g1 - a.g0) return GL_ERR_SHAPE;
  if (((uintptr_t)a.idx & 15) || ((uintptr_t)a.w & 15) || ((uintptr_t)a.dw & 7)) return GL_ERR_ALIGN;
  const int mode = a.shared ? (a.packed ? 2 : 1) : 0;
  const int64_t n = a.B * (a.g1 - a.g0) * kev;
  cudaStream_t st = (cudaStream_t)stream;
  switch (a.act) {
    case GL_ACT_IDENTITY: return event_launch<GL_ACT_IDENTITY>(a, mode, n, st);
    case GL_ACT_RELU: return event_launch<GL_ACT_RELU>(a, mode, n, st);
    case GL_ACT_GELU: return event_launch<GL_ACT_GELU>(a, mode, n, st);
    default: return GL_ERR_UNSUPPORTED;
  }
}
