// Fused Adam(W) step over fp32 parameters, reading the fp32 gradient and
// zeroing it in the same pass (sparse_pooling/optim.py:26-64, _adamw_kernel,
// with moments="fp32" and fp32 parameters: no master copy, no stochastic
// rounding, optim.py:107, 121).  Purely HBM-bound: 16 bytes read and 16 bytes
// written per element; float4 vectors with a grid-stride loop sized to the
// SM count.
#include "common.cuh"

namespace gl {

struct AdamCoef {
  float lr, b1, b2, eps, decay, bc1, bc2;
};

__device__ __forceinline__ void adam1(float& p, float& g, float& m, float& v, const AdamCoef& c) {
  m = c.b1 * m + (1.f - c.b1) * g;
  v = c.b2 * v + (1.f - c.b2) * g * g;
  const float upd = (m / c.bc1) / (sqrtf(v / c.bc2) + c.eps);
  p = p * c.decay - c.lr * upd;
}

__global__ void __launch_bounds__(256) adam_vec_kernel(float4* __restrict__ p, float4* __restrict__ g,
                                                       float4* __restrict__ m, float4* __restrict__ v, int64_t n4,
                                                       AdamCoef c, int zero) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    float4 pp = p[i], gg = g[i], mm = m[i], vv = v[i];
    adam1(pp.x, gg.x, mm.x, vv.x, c);
    adam1(pp.y, gg.y, mm.y, vv.y, c);
    adam1(pp.z, gg.z, mm.z, vv.z, c);
    adam1(pp.w, gg.w, mm.w, vv.w, c);
    p[i] = pp;
    m[i] = mm;
    v[i] = vv;
    if (zero) g[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

__global__ void __launch_bounds__(256) adam_scalar_kernel(float* __restrict__ p, float* __restrict__ g,
                                                          float* __restrict__ m, float* __restrict__ v, int64_t n,
                                                          AdamCoef c, int zero) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float pp = p[i], gg = g[i], mm = m[i], vv = v[i];
    adam1(pp, gg, mm, vv, c);
    p[i] = pp;
    m[i] = mm;
    v[i] = vv;
    if (zero) g[i] = 0.f;
  }
}

}  // namespace gl

using namespace gl;

extern "C" int gl_adam_f32(const GlAdamArgs* args, void* stream) {
  if (!args) return GL_ERR_NULL;
  const GlAdamArgs& a = *args;
  if (a.n < 0) return GL_ERR_SHAPE;
  if (a.n == 0) return GL_OK;
  if (!a.p || !a.g || !a.m || !a.v) return GL_ERR_NULL;
  int sms = 0;
  int rc = device_sm_count(&sms);
  if (rc) return rc;
  AdamCoef c{a.lr, a.beta1, a.beta2, a.eps, 1.f - a.lr * a.weight_decay, a.bc1, a.bc2};
  cudaStream_t st = (cudaStream_t)stream;
  const bool vec = !(((uintptr_t)a.p | (uintptr_t)a.g | (uintptr_t)a.m | (uintptr_t)a.v) & 15);
  const int64_t n4 = vec ? a.n / 4 : 0;
  const int64_t blocks_cap = (int64_t)sms * 8;
  if (n4 > 0) {
    int64_t blocks = (n4 + 255) / 256;
    if (blocks > blocks_cap) blocks = blocks_cap;
    adam_vec_kernel<<<(unsigned)blocks, 256, 0, st>>>((float4*)a.p, (float4*)a.g, (float4*)a.m, (float4*)a.v, n4,
                                                       c, a.zero_grad);
  }
  const int64_t tail = a.n - n4 * 4;
  if (tail > 0) {
    const int64_t off = n4 * 4;
    int64_t blocks = (tail + 255) / 256;
    if (blocks > blocks_cap) blocks = blocks_cap;
    adam_scalar_kernel<<<(unsigned)blocks, 256, 0, st>>>(a.p + off, a.g + off, a.m + off, a.v + off, tail, c,
                                                         a.zero_grad);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e);
  count_launches((n4 > 0) + (tail > 0));
  return GL_OK;
}
