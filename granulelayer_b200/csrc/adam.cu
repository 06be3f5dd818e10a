// Fused Adam(W) step, reading the fp32 gradient and zeroing it in the same pass
// (sparse_pooling/optim.py:26-64, _adamw_kernel).  fp32 arithmetic; parameters fp32 or bf16 (with an
// optional fp32 master copy, or stochastic rounding to bf16, optim.py:49-62); moments fp32 or bf16
// (stored round-to-nearest-even, optim.py:47-48).  Purely HBM-bound: the all-fp32 path moves
// 16 bytes in and 16 out per element with float4 vectors; every path uses a grid-stride loop sized
// to the SM count.
#include <cuda_bf16.h>

#include "common.cuh"

namespace gl {

struct AdamCoef {
  float lr, b1, b2, eps, decay, bc1, bc2;
};

__device__ __forceinline__ void adam1(float& p, float g, float& m, float& v, const AdamCoef& c) {
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

// A 32-bit hash of (seed, i) for stochastic rounding: a counter-based generator, so the noise of
// an element does not depend on the launch shape.  (Murmur3's 64-bit finaliser on the pair.)
__device__ __forceinline__ unsigned sr_hash(unsigned seed, uint64_t i) {
  uint64_t h = i * 0x9E3779B97F4A7C15ull ^ ((uint64_t)seed << 32 | seed);
  h ^= h >> 33;
  h *= 0xFF51AFD7ED558CCDull;
  h ^= h >> 33;
  h *= 0xC4CEB9FE1A85EC53ull;
  h ^= h >> 33;
  return (unsigned)h;
}

__device__ __forceinline__ float ld_any(const void* a, int64_t i, bool bf) {
  return bf ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(a)[i]) : reinterpret_cast<const float*>(a)[i];
}

__device__ __forceinline__ void st_any(void* a, int64_t i, float x, bool bf) {
  if (bf) reinterpret_cast<__nv_bfloat16*>(a)[i] = __float2bfloat16_rn(x);
  else reinterpret_cast<float*>(a)[i] = x;
}

// Any mix of storage types, one element per thread and step.
__global__ void __launch_bounds__(256) adam_any_kernel(void* __restrict__ p, float* __restrict__ g,
                                                       void* __restrict__ m, void* __restrict__ v,
                                                       float* __restrict__ master, int64_t n, AdamCoef c, int zero,
                                                       bool pbf, bool mbf, bool stochastic, unsigned seed) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const float gg = g[i];
    float mm = ld_any(m, i, mbf), vv = ld_any(v, i, mbf);
    float pp = master != nullptr ? master[i] : ld_any(p, i, pbf);
    adam1(pp, gg, mm, vv, c);
    st_any(m, i, mm, mbf);
    st_any(v, i, vv, mbf);
    if (zero) g[i] = 0.f;
    if (master != nullptr) master[i] = pp;
    if (pbf && master == nullptr && stochastic) {
      // noise below the bf16 ulp added to the fp32 bits, then truncation (optim.py:55-62)
      const unsigned bits = (__float_as_uint(pp) + (sr_hash(seed, (uint64_t)i) & 0xFFFFu)) & 0xFFFF0000u;
      reinterpret_cast<unsigned short*>(p)[i] = (unsigned short)(bits >> 16);
    } else {
      st_any(p, i, pp, pbf);
    }
  }
}

}  // namespace gl

using namespace gl;

extern "C" int gl_adam_f32(const GlAdamArgs* args, void* stream) {
  if (!args) return GL_ERR_NULL;
  const GlAdamArgs& a = *args;
  if (a.n < 0) return GL_ERR_SHAPE;
  if ((a.pdtype != GL_DTYPE_F32 && a.pdtype != GL_DTYPE_BF16) || (a.mdtype != GL_DTYPE_F32 && a.mdtype != GL_DTYPE_BF16))
    return GL_ERR_UNSUPPORTED;
  if (a.master && a.pdtype != GL_DTYPE_BF16) return GL_ERR_UNSUPPORTED;
  if (a.n == 0) return GL_OK;
  if (!a.p || !a.g || !a.m || !a.v) return GL_ERR_NULL;
  int sms = 0;
  int rc = device_sm_count(&sms);
  if (rc) return rc;
  AdamCoef c{a.lr, a.beta1, a.beta2, a.eps, 1.f - a.lr * a.weight_decay, a.bc1, a.bc2};
  cudaStream_t st = (cudaStream_t)stream;
  const int64_t blocks_cap = (int64_t)sms * 8;
  const bool all_f32 = a.pdtype == GL_DTYPE_F32 && a.mdtype == GL_DTYPE_F32;
  const bool vec = all_f32 && !(((uintptr_t)a.p | (uintptr_t)a.g | (uintptr_t)a.m | (uintptr_t)a.v) & 15);
  const int64_t n4 = vec ? a.n / 4 : 0;
  int launches = 0;
  if (n4 > 0) {
    int64_t blocks = (n4 + 255) / 256;
    if (blocks > blocks_cap) blocks = blocks_cap;
    adam_vec_kernel<<<(unsigned)blocks, 256, 0, st>>>((float4*)a.p, (float4*)a.g, (float4*)a.m, (float4*)a.v, n4,
                                                       c, a.zero_grad);
    ++launches;
  }
  const int64_t off = n4 * 4, tail = a.n - off;
  if (tail > 0) {
    const size_t pe = a.pdtype == GL_DTYPE_BF16 ? 2 : 4, me = a.mdtype == GL_DTYPE_BF16 ? 2 : 4;
    int64_t blocks = (tail + 255) / 256;
    if (blocks > blocks_cap) blocks = blocks_cap;
    adam_any_kernel<<<(unsigned)blocks, 256, 0, st>>>(
        (char*)a.p + off * pe, a.g + off, (char*)a.m + off * me, (char*)a.v + off * me,
        a.master ? a.master + off : nullptr, tail, c, a.zero_grad, a.pdtype == GL_DTYPE_BF16,
        a.mdtype == GL_DTYPE_BF16, a.stochastic != 0, a.seed);
    ++launches;
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e);
  count_launches(launches);
  return GL_OK;
}
