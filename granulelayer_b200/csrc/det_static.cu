// Allocation-free variant of the deterministic Mode-B backward (gl_bwd_shared_det_static_f32).
//
// gl_bwd_shared_det_f32 needs an int64 [B, D] scratch buffer (the exact fixed-point dX sums) that the
// caller allocates and zeroes.  Some callers cannot allocate device memory at the point where they run
// the backward: a plugin whose host framework owns every byte of device memory through its own pool
// and forbids side allocations, or a latency-bound loop where cudaMalloc / cudaFree, which may
// synchronise the device, are not acceptable.  This entry point keeps that scratch in a file-scope
// device array of fixed size instead, so the caller passes only the inputs (x, parameters, dL/dpre,
// the per-token scales) and the outputs (dx, dw, db).
//
// The array (GL_DET_STATIC_MAX_ELEMS int64 entries, 8 MiB) is part of the library's device image:
// every GPU that loads the library holds it until the process exits.  Host code may not pass the
// array's name to a kernel (on the host it names a stand-in, not device memory), so the first call
// on each device looks up its device address with cudaGetSymbolAddress while that device is current
// and caches it; that first call should come before any stream capture.  Every call clears the
// B * D entries it uses on the caller's stream before the backward runs, because the array keeps the
// previous call's sums.  All calls on a device share the one array: calls whose GPU work overlaps
// (different streams without ordering between them) race on it and give wrong results.
#include <mutex>

#include "common.cuh"

namespace gl {
namespace {

__device__ __align__(256) static int64_t g_det_dxq_scratch[GL_DET_STATIC_MAX_ELEMS];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
int64_t* g_scratch_ptr[kMaxDevices] = {};

// Device address of the scratch array on the current device, looked up once per device.
int scratch_address(int64_t** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return GL_ERR_DEVICE;
  }
  if (dev < 0 || dev >= kMaxDevices) return GL_ERR_DEVICE;
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_det_dxq_scratch);
    if (e != cudaSuccess || p == nullptr) {
      set_cuda_error(e != cudaSuccess ? e : cudaErrorInvalidSymbol);
      return GL_ERR_DEVICE;
    }
    g_scratch_ptr[dev] = static_cast<int64_t*>(p);
  }
  *out = g_scratch_ptr[dev];
  return GL_OK;
}

}  // namespace
}  // namespace gl

extern "C" int gl_bwd_shared_det_static_f32(const GlSharedArgs* args, const float* qscale, const float* qinv,
                                            void* stream) {
  if (!args) return GL_ERR_NULL;
  const GlSharedArgs& a = *args;
  if (a.B < 0 || a.D < 1) return GL_ERR_SHAPE;
  if (a.B > 0 && a.D > GL_DET_STATIC_MAX_ELEMS / a.B) return GL_ERR_CAPACITY;
  if (a.B == 0 || a.g1 <= a.g0) return gl_bwd_shared_det_f32(args, nullptr, qscale, qinv, stream);
  int64_t* dxq = nullptr;
  int rc = gl::scratch_address(&dxq);
  if (rc) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  cudaError_t e = cudaMemsetAsync(dxq, 0, (size_t)(a.B * a.D) * sizeof(int64_t), st);
  if (e != cudaSuccess) return gl::set_cuda_error(e);
  return gl_bwd_shared_det_f32(args, dxq, qscale, qinv, stream);
}
