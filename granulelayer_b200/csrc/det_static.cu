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
// array's name to a kernel (on the host it names a stand-in, not device memory), so every call looks
// up the array's device address with cudaGetSymbolAddress in the CUDA context current on the calling
// thread.  The lookup allocates nothing; it is made on every call rather than cached because the
// address belongs to a context, and a caller may run in a context of its own (a framework that
// creates contexts with the driver API) or after cudaDeviceReset.  The first call in a context can
// load the library's device code into that context, so make it before any stream capture.  Every
// call validates all its arguments first and then clears the B * D entries it uses on the caller's
// stream before the backward runs, because the array keeps the previous call's sums.  All calls on a
// device share the one array: calls whose GPU work overlaps (different streams without ordering
// between them) race on it and give wrong results.
#include "common.cuh"

namespace gl {
namespace {

__device__ __align__(256) static int64_t g_det_dxq_scratch[GL_DET_STATIC_MAX_ELEMS];

// Device address of the scratch array in the current context.
int scratch_address(int64_t** out) {
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_det_dxq_scratch);
  if (e != cudaSuccess || p == nullptr) {
    set_cuda_error(e != cudaSuccess ? e : cudaErrorInvalidSymbol);
    return GL_ERR_DEVICE;
  }
  *out = static_cast<int64_t*>(p);
  return GL_OK;
}

}  // namespace
}  // namespace gl

extern "C" int gl_bwd_shared_det_static_f32(const GlSharedArgs* args, const float* qscale, const float* qinv,
                                            void* stream) {
  if (!args) return GL_ERR_NULL;
  const GlSharedArgs& a = *args;
  int T = 0;
  int rc = gl::det_check_args(a, qscale, qinv, &T);  // nothing touches the shared scratch before this passes
  if (rc || !T) return rc;
  if (a.D > GL_DET_STATIC_MAX_ELEMS / a.B) return GL_ERR_CAPACITY;
  int64_t* dxq = nullptr;
  if ((rc = gl::scratch_address(&dxq))) return rc;
  cudaStream_t st = (cudaStream_t)stream;
  const cudaError_t e = cudaMemsetAsync(dxq, 0, (size_t)(a.B * a.D) * sizeof(int64_t), st);
  if (e != cudaSuccess) return gl::set_cuda_error(e);
  return gl_bwd_shared_det_f32(args, dxq, qscale, qinv, stream);
}
