// ABI identity, status strings and per-device launch state of the library
// (the pattern of the reference's abi.cu:9-62 and launch.cuh:15-82: version
// query, negative status codes, a per-device cache of kernel attributes
// guarded by a mutex).
#include <atomic>
#include <mutex>
#include <unordered_map>
#include <utility>

#include "common.cuh"

namespace gl {

static thread_local int g_last_cuda = 0;
static std::atomic<int64_t> g_launches{0};

void count_launches(int n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

int set_cuda_error(cudaError_t e) {
  g_last_cuda = (int)e;
  return GL_ERR_LAUNCH;
}

namespace {
std::mutex g_mu;
struct PairHash {
  size_t operator()(const std::pair<const void*, int>& k) const {
    return std::hash<const void*>()(k.first) ^ (std::hash<int>()(k.second) * 0x9e3779b97f4a7c15ull);
  }
};
std::unordered_map<std::pair<const void*, int>, size_t, PairHash> g_smem_set;  // (kernel, device) -> bytes
std::unordered_map<int, int> g_optin, g_sms;
}  // namespace

static int current_device(int* dev) {
  cudaError_t e = cudaGetDevice(dev);
  if (e != cudaSuccess) {
    g_last_cuda = (int)e;
    return GL_ERR_DEVICE;
  }
  return GL_OK;
}

int device_smem_optin(int* bytes) {
  int dev;
  int rc = current_device(&dev);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_optin.find(dev);
  if (it == g_optin.end()) {
    int v = 0;
    cudaError_t e = cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e != cudaSuccess) {
      g_last_cuda = (int)e;
      return GL_ERR_DEVICE;
    }
    it = g_optin.emplace(dev, v).first;
  }
  *bytes = it->second;
  return GL_OK;
}

int device_sm_count(int* sms) {
  int dev;
  int rc = current_device(&dev);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_sms.find(dev);
  if (it == g_sms.end()) {
    int v = 0;
    cudaError_t e = cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) {
      g_last_cuda = (int)e;
      return GL_ERR_DEVICE;
    }
    it = g_sms.emplace(dev, v).first;
  }
  *sms = it->second;
  return GL_OK;
}

int ensure_dynamic_smem(const void* func, size_t bytes) {
  int dev;
  int rc = current_device(&dev);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(g_mu);
  auto key = std::make_pair(func, dev);
  auto it = g_smem_set.find(key);
  if (it != g_smem_set.end() && it->second >= bytes) return GL_OK;
  const size_t want = bytes < 49152 ? 49152 : bytes;
  cudaError_t e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)want);
  if (e != cudaSuccess) {
    g_last_cuda = (int)e;
    return GL_ERR_SMEM;
  }
  g_smem_set[key] = want;
  return GL_OK;
}

}  // namespace gl

extern "C" int gl_abi_version(void) { return GL_ABI_VERSION; }

extern "C" int gl_last_cuda_error(void) { return gl::g_last_cuda; }

extern "C" int64_t gl_launch_count(void) { return gl::g_launches.load(std::memory_order_relaxed); }

extern "C" const char* gl_status_string(int status) {
  switch (status) {
    case GL_OK: return "ok";
    case GL_ERR_NULL: return "a required pointer is NULL";
    case GL_ERR_SHAPE: return "inconsistent sizes, strides or group range";
    case GL_ERR_ALIGN: return "a pointer is not aligned for vector access";
    case GL_ERR_UNSUPPORTED: return "unsupported pool, activation or token tile";
    case GL_ERR_SMEM: return "the token tile does not fit in shared memory";
    case GL_ERR_LAUNCH: return "CUDA launch failed";
    case GL_ERR_DEVICE: return "no usable CUDA device";
    case GL_ERR_CAPACITY: return "the problem exceeds the fixed scratch of the allocation-free entry point";
    default: return "unknown status";
  }
}
