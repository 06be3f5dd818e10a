// ABI identity, status strings and per-device launch state of the library
// (the pattern of the reference's abi.cu:9-62 and launch.cuh:15-82: version
// query, negative status codes, a per-device cache of kernel attributes
// guarded by a mutex).
#include <atomic>
#include <cstddef>
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

// ---- argument-struct layouts (gl_struct_layout / gl_struct_fields) ----
// One list of fields per struct, in declaration order; the offsets and the names are both generated
// from it, so a binding that compares both against its own declarations catches a missing, added,
// reordered or resized field.
#define GL_FWD_FIELDS(F)                                                                                         \
  F(x) F(idx) F(w) F(b) F(counts) F(pre) F(B) F(D) F(NB) F(g0) F(g1) F(ldx) F(ldp) F(pool) F(act) F(tokens)       \
  F(groups_per_cta) F(wabsmax) F(order) F(lidx) F(fmap) F(nfeat) F(fcap) F(winners) F(ldwin) F(stat) F(ldstat)   \
  F(param) F(k) F(wdtype) F(reserved3)
#define GL_BWD_FIELDS(F)                                                                                         \
  F(x) F(idx) F(w) F(b) F(counts) F(gpre) F(dx) F(dw) F(db) F(B) F(D) F(NB) F(g0) F(g1) F(ldx) F(ldg) F(lddx)     \
  F(pool) F(act) F(tokens) F(groups_per_cta) F(wabsmax) F(rowmax) F(order) F(lidx) F(fmap) F(nfeat) F(fcap)      \
  F(c2) F(c3) F(param) F(wdtype)
#define GL_ADAM_FIELDS(F)                                                                                        \
  F(p) F(g) F(m) F(v) F(n) F(lr) F(beta1) F(beta2) F(eps) F(weight_decay) F(bc1) F(bc2) F(zero_grad) F(master)   \
  F(pdtype) F(mdtype) F(stochastic) F(seed)
#define GL_SHARED_FIELDS(F)                                                                                      \
  F(x) F(idx) F(w) F(b) F(counts) F(pre) F(gpre) F(dx) F(dw) F(db) F(B) F(D) F(NB) F(C) F(g0) F(g1) F(ldx) F(ldp) \
  F(ldg) F(lddx) F(pool) F(act) F(packed) F(tokens) F(groups_per_cta) F(wdtype) F(winners) F(ldwin) F(stat)      \
  F(ldstat) F(c2) F(c3) F(param) F(k)
#define GL_SET_FIELDS(F) F(feat) F(buckets) F(chunks) F(rowmax) F(wabsmax) F(S) F(nchunks) F(max_chunk)
#define GL_EVENT_FIELDS(F)                                                                                       \
  F(x) F(idx) F(w) F(b) F(winners) F(coef) F(dx) F(dw) F(db) F(B) F(D) F(NB) F(C) F(g0) F(g1) F(ldx) F(ldwin)    \
  F(ldc) F(lddx) F(shared) F(packed) F(act) F(kev) F(wdtype) F(reserved)
#define GL_K16_FIELDS(F)                                                                                         \
  F(x) F(env) F(feat) F(buckets) F(q_off) F(rec_off) F(w) F(b) F(counts) F(pre) F(c1t) F(dx) F(dw) F(db) F(B)    \
  F(D) F(G) F(NB16) F(Q) F(S) F(nbuckets) F(ldx) F(ldp) F(ldc) F(lddx) F(act) F(tokens)

#define GL_NAME(f) #f ","

namespace {

template <typename S>
int write_layout(const int64_t* off, int nf, int64_t* out, int n) {
  if (!out || n < nf + 1) return GL_ERR_SHAPE;
  out[0] = (int64_t)sizeof(S);
  for (int i = 0; i < nf; ++i) out[i + 1] = off[i];
  return nf + 1;
}

#define GL_LAYOUT_CASE(ID, S, LIST)                                                  \
  case ID: {                                                                         \
    const int64_t off[] = {LIST(GL_OFF_##S)};                                        \
    return write_layout<S>(off, (int)(sizeof(off) / sizeof(off[0])), out, n);        \
  }
#define GL_OFF_GlFwdArgs(f) (int64_t) offsetof(GlFwdArgs, f),
#define GL_OFF_GlBwdArgs(f) (int64_t) offsetof(GlBwdArgs, f),
#define GL_OFF_GlAdamArgs(f) (int64_t) offsetof(GlAdamArgs, f),
#define GL_OFF_GlSharedArgs(f) (int64_t) offsetof(GlSharedArgs, f),
#define GL_OFF_GlSetArgs(f) (int64_t) offsetof(GlSetArgs, f),
#define GL_OFF_GlEventArgs(f) (int64_t) offsetof(GlEventArgs, f),
#define GL_OFF_GlK16Args(f) (int64_t) offsetof(GlK16Args, f),

}  // namespace

extern "C" int gl_struct_layout(int which, int64_t* out, int n) {
  switch (which) {
    GL_LAYOUT_CASE(0, GlFwdArgs, GL_FWD_FIELDS)
    GL_LAYOUT_CASE(1, GlBwdArgs, GL_BWD_FIELDS)
    GL_LAYOUT_CASE(2, GlAdamArgs, GL_ADAM_FIELDS)
    GL_LAYOUT_CASE(3, GlSharedArgs, GL_SHARED_FIELDS)
    GL_LAYOUT_CASE(4, GlSetArgs, GL_SET_FIELDS)
    GL_LAYOUT_CASE(5, GlEventArgs, GL_EVENT_FIELDS)
    GL_LAYOUT_CASE(6, GlK16Args, GL_K16_FIELDS)
    default: return GL_ERR_UNSUPPORTED;
  }
}

extern "C" const char* gl_struct_fields(int which) {
  switch (which) {
    case 0: return GL_FWD_FIELDS(GL_NAME);
    case 1: return GL_BWD_FIELDS(GL_NAME);
    case 2: return GL_ADAM_FIELDS(GL_NAME);
    case 3: return GL_SHARED_FIELDS(GL_NAME);
    case 4: return GL_SET_FIELDS(GL_NAME);
    case 5: return GL_EVENT_FIELDS(GL_NAME);
    case 6: return GL_K16_FIELDS(GL_NAME);
    default: return nullptr;
  }
}
