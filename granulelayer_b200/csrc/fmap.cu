// Per-group input feature maps for input locality (no counterpart in the reference).
//
// When the neurons of a group read only a small part of the input (the locality benchmark's
// windowed indices: 3 windows of 512 out of 16,384 features per group), the forward and
// backward kernels can stage just those columns of x instead of all D.  This kernel builds,
// for each group, the sorted list of the distinct features its valid (slot, k) records read,
// fmap[g][0 .. nf[g]-1], and the records rewritten as positions in that list,
// lidx[g][s][k] = rank of idx[g][s][k] in fmap[g] (int16, same shape as the indices).  With
// fmap == NULL it only counts nf[g] (the first pass: callers size fmap from max nf).
//
// One block per group: a D-bit presence bitmap in shared memory (atomicOr per record input),
// a block-wide exclusive scan of the words' population counts, then the list and the ranks.
#include "common.cuh"

namespace gl {

constexpr int kFmapThreads = 512;

__global__ void __launch_bounds__(kFmapThreads) group_fmap_kernel(const int16_t* __restrict__ idx,
                                                                  const int32_t* __restrict__ counts, int D,
                                                                  int64_t NB, int64_t g0, int cap,
                                                                  int32_t* __restrict__ nf,
                                                                  int16_t* __restrict__ fmap,
                                                                  int16_t* __restrict__ lidx) {
  extern __shared__ uint32_t sm_u32[];
  const int nwords = (D + 31) >> 5;
  uint32_t* bits = sm_u32;                 // [nwords]
  uint32_t* base = sm_u32 + nwords;        // [nwords] exclusive prefix of popcounts
  __shared__ uint32_t wsum[kFmapThreads / 32];
  const int64_t g = g0 + blockIdx.x;
  const int64_t slots = NB * 8;
  const int64_t ng = min((int64_t)counts[g], slots);
  const int16_t* gi = idx + g * slots * 8;
  for (int w = threadIdx.x; w < nwords; w += kFmapThreads) bits[w] = 0u;
  __syncthreads();
  for (int64_t e = threadIdx.x; e < ng * 8; e += kFmapThreads) {
    const int d = min((int)(uint16_t)__ldg(gi + e), D - 1);
    atomicOr(&bits[d >> 5], 1u << (d & 31));
  }
  __syncthreads();
  // exclusive scan of popcounts over the words: each thread takes a contiguous run of words
  const int per = (nwords + kFmapThreads - 1) / kFmapThreads;
  const int w0 = threadIdx.x * per, w1 = min(w0 + per, nwords);
  uint32_t local = 0;
  for (int w = w0; w < w1; ++w) local += __popc(bits[w]);
  // block scan of `local`
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t incl = local;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const uint32_t v = __shfl_up_sync(kFullMask, incl, off);
    if (lane >= off) incl += v;
  }
  if (lane == 31) wsum[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    uint32_t v = lane < kFmapThreads / 32 ? wsum[lane] : 0u;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const uint32_t u = __shfl_up_sync(kFullMask, v, off);
      if (lane >= off) v += u;
    }
    if (lane < kFmapThreads / 32) wsum[lane] = v;  // inclusive prefix over warps
  }
  __syncthreads();
  uint32_t run = incl - local + (warp ? wsum[warp - 1] : 0u);  // exclusive prefix of this thread's run
  for (int w = w0; w < w1; ++w) {
    base[w] = run;
    run += __popc(bits[w]);
  }
  __syncthreads();
  const int total = (int)wsum[kFmapThreads / 32 - 1];
  if (threadIdx.x == 0) nf[blockIdx.x] = total;
  if (fmap == nullptr) return;
  int16_t* gf = fmap + (int64_t)blockIdx.x * cap;
  for (int w = threadIdx.x; w < nwords; w += kFmapThreads) {
    uint32_t m = bits[w];
    int r = (int)base[w];
    while (m) {
      const int b = __ffs(m) - 1;
      if (r < cap) gf[r] = (int16_t)(w * 32 + b);
      ++r;
      m &= m - 1;
    }
  }
  if (lidx == nullptr) return;
  int16_t* gl_ = lidx + g * slots * 8;
  for (int64_t e = threadIdx.x; e < slots * 8; e += kFmapThreads) {
    int16_t v = 0;
    if (e < ng * 8) {
      const int d = min((int)(uint16_t)__ldg(gi + e), D - 1);
      const uint32_t below = bits[d >> 5] & ((1u << (d & 31)) - 1u);
      v = (int16_t)(base[d >> 5] + __popc(below));
    }
    gl_[e] = v;
  }
}

}  // namespace gl

using namespace gl;

extern "C" int gl_group_feature_map(const int16_t* idx, const int32_t* counts, int64_t D, int64_t NB, int64_t g0,
                                    int64_t g1, int32_t cap, int32_t* nf, int16_t* fmap, int16_t* lidx,
                                    void* stream) {
  if (D < 1 || D > 32767 || NB < 1 || g0 < 0 || g1 < g0 || cap < 0) return GL_ERR_SHAPE;
  if (g1 == g0) return GL_OK;
  if (!idx || !counts || !nf) return GL_ERR_NULL;
  if (lidx && !fmap) return GL_ERR_NULL;
  if (g1 - g0 > 2147483647LL) return GL_ERR_SHAPE;
  const size_t smem = (size_t)((D + 31) / 32) * 2 * sizeof(uint32_t);
  int rc = ensure_dynamic_smem((const void*)group_fmap_kernel, smem);
  if (rc) return rc;
  group_fmap_kernel<<<(unsigned)(g1 - g0), kFmapThreads, smem, (cudaStream_t)stream>>>(
      idx, counts, (int)D, NB, g0, cap, nf, fmap, lidx);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e);
  count_launches(1);
  return GL_OK;
}
