// Bank-aware processing order of the neurons of each group (no counterpart in the reference).
//
// The forward and backward kernels gather x from a shared-memory tile xs[d][T] (rows of
// 4T bytes) and the backward scatters into a dX tile of the same shape.  One shared-memory
// wavefront serves 128 bytes = 32/T rows from distinct bank groups (bank group of row d =
// d mod 32/T); the M = 32/T neurons whose rows one wavefront serves are consecutive
// processing positions (the forward's quarter-warp at T = 8 holds 4 neurons, the backward's
// warp step at T = 4 holds 8).  With random indices the M rows of gather k collide: the
// expected wavefront count is 2.12 (M = 4) and 2.60 (M = 8) instead of 1.
//
// A third mode (unit 48) builds units of 8 scored mod 8 whose halves are also scored mod 4, so
// one order serves both kernels (used for parameter storage kept in processing order).
//
// This kernel permutes the processing order within each group so that the M neurons of a
// unit have rows in distinct bank groups for as many of their 8 inputs as possible: a greedy
// pass keeps a pool of up to kOrderPool not-yet-placed neurons (in slot order) and fills each
// unit by picking, one at a time, the pool neuron that raises the unit's per-input maximum
// bank-group multiplicity least (ties: fewest collisions, then the lowest pool position); the
// picked neuron's pool entry takes the next slot.  The result depends only on the indices and
// is deterministic.  Positions >= n_g keep the identity (padding slots).  Storage order of the
// parameters is unchanged: the kernels read order[g][position] to find the slot they process.
#include "common.cuh"

namespace gl {

constexpr int kOrderWarps = 4;
constexpr int kOrderPool = 1024;

// Bank groups (index mod M) of a record's 8 inputs, 4 bits each; M <= 8, so unit counts fit 4 bits.
template <int M>
__device__ __forceinline__ uint32_t order_residues(const int16_t* __restrict__ rec, int dmax) {
  const Rec8 r = load_rec8(rec, dmax);
  uint32_t v = 0;
#pragma unroll
  for (int k = 0; k < 8; ++k) v |= (uint32_t)(r.i[k] & (M - 1)) << (4 * k);
  return v;
}

// Marginal cost of adding a neuron with bank groups r (4 bits per input) to a unit whose per-input
// bin counts are cnt[k] (4 bits per bin) and maxima mx (4 bits per input): 64 per input whose
// maximum would grow, plus the collisions.
template <int M>
__device__ __forceinline__ int order_score(uint32_t r, const uint32_t (&cnt)[8], uint32_t mx) {
  int sc = 0;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int b = (r >> (4 * k)) & (M - 1);
    const int c = (cnt[k] >> (4 * b)) & 15;
    const int m = (mx >> (4 * k)) & 15;
    sc += (c + 1 > m ? 64 : 0) + c;
  }
  return sc;
}

template <int M>
__device__ __forceinline__ void order_add(uint32_t r, uint32_t (&cnt)[8], uint32_t& mx) {
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int b = (r >> (4 * k)) & (M - 1);
    const int c = ((cnt[k] >> (4 * b)) & 15) + 1;
    cnt[k] += 1u << (4 * b);
    if (c > (int)((mx >> (4 * k)) & 15)) mx = (mx & ~(15u << (4 * k))) | ((uint32_t)c << (4 * k));
  }
}

// MODE 4 / 8: units of MODE neurons scored mod MODE.  MODE 48: units of 8 scored mod 8 whose two
// halves are also scored mod 4 (serves the backward's tile of 4 tokens and the forward's of 8).
template <int MODE>
__global__ void __launch_bounds__(kOrderWarps * 32) group_order_kernel(const int16_t* __restrict__ idx,
                                                                       const int32_t* __restrict__ counts, int D,
                                                                       int64_t NB, int64_t g0, int64_t g1,
                                                                       int32_t* __restrict__ order) {
  constexpr int UNIT = MODE == 4 ? 4 : 8;
  constexpr int MB = MODE == 4 ? 4 : 8;  // bins of the unit score
  __shared__ int pool_s[kOrderWarps][kOrderPool];
  __shared__ uint32_t pool_r[kOrderWarps][kOrderPool];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t g = g0 + (int64_t)blockIdx.x * kOrderWarps + warp;
  if (g >= g1) return;  // warp-uniform
  const int slots = (int)(NB * 8);
  const int ng = min(max(__ldg(counts + g), 0), slots);
  const int16_t* gidx = idx + g * (int64_t)slots * 8;
  int32_t* gout = order + (g - g0) * (int64_t)slots;
  int* ps = pool_s[warp];
  uint32_t* pr = pool_r[warp];
  int psize = min(ng, kOrderPool);
  for (int i = lane; i < psize; i += 32) {
    ps[i] = i;
    pr[i] = order_residues<8>(gidx + (int64_t)i * 8, D - 1);
  }
  for (int s = ng + lane; s < slots; s += 32) gout[s] = s;
  __syncwarp();
  int next = psize;
  int pos = 0;
  while (pos < ng) {
    uint32_t cnt[8] = {0, 0, 0, 0, 0, 0, 0, 0}, cq[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    uint32_t mx = 0, mq = 0;
    for (int j = 0; j < UNIT && pos < ng; ++j, ++pos) {
      if (MODE == 48 && j == 4) {
#pragma unroll
        for (int k = 0; k < 8; ++k) cq[k] = 0;
        mq = 0;
      }
      int best = 0x7fffffff, besti = 0x7fffffff;
      for (int i = lane; i < psize; i += 32) {
        const uint32_t r = pr[i];
        int sc = order_score<MB>(r, cnt, mx);
        if (MODE == 48) sc += order_score<4>(r, cq, mq);
        if (sc < best) {
          best = sc;
          besti = i;
        }
      }
#pragma unroll
      for (int off = 16; off; off >>= 1) {
        const int ob = __shfl_xor_sync(kFullMask, best, off);
        const int oi = __shfl_xor_sync(kFullMask, besti, off);
        if (ob < best || (ob == best && oi < besti)) {
          best = ob;
          besti = oi;
        }
      }
      const int pick = ps[besti];
      const uint32_t r = pr[besti];
      order_add<MB>(r, cnt, mx);
      if (MODE == 48) order_add<4>(r, cq, mq);
      __syncwarp();
      if (lane == 0) {
        gout[pos] = pick;
        if (next < ng) {
          ps[besti] = next;
          pr[besti] = order_residues<8>(gidx + (int64_t)next * 8, D - 1);
        } else {
          ps[besti] = ps[psize - 1];
          pr[besti] = pr[psize - 1];
        }
      }
      if (next < ng) ++next; else --psize;
      __syncwarp();
    }
  }
}

}  // namespace gl

using namespace gl;

extern "C" int gl_group_order(const int16_t* idx, const int32_t* counts, int64_t D, int64_t NB, int64_t g0,
                              int64_t g1, int32_t unit, int32_t* out, void* stream) {
  if (D < 1 || D > 32767 || NB < 1 || g0 < 0 || g1 < g0) return GL_ERR_SHAPE;
  if (NB * 8 > 2147483647LL) return GL_ERR_SHAPE;
  if (unit != 4 && unit != 8 && unit != 48) return GL_ERR_UNSUPPORTED;
  if (g1 == g0) return GL_OK;
  if (!idx || !counts || !out) return GL_ERR_NULL;
  if ((uintptr_t)idx & 15) return GL_ERR_ALIGN;
  const int64_t blocks = (g1 - g0 + kOrderWarps - 1) / kOrderWarps;
  if (blocks > 2147483647LL) return GL_ERR_SHAPE;
  cudaStream_t st = (cudaStream_t)stream;
  const dim3 grid((unsigned)blocks);
  if (unit == 4) group_order_kernel<4><<<grid, kOrderWarps * 32, 0, st>>>(idx, counts, (int)D, NB, g0, g1, out);
  else if (unit == 8) group_order_kernel<8><<<grid, kOrderWarps * 32, 0, st>>>(idx, counts, (int)D, NB, g0, g1, out);
  else group_order_kernel<48><<<grid, kOrderWarps * 32, 0, st>>>(idx, counts, (int)D, NB, g0, g1, out);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_cuda_error(e);
  count_launches(1);
  return GL_OK;
}
