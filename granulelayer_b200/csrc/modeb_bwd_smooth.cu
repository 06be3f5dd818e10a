// Mode B backward: the LogMeanExp / power-mean / softmax-weighted instantiations (dz from the
// reference's coefficients through pool_dz; the kernel is in modeb_bwd.cuh).
#include "modeb_bwd.cuh"

namespace gl {

int mb_bwd_launch_smooth(const MbParams& p, int T, int act, bool packed, cudaStream_t st) {
  return mb_bwd_dispatch<true>(p, T, act, packed, st);
}

}  // namespace gl
