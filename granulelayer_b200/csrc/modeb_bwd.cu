// Mode B backward: the mean / sum instantiations and the launch entry (the kernel is in
// modeb_bwd.cuh; the smooth pools' instantiations are in modeb_bwd_smooth.cu, compiled in parallel).
#include "modeb_bwd.cuh"

namespace gl {

int mb_bwd_launch(const MbParams& p, int T, int act, bool packed, cudaStream_t st) {
  if (p.pool >= GL_POOL_LME) return mb_bwd_launch_smooth(p, T, act, packed, st);
  return mb_bwd_dispatch<false>(p, T, act, packed, st);
}

}  // namespace gl
