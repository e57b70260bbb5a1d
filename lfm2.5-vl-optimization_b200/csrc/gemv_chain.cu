// Chained decode GEMV: a list of weight-only int8 GEMVs y_l = bf16((x_l . W_l^T) * s_l), one after the other, each
// with the arithmetic of lfm2q_gemv's x-sliced int8 path (gemv.cu) where its token buffer fits (else the bf16 path),
// launched back to back with programmatic dependent launch.
//
// Reference: the decode step runs its GEMVs back to back inside one captured CUDA graph (src/lfm2opt/runtime.py:
// 223-244 `StaticDecoder._linear`, :247-294 `_step_fused`), one launch of gemv (kernels/lfm2_decode.cu:576-714,
// binding kernels/lfm2_decode.cpp:73-85) per linear.
//
// Why plain launches. Every GEMV of a decode step depends on the whole output of the one before, so each step of the
// chain has a fixed critical path: the producer's stores reach L2, the consumer learns of it, reads x and reduces.
// Measured on B200 with the weights already in L2 (16 x 2048 x 2048): 3.0 us per dependent GEMV for graph launches,
// 5.9 us for a persistent cooperative kernel synchronising its blocks through global counters (an earlier version of
// this file): the launch path is the cheaper barrier. The weight stream of the next layer is overlapped by the deep
// kernel itself (its blocks are resident beside the running layer's and fill their rings before the dependency
// wait). Bulk L2 prefetches of the layers ahead (a 48 MB window kept ahead of the running layer, another earlier
// version) made the 65-GEMV stack slower, 534 vs 467 us, as did L2 prefetches of each block's next row group.
#include <cuda_runtime.h>

#include "launch.h"

namespace lfm2q {

cudaError_t launch_gemv_chain(const ChainLayer *L, int n, int B, bool pdl, cudaStream_t st) {
  for (int l = 0; l < n; ++l)
    if (const cudaError_t e = launch_gemv_sliced(L[l].W, L[l].scale, L[l].x, L[l].y, L[l].N, L[l].K, B, pdl, st))
      return e;
  return cudaSuccess;
}

}  // namespace lfm2q
