// Chained decode GEMV: a list of weight-only int8 GEMVs y_l = bf16((x_l . W_l^T) * s_l), one after the other, each
// with the arithmetic of lfm2q_gemv's x-sliced int8 path (gemv.cu) where its token buffer fits (else the bf16 path),
// launched back to back with programmatic dependent launch, and with the weights of the layers ahead streamed into L2
// while the earlier layers run.
//
// Reference: the decode step runs its GEMVs back to back inside one captured CUDA graph (src/lfm2opt/runtime.py:
// 223-244 `StaticDecoder._linear`, :247-294 `_step_fused`), one launch of gemv (kernels/lfm2_decode.cu:576-714,
// binding kernels/lfm2_decode.cpp:73-85) per linear.
//
// Why launches and an L2 window. Every GEMV of a decode step depends on the whole output of the one before, so each
// step of the chain has a fixed critical path: the producer's stores reach L2, the consumer learns of it, reads x and
// reduces. Measured on B200 with the weights already in L2 (16 x 2048 x 2048): 3.0 us per dependent GEMV for graph
// launches, 5.9 us for a persistent cooperative kernel synchronising its blocks through global counters (an earlier
// version of this file) - the launch path is the cheaper barrier. What the launches lose is the HBM stream: a 4 MB
// GEMV needs 0.65 us of HBM time but its weights only start to move when it starts. So launch l issues, before its
// dependency wait, bulk L2 prefetches of the next stretch of the list's weights: the frontier of requested bytes is
// kept CH_L2_WINDOW bytes past the end of layer l (126 MB of L2), every block requesting its share of each range.
// By the time a layer runs, its weights are mostly in L2 and HBM has been busy meanwhile.
#include <cuda_runtime.h>

#include <algorithm>
#include <vector>

#include "launch.h"

namespace lfm2q {
namespace {
constexpr long long CH_L2_WINDOW = 48ll << 20;  // bytes of weights requested ahead of the running layer
}  // namespace

cudaError_t launch_gemv_chain(const ChainLayer *L, int n, int B, bool pdl, cudaStream_t st) {
  // weight bytes of the list laid end to end: layer q occupies [start[q], start[q + 1])
  std::vector<long long> start(n + 1, 0);
  for (int l = 0; l < n; ++l) start[l + 1] = start[l] + (long long)L[l].N * L[l].K;
  long long frontier = 0;  // bytes requested into L2 so far
  int q = 0;
  for (int l = 0; l < n; ++l) {
    // the layers after this one, up to the window (the running layer streams its own weights through its rings)
    L2Prefetch pf = {};
    frontier = std::max(frontier, start[l + 1]);
    const long long target = std::min(start[n], start[l + 1] + CH_L2_WINDOW);
    while (frontier < target && pf.cnt < 8) {
      while (start[q + 1] <= frontier) ++q;
      const long long end = std::min(target, start[q + 1]);
      pf.p[pf.cnt] = L[q].W + (frontier - start[q]);  // offsets are multiples of 64 bytes: K % 64 == 0
      pf.n[pf.cnt] = (unsigned long long)(end - frontier);
      ++pf.cnt;
      frontier = end;
    }
    if (const cudaError_t e = launch_gemv_pf(L[l].W, L[l].scale, L[l].x, L[l].y, L[l].N, L[l].K, B, pf, pdl, st)) return e;
  }
  return cudaSuccess;
}

}  // namespace lfm2q
