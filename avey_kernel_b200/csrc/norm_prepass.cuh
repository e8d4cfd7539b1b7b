// Streaming pre-pass of the tcgen05 path: per-row sums of squares of z_tr
// (fp32), 4 bytes per row, into the caller's workspace. One warp per row,
// 16-byte loads; rows are 16-byte aligned on this path. It lets the fused
// kernel that follows start at once (programmatic dependent launch); that
// kernel waits for these sums only before its P phase.
//
// Reference: the row L2 norm inside F.normalize (avey_kernels/ops.py:73 and
// :113); only the sum of squares is produced here, the division by
// max(sqrt(.), norm_eps) is applied to the Gram tile in the fused kernel.
#pragma once

#include "common.cuh"
#include "ptx.cuh"

namespace avey {

constexpr int kPrepassThreads = 256;

template <typename T>
__global__ void __launch_bounds__(kPrepassThreads) norm_prepass(const FwdArgs args) {
  griddep_launch_dependents();
  const int warp = (blockIdx.x * kPrepassThreads + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int nwarps = (gridDim.x * kPrepassThreads) >> 5;
  const int rows = args.batch * args.ctx;
  const int nvec = args.feat / 8;  // 16-byte vectors per row (feat % 8 == 0 here)
  const uint64_t keep = l2_policy_evict_last();  // the fused kernel reads z_tr next
  for (int r = warp; r < rows; r += nwarps) {
    const int b = r / args.ctx, n = r - b * args.ctx;
    const uint4* row = reinterpret_cast<const uint4*>(static_cast<const T*>(args.z_tr) +
                                                      static_cast<int64_t>(b) * args.zr_bs +
                                                      static_cast<int64_t>(n) * args.zr_rs);
    float s = 0.f;
    for (int v = lane; v < nvec; v += 32) {
      const uint4 q = ld_global_nc_v4_hint(row + v, keep);
      const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const uint16_t lo = static_cast<uint16_t>(w[e] & 0xFFFFu);
        const uint16_t hi = static_cast<uint16_t>(w[e] >> 16);
        const float a = Elem<T>::to_f(*reinterpret_cast<const T*>(&lo));
        const float c = Elem<T>::to_f(*reinterpret_cast<const T*>(&hi));
        s = fmaf(a, a, s);
        s = fmaf(c, c, s);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) args.sumsq[r] = s;
  }
}

}  // namespace avey
