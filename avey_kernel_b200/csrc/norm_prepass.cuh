// Streaming pre-pass of the tcgen05 path: per-row sums of squares of z_tr
// (fp32), 4 bytes per row, into the caller's workspace. Two rows per warp
// step, 16-byte loads; rows are 16-byte aligned on this path. It lets the fused
// kernel that follows start at once (programmatic dependent launch); that
// kernel waits for these sums only before its P phase.
//
// Reference: the row L2 norm inside F.normalize (avey_kernels/ops.py:68 and
// :108); only the sum of squares is produced here, the division by
// max(sqrt(.), norm_eps) is applied to the Gram tile in the fused kernel.
#pragma once

#include "common.cuh"
#include "ptx.cuh"

namespace avey {

constexpr int kPrepassThreads = 256;

// Sum of squares of the 16-bit pairs in one 16-byte vector.
template <typename T>
__device__ __forceinline__ float sumsq_v4(const uint4 q, float s) {
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
  return s;
}

// Each warp takes two rows per step and issues all of their loads (up to
// four 16-byte vectors per lane and row, 1024 features) before using any, so
// a row costs one memory round trip instead of one per vector.
template <typename T>
__global__ void __launch_bounds__(kPrepassThreads) norm_prepass(const FwdArgs args) {
  griddep_launch_dependents();
  const int warp = (blockIdx.x * kPrepassThreads + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int nwarps = (gridDim.x * kPrepassThreads) >> 5;
  const int rows = args.batch * args.ctx;
  const int nvec = args.feat / 8;  // 16-byte vectors per row (feat % 8 == 0 here)
  const uint64_t keep = l2_policy_evict_last();  // the fused kernel reads z_tr next
  auto row_ptr = [&](int r) {
    const int b = r / args.ctx, n = r - b * args.ctx;
    return reinterpret_cast<const uint4*>(static_cast<const T*>(args.z_tr) +
                                          static_cast<int64_t>(b) * args.zr_bs +
                                          static_cast<int64_t>(n) * args.zr_rs);
  };
  for (int r0 = 2 * warp; r0 < rows; r0 += 2 * nwarps) {
    const bool two = r0 + 1 < rows;
    const uint4* ra = row_ptr(r0);
    const uint4* rb = two ? row_ptr(r0 + 1) : ra;
    float sa = 0.f, sb = 0.f;
    for (int v0 = 0; v0 < nvec; v0 += 128) {
      uint4 qa[4], qb[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int v = v0 + 32 * u + lane;
        qa[u] = v < nvec ? ld_global_nc_v4_hint(ra + v, keep) : make_uint4(0u, 0u, 0u, 0u);
        qb[u] = (two && v < nvec) ? ld_global_nc_v4_hint(rb + v, keep) : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        sa = sumsq_v4<T>(qa[u], sa);
        sb = sumsq_v4<T>(qb[u], sb);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      sa += __shfl_xor_sync(0xffffffffu, sa, o);
      sb += __shfl_xor_sync(0xffffffffu, sb, o);
    }
    if (lane == 0) {
      args.sumsq[r0] = sa;
      if (two) args.sumsq[r0 + 1] = sb;
    }
  }
}

// The pre-summed form (avey_fwd_presummed_v1): the producer of z_tr (the
// enricher's GEMM epilogue) already wrote the row sums of squares as partial
// planes of `rows` floats; they are added in plane order into the workspace
// (4 bytes per plane and row instead of a pass over z_tr). Launched where
// norm_prepass would be, with the same programmatic dependent launch.
__global__ void __launch_bounds__(kPrepassThreads)
    sumsq_planes(const float* __restrict__ planes, int nplanes, int64_t rows, float* __restrict__ out) {
  griddep_launch_dependents();
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * kPrepassThreads + threadIdx.x; r < rows;
       r += static_cast<int64_t>(gridDim.x) * kPrepassThreads) {
    float s = 0.f;
    for (int p = 0; p < nplanes; ++p) s += __ldg(planes + p * rows + r);
    out[r] = s;
  }
}

}  // namespace avey
