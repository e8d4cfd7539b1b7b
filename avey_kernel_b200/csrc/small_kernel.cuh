// Row-tile CUDA-core kernel for small fp32 problems (contexts up to 512 and a
// few hundred query tiles in all): the latency path. On such inputs the 3xTF32
// kernel pair runs a handful of CTAs through a long serial pipeline; this
// kernel gives each query tile of 8 rows to a (2, 1, 1) cluster whose two CTAs
// take one half of the tile's keys each, so config 1 (B = 2, 256 tokens)
// spreads over 128 SMs, and every key row is read from global memory once
// per CTA that needs it:
//
//   key blocks of kb rows (128, or 64 for rows of more than 512 bytes) are
//   copied to shared memory with cp.async, two blocks in flight; per block
//   phase 1  S = Z_q Z_k^T for the 8 query rows: 512 / kb threads per key,
//            each over its slice of the features (the key's sum of squares
//            comes from the same loads); the slices are summed in a fixed
//            order, then P = S * rinv_q * rinv_k * V under the masks goes to
//            shared memory, key-major, with the Avey-B row sums;
//   phase 2  O += P Z from the same shared block: a warp owns 4 features per
//            lane (128 per warp) for its share of the block's keys;
//   combine  each CTA sums its warps' partial O in a fixed order; after a
//            cluster barrier the even CTA finishes rows 0-3 and the odd one
//            rows 4-7, adding the peer's partial O and row sums read through
//            distributed shared memory, then the divide, bias, activation,
//            gate and row mask.
// The products run as packed fp32 pairs (fma.rn.f32x2, one instruction for
// two fused multiply-adds): phase 1 keeps the even and odd features' sums of
// each row apart and adds them at the end, phase 2 pairs neighbouring output
// features. Arithmetic is fp32 like the reference's (ops.py:63); rows that are
// padding are zero-filled as they are copied (ops.py:64-67), so NaN padding
// reaches no product.
#pragma once

#include "common.cuh"
#include "ptx.cuh"

namespace avey {

constexpr int kSmRows = 8;  // query rows per cluster
constexpr int kSmThreads = 512;
constexpr int kSmWarps = kSmThreads / 32;
constexpr int kSmMaxCtx = 512;
constexpr int kSmMaxRowBytes = 1024;                        // features x 4 bytes
constexpr int kSmRedBytes = kSmWarps * kSmRows * 128 * 4;  // phase-2 partial sums
constexpr int kSmMaxOut = kSmRows / 2 * kSmMaxRowBytes / 4 / kSmThreads;  // outputs per thread
constexpr int kSmRptMax = kSmRows * 128 / kSmThreads;  // P rows per thread (128-key blocks)
static_assert(kSmRptMax >= 1 && kSmMaxOut >= 1, "512 threads: 4 or 8 threads per key");

// Shared-memory layout of one CTA (byte offsets), chosen by the host from the
// feature count.
struct SmallGeom {
  int kb;      // keys per block: 128, or 64 for rows above 512 bytes
  int stride;  // bytes per staged row: row bytes + 16 (spreads rows over the banks)
  int zbuf;    // offset of the second key block
  int qbuf;    // the 8 query rows
  int part;    // phase-1 partial sums [threads / kb][9][kb]
  int pbuf;    // P [kb][8][2] (each value twice: the pair operand of phase 2)
  int osum;    // this CTA's partial O [8][features]
  int misc;    // rq, den, dpart, row flags, key mask
  int smem;    // total
};

inline SmallGeom small_geom(int feat) {
  SmallGeom g{};
  const int row = feat * 4;
  g.kb = row <= 512 ? 128 : 64;
  g.stride = row + 16;
  g.zbuf = g.kb * g.stride;
  int z_end = 2 * g.zbuf;
  if (z_end < kSmRedBytes) z_end = kSmRedBytes;  // the partial sums reuse the key blocks
  g.qbuf = z_end;
  g.part = g.qbuf + kSmRows * g.stride;
  g.pbuf = g.part + 9 * kSmThreads * 4;
  g.osum = g.pbuf + g.kb * kSmRows * 8;
  g.misc = g.osum + kSmRows * row;
  g.smem = g.misc + (kSmRows * 2 + kSmWarps * kSmRows + kSmRows) * 4 + kSmMaxCtx + 16;
  return g;
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_0() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// d = a * b + c on two packed fp32 lanes (the low word is lane 0), each lane
// rounded as fmaf rounds it.
__device__ __forceinline__ uint64_t fma_f32x2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ float2 unpack_f32x2(uint64_t v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}
__device__ __forceinline__ float ld_cluster_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

// 16 warps per CTA (4 per scheduler) hide the latency of each phase; the
// launch bound keeps the registers at 128 per thread.
__global__ void __launch_bounds__(kSmThreads, 1)
    small_contextualize(const FwdArgs args, const SmallGeom g) {
  extern __shared__ __align__(16) char sm_raw[];
  char* zb = sm_raw;                                        // [2][kb][stride]
  char* qb = sm_raw + g.qbuf;                               // [8][stride]
  float* part = reinterpret_cast<float*>(sm_raw + g.part);  // [kpt][9][kb]
  float* pbuf = reinterpret_cast<float*>(sm_raw + g.pbuf);  // [kb][8][2]
  float* osum = reinterpret_cast<float*>(sm_raw + g.osum);  // [8][D]
  float* rq = reinterpret_cast<float*>(sm_raw + g.misc);    // [8] inverse query norms
  float* den = rq + kSmRows;                                // [8] this CTA's Avey-B row sums
  float* dpart = den + kSmRows;                             // [kb / 32][8]
  int* row_ok_s = reinterpret_cast<int*>(dpart + kSmWarps * kSmRows);  // [8]
  uint8_t* kv_s = reinterpret_cast<uint8_t*>(row_ok_s + kSmRows);      // [512]
  __shared__ int last_valid_s;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t rank = cluster_rank();
  const int b = blockIdx.y;
  const int C = args.ctx, D = args.feat;
  const int nqt = (C + kSmRows - 1) / kSmRows;
  const int item = static_cast<int>(blockIdx.x) >> 1;
  const int qt = args.causal ? nqt - 1 - item : item;
  const int q0 = qt * kSmRows;
  const int kb = g.kb, kpt = kSmThreads / kb, stride = g.stride;
  const int row_bytes = D * 4;
  const int nseg = row_bytes / 16;
  const float* zr = static_cast<const float*>(args.z_tr) + static_cast<int64_t>(b) * args.zr_bs;

  // Valid positions: all of them without a padding mask (no barrier before
  // the first copies); with one, the row's mask is cached in shared memory
  // (C <= 512 here) with its last valid position.
  const bool masked = args.has_valid != 0;
  int kv_end = C;
  if (masked) {
    if (tid == 0) last_valid_s = -1;
    __syncthreads();
    int last = -1;
    for (int j = tid; j < C; j += kSmThreads) {
      const uint8_t ok = mask_ok(args, b, j) ? 1 : 0;
      kv_s[j] = ok;
      if (ok) last = j;
    }
    if (last >= 0) atomicMax(&last_valid_s, last);
    __syncthreads();
    kv_end = last_valid_s + 1;
  }
  auto kv = [&](int j) { return !masked || kv_s[j] != 0; };
  const int key_end = args.causal ? min(kv_end, q0 + kSmRows) : kv_end;
  // This CTA's keys: the even CTA the first half (rounded up to 32 keys).
  const int half = min(key_end, (((key_end + 1) >> 1) + 31) & ~31);
  const int kbeg = rank ? half : 0, kend = rank ? key_end : half;
  const int nblk = (kend - kbeg + kb - 1) / kb;
  if (tid < kSmRows) {
    const int i = q0 + tid;
    row_ok_s[tid] = (i < C && kv(i)) ? 1 : 0;
    den[tid] = 0.f;
  }

  // Copies rows [r0, r0 + n) of z_tr into `dst` (rows of `stride` bytes), a
  // warp per row and a lane per 16 bytes; rows that are padding or at or past
  // `end` are zero-filled without a read.
  auto copy_rows = [&](char* dst, int r0, int n, int end) {
    const uint32_t base = smem_u32(dst);
    for (int r = warp; r < n; r += kSmWarps) {
      const int j = r0 + r;
      const bool ok = j < end && kv(j);
      const char* src = reinterpret_cast<const char*>(zr + static_cast<int64_t>(ok ? j : 0) * args.zr_rs);
      for (int s = lane; s < nseg; s += 32)
        cp_async16(base + r * stride + 16 * s, src + 16 * s, ok ? 16u : 0u);
    }
  };
  copy_rows(qb, q0, kSmRows, C);
  if (nblk > 0) copy_rows(zb, kbeg, kb, kend);
  cp_async_commit();
  if (nblk > 1) copy_rows(zb + g.zbuf, kbeg + kb, kb, kend);
  cp_async_commit();

  // Gate and bias of this CTA's outputs (rows 4 rank .. 4 rank + 3), fetched
  // now so their latency hides behind the products.
  const int r_lo = 4 * static_cast<int>(rank);
  float gate[kSmMaxOut], bv[kSmMaxOut];
#pragma unroll
  for (int m = 0; m < kSmMaxOut; ++m) {
    const int idx = tid + m * kSmThreads;
    const int r = r_lo + idx / D, f = idx % D, i = q0 + r;
    gate[m] = 1.f, bv[m] = 0.f;
    if (idx < 4 * D && i < C) {
      if (args.has_zl)
        gate[m] = __ldg(static_cast<const float*>(args.z_tl) + static_cast<int64_t>(b) * args.zl_bs +
                        static_cast<int64_t>(i) * args.zl_rs + f);
      if (args.has_bias) bv[m] = __ldg(static_cast<const float*>(args.bias) + f);
    }
  }

  const float norm_eps = args.norm_eps_f;
  const int kk = tid % kb, h = tid / kb;  // phase 1: key kk, feature slice h
  const int seg_bytes = row_bytes / kpt;
  const int rpt = kSmRows / kpt;  // P rows of this thread: h * rpt ...
  const int nfg = D <= 128 ? 1 : 2;  // phase 2: feature groups of 128
  const int ks = kSmWarps / nfg;     // key shares per feature group
  const int fg = warp % nfg, ksp = warp / nfg;
  const int f2 = fg * 128 + 4 * lane;  // first feature of the lane in phase 2
  uint64_t acc2[kSmRows][2] = {};      // [row][feature pair]

  for (int n = 0; n < nblk; ++n) {
    const int k0 = kbeg + n * kb;
    char* zcur = zb + (n & 1) * g.zbuf;
    // V of this thread's P entries, fetched before the wait.
    float vreg[kSmRptMax];
#pragma unroll
    for (int u = 0; u < kSmRptMax; ++u) vreg[u] = 1.f;
    {
      const int j = k0 + kk;
      if (args.has_v && j < kend)
#pragma unroll
        for (int u = 0; u < kSmRptMax; ++u) {
          const int i = q0 + h * rpt + u;
          if (u < rpt && i < C)
            vreg[u] = __ldg(static_cast<const float*>(args.v) + static_cast<int64_t>(i) * args.v_rs + j);
        }
    }
    cp_async_wait_1();  // this block's group; the next block's may stay in flight
    __syncthreads();
    if (n == 0 && warp < kSmRows) {  // inverse query norms, a warp per row
      float ss = 0.f;
      for (int s = lane; s < nseg; s += 32) {
        const float4 x = *reinterpret_cast<const float4*>(qb + warp * stride + 16 * s);
        ss = fmaf(x.x, x.x, fmaf(x.y, x.y, fmaf(x.z, x.z, fmaf(x.w, x.w, ss))));
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      if (lane == 0) rq[warp] = 1.f / fmaxf(sqrtf(ss), norm_eps);
    }

    // ---- phase 1: partial dot products of key kk with the 8 query rows
    // (even and odd features in the two lanes of each pair).
    {
      uint64_t acc[kSmRows] = {};
      uint64_t ssq = 0;
      const char* zrow = zcur + kk * stride + h * seg_bytes;
      const char* qrow = qb + h * seg_bytes;
#pragma unroll 2
      for (int c = 0; c < seg_bytes; c += 16) {
        const ulonglong2 z = *reinterpret_cast<const ulonglong2*>(zrow + c);
        ssq = fma_f32x2(z.x, z.x, ssq);
        ssq = fma_f32x2(z.y, z.y, ssq);
#pragma unroll
        for (int r = 0; r < kSmRows; ++r) {
          const ulonglong2 q = *reinterpret_cast<const ulonglong2*>(qrow + r * stride + c);
          acc[r] = fma_f32x2(q.x, z.x, acc[r]);
          acc[r] = fma_f32x2(q.y, z.y, acc[r]);
        }
      }
#pragma unroll
      for (int r = 0; r < kSmRows; ++r) {
        const float2 a = unpack_f32x2(acc[r]);
        part[(h * 9 + r) * kb + kk] = a.x + a.y;
      }
      const float2 s2 = unpack_f32x2(ssq);
      part[(h * 9 + 8) * kb + kk] = s2.x + s2.y;
    }
    __syncthreads();

    // ---- P entries of key kk for rows h * rpt .. h * rpt + rpt - 1.
    {
      const int j = k0 + kk;
      float ss = 0.f;
      for (int hh = 0; hh < kpt; ++hh) ss += part[(hh * 9 + 8) * kb + kk];
      const float rk = 1.f / fmaxf(sqrtf(ss), norm_eps);
      const bool key_ok = j < kend && kv(j);
#pragma unroll
      for (int u = 0; u < kSmRptMax; ++u) {
        if (u >= rpt) break;  // uniform across the warp
        const int r = h * rpt + u, i = q0 + r;
        float s = 0.f;
        for (int hh = 0; hh < kpt; ++hh) s += part[(hh * 9 + r) * kb + kk];
        const bool ok = key_ok && row_ok_s[r] && (!args.causal || j <= i);
        const float p = ok ? s * rq[r] * rk * vreg[u] : 0.f;
        *reinterpret_cast<float2*>(pbuf + (kk * kSmRows + r) * 2) = make_float2(p, p);
        if (args.normalize) {
          float sm = p;
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) sm += __shfl_xor_sync(0xffffffffu, sm, o);
          if (lane == 0) dpart[(kk >> 5) * kSmRows + r] = sm;
        }
      }
    }
    __syncthreads();
    if (args.normalize && tid < kSmRows) {
      // The key groups of the block in order (deterministic).
      float sm = 0.f;
      for (int kg = 0; kg < kb / 32; ++kg) sm += dpart[kg * kSmRows + tid];
      den[tid] += sm;
    }

    // ---- phase 2: O += P Z over this warp's share of the block's keys.
    {
      const int kn = min(kb, kend - k0);
      const int per = kb / ks;
      const int kb0 = ksp * per, kb1 = min(kb0 + per, kn);
      if (f2 < D) {
        const char* zcol = zcur + 4 * f2;
#pragma unroll 4
        for (int k = kb0; k < kb1; ++k) {
          const ulonglong2* pp = reinterpret_cast<const ulonglong2*>(pbuf + k * kSmRows * 2);
          const ulonglong2 z = *reinterpret_cast<const ulonglong2*>(zcol + k * stride);
#pragma unroll
          for (int rr = 0; rr < kSmRows / 2; ++rr) {
            const ulonglong2 p = pp[rr];  // rows 2 rr and 2 rr + 1, each value twice
            acc2[2 * rr][0] = fma_f32x2(p.x, z.x, acc2[2 * rr][0]);
            acc2[2 * rr][1] = fma_f32x2(p.x, z.y, acc2[2 * rr][1]);
            acc2[2 * rr + 1][0] = fma_f32x2(p.y, z.x, acc2[2 * rr + 1][0]);
            acc2[2 * rr + 1][1] = fma_f32x2(p.y, z.y, acc2[2 * rr + 1][1]);
          }
        }
      }
    }
    __syncthreads();  // the block's buffer and P are free again
    if (n + 2 < nblk) copy_rows(zcur, k0 + 2 * kb, kb, kend);
    cp_async_commit();
  }
  cp_async_wait_0();
  __syncthreads();

  // ---- this CTA's partial O: the warps' sums in order.
  float* red = reinterpret_cast<float*>(zb);  // [8 warps][8 rows][128]
#pragma unroll
  for (int r = 0; r < kSmRows; ++r)
    *reinterpret_cast<ulonglong2*>(red + (warp * kSmRows + r) * 128 + 4 * lane) =
        make_ulonglong2(acc2[r][0], acc2[r][1]);
  __syncthreads();
  for (int idx = tid; idx < kSmRows * D; idx += kSmThreads) {
    const int r = idx / D, f = idx - r * D;
    const int fgr = f >> 7, fl = f & 127;
    float o = 0.f;
    for (int s = 0; s < ks; ++s) o += red[((s * nfg + fgr) * kSmRows + r) * 128 + fl];
    osum[idx] = o;
  }
  cluster_sync();  // both partial sums are complete and visible to the peer

  // ---- rows 4 rank .. 4 rank + 3: even CTA's sum + odd CTA's sum.
  const uint32_t peer = rank ^ 1u;
  const uint32_t osum_peer = mapa_shared(smem_u32(osum), peer);
  const uint32_t den_peer = mapa_shared(smem_u32(den), peer);
  const float eps = args.eps_f;
  float* out = static_cast<float*>(args.out) + static_cast<int64_t>(b) * args.o_bs;
#pragma unroll
  for (int m = 0; m < kSmMaxOut; ++m) {
    const int idx = tid + m * kSmThreads;
    const int r = r_lo + idx / D, f = idx % D, i = q0 + r;
    if (idx >= 4 * D || i >= C) continue;
    float y = 0.f;
    if (row_ok_s[r]) {
      const int e = r * D + f;
      const float mine = osum[e], other = ld_cluster_f32(osum_peer + 4u * static_cast<uint32_t>(e));
      const float o = rank ? other + mine : mine + other;
      if (args.normalize) {
        const float dm = den[r], dp = ld_cluster_f32(den_peer + 4u * static_cast<uint32_t>(r));
        y = o / ((rank ? dp + dm : dm + dp) + eps);
      } else {
        y = o;
      }
      y += bv[m];
      y = activate<float>(y, args.act);
      y *= gate[m];
    }
    out[static_cast<int64_t>(i) * args.o_rs + f] = y;
  }
  // The peer has read this CTA's shared memory (no data is published here, so
  // the arrive needs no release).
  asm volatile("barrier.cluster.arrive.relaxed.aligned;\n\tbarrier.cluster.wait.aligned;" ::: "memory");
}

}  // namespace avey
