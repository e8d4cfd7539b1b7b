// Two-phase CUDA-core kernel: the path for fp32 inputs and for 16-bit inputs
// the tensor-core kernels do not take (feature counts that are not a multiple
// of 8, unaligned views, contexts above 8192). fp64 keeps simt_contextualize.
//
// One CTA owns 32 query rows of one batch row (two CTAs per SM):
//   phase 1  S = Z_q Z_k^T (once per query tile when the row has at most 512
//            allowed keys, else once per feature pass and 512-key super-block),
//            in blocks of 256 keys: 8 x 4 register tiles
//            per thread over feature-major shared tiles of 32 features; the
//            key rows' sums of squares are accumulated from the same tiles.
//            P = S * rinv_q * rinv_k * V under the masks goes to shared memory
//            (key-major, 32 rows per key), with the Avey-B row sums.
//   phase 2  O = P Z in passes of 256 output features: 8 x 4 register tiles,
//            Z streamed in chunks of 32 keys; then the epilogue (divide,
//            bias, activation, gate, row mask).
// Rows that are padding are zeroed as they are loaded (ops.py:64-67), so a
// NaN in them cannot reach any product. Arithmetic is fp32 like the
// reference's (ops.py:63); S is computed once per query tile instead of once
// per output-feature tile as in simt_contextualize and the reference's Triton
// kernel (_triton.py:78-105).
#pragma once

#include "common.cuh"

namespace avey {

constexpr int kS2Rows = 32;       // query rows per CTA
constexpr int kS2Keys = 256;      // keys per phase-1 block
constexpr int kS2Feat = 256;      // output features per phase-2 pass
constexpr int kS2Chunk = 32;      // features (phase 1) / keys (phase 2) per staged chunk
constexpr int kS2Threads = 256;
constexpr int kS2MaxCtx = 512;
constexpr int kS2KStride = kS2Keys + 4;  // floats per row of the K / Z staging tile
constexpr int kS2SmemBytes =
    (kS2Chunk * kS2Rows + kS2Chunk * kS2KStride + kS2MaxCtx * kS2Rows + kS2MaxCtx + 4 * kS2Rows) *
        4 +
    kS2MaxCtx;

// Four consecutive elements of a row starting at p (n_ok of them in range),
// as fp32; vectorised when the row is 16-byte aligned fp32.
template <typename T>
__device__ __forceinline__ float4 s2_load4(const T* p, int n_ok, bool vec) {
  if constexpr (std::is_same<T, float>::value) {
    if (vec && n_ok >= 4) return __ldg(reinterpret_cast<const float4*>(p));
  }
  float v[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) v[e] = e < n_ok ? Elem<T>::load(p + e) : 0.f;
  return make_float4(v[0], v[1], v[2], v[3]);
}

// LONG: the instantiation for contexts above 512 (it also carries the
// super-block loop, whose live accumulators cost registers the short one keeps).
template <typename T, bool LONG>
__global__ void __launch_bounds__(kS2Threads, 2) simt2_contextualize(const FwdArgs args) {
  extern __shared__ __align__(16) float s2_smem[];
  float* qs = s2_smem;                       // [32 features][32 rows]
  float* ks = qs + kS2Chunk * kS2Rows;       // [32 features][256 keys] / [32 keys][256 features]
  float* ps = ks + kS2Chunk * kS2KStride;    // [512 keys][32 rows]
  float* rk = ps + kS2MaxCtx * kS2Rows;      // inverse key norms
  float* rq = rk + kS2MaxCtx;                // inverse query norms
  float* den = rq + kS2Rows;                 // Avey-B row sums
  float* dpart = den + kS2Rows;              // [2][32] per-warp partial row sums
  // Validity per position: cached in shared memory for rows of at most 512
  // positions; the LONG instantiation reads the mask from global memory.
  uint8_t* kv_s = reinterpret_cast<uint8_t*>(dpart + 2 * kS2Rows);
  __shared__ int last_valid_s;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int b = blockIdx.y;
  const int C = args.ctx, D = args.feat;
  const int nqt = (C + kS2Rows - 1) / kS2Rows;
  const int qt = args.causal ? nqt - 1 - static_cast<int>(blockIdx.x) : static_cast<int>(blockIdx.x);
  const int q0 = qt * kS2Rows;
  const T* zr = static_cast<const T*>(args.z_tr) + static_cast<int64_t>(b) * args.zr_bs;
  const bool vec = std::is_same<T, float>::value &&
                   (reinterpret_cast<uintptr_t>(args.z_tr) & 15u) == 0 && (args.zr_rs & 3) == 0 &&
                   (args.zr_bs & 3) == 0;

  // Position j < C is a valid (non-padding) row.
  auto kv = [&](int j) -> bool {
    if constexpr (LONG) return mask_ok(args, b, j);
    else return kv_s[j] != 0;
  };
  if (tid == 0) last_valid_s = -1;
  __syncthreads();
  {
    int last = -1;
    for (int j = tid; j < C; j += kS2Threads) {
      const uint8_t ok = mask_ok(args, b, j) ? 1 : 0;
      if constexpr (!LONG) kv_s[j] = ok;  // C <= 512 here (the host's choice)
      if (ok) last = j;
    }
    if (last >= 0) atomicMax(&last_valid_s, last);
  }
  if (tid < kS2Rows) den[tid] = 0.f;
  __syncthreads();
  const int kv_end = last_valid_s + 1;
  const int key_end = args.causal ? min(kv_end, q0 + kS2Rows) : kv_end;
  const float norm_eps = args.norm_eps_f;

  // Inverse norms of the 32 query rows (a warp per row).
  for (int r = warp; r < kS2Rows; r += kS2Threads / 32) {
    const int i = q0 + r;
    float ss = 0.f;
    if (i < C && kv(i))
      for (int c = lane; c < D; c += 32) {
        const float x = Elem<T>::load(zr + static_cast<int64_t>(i) * args.zr_rs + c);
        ss = fmaf(x, x, ss);
      }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) rq[r] = 1.f / fmaxf(sqrtf(ss), norm_eps);
  }

  // ---------------- phase 1: P for keys [sb, se) (se - sb <= 512) into ps,
  // blocks of 256 keys; the row sums accumulate when `rowsum` is set.
  auto phase1 = [&](int sb, int se, bool rowsum) {
    const int tr = tid >> 6;   // rows 8 tr .. 8 tr + 7
    const int tk = tid & 63;   // keys 4 tk .. 4 tk + 3 of the block
    for (int k0 = sb; k0 < se; k0 += kS2Keys) {
      float acc[8][4];
      float ksq[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int r = 0; r < 8; ++r)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[r][j] = 0.f;
      for (int c0 = 0; c0 < D; c0 += kS2Chunk) {
        __syncthreads();
        {  // query chunk: 32 rows x 32 features, one 4-vector per thread
          const int row = tid >> 3, c4 = tid & 7, i = q0 + row, c = c0 + 4 * c4;
          float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
          if (i < C && kv(i) && c < D) x = s2_load4<T>(zr + static_cast<int64_t>(i) * args.zr_rs + c, D - c, vec);
          qs[(4 * c4 + 0) * kS2Rows + row] = x.x;
          qs[(4 * c4 + 1) * kS2Rows + row] = x.y;
          qs[(4 * c4 + 2) * kS2Rows + row] = x.z;
          qs[(4 * c4 + 3) * kS2Rows + row] = x.w;
        }
#pragma unroll
        for (int m = 0; m < 8; ++m) {  // key chunk: 256 keys x 32 features
          const int e = tid + m * kS2Threads;
          const int key = e >> 3, c4 = e & 7, j = k0 + key, c = c0 + 4 * c4;
          float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
          if (j < se && kv(j) && c < D) x = s2_load4<T>(zr + static_cast<int64_t>(j) * args.zr_rs + c, D - c, vec);
          ks[(4 * c4 + 0) * kS2KStride + key] = x.x;
          ks[(4 * c4 + 1) * kS2KStride + key] = x.y;
          ks[(4 * c4 + 2) * kS2KStride + key] = x.z;
          ks[(4 * c4 + 3) * kS2KStride + key] = x.w;
        }
        __syncthreads();
#pragma unroll 8
        for (int c = 0; c < kS2Chunk; ++c) {
          const float4 qa = *reinterpret_cast<const float4*>(&qs[c * kS2Rows + 8 * tr]);
          const float4 qb = *reinterpret_cast<const float4*>(&qs[c * kS2Rows + 8 * tr + 4]);
          const float4 kk = *reinterpret_cast<const float4*>(&ks[c * kS2KStride + 4 * tk]);
          const float q[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
          const float k[4] = {kk.x, kk.y, kk.z, kk.w};
#pragma unroll
          for (int r = 0; r < 8; ++r)
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[r][j] = fmaf(q[r], k[j], acc[r][j]);
          if (tr == 0)
#pragma unroll
            for (int j = 0; j < 4; ++j) ksq[j] = fmaf(k[j], k[j], ksq[j]);
        }
      }
      // Inverse key norms of the block (keys past the range are 0 rows).
      if (tr == 0)
#pragma unroll
        for (int j = 0; j < 4; ++j) rk[k0 - sb + 4 * tk + j] = 1.f / fmaxf(sqrtf(ksq[j]), norm_eps);
      __syncthreads();
      float dsum[8];
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        const int row = 8 * tr + r, i = q0 + row;
        const bool row_ok = i < C && kv(i);
        float pv[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int key = k0 + 4 * tk + j;
          float p = 0.f;
          const bool ok = row_ok && key < se && kv(key) && (!args.causal || key <= i);
          if (ok) {
            p = acc[r][j] * rq[row] * rk[key - sb];
            if (args.has_v)
              p *= Elem<T>::load(static_cast<const T*>(args.v) + static_cast<int64_t>(i) * args.v_rs + key);
          }
          pv[j] = p;
        }
        dsum[r] = (pv[0] + pv[1]) + (pv[2] + pv[3]);
#pragma unroll
        for (int j = 0; j < 4; ++j) ps[(k0 - sb + 4 * tk + j) * kS2Rows + row] = pv[j];
      }
      if (rowsum) {
        // Row sums: a fixed-order warp reduction, then the two warps of each
        // row group in order (deterministic).
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          float sm = dsum[r];
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) sm += __shfl_xor_sync(0xffffffffu, sm, o);
          if (lane == 0) dpart[(warp & 1) * kS2Rows + 8 * tr + r] = sm;
        }
        __syncthreads();
        if (tid < kS2Rows) den[tid] += dpart[tid] + dpart[kS2Rows + tid];
      }
    }
    __syncthreads();
  };

  // ---------------- phase 2: acc += P[keys sb..se) Z[keys, f0 .. f0 + 255].
  const int tr = tid >> 6;   // rows 8 tr .. 8 tr + 7
  const int tf = tid & 63;   // features 4 tf .. 4 tf + 3 of the pass
  auto phase2 = [&](int sb, int se, int f0, float (&acc)[8][4]) {
    for (int kc = sb; kc < se; kc += kS2Chunk) {
      __syncthreads();
#pragma unroll
      for (int m = 0; m < 8; ++m) {  // Z chunk: 32 keys x 256 features
        const int e = tid + m * kS2Threads;
        const int key = e >> 6, f4 = e & 63, j = kc + key, f = f0 + 4 * f4;
        float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
        if (j < se && kv(j) && f < D) x = s2_load4<T>(zr + static_cast<int64_t>(j) * args.zr_rs + f, D - f, vec);
        *reinterpret_cast<float4*>(&ks[key * kS2KStride + 4 * f4]) = x;
      }
      __syncthreads();
      const int kn = min(kS2Chunk, se - kc);
      for (int k = 0; k < kn; ++k) {
        const float4 pa = *reinterpret_cast<const float4*>(&ps[(kc - sb + k) * kS2Rows + 8 * tr]);
        const float4 pb = *reinterpret_cast<const float4*>(&ps[(kc - sb + k) * kS2Rows + 8 * tr + 4]);
        const float4 zz = *reinterpret_cast<const float4*>(&ks[k * kS2KStride + 4 * tf]);
        const float p[8] = {pa.x, pa.y, pa.z, pa.w, pb.x, pb.y, pb.z, pb.w};
        const float z[4] = {zz.x, zz.y, zz.z, zz.w};
#pragma unroll
        for (int r = 0; r < 8; ++r)
#pragma unroll
          for (int c = 0; c < 4; ++c) acc[r][c] = fmaf(p[r], z[c], acc[r][c]);
      }
    }
  };

  const float eps = args.eps_f;
  const T* zl = args.has_zl ? static_cast<const T*>(args.z_tl) + static_cast<int64_t>(b) * args.zl_bs
                            : nullptr;
  T* out = static_cast<T*>(args.out) + static_cast<int64_t>(b) * args.o_bs;
  auto epilogue = [&](int f0, const float (&acc)[8][4]) {
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const int row = 8 * tr + r, i = q0 + row;
      if (i >= C) continue;
      const bool row_ok = kv(i) != 0;
      const float inv = args.normalize ? 1.f / (den[row] + eps) : 1.f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int f = f0 + 4 * tf + c;
        if (f >= D) continue;
        float y = 0.f;
        if (row_ok) {
          y = args.normalize ? acc[r][c] * inv : acc[r][c];
          if (args.has_bias) y += Elem<T>::load(static_cast<const T*>(args.bias) + f);
          y = activate<float>(y, args.act);
          if (zl) y *= Elem<T>::load(zl + static_cast<int64_t>(i) * args.zl_rs + f);
        }
        out[static_cast<int64_t>(i) * args.o_rs + f] = store_cast<T, float>(y);
      }
    }
  };

  if (!LONG || key_end <= kS2MaxCtx) {
    // P for every key fits in shared memory: S once, then every feature pass.
    phase1(0, key_end, args.normalize != 0);
    for (int f0 = 0; f0 < D; f0 += kS2Feat) {
      float acc[8][4] = {};
      phase2(0, key_end, f0, acc);
      epilogue(f0, acc);
    }
  } else if constexpr (LONG) {
    // Longer rows: super-blocks of 512 keys, S recomputed for each feature
    // pass (the row sums are taken in the first pass).
    for (int f0 = 0; f0 < D; f0 += kS2Feat) {
      float acc[8][4] = {};
      for (int sb = 0; sb < key_end; sb += kS2MaxCtx) {
        const int se = min(key_end, sb + kS2MaxCtx);
        phase1(sb, se, args.normalize != 0 && f0 == 0);
        phase2(sb, se, f0, acc);
      }
      epilogue(f0, acc);
    }
  }
}

}  // namespace avey
