// General CUDA-core contextualizer kernel: any dtype (f32 / f16 / bf16 / f64),
// any feature count and any row / batch strides. It is the kernel for fp32 and
// fp64 inputs and for shapes the tcgen05 kernel does not take (feature counts
// that are not a multiple of 8, unaligned views, contexts above 512).
//
// One CTA owns 16 query rows x 128 output features of one batch row and
// streams 32-key tiles: the raw Gram tile Z_q Z_k^T is accumulated over 32-wide
// feature chunks staged in shared memory, scaled by both inverse row norms, V
// and the masks into P, and then P Z_k is accumulated into registers (one
// output feature per thread, 16 rows). Arithmetic is in A (fp32, or fp64 for
// fp64 inputs), like the reference's fp32 accumulation (ops.py:63).
#pragma once

#include "common.cuh"

namespace avey {

constexpr int kSimtRows = 16;     // query rows per CTA
constexpr int kSimtFeat = 128;    // output features per CTA (= threads)
constexpr int kSimtKeys = 32;     // keys per tile
constexpr int kSimtChunk = 32;    // features per Gram staging chunk

template <typename T, typename A>
__device__ __forceinline__ A ld_acc(const T* p) {
  if constexpr (sizeof(T) == 2) {
    return static_cast<A>(Elem<T>::load(p));
  } else {
    return static_cast<A>(__ldg(p));
  }
}

template <typename T, typename A>
__global__ void __launch_bounds__(kSimtFeat) simt_contextualize(const FwdArgs args) {
  const int tid = threadIdx.x;
  const int b = blockIdx.z;
  const int q0 = blockIdx.x * kSimtRows;
  const int f = blockIdx.y * kSimtFeat + tid;
  const int C = args.ctx, D = args.feat;
  const A eps = sizeof(A) == 8 ? static_cast<A>(args.eps_d) : static_cast<A>(args.eps_f);
  const A norm_eps =
      sizeof(A) == 8 ? static_cast<A>(args.norm_eps_d) : static_cast<A>(args.norm_eps_f);

  const T* zr = static_cast<const T*>(args.z_tr) + static_cast<int64_t>(b) * args.zr_bs;

  __shared__ A q_s[kSimtRows][kSimtChunk + 1];
  __shared__ A k_s[kSimtKeys][kSimtChunk + 1];
  __shared__ A p_s[kSimtRows][kSimtKeys];
  __shared__ A rq_s[kSimtRows];
  __shared__ A kss_s[kSimtKeys];
  __shared__ A den_s[kSimtRows];
  __shared__ int qvalid_s[kSimtRows];
  __shared__ int kvalid_s[kSimtKeys];
  __shared__ int last_valid_s;

  // Last valid position of this batch row: keys past it contribute nothing.
  if (tid == 0) last_valid_s = -1;
  __syncthreads();
  if (args.has_valid) {
    int last = -1;
    for (int j = tid; j < C; j += kSimtFeat)
      if (mask_ok(args, b, j)) last = j;
    if (last >= 0) atomicMax(&last_valid_s, last);
  }
  if (tid < kSimtRows) {
    const int i = q0 + tid;
    qvalid_s[tid] = (i < C) && mask_ok(args, b, i);
    den_s[tid] = A(0);
  }
  __syncthreads();
  const int key_end0 = args.has_valid ? last_valid_s + 1 : C;
  const int key_end = args.causal ? min(key_end0, min(C, q0 + kSimtRows)) : key_end0;

  // Inverse L2 norms of the query rows (invalid rows are masked anyway).
  {
    const int warp = tid >> 5, lane = tid & 31;
    for (int r = warp; r < kSimtRows; r += kSimtFeat / 32) {
      const int i = q0 + r;
      A ss = A(0);
      if (i < C)
        for (int c = lane; c < D; c += 32) {
          const A x = ld_acc<T, A>(zr + static_cast<int64_t>(i) * args.zr_rs + c);
          ss += x * x;
        }
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      if (lane == 0) rq_s[r] = A(1) / max(sqrt(ss), norm_eps);
    }
  }

  A acc[kSimtRows];
#pragma unroll
  for (int r = 0; r < kSimtRows; ++r) acc[r] = A(0);

  for (int k0 = 0; k0 < key_end; k0 += kSimtKeys) {
    // Raw Gram tile G[r][kk] = z_{q0+r} . z_{k0+kk}, four entries per thread.
    A g[4] = {A(0), A(0), A(0), A(0)};
    if (tid < kSimtKeys) kss_s[tid] = A(0);
    for (int c0 = 0; c0 < D; c0 += kSimtChunk) {
      __syncthreads();
      for (int e = tid; e < (kSimtRows + kSimtKeys) * kSimtChunk; e += kSimtFeat) {
        const int row = e / kSimtChunk, c = c0 + e % kSimtChunk;
        const int src = row < kSimtRows ? q0 + row : k0 + row - kSimtRows;
        A x = A(0);
        if (src < C && c < D) x = ld_acc<T, A>(zr + static_cast<int64_t>(src) * args.zr_rs + c);
        if (row < kSimtRows)
          q_s[row][e % kSimtChunk] = x;
        else
          k_s[row - kSimtRows][e % kSimtChunk] = x;
      }
      __syncthreads();
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const int e = tid + m * kSimtFeat;
        const int r = e / kSimtKeys, kk = e % kSimtKeys;
        A s = g[m];
#pragma unroll 8
        for (int c = 0; c < kSimtChunk; ++c) s += q_s[r][c] * k_s[kk][c];
        g[m] = s;
      }
      if (tid < kSimtKeys) {
        A s = kss_s[tid];
#pragma unroll 8
        for (int c = 0; c < kSimtChunk; ++c) s += k_s[tid][c] * k_s[tid][c];
        kss_s[tid] = s;
      }
    }
    if (tid < kSimtKeys) {
      const int j = k0 + tid;
      kvalid_s[tid] = (j < key_end) && mask_ok(args, b, j);
    }
    __syncthreads();
    // P = G * rinv_q * rinv_k * V, masked by select so NaN padding cannot leak.
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const int e = tid + m * kSimtFeat;
      const int r = e / kSimtKeys, kk = e % kSimtKeys;
      const int i = q0 + r, j = k0 + kk;
      A p = A(0);
      const bool ok = qvalid_s[r] && kvalid_s[kk] && (!args.causal || j <= i);
      if (ok) {
        p = g[m] * rq_s[r] * (A(1) / max(sqrt(kss_s[kk]), norm_eps));
        if (args.has_v)
          p *= ld_acc<T, A>(static_cast<const T*>(args.v) + static_cast<int64_t>(i) * args.v_rs + j);
      }
      p_s[r][kk] = p;
    }
    __syncthreads();
    if (args.normalize && tid < kSimtRows) {
      A s = A(0);
      for (int kk = 0; kk < kSimtKeys; ++kk) s += p_s[tid][kk];
      den_s[tid] += s;
    }
    // acc[r] += sum_kk P[r][kk] * z_{k0+kk}[f]; invalid keys read as zero.
    if (f < D) {
      const int kmax = min(kSimtKeys, key_end - k0);
      for (int kk = 0; kk < kmax; ++kk) {
        if (!kvalid_s[kk]) continue;
        const A z = ld_acc<T, A>(zr + static_cast<int64_t>(k0 + kk) * args.zr_rs + f);
#pragma unroll
        for (int r = 0; r < kSimtRows; ++r) acc[r] += p_s[r][kk] * z;
      }
    }
  }
  __syncthreads();

  if (f >= D) return;
  const A bias = args.has_bias ? ld_acc<T, A>(static_cast<const T*>(args.bias) + f) : A(0);
  const T* zl = args.has_zl ? static_cast<const T*>(args.z_tl) + static_cast<int64_t>(b) * args.zl_bs
                            : nullptr;
  T* out = static_cast<T*>(args.out) + static_cast<int64_t>(b) * args.o_bs;
#pragma unroll
  for (int r = 0; r < kSimtRows; ++r) {
    const int i = q0 + r;
    if (i >= C) break;
    A y = A(0);
    if (qvalid_s[r]) {
      y = acc[r];
      if (args.normalize) y = y / (den_s[r] + eps);
      y = activate<A>(y + bias, args.act);
      if (zl) y *= ld_acc<T, A>(zl + static_cast<int64_t>(i) * args.zl_rs + f);
    }
    out[static_cast<int64_t>(i) * args.o_rs + f] = store_cast<T, A>(y);
  }
}

}  // namespace avey
