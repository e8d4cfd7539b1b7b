// Backward of the contextualizer: the elementwise and reduction steps that
// sit between the batched GEMMs of the gradient.
//
// Per batch row (Z = z_tr with padded rows zeroed, r = 1 / max(||Z||, ne),
// z^ = r Z, G = z^ z^T, S = G (.) V (.) M, num = S Z, den = rowsum(S) + eps, Y0 = num /
// den for Avey-B (num for Avey), Ypre = Y0 + bias, out = act(Ypre) (.) gate,
// rows of padded queries zeroed), the gradient is
//
//   dYpre = dout (.) gate (.) act'(Ypre)     dgate = dout (.) act(Ypre)
//   dbias = sum over rows of dYpre
//   dnum  = dYpre / den,  dden_i = -sum_f dYpre_if Y0_if / den_i   (Avey-B)
//   dS    = (dnum Z^T + dden 1^T) (.) M         dV = sum_b dS (.) G
//   dG    = dS (.) V,  dz^ = (dG + dG^T) z^,    dZ = S^T dnum + dz^ through
//           the normalisation (dz^ - z^ (z^ . dz^)) / ||Z||  (or dz^ / ne when
//           ||Z|| < ne), zero on padded rows.
//
// The five products are plain batched GEMMs run by the caller between these
// steps, all on Z itself (exact in the input type): Gr = Z Z^T (G = r_i r_j Gr),
// num = S Z, dnum Z^T, S^T dnum and (dGsym diag(r)) Z = dz^. Folding the norms
// into the fp32 steps instead of rounding z^ to a 16-bit GEMM operand keeps the
// Gram exact to fp32, as in the forward kernels. Every step here is one launch
// that streams its operands once; reductions (dbias, dV, dden) use fixed
// orders, so gradients are bitwise reproducible.
//
// Reference: torch autograd through avey_kernels/ops.py:61-91 (_reference):
// masked_fill before the arithmetic (ops.py:64-67), F.normalize (68), the
// masks (69-77), numerator / denominator (78-80), bias (81-82), activation
// (ops.py:49-58), gate and final row mask (84-90).
#pragma once

#include <type_traits>

#include "common.cuh"

namespace avey {

// Plain-old-data copy of AveyBwdParams for kernels.
struct BwdArgs {
  const void* z_tr;
  const void* v;
  const void* z_tl;
  const void* bias;
  const uint8_t* valid;
  const void* gout;
  int64_t zr_bs, zr_rs, v_rs, zl_bs, zl_rs, va_bs, va_rs, go_bs, go_rs;
  int64_t gr_bs, gr_rs;  // strides of grad_z_tr and grad_z_tl (elements)
  int batch, ctx, feat;
  double eps, norm_eps;
  int causal, normalize, act;
  void* zm;     // [B, C, d]  GEMM type: Z (padded rows zeroed)
  void* norms;  // [B, C]     acc: ||Z||, -1 on padded rows
  void* g;      // [B, C, C]  acc: Z Z^T
  void* s;      // [B, C, C]  GEMM type: S
  void* den;    // [B, C]     acc: rowsum(S) + eps
  void* num;    // [B, C, d]  acc: S Z
  void* dnum;   // [B, C, d]  GEMM type
  void* dden;   // [B, C]     acc
  void* ds0;    // [B, C, C]  acc: dnum Z^T
  void* dgsym;  // [B, C, C]  GEMM type: (dG + dG^T) diag(r)
  void* dzd;    // [B, C, d]  acc: S^T dnum
  void* dzh;    // [B, C, d]  acc: dz^ = dgsym Z
  void* part;   // acc partial sums (dbias, dV)
  void* gz_tr;  // [B, C, d]  input type, strides gr_bs / gr_rs
  void* gv;     // [C, C]
  void* gz_tl;  // [B, C, d]
  void* gbias;  // [d]
};

constexpr int kBwdThreads = 256;
constexpr int kBwdEpiRows = 64;   // rows per epilogue block (8 per warp)
constexpr int kBwdEpiChunk = 256; // features per epilogue pass (8 per lane)
constexpr int kBwdTile = 32;      // dscores tile edge

template <typename A, typename T>
__device__ __forceinline__ A ld_as(const T* p) {
  if constexpr (std::is_same<T, __half>::value || std::is_same<T, __nv_bfloat16>::value) {
    return static_cast<A>(Elem<T>::load(p));
  } else {
    return static_cast<A>(__ldg(p));
  }
}

template <typename T, typename A>
__device__ __forceinline__ void st_as(T* p, A x) {
  *p = store_cast<T, A>(x);
}

// r = 1 / max(||Z||, ne) of row `row` (flattened batch x context index).
template <typename A>
__device__ __forceinline__ A inv_norm(const BwdArgs& a, int64_t row) {
  const A n = static_cast<const A*>(a.norms)[row];
  const A ne = static_cast<A>(a.norm_eps);
  return A(1) / (n > ne ? n : ne);
}

// Element offset of row (b, n) in grad_z_tr / grad_z_tl.
__device__ __forceinline__ int64_t grad_off(const BwdArgs& a, int b, int n) {
  return static_cast<int64_t>(b) * a.gr_bs + static_cast<int64_t>(n) * a.gr_rs;
}

__device__ __forceinline__ bool row_valid(const BwdArgs& a, int b, int n) {
  return !a.valid || a.valid[static_cast<int64_t>(b) * a.va_bs + static_cast<int64_t>(n) * a.va_rs] != 0;
}

// Row (b, n) = flat row r of zm. A caller without a padding mask whose GEMM
// type is the input type may pass no zm (it equals z_tr then): the row is
// read from z_tr through its strides.
template <typename G>
__device__ __forceinline__ const G* zm_row(const BwdArgs& a, int64_t r, int b, int n) {
  if (a.zm) return static_cast<const G*>(a.zm) + r * a.feat;
  return static_cast<const G*>(a.z_tr) + static_cast<int64_t>(b) * a.zr_bs +
         static_cast<int64_t>(n) * a.zr_rs;
}

template <typename A>
__device__ __forceinline__ A warp_sum(A x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
  return x;
}

// Derivative of the activations of the reference (ops.py:49-58) at x, with
// torch's conventions: relu' = [x > 0]; relu2' = 2 max(x, 0); silu' =
// s (1 + x (1 - s)); tanh-gelu' = 0.5 (1 + t) + 0.5 x (1 - t^2) k (1 + 3 c x^2),
// t = tanh(k (x + c x^3)), k = sqrt(2 / pi), c = 0.044715.
template <typename A>
__device__ __forceinline__ A activate_grad(A x, int act) {
  switch (act) {
    case 1:
      return x > A(0) ? A(1) : A(0);
    case 2:
      return x > A(0) ? A(2) * x : A(0);
    case 3: {
      const A sg = sigmoid_stable(x);
      return sg * (A(1) + x * (A(1) - sg));
    }
    case 4: {
      const A k = A(0.7978845608028654), c = A(0.044715);
      const A t = tanh(k * (x + c * x * x * x));
      return A(0.5) * (A(1) + t) + A(0.5) * x * (A(1) - t * t) * k * (A(1) + A(3) * c * x * x);
    }
    default:
      return A(1);
  }
}

// Step 1: Z (padded rows zeroed) in the GEMM type and ||Z|| per row. One warp
// per row.
template <typename T, typename G, typename A>
__global__ void __launch_bounds__(kBwdThreads) bwd_prep(const BwdArgs a) {
  const int lane = threadIdx.x & 31;
  const int64_t rows = static_cast<int64_t>(a.batch) * a.ctx;
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * (kBwdThreads / 32);
  const int d = a.feat;
  const T* z = static_cast<const T*>(a.z_tr);
  G* zm = static_cast<G*>(a.zm);
  for (int64_t r = (static_cast<int64_t>(blockIdx.x) * kBwdThreads + threadIdx.x) >> 5; r < rows;
       r += nwarps) {
    const int b = static_cast<int>(r / a.ctx), n = static_cast<int>(r % a.ctx);
    const bool ok = row_valid(a, b, n);
    const T* zr = z + static_cast<int64_t>(b) * a.zr_bs + static_cast<int64_t>(n) * a.zr_rs;
    A ss = 0;
    if (ok)
      for (int f = lane; f < d; f += 32) {
        const A x = ld_as<A>(zr + f);
        ss += x * x;
      }
    ss = warp_sum(ss);
    if (zm)
      for (int f = lane; f < d; f += 32) st_as<G>(zm + r * d + f, ok ? ld_as<A>(zr + f) : A(0));
    if (lane == 0) static_cast<A*>(a.norms)[r] = ok ? sqrt(ss) : A(-1);  // -1 marks padding
  }
}

// Step 2: S = r_i r_j Gr (.) V (.) M (GEMM type) and den = rowsum(S) + eps.
// One warp per (batch, query) row.
template <typename T, typename G, typename A>
__global__ void __launch_bounds__(kBwdThreads) bwd_scores(const BwdArgs a) {
  const int lane = threadIdx.x & 31;
  const int64_t rows = static_cast<int64_t>(a.batch) * a.ctx;
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * (kBwdThreads / 32);
  const int C = a.ctx;
  const A* gr = static_cast<const A*>(a.g);
  G* s = static_cast<G*>(a.s);
  const T* v = static_cast<const T*>(a.v);
  for (int64_t r = (static_cast<int64_t>(blockIdx.x) * kBwdThreads + threadIdx.x) >> 5; r < rows;
       r += nwarps) {
    const int b = static_cast<int>(r / C), i = static_cast<int>(r % C);
    const A ri = inv_norm<A>(a, r);
    A sum = 0;
    for (int j = lane; j < C; j += 32) {
      const bool allowed = (!a.causal || j <= i) && row_valid(a, b, j);
      A x = A(0);
      if (allowed) {
        x = gr[r * C + j] * ri * inv_norm<A>(a, static_cast<int64_t>(b) * C + j);
        if (v) x *= ld_as<A>(v + static_cast<int64_t>(i) * a.v_rs + j);
      }
      st_as<G>(s + r * C + j, x);
      sum += x;
    }
    sum = warp_sum(sum);
    if (lane == 0) static_cast<A*>(a.den)[r] = sum + static_cast<A>(a.eps);
  }
}

// Step 3: epilogue backward. A block owns 64 consecutive (batch, query) rows
// (8 per warp) and walks the features in passes of 256 (8 per lane): it
// writes dgate and dnum, the per-row dden, and its partial dbias (one row of
// `part` per block, summed in block order by bwd_reduce).
template <typename T, typename G, typename A>
__global__ void __launch_bounds__(kBwdThreads) bwd_epilogue(const BwdArgs a) {
  __shared__ A red[kBwdThreads / 32][kBwdEpiChunk];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t rows = static_cast<int64_t>(a.batch) * a.ctx;
  const int d = a.feat, C = a.ctx;
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * kBwdEpiRows + warp * (kBwdEpiRows / 8);
  const A* num = static_cast<const A*>(a.num);
  const A* den = static_cast<const A*>(a.den);
  const T* bias = static_cast<const T*>(a.bias);
  const T* zl = static_cast<const T*>(a.z_tl);
  const T* go = static_cast<const T*>(a.gout);
  G* dnum = static_cast<G*>(a.dnum);
  T* gzl = static_cast<T*>(a.gz_tl);
  A dd[kBwdEpiRows / 8];
#pragma unroll
  for (int k = 0; k < kBwdEpiRows / 8; ++k) dd[k] = 0;
  for (int f0 = 0; f0 < d; f0 += kBwdEpiChunk) {
    A db[kBwdEpiChunk / 32];
#pragma unroll
    for (int q = 0; q < kBwdEpiChunk / 32; ++q) db[q] = 0;
#pragma unroll
    for (int k = 0; k < kBwdEpiRows / 8; ++k) {
      const int64_t r = r0 + k;
      if (r >= rows) break;
      const int b = static_cast<int>(r / C), n = static_cast<int>(r % C);
      const bool ok = row_valid(a, b, n);
      const A dn = a.normalize ? den[r] : A(1);
      const T* gor = go + static_cast<int64_t>(b) * a.go_bs + static_cast<int64_t>(n) * a.go_rs;
      const T* zlr = zl ? zl + static_cast<int64_t>(b) * a.zl_bs + static_cast<int64_t>(n) * a.zl_rs
                        : nullptr;
#pragma unroll
      for (int q = 0; q < kBwdEpiChunk / 32; ++q) {
        const int f = f0 + 32 * q + lane;
        if (f >= d) break;
        const A y0 = num[r * d + f] / dn;
        const A ypre = y0 + (bias ? ld_as<A>(bias + f) : A(0));
        const A g = ok ? ld_as<A>(gor + f) : A(0);
        A da = g;
        if (zlr) {
          const A gate = ok ? ld_as<A>(zlr + f) : A(0);
          if (gzl) st_as<T>(gzl + grad_off(a, b, n) + f, ok ? g * activate(ypre, a.act) : A(0));
          da = g * gate;
        }
        const A dy = ok ? da * activate_grad(ypre, a.act) : A(0);
        st_as<G>(dnum + r * d + f, dy / dn);
        dd[k] += dy * y0;
        db[q] += dy;
      }
    }
#pragma unroll
    for (int q = 0; q < kBwdEpiChunk / 32; ++q) red[warp][32 * q + lane] = db[q];
    __syncthreads();
    {
      const int f = f0 + threadIdx.x;
      if (threadIdx.x < kBwdEpiChunk && f < d) {
        A t = 0;
#pragma unroll
        for (int w = 0; w < kBwdThreads / 32; ++w) t += red[w][threadIdx.x];
        static_cast<A*>(a.part)[static_cast<int64_t>(blockIdx.x) * d + f] = t;
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int k = 0; k < kBwdEpiRows / 8; ++k) {
    const int64_t r = r0 + k;
    const A t = warp_sum(dd[k]);
    if (lane == 0 && r < rows)
      static_cast<A*>(a.dden)[r] = a.normalize ? -t / static_cast<const A*>(a.den)[r] : A(0);
  }
}

// Step 4: dS = (dnum Z^T + dden) (.) M, dGsym = (dG + dG^T) diag(r) with
// dG = dS (.) V, and the partial dV = sum over a group of batch rows of
// dS (.) G (G = r_i r_j Gr). A block
// owns a pair of 32 x 32 tiles (I, J), (J, I) with I <= J, so both halves of
// the symmetrised sum are formed in one place (through shared memory), and
// loops over its group of batch rows; blockIdx.y picks the group.
template <typename T, typename G, typename A>
__global__ void __launch_bounds__(kBwdThreads) bwd_dscores(const BwdArgs a, int bpg) {
  __shared__ A tr[kBwdTile][kBwdTile + 1];
  __shared__ A ts[kBwdTile][kBwdTile + 1];
  // Per batch row: r and key validity of the positions I0 + t and J0 + t.
  __shared__ A rs[2][kBwdTile];
  __shared__ int vs[2][kBwdTile];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int C = a.ctx;
  // Pair index -> (I, J), I <= J: row I holds pairs J = I .. nt-1.
  const int nt = (C + kBwdTile - 1) / kBwdTile;
  int p = blockIdx.x, I = 0;
  while (p >= nt - I) {
    p -= nt - I;
    ++I;
  }
  const int J = I + p;
  const bool diag = I == J;
  const int b0 = blockIdx.y * bpg, b1 = min(a.batch, b0 + bpg);
  const A* ds0 = static_cast<const A*>(a.ds0);
  const A* gr = static_cast<const A*>(a.g);
  const A* dden = static_cast<const A*>(a.dden);
  const T* v = static_cast<const T*>(a.v);
  G* dgs = static_cast<G*>(a.dgsym);
  constexpr int kR = kBwdTile / 8;
  // (i, j) of tile (I, J) and (i2, j2) of tile (J, I) for this thread.
  A vij[kR], vji[kR], acc1[kR], acc2[kR];
#pragma unroll
  for (int k = 0; k < kR; ++k) {
    const int i = I * kBwdTile + ty + 8 * k, j = J * kBwdTile + tx;
    const int i2 = J * kBwdTile + ty + 8 * k, j2 = I * kBwdTile + tx;
    vij[k] = (v && i < C && j < C) ? ld_as<A>(v + static_cast<int64_t>(i) * a.v_rs + j) : A(1);
    vji[k] = (v && i2 < C && j2 < C) ? ld_as<A>(v + static_cast<int64_t>(i2) * a.v_rs + j2) : A(1);
    acc1[k] = acc2[k] = 0;
  }
  for (int b = b0; b < b1; ++b) {
    const int64_t base = static_cast<int64_t>(b) * C * C;
    const int64_t rb = static_cast<int64_t>(b) * C;  // first row of batch b
    if (threadIdx.x < 2 * kBwdTile) {
      const int side = threadIdx.x / kBwdTile, t = threadIdx.x % kBwdTile;
      const int pos = (side ? J : I) * kBwdTile + t;
      rs[side][t] = pos < C ? inv_norm<A>(a, rb + pos) : A(0);
      vs[side][t] = pos < C && row_valid(a, b, pos);
    }
    __syncthreads();
    // r of the key columns of both tiles: J0 + tx and I0 + tx.
    const A rj1 = rs[1][tx], rj2 = rs[0][tx];
    const bool vj1 = vs[1][tx] != 0, vj2 = vs[0][tx] != 0;
    A dg1[kR];
#pragma unroll
    for (int k = 0; k < kR; ++k) {
      const int i = I * kBwdTile + ty + 8 * k, j = J * kBwdTile + tx;
      A x = 0;
      if (i < C && j < C && (!a.causal || j <= i) && vj1) {
        x = ds0[base + static_cast<int64_t>(i) * C + j];
        if (a.normalize) x += dden[rb + i];
        if (a.gv) acc1[k] += x * gr[base + static_cast<int64_t>(i) * C + j] * rs[0][ty + 8 * k] * rj1;
      }
      dg1[k] = x * vij[k];
      if (!diag) {
        const int i2 = J * kBwdTile + ty + 8 * k, j2 = I * kBwdTile + tx;
        A y = 0;
        if (i2 < C && j2 < C && (!a.causal || j2 <= i2) && vj2) {
          y = ds0[base + static_cast<int64_t>(i2) * C + j2];
          if (a.normalize) y += dden[rb + i2];
          if (a.gv) acc2[k] += y * gr[base + static_cast<int64_t>(i2) * C + j2] * rs[1][ty + 8 * k] * rj2;
        }
        tr[ty + 8 * k][tx] = y * vji[k];  // dG of tile (J, I) at (i2 - J0, j2 - I0)
      } else {
        tr[ty + 8 * k][tx] = dg1[k];
      }
    }
    __syncthreads();
    // dGsym (I, J)[r][c] = dG(I, J)[r][c] + dG(J, I)[c][r], stored with its
    // column scaled by r of that key.
#pragma unroll
    for (int k = 0; k < kR; ++k) {
      const int rr = ty + 8 * k;
      const int i = I * kBwdTile + rr, j = J * kBwdTile + tx;
      const A sym = dg1[k] + tr[tx][rr];
      ts[rr][tx] = sym;
      if (i < C && j < C) st_as<G>(dgs + base + static_cast<int64_t>(i) * C + j, sym * rj1);
    }
    __syncthreads();
    if (!diag) {
      // Tile (J, I) is the transpose of tile (I, J).
#pragma unroll
      for (int k = 0; k < kR; ++k) {
        const int rr = ty + 8 * k;
        const int i2 = J * kBwdTile + rr, j2 = I * kBwdTile + tx;
        if (i2 < C && j2 < C)
          st_as<G>(dgs + base + static_cast<int64_t>(i2) * C + j2, ts[tx][rr] * rj2);
      }
    }
    __syncthreads();
  }
  if (a.gv) {
    A* part = static_cast<A*>(a.part) + static_cast<int64_t>(blockIdx.y) * C * C;
#pragma unroll
    for (int k = 0; k < kR; ++k) {
      const int i = I * kBwdTile + ty + 8 * k, j = J * kBwdTile + tx;
      if (i < C && j < C) part[static_cast<int64_t>(i) * C + j] = acc1[k];
      if (!diag) {
        const int i2 = J * kBwdTile + ty + 8 * k, j2 = I * kBwdTile + tx;
        if (i2 < C && j2 < C) part[static_cast<int64_t>(i2) * C + j2] = acc2[k];
      }
    }
  }
}

// Step 5: dZ = S^T dnum + the normalisation backward of dz^, zero on padded
// rows, in the input type. One warp per row.
template <typename T, typename G, typename A>
__global__ void __launch_bounds__(kBwdThreads) bwd_final(const BwdArgs a) {
  const int lane = threadIdx.x & 31;
  const int64_t rows = static_cast<int64_t>(a.batch) * a.ctx;
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * (kBwdThreads / 32);
  const int d = a.feat;
  const A* dzh = static_cast<const A*>(a.dzh);
  const A* dzd = static_cast<const A*>(a.dzd);
  T* gz = static_cast<T*>(a.gz_tr);
  for (int64_t r = (static_cast<int64_t>(blockIdx.x) * kBwdThreads + threadIdx.x) >> 5; r < rows;
       r += nwarps) {
    const int b = static_cast<int>(r / a.ctx), n = static_cast<int>(r % a.ctx);
    const G* zr = zm_row<G>(a, r, b, n);
    const bool ok = row_valid(a, b, n);
    const A norm = static_cast<const A*>(a.norms)[r];
    const A ne = static_cast<A>(a.norm_eps);
    const bool scaled = norm >= ne;  // F.normalize divides by the norm itself
    const A rinv = A(1) / (scaled ? norm : ne);
    A dot = 0;
    if (ok && scaled)
      for (int f = lane; f < d; f += 32) dot += ld_as<A>(zr + f) * rinv * dzh[r * d + f];
    dot = warp_sum(dot);
    for (int f = lane; f < d; f += 32) {
      A g = 0;
      if (ok) {
        const A zhat = ld_as<A>(zr + f) * rinv;
        g = (dzh[r * d + f] - (scaled ? zhat * dot : A(0))) * rinv + dzd[r * d + f];
      }
      st_as<T>(gz + grad_off(a, b, n) + f, g);
    }
  }
}

// ---------------------------------------------------------------------------
// Vector forms of steps 1, 2, 3 and 5 (fp32 accumulation; bf16, fp16 and fp32
// inputs): every lane moves 8 consecutive elements per access (16-byte loads
// and stores of 16-bit data, two of fp32). The host picks them when the row
// lengths are multiples of 8 and every strided row starts 16-byte aligned.

template <typename T>
__device__ __forceinline__ void ld8(const T* p, float (&v)[8]);
template <>
__device__ __forceinline__ void ld8<__nv_bfloat16>(const __nv_bfloat16* p, float (&v)[8]) {
  const uint4 q = __ldg(reinterpret_cast<const uint4*>(p));
  const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    v[2 * e] = __uint_as_float(w[e] << 16);
    v[2 * e + 1] = __uint_as_float(w[e] & 0xFFFF0000u);
  }
}
template <>
__device__ __forceinline__ void ld8<__half>(const __half* p, float (&v)[8]) {
  const uint4 q = __ldg(reinterpret_cast<const uint4*>(p));
  const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[e]));
    v[2 * e] = f.x;
    v[2 * e + 1] = f.y;
  }
}
template <>
__device__ __forceinline__ void ld8<float>(const float* p, float (&v)[8]) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(p));
  const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

template <typename T>
__device__ __forceinline__ void st8(T* p, const float (&v)[8]);
template <>
__device__ __forceinline__ void st8<__nv_bfloat16>(__nv_bfloat16* p, const float (&v)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    __nv_bfloat162 h = __floats2bfloat162_rn(v[2 * e], v[2 * e + 1]);
    w[e] = *reinterpret_cast<uint32_t*>(&h);
  }
  *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
}
template <>
__device__ __forceinline__ void st8<__half>(__half* p, const float (&v)[8]) {
  uint32_t w[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    __half2 h = __floats2half2_rn(v[2 * e], v[2 * e + 1]);
    w[e] = *reinterpret_cast<uint32_t*>(&h);
  }
  *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
}
template <>
__device__ __forceinline__ void st8<float>(float* p, const float (&v)[8]) {
  reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
  reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
}

// Step 1, vector form.
template <typename T, typename G>
__global__ void __launch_bounds__(kBwdThreads) bwd_prep_v8(const BwdArgs a) {
  const int lane = threadIdx.x & 31;
  const int64_t rows = static_cast<int64_t>(a.batch) * a.ctx;
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * (kBwdThreads / 32);
  const int nv = a.feat / 8;
  const T* __restrict__ z = static_cast<const T*>(a.z_tr);
  G* __restrict__ zm = static_cast<G*>(a.zm);
  for (int64_t r = (static_cast<int64_t>(blockIdx.x) * kBwdThreads + threadIdx.x) >> 5; r < rows;
       r += nwarps) {
    const int b = static_cast<int>(r / a.ctx), n = static_cast<int>(r % a.ctx);
    const bool ok = row_valid(a, b, n);
    const T* zr = z + static_cast<int64_t>(b) * a.zr_bs + static_cast<int64_t>(n) * a.zr_rs;
    float ss = 0.f;
    for (int v = lane; v < nv; v += 32) {
      float x[8];
      if (ok) {
        ld8<T>(zr + 8 * v, x);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) x[e] = 0.f;
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) ss = fmaf(x[e], x[e], ss);
      if (zm) st8<G>(zm + r * a.feat + 8 * v, x);
    }
    ss = warp_sum(ss);
    if (lane == 0) static_cast<float*>(a.norms)[r] = ok ? sqrtf(ss) : -1.f;  // -1 marks padding
  }
}

// Step 2, vector form: a lane takes 8 consecutive keys.
template <typename T, typename G>
__global__ void __launch_bounds__(kBwdThreads) bwd_scores_v8(const BwdArgs a) {
  const int lane = threadIdx.x & 31;
  const int64_t rows = static_cast<int64_t>(a.batch) * a.ctx;
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * (kBwdThreads / 32);
  const int C = a.ctx;
  const float* __restrict__ gr = static_cast<const float*>(a.g);
  const float* __restrict__ norms = static_cast<const float*>(a.norms);
  G* __restrict__ s = static_cast<G*>(a.s);
  const T* __restrict__ v = static_cast<const T*>(a.v);
  const float ne = static_cast<float>(a.norm_eps);
  for (int64_t r = (static_cast<int64_t>(blockIdx.x) * kBwdThreads + threadIdx.x) >> 5; r < rows;
       r += nwarps) {
    const int b = static_cast<int>(r / C), i = static_cast<int>(r % C);
    const float ri = 1.f / fmaxf(norms[r], ne);
    const float* nb = norms + static_cast<int64_t>(b) * C;
    float sum = 0.f;
    for (int j0 = 8 * lane; j0 < C; j0 += 256) {
      float x[8], nk[8], vv[8];
      if (a.causal && j0 > i) {  // every key of the vector lies after the query
#pragma unroll
        for (int e = 0; e < 8; ++e) x[e] = 0.f;
        st8<G>(s + r * C + j0, x);
        continue;
      }
      ld8<float>(gr + r * C + j0, x);
      ld8<float>(nb + j0, nk);
      if (v) ld8<T>(v + static_cast<int64_t>(i) * a.v_rs + j0, vv);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int j = j0 + e;
        const bool allowed = (!a.causal || j <= i) && nk[e] >= 0.f;  // padding has norm -1
        float y = x[e] * ri * (1.f / fmaxf(nk[e], ne));
        if (v) y *= vv[e];
        x[e] = allowed ? y : 0.f;
        sum += x[e];
      }
      st8<G>(s + r * C + j0, x);
    }
    sum = warp_sum(sum);
    if (lane == 0) static_cast<float*>(a.den)[r] = sum + static_cast<float>(a.eps);
  }
}

// Step 3, vector form: a warp takes kBwdEpiRowsV8 rows, a lane 8 consecutive
// features of up to S slots (256 S features) per pass, keeping its dbias
// partial sums in registers across the rows; the block sums its 8 warps in
// order. The activation and S (2 or 3, the host picks the fewest passes) are
// template parameters. dden is accumulated in place (one warp owns a row) and
// finished after the last pass.
constexpr int kBwdEpiMaxSlots = 3;
constexpr int kBwdEpiRowsV8 = 32;  // rows per block (4 per warp)

template <int ACT>
__device__ __forceinline__ float act_grad_fn(float x) {
  if constexpr (ACT == 1) {
    return x > 0.f ? 1.f : 0.f;
  } else if constexpr (ACT == 2) {
    return x > 0.f ? 2.f * x : 0.f;
  } else if constexpr (ACT == 3) {
    const float sg = sigmoid_stable(x);
    return sg * (1.f + x * (1.f - sg));
  } else if constexpr (ACT == 4) {
    const float k = 0.7978845608028654f, c = 0.044715f;
    const float t = tanhf(k * (x + c * x * x * x));
    return 0.5f * (1.f + t) + 0.5f * x * (1.f - t * t) * k * (1.f + 3.f * c * x * x);
  } else {
    return 1.f;
  }
}

// Three blocks per SM (at most 85 registers a thread): each warp has one row's
// loads in flight at a time, so the kernel needs the warps to cover HBM latency
// (96 registers and two blocks per SM measured ~9 us slower on config 2).
template <typename T, typename G, int ACT, int S>
__global__ void __launch_bounds__(kBwdThreads, 3) bwd_epilogue_v8(const BwdArgs a) {
  static_assert(S >= 1 && S <= kBwdEpiMaxSlots, "feature slots per pass");
  __shared__ float red[kBwdThreads / 32][S * 256];
  constexpr int kRows = kBwdEpiRowsV8 / (kBwdThreads / 32);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t rows = static_cast<int64_t>(a.batch) * a.ctx;
  const int d = a.feat, C = a.ctx, nv = d / 8;
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * kBwdEpiRowsV8 + warp * kRows;
  const float* __restrict__ num = static_cast<const float*>(a.num);
  const float* __restrict__ den = static_cast<const float*>(a.den);
  float* __restrict__ dden = static_cast<float*>(a.dden);
  const T* __restrict__ bias = static_cast<const T*>(a.bias);
  const T* __restrict__ zl = static_cast<const T*>(a.z_tl);
  const T* __restrict__ go = static_cast<const T*>(a.gout);
  G* __restrict__ dnum = static_cast<G*>(a.dnum);
  T* __restrict__ gzl = static_cast<T*>(a.gz_tl);
  for (int w0 = 0; w0 < nv; w0 += 32 * S) {
    float db[S][8];
#pragma unroll
    for (int q = 0; q < S; ++q)
#pragma unroll
      for (int e = 0; e < 8; ++e) db[q][e] = 0.f;
#pragma unroll 1
    for (int k = 0; k < kRows; ++k) {
      const int64_t r = r0 + k;
      if (r >= rows) break;
      const int b = static_cast<int>(r / C), n = static_cast<int>(r % C);
      const bool ok = row_valid(a, b, n);
      const float dn = a.normalize ? den[r] : 1.f;
      const float rdn = 1.f / dn;
      const T* gor = go + static_cast<int64_t>(b) * a.go_bs + static_cast<int64_t>(n) * a.go_rs;
      const T* zlr = zl ? zl + static_cast<int64_t>(b) * a.zl_bs + static_cast<int64_t>(n) * a.zl_rs
                        : nullptr;
      float dsum = 0.f;
#pragma unroll
      for (int q = 0; q < S; ++q) {
        const int v = w0 + 32 * q + lane;
        if (v >= nv) break;
        const int f0 = 8 * v;
        float nm[8], g[8], bb[8], gt[8], dy[8], dz[8];
        ld8<float>(num + r * d + f0, nm);
        if (ok) {
          ld8<T>(gor + f0, g);
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e) g[e] = 0.f;
        }
        if (bias) {
          ld8<T>(bias + f0, bb);
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e) bb[e] = 0.f;
        }
        if (zlr && ok) {
          ld8<T>(zlr + f0, gt);
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e) gt[e] = zlr ? 0.f : 1.f;
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float y0 = nm[e] * rdn;
          const float ypre = y0 + bb[e];
          dz[e] = ok ? g[e] * act_fn<ACT>(ypre) : 0.f;
          dy[e] = ok ? g[e] * gt[e] * act_grad_fn<ACT>(ypre) : 0.f;
          dsum = fmaf(dy[e], y0, dsum);
          db[q][e] += dy[e];
          dy[e] *= rdn;
        }
        if (gzl) st8<T>(gzl + grad_off(a, b, n) + f0, dz);
        st8<G>(dnum + r * d + f0, dy);
      }
      dsum = warp_sum(dsum);
      if (lane == 0) dden[r] = (w0 == 0 ? 0.f : dden[r]) + dsum;
    }
#pragma unroll
    for (int q = 0; q < S; ++q)
#pragma unroll
      for (int e = 0; e < 8; ++e) red[warp][(32 * q + lane) * 8 + e] = db[q][e];
    __syncthreads();
    for (int t = threadIdx.x; t < S * 256; t += kBwdThreads) {
      const int f = 8 * w0 + t;
      if (f < d) {
        float acc = 0.f;
#pragma unroll
        for (int w = 0; w < kBwdThreads / 32; ++w) acc += red[w][t];
        static_cast<float*>(a.part)[static_cast<int64_t>(blockIdx.x) * d + f] = acc;
      }
    }
    __syncthreads();
  }
  if (lane == 0)
    for (int k = 0; k < kRows; ++k) {
      const int64_t r = r0 + k;
      if (r < rows) dden[r] = a.normalize ? -dden[r] / den[r] : 0.f;
    }
}

// Step 5, vector form.
template <typename T, typename G>
__global__ void __launch_bounds__(kBwdThreads) bwd_final_v8(const BwdArgs a) {
  const int lane = threadIdx.x & 31;
  const int64_t rows = static_cast<int64_t>(a.batch) * a.ctx;
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * (kBwdThreads / 32);
  const int d = a.feat, nv = d / 8;
  const float* __restrict__ dzh = static_cast<const float*>(a.dzh);
  const float* __restrict__ dzd = static_cast<const float*>(a.dzd);
  T* __restrict__ gz = static_cast<T*>(a.gz_tr);
  const float ne = static_cast<float>(a.norm_eps);
  for (int64_t r = (static_cast<int64_t>(blockIdx.x) * kBwdThreads + threadIdx.x) >> 5; r < rows;
       r += nwarps) {
    const int b = static_cast<int>(r / a.ctx), n = static_cast<int>(r % a.ctx);
    const G* __restrict__ zr = zm_row<G>(a, r, b, n);
    const float norm = static_cast<const float*>(a.norms)[r];
    const bool ok = norm >= 0.f;  // padding has norm -1
    const bool scaled = norm >= ne;
    const float rinv = 1.f / (scaled ? norm : ne);
    float dot = 0.f;
    if (ok && scaled)
      for (int v = lane; v < nv; v += 32) {
        float z[8], h[8];
        ld8<G>(zr + 8 * v, z);
        ld8<float>(dzh + r * d + 8 * v, h);
#pragma unroll
        for (int e = 0; e < 8; ++e) dot = fmaf(z[e] * rinv, h[e], dot);
      }
    dot = warp_sum(dot);
    for (int v = lane; v < nv; v += 32) {
      float o[8];
      if (ok) {
        float z[8], h[8], dd[8];
        ld8<G>(zr + 8 * v, z);
        ld8<float>(dzh + r * d + 8 * v, h);
        ld8<float>(dzd + r * d + 8 * v, dd);
#pragma unroll
        for (int e = 0; e < 8; ++e)
          o[e] = (h[e] - (scaled ? z[e] * rinv * dot : 0.f)) * rinv + dd[e];
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = 0.f;
      }
      st8<T>(gz + grad_off(a, b, n) + 8 * v, o);
    }
  }
}

template <typename G>
__device__ __forceinline__ void st4(G* p, const float (&v)[4]);
template <>
__device__ __forceinline__ void st4<__nv_bfloat16>(__nv_bfloat16* p, const float (&v)[4]) {
  __nv_bfloat162 lo = __floats2bfloat162_rn(v[0], v[1]), hi = __floats2bfloat162_rn(v[2], v[3]);
  *reinterpret_cast<uint2*>(p) =
      make_uint2(*reinterpret_cast<uint32_t*>(&lo), *reinterpret_cast<uint32_t*>(&hi));
}
template <>
__device__ __forceinline__ void st4<float>(float* p, const float (&v)[4]) {
  *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
}

// Step 4, vector form (fp32 accumulation, contexts a multiple of 8): a thread
// owns 4 consecutive columns of one row of each tile (float4 loads), the
// next batch row's operands are loaded while the current one is computed,
// the transposes go through double-buffered shared tiles (two barriers per
// batch row), and the norms and key validity come straight from global memory.
struct DsIn {
  float4 ds, g, nk;  // ds0 and Gr of 4 columns, norms of their keys
  float nq, dd;      // norm of the row's query, its dden
};

// dG of 4 columns (j .. j+3) of query row i, the dV partial sums, and r of
// the 4 keys.
__device__ __forceinline__ void ds_compute(const BwdArgs& a, const DsIn& x, int b, int i, int j,
                                           bool in, const float (&v)[4], float (&acc)[4],
                                           float (&dg)[4], float (&rk)[4]) {
  const float ne = static_cast<float>(a.norm_eps);
  const float xs[4] = {x.ds.x, x.ds.y, x.ds.z, x.ds.w};
  const float gs[4] = {x.g.x, x.g.y, x.g.z, x.g.w};
  const float ns[4] = {x.nk.x, x.nk.y, x.nk.z, x.nk.w};
  const float rq = 1.f / fmaxf(x.nq, ne);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    rk[e] = in ? 1.f / fmaxf(ns[e], ne) : 0.f;
    const bool ok = in && (!a.causal || j + e <= i) && ns[e] >= 0.f;  // padding has norm -1
    const float dsm = ok ? xs[e] + x.dd : 0.f;
    // Selected, not multiplied by zero: under the causal mask the tiles of Gr
    // and ds0 above the diagonal may be left unwritten by their GEMMs.
    if (ok) acc[e] = fmaf(dsm, gs[e] * rq * rk[e], acc[e]);
    dg[e] = dsm * v[e];
  }
}

// cp.async copies of 16 / 4 bytes from global to shared memory (completion
// tracked per thread by commit / wait groups).
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
               "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(dst))),
               "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// One batch row's two large operands of one dscores tile (ds0 and Gr, 4 KB
// each), field by field so that the threads' 16-byte slots are contiguous
// (conflict-free float4 reads). The small per-row operands (key norms, query
// norm, dden) go through registers, loaded one batch row ahead.
struct DsStage {
  float4 ds[kBwdThreads];
  float4 g[kBwdThreads];
};
constexpr int kDsStages = 3;

struct DsSmall {
  float4 nk;      // norms of the 4 keys
  float nq, dd;   // norm of the query, its dden
};

__device__ __forceinline__ DsSmall ds_small(const BwdArgs& a, int64_t rb, int i, int j, bool in) {
  DsSmall x;
  x.nk = make_float4(0.f, 0.f, 0.f, 0.f);
  x.nq = 1.f;
  x.dd = 0.f;
  if (in) {
    const float* nrm = static_cast<const float*>(a.norms);
    x.nk = __ldg(reinterpret_cast<const float4*>(nrm + rb + j));
    x.nq = __ldg(nrm + rb + i);
    if (a.normalize) x.dd = __ldg(static_cast<const float*>(a.dden) + rb + i);
  }
  return x;
}

// Issue the copies of this thread's operands of tile row i, columns j..j+3.
__device__ __forceinline__ void ds_issue(const BwdArgs& a, DsStage& st, int64_t base, int i, int j,
                                         bool in, bool want_g) {
  const int t = threadIdx.x;
  if (!in) return;
  const int64_t off = base + static_cast<int64_t>(i) * a.ctx + j;
  cp_async16(&st.ds[t], static_cast<const float*>(a.ds0) + off);
  if (want_g) cp_async16(&st.g[t], static_cast<const float*>(a.g) + off);
}

__device__ __forceinline__ DsIn ds_read(const DsStage& st, const DsSmall& sm, bool in, bool want_g) {
  const int t = threadIdx.x;
  DsIn x;
  x.ds = x.g = make_float4(0.f, 0.f, 0.f, 0.f);
  x.nk = sm.nk;
  x.nq = sm.nq;
  x.dd = sm.dd;
  if (in) {
    x.ds = st.ds[t];
    if (want_g) x.g = st.g[t];
  }
  return x;
}

template <typename T, typename G>
__global__ void __launch_bounds__(kBwdThreads, 3) bwd_dscores_v4(const BwdArgs a, int bpg) {
  __shared__ float tr[2][kBwdTile][kBwdTile + 1];
  __shared__ float ts[2][kBwdTile][kBwdTile + 1];
  const int row = threadIdx.x >> 3, c4 = (threadIdx.x & 7) * 4;
  const int C = a.ctx;
  const int nt = C / kBwdTile + (C % kBwdTile ? 1 : 0);
  int p = blockIdx.x, I = 0;
  while (p >= nt - I) {
    p -= nt - I;
    ++I;
  }
  const int J = I + p;
  const bool diag = I == J;
  const int I0 = I * kBwdTile, J0 = J * kBwdTile;
  const int b0 = blockIdx.y * bpg, b1 = min(a.batch, b0 + bpg);
  const T* v = static_cast<const T*>(a.v);
  G* dgs = static_cast<G*>(a.dgsym);
  const bool want_g = a.gv != nullptr;
  // Tile (I, J): row i1 = I0 + row, columns j1 = J0 + c4 + e. Tile (J, I):
  // row i2 = J0 + row, columns j2 = I0 + c4 + e. Four columns are in range
  // together (C is a multiple of 8, tiles start at multiples of 32).
  const int i1 = I0 + row, i2 = J0 + row, j1 = J0 + c4, j2 = I0 + c4;
  const bool in1 = i1 < C && j1 < C, in2 = !diag && i2 < C && j2 < C;
  float v1[4], v2[4], acc1[4] = {0.f, 0.f, 0.f, 0.f}, acc2[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    v1[e] = (v && in1) ? ld_as<float>(v + static_cast<int64_t>(i1) * a.v_rs + j1 + e) : 1.f;
    v2[e] = (v && in2) ? ld_as<float>(v + static_cast<int64_t>(i2) * a.v_rs + j2 + e) : 1.f;
  }
  // Operands stream through a kDsStages-deep shared-memory ring filled with
  // cp.async: each thread copies and later reads only its own slots, so the
  // ring needs no block barrier, and the loads of later batch rows are in
  // flight while this one is computed.
  extern __shared__ __align__(16) uint8_t ds_smem[];
  DsStage* ring1 = reinterpret_cast<DsStage*>(ds_smem);
  DsStage* ring2 = ring1 + kDsStages;
  const int nb = b1 - b0;
#pragma unroll
  for (int k = 0; k < kDsStages - 1; ++k) {
    if (k < nb) {
      const int64_t base = static_cast<int64_t>(b0 + k) * C * C;
      ds_issue(a, ring1[k], base, i1, j1, in1, want_g);
      ds_issue(a, ring2[k], base, i2, j2, in2, want_g);
    }
    cp_async_commit();
  }
  DsSmall s1 = ds_small(a, static_cast<int64_t>(b0) * C, i1, j1, in1 && nb > 0);
  DsSmall s2 = ds_small(a, static_cast<int64_t>(b0) * C, i2, j2, in2 && nb > 0);
  int buf = 0;
  for (int it = 0; it < nb; ++it, buf ^= 1) {
    const int b = b0 + it;
    const int64_t base = static_cast<int64_t>(b) * C * C;
    {
      const int ahead = it + kDsStages - 1;
      if (ahead < nb) {
        const int64_t abase = static_cast<int64_t>(b0 + ahead) * C * C;
        ds_issue(a, ring1[ahead % kDsStages], abase, i1, j1, in1, want_g);
        ds_issue(a, ring2[ahead % kDsStages], abase, i2, j2, in2, want_g);
      }
      cp_async_commit();
    }
    // The next batch row's small operands, in flight while this row is computed.
    const bool more = it + 1 < nb;
    const DsSmall n1 = ds_small(a, static_cast<int64_t>(b + 1) * C, i1, j1, in1 && more);
    const DsSmall n2 = ds_small(a, static_cast<int64_t>(b + 1) * C, i2, j2, in2 && more);
    cp_async_wait<kDsStages - 1>();  // this batch row's group has landed
    const DsIn x1 = ds_read(ring1[it % kDsStages], s1, in1, want_g);
    const DsIn x2 = ds_read(ring2[it % kDsStages], s2, in2, want_g);
    s1 = n1;
    s2 = n2;
    float dg1[4], r1[4], dg2[4], r2[4];
    ds_compute(a, x1, b, i1, j1, in1, v1, acc1, dg1, r1);
    if (!diag) {
      ds_compute(a, x2, b, i2, j2, in2, v2, acc2, dg2, r2);
#pragma unroll
      for (int e = 0; e < 4; ++e) tr[buf][row][c4 + e] = dg2[e];
    } else {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        tr[buf][row][c4 + e] = dg1[e];
        r2[e] = r1[e];
      }
    }
    __syncthreads();
    // dGsym (I, J)[row][c] = dG(I, J)[row][c] + dG(J, I)[c][row], column c
    // scaled by r of key J0 + c.
    float sym[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      sym[e] = dg1[e] + tr[buf][c4 + e][row];
      ts[buf][row][c4 + e] = sym[e];
      sym[e] *= r1[e];
    }
    if (in1) st4<G>(dgs + base + static_cast<int64_t>(i1) * C + j1, sym);
    __syncthreads();
    if (in2) {
      // Tile (J, I) is the transpose of tile (I, J); column c scaled by r of
      // key I0 + c.
      float t4[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) t4[e] = ts[buf][c4 + e][row] * r2[e];
      st4<G>(dgs + base + static_cast<int64_t>(i2) * C + j2, t4);
    }
  }
  if (want_g) {
    float* part = static_cast<float*>(a.part) + static_cast<int64_t>(blockIdx.y) * C * C;
    if (in1)
      *reinterpret_cast<float4*>(part + static_cast<int64_t>(i1) * C + j1) =
          make_float4(acc1[0], acc1[1], acc1[2], acc1[3]);
    if (in2)
      *reinterpret_cast<float4*>(part + static_cast<int64_t>(i2) * C + j2) =
          make_float4(acc2[0], acc2[1], acc2[2], acc2[3]);
  }
}

// out[k] = sum over p of part[p][k], p in order: the warps of a block take
// interleaved p (as many warps as parts, up to 32), then combine in warp
// order: deterministic.
constexpr int kBwdReduceThreads = 1024;
template <typename T, typename A>
__global__ void __launch_bounds__(kBwdReduceThreads) bwd_reduce(const A* part, int nparts,
                                                                int64_t n, T* out) {
  __shared__ A red[kBwdReduceThreads / 32][32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const int64_t k = static_cast<int64_t>(blockIdx.x) * 32 + lane;
  A t = 0;
  if (k < n) {
    int p = warp;
    for (; p + 7 * nw < nparts; p += 8 * nw) {  // eight loads in flight, added in order
      A v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = part[static_cast<int64_t>(p + u * nw) * n + k];
#pragma unroll
      for (int u = 0; u < 8; ++u) t += v[u];
    }
    for (; p < nparts; p += nw) t += part[static_cast<int64_t>(p) * n + k];
  }
  red[warp][lane] = t;
  __syncthreads();
  if (warp == 0 && k < n) {
    A s = 0;
    for (int w = 0; w < nw; ++w) s += red[w][lane];
    st_as<T>(out + k, s);
  }
}

// The same sums for many columns of at most 32 parts (dV: C x C columns, one
// part per batch group): one thread per column adds the parts in order, eight
// loads in flight. For nparts <= 32 bwd_reduce adds in the same order (one part
// per warp, warps combined in order), so the two forms give the same bits.
constexpr int kBwdReduceColThreads = 256;
template <typename T, typename A>
__global__ void __launch_bounds__(kBwdReduceColThreads) bwd_reduce_cols(const A* part, int nparts,
                                                                        int64_t n, T* out) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kBwdReduceColThreads;
  for (int64_t k = static_cast<int64_t>(blockIdx.x) * kBwdReduceColThreads + threadIdx.x; k < n;
       k += stride) {
    A t = 0;
    int p = 0;
    for (; p + 8 <= nparts; p += 8) {
      A v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = part[static_cast<int64_t>(p + u) * n + k];
#pragma unroll
      for (int u = 0; u < 8; ++u) t += v[u];
    }
    for (; p < nparts; ++p) t += part[static_cast<int64_t>(p) * n + k];
    st_as<T>(out + k, t);
  }
}

}  // namespace avey
