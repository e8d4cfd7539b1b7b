// Batched tcgen05 matrix product for 16-bit operands (bf16 / f16) with fp32
// accumulation in tensor memory:
//
//   C[b] = A[b] B[b]                                  (fp32 output), or
//   C[b] = act(A[b] B[b] + bias) (.) gate[b]          (16-bit output)
//
// with A [m x k], B [k x n]. Each operand is K-major (k contiguous) or
// MN-major (m / n contiguous), so transposed operands need no copy, and an
// operand may be shared by every batch entry (batch stride 0). It serves:
//
//  * the backward pass of the contextualizer: its five contractions
//    (g = zm zm^T, num = s zm, ds0 = dnum zm^T, dzd = s^T dnum,
//    dzh = dgsym zm), with the causal structure of s used to skip work:
//    whole output tiles above the diagonal (kGemmLowerOut: only c[i][j] with
//    j <= i is consumed) and the zero part of a triangular A in the K loop
//    (kGemmKLower: A[i][k] = 0 for k > i; kGemmKUpper: A[i][k] = 0 for k < i);
//  * the enricher projection x W^T + bias with its activation, whose output
//    feeds the contextualizer, with partial row sums of squares of its tail
//    columns written from the epilogue (the contextualizer then needs no
//    pre-pass over z_tr);
//  * the static (position-wise or token-mixing) layers, with the gate.
//
// Structure: persistent CTAs (one per SM, tiles of 128 x 256 taken round
// robin), warp 0 issues TMA (4 stages of a 128 x 64 A tile and a 64 x 256 B
// tile, 128-byte swizzle), warp 1 issues tcgen05.mma (M = 128, N = 256, K = 16)
// into one of two 256-column TMEM accumulators, and warps 4-11 drain the other
// accumulator (thread = output row, 32 columns per tcgen05.ld) through
// per-warp staging tiles and TMA tensor stores, so a tile's epilogue overlaps
// the next tile's main loop. Every wait is bounded (ptx.cuh).
#pragma once

#include "tc_long.cuh"

namespace avey {

constexpr int kGmThreads = 384;
constexpr int kGmBM = 128, kGmBN = 256, kGmBK = 64;
constexpr int kGmStages = 4;
constexpr int kGmABytes = kGmBM * kGmBK * 2;         // 16 KB
constexpr int kGmBBytes = kGmBN * kGmBK * 2;         // 32 KB
constexpr int kGmStageBytes = kGmABytes + kGmBBytes;  // 48 KB
constexpr int kGmMnBox = 64 * kGmBK * 2;              // one {64 (m or n), 64 (k)} box: 8 KB
constexpr int kGmStageTile = 4096;  // a warp's staging tile: 32 x 32 fp32 (or two 32 x 32 16-bit)
constexpr int kGmCtrlBytes = 1024;
constexpr int kGmSmem = 1024 + kGmStages * kGmStageBytes + 8 * kGmStageTile + kGmCtrlBytes;

enum GemmMode { kGemmDense = 0, kGemmLowerOut = 1, kGemmKLower = 2, kGemmKUpper = 3 };

struct GemmGeom {
  int batch, m, n, k;
  int n_mt, n_nt;       // row and column tiles per batch entry
  int mode;             // GemmMode
  int a_mn, b_mn;       // operand is MN-major (else K-major)
  int a_batched, b_batched;
  int total_tiles;
  int has_bias, has_gate;
  int sumsq_col0;       // 16-bit output: first column of the row sums of squares (multiple of 128)
  const void* bias;     // [n], operand type
  const void* gate;     // [batch][m][n], operand type
  int64_t gate_bs, gate_rs;
  float* sumsq;         // planes [(n - col0) / 128][batch * m], or null
};

struct GemmCtrl {
  uint64_t full[kGmStages], empty[kGmStages];
  uint64_t acc_full[2], acc_empty[2];
  uint32_t tmem_base;
};
static_assert(sizeof(GemmCtrl) <= kGmCtrlBytes, "control block too large");

struct GemmTile {
  int b, mt, nt;
  int k0;  // first K block (of kGmBK)
  int nk;  // K blocks
};

// Output tiles per row tile: all of them, or under kGemmLowerOut those with a
// column at or below the tile's last row.
__device__ __forceinline__ int gemm_cols_of(const GemmGeom& g, int mt) {
  return g.mode == kGemmLowerOut ? min(g.n_nt, (mt * kGmBM + kGmBM - 1) / kGmBN + 1) : g.n_nt;
}

// Tile t of the launch: row tiles in order (the longest K ranges first under
// kGemmKLower), then batch entries, then column tiles, so neighbouring CTAs
// share the A row block.
__device__ __forceinline__ GemmTile gemm_tile(const GemmGeom& g, int t) {
  GemmTile c{0, 0, 0, 0, 0};
  int rem = t;
  for (int o = 0; o < g.n_mt; ++o) {
    const int mt = g.mode == kGemmKLower ? g.n_mt - 1 - o : o;
    const int cnt = gemm_cols_of(g, mt);
    const int per = cnt * g.batch;
    if (rem < per) {
      c.mt = mt;
      c.b = rem / cnt;
      c.nt = rem % cnt;
      break;
    }
    rem -= per;
  }
  int klo = 0, khi = g.k;
  if (g.mode == kGemmKLower) khi = min(g.k, (c.mt + 1) * kGmBM);
  if (g.mode == kGemmKUpper) klo = min(g.k, c.mt * kGmBM);
  c.k0 = klo / kGmBK;
  c.nk = khi > klo ? (khi - c.k0 * kGmBK + kGmBK - 1) / kGmBK : 0;
  return c;
}

__device__ __forceinline__ void st_stage_f32(uint32_t stage, int lane, const uint32_t (&o)[32]) {
  // 32 rows x 128 bytes with the 128-byte swizzle (16-byte chunk q of row r at q ^ (r % 8)).
#pragma unroll
  for (int q = 0; q < 8; ++q)
    st_shared_v4(stage + lane * 128 + ((q ^ (lane & 7)) << 4), o[4 * q], o[4 * q + 1], o[4 * q + 2],
                 o[4 * q + 3]);
}

template <typename T, bool OUT16, int ACT>
__global__ void __launch_bounds__(kGmThreads, 1)
    tc_gemm(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
            const __grid_constant__ CUtensorMap map_c, const GemmGeom g) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* base_ptr = smem_raw + (base - raw);
  const uint32_t stages = base;
  const uint32_t staging = base + kGmStages * kGmStageBytes;
  GemmCtrl* ctrl = reinterpret_cast<GemmCtrl*>(base_ptr + kGmStages * kGmStageBytes + 8 * kGmStageTile);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int s = 0; s < kGmStages; ++s) {
      mbar_init(smem_u32(&ctrl->full[s]), 1);
      mbar_init(smem_u32(&ctrl->empty[s]), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&ctrl->acc_full[i]), 1);
      mbar_init(smem_u32(&ctrl->acc_empty[i]), 8);  // every epilogue warp, once per tile
    }
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_a);
    tma_prefetch_desc(&map_b);
    tma_prefetch_desc(&map_c);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&ctrl->tmem_base), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctrl->tmem_base;
  const uint32_t fmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;

  if (warp == 0) {
    // ============================================================ TMA producer
    if (lane == 0) {
      const uint64_t keep = l2_policy_evict_last();  // operands are re-read by other tiles
      int st = 0, fills = 0;
      uint32_t ph = 0;
      for (int t = blockIdx.x; t < g.total_tiles; t += gridDim.x) {
        const GemmTile c = gemm_tile(g, t);
        const int ab = g.a_batched ? c.b : 0, bb = g.b_batched ? c.b : 0;
        for (int kk = 0; kk < c.nk; ++kk) {
          if (fills >= kGmStages && !mbar_wait(smem_u32(&ctrl->empty[st]), ph ^ 1u)) break;
          const uint32_t full = smem_u32(&ctrl->full[st]);
          const uint32_t sa = stages + st * kGmStageBytes, sb = sa + kGmABytes;
          const int kx = (c.k0 + kk) * kGmBK;
          mbar_arrive_expect_tx(full, kGmStageBytes);
          if (!g.a_mn) {
            tma_load_3d_hint(sa, &map_a, full, kx, c.mt * kGmBM, ab, keep);
          } else {
            tma_load_3d_hint(sa, &map_a, full, c.mt * kGmBM, kx, ab, keep);
            tma_load_3d_hint(sa + kGmMnBox, &map_a, full, c.mt * kGmBM + 64, kx, ab, keep);
          }
          if (!g.b_mn) {
            tma_load_3d_hint(sb, &map_b, full, kx, c.nt * kGmBN, bb, keep);
          } else {
#pragma unroll
            for (int i = 0; i < kGmBN / 64; ++i)
              tma_load_3d_hint(sb + i * kGmMnBox, &map_b, full, c.nt * kGmBN + i * 64, kx, bb, keep);
          }
          ++fills;
          if (++st == kGmStages) {
            st = 0;
            ph ^= 1u;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ============================================================ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(fmt, kGmBM, kGmBN, static_cast<uint32_t>(g.a_mn),
                                       static_cast<uint32_t>(g.b_mn));
      // K-major: 16 k (32 bytes) per MMA inside the 128-byte swizzled rows;
      // MN-major: 16 k rows (2 KB) per MMA, 64-wide m / n groups 8 KB apart.
      const uint64_t da0 = g.a_mn ? smem_desc_sw128(stages, kGmMnBox, 1024) : smem_desc_sw128(stages, 16, 1024);
      const uint64_t db0 = g.b_mn ? smem_desc_sw128(stages + kGmABytes, kGmMnBox, 1024)
                                  : smem_desc_sw128(stages + kGmABytes, 16, 1024);
      const uint32_t ka = g.a_mn ? (2048u >> 4) : 2u, kb = g.b_mn ? (2048u >> 4) : 2u;
      int st = 0, it = 0;
      uint32_t ph = 0;
      bool alive = true;
      for (int t = blockIdx.x; t < g.total_tiles && alive; t += gridDim.x, ++it) {
        const GemmTile c = gemm_tile(g, t);
        const int buf = it & 1;
        if (it >= 2) {
          if (!mbar_wait(smem_u32(&ctrl->acc_empty[buf]), ((it >> 1) - 1) & 1)) break;
          tc_fence_after();
        }
        const uint32_t d_tmem = tmem + static_cast<uint32_t>(buf * kGmBN);
        for (int kk = 0; kk < c.nk; ++kk) {
          if (!mbar_wait(smem_u32(&ctrl->full[st]), ph)) {
            alive = false;
            break;
          }
          tc_fence_after();
          const uint32_t adv = static_cast<uint32_t>(st * kGmStageBytes) >> 4;
#pragma unroll
          for (int k = 0; k < kGmBK / 16; ++k)
            tc_mma_f16(d_tmem, da0 + adv + ka * k, db0 + adv + kb * k, idesc,
                       (kk != 0 || k != 0) ? 1u : 0u);
          tc_commit(smem_u32(&ctrl->empty[st]));
          if (++st == kGmStages) {
            st = 0;
            ph ^= 1u;
          }
        }
        if (!alive) break;
        if (c.nk == 0)
          mbar_arrive(smem_u32(&ctrl->acc_full[buf]));  // empty K range: the tile is zero
        else
          tc_commit(smem_u32(&ctrl->acc_full[buf]));
      }
    }
  } else if (warp >= 4) {
    // ============================================================ epilogue
    const int h = (warp - 4) >> 2;  // column half of the tile
    const int wq = warp & 3;        // TMEM lane quarter
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    const uint32_t stage = staging + static_cast<uint32_t>((warp - 4) * kGmStageTile);
    const uint64_t stream = l2_policy_evict_normal();
    int it = 0;
    for (int t = blockIdx.x; t < g.total_tiles; t += gridDim.x, ++it) {
      const GemmTile c = gemm_tile(g, t);
      const int buf = it & 1;
      if (!mbar_wait(smem_u32(&ctrl->acc_full[buf]), (it >> 1) & 1)) break;
      tc_fence_after();
      const int row0 = c.mt * kGmBM + wq * 32;
      const int m = row0 + lane;
      const int n_half = c.nt * kGmBN + h * 128;
      const uint32_t tb = tmem + lane_off + static_cast<uint32_t>(buf * kGmBN + h * 128);
      const bool rows_in = row0 < g.m;
      float ss = 0.f;  // row sum of squares over this half's columns (16-bit output)
      const T* grow = nullptr;
      if (OUT16 && g.has_gate && m < g.m)
        grow = static_cast<const T*>(g.gate) + static_cast<int64_t>(c.b) * g.gate_bs +
               static_cast<int64_t>(m) * g.gate_rs;
#pragma unroll 1
      for (int ch = 0; ch < 4; ++ch) {
        const int n0 = n_half + ch * 32;
        if (n0 >= g.n) break;  // uniform across the warp
        uint32_t o[32];
        if (c.nk > 0) {
          tmem_ld32(tb + ch * 32, o);
          tmem_wait_ld(o);
        } else {
#pragma unroll
          for (int q = 0; q < 32; ++q) o[q] = 0u;
        }
        if constexpr (!OUT16) {
          if (lane == 0) bulk_wait_read_all();  // the previous store has read the tile
          __syncwarp();
          st_stage_f32(stage, lane, o);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0 && rows_in) {
            tma_store_3d(&map_c, stage, n0, row0, c.b, stream);
            bulk_commit_group();
          }
        } else {
          float bv[32];
          if (g.has_bias) {
            const T* bp = static_cast<const T*>(g.bias) + n0;
#pragma unroll
            for (int q = 0; q < 32; ++q) bv[q] = n0 + q < g.n ? to_f32<T>(bp[q]) : 0.f;
          } else {
#pragma unroll
            for (int q = 0; q < 32; ++q) bv[q] = 0.f;
          }
          uint32_t gw[16];
          if (grow) load_raw32<T>(grow + n0, g.n - n0, (g.gate_rs & 7) == 0 && (g.gate_bs & 7) == 0 &&
                                                           (reinterpret_cast<uintptr_t>(g.gate) & 15u) == 0,
                                  gw, stream);
          const bool want_ss = g.sumsq && n0 >= g.sumsq_col0;
          uint32_t pk[16];
#pragma unroll
          for (int q = 0; q < 16; ++q) {
            float y0 = act_fn<ACT>(__uint_as_float(o[2 * q]) + bv[2 * q]);
            float y1 = act_fn<ACT>(__uint_as_float(o[2 * q + 1]) + bv[2 * q + 1]);
            if (grow) {
              y0 *= raw_at<T>(gw, 2 * q);
              y1 *= raw_at<T>(gw, 2 * q + 1);
            }
            pk[q] = pack2<T>(y0, y1);
            if (want_ss) {
              // Squares of the stored (rounded) values, columns past n excluded.
              const uint16_t lo = static_cast<uint16_t>(pk[q] & 0xFFFFu), hi = static_cast<uint16_t>(pk[q] >> 16);
              const float r0 = to_f32<T>(*reinterpret_cast<const T*>(&lo));
              const float r1 = to_f32<T>(*reinterpret_cast<const T*>(&hi));
              if (n0 + 2 * q < g.n) ss = fmaf(r0, r0, ss);
              if (n0 + 2 * q + 1 < g.n) ss = fmaf(r1, r1, ss);
            }
          }
          if (lane == 0) bulk_wait_read_1();  // two tiles per warp: the store two chunks back is done
          __syncwarp();
          if (rows_in)
            warp_tile_store(stage + (ch & 1) * 2048, pk, &map_c, n0, row0, c.b, stream, lane);
        }
      }
      // The accumulator has been read: the MMA may refill it.
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&ctrl->acc_empty[buf]));
      if (OUT16 && g.sumsq && n_half >= g.sumsq_col0 && n_half < g.n && m < g.m) {
        const int plane = (n_half - g.sumsq_col0) / 128;
        g.sumsq[static_cast<int64_t>(plane) * g.batch * g.m + static_cast<int64_t>(c.b) * g.m + m] = ss;
      }
    }
    if (lane == 0) bulk_wait_read_all();
  }

  // ---------------------------------------------------------------- teardown
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace avey
