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
//  * the static (position-wise or token-mixing) layers, with the gate;
//  * O = P Z of the long-context contextualizer (tc_long.cuh's P workspace
//    times z_tr), with the contextualizer's row scale in the epilogue.
//
// Structure: persistent CTAs (one per SM, tiles of 128 x 256 taken round
// robin, batch entry by batch entry), warp 0 issues TMA (4 stages of a
// 128 x 64 A tile and a 64 x 256 B tile, 128-byte swizzle), warp 1 issues
// tcgen05.mma (M = 128, N = 256, K = 16) into one of two 256-column TMEM
// accumulators, and warps 4-11 drain the other accumulator (thread = output
// row, 32 columns per tcgen05.ld, the next chunk's load in flight) through
// per-warp staging tiles and TMA tensor stores, so a tile's epilogue overlaps
// the next tile's main loop. A variant runs on CTA pairs (tc_gemm_pair, below).
// Every wait is bounded (ptx.cuh).
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
constexpr int kGmStageTile = 4096;  // a warp's two 2 KB staging tiles (32 x 16 fp32 or 32 x 32 16-bit each)
constexpr int kGmCtrlBytes = 1024;
constexpr int kGmSmem = 1024 + kGmStages * kGmStageBytes + 8 * kGmStageTile + kGmCtrlBytes;

enum GemmMode { kGemmDense = 0, kGemmLowerOut = 1, kGemmKLower = 2, kGemmKUpper = 3 };

struct GemmGeom {
  int batch, m, n, k;
  int bm;               // rows per output tile: 128 (one CTA) or 256 (a CTA pair)
  int n_mt, n_nt;       // row and column tiles per batch entry
  int mode;             // GemmMode
  int a_mn, b_mn;       // operand is MN-major (else K-major)
  int a_batched, b_batched;
  int total_tiles, tiles_per_batch;
  int has_bias, has_gate;
  int sumsq_col0;       // 16-bit output: first column of the row sums of squares (multiple of 128)
  const void* bias;     // [n], operand type
  const void* gate;     // [batch][m][n], operand type
  int64_t gate_bs, gate_rs;
  float* sumsq;         // planes [(n - col0) / 128][batch * m], or null
  // Contextualizer mix epilogue (O = P Z of the long-context path, 16-bit
  // output): each row scaled before the bias as tc_pv scales it, from the
  // rows' sums of squares (ctx_sumsq [batch * m]) and, for Avey-B, the partial
  // row sums of P (ctx_den [batch][ctx_groups][m]); null when unused.
  const float* ctx_sumsq;
  const float* ctx_den;
  int ctx_groups, ctx_causal, ctx_normalize, ctx_rq_in_p;
  float ctx_eps, ctx_norm_eps;
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
  return g.mode == kGemmLowerOut ? min(g.n_nt, (mt * g.bm + g.bm - 1) / kGmBN + 1) : g.n_nt;
}

// Tile t of the launch: batch entries outermost, so the CTAs working at one
// time share few operands in L2 (a batch entry's A and B are read from DRAM
// about once: batch-inner orders measured 1.6x the operand bytes); inside a
// batch entry, row tiles (the longest K ranges first under kGemmKLower), then
// column tiles, so neighbouring CTAs share the A row block.
__device__ __forceinline__ GemmTile gemm_tile(const GemmGeom& g, int t) {
  GemmTile c{0, 0, 0, 0, 0};
  c.b = t / g.tiles_per_batch;
  int rem = t - c.b * g.tiles_per_batch;
  for (int o = 0; o < g.n_mt; ++o) {
    const int mt = g.mode == kGemmKLower ? g.n_mt - 1 - o : o;
    const int cnt = gemm_cols_of(g, mt);
    if (rem < cnt) {
      c.mt = mt;
      c.nt = rem;
      break;
    }
    rem -= cnt;
  }
  int klo = 0, khi = g.k;
  if (g.mode == kGemmKLower) khi = min(g.k, (c.mt + 1) * g.bm);
  if (g.mode == kGemmKUpper) klo = min(g.k, c.mt * g.bm);
  c.k0 = klo / kGmBK;
  c.nk = khi > klo ? (khi - c.k0 * kGmBK + kGmBK - 1) / kGmBK : 0;
  return c;
}

// Drain this warp's 32 rows (first row `row0`) x 128 columns (half `h` of the
// 256-column tile) of one accumulator (`tb0`: TMEM address of column 0 of the
// buffer in this warp's lane quarter) into C, then release the accumulator by
// one arrival on `acc_empty` (this CTA's barrier, or with PAIR the pair
// leader's, as a shared::cluster address). fp32 output: 32 x 16 halves
// through two staging tiles and TMA stores; 16-bit output: row scale, bias,
// activation, gate, row sums of squares, 32 x 32 tiles.
template <typename T, bool OUT16, int ACT, bool PAIR>
__device__ __forceinline__ void gemm_drain_tile(const GemmGeom& g, const GemmTile& c, int row0,
                                                uint32_t tb0, int h, int lane, uint32_t stage,
                                                const CUtensorMap* map_c, uint64_t stream,
                                                uint32_t acc_empty) {
  const int m = row0 + lane;
  const int n_half = c.nt * kGmBN + h * 128;
  const uint32_t tb = tb0 + static_cast<uint32_t>(h * 128);
  const bool rows_in = row0 < g.m;
  float ss = 0.f;  // row sum of squares over this half's columns (16-bit output)
  const T* grow = nullptr;
  if (OUT16 && g.has_gate && m < g.m)
    grow = static_cast<const T*>(g.gate) + static_cast<int64_t>(c.b) * g.gate_bs +
           static_cast<int64_t>(m) * g.gate_rs;
  const bool bias_vec = (reinterpret_cast<uintptr_t>(g.bias) & 15u) == 0;
  // Row scale of the contextualizer mix (1 otherwise): 1 / max(||z_i||,
  // norm_eps) (unless it is already in P), divided by (row sum of P + eps) for
  // Avey-B, with the partial sums added in group order (as tc_pv does).
  float rs = 1.f;
  if (OUT16 && g.ctx_sumsq && m < g.m) {
    const int64_t r = static_cast<int64_t>(c.b) * g.m + m;
    const float rq = 1.f / fmaxf(sqrtf(g.ctx_sumsq[r]), g.ctx_norm_eps);
    const float os = g.ctx_rq_in_p ? 1.f : rq;
    if (g.ctx_normalize) {
      const int q_lo = (m / 128) * 128;
      const int nkeys = g.ctx_causal ? min(g.m, q_lo + 128) : g.m;
      const int ng = (nkeys + kLgGroupKeys - 1) / kLgGroupKeys;
      float den = 0.f;
      for (int gg = 0; gg < ng; ++gg)
        den += g.ctx_den[(static_cast<int64_t>(c.b) * g.ctx_groups + gg) * g.m + m];
      rs = os / (os * den + g.ctx_eps);
    } else {
      rs = os;
    }
  }
  const int nch = max(0, min(4, (g.n - n_half + 31) / 32));  // chunks of 32 columns in range
  // The staging tiles alternate chunk by chunk (and half by half for fp32)
  // within a tile; across tiles the stores of the last tile must have read
  // them first.
  if (lane == 0) bulk_wait_read_all();
  __syncwarp();
  // One 32-column chunk: stores (and sums) from registers `o`.
  // Gate words of the next chunk to emit (16-bit output with a gate).
  const bool gate_vec = (g.gate_rs & 7) == 0 && (g.gate_bs & 7) == 0 &&
                        (reinterpret_cast<uintptr_t>(g.gate) & 15u) == 0;
  uint32_t gn[16];
#pragma unroll
  for (int q = 0; q < 16; ++q) gn[q] = 0u;
  if (OUT16 && grow && nch > 0) load_raw32<T>(grow + n_half, g.n - n_half, gate_vec, gn, stream);
  auto emit = [&](int ch, const uint32_t (&o)[32]) {
    const int n0 = n_half + ch * 32;
    if constexpr (!OUT16) {
      // Two 16-column halves through two 2 KB staging tiles (64-byte rows,
      // 64-byte swizzle): a half waits only for the store two halves back.
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const uint32_t st_tile = stage + static_cast<uint32_t>(hh * 2048);
        if (lane == 0) bulk_wait_read_1();
        __syncwarp();
#pragma unroll
        for (int q = 0; q < 4; ++q)
          st_shared_v4(st_tile + lane * 64 + ((q ^ ((lane >> 1) & 3)) << 4), o[16 * hh + 4 * q],
                       o[16 * hh + 4 * q + 1], o[16 * hh + 4 * q + 2], o[16 * hh + 4 * q + 3]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0 && rows_in && n0 + 16 * hh < g.n) {
          tma_store_3d(map_c, st_tile, n0 + 16 * hh, row0, c.b, stream);
          bulk_commit_group();
        }
      }
    } else {
      // The chunk's 32 bias values as packed 16-bit pairs (converted where used).
      uint32_t bw[16];
      if (g.has_bias) {
        const T* bp = static_cast<const T*>(g.bias) + n0;
        if (bias_vec && n0 + 32 <= g.n) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint4 v = ld_global_nc_v4(bp + 8 * q);
            bw[4 * q] = v.x;
            bw[4 * q + 1] = v.y;
            bw[4 * q + 2] = v.z;
            bw[4 * q + 3] = v.w;
          }
        } else {
          const uint16_t* bh = reinterpret_cast<const uint16_t*>(bp);
#pragma unroll
          for (int q = 0; q < 16; ++q) {
            const uint32_t lo = n0 + 2 * q < g.n ? bh[2 * q] : 0u;
            const uint32_t hi = n0 + 2 * q + 1 < g.n ? bh[2 * q + 1] : 0u;
            bw[q] = lo | (hi << 16);
          }
        }
      } else {
#pragma unroll
        for (int q = 0; q < 16; ++q) bw[q] = 0u;  // +0.0 in both 16-bit formats
      }
      // This chunk's gate words (loaded one chunk ahead), then the next chunk's.
      uint32_t gw[16];
#pragma unroll
      for (int q = 0; q < 16; ++q) gw[q] = gn[q];
      if (grow && ch + 1 < nch) load_raw32<T>(grow + n0 + 32, g.n - n0 - 32, gate_vec, gn, stream);
      const bool want_ss = g.sumsq && n0 >= g.sumsq_col0;
      const bool whole = n0 + 32 <= g.n;
      uint32_t pk[16];
#pragma unroll
      for (int q = 0; q < 16; ++q) {
        float y0 = act_fn<ACT>(fmaf(__uint_as_float(o[2 * q]), rs, raw_at<T>(bw, 2 * q)));
        float y1 = act_fn<ACT>(fmaf(__uint_as_float(o[2 * q + 1]), rs, raw_at<T>(bw, 2 * q + 1)));
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
          if (whole || n0 + 2 * q < g.n) ss = fmaf(r0, r0, ss);
          if (whole || n0 + 2 * q + 1 < g.n) ss = fmaf(r1, r1, ss);
        }
      }
      if (lane == 0) bulk_wait_read_1();  // two tiles per warp: the store two chunks back is done
      __syncwarp();
      if (rows_in) warp_tile_store(stage + (ch & 1) * 2048, pk, map_c, n0, row0, c.b, stream, lane);
    }
  };
  if (c.nk > 0) {
    // TMEM loads run one chunk ahead of the stores.
    uint32_t oa[32], ob[32];
    if (nch > 0) tmem_ld32(tb, oa);
#pragma unroll 1
    for (int ch = 0; ch < nch; ch += 2) {
      tmem_wait_ld(oa);
      const bool has_b = ch + 1 < nch;
      if (has_b) tmem_ld32(tb + (ch + 1) * 32, ob);
      emit(ch, oa);
      if (has_b) {
        tmem_wait_ld(ob);
        if (ch + 2 < nch) tmem_ld32(tb + (ch + 2) * 32, oa);
        emit(ch + 1, ob);
      }
    }
  } else {
    uint32_t z[32];
#pragma unroll
    for (int q = 0; q < 32; ++q) z[q] = 0u;
#pragma unroll 1
    for (int ch = 0; ch < nch; ++ch) emit(ch, z);
  }
  // The accumulator has been read: the MMA may refill it.
  tc_fence_before();
  __syncwarp();
  if (lane == 0) {
    if (PAIR)
      mbar_arrive_cluster(acc_empty);
    else
      mbar_arrive(acc_empty);
  }
  if (OUT16 && g.sumsq && n_half >= g.sumsq_col0 && n_half < g.n && m < g.m) {
    const int plane = (n_half - g.sumsq_col0) / 128;
    g.sumsq[static_cast<int64_t>(plane) * g.batch * g.m + static_cast<int64_t>(c.b) * g.m + m] = ss;
  }
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
      gemm_drain_tile<T, OUT16, ACT, false>(g, c, c.mt * g.bm + wq * 32, tmem + lane_off + static_cast<uint32_t>(buf * kGmBN),
                                     h, lane, stage, &map_c, stream,
                                     smem_u32(&ctrl->acc_empty[buf]));
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

// ============================================================================
// The same product on CTA pairs (cta_group::2): a (2, 1, 1) cluster computes
// 256 x 256 output tiles, the even CTA (rank 0) holding rows 0-127 and the
// odd one rows 128-255. Each CTA loads its own 128 rows of the A tile and its
// half of the B tile's 256 columns (16 KB + 16 KB per 64-wide K block), so a
// CTA moves half the B bytes of the single-CTA kernel per MMA cycle; rank 0
// issues the M = 256 MMAs for both. Six 32 KB stages per CTA.
//
// Barriers: full[s] of rank 0 counts both CTAs' TMA bytes (their loads name
// it through its shared::cluster address); empty[s] and acc_full[b] of both
// CTAs are signalled by rank 0's commits (one plain commit per CTA, to a mapa address);
// acc_empty[b] of rank 0 counts the epilogue warps of both CTAs. Every wait
// is bounded, and both CTAs always reach the final cluster barrier.
// ============================================================================
constexpr int kG2Stages = 6;
constexpr int kG2HalfBytes = 128 * kGmBK * 2;          // 16 KB: 128 rows (A) or N-columns (B)
constexpr int kG2StageBytes = 2 * kG2HalfBytes;         // 32 KB per CTA
constexpr int kG2Smem = 1024 + kG2Stages * kG2StageBytes + 8 * kGmStageTile + kGmCtrlBytes;

struct Gemm2Ctrl {
  uint64_t full[kG2Stages], empty[kG2Stages];
  uint64_t acc_full[2], acc_empty[2];
  uint32_t tmem_base;
};
static_assert(sizeof(Gemm2Ctrl) <= kGmCtrlBytes, "control block too large");

template <typename T, bool OUT16, int ACT>
__global__ void __launch_bounds__(kGmThreads, 1)
    tc_gemm_pair(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                 const __grid_constant__ CUtensorMap map_c, const GemmGeom g) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* base_ptr = smem_raw + (base - raw);
  const uint32_t stages = base;
  const uint32_t staging = base + kG2Stages * kG2StageBytes;
  Gemm2Ctrl* ctrl = reinterpret_cast<Gemm2Ctrl*>(base_ptr + kG2Stages * kG2StageBytes + 8 * kGmStageTile);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  if (tid == 0) {
    for (int s = 0; s < kG2Stages; ++s) {
      mbar_init(smem_u32(&ctrl->full[s]), 1);
      mbar_init(smem_u32(&ctrl->empty[s]), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&ctrl->acc_full[i]), 1);
      mbar_init(smem_u32(&ctrl->acc_empty[i]), 16);  // 8 epilogue warps in each CTA
    }
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_a);
    tma_prefetch_desc(&map_b);
    tma_prefetch_desc(&map_c);
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(&ctrl->tmem_base), 512);
    tmem_relinquish_pair();
  }
  // Both CTAs' barriers are initialised and the TMEM is allocated before
  // either CTA signals the other.
  tc_fence_before();
  __syncwarp();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = ctrl->tmem_base;
  const uint32_t fmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;

  if (warp == 0) {
    // ============================================================ TMA producer (both CTAs)
    if (lane == 0) {
      const uint64_t keep = l2_policy_evict_last();
      int st = 0, fills = 0;
      uint32_t ph = 0;
      bool alive = true;
      for (int t = pair; t < g.total_tiles && alive; t += npairs) {
        const GemmTile c = gemm_tile(g, t);
        const int ab = g.a_batched ? c.b : 0, bb = g.b_batched ? c.b : 0;
        const int arow = c.mt * 256 + static_cast<int>(rank) * 128;  // this CTA's A rows
        const int bcol = c.nt * kGmBN + static_cast<int>(rank) * 128;  // this CTA's B columns
        for (int kk = 0; kk < c.nk; ++kk) {
          if (fills >= kG2Stages && !mbar_wait(smem_u32(&ctrl->empty[st]), ph ^ 1u)) {
            alive = false;
            break;
          }
          const uint32_t full = mapa_shared(smem_u32(&ctrl->full[st]), 0);
          const uint32_t sa = stages + st * kG2StageBytes, sb = sa + kG2HalfBytes;
          const int kx = (c.k0 + kk) * kGmBK;
          if (leader) mbar_arrive_expect_tx(smem_u32(&ctrl->full[st]), 2 * kG2StageBytes);
          if (!g.a_mn) {
            tma_load_3d_pair(sa, &map_a, full, kx, arow, ab, keep);
          } else {
            tma_load_3d_pair(sa, &map_a, full, arow, kx, ab, keep);
            tma_load_3d_pair(sa + kGmMnBox, &map_a, full, arow + 64, kx, ab, keep);
          }
          if (!g.b_mn) {
            tma_load_3d_pair(sb, &map_b, full, kx, bcol, bb, keep);
          } else {
            tma_load_3d_pair(sb, &map_b, full, bcol, kx, bb, keep);
            tma_load_3d_pair(sb + kGmMnBox, &map_b, full, bcol + 64, kx, bb, keep);
          }
          ++fills;
          if (++st == kG2Stages) {
            st = 0;
            ph ^= 1u;
          }
        }
      }
      // Wait until every stage this CTA filled has been released by the
      // leader's commits, so none of them is still in flight when it exits.
      for (int i = 0; i < kG2Stages && i < fills && alive; ++i) {
        // Stage (st - 1 - i) mod S was filled last in its own phase.
        const int s = (st - 1 - i + kG2Stages) % kG2Stages;
        const int uses = (fills - 1 - i) / kG2Stages;  // index of that stage's last fill
        if (!mbar_wait(smem_u32(&ctrl->empty[s]), uses & 1)) break;
      }
    }
  } else if (warp == 1) {
    // ============================================================ MMA issuer (rank 0 only)
    if (lane == 0 && leader) {
      const uint32_t idesc = idesc_f16(fmt, 256, kGmBN, static_cast<uint32_t>(g.a_mn),
                                       static_cast<uint32_t>(g.b_mn));
      const uint64_t da0 = g.a_mn ? smem_desc_sw128(stages, kGmMnBox, 1024) : smem_desc_sw128(stages, 16, 1024);
      const uint64_t db0 = g.b_mn ? smem_desc_sw128(stages + kG2HalfBytes, kGmMnBox, 1024)
                                  : smem_desc_sw128(stages + kG2HalfBytes, 16, 1024);
      const uint32_t ka = g.a_mn ? (2048u >> 4) : 2u, kb = g.b_mn ? (2048u >> 4) : 2u;
      int st = 0, it = 0;
      uint32_t ph = 0;
      bool alive = true;
      for (int t = pair; t < g.total_tiles && alive; t += npairs, ++it) {
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
          const uint32_t adv = static_cast<uint32_t>(st * kG2StageBytes) >> 4;
#pragma unroll
          for (int k = 0; k < kGmBK / 16; ++k)
            tc_mma_f16_pair(d_tmem, da0 + adv + ka * k, db0 + adv + kb * k, idesc,
                            (kk != 0 || k != 0) ? 1u : 0u);
          tc_commit_pair(smem_u32(&ctrl->empty[st]));
          tc_commit_pair(mapa_shared(smem_u32(&ctrl->empty[st]), 1));
          if (++st == kG2Stages) {
            st = 0;
            ph ^= 1u;
          }
        }
        if (!alive) break;
        if (c.nk == 0) {  // empty K range: the tile is zero
          mbar_arrive(smem_u32(&ctrl->acc_full[buf]));
          mbar_arrive_cluster(mapa_shared(smem_u32(&ctrl->acc_full[buf]), 1));
        } else {
          tc_commit_pair(smem_u32(&ctrl->acc_full[buf]));
          tc_commit_pair(mapa_shared(smem_u32(&ctrl->acc_full[buf]), 1));
        }
      }
    }
  } else if (warp >= 4) {
    // ============================================================ epilogue (both CTAs)
    const int h = (warp - 4) >> 2;
    const int wq = warp & 3;
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    const uint32_t stage = staging + static_cast<uint32_t>((warp - 4) * kGmStageTile);
    const uint64_t stream = l2_policy_evict_normal();
    int it = 0;
    for (int t = pair; t < g.total_tiles; t += npairs, ++it) {
      const GemmTile c = gemm_tile(g, t);
      const int buf = it & 1;
      if (!mbar_wait(smem_u32(&ctrl->acc_full[buf]), (it >> 1) & 1)) break;
      tc_fence_after();
      gemm_drain_tile<T, OUT16, ACT, true>(g, c, c.mt * 256 + static_cast<int>(rank) * 128 + wq * 32,
                                           tmem + lane_off + static_cast<uint32_t>(buf * kGmBN), h, lane,
                                           stage, &map_c, stream,
                                           mapa_shared(smem_u32(&ctrl->acc_empty[buf]), 0));
    }
    if (lane == 0) bulk_wait_read_all();
  }

  // ---------------------------------------------------------------- teardown
  tc_fence_before();
  __syncwarp();
  cluster_sync();  // no signal targets either CTA after this point
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 512);
  }
}

}  // namespace avey
