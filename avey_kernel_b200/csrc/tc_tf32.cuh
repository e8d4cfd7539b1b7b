// Tensor-core path for fp32 inputs: 3xTF32 on tcgen05 (kind::tf32).
//
// Every fp32 operand x is split into a tf32 head h = rna_tf32(x) and a tf32
// tail l = rna_tf32(x - h) (x = h + l to ~22 bits), and each product is
// formed as h_a h_b + h_a l_b + l_a h_b with fp32 accumulation: the 3-pass
// scheme the reference requests from Triton for fp32 inputs
// (input_precision="tf32x3", avey_kernels/_triton.py:92 and :105). The split
// is done in shared memory by the compute warps, between a stage's TMA
// arrival and its MMAs, so global memory only ever holds the fp32 inputs.
//
//   tf_gram_p  per (batch row, 128-query tile, group of up to 256 keys): G =
//              Z_q Z_k^T (3xTF32, 256 fp32 TMEM columns); the split also sums
//              the squares of every staged row, so the row norms need no
//              pre-pass. P = G * rinv_i * rinv_j * V under the masks, written
//              as fp32 to a [B, C, Cp] workspace, plus partial row sums.
//   tf_pv      per (batch row, 128-query tile, 256-feature group): O = P Z
//              (3xTF32). The split also transposes each staged Z block into
//              K-major order (feature rows of 32 keys), so both operands are
//              K-major as in the Gram; padded key rows of Z become zeros there,
//              so non-finite padding never meets a zero weight. Then the
//              epilogue of the other kernels (scale, bias, activation, gate,
//              row mask) and TMA stores.
//
// Both kernels hold two 96 KB stages (fp32 heads in place, tails beside them)
// and run one CTA per SM.
#pragma once

#include "tc_long.cuh"

namespace avey {

constexpr int kTfThreads = 256;
constexpr int kTfStages = 2;
constexpr int kTfChunk = 32;                          // fp32 features per 128-byte row
constexpr int kTfTile = 128 * kTfChunk * 4;           // one 128-row tile of a chunk: 16 KB
constexpr int kTfGramTiles = kLgGroupTiles + 1;       // key tiles of a group + the query tile
constexpr int kTfGramLo = kTfGramTiles * kTfTile;     // tails, after the heads: 48 KB
constexpr int kTfGramStage = 2 * kTfGramLo;           // 96 KB
constexpr int kTfPvKeys = 32;                         // keys per tf_pv stage
constexpr int kTfPvCols = 256;                        // output features per tf_pv item
constexpr int kTfPvA = 128 * kTfPvKeys * 4;           // P box {32 keys, 128 rows}: 16 KB
constexpr int kTfPvBox = 32 * kTfPvKeys * 4;          // Z box {32 features, 32 keys}: 4 KB
constexpr int kTfPvB = kTfPvCols * kTfPvKeys * 4;     // Z^T block {32 keys, 256 features}: 32 KB
// Stage layout: [P heads | Z as loaded, then the Z^T tails | P tails | Z^T heads].
constexpr int kTfPvLo = kTfPvA + kTfPvB;              // P tails: 48 KB after the P heads
constexpr int kTfPvBHi = kTfPvLo + kTfPvA;            // Z^T heads: 64 KB
constexpr int kTfPvStage = kTfPvBHi + kTfPvB;         // 96 KB
constexpr int kTfOutTile = 32 * 32 * 4;               // one warp's 32 x 32 fp32 staging tile
constexpr int kTfCtrlBytes = 4096;

struct TfGramCtrl {
  uint64_t full[kTfStages], split[kTfStages], empty[kTfStages];
  uint64_t s_full;
  uint32_t tmem_base;
  int last_valid;
  int exact;
  alignas(16) float rinv[kLgGroupKeys];
  uint32_t kbits[kLgGroupKeys / 32];
  uint8_t kvalid[kLgGroupKeys];
};
static_assert(sizeof(TfGramCtrl) <= kTfCtrlBytes, "control block too large");

struct TfPvCtrl {
  uint64_t full[kTfStages], split[kTfStages], empty[kTfStages];
  uint64_t o_full;
  uint32_t tmem_base;
  int last_valid;
  alignas(16) float bias[kTfPvCols];
  uint32_t kbits[kLongMaxContext / 32];  // allowed keys of the item's batch row and query tile
};
static_assert(sizeof(TfPvCtrl) <= kTfCtrlBytes, "control block too large");

// One staged 128-byte row (32 fp32 values; the swizzle only permutes its
// 16-byte pieces) split in place: heads where the values were, tails `lo_off`
// bytes further on; `zero` writes zeros to both instead. Returns the sum of
// squares of the row's values. The pieces are visited in the row's swizzled
// order (piece q at q ^ (row % 8)), so the 32 rows a warp splits at once
// spread over all banks.
__device__ __forceinline__ float tf32_split_row(uint32_t addr, uint32_t lo_off, bool zero) {
  const uint32_t sw = (addr >> 7) & 7u;
  uint4 v[8];
#pragma unroll
  for (int q = 0; q < 8; ++q) v[q] = ld_shared_v4(addr + ((q ^ sw) << 4));
  float s = 0.f;
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const float x[4] = {__uint_as_float(v[q].x), __uint_as_float(v[q].y), __uint_as_float(v[q].z),
                        __uint_as_float(v[q].w)};
    uint32_t h[4], l[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      s = fmaf(x[e], x[e], s);
      h[e] = tf32_rna(x[e]);
      l[e] = tf32_rna(x[e] - __uint_as_float(h[e]));
      if (zero) h[e] = l[e] = 0u;
    }
    st_shared_v4(addr + ((q ^ sw) << 4), h[0], h[1], h[2], h[3]);
    st_shared_v4(addr + lo_off + ((q ^ sw) << 4), l[0], l[1], l[2], l[3]);
  }
  return s;
}

// 32 consecutive fp32 values starting at p (16-byte aligned when vec); values
// at or past n_ok read as `fill`.
__device__ __forceinline__ void load_f32x32_global(const float* p, int n_ok, bool vec, float fill,
                                                   uint64_t policy, float (&w)[32]) {
  if (vec && n_ok >= 32) {
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const uint4 v = ld_global_nc_v4_hint(p + 4 * q, policy);
      w[4 * q] = __uint_as_float(v.x);
      w[4 * q + 1] = __uint_as_float(v.y);
      w[4 * q + 2] = __uint_as_float(v.z);
      w[4 * q + 3] = __uint_as_float(v.w);
    }
  } else {
#pragma unroll
    for (int e = 0; e < 32; ++e) w[e] = e < n_ok ? __ldg(p + e) : fill;
  }
}

// One warp's 32 x 32 fp32 tile (row = lane) through a 128-byte-swizzled
// staging tile to global memory with a TMA store.
__device__ __forceinline__ void warp_tile_store_f32(uint32_t stage, const uint32_t (&v)[32],
                                                   const CUtensorMap* map, int x, int y, int z,
                                                   uint64_t policy, int lane) {
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const int phys = q ^ (lane & 7);
    st_shared_v4(stage + lane * 128 + phys * 16, v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
  }
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    tma_store_3d(map, stage, x, y, z, policy);
    bulk_commit_group();
  }
}

// One 32-key chunk of P in fp32 for this thread's row: P = G * rk * rq * V
// under the allowed-key bits (select, so non-finite products of masked keys
// give 0), with the row sums accumulated for Avey-B.
template <bool MASKED, bool NORM, bool HAS_V>
__device__ __forceinline__ void p_chunk_f32(const uint32_t (&g)[32], const float (&rk)[32], float rqi,
                                            const float (&vw)[32], uint32_t okb, uint32_t (&pf)[32],
                                            float (&den)[4]) {
#pragma unroll
  for (int idx = 0; idx < 32; ++idx) {
    float p = __uint_as_float(g[idx]) * rk[idx];
    p *= rqi;
    if (HAS_V) p *= vw[idx];
    if (MASKED) p = ((okb >> idx) & 1u) ? p : 0.f;
    if (NORM) den[idx & 3] += p;
    pf[idx] = __float_as_uint(p);
  }
}

// ============================================================================
// tf_gram_p: G (3xTF32) with the row sums of squares, then P into the workspace.
// ============================================================================
__global__ void __launch_bounds__(kTfThreads, 1)
    tf_gram_p(const FwdArgs args, const __grid_constant__ CUtensorMap map_k,
              const __grid_constant__ CUtensorMap map_pst, const LongGeom geom) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* base_ptr = smem_raw + (base - raw);
  const uint32_t stage_addr = base;  // TMA stages; P staging tiles once the Gram is complete
  TfGramCtrl* ctrl = reinterpret_cast<TfGramCtrl*>(base_ptr + kTfStages * kTfGramStage);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int C = args.ctx, D = args.feat;
  const int b = blockIdx.y;
  // Item -> (query tile, key group), as in tc_gram_p.
  int qt = 0, kg = blockIdx.x;
  for (; qt < geom.n_qtiles; ++qt) {
    const int ng = lg_groups(qt, C, args.causal);
    if (kg < ng) break;
    kg -= ng;
  }
  const int q_lo = qt * 128;
  const int key0 = kg * kLgGroupKeys;

  if (tid == 0) {
    for (int s = 0; s < kTfStages; ++s) {
      mbar_init(smem_u32(&ctrl->full[s]), 1);
      mbar_init(smem_u32(&ctrl->split[s]), 4);  // the four compute warps
      mbar_init(smem_u32(&ctrl->empty[s]), 1);
    }
    mbar_init(smem_u32(&ctrl->s_full), 1);
    ctrl->last_valid = -1;
    ctrl->exact = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_k);
    tma_prefetch_desc(&map_pst);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&ctrl->tmem_base), kLgGroupKeys);
    tmem_relinquish();
  }
  __syncthreads();
  find_last_valid(args, b, &ctrl->last_valid);
  for (int j = tid; j < kLgGroupKeys; j += kTfThreads)
    ctrl->kvalid[j] = static_cast<uint8_t>(pos_valid(args, b, key0 + j));
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctrl->tmem_base;

  const int kv_end = ctrl->last_valid + 1;
  const int nkeys = args.causal ? min(kv_end, q_lo + 128) : kv_end;
  const bool skip = q_lo >= kv_end || key0 >= nkeys;
  const int nk = skip ? 0 : min(kLgGroupTiles, (nkeys - key0 + 127) / 128);
  const int q_in = (qt * 128 >= key0 && qt * 128 < key0 + nk * 128) ? (qt - key0 / 128) : -1;
  const int nchunk = (D + kTfChunk - 1) / kTfChunk;

  if (warp == 0) {
    if (!skip && lane == 0) {
      // ---- TMA producer: key tiles of the group (+ the query tile when it is
      // not one of them), one 32-feature chunk per stage.
      const uint64_t keep = l2_policy_evict_last();
      const uint32_t bytes = (nk + (q_in < 0 ? 1 : 0)) * kTfTile;
      int st = 0;
      uint32_t ph = 0;
      for (int c = 0; c < nchunk; ++c) {
        if (c >= kTfStages) mbar_wait(smem_u32(&ctrl->empty[st]), ph ^ 1u);
        const uint32_t full = smem_u32(&ctrl->full[st]);
        const uint32_t sa = stage_addr + st * kTfGramStage;
        mbar_arrive_expect_tx(full, bytes);
        for (int t = 0; t < nk; ++t)
          tma_load_3d_hint(sa + t * kTfTile, &map_k, full, c * kTfChunk, key0 + t * 128, b, keep);
        if (q_in < 0) tma_load_3d_hint(sa + nk * kTfTile, &map_k, full, c * kTfChunk, q_lo, b, keep);
        if (++st == kTfStages) {
          st = 0;
          ph ^= 1u;
        }
      }
    }
  } else if (warp == 1) {
    if (!skip && lane == 0) {
      // ---- MMA issuer: G[128 x 128 nk] in TMEM columns [0, 128 nk), three
      // tf32 products per 8-feature K step.
      const uint64_t d0 = smem_desc_sw128(stage_addr, 16, 1024);
      const uint32_t q_adv = static_cast<uint32_t>((q_in >= 0 ? q_in : nk) * kTfTile) >> 4;
      const uint32_t lo = static_cast<uint32_t>(kTfGramLo) >> 4;
      const uint32_t idesc = idesc_tf32(128, static_cast<uint32_t>(nk * 128), 0, 0);
      int st = 0;
      uint32_t ph = 0;
      for (int c = 0; c < nchunk; ++c) {
        mbar_wait(smem_u32(&ctrl->split[st]), ph);
        tc_fence_after();
        const uint64_t dk = d0 + static_cast<uint32_t>(st * kTfGramStage >> 4);
        const uint64_t dq = dk + q_adv;
#pragma unroll
        for (int k = 0; k < kTfChunk / 8; ++k) {
          tc_mma_tf32(tmem, dq + 2 * k, dk + 2 * k, idesc, (c != 0 || k != 0) ? 1u : 0u);
          tc_mma_tf32(tmem, dq + 2 * k, dk + lo + 2 * k, idesc, 1u);
          tc_mma_tf32(tmem, dq + lo + 2 * k, dk + 2 * k, idesc, 1u);
        }
        tc_commit(smem_u32(&ctrl->empty[st]));
        if (++st == kTfStages) {
          st = 0;
          ph ^= 1u;
        }
      }
      tc_commit(smem_u32(&ctrl->s_full));
    }
  } else if (warp >= 4) {
    // ---- compute warps: split every stage (thread = row of each tile) while
    // summing the rows' squares; then the norms and P chunks.
    const int cw = warp - 4, wq = warp & 3;
    const int row = wq * 32 + lane, i = q_lo + row;
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    if (!skip) {
      float ss_k0 = 0.f, ss_k1 = 0.f, ss_q = 0.f;
      {
        int st = 0;
        uint32_t ph = 0;
        for (int c = 0; c < nchunk; ++c) {
          mbar_wait(smem_u32(&ctrl->full[st]), ph);
          const uint32_t sa = stage_addr + st * kTfGramStage + row * 128;
          ss_k0 += tf32_split_row(sa, kTfGramLo, false);
          if (nk > 1) ss_k1 += tf32_split_row(sa + kTfTile, kTfGramLo, false);
          if (q_in < 0) ss_q += tf32_split_row(sa + nk * kTfTile, kTfGramLo, false);
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(smem_u32(&ctrl->split[st]));
          if (++st == kTfStages) {
            st = 0;
            ph ^= 1u;
          }
        }
      }
      if (q_in == 0) ss_q = ss_k0;
      if (q_in == 1) ss_q = ss_k1;
      // Inverse norms of the group's keys (0 outside the allowed set).
      int nonfinite = 0;
      const float ssk[2] = {ss_k0, ss_k1};
#pragma unroll
      for (int t = 0; t < kLgGroupTiles; ++t) {
        const int j = t * 128 + row, key = key0 + j;
        const float s2 = t < nk ? ssk[t] : 0.f;
        if (t < nk && key < C && !isfinite(s2)) nonfinite = 1;
        ctrl->rinv[j] = (t < nk && key < nkeys && ctrl->kvalid[j])
                            ? 1.f / fmaxf(sqrtf(s2), args.norm_eps_f)
                            : 0.f;
      }
      if (row < kLgGroupKeys / 32) {
        uint32_t m = 0u;
        for (int e = 0; e < 32; ++e) {
          const int j = row * 32 + e;
          if (key0 + j < nkeys && ctrl->kvalid[j]) m |= 1u << e;
        }
        ctrl->kbits[row] = m;
      }
      const bool row_ok = i < C && pos_valid(args, b, i);
      if (i < C && !isfinite(ss_q)) nonfinite = 1;
      if (nonfinite) ctrl->exact = 1;
      named_bar_sync(1, 128);
      const float rqi = row_ok ? 1.f / fmaxf(sqrtf(ss_q), args.norm_eps_f) : 0.f;
      const float* vrow = (args.has_v && i < C)
                              ? static_cast<const float*>(args.v) + static_cast<int64_t>(i) * args.v_rs + key0
                              : nullptr;
      const bool v_vec = (reinterpret_cast<uintptr_t>(args.v) & 15u) == 0 && (args.v_rs & 3) == 0;
      const uint64_t keep = l2_policy_evict_last();
      const int nch = nk * 4;
      const int vlim = C - key0;
      float vw[32], vn[32];
#pragma unroll
      for (int e = 0; e < 32; ++e) vw[e] = vn[e] = 1.f;
      if (vrow) load_f32x32_global(vrow, vlim, v_vec, 1.f, keep, vw);
      mbar_wait(smem_u32(&ctrl->s_full), 0);
      tc_fence_after();
      const bool exact = ctrl->exact != 0 || (args.has_valid && args.has_v);
      const int i0 = q_lo + wq * 32;
      const bool norm = args.normalize;
      float den4[4] = {0.f, 0.f, 0.f, 0.f};
      // The stages are idle once the Gram is complete: two staging tiles per warp.
      const uint32_t stage0 = stage_addr + cw * 2 * kTfOutTile;
#pragma unroll 1
      for (int ch = 0; ch < nch; ++ch) {
        const int c0 = ch * 32;
        uint32_t g[32];
        tmem_ld32(tmem + lane_off + c0, g);
        if (vrow && ch + 1 < nch) load_f32x32_global(vrow + c0 + 32, vlim - c0 - 32, v_vec, 1.f, keep, vn);
        const bool masked = exact || (args.causal && key0 + c0 + 31 > i0);
        uint32_t okb = 0u;
        if (masked) {
          okb = row_ok ? ctrl->kbits[c0 >> 5] : 0u;
          if (args.causal) {
            const int lim = i - (key0 + c0) + 1;
            okb &= lim >= 32 ? 0xFFFFFFFFu : (lim <= 0 ? 0u : ((1u << lim) - 1u));
          }
        }
        float rk[32];
        load_f32x32(&ctrl->rinv[c0], rk);
        tmem_wait_ld(g);
        uint32_t pf[32];
        if (args.has_v) {
          if (masked) {
            if (norm) p_chunk_f32<true, true, true>(g, rk, rqi, vw, okb, pf, den4);
            else p_chunk_f32<true, false, true>(g, rk, rqi, vw, okb, pf, den4);
          } else {
            if (norm) p_chunk_f32<false, true, true>(g, rk, rqi, vw, okb, pf, den4);
            else p_chunk_f32<false, false, true>(g, rk, rqi, vw, okb, pf, den4);
          }
        } else {
          if (masked) {
            if (norm) p_chunk_f32<true, true, false>(g, rk, rqi, vw, okb, pf, den4);
            else p_chunk_f32<true, false, false>(g, rk, rqi, vw, okb, pf, den4);
          } else {
            if (norm) p_chunk_f32<false, true, false>(g, rk, rqi, vw, okb, pf, den4);
            else p_chunk_f32<false, false, false>(g, rk, rqi, vw, okb, pf, den4);
          }
        }
        // The store two chunks back must have read its staging tile.
        if (lane == 0) bulk_wait_read_1();
        __syncwarp();
        if (key0 + c0 < C && i0 < C)
          warp_tile_store_f32(stage0 + (ch & 1) * kTfOutTile, pf, &map_pst, key0 + c0, i0, b, keep,
                              lane);  // P is read back by tf_pv soon: keep it in L2
        if (vrow) {
#pragma unroll
          for (int e = 0; e < 32; ++e) vw[e] = vn[e];
        }
      }
      if (norm && i < C)
        geom.den_part[(static_cast<int64_t>(b) * geom.n_groups + kg) * C + i] =
            (den4[0] + den4[1]) + (den4[2] + den4[3]);
      if (lane == 0) bulk_wait_read_all();
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kLgGroupKeys);
  }
}

// ============================================================================
// tf_pv: O = P Z (3xTF32) per 256-feature group, then the epilogue.
// ============================================================================
template <int ACT>
__global__ void __launch_bounds__(kTfThreads, 1)
    tf_pv(const FwdArgs args, const __grid_constant__ CUtensorMap map_p,
          const __grid_constant__ CUtensorMap map_z, const __grid_constant__ CUtensorMap map_o,
          const LongGeom geom) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* base_ptr = smem_raw + (base - raw);
  const uint32_t ring = base;  // TMA stages; output staging tiles in the epilogue
  TfPvCtrl* ctrl = reinterpret_cast<TfPvCtrl*>(base_ptr + kTfStages * kTfPvStage);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int C = args.ctx, D = args.feat;
  const int b = blockIdx.y;
  const int qi = blockIdx.x / geom.n_fgroups, fg = blockIdx.x % geom.n_fgroups;
  const int qt = args.causal ? geom.n_qtiles - 1 - qi : qi;
  const int q_lo = qt * 128;
  const int f_lo = fg * kTfPvCols;
  const int width = min(kTfPvCols, D - f_lo);

  if (tid == 0) {
    for (int s = 0; s < kTfStages; ++s) {
      mbar_init(smem_u32(&ctrl->full[s]), 1);
      mbar_init(smem_u32(&ctrl->split[s]), 4);
      mbar_init(smem_u32(&ctrl->empty[s]), 1);
    }
    mbar_init(smem_u32(&ctrl->o_full), 1);
    ctrl->last_valid = -1;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_p);
    tma_prefetch_desc(&map_z);
    tma_prefetch_desc(&map_o);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&ctrl->tmem_base), 256);
    tmem_relinquish();
  }
  __syncthreads();
  find_last_valid(args, b, &ctrl->last_valid);
  if (args.has_bias)
    for (int f = tid; f < width; f += kTfThreads)
      ctrl->bias[f] = static_cast<const float*>(args.bias)[f_lo + f];
  __syncthreads();
  const int kv_end = ctrl->last_valid + 1;
  const int nkeys = args.causal ? min(kv_end, q_lo + 128) : kv_end;
  const bool skip = q_lo >= kv_end;
  const int nkc = skip ? 0 : (nkeys + kTfPvKeys - 1) / kTfPvKeys;
  // Allowed keys (valid and below nkeys), one bit each, for the Z split.
  for (int w = tid; w < nkc; w += kTfThreads) {
    uint32_t m = 0u;
    for (int e = 0; e < 32; ++e) {
      const int key = w * 32 + e;
      if (key < nkeys && pos_valid(args, b, key)) m |= 1u << e;
    }
    ctrl->kbits[w] = m;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctrl->tmem_base;
  const int nfb = (width + 31) / 32;

  if (warp == 0) {
    if (!skip && lane == 0) {
      const uint64_t keep = l2_policy_evict_last();
      const uint32_t bytes = kTfPvA + nfb * kTfPvBox;
      int st = 0;
      uint32_t ph = 0;
      for (int kc = 0; kc < nkc; ++kc) {
        if (kc >= kTfStages) mbar_wait(smem_u32(&ctrl->empty[st]), ph ^ 1u);
        const uint32_t full = smem_u32(&ctrl->full[st]);
        const uint32_t sa = ring + st * kTfPvStage;
        mbar_arrive_expect_tx(full, bytes);
        tma_load_3d(sa, &map_p, full, kc * kTfPvKeys, q_lo, b);
        for (int i = 0; i < nfb; ++i)
          tma_load_3d_hint(sa + kTfPvA + i * kTfPvBox, &map_z, full, f_lo + i * 32, kc * kTfPvKeys, b,
                           keep);
        if (++st == kTfStages) {
          st = 0;
          ph ^= 1u;
        }
      }
    }
  } else if (warp == 1) {
    if (!skip && lane == 0) {
      // A: P and B: Z^T, both K-major (8 keys = 32 bytes per K step); heads
      // and tails as laid out by the split.
      const uint64_t d0 = smem_desc_sw128(ring, 16, 1024);
      const uint64_t e0 = smem_desc_sw128(ring + kTfPvBHi, 16, 1024);
      const uint32_t lo = static_cast<uint32_t>(kTfPvLo) >> 4;
      const uint32_t zlo = static_cast<uint32_t>(kTfPvBHi - kTfPvA) >> 4;  // Z^T tails sit below the heads
      const uint32_t idesc = idesc_tf32(128, static_cast<uint32_t>((width + 15) & ~15), 0, 0);
      int st = 0;
      uint32_t ph = 0;
      for (int kc = 0; kc < nkc; ++kc) {
        mbar_wait(smem_u32(&ctrl->split[st]), ph);
        tc_fence_after();
        const uint32_t adv = static_cast<uint32_t>(st * kTfPvStage) >> 4;
#pragma unroll
        for (int k = 0; k < kTfPvKeys / 8; ++k) {
          const uint64_t a = d0 + adv + 2 * k, bz = e0 + adv + 2 * k;
          tc_mma_tf32(tmem, a, bz, idesc, (kc != 0 || k != 0) ? 1u : 0u);
          tc_mma_tf32(tmem, a, bz - zlo, idesc, 1u);
          tc_mma_tf32(tmem, a + lo, bz, idesc, 1u);
        }
        tc_commit(smem_u32(&ctrl->empty[st]));
        if (++st == kTfStages) {
          st = 0;
          ph ^= 1u;
        }
      }
      tc_commit(smem_u32(&ctrl->o_full));
    }
  } else if (warp >= 4 && !skip) {
    // ---- split: P rows in place (thread = query row); then Z transposed to
    // K-major feature rows (thread = feature f and f + 128: its 32 keys are
    // read across the stage's key rows, keys outside the allowed set as 0),
    // heads into the Z^T head block, tails over the loaded Z once every
    // thread has read its values.
    const int t = tid - 128;
    int st = 0;
    uint32_t ph = 0;
    for (int kc = 0; kc < nkc; ++kc) {
      mbar_wait(smem_u32(&ctrl->full[st]), ph);
      const uint32_t sa = ring + st * kTfPvStage;
      tf32_split_row(sa + t * 128, kTfPvLo, false);
      const uint32_t kb = ctrl->kbits[kc];
      float zv[2][32];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int f = t + 128 * h, fc = f & 31;
        const uint32_t src = sa + kTfPvA + (f >> 5) * kTfPvBox + (fc & 3) * 4;
#pragma unroll
        for (int k = 0; k < 32; ++k) {
          float v = 0.f;
          if (f < nfb * 32)
            asm volatile("ld.shared.f32 %0, [%1];"
                         : "=f"(v)
                         : "r"(src + k * 128 + ((((fc >> 2) ^ (k & 7)) & 7) << 4)));
          zv[h][k] = ((kb >> k) & 1u) ? v : 0.f;
        }
      }
      named_bar_sync(2, 128);  // every thread has read the loaded Z: its space takes the tails
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int f = t + 128 * h;
        if (f < nfb * 32) {
          const uint32_t hi_row = sa + kTfPvBHi + f * 128, lo_row = sa + kTfPvA + f * 128;
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            uint32_t hv[4], lv[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float x = zv[h][4 * q + e];
              hv[e] = tf32_rna(x);
              lv[e] = tf32_rna(x - __uint_as_float(hv[e]));
            }
            const uint32_t off = static_cast<uint32_t>((q ^ (f & 7)) << 4);
            st_shared_v4(hi_row + off, hv[0], hv[1], hv[2], hv[3]);
            st_shared_v4(lo_row + off, lv[0], lv[1], lv[2], lv[3]);
          }
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&ctrl->split[st]));
      if (++st == kTfStages) {
        st = 0;
        ph ^= 1u;
      }
    }
  }
  __syncwarp();  // lanes 1-31 of the producer and MMA warps rejoin lane 0

  // Epilogue: after the last MMA the stages are idle, so they hold the output
  // staging tiles (two per warp), and all eight warps drain the accumulator:
  // the warps of one TMEM lane quarter (w and w + 4) take one half of the
  // columns each.
  {
    const int wq = warp & 3, half = warp >> 2;
    const int row = wq * 32 + lane, i = q_lo + row;
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    const uint32_t stage_w = ring + warp * 2 * kTfOutTile;
    if (skip) {
      // No valid query row in this tile: its output rows are zero.
#pragma unroll
      for (int q = 0; q < 8; ++q) st_shared_v4(stage_w + lane * 128 + q * 16, 0u, 0u, 0u, 0u);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        const uint64_t stream = l2_policy_evict_normal();
        const int nbf = (width + 31) / 32, nbr = (min(128, C - q_lo) + 31) / 32;
        for (int k = warp; k < nbf * nbr; k += 8)
          tma_store_3d(&map_o, stage_w, f_lo + (k % nbf) * 32, q_lo + (k / nbf) * 32, b, stream);
        bulk_commit_group();
        bulk_wait_read_all();
      }
    } else {
      griddep_wait();
      const bool row_ok = i < C && pos_valid(args, b, i);
      float den = 0.f;
      if (row_ok && args.normalize) {
        const int ng = (nkeys + kLgGroupKeys - 1) / kLgGroupKeys;
        for (int g = 0; g < ng; ++g)
          den += geom.den_part[(static_cast<int64_t>(b) * geom.n_groups + g) * C + i];
      }
      // rq is inside P (fp32 keeps its range), so O needs only the row sum.
      const float inv = args.normalize ? 1.f / (den + args.eps_f) : 1.f;
      const float* zl = args.has_zl ? static_cast<const float*>(args.z_tl) + static_cast<int64_t>(b) * args.zl_bs
                                    : nullptr;
      const float* zrow = (zl && i < C) ? zl + static_cast<int64_t>(i) * args.zl_rs : nullptr;
      const bool zl_vec = zl && (reinterpret_cast<uintptr_t>(args.z_tl) & 15u) == 0 &&
                          (args.zl_rs & 3) == 0 && (args.zl_bs & 3) == 0;
      const uint64_t stream = l2_policy_evict_normal();
      const bool has_bias = args.has_bias;
      const int nch = (width + 31) / 32, ch_mid = (nch + 1) / 2;
      const int c_lo = half ? ch_mid * 32 : 0, c_hi = half ? width : min(width, ch_mid * 32);
      float gn[32];
      if (zrow && c_lo < c_hi) load_f32x32_global(zrow + f_lo + c_lo, D - f_lo - c_lo, zl_vec, 0.f, stream, gn);
      mbar_wait(smem_u32(&ctrl->o_full), 0);
      tc_fence_after();
#pragma unroll 1
      for (int c0 = c_lo, n = 0; c0 < c_hi; c0 += 32, ++n) {
        uint32_t o[32];
        float gw[32];
        tmem_ld32(tmem + lane_off + c0, o);
#pragma unroll
        for (int e = 0; e < 32; ++e) gw[e] = gn[e];
        if (zrow && c0 + 32 < c_hi)
          load_f32x32_global(zrow + f_lo + c0 + 32, D - f_lo - c0 - 32, zl_vec, 0.f, stream, gn);
        float bv[32];
        load_bias32(&ctrl->bias[c0], has_bias, bv);
        tmem_wait_ld(o);
        uint32_t y32[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          float y = act_fn<ACT>(fmaf(__uint_as_float(o[e]), inv, bv[e]));
          if (zrow) y *= gw[e];
          y32[e] = __float_as_uint(row_ok ? y : 0.f);
        }
        // Two staging tiles: the store two chunks back must have read its tile.
        if (lane == 0) bulk_wait_read_1();
        __syncwarp();
        if (q_lo + wq * 32 < C)
          warp_tile_store_f32(stage_w + (n & 1) * kTfOutTile, y32, &map_o, f_lo + c0, q_lo + wq * 32, b,
                              stream, lane);
      }
      if (lane == 0) bulk_wait_read_all();
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

}  // namespace avey
