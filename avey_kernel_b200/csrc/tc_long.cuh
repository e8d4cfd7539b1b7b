// Tensor-core path for contexts longer than 512 tokens (two kernels after the
// row-norm pre-pass):
//
//   tc_gram_p  per (batch row, 128-query tile, group of up to 2 key tiles):
//              G = Z_q Z_k^T on tcgen05 (256 fp32 TMEM columns per CTA, two
//              CTAs per SM), P = G * rinv_j * V (* rinv_i for fp16) under the
//              masks, written as bf16/f16 to a [B, C, Cp] workspace, plus the
//              group's partial row sums of P (Avey-B).
//   tc_pv      per (batch row, 128-query tile, 256-feature group): O = P Z
//              on tcgen05 with P and Z streamed by TMA (P is K-major, Z is
//              MN-major), then the same epilogue as the fused kernel (scale,
//              bias, activation, gate, row mask) and TMA stores.
//
// Compared with the fused kernel (contexts <= 512) P makes one round trip
// through HBM (2 bytes per allowed (query, key) pair, written once and read
// once per feature group); S is never recomputed. The reference's Triton
// kernel (_triton.py:53-128) instead recomputes S for every output feature
// tile.
#pragma once

#include "tc_kernel.cuh"

namespace avey {

// tc_gram_p: groups of 256 keys (256 TMEM columns), one compute warpgroup,
// ~107 KB of shared memory: two CTAs share an SM, so one CTA's P phase (CUDA
// cores, TMA stores) overlaps the other's Gram phase (TMA loads, tcgen05).
constexpr int kLgWG = 1;                     // compute warpgroups
constexpr int kLgThreads = 128 + 128 * kLgWG;
constexpr int kLgGroupKeys = 256;            // keys per tc_gram_p item (TMEM columns)
constexpr int kLgGroupTiles = kLgGroupKeys / 128;
constexpr int kLgStageBytes = (1 + kLgGroupTiles) * kTcTileBytesA;  // query + key tiles, one chunk
constexpr int kLgStages = 2;
constexpr int kLgCtrlBytes = 2048;
constexpr int kLongMaxContext = 8192;

// tc_pv: 256 threads (producer warp, MMA warp, two idle warps, one warpgroup
// that waits for the accumulator; all eight warps then drain it) and ~99 KB of
// shared memory, so two CTAs share an SM and one's epilogue overlaps the
// other's main loop.
constexpr int kPvThreads = 256;
constexpr int kPvGroupCols = 256;            // output features per tc_pv item (TMEM columns)
constexpr int kPvChunkKeys = 64;             // keys per pipeline stage
constexpr int kPvABytes = 128 * kPvChunkKeys * 2;  // P box {64 keys, 128 rows}: 16 KB
constexpr int kPvBBoxBytes = 64 * kPvChunkKeys * 2;  // Z box {64 features, 64 keys}: 8 KB
constexpr int kPvStageBytes = kPvABytes + 4 * kPvBBoxBytes;  // 48 KB
constexpr int kPvStages = 2;
constexpr int kPvCtrlBytes = 1536;

struct LongGeom {
  int n_qtiles;     // query tiles per batch row
  int n_groups;     // key groups of the longest query tile (ceil(C / 512))
  int items;        // tc_gram_p items per batch row
  int n_fgroups;    // tc_pv feature groups per query tile
  int64_t p_rs;     // P workspace row stride (elements)
  int64_t p_bs;     // P workspace batch stride (elements)
  float* den_part;  // [batch][n_groups][ctx] partial row sums of P (Avey-B)
};

struct LgCtrl {
  uint64_t full[kLgStages], empty[kLgStages];
  uint64_t s_full;
  uint32_t tmem_base;
  int last_valid;
  int exact;
  alignas(16) float rinv[kLgGroupKeys];  // inverse norms of the group's keys (0: not allowed)
  uint32_t kbits[kLgGroupKeys / 32];
  uint8_t kvalid[kLgGroupKeys];
};
static_assert(sizeof(LgCtrl) <= kLgCtrlBytes, "control block too large");

struct PvCtrl {
  uint64_t full[kPvStages], empty[kPvStages], fixed[kPvStages];
  uint64_t o_full;
  uint32_t tmem_base;
  int last_valid;
  int fix;  // some key row the MMA reads outside the allowed set is not finite
  alignas(16) float bias[kPvGroupCols];
};
static_assert(sizeof(PvCtrl) <= kPvCtrlBytes, "control block too large");

// Last valid position of batch row b (-1 if none), computed by the whole CTA.
__device__ __forceinline__ void find_last_valid(const FwdArgs& args, int b, int* slot) {
  int last = -1;
  for (int j = threadIdx.x; j < args.ctx; j += blockDim.x)
    if (mask_ok(args, b, j)) last = j;
  if (last >= 0) atomicMax(slot, last);
}

__device__ __forceinline__ bool pos_valid(const FwdArgs& args, int b, int j) {
  return j < args.ctx && mask_ok(args, b, j);
}

// Key groups of query tile qt: keys [0, nkeys) in groups of 512.
__device__ __forceinline__ int lg_groups(int qt, int ctx, int causal) {
  const int nkeys = causal ? min(ctx, qt * 128 + 128) : ctx;
  return (nkeys + kLgGroupKeys - 1) / kLgGroupKeys;
}

// One warp's 32 x 32 tile (rows = lanes, 32 columns packed in pk) through a
// 64-byte-swizzled shared staging tile to global memory with a TMA store.
__device__ __forceinline__ void warp_tile_store(uint32_t stage, const uint32_t (&pk)[16],
                                               const CUtensorMap* map, int x, int y, int z,
                                               uint64_t policy, int lane) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int phys = q ^ ((lane >> 1) & 3);
    st_shared_v4(stage + lane * 64 + phys * 16, pk[4 * q], pk[4 * q + 1], pk[4 * q + 2],
                 pk[4 * q + 3]);
  }
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    tma_store_3d(map, stage, x, y, z, policy);
    bulk_commit_group();
  }
}

// ============================================================================
// tc_gram_p: G, then P into the workspace.
// ============================================================================
template <typename T>
__global__ void __launch_bounds__(kLgThreads, 2)
    tc_gram_p(const FwdArgs args, const __grid_constant__ CUtensorMap map_k,
              const __grid_constant__ CUtensorMap map_pst, const LongGeom geom) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* base_ptr = smem_raw + (base - raw);
  const uint32_t stage_addr = base;  // TMA stages; P staging tiles once the Gram is complete
  LgCtrl* ctrl = reinterpret_cast<LgCtrl*>(base_ptr + kLgStages * kLgStageBytes);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int C = args.ctx, D = args.feat;
  const int b = blockIdx.y;
  // Item -> (query tile, key group), query tiles in order.
  int qt = 0, kg = blockIdx.x;
  for (; qt < geom.n_qtiles; ++qt) {
    const int ng = lg_groups(qt, C, args.causal);
    if (kg < ng) break;
    kg -= ng;
  }
  const int q_lo = qt * 128;
  const int key0 = kg * kLgGroupKeys;

  if (tid == 0) {
    for (int s = 0; s < kLgStages; ++s) {
      mbar_init(smem_u32(&ctrl->full[s]), 1);
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
  for (int j = tid; j < kLgGroupKeys; j += kLgThreads)
    ctrl->kvalid[j] = static_cast<uint8_t>(pos_valid(args, b, key0 + j));
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctrl->tmem_base;

  const int kv_end = ctrl->last_valid + 1;
  const int nkeys = args.causal ? min(kv_end, q_lo + 128) : kv_end;
  const bool skip = q_lo >= kv_end || key0 >= nkeys;
  const int nk = skip ? 0 : min(kLgGroupTiles, (nkeys - key0 + 127) / 128);  // key tiles here
  const int q_in = (qt * 128 >= key0 && qt * 128 < key0 + nk * 128) ? (qt - key0 / 128) : -1;
  const int nchunk = (D + kTcChunk - 1) / kTcChunk;
  const uint32_t fmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;

  if (warp == 0) {
    if (!skip && lane == 0) {
      // ---- TMA producer: key tiles of the group (+ the query tile when it is
      // not one of them), one 64-feature chunk per stage.
      const uint64_t keep = l2_policy_evict_last();
      const uint32_t bytes = (nk + (q_in < 0 ? 1 : 0)) * kTcTileBytesA;
      int st = 0;
      uint32_t ph = 0;
      for (int c = 0; c < nchunk; ++c) {
        if (c >= kLgStages) mbar_wait(smem_u32(&ctrl->empty[st]), ph ^ 1u);
        const uint32_t full = smem_u32(&ctrl->full[st]);
        const uint32_t sa = stage_addr + st * kLgStageBytes;
        mbar_arrive_expect_tx(full, bytes);
        for (int t = 0; t < nk; ++t)
          tma_load_3d_hint(sa + t * kTcTileBytesA, &map_k, full, c * kTcChunk, key0 + t * 128, b,
                           keep);
        if (q_in < 0)
          tma_load_3d_hint(sa + nk * kTcTileBytesA, &map_k, full, c * kTcChunk, q_lo, b, keep);
        if (++st == kLgStages) {
          st = 0;
          ph ^= 1u;
        }
      }
    }
  } else if (warp == 1) {
    if (!skip && lane == 0) {
      // ---- MMA issuer: G[128 x 128 nk] in TMEM columns [0, 128 nk).
      const uint64_t d0 = smem_desc_sw128(stage_addr, 16, 1024);
      const uint32_t q_adv = static_cast<uint32_t>((q_in >= 0 ? q_in : nk) * kTcTileBytesA) >> 4;
      const uint32_t idesc_g1 = idesc_f16(fmt, 128, nk >= 2 ? 256 : 128, 0, 0);
      int st = 0;
      uint32_t ph = 0;
      for (int c = 0; c < nchunk; ++c) {
        mbar_wait(smem_u32(&ctrl->full[st]), ph);
        tc_fence_after();
        const uint64_t dk = d0 + static_cast<uint32_t>(st * kLgStageBytes >> 4);
        const uint64_t dq = dk + q_adv;
#pragma unroll
        for (int k = 0; k < kTcChunk / 16; ++k) {
          const uint32_t acc = (c != 0 || k != 0) ? 1u : 0u;
          tc_mma_f16(tmem, dq + 2 * k, dk + 2 * k, idesc_g1, acc);  // key tiles 0 and 1
        }
        tc_commit(smem_u32(&ctrl->empty[st]));
        if (++st == kLgStages) {
          st = 0;
          ph ^= 1u;
        }
      }
      tc_commit(smem_u32(&ctrl->s_full));
    }
  } else if (warp >= 4) {
    // ---- compute warps: inverse norms, then P chunks into the workspace.
    const int cw = warp - 4, wq = warp & 3;
    const int row = wq * 32 + lane, i = q_lo + row;
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    if (!skip) {
      griddep_wait();  // the row sums of squares come from norm_prepass
      const float* ssq = args.sumsq + static_cast<int64_t>(b) * C;
      const int tid_c = cw * 32 + lane;
      int nonfinite = 0;
      for (int j = tid_c; j < nk * 128; j += 128 * kLgWG) {
        const int key = key0 + j;
        const float s2 = key < C ? ssq[key] : 0.f;
        if (key < C && !isfinite(s2)) nonfinite = 1;
        ctrl->rinv[j] = (key < nkeys && ctrl->kvalid[j]) ? 1.f / fmaxf(sqrtf(s2), args.norm_eps_f) : 0.f;
      }
      if (tid_c < kLgGroupKeys / 32) {
        uint32_t m = 0u;
        for (int e = 0; e < 32; ++e) {
          const int j = tid_c * 32 + e;
          if (key0 + j < nkeys && ctrl->kvalid[j]) m |= 1u << e;
        }
        ctrl->kbits[tid_c] = m;
      }
      // The query rows' own finiteness (they need not be keys of this group).
      const bool row_ok = i < C && pos_valid(args, b, i);
      const float s2q = i < C ? ssq[i] : 0.f;
      if (i < C && !isfinite(s2q)) nonfinite = 1;
      if (nonfinite) ctrl->exact = 1;
      named_bar_sync(1, 128 * kLgWG);
      const float rqi = row_ok ? 1.f / fmaxf(sqrtf(s2q), args.norm_eps_f) : 0.f;
      const T* vrow = (args.has_v && i < C)
                          ? static_cast<const T*>(args.v) + static_cast<int64_t>(i) * args.v_rs + key0
                          : nullptr;
      const bool v_vec = (reinterpret_cast<uintptr_t>(args.v) & 15u) == 0 && (args.v_rs & 7) == 0;
      const uint64_t keep = l2_policy_evict_last();
      const uint64_t stream = l2_policy_evict_normal();
      // The warpgroup covers every key of the group, 32 per chunk.
      const int c_begin = 0;
      const int nch = nk * 4;
      const uint32_t one2 = pack2<T>(1.f, 1.f);
      uint32_t vw[16], vn[16], vnn[16];
#pragma unroll
      for (int q = 0; q < 16; ++q) vw[q] = vn[q] = vnn[q] = one2;
      const int vlim = C - key0;  // valid V columns from this group's first key
      if (vrow) {
        load_raw32<T>(vrow + c_begin, vlim - c_begin, v_vec, vw, keep);
        if (nch > 1) load_raw32<T>(vrow + c_begin + 32, vlim - c_begin - 32, v_vec, vn, keep);
      }
      mbar_wait(smem_u32(&ctrl->s_full), 0);
      tc_fence_after();
      const bool exact = ctrl->exact != 0 || (args.has_valid && args.has_v);
      const int i0 = q_lo + wq * 32;
      const bool norm = args.normalize;
      float den4[4] = {0.f, 0.f, 0.f, 0.f};
      // The stage ring is idle once the Gram is complete: two staging tiles per warp.
      const uint32_t stage0 = stage_addr + cw * 2 * kTcOutTileBytes;
#pragma unroll 1
      for (int ch = 0; ch < nch; ++ch) {
        const int c0 = c_begin + ch * 32;
        uint32_t g[32];
        tmem_ld32(tmem + lane_off + c0, g);
        if (vrow && ch + 2 < nch) load_raw32<T>(vrow + c0 + 64, vlim - c0 - 64, v_vec, vnn, keep);
        const bool masked = exact || (args.causal && key0 + c0 + 31 > i0);
        uint32_t okb = 0u;
        if (masked) {
          okb = row_ok ? ctrl->kbits[c0 >> 5] : 0u;
          if (args.causal) {
            const int lim = i - (key0 + c0) + 1;
            okb &= lim >= 32 ? 0xFFFFFFFFu : (lim <= 0 ? 0u : ((1u << lim) - 1u));
          }
        }
        float rk[32];  // the chunk's inverse key norms, loaded while the TMEM load is in flight
        load_f32x32(&ctrl->rinv[c0], rk);
        tmem_wait_ld(g);
        uint32_t pk[16];
        if (args.has_v) {
          if (masked) {
            if (norm) p_chunk<T, true, true, true>(g, rk, rqi, vw, okb, pk, den4);
            else p_chunk<T, true, false, true>(g, rk, rqi, vw, okb, pk, den4);
          } else {
            if (norm) p_chunk<T, false, true, true>(g, rk, rqi, vw, okb, pk, den4);
            else p_chunk<T, false, false, true>(g, rk, rqi, vw, okb, pk, den4);
          }
        } else {
          if (masked) {
            if (norm) p_chunk<T, true, true, false>(g, rk, rqi, vw, okb, pk, den4);
            else p_chunk<T, true, false, false>(g, rk, rqi, vw, okb, pk, den4);
          } else {
            if (norm) p_chunk<T, false, true, false>(g, rk, rqi, vw, okb, pk, den4);
            else p_chunk<T, false, false, false>(g, rk, rqi, vw, okb, pk, den4);
          }
        }
        // The store two chunks back must have read its staging tile.
        if (lane == 0) bulk_wait_read_1();
        __syncwarp();
        if (key0 + c0 < C && i0 < C)  // the box holds some of the tensor
          warp_tile_store(stage0 + (ch & 1) * kTcOutTileBytes, pk, &map_pst, key0 + c0, i0, b,
                          keep, lane);  // P is read back by tc_pv soon: keep it in L2
        if (vrow) {
#pragma unroll
          for (int q = 0; q < 16; ++q) {
            vw[q] = vn[q];
            vn[q] = vnn[q];
          }
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
// tc_pv: O = P Z per 256-feature group, then the epilogue.
// ============================================================================
template <typename T, int ACT>
__global__ void __launch_bounds__(kPvThreads, 2)
    tc_pv(const FwdArgs args, const __grid_constant__ CUtensorMap map_p,
          const __grid_constant__ CUtensorMap map_z, const __grid_constant__ CUtensorMap map_o,
          const LongGeom geom) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  uint8_t* base_ptr = smem_raw + (base - raw);
  const uint32_t ring = base;  // TMA stages; output staging tiles in the epilogue
  PvCtrl* ctrl = reinterpret_cast<PvCtrl*>(base_ptr + kPvStages * kPvStageBytes);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int C = args.ctx, D = args.feat;
  const int b = blockIdx.y;
  // Longest items first under the causal mask (later query tiles have more keys).
  const int qi = blockIdx.x / geom.n_fgroups, fg = blockIdx.x % geom.n_fgroups;
  const int qt = args.causal ? geom.n_qtiles - 1 - qi : qi;
  const int q_lo = qt * 128;
  const int f_lo = fg * kPvGroupCols;
  const int width = min(kPvGroupCols, D - f_lo);

  if (tid == 0) {
    for (int s = 0; s < kPvStages; ++s) {
      mbar_init(smem_u32(&ctrl->full[s]), 1);
      mbar_init(smem_u32(&ctrl->empty[s]), 1);
      mbar_init(smem_u32(&ctrl->fixed[s]), 4);  // warps 4-7, in fix mode
    }
    mbar_init(smem_u32(&ctrl->o_full), 1);
    ctrl->last_valid = -1;
    ctrl->fix = 0;
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
    for (int f = tid; f < width; f += kPvThreads)
      ctrl->bias[f] = to_f32<T>(static_cast<const T*>(args.bias)[f_lo + f]);
  __syncthreads();
  const int kv_end = ctrl->last_valid + 1;
  const int nkeys = args.causal ? min(kv_end, q_lo + 128) : kv_end;
  const bool skip = q_lo >= kv_end;
  const int nkc = skip ? 0 : (nkeys + kPvChunkKeys - 1) / kPvChunkKeys;
  const int nfb = (width + 63) / 64;
  const uint32_t fmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
  // The MMA reads whole 64-key chunks. With a padding mask some of their key
  // rows are outside the allowed set: P is exactly zero there, but 0 * Inf or
  // 0 * NaN in a padded row of z_tr would still reach O. If any such row is
  // not finite (its sum of squares, from norm_prepass, which completed before
  // the G/P launch did), warps 4-7 zero those rows of every stage before the
  // MMA reads it.
  if (!skip && args.has_valid) {
    const float* ssq = args.sumsq + static_cast<int64_t>(b) * C;
    const int kend = min(C, nkc * kPvChunkKeys);
    int bad = 0;
    for (int j = tid; j < kend; j += kPvThreads)
      if (!(j < nkeys && pos_valid(args, b, j)) && !isfinite(ssq[j])) bad = 1;
    if (bad) ctrl->fix = 1;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctrl->tmem_base;
  const bool fix = ctrl->fix != 0;

  if (warp == 0) {
    if (!skip && lane == 0) {
      const uint64_t keep = l2_policy_evict_last();
      const uint32_t bytes = kPvABytes + nfb * kPvBBoxBytes;
      int st = 0;
      uint32_t ph = 0;
      for (int kc = 0; kc < nkc; ++kc) {
        if (kc >= kPvStages) mbar_wait(smem_u32(&ctrl->empty[st]), ph ^ 1u);
        const uint32_t full = smem_u32(&ctrl->full[st]);
        const uint32_t sa = ring + st * kPvStageBytes;
        mbar_arrive_expect_tx(full, bytes);
        tma_load_3d(sa, &map_p, full, kc * kPvChunkKeys, q_lo, b);
        for (int i = 0; i < nfb; ++i)
          tma_load_3d_hint(sa + kPvABytes + i * kPvBBoxBytes, &map_z, full, f_lo + i * 64,
                           kc * kPvChunkKeys, b, keep);
        if (++st == kPvStages) {
          st = 0;
          ph ^= 1u;
        }
      }
    }
  } else if (warp == 1) {
    if (!skip && lane == 0) {
      const uint64_t d0 = smem_desc_sw128(ring, 16, 1024);  // A: P, K-major
      const uint64_t e0 = smem_desc_sw128(ring + kPvABytes, kPvBBoxBytes, 1024);  // B: Z, MN-major
      const uint32_t idesc = idesc_f16(fmt, 128, static_cast<uint32_t>((width + 15) & ~15), 0, 1);
      int st = 0;
      uint32_t ph = 0;
      for (int kc = 0; kc < nkc; ++kc) {
        mbar_wait(smem_u32(fix ? &ctrl->fixed[st] : &ctrl->full[st]), ph);
        tc_fence_after();
        const uint32_t adv = static_cast<uint32_t>(st * kPvStageBytes) >> 4;
#pragma unroll
        for (int k = 0; k < kPvChunkKeys / 16; ++k)
          tc_mma_f16(tmem, d0 + adv + 2 * k, e0 + adv + (2048 >> 4) * k, idesc,
                     (kc != 0 || k != 0) ? 1u : 0u);
        tc_commit(smem_u32(&ctrl->empty[st]));
        if (++st == kPvStages) {
          st = 0;
          ph ^= 1u;
        }
      }
      tc_commit(smem_u32(&ctrl->o_full));
    }
  } else if (warp >= 4 && fix && !skip) {
    // Fix mode: zero the Z rows of keys outside the allowed set in each stage.
    const int t = tid - 128;
    int st = 0;
    uint32_t ph = 0;
    for (int kc = 0; kc < nkc; ++kc) {
      mbar_wait(smem_u32(&ctrl->full[st]), ph);
      const uint32_t zb = ring + st * kPvStageBytes + kPvABytes;
      for (int r = t; r < nfb * kPvChunkKeys; r += 128) {
        const int kr = r % kPvChunkKeys, key = kc * kPvChunkKeys + kr;
        if (key < C && !(key < nkeys && pos_valid(args, b, key))) {
          const uint32_t ra = zb + (r / kPvChunkKeys) * kPvBBoxBytes + kr * 128;
#pragma unroll
          for (int q = 0; q < 8; ++q) st_shared_v4(ra + q * 16, 0u, 0u, 0u, 0u);
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&ctrl->fixed[st]));
      if (++st == kPvStages) {
        st = 0;
        ph ^= 1u;
      }
    }
  }
  __syncwarp();  // lanes 1-31 of the producer and MMA warps rejoin lane 0

  // Epilogue: after the last MMA the stage ring is idle, so it holds the
  // output staging tiles (two per warp), and all eight warps drain the
  // accumulator: the warps of one TMEM lane quarter (w and w + 4) take one
  // half of the columns each.
  if (!skip || (warp != 2 && warp != 3)) {  // padded tiles: warps 0, 1, 4-7 write the zeros
    const int wq = warp & 3, half = warp >> 2;
    const int row = wq * 32 + lane, i = q_lo + row;
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    const uint32_t stage_w = ring + warp * 2 * kTcOutTileBytes;
    if (skip) {
      // No valid query row in this tile: its output rows are zero. Each warp
      // zeroes a staging tile and stores it with TMA over its share of the
      // tile's 32 x 32 boxes (the tensor map clips rows past the context and
      // columns past d').
#pragma unroll
      for (int q = 0; q < 4; ++q) st_shared_v4(stage_w + lane * 64 + q * 16, 0u, 0u, 0u, 0u);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        const uint64_t stream = l2_policy_evict_normal();
        const int nbf = (width + 31) / 32, nbr = (min(128, C - q_lo) + 31) / 32;
        const int me = warp < 2 ? warp : warp - 2;  // warps 0, 1, 4..7
        for (int k = me; k < nbf * nbr; k += 6)
          tma_store_3d(&map_o, stage_w, f_lo + (k % nbf) * 32, q_lo + (k / nbf) * 32, b, stream);
        bulk_commit_group();
        bulk_wait_read_all();
      }
    } else {
      griddep_wait();  // P, the partial sums and the sums of squares come from earlier launches
      const bool row_ok = i < C && pos_valid(args, b, i);
      float rqi = 0.f, den = 0.f;
      if (row_ok) {
        rqi = 1.f / fmaxf(sqrtf(args.sumsq[static_cast<int64_t>(b) * C + i]), args.norm_eps_f);
        if (args.normalize) {
          const int ng = (nkeys + kLgGroupKeys - 1) / kLgGroupKeys;
          for (int g = 0; g < ng; ++g)
            den += geom.den_part[(static_cast<int64_t>(b) * geom.n_groups + g) * C + i];
        }
      }
      const float o_scale = kRowScaleInP<T> ? 1.f : rqi;
      const float inv = args.normalize ? o_scale / (o_scale * den + args.eps_f) : o_scale;
      const T* zl = args.has_zl ? static_cast<const T*>(args.z_tl) + static_cast<int64_t>(b) * args.zl_bs
                                : nullptr;
      const T* zrow = (zl && i < C) ? zl + static_cast<int64_t>(i) * args.zl_rs : nullptr;
      const bool zl_vec = zl && (reinterpret_cast<uintptr_t>(args.z_tl) & 15u) == 0 &&
                          (args.zl_rs & 7) == 0 && (args.zl_bs & 7) == 0;
      const uint64_t stream = l2_policy_evict_normal();
      const bool has_bias = args.has_bias;
      // This warp's half of the group's 32-column chunks.
      const int nch = (width + 31) / 32, ch_mid = (nch + 1) / 2;
      const int c_lo = half ? ch_mid * 32 : 0, c_hi = half ? width : min(width, ch_mid * 32);
      uint32_t gn[16];
      if (zrow && c_lo < c_hi) load_raw32<T>(zrow + f_lo + c_lo, D - f_lo - c_lo, zl_vec, gn, stream);
      mbar_wait(smem_u32(&ctrl->o_full), 0);
      tc_fence_after();
#pragma unroll 1
      for (int c0 = c_lo, n = 0; c0 < c_hi; c0 += 32, ++n) {
        uint32_t o[32], gw[16];
        tmem_ld32(tmem + lane_off + c0, o);
#pragma unroll
        for (int q = 0; q < 16; ++q) gw[q] = gn[q];
        if (zrow && c0 + 32 < c_hi) load_raw32<T>(zrow + f_lo + c0 + 32, D - f_lo - c0 - 32, zl_vec, gn, stream);
        float bv[32];
        load_bias32(&ctrl->bias[c0], has_bias, bv);
        tmem_wait_ld(o);
        uint32_t pk[16];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          float yv[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int idx = 4 * q + e;
            float y = act_fn<ACT>(fmaf(__uint_as_float(o[idx]), inv, bv[idx]));
            if (zrow) y *= raw_at<T>(gw, idx);
            yv[e] = row_ok ? y : 0.f;
          }
          pk[2 * q] = pack2<T>(yv[0], yv[1]);
          pk[2 * q + 1] = pack2<T>(yv[2], yv[3]);
        }
        // Two staging tiles: the store two chunks back must have read its tile.
        if (lane == 0) bulk_wait_read_1();
        __syncwarp();
        if (q_lo + wq * 32 < C)
          warp_tile_store(stage_w + (n & 1) * kTcOutTileBytes, pk, &map_o, f_lo + c0,
                          q_lo + wq * 32, b, stream, lane);
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
