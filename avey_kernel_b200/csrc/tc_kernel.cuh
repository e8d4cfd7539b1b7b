// Fused tcgen05 contextualizer kernel for bf16 / f16 inputs (sm_100a).
//
// One CTA owns one work item: 128 query rows (a "query tile") of one batch
// row, and computes the output row block [128, d'] in three phases that keep
// the similarity matrix on chip:
//
//  A. Gram phase. TMA streams 64-feature chunks of the query tile and of every
//     needed key tile (128-byte swizzle) into chunk stages that live in the
//     space of the phase-C ring (unused until phase C). The MMA warp
//     accumulates the raw Gram block G = Z_q Z_k^T (fp32) in TMEM, two key
//     tiles per MMA (N = 256), up to 512 keys = all 512 TMEM columns. The L2
//     normalisation is applied to G in phase B from per-row sums of squares,
//     which the compute warps take from the same phase-A stages while the
//     Gram runs (each stage is released by the MMAs and by them); in the
//     pre-pass variant (given row sums, or norm_prepass running concurrently
//     through programmatic dependent launch) they read them from the
//     workspace instead. No normalised copy of z_tr exists anywhere.
//  B. P phase. The compute warps read G from TMEM (thread = query row), form
//     P = G * rinv_i * rinv_j * V[i, j] under the causal / padding masks
//     (select, so NaN padding cannot leak), accumulate the signed row sum for
//     Avey-B in fp32, and write P back into TMEM as packed bf16 / f16 pairs
//     (tcgen05.st), over Gram columns the same thread has already read. P never
//     leaves the tensor memory.
//  C. Mix phase. TMA streams z_tr again as 64-key x 128-feature units (MN-major
//     B operand, 128-byte swizzle) through a 12-slot ring. The MMA warp computes
//     O = P Z with P read from TMEM (tcgen05.mma A-from-TMEM) for 128-feature
//     slices into two 128-column TMEM buffers. The compute warps drain each
//     slice: divide by (den + eps), add the bias, apply the activation,
//     multiply by the gate, zero padded rows, and write the tile through
//     shared memory with a TMA tensor store.
//
// Roles: warp 0 issues TMA (and L2 prefetches of the item's V rows and gate
// rows), warp 1 owns TMEM and issues MMAs, warps 4-11 are the compute warps
// (two warpgroups; warpgroup h drains slices s = h mod 2). Every wait is
// bounded (ptx.cuh): a wait that gives up raises the device flag, and all
// later waits in the grid return at once, so the kernel always terminates and
// frees its TMEM.
//
// Reference: the fused loop of avey_kernels/_triton.py:53-128 (S tile 83-92,
// V 93-96, masks 97-100, row sum 101-102, S.Z 103-105, divide 106-107, bias
// 108-110, activation 111-121, gate 122-125, masked store 126-128), plus the
// normalisation pre-pass it relies on (ops.py:107-108), fused here.
#pragma once

#include <cuda.h>

#include <type_traits>

#include "common.cuh"
#include "ptx.cuh"

namespace avey {

constexpr int kTcThreads = 384;
constexpr int kTcMaxKeys = 512;      // keys per work item (TMEM holds 512 fp32 columns)
constexpr int kTcUnitBytes = 32768;  // one phase-C ring slot (128 keys x 128 features)
constexpr int kTcUnitKeys = 128;     // keys per phase-C unit (one key tile)
constexpr int kTcSliceCols = 128;    // output features per phase-C slice (TMEM buffer)
constexpr int kTcOutTileBytes = 2048; // one warp's 32 x 32 output staging tile
constexpr int kTcOutStageBytes = 8 * kTcOutTileBytes;
constexpr int kTcZBoxBytes = 16384;  // one {64 features x 128 keys} box of a unit
constexpr int kTcMaxSlots = 6;
constexpr int kTcMaxStages = 12;  // 192 KB of ring / 16 KB stages (one key tile)
constexpr int kTcChunk = 64;                      // phase-A feature chunk (128-byte rows)
constexpr int kTcTileBytesA = 128 * kTcChunk * 2; // one 128-row tile of a chunk (16 KB)
constexpr int kTcMaxFeatures = 2048;  // bias staged in shared memory
constexpr int kTcCtrlBytes = 13312;

struct TcGeom {
  int nslot;     // phase-C ring slots
  int n_qtiles;  // query tiles per batch row
  int v_tma;     // V tiles reach shared memory by TMA (aligned V), else per-thread loads
  int test_stall;  // test hook: the TMA and MMA warps issue nothing, so waits run out
  int self_sums;   // the compute warps sum the key rows' squares from the phase-A stages
                   // (no row-sum pre-pass; args.sumsq is not read)
};

// TMEM column of the packed P pair holding key j (two keys per 32-bit column).
// With three or four key tiles, keys below 256 pack into [0, 128) and the rest
// into [256, 384): each warpgroup then writes only Gram columns it has already
// read, and [128, 256) / [384, 512) hold the two O buffers. With one or two key
// tiles P goes to [256, 384) and the O buffers to [0, 128) / [128, 256).
__device__ __forceinline__ uint32_t p_col(int j, int nk) {
  return nk >= 3 ? (j < 256 ? j >> 1 : 128 + (j >> 1)) : 256 + (j >> 1);
}
__device__ __forceinline__ uint32_t o_col(int buf, int nk) {
  return nk >= 3 ? (buf ? 384u : 128u) : (buf ? 128u : 0u);
}

// Shared-memory control block.
struct TcCtrl {
  uint64_t a_full[kTcMaxStages], a_empty[kTcMaxStages];
  uint64_t full[kTcMaxSlots], empty[kTcMaxSlots], fixed[kTcMaxSlots];
  uint64_t s_full, p_ready;
  uint64_t o_full[2], o_empty[2];
  uint32_t tmem_base;
  int last_valid;
  int fix;
  int exact;  // some key row's sum of squares is not finite: mask every P chunk exactly
  alignas(16) float rinv[kTcMaxKeys];  // sums of squares, then inverse norms (read as float4)
  float den[2][128];
  uint32_t kbits[kTcMaxKeys / 32];
  uint8_t kvalid[kTcMaxKeys];
  alignas(16) float bias[kTcMaxFeatures];  // read as float4
};
static_assert(sizeof(TcCtrl) <= kTcCtrlBytes, "control block too large");

template <typename T>
__device__ __forceinline__ float to_f32(T x);
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) {
  return __bfloat162float(x);
}
template <>
__device__ __forceinline__ float to_f32<__half>(__half x) {
  return __half2float(x);
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// With bf16 the query row's inverse norm rq is not multiplied into P: P/rq
// keeps bf16's relative precision (same exponent range as fp32), and the
// drain multiplies O by rq instead. fp16 keeps rq in P, whose range bounds it.
template <typename T>
constexpr bool kRowScaleInP = !std::is_same<T, __nv_bfloat16>::value;

// One 32-key chunk of P for this thread's row: P = G * rq * rk * V (rq only
// if kRowScaleInP), packed to 16-bit pairs. MASKED applies the allowed-key
// bits `okb` with a select (so a non-finite product of a masked key still
// gives 0); otherwise keys outside the allowed set already carry rk = 0. NORM
// accumulates the row sums of P; HAS_V multiplies by the weight row.
template <typename T, bool MASKED, bool NORM, bool HAS_V>
__device__ __forceinline__ void p_chunk(const uint32_t (&g)[32], const float (&rk)[32], float rqi,
                                        const uint32_t (&vw)[16], uint32_t okb, uint32_t (&pk)[16],
                                        float (&den)[4]);

// 32 consecutive fp32 values from shared memory, all loaded before any is
// used: shared-memory loads interleaved with arithmetic stall behind the
// tensor core's and TMA's shared-memory traffic (measured on the bias of the
// epilogue: 1.5 us per config-2 forward).
__device__ __forceinline__ void load_f32x32(const float* src, float (&v)[32]) {
  const float4* s4 = reinterpret_cast<const float4*>(src);
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    const float4 x = s4[q];
    v[4 * q] = x.x;
    v[4 * q + 1] = x.y;
    v[4 * q + 2] = x.z;
    v[4 * q + 3] = x.w;
  }
}

// The 32 bias values of one 32-feature output chunk (fp32, staged in shared
// memory), or zeros.
__device__ __forceinline__ void load_bias32(const float* bias, bool has_bias, float (&bv)[32]) {
  if (has_bias) {
    load_f32x32(bias, bv);
  } else {
#pragma unroll
    for (int q = 0; q < 32; ++q) bv[q] = 0.f;
  }
}

// Element e (0..31) of 32 packed 16-bit values.
template <typename T>
__device__ __forceinline__ float raw_at(const uint32_t (&w)[16], int e) {
  const uint32_t word = w[e >> 1];
  const uint16_t h = static_cast<uint16_t>((e & 1) ? (word >> 16) : (word & 0xFFFFu));
  return to_f32<T>(*reinterpret_cast<const T*>(&h));
}

template <typename T, bool MASKED, bool NORM, bool HAS_V>
__device__ __forceinline__ void p_chunk(const uint32_t (&g)[32], const float (&rk)[32], float rqi,
                                        const uint32_t (&vw)[16], uint32_t okb, uint32_t (&pk)[16],
                                        float (&den)[4]) {
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    float pv[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int idx = 4 * q + e;
      float p = __uint_as_float(g[idx]) * rk[idx];
      if (kRowScaleInP<T>) p *= rqi;
      if (HAS_V) p *= raw_at<T>(vw, idx);
      if (MASKED) p = ((okb >> idx) & 1u) ? p : 0.f;
      if (NORM) den[e] += p;
      pv[e] = p;
    }
    pk[2 * q] = pack2<T>(pv[0], pv[1]);
    pk[2 * q + 1] = pack2<T>(pv[2], pv[3]);
  }
}

// The two 16-bit values packed in w (low half first) as fp32.
template <typename T>
__device__ __forceinline__ float2 unpack2(uint32_t w) {
  T h[2];
  memcpy(h, &w, 4);
  return make_float2(to_f32<T>(h[0]), to_f32<T>(h[1]));
}

__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}
__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}
__device__ __forceinline__ uint4 ld_global_nc_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// The 32 weights V[row, c0 .. c0 + 31] of the TMA-staged V tiles: key tile
// c0 / 128 sits in ring slot c0 / 128 as two {64 keys, 128 rows} boxes with
// the 128-byte swizzle (16-byte chunk q of row r at position q ^ (r % 8)).
__device__ __forceinline__ void load_v_tile32(uint32_t ring_addr, int c0, int row, uint32_t (&w)[16]) {
  const int kk = c0 & 127;
  const uint32_t base = ring_addr + static_cast<uint32_t>((c0 >> 7) * kTcUnitBytes + (kk >> 6) * kTcZBoxBytes +
                                                          row * 128);
  const uint32_t j0 = static_cast<uint32_t>((kk & 63) >> 3);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const uint4 v = ld_shared_v4(base + (((j0 + q) ^ static_cast<uint32_t>(row & 7)) << 4));
    w[4 * q] = v.x;
    w[4 * q + 1] = v.y;
    w[4 * q + 2] = v.z;
    w[4 * q + 3] = v.w;
  }
}

// 32 consecutive 16-bit elements starting at p into w[16] (p 16-byte aligned
// when vec); elements at or past n_ok read as zero.
template <typename T>
__device__ __forceinline__ void load_raw32(const T* p, int n_ok, bool vec, uint32_t (&w)[16],
                                           uint64_t policy) {
  if (vec && n_ok >= 32) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint4 v = ld_global_nc_v4_hint(p + 8 * q, policy);
      w[4 * q] = v.x;
      w[4 * q + 1] = v.y;
      w[4 * q + 2] = v.z;
      w[4 * q + 3] = v.w;
    }
  } else {
    const uint16_t* h = reinterpret_cast<const uint16_t*>(p);
#pragma unroll
    for (int e = 0; e < 32; e += 2) {
      const uint32_t lo = e < n_ok ? h[e] : 0u;
      const uint32_t hi = e + 1 < n_ok ? h[e + 1] : 0u;
      w[e >> 1] = lo | (hi << 16);
    }
  }
}

template <typename T, int ACT>
__global__ void __launch_bounds__(kTcThreads, 1)
    tc_contextualize(const FwdArgs args, const __grid_constant__ CUtensorMap map_q,
                     const __grid_constant__ CUtensorMap map_z,
                     const __grid_constant__ CUtensorMap map_o,
                     const __grid_constant__ CUtensorMap map_v, const TcGeom geom) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte alignment for the swizzle atoms.
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* base_ptr = smem_raw + (base - raw_addr);
  // [phase-C ring (phase-A stages before it) | output staging | control block]
  const uint32_t ring_addr = base;
  const uint32_t stage_addr = base;
  const uint32_t out_stage_addr = ring_addr + static_cast<uint32_t>(geom.nslot * kTcUnitBytes);
  TcCtrl* ctrl = reinterpret_cast<TcCtrl*>(base_ptr + geom.nslot * kTcUnitBytes + kTcOutStageBytes);

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int nslot = geom.nslot;
  const int C = args.ctx, D = args.feat, B = args.batch;

  // Work item: causal items with more key tiles come first (longest first).
  const int item = blockIdx.x;
  const int qt = args.causal ? geom.n_qtiles - 1 - item / B : item / B;
  const int b = item % B;
  const int q_lo = qt * 128;


  // ---------------------------------------------------------------- setup
  if (tid == 0) {
    for (int s = 0; s < kTcMaxStages; ++s) {
      mbar_init(smem_u32(&ctrl->a_full[s]), 1);
      // Released by the MMAs' commit, and with self_sums also by every
      // compute warp once it has read the stage.
      mbar_init(smem_u32(&ctrl->a_empty[s]), geom.self_sums ? 9 : 1);
    }
    for (int s = 0; s < kTcMaxSlots; ++s) {
      mbar_init(smem_u32(&ctrl->full[s]), 1);
      mbar_init(smem_u32(&ctrl->empty[s]), 1);
      mbar_init(smem_u32(&ctrl->fixed[s]), 4);
    }
    mbar_init(smem_u32(&ctrl->s_full), 1);
    mbar_init(smem_u32(&ctrl->p_ready), 8);
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&ctrl->o_full[i]), 1);
      mbar_init(smem_u32(&ctrl->o_empty[i]), 8);  // every compute warp, once per slice
    }
    ctrl->last_valid = -1;
    ctrl->fix = 0;
    ctrl->exact = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_q);
    tma_prefetch_desc(&map_z);
    tma_prefetch_desc(&map_o);
    if (geom.v_tma) tma_prefetch_desc(&map_v);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&ctrl->tmem_base), 512);
    tmem_relinquish();
  }
  __syncthreads();
  // Without a pre-pass the launch may overlap the previous kernel of the
  // stream (programmatic dependent launch): the set-up above runs early, and
  // nothing is read from global memory before that kernel has finished.
  if (geom.self_sums) griddep_wait();
  // Key validity of this batch row and the last valid position.
  {
    int last = -1;
    for (int j = tid; j < kTcMaxKeys; j += kTcThreads) {
      const int ok = j < C && mask_ok(args, b, j);
      ctrl->kvalid[j] = static_cast<uint8_t>(ok);
      if (ok) last = j;
    }
    if (last >= 0) atomicMax(&ctrl->last_valid, last);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = ctrl->tmem_base;

  // ---------------------------------------------------------------- geometry
  const int kv_end = ctrl->last_valid + 1;  // == C without a mask
  const bool skip = q_lo >= kv_end;         // no valid query row in this tile
  const int nkeys = args.causal ? min(kv_end, q_lo + 128) : kv_end;
  const int nk = skip ? 0 : (nkeys + 127) / 128;       // key tiles
  const int nchunk = (D + kTcChunk - 1) / kTcChunk;     // phase-A feature chunks
  const int nslices = (D + kTcSliceCols - 1) / kTcSliceCols;  // output slices (phase C)
  const int nunits = skip ? 0 : (nkeys + kTcUnitKeys - 1) / kTcUnitKeys;  // units per slice
  const int units_c = nslices * nunits;
  const uint32_t fmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
  // Phase-A stages of this item: one 16 KB tile per key tile, as many stages
  // as the ring holds (up to 12 with one key tile).
  const int a_stage_bytes = max(nk, 1) * kTcTileBytesA;
  const int nst = min(kTcMaxStages, (nslot * kTcUnitBytes) / a_stage_bytes);
  // With an aligned V, its tiles (128 query rows x 128 keys, 32 KB each) take
  // the first nk ring slots after the Gram; the mix units follow them.
  const int nvt = (geom.v_tma && args.has_v && !skip) ? nk : 0;
  // Phase-C ring entries in order: the V tiles, then the units slice by slice.
  auto e_unit = [&](int s, int u) { return nvt + s * nunits + u; };

  if (warp == 0) {
    // ============================================================ TMA producer
    // One lane walks the whole schedule (a per-step branch on the lane index
    // would cost a reconvergence every step). Slot indices and barrier
    // parities advance incrementally (no divisions in the hot loop).
    if (!skip && lane == 0 && !geom.test_stall) {
      const uint64_t keep = l2_policy_evict_last();  // z_tr is read again (phase C, other CTAs)
      // Phase-A stage state.
      int a_st = 0, a_use = 0, c = 0;
      // Phase-A stages (bit per stage) released for the last time so far.
      uint32_t released = 0u;
      // Phase-C ring entry e goes to slot e % nslot once the slot's previous
      // entry (e - nslot) has been released on empty[] (its phase
      // (e / nslot) - 1); a slot's first entry waits only for the last use of
      // the phase-A stages that overlap its bytes, so V tiles and early units
      // load while the Gram's last chunks still run.
      auto claim = [&](int e) -> int {
        const int slot = e % nslot;
        if (e >= nslot) {
          mbar_wait(smem_u32(&ctrl->empty[slot]), ((e / nslot) - 1) & 1);
        } else {
          const int lo = (slot * kTcUnitBytes) / a_stage_bytes;
          const int hi = min(((slot + 1) * kTcUnitBytes - 1) / a_stage_bytes, min(nst, nchunk) - 1);
          for (int st_i = lo; st_i <= hi; ++st_i) {
            if ((released >> st_i) & 1u) continue;
            const int uses = (nchunk - st_i + nst - 1) / nst;  // chunks that went to stage st_i
            mbar_wait(smem_u32(&ctrl->a_empty[st_i]), (uses - 1) & 1);
            released |= 1u << st_i;
          }
        }
        return slot;
      };
      auto load_stage = [&]() {
        if (a_use > 0) mbar_wait(smem_u32(&ctrl->a_empty[a_st]), (a_use - 1) & 1);
        {
          const uint32_t full = smem_u32(&ctrl->a_full[a_st]);
          const uint32_t st = stage_addr + a_st * a_stage_bytes;
          // Key tiles 0 .. nk-1; the query tile is key tile qt (qt < nk in
          // both modes), so it is not loaded a second time.
          mbar_arrive_expect_tx(full, nk * kTcTileBytesA);
          for (int t = 0; t < nk; ++t)
            tma_load_3d_hint(st + t * kTcTileBytesA, &map_q, full, c * kTcChunk, t * 128, b, keep);
        }
        ++c;
        if (++a_st == nst) {
          a_st = 0;
          ++a_use;
        }
      };
      // Phase-A stages occupy the ring space: each phase-C entry claims its
      // slot only after the stages under it are released (claim above).
      while (c < nchunk) load_stage();
      // V tiles for the P phase: two {64 keys, 128 rows} boxes per key tile.
      for (int t = 0; t < nvt; ++t) {
        const int slot = claim(t);
        const uint32_t full = smem_u32(&ctrl->full[slot]);
        mbar_arrive_expect_tx(full, kTcUnitBytes);
        for (int bx = 0; bx < 2; ++bx)
          tma_load_3d_hint(ring_addr + slot * kTcUnitBytes + bx * kTcZBoxBytes, &map_v, full,
                           t * kTcUnitKeys + bx * 64, q_lo, 0, keep);
      }
      for (int sl = 0; sl < nslices; ++sl) {
        const int nbox = (min(kTcSliceCols, D - sl * kTcSliceCols) + 63) / 64;
        for (int uu = 0; uu < nunits; ++uu) {
          const int slot = claim(e_unit(sl, uu));
          const uint32_t full = smem_u32(&ctrl->full[slot]);
          const uint32_t dst = ring_addr + slot * kTcUnitBytes;
          mbar_arrive_expect_tx(full, nbox * kTcZBoxBytes);
          for (int i = 0; i < nbox; ++i)
            tma_load_3d_hint(dst + i * kTcZBoxBytes, &map_z, full, sl * kTcSliceCols + i * 64,
                             uu * kTcUnitKeys, b, keep);
        }
      }
    }
  } else if (warp == 1) {
    // ============================================================ MMA issuer
    // One lane issues everything (see the producer).
    if (!skip && lane == 0 && !geom.test_stall) {
      // Descriptors are advanced by adding (byte offset >> 4) to the start
      // address field; every address stays below 2^18, so nothing carries out.
      const uint64_t dq0 = smem_desc_sw128(stage_addr, 16, 1024);
      const uint32_t stage_adv = static_cast<uint32_t>(a_stage_bytes) >> 4;
      const uint32_t q_adv = static_cast<uint32_t>(qt * kTcTileBytesA) >> 4;
      const uint32_t idesc_g256 = idesc_f16(fmt, 128, 256, 0, 0);
      const uint32_t idesc_g128 = idesc_f16(fmt, 128, 128, 0, 0);
      const uint32_t idesc_g1 = nk >= 2 ? idesc_g256 : idesc_g128;
      const uint32_t idesc_g2 = nk >= 4 ? idesc_g256 : idesc_g128;
      int st = 0;
      uint32_t ph = 0;
      for (int c = 0; c < nchunk; ++c) {
        mbar_wait(smem_u32(&ctrl->a_full[st]), ph);
        tc_fence_after();
        {
          const uint64_t dk = dq0 + st * stage_adv;  // key tile 0 of this stage
          const uint64_t dq = dk + q_adv;              // the query tile (key tile qt)
          // Four 16-feature K steps (32 bytes each inside the 128-byte swizzled
          // rows); key tiles (0,1) and (2,3) are each one N = 256 MMA.
#pragma unroll
          for (int k = 0; k < kTcChunk / 16; ++k) {
            const uint32_t acc = (c != 0 || k != 0) ? 1u : 0u;
            tc_mma_f16(tmem, dq + 2 * k, dk + 2 * k, idesc_g1, acc);
            if (nk > 2)
              tc_mma_f16(tmem + 256, dq + 2 * k, dk + (2 * kTcTileBytesA >> 4) + 2 * k, idesc_g2,
                         acc);
          }
          tc_commit(smem_u32(&ctrl->a_empty[st]));
        }
        if (++st == nst) {
          st = 0;
          ph ^= 1u;
        }
      }
      tc_commit(smem_u32(&ctrl->s_full));
      mbar_wait(smem_u32(&ctrl->p_ready), 0);
      tc_fence_after();
      const bool fix = ctrl->fix != 0;
      const uint64_t dz0 = smem_desc_sw128(ring_addr, kTcZBoxBytes, 1024);
      uint32_t fpar = 0u;  // per slot: parity of the units it has held (phases of fixed[])
      for (int s = 0; s < nslices; ++s) {
        const int buf = s & 1;
        if (s >= 2) {
          mbar_wait(smem_u32(&ctrl->o_empty[buf]), ((s >> 1) - 1) & 1);
          tc_fence_after();
        }
        const int width = min(kTcSliceCols, D - s * kTcSliceCols);
        const uint32_t idesc_o = idesc_f16(fmt, 128, static_cast<uint32_t>((width + 15) & ~15), 0, 1);
        const uint32_t d_tmem = tmem + o_col(buf, nk);
        for (int uu = 0; uu < nunits; ++uu) {
          const int e = e_unit(s, uu);
          const int slot = e % nslot;
          if (fix) {
            mbar_wait(smem_u32(&ctrl->fixed[slot]), (fpar >> slot) & 1u);
            fpar ^= 1u << slot;
          }
          else mbar_wait(smem_u32(&ctrl->full[slot]), (e / nslot) & 1);
          tc_fence_after();
          {
            // P keys 128 uu .. +127 start at TMEM column p_col(128 uu); K steps
            // of 16 keys advance 8 columns of P and 16 rows (2 KB) of the Z unit.
            const uint32_t a_tmem = tmem + p_col(uu * kTcUnitKeys, nk);
            const uint64_t dz = dz0 + slot * (kTcUnitBytes >> 4);
#pragma unroll
            for (int k = 0; k < kTcUnitKeys / 16; ++k)
              tc_mma_f16_ts(d_tmem, a_tmem + 8 * k, dz + k * (2048 >> 4), idesc_o,
                            (uu != 0 || k != 0) ? 1u : 0u);
            tc_commit(smem_u32(&ctrl->empty[slot]));
          }
        }
        tc_commit(smem_u32(&ctrl->o_full[buf]));
      }
    }
  } else if (warp >= 4) {
    // ============================================================ compute warps
    const int cw = warp - 4;        // 0..7
    const int h = cw >> 2;          // warpgroup
    const int wq = warp & 3;        // TMEM lane quarter
    const int row = wq * 32 + lane; // query row within the tile
    const int i = q_lo + row;
    const uint32_t lane_off = static_cast<uint32_t>(wq * 32) << 16;
    const T* zl = args.has_zl ? static_cast<const T*>(args.z_tl) + static_cast<int64_t>(b) * args.zl_bs
                              : nullptr;
    T* out = static_cast<T*>(args.out) + static_cast<int64_t>(b) * args.o_bs;

    if (skip) {
      // Every query row of this tile is padding: the output rows are zero.
      // Each warp zeroes its 32 x 32 staging tile and stores it with TMA over
      // its share of the tile's 32 x 32 boxes (the tensor map clips columns
      // past d' and rows past the context).
      const uint32_t stage_z = out_stage_addr + cw * kTcOutTileBytes;
#pragma unroll
      for (int q = 0; q < 4; ++q) st_shared_v4(stage_z + lane * 64 + q * 16, 0u, 0u, 0u, 0u);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        const uint64_t stream = l2_policy_evict_normal();
        const int nbf = (D + 31) / 32, nbr = (min(128, C - q_lo) + 31) / 32;
        for (int k = cw; k < nbf * nbr; k += 8)
          tma_store_3d(&map_o, stage_z, (k % nbf) * 32, q_lo + (k / nbf) * 32, b, stream);
        bulk_commit_group();
        bulk_wait_read_all();
      }
      (void)out;
    } else {
      // Warm L2 with the gate of this warpgroup's part of the first output
      // slice (columns 64 h .. 64 h + 63); each drain warms the next slice's.
      // Warming the whole row here measured slower: the lines are evicted
      // again before phase C.
      if (args.has_zl && i < C && h * 64 < D) {
        const char* grow = reinterpret_cast<const char*>(zl + static_cast<int64_t>(i) * args.zl_rs +
                                                         h * 64);
        const int nbytes = min(64, D - h * 64) * 2;
        for (int l = 0; l < nbytes; l += 128) asm volatile("prefetch.global.L2 [%0];" ::"l"(grow + l));
      }
      // ---------------- phase A (compute warps): sums of squares of the key rows.
      if (geom.self_sums) {
        // From the phase-A stages, as the Gram consumes them: thread tid_c sums
        // key rows tid_c and tid_c + 256 over every 64-feature chunk. A row's
        // 128 bytes hold its 8 granules of 16 bytes in swizzled order (granule
        // g at g ^ (row & 7)); visiting granule k ^ (row & 7) at step k keeps
        // the 8 rows of each access phase on distinct banks.
        const int tid_c = cw * 32 + lane;
        float ss[2] = {0.f, 0.f};
        int st = 0;
        uint32_t ph = 0;
        for (int c = 0; c < nchunk; ++c) {
          const bool ok = mbar_wait(smem_u32(&ctrl->a_full[st]), ph);
          if (ok) {
            const uint32_t stage = stage_addr + st * a_stage_bytes;
#pragma unroll
            for (int q = 0; q < 2; ++q) {
              const int j = tid_c + 256 * q;
              if (j < nk * 128) {
                const uint32_t rowa = stage + (j >> 7) * kTcTileBytesA + (j & 127) * 128;
#pragma unroll
                for (int k = 0; k < 8; ++k) {
                  const uint4 v = ld_shared_v4(rowa + ((k ^ (j & 7)) << 4));
                  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                  for (int e = 0; e < 4; ++e) {
                    const float2 f = unpack2<T>(w[e]);
                    ss[q] = fmaf(f.x, f.x, fmaf(f.y, f.y, ss[q]));
                  }
                }
              }
            }
          }
          __syncwarp();
          if (lane == 0) mbar_arrive(smem_u32(&ctrl->a_empty[st]));
          if (++st == nst) {
            st = 0;
            ph ^= 1u;
          }
        }
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          const int j = tid_c + 256 * q;
          if (j < nk * 128) ctrl->rinv[j] = j < C ? ss[q] : 0.f;
        }
      } else {
        // From the row-sum pre-pass, which may still be running (programmatic
        // dependent launch): wait for it only here.
        griddep_wait();
        const float* ssq = args.sumsq + static_cast<int64_t>(b) * C;
        for (int j = cw * 32 + lane; j < nk * 128; j += 256) ctrl->rinv[j] = j < C ? ssq[j] : 0.f;
      }
      named_bar_sync(1, 256);
      {
        const int tid_c = cw * 32 + lane;
        const float norm_eps = args.norm_eps_f;
        int bad = 0, nonfinite = 0;
        for (int j = tid_c; j < nk * 128; j += 256) {
          const float s2 = ctrl->rinv[j];
          if (j < C && !isfinite(s2)) {
            nonfinite = 1;
            // Padded rows holding Inf / NaN would poison P.Z (0 * NaN): flag them.
            if (!ctrl->kvalid[j]) bad = 1;
          }
          // Keys outside the allowed set (padding, past nkeys) get a zero
          // inverse norm, which zeroes their P column without a select.
          ctrl->rinv[j] = (j < nkeys && ctrl->kvalid[j]) ? 1.f / fmaxf(sqrtf(s2), norm_eps) : 0.f;
        }
        if (bad) ctrl->fix = 1;
        if (nonfinite) ctrl->exact = 1;
        // Key bitmask: bit e of word w <=> key 32 w + e is valid and < nkeys.
        if (tid_c < kTcMaxKeys / 32) {
          uint32_t m = 0u;
          for (int e = 0; e < 32; ++e) {
            const int j = tid_c * 32 + e;
            if (j < nkeys && ctrl->kvalid[j]) m |= 1u << e;
          }
          ctrl->kbits[tid_c] = m;
        }
        if (args.has_bias)
          for (int f = tid_c; f < D; f += 256)
            ctrl->bias[f] = to_f32<T>(static_cast<const T*>(args.bias)[f]);
      }
      named_bar_sync(1, 256);

      // ---------------- phase B: P = G * rinv_i * rinv_j * V, masked, into TMEM
      const bool row_ok = i < C && ctrl->kvalid[i];
      const float rqi = row_ok ? ctrl->rinv[i] : 0.f;
      // V rows by per-thread loads only when its tiles do not come by TMA.
      const T* vrow = (args.has_v && i < C && nvt == 0)
                          ? static_cast<const T*>(args.v) + static_cast<int64_t>(i) * args.v_rs
                          : nullptr;
      const bool v_vec = (reinterpret_cast<uintptr_t>(args.v) & 15u) == 0 && (args.v_rs & 7) == 0;
      const uint64_t keep = l2_policy_evict_last();    // V: read by every batch row
      const uint64_t stream = l2_policy_evict_normal(); // gate and output: touched once
      float den4[4] = {0.f, 0.f, 0.f, 0.f};
      {
        // Key ranges of the two warpgroups (see p_col): with three or four key
        // tiles warpgroup 0 takes keys [0, 256) and warpgroup 1 the rest.
        const int split = nk >= 3 ? 256 : nk * 64;
        const int c_begin = h ? split : 0;
        const int nch = ((h ? nk * 128 : split) - c_begin) / 32;
        // V without a weight matrix is 1.0 everywhere (packed 16-bit ones).
        const uint32_t one2 = pack2<T>(1.f, 1.f);
        uint32_t vw[16], vn[16], vnn[16];
#pragma unroll
        for (int q = 0; q < 16; ++q) vw[q] = vn[q] = vnn[q] = one2;
        // The first two V chunks do not depend on the Gram: load them while
        // the MMAs still run.
        if (vrow) {
          load_raw32<T>(vrow + c_begin, C - c_begin, v_vec, vw, keep);
          if (nch > 1) load_raw32<T>(vrow + c_begin + 32, C - c_begin - 32, v_vec, vn, keep);
        }
        mbar_wait(smem_u32(&ctrl->s_full), 0);
        tc_fence_after();
        for (int t = 0; t < nvt; ++t) mbar_wait(smem_u32(&ctrl->full[t]), 0);
        // Chunks need per-key selects only where a mask bit can be 0 for a key
        // whose zero inverse norm does not already zero the product: keys above
        // the causal diagonal, non-finite rows (0 * Inf), and padded keys when a
        // weight matrix may hold non-finite values there. The choice is uniform
        // per warp (i0 = the warp's first row).
        const bool exact = ctrl->exact != 0 || (args.has_valid && args.has_v);
        const int i0 = q_lo + wq * 32;
        const bool norm = args.normalize;
#pragma unroll 1
        for (int ch = 0; ch < nch; ++ch) {
          const int c0 = c_begin + ch * 32;
          uint32_t g[32];
          tmem_ld32(tmem + lane_off + c0, g);
          if (vrow && ch + 2 < nch) load_raw32<T>(vrow + c0 + 64, C - c0 - 64, v_vec, vnn, keep);
          if (nvt) load_v_tile32(ring_addr, c0, row, vw);
          const bool masked = exact || (args.causal && c0 + 31 > i0);
          uint32_t okb = 0u;
          if (masked) {
            // Allowed keys of this chunk: valid, below nkeys, and j <= i if causal.
            okb = row_ok ? ctrl->kbits[c0 >> 5] : 0u;
            if (args.causal) {
              const int lim = i - c0 + 1;
              okb &= lim >= 32 ? 0xFFFFFFFFu : (lim <= 0 ? 0u : ((1u << lim) - 1u));
            }
          }
          // The chunk's 32 inverse key norms, loaded while the TMEM load is in flight.
          float rk[32];
          load_f32x32(&ctrl->rinv[c0], rk);
          tmem_wait_ld(g);
          uint32_t pk[16];
          if (args.has_v) {  // uniform; rows past the context multiply by ones
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
          // Packed pairs into TMEM columns this thread has already read.
          tmem_st16(tmem + lane_off + p_col(c0, nk), pk);
          if (vrow) {
#pragma unroll
            for (int q = 0; q < 16; ++q) {
              vw[q] = vn[q];
              vn[q] = vnn[q];
            }
          }
        }
      }
      const float den = (den4[0] + den4[1]) + (den4[2] + den4[3]);
      ctrl->den[h][row] = den;
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&ctrl->p_ready));
      named_bar_sync(1, 256);
      if (cw == 0 && lane == 0) {
        // Every compute warp is done with the V tiles: their slots go to the mix units.
        for (int t = 0; t < nvt; ++t) mbar_arrive(smem_u32(&ctrl->empty[t]));
      }
      // O (and the row sums) carry rq only if it went into P.
      const float o_scale = kRowScaleInP<T> ? 1.f : rqi;
      const float inv_den =
          args.normalize ? o_scale / (o_scale * (ctrl->den[0][row] + ctrl->den[1][row]) + args.eps_f)
                         : o_scale;
      const bool fix = ctrl->fix != 0;

      // ---------------- phase C: drain O slices (and, in fix mode, clean units)
      const bool zl_vec = zl && (reinterpret_cast<uintptr_t>(args.z_tl) & 15u) == 0 &&
                          (args.zl_rs & 7) == 0 && (args.zl_bs & 7) == 0;
      const T* zrow = (zl && i < C) ? zl + static_cast<int64_t>(i) * args.zl_rs : nullptr;
      const bool has_bias = args.has_bias;
      // Gate words for the next chunk to drain (prefetched one chunk ahead,
      // across slice boundaries too).
      uint32_t gn[16];
      // Output staging: each compute warp owns a 32-row x 32-column tile (2 KB,
      // 64-byte swizzle) that it fills from registers and writes out with one
      // TMA tensor store; lane 0 tracks the store's bulk group.
      const uint32_t stage_o = out_stage_addr + cw * kTcOutTileBytes;
      auto emit = [&](int f0, const uint32_t (&o)[32], const uint32_t (&gw)[16]) {
        float bv[32];
        load_bias32(&ctrl->bias[f0], has_bias, bv);
        uint32_t pk[16];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          float yv[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int idx = 4 * q + e;
            float y = act_fn<ACT>(fmaf(__uint_as_float(o[idx]), inv_den, bv[idx]));
            if (zrow) y *= raw_at<T>(gw, idx);
            yv[e] = row_ok ? y : 0.f;
          }
          pk[2 * q] = pack2<T>(yv[0], yv[1]);
          pk[2 * q + 1] = pack2<T>(yv[2], yv[3]);
        }
        // The previous store from this tile must have finished reading it.
        if (lane == 0) bulk_wait_read_all();
        __syncwarp();
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int phys = q ^ ((lane >> 1) & 3);  // 64-byte swizzle
          st_shared_v4(stage_o + lane * 64 + phys * 16, pk[4 * q], pk[4 * q + 1], pk[4 * q + 2],
                       pk[4 * q + 3]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_3d(&map_o, stage_o, f0, q_lo + wq * 32, b, stream);
          bulk_commit_group();
        }
      };
      // Drain slice s: chunks [ch_lo, ch_hi) of its 32-column chunks (both
      // warpgroups split every slice, so a slice is drained in half the time
      // and the MMA can refill its buffer sooner). Every compute warp waits
      // for and releases every slice, even with no chunk of it, which keeps
      // the two buffers' phases in step. In fix mode warpgroup 0 drains every
      // chunk alone and releases for both warpgroups.
      const int ch_lo = fix ? 0 : 2 * h, ch_hi = fix ? 4 : 2 * h + 2;
      const uint32_t rel_cnt = fix ? 2u : 1u;
      auto drain = [&](int s) {
        const int buf = s & 1;
        if (zrow && s + 1 < nslices) {
          const int f = (s + 1) * kTcSliceCols + ch_lo * 32;
          const int nbytes = min((ch_hi - ch_lo) * 32, D - f) * 2;
          const char* g2 = reinterpret_cast<const char*>(zrow + f);
          for (int l = 0; l < nbytes; l += 128) asm volatile("prefetch.global.L2 [%0];" ::"l"(g2 + l));
        }
        mbar_wait(smem_u32(&ctrl->o_full[buf]), (s >> 1) & 1);
        tc_fence_after();
        const int width = min(kTcSliceCols, D - s * kTcSliceCols);
        const int nch_o = min(ch_hi, (width + 31) / 32);
        const uint32_t tb = tmem + lane_off + o_col(buf, nk);
        // Gate words of the chunk after `f0` (the rest of this slice's range,
        // then the first chunk of the next slice), prefetched one chunk ahead.
        auto next_gate = [&](int ch, int f0) {
          if (zrow) {
            const int fn = ch + 1 < nch_o ? f0 + 32
                                          : (s + 1 < nslices ? (s + 1) * kTcSliceCols + ch_lo * 32 : D);
            if (fn < D) load_raw32<T>(zrow + fn, D - fn, zl_vec, gn, stream);
          }
        };
        // TMEM loads run one chunk ahead of the math.
        uint32_t oa[32], ob[32], gw[16];
        if (ch_lo < nch_o) tmem_ld32(tb + ch_lo * 32, oa);
#pragma unroll 1
        for (int ch = ch_lo; ch < nch_o; ch += 2) {
          const int f0 = s * kTcSliceCols + ch * 32;
          tmem_wait_ld(oa);
          const bool has_b = ch + 1 < nch_o;
          if (has_b) tmem_ld32(tb + (ch + 1) * 32, ob);
#pragma unroll
          for (int q = 0; q < 16; ++q) gw[q] = gn[q];
          next_gate(ch, f0);
          emit(f0, oa, gw);
          if (has_b) {
            tmem_wait_ld(ob);
            if (ch + 2 < nch_o) tmem_ld32(tb + (ch + 2) * 32, oa);
#pragma unroll
            for (int q = 0; q < 16; ++q) gw[q] = gn[q];
            next_gate(ch + 1, f0 + 32);
            emit(f0 + 32, ob, gw);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cnt(smem_u32(&ctrl->o_empty[buf]), rel_cnt);
      };
      if (zrow && ch_lo * 32 < D)
        load_raw32<T>(zrow + ch_lo * 32, D - ch_lo * 32, zl_vec, gn, stream);
      if (!fix || h == 0) {
        for (int s = 0; s < nslices; ++s) drain(s);
        if (lane == 0) bulk_wait_read_all();
      } else {
        // Fix mode: zero every padded key row of each mix unit before the MMA
        // reads it (warpgroup 1), while warpgroup 0 drains all slices.
        int sl = 0, uu = 0;
        for (int u = 0; u < units_c; ++u) {
          const int nbox = (min(kTcSliceCols, D - sl * kTcSliceCols) + 63) / 64;
          const int e = e_unit(sl, uu);
          const int slot = e % nslot;
          mbar_wait(smem_u32(&ctrl->full[slot]), (e / nslot) & 1);
          // Warpgroup 1 (128 threads) covers the unit's nbox x 64 rows.
          for (int idx = wq * 32 + lane; idx < nbox * kTcUnitKeys; idx += 128) {
            const int r = idx & (kTcUnitKeys - 1), box = idx / kTcUnitKeys;
            const int key = uu * kTcUnitKeys + r;
            if (key < C && !ctrl->kvalid[key]) {
              const uint32_t ra = ring_addr + slot * kTcUnitBytes + box * kTcZBoxBytes + r * 128;
#pragma unroll
              for (int q = 0; q < 8; ++q) st_shared_v4(ra + q * 16, 0u, 0u, 0u, 0u);
            }
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(smem_u32(&ctrl->fixed[slot]));
          if (++uu == nunits) {
            uu = 0;
            ++sl;
          }
        }
      }
    }
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
