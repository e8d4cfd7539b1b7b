// Fused tcgen05 contextualizer kernel for bf16 / f16 inputs (sm_100a).
//
// One CTA owns one work item: 128 query rows (a "query tile") of one batch
// row, and computes the whole output row block [128, d'] in three phases that
// keep the similarity matrix on chip:
//
//  A. Gram phase. TMA streams the query tile and every needed key tile in
//     64-feature chunks (128 x 64 bf16 = 16 KB units, 128-byte swizzle) through
//     a ring of shared-memory slots. The MMA warp accumulates the raw Gram
//     block G = Z_q Z_k^T (fp32) in TMEM, one 128-column tile per key tile
//     (up to 512 keys = all 512 TMEM columns). Meanwhile eight compute warps
//     read each key unit from shared memory and accumulate the row sums of
//     squares: the L2 normalisation is fused here, no normalised copy exists.
//  B. P phase. The compute warps read G from TMEM (thread = query row), form
//     P = G * rinv_i * rinv_j * V[i, j] under the causal / padding masks
//     (select, so NaN padding cannot leak), accumulate the signed row sum for
//     Avey-B in fp32, and write P as bf16 / f16 into shared memory in the
//     K-major 128-byte-swizzle layout the tensor core reads. P never reaches
//     global memory.
//  C. Mix phase. TMA streams z_tr again as 32-key x 256-feature units (MN-major
//     B operand) and the MMA warp computes O = P Z for 256-feature slices into
//     two TMEM buffers (256 columns each, reusing the Gram columns). The
//     compute warps drain each slice: divide by (den + eps), add the bias,
//     apply the activation, multiply by the gate, zero padded rows, store.
//
// Roles: warp 0 issues TMA, warp 1 owns TMEM and issues MMAs, warps 4-11 are
// the compute warps (two warpgroups; warpgroup h drains slices s = h mod 2).
// Every wait is bounded (ptx.cuh): a wait that gives up raises the device
// flag, and all later waits in the grid return at once, so the kernel always
// terminates and frees its TMEM.
//
// Reference: the fused loop of avey_kernels/_triton.py:53-128 (S tile 83-92,
// V 93-96, masks 97-100, row sum 101-102, S.Z 103-105, divide 106-107, bias
// 108-110, activation 111-121, gate 122-125, masked store 126-128), plus the
// normalisation pre-pass it relies on (ops.py:112-113), fused here.
#pragma once

#include <cuda.h>

#include <type_traits>

#include "common.cuh"
#include "ptx.cuh"

namespace avey {

constexpr int kTcThreads = 384;
constexpr int kTcMaxKeys = 512;      // keys per work item (TMEM holds 512 fp32 columns)
constexpr int kTcUnitBytes = 16384;  // one ring slot
constexpr int kTcMaxSlots = 8;
constexpr int kTcCtrlBytes = 4096;

struct TcGeom {
  int nslot;    // ring slots
  int p_bytes;  // bytes of the P region (16 KB per 64 keys)
  int n_qtiles; // query tiles per batch row
};

// Shared-memory control block (offsets in bytes).
struct TcCtrl {
  uint64_t full[kTcMaxSlots];
  uint64_t empty[kTcMaxSlots];
  uint64_t aux[kTcMaxSlots];
  uint64_t fixed[kTcMaxSlots];
  uint64_t s_full, p_ready;
  uint64_t o_full[2], o_empty[2];
  uint32_t tmem_base;
  int last_valid;
  int fix;
  int pad_[1];
  float rinv[kTcMaxKeys];  // sums of squares, then inverse norms
  float den[2][128];
  uint8_t kvalid[kTcMaxKeys];
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

// Unpack 8 16-bit values held in a uint4 to fp32.
template <typename T>
__device__ __forceinline__ void unpack8(const uint4& v, float (&f)[8]) {
  const T* h = reinterpret_cast<const T*>(&v);
#pragma unroll
  for (int i = 0; i < 8; ++i) f[i] = to_f32<T>(h[i]);
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

// Load 32 consecutive elements starting at p (p 16-byte aligned when vec).
template <typename T>
__device__ __forceinline__ void load32(const T* p, int n_ok, bool vec, float (&f)[32]) {
  if (vec && n_ok >= 32) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float t[8];
      unpack8<T>(ld_global_nc_v4(p + 8 * q), t);
#pragma unroll
      for (int e = 0; e < 8; ++e) f[8 * q + e] = t[e];
    }
  } else {
#pragma unroll
    for (int e = 0; e < 32; ++e) f[e] = e < n_ok ? to_f32<T>(p[e]) : 0.f;
  }
}

template <typename T>
__global__ void __launch_bounds__(kTcThreads, 1)
    tc_contextualize(const FwdArgs args, const __grid_constant__ CUtensorMap map_k,
                     const __grid_constant__ CUtensorMap map_z, const TcGeom geom) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte alignment for the 128-byte-swizzle atoms.
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* base_ptr = smem_raw + (base - raw_addr);
  const uint32_t p_addr = base;
  const uint32_t ring_addr = base + static_cast<uint32_t>(geom.p_bytes);
  TcCtrl* ctrl = reinterpret_cast<TcCtrl*>(base_ptr + geom.p_bytes + geom.nslot * kTcUnitBytes);

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int nslot = geom.nslot;
  const int C = args.ctx, D = args.feat, B = args.batch;

  // Work item: causal items with more key tiles come first (longest first).
  const int item = blockIdx.x;
  const int qt = args.causal ? geom.n_qtiles - 1 - item / B : item / B;
  const int b = item % B;
  const int q_lo = qt * 128;

  const uint8_t* va = args.has_valid ? args.valid + static_cast<int64_t>(b) * args.va_bs : nullptr;

  // ---------------------------------------------------------------- setup
  if (tid == 0) {
    for (int s = 0; s < kTcMaxSlots; ++s) {
      mbar_init(smem_u32(&ctrl->full[s]), 1);
      mbar_init(smem_u32(&ctrl->empty[s]), 1);
      mbar_init(smem_u32(&ctrl->aux[s]), 8);
      mbar_init(smem_u32(&ctrl->fixed[s]), 4);
    }
    mbar_init(smem_u32(&ctrl->s_full), 1);
    mbar_init(smem_u32(&ctrl->p_ready), 8);
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_u32(&ctrl->o_full[i]), 1);
      mbar_init(smem_u32(&ctrl->o_empty[i]), 4);
    }
    ctrl->last_valid = -1;
    ctrl->fix = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_k);
    tma_prefetch_desc(&map_z);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&ctrl->tmem_base), 512);
    tmem_relinquish();
  }
  __syncthreads();
  // Key validity of this batch row and the last valid position.
  {
    int last = -1;
    for (int j = tid; j < kTcMaxKeys; j += kTcThreads) {
      const int ok = j < C && (!va || va[static_cast<int64_t>(j) * args.va_rs] != 0);
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
  const int nk = skip ? 0 : (nkeys + 127) / 128;  // key tiles (phase A)
  const int nchunk = (D + 63) / 64;                // feature chunks (phase A)
  const int nslices = (D + 255) / 256;             // output slices (phase C)
  const int nunits = skip ? 0 : (nkeys + 31) / 32; // 32-key units per slice
  const int units_a = nchunk * (1 + nk);
  const uint32_t fmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;

  if (warp == 0) {
    // ============================================================ TMA producer
    if (lane == 0 && !skip) {
      // acount[s]: phase-A units placed in slot s so far; prev_a[s]: the slot's
      // last occupant was a phase-A unit (released by the MMA *and* the
      // compute warps' `aux` arrival).
      uint32_t acount[kTcMaxSlots];
      bool prev_a[kTcMaxSlots];
#pragma unroll
      for (int s = 0; s < kTcMaxSlots; ++s) {
        acount[s] = 0;
        prev_a[s] = false;
      }
      int u = 0;
      auto acquire = [&](int slot, int use) {
        if (use > 0) {
          mbar_wait(smem_u32(&ctrl->empty[slot]), (use - 1) & 1);
          if (prev_a[slot]) mbar_wait(smem_u32(&ctrl->aux[slot]), (acount[slot] - 1) & 1);
        }
      };
      for (int c = 0; c < nchunk; ++c) {
        for (int t = -1; t < nk; ++t) {
          const int slot = u % nslot, use = u / nslot;
          acquire(slot, use);
          const uint32_t full = smem_u32(&ctrl->full[slot]);
          mbar_arrive_expect_tx(full, kTcUnitBytes);
          tma_load_3d(ring_addr + slot * kTcUnitBytes, &map_k, full, c * 64,
                      (t < 0 ? qt : t) * 128, b);
          prev_a[slot] = true;
          ++acount[slot];
          ++u;
        }
      }
      for (int s = 0; s < nslices; ++s) {
        const int width = min(256, D - s * 256);
        const int nbox = (width + 63) / 64;
        for (int uu = 0; uu < nunits; ++uu) {
          const int slot = u % nslot, use = u / nslot;
          acquire(slot, use);
          prev_a[slot] = false;
          const uint32_t full = smem_u32(&ctrl->full[slot]);
          mbar_arrive_expect_tx(full, nbox * 4096);
          for (int i = 0; i < nbox; ++i)
            tma_load_3d(ring_addr + slot * kTcUnitBytes + i * 4096, &map_z, full,
                        s * 256 + i * 64, uu * 32, b);
          ++u;
        }
      }
    }
  } else if (warp == 1) {
    // ============================================================ MMA issuer
    if (lane == 0 && !skip) {
      const uint32_t idesc_g = idesc_f16(fmt, 128, 128, 0, 0);
      int u = 0;
      for (int c = 0; c < nchunk; ++c) {
        const int qslot = u % nslot;
        mbar_wait(smem_u32(&ctrl->full[qslot]), (u / nslot) & 1);
        tc_fence_after();
        const uint32_t qa = ring_addr + qslot * kTcUnitBytes;
        ++u;
        for (int t = 0; t < nk; ++t) {
          const int slot = u % nslot;
          mbar_wait(smem_u32(&ctrl->full[slot]), (u / nslot) & 1);
          tc_fence_after();
          const uint32_t ka = ring_addr + slot * kTcUnitBytes;
#pragma unroll
          for (int k = 0; k < 4; ++k)
            tc_mma_f16(tmem + t * 128, smem_desc_sw128(qa + k * 32, 16, 1024),
                       smem_desc_sw128(ka + k * 32, 16, 1024), idesc_g, (c | k) != 0);
          tc_commit(smem_u32(&ctrl->empty[slot]));
          ++u;
        }
        tc_commit(smem_u32(&ctrl->empty[qslot]));
      }
      tc_commit(smem_u32(&ctrl->s_full));
      mbar_wait(smem_u32(&ctrl->p_ready), 0);
      tc_fence_after();
      const bool fix = ctrl->fix != 0;
      uint32_t fixcount[kTcMaxSlots];
#pragma unroll
      for (int s = 0; s < kTcMaxSlots; ++s) fixcount[s] = 0;
      for (int s = 0; s < nslices; ++s) {
        const int buf = s & 1;
        if (s >= 2) {
          mbar_wait(smem_u32(&ctrl->o_empty[buf]), ((s >> 1) - 1) & 1);
          tc_fence_after();
        }
        const int width = min(256, D - s * 256);
        const uint32_t n_mma = static_cast<uint32_t>((width + 15) & ~15);
        const uint32_t idesc_o = idesc_f16(fmt, 128, n_mma, 0, 1);
        for (int uu = 0; uu < nunits; ++uu) {
          const int slot = u % nslot;
          if (fix)
            mbar_wait(smem_u32(&ctrl->fixed[slot]), (fixcount[slot]++) & 1);
          else
            mbar_wait(smem_u32(&ctrl->full[slot]), (u / nslot) & 1);
          tc_fence_after();
          const uint32_t za = ring_addr + slot * kTcUnitBytes;
#pragma unroll
          for (int k = 0; k < 2; ++k) {
            const int j0 = uu * 32 + k * 16;
            const uint32_t pa = p_addr + (j0 >> 6) * 16384 + ((j0 & 63) >> 4) * 32;
            tc_mma_f16(tmem + buf * 256, smem_desc_sw128(pa, 16, 1024),
                       smem_desc_sw128(za + k * 2048, 4096, 1024), idesc_o, (uu | k) != 0);
          }
          tc_commit(smem_u32(&ctrl->empty[slot]));
          ++u;
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
      const int rows = min(128, C - q_lo);
      for (int e = (cw * 32 + lane) * 8; e < rows * D; e += 256 * 8) {
        for (int k = 0; k < 8 && e + k < rows * D; ++k) {
          const int r = (e + k) / D, f = (e + k) % D;
          out[static_cast<int64_t>(q_lo + r) * args.o_rs + f] = store_cast<T, float>(0.f);
        }
      }
    } else {
      // ---------------- phase A: sums of squares of every key row, from smem
      float ss[4][4];
#pragma unroll
      for (int t = 0; t < 4; ++t)
#pragma unroll
        for (int q = 0; q < 4; ++q) ss[t][q] = 0.f;
      {
        // The compute warps step through every phase-A unit (query units too,
        // without reading them) so that they observe each phase of each slot's
        // barrier in order; the producer waits for their `aux` arrival before
        // refilling a phase-A slot.
        int u = 0;
        for (int c = 0; c < nchunk; ++c) {
          {
            const int slot = u % nslot;
            mbar_wait(smem_u32(&ctrl->full[slot]), (u / nslot) & 1);
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&ctrl->aux[slot]));
            ++u;
          }
          for (int t = 0; t < nk; ++t) {
            const int slot = u % nslot;
            mbar_wait(smem_u32(&ctrl->full[slot]), (u / nslot) & 1);
            const uint32_t ua = ring_addr + slot * kTcUnitBytes;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const int r = cw * 16 + q * 4 + (lane >> 3);
              const int phys = (lane & 7) ^ (r & 7);
              float f[8];
              unpack8<T>(ld_shared_v4(ua + r * 128 + phys * 16), f);
              float s = 0.f;
#pragma unroll
              for (int e = 0; e < 8; ++e) s = fmaf(f[e], f[e], s);
              s += __shfl_xor_sync(0xffffffffu, s, 1);
              s += __shfl_xor_sync(0xffffffffu, s, 2);
              s += __shfl_xor_sync(0xffffffffu, s, 4);
#pragma unroll
              for (int tt = 0; tt < 4; ++tt)
                if (tt == t) ss[tt][q] += s;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&ctrl->aux[slot]));
            ++u;
          }
        }
      }
      if ((lane & 7) == 0) {
#pragma unroll
        for (int t = 0; t < 4; ++t)
#pragma unroll
          for (int q = 0; q < 4; ++q)
            if (t < nk) ctrl->rinv[t * 128 + cw * 16 + q * 4 + (lane >> 3)] = ss[t][q];
      }
      named_bar_sync(1, 256);
      {
        const int tid_c = cw * 32 + lane;
        const float norm_eps = args.norm_eps_f;
        int bad = 0;
        for (int j = tid_c; j < nk * 128; j += 256) {
          const float s2 = ctrl->rinv[j];
          // Padded rows holding Inf / NaN would poison P.Z (0 * NaN): flag them.
          if (j < C && !ctrl->kvalid[j] && !isfinite(s2)) bad = 1;
          ctrl->rinv[j] = 1.f / fmaxf(sqrtf(s2), norm_eps);
        }
        if (bad) ctrl->fix = 1;
      }
      named_bar_sync(1, 256);

      // ---------------- phase B: P = G * rinv_i * rinv_j * V, masked, to smem
      mbar_wait(smem_u32(&ctrl->s_full), 0);
      tc_fence_after();
      const bool row_ok = i < C && ctrl->kvalid[i];
      const float rqi = row_ok ? ctrl->rinv[i] : 0.f;
      const T* vrow = (args.has_v && i < C) ? static_cast<const T*>(args.v) + static_cast<int64_t>(i) * args.v_rs
                                            : nullptr;
      const bool v_vec = (reinterpret_cast<uintptr_t>(args.v) & 15u) == 0 && (args.v_rs & 7) == 0;
      float den = 0.f;
      const int half_cols = nk * 64;
      for (int ch = 0; ch < half_cols / 32; ++ch) {
        const int c0 = h * half_cols + ch * 32;
        uint32_t g[32];
        tmem_ld32(tmem + lane_off + c0, g);
        tmem_wait_ld();
        float vv[32];
        if (vrow)
          load32<T>(vrow + c0, C - c0, v_vec, vv);
        else
#pragma unroll
          for (int e = 0; e < 32; ++e) vv[e] = 1.f;
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          float p2[2];
#pragma unroll
          for (int k = 0; k < 2; ++k) {
            const int j = c0 + e + k;
            const bool ok = row_ok && j < nkeys && ctrl->kvalid[j] && (!args.causal || j <= i);
            const float p = __uint_as_float(g[e + k]) * rqi * ctrl->rinv[j] * vv[e + k];
            p2[k] = ok ? p : 0.f;
            den += p2[k];
          }
          pk[e >> 1] = pack2<T>(p2[0], p2[1]);
        }
        const uint32_t chunk = p_addr + (c0 >> 6) * 16384 + row * 128;
        const int ubase = (c0 & 63) >> 3;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int phys = (ubase + q) ^ (row & 7);
          st_shared_v4(chunk + phys * 16, pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
        }
      }
      ctrl->den[h][row] = den;
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&ctrl->p_ready));
      named_bar_sync(1, 256);
      const float inv_den =
          args.normalize ? 1.f / (ctrl->den[0][row] + ctrl->den[1][row] + args.eps_f) : 1.f;
      const bool fix = ctrl->fix != 0;

      // ---------------- phase C: drain O slices (and, in fix mode, clean units)
      const bool zl_vec = zl && (reinterpret_cast<uintptr_t>(args.z_tl) & 15u) == 0 &&
                          (args.zl_rs & 7) == 0 && (args.zl_bs & 7) == 0;
      const bool o_vec = (reinterpret_cast<uintptr_t>(args.out) & 15u) == 0 &&
                         (args.o_rs & 7) == 0 && (args.o_bs & 7) == 0;
      const bool b_vec = args.has_bias && (reinterpret_cast<uintptr_t>(args.bias) & 15u) == 0;
      auto drain = [&](int s, int buf) {
        mbar_wait(smem_u32(&ctrl->o_full[buf]), (s >> 1) & 1);
        tc_fence_after();
        const int width = min(256, D - s * 256);
        for (int ch = 0; ch < (width + 31) / 32; ++ch) {
          const int f0 = s * 256 + ch * 32;
          uint32_t o[32];
          tmem_ld32(tmem + lane_off + buf * 256 + ch * 32, o);
          tmem_wait_ld();
          if (i >= C) continue;
          float bias[32], gate[32];
          if (args.has_bias)
            load32<T>(static_cast<const T*>(args.bias) + f0, D - f0, b_vec, bias);
          else
#pragma unroll
            for (int e = 0; e < 32; ++e) bias[e] = 0.f;
          if (zl)
            load32<T>(zl + static_cast<int64_t>(i) * args.zl_rs + f0, D - f0, zl_vec, gate);
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            float y2[2];
#pragma unroll
            for (int k = 0; k < 2; ++k) {
              float y = activate<float>(__uint_as_float(o[e + k]) * inv_den + bias[e + k], args.act);
              if (zl) y *= gate[e + k];
              y2[k] = row_ok ? y : 0.f;
            }
            pk[e >> 1] = pack2<T>(y2[0], y2[1]);
          }
          T* dst = out + static_cast<int64_t>(i) * args.o_rs + f0;
          if (o_vec && f0 + 32 <= D) {
#pragma unroll
            for (int q = 0; q < 4; ++q)
              *reinterpret_cast<uint4*>(dst + 8 * q) =
                  make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
          } else {
            const T* hv = reinterpret_cast<const T*>(pk);
            for (int e = 0; e < 32 && f0 + e < D; ++e) dst[e] = hv[e];
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&ctrl->o_empty[buf]));
      };
      if (!fix) {
        for (int s = h; s < nslices; s += 2) drain(s, h);
      } else if (h == 0) {
        for (int s = 0; s < nslices; ++s) drain(s, s & 1);
      } else {
        // Fix mode: zero every padded key row of each mix unit before the MMA
        // reads it (warpgroup 1), while warpgroup 0 drains all slices.
        int u = units_a;
        for (int s = 0; s < nslices; ++s) {
          const int width = min(256, D - s * 256);
          const int nbox = (width + 63) / 64;
          for (int uu = 0; uu < nunits; ++uu) {
            const int slot = u % nslot;
            mbar_wait(smem_u32(&ctrl->full[slot]), (u / nslot) & 1);
            const int key = uu * 32 + lane;
            if (wq < nbox && key < C && !ctrl->kvalid[key]) {
              const uint32_t ra = ring_addr + slot * kTcUnitBytes + wq * 4096 + lane * 128;
#pragma unroll
              for (int q = 0; q < 8; ++q) st_shared_v4(ra + q * 16, 0u, 0u, 0u, 0u);
            }
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&ctrl->fixed[slot]));
            ++u;
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
