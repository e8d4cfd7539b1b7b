// C ABI of the backward steps (declared in include/avey_b200.h): argument
// checks, type dispatch and launches of bwd_kernels.cuh.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <mutex>
#include <type_traits>

#include "avey_b200.h"
#include "bwd_kernels.cuh"

namespace avey_host {
int set_error(int code, const char* msg);
int clear_error();
void count_launches(int n);
}  // namespace avey_host

namespace {

int fail(int code, const char* msg) { return avey_host::set_error(code, msg); }

int expected_gemm_dtype(int dtype) {
  switch (dtype) {
    case AVEY_BF16: return AVEY_BF16;
    case AVEY_F16:
    case AVEY_F32: return AVEY_F32;
    case AVEY_F64: return AVEY_F64;
    default: return -1;
  }
}

int acc_size(const AveyBwdParams* p) { return p->dtype == AVEY_F64 ? 8 : 4; }

bool vec_ok(const AveyBwdParams* p);

// Epilogue blocks: 64 rows each in the scalar form, 32 in the vector form.
int64_t epi_blocks(const AveyBwdParams* p) {
  const int rows = vec_ok(p) ? avey::kBwdEpiRowsV8 : avey::kBwdEpiRows;
  return (p->batch * p->context + rows - 1) / rows;
}

// dscores grid: tile pairs x batch groups, enough CTAs to fill the GPU.
void dscores_grid(const AveyBwdParams* p, int* pairs, int* groups, int* per_group) {
  const int nt = static_cast<int>((p->context + avey::kBwdTile - 1) / avey::kBwdTile);
  *pairs = nt * (nt + 1) / 2;
  int g = std::max(1, std::min(static_cast<int>(p->batch), (1184 + *pairs - 1) / *pairs));
  g = std::min(g, 16);  // bounds the dV partial sums (16 x C x C)
  *per_group = static_cast<int>((p->batch + g - 1) / g);
  *groups = static_cast<int>((p->batch + *per_group - 1) / *per_group);
}

uint64_t workspace_bytes(const AveyBwdParams* p) {
  int pairs, groups, per;
  dscores_grid(p, &pairs, &groups, &per);
  const uint64_t epi = static_cast<uint64_t>(epi_blocks(p)) * p->features;
  const uint64_t ds = p->v ? static_cast<uint64_t>(groups) * p->context * p->context : 0;
  return std::max(epi, ds) * acc_size(p);
}

int validate(const AveyBwdParams* p) {
  if (!p) return fail(AVEY_ERR_ARGUMENT, "params is NULL");
  if (p->struct_size != sizeof(AveyBwdParams))
    return fail(AVEY_ERR_ARGUMENT, "struct_size does not match sizeof(AveyBwdParams)");
  if (expected_gemm_dtype(p->dtype) < 0) return fail(AVEY_ERR_ARGUMENT, "unknown dtype");
  if (p->gemm_dtype != expected_gemm_dtype(p->dtype))
    return fail(AVEY_ERR_ARGUMENT, "gemm_dtype must be bf16 for bf16 inputs, f32 for f16/f32, f64 for f64");
  if (p->batch < 1 || p->context < 1 || p->features < 1 || p->batch > 65535 ||
      p->context > (1 << 16) || p->features > (1 << 24))
    return fail(AVEY_ERR_ARGUMENT, "batch, context and features out of range");
  if (p->activation < 0 || p->activation > 4) return fail(AVEY_ERR_ARGUMENT, "unknown activation");
  if (!std::isfinite(p->eps) || p->eps <= 0 || !std::isfinite(p->norm_eps) || p->norm_eps <= 0)
    return fail(AVEY_ERR_ARGUMENT, "eps and norm_eps must be finite and positive");
  if (!p->z_tr || p->z_tr_row_stride < p->features || p->z_tr_batch_stride < 0 ||
      (p->z_tl && (p->z_tl_row_stride < p->features || p->z_tl_batch_stride < 0)) ||
      (p->v && p->v_row_stride < p->context) || p->valid_batch_stride < 0 ||
      p->valid_row_stride < 0 || p->grad_batch_stride < 0 ||
      (p->grad_row_stride && p->grad_row_stride < p->features))
    return fail(AVEY_ERR_ARGUMENT, "z_tr is required and strides must cover the rows");
  return AVEY_OK;
}

avey::BwdArgs make_args(const AveyBwdParams* p) {
  avey::BwdArgs a{};
  a.z_tr = p->z_tr;
  a.v = p->v;
  a.z_tl = p->z_tl;
  a.bias = p->bias;
  a.valid = p->valid;
  a.gout = p->grad_out;
  a.zr_bs = p->z_tr_batch_stride;
  a.zr_rs = p->z_tr_row_stride;
  a.v_rs = p->v_row_stride;
  a.zl_bs = p->z_tl_batch_stride;
  a.zl_rs = p->z_tl_row_stride;
  a.va_bs = p->valid_batch_stride;
  a.va_rs = p->valid_row_stride;
  a.go_bs = p->grad_out_batch_stride;
  a.go_rs = p->grad_out_row_stride;
  // grad_z_tr / grad_z_tl: contiguous unless strides are given.
  a.gr_rs = p->grad_row_stride ? p->grad_row_stride : p->features;
  a.gr_bs = p->grad_batch_stride ? p->grad_batch_stride : p->context * a.gr_rs;
  a.batch = static_cast<int>(p->batch);
  a.ctx = static_cast<int>(p->context);
  a.feat = static_cast<int>(p->features);
  a.eps = p->eps;
  a.norm_eps = p->norm_eps;
  a.causal = p->causal != 0;
  a.normalize = p->normalize != 0;
  a.act = p->activation;
  a.zm = p->zm;
  a.norms = p->norms;
  a.g = p->g;
  a.s = p->s;
  a.den = p->den;
  a.num = p->num;
  a.dnum = p->dnum;
  a.dden = p->dden;
  a.ds0 = p->ds0;
  a.dgsym = p->dgsym;
  a.dzd = p->dzd;
  a.dzh = p->dzh;
  a.part = p->workspace;
  a.gz_tr = p->grad_z_tr;
  a.gv = p->v ? p->grad_v : nullptr;
  a.gz_tl = p->z_tl ? p->grad_z_tl : nullptr;
  a.gbias = p->bias ? p->grad_bias : nullptr;
  return a;
}

int launched(int n) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    char buf[256];
    snprintf(buf, sizeof(buf), "backward launch: %s", cudaGetErrorString(e));
    return fail(AVEY_ERR_LAUNCH, buf);
  }
  avey_host::count_launches(n);
  return avey_host::clear_error();
}

bool al16(const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; }

// The vector forms need 8-element rows everywhere and 16-byte aligned rows
// in every strided input (fp64 keeps the scalar forms).
bool vec_ok(const AveyBwdParams* p) {
  if (p->dtype == AVEY_F64 || p->context % 8 || p->features % 8) return false;
  auto rows_ok = [](const void* q, int64_t bs, int64_t rs) {
    return !q || (al16(q) && bs % 8 == 0 && rs % 8 == 0);
  };
  return rows_ok(p->z_tr, p->z_tr_batch_stride, p->z_tr_row_stride) &&
         rows_ok(p->z_tl, p->z_tl_batch_stride, p->z_tl_row_stride) &&
         rows_ok(p->grad_out, p->grad_out_batch_stride, p->grad_out_row_stride) &&
         rows_ok(p->v, 0, p->v_row_stride) && (!p->bias || al16(p->bias)) &&
         rows_ok(p->grad_z_tr, p->grad_batch_stride, p->grad_row_stride) &&
         rows_ok(p->grad_z_tl, p->grad_batch_stride, p->grad_row_stride);
}

// One warp per partial sum, up to 32 warps.
unsigned reduce_threads(int64_t nparts) {
  return static_cast<unsigned>(32 * std::min<int64_t>(32, std::max<int64_t>(1, nparts)));
}

int row_grid(const AveyBwdParams* p) {
  const int64_t warps = p->batch * p->context;
  return static_cast<int>(std::min<int64_t>((warps + 7) / 8, 148 * 16));
}

// zm equals z_tr when nothing is padded and the GEMM type is the input type;
// the caller may then pass no zm and give z_tr (strided) to the GEMMs.
bool zm_optional(const AveyBwdParams* p) { return !p->valid && p->gemm_dtype == p->dtype; }

// Feature slots (256 features each) per epilogue pass: three when that takes
// fewer passes over the rows than two (d' = 768: one pass instead of two),
// else two (d' = 384 would leave most of a third slot idle).
int epi_slots(const AveyBwdParams* p) {
  const int64_t nv = p->features / 8;
  const int64_t p2 = (nv + 63) / 64, p3 = (nv + 95) / 96;
  return p3 < p2 ? 3 : 2;
}

template <typename T, typename G, int S>
void launch_epilogue_v8(int activation, unsigned grid, cudaStream_t st, const avey::BwdArgs& a) {
  constexpr int kT = avey::kBwdThreads;
  switch (activation) {
    case 1: avey::bwd_epilogue_v8<T, G, 1, S><<<grid, kT, 0, st>>>(a); break;
    case 2: avey::bwd_epilogue_v8<T, G, 2, S><<<grid, kT, 0, st>>>(a); break;
    case 3: avey::bwd_epilogue_v8<T, G, 3, S><<<grid, kT, 0, st>>>(a); break;
    case 4: avey::bwd_epilogue_v8<T, G, 4, S><<<grid, kT, 0, st>>>(a); break;
    default: avey::bwd_epilogue_v8<T, G, 0, S><<<grid, kT, 0, st>>>(a); break;
  }
}

template <typename T, typename G, typename A>
int run_step(const AveyBwdParams* p, int step, cudaStream_t st) {
  const avey::BwdArgs a = make_args(p);
  constexpr int kT = avey::kBwdThreads;
  constexpr bool kHasVec = !std::is_same<A, double>::value;
  const bool vec = kHasVec && vec_ok(p);
  switch (step) {
    case AVEY_BWD_PREP:
      if (!p->norms) return fail(AVEY_ERR_ARGUMENT, "prep needs norms");
      if (!p->zm && !zm_optional(p))
        return fail(AVEY_ERR_ARGUMENT, "zm may be NULL only without valid and with gemm_dtype == dtype");
      if constexpr (kHasVec) {
        if (vec) {
          avey::bwd_prep_v8<T, G><<<row_grid(p), kT, 0, st>>>(a);
          return launched(1);
        }
      }
      avey::bwd_prep<T, G, A><<<row_grid(p), kT, 0, st>>>(a);
      return launched(1);
    case AVEY_BWD_SCORES:
      if (!p->g || !p->s || !p->den || !p->norms)
        return fail(AVEY_ERR_ARGUMENT, "scores needs g, s, den, norms");
      if constexpr (kHasVec) {
        if (vec) {
          avey::bwd_scores_v8<T, G><<<row_grid(p), kT, 0, st>>>(a);
          return launched(1);
        }
      }
      avey::bwd_scores<T, G, A><<<row_grid(p), kT, 0, st>>>(a);
      return launched(1);
    case AVEY_BWD_EPILOGUE: {
      if (!p->num || !p->den || !p->dnum || !p->dden || !p->grad_out || !p->workspace ||
          p->workspace_bytes < workspace_bytes(p))
        return fail(AVEY_ERR_ARGUMENT, "epilogue needs num, den, dnum, dden, grad_out, workspace");
      const int64_t nb = epi_blocks(p);
      bool done = false;
      if constexpr (kHasVec) {
        if (vec) {
          if (epi_slots(p) == 3)
            launch_epilogue_v8<T, G, 3>(p->activation, static_cast<unsigned>(nb), st, a);
          else
            launch_epilogue_v8<T, G, 2>(p->activation, static_cast<unsigned>(nb), st, a);
          done = true;
        }
      }
      if (!done) avey::bwd_epilogue<T, G, A><<<static_cast<unsigned>(nb), kT, 0, st>>>(a);
      int n = 1;
      if (a.gbias) {
        avey::bwd_reduce<T, A><<<static_cast<unsigned>((p->features + 31) / 32), reduce_threads(nb), 0, st>>>(
            static_cast<const A*>(p->workspace), static_cast<int>(nb), p->features,
            static_cast<T*>(p->grad_bias));
        ++n;
      }
      return launched(n);
    }
    case AVEY_BWD_DSCORES: {
      if (!p->ds0 || !p->g || !p->dden || !p->dgsym || !p->norms || (a.gv && (!p->workspace ||
                                                             p->workspace_bytes < workspace_bytes(p))))
        return fail(AVEY_ERR_ARGUMENT, "dscores needs ds0, g, dden, dgsym (and workspace for grad_v)");
      int pairs, groups, per;
      dscores_grid(p, &pairs, &groups, &per);
      bool vdone = false;
      if constexpr (kHasVec) {
        if (vec) {
          // The cp.async operand ring: 2 tiles x kDsStages batch rows (48 KB).
          constexpr int kRing = 2 * avey::kDsStages * static_cast<int>(sizeof(avey::DsStage));
          int dev = 0;
          cudaGetDevice(&dev);
          static std::once_flag once[64];
          static cudaError_t attr_err[64];
          std::call_once(once[dev & 63], [&] {
            attr_err[dev & 63] = cudaFuncSetAttribute(
                avey::bwd_dscores_v4<T, G>, cudaFuncAttributeMaxDynamicSharedMemorySize, kRing);
          });
          if (attr_err[dev & 63] != cudaSuccess)
            return fail(AVEY_ERR_CUDA, "cudaFuncSetAttribute(bwd_dscores_v4) failed");
          avey::bwd_dscores_v4<T, G><<<dim3(pairs, groups), kT, kRing, st>>>(a, per);
          vdone = true;
        }
      }
      if (!vdone) avey::bwd_dscores<T, G, A><<<dim3(pairs, groups), kT, 0, st>>>(a, per);
      int n = 1;
      if (a.gv) {
        const int64_t cc = p->context * p->context;
        const A* part = static_cast<const A*>(p->workspace);
        if (groups <= 32) {
          constexpr int kRt = avey::kBwdReduceColThreads;
          const int64_t blocks = std::min<int64_t>((cc + kRt - 1) / kRt, 148 * 8);
          avey::bwd_reduce_cols<T, A><<<static_cast<unsigned>(blocks), kRt, 0, st>>>(
              part, groups, cc, static_cast<T*>(p->grad_v));
        } else {
          avey::bwd_reduce<T, A><<<static_cast<unsigned>((cc + 31) / 32), reduce_threads(groups), 0, st>>>(
              part, groups, cc, static_cast<T*>(p->grad_v));
        }
        ++n;
      }
      return launched(n);
    }
    case AVEY_BWD_FINAL:
      if (!p->norms || !p->dzh || !p->dzd || !p->grad_z_tr)
        return fail(AVEY_ERR_ARGUMENT, "final needs norms, dzh, dzd, grad_z_tr");
      if (!p->zm && !zm_optional(p))
        return fail(AVEY_ERR_ARGUMENT, "zm may be NULL only without valid and with gemm_dtype == dtype");
      if constexpr (kHasVec) {
        if (vec) {
          avey::bwd_final_v8<T, G><<<row_grid(p), kT, 0, st>>>(a);
          return launched(1);
        }
      }
      avey::bwd_final<T, G, A><<<row_grid(p), kT, 0, st>>>(a);
      return launched(1);
    default:
      return fail(AVEY_ERR_ARGUMENT, "unknown backward step");
  }
}

}  // namespace

extern "C" {

int avey_bwd_workspace_size(const AveyBwdParams* p, uint64_t* bytes) {
  int rc = validate(p);
  if (rc != AVEY_OK) return rc;
  if (!bytes) return fail(AVEY_ERR_ARGUMENT, "bytes is NULL");
  *bytes = workspace_bytes(p);
  return avey_host::clear_error();
}

int avey_bwd_step_v1(const AveyBwdParams* p, int step, void* stream) {
  int rc = validate(p);
  if (rc != AVEY_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  switch (p->dtype) {
    case AVEY_BF16: return run_step<__nv_bfloat16, __nv_bfloat16, float>(p, step, st);
    case AVEY_F16: return run_step<__half, float, float>(p, step, st);
    case AVEY_F32: return run_step<float, float, float>(p, step, st);
    case AVEY_F64: return run_step<double, double, double>(p, step, st);
    default: return fail(AVEY_ERR_ARGUMENT, "unknown dtype");
  }
}

}  // extern "C"
