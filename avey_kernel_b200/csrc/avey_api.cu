// C ABI of libavey_b200.so (declared in include/avey_b200.h): argument
// validation, kernel selection, TMA descriptor encoding and launches.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "avey_b200.h"
#include "common.cuh"
#include "ptx.cuh"
#include "simt_kernel.cuh"
#include "tc_kernel.cuh"

namespace {

thread_local std::string g_last_error;
std::atomic<uint64_t> g_launches{0};

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int ok() {
  g_last_error.clear();
  return AVEY_OK;
}

enum Reason {
  kReasonNone = 0,
  kReasonDtype = 1,      // tcgen05 kernel needs bf16 or f16
  kReasonContext = 2,    // more than 512 tokens per row
  kReasonAlignment = 3,  // base / strides not 16-byte aligned (TMA, vector I/O)
  kReasonForced = 4,     // caller asked for the CUDA-core kernel
};

constexpr int kMaxDynSmem = 232448;  // 227 KB opt-in per block on sm_100

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int elem_size(int dtype) {
  switch (dtype) {
    case AVEY_F32: return 4;
    case AVEY_F16: return 2;
    case AVEY_BF16: return 2;
    case AVEY_F64: return 8;
    default: return 0;
  }
}

int validate(const AveyFwdParams* p) {
  if (!p) return fail(AVEY_ERR_ARGUMENT, "params is NULL");
  if (p->struct_size != sizeof(AveyFwdParams))
    return fail(AVEY_ERR_ARGUMENT, "struct_size %u != sizeof(AveyFwdParams) %zu", p->struct_size,
                sizeof(AveyFwdParams));
  if (elem_size(p->dtype) == 0) return fail(AVEY_ERR_ARGUMENT, "unknown dtype %d", p->dtype);
  if (p->batch < 1 || p->context < 1 || p->features < 1)
    return fail(AVEY_ERR_ARGUMENT, "batch, context and features must be >= 1");
  if (p->batch > 65535 || p->context > (1 << 24) || p->features > (1 << 24))
    return fail(AVEY_ERR_ARGUMENT, "shape [%lld, %lld, %lld] exceeds the supported range",
                (long long)p->batch, (long long)p->context, (long long)p->features);
  if (!p->z_tr || !p->out) return fail(AVEY_ERR_ARGUMENT, "z_tr and out are required");
  if (p->activation < 0 || p->activation > 4)
    return fail(AVEY_ERR_ARGUMENT, "unknown activation %d", p->activation);
  if (p->kernel < 0 || p->kernel > 2) return fail(AVEY_ERR_ARGUMENT, "unknown kernel %d", p->kernel);
  if (!std::isfinite(p->eps) || p->eps <= 0 || !std::isfinite(p->norm_eps) || p->norm_eps <= 0)
    return fail(AVEY_ERR_ARGUMENT, "eps and norm_eps must be finite and positive");
  if (p->z_tr_row_stride < p->features || p->out_row_stride < p->features ||
      (p->z_tl && p->z_tl_row_stride < p->features) || (p->v && p->v_row_stride < p->context))
    return fail(AVEY_ERR_ARGUMENT, "row strides must be at least the row length");
  if (p->z_tr_batch_stride < 0 || p->out_batch_stride < 0 || p->z_tl_batch_stride < 0 ||
      p->valid_batch_stride < 0 || p->valid_row_stride < 0)
    return fail(AVEY_ERR_ARGUMENT, "negative strides are not supported");
  return AVEY_OK;
}

int device_arch_ok(int* major_out) {
  int dev = 0, major = 0, minor = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail(AVEY_ERR_CUDA, "cudaGetDevice failed");
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  if (major_out) *major_out = major;
  if (major != 10 || minor != 0)
    return fail(AVEY_ERR_ARCH, "device %d is sm_%d%d; this library is built for sm_100a", dev, major,
                minor);
  return AVEY_OK;
}

int tc_reason(const AveyFwdParams* p) {
  if (p->kernel == AVEY_KERNEL_SIMT) return kReasonForced;
  if (p->dtype != AVEY_BF16 && p->dtype != AVEY_F16) return kReasonDtype;
  if (p->context > avey::kTcMaxKeys) return kReasonContext;
  const bool a = aligned16(p->z_tr) && aligned16(p->out) && (!p->z_tl || aligned16(p->z_tl)) &&
                 (p->z_tr_row_stride % 8 == 0) && (p->out_row_stride % 8 == 0) &&
                 (p->z_tr_batch_stride % 8 == 0 || p->batch == 1) &&
                 (p->out_batch_stride % 8 == 0 || p->batch == 1) && (p->features % 8 == 0) &&
                 (!p->z_tl || ((p->z_tl_row_stride % 8 == 0) &&
                               (p->z_tl_batch_stride % 8 == 0 || p->batch == 1)));
  if (!a) return kReasonAlignment;
  return kReasonNone;
}

struct TcLayout {
  avey::TcGeom geom;
  int smem;
};

TcLayout tc_layout(const AveyFwdParams* p) {
  TcLayout l{};
  const int ctx = static_cast<int>(p->context);
  const int nk_max = (ctx + 127) / 128;
  l.geom.p_bytes = nk_max * 2 * avey::kTcUnitBytes;
  const int room = kMaxDynSmem - 1024 - avey::kTcCtrlBytes - l.geom.p_bytes;
  int nslot = room / avey::kTcUnitBytes;
  if (nslot > avey::kTcMaxSlots) nslot = avey::kTcMaxSlots;
  l.geom.nslot = nslot;
  l.geom.n_qtiles = nk_max;
  l.smem = 1024 + l.geom.p_bytes + nslot * avey::kTcUnitBytes + avey::kTcCtrlBytes;
  return l;
}

avey::FwdArgs make_args(const AveyFwdParams* p) {
  avey::FwdArgs a{};
  a.z_tr = p->z_tr;
  a.v = p->v;
  a.z_tl = p->z_tl;
  a.bias = p->bias;
  a.valid = p->valid;
  a.out = p->out;
  a.zr_bs = p->z_tr_batch_stride;
  a.zr_rs = p->z_tr_row_stride;
  a.v_rs = p->v_row_stride;
  a.zl_bs = p->z_tl_batch_stride;
  a.zl_rs = p->z_tl_row_stride;
  a.va_bs = p->valid_batch_stride;
  a.va_rs = p->valid_row_stride;
  a.o_bs = p->out_batch_stride;
  a.o_rs = p->out_row_stride;
  a.batch = static_cast<int>(p->batch);
  a.ctx = static_cast<int>(p->context);
  a.feat = static_cast<int>(p->features);
  a.eps_f = static_cast<float>(p->eps);
  a.norm_eps_f = static_cast<float>(p->norm_eps);
  a.eps_d = p->eps;
  a.norm_eps_d = p->norm_eps;
  a.causal = p->causal != 0;
  a.normalize = p->normalize != 0;
  a.act = p->activation;
  a.has_v = p->v != nullptr;
  a.has_zl = p->z_tl != nullptr;
  a.has_bias = p->bias != nullptr;
  a.has_valid = p->valid != nullptr;
  return a;
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// 3-D map over z_tr viewed as [batch][context][features] with a box of
// `box_rows` rows x 64 features, 128-byte swizzle, zero fill out of bounds.
int encode_zmap(const AveyFwdParams* p, int box_rows, CUtensorMap* map) {
  auto fn = encode_fn();
  if (!fn) return fail(AVEY_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  const int es = elem_size(p->dtype);
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(p->features), static_cast<cuuint64_t>(p->context),
                        static_cast<cuuint64_t>(p->batch)};
  int64_t bs = p->z_tr_batch_stride;
  if (p->batch == 1) bs = p->z_tr_row_stride * p->context;  // unused; any aligned value
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(p->z_tr_row_stride * es),
                           static_cast<cuuint64_t>(((bs * es) + 15) / 16 * 16)};
  cuuint32_t box[3] = {64, static_cast<cuuint32_t>(box_rows), 1};
  cuuint32_t estr[3] = {1, 1, 1};
  const CUtensorMapDataType dt =
      p->dtype == AVEY_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  const CUresult r = fn(map, dt, 3, const_cast<void*>(p->z_tr), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(AVEY_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return AVEY_OK;
}

template <typename T>
int launch_tc(const AveyFwdParams* p, cudaStream_t stream) {
  static std::once_flag attr_once[64];
  int dev = 0;
  cudaGetDevice(&dev);
  cudaError_t attr_err = cudaSuccess;
  std::call_once(attr_once[dev & 63], [&] {
    attr_err = cudaFuncSetAttribute(avey::tc_contextualize<T>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxDynSmem);
  });
  if (attr_err != cudaSuccess)
    return fail(AVEY_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(attr_err));
  CUtensorMap map_k, map_z;
  int rc = encode_zmap(p, 128, &map_k);
  if (rc != AVEY_OK) return rc;
  rc = encode_zmap(p, 32, &map_z);
  if (rc != AVEY_OK) return rc;
  const TcLayout l = tc_layout(p);
  const avey::FwdArgs args = make_args(p);
  const unsigned grid = static_cast<unsigned>(p->batch * l.geom.n_qtiles);
  avey::tc_contextualize<T><<<grid, avey::kTcThreads, l.smem, stream>>>(args, map_k, map_z, l.geom);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(AVEY_ERR_LAUNCH, "tcgen05 kernel launch: %s", cudaGetErrorString(e));
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return ok();
}

template <typename T, typename A>
int launch_simt(const AveyFwdParams* p, cudaStream_t stream) {
  const avey::FwdArgs args = make_args(p);
  const dim3 grid(static_cast<unsigned>((p->context + avey::kSimtRows - 1) / avey::kSimtRows),
                  static_cast<unsigned>((p->features + avey::kSimtFeat - 1) / avey::kSimtFeat),
                  static_cast<unsigned>(p->batch));
  avey::simt_contextualize<T, A><<<grid, avey::kSimtFeat, 0, stream>>>(args);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(AVEY_ERR_LAUNCH, "CUDA-core kernel launch: %s", cudaGetErrorString(e));
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return ok();
}

}  // namespace

extern "C" {

int avey_fwd_plan(const AveyFwdParams* p, AveyPlan* plan) {
  int rc = validate(p);
  if (rc != AVEY_OK) return rc;
  if (!plan) return fail(AVEY_ERR_ARGUMENT, "plan is NULL");
  const int reason = tc_reason(p);
  if (p->kernel == AVEY_KERNEL_TCGEN05 && reason != kReasonNone)
    return fail(AVEY_ERR_UNSUPPORTED, "tcgen05 kernel cannot run these inputs (reason %d)", reason);
  std::memset(plan, 0, sizeof(*plan));
  plan->reason = reason;
  plan->launches = 1;
  if (reason == kReasonNone) {
    const TcLayout l = tc_layout(p);
    plan->kernel = AVEY_KERNEL_TCGEN05;
    plan->grid = static_cast<int32_t>(p->batch * l.geom.n_qtiles);
    plan->block = avey::kTcThreads;
    plan->smem_bytes = l.smem;
  } else {
    plan->kernel = AVEY_KERNEL_SIMT;
    plan->grid = static_cast<int32_t>(((p->context + 15) / 16) * ((p->features + 127) / 128) *
                                      p->batch);
    plan->block = avey::kSimtFeat;
    plan->smem_bytes = 0;
  }
  return ok();
}

int avey_fwd_v1(const AveyFwdParams* p, void* stream_ptr) {
  AveyPlan plan;
  int rc = avey_fwd_plan(p, &plan);
  if (rc != AVEY_OK) return rc;
  rc = device_arch_ok(nullptr);
  if (rc != AVEY_OK) return rc;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  if (plan.kernel == AVEY_KERNEL_TCGEN05) {
    return p->dtype == AVEY_BF16 ? launch_tc<__nv_bfloat16>(p, stream)
                                 : launch_tc<__half>(p, stream);
  }
  switch (p->dtype) {
    case AVEY_F32: return launch_simt<float, float>(p, stream);
    case AVEY_F16: return launch_simt<__half, float>(p, stream);
    case AVEY_BF16: return launch_simt<__nv_bfloat16, float>(p, stream);
    case AVEY_F64: return launch_simt<double, double>(p, stream);
    default: return fail(AVEY_ERR_ARGUMENT, "unknown dtype");
  }
}

const char* avey_last_error(void) { return g_last_error.c_str(); }

int avey_device_status(uint32_t* flags, int clear) {
  if (!flags) return fail(AVEY_ERR_ARGUMENT, "flags is NULL");
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return fail(AVEY_ERR_CUDA, "cudaDeviceSynchronize: %s", cudaGetErrorString(e));
  unsigned int v = 0;
  e = cudaMemcpyFromSymbol(&v, avey::g_devflags, sizeof(v));
  if (e != cudaSuccess) return fail(AVEY_ERR_CUDA, "reading the status word: %s", cudaGetErrorString(e));
  *flags = v;
  if (clear) {
    const unsigned int zero = 0;
    e = cudaMemcpyToSymbol(avey::g_devflags, &zero, sizeof(zero));
    if (e != cudaSuccess) return fail(AVEY_ERR_CUDA, "clearing the status word: %s", cudaGetErrorString(e));
  }
  return ok();
}

uint64_t avey_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int avey_abi_version(void) { return AVEY_ABI_VERSION; }

}  // extern "C"
