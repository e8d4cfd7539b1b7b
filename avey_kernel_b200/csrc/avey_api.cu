// C ABI of libavey_b200.so (declared in include/avey_b200.h): argument
// validation, kernel selection, TMA descriptor encoding and launches.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
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
#include "norm_prepass.cuh"
#include "simt_kernel.cuh"
#include "simt2_kernel.cuh"
#include "small_kernel.cuh"
#include "tc_kernel.cuh"
#include "tc_long.cuh"
#include "tc_tf32.cuh"
#include "tc_gemm.cuh"

namespace {

thread_local std::string g_last_error;
std::atomic<uint64_t> g_launches{0};
// Test hook (avey_test_hooks_v1): the fused kernel's TMA and MMA warps issue nothing.
std::atomic<int> g_test_stall{0};

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
  kReasonDtype = 1,      // tcgen05 kernels take bf16, f16 and fp32 (3xTF32)
  kReasonContext = 2,    // more than 8192 tokens per row (or more than 512 without a workspace)
  kReasonAlignment = 3,  // base / strides not 16-byte aligned (TMA, vector I/O)
  kReasonForced = 4,     // caller asked for the CUDA-core kernel
  kReasonFeatures = 5,   // more than 2048 features (bias is staged in shared memory)
  kReasonSmall = 6,      // small fp32 problem: the 8-row CUDA-core kernel finishes first
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
  if (p->valid && p->lengths)
    return fail(AVEY_ERR_ARGUMENT, "pass the mask as valid or as lengths, not both");
  if (p->z_tr_batch_stride < 0 || p->out_batch_stride < 0 || p->z_tl_batch_stride < 0 ||
      p->valid_batch_stride < 0 || p->valid_row_stride < 0)
    return fail(AVEY_ERR_ARGUMENT, "negative strides are not supported");
  return AVEY_OK;
}

constexpr int kMaxDevices = 64;

// The current device, checked to be sm_100 once per device (the compute
// capability is queried on the first call only).
int device_arch_ok(int* dev_out) {
  static std::once_flag once[kMaxDevices];
  static int cc[kMaxDevices];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return fail(AVEY_ERR_CUDA, "cannot determine the current device");
  std::call_once(once[dev], [dev] {
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    cc[dev] = 10 * major + minor;
  });
  if (dev_out) *dev_out = dev;
  if (cc[dev] != 100)
    return fail(AVEY_ERR_ARCH, "device %d is sm_%d; this library is built for sm_100a", dev, cc[dev]);
  return AVEY_OK;
}

// Opt kernel K into `bytes` of dynamic shared memory, once per device. The
// outcome is kept per device and returned on every call, so a failure is
// reported as itself each time instead of as a later launch error.
template <auto K>
cudaError_t smem_opt_in(int bytes) {
  static std::once_flag once[kMaxDevices];
  static cudaError_t err[kMaxDevices];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::call_once(once[dev], [dev, bytes] {
    err[dev] = cudaFuncSetAttribute(K, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  });
  return err[dev];
}

// Contexts up to 512 run the fused kernel; longer ones (up to 8192) the
// two-kernel path of tc_long.cuh, whose P round trip needs a large workspace;
// `allow_long` is false for the no-allocation entry point.
bool small_pick(const AveyFwdParams* p);

int tc_reason(const AveyFwdParams* p, bool allow_long = true) {
  if (p->kernel == AVEY_KERNEL_SIMT) return kReasonForced;
  if (p->kernel == AVEY_KERNEL_AUTO && small_pick(p)) return kReasonSmall;
  if (p->dtype != AVEY_BF16 && p->dtype != AVEY_F16 && p->dtype != AVEY_F32) return kReasonDtype;
  if (p->context > (allow_long ? avey::kLongMaxContext : avey::kTcMaxKeys)) return kReasonContext;
  if (p->features > avey::kTcMaxFeatures) return kReasonFeatures;
  // Elements per 16 bytes: rows, batch strides and the feature count must be
  // whole 16-byte units (TMA strides, vector loads of the gate).
  const int64_t u = 16 / elem_size(p->dtype);
  const bool a = aligned16(p->z_tr) && aligned16(p->out) && (!p->z_tl || aligned16(p->z_tl)) &&
                 (p->z_tr_row_stride % u == 0) && (p->out_row_stride % u == 0) &&
                 (p->z_tr_batch_stride % u == 0 || p->batch == 1) &&
                 (p->out_batch_stride % u == 0 || p->batch == 1) && (p->features % u == 0) &&
                 (!p->z_tl || ((p->z_tl_row_stride % u == 0) &&
                               (p->z_tl_batch_stride % u == 0 || p->batch == 1)));
  if (!a) return kReasonAlignment;
  return kReasonNone;
}

struct TcLayout {
  avey::TcGeom geom;
  int smem;
};

// Shared memory: [phase-C ring | output staging | control block]. The phase-A
// stages (every key tile's chunk, 16 KB each; the query tile is one of the key
// tiles) use the ring's space before phase C; P itself lives in tensor memory.
TcLayout tc_layout(const AveyFwdParams* p) {
  TcLayout l{};
  const int ctx = static_cast<int>(p->context);
  const int nk_max = (ctx + 127) / 128;
  const int room = kMaxDynSmem - 1024 - avey::kTcCtrlBytes - avey::kTcOutStageBytes;
  int nslot = room / avey::kTcUnitBytes;
  if (nslot > avey::kTcMaxSlots) nslot = avey::kTcMaxSlots;
  l.geom.nslot = nslot;
  l.geom.n_qtiles = nk_max;
  // V tiles by TMA need a 16-byte aligned base and rows of multiples of 8 elements.
  l.geom.v_tma = p->v && aligned16(p->v) && (p->v_row_stride % 8 == 0);
  l.geom.test_stall = g_test_stall.load(std::memory_order_relaxed);
  l.smem = 1024 + nslot * avey::kTcUnitBytes + avey::kTcOutStageBytes + avey::kTcCtrlBytes;
  return l;
}

bool is_long(const AveyFwdParams* p) { return p->context > avey::kTcMaxKeys; }

// Inputs that run a kernel pair with a P workspace (G/P, then P.Z): 16-bit
// rows above 512 tokens, and every fp32 input (3xTF32 kernels).
bool is_pair(const AveyFwdParams* p) { return is_long(p) || p->dtype == AVEY_F32; }
bool is_tf32(const AveyFwdParams* p) { return p->dtype == AVEY_F32; }

// Long-context path: grid shapes, shared memory and the workspace layout
// [row sums of squares | partial row sums of P | P (bf16/f16, rows padded to
// 64 elements)], each part 256-byte aligned.
// P workspace of one batch slice of the long path. Slices of 32 MB (P read
// back from L2, DRAM traffic 367 -> 292 MB at config 4) measured slower (227
// against 193 us: eight smaller launches with their tails), so a slice holds
// up to 256 MB: config 4 runs as one slice, and only larger batches are cut
// into slices, which also bounds the workspace.
constexpr uint64_t kLongSliceBytes = 256ull << 20;

struct LongLayout {
  avey::LongGeom geom;
  int gp_items;
  int slice_rows;  // batch rows per G/P + P.Z launch pair
  int smem_gp, smem_pv;
  uint64_t off_den, off_p, total;
};

uint64_t align256(uint64_t x) { return (x + 255u) & ~uint64_t(255); }

LongLayout long_layout(const AveyFwdParams* p) {
  LongLayout l{};
  const int64_t B = p->batch, C = p->context, D = p->features;
  l.geom.n_qtiles = static_cast<int>((C + 127) / 128);
  l.geom.n_groups = static_cast<int>((C + avey::kLgGroupKeys - 1) / avey::kLgGroupKeys);
  int items = 0;
  for (int qt = 0; qt < l.geom.n_qtiles; ++qt) {
    const int64_t nkeys = p->causal ? std::min<int64_t>(C, qt * 128 + 128) : C;
    items += static_cast<int>((nkeys + avey::kLgGroupKeys - 1) / avey::kLgGroupKeys);
  }
  l.gp_items = items;
  l.geom.items = items;
  l.geom.n_fgroups = static_cast<int>((D + avey::kPvGroupCols - 1) / avey::kPvGroupCols);
  const int64_t cp = (C + 63) / 64 * 64;
  l.geom.p_rs = cp;
  l.geom.p_bs = C * cp;
  const uint64_t p_es = is_tf32(p) ? 4u : 2u;  // P is fp32 on the 3xTF32 path
  const uint64_t p_row_bytes = static_cast<uint64_t>(C * cp) * p_es;
  l.slice_rows = static_cast<int>(std::max<uint64_t>(
      1, std::min<uint64_t>(static_cast<uint64_t>(B), kLongSliceBytes / p_row_bytes)));
  l.off_den = align256(static_cast<uint64_t>(B * C) * sizeof(float));
  l.off_p = l.off_den + align256(static_cast<uint64_t>(B * l.geom.n_groups * C) * sizeof(float));
  l.total = l.off_p + static_cast<uint64_t>(l.slice_rows) * p_row_bytes;
  if (is_tf32(p)) {
    l.geom.n_fgroups = static_cast<int>((D + avey::kTfPvCols - 1) / avey::kTfPvCols);
    l.smem_gp = 1024 + avey::kTfStages * avey::kTfGramStage + avey::kTfCtrlBytes;
    l.smem_pv = 1024 + avey::kTfStages * avey::kTfPvStage + avey::kTfCtrlBytes;
  } else {
    l.smem_gp = 1024 + avey::kLgStages * avey::kLgStageBytes + avey::kLgCtrlBytes;
    l.smem_pv = 1024 + avey::kPvStages * avey::kPvStageBytes + avey::kPvCtrlBytes;
  }
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
  a.has_valid = p->valid != nullptr || p->lengths != nullptr;
  a.sumsq = static_cast<float*>(p->workspace);
  a.lengths = p->lengths;
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

// Encoded tensor maps, cached per process: a map is a pure function of its
// encode arguments (device, base address, shape, strides, box, element type),
// so callers that reuse buffers (training loops, graph warm-ups, benchmarks)
// skip the driver call. Small and mutex-guarded; the oldest entry is replaced.
struct MapKey {
  int dev, dtype, box_cols, box_rows;
  const void* base;
  uint64_t dims[3], strides[2];
  bool operator==(const MapKey& o) const { return std::memcmp(this, &o, sizeof(MapKey)) == 0; }
};
struct MapCache {
  static constexpr int kEntries = 64;
  std::mutex mu;
  MapKey keys[kEntries];
  CUtensorMap maps[kEntries];
  int used = 0, next = 0;
};
MapCache& map_cache() {
  static MapCache c;
  return c;
}

// Encode (or fetch) a 3-D tiled map: dims {inner, rows, batch}, strides in bytes.
int encode_cached(int dtype, const void* base, const cuuint64_t (&dims)[3], const cuuint64_t (&strides)[2],
                  int box_cols, int box_rows, CUtensorMap* map) {
  MapKey k;
  std::memset(&k, 0, sizeof(k));  // padding bytes take part in the comparison
  cudaGetDevice(&k.dev);
  k.dtype = dtype;
  k.box_cols = box_cols;
  k.box_rows = box_rows;
  k.base = base;
  for (int i = 0; i < 3; ++i) k.dims[i] = dims[i];
  for (int i = 0; i < 2; ++i) k.strides[i] = strides[i];
  MapCache& c = map_cache();
  {
    std::lock_guard<std::mutex> lock(c.mu);
    for (int i = 0; i < c.used; ++i)
      if (c.keys[i] == k) {
        *map = c.maps[i];
        return AVEY_OK;
      }
  }
  auto fn = encode_fn();
  if (!fn) return fail(AVEY_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  const int es = elem_size(dtype);
  cuuint32_t box[3] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows), 1};
  const CUtensorMapSwizzle swz =
      box_cols * es == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B;
  cuuint32_t estr[3] = {1, 1, 1};
  const CUtensorMapDataType dt = dtype == AVEY_BF16  ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                 : dtype == AVEY_F32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                                     : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  cuuint64_t d[3] = {dims[0], dims[1], dims[2]};
  cuuint64_t st[2] = {strides[0], strides[1]};
  const CUresult r = fn(map, dt, 3, const_cast<void*>(base), d, st, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(AVEY_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  std::lock_guard<std::mutex> lock(c.mu);
  const int slot = c.used < MapCache::kEntries ? c.used++ : (c.next++ % MapCache::kEntries);
  c.keys[slot] = k;
  c.maps[slot] = *map;
  return AVEY_OK;
}

// 3-D map over z_tr viewed as [batch][context][features] with a box of
// `box_rows` rows x `box_cols` features (64-byte swizzle for 32 columns,
// 128-byte swizzle for 64), zero fill out of bounds.
int encode_map(const AveyFwdParams* p, const void* base, int64_t batch_stride, int64_t row_stride,
               int box_cols, int box_rows, CUtensorMap* map) {
  const int es = elem_size(p->dtype);
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(p->features), static_cast<cuuint64_t>(p->context),
                              static_cast<cuuint64_t>(p->batch)};
  int64_t bs = batch_stride;
  if (p->batch == 1) bs = row_stride * p->context;  // unused; any aligned value
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(row_stride * es),
                                 static_cast<cuuint64_t>(((bs * es) + 15) / 16 * 16)};
  return encode_cached(p->dtype, base, dims, strides, box_cols, box_rows, map);
}

// 3-D map with explicit sizes: dims {inner, rows, batch}, strides in bytes.
int encode_map_dims(int dtype, const void* base, uint64_t inner, uint64_t rows, uint64_t batch,
                    uint64_t row_bytes, uint64_t batch_bytes, int box_cols, int box_rows,
                    CUtensorMap* map) {
  const cuuint64_t dims[3] = {inner, rows, batch};
  const cuuint64_t strides[2] = {row_bytes, batch > 1 ? batch_bytes : row_bytes * rows};
  return encode_cached(dtype, base, dims, strides, box_cols, box_rows, map);
}

// Row sums of squares of z_tr, written into the workspace before the main
// kernels: the pre-pass over z_tr, or (avey_fwd_presummed_v1) the sum of the
// caller's partial planes. Both let the next launch start at once
// (programmatic dependent launch).
struct PreSum {
  const float* planes = nullptr;
  int n = 0;
  // Without planes: the fused kernel sums the rows' squares itself, unless
  // prepass is set (norm_prepass writes them to the workspace first).
  bool prepass = false;
};

template <typename T>
int launch_row_sums(const AveyFwdParams* p, const avey::FwdArgs& args, const PreSum& ps,
                    cudaStream_t stream) {
  const int rows = static_cast<int>(p->batch * p->context);
  if (ps.planes) {
    const int blocks = std::min(148 * 4, (rows + avey::kPrepassThreads - 1) / avey::kPrepassThreads);
    avey::sumsq_planes<<<blocks, avey::kPrepassThreads, 0, stream>>>(ps.planes, ps.n, rows, args.sumsq);
  } else {
    const int pre_blocks = std::min(148 * 8, (rows + 7) / 8);
    avey::norm_prepass<T><<<pre_blocks, avey::kPrepassThreads, 0, stream>>>(args);
  }
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(AVEY_ERR_LAUNCH, "row-sum launch: %s", cudaGetErrorString(e));
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return AVEY_OK;
}

// The contextualizer's per-row scale for the GEMM epilogue (O = P Z of the
// long-context path; see GemmGeom::ctx_*).
struct CtxMix {
  const float* sumsq;
  const float* den;
  int groups, causal, normalize, rq_in_p;
  float eps, norm_eps;
};
int validate_gemm(const AveyGemmParams* p);
template <typename T, bool OUT16, int ACT>
int launch_gemm(const AveyGemmParams* p, cudaStream_t stream, const CtxMix* ctx);

template <typename T, int ACT>
int launch_long(const AveyFwdParams* p, cudaStream_t stream, const PreSum& ps) {
  cudaError_t attr_err = smem_opt_in<avey::tc_gram_p<T>>(kMaxDynSmem);
  if (attr_err == cudaSuccess) attr_err = smem_opt_in<avey::tc_pv<T, ACT>>(kMaxDynSmem);
  if (attr_err != cudaSuccess)
    return fail(AVEY_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(attr_err));
  LongLayout l = long_layout(p);
  if (!p->workspace || p->workspace_bytes < l.total ||
      (reinterpret_cast<uintptr_t>(p->workspace) & 255u))
    return fail(AVEY_ERR_ARGUMENT,
                "the long-context tcgen05 path needs a 256-byte aligned workspace of %llu bytes",
                (unsigned long long)l.total);
  uint8_t* ws = static_cast<uint8_t*>(p->workspace);
  float* den_base = reinterpret_cast<float*>(ws + l.off_den);
  void* pbuf = ws + l.off_p;
  const uint64_t C = static_cast<uint64_t>(p->context);
  const uint64_t prow = static_cast<uint64_t>(l.geom.p_rs) * 2u, pbat = static_cast<uint64_t>(l.geom.p_bs) * 2u;
  const avey::FwdArgs all = make_args(p);
  // 1. Row sums of squares of every row.
  int rc0 = launch_row_sums<T>(p, all, ps, stream);
  if (rc0 != AVEY_OK) return rc0;
  cudaError_t e = cudaSuccess;
  // 2./3. Per batch slice: G and P per (query tile, key group) into the P
  // workspace (written with an L2 evict-last hint), then O = P Z and the
  // epilogue; a slice's P is small enough to be read back from L2.
  const int es = elem_size(p->dtype);
  for (int64_t b0 = 0; b0 < p->batch; b0 += l.slice_rows) {
    AveyFwdParams q = *p;
    q.batch = std::min<int64_t>(l.slice_rows, p->batch - b0);
    q.z_tr = static_cast<const uint8_t*>(p->z_tr) + b0 * p->z_tr_batch_stride * es;
    if (p->z_tl) q.z_tl = static_cast<const uint8_t*>(p->z_tl) + b0 * p->z_tl_batch_stride * es;
    q.out = static_cast<uint8_t*>(p->out) + b0 * p->out_batch_stride * es;
    if (p->valid) q.valid = p->valid + b0 * p->valid_batch_stride;
    if (p->lengths) q.lengths = p->lengths + b0;
    const uint64_t nb = static_cast<uint64_t>(q.batch);
    CUtensorMap map_k, map_pst, map_p, map_z, map_o;
    int rc = encode_map(&q, q.z_tr, q.z_tr_batch_stride, q.z_tr_row_stride, avey::kTcChunk, 128, &map_k);
    if (rc == AVEY_OK) rc = encode_map_dims(q.dtype, pbuf, C, C, nb, prow, pbat, 32, 32, &map_pst);
    if (rc == AVEY_OK) rc = encode_map_dims(q.dtype, pbuf, C, C, nb, prow, pbat, 64, 128, &map_p);
    if (rc == AVEY_OK)
      rc = encode_map(&q, q.z_tr, q.z_tr_batch_stride, q.z_tr_row_stride, 64, avey::kPvChunkKeys, &map_z);
    if (rc == AVEY_OK) rc = encode_map(&q, q.out, q.out_batch_stride, q.out_row_stride, 32, 32, &map_o);
    if (rc != AVEY_OK) return rc;
    avey::FwdArgs args = make_args(&q);
    args.sumsq = all.sumsq + b0 * static_cast<int64_t>(C);
    avey::LongGeom geom = l.geom;
    geom.den_part = den_base + b0 * geom.n_groups * static_cast<int64_t>(C);
    // The first slice's G/P launch is a programmatic dependent of the pre-pass
    // (it waits for the sums only before forming P); later ones follow in
    // plain stream order.
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(l.gp_items), static_cast<unsigned>(q.batch));
    cfg.blockDim = dim3(avey::kLgThreads);
    cfg.dynamicSmemBytes = static_cast<size_t>(l.smem_gp);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = b0 == 0 ? 1 : 0;
    e = cudaLaunchKernelEx(&cfg, avey::tc_gram_p<T>, args, map_k, map_pst, geom);
    if (e != cudaSuccess) return fail(AVEY_ERR_LAUNCH, "tc_gram_p launch: %s", cudaGetErrorString(e));
    g_launches.fetch_add(1, std::memory_order_relaxed);
    if (!p->valid && !p->lengths) {
      // No padding mask: O = P Z runs on the persistent tcgen05 GEMM (the K
      // loop of each 128-row tile stops at its diagonal under the causal
      // mask, where P is zero beyond it), its epilogue scaling each row as
      // tc_pv does, then bias, activation and gate.
      AveyGemmParams gp;
      std::memset(&gp, 0, sizeof(gp));
      gp.struct_size = sizeof(gp);
      gp.dtype = q.dtype;
      gp.out_dtype = q.dtype;
      gp.mode = q.causal ? AVEY_GEMM_K_LOWER : AVEY_GEMM_DENSE;
      gp.batch = q.batch;
      gp.m = q.context;
      gp.n = q.features;
      gp.k = q.context;
      const bool many = q.batch > 1;
      gp.a = pbuf;
      gp.a_batch_stride = many ? geom.p_bs : 0;
      gp.a_ld = geom.p_rs;
      gp.a_major = AVEY_MAJOR_K;
      gp.b = q.z_tr;
      gp.b_batch_stride = many ? q.z_tr_batch_stride : 0;
      gp.b_ld = q.z_tr_row_stride;
      gp.b_major = AVEY_MAJOR_MN;
      gp.c = q.out;
      gp.c_batch_stride = many ? q.out_batch_stride : 0;
      gp.c_ld = q.out_row_stride;
      gp.bias = q.bias;
      gp.gate = q.z_tl;
      gp.gate_batch_stride = q.z_tl ? (many ? q.z_tl_batch_stride : 0) : 0;
      gp.gate_ld = q.z_tl ? q.z_tl_row_stride : 0;
      gp.activation = ACT;
      gp.kernel = AVEY_GEMM_KERNEL_SINGLE;
      rc = validate_gemm(&gp);
      if (rc != AVEY_OK) return rc;
      const CtxMix cm{args.sumsq, geom.den_part, geom.n_groups, q.causal != 0, q.normalize != 0,
                      avey::kRowScaleInP<T> ? 1 : 0, args.eps_f, args.norm_eps_f};
      rc = launch_gemm<T, true, ACT>(&gp, stream, &cm);
      if (rc != AVEY_OK) return rc;
    } else {
      avey::tc_pv<T, ACT><<<dim3(static_cast<unsigned>(geom.n_qtiles * geom.n_fgroups),
                                 static_cast<unsigned>(q.batch)),
                            avey::kPvThreads, static_cast<size_t>(l.smem_pv), stream>>>(
          args, map_p, map_z, map_o, geom);
      e = cudaGetLastError();
      if (e != cudaSuccess) return fail(AVEY_ERR_LAUNCH, "tc_pv launch: %s", cudaGetErrorString(e));
      g_launches.fetch_add(1, std::memory_order_relaxed);
    }
  }
  return ok();
}

// fp32 inputs: per batch slice, tf_gram_p (G in 3xTF32 with the row norms
// from its own split, P as fp32 into the workspace) then tf_pv (O = P Z in
// 3xTF32 and the epilogue). No pre-pass: the split sums the squares.
template <int ACT>
int launch_tf32(const AveyFwdParams* p, cudaStream_t stream) {
  cudaError_t attr_err = smem_opt_in<avey::tf_gram_p>(kMaxDynSmem);
  if (attr_err == cudaSuccess) attr_err = smem_opt_in<avey::tf_pv<ACT>>(kMaxDynSmem);
  if (attr_err != cudaSuccess)
    return fail(AVEY_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(attr_err));
  LongLayout l = long_layout(p);
  if (!p->workspace || p->workspace_bytes < l.total ||
      (reinterpret_cast<uintptr_t>(p->workspace) & 255u))
    return fail(AVEY_ERR_ARGUMENT,
                "the fp32 tcgen05 path needs a 256-byte aligned workspace of %llu bytes",
                (unsigned long long)l.total);
  uint8_t* ws = static_cast<uint8_t*>(p->workspace);
  float* den_base = reinterpret_cast<float*>(ws + l.off_den);
  void* pbuf = ws + l.off_p;
  const uint64_t C = static_cast<uint64_t>(p->context);
  const uint64_t prow = static_cast<uint64_t>(l.geom.p_rs) * 4u, pbat = static_cast<uint64_t>(l.geom.p_bs) * 4u;
  for (int64_t b0 = 0; b0 < p->batch; b0 += l.slice_rows) {
    AveyFwdParams q = *p;
    q.batch = std::min<int64_t>(l.slice_rows, p->batch - b0);
    q.z_tr = static_cast<const float*>(p->z_tr) + b0 * p->z_tr_batch_stride;
    if (p->z_tl) q.z_tl = static_cast<const float*>(p->z_tl) + b0 * p->z_tl_batch_stride;
    q.out = static_cast<float*>(p->out) + b0 * p->out_batch_stride;
    if (p->valid) q.valid = p->valid + b0 * p->valid_batch_stride;
    if (p->lengths) q.lengths = p->lengths + b0;
    const uint64_t nb = static_cast<uint64_t>(q.batch);
    CUtensorMap map_k, map_pst, map_p, map_z, map_o;
    int rc = encode_map(&q, q.z_tr, q.z_tr_batch_stride, q.z_tr_row_stride, avey::kTfChunk, 128, &map_k);
    if (rc == AVEY_OK) rc = encode_map_dims(AVEY_F32, pbuf, C, C, nb, prow, pbat, 32, 32, &map_pst);
    if (rc == AVEY_OK) rc = encode_map_dims(AVEY_F32, pbuf, C, C, nb, prow, pbat, avey::kTfPvKeys, 128, &map_p);
    if (rc == AVEY_OK)
      rc = encode_map(&q, q.z_tr, q.z_tr_batch_stride, q.z_tr_row_stride, 32, avey::kTfPvKeys, &map_z);
    if (rc == AVEY_OK) rc = encode_map(&q, q.out, q.out_batch_stride, q.out_row_stride, 32, 32, &map_o);
    if (rc != AVEY_OK) return rc;
    const avey::FwdArgs args = make_args(&q);
    avey::LongGeom geom = l.geom;
    geom.den_part = den_base + b0 * geom.n_groups * static_cast<int64_t>(C);
    avey::tf_gram_p<<<dim3(static_cast<unsigned>(l.gp_items), static_cast<unsigned>(q.batch)),
                      avey::kTfThreads, static_cast<size_t>(l.smem_gp), stream>>>(args, map_k, map_pst, geom);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(AVEY_ERR_LAUNCH, "tf_gram_p launch: %s", cudaGetErrorString(e));
    g_launches.fetch_add(1, std::memory_order_relaxed);
    avey::tf_pv<ACT><<<dim3(static_cast<unsigned>(geom.n_qtiles * geom.n_fgroups),
                            static_cast<unsigned>(q.batch)),
                       avey::kTfThreads, static_cast<size_t>(l.smem_pv), stream>>>(
        args, map_p, map_z, map_o, geom);
    e = cudaGetLastError();
    if (e != cudaSuccess) return fail(AVEY_ERR_LAUNCH, "tf_pv launch: %s", cudaGetErrorString(e));
    g_launches.fetch_add(1, std::memory_order_relaxed);
  }
  return ok();
}

int launch_tf32_act(const AveyFwdParams* p, cudaStream_t stream) {
  switch (p->activation) {
    case AVEY_ACT_RELU: return launch_tf32<AVEY_ACT_RELU>(p, stream);
    case AVEY_ACT_RELU2: return launch_tf32<AVEY_ACT_RELU2>(p, stream);
    case AVEY_ACT_SILU: return launch_tf32<AVEY_ACT_SILU>(p, stream);
    case AVEY_ACT_GELU: return launch_tf32<AVEY_ACT_GELU>(p, stream);
    default: return launch_tf32<AVEY_ACT_IDENTITY>(p, stream);
  }
}

template <typename T, int ACT>
int launch_tc(const AveyFwdParams* p, cudaStream_t stream, const PreSum& ps) {
  if (is_long(p)) return launch_long<T, ACT>(p, stream, ps);
  const cudaError_t attr_err = smem_opt_in<avey::tc_contextualize<T, ACT>>(kMaxDynSmem);
  if (attr_err != cudaSuccess)
    return fail(AVEY_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(attr_err));
  CUtensorMap map_q, map_z, map_o, map_v;
  std::memset(&map_v, 0, sizeof(map_v));
  int rc = encode_map(p, p->z_tr, p->z_tr_batch_stride, p->z_tr_row_stride, avey::kTcChunk, 128,
                      &map_q);
  if (rc != AVEY_OK) return rc;
  rc = encode_map(p, p->z_tr, p->z_tr_batch_stride, p->z_tr_row_stride, 64, avey::kTcUnitKeys,
                  &map_z);
  if (rc != AVEY_OK) return rc;
  rc = encode_map(p, p->out, p->out_batch_stride, p->out_row_stride, 32, 32, &map_o);
  if (rc != AVEY_OK) return rc;
  if (tc_layout(p).geom.v_tma) {
    // V [query, key] as a 2-D map (one "batch"): {64 keys, 128 query rows} boxes.
    rc = encode_map_dims(p->dtype, p->v, static_cast<uint64_t>(p->context),
                         static_cast<uint64_t>(p->context), 1,
                         static_cast<uint64_t>(p->v_row_stride) * elem_size(p->dtype), 0, 64, 128,
                         &map_v);
    if (rc != AVEY_OK) return rc;
  }
  const avey::FwdArgs args = make_args(p);
  TcLayout l = tc_layout(p);
  l.geom.self_sums = (ps.planes || ps.prepass) ? 0 : 1;
  const uint64_t need = static_cast<uint64_t>(p->batch) * p->context * sizeof(float);
  if (!l.geom.self_sums &&
      (!p->workspace || p->workspace_bytes < need || (reinterpret_cast<uintptr_t>(p->workspace) & 3u)))
    return fail(AVEY_ERR_ARGUMENT,
                "the row sums of squares need a 4-byte aligned workspace of %llu bytes",
                (unsigned long long)need);
  // 1. Row sums of squares into the workspace, from given planes or by the
  //    pre-pass (the first launch lets the second start at once); otherwise
  //    the fused kernel sums the rows itself.
  if (!l.geom.self_sums) {
    rc = launch_row_sums<T>(p, args, ps, stream);
    if (rc != AVEY_OK) return rc;
  }
  cudaError_t e = cudaSuccess;
  // 2. The fused kernel as a programmatic dependent of the previous launch:
  //    after the pre-pass it waits for the sums only before its P phase;
  //    otherwise it waits once its set-up is done, before reading any input.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(p->batch * l.geom.n_qtiles));
  cfg.blockDim = dim3(avey::kTcThreads);
  cfg.dynamicSmemBytes = static_cast<size_t>(l.smem);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, avey::tc_contextualize<T, ACT>, args, map_q, map_z, map_o, map_v, l.geom);
  if (e != cudaSuccess) return fail(AVEY_ERR_LAUNCH, "tcgen05 kernel launch: %s", cudaGetErrorString(e));
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return ok();
}

template <typename T>
int launch_tc_act(const AveyFwdParams* p, cudaStream_t stream, const PreSum& ps = PreSum{}) {
  switch (p->activation) {
    case AVEY_ACT_RELU: return launch_tc<T, AVEY_ACT_RELU>(p, stream, ps);
    case AVEY_ACT_RELU2: return launch_tc<T, AVEY_ACT_RELU2>(p, stream, ps);
    case AVEY_ACT_SILU: return launch_tc<T, AVEY_ACT_SILU>(p, stream, ps);
    case AVEY_ACT_GELU: return launch_tc<T, AVEY_ACT_GELU>(p, stream, ps);
    default: return launch_tc<T, AVEY_ACT_IDENTITY>(p, stream, ps);
  }
}

// The two-phase CUDA-core kernel takes every fp32 and 16-bit input the
// tensor-core kernels do not; fp64 keeps simt_contextualize.
bool use_simt2(const AveyFwdParams* p) { return p->dtype != AVEY_F64; }

// fp32 inputs the 8-row kernel (small_kernel.cuh) takes: contexts up to 512,
// feature counts that are multiples of 32 with rows of at most 1 KB, and z_tr
// rows it can copy in 16-byte pieces.
bool small_ok(const AveyFwdParams* p) {
  if (p->dtype != AVEY_F32) return false;
  if (p->context > avey::kSmMaxCtx || p->features % 32 != 0 ||
      p->features * 4 > avey::kSmMaxRowBytes)
    return false;
  return aligned16(p->z_tr) && p->z_tr_row_stride % 4 == 0 &&
         (p->z_tr_batch_stride % 4 == 0 || p->batch == 1);
}

// Where the 8-row kernel finishes before the 3xTF32 kernel pair: each query
// tile of 8 rows runs on a CTA pair, one CTA per SM, so a wave is 74 tiles
// on the 148 SMs of a B200 and costs about 9 us (11.5 us at 512 tokens);
// the pair takes about 20 / 25 / 37 / 51 us at 64 / 128 / 256 / 512 tokens
// (fp32, Avey causal, 128 features, few rows). Measured: 9.8 against 36.8 us
// at config 1 (64 tiles), 35.1 against 37.2 us at 8 x 256 tokens (256 tiles),
// 25.7 against 20.6 us at 24 x 64 tokens (192 tiles). So AUTO picks it
// (reason kReasonSmall) for up to 4 waves of tiles above 128 tokens and up to
// 2 waves at or below; a forced AVEY_KERNEL_SIMT keeps the two-phase kernel.
constexpr int64_t kSmallTilesPerWave = 74;

bool small_pick(const AveyFwdParams* p) {
  if (!small_ok(p)) return false;
  const int64_t tiles = p->batch * ((p->context + avey::kSmRows - 1) / avey::kSmRows);
  return tiles <= (p->context > 128 ? 4 : 2) * kSmallTilesPerWave;
}

int launch_small(const AveyFwdParams* p, cudaStream_t stream) {
  const avey::SmallGeom g = avey::small_geom(static_cast<int>(p->features));
  // The opt-in is made once per device, so it names the largest layout (the
  // 128-key blocks of 512-byte rows and the 64-key blocks of 1 KB rows; the
  // kernel's static shared memory comes on top).
  const int smem_max = std::max(avey::small_geom(128).smem, avey::small_geom(256).smem);
  const cudaError_t attr_err = smem_opt_in<avey::small_contextualize>(smem_max);
  if (attr_err != cudaSuccess)
    return fail(AVEY_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(attr_err));
  const avey::FwdArgs args = make_args(p);
  // A (2, 1, 1) cluster per query tile: the two CTAs split the tile's keys.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(2 * ((p->context + avey::kSmRows - 1) / avey::kSmRows)),
                     static_cast<unsigned>(p->batch));
  cfg.blockDim = dim3(avey::kSmThreads);
  cfg.dynamicSmemBytes = static_cast<size_t>(g.smem);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, avey::small_contextualize, args, g);
  if (e != cudaSuccess) return fail(AVEY_ERR_LAUNCH, "CUDA-core kernel launch: %s", cudaGetErrorString(e));
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return ok();
}

template <typename T, bool LONG>
int launch_simt2(const AveyFwdParams* p, cudaStream_t stream) {
  const cudaError_t attr_err = smem_opt_in<avey::simt2_contextualize<T, LONG>>(avey::kS2SmemBytes);
  if (attr_err != cudaSuccess)
    return fail(AVEY_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(attr_err));
  const avey::FwdArgs args = make_args(p);
  const dim3 grid(static_cast<unsigned>((p->context + avey::kS2Rows - 1) / avey::kS2Rows),
                  static_cast<unsigned>(p->batch));
  avey::simt2_contextualize<T, LONG><<<grid, avey::kS2Threads, avey::kS2SmemBytes, stream>>>(args);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(AVEY_ERR_LAUNCH, "CUDA-core kernel launch: %s", cudaGetErrorString(e));
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

// ---------------------------------------------------------------------------
// Batched tcgen05 matrix product (avey_gemm_v1).

int sm_count() {
  static std::once_flag once[kMaxDevices];
  static int count[kMaxDevices];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
  std::call_once(once[dev], [dev] {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n < 1) n = 148;
    count[dev] = n;
  });
  return count[dev];
}

// Output tiles of one batch entry (the kernel's gemm_cols_of summed over row tiles).
int64_t gemm_tiles_per_batch(const avey::GemmGeom& g) {
  int64_t n = 0;
  for (int mt = 0; mt < g.n_mt; ++mt)
    n += g.mode == avey::kGemmLowerOut
             ? std::min<int64_t>(g.n_nt, (static_cast<int64_t>(mt) * g.bm + g.bm - 1) / avey::kGmBN + 1)
             : g.n_nt;
  return n;
}

int validate_gemm(const AveyGemmParams* p) {
  if (!p) return fail(AVEY_ERR_ARGUMENT, "params is NULL");
  if (p->struct_size != sizeof(AveyGemmParams))
    return fail(AVEY_ERR_ARGUMENT, "struct_size %u != sizeof(AveyGemmParams) %zu", p->struct_size,
                sizeof(AveyGemmParams));
  if (p->dtype != AVEY_BF16 && p->dtype != AVEY_F16)
    return fail(AVEY_ERR_ARGUMENT, "avey_gemm_v1 takes bf16 or f16 operands (dtype %d)", p->dtype);
  if (p->out_dtype != AVEY_F32 && p->out_dtype != p->dtype)
    return fail(AVEY_ERR_ARGUMENT, "out_dtype must be AVEY_F32 or the operand dtype");
  if (p->mode < AVEY_GEMM_DENSE || p->mode > AVEY_GEMM_K_UPPER)
    return fail(AVEY_ERR_ARGUMENT, "unknown mode %d", p->mode);
  if (p->batch < 1 || p->m < 1 || p->n < 1 || p->k < 1 || p->batch > 65535 || p->m > (1 << 24) ||
      p->n > (1 << 24) || p->k > (1 << 24))
    return fail(AVEY_ERR_ARGUMENT, "batch, m, n, k must be in [1, 2^24] (batch <= 65535)");
  if (!p->a || !p->b || !p->c) return fail(AVEY_ERR_ARGUMENT, "a, b and c are required");
  if ((p->a_major != AVEY_MAJOR_K && p->a_major != AVEY_MAJOR_MN) ||
      (p->b_major != AVEY_MAJOR_K && p->b_major != AVEY_MAJOR_MN))
    return fail(AVEY_ERR_ARGUMENT, "a_major / b_major must be AVEY_MAJOR_K or AVEY_MAJOR_MN");
  const int64_t a_inner = p->a_major == AVEY_MAJOR_K ? p->k : p->m;
  const int64_t b_inner = p->b_major == AVEY_MAJOR_K ? p->k : p->n;
  if (p->a_ld < a_inner || p->b_ld < b_inner || p->c_ld < p->n)
    return fail(AVEY_ERR_ARGUMENT, "leading dimensions must be at least the contiguous extent");
  if (p->a_batch_stride < 0 || p->b_batch_stride < 0 || p->c_batch_stride < 0)
    return fail(AVEY_ERR_ARGUMENT, "negative batch strides are not supported");
  const int es = 2, oes = p->out_dtype == AVEY_F32 ? 4 : 2;
  auto whole16 = [](int64_t elems, int size) { return (elems * size) % 16 == 0; };
  if (!aligned16(p->a) || !aligned16(p->b) || !aligned16(p->c) || !whole16(p->a_ld, es) ||
      !whole16(p->b_ld, es) || !whole16(p->c_ld, oes) || !whole16(p->a_batch_stride, es) ||
      !whole16(p->b_batch_stride, es) || (p->batch > 1 && !whole16(p->c_batch_stride, oes)))
    return fail(AVEY_ERR_ARGUMENT,
                "avey_gemm_v1 needs 16-byte aligned bases and strides that are whole 16-byte units");
  if (p->out_dtype == AVEY_F32 && (p->bias || p->gate || p->sumsq || p->activation != AVEY_ACT_IDENTITY))
    return fail(AVEY_ERR_ARGUMENT, "bias, gate, activation and sumsq need a 16-bit output");
  if (p->activation < 0 || p->activation > 4)
    return fail(AVEY_ERR_ARGUMENT, "unknown activation %d", p->activation);
  if (p->gate && (p->gate_ld < p->n || p->gate_batch_stride < 0))
    return fail(AVEY_ERR_ARGUMENT, "gate strides must cover a [batch][m][n] array");
  if (p->sumsq && (p->sumsq_col0 < 0 || p->sumsq_col0 % 128 != 0 || p->sumsq_col0 >= p->n))
    return fail(AVEY_ERR_ARGUMENT, "sumsq_col0 must be a multiple of 128 below n");
  if (p->kernel < AVEY_GEMM_KERNEL_AUTO || p->kernel > AVEY_GEMM_KERNEL_PAIR)
    return fail(AVEY_ERR_ARGUMENT, "unknown GEMM kernel %d", p->kernel);
  return AVEY_OK;
}

template <typename T, bool OUT16, int ACT>
int launch_gemm(const AveyGemmParams* p, cudaStream_t stream, const CtxMix* ctx) {
  // AUTO: one CTA per tile. With the current epilogue the pair measured slower
  // on every shape tried (4096^3 bf16: 109.0 against 103.2 us; the enricher
  // shape 75.2 against 71.6 us; num = s zm 41.4 against 36.8 us), so pairs
  // run only when asked for.
  const bool pair = p->kernel == AVEY_GEMM_KERNEL_PAIR;
  constexpr auto K1 = avey::tc_gemm<T, OUT16, ACT>;
  constexpr auto K2 = avey::tc_gemm_pair<T, OUT16, ACT>;
  const cudaError_t attr_err = pair ? smem_opt_in<K2>(avey::kG2Smem) : smem_opt_in<K1>(avey::kGmSmem);
  if (attr_err != cudaSuccess)
    return fail(AVEY_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(attr_err));
  avey::GemmGeom g{};
  g.batch = static_cast<int>(p->batch);
  g.m = static_cast<int>(p->m);
  g.n = static_cast<int>(p->n);
  g.k = static_cast<int>(p->k);
  g.bm = pair ? 256 : avey::kGmBM;
  g.n_mt = static_cast<int>((p->m + g.bm - 1) / g.bm);
  g.n_nt = static_cast<int>((p->n + avey::kGmBN - 1) / avey::kGmBN);
  g.mode = p->mode;
  g.a_mn = p->a_major == AVEY_MAJOR_MN;
  g.b_mn = p->b_major == AVEY_MAJOR_MN;
  g.a_batched = p->a_batch_stride != 0 && p->batch > 1;
  g.b_batched = p->b_batch_stride != 0 && p->batch > 1;
  const int64_t per_batch = gemm_tiles_per_batch(g);
  const int64_t tiles = per_batch * p->batch;
  if (tiles > (1ll << 30)) return fail(AVEY_ERR_ARGUMENT, "too many output tiles");
  g.total_tiles = static_cast<int>(tiles);
  g.tiles_per_batch = static_cast<int>(per_batch);
  g.has_bias = p->bias != nullptr;
  g.has_gate = p->gate != nullptr;
  g.bias = p->bias;
  g.gate = p->gate;
  g.gate_bs = p->gate_batch_stride;
  g.gate_rs = p->gate_ld;
  g.sumsq = p->sumsq;
  g.sumsq_col0 = p->sumsq_col0;
  if (ctx) {
    g.ctx_sumsq = ctx->sumsq;
    g.ctx_den = ctx->den;
    g.ctx_groups = ctx->groups;
    g.ctx_causal = ctx->causal;
    g.ctx_normalize = ctx->normalize;
    g.ctx_rq_in_p = ctx->rq_in_p;
    g.ctx_eps = ctx->eps;
    g.ctx_norm_eps = ctx->norm_eps;
  }
  // Operand maps: {contiguous extent, other extent, batch}; boxes of 64
  // contiguous elements (128 bytes, 128-byte swizzle) by 128 rows (A, K-major),
  // 256 rows (B, K-major) or 64 k rows (MN-major operands).
  const uint64_t ab = g.a_batched ? static_cast<uint64_t>(p->batch) : 1u;
  const uint64_t bb = g.b_batched ? static_cast<uint64_t>(p->batch) : 1u;
  CUtensorMap map_a, map_b, map_c;
  int rc = g.a_mn
               ? encode_map_dims(p->dtype, p->a, p->m, p->k, ab, p->a_ld * 2, p->a_batch_stride * 2, 64, 64, &map_a)
               : encode_map_dims(p->dtype, p->a, p->k, p->m, ab, p->a_ld * 2, p->a_batch_stride * 2, 64,
                                 avey::kGmBM, &map_a);
  if (rc != AVEY_OK) return rc;
  // K-major B: each CTA of a pair loads 128 of the tile's 256 columns.
  rc = g.b_mn ? encode_map_dims(p->dtype, p->b, p->n, p->k, bb, p->b_ld * 2, p->b_batch_stride * 2, 64, 64, &map_b)
              : encode_map_dims(p->dtype, p->b, p->k, p->n, bb, p->b_ld * 2, p->b_batch_stride * 2, 64,
                                pair ? 128 : avey::kGmBN, &map_b);
  if (rc != AVEY_OK) return rc;
  // Output boxes: 32 x 32 16-bit values, or 32 rows x 16 fp32 values (two
  // per 32-column chunk, double-buffered); both 64-byte rows.
  const int oes = OUT16 ? 2 : 4;
  rc = encode_map_dims(p->out_dtype, p->c, p->n, p->m, p->batch, p->c_ld * oes, p->c_batch_stride * oes,
                       OUT16 ? 32 : 16, 32, &map_c);
  if (rc != AVEY_OK) return rc;
  cudaError_t e = cudaSuccess;
  if (!pair) {
    const int grid = static_cast<int>(std::min<int64_t>(tiles, sm_count()));
    K1<<<grid, avey::kGmThreads, avey::kGmSmem, stream>>>(map_a, map_b, map_c, g);
    e = cudaGetLastError();
  } else {
    // Persistent CTA pairs: (2, 1, 1) clusters, one pair per two SMs.
    const int pairs = static_cast<int>(std::min<int64_t>(tiles, sm_count() / 2));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs));
    cfg.blockDim = dim3(avey::kGmThreads);
    cfg.dynamicSmemBytes = static_cast<size_t>(avey::kG2Smem);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, K2, map_a, map_b, map_c, g);
  }
  if (e != cudaSuccess) return fail(AVEY_ERR_LAUNCH, "tc_gemm launch: %s", cudaGetErrorString(e));
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return ok();
}

template <typename T>
int launch_gemm_out(const AveyGemmParams* p, cudaStream_t stream) {
  if (p->out_dtype == AVEY_F32) return launch_gemm<T, false, AVEY_ACT_IDENTITY>(p, stream, nullptr);
  switch (p->activation) {
    case AVEY_ACT_RELU: return launch_gemm<T, true, AVEY_ACT_RELU>(p, stream, nullptr);
    case AVEY_ACT_RELU2: return launch_gemm<T, true, AVEY_ACT_RELU2>(p, stream, nullptr);
    case AVEY_ACT_SILU: return launch_gemm<T, true, AVEY_ACT_SILU>(p, stream, nullptr);
    case AVEY_ACT_GELU: return launch_gemm<T, true, AVEY_ACT_GELU>(p, stream, nullptr);
    default: return launch_gemm<T, true, AVEY_ACT_IDENTITY>(p, stream, nullptr);
  }
}

}  // namespace

// Shared with the backward translation unit (avey_bwd.cu): one last-error
// string per thread and one launch counter for the whole library.
namespace avey_host {
int set_error(int code, const char* msg) { return fail(code, "%s", msg); }
int clear_error() { return ok(); }
void count_launches(int n) { g_launches.fetch_add(static_cast<uint64_t>(n), std::memory_order_relaxed); }
}  // namespace avey_host

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
  if (reason == kReasonNone && is_pair(p)) {
    const LongLayout l = long_layout(p);
    plan->kernel = AVEY_KERNEL_TCGEN05;
    // (16-bit: the pre-pass, then) a G/P + P.Z launch pair per batch slice.
    plan->launches = (is_tf32(p) ? 0 : 1) +
                     2 * static_cast<int32_t>((p->batch + l.slice_rows - 1) / l.slice_rows);
    plan->grid = static_cast<int32_t>(std::min<int64_t>(p->batch, l.slice_rows) * l.gp_items);
    plan->block = is_tf32(p) ? avey::kTfThreads : avey::kLgThreads;
    plan->smem_bytes = std::max(l.smem_gp, l.smem_pv);
  } else if (reason == kReasonNone) {
    const TcLayout l = tc_layout(p);
    plan->kernel = AVEY_KERNEL_TCGEN05;
    plan->launches = 1;  // the fused kernel sums the rows' squares itself
    plan->grid = static_cast<int32_t>(p->batch * l.geom.n_qtiles);
    plan->block = avey::kTcThreads;
    plan->smem_bytes = l.smem;
  } else if (reason == kReasonSmall) {
    plan->kernel = AVEY_KERNEL_SIMT;
    plan->grid = static_cast<int32_t>(2 * ((p->context + avey::kSmRows - 1) / avey::kSmRows) * p->batch);
    plan->block = avey::kSmThreads;
    plan->smem_bytes = avey::small_geom(static_cast<int>(p->features)).smem;
  } else if (use_simt2(p)) {
    plan->kernel = AVEY_KERNEL_SIMT;
    plan->grid = static_cast<int32_t>(((p->context + avey::kS2Rows - 1) / avey::kS2Rows) * p->batch);
    plan->block = avey::kS2Threads;
    plan->smem_bytes = avey::kS2SmemBytes;
  } else {
    plan->kernel = AVEY_KERNEL_SIMT;
    plan->grid = static_cast<int32_t>(((p->context + 15) / 16) * ((p->features + 127) / 128) *
                                      p->batch);
    plan->block = avey::kSimtFeat;
    plan->smem_bytes = 0;
  }
  return ok();
}

int avey_fwd_workspace_size(const AveyFwdParams* p, uint64_t* bytes) {
  AveyPlan plan;
  const int rc = avey_fwd_plan(p, &plan);
  if (rc != AVEY_OK) return rc;
  if (!bytes) return fail(AVEY_ERR_ARGUMENT, "bytes is NULL");
  // The fused kernel (up to 512 tokens, 16-bit) sums the rows' squares itself.
  *bytes = (plan.kernel == AVEY_KERNEL_TCGEN05 && is_pair(p)) ? long_layout(p).total : 0u;
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
    if (is_tf32(p)) return launch_tf32_act(p, stream);
    return p->dtype == AVEY_BF16 ? launch_tc_act<__nv_bfloat16>(p, stream)
                                 : launch_tc_act<__half>(p, stream);
  }
  if (plan.reason == kReasonSmall) return launch_small(p, stream);
  if (use_simt2(p)) {
    const bool lng = p->context > avey::kS2MaxCtx;
    switch (p->dtype) {
      case AVEY_F32: return lng ? launch_simt2<float, true>(p, stream) : launch_simt2<float, false>(p, stream);
      case AVEY_F16: return lng ? launch_simt2<__half, true>(p, stream) : launch_simt2<__half, false>(p, stream);
      default:
        return lng ? launch_simt2<__nv_bfloat16, true>(p, stream)
                   : launch_simt2<__nv_bfloat16, false>(p, stream);
    }
  }
  switch (p->dtype) {
    case AVEY_F32: return launch_simt<float, float>(p, stream);
    case AVEY_F16: return launch_simt<__half, float>(p, stream);
    case AVEY_BF16: return launch_simt<__nv_bfloat16, float>(p, stream);
    case AVEY_F64: return launch_simt<double, double>(p, stream);
    default: return fail(AVEY_ERR_ARGUMENT, "unknown dtype");
  }
}

// ---------------------------------------------------------------------------
// No-allocation entry point: scratch in a file-scope device array.
}  // extern "C"

namespace {

// One float (row sum of squares) per row of z_tr. Host code must not use the
// name as a device address; its address comes from cudaGetSymbolAddress.
__device__ __align__(256) float g_noalloc_sumsq[AVEY_NOALLOC_MAX_ROWS];

std::once_flag g_noalloc_once[kMaxDevices];
void* g_noalloc_ptr[kMaxDevices];
cudaError_t g_noalloc_err[kMaxDevices];

}  // namespace

extern "C" {

int avey_fwd_noalloc_v1(const AveyFwdParams* p, void* stream) {
  AveyPlan plan;
  int rc = avey_fwd_plan(p, &plan);
  if (rc != AVEY_OK) return rc;
  AveyFwdParams q = *p;
  // Contexts above 512 and fp32 inputs would take a tensor-core kernel pair
  // whose P workspace this entry point does not have: they run a CUDA-core
  // kernel (small fp32 problems the 8-row kernel, as avey_fwd_v1 does).
  if (is_pair(p) && plan.reason != kReasonSmall) {
    if (p->kernel == AVEY_KERNEL_TCGEN05)
      return fail(AVEY_ERR_UNSUPPORTED,
                  "the no-allocation entry point runs contexts above 512 and fp32 inputs on CUDA "
                  "cores only");
    q.kernel = AVEY_KERNEL_SIMT;
  }
  // Only the fused tensor-core path reads scratch (one float per row); the
  // CUDA-core kernels need none and have no row limit here.
  if (plan.kernel != AVEY_KERNEL_TCGEN05 || is_pair(p)) return avey_fwd_v1(&q, stream);
  const uint64_t rows = static_cast<uint64_t>(p->batch) * static_cast<uint64_t>(p->context);
  if (rows > AVEY_NOALLOC_MAX_ROWS)
    return fail(AVEY_ERR_ARGUMENT,
                "batch x context = %llu rows exceeds the no-allocation limit of %u rows",
                (unsigned long long)rows, AVEY_NOALLOC_MAX_ROWS);
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return fail(AVEY_ERR_CUDA, "cannot determine the current device");
  // Once per device, with that device current: the array's device address.
  std::call_once(g_noalloc_once[dev], [dev] {
    void* ptr = nullptr;
    g_noalloc_err[dev] = cudaGetSymbolAddress(&ptr, g_noalloc_sumsq);
    g_noalloc_ptr[dev] = g_noalloc_err[dev] == cudaSuccess ? ptr : nullptr;
  });
  if (g_noalloc_err[dev] != cudaSuccess || !g_noalloc_ptr[dev])
    return fail(AVEY_ERR_CUDA, "cudaGetSymbolAddress(no-allocation scratch): %s",
                cudaGetErrorString(g_noalloc_err[dev]));
  q.workspace = g_noalloc_ptr[dev];
  q.workspace_bytes = static_cast<uint64_t>(AVEY_NOALLOC_MAX_ROWS) * sizeof(float);
  // The pre-pass variant of the fused kernel: row sums of squares in the
  // array, read back by the kernel.
  rc = device_arch_ok(nullptr);
  if (rc != AVEY_OK) return rc;
  PreSum pre;
  pre.prepass = true;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return q.dtype == AVEY_BF16 ? launch_tc_act<__nv_bfloat16>(&q, s, pre)
                              : launch_tc_act<__half>(&q, s, pre);
}

int avey_gemm_v1(const AveyGemmParams* p, void* stream) {
  int rc = validate_gemm(p);
  if (rc != AVEY_OK) return rc;
  rc = device_arch_ok(nullptr);
  if (rc != AVEY_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return p->dtype == AVEY_BF16 ? launch_gemm_out<__nv_bfloat16>(p, s) : launch_gemm_out<__half>(p, s);
}

int avey_fwd_presummed_v1(const AveyFwdParams* p, const float* sumsq, int planes, void* stream_ptr) {
  AveyPlan plan;
  int rc = avey_fwd_plan(p, &plan);
  if (rc != AVEY_OK) return rc;
  if (!sumsq || planes < 1 || planes > 64)
    return fail(AVEY_ERR_ARGUMENT, "sumsq must hold 1 to 64 planes of row sums of squares");
  // Paths without the row-sum pre-pass (CUDA cores, 3xTF32) ignore the sums.
  if (plan.kernel != AVEY_KERNEL_TCGEN05 || is_tf32(p)) return avey_fwd_v1(p, stream_ptr);
  rc = device_arch_ok(nullptr);
  if (rc != AVEY_OK) return rc;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  const PreSum ps{sumsq, planes};
  return p->dtype == AVEY_BF16 ? launch_tc_act<__nv_bfloat16>(p, stream, ps)
                               : launch_tc_act<__half>(p, stream, ps);
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

int avey_test_hooks_v1(long long wait_limit_cycles, int stall) {
  if (wait_limit_cycles <= 0) wait_limit_cycles = avey::kWaitLimitCycles;
  const cudaError_t e = cudaMemcpyToSymbol(avey::g_wait_limit, &wait_limit_cycles, sizeof(long long));
  if (e != cudaSuccess) return fail(AVEY_ERR_CUDA, "setting the wait limit: %s", cudaGetErrorString(e));
  g_test_stall.store(stall ? 1 : 0, std::memory_order_relaxed);
  return ok();
}

int avey_abi_version(void) { return AVEY_ABI_VERSION; }


}  // extern "C"
