// Element-type traits, the activation epilogue and the launch parameters that
// both kernel families share.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>

namespace avey {

// Plain-old-data copy of the C-ABI parameters, passed by value to kernels.
struct FwdArgs {
  const void* z_tr;
  const void* v;
  const void* z_tl;
  const void* bias;
  const uint8_t* valid;
  void* out;
  int64_t zr_bs, zr_rs;  // z_tr batch / row strides (elements)
  int64_t v_rs;
  int64_t zl_bs, zl_rs;
  int64_t va_bs, va_rs;  // valid batch / position strides (bytes)
  int64_t o_bs, o_rs;
  int batch, ctx, feat;
  float eps_f, norm_eps_f;
  double eps_d, norm_eps_d;
  int causal, normalize, act;
  int has_v, has_zl, has_bias, has_valid;  // has_valid: a byte mask or prefix lengths
  float* sumsq;  // workspace: per-row sums of squares of z_tr [batch][ctx] (tcgen05 path)
  const int32_t* lengths;  // [batch] prefix lengths (instead of valid), or null
};

// Position j of batch row b is valid (not padding): j < lengths[b] with the
// prefix-length form of the mask, valid[b][j] != 0 with the byte mask, always
// without either. Callers keep j < ctx.
__device__ __forceinline__ bool mask_ok(const FwdArgs& a, int b, int j) {
  if (a.lengths) return j < __ldg(a.lengths + b);
  return !a.valid ||
         a.valid[static_cast<int64_t>(b) * a.va_bs + static_cast<int64_t>(j) * a.va_rs] != 0;
}

template <typename T>
struct Elem;
template <>
struct Elem<float> {
  __device__ static float load(const float* p) { return __ldg(p); }
  __device__ static float to_f(float x) { return x; }
  __device__ static float from_f(float x) { return x; }
};
template <>
struct Elem<double> {
  __device__ static double load(const double* p) { return __ldg(p); }
};
template <>
struct Elem<__half> {
  __device__ static float load(const __half* p) { return __half2float(__ldg(p)); }
  __device__ static float to_f(__half x) { return __half2float(x); }
  __device__ static __half from_f(float x) { return __float2half_rn(x); }
};
template <>
struct Elem<__nv_bfloat16> {
  __device__ static float load(const __nv_bfloat16* p) { return __bfloat162float(__ldg(p)); }
  __device__ static float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
  __device__ static __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
};

template <typename T, typename A>
__device__ __forceinline__ T store_cast(A x) {
  if constexpr (sizeof(T) == sizeof(A)) {
    return static_cast<T>(x);
  } else if constexpr (sizeof(T) == 2) {
    return Elem<T>::from_f(static_cast<float>(x));
  } else {
    return static_cast<T>(x);
  }
}

// exp(-|x|) based logistic that neither overflows nor loses the small tail.
__device__ __forceinline__ float sigmoid_stable(float x) {
  const float e = expf(-fabsf(x));
  return x >= 0.f ? 1.f / (1.f + e) : e / (1.f + e);
}
__device__ __forceinline__ double sigmoid_stable(double x) {
  const double e = exp(-fabs(x));
  return x >= 0.0 ? 1.0 / (1.0 + e) : e / (1.0 + e);
}

// Activations of the reference (ops.py:49-58); ids as in _triton.py:169.
// relu keeps NaN (x < 0 is false for NaN), as torch.relu does.
template <typename A>
__device__ __forceinline__ A activate(A x, int act) {
  switch (act) {
    case 1:
      return x < A(0) ? A(0) : x;
    case 2: {
      const A r = x < A(0) ? A(0) : x;
      return r * r;
    }
    case 3:
      return x * sigmoid_stable(x);
    case 4: {
      // tanh-approximate gelu: 0.5 x (1 + tanh(t)) = x * sigmoid(2 t),
      // t = sqrt(2 / pi) * (x + 0.044715 x^3).
      const A t = A(0.7978845608028654) * (x + A(0.044715) * x * x * x);
      return x * sigmoid_stable(A(2) * t);
    }
    default:
      return x;
  }
}

// Activation with the id fixed at compile time (one case per kernel instance).
template <int ACT>
__device__ __forceinline__ float act_fn(float x) {
  if constexpr (ACT == 1) {
    return x < 0.f ? 0.f : x;
  } else if constexpr (ACT == 2) {
    const float r = x < 0.f ? 0.f : x;
    return r * r;
  } else if constexpr (ACT == 3) {
    return x * sigmoid_stable(x);
  } else if constexpr (ACT == 4) {
    const float t = 0.7978845608028654f * (x + 0.044715f * x * x * x);
    return x * sigmoid_stable(2.f * t);
  } else {
    return x;
  }
}

}  // namespace avey
