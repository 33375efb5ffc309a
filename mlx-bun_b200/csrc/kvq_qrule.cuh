#pragma once
// kvq_qrule.cuh — the affine group-quantize rule of MLX's quantize as this
// library applies it on the device (shared by the append kernel and the
// fused projection epilogue, so both produce the same codes):
//   s0 = (max - min) / (2^bits - 1), at least kQuantEps;
//   anchor = the extreme of larger magnitude, s0 signed towards it;
//   q0 = round(anchor / s0); scale = anchor / q0, bias = anchor (q0 != 0),
//   else scale = s0, bias = 0;
//   code = clamp(round((w - bias) / scale), 0, 2^bits - 1), with the
//   unrounded f32 scale; round half away from zero; IEEE division.
// The stored scale and bias are the f32 values rounded to the dtype.
#include <cuda_runtime.h>

namespace kvq {

constexpr float kQuantEps = 1e-7f;  // constant-group guard shared with the oracle

// scale and bias of a group whose elements span [mn, mx]; NB = 2^bits - 1
__device__ __forceinline__ void quant_params(float mn, float mx, float NB, float& scale,
                                             float& bias) {
  float s0 = (mx - mn) / NB;
  if (!(s0 >= kQuantEps)) s0 = kQuantEps;
  const bool neg = fabsf(mn) > fabsf(mx);
  const float anchor = neg ? mn : mx;
  s0 = neg ? s0 : -s0;
  const float q0 = roundf(anchor / s0);
  if (q0 != 0.0f) {
    scale = anchor / q0;
    bias = anchor;
  } else {
    scale = s0;
    bias = 0.0f;
  }
}

// the code of one element
__device__ __forceinline__ uint32_t quant_code(float w, float scale, float bias, float NB) {
  float c = roundf((w - bias) / scale);
  c = fminf(fmaxf(c, 0.0f), NB);
  return (uint32_t)c;
}

}  // namespace kvq
