// weight_value.cuh -- the dequantized f32 value of one base-weight element, read from the device
// layout of quant.cu (Q8_0 / Q4_K code and scale planes, or the original F16 / F32 values).
#pragma once

#include "sa3k_internal.h"

namespace sa3k {

// Dequantized value of (o, i) from the device layout, f32, bit-identical to ggml's to_float.
__device__ __forceinline__ float wval(const Weight& w, int64_t o, int64_t i) {
  switch (w.type) {
    case kTypeQ8_0:
      return (float)w.codes[o * w.in + i] * w.scales[(i >> 5) * w.out + o];
    case kTypeQ4_K: {
      const uint8_t b = reinterpret_cast<const uint8_t*>(w.codes)[o * (w.in / 2) + (i >> 1)];
      const int q = (i & 1) ? (b >> 4) : (b & 15);
      const float2 s = reinterpret_cast<const float2*>(w.scales)[(i >> 5) * w.out + o];
      return s.x * (float)q - s.y;
    }
    case kTypeF16:
      return __half2float(reinterpret_cast<const __half*>(w.raw)[o * w.in + i]);
    default:
      return reinterpret_cast<const float*>(w.raw)[o * w.in + i];
  }
}

}  // namespace sa3k
