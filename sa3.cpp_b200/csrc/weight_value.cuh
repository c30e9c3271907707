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

// The same values for the four elements (o, i .. i+3), i a multiple of 4, with one vector load of
// codes (and one scale: the four lie in one 32-element block): bit-identical to four wval calls.
__device__ __forceinline__ void wval4(const Weight& w, int64_t o, int64_t i, float (&v)[4]) {
  switch (w.type) {
    case kTypeQ8_0: {
      const char4 q = *reinterpret_cast<const char4*>(w.codes + o * w.in + i);
      const float d = w.scales[(i >> 5) * w.out + o];
      v[0] = (float)q.x * d; v[1] = (float)q.y * d; v[2] = (float)q.z * d; v[3] = (float)q.w * d;
      return;
    }
    case kTypeQ4_K: {
      const uint16_t b = *reinterpret_cast<const uint16_t*>(reinterpret_cast<const uint8_t*>(w.codes) +
                                                            o * (w.in / 2) + (i >> 1));
      const float2 s = reinterpret_cast<const float2*>(w.scales)[(i >> 5) * w.out + o];
      v[0] = s.x * (float)(b & 15) - s.y;
      v[1] = s.x * (float)((b >> 4) & 15) - s.y;
      v[2] = s.x * (float)((b >> 8) & 15) - s.y;
      v[3] = s.x * (float)(b >> 12) - s.y;
      return;
    }
    default:
      for (int c = 0; c < 4; ++c) v[c] = wval(w, o, i + c);
  }
}

}  // namespace sa3k
