// Two-digit int8 activations: the arithmetic of the tolerance paths (the
// tcgen05 grouped GEMMs of expert_tc.cu, expert parallelism in ep.cu and the
// digit decode kernel of decode_digits.cu).
//
// An activation row v is written as two signed int8 digits with a per-row
// scale:
//     s = max|v| / 127 (1 for an all-zero row),  t = v / s,
//     d1 = rint(t),  d2 = rint((t - d1) * 254),   v ~= s * (d1 + d2 / 254),
// so the per-element error is at most max|v| / 64516.  An INT8 weight row w
// is then dotted with both digit planes in exact int32 arithmetic
// (D1 = sum w * d1, D2 = sum w * d2; |D| < 2^31 for rows up to 65536), and
// the epilogue forms s * D1 + (s / 254) * D2 in fp32.  Every kernel takes
// these functions, so equal int32 sums give bit-identical outputs on every
// path, whatever hardware produced the sums (tensor cores or dp4a).
#pragma once

#include <cstdint>

namespace moe {
namespace digits {

__device__ __forceinline__ float row_scale(float amax) {
  return amax > 0.0f ? amax / 127.0f : 1.0f;
}

// Digits of v given inv = 1 / row_scale(amax).
__device__ __forceinline__ void split(float v, float inv, int &d1, int &d2) {
  const float t = v * inv;
  const float a1 = fminf(fmaxf(rintf(t), -127.0f), 127.0f);
  const float a2 = fminf(fmaxf(rintf((t - a1) * 254.0f), -127.0f), 127.0f);
  d1 = (int)a1;
  d2 = (int)a2;
}

// Four values -> (low-plane word, high-plane word), byte k = element k.
__device__ __forceinline__ uint32_t split4(float v0, float v1, float v2, float v3, float inv,
                                           uint32_t &plane2) {
  const float in[4] = {v0, v1, v2, v3};
  uint32_t p1 = 0, p2 = 0;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    int d1, d2;
    split(in[k], inv, d1, d2);
    p1 |= (uint32_t)(uint8_t)(int8_t)d1 << (8 * k);
    p2 |= (uint32_t)(uint8_t)(int8_t)d2 << (8 * k);
  }
  plane2 = p2;
  return p1;
}

// s * D1 + (s / 254) * D2, with s2 = s / 254 precomputed.
__device__ __forceinline__ float dot(int32_t d1, int32_t d2, float s1, float s2) {
  return fmaf(s1, (float)d1, s2 * (float)d2);
}

// Gate/up epilogue: g = dot_g * s_g, u = dot_u * s_u, act = silu(g) * u (the
// hardware exp: this is the tolerance path).
__device__ __forceinline__ float swiglu(int32_t g1, int32_t g2, int32_t u1, int32_t u2, float s1,
                                        float s2, float sg, float su) {
  const float gg = dot(g1, g2, s1, s2) * sg, uu = dot(u1, u2, s1, s2) * su;
  return __fdividef(gg, 1.0f + __expf(-gg)) * uu;
}

// Down epilogue: y = dot_d * s_d.
__device__ __forceinline__ float down(int32_t d1, int32_t d2, float s1, float s2, float sd) {
  return dot(d1, d2, s1, s2) * sd;
}

}  // namespace digits
}  // namespace moe
