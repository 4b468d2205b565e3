// Shared device helpers for the MoE-layer kernels (sm_100a).
//
// Floating-point contract: every arithmetic step that has to match the
// reference engine's CPU INT8 path bit for bit is written with the _rn
// intrinsics (__fmul_rn / __fadd_rn / __fmaf_rn / __fdiv_rn / __fsqrt_rn),
// which nvcc never contracts or reassociates, so the order below *is* the
// order executed.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace moe {

// Device status word bits (read back by moe_sync_status()).
enum : uint32_t {
  kStatusNonFinite = 1u << 0,  // non-finite input or output (reference `finite`)
  kStatusTimeout = 1u << 1,    // a bounded device-side wait gave up
  kStatusBadRoute = 1u << 2,   // routing produced an out-of-range expert id
};

constexpr int kMaxExperts = 256;
constexpr int kMaxTopK = 16;

__device__ __forceinline__ void set_status(uint32_t *status, uint32_t bit) {
  if (status) atomicOr(status, bit);
}

// ---------------------------------------------------------------------------
// Exact int8 -> f32 for four packed bytes: bias each byte to unsigned, place
// it in the mantissa of 2^23 (0x4B0000xx) with a byte permute, subtract
// 2^23 + 128.  Exact for every byte value.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void i8x4_to_f32(uint32_t w, float &a, float &b, float &c,
                                            float &d) {
  const uint32_t u = w ^ 0x80808080u;
  const float m = 8388736.0f;  // 2^23 + 128
  a = __fsub_rn(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7540)), m);
  b = __fsub_rn(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7541)), m);
  c = __fsub_rn(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7542)), m);
  d = __fsub_rn(__uint_as_float(__byte_perm(u, 0x4B000000u, 0x7543)), m);
}

// ---------------------------------------------------------------------------
// expf, bit-identical to the host libm expf that the reference's Rust
// `f32::exp` calls (glibc >= 2.28, FMA build).  Method: the table-driven
// single-precision exp published by Szabolcs Nagy (ARM optimized-routines):
// k = round(x * 32/ln2), r = x * 32/ln2 - k, exp(x) = 2^(k/32) * P(r) with a
// cubic P evaluated in double with FMAs.  The 2^(i/32) table is generated at
// build time from exact decimal arithmetic (gen_tables.py).  Equality with
// the host expf over every float input is checked by the test-suite.
// ---------------------------------------------------------------------------
#include "_gen/exp_table.inc"  // defines kPow2Tab[32] (double bit patterns)

__device__ __forceinline__ float expf_ref(float x) {
  if (x < -0x1.9fe368p6f) return 0.0f;
  if (x > 0x1.62e42ep6f) return __int_as_float(0x7f800000);
  const double inv_ln2_n = 0x1.71547652b82fep+0 * 32.0;
  const double shift = 0x1.8p+52;
  const double c0 = 0x1.c6af84b912394p-5 / (32.0 * 32.0 * 32.0);
  const double c1 = 0x1.ebfce50fac4f3p-3 / (32.0 * 32.0);
  const double c2 = 0x1.62e42ff0c52d6p-1 / 32.0;
  const double xd = (double)x;
  double kd = __fma_rn(inv_ln2_n, xd, shift);
  const unsigned long long ki = (unsigned long long)__double_as_longlong(kd);
  kd = __dsub_rn(kd, shift);
  const double r = __fma_rn(inv_ln2_n, xd, -kd);
  unsigned long long bits = kPow2Tab[ki & 31] + ((ki >> 5) << 52);
  const double sc = __longlong_as_double((long long)bits);
  const double z = __fma_rn(c0, r, c1);
  const double r2 = __dmul_rn(r, r);
  double y = __fma_rn(c2, r, 1.0);
  y = __fma_rn(z, r2, y);
  y = __dmul_rn(y, sc);
  return __double2float_rn(y);
}

// f32::total_cmp order key: larger key == later in total order.
__device__ __forceinline__ uint32_t total_order_u32(float f) {
  const int32_t i = __float_as_int(f);
  const int32_t k = i ^ (int32_t)(((uint32_t)(i >> 31)) >> 1);
  return (uint32_t)k ^ 0x80000000u;  // signed order -> unsigned order
}

__device__ __forceinline__ bool is_finite_f(float v) { return isfinite(v); }

// Bounded spin on a 32-bit flag in global memory until (*p >= target).
// Returns false (and records kStatusTimeout) after `limit` polls.
__device__ __forceinline__ bool spin_until_geq(const volatile uint32_t *p, uint32_t target,
                                               uint32_t *status, long long limit) {
  for (long long it = 0; it < limit; ++it) {
    if (*p >= target) return true;
    __nanosleep(64);
  }
  set_status(status, kStatusTimeout);
  return false;
}

}  // namespace moe
