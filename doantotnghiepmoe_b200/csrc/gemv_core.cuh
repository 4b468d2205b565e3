// Device building blocks of the exact-order INT8 GEMV (shared by the
// per-phase kernels in expert_gemv.cu and the fused decode kernel).
//
// Arithmetic is the reference's AVX2 path, operation for operation
// (src/int8_expert.rs:380-458 `dot_i8_f32_avx2`, :653-781
// `dot_i8_f32_pair_avx2`, :1058-1127 the `_seq` row loops):
//   * a row dot of length n keeps 32 accumulators = 4 banks x 8 lanes; lane l
//     of bank b is an FMA chain over elements 32c + 8b + l, c = 0 .. n/32-1;
//   * banks fold as (b0 + b1) + (b2 + b3); leftover 8-chunks FMA into that;
//   * 8 -> 4 -> 2 -> 1 fold ((t0+t4)+(t2+t6)) + ((t1+t5)+(t3+t7)); scalar tail
//     with separate multiply and add;
//   * g = dot_g * s_g, u = dot_u * s_u, act = (g / (1 + exp(-g))) * u;
//     y = dot_d(act) * s_d.
// One thread holds one bank (its 8 lanes) of one row for up to kTG tokens,
// so the four banks of a row sit in four adjacent lanes and fold with warp
// shuffles.  Results are bit-identical to the CPU path.
//
// Weight formats (template kQ): 8 = one int8 per element; 4 = INT4, two
// signed nibbles per byte, element 2i in the low nibble
// (src/int8_expert.rs:473-649, :785-952).  INT4 rows are n/2 bytes and the
// per-element arithmetic is the same, so the 8 weights of a (chunk, bank)
// are 8 bytes or one 32-bit word.
#pragma once

#include "common.cuh"

namespace moe {
namespace gemv {

constexpr int kPF = 8;              // chunk-steps per register batch (two batches in flight)
constexpr int kTG = 4;              // tokens per pass
constexpr int kGURowsPerWarp = 4;   // gate/up: 8 lanes per row (4 gate + 4 up banks)
constexpr int kDNRowsPerWarp = 8;   // down: 4 lanes per row

// Streaming 8-byte weight load: read once, never reused by this CTA, and
// marked evict-first in L2 so the stream does not push the kernel's code,
// the routers or the activations out of L2.
__device__ __forceinline__ uint2 ldg_stream8(const int8_t *p) {
  uint64_t pol;
  asm("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  uint2 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v2.u32 {%0, %1}, [%2], %3;"
               : "=r"(v.x), "=r"(v.y)
               : "l"(p), "l"(pol));
  return v;
}

__device__ __forceinline__ uint32_t ldg_stream4(const int8_t *p) {
  uint64_t pol;
  asm("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  uint32_t v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.u32 %0, [%1], %2;"
               : "=r"(v)
               : "l"(p), "l"(pol));
  return v;
}

template <bool kVec>
__device__ __forceinline__ uint2 load_w8_raw(const int8_t *p) {
  if (kVec) return ldg_stream8(p);
  uint2 v;
  v.x = (uint32_t)(uint8_t)p[0] | ((uint32_t)(uint8_t)p[1] << 8) |
        ((uint32_t)(uint8_t)p[2] << 16) | ((uint32_t)(uint8_t)p[3] << 24);
  v.y = (uint32_t)(uint8_t)p[4] | ((uint32_t)(uint8_t)p[5] << 8) |
        ((uint32_t)(uint8_t)p[6] << 16) | ((uint32_t)(uint8_t)p[7] << 24);
  return v;
}

// Raw bytes of one (chunk, bank): 8 elements.
template <int kQ>
struct WRaw {
  using T = uint2;
};
template <>
struct WRaw<4> {
  using T = uint32_t;
};

template <int kQ, bool kVec>
__device__ __forceinline__ typename WRaw<kQ>::T load_wq(const int8_t *p) {
  if constexpr (kQ == 8) {
    return load_w8_raw<kVec>(p);
  } else {
    if (kVec) return ldg_stream4(p);
    return (uint32_t)(uint8_t)p[0] | ((uint32_t)(uint8_t)p[1] << 8) |
           ((uint32_t)(uint8_t)p[2] << 16) | ((uint32_t)(uint8_t)p[3] << 24);
  }
}

// The 8 weights of a (chunk, bank) as floats, in element order (exact).
__device__ __forceinline__ void decode8(const uint2 r, float w[8]) {
  i8x4_to_f32(r.x, w[0], w[1], w[2], w[3]);
  i8x4_to_f32(r.y, w[4], w[5], w[6], w[7]);
}
// Nibble k of the word is element k: u = bits [4k, 4k + 4), value
// (u ^ 8) - 8, formed exactly in the mantissa of 2^23.
__device__ __forceinline__ void decode8(const uint32_t r, float w[8]) {
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const uint32_t u = (r >> (4 * k)) & 0xFu;
    w[k] = __fsub_rn(__uint_as_float(0x4B000000u | (u ^ 8u)), 8388616.0f);
  }
}

// Element i of a row as a float (leftover chunks and the tail).
template <int kQ>
__device__ __forceinline__ float w_at(const int8_t *__restrict__ wrow, int i) {
  if constexpr (kQ == 8) {
    return (float)wrow[i];
  } else {
    const int8_t b = wrow[i >> 1];
    return (float)((i & 1) ? (b >> 4) : ((int8_t)(b << 4) >> 4));
  }
}

template <bool kVec>
__device__ __forceinline__ void load_x8(const float *p, float x[8]) {
  if (kVec) {
    const float4 a = *reinterpret_cast<const float4 *>(p);
    const float4 b = *reinterpret_cast<const float4 *>(p + 4);
    x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
    x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
  } else {
#pragma unroll
    for (int l = 0; l < 8; ++l) x[l] = p[l];
  }
}

// Bank `bank` of a row dot for ng (<= kTG) tokens whose inputs sit in smem
// rows xs + t*ld.  Weights are fetched kPF chunk-steps ahead into registers so
// that enough bytes are in flight to cover HBM latency; the FMA chains still
// run strictly in chunk order.
template <int kQ, bool kVec, int PF>
__device__ __forceinline__ void load_batch(typename WRaw<kQ>::T (&raw)[PF],
                                           const int8_t *__restrict__ wrow, int c0, int nc,
                                           int bank) {
#pragma unroll
  for (int i = 0; i < PF; ++i)
    if (c0 + i < nc) raw[i] = load_wq<kQ, kVec>(wrow + (32 * (c0 + i) + 8 * bank) * kQ / 8);
}

template <int kQ, bool kVec, int TG, int PF>
__device__ __forceinline__ void fma_batch(const typename WRaw<kQ>::T (&raw)[PF],
                                          const float *__restrict__ xs, int ld, int c0, int nc,
                                          int bank, int ng, float acc[TG][8]) {
#pragma unroll
  for (int i = 0; i < PF; ++i) {
    if (c0 + i < nc) {
      const int off = 32 * (c0 + i) + 8 * bank;
      float w[8];
      decode8(raw[i], w);
#pragma unroll
      for (int t = 0; t < TG; ++t) {
        if (t < ng) {
          float x[8];
          load_x8<kVec>(xs + t * ld + off, x);
#pragma unroll
          for (int l = 0; l < 8; ++l) acc[t][l] = __fmaf_rn(w[l], x[l], acc[t][l]);
        }
      }
    }
    // Ordering fence: keeps the scheduler from hoisting the shared-memory
    // loads of every later chunk-step (which exhausts registers).
    asm volatile("" ::: "memory");
  }
}

// Bank `bank` of a row dot for ng (<= TG) tokens whose inputs sit in smem
// rows xs + t*ld.  Weights stream through two register batches of PF
// chunk-steps: the loads of batch k+1 are in flight while batch k is
// multiplied, so memory latency overlaps the FMA chains, which still run
// strictly in chunk order.
template <int kQ, bool kVec, int TG = kTG, int PF = kPF>
__device__ __forceinline__ void bank_chain(const int8_t *__restrict__ wrow,
                                           const float *__restrict__ xs, int ld, int n, int bank,
                                           int ng, float acc[TG][8]) {
#pragma unroll
  for (int t = 0; t < TG; ++t)
#pragma unroll
    for (int l = 0; l < 8; ++l) acc[t][l] = 0.0f;
  const int nc = n / 32;
  typename WRaw<kQ>::T ra[PF], rb[PF];
  load_batch<kQ, kVec, PF>(ra, wrow, 0, nc, bank);
  for (int c0 = 0; c0 < nc; c0 += 2 * PF) {
    load_batch<kQ, kVec, PF>(rb, wrow, c0 + PF, nc, bank);
    fma_batch<kQ, kVec, TG, PF>(ra, xs, ld, c0, nc, bank, ng, acc);
    load_batch<kQ, kVec, PF>(ra, wrow, c0 + 2 * PF, nc, bank);
    fma_batch<kQ, kVec, TG, PF>(rb, xs, ld, c0 + PF, nc, bank, ng, acc);
  }
}

// Fold the four banks held by lanes L..L+3 into lane L's `tot`, then finish
// the dot there: leftover 8-chunks, horizontal fold, scalar tail.
template <int kQ>
__device__ __forceinline__ float fold_and_finish(const float acc[8], const int8_t *__restrict__ wrow,
                                                 const float *__restrict__ x, int n,
                                                 bool leader) {
  float b1[8], b2[8], b3[8];
#pragma unroll
  for (int l = 0; l < 8; ++l) {
    b1[l] = __shfl_down_sync(0xffffffffu, acc[l], 1);
    b2[l] = __shfl_down_sync(0xffffffffu, acc[l], 2);
    b3[l] = __shfl_down_sync(0xffffffffu, acc[l], 3);
  }
  if (!leader) return 0.0f;
  float tot[8];
#pragma unroll
  for (int l = 0; l < 8; ++l) tot[l] = __fadd_rn(__fadd_rn(acc[l], b1[l]), __fadd_rn(b2[l], b3[l]));
  int i = 32 * (n / 32);
  for (; i + 8 <= n; i += 8)
#pragma unroll
    for (int l = 0; l < 8; ++l) tot[l] = __fmaf_rn(w_at<kQ>(wrow, i + l), x[i + l], tot[l]);
  const float s0 = __fadd_rn(tot[0], tot[4]), s1 = __fadd_rn(tot[1], tot[5]);
  const float s2 = __fadd_rn(tot[2], tot[6]), s3 = __fadd_rn(tot[3], tot[7]);
  float s = __fadd_rn(__fadd_rn(s0, s2), __fadd_rn(s1, s3));
  for (; i < n; ++i) s = __fadd_rn(s, __fmul_rn(w_at<kQ>(wrow, i), x[i]));
  return s;
}

// Stage ng input rows (gathered through r_token) into smem.  Loads are
// issued in batches of kSB per thread before any store, so a row costs about
// one memory round trip instead of one per loop trip.  They go through L2
// (ld.cg): in the fused decode kernel the rows were written by other CTAs
// of the same launch, which L1 does not see.
constexpr int kSB = 4;
template <bool kVec>
__device__ __forceinline__ void stage_rows(float *__restrict__ xs, const float *__restrict__ src,
                                           const int32_t *__restrict__ r_token, int g0, int ng,
                                           int n) {
  if (kVec) {
    const int n4 = n / 4, total = ng * n4;
    for (int base = 0; base < total; base += blockDim.x * kSB) {
      float4 v[kSB];
#pragma unroll
      for (int k = 0; k < kSB; ++k) {
        const int i = base + k * blockDim.x + threadIdx.x;
        if (i < total) {
          const int t = i / n4, c = i % n4;
          const int row = r_token ? r_token[g0 + t] : g0 + t;
          v[k] = __ldcg(reinterpret_cast<const float4 *>(src + (size_t)row * n) + c);
        }
      }
#pragma unroll
      for (int k = 0; k < kSB; ++k) {
        const int i = base + k * blockDim.x + threadIdx.x;
        if (i < total) reinterpret_cast<float4 *>(xs)[(i / n4) * n4 + i % n4] = v[k];
      }
    }
  } else {
    for (int i = threadIdx.x; i < ng * n; i += blockDim.x) {
      const int t = i / n, c = i % n;
      const int row = r_token ? r_token[g0 + t] : g0 + t;
      xs[t * n + c] = __ldcg(src + (size_t)row * n + c);
    }
  }
}


// One gate/up item: rows [row0, row0 + 4 * nwarps) of expert (W, S) for the
// routes [r0, r1); lane layout per warp: 4 rows x (4 gate + 4 up banks).
// Called by every thread of the CTA (it stages inputs with __syncthreads).
template <bool kVec, int TG = kTG, int PF = kPF, int kQ = 8>
__device__ __forceinline__ void gate_up_item(const int8_t *__restrict__ W,
                                             const float *__restrict__ S, int H, int I, int row0,
                                             int r0, int r1, const int32_t *r_token,
                                             const float *__restrict__ x, float *xs,
                                             float *__restrict__ act) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q = lane & 7, bank = q & 3;
  const bool is_up = q >= 4;
  const int row = row0 + warp * kGURowsPerWarp + (lane >> 3);
  const bool row_ok = row < I;
  const size_t hb = (size_t)H * kQ / 8;  // bytes per row
  const int8_t *wrow = W + (is_up ? (size_t)I * hb : 0) + (size_t)(row_ok ? row : 0) * hb;
  for (int g0 = r0; g0 < r1; g0 += TG) {
    const int ng = min(TG, r1 - g0);
    __syncthreads();
    stage_rows<kVec>(xs, x, r_token, g0, ng, H);
    __syncthreads();
    float acc[TG][8];
    bank_chain<kQ, kVec, TG, PF>(wrow, xs, H, H, bank, ng, acc);
#pragma unroll
    for (int t = 0; t < TG; ++t) {
      if (t < ng) {
        const float dot = fold_and_finish<kQ>(acc[t], wrow, xs + t * H, H, bank == 0);
        const float v = __fmul_rn(dot, row_ok ? S[(is_up ? I : 0) + row] : 0.0f);
        const float u = __shfl_down_sync(0xffffffffu, v, 4);
        if (q == 0 && row_ok) {
          const float g = v;
          const float den = __fadd_rn(1.0f, expf_ref(-g));
          const float silu = __fdiv_rn(g, den);
          act[(size_t)(g0 + t) * I + row] = __fmul_rn(silu, u);
        }
      }
    }
  }
}

// One down item: rows [row0, row0 + 8 * nwarps) of expert (W, S) for routes
// [r0, r1); lane layout per warp: 8 rows x 4 banks.  `emit(route, row, y)`
// receives y = dot * s_d.  Returns false if any y is not finite.
template <bool kVec, int TG = kTG, int PF = kPF, int kQ = 8, typename Emit>
__device__ __forceinline__ bool down_item(const int8_t *__restrict__ W, const float *__restrict__ S,
                                          int H, int I, int row0, int r0, int r1,
                                          const float *__restrict__ act, float *xs, Emit emit) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bank = lane & 3;
  const int row = row0 + warp * kDNRowsPerWarp + (lane >> 2);
  const bool row_ok = row < H;
  const size_t hb = (size_t)H * kQ / 8, ib = (size_t)I * kQ / 8;  // bytes per row
  const int8_t *wrow = W + 2 * (size_t)I * hb + (size_t)(row_ok ? row : 0) * ib;
  const float *Sd = S + 2 * I;
  bool good = true;
  for (int g0 = r0; g0 < r1; g0 += TG) {
    const int ng = min(TG, r1 - g0);
    __syncthreads();
    stage_rows<kVec>(xs, act, nullptr, g0, ng, I);
    __syncthreads();
    float acc[TG][8];
    bank_chain<kQ, kVec, TG, PF>(wrow, xs, I, I, bank, ng, acc);
#pragma unroll
    for (int t = 0; t < TG; ++t) {
      if (t < ng) {
        const float dot = fold_and_finish<kQ>(acc[t], wrow, xs + t * I, I, bank == 0);
        if (bank == 0 && row_ok) {
          const float y = __fmul_rn(dot, Sd[row]);
          good &= is_finite_f(y);
          emit(g0 + t, row, y);
        }
      }
    }
  }
  return good;
}

}  // namespace gemv
}  // namespace moe
