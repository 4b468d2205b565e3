// Weight-tile ring for the exact-order GEMV of the single-launch decode
// kernel.
//
// The arithmetic is gemv_core.cuh's (the reference's AVX2 row dot,
// src/int8_expert.rs:380-458 and :473-649: one thread per (row, bank), 8
// FMA chains in chunk order, the same bank fold and tail).  Only the way the
// weight bytes reach the thread changes: instead of each thread fetching its
// own 8 (INT8) or 4 (INT4) bytes per chunk-step from global memory, the
// CTA's weight rows stream through a ring of shared-memory stages filled by
// TMA, one 8 KB tile per stage:
//   gate/up item: gate rows [row0, row0+32) and up rows [I+row0, +32), each
//                 a 32 x 128-byte box of the layer's gate/up tensor map;
//   down item:    rows [row0, row0+64), a 64 x 128-byte box of the down map.
// A stage covers 128 bytes of every row: 4 chunk-steps of INT8, 8 of INT4.
// Tiles land with the 128-byte swizzle (16-byte unit u of tile row r is
// stored at unit u ^ (r & 7)); each warp's lanes are assigned to rows so that
// its weight reads from a stage hit every shared-memory bank equally.
//
// The caller orders earlier generic-proxy writes to the ring's memory (the
// router's staging rows) with one proxy fence per layer; within the expert
// phases only TMA writes the ring.
//
// Pipeline (one pass = one token group of one item): thread 0 issues the
// pass's first kTileStages stages, each counted on its slot's mbarrier
// (transaction bytes); all threads wait on the slot, run the stage's
// chunk-steps, and meet at one barrier (which also votes on a failed wait)
// before thread 0 refills the slot with the pass's next stage.  Nothing is
// in flight between passes.  Waits are bounded: on expiry the pass drains
// its own copies in flight (at most kTileStages, each wait bounded), marks
// the ring dead and returns false; the caller records kStatusTimeout.
#pragma once

#include "gemv_core.cuh"
#include "tma_ptx.cuh"

namespace moe {
namespace gemv {

constexpr int kTileStages = 4;         // ring depth (stages in flight)
constexpr int kTileK = 128;            // bytes of each row per stage (one swizzle span)
constexpr int kTileGURows = 32;        // gate rows (and up rows) per gate/up tile
constexpr int kTileDNRows = 64;        // down rows per down tile
constexpr uint32_t kTileBytes = 8192;  // one stage: 2 x 32 x 128 or 64 x 128 bytes
constexpr size_t kTileRingBytes = (size_t)kTileStages * kTileBytes;

struct TileRing {
  uint8_t *buf;    // kTileStages x kTileBytes of shared memory, 1024-byte aligned
  uint64_t *full;  // kTileStages mbarriers (arrival count 1)
  uint32_t seq;    // stages consumed so far by this CTA (the same in every thread)
  bool dead;       // a wait gave up; the ring is not used again in this launch
};

// Gate/up stage s of item (e, row0) into the slot of sequence number u.
__device__ __forceinline__ void issue_gu(TileRing &rg, const void *map, int e, int row0, int I,
                                         int s, uint32_t u) {
  const int slot = (int)(u % kTileStages);
  uint8_t *dst = rg.buf + (size_t)slot * kTileBytes;
  tma::mbar_expect_tx(&rg.full[slot], kTileBytes);
  tma::load_3d(dst, map, &rg.full[slot], s * kTileK, row0, e);
  tma::load_3d(dst + kTileBytes / 2, map, &rg.full[slot], s * kTileK, I + row0, e);
}

// Down stage s of item (e, row0) into the slot of sequence number u.
__device__ __forceinline__ void issue_dn(TileRing &rg, const void *map, int e, int row0, int s,
                                         uint32_t u) {
  const int slot = (int)(u % kTileStages);
  tma::mbar_expect_tx(&rg.full[slot], kTileBytes);
  tma::load_3d(rg.buf + (size_t)slot * kTileBytes, map, &rg.full[slot], s * kTileK, row0, e);
}

// Raw weights of chunk-step cc (counted inside the stage) for bank `bank`
// from a swizzled 128-byte tile row with swizzle key sw = row & 7.
template <int kQ>
__device__ __forceinline__ typename WRaw<kQ>::T tile_w(const uint8_t *row, uint32_t sw, int cc,
                                                       int bank) {
  if constexpr (kQ == 8) {
    const uint32_t unit = (uint32_t)(2 * cc + (bank >> 1)) ^ sw;
    return *reinterpret_cast<const uint2 *>(row + unit * 16 + (bank & 1) * 8);
  } else {
    const uint32_t unit = (uint32_t)cc ^ sw;
    return *reinterpret_cast<const uint32_t *>(row + unit * 16 + bank * 4);
  }
}

// One chunk-step of bank `bank` for ng (<= TG) tokens: inputs at xs + t*ld
// + off, off = 32 c + 8 bank.
template <int kQ, int TG>
__device__ __forceinline__ void fma_chunk(typename WRaw<kQ>::T raw, const float *__restrict__ xs,
                                          int ld, int off, int ng, float acc[TG][8]) {
  float w[8];
  decode8(raw, w);
#pragma unroll
  for (int t = 0; t < TG; ++t) {
    if (t < ng) {
      float x[8];
      load_x8<true>(xs + t * ld + off, x);
#pragma unroll
      for (int l = 0; l < 8; ++l) acc[t][l] = __fmaf_rn(w[l], x[l], acc[t][l]);
    }
  }
}

// Thread 0: the first stages of a pass.
template <typename Issue>
__device__ __forceinline__ void tile_prologue(const TileRing &rg, int nst, Issue issue) {
  const int n = min(kTileStages, nst);
  for (int s = 0; s < n; ++s) issue(s, rg.seq + (uint32_t)s);
}

// One pass of nst stages over the item's tile rows: the thread's row sits at
// byte tile_off of each stage, its bank's chains accumulate into acc for ng
// tokens.  nc = row length / 32 (chunk-steps).  Called by every thread;
// returns false on every thread when a wait gave up.
template <int kQ, int TG, typename Issue>
__device__ __forceinline__ bool tile_pass(TileRing &rg, int nst, int nc, int tile_off,
                                          uint32_t sw, int bank, const float *__restrict__ xs,
                                          int ld, int ng, float acc[TG][8], Issue issue) {
  constexpr int kCPS = kTileK * 8 / kQ / 32;  // chunk-steps per stage: 4 (INT8), 8 (INT4)
#pragma unroll
  for (int t = 0; t < TG; ++t)
#pragma unroll
    for (int l = 0; l < 8; ++l) acc[t][l] = 0.0f;
  for (int s = 0; s < nst; ++s) {
    const uint32_t u = rg.seq + (uint32_t)s;
    const int slot = (int)(u % kTileStages);
    const bool got = tma::mbar_wait(&rg.full[slot], (u / kTileStages) & 1u, nullptr);
    if (got) {
      const uint8_t *row = rg.buf + (size_t)slot * kTileBytes + tile_off;
#pragma unroll
      for (int cc = 0; cc < kCPS; ++cc) {
        const int c = s * kCPS + cc;
        if (c < nc) fma_chunk<kQ, TG>(tile_w<kQ>(row, sw, cc, bank), xs, ld, 32 * c + 8 * bank, ng, acc);
      }
    }
    if (__syncthreads_or(!got)) {
      // Stages s .. min(nst, s + kTileStages) - 1 were issued and not
      // consumed (at most kTileStages): wait for them (bounded) before the
      // memory is reused.
      if (threadIdx.x == 0)
        for (int d = s; d < min(nst, s + kTileStages); ++d) {
          const uint32_t ud = rg.seq + (uint32_t)d;
          tma::mbar_wait(&rg.full[ud % kTileStages], (ud / kTileStages) & 1u, nullptr);
        }
      __syncthreads();
      // If a drain wait gave up too, a copy may still land in the ring: the
      // ring's shared memory is never read or reused after this (callers
      // skip every later item, and the decode kernel returns at the end of
      // the layer).
      rg.dead = true;
      return false;
    }
    if (threadIdx.x == 0 && s + kTileStages < nst) issue(s + kTileStages, u + kTileStages);
  }
  rg.seq += (uint32_t)nst;
  return true;
}

// Gate/up item on the tile ring: rows [row0, row0 + 32) of expert e for the
// routes [r0, r1), map = the layer's gate/up tensor map (H % 32 == 0).  Lane
// group j (lanes 8j .. 8j+7) runs gate row group j on lanes 8j+0..3 and up
// row group j ^ 2 on lanes 8j+4..7; row group g of warp w is tile row
// (w & 1) + 2g + 8 (w >> 1).  Same outputs as gate_up_item.
template <int TG, int kQ>
__device__ __forceinline__ bool gate_up_tile_item(TileRing &rg, const void *map, int e,
                                                  const float *__restrict__ S, int H, int I,
                                                  int row0, int r0, int r1,
                                                  const int32_t *r_token,
                                                  const float *__restrict__ x, float *xs,
                                                  float *__restrict__ act) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int q = lane & 7, bank = q & 3, j = lane >> 3;
  const bool is_up = q >= 4;
  const int jr = is_up ? (j ^ 2) : j;
  const int tr = (warp & 1) + 2 * jr + 8 * (warp >> 1);
  const int row = row0 + tr;
  const bool row_ok = row < I;
  const int nst = (H * kQ / 8 + kTileK - 1) / kTileK;
  const int tile_off = (is_up ? (int)kTileBytes / 2 : 0) + tr * kTileK;
  const uint32_t sw = (uint32_t)tr & 7u;
  const float sc = row_ok ? S[(is_up ? I : 0) + row] : 0.0f;
  const int partner = ((j ^ 2) << 3) + 4;  // lane with the up dot of this group's gate row
  auto issue = [&](int s, uint32_t u) { issue_gu(rg, map, e, row0, I, s, u); };
  for (int g0 = r0; g0 < r1; g0 += TG) {
    const int ng = min(TG, r1 - g0);
    __syncthreads();
    if (threadIdx.x == 0) tile_prologue(rg, nst, issue);
    stage_rows<true>(xs, x, r_token, g0, ng, H);
    __syncthreads();
    float acc[TG][8];
    if (!tile_pass<kQ, TG>(rg, nst, H / 32, tile_off, sw, bank, xs, H, ng, acc, issue))
      return false;
#pragma unroll
    for (int t = 0; t < TG; ++t) {
      if (t < ng) {
        const float dot = fold_and_finish<kQ>(acc[t], nullptr, xs + t * H, H, bank == 0);
        const float v = __fmul_rn(dot, sc);
        const float u = __shfl_sync(0xffffffffu, v, partner);
        if (q == 0 && row_ok) {
          const float g = v;
          const float den = __fadd_rn(1.0f, expf_ref(-g));
          const float silu = __fdiv_rn(g, den);
          act[(size_t)(g0 + t) * I + row] = __fmul_rn(silu, u);
        }
      }
    }
  }
  return true;
}

// Down item on the tile ring: rows [row0, row0 + 64) of expert e for routes
// [r0, r1) (I % 32 == 0).  Lane group jj (lanes 4jj .. 4jj+3) of warp w runs
// tile row 8 (2 (w >> 1) + (jj >> 2)) + (w & 1) + 2 (jj & 3).  `emit(route,
// row, y)` receives y = dot * s_d; good turns false on a non-finite y.  Same
// outputs as down_item.
template <int TG, int kQ, typename Emit>
__device__ __forceinline__ bool down_tile_item(TileRing &rg, const void *map, int e,
                                               const float *__restrict__ S, int H, int I,
                                               int row0, int r0, int r1,
                                               const float *__restrict__ act, float *xs,
                                               bool &good, Emit emit) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bank = lane & 3, jj = lane >> 2;
  const int tr = 8 * (2 * (warp >> 1) + (jj >> 2)) + (warp & 1) + 2 * (jj & 3);
  const int row = row0 + tr;
  const bool row_ok = row < H;
  const int nst = (I * kQ / 8 + kTileK - 1) / kTileK;
  const int tile_off = tr * kTileK;
  const uint32_t sw = (uint32_t)tr & 7u;
  const float sd = row_ok ? S[2 * I + row] : 0.0f;
  auto issue = [&](int s, uint32_t u) { issue_dn(rg, map, e, row0, s, u); };
  for (int g0 = r0; g0 < r1; g0 += TG) {
    const int ng = min(TG, r1 - g0);
    __syncthreads();
    if (threadIdx.x == 0) tile_prologue(rg, nst, issue);
    stage_rows<true>(xs, act, nullptr, g0, ng, I);
    __syncthreads();
    float acc[TG][8];
    if (!tile_pass<kQ, TG>(rg, nst, I / 32, tile_off, sw, bank, xs, I, ng, acc, issue))
      return false;
#pragma unroll
    for (int t = 0; t < TG; ++t) {
      if (t < ng) {
        const float dot = fold_and_finish<kQ>(acc[t], nullptr, xs + t * I, I, bank == 0);
        if (bank == 0 && row_ok) {
          const float y = __fmul_rn(dot, sd);
          good &= is_finite_f(y);
          emit(g0 + t, row, y);
        }
      }
    }
  }
  return true;
}

}  // namespace gemv
}  // namespace moe
