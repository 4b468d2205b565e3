// Grouped INT8 expert GEMM on the 5th-generation tensor cores (tcgen05) for
// prefill-sized batches.
//
// Math.  The reference computes g = (W_g . x) * s_g, u = (W_u . x) * s_u,
// act = silu(g) * u, y = (W_d . act) * s_d with INT8 weights and FP32
// activations (src/int8_expert.rs:969-1055).  Here the INT8 weights go to
// the tensor cores untouched and each activation row r is written as two
// signed int8 digits with a per-row scale:
//     x_r ~= s_r * (d1 + d2 / 254),   s_r = max|x_r| / 127,
// so the per-element error is <= max|x_r| / 64516.  Both digit planes are
// multiplied with `tcgen05.mma ... kind::i8` into separate int32 TMEM
// accumulators (exact integer sums), and the epilogue forms
//     dot = s_r * D1 + (s_r / 254) * D2
// in fp32.  Against the CPU path the layer output stays within the 1e-3
// relative tolerance with a wide margin (the parity tests assert it).
//
// Kernel shapes.  Default (persistent): one CTA per SM walks the work items
// (64-route tile of one expert x weight rows), 576 threads:
//   warp 0  : TMA producer (3D tiled loads, 128B swizzle, mbarrier tx count),
//             one ring running on across items
//   warp 1  : TMEM allocator + single-thread MMA issuer, alternating between
//             two TMEM accumulator buffers
//   warps 2-17: epilogue, tcgen05.ld of the accumulators (warp w reads TMEM
//             lanes 32*(w%4) .. +31), draining one buffer while the MMAs
//             fill the other.
// MOE_TC_PERSISTENT=0: one CTA per (128-row weight tile, route tile of up to
// 128 routes), 192 threads, the same roles with 4 epilogue warps.
// Every mbarrier wait is bounded: on expiry the kernel records
// kStatusTimeout, stops issuing work, waits (bounded) for its in-flight
// copies, frees its TMEM and returns.
//
// Every tensor load targets this CTA's own shared memory only.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdlib>

#include "common.cuh"
#include "expert_tc.h"
#include "digits.cuh"
#include "tma_ptx.cuh"

namespace moe {
namespace tc {
namespace {

constexpr int BM = 128;          // weight rows per tile (UMMA M)
constexpr int BK = 128;          // int8 K elements per stage (= 128 B swizzle row)
constexpr int UK = 32;           // K per tcgen05.mma kind::i8
constexpr int kThreads = 192;
constexpr uint32_t kTileBytes = BM * BK;  // 16 KB weight tile; a digit tile is BN * 128 B

// ---------------------------------------------------------------------------
// PTX wrappers (mbarrier and TMA pieces live in tma_ptx.cuh)
// ---------------------------------------------------------------------------
using tma::mbar_expect_tx;
using tma::mbar_init;
using tma::mbar_try;
using tma::mbar_wait;
using tma::su32;

__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, uint64_t *bar,
                                            int c0, int c1, int c2) {
  tma::load_3d(dst, map, bar, c0, c1, c2);
}

__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   su32(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void fence_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t *bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          su32(bar))
      : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, int32_t v[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor, K-major operand with 128-byte swizzle:
// 8-row x 128-byte atoms, atoms 1024 B apart (SBO), version 1, layout 2.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor: s32 accumulate, s8 x s8, both K-major, M=128, N=BN.
template <int BN>
__host__ __device__ constexpr uint32_t idesc_i8() {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
         ((uint32_t)(BM >> 4) << 24);
}

struct Pipe {
  uint64_t full[4];
  uint64_t empty[4];
  uint64_t done;
  uint32_t tmem_base;
  int abort_flag;
  int consumed;
};

__device__ __forceinline__ uint8_t *align1024(uint8_t *p) {
  return reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(p) + 1023) & ~uintptr_t(1023));
}

// ---------------------------------------------------------------------------
// Mainloop shared by both GEMMs: NA weight tiles x NB digit tiles per stage,
// accumulator (a, b) at TMEM column (a * NB + b) * BN.
// ---------------------------------------------------------------------------
template <int NA, int NB, int S, int BN>
__device__ __forceinline__ void mainloop(Pipe &pp, uint8_t *tiles, const CUtensorMap *mapA,
                                         const CUtensorMap *mapB, const int a_row[NA], int a_e,
                                         int b_row, int nk, uint32_t tmem) {
  constexpr uint32_t kBTile = BN * BK;
  constexpr uint32_t kStageBytes = NA * kTileBytes + NB * kBTile;
  // the NB digit tiles of a stage are adjacent 8-row swizzle atoms, so one
  // MMA of N = NB * BN covers every plane: the weight tile is read from
  // shared memory once per K step rather than once per plane
  static_assert(NB * BN <= 256 && (NB * BN) % 16 == 0, "UMMA N");
  constexpr uint32_t kIdesc = idesc_i8<NB * BN>();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp == 0 && lane == 0) {
    int issued = 0;
    for (int kb = 0; kb < nk; ++kb) {
      const int s = kb % S;
      const int use = kb / S;
      if (use > 0 && !mbar_wait(&pp.empty[s], (use - 1) & 1, &pp.abort_flag)) {
        pp.abort_flag = 1;
        break;
      }
      uint8_t *st = tiles + s * kStageBytes;
      mbar_expect_tx(&pp.full[s], kStageBytes);
#pragma unroll
      for (int a = 0; a < NA; ++a)
        tma_load_3d(st + a * kTileBytes, mapA, &pp.full[s], kb * BK, a_row[a], a_e);
#pragma unroll
      for (int b = 0; b < NB; ++b)
        tma_load_3d(st + NA * kTileBytes + b * kBTile, mapB, &pp.full[s], kb * BK, b_row, b);
      ++issued;
    }
    // On abort, the stages issued but not yet consumed must land before the
    // CTA may exit (their bytes target this CTA's shared memory).
    if (pp.abort_flag) {
      const int from = *(volatile int *)&pp.consumed;
      for (int kb = from; kb < issued; ++kb) mbar_wait(&pp.full[kb % S], (kb / S) & 1, nullptr);
    }
  } else if (warp == 1 && lane == 0) {
    int kb = 0;
    for (; kb < nk; ++kb) {
      const int s = kb % S;
      if (!mbar_wait(&pp.full[s], (kb / S) & 1, &pp.abort_flag)) {
        pp.abort_flag = 1;
        break;
      }
      fence_after_sync();
      const uint32_t base = su32(tiles + s * kStageBytes);
#pragma unroll
      for (int k = 0; k < BK / UK; ++k) {
        const uint64_t bd = sw128_desc(base + NA * kTileBytes + k * UK);
#pragma unroll
        for (int a = 0; a < NA; ++a) {
          const uint64_t ad = sw128_desc(base + a * kTileBytes + k * UK);
          mma_i8(tmem + (uint32_t)(a * NB * BN), ad, bd, kIdesc, (kb > 0 || k > 0) ? 1u : 0u);
        }
      }
      mma_commit(&pp.empty[s]);
      pp.consumed = kb + 1;
    }
    // Signals the epilogue once every issued MMA has completed.
    mma_commit(&pp.done);
  }
}

__device__ __forceinline__ void setup(Pipe &pp, int stages, uint32_t ncols) {
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&pp.full[s], 1);
      mbar_init(&pp.empty[s], 1);
    }
    mbar_init(&pp.done, 1);
    pp.abort_flag = 0;
    pp.consumed = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) tmem_alloc(&pp.tmem_base, ncols);
  __syncthreads();
  fence_after_sync();
}

__device__ __forceinline__ void teardown(Pipe &pp, uint32_t ncols, uint32_t *status) {
  fence_before_sync();
  __syncthreads();
  if (threadIdx.x == 0 && pp.abort_flag) set_status(status, kStatusTimeout);
  if ((threadIdx.x >> 5) == 1) tmem_dealloc(pp.tmem_base, ncols);
}

// Dynamic smem: [Pipe | per-route epilogue table | pad | tiles (1024-aligned)].
struct RouteTab {
  float s1[128], s2[128], gate[128];
  int32_t tok[128], slot[128], rank[128];
};
constexpr size_t smem_bytes(int na, int nb, int bn, int stages) {
  return 1024 + sizeof(Pipe) + sizeof(RouteTab) + 1024 +
         (size_t)stages * (na * kTileBytes + nb * bn * BK);
}

// Named barrier among the four epilogue warps (ids 1.., 128 threads).
__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Max over the warp's 32 lanes of each of 16 per-lane values, as a butterfly
// reduce-scatter: at each step a lane keeps half of its columns and folds in
// its partner's copy of them, so 8 + 4 + 2 + 1 + 1 shuffles reduce all 16
// columns.  Lane l ends with the maximum of column (l >> 1) & 15 (lanes l
// and l ^ 1 hold the same column).  Exact: max does not depend on order.
__device__ __forceinline__ float warp_colmax16(float (&m)[16]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int half = 8, bit = 16; half >= 1; half >>= 1, bit >>= 1) {
    const bool hi = (lane & bit) != 0;
#pragma unroll
    for (int j = 0; j < half; ++j) {
      const float send = hi ? m[j] : m[j + half];
      const float keep = hi ? m[j + half] : m[j];
      m[j] = fmaxf(keep, __shfl_xor_sync(0xffffffffu, send, bit));
    }
  }
  return fmaxf(m[0], __shfl_xor_sync(0xffffffffu, m[0], 1));
}

// Expert-parallel return of a warp's 32 output rows (this lane: row j) for
// 16 route columns c0 .. c0 + 15 of the tile: int16 values with one scale per
// (route, 32-row block), q = rint(v * 32767 / m), m = max |v| over the block;
// the source rank multiplies back by m / 32767 (per-element error <= m /
// 65534).  No cross-warp synchronisation: each warp owns its block.
__device__ __forceinline__ void ep_store16(const TcArgs &a, const RouteTab &tab, int c0, int nr,
                                           int j, int jblk, float (&v)[16]) {
  const int lane = threadIdx.x & 31;
  float mx[16];
#pragma unroll
  for (int jj = 0; jj < 16; ++jj) mx[jj] = fabsf(v[jj]);
  const float m = warp_colmax16(mx);  // lane l: column (l >> 1) & 15
  const int hb = (a.H + 31) / 32;
#pragma unroll
  for (int jj = 0; jj < 16; ++jj) {
    const int c = c0 + jj;
    const float mc = __shfl_sync(0xffffffffu, m, 2 * jj);
    if (c < nr) {
      const size_t row = (size_t)tab.tok[c] * a.K + tab.slot[c];
      if (j < a.H) {
        const float f = mc > 0.0f ? 32767.0f / mc : 0.0f;
        const float q = fminf(fmaxf(rintf(v[jj] * f), -32767.0f), 32767.0f);
        a.peer_c16[tab.rank[c]][row * a.H + j] = (int16_t)q;
      }
      if (lane == 2 * jj) a.peer_cscale[tab.rank[c]][row * hb + jblk] = mc / 32767.0f;
    }
  }
}

// The same columns as fp32 rows (ret16 == 0), or as int16 rows with scales.
__device__ __forceinline__ void ep_store(const TcArgs &a, const RouteTab &tab, int c0, int nr,
                                         int j, int jblk, float (&v)[16]) {
  if (a.ret16) {
    ep_store16(a, tab, c0, nr, j, jblk, v);
    return;
  }
#pragma unroll
  for (int jj = 0; jj < 16; ++jj) {
    const int c = c0 + jj;
    if (c < nr && j < a.H)
      a.peer_c32[tab.rank[c]][((size_t)tab.tok[c] * a.K + tab.slot[c]) * a.H + j] = v[jj];
  }
}

// ---------------------------------------------------------------------------
// GEMM 1: gate/up.  A = gate rows [m0, m0+128) and up rows [I+m0, ...) of
// expert e; B = the two digit planes of the tile's routes.  BN routes per
// tile, S pipeline stages; MINB CTAs per SM.
// ---------------------------------------------------------------------------
template <int BN, int S, int MINB>
__global__ void __launch_bounds__(kThreads, MINB)
    gate_up_tc_kernel(const __grid_constant__ CUtensorMap mapW,
                      const __grid_constant__ CUtensorMap mapX, TcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  const int g = blockIdx.y;
  if (g >= *a.n_tiles) return;
  Pipe &pp = *reinterpret_cast<Pipe *>(smem_raw);
  RouteTab &tab = *reinterpret_cast<RouteTab *>(smem_raw + sizeof(Pipe));
  uint8_t *tiles = align1024(smem_raw + sizeof(Pipe) + sizeof(RouteTab));
  const int e = a.tile_expert[g], r0 = a.tile_row0[g], nr = a.tile_rows[g];
  const int m0 = blockIdx.x * BM;
  const int nk = (a.H + BK - 1) / BK;
  constexpr uint32_t kCols = 4 * BN;
  setup(pp, S, kCols);
  const int arow[2] = {m0, a.I + m0};
  mainloop<2, 2, S, BN>(pp, tiles, &mapW, &mapX, arow, e, r0, nk, pp.tmem_base);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp >= 2) {
    // while the mainloop runs: this tile's per-route scales into smem
    for (int c = threadIdx.x - 64; c < nr; c += 128) {
      tab.s1[c] = a.xs1[r0 + c];
      tab.s2[c] = a.xs2[r0 + c];
    }
    const int q = warp & 3;
    const int i = m0 + 32 * q + lane;  // weight row of this thread
    const float *Sc = a.s_ptr[e];
    const float sg = i < a.I ? Sc[i] : 0.0f, su = i < a.I ? Sc[a.I + i] : 0.0f;
    epi_sync();
    bool ok = mbar_wait(&pp.done, 0, &pp.abort_flag);
    if (!ok) pp.abort_flag = 1;
    ok = ok && !*(volatile int *)&pp.abort_flag;  // an aborted mainloop leaves partial sums
    if (ok) {
      fence_after_sync();
      const uint32_t trow = pp.tmem_base + ((uint32_t)(32 * q) << 16);
      for (int c0 = 0; c0 < BN; c0 += 16) {
        if (c0 >= nr) break;  // warp-uniform
        int32_t v[4][16];
#pragma unroll
        for (int acc = 0; acc < 4; ++acc) tmem_ld16(trow + acc * BN + c0, v[acc]);
        tmem_wait_ld();
        float mx[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int c = c0 + j;
          float act = 0.0f;
          if (c < nr) {
            const int r = r0 + c;
            const float s1 = tab.s1[c], s2 = tab.s2[c];
            // tolerance path: the hardware exp (the GEMV path keeps libm's)
            act = digits::swiglu(v[0][j], v[1][j], v[2][j], v[3][j], s1, s2, sg, su);
            if (i < a.I) a.act[(size_t)r * a.I + i] = act;
          }
          mx[j] = fabsf(act);
        }
        // max |act| over this warp's 32 rows, all 16 route columns at once
        const float m = warp_colmax16(mx);
        const int c = c0 + ((lane >> 1) & 15);
        if ((lane & 1) == 0 && c < nr) atomicMax(&a.act_amax[r0 + c], __float_as_uint(m));
      }
    }
  }
  teardown(pp, kCols, a.status);
}

// ---------------------------------------------------------------------------
// GEMM 2: down.  A = down rows [m0, m0+128) of expert e (K = I); B = the
// digit planes of the tile's activations.  Epilogue writes gate * y into the
// (token, slot) contribution row.
// ---------------------------------------------------------------------------
template <int BN, int S, int MINB>
__global__ void __launch_bounds__(kThreads, MINB)
    down_tc_kernel(const __grid_constant__ CUtensorMap mapW,
                   const __grid_constant__ CUtensorMap mapA, TcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  const int g = blockIdx.y;
  if (g >= *a.n_tiles) return;
  Pipe &pp = *reinterpret_cast<Pipe *>(smem_raw);
  RouteTab &tab = *reinterpret_cast<RouteTab *>(smem_raw + sizeof(Pipe));
  uint8_t *tiles = align1024(smem_raw + sizeof(Pipe) + sizeof(RouteTab));
  const int e = a.tile_expert[g], r0 = a.tile_row0[g], nr = a.tile_rows[g];
  const int m0 = blockIdx.x * BM;
  const int nk = (a.I + BK - 1) / BK;
  constexpr uint32_t kCols = 2 * BN;
  setup(pp, S, kCols);
  const int arow[1] = {m0};
  mainloop<1, 2, S, BN>(pp, tiles, &mapW, &mapA, arow, e, r0, nk, pp.tmem_base);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp >= 2) {
    for (int c = threadIdx.x - 64; c < nr; c += 128) {
      const int r = r0 + c;
      tab.s1[c] = a.as1[r];
      tab.s2[c] = a.as2[r];
      tab.gate[c] = a.r_gate[r];
      tab.tok[c] = a.r_token[r];
      tab.slot[c] = a.r_slot[r];
      tab.rank[c] = a.r_rank ? a.r_rank[r] : 0;
    }
    const int q = warp & 3;
    const int j = m0 + 32 * q + lane;  // output row (hidden index)
    const float sd = j < a.H ? a.s_ptr[e][2 * a.I + j] : 0.0f;
    epi_sync();
    bool ok = mbar_wait(&pp.done, 0, &pp.abort_flag);
    if (!ok) pp.abort_flag = 1;
    ok = ok && !*(volatile int *)&pp.abort_flag;  // an aborted mainloop leaves partial sums
    if (ok) {
      fence_after_sync();
      const uint32_t trow = pp.tmem_base + ((uint32_t)(32 * q) << 16);
      bool bad = false;
      for (int c0 = 0; c0 < BN; c0 += 16) {
        if (c0 >= nr) break;
        int32_t v[2][16];
        tmem_ld16(trow + c0, v[0]);
        tmem_ld16(trow + BN + c0, v[1]);
        tmem_wait_ld();
        float gy[16];
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) {
          const int c = c0 + jj;
          gy[jj] = 0.0f;
          if (c < nr && j < a.H) {
            const float y = digits::down(v[0][jj], v[1][jj], tab.s1[c], tab.s2[c], sd);
            bad |= !is_finite_f(y);
            gy[jj] = __fmul_rn(tab.gate[c], y);
            if (!a.r_rank) a.contrib[((size_t)tab.tok[c] * a.K + tab.slot[c]) * a.H + j] = gy[jj];
          }
        }
        // expert parallelism: the rows go straight to the source ranks'
        // buffers (peer memory over NVLink)
        if (a.r_rank) ep_store(a, tab, c0, nr, j, (m0 + 32 * q) / 32, gy);
      }
      if (bad) set_status(a.status, kStatusNonFinite);
    }
  }
  teardown(pp, kCols, a.status);
}

// ---------------------------------------------------------------------------
// Persistent variants: one CTA per SM walks the work items (route tile g,
// 128-row weight tile m) with a stride of gridDim.x.  The producer's TMA
// stages run on across work items; the MMA thread alternates between two
// TMEM accumulator buffers, so the epilogue of one item overlaps the
// mainloop of the next.  64-route tiles (two buffers of 4 x 64 columns for
// gate/up, 2 x 64 for down).
// ---------------------------------------------------------------------------
constexpr int PBN = 64;

struct PPipe {
  uint64_t full[8];
  uint64_t empty[8];
  uint64_t tfull[2];
  uint64_t tempty[2];
  uint64_t done;
  uint32_t tmem_base;
  int abort_flag;
  int consumed;
};

// The persistent kernels run kPEpiWarps epilogue warps (warps 2 ..): warp w
// reads TMEM lane quarter w % 4 (the hardware's rule), and the kPEpiGroups
// warps of a quarter split each item's columns (and, in the two-block down
// GEMM, its row blocks) between them.  The epilogue is issue-latency bound
// (dependent per-element chains), so more warps drain an item faster while
// the MMAs fill the other TMEM buffer.
constexpr int kPEpiWarps = 16;
constexpr int kPEpiGroups = kPEpiWarps / 4;
constexpr int kPThreads = 64 + 32 * kPEpiWarps;
static_assert(PBN % (16 * kPEpiGroups) == 0, "column split");

__device__ __forceinline__ void pepi_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(32 * kPEpiWarps) : "memory");
}

// Barrier among the epilogue warps that ORs a predicate over them, so every
// epilogue thread leaves the tile loop at the same item on an abort.
__device__ __forceinline__ bool epi_any(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, 1, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)v), "n"(32 * kPEpiWarps)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ void mbar_arrive_plain(uint64_t *bar) { tma::mbar_arrive(bar); }

__device__ __forceinline__ void psetup(PPipe &pp, int stages, uint32_t ncols) {
  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&pp.full[s], 1);
      mbar_init(&pp.empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&pp.tfull[b], 1);
      mbar_init(&pp.tempty[b], kPEpiWarps);  // one arrive per epilogue warp
    }
    mbar_init(&pp.done, 1);
    pp.abort_flag = 0;
    pp.consumed = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if ((threadIdx.x >> 5) == 1) tmem_alloc(&pp.tmem_base, ncols);
  __syncthreads();
  fence_after_sync();
}

// Producer (warp 0, one thread) and MMA issuer (warp 1, one thread) of the
// persistent kernels.  NA weight tiles (rows arow(m, a)) x NB digit tiles
// per stage; accumulator (a, b) of buffer buf at TMEM column
// buf * NA * NB * PBN + (a * NB + b) * PBN.
template <int NA, int NB, int S, typename ARow>
__device__ __forceinline__ void pmain(PPipe &pp, uint8_t *tiles, const CUtensorMap *mapA,
                                      const CUtensorMap *mapB, const TcArgs &a, int nwork,
                                      int nM, int nk, ARow arow) {
  constexpr uint32_t kBTile = PBN * BK;
  constexpr uint32_t kStageBytes = NA * kTileBytes + NB * kBTile;
  static_assert(NB * PBN <= 256 && (NB * PBN) % 16 == 0, "UMMA N");
  constexpr uint32_t kIdesc = idesc_i8<NB * PBN>();  // every plane in one MMA
  constexpr uint32_t kBufCols = NA * NB * PBN;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp == 0 && lane == 0) {
    int q = 0;
    for (int w = blockIdx.x; w < nwork; w += gridDim.x) {
      const int g = w / nM, m = w % nM;
      const int e = a.tile_expert[g], r0 = a.tile_row0[g];
      for (int kb = 0; kb < nk; ++kb, ++q) {
        const int s = q % S, use = q / S;
        if (use > 0 && !mbar_wait(&pp.empty[s], (use - 1) & 1, &pp.abort_flag)) {
          pp.abort_flag = 1;
          break;
        }
        uint8_t *st = tiles + s * kStageBytes;
        mbar_expect_tx(&pp.full[s], kStageBytes);
#pragma unroll
        for (int x = 0; x < NA; ++x)
          tma_load_3d(st + x * kTileBytes, mapA, &pp.full[s], kb * BK, arow(m, x), e);
#pragma unroll
        for (int b = 0; b < NB; ++b)
          tma_load_3d(st + NA * kTileBytes + b * kBTile, mapB, &pp.full[s], kb * BK, r0, b);
      }
      if (pp.abort_flag) break;
    }
    if (pp.abort_flag) {  // issued stages must land before the CTA may exit
      const int from = *(volatile int *)&pp.consumed;
      for (int k = from; k < q; ++k) mbar_wait(&pp.full[k % S], (k / S) & 1, nullptr);
    }
  } else if (warp == 1 && lane == 0) {
    int q = 0, j = 0;
    for (int w = blockIdx.x; w < nwork; w += gridDim.x, ++j) {
      const int buf = j & 1;
      if (j >= 2 && !mbar_wait(&pp.tempty[buf], ((j >> 1) - 1) & 1, &pp.abort_flag)) {
        pp.abort_flag = 1;
        break;
      }
      fence_after_sync();
      const uint32_t tmem = pp.tmem_base + (uint32_t)(buf * kBufCols);
      bool ok = true;
      for (int kb = 0; kb < nk; ++kb, ++q) {
        const int s = q % S;
        if (!mbar_wait(&pp.full[s], (q / S) & 1, &pp.abort_flag)) {
          pp.abort_flag = 1;
          ok = false;
          break;
        }
        fence_after_sync();
        const uint32_t base = su32(tiles + s * kStageBytes);
#pragma unroll
        for (int k = 0; k < BK / UK; ++k) {
          const uint64_t bd = sw128_desc(base + NA * kTileBytes + k * UK);
#pragma unroll
          for (int x = 0; x < NA; ++x) {
            const uint64_t ad = sw128_desc(base + x * kTileBytes + k * UK);
            mma_i8(tmem + (uint32_t)(x * NB * PBN), ad, bd, kIdesc, (kb > 0 || k > 0) ? 1u : 0u);
          }
        }
        mma_commit(&pp.empty[s]);
        pp.consumed = q + 1;
      }
      if (!ok) break;
      mma_commit(&pp.tfull[buf]);
    }
    mma_commit(&pp.done);  // every MMA issued by this CTA has completed
  }
}

__device__ __forceinline__ void pteardown(PPipe &pp, uint32_t ncols, uint32_t *status) {
  if (threadIdx.x == 32) mbar_wait(&pp.done, 0, nullptr);  // no MMA still writes TMEM
  fence_before_sync();
  __syncthreads();
  if (threadIdx.x == 0 && pp.abort_flag) set_status(status, kStatusTimeout);
  if ((threadIdx.x >> 5) == 1) tmem_dealloc(pp.tmem_base, ncols);
}

constexpr size_t psmem_bytes(int na, int nb, int stages) {
  return 1024 + sizeof(PPipe) + 2 * sizeof(RouteTab) + 1024 +
         (size_t)stages * (na * kTileBytes + nb * PBN * BK);
}

template <int S>
__global__ void __launch_bounds__(kPThreads, 1)
    gate_up_tc_pkernel(const __grid_constant__ CUtensorMap mapW,
                       const __grid_constant__ CUtensorMap mapX, TcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  PPipe &pp = *reinterpret_cast<PPipe *>(smem_raw);
  RouteTab *tabs = reinterpret_cast<RouteTab *>(smem_raw + sizeof(PPipe));
  uint8_t *tiles = align1024(smem_raw + sizeof(PPipe) + 2 * sizeof(RouteTab));
  const int nM = (a.I + BM - 1) / BM, nwork = *a.n_tiles * nM, nk = (a.H + BK - 1) / BK;
  constexpr uint32_t kCols = 2 * 4 * PBN;
  psetup(pp, S, kCols);
  const int I = a.I;
  pmain<2, 2, S>(pp, tiles, &mapW, &mapX, a, nwork, nM, nk,
                 [I](int m, int x) { return x * I + m * BM; });
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp >= 2) {
    const int qd = warp & 3, grp = (warp - 2) >> 2;
    constexpr int kNC = PBN / kPEpiGroups;  // columns of this warp's share
    int j = 0;
    for (int w = blockIdx.x; w < nwork; w += gridDim.x, ++j) {
      const int buf = j & 1, g = w / nM, m = w % nM;
      const int e = a.tile_expert[g], r0 = a.tile_row0[g], nr = a.tile_rows[g];
      RouteTab &tab = tabs[buf];
      const int i = m * BM + 32 * qd + lane;  // weight row of this thread
      const float *Sc = a.s_ptr[e];
      const float sg = i < I ? Sc[i] : 0.0f, su = i < I ? Sc[I + i] : 0.0f;
      pepi_sync();  // every epilogue warp is past the item that last used tab[buf]
      for (int c = threadIdx.x - 64; c < nr; c += 32 * kPEpiWarps) {
        tab.s1[c] = a.xs1[r0 + c];
        tab.s2[c] = a.xs2[r0 + c];
      }
      pepi_sync();
      const bool ok = mbar_wait(&pp.tfull[buf], (j >> 1) & 1, &pp.abort_flag);
      if (epi_any(!ok)) {  // uniform over the epilogue warps
        pp.abort_flag = 1;
        break;
      }
      fence_after_sync();
      const uint32_t trow =
          pp.tmem_base + (uint32_t)(buf * 4 * PBN) + ((uint32_t)(32 * qd) << 16);
      for (int c0 = grp * kNC; c0 < (grp + 1) * kNC; c0 += 16) {
        if (c0 >= nr) break;  // warp-uniform
        int32_t v[4][16];
#pragma unroll
        for (int acc = 0; acc < 4; ++acc) tmem_ld16(trow + acc * PBN + c0, v[acc]);
        tmem_wait_ld();
        float mx[16];
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) {
          const int c = c0 + jj;
          float act = 0.0f;
          if (c < nr) {
            const int r = r0 + c;
            const float s1 = tab.s1[c], s2 = tab.s2[c];
act = digits::swiglu(v[0][jj], v[1][jj], v[2][jj], v[3][jj], s1, s2, sg, su);
            if (i < I) a.act[(size_t)r * I + i] = act;
          }
          mx[jj] = fabsf(act);
        }
        const float m = warp_colmax16(mx);
        const int cm = c0 + ((lane >> 1) & 15);
        if ((lane & 1) == 0 && cm < nr) atomicMax(&a.act_amax[r0 + cm], __float_as_uint(m));
      }
      fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive_plain(&pp.tempty[buf]);
    }
  }
  pteardown(pp, kCols, a.status);
}

// NA weight row blocks per work item: with NA = 2 the item's digit tile is
// loaded once for 256 output rows (half the activation traffic of NA = 1).
// The kPEpiGroups epilogue warps of a TMEM lane quarter split the item's
// NA row blocks x 64 columns evenly.
template <int S, int NA>
__global__ void __launch_bounds__(kPThreads, 1)
    down_tc_pkernel(const __grid_constant__ CUtensorMap mapW,
                    const __grid_constant__ CUtensorMap mapA, TcArgs a) {
  static_assert(NA == 1 || NA == 2, "row blocks per item");
  extern __shared__ uint8_t smem_raw[];
  PPipe &pp = *reinterpret_cast<PPipe *>(smem_raw);
  RouteTab *tabs = reinterpret_cast<RouteTab *>(smem_raw + sizeof(PPipe));
  uint8_t *tiles = align1024(smem_raw + sizeof(PPipe) + 2 * sizeof(RouteTab));
  const int nM = (a.H + NA * BM - 1) / (NA * BM), nwork = *a.n_tiles * nM;
  const int nk = (a.I + BK - 1) / BK;
  constexpr uint32_t kBufCols = NA * 2 * PBN;
  constexpr uint32_t kCols = 2 * kBufCols;
  psetup(pp, S, kCols);
  pmain<NA, 2, S>(pp, tiles, &mapW, &mapA, a, nwork, nM, nk,
                  [](int m, int x) { return (NA * m + x) * BM; });
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp >= 2) {
    static_assert(kPEpiGroups % NA == 0, "row split");
    constexpr int kNC = PBN * NA / kPEpiGroups;  // columns of this warp's share
    const int qd = warp & 3, grp = (warp - 2) >> 2;
    const int x = grp % NA;                       // row block of the item
    const int cb = (grp / NA) * kNC, ce = cb + kNC;
    bool bad = false;
    int j = 0;
    for (int w = blockIdx.x; w < nwork; w += gridDim.x, ++j) {
      const int buf = j & 1, g = w / nM, m = w % nM;
      const int e = a.tile_expert[g], r0 = a.tile_row0[g], nr = a.tile_rows[g];
      RouteTab &tab = tabs[buf];
      const int rb = (NA * m + x) * BM + 32 * qd;  // first output row of this warp
      const int jr = rb + lane;                    // output row (hidden index)
      const float sd = jr < a.H ? a.s_ptr[e][2 * a.I + jr] : 0.0f;
      pepi_sync();
      for (int c = threadIdx.x - 64; c < nr; c += 32 * kPEpiWarps) {
        const int r = r0 + c;
        tab.s1[c] = a.as1[r];
        tab.s2[c] = a.as2[r];
        tab.gate[c] = a.r_gate[r];
        tab.tok[c] = a.r_token[r];
        tab.slot[c] = a.r_slot[r];
        tab.rank[c] = a.r_rank ? a.r_rank[r] : 0;
      }
      pepi_sync();
      const bool ok = mbar_wait(&pp.tfull[buf], (j >> 1) & 1, &pp.abort_flag);
      if (epi_any(!ok)) {  // uniform over the epilogue warps
        pp.abort_flag = 1;
        break;
      }
      fence_after_sync();
      const uint32_t trow = pp.tmem_base + (uint32_t)(buf * kBufCols + x * 2 * PBN) +
                            ((uint32_t)(32 * qd) << 16);
      if (rb < a.H) {  // warp-uniform: a row block past H has nothing to store
        for (int c0 = cb; c0 < ce; c0 += 16) {
          if (c0 >= nr) break;
          int32_t v[2][16];
          tmem_ld16(trow + c0, v[0]);
          tmem_ld16(trow + PBN + c0, v[1]);
          tmem_wait_ld();
          float gy[16];
#pragma unroll
          for (int jj = 0; jj < 16; ++jj) {
            const int c = c0 + jj;
            gy[jj] = 0.0f;
            if (c < nr && jr < a.H) {
              const float y = digits::down(v[0][jj], v[1][jj], tab.s1[c], tab.s2[c], sd);
              bad |= !is_finite_f(y);
              gy[jj] = __fmul_rn(tab.gate[c], y);
              if (!a.r_rank)
                a.contrib[((size_t)tab.tok[c] * a.K + tab.slot[c]) * a.H + jr] = gy[jj];
            }
          }
          if (a.r_rank) ep_store(a, tab, c0, nr, jr, rb / 32, gy);
        }
      }
      fence_before_sync();
      __syncwarp();
      if (lane == 0) mbar_arrive_plain(&pp.tempty[buf]);
    }
    if (bad) set_status(a.status, kStatusNonFinite);
  }
  pteardown(pp, kCols, a.status);
}

// ---------------------------------------------------------------------------
// Tile table and activation digit planes
// ---------------------------------------------------------------------------
// Tile table: tile t of the layer covers routes [row0, row0 + rows) of one
// expert.  One thread per active expert; block-wide exclusive scan of the
// per-expert tile counts (E <= 256).
__global__ void __launch_bounds__(256) build_tiles_kernel(const int32_t *seg_off,
                                                          const int32_t *active,
                                                          const int32_t *n_active, int bn,
                                                          int32_t *tile_expert,
                                                          int32_t *tile_row0, int32_t *tile_rows,
                                                          int32_t *n_tiles, int max_tiles) {
  __shared__ int32_t scan[256];
  const int j = threadIdx.x;
  const int na = *n_active;
  int e = -1, cnt = 0;
  if (j < na) {
    e = active[j];
    cnt = (seg_off[e + 1] - seg_off[e] + bn - 1) / bn;
  }
  scan[j] = cnt;
  __syncthreads();
  for (int o = 1; o < 256; o <<= 1) {  // inclusive Hillis-Steele scan
    const int v = j >= o ? scan[j - o] : 0;
    __syncthreads();
    scan[j] += v;
    __syncthreads();
  }
  const int first = scan[j] - cnt;
  for (int k = 0; k < cnt && first + k < max_tiles; ++k) {
    const int r = seg_off[e] + k * bn;
    tile_expert[first + k] = e;
    tile_row0[first + k] = r;
    tile_rows[first + k] = min(bn, seg_off[e + 1] - r);
  }
  if (j == 255) *n_tiles = min(scan[255], max_tiles);
}

// One warp per route row: s = max|v| / 127, d1 = rint(v/s), d2 = rint((v/s - d1) * 254).
// src rows are gathered through `rows` (null = identity).  Also resets the
// per-row amax used by the next stage when `amax_reset` is given.
__global__ void quantize_rows_kernel(const float *__restrict__ src, const int32_t *__restrict__ rows,
                                     const uint32_t *__restrict__ amax_in, int R,
                                     const int32_t *__restrict__ R_dev, int n,
                                     int8_t *__restrict__ q, size_t plane, float *__restrict__ s1,
                                     float *__restrict__ s2, uint32_t *__restrict__ amax_reset) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= R || (R_dev && warp >= *R_dev)) return;
  const int row = rows ? rows[warp] : warp;
  const float *x = src + (size_t)row * n;
  float amax;
  if (amax_in) {
    amax = __uint_as_float(amax_in[warp]);
  } else {
    amax = 0.0f;
#pragma unroll 4
    for (int c = lane * 4; c < n; c += 128) {
      const float4 v = *reinterpret_cast<const float4 *>(x + c);
      amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  }
  const float s = digits::row_scale(amax);
  const float inv = 1.0f / s;
  int8_t *q1 = q + (size_t)warp * n;
  int8_t *q2 = q + plane + (size_t)warp * n;
#pragma unroll 4
  for (int c = lane * 4; c < n; c += 128) {
    const float4 v = *reinterpret_cast<const float4 *>(x + c);
    uint32_t p2;
    const uint32_t p1 = digits::split4(v.x, v.y, v.z, v.w, inv, p2);
    *reinterpret_cast<uint32_t *>(q1 + c) = p1;
    *reinterpret_cast<uint32_t *>(q2 + c) = p2;
  }
  if (lane == 0) {
    s1[warp] = s;
    s2[warp] = s / 254.0f;
    if (amax_reset) amax_reset[warp] = 0u;
  }
}

// One CTA per token: the token's row is quantized once, with the same
// arithmetic as quantize_rows_kernel, and the digits are stored at each of
// its K routes' expert-sorted rows (r_pos; negative or out-of-range
// positions, which invalid routes leave, are skipped), with the per-route
// scales; the routes' activation amax is cleared for the gate/up epilogue.
// A thread owns 16 consecutive elements per pass (n % 16 == 0), so every
// digit store is 16 bytes.
constexpr int kQtThreads = 128;
__device__ __forceinline__ uint32_t digits4(const float4 v, float inv, uint32_t &hi) {
  return digits::split4(v.x, v.y, v.z, v.w, inv, hi);
}

__global__ void __launch_bounds__(kQtThreads, 4) quantize_tokens_kernel(
    const float *__restrict__ x, const int32_t *__restrict__ r_pos, int T, int K, int n,
    int8_t *__restrict__ q, size_t plane, float *__restrict__ s1, float *__restrict__ s2,
    uint32_t *__restrict__ amax_reset) {
  __shared__ float wmax[kQtThreads / 32];
  __shared__ int pos_s[kMaxTopK];
  const int t = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t R = (uint32_t)T * (uint32_t)K;
  if (tid < K) pos_s[tid] = r_pos[(size_t)t * K + tid];
  const float4 *row = reinterpret_cast<const float4 *>(x + (size_t)t * n);
  float amax = 0.0f;
  for (int c = tid * 16; c < n; c += kQtThreads * 16) {
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float4 v = row[c / 4 + w];
      amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if (lane == 0) wmax[warp] = amax;
  __syncthreads();
#pragma unroll
  for (int w = 0; w < kQtThreads / 32; ++w) amax = fmaxf(amax, wmax[w]);
  const float s = digits::row_scale(amax);
  const float inv = 1.0f / s;
  int pos[kMaxTopK];
#pragma unroll
  for (int k = 0; k < kMaxTopK; ++k) pos[k] = k < K ? pos_s[k] : -1;
  for (int c = tid * 16; c < n; c += kQtThreads * 16) {
    uint4 lo, hi;
    lo.x = digits4(row[c / 4 + 0], inv, hi.x);
    lo.y = digits4(row[c / 4 + 1], inv, hi.y);
    lo.z = digits4(row[c / 4 + 2], inv, hi.z);
    lo.w = digits4(row[c / 4 + 3], inv, hi.w);
#pragma unroll
    for (int k = 0; k < kMaxTopK; ++k)
      if ((uint32_t)pos[k] < R) {
        *reinterpret_cast<uint4 *>(q + (size_t)pos[k] * n + c) = lo;
        *reinterpret_cast<uint4 *>(q + plane + (size_t)pos[k] * n + c) = hi;
      }
  }
  if (tid < K && (uint32_t)pos_s[tid] < R) {
    s1[pos_s[tid]] = s;
    s2[pos_s[tid]] = s / 254.0f;
    if (amax_reset) amax_reset[pos_s[tid]] = 0u;
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

}  // namespace

bool encode_map3d(CUtensorMap *map, const void *base, uint64_t d0, uint64_t d1, uint64_t d2,
                  uint64_t stride1, uint64_t stride2, uint32_t box_rows) {
  auto enc = encoder();
  if (!enc) return false;
  if (((uintptr_t)base & 15) || (stride1 & 15) || (stride2 & 15)) return false;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {stride1, stride2};
  cuuint32_t box[3] = {(cuuint32_t)BK, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void *>(base), dims,
                         strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

cudaError_t launch_build_tiles(const int32_t *seg_off, const int32_t *active,
                               const int32_t *n_active, int bn, int32_t *tile_expert,
                               int32_t *tile_row0, int32_t *tile_rows, int32_t *n_tiles,
                               int max_tiles, cudaStream_t s) {
  build_tiles_kernel<<<1, 256, 0, s>>>(seg_off, active, n_active, bn, tile_expert, tile_row0,
                                       tile_rows, n_tiles, max_tiles);
  return cudaGetLastError();
}

cudaError_t launch_quantize_rows(const float *src, const int32_t *rows, const uint32_t *amax_in,
                                 int R, int n, int8_t *q, size_t plane, float *s1, float *s2,
                                 uint32_t *amax_reset, cudaStream_t s, const int32_t *R_dev) {
  if (R <= 0) return cudaSuccess;
  quantize_rows_kernel<<<(R + 7) / 8, 256, 0, s>>>(src, rows, amax_in, R, R_dev, n, q, plane, s1,
                                                   s2, amax_reset);
  return cudaGetLastError();
}

cudaError_t launch_quantize_tokens(const float *x, const int32_t *r_pos, int T, int K, int n,
                                   int8_t *q, size_t plane, float *s1, float *s2,
                                   uint32_t *amax_reset, cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  if (K > kMaxTopK || n % 16) return cudaErrorInvalidValue;
  quantize_tokens_kernel<<<T, kQtThreads, 0, s>>>(x, r_pos, T, K, n, q, plane, s1, s2,
                                                  amax_reset);
  return cudaGetLastError();
}

// Persistent tile loop with double-buffered accumulators for 64-route tiles:
// Persistent kernels (one CTA per SM walking 64-route work items, TMEM double
// buffered, 8 epilogue warps) for both GEMMs by default: measured on B200
// faster than one CTA per tile at Qwen3 T = 512, 1376 and 4096 and OLMoE
// T = 512.  MOE_TC_PERSISTENT=0 selects one CTA per tile, =2 persistent down
// only, =3 persistent gate/up only.
int persistent_mode() {
  static int v = -1;
  if (v < 0) {
    const char *env = getenv("MOE_TC_PERSISTENT");
    v = env ? atoi(env) : 1;
    if (v < 0 || v > 3) v = 1;
  }
  return v;
}
bool persistent_gu() { return persistent_mode() == 1 || persistent_mode() == 3; }
bool persistent_dn() { return persistent_mode() == 1 || persistent_mode() == 2; }

int tc_bn_dn_override() {
  static int v = -1;
  if (v < 0) {
    const char *env = getenv("MOE_TC_BN_DN");
    v = env ? atoi(env) : 0;
    if (v != 64 && v != 128) v = 0;
  }
  return v;
}

int tc_bn_override() {
  static int v = -1;
  if (v < 0) {
    const char *env = getenv("MOE_TC_BN");
    v = env ? atoi(env) : 0;
    if (v != 64 && v != 128) v = 0;
  }
  return v;
}

// Tile configurations.  BN = 64: 2 CTAs per SM (TMEM 4*64 and 2*64 columns,
// 96 KB of pipeline each).  BN = 128: gate/up one CTA per SM (512 TMEM
// columns, 3 stages), down two per SM.
template <int BN, int S, int MINB>
cudaError_t launch_gu(const CUtensorMap &mapW, const CUtensorMap &mapX, const TcArgs &a,
                      int max_tiles, cudaStream_t s) {
  const size_t smem = smem_bytes(2, 2, BN, S);
  auto k = gate_up_tc_kernel<BN, S, MINB>;
  cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  dim3 grid((a.I + BM - 1) / BM, max_tiles);
  k<<<grid, kThreads, smem, s>>>(mapW, mapX, a);
  return cudaGetLastError();
}

template <int BN, int S, int MINB>
cudaError_t launch_dn(const CUtensorMap &mapW, const CUtensorMap &mapA, const TcArgs &a,
                      int max_tiles, cudaStream_t s) {
  const size_t smem = smem_bytes(1, 2, BN, S);
  auto k = down_tc_kernel<BN, S, MINB>;
  cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  dim3 grid((a.H + BM - 1) / BM, max_tiles);
  k<<<grid, kThreads, smem, s>>>(mapW, mapA, a);
  return cudaGetLastError();
}

// Persistent kernels: one CTA per SM (at most one per work item).
int sm_count_cached() {
  static int n = 0;
  if (n == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

constexpr int kPStagesGU = 4, kPStagesDN = 6, kPStagesDN2 = 4;

// MOE_TC_DN_ROWS=1: one 128-row weight block per persistent down item
// (default two).
int dn_rows() {
  static int v = -1;
  if (v < 0) {
    const char *env = getenv("MOE_TC_DN_ROWS");
    v = env && atoi(env) == 1 ? 1 : 2;
  }
  return v;
}

cudaError_t launch_gate_up_tc(const CUtensorMap &mapW, const CUtensorMap &mapX, const TcArgs &a,
                              int bn, int max_tiles, cudaStream_t s) {
  if (bn == PBN && persistent_gu()) {
    const size_t smem = psmem_bytes(2, 2, kPStagesGU);
    auto k = gate_up_tc_pkernel<kPStagesGU>;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    const long long work = (long long)max_tiles * ((a.I + BM - 1) / BM);
    const int grid = (int)std::min<long long>(sm_count_cached(), std::max<long long>(work, 1));
    k<<<grid, kPThreads, smem, s>>>(mapW, mapX, a);
    return cudaGetLastError();
  }
  return bn == 64 ? launch_gu<64, 2, 2>(mapW, mapX, a, max_tiles, s)
                  : launch_gu<128, 3, 1>(mapW, mapX, a, max_tiles, s);
}

cudaError_t launch_down_tc(const CUtensorMap &mapW, const CUtensorMap &mapA, const TcArgs &a,
                           int bn, int max_tiles, cudaStream_t s) {
  if (bn == PBN && persistent_dn()) {
    const int na = dn_rows();
    const size_t smem = na == 2 ? psmem_bytes(2, 2, kPStagesDN2) : psmem_bytes(1, 2, kPStagesDN);
    auto k = na == 2 ? down_tc_pkernel<kPStagesDN2, 2> : down_tc_pkernel<kPStagesDN, 1>;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    const long long work = (long long)max_tiles * ((a.H + na * BM - 1) / (na * BM));
    const int grid = (int)std::min<long long>(sm_count_cached(), std::max<long long>(work, 1));
    k<<<grid, kPThreads, smem, s>>>(mapW, mapA, a);
    return cudaGetLastError();
  }
  return bn == 64 ? launch_dn<64, 3, 2>(mapW, mapA, a, max_tiles, s)
                  : launch_dn<128, 2, 2>(mapW, mapA, a, max_tiles, s);
}

}  // namespace tc
}  // namespace moe
