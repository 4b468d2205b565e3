// Router projection, softmax, top-k and the by-expert permutation.
//
// Reference semantics (juanhuy/DoanTotNghiepMOE):
//   logits   src/backend.rs:105-120 (`dot_product`: 8 lane accumulators over
//            chunks of 8, lanes folded in order, sequential tail) and
//            src/dense.rs:58-73 (`dot_bf16`, same order on widened BF16);
//   softmax  src/backend.rs:375-389 (max, exp(x - max), sequential sum, divide);
//   top-k    src/olmoe.rs:2595-2621 (total_cmp descending, ties -> lower id,
//            normalizer = sequential sum of the selected p when norm_topk_prob);
//   variant  src/router.rs:50-103 (`route_hidden`: sequential dot, sort by
//            score, softmax over the kept k);
//   permute  src/olmoe.rs:3474-3480 (`expert_uses`: experts ascending, tokens
//            ascending within an expert).
// Every floating-point step is the same IEEE operation in the same order, so
// logits, probabilities, ids and gates are bit-identical to the CPU path.
#include <cstdlib>

#include "common.cuh"
#include "kernels.h"
#include "route_core.cuh"

namespace moe {
namespace {

constexpr int kRouteThreads = 256;

// Small T (decode): one CTA per (token, 4 experts).  The token row and the 4
// router rows are staged into shared memory in one shot -- every thread
// issues its loads of a batch before the first store -- so the kernel pays
// about one memory round trip; then 32 threads run the 8-lane chains.
constexpr int kSmallTE = 4;
__global__ void __launch_bounds__(kRouteThreads) route_logits_small_kernel(RouteArgs a) {
  extern __shared__ float sm[];  // [1 + kSmallTE][H]
  const int tid = threadIdx.x;
  const int e0 = blockIdx.x * kSmallTE, t = blockIdx.y;
  const int H = a.H;
  float *hs = sm, *ws = sm + H;
  bool bad_input = false;
  constexpr int kBatch = 8;
  const int total = (1 + kSmallTE) * H;
  for (int base = 0; base < total; base += kRouteThreads * kBatch) {
    float v[kBatch];
#pragma unroll
    for (int k = 0; k < kBatch; ++k) {
      const int i = base + k * kRouteThreads + tid;
      v[k] = 0.0f;
      if (i < H) {
        v[k] = a.h[(size_t)t * H + i];
      } else if (i < total) {
        const int r = i / H - 1, c = i % H;
        if (e0 + r < a.E) v[k] = load_w(a.router, a.router_dtype, (size_t)(e0 + r) * H + c);
      }
    }
#pragma unroll
    for (int k = 0; k < kBatch; ++k) {
      const int i = base + k * kRouteThreads + tid;
      if (i < total) {
        sm[i] = v[k];
        if (i < H && blockIdx.x == 0 && !is_finite_f(v[k])) bad_input = true;
      }
    }
  }
  __syncthreads();
  if (bad_input) set_status(a.status, kStatusNonFinite);
  if (tid >= 8 * kSmallTE) return;
  const int lane = tid & 7, el = tid >> 3, e = e0 + el;
  const float *w = ws + (size_t)el * H;
  const int full = H / 8;
  float logit;
  if (a.router_dtype == kRouterF32Seq) {
    // src/router.rs:59-62: one sequential chain (from -0.0, Rust's f32 Sum)
    float acc = -0.0f;
    if (lane == 0)
      for (int c = 0; c < H; ++c) acc = __fadd_rn(acc, __fmul_rn(w[c], hs[c]));
    logit = acc;
  } else {
    float acc = 0.0f;  // `[0.0f32; 8]`, src/backend.rs:107
#pragma unroll 8
    for (int c = 0; c < full; ++c)
      acc = __fadd_rn(acc, __fmul_rn(w[8 * c + lane], hs[8 * c + lane]));
    float s = -0.0f;
    const int base = (tid & 31) & ~7;
#pragma unroll
    for (int l = 0; l < 8; ++l) s = __fadd_rn(s, __shfl_sync(0xffffffffu, acc, base + l));
    for (int i = full * 8; i < H; ++i) s = __fadd_rn(s, __fmul_rn(w[i], hs[i]));
    logit = s;
  }
  if (lane == 0 && e < a.E) {
    a.logits[(size_t)t * a.E + e] = logit;
    if (!is_finite_f(logit)) set_status(a.status, kStatusNonFinite);
  }
}

// Register-tiled logits for larger T.  A CTA covers kTT (32 or 16) tokens x
// 16 experts; thread (lane l, token group, expert group) owns lane l of the
// 8-lane chain of (kTT / 8) x 4 (token, expert) pairs, so each shared-memory
// load feeds several multiply-adds and every chain still runs in chunk order.
// The 16-token tile doubles the grid when 32-token tiles would leave SMs idle.
constexpr int kTE = 16, kCW = 128;  // experts, columns per pass
constexpr int kHStride = kCW + 2;   // padding: conflict-free token rows
template <int kTT>
__global__ void __launch_bounds__(256) route_logits_tiled_kernel(RouteArgs a) {
  constexpr int kTG = kTT / 8;      // tokens per thread
  __shared__ float hs[kTT][kHStride];
  __shared__ float ws[kTE][kCW];
  const int tid = threadIdx.x;
  const int l = tid & 7, st = tid >> 3;
  const int tg = st & 7, eg = st >> 3;  // 8 token groups x 4 expert groups
  const int t0 = blockIdx.y * kTT, e0 = blockIdx.x * kTE;
  const int H = a.H, full = H / 8;
  float acc[kTG][4];
#pragma unroll
  for (int i = 0; i < kTG; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
  bool bad_input = false;
  // Software pipeline: the loads of pass p+1 go out into registers before
  // pass p is computed, and are stored to shared memory after it.
  constexpr int kHPer = kTT * kCW / 256, kWPer = kTE * kCW / 256;
  float hreg[kHPer], wreg[kWPer];
  auto fetch = [&](int c0) {
    const int ncol = min(kCW, full * 8 - c0);
#pragma unroll
    for (int k = 0; k < kHPer; ++k) {
      const int i = k * 256 + tid, r = i / kCW, c = i % kCW;
      hreg[k] = (t0 + r < a.T && c < ncol) ? a.h[(size_t)(t0 + r) * H + c0 + c] : 0.0f;
    }
#pragma unroll
    for (int k = 0; k < kWPer; ++k) {
      const int i = k * 256 + tid, r = i / kCW, c = i % kCW;
      wreg[k] = (e0 + r < a.E && c < ncol)
                    ? load_w(a.router, a.router_dtype, (size_t)(e0 + r) * H + c0 + c)
                    : 0.0f;
    }
  };
  if (full > 0) fetch(0);
  for (int c0 = 0; c0 < full * 8; c0 += kCW) {
    const int ncol = min(kCW, full * 8 - c0);
#pragma unroll
    for (int k = 0; k < kHPer; ++k) {
      const int i = k * 256 + tid;
      hs[i / kCW][i % kCW] = hreg[k];
      if (blockIdx.x == 0 && !is_finite_f(hreg[k])) bad_input = true;
    }
#pragma unroll
    for (int k = 0; k < kWPer; ++k) {
      const int i = k * 256 + tid;
      ws[i / kCW][i % kCW] = wreg[k];
    }
    __syncthreads();
    if (c0 + kCW < full * 8) fetch(c0 + kCW);
    const int nchunk = ncol / 8;
#pragma unroll 4
    for (int c = 0; c < nchunk; ++c) {
      float hv[kTG], wv[4];
#pragma unroll
      for (int i = 0; i < kTG; ++i) hv[i] = hs[kTG * tg + i][8 * c + l];
#pragma unroll
      for (int j = 0; j < 4; ++j) wv[j] = ws[4 * eg + j][8 * c + l];
#pragma unroll
      for (int i = 0; i < kTG; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(wv[j], hv[i]));
    }
    __syncthreads();
  }
  // tail columns (H % 8) are folded below; the finite check must see them too
  if (blockIdx.x == 0)
    for (int i = tid; i < kTT * (H - full * 8); i += 256) {
      const int r = i / (H - full * 8), c = full * 8 + i % (H - full * 8);
      if (t0 + r < a.T && !is_finite_f(a.h[(size_t)(t0 + r) * H + c])) bad_input = true;
    }
  if (bad_input) set_status(a.status, kStatusNonFinite);
  const int base = (tid & 31) & ~7;
#pragma unroll
  for (int i = 0; i < kTG; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float s = -0.0f;
#pragma unroll
      for (int k = 0; k < 8; ++k) s = __fadd_rn(s, __shfl_sync(0xffffffffu, acc[i][j], base + k));
      const int t = t0 + kTG * tg + i, e = e0 + 4 * eg + j;
      if (l == 0 && t < a.T && e < a.E) {
        for (int c = full * 8; c < H; ++c)
          s = __fadd_rn(s, __fmul_rn(load_w(a.router, a.router_dtype, (size_t)e * H + c),
                                     a.h[(size_t)t * H + c]));
        a.logits[(size_t)t * a.E + e] = s;
        if (!is_finite_f(s)) set_status(a.status, kStatusNonFinite);
      }
    }
}

// Pipelined, register-blocked logits for f32 routers (H % 4 == 0, 16-byte
// aligned rows).  A thread owns lane l of the 8-lane chain of a PT x PE block
// of (token, expert) pairs, so each shared-memory word it loads feeds PE (or
// PT) multiply-adds: at PT = PE = 8 the shared-memory traffic per
// multiply-add is half that of a 4 x 4 block, and the FP32 pipe, not shared
// memory, bounds the kernel.  The 32 groups of 8 threads form 8 token groups
// x 4 expert groups; token (i, tg) is row 8 i + tg of the tile and expert
// (j, ge) is row 4 j + ge, so the four groups of a warp read four adjacent
// token rows (row stride = 8 words mod 32: no bank conflicts) and one shared
// expert row (a broadcast).  Columns arrive in 64-wide stages through a
// kStages-deep cp.async ring; columns past the last full chunk of 8 are zero
// filled (0 * 0 added to a lane sum that cannot be -0.0 leaves it unchanged)
// and folded after the chains, in the reference order.
//
// Non-finite input needs no separate scan: a non-finite h[t][c] makes the
// product in its lane chain, and so the logit of every expert for token t,
// non-finite, and the logit check below records it.
template <int PT, int PE, int CW, int S, int NT>
struct PipeTile {
  static constexpr int GE = NT / 64;  // expert groups (8 token groups)
  static constexpr int TT = 8 * PT, TE = GE * PE;
  static constexpr int kStride = CW + 8;  // words per smem row (= 8 mod 32)
  static constexpr int kStageWords = (TT + TE) * kStride;
  static constexpr int kRedWords = TT * TE * 9;
  static constexpr size_t kSmem =
      sizeof(float) * (size_t)(kStageWords * S > kRedWords ? kStageWords * S : kRedWords);
};

__device__ __forceinline__ void cp_async16_zfill(uint32_t dst, const float *src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src),
               "r"(valid ? 16 : 0)
               : "memory");
}

// CW columns per stage, an S-deep ring, NT threads: small blocks (little
// compute per stage) take wider stages, a deeper ring and 128-thread CTAs so
// that the copies in flight cover the memory latency and the grid covers
// every SM.  Each thread's copy rows and column are fixed for the whole
// kernel (row rb + k * (NT / (CW / 4)), column 4 * qc of every stage), so a
// copy costs a pointer add and a predicate.
//
// PK: the products of expert pairs (j, j + 1) come from one packed
// `mul.rn.f32x2` (per component the IEEE product, exactly __fmul_rn's), and
// each chain adds its product with a scalar __fadd_rn, which is never fused.
// A packed add as well was measured on B200 to change the logits' low bits
// (the multiply and add of a pair end up contracted), so it is not used.

__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float &lo, float &hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_mul_rn(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

template <int PT, int PE, int CW, int S, int NT, bool PK>
__global__ void __launch_bounds__(NT, PT * PE >= 64 ? 2 : 4)
    route_logits_pipe_kernel(RouteArgs a) {
  using Tile = PipeTile<PT, PE, CW, S, NT>;
  constexpr int TT = Tile::TT, TE = Tile::TE, kStride = Tile::kStride;
  constexpr int kQuads = CW / 4;               // 16-byte copies per row and stage
  constexpr int kRowsPer = NT / kQuads;        // rows one pass of the CTA covers
  constexpr int kNK = (TT + TE + kRowsPer - 1) / kRowsPer;
  static_assert(NT % kQuads == 0, "copy layout");
  extern __shared__ __align__(16) float psm[];
  const int tid = threadIdx.x;
  const int l = tid & 7, grp = tid >> 3;
  const int tg = grp & 7, ge = grp >> 3;
  const int t0 = blockIdx.y * TT, e0 = blockIdx.x * TE;
  const int H = a.H, full = H / 8, ncols = full * 8;
  const float *W = static_cast<const float *>(a.router);
  const int nstage = (ncols + CW - 1) / CW;

  const int rb = tid / kQuads, qc = tid % kQuads;
  const float *src[kNK];
  uint32_t rowok = 0;
#pragma unroll
  for (int k = 0; k < kNK; ++k) {
    const int r = rb + k * kRowsPer;
    bool ok;
    if (r < TT) {
      ok = t0 + r < a.T;
      src[k] = a.h + (size_t)(ok ? t0 + r : 0) * H + 4 * qc;
    } else {
      ok = r < TT + TE && e0 + r - TT < a.E;
      src[k] = W + (size_t)(ok ? e0 + r - TT : 0) * H + 4 * qc;
    }
    rowok |= (ok ? 1u : 0u) << k;
  }
  const uint32_t dst0 = (uint32_t)__cvta_generic_to_shared(psm) + 4u * (rb * kStride + 4 * qc);

  auto issue = [&](int st) {
    const uint32_t dst = dst0 + 4u * (st % S) * Tile::kStageWords;
    const int c0 = st * CW;
    const bool colok = c0 + 4 * qc < ncols;
#pragma unroll
    for (int k = 0; k < kNK; ++k) {
      if (kNK * kRowsPer > TT + TE && rb + k * kRowsPer >= TT + TE) break;
      const bool ok = colok && ((rowok >> k) & 1u);
      cp_async16_zfill(dst + 4u * k * kRowsPer * kStride, ok ? src[k] + c0 : src[k], ok);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };

  float acc[PT][PE];
#pragma unroll
  for (int i = 0; i < PT; ++i)
#pragma unroll
    for (int j = 0; j < PE; ++j) acc[i][j] = 0.0f;  // `[0.0f32; 8]`, src/backend.rs:107

#pragma unroll
  for (int st = 0; st < S - 1; ++st) {
    if (st < nstage) issue(st);
    else asm volatile("cp.async.commit_group;" ::: "memory");
  }
  for (int st = 0; st < nstage; ++st) {
    asm volatile("cp.async.wait_group %0;" ::"n"(S - 2) : "memory");
    __syncthreads();  // stage st visible; stage st - 1 fully consumed
    if (st + S - 1 < nstage) issue(st + S - 1);
    else asm volatile("cp.async.commit_group;" ::: "memory");
    const float *hs = psm + (st % S) * Tile::kStageWords + tg * kStride + l;
    const float *ws = psm + (st % S) * Tile::kStageWords + (TT + ge) * kStride + l;
#pragma unroll
    for (int c = 0; c < CW / 8; ++c) {
      float hv[PT], wv[PE];
#pragma unroll
      for (int i = 0; i < PT; ++i) hv[i] = hs[8 * i * kStride + 8 * c];
#pragma unroll
      for (int j = 0; j < PE; ++j) wv[j] = ws[Tile::GE * j * kStride + 8 * c];
      if constexpr (PK) {
        static_assert(PE % 2 == 0, "expert pairs");
        uint64_t w2[PE / 2];
#pragma unroll
        for (int jj = 0; jj < PE / 2; ++jj) w2[jj] = f2_pack(wv[2 * jj], wv[2 * jj + 1]);
#pragma unroll
        for (int i = 0; i < PT; ++i) {
          const uint64_t h2 = f2_pack(hv[i], hv[i]);
#pragma unroll
          for (int jj = 0; jj < PE / 2; ++jj) {
            float p0, p1;
            f2_unpack(f2_mul_rn(w2[jj], h2), p0, p1);
            acc[i][2 * jj] = __fadd_rn(acc[i][2 * jj], p0);
            acc[i][2 * jj + 1] = __fadd_rn(acc[i][2 * jj + 1], p1);
          }
        }
      } else {
#pragma unroll
        for (int i = 0; i < PT; ++i)
#pragma unroll
          for (int j = 0; j < PE; ++j)
            acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(wv[j], hv[i]));
      }
    }
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  __syncthreads();
  // lane sums to shared memory, then each thread folds whole pairs
  float *red = psm;
#pragma unroll
  for (int i = 0; i < PT; ++i)
#pragma unroll
    for (int j = 0; j < PE; ++j)
      red[((8 * i + tg) * TE + Tile::GE * j + ge) * 9 + l] = acc[i][j];
  __syncthreads();
  for (int p = tid; p < TT * TE; p += NT) {
    const int t = t0 + p / TE, e = e0 + p % TE;
    if (t >= a.T || e >= a.E) continue;
    float s = -0.0f;
#pragma unroll
    for (int k = 0; k < 8; ++k) s = __fadd_rn(s, red[p * 9 + k]);
    for (int c = ncols; c < H; ++c)
      s = __fadd_rn(s, __fmul_rn(W[(size_t)e * H + c], a.h[(size_t)t * H + c]));
    a.logits[(size_t)t * a.E + e] = s;
    if (!is_finite_f(s)) set_status(a.status, kStatusNonFinite);
  }
}

// MOE_ROUTE_F32X2=0 runs the pipelined logits with scalar multiplies.
bool route_packed() {
  static int v = -1;
  if (v < 0) {
    const char *env = getenv("MOE_ROUTE_F32X2");
    v = env && atoi(env) == 0 ? 0 : 1;
  }
  return v == 1;
}

// MOE_ROUTE_TILE=24|44 pins the block (PT, PE) for measurements; 1 selects
// the 4 x 4 scalar-staged kernel.
int route_tile_override() {
  static int v = -1;
  if (v < 0) {
    const char *env = getenv("MOE_ROUTE_TILE");
    v = env ? atoi(env) : 0;
    if (v != 1 && v != 24 && v != 44) v = 0;
  }
  return v;
}

template <int PT, int PE, int NT>
int pipe_ctas(const RouteArgs &a) {
  constexpr int TE = NT / 64 * PE, TT = 8 * PT;
  return ((a.E + TE - 1) / TE) * ((a.T + TT - 1) / TT);
}

template <int PT, int PE, int CW, int S, int NT, bool PK>
cudaError_t launch_pipe(const RouteArgs &a, cudaStream_t s) {
  using Tile = PipeTile<PT, PE, CW, S, NT>;
  constexpr size_t smem = Tile::kSmem;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(route_logits_pipe_kernel<PT, PE, CW, S, NT, PK>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  dim3 grid((a.E + Tile::TE - 1) / Tile::TE, (a.T + Tile::TT - 1) / Tile::TT);
  route_logits_pipe_kernel<PT, PE, CW, S, NT, PK><<<grid, NT, smem, s>>>(a);
  return cudaGetLastError();
}

// One warp per token (the selection itself is route_core.cuh select_token).
__global__ void __launch_bounds__(256) route_select_kernel(RouteArgs a) {
  __shared__ SelectScratch scratch[8];
  const int warp = threadIdx.x >> 5;
  const int t = blockIdx.x * 8 + warp;
  if (t >= a.T) return;
  select_token(a.logits + (size_t)t * a.E, a.E, a.K, a.norm_topk_prob, a.mode,
               a.ids + (size_t)t * a.K, a.gates + (size_t)t * a.K,
               a.probs ? a.probs + (size_t)t * a.E : nullptr, scratch[warp], a.status);
}

// Single-CTA stable counting sort of the T*K routes by expert.
// ---------------------------------------------------------------------------
// Permutation: a stable counting sort of the routes by expert.
// ---------------------------------------------------------------------------

// Exclusive prefix over threads 0..255 of the block of v (threads >= 256 take
// part and get meaningless results); `total` = sum over threads 0..255.
// wsum: 8 words of shared memory.  Contains two block barriers.
__device__ __forceinline__ int block_scan256(int v, int *wsum, int &total) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31 && w < 8) wsum[w] = x;
  __syncthreads();
  int pre = 0;
  total = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int t = wsum[i];
    if (i < w) pre += t;
    total += t;
  }
  __syncthreads();
  return pre + x - v;
}

// Expert segments, the active list and (optionally) the tile list from the
// per-expert counts; called by every thread of the block, thread e < 256
// holding cnt of expert e (0 past E).  Returns the segment start of expert
// tid.  Contains block barriers.
__device__ __forceinline__ int segments_and_tiles(const PermuteArgs &a, int cnt, int *wsum) {
  const int e = threadIdx.x, E = a.E;
  const bool mine = e < E && e < kMaxExperts;
  int total;
  const int seg = block_scan256(mine ? cnt : 0, wsum, total);
  int nact;
  const int apos = block_scan256(mine && cnt > 0 ? 1 : 0, wsum, nact);
  if (mine) {
    a.seg_off[e] = seg;
    if (cnt > 0) a.active[apos] = e;
  }
  if (e == 0) {
    a.seg_off[E] = total;
    *a.n_active = nact;
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const PermuteArgs::TileList &L = a.tiles[i];
    if (L.bn <= 0) continue;  // block-uniform
    const int nt = mine ? (cnt + L.bn - 1) / L.bn : 0;
    int ntot;
    const int first = block_scan256(nt, wsum, ntot);
    for (int k = 0; k < nt && first + k < L.max_tiles; ++k) {
      L.expert[first + k] = e;
      L.row0[first + k] = seg + k * L.bn;
      L.rows[first + k] = min(L.bn, cnt - k * L.bn);
    }
    if (e == 0) *L.count = min(ntot, L.max_tiles);
  }
  return seg;
}

// One CTA sorts up to kPermSingleMax routes (and any count when no scratch
// for the multi-CTA sort is given).  Routes go in tiles of 1024 in route
// order; inside a tile a route's rank comes from its warp's match mask plus a
// scan over the warps' counts for its expert (one warp scans one expert's 32
// warp counts with shuffles), on top of the expert's running offset.  The
// ids and gates of the first kPermPer tiles are loaded up front, so those
// tiles wait on no global load.
constexpr int kPermThreads = 1024;
constexpr int kPermPer = 8;
constexpr int kPermSingleMax = 2048;  // above: the three-kernel sort is faster (measured)
__global__ void __launch_bounds__(kPermThreads, 1) permute_kernel(PermuteArgs a) {
  __shared__ int32_t cnt[kMaxExperts];
  __shared__ int32_t run[kMaxExperts];
  __shared__ int32_t wcnt[kPermThreads / 32][kMaxExperts];
  __shared__ int32_t wsum[8];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int E = a.E, R = a.T * a.K;
  uint32_t eid[kPermPer];
  float gv[kPermPer];
#pragma unroll
  for (int k = 0; k < kPermPer; ++k) {
    const int r = k * kPermThreads + tid;
    eid[k] = r < R ? a.ids[r] : 0xFFFFFFFFu;
    gv[k] = (r < R && a.r_gate) ? a.gates[r] : 0.0f;
  }
  if (tid < kMaxExperts) cnt[tid] = 0;
  for (int i = tid; i < (kPermThreads / 32) * kMaxExperts; i += kPermThreads)
    (&wcnt[0][0])[i] = 0;
  __syncthreads();
#pragma unroll
  for (int k = 0; k < kPermPer; ++k)
    if (k * kPermThreads + tid < R) {
      if (eid[k] < (uint32_t)E) atomicAdd(&cnt[eid[k]], 1);
      else set_status(a.status, kStatusBadRoute);
    }
  for (int r = kPermPer * kPermThreads + tid; r < R; r += kPermThreads) {
    const uint32_t e = a.ids[r];
    if (e < (uint32_t)E) atomicAdd(&cnt[e], 1);
    else set_status(a.status, kStatusBadRoute);
  }
  __syncthreads();
  const int seg = segments_and_tiles(a, tid < kMaxExperts ? cnt[tid] : 0, wsum);
  if (tid < E) run[tid] = seg;
  __syncthreads();
  // one tile of 1024 routes (block-uniform call)
  auto tile = [&](int r, uint32_t e, float gate) {
    const bool valid = r < R;
    const bool ok = valid && e < (uint32_t)E;
    const unsigned mask = __match_any_sync(0xffffffffu, ok ? e : 0xFFFFFFFFu);
    const int intra = __popc(mask & ((1u << lane) - 1u));
    if (ok && intra == 0) wcnt[warp][e] = __popc(mask);
    __syncthreads();
    // wcnt[w][e] := position of warp w's first route to e; run[e] advances
    for (int ee = warp; ee < E; ee += kPermThreads / 32) {
      const int v = wcnt[lane][ee];
      int x = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
      }
      const int r0 = run[ee];
      wcnt[lane][ee] = r0 + x - v;
      __syncwarp();
      if (lane == 31) run[ee] = r0 + x;
    }
    __syncthreads();
    if (ok) {
      const int pos = wcnt[warp][e] + intra;
      a.r_token[pos] = r / a.K;
      a.r_slot[pos] = r % a.K;
      if (a.r_gate) a.r_gate[pos] = gate;
      if (a.r_pos) a.r_pos[r] = pos;
    } else if (valid && a.r_pos) {
      a.r_pos[r] = -1;  // an invalid expert id holds no sorted row
    }
    __syncthreads();
    for (int i = tid; i < (kPermThreads / 32) * E; i += kPermThreads) wcnt[i / E][i % E] = 0;
    __syncthreads();
  };
#pragma unroll
  for (int k = 0; k < kPermPer; ++k)
    if (k * kPermThreads < R) tile(k * kPermThreads + tid, eid[k], gv[k]);
  for (int base = kPermPer * kPermThreads; base < R; base += kPermThreads) {
    const int r = base + tid;
    const uint32_t e = r < R ? a.ids[r] : 0xFFFFFFFFu;
    tile(r, e, (r < R && a.r_gate) ? a.gates[r] : 0.0f);
  }
}

// Multi-CTA stable counting sort for large route counts: (1) per tile of
// 1024 routes, the per-expert counts and each route's rank inside its tile
// (warp match mask + earlier warps' counts); (2) one CTA turns the tile
// counts into per-tile offsets, the expert segments and the tile list; (3)
// every route is scattered to seg_off[e] + tile offset + rank in tile.  Same
// order as the single-CTA kernel: experts ascending, routes (tokens)
// ascending inside.
constexpr int kPermTile = 1024;

__global__ void __launch_bounds__(kPermTile) perm_hist_kernel(PermuteArgs a, int32_t *tilecnt,
                                                              int32_t *intra) {
  __shared__ int32_t wcnt[kPermTile / 32][kMaxExperts];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int E = a.E, R = a.T * a.K;
  for (int i = tid; i < (kPermTile / 32) * kMaxExperts; i += kPermTile) (&wcnt[0][0])[i] = 0;
  __syncthreads();
  const int r = blockIdx.x * kPermTile + tid;
  const bool valid = r < R;
  const uint32_t e = valid ? a.ids[r] : 0xFFFFFFFFu;
  const bool ok = valid && e < (uint32_t)E;
  if (valid && !ok) set_status(a.status, kStatusBadRoute);
  const unsigned mask = __match_any_sync(0xffffffffu, ok ? e : 0xFFFFFFFFu);
  const int in_warp = __popc(mask & ((1u << lane) - 1u));
  if (ok && in_warp == 0) wcnt[warp][e] = __popc(mask);
  __syncthreads();
  if (ok) {
    int rank = in_warp;
    for (int w = 0; w < warp; ++w) rank += wcnt[w][e];
    intra[r] = rank;
  }
  for (int ee = tid; ee < E; ee += kPermTile) {
    int tot = 0;
    for (int w = 0; w < kPermTile / 32; ++w) tot += wcnt[w][ee];
    tilecnt[(size_t)blockIdx.x * E + ee] = tot;
  }
}

__global__ void __launch_bounds__(kMaxExperts) perm_scan_kernel(PermuteArgs a, int32_t *tilecnt,
                                                                int ntiles) {
  __shared__ int32_t wsum[8];
  const int e = threadIdx.x, E = a.E;
  // running offsets of expert e over the tiles, loads batched 8 at a time
  int run = 0;
  if (e < E)
    for (int t0 = 0; t0 < ntiles; t0 += 8) {
      int c[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) c[k] = t0 + k < ntiles ? tilecnt[(size_t)(t0 + k) * E + e] : 0;
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if (t0 + k < ntiles) {
          tilecnt[(size_t)(t0 + k) * E + e] = run;
          run += c[k];
        }
    }
  segments_and_tiles(a, run, wsum);
}

__global__ void perm_scatter_kernel(PermuteArgs a, const int32_t *tilecnt,
                                    const int32_t *intra) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  const int R = a.T * a.K;
  if (r >= R) return;
  const uint32_t e = a.ids[r];
  if (e >= (uint32_t)a.E) {
    if (a.r_pos) a.r_pos[r] = -1;  // an invalid expert id holds no sorted row
    return;
  }
  const int pos = a.seg_off[e] + tilecnt[(size_t)(r / kPermTile) * a.E + e] + intra[r];
  a.r_token[pos] = r / a.K;
  a.r_slot[pos] = r % a.K;
  if (a.r_gate) a.r_gate[pos] = a.gates[r];
  if (a.r_pos) a.r_pos[r] = pos;
}

}  // namespace

size_t permute_scratch_words(int R, int E) {
  return (size_t)((R + kPermTile - 1) / kPermTile) * E + (size_t)R;
}

cudaError_t launch_route(const RouteArgs &a, cudaStream_t s, int *launches) {
  if (launches) *launches = 0;
  if (a.T <= 0) return cudaSuccess;
  const size_t small_smem = sizeof(float) * (size_t)(1 + kSmallTE) * a.H;
  const bool aligned16 =
      ((reinterpret_cast<uintptr_t>(a.h) | reinterpret_cast<uintptr_t>(a.router)) & 15) == 0;
  if (a.T >= 16 && a.router_dtype == kRouterF32 && a.H % 4 == 0 && aligned16 &&
      route_tile_override() != 1) {
    // the largest block that still gives about 1.7 CTAs per SM
    // 4 x 4 blocks while they still give about one CTA per SM, else 2 x 4
    const int pin = route_tile_override();
    cudaError_t e;
    const bool wide = pin == 44 || (pin != 24 && pipe_ctas<4, 4, 256>(a) >= 128);
    if (route_packed())
      e = wide ? launch_pipe<4, 4, 64, 4, 256, true>(a, s)
               : launch_pipe<2, 4, 128, 4, 256, true>(a, s);
    else
      e = wide ? launch_pipe<4, 4, 64, 4, 256, false>(a, s)
               : launch_pipe<2, 4, 128, 4, 256, false>(a, s);
    if (e != cudaSuccess) return e;
  } else if (a.T >= 16 && a.router_dtype != kRouterF32Seq) {
    const int ne = (a.E + kTE - 1) / kTE;
    if ((long long)ne * ((a.T + 31) / 32) >= 2 * 148) {
      route_logits_tiled_kernel<32><<<dim3(ne, (a.T + 31) / 32), 256, 0, s>>>(a);
    } else {
      route_logits_tiled_kernel<16><<<dim3(ne, (a.T + 15) / 16), 256, 0, s>>>(a);
    }
  } else {
    if (small_smem > 48 * 1024)
      cudaFuncSetAttribute(route_logits_small_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)small_smem);
    dim3 grid((a.E + kSmallTE - 1) / kSmallTE, a.T);
    route_logits_small_kernel<<<grid, kRouteThreads, small_smem, s>>>(a);
  }
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return err;
  route_select_kernel<<<(a.T + 7) / 8, 256, 0, s>>>(a);
  if (launches) *launches = 2;
  return cudaGetLastError();
}

// MOE_PERM_SINGLE_MAX overrides the route count up to which one CTA sorts.
int perm_single_max() {
  static int v = -1;
  if (v < 0) {
    const char *env = getenv("MOE_PERM_SINGLE_MAX");
    v = env ? atoi(env) : kPermSingleMax;
    if (v < 0) v = kPermSingleMax;
  }
  return v;
}

int permute_launches(const PermuteArgs &a) {
  const int R = a.T * a.K;
  return (R <= perm_single_max() || !a.scratch ||
          a.scratch_words < permute_scratch_words(R, a.E))
             ? 1
             : 3;
}

cudaError_t launch_permute(const PermuteArgs &a, cudaStream_t s) {
  const int R = a.T * a.K;
  if (R <= perm_single_max() || !a.scratch ||
      a.scratch_words < permute_scratch_words(R, a.E)) {
    permute_kernel<<<1, kPermThreads, 0, s>>>(a);
    return cudaGetLastError();
  }
  const int ntiles = (R + kPermTile - 1) / kPermTile;
  int32_t *tilecnt = a.scratch, *intra = a.scratch + (size_t)ntiles * a.E;
  perm_hist_kernel<<<ntiles, kPermTile, 0, s>>>(a, tilecnt, intra);
  perm_scan_kernel<<<1, kMaxExperts, 0, s>>>(a, tilecnt, ntiles);
  perm_scatter_kernel<<<(R + 255) / 256, 256, 0, s>>>(a, tilecnt, intra);
  return cudaGetLastError();
}

}  // namespace moe
