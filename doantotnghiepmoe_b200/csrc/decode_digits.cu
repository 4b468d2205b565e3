// Digit decode: one cooperative, persistent launch runs a whole MoE layer --
// or a stack of layers with RMSNorm and residual between them -- for decode
// batches, on the tolerance path.
//
// Routing is the reference's arithmetic bit for bit (the 8-lane router dot,
// softmax with libm's expf, top-k with ties to the lower index;
// src/backend.rs:105-120, :375-389, src/olmoe.rs:2589-2621), and so is the
// RMSNorm between stacked layers (src/backend.rs:341-359).  The experts use
// the two-digit int8 activations of digits.cuh: each weight row is dotted with
// both digit planes in exact int32 (__dp4a over 16-byte weight loads) and the
// epilogue is the tensor-core path's, so a layer's outputs are bit-identical
// to MOE_PATH_TENSOR's and within the 1e-3 tolerance of the CPU reference.
// Compared with the exact FP32 FMA chains (decode_fused.cu) a weight costs
// about half an instruction instead of five, so the weight stream runs at
// memory speed.
//
// Phases of one layer (G = gridDim.x CTAs, all co-resident):
//   R  router logits over tasks of (<= 4 tokens x 4 experts, or 1 expert when
//      tasks are scarce); a stacked layer normalises its staged token rows
//      first; the task of expert group 0 also writes the tokens' digit planes;
//   -- grid barrier --
//   S  top-k: with T <= 8 every CTA selects every token itself (one warp per
//      token); otherwise each token is selected once somewhere in the grid
//      and a second barrier publishes the routing;
//   P  every CTA sorts the T*K routes by expert in shared memory;
//   G  gate/up: the (active expert, weight row) pairs are split evenly over
//      the CTAs; a warp streams a gate row and its up row (16-byte loads,
//      evict-first) and dots them with the digit planes of every route of the
//      expert; SwiGLU -> act (fp32).  Single-token launches prefetch the down
//      rows they will need into L2 meanwhile;
//   -- grid barrier --
//   D  T = 1: every CTA owns a block of output rows, digitises the K
//      activation rows itself, runs all K experts' rows and combines in slot
//      order in registers (no further barrier);
//      T > 1: the (active expert, output row) pairs are split evenly; each
//      CTA digitises the activation rows of its experts' routes and writes
//      gate * y; a barrier, then the slot-ordered combine.
//   -- grid barrier before the next stacked layer --
// Every barrier wait is bounded (FusedArgs-style wait_cycles); on expiry the
// CTA records kStatusTimeout and returns.
#include <algorithm>

#include "common.cuh"
#include "digits.cuh"
#include "kernels.h"
#include "route_core.cuh"

namespace moe {
namespace {

constexpr int kDT = 256;         // threads per CTA
constexpr int kDW = kDT / 32;    // warps per CTA
constexpr int kRTT = 4;          // router task: tokens
constexpr int kRTE = 4;          // router task: experts
constexpr int kGR = 16;          // routes whose digit planes are staged at once
constexpr int kMaxChunks = 4;    // 16-byte chunks per lane of a row (rows <= 2048 bytes)

struct DTables {
  int32_t seg_off[kMaxExperts + 1];
  int32_t active[kMaxExperts];
  int32_t run[kMaxExperts];
  int32_t n_active;
  int32_t r_token[kFusedMaxRoutes];
  int32_t r_slot[kFusedMaxRoutes];
  float r_gate[kFusedMaxRoutes];
  uint32_t ids[kFusedMaxRoutes];   // token-major routing of the current layer
  float gates[kFusedMaxRoutes];
  int32_t wcnt[kDW][kMaxExperts];
  float s1[kMaxTopK > kGR ? kMaxTopK : kGR];  // scales of the staged digit rows
  float s2[kMaxTopK > kGR ? kMaxTopK : kGR];
  float inv[kRTT];                            // RMSNorm factors of the staged tokens
};

constexpr size_t align128(size_t n) { return (n + 127) & ~size_t(127); }
constexpr size_t kSelOff = align128(sizeof(DTables));
constexpr size_t kStageOff = align128(kSelOff + kDW * sizeof(SelectScratch));

__device__ __forceinline__ bool grid_sync(uint32_t *bar, uint32_t target, uint32_t *status,
                                          long long limit) {
  __shared__ int ok;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(bar, 1u);
    const long long t0 = clock64();
    int good = 1;
    while (*(volatile uint32_t *)bar < target) {
      if (clock64() - t0 > limit) {
        good = 0;
        set_status(status, kStatusTimeout);
        break;
      }
      __nanosleep(32);
    }
    __threadfence();
    ok = good;
  }
  __syncthreads();
  return ok != 0;
}

__device__ __forceinline__ void stamp(const DigitArgs &a, int idx) {
  if (a.phase_ts && blockIdx.x == 0 && threadIdx.x == 0) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    a.phase_ts[idx] = t;
  }
}

// 16 weight bytes, read once: no L1 allocation, evict-first in L2.
__device__ __forceinline__ uint4 ldg_stream16(const int8_t *p) {
  uint64_t pol;
  asm("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0, %1, %2, %3}, [%4], %5;"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p), "l"(pol));
  return v;
}

__device__ __forceinline__ void prefetch_l2(const void *p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

__device__ __forceinline__ void dp4(const uint4 w, const uint4 x, int &acc) {
  acc = __dp4a((int)w.x, (int)x.x, acc);
  acc = __dp4a((int)w.y, (int)x.y, acc);
  acc = __dp4a((int)w.z, (int)x.z, acc);
  acc = __dp4a((int)w.w, (int)x.w, acc);
}

__device__ __forceinline__ int warp_sum(int v) {
  return (int)__reduce_add_sync(0xffffffffu, (unsigned)v);
}

// ---------------------------------------------------------------------------
// R: router logits (exact order) + the token rows' digit planes.
// ---------------------------------------------------------------------------
__device__ void router_phase(const DigitArgs &a, const FusedLayer &L, const float *xin,
                             bool stacked, float *stage, DTables &tb) {
  const int T = a.T, E = a.E, H = a.H, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int TT = min(T, kRTT);
  const int ntt = (T + TT - 1) / TT;
  const int RE = ntt * ((E + kRTE - 1) / kRTE) * 2 < (int)gridDim.x ? 1 : kRTE;
  const int nte = (E + RE - 1) / RE;
  const int tasks = ntt * nte;
  const int full = H / 8;
  const bool seq = a.route_mode == kRouteTopkSoftmax && L.router_dtype == kRouterF32;
  for (int task = blockIdx.x; task < tasks; task += gridDim.x) {
    const int t0 = (task / nte) * TT, e0 = (task % nte) * RE;
    const int nt = min(TT, T - t0);
    bool bad = false;
    // stage rows [0, TT) tokens, [TT, TT + RE) router rows
    if (a.router_async) {
      const int q = H / 4;
      for (int i = tid; i < (TT + RE) * q; i += kDT) {
        const int r = i / q, c = (i % q) * 4;
        float *dst = stage + (size_t)r * H + c;
        const float *src = nullptr;
        if (r < TT) {
          if (r < nt) src = xin + (size_t)(t0 + r) * H + c;
        } else if (e0 + r - TT < E) {
          src = reinterpret_cast<const float *>(L.router) + (size_t)(e0 + r - TT) * H + c;
        }
        if (src) {
          asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                           (uint32_t)__cvta_generic_to_shared(dst)),
                       "l"(src)
                       : "memory");
        } else {
          *reinterpret_cast<float4 *>(dst) = make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
      asm volatile("cp.async.wait_all;" ::: "memory");
    } else {
      for (int i = tid; i < (TT + RE) * H; i += kDT) {
        const int r = i / H, c = i % H;
        float v = 0.0f;
        if (r < TT) {
          if (r < nt) v = __ldcg(xin + (size_t)(t0 + r) * H + c);
        } else if (e0 + r - TT < E) {
          v = load_w(L.router, L.router_dtype, (size_t)(e0 + r - TT) * H + c);
        }
        stage[i] = v;
      }
    }
    __syncthreads();
    for (int i = tid; i < nt * H; i += kDT)
      if (!is_finite_f(stage[i])) bad = true;
    if (stacked) {
      // RMSNorm of each staged token row (src/backend.rs:341-359): lanes 0..7
      // of warp r run the 8-lane sum of squares, then every thread scales.
      if (warp < nt) {
        const float *x = stage + (size_t)warp * H;
        float acc = 0.0f;
        if (lane < 8)
          for (int c = 0; c < full; ++c) {
            const float v = x[8 * c + lane];
            acc = __fadd_rn(acc, __fmul_rn(v, v));
          }
        float s = -0.0f;
#pragma unroll
        for (int l = 0; l < 8; ++l) s = __fadd_rn(s, __shfl_sync(0xffffffffu, acc, l));
        for (int i = full * 8; i < H; ++i) s = __fadd_rn(s, __fmul_rn(x[i], x[i]));
        if (lane == 0) {
          const float scale = __fsqrt_rn(__fadd_rn(__fdiv_rn(s, (float)H), a.eps));
          tb.inv[warp] = __fdiv_rn(1.0f, scale);
        }
      }
      __syncthreads();
      for (int i = tid; i < nt * H; i += kDT) {
        const int r = i / H, j = i % H;
        const float o = __fmul_rn(__fmul_rn(stage[i], tb.inv[r]), L.norm_w ? L.norm_w[j] : 1.0f);
        if (!is_finite_f(o)) bad = true;
        stage[i] = o;
      }
      __syncthreads();
    }
    if (bad) set_status(a.status, kStatusNonFinite);
    // 8 lanes per (token, expert) pair, whole warps (the fold is a shuffle)
    const int npairs = TT * RE;
    if (tid < ((8 * npairs + 31) & ~31)) {
      const int l8 = tid & 7, pair = tid >> 3;
      const bool live = pair < npairs;
      const int ti = live ? pair / RE : 0, ei = live ? pair % RE : 0;
      const float *hs = stage + (size_t)ti * H;
      const float *w = stage + (size_t)(TT + ei) * H;
      float logit;
      if (seq) {
        float acc = -0.0f;  // src/router.rs:59-62, Rust's f32 Sum folds from -0.0
        if (l8 == 0)
          for (int c = 0; c < H; ++c) acc = __fadd_rn(acc, __fmul_rn(w[c], hs[c]));
        logit = acc;
      } else {
        float acc = 0.0f;  // `[0.0f32; 8]`, src/backend.rs:107
#pragma unroll 8
        for (int c = 0; c < full; ++c)
          acc = __fadd_rn(acc, __fmul_rn(w[8 * c + l8], hs[8 * c + l8]));
        float s = -0.0f;
        const int base = lane & ~7;
#pragma unroll
        for (int l = 0; l < 8; ++l) s = __fadd_rn(s, __shfl_sync(0xffffffffu, acc, base + l));
        for (int i = full * 8; i < H; ++i) s = __fadd_rn(s, __fmul_rn(w[i], hs[i]));
        logit = s;
      }
      const int t = t0 + ti, e = e0 + ei;
      if (live && l8 == 0 && ti < nt && e < E) {
        a.logits[(size_t)t * E + e] = logit;
        if (!is_finite_f(logit)) set_status(a.status, kStatusNonFinite);
      }
    }
    // the token rows' digit planes, once per token (expert group 0)
    if (e0 == 0 && warp < nt) {
      const float *x = stage + (size_t)warp * H;
      float amax = 0.0f;
      for (int c = lane * 4; c < H; c += 128) {
        const float4 v = *reinterpret_cast<const float4 *>(x + c);
        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      const float s = digits::row_scale(amax);
      const float inv = 1.0f / s;
      const int t = t0 + warp;
      int8_t *q1 = a.xq + (size_t)t * 2 * H, *q2 = q1 + H;
      for (int c = lane * 4; c < H; c += 128) {
        const float4 v = *reinterpret_cast<const float4 *>(x + c);
        uint32_t p2;
        const uint32_t p1 = digits::split4(v.x, v.y, v.z, v.w, inv, p2);
        *reinterpret_cast<uint32_t *>(q1 + c) = p1;
        *reinterpret_cast<uint32_t *>(q2 + c) = p2;
      }
      if (lane == 0) {
        a.xs1[t] = s;
        a.xs2[t] = s / 254.0f;
      }
    }
    __syncthreads();
  }
}

// P: stable counting sort of the R routes (tb.ids, token-major) by expert:
// experts ascending, routes ascending inside (src/olmoe.rs:3474-3480).
__device__ void build_tables(int R, int K, int E, DTables &tb) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (int e = tid; e < E; e += kDT) tb.run[e] = 0;
  for (int i = tid; i < kDW * kMaxExperts; i += kDT) (&tb.wcnt[0][0])[i] = 0;
  __syncthreads();
  for (int r = tid; r < R; r += kDT) {
    const uint32_t e = tb.ids[r];
    if (e < (uint32_t)E) atomicAdd(&tb.run[e], 1);
  }
  __syncthreads();
  if (warp == 0) {
    int acc = 0, na = 0;
    for (int base = 0; base < E; base += 32) {
      const int e = base + lane;
      const int c = e < E ? tb.run[e] : 0;
      int inc = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += v;
      }
      const unsigned act = __ballot_sync(0xffffffffu, c > 0);
      if (e < E) {
        tb.seg_off[e] = acc + inc - c;
        tb.run[e] = acc + inc - c;
        if (c > 0) tb.active[na + __popc(act & ((1u << lane) - 1u))] = e;
      }
      acc += __shfl_sync(0xffffffffu, inc, 31);
      na += __popc(act);
    }
    if (lane == 0) {
      tb.seg_off[E] = acc;
      tb.n_active = na;
    }
  }
  __syncthreads();
  for (int base = 0; base < R; base += kDT) {
    const int r = base + tid;
    const bool valid = r < R;
    const uint32_t e = valid ? tb.ids[r] : 0xFFFFFFFFu;
    const bool ok = valid && e < (uint32_t)E;
    const unsigned mask = __match_any_sync(0xffffffffu, ok ? e : 0xFFFFFFFFu);
    const int intra = __popc(mask & ((1u << lane) - 1u));
    if (ok && intra == 0) tb.wcnt[warp][e] = __popc(mask);
    __syncthreads();
    if (ok) {
      int pos = tb.run[e] + intra;
      for (int w = 0; w < warp; ++w) pos += tb.wcnt[w][e];
      tb.r_token[pos] = r / K;
      tb.r_slot[pos] = r % K;
      tb.r_gate[pos] = tb.gates[r];
    }
    __syncthreads();
    for (int ee = tid; ee < E; ee += kDT) {
      int tot = 0;
      for (int w = 0; w < kDW; ++w) {
        tot += tb.wcnt[w][ee];
        tb.wcnt[w][ee] = 0;
      }
      tb.run[ee] += tot;
    }
    __syncthreads();
  }
}

// The CTA's share [u0, u1) of n units.
__device__ __forceinline__ void share(long long n, long long &u0, long long &u1) {
  u0 = n * blockIdx.x / gridDim.x;
  u1 = n * (blockIdx.x + 1) / gridDim.x;
}

// Bulk L2 prefetch of the down rows this CTA reads in D (same partition).
__device__ void prefetch_down(const DigitArgs &a, const FusedLayer &L, const DTables &tb) {
  if (threadIdx.x != 0) return;
  const int H = a.H, I = a.I;
  long long u0, u1;
  if (a.T == 1) {
    share(H, u0, u1);
    if (u1 <= u0) return;
    for (int k = 0; k < a.K; ++k) {
      const uint32_t e = tb.ids[k];
      if (e >= (uint32_t)a.E) continue;
      prefetch_l2(L.w_ptr[e] + (size_t)2 * I * H + (size_t)u0 * I, (uint32_t)((u1 - u0) * I));
    }
    return;
  }
  share((long long)tb.n_active * H, u0, u1);
  for (long long u = u0; u < u1;) {
    const int ai = (int)(u / H), j0 = (int)(u - (long long)ai * H);
    const int j1 = (int)std::min<long long>(H, j0 + (u1 - u));
    prefetch_l2(L.w_ptr[tb.active[ai]] + (size_t)2 * I * H + (size_t)j0 * I,
                (uint32_t)((j1 - j0) * I));
    u += j1 - j0;
  }
}

// G: gate/up over the CTA's share of the (active expert, row) pairs.  A warp
// takes two row pairs at a time, so 4 * NCH 16-byte loads per lane are in
// flight before the first dot (NCH = 16-byte chunks per lane of an H row).
template <int NCH>
__device__ void gate_up_phase(const DigitArgs &a, const FusedLayer &L, uint8_t *xd, DTables &tb) {
  constexpr int kRows = 2;
  const int H = a.H, I = a.I, K = a.K, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  long long u0, u1;
  share((long long)tb.n_active * I, u0, u1);
  for (long long u = u0; u < u1;) {
    const int ai = (int)(u / I), i0 = (int)(u - (long long)ai * I);
    const int i1 = (int)std::min<long long>(I, i0 + (u1 - u));
    u += i1 - i0;
    const int e = tb.active[ai], r0 = tb.seg_off[e], r1 = tb.seg_off[e + 1];
    const int8_t *W = L.w_ptr[e];
    const float *S = L.s_ptr[e];
    for (int rb = r0; rb < r1; rb += kGR) {
      const int nr = min(kGR, r1 - rb);
      // the digit planes of routes rb .. rb + nr (2H bytes each) and scales
      __syncthreads();
      const int q16 = 2 * H / 16;
      for (int idx = tid; idx < nr * q16; idx += kDT) {
        const int j = idx / q16, o = idx - j * q16;
        const uint4 v = __ldcg(reinterpret_cast<const uint4 *>(
                                   a.xq + (size_t)tb.r_token[rb + j] * 2 * H) + o);
        reinterpret_cast<uint4 *>(xd + (size_t)j * 2 * H)[o] = v;
      }
      if (tid < nr) {
        tb.s1[tid] = __ldcg(a.xs1 + tb.r_token[rb + tid]);
        tb.s2[tid] = __ldcg(a.xs2 + tb.r_token[rb + tid]);
      }
      __syncthreads();
      for (int ib = i0 + warp * kRows; ib < i1; ib += kDW * kRows) {
        uint4 wg[kRows][NCH], wu[kRows][NCH];
#pragma unroll
        for (int q = 0; q < kRows; ++q)
#pragma unroll
          for (int m = 0; m < NCH; ++m) {
            const int off = 16 * (lane + 32 * m), i = ib + q;
            if (i < i1 && off < H) {
              wg[q][m] = ldg_stream16(W + (size_t)i * H + off);
              wu[q][m] = ldg_stream16(W + (size_t)(I + i) * H + off);
            } else {
              wg[q][m] = wu[q][m] = make_uint4(0, 0, 0, 0);
            }
          }
        int mg1[kRows] = {}, mg2[kRows] = {}, mu1[kRows] = {}, mu2[kRows] = {};  // route `lane`
        for (int j = 0; j < nr; ++j) {
          const uint8_t *x1 = xd + (size_t)j * 2 * H, *x2 = x1 + H;
          int g1[kRows] = {}, g2[kRows] = {}, v1[kRows] = {}, v2[kRows] = {};
#pragma unroll
          for (int m = 0; m < NCH; ++m) {
            const int off = 16 * (lane + 32 * m);
            if (off < H) {
              const uint4 d1 = *reinterpret_cast<const uint4 *>(x1 + off);
              const uint4 d2 = *reinterpret_cast<const uint4 *>(x2 + off);
#pragma unroll
              for (int q = 0; q < kRows; ++q) {
                dp4(wg[q][m], d1, g1[q]);
                dp4(wg[q][m], d2, g2[q]);
                dp4(wu[q][m], d1, v1[q]);
                dp4(wu[q][m], d2, v2[q]);
              }
            }
          }
#pragma unroll
          for (int q = 0; q < kRows; ++q) {
            g1[q] = warp_sum(g1[q]);
            g2[q] = warp_sum(g2[q]);
            v1[q] = warp_sum(v1[q]);
            v2[q] = warp_sum(v2[q]);
            if (lane == j) {
              mg1[q] = g1[q];
              mg2[q] = g2[q];
              mu1[q] = v1[q];
              mu2[q] = v2[q];
            }
          }
        }
        if (lane < nr) {
          const int r = rb + lane;
          float *act = a.act + ((size_t)tb.r_token[r] * K + tb.r_slot[r]) * I;
#pragma unroll
          for (int q = 0; q < kRows; ++q) {
            const int i = ib + q;
            if (i < i1)
              act[i] = digits::swiglu(mg1[q], mg2[q], mu1[q], mu2[q], tb.s1[lane], tb.s2[lane],
                                      S[i], S[I + i]);
          }
        }
      }
    }
  }
}

// Digit planes of activation rows (I floats each, read through L2) into xd,
// one warp per row; scales into tb.s1 / tb.s2.  rows[j] = act row index.
__device__ void digitise_act(const DigitArgs &a, const int32_t *act_row, int nr, uint8_t *xd,
                             DTables &tb) {
  const int I = a.I, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int j = warp; j < nr; j += kDW) {
    const float *x = a.act + (size_t)act_row[j] * I;
    float amax = 0.0f;
    for (int c = lane * 4; c < I; c += 128) {
      const float4 v = __ldcg(reinterpret_cast<const float4 *>(x + c));
      amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float s = digits::row_scale(amax);
    const float inv = 1.0f / s;
    uint8_t *q1 = xd + (size_t)j * 2 * I, *q2 = q1 + I;
    for (int c = lane * 4; c < I; c += 128) {
      const float4 v = __ldcg(reinterpret_cast<const float4 *>(x + c));
      uint32_t p2;
      const uint32_t p1 = digits::split4(v.x, v.y, v.z, v.w, inv, p2);
      *reinterpret_cast<uint32_t *>(q1 + c) = p1;
      *reinterpret_cast<uint32_t *>(q2 + c) = p2;
    }
    if (lane == 0) {
      tb.s1[j] = s;
      tb.s2[j] = s / 254.0f;
    }
  }
}

// D for one token: the CTA's block of output rows over all K routes, combined
// in slot order in registers: out = base + g_0 y_0 + ... + g_{K-1} y_{K-1}.
// The rows of up to 8 experts are loaded before the first dot.
template <int NCI>
__device__ void down_single(const DigitArgs &a, const FusedLayer &L, const float *resid,
                            float *out, uint8_t *xd, DTables &tb) {
  constexpr int kE = 8;
  const int H = a.H, I = a.I, K = a.K, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  long long u0, u1;
  share(H, u0, u1);
  __shared__ int32_t rows[kMaxTopK];
  if (threadIdx.x < K) rows[threadIdx.x] = threadIdx.x;  // act row of slot k (token 0)
  __syncthreads();
  digitise_act(a, rows, K, xd, tb);
  __syncthreads();
  bool bad = false;
  for (int j = (int)u0 + warp; j < (int)u1; j += kDW) {
    int my1 = 0, my2 = 0;  // sums of slot `lane`
    for (int k0 = 0; k0 < K; k0 += kE) {
      uint4 w[kE][NCI];
#pragma unroll
      for (int kk = 0; kk < kE; ++kk) {
        const int k = k0 + kk;
        const uint32_t e = k < K ? tb.ids[k] : 0xFFFFFFFFu;
        const int8_t *Wr = e < (uint32_t)a.E
                               ? L.w_ptr[e] + (size_t)2 * I * H + (size_t)j * I
                               : nullptr;
#pragma unroll
        for (int m = 0; m < NCI; ++m) {
          const int off = 16 * (lane + 32 * m);
          w[kk][m] = (Wr && off < I) ? ldg_stream16(Wr + off) : make_uint4(0, 0, 0, 0);
        }
      }
#pragma unroll
      for (int kk = 0; kk < kE; ++kk) {
        const int k = k0 + kk;
        if (k >= K) break;
        const uint8_t *x1 = xd + (size_t)k * 2 * I, *x2 = x1 + I;
        int d1 = 0, d2 = 0;
#pragma unroll
        for (int m = 0; m < NCI; ++m) {
          const int off = 16 * (lane + 32 * m);
          if (off < I) {
            dp4(w[kk][m], *reinterpret_cast<const uint4 *>(x1 + off), d1);
            dp4(w[kk][m], *reinterpret_cast<const uint4 *>(x2 + off), d2);
          }
        }
        d1 = warp_sum(d1);
        d2 = warp_sum(d2);
        if (lane == k) {
          my1 = d1;
          my2 = d2;
        }
      }
    }
    float c = 0.0f;
    if (lane < K) {
      const uint32_t e = tb.ids[lane];
      if (e < (uint32_t)a.E) {
        const float y = digits::down(my1, my2, tb.s1[lane], tb.s2[lane], L.s_ptr[e][2 * I + j]);
        bad |= !is_finite_f(y);
        c = __fmul_rn(tb.gates[lane], y);
      }
    }
    float acc = resid ? __ldcg(resid + j) : 0.0f;
    for (int k = 0; k < K; ++k) acc = __fadd_rn(acc, __shfl_sync(0xffffffffu, c, k));
    if (lane == 0) {
      bad |= !is_finite_f(acc);
      out[j] = acc;
    }
  }
  if (bad) set_status(a.status, kStatusNonFinite);
}

// D for T > 1: the CTA's share of (active expert, output row) pairs; gate * y
// into contrib[token, slot, row].  A warp takes four rows at a time.
template <int NCI>
__device__ void down_items(const DigitArgs &a, const FusedLayer &L, uint8_t *xd, DTables &tb) {
  constexpr int kRows = 4;
  const int H = a.H, I = a.I, K = a.K, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __shared__ int32_t rows[kGR];
  long long u0, u1;
  share((long long)tb.n_active * H, u0, u1);
  bool bad = false;
  for (long long u = u0; u < u1;) {
    const int ai = (int)(u / H), j0 = (int)(u - (long long)ai * H);
    const int j1 = (int)std::min<long long>(H, j0 + (u1 - u));
    u += j1 - j0;
    const int e = tb.active[ai], r0 = tb.seg_off[e], r1 = tb.seg_off[e + 1];
    const int8_t *Wd = L.w_ptr[e] + (size_t)2 * I * H;
    const float *Sd = L.s_ptr[e] + 2 * I;
    for (int rb = r0; rb < r1; rb += kGR) {
      const int nr = min(kGR, r1 - rb);
      __syncthreads();
      if (threadIdx.x < nr)
        rows[threadIdx.x] = tb.r_token[rb + threadIdx.x] * K + tb.r_slot[rb + threadIdx.x];
      __syncthreads();
      digitise_act(a, rows, nr, xd, tb);
      __syncthreads();
      for (int jb = j0 + warp * kRows; jb < j1; jb += kDW * kRows) {
        uint4 w[kRows][NCI];
#pragma unroll
        for (int q = 0; q < kRows; ++q)
#pragma unroll
          for (int m = 0; m < NCI; ++m) {
            const int off = 16 * (lane + 32 * m), j = jb + q;
            w[q][m] = (j < j1 && off < I) ? ldg_stream16(Wd + (size_t)j * I + off)
                                          : make_uint4(0, 0, 0, 0);
          }
        int my1[kRows] = {}, my2[kRows] = {};
        for (int r = 0; r < nr; ++r) {
          const uint8_t *x1 = xd + (size_t)r * 2 * I, *x2 = x1 + I;
          int d1[kRows] = {}, d2[kRows] = {};
#pragma unroll
          for (int m = 0; m < NCI; ++m) {
            const int off = 16 * (lane + 32 * m);
            if (off < I) {
              const uint4 c1 = *reinterpret_cast<const uint4 *>(x1 + off);
              const uint4 c2 = *reinterpret_cast<const uint4 *>(x2 + off);
#pragma unroll
              for (int q = 0; q < kRows; ++q) {
                dp4(w[q][m], c1, d1[q]);
                dp4(w[q][m], c2, d2[q]);
              }
            }
          }
#pragma unroll
          for (int q = 0; q < kRows; ++q) {
            d1[q] = warp_sum(d1[q]);
            d2[q] = warp_sum(d2[q]);
            if (lane == r) {
              my1[q] = d1[q];
              my2[q] = d2[q];
            }
          }
        }
        if (lane < nr) {
#pragma unroll
          for (int q = 0; q < kRows; ++q) {
            const int j = jb + q;
            if (j < j1) {
              const float y = digits::down(my1[q], my2[q], tb.s1[lane], tb.s2[lane], Sd[j]);
              bad |= !is_finite_f(y);
              a.contrib[(size_t)rows[lane] * H + j] = __fmul_rn(tb.r_gate[rb + lane], y);
            }
          }
        }
      }
    }
  }
  if (bad) set_status(a.status, kStatusNonFinite);
}

// out[t] = base[t] + contrib[t, 0] + ... + contrib[t, K-1] (slot order),
// base = resid (or 0).
__device__ void combine_phase(const DigitArgs &a, const float *resid, float *out) {
  const int H = a.H, K = a.K;
  bool bad = false;
  const size_t n = (size_t)a.T * H;
  for (size_t i = blockIdx.x * (size_t)kDT + threadIdx.x; i < n; i += (size_t)gridDim.x * kDT) {
    const size_t t = i / H, j = i % H;
    float acc = resid ? __ldcg(resid + i) : 0.0f;
    for (int k = 0; k < K; ++k) acc = __fadd_rn(acc, __ldcg(a.contrib + (t * K + k) * H + j));
    bad |= !is_finite_f(acc);
    out[i] = acc;
  }
  if (bad) set_status(a.status, kStatusNonFinite);
}

template <int NCH, int NCI>
__global__ void __launch_bounds__(kDT, 2) digit_decode_kernel(DigitArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  DTables &tb = *reinterpret_cast<DTables *>(smem);
  SelectScratch *sel = reinterpret_cast<SelectScratch *>(smem + kSelOff);
  uint8_t *stage = smem + kStageOff;
  const int G = gridDim.x, T = a.T, K = a.K, R = T * K;
  const int warp = threadIdx.x >> 5;
  uint32_t nbar = 0;
  auto sync = [&]() {
    ++nbar;
    return grid_sync(a.bar, nbar * G, a.status, a.wait_cycles);
  };
  stamp(a, 0);
  for (int l = 0; l < a.n_layers; ++l) {
    const FusedLayer L = a.layers[l];
    // stacked: x is the residual stream (in `out`), normalised while staged
    const float *xin = a.stacked ? a.out : a.h_in;
    const float *resid = a.stacked ? a.out : a.resid;
    router_phase(a, L, xin, a.stacked != 0, reinterpret_cast<float *>(stage), tb);
    if (!sync()) return;
    // S: selection
    if (T <= kDW) {
      if (warp < T)
        select_token(a.logits + (size_t)warp * a.E, a.E, K, a.norm, a.route_mode,
                     tb.ids + warp * K, tb.gates + warp * K, nullptr, sel[warp], a.status);
      __syncthreads();
      if (blockIdx.x == 0)
        for (int r = threadIdx.x; r < R; r += kDT) {
          a.ids[r] = tb.ids[r];
          a.gates[r] = tb.gates[r];
        }
    } else {
      for (int t = blockIdx.x * kDW + warp; t < T; t += G * kDW)
        select_token(a.logits + (size_t)t * a.E, a.E, K, a.norm, a.route_mode, a.ids + t * K,
                     a.gates + t * K, nullptr, sel[warp], a.status);
      if (!sync()) return;
      for (int r = threadIdx.x; r < R; r += kDT) {
        tb.ids[r] = __ldcg(a.ids + r);
        tb.gates[r] = __ldcg(a.gates + r);
      }
      __syncthreads();
    }
    build_tables(R, K, a.E, tb);
    if (l == 0) stamp(a, 1);
    if (a.prefetch_down) prefetch_down(a, L, tb);
    gate_up_phase<NCH>(a, L, stage, tb);
    if (!sync()) return;
    if (l == 0) stamp(a, 2);
    if (T == 1) {
      down_single<NCI>(a, L, resid, a.out, stage, tb);
    } else {
      down_items<NCI>(a, L, stage, tb);
      if (!sync()) return;
      combine_phase(a, resid, a.out);
    }
    if (l == 0) stamp(a, 3);
    if (a.stacked && l + 1 < a.n_layers && !sync()) return;
  }
  if (blockIdx.x == 0 && a.ids_out)
    for (int r = threadIdx.x; r < R; r += kDT) {
      a.ids_out[r] = __ldcg(a.ids + r);
      a.gates_out[r] = __ldcg(a.gates + r);
    }
  __syncthreads();
  stamp(a, 4);
}

size_t digit_smem_bytes(int H, int I) {
  const size_t router = (size_t)(kRTT + kRTE) * H * sizeof(float);
  const size_t digits = (size_t)kGR * 2 * std::max(H, I);
  return kStageOff + std::max(router, digits);
}

}  // namespace

bool digit_decode_supported(int T, int H, int I, int E, int K) {
  return T >= 1 && T * K <= kFusedMaxRoutes && K <= kMaxTopK && E <= kMaxExperts &&
         H % 16 == 0 && I % 16 == 0 && H <= 32 * 16 * kMaxChunks &&
         I <= 32 * 16 * kMaxChunks && digit_smem_bytes(H, I) <= 113 * 1024;
}

cudaError_t launch_digit_decode(const DigitArgs &a_in, int sm_count, cudaStream_t s) {
  const size_t smem = digit_smem_bytes(a_in.H, a_in.I);
  // 16-byte chunks per lane of an H row and of an I row
  const int nch = (a_in.H / 16 + 31) / 32, nci = (a_in.I / 16 + 31) / 32;
  const void *fn = nch <= 2 ? (nci <= 2 ? (const void *)digit_decode_kernel<2, 2>
                                        : (const void *)digit_decode_kernel<2, 4>)
                            : (nci <= 2 ? (const void *)digit_decode_kernel<4, 2>
                                        : (const void *)digit_decode_kernel<4, 4>);
  static thread_local int cached_dev = -1, cached_grid = 0;
  static thread_local const void *cached_fn = nullptr;
  static thread_local size_t cached_smem = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev != cached_dev || smem != cached_smem || fn != cached_fn) {
    cudaError_t e =
        cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kDT, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorLaunchOutOfResources;
    cached_dev = dev;
    cached_smem = smem;
    cached_fn = fn;
    cached_grid = std::min(per_sm, 2) * sm_count;
  }
  cudaError_t e = cudaMemsetAsync(a_in.bar, 0, sizeof(uint32_t), s);
  if (e != cudaSuccess) return e;
  DigitArgs a = a_in;
  a.router_async = a_in.router_async && a_in.H % 4 == 0;
  void *params[] = {&a};
  return cudaLaunchCooperativeKernel(fn, dim3(cached_grid), dim3(kDT), params, smem, s);
}

}  // namespace moe
