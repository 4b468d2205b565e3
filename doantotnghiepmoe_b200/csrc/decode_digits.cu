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
// Every barrier wait is bounded (DigitArgs::wait_cycles); on expiry the CTA
// records kStatusTimeout and stops.  The barrier counters reset themselves at
// the end of each launch.
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
constexpr int kRowPad = 8;       // floats of padding per staged router-phase row


struct DTables {
  int32_t run[kMaxExperts];               // counting-sort scratch
  int32_t act_e[kMaxExperts];             // active experts, ascending id
  int32_t act_r0[kMaxExperts + 1];        // routes of active a: [act_r0[a], act_r0[a + 1])
  int32_t cost_g[kMaxExperts + 1];        // gate/up cost prefix over the active experts
  int32_t cost_d[kMaxExperts + 1];        // down cost prefix
  int32_t n_active;
  int32_t r_token[kFusedMaxRoutes];       // sorted route -> token, slot, gate
  int32_t r_slot[kFusedMaxRoutes];
  float r_gate[kFusedMaxRoutes];
  uint32_t ids[kFusedMaxRoutes];          // token-major routing of the current layer
  float gates[kFusedMaxRoutes];
  const int8_t *wp[kMaxExperts];          // the layer's expert pointers
  const float *sp[kMaxExperts];
  union {
    int32_t wcnt[kDW][kMaxExperts];       // tables: per-warp counts
    struct {
      uint32_t key[kDW][kMaxExperts];     // top-k: total-order keys of a warp's token
      float ex[kDW][kMaxExperts];         // softmax numerators
    } s;
  } u;
  float sel_v[kDW][kMaxTopK];
  uint32_t sel_i[kDW][kMaxTopK];
  float s1[kMaxTopK > kGR ? kMaxTopK : kGR];  // scales of the staged digit rows
  float s2[kMaxTopK > kGR ? kMaxTopK : kGR];
  float inv[kRTT];                            // RMSNorm factors of the staged tokens
};

constexpr size_t align128(size_t n) { return (n + 127) & ~size_t(127); }
constexpr size_t kStageOff = align128(sizeof(DTables));

__device__ __forceinline__ bool grid_sync(uint32_t *bar, uint32_t target, uint32_t *status,
                                          long long limit) {
  __shared__ int ok;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(bar, 1u);
    const long long t0 = clock64();
    int good = 1;
    // poll without sleeping for the first few microseconds (the usual wait
    // is one phase's tail), then back off
    for (int it = 0; *(volatile uint32_t *)bar < target; ++it) {
      if (clock64() - t0 > limit) {
        good = 0;
        set_status(status, kStatusTimeout);
        break;
      }
      if (it > 4096) __nanosleep(64);
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
// One token's digit planes by a whole CTA that has no router task: the row
// (RMS-normalised first in stacks, with the router tasks' exact arithmetic)
// is staged, its max |x| reduced over the CTA, and its planes and scales
// written.  Runs while the router tasks compute the logits, so the planes
// leave the router tasks' critical path.
// ---------------------------------------------------------------------------
__device__ void token_digits_cta(const DigitArgs &a, const FusedLayer &L, const float *xin,
                                 bool stacked, int t, float *stage, DTables &tb) {
  const int H = a.H, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int full = H / 8;
  float *x = stage;
  for (int c = tid; c < H; c += kDT) x[c] = __ldcg(xin + (size_t)t * H + c);
  __syncthreads();
  if (stacked) {
    // the router tasks' RMSNorm, operation for operation
    if (warp == 0) {
      float acc = 0.0f;
      if (lane < 8) {
        int c = 0;
        for (; c + 16 <= full; c += 16) {
          float p[16];
#pragma unroll
          for (int u = 0; u < 16; ++u) {
            const float v = x[8 * (c + u) + lane];
            p[u] = __fmul_rn(v, v);
          }
#pragma unroll
          for (int u = 0; u < 16; ++u) acc = __fadd_rn(acc, p[u]);
        }
        for (; c < full; ++c) {
          const float v = x[8 * c + lane];
          acc = __fadd_rn(acc, __fmul_rn(v, v));
        }
      }
      float sq = -0.0f;
#pragma unroll
      for (int l = 0; l < 8; ++l) sq = __fadd_rn(sq, __shfl_sync(0xffffffffu, acc, l));
      for (int i = full * 8; i < H; ++i) sq = __fadd_rn(sq, __fmul_rn(x[i], x[i]));
      if (lane == 0) {
        const float scale = __fsqrt_rn(__fadd_rn(__fdiv_rn(sq, (float)H), a.eps));
        tb.inv[0] = __fdiv_rn(1.0f, scale);
      }
    }
    __syncthreads();
    const float inv = tb.inv[0];
    for (int j = tid; j < H; j += kDT) {
      const float w = L.norm_w ? L.norm_w[j] : 1.0f;
      x[j] = __fmul_rn(__fmul_rn(x[j], inv), w);
    }
    __syncthreads();
  }
  // max |x| over the row (order-free), then the planes, 4 columns a thread
  float amax = 0.0f;
  for (int c = 4 * tid; c < H; c += 4 * kDT) {
    const float4 v = *reinterpret_cast<const float4 *>(x + c);
    amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  // per-warp maxima in the top-k scratch (unused until after the barrier)
  float *red = tb.u.s.ex[0];
  if (lane == 0) red[warp] = amax;
  __syncthreads();
  amax = 0.0f;
  for (int w = 0; w < kDW; ++w) amax = fmaxf(amax, red[w]);
  const float sc = digits::row_scale(amax);
  const float inv = 1.0f / sc;
  int8_t *q1 = a.xq + (size_t)t * 2 * H, *q2 = q1 + H;
  for (int c = 4 * tid; c < H; c += 4 * kDT) {
    const float4 v = *reinterpret_cast<const float4 *>(x + c);
    uint32_t p2;
    const uint32_t p1 = digits::split4(v.x, v.y, v.z, v.w, inv, p2);
    *reinterpret_cast<uint32_t *>(q1 + c) = p1;
    *reinterpret_cast<uint32_t *>(q2 + c) = p2;
  }
  if (tid == 0) {
    a.xs1[t] = sc;
    a.xs2[t] = sc / 254.0f;
  }
  __syncthreads();
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
  // staged rows are kRowPad floats longer than H, so the 4 expert rows a
  // warp reads at the same column fall in different banks
  const int RS = H + kRowPad;
  const bool seq = a.route_mode == kRouteTopkSoftmax && L.router_dtype == kRouterF32;
  // with CTAs to spare, CTAs [tasks, tasks + T) make the tokens' digit planes
  // while the router tasks run; otherwise the tasks of expert group 0 do
  const bool sep = tasks + T <= (int)gridDim.x;
  if (sep && (int)blockIdx.x >= tasks && (int)blockIdx.x < tasks + T)
    token_digits_cta(a, L, xin, stacked, (int)blockIdx.x - tasks, stage, tb);
  for (int task = blockIdx.x; task < tasks; task += gridDim.x) {
    const int t0 = (task / nte) * TT, e0 = (task % nte) * RE;
    const int nt = min(TT, T - t0);
    bool bad = false;
    // stage rows [0, TT) tokens, [TT, TT + RE) router rows
    if (a.router_async) {
      const int q = H / 4;
      for (int r = 0; r < TT + RE; ++r) {
        const float *row = nullptr;
        if (r < TT) {
          if (r < nt) row = xin + (size_t)(t0 + r) * H;
        } else if (e0 + r - TT < E) {
          row = reinterpret_cast<const float *>(L.router) + (size_t)(e0 + r - TT) * H;
        }
        for (int c = 4 * tid; c < 4 * q; c += 4 * kDT) {
          float *dst = stage + (size_t)r * RS + c;
          if (row) {
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(
                             (uint32_t)__cvta_generic_to_shared(dst)),
                         "l"(row + c)
                         : "memory");
          } else {
            *reinterpret_cast<float4 *>(dst) = make_float4(0.f, 0.f, 0.f, 0.f);
          }
        }
      }
      asm volatile("cp.async.wait_all;" ::: "memory");
    } else {
      for (int r = 0; r < TT + RE; ++r)
        for (int c = tid; c < H; c += kDT) {
          float v = 0.0f;
          if (r < TT) {
            if (r < nt) v = __ldcg(xin + (size_t)(t0 + r) * H + c);
          } else if (e0 + r - TT < E) {
            v = load_w(L.router, L.router_dtype, (size_t)(e0 + r - TT) * H + c);
          }
          stage[(size_t)r * RS + c] = v;
        }
    }
    __syncthreads();
    const bool sub = task == (int)blockIdx.x && a.sub_stamps;  // first task, profiling
    if (sub) stamp(a, 9);
    for (int r = 0; r < nt; ++r)
      for (int j = tid; j < H; j += kDT)
        if (!is_finite_f(stage[(size_t)r * RS + j])) bad = true;
    if (stacked) {
      // RMSNorm of each staged token row (src/backend.rs:341-359): lanes 0..7
      // of warp r run the 8-lane sum of squares, then every thread scales.
      if (warp < nt) {
        const float *x = stage + (size_t)warp * RS;
        float acc = 0.0f;
        if (lane < 8) {
          // blocks of 16 squares ahead of the dependent adds (same order)
          int c = 0;
          for (; c + 16 <= full; c += 16) {
            float p[16];
#pragma unroll
            for (int u = 0; u < 16; ++u) {
              const float v = x[8 * (c + u) + lane];
              p[u] = __fmul_rn(v, v);
            }
#pragma unroll
            for (int u = 0; u < 16; ++u) acc = __fadd_rn(acc, p[u]);
          }
          for (; c < full; ++c) {
            const float v = x[8 * c + lane];
            acc = __fadd_rn(acc, __fmul_rn(v, v));
          }
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
      for (int j = tid; j < H; j += kDT) {
        const float w = L.norm_w ? L.norm_w[j] : 1.0f;
        for (int r = 0; r < nt; ++r) {
          float &v = stage[(size_t)r * RS + j];
          const float o = __fmul_rn(__fmul_rn(v, tb.inv[r]), w);
          if (!is_finite_f(o)) bad = true;
          v = o;
        }
      }
      __syncthreads();
    }
    if (bad) set_status(a.status, kStatusNonFinite);
    if (sub) stamp(a, 10);
    // 8 lanes per (token, expert) pair, whole warps (the fold is a shuffle)
    const int npairs = TT * RE;
    if (tid < ((8 * npairs + 31) & ~31)) {
      const int l8 = tid & 7, pair = tid >> 3;
      const bool live = pair < npairs;
      const int ti = live ? pair / RE : 0, ei = live ? pair % RE : 0;
      const float *hs = stage + (size_t)ti * RS;
      const float *w = stage + (size_t)(TT + ei) * RS;
      float logit;
      if (seq) {
        float acc = -0.0f;  // src/router.rs:59-62, Rust's f32 Sum folds from -0.0
        if (l8 == 0)
          for (int c = 0; c < H; ++c) acc = __fadd_rn(acc, __fmul_rn(w[c], hs[c]));
        logit = acc;
      } else {
        float acc = 0.0f;  // `[0.0f32; 8]`, src/backend.rs:107
        // blocks of 16 products ahead of the dependent adds (same order)
        int c = 0;
        for (; c + 16 <= full; c += 16) {
          float p[16];
#pragma unroll
          for (int u = 0; u < 16; ++u) p[u] = __fmul_rn(w[8 * (c + u) + l8], hs[8 * (c + u) + l8]);
#pragma unroll
          for (int u = 0; u < 16; ++u) acc = __fadd_rn(acc, p[u]);
        }
        for (; c < full; ++c) acc = __fadd_rn(acc, __fmul_rn(w[8 * c + l8], hs[8 * c + l8]));
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
    if (sub) {
      __syncthreads();
      stamp(a, 11);
    }
    // the token rows' digit planes, once per token (expert group 0), on the
    // warps above the ones running the dot (token r on warp kDW - 1 - r)
    if (!sep && e0 == 0 && kDW - 1 - warp < nt) {
      const int r = kDW - 1 - warp;
      const float *x = stage + (size_t)r * RS;
      float amax = 0.0f;
      for (int c = lane * 4; c < H; c += 128) {
        const float4 v = *reinterpret_cast<const float4 *>(x + c);
        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      const float s = digits::row_scale(amax);
      const float inv = 1.0f / s;
      const int t = t0 + r;
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

// S: softmax and top-k of one token, by one warp (src/backend.rs:375-389,
// src/olmoe.rs:2595-2621; the Router::select_top_k variant, src/router.rs:
// 84-103, on raw scores).  Same arithmetic as select_token in route_core.cuh;
// the K winners are found by rank instead of K argmax rounds: a candidate's
// slot is the number of candidates before it in the reference's order
// (f32::total_cmp descending, ties to the lower expert id).
template <int kPer>
__device__ void select_rank(const float *lg, int E, int K, int norm_topk_prob, int mode,
                            uint32_t *ids, float *gates, uint32_t *key, float *sel_v,
                            uint32_t *sel_i, float *ex, uint32_t *status) {
  const int lane = threadIdx.x & 31;
  float v[kPer];
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int e = lane + 32 * j;
    v[j] = e < E ? __ldcg(lg + e) : __int_as_float(0xff800000);  // -inf pad
  }
  if (mode == kRouteSoftmaxTopk) {
    float mx = __int_as_float(0xff800000);
#pragma unroll
    for (int j = 0; j < kPer; ++j) mx = fmaxf(mx, v[j]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int e = lane + 32 * j;
      if (e < E) {
        v[j] = expf_ref(__fsub_rn(v[j], mx));
        ex[e] = v[j];
      }
    }
    __syncwarp();
    float sum = 0.0f;
    if (lane == 0) {
      // sequential in index order, loads batched ahead of the dependent adds
      sum = -0.0f;
      int e = 0;
      for (; e + 8 <= E; e += 8) {
        float v8[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v8[j] = ex[e + j];
#pragma unroll
        for (int j = 0; j < 8; ++j) sum = __fadd_rn(sum, v8[j]);
      }
      for (; e < E; ++e) sum = __fadd_rn(sum, ex[e]);
    }
    sum = __shfl_sync(0xffffffffu, sum, 0);
#pragma unroll
    for (int j = 0; j < kPer; ++j)
      if (lane + 32 * j < E) v[j] = __fdiv_rn(v[j], sum);
  } else {
    // partial_cmp treats -0.0 == +0.0: canonical zero, so ties go by index
#pragma unroll
    for (int j = 0; j < kPer; ++j)
      if (v[j] == 0.0f) v[j] = 0.0f;
  }
  uint32_t k[kPer];
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    k[j] = total_order_u32(v[j]);
    if (lane + 32 * j < E) key[lane + 32 * j] = k[j];
  }
  __syncwarp();
  int rank[kPer];
#pragma unroll
  for (int j = 0; j < kPer; ++j) rank[j] = 0;
  // 8 keys a step: their shared-memory loads issue back to back
  int f = 0;
  for (; f + 8 <= E; f += 8) {
    uint32_t kf[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) kf[u] = key[f + u];
#pragma unroll
    for (int u = 0; u < 8; ++u)
#pragma unroll
      for (int j = 0; j < kPer; ++j) {
        const int e = lane + 32 * j;
        rank[j] += (kf[u] > k[j]) || (kf[u] == k[j] && f + u < e);
      }
  }
  for (; f < E; ++f) {
    const uint32_t kf = key[f];
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int e = lane + 32 * j;
      rank[j] += (kf > k[j]) || (kf == k[j] && f < e);
    }
  }
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int e = lane + 32 * j;
    if (e < E && rank[j] < K) {
      sel_v[rank[j]] = v[j];
      sel_i[rank[j]] = (uint32_t)e;
    }
  }
  __syncwarp();
  if (mode == kRouteSoftmaxTopk) {
    float norm = 1.0f;
    if (norm_topk_prob) {
      if (lane == 0) {
        norm = -0.0f;
        for (int q = 0; q < K; ++q) norm = __fadd_rn(norm, sel_v[q]);
      }
      norm = __shfl_sync(0xffffffffu, norm, 0);
    }
    if (lane < K) {
      ids[lane] = sel_i[lane];
      gates[lane] = __fdiv_rn(sel_v[lane], norm);
      if (sel_i[lane] >= (uint32_t)E) set_status(status, kStatusBadRoute);
    }
  } else {
    float total = 0.0f;
    if (lane == 0) {
      const float mx = sel_v[0];
      total = -0.0f;
      for (int q = 0; q < K; ++q) {
        ex[q] = expf_ref(__fsub_rn(sel_v[q], mx));
        total = __fadd_rn(total, ex[q]);
      }
    }
    total = __shfl_sync(0xffffffffu, total, 0);
    __syncwarp();
    if (lane < K) {
      ids[lane] = sel_i[lane];
      gates[lane] = __fdiv_rn(ex[lane], total);
    }
  }
  __syncwarp();
}

__device__ __forceinline__ void select_one(const DigitArgs &a, int t, uint32_t *ids,
                                           float *gates, DTables &tb) {
  const int w = threadIdx.x >> 5;
  const float *lg = a.logits + (size_t)t * a.E;
  uint32_t *key = tb.u.s.key[w];
  float *ex = tb.u.s.ex[w];
  if (a.E <= 64)
    select_rank<2>(lg, a.E, a.K, a.norm, a.route_mode, ids, gates, key, tb.sel_v[w],
                   tb.sel_i[w], ex, a.status);
  else if (a.E <= 128)
    select_rank<4>(lg, a.E, a.K, a.norm, a.route_mode, ids, gates, key, tb.sel_v[w],
                   tb.sel_i[w], ex, a.status);
  else
    select_rank<kMaxExperts / 32>(lg, a.E, a.K, a.norm, a.route_mode, ids, gates, key,
                                  tb.sel_v[w], tb.sel_i[w], ex, a.status);
}

// P: the R routes (tb.ids, token-major) sorted by expert, stable
// (src/olmoe.rs:3474-3480: experts ascending, routes ascending inside), as
// active-expert ranges, plus the cost prefixes of the gate/up and down splits.
__device__ void build_tables(const DigitArgs &a, int R, DTables &tb) {
  const int K = a.K, E = a.E, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (R <= 32) {
    // one warp: a route's position counts the routes ordered before it
    if (warp == 0) {
      const uint32_t e = lane < R ? tb.ids[lane] : 0xFFFFFFFFu;
      const bool valid = e < (uint32_t)E;
      const unsigned same = __match_any_sync(0xffffffffu, valid ? e : 0xFFFFFFFFu);
      const bool first = valid && (__ffs(same) - 1) == lane;
      int pos = 0, act = 0;
      for (int l = 0; l < 32; ++l) {
        const uint32_t el = __shfl_sync(0xffffffffu, e, l);
        const bool fl = __shfl_sync(0xffffffffu, first, l);
        pos += el < (uint32_t)E && (el < e || (el == e && l < lane));
        act += fl && el < e;
      }
      if (valid) {
        tb.r_token[pos] = lane / K;
        tb.r_slot[pos] = lane % K;
        tb.r_gate[pos] = tb.gates[lane];
      }
      if (first) {
        tb.act_e[act] = (int)e;
        tb.act_r0[act] = pos;
      }
      const int na = __popc(__ballot_sync(0xffffffffu, first));
      const int nv = __popc(__ballot_sync(0xffffffffu, valid));
      if (lane == 0) {
        tb.n_active = na;
        tb.act_r0[na] = nv;
      }
    }
  } else {
    for (int e = tid; e < E; e += kDT) tb.run[e] = 0;
    for (int i = tid; i < kDW * E; i += kDT) tb.u.wcnt[i / E][i % E] = 0;
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
          tb.run[e] = acc + inc - c;
          if (c > 0) {
            const int ai = na + __popc(act & ((1u << lane) - 1u));
            tb.act_e[ai] = e;
            tb.act_r0[ai] = acc + inc - c;
          }
        }
        acc += __shfl_sync(0xffffffffu, inc, 31);
        na += __popc(act);
      }
      if (lane == 0) {
        tb.n_active = na;
        tb.act_r0[na] = acc;
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
      if (ok && intra == 0) tb.u.wcnt[warp][e] = __popc(mask);
      __syncthreads();
      if (ok) {
        int pos = tb.run[e] + intra;
        for (int w = 0; w < warp; ++w) pos += tb.u.wcnt[w][e];
        tb.r_token[pos] = r / K;
        tb.r_slot[pos] = r % K;
        tb.r_gate[pos] = tb.gates[r];
      }
      __syncthreads();
      for (int ee = tid; ee < E; ee += kDT) {
        int tot = 0;
        for (int w = 0; w < kDW; ++w) {
          tot += tb.u.wcnt[w][ee];
          tb.u.wcnt[w][ee] = 0;
        }
        tb.run[ee] += tot;
      }
      __syncthreads();
    }
  }
  __syncthreads();
  // cost prefixes: a gate/up row pair costs (routes + gate_w), a down row
  // (routes + down_w), in units of one route's dot products
  if (warp == 0) {
    const int na = tb.n_active;
    int cg = 0, cd = 0;
    for (int base = 0; base < na; base += 32) {
      const int ai = base + lane;
      const int r = ai < na ? tb.act_r0[ai + 1] - tb.act_r0[ai] : 0;
      int g = ai < na ? a.I * (r + a.gate_w) : 0, d = ai < na ? a.H * (r + a.down_w) : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int vg = __shfl_up_sync(0xffffffffu, g, o), vd = __shfl_up_sync(0xffffffffu, d, o);
        if (lane >= o) {
          g += vg;
          d += vd;
        }
      }
      if (ai < na) {
        tb.cost_g[ai + 1] = cg + g;
        tb.cost_d[ai + 1] = cd + d;
      }
      cg += __shfl_sync(0xffffffffu, g, 31);
      cd += __shfl_sync(0xffffffffu, d, 31);
    }
    if (lane == 0) {
      tb.cost_g[0] = 0;
      tb.cost_d[0] = 0;
    }
  }
  __syncthreads();
}

// P for one token, by the warp that selected it: the K routes' experts are
// distinct, so a route's sorted position is the number of smaller expert ids.
__device__ void tables_single(const DigitArgs &a, DTables &tb) {
  const int K = a.K, lane = threadIdx.x & 31;
  __syncwarp();
  const uint32_t e = lane < K ? tb.ids[lane] : 0xFFFFFFFFu;
  const bool valid = e < (uint32_t)a.E;
  int pos = 0;
  for (int l = 0; l < K; ++l) {
    const uint32_t el = __shfl_sync(0xffffffffu, e, l);
    pos += el < (uint32_t)a.E && el < e;
  }
  if (valid) {
    tb.r_token[pos] = 0;
    tb.r_slot[pos] = lane;
    tb.r_gate[pos] = tb.gates[lane];
    tb.act_e[pos] = (int)e;
    tb.act_r0[pos] = pos;
  }
  const int na = __popc(__ballot_sync(0xffffffffu, valid));
  if (lane <= na) {
    tb.cost_g[lane] = lane * a.I * (1 + a.gate_w);
    tb.cost_d[lane] = lane * a.H * (1 + a.down_w);
  }
  if (lane == 0) {
    tb.n_active = na;
    tb.act_r0[na] = na;
  }
  __syncwarp();
}

// This CTA's part of a cost-weighted split: the active experts a with rows
// [rows_lo, rows_hi) of n rows each, unit cost w_a = routes + w0.  CTA c owns
// cost [C c / G, C (c + 1) / G); a boundary inside expert a falls on row
// ceil((x - cost[a]) / w_a), so neighbouring CTAs meet exactly.
template <typename F>
__device__ __forceinline__ void for_each_share(const DTables &tb, const int32_t *cost, int n,
                                               int w0, F &&fn) {
  const int na = tb.n_active;
  const long long C = cost[na];
  const long long c0 = C * blockIdx.x / gridDim.x, c1 = C * (blockIdx.x + 1) / gridDim.x;
  for (int ai = 0; ai < na; ++ai) {
    if (cost[ai + 1] <= c0) continue;
    if (cost[ai] >= c1) break;
    const int r0 = tb.act_r0[ai], r1 = tb.act_r0[ai + 1];
    const long long w = r1 - r0 + w0;
    const long long lo = std::max<long long>(0, c0 - cost[ai]);
    const long long hi = std::min<long long>((long long)n * w, c1 - cost[ai]);
    const int row0 = (int)((lo + w - 1) / w), row1 = (int)std::min<long long>(n, (hi + w - 1) / w);
    if (row1 > row0) fn(ai, row0, row1, r0, r1);
  }
}

// The CTA's share [u0, u1) of n equal units.
__device__ __forceinline__ void share(long long n, long long &u0, long long &u1) {
  u0 = n * blockIdx.x / gridDim.x;
  u1 = n * (blockIdx.x + 1) / gridDim.x;
}

// Bulk L2 prefetch of the down rows this CTA reads in D (same partition).
__device__ void prefetch_down(const DigitArgs &a, const DTables &tb) {
  if (threadIdx.x != 0) return;
  const int H = a.H, I = a.I;
  if (a.T == 1) {
    long long u0, u1;
    share(H, u0, u1);
    if (u1 <= u0) return;
    for (int k = 0; k < a.K; ++k) {
      const uint32_t e = tb.ids[k];
      if (e >= (uint32_t)a.E) continue;
      prefetch_l2(tb.wp[e] + (size_t)2 * I * H + (size_t)u0 * I, (uint32_t)((u1 - u0) * I));
      // the rows' scales, widened to whole 16-byte blocks
      const uintptr_t s0 = reinterpret_cast<uintptr_t>(tb.sp[e] + 2 * I + u0) & ~uintptr_t(15);
      const uintptr_t s1 =
          (reinterpret_cast<uintptr_t>(tb.sp[e] + 2 * I + u1) + 15) & ~uintptr_t(15);
      prefetch_l2(reinterpret_cast<const void *>(s0), (uint32_t)(s1 - s0));
    }
    return;
  }
  for_each_share(tb, tb.cost_d, H, a.down_w, [&](int ai, int j0, int j1, int, int) {
    prefetch_l2(tb.wp[tb.act_e[ai]] + (size_t)2 * I * H + (size_t)j0 * I,
                (uint32_t)((j1 - j0) * I));
  });
}

// G: gate/up over the CTA's cost share of the (active expert, row pair)
// units.  A warp takes two row pairs at a time, so 4 * NCH 16-byte loads per
// lane are in flight before the first dot (NCH = 16-byte chunks per lane of
// an H row); the rows' scales are loaded with them.
template <int NCH>
__device__ void gate_up_phase(const DigitArgs &a, uint8_t *xd, DTables &tb) {
  constexpr int kRows = 2;
  const int H = a.H, I = a.I, K = a.K, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for_each_share(tb, tb.cost_g, I, a.gate_w, [&](int ai, int i0, int i1, int r0, int r1) {
    const int e = tb.act_e[ai];
    const int8_t *W = tb.wp[e];
    const float *S = tb.sp[e];
    // this share's gate and up rows head for L2 while the digits are staged
    if (tid == 0) {
      prefetch_l2(W + (size_t)i0 * H, (uint32_t)((i1 - i0) * H));
      prefetch_l2(W + (size_t)(I + i0) * H, (uint32_t)((i1 - i0) * H));
    }
    for (int rb = r0; rb < r1; rb += kGR) {
      const int nr = min(kGR, r1 - rb);
      // the digit planes of routes rb .. rb + nr (2H bytes each) and scales
      __syncthreads();
      const int q16 = 2 * H / 16;
      for (int j = 0; j < nr; ++j) {
        const uint4 *src =
            reinterpret_cast<const uint4 *>(a.xq + (size_t)tb.r_token[rb + j] * 2 * H);
        for (int o = tid; o < q16; o += kDT)
          reinterpret_cast<uint4 *>(xd + (size_t)j * 2 * H)[o] = __ldcg(src + o);
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
        float sg[kRows], su[kRows];
#pragma unroll
        for (int q = 0; q < kRows; ++q) {
          const int i = min(ib + q, i1 - 1);
          sg[q] = S[i];
          su[q] = S[I + i];
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
                                      sg[q], su[q]);
          }
        }
      }
    }
  });
}

// Digit planes of activation rows (I floats each, read through L2) into xd,
// one warp per row; scales into tb.s1 / tb.s2.  act_row[j] = act row index.
// Lane l owns the 16-element chunks l + 32 m (m < NCI) of the row, the same
// chunks its dot products read later; all of its loads go out before the
// row maximum is formed.
template <int NCI>
__device__ void digitise_act(const DigitArgs &a, const int32_t *act_row, int nr, uint8_t *xd,
                             DTables &tb) {
  const int I = a.I, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int j = warp; j < nr; j += kDW) {
    const float4 *x = reinterpret_cast<const float4 *>(a.act + (size_t)act_row[j] * I);
    float4 v[NCI][4];
    float amax = 0.0f;
#pragma unroll
    for (int m = 0; m < NCI; ++m) {
      const int c = 16 * (lane + 32 * m);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        v[m][q] = c < I ? __ldcg(x + c / 4 + q) : make_float4(0.f, 0.f, 0.f, 0.f);
        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[m][q].x), fabsf(v[m][q].y)),
                                 fmaxf(fabsf(v[m][q].z), fabsf(v[m][q].w))));
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float s = digits::row_scale(amax);
    const float inv = 1.0f / s;
    uint8_t *q1 = xd + (size_t)j * 2 * I, *q2 = q1 + I;
#pragma unroll
    for (int m = 0; m < NCI; ++m) {
      const int c = 16 * (lane + 32 * m);
      if (c < I) {
        uint32_t p1[4], p2[4];
#pragma unroll
        for (int q = 0; q < 4; ++q)
          p1[q] = digits::split4(v[m][q].x, v[m][q].y, v[m][q].z, v[m][q].w, inv, p2[q]);
        *reinterpret_cast<uint4 *>(q1 + c) = make_uint4(p1[0], p1[1], p1[2], p1[3]);
        *reinterpret_cast<uint4 *>(q2 + c) = make_uint4(p2[0], p2[1], p2[2], p2[3]);
      }
    }
    if (lane == 0) {
      tb.s1[j] = s;
      tb.s2[j] = s / 254.0f;
    }
  }
}

// D for one token: the CTA's block of output rows [u0, u1) over all K
// routes.  Warp w streams slot w's expert (and w + 8, ...): its rows of the
// block are contiguous, and all of them are loaded before the first dot.  The
// gate-weighted outputs meet in shared memory and each row is combined in slot
// order: out = base + g_0 y_0 + ... + g_{K-1} y_{K-1}.
template <int NCI>
__device__ void down_single(const DigitArgs &a, const float *resid, float *out, uint8_t *xd,
                            DTables &tb) {
  constexpr int kMaxRows = 8;  // rows of the block handled per pass
  const int H = a.H, I = a.I, K = a.K, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  long long u0, u1;
  share(H, u0, u1);
  const int nrows = (int)(u1 - u0);
  __shared__ int32_t rows[kMaxTopK];
  __shared__ float cs[kMaxRows][kMaxTopK];
  if (threadIdx.x < K) rows[threadIdx.x] = threadIdx.x;  // act row of slot k (token 0)
  __syncthreads();
  digitise_act<NCI>(a, rows, K, xd, tb);
  __syncthreads();
  bool bad = false;
  for (int r0 = 0; r0 < nrows; r0 += kMaxRows) {
    const int nr = min(kMaxRows, nrows - r0);
    for (int k = warp; k < K; k += kDW) {
      const uint32_t e = tb.ids[k];
      if (e >= (uint32_t)a.E) {
        if (lane < nr) cs[lane][k] = 0.0f;
        continue;
      }
      const int j0 = (int)u0 + r0;
      const int8_t *Wr = tb.wp[e] + (size_t)2 * I * H + (size_t)j0 * I;
      const float sd = lane < nr ? tb.sp[e][2 * I + j0 + lane] : 0.0f;
      uint4 w[kMaxRows][NCI];
#pragma unroll
      for (int q = 0; q < kMaxRows; ++q)
#pragma unroll
        for (int m = 0; m < NCI; ++m) {
          const int off = 16 * (lane + 32 * m);
          w[q][m] = (q < nr && off < I) ? ldg_stream16(Wr + (size_t)q * I + off)
                                        : make_uint4(0, 0, 0, 0);
        }
      const uint8_t *x1 = xd + (size_t)k * 2 * I, *x2 = x1 + I;
      uint4 c1[NCI], c2[NCI];
#pragma unroll
      for (int m = 0; m < NCI; ++m) {
        const int off = 16 * (lane + 32 * m);
        c1[m] = off < I ? *reinterpret_cast<const uint4 *>(x1 + off) : make_uint4(0, 0, 0, 0);
        c2[m] = off < I ? *reinterpret_cast<const uint4 *>(x2 + off) : make_uint4(0, 0, 0, 0);
      }
      int my1 = 0, my2 = 0;  // sums of row `lane`
#pragma unroll
      for (int q = 0; q < kMaxRows; ++q) {
        if (q >= nr) break;
        int d1 = 0, d2 = 0;
#pragma unroll
        for (int m = 0; m < NCI; ++m) {
          dp4(w[q][m], c1[m], d1);
          dp4(w[q][m], c2[m], d2);
        }
        d1 = warp_sum(d1);
        d2 = warp_sum(d2);
        if (lane == q) {
          my1 = d1;
          my2 = d2;
        }
      }
      if (lane < nr) {
        const float y = digits::down(my1, my2, tb.s1[k], tb.s2[k], sd);
        bad |= !is_finite_f(y);
        cs[lane][k] = __fmul_rn(tb.gates[k], y);
      }
    }
    __syncthreads();
    if (threadIdx.x < nr) {
      const int j = (int)u0 + r0 + threadIdx.x;
      float acc = resid ? __ldcg(resid + j) : 0.0f;
      for (int k = 0; k < K; ++k) acc = __fadd_rn(acc, cs[threadIdx.x][k]);
      bad |= !is_finite_f(acc);
      out[j] = acc;
    }
    __syncthreads();
  }
  if (bad) set_status(a.status, kStatusNonFinite);
}

// D for T > 1: the CTA's cost share of (active expert, output row) units;
// gate * y into contrib[token, slot, row].  A warp takes six rows at a time,
// with their scales.
template <int NCI>
__device__ void down_items(const DigitArgs &a, uint8_t *xd, DTables &tb) {
  constexpr int kRows = 6;
  const int H = a.H, I = a.I, K = a.K, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __shared__ int32_t rows[kGR];
  bool bad = false;
  for_each_share(tb, tb.cost_d, H, a.down_w, [&](int ai, int j0, int j1, int r0, int r1) {
    const int e = tb.act_e[ai];
    const int8_t *Wd = tb.wp[e] + (size_t)2 * I * H;
    const float *Sd = tb.sp[e] + 2 * I;
    for (int rb = r0; rb < r1; rb += kGR) {
      const int nr = min(kGR, r1 - rb);
      __syncthreads();
      if (threadIdx.x < nr)
        rows[threadIdx.x] = tb.r_token[rb + threadIdx.x] * K + tb.r_slot[rb + threadIdx.x];
      __syncthreads();
      digitise_act<NCI>(a, rows, nr, xd, tb);
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
        float sd[kRows];
#pragma unroll
        for (int q = 0; q < kRows; ++q) sd[q] = Sd[min(jb + q, j1 - 1)];
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
              const float y = digits::down(my1[q], my2[q], tb.s1[lane], tb.s2[lane], sd[q]);
              bad |= !is_finite_f(y);
              a.contrib[(size_t)rows[lane] * H + j] = __fmul_rn(tb.r_gate[rb + lane], y);
            }
          }
        }
      }
    }
  });
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

// The layers of one launch; false when a barrier wait gave up.
template <int NCH, int NCI>
__device__ bool run_layers(const DigitArgs &a, DTables &tb, uint8_t *stage) {
  const int G = gridDim.x, T = a.T, K = a.K, R = T * K;
  const int warp = threadIdx.x >> 5;
  uint32_t nbar = 0;
  auto sync = [&]() {
    ++nbar;
    return grid_sync(a.bar, nbar * G, a.status, a.wait_cycles);
  };
  for (int l = 0; l < a.n_layers; ++l) {
    const FusedLayer L = a.layers[l];
    const bool first = l == 0;
    // the layer's expert pointers, read while the router runs
    for (int e = threadIdx.x; e < a.E; e += kDT) {
      tb.wp[e] = L.w_ptr[e];
      tb.sp[e] = L.s_ptr[e];
    }
    // stacked: x is the residual stream (in `out`), normalised while staged
    const float *xin = a.stacked ? a.out : a.h_in;
    const float *resid = a.stacked ? a.out : a.resid;
    if (first) {
      DigitArgs a0 = a;
      a0.sub_stamps = a.phase_ts != nullptr;
      router_phase(a0, L, xin, a.stacked != 0, reinterpret_cast<float *>(stage), tb);
    } else {
      router_phase(a, L, xin, a.stacked != 0, reinterpret_cast<float *>(stage), tb);
    }
    if (first) stamp(a, 1);
    if (!sync()) return false;
    if (first) stamp(a, 2);
    // S: selection
    if (T <= kDW) {
      if (warp < T) select_one(a, warp, tb.ids + warp * K, tb.gates + warp * K, tb);
      if (T == 1 && warp == 0) tables_single(a, tb);
      __syncthreads();
      if (blockIdx.x == 0)
        for (int r = threadIdx.x; r < R; r += kDT) {
          a.ids[r] = tb.ids[r];
          a.gates[r] = tb.gates[r];
        }
    } else {
      // one token per CTA (warp 0) while T <= G: each selection has an SM's
      // FP64 units and shared-memory bandwidth to itself
      for (int t = blockIdx.x + G * warp; t < T; t += G * kDW)
        select_one(a, t, a.ids + t * K, a.gates + t * K, tb);
      if (first) {
        __syncthreads();
        stamp(a, 12);
      }
      if (!sync()) return false;
      for (int r = threadIdx.x; r < R; r += kDT) {
        tb.ids[r] = __ldcg(a.ids + r);
        tb.gates[r] = __ldcg(a.gates + r);
      }
      __syncthreads();
    }
    if (first) stamp(a, 3);
    if (T > 1) build_tables(a, R, tb);
    if (first) stamp(a, 4);
    if (a.prefetch_down) prefetch_down(a, tb);
    gate_up_phase<NCH>(a, stage, tb);
    if (first) stamp(a, 5);
    if (first && a.phase_ts && threadIdx.x == 0) {
      // per-CTA end of gate/up (profiling): [16 + 2048 + c]
      unsigned long long t;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
      a.phase_ts[16 + 2048 + blockIdx.x] = t;
    }
    if (!sync()) return false;
    if (first) stamp(a, 6);
    if (a.stacked && l + 1 < a.n_layers && threadIdx.x == 0) {
      // the next layer's router rows head for L2 while this layer's down
      // phase runs: each CTA prefetches one 16-byte-aligned slice
      const FusedLayer &N = a.layers[l + 1];
      const size_t rb = (size_t)a.E * a.H * (N.router_dtype == kRouterBF16 ? 2 : 4);
      const size_t per = ((rb + gridDim.x - 1) / gridDim.x + 15) & ~size_t(15);
      const size_t o = per * blockIdx.x;
      if (o < rb && (reinterpret_cast<uintptr_t>(N.router) & 15) == 0)
        prefetch_l2(static_cast<const uint8_t *>(N.router) + o,
                    (uint32_t)(std::min(per, (rb - o + 15) & ~size_t(15))));
    }
    if (T == 1) {
      down_single<NCI>(a, resid, a.out, stage, tb);
    } else {
      down_items<NCI>(a, stage, tb);
      if (!sync()) return false;
      combine_phase(a, resid, a.out);
    }
    if (first) stamp(a, 7);
    if (a.stacked && l + 1 < a.n_layers && !sync()) return false;
  }
  if (blockIdx.x == 0 && a.ids_out)
    for (int r = threadIdx.x; r < R; r += kDT) {
      a.ids_out[r] = __ldcg(a.ids + r);
      a.gates_out[r] = __ldcg(a.gates + r);
    }
  return true;
}

// bar[0] counts barrier arrivals, bar[1] exits: the last CTA to leave --
// after every other CTA has passed all of its barriers, or given up --
// zeroes both, so the next launch needs no reset of its own.
template <int NCH, int NCI>
__global__ void __launch_bounds__(kDT, 2) digit_decode_kernel(DigitArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  DTables &tb = *reinterpret_cast<DTables *>(smem);
  uint8_t *stage = smem + kStageOff;
  stamp(a, 0);
  unsigned long long t_start = 0;
  if (a.phase_ts && threadIdx.x == 0) asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_start));
  run_layers<NCH, NCI>(a, tb, stage);
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(a.bar + 1, 1u) == gridDim.x - 1) {
      atomicExch(a.bar, 0u);
      atomicExch(a.bar + 1, 0u);
      __threadfence();
    }
    if (a.phase_ts) {
      // per-CTA start and end (profiling): [16 + 2 c], [16 + 2 c + 1]
      unsigned long long t_end;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_end));
      a.phase_ts[16 + 2 * blockIdx.x] = t_start;
      a.phase_ts[16 + 2 * blockIdx.x + 1] = t_end;
    }
  }
  stamp(a, 8);
}

size_t digit_smem_bytes(int H, int I) {
  const size_t router = (size_t)(kRTT + kRTE) * (H + kRowPad) * sizeof(float);
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
  DigitArgs a = a_in;
  a.router_async = a_in.router_async && a_in.H % 4 == 0;
  void *params[] = {&a};
  return cudaLaunchCooperativeKernel(fn, dim3(cached_grid), dim3(kDT), params, smem, s);
}

}  // namespace moe
