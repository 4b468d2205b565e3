// Fused decode: one cooperative, persistent launch runs a whole MoE layer --
// or a stack of layers with RMSNorm and residual between them -- for small
// token counts (decode batches).  Arithmetic is exactly that of the phased
// kernels (route_core.cuh, gemv_core.cuh), so results stay bit-identical to
// the CPU path; what changes is scheduling:
//
//   R  router logits, tasks of (<= 4 tokens x 4 experts, or x 1 expert when
//      tasks are scarce) over all CTAs; the CTA that completes the last task
//      of a token runs its softmax/top-k (per-token arrival counter, no
//      barrier);
//   -- grid barrier --
//   P  every CTA rebuilds the by-expert permutation in shared memory from the
//      routing (small: T*K <= 1024 routes), then issues bulk L2 prefetches for
//      the weight rows of all its gate/up and down items so HBM streams from
//      here on;
//   (single-token launches stream G and D weights through the TMA tile ring
//   of gemv_tiles.cuh; larger ones load them per thread)
//   G  gate/up GEMV items (expert segment x 32 rows) -> activations;
//   -- grid barrier --
//   D  down GEMV items (expert segment x 64 rows) -> gate-weighted
//      contributions;
//   -- grid barrier --
//   C  slot-ordered combine (single layer: spread over every thread; stacked:
//      one CTA per token, which also runs the next layer's RMSNorm) and, for
//      stacks, a barrier before the next layer's router.
//
// All CTAs are co-resident (cudaLaunchCooperativeKernel).  Every barrier wait
// is bounded: on expiry the CTA records kStatusTimeout and returns.
// Data produced by other CTAs of the launch is read through L2 (ld.cg).
#include <algorithm>

#include "gemv_core.cuh"
#include "gemv_tiles.cuh"
#include "kernels.h"
#include "route_core.cuh"

namespace moe {
namespace {

using namespace gemv;

constexpr int kFT = 256;          // threads per CTA (8 warps)
constexpr int kRTT = 4;           // router task: tokens
constexpr int kRTE = 4;           // router task: experts
constexpr int kRowPad = 8;        // floats of padding per staged router row

struct Tables {
  uint64_t tile_full[kTileStages];  // weight-tile ring mbarriers
  int32_t seg_off[kMaxExperts + 1];
  int32_t active[kMaxExperts];
  int32_t run[kMaxExperts];
  int32_t n_active;
  int32_t last[kRTT];
  int32_t r_token[kFusedMaxRoutes];
  int32_t r_slot[kFusedMaxRoutes];
  float r_gate[kFusedMaxRoutes];
  int32_t wcnt[kFT / 32][kMaxExperts];
};

// Grid barrier; each wait gives up after `limit` SM clock cycles
// (FusedArgs::wait_cycles, the handle's wait bound) and records
// kStatusTimeout.
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

__device__ __forceinline__ void stamp(const FusedArgs &a, int idx) {
  if (a.phase_ts && blockIdx.x == 0 && threadIdx.x == 0) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    a.phase_ts[idx] = t;
  }
}

__device__ __forceinline__ void prefetch_l2(const void *p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// R: router logits for task tiles of up to kRTT tokens x RE experts, then
// the last-arriving CTA of each token runs its selection.  RE = kRTE when
// that gives every CTA work; with fewer tasks than half the grid (small T)
// RE = 1, which spreads the router rows over 4x more CTAs and shortens each
// task's staging and dot.
__device__ void router_phase(const FusedArgs &a, const FusedLayer &L, const float *hin,
                             float *stage, Tables &tb, SelectScratch *sel) {
  const int T = a.T, E = a.E, H = a.H, tid = threadIdx.x;
  const int TT = min(T, kRTT);
  const int ntt = (T + TT - 1) / TT;
  const int RE = ntt * ((E + kRTE - 1) / kRTE) * 2 < (int)gridDim.x ? 1 : kRTE;
  const int nte = (E + RE - 1) / RE;
  const int tasks = ntt * nte;
  const int full = H / 8;
  // staged rows are kRowPad floats longer than H, so the 4 expert rows a
  // warp reads at the same column fall in different banks
  const int RS = H + kRowPad;
  // Router::select_top_k (src/router.rs:59-62) uses a plain sequential dot
  const bool seq = a.route_mode == kRouteTopkSoftmax && L.router_dtype == kRouterF32;
  for (int task = blockIdx.x; task < tasks; task += gridDim.x) {
    const int t0 = (task / nte) * TT, e0 = (task % nte) * RE;
    const int nt = min(TT, T - t0);
    // stage rows: [0, TT) tokens, [TT, TT + RE) experts
    const int total = (TT + RE) * H;
    bool bad = false;
    if (a.router_async) {
      // 16-byte cp.async copies, all issued before the single wait: one
      // memory round trip for the whole task.
      const int q = H / 4;
      for (int i = tid; i < (TT + RE) * q; i += kFT) {
        const int r = i / q, c = (i % q) * 4;
        float *dst = stage + (size_t)r * RS + c;
        const float *src = nullptr;
        if (r < TT) {
          if (r < nt) src = hin + (size_t)(t0 + r) * H + c;
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
      __syncthreads();
      for (int i = tid; i < nt * H; i += kFT)
        if (!is_finite_f(stage[(size_t)(i / H) * RS + i % H])) bad = true;
    } else {
      constexpr int kB = 8;
      for (int base = 0; base < total; base += kFT * kB) {
        float v[kB];
#pragma unroll
        for (int k = 0; k < kB; ++k) {
          const int i = base + k * kFT + tid;
          v[k] = 0.0f;
          if (i < total) {
            const int r = i / H, c = i % H;
            if (r < TT) {
              if (r < nt) v[k] = __ldcg(hin + (size_t)(t0 + r) * H + c);
            } else if (e0 + r - TT < E) {
              v[k] = load_w(L.router, L.router_dtype, (size_t)(e0 + r - TT) * H + c);
            }
          }
        }
#pragma unroll
        for (int k = 0; k < kB; ++k) {
          const int i = base + k * kFT + tid;
          if (i < total) {
            stage[(size_t)(i / H) * RS + i % H] = v[k];
            if (i < TT * H && !is_finite_f(v[k])) bad = true;
          }
        }
      }
    }
    if (bad) set_status(a.status, kStatusNonFinite);
    __syncthreads();
    // 8 lanes per (token, expert) pair.  The lane fold below is a warp
    // shuffle, so whole warps enter: lanes past the last pair compute on row
    // 0 and write nothing (8 * TT * RE is not a multiple of 32 when RE = 1).
    const int npairs = TT * RE;
    if (tid < ((8 * npairs + 31) & ~31)) {
      const int lane = tid & 7, pair = tid >> 3;
      const bool live = pair < npairs;
      const int ti = live ? pair / RE : 0, ei = live ? pair % RE : 0;
      const float *hs = stage + (size_t)ti * RS;
      const float *w = stage + (size_t)(TT + ei) * RS;
      float logit;
      if (seq) {
        float acc = -0.0f;  // src/router.rs:59-62, Rust's f32 Sum folds from -0.0
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
      const int t = t0 + ti, e = e0 + ei;
      if (live && lane == 0 && ti < nt && e < E) {
        a.logits[(size_t)t * E + e] = logit;
        if (!is_finite_f(logit)) set_status(a.status, kStatusNonFinite);
      }
    }
    __syncthreads();
    if (tid == 0) {
      __threadfence();
      for (int ti = 0; ti < nt; ++ti)
        tb.last[ti] = atomicAdd(&a.tok_cnt[t0 + ti], 1u) == (uint32_t)(nte - 1);
      __threadfence();
    }
    __syncthreads();
    const int warp = tid >> 5;
    if (warp < nt && tb.last[warp]) {
      const int t = t0 + warp;
      select_token(a.logits + (size_t)t * E, E, a.K, a.norm, a.route_mode,
                   a.ids + (size_t)t * a.K, a.gates + (size_t)t * a.K, nullptr, sel[warp],
                   a.status);
      if ((tid & 31) == 0) a.tok_cnt[t] = 0;  // ready for the next layer / call
    }
    __syncthreads();
  }
}

// P: stable counting sort of the T*K routes by expert, in shared memory
// (src/olmoe.rs:3474-3480: experts ascending, tokens ascending inside).
__device__ void build_tables(const FusedArgs &a, Tables &tb) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int E = a.E, R = a.T * a.K;
  for (int e = tid; e < E; e += kFT) tb.run[e] = 0;
  for (int i = tid; i < (kFT / 32) * kMaxExperts; i += kFT) (&tb.wcnt[0][0])[i] = 0;
  __syncthreads();
  for (int r = tid; r < R; r += kFT) {
    const uint32_t e = __ldcg(a.ids + r);
    if (e < (uint32_t)E) atomicAdd(&tb.run[e], 1);
  }
  __syncthreads();
  if (warp == 0) {
    // exclusive prefix of the counts and the ascending list of active
    // experts, 32 experts per round
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
  for (int base = 0; base < R; base += kFT) {
    const int r = base + tid;
    const bool valid = r < R;
    const uint32_t e = valid ? __ldcg(a.ids + r) : 0xFFFFFFFFu;
    const bool ok = valid && e < (uint32_t)E;
    const unsigned mask = __match_any_sync(0xffffffffu, ok ? e : 0xFFFFFFFFu);
    const int intra = __popc(mask & ((1u << lane) - 1u));
    if (ok && intra == 0) tb.wcnt[warp][e] = __popc(mask);
    __syncthreads();
    if (ok) {
      int pos = tb.run[e] + intra;
      for (int w = 0; w < warp; ++w) pos += tb.wcnt[w][e];
      tb.r_token[pos] = r / a.K;
      tb.r_slot[pos] = r % a.K;
      tb.r_gate[pos] = __ldcg(a.gates + r);
    }
    __syncthreads();
    for (int ee = tid; ee < E; ee += kFT) {
      int tot = 0;
      for (int w = 0; w < kFT / 32; ++w) {
        tot += tb.wcnt[w][ee];
        tb.wcnt[w][ee] = 0;
      }
      tb.run[ee] += tot;
    }
    __syncthreads();
  }
}

// Per-thread weight loads stream in register batches of kDecodePF
// chunk-steps, two in flight.  Deeper batches did not help: on B200 a
// phase is bound by the exact FMA chains' issue rate (about 0.7 us per four
// chunk-steps, with or without the weights in L2) and by the grid barriers,
// not by the loads -- INT4 (half the bytes) runs at INT8 speed, and an
// 8-deep INT4 batch made the multi-route variant slower.
constexpr int kDecodePF = 4;
constexpr int kGURowsItem = kGURowsPerWarp * (kFT / 32);  // 32
constexpr int kDNRowsItem = kDNRowsPerWarp * (kFT / 32);  // 64
static_assert(kGURowsItem == kTileGURows && kDNRowsItem == kTileDNRows,
              "a decode work item is one weight tile");
constexpr int kTensorMapBytes = 128;  // sizeof(CUtensorMap)

// kTiles: weights stream through the TMA tile ring (every layer of the
// launch has tile maps); otherwise each thread loads its own weights.
template <bool kVec, bool kMulti, int kQ, bool kTiles>
__device__ void expert_phases(const FusedArgs &a, const FusedLayer &L, const float *hin,
                              float *stage, Tables &tb, TileRing &rg, uint32_t &nbar,
                              bool &alive) {
  const int H = a.H, I = a.I, G = gridDim.x;
  const int nseg = tb.n_active;
  const int nb_gu = (I + kGURowsItem - 1) / kGURowsItem;
  const int nb_dn = (H + kDNRowsItem - 1) / kDNRowsItem;
  // Bulk L2 prefetch of the weight blocks this CTA will stream: all of them
  // up front when the layer's active experts fit comfortably in L2 (batch-1
  // decode), otherwise two items ahead of use (larger batches would evict
  // their own prefetches).
  const size_t hb = (size_t)H * kQ / 8, ib = (size_t)I * kQ / 8;  // bytes per row
  const bool all_up_front = (size_t)nseg * 3 * I * hb <= ((size_t)64 << 20);
  const char *map_gu = static_cast<const char *>(L.tmaps);
  const char *map_dn = map_gu + kTensorMapBytes;
  // Scale slices go with their weight blocks when whole 16-byte runs
  // (full 32- or 64-row items of 16-byte aligned scale vectors).
  auto pf_gu = [&](int item) {
    if (threadIdx.x != 0 || !L.prefetch_ok || item >= nseg * nb_gu) return;
    const int e = tb.active[item / nb_gu], row0 = (item % nb_gu) * kGURowsItem;
    const int rows = min(kGURowsItem, I - row0);
    const int8_t *W = L.w_ptr[e];
    prefetch_l2(W + (size_t)row0 * hb, (uint32_t)(rows * hb));
    prefetch_l2(W + (size_t)(I + row0) * hb, (uint32_t)(rows * hb));
    const float *S = L.s_ptr[e];
    if (rows == kGURowsItem && I % 4 == 0 && ((uintptr_t)S & 15) == 0) {
      prefetch_l2(S + row0, kGURowsItem * sizeof(float));
      prefetch_l2(S + I + row0, kGURowsItem * sizeof(float));
    }
  };
  auto pf_dn = [&](int item) {
    if (threadIdx.x != 0 || !L.prefetch_ok || item >= nseg * nb_dn) return;
    const int e = tb.active[item / nb_dn], row0 = (item % nb_dn) * kDNRowsItem;
    const int rows = min(kDNRowsItem, H - row0);
    prefetch_l2(L.w_ptr[e] + 2 * (size_t)I * hb + (size_t)row0 * ib, (uint32_t)(rows * ib));
    const float *S = L.s_ptr[e];
    if (rows == kDNRowsItem && I % 2 == 0 && ((uintptr_t)S & 15) == 0)
      prefetch_l2(S + 2 * I + row0, kDNRowsItem * sizeof(float));
  };
  // The tile ring overlaps the router's staging rows: every thread orders
  // its generic-proxy writes there before the ring's TMA writes (thread 0
  // issues them after the barrier).  Within the expert phases only TMA
  // writes the ring.
  if constexpr (kTiles) {
    tma::fence_proxy_async_smem();
    __syncthreads();
  }
  if (all_up_front) {
    for (int item = blockIdx.x; item < nseg * nb_gu; item += G) pf_gu(item);
    for (int item = blockIdx.x; item < nseg * nb_dn; item += G) pf_dn(item);
  } else {
    pf_gu(blockIdx.x);
    pf_gu(blockIdx.x + G);
  }
  for (int item = blockIdx.x; item < nseg * nb_gu; item += G) {
    if (!all_up_front) {
      pf_gu(item + 2 * G);
      // the first down items of this CTA go out during its last gate/up item
      if (item + G >= nseg * nb_gu) {
        pf_dn(blockIdx.x);
        pf_dn(blockIdx.x + G);
      }
    }
    const int e = tb.active[item / nb_gu];
    const int r0 = tb.seg_off[e], r1 = tb.seg_off[e + 1];
    const int row0 = (item % nb_gu) * kGURowsItem;
    if constexpr (kTiles) {
      if (rg.dead) continue;
      const bool ok =
          (!kMulti || r1 - r0 == 1)
              ? gate_up_tile_item<1, kQ>(rg, map_gu, e, L.s_ptr[e], H, I, row0, r0, r1,
                                         tb.r_token, hin, stage, a.act)
              : gate_up_tile_item<kTG, kQ>(rg, map_gu, e, L.s_ptr[e], H, I, row0, r0, r1,
                                           tb.r_token, hin, stage, a.act);
      if (!ok) set_status(a.status, kStatusTimeout);
    } else if (!kMulti || r1 - r0 == 1)
      gate_up_item<kVec, 1, kDecodePF, kQ>(L.w_ptr[e], L.s_ptr[e], H, I, row0, r0,
                                                       r1, tb.r_token, hin, stage, a.act);
    else
      gate_up_item<kVec, 4, kDecodePF, kQ>(L.w_ptr[e], L.s_ptr[e], H, I, row0, r0,
                                                      r1, tb.r_token, hin, stage, a.act);
  }
  ++nbar;
  if (!grid_sync(a.bar, nbar * G, a.status, a.wait_cycles)) {
    alive = false;
    return;
  }
  stamp(a, 2);
  bool good = true;
  for (int item = blockIdx.x; item < nseg * nb_dn; item += G) {
    if (!all_up_front) pf_dn(item + 2 * G);
    const int e = tb.active[item / nb_dn];
    const int r0 = tb.seg_off[e], r1 = tb.seg_off[e + 1];
    const int row0 = (item % nb_dn) * kDNRowsItem;
    auto emit = [&](int r, int row, float y) {
      a.contrib[((size_t)tb.r_token[r] * a.K + tb.r_slot[r]) * H + row] = __fmul_rn(tb.r_gate[r], y);
    };
    if constexpr (kTiles) {
      if (rg.dead) continue;
      const bool ok =
          (!kMulti || r1 - r0 == 1)
              ? down_tile_item<1, kQ>(rg, map_dn, e, L.s_ptr[e], H, I, row0, r0, r1, a.act,
                                      stage, good, emit)
              : down_tile_item<kTG, kQ>(rg, map_dn, e, L.s_ptr[e], H, I, row0, r0, r1, a.act,
                                        stage, good, emit);
      if (!ok) set_status(a.status, kStatusTimeout);
    } else if (!kMulti || r1 - r0 == 1)
      good &= down_item<kVec, 1, kDecodePF, kQ>(L.w_ptr[e], L.s_ptr[e], H, I,
                                                            row0, r0, r1, a.act, stage, emit);
    else
      good &= down_item<kVec, 4, kDecodePF, kQ>(L.w_ptr[e], L.s_ptr[e], H, I,
                                                           row0, r0, r1, a.act, stage, emit);
  }
  if (!good) set_status(a.status, kStatusNonFinite);
  ++nbar;
  if (!grid_sync(a.bar, nbar * G, a.status, a.wait_cycles)) alive = false;
  stamp(a, 3);
}

// RMSNorm of token row x into h (src/backend.rs:341-359; gain w, or 1 when
// null): warp 0, lanes 0..7 run the 8-lane sum of squares; all threads scale.
__device__ void rms_row(const float *x, const float *w, float *h, int H, float eps, float *red,
                        uint32_t *status) {
  const int tid = threadIdx.x;
  if (tid < 32) {
    float acc = 0.0f;
    const int full = H / 8;
    if (tid < 8)
      for (int c = 0; c < full; ++c) {
        const float v = __ldcg(x + 8 * c + tid);
        acc = __fadd_rn(acc, __fmul_rn(v, v));
      }
    float s = -0.0f;
#pragma unroll
    for (int l = 0; l < 8; ++l) s = __fadd_rn(s, __shfl_sync(0xffffffffu, acc, l));
    for (int i = full * 8; i < H; ++i) {
      const float v = __ldcg(x + i);
      s = __fadd_rn(s, __fmul_rn(v, v));
    }
    if (tid == 0) {
      const float scale = __fsqrt_rn(__fadd_rn(__fdiv_rn(s, (float)H), eps));
      red[0] = __fdiv_rn(1.0f, scale);
    }
  }
  __syncthreads();
  const float inv = red[0];
  bool bad = false;
  for (int j = tid; j < H; j += kFT) {
    const float v = __ldcg(x + j);
    const float o = __fmul_rn(__fmul_rn(v, inv), w ? w[j] : 1.0f);
    bad |= !is_finite_f(v) || !is_finite_f(o);
    h[j] = o;
  }
  if (bad) set_status(status, kStatusNonFinite);
  __syncthreads();
}

// Shared-memory carve-up; every region starts on a 128-byte boundary (the
// staging area is read and written with float4).
constexpr size_t align128(size_t n) { return (n + 127) & ~size_t(127); }
constexpr size_t kSelOff = align128(sizeof(Tables));
constexpr size_t kStageOff = align128(kSelOff + 8 * sizeof(SelectScratch));

// kQ: the weight format of every layer in the launch (8 or 4 bits).
template <bool kVec, bool kMulti, int kQ, bool kTiles>
__global__ void __launch_bounds__(kFT, kMulti ? 1 : 2) fused_decode_kernel(FusedArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  Tables &tb = *reinterpret_cast<Tables *>(smem);
  SelectScratch *sel = reinterpret_cast<SelectScratch *>(smem + kSelOff);
  float *stage = reinterpret_cast<float *>(smem + kStageOff);
  __shared__ float red[1];
  const int G = gridDim.x, T = a.T, H = a.H, K = a.K;
  uint32_t nbar = 0;
  bool alive = true;
  const float *hin = a.h_in;
  stamp(a, 0);
  if (threadIdx.x == 0) {
    for (int i = 0; i < kTileStages; ++i) tma::mbar_init(&tb.tile_full[i], 1);
    tma::fence_mbar_init();
  }
  __syncthreads();
  const uintptr_t ring_at =
      reinterpret_cast<uintptr_t>(stage) + (size_t)kTG * (size_t)max(H, a.I) * sizeof(float);
  TileRing rg{reinterpret_cast<uint8_t *>((ring_at + 1023) & ~uintptr_t(1023)), tb.tile_full, 0u,
              false};
  if (a.stacked) {
    for (int t = blockIdx.x; t < T; t += G)
      rms_row(a.out + (size_t)t * H, a.layers[0].norm_w, a.hbuf + (size_t)t * H, H, a.eps, red,
              a.status);
    ++nbar;
    if (!grid_sync(a.bar, nbar * G, a.status, a.wait_cycles)) return;
    hin = a.hbuf;
  }
  for (int l = 0; l < a.n_layers; ++l) {
    const FusedLayer L = a.layers[l];
    // the tile maps' descriptors are fetched while the router runs
    if (kTiles && threadIdx.x == 0) {
      asm volatile("prefetch.tensormap [%0];" ::"l"(L.tmaps) : "memory");
      asm volatile("prefetch.tensormap [%0];" ::"l"(static_cast<const char *>(L.tmaps) +
                                                   kTensorMapBytes)
                   : "memory");
    }
    router_phase(a, L, hin, stage, tb, sel);
    ++nbar;
    if (!grid_sync(a.bar, nbar * G, a.status, a.wait_cycles)) return;
    if (l == 0) stamp(a, 1);
    build_tables(a, tb);
    expert_phases<kVec, kMulti, kQ, kTiles>(a, L, hin, stage, tb, rg, nbar, alive);
    // A dead ring (a stage wait gave up; kStatusTimeout is set) may still
    // have a copy in flight into its shared memory, which the next layer's
    // router staging overlaps: this CTA stops here, and the others' bounded
    // barrier waits end the launch.
    if (!alive || rg.dead) return;
    if (!a.stacked) {
      // C: out = resid + contrib[., 0] + ... + contrib[., K-1] (slot order)
      bool bad = false;
      for (size_t i = blockIdx.x * (size_t)kFT + threadIdx.x; i < (size_t)T * H;
           i += (size_t)G * kFT) {
        const size_t t = i / H, j = i % H;
        float acc = a.resid ? a.resid[i] : 0.0f;
        for (int k = 0; k < K; ++k) acc = __fadd_rn(acc, __ldcg(a.contrib + (t * K + k) * H + j));
        bad |= !is_finite_f(acc);
        a.out[i] = acc;
      }
      if (bad) set_status(a.status, kStatusNonFinite);
      if (blockIdx.x == 0 && a.ids_out)
        for (int r = threadIdx.x; r < T * K; r += kFT) {
          a.ids_out[r] = __ldcg(a.ids + r);
          a.gates_out[r] = __ldcg(a.gates + r);
        }
    } else {
      // C (stacked): x += contributions in slot order, then the next
      // layer's RMSNorm of this token.
      for (int t = blockIdx.x; t < T; t += G) {
        float *x = a.out + (size_t)t * H;
        bool bad = false;
        for (int j = threadIdx.x; j < H; j += kFT) {
          float acc = __ldcg(x + j);
          for (int k = 0; k < K; ++k)
            acc = __fadd_rn(acc, __ldcg(a.contrib + ((size_t)t * K + k) * H + j));
          bad |= !is_finite_f(acc);
          x[j] = acc;
        }
        if (bad) set_status(a.status, kStatusNonFinite);
        __syncthreads();
        if (l + 1 < a.n_layers)
          rms_row(x, a.layers[l + 1].norm_w, a.hbuf + (size_t)t * H, H, a.eps, red, a.status);
      }
      if (l + 1 < a.n_layers) {
        ++nbar;
        if (!grid_sync(a.bar, nbar * G, a.status, a.wait_cycles)) return;
      }
    }
  }
  __syncthreads();
  stamp(a, 4);
}

size_t fused_smem_bytes(int H, int I, bool tiles) {
  const size_t router = (size_t)(kRTT + kRTE) * (H + kRowPad) * sizeof(float);
  // token rows, then (tile variants) the weight-tile ring on a 1024-byte
  // boundary
  const size_t gemv = (size_t)kTG * std::max(H, I) * sizeof(float) +
                      (tiles ? 1024 + kTileRingBytes : 0);
  return kStageOff + std::max(router, gemv);
}

}  // namespace

bool fused_decode_supported(int T, int H, int I, int E, int K) {
  return T >= 1 && T * K <= kFusedMaxRoutes && H <= kFusedMaxH && I <= kFusedMaxH &&
         E <= kMaxExperts && fused_smem_bytes(H, I, true) <= 113 * 1024;
}

cudaError_t launch_fused_decode(const FusedArgs &a, int vec, int sm_count, uint32_t *bar,
                                cudaStream_t s) {
  const bool multi = a.T > 1;
  const bool tiles = a.tiles != 0 && !multi;
  const size_t smem = fused_smem_bytes(a.H, a.I, tiles);
  // vector loads need 8-byte weight rows (H, I multiples of 8) on top of the
  // caller's pointer-alignment check
  vec = vec && a.H % 8 == 0 && a.I % 8 == 0;
  // A single token per call means every expert segment holds one route:
  // the lighter single-route variant then fits two CTAs per SM.
  const void *fn;
  // Weight tiles serve single-token launches, where they measured faster
  // than per-thread loads (C0 47.7 vs 51.0 us per layer on B200).  With
  // several tokens each CTA runs several short items and restarting the
  // ring per item cost more than it saved (C2 4.28 vs 3.88 ms), so those
  // launches keep per-thread loads.  The tile variants stage their inputs
  // with 16-byte loads (the caller checked the alignment).
  if (tiles) {
    fn = a.int4 ? (const void *)fused_decode_kernel<true, false, 4, true>
                : (const void *)fused_decode_kernel<true, false, 8, true>;
  } else if (a.int4) {
    fn = vec ? (multi ? (const void *)fused_decode_kernel<true, true, 4, false>
                      : (const void *)fused_decode_kernel<true, false, 4, false>)
             : (multi ? (const void *)fused_decode_kernel<false, true, 4, false>
                      : (const void *)fused_decode_kernel<false, false, 4, false>);
  } else {
    fn = vec ? (multi ? (const void *)fused_decode_kernel<true, true, 8, false>
                      : (const void *)fused_decode_kernel<true, false, 8, false>)
             : (multi ? (const void *)fused_decode_kernel<false, true, 8, false>
                      : (const void *)fused_decode_kernel<false, false, 8, false>);
  }
  // The attribute and occupancy query run once per (device, variant, size).
  static thread_local int cached_dev = -1, cached_vec = -1, cached_grid = 0, cached_multi = -1,
                          cached_q = -1, cached_tiles = -1;
  static thread_local size_t cached_smem = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev != cached_dev || vec != cached_vec || smem != cached_smem ||
      (int)multi != cached_multi || a.int4 != cached_q || (int)tiles != cached_tiles) {
    cudaError_t e =
        cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kFT, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorLaunchOutOfResources;
    cached_dev = dev;
    cached_vec = vec;
    cached_smem = smem;
    cached_multi = multi;
    cached_q = a.int4;
    cached_tiles = tiles;
    cached_grid = std::min(per_sm, 2) * sm_count;
  }
  cudaError_t e = cudaMemsetAsync(bar, 0, sizeof(uint32_t), s);
  if (e != cudaSuccess) return e;
  FusedArgs args = a;
  args.bar = bar;
  args.router_async = a.router_async && a.H % 4 == 0;
  void *params[] = {&args};
  return cudaLaunchCooperativeKernel(fn, dim3(cached_grid), dim3(kFT), params, smem, s);
}

}  // namespace moe
