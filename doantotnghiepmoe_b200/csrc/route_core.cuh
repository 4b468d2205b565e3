// Warp-level pieces of the router shared by route.cu and the fused decode
// kernel.  Reference semantics: src/backend.rs:375-389 (softmax),
// src/olmoe.rs:2595-2621 (top-k, ties to the lower index, normalizer),
// src/router.rs:84-103 (the top-k-then-softmax variant).
#pragma once

#include "common.cuh"
#include "kernels.h"

namespace moe {

__device__ __forceinline__ float load_w(const void *W, int dtype, size_t idx) {
  if (dtype == kRouterBF16) {
    const uint16_t v = reinterpret_cast<const uint16_t *>(W)[idx];
    return __uint_as_float((uint32_t)v << 16);
  }
  return reinterpret_cast<const float *>(W)[idx];
}

struct SelectScratch {
  float ex[kMaxExperts];
  float sel_v[kMaxTopK];
  uint32_t sel_i[kMaxTopK];
};

// Softmax over all E logits in index order (mode kRouteSoftmaxTopk) or the
// raw scores (kRouteTopkSoftmax), then K rounds of a warp-wide argmax on
// (f32::total_cmp key, lower index first).  Called by all 32 lanes of a warp.
// lg may live in global memory written by other CTAs: it is read through L2.
// kPer = candidates per lane (E <= 32 * kPer); select_token below picks it.
template <int kPer>
__device__ __forceinline__ void select_token_t(const float *lg, int E, int K, int norm_topk_prob,
                                               int mode, uint32_t *ids, float *gates,
                                               float *probs, SelectScratch &sc,
                                               uint32_t *status) {
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
        sc.ex[e] = v[j];
      }
    }
    __syncwarp();
    float sum = 0.0f;
    if (lane == 0) {
      // sequential in index order; loads batched ahead of the dependent adds
      sum = -0.0f;
      int e = 0;
      for (; e + 8 <= E; e += 8) {
        float v8[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v8[j] = sc.ex[e + j];
#pragma unroll
        for (int j = 0; j < 8; ++j) sum = __fadd_rn(sum, v8[j]);
      }
      for (; e < E; ++e) sum = __fadd_rn(sum, sc.ex[e]);
    }
    sum = __shfl_sync(0xffffffffu, sum, 0);
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int e = lane + 32 * j;
      if (e < E) {
        v[j] = __fdiv_rn(v[j], sum);
        if (probs) probs[e] = v[j];
      }
    }
  } else {
    // partial_cmp treats -0.0 == +0.0; canonicalise zero so the total-order
    // key ties them (and the lower index wins, as in the reference sort).
#pragma unroll
    for (int j = 0; j < kPer; ++j)
      if (v[j] == 0.0f) v[j] = 0.0f;
  }
  // Each round: every lane takes its best remaining candidate (its candidates
  // run in ascending expert order, so a strict '>' keeps the lower index on a
  // tie), one warp max-reduction finds the winning key, one min-reduction
  // picks the lowest expert index among the lanes holding it.
  uint32_t taken = 0;  // bit j set when candidate j of this lane was selected
  for (int k = 0; k < K; ++k) {
    uint32_t bk = 0;
    int bj = -1;
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int e = lane + 32 * j;
      if (e < E && !(taken & (1u << j))) {
        const uint32_t key = total_order_u32(v[j]);
        if (bj < 0 || key > bk) {
          bk = key;
          bj = j;
        }
      }
    }
    const uint32_t mx = __reduce_max_sync(0xffffffffu, bj >= 0 ? bk : 0u);
    const uint32_t cand = (bj >= 0 && bk == mx) ? (uint32_t)(lane + 32 * bj) : 0xFFFFFFFFu;
    const uint32_t e = __reduce_min_sync(0xffffffffu, cand);
    if ((int)(e & 31) == lane) {
      const int j = (int)(e >> 5);
      taken |= 1u << j;
      float val = 0.0f;
#pragma unroll
      for (int jj = 0; jj < kPer; ++jj)
        if (jj == j) val = v[jj];
      sc.sel_v[k] = val;
      sc.sel_i[k] = e;
    }
    __syncwarp();
  }
  if (lane == 0) {
    if (mode == kRouteSoftmaxTopk) {
      float norm = 1.0f;
      if (norm_topk_prob) {
        norm = -0.0f;
        for (int k = 0; k < K; ++k) norm = __fadd_rn(norm, sc.sel_v[k]);
      }
      for (int k = 0; k < K; ++k) {
        ids[k] = sc.sel_i[k];
        gates[k] = __fdiv_rn(sc.sel_v[k], norm);
        if (sc.sel_i[k] >= (uint32_t)E) set_status(status, kStatusBadRoute);
      }
    } else {
      const float mx = sc.sel_v[0];
      float total = -0.0f;
      float ex[kMaxTopK];
      for (int k = 0; k < K; ++k) {
        ex[k] = expf_ref(__fsub_rn(sc.sel_v[k], mx));
        total = __fadd_rn(total, ex[k]);
      }
      for (int k = 0; k < K; ++k) {
        ids[k] = sc.sel_i[k];
        gates[k] = __fdiv_rn(ex[k], total);
      }
    }
  }
  __syncwarp();
}

__device__ __forceinline__ void select_token(const float *lg, int E, int K, int norm_topk_prob,
                                             int mode, uint32_t *ids, float *gates, float *probs,
                                             SelectScratch &sc, uint32_t *status) {
  if (E <= 64)
    select_token_t<2>(lg, E, K, norm_topk_prob, mode, ids, gates, probs, sc, status);
  else if (E <= 128)
    select_token_t<4>(lg, E, K, norm_topk_prob, mode, ids, gates, probs, sc, status);
  else
    select_token_t<kMaxExperts / 32>(lg, E, K, norm_topk_prob, mode, ids, gates, probs, sc,
                                     status);
}

}  // namespace moe
