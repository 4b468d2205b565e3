// Streaming decode: one cooperative, persistent launch runs a MoE layer (or a
// stack of layers with RMSNorm and residual between them) for decode-sized
// batches, laid out so that HBM streams the active experts' weights without
// gaps.  Arithmetic is the reference's, operation for operation (the same
// 8-lane router chains, softmax/top-k, 4-bank x 8-lane FMA chains, SiLU and
// slot-ordered combine as route_core.cuh / gemv_core.cuh), so results are
// bit-identical to the CPU path; only the schedule differs.
//
// Per layer:
//   R  Router logits in tasks of (TT tokens x TE experts) spread over the
//      CTAs.  A task stages its rows in shared memory (cp.async) and runs the
//      8-lane chains; a global task counter tells every CTA when all logits
//      exist.  In a stack the task first waits until the previous layer is
//      fully combined and runs the RMSNorm of its token rows itself.
//   S  Every CTA runs softmax/top-k for all tokens (a warp per token) and the
//      stable by-expert permutation in its own shared memory: no second round
//      trip through global memory.
//   W  Routes are cut into segments (one expert, up to TG of its routes).  The
//      gate/up rows of all segments, then their down rows, form two linear
//      work lists split evenly over the CTAs; a CTA walks its share as windows
//      of up to 128 weight rows.  A window is streamed column block by column
//      block (256 bytes of each of its rows per stage) through a ring of
//      shared-memory slots.  A thread owns one (row, bank) FMA chain for the
//      whole window and itself copies (cp.async, L2 evict-first) exactly the
//      bytes that chain reads, ring-depth - 1 stages ahead: each SM keeps
//      ~100 KB of weights in flight and no barrier sits between copy and use.
//      Accumulators stay in registers across stages.  The copies run ahead across window and gate/up -> down
//      boundaries: down weights are on chip before the activations they
//      multiply exist.
//   D  A down window first waits (bounded) on the per-segment counters of the
//      gate/up rows it needs, then reads the activations through L2 and writes
//      gate-weighted contributions.  Per-row-block counters let the CTA that
//      completes a block of rows combine it in slot order: there is no grid
//      barrier anywhere in the layer.
//
// Global counters come in two sets; launch n uses set n % 2 and zeroes the
// other set for launch n + 1, so a launch that gave up on a wait never leaves
// dirty counters behind.  Every wait is bounded; on expiry the CTA records
// kStatusTimeout, waits for its own copies and returns.
#include <algorithm>
#include <cstdio>

#include "gemv_core.cuh"
#include "kernels.h"
#include "route_core.cuh"

namespace moe {
namespace {

constexpr int kST = 512;                     // threads per CTA (16 warps, one CTA per SM)
constexpr int kCB = 256;                     // weight columns (bytes) per stage
constexpr int kPitch = kCB + 16;             // 16-byte skew per row: 8 rows read
                                             // conflict-free
constexpr int kWinRows = 128;                // weight rows per window (8 per warp)
constexpr int kWinPairs = kWinRows / 2;      // gate/up pairs per window
constexpr int kSlotBytes = kWinRows * kPitch;
constexpr int kXBytes = 64 * 1024;           // staged input rows of a window (<= 2 TG rows)
constexpr int kMaxNS = 8;                    // ring slots
constexpr int kBR = 64;                      // combine row block
constexpr long long kWaitCycles = 2000000000LL;  // ~1 s

// Counter words of one set (see kStreamCtrWords in kernels.h).
constexpr int kCtrLogit = 0;                 // router tasks done (launch-monotonic)
constexpr int kCtrComb = 1;                  // row blocks combined (launch-monotonic)
constexpr int kCtrSel = 2;                   // CTAs done selecting (launch-monotonic)
constexpr int kCtrGu = 32;                   // [kFusedMaxRoutes] gate/up rows per segment
constexpr int kCtrBlk = kCtrGu + kFusedMaxRoutes;  // [kFusedMaxH / kBR] (route,row) per block
static_assert(kCtrBlk + kFusedMaxH / kBR <= kStreamCtrWords, "counter set size");

__device__ __forceinline__ uint32_t su32(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(su32(dst)), "l"(src) : "memory");
}
// 8-byte copy into shared memory through L1, marked evict-first in L2: the
// weights stream once, so they should not push the kernel's code, the
// routers or the activations out of L2.
__device__ __forceinline__ void cp_async8_stream(void *dst, const void *src, uint64_t pol) {
  asm volatile("cp.async.ca.shared.global.L2::cache_hint [%0], [%1], 8, %2;" ::"r"(su32(dst)),
               "l"(src), "l"(pol)
               : "memory");
}
__device__ __forceinline__ uint64_t evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_all;" ::: "memory");
}
// Wait until at most n of this thread's most recent copy groups are pending.
__device__ __forceinline__ void cp_async_wait_pending(int n) {
  switch (n) {
    case 0: asm volatile("cp.async.wait_group 0;" ::: "memory"); break;
    case 1: asm volatile("cp.async.wait_group 1;" ::: "memory"); break;
    case 2: asm volatile("cp.async.wait_group 2;" ::: "memory"); break;
    case 3: asm volatile("cp.async.wait_group 3;" ::: "memory"); break;
    case 4: asm volatile("cp.async.wait_group 4;" ::: "memory"); break;
    case 5: asm volatile("cp.async.wait_group 5;" ::: "memory"); break;
    default: asm volatile("cp.async.wait_group 6;" ::: "memory"); break;
  }
}
// Bounded spin until *p >= target; thread-local result.
__device__ __forceinline__ bool wait_geq(const uint32_t *p, uint32_t target) {
  const volatile uint32_t *v = p;
  if (*v >= target) return true;
  const long long t0 = clock64();
  while (*v < target)
    if (clock64() - t0 > kWaitCycles) return false;
  return true;
}

struct Win {
  int p0, np;        // first linear row (pair for gate/up) and count
  int nseg;          // 1 or 2 segments
  int seg[2];        // segment ids
  int off1;          // first window row of segment 1
  int e[2];          // expert of each segment
  int r0[2], n[2];   // routes of each segment (permuted positions)
  int nx;            // staged input rows
  int xrow[8];       // gate/up: token rows; down: route positions
  int xslot[2][4];   // route t of segment j -> staged row
};

struct STables {
  int32_t seg_off[kMaxExperts + 1];
  int32_t active[kMaxExperts];
  int32_t seg_pref[kMaxExperts + 1];  // first segment of active expert a
  int32_t n_active, n_seg, n_valid;
  int32_t flag;                       // broadcast of a bounded wait's result
  int32_t n_comb;
  int32_t comb[8];
  float inv[8];                       // RMSNorm factors of a router task's rows
  Win win;
};

struct Layout {
  int R, rt_off, x_off, ring_off, ns, total;
};

__host__ __device__ inline int align128i(int n) { return (n + 127) & ~127; }

// Dynamic shared memory: tables, the route arrays, the staged input rows, the
// ring.  Identical on host and device.
__host__ __device__ inline Layout make_layout(int T, int K, int x_bytes, int ns) {
  Layout l;
  l.R = T * K;
  l.rt_off = align128i((int)sizeof(STables));
  l.x_off = align128i(l.rt_off + 3 * l.R * 4);
  l.ring_off = align128i(l.x_off + x_bytes);
  l.ns = ns;
  l.total = l.ring_off + ns * kSlotBytes;
  return l;
}

// Active-expert index holding segment s (largest a with seg_pref[a] <= s).
__device__ __forceinline__ int seg_active(const STables &tb, int s) {
  int lo = 0, hi = tb.n_active - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (tb.seg_pref[mid] <= s) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// Which expert and routes segment s holds.
__device__ __forceinline__ void seg_info(const STables &tb, int s, int TG, int &e, int &r0,
                                         int &n) {
  const int a = seg_active(tb, s);
  e = tb.active[a];
  r0 = tb.seg_off[e] + (s - tb.seg_pref[a]) * TG;
  n = min(TG, tb.seg_off[e + 1] - r0);
}

// Window starting at linear row p (< pend) of the gate/up list (down = false,
// one row = one gate/up pair, I per segment) or of the down list (H rows per
// segment): up to kWinPairs / kWinRows rows, at most two segments (the caps
// are <= I and <= H), whose input rows (<= 2 TG) are staged together.
// Written straight into shared memory by one thread.
__device__ void make_win(Win &w, const STables &tb, const int32_t *r_token, bool down, int p,
                         int pend, int H, int I, int TG) {
  const int per = down ? H : I;
  const int cap = down ? kWinRows : kWinPairs;
  const int lim = min(pend, p + cap);
  const int s0 = p / per;
  w.p0 = p;
  w.np = lim - p;
  w.seg[0] = s0;
  w.nseg = lim > (s0 + 1) * per ? 2 : 1;
  w.off1 = (s0 + 1) * per - p;
  int nx = 0;
  for (int j = 0; j < w.nseg; ++j) {
    int e, r0, n;
    seg_info(tb, s0 + j, TG, e, r0, n);
    w.seg[j] = s0 + j;
    w.e[j] = e;
    w.r0[j] = r0;
    w.n[j] = n;
    for (int t = 0; t < n; ++t) {
      const int key = down ? r0 + t : r_token[r0 + t];
      int q = 0;
      while (q < nx && w.xrow[q] != key) ++q;
      if (q == nx) w.xrow[nx++] = key;
      w.xslot[j][t] = q;
    }
  }
  w.nx = nx;
}

// This CTA's share [pb, pe) of the gate/up (phase 0) or down (phase 1) list.
__device__ __forceinline__ void cta_slice(const STables &tb, int phase, int H, int I, int &pb,
                                          int &pe) {
  const long long total = (long long)tb.n_seg * (phase ? H : I);
  pb = (int)(total * blockIdx.x / gridDim.x);
  pe = (int)(total * (blockIdx.x + 1) / gridDim.x);
}

__device__ __forceinline__ void stamp(const FusedArgs &a, int idx) {
  if (a.phase_ts && blockIdx.x == 0 && threadIdx.x == 0) {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    a.phase_ts[idx] = t;
  }
}

// ---------------------------------------------------------------------------
// R: router tasks
// ---------------------------------------------------------------------------
__device__ void router_tasks(const FusedArgs &a, const FusedLayer &L, int layer, float *stage,
                             STables &tb, uint32_t *ctr, bool &alive) {
  const int T = a.T, E = a.E, H = a.H, tid = threadIdx.x;
  const int TT = a.rtt, TE = a.rte;
  const int ntt = (T + TT - 1) / TT, nte = (E + TE - 1) / TE, ntasks = ntt * nte;
  const int nblk = (H + kBR - 1) / kBR;
  const int full = H / 8;
  const bool seq = a.route_mode == kRouteTopkSoftmax && L.router_dtype == kRouterF32;
  const float *src = a.stacked ? a.out : a.h_in;
  for (int task = blockIdx.x; task < ntasks; task += gridDim.x) {
    if (a.stacked && layer > 0) {
      // every block of the previous layer combined (x final), and every CTA
      // done reading the previous layer's logits (they are overwritten here)
      if (tid == 0) {
        tb.flag = wait_geq(ctr + kCtrComb, (uint32_t)(layer * nblk)) &&
                  wait_geq(ctr + kCtrSel, (uint32_t)(layer * gridDim.x));
        __threadfence();
      }
      __syncthreads();
      if (!tb.flag) {
        set_status(a.status, kStatusTimeout);
        alive = false;
        return;
      }
    }
    if (blockIdx.x == 0 && task == 0) {
      // per-layer counters, free once the previous layer is combined
      for (int i = tid; i < kFusedMaxRoutes + nblk; i += kST) ctr[kCtrGu + i] = 0;
      __syncthreads();
    }
    const int t0 = (task / nte) * TT, e0 = (task % nte) * TE;
    const int nt = min(TT, T - t0), ne = min(TE, E - e0);
    float *xs = stage;                       // [TT][H]
    float *ws = stage + (size_t)TT * H;      // [TE][H]
    const int q = H / 4;
    for (int i = tid; i < nt * q; i += kST) {
      const int r = i / q, c = (i % q) * 4;
      cp_async16(xs + (size_t)r * H + c, src + (size_t)(t0 + r) * H + c);
    }
    if (a.router_async) {
      for (int i = tid; i < ne * q; i += kST) {
        const int r = i / q, c = (i % q) * 4;
        cp_async16(ws + (size_t)r * H + c,
                   reinterpret_cast<const float *>(L.router) + (size_t)(e0 + r) * H + c);
      }
    } else {
      for (int i = tid; i < ne * H; i += kST)
        ws[i] = load_w(L.router, L.router_dtype, (size_t)e0 * H + i);
    }
    cp_async_wait_all();
    __syncthreads();
    if (a.stacked) {
      // RMSNorm of the staged rows (src/backend.rs:341-359; this layer's gain)
      // whole warps run the folds (the shuffles name all 32 lanes)
      if ((tid >> 5) < (8 * nt + 31) / 32) {
        const int ti = min(tid >> 3, nt - 1), l = tid & 7;
        const float *x = xs + (size_t)ti * H;
        float acc = 0.0f;
        for (int c = 0; c < full; ++c) acc = __fadd_rn(acc, __fmul_rn(x[8 * c + l], x[8 * c + l]));
        float s = -0.0f;
        const int base = (tid & 31) & ~7;
#pragma unroll
        for (int j = 0; j < 8; ++j) s = __fadd_rn(s, __shfl_sync(0xffffffffu, acc, base + j));
        for (int i = full * 8; i < H; ++i) s = __fadd_rn(s, __fmul_rn(x[i], x[i]));
        if (l == 0 && (tid >> 3) < nt) {
          const float scale = __fsqrt_rn(__fadd_rn(__fdiv_rn(s, (float)H), a.eps));
          tb.inv[ti] = __fdiv_rn(1.0f, scale);
        }
      }
      __syncthreads();
      bool bad = false;
      const bool write = (task % nte) == 0;
      for (int i = tid; i < nt * H; i += kST) {
        const float v = xs[i];
        const float o =
            __fmul_rn(__fmul_rn(v, tb.inv[i / H]), L.norm_w ? L.norm_w[i % H] : 1.0f);
        bad |= !is_finite_f(v) || !is_finite_f(o);
        xs[i] = o;
        if (write) a.hbuf[(size_t)t0 * H + i] = o;
      }
      if (bad) set_status(a.status, kStatusNonFinite);
      __syncthreads();
    } else {
      bool bad = false;
      for (int i = tid; i < nt * H; i += kST) bad |= !is_finite_f(xs[i]);
      if (bad) set_status(a.status, kStatusNonFinite);
    }
    // whole warps run the chains (the fold shuffles name all 32 lanes);
    // lanes past the last (token, expert) pair compute a copy of it
    if ((tid >> 5) < (8 * nt * ne + 31) / 32) {
      const int lane = tid & 7, pair = min(tid >> 3, nt * ne - 1);
      const bool own = (tid >> 3) < nt * ne;
      const int ti = pair / ne, ei = pair % ne;
      const float *hs = xs + (size_t)ti * H;
      const float *w = ws + (size_t)ei * H;
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
      if (lane == 0 && own) {
        a.logits[(size_t)(t0 + ti) * E + e0 + ei] = logit;
        if (!is_finite_f(logit)) set_status(a.status, kStatusNonFinite);
      }
    }
    __syncthreads();
    if (tid == 0) {
      __threadfence();
      atomicAdd(ctr + kCtrLogit, 1u);
    }
  }
  if (layer < 2) stamp(a, 8 * layer + 1);
  // all logits of this layer
  if (tid == 0) {
    tb.flag = wait_geq(ctr + kCtrLogit, (uint32_t)((layer + 1) * ntasks));
    __threadfence();
  }
  __syncthreads();
  if (layer < 2) stamp(a, 8 * layer + 2);
  if (!tb.flag) {
    set_status(a.status, kStatusTimeout);
    alive = false;
  }
}

// ---------------------------------------------------------------------------
// S: selection for every token, then the stable by-expert permutation
// (src/olmoe.rs:3474-3480: experts ascending, tokens ascending inside).
// Scratch lives in the (idle) ring.
// ---------------------------------------------------------------------------
__device__ void select_and_permute(const FusedArgs &a, unsigned char *scratch, STables &tb,
                                   int32_t *r_token, int32_t *r_slot, float *r_gate, int TG,
                                   int layer) {
  const int T = a.T, E = a.E, K = a.K, R = T * K, tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  constexpr int nw = kST / 32;
  uint32_t *ids_s = reinterpret_cast<uint32_t *>(scratch);
  float *gates_s = reinterpret_cast<float *>(scratch + 4 * kFusedMaxRoutes);
  int32_t *cnt = reinterpret_cast<int32_t *>(scratch + 8 * kFusedMaxRoutes);
  const int W = (T + 31) / 32;
  uint32_t *mask = reinterpret_cast<uint32_t *>(cnt + kMaxExperts);  // [E][W]
  SelectScratch *sel = reinterpret_cast<SelectScratch *>(
      scratch + 8 * kFusedMaxRoutes + 4 * kMaxExperts + 4 * kMaxExperts * (kStreamMaxT / 32));
  for (int i = tid; i < E; i += kST) cnt[i] = 0;
  for (int i = tid; i < E * W; i += kST) mask[i] = 0;
  for (int t = warp; t < T; t += nw)
    select_token(a.logits + (size_t)t * E, E, K, a.norm, a.route_mode, ids_s + t * K,
                 gates_s + t * K, nullptr, sel[warp], a.status);
  __syncthreads();
  if (layer < 2) stamp(a, 8 * layer + 7);
  if (blockIdx.x == 0) {
    for (int r = tid; r < R; r += kST) {
      a.ids[r] = ids_s[r];
      a.gates[r] = gates_s[r];
      if (a.ids_out) {
        a.ids_out[r] = ids_s[r];
        a.gates_out[r] = gates_s[r];
      }
    }
  }
  for (int r = tid; r < R; r += kST) {
    const uint32_t e = ids_s[r];
    if (e < (uint32_t)E) {
      const int t = r / K;
      atomicAdd(&cnt[e], 1);
      atomicOr(&mask[e * W + (t >> 5)], 1u << (t & 31));
    }
  }
  __syncthreads();
  if (warp == 0) {
    // exclusive scans over experts: lane owns experts [8*lane, 8*lane + 8)
    int c[8], ls = 0, la = 0, lg = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int e = 8 * lane + j;
      c[j] = e < E ? cnt[e] : 0;
      ls += c[j];
      la += c[j] > 0;
      lg += (c[j] + TG - 1) / TG;
    }
    int is = ls, ia = la, ig = lg;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int s1 = __shfl_up_sync(0xffffffffu, is, o);
      const int a1 = __shfl_up_sync(0xffffffffu, ia, o);
      const int g1 = __shfl_up_sync(0xffffffffu, ig, o);
      if (lane >= o) {
        is += s1;
        ia += a1;
        ig += g1;
      }
    }
    int off = is - ls, act = ia - la, sg = ig - lg;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int e = 8 * lane + j;
      if (e < E) {
        tb.seg_off[e] = off;
        if (c[j] > 0) {
          tb.active[act] = e;
          tb.seg_pref[act] = sg;
          ++act;
          sg += (c[j] + TG - 1) / TG;
        }
        off += c[j];
      }
    }
    if (lane == 31) {
      tb.seg_off[E] = is;
      tb.n_valid = is;
      tb.n_active = ia;
      tb.seg_pref[ia] = ig;
      tb.n_seg = ig;
    }
  }
  __syncthreads();
  for (int r = tid; r < R; r += kST) {
    const uint32_t e = ids_s[r];
    if (e < (uint32_t)E) {
      const int t = r / K;
      int rank = __popc(mask[e * W + (t >> 5)] & ((1u << (t & 31)) - 1u));
      for (int j = 0; j < (t >> 5); ++j) rank += __popc(mask[e * W + j]);
      const int pos = tb.seg_off[e] + rank;
      r_token[pos] = t;
      r_slot[pos] = r % K;
      r_gate[pos] = gates_s[r];
    }
  }
  __syncthreads();
}


// ---------------------------------------------------------------------------
// W/D: the streamed expert GEMVs of one layer (all threads)
// ---------------------------------------------------------------------------
template <int TG>
__device__ void expert_layer(const FusedArgs &a, const FusedLayer &L, STables &tb,
                             const int32_t *r_token, const int32_t *r_slot, const float *r_gate,
                             float *xs, unsigned char *ring, int ns, uint32_t *ctr, int layer,
                             bool &alive) {
  const int tid = threadIdx.x;
  const int H = a.H, I = a.I, K = a.K, T = a.T;
  const int ncb_gu = (H + kCB - 1) / kCB, ncb_dn = (I + kCB - 1) / kCB;
  int pb[2], pe[2];
  cta_slice(tb, 0, H, I, pb[0], pe[0]);
  cta_slice(tb, 1, H, I, pb[1], pe[1]);
  const int nwg = (pe[0] - pb[0] + kWinPairs - 1) / kWinPairs;
  const int nwin = nwg + (pe[1] - pb[1] + kWinRows - 1) / kWinRows;
  const int nst = nwg * ncb_gu + (nwin - nwg) * ncb_dn;
  const float *xsrc = a.stacked ? a.hbuf : a.h_in;

  // Copy issue: every thread copies exactly the bytes its own chain reads
  // (8 bytes of its bank in each 32-byte chunk of the column block) into its
  // private part of the slot, so no barrier is needed between copy and use.
  // Slot layout: [4 pairs of chunks][kST threads][16 bytes].
  const uint64_t pol = evict_first_policy();
  int iw = -1;
  const int8_t *src = nullptr;
  auto issue = [&](int s) {
    if (s < nst) {
      int w, cb;
      if (s < nwg * ncb_gu) {
        w = s / ncb_gu;
        cb = s % ncb_gu;
      } else {
        const int s2 = s - nwg * ncb_gu;
        w = nwg + s2 / ncb_dn;
        cb = s2 % ncb_dn;
      }
      const bool down = w >= nwg;
      if (w != iw) {
        iw = w;
        const int p0 = down ? pb[1] + (w - nwg) * kWinRows : pb[0] + w * kWinPairs;
        const int pw = min(down ? pe[1] : pe[0], p0 + (down ? kWinRows : kWinPairs));
        const int per = down ? H : I;
        const int i = down ? (tid >> 2) : (tid >> 3);
        src = nullptr;
        if (p0 + i < pw) {
          const int p = p0 + i, row = p % per;
          const int8_t *W = L.w_ptr[tb.active[seg_active(tb, p / per)]];
          src = down ? W + (size_t)2 * I * H + (size_t)row * I
                     : W + (((tid >> 2) & 1) ? (size_t)I * H : 0) + (size_t)row * H;
          src += 8 * (tid & 3);
        }
      }
      if (src) {
        const int n = down ? I : H;
        const int c0 = cb * kCB, nc = min(kCB, n - c0) / 32;
        unsigned char *dst = ring + (size_t)(s % ns) * kSlotBytes + (size_t)tid * 16;
#pragma unroll
        for (int c = 0; c < kCB / 32; ++c)
          if (c < nc)
            cp_async8_stream(dst + (c >> 1) * (kST * 16) + (c & 1) * 8, src + c0 + 32 * c, pol);
      }
    }
    cp_async_commit();  // one group per stage, empty ones included
  };

  for (int s = 0; s < ns - 1; ++s) issue(s);
  int s = 0;
  bool good = true;
  for (int wi = 0; wi < nwin; ++wi) {
    const bool down = wi >= nwg;
    if (wi == nwg && layer < 2) stamp(a, 8 * layer + 4);
    if (tid == 0)
      make_win(tb.win, tb, r_token, down,
               down ? pb[1] + (wi - nwg) * kWinRows : pb[0] + wi * kWinPairs,
               down ? pe[1] : pe[0], H, I, TG);
    __syncthreads();
    const Win &w = tb.win;
    if (down) {
      if (tid == 0) {
        int ok = 1;
        for (int jj = 0; jj < w.nseg && ok; ++jj) ok = wait_geq(ctr + kCtrGu + w.seg[jj], I);
        __threadfence();
        tb.flag = ok;
      }
      __syncthreads();
      if (!tb.flag) {
        set_status(a.status, kStatusTimeout);
        cp_async_wait_all();
        alive = false;
        return;
      }
    }
    const int n = down ? I : H;
    const int ncb = down ? ncb_dn : ncb_gu;
    {
      // the window's input rows, read through L2 (written by other CTAs)
      const int q = n / 4;
      for (int idx = tid; idx < w.nx * q; idx += kST) {
        const int r = idx / q, c = (idx % q) * 4;
        const float *sp = down ? a.act + (size_t)w.xrow[r] * I : xsrc + (size_t)w.xrow[r] * H;
        *reinterpret_cast<float4 *>(xs + (size_t)r * n + c) =
            __ldcg(reinterpret_cast<const float4 *>(sp + c));
      }
    }
    __syncthreads();
    // this thread's chain: gate/up lanes = 4 rows x (4 gate + 4 up banks),
    // down lanes = 8 rows x 4 banks
    int i, bank = tid & 3, is_up = 0;
    if (down) {
      i = tid >> 2;
    } else {
      i = tid >> 3;
      is_up = (tid >> 2) & 1;
    }
    const bool valid = i < w.np;
    const int j = (w.nseg == 2 && i >= w.off1) ? 1 : 0;
    const int nr = w.n[j];
    const int row = (w.p0 + (valid ? i : 0)) % (down ? H : I);
    const float *Sp = L.s_ptr[w.e[j]];
    const float scale = valid ? __ldg(Sp + (down ? 2 * I : (is_up ? I : 0)) + row) : 0.0f;
    int xo[TG];
#pragma unroll
    for (int t = 0; t < TG; ++t) xo[t] = (t < nr ? w.xslot[j][t] : 0) * n;
    float acc[TG][8];
#pragma unroll
    for (int t = 0; t < TG; ++t)
#pragma unroll
      for (int l = 0; l < 8; ++l) acc[t][l] = 0.0f;
    for (int cb = 0; cb < ncb; ++cb, ++s) {
      cp_async_wait_pending(ns - 2);  // this thread's bytes of stage s landed
      issue(s + ns - 1);              // into the slot stage s - 1 used (own bytes)
      if (valid) {
        const unsigned char *mine = ring + (size_t)(s % ns) * kSlotBytes + (size_t)tid * 16;
        const int c0 = cb * kCB, nc = min(kCB, n - c0) / 32;
        const float *xb = xs + c0 + 8 * bank;
#pragma unroll 2
        for (int cq = 0; cq < kCB / 64; ++cq) {
          if (2 * cq < nc) {
            const uint4 raw = *reinterpret_cast<const uint4 *>(mine + cq * (kST * 16));
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              float wv[8];
              i8x4_to_f32(h ? raw.z : raw.x, wv[0], wv[1], wv[2], wv[3]);
              i8x4_to_f32(h ? raw.w : raw.y, wv[4], wv[5], wv[6], wv[7]);
              const int c = 2 * cq + h;
#pragma unroll
              for (int t = 0; t < TG; ++t) {
                if (t < nr) {
                  const float4 xa = *reinterpret_cast<const float4 *>(xb + xo[t] + 32 * c);
                  const float4 xc = *reinterpret_cast<const float4 *>(xb + xo[t] + 32 * c + 4);
                  acc[t][0] = __fmaf_rn(wv[0], xa.x, acc[t][0]);
                  acc[t][1] = __fmaf_rn(wv[1], xa.y, acc[t][1]);
                  acc[t][2] = __fmaf_rn(wv[2], xa.z, acc[t][2]);
                  acc[t][3] = __fmaf_rn(wv[3], xa.w, acc[t][3]);
                  acc[t][4] = __fmaf_rn(wv[4], xc.x, acc[t][4]);
                  acc[t][5] = __fmaf_rn(wv[5], xc.y, acc[t][5]);
                  acc[t][6] = __fmaf_rn(wv[6], xc.z, acc[t][6]);
                  acc[t][7] = __fmaf_rn(wv[7], xc.w, acc[t][7]);
                }
              }
            }
          }
        }
      }
    }
    // epilogue: fold the four banks (lanes 4m .. 4m+3), finish the dot; a
    // warp may straddle two segments, so the shuffles run to the warp's
    // largest route count
    const int nrw = __reduce_max_sync(0xffffffffu, (unsigned)nr);
#pragma unroll
    for (int t = 0; t < TG; ++t) {
      if (t < nrw) {
        float b1[8], b2[8], b3[8];
#pragma unroll
        for (int l = 0; l < 8; ++l) {
          b1[l] = __shfl_down_sync(0xffffffffu, acc[t][l], 1);
          b2[l] = __shfl_down_sync(0xffffffffu, acc[t][l], 2);
          b3[l] = __shfl_down_sync(0xffffffffu, acc[t][l], 3);
        }
        float tot[8];
#pragma unroll
        for (int l = 0; l < 8; ++l)
          tot[l] = __fadd_rn(__fadd_rn(acc[t][l], b1[l]), __fadd_rn(b2[l], b3[l]));
        const float s0 = __fadd_rn(tot[0], tot[4]), s1 = __fadd_rn(tot[1], tot[5]);
        const float s2 = __fadd_rn(tot[2], tot[6]), s3 = __fadd_rn(tot[3], tot[7]);
        const float dot = __fadd_rn(__fadd_rn(s0, s2), __fadd_rn(s1, s3));
        const int r = w.r0[j] + t;
        if (!down) {
          const float v = __fmul_rn(dot, scale);
          const float u = __shfl_down_sync(0xffffffffu, v, 4);
          if ((tid & 7) == 0 && valid && t < nr) {
            const float g = v;
            const float den = __fadd_rn(1.0f, expf_ref(-g));
            a.act[(size_t)r * I + row] = __fmul_rn(__fdiv_rn(g, den), u);
          }
        } else if (bank == 0 && valid && t < nr) {
          const float y = __fmul_rn(dot, scale);
          good &= is_finite_f(y);
          a.contrib[((size_t)r_token[r] * K + r_slot[r]) * H + row] = __fmul_rn(r_gate[r], y);
        }
      }
    }
    __syncthreads();
    // publish: gate/up rows per segment, or (route,row) pairs per row block
    if (tid == 0) {
      __threadfence();
      tb.n_comb = 0;
      for (int jj = 0; jj < w.nseg; ++jj) {
        const int lo = jj == 0 ? 0 : w.off1;
        const int hi = (jj + 1 < w.nseg) ? w.off1 : w.np;
        if (!down) {
          atomicAdd(ctr + kCtrGu + w.seg[jj], (uint32_t)(hi - lo));
        } else {
          const int rlo = (w.p0 + lo) % H, rhi = rlo + (hi - lo);
          for (int m = rlo / kBR; m * kBR < rhi; ++m) {
            const int a0 = max(rlo, m * kBR), a1 = min(rhi, (m + 1) * kBR);
            const uint32_t add = (uint32_t)((a1 - a0) * w.n[jj]);
            const uint32_t target = (uint32_t)(tb.n_valid * (min(H, (m + 1) * kBR) - m * kBR));
            const uint32_t old = atomicAdd(ctr + kCtrBlk + m, add);
            if (old + add == target) tb.comb[tb.n_comb++] = m;
          }
        }
      }
      __threadfence();
    }
    __syncthreads();
    // combine the row blocks this window completed (slot order)
    const int n_comb = tb.n_comb;
    for (int cbk = 0; cbk < n_comb; ++cbk) {
      const int m = tb.comb[cbk];
      const int j0 = m * kBR, nrow = min(H, j0 + kBR) - j0;
      bool bad = false;
      for (int idx = tid; idx < T * nrow; idx += kST) {
        const int t = idx / nrow, jr = j0 + idx % nrow;
        const size_t o = (size_t)t * H + jr;
        float acc2 = a.stacked ? __ldcg(a.out + o) : (a.resid ? a.resid[o] : 0.0f);
        for (int kk = 0; kk < K; ++kk)
          acc2 = __fadd_rn(acc2, __ldcg(a.contrib + ((size_t)t * K + kk) * H + jr));
        bad |= !is_finite_f(acc2);
        a.out[o] = acc2;
      }
      if (bad) set_status(a.status, kStatusNonFinite);
    }
    if (n_comb > 0) {
      __syncthreads();
      if (tid == 0) {
        for (int cbk = 0; cbk < n_comb; ++cbk) ctr[kCtrBlk + tb.comb[cbk]] = 0;
        __threadfence();
        atomicAdd(ctr + kCtrComb, (uint32_t)n_comb);
      }
    }
  }
  if (nwg == nwin && layer < 2) stamp(a, 8 * layer + 4);
  cp_async_wait_all();
  if (!good) set_status(a.status, kStatusNonFinite);
  if (layer < 2) stamp(a, 8 * layer + 5);
}

template <int TG>
__global__ void __launch_bounds__(kST, 1) stream_decode_kernel(FusedArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  STables &tb = *reinterpret_cast<STables *>(smem);
  const Layout lay = make_layout(a.T, a.K, a.stream_xbytes, a.stream_ns);
  int32_t *r_token = reinterpret_cast<int32_t *>(smem + lay.rt_off);
  int32_t *r_slot = r_token + lay.R;
  float *r_gate = reinterpret_cast<float *>(r_slot + lay.R);
  float *xs = reinterpret_cast<float *>(smem + lay.x_off);
  unsigned char *ring = smem + lay.ring_off;
  const int ns = lay.ns;
  const int tid = threadIdx.x;
  uint32_t *ctr = a.ctr;
  stamp(a, 0);
  // the next launch's counter set (the previous launch, which used it, is done)
  if (blockIdx.x == gridDim.x - 1)
    for (int i = tid; i < kStreamCtrWords; i += kST) a.ctr_next[i] = 0;
  bool alive = true;
  for (int l = 0; l < a.n_layers && alive; ++l) {
    const FusedLayer L = a.layers[l];
    if (l == 1) stamp(a, 8);
    router_tasks(a, L, l, reinterpret_cast<float *>(ring), tb, ctr, alive);
    if (!alive) break;
    select_and_permute(a, ring, tb, r_token, r_slot, r_gate, TG, l);
    if (tid == 0 && a.stacked) atomicAdd(ctr + kCtrSel, 1u);
    if (l < 2) stamp(a, 8 * l + 3);
    expert_layer<TG>(a, L, tb, r_token, r_slot, r_gate, xs, ring, ns, ctr, l, alive);
    __syncthreads();
  }
  stamp(a, 6);
}

char g_diag[256];

}  // namespace

const char *stream_decode_diag() { return g_diag; }

bool stream_decode_supported(int T, int H, int I, int E, int K) {
  if (T < 1 || T > kStreamMaxT || T * K > kFusedMaxRoutes || E > kMaxExperts) return false;
  if (H % 32 != 0 || I % 32 != 0 || H < kWinRows || I < kWinPairs) return false;
  if (H > kFusedMaxH || I > kFusedMaxH) return false;
  const int TG = T == 1 ? 1 : 4;
  // staged input rows: a window's two segments, 2 TG rows of H or of I
  if ((size_t)2 * TG * H * 4 > (size_t)kXBytes || (size_t)2 * TG * I * 4 > (size_t)kXBytes)
    return false;
  return true;
}

cudaError_t launch_stream_decode(const FusedArgs &a_in, int sm_count, cudaStream_t s) {
  FusedArgs a = a_in;
  const int TG = a.T == 1 ? 1 : 4;
  const void *fn = TG == 1 ? (const void *)stream_decode_kernel<1>
                           : (const void *)stream_decode_kernel<4>;
  int dev = 0;
  cudaGetDevice(&dev);
  int max_smem = 0;
  cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  // staged input rows: a window needs at most 2 TG rows
  const int x_bytes = std::max(2 * TG * a.H * 4, 2 * TG * a.I * 4);
  int ns = kMaxNS;
  while (ns > 3 && make_layout(a.T, a.K, x_bytes, ns).total > max_smem) --ns;
  const Layout lay = make_layout(a.T, a.K, x_bytes, ns);
  if (lay.total > max_smem) return cudaErrorInvalidConfiguration;
  // router tasks: TT tokens x TE experts; staged rows and the selection
  // scratch live in the ring
  const int ring_bytes = ns * kSlotBytes;
  int TT = std::min(a.T, 8), TE = 1;
  while (TE < 8 && (long long)((a.T + TT - 1) / TT) * ((a.E + TE - 1) / TE) > sm_count) TE *= 2;
  while (TE > 1 && (TT + TE) * a.H * 4 > ring_bytes) TE /= 2;
  while (TT > 1 && (TT + TE) * a.H * 4 > ring_bytes) --TT;
  const size_t sel_bytes = 8 * kFusedMaxRoutes + 4 * kMaxExperts +
                           4 * kMaxExperts * (kStreamMaxT / 32) + (kST / 32) * sizeof(SelectScratch);
  if ((TT + TE) * a.H * 4 > ring_bytes || sel_bytes > (size_t)ring_bytes)
    return cudaErrorInvalidConfiguration;
  a.rtt = TT;
  a.rte = TE;
  a.stream_ns = ns;
  a.stream_xbytes = x_bytes;
  static thread_local int cached_dev = -1, cached_tg = -1, cached_smem = -1, cached_grid = 0;
  if (dev != cached_dev || TG != cached_tg || lay.total != cached_smem) {
    cudaError_t e =
        cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, lay.total);
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kST, lay.total);
    if (e != cudaSuccess) return e;
    cudaFuncAttributes fa{};
    cudaFuncGetAttributes(&fa, fn);
    snprintf(g_diag, sizeof g_diag,
             "stream decode: %d CTAs/SM, %d regs, max %d threads, static smem %zu, dynamic %d "
             "(opt-in max %d), ns %d",
             per_sm, fa.numRegs, fa.maxThreadsPerBlock, fa.sharedSizeBytes, lay.total, max_smem,
             ns);
    if (per_sm < 1) return cudaErrorLaunchOutOfResources;
    cached_dev = dev;
    cached_tg = TG;
    cached_smem = lay.total;
    cached_grid = sm_count;
  }
  void *params[] = {&a};
  return cudaLaunchCooperativeKernel(fn, dim3(cached_grid), dim3(kST), params, lay.total, s);
}

}  // namespace moe
