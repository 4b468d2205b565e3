// Internal launch interface between the C-ABI layer (moe_abi.cu) and the
// kernel translation units.  Nothing here crosses the public ABI.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace moe {

// Router + top-k (route.cu).  Reference: src/olmoe.rs:2589-2621 (decode),
// :3421-3466 (prefill); src/backend.rs:105-120, :375-389; src/dense.rs:58-73.
enum RouteMode : int {
  kRouteSoftmaxTopk = 0,  // OlmoeModel: softmax over all E, top-k by probability
  kRouteTopkSoftmax = 1,  // Router::select_top_k: top-k by score, softmax over k
};
enum RouterDtype : int { kRouterF32 = 0, kRouterBF16 = 1, kRouterF32Seq = 2 };

struct RouteArgs {
  const float *h;       // [T, H] MoE input
  const void *router;   // [E, H] f32 or bf16 bits
  int router_dtype;     // RouterDtype
  int T, H, E, K;
  int norm_topk_prob;
  int mode;             // RouteMode
  float *logits;        // [T, E] scratch (raw logits)
  uint32_t *ids;        // [T, K]
  float *gates;         // [T, K]
  float *probs;         // optional [T, E] post-softmax probabilities
  uint32_t *status;
};
// `launches` (optional) receives the number of kernels enqueued.
cudaError_t launch_route(const RouteArgs &a, cudaStream_t s, int *launches = nullptr);

// Stable bucket of routes by expert (src/olmoe.rs:3474-3480): experts in
// ascending id, tokens ascending inside an expert.
struct PermuteArgs {
  const uint32_t *ids;  // [T, K]
  const float *gates;   // [T, K]
  int T, K, E;
  int32_t *seg_off;     // [E + 1]
  int32_t *active;      // [E] expert ids with at least one route, ascending
  int32_t *n_active;    // [1]
  int32_t *r_token;     // [T*K] permuted position -> token
  int32_t *r_slot;      // [T*K] permuted position -> slot
  float *r_gate;        // [T*K] permuted position -> gate (may be null)
  int32_t *r_pos;       // [T*K] (t*K + slot) -> permuted position (may be null)
  uint32_t *status;
  // optional scratch for the multi-CTA sort (large T*K); without it, or too
  // small, one CTA sorts everything
  int32_t *scratch;
  size_t scratch_words;
  // optional: up to two tensor-core tile lists (those with bn > 0) -- tiles
  // of up to bn consecutive routes of one expert, experts ascending, at most
  // max_tiles of them
  struct TileList {
    int bn, max_tiles;
    int32_t *expert, *row0, *rows, *count;
  } tiles[2];
};
size_t permute_scratch_words(int R, int E);
cudaError_t launch_permute(const PermuteArgs &a, cudaStream_t s);
int permute_launches(const PermuteArgs &a);  // kernels launch_permute enqueues

// Grouped INT8 GEMV over expert segments (expert_gemv.cu), in the exact
// reduction order of the reference's AVX2 kernels.
struct GemvArgs {
  int H, I;
  const int8_t *const *w_ptr;  // [n_experts] -> 3*I*H int8 (gate | up | down)
  const float *const *s_ptr;   // [n_experts] -> 2*I+H f32
  const int32_t *active;       // [<= n_experts] expert index per segment
  const int32_t *n_active_dev; // device count of segments, or null
  int n_active_max;            // upper bound (grid sizing) / fixed count
  const int32_t *seg_off;      // [n_experts + 1] route ranges per expert
  const int32_t *r_token;      // route -> row of x (gate/up) ; may be null = identity
  const float *x;              // [*, H] inputs (gate/up)
  float *act;                  // [routes, I]
  // down
  const int32_t *r_slot;       // route -> slot (contrib mode)
  const float *r_gate;         // route -> gate weight (contrib mode)
  int K;                       // contrib stride
  float *contrib;              // contrib mode: [T, K, H] = gate * y
  float *y;                    // pairs mode: [routes, H]
  uint32_t *status;
  int sm_count;
  int vec;                     // 1: every expert base pointer is 8-byte aligned
  int int4;                    // 1: INT4 experts (3*I*H/2 bytes, two nibbles per byte)
};
cudaError_t launch_gate_up(const GemvArgs &a, cudaStream_t s);
cudaError_t launch_down(const GemvArgs &a, cudaStream_t s);

// out[t] = (resid ? resid[t] : 0) + sum_slot contrib[t, slot] (slot order);
// src/olmoe.rs:3147-3157, :3702-3714.
cudaError_t launch_combine(const float *contrib, const float *resid, float *out, int T, int K,
                           int H, uint32_t *status, cudaStream_t s);

// RMSNorm with unit gain (src/backend.rs:341-359) over [T, H].
cudaError_t launch_rmsnorm(const float *x, const float *w, float *out, int T, int H, float eps,
                           uint32_t *status, cudaStream_t s);

// Fused decode (decode_fused.cu): a whole layer, or a stack of layers with
// RMSNorm + residual, in one cooperative launch for small T.
constexpr int kFusedMaxRoutes = 1024;  // T * K per call
constexpr int kFusedMaxH = 2048;       // router staging holds 8 rows of H floats

struct FusedLayer {
  const int8_t *const *w_ptr;
  const float *const *s_ptr;
  const void *router;
  int router_dtype;   // RouterDtype of the stored router
  int prefetch_ok;    // expert bases 16-byte aligned, H and I multiples of 16
  const float *norm_w;  // stacks: gain [H] of the RMSNorm before this layer, null = 1
  int int4;             // INT4 experts: rows of n/2 bytes, two signed nibbles per byte
  // Device array of two 128-byte CUtensorMaps over the packed expert weights
  // (gate/up rows: 128 B x 32-row boxes; down rows: 128 B x 64-row boxes,
  // 128-byte swizzle), or null: the decode GEMV then loads weights per thread.
  const void *tmaps;
};

struct FusedArgs {
  int T, H, I, E, K, norm, route_mode;
  int n_layers;              // layers in this launch
  int stacked;               // 1: x <- x + MoE(RMSNorm(x)) per layer, x in `out`
  const FusedLayer *layers;  // device array [n_layers]
  const float *h_in;         // single layer: MoE input [T, H]
  const float *resid;        // single layer: residual [T, H] or null
  float *out;                // single layer: output; stacked: x, updated in place
  float *hbuf;               // stacked: normalized input [T, H]
  float eps;
  float *logits;             // [T, E]
  uint32_t *ids;             // [T, K]
  float *gates;              // [T, K]
  float *act;                // [T*K, I]
  float *contrib;            // [T, K, H]
  uint32_t *ids_out;         // optional copies of the routing (single layer)
  float *gates_out;
  uint32_t *tok_cnt;         // [T] arrival counters, zero between calls
  uint32_t *bar;             // grid barrier counter (zeroed by the launcher)
  uint32_t *status;
  int router_async;          // routers of every layer are 16-byte aligned f32 rows
  int int4;                  // every layer of the launch has INT4 experts
  int tiles;                 // every layer has weight-tile maps; 16-byte aligned inputs
  unsigned long long *phase_ts;  // optional [5] phase timestamps (profiling)
  long long wait_cycles;     // bound of each grid-barrier wait (SM clock cycles)
};
bool fused_decode_supported(int T, int H, int I, int E, int K);
cudaError_t launch_fused_decode(const FusedArgs &a, int vec, int sm_count, uint32_t *bar,
                                cudaStream_t s);

// Digit decode (decode_digits.cu): a whole layer, or a stack of layers with
// RMSNorm + residual, in one cooperative launch for decode batches, on the
// tolerance path (two-digit int8 activations, dp4a; results bit-identical to
// the tensor-core path, routing bit-identical to the CPU reference).  Every
// layer INT8 with 16-byte aligned expert rows (FusedLayer::prefetch_ok);
// 16-byte aligned f32 inputs.
struct DigitArgs {
  int T, H, I, E, K, norm, route_mode;
  int n_layers;              // layers in this launch
  int stacked;               // 1: x <- x + MoE(RMSNorm(x)) per layer, x in `out`
  const FusedLayer *layers;  // device array [n_layers]
  const float *h_in;         // single layer: MoE input [T, H]
  const float *resid;        // single layer: residual [T, H] or null
  float *out;                // single layer: output; stacked: x, updated in place
  float eps;
  float *logits;             // [T, E]
  uint32_t *ids;             // [T, K] routing of the latest layer
  float *gates;              // [T, K]
  uint32_t *ids_out;         // optional copies of the routing (single layer)
  float *gates_out;
  int8_t *xq;                // [T][2][H] token digit planes
  float *xs1, *xs2;          // [T] token scales s, s / 254
  float *act;                // [T*K, I] activations (token-major route order)
  float *contrib;            // [T, K, H] gate * y (T > 1)
  uint32_t *bar;             // [2] barrier arrivals, exits: zero before the first launch;
                             // every launch leaves them zero
  uint32_t *status;
  long long wait_cycles;     // bound of each grid-barrier wait (SM clock cycles)
  int router_async;          // routers of every layer are 16-byte aligned f32 rows
  int prefetch_down;         // prefetch the down rows into L2 during gate/up
  int gate_w, down_w;        // work-split costs: a row costs (its expert's routes + w)
  unsigned long long *phase_ts;  // optional phase timestamps (profiling)
  int sub_stamps;            // also stamp inside the router phase (set by the kernel)
};
bool digit_decode_supported(int T, int H, int I, int E, int K);
cudaError_t launch_digit_decode(const DigitArgs &a, int sm_count, cudaStream_t s);

// Expert parallelism (ep.cu): one route on the wire = two int8 digit planes
// of its token row + {s1, s2, gate, destination-local expert id}.
__host__ __device__ inline size_t ep_row_bytes(int H) { return (size_t)2 * H + 16; }
cudaError_t launch_ep_dest(const uint32_t *ids, const int32_t *owner, int R, int E,
                           uint32_t *dest, uint32_t *status, cudaStream_t s);
cudaError_t launch_ep_pack(const float *x, const int32_t *r_token, const int32_t *r_slot,
                           const float *r_gate, const uint32_t *ids, const int32_t *local_of,
                           int R, int K, int H, uint8_t *send, cudaStream_t s);
cudaError_t launch_ep_unpack_meta(const uint8_t *recv, int R, int H, int E_local,
                                  uint32_t *ids_local, float *gates, uint32_t *status,
                                  cudaStream_t s);
cudaError_t launch_ep_unpack_digits(const uint8_t *recv, const int32_t *src, int R, int H,
                                    int8_t *xq, size_t plane, float *s1, float *s2,
                                    uint32_t *amax_reset, cudaStream_t s);
cudaError_t launch_seg_counts(const int32_t *seg, int n, int32_t *cnt, cudaStream_t s);
cudaError_t launch_ep_gather_combine(const float *ret, const int32_t *pos, const float *resid,
                                     float *out, int T, int K, int H, uint32_t *status,
                                     cudaStream_t s);

// Expert parallelism over NVLink peer memory: one region per rank, mapped by
// every peer (CUDA IPC) at the same offsets.
constexpr int kEpMaxRanks = 8;
struct EpP2P {
  uint8_t *base[kEpMaxRanks];  // region of each rank, as mapped in this process
  int rank, nranks;
  size_t off_flags;            // uint32 [3][kEpMaxRanks]: A counts, B routes, C outputs
  size_t off_counts;           // int32 [2][nranks][E] route counts by source rank
  size_t off_xq, plane;        // int8 [2][RR][H] digit planes (plane = RR * H)
  size_t off_s1, off_s2, off_gate, off_rank, off_tok, off_slot, off_amax;  // [RR]
  size_t off_contrib;          // outputs of this rank's routes, written by their owners:
                               // int16 [T, K, H] (value = q * scale) when ret16, else f32
  size_t off_cscale;           // f32 [T, K, ceil(H / 32)] scales of the int16 rows
  int ret16;                   // return format (MOE_EP_RETURN)
  long long wait_cycles;       // bound of every flag wait (SM clock cycles)
};
// epoch: this rank's call counter in device memory; the publish kernel
// advances it, every later kernel of the call reads it.
cudaError_t launch_ep_publish(const int32_t *seg_off, int E, const EpP2P &p, uint32_t *epoch,
                              cudaStream_t s);
// One warp per token: quantize the row once, store it at each of its K
// routes' rows in the owners' buffers (r_pos: route -> position in this
// rank's expert-sorted order, as the permutation writes it).
cudaError_t launch_ep_dispatch(const float *x, const int32_t *seg_off, const uint32_t *ids,
                               const float *gates, const int32_t *r_pos, const int32_t *owner,
                               int E, int T, int K, int H, const EpP2P &p, const uint32_t *epoch,
                               uint32_t *done, int grid, uint32_t *status, cudaStream_t s);
cudaError_t launch_ep_recv_prep(const int32_t *owner, int E, const EpP2P &p,
                                const uint32_t *epoch, int32_t *seg_l, int32_t *active_l,
                                int32_t *n_active_l, int32_t *n_recv, uint32_t *status,
                                cudaStream_t s);
cudaError_t launch_ep_signal(const EpP2P &p, const uint32_t *epoch, cudaStream_t s);
// One thread waits, with the flag waits' bound, until flags[0..n) all reach
// `target`; on expiry kStatusTimeout goes into *status.  Used by the
// failure-path test (moe_debug_wait_flag) on a flag that nobody sets.
cudaError_t launch_wait_probe(const uint32_t *flags, int n, uint32_t target,
                              long long wait_cycles, uint32_t *status, cudaStream_t s);
cudaError_t launch_ep_wait_combine(const EpP2P &p, const uint32_t *epoch, const float *resid,
                                   float *out, int T, int K, int H, uint32_t *status,
                                   cudaStream_t s);

// Seeded synthetic expert weights, bit-identical to the host-side generator.
cudaError_t launch_synth_expert(uint64_t seed, int layer, int expert, int H, int I, int8_t *w,
                                float *sc, cudaStream_t s);

// expf restatement evaluated over a range of float bit patterns; writes a
// per-block mismatch count against `expected` (or the raw values when
// expected == null).  Used by the parity tests.
cudaError_t launch_expf_eval(uint32_t bits_lo, uint32_t count, float *out, cudaStream_t s);

// Read `bytes` (a multiple of 16, 16-byte aligned) once with 16-byte loads.
cudaError_t launch_stream_read(const void *buf, size_t bytes, uint32_t *sink, int sm_count,
                               cudaStream_t s);

}  // namespace moe
