// Host side of the C ABI declared in include/moe_b200.h.
//
// Ownership mirrors the reference: expert weights are borrowed device
// pointers (GpuExpertWeights, src/gpu.rs:1552-1566); the handle owns its
// device scratch and serialises calls with a mutex (src/gpu_expert.rs:241-261).
#include <dlfcn.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>

#include "ckpt.h"
#include "handle.h"

using namespace moe;

namespace moe {
namespace host {

void set_err(std::string &dst, const char *fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  dst = buf;
}

int sm_count_of(int device) {
  int n = 148;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device);
  return n;
}

const NcclApi &nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void *lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!lib) lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!lib) return;
    auto sym = [&](const char *n) { return dlsym(lib, n); };
    api.get_unique_id = (decltype(api.get_unique_id))sym("ncclGetUniqueId");
    api.comm_init_rank = (decltype(api.comm_init_rank))sym("ncclCommInitRank");
    api.comm_destroy = (decltype(api.comm_destroy))sym("ncclCommDestroy");
    api.send = (decltype(api.send))sym("ncclSend");
    api.recv = (decltype(api.recv))sym("ncclRecv");
    api.group_start = (decltype(api.group_start))sym("ncclGroupStart");
    api.group_end = (decltype(api.group_end))sym("ncclGroupEnd");
    api.error_string = (decltype(api.error_string))sym("ncclGetErrorString");
    api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.send &&
             api.recv && api.group_start && api.group_end && api.error_string;
  });
  return api;
}

}  // namespace host
}  // namespace moe

using namespace moe::host;

// ---------------------------------------------------------------------------
// GpuExpertKernels drop-in
// ---------------------------------------------------------------------------
struct moe_expert_kernels {
  int device = 0;
  size_t H = 0, I = 0, max_experts = 0;
  int sm_count = 148;
  cudaStream_t stream = nullptr;
  std::mutex mu;
  std::string err;
  float *d_in = nullptr, *d_act = nullptr, *d_out = nullptr;
  const int8_t **d_wptr = nullptr;
  const float **d_sptr = nullptr;
  int32_t *d_seg = nullptr, *d_tok_shared = nullptr;
  uint32_t *d_status = nullptr;
  float *h_in = nullptr, *h_out = nullptr;
  const void **h_ptrs = nullptr;  // pinned staging for the pointer arrays
};

extern "C" moe_status moe_expert_kernels_init(int device, size_t hidden, size_t intermediate,
                                              size_t max_experts, moe_expert_kernels **out) {
  if (!out) return MOE_ERR_INVALID;
  *out = nullptr;
  if (hidden == 0 || intermediate == 0 || max_experts == 0 || hidden > (1u << 20) ||
      intermediate > (1u << 20) || max_experts > 4096)
    return MOE_ERR_INVALID;
  if (cudaSetDevice(device) != cudaSuccess) return MOE_ERR_CUDA;
  auto *k = new moe_expert_kernels();
  k->device = device;
  k->H = hidden;
  k->I = intermediate;
  k->max_experts = max_experts;
  k->sm_count = sm_count_of(device);
  bool ok = cudaStreamCreateWithFlags(&k->stream, cudaStreamNonBlocking) == cudaSuccess;
  ok = ok && dalloc(&k->d_in, max_experts * hidden) == cudaSuccess;
  ok = ok && dalloc(&k->d_act, max_experts * intermediate) == cudaSuccess;
  ok = ok && dalloc(&k->d_out, max_experts * hidden) == cudaSuccess;
  ok = ok && dalloc(&k->d_wptr, max_experts) == cudaSuccess;
  ok = ok && dalloc(&k->d_sptr, max_experts) == cudaSuccess;
  ok = ok && dalloc(&k->d_seg, max_experts + 1) == cudaSuccess;
  ok = ok && dalloc(&k->d_tok_shared, max_experts) == cudaSuccess;
  ok = ok && dalloc(&k->d_status, 1) == cudaSuccess;
  ok = ok && cudaMallocHost(&k->h_in, max_experts * hidden * sizeof(float)) == cudaSuccess;
  ok = ok && cudaMallocHost(&k->h_out, max_experts * hidden * sizeof(float)) == cudaSuccess;
  ok = ok && cudaMallocHost(&k->h_ptrs, 2 * max_experts * sizeof(void *)) == cudaSuccess;
  if (ok) {
    std::vector<int32_t> seg(max_experts + 1);
    for (size_t i = 0; i <= max_experts; ++i) seg[i] = (int32_t)i;
    ok = cudaMemcpy(k->d_seg, seg.data(), seg.size() * 4, cudaMemcpyHostToDevice) == cudaSuccess;
    ok = ok && cudaMemset(k->d_tok_shared, 0, max_experts * 4) == cudaSuccess;
    ok = ok && cudaMemset(k->d_status, 0, 4) == cudaSuccess;
  }
  if (!ok) {
    moe_expert_kernels_destroy(k);
    return MOE_ERR_NOMEM;
  }
  *out = k;
  return MOE_OK;
}

extern "C" void moe_expert_kernels_destroy(moe_expert_kernels *k) {
  if (!k) return;
  {
    DeviceGuard g(k->device);
    if (k->stream) cudaStreamSynchronize(k->stream);
    cudaFree(k->d_in);
    cudaFree(k->d_act);
    cudaFree(k->d_out);
    cudaFree(k->d_wptr);
    cudaFree(k->d_sptr);
    cudaFree(k->d_seg);
    cudaFree(k->d_tok_shared);
    cudaFree(k->d_status);
    cudaFreeHost(k->h_in);
    cudaFreeHost(k->h_out);
    cudaFreeHost(k->h_ptrs);
    if (k->stream) cudaStreamDestroy(k->stream);
  }
  delete k;
}

extern "C" size_t moe_expert_kernels_max_experts(const moe_expert_kernels *k) {
  return k ? k->max_experts : 0;
}

extern "C" const char *moe_expert_kernels_last_error(const moe_expert_kernels *k) {
  return k ? k->err.c_str() : "null handle";
}

extern "C" moe_status moe_expert_forward_pairs(moe_expert_kernels *k, const void *const *d_weights,
                                               const void *const *d_scales,
                                               const size_t *weight_bytes,
                                               const size_t *scale_bytes, size_t n,
                                               const float *const *inputs, size_t n_inputs,
                                               float *const *outputs) {
  if (!k) return MOE_ERR_INVALID;
  std::lock_guard<std::mutex> lock(k->mu);
  const size_t H = k->H, I = k->I;
  // Validation order follows src/gpu_expert.rs:383-403.
  if (n_inputs != 1 && n_inputs != n) {
    set_err(k->err, "expert/input count mismatch");
    return MOE_ERR_INVALID;
  }
  if (n > k->max_experts) {
    set_err(k->err, "expert/output count mismatch");
    return MOE_ERR_INVALID;
  }
  if (n == 0) return MOE_OK;
  if (!d_weights || !d_scales || !inputs || !outputs) {
    set_err(k->err, "null pointer argument");
    return MOE_ERR_INVALID;
  }
  for (size_t j = 0; j < n; ++j) {
    if ((weight_bytes && weight_bytes[j] != 3 * H * I) ||
        (scale_bytes && scale_bytes[j] != (2 * I + H) * 4)) {
      set_err(k->err, "GPU expert compute supports INT8 experts of the loaded shape only");
      return MOE_ERR_INVALID;
    }
    if (!d_weights[j] || !d_scales[j] || !outputs[j] || (j < n_inputs && !inputs[j])) {
      set_err(k->err, "null expert, input or output pointer");
      return MOE_ERR_INVALID;
    }
    if ((uintptr_t)d_scales[j] & 3) {
      set_err(k->err, "expert scales must be 4-byte aligned");
      return MOE_ERR_INVALID;
    }
  }
  int vec = 1;
  for (size_t j = 0; j < n; ++j) vec &= ((uintptr_t)d_weights[j] & 7) == 0;
  DeviceGuard g(k->device);
  for (size_t j = 0; j < n_inputs; ++j) memcpy(k->h_in + j * H, inputs[j], H * sizeof(float));
  for (size_t j = 0; j < n; ++j) {
    k->h_ptrs[j] = d_weights[j];
    k->h_ptrs[k->max_experts + j] = d_scales[j];
  }
  cudaStream_t s = k->stream;
  cudaMemcpyAsync(k->d_in, k->h_in, n_inputs * H * sizeof(float), cudaMemcpyHostToDevice, s);
  cudaMemcpyAsync(k->d_wptr, k->h_ptrs, n * sizeof(void *), cudaMemcpyHostToDevice, s);
  cudaMemcpyAsync(k->d_sptr, k->h_ptrs + k->max_experts, n * sizeof(void *),
                  cudaMemcpyHostToDevice, s);
  GemvArgs a{};
  a.H = (int)H;
  a.I = (int)I;
  a.w_ptr = k->d_wptr;
  a.s_ptr = k->d_sptr;
  a.active = nullptr;
  a.n_active_dev = nullptr;
  a.n_active_max = (int)n;
  a.seg_off = k->d_seg;
  a.r_token = n_inputs == 1 ? k->d_tok_shared : nullptr;
  a.x = k->d_in;
  a.act = k->d_act;
  a.y = k->d_out;
  a.status = k->d_status;
  a.sm_count = k->sm_count;
  a.vec = vec;
  cudaError_t e = launch_gate_up(a, s);
  if (e == cudaSuccess) e = launch_down(a, s);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(k->h_out, k->d_out, n * H * sizeof(float), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) {
    set_err(k->err, "CUDA error in expert kernels: %s", cudaGetErrorString(e));
    return MOE_ERR_CUDA;
  }
  uint32_t st = 0;
  cudaMemcpy(&st, k->d_status, 4, cudaMemcpyDeviceToHost);
  if (st) cudaMemset(k->d_status, 0, 4);
  for (size_t j = 0; j < n; ++j) memcpy(outputs[j], k->h_out + j * H, H * sizeof(float));
  for (size_t i = 0; i < n * H; ++i)
    if (!std::isfinite(k->h_out[i])) {
      set_err(k->err, "GPU expert output is not finite");
      return MOE_ERR_NONFINITE;
    }
  return MOE_OK;
}

extern "C" moe_status moe_expert_forward(moe_expert_kernels *k, const void *const *d_weights,
                                         const void *const *d_scales, const size_t *weight_bytes,
                                         const size_t *scale_bytes, size_t n, const float *input,
                                         float *const *outputs) {
  const float *inputs[1] = {input};
  return moe_expert_forward_pairs(k, d_weights, d_scales, weight_bytes, scale_bytes, n, inputs, 1,
                                  outputs);
}

// ---------------------------------------------------------------------------
// MoE layer handle
// ---------------------------------------------------------------------------
namespace moe {
namespace host {

void drop_graphs(moe_handle *h) {
  for (auto &g : h->graphs) cudaGraphExecDestroy(g.exec);
  h->graphs.clear();
}

cudaStream_t pick(moe_handle *h, void *stream) {
  return stream ? reinterpret_cast<cudaStream_t>(stream) : h->stream;
}

moe_status cuda_fail(moe_handle *h, cudaError_t e, const char *what) {
  set_err(h->err, "%s: %s", what, cudaGetErrorString(e));
  return MOE_ERR_CUDA;
}

// Router + top-k + permutation for T tokens of `layer`.
// bn_gu > 0: the permutation also writes the tensor-core tile list of the
// gate/up GEMM, and (bn_dn > 0, != bn_gu) the down GEMM's.
moe_status run_route(moe_handle *h, const LayerSlot &L, const float *d_h, int T, uint32_t *ids,
                     float *gates, float *probs, cudaStream_t s, bool permute, int bn_gu,
                     int bn_dn) {
  RouteArgs ra{};
  ra.h = d_h;
  ra.router = L.router;
  ra.router_dtype = L.router_dtype;
  if (h->route_mode == MOE_ROUTE_TOPK_SOFTMAX && L.router_dtype == MOE_ROUTER_F32)
    ra.router_dtype = kRouterF32Seq;  // src/router.rs:59-62 sequential dot
  ra.T = T;
  ra.H = h->d.hidden;
  ra.E = h->d.num_experts;
  ra.K = h->d.top_k;
  ra.norm_topk_prob = h->d.norm_topk_prob;
  ra.mode = h->route_mode;
  ra.logits = h->logits;
  ra.ids = ids;
  ra.gates = gates;
  ra.probs = probs;
  ra.status = h->status;
  cudaEvent_t p0 = h->prof.begin(s);
  int nl = 0;
  cudaError_t e = launch_route(ra, s, &nl);
  h->prof.end("route", p0, s);
  if (e != cudaSuccess) return cuda_fail(h, e, "route launch");
  h->last_launches += nl;
  if (!permute) return MOE_OK;
  PermuteArgs pa{};
  pa.ids = ids;
  pa.gates = gates;
  pa.T = T;
  pa.K = h->d.top_k;
  pa.E = h->d.num_experts;
  pa.seg_off = h->seg_off;
  pa.active = h->active;
  pa.n_active = h->n_active;
  pa.r_token = h->r_token;
  pa.r_slot = h->r_slot;
  pa.r_gate = h->r_gate;
  pa.r_pos = h->r_pos;
  pa.status = h->status;
  pa.scratch = h->perm_scratch;
  pa.scratch_words = h->perm_scratch_words;
  if (bn_gu > 0)
    pa.tiles[0] = {bn_gu, h->max_tiles, h->tile_expert, h->tile_row0, h->tile_rows, h->n_tiles};
  if (bn_dn > 0 && bn_dn != bn_gu)
    pa.tiles[1] = {bn_dn, h->max_tiles, h->dtile_expert, h->dtile_row0, h->dtile_rows,
                   h->n_dtiles};
  p0 = h->prof.begin(s);
  e = launch_permute(pa, s);
  h->prof.end("permute", p0, s);
  if (e != cudaSuccess) return cuda_fail(h, e, "permute launch");
  h->last_launches += permute_launches(pa);
  return MOE_OK;
}

}  // namespace host
}  // namespace moe

namespace {

void free_handle(moe_handle *h) {
  drop_graphs(h);
  free_ep(h);
  for (auto &l : h->layers) {
    cudaFree(l.d_wptr);
    cudaFree(l.d_sptr);
    cudaFree(l.d_tmaps);
    cudaFree(l.own_w);
    cudaFree(l.own_s);
    cudaFree(l.own_r);
    cudaFree(l.own_n);
  }
  void *ptrs[] = {h->logits,  h->gates,     h->r_gate,    h->act,       h->contrib, h->hbuf,
                  h->io_in,   h->io_out,    h->io_resid,  h->ids,       h->status,  h->seg_off,
                  h->active,  h->n_active,  h->r_token,   h->r_slot,    h->r_pos,   h->xq,
                  h->aq,      h->xs1,       h->xs2,       h->as1,       h->as2,     h->act_amax,
                  h->tile_expert, h->tile_row0, h->tile_rows, h->n_tiles, h->d_flayers,
                  h->dtile_expert, h->dtile_row0, h->dtile_rows, h->n_dtiles,
                  h->tok_cnt, h->fbar, h->phase_ts, h->perm_scratch, h->probe_flag, h->dbar};
  for (void *p : ptrs) cudaFree(p);
  cudaFreeHost(h->h_pin_in);
  cudaFreeHost(h->h_pin_out);
  cudaFreeHost(h->h_pin_status);
  cudaFreeHost(h->h_pin_meta);
  for (auto ev : h->stage_ev)
    if (ev) cudaEventDestroy(ev);
  for (auto &row : h->io_ev)
    for (auto ev : row)
      if (ev) cudaEventDestroy(ev);
  for (auto st : h->io_stream)
    if (st) cudaStreamDestroy(st);
  if (h->own_stream) cudaStreamDestroy(h->own_stream);
}

moe_status check_layer(moe_handle *h, int layer, int T) {
  if (layer < 0 || layer >= (int)h->layers.size()) {
    set_err(h->err, "layer %d out of range [0, %d)", layer, (int)h->layers.size());
    return MOE_ERR_INVALID;
  }
  if (!h->layers[layer].set) {
    set_err(h->err, "layer %d has no weights", layer);
    return MOE_ERR_STATE;
  }
  if (T < 0 || T > h->d.max_tokens) {
    set_err(h->err, "token count %d outside [0, %d]", T, h->d.max_tokens);
    return MOE_ERR_INVALID;
  }
  return MOE_OK;
}

bool use_tensor_path(const moe_handle *h, const LayerSlot &L, int T, const float *d_h) {
  const bool avail = h->tc_ok && L.tc_ok && ((uintptr_t)d_h & 15) == 0;
  if (h->path == MOE_PATH_TENSOR) return avail;
  if (h->path == MOE_PATH_GEMV || h->path == MOE_PATH_GEMV_PHASED ||
      h->path == MOE_PATH_GEMV_FUSED || h->path == MOE_PATH_DIGITS)
    return false;
  return avail && T >= kTcMinTokens;
}

// The digit decode launch can run layers [first, first + n) at T tokens:
// INT8 layers with 16-byte aligned rows, 16-byte aligned f32 activations.
bool digits_available(const moe_handle *h, int T, int first, int n, const void *d_x,
                      const void *d_resid) {
  if (((uintptr_t)d_x & 15) || ((uintptr_t)d_resid & 15)) return false;
  if (!digit_decode_supported(T, h->d.hidden, h->d.intermediate, h->d.num_experts, h->d.top_k))
    return false;
  for (int l = first; l < first + n; ++l)
    if (h->flayers[l].int4 || !h->flayers[l].prefetch_ok) return false;
  return true;
}

bool use_digits(const moe_handle *h, int T, int first, int n, const void *d_x,
                const void *d_resid) {
  if (h->path == MOE_PATH_DIGITS) return true;  // availability is checked by the caller
  return h->path == MOE_PATH_AUTO && T < kTcMinTokens &&
         digits_available(h, T, first, n, d_x, d_resid);
}

DigitArgs digit_args(moe_handle *h, int T) {
  DigitArgs a{};
  a.T = T;
  a.H = h->d.hidden;
  a.I = h->d.intermediate;
  a.E = h->d.num_experts;
  a.K = h->d.top_k;
  a.norm = h->d.norm_topk_prob;
  a.route_mode = h->route_mode;
  a.logits = h->logits;
  a.ids = h->ids;
  a.gates = h->gates;
  a.xq = h->xq;
  a.xs1 = h->xs1;
  a.xs2 = h->xs2;
  a.act = h->act;
  a.contrib = h->contrib;
  a.bar = h->dbar;
  a.status = h->status;
  a.wait_cycles = h->wait_barrier_cycles;
  // the down rows of a single-token launch (<= K experts) fit in L2 beside
  // the gate/up stream
  a.prefetch_down = T == 1 && (size_t)h->d.top_k * h->d.hidden * h->d.intermediate <= (48u << 20);
  // MOE_DIGIT_PREFETCH=0 in the environment turns the down-row prefetch off
  static const bool prefetch_env = [] {
    const char *v = getenv("MOE_DIGIT_PREFETCH");
    return !(v && v[0] == '0');
  }();
  a.prefetch_down = a.prefetch_down && prefetch_env;
  // work-split costs (MOE_DIGIT_GW / MOE_DIGIT_DW override them for tuning)
  static const int gate_w = [] {
    const char *v = getenv("MOE_DIGIT_GW");
    return v ? std::max(0, atoi(v)) : 2;
  }();
  static const int down_w = [] {
    const char *v = getenv("MOE_DIGIT_DW");
    return v ? std::max(0, atoi(v)) : 3;
  }();
  a.gate_w = gate_w;
  a.down_w = down_w;
  if (h->prof.on) {
    a.phase_ts = h->phase_ts;
    h->phase_pending = true;
    h->phase_kind = 1;
  }
  return a;
}

bool use_fused(const moe_handle *h, int T) {
  return h->path != MOE_PATH_GEMV_PHASED &&
         fused_decode_supported(T, h->d.hidden, h->d.intermediate, h->d.num_experts,
                                h->d.top_k);
}

// One weight format over layers [first, first + n) (the single-launch kernel
// is compiled per format); -1 when they differ.
int layers_quant(const moe_handle *h, int first, int n) {
  const int q = h->flayers[first].int4;
  for (int l = first + 1; l < first + n; ++l)
    if (h->flayers[l].int4 != q) return -1;
  return q;
}

FusedArgs fused_args(moe_handle *h, int T) {
  FusedArgs f{};
  f.T = T;
  f.H = h->d.hidden;
  f.I = h->d.intermediate;
  f.E = h->d.num_experts;
  f.K = h->d.top_k;
  f.norm = h->d.norm_topk_prob;
  f.route_mode = h->route_mode;
  f.logits = h->logits;
  f.ids = h->ids;
  f.gates = h->gates;
  f.act = h->act;
  f.contrib = h->contrib;
  f.tok_cnt = h->tok_cnt;
  f.status = h->status;
  f.wait_cycles = h->wait_barrier_cycles;
  if (h->prof.on) {
    f.phase_ts = h->phase_ts;
    h->phase_pending = true;
    h->phase_kind = 0;
  }
  return f;
}

// Experts on the tensor cores: digit planes of the routed inputs, gate/up
// GEMM with SwiGLU epilogue, digit planes of the activations, down GEMM with
// the gate-weighted contribution epilogue, slot-ordered combine.
moe_status tensor_experts(moe_handle *h, const LayerSlot &L, const float *d_h,
                          const float *d_resid, float *d_out, int T, cudaStream_t s) {
  const int H = h->d.hidden, I = h->d.intermediate, K = h->d.top_k;
  const int R = T * K;
  const size_t Rcap = (size_t)h->d.max_tokens * K;
  const int bn = tc::tc_block_n(R, h->d.num_experts);
  cudaError_t e;
  // the tile lists came with the permutation (run_route with the same widths)
  cudaEvent_t p0 = h->prof.begin(s);
  e = tc::launch_quantize_tokens(d_h, h->r_pos, T, K, H, h->xq, Rcap * H, h->xs1, h->xs2,
                                 h->act_amax, s);
  h->prof.end("tc_prep", p0, s);
  if (e != cudaSuccess) return cuda_fail(h, e, "tensor prep launch");
  tc::TcArgs a{};
  a.H = H;
  a.I = I;
  a.K = K;
  a.tile_expert = h->tile_expert;
  a.tile_row0 = h->tile_row0;
  a.tile_rows = h->tile_rows;
  a.n_tiles = h->n_tiles;
  a.s_ptr = L.d_sptr;
  a.xs1 = h->xs1;
  a.xs2 = h->xs2;
  a.act = h->act;
  a.act_amax = h->act_amax;
  a.as1 = h->as1;
  a.as2 = h->as2;
  a.r_token = h->r_token;
  a.r_slot = h->r_slot;
  a.r_gate = h->r_gate;
  a.contrib = h->contrib;
  a.status = h->status;
  const int tiles = std::min(h->max_tiles, (R + bn - 1) / bn + std::min(h->d.num_experts, R));
  p0 = h->prof.begin(s);
  e = tc::launch_gate_up_tc(L.map_gu, bn == 64 ? h->map_x64 : h->map_x128, a, bn, tiles, s);
  h->prof.end("gate_up_tc", p0, s);
  if (e == cudaSuccess) {
    p0 = h->prof.begin(s);
    e = tc::launch_quantize_rows(h->act, nullptr, h->act_amax, R, I, h->aq, Rcap * I, h->as1,
                                 h->as2, nullptr, s);
    h->prof.end("tc_act_digits", p0, s);
  }
  if (e == cudaSuccess) {
    const int dbn = tc::tc_block_n_down(R, h->d.num_experts);
    int dtiles = tiles;
    if (dbn != bn) {  // its own list, written by the permutation
      a.tile_expert = h->dtile_expert;
      a.tile_row0 = h->dtile_row0;
      a.tile_rows = h->dtile_rows;
      a.n_tiles = h->n_dtiles;
      dtiles = std::min(h->max_tiles, (R + dbn - 1) / dbn + std::min(h->d.num_experts, R));
    }
    p0 = h->prof.begin(s);
    e = tc::launch_down_tc(L.map_dn, dbn == 64 ? h->map_a64 : h->map_a128, a, dbn, dtiles, s);
    h->prof.end("down_tc", p0, s);
  }
  if (e == cudaSuccess) {
    p0 = h->prof.begin(s);
    e = launch_combine(h->contrib, d_resid, d_out, T, K, H, h->status, s);
    h->prof.end("combine", p0, s);
  }
  if (e != cudaSuccess) return cuda_fail(h, e, "tensor expert launch");
  h->last_launches += 5;
  return MOE_OK;
}

moe_status layer_forward_locked(moe_handle *h, int layer, const float *d_h, const float *d_resid,
                                float *d_out, int T, uint32_t *d_ids, float *d_gates,
                                cudaStream_t s) {
  const LayerSlot &L = h->layers[layer];
  uint32_t *ids = d_ids ? d_ids : h->ids;
  float *gates = d_gates ? d_gates : h->gates;
  if (h->path == MOE_PATH_TENSOR && !use_tensor_path(h, L, T, d_h)) {
    set_err(h->err, "tensor-core path unavailable for layer %d (needs the packed expert layout, "
            "H and I multiples of 16, 16-byte aligned inputs)", layer);
    return MOE_ERR_STATE;
  }
  if (use_digits(h, T, layer, 1, d_h, d_resid)) {
    if (!digits_available(h, T, layer, 1, d_h, d_resid)) {
      set_err(h->err, "digit decode path unavailable for layer %d at T=%d (needs INT8 experts "
              "with 16-byte aligned rows, H and I multiples of 16 up to 2048, T*K <= %d, "
              "16-byte aligned inputs)", layer, T, kFusedMaxRoutes);
      return MOE_ERR_STATE;
    }
    DigitArgs a = digit_args(h, T);
    a.n_layers = 1;
    a.stacked = 0;
    a.layers = h->d_flayers + layer;
    a.h_in = d_h;
    a.resid = d_resid;
    a.out = d_out;
    a.ids_out = d_ids;
    a.gates_out = d_gates;
    if (!d_ids || !d_gates) a.ids_out = nullptr;
    a.router_async = h->layer_async[layer];
    cudaEvent_t p0 = h->prof.begin(s);
    cudaError_t e = launch_digit_decode(a, h->sm_count, s);
    h->prof.end("digit_decode", p0, s);
    if (e != cudaSuccess) return cuda_fail(h, e, "digit decode launch");
    h->last_launches += 1;
    if (d_ids && !d_gates) cudaMemcpyAsync(d_ids, h->ids, (size_t)T * h->d.top_k * 4,
                                           cudaMemcpyDeviceToDevice, s);
    if (d_gates && !d_ids) cudaMemcpyAsync(d_gates, h->gates, (size_t)T * h->d.top_k * 4,
                                           cudaMemcpyDeviceToDevice, s);
    return MOE_OK;
  }
  if (!use_tensor_path(h, L, T, d_h) && use_fused(h, T)) {
    FusedArgs f = fused_args(h, T);
    f.n_layers = 1;
    f.stacked = 0;
    f.layers = h->d_flayers + layer;
    f.h_in = d_h;
    f.resid = d_resid;
    f.out = d_out;
    f.ids_out = d_ids;
    f.gates_out = d_gates;
    f.int4 = L.int4;
    f.tiles = h->flayers[layer].tmaps != nullptr && ((uintptr_t)d_h & 15) == 0;
    if (!d_ids || !d_gates) f.ids_out = nullptr;
    const int vec = h->layer_vec[layer] && ((uintptr_t)d_h & 15) == 0;
    f.router_async = h->layer_async[layer] && ((uintptr_t)d_h & 15) == 0;
    cudaEvent_t p0 = h->prof.begin(s);
    cudaError_t e = launch_fused_decode(f, vec, h->sm_count, h->fbar, s);
    h->prof.end("fused_decode", p0, s);
    if (e != cudaSuccess) return cuda_fail(h, e, "fused decode launch");
    h->last_launches += 1;
    if (d_ids && !d_gates) cudaMemcpyAsync(d_ids, h->ids, (size_t)T * h->d.top_k * 4,
                                           cudaMemcpyDeviceToDevice, s);
    if (d_gates && !d_ids) cudaMemcpyAsync(d_gates, h->gates, (size_t)T * h->d.top_k * 4,
                                           cudaMemcpyDeviceToDevice, s);
    return MOE_OK;
  }
  const bool tc = use_tensor_path(h, L, T, d_h);
  const int R = T * h->d.top_k, E = h->d.num_experts;
  moe_status st = run_route(h, L, d_h, T, ids, gates, nullptr, s, true,
                            tc ? tc::tc_block_n(R, E) : 0, tc ? tc::tc_block_n_down(R, E) : 0);
  if (st != MOE_OK) return st;
  if (tc) return tensor_experts(h, L, d_h, d_resid, d_out, T, s);
  GemvArgs a{};
  a.H = h->d.hidden;
  a.I = h->d.intermediate;
  a.w_ptr = L.d_wptr;
  a.s_ptr = L.d_sptr;
  a.active = h->active;
  a.n_active_dev = h->n_active;
  a.n_active_max = std::min(h->d.num_experts, T * h->d.top_k);
  a.seg_off = h->seg_off;
  a.r_token = h->r_token;
  a.x = d_h;
  a.act = h->act;
  a.r_slot = h->r_slot;
  a.r_gate = h->r_gate;
  a.K = h->d.top_k;
  a.contrib = h->contrib;
  a.status = h->status;
  a.sm_count = h->sm_count;
  a.vec = L.vec && ((uintptr_t)d_h & 15) == 0;
  a.int4 = L.int4;
  cudaEvent_t p0 = h->prof.begin(s);
  cudaError_t e = launch_gate_up(a, s);
  h->prof.end("gate_up_gemv", p0, s);
  if (e == cudaSuccess) {
    p0 = h->prof.begin(s);
    e = launch_down(a, s);
    h->prof.end("down_gemv", p0, s);
  }
  if (e == cudaSuccess) {
    p0 = h->prof.begin(s);
    e = launch_combine(h->contrib, d_resid, d_out, T, h->d.top_k, h->d.hidden, h->status, s);
    h->prof.end("combine", p0, s);
  }
  if (e != cudaSuccess) return cuda_fail(h, e, "expert launch");
  h->last_launches += 3;
  return MOE_OK;
}

}  // namespace

extern "C" moe_status moe_create(int device, const moe_dims *dims, moe_handle **out) {
  if (!out || !dims) return MOE_ERR_INVALID;
  *out = nullptr;
  const moe_dims &d = *dims;
  if (d.hidden <= 0 || d.intermediate <= 0 || d.num_experts <= 0 || d.num_experts > kMaxExperts ||
      d.top_k <= 0 || d.top_k > kMaxTopK || d.top_k > d.num_experts || d.max_tokens <= 0 ||
      d.num_layers <= 0 || d.hidden > (1 << 16) || d.intermediate > (1 << 16))
    return MOE_ERR_INVALID;
  if (cudaSetDevice(device) != cudaSuccess) return MOE_ERR_CUDA;
  auto *h = new moe_handle();
  h->device = device;
  h->d = d;
  h->sm_count = sm_count_of(device);
  h->layers.resize(d.num_layers);
  const size_t T = d.max_tokens, H = d.hidden, I = d.intermediate, E = d.num_experts,
               K = d.top_k;
  bool ok = cudaStreamCreateWithFlags(&h->own_stream, cudaStreamNonBlocking) == cudaSuccess;
  h->stream = h->own_stream;
  ok = ok && dalloc(&h->logits, T * E) == cudaSuccess;
  ok = ok && dalloc(&h->ids, T * K) == cudaSuccess;
  ok = ok && dalloc(&h->gates, T * K) == cudaSuccess;
  ok = ok && dalloc(&h->r_gate, T * K) == cudaSuccess;
  ok = ok && dalloc(&h->r_token, T * K) == cudaSuccess;
  ok = ok && dalloc(&h->r_slot, T * K) == cudaSuccess;
  ok = ok && dalloc(&h->r_pos, T * K) == cudaSuccess;
  ok = ok && dalloc(&h->seg_off, E + 1) == cudaSuccess;
  ok = ok && dalloc(&h->active, E) == cudaSuccess;
  ok = ok && dalloc(&h->n_active, 1) == cudaSuccess;
  ok = ok && dalloc(&h->act, T * K * I) == cudaSuccess;
  ok = ok && dalloc(&h->contrib, T * K * H) == cudaSuccess;
  ok = ok && dalloc(&h->hbuf, T * H) == cudaSuccess;
  ok = ok && dalloc(&h->io_in, T * H) == cudaSuccess;
  ok = ok && dalloc(&h->io_out, T * H) == cudaSuccess;
  ok = ok && dalloc(&h->io_resid, T * H) == cudaSuccess;
  ok = ok && dalloc(&h->status, 1) == cudaSuccess;
  ok = ok && cudaMallocHost(&h->h_pin_in, 2 * T * H * sizeof(float)) == cudaSuccess;
  ok = ok && cudaMallocHost(&h->h_pin_out, T * H * sizeof(float)) == cudaSuccess;
  ok = ok && cudaMallocHost(&h->h_pin_status, 64) == cudaSuccess;
  ok = ok && cudaMallocHost(&h->h_pin_meta, 2 * T * K * sizeof(float)) == cudaSuccess;
  ok = ok && cudaMemset(h->status, 0, 4) == cudaSuccess;
  // tensor-core path scratch and the activation-side tensor maps
  const size_t R = T * K;
  h->max_tiles = (int)((R + 63) / 64 + std::min(E, R));  // bound for the 64-route tiles
  ok = ok && dalloc(&h->xq, 2 * R * H) == cudaSuccess;
  ok = ok && dalloc(&h->aq, 2 * R * I) == cudaSuccess;
  ok = ok && dalloc(&h->xs1, R) == cudaSuccess && dalloc(&h->xs2, R) == cudaSuccess;
  ok = ok && dalloc(&h->as1, R) == cudaSuccess && dalloc(&h->as2, R) == cudaSuccess;
  ok = ok && dalloc(&h->act_amax, R) == cudaSuccess;
  ok = ok && dalloc(&h->tile_expert, h->max_tiles) == cudaSuccess;
  ok = ok && dalloc(&h->tile_row0, h->max_tiles) == cudaSuccess;
  ok = ok && dalloc(&h->tile_rows, h->max_tiles) == cudaSuccess;
  ok = ok && dalloc(&h->n_tiles, 1) == cudaSuccess;
  ok = ok && dalloc(&h->dtile_expert, h->max_tiles) == cudaSuccess;
  ok = ok && dalloc(&h->dtile_row0, h->max_tiles) == cudaSuccess;
  ok = ok && dalloc(&h->dtile_rows, h->max_tiles) == cudaSuccess;
  ok = ok && dalloc(&h->n_dtiles, 1) == cudaSuccess;
  ok = ok && dalloc(&h->d_flayers, d.num_layers) == cudaSuccess;
  ok = ok && dalloc(&h->tok_cnt, T) == cudaSuccess && dalloc(&h->fbar, 1) == cudaSuccess;
  ok = ok && cudaMemset(h->tok_cnt, 0, T * sizeof(uint32_t)) == cudaSuccess;
  ok = ok && dalloc(&h->phase_ts, 16 + 3 * 1024) == cudaSuccess;  // + per-CTA start, end
  ok = ok && dalloc(&h->dbar, 2) == cudaSuccess &&
       cudaMemset(h->dbar, 0, 2 * sizeof(uint32_t)) == cudaSuccess;
  ok = ok && dalloc(&h->probe_flag, 1) == cudaSuccess &&
       cudaMemset(h->probe_flag, 0, sizeof(uint32_t)) == cudaSuccess;
  h->perm_scratch_words = permute_scratch_words((int)(T * K), (int)E);
  ok = ok && dalloc(&h->perm_scratch, h->perm_scratch_words) == cudaSuccess;
  h->flayers.assign(d.num_layers, FusedLayer{});
  h->layer_vec.assign(d.num_layers, 0);
  h->layer_async.assign(d.num_layers, 0);
  if (!ok) {
    free_handle(h);
    delete h;
    return MOE_ERR_NOMEM;
  }
  h->tc_ok = H % 16 == 0 && I % 16 == 0 &&
             tc::encode_map3d(&h->map_x64, h->xq, H, R, 2, H, R * H, 64) &&
             tc::encode_map3d(&h->map_x128, h->xq, H, R, 2, H, R * H, 128) &&
             tc::encode_map3d(&h->map_a64, h->aq, I, R, 2, I, R * I, 64) &&
             tc::encode_map3d(&h->map_a128, h->aq, I, R, 2, I, R * I, 128);
  *out = h;
  return MOE_OK;
}

extern "C" void moe_destroy(moe_handle *h) {
  if (!h) return;
  {
    DeviceGuard g(h->device);
    if (h->stream) cudaStreamSynchronize(h->stream);
    free_handle(h);
  }
  delete h;
}

extern "C" const char *moe_last_error(const moe_handle *h) {
  return h ? h->err.c_str() : "null handle";
}

extern "C" moe_status moe_set_stream(moe_handle *h, void *cuda_stream) {
  if (!h) return MOE_ERR_INVALID;
  std::lock_guard<std::mutex> lock(h->mu);
  h->stream = cuda_stream ? reinterpret_cast<cudaStream_t>(cuda_stream) : h->own_stream;
  return MOE_OK;
}

extern "C" moe_status moe_set_graphs(moe_handle *h, int enable) {
  if (!h) return MOE_ERR_INVALID;
  std::lock_guard<std::mutex> lock(h->mu);
  DeviceGuard g(h->device);
  drop_graphs(h);
  h->graphs_on = enable != 0;
  return MOE_OK;
}

extern "C" moe_status moe_set_route_mode(moe_handle *h, int mode) {
  if (!h || (mode != MOE_ROUTE_SOFTMAX_TOPK && mode != MOE_ROUTE_TOPK_SOFTMAX))
    return MOE_ERR_INVALID;
  std::lock_guard<std::mutex> lock(h->mu);
  h->route_mode = mode;
  return MOE_OK;
}

extern "C" moe_status moe_set_path(moe_handle *h, int path) {
  if (!h || path < MOE_PATH_AUTO || path > MOE_PATH_DIGITS) return MOE_ERR_INVALID;
  std::lock_guard<std::mutex> lock(h->mu);
  h->path = path;
  return MOE_OK;
}

extern "C" moe_status moe_set_wait_limit(moe_handle *h, uint64_t ns) {
  if (!h) return MOE_ERR_INVALID;
  std::lock_guard<std::mutex> lock(h->mu);
  if (ns == 0) {
    h->wait_barrier_cycles = kDefaultBarrierWaitCycles;
    h->wait_flag_cycles = kDefaultFlagWaitCycles;
  } else {
    // clock64() counts SM cycles: a bound in time becomes cycles at the
    // maximum SM clock (at a lower clock the wait lasts longer, never less)
    int khz = 0;
    if (cudaDeviceGetAttribute(&khz, cudaDevAttrClockRate, h->device) != cudaSuccess || khz <= 0)
      khz = 2000000;
    const double cyc = (double)ns * (double)khz * 1e-6;
    const long long c = cyc > 9e18 ? (long long)9e18 : std::max(1000LL, (long long)cyc);
    h->wait_barrier_cycles = c;
    h->wait_flag_cycles = c;
  }
  h->ep.P.wait_cycles = h->wait_flag_cycles;
  drop_graphs(h);  // captured launches carry the old bound
  return MOE_OK;
}

extern "C" moe_status moe_debug_wait_flag(moe_handle *h, void *stream) {
  if (!h) return MOE_ERR_INVALID;
  std::lock_guard<std::mutex> lock(h->mu);
  DeviceGuard g(h->device);
  cudaStream_t s = pick(h, stream);
  const cudaError_t e =
      launch_wait_probe(h->probe_flag, 1, 1u, h->wait_flag_cycles, h->status, s);
  return e == cudaSuccess ? MOE_OK : cuda_fail(h, e, "wait probe launch");
}

extern "C" moe_status moe_set_layer_q(moe_handle *h, int layer, const void *const *d_weights,
                                      const void *const *d_scales, const void *d_router,
                                      int router_dtype, int quant) {
  if (!h) return MOE_ERR_INVALID;
  std::lock_guard<std::mutex> lock(h->mu);
  drop_graphs(h);
  if (layer < 0 || layer >= (int)h->layers.size() || !d_weights || !d_scales || !d_router ||
      (router_dtype != MOE_ROUTER_F32 && router_dtype != MOE_ROUTER_BF16) ||
      (quant != MOE_QUANT_INT8 && quant != MOE_QUANT_INT4)) {
    set_err(h->err, "moe_set_layer: invalid argument");
    return MOE_ERR_INVALID;
  }
  const int int4 = quant == MOE_QUANT_INT4;
  if (int4 && ((h->d.hidden | h->d.intermediate) & 1)) {  // src/int8_expert.rs:116-118
    set_err(h->err, "hidden and intermediate must be even for INT4");
    return MOE_ERR_INVALID;
  }
  const int E = h->d.num_experts;
  int vec = 1;
  for (int e = 0; e < E; ++e) {
    if (!d_weights[e] || !d_scales[e] || ((uintptr_t)d_scales[e] & 3)) {
      set_err(h->err, "expert %d: null pointer or scales not 4-byte aligned", e);
      return MOE_ERR_INVALID;
    }
    vec &= ((uintptr_t)d_weights[e] & 7) == 0;
  }
  DeviceGuard g(h->device);
  LayerSlot &L = h->layers[layer];
  if (!L.d_wptr && (dalloc(&L.d_wptr, E) != cudaSuccess || dalloc(&L.d_sptr, E) != cudaSuccess))
    return MOE_ERR_NOMEM;
  cudaError_t e1 = cudaMemcpy(L.d_wptr, d_weights, E * sizeof(void *), cudaMemcpyHostToDevice);
  cudaError_t e2 = cudaMemcpy(L.d_sptr, d_scales, E * sizeof(void *), cudaMemcpyHostToDevice);
  if (e1 != cudaSuccess || e2 != cudaSuccess) return cuda_fail(h, e1 ? e1 : e2, "set_layer");
  L.router = d_router;
  L.router_dtype = router_dtype;
  L.vec = vec;
  L.int4 = int4;
  // Packed layout (expert e at base + e * 3IH, scales at sbase + e * (2I+H))
  // enables the tensor-core path (INT8 experts only).
  const size_t H = h->d.hidden, I = h->d.intermediate;
  const size_t wbytes = 3 * I * H / (int4 ? 2 : 1);
  bool packed = true;
  for (int e = 1; e < E && packed; ++e)
    packed = (const char *)d_weights[e] == (const char *)d_weights[0] + e * wbytes &&
             (const float *)d_scales[e] == (const float *)d_scales[0] + e * (2 * I + H);
  const char *wb = (const char *)d_weights[0];
  L.tc_ok = packed && !int4 && h->tc_ok &&
            tc::encode_map3d(&L.map_gu, wb, H, 2 * I, E, H, 3 * I * H, 128) &&
            tc::encode_map3d(&L.map_dn, wb + 2 * I * H, I, H, E, I, 3 * I * H, 128);
  bool align16 = true;
  for (int e = 0; e < E; ++e) align16 = align16 && ((uintptr_t)d_weights[e] & 15) == 0;
  FusedLayer &F = h->flayers[layer];
  F.w_ptr = L.d_wptr;
  F.s_ptr = L.d_sptr;
  F.router = d_router;
  F.router_dtype = router_dtype;
  F.int4 = int4;
  // bulk L2 prefetches need 16-byte aligned rows
  F.prefetch_ok = align16 && (H / (int4 ? 2 : 1)) % 16 == 0 && (I / (int4 ? 2 : 1)) % 16 == 0 &&
                  (!int4 || (H % 32 == 0 && I % 32 == 0));
  // Decode weight tiles: TMA boxes of 128 bytes x 32 (gate/up) or 64 (down)
  // rows over the packed layout; rows of whole 32-element chunks.
  // MOE_DECODE_TILES=0 keeps the per-thread weight loads.
  F.tmaps = nullptr;
  const size_t hb = int4 ? H / 2 : H, ib = int4 ? I / 2 : I;
  const char *tiles_env = getenv("MOE_DECODE_TILES");
  if (packed && align16 && H % 32 == 0 && I % 32 == 0 && hb >= 128 && ib >= 128 && H >= 64 &&
      !(tiles_env && tiles_env[0] == '0')) {
    CUtensorMap m[2];
    if (tc::encode_map3d(&m[0], wb, hb, 2 * I, E, hb, wbytes, 32) &&
        tc::encode_map3d(&m[1], wb + 2 * I * hb, ib, H, E, ib, wbytes, 64)) {
      // the maps are an optimisation: without room for them the layer keeps
      // per-thread weight loads
      if (L.d_tmaps || cudaMalloc(&L.d_tmaps, sizeof m) == cudaSuccess) {
        const cudaError_t em = cudaMemcpy(L.d_tmaps, m, sizeof m, cudaMemcpyHostToDevice);
        if (em != cudaSuccess) return cuda_fail(h, em, "set_layer");
        F.tmaps = L.d_tmaps;
      } else {
        L.d_tmaps = nullptr;
        cudaGetLastError();  // clear the (non-sticky) allocation error
      }
    }
  }
  h->layer_vec[layer] = vec;
  h->layer_async[layer] = router_dtype == MOE_ROUTER_F32 && ((uintptr_t)d_router & 15) == 0 &&
                          H % 4 == 0;
  const cudaError_t e3 =
      cudaMemcpy(h->d_flayers + layer, &F, sizeof(FusedLayer), cudaMemcpyHostToDevice);
  if (e3 != cudaSuccess) return cuda_fail(h, e3, "set_layer");
  L.set = true;
  if (L.own_w && L.own_w != d_weights[0]) {  // the slot no longer uses a loaded copy
    cudaFree(L.own_w);
    cudaFree(L.own_s);
    cudaFree(L.own_r);
    L.own_w = L.own_s = L.own_r = nullptr;
  }
  return MOE_OK;
}

extern "C" moe_status moe_set_layer(moe_handle *h, int layer, const void *const *d_weights,
                                    const void *const *d_scales, const void *d_router,
                                    int router_dtype) {
  return moe_set_layer_q(h, layer, d_weights, d_scales, d_router, router_dtype, MOE_QUANT_INT8);
}

namespace {
// IEEE binary16 -> binary32, exact (every half is a float).
float half_to_float(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1Fu, man = h & 0x3FFu;
  uint32_t bits;
  if (exp == 0x1F) {
    bits = sign | 0x7F800000u | (man << 13);  // inf / nan
  } else if (exp != 0) {
    bits = sign | ((exp + 112u) << 23) | (man << 13);
  } else if (man == 0) {
    bits = sign;  // signed zero
  } else {  // subnormal half: normalise
    int e = -1;
    do {
      man <<= 1;
      ++e;
    } while (!(man & 0x400u));
    bits = sign | ((uint32_t)(112 - e) << 23) | ((man & 0x3FFu) << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}
}  // namespace

extern "C" moe_status moe_set_layer_norm(moe_handle *h, int layer, const float *d_norm_w) {
  if (!h) return MOE_ERR_INVALID;
  std::lock_guard<std::mutex> lock(h->mu);
  if (layer < 0 || layer >= (int)h->layers.size() || ((uintptr_t)d_norm_w & 3)) {
    set_err(h->err, "moe_set_layer_norm: invalid argument");
    return MOE_ERR_INVALID;
  }
  drop_graphs(h);
  DeviceGuard g(h->device);
  FusedLayer &F = h->flayers[layer];
  F.norm_w = d_norm_w;
  const cudaError_t e =
      cudaMemcpy(h->d_flayers + layer, &F, sizeof(FusedLayer), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return cuda_fail(h, e, "set_layer_norm");
  LayerSlot &L = h->layers[layer];
  if (L.own_n && L.own_n != d_norm_w) {  // the slot no longer uses a loaded copy
    cudaFree(L.own_n);
    L.own_n = nullptr;
  }
  return MOE_OK;
}

extern "C" moe_status moe_load_layer(moe_handle *h, const moe_ckpt *c, int ckpt_layer,
                                     int layer, int keep_bf16) {
  if (!h || !c || ckpt_layer < 0) return MOE_ERR_INVALID;
  const size_t E = h->d.num_experts, H = h->d.hidden, I = h->d.intermediate;
  const size_t wcount = 3 * I * H, scount = 2 * I + H;
  auto fail = [&](moe_status st, const std::string &m) {
    std::lock_guard<std::mutex> lock(h->mu);
    set_err(h->err, "%s", m.c_str());
    return st;
  };
  if (layer < 0 || layer >= (int)h->layers.size()) return fail(MOE_ERR_INVALID, "layer out of range");
  // descriptors first, no payload read (src/olmoe.rs:1080-1099)
  // INT8: I8 [3IH]; INT4: U8 [3IH/2] (src/int8_expert.rs:107-122, src/olmoe.rs:1086-1091);
  // every expert of the layer in the same format
  std::vector<const CkptTensor *> wt(E), st(E);
  int int4 = -1;
  for (size_t e = 0; e < E; ++e) {
    const std::string pre = "model.layers." + std::to_string(ckpt_layer) + ".mlp.experts." +
                            std::to_string(e);
    wt[e] = ckpt_find(c, pre + ".merged_weight");
    st[e] = ckpt_find(c, pre + ".qs");
    if (!wt[e]) return fail(MOE_ERR_INVALID, "missing tensor: " + pre + ".merged_weight");
    if (!st[e]) return fail(MOE_ERR_INVALID, "missing tensor: " + pre + ".qs");
    const auto &ws = wt[e]->shape;
    int q = -1;
    if (wt[e]->dtype == MOE_DT_I8 && ws.size() == 1 && (size_t)ws[0] == wcount) q = 0;
    else if (wt[e]->dtype == MOE_DT_U8 && ws.size() == 1 && (size_t)ws[0] == wcount / 2 &&
             H % 2 == 0 && I % 2 == 0)
      q = 1;
    if (q < 0 || (int4 >= 0 && q != int4) || st[e]->dtype != MOE_DT_F32 ||
        st[e]->shape.size() != 1 || (size_t)st[e]->shape[0] != scount)
      return fail(MOE_ERR_INVALID, pre + ": invalid merged expert layout");
    int4 = q;
  }
  const size_t wbytes = int4 ? wcount / 2 : wcount;
  const std::string rname = "model.layers." + std::to_string(ckpt_layer) + ".mlp.gate.weight";
  const CkptTensor *rt = ckpt_find(c, rname);
  if (!rt) return fail(MOE_ERR_INVALID, "missing tensor: " + rname);
  if (rt->shape.size() != 2 || (size_t)rt->shape[0] != E || (size_t)rt->shape[1] != H ||
      (rt->dtype != MOE_DT_F32 && rt->dtype != MOE_DT_BF16 && rt->dtype != MOE_DT_F16))
    return fail(MOE_ERR_INVALID, rname + ": incorrect shape or dtype");
  // router on the host: finite values, kept bf16 or widened to f32
  std::vector<uint8_t> raw(rt->bytes);
  if (!ckpt_read(c, *rt, raw.data())) return fail(MOE_ERR_INVALID, rname + ": short read");
  const bool bf16 = rt->dtype == MOE_DT_BF16 && keep_bf16;
  std::vector<float> rf(E * H);
  for (size_t i = 0; i < E * H; ++i) {
    if (rt->dtype == MOE_DT_F32) {
      memcpy(&rf[i], &raw[4 * i], 4);
    } else {
      uint16_t b;
      memcpy(&b, &raw[2 * i], 2);
      if (rt->dtype == MOE_DT_F16) {
        rf[i] = half_to_float(b);
      } else {
        const uint32_t bits = (uint32_t)b << 16;
        memcpy(&rf[i], &bits, 4);
      }
    }
    if (!std::isfinite(rf[i])) return fail(MOE_ERR_NONFINITE, rname + ": non-finite value");
  }
  DeviceGuard g(h->device);
  int8_t *dw = nullptr;
  float *ds = nullptr;
  void *dr = nullptr;
  uint8_t *stage = nullptr;
  auto release = [&] {
    cudaFree(dw);
    cudaFree(ds);
    cudaFree(dr);
    cudaFreeHost(stage);
  };
  if (cudaMalloc(&dw, E * wbytes) != cudaSuccess || cudaMalloc(&ds, E * scount * 4) != cudaSuccess ||
      cudaMalloc(&dr, bf16 ? E * H * 2 : E * H * 4) != cudaSuccess ||
      cudaMallocHost(&stage, wbytes + scount * 4) != cudaSuccess) {
    release();
    return fail(MOE_ERR_NOMEM, "moe_load_layer: out of memory");
  }
  // experts one by one through a pinned staging buffer
  for (size_t e = 0; e < E; ++e) {
    float *sc = reinterpret_cast<float *>(stage + wbytes);
    if (!ckpt_read(c, *wt[e], stage) || !ckpt_read(c, *st[e], sc)) {
      release();
      return fail(MOE_ERR_INVALID, "expert " + std::to_string(e) + ": short read");
    }
    for (size_t i = 0; i < scount; ++i)
      if (!std::isfinite(sc[i]) || !(sc[i] > 0.0f)) {  // src/int8_expert.rs:151-153
        release();
        return fail(MOE_ERR_INVALID, "expert scales must be finite and positive");
      }
    if (cudaMemcpy(dw + e * wbytes, stage, wbytes, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(ds + e * scount, sc, scount * 4, cudaMemcpyHostToDevice) != cudaSuccess) {
      release();
      return fail(MOE_ERR_CUDA, "moe_load_layer: upload failed");
    }
  }
  const cudaError_t ce = bf16 ? cudaMemcpy(dr, raw.data(), E * H * 2, cudaMemcpyHostToDevice)
                              : cudaMemcpy(dr, rf.data(), E * H * 4, cudaMemcpyHostToDevice);
  cudaFreeHost(stage);
  stage = nullptr;
  if (ce != cudaSuccess) {
    release();
    return fail(MOE_ERR_CUDA, "moe_load_layer: router upload failed");
  }
  // the post-attention RMSNorm gain, when the checkpoint has it
  // (src/olmoe.rs:1057, applied at :2583-2588)
  const std::string nname =
      "model.layers." + std::to_string(ckpt_layer) + ".post_attention_layernorm.weight";
  float *dn = nullptr;
  if (const CkptTensor *nt = ckpt_find(c, nname)) {
    if (nt->shape.size() != 1 || (size_t)nt->shape[0] != H ||
        (nt->dtype != MOE_DT_F32 && nt->dtype != MOE_DT_BF16 && nt->dtype != MOE_DT_F16)) {
      release();
      return fail(MOE_ERR_INVALID, nname + ": incorrect shape or dtype");
    }
    std::vector<uint8_t> nraw(nt->bytes);
    std::vector<float> nw(H);
    if (!ckpt_read(c, *nt, nraw.data())) {
      release();
      return fail(MOE_ERR_INVALID, nname + ": short read");
    }
    for (size_t i = 0; i < H; ++i) {
      if (nt->dtype == MOE_DT_F32) {
        memcpy(&nw[i], &nraw[4 * i], 4);
      } else {
        uint16_t b;
        memcpy(&b, &nraw[2 * i], 2);
        if (nt->dtype == MOE_DT_F16) {
          nw[i] = half_to_float(b);
        } else {
          const uint32_t bits = (uint32_t)b << 16;
          memcpy(&nw[i], &bits, 4);
        }
      }
      if (!std::isfinite(nw[i])) {
        release();
        return fail(MOE_ERR_NONFINITE, nname + ": non-finite value");
      }
    }
    if (cudaMalloc(&dn, H * 4) != cudaSuccess ||
        cudaMemcpy(dn, nw.data(), H * 4, cudaMemcpyHostToDevice) != cudaSuccess) {
      cudaFree(dn);
      release();
      return fail(MOE_ERR_NOMEM, "moe_load_layer: norm upload failed");
    }
  }
  const moe_status st2 = moe_set_layer_packed_q(h, layer, dw, ds, dr,
                                                bf16 ? MOE_ROUTER_BF16 : MOE_ROUTER_F32,
                                                int4 ? MOE_QUANT_INT4 : MOE_QUANT_INT8);
  if (st2 != MOE_OK) {
    cudaFree(dn);
    release();
    return st2;
  }
  const moe_status st3 = moe_set_layer_norm(h, layer, dn);
  std::lock_guard<std::mutex> lock(h->mu);
  LayerSlot &L = h->layers[layer];
  L.own_w = dw;
  L.own_s = ds;
  L.own_r = dr;
  L.own_n = dn;
  return st3;
}

extern "C" moe_status moe_set_layer_packed_q(moe_handle *h, int layer, const void *d_experts,
                                             const float *d_scales, const void *d_router,
                                             int router_dtype, int quant) {
  if (!h || !d_experts || !d_scales) return MOE_ERR_INVALID;
  const size_t E = h->d.num_experts, H = h->d.hidden, I = h->d.intermediate;
  const size_t wbytes = 3 * I * H / (quant == MOE_QUANT_INT4 ? 2 : 1);
  std::vector<const void *> w(E), s(E);
  for (size_t e = 0; e < E; ++e) {
    w[e] = static_cast<const int8_t *>(d_experts) + e * wbytes;
    s[e] = d_scales + e * (2 * I + H);
  }
  return moe_set_layer_q(h, layer, w.data(), s.data(), d_router, router_dtype, quant);
}

extern "C" moe_status moe_set_layer_packed(moe_handle *h, int layer, const int8_t *d_experts,
                                           const float *d_scales, const void *d_router,
                                           int router_dtype) {
  return moe_set_layer_packed_q(h, layer, d_experts, d_scales, d_router, router_dtype,
                                MOE_QUANT_INT8);
}

extern "C" moe_status moe_route(moe_handle *h, int layer, const float *d_h, int T,
                                uint32_t *d_ids, float *d_gates, float *d_probs, void *stream) {
  if (!h || !d_h || !d_ids || !d_gates) return MOE_ERR_INVALID;
  std::lock_guard<std::mutex> lock(h->mu);
  drop_graphs(h);
  // routing needs only the router: a layer registered for expert
  // parallelism (moe_ep_set_layer) routes too
  moe_status st = check_layer(h, layer, T);
  if (st == MOE_ERR_STATE && h->layers[layer].router) {
    st = MOE_OK;
    if (T < 0 || T > h->d.max_tokens) {
      set_err(h->err, "token count %d outside [0, %d]", T, h->d.max_tokens);
      st = MOE_ERR_INVALID;
    }
  }
  if (st != MOE_OK || T == 0) return st;
  DeviceGuard g(h->device);
  h->last_launches = 0;
  return run_route(h, h->layers[layer], d_h, T, d_ids, d_gates, d_probs, pick(h, stream), false);
}

extern "C" moe_status moe_route_permute(moe_handle *h, int layer, const float *d_h, int T,
                                        uint32_t *d_ids, float *d_gates, int32_t *d_seg_off,
                                        int32_t *d_route_token, int32_t *d_route_slot,
                                        void *stream) {
  if (!h || !d_h || !d_ids || !d_gates || !d_seg_off || !d_route_token || !d_route_slot)
    return MOE_ERR_INVALID;
  std::lock_guard<std::mutex> lock(h->mu);
  moe_status st = check_layer(h, layer, T);
  if (st != MOE_OK || T == 0) return st;
  DeviceGuard g(h->device);
  h->last_launches = 0;
  cudaStream_t s = pick(h, stream);
  st = run_route(h, h->layers[layer], d_h, T, d_ids, d_gates, nullptr, s, true);
  if (st != MOE_OK) return st;
  const size_t R = (size_t)T * h->d.top_k;
  cudaMemcpyAsync(d_seg_off, h->seg_off, (h->d.num_experts + 1) * 4, cudaMemcpyDeviceToDevice, s);
  cudaMemcpyAsync(d_route_token, h->r_token, R * 4, cudaMemcpyDeviceToDevice, s);
  cudaError_t e = cudaMemcpyAsync(d_route_slot, h->r_slot, R * 4, cudaMemcpyDeviceToDevice, s);
  return e == cudaSuccess ? MOE_OK : cuda_fail(h, e, "route_permute copy");
}

extern "C" moe_status moe_layer_forward(moe_handle *h, int layer, const float *d_h,
                                        const float *d_resid, float *d_out, int T,
                                        uint32_t *d_ids, float *d_gates, void *stream) {
  if (!h || !d_h || !d_out) return MOE_ERR_INVALID;
  std::lock_guard<std::mutex> lock(h->mu);
  moe_status st = check_layer(h, layer, T);
  if (st != MOE_OK || T == 0) return st;
  DeviceGuard g(h->device);
  h->last_launches = 0;
  cudaStream_t s = pick(h, stream);
  const uint64_t key[10] = {1, (uint64_t)layer, (uint64_t)T, (uint64_t)d_h, (uint64_t)d_resid,
                            (uint64_t)d_out, (uint64_t)d_ids, (uint64_t)d_gates, (uint64_t)s,
                            (uint64_t)(h->path * 16 + h->route_mode)};
  return graphed(h, key, s, [&] {
    h->last_launches = 0;
    return layer_forward_locked(h, layer, d_h, d_resid, d_out, T, d_ids, d_gates, s);
  });
}

moe_status stack_forward_locked(moe_handle *h, int first_layer, int n_layers, float *d_x, int T,
                                float rms_eps, cudaStream_t s);

extern "C" moe_status moe_stack_forward(moe_handle *h, int first_layer, int n_layers, float *d_x,
                                        int T, float rms_eps, void *stream) {
  if (!h || !d_x || n_layers <= 0) return MOE_ERR_INVALID;
  std::lock_guard<std::mutex> lock(h->mu);
  for (int l = first_layer; l < first_layer + n_layers; ++l) {
    moe_status st = check_layer(h, l, T);
    if (st != MOE_OK) return st;
  }
  if (T == 0) return MOE_OK;
  DeviceGuard g(h->device);
  cudaStream_t s = pick(h, stream);
  h->last_launches = 0;
  uint32_t eps_bits;
  memcpy(&eps_bits, &rms_eps, 4);
  const uint64_t key[10] = {2, (uint64_t)first_layer, (uint64_t)n_layers, (uint64_t)T,
                            (uint64_t)d_x, eps_bits, (uint64_t)s,
                            (uint64_t)(h->path * 16 + h->route_mode), 0, 0};
  return graphed(h, key, s, [&] {
    h->last_launches = 0;
    return stack_forward_locked(h, first_layer, n_layers, d_x, T, rms_eps, s);
  });
}

moe_status stack_forward_locked(moe_handle *h, int first_layer, int n_layers, float *d_x, int T,
                                float rms_eps, cudaStream_t s) {
  bool vec_all = ((uintptr_t)d_x & 15) == 0;
  for (int l = first_layer; l < first_layer + n_layers; ++l) vec_all = vec_all && h->layer_vec[l];
  const int quant = layers_quant(h, first_layer, n_layers);
  if (use_digits(h, T, first_layer, n_layers, d_x, nullptr)) {
    if (!digits_available(h, T, first_layer, n_layers, d_x, nullptr)) {
      set_err(h->err, "digit decode path unavailable for layers [%d, %d) at T=%d (needs INT8 "
              "experts with 16-byte aligned rows, H and I multiples of 16 up to 2048, "
              "T*K <= %d, a 16-byte aligned x)", first_layer, first_layer + n_layers, T,
              kFusedMaxRoutes);
      return MOE_ERR_STATE;
    }
    DigitArgs a = digit_args(h, T);
    a.n_layers = n_layers;
    a.stacked = 1;
    a.layers = h->d_flayers + first_layer;
    a.out = d_x;
    a.eps = rms_eps;
    a.router_async = 1;
    for (int l = first_layer; l < first_layer + n_layers; ++l)
      a.router_async = a.router_async && h->layer_async[l];
    cudaEvent_t p0 = h->prof.begin(s);
    cudaError_t e = launch_digit_decode(a, h->sm_count, s);
    h->prof.end("digit_decode", p0, s);
    if (e != cudaSuccess) return cuda_fail(h, e, "digit decode launch");
    h->last_launches += 1;
    return MOE_OK;
  }
  // AUTO: the tensor-core layers when every layer can take them at T (as
  // single-layer calls do), else the exact single launch for small T
  bool all_tc = h->path == MOE_PATH_AUTO;
  for (int l = first_layer; all_tc && l < first_layer + n_layers; ++l)
    all_tc = use_tensor_path(h, h->layers[l], T, h->hbuf);
  if (h->path != MOE_PATH_TENSOR && !all_tc && use_fused(h, T) && quant >= 0) {
    FusedArgs f = fused_args(h, T);
    f.n_layers = n_layers;
    f.stacked = 1;
    f.int4 = quant;
    f.tiles = 1;
    for (int l = first_layer; l < first_layer + n_layers; ++l)
      f.tiles = f.tiles && h->flayers[l].tmaps != nullptr;
    f.layers = h->d_flayers + first_layer;
    f.out = d_x;
    f.hbuf = h->hbuf;
    f.eps = rms_eps;
    f.router_async = 1;
    for (int l = first_layer; l < first_layer + n_layers; ++l)
      f.router_async = f.router_async && h->layer_async[l];
    cudaEvent_t p0 = h->prof.begin(s);
    cudaError_t e = launch_fused_decode(f, vec_all ? 1 : 0, h->sm_count, h->fbar, s);
    h->prof.end("fused_decode", p0, s);
    if (e != cudaSuccess) return cuda_fail(h, e, "fused decode launch");
    h->last_launches += 1;
    return MOE_OK;
  }
  for (int l = first_layer; l < first_layer + n_layers; ++l) {
    cudaEvent_t p0 = h->prof.begin(s);
    cudaError_t e = launch_rmsnorm(d_x, h->flayers[l].norm_w, h->hbuf, T, h->d.hidden, rms_eps,
                                   h->status, s);
    h->prof.end("rmsnorm", p0, s);
    if (e != cudaSuccess) return cuda_fail(h, e, "rmsnorm launch");
    h->last_launches += 1;
    moe_status st = layer_forward_locked(h, l, h->hbuf, d_x, d_x, T, nullptr, nullptr, s);
    if (st != MOE_OK) return st;
  }
  return MOE_OK;
}

static moe_status status_error(moe_handle *h, uint32_t st) {
  if (st & kStatusTimeout) {
    set_err(h->err, "device wait timed out");
    return MOE_ERR_TIMEOUT;
  }
  if (st & kStatusNonFinite) {
    set_err(h->err, "non-finite computation result");
    return MOE_ERR_NONFINITE;
  }
  if (st & kStatusBadRoute) {
    set_err(h->err, "routing produced an invalid expert id");
    return MOE_ERR_INVALID;
  }
  return MOE_OK;
}

extern "C" moe_status moe_sync_status(moe_handle *h, void *stream) {
  if (!h) return MOE_ERR_INVALID;
  std::lock_guard<std::mutex> lock(h->mu);
  DeviceGuard g(h->device);
  cudaStream_t s = pick(h, stream);
  uint32_t st = 0;
  cudaError_t e = cudaMemcpyAsync(&st, h->status, 4, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(h, e, "sync_status");
  if (st) cudaMemsetAsync(h->status, 0, 4, s);
  return status_error(h, st);
}

// Host memory that the CUDA driver has pinned (cudaHostAlloc, cudaHostRegister,
// torch pin_memory) can be read and written by the copy engines directly.
static bool host_is_pinned(const void *p) {
  cudaPointerAttributes at{};
  if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return at.type == cudaMemoryTypeHost;
}

// Pageable buffers are staged through the handle's pinned buffers in chunks,
// so the host copy of one chunk overlaps the DMA of the previous one.
static constexpr size_t kStageChunk = 1u << 20;
static constexpr int kStageEvents = 16;

static size_t stage_chunk(size_t bytes) {
  return std::max(kStageChunk, ((bytes + kStageEvents - 1) / kStageEvents + 255) & ~(size_t)255);
}

static void h2d(void *dst, const void *src, size_t bytes, void *pin, bool pinned,
                cudaStream_t s) {
  if (pinned) {
    cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, s);
    return;
  }
  const size_t c = stage_chunk(bytes);
  for (size_t o = 0; o < bytes; o += c) {
    const size_t n = std::min(c, bytes - o);
    memcpy(static_cast<char *>(pin) + o, static_cast<const char *>(src) + o, n);
    cudaMemcpyAsync(static_cast<char *>(dst) + o, static_cast<char *>(pin) + o, n,
                    cudaMemcpyHostToDevice, s);
  }
}

// Token chunks of the host-buffer call.  A layer's result for a token
// depends on that token's row alone (routing, digitisation and the int32
// tensor-core sums are per route), so a chunk's outputs, ids and gates are
// bit-identical to the whole batch's.  Chunk c's layer runs on the handle's
// stream while chunk c + 1 comes in on one copy stream and chunk c - 1 goes
// back on another, so the PCIe transfers hide behind the tensor-core work.
// MOE_HOST_CHUNK sets the chunk in tokens (0: whole batch).
static constexpr int kHostChunksMax = 8;
static constexpr int kHostChunkDefault = 1024;

static int host_chunk_tokens(moe_handle *h, int layer, int T) {
  static int env = -1;
  if (env < 0) {
    const char *v = getenv("MOE_HOST_CHUNK");
    env = v ? std::max(0, atoi(v)) : kHostChunkDefault;
    if (env > 0) env = std::max(env, 256);
  }
  if (env == 0 || T < 2 * env) return T;
  const int n = std::min(kHostChunksMax, T / env);
  const int c = ((T + n - 1) / n + 15) & ~15;
  // every chunk, the last (shortest) one included, must take the tensor-core
  // path, whose outputs do not depend on the batch composition
  const LayerSlot &L = h->layers[layer];
  if (!use_tensor_path(h, L, c, h->io_in) || !use_tensor_path(h, L, T - (n - 1) * c, h->io_in))
    return T;
  return c;
}

static bool host_streams(moe_handle *h) {
  if (h->io_stream[0]) return true;
  bool ok = true;
  for (auto &st : h->io_stream)
    ok = ok && cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) == cudaSuccess;
  for (auto &row : h->io_ev)
    for (auto &ev : row)
      ok = ok && cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) == cudaSuccess;
  if (!ok) cudaGetLastError();
  return ok;
}

extern "C" moe_status moe_layer_forward_host(moe_handle *h, int layer, const float *h_in,
                                             const float *h_resid, float *h_out, int T,
                                             uint32_t *h_ids, float *h_gates) {
  if (!h || !h_in || !h_out) return MOE_ERR_INVALID;
  std::lock_guard<std::mutex> lock(h->mu);
  moe_status st = check_layer(h, layer, T);
  if (st != MOE_OK || T == 0) return st;
  DeviceGuard g(h->device);
  cudaStream_t s = h->stream;
  const size_t H = h->d.hidden, K = h->d.top_k;
  const size_t R = (size_t)T * K;
  const size_t bytes = (size_t)T * H * sizeof(float);
  int ct = host_chunk_tokens(h, layer, T);
  if (ct < T && !host_streams(h)) ct = T;
  const int nch = (T + ct - 1) / ct;
  // one chunk: everything in order on the handle's stream
  cudaStream_t si = nch > 1 ? h->io_stream[0] : s, so = nch > 1 ? h->io_stream[1] : s;
  const bool pin_in = host_is_pinned(h_in);
  const bool pin_resid = h_resid && host_is_pinned(h_resid);
  const bool pin_out = host_is_pinned(h_out);
  if (!pin_out && !h->stage_ev[0])
    for (auto &ev : h->stage_ev) cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
  // pageable outputs come back through the pinned staging in pieces, each
  // copied out on the host as soon as its event has fired
  const size_t piece = stage_chunk(bytes);
  std::vector<std::pair<size_t, size_t>> pieces;
  auto drain = [&] {
    cudaStreamSynchronize(si);
    cudaStreamSynchronize(s);
    cudaStreamSynchronize(so);
  };
  int launches = 0;
  for (int c = 0; c < nch; ++c) {
    const size_t t0 = (size_t)c * ct, tc = std::min((size_t)ct, (size_t)T - t0);
    const size_t o = t0 * H, cb = tc * H * sizeof(float);
    h2d(h->io_in + o, h_in + o, cb, h->h_pin_in + o, pin_in, si);
    if (h_resid)
      h2d(h->io_resid + o, h_resid + o, cb, h->h_pin_in + (size_t)T * H + o, pin_resid, si);
    if (si != s) {
      cudaEventRecord(h->io_ev[0][c], si);
      cudaStreamWaitEvent(s, h->io_ev[0][c], 0);
    }
    const float *d_h = h->io_in + o, *d_resid = h_resid ? h->io_resid + o : nullptr;
    float *d_out = h->io_out + o;
    uint32_t *d_ids = h->ids + t0 * K;
    float *d_gates = h->gates + t0 * K;
    const uint64_t key[10] = {1, (uint64_t)layer, (uint64_t)tc, (uint64_t)d_h,
                              (uint64_t)d_resid, (uint64_t)d_out, (uint64_t)d_ids,
                              (uint64_t)d_gates, (uint64_t)s,
                              (uint64_t)(h->path * 16 + h->route_mode)};
    h->last_launches = 0;
    st = graphed(h, key, s, [&] {
      h->last_launches = 0;
      return layer_forward_locked(h, layer, d_h, d_resid, d_out, (int)tc, d_ids, d_gates, s);
    });
    if (st != MOE_OK) {
      drain();
      return st;
    }
    launches += h->last_launches;
    if (so != s) {
      cudaEventRecord(h->io_ev[1][c], s);
      cudaStreamWaitEvent(so, h->io_ev[1][c], 0);
    }
    if (pin_out) {
      cudaMemcpyAsync(h_out + o, d_out, cb, cudaMemcpyDeviceToHost, so);
    } else {
      for (size_t p = 0; p < cb; p += piece) {
        const size_t n = std::min(piece, cb - p);
        cudaMemcpyAsync(reinterpret_cast<char *>(h->h_pin_out + o) + p,
                        reinterpret_cast<const char *>(d_out) + p, n, cudaMemcpyDeviceToHost,
                        so);
        cudaEventRecord(h->stage_ev[pieces.size()], so);
        pieces.emplace_back(o * sizeof(float) + p, n);
      }
    }
  }
  h->last_launches = launches;
  // ids, gates and the status word follow the last chunk's layer; the status
  // is cleared behind them, so the call needs one synchronisation per stream
  const bool pin_ids = h_ids && host_is_pinned(h_ids);
  const bool pin_gates = h_gates && host_is_pinned(h_gates);
  uint32_t *ids_dst = pin_ids ? h_ids : reinterpret_cast<uint32_t *>(h->h_pin_meta);
  float *gates_dst = pin_gates ? h_gates : h->h_pin_meta + R;
  if (h_ids) cudaMemcpyAsync(ids_dst, h->ids, R * 4, cudaMemcpyDeviceToHost, so);
  if (h_gates) cudaMemcpyAsync(gates_dst, h->gates, R * 4, cudaMemcpyDeviceToHost, so);
  cudaMemcpyAsync(h->h_pin_status, h->status, 4, cudaMemcpyDeviceToHost, so);
  cudaMemsetAsync(h->status, 0, 4, so);
  cudaError_t e = cudaSuccess;
  for (size_t i = 0; i < pieces.size() && e == cudaSuccess; ++i) {
    e = cudaEventSynchronize(h->stage_ev[i]);
    if (e == cudaSuccess)
      memcpy(reinterpret_cast<char *>(h_out) + pieces[i].first,
             reinterpret_cast<const char *>(h->h_pin_out) + pieces[i].first, pieces[i].second);
  }
  for (cudaStream_t x : {so, s, si}) {
    const cudaError_t e2 = cudaStreamSynchronize(x);
    if (e == cudaSuccess) e = e2;
  }
  if (e == cudaSuccess && h_ids && !pin_ids) memcpy(h_ids, ids_dst, R * 4);
  if (e == cudaSuccess && h_gates && !pin_gates) memcpy(h_gates, gates_dst, R * 4);
  if (e != cudaSuccess) return cuda_fail(h, e, "layer_forward_host");
  return status_error(h, *h->h_pin_status);
}

extern "C" moe_status moe_host_alloc(size_t bytes, void **out) {
  if (!out || bytes == 0) return MOE_ERR_INVALID;
  *out = nullptr;
  return cudaHostAlloc(out, bytes, cudaHostAllocPortable) == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

extern "C" moe_status moe_host_free(void *p) {
  if (!p) return MOE_OK;
  return cudaFreeHost(p) == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

extern "C" int moe_last_launch_count(const moe_handle *h) { return h ? h->last_launches : 0; }

extern "C" moe_status moe_synth_expert(uint64_t seed, int layer, int expert, int hidden,
                                       int intermediate, int8_t *d_weights, float *d_scales,
                                       void *stream) {
  if (!d_weights || !d_scales || hidden <= 0 || intermediate <= 0) return MOE_ERR_INVALID;
  cudaError_t e = launch_synth_expert(seed, layer, expert, hidden, intermediate, d_weights,
                                      d_scales, reinterpret_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

extern "C" moe_status moe_debug_expf(uint32_t bits_lo, uint32_t count, float *d_out,
                                     void *stream) {
  if (!d_out) return MOE_ERR_INVALID;
  cudaError_t e = launch_expf_eval(bits_lo, count, d_out, reinterpret_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

extern "C" moe_status moe_debug_stream_read(const void *d_buf, size_t bytes, uint32_t *d_sink,
                                            void *stream) {
  if (!d_buf || !d_sink || bytes % 16 || ((uintptr_t)d_buf & 15)) return MOE_ERR_INVALID;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return MOE_ERR_CUDA;
  const cudaError_t e = launch_stream_read(d_buf, bytes, d_sink, sm_count_of(dev),
                                           reinterpret_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? MOE_OK : MOE_ERR_CUDA;
}

extern "C" moe_status moe_profile_enable(moe_handle *h, int enable) {
  if (!h) return MOE_ERR_INVALID;
  std::lock_guard<std::mutex> lock(h->mu);
  h->prof.on = enable != 0;
  return MOE_OK;
}

extern "C" moe_status moe_profile_read(moe_handle *h, moe_kernel_time *out, int max_entries,
                                       int *n_entries) {
  if (!h || !n_entries || (max_entries > 0 && !out)) return MOE_ERR_INVALID;
  std::lock_guard<std::mutex> lock(h->mu);
  DeviceGuard g(h->device);
  std::vector<moe_kernel_time> acc;
  for (auto &r : h->prof.recs) {
    if (cudaEventSynchronize(r.b) != cudaSuccess) return cuda_fail(h, cudaGetLastError(), "profile");
    float ms = 0.0f;
    cudaEventElapsedTime(&ms, r.a, r.b);
    auto it = std::find_if(acc.begin(), acc.end(),
                           [&](const moe_kernel_time &k) { return strcmp(k.name, r.name) == 0; });
    if (it == acc.end()) {
      moe_kernel_time k{};
      snprintf(k.name, sizeof k.name, "%s", r.name);
      acc.push_back(k);
      it = acc.end() - 1;
    }
    it->launches += 1;
    it->total_ms += ms;
  }
  h->prof.recs.clear();
  h->prof.used = 0;
  if (h->phase_pending) {
    // phases of the most recent profiled fused launch (first layer; the
    // last entry runs to the end of the launch)
    std::vector<unsigned long long> all(16 + 3 * 1024, 0);
    unsigned long long *ts = all.data();
    if (cudaMemcpy(ts, h->phase_ts, all.size() * sizeof(unsigned long long),
                   cudaMemcpyDeviceToHost) == cudaSuccess) {
      static const char *names_f[4] = {"fused:router", "fused:gate_up", "fused:down",
                                       "fused:rest"};
      static const char *names_d[8] = {"digit:router", "digit:barrier", "digit:select",
                                       "digit:tables", "digit:gate_up", "digit:barrier2",
                                       "digit:down", "digit:rest"};
      const char *const *names = h->phase_kind ? names_d : names_f;
      const int nph = h->phase_kind ? 8 : 4;
      for (int i = 0; i < nph; ++i) {
        moe_kernel_time k{};
        snprintf(k.name, sizeof k.name, "%s", names[i]);
        k.launches = 1;
        k.total_ms = ts[i + 1] > ts[i] ? (float)((ts[i + 1] - ts[i]) * 1e-6) : 0.0f;
        acc.push_back(k);
      }
      if (h->phase_kind) {
        // spread of the CTAs' start and end times around CTA 0's start
        unsigned long long s0 = ~0ull, s1 = 0, e0 = ~0ull, e1 = 0;
        for (int c = 0; c < 1024; ++c) {
          const unsigned long long a0 = ts[16 + 2 * c], a1 = ts[16 + 2 * c + 1];
          if (!a0 || !a1 || a0 + 100000 < ts[0]) continue;  // older launches
          s0 = std::min(s0, a0), s1 = std::max(s1, a0), e0 = std::min(e0, a1), e1 = std::max(e1, a1);
        }
        if (s1 >= s0 && e1 >= e0 && s0 != ~0ull) {
          // spread of the CTAs' gate/up end times (first layer)
          unsigned long long g0 = ~0ull, g1 = 0;
          for (int c = 0; c < 1024; ++c) {
            const unsigned long long g = ts[16 + 2048 + c];
            if (g < s0 || g > e1) continue;
            g0 = std::min(g0, g), g1 = std::max(g1, g);
          }
          // router sub-phases of CTA 0's first task, and the distributed
          // selection (T > 8) before its barrier
          auto d = [&](int i, int j) { return ts[j] > ts[i] && ts[i] ? ts[j] - ts[i] : 0ull; };
          const char *nm[8] = {"digit:cta_start_spread", "digit:cta_end_spread",
                               "digit:first_to_last", "digit:gate_up_end_spread",
                               "digit:r_stage", "digit:r_norm", "digit:r_dot",
                               "digit:s_select"};
          const unsigned long long v[8] = {s1 - s0, e1 - e0, e1 - s0, g1 >= g0 ? g1 - g0 : 0,
                                           d(0, 9), d(9, 10), d(10, 11), d(2, 12)};
          for (int i = 0; i < 8; ++i) {
            moe_kernel_time k{};
            snprintf(k.name, sizeof k.name, "%s", nm[i]);
            k.launches = 1;
            k.total_ms = (float)(v[i] * 1e-6);
            acc.push_back(k);
          }
        }
      }
    }
    h->phase_pending = false;
  }
  const int n = std::min<int>((int)acc.size(), max_entries);
  for (int i = 0; i < n; ++i) out[i] = acc[i];
  *n_entries = (int)acc.size();
  return MOE_OK;
}

// Same stream of numbers as the test-side generator: splitmix64 counters,
// Box-Muller in double precision.
extern "C" moe_status moe_synth_normal_host(uint64_t seed, uint32_t kind, uint32_t layer,
                                            size_t n, float stddev, float *out) {
  if (!out) return MOE_ERR_INVALID;
  auto mix = [](uint64_t z) {
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
    return z ^ (z >> 31);
  };
  const uint64_t k0 = mix(seed ^ 0x6a09e667f3bcc909ULL);
  const uint64_t key = mix(k0 ^ ((uint64_t)kind << 48) ^ ((uint64_t)layer << 24));
  auto at = [&](uint64_t i) { return mix(key + (i + 1) * 0x9E3779B97F4A7C15ULL); };
  for (size_t j = 0; 2 * j < n; ++j) {
    const double a = (double)((at(2 * j) >> 11) + 1) * 0x1p-53;
    const double b = (double)(at(2 * j + 1) >> 11) * 0x1p-53;
    const double r = std::sqrt(-2.0 * std::log(a));
    const double th = 6.283185307179586 * b;
    out[2 * j] = (float)((double)stddev * r * std::cos(th));
    if (2 * j + 1 < n) out[2 * j + 1] = (float)((double)stddev * r * std::sin(th));
  }
  return MOE_OK;
}

