// moe_layer_forward_noalloc: one MoE layer that allocates no device memory.
//
// Who needs this: a host that budgets every byte of GPU memory itself (the
// reference engine's VRAM tier manager sizes its expert pool to what is left
// after its own buffers, so an allocation made behind its back can push it
// out of memory), and a host that calls the layer on a latency-critical
// decode thread, where cudaMalloc/cudaFree can block on or synchronise the
// device.  Such callers cannot use moe_create(), which allocates the
// per-handle scratch with cudaMalloc.
//
// How: every intermediate of the layer (logits, routing, permutation,
// activations, contributions, the status word) lives in one file-scope
// device array of kNoAllocScratchBytes.  The array is part of the loaded
// module, so each GPU that loads this library holds it from load until the
// process exits.  The call runs on the device that owns `stream` (the
// current device for the legacy default stream), made current for the
// duration of the call.  The array's address on that device is fetched once,
// with cudaGetSymbolAddress on the first call there; make that first call
// before any stream capture.  The address is cached for the life of the
// process, so the entry point must not be used again on a device after
// cudaDeviceReset() on it.  All calls share
// the one array: calls whose work overlaps on the GPU (two streams, two host
// threads) race on it and must be serialised by the caller.  The array keeps
// the previous call's contents; the only state that must start from zero
// (the status word) is cleared at the start of every call, and everything
// else is fully rewritten before it is read.
//
// The layer runs the same kernels as moe_layer_forward (router, permutation,
// exact-order INT8 GEMV experts, slot-ordered combine), so its results are
// identical to that entry point's.
#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "../../include/moe_b200.h"
#include "common.cuh"
#include "kernels.h"

namespace {

// the GEMV kernels stage this many input rows of H (gate/up) or I (down)
// floats in shared memory
constexpr int kGemvStagedRows = 4;

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;  // 8 MiB per GPU
constexpr int kMaxDevices = 64;

__device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_setup_mu;
void *g_scratch_ptr[kMaxDevices] = {};
int g_sm_count[kMaxDevices] = {};

__global__ void fill_expert_tables(const int8_t *experts, const float *scales, size_t wstride,
                                   size_t sstride, int E, const int8_t **wp, const float **sp) {
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < E; e += gridDim.x * blockDim.x) {
    wp[e] = experts + (size_t)e * wstride;
    sp[e] = scales + (size_t)e * sstride;
  }
}

void report(char *msg, size_t len, const char *fmt, ...) __attribute__((format(printf, 3, 4)));
void report(char *msg, size_t len, const char *fmt, ...) {
  if (!msg || len == 0) return;
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(msg, len, fmt, ap);
  va_end(ap);
}

size_t align256(size_t n) { return (n + 255) & ~size_t(255); }

}  // namespace

extern "C" moe_status moe_layer_forward_noalloc(const moe_dims *dims, const int8_t *d_experts,
                                                const float *d_scales, const void *d_router,
                                                int router_dtype, const float *d_h,
                                                const float *d_resid, float *d_out, int T,
                                                void *stream, char *err_msg, size_t err_len) {
  using namespace moe;
  if (err_msg && err_len) err_msg[0] = '\0';
  if (!dims || !d_experts || !d_scales || !d_router || !d_h || !d_out) {
    report(err_msg, err_len, "null argument");
    return MOE_ERR_INVALID;
  }
  const moe_dims &d = *dims;
  if (d.hidden <= 0 || d.intermediate <= 0 || d.hidden > (1 << 16) ||
      d.intermediate > (1 << 16) || d.num_experts <= 0 || d.num_experts > kMaxExperts ||
      d.top_k <= 0 || d.top_k > kMaxTopK || d.top_k > d.num_experts || T < 0 ||
      (router_dtype != MOE_ROUTER_F32 && router_dtype != MOE_ROUTER_BF16) ||
      ((uintptr_t)d_scales & 3)) {
    report(err_msg, err_len, "invalid dimensions, router dtype or scale alignment");
    return MOE_ERR_INVALID;
  }
  if (T == 0) return MOE_OK;
  const size_t H = d.hidden, I = d.intermediate, E = d.num_experts, K = d.top_k;
  const size_t R = (size_t)T * K;
  // Carve the scratch: every piece starts on a 256-byte boundary.
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t at = off;
    off += align256(bytes);
    return at;
  };
  const size_t o_status = take(4), o_seg = take((E + 1) * 4), o_active = take(E * 4),
               o_nactive = take(4), o_ids = take(R * 4), o_gates = take(R * 4),
               o_rtok = take(R * 4), o_rslot = take(R * 4), o_rgate = take(R * 4),
               o_rpos = take(R * 4), o_logits = take((size_t)T * E * 4),
               o_wp = take(E * sizeof(void *)), o_sp = take(E * sizeof(void *)),
               o_act = take(R * I * 4), o_contrib = take(R * H * 4);
  if (off > kNoAllocScratchBytes) {
    report(err_msg, err_len,
           "moe_layer_forward_noalloc: T=%d needs %zu bytes of scratch, more than the fixed "
           "%zu bytes; use fewer tokens per call or moe_layer_forward",
           T, off, kNoAllocScratchBytes);
    return MOE_ERR_INVALID;
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int prev = -1, dev = -1;
  if (cudaGetDevice(&prev) != cudaSuccess) {
    report(err_msg, err_len, "no usable current CUDA device");
    return MOE_ERR_CUDA;
  }
  dev = prev;
  // a stream of another device: run there (its copy of the array)
  if (s && cudaStreamGetDevice(s, &dev) != cudaSuccess) {
    cudaGetLastError();
    report(err_msg, err_len, "stream does not belong to a usable CUDA device");
    return MOE_ERR_INVALID;
  }
  if (dev < 0 || dev >= kMaxDevices) {
    report(err_msg, err_len, "device %d outside the supported range [0, %d)", dev, kMaxDevices);
    return MOE_ERR_INVALID;
  }
  struct Restore {
    int prev, dev;
    ~Restore() {
      if (prev != dev) cudaSetDevice(prev);
    }
  } restore{prev, dev};
  if (dev != prev && cudaSetDevice(dev) != cudaSuccess) {
    report(err_msg, err_len, "cannot make device %d current", dev);
    return MOE_ERR_CUDA;
  }
  // The GEMV kernels stage their input rows in shared memory: a shape that
  // would not fit is rejected here rather than failing at launch.
  int smem_max = 0;
  cudaDeviceGetAttribute(&smem_max, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  const size_t smem_need = sizeof(float) * kGemvStagedRows * std::max(H, I);
  if (smem_max > 0 && smem_need > (size_t)smem_max) {
    report(err_msg, err_len,
           "hidden %zu / intermediate %zu need %zu bytes of shared memory per block, more "
           "than the device's %d", H, I, smem_need, smem_max);
    return MOE_ERR_INVALID;
  }
  unsigned char *base = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_setup_mu);
    if (!g_scratch_ptr[dev]) {
      void *p = nullptr;
      const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
      if (e != cudaSuccess || !p) {
        report(err_msg, err_len, "cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
        return MOE_ERR_CUDA;
      }
      int sms = 148;
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      g_sm_count[dev] = sms;
      g_scratch_ptr[dev] = p;
    }
    base = static_cast<unsigned char *>(g_scratch_ptr[dev]);
  }
  uint32_t *status = reinterpret_cast<uint32_t *>(base + o_status);
  auto at = [&](size_t o) { return base + o; };

  cudaError_t e = cudaMemsetAsync(status, 0, 4, s);
  const int8_t **wp = reinterpret_cast<const int8_t **>(at(o_wp));
  const float **sp = reinterpret_cast<const float **>(at(o_sp));
  if (e == cudaSuccess) {
    fill_expert_tables<<<1, 256, 0, s>>>(d_experts, d_scales, 3 * I * H, 2 * I + H, (int)E, wp,
                                         sp);
    e = cudaGetLastError();
  }
  RouteArgs ra{};
  ra.h = d_h;
  ra.router = d_router;
  ra.router_dtype = router_dtype;
  ra.T = T;
  ra.H = (int)H;
  ra.E = (int)E;
  ra.K = (int)K;
  ra.norm_topk_prob = d.norm_topk_prob;
  ra.mode = kRouteSoftmaxTopk;
  ra.logits = reinterpret_cast<float *>(at(o_logits));
  ra.ids = reinterpret_cast<uint32_t *>(at(o_ids));
  ra.gates = reinterpret_cast<float *>(at(o_gates));
  ra.status = status;
  if (e == cudaSuccess) e = launch_route(ra, s);
  PermuteArgs pa{};
  pa.ids = ra.ids;
  pa.gates = ra.gates;
  pa.T = T;
  pa.K = (int)K;
  pa.E = (int)E;
  pa.seg_off = reinterpret_cast<int32_t *>(at(o_seg));
  pa.active = reinterpret_cast<int32_t *>(at(o_active));
  pa.n_active = reinterpret_cast<int32_t *>(at(o_nactive));
  pa.r_token = reinterpret_cast<int32_t *>(at(o_rtok));
  pa.r_slot = reinterpret_cast<int32_t *>(at(o_rslot));
  pa.r_gate = reinterpret_cast<float *>(at(o_rgate));
  pa.r_pos = reinterpret_cast<int32_t *>(at(o_rpos));
  pa.status = status;
  // pa.scratch stays null: launch_permute then sorts every route in one CTA,
  // whatever their count, and never takes its multi-CTA path (which needs
  // scratch of its own).
  if (e == cudaSuccess) e = launch_permute(pa, s);
  GemvArgs a{};
  a.H = (int)H;
  a.I = (int)I;
  a.w_ptr = wp;
  a.s_ptr = sp;
  a.active = pa.active;
  a.n_active_dev = pa.n_active;
  a.n_active_max = (int)std::min<size_t>(E, R);
  a.seg_off = pa.seg_off;
  a.r_token = pa.r_token;
  a.x = d_h;
  a.act = reinterpret_cast<float *>(at(o_act));
  a.r_slot = pa.r_slot;
  a.r_gate = pa.r_gate;
  a.K = (int)K;
  a.contrib = reinterpret_cast<float *>(at(o_contrib));
  a.status = status;
  a.sm_count = g_sm_count[dev];
  a.vec = ((uintptr_t)d_experts & 7) == 0 && ((3 * I * H) & 7) == 0 &&
          ((uintptr_t)d_h & 15) == 0;
  if (e == cudaSuccess) e = launch_gate_up(a, s);
  if (e == cudaSuccess) e = launch_down(a, s);
  if (e == cudaSuccess) e = launch_combine(a.contrib, d_resid, d_out, T, (int)K, (int)H, status, s);
  uint32_t st = 0;
  if (e == cudaSuccess) e = cudaMemcpyAsync(&st, status, 4, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) {
    report(err_msg, err_len, "CUDA error: %s", cudaGetErrorString(e));
    return MOE_ERR_CUDA;
  }
  if (st & kStatusTimeout) {
    report(err_msg, err_len, "device wait timed out");
    return MOE_ERR_TIMEOUT;
  }
  if (st & kStatusNonFinite) {
    report(err_msg, err_len, "non-finite computation result");
    return MOE_ERR_NONFINITE;
  }
  if (st & kStatusBadRoute) {
    report(err_msg, err_len, "routing produced an invalid expert id");
    return MOE_ERR_INVALID;
  }
  return MOE_OK;
}
