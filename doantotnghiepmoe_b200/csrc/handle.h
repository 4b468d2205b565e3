// Internal state of a moe_handle, shared by the C-ABI translation units
// (moe_abi.cu: single-GPU calls; ep_host.cu: expert parallelism).  Nothing
// here crosses the public ABI.
#pragma once

#include <cuda.h>
#include <nccl.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/moe_b200.h"
#include "common.cuh"
#include "expert_tc.h"
#include "kernels.h"

namespace moe {
namespace host {

// Calls of at least this many tokens take the tensor-core path under
// MOE_PATH_AUTO; smaller ones the single-launch digit decode.  Measured on
// B200 with 16- and 48-layer stacks (OLMoE E = 64, Qwen3 E = 128, K = 8):
// the digit launch wins at T = 8 (1.51 vs 1.58 ms, 4.63 vs 4.84 ms), the
// persistent tensor-core GEMMs from T = 12 (1.71 vs 1.78 ms) and by 24% at
// T = 24-32 and 37% at T = 64 (7.49 vs 11.90 ms).
constexpr int kTcMinTokens = 12;
// Default bounds of the device-side waits, in SM clock cycles: about 1 s for
// the single-launch kernels' grid barriers and 2 s for the expert-parallel
// flag waits at the maximum SM clock.
constexpr long long kDefaultBarrierWaitCycles = 2000000000LL;
constexpr long long kDefaultFlagWaitCycles = 4000000000LL;

void set_err(std::string &dst, const char *fmt, ...);

int sm_count_of(int device);

template <typename T>
cudaError_t dalloc(T **p, size_t count) {
  return cudaMalloc(reinterpret_cast<void **>(p), std::max<size_t>(count, 1) * sizeof(T));
}

struct DeviceGuard {
  int prev = -1;
  explicit DeviceGuard(int dev) {
    cudaGetDevice(&prev);
    if (prev != dev) cudaSetDevice(dev);
  }
  ~DeviceGuard() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

// CUDA-event bracketing of kernel launches (moe_profile_*).
struct Profiler {
  bool on = false;
  struct Rec {
    const char *name;
    cudaEvent_t a, b;
  };
  std::vector<cudaEvent_t> pool;
  size_t used = 0;
  std::vector<Rec> recs;
  cudaEvent_t take() {
    if (used == pool.size()) {
      cudaEvent_t e;
      if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
      pool.push_back(e);
    }
    return pool[used++];
  }
  // Returns the start event (or null when off / out of events).
  cudaEvent_t begin(cudaStream_t s) {
    if (!on || recs.size() >= 1 << 16) return nullptr;
    cudaEvent_t a = take();
    if (a) cudaEventRecord(a, s);
    return a;
  }
  void end(const char *name, cudaEvent_t a, cudaStream_t s) {
    if (!a) return;
    cudaEvent_t b = take();
    if (!b) return;
    cudaEventRecord(b, s);
    recs.push_back({name, a, b});
  }
  ~Profiler() {
    for (auto e : pool) cudaEventDestroy(e);
  }
};

struct LayerSlot {
  bool set = false;
  const int8_t **d_wptr = nullptr;  // device array [E]
  const float **d_sptr = nullptr;   // device array [E]
  const void *router = nullptr;
  int router_dtype = MOE_ROUTER_F32;
  int vec = 0;  // all expert bases 8-byte aligned -> vector weight loads
  int int4 = 0;  // INT4 experts (src/int8_expert.rs:473-649): GEMV paths only
  // tensor-core path: only for the packed layout (one 3D tensor map per GEMM)
  bool tc_ok = false;
  CUtensorMap map_gu{}, map_dn{};
  // decode weight-tile maps (FusedLayer::tmaps, two maps of 128 bytes), device copy
  void *d_tmaps = nullptr;
  // device copies made by moe_load_layer (owned by the handle)
  void *own_w = nullptr, *own_s = nullptr, *own_r = nullptr, *own_n = nullptr;
};
static_assert(sizeof(CUtensorMap) == 128, "FusedLayer::tmaps holds 128-byte maps");

// NCCL, resolved at run time: the process normally has it loaded already
// (PyTorch's copy); otherwise the system libnccl.so.2 is opened.
struct NcclApi {
  bool ok = false;
  ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*send)(const void *, size_t, ncclDataType_t, int, ncclComm_t,
                       cudaStream_t) = nullptr;
  ncclResult_t (*recv)(void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*group_start)() = nullptr;
  ncclResult_t (*group_end)() = nullptr;
  const char *(*error_string)(ncclResult_t) = nullptr;
};

const NcclApi &nccl();

struct EpLayer {
  bool set = false;
  const float **d_sptr = nullptr;  // [E_local] local scale rows
  CUtensorMap map_gu{}, map_dn{};  // over the packed local experts
};

struct EpState {
  bool on = false;
  int rank = 0, nranks = 1, E_local = 0;
  ncclComm_t comm = nullptr;
  int32_t *d_owner = nullptr, *d_dest_local = nullptr;  // [E]
  std::vector<EpLayer> layers;
  size_t r_local_cap = 0, r_recv_cap = 0;
  int max_tiles = 0;
  // dispatch side
  uint32_t *dest = nullptr;
  int32_t *seg_dest = nullptr, *act_dest = nullptr, *n_dest = nullptr, *stok = nullptr,
          *sslot = nullptr, *spos = nullptr, *scount = nullptr, *rcount = nullptr;
  float *sgate = nullptr, *ret = nullptr;
  uint8_t *send = nullptr, *recv = nullptr;
  int32_t *h_counts = nullptr;  // pinned [2 * nranks]
  // expert side
  uint32_t *ids_l = nullptr;
  float *gates_l = nullptr, *rgate_l = nullptr, *ybuf = nullptr, *act = nullptr;
  int32_t *seg_l = nullptr, *active_l = nullptr, *n_active_l = nullptr, *rtok_l = nullptr,
          *rslot_l = nullptr, *rpos_l = nullptr;
  int8_t *xq = nullptr, *aq = nullptr;
  float *xs1 = nullptr, *xs2 = nullptr, *as1 = nullptr, *as2 = nullptr;
  uint32_t *act_amax = nullptr;
  int32_t *tile_expert = nullptr, *tile_row0 = nullptr, *tile_rows = nullptr, *n_tiles = nullptr;
  // the down GEMM's tile list when its width differs from the gate/up one
  int32_t *dtile_expert = nullptr, *dtile_row0 = nullptr, *dtile_rows = nullptr,
          *n_dtiles = nullptr;
  CUtensorMap map_x64{}, map_x128{}, map_a64{}, map_a128{};
  std::vector<void *> allocs;
  // device-driven exchange over NVLink peer memory (CUDA IPC)
  bool p2p = false;
  std::string transport_note;       // why the collective-library path is in use
  void *region = nullptr;           // this rank's peer-visible region
  std::vector<void *> peer_maps;    // opened peer regions (closed at finalize)
  EpP2P P{};
  uint32_t *epoch = nullptr;        // device: calls so far (flag values)
  uint32_t *done = nullptr;         // dispatch completion counter (monotonic)
  int32_t *n_recv = nullptr;        // device count of received routes
  int dispatch_grid = 0;
};

}  // namespace host
}  // namespace moe

struct moe_handle {
  int device = 0;
  moe_dims d{};
  int sm_count = 148;
  cudaStream_t own_stream = nullptr, stream = nullptr;
  int route_mode = MOE_ROUTE_SOFTMAX_TOPK;
  int path = MOE_PATH_AUTO;
  std::mutex mu;
  std::string err;
  std::vector<moe::host::LayerSlot> layers;
  // scratch
  float *logits = nullptr, *gates = nullptr, *r_gate = nullptr, *act = nullptr,
        *contrib = nullptr, *hbuf = nullptr, *io_in = nullptr, *io_out = nullptr,
        *io_resid = nullptr;
  uint32_t *ids = nullptr, *status = nullptr;
  int32_t *seg_off = nullptr, *active = nullptr, *n_active = nullptr, *r_token = nullptr,
          *r_slot = nullptr, *r_pos = nullptr;
  float *h_pin_in = nullptr, *h_pin_out = nullptr;
  uint32_t *h_pin_status = nullptr;
  float *h_pin_meta = nullptr;  // [2][max_tokens * top_k]: ids, gates
  cudaEvent_t stage_ev[32] = {};  // chunked staging of pageable host outputs
  // host-buffer call in token chunks: copy-in and copy-out streams, and per
  // chunk the events "input arrived" and "layer done"
  cudaStream_t io_stream[2] = {};
  cudaEvent_t io_ev[2][8] = {};
  int last_launches = 0;
  moe::host::Profiler prof;
  // tensor-core path scratch
  bool tc_ok = false;
  int max_tiles = 0;
  int8_t *xq = nullptr, *aq = nullptr;  // [2][R][H], [2][R][I] digit planes
  float *xs1 = nullptr, *xs2 = nullptr, *as1 = nullptr, *as2 = nullptr;
  uint32_t *act_amax = nullptr;
  int32_t *tile_expert = nullptr, *tile_row0 = nullptr, *tile_rows = nullptr, *n_tiles = nullptr;
  // the down GEMM's tile list when its width differs from the gate/up one
  int32_t *dtile_expert = nullptr, *dtile_row0 = nullptr, *dtile_rows = nullptr,
          *n_dtiles = nullptr;
  CUtensorMap map_x64{}, map_x128{}, map_a64{}, map_a128{};  // digit planes, box 64/128 rows
  // fused decode
  moe::FusedLayer *d_flayers = nullptr;  // [num_layers]
  std::vector<moe::FusedLayer> flayers;
  std::vector<int> layer_vec;
  uint32_t *tok_cnt = nullptr, *fbar = nullptr;
  uint32_t *dbar = nullptr;                // digit decode barrier: arrivals, exits
  int phase_kind = 0;                      // stamps of: 0 the exact kernel, 1 the digit kernel
  int32_t *perm_scratch = nullptr;         // multi-CTA permutation
  size_t perm_scratch_words = 0;
  std::vector<int> layer_async;            // router rows are 16-byte aligned f32
  unsigned long long *phase_ts = nullptr;  // [8] single-launch kernel phase stamps
  bool phase_pending = false;
  // replayed launch sequences (see graphed())
  struct GraphEntry {
    uint64_t key[10];
    cudaGraphExec_t exec;
    int launches;
    uint64_t last_use;
  };
  std::vector<GraphEntry> graphs;
  uint64_t graph_clock = 0;
  bool graphs_on = true;
  // device-side wait bounds, in SM clock cycles (moe_set_wait_limit)
  long long wait_barrier_cycles = moe::host::kDefaultBarrierWaitCycles;
  long long wait_flag_cycles = moe::host::kDefaultFlagWaitCycles;
  uint32_t *probe_flag = nullptr;  // device word that nothing sets (moe_debug_wait_flag)
  moe::host::EpState ep;
};


namespace moe {
namespace host {

void free_ep(moe_handle *h);  // ep_host.cu
void drop_graphs(moe_handle *h);
cudaStream_t pick(moe_handle *h, void *stream);
moe_status cuda_fail(moe_handle *h, cudaError_t e, const char *what);
// Router + top-k (+ permutation and tensor-core tile lists) for T tokens.
moe_status run_route(moe_handle *h, const LayerSlot &L, const float *d_h, int T, uint32_t *ids,
                     float *gates, float *probs, cudaStream_t s, bool permute, int bn_gu = 0,
                     int bn_dn = 0);

// Replay a call's launch sequence as a CUDA graph.  The sequence is captured
// once per key (call kind, layer, token count, buffers, stream, path) and
// replayed afterwards, which removes the host launch cost and most of the
// gaps between the kernels.  Captures are only kept when every launch in the
// sequence takes its sizes from device memory or from the key; the cache is
// dropped whenever weights, path or routing mode change.  Profiling (events
// between kernels) and a caller's own stream capture use direct launches.
template <typename F>
moe_status graphed(moe_handle *h, const uint64_t (&key)[10], cudaStream_t s, F &&launch_all) {
  if (!h->graphs_on || h->prof.on) return launch_all();
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(s, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) {
    cudaGetLastError();
    return launch_all();
  }
  for (auto &g : h->graphs) {
    if (memcmp(g.key, key, sizeof key) != 0) continue;
    g.last_use = ++h->graph_clock;
    h->last_launches = g.launches;
    const cudaError_t e = cudaGraphLaunch(g.exec, s);
    return e == cudaSuccess ? MOE_OK : cuda_fail(h, e, "graph launch");
  }
  if (cudaStreamBeginCapture(s, cudaStreamCaptureModeRelaxed) != cudaSuccess) {
    cudaGetLastError();
    return launch_all();
  }
  const moe_status st = launch_all();
  cudaGraph_t graph = nullptr;
  const cudaError_t ec = cudaStreamEndCapture(s, &graph);
  cudaGraphExec_t exec = nullptr;
  const bool ok = st == MOE_OK && ec == cudaSuccess && graph &&
                  cudaGraphInstantiate(&exec, graph, 0) == cudaSuccess;
  if (graph) cudaGraphDestroy(graph);
  if (!ok) {
    cudaGetLastError();
    if (st != MOE_OK) return st;
    return launch_all();  // nothing ran during the failed capture
  }
  if (h->graphs.size() >= 32) {
    auto old = std::min_element(h->graphs.begin(), h->graphs.end(),
                                [](const auto &a, const auto &b) { return a.last_use < b.last_use; });
    cudaGraphExecDestroy(old->exec);
    h->graphs.erase(old);
  }
  moe_handle::GraphEntry g{};
  memcpy(g.key, key, sizeof key);
  g.exec = exec;
  g.launches = h->last_launches;
  g.last_use = ++h->graph_clock;
  h->graphs.push_back(g);
  const cudaError_t e = cudaGraphLaunch(exec, s);
  return e == cudaSuccess ? MOE_OK : cuda_fail(h, e, "graph launch");
}

}  // namespace host
}  // namespace moe
