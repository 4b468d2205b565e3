// Expert parallelism entry points of the C ABI (include/moe_b200.h, 2b): group
// set-up (NCCL communicator, peer-memory regions shared over CUDA IPC), the
// per-layer forward over the peer-memory transport and over NCCL
// point-to-point, and teardown.  The kernels are in ep.cu.
#include <cstdio>
#include <cstdlib>

#include "handle.h"

using namespace moe;
using namespace moe::host;

namespace moe {
namespace host {

void free_ep(moe_handle *h) {
  EpState &ep = h->ep;
  for (void *m : ep.peer_maps) cudaIpcCloseMemHandle(m);
  ep.peer_maps.clear();
  if (ep.region) cudaFree(ep.region);
  ep.region = nullptr;
  ep.p2p = false;
  if (ep.comm && nccl().ok) nccl().comm_destroy(ep.comm);
  ep.comm = nullptr;
  for (auto &l : ep.layers) cudaFree(l.d_sptr);
  ep.layers.clear();
  for (void *p : ep.allocs) cudaFree(p);
  ep.allocs.clear();
  cudaFreeHost(ep.h_counts);
  ep.h_counts = nullptr;
  ep.on = false;
}

}  // namespace host
}  // namespace moe

namespace {
template <typename T>
bool ep_alloc(EpState &ep, T **p, size_t count) {
  if (dalloc(p, count) != cudaSuccess) return false;
  ep.allocs.push_back(*p);
  return true;
}

moe_status nccl_fail(moe_handle *h, ncclResult_t r, const char *what) {
  set_err(h->err, "%s: %s", what, nccl().error_string ? nccl().error_string(r) : "nccl");
  return MOE_ERR_NCCL;
}
}  // namespace

namespace {
size_t align_up(size_t n, size_t a) { return (n + a - 1) / a * a; }

// Peer-memory transport: one region per rank holding everything peers write
// (flags, count matrix, the expert-sorted receive side of the tensor-core
// input, the [T, K, H] contribution buffer), shared through CUDA IPC handles
// that are exchanged once over the communicator.  On any failure the
// collective-library transport stays in use and the reason is kept.
void ep_setup_p2p(moe_handle *h, size_t Tm) {
  EpState &ep = h->ep;
  const int N = ep.nranks, E = h->d.num_experts, H = h->d.hidden, K = h->d.top_k;
  const char *env = getenv("MOE_EP_TRANSPORT");
  if (env && strcmp(env, "nccl") == 0) {
    ep.transport_note = "MOE_EP_TRANSPORT=nccl";
    return;
  }
  if (N > kEpMaxRanks) {
    ep.transport_note = "more ranks than the peer-memory transport supports";
    return;
  }
  const size_t RR = ep.r_recv_cap;
  EpP2P P{};
  size_t off = 0;
  P.off_flags = off;   off = align_up(off + 3 * kEpMaxRanks * 4, 1024);
  P.off_counts = off;  off = align_up(off + (size_t)2 * N * E * 4, 1024);
  P.off_xq = off;      P.plane = RR * H; off = align_up(off + 2 * RR * H, 1024);
  P.off_s1 = off;      off = align_up(off + RR * 4, 1024);
  P.off_s2 = off;      off = align_up(off + RR * 4, 1024);
  P.off_gate = off;    off = align_up(off + RR * 4, 1024);
  P.off_rank = off;    off = align_up(off + RR * 4, 1024);
  P.off_tok = off;     off = align_up(off + RR * 4, 1024);
  P.off_slot = off;    off = align_up(off + RR * 4, 1024);
  P.off_amax = off;    off = align_up(off + RR * 4, 1024);
  P.off_contrib = off; off = align_up(off + Tm * K * H * 4, 1024);  // room for f32 rows
  P.off_cscale = off;  off = align_up(off + Tm * K * ((H + 31) / 32) * 4, 1024);
  P.rank = ep.rank;
  P.nranks = N;
  // return rows as fp32 (default) or as int16 with a scale per 32 rows:
  // MOE_EP_RETURN=i16.  On 2 B200s the int16 epilogue cost more than the
  // halved traffic saved (down GEMM 331 vs 203 us at C4), so fp32 stays.
  const char *ret = getenv("MOE_EP_RETURN");
  P.ret16 = ret && strcmp(ret, "i16") == 0;
  P.wait_cycles = h->wait_flag_cycles;
  void *region = nullptr;
  if (cudaMalloc(&region, off) != cudaSuccess || cudaMemset(region, 0, off) != cudaSuccess) {
    cudaGetLastError();
    if (region) cudaFree(region);
    ep.transport_note = "peer region allocation failed";
    return;
  }
  cudaIpcMemHandle_t mine{};
  if (cudaIpcGetMemHandle(&mine, region) != cudaSuccess) {
    cudaGetLastError();
    cudaFree(region);
    ep.transport_note = "cudaIpcGetMemHandle failed";
    return;
  }
  // exchange the handles: every rank sends its 64 bytes to every other rank
  const size_t HB = sizeof(cudaIpcMemHandle_t);
  uint8_t *dh = nullptr;
  std::vector<uint8_t> all(N * HB);
  bool ok = cudaMalloc(&dh, N * HB) == cudaSuccess &&
            cudaMemcpy(dh + ep.rank * HB, &mine, HB, cudaMemcpyHostToDevice) == cudaSuccess;
  cudaStream_t s = h->stream;
  if (ok) {
    const NcclApi &api = nccl();
    ncclResult_t nr = api.group_start();
    for (int q = 0; q < N && nr == ncclSuccess; ++q) {
      if (q == ep.rank) continue;
      nr = api.send(dh + ep.rank * HB, HB, ncclUint8, q, ep.comm, s);
      if (nr == ncclSuccess) nr = api.recv(dh + q * HB, HB, ncclUint8, q, ep.comm, s);
    }
    const ncclResult_t ng = api.group_end();
    ok = nr == ncclSuccess && ng == ncclSuccess && cudaStreamSynchronize(s) == cudaSuccess &&
         cudaMemcpy(all.data(), dh, N * HB, cudaMemcpyDeviceToHost) == cudaSuccess;
  }
  if (dh) cudaFree(dh);
  std::vector<void *> maps;
  for (int q = 0; q < N && ok; ++q) {
    if (q == ep.rank) {
      P.base[q] = (uint8_t *)region;
      continue;
    }
    cudaIpcMemHandle_t hq;
    memcpy(&hq, all.data() + q * HB, HB);
    void *ptr = nullptr;
    if (cudaIpcOpenMemHandle(&ptr, hq, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
      cudaGetLastError();
      ok = false;
      break;
    }
    maps.push_back(ptr);
    P.base[q] = (uint8_t *)ptr;
  }
  // the tensor-core input maps now point at the region's receive side
  uint8_t *xq = (uint8_t *)region + P.off_xq;
  ok = ok && tc::encode_map3d(&ep.map_x64, xq, H, RR, 2, H, RR * H, 64) &&
       tc::encode_map3d(&ep.map_x128, xq, H, RR, 2, H, RR * H, 128) &&
       ep_alloc(ep, &ep.done, 1) && ep_alloc(ep, &ep.n_recv, 1) &&
       ep_alloc(ep, &ep.epoch, 1) && cudaMemset(ep.done, 0, 4) == cudaSuccess &&
       cudaMemset(ep.epoch, 0, 4) == cudaSuccess;
  if (!ok) {
    for (void *m : maps) cudaIpcCloseMemHandle(m);
    cudaFree(region);
    ep.transport_note = "CUDA IPC handle exchange / mapping failed";
    // restore the collective-library path's maps
    tc::encode_map3d(&ep.map_x64, ep.xq, H, RR, 2, H, RR * H, 64);
    tc::encode_map3d(&ep.map_x128, ep.xq, H, RR, 2, H, RR * H, 128);
    return;
  }
  ep.region = region;
  ep.peer_maps = maps;
  ep.P = P;
  ep.p2p = true;
  ep.dispatch_grid = 2 * h->sm_count;
  ep.transport_note.clear();
}
}  // namespace

extern "C" moe_status moe_ep_unique_id(unsigned char id_out[128]) {
  if (!id_out) return MOE_ERR_INVALID;
  if (!nccl().ok) return MOE_ERR_NCCL;
  ncclUniqueId id;
  if (nccl().get_unique_id(&id) != ncclSuccess) return MOE_ERR_NCCL;
  memcpy(id_out, id.internal, 128);
  return MOE_OK;
}

extern "C" moe_status moe_ep_init(moe_handle *h, int rank, int nranks,
                                  const unsigned char id[128], const int32_t *expert_owner) {
  if (!h || !id || !expert_owner || nranks < 1 || rank < 0 || rank >= nranks)
    return MOE_ERR_INVALID;
  std::lock_guard<std::mutex> lock(h->mu);
  drop_graphs(h);
  if (!nccl().ok) {
    set_err(h->err, "libnccl.so.2 not available");
    return MOE_ERR_NCCL;
  }
  const int E = h->d.num_experts, H = h->d.hidden, I = h->d.intermediate, K = h->d.top_k;
  if (H % 16 || I % 16 || !h->tc_ok) {
    set_err(h->err, "expert parallelism needs the tensor-core path (H, I multiples of 16)");
    return MOE_ERR_INVALID;
  }
  std::vector<int32_t> counts(nranks, 0), dest_local(E, -1);
  for (int e = 0; e < E; ++e) {
    const int o = expert_owner[e];
    if (o < 0 || o >= nranks) {
      set_err(h->err, "expert %d has owner %d outside [0, %d)", e, o, nranks);
      return MOE_ERR_INVALID;
    }
    dest_local[e] = counts[o]++;  // local index = rank of e among its owner's experts
  }
  DeviceGuard g(h->device);
  free_ep(h);
  EpState &ep = h->ep;
  ep.rank = rank;
  ep.nranks = nranks;
  ep.E_local = counts[rank];
  ncclUniqueId uid;
  memcpy(uid.internal, id, 128);
  const ncclResult_t nr = nccl().comm_init_rank(&ep.comm, nranks, uid, rank);
  if (nr != ncclSuccess) {
    ep.comm = nullptr;
    return nccl_fail(h, nr, "ncclCommInitRank");
  }
  const size_t Tm = h->d.max_tokens;
  ep.r_local_cap = Tm * K;
  ep.r_recv_cap = (size_t)nranks * Tm * K;
  const size_t RL = ep.r_local_cap, RR = ep.r_recv_cap, ROW = ep_row_bytes(H);
  ep.max_tiles = (int)((RR + 63) / 64 + std::min<size_t>(std::max(ep.E_local, 1), RR));
  bool ok = ep_alloc(ep, &ep.d_owner, E) && ep_alloc(ep, &ep.d_dest_local, E) &&
            ep_alloc(ep, &ep.dest, RL) && ep_alloc(ep, &ep.seg_dest, nranks + 1) &&
            ep_alloc(ep, &ep.act_dest, nranks) && ep_alloc(ep, &ep.n_dest, 1) &&
            ep_alloc(ep, &ep.stok, RL) && ep_alloc(ep, &ep.sslot, RL) &&
            ep_alloc(ep, &ep.spos, RL) && ep_alloc(ep, &ep.sgate, RL) &&
            ep_alloc(ep, &ep.scount, nranks) && ep_alloc(ep, &ep.rcount, nranks) &&
            ep_alloc(ep, &ep.send, RL * ROW) && ep_alloc(ep, &ep.recv, RR * ROW) &&
            ep_alloc(ep, &ep.ret, RL * H) && ep_alloc(ep, &ep.ids_l, RR) &&
            ep_alloc(ep, &ep.gates_l, RR) && ep_alloc(ep, &ep.rgate_l, RR) &&
            ep_alloc(ep, &ep.ybuf, RR * H) && ep_alloc(ep, &ep.act, RR * I) &&
            ep_alloc(ep, &ep.seg_l, std::max(ep.E_local, 1) + 1) &&
            ep_alloc(ep, &ep.active_l, std::max(ep.E_local, 1)) &&
            ep_alloc(ep, &ep.n_active_l, 1) && ep_alloc(ep, &ep.rtok_l, RR) &&
            ep_alloc(ep, &ep.rslot_l, RR) && ep_alloc(ep, &ep.rpos_l, RR) &&
            ep_alloc(ep, &ep.xq, 2 * RR * H) && ep_alloc(ep, &ep.aq, 2 * RR * I) &&
            ep_alloc(ep, &ep.xs1, RR) && ep_alloc(ep, &ep.xs2, RR) && ep_alloc(ep, &ep.as1, RR) &&
            ep_alloc(ep, &ep.as2, RR) && ep_alloc(ep, &ep.act_amax, RR) &&
            ep_alloc(ep, &ep.tile_expert, ep.max_tiles) &&
            ep_alloc(ep, &ep.tile_row0, ep.max_tiles) &&
            ep_alloc(ep, &ep.tile_rows, ep.max_tiles) && ep_alloc(ep, &ep.n_tiles, 1) &&
            ep_alloc(ep, &ep.dtile_expert, ep.max_tiles) &&
            ep_alloc(ep, &ep.dtile_row0, ep.max_tiles) &&
            ep_alloc(ep, &ep.dtile_rows, ep.max_tiles) && ep_alloc(ep, &ep.n_dtiles, 1) &&
            cudaMallocHost(&ep.h_counts, 2 * nranks * sizeof(int32_t)) == cudaSuccess;
  if (!ok) {
    free_ep(h);
    return MOE_ERR_NOMEM;
  }
  cudaMemcpy(ep.d_owner, expert_owner, E * sizeof(int32_t), cudaMemcpyHostToDevice);
  cudaMemcpy(ep.d_dest_local, dest_local.data(), E * sizeof(int32_t), cudaMemcpyHostToDevice);
  ok = tc::encode_map3d(&ep.map_x64, ep.xq, H, RR, 2, H, RR * H, 64) &&
       tc::encode_map3d(&ep.map_x128, ep.xq, H, RR, 2, H, RR * H, 128) &&
       tc::encode_map3d(&ep.map_a64, ep.aq, I, RR, 2, I, RR * I, 64) &&
       tc::encode_map3d(&ep.map_a128, ep.aq, I, RR, 2, I, RR * I, 128);
  if (!ok) {
    free_ep(h);
    set_err(h->err, "tensor map encoding failed for the expert-parallel buffers");
    return MOE_ERR_CUDA;
  }
  ep.layers.assign(h->d.num_layers, EpLayer{});
  ep.on = true;
  ep_setup_p2p(h, Tm);
  return MOE_OK;
}

extern "C" int moe_ep_transport(const moe_handle *h) {
  if (!h || !h->ep.on) return -1;
  return h->ep.p2p ? 1 : 0;
}

extern "C" moe_status moe_ep_finalize(moe_handle *h) {
  if (!h) return MOE_ERR_INVALID;
  std::lock_guard<std::mutex> lock(h->mu);
  DeviceGuard g(h->device);
  drop_graphs(h);
  free_ep(h);
  return MOE_OK;
}

extern "C" moe_status moe_ep_set_layer(moe_handle *h, int layer, const int8_t *d_experts_local,
                                       const float *d_scales_local, const void *d_router,
                                       int router_dtype) {
  if (!h || !d_router || (router_dtype != MOE_ROUTER_F32 && router_dtype != MOE_ROUTER_BF16))
    return MOE_ERR_INVALID;
  std::lock_guard<std::mutex> lock(h->mu);
  drop_graphs(h);
  EpState &ep = h->ep;
  if (!ep.on || layer < 0 || layer >= (int)ep.layers.size()) {
    set_err(h->err, "moe_ep_set_layer: call moe_ep_init first / layer out of range");
    return MOE_ERR_STATE;
  }
  const size_t H = h->d.hidden, I = h->d.intermediate;
  const int EL = ep.E_local;
  if (EL > 0 && (!d_experts_local || !d_scales_local || ((uintptr_t)d_experts_local & 15) ||
                 ((uintptr_t)d_scales_local & 3))) {
    set_err(h->err, "local experts: null or misaligned pointers");
    return MOE_ERR_INVALID;
  }
  DeviceGuard g(h->device);
  EpLayer &L = ep.layers[layer];
  if (!L.d_sptr && dalloc(&L.d_sptr, std::max(EL, 1)) != cudaSuccess) return MOE_ERR_NOMEM;
  std::vector<const float *> sp(std::max(EL, 1), nullptr);
  for (int e = 0; e < EL; ++e) sp[e] = d_scales_local + e * (2 * I + H);
  cudaMemcpy(L.d_sptr, sp.data(), sp.size() * sizeof(void *), cudaMemcpyHostToDevice);
  if (EL > 0) {
    const char *wb = (const char *)d_experts_local;
    if (!tc::encode_map3d(&L.map_gu, wb, H, 2 * I, EL, H, 3 * I * H, 128) ||
        !tc::encode_map3d(&L.map_dn, wb + 2 * I * H, I, H, EL, I, 3 * I * H, 128)) {
      set_err(h->err, "tensor map encoding failed for the local experts");
      return MOE_ERR_CUDA;
    }
  }
  // the router (replicated on every rank) lives in the ordinary layer slot
  LayerSlot &S = h->layers[layer];
  S.router = d_router;
  S.router_dtype = router_dtype;
  L.set = true;
  return MOE_OK;
}

namespace {
// One layer over the peer-memory transport; see ep.cu for the protocol.
moe_status ep_forward_p2p(moe_handle *h, int layer, const float *d_h, const float *d_resid,
                          float *d_out, int T, cudaStream_t s) {
  EpState &ep = h->ep;
  const int H = h->d.hidden, I = h->d.intermediate, K = h->d.top_k, E = h->d.num_experts;
  const int R = T * K;
  const size_t RR = ep.r_recv_cap;
  const LayerSlot &LS = h->layers[layer];
  const EpLayer &EL = ep.layers[layer];
  const EpP2P &P = ep.P;
  uint32_t *epoch = ep.epoch;  // advanced on the device by the publish kernel
  cudaError_t e = cudaSuccess;
  // 1. route and bucket the local routes by global expert
  cudaEvent_t p0 = nullptr;
  if (T > 0) {
    moe_status st = run_route(h, LS, d_h, T, h->ids, h->gates, nullptr, s, false);
    if (st != MOE_OK) return st;
    p0 = h->prof.begin(s);
    PermuteArgs pa{};
    pa.ids = h->ids;
    pa.gates = h->gates;
    pa.T = T;
    pa.K = K;
    pa.E = E;
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
    e = launch_permute(pa, s);
    h->prof.end("permute", p0, s);
    h->last_launches += permute_launches(pa);
  } else {
    e = cudaMemsetAsync(h->seg_off, 0, (E + 1) * sizeof(int32_t), s);
  }
  // 2. counts to every peer, 3. routes straight into the owners' buffers
  cudaEvent_t p1 = h->prof.begin(s);
  if (e == cudaSuccess) e = launch_ep_publish(h->seg_off, E, P, epoch, s);
  if (e == cudaSuccess)
    e = launch_ep_dispatch(d_h, h->seg_off, h->ids, h->gates, h->r_pos, ep.d_owner, E, T, K, H,
                           P, epoch, ep.done, ep.dispatch_grid, h->status, s);
  h->prof.end("ep_dispatch", p1, s);
  if (e != cudaSuccess) return cuda_fail(h, e, "ep dispatch");
  // 4. wait for every rank's routes; expert segments from the count matrix
  cudaEvent_t p2 = h->prof.begin(s);
  e = launch_ep_recv_prep(ep.d_owner, E, P, epoch, ep.seg_l, ep.active_l, ep.n_active_l,
                          ep.n_recv, h->status, s);
  // tile widths from the expected receive count (this rank's own route
  // count: the ranks route equal token counts)
  const int bn = tc::tc_block_n(std::max(R, 1), std::max(ep.E_local, 1));
  const int dbn = tc::tc_block_n_down(std::max(R, 1), std::max(ep.E_local, 1));
  if (e == cudaSuccess && ep.E_local > 0)
    e = tc::launch_build_tiles(ep.seg_l, ep.active_l, ep.n_active_l, bn, ep.tile_expert,
                               ep.tile_row0, ep.tile_rows, ep.n_tiles, ep.max_tiles, s);
  if (e == cudaSuccess && ep.E_local > 0 && dbn != bn)
    e = tc::launch_build_tiles(ep.seg_l, ep.active_l, ep.n_active_l, dbn, ep.dtile_expert,
                               ep.dtile_row0, ep.dtile_rows, ep.n_dtiles, ep.max_tiles, s);
  h->prof.end("ep_recv", p2, s);
  if (e != cudaSuccess) return cuda_fail(h, e, "ep receive");
  // 5. experts; the down epilogue writes each output row to its source rank
  if (ep.E_local > 0) {
    uint8_t *me = P.base[P.rank];
    tc::TcArgs a{};
    a.H = H;
    a.I = I;
    a.K = K;
    a.tile_expert = ep.tile_expert;
    a.tile_row0 = ep.tile_row0;
    a.tile_rows = ep.tile_rows;
    a.n_tiles = ep.n_tiles;
    a.s_ptr = EL.d_sptr;
    a.xs1 = (const float *)(me + P.off_s1);
    a.xs2 = (const float *)(me + P.off_s2);
    a.act = ep.act;
    a.act_amax = (uint32_t *)(me + P.off_amax);
    a.as1 = ep.as1;
    a.as2 = ep.as2;
    a.r_token = (const int32_t *)(me + P.off_tok);
    a.r_slot = (const int32_t *)(me + P.off_slot);
    a.r_gate = (const float *)(me + P.off_gate);
    a.r_rank = (const int32_t *)(me + P.off_rank);
    for (int q = 0; q < P.nranks; ++q) {
      a.peer_c16[q] = (int16_t *)(P.base[q] + P.off_contrib);
      a.peer_cscale[q] = (float *)(P.base[q] + P.off_cscale);
      a.peer_c32[q] = (float *)(P.base[q] + P.off_contrib);
    }
    a.contrib = nullptr;
    a.ret16 = P.ret16;
    a.status = h->status;
    cudaEvent_t p3 = h->prof.begin(s);
    e = tc::launch_gate_up_tc(EL.map_gu, bn == 64 ? ep.map_x64 : ep.map_x128, a, bn,
                              ep.max_tiles, s);
    h->prof.end("gate_up_tc", p3, s);
    p3 = h->prof.begin(s);
    if (e == cudaSuccess)
      e = tc::launch_quantize_rows(ep.act, nullptr, a.act_amax, (int)RR, I, ep.aq, RR * I,
                                   ep.as1, ep.as2, nullptr, s, ep.n_recv);
    h->prof.end("tc_act_digits", p3, s);
    if (dbn != bn) {
      a.tile_expert = ep.dtile_expert;
      a.tile_row0 = ep.dtile_row0;
      a.tile_rows = ep.dtile_rows;
      a.n_tiles = ep.n_dtiles;
    }
    p3 = h->prof.begin(s);
    if (e == cudaSuccess)
      e = tc::launch_down_tc(EL.map_dn, dbn == 64 ? ep.map_a64 : ep.map_a128, a, dbn,
                             ep.max_tiles, s);
    h->prof.end("down_tc", p3, s);
    if (e != cudaSuccess) return cuda_fail(h, e, "ep experts");
  }
  // 6. outputs are in: signal the sources; 7. combine this rank's tokens
  cudaEvent_t p4 = h->prof.begin(s);
  e = launch_ep_signal(P, epoch, s);
  if (e == cudaSuccess)
    e = launch_ep_wait_combine(P, epoch, d_resid, d_out, T, K, H, h->status, s);
  h->prof.end("ep_combine", p4, s);
  if (e != cudaSuccess) return cuda_fail(h, e, "ep combine");
  // publish, dispatch, receive, signal, combine; tile lists and the three
  // expert kernels when this rank owns experts
  h->last_launches += 5 + (ep.E_local > 0 ? 4 + (dbn != bn ? 1 : 0) : 0);
  return MOE_OK;
}
}  // namespace

extern "C" moe_status moe_ep_layer_forward(moe_handle *h, int layer, const float *d_h,
                                           const float *d_resid, float *d_out, int T,
                                           void *stream) {
  if (!h || !d_h || !d_out || ((uintptr_t)d_h & 15)) return MOE_ERR_INVALID;
  std::lock_guard<std::mutex> lock(h->mu);
  EpState &ep = h->ep;
  if (!ep.on || layer < 0 || layer >= (int)ep.layers.size() || !ep.layers[layer].set) {
    set_err(h->err, "expert-parallel layer %d not ready", layer);
    return MOE_ERR_STATE;
  }
  if (T < 0 || T > h->d.max_tokens) {
    set_err(h->err, "token count %d outside [0, %d]", T, h->d.max_tokens);
    return MOE_ERR_INVALID;
  }
  DeviceGuard g(h->device);
  cudaStream_t s = pick(h, stream);
  h->last_launches = 0;
  const int H = h->d.hidden, I = h->d.intermediate, K = h->d.top_k, E = h->d.num_experts;
  const int N = ep.nranks, R = T * K;
  const size_t ROW = ep_row_bytes(H), RR = ep.r_recv_cap;
  const LayerSlot &LS = h->layers[layer];
  const EpLayer &EL = ep.layers[layer];
  cudaError_t e = cudaSuccess;
  moe_status st = MOE_OK;
  if (ep.p2p) {
    const uint64_t key[10] = {3, (uint64_t)layer, (uint64_t)T, (uint64_t)d_h, (uint64_t)d_resid,
                              (uint64_t)d_out, (uint64_t)s, (uint64_t)h->route_mode, 0, 0};
    return graphed(h, key, s, [&] {
      h->last_launches = 0;
      return ep_forward_p2p(h, layer, d_h, d_resid, d_out, T, s);
    });
  }
  // 1. route the local tokens and bucket the routes by owner rank
  if (T > 0) {
    st = run_route(h, LS, d_h, T, h->ids, h->gates, nullptr, s, false);
    if (st != MOE_OK) return st;
    e = launch_ep_dest(h->ids, ep.d_owner, R, E, ep.dest, h->status, s);
    PermuteArgs pa{};
    pa.ids = ep.dest;
    pa.gates = h->gates;
    pa.T = T;
    pa.K = K;
    pa.E = N;
    pa.seg_off = ep.seg_dest;
    pa.active = ep.act_dest;
    pa.n_active = ep.n_dest;
    pa.r_token = ep.stok;
    pa.r_slot = ep.sslot;
    pa.r_gate = ep.sgate;
    pa.r_pos = ep.spos;
    pa.status = h->status;
    pa.scratch = h->perm_scratch;
    pa.scratch_words = h->perm_scratch_words;
    cudaEvent_t p0 = h->prof.begin(s);
    if (e == cudaSuccess) e = launch_permute(pa, s);
    if (e == cudaSuccess)
      e = launch_ep_pack(d_h, ep.stok, ep.sslot, ep.sgate, h->ids, ep.d_dest_local, R, K, H,
                         ep.send, s);
    if (e == cudaSuccess) e = launch_seg_counts(ep.seg_dest, N, ep.scount, s);
    h->prof.end("ep_dispatch_prep", p0, s);
  } else {
    e = cudaMemsetAsync(ep.scount, 0, N * sizeof(int32_t), s);
  }
  if (e != cudaSuccess) return cuda_fail(h, e, "ep dispatch prep");
  // 2. exchange counts, then the payload (the one host synchronisation)
  const NcclApi &api = nccl();
  cudaEvent_t p1 = h->prof.begin(s);
  ncclResult_t nr = api.group_start();
  for (int p = 0; p < N && nr == ncclSuccess; ++p) {
    nr = api.send(ep.scount + p, 1, ncclInt32, p, ep.comm, s);
    if (nr == ncclSuccess) nr = api.recv(ep.rcount + p, 1, ncclInt32, p, ep.comm, s);
  }
  const ncclResult_t ng = api.group_end();
  if (nr != ncclSuccess || ng != ncclSuccess) return nccl_fail(h, nr ? nr : ng, "count exchange");
  cudaMemcpyAsync(ep.h_counts, ep.scount, N * sizeof(int32_t), cudaMemcpyDeviceToHost, s);
  cudaMemcpyAsync(ep.h_counts + N, ep.rcount, N * sizeof(int32_t), cudaMemcpyDeviceToHost, s);
  e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(h, e, "count exchange");
  std::vector<size_t> soff(N + 1, 0), roff(N + 1, 0);
  for (int p = 0; p < N; ++p) {
    soff[p + 1] = soff[p] + ep.h_counts[p];
    roff[p + 1] = roff[p] + ep.h_counts[N + p];
  }
  const size_t Rr = roff[N];
  if (Rr > RR || soff[N] != (size_t)R) {
    set_err(h->err, "expert-parallel exchange sizes inconsistent (%zu received, cap %zu)", Rr, RR);
    return MOE_ERR_STATE;
  }
  nr = api.group_start();
  for (int p = 0; p < N && nr == ncclSuccess; ++p) {
    if (ep.h_counts[p])
      nr = api.send(ep.send + soff[p] * ROW, ep.h_counts[p] * ROW, ncclUint8, p, ep.comm, s);
    if (nr == ncclSuccess && ep.h_counts[N + p])
      nr = api.recv(ep.recv + roff[p] * ROW, ep.h_counts[N + p] * ROW, ncclUint8, p, ep.comm, s);
  }
  const ncclResult_t ng2 = api.group_end();
  h->prof.end("ep_dispatch_comm", p1, s);
  if (nr != ncclSuccess || ng2 != ncclSuccess) return nccl_fail(h, nr ? nr : ng2, "dispatch");
  // 3. experts on the received routes (tensor cores)
  const int Rri = (int)Rr;
  if (Rri > 0 && ep.E_local > 0) {
    cudaEvent_t p2 = h->prof.begin(s);
    e = launch_ep_unpack_meta(ep.recv, Rri, H, ep.E_local, ep.ids_l, ep.gates_l, h->status, s);
    PermuteArgs pl{};
    pl.ids = ep.ids_l;
    pl.gates = ep.gates_l;
    pl.T = Rri;
    pl.K = 1;
    pl.E = ep.E_local;
    pl.seg_off = ep.seg_l;
    pl.active = ep.active_l;
    pl.n_active = ep.n_active_l;
    pl.r_token = ep.rtok_l;
    pl.r_slot = ep.rslot_l;
    pl.r_gate = ep.rgate_l;
    pl.r_pos = ep.rpos_l;
    pl.status = h->status;
    if (e == cudaSuccess) e = launch_permute(pl, s);
    if (e == cudaSuccess)
      e = launch_ep_unpack_digits(ep.recv, ep.rtok_l, Rri, H, ep.xq, RR * H, ep.xs1, ep.xs2,
                                  ep.act_amax, s);
    const int bn = tc::tc_block_n(Rri, ep.E_local);
    const int dbn = tc::tc_block_n_down(Rri, ep.E_local);
    if (e == cudaSuccess)
      e = tc::launch_build_tiles(ep.seg_l, ep.active_l, ep.n_active_l, bn, ep.tile_expert,
                                 ep.tile_row0, ep.tile_rows, ep.n_tiles, ep.max_tiles, s);
    if (e == cudaSuccess && dbn != bn)
      e = tc::launch_build_tiles(ep.seg_l, ep.active_l, ep.n_active_l, dbn, ep.dtile_expert,
                                 ep.dtile_row0, ep.dtile_rows, ep.n_dtiles, ep.max_tiles, s);
    h->prof.end("ep_unpack", p2, s);
    tc::TcArgs a{};
    a.H = H;
    a.I = I;
    a.K = 1;  // outputs go to ybuf[received row]
    a.tile_expert = ep.tile_expert;
    a.tile_row0 = ep.tile_row0;
    a.tile_rows = ep.tile_rows;
    a.n_tiles = ep.n_tiles;
    a.s_ptr = EL.d_sptr;
    a.xs1 = ep.xs1;
    a.xs2 = ep.xs2;
    a.act = ep.act;
    a.act_amax = ep.act_amax;
    a.as1 = ep.as1;
    a.as2 = ep.as2;
    a.r_token = ep.rtok_l;
    a.r_slot = ep.rslot_l;
    a.r_gate = ep.rgate_l;
    a.contrib = ep.ybuf;
    a.status = h->status;
    const int tiles =
        std::min(ep.max_tiles, (Rri + bn - 1) / bn + std::min(ep.E_local, Rri));
    cudaEvent_t p3 = h->prof.begin(s);
    if (e == cudaSuccess)
      e = tc::launch_gate_up_tc(EL.map_gu, bn == 64 ? ep.map_x64 : ep.map_x128, a, bn, tiles, s);
    h->prof.end("gate_up_tc", p3, s);
    p3 = h->prof.begin(s);
    if (e == cudaSuccess)
      e = tc::launch_quantize_rows(ep.act, nullptr, ep.act_amax, Rri, I, ep.aq, RR * I, ep.as1,
                                   ep.as2, nullptr, s);
    h->prof.end("tc_act_digits", p3, s);
    int dtiles = tiles;
    if (dbn != bn) {
      a.tile_expert = ep.dtile_expert;
      a.tile_row0 = ep.dtile_row0;
      a.tile_rows = ep.dtile_rows;
      a.n_tiles = ep.n_dtiles;
      dtiles = std::min(ep.max_tiles, (Rri + dbn - 1) / dbn + std::min(ep.E_local, Rri));
    }
    p3 = h->prof.begin(s);
    if (e == cudaSuccess)
      e = tc::launch_down_tc(EL.map_dn, dbn == 64 ? ep.map_a64 : ep.map_a128, a, dbn, dtiles, s);
    h->prof.end("down_tc", p3, s);
    if (e != cudaSuccess) return cuda_fail(h, e, "ep experts");
  }
  // 4. send the gate-weighted outputs back; combine on the owner in slot order
  cudaEvent_t p4 = h->prof.begin(s);
  nr = api.group_start();
  for (int p = 0; p < N && nr == ncclSuccess; ++p) {
    if (ep.h_counts[N + p])
      nr = api.send(ep.ybuf + roff[p] * H, ep.h_counts[N + p] * (size_t)H, ncclFloat32, p,
                    ep.comm, s);
    if (nr == ncclSuccess && ep.h_counts[p])
      nr = api.recv(ep.ret + soff[p] * H, ep.h_counts[p] * (size_t)H, ncclFloat32, p, ep.comm, s);
  }
  const ncclResult_t ng3 = api.group_end();
  h->prof.end("ep_combine_comm", p4, s);
  if (nr != ncclSuccess || ng3 != ncclSuccess) return nccl_fail(h, nr ? nr : ng3, "combine");
  if (T > 0) {
    cudaEvent_t p5 = h->prof.begin(s);
    e = launch_ep_gather_combine(ep.ret, ep.spos, d_resid, d_out, T, K, H, h->status, s);
    h->prof.end("combine", p5, s);
    if (e != cudaSuccess) return cuda_fail(h, e, "ep combine");
  }
  h->last_launches += 12;
  return MOE_OK;
}
