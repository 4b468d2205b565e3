// Expert parallelism: kernels around the NCCL exchange (experts sharded over
// GPUs, one process per GPU).  The reference has no multi-GPU path; this is
// the dispatch/combine of the north star's expert-parallel configuration.
//
// A route travels as the tensor-core path's own input: the two int8 digit
// planes of its token row plus the two digit scales, the gate and the
// destination-local expert id (2H + 16 bytes; half of the fp32 row), so the
// receiving GPU multiplies exactly the integers the single-GPU path would.
// The gate-weighted expert outputs come back in fp32 and are summed on the
// owner of the token in slot order; results are bit-identical to the
// single-GPU tensor-core path.
#include <algorithm>
#include <cstdlib>
#include <cstring>

#include "common.cuh"
#include "digits.cuh"
#include "kernels.h"

namespace moe {
namespace {

__global__ void dest_kernel(const uint32_t *__restrict__ ids, const int32_t *__restrict__ owner,
                            int R, int E, uint32_t *__restrict__ dest, uint32_t *status) {
  for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < R; r += gridDim.x * blockDim.x) {
    const uint32_t e = ids[r];
    if (e >= (uint32_t)E) {
      set_status(status, kStatusBadRoute);
      dest[r] = 0;
    } else {
      dest[r] = (uint32_t)owner[e];
    }
  }
}

// One warp per send position p: quantize the token row into two int8 digits
// (s = max|x| / 127, d1 = rint(x/s), d2 = rint((x/s - d1) * 254)) -- the same
// function as the single-GPU path -- and append scales, gate, local id.
__global__ void pack_kernel(const float *__restrict__ x, const int32_t *__restrict__ r_token,
                            const int32_t *__restrict__ r_slot, const float *__restrict__ r_gate,
                            const uint32_t *__restrict__ ids, const int32_t *__restrict__ local_of,
                            int R, int K, int H, uint8_t *__restrict__ send) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= R) return;
  const int t = r_token[warp], slot = r_slot[warp];
  const float *xr = x + (size_t)t * H;
  float amax = 0.0f;
  for (int c = lane * 4; c < H; c += 128) {
    const float4 v = *reinterpret_cast<const float4 *>(xr + c);
    amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  const float s = digits::row_scale(amax);
  const float inv = 1.0f / s;
  uint8_t *row = send + (size_t)warp * ep_row_bytes(H);
  for (int c = lane * 4; c < H; c += 128) {
    const float4 v = *reinterpret_cast<const float4 *>(xr + c);
    uint32_t p2;
    const uint32_t p1 = digits::split4(v.x, v.y, v.z, v.w, inv, p2);
    *reinterpret_cast<uint32_t *>(row + c) = p1;
    *reinterpret_cast<uint32_t *>(row + H + c) = p2;
  }
  if (lane == 0) {
    float *meta = reinterpret_cast<float *>(row + 2 * H);
    meta[0] = s;
    meta[1] = s / 254.0f;
    meta[2] = r_gate[warp];
    meta[3] = __int_as_float(local_of[ids[(size_t)t * K + slot]]);
  }
}

__global__ void unpack_meta_kernel(const uint8_t *__restrict__ recv, int R, int H, int E_local,
                                   uint32_t *__restrict__ ids_local, float *__restrict__ gates,
                                   uint32_t *status) {
  for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < R; r += gridDim.x * blockDim.x) {
    const float *meta = reinterpret_cast<const float *>(recv + (size_t)r * ep_row_bytes(H) + 2 * H);
    const int e = __float_as_int(meta[3]);
    if (e < 0 || e >= E_local) {
      set_status(status, kStatusBadRoute);
      ids_local[r] = 0;
    } else {
      ids_local[r] = (uint32_t)e;
    }
    gates[r] = meta[2];
  }
}

// Permuted position q <- received row src[q]: digit planes and scales.
__global__ void unpack_digits_kernel(const uint8_t *__restrict__ recv,
                                     const int32_t *__restrict__ src, int R, int H,
                                     int8_t *__restrict__ xq, size_t plane, float *__restrict__ s1,
                                     float *__restrict__ s2, uint32_t *__restrict__ amax_reset) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= R) return;
  const uint8_t *row = recv + (size_t)src[warp] * ep_row_bytes(H);
  int8_t *q1 = xq + (size_t)warp * H;
  int8_t *q2 = xq + plane + (size_t)warp * H;
  for (int c = lane * 16; c < H; c += 512) {
    *reinterpret_cast<uint4 *>(q1 + c) = *reinterpret_cast<const uint4 *>(row + c);
    *reinterpret_cast<uint4 *>(q2 + c) = *reinterpret_cast<const uint4 *>(row + H + c);
  }
  if (lane == 0) {
    const float *meta = reinterpret_cast<const float *>(row + 2 * H);
    s1[warp] = meta[0];
    s2[warp] = meta[1];
    amax_reset[warp] = 0u;
  }
}

// out[t] = resid[t] (or 0) + ret[pos(t, 0)] + ... + ret[pos(t, K-1)], slot order.
__global__ void gather_combine_kernel(const float *__restrict__ ret,
                                      const int32_t *__restrict__ pos,
                                      const float *__restrict__ resid, float *__restrict__ out,
                                      int T, int K, int H, uint32_t *status) {
  bool bad = false;
  const size_t n = (size_t)T * H;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
       i += (size_t)gridDim.x * blockDim.x) {
    const size_t t = i / H, j = i % H;
    float acc = resid ? resid[i] : 0.0f;
    for (int k = 0; k < K; ++k) acc = __fadd_rn(acc, ret[(size_t)pos[t * K + k] * H + j]);
    bad |= !is_finite_f(acc);
    out[i] = acc;
  }
  if (bad) set_status(status, kStatusNonFinite);
}

}  // namespace

cudaError_t launch_ep_dest(const uint32_t *ids, const int32_t *owner, int R, int E,
                           uint32_t *dest, uint32_t *status, cudaStream_t s) {
  if (R <= 0) return cudaSuccess;
  dest_kernel<<<(R + 255) / 256, 256, 0, s>>>(ids, owner, R, E, dest, status);
  return cudaGetLastError();
}

cudaError_t launch_ep_pack(const float *x, const int32_t *r_token, const int32_t *r_slot,
                           const float *r_gate, const uint32_t *ids, const int32_t *local_of,
                           int R, int K, int H, uint8_t *send, cudaStream_t s) {
  if (R <= 0) return cudaSuccess;
  pack_kernel<<<(R + 7) / 8, 256, 0, s>>>(x, r_token, r_slot, r_gate, ids, local_of, R, K, H,
                                          send);
  return cudaGetLastError();
}

cudaError_t launch_ep_unpack_meta(const uint8_t *recv, int R, int H, int E_local,
                                  uint32_t *ids_local, float *gates, uint32_t *status,
                                  cudaStream_t s) {
  if (R <= 0) return cudaSuccess;
  unpack_meta_kernel<<<(R + 255) / 256, 256, 0, s>>>(recv, R, H, E_local, ids_local, gates,
                                                     status);
  return cudaGetLastError();
}

cudaError_t launch_ep_unpack_digits(const uint8_t *recv, const int32_t *src, int R, int H,
                                    int8_t *xq, size_t plane, float *s1, float *s2,
                                    uint32_t *amax_reset, cudaStream_t s) {
  if (R <= 0) return cudaSuccess;
  unpack_digits_kernel<<<(R + 7) / 8, 256, 0, s>>>(recv, src, R, H, xq, plane, s1, s2,
                                                   amax_reset);
  return cudaGetLastError();
}

cudaError_t launch_ep_gather_combine(const float *ret, const int32_t *pos, const float *resid,
                                     float *out, int T, int K, int H, uint32_t *status,
                                     cudaStream_t s) {
  if (T <= 0) return cudaSuccess;
  const size_t n = (size_t)T * H;
  const int blocks = (int)std::min<size_t>((n + 255) / 256, 148 * 8);
  gather_combine_kernel<<<blocks, 256, 0, s>>>(ret, pos, resid, out, T, K, H, status);
  return cudaGetLastError();
}

}  // namespace moe

namespace moe {
namespace {
__global__ void seg_counts_kernel(const int32_t *__restrict__ seg, int n, int32_t *__restrict__ cnt) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) cnt[i] = seg[i + 1] - seg[i];
}
}  // namespace

cudaError_t launch_seg_counts(const int32_t *seg, int n, int32_t *cnt, cudaStream_t s) {
  seg_counts_kernel<<<(n + 127) / 128, 128, 0, s>>>(seg, n, cnt);
  return cudaGetLastError();
}
}  // namespace moe

// ---------------------------------------------------------------------------
// Device-driven exchange over NVLink peer memory (CUDA IPC).  Every rank owns
// one region, mapped by all peers at the same offsets (EpP2P).  No host
// synchronisation and no collective library on the data path:
//   1. publish: this rank's per-expert route counts go into every peer's
//      count matrix, then flag A;
//   2. dispatch: after every rank's counts are in, each route is quantized
//      and written straight into its owner's expert-sorted tensor-core input
//      (digit planes, scales, gate, source rank/token/slot); the last CTA
//      raises flag B on every peer;
//   3. receive: the owner waits for flag B from every rank and derives its
//      expert segments from the count matrix;
//   4. the down GEMM's epilogue writes gate * y straight into the source
//      rank's [T, K, H] contribution buffer; flag C follows;
//   5. combine: the source waits for flag C from every rank and sums the
//      contributions in slot order.
// Flags carry the call's epoch (monotonic), so nothing is ever reset.  The
// epoch lives in device memory and the publish kernel advances it, so a
// captured sequence of these launches replays correctly.  Every wait is
// bounded; on expiry the kernel records kStatusTimeout and moves on.
// ---------------------------------------------------------------------------
namespace moe {
namespace {

// Wait until flags[0..n) all reach epoch; false once `limit` SM clock
// cycles have passed (the handle's wait bound, EpP2P::wait_cycles).
__device__ __forceinline__ bool ep_wait_flags(const uint32_t *flags, int n, uint32_t epoch,
                                              long long limit) {
  const long long t0 = clock64();
  for (int q = 0; q < n; ++q) {
    const volatile uint32_t *f = flags + q;
    while (*f < epoch)
      if (clock64() - t0 > limit) return false;
  }
  __threadfence_system();
  return true;
}

__global__ void wait_probe_kernel(const uint32_t *flags, int n, uint32_t target, long long limit,
                                  uint32_t *status) {
  if (threadIdx.x == 0 && !ep_wait_flags(flags, n, target, limit))
    set_status(status, kStatusTimeout);
}

__device__ __forceinline__ uint8_t *peer_at(const EpP2P &p, int rank, size_t off) {
  return p.base[rank] + off;
}

__global__ void ep_publish_kernel(const int32_t *__restrict__ seg_off, int E, EpP2P p,
                                  uint32_t *epoch_p) {
  __shared__ uint32_t ep_now;
  if (threadIdx.x == 0) {
    ep_now = *epoch_p + 1;
    *epoch_p = ep_now;
  }
  __syncthreads();
  const uint32_t epoch = ep_now;
  const int par = epoch & 1;
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    const int32_t c = seg_off[e + 1] - seg_off[e];
    for (int q = 0; q < p.nranks; ++q) {
      int32_t *cm = reinterpret_cast<int32_t *>(peer_at(p, q, p.off_counts));
      cm[((size_t)par * p.nranks + p.rank) * E + e] = c;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    for (int q = 0; q < p.nranks; ++q)
      reinterpret_cast<volatile uint32_t *>(peer_at(p, q, p.off_flags))[0 * kEpMaxRanks + p.rank] =
          epoch;
  }
}

// dest_base[e]: first position, in the owner's expert-sorted receive buffer,
// of this rank's routes to expert e = (routes of the owner's earlier local
// experts, all sources) + (routes to e from lower ranks).
__device__ void ep_dest_bases(const int32_t *cm, const int32_t *owner, int E, int me, int N,
                              int32_t *tot, int32_t *base) {
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int t = 0, before = 0;
    for (int q = 0; q < N; ++q) {
      const int c = cm[(size_t)q * E + e];
      t += c;
      if (q < me) before += c;
    }
    tot[e] = t;
    base[e] = before;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    const int o = owner[e];
    int s = 0;
    for (int e2 = 0; e2 < e; ++e2)
      if (owner[e2] == o) s += tot[e2];
    base[e] += s;
  }
  __syncthreads();
}

__global__ void __launch_bounds__(256) ep_dispatch_kernel(
    const float *__restrict__ x, const int32_t *__restrict__ seg_off,
    const uint32_t *__restrict__ ids, const float *__restrict__ gates,
    const int32_t *__restrict__ r_pos, const int32_t *__restrict__ owner, int E, int T, int K,
    int H, EpP2P p, const uint32_t *epoch_p, uint32_t *done, uint32_t *status, int per_token) {
  __shared__ int32_t tot[kMaxExperts], base[kMaxExperts], segs[kMaxExperts + 1];
  __shared__ int ok;
  const uint32_t epoch = *epoch_p;
  if (threadIdx.x == 0) {
    ok = ep_wait_flags(reinterpret_cast<const uint32_t *>(p.base[p.rank] + p.off_flags) +
                           0 * kEpMaxRanks,
                       p.nranks, epoch, p.wait_cycles);
    if (!ok) set_status(status, kStatusTimeout);
  }
  for (int e = threadIdx.x; e <= E; e += blockDim.x) segs[e] = seg_off[e];
  __syncthreads();
  const int par = epoch & 1;
  if (ok) {
    const int32_t *cm =
        reinterpret_cast<const int32_t *>(p.base[p.rank] + p.off_counts) + (size_t)par * p.nranks * E;
    ep_dest_bases(cm, owner, E, p.rank, p.nranks, tot, base);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (per_token) {
      // one warp per token: the row is quantized once and stored at each of
      // its K routes' rows in their owners' expert-sorted buffers
      for (int t = blockIdx.x * 8 + warp; t < T; t += gridDim.x * 8) {
        int q = 0, pos = 0, slot_ok = 0;
        float g = 0.0f;
        if (lane < K) {
          const uint32_t e = ids[(size_t)t * K + lane];
          const int r = r_pos[(size_t)t * K + lane];
          if (e < (uint32_t)E && r >= 0) {
            q = owner[e];
            pos = base[e] + (r - segs[e]);
            g = gates[(size_t)t * K + lane];
            slot_ok = 1;
          }
        }
        const unsigned vmask = __ballot_sync(0xffffffffu, slot_ok);
        uint8_t *dst[kMaxTopK];
  #pragma unroll
        for (int k = 0; k < kMaxTopK; ++k) {
          const int qk = __shfl_sync(0xffffffffu, q, k);
          const int pk = __shfl_sync(0xffffffffu, pos, k);
          dst[k] = peer_at(p, qk, p.off_xq) + (size_t)pk * H;
        }
        const float *xr = x + (size_t)t * H;
        // the single-GPU tensor path's two-digit quantization of the row
        float amax = 0.0f;
        for (int c = lane * 4; c < H; c += 128) {
          const float4 v = *reinterpret_cast<const float4 *>(xr + c);
          amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
        }
  #pragma unroll
        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        const float s = digits::row_scale(amax);
        const float inv = 1.0f / s;
        // 16 elements per lane per pass: 16-byte stores, 512 bytes per warp
        // instruction on the link (H is a multiple of 16)
        for (int c = lane * 16; c < H; c += 512) {
          uint32_t p1[4], p2[4];
  #pragma unroll
          for (int w4 = 0; w4 < 4; ++w4) {
            const float4 v = *reinterpret_cast<const float4 *>(xr + c + 4 * w4);
            p1[w4] = digits::split4(v.x, v.y, v.z, v.w, inv, p2[w4]);
          }
          const uint4 v1 = make_uint4(p1[0], p1[1], p1[2], p1[3]);
          const uint4 v2 = make_uint4(p2[0], p2[1], p2[2], p2[3]);
  #pragma unroll
          for (int k = 0; k < kMaxTopK; ++k)
            if ((vmask >> k) & 1u) {
              *reinterpret_cast<uint4 *>(dst[k] + c) = v1;
              *reinterpret_cast<uint4 *>(dst[k] + p.plane + c) = v2;
            }
        }
        if (slot_ok) {
          reinterpret_cast<float *>(peer_at(p, q, p.off_s1))[pos] = s;
          reinterpret_cast<float *>(peer_at(p, q, p.off_s2))[pos] = s / 254.0f;
          reinterpret_cast<float *>(peer_at(p, q, p.off_gate))[pos] = g;
          reinterpret_cast<int32_t *>(peer_at(p, q, p.off_rank))[pos] = p.rank;
          reinterpret_cast<int32_t *>(peer_at(p, q, p.off_tok))[pos] = t;
          reinterpret_cast<int32_t *>(peer_at(p, q, p.off_slot))[pos] = lane;
          reinterpret_cast<uint32_t *>(peer_at(p, q, p.off_amax))[pos] = 0u;
        }
      }
    } else {
      // one warp per route: it digitises its token's row (every route of a
      // token gets the same digits) and stores them at the route's row in its
      // owner's expert-sorted buffer.  With a warp per route rather than per
      // token, every SM issues peer stores.
      const int R = T * K;
      for (int r = blockIdx.x * 8 + warp; r < R; r += gridDim.x * 8) {
        const uint32_t e = ids[r];
        const int rp = r_pos[r];
        if (!(e < (uint32_t)E && rp >= 0)) continue;  // warp-uniform
        const int t = r / K, slot = r - t * K;
        const int q = owner[e];
        const int pos = base[e] + (rp - segs[e]);
        uint8_t *dst = peer_at(p, q, p.off_xq) + (size_t)pos * H;
        const float *xr = x + (size_t)t * H;
        // the single-GPU tensor path's two-digit quantization of the row
        float amax = 0.0f;
        for (int c = lane * 4; c < H; c += 128) {
          const float4 v = *reinterpret_cast<const float4 *>(xr + c);
          amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
        }
  #pragma unroll
        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        const float s = digits::row_scale(amax);
        const float inv = 1.0f / s;
        // 16 elements per lane per pass: 16-byte stores, 512 bytes per warp
        // instruction on the link (H is a multiple of 16)
        for (int c = lane * 16; c < H; c += 512) {
          uint32_t p1[4], p2[4];
  #pragma unroll
          for (int w4 = 0; w4 < 4; ++w4) {
            const float4 v = *reinterpret_cast<const float4 *>(xr + c + 4 * w4);
            p1[w4] = digits::split4(v.x, v.y, v.z, v.w, inv, p2[w4]);
          }
          *reinterpret_cast<uint4 *>(dst + c) = make_uint4(p1[0], p1[1], p1[2], p1[3]);
          *reinterpret_cast<uint4 *>(dst + p.plane + c) = make_uint4(p2[0], p2[1], p2[2], p2[3]);
        }
        if (lane == 0) {
          reinterpret_cast<float *>(peer_at(p, q, p.off_s1))[pos] = s;
          reinterpret_cast<float *>(peer_at(p, q, p.off_s2))[pos] = s / 254.0f;
          reinterpret_cast<float *>(peer_at(p, q, p.off_gate))[pos] = gates[r];
          reinterpret_cast<int32_t *>(peer_at(p, q, p.off_rank))[pos] = p.rank;
          reinterpret_cast<int32_t *>(peer_at(p, q, p.off_tok))[pos] = t;
          reinterpret_cast<int32_t *>(peer_at(p, q, p.off_slot))[pos] = slot;
          reinterpret_cast<uint32_t *>(peer_at(p, q, p.off_amax))[pos] = 0u;
        }
      }
    }
  }
  // the last CTA to finish raises flag B on every peer
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const uint32_t prev = atomicAdd(done, 1u);
    if (prev + 1 == epoch * gridDim.x) {
      __threadfence_system();
      for (int q = 0; q < p.nranks; ++q)
        reinterpret_cast<volatile uint32_t *>(peer_at(p, q, p.off_flags))[1 * kEpMaxRanks + p.rank] =
            epoch;
    }
  }
}

// One CTA: wait for every rank's routes, then this rank's expert segments
// (local expert order) from the count matrix.
__global__ void __launch_bounds__(256) ep_recv_prep_kernel(const int32_t *__restrict__ owner,
                                                           int E, EpP2P p,
                                                           const uint32_t *epoch_p,
                                                           int32_t *seg_l, int32_t *active_l,
                                                           int32_t *n_active_l,
                                                           int32_t *n_recv, uint32_t *status) {
  __shared__ int ok;
  const uint32_t epoch = *epoch_p;
  __shared__ int32_t tot[kMaxExperts];
  if (threadIdx.x == 0) {
    ok = ep_wait_flags(reinterpret_cast<const uint32_t *>(p.base[p.rank] + p.off_flags) +
                           1 * kEpMaxRanks,
                       p.nranks, epoch, p.wait_cycles);
    if (!ok) set_status(status, kStatusTimeout);
  }
  __syncthreads();
  const int par = epoch & 1;
  const int32_t *cm =
      reinterpret_cast<const int32_t *>(p.base[p.rank] + p.off_counts) + (size_t)par * p.nranks * E;
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int t = 0;
    if (ok)
      for (int q = 0; q < p.nranks; ++q) t += cm[(size_t)q * E + e];
    tot[e] = t;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int acc = 0, el = 0, na = 0;
    for (int e = 0; e < E; ++e) {
      if (owner[e] != p.rank) continue;
      seg_l[el] = acc;
      if (tot[e] > 0) active_l[na++] = el;
      acc += tot[e];
      ++el;
    }
    seg_l[el] = acc;
    *n_active_l = na;
    *n_recv = acc;
  }
}

__global__ void ep_signal_kernel(EpP2P p, const uint32_t *epoch_p) {
  const uint32_t epoch = *epoch_p;
  __threadfence_system();
  for (int q = 0; q < p.nranks; ++q)
    reinterpret_cast<volatile uint32_t *>(peer_at(p, q, p.off_flags))[2 * kEpMaxRanks + p.rank] =
        epoch;
}

// out[t] = resid[t] (or 0) + contrib[t, 0] + ... + contrib[t, K-1], slot
// order, once every rank's contributions are in.
__global__ void ep_wait_combine_kernel(EpP2P p, const uint32_t *epoch_p,
                                       const float *__restrict__ resid, float *__restrict__ out,
                                       int T, int K, int H, uint32_t *status) {
  __shared__ int ok;
  const uint32_t epoch = *epoch_p;
  if (threadIdx.x == 0) {
    ok = ep_wait_flags(reinterpret_cast<const uint32_t *>(p.base[p.rank] + p.off_flags) +
                           2 * kEpMaxRanks,
                       p.nranks, epoch, p.wait_cycles);
    if (!ok) set_status(status, kStatusTimeout);
  }
  __syncthreads();
  if (!ok) return;
  // the owners' int16 rows and their per-(route, 32-row block) scales
  const int16_t *q16 = reinterpret_cast<const int16_t *>(p.base[p.rank] + p.off_contrib);
  const float *sc = reinterpret_cast<const float *>(p.base[p.rank] + p.off_cscale);
  const int hb = (H + 31) / 32;
  bool bad = false;
  const bool vec = (H & 3) == 0 && K <= kMaxTopK &&
                   (((uintptr_t)out | (uintptr_t)resid) & 15) == 0 &&
                   (size_t)T * H / 4 < (1u << 31);
  if (!p.ret16 && vec) {
    // fp32 rows, 4 columns per thread with 32-bit index math; all K slot
    // loads issued before the first add, then the single-GPU combine's
    // slot order (bit-identical)
    const float *c32 = reinterpret_cast<const float *>(p.base[p.rank] + p.off_contrib);
    const uint32_t H4 = H / 4, n4 = (uint32_t)((size_t)T * H / 4);
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n4;
         i += gridDim.x * blockDim.x) {
      const uint32_t t = i / H4, j4 = i - t * H4;
      float4 acc = resid ? reinterpret_cast<const float4 *>(resid)[i] : make_float4(0, 0, 0, 0);
      float4 v[kMaxTopK];
#pragma unroll
      for (int k = 0; k < kMaxTopK; ++k)
        if (k < K)
          v[k] = __ldcg(reinterpret_cast<const float4 *>(c32 + ((size_t)t * K + k) * H) + j4);
#pragma unroll
      for (int k = 0; k < kMaxTopK; ++k)
        if (k < K) {
          acc.x = __fadd_rn(acc.x, v[k].x);
          acc.y = __fadd_rn(acc.y, v[k].y);
          acc.z = __fadd_rn(acc.z, v[k].z);
          acc.w = __fadd_rn(acc.w, v[k].w);
        }
      bad |= !(is_finite_f(acc.x) && is_finite_f(acc.y) && is_finite_f(acc.z) &&
               is_finite_f(acc.w));
      reinterpret_cast<float4 *>(out)[i] = acc;
    }
    if (bad) set_status(status, kStatusNonFinite);
    return;
  }
  if (!p.ret16) {
    // fp32 rows: slot order as the single-GPU combine (bit-identical)
    const float *c32 = reinterpret_cast<const float *>(p.base[p.rank] + p.off_contrib);
    const size_t n = (size_t)T * H;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x) {
      const size_t t = i / H, j = i % H;
      float acc = resid ? resid[i] : 0.0f;
      float v[kMaxTopK];
#pragma unroll
      for (int k = 0; k < kMaxTopK; ++k)
        if (k < K) v[k] = __ldcg(c32 + (t * K + k) * H + j);
#pragma unroll
      for (int k = 0; k < kMaxTopK; ++k)
        if (k < K) acc = __fadd_rn(acc, v[k]);
      bad |= !is_finite_f(acc);
      out[i] = acc;
    }
    if (bad) set_status(status, kStatusNonFinite);
    return;
  }
  // slot order as the single-GPU combine; 4 columns per thread (one scale
  // block), all K slot loads issued before the first add (the peers' stores
  // reached these buffers before their flags C, so the loads bypass L1)
  if (vec) {
    const uint32_t H4 = H / 4, n4 = (uint32_t)((size_t)T * H / 4);
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n4;
         i += gridDim.x * blockDim.x) {
      const uint32_t t = i / H4, j4 = i - t * H4, j = 4 * j4;
      float4 acc = resid ? reinterpret_cast<const float4 *>(resid)[i] : make_float4(0, 0, 0, 0);
      uint2 v[kMaxTopK];
      float f[kMaxTopK];
#pragma unroll
      for (int k = 0; k < kMaxTopK; ++k)
        if (k < K) {
          const size_t row = (size_t)t * K + k;
          v[k] = __ldcg(reinterpret_cast<const uint2 *>(q16 + row * H + j));
          f[k] = __ldcg(sc + row * hb + j / 32);
        }
#pragma unroll
      for (int k = 0; k < kMaxTopK; ++k)
        if (k < K) {
          acc.x = __fmaf_rn((float)(int16_t)(v[k].x & 0xFFFFu), f[k], acc.x);
          acc.y = __fmaf_rn((float)(int16_t)(v[k].x >> 16), f[k], acc.y);
          acc.z = __fmaf_rn((float)(int16_t)(v[k].y & 0xFFFFu), f[k], acc.z);
          acc.w = __fmaf_rn((float)(int16_t)(v[k].y >> 16), f[k], acc.w);
        }
      bad |= !(is_finite_f(acc.x) && is_finite_f(acc.y) && is_finite_f(acc.z) &&
               is_finite_f(acc.w));
      reinterpret_cast<float4 *>(out)[i] = acc;
    }
  } else {
    const size_t n = (size_t)T * H;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n;
         i += (size_t)gridDim.x * blockDim.x) {
      const size_t t = i / H, j = i % H;
      float acc = resid ? resid[i] : 0.0f;
      for (int k = 0; k < K; ++k) {
        const size_t row = t * K + k;
        acc = __fmaf_rn((float)__ldcg(q16 + row * H + j), __ldcg(sc + row * hb + j / 32), acc);
      }
      bad |= !is_finite_f(acc);
      out[i] = acc;
    }
  }
  if (bad) set_status(status, kStatusNonFinite);
}

}  // namespace

cudaError_t launch_ep_publish(const int32_t *seg_off, int E, const EpP2P &p, uint32_t *epoch,
                              cudaStream_t s) {
  ep_publish_kernel<<<1, 256, 0, s>>>(seg_off, E, p, epoch);
  return cudaGetLastError();
}

cudaError_t launch_ep_dispatch(const float *x, const int32_t *seg_off, const uint32_t *ids,
                               const float *gates, const int32_t *r_pos, const int32_t *owner,
                               int E, int T, int K, int H, const EpP2P &p, const uint32_t *epoch,
                               uint32_t *done, int grid, uint32_t *status, cudaStream_t s) {
  if (K > kMaxTopK) return cudaErrorInvalidValue;
  // One warp per token digitises a row once for all its routes; one warp
  // per route keeps every CTA busy when tokens are few.  By default a warp
  // per token while the tokens fill at least half of the grid's warps
  // (2 B200s, 2048 tokens a rank: 86.5 us per token vs 92.7 per route),
  // else a warp per route.  MOE_EP_DISPATCH=token|route pins the mode.
  static const int pin = [] {
    const char *v = getenv("MOE_EP_DISPATCH");
    if (v && strcmp(v, "route") == 0) return 0;
    if (v && strcmp(v, "token") == 0) return 1;
    return -1;
  }();
  const int per_token = pin >= 0 ? pin : (2 * T >= grid * 8 ? 1 : 0);
  ep_dispatch_kernel<<<grid, 256, 0, s>>>(x, seg_off, ids, gates, r_pos, owner, E, T, K, H, p,
                                          epoch, done, status, per_token);
  return cudaGetLastError();
}

cudaError_t launch_ep_recv_prep(const int32_t *owner, int E, const EpP2P &p,
                                const uint32_t *epoch, int32_t *seg_l, int32_t *active_l, int32_t *n_active_l,
                                int32_t *n_recv, uint32_t *status, cudaStream_t s) {
  ep_recv_prep_kernel<<<1, 256, 0, s>>>(owner, E, p, epoch, seg_l, active_l, n_active_l, n_recv,
                                        status);
  return cudaGetLastError();
}

cudaError_t launch_wait_probe(const uint32_t *flags, int n, uint32_t target,
                              long long wait_cycles, uint32_t *status, cudaStream_t s) {
  wait_probe_kernel<<<1, 32, 0, s>>>(flags, n, target, wait_cycles, status);
  return cudaGetLastError();
}

cudaError_t launch_ep_signal(const EpP2P &p, const uint32_t *epoch, cudaStream_t s) {
  ep_signal_kernel<<<1, 1, 0, s>>>(p, epoch);
  return cudaGetLastError();
}

cudaError_t launch_ep_wait_combine(const EpP2P &p, const uint32_t *epoch, const float *resid,
                                   float *out, int T, int K, int H, uint32_t *status,
                                   cudaStream_t s) {
  const size_t n = (size_t)T * H;
  const int blocks = (int)std::max<size_t>(1, std::min<size_t>((n + 255) / 256, 148 * 8));
  ep_wait_combine_kernel<<<blocks, 256, 0, s>>>(p, epoch, resid, out, T, K, H, status);
  return cudaGetLastError();
}

}  // namespace moe
