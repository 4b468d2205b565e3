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

#include "common.cuh"
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
  const float s = amax > 0.0f ? amax / 127.0f : 1.0f;
  const float inv = 1.0f / s;
  uint8_t *row = send + (size_t)warp * ep_row_bytes(H);
  for (int c = lane * 4; c < H; c += 128) {
    const float4 v = *reinterpret_cast<const float4 *>(xr + c);
    const float in[4] = {v.x, v.y, v.z, v.w};
    uint32_t p1 = 0, p2 = 0;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float q = in[k] * inv;
      const float a1 = fminf(fmaxf(rintf(q), -127.0f), 127.0f);
      const float a2 = fminf(fmaxf(rintf((q - a1) * 254.0f), -127.0f), 127.0f);
      p1 |= (uint32_t)(uint8_t)(int8_t)(int)a1 << (8 * k);
      p2 |= (uint32_t)(uint8_t)(int8_t)(int)a2 << (8 * k);
    }
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
