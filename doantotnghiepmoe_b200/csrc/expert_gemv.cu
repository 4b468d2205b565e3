// Grouped INT8 (or INT4) x FP32 GEMV over expert segments, one launch per phase
// (gate/up, then down): the decode-sized expert path used by the layer API
// and by the GpuExpertKernels drop-in.  The arithmetic lives in
// gemv_core.cuh; this file only maps work items to CTAs.
//
// Work decomposition: an item is (expert segment, block of rows); a
// persistent grid walks the items.  Tokens of the segment are staged through
// shared memory kTG at a time.
#include <algorithm>

#include "gemv_core.cuh"
#include "kernels.h"

namespace moe {
namespace {

using namespace gemv;
constexpr int kThreads = 128;  // 4 warps: small items, many CTAs per SM

__device__ __forceinline__ int seg_count(const GemvArgs &a) {
  return a.n_active_dev ? *a.n_active_dev : a.n_active_max;
}

template <bool kVec, int kQ>
__global__ void __launch_bounds__(kThreads) gate_up_kernel(GemvArgs a) {
  extern __shared__ float xs[];  // [kTG][H]
  const int rows_per_item = kGURowsPerWarp * (kThreads / 32);
  const int nblk = (a.I + rows_per_item - 1) / rows_per_item;
  const int nitems = seg_count(a) * nblk;
  for (int item = blockIdx.x; item < nitems; item += gridDim.x) {
    const int j = item / nblk, b = item % nblk;
    const int e = a.active ? a.active[j] : j;
    gate_up_item<kVec, kTG, kPF, kQ>(a.w_ptr[e], a.s_ptr[e], a.H, a.I, b * rows_per_item, a.seg_off[e],
                       a.seg_off[e + 1], a.r_token, a.x, xs, a.act);
  }
}

template <bool kVec, int kQ>
__global__ void __launch_bounds__(kThreads) down_kernel(GemvArgs a) {
  extern __shared__ float xs[];  // [kTG][I]
  const int rows_per_item = kDNRowsPerWarp * (kThreads / 32);
  const int nblk = (a.H + rows_per_item - 1) / rows_per_item;
  const int nitems = seg_count(a) * nblk;
  bool good = true;
  for (int item = blockIdx.x; item < nitems; item += gridDim.x) {
    const int j = item / nblk, b = item % nblk;
    const int e = a.active ? a.active[j] : j;
    if (a.contrib) {
      good &= down_item<kVec, kTG, kPF, kQ>(a.w_ptr[e], a.s_ptr[e], a.H, a.I, b * rows_per_item,
                              a.seg_off[e], a.seg_off[e + 1], a.act, xs,
                              [&](int r, int row, float y) {
                                const int tok = a.r_token[r], slot = a.r_slot[r];
                                a.contrib[((size_t)tok * a.K + slot) * a.H + row] =
                                    __fmul_rn(a.r_gate[r], y);
                              });
    } else {
      good &= down_item<kVec, kTG, kPF, kQ>(a.w_ptr[e], a.s_ptr[e], a.H, a.I, b * rows_per_item,
                              a.seg_off[e], a.seg_off[e + 1], a.act, xs,
                              [&](int r, int row, float y) { a.y[(size_t)r * a.H + row] = y; });
    }
  }
  if (!good) set_status(a.status, kStatusNonFinite);
}

int grid_for(int items, int sm_count) { return std::max(1, std::min(items, sm_count * 8)); }

}  // namespace

template <typename K>
void ensure_smem(K kernel, size_t smem) {
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
}

cudaError_t launch_gate_up(const GemvArgs &a, cudaStream_t s) {
  const int nblk = (a.I + kGURowsPerWarp * 4 - 1) / (kGURowsPerWarp * 4);
  const int grid = grid_for(a.n_active_max * nblk, a.sm_count);
  const size_t smem = sizeof(float) * kTG * a.H;
  auto go = [&](auto kernel) {
    ensure_smem(kernel, smem);
    kernel<<<grid, kThreads, smem, s>>>(a);
  };
  const bool vec = a.H % 8 == 0 && a.vec;
  if (a.int4) {
    if (vec) go(gate_up_kernel<true, 4>);
    else go(gate_up_kernel<false, 4>);
  } else {
    if (vec) go(gate_up_kernel<true, 8>);
    else go(gate_up_kernel<false, 8>);
  }
  return cudaGetLastError();
}

cudaError_t launch_down(const GemvArgs &a, cudaStream_t s) {
  const int nblk = (a.H + kDNRowsPerWarp * 4 - 1) / (kDNRowsPerWarp * 4);
  const int grid = grid_for(a.n_active_max * nblk, a.sm_count);
  const size_t smem = sizeof(float) * kTG * a.I;
  auto go = [&](auto kernel) {
    ensure_smem(kernel, smem);
    kernel<<<grid, kThreads, smem, s>>>(a);
  };
  const bool vec = a.I % 8 == 0 && a.vec;
  if (a.int4) {
    if (vec) go(down_kernel<true, 4>);
    else go(down_kernel<false, 4>);
  } else {
    if (vec) go(down_kernel<true, 8>);
    else go(down_kernel<false, 8>);
  }
  return cudaGetLastError();
}

}  // namespace moe
