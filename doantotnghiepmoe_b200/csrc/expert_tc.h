// Launch interface of the tcgen05 grouped expert GEMM (expert_tc.cu).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>

namespace moe {
namespace tc {

int persistent_mode();  // MOE_TC_PERSISTENT: 0 off, 1 both GEMMs (default), 2 down, 3 gate/up
int tc_bn_override();  // MOE_TC_BN (64 or 128), 0 when unset

// Routes per GEMM tile: 64, which the persistent kernels require.  With one
// CTA per tile (MOE_TC_PERSISTENT=0), 64-route tiles with two CTAs per SM
// also beat 128-route tiles on B200 (OLMoE T=512, Qwen3 T=4096): two
// pipelines per SM overlap one CTA's epilogue with the other's mainloop.
// MOE_TC_BN=128 selects the wide tile there.
inline int tc_block_n(int routes, int experts) {
  (void)routes;
  (void)experts;
  if (persistent_mode() == 1 || persistent_mode() == 3) return 64;
  if (const int o = tc_bn_override()) return o;
  return 64;
}

int tc_bn_dn_override();  // MOE_TC_BN_DN (64 or 128), 0 when unset

// Routes per down-GEMM tile.  The down GEMM has a short K (= I), so its
// CTAs are short-lived and per-CTA overheads weigh; 128-route tiles halve
// the CTA count once experts average 128 routes or more.  Measured on B200:
// Qwen3 T=4096 (256 routes per expert) 877 vs 921 us per layer, OLMoE T=512
// (64 per expert) a tie.  MOE_TC_BN_DN (64 or 128) pins the width.
inline int tc_block_n_down(int routes, int experts) {
  if (persistent_mode() == 1 || persistent_mode() == 2) return 64;
  if (const int o = tc_bn_dn_override()) return o;
  if (tc_bn_override()) return tc_bn_override();
  return routes >= 128 * experts ? 128 : 64;
}

struct TcArgs {
  int H, I, K;
  const int32_t *tile_expert;  // [max_tiles] expert of each route tile
  const int32_t *tile_row0;    // [max_tiles] first permuted route of the tile
  const int32_t *tile_rows;    // [max_tiles] routes in the tile (<= the tile width)
  const int32_t *n_tiles;      // device count of valid tiles
  const float *const *s_ptr;   // per-expert scales [gate I | up I | down H]
  const float *xs1, *xs2;      // per-route digit scales of the inputs
  float *act;                  // [R, I] fp32 activations
  uint32_t *act_amax;          // [R] max|act| bits, accumulated by GEMM 1
  const float *as1, *as2;      // per-route digit scales of the activations
  const int32_t *r_token, *r_slot;
  const float *r_gate;
  float *contrib;              // [T, K, H]
  // expert parallelism over peer memory: when r_rank is set, route r's row
  // goes to the source rank r_rank[r] as int16 values peer_c16[rank] [T, K, H]
  // with one scale per (route, 32-row block) in peer_cscale[rank]
  // [T, K, ceil(H / 32)]: value = q * scale (see ep_store16)
  // (ret16), or as fp32 rows peer_c32[rank] [T, K, H] (ret16 == 0)
  const int32_t *r_rank;
  int ret16;
  int16_t *peer_c16[8];
  float *peer_cscale[8];
  float *peer_c32[8];
  uint32_t *status;
};

// 3D uint8 tiled map with a 128 x 128 box and 128-byte swizzle.
bool encode_map3d(CUtensorMap *map, const void *base, uint64_t d0, uint64_t d1, uint64_t d2,
                  uint64_t stride1, uint64_t stride2, uint32_t box_rows);

cudaError_t launch_build_tiles(const int32_t *seg_off, const int32_t *active,
                               const int32_t *n_active, int bn, int32_t *tile_expert,
                               int32_t *tile_row0, int32_t *tile_rows, int32_t *n_tiles,
                               int max_tiles, cudaStream_t s);

// T token rows, each quantized once and stored at its K routes' sorted rows
// r_pos[t * K + k] (rows outside [0, T * K) are skipped).
cudaError_t launch_quantize_tokens(const float *x, const int32_t *r_pos, int T, int K, int n,
                                   int8_t *q, size_t plane, float *s1, float *s2,
                                   uint32_t *amax_reset, cudaStream_t s);

// R rows (grid size); when R_dev is given, rows at or past *R_dev are skipped.
cudaError_t launch_quantize_rows(const float *src, const int32_t *rows, const uint32_t *amax_in,
                                 int R, int n, int8_t *q, size_t plane, float *s1, float *s2,
                                 uint32_t *amax_reset, cudaStream_t s,
                                 const int32_t *R_dev = nullptr);

cudaError_t launch_gate_up_tc(const CUtensorMap &mapW, const CUtensorMap &mapX, const TcArgs &a,
                              int bn, int max_tiles, cudaStream_t s);
cudaError_t launch_down_tc(const CUtensorMap &mapW, const CUtensorMap &mapA, const TcArgs &a,
                           int bn, int max_tiles, cudaStream_t s);

}  // namespace tc
}  // namespace moe
