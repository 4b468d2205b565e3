/*
 * moe_b200.h -- C ABI of the B200 (sm_100a) MoE-layer hot path.
 *
 * Drop-in boundary for the MoE-TierEngine reference (Rust crate
 * `moe-tier-engine`, juanhuy/DoanTotNghiepMOE).  Plain C types only: device
 * pointers are `const void *` / typed pointers into CUDA device memory, a
 * stream is an opaque `void *` holding a `cudaStream_t` (NULL = the handle's
 * own stream).  Every entry point returns a moe_status; nothing throws across
 * the boundary.  Calls on one handle are serialised by an internal mutex,
 * like the reference's `Mutex<Scratch>` (src/gpu_expert.rs:241-261).
 *
 * Numerics: routing (logits, softmax, top-k ids and gates) and the INT8
 * SwiGLU expert GEMV path reproduce the reference's CPU arithmetic bit for
 * bit (src/backend.rs:105-120, :375-389; src/olmoe.rs:2589-2621;
 * src/int8_expert.rs:380-458, :653-781, :1058-1127).
 */
#ifndef MOE_B200_H
#define MOE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum moe_status {
  MOE_OK = 0,
  MOE_ERR_INVALID = 1,   /* bad argument / shape / count; nothing was launched */
  MOE_ERR_NONFINITE = 2, /* non-finite input or output (reference `finite`, src/backend.rs:325-330) */
  MOE_ERR_CUDA = 3,      /* CUDA runtime error; see moe_last_error() */
  MOE_ERR_NCCL = 4,      /* collective failure (expert-parallel calls) */
  MOE_ERR_TIMEOUT = 5,   /* a bounded device-side wait gave up */
  MOE_ERR_STATE = 6,     /* handle not ready (e.g. layer weights not set) */
  MOE_ERR_NOMEM = 7      /* device allocation failed */
} moe_status;

/* ------------------------------------------------------------------------
 * 1. GpuExpertKernels drop-in (src/gpu_expert.rs:250-495).
 *    Same argument meaning and error behaviour as the Rust type: shape or
 *    count mismatch -> MOE_ERR_INVALID before any launch (:384-403); a
 *    non-finite output -> MOE_ERR_NONFINITE (:492-493).  Inputs and outputs
 *    are HOST buffers; expert weights are DEVICE pointers borrowed for the
 *    call (GpuExpertWeights, src/gpu.rs:1552-1566).
 * ---------------------------------------------------------------------- */
typedef struct moe_expert_kernels moe_expert_kernels;

/* GpuExpertKernels::init (src/gpu_expert.rs:268). */
moe_status moe_expert_kernels_init(int device, size_t hidden, size_t intermediate,
                                   size_t max_experts, moe_expert_kernels **out);

/* GpuExpertKernels::forward_pairs (src/gpu_expert.rs:377): pair j runs
 * d_weights[j] / d_scales[j] (3*I*H int8 [gate|up|down], 2*I+H f32) on
 * inputs[n_inputs == 1 ? 0 : j] (H floats) into outputs[j] (H floats).
 * weight_bytes / scale_bytes give each expert's sizes for validation (may be
 * NULL to skip, matching `GpuExpertWeights::{weight_bytes, scale_bytes}`). */
moe_status moe_expert_forward_pairs(moe_expert_kernels *k, const void *const *d_weights,
                                    const void *const *d_scales, const size_t *weight_bytes,
                                    const size_t *scale_bytes, size_t n_experts,
                                    const float *const *inputs, size_t n_inputs,
                                    float *const *outputs);

/* GpuExpertKernels::forward (src/gpu_expert.rs:366): every expert on one input. */
moe_status moe_expert_forward(moe_expert_kernels *k, const void *const *d_weights,
                              const void *const *d_scales, const size_t *weight_bytes,
                              const size_t *scale_bytes, size_t n_experts, const float *input,
                              float *const *outputs);

size_t moe_expert_kernels_max_experts(const moe_expert_kernels *k); /* :362 */
const char *moe_expert_kernels_last_error(const moe_expert_kernels *k);
void moe_expert_kernels_destroy(moe_expert_kernels *k); /* Drop, :497-510 */

/* ------------------------------------------------------------------------
 * 2. MoE layer on the device: router projection -> softmax -> top-k ->
 *    permutation by expert -> INT8 SwiGLU experts -> slot-ordered combine.
 *    Replaces the host loop of OlmoeModel::step_inner (src/olmoe.rs:2583-3158)
 *    and OlmoeModel::prefill (src/olmoe.rs:3417-3714) for the MoE block.
 * ---------------------------------------------------------------------- */
typedef struct moe_handle moe_handle;

typedef struct moe_dims {
  int32_t hidden;         /* H  (config hidden_size) */
  int32_t intermediate;   /* I  (intermediate_size / moe_intermediate_size) */
  int32_t num_experts;    /* E  (<= 256; the reference caps at 128, src/olmoe.rs:72) */
  int32_t top_k;          /* K  (num_experts_per_tok, <= 16) */
  int32_t norm_topk_prob; /* 0/1 (src/olmoe.rs:2614-2621) */
  int32_t max_tokens;     /* largest T per call (sizes the scratch) */
  int32_t num_layers;     /* size of the layer table */
} moe_dims;

enum {
  MOE_ROUTER_F32 = 0,  /* f32 [E,H], 8-lane dot (src/backend.rs:105-120) */
  MOE_ROUTER_BF16 = 1, /* bf16 bits [E,H] (src/dense.rs:58-73) */
};

/* Expert weight formats (src/int8_expert.rs:14-17, :107-122). */
enum {
  MOE_QUANT_INT8 = 0, /* int8 per weight: 3*I*H bytes per expert */
  MOE_QUANT_INT4 = 1  /* two signed nibbles per byte, element 2i low: 3*I*H/2 bytes */
};

/* Routing semantics. */
enum {
  MOE_ROUTE_SOFTMAX_TOPK = 0, /* OlmoeModel (default): softmax over E, top-k, optional renorm */
  MOE_ROUTE_TOPK_SOFTMAX = 1  /* Router::select_top_k (src/router.rs:84-103) */
};

/* Expert GEMM back-end for a layer call. */
enum {
  MOE_PATH_AUTO = 0,        /* the digit decode launch for T < 12 when the layers allow it
                               (INT8, 16-byte aligned rows), else the exact GEMV; tensor
                               cores from T = 12 (the measured crossover on B200) */
  MOE_PATH_GEMV = 1,        /* exact-order INT8 GEMV (bit-identical to the CPU path); for
                               small T the whole layer runs as one cooperative launch */
  MOE_PATH_TENSOR = 2,      /* tcgen05 grouped GEMM (within the 1e-3 tolerance) */
  MOE_PATH_GEMV_PHASED = 3, /* exact-order GEMV, one launch per phase (no fusion) */
  MOE_PATH_GEMV_FUSED = 4,  /* same as MOE_PATH_GEMV: the register-prefetch single launch */
  MOE_PATH_DIGITS = 5       /* decode batches (T*K <= 1024) in one cooperative launch per
                               layer or stack: routing bit-identical to the CPU path, experts
                               on two-digit int8 activations with exact int32 dot products
                               (dp4a), outputs bit-identical to MOE_PATH_TENSOR and within
                               the 1e-3 tolerance; INT8 layers with 16-byte aligned experts,
                               H and I multiples of 16 (<= 2048) */
};

moe_status moe_create(int device, const moe_dims *dims, moe_handle **out);
void moe_destroy(moe_handle *h);
const char *moe_last_error(const moe_handle *h);
/* Replay each call's launch sequence as a CUDA graph (default on).  The
 * sequence is captured once per (call, layer, token count, buffers, stream,
 * path) and replayed afterwards; captures are dropped when weights, path or
 * routing mode change.  Calls run with direct launches while profiling is on
 * and inside a caller's own stream capture. */
moe_status moe_set_graphs(moe_handle *h, int enable);
/* Default stream for calls that pass stream == NULL. */
moe_status moe_set_stream(moe_handle *h, void *cuda_stream);
moe_status moe_set_route_mode(moe_handle *h, int route_mode);
moe_status moe_set_path(moe_handle *h, int path);

/* Register one layer's weights by borrowing device pointers (the pool owns
 * them, as with GpuExpertWeights).  d_weights[e] -> 3*I*H int8
 * [gate I*H | up I*H | down H*I] (src/int8_expert.rs:90-97), d_scales[e] ->
 * 2*I+H f32 [gate | up | down]; d_router -> [E,H] in router_dtype.
 * When the experts form one packed allocation (expert e at d_weights[0] +
 * e*3*I*H), the handle builds the layer's TMA tensor maps (a 256-byte device
 * buffer per slot): the tensor-core path and the batch-1 decode weight-tile
 * ring need them.  MOE_DECODE_TILES=0 in the environment at this call keeps
 * batch-1 decode on per-thread weight loads (bit-identical results). */
moe_status moe_set_layer(moe_handle *h, int layer, const void *const *d_weights,
                         const void *const *d_scales, const void *d_router, int router_dtype);

/* Same, for experts packed back to back: expert e at d_experts + e*3*I*H and
 * d_scales + e*(2*I+H). */
moe_status moe_set_layer_packed(moe_handle *h, int layer, const int8_t *d_experts,
                                const float *d_scales, const void *d_router, int router_dtype);

/* The same two calls with the experts' weight format (MOE_QUANT_*).  INT4
 * experts (H and I even) run on the exact GEMV paths -- the per-phase
 * launches and the single-launch decode kernel -- bit-identical to the
 * reference's INT4 AVX2 path (src/int8_expert.rs:519-637, :785-952); the
 * tensor-core prefill path and the streaming kernel take INT8 layers only,
 * so an INT4 layer uses the GEMV path at every T.  A stack mixing formats
 * runs one launch per phase. */
moe_status moe_set_layer_q(moe_handle *h, int layer, const void *const *d_weights,
                           const void *const *d_scales, const void *d_router, int router_dtype,
                           int quant);
moe_status moe_set_layer_packed_q(moe_handle *h, int layer, const void *d_experts,
                                  const float *d_scales, const void *d_router, int router_dtype,
                                  int quant);

/* Routing only: ids/gates [T,K] (device).  probs (optional, device [T,E])
 * receives the post-softmax probabilities.  Needs only the layer's router,
 * so it also serves layers registered with moe_ep_set_layer. */
moe_status moe_route(moe_handle *h, int layer, const float *d_h, int T, uint32_t *d_ids,
                     float *d_gates, float *d_probs, void *stream);

/* Routing + the by-expert permutation (src/olmoe.rs:3474-3480), device
 * outputs: seg_off [E+1], route_token / route_slot [T*K]. */
moe_status moe_route_permute(moe_handle *h, int layer, const float *d_h, int T,
                             uint32_t *d_ids, float *d_gates, int32_t *d_seg_off,
                             int32_t *d_route_token, int32_t *d_route_slot, void *stream);

/* One MoE layer: d_out[t] = (d_resid ? d_resid[t] : 0) + sum over slots, in
 * slot order, of gate * expert(d_h[t]).  All pointers are device memory;
 * stream-ordered and asynchronous.  d_ids / d_gates (optional) receive the
 * routing.  Non-finite values are recorded in the handle's device status
 * word; read it with moe_sync_status(). */
moe_status moe_layer_forward(moe_handle *h, int layer, const float *d_h, const float *d_resid,
                             float *d_out, int T, uint32_t *d_ids, float *d_gates, void *stream);

/* Stacked decode: for l in [first, first+n): x <- x + MoE_l(RMSNorm_l(x; eps)), in place
 * on d_x [T,H] (src/olmoe.rs:2583-2588 then :3147-3157 per layer).  RMSNorm_l scales by
 * layer l's post-attention gain (moe_set_layer_norm), or by 1 when none is set. */
moe_status moe_stack_forward(moe_handle *h, int first_layer, int n_layers, float *d_x, int T,
                             float rms_eps, void *stream);

/* The post-attention RMSNorm gain of a layer, [H] f32 device memory (borrowed),
 * used by moe_stack_forward: h = (x * (1 / sqrt(sum x^2 / H + eps))) * w
 * (src/backend.rs:341-359).  NULL restores the unit gain. */
moe_status moe_set_layer_norm(moe_handle *h, int layer, const float *d_norm_w);

/* Host-buffer variant of moe_layer_forward (copies in and out inside the
 * call, synchronous, checks the status word like the reference's `finite`).
 * Buffers in pinned host memory are read and written by DMA directly;
 * pageable ones go through the handle's pinned staging in chunks.  Buffers
 * from moe_host_alloc() take the fastest host-to-device path.  Batches of
 * at least 2 x 1024 tokens on the tensor-core path run in token chunks (up
 * to 8; MOE_HOST_CHUNK sets the chunk, 0 turns it off): a chunk's layer
 * overlaps the next chunk's copy in and the previous chunk's copy out, and
 * the results are bit-identical to one whole-batch call. */
moe_status moe_layer_forward_host(moe_handle *h, int layer, const float *h_in,
                                  const float *h_resid, float *h_out, int T, uint32_t *h_ids,
                                  float *h_gates);

/* Pinned host memory for the host-buffer calls (cudaHostAlloc, portable
 * across devices), to be kept and reused across calls; free it with
 * moe_host_free().  Device reads of it run at the link's full rate, which
 * memory pinned after allocation (cudaHostRegister) may not reach. */
moe_status moe_host_alloc(size_t bytes, void **out);
moe_status moe_host_free(void *p);

/* Synchronise the handle's stream (or `stream`), read and clear the device
 * status word: MOE_OK, MOE_ERR_NONFINITE or MOE_ERR_TIMEOUT. */
moe_status moe_sync_status(moe_handle *h, void *stream);

/* Bound of the device-side waits of this handle's kernels: the grid barriers
 * of the single-launch decode kernels and the expert-parallel flag waits, in
 * nanoseconds at the maximum SM clock (0 restores the defaults, about 1 s and
 * 2 s).  A wait that runs out records a timeout in the handle's status word,
 * which moe_sync_status() returns as MOE_ERR_TIMEOUT; the kernel stops its
 * work and returns, so the context stays usable.  The reference's engine
 * trips its GPU circuit breaker on such an error (src/gpu.rs:534-550).  The
 * mbarrier waits inside the tensor-core kernels keep their own bound. */
moe_status moe_set_wait_limit(moe_handle *h, uint64_t ns);

/* Failure-path probe (tests): one thread waits, with the handle's flag-wait
 * bound, on a device word of the handle that nothing ever sets.  The wait
 * runs out and the handle's status word records the timeout; nothing faults
 * or traps.  Asynchronous on `stream` (NULL = the handle's stream). */
moe_status moe_debug_wait_flag(moe_handle *h, void *stream);

/* Number of kernel launches issued by the last layer/stack call. */
int moe_last_launch_count(const moe_handle *h);

/* One MoE layer that allocates no device memory.  No counterpart in the
 * reference: it is for callers that cannot allocate on the GPU -- a host
 * whose own allocator or VRAM budget owns every byte (an allocation made
 * behind its back can push its expert pool out of memory), or a
 * latency-critical decode thread on which cudaMalloc/cudaFree would block
 * or synchronise the device.  It needs no moe_handle: weights are the packed
 * device layout of moe_set_layer_packed(), d_h / d_resid / d_out are device
 * [T,H] as in moe_layer_forward(), and the results equal that call's.
 * Intermediates live in a fixed 8 MiB device array inside this library that
 * every GPU loading the library holds until the process exits; a call whose
 * T needs more returns MOE_ERR_INVALID with the reason in err_msg (optional
 * buffer).  The call runs on the device that owns `stream` (NULL = the
 * legacy default stream of the current device).  The first call on each
 * device looks the array up with that device current, so make it before any
 * stream capture; the address is kept for the process, so do not call this
 * again on a device after cudaDeviceReset() on it.  Calls share the array:
 * calls that overlap on the GPU race on it.  Shapes whose GEMV staging does
 * not fit in shared memory are rejected with MOE_ERR_INVALID.  The call
 * synchronises `stream` and returns MOE_ERR_NONFINITE like
 * moe_layer_forward_host() when an input or output is not finite. */
moe_status moe_layer_forward_noalloc(const moe_dims *dims, const int8_t *d_experts,
                                     const float *d_scales, const void *d_router,
                                     int router_dtype, const float *d_h, const float *d_resid,
                                     float *d_out, int T, void *stream, char *err_msg,
                                     size_t err_len);

/* ------------------------------------------------------------------------
 * 2b. Expert parallelism (no counterpart in the reference, which runs on one
 *     device, src/gpu.rs:457-460).  One process per GPU; experts are owned by
 *     ranks, tokens stay on the rank that routes them.  Dispatch and combine
 *     run inside moe_ep_layer_forward: by default the kernels write straight
 *     into peer memory over NVLink (CUDA IPC, handles exchanged once at
 *     moe_ep_init; no host synchronisation per layer); without peer mappings,
 *     or with MOE_EP_TRANSPORT=nccl in the environment, as NCCL
 *     point-to-point exchanges.  Routing is the single-GPU routing bit for
 *     bit, and with the default fp32 returns the outputs equal the
 *     single-GPU tensor-core path bit for bit.  MOE_EP_RETURN=i16 sends each
 *     route's output row as int16 with one scale per 32 rows instead (error
 *     <= 1/65534 of the block's largest value; within 1e-4). 
 * ---------------------------------------------------------------------- */
/* 128-byte NCCL unique id; rank 0 creates it and the host shares it. */
moe_status moe_ep_unique_id(unsigned char id_out[128]);
/* Join the expert-parallel group.  expert_owner[e] = rank that holds expert
 * e (E entries, every rank the same table).  Must precede moe_ep_set_layer. */
moe_status moe_ep_init(moe_handle *h, int rank, int nranks, const unsigned char id[128],
                       const int32_t *expert_owner);
/* This rank's experts of a layer, packed in ascending global id order
 * (3*I*H int8 and 2*I+H f32 each), plus the full [E,H] router. */
moe_status moe_ep_set_layer(moe_handle *h, int layer, const int8_t *d_experts_local,
                            const float *d_scales_local, const void *d_router, int router_dtype);
/* One MoE layer over this rank's T_local tokens (device [T_local,H]); every
 * rank must call it with the same layer, in the same order. */
moe_status moe_ep_layer_forward(moe_handle *h, int layer, const float *d_h, const float *d_resid,
                                float *d_out, int T_local, void *stream);
/* Leave the group (destroys the communicator; also done by moe_destroy). */
moe_status moe_ep_finalize(moe_handle *h);
/* Transport in use: 1 = peer memory, 0 = NCCL point-to-point, -1 = no group. */
int moe_ep_transport(const moe_handle *h);

/* ------------------------------------------------------------------------
 * 3. Utilities for tests and benchmarks (no reference counterpart).
 * ---------------------------------------------------------------------- */
/* Per-kernel device timing: when enabled, every kernel the handle launches is
 * bracketed by CUDA events on its stream.  moe_profile_read synchronises,
 * then reports, per kernel name, the launch count and total milliseconds
 * since the previous read. */
typedef struct moe_kernel_time {
  char name[32];
  int32_t launches;
  float total_ms;
} moe_kernel_time;
moe_status moe_profile_enable(moe_handle *h, int enable);
moe_status moe_profile_read(moe_handle *h, moe_kernel_time *out, int max_entries,
                            int *n_entries);

/* ---- Merged-INT8 checkpoints --------------------------------------------
 * The safetensors shards written by the reference's converter
 * (tools/prepare_olmoe.py:85-94): per expert
 * `model.layers.{l}.mlp.experts.{e}.merged_weight` I8 [3*I*H] = [gate I x H |
 * up I x H | down H x I] and `.qs` F32 [2*I + H]; the router
 * `model.layers.{l}.mlp.gate.weight` F32, BF16 or F16 [E, H].  The shard
 * index makes the header checks of the reference's TensorIndex
 * (src/safetensors.rs:90-181) and rejects a malformed shard with
 * MOE_ERR_INVALID and the reason in `err`. */
typedef struct moe_ckpt moe_ckpt;
enum { MOE_DT_U8 = 0, MOE_DT_I8 = 1, MOE_DT_F16 = 2, MOE_DT_BF16 = 3, MOE_DT_F32 = 4 };
/* Index every *.safetensors file in `dir` (headers only). */
moe_status moe_ckpt_open(const char *dir, moe_ckpt **out, char *err, size_t err_len);
void moe_ckpt_close(moe_ckpt *c);
int moe_ckpt_num_tensors(const moe_ckpt *c);
/* dtype (MOE_DT_*), rank, up to 8 dimensions, payload bytes. */
moe_status moe_ckpt_tensor_info(const moe_ckpt *c, const char *name, int *dtype, int *ndim,
                                int64_t *shape, size_t *bytes);
/* Raw little-endian payload of one tensor into host memory. */
moe_status moe_ckpt_read(const moe_ckpt *c, const char *name, void *dst, size_t dst_bytes);
/* Load checkpoint layer `ckpt_layer` into the handle's layer slot `layer`:
 * the E experts go to one packed device allocation that the handle owns
 * (freed by moe_destroy, or when the slot is set again), the router to a
 * device copy (kept BF16 when stored BF16 and keep_bf16 != 0, else f32).
 * The checks are the reference's Int8Expert::load_into
 * (src/int8_expert.rs:90-170): I8 merged_weight of exactly 3*I*H elements,
 * F32 qs of 2*I + H, scales finite and > 0; a router of [E, H] with finite
 * values.  INT4 experts (U8 [3*I*H/2], every expert of the layer) load as
 * MOE_QUANT_INT4.  A
 * `model.layers.{l}.post_attention_layernorm.weight` [H] becomes the slot's
 * RMSNorm gain (moe_set_layer_norm), likewise owned by the handle. */
moe_status moe_load_layer(moe_handle *h, const moe_ckpt *c, int ckpt_layer, int layer,
                          int keep_bf16);

/* Seeded N(0, stddev^2) values on the host (Box-Muller in double precision);
 * kind/layer select an independent stream. */
moe_status moe_synth_normal_host(uint64_t seed, uint32_t kind, uint32_t layer, size_t n,
                                 float stddev, float *out);

/* Fill an expert with the seeded synthetic generator (int8 weights
 * U[-127,127], scales U[1e-4,1e-3]); bit-identical to the CPU generator. */
moe_status moe_synth_expert(uint64_t seed, int layer, int expert, int hidden, int intermediate,
                            int8_t *d_weights, float *d_scales, void *stream);
/* Evaluate the device expf used by the softmax on `count` consecutive float
 * bit patterns starting at bits_lo (device output). */
moe_status moe_debug_expf(uint32_t bits_lo, uint32_t count, float *d_out, void *stream);

/* Read `bytes` of device memory once (16-byte loads, eight in flight per
 * thread, a few CTAs per SM): the bandwidth ceiling of a single launch over
 * a given byte count, which the benchmark times beside the decode layer.
 * d_buf 16-byte aligned, bytes a multiple of 16; d_sink is one device word
 * the kernel almost never writes.  Asynchronous on `stream`. */
moe_status moe_debug_stream_read(const void *d_buf, size_t bytes, uint32_t *d_sink,
                                 void *stream);

#ifdef __cplusplus
}
#endif
#endif /* MOE_B200_H */
