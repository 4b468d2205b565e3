/*
 * CPU oracle for the MoE-layer hot path.  TEST INFRASTRUCTURE ONLY.
 *
 * This is a plain-C restatement of the reference engine's CPU INT8 path
 * (juanhuy/DoanTotNghiepMOE, Rust crate `moe-tier-engine`).  It exists so the
 * tests, `__graft_entry__.smoke()` and the `cpu_baseline` / `--impl reference`
 * legs of `bench.py` have something to check the CUDA path against and to time
 * beside it.  Nothing in the product library links, loads or calls it.
 *
 * Parity pins (see tests/golden/make_golden.py):
 *   - the reference's hand-computed known answer (tests/int8_loader.rs:40-62),
 *   - the reference's matvec-vs-f64 and paired-vs-separate tests
 *     (src/int8_expert.rs:1149-1183, :1188-1300) re-run against this code,
 *   - top-k tie cases (src/olmoe.rs:6496-6543), learned-router KAT
 *     (src/router.rs:118-140),
 *   - the five tiny model fixtures (tests/fixtures/olmoe and tests/fixtures/qwen3moe): the
 *     reference's own Transformers logits are reproduced to < 2e-5 with this
 *     oracle standing in for every MoE block of the model.
 *
 * Floating-point order follows the reference exactly; the file is compiled
 * with -ffp-contract=off so that only the explicit fmaf()/_mm256_fmadd_ps
 * calls fuse, exactly where the reference's AVX2 intrinsics fuse.
 */
#ifndef MOE_ORACLE_H
#define MOE_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    ORACLE_OK = 0,
    ORACLE_ERR_SHAPE = 1,
    ORACLE_ERR_NONFINITE = 2,
};

/* ---- dense router dot (src/backend.rs:105-120, src/dense.rs:58-73) ---- */
float oracle_dot_f32(const float *a, const float *b, size_t n);
float oracle_dot_bf16(const uint16_t *a, const float *b, size_t n);
/* plain sequential dot used by Router::route_hidden (src/router.rs:59-62) */
float oracle_dot_seq(const float *a, const float *b, size_t n);
/* logits[e] = W[e,:].h  (Matrix::multiply_loaded_into, src/backend.rs:69-89) */
int oracle_router_logits(const void *w, int bf16, int E, int H, const float *h,
                         float *logits);

/* ---- softmax / rmsnorm (src/backend.rs:341-389) ---- */
int oracle_softmax(float *v, int n);
int oracle_rms_norm(const float *x, const float *w, int n, float eps, float *out);

/* ---- top-k over probabilities (src/olmoe.rs:2595-2621) ----
 * ids[K] in slot order (descending p, ties -> lower index), gates[K] = p/normalizer. */
void oracle_topk(const float *p, int E, int K, int norm_topk_prob, uint32_t *ids,
                 float *gates);
/* Router::select_top_k variant (src/router.rs:84-103): sort raw scores, keep
 * K, softmax over the K. */
void oracle_select_topk_then_softmax(const float *scores, int E, int K,
                                     uint32_t *ids, float *gates);

/* ---- INT8 expert (src/int8_expert.rs) ----
 * weights: [gate I*H | up I*H | down H*I] int8 row-major; scales [2I+H].
 * mode 0 = AVX2 paired path (production on x86 with AVX2+FMA),
 * mode 1 = scalar fallback (dot_i8_f32_scalar). */
float oracle_dot_i8_avx2(const int8_t *q, const float *x, size_t n);
float oracle_dot_i8_scalar(const int8_t *q, const float *x, size_t n);
float oracle_dot_i4_avx2(const uint8_t *q, const float *x, size_t n);
float oracle_dot_i4_scalar(const uint8_t *q, const float *x, size_t n);
int oracle_expert_forward_q(const int8_t *w, const float *s, int H, int I, const float *x,
                            float *act, float *y, int mode, int int4);
int oracle_expert_forward(const int8_t *w, const float *s, int H, int I,
                          const float *x, float *act, float *y, int mode);

/* ---- exact softmax exponential used by the CUDA path, restated on CPU so
 * the tests can compare it with glibc expf over the whole input range ---- */
float oracle_expf_table(float x);
uint64_t oracle_expf_table_mismatches(uint32_t bits_lo, uint32_t bits_hi,
                                      uint32_t stride);
void oracle_expf_libm_range(uint32_t bits_lo, size_t count, float *out);

/* ---- one MoE layer over T tokens ----
 * router: [E,H] f32 (bf16=0) or bf16 bits (bf16=1)
 * experts: E * (3*I*H) int8, scales: E * (2I+H) f32
 * h: [T,H] MoE input (post-norm hidden).  out: [T,H].
 * If resid != NULL out = resid + sum_slot w*y (slot order), else starts at 0.
 * ids/gates: [T,K] routing outputs (may be NULL).
 * uses_* : optional prefill permutation (src/olmoe.rs:3474-3480): experts in
 * ascending id, tokens ascending within an expert.  seg_off[E+1],
 * use_token[T*K], use_slot[T*K], use_gate[T*K].
 * nthreads: 1 = serial; >1 = the reference's production schedule with that
 * many worker threads (decode: one expert per worker, src/olmoe.rs:2928-2934;
 * prefill: row-parallel matvec per routed token, src/olmoe.rs:3615-3629). */
typedef struct oracle_layer {
    int H, I, E, K, norm_topk_prob, router_bf16;
    const void *router;
    const int8_t *experts;
    const float *scales;
    const float *norm_w; /* post-attention RMSNorm gain [H] for stacks, NULL = 1 */
    int int4;            /* experts are packed INT4 nibbles (3*H*I/2 bytes each) */
} oracle_layer;

int oracle_layer_forward(const oracle_layer *L, int T, const float *h,
                         const float *resid, float *out, uint32_t *ids,
                         float *gates, int32_t *seg_off, int32_t *use_token,
                         int32_t *use_slot, float *use_gate, int mode,
                         int nthreads);

/* Stacked decode layers: x <- x + MoE(RMSNorm(x; w=1)) per layer.
 * x: [T,H] updated in place.  ids/gates (optional): [nlayers,T,K]. */
int oracle_stack_forward(const oracle_layer *layers, int nlayers, int T,
                         float *x, float eps, uint32_t *ids, float *gates,
                         int mode, int nthreads);

/* ---- seeded synthetic inputs (shared bit-for-bit with the CUDA generator) ---- */
uint64_t oracle_synth_key(uint64_t seed, uint32_t kind, uint32_t layer,
                          uint32_t expert);
void oracle_synth_expert(uint64_t seed, int layer, int expert, int H, int I,
                         int8_t *w, float *s);
void oracle_synth_normal(uint64_t seed, uint32_t kind, uint32_t layer,
                         size_t n, float stddev, float *out);

/* ---- generators of the reference's kernel tests (src/gpu_expert.rs:517-530,
 * src/int8_expert.rs:1188-1229) ---- */
void oracle_gen_xorshift32_expert(uint32_t seed, int H, int I, int8_t *w, float *s);
void oracle_gen_xorshift64_case(uint64_t seed, int H, int I, int8_t *w, float *s,
                                float *x);

#ifdef __cplusplus
}
#endif
#endif
