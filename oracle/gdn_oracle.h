/* gdn_oracle.h -- CPU restatement of the reference GatedDeltaNet decode step.
 *
 * TEST INFRASTRUCTURE ONLY. This is the checker the engine is compared
 * against; nothing in the shipped package links, loads or calls it. Only the
 * tests, __graft_entry__.smoke() and bench.py's CPU-baseline leg may use it.
 *
 * It restates c_impl/gdn_model.cpp's native decode arithmetic (gdn_forward,
 * c_impl/gdn_model.cpp:3532-3897) operation by operation, in the reference's
 * association order and without FMA contraction, so that in the reference
 * mode {native products, BF16 state, BF16 boundaries} it reproduces the
 * reference bit for bit. Parity pin: tests/golden holds digests of the
 * reference's own outputs (c_impl/gdn_model.cpp compiled natively through
 * oracle/hls_shim by oracle/Makefile) for seeded 1.3B weights and token
 * streams; tests/test_oracle_golden.py checks this file against them.
 *
 * Modes:
 *   native_product  1: every GEMV product rounded to BF16 with DAZ/FTZ
 *                      (c_impl/gdn_model.cpp:392-466); 0: exact products.
 *   bf16_state      1: recurrent state stored as BF16 (gdn_model.cpp:2268-2300);
 *                   0: FP32 state (the engine's layout).
 *   bf16_boundary   1: activations rounded to BF16 at every operator boundary
 *                      (the reference's all-BF16 transient contract);
 *                   0: FP32 boundaries (the "fp32 control").
 */
#ifndef GDN_ORACLE_H
#define GDN_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct {
    uint32_t vocab, hidden, layers, heads, head_dim, inter, conv;
    float eps;
} GdnOracleDims;

typedef struct {
    int native_product;
    int bf16_state;
    int bf16_boundary;
} GdnOracleMode;

/* Sizes in floats. */
size_t gdn_oracle_weight_floats(const GdnOracleDims *d);
size_t gdn_oracle_rec_floats(const GdnOracleDims *d);   /* [L][H][K][V] */
size_t gdn_oracle_conv_floats(const GdnOracleDims *d);  /* [L][q,k,v][W-1][hidden] */

/* Fill a weight blob (the .gdnw payload order) from the seeded generator
 * of gateddeltanet_b200/csrc/gdn_synth.h, using `threads` threads. */
void gdn_oracle_synth_weights(const GdnOracleDims *d, uint64_t seed, float *blob, int threads);

/* Seeded uniform token id i of stream `stream` (gdn_synth.h). */
int32_t gdn_oracle_synth_token(uint64_t seed, uint32_t stream, uint64_t i, uint32_t vocab);

/* Seeded BF16-exact initial state: rec ~ N(0, 0.05), conv tails ~ N(0, 0.5);
 * state_seed 0 gives zeros. */
void gdn_oracle_synth_state(const GdnOracleDims *d, uint64_t state_seed, float *rec, float *conv);

/* One decode step. rec/conv are updated in place. Any of logits /
 * final_hidden / argmax may be NULL. Returns 0, or -1 on bad arguments. */
int gdn_oracle_step(const GdnOracleDims *d, const float *blob, GdnOracleMode mode,
                    float *rec, float *conv, int32_t token,
                    float *logits, float *final_hidden, int32_t *argmax, int threads);

/* Primitive hooks for known-answer tests. */
uint16_t gdn_oracle_bf16_rne_bits(uint32_t fp32_bits);
uint32_t gdn_oracle_native_product_bits(uint16_t weight, uint16_t activation);
float gdn_oracle_row_dot(const float *w_row, const float *x, uint32_t k, int native_product);

/* Batch forms for the known-answer tests: out[i] = RNE bits of in[i];
 * out[j * n_w + i] = product bits of (w[i], a[j]). */
void gdn_oracle_bf16_rne_batch(const uint32_t *in, size_t n, uint16_t *out);
void gdn_oracle_native_product_grid(const uint16_t *w, size_t n_w, const uint16_t *a, size_t n_a, uint32_t *out);

/* gdn_compute_logits (c_impl/gdn_model.cpp:3930-3975): logits[v] =
 * sequential sum over i of the BF16-rounded product of lm_head[v][i] and
 * RNE(hidden[i]). blob is the .gdnw payload. */
void gdn_oracle_compute_logits(const GdnOracleDims *d, const float *blob, const float *hidden, float *logits,
                               int threads);

/* The gated delta rule for one head from the read pass on
 * (c_impl/gdn_model.cpp:2119-2300): S [K][V] updated in place from already
 * L2-normalised q/k, the decay and beta; o [V] receives the unrounded output. */
void gdn_oracle_delta_rule_head(float *S, const float *qn, const float *kn, const float *v,
                                float decay, float beta, int bf16_state, float *o);

#ifdef __cplusplus
}
#endif

#endif
