/* gdn_b200.h -- entry points of libgdn_b200.so beyond the reference's
 * c_impl/gdn_model.h. All return 0 on success and -1 on failure, with the
 * reason available from gdn_b200_last_error() (and printed to stderr, as the
 * reference's gdn_print_error does).
 */
#ifndef GDN_B200_H
#define GDN_B200_H

#include <stddef.h>
#include <stdint.h>

#include "gdn_model.h"

#ifdef __cplusplus
extern "C" {
#endif

/* CUDA device used by models and run states created afterwards on this
 * thread (default: device 0). One process per GPU is the intended layout.
 * No reference counterpart (the FPGA host selects its card through XRT,
 * c_impl/host.cpp:214-417). */
int gdn_b200_set_device(int device);

/* Message of the most recent failure on this thread ("" if none). */
const char *gdn_b200_last_error(void);

/* Fill `model` with seeded synthetic weights in the .gdnw blob order
 * (BF16-exact FP32 words; distributions in gateddeltanet_b200/csrc/gdn_synth.h)
 * instead of reading a file; afterwards the model behaves exactly as one
 * returned by gdn_model_load. Counterpart of the reference's weight writer
 * scripts/export_gdn_c.py:177-210 for a checkpoint that does not exist here. */
int gdn_b200_model_synth(GDNModel *model, const GDNWeightHeader *config, uint64_t seed);

/* Write `model` as a .gdnw file (60-byte header + FP32 words), the format
 * gdn_model_load reads (scripts/export_gdn_c.py:177-210). */
int gdn_b200_model_save(const GDNModel *model, const char *path);

/* Numeric contract of a stream. Three are supported:
 *   (1, 1, 1)  the default: the reference's own arithmetic (c_impl): every
 *              activation rounded to BF16 where the reference rounds it, each
 *              GEMV product rounded to BF16 with DAZ/FTZ before the sum
 *              (c_impl/gdn_model.cpp:392-466), the recurrent state stored in
 *              BF16 after each update (2268-2300), transcendental functions
 *              rounded as the host C library rounds them. Reproduces
 *              gdn_decode_step_host of the reference bit for bit.
 *   (1, 0, 0)  BF16 boundaries, exact products, FP32 state (the PyTorch/GPU
 *              arithmetic of the reference's training stack).
 *   (0, 0, 0)  the FP32 control of the parity gates: FP32 boundaries, exact
 *              products, FP32 state.
 * GEMV sums always follow the reference's reduction order. Other
 * combinations return -1. Switching between BF16 and FP32 state converts the
 * stream's state (FP32 -> BF16 rounds to nearest even). */
int gdn_b200_set_numerics(GDNRunState *state, int bf16_boundary, int bf16_products, int bf16_state);

/* Replace / read the decode state in the .gdnstate section layouts:
 * rec [layers][heads][K=256][V=256] FP32 and conv tails
 * [layers][q,k,v][conv_size-1][hidden] FP32, last row newest
 * (scripts/export_gdn_state.py:13-19, 340-362; c_impl/gdn_eval.cpp:202-267). */
int gdn_b200_state_upload(GDNRunState *state, const float *rec, size_t rec_floats, const float *conv,
                          size_t conv_floats);
int gdn_b200_state_download(GDNRunState *state, float *rec, size_t rec_floats, float *conv, size_t conv_floats);

/* .gdnstate files ("GDNSTAT1", c_impl/gdn_eval.cpp:202-267 and
 * c_impl/host.cpp:675-735: dims must match the model, no trailing bytes). */
int gdn_b200_state_load_file(GDNRunState *state, const char *path, int32_t *seed_token);
int gdn_b200_state_save_file(GDNRunState *state, const char *path, int32_t seed_token);

/* FP32 logits (vocab floats) and final normalised hidden vector (hidden
 * floats) of the most recent step; either pointer may be NULL. */
int gdn_b200_fetch_outputs(GDNRunState *state, float *logits, float *final_hidden);

/* Decode n tokens back to back without returning to the host between
 * steps. greedy = 0: teacher-forced, step i consumes tokens[i]; greedy = 1:
 * step 0 consumes tokens[0] and step i > 0 consumes step i-1's argmax
 * (the loop of c_impl/gdn_eval.cpp:336-440). argmax_out[i] receives step
 * i's token. If kernel_ms is not NULL it receives the device time of the n
 * steps (CUDA events on the stream). Embedding rows are gathered on the
 * device; the token ids cross PCIe once. */
int gdn_b200_decode_tokens(const GDNModel *model, GDNRunState *state, const int32_t *tokens, uint32_t n,
                           int greedy, int32_t *argmax_out, float *kernel_ms);

/* gdn_b200_decode_tokens without any device memory allocation: same
 * arguments, same results. No counterpart in the reference.
 *
 * For callers that must not allocate device memory while they decode -- a
 * server that has handed the rest of HBM to its own pool, or a loop that
 * cannot afford cudaMalloc/cudaFree synchronising the device. (The plain
 * gdn_b200_decode_tokens grows a per-run-state device buffer with cudaMalloc
 * whenever a call is longer than any before it.) The token ids and per-step
 * argmax live instead in a fixed 32 KB array in the library's device memory,
 * one per device.
 *
 * Limits: at most 4096 tokens per call (longer calls fail with an error
 * naming the limit; split the sequence). The first call on a device looks up
 * the array's address (cudaGetSymbolAddress); make that first call before
 * any stream capture begins on that device. All run states of a device share
 * the array, so calls that overlap in time on one device -- from several
 * threads, or on run states whose streams run concurrently -- race on it and
 * may read each other's tokens: issue them one at a time per device. */
int gdn_b200_decode_tokens_noalloc(const GDNModel *model, GDNRunState *state, const int32_t *tokens, uint32_t n,
                                   int greedy, int32_t *argmax_out, float *kernel_ms);

/* One decode step of `token` with the kernel's phase trace enabled: for every
 * CTA and phase (layer * 5 + {QKVG, state, O, gate/up, down}, then the LM
 * head) eight %globaltimer stamps in ns -- [0] consumers done with the
 * previous phase, [1] phase inputs arrived, [2] phase input built, [3] the
 * phase's chunks done, [6] input reductions done; [4], [5], [7] unused. Layout [cta][phase][8]; returns the
 * number of (cta, phase) records or -1. The B200 counterpart of the
 * reference's GDN_CALL_PROBE cycle stamps (c_impl/gdn_model.cpp:18-127). */
int gdn_b200_trace_step(const GDNModel *model, GDNRunState *state, int32_t token, uint64_t *trace_out,
                        size_t capacity);

/* The gated delta rule alone (BASELINE config[1] microbench): `slices`
 * (layer, head) recurrent states S [slices][256 (v)][256 (k)] FP32 (the
 * engine's layout: column v of the reference's S[k][v] is contiguous) are
 * advanced `steps` times in place from
 * L2-normalised q and k, v ([slices][256] each), decay and beta ([slices]),
 * as c_impl/gdn_model.cpp:2119-2300 does for one head: alpha = tree256(q.k),
 * r and p by sequential sums over k, delta = beta (v - decay r),
 * o = (decay p + alpha delta) / 16, S' = decay S + k delta^T (no rounding of
 * S). o receives the last step's FP32 outputs. All buffers are host memory;
 * the call uploads them, runs the steps (L2 flushed before each, so every
 * step streams S from HBM) and downloads S and o. ms_per_step, if not NULL,
 * receives the mean device time of one step (CUDA events around each kernel
 * only). */
int gdn_b200_delta_rule_step(uint32_t slices, float *S, const float *q, const float *k, const float *v,
                             const float *decay, const float *beta, float *o, uint32_t steps, float *ms_per_step);

/* Test hook for the failure path (no counterpart in the reference): until
 * called again with cta = -1, every decode step of `state` has CTA `cta`
 * leave out its outputs of phase `phase` (layer * 5 + 0 for QKVG, + 2 for O,
 * + 3 for gate/up, + 4 for down). The CTAs waiting for them give up after
 * their wait limit (2 s), the step returns -1 with the kernel's error, and
 * the run state stays usable (its recurrent state is then partly updated:
 * reload it). Nothing faults or hangs on the GPU. */
int gdn_b200_test_drop_outputs(GDNRunState *state, int cta, int phase);

/* Test hook (no counterpart in the reference): with on != 0 every GEMV of
 * `state` in the c_impl contract uses the exact emulation of the reference's
 * BF16 product (special values, DAZ, FTZ) instead of the packed BF16
 * multiply, which the kernel otherwise uses whenever no product of a phase
 * can fall below the normal range. Results are identical either way. */
int gdn_b200_test_force_exact_products(GDNRunState *state, int on);

/* Test hook (no counterpart in the reference): the exchange tag base of the
 * next launch of `state` (the host advances it by 5 L + 1 per launch; in the
 * BF16-boundary contracts only its low 16 bits reach the exchange words).
 * Lets a test start launches whose tags wrap past 0xffff, the tag of a word
 * that was never written since the exchange buffers were last refilled. */
int gdn_b200_test_set_epoch(GDNRunState *state, uint32_t epoch);

/* Test hook (no counterpart in the reference; host only, no GPU needed): the
 * chunk geometry gdn_b200_tp_attach gives the weight image of a model of
 * these sizes for `ncta` CTAs over all GPUs -- geom[0..3] = 64-column groups
 * per chunk of the QKVG, gate/up and LM-head tiles and of the O / DOWN rows
 * (4, 2, 2, 16 is the one-GPU image). With check_maps != 0 it also checks,
 * for that geometry and the one-GPU one, that the image layout maps and
 * their inverses are bijections onto every projection (the device re-layout
 * gathers through them). 0, or -1 with gdn_last_error(). */
int gdn_b200_test_image_geometry(uint32_t hidden, uint32_t intermediate, uint32_t vocab, uint32_t ncta,
                                 uint32_t *geom, int check_maps);

/* Reference-ABI compatibility for the run states created afterwards (also
 * GDN_B200_ABI_COMPAT=1 in the environment): gdn_run_state_init then builds
 * the reference's host images (32 packed shards with the BF16 state stripes,
 * the aux image; about 2.8 GB of host memory per run state) and selects the
 * c_impl arithmetic; state written through gdn_scatter_recurrent_state /
 * gdn_pack_conv_tails_bf16 is uploaded before the next step, and after every
 * step the device state is written back to the stripes and the head buffer,
 * so an unmodified reference driver (c_impl/gdn_eval.cpp) runs on this
 * library. Off by default. */
int gdn_b200_set_abi_compat(int on);

/* Number of SMs (CTAs) the decode kernel uses on the current device. */
int gdn_b200_grid_size(void);

/* ------------------------------------------- tensor-parallel decode
 * One decode stream over 2..8 GPUs, one run state per
 * GPU, each in its own process. Replaces the head/column split with an
 * allreduce of c_impl/gdn_model.cpp's GEMV calls by a row split: every output
 * row (and state column) is computed whole on one GPU and stored into every
 * GPU's exchange region over NVLink, so the step is the single-GPU step and
 * its results are identical bit for bit. The recurrent state and conv tails
 * are then split by owner: each rank updates only the columns and channels
 * its CTAs own (logits and tokens are complete on every rank).
 *   1. every rank: gdn_b200_tp_token(state, token) -> share the
 *      GDN_B200_TP_TOKEN_BYTES token with the others (all-gather);
 *   2. every rank: gdn_b200_tp_attach(state, rank, world, tokens) with the
 *      tokens in rank order, then a barrier before the first step;
 *   3. every rank makes the same decode calls with the same tokens, in step.
 * Ranks must sit on distinct devices with the same SM count. A rank that does
 * not take part lets the others' waits run out (2 s): the step returns -1;
 * attaching every rank again (step 2) and reloading the state recovers.
 * After the first tensor-parallel step a run state holds one rank's part of
 * the state until a full state is uploaded (gdn_b200_state_upload): while it
 * does, gdn_b200_state_download, gdn_b200_state_save_file, gdn_b200_prefill
 * and (after gdn_b200_tp_detach) single-GPU decode return -1. The parts come
 * out through gdn_b200_tp_state_download_part; the Python layer's
 * tensor_parallel.merge_state joins them into the full state.
 * The first attach of a model for a given world * grid allocates, on this
 * GPU, a copy of the weight image in that grid's chunk geometry (about the
 * size of the weights; kept with the model, reused, freed with it); -1 if
 * that allocation fails. */
#define GDN_B200_TP_TOKEN_BYTES 128
int gdn_b200_tp_token(GDNRunState *state, void *token);
int gdn_b200_tp_attach(GDNRunState *state, int rank, int world, const void *tokens);
/* back to single-GPU decode (the state stays partial: see above) */
int gdn_b200_tp_detach(GDNRunState *state);
/* This rank's part of a tensor-parallel state in the gdn_b200_state_download
 * layout (the columns and conv channels other ranks own hold stale values),
 * with the attachment it came from: *tp_grid CTAs per GPU, *tp_rank of
 * *tp_world GPUs (unit u of a phase with `total` units belongs to global CTA
 * c when c * total / (world * grid) <= u < (c + 1) * total / (world * grid),
 * and global CTA c to rank c / grid). -1 if the run state never took a
 * tensor-parallel step since its last full upload. */
int gdn_b200_tp_state_download_part(GDNRunState *state, float *rec, size_t rec_floats, float *conv,
                                    size_t conv_floats, int32_t *tp_grid, int32_t *tp_rank, int32_t *tp_world);

/* ---------------------------------------------------- multi-stream decode
 * Several independent decode streams on one GPU (no
 * counterpart in the reference, whose decode ABI is one stream per call):
 * every step advances each stream by one token and reads each weight byte
 * once for all of them. The projections run on the tensor cores (tcgen05)
 * with FP32 accumulation, so the batch follows the FP32-boundary contract
 * (FP32 activations and state, BF16 weights; every product exact, only the
 * summation order differs from c_impl/gdn_model.cpp's bank chains). Streams
 * start from zero state. The weight image (a tensor-core tile layout, 2.8 GB
 * for GDN-1.3B) is built once per model and device and shared by batches.
 * Functions return 0 / -1 (gdn_b200_last_error) unless stated. */
typedef struct GdnB200Batch GdnB200Batch;

/* NULL on error. streams: 1 .. 1024 (processed in passes of 80). */
GdnB200Batch *gdn_b200_batch_create(const GDNModel *model, uint32_t streams);
void gdn_b200_batch_free(GdnB200Batch *batch);
/* Kernel launches in one step (the step is one CUDA graph replay). */
uint32_t gdn_b200_batch_launches_per_step(const GdnB200Batch *batch);
/* Zero every stream's recurrent state and conv tails. */
int gdn_b200_batch_reset(GdnB200Batch *batch);
/* One stream's state in the host layouts of gdn_b200_state_upload:
 * rec [L][heads][K][V], conv tails [L][q,k,v][W-1][hidden]. */
int gdn_b200_batch_state_upload(GdnB200Batch *batch, uint32_t stream, const float *rec, size_t rec_floats,
                                const float *conv, size_t conv_floats);
int gdn_b200_batch_state_download(GdnB200Batch *batch, uint32_t stream, float *rec, size_t rec_floats, float *conv,
                                  size_t conv_floats);
/* One step from host memory: tokens[streams] in; argmax[streams] and, if not
 * NULL, logits[streams][vocab] (FP32) out. */
int gdn_b200_batch_step_host(GdnB200Batch *batch, const int32_t *tokens, int32_t *argmax, float *logits);
/* n steps with the token ids on the device: tokens[n][streams] (teacher
 * forced), or with greedy != 0 only tokens[0][streams] and then each
 * stream's own argmax. argmax_out[n][streams] may be NULL; device_ms, if not
 * NULL, receives the device time of the steps (CUDA events around the graph
 * replays). */
int gdn_b200_batch_decode_tokens(GdnB200Batch *batch, const int32_t *tokens, uint32_t n, int greedy,
                                 int32_t *argmax_out, float *device_ms);
/* Logits [streams][vocab] of the last step. */
int gdn_b200_batch_fetch_logits(GdnB200Batch *batch, float *logits);
/* Prefill: advance a run state by n prompt tokens at once (no logits), e.g.
 * the prompt before decoding starts. The projections run as tensor-core GEMMs
 * over up to 240 tokens at a time; the short convolution and the recurrence
 * run in token order on the run state's own state. FP32 arithmetic: the state
 * matches token-by-token decoding in the FP32-boundary contract within
 * summation-order differences. device_ms, if not NULL, receives the device
 * time. The counterpart of the reference's GPU prompt prefill
 * (scripts/export_gdn_state.py:157-201), which feeds its .gdnstate export. */
int gdn_b200_prefill(const GDNModel *model, GDNRunState *state, const int32_t *tokens, uint32_t n, float *device_ms);

/* Teacher-forced scoring of one window, c_impl/host.cpp:1954-1994
 * (score_window_hw): resets the run state to zero, feeds tokens = ctx ++ cont
 * in order except the last, and sums over every fed token i >= ctx_len - 1
 * the log-probability of tokens[i + 1] under that step's FP32 logits
 * (max-shifted log-softmax in double). logprob receives the sum, scored (if
 * not NULL) the number of scored tokens (cont_len). -1 if ctx_len or cont_len
 * is 0 or a token is out of range. use_prefill != 0 feeds the first
 * ctx_len - 1 tokens through gdn_b200_prefill (FP32) instead of decode steps. */
int gdn_b200_score_window(const GDNModel *model, GDNRunState *state, const int32_t *ctx, uint32_t ctx_len,
                          const int32_t *cont, uint32_t cont_len, int use_prefill, double *logprob, uint64_t *scored);

/* Test hook: y[n][m] = sum_k w[m][k] x[n][k] through one tensor-core tile-GEMM
 * launch (w BF16-exact FP32 words, x FP32 entering as three BF16 terms;
 * k a multiple of 64, n <= 80). */
int gdn_b200_test_tile_gemm(uint32_t m, uint32_t k, uint32_t n, const float *w, const float *x, float *y);

#ifdef __cplusplus
}
#endif

#endif
