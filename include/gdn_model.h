/* gdn_model.h -- the GatedDeltaNet decode C ABI, served by libgdn_b200.so.
 *
 * This header re-declares the decode interface of the reference's
 * c_impl/gdn_model.h without Xilinx types, so a host program written against
 * that header links against the B200 engine instead of the FPGA/native model.
 * Struct layouts, the .gdnw header, the workspace float offsets
 * (GDN_WS_OFF_*) and the return conventions (0 on success, -1 with a message
 * on stderr) are identical to the reference; each declaration cites the line
 * of c_impl/gdn_model.h (and of c_impl/gdn_model.cpp for behaviour) that it
 * replaces.
 *
 * What differs behind the interface (documented per entry point below):
 *   - Weights live once per GDNModel as a BF16 image in device memory; run
 *     states share it instead of each building 32 host shards.
 *   - The recurrent state is FP32 in device memory (the FPGA keeps BF16
 *     stripes in weight shards 28..31).
 *   - GDNRunState.workspace is a pinned host mirror of the ABI workspace:
 *     X receives the embedding row, X_NORM lane 0 receives the token id after
 *     each step, LOGITS is filled on request.
 */
#ifndef GDN_MODEL_H
#define GDN_MODEL_H

#include <stddef.h>
#include <stdint.h>

/* One 512-bit beat: 32 BF16 lanes or 16 FP32 lanes, little-endian.
 * Replaces `using Beat512 = ap_uint<512>` (c_impl/gdn_model.h:10); same size. */
typedef struct GDNBeat512 {
    uint64_t words[8];
} Beat512;

/* c_impl/gdn_model.h:23-24 */
#define GEMV_CHANNELS 32
#define GEMV_CLUSTERS 16

#ifdef __cplusplus
extern "C" {
#endif

/* .gdnw header, 60 bytes (c_impl/gdn_model.h:30-45; writer
 * scripts/export_gdn_c.py:29, 177-192). */
typedef struct {
    char magic[8];
    uint32_t version;
    uint32_t vocab_size;
    uint32_t hidden_size;
    uint32_t num_layers;
    uint32_t num_heads;
    uint32_t num_v_heads;
    uint32_t head_dim;
    uint32_t intermediate_size;
    uint32_t conv_size;
    uint32_t max_seq_len;
    int32_t bos_token_id;
    int32_t eos_token_id;
    float norm_eps;
} GDNWeightHeader;

/* Workspace layout in FLOATS (c_impl/gdn_model.h:54-75). */
#define GDN_WSF_HID     2048u
#define GDN_WSF_HEAD    16u
#define GDN_WSF_MLP     5632u
#define GDN_WSF_STATE   12582912u
#define GDN_WSF_HEADBUF 442368u
#define GDN_WSF_LOGITS  32000u
#define GDN_WS_OFF_X          ((size_t)0)
#define GDN_WS_OFF_X_NORM     (GDN_WS_OFF_X         + GDN_WSF_HID)
#define GDN_WS_OFF_Q          (GDN_WS_OFF_X_NORM    + GDN_WSF_HID)
#define GDN_WS_OFF_K          (GDN_WS_OFF_Q         + GDN_WSF_HID)
#define GDN_WS_OFF_V          (GDN_WS_OFF_K         + GDN_WSF_HID)
#define GDN_WS_OFF_A          (GDN_WS_OFF_V         + GDN_WSF_HID)
#define GDN_WS_OFF_B          (GDN_WS_OFF_A         + GDN_WSF_HEAD)
#define GDN_WS_OFF_GATE       (GDN_WS_OFF_B         + GDN_WSF_HEAD)
#define GDN_WS_OFF_ATTN       (GDN_WS_OFF_GATE      + GDN_WSF_HID)
#define GDN_WS_OFF_TMP_HIDDEN (GDN_WS_OFF_ATTN      + GDN_WSF_HID)
#define GDN_WS_OFF_MLP_GATE   (GDN_WS_OFF_TMP_HIDDEN + GDN_WSF_HID)
#define GDN_WS_OFF_MLP_UP     (GDN_WS_OFF_MLP_GATE  + GDN_WSF_MLP)
#define GDN_WS_OFF_REC_STATE  (GDN_WS_OFF_MLP_UP    + GDN_WSF_MLP)
#define GDN_WS_OFF_HEAD_BUF   (GDN_WS_OFF_REC_STATE + GDN_WSF_STATE)
#define GDN_WS_OFF_LOGITS     (GDN_WS_OFF_HEAD_BUF  + GDN_WSF_HEADBUF)
#define GDN_WS_FLOATS         (GDN_WS_OFF_LOGITS    + GDN_WSF_LOGITS)

/* Per-layer weight views into GDNModel.weight_data (c_impl/gdn_model.h:123-142). */
typedef struct {
    const float *attn_norm;
    const float *a_log;
    const float *dt_bias;
    const float *q_proj;
    const float *k_proj;
    const float *v_proj;
    const float *a_proj;
    const float *b_proj;
    const float *q_conv;
    const float *k_conv;
    const float *v_conv;
    const float *g_proj;
    const float *o_norm;
    const float *o_proj;
    const float *mlp_norm;
    const float *mlp_gate_proj;
    const float *mlp_up_proj;
    const float *mlp_down_proj;
} GDNLayerWeights;

/* c_impl/gdn_model.h:144-151 */
typedef struct {
    GDNWeightHeader config;
    float *weight_data;
    GDNLayerWeights *layers;
    const float *embeddings;
    const float *final_norm;
    const float *lm_head;
} GDNModel;

/* c_impl/gdn_model.h:153-160. In this engine: `workspace` is a pinned,
 * 64-byte aligned host mirror of GDN_WS_FLOATS floats; `x`,
 * `recurrent_state` and `head_buffer` are views into it (as in the
 * reference). `weight_shards[]` and `aux_weights` are NULL: the weights live
 * in the device image shared by every run state of the model. */
typedef struct {
    Beat512 *workspace;
    float *x;
    float *recurrent_state;
    float *head_buffer;
    Beat512 *weight_shards[GEMV_CHANNELS];
    Beat512 *aux_weights;
} GDNRunState;

/* c_impl/gdn_model.h:162-168 */
typedef struct {
    uint64_t calls;
    uint64_t special_inputs;
    uint64_t flushed_inputs;
    uint64_t flushed_outputs;
    uint64_t overflows;
} GDNMixedMulStats;

/* The FPGA image layouts of the reference's run state (c_impl/gdn_model.h:
 * 84-119): the recurrent state lives as BF16 stripes past the weights of
 * shards 28..31, the conv tails as BF16 in the first half of each per
 * layer/kind stripe of the workspace head buffer. */
#define GDN_RECURRENT_STATE_PORTS       4
#define GDN_RECURRENT_STATE_FIRST_PORT 28
#define GDN_RECURRENT_STATE_STRIPE_FLOATS (GDN_WSF_STATE / GDN_RECURRENT_STATE_PORTS)
#define GDN_RECURRENT_STATE_STRIPE_BF16_BEATS (GDN_RECURRENT_STATE_STRIPE_FLOATS / 32u)
#define GDN_CONV_TAIL_STRIPES (24u * 3u)
#define GDN_CONV_TAIL_FLOATS_PER_STRIPE (GDN_WSF_HEADBUF / GDN_CONV_TAIL_STRIPES)
#define GDN_CONV_TAIL_RESERVED_BEATS_PER_STRIPE (GDN_CONV_TAIL_FLOATS_PER_STRIPE / 16u)
#define GDN_CONV_TAIL_BF16_BEATS_PER_STRIPE (GDN_CONV_TAIL_FLOATS_PER_STRIPE / 32u)

/* Host image helpers, c_impl/gdn_model.h:170-195 (behaviour
 * c_impl/gdn_model.cpp:595-1080), implemented in gdn_abi_host.cpp with the
 * reference's exact layouts. The engine does not read these images; a run
 * state has them only in reference-ABI compatibility mode
 * (gdn_b200_set_abi_compat). */
size_t gdn_weight_shard_beats(const GDNWeightHeader *config);
size_t gdn_weight_shard_bytes(const GDNWeightHeader *config);
int gdn_validate_bf16_exact_weights(const float *weight_data, const GDNWeightHeader *config);
void gdn_build_weight_shards(const float *weight_data, const GDNWeightHeader *config, Beat512 *const shards[]);
int gdn_validate_weight_shards(const float *weight_data, const GDNWeightHeader *config, Beat512 *const shards[]);
size_t gdn_aux_image_beats(const GDNWeightHeader *config);
void gdn_build_aux_image(const float *weight_data, const GDNWeightHeader *config, Beat512 *aux_image);
int gdn_validate_aux_image(const Beat512 *aux_image, const float *weight_data, const GDNWeightHeader *config);
/* Writing state through these two also marks the owning run state (if any)
 * for upload before its next decode step. */
int gdn_scatter_recurrent_state(Beat512 *const state_stripes[], const float *recurrent_state,
                                size_t recurrent_state_floats);
int gdn_pack_conv_tails_bf16(Beat512 *workspace_head_buffer, const float *conv_tails, size_t conv_tail_floats);

/* Lane helpers of the reference's tests, c_impl/gdn_model.cpp:338-366. */
uint16_t gdn_test_fp32_to_bf16_rne_bits(uint32_t bits);
uint32_t gdn_test_bf16_to_fp32_bits(uint16_t bits);
void gdn_test_set_fp32_lane_bits(Beat512 *beat, uint32_t lane, uint32_t bits);
uint32_t gdn_test_get_fp32_lane_bits(const Beat512 *beat, uint32_t lane);
void gdn_test_set_bf16_lane_bits(Beat512 *beat, uint32_t lane, uint16_t bits);
uint16_t gdn_test_get_bf16_lane_bits(const Beat512 *beat, uint32_t lane);

/* Load a .gdnw file: header validation (magic "GDNWv1", version 1,
 * num_heads == num_v_heads, hidden == heads * head_dim) and the BF16-exactness
 * check of every word while reading. Returns 0, or -1 with a message.
 * Replaces c_impl/gdn_model.h:196 (behaviour c_impl/gdn_model.cpp:1082-1229). */
int gdn_model_load(GDNModel *model, const char *path);

/* Frees the weight blob and the model's device image (if any).
 * Replaces c_impl/gdn_model.h:197 (c_impl/gdn_model.cpp:1231-1235). */
void gdn_model_free(GDNModel *model);

/* Creates a decode stream: zero recurrent and conv state on the device, the
 * pinned host workspace, and (on first use of `model`) the device weight
 * image. -1 if max_tokens == 0 or max_tokens > max_seq_len, or if the model
 * shape is not supported by the engine (head_dim must be 256).
 * Replaces c_impl/gdn_model.h:199 (c_impl/gdn_model.cpp:1247-1294). */
int gdn_run_state_init(GDNRunState *state, const GDNModel *model, uint32_t max_tokens);

/* Replaces c_impl/gdn_model.h:200 (c_impl/gdn_model.cpp:1296-1305). */
void gdn_run_state_free(GDNRunState *state);

/* One decode step: range-check the token (-1 if out of range), copy its FP32
 * embedding row into workspace[X] and on to the device, run the 24 layers and
 * the LM head on the GPU, and return with the greedy token id (maximum logit,
 * lowest index on ties) written as a float into workspace[X_NORM] lane 0.
 * Synchronous. Replaces c_impl/gdn_model.h:263 (c_impl/gdn_model.cpp:3900-3928). */
int gdn_decode_step_host(const GDNModel *model, GDNRunState *state, const int32_t *token);

/* The reference's SLR-partitioned step (c_impl/gdn_model.h:264,
 * c_impl/gdn_model.cpp:7240-7258) computes the same step; here it is
 * gdn_decode_step_host. */
int gdn_decode_step_host_partitioned(const GDNModel *model, GDNRunState *state, const int32_t *token);

/* The reference's kernel top (c_impl/gdn_model.h:224-259): one token from the
 * FP32 embedding row in workspace[X] against the run state that owns
 * `workspace`; the 32 shard pointers and the aux image name the weights the
 * engine already holds on the device. -1 if the workspace is not a run state's. */
int gdn_forward(const Beat512 *aux_weights, Beat512 *workspace, const Beat512 *weight_data_mm0,
                const Beat512 *weight_data_mm1, const Beat512 *weight_data_mm2, const Beat512 *weight_data_mm3,
                const Beat512 *weight_data_mm4, const Beat512 *weight_data_mm5, const Beat512 *weight_data_mm6,
                const Beat512 *weight_data_mm7, const Beat512 *weight_data_mm8, const Beat512 *weight_data_mm9,
                const Beat512 *weight_data_mm10, const Beat512 *weight_data_mm11, const Beat512 *weight_data_mm12,
                const Beat512 *weight_data_mm13, const Beat512 *weight_data_mm14, const Beat512 *weight_data_mm15,
                const Beat512 *weight_data_mm16, const Beat512 *weight_data_mm17, const Beat512 *weight_data_mm18,
                const Beat512 *weight_data_mm19, const Beat512 *weight_data_mm20, const Beat512 *weight_data_mm21,
                const Beat512 *weight_data_mm22, const Beat512 *weight_data_mm23, const Beat512 *weight_data_mm24,
                const Beat512 *weight_data_mm25, const Beat512 *weight_data_mm26, const Beat512 *weight_data_mm27,
                Beat512 *weight_data_mm28, Beat512 *weight_data_mm29, Beat512 *weight_data_mm30,
                Beat512 *weight_data_mm31);

/* Independent scalar LM head on the host: logits_out[v] = sum_i
 * lm_head[v][i] * bf16(hidden[i]) with the reference's BF16 product rounding.
 * Replaces c_impl/gdn_model.h:266 (c_impl/gdn_model.cpp:3930-3975). */
void gdn_compute_logits(const GDNModel *model, const float *hidden, float *logits_out);

/* BF16 x BF16 product rounded to BF16 with DAZ/FTZ (the reference's GEMV
 * product contract), widened to FP32. The operands are raw BF16 bits.
 * Replaces c_impl/gdn_model.h:210 (c_impl/gdn_model.cpp:392-466), whose
 * arguments are ap_uint<16>. */
float gdn_native_bf16_mul_to_fp32(uint16_t weight, uint16_t activation);

/* After each subsequent step, copy the final normalised hidden vector
 * (hidden_size floats) and the full FP32 logits (vocab floats) to these host
 * buffers; NULL disables. Replaces c_impl/gdn_model.h:274
 * (c_impl/gdn_model.cpp:477-485). */
void gdn_set_native_debug_buffers(float *final_hidden, float *logits);

/* The engine computes exact BF16 products, so these report zero counts; kept
 * so callers of c_impl/gdn_model.h:213-214 link. */
void gdn_reset_mixed_mul_stats(void);
GDNMixedMulStats gdn_get_mixed_mul_stats(void);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif /* GDN_MODEL_H */
