/* Internal interface between the C-ABI host layer (gdn_host.cu) and the
 * decode kernel (gdn_decode.cu). Not installed; callers use include/gdn_model.h
 * and include/gdn_b200.h.
 *
 * Device image of one model (all pointers device memory, built once per
 * GDNModel and shared by every run state):
 *   per layer l, at wimg + l * layer_stride bytes, BF16 rows [out][in] whose
 *   columns are permuted inside every 512-column group: the group stores the
 *   first 8 columns of each of its 32 sixteen-column halves, then the last 8
 *   (so lane l of a warp reads half l with two conflict-free 16-byte loads):
 *     QKVGAB  [4H + 2nh][H]   rows q | k | v | g | a_proj | b_proj
 *     O       [H][H]          at + off_o
 *     GU      [2I][H]         at + off_gu, gate row i at 2i, up row i at 2i+1
 *     DOWN    [H][I]          at + off_down
 *   LM head  [V][H] BF16 at w_lm;   embeddings [V][H] BF16 at emb.
 *   aux FP32 per layer at aux + l * aux_stride floats:
 *     attn_norm[H] | o_norm[256] | mlp_norm[H] | conv_w[3][H][4] | a_log[nh] | dt_bias[nh]
 *   final_norm[H] FP32 at aux + L * aux_stride.
 * Per decode stream (run state):
 *   S      FP32 [L][nh][256 (v)][256 (k)]  -- column v of a head's S[k][v]
 *          is 1 KB contiguous, so a CTA's share of columns is one range
 *   tails  FP32 [L][3 (q,k,v)][H][4]       -- rows 0..2 of the conv window
 *          (row 2 newest) plus one pad lane, one 16-byte vector per channel
 *   exchange buffers (qkv, gate, ab, attn, y_o, m, y_down): one word per
 *          element carrying the value and the phase's tag (epoch + phase
 *          index) -- 32 bits {BF16 value, 16-bit tag} in the BF16-boundary
 *          contracts, 64 bits {FP32 value, 32-bit tag} in the FP32 one. A
 *          phase's producer CTAs store each word once with a single store;
 *          consumer CTAs poll the words until every tag matches, so a phase
 *          boundary costs one round trip instead of a grid barrier plus a
 *          load.
 */
#ifndef GDN_ENGINE_H
#define GDN_ENGINE_H

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace gdn {

constexpr int kHeadDim = 256;
constexpr int kConsumerWarps = 8;
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr int kThreads = kConsumerThreads;
constexpr int kSlotBytes = 16384;
constexpr int kSlots = 11;
constexpr int kMaxRowsPerChunk = 4;
constexpr int kColsPerChunk = 2;
constexpr int kPhasesPerLayer = 5;
constexpr int kTraceSlots = 8;

/* error codes written to DecodeStatus.err */
enum {
    kErrNone = 0,
    kErrExchangeTimeout = 1,
    kErrChunkTimeout = 2,
    kErrSlotTimeout = 3,
    kErrAborted = 4,
    kErrBadToken = 5,
};

/* Tensor-parallel decode: GPUs per run state at most. */
constexpr int kMaxTpRanks = 8;
/* 64-bit words {payload, tag} after the exchange words of a run state's
 * exchange region: per rank, its argmax value bits and index */
constexpr int kRankCandWords = 2 * kMaxTpRanks;

/* Small device-side status block; its first 64 bytes mirror the ABI's
 * workspace[X_NORM] line (lane 0 = token id as a float). */
struct DecodeStatus {
    float token_line[16];
    int32_t token;
    int32_t err;
    uint32_t err_cta;
    uint32_t err_where;
    uint32_t done;        /* LM-head ticket counter, reset by the last CTA */
    uint32_t pad[11];
};

typedef unsigned long long xword;  /* exchange word: {fp32 bits, tag} */

struct DecodeParams {
    /* shape */
    int H, I, V, L, nh;
    float eps;
    int bf16_boundary;   /* 1: round activations to BF16 at operator boundaries */
    int native_product;  /* 1: round every GEMV product to BF16 (DAZ/FTZ), the c_impl contract */
    int bf16_state;      /* 1: round the updated recurrent state to BF16 (c_impl storage) */
    /* weights */
    const uint8_t *wimg;
    size_t layer_stride, off_o, off_gu, off_down;
    const uint8_t *w_lm;
    const uint16_t *emb;
    const float *aux;
    size_t aux_stride;
    const float *exp_table;    /* 2^(j/64), j < 64, as hi[64] | lo[64] (gdn_math.h) */
    /* stream state */
    float *S;
    float *tails;
    /* exchange buffers */
    xword *qkv, *gate, *ab, *attn, *y_o, *m, *y_down;
    /* outputs */
    float *logits, *hidden_out;
    const float *x_embed;      /* FP32 embedding row, used when token_src == nullptr */
    const int32_t *token_src;  /* device token id: gather the embedding row on device */
    float *cand_val;
    int32_t *cand_idx;
    int32_t *token_out;        /* optional: receives the step's argmax token */
    DecodeStatus *status;
    uint32_t epoch;            /* tag of phase q of this launch is epoch + q */
    /* optional phase trace, %globaltimer ns: [cta][phase][kTraceSlots], phase =
     * layer * 5 + {A..E}, L * 5 = LM head. Slots: 0 consumers done with the
     * previous phase, 1 phase inputs arrived, 2 phase input built, 3 consumer
     * chunks done (warp 0), 6 input reduction (norm sums, head scalars) done;
     * 4, 5 and 7 unused. */
    unsigned long long *trace;
    /* test hook: CTA test_drop_cta stores none of its outputs of phase
     * test_drop_phase (layer * 5 + {A, C, D, E}), so the consumers' bounded
     * waits run out; -1: off */
    int test_drop_cta, test_drop_phase;
    /* tensor-parallel decode over tp_world GPUs (1: one GPU). This GPU's
     * CTAs are the global CTAs tp_rank * gridDim.x + blockIdx.x of
     * tp_world * gridDim.x, every unit partition runs over the global CTAs,
     * and every exchange word, logit and argmax candidate a CTA stores goes
     * to its own exchange region and, for each peer r, to address + tp_delta[r]
     * (the peer's region mapped into this process, byte offset; unused for
     * r == tp_rank). rank_cand: the kRankCandWords words of this GPU's region. */
    int tp_world, tp_rank;
    long long tp_delta[kMaxTpRanks];
    unsigned long long *rank_cand;
};

/* The isolated gated-delta-rule step (gdn_recurrence.cu): `slices` (layer,
 * head) states S [256 (v)][256 (k)] FP32 updated in place from L2-normalised
 * q, k and v ([slices][256] each), decay and beta ([slices]); o [slices][256]
 * receives the unrounded outputs. status: set to 1 by a CTA whose state copy
 * did not land within its wait limit. */
struct DeltaRuleParams {
    float *S;
    const float *q, *k, *v, *decay, *beta;
    float *o;
    int *status;
    uint32_t slices;
};
size_t delta_rule_smem_bytes();
cudaError_t launch_delta_rule(const DeltaRuleParams &p, cudaStream_t stream);

/* Tags one launch consumes; the host advances DecodeParams.epoch by this. */
inline uint32_t epoch_stride(int L) { return (uint32_t)(L * kPhasesPerLayer + 1); }

size_t decode_smem_bytes(int H, int I);
cudaError_t launch_decode(const DecodeParams &p, int grid, cudaStream_t stream);
/* acc[0] += log_softmax(logits)[*target] (double), acc[1] += 1 (gdn_score.cu) */
cudaError_t launch_score(const float *logits, uint32_t V, const int32_t *target, double *acc, cudaStream_t stream);

}  // namespace gdn

#endif
