/* Internal interface between the C-ABI host layer (gdn_host.cu) and the
 * decode kernel (gdn_decode.cu). Not installed; callers use include/gdn_model.h
 * and include/gdn_b200.h.
 *
 * Device image of one model (device memory, built once per GDNModel and
 * shared by every run state). BF16 rows [out][in]; a 64-column group of a
 * row is 128 bytes = eight 16-byte pieces of 8 columns, and the pieces are
 * stored XOR-permuted so that the kernel's warps read shared memory without
 * bank conflicts. Each projection is stored column-chunk-major, so that the
 * chunk a CTA needs (a column block of all its rows) is one contiguous copy:
 *   tiled projections (QKVG with 8-row tiles and 4 groups per chunk, GU and
 *     the LM head with 16-row tiles and 2):
 *     [column chunk j][tile t][group g of the chunk][row r][piece], logical
 *     piece p of row r at position p ^ (r & 7);
 *   row-major projections (O, DOWN): [column chunk j of 16 groups (the last
 *     may have fewer)][row][group g][piece], logical piece p of group g at
 *     position p ^ (g & 7);
 *   AB: rows a_0, b_0, a_1, b_1, ... (the a/b projections of each head next to
 *     each other), natural column order.
 * Per layer l, at wimg + l * layer_stride bytes:
 *   QKVG [4H][H] (rows q | k | v | g) | AB [2 nh][H] at off_ab | O [H][H] at
 *   off_o | GU [2I][H] at off_gu (gate row i at 2i, up row i at 2i + 1) |
 *   DOWN [H][I] at off_down.
 * LM head [V][H] (16-row tiles) at w_lm; embeddings [V][H] BF16, natural, at emb.
 * aux FP32 per layer at aux + l * aux_stride floats:
 *   attn_norm[H] | o_norm[256] | mlp_norm[H] | conv_w[3][H][4] | a_log[nh] | dt_bias[nh]
 *   final_norm[H] FP32 at aux + L * aux_stride.
 * decay_tab (BF16-boundary contracts): FP32 [L][nh][65536], the reference's
 *   decay exp(-exp(a_log) * softplus(a + dt_bias)) for every BF16 bit pattern
 *   of a, evaluated with the host C library (c_impl/gdn_model.cpp:2101-2105).
 * exp_exc: sorted bit patterns of the negative floats x whose host expf(x) is
 *   not the correctly rounded exp(x) (the kernel's exp is correctly rounded and
 *   consults the list where the rounding is in doubt).
 *
 * Per decode stream (run state):
 *   S      [L][nh * 256 columns v][256 k]: FP32 (1 KB per column) or BF16
 *          (512 B, the c_impl contract's storage); 16-byte piece p of column
 *          v stored at position p ^ (v & 7)
 *   tails  FP32 [L][3 (q,k,v)][H][4]: rows 0..2 of the conv window (row 2
 *          newest) plus one pad lane, one 16-byte vector per channel
 *   exchange buffers (qkv, gate, attn, y_o, m, y_down): one word per element
 *          carrying the value and the phase's tag (epoch + phase index) --
 *          32 bits {BF16 value, 16-bit tag} in the BF16-boundary contracts,
 *          64 bits {FP32 value, 32-bit tag} in the FP32 one.
 */
#ifndef GDN_ENGINE_H
#define GDN_ENGINE_H

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace gdn {

constexpr int kHeadDim = 256;
/* 16 warps: 15 consumers and the producer (a 17th warp would put five warps
 * on one of the SM's four register-file partitions and cap every thread at
 * 96 registers) */
constexpr int kConsumerWarps = 15;
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr int kProducerWarp = kConsumerWarps;      /* the last warp issues the ring's copies */
constexpr int kThreads = kConsumerThreads + 32;
/* 4 slots in flight per SM: more queues the latency-critical exchange
 * traffic behind the weight stream (measured with 28 KB slots: 6 slots 1.26,
 * 5 1.23, 4 1.18, 3 1.23 ms/token). The one-GPU image's chunks are 28 KB;
 * 32 KB slots let a tensor-parallel CTA of four 8-row tiles take a whole
 * QKVG phase in 4 chunks. */
constexpr int kSlotBytes = 32768;
constexpr int kSlots = 4;
constexpr int kPhasesPerLayer = 5;
constexpr int kTraceSlots = 8;
constexpr int kNarrowGroups = 16;    /* 64-column groups per chunk of O / DOWN in the one-GPU image (the last may have fewer) */
constexpr int kMaxNarrowRows = kConsumerWarps;  /* O / DOWN rows per CTA: one per consumer warp */
constexpr int kMaxStateCols = kConsumerWarps;   /* state columns per CTA: one per consumer warp */
constexpr int kTileRowsQKVG = 8, kGroupsQKVG = 4;
constexpr int kTileRowsGU = 16, kGroupsGU = 2;
constexpr int kTileRowsLM = 16, kGroupsLM = 2;
constexpr uint32_t kPassTiles = 7;   /* tiles of a tiled projection per pass (one warp per 8 rows of QKVG; 28 KB chunks in the one-GPU image) */
constexpr int kMaxExcBf16 = 8;       /* BF16-valued entries of the exp exception list, copied into the parameters */

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
    int bf16_state;      /* 1: recurrent state stored and rounded as BF16 (c_impl) */
    /* weights */
    const uint8_t *wimg;
    size_t layer_stride, off_ab, off_o, off_gu, off_down;
    const uint8_t *w_lm;
    const uint16_t *emb;
    const float *aux;
    size_t aux_stride;
    const float *exp_table;    /* 2^(j/64), j < 64, as hi[64] | lo[64] (gdn_math.h) */
    const float *decay_tab;    /* [L][nh][65536] (BF16-boundary contracts) */
    const uint32_t *exp_exc;   /* sorted negative-float bit patterns, exp_exc_n of them */
    uint32_t exp_exc_n;
    uint32_t exp_exc_bf16_n;
    uint32_t exp_exc_bf16[kMaxExcBf16];
    /* BF16-rounded products: the packed BF16 multiply is the reference's
     * product when no product can fall below the normal range, i.e. every
     * nonzero input has magnitude >= fast_x_min (2^-126 over the smallest
     * nonzero weight magnitude; +inf when a weight is subnormal or not
     * finite). Phases whose input fails the test use the exact emulation. */
    float fast_x_min;
    int force_exact;           /* test hook: always use the exact emulation */
    /* chunk geometry of the weight image (wimg, w_lm): 64-column groups per
     * chunk of the QKVG, gate/up and LM-head tiles, and of the O / DOWN rows
     * (a multiple of 8) */
    uint32_t g_qkvg, g_gu, g_lm, ng_narrow;
    /* 1: a tiled GEMV pass whose tiles leave at least half of the consumer
     * warps idle spreads its groups over them (tensor-parallel launches) */
    uint32_t split;
    /* stream state */
    void *S;
    float *tails;
    /* exchange buffers */
    xword *qkv, *gate, *attn, *y_o, *m, *y_down;
    /* outputs */
    float *logits, *hidden_out;
    const float *x_embed;      /* FP32 embedding row, used when token_src == nullptr */
    const int32_t *token_src;  /* device token id: gather the embedding row on device */
    int32_t token_imm;         /* >= 0 (and token_src null): the token id itself, gathered the same way */
    float *cand_val;
    int32_t *cand_idx;
    int32_t *token_out;        /* optional: receives the step's argmax token */
    DecodeStatus *status;
    uint32_t epoch;            /* tag of phase q of this launch is epoch + q */
    /* optional phase trace, %globaltimer ns: [cta][phase][kTraceSlots], phase =
     * layer * 5 + {A..E}, L * 5 = LM head. Slots: 0 consumers done with the
     * previous phase, 1 phase inputs arrived, 2 phase input built, 3 consumer
     * chunks done, 6 input reduction (norm sums, head scalars) done; 4, 5 and
     * 7 unused. */
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

size_t decode_smem_bytes(int H, int I, bool tp);  /* tp: a tensor-parallel launch (adds the split GEMV values) */
cudaError_t launch_decode(const DecodeParams &p, int grid, cudaStream_t stream);
/* acc[0] += log_softmax(logits)[*target] (double), acc[1] += 1 (gdn_score.cu) */
cudaError_t launch_score(const float *logits, uint32_t V, const int32_t *target, double *acc, cudaStream_t stream);
/* Run-state storage <-> FP32 [L*nh][256 v][256 k] in natural order (the layout
 * of the prefill and multi-stream kernels): `cols` columns of 256 values. */
cudaError_t launch_state_to_fp32(const void *S, int bf16, float *dst, size_t cols, cudaStream_t stream);
cudaError_t launch_state_from_fp32(const float *src, void *S, int bf16, size_t cols, cudaStream_t stream);

}  // namespace gdn

#endif
