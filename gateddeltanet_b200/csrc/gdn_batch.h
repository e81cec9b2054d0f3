/* Internal interface of the multi-stream decode engine (several independent
 * decode streams per GPU): gdn_batch.cu (kernels) and
 * gdn_batch_host.cu (C ABI). Not installed; callers use include/gdn_b200.h.
 *
 * Numeric contract: the reference's decode step with FP32 operator boundaries
 * and FP32 recurrent state (the "FP32 control" of the single-stream engine),
 * BF16 weights. The projections run on the tensor cores (tcgen05, FP32
 * accumulation in TMEM); an FP32 activation v enters them as three BF16 terms
 * h0 + h1 + h2 = v (h0 = bf16(v), h1 = bf16(v - h0), h2 = v - h0 - h1, all
 * exact), so every product is exact and only the accumulation order differs
 * from the reference's bank chains.
 *
 * Device layouts:
 *   tile image of a weight matrix [M][K] (BF16): blocks of 128 rows x 64
 *     columns, 16 KB each, in [m-tile][k-block] order, so k-block u of the
 *     flattened (tile, k-block) sequence is the u-th 16 KB block. Inside a
 *     block row r occupies bytes r*128 .. r*128+127 and its 16-byte chunk c
 *     (columns 8c .. 8c+7) sits at chunk position c ^ (r & 7): the K-major
 *     128-byte-swizzle layout the tensor core's shared-memory descriptor
 *     reads, so one bulk copy lands a block ready for tcgen05.mma. Rows past M
 *     are zero.
 *   activation tiles of a [N][K] operand (N = streams padded to 16): per
 *     64-column block kb, three terms, each N rows x 128 bytes in the same
 *     swizzle: element (n, k) of term t at
 *       kb * 3*N*128 + t * N*128 + n*128 + ((((k & 63) >> 3) ^ (n & 7)) << 4) + (k & 7)*2.
 *   per stream s: S FP32 [L][nh][v][k] (column v of a head's S[k][v] is 1 KB
 *     contiguous); conv tails FP32 [L][q,k,v][3][H] (row 2 newest, the
 *     reference's order); residual x FP32 [H]; the QKVGAB output FP32
 *     [4H + 2nh] (q, k, v after the short convolution and SiLU; g, a, b raw).
 */
#ifndef GDN_BATCH_H
#define GDN_BATCH_H

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace gdn {
namespace bt {

constexpr int kTileM = 128;
constexpr int kTileK = 64;
constexpr int kTerms = 3;
constexpr int kABlockBytes = kTileM * kTileK * 2;
constexpr int kMaxPassStreams = 128;  /* streams per GEMM pass (TMEM: 2 x 128 columns) */
constexpr int kGemmThreads = 224;     /* warps 0-3 epilogue, 4 A copies, 5 B copies, 6 MMA */

enum Epilogue : int {
    kEpiStore = 0,   /* out[n * out_stride + row] = y */
    kEpiQKV = 1,     /* rows < 3H: causal conv + SiLU with tail update; others stored raw */
    kEpiResid = 2,   /* resid[n * out_stride + row] += y */
    kEpiSwiGLU = 3,  /* rows (2i, 2i+1) = (gate_i, up_i): m_i = silu(g) * u as activation tiles */
    kEpiLogits = 4,  /* out[n * out_stride + row] = y, and the per-stream argmax key */
};

enum Error : uint32_t {
    kErrNone = 0,
    kErrWaitA = 1,
    kErrWaitB = 2,
    kErrWaitMma = 3,
    kErrWaitAcc = 4,
    kErrWaitDrain = 5,
    kErrBadToken = 6,
};

struct GemmParams {
    const uint8_t *a;      /* tile image, [m-tile][k-block] 16 KB blocks */
    const uint8_t *b;      /* activation tiles of this pass */
    uint32_t m;            /* valid rows */
    uint32_t kblocks;      /* K / 64 */
    uint32_t mtiles;       /* ceil(M / 128) */
    uint32_t npad;         /* streams of this pass, padded to a multiple of 16 */
    uint32_t nvalid;       /* streams of this pass */
    uint32_t stream0;      /* first stream of this pass (argmax keys, tails) */
    uint32_t a_slots, b_slots;
    float *partial;        /* [grid][max_local][npad][128] */
    uint32_t max_local;    /* partial slots per CTA */
    uint32_t *counters;    /* per m-tile arrival counters, zero between launches */
    int epi;
    float *out;            /* Store / Logits / Resid: [n][out_stride] (pass-relative n) */
    uint32_t out_stride;
    /* QKV: conv weights FP32 [3][H][4] of the layer; tails of stream 0 of the
     * pass at tails, stream stride tails_stride floats, layout [3][3][H] */
    const float *conv_w;
    float *tails;
    size_t tails_stride;
    uint32_t hidden;
    /* SwiGLU: activation tiles of the next GEMM (K = M / 2) */
    uint8_t *next_b;
    /* Logits: argmax keys, one per stream (absolute stream index) */
    unsigned long long *keys;
    uint32_t *status;      /* [0] error code, [1] where */
};

/* smem bytes of the GEMM for a pass of npad streams with the given slots */
size_t gemm_smem_bytes(uint32_t npad, uint32_t a_slots, uint32_t b_slots);
/* choose ring depths for npad streams within the shared-memory limit */
void gemm_slots(uint32_t npad, uint32_t *a_slots, uint32_t *b_slots);
/* CTAs of one launch: min(SM count, m-tiles x k-blocks) */
uint32_t gemm_grid(uint32_t mtiles, uint32_t kblocks, uint32_t sms);
/* partial slots one CTA can need */
uint32_t gemm_max_local(uint32_t mtiles, uint32_t kblocks, uint32_t grid);
cudaError_t launch_gemm(const GemmParams &p, uint32_t grid, cudaStream_t stream);

/* Per-stream kernels of one step. */
struct StepParams {
    uint32_t streams, npad_total;  /* all streams; npad of each pass is min(128, ...) */
    uint32_t hidden, heads, inter, vocab, layers;
    float eps;
    const uint16_t *emb;           /* BF16 [V][H] */
    const float *aux;              /* per layer: attn_norm | o_norm | mlp_norm | conv_w | a_log | dt_bias */
    size_t aux_stride;
    const float *final_norm;
    const int32_t *tokens;         /* [steps][streams] */
    uint32_t *step;                /* device step counter */
    int32_t *argmax_out;           /* [steps][streams] */
    int greedy;                    /* feed the previous argmax instead of tokens[step] (step > 0) */
    float *resid;                  /* [streams][H] */
    float *qkv;                    /* [streams][4H + 2nh] */
    float *attn;                   /* [streams][H] */
    float *state;                  /* [streams][L][nh][256][256] */
    size_t state_stride;           /* floats per stream */
    unsigned long long *keys;      /* [streams] */
    uint32_t *status;
};

/* Activation tiles for a set of passes: pass p covers streams [128p, 128p + 128)
 * and its tiles start at base + p * pass_stride bytes. */
struct TileOut {
    uint8_t *base;
    size_t pass_stride;
    uint32_t npad_last;            /* npad of the last pass */
    uint32_t passes;
};

/* x <- E[token] (layer 0) and RMSNorm(x) as activation tiles (K = H) */
cudaError_t launch_input(const StepParams &p, const float *norm_w, int embed, TileOut out, cudaStream_t stream);
/* recurrence of layer l: S, attn from the QKVGAB output */
cudaError_t launch_recur(const StepParams &p, uint32_t layer, cudaStream_t stream);
/* output norm x swish gate as activation tiles (K = H) */
cudaError_t launch_gate_norm(const StepParams &p, uint32_t layer, TileOut out, cudaStream_t stream);
/* argmax tokens of the step, step counter advance */
cudaError_t launch_finish(const StepParams &p, cudaStream_t stream);

size_t tile_pass_bytes(uint32_t npad, uint32_t k);

}  // namespace bt
}  // namespace gdn

#endif
