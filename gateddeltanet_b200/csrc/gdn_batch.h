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
 *     reference's order) in two buffers that alternate by step, so that the
 *     CTAs sharing a head read the old window while others write the new
 *     one; residual x FP32 [H].
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
constexpr int kMaxPassStreams = 80;   /* streams per GEMM pass: MMA N = 3 x 80 <= 256 */
constexpr int kGemmThreads = 224;     /* warps 0-3 epilogue, 4 A copies, 5 B copies, 6 MMA */

enum Error : uint32_t {
    kErrNone = 0,
    kErrWaitA = 1,
    kErrWaitB = 2,
    kErrWaitMma = 3,
    kErrWaitAcc = 4,
    kErrWaitDrain = 5,
    kErrBadToken = 6,
};

/* Unit partition of one projection: CTA c of `grid` takes the contiguous
 * (tile, k-block) units [unit_start(c), unit_start(c + 1)). */
__host__ __device__ __forceinline__ uint32_t unit_start(uint32_t c, uint32_t units, uint32_t grid) {
    return (uint32_t)(((uint64_t)c * units) / grid);
}
/* the CTA whose range holds unit u: the largest c with unit_start(c) <= u */
__host__ __device__ __forceinline__ uint32_t unit_owner(uint32_t u, uint32_t units, uint32_t grid) {
    return (uint32_t)((((uint64_t)(u + 1) * grid) + units - 1) / units) - 1u;
}

/* Split-K partial sums of one projection. The (tile, k-block) units are split
 * over the launch's CTAs in contiguous ranges; CTA c writes, for each tile
 * segment it covers (local index j = tile - its first tile), the FP32 block
 * [npad][128] (stream-major, rows of the tile contiguous) at
 *   base + pass * pass_stride + (c * max_local + j) * npad * 128
 * floats. The consumer of the projection sums the segments of a row's tile in
 * k order (deterministic), so no GEMM waits for another CTA. */
struct Partials {
    float *base;
    size_t pass_stride;   /* floats per pass */
    uint32_t units, grid, kblocks, max_local;
    uint32_t npad_last, passes;
};

struct GemmParams {
    const uint8_t *a;      /* tile image, [m-tile][k-block] 16 KB blocks */
    const uint8_t *b;      /* activation tiles of this pass */
    uint32_t kblocks;      /* K / 64 */
    uint32_t mtiles;       /* ceil(M / 128) */
    uint32_t npad;         /* streams of this pass, padded to a multiple of 16 */
    uint32_t a_slots, b_slots;
    float *partial;        /* this pass's slots */
    uint32_t max_local;    /* slots per CTA */
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
    uint32_t streams;
    uint32_t hidden, heads, inter, vocab, layers;
    float eps;
    const uint16_t *emb;           /* BF16 [V][H] */
    const float *aux;              /* per layer: attn_norm | o_norm | mlp_norm | conv_w | a_log | dt_bias */
    size_t aux_stride;
    const int32_t *tokens;         /* [steps][streams] */
    uint32_t *step;                /* device step counter */
    int32_t *argmax_out;           /* [steps][streams] */
    int greedy;                    /* feed the previous argmax instead of tokens[step] (step > 0) */
    float *resid;                  /* [streams][H] */
    float *attn;                   /* [streams][H] */
    float *state;                  /* [streams][L][nh][256][256] */
    size_t state_stride;           /* floats per stream */
    float *tails;                  /* [2][streams][L][3][3][H]: read buffer *tails_parity, write the other */
    size_t tails_stride;           /* floats per stream */
    size_t tails_buf;              /* floats per buffer */
    uint32_t *tails_parity;
    float *logits;                 /* [streams][V] */
    unsigned long long *keys;      /* [streams] */
    uint32_t *status;
};

/* Activation tiles for a set of passes: pass p covers streams [80p, 80p + 80)
 * and its tiles start at base + p * pass_stride bytes. */
struct TileOut {
    uint8_t *base;
    size_t pass_stride;
    uint32_t npad_last;            /* npad of the last pass */
    uint32_t passes;
};

/* x <- E[token] (mode 0) or x <- x + the projection's sums (mode 1, then x is
 * stored back); RMSNorm(x) with norm_w as activation tiles (K = H) */
cudaError_t launch_input(const StepParams &p, const float *norm_w, int mode, const Partials &add, TileOut out,
                         cudaStream_t stream);
/* causal conv + SiLU of q, k, v, norms and gates (prep, two launches), then
 * the recurrence of layer l; prep holds prep_floats() floats */
cudaError_t launch_recur(const StepParams &p, uint32_t layer, const Partials &qkv, float *prep, cudaStream_t stream);
size_t prep_floats(uint32_t streams, uint32_t heads);
/* prep, recurrence and output norm x swish gate of layer l in one kernel per
 * (stream, head); writes the O projection's activation tiles (K = H) */
cudaError_t launch_head(const StepParams &p, uint32_t layer, const Partials &qkv, TileOut out, cudaStream_t stream);
/* output norm x swish gate as activation tiles (K = H) */
cudaError_t launch_gate_norm(const StepParams &p, uint32_t layer, const Partials &qkv, TileOut out,
                             cudaStream_t stream);
/* prefill: conv, norms and the recurrence of layer l for the ntok tokens of a
 * chunk (the "streams" of its projections), on a single-stream run state's
 * S [L][nh][v][k] and tails [L][3][H][4]; new tails go to tails_out; the
 * outputs to p.attn [ntok][H] */
cudaError_t launch_prefill_head(const StepParams &p, uint32_t layer, const Partials &qkv, float *state,
                                const float *tails_in, float *tails_out, uint32_t ntok, cudaStream_t stream);
/* m = silu(gate) * up as activation tiles (K = I) */
cudaError_t launch_swiglu(const StepParams &p, const Partials &gu, TileOut out, cudaStream_t stream);
/* FP32 logits and the per-stream argmax keys */
cudaError_t launch_logits(const StepParams &p, const Partials &lm, cudaStream_t stream);
/* argmax tokens of the step, step counter and tail parity advance */
cudaError_t launch_finish(const StepParams &p, cudaStream_t stream);

size_t tile_pass_bytes(uint32_t npad, uint32_t k);

}  // namespace bt
}  // namespace gdn

#endif
