/* gdn_decode.cu -- one GatedDeltaNet decode token as a single persistent
 * sm_100a kernel.
 *
 * The reference computes a token as 24 x {a/b + QKVG GEMV with short conv and
 * gated delta rule, output norm/gate, o_proj, residual + norm, gate/up with
 * SwiGLU, down, residual + norm} and an LM head with argmax
 * (c_impl/gdn_model.cpp:3532-3897). At batch 1 every one of those steps is
 * bound by HBM bytes (2.8 GB of BF16 weights + 100 MB of FP32 state per
 * token), so the kernel is organised around keeping HBM busy:
 *
 *   - grid = one CTA per SM, launched cooperatively; each CTA owns a fixed
 *     slice of every phase's rows (and of the recurrent state's columns);
 *   - warp 8 of every CTA is a producer: one lane walks the CTA's whole
 *     token schedule of weight / state chunks and streams each chunk into an
 *     11-slot shared-memory ring with cp.async.bulk (TMA bulk copies,
 *     mbarrier completion, evict-first L2 policy for weights). Weights do
 *     not depend on activations, so the producer runs ahead across phase
 *     boundaries while the consumers wait for inputs;
 *   - warps 0..7 are consumers: per phase they build the phase's input vector
 *     in shared memory from the previous phase's outputs (residual add +
 *     RMSNorm, output norm x swish gate, ...), then each warp takes every 8th
 *     chunk: tree16 dot products in the reference's reduction order, and the
 *     phase's epilogue fused per row (short conv + SiLU + conv-window update,
 *     SwiGLU, LM-head logits + argmax).
 *
 * Phases per layer l: A QKVG+a/b rows, B state columns (gated delta rule),
 * C O rows, D gate/up row pairs, E down rows; after the last layer F LM head.
 * There is no grid barrier: a phase's outputs travel as 64-bit words that
 * carry the phase's tag next to the value, and each consumer CTA polls the
 * words it needs (gdn_engine.h). A CTA cannot run more than one phase ahead
 * of any CTA it reads from, so exchange buffers are reused every layer
 * without write-after-read hazards; the residual stream lives in each CTA's
 * shared memory (every CTA computes it identically).
 *
 * Every wait (mbarrier, exchange word) is bounded by %globaltimer; on expiry
 * the kernel records an error in DecodeStatus, stops issuing copies, waits
 * for the copies already in flight and returns. The host reports -1.
 */
#include "gdn_engine.h"
#include "gdn_math.h"

#include <cuda_runtime.h>
#include <type_traits>
#include <stdint.h>

namespace gdn {
constexpr uint64_t kWaitNs = 2000000000ull;  /* 2 s: normal waits are microseconds */

/* ------------------------------------------------------------ PTX helpers */

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ uint64_t gtimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n"
        " .reg .pred p;\n"
        " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n"
        "}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar,
                                         uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1], %2, [%3], %4;" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar), "l"(policy)
        : "memory");
}
__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ void named_sync(int id, int n) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ int ld_volatile_i32(const int32_t *p) {
    return *(const volatile int32_t *)p;
}

/* ------------------------------------------------------ numeric helpers */

/* FP32 -> BF16 round-to-nearest-even with canonical NaN, as FP32
 * (the reference's fp32_to_bf16_rne, c_impl/gdn_model.cpp:314-325). */
__device__ __forceinline__ float bf16_round(float v) {
    uint32_t b = __float_as_uint(v);
    const uint32_t mag = b & 0x7fffffffu;
    if (mag >= 0x7f800000u) {
        if (mag == 0x7f800000u) return v;
        return __uint_as_float((b & 0x80000000u) ? 0xffc00000u : 0x7fc00000u);
    }
    b = (b + 0x7fffu + ((b >> 16) & 1u)) & 0xffff0000u;
    return __uint_as_float(b);
}
template <int MODE>
__device__ __forceinline__ float bnd(float v) {
    return (MODE & 1) ? bf16_round(v) : v;
}

/* exp table (2^(j/64) as hi | lo) staged in shared memory at kernel start */
__device__ __forceinline__ const float *exp_table();

/* exp / sigmoid / silu / softplus of the reference (c_impl/gdn_model.cpp:
 * 1307-1330) on the primitives of gdn_math.h. */
__device__ __forceinline__ float exp_ref(float x) { return gdn_expf(x, exp_table()); }
__device__ __forceinline__ float sigmoid_ref(float x) { return gdn_sigmoidf(x, exp_table()); }
__device__ __forceinline__ float silu_ref(float x) { return __fmul_rn(x, sigmoid_ref(x)); }
__device__ __forceinline__ float softplus_ref(float x) {
    if (x > 20.0f) return x;
    if (x < -20.0f) return exp_ref(x);
    return log1pf(exp_ref(x));
}

/* The c_impl GEMV product (c_impl/gdn_model.cpp:392-462) for finite normal
 * BF16 operands: the exact product, flushed to a signed zero below
 * 0x007fc000, else rounded to BF16 (RNE). Subnormal operands, which the
 * reference flushes first, do not occur in BF16 weights/activations of
 * normal magnitude and are not special-cased. */
__device__ __forceinline__ float native_round(float p) {
    const uint32_t b = __float_as_uint(p);
    if ((b & 0x7fffffffu) < 0x007fc000u) return __uint_as_float(b & 0x80000000u);
    return __uint_as_float((b + 0x7fffu + ((b >> 16) & 1u)) & 0xffff0000u);
}

/* Butterfly sum: lane offsets 1, 2, 4, 8, 16 give the balanced pairwise tree
 * over each aligned block, so every lane ends with the same bits. */
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }
/* Two BF16-exact floats as one packed pair {lo, hi} (inputs of the
 * BF16-boundary contract's mixed-precision products). */
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
    return (__float_as_uint(lo) >> 16) | (__float_as_uint(hi) & 0xffff0000u);
}

/* Shared-memory position of input column c. Columns come in groups of 512
 * = 32 halves of 16; lane l owns half l of a group and reads its 16 inputs as
 * four float4 (quads q = 0..3) at group*512 + q*128 + 4*l, contiguous across
 * lanes. */
__device__ __forceinline__ int xs_pos(int c) {
    const int g = c >> 9, w = c & 511, half = w >> 4, i = w & 15;
    return (g << 9) + ((i >> 2) << 7) + (half << 2) + (i & 3);
}

/* ------------------------------------------------------------ schedule */

/* Where a CTA's share of one phase lives: units [u0, u1) of unit_bytes each,
 * upc units per ring chunk. The shape depends on the phase kind only (not on
 * the layer); kernel start tabulates it in shared memory. */
struct Geom {
    const uint8_t *src;
    uint32_t unit_bytes, upc, u0, u1;
};

enum { PH_QKVG = 0, PH_STATE = 1, PH_O = 2, PH_GU = 3, PH_DOWN = 4, PH_LM = 5 };

__device__ __forceinline__ Geom geom_compute(const DecodeParams &p, int ph, uint32_t cta, uint32_t ncta) {
    Geom g;
    uint32_t total;
    const uint32_t rowH = 2u * (uint32_t)p.H;
    uint32_t rpcH = (uint32_t)kSlotBytes / rowH;
    if (rpcH > (uint32_t)kMaxRowsPerChunk) rpcH = kMaxRowsPerChunk;
    g.src = nullptr;
    switch (ph) {
    case PH_QKVG:
        total = 4u * p.H + 2u * p.nh;
        g.unit_bytes = rowH;
        g.upc = rpcH;
        break;
    case PH_STATE:
        total = (uint32_t)p.nh * kHeadDim;
        g.unit_bytes = kHeadDim * 4u;
        g.upc = kColsPerChunk;
        break;
    case PH_O:
        total = (uint32_t)p.H;
        g.unit_bytes = rowH;
        g.upc = rpcH;
        break;
    case PH_GU:
        total = (uint32_t)p.I;
        g.unit_bytes = 2u * rowH;
        g.upc = rpcH / 2u > 0 ? rpcH / 2u : 1u;
        break;
    case PH_DOWN: {
        total = (uint32_t)p.H;
        g.unit_bytes = 2u * (uint32_t)p.I;
        uint32_t r = (uint32_t)kSlotBytes / g.unit_bytes;
        g.upc = r > (uint32_t)kMaxRowsPerChunk ? (uint32_t)kMaxRowsPerChunk : (r > 0 ? r : 1u);
        break;
    }
    default:
        total = (uint32_t)p.V;
        g.unit_bytes = rowH;
        g.upc = rpcH;
        break;
    }
    g.u0 = (uint32_t)(((uint64_t)cta * total) / ncta);
    g.u1 = (uint32_t)(((uint64_t)(cta + 1) * total) / ncta);
    return g;
}

/* Base address of phase ph's units in layer l (ignored for the LM head). */
__device__ __forceinline__ const uint8_t *phase_src(const DecodeParams &p, int l, int ph) {
    const uint8_t *lw = p.wimg + (size_t)l * p.layer_stride;
    switch (ph) {
    case PH_QKVG: return lw;
    case PH_STATE: return reinterpret_cast<const uint8_t *>(p.S + (size_t)l * p.nh * kHeadDim * kHeadDim);
    case PH_O: return lw + p.off_o;
    case PH_GU: return lw + p.off_gu;
    case PH_DOWN: return lw + p.off_down;
    default: return p.w_lm;
    }
}

/* ------------------------------------------------------ exchange words */

/* Exchange words. The BF16-boundary contracts (MODE & 1) only ever exchange
 * BF16-exact values, so their word is 32 bits: the value's upper half and a
 * 16-bit tag (the low half of epoch + phase; a word always holds either this
 * launch's tag or the previous launch's, which differs by the epoch stride).
 * The FP32 contract uses 64-bit words {FP32 value, 32-bit tag}. Either way one
 * aligned store publishes value and tag together. The buffers are sized for
 * 64-bit words; a 32-bit-word contract uses the first half of each. */
template <int MODE>
struct XW {
    typedef unsigned long long T;
};
template <>
struct XW<1> {
    typedef uint32_t T;
};
template <>
struct XW<3> {
    typedef uint32_t T;
};
template <>
struct XW<5> {
    typedef uint32_t T;
};
template <>
struct XW<7> {
    typedef uint32_t T;
};

template <int MODE>
__device__ __forceinline__ typename XW<MODE>::T *xw(xword *base) {
    return reinterpret_cast<typename XW<MODE>::T *>(base);
}
template <int MODE>
__device__ __forceinline__ const typename XW<MODE>::T *xw(const xword *base) {
    return reinterpret_cast<const typename XW<MODE>::T *>(base);
}

__device__ __forceinline__ uint32_t xword_of(uint32_t *, float v, uint32_t tag) {
    return (__float_as_uint(v) & 0xffff0000u) | (tag & 0xffffu);
}
__device__ __forceinline__ unsigned long long xword_of(unsigned long long *, float v, uint32_t tag) {
    return ((unsigned long long)tag << 32) | (unsigned long long)__float_as_uint(v);
}
__device__ __forceinline__ void xstore(uint32_t *p, uint32_t w) {
    asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(w) : "memory");
}
__device__ __forceinline__ void xstore(unsigned long long *p, unsigned long long w) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
/* system scope: a store into a peer GPU's memory, or a word a peer polls */
__device__ __forceinline__ void xstore_sys(uint32_t *p, uint32_t w) {
    asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(w) : "memory");
}
__device__ __forceinline__ void xstore_sys(unsigned long long *p, unsigned long long w) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
/* address of a word of this GPU's exchange region in peer r's region */
template <class T>
__device__ __forceinline__ T *peer_addr(const DecodeParams &p, T *a, int r) {
    return reinterpret_cast<T *>(reinterpret_cast<char *>(a) + p.tp_delta[r]);
}
/* store element i of exchange buffer `base`: here and, in tensor-parallel
 * decode, in every peer's copy of the buffer */
template <int MODE>
__device__ __forceinline__ void xput(const DecodeParams &p, xword *base, size_t i, float v, uint32_t tag) {
    auto *a = xw<MODE>(base) + i;
    const auto w = xword_of(a, v, tag);
    xstore(a, w);
    if (MODE & 4)
        for (int r = 0; r < p.tp_world; ++r)
            if (r != p.tp_rank) xstore_sys(peer_addr(p, a, r), w);
}
/* Exchange-word loads. `sys`: tensor-parallel decode, where peers store the
 * words (system-scope loads, so that they and the peers' system-scope stores
 * are morally strong). */
__device__ __forceinline__ uint32_t xget(const uint32_t *p, bool sys) {
    uint32_t w;
    if (sys) asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(w) : "l"(p) : "memory");
    else asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(w) : "l"(p) : "memory");
    return w;
}
__device__ __forceinline__ unsigned long long xget(const unsigned long long *p, bool sys) {
    unsigned long long w;
    if (sys) asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    else asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}
__device__ __forceinline__ void xget2(const uint32_t *p, uint32_t &a, uint32_t &b, bool sys) {
    if (sys) asm volatile("ld.relaxed.sys.global.v2.u32 {%0, %1}, [%2];" : "=r"(a), "=r"(b) : "l"(p) : "memory");
    else asm volatile("ld.relaxed.gpu.global.v2.u32 {%0, %1}, [%2];" : "=r"(a), "=r"(b) : "l"(p) : "memory");
}
__device__ __forceinline__ void xget2(const unsigned long long *p, unsigned long long &a, unsigned long long &b,
                                      bool sys) {
    if (sys) asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
    else asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
__device__ __forceinline__ bool xtag_is(uint32_t w, uint32_t tag) { return (w & 0xffffu) == (tag & 0xffffu); }
__device__ __forceinline__ bool xtag_is(unsigned long long w, uint32_t tag) { return (uint32_t)(w >> 32) == tag; }
__device__ __forceinline__ float xval(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }
__device__ __forceinline__ float xval(unsigned long long w) { return __uint_as_float((uint32_t)w); }

/* ------------------------------------------------------- shared memory */

/* Shared-memory layout: every region sits at a compile-time offset (so the
 * region pointers fold into immediate addresses instead of occupying
 * registers); only the size of the last region, xs, depends on the shape. */
constexpr size_t kOffRing = 0;
constexpr size_t kOffChain = kOffRing + (size_t)kSlots * kSlotBytes;
constexpr size_t kOffRed = kOffChain + (size_t)kConsumerWarps * 512 * 4;
constexpr size_t kOffHscal = kOffRed + 160 * 4;
constexpr size_t kOffWbest = kOffHscal + 16 * 4;
constexpr size_t kOffWbestI = kOffWbest + 8 * 4;
constexpr size_t kOffBars = kOffWbestI + 8 * 4;
constexpr size_t kOffFlags = kOffBars + kSlots * 8;
constexpr size_t kOffShape = kOffFlags + 16;          /* [6 phase kinds][8] u32, see PhaseShape */
constexpr size_t kOffIssued = kOffShape + 6 * 8 * 4;  /* [kSlots] u32 copies issued per ring slot */
constexpr size_t kOffExpTab = (kOffIssued + kSlots * 4 + 15) & ~(size_t)15;
constexpr size_t kOffXres = kOffExpTab + 128 * 4;
constexpr size_t kMaxHidden = 2048;
constexpr size_t kOffXs = kOffXres + kMaxHidden * 4;

extern __shared__ __align__(128) uint8_t smem_raw[];

/* Region accessors: constant offsets from the dynamic shared-memory base, so
 * they fold into immediate addresses and need no registers or stack. */
__device__ __forceinline__ uint8_t *sm_ring() { return smem_raw + kOffRing; }
/* permuted phase input, max(H, I) floats; phase B: qn | kn */
__device__ __forceinline__ float *sm_xs() { return reinterpret_cast<float *>(smem_raw + kOffXs); }
/* [2][256] normalised q/k of the CTA's (at most two) heads */
__device__ __forceinline__ float *sm_qn() { return sm_xs(); }
__device__ __forceinline__ float *sm_kn() { return sm_xs() + 2 * kHeadDim; }
/* residual stream, H floats (the same in every CTA) */
__device__ __forceinline__ float *sm_xres() { return reinterpret_cast<float *>(smem_raw + kOffXres); }
/* 160 floats: half sums [0,128), block partials [0,64), scalars [128,160) */
__device__ __forceinline__ float *sm_red() { return reinterpret_cast<float *>(smem_raw + kOffRed); }
/* [8 warps][512] per-warp GEMV bank partials */
__device__ __forceinline__ float *sm_chain() { return reinterpret_cast<float *>(smem_raw + kOffChain); }
/* [2][4] alpha, beta, decay per local head; [8, 16) per-head norm scales */
__device__ __forceinline__ float *sm_hscal() { return reinterpret_cast<float *>(smem_raw + kOffHscal); }
__device__ __forceinline__ float *sm_wbest() { return reinterpret_cast<float *>(smem_raw + kOffWbest); }
__device__ __forceinline__ int32_t *sm_wbest_i() { return reinterpret_cast<int32_t *>(smem_raw + kOffWbestI); }
__device__ __forceinline__ uint64_t *sm_full() { return reinterpret_cast<uint64_t *>(smem_raw + kOffBars); }
/* per phase kind: unit_bytes, upc, u0, u1, chunks; then [8] = chunks per layer */
__device__ __forceinline__ uint32_t *sm_shape() { return reinterpret_cast<uint32_t *>(smem_raw + kOffShape); }
__device__ __forceinline__ uint32_t *sm_issued() { return reinterpret_cast<uint32_t *>(smem_raw + kOffIssued); }
/* set by any thread of the CTA that gives up */
__device__ __forceinline__ volatile int32_t *sm_abort_flag() {
    return reinterpret_cast<volatile int32_t *>(smem_raw + kOffFlags);
}
/* thread 0's CTA-uniform go/stop, read after a barrier */
__device__ __forceinline__ volatile int32_t *sm_decision() {
    return reinterpret_cast<volatile int32_t *>(smem_raw + kOffFlags + 4);
}

size_t decode_smem_bytes(int H, int I) {
    return kOffXs + (size_t)4 * (H > I ? H : I);
}

__device__ __forceinline__ const float *exp_table() {
    return reinterpret_cast<const float *>(smem_raw + kOffExpTab);
}

/* This CTA's share of phase kind ph in layer l, from the table. */
__device__ __forceinline__ Geom geom(const DecodeParams &p, int l, int ph) {
    const uint32_t *t = sm_shape() + ph * 8;
    Geom g;
    g.unit_bytes = t[0];
    g.upc = t[1];
    g.u0 = t[2];
    g.u1 = t[3];
    g.src = phase_src(p, l, ph);
    return g;
}

/* A ring refill: chunk `idx` of layer `l` of the CTA's schedule (each layer's
 * phases A..E, then the LM head as layer L; idx may run past the end of the
 * layer and is carried into the next), into ring slot `slot`, whose
 * `count`-th copy it is (1-based). */
struct Refill {
    uint32_t l, idx, slot, count;
};

/* Start the bulk copy of a refill; nothing past the end of the schedule. One
 * lane calls this, once the slot's previous chunk has been read. Weights
 * stream with L2 evict_first, the recurrent state with evict_last (it is
 * written back right after). */
/* A resolved refill: what issue_refill copies (bytes == 0: nothing). */
struct RefillDesc {
    const uint8_t *src;
    uint32_t bytes, slot, count, state;
};

/* Resolve a refill against the shape table (shared-memory reads; done before
 * the chunk's own work so their latency overlaps it). */
__device__ __forceinline__ RefillDesc prepare_refill(const DecodeParams &p, Refill f) {
    RefillDesc d;
    d.bytes = 0;
    d.slot = f.slot;
    d.count = f.count;
    const uint32_t *sh = sm_shape();
    const uint32_t per_layer = sh[PH_LM * 8 + 7];
    uint32_t l = f.l, i = f.idx;
    while (l < (uint32_t)p.L && i >= per_layer) {
        i -= per_layer;
        ++l;
    }
    int ph;
    if (l >= (uint32_t)p.L) {
        if (i >= sh[PH_LM * 8 + 4]) return d;
        ph = PH_LM;
        l = 0;
    } else {
        ph = (int)(i >= sh[1 * 8 + 5]) + (int)(i >= sh[2 * 8 + 5]) + (int)(i >= sh[3 * 8 + 5]) +
             (int)(i >= sh[4 * 8 + 5]);
        i -= sh[ph * 8 + 5];
    }
    const uint32_t *t = sh + ph * 8;
    const uint32_t u = t[2] + i * t[1];
    const uint32_t n = (t[3] - u) < t[1] ? (t[3] - u) : t[1];
    d.bytes = n * t[0];
    d.src = phase_src(p, (int)l, ph) + (size_t)u * t[0];
    d.state = ph == PH_STATE;
    return d;
}

__device__ __forceinline__ void issue_refill(const RefillDesc &d) {
    if (d.bytes == 0) return;
    const uint32_t fb = smem_u32(&sm_full()[d.slot]);
    *reinterpret_cast<volatile uint32_t *>(sm_issued() + d.slot) = d.count;
    mbar_expect_tx(fb, d.bytes);
    bulk_g2s(smem_u32(sm_ring() + (size_t)d.slot * kSlotBytes), d.src, d.bytes, fb,
             d.state ? policy_evict_last() : policy_evict_first());
}

__device__ __forceinline__ void issue_chunk(const DecodeParams &p, Refill f) { issue_refill(prepare_refill(p, f)); }

/* --------------------------------------------------- block-level helpers */

/* Deterministic sum over the 256 consumer threads of N values each: warp
 * butterfly, then a fixed pairwise tree over the 8 warps. Over 256 inputs
 * held one per thread this is exactly the balanced tree of
 * gdn_tree_reduce_256 (c_impl/gdn_model.cpp:1336-1375). */
template <int N>
__device__ __forceinline__ void block_sum(float (&v)[N], float *red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int i = 0; i < N; ++i) v[i] = warp_sum(v[i]);
    if (lane == 0) {
#pragma unroll
        for (int i = 0; i < N; ++i) red[warp * 8 + i] = v[i];
    }
    named_sync(1, kConsumerThreads);
#pragma unroll
    for (int i = 0; i < N; ++i) {
        const float a = __fadd_rn(red[0 * 8 + i], red[1 * 8 + i]);
        const float b = __fadd_rn(red[2 * 8 + i], red[3 * 8 + i]);
        const float c = __fadd_rn(red[4 * 8 + i], red[5 * 8 + i]);
        const float d = __fadd_rn(red[6 * 8 + i], red[7 * 8 + i]);
        v[i] = __fadd_rn(__fadd_rn(a, b), __fadd_rn(c, d));
    }
    named_sync(1, kConsumerThreads);
}

__device__ __forceinline__ void trace_put(const DecodeParams &p, int phase, int slot) {
    if (p.trace != nullptr)
        p.trace[((size_t)blockIdx.x * (p.L * kPhasesPerLayer + 1) + phase) * kTraceSlots + slot] = gtimer();
}

__device__ __forceinline__ void raise_error(const DecodeParams &p, int code, uint32_t where) {
    if (atomicCAS(&p.status->err, 0, code) == 0) {
        p.status->err_cta = blockIdx.x;
        p.status->err_where = where;
    }
    *sm_abort_flag() = 1;
}

/* Spin on one exchange word until it carries `tag`; returns the last word
 * read, whose tag differs from `tag` on abort/timeout. */
template <bool SYS, class W>
__device__ __noinline__ W xwait(const DecodeParams &p, const W *a, uint32_t tag) {
    const uint64_t t0 = gtimer();
    uint32_t spins = 0;
    while (true) {
        const W w = xget(a, SYS);
        if (xtag_is(w, tag)) return w;
        if (*sm_abort_flag()) return w;
        if ((++spins & 63u) == 0) {
            if (ld_volatile_i32(&p.status->err) != 0) {
                *sm_abort_flag() = 1;
                return w;
            }
            if (gtimer() - t0 > kWaitNs) {
                raise_error(p, kErrExchangeTimeout, tag);
                return w;
            }
        }
    }
}

/* Warp-wide read of exchange words: lane word i (i < N, where use(i)) lives
 * at addr(i) and must carry tag tagof(i). PAIRS: words 2k and 2k + 1 are
 * adjacent and 16-byte aligned, and are fetched with one vector load. Callers
 * lay the words out so that a warp's loads are coalesced (consecutive lanes
 * at consecutive addresses): per-thread contiguous runs cost several times
 * more. Every load is issued at once, so data that is already there costs
 * one round trip. While words are missing, every lane re-reads its own
 * missing words, so the read completes one round trip after the last word
 * lands. All 32 lanes must call; lanes
 * that use no word take part in the protocol only. With PAIRS, use(2k) must
 * equal use(2k + 1). */
template <int N, bool PAIRS, bool SYS, class Addr, class TagOf, class Use>
__device__ __forceinline__ bool xread(const DecodeParams &p, const Addr &addr, const TagOf &tagof, const Use &use,
                                      float (&v)[N]) {
    typedef typename std::remove_const<typename std::remove_pointer<decltype(addr(0))>::type>::type W;
    const int lane = threadIdx.x & 31;
    constexpr bool sys = SYS;
    W w[N];
    if (PAIRS) {
#pragma unroll
        for (int i = 0; i < N; i += 2)
            if (use(i)) xget2(addr(i), w[i], w[i + 1], sys);
    } else {
#pragma unroll
        for (int i = 0; i < N; ++i)
            if (use(i)) w[i] = xget(addr(i), sys);
    }
    uint32_t missing = 0;
#pragma unroll
    for (int i = 0; i < N; ++i)
        if (use(i) && !xtag_is(w[i], tagof(i))) missing |= 1u << i;
    uint64_t t0 = 0;
    uint32_t rounds = 0;
    while (__any_sync(0xffffffffu, missing != 0)) {
        /* every lane re-reads its own missing words, so the read completes one
         * round trip after the last word lands; the words still missing after
         * the first read are the few of the slowest producers */
#pragma unroll
        for (int i = 0; i < N; ++i)
            if ((missing >> i) & 1u) w[i] = xget(addr(i), sys);
#pragma unroll
        for (int i = 0; i < N; ++i)
            if (((missing >> i) & 1u) && xtag_is(w[i], tagof(i))) missing &= ~(1u << i);
        if ((++rounds & 15u) == 0) {
            /* lane 0 decides for the warp: abort raised elsewhere, or timeout */
            int stop = 0;
            if (lane == 0) {
                if (*sm_abort_flag() != 0 || ld_volatile_i32(&p.status->err) != 0) stop = 1;
                else if (t0 == 0) t0 = gtimer();
                else if (gtimer() - t0 > kWaitNs) stop = 2;
            }
            stop = __shfl_sync(0xffffffffu, stop, 0);
            if (stop) {
                const uint32_t any = __ballot_sync(0xffffffffu, missing != 0);
                if (stop == 2 && lane == __ffs(any) - 1) raise_error(p, kErrExchangeTimeout, tagof(__ffs(missing) - 1));
                *sm_abort_flag() = 1;
                return false;
            }
        }
    }
#pragma unroll
    for (int i = 0; i < N; ++i)
        if (use(i)) v[i] = xval(w[i]);
    return true;
}

/* The coalesced element order of a whole-vector read: thread t's word i is
 * element 2t + 512 (i >> 1) + (i & 1) -- word pairs, consecutive threads on
 * consecutive pairs. n/256 words per thread for an n-element vector (n a
 * multiple of 512). */
__device__ __forceinline__ int vec_elem(int t, int i) { return 2 * t + 512 * (i >> 1) + (i & 1); }

/* Position of the packed BF16 pair of columns c, c + 1 (c even) in the packed
 * input: per 512-column group, uint4 j (columns 8j..8j+7 of a half) of half h
 * at (group << 6) + 32 j + h, so lane h reads its half with two conflict-free
 * 16-byte loads. */
__device__ __forceinline__ int xsp_pos(int c) {
    const int k = (c & 15) >> 1;
    return ((c >> 9) << 8) + ((k >> 2) << 7) + (((c & 511) >> 4) << 2) + (k & 3);
}

/* Read n exchange words (coalesced order) into the shared input: FP32 in the
 * permuted order of xs_pos, or, in the BF16-boundary contract, as packed
 * pairs at xsp_pos. n <= 5632, the workspace ABI's intermediate size. All
 * consumer threads call. */
constexpr int kMaxWordsPerThread = 22;
template <int MODE>
__device__ __forceinline__ bool xread_to_xs(const DecodeParams &p, const xword *src, int n, uint32_t tag) {
    const int t = threadIdx.x;
    const int per = n >> 8;
    float v[kMaxWordsPerThread];
    const bool ok = xread<kMaxWordsPerThread, true, (MODE & 4) != 0>(
        p, [&](int i) { return xw<MODE>(src) + vec_elem(t, i); }, [&](int) { return tag; },
        [&](int i) { return i < per; }, v);
    if ((MODE & 3) == 1) {
        uint32_t *xsp = reinterpret_cast<uint32_t *>(sm_xs());
#pragma unroll
        for (int j = 0; j < kMaxWordsPerThread; j += 2)
            if (j < per) xsp[xsp_pos(vec_elem(t, j))] = pack_bf16(v[j], v[j + 1]);
    } else {
#pragma unroll
        for (int j = 0; j < kMaxWordsPerThread; ++j)
            if (j < per) sm_xs()[xs_pos(vec_elem(t, j))] = v[j];
    }
    return ok;
}

/* Store this thread's phase-input elements (coalesced order of vec_elem,
 * count per <= 8, even) into the shared input of the phase's GEMV. */
template <int MODE>
__device__ __forceinline__ void store_input(const float (&o)[8], int per) {
    const int t = threadIdx.x;
    if ((MODE & 3) == 1) {
        uint32_t *xsp = reinterpret_cast<uint32_t *>(sm_xs());
#pragma unroll
        for (int i = 0; i < 8; i += 2)
            if (i < per) xsp[xsp_pos(vec_elem(t, i))] = pack_bf16(o[i], o[i + 1]);
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i)
            if (i < per) sm_xs()[xs_pos(vec_elem(t, i))] = o[i];
    }
}

/* Single-lane read of one exchange word. */
template <bool SYS, class W>
__device__ __forceinline__ bool xread1(const DecodeParams &p, const W *src, uint32_t tag, float &v) {
    W w = xget(src, SYS);
    if (!xtag_is(w, tag)) w = xwait<SYS>(p, src, tag);
    v = xval(w);
    return xtag_is(w, tag);
}

/* Wait until chunk q of the schedule sits in its ring slot; false on abort.
 * The slot's copy of q is issued only after the slot's previous chunk
 * (q - kSlots) has been read, but a warp may reach q earlier than that: it
 * first waits (in shared memory) for the issue, so that the mbarrier it then
 * waits on is never more than one phase ahead of the copy -- the parity test
 * cannot tell phase k from phase k - 2. */
__device__ __forceinline__ bool wait_full(const DecodeParams &p, uint32_t q) {
    const uint32_t slot = q % kSlots, k = q / kSlots;
    const uint32_t bar = smem_u32(&sm_full()[slot]);
    const volatile uint32_t *issued = sm_issued() + slot;
    if (*issued > k && mbar_try(bar, k & 1u)) return true;
    const uint64_t t0 = gtimer();
    while (true) {
        if (*issued > k && mbar_try(bar, k & 1u)) return true;
        if (*sm_abort_flag()) return false;
        if (gtimer() - t0 > kWaitNs) {
            raise_error(p, kErrChunkTimeout, q);
            return false;
        }
    }
}

/* Products of one BF16 weight with one input in the selected contract. */
template <int MODE>
__device__ __forceinline__ float prod(float w, float x) {
    const float p = __fmul_rn(w, x);
    return (MODE & 2) ? native_round(p) : p;
}

/* tree16 of one 16-column half (gemv32_tree16, c_impl/gdn_model.cpp:4004-4035):
 * ((p0+p1)+(p2+p3)) + ((p4+p5)+(p6+p7)) ... over the 16 products. With BF16
 * inputs and exact products a pair sum p0 + p1 equals fma(w1, x1, p0). */
template <int MODE>
__device__ __forceinline__ float tree16_half(const uint4 &w0, const uint4 &w1, const float4 &x0, const float4 &x1,
                                             const float4 &x2, const float4 &x3) {
    float s0, s1, s2, s3, s4, s5, s6, s7;
    if ((MODE & 3) == 1) {
        s0 = fmaf(bf_hi(w0.x), x0.y, __fmul_rn(bf_lo(w0.x), x0.x));
        s1 = fmaf(bf_hi(w0.y), x0.w, __fmul_rn(bf_lo(w0.y), x0.z));
        s2 = fmaf(bf_hi(w0.z), x1.y, __fmul_rn(bf_lo(w0.z), x1.x));
        s3 = fmaf(bf_hi(w0.w), x1.w, __fmul_rn(bf_lo(w0.w), x1.z));
        s4 = fmaf(bf_hi(w1.x), x2.y, __fmul_rn(bf_lo(w1.x), x2.x));
        s5 = fmaf(bf_hi(w1.y), x2.w, __fmul_rn(bf_lo(w1.y), x2.z));
        s6 = fmaf(bf_hi(w1.z), x3.y, __fmul_rn(bf_lo(w1.z), x3.x));
        s7 = fmaf(bf_hi(w1.w), x3.w, __fmul_rn(bf_lo(w1.w), x3.z));
    } else {
        s0 = __fadd_rn(prod<MODE>(bf_lo(w0.x), x0.x), prod<MODE>(bf_hi(w0.x), x0.y));
        s1 = __fadd_rn(prod<MODE>(bf_lo(w0.y), x0.z), prod<MODE>(bf_hi(w0.y), x0.w));
        s2 = __fadd_rn(prod<MODE>(bf_lo(w0.z), x1.x), prod<MODE>(bf_hi(w0.z), x1.y));
        s3 = __fadd_rn(prod<MODE>(bf_lo(w0.w), x1.z), prod<MODE>(bf_hi(w0.w), x1.w));
        s4 = __fadd_rn(prod<MODE>(bf_lo(w1.x), x2.x), prod<MODE>(bf_hi(w1.x), x2.y));
        s5 = __fadd_rn(prod<MODE>(bf_lo(w1.y), x2.z), prod<MODE>(bf_hi(w1.y), x2.w));
        s6 = __fadd_rn(prod<MODE>(bf_lo(w1.z), x3.x), prod<MODE>(bf_hi(w1.z), x3.y));
        s7 = __fadd_rn(prod<MODE>(bf_lo(w1.w), x3.z), prod<MODE>(bf_hi(w1.w), x3.w));
    }
    const float a0 = __fadd_rn(s0, s1), a1 = __fadd_rn(s2, s3), a2 = __fadd_rn(s4, s5), a3 = __fadd_rn(s6, s7);
    return __fadd_rn(__fadd_rn(a0, a1), __fadd_rn(a2, a3));
}

/* w.lo * x.lo + w.hi * x.hi of packed BF16 pairs as the reference's pair sum
 * (lo product + hi product, both exact, one rounding): mixed-precision FMA
 * with BF16 multiplicands and FP32 addend, which multiplies exactly and rounds
 * once; the first FMA adds -0.0 so an exact zero product keeps its sign. */
__device__ __forceinline__ float pair_sum(uint32_t w, uint32_t x) {
    float d;
    asm("{\n .reg .b16 wl, wh, xl, xh;\n mov.b32 {wl, wh}, %1;\n mov.b32 {xl, xh}, %2;\n"
        " fma.rn.f32.bf16 %0, wl, xl, 0f80000000;\n fma.rn.f32.bf16 %0, wh, xh, %0;\n}"
        : "=f"(d)
        : "r"(w), "r"(x));
    return d;
}

/* tree16 of one 16-column half from packed pairs (same order as tree16_half). */
__device__ __forceinline__ float tree16_mx(const uint4 &w0, const uint4 &w1, const uint4 &x0, const uint4 &x1) {
    const float s0 = pair_sum(w0.x, x0.x), s1 = pair_sum(w0.y, x0.y), s2 = pair_sum(w0.z, x0.z),
                s3 = pair_sum(w0.w, x0.w);
    const float s4 = pair_sum(w1.x, x1.x), s5 = pair_sum(w1.y, x1.y), s6 = pair_sum(w1.z, x1.z),
                s7 = pair_sum(w1.w, x1.w);
    const float a0 = __fadd_rn(s0, s1), a1 = __fadd_rn(s2, s3), a2 = __fadd_rn(s4, s5), a3 = __fadd_rn(s6, s7);
    return __fadd_rn(__fadd_rn(a0, a1), __fadd_rn(a2, a3));
}

/* Chain scratch layout: row r, bank b holds C = K/64 positions at
 * (4r + b) C. Position q = 8g + j (group g, lane group j) is stored at
 * 8 (g ^ b) + j when G % 4 == 0 -- otherwise the four banks of a row would
 * land on the same shared-memory banks; the XOR keeps every aligned run of 8
 * positions contiguous (stage 2 reads float4). */

/* Stage 1 for a compile-time shape (G groups, NR rows, MODE 1): every
 * address folds to an immediate and each group's loads are issued before its
 * products, the same arithmetic as the general loop of warp_dot. */
template <int G, int NR>
__device__ __forceinline__ void dot_fixed(const uint8_t *slot, const float *xs, float *chain, int lane) {
    constexpr int K = G * 512, C = G * 8;
    constexpr bool kSwizzle = (G % 4) == 0;
    const int b_own = lane & 3;
    float *park = chain + b_own * C + (lane >> 2);
    const uint4 *xsp4 = reinterpret_cast<const uint4 *>(xs);
#pragma unroll
    for (int g = 0; g < G; ++g) {
        const uint4 x0 = xsp4[(g << 6) + lane], x1 = xsp4[(g << 6) + 32 + lane];
        uint4 wa[NR], wb[NR];
#pragma unroll
        for (int r = 0; r < NR; ++r) {
            const uint4 *wr = reinterpret_cast<const uint4 *>(slot + (size_t)r * K * 2) + (g << 6);
            wa[r] = wr[lane];
            wb[r] = wr[32 + lane];
        }
#pragma unroll
        for (int r = 0; r < NR; ++r)
            park[r * 4 * C + ((kSwizzle ? (g ^ b_own) : g) << 3)] = tree16_mx(wa[r], wb[r], x0, x1);
    }
}

/* Stage 2 for a compile-time chain length C: the bank's C partials (XOR
 * layout of dot_fixed when C % 32 == 0) are loaded first, then summed in
 * position order from 0.0f. */
template <int C>
__device__ __forceinline__ float chain_sum_fixed(const float *c, int b) {
    const int sw = (C % 32 == 0) ? (b << 3) : 0;
    float4 v[C / 4];
#pragma unroll
    for (int k = 0; k < C / 4; ++k) v[k] = *reinterpret_cast<const float4 *>(c + ((4 * k) ^ sw));
    float acc = 0.0f;
#pragma unroll
    for (int k = 0; k < C / 4; ++k) {
        acc = __fadd_rn(acc, v[k].x);
        acc = __fadd_rn(acc, v[k].y);
        acc = __fadd_rn(acc, v[k].z);
        acc = __fadd_rn(acc, v[k].w);
    }
    return acc;
}

/* Dot products of up to 4 BF16 rows (contiguous in a ring slot, columns
 * permuted per 512-column group) with the shared input, summed in the
 * reference's order (c_impl/gdn_model.cpp:4444-4586):
 *   stage 1: lane l computes tree16 of half l of every group and parks it in
 *            the warp's chain scratch at bank (half & 3) -- lo/hi half x
 *            even/odd 32-column beat -- position half >> 2;
 *   stage 2: lane 4r + b accumulates bank b of row r sequentially from 0;
 *            row = (bank0 + bank1) + (bank2 + bank3).
 * Rows flagged in `tiny` (the a/b projections, c_impl/gdn_model.cpp:1501-1535)
 * instead take one sequential chain over all halves in column order.
 * In the BF16-boundary contract (MODE 1) the input is BF16-exact and is
 * kept as packed pairs (xsp_pos), and tree16_mx forms the products; in the
 * other contracts the FP32 input is read in the order of xs_pos.
 * Every lane returns all row sums. */
template <int MODE>
__device__ __forceinline__ void warp_dot(const uint8_t *slot, int K, int nrows, unsigned tiny, const float *xs,
                                         float *chain, const RefillDesc &refill, float (&out)[4]) {
    const int lane = threadIdx.x & 31;
    const int G = K >> 9;           /* 512-column groups */
    const int C = K >> 6;           /* halves per bank of one row */
    const int b_own = lane & 3;
    /* stage-1 parking slot of group g: bank b_own, position 8g + lane/4, with
     * the group index XOR-ed by the bank when G % 4 == 0 (chain_pos) */
    const int sw = (G & 3) ? 0 : b_own;
    float *park = chain + b_own * C + (lane >> 2);
    if ((MODE & 3) == 1 && K == 2048 && nrows == 4 && tiny == 0) {
        dot_fixed<4, 4>(slot, xs, chain, lane); /* the K = H = 2048 phases, full chunks */
    } else if ((MODE & 3) == 1 && K == 5632 && nrows == 1) {
        dot_fixed<11, 1>(slot, xs, chain, lane); /* the down projection, I = 5632 */
    } else if ((MODE & 3) == 1) {
        /* packed BF16 input in shared memory */
        const uint4 *xsp4 = reinterpret_cast<const uint4 *>(xs);
#pragma unroll 2
        for (int g = 0; g < G; ++g) {
            const uint4 x0 = xsp4[(g << 6) + lane], x1 = xsp4[(g << 6) + 32 + lane];
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                if (r < nrows) {
                    const uint4 *wr = reinterpret_cast<const uint4 *>(slot + (size_t)r * K * 2) + (g << 6);
                    park[r * 4 * C + ((g ^ sw) << 3)] = tree16_mx(wr[lane], wr[32 + lane], x0, x1);
                }
            }
        }
    } else {
        const float4 *xs4 = reinterpret_cast<const float4 *>(xs);
        for (int g = 0; g < G; ++g) {
            const float4 x0 = xs4[(g << 7) + lane];
            const float4 x1 = xs4[(g << 7) + 32 + lane];
            const float4 x2 = xs4[(g << 7) + 64 + lane];
            const float4 x3 = xs4[(g << 7) + 96 + lane];
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                if (r < nrows) {
                    const uint4 *wr = reinterpret_cast<const uint4 *>(slot + (size_t)r * K * 2) + (g << 6);
                    /* the a/b projections multiply exactly even in the c_impl
                     * contract (c_impl/gdn_model.cpp:1517-1520) */
                    const float d = ((MODE & 2) && ((tiny >> r) & 1u))
                                        ? tree16_half<MODE & 1>(wr[lane], wr[32 + lane], x0, x1, x2, x3)
                                        : tree16_half<MODE>(wr[lane], wr[32 + lane], x0, x1, x2, x3);
                    park[r * 4 * C + ((g ^ sw) << 3)] = d;
                }
            }
        }
    }
    /* the weights have been read: refill the ring slot before the bank
     * chains and the epilogue */
    __syncwarp();
    if (lane == 0) issue_refill(refill);
    const int r = lane >> 2, b = lane & 3;
    float acc = 0.0f;
    const bool is_tiny = r < nrows && ((tiny >> r) & 1u);
    if ((MODE & 3) == 1 && K == 2048 && nrows == 4 && tiny == 0) {
        if (r < 4) acc = chain_sum_fixed<32>(chain + (r * 4 + b) * 32, b);
    } else if ((MODE & 3) == 1 && K == 5632 && nrows == 1) {
        if (r == 0) acc = chain_sum_fixed<88>(chain + b * 88, b);
    } else if (r < nrows) {
        if (!is_tiny) {
            const float *c = chain + (r * 4 + b) * C;
            const int swb = (G & 3) ? 0 : (b << 3);
            for (int k = 0; k < C; k += 4) {
                const float4 v = *reinterpret_cast<const float4 *>(c + (k ^ swb));
                acc = __fadd_rn(acc, v.x);
                acc = __fadd_rn(acc, v.y);
                acc = __fadd_rn(acc, v.z);
                acc = __fadd_rn(acc, v.w);
            }
        } else if (b == 0) {
            const float *c = chain + r * 4 * C;
            const int sw1 = (G & 3) ? 0 : 8, sw2 = (G & 3) ? 0 : 16, sw3 = (G & 3) ? 0 : 24;
            for (int k = 0; k < C; ++k) {
                acc = __fadd_rn(acc, c[k]);
                acc = __fadd_rn(acc, c[C + (k ^ sw1)]);
                acc = __fadd_rn(acc, c[2 * C + (k ^ sw2)]);
                acc = __fadd_rn(acc, c[3 * C + (k ^ sw3)]);
            }
        }
    }
    const float t = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 1));  /* b=0: bank0+bank1, b=2: bank2+bank3 */
    const float t2 = __shfl_down_sync(0xffffffffu, t, 2);
    const float total = is_tiny ? acc : __fadd_rn(t, t2);
#pragma unroll
    for (int q = 0; q < 4; ++q) out[q] = __shfl_sync(0xffffffffu, total, q << 2);
    __syncwarp();
}

/* ---------------------------------------------------------- prologues */

/* Sequential sum of n (multiple of 4) floats in shared memory, in index
 * order from 0.0f (one thread). */
__device__ __forceinline__ float seq_sum(const float *a, int n) {
    float sum = 0.0f;
#pragma unroll 8
    for (int j = 0; j < n; j += 4) {
        const float4 v = *reinterpret_cast<const float4 *>(a + j);
        sum = __fadd_rn(sum, v.x);
        sum = __fadd_rn(sum, v.y);
        sum = __fadd_rn(sum, v.z);
        sum = __fadd_rn(sum, v.w);
    }
    return sum;
}

/* Residual add + RMSNorm into the permuted shared input, in the reference's
 * order (c_impl/gdn_model.cpp:1394-1476, 3351-3452). Elementwise work runs in
 * the coalesced order of vec_elem: x = round(xres + y) (or the embedding for
 * layer 0). Thread t < H/16 then sums the squares of the 16-column half t
 * (beat t/2, half t%2) sequentially; lane 0 of every warp sums the H/16 half
 * sums sequentially (redundantly, so no third barrier); scale = 1/sqrtf(sum/H
 * + eps); out = round((x*scale)*w). */
template <int MODE>
__device__ __forceinline__ bool prologue_norm(const DecodeParams &p, const xword *y, uint32_t tag,
                                              const float *w, bool embed, float *hidden, int pidx) {
    const int t = threadIdx.x, lane = t & 31;
    const int halves = p.H >> 4;
    const int per = p.H >> 8; /* even, <= 8 */
    bool ok = true;
    float x[8], wv[8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
        if (i < per) wv[i] = __ldg(w + vec_elem(t, i));
    if (embed) {
        if (p.token_src != nullptr) {
            const uint32_t *e2 = reinterpret_cast<const uint32_t *>(p.emb + (size_t)(*p.token_src) * p.H);
#pragma unroll
            for (int i = 0; i < 8; i += 2) {
                if (i < per) {
                    const uint32_t ew = __ldg(e2 + (vec_elem(t, i) >> 1));
                    x[i] = bnd<MODE>(bf_lo(ew));
                    x[i + 1] = bnd<MODE>(bf_hi(ew));
                }
            }
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i)
                if (i < per) x[i] = bnd<MODE>(p.x_embed[vec_elem(t, i)]);
        }
    } else {
        float yv[8];
        ok = xread<8, true, (MODE & 4) != 0>(p, [&](int i) { return xw<MODE>(y) + vec_elem(t, i); }, [&](int) { return tag; },
                            [&](int i) { return i < per; }, yv);
#pragma unroll
        for (int i = 0; i < 8; ++i)
            if (i < per) x[i] = bnd<MODE>(__fadd_rn(sm_xres()[vec_elem(t, i)], yv[i]));
    }
    if (t == 0) trace_put(p, pidx, 1);
#pragma unroll
    for (int i = 0; i < 8; ++i)
        if (i < per) sm_xres()[vec_elem(t, i)] = x[i];
    named_sync(1, kConsumerThreads);
    if (t < halves) {
        const float4 *h4 = reinterpret_cast<const float4 *>(sm_xres() + 16 * t);
        float hs = 0.0f;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float4 v = h4[q];
            hs = __fadd_rn(hs, __fmul_rn(v.x, v.x));
            hs = __fadd_rn(hs, __fmul_rn(v.y, v.y));
            hs = __fadd_rn(hs, __fmul_rn(v.z, v.z));
            hs = __fadd_rn(hs, __fmul_rn(v.w, v.w));
        }
        sm_red()[t] = hs;
    }
    named_sync(1, kConsumerThreads);
    float scale = 0.0f;
    if (lane == 0) {
        const float sum = seq_sum(sm_red(), halves);
        scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, (float)p.H), p.eps)));
        if (t == 0) trace_put(p, pidx, 6);
    }
    scale = __shfl_sync(0xffffffffu, scale, 0);
    float o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        if (i < per) {
            o[i] = bnd<MODE>(__fmul_rn(__fmul_rn(x[i], scale), wv[i]));
            if (hidden != nullptr) hidden[vec_elem(t, i)] = o[i];
        }
    }
    store_input<MODE>(o, per);
    return ok;
}

/* Per-head RMSNorm of the attention output times swish(gate) in the
 * reference's order (c_impl/gdn_model.cpp:3226-3349): per head, 16 half sums
 * of 16 sequential squares, summed sequentially; scale = 1/sqrtf(sum/256 +
 * eps); out = round(((a*scale)*w) * g * sigmoid(g)). Gate and attention words
 * are read together in the coalesced order of vec_elem; every warp derives
 * the head scales itself (lanes 0..nh-1), so three barriers suffice. */
template <int MODE>
__device__ __forceinline__ bool prologue_norm_gate(const DecodeParams &p, const float *o_norm,
                                                   uint32_t tag_a, uint32_t tag_b, int pidx) {
    const int t = threadIdx.x, lane = t & 31;
    const int halves = p.H >> 4;
    const int per = p.H >> 8; /* even, <= 8 */
    float *a_sh = sm_chain();  /* H <= 2048 floats: fits the 16 KB scratch */
    float wv[8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
        if (i < per) wv[i] = __ldg(o_norm + (vec_elem(t, i) & (kHeadDim - 1)));
    /* words [0, per): gate; [8, 8 + per): attention output */
    float v[16];
    const bool ok = xread<16, true, (MODE & 4) != 0>(
        p, [&](int i) { return i < 8 ? xw<MODE>(p.gate) + vec_elem(t, i) : xw<MODE>(p.attn) + vec_elem(t, i - 8); },
        [&](int i) { return i < 8 ? tag_a : tag_b; }, [&](int i) { return (i & 7) < per; }, v);
    if (t == 0) trace_put(p, pidx, 1);
#pragma unroll
    for (int i = 0; i < 8; ++i)
        if (i < per) a_sh[vec_elem(t, i)] = v[8 + i];
    named_sync(1, kConsumerThreads);
    if (t < halves) {
        const float4 *h4 = reinterpret_cast<const float4 *>(a_sh + 16 * t);
        float hs = 0.0f;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float4 a = h4[q];
            hs = __fadd_rn(hs, __fmul_rn(a.x, a.x));
            hs = __fadd_rn(hs, __fmul_rn(a.y, a.y));
            hs = __fadd_rn(hs, __fmul_rn(a.z, a.z));
            hs = __fadd_rn(hs, __fmul_rn(a.w, a.w));
        }
        sm_red()[t] = hs;
    }
    named_sync(1, kConsumerThreads);
    float hscale = 0.0f;
    if (lane < p.nh) {
        float sum = 0.0f;
#pragma unroll
        for (int j = 0; j < 16; ++j) sum = __fadd_rn(sum, sm_red()[16 * lane + j]);
        hscale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, 256.0f), p.eps)));
    }
    if (t == 0) trace_put(p, pidx, 6);
    float o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float scale = __shfl_sync(0xffffffffu, hscale, (vec_elem(t, i) >> 8) & 31);
        if (i < per) {
            const float gv = v[i];
            const float normalized = __fmul_rn(__fmul_rn(v[8 + i], scale), wv[i]);
            o[i] = bnd<MODE>(__fmul_rn(__fmul_rn(normalized, gv), sigmoid_ref(gv)));
        }
    }
    store_input<MODE>(o, per);
    return ok;
}

/* q/k L2 norms (balanced tree order of gdn_tree_reduce_256), alpha, beta
 * and decay for the CTA's heads (c_impl/gdn_model.cpp:2059-2124); all reads
 * are issued before any reduction. */
template <int MODE>
__device__ __forceinline__ bool prologue_state(const DecodeParams &p, int l, int h0, int h1,
                                            uint32_t tag) {
    const int t = threadIdx.x;
    const int nhl = h1 - h0 + 1; /* 1 or 2 */
    const float *aux = p.aux + (size_t)l * p.aux_stride;
    const float *a_log = aux + 14 * p.H + kHeadDim;
    const float *dt_bias = a_log + p.nh;
    float qk[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    float av = 0.0f, bv = 0.0f, alog = 0.0f, dtb = 0.0f;
    bool ok = true;
    if (t < 2 * nhl) {
        const int h = h0 + (t >> 1);
        alog = __ldg(a_log + h);
        dtb = __ldg(dt_bias + h);
    }
    {
        /* words: q h0, k h0 [, q h1, k h1] at stride H between q and k */
        float v4[4];
        const typename XW<MODE>::T *base = xw<MODE>(p.qkv) + h0 * kHeadDim + t;
        float vq[2], vk[2];
        ok = xread<2, false, (MODE & 4) != 0>(p, [&](int i) { return base + i * kHeadDim; }, [&](int) { return tag; },
                             [&](int i) { return i < nhl; }, vq) &&
             ok;
        ok = xread<2, false, (MODE & 4) != 0>(p, [&](int i) { return base + p.H + i * kHeadDim; }, [&](int) { return tag; },
                             [&](int i) { return i < nhl; }, vk) &&
             ok;
        v4[0] = vq[0];
        v4[1] = vk[0];
        v4[2] = nhl > 1 ? vq[1] : 0.0f;
        v4[3] = nhl > 1 ? vk[1] : 0.0f;
#pragma unroll
        for (int i = 0; i < 4; ++i) qk[i] = v4[i];
    }
    if (t < 2 * nhl) {
        const int h = h0 + (t >> 1);
        ok = xread1<(MODE & 4) != 0>(p, xw<MODE>(p.ab) + ((t & 1) ? p.nh + h : h), tag, (t & 1) ? bv : av) && ok;
    }
    float sq[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) sq[i] = __fmul_rn(qk[i], qk[i]);
    block_sum<4>(sq, sm_red());
    float al[2];
#pragma unroll
    for (int hs = 0; hs < 2; ++hs) {
        const float q_inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(sq[2 * hs], 1e-6f)));
        const float k_inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(sq[2 * hs + 1], 1e-6f)));
        const float qn = __fmul_rn(qk[2 * hs], q_inv), kn = __fmul_rn(qk[2 * hs + 1], k_inv);
        if (hs < nhl) {
            sm_qn()[hs * kHeadDim + t] = qn;
            sm_kn()[hs * kHeadDim + t] = kn;
        }
        al[hs] = __fmul_rn(qn, kn);
    }
    block_sum<2>(al, sm_red() + 32);
    /* beta and decay: thread 2h read a_h, thread 2h+1 read b_h (full-warp
     * shuffle; only threads 0..3 use the result) */
    const float other = __shfl_xor_sync(0xffffffffu, (t & 1) ? bv : av, 1);
    if (t < 2 * nhl) {
        const int hs = t >> 1;
        if ((t & 1) == 0) {
            const float b_h = other;
            const float beta = sigmoid_ref(b_h);
            const float decay_in = __fadd_rn(av, dtb);
            const float decay_val = __fmul_rn(-exp_ref(alog), softplus_ref(decay_in));
            sm_hscal()[hs * 4 + 0] = al[hs];
            sm_hscal()[hs * 4 + 1] = beta;
            sm_hscal()[hs * 4 + 2] = exp_ref(decay_val);
        }
    }
    return ok;
}

/* One chunk of the recurrence (phase B): columns u .. u + n - 1 of the layer's
 * state in ring slot `buf`; lane j < n reads column u + j. A separate,
 * non-inlined function: its long add chains get their own register
 * allocation instead of competing with the GEMV path of the chunk loop. */
template <int MODE>
__device__ __noinline__ void state_chunk(const DecodeParams &p, const uint8_t *buf, uint32_t u, uint32_t n, int h0,
                                         int l, float vv, uint32_t tag_out) {
    const int lane = threadIdx.x & 31;
    /* read pass, sequential over k for each column, c_impl/gdn_model.cpp:
     * 2184-2210: lane j < n runs the r chain of column u + j (sum S k_n),
     * lane 16 + j its p chain (sum S q_n) -- one chain per lane */
    static_assert(kColsPerChunk <= 16, "a state chunk's columns map to lanes j and 16 + j");
    float acc = 0.0f;
    const int cj = lane & 15;
    if (cj < (int)n) {
        const int hs = (int)((u + cj) >> 8) - h0;
        const float4 *col = reinterpret_cast<const float4 *>(buf) + cj * (kHeadDim / 4);
        const float4 *vec4 = reinterpret_cast<const float4 *>((lane < 16 ? sm_kn() : sm_qn()) + hs * kHeadDim);
#pragma unroll 8
        for (int k = 0; k < kHeadDim / 4; ++k) {
            const float4 sv = col[k], xv = vec4[k];
            acc = __fadd_rn(acc, __fmul_rn(sv.x, xv.x));
            acc = __fadd_rn(acc, __fmul_rn(sv.y, xv.y));
            acc = __fadd_rn(acc, __fmul_rn(sv.z, xv.z));
            acc = __fadd_rn(acc, __fmul_rn(sv.w, xv.w));
        }
    }
    for (uint32_t j = 0; j < n; ++j) {
        const uint32_t c = u + j;
        const int hs = (int)(c >> 8) - h0;
        const float rj = __shfl_sync(0xffffffffu, acc, j);
        const float pj = __shfl_sync(0xffffffffu, acc, 16 + j);
        const float vj = __shfl_sync(0xffffffffu, vv, j);
        const float alpha = sm_hscal()[hs * 4 + 0];
        const float beta = sm_hscal()[hs * 4 + 1];
        const float decay = sm_hscal()[hs * 4 + 2];
        /* c_impl/gdn_model.cpp:2214-2243 */
        const float delta = __fmul_rn(beta, __fsub_rn(vj, __fmul_rn(decay, rj)));
        const float o =
            __fmul_rn(0.0625f, __fadd_rn(__fmul_rn(decay, pj), __fmul_rn(alpha, delta)));
        if (lane == 0) xput<MODE>(p, p.attn, c, bnd<MODE>(o), tag_out);
        /* update, c_impl/gdn_model.cpp:2268-2300 */
        const float *colp = reinterpret_cast<const float *>(buf) + j * kHeadDim + lane * 8;
        const float *knp = sm_kn() + hs * kHeadDim + lane * 8;
        const float4 s0 = *reinterpret_cast<const float4 *>(colp);
        const float4 s1 = *reinterpret_cast<const float4 *>(colp + 4);
        const float4 k0 = *reinterpret_cast<const float4 *>(knp);
        const float4 k1 = *reinterpret_cast<const float4 *>(knp + 4);
        float4 n0, n1;
        n0.x = __fadd_rn(__fmul_rn(decay, s0.x), __fmul_rn(k0.x, delta));
        n0.y = __fadd_rn(__fmul_rn(decay, s0.y), __fmul_rn(k0.y, delta));
        n0.z = __fadd_rn(__fmul_rn(decay, s0.z), __fmul_rn(k0.z, delta));
        n0.w = __fadd_rn(__fmul_rn(decay, s0.w), __fmul_rn(k0.w, delta));
        n1.x = __fadd_rn(__fmul_rn(decay, s1.x), __fmul_rn(k1.x, delta));
        n1.y = __fadd_rn(__fmul_rn(decay, s1.y), __fmul_rn(k1.y, delta));
        n1.z = __fadd_rn(__fmul_rn(decay, s1.z), __fmul_rn(k1.z, delta));
        n1.w = __fadd_rn(__fmul_rn(decay, s1.w), __fmul_rn(k1.w, delta));
        if (p.bf16_state) {
            n0.x = bf16_round(n0.x); n0.y = bf16_round(n0.y);
            n0.z = bf16_round(n0.z); n0.w = bf16_round(n0.w);
            n1.x = bf16_round(n1.x); n1.y = bf16_round(n1.y);
            n1.z = bf16_round(n1.z); n1.w = bf16_round(n1.w);
        }
        float *dst = p.S + ((size_t)l * p.nh * kHeadDim + c) * kHeadDim + lane * 8;
        __stcg(reinterpret_cast<float4 *>(dst), n0);
        __stcg(reinterpret_cast<float4 *>(dst + 4), n1);
    }
}

/* ------------------------------------------------------------ the kernel */

template <int MODE>
__global__ void __launch_bounds__(kThreads, 1) gdn_decode_kernel(const __grid_constant__ DecodeParams p) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    /* the global CTA index: unit partitions run over every GPU's CTAs */
    const uint32_t cta = (uint32_t)p.tp_rank * gridDim.x + blockIdx.x, ncta = (uint32_t)p.tp_world * gridDim.x;

    if (threadIdx.x < 128)
        reinterpret_cast<float *>(smem_raw + kOffExpTab)[threadIdx.x] = __ldg(p.exp_table + threadIdx.x);
    if (threadIdx.x < 6) {
        const Geom g = geom_compute(p, threadIdx.x, cta, ncta);
        uint32_t *t = sm_shape() + threadIdx.x * 8;
        t[0] = g.unit_bytes;
        t[1] = g.upc;
        t[2] = g.u0;
        t[3] = g.u1;
        t[4] = (g.u1 - g.u0 + g.upc - 1) / g.upc;
    }
    if (threadIdx.x >= 32 && threadIdx.x < 32 + kSlots) sm_issued()[threadIdx.x - 32] = 0;
    if (threadIdx.x == 64) {
        for (int i = 0; i < kSlots; ++i) mbar_init(smem_u32(&sm_full()[i]), 1);
        *sm_abort_flag() = 0;
        *sm_decision() = 1;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        /* chunk index of each phase's first chunk inside a layer, chunks per layer */
        uint32_t acc = 0;
        for (int ph = 0; ph < kPhasesPerLayer; ++ph) {
            sm_shape()[ph * 8 + 5] = acc;
            acc += sm_shape()[ph * 8 + 4];
        }
        sm_shape()[PH_LM * 8 + 5] = 0;
        sm_shape()[PH_LM * 8 + 7] = acc;
        for (uint32_t q = 0; q < (uint32_t)kSlots; ++q) issue_chunk(p, Refill{0u, q, q, 1u});
    }
    __syncthreads();

    {
        /* ---------------------------------------------- consumer warps */
        uint32_t seq = 0;
        float best = -3.402823466e38f;
        int32_t best_i = 0;
        bool ok = true;
        /* the layer, phase and chunk loops stay rolled: unrolled, every phase
         * kind gets its own copy of the chunk code and the kernel outgrows the
         * instruction caches */
#pragma unroll 1
        for (int l = 0; l <= p.L && ok; ++l) {
            const int nph = (l < p.L) ? kPhasesPerLayer : 1;
            const float *aux = p.aux + (size_t)(l < p.L ? l : 0) * p.aux_stride;
            const uint32_t tag_base = p.epoch + (uint32_t)(l * kPhasesPerLayer);
#pragma unroll 1
            for (int pi = 0; pi < nph && ok; ++pi) {
                const int ph = (l < p.L) ? pi : PH_LM;
                const int pidx = l * kPhasesPerLayer + pi;
                const Geom g = geom(p, l < p.L ? l : 0, ph);
                /* every consumer warp is done with the previous phase's chunks
                 * (shared inputs may be overwritten) */
                named_sync(1, kConsumerThreads);
                if (threadIdx.x == 0) trace_put(p, pidx, 0);
                int h0 = 0, h1 = 0;
                bool in_ok = true;
                /* the residual-stream RMSNorm phases (A, D, LM head) share one
                 * call site, so its body is instantiated once */
                bool norm_phase = false, embed = false;
                const xword *ny = nullptr;
                uint32_t ntag = 0;
                const float *nw = aux;
                float *hidden = nullptr;
                switch (ph) {
                case PH_QKVG:
                    norm_phase = true;
                    if (l == 0) {
                        if (p.token_src != nullptr) {
                            const int32_t tok = *p.token_src;
                            if (tok < 0 || tok >= p.V) {
                                /* every consumer thread reads the same token: uniform exit */
                                if (threadIdx.x == 0) raise_error(p, kErrBadToken, (uint32_t)tok);
                                ok = false;
                                break;
                            }
                        }
                        embed = true;
                    } else {
                        ny = p.y_down;
                        ntag = tag_base - kPhasesPerLayer + PH_DOWN;
                    }
                    break;
                case PH_STATE:
                    if (g.u1 > g.u0) {
                        h0 = (int)(g.u0 >> 8);
                        h1 = (int)((g.u1 - 1) >> 8);
                        in_ok = prologue_state<MODE>(p, l, h0, h1, tag_base + PH_QKVG);
                        if (threadIdx.x == 0) trace_put(p, pidx, 1);
                    }
                    break;
                case PH_O:
                    in_ok = prologue_norm_gate<MODE>(p, aux + p.H, tag_base + PH_QKVG, tag_base + PH_STATE, pidx);
                    break;
                case PH_GU:
                    norm_phase = true;
                    ny = p.y_o;
                    ntag = tag_base + PH_O;
                    nw = aux + p.H + kHeadDim;
                    break;
                case PH_DOWN:
                    in_ok = xread_to_xs<MODE>(p, p.m, p.I, tag_base + PH_GU);
                    if (threadIdx.x == 0) trace_put(p, pidx, 1);
                    break;
                default:
                    norm_phase = true;
                    ny = p.y_down;
                    ntag = p.epoch + (uint32_t)((p.L - 1) * kPhasesPerLayer + PH_DOWN);
                    nw = p.aux + (size_t)p.L * p.aux_stride;
                    hidden = blockIdx.x == 0 ? p.hidden_out : nullptr;
                    break;
                }
                if (ok && norm_phase) in_ok = prologue_norm<MODE>(p, ny, ntag, nw, embed, hidden, pidx);
                if (!ok) break;
                (void)in_ok;  /* a failed read has raised the abort flag */
                if (threadIdx.x == 0) *sm_decision() = (*sm_abort_flag() == 0) ? 1 : 0;
                named_sync(1, kConsumerThreads);
                if (*sm_decision() == 0) { ok = false; break; }
                if (threadIdx.x == 0) trace_put(p, pidx, 2);
                const uint32_t tag_out = tag_base + (uint32_t)ph;
                /* chunks of this phase: warp w takes every 8th. A warp that
                 * gives up (abort) skips its remaining chunks but keeps walking
                 * the schedule, so all consumer warps meet the same named
                 * barriers; the stop is taken uniformly at the next phase. */
                /* chunk kk of this phase is chunk first + kk of layer l's
                 * schedule (the LM head is layer L) */
                const uint32_t first = (ph == PH_LM) ? 0u : sm_shape()[ph * 8 + 5];
                uint32_t kk = 0;
#pragma unroll 1
                for (uint32_t u = g.u0; u < g.u1; u += g.upc, ++seq, ++kk) {
                    if ((int)(seq % kConsumerWarps) != warp) continue;
                    if (*sm_abort_flag()) continue;
                    const uint32_t n = (g.u1 - u) < g.upc ? (g.u1 - u) : g.upc;
                    const uint32_t slot = seq % kSlots;
                    /* the slot's next chunk, kSlots further on (resolved by lane 0
                     * now, issued once the slot has been read) */
                    RefillDesc refill;
                    refill.bytes = 0;
                    if (lane == 0) refill = prepare_refill(p, Refill{(uint32_t)l, first + kk + kSlots, slot, seq / kSlots + 2u});
                    const uint8_t *buf = sm_ring() + (size_t)slot * kSlotBytes;

                    /* per-row side inputs, fetched before waiting for the chunk */
                    float4 tail = make_float4(0.f, 0.f, 0.f, 0.f), cw = tail;
                    int row_kind = -1;
                    if (ph == PH_QKVG && lane < (int)n) {
                        const uint32_t r = u + lane;
                        if (r < 3u * p.H) {
                            row_kind = (int)(r / (uint32_t)p.H);
                            const uint32_t d = r - (uint32_t)row_kind * p.H;
                            tail = __ldcg(reinterpret_cast<const float4 *>(
                                p.tails + (((size_t)l * 3 + row_kind) * p.H + d) * 4));
                            cw = __ldg(reinterpret_cast<const float4 *>(
                                aux + 2 * p.H + kHeadDim + ((size_t)row_kind * p.H + d) * 4));
                        }
                    }
                    float vv = 0.0f;
                    if (ph == PH_STATE && lane < (int)n)
                        xread1<(MODE & 4) != 0>(p, xw<MODE>(p.qkv) + 2 * p.H + u + lane, tag_base + PH_QKVG, vv);

                    if (!wait_full(p, seq)) continue;

                    if (ph == PH_STATE) {
                        state_chunk<MODE>(p, buf, u, n, h0, l, vv, tag_out);
                    } else {
                        const int K = (ph == PH_DOWN) ? p.I : p.H;
                        float out[4];
                        unsigned tiny = 0;
                        if (ph == PH_QKVG) {
                            for (uint32_t j = 0; j < n; ++j)
                                if (u + j >= 4u * p.H) tiny |= 1u << j;
                        }
                        warp_dot<MODE>(buf, K, (int)((ph == PH_GU) ? 2 * n : n), tiny, sm_xs(),
                                       sm_chain() + warp * 512, refill, out);
                        float y = out[0];
                        if (lane == 1) y = out[1];
                        if (lane == 2) y = out[2];
                        if (lane == 3) y = out[3];
                        const bool drop = (int)cta == p.test_drop_cta && pidx == p.test_drop_phase;
                        switch (drop ? -1 : ph) {
                        case PH_QKVG:
                            if (lane < (int)n) {
                                const uint32_t r = u + lane;
                                const float raw = bnd<MODE>(y);
                                if (row_kind >= 0) {
                                    /* depthwise conv over [t0 t1 t2 new] + SiLU, left to right
                                     * (c_impl/gdn_model.cpp:1630-1650), then the window shift */
                                    const float sum = __fadd_rn(
                                        __fadd_rn(__fadd_rn(__fmul_rn(tail.x, cw.x), __fmul_rn(tail.y, cw.y)),
                                                  __fmul_rn(tail.z, cw.z)),
                                        __fmul_rn(raw, cw.w));
                                    xput<MODE>(p, p.qkv, r, bnd<MODE>(silu_ref(sum)), tag_out);
                                    const uint32_t d = r - (uint32_t)row_kind * p.H;
                                    __stcg(reinterpret_cast<float4 *>(
                                               p.tails + (((size_t)l * 3 + row_kind) * p.H + d) * 4),
                                           make_float4(tail.y, tail.z, raw, 0.0f));
                                } else if (r < 4u * p.H) {
                                    xput<MODE>(p, p.gate, r - 3u * p.H, raw, tag_out);
                                } else {
                                    xput<MODE>(p, p.ab, r - 4u * p.H, raw, tag_out);
                                }
                            }
                            break;
                        case PH_O:
                            if (lane < (int)n) xput<MODE>(p, p.y_o, u + lane, bnd<MODE>(y), tag_out);
                            break;
                        case PH_DOWN:
                            if (lane < (int)n) xput<MODE>(p, p.y_down, u + lane, bnd<MODE>(y), tag_out);
                            break;
                        case PH_GU: {
                            /* rows [g_u, u_u, g_u+1, u_u+1]; SwiGLU as c_impl/gdn_model.cpp:4751-4770 */
                            const float gv = bnd<MODE>(lane == 0 ? out[0] : out[2]);
                            const float uv = bnd<MODE>(lane == 0 ? out[1] : out[3]);
                            if (lane < (int)n) xput<MODE>(p, p.m, u + lane, bnd<MODE>(__fmul_rn(silu_ref(gv), uv)), tag_out);
                            break;
                        }
                        case -1: /* outputs left out on purpose (test hook) */
                            break;
                        default:
                            if (lane < (int)n) {
                                p.logits[u + lane] = y;
                                if (MODE & 4)
                                    for (int r = 0; r < p.tp_world; ++r)
                                        if (r != p.tp_rank) *peer_addr(p, p.logits + u + lane, r) = y;
                            }
#pragma unroll
                            for (int j = 0; j < 4; ++j) {
                                if (j < (int)n && out[j] > best) {
                                    best = out[j];
                                    best_i = (int32_t)(u + j);
                                }
                            }
                            break;
                        }
                    }
                    __syncwarp();
                    if (ph == PH_STATE && lane == 0) issue_refill(refill);
                }
                if (threadIdx.x == 0) trace_put(p, pidx, 3);
            }
        }

        /* LM-head argmax: warps -> CTA candidate -> the last CTA picks the token */
        named_sync(1, kConsumerThreads);
        if (threadIdx.x == 0) *sm_decision() = (ok && *sm_abort_flag() == 0) ? 1 : 0;
        named_sync(1, kConsumerThreads);
        if (*sm_decision() != 0) {
            if (lane == 0) {
                sm_wbest()[warp] = best;
                sm_wbest_i()[warp] = best_i;
            }
            named_sync(1, kConsumerThreads);
            if (threadIdx.x == 0) {
                float b = sm_wbest()[0];
                int32_t bi = sm_wbest_i()[0];
                for (int w = 1; w < kConsumerWarps; ++w) {
                    const float v = sm_wbest()[w];
                    const int32_t vi = sm_wbest_i()[w];
                    if (v > b || (v == b && vi < bi)) { b = v; bi = vi; }
                }
                p.cand_val[blockIdx.x] = b;
                p.cand_idx[blockIdx.x] = bi;
                /* tensor-parallel: the logits this CTA stored into the peers'
                 * regions are visible there before its GPU's candidate is */
                if (MODE & 4) __threadfence_system();
                else __threadfence();
                const uint32_t ticket = atomicAdd(&p.status->done, 1u);
                if (ticket == gridDim.x - 1) {
                    __threadfence();
                    float gb = __ldcg(p.cand_val);
                    int32_t gi = __ldcg(p.cand_idx);
                    for (uint32_t c = 1; c < gridDim.x; ++c) {
                        const float v = __ldcg(p.cand_val + c);
                        const int32_t vi = __ldcg(p.cand_idx + c);
                        if (v > gb || (v == gb && vi < gi)) { gb = v; gi = vi; }
                    }
                    if (MODE & 4) {
                        /* this GPU's candidate to every GPU, then all of them
                         * merged in rank order (strict >, lowest index on ties:
                         * the order of the CTAs does not matter) */
                        const uint32_t ctag = p.epoch;
                        const unsigned long long wv = ((unsigned long long)ctag << 32) | __float_as_uint(gb);
                        const unsigned long long wi = ((unsigned long long)ctag << 32) | (uint32_t)gi;
                        __threadfence_system();
                        unsigned long long *mine = p.rank_cand + 2 * p.tp_rank;
                        for (int r = 0; r < p.tp_world; ++r) {
                            unsigned long long *dst = r == p.tp_rank ? mine : peer_addr(p, mine, r);
                            xstore_sys(dst, wv);
                            xstore_sys(dst + 1, wi);
                        }
                        for (int r = 0; r < p.tp_world; ++r) {
                            const unsigned long long v = xwait<true>(p, p.rank_cand + 2 * r, ctag);
                            const unsigned long long vi = xwait<true>(p, p.rank_cand + 2 * r + 1, ctag);
                            if (!xtag_is(v, ctag) || !xtag_is(vi, ctag)) break;  /* error raised */
                            const float fv = xval(v);
                            const int32_t iv = (int32_t)(uint32_t)vi;
                            if (r == 0 || fv > gb || (fv == gb && iv < gi)) { gb = fv; gi = iv; }
                        }
                        /* the peers' logits, released before their candidates */
                        __threadfence_system();
                    }
                    p.status->token = gi;
                    if (p.token_out != nullptr) *p.token_out = gi;
                    p.status->token_line[0] = (float)gi;
                    for (int i = 1; i < 16; ++i) p.status->token_line[i] = 0.0f;
                    p.status->done = 0u;
                }
            }
        }
    }
    __syncthreads();
    /* Every bulk copy issued into the ring must land before the CTA exits
     * (only a CTA that gave up mid-schedule can have one in flight; each
     * slot has at most one, its latest). */
    if (threadIdx.x == 0) {
        for (int i = 0; i < kSlots; ++i) {
            const uint32_t n = sm_issued()[i];
            if (n == 0) continue;
            const uint32_t bar = smem_u32(&sm_full()[i]);
            const uint64_t t0 = gtimer();
            while (!mbar_try(bar, (n - 1) & 1u))
                if (gtimer() - t0 > kWaitNs) break;
        }
    }
}

template <int MODE>
static cudaError_t launch_mode(const DecodeParams &p, int grid, cudaStream_t stream, size_t smem) {
    void *args[] = {const_cast<DecodeParams *>(&p)};
    const cudaError_t e =
        cudaFuncSetAttribute(gdn_decode_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    return cudaLaunchCooperativeKernel((const void *)gdn_decode_kernel<MODE>, dim3(grid), dim3(kThreads), args, smem,
                                       stream);
}

/* MODE bit 0: BF16 boundaries; bit 1: BF16-rounded products (needs bit 0); bit 2:
 * tensor-parallel decode. */
cudaError_t launch_decode(const DecodeParams &p, int grid, cudaStream_t stream) {
    const size_t smem = decode_smem_bytes(p.H, p.I);
    if (!p.bf16_boundary && p.native_product) return cudaErrorInvalidValue;
    /* MODE bit 2: tensor-parallel decode (peer stores, system-scope exchange) */
    if (p.tp_world > 1) {
        if (!p.bf16_boundary) return launch_mode<4>(p, grid, stream, smem);
        return p.native_product ? launch_mode<7>(p, grid, stream, smem) : launch_mode<5>(p, grid, stream, smem);
    }
    if (!p.bf16_boundary) return launch_mode<0>(p, grid, stream, smem);
    return p.native_product ? launch_mode<3>(p, grid, stream, smem) : launch_mode<1>(p, grid, stream, smem);
}

}  // namespace gdn
