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
 *     token schedule of weight / state chunks and streams each chunk into a
 *     12-slot shared-memory ring with cp.async.bulk (TMA bulk copies,
 *     mbarrier completion, evict-first L2 policy for weights). Weights do
 *     not depend on activations, so the producer runs ahead across phase
 *     boundaries while the consumers wait at grid barriers;
 *   - warps 0..7 are consumers: per phase they pass a grid barrier, build the
 *     phase's input vector in shared memory (residual add + RMSNorm, output
 *     norm x swish gate, ...), then each warp takes every 8th chunk: 16-byte
 *     vector reads of BF16 weights, FP32 FMA, butterfly warp reductions, and
 *     the phase's epilogue fused per row (short conv + SiLU + conv-window
 *     update, SwiGLU, LM-head logits + argmax).
 *
 * Phases per layer l: A QKVG+a/b rows, B state columns (gated delta rule),
 * C O rows, D gate/up row pairs, E down rows; after the last layer F LM head.
 * Five grid barriers per layer (none before layer 0's A).
 *
 * Every wait (mbarrier, grid barrier) is bounded by %globaltimer; on expiry
 * the kernel records an error in DecodeStatus, stops issuing copies, waits
 * for the copies already in flight and returns. The host reports -1.
 */
#include "gdn_engine.h"

#include <cuda_runtime.h>
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
template <bool BF16B>
__device__ __forceinline__ float bnd(float v) {
    return BF16B ? bf16_round(v) : v;
}

/* gdn_sigmoid / gdn_softplus with IEEE single-rounding operations
 * (c_impl/gdn_model.cpp:1307-1330). */
__device__ __forceinline__ float sigmoid_ref(float x) {
    if (x >= 0.0f) {
        const float z = expf(-x);
        return __fdiv_rn(1.0f, __fadd_rn(1.0f, z));
    }
    const float z = expf(x);
    return __fdiv_rn(z, __fadd_rn(1.0f, z));
}
__device__ __forceinline__ float silu_ref(float x) { return __fmul_rn(x, sigmoid_ref(x)); }
__device__ __forceinline__ float softplus_ref(float x) {
    if (x > 20.0f) return x;
    if (x < -20.0f) return expf(x);
    return log1pf(expf(x));
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

/* Shared-memory position of input column c: lane l of a 256-column step
 * reads its 8 columns as two float4 that are contiguous across lanes. */
__device__ __forceinline__ int xs_pos(int c) {
    const int s = c >> 8, w = c & 255, l = w >> 3, j = w & 7;
    return (s << 8) + (j < 4 ? (l << 2) + j : 128 + (l << 2) + (j - 4));
}

/* ------------------------------------------------------------ schedule */

struct Geom {
    const uint8_t *src;
    uint32_t unit_bytes, upc, u0, u1;
};

enum { PH_QKVG = 0, PH_STATE = 1, PH_O = 2, PH_GU = 3, PH_DOWN = 4, PH_LM = 5 };

__device__ __forceinline__ Geom geom(const DecodeParams &p, int l, int ph, uint32_t cta, uint32_t ncta) {
    Geom g;
    uint32_t total;
    const uint8_t *lw = p.wimg + (size_t)l * p.layer_stride;
    const uint32_t rowH = 2u * (uint32_t)p.H;
    uint32_t rpcH = (uint32_t)kSlotBytes / rowH;
    if (rpcH > (uint32_t)kMaxRowsPerChunk) rpcH = kMaxRowsPerChunk;
    switch (ph) {
    case PH_QKVG:
        total = 4u * p.H + 2u * p.nh;
        g.src = lw;
        g.unit_bytes = rowH;
        g.upc = rpcH;
        break;
    case PH_STATE:
        total = (uint32_t)p.nh * kHeadDim;
        g.src = reinterpret_cast<const uint8_t *>(p.S + (size_t)l * p.nh * kHeadDim * kHeadDim);
        g.unit_bytes = kHeadDim * 4u;
        g.upc = kColsPerChunk;
        break;
    case PH_O:
        total = (uint32_t)p.H;
        g.src = lw + p.off_o;
        g.unit_bytes = rowH;
        g.upc = rpcH;
        break;
    case PH_GU:
        total = (uint32_t)p.I;
        g.src = lw + p.off_gu;
        g.unit_bytes = 2u * rowH;
        g.upc = rpcH / 2u > 0 ? rpcH / 2u : 1u;
        break;
    case PH_DOWN: {
        total = (uint32_t)p.H;
        g.src = lw + p.off_down;
        g.unit_bytes = 2u * (uint32_t)p.I;
        uint32_t r = (uint32_t)kSlotBytes / g.unit_bytes;
        g.upc = r > (uint32_t)kMaxRowsPerChunk ? (uint32_t)kMaxRowsPerChunk : (r > 0 ? r : 1u);
        break;
    }
    default:
        total = (uint32_t)p.V;
        g.src = p.w_lm;
        g.unit_bytes = rowH;
        g.upc = rpcH;
        break;
    }
    g.u0 = (uint32_t)(((uint64_t)cta * total) / ncta);
    g.u1 = (uint32_t)(((uint64_t)(cta + 1) * total) / ncta);
    return g;
}

/* ------------------------------------------------------- shared memory */

struct Smem {
    uint8_t *ring;
    float *xs;        /* permuted phase input, max(H, I) floats */
    float *qn, *kn;   /* [2][256] normalised q/k of the CTA's (at most two) heads */
    float *red;       /* [8 warps][8 values] reduction scratch */
    float *hscal;     /* [2][4]: alpha, beta, decay per local head */
    float *wbest;     /* [8] */
    int32_t *wbest_i; /* [8] */
    uint64_t *full, *empty;
    volatile int32_t *abort_flag;  /* set by any thread of the CTA that gives up */
    volatile int32_t *decision;    /* thread 0's CTA-uniform go/stop, read after a barrier */
};

__device__ __forceinline__ Smem carve(uint8_t *base, int H, int I) {
    Smem s;
    size_t off = 0;
    s.ring = base;
    off += (size_t)kSlots * kSlotBytes;
    s.xs = reinterpret_cast<float *>(base + off);
    off += (size_t)4 * (H > I ? H : I);
    s.qn = reinterpret_cast<float *>(base + off);
    off += 2 * kHeadDim * 4;
    s.kn = reinterpret_cast<float *>(base + off);
    off += 2 * kHeadDim * 4;
    s.red = reinterpret_cast<float *>(base + off);
    off += 64 * 4;
    s.hscal = reinterpret_cast<float *>(base + off);
    off += 8 * 4;
    s.wbest = reinterpret_cast<float *>(base + off);
    off += 8 * 4;
    s.wbest_i = reinterpret_cast<int32_t *>(base + off);
    off += 8 * 4;
    off = (off + 7) & ~(size_t)7;
    s.full = reinterpret_cast<uint64_t *>(base + off);
    off += kSlots * 8;
    s.empty = reinterpret_cast<uint64_t *>(base + off);
    off += kSlots * 8;
    s.abort_flag = reinterpret_cast<volatile int32_t *>(base + off);
    s.decision = reinterpret_cast<volatile int32_t *>(base + off + 4);
    return s;
}

size_t decode_smem_bytes(int H, int I) {
    size_t off = (size_t)kSlots * kSlotBytes + (size_t)4 * (H > I ? H : I) + 4 * kHeadDim * 4 + 64 * 4 +
                 8 * 4 * 3;
    off = (off + 7) & ~(size_t)7;
    off += 2 * kSlots * 8 + 16;
    return off;
}

/* --------------------------------------------------- block-level helpers */

/* Deterministic sum over the 256 consumer threads of N values each: warp
 * butterfly, then a fixed pairwise tree over the 8 warps. */
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

/* Grid barrier among the consumer warps of all CTAs. Returns false when the
 * kernel is aborting (timeout here or an error raised by another CTA). The
 * answer is decided by thread 0 and published through s.decision before the
 * closing barrier, so every consumer thread sees the same value even if the
 * producer raises the abort flag meanwhile. */
__device__ bool grid_sync(const DecodeParams &p, uint32_t index, const Smem &s) {
    named_sync(1, kConsumerThreads);
    if (threadIdx.x == 0 && *s.abort_flag == 0) {
        const uint32_t target = p.bar_base + (index + 1u) * gridDim.x;
        __threadfence();
        atomicAdd(&p.status->bar, 1u);
        uint64_t t0 = 0;
        uint32_t spins = 0;
        while (true) {
            const uint32_t v = ld_acquire(&p.status->bar);
            if ((int32_t)(v - target) >= 0) break;
            if ((++spins & 255u) == 0) {
                if (ld_volatile_i32(&p.status->err) != 0) {
                    *s.abort_flag = 1;
                    break;
                }
                const uint64_t now = gtimer();
                if (t0 == 0) t0 = now;
                else if (now - t0 > kWaitNs) {
                    if (atomicCAS(&p.status->err, 0, kErrBarrierTimeout) == 0) {
                        p.status->err_cta = blockIdx.x;
                        p.status->err_where = index;
                    }
                    *s.abort_flag = 1;
                    break;
                }
            }
        }
        __threadfence();
    }
    if (threadIdx.x == 0) *s.decision = (*s.abort_flag == 0) ? 1 : 0;
    named_sync(1, kConsumerThreads);
    return *s.decision != 0;
}

/* Wait for a ring slot to be filled; false on abort. */
__device__ __forceinline__ bool wait_full(const DecodeParams &p, const Smem &s, uint32_t slot, uint32_t parity) {
    const uint32_t bar = smem_u32(&s.full[slot]);
    if (mbar_try(bar, parity)) return true;
    const uint64_t t0 = gtimer();
    while (true) {
        if (mbar_try(bar, parity)) return true;
        if (*s.abort_flag) return false;
        if (gtimer() - t0 > kWaitNs) {
            if (atomicCAS(&p.status->err, 0, kErrChunkTimeout) == 0) {
                p.status->err_cta = blockIdx.x;
                p.status->err_where = slot;
            }
            *s.abort_flag = 1;
            return false;
        }
    }
}

/* Dot products of up to 4 BF16 rows (contiguous in a ring slot) with the
 * permuted input vector; every lane returns all sums. */
__device__ __forceinline__ void warp_dot(const uint8_t *slot, int K, int nrows, const float *xs, float (&out)[4]) {
    const int lane = threadIdx.x & 31;
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    const int steps = K >> 8;
    for (int st = 0; st < steps; ++st) {
        const float4 xa = *reinterpret_cast<const float4 *>(xs + (st << 8) + (lane << 2));
        const float4 xb = *reinterpret_cast<const float4 *>(xs + (st << 8) + 128 + (lane << 2));
        const int col = (st << 8) + (lane << 3);
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            if (r < nrows) {
                const uint4 w = *reinterpret_cast<const uint4 *>(slot + ((size_t)r * K + col) * 2);
                float a = acc[r];
                a = fmaf(bf_lo(w.x), xa.x, a);
                a = fmaf(bf_hi(w.x), xa.y, a);
                a = fmaf(bf_lo(w.y), xa.z, a);
                a = fmaf(bf_hi(w.y), xa.w, a);
                a = fmaf(bf_lo(w.z), xb.x, a);
                a = fmaf(bf_hi(w.z), xb.y, a);
                a = fmaf(bf_lo(w.w), xb.z, a);
                a = fmaf(bf_hi(w.w), xb.w, a);
                acc[r] = a;
            }
        }
    }
#pragma unroll
    for (int r = 0; r < 4; ++r) out[r] = warp_sum(acc[r]);
}

/* ---------------------------------------------------------- prologues */

/* x = round(a + b) (or the embedding for layer 0), optional store of x,
 * then RMSNorm with weight w into the permuted shared input
 * (c_impl/gdn_model.cpp:3351-3452, 1394-1476). */
template <bool BF16B>
__device__ void prologue_residual_norm(const DecodeParams &p, const Smem &s, const float *a, const float *b,
                                       const float *w, float *x_store, bool embed) {
    const int t = threadIdx.x;
    const int H = p.H;
    const int per = H >> 8;
    float xv[8];
    float sq[1] = {0.0f};
    int32_t tok = -1;
    if (embed && p.token_src != nullptr) tok = *p.token_src;
    for (int j = 0; j < per; ++j) {
        const int i = t + (j << 8);
        float x;
        if (embed) {
            if (p.token_src != nullptr) {
                const uint16_t e = p.emb[(size_t)tok * H + i];
                x = __uint_as_float((uint32_t)e << 16);
            } else {
                x = p.x_embed[i];
            }
            x = bnd<BF16B>(x);
        } else {
            x = bnd<BF16B>(__fadd_rn(__ldcg(a + i), __ldcg(b + i)));
        }
        xv[j] = x;
        sq[0] = fmaf(x, x, sq[0]);
        if (x_store != nullptr) x_store[i] = x;
    }
    block_sum<1>(sq, s.red);
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sq[0], (float)H), p.eps)));
    for (int j = 0; j < per; ++j) {
        const int i = t + (j << 8);
        s.xs[xs_pos(i)] = bnd<BF16B>(__fmul_rn(__fmul_rn(xv[j], scale), __ldg(w + i)));
    }
}

/* Per-head RMSNorm of the attention output times swish(gate), into the
 * permuted shared input (c_impl/gdn_model.cpp:3226-3349). Element i = t +
 * 256 j belongs to head j. */
template <bool BF16B>
__device__ void prologue_norm_gate(const DecodeParams &p, const Smem &s, const float *o_norm) {
    const int t = threadIdx.x;
    float av[8], sq[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        sq[j] = 0.0f;
        av[j] = 0.0f;
        if (j < p.nh) {
            av[j] = __ldcg(p.attn + t + (j << 8));
            sq[j] = __fmul_rn(av[j], av[j]);
        }
    }
    block_sum<8>(sq, s.red);
    const float w = __ldg(o_norm + t);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        if (j < p.nh) {
            const int i = t + (j << 8);
            const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sq[j], 256.0f), p.eps)));
            const float g = __ldcg(p.gate + i);
            const float normalized = __fmul_rn(__fmul_rn(av[j], scale), w);
            s.xs[xs_pos(i)] = bnd<BF16B>(__fmul_rn(__fmul_rn(normalized, g), sigmoid_ref(g)));
        }
    }
}

/* q/k L2 norms (balanced tree order of gdn_tree_reduce_256), alpha, beta
 * and decay for the CTA's heads (c_impl/gdn_model.cpp:2059-2124). */
__device__ void prologue_state(const DecodeParams &p, const Smem &s, int l, int h0, int h1) {
    const int t = threadIdx.x;
    const float *aux = p.aux + (size_t)l * p.aux_stride;
    const float *a_log = aux + 14 * p.H + kHeadDim;
    const float *dt_bias = a_log + p.nh;
    for (int hs = 0; hs <= h1 - h0; ++hs) {
        const int h = h0 + hs;
        const float q = __ldcg(p.qkv + h * kHeadDim + t);
        const float k = __ldcg(p.qkv + p.H + h * kHeadDim + t);
        float v2[2] = {__fmul_rn(q, q), __fmul_rn(k, k)};
        block_sum<2>(v2, s.red);
        const float q_inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(v2[0], 1e-6f)));
        const float k_inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(v2[1], 1e-6f)));
        const float qn = __fmul_rn(q, q_inv), kn = __fmul_rn(k, k_inv);
        s.qn[hs * kHeadDim + t] = qn;
        s.kn[hs * kHeadDim + t] = kn;
        float al[1] = {__fmul_rn(qn, kn)};
        block_sum<1>(al, s.red);
        if (t == 0) {
            const float beta = sigmoid_ref(__ldcg(p.ab + p.nh + h));
            const float decay_in = __fadd_rn(__ldcg(p.ab + h), __ldg(dt_bias + h));
            const float decay_val = __fmul_rn(-expf(__ldg(a_log + h)), softplus_ref(decay_in));
            s.hscal[hs * 4 + 0] = al[0];
            s.hscal[hs * 4 + 1] = beta;
            s.hscal[hs * 4 + 2] = expf(decay_val);
        }
    }
    named_sync(1, kConsumerThreads);
}

/* ------------------------------------------------------------ the kernel */

template <bool BF16B>
__global__ void __launch_bounds__(kThreads, 1) gdn_decode_kernel(const DecodeParams p) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    const Smem s = carve(smem_raw, p.H, p.I);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t cta = blockIdx.x, ncta = gridDim.x;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kSlots; ++i) {
            mbar_init(smem_u32(&s.full[i]), 1);
            mbar_init(smem_u32(&s.empty[i]), 1);
        }
        *s.abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    if (warp == kConsumerWarps) {
        /* ------------------------------------------------ producer warp */
        if (lane == 0) {
            const uint64_t pol_w = policy_evict_first();
            const uint64_t pol_s = policy_evict_last();
            uint32_t seq = 0;
            bool ok = true;
            for (int l = 0; l <= p.L && ok; ++l) {
                const int nph = (l < p.L) ? kPhasesPerLayer : 1;
                for (int pi = 0; pi < nph && ok; ++pi) {
                    const int ph = (l < p.L) ? pi : PH_LM;
                    const Geom g = geom(p, l < p.L ? l : 0, ph, cta, ncta);
                    for (uint32_t u = g.u0; u < g.u1; u += g.upc, ++seq) {
                        const uint32_t n = (g.u1 - u) < g.upc ? (g.u1 - u) : g.upc;
                        const uint32_t slot = seq % kSlots;
                        if (seq >= (uint32_t)kSlots) {
                            const uint32_t bar = smem_u32(&s.empty[slot]);
                            const uint32_t par = ((seq / kSlots) + 1u) & 1u;
                            if (!mbar_try(bar, par)) {
                                const uint64_t t0 = gtimer();
                                while (!mbar_try(bar, par)) {
                                    if (*s.abort_flag) { ok = false; break; }
                                    if (gtimer() - t0 > kWaitNs) {
                                        if (atomicCAS(&p.status->err, 0, kErrSlotTimeout) == 0) {
                                            p.status->err_cta = cta;
                                            p.status->err_where = seq;
                                        }
                                        *s.abort_flag = 1;
                                        ok = false;
                                        break;
                                    }
                                }
                                if (!ok) break;
                            }
                        }
                        if (*s.abort_flag) { ok = false; break; }
                        const uint32_t bytes = n * g.unit_bytes;
                        const uint32_t fb = smem_u32(&s.full[slot]);
                        mbar_expect_tx(fb, bytes);
                        bulk_g2s(smem_u32(s.ring + (size_t)slot * kSlotBytes), g.src + (size_t)u * g.unit_bytes,
                                 bytes, fb, ph == PH_STATE ? pol_s : pol_w);
                    }
                }
            }
            /* Drain: every issued copy must land before the CTA may exit. */
            const uint32_t issued = seq;
            const uint32_t first = issued > (uint32_t)kSlots ? issued - kSlots : 0u;
            for (uint32_t q = first; q < issued; ++q) {
                const uint32_t bar = smem_u32(&s.full[q % kSlots]);
                const uint32_t par = (q / kSlots) & 1u;
                const uint64_t t0 = gtimer();
                while (!mbar_try(bar, par)) {
                    if (gtimer() - t0 > kWaitNs) break;
                }
            }
        }
        __syncwarp();
    } else {
        /* ---------------------------------------------- consumer warps */
        uint32_t seq = 0;
        uint32_t bar_index = 0;
        float best = -3.402823466e38f;
        int32_t best_i = 0;
        bool ok = true;
        for (int l = 0; l <= p.L && ok; ++l) {
            const int nph = (l < p.L) ? kPhasesPerLayer : 1;
            const float *aux = p.aux + (size_t)(l < p.L ? l : 0) * p.aux_stride;
            for (int pi = 0; pi < nph && ok; ++pi) {
                const int ph = (l < p.L) ? pi : PH_LM;
                const Geom g = geom(p, l < p.L ? l : 0, ph, cta, ncta);
                if (!(l == 0 && ph == PH_QKVG)) {
                    if (!grid_sync(p, bar_index++, s)) { ok = false; break; }
                }
                int h0 = 0, h1 = 0;
                /* phase input */
                switch (ph) {
                case PH_QKVG:
                    if (l == 0) {
                        if (p.token_src != nullptr) {
                            const int32_t tok = *p.token_src;
                            if (tok < 0 || tok >= p.V) {
                                /* every consumer thread reads the same token: uniform exit */
                                if (threadIdx.x == 0) {
                                    atomicCAS(&p.status->err, 0, kErrBadToken);
                                    *s.abort_flag = 1;
                                }
                                ok = false;
                                break;
                            }
                        }
                        prologue_residual_norm<BF16B>(p, s, nullptr, nullptr, aux, cta == 0 ? p.x_in : nullptr, true);
                    } else {
                        prologue_residual_norm<BF16B>(p, s, p.x_mid, p.y_down, aux, cta == 0 ? p.x_in : nullptr,
                                                      false);
                    }
                    break;
                case PH_STATE:
                    if (g.u1 > g.u0) {
                        h0 = (int)(g.u0 >> 8);
                        h1 = (int)((g.u1 - 1) >> 8);
                        prologue_state(p, s, l, h0, h1);
                    }
                    break;
                case PH_O:
                    prologue_norm_gate<BF16B>(p, s, aux + p.H);
                    break;
                case PH_GU:
                    prologue_residual_norm<BF16B>(p, s, p.x_in, p.y_o, aux + p.H + kHeadDim,
                                                  cta == 0 ? p.x_mid : nullptr, false);
                    break;
                case PH_DOWN:
                    for (int i = threadIdx.x; i < p.I; i += kConsumerThreads) s.xs[xs_pos(i)] = __ldcg(p.m + i);
                    break;
                default: {
                    const float *final_norm = p.aux + (size_t)p.L * p.aux_stride;
                    prologue_residual_norm<BF16B>(p, s, p.x_mid, p.y_down, final_norm, nullptr, false);
                    break;
                }
                }
                if (!ok) break;
                named_sync(1, kConsumerThreads);
                if (ph == PH_LM && cta == 0 && p.hidden_out != nullptr) {
                    for (int i = threadIdx.x; i < p.H; i += kConsumerThreads) p.hidden_out[i] = s.xs[xs_pos(i)];
                }

                /* chunks of this phase: warp w takes every 8th */
                /* A warp that gives up (abort) skips its remaining chunks but
                 * keeps walking the schedule, so that all consumer warps meet
                 * the same named barriers; the stop is taken uniformly at the
                 * next grid_sync. */
                for (uint32_t u = g.u0; u < g.u1; u += g.upc, ++seq) {
                    if ((int)(seq % kConsumerWarps) != warp) continue;
                    if (*s.abort_flag) continue;
                    const uint32_t n = (g.u1 - u) < g.upc ? (g.u1 - u) : g.upc;
                    const uint32_t slot = seq % kSlots;
                    const uint8_t *buf = s.ring + (size_t)slot * kSlotBytes;

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

                    if (!wait_full(p, s, slot, (seq / kSlots) & 1u)) continue;

                    if (ph == PH_STATE) {
                        for (uint32_t j = 0; j < n; ++j) {
                            const uint32_t c = u + j;
                            const int hs = (int)(c >> 8) - h0;
                            const float *col = reinterpret_cast<const float *>(buf) + j * kHeadDim + lane * 8;
                            const float4 s0 = *reinterpret_cast<const float4 *>(col);
                            const float4 s1 = *reinterpret_cast<const float4 *>(col + 4);
                            const float *qn = s.qn + hs * kHeadDim + lane * 8;
                            const float *kn = s.kn + hs * kHeadDim + lane * 8;
                            const float4 q0 = *reinterpret_cast<const float4 *>(qn);
                            const float4 q1 = *reinterpret_cast<const float4 *>(qn + 4);
                            const float4 k0 = *reinterpret_cast<const float4 *>(kn);
                            const float4 k1 = *reinterpret_cast<const float4 *>(kn + 4);
                            float r = 0.0f, pp = 0.0f;
                            r = fmaf(s0.x, k0.x, r); pp = fmaf(s0.x, q0.x, pp);
                            r = fmaf(s0.y, k0.y, r); pp = fmaf(s0.y, q0.y, pp);
                            r = fmaf(s0.z, k0.z, r); pp = fmaf(s0.z, q0.z, pp);
                            r = fmaf(s0.w, k0.w, r); pp = fmaf(s0.w, q0.w, pp);
                            r = fmaf(s1.x, k1.x, r); pp = fmaf(s1.x, q1.x, pp);
                            r = fmaf(s1.y, k1.y, r); pp = fmaf(s1.y, q1.y, pp);
                            r = fmaf(s1.z, k1.z, r); pp = fmaf(s1.z, q1.z, pp);
                            r = fmaf(s1.w, k1.w, r); pp = fmaf(s1.w, q1.w, pp);
                            r = warp_sum(r);
                            pp = warp_sum(pp);
                            const float alpha = s.hscal[hs * 4 + 0];
                            const float beta = s.hscal[hs * 4 + 1];
                            const float decay = s.hscal[hs * 4 + 2];
                            const float vv = __ldcg(p.qkv + 2 * p.H + c);
                            /* c_impl/gdn_model.cpp:2214-2243, 2268-2300 */
                            const float delta = __fmul_rn(beta, __fsub_rn(vv, __fmul_rn(decay, r)));
                            const float o = __fmul_rn(0.0625f, __fadd_rn(__fmul_rn(decay, pp), __fmul_rn(alpha, delta)));
                            if (lane == 0) p.attn[c] = bnd<BF16B>(o);
                            float4 n0, n1;
                            n0.x = __fadd_rn(__fmul_rn(decay, s0.x), __fmul_rn(k0.x, delta));
                            n0.y = __fadd_rn(__fmul_rn(decay, s0.y), __fmul_rn(k0.y, delta));
                            n0.z = __fadd_rn(__fmul_rn(decay, s0.z), __fmul_rn(k0.z, delta));
                            n0.w = __fadd_rn(__fmul_rn(decay, s0.w), __fmul_rn(k0.w, delta));
                            n1.x = __fadd_rn(__fmul_rn(decay, s1.x), __fmul_rn(k1.x, delta));
                            n1.y = __fadd_rn(__fmul_rn(decay, s1.y), __fmul_rn(k1.y, delta));
                            n1.z = __fadd_rn(__fmul_rn(decay, s1.z), __fmul_rn(k1.z, delta));
                            n1.w = __fadd_rn(__fmul_rn(decay, s1.w), __fmul_rn(k1.w, delta));
                            float *dst = p.S + ((size_t)l * p.nh * kHeadDim + c) * kHeadDim + lane * 8;
                            __stcg(reinterpret_cast<float4 *>(dst), n0);
                            __stcg(reinterpret_cast<float4 *>(dst + 4), n1);
                        }
                    } else {
                        const int K = (ph == PH_DOWN) ? p.I : p.H;
                        float out[4];
                        warp_dot(buf, K, (int)((ph == PH_GU) ? 2 * n : n), s.xs, out);
                        switch (ph) {
                        case PH_QKVG: {
                            float y = out[0];
                            if (lane == 1) y = out[1];
                            if (lane == 2) y = out[2];
                            if (lane == 3) y = out[3];
                            if (lane < (int)n) {
                                const uint32_t r = u + lane;
                                const float raw = bnd<BF16B>(y);
                                if (row_kind >= 0) {
                                    /* depthwise conv over [t0 t1 t2 new] + SiLU, left to right
                                     * (c_impl/gdn_model.cpp:1630-1650), then the window shift */
                                    const float sum = __fadd_rn(
                                        __fadd_rn(__fadd_rn(__fmul_rn(tail.x, cw.x), __fmul_rn(tail.y, cw.y)),
                                                  __fmul_rn(tail.z, cw.z)),
                                        __fmul_rn(raw, cw.w));
                                    p.qkv[r] = bnd<BF16B>(silu_ref(sum));
                                    const uint32_t d = r - (uint32_t)row_kind * p.H;
                                    __stcg(reinterpret_cast<float4 *>(
                                               p.tails + (((size_t)l * 3 + row_kind) * p.H + d) * 4),
                                           make_float4(tail.y, tail.z, raw, 0.0f));
                                } else if (r < 4u * p.H) {
                                    p.gate[r - 3u * p.H] = raw;
                                } else {
                                    p.ab[r - 4u * p.H] = raw;
                                }
                            }
                            break;
                        }
                        case PH_O:
                        case PH_DOWN: {
                            float y = out[0];
                            if (lane == 1) y = out[1];
                            if (lane == 2) y = out[2];
                            if (lane == 3) y = out[3];
                            if (lane < (int)n) (ph == PH_O ? p.y_o : p.y_down)[u + lane] = bnd<BF16B>(y);
                            break;
                        }
                        case PH_GU: {
                            /* rows [g_u, u_u, g_u+1, u_u+1]; SwiGLU as c_impl/gdn_model.cpp:4751-4770 */
                            const float gv = bnd<BF16B>(lane == 0 ? out[0] : out[2]);
                            const float uv = bnd<BF16B>(lane == 0 ? out[1] : out[3]);
                            if (lane < (int)n) p.m[u + lane] = bnd<BF16B>(__fmul_rn(silu_ref(gv), uv));
                            break;
                        }
                        default: {
                            float y = out[0];
                            if (lane == 1) y = out[1];
                            if (lane == 2) y = out[2];
                            if (lane == 3) y = out[3];
                            if (lane < (int)n) p.logits[u + lane] = y;
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
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive(smem_u32(&s.empty[slot]));
                }
            }
        }

        /* LM-head argmax: warps -> CTA candidate -> the last CTA picks the token */
        if (ok) {
            if (threadIdx.x == 0) *s.decision = (*s.abort_flag == 0) ? 1 : 0;
            named_sync(1, kConsumerThreads);
            ok = *s.decision != 0;
        }
        if (ok) {
            if (lane == 0) {
                s.wbest[warp] = best;
                s.wbest_i[warp] = best_i;
            }
            named_sync(1, kConsumerThreads);
            if (threadIdx.x == 0) {
                float b = s.wbest[0];
                int32_t bi = s.wbest_i[0];
                for (int w = 1; w < kConsumerWarps; ++w) {
                    const float v = s.wbest[w];
                    const int32_t vi = s.wbest_i[w];
                    if (v > b || (v == b && vi < bi)) { b = v; bi = vi; }
                }
                p.cand_val[cta] = b;
                p.cand_idx[cta] = bi;
                __threadfence();
                const uint32_t ticket = atomicAdd(&p.status->done, 1u);
                if (ticket == ncta - 1) {
                    __threadfence();
                    float gb = __ldcg(p.cand_val);
                    int32_t gi = __ldcg(p.cand_idx);
                    for (uint32_t c = 1; c < ncta; ++c) {
                        const float v = __ldcg(p.cand_val + c);
                        const int32_t vi = __ldcg(p.cand_idx + c);
                        if (v > gb || (v == gb && vi < gi)) { gb = v; gi = vi; }
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
}

cudaError_t launch_decode(const DecodeParams &p, int grid, cudaStream_t stream) {
    const size_t smem = decode_smem_bytes(p.H, p.I);
    void *args[] = {const_cast<DecodeParams *>(&p)};
    cudaError_t e;
    if (p.bf16_boundary) {
        e = cudaFuncSetAttribute(gdn_decode_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        return cudaLaunchCooperativeKernel((const void *)gdn_decode_kernel<true>, dim3(grid), dim3(kThreads), args,
                                           smem, stream);
    }
    e = cudaFuncSetAttribute(gdn_decode_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    return cudaLaunchCooperativeKernel((const void *)gdn_decode_kernel<false>, dim3(grid), dim3(kThreads), args,
                                       smem, stream);
}

}  // namespace gdn
