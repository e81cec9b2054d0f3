/* gdn_batch.cu -- the multi-stream decode engine's kernels (BASELINE
 * config[3]): B independent decode streams advance one token per step, and
 * every weight byte is read once per step for all of them.
 *
 * One step is, per layer (c_impl/gdn_model.cpp:3719-3897 for one stream):
 *   QKVGAB projection (tile GEMM, epilogue: causal conv + SiLU with the tail
 *     update, :1543-1660, :5113-5127)
 *   gated delta rule per (stream, head, 64 state columns) (:1932-2340)
 *   output norm x swish gate per (stream, head) (:3226-3349)
 *   O projection (tile GEMM, epilogue: residual add, :3351-3452)
 *   MLP RMSNorm per stream (:3379-3452)
 *   gate/up projection (tile GEMM, epilogue: SwiGLU, :4751-4770)
 *   down projection (tile GEMM, epilogue: residual add, :3836-3842)
 *   next RMSNorm per stream
 * then the LM head (tile GEMM, epilogue: FP32 logits and the strict-">"
 * lowest-index argmax per stream, :4775-4925).
 *
 * Tile GEMM (tcgen05): D[row][n] = sum_k W[row][k] x[n][k] for a 128-row tile
 * and all n streams of a pass, accumulated in TMEM. The (tile, 64-column
 * block) units of a projection are split evenly over the SMs (each CTA takes a
 * contiguous unit range, so a tile may be shared by two or three CTAs); a CTA
 * accumulates each of its tile segments in one of two TMEM buffers, and a
 * tile split over several CTAs is summed by the last CTA to finish it, in
 * k order (deterministic). Warp roles: one thread streams the weight blocks
 * (16 KB bulk copies, L2 evict-first) through an 8-10 slot ring, one streams
 * the activation blocks, one issues the MMAs (three per 16-column step: one
 * per BF16 term of the activations), and four warps drain TMEM and run the
 * epilogue while the next segment accumulates. Every wait is bounded (2 s) and
 * reports through the status word.
 */
#include "gdn_batch.h"

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace gdn {
namespace bt {

namespace {

constexpr uint64_t kWaitNs = 2000000000ull;
constexpr size_t kSmemLimit = 232448;  /* 227 KB per CTA */
constexpr size_t kSmemAlign = 1024;    /* the 128-byte swizzle repeats every 1 KB */
constexpr size_t kSmemTail = 512;      /* barriers and flags */

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
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
    asm volatile("barrier.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}
/* AND of v over the n threads of named barrier id (every one of them gets it) */
__device__ __forceinline__ bool named_all(int id, int n, bool v) {
    uint32_t r;
    asm volatile(
        "{\n"
        " .reg .pred p, q;\n"
        " setp.ne.u32 p, %1, 0;\n"
        " barrier.red.and.pred q, %2, %3, p;\n"
        " selp.u32 %0, 1, 0, q;\n"
        "}\n"
        : "=r"(r)
        : "r"((uint32_t)v), "r"(id), "r"(n)
        : "memory");
    return r != 0;
}

/* ---- tcgen05 ---- */

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

/* Shared-memory matrix descriptor, K-major operand in the 128-byte swizzle:
 * start address >> 4 (bits 0-13), leading byte offset 16 B (unused by this
 * layout, bits 16-29), stride byte offset 1024 B between 8-row groups (bits
 * 32-45), descriptor version 1 (bits 46-47), base offset 0, layout type 2 =
 * 128-byte swizzle (bits 61-63). */
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
    return (uint64_t)((addr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

/* Instruction descriptor of kind::f16: D FP32 (bits 4-5 = 1), A and B BF16
 * (bits 7-9 = 1, 10-12 = 1), both K-major, N >> 3 at bits 17-22, M >> 4 at
 * bits 24-28. */
__host__ __device__ constexpr uint32_t instr_desc(uint32_t m, uint32_t n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((n >> 3) << 17) | ((m >> 4) << 24);
}

__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n"
        " .reg .pred p;\n"
        " setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n"
        "}\n" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void tc_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}
/* 16 consecutive FP32 columns of this thread's TMEM lane */
__device__ __forceinline__ void tc_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    __syncwarp();
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
        "%14, %15}, [%16];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

/* ---- the reference's scalar functions (c_impl/gdn_model.cpp:1307-1330) ---- */

__device__ __forceinline__ float sigmoid_ref(float x) {
    if (x >= 0.0f) return __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-x)));
    const float z = expf(x);
    return __fdiv_rn(z, __fadd_rn(1.0f, z));
}
__device__ __forceinline__ float silu_ref(float x) { return __fmul_rn(x, sigmoid_ref(x)); }
__device__ __forceinline__ float softplus_ref(float x) {
    if (x > 20.0f) return x;
    if (x < -20.0f) return expf(x);
    return log1pf(expf(x));
}

/* ---- activation tiles ---- */

__device__ __forceinline__ size_t tile_off(uint32_t npad, uint32_t n, uint32_t k) {
    const uint32_t kb = k >> 6, kk = k & 63;
    return (size_t)kb * (kTerms * npad * 128u) + (size_t)n * 128u + ((((kk >> 3) ^ (n & 7u)) << 4) | ((kk & 7u) << 1));
}
/* v = h0 + h1 + h2 exactly (each residual of a rounding to BF16 is exact in FP32) */
__device__ __forceinline__ void split3(float v, uint16_t &h0, uint16_t &h1, uint16_t &h2) {
    const __nv_bfloat16 b0 = __float2bfloat16_rn(v);
    const float r1 = __fsub_rn(v, __bfloat162float(b0));
    const __nv_bfloat16 b1 = __float2bfloat16_rn(r1);
    const float r2 = __fsub_rn(r1, __bfloat162float(b1));
    const __nv_bfloat16 b2 = __float2bfloat16_rn(r2);
    h0 = __bfloat16_as_ushort(b0);
    h1 = __bfloat16_as_ushort(b1);
    h2 = __bfloat16_as_ushort(b2);
}
__device__ __forceinline__ void put_act(uint8_t *tiles, uint32_t npad, uint32_t n, uint32_t k, float v) {
    uint16_t h0, h1, h2;
    split3(v, h0, h1, h2);
    uint8_t *p = tiles + tile_off(npad, n, k);
    const size_t term = (size_t)npad * 128u;
    *reinterpret_cast<uint16_t *>(p) = h0;
    *reinterpret_cast<uint16_t *>(p + term) = h1;
    *reinterpret_cast<uint16_t *>(p + 2 * term) = h2;
}
/* eight consecutive k (k % 8 == 0) of stream n: one 16-byte chunk per term */
__device__ __forceinline__ void put_act8(uint8_t *tiles, uint32_t npad, uint32_t n, uint32_t k, const float (&v)[8]) {
    uint32_t w0[4], w1[4], w2[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        uint16_t a0, a1, a2, b0, b1, b2;
        split3(v[2 * i], a0, a1, a2);
        split3(v[2 * i + 1], b0, b1, b2);
        w0[i] = (uint32_t)a0 | ((uint32_t)b0 << 16);
        w1[i] = (uint32_t)a1 | ((uint32_t)b1 << 16);
        w2[i] = (uint32_t)a2 | ((uint32_t)b2 << 16);
    }
    uint8_t *p = tiles + tile_off(npad, n, k);
    const size_t term = (size_t)npad * 128u;
    *reinterpret_cast<uint4 *>(p) = make_uint4(w0[0], w0[1], w0[2], w0[3]);
    *reinterpret_cast<uint4 *>(p + term) = make_uint4(w1[0], w1[1], w1[2], w1[3]);
    *reinterpret_cast<uint4 *>(p + 2 * term) = make_uint4(w2[0], w2[1], w2[2], w2[3]);
}

__device__ __forceinline__ void report(uint32_t *status, uint32_t code, uint32_t where) {
    if (atomicCAS(status, 0u, code) == 0u) atomicExch(status + 1, where);
}

/* argmax key: larger value first, then the lower row; NaN never wins and -0
 * equals +0 (the reference's strict ">" scan from row 0) */
__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t row) {
    if (v != v) return 0ull;
    uint32_t b = __float_as_uint(v == 0.0f ? 0.0f : v);
    b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return ((unsigned long long)b << 32) | (unsigned long long)(0xFFFFFFFFu - row);
}

/* ---- unit partition of one projection ---- */

__host__ __device__ __forceinline__ uint32_t unit_start(uint32_t c, uint32_t units, uint32_t grid) {
    return (uint32_t)(((uint64_t)c * units) / grid);
}
/* the CTA whose range holds unit u: the largest c with unit_start(c) <= u */
__host__ __device__ __forceinline__ uint32_t unit_owner(uint32_t u, uint32_t units, uint32_t grid) {
    return (uint32_t)((((uint64_t)(u + 1) * grid) + units - 1) / units) - 1u;
}

/* shared-memory layout of the GEMM */
struct GemmSmem {
    uint32_t a0, b0, bblock;                 /* ring bases (shared addresses), B block bytes */
    uint32_t full_a, empty_a, full_b, empty_b, acc_full, acc_empty, drain;  /* barrier arrays */
    uint32_t *tmem_slot, *abort, *flag;
};

__device__ __forceinline__ bool wait_bar(uint32_t bar, uint32_t parity, volatile uint32_t *abort) {
    if (mbar_try(bar, parity)) return true;
    const uint64_t t0 = gtimer();
    while (true) {
        if (mbar_try(bar, parity)) return true;
        if (*abort) return false;
        if (gtimer() - t0 > kWaitNs) return false;
    }
}

/* The epilogue of y = D[row][n] of the pass; called by all 32 lanes of a warp
 * with the same n (rows r .. r + 31). */
__device__ __forceinline__ void epilogue(const GemmParams &p, float y, uint32_t n, uint32_t row, bool valid) {
    const float partner = __shfl_xor_sync(0xffffffffu, y, 1);
    const bool live = valid && n < p.nvalid;
    if (p.epi == kEpiLogits) {
        unsigned long long key = live ? argmax_key(y, row) : 0ull;
        if (live) p.out[(size_t)n * p.out_stride + row] = y;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
            key = other > key ? other : key;
        }
        if ((threadIdx.x & 31u) == 0 && n < p.nvalid && key != 0ull) atomicMax(p.keys + p.stream0 + n, key);
        return;
    }
    if (!live) return;
    switch (p.epi) {
        case kEpiStore:
            p.out[(size_t)n * p.out_stride + row] = y;
            break;
        case kEpiResid: {
            float *r = p.out + (size_t)n * p.out_stride + row;
            *r = __fadd_rn(*r, y);
            break;
        }
        case kEpiQKV: {
            const uint32_t H = p.hidden;
            float v = y;
            if (row < 3 * H) {
                /* window = [t0, t1, t2, new], summed left to right (:1543-1660) */
                const uint32_t kind = row / H, ch = row - kind * H;
                const float4 w = reinterpret_cast<const float4 *>(p.conv_w)[(size_t)kind * H + ch];
                float *t = p.tails + (size_t)n * p.tails_stride + (size_t)kind * 3 * H + ch;
                const float t0 = t[0], t1 = t[H], t2 = t[2 * H];
                float sum = __fadd_rn(__fmul_rn(t0, w.x), __fmul_rn(t1, w.y));
                sum = __fadd_rn(sum, __fmul_rn(t2, w.z));
                sum = __fadd_rn(sum, __fmul_rn(y, w.w));
                v = silu_ref(sum);
                t[0] = t1;
                t[H] = t2;
                t[2 * H] = y;
            }
            p.out[(size_t)n * p.out_stride + row] = v;
            break;
        }
        case kEpiSwiGLU:
            /* row 2i = gate_i, row 2i + 1 = up_i (:4751-4770) */
            if ((row & 1u) == 0) put_act(p.next_b, p.npad, n, row >> 1, __fmul_rn(silu_ref(y), partner));
            break;
        default:
            break;
    }
}

__global__ void __launch_bounds__(kGemmThreads, 1) tile_gemm_kernel(const __grid_constant__ GemmParams p) {
    extern __shared__ uint8_t dsm_raw[];
    const uint32_t raw = smem_u32(dsm_raw);
    const uint32_t pad = (uint32_t)((kSmemAlign - (raw & (kSmemAlign - 1))) & (kSmemAlign - 1));
    uint8_t *dsm = dsm_raw + pad;
    const uint32_t base = raw + pad;
    const uint32_t SA = p.a_slots, SB = p.b_slots;
    GemmSmem s;
    s.bblock = kTerms * p.npad * 128u;
    s.a0 = base;
    s.b0 = base + SA * (uint32_t)kABlockBytes;
    const uint32_t bars = s.b0 + SB * s.bblock;
    s.full_a = bars;
    s.empty_a = s.full_a + 8 * SA;
    s.full_b = s.empty_a + 8 * SA;
    s.empty_b = s.full_b + 8 * SB;
    s.acc_full = s.empty_b + 8 * SB;
    s.acc_empty = s.acc_full + 16;
    s.drain = s.acc_empty + 16;
    uint8_t *tail = dsm + (s.drain + 8 - base);
    s.tmem_slot = reinterpret_cast<uint32_t *>(tail);
    s.abort = reinterpret_cast<uint32_t *>(tail + 4);
    s.flag = reinterpret_cast<uint32_t *>(tail + 8);
    volatile uint32_t *abort = s.abort;

    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t units = p.mtiles * p.kblocks, G = gridDim.x, c = blockIdx.x;
    const uint32_t u0 = unit_start(c, units, G), u1 = unit_start(c + 1, units, G);
    const uint32_t KB = p.kblocks;
    uint32_t acc_cols = 32;  /* a power of two >= npad: both buffers start aligned */
    while (acc_cols < p.npad) acc_cols <<= 1;
    const uint32_t ncols = 2 * acc_cols;

    if (tid == 0) {
        for (uint32_t i = 0; i < SA; ++i) {
            mbar_init(s.full_a + 8 * i, 1);
            mbar_init(s.empty_a + 8 * i, 1);
        }
        for (uint32_t i = 0; i < SB; ++i) {
            mbar_init(s.full_b + 8 * i, 1);
            mbar_init(s.empty_b + 8 * i, 1);
        }
        for (uint32_t i = 0; i < 2; ++i) {
            mbar_init(s.acc_full + 8 * i, 1);
            mbar_init(s.acc_empty + 8 * i, 128);
        }
        mbar_init(s.drain, 1);
        *s.abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
        __syncwarp();
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(s.tmem_slot)),
                     "r"(ncols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *s.tmem_slot;

    if (warp == 4) {
        /* weight blocks: unit u is the u-th 16 KB block of the tile image */
        if (lane == 0) {
            const uint64_t pol = policy_evict_first();
            uint32_t i = 0;
            for (uint32_t u = u0; u < u1; ++u, ++i) {
                const uint32_t sl = i % SA;
                if (i >= SA && !wait_bar(s.empty_a + 8 * sl, ((i / SA) - 1) & 1u, abort)) {
                    if (!*abort) report(p.status, kErrWaitA, c);
                    *abort = 1;
                    break;
                }
                mbar_expect_tx(s.full_a + 8 * sl, kABlockBytes);
                bulk_g2s(s.a0 + sl * kABlockBytes, p.a + (size_t)u * kABlockBytes, kABlockBytes, s.full_a + 8 * sl,
                         pol);
            }
            /* copies already issued land before the CTA exits (an abort does not stop them) */
            for (uint32_t j = i > SA ? i - SA : 0; j < i; ++j) {
                const uint64_t t0 = gtimer();
                while (!mbar_try(s.full_a + 8 * (j % SA), (j / SA) & 1u) && gtimer() - t0 < kWaitNs) {
                }
            }
        }
    } else if (warp == 5) {
        /* activation blocks: k-block u % KB of the pass's tiles */
        if (lane == 0) {
            const uint64_t pol = policy_evict_last();
            uint32_t i = 0;
            for (uint32_t u = u0; u < u1; ++u, ++i) {
                const uint32_t sl = i % SB;
                if (i >= SB && !wait_bar(s.empty_b + 8 * sl, ((i / SB) - 1) & 1u, abort)) {
                    if (!*abort) report(p.status, kErrWaitB, c);
                    *abort = 1;
                    break;
                }
                mbar_expect_tx(s.full_b + 8 * sl, s.bblock);
                bulk_g2s(s.b0 + sl * s.bblock, p.b + (size_t)(u % KB) * s.bblock, s.bblock, s.full_b + 8 * sl, pol);
            }
            const uint32_t lo = i > SB ? i - SB : 0;
            for (uint32_t j = lo; j < i; ++j) {
                const uint64_t t0 = gtimer();
                while (!mbar_try(s.full_b + 8 * (j % SB), (j / SB) & 1u) && gtimer() - t0 < kWaitNs) {
                }
            }
        }
    } else if (warp == 6) {
        if (lane == 0) {
            const uint32_t idesc = instr_desc(kTileM, p.npad);
            const uint32_t term_bytes = p.npad * 128u;
            uint32_t i = 0, seg = 0;
            bool ok = true;
            for (uint32_t t = u0 / KB; ok && t * KB < u1; ++t, ++seg) {
                const uint32_t ua = max(u0, t * KB), ub = min(u1, (t + 1) * KB);
                const uint32_t acc = seg & 1u;
                if (seg >= 2 && !wait_bar(s.acc_empty + 8 * acc, ((seg >> 1) - 1) & 1u, abort)) {
                    if (!*abort) report(p.status, kErrWaitAcc, c);
                    *abort = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t d = tmem + acc * acc_cols;
                for (uint32_t u = ua; u < ub; ++u, ++i) {
                    const uint32_t sa = i % SA, sb = i % SB;
                    if (!wait_bar(s.full_a + 8 * sa, (i / SA) & 1u, abort) ||
                        !wait_bar(s.full_b + 8 * sb, (i / SB) & 1u, abort)) {
                        if (!*abort) report(p.status, kErrWaitMma, c);
                        *abort = 1;
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t abase = s.a0 + sa * kABlockBytes, bbase = s.b0 + sb * s.bblock;
#pragma unroll
                    for (uint32_t term = 0; term < kTerms; ++term) {
#pragma unroll
                        for (uint32_t kk = 0; kk < kTileK / 16; ++kk) {
                            const uint64_t ad = smem_desc(abase + kk * 32u);
                            const uint64_t bd = smem_desc(bbase + term * term_bytes + kk * 32u);
                            tc_mma(d, ad, bd, idesc, (u == ua && term == 0 && kk == 0) ? 0u : 1u);
                        }
                    }
                    tc_commit(s.empty_a + 8 * sa);
                    tc_commit(s.empty_b + 8 * sb);
                }
                if (ok) tc_commit(s.acc_full + 8 * acc);
            }
            /* every MMA issued has completed before TMEM is released */
            tc_commit(s.drain);
            const uint64_t t0 = gtimer();
            while (!mbar_try(s.drain, 0) && gtimer() - t0 < kWaitNs) {
            }
        }
    } else {
        /* warps 0-3: TMEM lanes 32w .. 32w + 31 = rows of the tile */
        const uint32_t r = tid;  /* 0..127 */
        uint32_t seg = 0;
        for (uint32_t t = u0 / KB; t * KB < u1; ++t, ++seg) {
            const uint32_t ua = max(u0, t * KB), ub = min(u1, (t + 1) * KB);
            const uint32_t acc = seg & 1u;
            const bool whole = (ua == t * KB) && (ub == (t + 1) * KB);
            const uint32_t row = t * kTileM + r;
            const bool valid = row < p.m;
            /* the 128 epilogue threads leave together or not at all */
            const bool got = wait_bar(s.acc_full + 8 * acc, (seg >> 1) & 1u, abort);
            if (!named_all(1, 128, got)) {
                if (!got && !*abort) report(p.status, kErrWaitAcc, c);
                *abort = 1;
                break;
            }
            tc_fence_after();
            const uint32_t taddr = tmem + acc * acc_cols + ((warp * 32u) << 16);
            const uint32_t local = t - u0 / KB;
            float *slot = p.partial + ((size_t)c * p.max_local + local) * p.npad * kTileM;
            for (uint32_t c0 = 0; c0 < p.npad; c0 += 16) {
                float v[16];
                tc_ld16(taddr + c0, v);
                if (whole) {
#pragma unroll
                    for (int j = 0; j < 16; ++j) epilogue(p, v[j], c0 + j, row, valid);
                } else {
#pragma unroll
                    for (int j = 0; j < 16; ++j) slot[(size_t)(c0 + j) * kTileM + r] = v[j];
                }
            }
            tc_fence_before();
            mbar_arrive(s.acc_empty + 8 * acc);
            if (whole) continue;
            /* split tile: the last of its CTAs sums the segments in k order */
            __threadfence();
            named_sync(1, 128);
            if (r == 0) {
                const uint32_t cf = unit_owner(t * KB, units, G), cl = unit_owner(t * KB + KB - 1, units, G);
                const uint32_t prev = atomicAdd(p.counters + t, 1u);
                *s.flag = (prev + 1 == cl - cf + 1) ? 1u : 0u;
            }
            named_sync(1, 128);
            if (*s.flag) {
                __threadfence();
                const uint32_t cf = unit_owner(t * KB, units, G), cl = unit_owner(t * KB + KB - 1, units, G);
                for (uint32_t n = 0; n < p.npad; ++n) {
                    float y = 0.0f;
                    for (uint32_t cc = cf; cc <= cl; ++cc) {
                        const uint32_t lc = t - unit_start(cc, units, G) / KB;
                        const float *sl = p.partial + ((size_t)cc * p.max_local + lc) * p.npad * kTileM;
                        y = (cc == cf) ? __ldcg(sl + (size_t)n * kTileM + r) : __fadd_rn(y, __ldcg(sl + (size_t)n * kTileM + r));
                    }
                    epilogue(p, y, n, row, valid);
                }
                if (r == 0) p.counters[t] = 0;
            }
            named_sync(1, 128);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ncols) : "memory");
    }
}


/* ---- per-stream kernels ---- */

/* Pass-relative placement of stream s in a TileOut. */
__device__ __forceinline__ uint8_t *pass_tiles(const TileOut &o, uint32_t s, uint32_t &n, uint32_t &npad) {
    const uint32_t pass = s / kMaxPassStreams;
    n = s - pass * kMaxPassStreams;
    npad = (pass + 1 == o.passes) ? o.npad_last : (uint32_t)kMaxPassStreams;
    return o.base + (size_t)pass * o.pass_stride;
}

/* RMSNorm of the residual of stream blockIdx.x (c_impl/gdn_model.cpp:1394-1476):
 * per 16-element half a sequential sum of squares, the halves summed in
 * order; scale = 1/sqrtf(sum/H + eps); out = (x * scale) * w, written as the
 * activation tiles of the next projection. At layer 0 the residual is first
 * loaded with the token's embedding row (:3719-3731). */
__global__ void __launch_bounds__(256) input_kernel(const StepParams p, const float *__restrict__ norm_w, int embed,
                                                    TileOut out) {
    __shared__ float half_sum[256];
    __shared__ float scale_s;
    const uint32_t s = blockIdx.x, H = p.hidden, t = threadIdx.x;
    float *x = p.resid + (size_t)s * H;
    if (embed) {
        const uint32_t step = *p.step;
        int32_t tok = (p.greedy && step > 0) ? p.argmax_out[(size_t)(step - 1) * p.streams + s]
                                             : p.tokens[(size_t)step * p.streams + s];
        if (tok < 0 || (uint32_t)tok >= p.vocab) {
            if (t == 0) report(p.status, kErrBadToken, s);
            tok = 0;
        }
        const uint16_t *e = p.emb + (size_t)tok * H;
        for (uint32_t j = t; j < H; j += 256) x[j] = __uint_as_float((uint32_t)e[j] << 16);
        __syncthreads();
    }
    for (uint32_t hf = t; hf < H / 16; hf += 256) {
        float acc = 0.0f;
#pragma unroll
        for (int k = 0; k < 16; ++k) {
            const float v = x[hf * 16 + k];
            acc = __fadd_rn(acc, __fmul_rn(v, v));
        }
        half_sum[hf] = acc;
    }
    __syncthreads();
    if (t == 0) {
        float sum = 0.0f;
        for (uint32_t hf = 0; hf < H / 16; ++hf) sum = __fadd_rn(sum, half_sum[hf]);
        scale_s = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(sum, (float)H), p.eps)));
    }
    __syncthreads();
    const float scale = scale_s;
    uint32_t n, npad;
    uint8_t *tiles = pass_tiles(out, s, n, npad);
    for (uint32_t c8 = t; c8 < H / 8; c8 += 256) {
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t j = c8 * 8 + i;
            v[i] = __fmul_rn(__fmul_rn(x[j], scale), norm_w[j]);
        }
        put_act8(tiles, npad, n, c8 * 8, v);
    }
}

/* The gated delta rule for 64 state columns of one head of one stream
 * (c_impl/gdn_model.cpp:1932-2340 in the FP32 contract): q, k L2-normalised
 * (tree256 sums, :2059-2092), beta = sigmoid(b), decay = exp(-exp(a_log) *
 * softplus(a + dt_bias)) (:2101-2105), alpha = tree256(qn . kn) (:2119-2124);
 * per column v: r = S[:, v] . kn, p = S[:, v] . qn, delta = beta (v - decay r),
 * o = (decay p + alpha delta) / 16, S'[:, v] = decay S[:, v] + kn delta. A warp
 * owns eight columns; lane l holds k = 4l .. 4l+3 and 128+4l .. 128+4l+3 of a
 * column, the two dot products are warp sums. */
constexpr uint32_t kRecurCols = 64;
__global__ void __launch_bounds__(256) recur_kernel(const StepParams p, uint32_t layer) {
    __shared__ __align__(16) float qn[256], kn[256];
    __shared__ float red[2][8];
    __shared__ float scal[3];
    const uint32_t nh = p.heads, H = p.hidden;
    const uint32_t cb = blockIdx.x % (256 / kRecurCols);
    const uint32_t h = (blockIdx.x / (256 / kRecurCols)) % nh;
    const uint32_t s = blockIdx.x / ((256 / kRecurCols) * nh);
    const uint32_t t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const uint32_t qkv_stride = 4 * H + 2 * nh;
    const float *row = p.qkv + (size_t)s * qkv_stride;
    const float q = row[h * 256 + t], k = row[H + h * 256 + t];
    float sq = __fmul_rn(q, q), sk = __fmul_rn(k, k);
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        sq = __fadd_rn(sq, __shfl_xor_sync(0xffffffffu, sq, o));
        sk = __fadd_rn(sk, __shfl_xor_sync(0xffffffffu, sk, o));
    }
    if (lane == 0) {
        red[0][warp] = sq;
        red[1][warp] = sk;
    }
    __syncthreads();
    const float tq = __fadd_rn(__fadd_rn(__fadd_rn(red[0][0], red[0][1]), __fadd_rn(red[0][2], red[0][3])),
                               __fadd_rn(__fadd_rn(red[0][4], red[0][5]), __fadd_rn(red[0][6], red[0][7])));
    const float tk = __fadd_rn(__fadd_rn(__fadd_rn(red[1][0], red[1][1]), __fadd_rn(red[1][2], red[1][3])),
                               __fadd_rn(__fadd_rn(red[1][4], red[1][5]), __fadd_rn(red[1][6], red[1][7])));
    const float q_inv = __fdiv_rn(1.0f, sqrtf(__fadd_rn(tq, 1e-6f)));
    const float k_inv = __fdiv_rn(1.0f, sqrtf(__fadd_rn(tk, 1e-6f)));
    const float qv = __fmul_rn(q, q_inv), kv = __fmul_rn(k, k_inv);
    qn[t] = qv;
    kn[t] = kv;
    float a = __fmul_rn(qv, kv);
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) a = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, o));
    __syncthreads();
    if (lane == 0) red[0][warp] = a;
    if (t == 0) {
        const float *aux = p.aux + (size_t)layer * p.aux_stride;
        const float *a_log = aux + 14 * H + 256, *dt_bias = a_log + nh;
        const float av = row[4 * H + h], bv = row[4 * H + nh + h];
        scal[1] = sigmoid_ref(bv);
        const float dv = __fmul_rn(-expf(a_log[h]), softplus_ref(__fadd_rn(av, dt_bias[h])));
        scal[2] = expf(dv);
    }
    __syncthreads();
    const float alpha = __fadd_rn(__fadd_rn(__fadd_rn(red[0][0], red[0][1]), __fadd_rn(red[0][2], red[0][3])),
                                  __fadd_rn(__fadd_rn(red[0][4], red[0][5]), __fadd_rn(red[0][6], red[0][7])));
    const float beta = scal[1], decay = scal[2];
    const float4 k0 = reinterpret_cast<const float4 *>(kn)[lane], k1 = reinterpret_cast<const float4 *>(kn)[32 + lane];
    const float4 q0 = reinterpret_cast<const float4 *>(qn)[lane], q1 = reinterpret_cast<const float4 *>(qn)[32 + lane];
    const uint32_t c0 = cb * kRecurCols + warp * 8;
    float *S = p.state + (size_t)s * p.state_stride + (((size_t)layer * nh + h) * 256 + c0) * 256;
    float4 a0[8], a1[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        a0[i] = __ldcs(reinterpret_cast<const float4 *>(S + (size_t)i * 256) + lane);
        a1[i] = __ldcs(reinterpret_cast<const float4 *>(S + (size_t)i * 256) + 32 + lane);
    }
    float *attn = p.attn + (size_t)s * H + h * 256;
    const float *vrow = row + 2 * H + h * 256;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        float r = __fmul_rn(a0[i].x, k0.x), pp = __fmul_rn(a0[i].x, q0.x);
        r = __fadd_rn(r, __fmul_rn(a0[i].y, k0.y)); pp = __fadd_rn(pp, __fmul_rn(a0[i].y, q0.y));
        r = __fadd_rn(r, __fmul_rn(a0[i].z, k0.z)); pp = __fadd_rn(pp, __fmul_rn(a0[i].z, q0.z));
        r = __fadd_rn(r, __fmul_rn(a0[i].w, k0.w)); pp = __fadd_rn(pp, __fmul_rn(a0[i].w, q0.w));
        r = __fadd_rn(r, __fmul_rn(a1[i].x, k1.x)); pp = __fadd_rn(pp, __fmul_rn(a1[i].x, q1.x));
        r = __fadd_rn(r, __fmul_rn(a1[i].y, k1.y)); pp = __fadd_rn(pp, __fmul_rn(a1[i].y, q1.y));
        r = __fadd_rn(r, __fmul_rn(a1[i].z, k1.z)); pp = __fadd_rn(pp, __fmul_rn(a1[i].z, q1.z));
        r = __fadd_rn(r, __fmul_rn(a1[i].w, k1.w)); pp = __fadd_rn(pp, __fmul_rn(a1[i].w, q1.w));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            r = __fadd_rn(r, __shfl_xor_sync(0xffffffffu, r, o));
            pp = __fadd_rn(pp, __shfl_xor_sync(0xffffffffu, pp, o));
        }
        const uint32_t col = c0 + i;
        const float delta = __fmul_rn(beta, __fsub_rn(vrow[col], __fmul_rn(decay, r)));
        if (lane == 0) attn[col] = __fmul_rn(0.0625f, __fadd_rn(__fmul_rn(decay, pp), __fmul_rn(alpha, delta)));
        float4 n0, n1;
        n0.x = __fadd_rn(__fmul_rn(decay, a0[i].x), __fmul_rn(k0.x, delta));
        n0.y = __fadd_rn(__fmul_rn(decay, a0[i].y), __fmul_rn(k0.y, delta));
        n0.z = __fadd_rn(__fmul_rn(decay, a0[i].z), __fmul_rn(k0.z, delta));
        n0.w = __fadd_rn(__fmul_rn(decay, a0[i].w), __fmul_rn(k0.w, delta));
        n1.x = __fadd_rn(__fmul_rn(decay, a1[i].x), __fmul_rn(k1.x, delta));
        n1.y = __fadd_rn(__fmul_rn(decay, a1[i].y), __fmul_rn(k1.y, delta));
        n1.z = __fadd_rn(__fmul_rn(decay, a1[i].z), __fmul_rn(k1.z, delta));
        n1.w = __fadd_rn(__fmul_rn(decay, a1[i].w), __fmul_rn(k1.w, delta));
        __stcs(reinterpret_cast<float4 *>(S + (size_t)i * 256) + lane, n0);
        __stcs(reinterpret_cast<float4 *>(S + (size_t)i * 256) + 32 + lane, n1);
    }
}

/* Output RMSNorm x swish gate of one head of one stream (c_impl/gdn_model.cpp:
 * 3226-3349): per 16-element half a sequential sum of squares, halves summed
 * in order; scale = 1/sqrtf(sum/256 + eps); out = ((a * scale) * w) * g *
 * sigmoid(g), written as activation tiles of the O projection. */
__global__ void __launch_bounds__(256) gate_norm_kernel(const StepParams p, uint32_t layer, TileOut out) {
    __shared__ float half_sum[16];
    __shared__ float scale_s;
    const uint32_t nh = p.heads, H = p.hidden;
    const uint32_t h = blockIdx.x % nh, s = blockIdx.x / nh, t = threadIdx.x;
    const float *a = p.attn + (size_t)s * H + h * 256;
    if (t < 16) {
        float acc = 0.0f;
#pragma unroll
        for (int k = 0; k < 16; ++k) {
            const float v = a[t * 16 + k];
            acc = __fadd_rn(acc, __fmul_rn(v, v));
        }
        half_sum[t] = acc;
    }
    __syncthreads();
    if (t == 0) {
        float sum = 0.0f;
        for (int i = 0; i < 16; ++i) sum = __fadd_rn(sum, half_sum[i]);
        scale_s = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(sum, 256.0f), p.eps)));
    }
    __syncthreads();
    if (t < 32) {
        const float *w = p.aux + (size_t)layer * p.aux_stride + H;  /* o_norm */
        const float *g = p.qkv + (size_t)s * (4 * H + 2 * nh) + 3 * H + h * 256;
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t j = t * 8 + i;
            const float gv = g[j];
            const float nrm = __fmul_rn(__fmul_rn(a[j], scale_s), w[j]);
            v[i] = __fmul_rn(__fmul_rn(nrm, gv), sigmoid_ref(gv));
        }
        uint32_t n, npad;
        uint8_t *tiles = pass_tiles(out, s, n, npad);
        put_act8(tiles, npad, n, h * 256 + t * 8, v);
    }
}

/* Tokens of the step from the argmax keys; keys cleared; step advanced. */
__global__ void __launch_bounds__(256) finish_kernel(const StepParams p) {
    const uint32_t step = *p.step;
    for (uint32_t s = threadIdx.x; s < p.streams; s += 256) {
        const unsigned long long key = p.keys[s];
        p.argmax_out[(size_t)step * p.streams + s] = key ? (int32_t)(0xFFFFFFFFu - (uint32_t)key) : 0;
        p.keys[s] = 0ull;
    }
    __syncthreads();
    if (threadIdx.x == 0) *p.step = step + 1;
}

}  // namespace

size_t gemm_smem_bytes(uint32_t npad, uint32_t a_slots, uint32_t b_slots) {
    return kSmemAlign + (size_t)a_slots * kABlockBytes + (size_t)b_slots * kTerms * npad * 128u + kSmemTail;
}

void gemm_slots(uint32_t npad, uint32_t *a_slots, uint32_t *b_slots) {
    const size_t bblock = (size_t)kTerms * npad * 128u;
    const uint32_t sb = bblock >= 24576 ? 2u : 4u;
    size_t room = kSmemLimit - kSmemAlign - kSmemTail - sb * bblock;
    uint32_t sa = (uint32_t)(room / kABlockBytes);
    if (sa > 10) sa = 10;
    *a_slots = sa;
    *b_slots = sb;
}

uint32_t gemm_grid(uint32_t mtiles, uint32_t kblocks, uint32_t sms) {
    const uint32_t units = mtiles * kblocks;
    return units < sms ? units : sms;
}

uint32_t gemm_max_local(uint32_t mtiles, uint32_t kblocks, uint32_t grid) {
    const uint32_t units = mtiles * kblocks;
    uint32_t mx = 1;
    for (uint32_t c = 0; c < grid; ++c) {
        const uint32_t a = unit_start(c, units, grid), b = unit_start(c + 1, units, grid);
        if (b <= a) continue;
        const uint32_t n = (b - 1) / kblocks - a / kblocks + 1;
        if (n > mx) mx = n;
    }
    return mx;
}

size_t tile_pass_bytes(uint32_t npad, uint32_t k) { return (size_t)(k / kTileK) * kTerms * npad * 128u; }

cudaError_t launch_gemm(const GemmParams &p, uint32_t grid, cudaStream_t stream) {
    const size_t smem = gemm_smem_bytes(p.npad, p.a_slots, p.b_slots);
    cudaError_t e = cudaFuncSetAttribute(tile_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    tile_gemm_kernel<<<grid, kGemmThreads, smem, stream>>>(p);
    return cudaGetLastError();
}


cudaError_t launch_input(const StepParams &p, const float *norm_w, int embed, TileOut out, cudaStream_t stream) {
    input_kernel<<<p.streams, 256, 0, stream>>>(p, norm_w, embed, out);
    return cudaGetLastError();
}

cudaError_t launch_recur(const StepParams &p, uint32_t layer, cudaStream_t stream) {
    recur_kernel<<<p.streams * p.heads * (256 / kRecurCols), 256, 0, stream>>>(p, layer);
    return cudaGetLastError();
}

cudaError_t launch_gate_norm(const StepParams &p, uint32_t layer, TileOut out, cudaStream_t stream) {
    gate_norm_kernel<<<p.streams * p.heads, 256, 0, stream>>>(p, layer, out);
    return cudaGetLastError();
}

cudaError_t launch_finish(const StepParams &p, cudaStream_t stream) {
    finish_kernel<<<1, 256, 0, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace bt
}  // namespace gdn
