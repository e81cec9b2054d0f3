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
 * the activation blocks, one issues the MMAs (one per 16-column step, N =
 * three BF16 terms x streams), and four warps drain TMEM (summing the terms)
 * while the next segment accumulates. Every wait is bounded (2 s) and
 * reports through the status word.
 */
#include "gdn_batch.h"

#include <cuda_bf16.h>

#include <algorithm>
#include <cstring>
#include <utility>
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

/* Programmatic dependent launch: every kernel of the step lets the next one
 * start (launch_dependents) and waits for the previous one (wait) only where
 * it first needs that kernel's results, so weight copies and state loads that
 * depend on nothing overlap the previous kernel's tail. */
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

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

    pdl_trigger();
    const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t units = p.mtiles * p.kblocks, G = gridDim.x, c = blockIdx.x;
    const uint32_t u0 = unit_start(c, units, G), u1 = unit_start(c + 1, units, G);
    const uint32_t KB = p.kblocks;
    /* TMEM: one accumulator holds the three term columns of every stream
     * (3 * npad <= 240 columns); two of them, a power of two apart, so the
     * next segment accumulates while the epilogue drains the last one */
    uint32_t acc_cols = 32;
    while (acc_cols < kTerms * p.npad) acc_cols <<= 1;
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
        /* activation blocks: k-block u % KB of the pass's tiles, written by
         * the previous kernel */
        if (lane == 0) {
            pdl_wait();
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
            /* N = 3 * npad: the three BF16 terms of the activations are 3 * npad
             * consecutive rows of the activation block, so one MMA per 16
             * columns covers them all and reads the weight tile once */
            const uint32_t idesc = instr_desc(kTileM, kTerms * p.npad);
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
                    for (uint32_t kk = 0; kk < kTileK / 16; ++kk)
                        tc_mma(d, smem_desc(abase + kk * 32u), smem_desc(bbase + kk * 32u), idesc,
                               (u == ua && kk == 0) ? 0u : 1u);
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
        /* warps 0-3: TMEM lanes 32w .. 32w + 31 = rows of the tile; each
         * segment's accumulator goes to its partial slot (the projection's
         * consumer sums the slots of a tile) */
        const uint32_t r = tid;  /* 0..127 */
        pdl_wait();  /* the partial slots may still be read by the previous kernel */
        uint32_t seg = 0;
        for (uint32_t t = u0 / KB; t * KB < u1; ++t, ++seg) {
            const uint32_t acc = seg & 1u;
            /* the 128 epilogue threads leave together or not at all */
            const bool got = wait_bar(s.acc_full + 8 * acc, (seg >> 1) & 1u, abort);
            if (!named_all(1, 128, got)) {
                if (!got && !*abort) report(p.status, kErrWaitAcc, c);
                *abort = 1;
                break;
            }
            tc_fence_after();
            const uint32_t taddr = tmem + acc * acc_cols + ((warp * 32u) << 16);
            float *slot = p.partial + ((size_t)c * p.max_local + (t - u0 / KB)) * p.npad * kTileM + r;
            for (uint32_t c0 = 0; c0 < p.npad; c0 += 16) {
                float v0[16], v1[16], v2[16];
                tc_ld16(taddr + c0, v0);
                tc_ld16(taddr + p.npad + c0, v1);
                tc_ld16(taddr + 2 * p.npad + c0, v2);
#pragma unroll
                for (int j = 0; j < 16; ++j)
                    __stcg(slot + (size_t)(c0 + j) * kTileM, __fadd_rn(v0[j], __fadd_rn(v1[j], v2[j])));
            }
            tc_fence_before();
            mbar_arrive(s.acc_empty + 8 * acc);
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

/* Rows row0 .. row0 + 7 (row0 % 8 == 0) of stream s of a projection: the sum
 * of the tile's partial slots in k order. The loads of up to four segments
 * are in flight together. */
__device__ __forceinline__ void psum8(const Partials &v, uint32_t s, uint32_t row0, float (&out)[8]) {
    const uint32_t pass = s / kMaxPassStreams, n = s - pass * kMaxPassStreams;
    const uint32_t npad = (pass + 1 == v.passes) ? v.npad_last : (uint32_t)kMaxPassStreams;
    const uint32_t KB = v.kblocks, t = row0 / kTileM, r = row0 - t * kTileM;
    const uint32_t cf = unit_owner(t * KB, v.units, v.grid), cl = unit_owner(t * KB + KB - 1, v.units, v.grid);
    const uint32_t ns = cl - cf + 1;
    const float *base = v.base + pass * v.pass_stride + (size_t)n * kTileM + r;
    const size_t slot = (size_t)npad * kTileM;
    for (uint32_t k0 = 0; k0 < ns; k0 += 4) {
        float4 x[4][2];
#pragma unroll
        for (uint32_t k = 0; k < 4; ++k) {
            if (k0 + k < ns) {
                const uint32_t cc = cf + k0 + k;
                const uint32_t lc = t - unit_start(cc, v.units, v.grid) / KB;
                const float4 *q = reinterpret_cast<const float4 *>(base + ((size_t)cc * v.max_local + lc) * slot);
                x[k][0] = __ldcg(q);
                x[k][1] = __ldcg(q + 1);
            }
        }
#pragma unroll
        for (uint32_t k = 0; k < 4; ++k) {
            if (k0 + k < ns) {
                const float e[8] = {x[k][0].x, x[k][0].y, x[k][0].z, x[k][0].w,
                                    x[k][1].x, x[k][1].y, x[k][1].z, x[k][1].w};
#pragma unroll
                for (int i = 0; i < 8; ++i) out[i] = (k0 + k == 0) ? e[i] : __fadd_rn(out[i], e[i]);
            }
        }
    }
}

/* RMSNorm of the residual of stream blockIdx.x (c_impl/gdn_model.cpp:1394-1476
 * in the FP32 contract): scale = 1/sqrtf(sum(x^2)/H + eps), out = (x * scale)
 * * w, written as the activation tiles of the next projection. Mode 0 (layer 0)
 * loads the residual with the token's embedding row (:3719-3731); mode 1
 * first adds the sums of the previous projection (the residual add of
 * :3351-3452, :3836-3842). Each thread keeps its (at most two) 8-element
 * chunks in registers; every load is issued before the first dependent use. */
__global__ void __launch_bounds__(256) input_kernel(const StepParams p, const float *__restrict__ norm_w, int mode,
                                                    const Partials add, TileOut out) {
    __shared__ float wsum[8];
    pdl_trigger();
    const uint32_t s = blockIdx.x, H = p.hidden, t = threadIdx.x, nch = H / 8;
    /* the norm weights do not depend on the previous kernel */
    float w[2][8];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const uint32_t c8 = t + 256 * r;
        if (c8 < nch) {
            const float4 w0 = reinterpret_cast<const float4 *>(norm_w)[2 * c8];
            const float4 w1 = reinterpret_cast<const float4 *>(norm_w)[2 * c8 + 1];
            w[r][0] = w0.x; w[r][1] = w0.y; w[r][2] = w0.z; w[r][3] = w0.w;
            w[r][4] = w1.x; w[r][5] = w1.y; w[r][6] = w1.z; w[r][7] = w1.w;
        }
    }
    pdl_wait();
    float *x = p.resid + (size_t)s * H;
    int32_t tok = 0;
    if (mode == 0) {
        const uint32_t step = __ldcg(p.step);
        tok = (p.greedy && step > 0) ? __ldcg(p.argmax_out + (size_t)(step - 1) * p.streams + s)
                                     : __ldcg(p.tokens + (size_t)step * p.streams + s);
        if (tok < 0 || (uint32_t)tok >= p.vocab) {
            if (t == 0) report(p.status, kErrBadToken, s);
            tok = 0;
        }
    }
    float v[2][8];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const uint32_t c8 = t + 256 * r;
        if (c8 >= nch) continue;
        if (mode == 0) {
            const uint4 e = *reinterpret_cast<const uint4 *>(p.emb + (size_t)tok * H + c8 * 8);
            const uint32_t ew[4] = {e.x, e.y, e.z, e.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                v[r][2 * i] = __uint_as_float(ew[i] << 16);
                v[r][2 * i + 1] = __uint_as_float(ew[i] & 0xFFFF0000u);
            }
        } else {
            const float4 a0 = __ldcg(reinterpret_cast<const float4 *>(x) + 2 * c8);
            const float4 a1 = __ldcg(reinterpret_cast<const float4 *>(x) + 2 * c8 + 1);
            float y[8];
            psum8(add, s, c8 * 8, y);
            const float xa[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
#pragma unroll
            for (int i = 0; i < 8; ++i) v[r][i] = __fadd_rn(xa[i], y[i]);
        }
        reinterpret_cast<float4 *>(x)[2 * c8] = make_float4(v[r][0], v[r][1], v[r][2], v[r][3]);
        reinterpret_cast<float4 *>(x)[2 * c8 + 1] = make_float4(v[r][4], v[r][5], v[r][6], v[r][7]);
    }
    float acc = 0.0f;
#pragma unroll
    for (int r = 0; r < 2; ++r)
        if (t + 256 * r < nch) {
#pragma unroll
            for (int i = 0; i < 8; ++i) acc = __fadd_rn(acc, __fmul_rn(v[r][i], v[r][i]));
        }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o));
    if ((t & 31) == 0) wsum[t >> 5] = acc;
    __syncthreads();
    float sum = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) sum = __fadd_rn(sum, wsum[i]);
    const float scale = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(sum, (float)H), p.eps)));
    uint32_t n, npad;
    uint8_t *tiles = pass_tiles(out, s, n, npad);
#pragma unroll
    for (int r = 0; r < 2; ++r) {
        const uint32_t c8 = t + 256 * r;
        if (c8 >= nch) continue;
        float o[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = __fmul_rn(__fmul_rn(v[r][i], scale), w[r][i]);
        put_act8(tiles, npad, n, c8 * 8, o);
    }
}

/* Causal conv + SiLU of 8 channels (:1543-1660): window [t0, t1, t2, new]
 * summed left to right; the new window [t1, t2, new] goes to the other tail
 * buffer when `write` is set. */
__device__ __forceinline__ void conv8(const float *__restrict__ tr, float *__restrict__ tw, uint32_t H,
                                      const float *__restrict__ w4, const float (&y)[8], bool write, float (&o)[8]) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float t0 = __ldcg(tr + i), t1 = __ldcg(tr + H + i), t2 = __ldcg(tr + 2 * H + i);
        const float4 w = reinterpret_cast<const float4 *>(w4)[i];
        float sum = __fadd_rn(__fmul_rn(t0, w.x), __fmul_rn(t1, w.y));
        sum = __fadd_rn(sum, __fmul_rn(t2, w.z));
        sum = __fadd_rn(sum, __fmul_rn(y[i], w.w));
        o[i] = silu_ref(sum);
        if (write) {
            tw[i] = t1;
            tw[H + i] = t2;
            tw[2 * H + i] = y[i];
        }
    }
}

/* Per (stream, head), the inputs of the gated delta rule (c_impl/gdn_model.cpp:
 * 1932-2124 in the FP32 contract): q, k, v of the head after the causal conv +
 * SiLU (new tails to the other buffer), q and k L2-normalised (tree256 sums,
 * :2059-2092), alpha = tree256(qn . kn) (:2119-2124), beta = sigmoid(b) and
 * decay = exp(-exp(a_log) * softplus(a + dt_bias)) (:2101-2105). Output
 * prep[s][h] = {alpha, beta, decay, 0, qn[256], kn[256], v[256]}. */
constexpr uint32_t kPrepFloats = 4 + 3 * 256;
__global__ void __launch_bounds__(128) prep_kernel(const StepParams p, uint32_t layer, const Partials qkv,
                                                   float *__restrict__ prep) {
    __shared__ __align__(16) float qs[256], ks[256];
    __shared__ float red[3][4];
    __shared__ float scal[2];
    pdl_trigger();
    pdl_wait();
    const uint32_t nh = p.heads, H = p.hidden;
    const uint32_t h = blockIdx.x % nh, s = blockIdx.x / nh, t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const float *aux = p.aux + (size_t)layer * p.aux_stride;
    float *out = prep + ((size_t)s * nh + h) * kPrepFloats;
    if (t < 96) {
        const uint32_t kind = t >> 5, ch = h * 256 + (t & 31) * 8;
        float y[8], o[8];
        psum8(qkv, s, kind * H + ch, y);
        const uint32_t par = __ldcg(p.tails_parity);
        const size_t toff = (size_t)s * p.tails_stride + ((size_t)layer * 3 + kind) * 3 * H + ch;
        conv8(p.tails + par * p.tails_buf + toff, p.tails + (par ^ 1u) * p.tails_buf + toff, H,
              aux + 2 * H + 256 + ((size_t)kind * H + ch) * 4, y, true, o);
        float *dst = kind == 0 ? qs + (t & 31) * 8 : (kind == 1 ? ks + (t & 31) * 8 : out + 4 + 512 + (t & 31) * 8);
#pragma unroll
        for (int i = 0; i < 8; ++i) dst[i] = o[i];
    } else if (t == 96 || t == 97) {
        /* a (t = 96) and b (t = 97) of the head */
        const uint32_t row = t == 96 ? h : nh + h;
        float y8[8];
        psum8(qkv, s, 4 * H + (row & ~7u), y8);
        float yv = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; ++i) yv = ((uint32_t)i == (row & 7u)) ? y8[i] : yv;
        if (t == 97) {
            scal[0] = sigmoid_ref(yv);
        } else {
            const float *a_log = aux + 14 * H + 256, *dt_bias = a_log + nh;
            scal[1] = expf(__fmul_rn(-expf(a_log[h]), softplus_ref(__fadd_rn(yv, dt_bias[h]))));
        }
    }
    __syncthreads();
    /* tree256: thread t holds elements 2t, 2t+1 (first level), the warp
     * butterfly the next five levels, then (w0 + w1) + (w2 + w3) */
    const float2 q2 = reinterpret_cast<const float2 *>(qs)[t], k2 = reinterpret_cast<const float2 *>(ks)[t];
    float sq = __fadd_rn(__fmul_rn(q2.x, q2.x), __fmul_rn(q2.y, q2.y));
    float sk = __fadd_rn(__fmul_rn(k2.x, k2.x), __fmul_rn(k2.y, k2.y));
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
    const float tq = __fadd_rn(__fadd_rn(red[0][0], red[0][1]), __fadd_rn(red[0][2], red[0][3]));
    const float tk = __fadd_rn(__fadd_rn(red[1][0], red[1][1]), __fadd_rn(red[1][2], red[1][3]));
    const float q_inv = __fdiv_rn(1.0f, sqrtf(__fadd_rn(tq, 1e-6f)));
    const float k_inv = __fdiv_rn(1.0f, sqrtf(__fadd_rn(tk, 1e-6f)));
    const float2 qn = make_float2(__fmul_rn(q2.x, q_inv), __fmul_rn(q2.y, q_inv));
    const float2 kn = make_float2(__fmul_rn(k2.x, k_inv), __fmul_rn(k2.y, k_inv));
    reinterpret_cast<float2 *>(out + 4)[t] = qn;
    reinterpret_cast<float2 *>(out + 4 + 256)[t] = kn;
    float a = __fadd_rn(__fmul_rn(qn.x, kn.x), __fmul_rn(qn.y, kn.y));
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) a = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, o));
    if (lane == 0) red[2][warp] = a;
    __syncthreads();
    if (t == 0) {
        out[0] = __fadd_rn(__fadd_rn(red[2][0], red[2][1]), __fadd_rn(red[2][2], red[2][3]));
        out[1] = scal[0];
        out[2] = scal[1];
        out[3] = 0.0f;
    }
}

/* The gated delta rule for 64 state columns of one head of one stream
 * (c_impl/gdn_model.cpp:2184-2300 in the FP32 contract), from prep_kernel's
 * inputs: per column v, r = S[:, v] . kn, p = S[:, v] . qn, delta = beta (v -
 * decay r), o = (decay p + alpha delta) / 16, S'[:, v] = decay S[:, v] +
 * kn delta. A warp owns eight columns; lane l holds k = 4l .. 4l+3 and
 * 128+4l .. 128+4l+3 of a column, the two dot products are warp sums. S is
 * read and written once, with streaming (evict-first) accesses. */
constexpr uint32_t kRecurCols = 64;
__global__ void __launch_bounds__(256) recur_kernel(const StepParams p, uint32_t layer, const float *prep) {
    const uint32_t nh = p.heads, H = p.hidden;
    const uint32_t cb = blockIdx.x % (256 / kRecurCols);
    const uint32_t h = (blockIdx.x / (256 / kRecurCols)) % nh;
    const uint32_t s = blockIdx.x / ((256 / kRecurCols) * nh);
    const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint32_t c0 = cb * kRecurCols + warp * 8;
    float *S = p.state + (size_t)s * p.state_stride + (((size_t)layer * nh + h) * 256 + c0) * 256;
    pdl_trigger();
    /* S was last written by this layer's recurrence one step earlier: it is
     * loaded before waiting for prep_kernel */
    float4 a0[8], a1[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        a0[i] = __ldcg(reinterpret_cast<const float4 *>(S + (size_t)i * 256) + lane);
        a1[i] = __ldcg(reinterpret_cast<const float4 *>(S + (size_t)i * 256) + 32 + lane);
    }
    pdl_wait();
    const float *in = prep + ((size_t)s * nh + h) * kPrepFloats;
    const float alpha = __ldcg(in), beta = __ldcg(in + 1), decay = __ldcg(in + 2);
    const float4 q0 = __ldcg(reinterpret_cast<const float4 *>(in + 4) + lane);
    const float4 q1 = __ldcg(reinterpret_cast<const float4 *>(in + 4) + 32 + lane);
    const float4 k0 = __ldcg(reinterpret_cast<const float4 *>(in + 4 + 256) + lane);
    const float4 k1 = __ldcg(reinterpret_cast<const float4 *>(in + 4 + 256) + 32 + lane);
    const float vv = lane < 8 ? __ldcg(in + 4 + 512 + c0 + lane) : 0.0f;
    float *attn = p.attn + (size_t)s * H + h * 256;
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
        const float v = __shfl_sync(0xffffffffu, vv, i);
        const float delta = __fmul_rn(beta, __fsub_rn(v, __fmul_rn(decay, r)));
        if (lane == 0) attn[c0 + i] = __fmul_rn(0.0625f, __fadd_rn(__fmul_rn(decay, pp), __fmul_rn(alpha, delta)));
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

/* One head of one stream, layer l, in one CTA: the recurrence's inputs (as
 * prep_kernel: conv + SiLU with the tail update, L2 norms, alpha, beta,
 * decay), the gated delta rule over all 256 state columns (as recur_kernel),
 * and the output RMSNorm x swish gate (as gate_norm_kernel) written as the O
 * projection's activation tiles. Warp w owns columns 32w .. 32w+31 (32 KB,
 * contiguous) and streams them through its own three-slot shared-memory ring
 * of 4-column bulk copies (4 KB); the first three copies are issued before
 * the kernel waits for the QKVGAB projection, so they overlap the prologue.
 * Every ring wait is bounded (2 s) and reports through the status word. */
constexpr int kHeadCols = 4;                      /* columns per copy */
constexpr int kHeadSlots = 3;                     /* copies in flight per warp */
constexpr uint32_t kHeadSlotBytes = kHeadCols * 1024u;
constexpr size_t kHeadSmem = 8 * kHeadSlots * kHeadSlotBytes + 8 * kHeadSlots * 8 + 4 * 256 * 4 + 64;
__global__ void __launch_bounds__(256, 2) head_kernel(const StepParams p, uint32_t layer, const Partials qkv,
                                                      TileOut out) {
    extern __shared__ __align__(128) uint8_t hsm[];
    float *ring = reinterpret_cast<float *>(hsm);                                   /* [8 warps][slots][4][256] */
    uint64_t *bars = reinterpret_cast<uint64_t *>(hsm + 8 * kHeadSlots * kHeadSlotBytes);  /* [8][slots] */
    float *qs = reinterpret_cast<float *>(hsm + 8 * kHeadSlots * kHeadSlotBytes + 8 * kHeadSlots * 8);
    float *ks = qs + 256, *vs = ks + 256, *os = vs + 256;
    float *red = os + 256;  /* [3][4] + 2 */
    float *scal = red + 12;
    pdl_trigger();
    const uint32_t nh = p.heads, H = p.hidden;
    const uint32_t h = blockIdx.x % nh, s = blockIdx.x / nh, t = threadIdx.x, lane = t & 31, warp = t >> 5;
    float *S = p.state + (size_t)s * p.state_stride + (((size_t)layer * nh + h) * 256 + warp * 32) * 256;
    float *wring = ring + (size_t)warp * kHeadSlots * kHeadCols * 256;
    const uint32_t wbar = smem_u32(bars + warp * kHeadSlots);
    if (lane == 0) {
        for (int i = 0; i < kHeadSlots; ++i) mbar_init(wbar + 8 * i, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        /* S was last written by this layer's recurrence one step earlier */
        for (int i = 0; i < kHeadSlots; ++i) {
            mbar_expect_tx(wbar + 8 * i, kHeadSlotBytes);
            bulk_g2s(smem_u32(wring + (size_t)i * kHeadCols * 256), S + (size_t)i * kHeadCols * 256, kHeadSlotBytes,
                     wbar + 8 * i, policy_evict_first());
        }
    }
    __syncwarp();
    pdl_wait();
    const float *aux = p.aux + (size_t)layer * p.aux_stride;
    if (t < 96) {
        const uint32_t kind = t >> 5, ch = h * 256 + (t & 31) * 8;
        float y[8], o[8];
        psum8(qkv, s, kind * H + ch, y);
        const uint32_t par = __ldcg(p.tails_parity);
        const size_t toff = (size_t)s * p.tails_stride + ((size_t)layer * 3 + kind) * 3 * H + ch;
        conv8(p.tails + par * p.tails_buf + toff, p.tails + (par ^ 1u) * p.tails_buf + toff, H,
              aux + 2 * H + 256 + ((size_t)kind * H + ch) * 4, y, true, o);
        float *dst = (kind == 0 ? qs : (kind == 1 ? ks : vs)) + (t & 31) * 8;
#pragma unroll
        for (int i = 0; i < 8; ++i) dst[i] = o[i];
    } else if (t == 96 || t == 97) {
        const uint32_t row = t == 96 ? h : nh + h;
        float y8[8];
        psum8(qkv, s, 4 * H + (row & ~7u), y8);
        float yv = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; ++i) yv = ((uint32_t)i == (row & 7u)) ? y8[i] : yv;
        if (t == 97) {
            scal[0] = sigmoid_ref(yv);
        } else {
            const float *a_log = aux + 14 * H + 256, *dt_bias = a_log + nh;
            scal[1] = expf(__fmul_rn(-expf(a_log[h]), softplus_ref(__fadd_rn(yv, dt_bias[h]))));
        }
    }
    __syncthreads();
    /* tree256 of q^2, k^2 (threads 0-127 hold pairs), then of qn . kn */
    if (t < 128) {
        const float2 q2 = reinterpret_cast<const float2 *>(qs)[t], k2 = reinterpret_cast<const float2 *>(ks)[t];
        float sq = __fadd_rn(__fmul_rn(q2.x, q2.x), __fmul_rn(q2.y, q2.y));
        float sk = __fadd_rn(__fmul_rn(k2.x, k2.x), __fmul_rn(k2.y, k2.y));
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            sq = __fadd_rn(sq, __shfl_xor_sync(0xffffffffu, sq, o));
            sk = __fadd_rn(sk, __shfl_xor_sync(0xffffffffu, sk, o));
        }
        if (lane == 0) {
            red[warp] = sq;
            red[4 + warp] = sk;
        }
    }
    __syncthreads();
    const float q_inv = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fadd_rn(__fadd_rn(red[0], red[1]), __fadd_rn(red[2], red[3])),
                                                        1e-6f)));
    const float k_inv = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fadd_rn(__fadd_rn(red[4], red[5]), __fadd_rn(red[6], red[7])),
                                                        1e-6f)));
    if (t < 128) {
        const float2 q2 = reinterpret_cast<const float2 *>(qs)[t], k2 = reinterpret_cast<const float2 *>(ks)[t];
        const float2 qn = make_float2(__fmul_rn(q2.x, q_inv), __fmul_rn(q2.y, q_inv));
        const float2 kn = make_float2(__fmul_rn(k2.x, k_inv), __fmul_rn(k2.y, k_inv));
        float a = __fadd_rn(__fmul_rn(qn.x, kn.x), __fmul_rn(qn.y, kn.y));
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) a = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, o));
        if (lane == 0) red[8 + warp] = a;
    }
    __syncthreads();  /* every q_inv / k_inv read is done before qs / ks are overwritten */
    if (t < 128) {
        const float2 q2 = reinterpret_cast<const float2 *>(qs)[t], k2 = reinterpret_cast<const float2 *>(ks)[t];
        reinterpret_cast<float2 *>(qs)[t] = make_float2(__fmul_rn(q2.x, q_inv), __fmul_rn(q2.y, q_inv));
        reinterpret_cast<float2 *>(ks)[t] = make_float2(__fmul_rn(k2.x, k_inv), __fmul_rn(k2.y, k_inv));
    }
    __syncthreads();
    const float alpha = __fadd_rn(__fadd_rn(red[8], red[9]), __fadd_rn(red[10], red[11]));
    const float beta = scal[0], decay = scal[1];
    const float4 k0 = reinterpret_cast<const float4 *>(ks)[lane], k1 = reinterpret_cast<const float4 *>(ks)[32 + lane];
    const float4 q0 = reinterpret_cast<const float4 *>(qs)[lane], q1 = reinterpret_cast<const float4 *>(qs)[32 + lane];
    bool ok = true;
#pragma unroll 1
    for (int b = 0; b < 32 / kHeadCols; ++b) {
        const int sl = b % kHeadSlots;
        /* bounded wait for the batch; the warp agrees on the outcome */
        bool got = mbar_try(wbar + 8 * sl, (b / kHeadSlots) & 1);
        if (!got) {
            const uint64_t t0 = gtimer();
            while (!(got = mbar_try(wbar + 8 * sl, (b / kHeadSlots) & 1)) && gtimer() - t0 < kWaitNs) {
            }
        }
        if (!__all_sync(0xffffffffu, got)) {
            if (lane == 0) report(p.status, kErrWaitA, blockIdx.x);
            ok = false;
            break;
        }
        const float *src = wring + (size_t)sl * kHeadCols * 256;
        float4 a0[kHeadCols], a1[kHeadCols];
#pragma unroll
        for (int i = 0; i < kHeadCols; ++i) {
            a0[i] = reinterpret_cast<const float4 *>(src + (size_t)i * 256)[lane];
            a1[i] = reinterpret_cast<const float4 *>(src + (size_t)i * 256)[32 + lane];
        }
        float *Sb = S + (size_t)b * kHeadCols * 256;
#pragma unroll
        for (int i = 0; i < kHeadCols; ++i) {
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
            const uint32_t col = warp * 32 + b * kHeadCols + i;
            const float delta = __fmul_rn(beta, __fsub_rn(vs[col], __fmul_rn(decay, r)));
            if (lane == 0) os[col] = __fmul_rn(0.0625f, __fadd_rn(__fmul_rn(decay, pp), __fmul_rn(alpha, delta)));
            float4 n0, n1;
            n0.x = __fadd_rn(__fmul_rn(decay, a0[i].x), __fmul_rn(k0.x, delta));
            n0.y = __fadd_rn(__fmul_rn(decay, a0[i].y), __fmul_rn(k0.y, delta));
            n0.z = __fadd_rn(__fmul_rn(decay, a0[i].z), __fmul_rn(k0.z, delta));
            n0.w = __fadd_rn(__fmul_rn(decay, a0[i].w), __fmul_rn(k0.w, delta));
            n1.x = __fadd_rn(__fmul_rn(decay, a1[i].x), __fmul_rn(k1.x, delta));
            n1.y = __fadd_rn(__fmul_rn(decay, a1[i].y), __fmul_rn(k1.y, delta));
            n1.z = __fadd_rn(__fmul_rn(decay, a1[i].z), __fmul_rn(k1.z, delta));
            n1.w = __fadd_rn(__fmul_rn(decay, a1[i].w), __fmul_rn(k1.w, delta));
            __stcs(reinterpret_cast<float4 *>(Sb + (size_t)i * 256) + lane, n0);
            __stcs(reinterpret_cast<float4 *>(Sb + (size_t)i * 256) + 32 + lane, n1);
        }
        /* the slot's data has been used by every lane: refill it with batch b + slots */
        __syncwarp();
        if (lane == 0 && b + kHeadSlots < 32 / kHeadCols) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            mbar_expect_tx(wbar + 8 * sl, kHeadSlotBytes);
            bulk_g2s(smem_u32(wring + (size_t)sl * kHeadCols * 256), S + (size_t)(b + kHeadSlots) * kHeadCols * 256,
                     kHeadSlotBytes, wbar + 8 * sl, policy_evict_first());
        }
    }
    if (!ok && lane == 0) {
        /* copies issued and not consumed land before the CTA exits */
        for (int i = 0; i < kHeadSlots; ++i) {
            const uint64_t t0 = gtimer();
            while (!mbar_try(wbar + 8 * i, 0) && !mbar_try(wbar + 8 * i, 1) && gtimer() - t0 < kWaitNs) {
            }
        }
    }
    __syncthreads();
    /* output RMSNorm x swish gate (:3226-3349), warp 0: 8 elements per lane */
    if (warp == 0) {
        const float4 o0 = reinterpret_cast<const float4 *>(os)[2 * lane], o1 = reinterpret_cast<const float4 *>(os)[2 * lane + 1];
        const float av[8] = {o0.x, o0.y, o0.z, o0.w, o1.x, o1.y, o1.z, o1.w};
        float g[8];
        psum8(qkv, s, 3 * H + h * 256 + lane * 8, g);
        float acc = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; ++i) acc = __fadd_rn(acc, __fmul_rn(av[i], av[i]));
        const float half = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 1));
        float sum = 0.0f;
#pragma unroll
        for (int j = 0; j < 16; ++j) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, half, 2 * j));
        const float scale = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(sum, 256.0f), p.eps)));
        const float *w = aux + H + lane * 8; /* o_norm */
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float nrm = __fmul_rn(__fmul_rn(av[i], scale), w[i]);
            v[i] = __fmul_rn(__fmul_rn(nrm, g[i]), sigmoid_ref(g[i]));
        }
        uint32_t n, npad;
        uint8_t *tiles = pass_tiles(out, s, n, npad);
        put_act8(tiles, npad, n, h * 256 + lane * 8, v);
    }
}

/* Prefill of one head, 64 state columns (block cb), over the ntok tokens of a
 * chunk, in token order (c_impl/gdn_model.cpp:1543-1660 and :1932-2340 per
 * token, FP32 contract). The tokens are the "streams" of the chunk's
 * projections. In sub-chunks of kSub tokens: the raw q, k (all 256 channels of
 * the head) and v (the block's 64) of every token from the QKVGAB partial
 * sums, the causal conv over time (window from the run state's tails, then
 * from the previous tokens), SiLU, L2 norms, alpha, beta, decay -- all in
 * parallel over tokens; then the recurrence, token by token, on the block's
 * state held in registers (warp w: columns w*8 .. w*8+7, lane l: k = 4l..4l+3
 * and 128+4l..128+4l+3). S is read once and written once per chunk. The
 * window's last three raw rows become the new tails, written to tails_out
 * (this block's q/k quarter and its v channels) so the four blocks of a head
 * never race on the tails they read. Layouts of the single-stream run state:
 * S [L][nh][v][k], tails [L][q,k,v][H][4] (rows 0..2 oldest to newest). */
constexpr int kSub = 16;
constexpr int kPrefCh = 576;  /* q 256 | k 256 | v 64 */
constexpr size_t kPrefillSmem = (size_t)(kSub + 3) * kPrefCh * 4 + (size_t)kSub * kPrefCh * 4 + (size_t)kSub * 4 * 4 + 64;
__global__ void __launch_bounds__(256, 1) prefill_head_kernel(const StepParams p, uint32_t layer, const Partials qkv,
                                                              float *state, const float *tails_in, float *tails_out,
                                                              uint32_t ntok) {
    extern __shared__ __align__(16) float psm[];
    float *raw = psm;                                  /* [kSub + 3][576]: rows 0..2 = the three tokens before */
    float *act = raw + (kSub + 3) * kPrefCh;           /* [kSub][576] */
    float *sc = act + kSub * kPrefCh;                  /* [kSub][4]: alpha, beta, decay, - */
    pdl_trigger();
    pdl_wait();
    const uint32_t nh = p.heads, H = p.hidden;
    const uint32_t cb = blockIdx.x & 3u, h = blockIdx.x >> 2;
    const uint32_t t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const float *aux = p.aux + (size_t)layer * p.aux_stride;
    auto gch = [&](uint32_t c) -> uint32_t {  /* channel c of the block -> (kind, global channel) */
        return c < 512 ? h * 256 + (c & 255u) : h * 256 + cb * 64 + (c - 512);
    };
    auto kind_of = [](uint32_t c) -> uint32_t { return c < 256 ? 0u : (c < 512 ? 1u : 2u); };
    float *S = state + ((((size_t)layer * nh + h) * 256) + cb * 64 + warp * 8) * 256;
    float4 a0[8], a1[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        a0[i] = __ldcg(reinterpret_cast<const float4 *>(S + (size_t)i * 256) + lane);
        a1[i] = __ldcg(reinterpret_cast<const float4 *>(S + (size_t)i * 256) + 32 + lane);
    }
    for (uint32_t c = t; c < (uint32_t)kPrefCh; c += 256) {
        const uint32_t kind = kind_of(c);
        const float4 tv = __ldcg(reinterpret_cast<const float4 *>(tails_in) + ((size_t)layer * 3 + kind) * H + gch(c));
        raw[c] = tv.x;
        raw[kPrefCh + c] = tv.y;
        raw[2 * kPrefCh + c] = tv.z;
    }
    for (uint32_t j0 = 0; j0 < ntok; j0 += kSub) {
        const uint32_t nj = min((uint32_t)kSub, ntok - j0);
        __syncthreads();
        /* raw projections of the sub-chunk's tokens, and a, b */
        for (uint32_t idx = t; idx < nj * (kPrefCh / 8); idx += 256) {
            const uint32_t j = idx / (kPrefCh / 8), c8 = idx % (kPrefCh / 8);
            const uint32_t c = c8 * 8;
            float y[8];
            psum8(qkv, j0 + j, kind_of(c) * H + gch(c), y);
#pragma unroll
            for (int i = 0; i < 8; ++i) raw[(3 + j) * kPrefCh + c + i] = y[i];
        }
        for (uint32_t idx = t; idx < 2 * nj; idx += 256) {
            const uint32_t j = idx >> 1, which = idx & 1u;
            const uint32_t row = which == 0 ? h : nh + h;
            float y8[8];
            psum8(qkv, j0 + j, 4 * H + (row & ~7u), y8);
            float yv = 0.0f;
#pragma unroll
            for (int i = 0; i < 8; ++i) yv = ((uint32_t)i == (row & 7u)) ? y8[i] : yv;
            if (which == 1) {
                sc[j * 4 + 1] = sigmoid_ref(yv);
            } else {
                const float *a_log = aux + 14 * H + 256, *dt_bias = a_log + nh;
                sc[j * 4 + 2] = expf(__fmul_rn(-expf(a_log[h]), softplus_ref(__fadd_rn(yv, dt_bias[h]))));
            }
        }
        __syncthreads();
        /* conv over time + SiLU: token j's window is raw rows j .. j+3 */
        for (uint32_t idx = t; idx < nj * kPrefCh; idx += 256) {
            const uint32_t j = idx / kPrefCh, c = idx % kPrefCh;
            const float4 w = reinterpret_cast<const float4 *>(aux + 2 * H + 256)[(size_t)kind_of(c) * H + gch(c)];
            float sum = __fadd_rn(__fmul_rn(raw[j * kPrefCh + c], w.x), __fmul_rn(raw[(j + 1) * kPrefCh + c], w.y));
            sum = __fadd_rn(sum, __fmul_rn(raw[(j + 2) * kPrefCh + c], w.z));
            sum = __fadd_rn(sum, __fmul_rn(raw[(j + 3) * kPrefCh + c], w.w));
            act[j * kPrefCh + c] = silu_ref(sum);
        }
        __syncthreads();
        /* L2 norms and alpha per token (tree256: 8 per lane, then the butterfly); warp w: tokens w, w + 8 */
        for (uint32_t j = warp; j < nj; j += 8) {
            float *q = act + j * kPrefCh, *k = q + 256;
            float qv[8], kv[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                qv[i] = q[lane * 8 + i];
                kv[i] = k[lane * 8 + i];
            }
            auto tree8 = [](const float (&v)[8], bool sq) -> float {
                float l1[4];
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    l1[i] = sq ? __fadd_rn(__fmul_rn(v[2 * i], v[2 * i]), __fmul_rn(v[2 * i + 1], v[2 * i + 1]))
                               : __fadd_rn(v[2 * i], v[2 * i + 1]);
                return __fadd_rn(__fadd_rn(l1[0], l1[1]), __fadd_rn(l1[2], l1[3]));
            };
            float sq = tree8(qv, true), sk = tree8(kv, true);
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                sq = __fadd_rn(sq, __shfl_xor_sync(0xffffffffu, sq, o));
                sk = __fadd_rn(sk, __shfl_xor_sync(0xffffffffu, sk, o));
            }
            const float qi = __fdiv_rn(1.0f, sqrtf(__fadd_rn(sq, 1e-6f)));
            const float ki = __fdiv_rn(1.0f, sqrtf(__fadd_rn(sk, 1e-6f)));
            float pr[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                qv[i] = __fmul_rn(qv[i], qi);
                kv[i] = __fmul_rn(kv[i], ki);
                pr[i] = __fmul_rn(qv[i], kv[i]);
                q[lane * 8 + i] = qv[i];
                k[lane * 8 + i] = kv[i];
            }
            float al = tree8(pr, false);
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) al = __fadd_rn(al, __shfl_xor_sync(0xffffffffu, al, o));
            if (lane == 0) sc[j * 4] = al;
        }
        __syncthreads();
        /* the recurrence, token by token */
        for (uint32_t j = 0; j < nj; ++j) {
            const float *q = act + j * kPrefCh, *k = q + 256, *v = q + 512;
            const float4 k0 = reinterpret_cast<const float4 *>(k)[lane], k1 = reinterpret_cast<const float4 *>(k)[32 + lane];
            const float4 q0 = reinterpret_cast<const float4 *>(q)[lane], q1 = reinterpret_cast<const float4 *>(q)[32 + lane];
            const float alpha = sc[j * 4], beta = sc[j * 4 + 1], decay = sc[j * 4 + 2];
            float *attn = p.attn + (size_t)(j0 + j) * H + h * 256 + cb * 64 + warp * 8;
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
                const float delta = __fmul_rn(beta, __fsub_rn(v[warp * 8 + i], __fmul_rn(decay, r)));
                if (lane == 0) attn[i] = __fmul_rn(0.0625f, __fadd_rn(__fmul_rn(decay, pp), __fmul_rn(alpha, delta)));
                a0[i].x = __fadd_rn(__fmul_rn(decay, a0[i].x), __fmul_rn(k0.x, delta));
                a0[i].y = __fadd_rn(__fmul_rn(decay, a0[i].y), __fmul_rn(k0.y, delta));
                a0[i].z = __fadd_rn(__fmul_rn(decay, a0[i].z), __fmul_rn(k0.z, delta));
                a0[i].w = __fadd_rn(__fmul_rn(decay, a0[i].w), __fmul_rn(k0.w, delta));
                a1[i].x = __fadd_rn(__fmul_rn(decay, a1[i].x), __fmul_rn(k1.x, delta));
                a1[i].y = __fadd_rn(__fmul_rn(decay, a1[i].y), __fmul_rn(k1.y, delta));
                a1[i].z = __fadd_rn(__fmul_rn(decay, a1[i].z), __fmul_rn(k1.z, delta));
                a1[i].w = __fadd_rn(__fmul_rn(decay, a1[i].w), __fmul_rn(k1.w, delta));
            }
        }
        __syncthreads();
        /* the last three raw rows start the next window */
        for (uint32_t idx = t; idx < 3 * kPrefCh; idx += 256) {
            const uint32_t r = idx / kPrefCh, c = idx % kPrefCh;
            raw[r * kPrefCh + c] = raw[(nj + r) * kPrefCh + c];
        }
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        reinterpret_cast<float4 *>(S + (size_t)i * 256)[lane] = a0[i];
        reinterpret_cast<float4 *>(S + (size_t)i * 256)[32 + lane] = a1[i];
    }
    for (uint32_t c = t; c < (uint32_t)kPrefCh; c += 256) {
        const uint32_t kind = kind_of(c);
        if (kind < 2 && ((c & 255u) >> 6) != cb) continue;  /* q/k tails: this block's quarter */
        reinterpret_cast<float4 *>(tails_out)[((size_t)layer * 3 + kind) * H + gch(c)] =
            make_float4(raw[c], raw[kPrefCh + c], raw[2 * kPrefCh + c], 0.0f);
    }
}

/* Output RMSNorm x swish gate of one head of one stream (c_impl/gdn_model.cpp:
 * 3226-3349): sums of squares per 8 elements, then per 16-element half, the
 * halves summed in order; scale = 1/sqrtf(sum/256 + eps); out = ((a * scale)
 * * w) * g * sigmoid(g), written as activation tiles of the O projection. */
__global__ void __launch_bounds__(32) gate_norm_kernel(const StepParams p, uint32_t layer, const Partials qkv,
                                                       TileOut out) {
    pdl_trigger();
    pdl_wait();
    const uint32_t nh = p.heads, H = p.hidden;
    const uint32_t h = blockIdx.x % nh, s = blockIdx.x / nh, t = threadIdx.x;
    const float *a = p.attn + (size_t)s * H + h * 256 + t * 8;
    const float4 a0 = __ldcg(reinterpret_cast<const float4 *>(a)), a1 = __ldcg(reinterpret_cast<const float4 *>(a) + 1);
    const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
    float g[8];
    psum8(qkv, s, 3 * H + h * 256 + t * 8, g);
    float acc = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) acc = __fadd_rn(acc, __fmul_rn(av[i], av[i]));
    /* halves: lanes (2j, 2j+1); then the 16 halves in order */
    const float half = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 1));
    float sum = 0.0f;
#pragma unroll
    for (int j = 0; j < 16; ++j) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, half, 2 * j));
    const float scale = __fdiv_rn(1.0f, sqrtf(__fadd_rn(__fdiv_rn(sum, 256.0f), p.eps)));
    const float *w = p.aux + (size_t)layer * p.aux_stride + H + t * 8; /* o_norm */
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float nrm = __fmul_rn(__fmul_rn(av[i], scale), w[i]);
        v[i] = __fmul_rn(__fmul_rn(nrm, g[i]), sigmoid_ref(g[i]));
    }
    uint32_t n, npad;
    uint8_t *tiles = pass_tiles(out, s, n, npad);
    put_act8(tiles, npad, n, h * 256 + t * 8, v);
}

/* m_i = silu(gate_i) * up_i (c_impl/gdn_model.cpp:4751-4770; gate row i at 2i,
 * up at 2i + 1), eight m per thread, as activation tiles of the down projection. */
__global__ void __launch_bounds__(256) swiglu_kernel(const StepParams p, const Partials gu, TileOut out) {
    pdl_trigger();
    pdl_wait();
    const uint32_t chunks = p.inter / 8;
    const uint32_t s = blockIdx.x % p.streams, part = blockIdx.x / p.streams;
    const uint32_t c8 = part * 256 + threadIdx.x;
    if (c8 >= chunks) return;
    float lo[8], hi[8];
    psum8(gu, s, c8 * 16, lo);
    psum8(gu, s, c8 * 16 + 8, hi);
    const float y[16] = {lo[0], lo[1], lo[2], lo[3], lo[4], lo[5], lo[6], lo[7],
                         hi[0], hi[1], hi[2], hi[3], hi[4], hi[5], hi[6], hi[7]};
    float m[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) m[i] = __fmul_rn(silu_ref(y[2 * i]), y[2 * i + 1]);
    uint32_t n, npad;
    uint8_t *tiles = pass_tiles(out, s, n, npad);
    put_act8(tiles, npad, n, c8 * 8, m);
}

/* FP32 logits (not rounded) and the per-stream argmax: largest value, lowest
 * row on ties (c_impl/gdn_model.cpp:4775-4925), as a packed key. */
__global__ void __launch_bounds__(256) logits_kernel(const StepParams p, const Partials lm) {
    __shared__ unsigned long long best[8];
    pdl_trigger();
    pdl_wait();
    const uint32_t s = blockIdx.x % p.streams, part = blockIdx.x / p.streams;
    const uint32_t c8 = part * 256 + threadIdx.x;
    unsigned long long key = 0ull;
    if (c8 * 8 < p.vocab) {
        float y[8];
        psum8(lm, s, c8 * 8, y);
        float *dst = p.logits + (size_t)s * p.vocab + c8 * 8;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            if (c8 * 8 + i < p.vocab) {
                dst[i] = y[i];
                const unsigned long long kk = argmax_key(y[i], c8 * 8 + i);
                key = kk > key ? kk : key;
            }
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
        key = other > key ? other : key;
    }
    if ((threadIdx.x & 31) == 0) best[threadIdx.x >> 5] = key;
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned long long b = best[0];
        for (int w = 1; w < 8; ++w) b = best[w] > b ? best[w] : b;
        if (b != 0ull) atomicMax(p.keys + s, b);
    }
}

/* Tokens of the step from the argmax keys; keys cleared; step and tail parity advanced. */
__global__ void __launch_bounds__(256) finish_kernel(const StepParams p) {
    pdl_trigger();
    pdl_wait();
    const uint32_t step = __ldcg(p.step);
    for (uint32_t s = threadIdx.x; s < p.streams; s += 256) {
        const unsigned long long key = __ldcg(p.keys + s);
        p.argmax_out[(size_t)step * p.streams + s] = key ? (int32_t)(0xFFFFFFFFu - (uint32_t)key) : 0;
        p.keys[s] = 0ull;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        *p.step = step + 1;
        *p.tails_parity ^= 1u;
    }
}

}  // namespace

size_t gemm_smem_bytes(uint32_t npad, uint32_t a_slots, uint32_t b_slots) {
    return kSmemAlign + (size_t)a_slots * kABlockBytes + (size_t)b_slots * kTerms * npad * 128u + kSmemTail;
}

void gemm_slots(uint32_t npad, uint32_t *a_slots, uint32_t *b_slots) {
    /* activation blocks come from L2 (a microsecond or more under load): up to
     * 96 KB of them in flight, at least two; the weight ring takes the rest
     * (at most 10 blocks) */
    const size_t bblock = (size_t)kTerms * npad * 128u;
    const size_t budget = kSmemLimit - kSmemAlign - kSmemTail;
    uint32_t sb = (uint32_t)std::max<size_t>(2, std::min<size_t>(8, (96 * 1024) / bblock));
    while (sb > 2 && sb * bblock + 6 * (size_t)kABlockBytes > budget) --sb;
    uint32_t sa = (uint32_t)((budget - sb * bblock) / kABlockBytes);
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

/* Launch with programmatic stream serialization (see pdl_wait). */
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), uint32_t grid, uint32_t block, size_t smem, cudaStream_t stream,
                       Args &&...args) {
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(block);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

cudaError_t launch_gemm(const GemmParams &p, uint32_t grid, cudaStream_t stream) {
    const size_t smem = gemm_smem_bytes(p.npad, p.a_slots, p.b_slots);
    cudaError_t e = cudaFuncSetAttribute(tile_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    return launch_pdl(tile_gemm_kernel, grid, kGemmThreads, smem, stream, p);
}

cudaError_t launch_input(const StepParams &p, const float *norm_w, int mode, const Partials &add, TileOut out,
                         cudaStream_t stream) {
    return launch_pdl(input_kernel, p.streams, 256, 0, stream, p, norm_w, mode, add, out);
}

cudaError_t launch_recur(const StepParams &p, uint32_t layer, const Partials &qkv, float *prep, cudaStream_t stream) {
    cudaError_t e = launch_pdl(prep_kernel, p.streams * p.heads, 128, 0, stream, p, layer, qkv, prep);
    if (e != cudaSuccess) return e;
    return launch_pdl(recur_kernel, p.streams * p.heads * (256 / kRecurCols), 256, 0, stream, p, layer,
                      (const float *)prep);
}

size_t prep_floats(uint32_t streams, uint32_t heads) { return (size_t)streams * heads * kPrepFloats; }

cudaError_t launch_head(const StepParams &p, uint32_t layer, const Partials &qkv, TileOut out, cudaStream_t stream) {
    const cudaError_t e = cudaFuncSetAttribute(head_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kHeadSmem);
    if (e != cudaSuccess) return e;
    return launch_pdl(head_kernel, p.streams * p.heads, 256, kHeadSmem, stream, p, layer, qkv, out);
}

cudaError_t launch_prefill_head(const StepParams &p, uint32_t layer, const Partials &qkv, float *state,
                                const float *tails_in, float *tails_out, uint32_t ntok, cudaStream_t stream) {
    const cudaError_t e =
        cudaFuncSetAttribute(prefill_head_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPrefillSmem);
    if (e != cudaSuccess) return e;
    return launch_pdl(prefill_head_kernel, p.heads * 4, 256, kPrefillSmem, stream, p, layer, qkv, state, tails_in,
                      tails_out, ntok);
}

cudaError_t launch_gate_norm(const StepParams &p, uint32_t layer, const Partials &qkv, TileOut out,
                             cudaStream_t stream) {
    return launch_pdl(gate_norm_kernel, p.streams * p.heads, 32, 0, stream, p, layer, qkv, out);
}

cudaError_t launch_swiglu(const StepParams &p, const Partials &gu, TileOut out, cudaStream_t stream) {
    const uint32_t parts = (p.inter / 8 + 255) / 256;
    return launch_pdl(swiglu_kernel, p.streams * parts, 256, 0, stream, p, gu, out);
}

cudaError_t launch_logits(const StepParams &p, const Partials &lm, cudaStream_t stream) {
    const uint32_t parts = (p.vocab / 8 + 255) / 256 + 1;
    return launch_pdl(logits_kernel, p.streams * parts, 256, 0, stream, p, lm);
}

cudaError_t launch_finish(const StepParams &p, cudaStream_t stream) {
    return launch_pdl(finish_kernel, 1, 256, 0, stream, p);
}

}  // namespace bt
}  // namespace gdn
