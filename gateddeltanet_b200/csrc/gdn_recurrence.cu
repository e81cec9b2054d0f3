/* gdn_recurrence.cu -- the gated delta rule as an isolated step (BASELINE
 * config[1]): for every (layer, head) slice the recurrent state S FP32 is read
 * once and written once, from already L2-normalised q, k, the value v, the
 * decay and beta of the slice (c_impl/gdn_model.cpp:2119-2300):
 *
 *   alpha = tree256(q (.) k)                     (:2119-2124, gdn_tree_reduce_256)
 *   r[v]  = sum_k S[k][v] k[k], p[v] = sum_k S[k][v] q[k], sequential in k
 *                                                (:2184-2210)
 *   delta = beta (v - decay r),  o = (1/16)(decay p + alpha delta)   (:2214-2243)
 *   S'[k][v] = decay S[k][v] + k[k] delta[v]     (:2268-2300)
 *
 * S is stored as the decode engine keeps it, [v][k] (column v of the
 * reference's S[k][v] is 1 KB contiguous). The step is a pipeline: one CTA
 * per SM walks its contiguous range of 32-column blocks. A producer warp
 * stages each block (one 1 KB bulk copy per column, into rows padded by 16
 * bytes so that a lane per column reads without bank conflicts) with the
 * slice's q and k into a 4-slot ring; two warps run the block's r and p
 * chains (a lane per column); four warps load the block's scalars and v
 * ahead, form alpha, delta and the outputs, then update the block and store
 * it with coalesced 16-byte stores while the chain warps are already on the
 * next block. S crosses HBM once each way. (Measured slower: one 32 KB copy
 * per block with the chain lanes skewed against bank conflicts, eight 4 KB
 * copies of padded four-column groups with two pairs of chain warps, six
 * slots. Measured no faster: one TMA tensor copy per block -- a 3-D view of
 * S with the 128-byte swizzle, conflict-free for a lane per column -- in
 * place of the 32 column copies, 27.2 us against 26.3, and with it two
 * pairs of chain warps on alternate blocks, 27.0 us.)
 * Every wait is bounded: a CTA whose copy does not land in 2 s records the
 * error and leaves.
 */
#include "gdn_engine.h"

#include <cuda_runtime.h>
#include <stdint.h>

namespace gdn {

namespace {

constexpr int kDK = 256, kDV = 256;
constexpr int kColsB = 32, kBlocksPerSlice = kDV / kColsB;  /* 32-column blocks */
constexpr int kSlotsDR = 4;
constexpr int kRowB = kDK + 4;                               /* padded column stride, floats (1040 bytes) */
/* warps: 0 the r chains, 1 the p chains, 2..5 alpha / delta / update, 6 the producer */
constexpr int kChainWarps = 2, kUpdWarps = 4, kUpdThreads = kUpdWarps * 32;
constexpr int kThreadsDR = (kChainWarps + kUpdWarps + 1) * 32;
constexpr int kProdWarpDR = kChainWarps + kUpdWarps;
__host__ __device__ constexpr size_t col_off(int c) { return (size_t)c * kRowB * 4; }

/* slot: S block [32][260] | q [256] | k [256] | r [32] | p [32] | delta [32] | alpha partials [4] */
constexpr size_t kSlotS = 0;
constexpr size_t kSlotQ = kSlotS + (size_t)kColsB * kRowB * 4;
constexpr size_t kSlotK = kSlotQ + kDK * 4;
constexpr size_t kSlotR = kSlotK + kDK * 4;
constexpr size_t kSlotP = kSlotR + kColsB * 4;
constexpr size_t kSlotD = kSlotP + kColsB * 4;
constexpr size_t kSlotW = kSlotD + kColsB * 4;
constexpr size_t kSlotBytesDR = (kSlotW + 4 * 4 + 127) & ~(size_t)127;
constexpr size_t kOffBarsDR = kSlotsDR * kSlotBytesDR;  /* full[4] | chains[4] | empty[4] | abort flag */
constexpr size_t kSmemDR = kOffBarsDR + 3 * kSlotsDR * 8 + 16;
constexpr uint64_t kWaitNsDR = 2000000000ull;

__device__ __forceinline__ uint32_t smem_addr(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ uint64_t now_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ bool mbar_test(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred q;\n mbarrier.try_wait.parity.shared::cta.b64 q, [%1], %2, %3;\n selp.u32 %0, 1, 0, q;\n}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(20000u)
        : "memory");
    return ok != 0;
}
/* Warp-wide wait for phase `parity` of a barrier (every lane observes the
 * completion); false on abort, decided by lane 0 for the whole warp: the
 * limit ran out here, or another warp raised the flag. */
__device__ __forceinline__ bool mbar_wait_warp(uint32_t bar, uint32_t parity, volatile int *abort_flag,
                                               const DeltaRuleParams &p) {
    const uint64_t t0 = now_ns();
    bool done = mbar_test(bar, parity);
    while (!__all_sync(0xffffffffu, done)) {
        int stop = 0;
        if ((threadIdx.x & 31) == 0) {
            if (*abort_flag) {
                stop = 1;
            } else if (now_ns() - t0 > kWaitNsDR) {
                *abort_flag = 1;
                atomicExch(p.status, 1);
                stop = 1;
            }
        }
        if (__shfl_sync(0xffffffffu, stop, 0)) return false;
        if (!done) done = mbar_test(bar, parity);
    }
    return true;
}
__device__ __forceinline__ void mbar_arrive1(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
/* barrier of the update warps that also ORs a predicate over them */
__device__ __forceinline__ bool upd_sync_or(bool v) {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred a, b;\n setp.ne.u32 a, %1, 0;\n barrier.red.or.pred b, 1, %2, a;\n selp.u32 %0, 1, 0, b;\n}\n"
        : "=r"(r)
        : "r"((uint32_t)v), "r"(kUpdThreads)
        : "memory");
    return r != 0;
}

__global__ void __launch_bounds__(kThreadsDR, 1) delta_rule_kernel(const __grid_constant__ DeltaRuleParams p) {
    extern __shared__ __align__(128) uint8_t dsm[];
    uint64_t *full = reinterpret_cast<uint64_t *>(dsm + kOffBarsDR);
    uint64_t *chains = full + kSlotsDR, *empty = chains + kSlotsDR;
    volatile int *abort_flag = reinterpret_cast<volatile int *>(empty + kSlotsDR);
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const uint32_t nb = p.slices * kBlocksPerSlice;
    const uint32_t b0 = (uint32_t)(((uint64_t)blockIdx.x * nb) / gridDim.x);
    const uint32_t b1 = (uint32_t)(((uint64_t)(blockIdx.x + 1) * nb) / gridDim.x);
    if (t == 0) {
        for (int i = 0; i < kSlotsDR; ++i) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(&full[i])) : "memory");
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 2;" ::"r"(smem_addr(&chains[i])) : "memory");
            asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(&empty[i])), "r"(kUpdWarps)
                         : "memory");
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    if (warp == kProdWarpDR) {
        /* producer: 32 column copies (a lane each) plus q and k per block */
        for (uint32_t b = b0; b < b1; ++b) {
            const uint32_t i = b - b0, slot = i % kSlotsDR, n = i / kSlotsDR;
            uint8_t *sl = dsm + slot * kSlotBytesDR;
            if (n > 0 && !mbar_wait_warp(smem_addr(&empty[slot]), (n - 1) & 1u, abort_flag, p)) return;
            const uint32_t slice = b / kBlocksPerSlice, cb = b % kBlocksPerSlice;
            if (lane == 0)
                asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(&full[slot])),
                             "r"((uint32_t)((kColsB + 2) * kDK * 4))
                             : "memory");
            __syncwarp();
            /* a column (1 KB, into its padded row) per lane; lanes 0, 1 also q and k */
            const float *src = p.S + ((size_t)slice * kDV + (size_t)cb * kColsB + lane) * kDK;
            asm volatile(
                "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                    smem_addr(sl + kSlotS + col_off(lane))),
                "l"(src), "r"((uint32_t)(kDK * 4)), "r"(smem_addr(&full[slot]))
                : "memory");
            if (lane < 2)
                asm volatile(
                    "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                        smem_addr(sl + (lane == 0 ? kSlotQ : kSlotK))),
                    "l"((lane == 0 ? p.q : p.k) + (size_t)slice * kDK), "r"((uint32_t)(kDK * 4)),
                    "r"(smem_addr(&full[slot]))
                    : "memory");
        }
        return;
    }
    if (warp < kChainWarps) {
        /* warp 0: r = S k, warp 1: p = S q; lane = column, sequential in k */
        const bool is_r = warp == 0;
        for (uint32_t b = b0; b < b1; ++b) {
            const uint32_t i = b - b0, slot = i % kSlotsDR, n = i / kSlotsDR;
            uint8_t *sl = dsm + slot * kSlotBytesDR;
            if (!mbar_wait_warp(smem_addr(&full[slot]), n & 1u, abort_flag, p)) return;
            const float4 *col = reinterpret_cast<const float4 *>(sl + kSlotS + col_off(lane));
            const float4 *vec4 = reinterpret_cast<const float4 *>(sl + (is_r ? kSlotK : kSlotQ));
            float acc = 0.0f;
#pragma unroll 4
            for (int k4 = 0; k4 < kDK / 4; ++k4) {
                const float4 sv = col[k4], xv = vec4[k4];
                acc = __fadd_rn(acc, __fmul_rn(sv.x, xv.x));
                acc = __fadd_rn(acc, __fmul_rn(sv.y, xv.y));
                acc = __fadd_rn(acc, __fmul_rn(sv.z, xv.z));
                acc = __fadd_rn(acc, __fmul_rn(sv.w, xv.w));
            }
            reinterpret_cast<float *>(sl + (is_r ? kSlotR : kSlotP))[lane] = acc;
            __syncwarp();
            if (lane == 0) mbar_arrive1(smem_addr(&chains[slot]));
        }
        return;
    }
    /* warps 2..5: alpha, delta, outputs and the update of every block */
    const int u = t - kChainWarps * 32, uw = u >> 5;
    for (uint32_t b = b0; b < b1; ++b) {
        const uint32_t i = b - b0, slot = i % kSlotsDR, n = i / kSlotsDR;
        uint8_t *sl = dsm + slot * kSlotBytesDR;
        const uint32_t slice = b / kBlocksPerSlice, cb = b % kBlocksPerSlice;
        const float *qs = reinterpret_cast<const float *>(sl + kSlotQ);
        const float *ks = reinterpret_cast<const float *>(sl + kSlotK);
        float *ws = reinterpret_cast<float *>(sl + kSlotW);
        float *ds = reinterpret_cast<float *>(sl + kSlotD);
        /* the block's scalars and v: loaded before the waits, so the round
         * trip overlaps the copy and the chains */
        const size_t vi = (size_t)slice * kDV + (size_t)cb * kColsB + (u & (kColsB - 1));
        const float decay = __ldg(p.decay + slice), beta = __ldg(p.beta + slice), vv = __ldg(p.v + vi);
        bool ok = mbar_wait_warp(smem_addr(&full[slot]), n & 1u, abort_flag, p);
        if (upd_sync_or(!ok)) return;
        /* alpha = tree256(q (.) k): thread u holds elements 2u and 2u+1 (the
         * first level), the warp butterfly the next five, then
         * (w0 + w1) + (w2 + w3) */
        const float2 q2 = reinterpret_cast<const float2 *>(qs)[u], k2 = reinterpret_cast<const float2 *>(ks)[u];
        float a = __fadd_rn(__fmul_rn(q2.x, k2.x), __fmul_rn(q2.y, k2.y));
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) a = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, o));
        if (lane == 0) ws[uw] = a;
        ok = mbar_wait_warp(smem_addr(&chains[slot]), n & 1u, abort_flag, p);
        if (upd_sync_or(!ok)) return;
        const float alpha = __fadd_rn(__fadd_rn(ws[0], ws[1]), __fadd_rn(ws[2], ws[3]));
        if (u < kColsB) {
            const float r = reinterpret_cast<const float *>(sl + kSlotR)[u];
            const float pp = reinterpret_cast<const float *>(sl + kSlotP)[u];
            const float delta = __fmul_rn(beta, __fsub_rn(vv, __fmul_rn(decay, r)));
            p.o[vi] = __fmul_rn(0.0625f, __fadd_rn(__fmul_rn(decay, pp), __fmul_rn(alpha, delta)));
            ds[u] = delta;
        }
        upd_sync_or(false);
        /* update and store: thread u its 16 bytes k = 4 (u & 63) .. +3 of
         * columns (u >> 6) + 2 j -- 512-byte warp stores */
        const int k4 = u & 63;
        const float4 kk = reinterpret_cast<const float4 *>(ks)[k4];
        float *S = p.S + ((size_t)slice * kDV + (size_t)cb * kColsB) * kDK;
#pragma unroll 4
        for (int c = u >> 6; c < kColsB; c += kUpdThreads / 64) {
            const float4 s4 = reinterpret_cast<const float4 *>(sl + kSlotS + col_off(c))[k4];
            const float d = ds[c];
            float4 n4;
            n4.x = __fadd_rn(__fmul_rn(decay, s4.x), __fmul_rn(kk.x, d));
            n4.y = __fadd_rn(__fmul_rn(decay, s4.y), __fmul_rn(kk.y, d));
            n4.z = __fadd_rn(__fmul_rn(decay, s4.z), __fmul_rn(kk.z, d));
            n4.w = __fadd_rn(__fmul_rn(decay, s4.w), __fmul_rn(kk.w, d));
            __stcs(reinterpret_cast<float4 *>(S + (size_t)c * kDK) + k4, n4);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive1(smem_addr(&empty[slot]));
    }
}


}  // namespace

size_t delta_rule_smem_bytes() { return kSmemDR; }

cudaError_t launch_delta_rule(const DeltaRuleParams &p, cudaStream_t stream) {
    cudaError_t e = cudaFuncSetAttribute(delta_rule_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemDR);
    if (e != cudaSuccess) return e;
    int dev = 0, sms = 0;
    if ((e = cudaGetDevice(&dev)) != cudaSuccess) return e;
    if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
    /* one CTA per SM, at most one per block */
    const uint32_t nb = p.slices * kBlocksPerSlice;
    const uint32_t grid = (uint32_t)sms < nb ? (uint32_t)sms : nb;
    delta_rule_kernel<<<grid, kThreadsDR, kSmemDR, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace gdn
