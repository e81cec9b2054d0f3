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
 * reference's S[k][v] is 1 KB contiguous). One CTA per 64-column block of a
 * slice: the 64 columns are staged in shared memory by 1 KB bulk copies into
 * rows padded by 16 bytes (so a lane per column reads conflict-free), two
 * warps run the r chains and two the p chains, then all four update the block
 * and store it with coalesced 16-byte stores. S crosses HBM once each way;
 * three CTAs fit an SM, so one block's copy overlaps another's chains.
 * (Measured slower: a persistent CTA per SM with a three-block ring, fed by
 * bulk or by cp.async copies -- four warps per SM leave the chains exposed.)
 */
#include "gdn_engine.h"

#include <cuda_runtime.h>
#include <stdint.h>

namespace gdn {

namespace {

constexpr int kDK = 256, kDV = 256, kCols = 64, kBlocksPerSlice = kDV / kCols;
constexpr int kThreadsDR = 128;

__device__ __forceinline__ uint32_t smem_addr(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

/* shared memory: S block [64][256 + 4] | q [256] | k [256] | r [64] | p [64] | delta [64] | warp partials [4] */
constexpr int kRow = kDK + 4;  /* padded column stride in floats (1040 bytes) */
constexpr size_t kOffS = 0;
constexpr size_t kOffQ = kOffS + (size_t)kCols * kRow * 4;
constexpr size_t kOffK = kOffQ + kDK * 4;
constexpr size_t kOffR = kOffK + kDK * 4;
constexpr size_t kOffP = kOffR + kCols * 4;
constexpr size_t kOffD = kOffP + kCols * 4;
constexpr size_t kOffW = kOffD + kCols * 4;
constexpr size_t kOffBar = (kOffW + 4 * 4 + 7) & ~(size_t)7;
constexpr size_t kSmemDR = kOffBar + 8;
constexpr uint64_t kWaitNsDR = 2000000000ull;

__device__ __forceinline__ uint64_t now_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__global__ void __launch_bounds__(kThreadsDR) delta_rule_kernel(const __grid_constant__ DeltaRuleParams p) {
    extern __shared__ __align__(128) uint8_t dsm[];
    float *sb = reinterpret_cast<float *>(dsm + kOffS);
    float *qs = reinterpret_cast<float *>(dsm + kOffQ);
    float *ks = reinterpret_cast<float *>(dsm + kOffK);
    float *rs = reinterpret_cast<float *>(dsm + kOffR);
    float *ps = reinterpret_cast<float *>(dsm + kOffP);
    float *ds = reinterpret_cast<float *>(dsm + kOffD);
    float *ws = reinterpret_cast<float *>(dsm + kOffW);
    uint64_t *bar = reinterpret_cast<uint64_t *>(dsm + kOffBar);
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const uint32_t slice = blockIdx.x / kBlocksPerSlice, cb = blockIdx.x % kBlocksPerSlice;
    /* the block: columns cb*64 .. cb*64+63 of the slice, 1 KB each */
    float *S = p.S + (size_t)slice * kDK * kDV + (size_t)cb * kCols * kDK;

    if (t == 0) {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(bar)) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    if (warp == 0) {
        /* lane 0 posts the byte count, then every lane copies two columns */
        if (lane == 0)
            asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
                         "r"((uint32_t)(kCols * kDK * 4))
                         : "memory");
        __syncwarp();
#pragma unroll
        for (int j = 0; j < kCols / 32; ++j) {
            const int c = lane + 32 * j;
            asm volatile(
                "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                    smem_addr(sb + (size_t)c * kRow)),
                "l"(S + (size_t)c * kDK), "r"((uint32_t)(kDK * 4)), "r"(smem_addr(bar))
                : "memory");
        }
    }
    /* q, k of the slice, and alpha = tree256(q (.) k): thread t holds elements
     * 2t and 2t+1 (first tree level), the warp butterfly the next five, then
     * (w0 + w1) + (w2 + w3) */
    const float2 q2 = reinterpret_cast<const float2 *>(p.q + (size_t)slice * kDK)[t];
    const float2 k2 = reinterpret_cast<const float2 *>(p.k + (size_t)slice * kDK)[t];
    reinterpret_cast<float2 *>(qs)[t] = q2;
    reinterpret_cast<float2 *>(ks)[t] = k2;
    float a = __fadd_rn(__fmul_rn(q2.x, k2.x), __fmul_rn(q2.y, k2.y));
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) a = __fadd_rn(a, __shfl_xor_sync(0xffffffffu, a, o));
    if (lane == 0) ws[warp] = a;
    __syncthreads();
    const float alpha = __fadd_rn(__fadd_rn(ws[0], ws[1]), __fadd_rn(ws[2], ws[3]));

    /* wait for the block; bounded: after the limit the CTA records the error
     * and leaves (a bulk copy that has not landed in 2 s is not waited for
     * any longer) */
    {
        const uint64_t t0 = now_ns();
        uint32_t done = 0;
        bool timed_out = false;
        while (true) {
            asm volatile(
                "{\n .reg .pred q;\n mbarrier.try_wait.parity.shared::cta.b64 q, [%1], 0;\n selp.u32 %0, 1, 0, q;\n}\n"
                : "=r"(done)
                : "r"(smem_addr(bar))
                : "memory");
            if (done) break;
            if (now_ns() - t0 > kWaitNsDR) {
                timed_out = true;
                break;
            }
        }
        if (__syncthreads_or(timed_out)) {
            if (t == 0) atomicExch(p.status, 1);
            return;
        }
    }

    /* read pass: warps 0-1 the r chains, warps 2-3 the p chains, lane = column */
    {
        const int c = t & (kCols - 1);
        const float4 *col = reinterpret_cast<const float4 *>(sb + (size_t)c * kRow);
        const float4 *vec4 = reinterpret_cast<const float4 *>((warp < 2) ? ks : qs);
        float acc = 0.0f;
#pragma unroll 4
        for (int k4 = 0; k4 < kDK / 4; ++k4) {
            const float4 sv = col[k4], xv = vec4[k4];
            acc = __fadd_rn(acc, __fmul_rn(sv.x, xv.x));
            acc = __fadd_rn(acc, __fmul_rn(sv.y, xv.y));
            acc = __fadd_rn(acc, __fmul_rn(sv.z, xv.z));
            acc = __fadd_rn(acc, __fmul_rn(sv.w, xv.w));
        }
        ((warp < 2) ? rs : ps)[c] = acc;
    }
    __syncthreads();
    const float decay = p.decay[slice], beta = p.beta[slice];
    if (t < kCols) {
        const size_t vi = (size_t)slice * kDV + (size_t)cb * kCols + t;
        const float delta = __fmul_rn(beta, __fsub_rn(p.v[vi], __fmul_rn(decay, rs[t])));
        p.o[vi] = __fmul_rn(0.0625f, __fadd_rn(__fmul_rn(decay, ps[t]), __fmul_rn(alpha, delta)));
        ds[t] = delta;
    }
    __syncthreads();
    /* update and store: thread t its 16 bytes k = 4 (t & 63) .. +3 of columns
     * (t >> 6) + 2 i -- 512-byte warp stores */
    const int k4 = t & 63;
    const float4 kk = reinterpret_cast<const float4 *>(ks)[k4];
#pragma unroll 4
    for (int c = t >> 6; c < kCols; c += kThreadsDR / 64) {
        const float4 s4 = reinterpret_cast<const float4 *>(sb + (size_t)c * kRow)[k4];
        const float d = ds[c];
        float4 n4;
        n4.x = __fadd_rn(__fmul_rn(decay, s4.x), __fmul_rn(kk.x, d));
        n4.y = __fadd_rn(__fmul_rn(decay, s4.y), __fmul_rn(kk.y, d));
        n4.z = __fadd_rn(__fmul_rn(decay, s4.z), __fmul_rn(kk.z, d));
        n4.w = __fadd_rn(__fmul_rn(decay, s4.w), __fmul_rn(kk.w, d));
        __stcs(reinterpret_cast<float4 *>(S + (size_t)c * kDK) + k4, n4);
    }
}

}  // namespace

size_t delta_rule_smem_bytes() { return kSmemDR; }

cudaError_t launch_delta_rule(const DeltaRuleParams &p, cudaStream_t stream) {
    const cudaError_t e =
        cudaFuncSetAttribute(delta_rule_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemDR);
    if (e != cudaSuccess) return e;
    delta_rule_kernel<<<p.slices * kBlocksPerSlice, kThreadsDR, kSmemDR, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace gdn
