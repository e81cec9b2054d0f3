/* gdn_score.cu -- teacher-forced scoring on the device (c_impl/host.cpp:
 * 1954-1994, score_window_hw): after a decode step, the log-probability of the
 * next token under the step's FP32 logits, log-softmax in double:
 *   m = max_v logits[v], sum = sum_v exp((double)logits[v] - m),
 *   logprob += ((double)logits[target] - m) - log(sum)
 * accumulated into acc[0] (acc[1] counts the scored tokens). One CTA; the
 * reference's sequential sums become a tree (double: the order shows only in
 * the last bits). */
#include <cuda_runtime.h>
#include <stdint.h>

namespace gdn {

namespace {

constexpr int kScoreThreads = 1024;

__global__ void __launch_bounds__(kScoreThreads) score_kernel(const float *__restrict__ logits, uint32_t V,
                                                              const int32_t *__restrict__ target, double *acc) {
    __shared__ float wmax[32];
    __shared__ double wsum[32];
    const uint32_t t = threadIdx.x, lane = t & 31, warp = t >> 5;
    float m = -3.402823466e38f;
    for (uint32_t v = t; v < V; v += kScoreThreads) m = fmaxf(m, logits[v]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) wmax[warp] = m;
    __syncthreads();
    m = wmax[0];
    for (int w = 1; w < kScoreThreads / 32; ++w) m = fmaxf(m, wmax[w]);
    const double md = (double)m;
    double s = 0.0;
    for (uint32_t v = t; v < V; v += kScoreThreads) s += exp((double)logits[v] - md);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) wsum[warp] = s;
    __syncthreads();
    if (t == 0) {
        double sum = 0.0;
        for (int w = 0; w < kScoreThreads / 32; ++w) sum += wsum[w];
        const int32_t tg = *target;
        acc[0] += ((double)logits[tg] - md) - log(sum);
        acc[1] += 1.0;
    }
}

}  // namespace

cudaError_t launch_score(const float *logits, uint32_t V, const int32_t *target, double *acc, cudaStream_t stream) {
    score_kernel<<<1, kScoreThreads, 0, stream>>>(logits, V, target, acc);
    return cudaGetLastError();
}

}  // namespace gdn
