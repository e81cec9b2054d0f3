/* gdn_decode.cu -- one GatedDeltaNet decode token as a single persistent
 * sm_100a kernel.
 *
 * The reference computes a token as 24 x {a/b + QKVG GEMV with short conv and
 * gated delta rule, output norm/gate, o_proj, residual + norm, gate/up with
 * SwiGLU, down, residual + norm} and an LM head with argmax
 * (c_impl/gdn_model.cpp:3532-3897). At batch 1 every step is bound by HBM
 * bytes (2.8 GB of BF16 weights + the recurrent state per token), so the
 * kernel is organised around keeping HBM busy:
 *
 *   - grid = one CTA per SM, launched cooperatively; each CTA owns a fixed
 *     slice of every phase's rows and of the recurrent state's columns;
 *   - warp 15 of every CTA is the producer: one lane walks the CTA's whole
 *     token schedule (built once per launch in shared memory) and streams
 *     each chunk (up to 32 KB) into a 4-slot shared-memory ring with one
 *     cp.async.bulk copy per chunk (mbarrier completion, evict-first L2
 *     policy for weights, evict-last for the state). Weights do not depend
 *     on activations, so it runs ahead across phase boundaries while the
 *     consumers wait for inputs;
 *   - warps 0..14 consume every chunk together, each on its own rows, so a
 *     slot is held only while the CTA works on it. A chunk holds a column
 *     block of all the CTA's rows; each lane owns one of a row's four bank
 *     chains (c_impl/gdn_model.cpp:4444-4586) and keeps it in a register
 *     across the chunks, so the reference's reduction order costs no shared
 *     memory traffic. The O and DOWN projections (a dozen rows per CTA)
 *     instead give a warp one row and eight column groups per chunk; the
 *     chain's eight tree16 values are gathered by warp shuffles.
 *
 * Phases per layer l: A QKVG rows (+ short conv, SiLU), B a/b rows and the
 * state columns (gated delta rule), C O rows, D gate/up row pairs (SwiGLU),
 * E down rows; after the last layer the LM head. There is no grid barrier: a
 * phase's outputs travel as words that carry the phase's tag next to the
 * value (32-bit {BF16, 16-bit tag} words in the BF16-boundary contracts,
 * 64-bit {FP32, 32-bit tag} in the FP32 one), and each consumer CTA polls the
 * words it needs. A CTA cannot run
 * more than one phase ahead of any CTA it reads from, so exchange buffers are
 * reused every layer without write-after-read hazards; the residual stream
 * lives in each CTA's shared memory (every CTA computes it identically).
 *
 * Every wait (mbarrier, exchange word) is bounded by %globaltimer; on expiry
 * the kernel records an error in DecodeStatus, stops issuing copies, waits
 * for the copies already in flight and returns. The host reports -1.
 */
#include "gdn_engine.h"
#include "gdn_math.h"

#include <atomic>
#include <cuda_runtime.h>
#include <type_traits>
#include <stdint.h>

namespace gdn {
constexpr uint64_t kWaitNs = 2000000000ull;  /* 2 s: normal waits are microseconds */
/* The producer waits for slots the consumers hold; a consumer stuck on its
 * inputs gives up (and reports why) first. */
constexpr uint64_t kSlotWaitNs = 2 * kWaitNs;

/* MODE bits: 1 BF16 boundaries, 2 BF16-rounded products, 4 tensor-parallel,
 * 8 BF16 state storage. Instantiated: 0 (FP32 control), 1 (engine), 11 (the
 * c_impl contract) and their tensor-parallel forms 4, 5, 15. */
template <int MODE>
struct Mode {
    static constexpr bool kBf16 = (MODE & 1) != 0;
    static constexpr bool kNative = (MODE & 2) != 0;
    static constexpr bool kTp = (MODE & 4) != 0;
    static constexpr bool kBf16State = (MODE & 8) != 0;
};

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
__device__ __forceinline__ void mbar_arrive_n(uint32_t bar, uint32_t n) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(n) : "memory");
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
/* The same test, suspending the thread in hardware (up to `ns`) until the
 * phase completes, so that waiting warps take no issue slots. */
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, uint32_t ns) {
    uint32_t ok;
    asm volatile(
        "{\n"
        " .reg .pred p;\n"
        " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
        " selp.u32 %0, 1, 0, p;\n"
        "}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(ns)
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
__device__ __forceinline__ int ld_volatile_i32(const int32_t *p) {
    return *(const volatile int32_t *)p;
}
__device__ __forceinline__ uint4 lds128(const uint8_t *p) { return *reinterpret_cast<const uint4 *>(p); }
/* 16-byte asynchronous global -> shared copies (L2-coherent), waited for by
 * the issuing thread */
__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

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
    return Mode<MODE>::kBf16 ? bf16_round(v) : v;
}
__device__ __forceinline__ float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

/* The reference's BF16 x BF16 -> BF16 product with its special cases, DAZ and
 * FTZ (gdn_native_bf16_product_bits, c_impl/gdn_model.cpp:392-462), as FP32.
 * The exact emulation, used only for phase inputs outside the fast path's
 * range. */
__device__ __noinline__ float native_product(uint32_t lhs, uint32_t rhs) {
    const uint32_t le = (lhs >> 7) & 0xffu, re = (rhs >> 7) & 0xffu;
    const bool lnan = le == 0xffu && (lhs & 0x7fu), rnan = re == 0xffu && (rhs & 0x7fu);
    const bool linf = le == 0xffu && !(lhs & 0x7fu), rinf = re == 0xffu && !(rhs & 0x7fu);
    const bool lz = le == 0, rz = re == 0;
    const uint32_t sign = (lhs ^ rhs) & 0x8000u;
    if (lnan || rnan || (linf && rz) || (rinf && lz)) return __uint_as_float(0x7fc00000u);
    if (linf || rinf) return __uint_as_float((sign | 0x7f80u) << 16);
    if (lz || rz) return __uint_as_float(sign << 16);
    const float prod = __fmul_rn(__uint_as_float(lhs << 16), __uint_as_float(rhs << 16));
    const uint32_t pb = __float_as_uint(prod), mag = pb & 0x7fffffffu;
    if (mag == 0x7f800000u) return __uint_as_float(pb & 0xffff0000u);
    if (mag < 0x007fc000u) return __uint_as_float(pb & 0x80000000u);
    const uint32_t res = ((pb + 0x7fffu + ((pb >> 16) & 1u)) >> 16) & 0xffffu;
    if ((res & 0x7f80u) == 0) return __uint_as_float((res & 0x8000u) << 16);
    return __uint_as_float(res << 16);
}

/* exp table (2^(j/64) as hi | lo) staged in shared memory at kernel start */
__device__ __forceinline__ const float *exp_table();

/* exp / sigmoid / silu / softplus of the reference (c_impl/gdn_model.cpp:
 * 1307-1330) on the primitives of gdn_math.h (the FP32 control contract). */
__device__ __forceinline__ float exp_ref(float x) { return gdn_expf(x, exp_table()); }
__device__ __forceinline__ float sigmoid_ref(float x) { return gdn_sigmoidf(x, exp_table()); }
__device__ __forceinline__ float softplus_ref(float x) {
    if (x > 20.0f) return x;
    if (x < -20.0f) return exp_ref(x);
    return log1pf(exp_ref(x));
}

/* ---------------------------------------- exp as the host C library rounds it
 *
 * The reference evaluates expf with the host C library, which rounds a small
 * fraction of inputs (7.6e-5 of them) to the neighbour of the correctly
 * rounded value. The kernel's exp (gdn_expf_zone) is correctly rounded outside
 * a narrow zone around rounding boundaries and reports when an input is in it
 * (0.4 % of inputs; every input the library rounds the other way lies in it).
 * There the value is recomputed in double precision, and the other
 * neighbour is taken for the inputs on the host-built exception list. */

/* The float neighbour of e = RN(d) on d's side, for d > 0. */
__device__ __forceinline__ float exp_neighbour(float e, double d) {
    const double ed = (double)e;
    if (d > ed) return __uint_as_float(__float_as_uint(e) + 1u);
    if (d < ed && e > 0.0f) return __uint_as_float(__float_as_uint(e) - 1u);
    return e;
}

/* Binary search of the host-built exception list (global memory). */
__device__ __noinline__ bool exp_exc_contains(const DecodeParams &p, float a) {
    const uint32_t key = __float_as_uint(a);
    uint32_t lo = 0, hi = p.exp_exc_n;
    while (lo < hi) {
        const uint32_t mid = (lo + hi) >> 1;
        const uint32_t v = __ldg(p.exp_exc + mid);
        if (v == key) return true;
        if (v < key) lo = mid + 1;
        else hi = mid;
    }
    return false;
}

/* sigmoid(x) of a BF16-valued x as the reference computes it with the host
 * library (beta, the output gate, SwiGLU). Of the BF16 inputs only the
 * handful in p.exp_exc_bf16 round differently, so the check is a short scan. */
__device__ __noinline__ float exp_bf16in_slow(const DecodeParams &p, float a) {
    const double d = exp((double)a);
    const float e = __double2float_rn(d);
    const uint32_t key = __float_as_uint(a);
    for (uint32_t i = 0; i < p.exp_exc_bf16_n; ++i)
        if (p.exp_exc_bf16[i] == key) return exp_neighbour(e, d);
    return e;
}
__device__ __forceinline__ float sigmoid_bf16in(const DecodeParams &p, float x) {
    const bool pos = x >= 0.0f;
    const float a = pos ? -x : x;
    bool zone;
    float z = gdn_expf_zone(a, exp_table(), &zone);
    if (zone) {
        z = exp_bf16in_slow(p, a);
        return __fdiv_rn(pos ? 1.0f : z, __fadd_rn(1.0f, z));
    }
    return gdn_divf(pos ? 1.0f : z, __fadd_rn(1.0f, z));
}

/* BF16 output of silu(x) = x * sigmoid(x) for an arbitrary FP32 x (the
 * short conv, c_impl/gdn_model.cpp:1630-1653) as the reference computes it.
 * In the doubt zone both candidate exps are tried; only when they give
 * different BF16 outputs is the full exception list searched. */
template <int MODE>
__device__ __noinline__ float silu_conv_slow(const DecodeParams &p, float x, float a) {
    const bool pos = x >= 0.0f;
    const double d = exp((double)a);
    const float e = __double2float_rn(d);
    const float alt = exp_neighbour(e, d);
    const float o1 = bnd<MODE>(__fmul_rn(x, __fdiv_rn(pos ? 1.0f : e, __fadd_rn(1.0f, e))));
    if (alt == e) return o1;
    const float o2 = bnd<MODE>(__fmul_rn(x, __fdiv_rn(pos ? 1.0f : alt, __fadd_rn(1.0f, alt))));
    if (__float_as_uint(o1) == __float_as_uint(o2)) return o1;
    return exp_exc_contains(p, a) ? o2 : o1;
}
template <int MODE>
__device__ __forceinline__ float silu_conv(const DecodeParams &p, float x) {
    if (!Mode<MODE>::kBf16) return bnd<MODE>(__fmul_rn(x, sigmoid_ref(x)));
    const bool pos = x >= 0.0f;
    const float a = pos ? -x : x;
    bool zone;
    const float z = gdn_expf_zone(a, exp_table(), &zone);
    if (zone) return silu_conv_slow<MODE>(p, x, a);
    return bnd<MODE>(__fmul_rn(x, gdn_divf(pos ? 1.0f : z, __fadd_rn(1.0f, z))));
}
/* sigmoid of a BF16-valued input in the selected contract */
template <int MODE>
__device__ __forceinline__ float sigmoid_b(const DecodeParams &p, float x) {
    return Mode<MODE>::kBf16 ? sigmoid_bf16in(p, x) : sigmoid_ref(x);
}

/* ------------------------------------------------ GEMV product kernels */

/* w.lo * x.lo + w.hi * x.hi of packed BF16 pairs as the reference's pair sum
 * (lo product + hi product, both exact, one rounding): mixed-precision FMA
 * with BF16 multiplicands and FP32 addend; the first FMA adds -0.0 so an
 * exact zero product keeps its sign. */
__device__ __forceinline__ float pair_sum(uint32_t w, uint32_t x) {
    float d;
    asm("{\n .reg .b16 wl, wh, xl, xh;\n mov.b32 {wl, wh}, %1;\n mov.b32 {xl, xh}, %2;\n"
        " fma.rn.f32.bf16 %0, wl, xl, 0f80000000;\n fma.rn.f32.bf16 %0, wh, xh, %0;\n}"
        : "=f"(d)
        : "r"(w), "r"(x));
    return d;
}
/* The c_impl pair sum: both products rounded to BF16 (RNE) by the packed BF16
 * multiply, then added once in FP32 (lo + hi exactly as hi * 1 + lo). Equal
 * to the reference's product (c_impl/gdn_model.cpp:392-462) whenever no
 * product falls below the normal range; the kernel checks that per phase. */
__device__ __forceinline__ float pair_sum_native(uint32_t w, uint32_t x) {
    float d;
    asm("{\n .reg .b32 p, lo;\n .reg .b16 pl, ph, one;\n mul.rn.bf16x2 p, %1, %2;\n"
        " shl.b32 lo, p, 16;\n mov.b32 {pl, ph}, p;\n mov.b16 one, 0x3f80;\n"
        " fma.rn.f32.bf16 %0, ph, one, lo;\n}"
        : "=f"(d)
        : "r"(w), "r"(x));
    return d;
}
__device__ __forceinline__ float pair_sum_exact_native(uint32_t w, uint32_t x) {
    return __fadd_rn(native_product(w & 0xffffu, x & 0xffffu), native_product(w >> 16, x >> 16));
}

/* tree16 of one 16-column half (gemv32_tree16, c_impl/gdn_model.cpp:4004-4035):
 * ((s0+s1)+(s2+s3)) + ((s4+s5)+(s6+s7)) over the eight pair sums, from
 * packed BF16 weights (w0: columns 0..7, w1: 8..15) and inputs. KIND 0:
 * exact products (engine), 1: BF16-rounded products (c_impl), 2: the exact
 * emulation of the c_impl product. */
template <int KIND>
__device__ __forceinline__ float ps(uint32_t w, uint32_t x) {
    return KIND == 0 ? pair_sum(w, x) : KIND == 1 ? pair_sum_native(w, x) : pair_sum_exact_native(w, x);
}
template <int KIND>
__device__ __forceinline__ float tree16_bf(const uint4 &w0, const uint4 &w1, const uint4 &x0, const uint4 &x1) {
    const float s0 = ps<KIND>(w0.x, x0.x), s1 = ps<KIND>(w0.y, x0.y), s2 = ps<KIND>(w0.z, x0.z),
                s3 = ps<KIND>(w0.w, x0.w);
    const float s4 = ps<KIND>(w1.x, x1.x), s5 = ps<KIND>(w1.y, x1.y), s6 = ps<KIND>(w1.z, x1.z),
                s7 = ps<KIND>(w1.w, x1.w);
    const float a0 = __fadd_rn(s0, s1), a1 = __fadd_rn(s2, s3), a2 = __fadd_rn(s4, s5), a3 = __fadd_rn(s6, s7);
    return __fadd_rn(__fadd_rn(a0, a1), __fadd_rn(a2, a3));
}
/* The FP32 control: BF16 weights times FP32 inputs (16 floats), each product
 * rounded to FP32, then the same tree. */
__device__ __forceinline__ float pair_f32(uint32_t w, float xa, float xb) {
    return __fadd_rn(__fmul_rn(bf_lo(w), xa), __fmul_rn(bf_hi(w), xb));
}
__device__ __forceinline__ float tree16_f32(const uint4 &w0, const uint4 &w1, const float4 &x0, const float4 &x1,
                                            const float4 &x2, const float4 &x3) {
    const float s0 = pair_f32(w0.x, x0.x, x0.y), s1 = pair_f32(w0.y, x0.z, x0.w);
    const float s2 = pair_f32(w0.z, x1.x, x1.y), s3 = pair_f32(w0.w, x1.z, x1.w);
    const float s4 = pair_f32(w1.x, x2.x, x2.y), s5 = pair_f32(w1.y, x2.z, x2.w);
    const float s6 = pair_f32(w1.z, x3.x, x3.y), s7 = pair_f32(w1.w, x3.z, x3.w);
    const float a0 = __fadd_rn(s0, s1), a1 = __fadd_rn(s2, s3), a2 = __fadd_rn(s4, s5), a3 = __fadd_rn(s6, s7);
    return __fadd_rn(__fadd_rn(a0, a1), __fadd_rn(a2, a3));
}

/* ------------------------------------------------------ exchange words */

/* The BF16-boundary contracts only ever exchange BF16-exact values, so their
 * word is 32 bits: the value's upper half and a 16-bit tag (the low half of
 * epoch + phase; a word always holds either this launch's tag or the
 * previous launch's, which differs by the epoch stride). The FP32 contract
 * uses 64-bit words {FP32 value, 32-bit tag}. Either way one aligned store
 * publishes value and tag together. The buffers are sized for 64-bit words;
 * a 32-bit-word contract uses the first half of each. */
template <int MODE, bool B = Mode<MODE>::kBf16>
struct XW {
    typedef unsigned long long T;
};
template <int MODE>
struct XW<MODE, true> {
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
    if (Mode<MODE>::kTp)
        for (int r = 0; r < p.tp_world; ++r)
            if (r != p.tp_rank) xstore_sys(peer_addr(p, a, r), w);
}
/* store gate element i: in the BF16-boundary contracts with sigmoid(g)
 * beside it (gword), so the output gate's consumers need no exp */
template <int MODE>
__device__ __forceinline__ void xput_gate(const DecodeParams &p, size_t i, float g, float sg, uint32_t tag) {
    if (!Mode<MODE>::kBf16) {
        xput<MODE>(p, p.gate, i, g, tag);
        return;
    }
    unsigned long long *a = reinterpret_cast<unsigned long long *>(p.gate) + i;
    const unsigned long long w =
        ((unsigned long long)((__float_as_uint(g) & 0xffff0000u) | (tag & 0xffffu)) << 32) | __float_as_uint(sg);
    xstore(a, w);
    if (Mode<MODE>::kTp)
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
/* The gate words of the BF16-boundary contracts are 64 bits: sigmoid(g) as
 * FP32 in the low half (computed once, by the CTA that computes the gate
 * row), the BF16 g and the 16-bit tag in the high half. */
struct gword {
    unsigned long long v;
};
__device__ __forceinline__ gword xget(const gword *p, bool sys) {
    return gword{xget(reinterpret_cast<const unsigned long long *>(p), sys)};
}
__device__ __forceinline__ bool xtag_is(gword w, uint32_t tag) { return ((uint32_t)(w.v >> 32) & 0xffffu) == (tag & 0xffffu); }
__device__ __forceinline__ float gword_g(gword w) { return __uint_as_float((uint32_t)(w.v >> 32) & 0xffff0000u); }
__device__ __forceinline__ float gword_sig(gword w) { return __uint_as_float((uint32_t)w.v); }
__device__ __forceinline__ bool xtag_is(uint32_t w, uint32_t tag) { return (w & 0xffffu) == (tag & 0xffffu); }
__device__ __forceinline__ bool xtag_is(unsigned long long w, uint32_t tag) { return (uint32_t)(w >> 32) == tag; }
__device__ __forceinline__ float xval(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }
__device__ __forceinline__ float xval(unsigned long long w) { return __uint_as_float((uint32_t)w); }

/* ------------------------------------------------------- shared memory */

/* Every region sits at a compile-time offset (region pointers fold into
 * immediate addresses); only the size of the last region, xs, depends on the
 * shape. */
constexpr size_t kMaxHidden = 2048;
constexpr size_t kOffRing = 0;
constexpr size_t kOffXres = kOffRing + (size_t)kSlots * kSlotBytes;      /* residual stream, H floats */
constexpr size_t kOffScratch = kOffXres + kMaxHidden * 4;               /* 8 KB, per phase */
constexpr size_t kOffRed = kOffScratch + kMaxHidden * 4;                 /* 320 floats */
constexpr size_t kOffHscal = kOffRed + 320 * 4;                          /* 64 floats */
constexpr size_t kOffWbest = kOffHscal + 64 * 4;                         /* 16 floats */
constexpr size_t kOffWbestI = kOffWbest + 16 * 4;                        /* 16 ints */
constexpr size_t kOffBars = kOffWbestI + 16 * 4;                         /* full[kSlots], empty[kSlots] */
constexpr size_t kOffIssued = kOffBars + 2 * kSlots * 8;                 /* [kSlots] u32 */
constexpr size_t kOffFlags = kOffIssued + kSlots * 4;                    /* abort, decision, exact[2] */
constexpr size_t kOffSched = (kOffFlags + 16 + 15) & ~(size_t)15;        /* the CTA's Sched (256 bytes) */
constexpr size_t kOffExpTab = kOffSched + 256;                           /* 128 floats */
constexpr size_t kOffNormW = kOffExpTab + 128 * 4;                       /* next RMSNorm weights, H floats */
constexpr size_t kOffONorm = kOffNormW + kMaxHidden * 4;                 /* next output-norm weights, 256 */
constexpr size_t kOffXs = kOffONorm + kHeadDim * 4;                      /* phase input */
constexpr size_t kSplitBytes = 28672;  /* tensor-parallel launches: split GEMV tree16 values, after xs */

extern __shared__ __align__(128) uint8_t smem_raw[];

__device__ __forceinline__ uint8_t *sm_slot(uint32_t s) { return smem_raw + kOffRing + (size_t)s * kSlotBytes; }
__device__ __forceinline__ float *sm_xres() { return reinterpret_cast<float *>(smem_raw + kOffXres); }
__device__ __forceinline__ float *sm_scratch() { return reinterpret_cast<float *>(smem_raw + kOffScratch); }
/* phase B: normalised q and k of the CTA's (at most two) heads, then the a/b
 * tree16 values [4][H/16] */
__device__ __forceinline__ float *sm_qn() { return sm_scratch(); }
__device__ __forceinline__ float *sm_kn() { return sm_scratch() + 2 * kHeadDim; }
__device__ __forceinline__ float *sm_park() { return sm_scratch() + 4 * kHeadDim; }
__device__ __forceinline__ float *sm_red() { return reinterpret_cast<float *>(smem_raw + kOffRed); }
/* [hs * 8 + {0 alpha, 1 beta, 2 decay, 3 a, 4 b}] per local head; [16 + j]
 * delta of state column j */
__device__ __forceinline__ float *sm_hscal() { return reinterpret_cast<float *>(smem_raw + kOffHscal); }
__device__ __forceinline__ float *sm_wbest() { return reinterpret_cast<float *>(smem_raw + kOffWbest); }
__device__ __forceinline__ int32_t *sm_wbest_i() { return reinterpret_cast<int32_t *>(smem_raw + kOffWbestI); }
__device__ __forceinline__ uint64_t *sm_full() { return reinterpret_cast<uint64_t *>(smem_raw + kOffBars); }
__device__ __forceinline__ uint64_t *sm_empty() { return reinterpret_cast<uint64_t *>(smem_raw + kOffBars) + kSlots; }
__device__ __forceinline__ volatile uint32_t *sm_issued() {
    return reinterpret_cast<volatile uint32_t *>(smem_raw + kOffIssued);
}
/* set by any thread of the CTA that gives up */
__device__ __forceinline__ volatile int32_t *sm_abort_flag() {
    return reinterpret_cast<volatile int32_t *>(smem_raw + kOffFlags);
}
/* thread 0's CTA-uniform go/stop, read after a barrier */
__device__ __forceinline__ volatile int32_t *sm_decision() {
    return reinterpret_cast<volatile int32_t *>(smem_raw + kOffFlags + 4);
}
/* [phase parity]: 1 when the phase's GEMV input is outside the BF16 fast
 * path's range (two flags, so the next phase's is cleared while nobody reads
 * it) */
__device__ __forceinline__ volatile int32_t *sm_exact() {
    return reinterpret_cast<volatile int32_t *>(smem_raw + kOffFlags + 8);
}
__device__ __forceinline__ const float *exp_table() {
    return reinterpret_cast<const float *>(smem_raw + kOffExpTab);
}
__device__ __forceinline__ uint8_t *sm_xs() { return smem_raw + kOffXs; }
__device__ __forceinline__ size_t xs_bytes(int H, int I) { return ((size_t)4 * (H > I ? H : I) + 15) & ~(size_t)15; }
__device__ __forceinline__ float *sm_split(const DecodeParams &p) {
    return reinterpret_cast<float *>(smem_raw + kOffXs + xs_bytes(p.H, p.I));
}
/* Norm weights, copied in (cp.async) right after their previous user's
 * prologue: a global load in a prologue costs a round trip through a memory
 * system saturated by the ring's copies */
__device__ __forceinline__ float *sm_normw() { return reinterpret_cast<float *>(smem_raw + kOffNormW); }
__device__ __forceinline__ float *sm_onorm() { return reinterpret_cast<float *>(smem_raw + kOffONorm); }
/* All consumer threads: start copying n floats (n a multiple of 4) into shared memory. */
__device__ __forceinline__ void prefetch_floats(float *dst, const float *src, int n) {
    for (int i = threadIdx.x; i < n / 4; i += kConsumerThreads) cp_async16(smem_u32(dst + 4 * i), src + 4 * i);
    cp_async_commit();
}
/* The same by the consumer warps from w0 on (the warps a GEMV leaves idle:
 * the copy then costs the working warps nothing); all of them when w0 is
 * past the last consumer warp. */
__device__ __forceinline__ void prefetch_floats_idle(float *dst, const float *src, int n, uint32_t w0) {
    if (w0 >= (uint32_t)kConsumerWarps) w0 = 0;
    const int i0 = (int)threadIdx.x - (int)(w0 * 32u), nthr = (kConsumerWarps - (int)w0) * 32;
    if (i0 < 0) return;
    for (int i = i0; i < n / 4; i += nthr) cp_async16(smem_u32(dst + 4 * i), src + 4 * i);
    cp_async_commit();
}

size_t decode_smem_bytes(int H, int I, bool tp) {
    const size_t xs = ((size_t)4 * (H > I ? H : I) + 15) & ~(size_t)15;
    return kOffXs + xs + (tp ? kSplitBytes : 0);
}

/* Phase input x in shared memory, element e: BF16 (2 bytes) in the
 * BF16-boundary contracts, FP32 in the FP32 control; per 64-column group g,
 * 16-byte piece p stored at position p ^ (g & 7) (conflict-free reads by the
 * GEMV lanes of both layouts). */
template <int MODE>
__device__ __forceinline__ uint32_t xs_off(int e) {
    const int g = e >> 6, c = e & 63;
    if (Mode<MODE>::kBf16) return (uint32_t)((g << 7) + ((((c >> 3) ^ (g & 7))) << 4) + ((c & 7) << 1));
    return (uint32_t)((g << 8) + ((((c >> 2) ^ (g & 7))) << 4) + ((c & 3) << 2));
}
template <int MODE>
__device__ __forceinline__ void xs_put(int e, float v) {
    if (Mode<MODE>::kBf16)
        *reinterpret_cast<uint16_t *>(sm_xs() + xs_off<MODE>(e)) = (uint16_t)(__float_as_uint(v) >> 16);
    else
        *reinterpret_cast<float *>(sm_xs() + xs_off<MODE>(e)) = v;
}
/* the fast BF16 product needs every nonzero input >= fast_x_min and finite */
__device__ __forceinline__ bool fast_ok(const DecodeParams &p, float v) {
    const float a = fabsf(v);
    return a == 0.0f || (a >= p.fast_x_min && a <= 3.4028234663852886e38f);
}

/* ----------------------------------------------------------- status */

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
 * at addr(i) and must carry tag tagof(i). Callers lay the words out so that a
 * warp's loads are coalesced (consecutive lanes at consecutive addresses).
 * Every load is issued at once, so data that is already there costs one
 * round trip; while words are missing, every lane re-reads its own missing
 * words, so the read completes one round trip after the last word lands.
 * All 32 lanes must call; lanes that use no word take part in the protocol
 * only. */
template <int N, bool SYS, class Addr, class TagOf, class Use, class W>
__device__ __forceinline__ uint32_t xissue(const Addr &addr, const TagOf &tagof, const Use &use, W (&w)[N]) {
#pragma unroll
    for (int i = 0; i < N; ++i)
        if (use(i)) w[i] = xget(addr(i), SYS);
    uint32_t missing = 0;
#pragma unroll
    for (int i = 0; i < N; ++i)
        if (use(i) && !xtag_is(w[i], tagof(i))) missing |= 1u << i;
    return missing;
}
template <int N, bool SYS, class Addr, class TagOf, class W>
__device__ __forceinline__ bool xfinish(const DecodeParams &p, const Addr &addr, const TagOf &tagof, W (&w)[N],
                                        uint32_t missing) {
    const int lane = threadIdx.x & 31;
    uint64_t t0 = 0;
    uint32_t rounds = 0;
    while (__any_sync(0xffffffffu, missing != 0)) {
        /* every lane re-reads its own missing words, so the read completes one
         * round trip after the last word lands */
#pragma unroll
        for (int i = 0; i < N; ++i)
            if ((missing >> i) & 1u) w[i] = xget(addr(i), SYS);
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
    return true;
}
/* Warp-wide read of exchange words: lane word i (i < N, where use(i)) lives
 * at addr(i) and must carry tag tagof(i). Callers lay the words out so that a
 * warp's loads are coalesced (consecutive lanes at consecutive addresses).
 * Every load is issued at once, so data that is already there costs one
 * round trip; while words are missing, every lane re-reads its own missing
 * words. All 32 lanes must call; lanes that use no word take part in the
 * protocol only. */
template <int N, bool SYS, class Addr, class TagOf, class Use>
__device__ __forceinline__ bool xread(const DecodeParams &p, const Addr &addr, const TagOf &tagof, const Use &use,
                                      float (&v)[N]) {
    typedef typename std::remove_const<typename std::remove_pointer<decltype(addr(0))>::type>::type W;
    W w[N];
    const uint32_t missing = xissue<N, SYS>(addr, tagof, use, w);
    const bool ok = xfinish<N, SYS>(p, addr, tagof, w, missing);
#pragma unroll
    for (int i = 0; i < N; ++i)
        if (use(i)) v[i] = xval(w[i]);
    return ok;
}

/* Element i of a whole-vector read by consumer thread t: t + 480 i
 * (coalesced across each warp); elements past the vector's end are unused. */
__device__ __forceinline__ int vec_elem(int t, int i) { return t + kConsumerThreads * i; }

/* Read n exchange words (at most 12 per thread) into the shared phase input,
 * recording whether they are in the fast path's range. All consumer threads
 * call. */
constexpr int kMaxWordsPerThread = 12;
template <int MODE>
__device__ __noinline__ bool xread_to_xs(const DecodeParams &p, const xword *src, int n, uint32_t tag, int xf) {
    const int t = threadIdx.x;
    float v[kMaxWordsPerThread];
    const bool ok = xread<kMaxWordsPerThread, Mode<MODE>::kTp>(
        p, [&](int i) { return xw<MODE>(src) + vec_elem(t, i); }, [&](int) { return tag; },
        [&](int i) { return vec_elem(t, i) < n; }, v);
    bool fast = true;
#pragma unroll
    for (int i = 0; i < kMaxWordsPerThread; ++i)
        if (vec_elem(t, i) < n) {
            xs_put<MODE>(vec_elem(t, i), v[i]);
            fast = fast && fast_ok(p, v[i]);
        }
    if (Mode<MODE>::kNative && !fast) sm_exact()[xf] = 1;
    return ok;
}

/* Wait until chunk q of the schedule sits in its ring slot; false on abort.
 * The slot's copy of q is issued only after every warp is done with the
 * slot's previous chunk (q - kSlots), but a warp that took no part in some
 * chunks may reach q earlier than that: it first sees the issue (in shared
 * memory), so that the mbarrier phase it then tests is never more than one
 * behind -- the parity test cannot tell phase k from phase k - 2. Every lane
 * waits itself (suspended in hardware; observing the completed phase makes
 * the copied bytes visible to it); a vote makes the result warp-uniform. */
__device__ __forceinline__ bool wait_full(const DecodeParams &p, uint32_t q) {
    const uint32_t slot = q % kSlots, k = q / kSlots;
    const uint32_t bar = smem_u32(&sm_full()[slot]);
    bool ok = sm_issued()[slot] > k && mbar_try(bar, k & 1u);
    if (!__all_sync(0xffffffffu, ok)) {
        const uint64_t t0 = gtimer();
        while (!ok) {
            ok = sm_issued()[slot] > k && mbar_wait(bar, k & 1u, 20000u);
            if (!ok && (*sm_abort_flag() || gtimer() - t0 > kWaitNs)) break;
        }
        if (!__all_sync(0xffffffffu, ok)) {
            if ((threadIdx.x & 31) == 0 && !*sm_abort_flag()) raise_error(p, kErrChunkTimeout, q);
            return false;
        }
    }
    return true;
}
/* A warp is done with chunk q's slot. */
__device__ __forceinline__ void release(uint32_t q) {
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(smem_u32(&sm_empty()[q % kSlots]));
}

/* ------------------------------------------------------------ schedule */

/* Units of a phase owned by CTA `cta` of `ncta`: [cta n / ncta, (cta+1) n / ncta). */
struct Span {
    uint32_t u0, u1;
};
/* a * b / c, in 32 bits when the product fits */
__device__ __forceinline__ uint32_t mul_div(uint32_t a, uint32_t b, uint32_t c) {
    const uint64_t m = (uint64_t)a * b;
    return (m >> 32) ? (uint32_t)(m / c) : (uint32_t)m / c;
}
__device__ __forceinline__ Span span_of(uint32_t total, uint32_t cta, uint32_t ncta) {
    return Span{mul_div(cta, total, ncta), mul_div(cta + 1, total, ncta)};
}

/* A tiled (wide) projection: T tiles of TR rows, G 64-column groups per
 * chunk, at most P tiles (one warp per 8 rows, at most kSlotBytes) per pass.
 * Stored column-chunk-major, so the chunk of tiles [a, b) is one copy. */
/* Parts a tiled GEMV pass of `units` 8-row units splits into: 1 (each
 * unit's warp works every group) unless splitting is on and the units leave
 * at least half of the consumer warps idle; then part k of a unit forms the
 * tree16 values of the unit's groups g with g % parts == k into shared
 * memory, and the unit's own warp adds them in group order. `items`: groups
 * per row; `bytes`: the values' size per unit. (The O / DOWN rows are not
 * split: a warp's share of a row is a few hundred cycles, less than the
 * split's two barriers and chain.) */
__device__ __forceinline__ uint32_t split_parts(uint32_t on, uint32_t units, uint32_t items, uint32_t bytes) {
    if (!on || units == 0 || 2u * units > (uint32_t)kConsumerWarps || units * bytes > kSplitBytes) return 1u;
    return min((uint32_t)kConsumerWarps / units, items);
}
struct Wide {
    const uint8_t *base;
    uint32_t TR, G, P, K, T, t0, t1;
    __device__ __forceinline__ uint32_t passes() const { return (t1 - t0 + P - 1) / P; }
    __device__ __forceinline__ uint32_t chunks_per_pass() const { return K / 64 / G; }
    __device__ __forceinline__ uint32_t piece() const { return G * TR * 128; }  /* one tile's share of a chunk */
    /* parts of a pass of n tiles (on: DecodeParams.split) */
    __device__ __forceinline__ uint32_t parts(uint32_t on, uint32_t n) const {
        return split_parts(on, n * (TR / 8), K / 64, K / 64 * 128);
    }
};
/* A narrow projection of R rows: rows [r0, r1), kNarrowGroups groups per
 * chunk (the last chunk may have fewer); stored column-chunk-major, so a
 * chunk of the rows is one copy. */
struct Narrow {
    const uint8_t *base;
    uint32_t K, R, r0, r1;
    __device__ __forceinline__ uint32_t chunks() const { return (K / 64 + kNarrowGroups - 1) / kNarrowGroups; }
    __device__ __forceinline__ uint32_t groups(uint32_t j) const { return min((uint32_t)kNarrowGroups, K / 64 - j * kNarrowGroups); }
    /* byte offset of chunk j's row r */
    __device__ __forceinline__ size_t off(uint32_t j, uint32_t r) const {
        return ((size_t)j * kNarrowGroups * R + (size_t)r * groups(j)) * 128u;
    }
    /* the same in a tensor-parallel image of NG groups per chunk (DecodeParams.ng_narrow) */
    __device__ __forceinline__ uint32_t chunks_ng(uint32_t NG) const { return (K / 64 + NG - 1) / NG; }
    __device__ __forceinline__ uint32_t groups_ng(uint32_t NG, uint32_t j) const { return min(NG, K / 64 - j * NG); }
    __device__ __forceinline__ size_t off_ng(uint32_t NG, uint32_t j, uint32_t r) const {
        return ((size_t)j * NG * R + (size_t)r * groups_ng(NG, j)) * 128u;
    }
};

__device__ __forceinline__ const uint8_t *layer_base(const DecodeParams &p, int l) {
    return p.wimg + (size_t)l * p.layer_stride;
}
/* TP: a tensor-parallel launch, whose image has the groups per chunk of
 * DecodeParams (g_qkvg, g_gu, g_lm, ng_narrow) */
template <bool TP>
__device__ __forceinline__ Wide wide_qkvg(const DecodeParams &p, int l, uint32_t cta, uint32_t ncta) {
    const uint32_t T = 4u * p.H / kTileRowsQKVG;
    const Span s = span_of(T, cta, ncta);
    return Wide{layer_base(p, l), kTileRowsQKVG, TP ? p.g_qkvg : kGroupsQKVG, kPassTiles, (uint32_t)p.H, T, s.u0, s.u1};
}
template <bool TP>
__device__ __forceinline__ Wide wide_gu(const DecodeParams &p, int l, uint32_t cta, uint32_t ncta) {
    const uint32_t T = 2u * p.I / kTileRowsGU;
    const Span s = span_of(T, cta, ncta);
    return Wide{layer_base(p, l) + p.off_gu, kTileRowsGU, TP ? p.g_gu : kGroupsGU, kPassTiles, (uint32_t)p.H, T, s.u0,
                s.u1};
}
template <bool TP>
__device__ __forceinline__ Wide wide_lm(const DecodeParams &p, uint32_t cta, uint32_t ncta) {
    const uint32_t T = (uint32_t)p.V / kTileRowsLM;
    const Span s = span_of(T, cta, ncta);
    return Wide{p.w_lm, kTileRowsLM, TP ? p.g_lm : kGroupsLM, kPassTiles, (uint32_t)p.H, T, s.u0, s.u1};
}
__device__ __forceinline__ Narrow narrow_o(const DecodeParams &p, int l, uint32_t cta, uint32_t ncta) {
    const Span s = span_of((uint32_t)p.H, cta, ncta);
    return Narrow{layer_base(p, l) + p.off_o, (uint32_t)p.H, (uint32_t)p.H, s.u0, s.u1};
}
__device__ __forceinline__ Narrow narrow_down(const DecodeParams &p, int l, uint32_t cta, uint32_t ncta) {
    const Span s = span_of((uint32_t)p.H, cta, ncta);
    return Narrow{layer_base(p, l) + p.off_down, (uint32_t)p.I, (uint32_t)p.H, s.u0, s.u1};
}
template <int MODE>
__device__ __forceinline__ uint32_t state_col_bytes() { return Mode<MODE>::kBf16State ? 512u : 1024u; }

/* Warps taking part in the a/b chunk and the state chunk of phase B. */
__device__ __forceinline__ uint32_t ab_warps(const DecodeParams &p, uint32_t rows) {
    const uint32_t w = (rows * ((uint32_t)p.H >> 4) + 31) / 32;
    return w < (uint32_t)kConsumerWarps ? w : (uint32_t)kConsumerWarps;
}
__device__ __forceinline__ uint32_t state_warps(uint32_t cols) { return cols > 2 ? cols : 2; }

/* ------------------------------------------------------------ producer */

/* Lane 0 claims the slot of chunk q (its previous chunk released by every
 * warp), marks the warps that sit the chunk out as done with it, and arms the
 * full barrier for `bytes`. Returns false (and stops the producer) on abort
 * or timeout. All lanes call. */
__device__ __forceinline__ bool claim_slot(const DecodeParams &p, uint32_t q, uint32_t active, uint32_t bytes) {
    int ok = 1;
    if ((threadIdx.x & 31) == 0) {
        const uint32_t slot = q % kSlots, k = q / kSlots;
        if (k > 0) {
            const uint32_t bar = smem_u32(&sm_empty()[slot]);
            const uint64_t t0 = gtimer();
            while (!mbar_wait(bar, (k - 1) & 1u, 20000u)) {
                if (*sm_abort_flag()) { ok = 0; break; }
                if (gtimer() - t0 > kSlotWaitNs) {
                    raise_error(p, kErrSlotTimeout, q);
                    ok = 0;
                    break;
                }
            }
        }
        if (ok && *sm_abort_flag()) ok = 0;
        if (ok) {
            if (active < (uint32_t)kConsumerWarps) mbar_arrive_n(smem_u32(&sm_empty()[slot]), kConsumerWarps - active);
            mbar_expect_tx(smem_u32(&sm_full()[slot]), bytes);
            sm_issued()[slot] = k + 1;
        }
    }
    return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

/* The CTA's chunk schedule, in the order the consumers take the chunks: per
 * layer the QKVG chunks, the a/b rows of its heads, its state columns, the
 * O chunks, the gate/up chunks, the DOWN chunks; then the LM head's. Built
 * once per launch (the partitions do not depend on the layer: chunk
 * addresses of layer l are layer 0's plus l * layer_stride), so the producer
 * walks it with a few multiplies per chunk. */
struct Chunk {
    const uint8_t *src;
    uint32_t bytes, active;  /* copy size; consumer warps that take part */
    bool state;              /* a state chunk (kept in L2 across tokens) */
};
struct Sched {
    Wide qkvg, gu, lm;
    Narrow o, down;
    uint32_t h0, ab_rows, c0, ncols, cb;
};
struct Cursor {
    int l;
    uint32_t seg, k;
};
constexpr uint32_t kSegsPerLayer = 6;

static_assert(sizeof(Sched) <= 256, "the schedule's shared-memory region holds 256 bytes");
/* The CTA's schedule, built once per launch (gdn_decode_kernel's start) */
__device__ __forceinline__ Sched *sm_sched() { return reinterpret_cast<Sched *>(smem_raw + kOffSched); }
/* Lane 0 of consumer warps 0..5 each fill one part (the partitions' divisions
 * run in parallel and once per launch, not in every phase's setup). */
template <int MODE>
__device__ __forceinline__ void build_sched(const DecodeParams &p, uint32_t cta, uint32_t ncta) {
    const int warp = threadIdx.x >> 5;
    if ((threadIdx.x & 31) != 0 || warp > 5) return;
    Sched *s = sm_sched();
    switch (warp) {
    case 0: s->qkvg = wide_qkvg<Mode<MODE>::kTp>(p, 0, cta, ncta); break;
    case 1: s->gu = wide_gu<Mode<MODE>::kTp>(p, 0, cta, ncta); break;
    case 2: s->lm = wide_lm<Mode<MODE>::kTp>(p, cta, ncta); break;
    case 3: s->o = narrow_o(p, 0, cta, ncta); break;
    case 4: s->down = narrow_down(p, 0, cta, ncta); break;
    default: {
        const Span sc = span_of((uint32_t)p.nh * kHeadDim, cta, ncta);
        s->h0 = sc.u0 >> 8;
        s->ab_rows = 2u * (((sc.u1 - 1) >> 8) - s->h0 + 1);
        s->c0 = sc.u0;
        s->ncols = sc.u1 - sc.u0;
        s->cb = state_col_bytes<MODE>();
    }
    }
}
__device__ __forceinline__ uint32_t wide_count(const Wide &w) { return w.passes() * w.chunks_per_pass(); }
template <bool TP>
__device__ __forceinline__ Chunk wide_chunk(const DecodeParams &p, const Wide &w, size_t shift, uint32_t k) {
    const uint32_t cpp = w.chunks_per_pass(), pass = k / cpp, j = k - pass * cpp;
    const uint32_t pt0 = w.t0 + pass * w.P, n = min(w.P, w.t1 - pt0);
    if (TP) {
        const uint32_t sf = w.parts(p.split, n);
        /* the chunk's G consecutive groups fall to min(G, sf) parts */
        return Chunk{w.base + shift + ((size_t)j * w.T + pt0) * w.piece(), n * w.piece(),
                     n * (w.TR / 8) * (sf > 1 ? min(w.G, sf) : 1u), false};
    }
    return Chunk{w.base + shift + ((size_t)j * w.T + pt0) * w.piece(), n * w.piece(), n * (w.TR / 8), false};
}
template <bool TP>
__device__ __forceinline__ Chunk narrow_chunk(const DecodeParams &p, const Narrow &w, size_t shift, uint32_t j) {
    const uint32_t n = w.r1 - w.r0;
    if (TP) {
        const uint32_t NG = p.ng_narrow;
        return Chunk{w.base + shift + w.off_ng(NG, j, w.r0), n * w.groups_ng(NG, j) * 128u, n, false};
    }
    return Chunk{w.base + shift + w.off(j, w.r0), n * w.groups(j) * 128u, n, false};
}
/* Chunk c of the schedule, advancing c; false past the end. */
template <bool TP>
__device__ __forceinline__ bool sched_next(const DecodeParams &p, const Sched &s, Cursor &c, Chunk &out) {
    while (c.l <= p.L) {
        const size_t shift = (size_t)c.l * p.layer_stride;
        uint32_t count;
        if (c.l == p.L) {
            count = wide_count(s.lm);
            if (c.k < count) { out = wide_chunk<TP>(p, s.lm, 0, c.k++); return true; }
        } else {
            switch (c.seg) {
            case 0: count = wide_count(s.qkvg); if (c.k < count) { out = wide_chunk<TP>(p, s.qkvg, shift, c.k++); return true; } break;
            case 1:
                if (c.k == 0) {
                    ++c.k;
                    out = Chunk{layer_base(p, c.l) + p.off_ab + (size_t)2 * s.h0 * p.H * 2, s.ab_rows * p.H * 2,
                                ab_warps(p, s.ab_rows), false};
                    return true;
                }
                break;
            case 2:
                if (c.k == 0) {
                    ++c.k;
                    out = Chunk{reinterpret_cast<const uint8_t *>(p.S) + ((size_t)c.l * p.nh * kHeadDim + s.c0) * s.cb,
                                s.ncols * s.cb, state_warps(s.ncols), true};
                    return true;
                }
                break;
            case 3: count = TP ? s.o.chunks_ng(p.ng_narrow) : s.o.chunks(); if (c.k < count) { out = narrow_chunk<TP>(p, s.o, shift, c.k++); return true; } break;
            case 4: count = wide_count(s.gu); if (c.k < count) { out = wide_chunk<TP>(p, s.gu, shift, c.k++); return true; } break;
            default: count = TP ? s.down.chunks_ng(p.ng_narrow) : s.down.chunks(); if (c.k < count) { out = narrow_chunk<TP>(p, s.down, shift, c.k++); return true; } break;
            }
        }
        c.k = 0;
        if (c.l == p.L || ++c.seg == kSegsPerLayer) { c.seg = 0; ++c.l; }
    }
    return false;
}

/* The producer warp: walks the CTA's schedule, one chunk per ring slot
 * (lane 0 issues the copy). (Measured slower: prefetching the chunks past
 * the ring into L2 with cp.async.bulk.prefetch.L2, continuously 128-512 KB
 * ahead or only while the consumers wait for inputs.) */
template <int MODE>
__device__ void producer(const DecodeParams &p, uint32_t cta, uint32_t ncta) {
    const int lane = threadIdx.x & 31;
    const uint64_t pol_w = policy_evict_first(), pol_s = policy_evict_last();
    (void)cta;
    (void)ncta;
    const Sched s = *sm_sched();
    Cursor d{0, 0, 0};
    Chunk ch;
    for (uint32_t q = 0; sched_next<Mode<MODE>::kTp>(p, s, d, ch); ++q) {
        if (!claim_slot(p, q, ch.active, ch.bytes)) return;
        if (lane == 0)
            bulk_g2s(smem_u32(sm_slot(q % kSlots)), ch.src, ch.bytes, smem_u32(&sm_full()[q % kSlots]),
                     ch.state ? pol_s : pol_w);
    }
}

/* ---------------------------------------------------- consumer GEMVs */

/* tree16 of the 16 columns [64 g + 16 b, 64 g + 16 b + 16) of a weight row
 * whose 64-column group sits at `wrow` with piece swizzle `wsw`, against the
 * shared phase input. KIND: 0 exact products, 1 BF16-rounded (fast), 2 the
 * exact emulation of the BF16-rounded product, 3 the FP32 control. */
template <int KIND>
__device__ __forceinline__ float tree16_at(const uint8_t *wrow, uint32_t wsw, uint32_t g, uint32_t b) {
    const uint4 w0 = lds128(wrow + (((2u * b) ^ wsw) << 4));
    const uint4 w1 = lds128(wrow + (((2u * b + 1u) ^ wsw) << 4));
    if (KIND == 3) {
        const uint8_t *xp = sm_xs() + (g << 8);
        const uint4 a0 = lds128(xp + (((4u * b) ^ (g & 7u)) << 4));
        const uint4 a1 = lds128(xp + (((4u * b + 1u) ^ (g & 7u)) << 4));
        const uint4 a2 = lds128(xp + (((4u * b + 2u) ^ (g & 7u)) << 4));
        const uint4 a3 = lds128(xp + (((4u * b + 3u) ^ (g & 7u)) << 4));
        return tree16_f32(w0, w1, *reinterpret_cast<const float4 *>(&a0), *reinterpret_cast<const float4 *>(&a1),
                          *reinterpret_cast<const float4 *>(&a2), *reinterpret_cast<const float4 *>(&a3));
    }
    const uint8_t *xp = sm_xs() + (g << 7);
    const uint4 x0 = lds128(xp + (((2u * b) ^ (g & 7u)) << 4));
    const uint4 x1 = lds128(xp + (((2u * b + 1u) ^ (g & 7u)) << 4));
    return tree16_bf<KIND < 3 ? KIND : 0>(w0, w1, x0, x1);
}

/* One pass of a tiled projection: tiles [pt0, pt0 + n), chunks q .. q +
 * chunks_per_pass - 1 of the schedule (the counter is passed by value: a
 * counter in local memory costs an L2 round trip per chunk). Warp w works on rows 8 (w % (TR/8))
 * .. + 7 of tile w / (TR/8); lane (r = lane / 4, b = lane % 4) keeps the
 * sequential chain of bank b of its row over the K / 64 groups (the
 * reference's bank accumulation, c_impl/gdn_model.cpp:4444-4586). Returns
 * the row's (b0 + b1) + (b2 + b3) in lanes with b == 0 of active warps. */
constexpr uint32_t kPair = 1;  /* chunks taken together by a warp (2 measured slower: fewer slots in flight) */
constexpr uint32_t kMaxG = 4;   /* groups per chunk of a tiled projection, at most */

/* A pass of a tiled projection split into sf parts (every consumer warp
 * calls it): warp (unit u = warp % units, part k = warp / units) forms the
 * tree16 values of the groups g % sf == k of unit u's rows into shared
 * memory, then unit u's own warp (k == 0, the warp that owns the rows
 * unsplit) adds them in group order -- the same chain as wide_chunks. */
template <int KIND>
__device__ __forceinline__ float wide_split(const DecodeParams &p, const Wide &w, uint32_t n, uint32_t q, uint32_t sf) {
    const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t wpt = w.TR / 8, units = n * wpt, unit = warp % units, part = warp / units;
    const uint32_t tw = unit / wpt, rr = (unit % wpt) * 8u + (lane >> 2), b = lane & 3u;
    const uint32_t ng = w.K / 64;
    float *vals = sm_split(p) + unit * ng * 32u + lane;
    named_sync(1, kConsumerThreads); /* the previous split's chain reads are done */
    if (part < sf) {
        const uint32_t cpp = w.chunks_per_pass();
        for (uint32_t j = 0; j < cpp; ++j) {
            const uint32_t ga = j * w.G, g1 = ga + w.G;
            const uint32_t gf = ga + (part + sf - ga % sf) % sf; /* the part's first group of the chunk */
            if (gf >= g1) continue;
            if (!wait_full(p, q + j)) continue;
            const uint8_t *tile = sm_slot((q + j) % kSlots) + tw * w.piece() + rr * 128u;
            for (uint32_t g = gf; g < g1; g += sf) vals[g * 32u] = tree16_at<KIND>(tile + (g - ga) * w.TR * 128u, rr & 7u, g, b);
            release(q + j);
        }
    }
    named_sync(1, kConsumerThreads);
    float acc = 0.0f;
    if (warp < units) {
#pragma unroll 8
        for (uint32_t g = 0; g < ng; ++g) acc = __fadd_rn(acc, vals[g * 32u]);
    }
    const float t = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 1));
    return __fadd_rn(t, __shfl_down_sync(0xffffffffu, t, 2));
}

/* The same for the tensor-parallel images: any G, in blocks of kMaxG groups
 * (the chain in group order). */
template <int KIND>
__device__ __forceinline__ float wide_chunks_any(const DecodeParams &p, const Wide &w, uint32_t n, uint32_t q) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t wpt = w.TR / 8;
    const uint32_t tw = (uint32_t)warp / wpt;
    const uint32_t rr = ((uint32_t)warp % wpt) * 8u + ((uint32_t)lane >> 2), b = (uint32_t)lane & 3u;
    float acc = 0.0f;
    if (tw < n) {
        const uint32_t cpp = w.chunks_per_pass();
        for (uint32_t j = 0; j < cpp; ++j, ++q) {
            if (!wait_full(p, q)) continue;
            const uint8_t *tile = sm_slot(q % kSlots) + tw * w.piece() + rr * 128u;
            for (uint32_t gb = 0; gb < w.G; gb += kMaxG) {
                float t[kMaxG];
#pragma unroll
                for (uint32_t gi = 0; gi < kMaxG; ++gi)
                    t[gi] = gb + gi < w.G ? tree16_at<KIND>(tile + (gb + gi) * w.TR * 128u, rr & 7u, j * w.G + gb + gi, b)
                                          : 0.0f;
#pragma unroll
                for (uint32_t gi = 0; gi < kMaxG; ++gi)
                    if (gb + gi < w.G) acc = __fadd_rn(acc, t[gi]);
            }
            release(q);
        }
    }
    const float t = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 1));
    return __fadd_rn(t, __shfl_down_sync(0xffffffffu, t, 2));
}

/* TP: a tensor-parallel launch (the image's geometry; split when the pass
 * leaves warps idle). */
template <int KIND, bool TP>
__device__ __forceinline__ float wide_chunks(const DecodeParams &p, const Wide &w, uint32_t n, uint32_t q) {
    if (TP) {
        const uint32_t sf = w.parts(p.split, n);
        return sf > 1 ? wide_split<KIND>(p, w, n, q, sf) : wide_chunks_any<KIND>(p, w, n, q);
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t wpt = w.TR / 8;
    const uint32_t tw = (uint32_t)warp / wpt;
    const uint32_t rr = ((uint32_t)warp % wpt) * 8u + ((uint32_t)lane >> 2), b = (uint32_t)lane & 3u;
    float acc = 0.0f;
    if (tw < n) {
        const uint32_t cpp = w.chunks_per_pass();
        for (uint32_t j = 0; j < cpp; j += kPair, q += kPair) {
            const uint32_t u = min(kPair, cpp - j);
            bool ok = true;
            for (uint32_t i = 0; i < u; ++i) ok = wait_full(p, q + i) && ok;
            if (!ok) continue;
            float t[kPair][kMaxG];
#pragma unroll
            for (uint32_t i = 0; i < kPair; ++i) {
                const uint8_t *tile = sm_slot((q + i) % kSlots) + tw * w.piece() + rr * 128u;
#pragma unroll
                for (uint32_t gi = 0; gi < kMaxG; ++gi)
                    t[i][gi] = (i < u && gi < w.G)
                                   ? tree16_at<KIND>(tile + gi * w.TR * 128u, rr & 7u, (j + i) * w.G + gi, b)
                                   : 0.0f;
            }
#pragma unroll
            for (uint32_t i = 0; i < kPair; ++i)
#pragma unroll
                for (uint32_t gi = 0; gi < kMaxG; ++gi)
                    if (i < u && gi < w.G) acc = __fadd_rn(acc, t[i][gi]);
            for (uint32_t i = 0; i < u; ++i) release(q + i);
        }
    }
    const float t = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 1));
    return __fadd_rn(t, __shfl_down_sync(0xffffffffu, t, 2));
}

/* The same for the tensor-parallel images: chunks of any multiple of 8
 * groups, in blocks of 8 (lane (b, s): group 8 m + s). */
template <int KIND>
__device__ __forceinline__ float narrow_chunks_any(const DecodeParams &p, const Narrow &w, uint32_t q) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t b = (uint32_t)lane >> 3, s = (uint32_t)lane & 7u;
    float acc = 0.0f;
    if ((uint32_t)warp < w.r1 - w.r0) {
        const uint32_t NG = p.ng_narrow, nc = w.chunks_ng(NG);
        for (uint32_t j = 0; j < nc; ++j, ++q) {
            const uint32_t ng = w.groups_ng(NG, j);
            if (!wait_full(p, q)) continue;
            const uint8_t *row = sm_slot(q % kSlots) + warp * ng * 128u;
            const uint32_t g0 = j * NG;
            for (uint32_t gb = 0; gb < ng; gb += 8) {
                const uint32_t g = g0 + gb + s;
                const float t0 = tree16_at<KIND>(row + (gb + s) * 128u, g & 7u, g, b);
                acc = __fadd_rn(acc, t0);
#pragma unroll
                for (int k = 1; k < 8; ++k) acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, t0, k));
            }
            release(q);
        }
    }
    const float t = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 8));
    return __fadd_rn(t, __shfl_down_sync(0xffffffffu, t, 16));
}

/* A narrow projection: warp w owns row r0 + w; lane (b = lane / 8, s = lane
 * % 8) computes the tree16 of bank b of groups s and s + 8 of a chunk, and
 * lane (b, 0) adds a chunk's values in group order to the bank's chain
 * (gathered by warp shuffles). Returns (b0 + b1) + (b2 + b3) in lane 0 of
 * active warps. */
template <int KIND, bool TP>
__device__ __forceinline__ float narrow_chunks(const DecodeParams &p, const Narrow &w, uint32_t q) {
    if (TP) return narrow_chunks_any<KIND>(p, w, q);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t b = (uint32_t)lane >> 3, s = (uint32_t)lane & 7u;
    float acc = 0.0f;
    if ((uint32_t)warp < w.r1 - w.r0) {
        const uint32_t nc = w.chunks();
        for (uint32_t j = 0; j < nc; ++j, ++q) {
            const uint32_t ng = w.groups(j);
            if (!wait_full(p, q)) continue;
            const uint8_t *row = sm_slot(q % kSlots) + warp * ng * 128u;
            const uint32_t g0 = j * kNarrowGroups;
            const float t0 = tree16_at<KIND>(row + s * 128u, s, g0 + s, b);
            const float t1 = ng > 8 ? tree16_at<KIND>(row + (8 + s) * 128u, s, g0 + 8 + s, b) : 0.0f;
            release(q);
            acc = __fadd_rn(acc, t0);
#pragma unroll
            for (int k = 1; k < 8; ++k) acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, t0, k));
            if (ng > 8) {
                acc = __fadd_rn(acc, t1);
#pragma unroll
                for (int k = 1; k < 8; ++k) acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, t1, k));
            }
        }
    }
    const float t = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 8));
    return __fadd_rn(t, __shfl_down_sync(0xffffffffu, t, 16));
}

/* The GEMV kind of the contract and phase (exact: the input failed the fast
 * path's range test, or the test hook). */
template <int MODE, class F>
__device__ __forceinline__ float gemv_dispatch(bool exact, const F &f) {
    if (!Mode<MODE>::kBf16) return f(std::integral_constant<int, 3>());
    if (!Mode<MODE>::kNative) return f(std::integral_constant<int, 0>());
    if (exact) return f(std::integral_constant<int, 2>());
    return f(std::integral_constant<int, 1>());
}

/* ---------------------------------------------------------- prologues */

constexpr int kMaxPer = ((int)kMaxHidden + kConsumerThreads - 1) / kConsumerThreads;  /* hidden elements per consumer thread */

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
/* Sequential sum, in index order from 0.0f, of the n floats at a (shared
 * memory, 16-byte aligned). Every lane of the calling warp forms it and
 * returns it. */
__device__ __forceinline__ float seq_sum_bcast(const float *a, int n) {
    /* every lane reads the same 16 bytes (one shared-memory wavefront): the
     * shuffle unit, which all warps of the SM share, stays out of the chain */
    const float4 *a4 = reinterpret_cast<const float4 *>(a);
    float sum = 0.0f;
    int k = 0;
    for (; k + 8 <= (n >> 2); k += 8) {
        float4 v[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = a4[k + i];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            sum = __fadd_rn(sum, v[i].x);
            sum = __fadd_rn(sum, v[i].y);
            sum = __fadd_rn(sum, v[i].z);
            sum = __fadd_rn(sum, v[i].w);
        }
    }
    for (int i = 4 * k; i < n; ++i) sum = __fadd_rn(sum, a[i]);
    return sum;
}

/* Sum of squares of 16 consecutive floats, sequential from 0.0f. */
__device__ __forceinline__ float sq16(const float *a) {
    float hs = 0.0f;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const float4 v = reinterpret_cast<const float4 *>(a)[q];
        hs = __fadd_rn(hs, __fmul_rn(v.x, v.x));
        hs = __fadd_rn(hs, __fmul_rn(v.y, v.y));
        hs = __fadd_rn(hs, __fmul_rn(v.z, v.z));
        hs = __fadd_rn(hs, __fmul_rn(v.w, v.w));
    }
    return hs;
}

/* Residual add + RMSNorm into the shared phase input, in the reference's
 * order (c_impl/gdn_model.cpp:1394-1476, 3351-3452): x = round(xres + y) (or
 * the embedding row for layer 0); thread t < H/16 sums the squares of the
 * 16-column half t (beat t/2, half t%2) sequentially; lane 0 of every warp
 * sums the H/16 half sums sequentially (redundantly, so no third barrier);
 * scale = 1/sqrtf(sum/H + eps); out = round((x*scale)*w). */
template <int MODE>
__device__ __noinline__ bool prologue_norm(const DecodeParams &p, const xword *y, uint32_t tag,
                                              const float *w, bool embed, float *hidden, int pidx, int xf) {
    const int t = threadIdx.x;
    const int halves = p.H >> 4;
    bool ok = true;
    float x[kMaxPer];
    (void)w;
    cp_async_wait_all();  /* this thread's share of the weights; the barrier below publishes all shares */
    if (embed) {
        if (p.token_src != nullptr || p.token_imm >= 0) {
            const int32_t tok = p.token_src != nullptr ? *p.token_src : p.token_imm;
            const uint16_t *e = p.emb + (size_t)tok * p.H;
#pragma unroll
            for (int i = 0; i < kMaxPer; ++i)
                if (vec_elem(t, i) < p.H) x[i] = bnd<MODE>(__uint_as_float((uint32_t)__ldg(e + vec_elem(t, i)) << 16));
        } else {
#pragma unroll
            for (int i = 0; i < kMaxPer; ++i)
                if (vec_elem(t, i) < p.H) x[i] = bnd<MODE>(p.x_embed[vec_elem(t, i)]);
        }
    } else {
        float yv[kMaxPer];
        ok = xread<kMaxPer, Mode<MODE>::kTp>(p, [&](int i) { return xw<MODE>(y) + vec_elem(t, i); },
                                             [&](int) { return tag; }, [&](int i) { return vec_elem(t, i) < p.H; }, yv);
#pragma unroll
        for (int i = 0; i < kMaxPer; ++i)
            if (vec_elem(t, i) < p.H) x[i] = bnd<MODE>(__fadd_rn(sm_xres()[vec_elem(t, i)], yv[i]));
    }
    if (t == 0) trace_put(p, pidx, 1);
#pragma unroll
    for (int i = 0; i < kMaxPer; ++i)
        if (vec_elem(t, i) < p.H) sm_xres()[vec_elem(t, i)] = x[i];
    named_sync(1, kConsumerThreads);
    if (t < halves) sm_red()[t] = sq16(sm_xres() + 16 * t);
    named_sync(1, kConsumerThreads);
    if (t == 0) trace_put(p, pidx, 4);
    /* every warp forms the sum itself: no third barrier (and a single warp
     * doing it while the others wait at a barrier measured far slower) */
    const float sum = seq_sum_bcast(sm_red(), halves);
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, (float)p.H), p.eps)));
    if (t == 0) trace_put(p, pidx, 6);
    bool fast = true;
#pragma unroll
    for (int i = 0; i < kMaxPer; ++i) {
        if (vec_elem(t, i) < p.H) {
            const float o = bnd<MODE>(__fmul_rn(__fmul_rn(x[i], scale), sm_normw()[vec_elem(t, i)]));
            if (hidden != nullptr) hidden[vec_elem(t, i)] = o;
            xs_put<MODE>(vec_elem(t, i), o);
            fast = fast && fast_ok(p, o);
        }
    }
    if (Mode<MODE>::kNative && !fast) sm_exact()[xf] = 1;
    return ok;
}

/* Per-head RMSNorm of the attention output times swish(gate) in the
 * reference's order (c_impl/gdn_model.cpp:3226-3349, production form
 * :5720-5835): per head, 16 half sums of 16 sequential squares, summed
 * sequentially; scale = 1/sqrtf(sum/256 + eps); out = round(((a*scale)*w) *
 * g * sigmoid(g)). Gate and attention words are read together. */
template <int MODE>
__device__ __noinline__ bool prologue_norm_gate(const DecodeParams &p, const float *o_norm, uint32_t tag_g,
                                                   uint32_t tag_a, int pidx, int xf) {
    const int t = threadIdx.x, lane = t & 31;
    const int halves = p.H >> 4;
    float *a_sh = sm_scratch();
    (void)o_norm;
    cp_async_wait_all();
    /* v[i]: gate g; v[kMaxPer + i]: attention output; sg[i]: sigmoid(g) */
    float v[2 * kMaxPer], sg[kMaxPer];
    bool ok;
    if (Mode<MODE>::kBf16) {
        /* both reads issued before either is polled */
        const gword *gw = reinterpret_cast<const gword *>(p.gate);
        const auto *aw = xw<MODE>(p.attn);
        auto use = [&](int i) { return vec_elem(t, i) < p.H; };
        auto ga = [&](int i) { return gw + vec_elem(t, i); };
        auto aa = [&](int i) { return aw + vec_elem(t, i); };
        gword g[kMaxPer];
        typename XW<MODE>::T a[kMaxPer];
        const uint32_t mg = xissue<kMaxPer, Mode<MODE>::kTp>(ga, [&](int) { return tag_g; }, use, g);
        const uint32_t ma = xissue<kMaxPer, Mode<MODE>::kTp>(aa, [&](int) { return tag_a; }, use, a);
        ok = xfinish<kMaxPer, Mode<MODE>::kTp>(p, ga, [&](int) { return tag_g; }, g, mg);
        ok = xfinish<kMaxPer, Mode<MODE>::kTp>(p, aa, [&](int) { return tag_a; }, a, ma) && ok;
#pragma unroll
        for (int i = 0; i < kMaxPer; ++i) {
            v[i] = gword_g(g[i]);
            sg[i] = gword_sig(g[i]);
            v[kMaxPer + i] = xval(a[i]);
        }
    } else {
        ok = xread<2 * kMaxPer, Mode<MODE>::kTp>(
            p,
            [&](int i) {
                return i < kMaxPer ? xw<MODE>(p.gate) + vec_elem(t, i) : xw<MODE>(p.attn) + vec_elem(t, i - kMaxPer);
            },
            [&](int i) { return i < kMaxPer ? tag_g : tag_a; }, [&](int i) { return vec_elem(t, i % kMaxPer) < p.H; }, v);
    }
    if (t == 0) trace_put(p, pidx, 1);
#pragma unroll
    for (int i = 0; i < kMaxPer; ++i)
        if (vec_elem(t, i) < p.H) a_sh[vec_elem(t, i)] = v[kMaxPer + i];
    named_sync(1, kConsumerThreads);
    if (t < halves) sm_red()[t] = sq16(a_sh + 16 * t);
    named_sync(1, kConsumerThreads);
    if (t == 0) trace_put(p, pidx, 4);
    float hscale = 0.0f;
    if (lane < p.nh) {
        float sum = 0.0f;
#pragma unroll
        for (int j = 0; j < 16; ++j) sum = __fadd_rn(sum, sm_red()[16 * lane + j]);
        hscale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum, 256.0f), p.eps)));
    }
    if (t == 0) trace_put(p, pidx, 6);
    bool fast = true;
#pragma unroll
    for (int i = 0; i < kMaxPer; ++i) {
        const float scale = __shfl_sync(0xffffffffu, hscale, (vec_elem(t, i) >> 8) & 31);
        if (vec_elem(t, i) < p.H) {
            const float gv = v[i];
            const float normalized = __fmul_rn(__fmul_rn(v[kMaxPer + i], scale), sm_onorm()[vec_elem(t, i) & (kHeadDim - 1)]);
            const float sig = Mode<MODE>::kBf16 ? sg[i] : sigmoid_ref(gv);
            const float o = bnd<MODE>(__fmul_rn(__fmul_rn(normalized, gv), sig));
            xs_put<MODE>(vec_elem(t, i), o);
            fast = fast && fast_ok(p, o);
        }
    }
    if (Mode<MODE>::kNative && !fast) sm_exact()[xf] = 1;
    return ok;
}

/* ---------------------------------------------------------- phase B */

/* Butterfly sum: lane offsets 1, 2, 4, 8, 16 give the balanced pairwise tree
 * over each aligned block, so every lane ends with the same bits. */
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
/* Deterministic sums over warps 0..7 (256 threads, one value each per sum)
 * of N values: warp butterfly, then a fixed pairwise tree over the 8 warps.
 * Over 256 inputs held one per thread this is exactly the balanced tree of
 * gdn_tree_reduce_256 (c_impl/gdn_model.cpp:1336-1375). All consumer threads
 * call (warps 8.. contribute nothing) and receive the sums. */
template <int N>
__device__ __forceinline__ void block_sum8(float (&v)[N], float *red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (warp < 8) {  /* the other warps' values are not part of the sums */
#pragma unroll
        for (int i = 0; i < N; ++i) v[i] = warp_sum(v[i]);
    }
    if (lane == 0 && warp < 8) {
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

/* Phase B of layer l for state columns [c0, c1) (heads h0..h1):
 *   1. the a/b projection rows of the CTA's heads from the a/b chunk and the
 *      phase-A input still in shared memory: exact products, one sequential
 *      chain of tree16 values per row (gdn_gemv_tiny_ab, c_impl/
 *      gdn_model.cpp:1501-1535); beta = sigmoid(b), decay (2101-2105);
 *   2. q, k of the heads and v of the columns from phase A's outputs; q/k L2
 *      norms and alpha = <q_n, k_n> (2059-2124);
 *   3. the gated delta rule on the state chunk: read pass r = S k_n, p = S
 *      q_n sequential over k (2184-2210), delta and the output (2214-2243),
 *      update S' = decay S + k_n delta (2268-2300), written back. */
template <int MODE>
__device__ __noinline__ bool phase_state(const DecodeParams &p, int l, uint32_t q, uint32_t c0, uint32_t c1,
                                         uint32_t tag_in, uint32_t tag_out, int pidx) {
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const uint32_t h0 = c0 >> 8, h1 = (c1 - 1) >> 8, nhl = h1 - h0 + 1, n = c1 - c0;
    const uint32_t halves = (uint32_t)p.H >> 4, rows = 2 * nhl;
    bool ok = true;
    /* q, k of both heads (element t of each, threads 0..255), v of column
     * c0 + t: the loads go out now and are polled after the a/b rows, so
     * their round trip overlaps that work */
    const bool qk = t < kHeadDim;
    const auto *qb = xw<MODE>(p.qkv);
    auto qaddr = [&](int k) {
        return k == 4 ? qb + 2 * p.H + c0 + t : qb + (k & 1) * p.H + (h0 + (uint32_t)(k >> 1)) * kHeadDim + t;
    };
    auto qtag = [&](int) { return tag_in; };
    auto quse = [&](int k) { return k == 4 ? (uint32_t)t < n : qk && (uint32_t)(k >> 1) < nhl; };
    typename XW<MODE>::T qw[5];
    const uint32_t qmiss = xissue<5, Mode<MODE>::kTp>(qaddr, qtag, quse, qw);
    /* 1. a/b rows: thread (row, half) forms one tree16, warp row chains them */
    if ((uint32_t)warp < ab_warps(p, rows)) {
        if (wait_full(p, q)) {
            for (uint32_t idx = (uint32_t)t; idx < rows * halves; idx += kConsumerThreads) {
                const uint32_t row = idx / halves, hf = idx % halves;
                const uint8_t *wr = sm_slot(q % kSlots) + ((size_t)row * p.H + hf * 16) * 2;
                const uint4 w0 = lds128(wr), w1 = lds128(wr + 16);
                const uint32_t g = hf >> 2, b = hf & 3u;
                float x[16];
                if (Mode<MODE>::kBf16) {
                    const uint8_t *xp = sm_xs() + (g << 7);
                    const uint4 x0 = lds128(xp + (((2u * b) ^ (g & 7u)) << 4));
                    const uint4 x1 = lds128(xp + (((2u * b + 1u) ^ (g & 7u)) << 4));
                    const uint32_t xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        x[2 * i] = bf_lo(xv[i]);
                        x[2 * i + 1] = bf_hi(xv[i]);
                    }
                } else {
                    const uint8_t *xp = sm_xs() + (g << 8);
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const float4 v4 = *reinterpret_cast<const float4 *>(xp + (((4u * b + i) ^ (g & 7u)) << 4));
                        x[4 * i] = v4.x;
                        x[4 * i + 1] = v4.y;
                        x[4 * i + 2] = v4.z;
                        x[4 * i + 3] = v4.w;
                    }
                }
                const uint32_t wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
                float s[8];
#pragma unroll
                for (int i = 0; i < 8; ++i)
                    s[i] = __fadd_rn(__fmul_rn(bf_lo(wv[i]), x[2 * i]), __fmul_rn(bf_hi(wv[i]), x[2 * i + 1]));
                const float a0 = __fadd_rn(s[0], s[1]), a1 = __fadd_rn(s[2], s[3]);
                const float a2 = __fadd_rn(s[4], s[5]), a3 = __fadd_rn(s[6], s[7]);
                sm_park()[row * 128 + hf] = __fadd_rn(__fadd_rn(a0, a1), __fadd_rn(a2, a3));
            }
            release(q);
        }
    }
    ++q;
    named_sync(1, kConsumerThreads);
    if ((uint32_t)warp < rows) {
        /* one sequential chain over the row's halves in column order */
        const float acc = seq_sum_bcast(sm_park() + warp * 128, (int)halves);
        /* row 2 hs: a of head h0 + hs, row 2 hs + 1: b */
        if (lane == 0) sm_hscal()[(warp >> 1) * 8 + 3 + (warp & 1)] = bnd<MODE>(acc);
    }
    named_sync(1, kConsumerThreads);
    if (t == 0) trace_put(p, pidx, 4);
    /* beta and decay per head (lane 0 of warps 0, 1); the decay table load
     * overlaps the wait for q and k */
    if (lane == 0 && (uint32_t)warp < nhl) {
        const uint32_t hs = (uint32_t)warp, h = h0 + hs;
        const float a = sm_hscal()[hs * 8 + 3], bb = sm_hscal()[hs * 8 + 4];
        float decay;
        if (Mode<MODE>::kBf16) {
            decay = __ldg(p.decay_tab + ((size_t)l * p.nh + h) * 65536u + (__float_as_uint(a) >> 16));
        } else {
            const float *aux = p.aux + (size_t)l * p.aux_stride;
            const float alog = __ldg(aux + 14 * p.H + kHeadDim + h), dtb = __ldg(aux + 14 * p.H + kHeadDim + p.nh + h);
            decay = exp_ref(__fmul_rn(-exp_ref(alog), softplus_ref(__fadd_rn(a, dtb))));
        }
        sm_hscal()[hs * 8 + 1] = sigmoid_b<MODE>(p, bb);
        sm_hscal()[hs * 8 + 2] = decay;
    }
    /* 2. q, k and v arrive */
    float w5[5];
    ok = xfinish<5, Mode<MODE>::kTp>(p, qaddr, qtag, qw, qmiss) && ok;
#pragma unroll
    for (int k = 0; k < 5; ++k) w5[k] = quse(k) ? xval(qw[k]) : 0.0f;
    if (t == 0) trace_put(p, pidx, 1);
    {
        float sq[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) sq[i] = __fmul_rn(w5[i], w5[i]);
        block_sum8<4>(sq, sm_red());
        float al[2];
#pragma unroll
        for (uint32_t hs = 0; hs < 2; ++hs) {
            const float q_inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(sq[2 * hs], 1e-6f)));
            const float k_inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(sq[2 * hs + 1], 1e-6f)));
            const float qn = __fmul_rn(w5[2 * hs], q_inv), kn = __fmul_rn(w5[2 * hs + 1], k_inv);
            if (t < kHeadDim && hs < nhl) {
                sm_qn()[hs * kHeadDim + t] = qn;
                sm_kn()[hs * kHeadDim + t] = kn;
            }
            al[hs] = __fmul_rn(qn, kn);
        }
        block_sum8<2>(al, sm_red() + 64);
        if (t == 0) {
            sm_hscal()[0] = al[0];
            if (nhl > 1) sm_hscal()[8] = al[1];
        }
    }
    named_sync(1, kConsumerThreads);
    if (t == 0) trace_put(p, pidx, 6);
    /* 3. the state chunk */
    const uint32_t cb = state_col_bytes<MODE>();
    const bool part = (uint32_t)warp < state_warps(n);
    bool have = false;
    if (part) have = wait_full(p, q);
    const uint8_t *slot = sm_slot(q % kSlots);
    /* read pass: warp 0 lane j runs the r chain of column c0 + j, warp 1 the p chain */
    if (have && warp < 2 && (uint32_t)lane < n) {
        const uint32_t v = c0 + lane, hs = (v >> 8) - h0, sw = v & 7u;
        const float *vec = (warp == 0 ? sm_kn() : sm_qn()) + hs * kHeadDim;
        const uint8_t *col = slot + lane * cb;
        float acc = 0.0f;
        if (Mode<MODE>::kBf16State) {
            /* the next piece's loads are issued before this piece's chain */
            uint4 sn = lds128(col + (sw << 4));
            float4 x0n = *reinterpret_cast<const float4 *>(vec), x1n = *reinterpret_cast<const float4 *>(vec + 4);
#pragma unroll 4
            for (uint32_t c = 0; c < 32; ++c) {
                const uint4 s = sn;
                const float4 x0 = x0n, x1 = x1n;
                if (c + 1 < 32) {
                    sn = lds128(col + (((c + 1) ^ sw) << 4));
                    x0n = *reinterpret_cast<const float4 *>(vec + 8 * (c + 1));
                    x1n = *reinterpret_cast<const float4 *>(vec + 8 * (c + 1) + 4);
                }
                acc = __fadd_rn(acc, __fmul_rn(bf_lo(s.x), x0.x));
                acc = __fadd_rn(acc, __fmul_rn(bf_hi(s.x), x0.y));
                acc = __fadd_rn(acc, __fmul_rn(bf_lo(s.y), x0.z));
                acc = __fadd_rn(acc, __fmul_rn(bf_hi(s.y), x0.w));
                acc = __fadd_rn(acc, __fmul_rn(bf_lo(s.z), x1.x));
                acc = __fadd_rn(acc, __fmul_rn(bf_hi(s.z), x1.y));
                acc = __fadd_rn(acc, __fmul_rn(bf_lo(s.w), x1.z));
                acc = __fadd_rn(acc, __fmul_rn(bf_hi(s.w), x1.w));
            }
        } else {
#pragma unroll 4
            for (uint32_t c = 0; c < 64; ++c) {
                const float4 s = *reinterpret_cast<const float4 *>(col + ((c ^ sw) << 4));
                const float4 x0 = *reinterpret_cast<const float4 *>(vec + 4 * c);
                acc = __fadd_rn(acc, __fmul_rn(s.x, x0.x));
                acc = __fadd_rn(acc, __fmul_rn(s.y, x0.y));
                acc = __fadd_rn(acc, __fmul_rn(s.z, x0.z));
                acc = __fadd_rn(acc, __fmul_rn(s.w, x0.w));
            }
        }
        sm_hscal()[16 + 16 * warp + lane] = acc;  /* r at [16, 32), p at [32, 48) */
    }
    named_sync(1, kConsumerThreads);
    if (t == 0) trace_put(p, pidx, 5);
    if (have && warp == 0 && (uint32_t)lane < n) {
        const uint32_t v = c0 + lane, hs = (v >> 8) - h0;
        const float r = sm_hscal()[16 + lane], pp = sm_hscal()[32 + lane];
        const float alpha = sm_hscal()[hs * 8 + 0], beta = sm_hscal()[hs * 8 + 1], decay = sm_hscal()[hs * 8 + 2];
        const float delta = __fmul_rn(beta, __fsub_rn(w5[4], __fmul_rn(decay, r)));
        const float o = __fmul_rn(0.0625f, __fadd_rn(__fmul_rn(decay, pp), __fmul_rn(alpha, delta)));
        xput<MODE>(p, p.attn, v, bnd<MODE>(o), tag_out);
        sm_hscal()[48 + lane] = delta;
    }
    named_sync(1, kConsumerThreads);
    /* update: warp j writes column c0 + j back (16-byte pieces, swizzled) */
    if (have && (uint32_t)warp < n) {
        const uint32_t j = (uint32_t)warp, v = c0 + j, hs = (v >> 8) - h0, sw = v & 7u;
        const float decay = sm_hscal()[hs * 8 + 2], delta = sm_hscal()[48 + j];
        const float *kn = sm_kn() + hs * kHeadDim;
        const uint8_t *col = slot + j * cb;
        uint8_t *dst = reinterpret_cast<uint8_t *>(p.S) + ((size_t)l * p.nh * kHeadDim + v) * cb;
        if (Mode<MODE>::kBf16State) {
            const uint32_t c = (uint32_t)lane;
            const uint4 s = lds128(col + ((c ^ sw) << 4));
            const float4 k0 = *reinterpret_cast<const float4 *>(kn + 8 * c);
            const float4 k1 = *reinterpret_cast<const float4 *>(kn + 8 * c + 4);
            const float kk[8] = {k0.x, k0.y, k0.z, k0.w, k1.x, k1.y, k1.z, k1.w};
            const uint32_t sv[4] = {s.x, s.y, s.z, s.w};
            uint32_t o[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float lo = bf16_round(__fadd_rn(__fmul_rn(decay, bf_lo(sv[i])), __fmul_rn(kk[2 * i], delta)));
                const float hi =
                    bf16_round(__fadd_rn(__fmul_rn(decay, bf_hi(sv[i])), __fmul_rn(kk[2 * i + 1], delta)));
                o[i] = (__float_as_uint(lo) >> 16) | (__float_as_uint(hi) & 0xffff0000u);
            }
            *reinterpret_cast<uint4 *>(dst + ((c ^ sw) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
        } else {
#pragma unroll
            for (uint32_t half = 0; half < 2; ++half) {
                const uint32_t c = (uint32_t)lane + 32u * half;
                const float4 s = *reinterpret_cast<const float4 *>(col + ((c ^ sw) << 4));
                const float4 k0 = *reinterpret_cast<const float4 *>(kn + 4 * c);
                float4 o;
                o.x = __fadd_rn(__fmul_rn(decay, s.x), __fmul_rn(k0.x, delta));
                o.y = __fadd_rn(__fmul_rn(decay, s.y), __fmul_rn(k0.y, delta));
                o.z = __fadd_rn(__fmul_rn(decay, s.z), __fmul_rn(k0.z, delta));
                o.w = __fadd_rn(__fmul_rn(decay, s.w), __fmul_rn(k0.w, delta));
                *reinterpret_cast<float4 *>(dst + ((c ^ sw) << 4)) = o;
            }
        }
    }
    if (have) release(q);
    if (t == 0) trace_put(p, pidx, 7);
    ++q;
    return ok;
}

/* ------------------------------------------------------------ the kernel */

enum { PH_QKVG = 0, PH_STATE = 1, PH_O = 2, PH_GU = 3, PH_DOWN = 4, PH_LM = 5 };

/* argmax merge: larger value, lowest index on ties (c_impl/gdn_model.cpp:4775-4925) */
__device__ __forceinline__ void better(float &b, int32_t &bi, float v, int32_t vi) {
    if (v > b || (v == b && vi < bi)) {
        b = v;
        bi = vi;
    }
}

template <int MODE>
__global__ void __launch_bounds__(kThreads, 1) gdn_decode_kernel(const __grid_constant__ DecodeParams p) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, t = threadIdx.x;
    /* the global CTA index: unit partitions run over every GPU's CTAs */
    const uint32_t cta = (uint32_t)p.tp_rank * gridDim.x + blockIdx.x, ncta = (uint32_t)p.tp_world * gridDim.x;

    if (t < 128) reinterpret_cast<float *>(smem_raw + kOffExpTab)[t] = __ldg(p.exp_table + t);
    if (t < kSlots) sm_issued()[t] = 0;
    if (t == 64) {
        for (int i = 0; i < kSlots; ++i) {
            mbar_init(smem_u32(&sm_full()[i]), 1);
            mbar_init(smem_u32(&sm_empty()[i]), kConsumerWarps);
        }
        *sm_abort_flag() = 0;
        *sm_decision() = 1;
        sm_exact()[0] = 0;
        sm_exact()[1] = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    build_sched<MODE>(p, cta, ncta);
    __syncthreads();

    if (warp == kProducerWarp) {
        producer<MODE>(p, cta, ncta);
    } else {
        prefetch_floats(sm_normw(), p.aux, p.H);
        prefetch_floats(sm_onorm(), p.aux + p.H, kHeadDim);
        uint32_t q = 0;
        float best = -3.402823466e38f;
        int32_t best_i = 0x7fffffff;
        bool ok = true;
        const Span sc{sm_sched()->c0, sm_sched()->c0 + sm_sched()->ncols};
        /* the layer and phase loops stay rolled: unrolled, every phase kind
         * gets its own copy of the chunk code and the kernel outgrows the
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
                const int xf = pidx & 1;
                const uint32_t tag_out = tag_base + (uint32_t)ph;
                /* every consumer warp is done with the previous phase (shared
                 * inputs may be overwritten) */
                named_sync(1, kConsumerThreads);
                if (t == 0) {
                    trace_put(p, pidx, 0);
                    sm_exact()[xf ^ 1] = 0;
                }
                switch (ph) {
                case PH_QKVG:
                    if (l == 0) {
                        if (p.token_src != nullptr || p.token_imm >= 0) {
                            const int32_t tok = p.token_src != nullptr ? *p.token_src : p.token_imm;
                            if (tok < 0 || tok >= p.V) {
                                /* every consumer thread reads the same token: uniform exit */
                                if (t == 0) raise_error(p, kErrBadToken, (uint32_t)tok);
                                ok = false;
                                break;
                            }
                        }
                        prologue_norm<MODE>(p, nullptr, 0, aux, true, nullptr, pidx, xf);
                    } else {
                        prologue_norm<MODE>(p, p.y_down, tag_base - kPhasesPerLayer + PH_DOWN, aux, false, nullptr,
                                            pidx, xf);
                    }
                    break;
                case PH_STATE:
                    break;
                case PH_O:
                    prologue_norm_gate<MODE>(p, aux + p.H, tag_base + PH_QKVG, tag_base + PH_STATE, pidx, xf);
                    break;
                case PH_GU:
                    prologue_norm<MODE>(p, p.y_o, tag_base + PH_O, aux + p.H + kHeadDim, false, nullptr, pidx, xf);
                    break;
                case PH_DOWN:
                    xread_to_xs<MODE>(p, p.m, p.I, tag_base + PH_GU, xf);
                    if (t == 0) trace_put(p, pidx, 1);
                    break;
                default:
                    prologue_norm<MODE>(p, p.y_down, p.epoch + (uint32_t)((p.L - 1) * kPhasesPerLayer + PH_DOWN),
                                        p.aux + (size_t)p.L * p.aux_stride, false,
                                        blockIdx.x == 0 ? p.hidden_out : nullptr, pidx, xf);
                    break;
                }
                if (!ok) break;
                /* a failed read has raised the abort flag */
                if (t == 0) *sm_decision() = (*sm_abort_flag() == 0) ? 1 : 0;
                named_sync(1, kConsumerThreads);
                if (*sm_decision() == 0) { ok = false; break; }
                if (t == 0) trace_put(p, pidx, 2);
                /* the prologue is done with its norm weights: fetch the next ones */
                if (ph == PH_QKVG) {
                    const Wide &g = sm_sched()->qkvg;
                    prefetch_floats_idle(sm_normw(), aux + p.H + kHeadDim, p.H,
                                         min(g.P, g.t1 - g.t0) * (g.TR / 8));                 /* mlp_norm[l] */
                } else if (ph == PH_GU) {
                    const Wide &g = sm_sched()->gu;
                    prefetch_floats_idle(sm_normw(),
                                         l + 1 < p.L ? aux + p.aux_stride : p.aux + (size_t)p.L * p.aux_stride, p.H,
                                         min(g.P, g.t1 - g.t0) * (g.TR / 8));                 /* attn_norm[l+1] / final */
                } else if (ph == PH_O && l + 1 < p.L) {
                    prefetch_floats_idle(sm_onorm(), aux + p.aux_stride + p.H, kHeadDim,
                                         sm_sched()->o.r1 - sm_sched()->o.r0);                /* o_norm[l+1] */
                }
                const bool exact = Mode<MODE>::kNative && (sm_exact()[xf] != 0 || p.force_exact != 0);
                const bool drop = (int)cta == p.test_drop_cta && pidx == p.test_drop_phase;
                if (ph == PH_STATE) {
                    phase_state<MODE>(p, l, q, sc.u0, sc.u1, tag_base + PH_QKVG, tag_out, pidx);
                    q += 2;
                } else if (ph == PH_O || ph == PH_DOWN) {
                    Narrow w = ph == PH_O ? sm_sched()->o : sm_sched()->down;
                    w.base += (size_t)l * p.layer_stride;
                    const uint32_t q0 = q;
                    const float total = gemv_dispatch<MODE>(
                        exact, [&, q0](auto K) { return narrow_chunks<decltype(K)::value, Mode<MODE>::kTp>(p, w, q0); });
                    q += Mode<MODE>::kTp ? w.chunks_ng(p.ng_narrow) : w.chunks();
                    if (!drop && lane == 0 && (uint32_t)warp < w.r1 - w.r0)
                        xput<MODE>(p, ph == PH_O ? p.y_o : p.y_down, w.r0 + warp, bnd<MODE>(total), tag_out);
                } else {
                    Wide w = ph == PH_QKVG ? sm_sched()->qkvg : ph == PH_GU ? sm_sched()->gu : sm_sched()->lm;
                    if (ph != PH_LM) w.base += (size_t)l * p.layer_stride;
                    const uint32_t wpt = w.TR / 8, tw = (uint32_t)warp / wpt;
                    const uint32_t rr = ((uint32_t)warp % wpt) * 8u + ((uint32_t)lane >> 2);
                    const bool head = (lane & 3) == 0;
                    for (uint32_t pass = 0; pass < w.passes(); ++pass) {
                        const uint32_t pt0 = w.t0 + pass * w.P, n = min(w.P, w.t1 - pt0);
                        const bool active = tw < n;
                        const uint32_t row = (pt0 + tw) * w.TR + rr;
                        /* QKVG: the row's conv window and weights, copied into shared
                         * memory while the chunks stream (held in registers across the
                         * chunk loop they would spill) */
                        float4 *tw_sh = reinterpret_cast<float4 *>(sm_scratch()) + 2 * (warp * 8 + (lane >> 2));
                        const bool conv_row = ph == PH_QKVG && active && head && row < 3u * p.H;
                        /* q, k or v row (no division: a compare per kind) */
                        const uint32_t kind = (uint32_t)(row >= (uint32_t)p.H) + (uint32_t)(row >= 2u * p.H);
                        const uint32_t d = row - kind * (uint32_t)p.H;
                        if (conv_row) {
                            cp_async16(smem_u32(tw_sh), p.tails + (((size_t)l * 3 + kind) * p.H + d) * 4);
                            cp_async16(smem_u32(tw_sh + 1), aux + 2 * p.H + kHeadDim + ((size_t)kind * p.H + d) * 4);
                            cp_async_commit();
                        }
                        const uint32_t q0 = q;
                        const float total = gemv_dispatch<MODE>(
                            exact, [&, q0](auto K) { return wide_chunks<decltype(K)::value, Mode<MODE>::kTp>(p, w, n, q0); });
                        q += w.chunks_per_pass();
                        const float up = __shfl_down_sync(0xffffffffu, total, 4);
                        if (!active || !head || drop) continue;
                        if (ph == PH_QKVG) {
                            const float raw = bnd<MODE>(total);
                            if (conv_row) {
                                cp_async_wait_all();
                                const float4 tail = tw_sh[0], cw = tw_sh[1];
                                /* depthwise conv over [t0 t1 t2 new] + SiLU, left to right
                                 * (c_impl/gdn_model.cpp:1630-1653), then the window shift */
                                const float sum = __fadd_rn(
                                    __fadd_rn(__fadd_rn(__fmul_rn(tail.x, cw.x), __fmul_rn(tail.y, cw.y)),
                                              __fmul_rn(tail.z, cw.z)),
                                    __fmul_rn(raw, cw.w));
                                xput<MODE>(p, p.qkv, row, silu_conv<MODE>(p, sum), tag_out);
                                __stcg(reinterpret_cast<float4 *>(p.tails + (((size_t)l * 3 + kind) * p.H + d) * 4),
                                       make_float4(tail.y, tail.z, raw, 0.0f));
                            } else {
                                xput_gate<MODE>(p, row - 3u * p.H, raw, Mode<MODE>::kBf16 ? sigmoid_b<MODE>(p, raw) : 0.0f,
                                                tag_out);
                            }
                        } else if (ph == PH_GU) {
                            /* rows 2i (gate) and 2i + 1 (up); SwiGLU as c_impl/gdn_model.cpp:4751-4770 */
                            if ((rr & 1u) == 0) {
                                const float gv = bnd<MODE>(total), uv = bnd<MODE>(up);
                                xput<MODE>(p, p.m, row >> 1,
                                           bnd<MODE>(__fmul_rn(__fmul_rn(gv, sigmoid_b<MODE>(p, gv)), uv)), tag_out);
                            }
                        } else {
                            p.logits[row] = total;
                            if (Mode<MODE>::kTp)
                                for (int r = 0; r < p.tp_world; ++r)
                                    if (r != p.tp_rank) *peer_addr(p, p.logits + row, r) = total;
                            better(best, best_i, total, (int32_t)row);
                        }
                    }
                }
                if (t == 0) trace_put(p, pidx, 3);
            }
        }

        /* LM-head argmax: warps -> CTA candidate -> the last CTA picks the token */
        named_sync(1, kConsumerThreads);
        if (t == 0) *sm_decision() = (ok && *sm_abort_flag() == 0) ? 1 : 0;
        named_sync(1, kConsumerThreads);
        if (*sm_decision() != 0) {
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const float v = __shfl_xor_sync(0xffffffffu, best, o);
                const int32_t vi = __shfl_xor_sync(0xffffffffu, best_i, o);
                better(best, best_i, v, vi);
            }
            if (lane == 0) {
                sm_wbest()[warp] = best;
                sm_wbest_i()[warp] = best_i;
            }
            named_sync(1, kConsumerThreads);
            if (t == 0) {
                float b = sm_wbest()[0];
                int32_t bi = sm_wbest_i()[0];
                for (int w = 1; w < kConsumerWarps; ++w) better(b, bi, sm_wbest()[w], sm_wbest_i()[w]);
                p.cand_val[blockIdx.x] = b;
                p.cand_idx[blockIdx.x] = bi;
                /* tensor-parallel: the logits this CTA stored into the peers'
                 * regions are visible there before its GPU's candidate is */
                if (Mode<MODE>::kTp) __threadfence_system();
                else __threadfence();
                const uint32_t ticket = atomicAdd(&p.status->done, 1u);
                if (ticket == gridDim.x - 1) {
                    __threadfence();
                    float gb = __ldcg(p.cand_val);
                    int32_t gi = __ldcg(p.cand_idx);
                    for (uint32_t c = 1; c < gridDim.x; ++c) better(gb, gi, __ldcg(p.cand_val + c), __ldcg(p.cand_idx + c));
                    if (Mode<MODE>::kTp) {
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
                            if (r == 0) {
                                gb = fv;
                                gi = iv;
                            } else {
                                better(gb, gi, fv, iv);
                            }
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
    if (t == 0) {
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
    /* the shared-memory opt-in, once per device and size (it costs a driver
     * call per launch otherwise) */
    static std::atomic<size_t> smem_set[64];
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::atomic<size_t> &done = smem_set[dev & 63];
    if (dev >= 64 || done.load(std::memory_order_acquire) < smem) {
        e = cudaFuncSetAttribute(gdn_decode_kernel<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        if (dev < 64) done.store(smem, std::memory_order_release);
    }
    return cudaLaunchCooperativeKernel((const void *)gdn_decode_kernel<MODE>, dim3(grid), dim3(kThreads), args, smem,
                                       stream);
}

/* The contracts: FP32 control (boundaries, products and state FP32), engine
 * (BF16 boundaries, exact products, FP32 state), c_impl (BF16 boundaries,
 * BF16-rounded products, BF16 state); tensor-parallel forms of each. */
cudaError_t launch_decode(const DecodeParams &p, int grid, cudaStream_t stream) {
    const size_t smem = decode_smem_bytes(p.H, p.I, p.tp_world > 1);
    const bool fp32 = !p.bf16_boundary && !p.native_product && !p.bf16_state;
    const bool engine = p.bf16_boundary && !p.native_product && !p.bf16_state;
    const bool cimpl = p.bf16_boundary && p.native_product && p.bf16_state;
    if (!(fp32 || engine || cimpl)) return cudaErrorInvalidValue;
    if (p.tp_world > 1) {
        if (fp32) return launch_mode<4>(p, grid, stream, smem);
        return engine ? launch_mode<5>(p, grid, stream, smem) : launch_mode<15>(p, grid, stream, smem);
    }
    if (fp32) return launch_mode<0>(p, grid, stream, smem);
    return engine ? launch_mode<1>(p, grid, stream, smem) : launch_mode<11>(p, grid, stream, smem);
}

/* ------------------------------------------- state layout conversions */

/* Run-state storage (16-byte pieces of column v at p ^ (v & 7); FP32 or
 * BF16) <-> natural FP32 [column][256]. One thread per 16-byte piece. */
__global__ void state_to_fp32_kernel(const uint8_t *S, int bf16, float *dst, size_t cols) {
    const size_t pieces = cols * (bf16 ? 32 : 64);
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < pieces; i += (size_t)gridDim.x * blockDim.x) {
        const size_t col = bf16 ? i >> 5 : i >> 6;
        const uint32_t c = (uint32_t)(bf16 ? i & 31 : i & 63), pc = c ^ (uint32_t)(col & 7);
        if (bf16) {
            const uint4 s = *reinterpret_cast<const uint4 *>(S + col * 512 + pc * 16);
            float *d = dst + col * 256 + c * 8;
            const uint32_t sv[4] = {s.x, s.y, s.z, s.w};
            for (int k = 0; k < 4; ++k) {
                d[2 * k] = bf_lo(sv[k]);
                d[2 * k + 1] = bf_hi(sv[k]);
            }
        } else {
            *reinterpret_cast<float4 *>(dst + col * 256 + c * 4) =
                *reinterpret_cast<const float4 *>(S + col * 1024 + pc * 16);
        }
    }
}
__global__ void state_from_fp32_kernel(const float *src, uint8_t *S, int bf16, size_t cols) {
    const size_t pieces = cols * (bf16 ? 32 : 64);
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < pieces; i += (size_t)gridDim.x * blockDim.x) {
        const size_t col = bf16 ? i >> 5 : i >> 6;
        const uint32_t c = (uint32_t)(bf16 ? i & 31 : i & 63), pc = c ^ (uint32_t)(col & 7);
        if (bf16) {
            const float *s = src + col * 256 + c * 8;
            uint32_t o[4];
            for (int k = 0; k < 4; ++k)
                o[k] = (__float_as_uint(bf16_round(s[2 * k])) >> 16) | (__float_as_uint(bf16_round(s[2 * k + 1])) & 0xffff0000u);
            *reinterpret_cast<uint4 *>(S + col * 512 + pc * 16) = make_uint4(o[0], o[1], o[2], o[3]);
        } else {
            *reinterpret_cast<float4 *>(S + col * 1024 + pc * 16) =
                *reinterpret_cast<const float4 *>(src + col * 256 + c * 4);
        }
    }
}
cudaError_t launch_state_to_fp32(const void *S, int bf16, float *dst, size_t cols, cudaStream_t stream) {
    state_to_fp32_kernel<<<592, 256, 0, stream>>>(reinterpret_cast<const uint8_t *>(S), bf16, dst, cols);
    return cudaGetLastError();
}
cudaError_t launch_state_from_fp32(const float *src, void *S, int bf16, size_t cols, cudaStream_t stream) {
    state_from_fp32_kernel<<<592, 256, 0, stream>>>(src, reinterpret_cast<uint8_t *>(S), bf16, cols);
    return cudaGetLastError();
}

}  // namespace gdn
