/* Seeded synthetic inputs for GatedDeltaNet decode: weights, token streams and
 * recurrent state, generated deterministically from (seed, tensor, index).
 *
 * There is no checkpoint and no dataset on this machine, so every run (engine,
 * CPU oracle, reference build) rebuilds the same tensors from a master seed.
 * The generator is counter based: element i of tensor t depends only on
 * (seed, t, i), so callers may fill any sub-range from any thread and obtain
 * identical bits.
 *
 * Distributions (the unspecified ones follow the FLA-style
 * initialisation of lit_gpt/gated_delta_net.py:105-121 in the reference):
 *   linear weights (embeddings, q/k/v/g/o, a/b proj, gate/up/down, lm_head): N(0, 0.02)
 *   norm weights (attn_norm, o_norm, mlp_norm, final_norm):                 1.0
 *   short-conv kernels (q/k/v_conv, fan-in 4):                               U(-0.5, 0.5)
 *   A_log = log(U(0, 16));  dt_bias = softplus^-1(clamp(exp(U(ln 1e-3, ln 0.1)), 1e-4))
 * Every value is rounded to BF16 (round-to-nearest-even) and stored as an FP32
 * word, because the .gdnw loader accepts BF16-exact words only
 * (c_impl/gdn_model.cpp:1190-1216).
 *
 * Tensor ids follow the .gdnw blob order (scripts/export_gdn_c.py:138-166):
 *   0 = embeddings, then per layer l the 18 tensors at 1 + 18*l + j
 *   (j = GDN_SYNTH_* below), then final_norm, then lm_head.
 */
#ifndef GDN_SYNTH_H
#define GDN_SYNTH_H

#include <math.h>
#include <stdint.h>
#include <string.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    GDN_SYNTH_ATTN_NORM = 0,
    GDN_SYNTH_A_LOG,
    GDN_SYNTH_DT_BIAS,
    GDN_SYNTH_Q_PROJ,
    GDN_SYNTH_K_PROJ,
    GDN_SYNTH_V_PROJ,
    GDN_SYNTH_A_PROJ,
    GDN_SYNTH_B_PROJ,
    GDN_SYNTH_Q_CONV,
    GDN_SYNTH_K_CONV,
    GDN_SYNTH_V_CONV,
    GDN_SYNTH_G_PROJ,
    GDN_SYNTH_O_NORM,
    GDN_SYNTH_O_PROJ,
    GDN_SYNTH_MLP_NORM,
    GDN_SYNTH_MLP_GATE,
    GDN_SYNTH_MLP_UP,
    GDN_SYNTH_MLP_DOWN,
    GDN_SYNTH_TENSORS_PER_LAYER
};

enum {
    GDN_DIST_NORMAL_002 = 0, /* N(0, 0.02) */
    GDN_DIST_ONES,
    GDN_DIST_CONV,           /* U(-0.5, 0.5) */
    GDN_DIST_A_LOG,
    GDN_DIST_DT_BIAS
};

/* Stream ids outside the weight range (token streams, states). */
#define GDN_SYNTH_STREAM_TOKENS   0x70000000u
#define GDN_SYNTH_STREAM_STATE    0x71000000u
#define GDN_SYNTH_STREAM_MICRO    0x72000000u

static inline uint64_t gdn_synth_mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

static inline uint64_t gdn_synth_key(uint64_t seed, uint64_t stream) {
    return gdn_synth_mix64(seed ^ gdn_synth_mix64(stream * 0xD1B54A32D192ED03ull + 0x1234567ull));
}

/* Position idx of a splitmix64 sequence keyed by (seed, stream). */
static inline uint64_t gdn_synth_u64(uint64_t key, uint64_t idx) {
    return gdn_synth_mix64(key + (idx + 1u) * 0x9E3779B97F4A7C15ull);
}

/* Uniform double in the open interval (0, 1). */
static inline double gdn_synth_unit(uint64_t r) {
    return ((double)(r >> 11) + 0.5) * (1.0 / 9007199254740992.0);
}

static inline uint32_t gdn_synth_f32_bits(float v) {
    uint32_t b;
    memcpy(&b, &v, 4);
    return b;
}

static inline float gdn_synth_bits_f32(uint32_t b) {
    float v;
    memcpy(&v, &b, 4);
    return v;
}

/* FP32 -> BF16 round-to-nearest-even, NaN canonicalised; returned widened. */
static inline float gdn_synth_round_bf16(float v) {
    uint32_t b = gdn_synth_f32_bits(v);
    uint32_t mag = b & 0x7fffffffu;
    if (mag >= 0x7f800000u) {
        if (mag == 0x7f800000u) return v;
        return gdn_synth_bits_f32((b & 0x80000000u) ? 0xffc00000u : 0x7fc00000u);
    }
    b = (b + 0x7fffu + ((b >> 16) & 1u)) & 0xffff0000u;
    return gdn_synth_bits_f32(b);
}

/* Distribution of tensor `tensor_id` in the blob order. */
static inline int gdn_synth_tensor_dist(uint32_t tensor_id, uint32_t num_layers) {
    if (tensor_id == 0) return GDN_DIST_NORMAL_002;                     /* embeddings */
    if (tensor_id == 1 + GDN_SYNTH_TENSORS_PER_LAYER * num_layers) return GDN_DIST_ONES; /* final_norm */
    if (tensor_id == 2 + GDN_SYNTH_TENSORS_PER_LAYER * num_layers) return GDN_DIST_NORMAL_002; /* lm_head */
    switch ((tensor_id - 1) % GDN_SYNTH_TENSORS_PER_LAYER) {
    case GDN_SYNTH_ATTN_NORM:
    case GDN_SYNTH_O_NORM:
    case GDN_SYNTH_MLP_NORM: return GDN_DIST_ONES;
    case GDN_SYNTH_A_LOG: return GDN_DIST_A_LOG;
    case GDN_SYNTH_DT_BIAS: return GDN_DIST_DT_BIAS;
    case GDN_SYNTH_Q_CONV:
    case GDN_SYNTH_K_CONV:
    case GDN_SYNTH_V_CONV: return GDN_DIST_CONV;
    default: return GDN_DIST_NORMAL_002;
    }
}

/* Fill dst[0 .. end-begin) with elements [begin, end) of a tensor, already
 * rounded to BF16 and stored as FP32 words. Normal values come from
 * Box-Muller pairs (element 2j uses the cosine branch, 2j+1 the sine branch of
 * pair j), so any sub-range reproduces the same bits. */
static inline void gdn_synth_fill(float *dst, uint64_t seed, uint32_t tensor_id,
                                  int dist, uint64_t begin, uint64_t end) {
    const uint64_t key = gdn_synth_key(seed, tensor_id);
    uint64_t i = begin;
    while (i < end) {
        float value;
        switch (dist) {
        case GDN_DIST_ONES:
            value = 1.0f;
            break;
        case GDN_DIST_CONV:
            value = (float)(gdn_synth_unit(gdn_synth_u64(key, i)) - 0.5);
            break;
        case GDN_DIST_A_LOG:
            value = (float)log(16.0 * gdn_synth_unit(gdn_synth_u64(key, i)));
            break;
        case GDN_DIST_DT_BIAS: {
            const double lo = log(0.001), hi = log(0.1);
            double dt = exp(gdn_synth_unit(gdn_synth_u64(key, i)) * (hi - lo) + lo);
            if (dt < 1e-4) dt = 1e-4;
            value = (float)(dt + log(-expm1(-dt)));
            break;
        }
        default: {
            const uint64_t pair = i >> 1;
            const double u1 = gdn_synth_unit(gdn_synth_u64(key, 2 * pair));
            const double u2 = gdn_synth_unit(gdn_synth_u64(key, 2 * pair + 1));
            const double r = sqrt(-2.0 * log(u1)) * 0.02;
            const double th = 6.283185307179586 * u2;
            if ((i & 1u) == 0 && i + 1 < end) {
                /* both members of the pair are wanted: share the radius */
                dst[i - begin] = gdn_synth_round_bf16((float)(r * cos(th)));
                dst[i + 1 - begin] = gdn_synth_round_bf16((float)(r * sin(th)));
                i += 2;
                continue;
            }
            value = (float)(r * ((i & 1u) ? sin(th) : cos(th)));
            break;
        }
        }
        dst[i - begin] = gdn_synth_round_bf16(value);
        ++i;
    }
}

/* Seeded uniform token ids in [0, vocab): element i of stream `stream`. */
static inline int32_t gdn_synth_token(uint64_t seed, uint32_t stream, uint64_t i, uint32_t vocab) {
    const uint64_t r = gdn_synth_u64(gdn_synth_key(seed, GDN_SYNTH_STREAM_TOKENS + stream), i);
    return (int32_t)(((r >> 32) * (uint64_t)vocab) >> 32);
}

/* N(0, sigma) fp32 value i of an auxiliary stream (microbench state/inputs);
 * not rounded. */
static inline float gdn_synth_normal(uint64_t seed, uint32_t stream, uint64_t i, double sigma) {
    const uint64_t key = gdn_synth_key(seed, stream);
    const uint64_t pair = i >> 1;
    const double u1 = gdn_synth_unit(gdn_synth_u64(key, 2 * pair));
    const double u2 = gdn_synth_unit(gdn_synth_u64(key, 2 * pair + 1));
    const double r = sqrt(-2.0 * log(u1)) * sigma;
    const double th = 6.283185307179586 * u2;
    return (float)(r * ((i & 1u) ? sin(th) : cos(th)));
}

#ifdef __cplusplus
}
#endif

#endif /* GDN_SYNTH_H */
