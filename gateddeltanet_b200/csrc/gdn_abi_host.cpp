/* gdn_abi_host.cpp -- the reference's host-side image helpers (c_impl/
 * gdn_model.h:170-195, behaviour c_impl/gdn_model.cpp:338-366, 595-1080),
 * restated so that a caller of the reference's ABI links and runs unchanged:
 * the 32 packed-BF16 GEMV shards of the FPGA's HBM ports, the packed aux
 * image, the recurrent-state stripes at the tails of shards 28..31 and the
 * BF16 conv-tail packing of the workspace head buffer. The layouts are the
 * reference's formats (a caller may read them back, e.g. c_impl/gdn_eval.cpp's
 * state dump), so they are reproduced exactly; the engine itself never reads
 * the shards -- it keeps its own device image -- but state written through
 * gdn_scatter_recurrent_state / gdn_pack_conv_tails_bf16 is picked up by the
 * next decode step of the run state that owns those buffers (gdn_host.cu).
 *
 * A 512-bit beat holds 32 BF16 lanes (lane i = bytes 2i, 2i+1) or 16 FP32
 * lanes (lane i = bytes 4i .. 4i+3), little-endian, as the reference's native
 * build stores ap_uint<512> (c_impl/gdn_model.cpp:225-274).
 */
#include "../../include/gdn_model.h"

#include <atomic>
#include <cstdio>
#include <cstring>
#include <thread>
#include <vector>

namespace gdn {
void host_note_state_write(const void *buffer);
}

namespace {

constexpr uint32_t kStatePorts = 4;      /* GDN_RECURRENT_STATE_PORTS, c_impl/gdn_model.h:84 */
constexpr uint32_t kDV = 256;            /* value_dim */
constexpr size_t kConvStripes = 24u * 3u;
constexpr size_t kConvFloatsPerStripe = GDN_WSF_HEADBUF / kConvStripes;

inline uint32_t f2u(float v) {
    uint32_t b;
    memcpy(&b, &v, 4);
    return b;
}
inline float u2f(uint32_t b) {
    float v;
    memcpy(&v, &b, 4);
    return v;
}
inline void set_bf16(Beat512 &b, uint32_t lane, uint16_t v) { memcpy(reinterpret_cast<uint8_t *>(&b) + 2 * lane, &v, 2); }
inline uint16_t get_bf16(const Beat512 &b, uint32_t lane) {
    uint16_t v;
    memcpy(&v, reinterpret_cast<const uint8_t *>(&b) + 2 * lane, 2);
    return v;
}
inline void set_fp32(Beat512 &b, uint32_t lane, uint32_t v) { memcpy(reinterpret_cast<uint8_t *>(&b) + 4 * lane, &v, 4); }
inline uint32_t get_fp32(const Beat512 &b, uint32_t lane) {
    uint32_t v;
    memcpy(&v, reinterpret_cast<const uint8_t *>(&b) + 4 * lane, 4);
    return v;
}
/* upper half of a BF16-exact FP32 word */
inline uint16_t bf16_of(float v) { return (uint16_t)(f2u(v) >> 16); }

template <typename F>
void parallel_for(size_t n, F fn) {
    unsigned hw = std::thread::hardware_concurrency();
    const size_t t = std::min<size_t>(std::max(1u, std::min(hw, 64u)), n ? n : 1);
    if (t <= 1) {
        fn((size_t)0, n);
        return;
    }
    std::vector<std::thread> th;
    for (size_t i = 0; i < t; ++i) th.emplace_back([=] { fn(n * i / t, n * (i + 1) / t); });
    for (auto &x : th) x.join();
}

/* blob geometry (c_impl/gdn_model.cpp:515-587) */
size_t layer_floats(const GDNWeightHeader *c) {
    const size_t H = c->hidden_size, nh = c->num_heads, hd = c->head_dim, I = c->intermediate_size, cs = c->conv_size;
    return H + 2 * nh + 3 * H * H + 2 * nh * H + 3 * H * cs + H * H + hd + H * H + H + 2 * I * H + H * I;
}
size_t layer_offset(const GDNWeightHeader *c, uint32_t l) {
    return (size_t)c->vocab_size * c->hidden_size + (size_t)l * layer_floats(c);
}
size_t final_norm_offset(const GDNWeightHeader *c) { return layer_offset(c, c->num_layers); }
size_t total_floats(const GDNWeightHeader *c) { return final_norm_offset(c) + c->hidden_size + (size_t)c->vocab_size * c->hidden_size; }

/* The rows [row0, row0 + rows) of a [.][cols] matrix, in groups of eight rows:
 * per group, per 32-column beat, one beat per row (c_impl/gdn_model.cpp:611-633). */
struct RowBlock {
    const float *src;
    size_t rows, cols;
    size_t beats() const { return rows * (cols / 32); }
    Beat512 beat(size_t i) const {
        const size_t per_group = 8 * (cols / 32);
        const size_t group = i / per_group, within = i % per_group;
        const size_t wb = within / 8, row = group * 8 + within % 8;
        Beat512 b;
        const float *r = src + row * cols + wb * 32;
        for (uint32_t lane = 0; lane < 32; ++lane) set_bf16(b, lane, bf16_of(r[lane]));
        return b;
    }
};

/* Walk of the shard image (c_impl/gdn_model.cpp:690-759): fn(channel, beat
 * offset in the channel's shard, block) for every block in shard order. */
template <typename F>
void walk_shards(const float *wd, const GDNWeightHeader *c, F fn) {
    const size_t H = c->hidden_size, I = c->intermediate_size, nh = c->num_heads, hd = c->head_dim,
                 cs = c->conv_size, CH = GEMV_CHANNELS;
    size_t soff = 0;
    for (uint32_t l = 0; l < c->num_layers; ++l) {
        const size_t base = layer_offset(c, l);
        const size_t q = base + H + 2 * nh, k = q + H * H, v = k + H * H;
        const size_t g = v + H * H + 2 * nh * H + 3 * H * cs;
        const size_t o = g + H * H + hd, mg = o + H * H + H, mu = mg + I * H, md = mu + I * H;
        const size_t qkvg[4] = {q, k, v, g};
        const size_t qrows = (4 * hd) / CH;
        for (size_t ch = 0; ch < CH; ++ch) {
            const size_t kind = ch / (CH / 4), seg = ch % (CH / 4);
            size_t dst = soff;
            for (size_t head = 0; head < nh; ++head) {
                const RowBlock blk{wd + qkvg[kind] + (head * hd + seg * qrows) * H, qrows, H};
                fn(ch, dst, blk);
                dst += blk.beats();
            }
        }
        soff += nh * qrows * (H / 32);
        const size_t orows = H / CH;
        for (size_t ch = 0; ch < CH; ++ch) fn(ch, soff, RowBlock{wd + o + ch * orows * H, orows, H});
        soff += orows * (H / 32);
        const size_t gurows = I / (CH / 2);
        const size_t gu[2] = {mg, mu};
        for (size_t ch = 0; ch < CH; ++ch) fn(ch, soff, RowBlock{wd + gu[ch & 1] + (ch >> 1) * gurows * H, gurows, H});
        soff += gurows * (H / 32);
        const size_t drows = H / CH;
        for (size_t ch = 0; ch < CH; ++ch) fn(ch, soff, RowBlock{wd + md + ch * drows * I, drows, I});
        soff += drows * (I / 32);
    }
    const size_t lm = final_norm_offset(c) + H, lrows = c->vocab_size / CH;
    for (size_t ch = 0; ch < CH; ++ch) fn(ch, soff, RowBlock{wd + lm + ch * lrows * H, lrows, H});
}

/* aux image geometry (c_impl/gdn_model.cpp:937-1028) */
size_t aux_layer_beats(const GDNWeightHeader *c) {
    const size_t H = c->hidden_size, nh = c->num_heads, hd = c->head_dim, cs = c->conv_size;
    return H / 32 + 1 + hd / 32 + H / 32 + (2 * nh * H) / 32 + (3 * H * cs) / 32;
}
struct AuxSources {
    const float *attn_norm, *a_log, *dt_bias, *a_proj, *b_proj, *q_conv, *k_conv, *v_conv, *o_norm, *mlp_norm;
};
AuxSources aux_sources(const float *wd, const GDNWeightHeader *c, uint32_t l) {
    const size_t H = c->hidden_size, nh = c->num_heads, hd = c->head_dim, cs = c->conv_size;
    const float *b = wd + layer_offset(c, l);
    AuxSources s;
    s.attn_norm = b;
    s.a_log = b + H;
    s.dt_bias = s.a_log + nh;
    s.a_proj = s.dt_bias + nh + 3 * H * H;
    s.b_proj = s.a_proj + nh * H;
    s.q_conv = s.b_proj + nh * H;
    s.k_conv = s.q_conv + H * cs;
    s.v_conv = s.k_conv + H * cs;
    s.o_norm = s.v_conv + H * cs + H * H;
    s.mlp_norm = s.o_norm + hd + H * H;
    return s;
}
/* fn(beat index, lane, kind, value bits): kind 0 = BF16 lane of a BF16-exact
 * source, 1 = FP32 lane */
template <typename F>
void walk_aux(const float *wd, const GDNWeightHeader *c, F fn) {
    const size_t H = c->hidden_size, nh = c->num_heads, hd = c->head_dim, cs = c->conv_size;
    const size_t per = aux_layer_beats(c);
    const size_t o_scal = H / 32, o_onorm = o_scal + 1, o_mlp = o_onorm + hd / 32, o_ab = o_mlp + H / 32;
    const size_t o_conv = o_ab + (2 * nh * H) / 32, conv_beats = (H * cs) / 32;
    auto lanes = [&](size_t beat0, const float *src, size_t n) {
        for (size_t i = 0; i < n; ++i) fn(beat0 + i / 32, (uint32_t)(i % 32), 0, f2u(src[i]));
    };
    for (uint32_t l = 0; l < c->num_layers; ++l) {
        const AuxSources s = aux_sources(wd, c, l);
        const size_t L0 = (size_t)l * per;
        lanes(L0, s.attn_norm, H);
        for (size_t h = 0; h < nh; ++h) {
            fn(L0 + o_scal, (uint32_t)h, 1, f2u(s.a_log[h]));
            fn(L0 + o_scal, (uint32_t)(nh + h), 1, f2u(s.dt_bias[h]));
        }
        lanes(L0 + o_onorm, s.o_norm, hd);
        lanes(L0 + o_mlp, s.mlp_norm, H);
        for (size_t ci = 0; ci < 2 * nh; ++ci) {
            const float *row = ci < nh ? s.a_proj + ci * H : s.b_proj + (ci - nh) * H;
            for (size_t j = 0; j < H / 32; ++j)
                for (uint32_t lane = 0; lane < 32; ++lane)
                    fn(L0 + o_ab + j * (2 * nh) + ci, lane, 0, f2u(row[j * 32 + lane]));
        }
        lanes(L0 + o_conv, s.q_conv, H * cs);
        lanes(L0 + o_conv + conv_beats, s.k_conv, H * cs);
        lanes(L0 + o_conv + 2 * conv_beats, s.v_conv, H * cs);
    }
    lanes((size_t)c->num_layers * per, wd + final_norm_offset(c), H);
}

/* Stripe placement of recurrent value (row, v): port, beat, lane
 * (c_impl/gdn_model.cpp:850-890). */
inline void stripe_pos(size_t row, uint32_t v, uint32_t &port, size_t &beat, uint32_t &lane) {
    const uint32_t high = v >> 7, pair = (v >> 6) & 1u, sub = (v >> 5) & 1u, island = (v >> 4) & 1u, l = v & 15u;
    port = (high << 1) | island;
    beat = row * 2 + pair;
    lane = sub * 16 + l;
}

}  // namespace

/* Inverse forms for the engine's state sync (gdn_host.cu). */
namespace gdn {
namespace abi {
size_t shard_beats(const GDNWeightHeader *c);
void gather_recurrent_state(Beat512 *const stripes[], float *rec, size_t floats) {
    parallel_for(floats / kDV, [&](size_t r0, size_t r1) {
        for (size_t row = r0; row < r1; ++row)
            for (uint32_t v = 0; v < kDV; ++v) {
                uint32_t port, lane;
                size_t beat;
                stripe_pos(row, v, port, beat, lane);
                rec[row * kDV + v] = u2f((uint32_t)get_bf16(stripes[port][beat], lane) << 16);
            }
    });
}
void unpack_conv_tails(const Beat512 *head, float *conv, size_t floats) {
    for (size_t stripe = 0; stripe < kConvStripes; ++stripe)
        for (size_t i = 0; i < kConvFloatsPerStripe && stripe * kConvFloatsPerStripe + i < floats; ++i)
            conv[stripe * kConvFloatsPerStripe + i] =
                u2f((uint32_t)get_bf16(head[stripe * (kConvFloatsPerStripe / 16) + i / 32], (uint32_t)(i % 32)) << 16);
}
/* FP32 -> BF16 nearest even; NaN becomes the canonical 0x7fc0 / 0xffc0, Inf
 * is kept (fp32_to_bf16_rne, c_impl/gdn_model.cpp:314-325) */
inline uint16_t rne(float v) {
    const uint32_t b = f2u(v), mag = b & 0x7fffffffu;
    if (mag >= 0x7f800000u) {
        if (mag == 0x7f800000u) return (uint16_t)(b >> 16);
        return (uint16_t)((b & 0x80000000u) ? 0xffc0u : 0x7fc0u);
    }
    return (uint16_t)((b + 0x7fffu + ((b >> 16) & 1u)) >> 16);
}
void store_recurrent_state(Beat512 *const stripes[], const float *rec, size_t floats) {
    parallel_for(floats / kDV, [&](size_t r0, size_t r1) {
        for (size_t row = r0; row < r1; ++row)
            for (uint32_t v = 0; v < kDV; ++v) {
                uint32_t port, lane;
                size_t beat;
                stripe_pos(row, v, port, beat, lane);
                set_bf16(stripes[port][beat], lane, rne(rec[row * kDV + v]));
            }
    });
}
void store_conv_tails(Beat512 *head, const float *conv, size_t floats) {
    memset(head, 0, (GDN_WSF_HEADBUF / 16u) * sizeof(Beat512));
    for (size_t stripe = 0; stripe < kConvStripes; ++stripe)
        for (size_t i = 0; i < kConvFloatsPerStripe && stripe * kConvFloatsPerStripe + i < floats; ++i)
            set_bf16(head[stripe * (kConvFloatsPerStripe / 16) + i / 32], (uint32_t)(i % 32),
                     rne(conv[stripe * kConvFloatsPerStripe + i]));
}
}  // namespace abi
}  // namespace gdn

extern "C" {

/* c_impl/gdn_model.cpp:674-688 */
size_t gdn_weight_shard_beats(const GDNWeightHeader *c) {
    const size_t H = c->hidden_size, I = c->intermediate_size, V = c->vocab_size, CH = GEMV_CHANNELS;
    const size_t per_layer = 5 * (H / CH) * (H / 32) + 2 * (I / CH) * (H / 32) + (H / CH) * (I / 32);
    return (size_t)c->num_layers * per_layer + (V / CH) * (H / 32);
}
size_t gdn_weight_shard_bytes(const GDNWeightHeader *c) { return gdn_weight_shard_beats(c) * sizeof(Beat512); }

/* c_impl/gdn_model.cpp:595-609 */
int gdn_validate_bf16_exact_weights(const float *wd, const GDNWeightHeader *c) {
    const size_t n = total_floats(c);
    for (size_t i = 0; i < n; ++i)
        if (f2u(wd[i]) & 0xffffu) {
            fprintf(stderr, "gdn: weight %zu is not BF16-exact (bits=0x%08x)\n", i, f2u(wd[i]));
            return -1;
        }
    return 0;
}

/* c_impl/gdn_model.cpp:690-759 */
void gdn_build_weight_shards(const float *wd, const GDNWeightHeader *c, Beat512 *const shards[]) {
    std::vector<std::pair<size_t, std::pair<size_t, RowBlock>>> blocks;
    walk_shards(wd, c, [&](size_t ch, size_t off, const RowBlock &b) { blocks.push_back({ch, {off, b}}); });
    parallel_for(blocks.size(), [&](size_t lo, size_t hi) {
        for (size_t i = lo; i < hi; ++i) {
            Beat512 *dst = shards[blocks[i].first] + blocks[i].second.first;
            const RowBlock &b = blocks[i].second.second;
            for (size_t j = 0; j < b.beats(); ++j) dst[j] = b.beat(j);
        }
    });
}

/* c_impl/gdn_model.cpp:761-848 */
int gdn_validate_weight_shards(const float *wd, const GDNWeightHeader *c, Beat512 *const shards[]) {
    const size_t H = c->hidden_size, I = c->intermediate_size, nh = c->num_heads, hd = c->head_dim;
    if (H != nh * hd || H % 32 || I % 32 || (4 * hd) % GEMV_CHANNELS || GEMV_CHANNELS % 4) {
        fprintf(stderr, "gdn: packed BF16 shard geometry is incompatible with the model\n");
        return -1;
    }
    for (int ch = 0; ch < GEMV_CHANNELS; ++ch)
        if (shards[ch] == nullptr) {
            fprintf(stderr, "gdn: run state has no host shard image (enable gdn_b200_set_abi_compat)\n");
            return -1;
        }
    std::vector<std::pair<size_t, std::pair<size_t, RowBlock>>> blocks;
    walk_shards(wd, c, [&](size_t ch, size_t off, const RowBlock &b) { blocks.push_back({ch, {off, b}}); });
    std::atomic<int> bad{0};
    parallel_for(blocks.size(), [&](size_t lo, size_t hi) {
        for (size_t i = lo; i < hi && !bad.load(std::memory_order_relaxed); ++i) {
            const size_t ch = blocks[i].first, off = blocks[i].second.first;
            const RowBlock &b = blocks[i].second.second;
            for (size_t j = 0; j < b.beats(); ++j) {
                const Beat512 e = b.beat(j);
                if (memcmp(&e, shards[ch] + off + j, sizeof(Beat512)) != 0) {
                    if (bad.exchange(1) == 0)
                        fprintf(stderr, "gdn: packed shard mismatch channel=%zu beat=%zu\n", ch, off + j);
                    break;
                }
            }
        }
    });
    return bad.load() ? -1 : 0;
}

/* c_impl/gdn_model.cpp:937-940 */
size_t gdn_aux_image_beats(const GDNWeightHeader *c) {
    return (size_t)c->num_layers * aux_layer_beats(c) + c->hidden_size / 32;
}

/* c_impl/gdn_model.cpp:975-1027 */
void gdn_build_aux_image(const float *wd, const GDNWeightHeader *c, Beat512 *image) {
    memset(image, 0, gdn_aux_image_beats(c) * sizeof(Beat512));
    walk_aux(wd, c, [&](size_t beat, uint32_t lane, int kind, uint32_t bits) {
        if (kind == 0) set_bf16(image[beat], lane, (uint16_t)(bits >> 16));
        else set_fp32(image[beat], lane, bits);
    });
}

/* c_impl/gdn_model.cpp:1029-1080 */
int gdn_validate_aux_image(const Beat512 *image, const float *wd, const GDNWeightHeader *c) {
    if (c->hidden_size % 32 || c->head_dim % 32 || (c->hidden_size * c->conv_size) % 32 || 2 * c->num_heads > 16) {
        fprintf(stderr, "gdn: aux image layout incompatible with the model\n");
        return -1;
    }
    int bad = 0;
    walk_aux(wd, c, [&](size_t beat, uint32_t lane, int kind, uint32_t bits) {
        if (bad) return;
        const bool ok = kind == 0 ? ((bits & 0xffffu) == 0 && get_bf16(image[beat], lane) == (uint16_t)(bits >> 16))
                                  : get_fp32(image[beat], lane) == bits;
        if (!ok) {
            fprintf(stderr, "gdn: aux image mismatch beat=%zu lane=%u\n", beat, lane);
            bad = 1;
        }
    });
    return bad ? -1 : 0;
}

/* c_impl/gdn_model.cpp:850-890: value v of 256-value row r goes to port
 * (v / 128) * 2 + (v / 16) % 2, beat 2r + (v / 64) % 2, lane ((v / 32) % 2) * 16
 * + v % 16; every value must be BF16-exact. */
int gdn_scatter_recurrent_state(Beat512 *const stripes[], const float *rec, size_t floats) {
    if (floats % kDV) {
        fprintf(stderr, "gdn: recurrent state is not a whole 256-value row\n");
        return -1;
    }
    for (size_t i = 0; i < floats; ++i)
        if (f2u(rec[i]) & 0xffffu) {
            fprintf(stderr, "gdn: recurrent state %zu is not BF16-exact (bits=0x%08x)\n", i, f2u(rec[i]));
            return -1;
        }
    parallel_for(floats / kDV, [&](size_t r0, size_t r1) {
        for (size_t row = r0; row < r1; ++row)
            for (uint32_t v = 0; v < kDV; ++v) {
                uint32_t port, lane;
                size_t beat;
                stripe_pos(row, v, port, beat, lane);
                set_bf16(stripes[port][beat], lane, bf16_of(rec[row * kDV + v]));
            }
    });
    gdn::host_note_state_write(stripes[0]);
    return 0;
}

/* c_impl/gdn_model.cpp:892-935: per layer/kind stripe of (conv-1) x hidden
 * values, BF16 lanes in the first half of the stripe's FP32-sized reservation. */
int gdn_pack_conv_tails_bf16(Beat512 *head, const float *conv, size_t floats) {
    if (floats != GDN_WSF_HEADBUF) {
        fprintf(stderr, "gdn: convolution-tail size does not match workspace ABI\n");
        return -1;
    }
    for (size_t i = 0; i < floats; ++i)
        if (f2u(conv[i]) & 0xffffu) {
            fprintf(stderr, "gdn: convolution tail %zu is not BF16-exact (bits=0x%08x)\n", i, f2u(conv[i]));
            return -1;
        }
    memset(head, 0, (GDN_WSF_HEADBUF / 16u) * sizeof(Beat512));
    for (size_t stripe = 0; stripe < kConvStripes; ++stripe)
        for (size_t i = 0; i < kConvFloatsPerStripe; ++i)
            set_bf16(head[stripe * (kConvFloatsPerStripe / 16) + i / 32], (uint32_t)(i % 32),
                     bf16_of(conv[stripe * kConvFloatsPerStripe + i]));
    gdn::host_note_state_write(head);
    return 0;
}

/* c_impl/gdn_model.cpp:338-366 */
uint16_t gdn_test_fp32_to_bf16_rne_bits(uint32_t bits) { return gdn::abi::rne(u2f(bits)); }
uint32_t gdn_test_bf16_to_fp32_bits(uint16_t bits) { return (uint32_t)bits << 16; }
void gdn_test_set_fp32_lane_bits(Beat512 *beat, uint32_t lane, uint32_t bits) { set_fp32(*beat, lane, bits); }
uint32_t gdn_test_get_fp32_lane_bits(const Beat512 *beat, uint32_t lane) { return get_fp32(*beat, lane); }
void gdn_test_set_bf16_lane_bits(Beat512 *beat, uint32_t lane, uint16_t bits) { set_bf16(*beat, lane, bits); }
uint16_t gdn_test_get_bf16_lane_bits(const Beat512 *beat, uint32_t lane) { return get_bf16(*beat, lane); }

}  // extern "C"

namespace gdn {
namespace abi {
size_t shard_beats(const GDNWeightHeader *c) { return gdn_weight_shard_beats(c); }
}  // namespace abi
}  // namespace gdn
