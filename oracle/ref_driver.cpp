/* gdn_ref_driver -- runs the REFERENCE decode model (c_impl/gdn_model.cpp,
 * compiled natively through oracle/hls_shim) on seeded synthetic inputs.
 *
 * TEST INFRASTRUCTURE ONLY. Two uses:
 *   1. golden generation: per-step logits, argmax and final hidden vector,
 *      plus the post-run recurrent/conv state, written to a binary file that
 *      tests/golden/make_golden.py digests into committed fixtures;
 *   2. the CPU baseline of bench.py --impl reference: the reference's own
 *      gdn_decode_step_host timed per token with CLOCK_MONOTONIC, as
 *      c_impl/gdn_eval.cpp:182-186, 337, 435 does.
 *
 * The flow mirrors c_impl/gdn_eval.cpp: gdn_model_load (here from an
 * in-memory file, memfd), gdn_run_state_init, state upload through
 * gdn_scatter_recurrent_state / gdn_pack_conv_tails_bf16 (gdn_eval.cpp:
 * 202-267), then gdn_decode_step_host per token with the native debug
 * buffers capturing the final hidden vector and the logits
 * (gdn_eval.cpp:336-399). The model shape is the reference's compiled one
 * (GDN-1.3B); weights come from gateddeltanet_b200/csrc/gdn_synth.h.
 */
#include "gdn_model.h"

#include "../gateddeltanet_b200/csrc/gdn_synth.h"
#include "gdn_oracle.h"

#include <sys/mman.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <ctime>
#include <string>
#include <vector>

static const size_t GDN_DV_CONST = 256; /* value dim of the compiled shape */

static double monotonic_ms() {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (double)ts.tv_sec * 1000.0 + (double)ts.tv_nsec / 1.0e6;
}

static void die(const char *msg) {
    std::fprintf(stderr, "gdn_ref_driver: %s\n", msg);
    std::exit(1);
}

static uint16_t bf16_lane(const Beat512 &beat, uint32_t lane) {
    uint16_t v;
    std::memcpy(&v, reinterpret_cast<const unsigned char *>(&beat) + 2 * lane, 2);
    return v;
}

static float bf16_to_f(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

/* Known-answer grids over the reference's own primitives, written raw:
 *   RNE set A: x = i * 65521 (mod 2^32), i < 65536
 *   RNE set B: x = (h << 16) | l, h < 65536, l in {0, 0x7fff, 0x8000, 0x8001, 0xffff}
 *   product grid: every BF16 weight pattern (65536) x the 32 activations below
 * through gdn_test_fp32_to_bf16_rne_bits and gdn_native_bf16_mul_to_fp32
 * (c_impl/gdn_model.cpp:314-325, 392-466). tests/test_oracle_golden.py
 * rebuilds the same grids. */
static const uint16_t kGridActivations[32] = {
    0x0000, 0x8000, 0x0001, 0x807f, 0x0080, 0x8080, 0x3f80, 0xbf80, 0x7f80, 0xff80, 0x7fc0,
    0x7f81, 0x7f7f, 0xff7f, 0x3f81, 0x4000, 0x00ff, 0x3e4c, 0xc2f7, 0x1f00, 0x2000, 0x2080,
    0x5f00, 0x6000, 0x0100, 0x3c00, 0x3b80, 0x1c3f, 0x23a1, 0x9e77, 0x4b19, 0xd0e3};

static int dump_primitives(const char *path) {
    FILE *f = std::fopen(path, "wb");
    if (f == nullptr) die("cannot open primitives output");
    std::vector<uint16_t> rne;
    for (uint32_t i = 0; i < 65536u; ++i) rne.push_back(gdn_test_fp32_to_bf16_rne_bits(i * 65521u));
    const uint32_t lows[5] = {0x0000u, 0x7fffu, 0x8000u, 0x8001u, 0xffffu};
    for (uint32_t h = 0; h < 65536u; ++h)
        for (uint32_t k = 0; k < 5; ++k) rne.push_back(gdn_test_fp32_to_bf16_rne_bits((h << 16) | lows[k]));
    std::vector<uint32_t> prod;
    prod.reserve(65536u * 32u);
    for (uint32_t j = 0; j < 32; ++j)
        for (uint32_t w = 0; w < 65536u; ++w) {
            const float v = gdn_native_bf16_mul_to_fp32(Bf16Bits(w), Bf16Bits(kGridActivations[j]));
            uint32_t b;
            std::memcpy(&b, &v, 4);
            prod.push_back(b);
        }
    std::fwrite("GDNPRIM1", 1, 8, f);
    const uint32_t n[2] = {(uint32_t)rne.size(), (uint32_t)prod.size()};
    std::fwrite(n, 4, 2, f);
    std::fwrite(rne.data(), 2, rne.size(), f);
    std::fwrite(prod.data(), 4, prod.size(), f);
    std::fclose(f);
    return 0;
}

/* The reference's host image helpers on seeded inputs (layout goldens):
 *   the 32 weight shards and the aux image of a small seeded model (the
 *   builders are shape-driven: vocab 4096, hidden 512, 2 layers, 2 heads,
 *   intermediate 1536), the four state stripes of a seeded BF16 state of that
 *   model, and the conv-tail packing of a seeded GDN_WSF_HEADBUF-float array,
 * written raw in that order (c_impl/gdn_model.cpp:674-935, 937-1027).
 * tests/test_abi_layouts_cpu.py rebuilds the same images with
 * libgdn_b200.so's restatement and compares digests. */
static int dump_layouts(const char *path) {
    GdnOracleDims d = {4096, 512, 2, 2, 256, 1536, 4, 1e-6f};
    GDNWeightHeader hdr;
    std::memset(&hdr, 0, sizeof(hdr));
    std::memcpy(hdr.magic, "GDNWv1\0\0", 8);
    hdr.version = 1;
    hdr.vocab_size = d.vocab;
    hdr.hidden_size = d.hidden;
    hdr.num_layers = d.layers;
    hdr.num_heads = d.heads;
    hdr.num_v_heads = d.heads;
    hdr.head_dim = d.head_dim;
    hdr.intermediate_size = d.inter;
    hdr.conv_size = d.conv;
    hdr.max_seq_len = 2048;
    hdr.norm_eps = d.eps;
    std::vector<float> blob(gdn_oracle_weight_floats(&d));
    gdn_oracle_synth_weights(&d, 4321, blob.data(), 8);
    const size_t sb = gdn_weight_shard_beats(&hdr);
    std::vector<Beat512> shard_mem((size_t)GEMV_CHANNELS * sb);
    Beat512 *shards[GEMV_CHANNELS];
    for (int c = 0; c < GEMV_CHANNELS; ++c) shards[c] = shard_mem.data() + (size_t)c * sb;
    gdn_build_weight_shards(blob.data(), &hdr, shards);
    std::vector<Beat512> aux(gdn_aux_image_beats(&hdr));
    gdn_build_aux_image(blob.data(), &hdr, aux.data());
    const size_t rec_floats = (size_t)d.layers * d.heads * 256 * 256;
    std::vector<float> rec(rec_floats);
    for (size_t i = 0; i < rec_floats; ++i) rec[i] = gdn_synth_round_bf16(gdn_synth_normal(77, GDN_SYNTH_STREAM_STATE, i, 0.05));
    const size_t stripe_beats = rec_floats / 256 * 2;
    std::vector<Beat512> stripe_mem(4 * stripe_beats);
    Beat512 *stripes[4];
    for (int p = 0; p < 4; ++p) stripes[p] = stripe_mem.data() + (size_t)p * stripe_beats;
    if (gdn_scatter_recurrent_state(stripes, rec.data(), rec_floats) != 0) die("scatter failed");
    std::vector<float> conv(GDN_WSF_HEADBUF);
    for (size_t i = 0; i < conv.size(); ++i) conv[i] = gdn_synth_round_bf16(gdn_synth_normal(78, GDN_SYNTH_STREAM_STATE + 1, i, 0.5));
    std::vector<Beat512> head(GDN_WSF_HEADBUF / 16);
    if (gdn_pack_conv_tails_bf16(head.data(), conv.data(), conv.size()) != 0) die("conv pack failed");
    FILE *f = std::fopen(path, "wb");
    if (f == nullptr) die("cannot open layouts output");
    std::fwrite("GDNLAYT1", 1, 8, f);
    const uint64_t n[4] = {sb, aux.size(), stripe_beats, head.size()};
    std::fwrite(n, 8, 4, f);
    std::fwrite(shard_mem.data(), sizeof(Beat512), shard_mem.size(), f);
    std::fwrite(aux.data(), sizeof(Beat512), aux.size(), f);
    std::fwrite(stripe_mem.data(), sizeof(Beat512), stripe_mem.size(), f);
    std::fwrite(head.data(), sizeof(Beat512), head.size(), f);
    std::fclose(f);
    return 0;
}

int main(int argc, char **argv) {
    if (argc == 3 && std::string(argv[1]) == "--primitives") return dump_primitives(argv[2]);
    if (argc == 3 && std::string(argv[1]) == "--layouts") return dump_layouts(argv[2]);
    uint64_t seed = 1234;
    uint64_t stream_seed = 99;
    uint32_t stream_id = 0;
    uint32_t steps = 2;
    uint32_t warmup = 0;
    double budget_ms = 0.0;   /* >0: stop timing after this much wall time */
    uint64_t state_seed = 0;  /* 0: zero initial state */
    int greedy = 0;
    int partitioned = 0;
    int threads = 8;
    const char *out_path = nullptr;
    for (int i = 1; i < argc; ++i) {
        std::string a = argv[i];
        auto next = [&]() -> const char * {
            if (i + 1 >= argc) die("missing value");
            return argv[++i];
        };
        if (a == "--seed") seed = std::strtoull(next(), nullptr, 10);
        else if (a == "--stream-seed") stream_seed = std::strtoull(next(), nullptr, 10);
        else if (a == "--stream") stream_id = (uint32_t)std::strtoul(next(), nullptr, 10);
        else if (a == "--steps") steps = (uint32_t)std::strtoul(next(), nullptr, 10);
        else if (a == "--warmup") warmup = (uint32_t)std::strtoul(next(), nullptr, 10);
        else if (a == "--budget-ms") budget_ms = std::atof(next());
        else if (a == "--state-seed") state_seed = std::strtoull(next(), nullptr, 10);
        else if (a == "--greedy") greedy = 1;
        else if (a == "--partitioned") partitioned = 1;
        else if (a == "--threads") threads = std::atoi(next());
        else if (a == "--out") out_path = next();
        else die(("unknown argument " + a).c_str());
    }

    /* The compiled reference shape (c_impl/gdn_model.cpp:133-155). */
    GdnOracleDims d = {32000, 2048, 24, 8, 256, 5632, 4, 1e-6f};
    GDNWeightHeader hdr;
    std::memset(&hdr, 0, sizeof(hdr));
    std::memcpy(hdr.magic, "GDNWv1\0\0", 8);
    hdr.version = 1;
    hdr.vocab_size = d.vocab;
    hdr.hidden_size = d.hidden;
    hdr.num_layers = d.layers;
    hdr.num_heads = d.heads;
    hdr.num_v_heads = d.heads;
    hdr.head_dim = d.head_dim;
    hdr.intermediate_size = d.inter;
    hdr.conv_size = d.conv;
    hdr.max_seq_len = 2048;
    hdr.bos_token_id = 1;
    hdr.eos_token_id = 2;
    hdr.norm_eps = d.eps;

    double t_gen = monotonic_ms();
    const size_t nfloats = gdn_oracle_weight_floats(&d);
    std::vector<float> blob(nfloats);
    gdn_oracle_synth_weights(&d, seed, blob.data(), threads);
    int fd = memfd_create("gdnw", 0);
    if (fd < 0) die("memfd_create failed");
    if (write(fd, &hdr, sizeof(hdr)) != (ssize_t)sizeof(hdr)) die("header write failed");
    {
        const char *p = reinterpret_cast<const char *>(blob.data());
        size_t left = nfloats * sizeof(float);
        while (left > 0) {
            const size_t chunk = left < ((size_t)1 << 30) ? left : ((size_t)1 << 30);
            const ssize_t w = write(fd, p, chunk);
            if (w <= 0) die("blob write failed");
            p += w;
            left -= (size_t)w;
        }
    }
    std::vector<float>().swap(blob);
    char path[64];
    std::snprintf(path, sizeof(path), "/proc/self/fd/%d", fd);
    GDNModel model;
    if (gdn_model_load(&model, path) != 0) die("gdn_model_load failed");
    close(fd);
    GDNRunState st;
    if (gdn_run_state_init(&st, &model, model.config.max_seq_len) != 0) die("run state init failed");
    std::fprintf(stderr, "[ref] model ready in %.1f s\n", (monotonic_ms() - t_gen) / 1000.0);

    /* Initial state: zero, or seeded BF16-exact values (S ~ N(0, 0.05),
     * tails ~ N(0, 0.5)); uploaded exactly as gdn_eval.cpp:226-260 does. */
    const size_t rec_count = gdn_oracle_rec_floats(&d);
    const size_t conv_count = gdn_oracle_conv_floats(&d);
    std::vector<float> rec(rec_count, 0.0f), conv(conv_count, 0.0f);
    if (state_seed != 0) {
        for (size_t i = 0; i < rec_count; ++i)
            rec[i] = gdn_synth_round_bf16(gdn_synth_normal(state_seed, GDN_SYNTH_STREAM_STATE, i, 0.05));
        for (size_t i = 0; i < conv_count; ++i)
            conv[i] = gdn_synth_round_bf16(gdn_synth_normal(state_seed, GDN_SYNTH_STREAM_STATE + 1, i, 0.5));
    }
    std::memcpy(st.recurrent_state, rec.data(), rec_count * sizeof(float));
    Beat512 *stripes[GDN_RECURRENT_STATE_PORTS];
    const size_t shard_beats = gdn_weight_shard_beats(&model.config);
    for (int p = 0; p < GDN_RECURRENT_STATE_PORTS; ++p)
        stripes[p] = st.weight_shards[GDN_RECURRENT_STATE_FIRST_PORT + p] + shard_beats;
    if (gdn_scatter_recurrent_state(stripes, st.recurrent_state, rec_count) != 0) die("scatter failed");
    if (gdn_pack_conv_tails_bf16(reinterpret_cast<Beat512 *>(st.head_buffer), conv.data(), conv_count) != 0)
        die("conv pack failed");

    std::vector<float> hidden(d.hidden), logits(d.vocab);
    gdn_set_native_debug_buffers(hidden.data(), logits.data());

    FILE *out = nullptr;
    if (out_path != nullptr) {
        out = std::fopen(out_path, "wb");
        if (out == nullptr) die("cannot open output");
        const uint32_t h[4] = {steps, d.vocab, d.hidden, 0};
        std::fwrite("GDNREF01", 1, 8, out);
        std::fwrite(h, 4, 4, out);
    }

    int32_t prev = gdn_synth_token(stream_seed, stream_id, 0, d.vocab);
    std::vector<double> times;
    double timed_total = 0.0;
    uint32_t timed_steps = 0;
    const double t_run = monotonic_ms();
    for (uint32_t s = 0; s < warmup + steps; ++s) {
        const int32_t tok = (greedy && s > 0) ? prev : gdn_synth_token(stream_seed, stream_id, s, d.vocab);
        int32_t arg = tok;
        const double t0 = monotonic_ms();
        const int rc = partitioned ? gdn_decode_step_host_partitioned(&model, &st, &arg)
                                   : gdn_decode_step_host(&model, &st, &arg);
        const double ms = monotonic_ms() - t0;
        if (rc != 0) die("decode step failed");
        const float *ws = reinterpret_cast<const float *>(st.workspace);
        const int32_t pick = (int32_t)ws[GDN_WS_OFF_X_NORM];
        prev = pick;
        if (s >= warmup) {
            times.push_back(ms);
            timed_total += ms;
            ++timed_steps;
            if (out != nullptr) {
                std::fwrite(&tok, 4, 1, out);
                std::fwrite(&pick, 4, 1, out);
                std::fwrite(&ms, 8, 1, out);
                std::fwrite(logits.data(), 4, d.vocab, out);
                std::fwrite(hidden.data(), 4, d.hidden, out);
            }
            if (budget_ms > 0.0 && monotonic_ms() - t_run > budget_ms) break;
        }
    }
    if (out != nullptr) {
        /* post-run state back to the .gdnstate layouts (inverse of
         * gdn_scatter_recurrent_state, c_impl/gdn_model.cpp:850-890, and of
         * gdn_pack_conv_tails_bf16, :892-929) */
        const size_t rows = rec_count / GDN_DV_CONST;
        for (size_t row = 0; row < rows; ++row)
            for (uint32_t port = 0; port < 4; ++port)
                for (uint32_t pair = 0; pair < 2; ++pair) {
                    const Beat512 &beat = stripes[port][row * 2 + pair];
                    for (uint32_t sub = 0; sub < 2; ++sub)
                        for (uint32_t lane = 0; lane < 16; ++lane) {
                            const uint32_t v = (port >> 1) * 128u + pair * 64u + sub * 32u + (port & 1u) * 16u + lane;
                            rec[row * GDN_DV_CONST + v] = bf16_to_f(bf16_lane(beat, sub * 16u + lane));
                        }
                }
        const Beat512 *hb = reinterpret_cast<const Beat512 *>(st.head_buffer);
        for (size_t stripe = 0; stripe < GDN_CONV_TAIL_STRIPES; ++stripe)
            for (uint32_t beat = 0; beat < GDN_CONV_TAIL_BF16_BEATS_PER_STRIPE; ++beat)
                for (uint32_t lane = 0; lane < 32; ++lane)
                    conv[stripe * GDN_CONV_TAIL_FLOATS_PER_STRIPE + beat * 32u + lane] =
                        bf16_to_f(bf16_lane(hb[stripe * GDN_CONV_TAIL_RESERVED_BEATS_PER_STRIPE + beat], lane));
        std::fwrite(rec.data(), 4, rec_count, out);
        std::fwrite(conv.data(), 4, conv_count, out);
        /* patch the real step count */
        std::fseek(out, 8, SEEK_SET);
        std::fwrite(&timed_steps, 4, 1, out);
        std::fclose(out);
    }
    std::vector<double> sorted = times;
    std::sort(sorted.begin(), sorted.end());
    const double median = sorted.empty() ? 0.0 : sorted[sorted.size() / 2];
    std::printf("{\"impl\": \"reference-native\", \"steps\": %u, \"mean_ms_per_token\": %.3f, "
                "\"median_ms_per_token\": %.3f, \"threads\": %d}\n",
                timed_steps, timed_steps ? timed_total / timed_steps : 0.0, median,
                partitioned ? 3 : 1);
    gdn_set_native_debug_buffers(nullptr, nullptr);
    gdn_run_state_free(&st);
    gdn_model_free(&model);
    return 0;
}
