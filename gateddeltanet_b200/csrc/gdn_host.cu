/* gdn_host.cu -- the C ABI of libgdn_b200.so (include/gdn_model.h,
 * include/gdn_b200.h): model loading, the shared device weight image, decode
 * streams (run states) and the host-side checks.
 *
 * Reference behaviour kept (c_impl/gdn_model.cpp unless noted):
 *   gdn_model_load          header checks :1082-1100, BF16-exact words :1190-1216
 *   gdn_run_state_init      max_tokens range :1247-1252
 *   gdn_decode_step_host    token range :3900-3905, embedding row -> workspace[X]
 *   token line              workspace[X_NORM] lane 0 = argmax as float :3873-3877
 *   gdn_compute_logits      scalar LM head with BF16 product rounding :3930-3975
 *   .gdnstate               c_impl/gdn_eval.cpp:202-267, c_impl/host.cpp:675-735
 */
#include "gdn_engine.h"
#include "gdn_math.h"
#include "gdn_synth.h"

#include "../../include/gdn_b200.h"
#include "../../include/gdn_model.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

namespace gdn {
namespace abi {
void gather_recurrent_state(Beat512 *const stripes[], float *rec, size_t floats);
void unpack_conv_tails(const Beat512 *head, float *conv, size_t floats);
void store_recurrent_state(Beat512 *const stripes[], const float *rec, size_t floats);
void store_conv_tails(Beat512 *head, const float *conv, size_t floats);
}  // namespace abi
}  // namespace gdn


namespace {

thread_local std::string g_last_error;
thread_local int g_device = 0;

int fail(const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    fprintf(stderr, "%s\n", buf);
    return -1;
}

#define CUDA_OK(call)                                                                        \
    do {                                                                                     \
        cudaError_t e_ = (call);                                                             \
        if (e_ != cudaSuccess) return fail("gdn_b200: %s failed: %s", #call, cudaGetErrorString(e_)); \
    } while (0)

constexpr size_t kHeaderBytes = 60;

static_assert(sizeof(GDNWeightHeader) == kHeaderBytes, "GDNWeightHeader must be 60 bytes");

inline uint32_t f2u(float v) { uint32_t b; memcpy(&b, &v, 4); return b; }
inline float u2f(uint32_t b) { float v; memcpy(&v, &b, 4); return v; }

int hw_threads() {
    unsigned n = std::thread::hardware_concurrency();
    if (n == 0) n = 4;
    return (int)std::min(n, 64u);
}

template <typename F>
void parallel_for(size_t n, F fn) {
    const int t = (int)std::min<size_t>((size_t)hw_threads(), n ? n : 1);
    if (t <= 1) { fn((size_t)0, n); return; }
    std::vector<std::thread> th;
    for (int i = 0; i < t; ++i) {
        const size_t b = n * (size_t)i / (size_t)t, e = n * (size_t)(i + 1) / (size_t)t;
        th.emplace_back([=] { fn(b, e); });
    }
    for (auto &x : th) x.join();
}

/* ------------------------------------------------------- blob geometry */

size_t layer_floats(const GDNWeightHeader &c) {
    const size_t H = c.hidden_size, nh = c.num_heads, hd = c.head_dim, I = c.intermediate_size, cs = c.conv_size;
    return H + 2 * nh + 3 * H * H + 2 * nh * H + 3 * H * cs + H * H + hd + H * H + H + 2 * I * H + H * I;
}
size_t total_floats(const GDNWeightHeader &c) {
    return (size_t)c.vocab_size * c.hidden_size + (size_t)c.num_layers * layer_floats(c) + c.hidden_size +
           (size_t)c.vocab_size * c.hidden_size;
}

/* gdn_validate_config, c_impl/gdn_model.cpp:1082-1100 */
int validate_config(const GDNWeightHeader &c) {
    if (memcmp(c.magic, "GDNWv1", 6) != 0 || c.version != 1) return fail("unsupported weight file");
    if (c.num_heads != c.num_v_heads) return fail("expected num_heads == num_v_heads");
    if (c.hidden_size != c.num_heads * c.head_dim) return fail("expected hidden_size == num_heads * head_dim");
    return 0;
}

/* gdn_assign_weight_views, c_impl/gdn_model.cpp:1102-1159 (same blob order) */
void assign_views(GDNModel *m) {
    const GDNWeightHeader &c = m->config;
    const size_t H = c.hidden_size, nh = c.num_heads, hd = c.head_dim, I = c.intermediate_size, cs = c.conv_size;
    float *p = m->weight_data;
    m->embeddings = p;
    p += (size_t)c.vocab_size * H;
    for (uint32_t l = 0; l < c.num_layers; ++l) {
        GDNLayerWeights *w = &m->layers[l];
        w->attn_norm = p; p += H;
        w->a_log = p; p += nh;
        w->dt_bias = p; p += nh;
        w->q_proj = p; p += H * H;
        w->k_proj = p; p += H * H;
        w->v_proj = p; p += H * H;
        w->a_proj = p; p += nh * H;
        w->b_proj = p; p += nh * H;
        w->q_conv = p; p += H * cs;
        w->k_conv = p; p += H * cs;
        w->v_conv = p; p += H * cs;
        w->g_proj = p; p += H * H;
        w->o_norm = p; p += hd;
        w->o_proj = p; p += H * H;
        w->mlp_norm = p; p += H;
        w->mlp_gate_proj = p; p += I * H;
        w->mlp_up_proj = p; p += I * H;
        w->mlp_down_proj = p; p += H * I;
    }
    m->final_norm = p;
    p += H;
    m->lm_head = p;
}

/* Shape limits of this engine (beyond the reference's own header checks). */
int engine_supports(const GDNWeightHeader &c) {
    const uint32_t H = c.hidden_size, I = c.intermediate_size;
    if (c.head_dim != 256) return fail("gdn_b200: head_dim must be 256 (got %u)", c.head_dim);
    if (c.conv_size != 4) return fail("gdn_b200: conv_size must be 4 (got %u)", c.conv_size);
    if (H % 512 || I % 512 || H == 0 || I == 0) return fail("gdn_b200: hidden and intermediate must be multiples of 512");
    if (c.vocab_size % 16) return fail("gdn_b200: vocab must be a multiple of 16 (the LM head's 16-row tiles)");
    if (c.num_heads > 8 || H > GDN_WSF_HID) return fail("gdn_b200: at most 8 heads (hidden <= 2048)");
    if (I > GDN_WSF_MLP || c.vocab_size > GDN_WSF_LOGITS || c.vocab_size == 0)
        return fail("gdn_b200: intermediate/vocab exceed the workspace ABI");
    if ((size_t)c.num_layers * c.num_heads * 256 * 256 > GDN_WSF_STATE ||
        (size_t)c.num_layers * 3 * 3 * H > GDN_WSF_HEADBUF || c.num_layers == 0)
        return fail("gdn_b200: layer count exceeds the workspace ABI");
    return 0;
}

/* Per-CTA limits of the decode kernel for `ncta` CTAs: every CTA owns units
 * of every phase (so that no CTA can run two phases ahead of one it reads
 * from), at most one O / DOWN row and one state column per consumer warp. */
int engine_grid_ok(const GDNWeightHeader &c, int ncta, bool report = true) {
    const uint32_t H = c.hidden_size, cols = c.num_heads * 256;
    const uint32_t units[] = {4 * H / gdn::kTileRowsQKVG, cols, H, 2 * c.intermediate_size / gdn::kTileRowsGU,
                              c.vocab_size / gdn::kTileRowsLM};
    for (uint32_t u : units)
        if (u < (uint32_t)ncta) return report ? fail("gdn_b200: %d CTAs exceed the %u units of a phase", ncta, u) : -1;
    const uint32_t narrow_rows = std::min<uint32_t>(gdn::kMaxNarrowRows, gdn::kSlotBytes / (gdn::kNarrowGroups * 128));
    if ((H + ncta - 1) / ncta > narrow_rows || (cols + ncta - 1) / ncta > (uint32_t)gdn::kMaxStateCols)
        return report ? fail("gdn_b200: %d CTAs are too few for this model (at most %u O/DOWN rows and %d state "
                             "columns per CTA)", ncta, narrow_rows, gdn::kMaxStateCols)
                      : -1;
    return 0;
}

/* ------------------------------------------------- device weight image */

/* Chunk geometry of a weight image: 64-column groups per chunk of the tiled
 * projections and of the O / DOWN rows (the defaults: the one-GPU image). */
struct ImageGeom {
    uint32_t g_qkvg = gdn::kGroupsQKVG, g_gu = gdn::kGroupsGU, g_lm = gdn::kGroupsLM, ng = gdn::kNarrowGroups;
    bool operator==(const ImageGeom &o) const {
        return g_qkvg == o.g_qkvg && g_gu == o.g_gu && g_lm == o.g_lm && ng == o.ng;
    }
};

struct DeviceModel {
    int device = 0;
    int refs = 0;
    GDNWeightHeader cfg;
    uint8_t *wimg = nullptr;
    size_t layer_stride = 0, off_ab = 0, off_o = 0, off_gu = 0, off_down = 0;
    uint8_t *w_lm = nullptr;
    uint16_t *emb = nullptr;
    float *aux = nullptr;
    size_t aux_stride = 0;
    float *exp_table = nullptr;
    float *decay_tab = nullptr;     /* [L][nh][65536], see gdn_engine.h */
    uint32_t *exp_exc = nullptr;    /* the host library's expf exceptions, device copy */
    uint32_t exp_exc_n = 0;
    float fast_x_min = INFINITY;    /* DecodeParams.fast_x_min */
    uint32_t exp_exc_bf16[gdn::kMaxExcBf16] = {};  /* the BF16-valued entries of exp_exc */
    uint32_t exp_exc_bf16_n = 0;
    bool model_alive = true;
    /* the same weights in the chunk geometries of tensor-parallel grids
     * (built from wimg / w_lm on first use, guarded by g_mu) */
    struct Image {
        ImageGeom g;
        uint8_t *wimg, *w_lm;
    };
    std::vector<Image> images;
};

std::mutex g_mu;
std::map<const float *, DeviceModel *> g_models;  /* keyed by GDNModel.weight_data */

inline uint16_t hi16(float v) { return (uint16_t)(f2u(v) >> 16); }

/* Device image positions -> natural (row, column) of a projection (layouts
 * in gdn_engine.h). Tiled: element i of [K/(64 G) column chunks][T tiles][G
 * groups][TR rows][64]; row-major: element i of [K/512 column chunks][R
 * rows][8 groups][64]. In both, the 16-byte pieces of a 128-byte group are
 * permuted (by the row in tiles, by the group otherwise). */
__host__ __device__ inline void tiled_src(size_t i, size_t TR, size_t G, size_t rows, size_t *row, size_t *col) {
    const size_t T = rows / TR, chunk = T * G * TR * 64;
    const size_t j = i / chunk, rem = i % chunk;
    const size_t t = rem / (G * TR * 64), rem2 = rem % (G * TR * 64);
    const size_t gi = rem2 / (TR * 64), r = (rem2 % (TR * 64)) / 64, c = rem2 % 64;
    *row = t * TR + r;
    *col = (j * G + gi) * 64 + (((c >> 3) ^ (r & 7)) << 3) + (c & 7);
}
/* NG: groups per column chunk (gdn::kNarrowGroups in the one-GPU image) */
__host__ __device__ inline void rowmajor_src(size_t i, size_t rows, size_t K, size_t NG, size_t *row, size_t *col) {
    const size_t groups = K / 64;
    const size_t j = i / (rows * NG * 64), rem = i - j * rows * NG * 64;
    const size_t ng = groups - j * NG < NG ? groups - j * NG : NG;
    const size_t cc = rem % (ng * 64), g = j * NG + cc / 64, c = cc % 64;
    *row = rem / (ng * 64);
    *col = g * 64 + (((c >> 3) ^ (g & 7)) << 3) + (c & 7);
}
/* The inverses: image position of natural (row, col). */
__host__ __device__ inline size_t tiled_pos(size_t row, size_t col, size_t TR, size_t G, size_t rows) {
    const size_t T = rows / TR, t = row / TR, r = row % TR, gg = col / 64, j = gg / G, gi = gg % G, ci = col % 64;
    const size_t c = (((ci >> 3) ^ (r & 7)) << 3) | (ci & 7);
    return ((j * T + t) * G + gi) * TR * 64 + r * 64 + c;
}
__host__ __device__ inline size_t rowmajor_pos(size_t row, size_t col, size_t rows, size_t K, size_t NG) {
    const size_t groups = K / 64, g = col / 64, j = g / NG, ci = col % 64;
    const size_t ng = groups - j * NG < NG ? groups - j * NG : NG;
    const size_t c = (((ci >> 3) ^ (g & 7)) << 3) | (ci & 7);
    return j * rows * NG * 64 + row * ng * 64 + (g - j * NG) * 64 + c;
}

/* The geometry for `ncta` CTAs (all GPUs of a tensor-parallel launch): the
 * fewest chunks per phase whose largest copy still fits a ring slot. A
 * tiled projection of T tiles gives a CTA at most ceil(T / ncta) tiles (at
 * most kPassTiles of them per pass), an O / DOWN row set ceil(H / ncta)
 * rows. */
ImageGeom image_geometry(const GDNWeightHeader &c, uint32_t ncta) {
    const uint32_t H = c.hidden_size, I = c.intermediate_size;
    auto wide = [&](uint32_t T, uint32_t TR) {
        const uint32_t n = std::min(gdn::kPassTiles, (T + ncta - 1) / ncta);
        uint32_t G = 1;
        while ((H / 64) % (2 * G) == 0 && n * 2 * G * TR * 128 <= (uint32_t)gdn::kSlotBytes) G *= 2;
        return G;
    };
    ImageGeom g;
    g.g_qkvg = wide(4 * H / gdn::kTileRowsQKVG, gdn::kTileRowsQKVG);
    g.g_gu = wide(2 * I / gdn::kTileRowsGU, gdn::kTileRowsGU);
    g.g_lm = wide(c.vocab_size / gdn::kTileRowsLM, gdn::kTileRowsLM);
    const uint32_t rows = (H + ncta - 1) / ncta;
    g.ng = std::min<uint32_t>((uint32_t)gdn::kSlotBytes / (rows * 128) / 8 * 8, std::max(H, I) / 64);
    return g;
}

/* The reference's scalar functions with the host C library
 * (c_impl/gdn_model.cpp:1307-1330). */
float host_softplus(float x) {
    if (x > 20.0f) return x;
    if (x < -20.0f) return expf(x);
    return log1pf(expf(x));
}

/* Negative floats x in [-104, 0] whose host expf(x) differs from the
 * correctly rounded exp(x) (taken as the double-precision exp rounded to
 * float), in increasing bit order; computed once per process. */
const std::vector<uint32_t> &host_exp_exceptions() {
    static std::once_flag once;
    static std::vector<uint32_t> exc;
    std::call_once(once, [] {
        const uint64_t lo = 0x80000000ull, hi = 0xC2D00001ull; /* -0 .. -104 */
        const int nt = hw_threads();
        std::vector<std::vector<uint32_t>> part(nt);
        std::vector<std::thread> th;
        for (int k = 0; k < nt; ++k)
            th.emplace_back([&, k] {
                const uint64_t b = lo + (hi - lo) * k / nt, e = lo + (hi - lo) * (k + 1) / nt;
                for (uint64_t u = b; u < e; ++u) {
                    const float x = u2f((uint32_t)u);
                    const float g = expf(x), c = (float)exp((double)x);
                    if (f2u(g) != f2u(c)) part[k].push_back((uint32_t)u);
                }
            });
        for (auto &x : th) x.join();
        for (auto &v : part) exc.insert(exc.end(), v.begin(), v.end());
    });
    return exc;
}

void free_device_model(DeviceModel *dm) {
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(dm->device);
    cudaFree(dm->wimg);
    cudaFree(dm->w_lm);
    for (auto &im : dm->images) {
        cudaFree(im.wimg);
        cudaFree(im.w_lm);
    }
    cudaFree(dm->emb);
    cudaFree(dm->aux);
    cudaFree(dm->exp_table);
    cudaFree(dm->decay_tab);
    cudaFree(dm->exp_exc);
    cudaSetDevice(prev);
    delete dm;
}

/* Upload n BF16 values produced by fill(dst, begin, end) through a pinned
 * staging buffer. */
template <typename F>
int upload_bf16(uint16_t *dst, size_t n, F fill) {
    const size_t chunk = (size_t)64 << 20;  /* values per staging pass */
    uint16_t *stage = nullptr;
    CUDA_OK(cudaMallocHost(&stage, std::min(n, chunk) * 2));
    for (size_t b = 0; b < n; b += chunk) {
        const size_t e = std::min(n, b + chunk);
        parallel_for(e - b, [&](size_t lo, size_t hi) { fill(stage, b + lo, b + hi, lo); });
        const cudaError_t err = cudaMemcpy(dst + b, stage, (e - b) * 2, cudaMemcpyHostToDevice);
        if (err != cudaSuccess) {
            cudaFreeHost(stage);
            return fail("gdn_b200: weight upload failed: %s", cudaGetErrorString(err));
        }
    }
    cudaFreeHost(stage);
    return 0;
}

/* Smallest nonzero weight magnitude of the rounded-product GEMVs, and whether
 * any of their weights is subnormal or not finite. */
void gemv_weight_range(const GDNModel *model, float *wmin, bool *bad) {
    const GDNWeightHeader &c = model->config;
    const size_t H = c.hidden_size, I = c.intermediate_size;
    std::vector<std::pair<const float *, size_t>> spans;
    for (uint32_t l = 0; l < c.num_layers; ++l) {
        const GDNLayerWeights &w = model->layers[l];
        for (const float *pp : {w.q_proj, w.k_proj, w.v_proj, w.g_proj, w.o_proj}) spans.push_back({pp, H * H});
        for (const float *pp : {w.mlp_gate_proj, w.mlp_up_proj, w.mlp_down_proj}) spans.push_back({pp, I * H});
    }
    spans.push_back({model->lm_head, (size_t)c.vocab_size * H});
    std::mutex mu;
    float best = INFINITY;
    bool any_bad = false;
    for (auto &sp : spans) {
        parallel_for(sp.second, [&](size_t b, size_t e) {
            float m = INFINITY;
            bool bd = false;
            for (size_t i = b; i < e; ++i) {
                const uint32_t u = f2u(sp.first[i]) & 0x7fffffffu;
                if (u == 0) continue;
                if (u < 0x00800000u || u >= 0x7f800000u) bd = true;
                else m = std::min(m, u2f(u));
            }
            std::lock_guard<std::mutex> lock(mu);
            best = std::min(best, m);
            any_bad = any_bad || bd;
        });
    }
    *wmin = best;
    *bad = any_bad;
}

DeviceModel *build_device_model(const GDNModel *model) {
    const GDNWeightHeader &c = model->config;
    const size_t H = c.hidden_size, nh = c.num_heads, I = c.intermediate_size, V = c.vocab_size, L = c.num_layers;
    DeviceModel *dm = new DeviceModel();
    dm->cfg = c;
    dm->device = g_device;
    const size_t rows_a = 4 * H;
    dm->off_ab = rows_a * H * 2;
    dm->off_o = dm->off_ab + 2 * nh * H * 2;
    dm->off_gu = dm->off_o + H * H * 2;
    dm->off_down = dm->off_gu + 2 * I * H * 2;
    dm->layer_stride = ((dm->off_down + H * I * 2) + 255) & ~(size_t)255;
    dm->aux_stride = (14 * H + 256 + 2 * nh + 3) & ~(size_t)3;
    const size_t decay_n = L * nh * 65536;
    if (cudaMalloc(&dm->wimg, dm->layer_stride * L) != cudaSuccess || cudaMalloc(&dm->w_lm, V * H * 2) != cudaSuccess ||
        cudaMalloc(&dm->emb, V * H * 2) != cudaSuccess ||
        cudaMalloc(&dm->aux, (dm->aux_stride * L + H) * sizeof(float)) != cudaSuccess ||
        cudaMalloc(&dm->decay_tab, decay_n * sizeof(float)) != cudaSuccess) {
        fail("gdn_b200: device weight image allocation failed (%.2f GB)",
             (double)(dm->layer_stride * L + 2 * V * H * 2) / 1e9);
        free_device_model(dm);
        return nullptr;
    }
    /* per layer: QKVG (8-row tiles), AB, O (row-major), GU (16-row tiles),
     * DOWN (row-major), as one contiguous range */
    for (size_t l = 0; l < L; ++l) {
        const GDNLayerWeights &w = model->layers[l];
        uint16_t *base = reinterpret_cast<uint16_t *>(dm->wimg + l * dm->layer_stride);
        const size_t n = dm->off_down / 2 + H * I;
        const int rc = upload_bf16(base, n, [&](uint16_t *st, size_t b, size_t e, size_t so) {
            for (size_t i = b; i < e; ++i) {
                size_t r, col;
                const float *src;
                if (i < dm->off_ab / 2) {
                    tiled_src(i, gdn::kTileRowsQKVG, gdn::kGroupsQKVG, 4 * H, &r, &col);
                    const float *m = r < H ? w.q_proj : r < 2 * H ? w.k_proj : r < 3 * H ? w.v_proj : w.g_proj;
                    src = m + (r % H) * H + col;
                } else if (i < dm->off_o / 2) {
                    const size_t j = i - dm->off_ab / 2;
                    r = j / H;
                    src = ((r & 1) ? w.b_proj : w.a_proj) + (r >> 1) * H + j % H;
                } else if (i < dm->off_gu / 2) {
                    rowmajor_src(i - dm->off_o / 2, H, H, gdn::kNarrowGroups, &r, &col);
                    src = w.o_proj + r * H + col;
                } else if (i < dm->off_down / 2) {
                    tiled_src(i - dm->off_gu / 2, gdn::kTileRowsGU, gdn::kGroupsGU, 2 * I, &r, &col);
                    src = ((r & 1) ? w.mlp_up_proj : w.mlp_gate_proj) + (r >> 1) * H + col;
                } else {
                    rowmajor_src(i - dm->off_down / 2, H, I, gdn::kNarrowGroups, &r, &col);
                    src = w.mlp_down_proj + r * I + col;
                }
                st[so + (i - b)] = hi16(*src);
            }
        });
        if (rc != 0) { free_device_model(dm); return nullptr; }
    }
    if (upload_bf16(reinterpret_cast<uint16_t *>(dm->w_lm), V * H,
                    [&](uint16_t *st, size_t b, size_t e, size_t so) {
                        for (size_t i = b; i < e; ++i) {
                            size_t r, col;
                            tiled_src(i, gdn::kTileRowsLM, gdn::kGroupsLM, V, &r, &col);
                            st[so + (i - b)] = hi16(model->lm_head[r * H + col]);
                        }
                    }) != 0 ||
        upload_bf16(dm->emb, V * H, [&](uint16_t *st, size_t b, size_t e, size_t so) {
            for (size_t i = b; i < e; ++i) st[so + (i - b)] = hi16(model->embeddings[i]);
        }) != 0) {
        free_device_model(dm);
        return nullptr;
    }
    /* aux (FP32): attn_norm | o_norm | mlp_norm | conv_w[3][H][4] | a_log | dt_bias, then final_norm */
    std::vector<float> aux(dm->aux_stride * L + H, 0.0f);
    for (size_t l = 0; l < L; ++l) {
        const GDNLayerWeights &w = model->layers[l];
        float *a = aux.data() + l * dm->aux_stride;
        memcpy(a, w.attn_norm, H * 4);
        memcpy(a + H, w.o_norm, 256 * 4);
        memcpy(a + H + 256, w.mlp_norm, H * 4);
        memcpy(a + 2 * H + 256, w.q_conv, H * 4 * 4);
        memcpy(a + 6 * H + 256, w.k_conv, H * 4 * 4);
        memcpy(a + 10 * H + 256, w.v_conv, H * 4 * 4);
        memcpy(a + 14 * H + 256, w.a_log, nh * 4);
        memcpy(a + 14 * H + 256 + nh, w.dt_bias, nh * 4);
    }
    memcpy(aux.data() + dm->aux_stride * L, model->final_norm, H * 4);
    /* decay = exp(-exp(a_log) * softplus(a + dt_bias)) for every BF16 a, with
     * the host library, in the reference's operation order
     * (c_impl/gdn_model.cpp:2101-2105) */
    std::vector<float> decay(decay_n);
    parallel_for(L * nh, [&](size_t b, size_t e) {
        for (size_t lh = b; lh < e; ++lh) {
            const GDNLayerWeights &w = model->layers[lh / nh];
            const float alog = w.a_log[lh % nh], dtb = w.dt_bias[lh % nh];
            const float ea = expf(alog);
            for (uint32_t bits = 0; bits < 65536u; ++bits) {
                const float a = u2f(bits << 16);
                const float decay_in = a + dtb;
                const float decay_val = -ea * host_softplus(decay_in);
                decay[lh * 65536 + bits] = expf(decay_val);
            }
        }
    });
    const std::vector<uint32_t> &exc = host_exp_exceptions();
    dm->exp_exc_n = (uint32_t)exc.size();
    for (uint32_t u : exc) {
        if ((u & 0xffffu) != 0) continue;
        if (dm->exp_exc_bf16_n == (uint32_t)gdn::kMaxExcBf16) {
            fail("gdn_b200: the host library's exp has more than %d exceptions at BF16 inputs", gdn::kMaxExcBf16);
            free_device_model(dm);
            return nullptr;
        }
        dm->exp_exc_bf16[dm->exp_exc_bf16_n++] = u;
    }
    float wmin = INFINITY;
    bool wbad = false;
    gemv_weight_range(model, &wmin, &wbad);
    dm->fast_x_min = (wbad || !(wmin > 0.0f)) ? INFINITY : (float)(ldexp(1.0, -126) / (double)wmin * (1.0 + 1e-6));
    float table[128];
    gdn_exp_table_fill(table);
    if (cudaMemcpy(dm->aux, aux.data(), aux.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(dm->decay_tab, decay.data(), decay_n * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMalloc(&dm->exp_exc, std::max<size_t>(exc.size(), 1) * 4) != cudaSuccess ||
        (exc.size() && cudaMemcpy(dm->exp_exc, exc.data(), exc.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess) ||
        cudaMalloc(&dm->exp_table, sizeof(table)) != cudaSuccess ||
        cudaMemcpy(dm->exp_table, table, sizeof(table), cudaMemcpyHostToDevice) != cudaSuccess) {
        fail("gdn_b200: aux upload failed");
        free_device_model(dm);
        return nullptr;
    }
    return dm;
}

/* Piece i (8 BF16 values, consecutive columns in every geometry) of a
 * projection in groups-per-chunk `gd`, gathered from its copy in `gs`;
 * kind 0 tiled (TR-row tiles), 1 row-major O / DOWN rows. */
__global__ void reimage_kernel(uint4 *dst, const uint4 *src, size_t pieces, int kind, uint32_t TR, uint32_t gs,
                               uint32_t gd, size_t rows, size_t K) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < pieces; i += (size_t)gridDim.x * blockDim.x) {
        size_t r, c, j;
        if (kind == 0) {
            tiled_src(i * 8, TR, gd, rows, &r, &c);
            j = tiled_pos(r, c, TR, gs, rows);
        } else {
            rowmajor_src(i * 8, rows, K, gd, &r, &c);
            j = rowmajor_pos(r, c, rows, K, gs);
        }
        dst[i] = src[j / 8];
    }
}

/* The weight image (QKVG ... DOWN of every layer, and the LM head) in
 * geometry g: the one-GPU image itself for the default geometry, else a copy
 * re-laid on the device from it on first use and kept with the model. */
int device_image(DeviceModel *dm, const ImageGeom &g, cudaStream_t st, uint8_t **wimg, uint8_t **w_lm) {
    if (g == ImageGeom()) {
        *wimg = dm->wimg;
        *w_lm = dm->w_lm;
        return 0;
    }
    std::lock_guard<std::mutex> lock(g_mu);
    for (const auto &im : dm->images)
        if (im.g == g) {
            *wimg = im.wimg;
            *w_lm = im.w_lm;
            return 0;
        }
    const GDNWeightHeader &c = dm->cfg;
    const size_t H = c.hidden_size, I = c.intermediate_size, V = c.vocab_size, L = c.num_layers;
    DeviceModel::Image im{g, nullptr, nullptr};
    if (cudaMalloc(&im.wimg, dm->layer_stride * L) != cudaSuccess || cudaMalloc(&im.w_lm, V * H * 2) != cudaSuccess) {
        cudaFree(im.wimg);
        return fail("gdn_b200: tensor-parallel weight image allocation failed (%.2f GB)",
                    (double)(dm->layer_stride * L + V * H * 2) / 1e9);
    }
    auto run = [&](uint8_t *dst, const uint8_t *src, size_t elems, int kind, uint32_t TR, uint32_t gs, uint32_t gd,
                   size_t rows, size_t K) {
        reimage_kernel<<<1184, 256, 0, st>>>(reinterpret_cast<uint4 *>(dst), reinterpret_cast<const uint4 *>(src),
                                             elems / 8, kind, TR, gs, gd, rows, K);
    };
    for (size_t l = 0; l < L; ++l) {
        uint8_t *d = im.wimg + l * dm->layer_stride;
        const uint8_t *s0 = dm->wimg + l * dm->layer_stride;
        run(d, s0, 4 * H * H, 0, gdn::kTileRowsQKVG, gdn::kGroupsQKVG, g.g_qkvg, 4 * H, H);
        cudaMemcpyAsync(d + dm->off_ab, s0 + dm->off_ab, dm->off_o - dm->off_ab, cudaMemcpyDeviceToDevice, st);
        run(d + dm->off_o, s0 + dm->off_o, H * H, 1, 0, gdn::kNarrowGroups, g.ng, H, H);
        run(d + dm->off_gu, s0 + dm->off_gu, 2 * I * H, 0, gdn::kTileRowsGU, gdn::kGroupsGU, g.g_gu, 2 * I, H);
        run(d + dm->off_down, s0 + dm->off_down, H * I, 1, 0, gdn::kNarrowGroups, g.ng, H, I);
    }
    run(im.w_lm, dm->w_lm, V * H, 0, gdn::kTileRowsLM, gdn::kGroupsLM, g.g_lm, V, H);
    const cudaError_t e = cudaStreamSynchronize(st);
    const cudaError_t e2 = cudaGetLastError();
    if (e != cudaSuccess || e2 != cudaSuccess) {
        cudaFree(im.wimg);
        cudaFree(im.w_lm);
        return fail("gdn_b200: building the tensor-parallel weight image failed: %s",
                    cudaGetErrorString(e != cudaSuccess ? e : e2));
    }
    dm->images.push_back(im);
    *wimg = im.wimg;
    *w_lm = im.w_lm;
    return 0;
}

/* ------------------------------------------------------- decode streams */

struct Stream {
    DeviceModel *dm = nullptr;
    int device = 0;
    int grid = 0;
    /* numeric contract: the reference's own (c_impl) unless gdn_b200_set_numerics chooses another */
    int bf16_boundary = 1;
    int native_product = 1;
    int bf16_state = 1;
    int force_exact = 0;   /* test hook: exact emulation of the BF16 product in every phase */
    cudaStream_t stream = nullptr;
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;
    float *S = nullptr, *tails = nullptr, *acts = nullptr;
    gdn::xword *xbuf = nullptr;  /* exchange words: qkv | gate | attn | y_o | m | y_down */
    size_t xwords = 0;
    gdn::xword *qkv, *gate, *attn, *y_o, *m, *y_down;
    float *logits, *hidden, *x_embed, *cand_val;
    int32_t *cand_idx = nullptr;
    gdn::DecodeStatus *status = nullptr;
    gdn::DecodeStatus *status_host = nullptr;
    int32_t *tokens = nullptr, *argmax = nullptr;
    size_t tokens_cap = 0;
    uint32_t epoch = 0;   /* exchange tag base of the next launch */
    int test_drop_cta = -1, test_drop_phase = -1;
    float *ws = nullptr;  /* pinned ABI workspace (host) */
    /* reference-ABI compatibility (gdn_b200_set_abi_compat): the host shard and
     * aux images of c_impl/gdn_model.cpp:1247-1294, whose state stripes
     * (shards 28..31 past the weights) and workspace head buffer mirror the
     * device state */
    bool compat = false;
    bool host_dirty = false;
    Beat512 *shards[GEMV_CHANNELS] = {};
    Beat512 *aux = nullptr;
    size_t shard_beats = 0;
    /* tensor-parallel decode (gdn_b200_tp_attach): the peers' exchange
     * regions mapped into this process */
    int tp_world = 1, tp_rank = 0;
    int tp_grid = 0;      /* CTAs per GPU while attached: every phase must keep a unit for each CTA of all GPUs */
    /* the weight image of the attached grid's chunk geometry */
    ImageGeom tp_geom;
    uint8_t *tp_wimg = nullptr, *tp_lm = nullptr;
    /* the state holds one rank's part since a tensor-parallel step (until a
     * full upload); part_* is the attachment that step ran under */
    bool tp_part = false;
    int part_grid = 0, part_rank = 0, part_world = 1;
    void *tp_peer[gdn::kMaxTpRanks] = {};
    unsigned long long *rank_cand = nullptr;
    size_t xbytes = 0;   /* bytes of the exchange region: words, rank candidates, logits */
};

std::map<const void *, Stream *> g_streams;  /* keyed by GDNRunState.workspace */
bool g_abi_compat = false;                   /* gdn_b200_set_abi_compat / GDN_B200_ABI_COMPAT=1 */

float *g_debug_hidden = nullptr;
float *g_debug_logits = nullptr;

Stream *find_stream(GDNRunState *state) {
    std::lock_guard<std::mutex> lock(g_mu);
    auto it = g_streams.find(state ? (const void *)state->workspace : nullptr);
    return it == g_streams.end() ? nullptr : it->second;
}

/* Host [L][h][k][v] / [L][kind][row][H] state <-> the device's storage
 * ([L][h][v][k] columns, FP32 or BF16, pieces permuted; gdn_engine.h) /
 * [L][kind][H][4] tails. The recurrent state passes through a natural FP32
 * [L][h][v][k] device buffer and the layout kernels of gdn_decode.cu. */
int upload_state(Stream &st, const float *rec, const float *conv) {
    Stream *s = &st;
    const GDNWeightHeader &c = s->dm->cfg;
    const size_t L = c.num_layers, nh = c.num_heads, H = c.hidden_size;
    const size_t rec_floats = L * nh * 256 * 256;
    std::vector<float> S(rec_floats), T(L * 3 * H * 4, 0.0f);
    parallel_for(L * nh, [&](size_t b, size_t e) {
        for (size_t lh = b; lh < e; ++lh)
            for (size_t k = 0; k < 256; ++k)
                for (size_t v = 0; v < 256; ++v) S[(lh * 256 + v) * 256 + k] = rec[(lh * 256 + k) * 256 + v];
    });
    for (size_t lk = 0; lk < L * 3; ++lk)
        for (size_t d = 0; d < H; ++d)
            for (size_t r = 0; r < 3; ++r) T[(lk * H + d) * 4 + r] = conv[(lk * 3 + r) * H + d];
    CUDA_OK(cudaSetDevice(s->device));
    float *tmp = nullptr;
    CUDA_OK(cudaMalloc(&tmp, rec_floats * 4));
    cudaError_t e = cudaMemcpyAsync(tmp, S.data(), rec_floats * 4, cudaMemcpyHostToDevice, s->stream);
    if (e == cudaSuccess) e = gdn::launch_state_from_fp32(tmp, s->S, s->bf16_state, L * nh * 256, s->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(s->tails, T.data(), T.size() * 4, cudaMemcpyHostToDevice, s->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s->stream);
    cudaFree(tmp);
    if (e != cudaSuccess) return fail("gdn_b200: state upload failed: %s", cudaGetErrorString(e));
    return 0;
}

int download_state(Stream &st, float *rec, float *conv) {
    Stream *s = &st;
    const GDNWeightHeader &c = s->dm->cfg;
    const size_t L = c.num_layers, nh = c.num_heads, H = c.hidden_size;
    const size_t rec_floats = L * nh * 256 * 256;
    std::vector<float> S(rec_floats), T(L * 3 * H * 4);
    CUDA_OK(cudaSetDevice(s->device));
    float *tmp = nullptr;
    CUDA_OK(cudaMalloc(&tmp, rec_floats * 4));
    cudaError_t e = gdn::launch_state_to_fp32(s->S, s->bf16_state, tmp, L * nh * 256, s->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(S.data(), tmp, rec_floats * 4, cudaMemcpyDeviceToHost, s->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(T.data(), s->tails, T.size() * 4, cudaMemcpyDeviceToHost, s->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s->stream);
    cudaFree(tmp);
    if (e != cudaSuccess) return fail("gdn_b200: state download failed: %s", cudaGetErrorString(e));
    parallel_for(L * nh, [&](size_t b, size_t e2) {
        for (size_t lh = b; lh < e2; ++lh)
            for (size_t k = 0; k < 256; ++k)
                for (size_t v = 0; v < 256; ++v) rec[(lh * 256 + k) * 256 + v] = S[(lh * 256 + v) * 256 + k];
    });
    for (size_t lk = 0; lk < L * 3; ++lk)
        for (size_t d = 0; d < H; ++d)
            for (size_t r = 0; r < 3; ++r) conv[(lk * 3 + r) * H + d] = T[(lk * H + d) * 4 + r];
    return 0;
}

/* Reference-ABI compatibility: state written by the caller into the host
 * stripes / head buffer (gdn_scatter_recurrent_state, gdn_pack_conv_tails_bf16)
 * goes to the device before the next step, and after every step the device
 * state is written back there (BF16, the c_impl state format), so callers that
 * read the stripes (c_impl/gdn_eval.cpp's state dump) see the current state. */
Beat512 *stripe(Stream &s, int p) { return s.shards[GDN_RECURRENT_STATE_FIRST_PORT + p] + s.shard_beats; }

int compat_pull(Stream &s) {
    const GDNWeightHeader &c = s.dm->cfg;
    const size_t rec_floats = (size_t)c.num_layers * c.num_heads * 256 * 256;
    const size_t conv_floats = (size_t)c.num_layers * 9 * c.hidden_size;
    std::vector<float> rec(rec_floats), conv(conv_floats);
    Beat512 *st[4] = {stripe(s, 0), stripe(s, 1), stripe(s, 2), stripe(s, 3)};
    gdn::abi::gather_recurrent_state(st, rec.data(), rec_floats);
    gdn::abi::unpack_conv_tails(reinterpret_cast<const Beat512 *>(s.ws + GDN_WS_OFF_HEAD_BUF), conv.data(), conv_floats);
    s.host_dirty = false;
    return upload_state(s, rec.data(), conv.data());
}

int compat_push(Stream &s) {
    const GDNWeightHeader &c = s.dm->cfg;
    const size_t rec_floats = (size_t)c.num_layers * c.num_heads * 256 * 256;
    const size_t conv_floats = (size_t)c.num_layers * 9 * c.hidden_size;
    std::vector<float> rec(rec_floats), conv(conv_floats);
    if (download_state(s, rec.data(), conv.data()) != 0) return -1;
    Beat512 *st[4] = {stripe(s, 0), stripe(s, 1), stripe(s, 2), stripe(s, 3)};
    gdn::abi::store_recurrent_state(st, rec.data(), rec_floats);
    gdn::abi::store_conv_tails(reinterpret_cast<Beat512 *>(s.ws + GDN_WS_OFF_HEAD_BUF), conv.data(), conv_floats);
    return 0;
}

gdn::DecodeParams make_params(const Stream &s) {
    const DeviceModel &dm = *s.dm;
    gdn::DecodeParams p;
    memset(&p, 0, sizeof(p));
    p.H = (int)dm.cfg.hidden_size;
    p.I = (int)dm.cfg.intermediate_size;
    p.V = (int)dm.cfg.vocab_size;
    p.L = (int)dm.cfg.num_layers;
    p.nh = (int)dm.cfg.num_heads;
    p.eps = dm.cfg.norm_eps;
    p.bf16_boundary = s.bf16_boundary;
    p.native_product = s.native_product;
    p.bf16_state = s.bf16_state;
    const bool tp = s.tp_world > 1;
    p.wimg = tp ? s.tp_wimg : dm.wimg;
    p.w_lm = tp ? s.tp_lm : dm.w_lm;
    const ImageGeom geom = tp ? s.tp_geom : ImageGeom();
    p.g_qkvg = geom.g_qkvg;
    p.g_gu = geom.g_gu;
    p.g_lm = geom.g_lm;
    p.ng_narrow = geom.ng;
    p.split = tp ? 1u : 0u;
    p.layer_stride = dm.layer_stride;
    p.off_ab = dm.off_ab;
    p.off_o = dm.off_o;
    p.off_gu = dm.off_gu;
    p.off_down = dm.off_down;
    p.emb = dm.emb;
    p.aux = dm.aux;
    p.aux_stride = dm.aux_stride;
    p.exp_table = dm.exp_table;
    p.decay_tab = dm.decay_tab;
    p.exp_exc = dm.exp_exc;
    p.exp_exc_n = dm.exp_exc_n;
    p.exp_exc_bf16_n = dm.exp_exc_bf16_n;
    for (uint32_t i = 0; i < dm.exp_exc_bf16_n; ++i) p.exp_exc_bf16[i] = dm.exp_exc_bf16[i];
    p.fast_x_min = dm.fast_x_min;
    p.force_exact = s.force_exact;
    p.S = s.S;
    p.tails = s.tails;
    p.y_o = s.y_o;
    p.y_down = s.y_down;
    p.qkv = s.qkv;
    p.gate = s.gate;
    p.attn = s.attn;
    p.m = s.m;
    p.logits = s.logits;
    p.hidden_out = s.hidden;
    p.x_embed = s.x_embed;
    p.token_src = nullptr;
    p.token_imm = -1;
    p.cand_val = s.cand_val;
    p.cand_idx = s.cand_idx;
    p.token_out = nullptr;
    p.status = s.status;
    p.epoch = s.epoch;
    p.test_drop_cta = s.test_drop_cta;
    p.test_drop_phase = s.test_drop_phase;
    p.tp_world = s.tp_world;
    p.tp_rank = s.tp_rank;
    for (int r = 0; r < gdn::kMaxTpRanks; ++r)
        p.tp_delta[r] = s.tp_peer[r] == nullptr ? 0
                                                : (long long)(reinterpret_cast<char *>(s.tp_peer[r]) -
                                                              reinterpret_cast<char *>(s.xbuf));
    p.rank_cand = s.rank_cand;
    return p;
}

/* A run state that holds one rank's part of a tensor-parallel state. */
int refuse_part(const Stream &s, const char *what) {
    return fail("gdn_b200: %s: the run state holds rank %d's part of a tensor-parallel state (%s); join the "
                "ranks' parts (gdn_b200_tp_state_download_part, tensor_parallel.merge_state) and upload the full "
                "state first",
                what, s.part_rank, s.tp_world > 1 ? "attached" : "since its last tensor-parallel step");
}

int launch(Stream &s, gdn::DecodeParams &p) {
    if (s.tp_world == 1 && s.tp_part) return refuse_part(s, "single-GPU decode");
    if (s.tp_world > 1) {
        s.tp_part = true;
        s.part_grid = s.tp_grid;
        s.part_rank = s.tp_rank;
        s.part_world = s.tp_world;
    }
    p.epoch = s.epoch;
    const cudaError_t e = gdn::launch_decode(p, s.tp_world > 1 ? s.tp_grid : s.grid, s.stream);
    if (e != cudaSuccess) return fail("gdn_b200: decode launch failed: %s", cudaGetErrorString(e));
    s.epoch += gdn::epoch_stride(p.L);
    return 0;
}

/* After a synchronised step: read the status block and recover from a
 * kernel-reported error (the counters are reset so the stream stays usable). */
int check_status(Stream &s) {
    if (s.status_host->err == gdn::kErrNone) return 0;
    const int err = s.status_host->err;
    const unsigned cta = s.status_host->err_cta, where = s.status_host->err_where;
    cudaMemsetAsync(s.status, 0, sizeof(gdn::DecodeStatus), s.stream);
    cudaStreamSynchronize(s.stream);
    static const char *names[] = {"none", "exchange wait timeout", "chunk wait timeout", "ring slot timeout",
                                  "aborted", "token id out of range"};
    return fail("gdn_b200: decode kernel reported %s (cta %u, at %u)", names[err >= 0 && err <= 5 ? err : 4], cta,
                where);
}

/* A launch of a multi-token loop failed: the launches already queued still
 * run; wait for them and report what the kernel recorded (or the launch
 * error) before returning -1, so the caller sees a settled run state. */
int abort_loop(Stream &s, int launched) {
    const std::string launch_err = g_last_error;
    cudaStreamSynchronize(s.stream);
    if (cudaMemcpy(s.status_host, s.status, sizeof(gdn::DecodeStatus), cudaMemcpyDeviceToHost) == cudaSuccess &&
        s.status_host->err != gdn::kErrNone && check_status(s) != 0)
        return fail("%s (after %d launched steps; %s)", g_last_error.c_str(), launched, launch_err.c_str());
    return fail("%s (after %d launched steps)", launch_err.c_str(), launched);
}

int sync_and_check(Stream &s) {
    cudaError_t e = cudaMemcpyAsync(s.status_host, s.status, sizeof(gdn::DecodeStatus), cudaMemcpyDeviceToHost,
                                    s.stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s.stream);
    if (e != cudaSuccess) return fail("gdn_b200: decode step failed: %s", cudaGetErrorString(e));
    return check_status(s);
}

/* BF16 x BF16 -> BF16 product with DAZ/FTZ, the reference's GEMV product
 * contract (c_impl/gdn_model.cpp:392-462), as FP32 bits. */
uint32_t native_product_bits(uint16_t lhs, uint16_t rhs) {
    const uint32_t le = (lhs >> 7) & 0xffu, re = (rhs >> 7) & 0xffu;
    const bool lnan = le == 0xffu && (lhs & 0x7fu), rnan = re == 0xffu && (rhs & 0x7fu);
    const bool linf = le == 0xffu && !(lhs & 0x7fu), rinf = re == 0xffu && !(rhs & 0x7fu);
    const bool lz = le == 0, rz = re == 0;
    const uint32_t sign = (uint32_t)((lhs ^ rhs) & 0x8000u);
    if (lnan || rnan || (linf && rz) || (rinf && lz)) return 0x7fc00000u;
    if (linf || rinf) return (sign | 0x7f80u) << 16;
    if (lz || rz) return sign << 16;
    volatile float prod = u2f((uint32_t)lhs << 16) * u2f((uint32_t)rhs << 16);
    const uint32_t pb = f2u(prod), mag = pb & 0x7fffffffu;
    if (mag == 0x7f800000u) return pb & 0xffff0000u;
    if (mag < 0x007fc000u) return pb & 0x80000000u;
    const uint32_t res = ((pb + 0x7fffu + ((pb >> 16) & 1u)) >> 16) & 0xffffu;
    if ((res & 0x7f80u) == 0) return (res & 0x8000u) << 16;
    return res << 16;
}

uint16_t bf16_rne_bits(float v) {
    const uint32_t b = f2u(v), mag = b & 0x7fffffffu;
    if (mag >= 0x7f800000u) {
        if (mag == 0x7f800000u) return (uint16_t)(b >> 16);
        return (uint16_t)((b & 0x80000000u) ? 0xffc0u : 0x7fc0u);
    }
    return (uint16_t)((b + 0x7fffu + ((b >> 16) & 1u)) >> 16);
}

}  // namespace

/* Shared with the multi-stream layer (gdn_batch_host.cu): one error string and
 * one device selection per thread for the whole library. */
namespace gdn {
/* A caller wrote state through the reference's packing functions into buffers
 * of a run state: mark it for upload before its next step. */
void host_note_state_write(const void *buffer) {
    std::lock_guard<std::mutex> lock(g_mu);
    for (auto &kv : g_streams) {
        Stream *s = kv.second;
        if (!s->compat) continue;
        if (buffer == (const void *)(s->ws + GDN_WS_OFF_HEAD_BUF) ||
            buffer == (const void *)(s->shards[GDN_RECURRENT_STATE_FIRST_PORT] + s->shard_beats))
            s->host_dirty = true;
    }
}
int host_fail(const char *msg) { return fail("%s", msg); }
int host_device() { return g_device; }
/* The recurrent state of a run state as FP32 [L][nh][v][k] in natural order
 * (the layout of the prefill kernels), in a device buffer that
 * host_state_end writes back into the run state's own storage (rounded to
 * BF16 when the run state keeps BF16 state) and frees. Tails: FP32
 * [L][3][H][4], the run state's own buffer. */
int host_state_begin(GDNRunState *state, float **S, float **tails, int *device, cudaStream_t *stream) {
    Stream *s = find_stream(state);
    if (s == nullptr) return fail("gdn_b200: unknown run state");
    if (s->tp_world > 1 || s->tp_part) return refuse_part(*s, "prefill");
    const GDNWeightHeader &c = s->dm->cfg;
    const size_t cols = (size_t)c.num_layers * c.num_heads * 256;
    CUDA_OK(cudaSetDevice(s->device));
    float *tmp = nullptr;
    CUDA_OK(cudaMalloc(&tmp, cols * 256 * 4));
    const cudaError_t e = gdn::launch_state_to_fp32(s->S, s->bf16_state, tmp, cols, s->stream);
    if (e != cudaSuccess) {
        cudaFree(tmp);
        return fail("gdn_b200: state conversion failed: %s", cudaGetErrorString(e));
    }
    *S = tmp;
    *tails = s->tails;
    *device = s->device;
    *stream = s->stream;
    return 0;
}
int host_state_end(GDNRunState *state, float *S, bool write_back) {
    Stream *s = find_stream(state);
    if (s == nullptr) {
        cudaFree(S);
        return fail("gdn_b200: unknown run state");
    }
    const GDNWeightHeader &c = s->dm->cfg;
    const size_t cols = (size_t)c.num_layers * c.num_heads * 256;
    cudaError_t e = cudaSuccess;
    if (write_back) e = gdn::launch_state_from_fp32(S, s->S, s->bf16_state, cols, s->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s->stream);
    cudaFree(S);
    if (e != cudaSuccess) return fail("gdn_b200: state conversion failed: %s", cudaGetErrorString(e));
    return 0;
}
}  // namespace gdn

/* ================================================================ C ABI */

extern "C" {

int gdn_b200_set_device(int device) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n)
        return fail("gdn_b200: no CUDA device %d", device);
    g_device = device;
    CUDA_OK(cudaSetDevice(device));
    return 0;
}

const char *gdn_b200_last_error(void) { return g_last_error.c_str(); }

int gdn_b200_grid_size(void) {
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, g_device) != cudaSuccess) return -1;
    return sms;
}

int gdn_model_load(GDNModel *model, const char *path) {
    memset(model, 0, sizeof(*model));
    FILE *f = fopen(path, "rb");
    if (f == nullptr) return fail("fopen weights: %s", path);
    if (fread(&model->config, 1, kHeaderBytes, f) != kHeaderBytes) {
        fclose(f);
        return fail("failed to read weight header");
    }
    if (validate_config(model->config) != 0) { fclose(f); return -1; }
    const size_t n = total_floats(model->config);
    model->weight_data = (float *)malloc(n * sizeof(float));
    model->layers = (GDNLayerWeights *)calloc(model->config.num_layers, sizeof(GDNLayerWeights));
    if (model->weight_data == nullptr || model->layers == nullptr) {
        fclose(f);
        gdn_model_free(model);
        return fail("malloc failed");
    }
    /* Read in chunks and validate each chunk's BF16-exactness while reading
     * (c_impl/gdn_model.cpp:1190-1216), so a non-BF16 blob fails early. */
    const size_t chunk = (size_t)64 << 20;
    for (size_t b = 0; b < n; b += chunk) {
        const size_t req = std::min(chunk, n - b);
        if (fread(model->weight_data + b, sizeof(float), req, f) != req) {
            fclose(f);
            gdn_model_free(model);
            return fail("failed to read weight payload");
        }
        std::atomic<size_t> bad{(size_t)-1};
        const float *w = model->weight_data + b;
        parallel_for(req, [&](size_t lo, size_t hi) {
            for (size_t i = lo; i < hi; ++i)
                if (f2u(w[i]) & 0xffffu) {
                    size_t cur = bad.load();
                    while (i < cur && !bad.compare_exchange_weak(cur, i)) {
                    }
                    return;
                }
        });
        if (bad.load() != (size_t)-1) {
            const size_t i = b + bad.load();
            fclose(f);
            fail("gdn: weight %zu is not BF16-exact (bits=0x%08x)", i, f2u(model->weight_data[i]));
            gdn_model_free(model);
            return fail("dense packing requires a BF16-exact FP32-word checkpoint");
        }
    }
    fclose(f);
    assign_views(model);
    return 0;
}

int gdn_b200_model_synth(GDNModel *model, const GDNWeightHeader *config, uint64_t seed) {
    memset(model, 0, sizeof(*model));
    model->config = *config;
    if (validate_config(model->config) != 0) return -1;
    const GDNWeightHeader &c = model->config;
    const size_t n = total_floats(c);
    model->weight_data = (float *)malloc(n * sizeof(float));
    model->layers = (GDNLayerWeights *)calloc(c.num_layers, sizeof(GDNLayerWeights));
    if (model->weight_data == nullptr || model->layers == nullptr) {
        gdn_model_free(model);
        return fail("malloc failed");
    }
    /* tensor table in blob order */
    struct T { size_t off, size; uint32_t id; };
    std::vector<T> tensors;
    const size_t H = c.hidden_size, nh = c.num_heads, hd = c.head_dim, I = c.intermediate_size, cs = c.conv_size;
    const size_t sizes[GDN_SYNTH_TENSORS_PER_LAYER] = {H, nh, nh, H * H, H * H, H * H, nh * H, nh * H, H * cs,
                                                       H * cs, H * cs, H * H, hd, H * H, H, I * H, I * H, H * I};
    size_t off = 0;
    uint32_t id = 0;
    tensors.push_back({off, (size_t)c.vocab_size * H, id++});
    off += (size_t)c.vocab_size * H;
    for (uint32_t l = 0; l < c.num_layers; ++l)
        for (int j = 0; j < GDN_SYNTH_TENSORS_PER_LAYER; ++j) {
            tensors.push_back({off, sizes[j], id++});
            off += sizes[j];
        }
    tensors.push_back({off, H, id++});
    off += H;
    tensors.push_back({off, (size_t)c.vocab_size * H, id++});
    const size_t piece = (size_t)1 << 20;
    const size_t pieces = (n + piece - 1) / piece;
    parallel_for(pieces, [&](size_t pb, size_t pe) {
        size_t ti = 0;
        for (size_t pc = pb; pc < pe; ++pc) {
            const size_t lo = pc * piece, hi = std::min(n, lo + piece);
            while (ti < tensors.size() && tensors[ti].off + tensors[ti].size <= lo) ++ti;
            for (size_t k = ti; k < tensors.size() && tensors[k].off < hi; ++k) {
                const size_t b0 = std::max(lo, tensors[k].off), e0 = std::min(hi, tensors[k].off + tensors[k].size);
                gdn_synth_fill(model->weight_data + b0, seed, tensors[k].id,
                               gdn_synth_tensor_dist(tensors[k].id, c.num_layers), b0 - tensors[k].off,
                               e0 - tensors[k].off);
            }
        }
    });
    assign_views(model);
    return 0;
}

int gdn_b200_model_save(const GDNModel *model, const char *path) {
    FILE *f = fopen(path, "wb");
    if (f == nullptr) return fail("cannot create %s", path);
    const size_t n = total_floats(model->config);
    const bool ok = fwrite(&model->config, 1, kHeaderBytes, f) == kHeaderBytes &&
                    fwrite(model->weight_data, sizeof(float), n, f) == n;
    fclose(f);
    return ok ? 0 : fail("write failed: %s", path);
}

void gdn_model_free(GDNModel *model) {
    if (model == nullptr) return;
    {
        std::lock_guard<std::mutex> lock(g_mu);
        auto it = g_models.find(model->weight_data);
        if (it != g_models.end()) {
            DeviceModel *dm = it->second;
            g_models.erase(it);
            dm->model_alive = false;
            if (dm->refs == 0) free_device_model(dm);
        }
    }
    free(model->weight_data);
    free(model->layers);
    memset(model, 0, sizeof(*model));
}

int gdn_run_state_init(GDNRunState *state, const GDNModel *model, uint32_t max_tokens) {
    memset(state, 0, sizeof(*state));
    if (max_tokens == 0 || max_tokens > model->config.max_seq_len) return fail("invalid max_tokens for run state");
    if (engine_supports(model->config) != 0) return -1;
    CUDA_OK(cudaSetDevice(g_device));
    DeviceModel *dm = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_mu);
        auto it = g_models.find(model->weight_data);
        if (it != g_models.end()) dm = it->second;
    }
    if (dm == nullptr) {
        dm = build_device_model(model);
        if (dm == nullptr) return -1;
        std::lock_guard<std::mutex> lock(g_mu);
        g_models[model->weight_data] = dm;
    }
    if (dm->device != g_device) return fail("gdn_b200: model image lives on device %d, run state on %d", dm->device, g_device);

    Stream *s = new Stream();
    s->dm = dm;
    s->device = g_device;
    /* one CTA per SM, but never more CTAs than units of the smallest phase:
     * every CTA owns work in every phase (the exchange ordering relies on it) */
    s->grid = gdn_b200_grid_size();
    {
        const GDNWeightHeader &hc = model->config;
        const int units[] = {(int)(4 * hc.hidden_size / gdn::kTileRowsQKVG), (int)(hc.num_heads * 256),
                             (int)hc.hidden_size, (int)(2 * hc.intermediate_size / gdn::kTileRowsGU),
                             (int)(hc.vocab_size / gdn::kTileRowsLM)};
        for (int u : units) s->grid = std::min(s->grid, u);
    }
    if (engine_grid_ok(model->config, s->grid) != 0) return -1;
    const GDNWeightHeader &c = model->config;
    const size_t H = c.hidden_size, I = c.intermediate_size, V = c.vocab_size, nh = c.num_heads, L = c.num_layers;
    auto cleanup = [&](int rc) {
        if (s->stream) cudaStreamDestroy(s->stream);
        if (s->ev0) cudaEventDestroy(s->ev0);
        if (s->ev1) cudaEventDestroy(s->ev1);
        cudaFree(s->S);
        cudaFree(s->tails);
        cudaFree(s->acts);
        cudaFree(s->xbuf);
        cudaFree(s->status);
        cudaFreeHost(s->status_host);
        cudaFreeHost(s->ws);
        delete s;
        return rc;
    };
    if (cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreate(&s->ev0) != cudaSuccess || cudaEventCreate(&s->ev1) != cudaSuccess)
        return cleanup(fail("gdn_b200: stream creation failed"));
    const size_t s_bytes = L * nh * 256 * 256 * sizeof(float);
    const size_t t_bytes = L * 3 * H * 4 * sizeof(float);
    const size_t act_floats = H + H + 2 * (size_t)s->grid + 64;
    /* the exchange region (one allocation, the one a tensor-parallel peer
     * maps): exchange words, the per-rank argmax candidates, logits */
    const size_t xwords = 3 * H + H + H + H + I + H;
    s->xwords = xwords + gdn::kRankCandWords;
    s->xbytes = s->xwords * sizeof(gdn::xword) + V * sizeof(float);
    if (cudaMalloc(&s->S, s_bytes) != cudaSuccess || cudaMalloc(&s->tails, t_bytes) != cudaSuccess ||
        cudaMalloc(&s->acts, act_floats * sizeof(float)) != cudaSuccess ||
        cudaMalloc(&s->xbuf, s->xbytes) != cudaSuccess ||
        cudaMalloc(&s->status, sizeof(gdn::DecodeStatus)) != cudaSuccess ||
        cudaMallocHost(&s->status_host, sizeof(gdn::DecodeStatus)) != cudaSuccess ||
        cudaHostAlloc(&s->ws, GDN_WS_FLOATS * sizeof(float), cudaHostAllocDefault) != cudaSuccess)
        return cleanup(fail("gdn_b200: run state allocation failed"));
    gdn::xword *x = s->xbuf;
    s->qkv = x; x += 3 * H;
    s->gate = x; x += H;
    s->attn = x; x += H;
    s->y_o = x; x += H;
    s->m = x; x += I;
    s->y_down = x;
    s->rank_cand = reinterpret_cast<unsigned long long *>(s->xbuf + xwords);
    s->logits = reinterpret_cast<float *>(s->xbuf + s->xwords);
    float *a = s->acts;
    s->hidden = a; a += H;
    s->x_embed = a; a += H;
    s->cand_val = a; a += s->grid;
    s->cand_idx = reinterpret_cast<int32_t *>(a);
    /* exchange words start as all ones: tag 0xffff (32-bit words) or
     * 0xffffffff (64-bit words), which the first launches (epoch 0, tags
     * 0 .. 5L) never use; every refill with ones also restarts the epoch */
    if (cudaMemsetAsync(s->S, 0, s_bytes, s->stream) != cudaSuccess ||
        cudaMemsetAsync(s->tails, 0, t_bytes, s->stream) != cudaSuccess ||
        cudaMemsetAsync(s->acts, 0, act_floats * sizeof(float), s->stream) != cudaSuccess ||
        cudaMemsetAsync(s->xbuf, 0xff, s->xwords * sizeof(gdn::xword), s->stream) != cudaSuccess ||
        cudaMemsetAsync(s->logits, 0, V * sizeof(float), s->stream) != cudaSuccess ||
        cudaMemsetAsync(s->status, 0, sizeof(gdn::DecodeStatus), s->stream) != cudaSuccess ||
        cudaStreamSynchronize(s->stream) != cudaSuccess)
        return cleanup(fail("gdn_b200: run state initialisation failed"));
    memset(s->ws, 0, GDN_WS_FLOATS * sizeof(float));
    state->workspace = reinterpret_cast<Beat512 *>(s->ws);
    state->x = s->ws + GDN_WS_OFF_X;
    state->recurrent_state = s->ws + GDN_WS_OFF_REC_STATE;
    state->head_buffer = s->ws + GDN_WS_OFF_HEAD_BUF;
    const char *env = getenv("GDN_B200_ABI_COMPAT");
    if (g_abi_compat || (env != nullptr && env[0] == '1')) {
        /* the reference's run state: 32 packed shards (28..31 followed by the
         * BF16 state stripes) and the aux image (c_impl/gdn_model.cpp:1266-1293),
         * and the reference's own arithmetic */
        s->compat = true;
        s->shard_beats = gdn_weight_shard_beats(&c);
        for (int ch = 0; ch < GEMV_CHANNELS; ++ch) {
            const bool st = ch >= GDN_RECURRENT_STATE_FIRST_PORT && ch < GDN_RECURRENT_STATE_FIRST_PORT + 4;
            const size_t beats = s->shard_beats + (st ? GDN_RECURRENT_STATE_STRIPE_BF16_BEATS : 0);
            s->shards[ch] = static_cast<Beat512 *>(aligned_alloc(64, beats * sizeof(Beat512)));
            if (s->shards[ch] == nullptr) {
                for (int j = 0; j < ch; ++j) free(s->shards[j]);
                return cleanup(fail("gdn_b200: host shard allocation failed"));
            }
            if (st) memset(s->shards[ch] + s->shard_beats, 0, GDN_RECURRENT_STATE_STRIPE_BF16_BEATS * sizeof(Beat512));
        }
        gdn_build_weight_shards(model->weight_data, &c, s->shards);
        s->aux = static_cast<Beat512 *>(aligned_alloc(64, gdn_aux_image_beats(&c) * sizeof(Beat512)));
        if (s->aux == nullptr) {
            for (auto &p : s->shards) free(p);
            return cleanup(fail("gdn_b200: aux image allocation failed"));
        }
        gdn_build_aux_image(model->weight_data, &c, s->aux);
        for (int ch = 0; ch < GEMV_CHANNELS; ++ch) state->weight_shards[ch] = s->shards[ch];
        state->aux_weights = s->aux;
        s->bf16_boundary = 1;
        s->native_product = 1;
        s->bf16_state = 1;
    }
    {
        std::lock_guard<std::mutex> lock(g_mu);
        dm->refs++;
        g_streams[state->workspace] = s;
    }
    return 0;
}

/* ----------------------------------------------- tensor-parallel decode */

/* What a rank publishes so that its peers can map its exchange region
 * (GDN_B200_TP_TOKEN_BYTES). */
struct TpToken {
    cudaIpcMemHandle_t handle;
    uint32_t grid;
    uint32_t pad;
    uint64_t xbytes;
    char bus[48];   /* PCI bus id of the run state's device */
};
static_assert(sizeof(TpToken) == GDN_B200_TP_TOKEN_BYTES, "TpToken size");

static void tp_close(Stream &s) {
    for (int r = 0; r < gdn::kMaxTpRanks; ++r) {
        if (s.tp_peer[r] != nullptr) cudaIpcCloseMemHandle(s.tp_peer[r]);
        s.tp_peer[r] = nullptr;
    }
    s.tp_world = 1;
    s.tp_rank = 0;
    s.tp_geom = ImageGeom();
    s.tp_wimg = s.tp_lm = nullptr;
}

static int tp_token_of(Stream &s, TpToken &t) {
    memset(&t, 0, sizeof(t));
    CUDA_OK(cudaSetDevice(s.device));
    CUDA_OK(cudaIpcGetMemHandle(&t.handle, s.xbuf));
    t.grid = (uint32_t)s.grid;
    t.xbytes = s.xbytes;
    CUDA_OK(cudaDeviceGetPCIBusId(t.bus, (int)sizeof(t.bus) - 1, s.device));
    return 0;
}

int gdn_b200_tp_token(GDNRunState *state, void *token) {
    Stream *s = find_stream(state);
    if (s == nullptr) return fail("gdn_b200: unknown run state");
    if (token == nullptr) return fail("gdn_b200_tp_token: null token");
    TpToken t;
    if (tp_token_of(*s, t) != 0) return -1;
    memcpy(token, &t, sizeof(t));
    return 0;
}

int gdn_b200_tp_attach(GDNRunState *state, int rank, int world, const void *tokens) {
    Stream *s = find_stream(state);
    if (s == nullptr) return fail("gdn_b200: unknown run state");
    if (world < 1 || world > gdn::kMaxTpRanks || rank < 0 || rank >= world)
        return fail("gdn_b200_tp_attach: rank %d of %d out of range (at most %d GPUs)", rank, world, gdn::kMaxTpRanks);
    if (tokens == nullptr) return fail("gdn_b200_tp_attach: null tokens");
    if (s->compat) return fail("gdn_b200_tp_attach: not available in the reference-ABI compatibility mode");
    const TpToken *t = static_cast<const TpToken *>(tokens);
    TpToken mine;
    if (tp_token_of(*s, mine) != 0) return -1;
    if (memcmp(&t[rank], &mine, sizeof(mine)) != 0)
        return fail("gdn_b200_tp_attach: token %d is not this run state's", rank);
    for (int r = 0; r < world; ++r) {
        if (t[r].grid != mine.grid || t[r].xbytes != mine.xbytes)
            return fail("gdn_b200_tp_attach: rank %d has another grid (%u) or exchange size than this GPU (%u)", r,
                        t[r].grid, mine.grid);
        for (int q = 0; q < r; ++q)
            if (strncmp(t[q].bus, t[r].bus, sizeof(t[r].bus)) == 0)
                return fail("gdn_b200_tp_attach: ranks %d and %d share the device %s", q, r, t[r].bus);
    }
    CUDA_OK(cudaSetDevice(s->device));
    CUDA_OK(cudaStreamSynchronize(s->stream));
    tp_close(*s);
    for (int r = 0; r < world; ++r) {
        if (r == rank) continue;
        const cudaError_t e = cudaIpcOpenMemHandle(&s->tp_peer[r], t[r].handle, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            s->tp_peer[r] = nullptr;
            tp_close(*s);
            return fail("gdn_b200_tp_attach: mapping rank %d's exchange region failed: %s", r, cudaGetErrorString(e));
        }
    }
    /* the largest per-GPU grid whose world * grid CTAs all own units of
     * every phase (the GU projection's 16-row tiles run out first) */
    int g = s->grid;
    while (g > 0 && engine_grid_ok(s->dm->cfg, world * g, false) != 0) --g;
    if (g == 0) {
        tp_close(*s);
        return fail("gdn_b200_tp_attach: no grid fits %d GPUs for this model", world);
    }
    const ImageGeom geom = image_geometry(s->dm->cfg, (uint32_t)(world * g));
    if (device_image(s->dm, geom, s->stream, &s->tp_wimg, &s->tp_lm) != 0) {
        tp_close(*s);
        return -1;
    }
    s->tp_geom = geom;
    s->tp_grid = g;
    s->tp_world = world;
    s->tp_rank = rank;
    /* every rank starts from the same tags */
    s->epoch = 0;
    CUDA_OK(cudaMemsetAsync(s->xbuf, 0xff, s->xwords * sizeof(gdn::xword), s->stream));
    CUDA_OK(cudaStreamSynchronize(s->stream));
    return 0;
}

int gdn_b200_tp_detach(GDNRunState *state) {
    Stream *s = find_stream(state);
    if (s == nullptr) return fail("gdn_b200: unknown run state");
    CUDA_OK(cudaSetDevice(s->device));
    CUDA_OK(cudaStreamSynchronize(s->stream));
    tp_close(*s);
    CUDA_OK(cudaMemsetAsync(s->xbuf, 0xff, s->xwords * sizeof(gdn::xword), s->stream));
    CUDA_OK(cudaStreamSynchronize(s->stream));
    s->epoch = 0;
    return 0;
}

void gdn_run_state_free(GDNRunState *state) {
    if (state == nullptr || state->workspace == nullptr) return;
    Stream *s = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_mu);
        auto it = g_streams.find(state->workspace);
        if (it != g_streams.end()) {
            s = it->second;
            g_streams.erase(it);
        }
    }
    if (s != nullptr) {
        int prev = 0;
        cudaGetDevice(&prev);
        cudaSetDevice(s->device);
        cudaStreamSynchronize(s->stream);
        tp_close(*s);
        cudaStreamDestroy(s->stream);
        cudaEventDestroy(s->ev0);
        cudaEventDestroy(s->ev1);
        cudaFree(s->S);
        cudaFree(s->tails);
        cudaFree(s->acts);
        cudaFree(s->xbuf);
        cudaFree(s->status);
        cudaFree(s->tokens);
        cudaFree(s->argmax);
        cudaFreeHost(s->status_host);
        cudaFreeHost(s->ws);
        for (auto &p : s->shards) free(p);
        free(s->aux);
        cudaSetDevice(prev);
        std::lock_guard<std::mutex> lock(g_mu);
        DeviceModel *dm = s->dm;
        if (--dm->refs == 0 && !dm->model_alive) free_device_model(dm);
        delete s;
    }
    memset(state, 0, sizeof(*state));
}

int gdn_b200_set_numerics(GDNRunState *state, int bf16_boundary, int bf16_products, int bf16_state) {
    Stream *s = find_stream(state);
    if (s == nullptr) return fail("gdn_b200: unknown run state");
    const int boundary = bf16_boundary ? 1 : 0, products = bf16_products ? 1 : 0, bstate = bf16_state ? 1 : 0;
    const bool fp32 = !boundary && !products && !bstate, engine = boundary && !products && !bstate,
               cimpl = boundary && products && bstate;
    if (!(fp32 || engine || cimpl))
        return fail("gdn_b200: numerics (%d, %d, %d) is not a contract of this engine: (1, 1, 1) the reference's "
                    "own (c_impl), (1, 0, 0) exact products with FP32 state, (0, 0, 0) the FP32 control",
                    boundary, products, bstate);
    if (s->tp_world > 1)
        return fail("gdn_b200: numerics cannot change while the run state is attached for tensor parallelism "
                    "(every rank must run the same contract): detach every rank first");
    CUDA_OK(cudaSetDevice(s->device));
    if (bstate != s->bf16_state) {
        /* the state changes storage (BF16 <-> FP32): convert it in place */
        const GDNWeightHeader &c = s->dm->cfg;
        const size_t cols = (size_t)c.num_layers * c.num_heads * 256;
        float *tmp = nullptr;
        CUDA_OK(cudaMalloc(&tmp, cols * 256 * 4));
        cudaError_t e = gdn::launch_state_to_fp32(s->S, s->bf16_state, tmp, cols, s->stream);
        if (e == cudaSuccess) e = gdn::launch_state_from_fp32(tmp, s->S, bstate, cols, s->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s->stream);
        cudaFree(tmp);
        if (e != cudaSuccess) return fail("gdn_b200: state conversion failed: %s", cudaGetErrorString(e));
    }
    if (boundary != s->bf16_boundary) {
        /* the exchange word width follows the boundary contract (32-bit words
         * for BF16 boundaries, 64-bit for FP32): start the buffers over, and
         * the tags with them */
        CUDA_OK(cudaMemsetAsync(s->xbuf, 0xff, s->xwords * sizeof(gdn::xword), s->stream));
        CUDA_OK(cudaStreamSynchronize(s->stream));
        s->epoch = 0;
    }
    s->bf16_boundary = boundary;
    s->native_product = products;
    s->bf16_state = bstate;
    return 0;
}

int gdn_b200_test_force_exact_products(GDNRunState *state, int on) {
    Stream *s = find_stream(state);
    if (s == nullptr) return fail("gdn_b200: unknown run state");
    s->force_exact = on ? 1 : 0;
    return 0;
}

int gdn_b200_test_set_epoch(GDNRunState *state, uint32_t epoch) {
    Stream *s = find_stream(state);
    if (s == nullptr) return fail("gdn_b200: unknown run state");
    s->epoch = epoch;
    return 0;
}

namespace {
/* Pieces (8 values) of a projection: the image map of piece i lands in range
 * at a piece boundary and its inverse gives i back, so the map is a
 * bijection of the projection's pieces. */
bool tiled_map_ok(size_t TR, size_t G, size_t rows, size_t K) {
    std::atomic<bool> ok{true};
    parallel_for(rows * K / 8, [&](size_t b, size_t e) {
        for (size_t i = b; i < e && ok.load(std::memory_order_relaxed); ++i) {
            size_t r, c;
            tiled_src(i * 8, TR, G, rows, &r, &c);
            if (r >= rows || c >= K || c % 8 != 0 || tiled_pos(r, c, TR, G, rows) != i * 8) ok = false;
        }
    });
    return ok;
}
bool rowmajor_map_ok(size_t rows, size_t K, size_t NG) {
    std::atomic<bool> ok{true};
    parallel_for(rows * K / 8, [&](size_t b, size_t e) {
        for (size_t i = b; i < e && ok.load(std::memory_order_relaxed); ++i) {
            size_t r, c;
            rowmajor_src(i * 8, rows, K, NG, &r, &c);
            if (r >= rows || c >= K || c % 8 != 0 || rowmajor_pos(r, c, rows, K, NG) != i * 8) ok = false;
        }
    });
    return ok;
}
}  // namespace

int gdn_b200_test_image_geometry(uint32_t hidden, uint32_t intermediate, uint32_t vocab, uint32_t ncta,
                                 uint32_t *geom, int check_maps) {
    if (geom == nullptr || ncta == 0) return fail("gdn_b200_test_image_geometry: null geometry or no CTAs");
    if (hidden == 0 || intermediate == 0 || hidden % 512 || intermediate % 512 || vocab == 0 || vocab % 16)
        return fail("gdn_b200_test_image_geometry: hidden and intermediate must be multiples of 512, vocab of 16");
    GDNWeightHeader c;
    memset(&c, 0, sizeof(c));
    c.hidden_size = hidden;
    c.intermediate_size = intermediate;
    c.vocab_size = vocab;
    const ImageGeom g = image_geometry(c, ncta);
    geom[0] = g.g_qkvg;
    geom[1] = g.g_gu;
    geom[2] = g.g_lm;
    geom[3] = g.ng;
    if (check_maps) {
        const size_t H = hidden, I = intermediate, V = vocab;
        for (const ImageGeom &m : {g, ImageGeom()}) {
            if (!tiled_map_ok(gdn::kTileRowsQKVG, m.g_qkvg, 4 * H, H) || !tiled_map_ok(gdn::kTileRowsGU, m.g_gu, 2 * I, H) ||
                !tiled_map_ok(gdn::kTileRowsLM, m.g_lm, V, H) || !rowmajor_map_ok(H, H, m.ng) ||
                !rowmajor_map_ok(H, I, m.ng))
                return fail("gdn_b200_test_image_geometry: a layout map of geometry (%u, %u, %u, %u) is not a bijection",
                            m.g_qkvg, m.g_gu, m.g_lm, m.ng);
        }
    }
    return 0;
}

int gdn_b200_test_drop_outputs(GDNRunState *state, int cta, int phase) {
    Stream *s = find_stream(state);
    if (s == nullptr) return fail("gdn_b200: unknown run state");
    if (cta >= s->grid) return fail("gdn_b200_test_drop_outputs: cta %d out of range", cta);
    if (cta >= 0 && (phase < 0 || phase % gdn::kPhasesPerLayer == 1))
        return fail("gdn_b200_test_drop_outputs: phase %d is not a GEMV phase (layer * 5 + {0, 2, 3, 4})", phase);
    s->test_drop_cta = cta < 0 ? -1 : cta;
    s->test_drop_phase = cta < 0 ? -1 : phase;
    return 0;
}

/* One step from the FP32 embedding row in workspace[X]: the body of the
 * reference's gdn_forward (c_impl/gdn_model.cpp:3719-3897). */
static int forward_from_workspace(Stream &st, int32_t token = -1) {
    Stream *s = &st;
    const GDNWeightHeader &c = s->dm->cfg;
    const size_t H = c.hidden_size;
    CUDA_OK(cudaSetDevice(s->device));
    if (s->compat && s->host_dirty && compat_pull(*s) != 0) return -1;
    gdn::DecodeParams p = make_params(*s);
    if (token >= 0) {
        /* workspace[X] holds that token's embedding row: the kernel gathers
         * the same row from its own copy, given the id as an argument */
        p.token_imm = token;
    } else {
        CUDA_OK(cudaMemcpyAsync(s->x_embed, s->ws + GDN_WS_OFF_X, H * sizeof(float), cudaMemcpyHostToDevice,
                                s->stream));
    }
    if (launch(*s, p) != 0) return -1;
    if (g_debug_hidden != nullptr)
        CUDA_OK(cudaMemcpyAsync(g_debug_hidden, s->hidden, H * sizeof(float), cudaMemcpyDeviceToHost, s->stream));
    if (g_debug_logits != nullptr)
        CUDA_OK(cudaMemcpyAsync(g_debug_logits, s->logits, c.vocab_size * sizeof(float), cudaMemcpyDeviceToHost,
                                s->stream));
    /* the status block's read-back carries the token line: workspace[X_NORM]
     * (64 bytes, c_impl/host.cpp:1011-1017) */
    const int rc = sync_and_check(*s);
    memcpy(s->ws + GDN_WS_OFF_X_NORM, s->status_host->token_line, 64);
    if (rc != 0) return rc;
    return s->compat ? compat_push(*s) : 0;
}

int gdn_decode_step_host(const GDNModel *model, GDNRunState *state, const int32_t *token) {
    if (*token < 0 || (uint32_t)*token >= model->config.vocab_size) return fail("token id out of range");
    Stream *s = find_stream(state);
    if (s == nullptr) return fail("gdn_b200: unknown run state");
    const size_t H = model->config.hidden_size;
    /* the host writes the FP32 embedding row into workspace[X]
     * (c_impl/gdn_model.cpp:3906-3908; c_impl/host.cpp:955-960) */
    memcpy(state->x, model->embeddings + (size_t)*token * H, H * sizeof(float));
    return forward_from_workspace(*s, *token);
}

/* The SLR-partitioned C model of the reference computes the same step
 * (c_impl/gdn_model.cpp:7216-7258); here it is the same engine call. */
int gdn_decode_step_host_partitioned(const GDNModel *model, GDNRunState *state, const int32_t *token) {
    return gdn_decode_step_host(model, state, token);
}

/* The kernel top of the reference (c_impl/gdn_model.h:224-259): one token from
 * the embedding row the host wrote into workspace[X], against the run state
 * whose workspace this is; the shard and aux pointers name the same weights the
 * engine holds on the device. The state it decodes from is that run state's
 * (after any caller write through gdn_scatter_recurrent_state /
 * gdn_pack_conv_tails_bf16). Returns 0, or -1 for an unknown workspace. */
int gdn_forward(const Beat512 *aux_weights, Beat512 *workspace, const Beat512 *mm0, const Beat512 *mm1,
                const Beat512 *mm2, const Beat512 *mm3, const Beat512 *mm4, const Beat512 *mm5, const Beat512 *mm6,
                const Beat512 *mm7, const Beat512 *mm8, const Beat512 *mm9, const Beat512 *mm10, const Beat512 *mm11,
                const Beat512 *mm12, const Beat512 *mm13, const Beat512 *mm14, const Beat512 *mm15,
                const Beat512 *mm16, const Beat512 *mm17, const Beat512 *mm18, const Beat512 *mm19,
                const Beat512 *mm20, const Beat512 *mm21, const Beat512 *mm22, const Beat512 *mm23,
                const Beat512 *mm24, const Beat512 *mm25, const Beat512 *mm26, const Beat512 *mm27, Beat512 *mm28,
                Beat512 *mm29, Beat512 *mm30, Beat512 *mm31) {
    (void)aux_weights;
    const void *unused[] = {mm0, mm1, mm2, mm3, mm4, mm5, mm6, mm7, mm8, mm9, mm10, mm11, mm12, mm13, mm14, mm15,
                            mm16, mm17, mm18, mm19, mm20, mm21, mm22, mm23, mm24, mm25, mm26, mm27, mm28, mm29, mm30,
                            mm31};
    for (const void *q : unused) (void)q;
    Stream *s = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_mu);
        auto it = g_streams.find((const void *)workspace);
        if (it != g_streams.end()) s = it->second;
    }
    if (s == nullptr) return fail("gdn_forward: workspace does not belong to a run state of this library");
    return forward_from_workspace(*s);
}

/* Reference-ABI compatibility for run states created after the call (also
 * GDN_B200_ABI_COMPAT=1 in the environment): host shard and aux images,
 * c_impl arithmetic, and the state stripes / head buffer kept in step with the
 * device state. */
int gdn_b200_set_abi_compat(int on) {
    g_abi_compat = on != 0;
    return 0;
}

int gdn_b200_decode_tokens(const GDNModel *model, GDNRunState *state, const int32_t *tokens, uint32_t n, int greedy,
                           int32_t *argmax_out, float *kernel_ms) {
    Stream *s = find_stream(state);
    if (s == nullptr) return fail("gdn_b200: unknown run state");
    if (n == 0) return 0;
    const uint32_t V = model->config.vocab_size;
    for (uint32_t i = 0; i < (greedy ? 1u : n); ++i)
        if (tokens[i] < 0 || (uint32_t)tokens[i] >= V) return fail("token id out of range");
    CUDA_OK(cudaSetDevice(s->device));
    if (s->tokens_cap < n) {
        cudaFree(s->tokens);
        cudaFree(s->argmax);
        s->tokens = nullptr;
        s->argmax = nullptr;
        s->tokens_cap = 0;
        CUDA_OK(cudaMalloc(&s->tokens, n * sizeof(int32_t)));
        CUDA_OK(cudaMalloc(&s->argmax, n * sizeof(int32_t)));
        s->tokens_cap = n;
    }
    CUDA_OK(cudaMemcpyAsync(s->tokens, tokens, (greedy ? 1u : n) * sizeof(int32_t), cudaMemcpyHostToDevice, s->stream));
    gdn::DecodeParams p = make_params(*s);
    CUDA_OK(cudaEventRecord(s->ev0, s->stream));
    for (uint32_t i = 0; i < n; ++i) {
        p.token_src = (greedy && i > 0) ? s->argmax + (i - 1) : s->tokens + i;
        p.token_out = s->argmax + i;
        if (launch(*s, p) != 0) return abort_loop(*s, (int)i);
    }
    CUDA_OK(cudaEventRecord(s->ev1, s->stream));
    if (argmax_out != nullptr)
        CUDA_OK(cudaMemcpyAsync(argmax_out, s->argmax, n * sizeof(int32_t), cudaMemcpyDeviceToHost, s->stream));
    CUDA_OK(cudaMemcpyAsync(s->ws + GDN_WS_OFF_X_NORM, s->status->token_line, 64, cudaMemcpyDeviceToHost, s->stream));
    const int rc = sync_and_check(*s);
    if (rc != 0) return rc;
    if (kernel_ms != nullptr) CUDA_OK(cudaEventElapsedTime(kernel_ms, s->ev0, s->ev1));
    return 0;
}

/* ------------------------------------------- allocation-free decode loop */

/* Scratch of gdn_b200_decode_tokens_noalloc: the step token ids in
 * [0, kNoAllocMaxTokens) and the per-step argmax in [kNoAllocMaxTokens,
 * 2 kNoAllocMaxTokens), 32 KB. A __device__ variable has one instance per
 * device, so every device has its own copy; all run states of a device share
 * it. Nothing in it has to start at zero: a call writes every entry it reads
 * (the token ids by its host-to-device copy, the argmax of step i by step i)
 * before reading it. */
constexpr uint32_t kNoAllocMaxTokens = 4096;
static __device__ __align__(256) int32_t g_noalloc_scratch[2 * kNoAllocMaxTokens];

/* Device address of the scratch on `device`, looked up once per device with
 * cudaGetSymbolAddress and cached; nullptr (error in *err) if unavailable. */
static int32_t *noalloc_scratch(int device, cudaError_t *err) {
    static std::mutex mu;
    static int32_t *addr[256] = {};
    std::lock_guard<std::mutex> lock(mu);
    *err = cudaSuccess;
    if (device < 0 || device >= 256) {
        *err = cudaErrorInvalidDevice;
        return nullptr;
    }
    if (addr[device] == nullptr) {
        void *p = nullptr;
        *err = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (*err != cudaSuccess) return nullptr;
        addr[device] = static_cast<int32_t *>(p);
    }
    return addr[device];
}

int gdn_b200_decode_tokens_noalloc(const GDNModel *model, GDNRunState *state, const int32_t *tokens, uint32_t n,
                                   int greedy, int32_t *argmax_out, float *kernel_ms) {
    Stream *s = find_stream(state);
    if (s == nullptr) return fail("gdn_b200: unknown run state");
    if (n == 0) return 0;
    if (n > kNoAllocMaxTokens)
        return fail("gdn_b200_decode_tokens_noalloc: at most %u tokens per call (got %u); split the sequence",
                    kNoAllocMaxTokens, n);
    const uint32_t V = model->config.vocab_size;
    for (uint32_t i = 0; i < (greedy ? 1u : n); ++i)
        if (tokens[i] < 0 || (uint32_t)tokens[i] >= V) return fail("token id out of range");
    CUDA_OK(cudaSetDevice(s->device));
    cudaError_t serr = cudaSuccess;
    int32_t *scratch = noalloc_scratch(s->device, &serr);
    if (scratch == nullptr)
        return fail("gdn_b200_decode_tokens_noalloc: scratch address unavailable: %s", cudaGetErrorString(serr));
    int32_t *dtok = scratch, *dmax = scratch + kNoAllocMaxTokens;
    CUDA_OK(cudaMemcpyAsync(dtok, tokens, (greedy ? 1u : n) * sizeof(int32_t), cudaMemcpyHostToDevice, s->stream));
    gdn::DecodeParams p = make_params(*s);
    CUDA_OK(cudaEventRecord(s->ev0, s->stream));
    for (uint32_t i = 0; i < n; ++i) {
        p.token_src = (greedy && i > 0) ? dmax + (i - 1) : dtok + i;
        p.token_out = dmax + i;
        if (launch(*s, p) != 0) return abort_loop(*s, (int)i);
    }
    CUDA_OK(cudaEventRecord(s->ev1, s->stream));
    if (argmax_out != nullptr)
        CUDA_OK(cudaMemcpyAsync(argmax_out, dmax, n * sizeof(int32_t), cudaMemcpyDeviceToHost, s->stream));
    CUDA_OK(cudaMemcpyAsync(s->ws + GDN_WS_OFF_X_NORM, s->status->token_line, 64, cudaMemcpyDeviceToHost, s->stream));
    const int rc = sync_and_check(*s);
    if (rc != 0) return rc;
    if (kernel_ms != nullptr) CUDA_OK(cudaEventElapsedTime(kernel_ms, s->ev0, s->ev1));
    return 0;
}

int gdn_b200_delta_rule_step(uint32_t slices, float *S, const float *q, const float *k, const float *v,
                             const float *decay, const float *beta, float *o, uint32_t steps, float *ms_per_step) {
    if (slices == 0 || steps == 0 || S == nullptr || q == nullptr || k == nullptr || v == nullptr ||
        decay == nullptr || beta == nullptr || o == nullptr)
        return fail("gdn_b200_delta_rule_step: empty or missing argument");
    CUDA_OK(cudaSetDevice(g_device));
    const size_t s_bytes = (size_t)slices * 256 * 256 * sizeof(float), vec_bytes = (size_t)slices * 256 * sizeof(float);
    const size_t flush_bytes = (size_t)256 << 20; /* twice the L2 */
    float *dS = nullptr, *dvec = nullptr;
    int *dstatus = nullptr;
    void *dflush = nullptr;
    cudaStream_t st = nullptr;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    int rc = 0;
    auto release = [&]() {
        cudaFree(dS);
        cudaFree(dvec);
        cudaFree(dstatus);
        cudaFree(dflush);
        if (e0) cudaEventDestroy(e0);
        if (e1) cudaEventDestroy(e1);
        if (st) cudaStreamDestroy(st);
    };
    if (cudaMalloc(&dS, s_bytes) != cudaSuccess || cudaMalloc(&dvec, 4 * vec_bytes + 2 * slices * sizeof(float)) != cudaSuccess ||
        cudaMalloc(&dstatus, sizeof(int)) != cudaSuccess || cudaMalloc(&dflush, flush_bytes) != cudaSuccess ||
        cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) != cudaSuccess || cudaEventCreate(&e0) != cudaSuccess ||
        cudaEventCreate(&e1) != cudaSuccess) {
        release();
        return fail("gdn_b200_delta_rule_step: allocation failed");
    }
    float *dq = dvec, *dk = dq + slices * 256, *dv = dk + slices * 256, *dout = dv + slices * 256;
    float *ddecay = dout + slices * 256, *dbeta = ddecay + slices;
    gdn::DeltaRuleParams prm{dS, dq, dk, dv, ddecay, dbeta, dout, dstatus, slices};
    double total_ms = 0.0;
    if (cudaMemcpyAsync(dS, S, s_bytes, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(dq, q, vec_bytes, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(dk, k, vec_bytes, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(dv, v, vec_bytes, cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(ddecay, decay, slices * sizeof(float), cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemcpyAsync(dbeta, beta, slices * sizeof(float), cudaMemcpyHostToDevice, st) != cudaSuccess ||
        cudaMemsetAsync(dstatus, 0, sizeof(int), st) != cudaSuccess)
        rc = fail("gdn_b200_delta_rule_step: upload failed");
    for (uint32_t i = 0; rc == 0 && i < steps; ++i) {
        float ms = 0.0f;
        if (cudaMemsetAsync(dflush, (int)(i & 0xff), flush_bytes, st) != cudaSuccess ||
            cudaEventRecord(e0, st) != cudaSuccess || gdn::launch_delta_rule(prm, st) != cudaSuccess ||
            cudaEventRecord(e1, st) != cudaSuccess || cudaEventSynchronize(e1) != cudaSuccess ||
            cudaEventElapsedTime(&ms, e0, e1) != cudaSuccess)
            rc = fail("gdn_b200_delta_rule_step: step %u failed: %s", i, cudaGetErrorString(cudaGetLastError()));
        total_ms += ms;
    }
    int status = 0;
    if (rc == 0 && (cudaMemcpyAsync(S, dS, s_bytes, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
                    cudaMemcpyAsync(o, dout, vec_bytes, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
                    cudaMemcpyAsync(&status, dstatus, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
                    cudaStreamSynchronize(st) != cudaSuccess))
        rc = fail("gdn_b200_delta_rule_step: download failed");
    if (rc == 0 && status != 0) rc = fail("gdn_b200_delta_rule_step: a state copy did not land in time");
    if (rc == 0 && ms_per_step != nullptr) *ms_per_step = (float)(total_ms / steps);
    release();
    return rc;
}

/* Teacher-forced scoring of one window, c_impl/host.cpp:1954-1994
 * (score_window_hw): the state is reset, tokens = ctx ++ cont are fed in
 * order except the last, and after each fed token i >= ctx_len - 1 the
 * log-probability of tokens[i + 1] under the step's FP32 logits is added
 * (gdn_score.cu). With use_prefill the first ctx_len - 1 tokens go through
 * gdn_b200_prefill instead of one decode step each. */
int gdn_b200_score_window(const GDNModel *model, GDNRunState *state, const int32_t *ctx, uint32_t ctx_len,
                          const int32_t *cont, uint32_t cont_len, int use_prefill, double *logprob, uint64_t *scored) {
    Stream *s = find_stream(state);
    if (s == nullptr) return fail("gdn_b200: unknown run state");
    if (ctx == nullptr || cont == nullptr || ctx_len == 0 || cont_len == 0 || logprob == nullptr)
        return fail("gdn_b200: invalid scoring window");
    const GDNWeightHeader &c = model->config;
    const uint32_t V = c.vocab_size, n = ctx_len + cont_len;
    std::vector<int32_t> tokens(ctx, ctx + ctx_len);
    tokens.insert(tokens.end(), cont, cont + cont_len);
    for (uint32_t i = 0; i < n; ++i)
        if (tokens[i] < 0 || (uint32_t)tokens[i] >= V) return fail("gdn_b200: scoring token %d out of range", tokens[i]);
    CUDA_OK(cudaSetDevice(s->device));
    const size_t L = c.num_layers, nh = c.num_heads, H = c.hidden_size;
    CUDA_OK(cudaMemsetAsync(s->S, 0, L * nh * 256 * 256 * sizeof(float), s->stream));
    CUDA_OK(cudaMemsetAsync(s->tails, 0, L * 3 * H * 4 * sizeof(float), s->stream));
    if (s->tokens_cap < n) {
        cudaFree(s->tokens);
        cudaFree(s->argmax);
        s->tokens = nullptr;
        s->argmax = nullptr;
        s->tokens_cap = 0;
        CUDA_OK(cudaMalloc(&s->tokens, n * sizeof(int32_t)));
        CUDA_OK(cudaMalloc(&s->argmax, n * sizeof(int32_t)));
        s->tokens_cap = n;
    }
    double *acc = nullptr;
    CUDA_OK(cudaMalloc(&acc, 2 * sizeof(double)));
    int rc = 0;
    uint32_t first = 0;
    if (use_prefill && ctx_len >= 2) {
        CUDA_OK(cudaStreamSynchronize(s->stream));
        rc = gdn_b200_prefill(model, state, tokens.data(), ctx_len - 1, nullptr);
        first = ctx_len - 1;
    }
    if (rc == 0 && (cudaMemsetAsync(acc, 0, 2 * sizeof(double), s->stream) != cudaSuccess ||
                    cudaMemcpyAsync(s->tokens, tokens.data(), n * sizeof(int32_t), cudaMemcpyHostToDevice,
                                    s->stream) != cudaSuccess))
        rc = fail("gdn_b200: scoring setup failed");
    gdn::DecodeParams p = make_params(*s);
    for (uint32_t i = first; rc == 0 && i + 1 < n; ++i) {
        p.token_src = s->tokens + i;
        p.token_out = s->argmax + i;
        if (launch(*s, p) != 0) rc = -1;
        else if (i + 1 >= ctx_len && gdn::launch_score(s->logits, V, s->tokens + i + 1, acc, s->stream) != cudaSuccess)
            rc = fail("gdn_b200: scoring launch failed");
    }
    double h[2] = {0.0, 0.0};
    if (rc == 0 && cudaMemcpyAsync(h, acc, sizeof(h), cudaMemcpyDeviceToHost, s->stream) != cudaSuccess)
        rc = fail("gdn_b200: scoring read-back failed");
    if (rc == 0) rc = sync_and_check(*s);
    cudaFree(acc);
    if (rc != 0) return rc;
    *logprob = h[0];
    if (scored) *scored = (uint64_t)h[1];
    return 0;
}

int gdn_b200_trace_step(const GDNModel *model, GDNRunState *state, int32_t token, uint64_t *trace_out,
                        size_t capacity) {
    Stream *s = find_stream(state);
    if (s == nullptr) return fail("gdn_b200: unknown run state");
    if (token < 0 || (uint32_t)token >= model->config.vocab_size) return fail("token id out of range");
    const size_t n = (size_t)s->grid * (model->config.num_layers * gdn::kPhasesPerLayer + 1) * gdn::kTraceSlots;
    if (trace_out == nullptr || capacity < n) return fail("gdn_b200: trace buffer needs %zu entries", n);
    CUDA_OK(cudaSetDevice(s->device));
    unsigned long long *dtrace = nullptr;
    int32_t *dtok = nullptr;
    CUDA_OK(cudaMalloc(&dtrace, n * sizeof(uint64_t)));
    if (cudaMalloc(&dtok, sizeof(int32_t)) != cudaSuccess) {
        cudaFree(dtrace);
        return fail("gdn_b200: trace allocation failed");
    }
    cudaMemsetAsync(dtrace, 0, n * sizeof(uint64_t), s->stream);
    cudaMemcpyAsync(dtok, &token, sizeof(int32_t), cudaMemcpyHostToDevice, s->stream);
    gdn::DecodeParams p = make_params(*s);
    p.token_src = dtok;
    p.trace = dtrace;
    int rc = launch(*s, p);
    if (rc == 0) rc = sync_and_check(*s);
    if (rc == 0 && cudaMemcpy(trace_out, dtrace, n * sizeof(uint64_t), cudaMemcpyDeviceToHost) != cudaSuccess)
        rc = fail("gdn_b200: trace copy failed");
    cudaFree(dtrace);
    cudaFree(dtok);
    return rc == 0 ? (int)(n / gdn::kTraceSlots) : rc;
}

int gdn_b200_fetch_outputs(GDNRunState *state, float *logits, float *final_hidden) {
    Stream *s = find_stream(state);
    if (s == nullptr) return fail("gdn_b200: unknown run state");
    CUDA_OK(cudaSetDevice(s->device));
    if (logits != nullptr)
        CUDA_OK(cudaMemcpyAsync(logits, s->logits, s->dm->cfg.vocab_size * sizeof(float), cudaMemcpyDeviceToHost,
                                s->stream));
    if (final_hidden != nullptr)
        CUDA_OK(cudaMemcpyAsync(final_hidden, s->hidden, s->dm->cfg.hidden_size * sizeof(float),
                                cudaMemcpyDeviceToHost, s->stream));
    CUDA_OK(cudaStreamSynchronize(s->stream));
    return 0;
}

int gdn_b200_state_upload(GDNRunState *state, const float *rec, size_t rec_floats, const float *conv,
                          size_t conv_floats) {
    Stream *s = find_stream(state);
    if (s == nullptr) return fail("gdn_b200: unknown run state");
    const GDNWeightHeader &c = s->dm->cfg;
    const size_t L = c.num_layers, nh = c.num_heads, H = c.hidden_size;
    if (rec_floats != L * nh * 256 * 256 || conv_floats != L * 3 * 3 * H)
        return fail("gdn_b200: state sizes do not match the model (rec %zu, conv %zu)", rec_floats, conv_floats);
    if (upload_state(*s, rec, conv) != 0) return -1;
    s->tp_part = false;  /* a full state again */
    return 0;
}

int gdn_b200_state_download(GDNRunState *state, float *rec, size_t rec_floats, float *conv, size_t conv_floats) {
    Stream *s = find_stream(state);
    if (s == nullptr) return fail("gdn_b200: unknown run state");
    const GDNWeightHeader &c = s->dm->cfg;
    const size_t L = c.num_layers, nh = c.num_heads, H = c.hidden_size;
    if (rec_floats != L * nh * 256 * 256 || conv_floats != L * 3 * 3 * H)
        return fail("gdn_b200: state sizes do not match the model");
    if (s->tp_world > 1 || s->tp_part) return refuse_part(*s, "state download");
    return download_state(*s, rec, conv);
}

int gdn_b200_tp_state_download_part(GDNRunState *state, float *rec, size_t rec_floats, float *conv,
                                    size_t conv_floats, int32_t *tp_grid, int32_t *tp_rank, int32_t *tp_world) {
    Stream *s = find_stream(state);
    if (s == nullptr) return fail("gdn_b200: unknown run state");
    const GDNWeightHeader &c = s->dm->cfg;
    const size_t L = c.num_layers, nh = c.num_heads, H = c.hidden_size;
    if (rec_floats != L * nh * 256 * 256 || conv_floats != L * 3 * 3 * H)
        return fail("gdn_b200: state sizes do not match the model");
    if (!s->tp_part)
        return fail("gdn_b200: the run state took no tensor-parallel step since its last full upload "
                    "(gdn_b200_state_download gives its state)");
    if (download_state(*s, rec, conv) != 0) return -1;
    if (tp_grid != nullptr) *tp_grid = s->part_grid;
    if (tp_rank != nullptr) *tp_rank = s->part_rank;
    if (tp_world != nullptr) *tp_world = s->part_world;
    return 0;
}

int gdn_b200_state_load_file(GDNRunState *state, const char *path, int32_t *seed_token) {
    Stream *s = find_stream(state);
    if (s == nullptr) return fail("gdn_b200: unknown run state");
    FILE *f = fopen(path, "rb");
    if (f == nullptr) return fail("cannot open .gdnstate file");
    char magic[8];
    uint32_t v[9];
    if (fread(magic, 1, 8, f) != 8 || memcmp(magic, "GDNSTAT1", 8) != 0) {
        fclose(f);
        return fail(".gdnstate: bad magic (expected GDNSTAT1)");
    }
    if (fread(v, sizeof(uint32_t), 9, f) != 9) { fclose(f); return fail(".gdnstate: truncated header"); }
    const GDNWeightHeader &c = s->dm->cfg;
    if (v[0] != 1 || v[1] != c.num_layers || v[2] != c.num_heads || v[3] != c.head_dim || v[4] != c.head_dim ||
        v[5] != c.hidden_size || v[6] != c.conv_size) {
        fclose(f);
        return fail(".gdnstate: dims do not match the loaded model");
    }
    if (fseek(f, (long)v[7] * 4, SEEK_CUR) != 0) { fclose(f); return fail(".gdnstate: cannot skip prompt ids"); }
    const size_t nrec = (size_t)v[1] * v[2] * v[3] * v[4], nconv = (size_t)v[1] * 3 * (v[6] - 1) * v[5];
    std::vector<float> rec(nrec), conv(nconv);
    if (fread(rec.data(), 4, nrec, f) != nrec) { fclose(f); return fail(".gdnstate: truncated recurrent section"); }
    if (fread(conv.data(), 4, nconv, f) != nconv) { fclose(f); return fail(".gdnstate: truncated conv section"); }
    char extra;
    const bool trailing = fread(&extra, 1, 1, f) == 1;
    fclose(f);
    if (trailing) return fail(".gdnstate: unexpected trailing bytes");
    if (seed_token != nullptr) *seed_token = (int32_t)v[8];
    return gdn_b200_state_upload(state, rec.data(), nrec, conv.data(), nconv);
}

int gdn_b200_state_save_file(GDNRunState *state, const char *path, int32_t seed_token) {
    Stream *s = find_stream(state);
    if (s == nullptr) return fail("gdn_b200: unknown run state");
    const GDNWeightHeader &c = s->dm->cfg;
    const size_t nrec = (size_t)c.num_layers * c.num_heads * 256 * 256, nconv = (size_t)c.num_layers * 3 * 3 * c.hidden_size;
    std::vector<float> rec(nrec), conv(nconv);
    if (gdn_b200_state_download(state, rec.data(), nrec, conv.data(), nconv) != 0) return -1;
    FILE *f = fopen(path, "wb");
    if (f == nullptr) return fail("cannot create %s", path);
    const uint32_t v[9] = {1, c.num_layers, c.num_heads, c.head_dim, c.head_dim, c.hidden_size, c.conv_size, 0,
                           (uint32_t)seed_token};
    bool ok = fwrite("GDNSTAT1", 1, 8, f) == 8 && fwrite(v, 4, 9, f) == 9 && fwrite(rec.data(), 4, nrec, f) == nrec &&
              fwrite(conv.data(), 4, nconv, f) == nconv;
    fclose(f);
    return ok ? 0 : fail("write failed: %s", path);
}

void gdn_compute_logits(const GDNModel *model, const float *hidden, float *logits_out) {
    const uint32_t V = model->config.vocab_size, H = model->config.hidden_size;
    std::vector<uint16_t> act(H);
    for (uint32_t i = 0; i < H; ++i) act[i] = bf16_rne_bits(hidden[i]);
    parallel_for(V, [&](size_t b, size_t e) {
        for (size_t v = b; v < e; ++v) {
            const float *row = model->lm_head + v * H;
            float sum = 0.0f;
            for (uint32_t i = 0; i < H; ++i) sum += u2f(native_product_bits(hi16(row[i]), act[i]));
            logits_out[v] = sum;
        }
    });
}

float gdn_native_bf16_mul_to_fp32(uint16_t weight, uint16_t activation) {
    return u2f(native_product_bits(weight, activation));
}

void gdn_set_native_debug_buffers(float *final_hidden, float *logits) {
    g_debug_hidden = final_hidden;
    g_debug_logits = logits;
}

void gdn_reset_mixed_mul_stats(void) {}

GDNMixedMulStats gdn_get_mixed_mul_stats(void) {
    GDNMixedMulStats s;
    memset(&s, 0, sizeof(s));
    return s;
}

}  // extern "C"
