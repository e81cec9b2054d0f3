/* gdn_batch_host.cu -- C ABI of the multi-stream decode engine
 * (include/gdn_b200.h, "multi-stream decode"): the tensor-core tile image of a
 * model, the batch object (B streams' states and the step's buffers), the
 * captured step graph, and the state transfers.
 *
 * A step advances every stream by one token: the per-layer kernel sequence of
 * gdn_batch.cu, captured once into a CUDA graph and replayed (the kernels read
 * the step index from a device counter, so one graph serves every step).
 * Streams are handled in passes of up to 80 (the tile GEMM's N is three
 * BF16 terms x streams <= 256); each
 * projection is one GEMM launch per pass.
 */
#include "gdn_batch.h"

#include "../../include/gdn_b200.h"
#include "../../include/gdn_model.h"

#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

namespace gdn {
int host_fail(const char *msg);
int host_device();
int host_state_begin(GDNRunState *state, float **S, float **tails, int *device, cudaStream_t *stream);
int host_state_end(GDNRunState *state, float *S, bool write_back);
}  // namespace gdn

using namespace gdn::bt;

namespace {

int bfail(const char *fmt, ...) __attribute__((format(printf, 1, 2)));
int bfail(const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    return gdn::host_fail(buf);
}

#define BT_OK(call)                                                                                \
    do {                                                                                           \
        cudaError_t e_ = (call);                                                                   \
        if (e_ != cudaSuccess) return bfail("gdn_b200 batch: %s failed: %s", #call, cudaGetErrorString(e_)); \
    } while (0)

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

inline uint16_t hi16(float v) {
    uint32_t b;
    memcpy(&b, &v, 4);
    return (uint16_t)(b >> 16);
}

/* ------------------------------------------------------------ tile image */

struct Matrix {
    uint32_t m, k;
    size_t off;  /* bytes from the image base */
    uint32_t mtiles() const { return (m + kTileM - 1) / kTileM; }
    uint32_t kblocks() const { return k / kTileK; }
    size_t bytes() const { return (size_t)mtiles() * kblocks() * kABlockBytes; }
};

struct TileModel {
    int device = 0;
    int refs = 0;
    GDNWeightHeader cfg;
    uint8_t *img = nullptr;  /* per layer: QKVGAB | O | GU | DOWN, then the LM head */
    size_t layer_bytes = 0;
    Matrix qkv, o, gu, down, lm;
    uint16_t *emb = nullptr;
    float *aux = nullptr;
    size_t aux_stride = 0;
};

std::mutex g_bmu;
std::map<std::pair<const float *, int>, TileModel *> g_tile_models;

void free_tile_model(TileModel *tm) {
    cudaFree(tm->img);
    cudaFree(tm->emb);
    cudaFree(tm->aux);
    delete tm;
}

/* Row r of a matrix as BF16-exact FP32 words; nullptr = zero row. */
using RowFn = const float *(*)(const GDNModel *, uint32_t layer, uint32_t r);

const float *row_qkv(const GDNModel *m, uint32_t l, uint32_t r) {
    const GDNLayerWeights &w = m->layers[l];
    const uint32_t H = m->config.hidden_size, nh = m->config.num_heads;
    if (r < H) return w.q_proj + (size_t)r * H;
    if (r < 2 * H) return w.k_proj + (size_t)(r - H) * H;
    if (r < 3 * H) return w.v_proj + (size_t)(r - 2 * H) * H;
    if (r < 4 * H) return w.g_proj + (size_t)(r - 3 * H) * H;
    if (r < 4 * H + nh) return w.a_proj + (size_t)(r - 4 * H) * H;
    if (r < 4 * H + 2 * nh) return w.b_proj + (size_t)(r - 4 * H - nh) * H;
    return nullptr;
}
const float *row_o(const GDNModel *m, uint32_t l, uint32_t r) {
    return m->layers[l].o_proj + (size_t)r * m->config.hidden_size;
}
const float *row_gu(const GDNModel *m, uint32_t l, uint32_t r) {
    const GDNLayerWeights &w = m->layers[l];
    return ((r & 1) ? w.mlp_up_proj : w.mlp_gate_proj) + (size_t)(r >> 1) * m->config.hidden_size;
}
const float *row_down(const GDNModel *m, uint32_t l, uint32_t r) {
    return m->layers[l].mlp_down_proj + (size_t)r * m->config.intermediate_size;
}
const float *row_lm(const GDNModel *m, uint32_t, uint32_t r) {
    return r < m->config.vocab_size ? m->lm_head + (size_t)r * m->config.hidden_size : nullptr;
}

/* One 16 KB block (tile mt, k-block kb): row r at r*128 bytes, its 16-byte
 * chunk c at chunk position c ^ (r & 7). */
void fill_block(uint8_t *dst, const GDNModel *model, uint32_t layer, RowFn rowf, const Matrix &mx, uint32_t mt,
                uint32_t kb) {
    uint16_t *d = reinterpret_cast<uint16_t *>(dst);
    for (uint32_t r = 0; r < (uint32_t)kTileM; ++r) {
        const uint32_t row = mt * kTileM + r;
        const float *src = row < mx.m ? rowf(model, layer, row) : nullptr;
        for (uint32_t c = 0; c < 8; ++c) {
            uint16_t *chunk = d + r * 64 + ((c ^ (r & 7)) * 8);
            for (uint32_t e = 0; e < 8; ++e) chunk[e] = src ? hi16(src[kb * 64 + c * 8 + e]) : (uint16_t)0;
        }
    }
}

int upload_matrix(uint8_t *dev, const GDNModel *model, uint32_t layer, RowFn rowf, const Matrix &mx,
                  std::vector<uint8_t> &stage) {
    const uint32_t MT = mx.mtiles(), KB = mx.kblocks();
    const size_t blocks = (size_t)MT * KB;
    const size_t per_pass = stage.size() / kABlockBytes;
    for (size_t b0 = 0; b0 < blocks; b0 += per_pass) {
        const size_t b1 = std::min(blocks, b0 + per_pass);
        parallel_for(b1 - b0, [&](size_t lo, size_t hi) {
            for (size_t i = lo; i < hi; ++i) {
                const size_t b = b0 + i;
                fill_block(stage.data() + i * kABlockBytes, model, layer, rowf, mx, (uint32_t)(b / KB),
                           (uint32_t)(b % KB));
            }
        });
        BT_OK(cudaMemcpy(dev + b0 * kABlockBytes, stage.data(), (b1 - b0) * kABlockBytes, cudaMemcpyHostToDevice));
    }
    return 0;
}

TileModel *build_tile_model(const GDNModel *model) {
    const GDNWeightHeader &c = model->config;
    const uint32_t H = c.hidden_size, nh = c.num_heads, I = c.intermediate_size, V = c.vocab_size, L = c.num_layers;
    TileModel *tm = new TileModel();
    tm->cfg = c;
    tm->device = gdn::host_device();
    tm->qkv = {4 * H + 2 * nh, H, 0};
    tm->o = {H, H, tm->qkv.bytes()};
    tm->gu = {2 * I, H, tm->o.off + tm->o.bytes()};
    tm->down = {H, I, tm->gu.off + tm->gu.bytes()};
    tm->layer_bytes = tm->down.off + tm->down.bytes();
    tm->lm = {V, H, tm->layer_bytes * L};
    tm->aux_stride = ((size_t)14 * H + 256 + 2 * nh + 3) & ~(size_t)3;
    const size_t img_bytes = tm->lm.off + tm->lm.bytes();
    if (cudaMalloc(&tm->img, img_bytes) != cudaSuccess || cudaMalloc(&tm->emb, (size_t)V * H * 2) != cudaSuccess ||
        cudaMalloc(&tm->aux, (tm->aux_stride * L + H) * sizeof(float)) != cudaSuccess) {
        bfail("gdn_b200 batch: tile image allocation failed (%.2f GB)", (double)img_bytes / 1e9);
        free_tile_model(tm);
        return nullptr;
    }
    std::vector<uint8_t> stage((size_t)4096 * kABlockBytes);
    for (uint32_t l = 0; l < L; ++l) {
        uint8_t *base = tm->img + (size_t)l * tm->layer_bytes;
        if (upload_matrix(base + tm->qkv.off, model, l, row_qkv, tm->qkv, stage) ||
            upload_matrix(base + tm->o.off, model, l, row_o, tm->o, stage) ||
            upload_matrix(base + tm->gu.off, model, l, row_gu, tm->gu, stage) ||
            upload_matrix(base + tm->down.off, model, l, row_down, tm->down, stage)) {
            free_tile_model(tm);
            return nullptr;
        }
    }
    if (upload_matrix(tm->img + tm->lm.off, model, 0, row_lm, tm->lm, stage)) {
        free_tile_model(tm);
        return nullptr;
    }
    std::vector<uint16_t> emb((size_t)V * H);
    parallel_for(emb.size(), [&](size_t b, size_t e) {
        for (size_t i = b; i < e; ++i) emb[i] = hi16(model->embeddings[i]);
    });
    std::vector<float> aux(tm->aux_stride * L + H, 0.0f);
    for (uint32_t l = 0; l < L; ++l) {
        const GDNLayerWeights &w = model->layers[l];
        float *a = aux.data() + l * tm->aux_stride;
        memcpy(a, w.attn_norm, H * 4);
        memcpy(a + H, w.o_norm, 256 * 4);
        memcpy(a + H + 256, w.mlp_norm, H * 4);
        memcpy(a + 2 * H + 256, w.q_conv, (size_t)H * 4 * 4);
        memcpy(a + 6 * H + 256, w.k_conv, (size_t)H * 4 * 4);
        memcpy(a + 10 * H + 256, w.v_conv, (size_t)H * 4 * 4);
        memcpy(a + 14 * H + 256, w.a_log, nh * 4);
        memcpy(a + 14 * H + 256 + nh, w.dt_bias, nh * 4);
    }
    memcpy(aux.data() + tm->aux_stride * L, model->final_norm, H * 4);
    if (cudaMemcpy(tm->emb, emb.data(), emb.size() * 2, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(tm->aux, aux.data(), aux.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess) {
        bfail("gdn_b200 batch: embedding/aux upload failed");
        free_tile_model(tm);
        return nullptr;
    }
    return tm;
}

}  // namespace

/* ------------------------------------------------------------- the batch */

struct GdnB200Batch {
    TileModel *tm = nullptr;
    int device = 0;
    cudaStream_t stream = nullptr;
    uint32_t streams = 0, passes = 0, npad_last = 0, sms = 0;
    uint32_t cap_steps = 0;
    size_t state_stride = 0, tails_stride = 0;
    float *state = nullptr, *tails = nullptr, *resid = nullptr, *attn = nullptr, *logits = nullptr;
    uint8_t *xb = nullptr, *mb = nullptr;
    size_t xb_stride = 0, mb_stride = 0;
    float *partial = nullptr;
    size_t partial_pass = 0;  /* floats per pass */
    float *prep = nullptr;    /* recurrence inputs per (stream, head) */
    uint32_t *status = nullptr, *step = nullptr, *parity = nullptr;
    unsigned long long *keys = nullptr;
    int32_t *tokens = nullptr, *argmax = nullptr;
    int greedy = 0;
    cudaGraphExec_t graph[2] = {nullptr, nullptr};  /* teacher-forced, greedy */
    cudaEvent_t ev0 = nullptr, ev1 = nullptr;
    uint32_t launches_per_step = 0;
};

namespace {

uint32_t pass_npad(const GdnB200Batch *b, uint32_t pass) {
    return pass + 1 == b->passes ? b->npad_last : (uint32_t)kMaxPassStreams;
}
StepParams step_params(const GdnB200Batch *b, int greedy) {
    const GDNWeightHeader &c = b->tm->cfg;
    StepParams p;
    memset(&p, 0, sizeof(p));
    p.streams = b->streams;
    p.hidden = c.hidden_size;
    p.heads = c.num_heads;
    p.inter = c.intermediate_size;
    p.vocab = c.vocab_size;
    p.layers = c.num_layers;
    p.eps = c.norm_eps;
    p.emb = b->tm->emb;
    p.aux = b->tm->aux;
    p.aux_stride = b->tm->aux_stride;
    p.tokens = b->tokens;
    p.step = b->step;
    p.argmax_out = b->argmax;
    p.greedy = greedy;
    p.resid = b->resid;
    p.attn = b->attn;
    p.state = b->state;
    p.state_stride = b->state_stride;
    p.tails = b->tails;
    p.tails_stride = b->tails_stride;
    p.tails_buf = (size_t)b->streams * b->tails_stride;
    p.tails_parity = b->parity;
    p.logits = b->logits;
    p.keys = b->keys;
    p.status = b->status;
    return p;
}

/* One projection over every pass; *view describes where its partial sums are. */
int gemm_all(GdnB200Batch *b, const Matrix &mx, const uint8_t *a, const uint8_t *bt, size_t bt_stride, Partials *view,
             uint32_t *launches) {
    const uint32_t grid = gemm_grid(mx.mtiles(), mx.kblocks(), b->sms);
    const uint32_t max_local = gemm_max_local(mx.mtiles(), mx.kblocks(), grid);
    for (uint32_t ps = 0; ps < b->passes; ++ps) {
        GemmParams p;
        memset(&p, 0, sizeof(p));
        p.a = a;
        p.b = bt + ps * bt_stride;
        p.kblocks = mx.kblocks();
        p.mtiles = mx.mtiles();
        p.npad = pass_npad(b, ps);
        gemm_slots(p.npad, &p.a_slots, &p.b_slots);
        p.partial = b->partial + ps * b->partial_pass;
        p.max_local = max_local;
        p.status = b->status;
        BT_OK(launch_gemm(p, grid, b->stream));
        ++*launches;
    }
    view->base = b->partial;
    view->pass_stride = b->partial_pass;
    view->units = mx.mtiles() * mx.kblocks();
    view->grid = grid;
    view->kblocks = mx.kblocks();
    view->max_local = max_local;
    view->npad_last = b->npad_last;
    view->passes = b->passes;
    return 0;
}

int enqueue_step(GdnB200Batch *b, int greedy, uint32_t *launches) {
    const GDNWeightHeader &c = b->tm->cfg;
    const uint32_t L = c.num_layers, H = c.hidden_size;
    const StepParams sp = step_params(b, greedy);
    const TileOut xo = {b->xb, b->xb_stride, b->npad_last, b->passes};
    const TileOut mo = {b->mb, b->mb_stride, b->npad_last, b->passes};
    const TileModel *tm = b->tm;
    Partials none, qkv, o, gu, down, lm;
    memset(&none, 0, sizeof(none));
    *launches = 0;
    BT_OK(launch_input(sp, tm->aux, 0, none, xo, b->stream));
    ++*launches;
    for (uint32_t l = 0; l < L; ++l) {
        const uint8_t *w = tm->img + (size_t)l * tm->layer_bytes;
        const float *aux = tm->aux + (size_t)l * tm->aux_stride;
        if (gemm_all(b, tm->qkv, w + tm->qkv.off, b->xb, b->xb_stride, &qkv, launches)) return -1;
        BT_OK(launch_head(sp, l, qkv, xo, b->stream));
        ++*launches;
        if (gemm_all(b, tm->o, w + tm->o.off, b->xb, b->xb_stride, &o, launches)) return -1;
        BT_OK(launch_input(sp, aux + H + 256, 1, o, xo, b->stream));
        ++*launches;
        if (gemm_all(b, tm->gu, w + tm->gu.off, b->xb, b->xb_stride, &gu, launches)) return -1;
        BT_OK(launch_swiglu(sp, gu, mo, b->stream));
        ++*launches;
        if (gemm_all(b, tm->down, w + tm->down.off, b->mb, b->mb_stride, &down, launches)) return -1;
        const float *next_norm = l + 1 < L ? tm->aux + (size_t)(l + 1) * tm->aux_stride : tm->aux + tm->aux_stride * L;
        BT_OK(launch_input(sp, next_norm, 1, down, xo, b->stream));
        ++*launches;
    }
    if (gemm_all(b, tm->lm, tm->img + tm->lm.off, b->xb, b->xb_stride, &lm, launches)) return -1;
    BT_OK(launch_logits(sp, lm, b->stream));
    BT_OK(launch_finish(sp, b->stream));
    *launches += 2;
    return 0;
}

int capture(GdnB200Batch *b, int greedy) {
    cudaGraph_t g = nullptr;
    uint32_t launches = 0;
    BT_OK(cudaStreamBeginCapture(b->stream, cudaStreamCaptureModeThreadLocal));
    const int rc = enqueue_step(b, greedy, &launches);
    const cudaError_t e = cudaStreamEndCapture(b->stream, &g);
    if (rc != 0) {
        if (g) cudaGraphDestroy(g);
        return -1;
    }
    BT_OK(e);
    const cudaError_t ie = cudaGraphInstantiate(&b->graph[greedy], g, 0);
    cudaGraphDestroy(g);
    BT_OK(ie);
    b->launches_per_step = launches;
    return 0;
}

int check_status(GdnB200Batch *b) {
    uint32_t st[2] = {0, 0};
    BT_OK(cudaMemcpyAsync(st, b->status, sizeof(st), cudaMemcpyDeviceToHost, b->stream));
    BT_OK(cudaStreamSynchronize(b->stream));
    if (st[0] != kErrNone) {
        static const char *names[] = {"none", "weight-block wait timeout", "activation-block wait timeout",
                                      "MMA operand wait timeout", "accumulator wait timeout", "drain timeout",
                                      "token out of range"};
        const char *nm = st[0] < sizeof(names) / sizeof(names[0]) ? names[st[0]] : "unknown";
        /* a failed step can leave argmax keys mid-count */
        cudaMemsetAsync(b->status, 0, 2 * sizeof(uint32_t), b->stream);
        cudaMemsetAsync(b->keys, 0, (size_t)b->streams * 8, b->stream);
        cudaStreamSynchronize(b->stream);
        return bfail("gdn_b200 batch: step failed on the device: %s (at %u)", nm, st[1]);
    }
    return 0;
}

void free_batch(GdnB200Batch *b) {
    cudaSetDevice(b->device);
    if (b->stream) cudaStreamSynchronize(b->stream);
    for (auto &g : b->graph)
        if (g) cudaGraphExecDestroy(g);
    if (b->ev0) cudaEventDestroy(b->ev0);
    if (b->ev1) cudaEventDestroy(b->ev1);
    void *ptrs[] = {b->state, b->tails, b->resid, b->attn, b->logits, b->xb, b->mb, b->prep,
                    b->partial, b->status, b->step, b->parity, b->keys, b->tokens, b->argmax};
    for (void *p : ptrs) cudaFree(p);
    if (b->stream) cudaStreamDestroy(b->stream);
    if (b->tm) {
        std::lock_guard<std::mutex> lk(g_bmu);
        if (--b->tm->refs == 0) {
            for (auto it = g_tile_models.begin(); it != g_tile_models.end(); ++it)
                if (it->second == b->tm) {
                    g_tile_models.erase(it);
                    break;
                }
            free_tile_model(b->tm);
        }
    }
    delete b;
}

/* The tile image of a model on a device, built on first use; one reference taken. */
TileModel *acquire_tile_model(const GDNModel *model, int device) {
    std::lock_guard<std::mutex> lk(g_bmu);
    auto key = std::make_pair((const float *)model->weight_data, device);
    auto it = g_tile_models.find(key);
    if (it == g_tile_models.end()) {
        TileModel *tm = build_tile_model(model);
        if (tm == nullptr) return nullptr;
        it = g_tile_models.emplace(key, tm).first;
    }
    ++it->second->refs;
    return it->second;
}

int batch_supports(const GDNWeightHeader &c, uint32_t streams) {
    if (streams == 0 || streams > 1024) return bfail("gdn_b200 batch: streams must be 1..1024 (got %u)", streams);
    if (c.head_dim != 256 || c.conv_size != 4 || c.hidden_size != c.num_heads * 256)
        return bfail("gdn_b200 batch: needs head_dim 256, conv 4, hidden = heads x 256");
    if (c.hidden_size % 512 || c.intermediate_size % 64 || c.hidden_size > 4096)
        return bfail("gdn_b200 batch: hidden must be a multiple of 512 (<= 4096), intermediate of 64");
    return 0;
}

}  // namespace

extern "C" {

GdnB200Batch *gdn_b200_batch_create(const GDNModel *model, uint32_t streams) {
    if (model == nullptr || model->weight_data == nullptr) {
        bfail("gdn_b200 batch: no model");
        return nullptr;
    }
    const GDNWeightHeader &c = model->config;
    if (batch_supports(c, streams) != 0) return nullptr;
    GdnB200Batch *b = new GdnB200Batch();
    b->device = gdn::host_device();
    if (cudaSetDevice(b->device) != cudaSuccess) {
        bfail("gdn_b200 batch: cannot select device %d", b->device);
        delete b;
        return nullptr;
    }
    b->tm = acquire_tile_model(model, b->device);
    if (b->tm == nullptr) {
        delete b;
        return nullptr;
    }
    const uint32_t H = c.hidden_size, nh = c.num_heads, I = c.intermediate_size, V = c.vocab_size, L = c.num_layers;
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, b->device);
    b->sms = (uint32_t)sms;
    b->streams = streams;
    b->passes = (streams + kMaxPassStreams - 1) / kMaxPassStreams;
    const uint32_t last = streams - (b->passes - 1) * kMaxPassStreams;
    b->npad_last = (last + 15) / 16 * 16;
    b->cap_steps = 4096;
    b->state_stride = (size_t)L * nh * 256 * 256;
    b->tails_stride = (size_t)L * 9 * H;
    b->xb_stride = tile_pass_bytes(kMaxPassStreams, H);
    b->mb_stride = tile_pass_bytes(kMaxPassStreams, I);
    /* partial slots: the largest grid x slots of any projection, 80 streams x 128 rows each, per pass */
    const TileModel *tm = b->tm;
    size_t slots = 0;
    for (const Matrix *mx : {&tm->qkv, &tm->o, &tm->gu, &tm->down, &tm->lm}) {
        const uint32_t g = gemm_grid(mx->mtiles(), mx->kblocks(), b->sms);
        slots = std::max<size_t>(slots, (size_t)g * gemm_max_local(mx->mtiles(), mx->kblocks(), g));
    }
    b->partial_pass = slots * kMaxPassStreams * kTileM;
    const size_t S = streams;
    bool ok = cudaStreamCreateWithFlags(&b->stream, cudaStreamNonBlocking) == cudaSuccess &&
              cudaEventCreate(&b->ev0) == cudaSuccess && cudaEventCreate(&b->ev1) == cudaSuccess &&
              cudaMalloc(&b->state, S * b->state_stride * 4) == cudaSuccess &&
              cudaMalloc(&b->tails, 2 * S * b->tails_stride * 4) == cudaSuccess &&
              cudaMalloc(&b->resid, S * H * 4) == cudaSuccess &&
              cudaMalloc(&b->attn, S * H * 4) == cudaSuccess && cudaMalloc(&b->logits, S * V * 4) == cudaSuccess &&
              cudaMalloc(&b->prep, prep_floats(streams, c.num_heads) * 4) == cudaSuccess &&
              cudaMalloc(&b->xb, b->passes * b->xb_stride) == cudaSuccess &&
              cudaMalloc(&b->mb, b->passes * b->mb_stride) == cudaSuccess &&
              cudaMalloc(&b->partial, b->passes * b->partial_pass * 4) == cudaSuccess &&
              cudaMalloc(&b->status, 2 * 4) == cudaSuccess && cudaMalloc(&b->step, 4) == cudaSuccess &&
              cudaMalloc(&b->parity, 4) == cudaSuccess && cudaMalloc(&b->keys, S * 8) == cudaSuccess &&
              cudaMalloc(&b->tokens, (size_t)b->cap_steps * S * 4) == cudaSuccess &&
              cudaMalloc(&b->argmax, (size_t)b->cap_steps * S * 4) == cudaSuccess;
    if (!ok) {
        bfail("gdn_b200 batch: allocation for %u streams failed (%.2f GB of state)", streams,
              (double)(S * b->state_stride * 4) / 1e9);
        free_batch(b);
        return nullptr;
    }
    ok = cudaMemsetAsync(b->state, 0, S * b->state_stride * 4, b->stream) == cudaSuccess &&
         cudaMemsetAsync(b->tails, 0, 2 * S * b->tails_stride * 4, b->stream) == cudaSuccess &&
         cudaMemsetAsync(b->xb, 0, b->passes * b->xb_stride, b->stream) == cudaSuccess &&
         cudaMemsetAsync(b->mb, 0, b->passes * b->mb_stride, b->stream) == cudaSuccess &&
         cudaMemsetAsync(b->status, 0, 8, b->stream) == cudaSuccess &&
         cudaMemsetAsync(b->keys, 0, S * 8, b->stream) == cudaSuccess &&
         cudaMemsetAsync(b->step, 0, 4, b->stream) == cudaSuccess &&
         cudaMemsetAsync(b->parity, 0, 4, b->stream) == cudaSuccess &&
         cudaStreamSynchronize(b->stream) == cudaSuccess;
    if (!ok || capture(b, 0) != 0 || capture(b, 1) != 0) {
        if (!ok) bfail("gdn_b200 batch: buffer initialisation failed");
        free_batch(b);
        return nullptr;
    }
    return b;
}

void gdn_b200_batch_free(GdnB200Batch *batch) {
    if (batch) free_batch(batch);
}

uint32_t gdn_b200_batch_launches_per_step(const GdnB200Batch *batch) { return batch ? batch->launches_per_step : 0; }

int gdn_b200_batch_reset(GdnB200Batch *b) {
    if (b == nullptr) return bfail("gdn_b200 batch: null batch");
    BT_OK(cudaSetDevice(b->device));
    BT_OK(cudaMemsetAsync(b->state, 0, (size_t)b->streams * b->state_stride * 4, b->stream));
    BT_OK(cudaMemsetAsync(b->tails, 0, 2 * (size_t)b->streams * b->tails_stride * 4, b->stream));
    BT_OK(cudaStreamSynchronize(b->stream));
    return 0;
}

/* the tail buffer the next step reads */
static int tails_read_buffer(GdnB200Batch *b, float **buf) {
    uint32_t par = 0;
    BT_OK(cudaMemcpyAsync(&par, b->parity, 4, cudaMemcpyDeviceToHost, b->stream));
    BT_OK(cudaStreamSynchronize(b->stream));
    *buf = b->tails + (size_t)(par & 1u) * b->streams * b->tails_stride;
    return 0;
}

int gdn_b200_batch_state_upload(GdnB200Batch *b, uint32_t s, const float *rec, size_t rec_floats, const float *conv,
                                size_t conv_floats) {
    if (b == nullptr || s >= b->streams) return bfail("gdn_b200 batch: bad stream index");
    const GDNWeightHeader &c = b->tm->cfg;
    const size_t L = c.num_layers, nh = c.num_heads, H = c.hidden_size;
    if (rec_floats != L * nh * 256 * 256 || conv_floats != L * 9 * H)
        return bfail("gdn_b200 batch: state sizes do not match the model (rec %zu, conv %zu)", rec_floats, conv_floats);
    /* [L][h][k][v] -> [L][h][v][k]; conv tails keep [L][kind][row][H] */
    std::vector<float> S(rec_floats);
    parallel_for(L * nh, [&](size_t lo, size_t hi) {
        for (size_t lh = lo; lh < hi; ++lh)
            for (size_t k = 0; k < 256; ++k)
                for (size_t v = 0; v < 256; ++v) S[(lh * 256 + v) * 256 + k] = rec[(lh * 256 + k) * 256 + v];
    });
    BT_OK(cudaSetDevice(b->device));
    float *tails = nullptr;
    if (tails_read_buffer(b, &tails) != 0) return -1;
    BT_OK(cudaMemcpyAsync(b->state + s * b->state_stride, S.data(), rec_floats * 4, cudaMemcpyHostToDevice, b->stream));
    BT_OK(cudaMemcpyAsync(tails + s * b->tails_stride, conv, conv_floats * 4, cudaMemcpyHostToDevice, b->stream));
    BT_OK(cudaStreamSynchronize(b->stream));
    return 0;
}

int gdn_b200_batch_state_download(GdnB200Batch *b, uint32_t s, float *rec, size_t rec_floats, float *conv,
                                  size_t conv_floats) {
    if (b == nullptr || s >= b->streams) return bfail("gdn_b200 batch: bad stream index");
    const GDNWeightHeader &c = b->tm->cfg;
    const size_t L = c.num_layers, nh = c.num_heads, H = c.hidden_size;
    if (rec_floats != L * nh * 256 * 256 || conv_floats != L * 9 * H)
        return bfail("gdn_b200 batch: state sizes do not match the model");
    std::vector<float> S(rec_floats);
    BT_OK(cudaSetDevice(b->device));
    float *tails = nullptr;
    if (tails_read_buffer(b, &tails) != 0) return -1;
    BT_OK(cudaMemcpyAsync(S.data(), b->state + s * b->state_stride, rec_floats * 4, cudaMemcpyDeviceToHost, b->stream));
    BT_OK(cudaMemcpyAsync(conv, tails + s * b->tails_stride, conv_floats * 4, cudaMemcpyDeviceToHost, b->stream));
    BT_OK(cudaStreamSynchronize(b->stream));
    parallel_for(L * nh, [&](size_t lo, size_t hi) {
        for (size_t lh = lo; lh < hi; ++lh)
            for (size_t k = 0; k < 256; ++k)
                for (size_t v = 0; v < 256; ++v) rec[(lh * 256 + k) * 256 + v] = S[(lh * 256 + v) * 256 + k];
    });
    return 0;
}

int gdn_b200_batch_step_host(GdnB200Batch *b, const int32_t *tokens, int32_t *argmax, float *logits) {
    if (b == nullptr || tokens == nullptr) return bfail("gdn_b200 batch: null argument");
    const uint32_t V = b->tm->cfg.vocab_size;
    for (uint32_t s = 0; s < b->streams; ++s)
        if (tokens[s] < 0 || (uint32_t)tokens[s] >= V)
            return bfail("gdn_b200 batch: token %d of stream %u out of range", tokens[s], s);
    BT_OK(cudaSetDevice(b->device));
    BT_OK(cudaMemcpyAsync(b->tokens, tokens, (size_t)b->streams * 4, cudaMemcpyHostToDevice, b->stream));
    BT_OK(cudaMemsetAsync(b->step, 0, 4, b->stream));
    BT_OK(cudaGraphLaunch(b->graph[0], b->stream));
    if (argmax) BT_OK(cudaMemcpyAsync(argmax, b->argmax, (size_t)b->streams * 4, cudaMemcpyDeviceToHost, b->stream));
    if (logits)
        BT_OK(cudaMemcpyAsync(logits, b->logits, (size_t)b->streams * V * 4, cudaMemcpyDeviceToHost, b->stream));
    return check_status(b);
}

int gdn_b200_batch_decode_tokens(GdnB200Batch *b, const int32_t *tokens, uint32_t n, int greedy, int32_t *argmax_out,
                                 float *device_ms) {
    if (b == nullptr || tokens == nullptr || n == 0) return bfail("gdn_b200 batch: bad arguments");
    const uint32_t V = b->tm->cfg.vocab_size, S = b->streams;
    const size_t need = greedy ? S : (size_t)n * S;
    for (size_t i = 0; i < need; ++i)
        if (tokens[i] < 0 || (uint32_t)tokens[i] >= V) return bfail("gdn_b200 batch: token %d out of range", tokens[i]);
    BT_OK(cudaSetDevice(b->device));
    float total_ms = 0.0f;
    std::vector<int32_t> carry;
    for (uint32_t s0 = 0; s0 < n; s0 += b->cap_steps) {
        const uint32_t steps = std::min(b->cap_steps, n - s0);
        if (greedy) {
            const int32_t *first = s0 == 0 ? tokens : carry.data();
            BT_OK(cudaMemcpyAsync(b->tokens, first, (size_t)S * 4, cudaMemcpyHostToDevice, b->stream));
        } else {
            BT_OK(cudaMemcpyAsync(b->tokens, tokens + (size_t)s0 * S, (size_t)steps * S * 4, cudaMemcpyHostToDevice,
                                  b->stream));
        }
        BT_OK(cudaMemsetAsync(b->step, 0, 4, b->stream));
        BT_OK(cudaEventRecord(b->ev0, b->stream));
        for (uint32_t i = 0; i < steps; ++i) BT_OK(cudaGraphLaunch(b->graph[greedy ? 1 : 0], b->stream));
        BT_OK(cudaEventRecord(b->ev1, b->stream));
        if (argmax_out)
            BT_OK(cudaMemcpyAsync(argmax_out + (size_t)s0 * S, b->argmax, (size_t)steps * S * 4, cudaMemcpyDeviceToHost,
                                  b->stream));
        if (check_status(b) != 0) return -1;
        float ms = 0.0f;
        BT_OK(cudaEventElapsedTime(&ms, b->ev0, b->ev1));
        total_ms += ms;
        if (greedy) {
            carry.resize(S);
            BT_OK(cudaMemcpy(carry.data(), b->argmax + (size_t)(steps - 1) * S, (size_t)S * 4, cudaMemcpyDeviceToHost));
        }
    }
    if (device_ms) *device_ms = total_ms;
    return 0;
}

int gdn_b200_batch_fetch_logits(GdnB200Batch *b, float *logits) {
    if (b == nullptr || logits == nullptr) return bfail("gdn_b200 batch: null argument");
    BT_OK(cudaSetDevice(b->device));
    BT_OK(cudaMemcpyAsync(logits, b->logits, (size_t)b->streams * b->tm->cfg.vocab_size * 4, cudaMemcpyDeviceToHost,
                          b->stream));
    BT_OK(cudaStreamSynchronize(b->stream));
    return 0;
}


/* Prefill (no reference counterpart in the C ABI; the reference builds prompt
 * state with FLA's chunked kernel, scripts/export_gdn_state.py:157-201): the
 * prompt's tokens, up to 240 at a time, are the "streams" of the tile-GEMM
 * projections, norms and SwiGLU; prefill_head_kernel runs the conv and the
 * recurrence in token order on the run state's own S and tails. FP32
 * contract; the run state ends as if the tokens had been decoded one by one
 * (within FP32 summation-order differences), with no logits computed. */
static int prefill_on(const GDNModel *model, const int32_t *tokens, uint32_t n, float *device_ms, float *S,
                      float *tails, int device, cudaStream_t stream) {
    const GDNWeightHeader &c = model->config;
    if (batch_supports(c, 1) != 0) return -1;
    for (uint32_t i = 0; i < n; ++i)
        if (tokens[i] < 0 || (uint32_t)tokens[i] >= c.vocab_size)
            return bfail("gdn_b200 prefill: token %d at %u out of range", tokens[i], i);
    BT_OK(cudaSetDevice(device));
    /* the tile image stays cached with the model once built */
    TileModel *tm = acquire_tile_model(model, device);
    if (tm == nullptr) return -1;
    const uint32_t H = c.hidden_size, I = c.intermediate_size, L = c.num_layers;
    constexpr uint32_t kChunk = 3 * kMaxPassStreams;
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    size_t slots = 0;
    for (const Matrix *mx : {&tm->qkv, &tm->o, &tm->gu, &tm->down}) {
        const uint32_t g = gemm_grid(mx->mtiles(), mx->kblocks(), (uint32_t)sms);
        slots = std::max<size_t>(slots, (size_t)g * gemm_max_local(mx->mtiles(), mx->kblocks(), g));
    }
    const size_t part_pass = slots * kMaxPassStreams * kTileM;
    const size_t xb_stride = tile_pass_bytes(kMaxPassStreams, H), mb_stride = tile_pass_bytes(kMaxPassStreams, I);
    const size_t tails_floats = (size_t)L * 3 * H * 4;
    float *resid = nullptr, *attn = nullptr, *partial = nullptr, *tails_new = nullptr;
    uint8_t *xb = nullptr, *mb = nullptr;
    int32_t *dtok = nullptr;
    uint32_t *step = nullptr, *status = nullptr;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    int rc = 0;
    auto cleanup = [&]() {
        cudaStreamSynchronize(stream);
        void *ptrs[] = {resid, attn, partial, tails_new, xb, mb, dtok, step, status};
        for (void *q : ptrs) cudaFree(q);
        if (e0) cudaEventDestroy(e0);
        if (e1) cudaEventDestroy(e1);
    };
    if (cudaMalloc(&resid, (size_t)kChunk * H * 4) != cudaSuccess || cudaMalloc(&attn, (size_t)kChunk * H * 4) != cudaSuccess ||
        cudaMalloc(&partial, 3 * part_pass * 4) != cudaSuccess || cudaMalloc(&tails_new, tails_floats * 4) != cudaSuccess ||
        cudaMalloc(&xb, 3 * xb_stride) != cudaSuccess || cudaMalloc(&mb, 3 * mb_stride) != cudaSuccess ||
        cudaMalloc(&dtok, (size_t)kChunk * 4) != cudaSuccess || cudaMalloc(&step, 4) != cudaSuccess ||
        cudaMalloc(&status, 8) != cudaSuccess || cudaEventCreate(&e0) != cudaSuccess || cudaEventCreate(&e1) != cudaSuccess) {
        cleanup();
        return bfail("gdn_b200 prefill: allocation failed");
    }
    cudaMemsetAsync(xb, 0, 3 * xb_stride, stream);
    cudaMemsetAsync(mb, 0, 3 * mb_stride, stream);
    cudaMemsetAsync(step, 0, 4, stream);
    cudaMemsetAsync(status, 0, 8, stream);
    cudaEventRecord(e0, stream);
    for (uint32_t j0 = 0; j0 < n && rc == 0; j0 += kChunk) {
        const uint32_t ntok = std::min(kChunk, n - j0);
        const uint32_t passes = (ntok + kMaxPassStreams - 1) / kMaxPassStreams;
        const uint32_t last = ntok - (passes - 1) * kMaxPassStreams, npad_last = (last + 15) / 16 * 16;
        auto npad_of = [&](uint32_t ps) { return ps + 1 == passes ? npad_last : (uint32_t)kMaxPassStreams; };
        StepParams sp;
        memset(&sp, 0, sizeof(sp));
        sp.streams = ntok;
        sp.hidden = H;
        sp.heads = c.num_heads;
        sp.inter = I;
        sp.vocab = c.vocab_size;
        sp.layers = L;
        sp.eps = c.norm_eps;
        sp.emb = tm->emb;
        sp.aux = tm->aux;
        sp.aux_stride = tm->aux_stride;
        sp.tokens = dtok;
        sp.step = step;
        sp.resid = resid;
        sp.attn = attn;
        sp.status = status;
        const TileOut xo = {xb, xb_stride, npad_last, passes}, mo = {mb, mb_stride, npad_last, passes};
        auto gemm = [&](const Matrix &mx, const uint8_t *a, const uint8_t *bt, size_t bt_stride, Partials *view) -> int {
            const uint32_t grid = gemm_grid(mx.mtiles(), mx.kblocks(), (uint32_t)sms);
            const uint32_t max_local = gemm_max_local(mx.mtiles(), mx.kblocks(), grid);
            for (uint32_t ps = 0; ps < passes; ++ps) {
                GemmParams p;
                memset(&p, 0, sizeof(p));
                p.a = a;
                p.b = bt + ps * bt_stride;
                p.kblocks = mx.kblocks();
                p.mtiles = mx.mtiles();
                p.npad = npad_of(ps);
                gemm_slots(p.npad, &p.a_slots, &p.b_slots);
                p.partial = partial + ps * part_pass;
                p.max_local = max_local;
                p.status = status;
                BT_OK(launch_gemm(p, grid, stream));
            }
            *view = Partials{partial, part_pass, mx.mtiles() * mx.kblocks(), grid, mx.kblocks(), max_local, npad_last,
                             passes};
            return 0;
        };
        if (cudaMemcpyAsync(dtok, tokens + j0, (size_t)ntok * 4, cudaMemcpyHostToDevice, stream) != cudaSuccess) {
            rc = bfail("gdn_b200 prefill: token upload failed");
            break;
        }
        Partials none, qkv, o, gu, down;
        memset(&none, 0, sizeof(none));
        if (launch_input(sp, tm->aux, 0, none, xo, stream) != cudaSuccess) rc = -1;
        for (uint32_t l = 0; l < L && rc == 0; ++l) {
            const uint8_t *w = tm->img + (size_t)l * tm->layer_bytes;
            const float *aux = tm->aux + (size_t)l * tm->aux_stride;
            if (gemm(tm->qkv, w + tm->qkv.off, xb, xb_stride, &qkv) ||
                launch_prefill_head(sp, l, qkv, S, tails, tails_new, ntok, stream) != cudaSuccess ||
                launch_gate_norm(sp, l, qkv, xo, stream) != cudaSuccess ||
                gemm(tm->o, w + tm->o.off, xb, xb_stride, &o) ||
                launch_input(sp, aux + H + 256, 1, o, xo, stream) != cudaSuccess ||
                gemm(tm->gu, w + tm->gu.off, xb, xb_stride, &gu) || launch_swiglu(sp, gu, mo, stream) != cudaSuccess ||
                gemm(tm->down, w + tm->down.off, mb, mb_stride, &down)) {
                rc = -1;
                break;
            }
            if (l + 1 < L && launch_input(sp, tm->aux + (size_t)(l + 1) * tm->aux_stride, 1, down, xo, stream) != cudaSuccess)
                rc = -1;
        }
        if (rc == 0 && cudaMemcpyAsync(tails, tails_new, tails_floats * 4, cudaMemcpyDeviceToDevice, stream) != cudaSuccess)
            rc = bfail("gdn_b200 prefill: tail copy failed");
    }
    if (rc != 0 && gdn_b200_last_error()[0] == 0) bfail("gdn_b200 prefill: launch failed: %s", cudaGetErrorString(cudaGetLastError()));
    cudaEventRecord(e1, stream);
    uint32_t st[2] = {0, 0};
    const cudaError_t se = cudaMemcpyAsync(st, status, 8, cudaMemcpyDeviceToHost, stream);
    const cudaError_t ss = cudaStreamSynchronize(stream);
    if (rc == 0 && (se != cudaSuccess || ss != cudaSuccess))
        rc = bfail("gdn_b200 prefill: %s", cudaGetErrorString(se != cudaSuccess ? se : ss));
    if (rc == 0 && st[0] != 0) rc = bfail("gdn_b200 prefill: device error %u at %u", st[0], st[1]);
    if (rc == 0 && device_ms) cudaEventElapsedTime(device_ms, e0, e1);
    cleanup();
    return rc;
}

/* The run state's recurrent state is converted to natural FP32 for the
 * prefill kernels and written back into its own storage afterwards (rounded
 * to BF16 when the run state keeps the c_impl contract's BF16 state). */
int gdn_b200_prefill(const GDNModel *model, GDNRunState *state, const int32_t *tokens, uint32_t n, float *device_ms) {
    if (model == nullptr || state == nullptr || (tokens == nullptr && n > 0))
        return bfail("gdn_b200 prefill: null argument");
    if (n == 0) {
        if (device_ms) *device_ms = 0.0f;
        return 0;
    }
    float *S = nullptr, *tails = nullptr;
    int device = 0;
    cudaStream_t stream = nullptr;
    if (gdn::host_state_begin(state, &S, &tails, &device, &stream) != 0) return -1;
    const int rc = prefill_on(model, tokens, n, device_ms, S, tails, device, stream);
    const int rc2 = gdn::host_state_end(state, S, rc == 0);
    return rc != 0 ? rc : rc2;
}

/* Test hook: Y[n][m] = sum_k W[m][k] X[n][k] through one tile-GEMM launch
 * (W BF16-exact FP32 words [m][k], X FP32 [n][k] split into three BF16 terms
 * as the engine does; k a multiple of 64, n <= 80). */
int gdn_b200_test_tile_gemm(uint32_t m, uint32_t k, uint32_t n, const float *w, const float *x, float *y) {
    if (m == 0 || k == 0 || k % kTileK || n == 0 || n > (uint32_t)kMaxPassStreams || !w || !x || !y)
        return bfail("gdn_b200 batch: bad tile-GEMM test shape");
    BT_OK(cudaSetDevice(gdn::host_device()));
    int sms = 0;
    BT_OK(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, gdn::host_device()));
    const Matrix mx = {m, k, 0};
    const uint32_t npad = (n + 15) / 16 * 16;
    std::vector<uint8_t> img(mx.bytes(), 0);
    for (uint32_t b = 0; b < mx.mtiles() * mx.kblocks(); ++b) {
        const uint32_t mt = b / mx.kblocks(), kb = b % mx.kblocks();
        uint16_t *d = reinterpret_cast<uint16_t *>(img.data() + (size_t)b * kABlockBytes);
        for (uint32_t r = 0; r < (uint32_t)kTileM; ++r) {
            const uint32_t row = mt * kTileM + r;
            if (row >= m) continue;
            for (uint32_t c = 0; c < 8; ++c)
                for (uint32_t e = 0; e < 8; ++e)
                    d[r * 64 + ((c ^ (r & 7)) * 8) + e] = hi16(w[(size_t)row * k + kb * 64 + c * 8 + e]);
        }
    }
    auto rne = [](float v) -> uint16_t {
        uint32_t bits;
        memcpy(&bits, &v, 4);
        return (uint16_t)((bits + 0x7FFFu + ((bits >> 16) & 1u)) >> 16);
    };
    auto widen = [](uint16_t h) -> float {
        const uint32_t bits = (uint32_t)h << 16;
        float v;
        memcpy(&v, &bits, 4);
        return v;
    };
    std::vector<uint8_t> act(tile_pass_bytes(npad, k), 0);
    for (uint32_t s = 0; s < n; ++s)
        for (uint32_t kk = 0; kk < k; ++kk) {
            const float v = x[(size_t)s * k + kk];
            const uint16_t h0 = rne(v);
            const float r1 = v - widen(h0);
            const uint16_t h1 = rne(r1);
            const float r2 = r1 - widen(h1);
            const uint16_t h2 = rne(r2);
            const uint16_t hs[3] = {h0, h1, h2};
            const uint32_t kb = kk >> 6, k6 = kk & 63;
            for (int t = 0; t < kTerms; ++t) {
                const size_t off = (size_t)kb * kTerms * npad * 128 + (size_t)t * npad * 128 + (size_t)s * 128 +
                                   ((((k6 >> 3) ^ (s & 7)) << 4) | ((k6 & 7) << 1));
                memcpy(act.data() + off, &hs[t], 2);
            }
        }
    const uint32_t grid = gemm_grid(mx.mtiles(), mx.kblocks(), (uint32_t)sms);
    const uint32_t max_local = gemm_max_local(mx.mtiles(), mx.kblocks(), grid);
    const size_t part_floats = (size_t)grid * max_local * npad * kTileM;
    uint8_t *d_img = nullptr, *d_act = nullptr;
    float *d_part = nullptr;
    uint32_t *d_status = nullptr;
    int rc = 0;
    if (cudaMalloc(&d_img, img.size()) != cudaSuccess || cudaMalloc(&d_act, act.size()) != cudaSuccess ||
        cudaMalloc(&d_part, part_floats * 4) != cudaSuccess || cudaMalloc(&d_status, 8) != cudaSuccess) {
        rc = bfail("gdn_b200 batch: test allocation failed");
    } else {
        cudaMemcpy(d_img, img.data(), img.size(), cudaMemcpyHostToDevice);
        cudaMemcpy(d_act, act.data(), act.size(), cudaMemcpyHostToDevice);
        cudaMemset(d_status, 0, 8);
        GemmParams p;
        memset(&p, 0, sizeof(p));
        p.a = d_img;
        p.b = d_act;
        p.kblocks = mx.kblocks();
        p.mtiles = mx.mtiles();
        p.npad = npad;
        gemm_slots(npad, &p.a_slots, &p.b_slots);
        p.partial = d_part;
        p.max_local = max_local;
        p.status = d_status;
        std::vector<float> part(part_floats);
        cudaError_t e = launch_gemm(p, grid, nullptr);
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
        uint32_t st[2] = {0, 0};
        if (e == cudaSuccess) e = cudaMemcpy(st, d_status, 8, cudaMemcpyDeviceToHost);
        if (e == cudaSuccess) e = cudaMemcpy(part.data(), d_part, part_floats * 4, cudaMemcpyDeviceToHost);
        if (e != cudaSuccess) rc = bfail("gdn_b200 batch: test GEMM failed: %s", cudaGetErrorString(e));
        else if (st[0] != 0) rc = bfail("gdn_b200 batch: test GEMM reported error %u at CTA %u", st[0], st[1]);
        else {
            /* the consumers' sum: segments of a tile in k order */
            const uint32_t units = mx.mtiles() * mx.kblocks(), KB = mx.kblocks();
            for (uint32_t row = 0; row < m; ++row) {
                const uint32_t t = row / kTileM, r = row % kTileM;
                const uint32_t cf = unit_owner(t * KB, units, grid), cl = unit_owner(t * KB + KB - 1, units, grid);
                for (uint32_t s = 0; s < n; ++s) {
                    float acc = 0.0f;
                    for (uint32_t cc = cf; cc <= cl; ++cc) {
                        const uint32_t lc = t - unit_start(cc, units, grid) / KB;
                        const float v = part[((size_t)cc * max_local + lc) * npad * kTileM + (size_t)s * kTileM + r];
                        acc = cc == cf ? v : acc + v;
                    }
                    y[(size_t)s * m + row] = acc;
                }
            }
        }
    }
    cudaFree(d_img);
    cudaFree(d_act);
    cudaFree(d_part);
    cudaFree(d_status);
    return rc;
}

}  // extern "C"
