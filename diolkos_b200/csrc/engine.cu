// engine.cu -- the decode engine behind dk_model_* (include/diolkos.h).
//
// One dk_model holds a LLaMA-2 model (or one tensor-parallel shard of it) in HBM:
//   * packed Q8_0 weights in one allocation: per layer the fused [wq; wk; wv] matrix, wo, the
//     row-interleaved [w1_0; w3_0; w1_1; w3_1; ...] matrix (so SwiGLU pairs arrive together) and
//     w2; the embedding table and lm_head; fp32 norm weights;
//   * the KV cache, [layer][kv_head][seq_len][head_size], bf16 (truncating, like the reference) or
//     fp32;
//   * activations, the RoPE (cos, sin) table, the token buffer and the current position.
// The per-token step (reference forward, src/transformer.c:55-239) is 5 kernels per layer plus
// the classifier, launched with programmatic dependent launch and captured once into a CUDA
// graph; `pos` and the tokens live in device memory, so the same graph serves every position and
// greedy decoding replays it back to back without the host in the loop.
#include <cmath>
#include <cstdlib>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <vector>

#include "dk_internal.h"

namespace dk {

int *device_error_word() {
    static std::mutex mu;
    static int *words[64] = {nullptr};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lk(mu);
    if (!words[dev]) {
        int *p = nullptr;
        if (cudaMalloc(&p, sizeof(int)) != cudaSuccess) return nullptr;
        if (cudaMemset(p, 0, sizeof(int)) != cudaSuccess) return nullptr;
        words[dev] = p;
    }
    return words[dev];
}

// HF rotate-half RoPE coefficients (src/transformer.c:90-95): for position p and j < hs/2,
// freq = 1/powf(10000, 2j/(float)hs), val = p*freq, (cosf(val), sinf(val)).  Computed on the host
// with the C library's single-precision functions and uploaded once.
static void rope_table(std::vector<float> &t, int seq_len, int hs) {
    t.resize((size_t)seq_len * hs);
    for (int p = 0; p < seq_len; ++p)
        for (int j = 0; j < hs / 2; ++j) {
            const float freq = 1.0f / powf(10000.0f, (float)(2 * j) / (float)hs);
            const float val = (float)p * freq;
            t[(size_t)p * hs + 2 * j] = cosf(val);
            t[(size_t)p * hs + 2 * j + 1] = sinf(val);
        }
}

}  // namespace dk

using namespace dk;

struct dk_layer {
    uint8_t *wqkv = nullptr, *wo = nullptr, *w13 = nullptr, *w2 = nullptr;
    float *rms_att = nullptr, *rms_ffn = nullptr;
};

struct dk_model {
    // global config
    int dim, hidden, n_layers, n_heads, n_kv_heads, vocab, seq_len, kv_type, device, rank, world;
    int hs, kv_dim;
    // this rank's shard: heads [rank*l_heads, ...), hidden rows [rank*l_hidden, ...), classifier rows
    // [vocab_off, vocab_off + l_vocab); l_dim / l_kv_dim = its q / k columns of the attention
    int l_heads, l_kv_heads, l_hidden, l_dim, l_kv_dim, l_vocab, vocab_off;
    int num_sms;
    cudaStream_t stream = nullptr;
    // weights
    uint8_t *warena = nullptr;
    size_t warena_bytes = 0;
    uint8_t *emb = nullptr, *wcls = nullptr;
    float *rms_final = nullptr;
    std::vector<dk_layer> layers;
    std::vector<uint8_t> have;  // [(n_layers + 1) * DK_W_COUNT]
    // activations and state
    uint8_t *aarena = nullptr;
    float *x = nullptr, *qkv = nullptr, *xb = nullptr, *hb = nullptr, *logits = nullptr, *rope = nullptr;
    float *attn_work = nullptr;
    unsigned *attn_count = nullptr;
    unsigned long long *amax_part = nullptr;
    unsigned *amax_count = nullptr;
    int *tokens = nullptr, *pos = nullptr, *n_forced = nullptr, *err = nullptr;
    void *kcache = nullptr, *vcache = nullptr;
    size_t kv_layer_elems = 0;
    int attn_splits = 1;
    // staging for weight upload
    uint8_t *stage = nullptr;
    size_t stage_bytes = 0;
    // pinned host scratch
    int *h_small = nullptr;
    // plans
    GemvPlan p_qkv, p_wo, p_w13, p_w2, p_cls;
    int emb_T = 32;  // tile height of the packed embedding table
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    int kernels_per_step = 0;
    bool finalized = false;
    // tensor-parallel exchange area (world > 1): this rank's, exported over CUDA IPC, and the peers'
    // mappings of theirs.  Layout: float recv[2][world][dim] | u64 cnt[2] | u64 keys[8] | u64 keys_cnt.
    uint8_t *comm = nullptr;
    size_t comm_bytes = 0, comm_ctl = 0;  // comm_ctl: offset of cnt[0]
    std::vector<void *> peer_base;        // [world]; this rank's entry is `comm`
    std::vector<bool> peer_opened;
    void **d_ptrs = nullptr;              // device pointer tables (see comm_tables)
    float *x2 = nullptr;                  // second residual buffer (the reduces ping-pong x <-> x2)
    unsigned long long *x64 = nullptr;    // persistent step, tensor parallel: the tagged residual, [2][dim]
    size_t comm_t64 = 0;                  // offset of the tagged receive areas, u64 [2][world][dim]
    unsigned long long *epoch = nullptr;  // decode steps completed (the exchange counters' epoch)
    bool connected = false;
    // persistent decode step (step.cu): the op list on the device, its dependency counters and plan
    bool use_step = true;                 // false: one kernel per GEMV / attention (DIOLKOS_STEP=kernels)
    StepOp *d_ops = nullptr;
    int n_ops = 0;
    unsigned long long *step_cnt = nullptr;  // [n_layers][5]: qkv, attention, wo, w1|w3, w2
    // the persistent step's attention plan (step_attn_plan): narrow items up to step_wide_from positions,
    // wide ones beyond; step_splits = the larger split count, the layout stride of the split scratch
    int step_narrow_splits = 1, step_wide_splits = 1, step_wide_chunk = 16, step_wide_from = 0x7fffffff;
    int step_splits = 1;
    StepArgs step;
    unsigned long long *d_trace = nullptr;  // DIOLKOS_STEP_TRACE=1: the persistent step's timeline
    std::vector<StepOp> h_ops;            // the op list as uploaded (diagnostics rewrite it)
    uint8_t *dump = nullptr;              // dk_model_dump_enable: per GEMV op input | int8 | scales
    std::vector<int> dump_ops;            // indices of the GEMV ops, step order
    // prompt prefill (tensor-core matmuls over chunks of up to pchunk positions), allocated on first use
    uint8_t *parena = nullptr;
    int pchunk = 0;
    float *px = nullptr, *pqkv = nullptr, *pxb = nullptr, *phb = nullptr, *pwork = nullptr, *pxs = nullptr;
    int8_t *pxq = nullptr;
    unsigned *pcount = nullptr;
    PrefillGroup *pgroups = nullptr;      // the attention's position groups of the current chunk
    float *ppart = nullptr;               // tensor parallel: this rank's wo / w2 partial rows [chunk][dim]
    size_t comm_pre = 0;                  // offset of the prefill receive areas in `comm`
    unsigned long long pex[2] = {0, 0};   // prefill exchanges done per parity (counter targets)
    bool prefill_broken = false;          // a tensor-parallel prefill exchange failed: prefill refused
    PrefillGroup *h_groups = nullptr;     // pinned: one slot of pchunk groups per chunk of the sequence
    int pslots = 0;
    std::vector<cudaEvent_t> pslot_done;  // recorded after each slot's upload: rewrite only after it
    size_t pwork_stride = 0, pcount_stride = 0;
};

static size_t align256(size_t v) { return (v + 255) & ~(size_t)255; }
// Positions per prefill chunk: the tensor-core matmul's token tiles are 32 wide; 256 positions keep
// the per-position attention scratch of a 7B-shape model near 100 MB.
static constexpr int kPrefillChunk = 256;
// Capacity of the per-CTA argmax partials, in CTAs per SM (plan_gemv never launches more).
static constexpr int kMaxGemvGrid = 4;

static int need(dk_model *m) {
    if (!m) return set_error(DK_ERR_INVALID, "null dk_model");
    cudaError_t e = cudaSetDevice(m->device);
    return cuda_status(e, "cudaSetDevice");
}

extern "C" {

dk_model *dk_model_create(const int *cfg, int kv_type, int device, int tp_rank, int tp_world) {
    if (!cfg) {
        set_error(DK_ERR_INVALID, "dk_model_create: null cfg");
        return nullptr;
    }
    const int dim = cfg[0], hidden = cfg[1], L = cfg[2], H = cfg[3], KVH = cfg[4], V = cfg[5], S = cfg[6];
    if (dim <= 0 || hidden <= 0 || L <= 0 || H <= 0 || KVH <= 0 || V <= 0 || S <= 0 || dim % H || H % KVH ||
        dim % 32 || hidden % 32 || (dim / H) % 4 || dim / H > 128 || H / KVH > 8) {
        set_error(DK_ERR_INVALID, "dk_model_create: unsupported config dim=%d hidden=%d layers=%d heads=%d kv=%d",
                  dim, hidden, L, H, KVH);
        return nullptr;
    }
    if (tp_world < 1 || tp_world > 8 || tp_rank < 0 || tp_rank >= tp_world) {
        set_error(DK_ERR_INVALID, "dk_model_create: tensor-parallel rank %d of %d (1 to 8 ranks)", tp_rank, tp_world);
        return nullptr;
    }
    if (tp_world > 1 && (H % tp_world || KVH % tp_world || hidden % (32 * tp_world) || ((dim / H) * (H / tp_world)) % 32)) {
        set_error(DK_ERR_INVALID,
                  "dk_model_create: %d ranks need heads, kv heads divisible by the ranks, hidden/ranks and "
                  "head_size*heads/ranks multiples of 32 (heads=%d kv=%d hidden=%d)",
                  tp_world, H, KVH, hidden);
        return nullptr;
    }
    if (kv_type != DK_KV_BF16 && kv_type != DK_KV_F32) {
        set_error(DK_ERR_INVALID, "dk_model_create: bad kv_type %d", kv_type);
        return nullptr;
    }
    if (cudaSetDevice(device) != cudaSuccess) {
        set_error(DK_ERR_CUDA, "dk_model_create: cudaSetDevice(%d) failed", device);
        return nullptr;
    }
    dk_model *m = new dk_model();
    m->dim = dim; m->hidden = hidden; m->n_layers = L; m->n_heads = H; m->n_kv_heads = KVH;
    m->vocab = V; m->seq_len = S; m->kv_type = kv_type; m->device = device;
    m->rank = tp_rank; m->world = tp_world;
    m->hs = dim / H;
    m->kv_dim = dim * KVH / H;
    m->l_heads = H / tp_world;
    m->l_kv_heads = KVH / tp_world;
    m->l_hidden = hidden / tp_world;
    m->l_dim = m->l_heads * m->hs;
    m->l_kv_dim = m->l_kv_heads * m->hs;
    {
        const int per = (V + tp_world - 1) / tp_world;
        m->vocab_off = tp_rank * per;
        m->l_vocab = std::max(0, std::min(V - m->vocab_off, per));
    }
    if (m->l_vocab < 1) {
        set_error(DK_ERR_INVALID, "dk_model_create: rank %d gets no classifier rows", tp_rank);
        delete m;
        return nullptr;
    }
    cudaDeviceGetAttribute(&m->num_sms, cudaDevAttrMultiProcessorCount, device);
    m->layers.resize(L);
    m->have.assign((size_t)(L + 1) * DK_W_COUNT, 0);

    auto fail = [&](const char *what) -> dk_model * {
        set_error(DK_ERR_NOMEM, "dk_model_create: %s", what);
        dk_model_destroy(m);
        return nullptr;
    };
    if (cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking) != cudaSuccess) return fail("stream");

    // ---- GEMV plans on this rank's shapes (they fix each matrix's tile height, hence its packed size)
    const int qkv_rows = m->l_dim + 2 * m->l_kv_dim, lh = m->l_hidden;
    m->p_qkv = plan_gemv(dim, qkv_rows, EPI_STORE, m->num_sms);
    m->p_wo = plan_gemv(m->l_dim, dim, EPI_ADD, m->num_sms);
    m->p_w13 = plan_gemv(dim, 2 * lh, EPI_SWIGLU, m->num_sms);
    m->p_w2 = plan_gemv(lh, dim, EPI_ADD, m->num_sms);
    m->p_cls = plan_gemv(dim, m->l_vocab, EPI_ARGMAX, m->num_sms);
    m->emb_T = gemv_tile_rows(V, EPI_STORE, m->num_sms);
    if (!gemv_supported(dim, qkv_rows, EPI_STORE) || !gemv_supported(dim, 2 * lh, EPI_SWIGLU) ||
        !gemv_supported(lh, dim, EPI_ADD) || !gemv_supported(m->l_dim, dim, EPI_ADD) ||
        !gemv_supported(dim, m->l_vocab, EPI_ARGMAX)) {
        set_error(DK_ERR_INVALID, "dk_model_create: matrix shapes exceed the GEMV's shared-memory budget");
        dk_model_destroy(m);
        return nullptr;
    }

    // ---- weights (zeroed: the pad rows of ragged last tiles and the pad bytes of segments stay 0)
    const size_t b_qkv = align256(q8_packed_bytes(dim, qkv_rows, m->p_qkv.T));
    const size_t b_wo = align256(q8_packed_bytes(m->l_dim, dim, m->p_wo.T));
    const size_t b_w13 = align256(q8_packed_bytes(dim, 2 * lh, m->p_w13.T));
    const size_t b_w2 = align256(q8_packed_bytes(lh, dim, m->p_w2.T));
    const size_t b_norm = align256((size_t)dim * 4);
    const size_t b_emb = align256(q8_packed_bytes(dim, V, m->emb_T));
    const size_t b_cls = align256(q8_packed_bytes(dim, m->l_vocab, m->p_cls.T));
    const size_t per_layer = b_qkv + b_wo + b_w13 + b_w2 + 2 * b_norm;
    m->warena_bytes = per_layer * L + b_emb + b_cls + b_norm;
    if (cudaMalloc(&m->warena, m->warena_bytes) != cudaSuccess) return fail("weight memory");
    if (cudaMemsetAsync(m->warena, 0, m->warena_bytes, m->stream) != cudaSuccess) return fail("weight memset");
    uint8_t *p = m->warena;
    m->emb = p; p += b_emb;
    m->wcls = p; p += b_cls;
    m->rms_final = reinterpret_cast<float *>(p); p += b_norm;
    for (int l = 0; l < L; ++l) {
        dk_layer &ly = m->layers[l];
        ly.wqkv = p; p += b_qkv;
        ly.wo = p; p += b_wo;
        ly.w13 = p; p += b_w13;
        ly.w2 = p; p += b_w2;
        ly.rms_att = reinterpret_cast<float *>(p); p += b_norm;
        ly.rms_ffn = reinterpret_cast<float *>(p); p += b_norm;
    }

    // ---- KV cache
    const size_t esz = kv_type == DK_KV_F32 ? 4 : 2;
    m->kv_layer_elems = (size_t)m->l_kv_heads * S * m->hs;
    if (cudaMalloc(&m->kcache, m->kv_layer_elems * L * esz) != cudaSuccess) return fail("key cache");
    if (cudaMalloc(&m->vcache, m->kv_layer_elems * L * esz) != cudaSuccess) return fail("value cache");
    cudaMemsetAsync(m->kcache, 0, m->kv_layer_elems * L * esz, m->stream);
    cudaMemsetAsync(m->vcache, 0, m->kv_layer_elems * L * esz, m->stream);

    // ---- activations and small state
    m->attn_splits = attn_max_splits(S, m->l_kv_heads, m->num_sms);
    {
        const char *mode = getenv("DIOLKOS_STEP");
        m->use_step = !(mode && strcmp(mode, "kernels") == 0);
    }
    // The persistent step's attention.  Narrow form (contexts up to step_wide_from positions): one
    // (KV head, split) item per 2-warp group of the grid (at most one wave: the split count is rounded
    // down), splits of at least 16 positions.  Wide form: at most
    // one wave of CTA-wide items, splits of at least step_min_chunk positions.  DIOLKOS_ATTN_WIDE_FROM moves
    // the switch (0: the wide form throughout; a value >= the context: the narrow form throughout);
    // DIOLKOS_ATTN_WIDE_CHUNK sets the wide form's shortest split (positions).
    {
        const int kv_mul = m->l_heads / m->l_kv_heads;
        m->step_narrow_splits =
            std::max(1, std::min(step_attn_item_slots(m->num_sms, kAttnNarrowWarps) / m->l_kv_heads, (S + 15) / 16));
        m->step_wide_chunk = step_min_chunk(kv_mul);
        if (const char *e = getenv("DIOLKOS_ATTN_WIDE_CHUNK")) m->step_wide_chunk = std::max(16, atoi(e));
        m->step_wide_splits =
            std::max(1, std::min(step_attn_item_slots(m->num_sms, kAttnWideWarps) / m->l_kv_heads,
                                 (S + m->step_wide_chunk - 1) / m->step_wide_chunk));
        m->step_wide_from = kStepWideFrom;
        // The wide form runs one wave of CTA-wide items.  Where they would leave more than a tenth of the
        // CTAs idle (the 7B shape on one GPU: 4 splits x 32 KV heads = 128 of 148), the narrow form's
        // full wave is the faster one at every context length.
        if ((long long)m->step_wide_splits * m->l_kv_heads * 10 < (long long)m->num_sms * 9)
            m->step_wide_from = 0x7fffffff;
        if (const char *e = getenv("DIOLKOS_ATTN_WIDE_FROM")) m->step_wide_from = std::max(0, atoi(e));
        m->step_splits = std::max(m->step_narrow_splits, m->step_wide_splits);
    }
    const int work_splits = std::max(m->attn_splits, m->step_splits);
    const size_t sz_x = align256((size_t)dim * 4), sz_qkv = align256((size_t)qkv_rows * 4);
    const size_t sz_hb = align256((size_t)lh * 4), sz_logits = align256((size_t)m->l_vocab * 4);
    const size_t sz_rope = align256((size_t)S * m->hs * 4);
    const size_t sz_work = align256((size_t)m->l_heads * work_splits * (m->hs + 2) * 4);
    const size_t sz_stepcnt = align256((size_t)L * 5 * 8);
    const size_t sz_cnt = align256((size_t)m->l_kv_heads * 4);
    const size_t sz_part = align256((size_t)kMaxGemvGrid * m->num_sms * 8);
    const size_t sz_tok = align256((size_t)(S + 1) * 4);
    const size_t sz_x64 = tp_world > 1 ? 2 * align256((size_t)dim * 8) : 0;
    const size_t total = sz_x * 3 + sz_qkv + sz_hb + sz_logits + sz_rope + sz_work + sz_cnt + sz_part + 256 + sz_tok +
                         4 * 256 + sz_stepcnt + sz_x64;
    if (cudaMalloc(&m->aarena, total) != cudaSuccess) return fail("activation memory");
    cudaMemsetAsync(m->aarena, 0, total, m->stream);
    p = m->aarena;
    m->x = reinterpret_cast<float *>(p); p += sz_x;
    m->x2 = reinterpret_cast<float *>(p); p += sz_x;
    m->xb = reinterpret_cast<float *>(p); p += sz_x;
    m->qkv = reinterpret_cast<float *>(p); p += sz_qkv;
    m->hb = reinterpret_cast<float *>(p); p += sz_hb;
    m->logits = reinterpret_cast<float *>(p); p += sz_logits;
    m->rope = reinterpret_cast<float *>(p); p += sz_rope;
    m->attn_work = reinterpret_cast<float *>(p); p += sz_work;
    m->attn_count = reinterpret_cast<unsigned *>(p); p += sz_cnt;
    m->amax_part = reinterpret_cast<unsigned long long *>(p); p += sz_part;
    m->amax_count = reinterpret_cast<unsigned *>(p); p += 256;
    m->tokens = reinterpret_cast<int *>(p); p += sz_tok;
    m->pos = reinterpret_cast<int *>(p); p += 256;
    m->n_forced = reinterpret_cast<int *>(p); p += 256;
    m->err = reinterpret_cast<int *>(p); p += 256;
    m->epoch = reinterpret_cast<unsigned long long *>(p); p += 256;
    m->step_cnt = reinterpret_cast<unsigned long long *>(p); p += sz_stepcnt;
    if (sz_x64) {  // zeroed with the arena: tag 0 is never a live tag
        m->x64 = reinterpret_cast<unsigned long long *>(p);
        p += sz_x64;
    }

    // ---- tensor-parallel exchange area (its own allocation: it is exported to the peers over IPC)
    if (tp_world > 1) {
        m->comm_ctl = align256((size_t)2 * tp_world * dim * 4);
        // then the prefill's two receive areas, [rank][chunk position][dim] floats each
        m->comm_pre = m->comm_ctl + 256;
        m->comm_t64 = m->comm_pre + 2 * align256((size_t)tp_world * std::min(kPrefillChunk, S) * dim * 4);
        // then the persistent step's tagged receive areas (zeroed: tag 0 is never a live tag)
        m->comm_bytes = m->comm_t64 + 2 * align256((size_t)tp_world * dim * 8);
        if (cudaMalloc(&m->comm, m->comm_bytes) != cudaSuccess) return fail("exchange area");
        if (cudaMemset(m->comm, 0, m->comm_bytes) != cudaSuccess) return fail("exchange area clear");
        if (cudaMalloc(&m->d_ptrs, 12 * 8 * sizeof(void *)) != cudaSuccess) return fail("peer pointer tables");
        m->peer_base.assign(tp_world, nullptr);
        m->peer_opened.assign(tp_world, false);
        m->peer_base[tp_rank] = m->comm;
    }

    std::vector<float> rt;
    rope_table(rt, S, m->hs);
    if (cudaMemcpyAsync(m->rope, rt.data(), rt.size() * 4, cudaMemcpyHostToDevice, m->stream) != cudaSuccess)
        return fail("rope upload");
    if (cudaMallocHost(&m->h_small, 4096) != cudaSuccess) return fail("pinned scratch");
    if (cudaStreamSynchronize(m->stream) != cudaSuccess) return fail("init sync");

    return m;
}

void dk_model_destroy(dk_model *m) {
    if (!m) return;
    cudaSetDevice(m->device);
    if (m->stream) cudaStreamSynchronize(m->stream);
    if (m->exec) cudaGraphExecDestroy(m->exec);
    if (m->graph) cudaGraphDestroy(m->graph);
    cudaFree(m->warena);
    cudaFree(m->kcache);
    cudaFree(m->vcache);
    cudaFree(m->aarena);
    cudaFree(m->stage);
    for (size_t q = 0; q < m->peer_base.size(); ++q)
        if (m->peer_opened[q]) cudaIpcCloseMemHandle(m->peer_base[q]);
    cudaFree(m->comm);
    cudaFree(m->d_ptrs);
    cudaFree(m->d_ops);
    cudaFree(m->d_trace);
    cudaFree(m->dump);
    cudaFree(m->parena);
    if (m->h_groups) cudaFreeHost(m->h_groups);
    for (cudaEvent_t e : m->pslot_done)
        if (e) cudaEventDestroy(e);
    if (m->h_small) cudaFreeHost(m->h_small);
    if (m->stream) cudaStreamDestroy(m->stream);
    delete m;
}

}  // extern "C"

// Shape of one weight: rows x cols of the full (unsharded) matrix; cols == 0 for norm vectors.
static int weight_shape(const dk_model *m, int which, int &rows, int &cols) {
    switch (which) {
    case DK_W_EMB: case DK_W_WCLS: rows = m->vocab; cols = m->dim; return 1;
    case DK_W_WQ: case DK_W_WO: rows = m->dim; cols = m->dim; return 1;
    case DK_W_WK: case DK_W_WV: rows = m->kv_dim; cols = m->dim; return 1;
    case DK_W_W1: case DK_W_W3: rows = m->hidden; cols = m->dim; return 1;
    case DK_W_W2: rows = m->dim; cols = m->hidden; return 1;
    case DK_W_RMS_FINAL: case DK_W_RMS_ATT: case DK_W_RMS_FFN: rows = m->dim; cols = 0; return 0;
    default: return -1;
    }
}

static int set_weight_impl(dk_model *m, int which, int layer, const void *q, const float *scale, bool on_device) {
    if (int r = need(m)) return r;
    if (m->finalized) return set_error(DK_ERR_STATE, "dk_model_set_weight: model already finalized");
    int rows = 0, cols = 0;
    const int kind = weight_shape(m, which, rows, cols);
    if (kind < 0) return set_error(DK_ERR_INVALID, "dk_model_set_weight: unknown weight id %d", which);
    const bool per_layer = which >= DK_W_RMS_ATT;
    if (per_layer ? (layer < 0 || layer >= m->n_layers) : (layer != -1))
        return set_error(DK_ERR_INVALID, "dk_model_set_weight: bad layer %d for weight %d", layer, which);
    if (!q || (kind == 1 && !scale)) return set_error(DK_ERR_INVALID, "dk_model_set_weight: null data");
    cudaStream_t st = m->stream;
    const cudaMemcpyKind dir = on_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;

    if (kind == 0) {  // fp32 norm vector
        float *dst = which == DK_W_RMS_FINAL ? m->rms_final
                     : which == DK_W_RMS_ATT ? m->layers[layer].rms_att : m->layers[layer].rms_ffn;
        if (int r = cuda_status(cudaMemcpyAsync(dst, q, (size_t)rows * 4, dir, st), "norm upload")) return r;
        if (int r = cuda_status(cudaStreamSynchronize(st), "norm upload sync")) return r;
    } else {
        const size_t nq = (size_t)rows * cols, ns = nq / 32;
        const int8_t *src_q = static_cast<const int8_t *>(q);
        const float *src_s = scale;
        if (!on_device) {
            const size_t need_bytes = align256(nq) + ns * 4;
            if (need_bytes > m->stage_bytes) {
                if (m->stage) {
                    cudaStreamSynchronize(st);
                    cudaFree(m->stage);
                    m->stage = nullptr;
                    m->stage_bytes = 0;
                }
                if (cudaMalloc(&m->stage, need_bytes) != cudaSuccess)
                    return set_error(DK_ERR_NOMEM, "dk_model_set_weight: staging buffer of %zu bytes", need_bytes);
                m->stage_bytes = need_bytes;
            }
            if (int r = cuda_status(cudaMemcpyAsync(m->stage, q, nq, cudaMemcpyHostToDevice, st), "weight upload"))
                return r;
            if (int r = cuda_status(cudaMemcpyAsync(m->stage + align256(nq), scale, ns * 4, cudaMemcpyHostToDevice, st),
                                    "scale upload"))
                return r;
            src_q = reinterpret_cast<const int8_t *>(m->stage);
            src_s = reinterpret_cast<const float *>(m->stage + align256(nq));
        }
        // This rank's part of the full matrix: rows [r0, r0 + nrows) and columns [c0, c0 + ncols),
        // packed into rows row0, row0 + step, ... of the local matrix.
        uint8_t *dst = nullptr;
        int row0 = 0, step = 1, T = 32, r0 = 0, nrows = rows, c0 = 0, ncols = cols;
        const dk_layer *ly = per_layer ? &m->layers[layer] : nullptr;
        switch (which) {
        case DK_W_EMB: dst = m->emb; T = m->emb_T; break;
        case DK_W_WCLS: dst = m->wcls; T = m->p_cls.T; r0 = m->vocab_off; nrows = m->l_vocab; break;
        case DK_W_WQ: dst = ly->wqkv; T = m->p_qkv.T; r0 = m->rank * m->l_dim; nrows = m->l_dim; break;
        case DK_W_WK:
            dst = ly->wqkv; row0 = m->l_dim; T = m->p_qkv.T; r0 = m->rank * m->l_kv_dim; nrows = m->l_kv_dim;
            break;
        case DK_W_WV:
            dst = ly->wqkv; row0 = m->l_dim + m->l_kv_dim; T = m->p_qkv.T; r0 = m->rank * m->l_kv_dim;
            nrows = m->l_kv_dim;
            break;
        case DK_W_WO: dst = ly->wo; T = m->p_wo.T; c0 = m->rank * m->l_dim; ncols = m->l_dim; break;
        case DK_W_W1:
            dst = ly->w13; row0 = 0; step = 2; T = m->p_w13.T; r0 = m->rank * m->l_hidden; nrows = m->l_hidden;
            break;
        case DK_W_W3:
            dst = ly->w13; row0 = 1; step = 2; T = m->p_w13.T; r0 = m->rank * m->l_hidden; nrows = m->l_hidden;
            break;
        case DK_W_W2: dst = ly->w2; T = m->p_w2.T; c0 = m->rank * m->l_hidden; ncols = m->l_hidden; break;
        default: break;
        }
        if (int r = cuda_status(launch_pack_rows(dst, ncols, T, src_q + (size_t)r0 * cols, src_s + (size_t)r0 * (cols / 32),
                                                 nrows, row0, step, st, cols, c0),
                                "pack rows"))
            return r;
        // The staging buffer is reused by the next call, and a caller may free its device source
        // buffers as soon as this returns: wait for the copy.
        if (int r = cuda_status(cudaStreamSynchronize(st), "weight upload sync")) return r;
    }
    m->have[(size_t)(per_layer ? layer : m->n_layers) * DK_W_COUNT + which] = 1;
    return DK_OK;
}

// Offsets inside a rank's exchange area and the device pointer tables built from the peers' mappings:
// table t (8 entries, one per rank) at d_ptrs + 8*t: 0/1 receive areas of parity 0/1, 2/3 their
// counters, 4 the argmax key arrays, 5 their counters, 6..9 the prefill's receive areas and counters,
// 10/11 the persistent step's tagged receive areas of parity 0/1.
static size_t comm_recv_off(const dk_model *m, int par) { return (size_t)par * m->world * m->dim * 4; }
static size_t comm_cnt_off(const dk_model *m, int par) { return m->comm_ctl + 8 * (size_t)par; }
static size_t comm_keys_off(const dk_model *m) { return m->comm_ctl + 16; }
static size_t comm_keys_cnt_off(const dk_model *m) { return m->comm_ctl + 16 + 64; }
static size_t comm_pcnt_off(const dk_model *m, int par) { return m->comm_ctl + 128 + 8 * (size_t)par; }
static size_t comm_t64_off(const dk_model *m, int par) {
    return m->comm_t64 + (size_t)par * align256((size_t)m->world * m->dim * 8);
}
static size_t comm_pre_off(const dk_model *m, int par) {
    return m->comm_pre + (size_t)par * align256((size_t)m->world * std::min(kPrefillChunk, m->seq_len) * m->dim * 4);
}

static int enqueue_step(dk_model *m, cudaStream_t st) {
    int launches = 0;
    // The first kernel of the step has no kernel predecessor inside the graph, so it is launched
    // without the programmatic-dependency attribute; every later kernel overlaps its weight
    // prefetch with the tail of the previous one.
    auto base_args = [&](const uint8_t *w, int n, int d, int pro, int epi, const float *x, const float *norm,
                         float *out) {
        GemvArgs a;
        a.w = w; a.n = n; a.d = d; a.pro = pro; a.epi = epi; a.x = x; a.norm_w = norm; a.out = out;
        a.emb = m->emb; a.emb_T = m->emb_T; a.tokens = m->tokens; a.pos = m->pos; a.n_forced = m->n_forced;
        a.seq_len = m->seq_len; a.amax_part = m->amax_part; a.amax_count = m->amax_count; a.err = m->err;
        a.tp_rank = m->rank; a.tp_world = m->world; a.epoch = m->epoch; a.epoch_rw = m->epoch;
        a.row_offset = m->vocab_off; a.vocab = m->vocab;
        return a;
    };
    auto launch = [&](const char *what, const GemvPlan &p, const GemvArgs &a) -> int {
        const bool pdl = launches > 0;
        ++launches;
        return cuda_status(launch_gemv(a, p, st, pdl), what);
    };
    const bool tp = m->world > 1;
    void *const *tab = reinterpret_cast<void *const *>(m->d_ptrs);
    // Tensor parallel: this rank's partial rows of wo / w2 go to every rank (EPI_PEER, exchange point
    // parity 0 / 1); the next GEMV waits for all of them and adds them to x in rank order
    // (PRO_RMS_REDUCE), writing the new residual to the other of the two x buffers.
    auto peer_epi = [&](GemvArgs &a, int par) {
        a.peer_recv = reinterpret_cast<float *const *>(tab + 8 * par);
        a.peer_cnt = reinterpret_cast<unsigned long long *const *>(tab + 8 * (2 + par));
    };
    float *X[2] = {m->x, m->x2};
    int cur = 0;
    auto reduce_pro = [&](GemvArgs &a, int par, int index) {
        a.x = X[cur];
        a.x_out = X[1 - cur];
        a.recv = reinterpret_cast<const float *>(m->comm + comm_recv_off(m, par));
        a.cnt = reinterpret_cast<const unsigned long long *>(m->comm + comm_cnt_off(m, par));
        a.red_index = index;
        a.red_period = m->n_layers;
        cur = 1 - cur;
    };
    const int qkv_rows = m->l_dim + 2 * m->l_kv_dim;
    const size_t esz = m->kv_type == DK_KV_F32 ? 4 : 2;
    for (int l = 0; l < m->n_layers; ++l) {
        const dk_layer &ly = m->layers[l];
        {
            GemvArgs a = base_args(ly.wqkv, m->dim, qkv_rows, l == 0 ? PRO_EMB_RMS : PRO_RMS, EPI_STORE, X[cur],
                                   ly.rms_att, m->qkv);
            if (tp && l > 0) {
                a.pro = PRO_RMS_REDUCE;
                reduce_pro(a, 1, l - 1);
            }
            if (int r = launch("qkv gemv", m->p_qkv, a)) return r;
        }
        AttnArgs at;
        at.qkv = m->qkv; at.rope = m->rope;
        at.k_cache = static_cast<uint8_t *>(m->kcache) + (size_t)l * m->kv_layer_elems * esz;
        at.v_cache = static_cast<uint8_t *>(m->vcache) + (size_t)l * m->kv_layer_elems * esz;
        at.out = m->xb; at.work = m->attn_work; at.count = m->attn_count; at.pos = m->pos;
        at.n_heads = m->l_heads; at.n_kv_heads = m->l_kv_heads; at.head_size = m->hs; at.seq_len = m->seq_len;
        at.kv_f32 = m->kv_type == DK_KV_F32; at.max_splits = m->attn_splits; at.min_chunk = kAttnMinChunk; at.err = m->err;
        ++launches;
        if (int r = cuda_status(launch_attention(at, st, true), "attention")) return r;
        {
            GemvArgs a = base_args(ly.wo, m->l_dim, m->dim, PRO_F32, tp ? EPI_PEER : EPI_ADD, m->xb, nullptr, X[cur]);
            if (tp) peer_epi(a, 0);
            if (int r = launch("wo gemv", m->p_wo, a)) return r;
        }
        {
            GemvArgs a = base_args(ly.w13, m->dim, 2 * m->l_hidden, PRO_RMS, EPI_SWIGLU, X[cur], ly.rms_ffn, m->hb);
            if (tp) {
                a.pro = PRO_RMS_REDUCE;
                reduce_pro(a, 0, l);
            }
            if (int r = launch("w1/w3 gemv", m->p_w13, a)) return r;
        }
        {
            GemvArgs a = base_args(ly.w2, m->l_hidden, m->dim, PRO_F32, tp ? EPI_PEER : EPI_ADD, m->hb, nullptr, X[cur]);
            if (tp) peer_epi(a, 1);
            if (int r = launch("w2 gemv", m->p_w2, a)) return r;
        }
    }
    if (m->p_cls.grid > kMaxGemvGrid * m->num_sms)
        return set_error(DK_ERR_INVALID, "classifier grid %d exceeds the argmax partials", m->p_cls.grid);
    {
        GemvArgs a = base_args(m->wcls, m->dim, m->l_vocab, PRO_RMS, EPI_ARGMAX, X[cur], m->rms_final, m->logits);
        if (tp) {
            a.pro = PRO_RMS_REDUCE;
            reduce_pro(a, 1, m->n_layers - 1);
            a.peer_amax = reinterpret_cast<unsigned long long *const *>(tab + 8 * 4);
            a.peer_amax_cnt = reinterpret_cast<unsigned long long *const *>(tab + 8 * 5);
            a.amax_keys = reinterpret_cast<const unsigned long long *>(m->comm + comm_keys_off(m));
            a.amax_keys_cnt = reinterpret_cast<const unsigned long long *>(m->comm + comm_keys_cnt_off(m));
        }
        if (int r = launch("classifier gemv", m->p_cls, a)) return r;
    }
    m->kernels_per_step = launches;
    return DK_OK;
}

// The persistent step (step.cu): the step's op list -- per layer q|k|v GEMV, attention, wo GEMV, w1|w3
// GEMV, w2 GEMV; then the classifier -- with the same arguments the per-kernel path gives each launch,
// the dependency counters that replace the kernel boundaries, and the shared-memory plan.
// The persistent step's attention plan, shared by the decode step and the prompt prefill (step_attn_plan).
static void step_attn_fields(const dk_model *m, AttnArgs &t) {
    t.max_splits = m->step_splits;
    t.min_chunk = 16;
    t.narrow_max_splits = m->step_narrow_splits;
    t.narrow_min_chunk = 16;
    t.wide_max_splits = m->step_wide_splits;
    t.wide_min_chunk = m->step_wide_chunk;
    t.wide_from = m->step_wide_from;
}

static int build_step(dk_model *m) {
    const bool tp = m->world > 1;
    void *const *tab = reinterpret_cast<void *const *>(m->d_ptrs);
    std::vector<StepOp> ops;
    auto cnt = [&](int l, int k) { return m->step_cnt + (size_t)l * 5 + k; };
    auto gemv_op = [&](const uint8_t *w, int n, int d, int pro, int epi, const float *x, const float *norm, float *out,
                       const GemvPlan &p) {
        StepOp op;
        op.kind = OP_GEMV;
        GemvArgs &a = op.g;
        a.w = w; a.n = n; a.d = d; a.pro = pro; a.epi = epi; a.x = x; a.norm_w = norm; a.out = out;
        a.emb = m->emb; a.emb_T = m->emb_T; a.tokens = m->tokens; a.pos = m->pos; a.n_forced = m->n_forced;
        a.seq_len = m->seq_len; a.amax_part = m->amax_part; a.amax_count = m->amax_count; a.err = m->err;
        a.tp_rank = m->rank; a.tp_world = m->world; a.epoch = m->epoch; a.epoch_rw = m->epoch;
        a.row_offset = m->vocab_off; a.vocab = m->vocab;
        op.T = p.T;
        op.ntiles = p.ntiles;
        return op;
    };
    float *X[2] = {m->x, m->x2};
    int cur = 0;
    // Tensor parallel: the tagged exchange (dk_kernels.h, GemvArgs::tagged).  Event k of a step: 0 the
    // embedding row, 2l+1 the reduce after layer l's wo, 2l+2 the reduce after its w2; the reduce of event
    // k reads the tagged residual x64[(k-1) & 1] and writes x64[k & 1].
    const int n_gather = std::min(16, m->num_sms);
    auto x64 = [&](int k) { return m->x64 + (size_t)(k & 1) * (align256((size_t)m->dim * 8) / 8); };
    auto tagged = [&](GemvArgs &a, int k) {
        a.tagged = 1;
        a.tag_k = k;
        a.tag_period = 2 * m->n_layers + 1;
        a.n_gather = n_gather;
    };
    auto reduce_pro = [&](StepOp &op, int par, int k) {
        GemvArgs &a = op.g;
        a.pro = PRO_RMS_REDUCE;
        tagged(a, k);
        a.x64 = x64(k - 1);
        a.x64_out = x64(k);
        a.recv64 = reinterpret_cast<const unsigned long long *>(m->comm + comm_t64_off(m, par));
    };
    auto peer_epi = [&](StepOp &op, int par, int k) {
        tagged(op.g, k);
        op.g.peer_recv64 = reinterpret_cast<unsigned long long *const *>(tab + 8 * (10 + par));
    };
    const int qkv_rows = m->l_dim + 2 * m->l_kv_dim;
    const size_t esz = m->kv_type == DK_KV_F32 ? 4 : 2;
    for (int l = 0; l < m->n_layers; ++l) {
        const dk_layer &ly = m->layers[l];
        StepOp q = gemv_op(ly.wqkv, m->dim, qkv_rows, l == 0 ? PRO_EMB_RMS : PRO_RMS, EPI_STORE, X[cur], ly.rms_att,
                           m->qkv, m->p_qkv);
        if (l == 0 && tp) {  // the embedding row starts the tagged residual chain (event 0)
            tagged(q.g, 0);
            q.g.x64_out = x64(0);
        }
        if (l > 0) {
            if (tp) {
                reduce_pro(q, 1, 2 * l);
            } else {
                q.wait_cnt = cnt(l - 1, 4);
                q.wait_units = (unsigned long long)m->dim;
            }
        }
        q.done_cnt = cnt(l, 0);
        ops.push_back(q);

        StepOp at;
        at.kind = OP_ATTN;
        AttnArgs &t = at.at;
        t.qkv = m->qkv; t.rope = m->rope;
        t.k_cache = static_cast<uint8_t *>(m->kcache) + (size_t)l * m->kv_layer_elems * esz;
        t.v_cache = static_cast<uint8_t *>(m->vcache) + (size_t)l * m->kv_layer_elems * esz;
        t.out = m->xb; t.work = m->attn_work; t.count = m->attn_count; t.pos = m->pos;
        t.n_heads = m->l_heads; t.n_kv_heads = m->l_kv_heads; t.head_size = m->hs; t.seq_len = m->seq_len;
        t.kv_f32 = m->kv_type == DK_KV_F32; step_attn_fields(m, t); t.err = m->err;
        at.wait_cnt = cnt(l, 0);
        at.wait_units = (unsigned long long)qkv_rows;
        at.done_cnt = cnt(l, 1);
        ops.push_back(at);

        StepOp o = gemv_op(ly.wo, m->l_dim, m->dim, PRO_F32, tp ? EPI_PEER : EPI_ADD, m->xb, nullptr, X[cur], m->p_wo);
        o.wait_cnt = cnt(l, 1);
        o.wait_units = (unsigned long long)m->l_dim;
        if (tp) peer_epi(o, 0, 2 * l + 1);
        else o.done_cnt = cnt(l, 2);
        ops.push_back(o);

        StepOp u = gemv_op(ly.w13, m->dim, 2 * m->l_hidden, PRO_RMS, EPI_SWIGLU, X[cur], ly.rms_ffn, m->hb, m->p_w13);
        if (tp) {
            reduce_pro(u, 0, 2 * l + 1);
        } else {
            u.wait_cnt = cnt(l, 2);
            u.wait_units = (unsigned long long)m->dim;
        }
        u.done_cnt = cnt(l, 3);
        ops.push_back(u);

        StepOp d = gemv_op(ly.w2, m->l_hidden, m->dim, PRO_F32, tp ? EPI_PEER : EPI_ADD, m->hb, nullptr, X[cur], m->p_w2);
        d.wait_cnt = cnt(l, 3);
        d.wait_units = (unsigned long long)m->l_hidden;
        if (tp) peer_epi(d, 1, 2 * l + 2);
        else d.done_cnt = cnt(l, 4);
        ops.push_back(d);
    }
    {
        StepOp c = gemv_op(m->wcls, m->dim, m->l_vocab, PRO_RMS, EPI_ARGMAX, X[cur], m->rms_final, m->logits, m->p_cls);
        if (tp) {
            reduce_pro(c, 1, 2 * m->n_layers);
            c.g.peer_amax = reinterpret_cast<unsigned long long *const *>(tab + 8 * 4);
            c.g.peer_amax_cnt = reinterpret_cast<unsigned long long *const *>(tab + 8 * 5);
            c.g.amax_keys = reinterpret_cast<const unsigned long long *>(m->comm + comm_keys_off(m));
            c.g.amax_keys_cnt = reinterpret_cast<const unsigned long long *>(m->comm + comm_keys_cnt_off(m));
        } else {
            c.wait_cnt = cnt(m->n_layers - 1, 4);
            c.wait_units = (unsigned long long)m->dim;
        }
        ops.push_back(c);
    }

    // shared memory: the ring, the activation (or attention scratch), the control block
    size_t slot = 0, act = step_attn_scratch_bytes(m->l_heads, m->l_kv_heads, m->hs);
    for (const StepOp &op : ops)
        if (op.kind == OP_GEMV) {
            slot = std::max(slot, (size_t)op.T * q8_blk_bytes(std::min(op.g.n, 512)));
            act = std::max(act, gemv_x_bytes(op.g.n));
        }
    StepArgs &sa = m->step;
    sa.slot = (slot + 127) & ~(size_t)127;
    sa.xoff = 0;  // set below
    const size_t budget = 227 * 1024, tail = ((act + 127) & ~(size_t)127) + step_ctl_bytes();
    int S = budget > tail ? (int)((budget - tail) / sa.slot) : 0;
    S = std::min(S, kStepMaxSlots);
    S -= S % kStepProducers;
    if (S < 2 * kStepProducers)
        return set_error(DK_ERR_INVALID, "persistent step: the activation (%zu bytes) leaves no room for the ring", act);
    sa.S = S;
    int nc = 4;  // measured best on B200 for the LLaMA shapes (more warps spin on the token flags)
    if (const char *e = getenv("DIOLKOS_STEP_NC")) nc = atoi(e);
    // A consumer waits on a slot's full barrier by parity, which is sound once the slot's previous stage
    // has landed: the token chain guarantees that for S >= 2 NC + 2 (units of two stages, step.cu).
    sa.NC = std::max(1, std::min(std::min(nc, (S - 2) / 2), kStepMaxConsumers));
    // Copies in flight per CTA.  While the compute warps wait for an op's input, build its activation or
    // run attention, the stream's queued copies delay their stores and L2 loads, so the producers keep
    // fewer in flight then (2) than while the stages are consumed (8).  Measured on B200, 7B decode:
    // one cap throughout 505 / 515 / 512 / 470 tok/s (as many as the ring allows / 4 / 6 / 2); 2 in the
    // waits with 4 / 6 / 8 otherwise 541 / 544 / 544, with 4 otherwise and 8 in the waits 523.
    sa.inflight = std::min(S, 8);
    if (const char *e = getenv("DIOLKOS_STEP_INFLIGHT")) sa.inflight = std::max(0, std::min(S, atoi(e) & ~(kStepProducers - 1)));
    sa.inflight_crit = std::min(S, 2);
    if (const char *e = getenv("DIOLKOS_STEP_INFLIGHT_CRIT"))
        sa.inflight_crit = std::max(0, std::min(S, atoi(e) & ~(kStepProducers - 1)));
    sa.xoff = (size_t)S * sa.slot;
    sa.ctl_off = sa.xoff + ((act + 127) & ~(size_t)127);
    sa.smem = sa.ctl_off + step_ctl_bytes();
    sa.epoch = m->epoch;
    sa.epoch_rw = m->epoch;
    sa.pos = m->pos;
    sa.seq_len = m->seq_len;
    sa.err = m->err;
    m->n_ops = (int)ops.size();
    m->h_ops = ops;
    m->dump_ops.clear();
    for (int i = 0; i < (int)ops.size(); ++i)
        if (ops[i].kind == OP_GEMV) m->dump_ops.push_back(i);
    if (cudaMalloc(&m->d_ops, ops.size() * sizeof(StepOp)) != cudaSuccess)
        return set_error(DK_ERR_NOMEM, "persistent step: op list");
    if (int r = cuda_status(cudaMemcpy(m->d_ops, ops.data(), ops.size() * sizeof(StepOp), cudaMemcpyHostToDevice),
                            "persistent step: op upload"))
        return r;
    sa.ops = m->d_ops;
    sa.nops = m->n_ops;
    if (const char *e = getenv("DIOLKOS_STEP_TRACE"))
        if (atoi(e) > 0) {
            const size_t tb = ((size_t)m->num_sms * m->n_ops * 8 + kStageTraceEntries) * 8;
            if (cudaMalloc(&m->d_trace, tb) != cudaSuccess || cudaMemset(m->d_trace, 0, tb) != cudaSuccess)
                return set_error(DK_ERR_NOMEM, "persistent step: trace buffer");
            sa.trace = m->d_trace;
            sa.stage_trace = m->d_trace + (size_t)m->num_sms * m->n_ops * 8;
            sa.stage_op0 = m->n_layers > 1 ? 5 : 0;  // the second layer's five ops
        }
    const int per_sm = step_max_ctas_per_sm(sa.smem);
    if (per_sm < 1)
        return set_error(DK_ERR_INVALID, "persistent step: %zu bytes of shared memory per CTA do not fit an SM", sa.smem);
    return DK_OK;
}

static int enqueue_step_persistent(dk_model *m, cudaStream_t st) {
    m->kernels_per_step = 1;
    return cuda_status(launch_step(m->step, m->num_sms, st), "persistent step");
}

extern "C" {

int dk_model_set_weight(dk_model *m, int which, int layer, const void *q, const float *scale) {
    return set_weight_impl(m, which, layer, q, scale, false);
}

int dk_model_set_weight_device(dk_model *m, int which, int layer, const void *q, const float *scale) {
    return set_weight_impl(m, which, layer, q, scale, true);
}

int dk_model_comm_handle(dk_model *m, void *handle) {
    if (int r = need(m)) return r;
    if (m->world < 2 || !m->comm) return set_error(DK_ERR_STATE, "dk_model_comm_handle: not a tensor-parallel model");
    if (!handle) return set_error(DK_ERR_INVALID, "dk_model_comm_handle: null handle");
    cudaIpcMemHandle_t h;
    if (int r = cuda_status(cudaIpcGetMemHandle(&h, m->comm), "cudaIpcGetMemHandle")) return r;
    static_assert(sizeof(h) == DK_COMM_HANDLE_BYTES, "IPC handle size");
    memcpy(handle, &h, sizeof(h));
    return DK_OK;
}

int dk_model_comm_connect(dk_model *m, const void *handles) {
    if (int r = need(m)) return r;
    if (m->world < 2 || !m->comm) return set_error(DK_ERR_STATE, "dk_model_comm_connect: not a tensor-parallel model");
    if (m->connected) return set_error(DK_ERR_STATE, "dk_model_comm_connect: already connected");
    if (!handles) return set_error(DK_ERR_INVALID, "dk_model_comm_connect: null handles");
    for (int q = 0; q < m->world; ++q) {
        if (q == m->rank) continue;
        cudaIpcMemHandle_t h;
        memcpy(&h, static_cast<const uint8_t *>(handles) + (size_t)q * DK_COMM_HANDLE_BYTES, sizeof(h));
        void *ptr = nullptr;
        const cudaError_t e = cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess)
            return set_error(DK_ERR_COMM, "dk_model_comm_connect: opening rank %d's exchange area: %s", q,
                             cudaGetErrorString(e));
        m->peer_base[q] = ptr;
        m->peer_opened[q] = true;
    }
    std::vector<void *> t(12 * 8, nullptr);
    for (int q = 0; q < m->world; ++q) {
        uint8_t *b = static_cast<uint8_t *>(m->peer_base[q]);
        t[0 * 8 + q] = b + comm_recv_off(m, 0);
        t[1 * 8 + q] = b + comm_recv_off(m, 1);
        t[2 * 8 + q] = b + comm_cnt_off(m, 0);
        t[3 * 8 + q] = b + comm_cnt_off(m, 1);
        t[4 * 8 + q] = b + comm_keys_off(m);
        t[5 * 8 + q] = b + comm_keys_cnt_off(m);
        t[6 * 8 + q] = b + comm_pre_off(m, 0);  // prefill receive areas and counters
        t[7 * 8 + q] = b + comm_pre_off(m, 1);
        t[8 * 8 + q] = b + comm_pcnt_off(m, 0);
        t[9 * 8 + q] = b + comm_pcnt_off(m, 1);
        t[10 * 8 + q] = b + comm_t64_off(m, 0);  // the persistent step's tagged receive areas
        t[11 * 8 + q] = b + comm_t64_off(m, 1);
    }
    if (int r = cuda_status(cudaMemcpy(m->d_ptrs, t.data(), t.size() * sizeof(void *), cudaMemcpyHostToDevice),
                            "peer table upload"))
        return r;
    m->connected = true;
    return DK_OK;
}

int dk_model_finalize(dk_model *m) {
    if (int r = need(m)) return r;
    if (m->finalized) return DK_OK;
    if (m->world > 1 && !m->connected)
        return set_error(DK_ERR_STATE, "dk_model_finalize: connect the ranks first (dk_model_comm_connect)");
    for (int l = 0; l <= m->n_layers; ++l)
        for (int w = 0; w < DK_W_COUNT; ++w) {
            const bool per_layer = w >= DK_W_RMS_ATT;
            if (per_layer != (l < m->n_layers)) continue;
            if (!m->have[(size_t)l * DK_W_COUNT + w])
                return set_error(DK_ERR_STATE, "dk_model_finalize: weight %d of layer %d was never set", w,
                                 per_layer ? l : -1);
        }
    if (int r = cuda_status(cudaStreamSynchronize(m->stream), "finalize sync")) return r;
    cudaFree(m->stage);
    m->stage = nullptr;
    m->stage_bytes = 0;
    if (m->use_step)
        if (int r = build_step(m)) return r;
    // Capture one decode step.
    if (int r = cuda_status(cudaStreamBeginCapture(m->stream, cudaStreamCaptureModeThreadLocal), "begin capture"))
        return r;
    const int rs = m->use_step ? enqueue_step_persistent(m, m->stream) : enqueue_step(m, m->stream);
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamEndCapture(m->stream, &g);
    if (rs) {
        if (g) cudaGraphDestroy(g);
        return rs;
    }
    if (int r = cuda_status(e, "end capture")) return r;
    m->graph = g;
    if (int r = cuda_status(cudaGraphInstantiate(&m->exec, g, 0), "graph instantiate")) return r;
    m->finalized = true;
    return DK_OK;
}

int dk_model_set_tokens(dk_model *m, const int *tokens, int n_tokens, int n_forced) {
    if (int r = need(m)) return r;
    if (n_tokens < 0 || n_tokens > m->seq_len + 1 || n_forced < 0)
        return set_error(DK_ERR_INVALID, "dk_model_set_tokens: bad sizes");
    for (int i = 0; i < n_tokens; ++i)
        if (tokens[i] < 0 || tokens[i] >= m->vocab)
            return set_error(DK_ERR_INVALID, "dk_model_set_tokens: token %d out of range", tokens[i]);
    if (n_tokens && cudaMemcpyAsync(m->tokens, tokens, (size_t)n_tokens * 4, cudaMemcpyHostToDevice, m->stream))
        return set_error(DK_ERR_CUDA, "dk_model_set_tokens: copy failed");
    m->h_small[0] = n_forced;
    if (int r = cuda_status(cudaMemcpyAsync(m->n_forced, m->h_small, 4, cudaMemcpyHostToDevice, m->stream), "n_forced"))
        return r;
    return cuda_status(cudaStreamSynchronize(m->stream), "dk_model_set_tokens");
}

int dk_model_enqueue_steps(dk_model *m, int pos0, int n_steps) {
    if (int r = need(m)) return r;
    if (!m->finalized) return set_error(DK_ERR_STATE, "dk_model_enqueue_steps: model not finalized");
    if (pos0 < 0 || n_steps < 0 || pos0 + n_steps > m->seq_len)
        return set_error(DK_ERR_INVALID, "dk_model_enqueue_steps: positions [%d, %d) exceed seq_len %d", pos0,
                         pos0 + n_steps, m->seq_len);
    m->h_small[1] = pos0;
    if (int r = cuda_status(cudaMemcpyAsync(m->pos, m->h_small + 1, 4, cudaMemcpyHostToDevice, m->stream), "pos"))
        return r;
    for (int i = 0; i < n_steps; ++i)
        if (int r = cuda_status(cudaGraphLaunch(m->exec, m->stream), "graph launch")) return r;
    return DK_OK;
}

int dk_model_get_tokens(dk_model *m, int *tokens, int n_tokens) {
    if (int r = need(m)) return r;
    if (n_tokens < 0 || n_tokens > m->seq_len + 1) return set_error(DK_ERR_INVALID, "dk_model_get_tokens: bad size");
    if (int r = cuda_status(cudaMemcpyAsync(tokens, m->tokens, (size_t)n_tokens * 4, cudaMemcpyDeviceToHost, m->stream),
                            "token readback"))
        return r;
    return cuda_status(cudaStreamSynchronize(m->stream), "token readback sync");
}

int dk_model_sync(dk_model *m) {
    if (int r = need(m)) return r;
    return cuda_status(cudaStreamSynchronize(m->stream), "dk_model_sync");
}

void *dk_model_stream(dk_model *m) { return m ? (void *)m->stream : nullptr; }

int dk_model_device_error(dk_model *m) {
    if (need(m)) return DK_ERR_CUDA;
    int v = 0;
    if (cudaMemcpyAsync(m->h_small + 2, m->err, 4, cudaMemcpyDeviceToHost, m->stream) != cudaSuccess) return DK_ERR_CUDA;
    if (cudaStreamSynchronize(m->stream) != cudaSuccess) return DK_ERR_CUDA;
    v = m->h_small[2];
    return v;
}

int dk_model_kernels_per_step(dk_model *m) { return m ? m->kernels_per_step : 0; }

int dk_model_trace(dk_model *m, unsigned long long *out, size_t n, int *grid, int *n_ops) {
    if (int r = need(m)) return r;
    if (grid) *grid = m->num_sms;
    if (n_ops) *n_ops = m->n_ops;
    if (!m->d_trace) return set_error(DK_ERR_STATE, "dk_model_trace: tracing is off (DIOLKOS_STEP_TRACE=1 at creation)");
    size_t total = (size_t)m->num_sms * m->n_ops * 8;
    if (!out || n < total) return set_error(DK_ERR_INVALID, "dk_model_trace: need %zu entries", total);
    if (n >= total + kStageTraceEntries) total += kStageTraceEntries;  // the per-stage timeline too
    return cuda_status(cudaMemcpy(out, m->d_trace, total * 8, cudaMemcpyDeviceToHost), "dk_model_trace");
}

// Diagnostics layout: GEMV op k (step order) with n_k input columns occupies, at 256-byte aligned
// offsets, n_k floats of input, n_k int8 values and n_k/32 float scales.
static size_t dump_layout(const dk_model *m, std::vector<size_t> *off) {
    size_t o = 0;
    for (int i : m->dump_ops) {
        const size_t n = (size_t)m->h_ops[i].g.n;
        if (off) off->push_back(o);
        o += align256(4 * n) + align256(n) + align256(n / 8);
    }
    return o;
}

int dk_model_dump_enable(dk_model *m, int on) {
    if (int r = need(m)) return r;
    if (!m->finalized || !m->use_step)
        return set_error(DK_ERR_STATE, "dk_model_dump_enable: needs a finalized model on the persistent step");
    if (int r = cuda_status(cudaStreamSynchronize(m->stream), "dk_model_dump_enable: sync")) return r;
    std::vector<size_t> off;
    const size_t bytes = dump_layout(m, &off);
    if (on && !m->dump) {
        if (cudaMalloc(&m->dump, bytes) != cudaSuccess) return set_error(DK_ERR_NOMEM, "dk_model_dump_enable");
        if (int r = cuda_status(cudaMemset(m->dump, 0, bytes), "dk_model_dump_enable: clear")) return r;
    }
    std::vector<StepOp> ops = m->h_ops;
    for (size_t k = 0; k < m->dump_ops.size(); ++k) {
        GemvArgs &a = ops[m->dump_ops[k]].g;
        const size_t n = (size_t)a.n;
        a.dump_in = on ? reinterpret_cast<float *>(m->dump + off[k]) : nullptr;
        a.dump_q = on ? reinterpret_cast<int8_t *>(m->dump + off[k] + align256(4 * n)) : nullptr;
        a.dump_s = on ? reinterpret_cast<float *>(m->dump + off[k] + align256(4 * n) + align256(n)) : nullptr;
    }
    // The captured graph reads the op list from this device array at every launch.
    return cuda_status(cudaMemcpy(m->d_ops, ops.data(), ops.size() * sizeof(StepOp), cudaMemcpyHostToDevice),
                       "dk_model_dump_enable: op upload");
}

int dk_model_dump_read(dk_model *m, float *in, int8_t *q, float *s) {
    if (int r = need(m)) return r;
    if (!m->dump) return set_error(DK_ERR_STATE, "dk_model_dump_read: dumps are off (dk_model_dump_enable)");
    std::vector<size_t> off;
    const size_t bytes = dump_layout(m, &off);
    std::vector<uint8_t> h(bytes);
    if (int r = cuda_status(cudaStreamSynchronize(m->stream), "dk_model_dump_read: sync")) return r;
    if (int r = cuda_status(cudaMemcpy(h.data(), m->dump, bytes, cudaMemcpyDeviceToHost), "dk_model_dump_read")) return r;
    size_t e = 0;
    for (size_t k = 0; k < m->dump_ops.size(); ++k) {
        const size_t n = (size_t)m->h_ops[m->dump_ops[k]].g.n;
        if (in) memcpy(in + e, h.data() + off[k], 4 * n);
        if (q) memcpy(q + e, h.data() + off[k] + align256(4 * n), n);
        if (s) memcpy(s + e / 32, h.data() + off[k] + align256(4 * n) + align256(n), n / 8);
        e += n;
    }
    return DK_OK;
}

int dk_model_kv_write(dk_model *m, int layer, int pos0, int n_pos, const void *k, const void *v, int src_type) {
    if (int r = need(m)) return r;
    if (layer < 0 || layer >= m->n_layers || pos0 < 0 || n_pos < 0 || pos0 + n_pos > m->seq_len || !k || !v ||
        (src_type != DK_KV_BF16 && src_type != DK_KV_F32))
        return set_error(DK_ERR_INVALID, "dk_model_kv_write: bad arguments");
    if (n_pos == 0) return DK_OK;
    if (int r = cuda_status(cudaStreamSynchronize(m->stream), "dk_model_kv_write: sync")) return r;
    const size_t esz = m->kv_type == DK_KV_F32 ? 4 : 2;
    const int hs = m->hs, kvd = m->kv_dim;
    // this rank's KV heads, [head][position][hs] in the cache's element type
    std::vector<uint8_t> buf((size_t)m->l_kv_heads * n_pos * hs * esz);
    for (int w = 0; w < 2; ++w) {
        const void *src = w == 0 ? k : v;
        for (int h = 0; h < m->l_kv_heads; ++h) {
            const int hg = m->rank * m->l_kv_heads + h;
            for (int p = 0; p < n_pos; ++p)
                for (int d = 0; d < hs; ++d) {
                    const size_t from = (size_t)p * kvd + (size_t)hg * hs + d;
                    uint32_t u;  // the value's fp32 bits
                    if (src_type == DK_KV_BF16) u = (uint32_t)static_cast<const uint16_t *>(src)[from] << 16;
                    else memcpy(&u, static_cast<const float *>(src) + from, 4);
                    const size_t at = ((size_t)h * n_pos + p) * hs + d;
                    if (esz == 2) reinterpret_cast<uint16_t *>(buf.data())[at] = (uint16_t)(u >> 16);  // truncation
                    else memcpy(buf.data() + 4 * at, &u, 4);
                }
        }
        uint8_t *base = static_cast<uint8_t *>(w == 0 ? m->kcache : m->vcache) + (size_t)layer * m->kv_layer_elems * esz;
        for (int h = 0; h < m->l_kv_heads; ++h)
            if (int r = cuda_status(cudaMemcpyAsync(base + ((size_t)h * m->seq_len + pos0) * hs * esz,
                                                    buf.data() + (size_t)h * n_pos * hs * esz, (size_t)n_pos * hs * esz,
                                                    cudaMemcpyHostToDevice, m->stream),
                                    "dk_model_kv_write"))
                return r;
        // stream order puts the rows before the next step; the host buffer must outlive the copies
        if (int r = cuda_status(cudaStreamSynchronize(m->stream), "dk_model_kv_write: sync")) return r;
    }
    return DK_OK;
}

int dk_model_kv_read(dk_model *m, int layer, int pos0, int n_pos, void *k, void *v) {
    if (int r = need(m)) return r;
    if (layer < 0 || layer >= m->n_layers || pos0 < 0 || n_pos < 0 || pos0 + n_pos > m->seq_len || !k || !v)
        return set_error(DK_ERR_INVALID, "dk_model_kv_read: bad arguments");
    if (n_pos == 0) return DK_OK;
    const size_t esz = m->kv_type == DK_KV_F32 ? 4 : 2;
    const int hs = m->hs, lkvd = m->l_kv_heads * hs;
    std::vector<uint8_t> buf((size_t)m->l_kv_heads * n_pos * hs * esz);
    for (int w = 0; w < 2; ++w) {
        const uint8_t *base =
            static_cast<const uint8_t *>(w == 0 ? m->kcache : m->vcache) + (size_t)layer * m->kv_layer_elems * esz;
        for (int h = 0; h < m->l_kv_heads; ++h)
            if (int r = cuda_status(cudaMemcpyAsync(buf.data() + (size_t)h * n_pos * hs * esz,
                                                    base + ((size_t)h * m->seq_len + pos0) * hs * esz,
                                                    (size_t)n_pos * hs * esz, cudaMemcpyDeviceToHost, m->stream),
                                    "dk_model_kv_read"))
                return r;
        if (int r = cuda_status(cudaStreamSynchronize(m->stream), "dk_model_kv_read: sync")) return r;
        uint8_t *dst = static_cast<uint8_t *>(w == 0 ? k : v);
        for (int h = 0; h < m->l_kv_heads; ++h)
            for (int p = 0; p < n_pos; ++p)
                memcpy(dst + ((size_t)p * lkvd + (size_t)h * hs) * esz, buf.data() + ((size_t)h * n_pos + p) * hs * esz,
                       (size_t)hs * esz);
    }
    return DK_OK;
}

size_t dk_model_weight_bytes(dk_model *m) {
    if (!m) return 0;
    // Bytes the GEMVs of one step stream on this rank (pad rows included): every layer's four
    // matrices + the classifier rows.
    const size_t per_layer = q8_packed_bytes(m->dim, m->l_dim + 2 * m->l_kv_dim, m->p_qkv.T) +
                             q8_packed_bytes(m->l_dim, m->dim, m->p_wo.T) +
                             q8_packed_bytes(m->dim, 2 * m->l_hidden, m->p_w13.T) +
                             q8_packed_bytes(m->l_hidden, m->dim, m->p_w2.T);
    return per_layer * m->n_layers + q8_packed_bytes(m->dim, m->l_vocab, m->p_cls.T);
}

int dk_model_forward(dk_model *m, int token, int pos, float *logits) {
    if (int r = need(m)) return r;
    if (!m->finalized) return set_error(DK_ERR_STATE, "dk_model_forward: model not finalized");
    if (pos < 0 || pos >= m->seq_len) return set_error(DK_ERR_INVALID, "dk_model_forward: pos %d out of range", pos);
    if (token < 0 || token >= m->vocab) return set_error(DK_ERR_INVALID, "dk_model_forward: token %d out of range", token);
    m->h_small[8] = token;
    m->h_small[9] = pos;
    m->h_small[10] = m->seq_len + 1;  // nothing forced: the argmax is written but not used
    cudaStream_t st = m->stream;
    if (cudaMemcpyAsync(m->tokens + pos, m->h_small + 8, 4, cudaMemcpyHostToDevice, st) ||
        cudaMemcpyAsync(m->pos, m->h_small + 9, 4, cudaMemcpyHostToDevice, st) ||
        cudaMemcpyAsync(m->n_forced, m->h_small + 10, 4, cudaMemcpyHostToDevice, st))
        return set_error(DK_ERR_CUDA, "dk_model_forward: step upload failed");
    if (int r = cuda_status(cudaGraphLaunch(m->exec, st), "graph launch")) return r;
    if (logits) {
        if (int r = cuda_status(cudaMemcpyAsync(logits + m->vocab_off, m->logits, (size_t)m->l_vocab * 4,
                                                cudaMemcpyDeviceToHost, st),
                                "logits readback"))
            return r;
    }
    if (int r = cuda_status(cudaStreamSynchronize(st), "dk_model_forward")) return r;
    const int dev_err = dk_model_device_error(m);
    if (dev_err) return set_error(dev_err, "dk_model_forward: device error word 0x%x", dev_err);
    return DK_OK;
}

static bool prefill_available(const dk_model *m) {
    return m->use_step && (m->world == 1 || (m->connected && !m->prefill_broken));
}

static int prefill_alloc(dk_model *m) {
    if (m->pchunk) return DK_OK;  // set last, once everything below succeeded
    // a previous attempt that failed part-way: start over
    cudaFree(m->parena);
    m->parena = nullptr;
    if (m->h_groups) cudaFreeHost(m->h_groups);
    m->h_groups = nullptr;
    for (cudaEvent_t e : m->pslot_done)
        if (e) cudaEventDestroy(e);
    m->pslot_done.clear();
    const int C = std::min(kPrefillChunk, m->seq_len);
    const int qkv_rows = m->l_dim + 2 * m->l_kv_dim;
    const int nmax = std::max(std::max(m->dim, m->l_dim), m->l_hidden);
    m->pwork_stride = (size_t)m->l_heads * m->step_splits * (m->hs + 2);
    m->pcount_stride = (size_t)m->l_kv_heads;
    const size_t sz_x = align256((size_t)C * m->dim * 4), sz_qkv = align256((size_t)C * qkv_rows * 4);
    const size_t sz_xb = align256((size_t)C * m->l_dim * 4), sz_hb = align256((size_t)C * m->l_hidden * 4);
    const size_t sz_xq = align256((size_t)C * nmax), sz_xs = align256((size_t)C * (nmax / 32) * 4);
    const size_t sz_work = align256((size_t)C * m->pwork_stride * 4), sz_cnt = align256((size_t)C * m->pcount_stride * 4);
    const size_t sz_groups = align256((size_t)C * sizeof(PrefillGroup));
    const size_t sz_ppart = m->world > 1 ? align256((size_t)C * m->dim * 4) : 0;
    const size_t total = sz_x + sz_qkv + sz_xb + sz_hb + sz_xq + sz_xs + sz_work + sz_cnt + sz_groups + sz_ppart;
    if (cudaMalloc(&m->parena, total) != cudaSuccess) {
        m->parena = nullptr;
        return set_error(DK_ERR_NOMEM, "prefill: %zu bytes of scratch", total);
    }
    // the attention counters must start at zero (each position's merging split resets its own)
    if (int r = cuda_status(cudaMemsetAsync(m->parena, 0, total, m->stream), "prefill scratch clear")) return r;
    uint8_t *p = m->parena;
    m->px = reinterpret_cast<float *>(p); p += sz_x;
    m->pqkv = reinterpret_cast<float *>(p); p += sz_qkv;
    m->pxb = reinterpret_cast<float *>(p); p += sz_xb;
    m->phb = reinterpret_cast<float *>(p); p += sz_hb;
    m->pxq = reinterpret_cast<int8_t *>(p); p += sz_xq;
    m->pxs = reinterpret_cast<float *>(p); p += sz_xs;
    m->pwork = reinterpret_cast<float *>(p); p += sz_work;
    m->pcount = reinterpret_cast<unsigned *>(p); p += sz_cnt;
    m->pgroups = reinterpret_cast<PrefillGroup *>(p); p += sz_groups;
    m->ppart = sz_ppart ? reinterpret_cast<float *>(p) : nullptr;
    // the group tables go up from pinned memory (a pageable source may synchronise the stream)
    m->pslots = (m->seq_len + C - 1) / C;
    if (cudaMallocHost(&m->h_groups, (size_t)m->pslots * C * sizeof(PrefillGroup)) != cudaSuccess) {
        m->h_groups = nullptr;
        return set_error(DK_ERR_NOMEM, "prefill: pinned group tables");
    }
    m->pslot_done.assign(m->pslots, nullptr);
    for (auto &e : m->pslot_done)
        if (int r = cuda_status(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "prefill: slot event")) return r;
    m->pchunk = C;
    return DK_OK;
}

// One chunk of the prompt: positions pos0 .. pos0+n-1 through every layer.  The same arithmetic as the
// decode step at each of those positions (the reference runs forward() once per prompt token,
// src/transformer.c:61-232): Q8_0 activations from the step's own prologue code, the matmuls on the
// tensor cores with the GEMV's summation order, RoPE / KV-cache writes and attention from the step's
// attention items with the step's split plan -- so the cache entries are the decode step's, bit for
// bit, and decoding continues from pos0+n as if every prompt token had been stepped.
static int prefill_chunk(dk_model *m, int pos0, int n, cudaStream_t st) {
    const int qkv_rows = m->l_dim + 2 * m->l_kv_dim;
    const size_t esz = m->kv_type == DK_KV_F32 ? 4 : 2;
    auto act = [&](int pro, const float *x, const float *norm, int cols) -> cudaError_t {
        GemvArgs a;
        a.n = cols; a.pro = pro; a.x = x; a.norm_w = norm; a.emb = m->emb; a.emb_T = m->emb_T;
        a.vocab = m->vocab; a.err = m->err;
        return launch_prefill_act(a, n, m->tokens + pos0, m->pxq, m->pxs, st);
    };
    // Tensor parallel: the wo / w2 partial rows (this rank's columns) go to every rank; once all ranks'
    // rows are in, x += (partial_0 + partial_1 + ...) in rank order -- the decode step's reduce.
    const bool tp = m->world > 1;
    const int C = m->pchunk;
    auto exchange = [&](int par) -> cudaError_t {
        const size_t nf = (size_t)n * m->dim;
        cudaError_t e = launch_prefill_scatter(m->ppart, reinterpret_cast<float *const *>(m->d_ptrs + 8 * (6 + par)),
                                               m->world, (size_t)m->rank * C * m->dim, nf, st);
        if (!e) e = launch_prefill_signal(reinterpret_cast<unsigned long long *const *>(m->d_ptrs + 8 * (8 + par)),
                                          m->world, st);
        // The counter target counts only exchanges whose signal was enqueued: every peer counts the same ones.
        if (!e) m->pex[par] += 1;
        if (!e) e = launch_prefill_wait(reinterpret_cast<const unsigned long long *>(m->comm + comm_pcnt_off(m, par)),
                                        m->pex[par] * (unsigned long long)m->world, m->err, st);
        if (!e) e = launch_prefill_reduce(m->px, reinterpret_cast<const float *>(m->comm + comm_pre_off(m, par)),
                                          (size_t)C * m->dim, m->world, nf, st);
        // After a failed exchange this rank's count may no longer match its peers': later prefills would wait
        // for a wrong target, so tensor-parallel prefill is refused from here on.
        if (e) m->prefill_broken = true;
        return e;
    };
    auto mm = [&](const uint8_t *w, int cols, int rows, int T, int epi, float *out) -> cudaError_t {
        GemmArgs g;
        g.w = w; g.n = cols; g.d = rows; g.T = T; g.xq = m->pxq; g.xs = m->pxs; g.ntok = n; g.epi = epi;
        g.out = out; g.err = m->err;
        return launch_gemm(g, st);
    };
    AttnArgs t;
    t.qkv = m->pqkv; t.rope = m->rope;
    t.out = m->pxb; t.work = m->pwork; t.count = m->pcount; t.pos = m->pos;
    t.n_heads = m->l_heads; t.n_kv_heads = m->l_kv_heads; t.head_size = m->hs; t.seq_len = m->seq_len;
    t.kv_f32 = m->kv_type == DK_KV_F32; step_attn_fields(m, t); t.err = m->err;
    // the attention's position groups (the same for every layer), planned into this chunk's pinned slot
    // once that slot's previous upload is done; stream order keeps the upload behind the previous
    // chunk's kernels
    const int slot = (pos0 / C) % m->pslots;
    PrefillGroup *hg = m->h_groups + (size_t)slot * C;
    if (int r = cuda_status(cudaEventSynchronize(m->pslot_done[slot]), "prefill: group slot")) return r;
    long long items = 0, narrow_items = 0;
    const int ngroups = prefill_attn_plan(t, pos0, n, hg, &items, &narrow_items);
    if (int r = cuda_status(cudaMemcpyAsync(m->pgroups, hg, (size_t)ngroups * sizeof(PrefillGroup),
                                            cudaMemcpyHostToDevice, st),
                            "prefill: group table"))
        return r;
    if (int r = cuda_status(cudaEventRecord(m->pslot_done[slot], st), "prefill: group slot")) return r;
    for (int l = 0; l < m->n_layers; ++l) {
        const dk_layer &ly = m->layers[l];
        cudaError_t e = act(l == 0 ? PRO_EMB_RMS : PRO_RMS, m->px, ly.rms_att, m->dim);
        if (!e) e = mm(ly.wqkv, m->dim, qkv_rows, m->p_qkv.T, EPI_STORE, m->pqkv);
        t.k_cache = static_cast<uint8_t *>(m->kcache) + (size_t)l * m->kv_layer_elems * esz;
        t.v_cache = static_cast<uint8_t *>(m->vcache) + (size_t)l * m->kv_layer_elems * esz;
        if (!e) e = launch_prefill_kv(t, pos0, n, (size_t)qkv_rows, st);
        // The last layer's attention and MLP feed only these positions' logits, which nothing reads: the
        // decode step recomputes the last prompt position.  Its K/V rows are all that is kept.
        if (!e && l == m->n_layers - 1) break;
        if (!e) e = launch_prefill_attn(t, pos0, m->pgroups, ngroups, items, narrow_items, (size_t)qkv_rows, (size_t)m->l_dim,
                                        m->pwork_stride, m->pcount_stride, st);
        if (!e) e = act(PRO_F32, m->pxb, nullptr, m->l_dim);
        if (!e) e = tp ? mm(ly.wo, m->l_dim, m->dim, m->p_wo.T, EPI_STORE, m->ppart)
                       : mm(ly.wo, m->l_dim, m->dim, m->p_wo.T, EPI_ADD, m->px);
        if (!e && tp) e = exchange(0);
        if (!e) e = act(PRO_RMS, m->px, ly.rms_ffn, m->dim);
        if (!e) e = mm(ly.w13, m->dim, 2 * m->l_hidden, m->p_w13.T, EPI_SWIGLU, m->phb);
        if (!e) e = act(PRO_F32, m->phb, nullptr, m->l_hidden);
        if (!e) e = tp ? mm(ly.w2, m->l_hidden, m->dim, m->p_w2.T, EPI_STORE, m->ppart)
                       : mm(ly.w2, m->l_hidden, m->dim, m->p_w2.T, EPI_ADD, m->px);
        if (!e && tp) e = exchange(1);
        if (e) return set_error(DK_ERR_CUDA, "prefill layer %d: %s", l, cudaGetErrorString(e));
    }
    return DK_OK;
}

// Enqueues the prefill of positions [pos0, pos0 + n) in chunks (no synchronisation).
static int enqueue_prefill(dk_model *m, int pos0, int n) {
    if (int r = prefill_alloc(m)) return r;
    for (int c = 0; c < n; c += m->pchunk)
        if (int r = prefill_chunk(m, pos0 + c, std::min(m->pchunk, n - c), m->stream)) return r;
    return DK_OK;
}

int dk_model_prefill(dk_model *m, int pos0, int n_positions) {
    if (int r = need(m)) return r;
    if (!m->finalized) return set_error(DK_ERR_STATE, "dk_model_prefill: model not finalized");
    if (!prefill_available(m))
        return set_error(DK_ERR_STATE, "dk_model_prefill: needs the persistent step (and connected ranks whose prefill exchanges never failed)");
    if (pos0 < 0 || n_positions < 0 || pos0 + n_positions > m->seq_len)
        return set_error(DK_ERR_INVALID, "dk_model_prefill: positions [%d, %d) exceed seq_len %d", pos0,
                         pos0 + n_positions, m->seq_len);
    if (n_positions == 0) return DK_OK;
    return enqueue_prefill(m, pos0, n_positions);
}

int dk_model_generate(dk_model *m, const int *prompt, int n_prompt, int steps, int *out, int *n_out) {
    if (int r = need(m)) return r;
    if (!m->finalized) return set_error(DK_ERR_STATE, "dk_model_generate: model not finalized");
    if (!prompt || n_prompt < 1) return set_error(DK_ERR_INVALID, "dk_model_generate: expected at least 1 prompt token");
    if (steps > m->seq_len) steps = m->seq_len;
    if (steps < 0) steps = 0;
    for (int i = 0; i < n_prompt; ++i)
        if (prompt[i] < 0 || prompt[i] >= m->vocab)
            return set_error(DK_ERR_INVALID, "dk_model_generate: prompt token %d out of range", prompt[i]);
    const int nt = n_prompt < m->seq_len + 1 ? n_prompt : m->seq_len + 1;
    if (int r = dk_model_set_tokens(m, prompt, nt, n_prompt)) return r;
    // The prompt positions whose next token is forced (all but the last prompt token) go through the
    // batched prefill; the decode steps continue from there.  DIOLKOS_PREFILL=0 steps them one by one.
    int pre = 0;
    if (prefill_available(m)) {
        const char *e = getenv("DIOLKOS_PREFILL");
        if (!(e && strcmp(e, "0") == 0)) pre = std::min(n_prompt - 1, steps);
    }
    if (pre > 0)
        if (int r = enqueue_prefill(m, 0, pre)) return r;
    if (int r = dk_model_enqueue_steps(m, pre, steps - pre)) return r;
    std::vector<int> toks((size_t)steps + 1);
    if (int r = dk_model_get_tokens(m, toks.data(), steps + 1)) return r;
    const int dev_err = dk_model_device_error(m);
    if (dev_err) return set_error(dev_err, "dk_model_generate: device error word 0x%x", dev_err);
    // Replay the reference loop's bookkeeping on the tokens the device produced.
    int count = 0;
    for (int pos = 0; pos < steps; ++pos) {
        int next;
        if (pos < n_prompt - 1) {
            next = prompt[pos + 1];
        } else {
            next = toks[(size_t)pos + 1];
            if (out) out[count] = next;
            ++count;
        }
        if (next == 1) break;
    }
    if (n_out) *n_out = count;
    return DK_OK;
}

}  // extern "C"
