// api.cpp -- the C ABI of include/jeromoe.h: contexts, HBM admission, layer
// upload into the device layout, and the batched forward.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <memory>
#include <mutex>
#include <string>
#include <cmath>
#include <vector>

#include "../../include/jeromoe.h"
#include "ep_p2p.h"
#include "ep_plan.h"
#include "kernels.h"
#include "layout.h"
#include "moe_device.h"
#include "nccl_dl.h"

using namespace jmoe;

namespace {

thread_local std::string g_last_error;

constexpr int kMaxExperts = 256;
constexpr int kMaxTopK = 16;
constexpr int kMaxGroups = 32;

struct LayerStore {
    bool present = false;
    int H = 0, E = 0, k = 0, I = 0, S = 0;
    int route_mode = 0, normalize = 1, n_groups = 0, topk_groups = 0;
    float routed_scale = 1.0f;
    void *block = nullptr;          // one cudaMalloc for the whole layer
    size_t block_bytes = 0, gguf_bytes = 0;
    const float *router = nullptr, *logit_bias = nullptr, *sel_bias = nullptr;
    float *ffn_norm = nullptr;      // moe_layer_set_ffn_norm: RMSNorm weight [H] (own allocation)
    float norm_eps = 0.0f;
    LayerDev dev{};
    LayerMaps maps{};
};

struct Scratch {
    void *block = nullptr;
    size_t bytes = 0;
    // capacities this block was carved for
    int Tm = 0, H = 0, E = 0, k = 0, W = 0;
    bool af = false;
    float *x = nullptr, *out = nullptr;
    int8_t *xq = nullptr;
    float *xd = nullptr, *xs = nullptr, *logits = nullptr, *sel_w = nullptr;
    int32_t *sel_idx = nullptr;
    int *sync = nullptr;
    uint32_t *mask = nullptr;
    int32_t *wprefix = nullptr, *offsets = nullptr, *perm_token = nullptr, *n_active = nullptr, *slot_of = nullptr;
    Problem *problems = nullptr;
    int8_t *aq = nullptr;
    float *ad = nullptr, *as = nullptr, *af_buf = nullptr, *y = nullptr;
    int *err = nullptr;
    int32_t *tile_off = nullptr;
    void *a16 = nullptr, *a16dn = nullptr;   // tensor-core path operands (f16)
    void *x16 = nullptr;                     // fused small-batch launch: f16 token rows
    int32_t *dep = nullptr;                  // fused expert launch: chunk counters, then the CTA ticket
    int dep_cap = 0;
    bool tc = false;
    int slots_cap = 0;
};

}  // namespace

namespace {

// CUDA events recorded after each kernel of a forward while profiling is on;
// folded into per-kernel totals by moe_profile_read.
struct Profiler {
    bool on = false;
    cudaStream_t stream = nullptr;
    std::vector<cudaEvent_t> pool;
    size_t used = 0;
    std::vector<std::pair<const char *, cudaEvent_t>> marks;   // name == nullptr: forward begins
    int forwards = 0;
    std::vector<std::pair<std::string, std::pair<double, int64_t>>> totals;

    static void mark_cb(void *user, const char *kernel)
    {
        Profiler *p = static_cast<Profiler *>(user);
        if (p->used == p->pool.size()) {
            cudaEvent_t ev;
            if (cudaEventCreate(&ev) != cudaSuccess) return;
            p->pool.push_back(ev);
        }
        cudaEvent_t ev = p->pool[p->used++];
        if (cudaEventRecord(ev, p->stream) != cudaSuccess) return;
        p->marks.emplace_back(kernel, ev);
        if (!kernel) p->forwards++;
    }

    void add(const char *name, double ms)
    {
        for (auto &t : totals)
            if (t.first == name) { t.second.first += ms; t.second.second++; return; }
        totals.push_back({name, {ms, 1}});
    }

    void release()
    {
        for (auto ev : pool) cudaEventDestroy(ev);
        pool.clear();
        marks.clear();
        used = 0;
    }
};

}  // namespace

namespace {

// Bound of each peer-flag wait of the peer-memory exchange (about 2 s at 2 GHz).
constexpr long long kEpWaitCycles = 4000000000LL;

// Expert-parallel state of a context: the communicator and a device arena for
// the exchange buffers and the local expert stage, grown on demand.
struct EpState {
    int rank = 0, world = 0;   // world == 0: not in expert-parallel mode
    ncclComm_t comm = nullptr;
    void *arena = nullptr;
    size_t arena_bytes = 0;
    int rows_cap = 0, send_cap = 0, H = 0, W = 0, E = 0;   // dims the arena was carved for
    bool tc = false;
    int32_t *all_off = nullptr;   // [world][E+1]
    uint8_t *send_buf = nullptr, *recv_buf = nullptr;
    int8_t *xq = nullptr;
    float *xd = nullptr, *xs = nullptr;
    int32_t *perm = nullptr;      // local slot -> received row
    uint8_t *plan_dev = nullptr;  // n_active | problems | segments (one upload)
    int8_t *aq = nullptr;
    float *ad = nullptr, *as = nullptr, *y = nullptr;
    int32_t *tile_off = nullptr, *zero = nullptr;
    void *a16 = nullptr, *a16dn = nullptr;
    int32_t *h_off = nullptr;     // pinned: all-gathered offsets
    uint8_t *h_plan = nullptr;    // pinned: plan upload staging
    size_t h_off_bytes = 0, h_plan_bytes = 0;
    uint8_t *small = nullptr;     // device: set-up all-gathers (flags, IPC handles)
    // exchange over peer memory (batches up to kEpP2PMaxTokens per rank)
    int p2p_state = 0;            // 0 not set up, 1 ready, -1 off for the current dims
    EpP2PLayout p2p{};
    uint8_t *p2p_arena = nullptr;
    uint8_t *p2p_peer[kEpMaxRanks] = {};
    uint32_t p2p_epoch = 0;
    bool p2p_broken = false;      // a flag wait failed: unusable until moe_ep_reset
    uint32_t dbg_skew = 0;        // test hook (moe_debug_ep_fault): the next forward waits for a skewed epoch
    long long dbg_wait_cycles = 0;   // test hook: bound of the flag waits (0: the default)
};

}  // namespace

struct moe_ctx {
    moe_device_spec spec{};
    cudaStream_t own_stream = nullptr;
    cudaStream_t stream = nullptr;
    std::vector<LayerStore> layers;
    Scratch scratch;
    int upload_count = 0;
    std::string last_error;
    // last forward, for moe_debug_permutation
    int last_layer = -1, last_T = 0;
    int32_t *dbg_isum = nullptr;   // moe_debug_capture_block_sums
    uint64_t dbg_isum_cap = 0;
    int num_sms = 148;
    int *status_host = nullptr;   // pinned word for the device status flag
    float *stack_buf = nullptr;   // moe_prefill_ffn_layers: the hidden rows on the device
    size_t stack_buf_n = 0;
    // the LM head (moe_lm_head_upload / moe_lm_head)
    struct Head {
        bool uploaded = false;   // moe_lm_head_upload was called
        bool has = false;        // a head tensor exists (output.weight or the tied token_embd.weight)
        bool shaped = false;     // GGUF [hidden, rows]; else rows = elements / hidden
        int hidden = 0, rows = 0;
        void *block = nullptr;   // the head in device layout
        DevMatrix m{};
        MatMaps maps{};
        void *buf = nullptr;     // call buffers
        size_t buf_bytes = 0;
        int *errw = nullptr;     // the status word at the start of buf
        MatMaps maps_tc{};       // tensor-core boxes (128 rows), when tc
        bool tc = false;         // the head suits the int8 tensor-core down launch
    } head;
    Profiler prof;
    EpState ep;
};

namespace {

int fail(moe_ctx *ctx, int code, const char *fmt, ...)
{
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    if (ctx) ctx->last_error = buf;
    g_last_error = buf;
    return code;
}

int cuda_fail(moe_ctx *ctx, cudaError_t e, const char *what)
{
    return fail(ctx, MOE_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

#define CUDA_TRY(ctx, call, what)                            \
    do {                                                     \
        cudaError_t e_ = (call);                             \
        if (e_ != cudaSuccess) return cuda_fail(ctx, e_, what); \
    } while (0)

// ------------------------------------------------------------ validation

struct MatSpec {
    int type = 0, rows = 0, cols = 0, experts = 0;
    const uint8_t *data = nullptr;
    bool present = false;
};

const char *quant_name(int q)
{
    switch (q) {
    case MOE_QUANT_F32: return "F32";
    case MOE_QUANT_Q8_0: return "Q8_0";
    case MOE_QUANT_Q4_K: return "Q4_K";
    default: return "unsupported";
    }
}

// A GGUF tensor [in, out(, E)] -> rows = out, cols = in.
int check_tensor(moe_ctx *ctx, const moe_tensor &t, const char *name, int want_dims, int cols, int experts,
                 MatSpec *out)
{
    out->present = t.data != nullptr;
    if (!out->present) return MOE_OK;
    if (t.quant != MOE_QUANT_F32 && t.quant != MOE_QUANT_Q8_0 && t.quant != MOE_QUANT_Q4_K)
        return fail(ctx, MOE_ERR_CAPABILITY_MISMATCH, "unsupported weight quantization %d for tensor '%s'",
                    t.quant, name);
    if (t.n_dims != want_dims)
        return fail(ctx, MOE_ERR_TENSOR_BOUNDS, "tensor '%s' has %d dims, expected %d", name, t.n_dims, want_dims);
    if (t.shape[0] != cols)
        return fail(ctx, MOE_ERR_TENSOR_BOUNDS, "tensor '%s' input dim %lld != %d", name, (long long)t.shape[0], cols);
    if (t.shape[1] <= 0 || t.shape[1] > (1 << 20))
        return fail(ctx, MOE_ERR_TENSOR_BOUNDS, "tensor '%s' output dim %lld out of range", name,
                    (long long)t.shape[1]);
    if (want_dims == 3 && t.shape[2] != experts)
        return fail(ctx, MOE_ERR_TENSOR_BOUNDS, "tensor '%s' holds %lld experts, expected %d", name,
                    (long long)t.shape[2], experts);
    size_t rb = gguf_row_bytes(t.quant, cols);
    if (!rb)
        return fail(ctx, MOE_ERR_CAPABILITY_MISMATCH, "tensor '%s': %d columns are not whole %s blocks", name, cols,
                    quant_name(t.quant));
    size_t need = rb * (size_t)t.shape[1] * (want_dims == 3 ? (size_t)experts : 1);
    if (t.nbytes != need)
        return fail(ctx, MOE_ERR_TENSOR_BOUNDS, "tensor '%s': %llu bytes, shape needs %llu", name,
                    (unsigned long long)t.nbytes, (unsigned long long)need);
    out->type = t.quant;
    out->rows = (int)t.shape[1];
    out->cols = cols;
    out->experts = want_dims == 3 ? experts : 1;
    out->data = static_cast<const uint8_t *>(t.data);
    return MOE_OK;
}

struct Validated {
    int H, E, k, I, S;
    MatSpec gate, up, down, sg, su, sd;
    const float *router, *logit_bias, *sel_bias;
};

int validate_desc(moe_ctx *ctx, const moe_layer_desc *d, Validated *v)
{
    if (!d) return fail(ctx, MOE_ERR_INVALID_ARGS, "null layer descriptor");
    const int H = d->hidden;
    if (H <= 0) return fail(ctx, MOE_ERR_INVALID_ARGS, "hidden must be positive");
    if (!d->router.data)
        return fail(ctx, MOE_ERR_CAPABILITY_MISMATCH,
                    "layer has no router tensor; the dense fallback stays on the host path");
    if (d->router.quant != MOE_QUANT_F32)
        return fail(ctx, MOE_ERR_CAPABILITY_MISMATCH, "router must be F32");
    if (d->router.n_dims != 2 || d->router.shape[0] != H)
        return fail(ctx, MOE_ERR_TENSOR_BOUNDS, "router shape must be [hidden, experts]");
    int E = (int)std::min<int64_t>(d->router.shape[1], d->num_experts);
    if (E <= 0 || d->top_k <= 0)
        return fail(ctx, MOE_ERR_CAPABILITY_MISMATCH, "num_experts and top_k must be positive");
    if ((uint64_t)d->router.nbytes != (uint64_t)d->router.shape[1] * H * 4)
        return fail(ctx, MOE_ERR_TENSOR_BOUNDS, "router byte length does not match its shape");
    if (E > kMaxExperts)
        return fail(ctx, MOE_ERR_CAPABILITY_MISMATCH, "%d experts exceed the supported %d", E, kMaxExperts);
    if (d->top_k > kMaxTopK || d->top_k > E)
        return fail(ctx, MOE_ERR_CAPABILITY_MISMATCH, "top_k %d unsupported (max %d, experts %d)", d->top_k,
                    kMaxTopK, E);
    if (d->route_mode == MOE_ROUTE_GROUP_LIMITED) {
        if (d->n_groups <= 1 || d->n_groups > kMaxGroups || E % d->n_groups || d->topk_groups <= 0 ||
            d->topk_groups >= d->n_groups)
            return fail(ctx, MOE_ERR_CAPABILITY_MISMATCH, "bad group-limited routing (%d groups, keep %d, %d experts)",
                        d->n_groups, d->topk_groups, E);
        if (d->top_k > d->topk_groups * (E / d->n_groups))
            return fail(ctx, MOE_ERR_CAPABILITY_MISMATCH, "top_k exceeds the experts of the kept groups");
    } else if (d->route_mode != MOE_ROUTE_SOFTMAX_TOPK) {
        return fail(ctx, MOE_ERR_INVALID_ARGS, "unknown route_mode %d", d->route_mode);
    }
    for (const moe_tensor *b : {&d->exp_probs_b, &d->logit_bias}) {
        if (b->data && (b->quant != MOE_QUANT_F32 || b->nbytes < (uint64_t)E * 4))
            return fail(ctx, MOE_ERR_TENSOR_BOUNDS, "router bias must be F32 with at least %d values", E);
    }
    int rc;
    if ((rc = check_tensor(ctx, d->gate_exps, "ffn_gate_exps", 3, H, E, &v->gate))) return rc;
    if ((rc = check_tensor(ctx, d->up_exps, "ffn_up_exps", 3, H, E, &v->up))) return rc;
    if (!v->gate.present || !v->up.present || !d->down_exps.data)
        return fail(ctx, MOE_ERR_CAPABILITY_MISMATCH,
                    "layer lacks stacked expert tensors; the dense fallback stays on the host path");
    const int I = v->gate.rows;
    if (v->up.rows != I) return fail(ctx, MOE_ERR_TENSOR_BOUNDS, "gate/up expert widths differ");
    if ((rc = check_tensor(ctx, d->down_exps, "ffn_down_exps", 3, I, E, &v->down))) return rc;
    if (v->down.rows != H) return fail(ctx, MOE_ERR_TENSOR_BOUNDS, "down expert output dim != hidden");
    if (v->gate.type != v->up.type)
        return fail(ctx, MOE_ERR_CAPABILITY_MISMATCH, "gate and up experts must share a quantization");
    if ((v->gate.type == MOE_QUANT_F32) != (v->down.type == MOE_QUANT_F32))
        return fail(ctx, MOE_ERR_CAPABILITY_MISMATCH, "F32 experts must be F32 in all three matrices");
    if (v->gate.type != MOE_QUANT_F32 && (I % 32))
        return fail(ctx, MOE_ERR_CAPABILITY_MISMATCH, "expert width %d is not a multiple of 32", I);
    int S = 0;
    v->sg = v->su = v->sd = MatSpec{};
    if (d->use_shared_expert && d->gate_shexp.data && d->up_shexp.data && d->down_shexp.data) {
        if ((rc = check_tensor(ctx, d->gate_shexp, "ffn_gate_shexp", 2, H, 1, &v->sg))) return rc;
        if ((rc = check_tensor(ctx, d->up_shexp, "ffn_up_shexp", 2, H, 1, &v->su))) return rc;
        S = v->sg.rows;
        if (v->su.rows != S) return fail(ctx, MOE_ERR_TENSOR_BOUNDS, "shared gate/up widths differ");
        if ((rc = check_tensor(ctx, d->down_shexp, "ffn_down_shexp", 2, S, 1, &v->sd))) return rc;
        if (v->sd.rows != H) return fail(ctx, MOE_ERR_TENSOR_BOUNDS, "shared down output dim != hidden");
        if (v->sg.type != v->su.type)
            return fail(ctx, MOE_ERR_CAPABILITY_MISMATCH, "shared gate and up must share a quantization");
        if ((v->sg.type == MOE_QUANT_F32) != (v->sd.type == MOE_QUANT_F32))
            return fail(ctx, MOE_ERR_CAPABILITY_MISMATCH, "F32 shared expert must be F32 in all three matrices");
        if (v->sg.type != MOE_QUANT_F32 && (S % 32))
            return fail(ctx, MOE_ERR_CAPABILITY_MISMATCH, "shared width %d is not a multiple of 32", S);
    }
    v->H = H; v->E = E; v->k = d->top_k; v->I = I; v->S = S;
    v->router = static_cast<const float *>(d->router.data);
    v->logit_bias = static_cast<const float *>(d->logit_bias.data);
    v->sel_bias = static_cast<const float *>(d->exp_probs_b.data);
    return MOE_OK;
}

// --------------------------------------------------------- device sizing

size_t layer_device_bytes(const Validated &v)
{
    size_t b = align_up((size_t)v.E * v.H * 4, 256) + 2 * align_up((size_t)v.E * 4, 256);
    auto mat = [&](const MatSpec &m) {
        if (!m.present) return (size_t)0;
        MatrixPlan p = plan_matrix(m.type, m.rows, m.cols, m.experts);
        return align_up(p.qs_bytes, 256) + align_up(p.meta_bytes, 256);
    };
    return b + mat(v.gate) + mat(v.up) + mat(v.down) + mat(v.sg) + mat(v.su) + mat(v.sd);
}

struct ScratchDims {
    int Tm, H, E, k, W;
    bool af;
    bool tc;   // buffers of the tensor-core expert path
};

// Carves the scratch block (or only measures it when base == nullptr).
size_t carve_scratch(const ScratchDims &d, uint8_t *base, Scratch *s)
{
    size_t off = 0;
    auto take = [&](size_t bytes) -> uint8_t * {
        uint8_t *p = base ? base + off : nullptr;
        off += align_up(bytes ? bytes : 1, 256);
        return p;
    };
    const size_t Tm = (size_t)std::max(d.Tm, 1), H = d.H, E = d.E, k = d.k, W = std::max(d.W, 32);
    const size_t mw = (Tm + 31) / 32, slots = Tm * k + Tm;
    const size_t maxp = std::min(E, Tm * k) + 1;
    Scratch t;
    t.x = (float *)take(Tm * H * 4);
    t.out = (float *)take(Tm * H * 4);
    t.xq = (int8_t *)take(Tm * H);
    t.xd = (float *)take(Tm * (H / 32 + 1) * 4);
    t.xs = (float *)take(Tm * (H / 32 + 1) * 4);
    t.logits = (float *)take(Tm * E * 4);
    t.sel_idx = (int32_t *)take(Tm * k * 4);
    t.sel_w = (float *)take(Tm * k * 4);
    uint8_t *sync_mask = take(kRoutingTicketBytes + E * mw * 4);   // routing tickets, then the masks (one memset)
    t.sync = (int *)sync_mask;
    t.mask = sync_mask ? (uint32_t *)(sync_mask + kRoutingTicketBytes) : nullptr;
    t.wprefix = (int32_t *)take(E * mw * 4);
    t.offsets = (int32_t *)take((E + 1) * 4);
    t.perm_token = (int32_t *)take(slots * 4);
    t.slot_of = (int32_t *)take(Tm * k * 4);
    t.problems = (Problem *)take(maxp * sizeof(Problem));
    t.n_active = (int32_t *)take(4);
    t.aq = (int8_t *)take(slots * W);
    t.ad = (float *)take(slots * (W / 32) * 4);
    t.as = (float *)take(slots * (W / 32) * 4);
    t.af_buf = d.af ? (float *)take(slots * W * 4) : nullptr;
    t.y = (float *)take(slots * H * 4);
    t.err = (int *)take(4);
    t.tile_off = (int32_t *)take(4 * (size_t)kTileOffStride * 4);
    t.a16 = d.tc ? take(slots * H * 2) : nullptr;
    // f16 operands: the down operand of both tensor-core paths, and the token
    // rows of the fused small-batch launch (batches below the prefill path)
    const size_t Tx = std::min<size_t>(Tm, MOE_TENSOR_CORE_MIN_TOKENS - 1), slots_x = Tx * k + Tx;
    t.a16dn = take((d.tc ? slots : slots_x) * W * 2);
    t.x16 = take(Tx * H * 2);
    // chunk counters: this context's forwards, and the fused launch over the
    // rows an expert-parallel forward receives (up to kEpMaxRanks sources, f16
    // items of at least 16 slots)
    t.dep_cap = std::max(dep_entries((int)Tm, (int)k, (int)E), (int)((kEpMaxRanks * Tm * k) / 16 + E + 2));
    t.dep = (int32_t *)take(((size_t)t.dep_cap + 1) * 4);
    if (s && base) {
        void *blk = s->block;
        *s = t;
        s->block = blk;
        s->Tm = d.Tm; s->H = d.H; s->E = d.E; s->k = d.k; s->W = d.W; s->af = d.af; s->tc = d.tc;
        s->slots_cap = (int)slots;
        s->bytes = off;
    }
    return off;
}

bool tc_possible(const moe_device_spec &spec)
{
    if (spec.flags & MOE_FLAG_TENSOR_CORES_NEVER) return false;
    return (spec.flags & MOE_FLAG_TENSOR_CORES_ALWAYS) || spec.max_tokens >= MOE_TENSOR_CORE_MIN_TOKENS;
}

ScratchDims scratch_dims(int Tm, const Validated &v, bool tc)
{
    ScratchDims d;
    d.Tm = Tm; d.H = v.H; d.E = v.E; d.k = v.k;
    d.W = std::max(v.I, v.S);
    d.af = v.down.type == MOE_QUANT_F32 || (v.S && v.sd.type == MOE_QUANT_F32);
    d.tc = tc && v.gate.type != MOE_QUANT_F32;
    return d;
}

// Buffers are used as dense arrays with the layer's own dims (and the
// scratch's W as the row stride of the SwiGLU buffers), so a block carved for
// dims that are all at least as large serves the layer.
bool covers(const Scratch &s, const ScratchDims &d)
{
    return s.block && s.Tm >= d.Tm && s.H >= d.H && s.E >= d.E && s.k >= d.k && s.W >= d.W && (s.af || !d.af) &&
           (s.tc || !d.tc);
}

ScratchDims merge(const Scratch &s, const ScratchDims &d)
{
    if (!s.block) return d;
    ScratchDims m = d;
    m.Tm = std::max(s.Tm, d.Tm);
    m.H = std::max(s.H, d.H);
    m.E = std::max(s.E, d.E);
    m.k = std::max(s.k, d.k);
    m.W = std::max(s.W, d.W);
    m.af = s.af || d.af;
    m.tc = s.tc || d.tc;
    return m;
}

DevMatrix to_dev(const MatrixPlan &p, const uint8_t *qs, const uint8_t *meta)
{
    DevMatrix m;
    m.type = p.type; m.rows = p.rows; m.cols = p.cols; m.n_experts = p.n_experts;
    m.qs = qs; m.meta = meta;
    m.qs_estride = p.qs_estride; m.meta_estride = p.meta_estride;
    m.qs_rstride = p.qs_rstride; m.meta_rstride = p.meta_rstride;
    return m;
}

// The tensor-core path takes quantised matrices whose rows are whole 128-row
// tiles and whose K is whole 64-value steps, when the scratch holds its buffers.
bool tc_matrix_ok(const DevMatrix &m)
{
    return (m.type == FMT_Q4_K || m.type == FMT_Q8_0) && m.rows % 128 == 0 && m.cols % 64 == 0;
}

// Batches below the f16 tensor-core path: the int8 tensor-core path
// (decode_tc.cu) from MOE_INT8_TENSOR_CORE_MIN_TOKENS tokens when the layer
// has a shared expert (all T tokens on one expert, which the streaming kernels
// re-stream per 8-token tile), Q8_0 experts, or at least six routed rows per
// expert on average; the weight-streaming kernels otherwise. Measured on B200:
// Qwen3-MoE Q4_K (E 128, top-8) streams faster up to 64 tokens (4 rows per
// expert) and the tensor cores win from 128; Q8_0 and shared-expert layers
// win on the tensor cores from 32 tokens.
bool use_int8_tc(const moe_device_spec &spec, const LayerStore &L, int T, int rows)
{
    if (spec.flags & MOE_FLAG_INT8_TENSOR_CORES_NEVER) return false;
    if (spec.flags & MOE_FLAG_INT8_TENSOR_CORES_ALWAYS) return true;
    if (T < MOE_INT8_TENSOR_CORE_MIN_TOKENS) return false;
    return L.S > 0 || L.dev.gate.type == FMT_Q8_0 || (int64_t)rows >= 6 * (int64_t)L.E;
}

// Batches below the f16 prefill path run the experts as one fused f16
// tensor-core launch (experts_tc.cu) unless a flag forces the int8 paths.
bool use_fused_tc(const moe_device_spec &spec, int T)
{
    if (spec.flags & (MOE_FLAG_FUSED_TC_NEVER | MOE_FLAG_INT8_TENSOR_CORES_NEVER | MOE_FLAG_INT8_TENSOR_CORES_ALWAYS))
        return false;
    // below MOE_FUSED_MIN_TOKENS the streaming kernels, unless a flag names a fused form
    if (T < MOE_FUSED_MIN_TOKENS && !(spec.flags & (MOE_FLAG_FUSED_I8_NEVER | MOE_FLAG_FUSED_I8_ALWAYS))) return false;
    return T < MOE_TENSOR_CORE_MIN_TOKENS;
}

// Between the two fused launches: integer operands while the routed slots
// per expert stay few (the int8 epilogue's work grows with the slots of an
// item, the f16 expansion's does not), f16 operands above.
bool use_fused_i8(const moe_device_spec &spec, const LayerStore &L, int T)
{
    if (spec.flags & MOE_FLAG_FUSED_I8_NEVER) return false;
    if (spec.flags & MOE_FLAG_FUSED_I8_ALWAYS) return true;
    return (int64_t)T * L.k <= (int64_t)MOE_FUSED_I8_MAX_SLOTS_PER_EXPERT * L.E;
}

bool use_tensor_cores(const moe_device_spec &spec, const LayerStore &L, const Scratch &s, int T)
{
    if (!s.tc || (spec.flags & MOE_FLAG_TENSOR_CORES_NEVER)) return false;
    if (!(spec.flags & MOE_FLAG_TENSOR_CORES_ALWAYS) && T < MOE_TENSOR_CORE_MIN_TOKENS) return false;
    if (!tc_matrix_ok(L.dev.gate) || !tc_matrix_ok(L.dev.up) || !tc_matrix_ok(L.dev.down)) return false;
    if (L.S && (!tc_matrix_ok(L.dev.sh_gate) || !tc_matrix_ok(L.dev.sh_up) || !tc_matrix_ok(L.dev.sh_down)))
        return false;
    return L.E + 2 <= kTileOffStride;
}

void free_layer(LayerStore &L)
{
    if (L.block) cudaFree(L.block);
    if (L.ffn_norm) cudaFree(L.ffn_norm);
    L = LayerStore{};
}

// Parameters of a forward over this context's T tokens (routing, local slots,
// combine); buffers from the scratch, or the caller's device buffers.
FwdParams local_params(moe_ctx *ctx, const LayerStore &L, int T, int ptr_kind, const float *x, float *out,
                       int32_t *sel_idx, float *sel_w)
{
    Scratch &s = ctx->scratch;
    FwdParams p{};
    p.T = T; p.H = L.H; p.E = L.E; p.k = L.k; p.I = L.I; p.S = L.S;
    p.route_mode = L.route_mode; p.normalize = L.normalize;
    p.n_groups = L.n_groups; p.topk_groups = L.topk_groups; p.routed_scale = L.routed_scale;
    p.mask_words = (T + 31) / 32;
    p.quant_x = L.dev.gate.type != FMT_F32 || (L.S && L.dev.sh_gate.type != FMT_F32);
    p.max_problems = std::min(L.E, T * L.k) + (L.S ? 1 : 0);
    p.router = L.router; p.logit_bias = L.logit_bias; p.sel_bias = L.sel_bias;
    p.x = ptr_kind == MOE_PTR_DEVICE ? x : s.x;
    p.out = ptr_kind == MOE_PTR_DEVICE ? out : s.out;
    p.xq = s.xq; p.xd = s.xd; p.xs = s.xs; p.logits = s.logits;
    p.sel_idx = (ptr_kind == MOE_PTR_DEVICE && sel_idx) ? sel_idx : s.sel_idx;
    p.sel_w = (ptr_kind == MOE_PTR_DEVICE && sel_w) ? sel_w : s.sel_w;
    p.sync = s.sync; p.mask = s.mask; p.wprefix = s.wprefix; p.offsets = s.offsets; p.perm_token = s.perm_token;
    p.slot_of = s.slot_of;
    p.problems = s.problems; p.n_active = s.n_active;
    p.aq = s.aq; p.ad = s.ad; p.as = s.as; p.af = s.af_buf; p.W = s.W; p.y = s.y;
    p.y_rows = nullptr;
    p.err = s.err;
    p.tile_off = s.tile_off;
    p.a16 = s.a16; p.a16dn = s.a16dn;
    p.a16_stride = s.H; p.a16dn_stride = s.W; p.slots_cap = s.slots_cap;
    p.dep = s.dep;
    p.dep_done = s.dep ? s.dep + s.dep_cap : nullptr;
    const uint64_t isum_need = (uint64_t)T * (L.k + (L.S ? 1 : 0)) * 2 * L.I * (L.H / 32);
    p.dbg_isum = ctx->dbg_isum && isum_need <= ctx->dbg_isum_cap ? ctx->dbg_isum : nullptr;
    p.dep_cap = s.dep_cap;
    p.x16 = T < MOE_TENSOR_CORE_MIN_TOKENS ? s.x16 : nullptr;
    p.use_tc = use_tensor_cores(ctx->spec, L, s, T);
    const bool fused = !p.use_tc && use_fused_tc(ctx->spec, T);
    p.use_xi8 = fused && use_fused_i8(ctx->spec, L, T) && fused_i8_ok(p, L.dev);
    p.use_xtc = fused && !p.use_xi8 && fused_experts_ok(p, L.dev);
    if (!p.use_xtc) p.x16 = nullptr;   // the routing writes the f16 rows only for the f16 fused launch
    p.use_dtc = !p.use_tc && !p.use_xtc && !p.use_xi8 && use_int8_tc(ctx->spec, L, T, T * L.k) && decode_tc_ok(p, L.dev);
    return p;
}

// ------------------------------------------------------ expert parallelism

struct EpDims {
    int world, E, H, W, rows, send;   // rows: received-slot capacity; send: sent-row capacity
    bool tc;
};

// Bytes of the plan upload: n_active (padded to 16) | problems [E] | segments [world * E].
size_t ep_plan_bytes(int world, int E)
{
    return 16 + align_up((size_t)E * sizeof(Problem), 16) + (size_t)world * E * sizeof(EpSegment);
}

// Carves the expert-parallel arena (or only measures it when base == nullptr).
size_t ep_carve(const EpDims &d, uint8_t *base, EpState *ep)
{
    size_t off = 0;
    auto take = [&](size_t bytes) -> uint8_t * {
        uint8_t *q = base ? base + off : nullptr;
        off += align_up(bytes ? bytes : 1, 256);
        return q;
    };
    const size_t R = (size_t)std::max(d.rows, 1), H = d.H, W = std::max(d.W, 32), rb = ep_row_bytes(d.H);
    EpState t;
    t.all_off = (int32_t *)take((size_t)d.world * (d.E + 1) * 4);
    t.send_buf = take((size_t)std::max(d.send, 1) * rb);
    t.recv_buf = take(R * rb);
    t.xq = (int8_t *)take(R * H);
    t.xd = (float *)take(R * (H / 32) * 4);
    t.xs = (float *)take(R * (H / 32) * 4);
    t.perm = (int32_t *)take(R * 4);
    t.plan_dev = take(ep_plan_bytes(d.world, d.E));
    t.aq = (int8_t *)take(R * W);
    t.ad = (float *)take(R * (W / 32) * 4);
    t.as = (float *)take(R * (W / 32) * 4);
    t.y = (float *)take(R * H * 4);
    t.tile_off = (int32_t *)take(4 * (size_t)kTileOffStride * 4);
    t.zero = (int32_t *)take(4);
    t.a16 = d.tc ? take(R * H * 2) : nullptr;
    t.a16dn = d.tc ? take(R * W * 2) : nullptr;
    if (ep && base) {
        ep->all_off = t.all_off; ep->send_buf = t.send_buf; ep->recv_buf = t.recv_buf;
        ep->xq = t.xq; ep->xd = t.xd; ep->xs = t.xs; ep->perm = t.perm; ep->plan_dev = t.plan_dev;
        ep->aq = t.aq; ep->ad = t.ad; ep->as = t.as; ep->y = t.y; ep->tile_off = t.tile_off; ep->zero = t.zero;
        ep->a16 = t.a16; ep->a16dn = t.a16dn;
        ep->rows_cap = (int)R; ep->send_cap = std::max(d.send, 1); ep->H = d.H; ep->W = (int)W; ep->E = d.E;
        ep->tc = d.tc;
        ep->arena_bytes = off;
    }
    return off;
}

// Grows the arena (and the pinned staging) to hold d.
int ep_reserve(moe_ctx *ctx, EpDims d)
{
    EpState &ep = ctx->ep;
    const bool fits = ep.arena && ep.rows_cap >= d.rows && ep.send_cap >= d.send && ep.H >= d.H &&
                      ep.W >= std::max(d.W, 32) && ep.E >= d.E && (ep.tc || !d.tc);
    if (!fits) {
        if (ep.arena) {
            // an earlier device-pointer forward may still be using the old arena
            CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
            d.rows = std::max(d.rows, 2 * ep.rows_cap);
            d.send = std::max(d.send, ep.send_cap);
            d.H = std::max(d.H, ep.H);
            d.W = std::max(d.W, ep.W);
            d.E = std::max(d.E, ep.E);
            d.tc = d.tc || ep.tc;
            cudaFree(ep.arena);
            ep.arena = nullptr;
        }
        d.rows = std::max(d.rows, 256);
        const size_t bytes = ep_carve(d, nullptr, nullptr);
        void *blk = nullptr;
        CUDA_TRY(ctx, cudaMalloc(&blk, bytes), "cudaMalloc(expert-parallel arena)");
        ep.arena = blk;
        ep_carve(d, static_cast<uint8_t *>(blk), &ep);
        CUDA_TRY(ctx, cudaMemset(ep.zero, 0, 4), "cudaMemset");
        CUDA_TRY(ctx, cudaDeviceSynchronize(), "cudaDeviceSynchronize");   // before any context-stream use
    }
    const size_t off_bytes = (size_t)ep.world * (ep.E + 1) * 4, plan_bytes = ep_plan_bytes(ep.world, ep.E);
    if (ep.h_off_bytes < off_bytes) {
        if (ep.h_off) cudaFreeHost(ep.h_off);
        ep.h_off = nullptr;
        CUDA_TRY(ctx, cudaMallocHost(&ep.h_off, off_bytes), "cudaMallocHost");
        ep.h_off_bytes = off_bytes;
    }
    if (ep.h_plan_bytes < plan_bytes) {
        if (ep.h_plan) cudaFreeHost(ep.h_plan);
        ep.h_plan = nullptr;
        CUDA_TRY(ctx, cudaMallocHost(&ep.h_plan, plan_bytes), "cudaMallocHost");
        ep.h_plan_bytes = plan_bytes;
    }
    return MOE_OK;
}

// Profiling names of the replicated shared-expert pass of an expert-parallel
// forward, so its launches are not folded into the routed expert stage's.
void shared_mark_cb(void *user, const char *kernel)
{
    const Marker *inner = static_cast<const Marker *>(user);
    const char *name = kernel;
    if (kernel && !strcmp(kernel, "prefill_prep")) name = "shared_prefill_prep";
    else if (kernel && !strcmp(kernel, "gate_up_tc")) name = "shared_gate_up_tc";
    else if (kernel && !strcmp(kernel, "down_tc")) name = "shared_down_tc";
    inner->mark(name);
}

// Unmaps the peers' arenas and frees this rank's (every rank is idle here).
void ep_p2p_release(EpState &ep)
{
    for (int g = 0; g < kEpMaxRanks; g++) {
        if (ep.p2p_peer[g] && ep.p2p_peer[g] != ep.p2p_arena) cudaIpcCloseMemHandle(ep.p2p_peer[g]);
        ep.p2p_peer[g] = nullptr;
    }
    if (ep.p2p_arena) cudaFree(ep.p2p_arena);
    ep.p2p_arena = nullptr;
    ep.p2p_state = 0;
}

int nccl_fail(moe_ctx *ctx, const NcclApi *nc, ncclResult_t r, const char *what)
{
    return fail(ctx, MOE_ERR_NCCL, "%s: %s", what, nc ? nc->GetErrorString(r) : "NCCL unavailable");
}

#define NCCL_TRY(ctx, nc, call, what)                              \
    do {                                                           \
        ncclResult_t r_ = (call);                                  \
        if (r_ != ncclSuccess) return nccl_fail(ctx, nc, r_, what); \
    } while (0)

// Every rank's int v, all-gathered through NCCL (set-up only; synchronises).
int ep_allgather_int(moe_ctx *ctx, const NcclApi *nc, int v, int *out)
{
    EpState &ep = ctx->ep;
    cudaStream_t st = ctx->stream;
    int32_t *d = reinterpret_cast<int32_t *>(ep.small);
    CUDA_TRY(ctx, cudaMemcpyAsync(d, &v, 4, cudaMemcpyHostToDevice, st), "copy");
    NCCL_TRY(ctx, nc, nc->AllGather(d, d + 16, 1, ncclInt32, ep.comm, st), "ncclAllGather");
    CUDA_TRY(ctx, cudaMemcpyAsync(out, d + 16, (size_t)ep.world * 4, cudaMemcpyDeviceToHost, st), "copy");
    CUDA_TRY(ctx, cudaStreamSynchronize(st), "set-up");
    return MOE_OK;
}

// Decides, collectively, whether this layer's forward uses the exchange over
// peer memory, and (re)builds the arenas and their mappings when it does and
// the current ones do not fit. Every rank reaches this at the same forward.
int ep_p2p_prepare(moe_ctx *ctx, const LayerStore &L, bool *use)
{
    EpState &ep = ctx->ep;
    const NcclApi *nc = nccl_api();
    *use = false;
    const int G = ep.world, me = ep.rank;
    const int W = std::max(L.I, L.S), cap = ctx->spec.max_tokens * L.k, slots_y = cap + ctx->spec.max_tokens;
    const bool fits = ep.p2p_state == 1 && ep.p2p.world == G && ep.p2p.E == L.E && ep.p2p.H == L.H &&
                      ep.p2p.W >= W && ep.p2p.cap >= cap && ep.p2p.slots_y >= slots_y;
    if (fits) { *use = true; return MOE_OK; }
    if (ep.p2p_state == -1 && ep.p2p.world == G && ep.p2p.E == L.E && ep.p2p.H == L.H && ep.p2p.cap >= cap)
        return MOE_OK;   // already decided against for these dims
    const bool want = !(ctx->spec.flags & MOE_FLAG_EP_NCCL_ONLY) && G <= kEpMaxRanks &&
                      ctx->spec.max_tokens <= kEpP2PMaxTokens && L.H % 64 == 0 && L.E % G == 0 &&
                      L.E <= 256;
    int all[kEpMaxRanks * 2] = {};
    int rc;
    if (G > kEpMaxRanks) {
        ep.p2p_state = -1;
        return MOE_OK;
    }
    // the arenas must have one layout on every rank: same max_tokens everywhere
    if ((rc = ep_allgather_int(ctx, nc, want ? ctx->spec.max_tokens : 0, all))) return rc;
    bool agree = true;
    for (int g = 0; g < G; g++) agree = agree && all[g] == ctx->spec.max_tokens && all[g] > 0;
    // every rank is past its previous forwards here (the all-gather ran on every stream)
    ep_p2p_release(ep);
    ep.p2p = ep_p2p_layout(G, L.E, L.H, W, cap, slots_y);
    if (!agree) {
        ep.p2p_state = -1;
        return MOE_OK;
    }
    void *arena = nullptr;
    CUDA_TRY(ctx, cudaMalloc(&arena, ep.p2p.bytes), "cudaMalloc(peer-exchange arena)");
    ep.p2p_arena = static_cast<uint8_t *>(arena);
    CUDA_TRY(ctx, cudaMemset(arena, 0, ep.p2p.bytes), "cudaMemset(peer-exchange arena)");
    CUDA_TRY(ctx, cudaDeviceSynchronize(), "cudaDeviceSynchronize");   // zero before peers map it
    ep.p2p_peer[me] = ep.p2p_arena;
    int ok = 1;
    if (G > 1) {
        cudaIpcMemHandle_t h;
        CUDA_TRY(ctx, cudaIpcGetMemHandle(&h, arena), "cudaIpcGetMemHandle");
        static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
        uint8_t *d = ep.small;
        cudaStream_t st = ctx->stream;
        CUDA_TRY(ctx, cudaMemcpyAsync(d, &h, 64, cudaMemcpyHostToDevice, st), "copy");
        NCCL_TRY(ctx, nc, nc->AllGather(d, d + 1024, 64, ncclUint8, ep.comm, st), "ncclAllGather");
        cudaIpcMemHandle_t hs[kEpMaxRanks];
        CUDA_TRY(ctx, cudaMemcpyAsync(hs, d + 1024, (size_t)G * 64, cudaMemcpyDeviceToHost, st), "copy");
        CUDA_TRY(ctx, cudaStreamSynchronize(st), "set-up");
        for (int g = 0; g < G && ok; g++) {
            if (g == me) continue;
            void *ptr = nullptr;
            if (cudaIpcOpenMemHandle(&ptr, hs[g], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
                cudaGetLastError();
                ok = 0;
            } else {
                ep.p2p_peer[g] = static_cast<uint8_t *>(ptr);
            }
        }
        if ((rc = ep_allgather_int(ctx, nc, ok, all))) return rc;
        for (int g = 0; g < G; g++) ok = ok && all[g] == 1;
    }
    if (!ok) {   // some rank could not map a peer: every rank falls back together
        ep_p2p_release(ep);
        ep.p2p_state = -1;
        return MOE_OK;
    }
    CUDA_TRY(ctx, cudaMemcpy(ep.p2p_arena + ep.p2p.o_peers, ep.p2p_peer, sizeof(ep.p2p_peer), cudaMemcpyHostToDevice),
             "copy peer table");
    ep.p2p_epoch = 0;
    ep.p2p_state = 1;
    *use = true;
    return MOE_OK;
}

}  // namespace

// ================================================================= C ABI

extern "C" {

int moe_ctx_create(const moe_device_spec *spec, moe_ctx **out)
{
    if (!spec || !out) return fail(nullptr, MOE_ERR_INVALID_ARGS, "null argument");
    *out = nullptr;
    if (spec->max_tokens <= 0 || spec->max_layers <= 0 || spec->max_layers > 4096)
        return fail(nullptr, MOE_ERR_INVALID_ARGS, "max_tokens and max_layers must be positive");
    int ndev = 0;
    cudaError_t e = cudaGetDeviceCount(&ndev);
    if (e != cudaSuccess || ndev == 0)
        return fail(nullptr, MOE_ERR_RESOURCE_EXHAUSTED, "no CUDA device available (%s)", cudaGetErrorName(e));
    if (spec->device < 0 || spec->device >= ndev)
        return fail(nullptr, MOE_ERR_INVALID_ARGS, "device %d out of range (%d devices)", spec->device, ndev);
    if ((e = cudaSetDevice(spec->device)) != cudaSuccess) return cuda_fail(nullptr, e, "cudaSetDevice");
    std::unique_ptr<moe_ctx> ctx(new moe_ctx());
    ctx->spec = *spec;
    ctx->layers.resize(spec->max_layers);
    if ((e = cudaStreamCreateWithFlags(&ctx->own_stream, cudaStreamNonBlocking)) != cudaSuccess)
        return cuda_fail(nullptr, e, "cudaStreamCreate");
    ctx->stream = ctx->own_stream;
    if ((e = cudaDeviceGetAttribute(&ctx->num_sms, cudaDevAttrMultiProcessorCount, spec->device)) != cudaSuccess)
        return cuda_fail(nullptr, e, "cudaDeviceGetAttribute");
    if ((e = cudaMallocHost(&ctx->status_host, sizeof(int))) != cudaSuccess)
        return cuda_fail(nullptr, e, "cudaMallocHost");
    *ctx->status_host = 0;
    *out = ctx.release();
    return MOE_OK;
}

int moe_ctx_destroy(moe_ctx *ctx)
{
    if (!ctx) return MOE_OK;
    cudaSetDevice(ctx->spec.device);
    cudaStreamSynchronize(ctx->stream);
    for (auto &L : ctx->layers) free_layer(L);
    if (ctx->scratch.block) cudaFree(ctx->scratch.block);
    ctx->prof.release();
    if (ctx->status_host) cudaFreeHost(ctx->status_host);
    if (ctx->stack_buf) cudaFree(ctx->stack_buf);
    if (ctx->head.block) cudaFree(ctx->head.block);
    if (ctx->head.buf) cudaFree(ctx->head.buf);
    EpState &ep = ctx->ep;
    if (ep.comm) {
        if (const NcclApi *nc = nccl_api()) nc->CommDestroy(ep.comm);
    }
    ep_p2p_release(ep);
    if (ep.arena) cudaFree(ep.arena);
    if (ep.small) cudaFree(ep.small);
    if (ep.h_off) cudaFreeHost(ep.h_off);
    if (ep.h_plan) cudaFreeHost(ep.h_plan);
    if (ctx->own_stream) cudaStreamDestroy(ctx->own_stream);
    delete ctx;
    return MOE_OK;
}

int moe_ctx_set_stream(moe_ctx *ctx, void *stream)
{
    if (!ctx) return fail(nullptr, MOE_ERR_INVALID_ARGS, "null context");
    ctx->stream = stream ? static_cast<cudaStream_t>(stream) : ctx->own_stream;
    return MOE_OK;
}

int moe_admission_check(const moe_device_spec *spec, const moe_layer_desc *layers, int32_t n_layers,
                        const moe_mem_inspector *inspector, moe_footprint *out)
{
    if (!spec || !out || n_layers < 0 || (n_layers > 0 && !layers))
        return fail(nullptr, MOE_ERR_INVALID_ARGS, "null argument");
    memset(out, 0, sizeof *out);
    uint64_t weights = 0, scratch = 0;
    ScratchDims acc{};
    bool have = false;
    for (int i = 0; i < n_layers; i++) {
        Validated v;
        int rc = validate_desc(nullptr, &layers[i], &v);
        if (rc) return rc;
        weights += layer_device_bytes(v);
        ScratchDims d = scratch_dims(std::min(spec->max_tokens, 64), v, false);
        if (!have) { acc = d; have = true; }
        else {
            acc.H = std::max(acc.H, d.H); acc.E = std::max(acc.E, d.E); acc.k = std::max(acc.k, d.k);
            acc.W = std::max(acc.W, d.W); acc.af = acc.af || d.af;
        }
    }
    uint64_t prefill = 0;
    if (have) {
        scratch = carve_scratch(acc, nullptr, nullptr);
        if (spec->max_tokens > 64) {
            ScratchDims full = acc;
            full.Tm = spec->max_tokens;
            full.tc = tc_possible(*spec);
            prefill = carve_scratch(full, nullptr, nullptr) - scratch;
        }
    }
    uint64_t free_b = 0, total_b = 0;
    if (inspector) {
        free_b = inspector->free_bytes;
        total_b = inspector->total_bytes;
    } else {
        size_t f = 0, t = 0;
        cudaError_t e = cudaSetDevice(spec->device);
        if (e == cudaSuccess) e = cudaMemGetInfo(&f, &t);
        if (e != cudaSuccess) return cuda_fail(nullptr, e, "cudaMemGetInfo");
        free_b = f; total_b = t;
    }
    (void)total_b;
    const uint64_t budget = free_b > spec->reserve_bytes ? free_b - spec->reserve_bytes : 0;
    out->weight_bytes = weights;
    out->scratch_bytes = scratch;
    out->total_required_bytes = weights + scratch;
    out->budget_bytes = budget;
    if (weights + scratch > budget)
        return fail(nullptr, MOE_ERR_INSUFFICIENT_MEMORY,
                    "device footprint %llu bytes (weights %llu + scratch %llu) exceeds budget %llu bytes",
                    (unsigned long long)(weights + scratch), (unsigned long long)weights,
                    (unsigned long long)scratch, (unsigned long long)budget);
    // optional prefill arena: dropped, not fatal, when it does not fit
    if (weights + scratch + prefill <= budget) {
        out->prefill_arena_bytes = prefill;
        out->prefill_enabled = 1;
    } else {
        out->prefill_arena_bytes = 0;
        out->prefill_enabled = 0;
    }
    return MOE_OK;
}

int moe_layer_upload(moe_ctx *ctx, int32_t layer, const moe_layer_desc *desc)
{
    if (!ctx) return fail(nullptr, MOE_ERR_INVALID_ARGS, "null context");
    if (layer < 0 || layer >= (int)ctx->layers.size())
        return fail(ctx, MOE_ERR_INVALID_ARGS, "layer %d outside 0..%d", layer, (int)ctx->layers.size() - 1);
    Validated v;
    int rc = validate_desc(ctx, desc, &v);
    if (rc) return rc;
    if (ctx->ep.world) {
        // expert parallel: this rank keeps its contiguous share of the routed experts
        const int G = ctx->ep.world;
        if (v.E % G)
            return fail(ctx, MOE_ERR_CAPABILITY_MISMATCH, "%d experts do not split over %d ranks", v.E, G);
        if (v.gate.type == MOE_QUANT_F32)
            return fail(ctx, MOE_ERR_CAPABILITY_MISMATCH, "expert parallelism needs quantised expert stacks");
        const int El = v.E / G, e0 = ctx->ep.rank * El;
        for (MatSpec *m : {&v.gate, &v.up, &v.down}) {
            m->data += (size_t)e0 * m->rows * gguf_row_bytes(m->type, m->cols);
            m->experts = El;
        }
    }
    CUDA_TRY(ctx, cudaSetDevice(ctx->spec.device), "cudaSetDevice");

    // admission against free HBM before allocating anything
    const size_t wbytes = layer_device_bytes(v);
    ScratchDims sd = merge(ctx->scratch, scratch_dims(ctx->spec.max_tokens, v, tc_possible(ctx->spec)));
    const size_t sbytes_new = covers(ctx->scratch, sd) ? 0 : carve_scratch(sd, nullptr, nullptr);
    size_t freeb = 0, totalb = 0;
    CUDA_TRY(ctx, cudaMemGetInfo(&freeb, &totalb), "cudaMemGetInfo");
    const size_t reclaim = ctx->layers[layer].block_bytes + (sbytes_new ? ctx->scratch.bytes : 0);
    const size_t avail = freeb + reclaim > ctx->spec.reserve_bytes ? freeb + reclaim - ctx->spec.reserve_bytes : 0;
    if (wbytes + sbytes_new > avail)
        return fail(ctx, MOE_ERR_INSUFFICIENT_MEMORY, "layer %d needs %zu bytes (+%zu scratch), %zu available",
                    layer, wbytes, sbytes_new, avail);

    // host staging in device layout
    std::vector<uint8_t> host(wbytes, 0);
    size_t off = 0;
    auto take = [&](size_t bytes) { size_t o = off; off += align_up(bytes, 256); return o; };
    const size_t o_router = take((size_t)v.E * v.H * 4);
    const size_t o_lb = take((size_t)v.E * 4), o_sb = take((size_t)v.E * 4);
    memcpy(host.data() + o_router, v.router, (size_t)v.E * v.H * 4);
    if (v.logit_bias) memcpy(host.data() + o_lb, v.logit_bias, (size_t)v.E * 4);
    if (v.sel_bias) memcpy(host.data() + o_sb, v.sel_bias, (size_t)v.E * 4);
    struct Placed { MatrixPlan plan; size_t qs, meta; bool present; };
    auto place = [&](const MatSpec &m) {
        Placed p{};
        p.present = m.present;
        if (!m.present) return p;
        p.plan = plan_matrix(m.type, m.rows, m.cols, m.experts);
        p.qs = take(p.plan.qs_bytes);
        p.meta = take(p.plan.meta_bytes);
        repack_rows(p.plan, m.data, host.data() + p.qs, p.plan.meta_bytes ? host.data() + p.meta : nullptr);
        return p;
    };
    Placed pg = place(v.gate), pu = place(v.up), pd = place(v.down);
    Placed psg = place(v.sg), psu = place(v.su), psd = place(v.sd);

    // device buffers: release the old layer and grow the scratch if needed
    CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
    free_layer(ctx->layers[layer]);
    if (sbytes_new) {
        if (ctx->scratch.block) cudaFree(ctx->scratch.block);
        ctx->scratch = Scratch{};
        void *blk = nullptr;
        CUDA_TRY(ctx, cudaMalloc(&blk, sbytes_new), "cudaMalloc(scratch)");
        ctx->scratch.block = blk;
        carve_scratch(sd, static_cast<uint8_t *>(blk), &ctx->scratch);
        CUDA_TRY(ctx, cudaMemset(ctx->scratch.err, 0, sizeof(int)), "cudaMemset(status)");
        CUDA_TRY(ctx, cudaMemset(ctx->scratch.sync, 0, kRoutingTicketBytes), "cudaMemset(routing tickets)");
        CUDA_TRY(ctx, cudaMemset(ctx->scratch.dep, 0, ((size_t)ctx->scratch.dep_cap + 1) * 4),
                 "cudaMemset(chunk counters)");
        CUDA_TRY(ctx, cudaDeviceSynchronize(), "cudaDeviceSynchronize");   // the context stream does not wait for it
    }
    LayerStore &L = ctx->layers[layer];
    void *blk = nullptr;
    CUDA_TRY(ctx, cudaMalloc(&blk, wbytes), "cudaMalloc(layer)");
    cudaError_t e = cudaMemcpy(blk, host.data(), wbytes, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        cudaFree(blk);
        return cuda_fail(ctx, e, "cudaMemcpy(layer)");
    }
    uint8_t *base = static_cast<uint8_t *>(blk);
    L.present = true;
    L.block = blk;
    L.block_bytes = wbytes;
    L.H = v.H; L.E = v.E; L.k = v.k; L.I = v.I; L.S = v.S;
    L.route_mode = desc->route_mode;
    L.normalize = desc->normalize;
    L.n_groups = desc->n_groups;
    L.topk_groups = desc->topk_groups;
    L.routed_scale = desc->routed_scale;
    L.router = reinterpret_cast<const float *>(base + o_router);
    L.logit_bias = v.logit_bias ? reinterpret_cast<const float *>(base + o_lb) : nullptr;
    L.sel_bias = v.sel_bias ? reinterpret_cast<const float *>(base + o_sb) : nullptr;
    auto dev = [&](const Placed &p) {
        if (!p.present) return DevMatrix{};
        DevMatrix m = to_dev(p.plan, base + p.qs, p.plan.meta_bytes ? base + p.meta : nullptr);
        plan_slices(m);
        return m;
    };
    L.dev.gate = dev(pg); L.dev.up = dev(pu); L.dev.down = dev(pd);
    L.dev.sh_gate = dev(psg); L.dev.sh_up = dev(psu); L.dev.sh_down = dev(psd);
    // TMA descriptors: each quantised stack is a dense [E*rows][row bytes] array
    struct MapSet { const DevMatrix *m; MatMaps *stream, *tc; };
    const MapSet mats[] = {{&L.dev.gate, &L.maps.gate, &L.maps.gate_tc},
                           {&L.dev.up, &L.maps.up, &L.maps.up_tc},
                           {&L.dev.down, &L.maps.down, &L.maps.down_tc},
                           {&L.dev.sh_gate, &L.maps.sh_gate, &L.maps.sh_gate_tc},
                           {&L.dev.sh_up, &L.maps.sh_up, &L.maps.sh_up_tc},
                           {&L.dev.sh_down, &L.maps.sh_down, &L.maps.sh_down_tc}};
    for (const auto &mm : mats) {
        const DevMatrix &m = *mm.m;
        if (m.rows && m.type != FMT_F32 &&
            (m.qs_estride != m.qs_rstride * m.rows || m.meta_estride != m.meta_rstride * m.rows)) {
            free_layer(L);
            return fail(ctx, MOE_ERR_CAPABILITY_MISMATCH, "expert slabs are not dense (rows %d)", m.rows);
        }
        int r = make_matrix_maps(m, mm.stream, 32);
        if (r == 0 && m.rows % 128 == 0) r = make_matrix_maps(m, mm.tc, 128);
        if (r != 0) {
            free_layer(L);
            return fail(ctx, MOE_ERR_CUDA, "cuTensorMapEncodeTiled failed (CUresult %d)", r);
        }
    }
    L.gguf_bytes = (size_t)v.E * v.H * 4;   // the router is replicated; expert stacks count this rank's share
    for (const MatSpec *m : {&v.gate, &v.up, &v.down, &v.sg, &v.su, &v.sd})
        if (m->present) L.gguf_bytes += gguf_row_bytes(m->type, m->cols) * m->rows * m->experts;
    ctx->upload_count++;
    return MOE_OK;
}

// moe_forward, and with block = true moe_forward_block: out = x + block(rmsnorm(x)).
static int forward_impl(moe_ctx *ctx, int32_t layer, int32_t T, const float *x, float *out, int32_t *sel_idx,
                        float *sel_w, int32_t ptr_kind, bool block)
{
    if (!ctx) return fail(nullptr, MOE_ERR_INVALID_ARGS, "null context");
    if (layer < 0 || layer >= (int)ctx->layers.size())
        return fail(ctx, MOE_ERR_INVALID_ARGS, "layer %d outside 0..%d", layer, (int)ctx->layers.size() - 1);
    LayerStore &L = ctx->layers[layer];
    if (!L.present) return fail(ctx, MOE_ERR_NOT_UPLOADED, "layer %d was never uploaded", layer);
    if (T < 0) return fail(ctx, MOE_ERR_INVALID_ARGS, "negative token count");
    if (T > ctx->spec.max_tokens)
        return fail(ctx, MOE_ERR_CONTEXT_LENGTH, "T=%d exceeds max_tokens=%d", T, ctx->spec.max_tokens);
    if (ptr_kind != MOE_PTR_HOST && ptr_kind != MOE_PTR_DEVICE)
        return fail(ctx, MOE_ERR_INVALID_ARGS, "unknown pointer kind %d", ptr_kind);
    if (T == 0) return MOE_OK;
    if (!x || !out) return fail(ctx, MOE_ERR_INVALID_ARGS, "null x or out");
    if (ptr_kind == MOE_PTR_DEVICE && (((uintptr_t)x | (uintptr_t)out) & 15))
        return fail(ctx, MOE_ERR_INVALID_ARGS, "device x and out must be 16-byte aligned");
    if (block && !L.ffn_norm)
        return fail(ctx, MOE_ERR_INVALID_ARGS, "layer %d has no ffn_norm (moe_layer_set_ffn_norm)", layer);
    CUDA_TRY(ctx, cudaSetDevice(ctx->spec.device), "cudaSetDevice");
    Scratch &s = ctx->scratch;
    cudaStream_t st = ctx->stream;
    FwdParams p = local_params(ctx, L, T, ptr_kind, x, out, sel_idx, sel_w);

    if (block) {
        // host: the residual stream goes to s.out, which the combine updates in
        // place; device: read from x, written to out (which may be x). The
        // normalised tokens go to s.x, the routing's input.
        const float *hidden = x;
        if (ptr_kind == MOE_PTR_HOST) {
            CUDA_TRY(ctx, cudaMemcpyAsync(s.out, x, (size_t)T * L.H * 4, cudaMemcpyHostToDevice, st), "copy hidden");
            hidden = s.out;
        }
        p.norm_in = hidden;
        p.norm_out = s.x;
        p.norm_w = L.ffn_norm;
        p.norm_eps = L.norm_eps;
        p.residual = hidden;
        p.x = s.x;
    } else if (ptr_kind == MOE_PTR_HOST) {
        CUDA_TRY(ctx, cudaMemcpyAsync(s.x, x, (size_t)T * L.H * 4, cudaMemcpyHostToDevice, st), "copy x");
    }
    Marker mk{nullptr, nullptr};
    if (ctx->prof.on) {
        ctx->prof.stream = st;
        mk = Marker{&Profiler::mark_cb, &ctx->prof};
    }
    int err = launch_forward(p, L.dev, L.maps, st, mk, ctx->num_sms);
    if (err != cudaSuccess) return cuda_fail(ctx, (cudaError_t)err, "forward launch");
    ctx->last_layer = layer;
    ctx->last_T = T;
    if (ptr_kind == MOE_PTR_HOST) {
        CUDA_TRY(ctx, cudaMemcpyAsync(out, s.out, (size_t)T * L.H * 4, cudaMemcpyDeviceToHost, st), "copy out");
        if (sel_idx)
            CUDA_TRY(ctx, cudaMemcpyAsync(sel_idx, s.sel_idx, (size_t)T * L.k * 4, cudaMemcpyDeviceToHost, st),
                     "copy sel_idx");
        if (sel_w)
            CUDA_TRY(ctx, cudaMemcpyAsync(sel_w, s.sel_w, (size_t)T * L.k * 4, cudaMemcpyDeviceToHost, st),
                     "copy sel_w");
        CUDA_TRY(ctx, cudaMemcpyAsync(ctx->status_host, s.err, sizeof(int), cudaMemcpyDeviceToHost, st),
                 "copy status");
        CUDA_TRY(ctx, cudaStreamSynchronize(st), "forward");
        if (*ctx->status_host) {
            cudaMemsetAsync(s.err, 0, sizeof(int), st);
            return fail(ctx, MOE_ERR_TIMEOUT, "a bounded device wait ran out in layer %d (status %d)", layer,
                        *ctx->status_host);
        }
    }
    return MOE_OK;
}

int moe_forward(moe_ctx *ctx, int32_t layer, int32_t T, const float *x, float *out, int32_t *sel_idx,
                float *sel_w, int32_t ptr_kind)
{
    return forward_impl(ctx, layer, T, x, out, sel_idx, sel_w, ptr_kind, false);
}

int moe_forward_block(moe_ctx *ctx, int32_t layer, int32_t T, const float *hidden, float *out, int32_t *sel_idx,
                      float *sel_w, int32_t ptr_kind)
{
    return forward_impl(ctx, layer, T, hidden, out, sel_idx, sel_w, ptr_kind, true);
}

// Layer-major prefill of a stack of MoE FFN sublayers: every layer takes all T
// tokens at once (moe_forward_block in place on the device), in layer order.
// For a stack of FFN sublayers this equals the reference's token-major prefill
// (run_prefill_with_hidden, src/qwen_deepseek.rs:2217-2316: every layer per
// token), because each sublayer treats its tokens independently; with host
// pointers the rows cross PCIe once each way for the whole stack.
int moe_prefill_ffn_layers(moe_ctx *ctx, int32_t first_layer, int32_t n_layers, int32_t T, float *hidden,
                           int32_t ptr_kind)
{
    if (!ctx || (!hidden && T > 0)) return fail(ctx, MOE_ERR_INVALID_ARGS, "null argument");
    if (n_layers < 0 || first_layer < 0 || first_layer + n_layers > (int)ctx->layers.size())
        return fail(ctx, MOE_ERR_INVALID_ARGS, "layers %d..%d outside 0..%d", first_layer, first_layer + n_layers - 1,
                    (int)ctx->layers.size() - 1);
    if (ptr_kind != MOE_PTR_HOST && ptr_kind != MOE_PTR_DEVICE)
        return fail(ctx, MOE_ERR_INVALID_ARGS, "ptr_kind must be MOE_PTR_HOST or MOE_PTR_DEVICE");
    if (T < 0 || T > ctx->spec.max_tokens)
        return fail(ctx, MOE_ERR_CONTEXT_LENGTH, "T = %d outside 0..max_tokens %d", T, ctx->spec.max_tokens);
    if (T == 0 || n_layers == 0) return MOE_OK;
    const int H = ctx->layers[first_layer].H;
    for (int l = first_layer; l < first_layer + n_layers; l++) {
        const LayerStore &L = ctx->layers[l];
        if (!L.present) return fail(ctx, MOE_ERR_NOT_UPLOADED, "layer %d was never uploaded", l);
        if (L.H != H) return fail(ctx, MOE_ERR_INVALID_ARGS, "layer %d has hidden %d, layer %d %d", l, L.H,
                                  first_layer, H);
    }
    CUDA_TRY(ctx, cudaSetDevice(ctx->spec.device), "cudaSetDevice");
    cudaStream_t st = ctx->stream;
    const size_t n = (size_t)T * H;
    float *rows = hidden;
    if (ptr_kind == MOE_PTR_HOST) {
        if (ctx->stack_buf_n < n) {
            CUDA_TRY(ctx, cudaStreamSynchronize(st), "cudaStreamSynchronize");
            if (ctx->stack_buf) cudaFree(ctx->stack_buf);
            ctx->stack_buf = nullptr;
            ctx->stack_buf_n = 0;
            CUDA_TRY(ctx, cudaMalloc(&ctx->stack_buf, n * 4), "cudaMalloc(prefill rows)");
            ctx->stack_buf_n = n;
        }
        rows = ctx->stack_buf;
        CUDA_TRY(ctx, cudaMemcpyAsync(rows, hidden, n * 4, cudaMemcpyHostToDevice, st), "copy hidden");
    }
    for (int l = first_layer; l < first_layer + n_layers; l++) {
        const int rc = forward_impl(ctx, l, T, rows, rows, nullptr, nullptr, MOE_PTR_DEVICE, true);
        if (rc != MOE_OK) return rc;
    }
    if (ptr_kind == MOE_PTR_HOST) {
        CUDA_TRY(ctx, cudaMemcpyAsync(hidden, rows, n * 4, cudaMemcpyDeviceToHost, st), "copy hidden");
        int32_t status = 0;
        const int rc = moe_device_status(ctx, &status);   // synchronises the stream
        if (rc != MOE_OK) return rc;
        if (status) return fail(ctx, MOE_ERR_TIMEOUT, "a bounded device wait ran out (status %d)", status);
    }
    return MOE_OK;
}

// The LM head of project_lm_head (src/qwen_deepseek.rs:584-632): output.weight
// when present, else the tied token_embd.weight; GGUF [hidden, rows] (rows =
// vocabulary). A tensor of another shape is kept as elements / hidden rows,
// used only by calls whose logit count equals them (the reference's second
// branch); a head that fits neither leaves the synthetic logits.
int moe_lm_head_upload(moe_ctx *ctx, const moe_tensor *output_weight, const moe_tensor *token_embd, int32_t hidden)
{
    if (!ctx) return fail(nullptr, MOE_ERR_INVALID_ARGS, "null context");
    if (hidden <= 0) return fail(ctx, MOE_ERR_INVALID_ARGS, "hidden must be positive");
    const moe_tensor *t = output_weight && output_weight->data ? output_weight
                          : (token_embd && token_embd->data ? token_embd : nullptr);
    if (t && t->quant != MOE_QUANT_F32 && t->quant != MOE_QUANT_Q8_0 && t->quant != MOE_QUANT_Q4_K)
        return fail(ctx, MOE_ERR_CAPABILITY_MISMATCH, "unsupported LM head quantization %d", t->quant);
    if (t && (t->n_dims < 1 || t->n_dims > 4)) return fail(ctx, MOE_ERR_TENSOR_BOUNDS, "LM head dims %d", t->n_dims);
    CUDA_TRY(ctx, cudaSetDevice(ctx->spec.device), "cudaSetDevice");
    CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
    moe_ctx::Head &hd = ctx->head;
    if (hd.block) cudaFree(hd.block);
    hd = moe_ctx::Head{hd.uploaded, false, false, hidden, 0, nullptr, DevMatrix{}, MatMaps{}, hd.buf, hd.buf_bytes, hd.errw};
    hd.uploaded = true;
    if (!t) return MOE_OK;
    hd.has = true;
    hd.shaped = t->n_dims == 2 && t->shape[0] == hidden && t->shape[1] > 0;
    int64_t rows = 0;
    if (hd.shaped) {
        rows = t->shape[1];
    } else {
        int64_t n = 1;
        for (int i = 0; i < t->n_dims; i++) n *= t->shape[i];
        rows = n > 0 && n % hidden == 0 ? n / hidden : 0;
    }
    if (rows <= 0) return MOE_OK;   // a head that fits no branch: synthetic logits, as the reference
    if (rows > (1 << 24)) return fail(ctx, MOE_ERR_TENSOR_BOUNDS, "LM head rows %lld out of range", (long long)rows);
    const size_t rb = gguf_row_bytes(t->quant, hidden);
    if (!rb)
        return fail(ctx, MOE_ERR_CAPABILITY_MISMATCH, "LM head: %d columns are not whole %s blocks", hidden,
                    quant_name(t->quant));
    if (t->nbytes != rb * (size_t)rows)
        return fail(ctx, MOE_ERR_TENSOR_BOUNDS, "LM head: %llu bytes, shape needs %llu",
                    (unsigned long long)t->nbytes, (unsigned long long)(rb * (size_t)rows));
    MatrixPlan plan = plan_matrix(t->quant, (int)rows, hidden, 1);
    const size_t o_meta = align_up(plan.qs_bytes, 256);
    const size_t bytes = o_meta + align_up(plan.meta_bytes, 256);
    std::vector<uint8_t> host(bytes, 0);
    repack_rows(plan, static_cast<const uint8_t *>(t->data), host.data(),
                plan.meta_bytes ? host.data() + o_meta : nullptr);
    void *blk = nullptr;
    if (cudaMalloc(&blk, bytes) != cudaSuccess) {
        cudaGetLastError();
        hd.has = false;
        return fail(ctx, MOE_ERR_INSUFFICIENT_MEMORY, "LM head needs %zu bytes of device memory", bytes);
    }
    cudaError_t e = cudaMemcpy(blk, host.data(), bytes, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        cudaFree(blk);
        hd.has = false;
        return cuda_fail(ctx, e, "cudaMemcpy(LM head)");
    }
    uint8_t *base = static_cast<uint8_t *>(blk);
    hd.block = blk;
    hd.rows = (int)rows;
    hd.m = to_dev(plan, base, plan.meta_bytes ? base + o_meta : nullptr);
    plan_slices(hd.m);
    int r = make_matrix_maps(hd.m, &hd.maps, 32);
    if (r != 0) return fail(ctx, MOE_ERR_CUDA, "cuTensorMapEncodeTiled failed (CUresult %d)", r);
    hd.tc = t->quant != MOE_QUANT_F32 && rows % 128 == 0 && hidden % (t->quant == MOE_QUANT_Q4_K ? 256 : 128) == 0;
    if (hd.tc && (r = make_matrix_maps(hd.m, &hd.maps_tc, 128)) != 0)
        return fail(ctx, MOE_ERR_CUDA, "cuTensorMapEncodeTiled failed (CUresult %d)", r);
    return MOE_OK;
}

// Rows of normed activations from which the LM head's product runs on the
// int8 tensor cores (decode_tc.cu down launch) instead of the streaming kernel,
// and from which on the f16 tensor-core GEMM (prefill.cu, one dense problem):
// measured crossovers on a 151936 x 2048 head (16 rows: Q4_K f16 145 us vs int8
// 206, Q8_0 f16 137 vs int8 147; 8 rows: int8 100-126 vs f16 about 140).
constexpr int kLmHeadTcMinTokens = 8;
constexpr int kLmHeadF16MinTokensQ4K = 16, kLmHeadF16MinTokensQ80 = 16;

// logits [T x n_logits] of T normed rows [T x hidden], each row as
// project_lm_head: the head's first min(n_logits, rows) rows as a quantised
// matrix-vector product (int8 activation blocks, as the experts), the rest
// normed[i mod hidden] * 0.05; without a usable head the synthetic logits.
int moe_lm_head(moe_ctx *ctx, int32_t T, const float *normed, float *logits, int32_t n_logits, int32_t ptr_kind)
{
    if (!ctx) return fail(nullptr, MOE_ERR_INVALID_ARGS, "null context");
    moe_ctx::Head &hd = ctx->head;
    if (!hd.uploaded) return fail(ctx, MOE_ERR_NOT_UPLOADED, "no LM head was uploaded (moe_lm_head_upload)");
    if (T < 0 || n_logits < 0) return fail(ctx, MOE_ERR_INVALID_ARGS, "negative token or logit count");
    if (T > ctx->spec.max_tokens)
        return fail(ctx, MOE_ERR_CONTEXT_LENGTH, "T = %d exceeds max_tokens %d", T, ctx->spec.max_tokens);
    if (ptr_kind != MOE_PTR_HOST && ptr_kind != MOE_PTR_DEVICE)
        return fail(ctx, MOE_ERR_INVALID_ARGS, "ptr_kind must be MOE_PTR_HOST or MOE_PTR_DEVICE");
    if (T == 0 || n_logits == 0) return MOE_OK;
    if (!normed || !logits) return fail(ctx, MOE_ERR_INVALID_ARGS, "null argument");
    CUDA_TRY(ctx, cudaSetDevice(ctx->spec.device), "cudaSetDevice");
    cudaStream_t st = ctx->stream;
    const int H = hd.hidden;
    const bool product = hd.has && hd.rows > 0 && (hd.shaped || hd.rows == n_logits);
    const int target = product ? std::min(n_logits, hd.rows) : 0;
    // the product's kernel: 0 streaming, 1 int8 tensor cores (from
    // kLmHeadTcMinTokens rows), 2 f16 tensor-core GEMM (from kLmHeadF16MinTokens);
    // the flags force one. Tensor-core items cover 128 head rows, so the product
    // then spans target rounded up to 128 (at most the head's rows).
    const unsigned fl = (unsigned)ctx->spec.flags;
    int path = 0;
    if (product && hd.tc) {
        if (fl & MOE_FLAG_INT8_TENSOR_CORES_NEVER) path = 0;
        else if (fl & MOE_FLAG_INT8_TENSOR_CORES_ALWAYS) path = 1;
        else if (fl & MOE_FLAG_TENSOR_CORES_ALWAYS) path = 2;
        else if (T >= (hd.m.type == FMT_Q4_K ? kLmHeadF16MinTokensQ4K : kLmHeadF16MinTokensQ80) &&
                 !(fl & MOE_FLAG_TENSOR_CORES_NEVER))
            path = 2;
        else if (T >= kLmHeadTcMinTokens) path = 1;
    }
    const bool tc = path != 0;
    const int yrows = tc ? (target + 127) / 128 * 128 : target;
    const bool direct = ptr_kind == MOE_PTR_DEVICE && target == n_logits && yrows == target;
    // call buffers: the status word and the problem first (fixed offsets, so the
    // word is zero from its allocation on), then normed rows, int8 blocks,
    // product rows, logits
    size_t off = 0;
    auto take = [&](size_t b) { size_t o = off; off += align_up(b ? b : 1, 256); return o; };
    const size_t o_e = take(16), o_p = take(sizeof(Problem) + 16), o_x = take((size_t)T * H * 4),
                 o_q = take((size_t)T * H), o_d = take((size_t)T * (H / 32) * 4), o_s = take((size_t)T * (H / 32) * 4),
                 o_y = take(direct ? 0 : (size_t)T * std::max(yrows, 1) * 4), o_l = take((size_t)T * n_logits * 4),
                 o_h = take(path == 2 ? (size_t)T * H * 2 : 0), o_t = take(path == 2 ? 4 * kTileOffStride * 4 : 0);
    if (hd.buf_bytes < off) {
        CUDA_TRY(ctx, cudaStreamSynchronize(st), "cudaStreamSynchronize");
        if (hd.buf) cudaFree(hd.buf);
        hd.buf = nullptr;
        hd.buf_bytes = 0;
        hd.errw = nullptr;
        CUDA_TRY(ctx, cudaMalloc(&hd.buf, off), "cudaMalloc(LM head buffers)");
        hd.buf_bytes = off;
        // on the call's stream: the context stream does not wait for the legacy stream
        CUDA_TRY(ctx, cudaMemsetAsync(hd.buf, 0, off, st), "cudaMemset(LM head buffers)");
    }
    uint8_t *b = static_cast<uint8_t *>(hd.buf);
    // the device status word: the context's, or (no layer uploaded yet) one of the head's own
    int *errw = ctx->scratch.err ? ctx->scratch.err : reinterpret_cast<int *>(b + o_e);
    hd.errw = reinterpret_cast<int *>(b + o_e);
    const float *x = normed;
    if (ptr_kind == MOE_PTR_HOST) {
        CUDA_TRY(ctx, cudaMemcpyAsync(b + o_x, normed, (size_t)T * H * 4, cudaMemcpyHostToDevice, st), "copy rows");
        x = reinterpret_cast<const float *>(b + o_x);
    }
    float *lg = ptr_kind == MOE_PTR_DEVICE ? logits : reinterpret_cast<float *>(b + o_l);
    cudaError_t e;
    if (product) {
        FwdParams pl{};
        pl.T = T; pl.H = yrows; pl.E = 1; pl.k = 1; pl.I = H; pl.S = 0; pl.W = H;
        pl.max_problems = 1;
        pl.problems = reinterpret_cast<Problem *>(b + o_p);
        pl.n_active = reinterpret_cast<int32_t *>(b + o_p + sizeof(Problem));
        pl.err = errw;
        pl.y = direct ? lg : reinterpret_cast<float *>(b + o_y);
        LayerDev Lh{};
        Lh.down = hd.m;
        Lh.down.rows = yrows;   // the first rows of the head (rows are contiguous)
        LayerMaps lm{};
        lm.down = hd.maps;
        lm.down_tc = hd.maps_tc;
        if (hd.m.type == FMT_F32) {
            pl.af = const_cast<float *>(x);
        } else {
            pl.aq = reinterpret_cast<int8_t *>(b + o_q);
            pl.ad = reinterpret_cast<float *>(b + o_d);
            pl.as = reinterpret_cast<float *>(b + o_s);
            if ((e = (cudaError_t)launch_quantize_rows(x, T, H, pl.aq, pl.ad, pl.as, st)) != cudaSuccess)
                return cuda_fail(ctx, e, "LM head activation blocks");
        }
        if (path == 2) {
            pl.xq = pl.aq;
            pl.xd = pl.ad;
            pl.a16dn = b + o_h;
            pl.a16dn_stride = H;
            pl.slots_cap = T;
            pl.tile_off = reinterpret_cast<int32_t *>(b + o_t);
        }
        if (path != 2 && (e = launch_lm_head_prep(pl.problems, pl.n_active, T, st)) != cudaSuccess)
            return cuda_fail(ctx, e, "LM head problem");
        if (path == 2 && dense_f16_ok(pl, Lh)) e = launch_dense_f16(pl, Lh, lm, ctx->num_sms, st);
        else if (path == 1 && decode_tc_down_ok(pl, Lh)) e = launch_decode_tc_down(pl, Lh, lm, ctx->num_sms, st);
        else if (path == 0) e = launch_down(pl, Lh, lm, 0, ctx->num_sms, st);
        else e = cudaErrorInvalidValue;   // the checks above admit every tensor-core head
        if (e != cudaSuccess) return cuda_fail(ctx, e, "LM head");
        if (!direct && (e = launch_lm_head_scatter(pl.y, yrows, target, x, H, lg, n_logits, T, ctx->num_sms, st)) !=
                           cudaSuccess)
            return cuda_fail(ctx, e, "LM head rows");
    } else if ((e = launch_lm_head_synth(x, H, lg, n_logits, T, st)) != cudaSuccess) {
        return cuda_fail(ctx, e, "LM head (synthetic)");
    }
    if (ptr_kind == MOE_PTR_HOST) {
        CUDA_TRY(ctx, cudaMemcpyAsync(logits, lg, (size_t)T * n_logits * 4, cudaMemcpyDeviceToHost, st), "copy logits");
        CUDA_TRY(ctx, cudaMemcpyAsync(ctx->status_host, errw, sizeof(int), cudaMemcpyDeviceToHost, st), "copy status");
        CUDA_TRY(ctx, cudaStreamSynchronize(st), "LM head");
        if (*ctx->status_host) {
            const int code = *ctx->status_host;
            cudaMemsetAsync(errw, 0, sizeof(int), st);
            return fail(ctx, MOE_ERR_TIMEOUT, "a bounded device wait ran out in the LM head (status %d)", code);
        }
    }
    return MOE_OK;
}

int moe_layer_set_ffn_norm(moe_ctx *ctx, int32_t layer, const float *weight, float eps)
{
    if (!ctx) return fail(nullptr, MOE_ERR_INVALID_ARGS, "null context");
    if (layer < 0 || layer >= (int)ctx->layers.size())
        return fail(ctx, MOE_ERR_INVALID_ARGS, "layer %d outside 0..%d", layer, (int)ctx->layers.size() - 1);
    LayerStore &L = ctx->layers[layer];
    if (!L.present) return fail(ctx, MOE_ERR_NOT_UPLOADED, "layer %d was never uploaded", layer);
    if (!std::isfinite(eps) || eps < 0.0f) return fail(ctx, MOE_ERR_INVALID_ARGS, "eps must be finite and >= 0");
    // missing or non-finite weights read as 1.0 (read_f32_weight_or_default)
    std::vector<float> w((size_t)L.H, 1.0f);
    if (weight)
        for (int h = 0; h < L.H; h++)
            if (std::isfinite(weight[h])) w[h] = weight[h];
    CUDA_TRY(ctx, cudaSetDevice(ctx->spec.device), "cudaSetDevice");
    if (!L.ffn_norm) CUDA_TRY(ctx, cudaMalloc(&L.ffn_norm, (size_t)L.H * 4), "ffn_norm allocation");
    CUDA_TRY(ctx, cudaMemcpy(L.ffn_norm, w.data(), (size_t)L.H * 4, cudaMemcpyHostToDevice), "copy ffn_norm");
    L.norm_eps = eps;
    return MOE_OK;
}

int moe_device_status(moe_ctx *ctx, int32_t *status)
{
    if (!ctx || !status) return fail(nullptr, MOE_ERR_INVALID_ARGS, "null argument");
    *status = 0;
    // the context's word, or (LM head calls before any layer upload) the head's own
    int *word = ctx->scratch.err ? ctx->scratch.err : ctx->head.errw;
    CUDA_TRY(ctx, cudaSetDevice(ctx->spec.device), "cudaSetDevice");
    if (!word) {
        CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream), "status sync");
        return MOE_OK;
    }
    CUDA_TRY(ctx, cudaMemcpyAsync(ctx->status_host, word, sizeof(int), cudaMemcpyDeviceToHost, ctx->stream),
             "copy status");
    CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream), "status sync");
    *status = *ctx->status_host;
    if (*status) {
        CUDA_TRY(ctx, cudaMemsetAsync(word, 0, sizeof(int), ctx->stream), "clear status");
        if (ctx->ep.world && (*status == kErrEpTimeout || *status == kErrEpDesync)) {
            ctx->ep.p2p_broken = true;
            return fail(ctx, MOE_ERR_TIMEOUT,
                        "a bounded peer-rank wait failed (status %d); call moe_ep_reset on every rank", *status);
        }
        return fail(ctx, MOE_ERR_TIMEOUT, "a bounded device wait ran out (status %d)", *status);
    }
    return MOE_OK;
}

int moe_ep_reset(moe_ctx *ctx)
{
    if (!ctx) return fail(nullptr, MOE_ERR_INVALID_ARGS, "null context");
    EpState &ep = ctx->ep;
    if (!ep.world) return fail(ctx, MOE_ERR_INVALID_ARGS, "moe_ep_init was not called on this context");
    const NcclApi *nc = nccl_api();
    if (!nc) return fail(ctx, MOE_ERR_NCCL, "NCCL unavailable");
    CUDA_TRY(ctx, cudaSetDevice(ctx->spec.device), "cudaSetDevice");
    int all[kEpMaxRanks] = {};
    int rc;
    // every rank has finished its own forwards before any arena is cleared ...
    CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
    if ((rc = ep_allgather_int(ctx, nc, 1, all))) return rc;
    if (ep.p2p_arena) CUDA_TRY(ctx, cudaMemset(ep.p2p_arena + ep.p2p.o_flags, 0, ep.p2p.o_peers - ep.p2p.o_flags),
                               "cudaMemset(peer-exchange arena)");
    if (ep.p2p_arena) CUDA_TRY(ctx, cudaMemset(ep.p2p_arena + ep.p2p.o_misc, 0, 128), "cudaMemset(tickets)");
    if (ctx->scratch.err) CUDA_TRY(ctx, cudaMemset(ctx->scratch.err, 0, sizeof(int)), "cudaMemset(status)");
    CUDA_TRY(ctx, cudaDeviceSynchronize(), "cudaDeviceSynchronize");
    ep.p2p_epoch = 0;
    ep.p2p_broken = false;
    ep.dbg_skew = 0;
    // ... and before any rank's next forward writes into a peer's arena
    return ep_allgather_int(ctx, nc, 1, all);
}

int moe_debug_ep_fault(moe_ctx *ctx, uint32_t epoch_skew, int64_t wait_cycles)
{
    if (!ctx) return fail(nullptr, MOE_ERR_INVALID_ARGS, "null context");
    if (!ctx->ep.world) return fail(ctx, MOE_ERR_INVALID_ARGS, "moe_ep_init was not called on this context");
    if (wait_cycles < 0) return fail(ctx, MOE_ERR_INVALID_ARGS, "negative wait bound");
    ctx->ep.dbg_skew = epoch_skew;
    ctx->ep.dbg_wait_cycles = wait_cycles;
    return MOE_OK;
}

int moe_residency_summary(const moe_ctx *ctx, moe_residency *out)
{
    if (!ctx || !out) return fail(nullptr, MOE_ERR_INVALID_ARGS, "null argument");
    memset(out, 0, sizeof *out);
    for (const auto &L : ctx->layers) {
        if (!L.present) continue;
        out->layers_resident++;
        out->resident_bytes += L.block_bytes;
        out->gguf_bytes += L.gguf_bytes;
    }
    out->upload_count = ctx->upload_count;
    out->scratch_bytes = ctx->scratch.bytes;
    return MOE_OK;
}

int moe_ctx_set_profiling(moe_ctx *ctx, int32_t enabled)
{
    if (!ctx) return fail(nullptr, MOE_ERR_INVALID_ARGS, "null context");
    ctx->prof.on = enabled != 0;
    return MOE_OK;
}

int moe_profile_read(moe_ctx *ctx, moe_kernel_time *out, int32_t cap, int32_t *n_kernels, int32_t *n_forwards)
{
    if (!ctx || (cap > 0 && !out)) return fail(nullptr, MOE_ERR_INVALID_ARGS, "null argument");
    CUDA_TRY(ctx, cudaSetDevice(ctx->spec.device), "cudaSetDevice");
    Profiler &pf = ctx->prof;
    if (!pf.marks.empty()) CUDA_TRY(ctx, cudaStreamSynchronize(pf.stream), "profile sync");
    pf.totals.clear();
    cudaEvent_t prev = nullptr;
    for (auto &m : pf.marks) {
        if (m.first && prev) {
            float ms = 0.0f;
            CUDA_TRY(ctx, cudaEventElapsedTime(&ms, prev, m.second), "cudaEventElapsedTime");
            pf.add(m.first, ms);
        }
        prev = m.second;
    }
    const int n = (int)pf.totals.size();
    for (int i = 0; i < n && i < cap; i++) {
        memset(&out[i], 0, sizeof out[i]);
        snprintf(out[i].name, sizeof out[i].name, "%s", pf.totals[i].first.c_str());
        out[i].total_ms = pf.totals[i].second.first;
        out[i].launches = pf.totals[i].second.second;
    }
    if (n_kernels) *n_kernels = n;
    if (n_forwards) *n_forwards = pf.forwards;
    pf.marks.clear();
    pf.used = 0;
    pf.forwards = 0;
    return MOE_OK;
}

const char *moe_last_error_message(const moe_ctx *ctx)
{
    if (ctx) return ctx->last_error.c_str();
    return g_last_error.c_str();
}

int moe_debug_permutation(moe_ctx *ctx, int32_t *offsets, int32_t *perm_token, int32_t *T_out)
{
    if (!ctx || !offsets || !perm_token) return fail(nullptr, MOE_ERR_INVALID_ARGS, "null argument");
    if (ctx->last_layer < 0) return fail(ctx, MOE_ERR_INVALID_ARGS, "no forward has run on this context");
    const LayerStore &L = ctx->layers[ctx->last_layer];
    CUDA_TRY(ctx, cudaSetDevice(ctx->spec.device), "cudaSetDevice");
    CUDA_TRY(ctx, cudaStreamSynchronize(ctx->stream), "sync");
    CUDA_TRY(ctx, cudaMemcpy(offsets, ctx->scratch.offsets, (size_t)(L.E + 1) * 4, cudaMemcpyDeviceToHost),
             "copy offsets");
    CUDA_TRY(ctx, cudaMemcpy(perm_token, ctx->scratch.perm_token, (size_t)ctx->last_T * L.k * 4,
                             cudaMemcpyDeviceToHost),
             "copy perm");
    if (T_out) *T_out = ctx->last_T;
    return MOE_OK;
}

int moe_debug_capture_block_sums(moe_ctx *ctx, int32_t *device_buf, uint64_t n_ints)
{
    if (!ctx) return fail(nullptr, MOE_ERR_INVALID_ARGS, "null context");
    if (!device_buf != !n_ints) return fail(ctx, MOE_ERR_INVALID_ARGS, "buffer and size go together");
    ctx->dbg_isum = device_buf;
    ctx->dbg_isum_cap = n_ints;
    return MOE_OK;
}

int moe_debug_block_dots(int32_t device, int32_t quant, const void *w, const float *x, int32_t n, int32_t cols,
                         int32_t *isum, int8_t *xq, float *xd)
{
    if (!w || !x || !isum || n <= 0) return fail(nullptr, MOE_ERR_INVALID_ARGS, "null argument");
    if (quant != MOE_QUANT_Q8_0 && quant != MOE_QUANT_Q4_K)
        return fail(nullptr, MOE_ERR_CAPABILITY_MISMATCH, "block dots need Q8_0 or Q4_K");
    if (!gguf_row_bytes(quant, cols)) return fail(nullptr, MOE_ERR_TENSOR_BOUNDS, "cols not whole blocks");
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) return cuda_fail(nullptr, e, "cudaSetDevice");
    MatrixPlan plan = plan_matrix(quant, n, cols, 1);
    std::vector<uint8_t> hq(plan.qs_bytes), hm(plan.meta_bytes);
    repack_rows(plan, static_cast<const uint8_t *>(w), hq.data(), hm.data());
    const size_t nb = (size_t)n * (cols / 32);
    uint8_t *dq = nullptr, *dm = nullptr, *dxq = nullptr;
    float *dx = nullptr, *dxd = nullptr, *dxs = nullptr;
    int32_t *dis = nullptr;
    int rc = MOE_OK;
    do {
        if ((e = cudaMalloc(&dq, plan.qs_bytes)) || (e = cudaMalloc(&dm, plan.meta_bytes)) ||
            (e = cudaMalloc(&dxq, (size_t)n * cols)) || (e = cudaMalloc(&dx, (size_t)n * cols * 4)) ||
            (e = cudaMalloc(&dxd, nb * 4)) || (e = cudaMalloc(&dxs, nb * 4)) || (e = cudaMalloc(&dis, nb * 4))) {
            rc = cuda_fail(nullptr, e, "cudaMalloc(probe)");
            break;
        }
        if ((e = cudaMemcpy(dq, hq.data(), plan.qs_bytes, cudaMemcpyHostToDevice)) ||
            (e = cudaMemcpy(dm, hm.data(), plan.meta_bytes, cudaMemcpyHostToDevice)) ||
            (e = cudaMemcpy(dx, x, (size_t)n * cols * 4, cudaMemcpyHostToDevice))) {
            rc = cuda_fail(nullptr, e, "cudaMemcpy(probe)");
            break;
        }
        DevMatrix m = to_dev(plan, dq, dm);
        if ((e = (cudaError_t)launch_quantize_rows(dx, n, cols, (int8_t *)dxq, dxd, dxs, nullptr)) ||
            (e = (cudaError_t)launch_block_dots(m, (const int8_t *)dxq, n, dis, nullptr)) ||
            (e = cudaDeviceSynchronize())) {
            rc = cuda_fail(nullptr, e, "probe kernels");
            break;
        }
        if ((e = cudaMemcpy(isum, dis, nb * 4, cudaMemcpyDeviceToHost)) ||
            (xq && (e = cudaMemcpy(xq, dxq, (size_t)n * cols, cudaMemcpyDeviceToHost))) ||
            (xd && (e = cudaMemcpy(xd, dxd, nb * 4, cudaMemcpyDeviceToHost)))) {
            rc = cuda_fail(nullptr, e, "cudaMemcpy(probe out)");
            break;
        }
    } while (0);
    cudaFree(dq); cudaFree(dm); cudaFree(dxq); cudaFree(dx); cudaFree(dxd); cudaFree(dxs); cudaFree(dis);
    return rc;
}

int moe_ep_unique_id(uint8_t *id_out)
{
    if (!id_out) return fail(nullptr, MOE_ERR_INVALID_ARGS, "null id buffer");
    const char *why = nullptr;
    const NcclApi *nc = nccl_api(&why);
    if (!nc) return fail(nullptr, MOE_ERR_NCCL, "%s", why);
    ncclUniqueId uid;
    NCCL_TRY(nullptr, nc, nc->GetUniqueId(&uid), "ncclGetUniqueId");
    static_assert(sizeof(uid.internal) == MOE_EP_ID_BYTES, "NCCL unique id size");
    memcpy(id_out, uid.internal, MOE_EP_ID_BYTES);
    return MOE_OK;
}

int moe_ep_init(moe_ctx *ctx, int32_t rank, int32_t world, const uint8_t *id)
{
    if (!ctx || !id) return fail(ctx, MOE_ERR_INVALID_ARGS, "null argument");
    if (world < 1 || rank < 0 || rank >= world)
        return fail(ctx, MOE_ERR_INVALID_ARGS, "rank %d outside a world of %d", rank, world);
    if (ctx->ep.world) return fail(ctx, MOE_ERR_INVALID_ARGS, "context is already expert-parallel");
    for (const auto &L : ctx->layers)
        if (L.present) return fail(ctx, MOE_ERR_INVALID_ARGS, "moe_ep_init must come before the layer uploads");
    const char *why = nullptr;
    const NcclApi *nc = nccl_api(&why);
    if (!nc) return fail(ctx, MOE_ERR_NCCL, "%s", why);
    CUDA_TRY(ctx, cudaSetDevice(ctx->spec.device), "cudaSetDevice");
    ncclUniqueId uid;
    memcpy(uid.internal, id, MOE_EP_ID_BYTES);
    ncclComm_t comm = nullptr;
    NCCL_TRY(ctx, nc, nc->CommInitRank(&comm, world, uid, rank), "ncclCommInitRank");
    ctx->ep.comm = comm;
    ctx->ep.rank = rank;
    ctx->ep.world = world;
    void *small = nullptr;
    CUDA_TRY(ctx, cudaMalloc(&small, 8192), "cudaMalloc(expert-parallel set-up buffer)");
    ctx->ep.small = static_cast<uint8_t *>(small);
    return MOE_OK;
}

int moe_ep_plan(int32_t rank, int32_t world, int32_t E, const int32_t *all_offsets, int32_t *send_cnt,
                int32_t *send_off, int32_t *recv_cnt, int32_t *recv_off, int32_t *problems, int32_t *n_problems,
                int32_t *segments, int32_t *n_segments)
{
    if (!all_offsets || !send_cnt || !send_off || !recv_cnt || !recv_off || !problems || !n_problems || !segments ||
        !n_segments)
        return fail(nullptr, MOE_ERR_INVALID_ARGS, "null argument");
    EpPlan plan;
    if (!ep_plan(rank, world, E, all_offsets, plan))
        return fail(nullptr, MOE_ERR_INVALID_ARGS, "bad plan input (rank %d, world %d, %d experts)", rank, world, E);
    for (int r = 0; r < world; r++) {
        send_cnt[r] = plan.send_cnt[r];
        send_off[r] = plan.send_off[r];
        recv_cnt[r] = plan.recv_cnt[r];
        recv_off[r] = plan.recv_off[r];
    }
    *n_problems = (int32_t)plan.problems.size();
    for (size_t i = 0; i < plan.problems.size(); i++) {
        problems[3 * i] = plan.problems[i].expert;
        problems[3 * i + 1] = plan.problems[i].slot0;
        problems[3 * i + 2] = plan.problems[i].count;
    }
    *n_segments = (int32_t)plan.segs.size();
    for (size_t i = 0; i < plan.segs.size(); i++) {
        segments[3 * i] = plan.segs[i].slot_base;
        segments[3 * i + 1] = plan.segs[i].row_base;
        segments[3 * i + 2] = plan.segs[i].count;
    }
    return MOE_OK;
}

// Expert-parallel forward: route the local tokens, all-gather the slot
// offsets (the one host synchronisation), send each routed row to the rank
// that owns its expert, run the local experts over the received rows (outputs
// written at their received row), send the outputs back, then the local
// shared expert and the combine.
// The rest of an expert-parallel forward through peer memory, after local
// routing: plan (offsets exchanged by the ranks' kernels), dispatch of the
// routed rows into their owners' inboxes, the local experts reading the
// received rows in place, return of the outputs into the sources' output
// inboxes, the replicated shared expert and the combine. No host
// synchronisation; every cross-GPU wait is a bounded spin in a kernel.
static int ep_forward_p2p(moe_ctx *ctx, LayerStore &L, FwdParams p, int T, int ptr_kind, float *out,
                          int32_t *sel_idx, float *sel_w, const Marker &mk, int layer)
{
    EpState &ep = ctx->ep;
    Scratch &s = ctx->scratch;
    cudaStream_t st = ctx->stream;
    const EpP2PLayout &l = ep.p2p;
    uint8_t *A = ep.p2p_arena;
    const int G = ep.world, me = ep.rank, E = L.E, El = E / G, H = L.H;
    cudaError_t ce;
    ep.p2p_epoch++;
    EpP2PArgs a{};
    a.peers = reinterpret_cast<uint8_t *const *>(A + l.o_peers);
    a.own = A;
    a.rank = me; a.world = G; a.E = E; a.El = El; a.e0 = me * El; a.H = H; a.cap = l.cap;
    a.rb = l.rb; a.o_flags = l.o_flags; a.o_off = l.o_off; a.o_xin = l.o_xin; a.o_yin = l.o_yin;
    a.epoch = ep.p2p_epoch;
    a.wait_epoch = ep.p2p_epoch + ep.dbg_skew;
    a.wait_cycles = ep.dbg_wait_cycles > 0 ? ep.dbg_wait_cycles : kEpWaitCycles;
    ep.dbg_skew = 0;
    a.err = s.err;
    int32_t *misc = reinterpret_cast<int32_t *>(A + l.o_misc);
    a.ok = misc + 16;
    a.ticket = misc;
    a.n_active = misc + 4;
    a.total = misc + 8;
    a.problems = reinterpret_cast<Problem *>(A + l.o_prob);
    a.perm = reinterpret_cast<int32_t *>(A + l.o_perm);
    a.ret = reinterpret_cast<int2 *>(A + l.o_ret);
    a.offsets = s.offsets; a.perm_token = p.perm_token; a.xq = p.xq; a.xd = p.xd; a.xs = p.xs;
    a.n_slots = T * L.k;
    a.y = reinterpret_cast<const float *>(A + l.o_y);

    // the local experts over the received rows, read in place: packed int8
    // rows, or (the fused launch) the f16 rows the sources wrote
    FwdParams pe{};
    pe.T = G * l.cap; pe.H = H; pe.E = El; pe.k = 1; pe.I = L.I; pe.S = 0;
    pe.quant_x = 1;
    pe.max_problems = std::max(El, 1);
    pe.xq = reinterpret_cast<int8_t *>(A + l.o_xin);
    pe.xd = reinterpret_cast<float *>(A + l.o_xin + H);
    pe.xs = pe.xd + H / 32;
    pe.x_qstride = (int)l.rb;
    pe.x_dstride = (int)(l.rb / 4);
    pe.perm_token = a.perm; pe.problems = a.problems; pe.n_active = a.n_active;
    pe.aq = reinterpret_cast<int8_t *>(A + l.o_aq);
    pe.ad = reinterpret_cast<float *>(A + l.o_ad);
    pe.as = reinterpret_cast<float *>(A + l.o_as);
    pe.af = nullptr; pe.W = l.W;
    pe.y = reinterpret_cast<float *>(A + l.o_y); pe.y_rows = nullptr;
    pe.err = s.err;
    pe.use_tc = 0;
    // the fused f16 launch over the received rows: one pass over the local
    // experts' weights for up to 32 rows per expert (the per-source rows of
    // every rank together), gate/up + SwiGLU + down in one launch
    FwdParams pf = pe;
    pf.x_qstride = 0;   // its operands are the f16 rows below, not the packed int8 rows
    pf.x16 = A + l.o_x16;
    pf.a16dn = A + l.o_a16dn;
    pf.a16dn_stride = l.W;
    pf.dep = s.dep; pf.dep_done = s.dep ? s.dep + s.dep_cap : nullptr; pf.dep_cap = s.dep_cap;
    // its down epilogue stores each output row straight into the source rank's
    // output inbox and its last CTA raises the outputs flag: no return pass
    pf.y_peer = a.peers;
    pf.y_ret = a.ret;
    pf.y_peer_off = l.o_yin;
    pf.y_flag_off = l.o_flags + ((size_t)kEpPhaseOut * kEpMaxRanks + me) * 4;
    pf.y_epoch = a.epoch;
    pf.y_world = G;
    pf.y_ok = a.ok;
    // (the same flags as the single-GPU policy pin the streaming or int8 paths)
    const bool fused = use_fused_tc(ctx->spec, T) && (long long)G * l.cap / 16 + El + 2 <= s.dep_cap &&
                       fused_experts_ok(pf, L.dev);
    pe.use_dtc = !fused && use_int8_tc(ctx->spec, L, T, T * L.k) && decode_tc_ok(pe, L.dev);
    a.o_x16 = fused ? l.o_x16 : 0;   // the fused launch takes the rows as f16 straight from the dispatch

    // rows (with the slot offsets) out first; the plan waits for every source's
    if ((ce = launch_ep_p2p_dispatch(a, ctx->num_sms, st)) != cudaSuccess) return cuda_fail(ctx, ce, "ep dispatch");
    mk.mark("ep_dispatch");
    if ((ce = launch_ep_p2p_plan(a, st)) != cudaSuccess) return cuda_fail(ctx, ce, "ep plan");
    mk.mark("ep_plan");

    if (fused) {
        if ((ce = launch_fused_experts(pf, L.dev, L.maps, 0, ctx->num_sms, st)) != cudaSuccess)
            return cuda_fail(ctx, ce, "experts (fused f16 tensor cores)");
        mk.mark("experts_tc");
    } else if (pe.use_dtc) {
        if ((ce = launch_decode_tc(pe, L.dev, L.maps, ctx->num_sms, mk, st)) != cudaSuccess)
            return cuda_fail(ctx, ce, "experts (int8 tensor cores)");
    } else {
        if ((ce = launch_gate_up(pe, L.dev, L.maps, 0, ctx->num_sms, st)) != cudaSuccess)
            return cuda_fail(ctx, ce, "gate_up");
        mk.mark("gate_up");
        if ((ce = launch_down(pe, L.dev, L.maps, 0, ctx->num_sms, st)) != cudaSuccess) return cuda_fail(ctx, ce, "down");
        mk.mark("down");
    }
    if (!fused) {
        if ((ce = launch_ep_p2p_return(a, ctx->num_sms, st)) != cudaSuccess) return cuda_fail(ctx, ce, "ep return");
        mk.mark("ep_return");
    }

    p.y = reinterpret_cast<float *>(A + l.o_yin);   // routed outputs arrive here; shared rows follow
    if (T > 0 && L.S > 0) {
        if (p.use_tc) {
            FwdParams ps = p;
            ps.n_active = misc + 12;   // a zero word: no routed problems in this pass
            if ((ce = launch_prefill(ps, L.dev, L.maps, ctx->num_sms, mk, st)) != cudaSuccess)
                return cuda_fail(ctx, ce, "shared expert (tensor cores)");
        } else if (p.use_dtc) {
            if ((ce = launch_decode_tc(p, L.dev, L.maps, ctx->num_sms, Marker{nullptr, nullptr}, st, true)) !=
                cudaSuccess)
                return cuda_fail(ctx, ce, "shared expert (int8 tensor cores)");
        } else {
            if ((ce = launch_gate_up(p, L.dev, L.maps, 1, ctx->num_sms, st)) != cudaSuccess)
                return cuda_fail(ctx, ce, "shared gate_up");
            if ((ce = launch_down(p, L.dev, L.maps, 1, ctx->num_sms, st)) != cudaSuccess)
                return cuda_fail(ctx, ce, "shared down");
        }
        mk.mark("shared");
    }
    if ((ce = launch_ep_p2p_wait(a, kEpPhaseOut, st)) != cudaSuccess) return cuda_fail(ctx, ce, "ep wait");
    mk.mark("ep_wait");
    if (T > 0) {
        if ((ce = launch_combine(p, st)) != cudaSuccess) return cuda_fail(ctx, ce, "combine");
        mk.mark("combine");
    }
    ctx->last_layer = layer;
    ctx->last_T = T;
    if (ptr_kind == MOE_PTR_HOST) {
        if (T > 0) {
            CUDA_TRY(ctx, cudaMemcpyAsync(out, s.out, (size_t)T * H * 4, cudaMemcpyDeviceToHost, st), "copy out");
            if (sel_idx)
                CUDA_TRY(ctx, cudaMemcpyAsync(sel_idx, s.sel_idx, (size_t)T * L.k * 4, cudaMemcpyDeviceToHost, st),
                         "copy sel_idx");
            if (sel_w)
                CUDA_TRY(ctx, cudaMemcpyAsync(sel_w, s.sel_w, (size_t)T * L.k * 4, cudaMemcpyDeviceToHost, st),
                         "copy sel_w");
        }
        CUDA_TRY(ctx, cudaMemcpyAsync(ctx->status_host, s.err, sizeof(int), cudaMemcpyDeviceToHost, st),
                 "copy status");
        CUDA_TRY(ctx, cudaStreamSynchronize(st), "forward");
        if (*ctx->status_host) {
            const int code = *ctx->status_host;
            cudaMemsetAsync(s.err, 0, sizeof(int), st);
            if (code == kErrEpTimeout || code == kErrEpDesync) {
                ep.p2p_broken = true;
                return fail(ctx, MOE_ERR_TIMEOUT,
                            "a bounded peer-rank wait %s in layer %d (status %d); the exchange state is lost: "
                            "call moe_ep_reset on every rank",
                            code == kErrEpTimeout ? "ran out" : "saw a later forward", layer, code);
            }
            return fail(ctx, MOE_ERR_TIMEOUT, "a bounded device wait ran out in layer %d (status %d)", layer, code);
        }
    }
    return MOE_OK;
}

int moe_forward_ep(moe_ctx *ctx, int32_t layer, int32_t T, const float *x, float *out, int32_t *sel_idx,
                   float *sel_w, int32_t ptr_kind)
{
    if (!ctx) return fail(nullptr, MOE_ERR_INVALID_ARGS, "null context");
    EpState &ep = ctx->ep;
    if (!ep.world) return fail(ctx, MOE_ERR_INVALID_ARGS, "moe_ep_init was not called on this context");
    if (layer < 0 || layer >= (int)ctx->layers.size())
        return fail(ctx, MOE_ERR_INVALID_ARGS, "layer %d outside 0..%d", layer, (int)ctx->layers.size() - 1);
    LayerStore &L = ctx->layers[layer];
    if (!L.present) return fail(ctx, MOE_ERR_NOT_UPLOADED, "layer %d was never uploaded", layer);
    if (T < 0) return fail(ctx, MOE_ERR_INVALID_ARGS, "negative token count");
    if (T > ctx->spec.max_tokens)
        return fail(ctx, MOE_ERR_CONTEXT_LENGTH, "T=%d exceeds max_tokens=%d", T, ctx->spec.max_tokens);
    if (ptr_kind != MOE_PTR_HOST && ptr_kind != MOE_PTR_DEVICE)
        return fail(ctx, MOE_ERR_INVALID_ARGS, "unknown pointer kind %d", ptr_kind);
    if (T > 0 && (!x || !out)) return fail(ctx, MOE_ERR_INVALID_ARGS, "null x or out");
    if (T > 0 && ptr_kind == MOE_PTR_DEVICE && (((uintptr_t)x | (uintptr_t)out) & 15))
        return fail(ctx, MOE_ERR_INVALID_ARGS, "device x and out must be 16-byte aligned");
    if (ep.p2p_broken)
        return fail(ctx, MOE_ERR_TIMEOUT,
                    "the peer exchange failed in an earlier forward; call moe_ep_reset on every rank first");
    const NcclApi *nc = nccl_api();
    if (!nc) return fail(ctx, MOE_ERR_NCCL, "NCCL unavailable");
    CUDA_TRY(ctx, cudaSetDevice(ctx->spec.device), "cudaSetDevice");
    Scratch &s = ctx->scratch;
    cudaStream_t st = ctx->stream;
    const int G = ep.world, me = ep.rank, E = L.E, El = E / G, H = L.H;
    FwdParams p = local_params(ctx, L, T, ptr_kind, x, out, sel_idx, sel_w);
    Marker mk{nullptr, nullptr};
    if (ctx->prof.on) {
        ctx->prof.stream = st;
        mk = Marker{&Profiler::mark_cb, &ctx->prof};
    }
    int rc;
    bool p2p = false;   // small batches: exchange over peer memory, no host synchronisation
    if ((rc = ep_p2p_prepare(ctx, L, &p2p))) return rc;
    // the arena's all-gather buffer and pinned staging (rows and sends sized below)
    EpDims dims{G, E, H, std::max(L.I, s.W), 1, std::max(T * L.k, 1), tc_possible(ctx->spec)};
    if (!p2p && (rc = ep_reserve(ctx, dims))) return rc;

    mk.mark(nullptr);
    cudaError_t ce;
    if (T > 0) {
        if (ptr_kind == MOE_PTR_HOST)
            CUDA_TRY(ctx, cudaMemcpyAsync(s.x, x, (size_t)T * H * 4, cudaMemcpyHostToDevice, st), "copy x");
        if ((ce = launch_routing(p, st, mk)) != cudaSuccess) return cuda_fail(ctx, ce, "routing");
    } else {
        CUDA_TRY(ctx, cudaMemsetAsync(s.offsets, 0, (size_t)(E + 1) * 4, st), "memset");
    }
    if (p2p) return ep_forward_p2p(ctx, L, p, T, ptr_kind, out, sel_idx, sel_w, mk, layer);

    // exchange sizes: every rank's slot offsets by expert
    NCCL_TRY(ctx, nc, nc->AllGather(s.offsets, ep.all_off, (size_t)E + 1, ncclInt32, ep.comm, st), "ncclAllGather");
    CUDA_TRY(ctx, cudaMemcpyAsync(ep.h_off, ep.all_off, (size_t)G * (E + 1) * 4, cudaMemcpyDeviceToHost, st),
             "copy offsets");
    CUDA_TRY(ctx, cudaStreamSynchronize(st), "exchange sizes");
    mk.mark("ep_sizes");
    EpPlan plan;
    if (!ep_plan(me, G, E, ep.h_off, plan)) return fail(ctx, MOE_ERR_CUDA, "inconsistent slot offsets from the ranks");
    dims.rows = plan.n_recv;
    if ((rc = ep_reserve(ctx, dims))) return rc;
    const size_t rb = ep_row_bytes(H);

    // plan upload: n_active | problems | segments
    {
        uint8_t *h = ep.h_plan;
        *reinterpret_cast<int32_t *>(h) = (int32_t)plan.problems.size();
        Problem *hp = reinterpret_cast<Problem *>(h + 16);
        for (size_t i = 0; i < plan.problems.size(); i++)
            hp[i] = Problem{plan.problems[i].expert, plan.problems[i].slot0, plan.problems[i].count, 0};
        EpSegment *hs = reinterpret_cast<EpSegment *>(h + 16 + align_up((size_t)ep.E * sizeof(Problem), 16));
        for (size_t i = 0; i < plan.segs.size(); i++) hs[i] = plan.segs[i];
        CUDA_TRY(ctx, cudaMemcpyAsync(ep.plan_dev, h, ep_plan_bytes(G, ep.E), cudaMemcpyHostToDevice, st),
                 "copy plan");
    }
    int32_t *d_nact = reinterpret_cast<int32_t *>(ep.plan_dev);
    Problem *d_prob = reinterpret_cast<Problem *>(ep.plan_dev + 16);
    const void *d_segs = ep.plan_dev + 16 + align_up((size_t)ep.E * sizeof(Problem), 16);
    if ((ce = launch_ep_segments(d_segs, (int)plan.segs.size(), ep.perm, ctx->num_sms, st)) != cudaSuccess)
        return cuda_fail(ctx, ce, "ep segments");

    // dispatch: routed rows to the owners of their experts
    if (T > 0 && (ce = launch_ep_pack(p.xq, p.xd, p.xs, p.perm_token, T * L.k, H, ep.send_buf, ctx->num_sms, st)) !=
                     cudaSuccess)
        return cuda_fail(ctx, ce, "ep pack");
    NCCL_TRY(ctx, nc, nc->GroupStart(), "ncclGroupStart");
    for (int r = 0; r < G; r++) {
        if (plan.send_cnt[r])
            NCCL_TRY(ctx, nc,
                     nc->Send(ep.send_buf + (size_t)plan.send_off[r] * rb, (size_t)plan.send_cnt[r] * rb, ncclUint8,
                              r, ep.comm, st),
                     "ncclSend");
        if (plan.recv_cnt[r])
            NCCL_TRY(ctx, nc,
                     nc->Recv(ep.recv_buf + (size_t)plan.recv_off[r] * rb, (size_t)plan.recv_cnt[r] * rb, ncclUint8,
                              r, ep.comm, st),
                     "ncclRecv");
    }
    NCCL_TRY(ctx, nc, nc->GroupEnd(), "ncclGroupEnd");
    if ((ce = launch_ep_unpack(ep.recv_buf, plan.n_recv, H, ep.xq, ep.xd, ep.xs, ctx->num_sms, st)) != cudaSuccess)
        return cuda_fail(ctx, ce, "ep unpack");
    mk.mark("ep_dispatch");

    // the local experts over the received rows
    if (plan.n_recv > 0) {
        FwdParams pe{};
        pe.T = plan.n_recv; pe.H = H; pe.E = El; pe.k = 1; pe.I = L.I; pe.S = 0;
        pe.quant_x = 1;
        pe.max_problems = std::max(El, 1);
        pe.xq = ep.xq; pe.xd = ep.xd; pe.xs = ep.xs;
        pe.perm_token = ep.perm; pe.problems = d_prob; pe.n_active = d_nact;
        pe.aq = ep.aq; pe.ad = ep.ad; pe.as = ep.as; pe.af = nullptr; pe.W = ep.W;
        pe.y = ep.y; pe.y_rows = ep.perm;
        pe.err = s.err;
        pe.tile_off = ep.tile_off;
        pe.a16 = ep.a16; pe.a16dn = ep.a16dn; pe.a16_stride = H; pe.a16dn_stride = ep.W; pe.slots_cap = ep.rows_cap;
        Scratch tcs{};
        tcs.tc = ep.tc;
        pe.use_tc = use_tensor_cores(ctx->spec, L, tcs, plan.n_recv);
        pe.use_dtc = !pe.use_tc && use_int8_tc(ctx->spec, L, T, T * L.k) && decode_tc_ok(pe, L.dev);
        if (pe.use_tc) {
            if ((ce = launch_prefill(pe, L.dev, L.maps, ctx->num_sms, mk, st)) != cudaSuccess)
                return cuda_fail(ctx, ce, "experts (tensor cores)");
        } else if (pe.use_dtc) {
            if ((ce = launch_decode_tc(pe, L.dev, L.maps, ctx->num_sms, mk, st)) != cudaSuccess)
                return cuda_fail(ctx, ce, "experts (int8 tensor cores)");
        } else {
            if ((ce = launch_gate_up(pe, L.dev, L.maps, 0, ctx->num_sms, st)) != cudaSuccess)
                return cuda_fail(ctx, ce, "gate_up");
            mk.mark("gate_up");
            if ((ce = launch_down(pe, L.dev, L.maps, 0, ctx->num_sms, st)) != cudaSuccess)
                return cuda_fail(ctx, ce, "down");
            mk.mark("down");
        }
    }

    // combine exchange: outputs back to their source ranks, in the sources' slot order
    NCCL_TRY(ctx, nc, nc->GroupStart(), "ncclGroupStart");
    for (int r = 0; r < G; r++) {
        if (plan.recv_cnt[r])
            NCCL_TRY(ctx, nc,
                     nc->Send(ep.y + (size_t)plan.recv_off[r] * H, (size_t)plan.recv_cnt[r] * H, ncclFloat32, r,
                              ep.comm, st),
                     "ncclSend");
        if (plan.send_cnt[r])
            NCCL_TRY(ctx, nc,
                     nc->Recv(s.y + (size_t)plan.send_off[r] * H, (size_t)plan.send_cnt[r] * H, ncclFloat32, r,
                              ep.comm, st),
                     "ncclRecv");
    }
    NCCL_TRY(ctx, nc, nc->GroupEnd(), "ncclGroupEnd");
    mk.mark("ep_return");

    if (T > 0) {
        if (L.S > 0) {   // the replicated shared expert over the local tokens
            if (p.use_tc) {
                FwdParams ps = p;
                ps.n_active = ep.zero;   // no routed problems in this pass
                const Marker smk{mk.fn ? &shared_mark_cb : nullptr, const_cast<Marker *>(&mk)};
                if ((ce = launch_prefill(ps, L.dev, L.maps, ctx->num_sms, smk, st)) != cudaSuccess)
                    return cuda_fail(ctx, ce, "shared expert (tensor cores)");
            } else if (p.use_dtc) {
                if ((ce = launch_decode_tc(p, L.dev, L.maps, ctx->num_sms, Marker{nullptr, nullptr}, st, true)) !=
                    cudaSuccess)
                    return cuda_fail(ctx, ce, "shared expert (int8 tensor cores)");
                mk.mark("shared");
            } else {
                if ((ce = launch_gate_up(p, L.dev, L.maps, 1, ctx->num_sms, st)) != cudaSuccess)
                    return cuda_fail(ctx, ce, "shared gate_up");
                if ((ce = launch_down(p, L.dev, L.maps, 1, ctx->num_sms, st)) != cudaSuccess)
                    return cuda_fail(ctx, ce, "shared down");
                mk.mark("shared");
            }
        }
        if ((ce = launch_combine(p, st)) != cudaSuccess) return cuda_fail(ctx, ce, "combine");
        mk.mark("combine");
    }
    ctx->last_layer = layer;
    ctx->last_T = T;
    if (ptr_kind == MOE_PTR_HOST) {
        if (T > 0) {
            CUDA_TRY(ctx, cudaMemcpyAsync(out, s.out, (size_t)T * H * 4, cudaMemcpyDeviceToHost, st), "copy out");
            if (sel_idx)
                CUDA_TRY(ctx, cudaMemcpyAsync(sel_idx, s.sel_idx, (size_t)T * L.k * 4, cudaMemcpyDeviceToHost, st),
                         "copy sel_idx");
            if (sel_w)
                CUDA_TRY(ctx, cudaMemcpyAsync(sel_w, s.sel_w, (size_t)T * L.k * 4, cudaMemcpyDeviceToHost, st),
                         "copy sel_w");
        }
        CUDA_TRY(ctx, cudaMemcpyAsync(ctx->status_host, s.err, sizeof(int), cudaMemcpyDeviceToHost, st),
                 "copy status");
        CUDA_TRY(ctx, cudaStreamSynchronize(st), "forward");
        if (*ctx->status_host) {
            cudaMemsetAsync(s.err, 0, sizeof(int), st);
            return fail(ctx, MOE_ERR_TIMEOUT, "a bounded device wait ran out in layer %d (status %d)", layer,
                        *ctx->status_host);
        }
    }
    return MOE_OK;
}

uint64_t moe_row_bytes(int32_t quant, int32_t cols) { return gguf_row_bytes(quant, cols); }

}  // extern "C"

void jmoe::record_error(const char *msg) { g_last_error = msg ? msg : ""; }

extern "C" {

}  // extern "C"
