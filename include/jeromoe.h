/*
 * jeromoe.h -- C ABI of the B200 (sm_100a) mixture-of-experts FFN path.
 *
 * This is the drop-in boundary for jero-engine's MoE block. Each entry point
 * names the reference interface it replaces (paths relative to the
 * jero-engine source tree). Plain pointers and sizes only; no CUDA or torch
 * types appear in the signatures (streams are passed as void*).
 *
 * Threading: one context per model and device, one CUDA stream per context.
 * Calls on one context must be serialised by the caller (the reference runs
 * the block under the engine's cycle-exclusive step, src/engine.rs:251-274).
 * No entry point aborts the process; every failure returns a status code and
 * leaves a message for moe_last_error_message().
 */
#ifndef JEROMOE_H
#define JEROMOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MOE_ABI_VERSION 1

/* Status codes. 2, 10, 11, 12 and 14 are the worker exit codes that the
 * reference maps its K3Error variants to (src/worker/error.rs:10-32, which
 * stops at 14); 15 and 16 extend that list for ContextLengthExceeded and for a
 * layer that was never uploaded, and 20-22 are device-side failures that the
 * reference (a CPU runtime) does not have. */
typedef enum moe_status {
    MOE_OK = 0,
    MOE_ERR_INVALID_ARGS = 2,          /* null pointer, bad count, unknown flag */
    MOE_ERR_CAPABILITY_MISMATCH = 10,  /* K3Error::CapabilityMismatch: unsupported quant/shape */
    MOE_ERR_INSUFFICIENT_MEMORY = 11,  /* K3Error::InsufficientLockableMemory, for device HBM */
    MOE_ERR_RESOURCE_EXHAUSTED = 12,   /* no CUDA device, allocation failure */
    MOE_ERR_CONTEXT_LENGTH = 15,       /* K3Error::ContextLengthExceeded: T > max_tokens */
    MOE_ERR_TENSOR_BOUNDS = 14,        /* K3Error::TensorBoundsError: byte size/shape mismatch */
    MOE_ERR_NOT_UPLOADED = 16,         /* forward on a layer that was never uploaded */
    MOE_ERR_CUDA = 20,                 /* CUDA runtime error (message has the name) */
    MOE_ERR_NCCL = 21,                 /* NCCL error in expert-parallel mode */
    MOE_ERR_TIMEOUT = 22               /* a bounded device or collective wait ran out */
} moe_status;

/* GGUF ggml_type ids, as the reference's QuantType (jero-core) names them. */
typedef enum moe_quant {
    MOE_QUANT_F32 = 0,
    MOE_QUANT_Q8_0 = 8,   /* 32 values / 34 B: f16 d, 32 x int8 */
    MOE_QUANT_Q4_K = 12   /* 256 values / 144 B: f16 d, f16 dmin, 12 B scales, 128 B nibbles */
} moe_quant;

/* A weight tensor as the reference's jero_core::TensorView describes it: GGUF
 * bytes (host memory, e.g. a view into the mlocked mmap) plus quant and shape.
 * shape[] is in GGUF order: [in, out] for matrices, [in, out, experts] for the
 * stacked expert tensors (src/qwen_deepseek.rs:2684-2698). data == NULL means
 * the tensor is absent (ModelWeights::contains_tensor == false). */
typedef struct moe_tensor {
    const void *data;
    uint64_t nbytes;
    int32_t quant;
    int32_t n_dims;
    int64_t shape[4];
} moe_tensor;

/* Routing modes. MOE_ROUTE_SOFTMAX_TOPK with normalize=1 is the reference's
 * only mode (select_top_k_experts, src/gemma.rs:362-442, plus the exp_probs_b
 * variant, src/qwen_deepseek.rs:773-831). The rest is build-defined. */
typedef enum moe_route {
    MOE_ROUTE_SOFTMAX_TOPK = 0,
    MOE_ROUTE_GROUP_LIMITED = 1   /* keep topk_groups of n_groups by best member, then top-k */
} moe_route;

/* One MoE layer: the tensors dispatch_qwen3_moe_ffn looks up by name
 * (src/qwen_deepseek.rs:860-932) plus the recipe's MoeDispatchSpec fields
 * (src/qwen_deepseek.rs:81-87). */
typedef struct moe_layer_desc {
    int32_t hidden;          /* H = norm_ffn_in.len() */
    int32_t num_experts;     /* E */
    int32_t top_k;           /* k */
    int32_t expert_ffn_dim;  /* I (validated against the expert tensors) */
    int32_t use_shared_expert;
    int32_t route_mode;      /* moe_route */
    int32_t normalize;       /* 1 = renormalise chosen weights (reference behaviour) */
    int32_t n_groups;        /* MOE_ROUTE_GROUP_LIMITED only */
    int32_t topk_groups;
    float   routed_scale;    /* multiplies weights when normalize == 0 (1.0 = raw softmax) */
    moe_tensor router;       /* blk.L.ffn_gate_inp.weight   [H, E] f32 */
    moe_tensor exp_probs_b;  /* blk.L.exp_probs_b.bias      [E] f32, optional (selection only) */
    moe_tensor logit_bias;   /* build-defined [E] f32, optional: added to the logits */
    moe_tensor gate_exps;    /* blk.L.ffn_gate_exps.weight  [H, I, E] */
    moe_tensor up_exps;      /* blk.L.ffn_up_exps.weight    [H, I, E] */
    moe_tensor down_exps;    /* blk.L.ffn_down_exps.weight  [I, H, E] */
    moe_tensor gate_shexp;   /* blk.L.ffn_gate_shexp.weight [H, S], optional */
    moe_tensor up_shexp;     /* blk.L.ffn_up_shexp.weight   [H, S], optional */
    moe_tensor down_shexp;   /* blk.L.ffn_down_shexp.weight [S, H], optional */
} moe_layer_desc;

typedef struct moe_device_spec {
    int32_t device;            /* CUDA ordinal */
    int32_t max_tokens;        /* largest T one forward may take (sizes the scratch) */
    int32_t max_layers;        /* layer slots in the device store */
    int32_t flags;             /* MOE_FLAG_* */
    uint64_t reserve_bytes;    /* HBM left free for other users of the device */
} moe_device_spec;

/* Expert path selection. By default forwards with at least
 * MOE_TENSOR_CORE_MIN_TOKENS tokens run the experts as tensor-core GEMMs
 * (f16 operands, f32 accumulation) and smaller ones as int8 weight-streaming
 * kernels; these flags force one path for every forward of the context. */
#define MOE_FLAG_TENSOR_CORES_ALWAYS 1
#define MOE_FLAG_TENSOR_CORES_NEVER 2
/* Expert parallelism: exchange through NCCL even for batches that would use
 * the peer-memory exchange (see moe_forward_ep). */
#define MOE_FLAG_EP_NCCL_ONLY 4
#define MOE_TENSOR_CORE_MIN_TOKENS 256
/* Below MOE_TENSOR_CORE_MIN_TOKENS, forwards with at least
 * MOE_INT8_TENSOR_CORE_MIN_TOKENS tokens run the experts on the tensor cores
 * with integer operands (the GGUF quants and the int8 activation blocks,
 * exact int32 block sums, f32 block scaling) when the layer has a shared
 * expert, Q8_0 experts, or at least six routed rows per expert on average;
 * other small batches run on the int8 weight-streaming kernels. These flags
 * force one of the two. */
#define MOE_FLAG_INT8_TENSOR_CORES_NEVER 8
#define MOE_FLAG_INT8_TENSOR_CORES_ALWAYS 16
#define MOE_INT8_TENSOR_CORE_MIN_TOKENS 16
/* By default, forwards below MOE_TENSOR_CORE_MIN_TOKENS run the whole expert
 * FFN (gate/up, SwiGLU, down) as one launch on the tensor cores with f16
 * operands: each weight value is expanded from its GGUF block once, the block
 * scales folded in, and accumulated over the whole K in f32. This flag turns
 * that off (the int8 paths above then apply); the two MOE_FLAG_INT8_* flags
 * also select the int8 paths. */
#define MOE_FLAG_FUSED_TC_NEVER 32
/* The fused launch has two forms: integer operands (tcgen05 kind::i8 on the
 * GGUF quants and the int8 activation blocks, exact int32 block sums scaled
 * per block in f32) when the routed slots per expert average at most
 * MOE_FUSED_I8_MAX_SLOTS_PER_EXPERT, f16 operands above. These flags force one. */
#define MOE_FLAG_FUSED_I8_NEVER 64
#define MOE_FLAG_FUSED_I8_ALWAYS 128
#define MOE_FUSED_I8_MAX_SLOTS_PER_EXPERT 8
/* A forward of fewer than MOE_FUSED_MIN_TOKENS tokens (one token: each routed
 * expert has one slot) runs the streaming int8 kernels rather than a fused
 * launch: their short per-tile chains beat the fused launch's serial K steps
 * when only k experts stream. MOE_FLAG_FUSED_I8_NEVER / ALWAYS still force the
 * fused launch. */
#define MOE_FUSED_MIN_TOKENS 2

/* Memory the admission check compares against. The real inspector reads
 * cudaMemGetInfo on spec->device; tests pass a fixed one, as the reference's
 * MockMemoryInspector does (src/memory.rs:1519-1547). */
typedef struct moe_mem_inspector {
    uint64_t free_bytes;
    uint64_t total_bytes;
} moe_mem_inspector;

/* Device footprint, the HBM counterpart of MemoryFootprint (src/memory.rs:792-829). */
typedef struct moe_footprint {
    uint64_t weight_bytes;          /* device-layout bytes of all layers */
    uint64_t scratch_bytes;         /* per-forward working set for max_tokens */
    uint64_t total_required_bytes;  /* weight + scratch */
    uint64_t budget_bytes;          /* free - reserve */
    uint64_t prefill_arena_bytes;   /* optional tensor-core prefill workspace (0 if downgraded) */
    int32_t  prefill_enabled;       /* 0 when the optional arena did not fit */
    int32_t  _pad;
} moe_footprint;

/* Residency counters, the device counterpart of RepackSummary (src/weights.rs:34-49). */
typedef struct moe_residency {
    int32_t layers_resident;
    int32_t upload_count;
    uint64_t resident_bytes;        /* device bytes held by layer weights */
    uint64_t gguf_bytes;            /* GGUF bytes those uploads consumed */
    uint64_t scratch_bytes;
} moe_residency;

typedef struct moe_ctx moe_ctx;

/* Pointer kinds for moe_forward. */
#define MOE_PTR_HOST 0    /* host buffers; the call copies in/out and returns when done */
#define MOE_PTR_DEVICE 1  /* device buffers on spec->device; asynchronous on the context stream */

/* Creates a context on one device. Replaces the model-scoped state that
 * LockedModelWeights::open_with_admission sets up (src/weights.rs:626-638). */
int moe_ctx_create(const moe_device_spec *spec, moe_ctx **out);

/* Frees every device buffer; like Drop for LockedModelWeights (src/weights.rs:1146-1171). */
int moe_ctx_destroy(moe_ctx *ctx);

/* Runs subsequent work on a caller-provided cudaStream_t (NULL = the context's own). */
int moe_ctx_set_stream(moe_ctx *ctx, void *cuda_stream);

/* Checks that n layers plus the forward scratch fit in device memory, with the
 * fail-closed and optional-arena-downgrade rules of
 * check_footprint_against_inspector (src/memory.rs:1576-1605).
 * inspector == NULL reads cudaMemGetInfo. Never allocates. */
int moe_admission_check(const moe_device_spec *spec, const moe_layer_desc *layers, int32_t n_layers,
                        const moe_mem_inspector *inspector, moe_footprint *out);

/* Validates one layer's tensors and uploads them once into device-resident,
 * expert-major, 128-byte-aligned layouts (the device side of
 * prepare_repacked_weights, src/weights.rs:776-868, which leaves the 3-D expert
 * stacks as mmap views, src/weights.rs:89-92). Re-uploading a layer replaces it. */
int moe_layer_upload(moe_ctx *ctx, int32_t layer, const moe_layer_desc *desc);

/* The batched MoE block: T tokens of x [T x H] f32 -> out [T x H] f32, with
 * the chosen experts sel_idx [T x k] and weights sel_w [T x k] in rank order.
 * Row t of the result equals dispatch_qwen3_moe_ffn(out_t, x_t, layer, ...)
 * (src/qwen_deepseek.rs:847-951) for that token. sel_idx / sel_w may be NULL. */
int moe_forward(moe_ctx *ctx, int32_t layer, int32_t T, const float *x, float *out,
                int32_t *sel_idx, float *sel_w, int32_t ptr_kind);

/* The FFN pre-norm of an uploaded layer for moe_forward_block: the RMSNorm
 * weight [H] f32 in host memory (blk.L.ffn_norm.weight) and eps. NULL weight,
 * or a non-finite entry, reads as 1.0, as read_f32_weight_or_default does
 * (src/qwen_deepseek.rs:491-519, used at :1279-1284). A re-upload of the layer
 * drops the norm. */
int moe_layer_set_ffn_norm(moe_ctx *ctx, int32_t layer, const float *weight, float eps);

/* The FFN sublayer around the MoE block for T tokens of the residual stream:
 * out = hidden + MoE(rmsnorm(hidden, ffn_norm, eps)), the reference's
 * src/qwen_deepseek.rs:1279-1306 (rmsnorm_standard, dispatch_qwen3_moe_ffn,
 * hidden += ffn_out) for a MoE layer, without the host round trip between
 * the norm, the block and the residual add. out may equal hidden. The norm
 * uses a fixed f32 order (lane partials (h/4) mod 32 of x*x as fmaf chains,
 * xor butterfly, mean, + eps, 1/sqrt, x * inv * w), the same in the oracle;
 * the reference kernel's order is not visible. Needs moe_layer_set_ffn_norm. */
int moe_forward_block(moe_ctx *ctx, int32_t layer, int32_t T, const float *hidden, float *out,
                      int32_t *sel_idx, float *sel_w, int32_t ptr_kind);

/* Layer-major prefill of a stack of MoE FFN sublayers: layers first_layer ..
 * first_layer + n_layers - 1 (uploaded, with their FFN norm set, one hidden
 * width) each take all T tokens at once, in layer order, in place on hidden
 * [T x H] (moe_forward_block per layer). For such a stack this equals the
 * reference's token-major prefill loop, run_prefill_with_hidden
 * (src/qwen_deepseek.rs:2217-2316), since each sublayer treats its tokens
 * independently (the attention sublayers between them stay on the host path).
 * MOE_PTR_HOST: one copy each way for the whole stack, synchronous;
 * MOE_PTR_DEVICE: asynchronous on the context's stream. */
int moe_prefill_ffn_layers(moe_ctx *ctx, int32_t first_layer, int32_t n_layers, int32_t T, float *hidden,
                           int32_t ptr_kind);

/* The LM head, project_lm_head (src/qwen_deepseek.rs:584-632), on the device.
 * Upload: the head is output_weight when present, else token_embd (the tied
 * embedding alias the reference resolves by tensor presence); GGUF [hidden,
 * vocab] F32 / Q8_0 / Q4_K (other types: MOE_ERR_CAPABILITY_MISMATCH). Both
 * absent (NULL or data NULL) is allowed: calls then give the reference's
 * synthetic logits. A tensor of another shape is kept as elements / hidden
 * rows and used only when a call's n_logits equals them (the reference's
 * second branch); otherwise the synthetic logits. A new upload replaces the
 * head. */
int moe_lm_head_upload(moe_ctx *ctx, const moe_tensor *output_weight, const moe_tensor *token_embd, int32_t hidden);
/* logits [T x n_logits] of T final-normed rows normed [T x hidden]: per row
 * the head's first min(n_logits, rows) rows, then normed[i mod hidden] * 0.05
 * for the logits past them; without a usable head base + normed[i mod hidden]
 * * 0.1 + (i mod 13) * 0.01 with base = tanh(sum(normed) / 16). T <= max_tokens.
 * The product uses the int8 activation blocks of the expert paths: integer
 * block sums below 16 rows (streaming kernel, or the int8 tensor cores from 8
 * rows on heads of whole 128-row tiles), the f16 tensor-core GEMM from 16
 * rows on such heads (within the same 1e-2 row tolerance); the MOE_FLAG_*
 * tensor-core flags force a form. MOE_PTR_HOST: synchronous; MOE_PTR_DEVICE:
 * asynchronous on the context's stream (status via moe_device_status). */
int moe_lm_head(moe_ctx *ctx, int32_t T, const float *normed, float *logits, int32_t n_logits, int32_t ptr_kind);

int moe_residency_summary(const moe_ctx *ctx, moe_residency *out);

/* Reads and clears the device status word of ctx (synchronises the context
 * stream). *status != 0 (and MOE_ERR_TIMEOUT) when a bounded wait inside a
 * kernel gave up since the last check; host-pointer forwards check it themselves. */
int moe_device_status(moe_ctx *ctx, int32_t *status);

/* ---- per-kernel timing (the device counterpart of PassTiming, src/engine.rs:136) ---- */

typedef struct moe_kernel_time {
    char name[32];       /* kernel of the forward sequence ("router", "gate_up", ...) */
    double total_ms;     /* summed CUDA-event durations on the context stream */
    int64_t launches;
} moe_kernel_time;

/* While enabled, every forward records a CUDA event after each of its kernels
 * on the context stream (no host synchronisation). */
int moe_ctx_set_profiling(moe_ctx *ctx, int32_t enabled);

/* Synchronises the context stream, folds the recorded events into per-kernel
 * totals and clears them. Returns up to cap entries; *n_kernels gets the number
 * of distinct kernels, *n_forwards the forwards timed since the last read. */
int moe_profile_read(moe_ctx *ctx, moe_kernel_time *out, int32_t cap, int32_t *n_kernels, int32_t *n_forwards);

/* Message of the last failure on ctx (or of the last context-free failure when
 * ctx == NULL). Valid until the next call on the same context. */
const char *moe_last_error_message(const moe_ctx *ctx);

/* ---- parity probes (test support; same device code as the forward path) ---- */

/* Copies the dispatch permutation of the last forward on ctx to host memory:
 * offsets [E+1] (slot range of each expert) and perm_token [T*k] (token of
 * each slot, experts ascending, tokens ascending inside an expert). */
int moe_debug_permutation(moe_ctx *ctx, int32_t *offsets, int32_t *perm_token, int32_t *T_out);

/* Parity probe of the int8 tensor-core expert paths (the per-projection
 * launches and the fused small-batch launch): while device_buf is set
 * (n_ints int32 on the context's device; NULL, 0 turns it off), forwards that
 * run such a path store the raw int32 sum of every 32-value block of the routed
 * gate/up products before any scaling, at
 * [slot][0 gate / 1 up][row of I][block of H/32] (slots as in
 * moe_debug_permutation). Forwards whose sums do not fit store nothing. */
int moe_debug_capture_block_sums(moe_ctx *ctx, int32_t *device_buf, uint64_t n_ints);

/* Quantises rows x [n x cols] f32 with the forward path's activation
 * quantiser and returns the int32 sum of each 32-value block against GGUF
 * rows w (host bytes, quant Q8_0 or Q4_K, n rows): isum [n x cols/32].
 * xq [n x cols] and xd [n x cols/32] receive the quantised activations. */
int moe_debug_block_dots(int32_t device, int32_t quant, const void *w, const float *x, int32_t n,
                         int32_t cols, int32_t *isum, int8_t *xq, float *xd);

/* Tensor-core throughput probe (measurement support): n_mma back-to-back
 * tcgen05.mma of one shape on every SM of `device`, operands in shared memory
 * (a_tmem = 1: A in TMEM, m = 128 only), issued by n_acc warps (1..4) of
 * each CTA, or for n_acc < 0 by lanes 0..-n_acc-1 (up to 8) of one warp, each
 * issuer into its own accumulator (|n_acc| * n <= 256); kind 0 = f16 inputs with f32 accumulation
 * (K = 16 per MMA), kind 1 = int8 (s8 x s8, s32 accumulation, K = 32).
 * *tops: dense tera-operations per second over the whole launch (2*m*n*K per
 * MMA); *cycles_per_mma: SM clock cycles per MMA of one issuing warp on the
 * slowest SM. m = 64 or
 * 128, n = 16..256 in steps of 16. No counterpart in the reference; it
 * measures the peaks the expert GEMMs are held against. */
int moe_probe_tensor(int32_t device, int32_t kind, int32_t m, int32_t n, int32_t a_tmem, int32_t n_acc,
                     int32_t ctas_per_sm, int32_t n_mma, double *tops, double *cycles_per_mma);

/* ---- routing without allocation ----
 * No counterpart in the reference. For callers that cannot allocate device
 * memory or let a library do it (a runtime that owns all device memory
 * through its own pool, or a decode loop held to zero allocations): the
 * router logits, top-k selection and dispatch permutation of T tokens, with
 * the kernels' working memory in one fixed 2 MiB static device array instead
 * of a context. All pointers are device pointers on `device`; x [T x H] and
 * router [E x H] f32 (16-byte aligned), logit_bias / sel_bias [E] or NULL
 * (as moe_layer_desc's logit_bias / exp_probs_b); outputs sel_idx, sel_w
 * [T x top_k], offsets [E+1], perm_token [T x top_k] as moe_forward and
 * moe_debug_permutation report them. n_groups > 0 selects group-limited
 * routing. Limits: T <= 1024, E <= 256, top_k <= 16; larger shapes return
 * MOE_ERR_CONTEXT_LENGTH. Asynchronous on `stream` (a cudaStream_t). The
 * first call on a device resolves the array's address, so make it before
 * capturing the stream into a graph. Every call shares the array: calls that
 * overlap on the GPU race. The calling thread's current device is the same
 * after the call. Errors: moe_last_error_message(NULL). */
int moe_route_noalloc(int32_t device, const float *x, const float *router, const float *logit_bias,
                      const float *sel_bias, int32_t T, int32_t H, int32_t E, int32_t top_k, int32_t normalize,
                      float routed_scale, int32_t n_groups, int32_t topk_groups, int32_t *sel_idx, float *sel_w,
                      int32_t *offsets, int32_t *perm_token, void *stream);

/* ---- expert parallelism (one process per GPU) ----
 * No counterpart in the reference, which runs the block on one host. A world
 * of G contexts (one per GPU, typically one process each) shards the routed
 * experts: rank g holds experts [g*E/G, (g+1)*E/G) of every layer, the router
 * and the shared expert are replicated, and each rank routes its own tokens.
 * A forward exchanges the routed token rows (int8 activation blocks with
 * their scales) with the owning ranks and the expert outputs back over NCCL
 * (send/recv, one group per direction); the combine is local. Row t of a
 * rank's result equals moe_forward of that rank's tokens on one GPU holding
 * all experts.
 *
 * Bootstrap: one rank calls moe_ep_unique_id and passes the bytes to every
 * rank out of band; each rank then calls moe_ep_init before uploading layers.
 * Every rank must call moe_forward_ep for the same layers in the same order
 * (T may differ per rank, 0 included). NCCL is loaded at run time
 * (libnccl.so.2, the one already in the process when there is one). */
#define MOE_EP_ID_BYTES 128

int moe_ep_unique_id(uint8_t *id_out);

/* Binds ctx to rank `rank` of `world` (E of every layer must be a multiple of
 * world). Collective: blocks until all ranks have joined. world == 1 is
 * allowed (an exchange with itself). */
int moe_ep_init(moe_ctx *ctx, int32_t rank, int32_t world, const uint8_t *id);

/* moe_forward for this rank's T tokens with the experts sharded across the
 * world. Host synchronisation: once per call, after the all-gather of the
 * per-expert slot counts (the exchange sizes). */
int moe_forward_ep(moe_ctx *ctx, int32_t layer, int32_t T, const float *x, float *out,
                   int32_t *sel_idx, float *sel_w, int32_t ptr_kind);

/* After moe_forward_ep (or moe_device_status) reports MOE_ERR_TIMEOUT for a
 * peer-rank wait -- a peer's flag that did not arrive within the bound, or one
 * already past the current forward -- the exchange state of the world is lost:
 * the failing rank stored nothing into any peer's memory for that forward, its
 * peers' waits run out too, and every later moe_forward_ep fails until every
 * rank has called moe_ep_reset. Collective: clears this rank's exchange flags
 * and counters, with a rendezvous before and after so that no rank writes into
 * a peer before the peer is clean. No counterpart in the reference. */
int moe_ep_reset(moe_ctx *ctx);

/* Fault injection for tests (no counterpart in the reference): the next
 * moe_forward_ep on ctx waits for a flag epoch skewed by epoch_skew (a flag
 * nothing raises), and every peer-flag wait from now on is bounded by
 * wait_cycles SM clock cycles (0: the default, about 2 s). Makes a bounded
 * device wait run out without a device fault. */
int moe_debug_ep_fault(moe_ctx *ctx, uint32_t epoch_skew, int64_t wait_cycles);

/* The exchange plan of one rank, as moe_forward_ep computes it from the
 * all-gathered slot offsets all_offsets [world][E+1] (host work only):
 * send_cnt / send_off / recv_cnt / recv_off [world] rows per peer; problems
 * [E/world][3] = (local expert, first slot, slot count) for the local experts
 * that received rows, in expert order (*n_problems of them); segments
 * [world*E/world][3] = (first slot, first received row, rows) of each
 * (local expert, source rank) pair (*n_segments). */
int moe_ep_plan(int32_t rank, int32_t world, int32_t E, const int32_t *all_offsets, int32_t *send_cnt,
                int32_t *send_off, int32_t *recv_cnt, int32_t *recv_off, int32_t *problems, int32_t *n_problems,
                int32_t *segments, int32_t *n_segments);

/* ---- host utilities (no device work) ---- */

/* GGUF row bytes for cols values of quant (0 if cols is not a whole number of blocks). */
uint64_t moe_row_bytes(int32_t quant, int32_t cols);

/* The repository's quantiser: f32 rows -> GGUF Q8_0 / Q4_K bytes. */
int moe_quantize_rows(int32_t quant, const float *src, int64_t rows, int32_t cols, void *dst,
                      int32_t n_threads);

/* Seeded N(0, sigma^2) values: element i of (seed, stream) is a fixed function
 * of the three numbers (counter-based splitmix64 + Box-Muller). */
int moe_gen_normal(uint64_t seed, uint64_t stream, uint64_t n, float sigma, float *dst,
                   int32_t n_threads);

#ifdef __cplusplus
}
#endif
#endif
