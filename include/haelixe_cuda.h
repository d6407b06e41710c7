/*
 * haelixe_cuda.h - C ABI of the B200 (sm_100a) fused attention library.
 *
 * This is the boundary that haelixe's Rust crate binds through `extern "C"`
 * (a build.rs step compiles this library with nvcc and links it).
 * Plain pointers and sizes only: device pointers are raw CUDA device
 * addresses on the context's device, host pointers are ordinary host memory.
 *
 * Reference interfaces replaced (paths inside sethigris/haelixe):
 *   hx_ctx_create / hx_ctx_destroy    <- GpuContext::new (src/gpu/mod.rs:38)
 *                                        and Device::gpu (src/device.rs:16-18)
 *   hx_alloc / hx_free / hx_arena_*   <- GpuMemoryArena::allocate / free / reset
 *                                        (src/gpu/arena.rs:25,64,76), and
 *                                        GpuAllocation::drop (arena.rs:113-131)
 *   hx_bin_size                       <- get_bin_size (src/gpu/arena.rs:84-91)
 *   hx_copy_h2d / hx_copy_d2h         <- Tensor::to upload / download_from_gpu
 *                                        (src/tensor.rs:300-391)
 *   hx_flash_attention_fwd            <- GpuContext::flash_attention_gpu
 *                                        (src/gpu/mod.rs:1336-1418), called by
 *                                        Tensor::flash_attention (src/tensor.rs:644-666)
 *   hx_flash_attention_bwd            <- FlashAttentionOp::backward
 *                                        (src/ops/flash_attention.rs:16-39)
 *   hx_attn_fwd_strided / _bwd_strided   the same two operations on strided
 *                                        [B,H,S,D] views, replacing the
 *                                        view/transpose/view head split of
 *                                        MultiHeadAttention::forward
 *                                        (src/nn/attention.rs:62-73,91-94)
 *   hx_rope_fwd / hx_rope_bwd         <- rope_forward / rope_backward
 *                                        (src/kernels/rope.rs:5-82)
 *   hx_linear_fwd / hx_linear_bwd     <- Linear::forward (src/nn/linear.rs:54-56)
 *                                        and the matmul/add backward it records
 *   hx_rmsnorm_fwd / hx_rmsnorm_bwd   <- rms_norm_forward / rms_norm_backward
 *                                        (src/kernels/rms_norm.rs:20-132)
 *   hx_add                            <- kernels::add (src/kernels/binary.rs:40), the
 *                                        autograd walk's gradient accumulation
 *   hx_gelu_fwd / hx_gelu_bwd         <- gelu / gelu_backward
 *                                        (src/kernels/activations.rs:192-237)
 *   hx_linear_residual_fwd            <- Linear::forward followed by the residual
 *                                        add of TransformerBlock::forward
 *                                        (src/nn/transformer.rs:26-40)
 *   hx_cross_entropy                  <- Tensor::cross_entropy (src/tensor.rs:754-801)
 *                                        with cross_entropy_forward/_backward
 *                                        (src/kernels/loss.rs:46-117)
 *   hx_adamw_step                     <- AdamW::step (src/optim.rs:128-199)
 *   hx_embedding_fwd / _bwd              a token embedding (the reference has none)
 *   hx_attn_bwd_rope_strided          <- FlashAttentionOp::backward followed by
 *                                        rope_backward of dq and dk (the rope ->
 *                                        attention order of src/nn/attention.rs:76-78)
 *
 * Error behaviour: every entry point returns 0 (HX_OK) or a negative
 * hx_status. The reference panics instead (e.g. src/tensor.rs:652,
 * src/gpu/mod.rs:45); a Rust wrapper turns a non-zero status into
 * `panic!` with the text of hx_last_error. All work is enqueued on the
 * context's stream and is asynchronous to the host, except the copies,
 * hx_sync and calls that must read a device status word.
 */
#ifndef HAELIXE_CUDA_H
#define HAELIXE_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define HX_ABI_VERSION 1

typedef struct hx_ctx hx_ctx;

typedef enum hx_dtype {
    HX_F32 = 0,  /* f32 storage, f32 arithmetic (the reference's only GPU dtype) */
    HX_BF16 = 1, /* bf16 storage, f32 accumulation (src/dtype.rs:4-13 BF16) */
} hx_dtype;

typedef enum hx_status {
    HX_OK = 0,
    HX_ERR_INVALID = -1,     /* null pointer, bad shape, stride or alignment */
    HX_ERR_UNSUPPORTED = -2, /* well-formed but not supported (e.g. head_dim > 256) */
    HX_ERR_CUDA = -3,        /* a CUDA runtime call failed */
    HX_ERR_OOM = -4,         /* device memory exhausted */
    HX_ERR_TIMEOUT = -5,     /* a bounded device-side wait expired; the context stays usable */
    HX_ERR_NCCL = -6,        /* a collective failed */
} hx_status;

/* Shape and element strides of one attention operand viewed as [B, H, S, D]
 * with D contiguous. q, k, v, o, dO, dQ, dK and dV of one call share it.
 * The reference's contiguous [B*H, S, D] tensors are B = B*H, H = 1,
 * stride_s = D, stride_b = S*D (what hx_flash_attention_* pass).
 * B, H or S of 0 is an empty problem: the attention and RoPE calls return
 * HX_OK without touching their operands (which may be NULL); D must be
 * positive. */
typedef struct hx_attn_shape {
    int32_t B, H, S, D;
    int64_t stride_b, stride_h, stride_s;
} hx_attn_shape;

typedef struct hx_arena_stats {
    uint64_t live_bytes;   /* binned bytes handed out and not yet returned */
    uint64_t cached_bytes; /* binned bytes parked in the free lists */
    uint64_t cached_slabs; /* number of parked slabs */
    uint64_t cached_bins;  /* number of distinct bin sizes with parked slabs */
    uint64_t hits;         /* allocations served from a free list */
    uint64_t misses;       /* allocations that went to the CUDA pool */
} hx_arena_stats;

/* ---- library / context ---------------------------------------------------- */
int hx_abi_version(void);
const char* hx_status_string(int status);

/* Creates a context on `device`: its own non-blocking stream, a binning arena
 * over a cudaMallocAsync pool, and a device status word for bounded waits. */
int hx_ctx_create(int device, hx_ctx** out);
int hx_ctx_destroy(hx_ctx* ctx);
int hx_ctx_device(const hx_ctx* ctx, int* device);
/* The cudaStream_t the context enqueues on (as void*). */
void* hx_ctx_stream(hx_ctx* ctx);
/* Enqueue on `stream` (a cudaStream_t; NULL is CUDA's legacy default stream). */
int hx_ctx_set_stream(hx_ctx* ctx, void* stream);
/* Go back to the context's own stream. */
int hx_ctx_use_own_stream(hx_ctx* ctx);
/* Blocks until the stream drains; reports a pending device timeout. */
int hx_sync(hx_ctx* ctx);
/* Copies the last error text (NUL-terminated) into buf. */
int hx_last_error(const hx_ctx* ctx, char* buf, size_t len);

/* ---- binning arena (src/gpu/arena.rs) -------------------------------------- */
/* Power-of-two bin with a 512-byte floor (arena.rs:84-91). */
uint64_t hx_bin_size(uint64_t requested_bytes);
/* Returns a slab of hx_bin_size(bytes) bytes, 256-byte aligned, stream-ordered. */
int hx_alloc(hx_ctx* ctx, uint64_t bytes, void** ptr);
/* Returns the slab to its bin: the caller calls this when its last reference
 * drops (the Arc strong_count==1 rule of arena.rs:126). */
int hx_free(hx_ctx* ctx, void* ptr);
/* Releases every parked slab back to the CUDA pool (arena.rs:76-80). */
int hx_arena_reset(hx_ctx* ctx);
/* Caps the bytes the arena may hold (handed out plus parked; 0 = no cap, the
 * reference's behaviour). An allocation past the cap first releases the
 * parked slabs, then fails with HX_ERR_OOM instead of growing the pool: a
 * memory budget for callers that share the GPU, and a way to test exhaustion. */
int hx_arena_set_limit(hx_ctx* ctx, uint64_t bytes);
int hx_arena_stats_get(const hx_ctx* ctx, hx_arena_stats* out);

/* ---- transfers --------------------------------------------------------------- */
int hx_copy_h2d(hx_ctx* ctx, void* dst_dev, const void* src_host, uint64_t bytes);
int hx_copy_d2h(hx_ctx* ctx, void* dst_host, const void* src_dev, uint64_t bytes);
int hx_copy_h2d_async(hx_ctx* ctx, void* dst_dev, const void* src_host, uint64_t bytes);
int hx_copy_d2h_async(hx_ctx* ctx, void* dst_host, const void* src_dev, uint64_t bytes);
int hx_host_alloc_pinned(uint64_t bytes, void** ptr);
int hx_host_free_pinned(void* ptr);

/* ---- fused attention, contiguous [BH, S, D] (the reference's layout) -------- */
/* o = softmax(scale * q k^T [+ causal mask]) v ; lse[BH*S] (f32, may be NULL
 * only when no backward follows) receives the per-row log-sum-exp. Without it
 * the tcgen05 kernels write a temporary one from the context's arena.
 * Mirrors the reference's Params{bh, seq_len, head_dim, scale}
 * (src/gpu/mod.rs:1354) plus the causal flag the reference lacks. */
int hx_flash_attention_fwd(hx_ctx* ctx, hx_dtype dtype, const void* q, const void* k,
                           const void* v, void* o, float* lse, int bh, int seq_len,
                           int head_dim, float scale, int causal);

/* Bytes of device workspace hx_*_bwd needs for this problem. */
int hx_attn_bwd_workspace_size(hx_dtype dtype, const hx_attn_shape* shape, uint64_t* bytes);

/* dq, dk, dv of the forward above for upstream gradient dout, from the saved
 * o and lse. workspace may be NULL: the call then takes it from the context's
 * arena and gives it back. Returns the gradients in the order [q, k, v] of
 * FlashAttentionOp::backward (src/ops/flash_attention.rs:38), with the
 * softmax scale applied to dq and dk. */
int hx_flash_attention_bwd(hx_ctx* ctx, hx_dtype dtype, const void* q, const void* k,
                           const void* v, const void* o, const void* dout, const float* lse,
                           void* dq, void* dk, void* dv, void* workspace,
                           uint64_t workspace_bytes, int bh, int seq_len, int head_dim,
                           float scale, int causal);

/* Same result as hx_flash_attention_bwd, but allocates no device memory: the
 * workspace lives in a fixed 64 MiB array compiled into the library (held on
 * every GPU that loads it until the process exits). No counterpart in the
 * reference; it exists for callers that cannot let a library allocate (a
 * runtime that gave all device memory to its own pool, a loop that cannot
 * afford cudaMalloc's synchronisation, an operator callback that must not
 * allocate). bf16 with head_dim 64 or 128 only. Problems whose workspace
 * (hx_attn_bwd_workspace_size) exceeds 64 MiB return HX_ERR_INVALID. Calls
 * share the array: calls that overlap on the GPU race, so serialize them.
 * The first call on a device resolves the array's address and keeps it; make
 * it before any stream capture, and do not call this after cudaDeviceReset.
 * A non-finite scale returns HX_ERR_INVALID. It ignores no setting silently:
 * a context forced onto the SIMT path (hx_set_force_simt) returns
 * HX_ERR_UNSUPPORTED. */
int hx_flash_attention_bwd_noalloc(hx_ctx* ctx, hx_dtype dtype, const void* q, const void* k,
                                   const void* v, const void* o, const void* dout,
                                   const float* lse, void* dq, void* dk, void* dv, int bh,
                                   int seq_len, int head_dim, float scale, int causal);

/* ---- fused attention on strided [B, H, S, D] views ------------------------- */
/* lse is contiguous [B, H, S]. */
int hx_attn_fwd_strided(hx_ctx* ctx, hx_dtype dtype, const hx_attn_shape* shape, const void* q,
                        const void* k, const void* v, void* o, float* lse, float scale,
                        int causal);
int hx_attn_bwd_strided(hx_ctx* ctx, hx_dtype dtype, const hx_attn_shape* shape, const void* q,
                        const void* k, const void* v, const void* o, const void* dout,
                        const float* lse, void* dq, void* dk, void* dv, void* workspace,
                        uint64_t workspace_bytes, float scale, int causal);

/* hx_attn_bwd_strided for attention applied to rotary-embedded q and k (the
 * order of MultiHeadAttention::forward, src/nn/attention.rs:76-78): q and k are
 * the rotated tensors the forward used, and dq, dk come back as gradients with
 * respect to the tensors before the rotation, i.e. hx_rope_bwd with rope_base
 * already applied (rope_backward, src/kernels/rope.rs:44-82). On the tcgen05
 * path the inverse rotation is part of the kernels' last writes of dk and dq. */
int hx_attn_bwd_rope_strided(hx_ctx* ctx, hx_dtype dtype, const hx_attn_shape* shape, const void* q,
                             const void* k, const void* v, const void* o, const void* dout,
                             const float* lse, void* dq, void* dk, void* dv, void* workspace,
                             uint64_t workspace_bytes, float scale, int causal, float rope_base);

/* ---- rotary embedding (src/kernels/rope.rs) ---------------------------------- */
/* Rotates interleaved pairs (2i, 2i+1) of every [.., S, D] row by
 * theta = s * base^(-2i/D), s the row's sequence index; bwd rotates by -theta.
 * x and out may alias. */
int hx_rope_fwd(hx_ctx* ctx, hx_dtype dtype, const hx_attn_shape* shape, const void* x, void* out,
                float base);
int hx_rope_bwd(hx_ctx* ctx, hx_dtype dtype, const hx_attn_shape* shape, const void* g, void* out,
                float base);
/* Q and K (same shape and strides) rotated as hx_rope_fwd does, in one
 * launch: the two rotations that precede the attention
 * (src/nn/attention.rs:76-78). Each output may alias its input. */
int hx_rope_fwd_qk(hx_ctx* ctx, hx_dtype dtype, const hx_attn_shape* shape, const void* q, const void* k,
                   void* q_out, void* k_out, float base);

/* ---- the attention block around the kernel (src/nn/attention.rs:46-98) ------------ */
/* y[rows, out] = x[rows, in] w[in, out] + b[out] (Linear::forward,
 * src/nn/linear.rs:54-56, weight stored [in, out] as in linear.rs:41); b may be
 * NULL. All row-major and contiguous, f32 accumulation. bf16: this library's
 * tcgen05 GEMM (bias added in f32 before the one bf16 rounding) whenever the
 * operands are 16-byte aligned with row lengths that are multiples of 8
 * elements, else cuBLAS. f32: cuBLAS without TF32 (the reference multiplies
 * in f32, src/kernels/matmul.rs). */
int hx_linear_fwd(hx_ctx* ctx, hx_dtype dtype, const void* x, const void* w, const void* b, void* y,
                  int rows, int in_features, int out_features);
/* Its backward: dx = dy w^T, dw = x^T dy, db = column sums of dy; each of
 * dx, dw, db may be NULL to skip it. */
int hx_linear_bwd(hx_ctx* ctx, hx_dtype dtype, const void* x, const void* w, const void* dy, void* dx,
                  void* dw, void* db, int rows, int in_features, int out_features);
/* RMSNorm over the last dimension (src/kernels/rms_norm.rs:20-55):
 * y = x / sqrt(mean(x^2) + eps) * w per row of `hidden` elements. */
int hx_rmsnorm_fwd(hx_ctx* ctx, hx_dtype dtype, const void* x, const void* w, void* y, int rows,
                   int hidden, float eps);
/* Its backward (src/kernels/rms_norm.rs:57-132): dx, and dw in f32 summed
 * over the rows. */
int hx_rmsnorm_bwd(hx_ctx* ctx, hx_dtype dtype, const void* dy, const void* x, const void* w, void* dx,
                   float* dw, int rows, int hidden, float eps);

/* out = a + b over n elements (src/kernels/binary.rs:40-60 for equal shapes): the
 * gradient accumulation of the autograd walk (src/tensor.rs:211-214); out may
 * alias a or b. */
int hx_add(hx_ctx* ctx, hx_dtype dtype, const void* a, const void* b, void* out, uint64_t n);

/* GELU, tanh form, element-wise over n elements (src/kernels/activations.rs:192-209),
 * used by FeedForward (src/nn/mlp.rs); x and y may alias. */
int hx_gelu_fwd(hx_ctx* ctx, hx_dtype dtype, const void* x, void* y, uint64_t n);
/* Its exact derivative times dy (activations.rs:211-237). */
int hx_gelu_bwd(hx_ctx* ctx, hx_dtype dtype, const void* dy, const void* x, void* dx, uint64_t n);

/* ---- the training step around the block stack (src/nn/transformer.rs, src/optim.rs) --- */
/* y = residual + x w + b: Linear::forward followed by TransformerBlock's
 * residual add (src/nn/transformer.rs:32, 37); b and residual may be NULL,
 * residual may alias y. Same layout and arithmetic as hx_linear_fwd. Its
 * backward is hx_linear_bwd plus d(residual) = dy. */
int hx_linear_residual_fwd(hx_ctx* ctx, hx_dtype dtype, const void* x, const void* w, const void* b,
                           const void* residual, void* y, int rows, int in_features, int out_features);

/* Mean cross-entropy of logits[rows, classes] (row-major) against targets[rows]
 * (src/kernels/loss.rs:46-82): loss[0] = mean over rows of logsumexp(row) -
 * row[target], written to device memory. When dlogits is not NULL it also
 * writes the gradient of that mean, (softmax(row) - onehot(target)) / rows
 * (loss.rs:86-117; like ops/cross_entropy.rs the upstream gradient is taken
 * as 1), in `dtype`. A target >= classes makes the loss NaN (the reference
 * panics on the out-of-range index). */
int hx_cross_entropy(hx_ctx* ctx, hx_dtype dtype, const void* logits, const uint32_t* targets, float* loss,
                     void* dlogits, int rows, int classes);

/* One tensor of an AdamW step: f32 master weights and moments, the gradient in
 * grad_dtype, and an optional bf16 copy of the updated weights (NULL for none)
 * for bf16 storage with f32 master weights. */
typedef struct hx_adamw_tensor {
    float* param;
    const void* grad;
    float* m;
    float* v;
    void* param_lowp;
    uint64_t n;
    int32_t grad_dtype; /* hx_dtype */
    int32_t reserved;   /* 0 */
} hx_adamw_tensor;

/* AdamW::step (src/optim.rs:128-199) over `count` tensors with step number
 * `step` >= 1 (the reference's step_count after its increment): decoupled
 * weight decay, then the moment updates and the bias-corrected step, each
 * element in the reference's order and rounding. m and v start as zeros (the
 * caller allocates them). bc1 = 1 - beta1^step and bc2 = 1 - beta2^step are
 * formed on the host by f32 binary exponentiation, as Rust's f32::powi. */
int hx_adamw_step(hx_ctx* ctx, const hx_adamw_tensor* tensors, int count, float lr, float beta1, float beta2,
                  float eps, float weight_decay, int step);

/* out[t, :] = table[ids[t], :] for t < tokens; table [vocab, dim] row-major.
 * An id >= vocab writes a NaN row. */
int hx_embedding_fwd(hx_ctx* ctx, hx_dtype dtype, const void* table, const uint32_t* ids, void* out,
                     uint64_t tokens, int vocab, int dim);
/* dtable[ids[t], :] += dout[t, :] in f32 (dtable is accumulated into, not
 * cleared); ids >= vocab are skipped. */
int hx_embedding_bwd(hx_ctx* ctx, hx_dtype dtype, const void* dout, const uint32_t* ids, float* dtable,
                     uint64_t tokens, int vocab, int dim);

/* ---- multi-GPU head sharding ------------------------------------------------------ */
/* After an all-gather of per-rank head shards, shards holds n_shards
 * contiguous blocks [B, H_shard, S, D]; writes them as [B, H, S, D]
 * (out_layout 0) or [B, S, H, D] (out_layout 1, the merged-heads layout of
 * src/nn/attention.rs:91-94), H = n_shards * H_shard. */
int hx_reassemble_heads(hx_ctx* ctx, hx_dtype dtype, const void* shards, void* out, int n_shards,
                        int B, int H_shard, int S, int D, int out_layout);

/* ---- the arena as a process's tensor allocator ------------------------------------ */
/* The reference takes every tensor's device storage from its GpuMemoryArena
 * (src/gpu/arena.rs:13-145, Tensor storage via src/storage.rs:17-26). These
 * two functions have the signatures torch's pluggable-allocator interface
 * calls (size, device, cudaStream_t as void*), so a Python host can route all
 * of its CUDA tensors through one arena per device: power-of-two bins with a
 * 512-byte floor, slabs parked on free and reused. A slab freed on one stream
 * and reused on another waits for an event of its last use. The arena's
 * context (for hx_arena_stats_get) is hx_torch_arena_context(device). */
void* hx_torch_malloc(size_t size, int device, void* stream);
void hx_torch_free(void* ptr, size_t size, int device, void* stream);
hx_ctx* hx_torch_arena_context(int device);

/* ---- the head-sharding exchange: NCCL all-gather + reassembly ------------------ */
/* The reference runs on one device and has no collective. Its multi-head
 * layer merges the per-head outputs after the attention
 * (src/nn/attention.rs:91-94, transpose(1, 2) + view to [B, S, H*D]); with
 * heads sharded across GPUs that merge needs every rank's heads, which these
 * entry points gather over NCCL (NVLink / NVSwitch) and reassemble.
 *
 * A group holds NCCL communicator ranks: one per process
 * (hx_group_create_rank, the id from hx_group_unique_id shared by the
 * caller) or all of them in one process (hx_group_create; drive each member
 * from its own host thread). NCCL is loaded at run time (libnccl.so.2);
 * without it these return HX_ERR_UNSUPPORTED. Every call that can wait on a
 * peer (initialisation, a gather, hx_group_sync) gives up after timeout_ms:
 * the communicator is aborted and HX_ERR_NCCL returned, with the reason in
 * hx_group_last_error; an aborted group only accepts hx_group_destroy.
 * flags: HX_GROUP_REGISTER registers the gather buffer with NCCL
 * (ncclCommRegister); HX_GROUP_SYMMETRIC registers it as a symmetric window
 * (collective, NCCL >= 2.27); HX_GROUP_COPY_ENGINE asks NCCL >= 2.28 to run
 * collectives on the copy engines where it can (CTA policy "zero"). */
#define HX_GROUP_ID_BYTES 128
typedef struct hx_group hx_group;
enum { HX_GROUP_REGISTER = 1, HX_GROUP_SYMMETRIC = 2, HX_GROUP_COPY_ENGINE = 4 };
/* Writes HX_GROUP_ID_BYTES bytes (an ncclUniqueId) to id. */
int hx_group_unique_id(void* id);
/* This process's rank `rank` of `nranks`, on `device`. *out is set even on
 * failure (for hx_group_last_error); destroy it either way. */
int hx_group_create_rank(int device, int nranks, int rank, const void* id, int flags, int timeout_ms,
                         hx_group** out);
/* All n ranks in this process, rank i on devices[i] (distinct devices). */
int hx_group_create(int n, const int* devices, int flags, int timeout_ms, hx_group** out);
int hx_group_destroy(hx_group* group);
int hx_group_abort(hx_group* group);
int hx_group_set_timeout(hx_group* group, int timeout_ms);
int hx_group_info(const hx_group* group, int* nranks, int* members, int* nccl_version);
int hx_group_last_error(const hx_group* group, char* buf, uint64_t n);
/* Device buffer of nranks packed slots of slot_bytes each (rank r's slot at
 * base + r * slot_bytes), owned by the group. A shard written into the
 * member's own slot is gathered in place. Collective when the group was made
 * with HX_GROUP_SYMMETRIC. */
int hx_group_gather_buffer(hx_group* group, int member, uint64_t slot_bytes, void** base);
/* Gathers every rank's shard [B, H_shard, S, D] (contiguous) into the gather
 * buffer and, if merged is not NULL, reassembles it as [B, H, S, D]
 * (layout 0) or [B, S, H, D] (layout 1), H = nranks * H_shard. Layout 2: the
 * shard is stored [B, S, H_shard, D] (the head-split view of a projection's
 * [B, S, H_shard*D] rows) and merged is [B, S, H, D], assembled by one 2D copy
 * per rank on the copy engines instead of a kernel. Runs on the
 * member's own side stream, after the work already queued on ctx's stream;
 * it returns once the work is enqueued. Order later work on ctx's stream
 * after it with hx_group_wait, or block the host with hx_group_sync. */
int hx_allgather_heads(hx_group* group, int member, hx_ctx* ctx, hx_dtype dtype, const void* shard,
                       void* merged, int B, int H_shard, int S, int D, int layout);
/* Makes ctx's stream wait (on the device) for the member's last gather. */
int hx_group_wait(hx_group* group, int member, hx_ctx* ctx);
/* Blocks the host until the member's last gather is done, or the timeout. */
int hx_group_sync(hx_group* group, int member);

/* ---- diagnostics --------------------------------------------------------------- */
/* Number of kernels this context has launched so far. */
uint64_t hx_kernel_launches(const hx_ctx* ctx);
/* Which kernel family the last attention call used on this context:
 * 0 none, 1 SIMT (any other head_dim, or forced), 2 tcgen05 (head_dim 64 or
 * 128: bf16 directly, f32 as f16 hi/lo operand planes with three MMAs per
 * product and a workspace from the context's arena in the forward). */
int hx_last_path(const hx_ctx* ctx);
/* Forces the SIMT kernels (1) or restores automatic selection (0). */
int hx_set_force_simt(hx_ctx* ctx, int force);
/* Which GEMM ran the last Linear product on this context: 0 none, 1 cuBLAS,
 * 2 the tcgen05 kernel. */
int hx_last_gemm_path(const hx_ctx* ctx);
/* bf16 Linear GEMMs: 0 = the tcgen05 kernel where it applies, its tile
 * chosen from the shape (default); 1 = always cuBLAS; 2, 3, 4 = the tcgen05
 * kernel with 128x128, 128x256 or 256x256 output tiles. */
int hx_set_gemm_backend(hx_ctx* ctx, int backend);
/* Exercises the kernels' failure path: enqueues one CTA whose bounded
 * mbarrier wait can never complete. After the wait limit (2 s) it records the
 * expiry in the context's status word and exits normally (no trap, no hang),
 * so the next hx_sync returns HX_ERR_TIMEOUT and later calls work as usual. */
int hx_selftest_wait_timeout(hx_ctx* ctx);

#ifdef __cplusplus
}
#endif

#endif /* HAELIXE_CUDA_H */
