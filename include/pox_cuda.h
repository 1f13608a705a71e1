/*
 * pox_cuda.h -- C ABI of the B200 (sm_100a) CUDA backend for ParaOxidizer's decode hot path.
 *
 * Plain pointers and sizes only: no C++ or torch types cross this boundary, so the Rust side
 * binds it with an `extern "C"` block. Every entry point cites the reference interface it
 * replaces; paths are relative to the reference repository root.
 *
 * Layout contract: all weight buffers are the unchanged `.pox` payloads
 * (crates/paraoxidizer-format/src/pox.rs:434-495): INT4 = packed nibbles (low nibble = even
 * column, kernels.rs:15-23) per row of ceil(cols/2) bytes, scale_data = per (row, group) an
 * f16 scale then an f16 min (kernels.rs:57-62); INT8 = int8 per element plus one f32
 * per-tensor scale (kernels.rs:131-154); outliers = u32 count | u32 flat indices | f16 values
 * (outlier.rs:99-110), whose values REPLACE the dequantized weight (kernels.rs:211-219).
 *
 * Errors: every call returns a pox_status. The reference returns Result<(), PoxError>; a
 * caller maps POX_ERR_LAYOUT to PoxError::Quantization and the rest to PoxError::Runtime
 * (crates/paraoxidizer-core/src/error.rs:25-26,50-51). pox_cuda_last_error() gives the message
 * of the last failure on the calling thread.
 *
 * Threading: a context may be shared by threads (the engine is shared through Arc across
 * spawn_blocking tasks, crates/paraoxidizer-serve/src/server.rs:136); calls on one context
 * are serialized internally. Synchronous calls return after the result is in host memory.
 */
#ifndef POX_CUDA_H
#define POX_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    POX_OK = 0,
    POX_ERR_LAYOUT = 1,      /* buffer sizes / dimensions inconsistent (PoxError::Quantization) */
    POX_ERR_UNSUPPORTED = 2, /* valid input this backend does not handle: caller uses the CPU path */
    POX_ERR_CUDA = 3,        /* CUDA runtime failure (PoxError::Runtime) */
    POX_ERR_NCCL = 4,        /* collective failure */
    POX_ERR_TIMEOUT = 5,     /* a bounded wait ran out */
    POX_ERR_OOM = 6,         /* device memory or paged-KV blocks exhausted */
    POX_ERR_INVALID = 7,     /* null pointer, bad handle or argument */
    POX_ERR_FORMAT = 8,      /* malformed .pox container (PoxError::Format / InvalidMagic / UnsupportedVersion /
                                Security / Json) */
    POX_ERR_INTEGRITY = 9    /* a tensor's SHA-256 differs from its index entry (PoxError::IntegrityHashMismatch) */
} pox_status;

/* DType codes, crates/paraoxidizer-core/src/tensor.rs:4-20 */
typedef enum { POX_F32 = 0, POX_F16 = 1, POX_BF16 = 2, POX_I8 = 3, POX_I4 = 4 } pox_dtype;

typedef struct pox_cuda_ctx pox_cuda_ctx;
typedef struct pox_tensor pox_tensor;

/* ---- library / context ------------------------------------------------------------------ */

/* Message of the last failed call on this thread ("" if none). */
const char* pox_cuda_last_error(void);
/* Library version string. */
const char* pox_cuda_version(void);
/* Number of CUDA devices visible (0 when there is no GPU). */
int pox_cuda_device_count(int* out);

/* Replaces MetalBackend::new() -> Option<Arc<Self>> (crates/paraoxidizer-runtime/src/
 * metal_backend.rs:64-82; the non-macOS stub returning None is :193-195). On failure *out is
 * NULL and the caller keeps the CPU path, as the engine does with None (engine.rs:97,174-207). */
int pox_cuda_create(int device, pox_cuda_ctx** out);
/* Frees every device buffer the context owns (resident tensors included). */
void pox_cuda_destroy(pox_cuda_ctx* ctx);
/* Waits for all work issued on the context's stream. */
int pox_cuda_synchronize(pox_cuda_ctx* ctx);
/* The context's CUDA stream (a cudaStream_t), for callers that chain async calls. */
void* pox_cuda_stream(pox_cuda_ctx* ctx);

/* ---- reference-shaped GEMV entry points (host slices, synchronous) ---------------------- */

/* Replaces MetalBackend::gemv_int4(&self, packed_weights, scale_data, rows, cols, group_size,
 * x, y) (metal_backend.rs:85-181): y[r] = sum_c (min_g + q*scale_g) * x[c].
 * rows == 0 || cols == 0 -> POX_OK with nothing written (:95-97).
 * scale_len < rows*ceil(cols/gs)*4 or packed_len < rows*ceil(cols/2) -> POX_ERR_LAYOUT
 * (:99-108). x needs cols floats, y rows floats (else POX_ERR_LAYOUT).
 * If (packed, scale_data) were registered by pox_cuda_tensor_upload, the resident copy is
 * used and only x and y cross the bus; otherwise the weights are copied for this call only,
 * as the Metal backend does (:111-129). */
int pox_cuda_gemv_int4(pox_cuda_ctx* ctx, const uint8_t* packed_weights, size_t packed_len,
                       const uint8_t* scale_data, size_t scale_len, size_t rows, size_t cols,
                       size_t group_size, const float* x, size_t x_len, float* y, size_t y_len);

/* Replaces quant::gemv_int4(packed, scale_data, group_size, rows, cols, outliers, x, y)
 * (crates/paraoxidizer-quant/src/kernels.rs:177-226) with the outlier table given in its
 * serialized .pox form (outlier.rs:99-110; NULL/len < 4 = no outliers, outlier.rs:113-115).
 * A table whose count runs past outlier_len -> POX_ERR_LAYOUT (from_bytes Err, :116-124).
 * Entries whose flat index is >= rows*cols are ignored, duplicates: the last entry wins. */
int pox_cuda_gemv_int4_outliers(pox_cuda_ctx* ctx, const uint8_t* packed_weights, size_t packed_len,
                                const uint8_t* scale_data, size_t scale_len, size_t group_size,
                                size_t rows, size_t cols, const uint8_t* outlier_data,
                                size_t outlier_len, const float* x, size_t x_len, float* y,
                                size_t y_len);

/* Replaces quant::gemv_int8(q_weights, scale_data, rows, cols, x, y) (kernels.rs:229-255):
 * y[r] = sum_c q*scale*x[c] with the single f32 per-tensor scale. x_len < cols, y_len < rows,
 * q_len < rows*cols or scale_len < 4 -> POX_ERR_LAYOUT (:237-241). The runtime's I8 path
 * ignores outlier tables (engine.rs:232-234), so this entry point takes none. */
int pox_cuda_gemv_int8(pox_cuda_ctx* ctx, const uint8_t* q_weights, size_t q_len,
                       const uint8_t* scale_data, size_t scale_len, size_t rows, size_t cols,
                       const float* x, size_t x_len, float* y, size_t y_len);

/* ---- resident tensors: upload once, then call with device pointers ---------------------- */

/* One .pox tensor (TensorMeta, crates/paraoxidizer-core/src/tensor.rs:116-128, plus the three
 * payload slices PoxFile::get_{tensor,scale,outlier}_data return, pox.rs:311-353). */
typedef struct {
    int dtype;            /* POX_I4, POX_I8 or POX_F16 */
    size_t rows, cols;    /* shape [rows, cols] (meta.shape.dims()[0..2]) */
    size_t group_size;    /* INT4: group size (meta.group_size). INT8: 0 = the .pox layout, one f32
                             per-tensor scale (kernels.rs:131-154); 1 = an extension with one f16 scale
                             per output row (scales = rows x 2 bytes LE; the reference's rules applied per
                             row: max_abs / 127 rounded to f16, q = round(w / that scale)). F16: ignored. */
    const uint8_t* data;  size_t data_len;
    const uint8_t* scales; size_t scale_len;   /* may be NULL for F16 */
    const uint8_t* outliers; size_t outlier_len; /* may be NULL; ignored for I8 (engine.rs:232) */
} pox_tensor_desc;

/* Uploads the tensor to HBM once, in the backend's device layout (data and scales may be host or
 * device memory; outlier tables are read on the host) (INT4/INT8 weights re-tiled
 * for 128-bit loads and tensor-core fragments; outlier table turned into a per-row CSR with
 * precomputed corrections). Replaces the per-call copies of metal_backend.rs:111-129 and the
 * per-call SparseOutlierTable::from_bytes of engine.rs:150-151. The host pointers are
 * remembered so that pox_cuda_gemv_int4* / pox_cuda_gemv_int8 calls on the same slices reuse the
 * resident copy. The match is by identity, not content: same addresses and lengths of the data,
 * scale and outlier slices, same shape, dtype and group size. So the caller must not modify those
 * host bytes, or free them and put another tensor at the same addresses, while the resident tensor
 * is alive (free it first): the calls would keep using the old resident copy. In the reference
 * these slices are an immutable mmap that outlives the engine (pox.rs:171-175). */
int pox_cuda_tensor_upload(pox_cuda_ctx* ctx, const pox_tensor_desc* desc, pox_tensor** out);
/* Frees a resident tensor (NULL is a no-op). */
int pox_cuda_tensor_free(pox_cuda_ctx* ctx, pox_tensor* t);
/* Shape and footprint of a resident tensor; any out pointer may be NULL. */
int pox_cuda_tensor_info(const pox_tensor* t, size_t* rows, size_t* cols, size_t* outlier_count,
                         size_t* device_bytes);
/* Name of the kernel a GEMV of this tensor at `batch` rows of x runs (per launch of up to 8 rows
 * for the batch <= 8 kernel): "gemv_tc_kernel" (mma.sync, batch <= 8), "gemm_tq_kernel"
 * (tcgen05 kind::i8; also below batch 9 where it was measured faster: INT4 without outliers with
 * cols >= 8192 from batch 6, INT8 with >= 16 M weights from batch 2), "gemm_tc05_kernel"
 * (tcgen05 kind::f16) or "gemv_generic" (raw .pox layout).
 * NULL if t is NULL. No counterpart in the reference (it has one CPU loop per dtype); it lets a
 * caller or a benchmark report which path served a call. */
const char* pox_cuda_tensor_gemv_kernel(const pox_tensor* t, size_t batch);

/* y[b][r] = sum_c W[r][c] * x[b][c] for b < batch, on device pointers, asynchronously on
 * `stream` (a cudaStream_t; NULL = the context's stream). x: [batch][cols] f32, y:
 * [batch][rows] f32, both device memory. Replaces project_tensor's per-dtype GEMV
 * (crates/paraoxidizer-runtime/src/engine.rs:131-291) for a resident weight. */
int pox_cuda_tensor_gemv(pox_cuda_ctx* ctx, const pox_tensor* t, const float* x_dev, size_t batch,
                         float* y_dev, void* stream);
/* Same with host x/y: copies x in and y out, synchronous. */
int pox_cuda_tensor_gemv_host(pox_cuda_ctx* ctx, const pox_tensor* t, const float* x, size_t batch,
                              float* y);
/* Same GEMV as pox_cuda_tensor_gemv, for callers that cannot allocate device memory once they
 * are running (an engine that reserved its HBM at start-up, a host runtime that only hands over
 * buffers it owns). No counterpart in the reference: it exists only because this backend's
 * GEMV needs scratch for the prepared x. That scratch is a fixed 1 MiB + 16 KiB array in device
 * memory, shared by every call on a device and held until the process exits; the call allocates
 * and frees nothing. Limit: cols <= 32768 (larger -> POX_ERR_UNSUPPORTED). Calls whose kernels
 * overlap on the same device (other streams or contexts) race on the shared array: serialize
 * them. The first call on a device looks up the array's device address (again after a context of
 * that device is destroyed), so make that first call before any stream capture. The call returns
 * before its kernels finish: a bounded wait that runs out inside them is returned as POX_ERR_TIMEOUT
 * by the next call of this entry point on the context (which then launches nothing) or by
 * pox_cuda_synchronize. */
int pox_cuda_tensor_gemv_noalloc(pox_cuda_ctx* ctx, const pox_tensor* t, const float* x_dev, size_t batch,
                                 float* y_dev, void* stream);
/* Operation fused into a GEMV's input (the decode step's RMSNorm before q/k/v and gate/up,
 * engine.rs:294-350, and SwiGLU before down, engine.rs:671-677). Row b of the GEMV input is
 *   POX_OP_NONE:   x[b * ld_x + k]
 *   POX_OP_RMSNORM: x[b * ld_x + k] * (1 / sqrt(sum_k x^2 / cols + eps)) * f16 norm_w[k] (norm_w may be NULL)
 *   POX_OP_SWIGLU:  g / (1 + exp(-g)) * up[b * ld_up + k] with g = x[b * ld_x + k]
 * ld_x / ld_up of 0 mean cols. norm_w and up are device pointers. */
typedef enum { POX_OP_NONE = 0, POX_OP_RMSNORM = 1, POX_OP_SWIGLU = 2 } pox_gemv_op_mode;
typedef struct {
    int mode;
    const uint16_t* norm_w;
    float eps;
    const float* up;
    uint32_t ld_x, ld_up;
} pox_gemv_op;
/* y = op(x) W^T (+ resid when resid_dev is non-NULL; resid may alias y), on device pointers,
 * asynchronous on `stream`. Tensors in the tiled layout only (INT4 with cols and group size
 * multiples of 128, INT8 with cols % 64 == 0, F16 with cols % 32 == 0); otherwise
 * POX_ERR_UNSUPPORTED. */
int pox_cuda_tensor_gemv_ex(pox_cuda_ctx* ctx, const pox_tensor* t, const float* x_dev, size_t batch, float* y_dev,
                            const pox_gemv_op* op, const float* resid_dev, void* stream);
/* quantize_int4_group (crates/paraoxidizer-quant/src/kernels.rs:26-82) on the GPU, bit-exact:
 * w_dev [numel] f32 (device) -> packed_dev [numel / 2] and scales_dev [numel / group_size * 4]
 * (device), the .pox INT4 payloads. numel must be a multiple of an even group_size.
 * Asynchronous on `stream` (NULL: the context's stream). */
int pox_cuda_quantize_int4(pox_cuda_ctx* ctx, const float* w_dev, size_t numel, size_t group_size,
                           uint8_t* packed_dev, uint8_t* scales_dev, void* stream);
/* extract_and_zero_outliers (crates/paraoxidizer-quant/src/outlier.rs:57-85) on the GPU, bit-exact:
 * the mean and the variance sum are the reference's sequential f32 sums in index order (one thread,
 * IEEE round-to-nearest adds, the square a separate multiply), std = sqrt(var_sum / n), threshold =
 * sigma * std; every element with |w - mean| > threshold (strict) goes, in ascending index order, into
 * the .pox outlier table (count:u32 | indices:u32[count] | f16 values rounded to nearest even,
 * outlier.rs:99-110) and is zeroed in w_dev (device, n floats). sigma is the policy's multiplier
 * (Conservative 4.5, Automatic 3.5, Aggressive 2.8; outlier.rs:9-35). The table goes to host memory
 * `table` (table_cap bytes); *table_len = its length, 0 where the reference returns None (no outlier
 * or n == 0). A buffer too small: nothing is modified, *table_len is set, POX_ERR_LAYOUT. n <= 2^32.
 * Synchronous; the two sums take about 4 ns per element. */
int pox_cuda_extract_outliers(pox_cuda_ctx* ctx, float* w_dev, size_t n, float sigma, uint8_t* table,
                              size_t table_cap, size_t* table_len);
/* Dequantizes a resident tensor into out_dev ([rows][cols] f32, device), bit-exact with
 * dequantize_int4_group / dequantize_int8_symmetric (kernels.rs:85-128,157-173) followed by
 * SparseOutlierTable::apply_to (outlier.rs:88-95). Asynchronous on `stream`. */
int pox_cuda_tensor_dequant(pox_cuda_ctx* ctx, const pox_tensor* t, float* out_dev, void* stream);
/* Host-output variant of pox_cuda_tensor_dequant, synchronous; out holds rows*cols floats. */
int pox_cuda_tensor_dequant_host(pox_cuda_ctx* ctx, const pox_tensor* t, float* out);

/* ---- decode step of a Llama-architecture model ------------------------------------------- */

/* ModelConfig fields the decode path uses (crates/paraoxidizer-core/src/arch.rs:96-112;
 * head_dim = hidden / heads, arch.rs:135-137). */
typedef struct {
    uint32_t hidden, intermediate, layers, heads, kv_heads, vocab;
    float rms_eps, rope_theta;
} pox_llama_config;

typedef struct pox_model pox_model;

/* A model on the context's device with a paged fp16 KV cache of kv_blocks pages of 16 tokens
 * (the page size of crates/paraoxidizer-runtime/src/paged_cache.rs:4) for up to max_batch
 * sequences of up to max_blocks_per_seq pages each. Replaces the engine state of PoxEngine
 * (engine.rs:86-104) plus its contiguous f32 KvCache (engine.rs:10-84). */
int pox_cuda_model_create(pox_cuda_ctx* ctx, const pox_llama_config* cfg, uint32_t max_batch, uint32_t kv_blocks,
                          uint32_t max_blocks_per_seq, pox_model** out);
void pox_cuda_model_destroy(pox_model* m);
/* model.embed_tokens.weight, model.norm.weight, lm_head.weight as f16 (.pox F16 payloads):
 * [vocab][hidden], [hidden], [vocab][hidden]. */
int pox_cuda_model_set_embeddings(pox_model* m, const uint16_t* embed, const uint16_t* final_norm,
                                  const uint16_t* lm_head);
/* Layer `layer`: proj[7] = q, k, v, o, gate, up, down projections (INT4 .pox tensors, optional
 * outlier tables), input_layernorm and post_attention_layernorm weights as f16 [hidden]. q/k/v and
 * gate/up are concatenated into one resident tensor each. */
int pox_cuda_model_set_layer(pox_model* m, uint32_t layer, const pox_tensor_desc* proj, const uint16_t* attn_norm,
                             const uint16_t* mlp_norm);
/* Layer `layer` from resident tensors (e.g. uploaded from device payloads): qkv = q, k, v
 * projections stacked by rows, gate_up = gate, up stacked by rows, all INT4 in the tiled layout.
 * The model takes ownership of the four tensors (freed with it). Norm weights: host f16. */
int pox_cuda_model_set_layer_tensors(pox_model* m, uint32_t layer, pox_tensor* qkv, pox_tensor* o, pox_tensor* gate_up,
                                     pox_tensor* down, const uint16_t* attn_norm, const uint16_t* mlp_norm);
/* One decode step for `batch` sequences (engine.rs:411-716 forward_token, batched): row b feeds
 * tokens[b] at positions[b], its KV pages listed in block_tables[b * max_blocks_per_seq + j]
 * (page j holds positions 16 j .. 16 j + 15; paged_cache.rs:149-162). logits [batch][vocab]
 * (non-finite -> 0, engine.rs:709-713) and the greedy next tokens (sampler.rs:55-65) are written
 * to host memory when non-NULL. Synchronous. */
int pox_cuda_model_decode(pox_model* m, uint32_t batch, const uint32_t* tokens, const uint32_t* positions,
                          const int32_t* block_tables, float* logits, uint32_t* next_tokens);
/* Prefill: `rows` tokens through the model in one pass, replacing the token-by-token prefill of
 * forward_sequence (crates/paraoxidizer-runtime/src/engine.rs:758-762). Row r feeds tokens[r] at
 * positions[r] with its sequence's pages in block_tables[r * max_blocks_per_seq ..]; rows may belong
 * to several sequences, and every row's k and v are written to the pages before any row attends, so
 * each row attends to positions 0..positions[r] of its table, rows of the same pass included (the
 * projections run as tensor-core GEMMs over the rows). logits [n_out][vocab] (this rank's slice) and
 * the greedy next tokens [n_out] of rows out_rows[0 .. n_out) (typically each sequence's last
 * prompt row) are written to host memory when non-NULL. rows <= max_batch (split longer prompts into
 * passes: later passes see the pages earlier ones wrote). Synchronous. */
int pox_cuda_model_prefill(pox_model* m, uint32_t rows, const uint32_t* tokens, const uint32_t* positions,
                           const int32_t* block_tables, uint32_t n_out, const uint32_t* out_rows, float* logits,
                           uint32_t* next_tokens);
/* Device-pointer variant, asynchronous on `stream` (NULL: the context's stream). NULL inputs keep
 * the model's current device buffers (pox_cuda_model_buffers); advance != 0 then feeds the greedy
 * tokens back and increments the positions on the device, so consecutive calls decode greedily.
 * The pages for every position a step reaches must be in the block tables already (reserve them
 * before a run of steps): a position at or beyond 16 max_blocks_per_seq or a page entry outside
 * [0, kv_blocks) is caught on the device, that part of the attention is left out, and the next
 * pox_cuda_synchronize returns POX_ERR_INVALID. */
int pox_cuda_model_decode_device(pox_model* m, uint32_t batch, const uint32_t* tokens_dev,
                                 const uint32_t* positions_dev, const int32_t* block_tables_dev, float* logits_dev,
                                 uint32_t* next_dev, int advance, void* stream);
/* enable = 1: decode steps of batch 1..4 run every layer in one persistent kernel (one CTA per SM:
 * eight warps prepare inputs, run the weight tiles and the attention items, one warp streams the
 * weights in 34 KB bulk copies ahead of them across projections and layers; grid barriers with
 * bounded waits between the projections) when the model qualifies: one GPU, head_dim 128 with 4..8
 * query heads per kv head, all projections INT4 with group size 128 and no outliers. Other steps,
 * and prefill, take one launch per projection. Default 0 (one launch per projection for every step):
 * on B200 the persistent kernel is not yet the faster of the two. No counterpart in the reference. */
int pox_cuda_model_set_persistent(pox_model* m, int enable);
/* 1 if a decode step of `batch` rows of this model runs as the persistent kernel, else 0. */
int pox_cuda_model_step_persistent(const pox_model* m, uint32_t batch);
/* Loads a batch state into the model's device buffers without running a step (host arrays:
 * tokens [batch], positions [batch], block_tables [batch][max_blocks_per_seq]); a following
 * pox_cuda_model_decode_device with NULL inputs continues from it. Synchronous. Every page up to
 * each row's position must be a block in [0, kv_blocks) (POX_ERR_INVALID otherwise; later pages may
 * be -1 = not yet allocated, as BlockTable leaves them). */
int pox_cuda_model_set_state(pox_model* m, uint32_t batch, const uint32_t* tokens, const uint32_t* positions,
                             const int32_t* block_tables);
/* The model's device buffers (any out pointer may be NULL): tokens [max_batch], positions
 * [max_batch], block tables [max_batch][max_blocks_per_seq], logits [max_batch][vocab], next
 * tokens [max_batch]. */
int pox_cuda_model_buffers(pox_model* m, uint32_t** tokens_dev, uint32_t** positions_dev, int32_t** block_tables_dev,
                           float** logits_dev, uint32_t** next_dev);

/* Paged GQA decode attention over an fp16 KV cache that already holds every position attended: the
 * attention of forward_token (crates/paraoxidizer-runtime/src/engine.rs:580-641) on the pages of
 * crates/paraoxidizer-runtime/src/paged_cache.rs:149-162 (page = position / 16, slot = position % 16),
 * exported for a kernel-level check. For batch row b and query head h (kv head h / (heads / kv_heads)):
 *   out[b][h] = sum over t <= positions[b] of p_t v_t,  p = softmax_t(q[b][h] . k_t / sqrt(head_dim))
 * with the reference's guards (non-finite max -> 0, non-finite terms -> 0, 1 / sum only when the sum
 * is > 1e-9). Device memory: q_dev [batch][heads][head_dim] f32 (already rotated), k_pages_dev and
 * v_pages_dev [num_blocks][kv_heads][16][head_dim] f16 bits (16-byte aligned), block_tables_dev
 * [batch][max_blocks_per_seq] int32, positions_dev [batch] u32 (last position attended), out_dev
 * [batch][heads][head_dim] f32. head_dim 32, 64 or 128 with at most 8 query heads per kv head (else
 * POX_ERR_UNSUPPORTED). Asynchronous on `stream` (NULL: the context's stream). A position at or
 * beyond 16 max_blocks_per_seq (that row's output is 0) or a page entry outside [0, num_blocks) (the
 * page is left out) is caught on the device, and the next pox_cuda_synchronize returns
 * POX_ERR_INVALID. The first call, and one with larger sizes, allocates the split partials: make it
 * before any stream capture. The decode step runs the same kernels with RoPE and the KV append fused. */
int pox_cuda_paged_attention(pox_cuda_ctx* ctx, const float* q_dev, const uint16_t* k_pages_dev,
                             const uint16_t* v_pages_dev, const int32_t* block_tables_dev,
                             const uint32_t* positions_dev, uint32_t batch, uint32_t heads, uint32_t kv_heads,
                             uint32_t head_dim, uint32_t num_blocks, uint32_t max_blocks_per_seq, float* out_dev,
                             void* stream);

/* ---- tensor-parallel decode across the GPUs of one node (one process and context per GPU) ----
 * The reference decodes on one device; the shard layout is the standard Megatron split, chosen so
 * that every .pox payload shards into contiguous row ranges or 128-aligned column ranges:
 *   q, k, v, gate, up, lm_head: split by rows (rank r holds heads [r nq/tp, (r+1) nq/tp), kv heads
 *     [r nkv/tp, ...), FFN rows [r I/tp, ...), vocab rows [r V/tp, ...));
 *   o, down: split by columns (K), their partial outputs summed by one allreduce each per layer;
 *   embedding and norms: replicated.
 * Rank r of tp_size is created with the whole model's configuration; the tensors given to
 * set_layer / set_layer_tensors and the lm_head given to set_embeddings are rank r's shards, and
 * logits are the rank's vocab slice [batch][vocab / tp_size]. Every rank calls every decode entry
 * point with the same batch state; the greedy tokens (first maximum over the whole vocab) are the
 * same on every rank. tp_size 1 is pox_cuda_model_create. Requires heads, kv_heads and vocab
 * divisible by tp_size and intermediate by 128 tp_size. */
int pox_cuda_model_create_tp(pox_cuda_ctx* ctx, const pox_llama_config* cfg, uint32_t max_batch, uint32_t kv_blocks,
                             uint32_t max_blocks_per_seq, uint32_t tp_rank, uint32_t tp_size, pox_model** out);

/* Allreduce / gather implementation of a tensor-parallel model. */
#define POX_COMM_NCCL 1 /* ncclAllReduce / ncclAllGather on the decode stream */
#define POX_COMM_PEER 2 /* one-shot exchange over CUDA IPC peer memory (NVLink loads, flag handshake) */

/* A fresh NCCL unique id (128 bytes), made by one rank and sent to the others. */
int pox_cuda_comm_unique_id(uint8_t id[128]);
/* Joins the NCCL communicator of the tp_size ranks; collective (every rank, same id). */
int pox_cuda_model_comm_nccl(pox_model* m, const uint8_t id[128]);
/* The CUDA IPC handle (64 bytes) of this rank's exchange buffer (flags + two data slots). */
int pox_cuda_model_comm_ipc_handle(pox_model* m, uint8_t handle[64]);
/* Opens every rank's exchange buffer: handles = tp_size x 64 bytes in rank order (this rank's own
 * entry is ignored). A waiting rank gives up after about two seconds and the step reports
 * POX_ERR_TIMEOUT. */
int pox_cuda_model_comm_peer(pox_model* m, const uint8_t* handles);
/* Selects the exchange of the decode step (POX_COMM_NCCL or POX_COMM_PEER; set up first). Every
 * rank must select the same mode. */
int pox_cuda_model_comm_mode(pox_model* m, int mode);

/* Failure-detection check of the peer exchange on this context's GPU: runs one allreduce of a
 * two-rank group whose second rank never arrives (its arrival flags are a local buffer that
 * nothing writes). Returns POX_OK when the arrival wait ran out within its limit, was reported
 * as a kernel error (POX_ERR_TIMEOUT internally, then cleared) and set the sticky abort word;
 * *wait_seconds (may be NULL) = the kernel's duration. The context stays usable. No counterpart
 * in the reference (one process, no exchanges). */
int pox_cuda_comm_check_missing_rank(pox_cuda_ctx* ctx, double* wait_seconds);

/* ---- the .pox container on the host (crates/paraoxidizer-format/src/pox.rs) --------------------- */

typedef struct pox_file pox_file;

/* One entry of the tensor index: TensorMeta (crates/paraoxidizer-core/src/tensor.rs:116-128). Offsets
 * are absolute in the file; name and sha256 (lower-case hex) stay valid while the file is open. */
typedef struct {
    const char* name;
    int dtype;              /* POX_F32 .. POX_I4; -1 for the F8E4M3 / F8E5M2 entries this backend does not serve */
    uint32_t group_size;    /* QuantGroupSize: 0 (None), 32, 64, 128 or 256 */
    uint32_t rank;          /* shape rank (first 8 dims in dims) */
    uint64_t dims[8];
    uint64_t data_offset, data_len, scale_offset, scale_len, outlier_offset, outlier_len;
    const char* sha256;
} pox_tensor_meta;

/* Replaces PoxFile::open (pox.rs:171-175, from_mmap :248-310): maps the file read-only, checks the
 * 128-byte header (magic "POX\x01", version 1) and the bounds of every section, and parses the JSON
 * metadata, tensor index, quant plan, manifest and signature. POX_ERR_FORMAT with the reference's
 * message on a malformed file, POX_ERR_INVALID when it cannot be opened. */
int pox_file_open(const char* path, pox_file** out);
/* Replaces PoxFile::from_bytes (pox.rs:177-246): the same checks on a byte buffer, which is copied. */
int pox_file_from_bytes(const uint8_t* bytes, size_t len, pox_file** out);
void pox_file_close(pox_file* f);
int pox_file_tensor_count(const pox_file* f, size_t* n);
int pox_file_tensor_meta(const pox_file* f, size_t index, pox_tensor_meta* out);
/* tensor_map lookup (pox.rs:199-202; a repeated name maps to its last entry). POX_ERR_INVALID if absent. */
int pox_file_find(const pox_file* f, const char* name, size_t* index);
/* get_tensor_data / get_scale_data / get_outlier_data (pox.rs:311-353): zero-copy slices of the file.
 * *ptr = NULL, *len = 0 where the reference returns None (unknown name, empty scale / outlier section,
 * a range past the end). */
int pox_file_tensor_data(const pox_file* f, const char* name, const uint8_t** ptr, size_t* len);
int pox_file_scale_data(const pox_file* f, const char* name, const uint8_t** ptr, size_t* len);
int pox_file_outlier_data(const pox_file* f, const char* name, const uint8_t** ptr, size_t* len);
/* metadata.model_config (ModelConfig, crates/paraoxidizer-core/src/arch.rs:96-112) as the decode
 * configuration; *tie_word_embeddings (may be NULL) = its tie_word_embeddings flag. */
int pox_file_model_config(const pox_file* f, pox_llama_config* cfg, int* tie_word_embeddings);
/* Replaces PoxFile::verify_integrity (pox.rs:356-383): SHA-256 of data || scales || outliers of every
 * tensor against its index entry; the first mismatch in index order -> POX_ERR_INTEGRITY. The tensors
 * are hashed by `threads` host threads (<= 0: one per core). */
int pox_file_verify_integrity(const pox_file* f, int threads);
/* Rank tp_rank's shard of a 2-D INT4 tensor for tensor-parallel decode, in .pox payload form: split 0 =
 * rows [r tp_rank, r (tp_rank + 1)) with r = rows / tp_size, split 1 = columns likewise (whole groups);
 * outlier entries outside the shard dropped, the rest re-indexed to the shard, order kept. With buffers
 * too small (or NULL) the sizes are stored and POX_ERR_LAYOUT returned. No counterpart in the reference
 * (one device). */
int pox_file_tensor_shard(const pox_file* f, const char* name, int split, uint32_t tp_rank, uint32_t tp_size,
                          uint8_t* data, size_t* data_len, uint8_t* scales, size_t* scale_len, uint8_t* outliers,
                          size_t* outlier_len);
/* A decode model built from a .pox file on the context's GPU: the engine's tensors (engine.rs:424-713;
 * model.embed_tokens / model.norm / lm_head F16, the seven INT4 projections of every layer with their
 * outlier tables, input / post-attention norms F16; tie_word_embeddings without lm_head uses the
 * embedding) uploaded once, as rank tp_rank of tp_size (pox_cuda_model_create_tp's split). Other dtypes
 * -> POX_ERR_UNSUPPORTED. The file may be closed afterwards. */
int pox_cuda_model_load(pox_cuda_ctx* ctx, const pox_file* f, uint32_t max_batch, uint32_t kv_blocks,
                        uint32_t max_blocks_per_seq, uint32_t tp_rank, uint32_t tp_size, pox_model** out);

#ifdef __cplusplus
}
#endif

#endif /* POX_CUDA_H */
