/*
 * qxcuda.h — C ABI of libqxcuda, the B200 (sm_100a) implementation of qx's
 * grouped-query-attention hot path: RoPE, bounded KV-cache append, split-KV
 * flash decode with a log-sum-exp combine, causal prefill, and the partial
 * (m, l, O) exchange format for a KV cache split across GPUs.
 *
 * Plain C types only: device pointers are `void*`, sizes are integers,
 * errors are status codes plus a per-context message. A Rust `qx-cuda`
 * crate binds these symbols one-to-one through an `extern "C"` block.
 *
 * Reference interfaces replaced (paths within blasrodri/qx):
 *   crates/qx-runtime/src/lib.rs:350-432     KvCache (new/len/is_empty/reset/append)
 *   crates/qx-runtime/src/lib.rs:434-442     apply_granite_rope
 *   crates/qx-runtime/src/lib.rs:444-452     granite_attention_decode
 *   crates/qx-runtime-v2/src/lib.rs:6566-6636 ExecutionPlan KV byte plan
 *   crates/qx-runtime-v2/src/lib.rs:6837-6860 GpuRuntimeBuffers::kv_key_buffer/kv_value_buffer
 *   crates/qx-runtime-v2/src/lib.rs:6863-6968 encode_attention_layer[_with_plan] (RoPE/KV + attention stage)
 *   crates/qx-runtime-v2/src/lib.rs:1793-1821 PreparedAttentionStack::encode (24-layer stack)
 *   crates/qx-runtime-v2/src/lib.rs:3265-3310 checkpoint_kv / rollback_kv / commit_kv
 *   crates/qx-runtime-v2/src/lib.rs:904-1024  Qwen attention stage (qk-norm RoPE, store KV, GQA)
 *   crates/qx-metal/src/lib.rs:14488         MetalContext::run_qwen_gqa_attention
 *   crates/qx-metal/src/lib.rs:9404-9440     DecodeGraph::finish (errors surface at wait)
 *
 * Threading: one qxc_ctx per host thread (like the reference's DecodeGraph,
 * which is not Send). Calls that take device pointers are asynchronous on the
 * context's stream; qxc_sync waits and reports device-side errors. Calls that
 * take host pointers are synchronous.
 */
#ifndef QXCUDA_H
#define QXCUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QXC_ABI_VERSION 1

typedef enum qxc_status {
  QXC_OK = 0,
  QXC_ERR_INVALID_ARG = 1,   /* shape, size, dtype or null pointer */
  QXC_ERR_POSITION = 2,      /* non-sequential or >= capacity (qx-runtime lib.rs:385-398) */
  QXC_ERR_NONFINITE = 3,     /* non-finite RoPE input/output or softmax (the reference panics) */
  QXC_ERR_CUDA = 4,
  QXC_ERR_NCCL = 5,
  QXC_ERR_TIMEOUT = 6,       /* a bounded device-side wait gave up */
  QXC_ERR_UNSUPPORTED = 7,
  QXC_ERR_OUT_OF_MEMORY = 8
} qxc_status;

typedef enum qxc_model {
  QXC_MODEL_GRANITE = 0, /* 16 q heads, 8 kv heads, head_dim 64, scale 1/64, pinned RoPE theta 1e4 */
  QXC_MODEL_QWEN3 = 1    /* 32 q heads, 4 kv heads, head_dim 128, scale 1/sqrt(128), QK-RMSNorm, RoPE theta 1e6 */
} qxc_model;

typedef enum qxc_dtype { QXC_F32 = 0, QXC_BF16 = 1, QXC_F16 = 2 } qxc_dtype;

/* Decode flags. */
#define QXC_DECODE_NO_ADVANCE 0x1 /* do not advance the cursor (caller advances after the last layer) */
#define QXC_DECODE_NATIVE_EXP 0x2 /* hardware exp2 instead of qx's pinned exp_f32 (Granite) */
#define QXC_DECODE_PINNED_EXP 0x4 /* qx's pinned exp_f32 (default for Granite; Qwen defaults to native) */

typedef struct qxc_ctx qxc_ctx;
typedef struct qxc_kv qxc_kv;

/* ---- library / context ------------------------------------------------ */
int qxc_abi_version(void);
const char* qxc_status_string(qxc_status status);
/* One context per host thread; `device` is the CUDA ordinal. */
qxc_status qxc_init(int device, qxc_ctx** out);
void qxc_destroy(qxc_ctx* ctx);
/* Use the caller's cudaStream_t (NULL restores the context's own stream). */
qxc_status qxc_set_stream(qxc_ctx* ctx, void* cuda_stream);
void* qxc_get_stream(qxc_ctx* ctx);
/* Wait for all work on the context stream, then report any device-side
 * error (non-finite values, bounded-wait timeouts) recorded since the last
 * sync. Mirrors DecodeGraph::finish (qx-metal lib.rs:9404-9440). */
qxc_status qxc_sync(qxc_ctx* ctx);
/* Message of the last failing call on this context ("" when none). */
const char* qxc_last_error(const qxc_ctx* ctx);
/* Number of kernels this context has launched so far. */
uint64_t qxc_launch_count(const qxc_ctx* ctx);
/* Cache positions per split chosen by the last decode call on this context. */
int32_t qxc_last_split(const qxc_ctx* ctx);
/* (new; host only, no device) The automatic split the decode calls choose:
 * cache rows per split for `n` sequences of attend[i] rows, `units` work
 * units per sequence (layers x kv heads, or kv-head pairs on the 16-bit
 * Granite path), `slots` CTAs resident on the GPU at once, at most
 * `max_splits` splits, `tile` rows per pipeline tile (64 on the CUDA-core
 * kernels, 128 on the tensor-core ones). 0 on a bad argument. */
int32_t qxc_auto_split(int32_t slots, const int32_t* attend, int32_t n, int32_t units, int32_t max_splits,
                       int32_t tile);

/* ---- KV cache arena ---------------------------------------------------- */
typedef struct qxc_kv_desc {
  int32_t model;       /* qxc_model */
  int32_t layers;      /* >= 1 */
  int32_t sequences;   /* >= 1, independent cursors */
  int32_t capacity;    /* slots per sequence (Granite: 1..=4096, ExecutionPlan::granite :6589) */
  int32_t key_dtype;   /* qxc_dtype of stored keys */
  int32_t value_dtype; /* qxc_dtype of stored values */
  int32_t first_position; /* absolute position of slot 0 (KV-length shards); 0 otherwise */
} qxc_kv_desc;

/* Bytes the arena holds for keys and values, without allocating
 * (ExecutionPlan::kv_key_bytes/kv_value_bytes, qx-runtime-v2 lib.rs:6640-6656). */
qxc_status qxc_kv_bytes(const qxc_kv_desc* desc, size_t* key_bytes, size_t* value_bytes);
/* One device allocation; layout per (sequence, layer):
 * keys [capacity][kv_heads][head_dim], values likewise (position-major, the
 * reference's layout). Cursors start at 0. */
qxc_status qxc_kv_create(qxc_ctx* ctx, const qxc_kv_desc* desc, qxc_kv** out);
void qxc_kv_destroy(qxc_kv* kv);
/* KvCache::len / is_empty / reset (qx-runtime lib.rs:370-380). seq < 0 in reset: all. */
qxc_status qxc_kv_len(const qxc_kv* kv, int32_t seq, int32_t* length);
qxc_status qxc_kv_reset(qxc_kv* kv, int32_t seq);
/* Set a cursor after loading a prefix with qxc_kv_write (0 <= length <= capacity). */
qxc_status qxc_kv_set_len(qxc_kv* kv, int32_t seq, int32_t length);
/* Speculative cursor (qx-runtime-v2 lib.rs:3265-3310): no KV copies. */
qxc_status qxc_kv_checkpoint(const qxc_kv* kv, int32_t seq, int32_t* sequence_len);
qxc_status qxc_kv_rollback(qxc_kv* kv, int32_t seq, int32_t sequence_len);
qxc_status qxc_kv_commit(qxc_kv* kv, int32_t seq, int32_t sequence_len, int32_t accepted_prefix);
/* Device views of one (sequence, layer) cache (kv_key_buffer / kv_value_buffer). */
qxc_status qxc_kv_key_buffer(qxc_kv* kv, int32_t seq, int32_t layer, void** device_ptr, size_t* bytes);
qxc_status qxc_kv_value_buffer(qxc_kv* kv, int32_t seq, int32_t layer, void** device_ptr, size_t* bytes);
/* Synchronous host copies of slots [begin, begin+count) of one (sequence,
 * layer); either host pointer may be NULL. */
qxc_status qxc_kv_read(qxc_kv* kv, int32_t seq, int32_t layer, int32_t begin, int32_t count,
                       void* host_keys, void* host_values);
qxc_status qxc_kv_write(qxc_kv* kv, int32_t seq, int32_t layer, int32_t begin, int32_t count,
                        const void* host_keys, const void* host_values);

/* ---- paged arenas -------------------------------------------------------- */
/* A paged arena replaces the fixed [capacity] cache per (sequence, layer) for
 * serving many sequences of uneven length (new; the reference plans one
 * fixed-size cache per layer, qx-runtime-v2 lib.rs:6566-6636). Per layer, a
 * pool of `pool_pages` pages of `page_size` rows ([page][kv_heads][head_dim]);
 * each sequence has one block table, shared by its layers, mapping its logical
 * pages to physical pages. Pages are mapped on demand, in order, by the calls
 * that write rows (decode, verify, partials, qxc_kv_write) and by
 * qxc_kv_set_len; a call the pool cannot serve fails with
 * QXC_ERR_OUT_OF_MEMORY and maps nothing. qxc_kv_reset returns a sequence's
 * pages to the pool; rollback / commit keep them for the sequence's regrowth;
 * qxc_kv_trim returns the pages past its length. desc->capacity is the
 * longest sequence. The decode, verify, partials and hash entry points read
 * rows through the table with the same results as a contiguous arena;
 * qxc_prefill and the contiguous views (qxc_kv_key_buffer / value_buffer)
 * return QXC_ERR_UNSUPPORTED. */
typedef struct qxc_kv_paging {
  int32_t page_size;  /* rows per page: a power of two in 64..=4096 (a 64-row TMA box never straddles pages) */
  int32_t pool_pages; /* physical pages per layer, shared by all sequences */
} qxc_kv_paging;

qxc_status qxc_kv_paged_bytes(const qxc_kv_desc* desc, const qxc_kv_paging* paging, size_t* key_bytes,
                              size_t* value_bytes);
qxc_status qxc_kv_create_paged(qxc_ctx* ctx, const qxc_kv_desc* desc, const qxc_kv_paging* paging, qxc_kv** out);
/* Pages mapped by `seq` (seq < 0: by all sequences) and pages free in the pool. */
qxc_status qxc_kv_page_stats(const qxc_kv* kv, int32_t seq, int32_t* mapped_pages, int32_t* free_pages);
/* Return the pages of `seq` past its current length to the pool (no-op on a
 * contiguous arena). */
qxc_status qxc_kv_trim(qxc_kv* kv, int32_t seq);
/* Device view of a paged arena's whole key (or value) page pool,
 * [layers][pool_pages][page_size][kv_heads][head_dim], e.g. to initialise
 * it; physical page p of layer l starts at row (l * pool_pages + p) * page_size. */
qxc_status qxc_kv_pool_buffer(qxc_kv* kv, int32_t key, void** device_ptr, size_t* bytes);

/* ---- decode ------------------------------------------------------------ */
/* Stream ordering. Every kernel here is launched as a programmatic
 * dependent of the stream's previous kernel. A single-sequence decode on a
 * contiguous Qwen arena may start reading cached rows before the previous
 * kernel has finished: it reads only rows that no earlier launch of this
 * context can still be writing. A caller that writes the arena with its own
 * kernel on the same stream must not launch that kernel with programmatic
 * stream serialization and trigger its dependents before the writes (plain
 * launches, copies and events need nothing). */
/* One token step for `seq_count` sequences over layers
 * [layer_begin, layer_begin + layer_count). Per (sequence, layer): RoPE on
 * q and k at `position` (Qwen: per-head RMSNorm first), append k/v into slot
 * `position`, attend over slots [0, position]. Tensors are packed
 * [seq_count][layer_count][heads * head_dim]:
 *   q, out: query heads; k, v: kv heads.
 * positions[i] must equal sequence seq_ids[i]'s length (KvCache::append
 * :382-405), else QXC_ERR_POSITION and nothing is launched. Unless
 * QXC_DECODE_NO_ADVANCE, each cursor advances by one. */
typedef struct qxc_decode_args {
  int32_t layer_begin;
  int32_t layer_count;
  int32_t seq_count;
  const int32_t* seq_ids;   /* host [seq_count]; NULL = 0..seq_count-1 */
  const int32_t* positions; /* host [seq_count] */
  const void* q;            /* device, q_dtype */
  const void* k;            /* device, in_dtype */
  const void* v;            /* device, in_dtype */
  void* out;                /* device, out_dtype */
  float* q_rot_out;         /* optional device f32 rotated query (V2 writes it back), NULL to skip */
  const float* q_norm;      /* Qwen: device [128] RMSNorm weight for q, NULL = 1.0 */
  const float* k_norm;      /* Qwen: device [128] RMSNorm weight for k, NULL = 1.0 */
  int32_t q_dtype;          /* F32 or BF16 (Qwen: BF16 or F16, the KV type) */
  int32_t in_dtype;         /* dtype of k and v inputs */
  int32_t out_dtype;        /* F32, BF16 or F16 */
  int32_t flags;            /* QXC_DECODE_* */
  int32_t split;            /* cache positions per CTA split, multiple of 64; 0 = automatic */
} qxc_decode_args;
qxc_status qxc_decode(qxc_ctx* ctx, qxc_kv* kv, const qxc_decode_args* args);
/* Same with q, k, v, out (and q_rot_out) in HOST memory, synchronous. When
 * every one of them is pinned memory the device can address (cudaHostAlloc,
 * or cudaHostRegister with cudaHostRegisterMapped) the kernels read and write
 * it in place over PCIe; otherwise the call copies in, decodes, copies out. */
qxc_status qxc_decode_host(qxc_ctx* ctx, qxc_kv* kv, const qxc_decode_args* args);

/* granite_attention_decode (qx-runtime lib.rs:444-452): host arrays
 * q[1024], k[512], v[512] -> out[1024] on sequence 0, layer 0 of a Granite
 * arena. Synchronous; QXC_ERR_POSITION when position != length. */
qxc_status qxc_granite_attention_decode(qxc_ctx* ctx, qxc_kv* kv, const float* q, const float* k,
                                        const float* v, int32_t position, float* out);
/* apply_granite_rope (qx-runtime lib.rs:434-442) in place on host arrays
 * q[1024], k[512], computed on the device with qx's pinned sin/cos. */
qxc_status qxc_apply_granite_rope(qxc_ctx* ctx, float* q, float* k, int32_t position);

/* ---- speculative verify (K candidate tokens of one sequence) -------------- */
/* Replaces the reference's batched verifier attention stage:
 * GpuRuntimeBuffers encode_rope_kv_batch + encode_attention_batch_with_plan
 * (qx-runtime-v2 lib.rs:3722-3760; qx-metal lib.rs:8105-8260). Appends the
 * RoPE'd keys and the values of positions start..start+tokens-1 (start must
 * equal the sequence's length, start+tokens <= capacity, else
 * QXC_ERR_POSITION), then token t attends positions [0, start+t]: the same
 * rows and the same outputs as `tokens` successive qxc_decode calls. The
 * length advances by `tokens` (unless QXC_DECODE_NO_ADVANCE); take a
 * qxc_kv_checkpoint before and qxc_kv_commit the accepted prefix after.
 * Layouts: q/out [tokens][layer_count][Hq*D], k/v [tokens][layer_count][Hkv*D],
 * device pointers; asynchronous on the context's stream. */
typedef struct {
  int32_t seq;
  int32_t layer_begin;
  int32_t layer_count;
  int32_t start;
  int32_t tokens;
  const void* q;
  const void* k;
  const void* v;
  void* out;
  const float* q_norm; /* Qwen RMSNorm weights [128] (null: 1.0) */
  const float* k_norm;
  int32_t q_dtype;
  int32_t in_dtype;
  int32_t out_dtype;
  int32_t flags;
  int32_t split; /* 0: automatic */
} qxc_verify_args;

/* Granite, 2 to 4 candidates: every cache tile is read once and scored
 * against all candidates' queries (one work item per layer, kv head and
 * split). QXC_VERIFY_PER_TOKEN in flags forces one causal decode entry per
 * candidate instead (each reads the cache: the layout Qwen and longer
 * drafts use). */
#define QXC_VERIFY_PER_TOKEN 0x8
qxc_status qxc_decode_verify(qxc_ctx* ctx, qxc_kv* kv, const qxc_verify_args* args);

/* ---- Q4 projections around attention (Granite layer) --------------------- */
/* A Q4 matrix in the reference's row-major layout with group 32
 * (qx-quant QuantizedTensor, layout RowMajor): per row and group, an FP16
 * scale and 16 bytes of codes, low nibble first; value = (code - 7) * scale. */
typedef struct {
  int32_t rows;
  int32_t cols;            /* a multiple of 32, at most 4096 */
  const uint8_t* codes;    /* device [rows][cols/32][16] */
  const uint16_t* scales;  /* device [rows][cols/32] FP16 bit patterns */
} qxc_q4_matrix;

/* y = W x (QuantizedTensor::mat_vec_simd32, qx-quant lib.rs:892-933), or
 * with rms_weight != NULL y = W (cpu_rms_norm_simd(x, rms_weight),
 * qx-runtime-v2 lib.rs:4924-4946; then cols must be 1024). Bit-identical
 * to the reference's CPU routines. Device pointers, asynchronous. */
qxc_status qxc_q4_mat_vec(qxc_ctx* ctx, const qxc_q4_matrix* w, const float* x, const float* rms_weight,
                          float* y);

/* The attention sub-layer of a Granite layer with Q4 weights, for one token
 * (GpuRuntimeBuffers::encode_attention_layer, qx-runtime-v2 lib.rs:6916-6994;
 * CPU twin CpuQ4Reference::step :4680-4706): RMSNorm(hidden_in, input_norm)
 * -> Q4 q/k/v projections -> RoPE, KV append at `position` and GQA attention
 * (qxc_decode) -> Q4 o-projection -> hidden_out = fma(0.22, o, hidden_in).
 * Same position rules as qxc_decode. Device pointers, asynchronous. */
typedef struct {
  int32_t seq;
  int32_t layer;
  int32_t position;
  const float* hidden_in;   /* [1024] */
  float* hidden_out;        /* [1024] */
  const float* input_norm;  /* [1024] */
  qxc_q4_matrix q_proj;     /* 1024 x 1024 */
  qxc_q4_matrix k_proj;     /* 512 x 1024 */
  qxc_q4_matrix v_proj;     /* 512 x 1024 */
  qxc_q4_matrix o_proj;     /* 1024 x 1024 */
  float* attention_out;     /* optional [1024]: attention before the o-projection */
  int32_t flags;
  int32_t split;
} qxc_layer_args;

qxc_status qxc_attention_layer(qxc_ctx* ctx, qxc_kv* kv, const qxc_layer_args* args);

/* The attention sub-layers of `layer_count` consecutive layers for one token
 * (PreparedAttentionStack::encode, qx-runtime-v2 lib.rs:1793-1821, which
 * runs encode_attention_layer :6916-6994 for every layer, the hidden state
 * passed from each layer to the next): for each layer in order,
 * hidden = fma(0.22, o_proj(attention(RoPE(q, k, v of
 * RMSNorm(hidden)))), hidden), appending the new token at `position` to every
 * layer's cache. hidden_out receives the last layer's output; the
 * intermediate states stay in the context. Same arithmetic and position
 * rules as qxc_attention_layer. An fp32 contiguous arena on a GPU of at
 * least 128 SMs with 16-byte aligned Q4 rows runs every layer in one
 * persistent cooperative launch (up to 32 layers per launch), its KV stream
 * overlapping the dependent steps; other arenas run qxc_attention_layer per
 * layer. `layers` is a host array of layer_count weight sets (device
 * pointers). The cursor advances by one unless QXC_DECODE_NO_ADVANCE.
 * split: cached rows per attention item (a multiple of 64, at most 256, at
 * most 16 items per kv head), or 0 for the library's choice. */
typedef struct {
  const float* input_norm;  /* [1024] */
  qxc_q4_matrix q_proj;     /* 1024 x 1024 */
  qxc_q4_matrix k_proj;     /* 512 x 1024 */
  qxc_q4_matrix v_proj;     /* 512 x 1024 */
  qxc_q4_matrix o_proj;     /* 1024 x 1024 */
} qxc_layer_weights;

typedef struct {
  int32_t seq;
  int32_t layer_begin;
  int32_t layer_count;
  int32_t position;
  const float* hidden_in;   /* [1024] */
  float* hidden_out;        /* [1024] */
  const qxc_layer_weights* layers;  /* host [layer_count] */
  int32_t flags;
  int32_t split;
} qxc_stack_args;

qxc_status qxc_attention_stack(qxc_ctx* ctx, qxc_kv* kv, const qxc_stack_args* args);

/* ---- commitments of KV slots and residual checkpoints (BLAKE3) ----------- */
/* Replaces the reference's verification-hash stage
 * (GpuDecodeGraph::encode_verification_hashes, qx-metal lib.rs:9247-9330,
 * kernels/verification_hash.metal; called per token at qx-runtime-v2
 * lib.rs:2215 and :2440). For token `token` of `seq`, position p in
 * 0..layers (the arena's layer count) writes 64 bytes at digests + 64 p:
 *   [0, 32)  state_hash_v1 of residual snapshot p (residuals + p * stride) when
 *            p == 0, (p % checkpoint_interval) == 0 or p == layers; else zeros
 *   [32, 64) kv_leaf_hash_v1(p - 1, token, key row, value row) read from the
 *            arena; zeros at p == 0
 * (qx-commit state.rs:213-257, :334-368). residual_stride is a power-of-two
 * number of 256-byte chunks, at most 16; the arena's rows must be 1 to 8
 * chunks (every arena type is); token < the sequence's length, else
 * QXC_ERR_POSITION. residuals 16-byte aligned. Device pointers, asynchronous. */
typedef struct {
  int32_t seq;
  int32_t token;
  const void* residuals;   /* (layers + 1) * residual_stride bytes */
  int64_t residual_stride; /* bytes */
  int32_t checkpoint_interval; /* 1..layers */
  uint8_t* digests;        /* (layers + 1) * 64 bytes */
} qxc_verification_hash_args;

qxc_status qxc_verification_hashes(qxc_ctx* ctx, qxc_kv* kv, const qxc_verification_hash_args* args);

/* kv_leaf_hash_v1(layer, token, key row, value row) of every slot of
 * [layer_begin, +layer_count) x [token_begin, +token_count) of `seq`, into
 * digests[layer_count][token_count][32] (device): the commitments of a whole
 * prefill or accepted speculative prefix in one launch. Rows must lie below
 * the sequence's length (else QXC_ERR_POSITION). flags picks the kernel
 * layout (QXC_HASH_*; 0 chooses by range size; the digests are the same).
 * Asynchronous. */
#define QXC_HASH_AUTO 0
#define QXC_HASH_PER_CHUNK 1 /* a lane per 256-byte chunk: lowest latency */
#define QXC_HASH_PER_SLOT 2  /* a lane per slot: highest throughput on large ranges */
qxc_status qxc_kv_slot_hashes(qxc_ctx* ctx, qxc_kv* kv, int32_t seq, int32_t layer_begin, int32_t layer_count,
                              int32_t token_begin, int32_t token_count, uint8_t* digests, int32_t flags);

/* Measurement helper: BLAKE3 block compressions per second on this device
 * with no memory traffic (every SM's integer pipes busy) — the ceiling the
 * hash kernels are compared against. Synchronous; about 10 ms. */
qxc_status qxc_blake3_compress_rate(qxc_ctx* ctx, double* compressions_per_second);

/* Consensus-math conformance: for each of n inputs x, out[4i..4i+3] = the
 * bits of the device's pinned exp_f32(x), rsqrt_f32(x) and the (sin, cos) of
 * granite_rope_sin_cos((uint32)x, i % 32), quiet NaN 0x7fc00000 where the
 * function has no value. Host pointers; synchronous. Replaces
 * MetalContext::run_consensus_math_conformance (qx-metal/src/lib.rs:9622-9690,
 * kernel kernels/consensus_math.metal:102-112); its test compares these bits
 * with the CPU functions (qx-metal/src/lib.rs:15488-15511). */
qxc_status qxc_consensus_math_conformance(qxc_ctx* ctx, const float* inputs, int32_t n, uint32_t* out);

/* ---- causal prefill ------------------------------------------------------ */
/* Prompt prefill of `length` tokens into an EMPTY (sequence, layer) of a
 * Granite arena (cursor must be 0): RoPE on q and k at positions
 * 0..length-1, all rows written to the cache, causal attention with fp32
 * accumulation on tcgen05 tensor cores. q:[L][16][64], k,v:[L][8][64]
 * (BF16), out:[L][16][64] (F32 or BF16). The cursor of `seq` becomes
 * `length` (unless QXC_DECODE_NO_ADVANCE). Requires bf16 KV. */
typedef struct qxc_prefill_args {
  int32_t seq;
  int32_t layer;
  int32_t length;
  const void* q;
  const void* k;
  const void* v;
  void* out;
  int32_t in_dtype;  /* BF16 */
  int32_t out_dtype; /* F32 or BF16 */
  int32_t flags;
} qxc_prefill_args;
qxc_status qxc_prefill(qxc_ctx* ctx, qxc_kv* kv, const qxc_prefill_args* args);

/* ---- KV-length split across GPUs --------------------------------------- */
/* Partial attention of one (sequence, layer) over this arena's slots
 * [first_position, first_position + length): per query head the triple
 * (m, l, O[head_dim]) with O unnormalised relative to m, written as f32
 * [q_heads][head_dim + 2] = {O..., m, l}. When `append` is non-zero this
 * shard owns the new token: RoPE at absolute `position`, append into slot
 * position - first_position, and include it. q/k/v as in qxc_decode for
 * one sequence and one layer. */
typedef struct qxc_partial_args {
  int32_t seq;
  int32_t layer;
  int32_t position; /* absolute position of the new token (RoPE angle) */
  int32_t append;   /* 1 on the shard that owns `position` */
  const void* q;
  const void* k;
  const void* v;
  const float* q_norm;
  const float* k_norm;
  float* partials;  /* device [q_heads][head_dim + 2] */
  int32_t q_dtype;
  int32_t in_dtype;
  int32_t flags;
  int32_t split;
} qxc_partial_args;
qxc_status qxc_decode_partials(qxc_ctx* ctx, qxc_kv* kv, const qxc_partial_args* args);
/* Exchange + merge over NVLink in one kernel, replacing the all-gather of the
 * partials and qxc_lse_merge when every rank's GPU can address every other's
 * memory (one node). A peer group is each rank's exchange area (about 540 KB
 * at 8 ranks); every rank creates one, exports its handle, and attaches every
 * other rank's, then each step calls qxc_exchange_merge with this rank's
 * partials from qxc_decode_partials. The kernel stores the partials into every
 * rank's area with peer stores, each value paired with the step's tag in one
 * 8-byte store (no memory fence), waits until every rank's values of its query
 * head carry the tag (bounded: QXC_ERR_TIMEOUT at qxc_sync) and merges in
 * rank order. A timed-out exchange leaves the group failed for good: every
 * later exchange on it (this call or qxc_decode_exchange) returns
 * QXC_ERR_TIMEOUT, at the call once the failure has been recorded, else at
 * qxc_sync without pushing or merging anything; destroy and re-create the
 * groups on every rank to go on. The merged output: the
 * output equals qxc_lse_merge over the gathered partials, bit for bit, on
 * every rank. Every rank must issue the same sequence of exchange calls. */
#define QXC_PEER_HANDLE_BYTES 64
typedef struct qxc_peer_group qxc_peer_group;
qxc_status qxc_peer_group_create(qxc_ctx* ctx, int32_t rank, int32_t world, qxc_peer_group** out);
void qxc_peer_group_destroy(qxc_peer_group* group);
/* The CUDA IPC handle of this rank's area (QXC_PEER_HANDLE_BYTES bytes), for
 * the other processes' qxc_peer_group_open. */
qxc_status qxc_peer_group_handle(const qxc_peer_group* group, void* handle);
qxc_status qxc_peer_group_open(qxc_peer_group* group, int32_t peer, const void* handle);
/* One process driving several GPUs: attach another group's area directly
 * (qxc_peer_group_base of that group); enables peer access when needed. */
qxc_status qxc_peer_group_base(const qxc_peer_group* group, void** base);
qxc_status qxc_peer_group_set_peer(qxc_peer_group* group, int32_t peer, void* base);
qxc_status qxc_exchange_merge(qxc_ctx* ctx, qxc_peer_group* group, int32_t model, const float* partials, void* out,
                              int32_t out_dtype);
/* qxc_decode_partials and qxc_exchange_merge in one pass, with the exchange
 * fused into the split merge: the kernel that combines this rank's KV splits
 * stores the combined partial of each (query head, 32 dims) into every rank's
 * area and merges all ranks' into out [q_heads][head_dim] (out_dtype), so no
 * separate exchange launch runs. args->partials is not used. Same output as
 * qxc_decode_partials + qxc_exchange_merge, bit for bit, when the range has
 * one split or more than 8 (with 2 to 8, qxc_decode_partials combines them
 * inside the decode kernel, in another order: equal within fp32 rounding).
 * Every rank must call it for the same steps, and not mix it with
 * qxc_exchange_merge on one group. */
qxc_status qxc_decode_exchange(qxc_ctx* ctx, qxc_kv* kv, const qxc_partial_args* args, qxc_peer_group* group,
                               void* out, int32_t out_dtype);
/* Log-sum-exp merge of n_parts partial sets [n_parts][q_heads][head_dim+2]
 * (device) into out [q_heads][head_dim] (device, out_dtype):
 * M = max m_i, O = sum e^(m_i-M) O_i / sum e^(m_i-M) l_i. */
qxc_status qxc_lse_merge(qxc_ctx* ctx, int32_t model, int32_t n_parts, const float* partials, void* out,
                         int32_t out_dtype);

/* ---- allocation-free decode ----------------------------------------------
 * No counterpart in the reference (qx's Metal path has no such entry point).
 * For callers that must not let a library allocate device memory: a host
 * runtime that sizes one arena up front and forbids allocation afterwards,
 * or code whose device memory comes from its own pool. One Granite decode
 * step (RoPE, append into slot `position`, attention over slots
 * [0, position]) on one layer's cache given as plain device pointers, with
 * the split-KV scratch taken from a 128 KiB static device array inside the
 * library instead of cudaMalloc. No context or arena is needed.
 *   - The first call on each device (with that device current) does a
 *     one-time set-up; make it before any stream capture on that device.
 *   - Every call on a device shares the one static array: calls whose
 *     kernels can overlap on the GPU race; order them on one stream.
 *   - A request whose split-KV partials exceed the array returns
 *     QXC_ERR_INVALID_ARG (use a larger `split`).
 * Asynchronous on `cuda_stream`; `message` (may be NULL) receives the
 * reason of a rejected call. */
typedef struct qxc_static_decode_args {
  void* key_cache;        /* device [capacity][8][64], key_dtype */
  void* value_cache;      /* device [capacity][8][64], value_dtype */
  int32_t capacity;       /* slots, 1..=4096 */
  int32_t key_dtype;      /* F32/F32, F32/F16, F16/F32, F16/F16 or BF16/BF16 */
  int32_t value_dtype;
  int32_t position;       /* slot of the new token; slots [0, position) hold the prefix */
  const void* q;          /* device [16][64], q_dtype */
  const void* k;          /* device [8][64], in_dtype */
  const void* v;          /* device [8][64], in_dtype */
  void* out;              /* device [16][64], out_dtype */
  int32_t q_dtype;
  int32_t in_dtype;
  int32_t out_dtype;
  int32_t flags;          /* QXC_DECODE_NATIVE_EXP to use hardware exp2 */
  int32_t split;          /* cache positions per split, multiple of 64; 0 = automatic */
  unsigned* device_error; /* optional device word set non-zero on a device-side error */
} qxc_static_decode_args;
qxc_status qxc_granite_decode_static_scratch(const qxc_static_decode_args* args, void* cuda_stream, char* message,
                                             size_t message_len);

#ifdef __cplusplus
}
#endif
#endif /* QXCUDA_H */
