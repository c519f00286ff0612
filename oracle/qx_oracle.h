/*
 * qx_oracle.h — CPU restatement of qx's grouped-query-attention path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the parity checker for the CUDA
 * implementation in qx_b200/. Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / reference arm of bench.py may load it. The product path
 * never links, loads or calls it.
 *
 * Every function restates the reference algorithm in plain C with the same
 * constants and the same operation order. Citations are to files of the
 * reference project (blasrodri/qx):
 *   crates/qx-consensus-math/src/lib.rs   pinned exp / rsqrt / sin-cos / RoPE
 *   crates/qx-runtime/src/lib.rs          KvCache, rotate_heads, decode
 *   tools/qx-qwen-parity/src/main.rs      Qwen QK-norm RoPE and GQA oracle
 *
 * Built with -O2 -ffp-contract=off and no fast-math so that every multiply
 * and add rounds separately, exactly as the Rust source (which never
 * contracts) does. fmaf() is the IEEE fused multiply-add, like libm::fmaf.
 */
#ifndef QX_ORACLE_H
#define QX_ORACLE_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes; numerically equal to the product's qxc_status values. */
enum {
  QXO_OK = 0,
  QXO_ERR_INVALID_ARG = 1,
  QXO_ERR_POSITION = 2,
  QXO_ERR_NONFINITE = 3
};

/* Storage element types for KV caches and 16-bit tensors. */
enum { QXO_F32 = 0, QXO_BF16 = 1, QXO_F16 = 2 };

/* ---- qx-consensus-math (crates/qx-consensus-math/src/lib.rs) ---- */
int qxo_exp_f32(float x, float* out);                         /* :70-110  */
int qxo_rsqrt_f32(float x, float* out);                       /* :114-128 */
int qxo_sin_cos_f32(float angle, float* s, float* c);         /* :148-189 */
int qxo_granite_rope_sin_cos(uint32_t position, uint32_t pair,
                             float* s, float* c);             /* :192-195 */
int qxo_granite_rope_pair(uint32_t position, uint32_t pair, float left,
                          float right, float* first,
                          float* second);                     /* :199-207 */
uint32_t qxo_granite_inverse_frequency_bits(uint32_t pair);   /* :28-61   */
float qxo_reduce_simd32(const float* lanes);  /* qx-runtime lib.rs:2298-2306 */

/* Error-bound sweeps from the consensus-math unit tests (:217-254,:298-311). */
float qxo_exp_worst_relative_error(void);
float qxo_rsqrt_worst_relative_error(void);
float qxo_rope_worst_absolute_error(void);

/* ---- element conversions (IEEE round-to-nearest-even) ---- */
uint16_t qxo_f32_to_bf16(float f);
float qxo_bf16_to_f32(uint16_t b);
uint16_t qxo_f32_to_f16(float f);
float qxo_f16_to_f32(uint16_t h);

/* ---- Granite (qx-runtime) ---- */
/* rotate_heads (:2439-2453) on `heads` heads of 64 values, in place.
 * Returns QXO_ERR_NONFINITE where the reference panics. */
int qxo_rotate_heads(float* values, int heads, uint32_t position);
/* cpu_rotate_heads (qx-runtime-v2 lib.rs:4957-4970), the V2 CPU twin's
 * RoPE: the same sin/cos, each product and sum rounded separately (no fma). */
int qxo_cpu_rotate_heads(float* values, int heads, uint32_t position);

/* granite_attention_decode[_simd] (:444-552) on one KvCache.
 * keys/values: [max_context][8][64] of key_dtype / value_dtype elements
 * (F32 reproduces the reference exactly; BF16/F16 store the rotated key and
 * the value rounded to that type and read them back widened).
 * *length is the KvCache cursor; it advances by one on success.
 * hierarchical=1 selects the 256-thread / 16x32-chunk variant, which the
 * reference only supports up to 512 cached positions. */
int qxo_granite_attention_decode(const float* query, const float* key,
                                 const float* value, int position,
                                 void* keys, void* values, int key_dtype,
                                 int value_dtype, int* length,
                                 int max_context, int hierarchical,
                                 float* output);

/* Many independent caches (one per sequence x layer) in one call; OpenMP
 * over units when threads > 1. statuses[u] receives each unit's status. */
int qxo_granite_attention_decode_many(
    int n_units, const float* const* query, const float* const* key,
    const float* const* value, const int* positions, void* const* keys,
    void* const* values, int key_dtype, int value_dtype, int* lengths,
    int max_context, int hierarchical, float* const* output, int threads,
    int* statuses);

/* Causal prefill defined as the decode oracle iterated over positions
 * 0..L-1 on an empty cache (the reference's prompt prefill is sequential
 * one-token decode). q:[L][16][64], k,v:[L][8][64] in in_dtype (BF16 or
 * F32); keys/values receive the cache in kv_dtype; out:[L][16][64] f32. */
int qxo_granite_prefill(const void* q, const void* k, const void* v,
                        int in_dtype, int length, void* keys, void* values,
                        int kv_dtype, float* output, int threads);

/* ---- Qwen3 (tools/qx-qwen-parity/src/main.rs) ---- */
/* cpu_qk_norm_rope (:1170-1210) with dtype selecting the 16-bit format
 * (F16 as the reference is written, BF16 for bf16 KV). */
void qxo_qwen_qk_norm_rope(const uint16_t* query, const uint16_t* key,
                           const float* query_norm, const float* key_norm,
                           uint32_t position, int dtype, uint16_t* query_out,
                           uint16_t* key_out);
/* The cos/sin values the reference evaluates for one position (64 pairs). */
void qxo_qwen_rope_table(uint32_t position, float* cosine, float* sine);
/* cpu_gqa_attention (:1218-1258): output before the final 16-bit rounding
 * in out_f32, and rounded to dtype in out_bits when out_bits != NULL. */
void qxo_qwen_gqa_attention(const uint16_t* query, const uint16_t* key_cache,
                            const uint16_t* value_cache, int context,
                            int dtype, float* out_f32, uint16_t* out_bits,
                            int threads);

/* ---- the attention half of a Granite layer with Q4 projections
 *      (qx-runtime-v2 CpuQ4Reference::step, lib.rs:4680-4706) ---- */
/* cpu_rms_norm_simd (qx-runtime-v2 lib.rs:4924-4946): HIDDEN = 1024,
 * 256 fma partials, two reduce_simd32 levels, consensus rsqrt, then
 * (x * scale) * weight. Returns 0 when the RMS is not positive finite. */
int qxo_rms_norm_simd(const float* input, const float* weight, float* out);
/* QuantizedTensor::quantize for Q4, group 32, row-major layout
 * (qx-quant lib.rs:313-360 and pack_scaled :1383-1404): scales[row][group]
 * as FP16 bits, codes[row][group][16 bytes], low nibble first. */
void qxo_q4_quantize(const float* src, int rows, int cols, uint8_t* codes, uint16_t* scales);
/* QuantizedTensor::mat_vec_simd32 for that layout (qx-quant lib.rs:892-933,
 * decode_scaled :1472-1485): column c accumulates into lane c % 32 by fma,
 * then the (16, 8, 4, 2, 1) lane tree. */
void qxo_q4_mat_vec_simd32(const uint8_t* codes, const uint16_t* scales, int rows, int cols,
                           const float* input, float* out);
/* One attention sub-layer: normalized = rms_norm(hidden, input_norm);
 * q/k/v = Q4 mat-vecs; RoPE; attention at `position` on `cache`;
 * out[i] = fma(RESIDUAL_MULTIPLIER = 0.22, o_proj(attention)[i], hidden[i]).
 * cpu_twin = 0 follows the V2 GPU stage (qx-runtime-v2 lib.rs:6916-6994:
 * the Metal fma RoPE, i.e. rotate_heads, and V1's plain attention);
 * cpu_twin = 1 follows the V2 CPU twin CpuQ4Reference::step exactly
 * (lib.rs:4686-4706: cpu_rotate_heads, CpuQ4Cache::attend, <= 512
 * positions). Weights as qxo_q4_quantize writes them; attention_out
 * (optional, [1024]) receives the attention output. Returns QXO_OK or
 * the decode's error status. */
int qxo_granite_attention_layer(const float* hidden, const float* input_norm,
                                const uint8_t* q_codes, const uint16_t* q_scales,
                                const uint8_t* k_codes, const uint16_t* k_scales,
                                const uint8_t* v_codes, const uint16_t* v_scales,
                                const uint8_t* o_codes, const uint16_t* o_scales,
                                int position, float* keys, float* values, int* length,
                                int capacity, int cpu_twin, float* out, float* attention_out);

/* ---- KV-slot commitments (qx-commit state.rs:213-251 and :334-368) ---- */
/* BLAKE3 (the blake3 crate 1.8.7, Cargo.lock:656-657; the published
 * algorithm) of an input of at most 1024 bytes, i.e. one chunk: every
 * commitment input on this path fits one. Returns 0 for longer inputs. */
int qxo_blake3_single_chunk(const uint8_t* input, size_t len, uint8_t out[32]);
/* chunk_tree_hash (state.rs:213-251): 256-byte leaves hashed as
 * hash_domain(leaf_domain, [u32 index LE, chunk]), padded with the empty
 * leaf hash_domain(QX:MERKLE:EMPTY:V1, [tree_domain]) to a power of two,
 * reduced by BLAKE3(left || right). Returns 0 on empty input. */
int qxo_chunk_tree_hash(const uint8_t* bytes, size_t len, const char* leaf_domain, const char* tree_domain,
                        uint8_t out[32]);
/* kv_leaf_hash_v1 (state.rs:334-368): the K and V chunk-tree roots bound to
 * (layer, token) under QX:KV:V1. */
int qxo_kv_leaf_hash(uint16_t layer, uint32_t token, const uint8_t* key_bytes, size_t key_len,
                     const uint8_t* value_bytes, size_t value_len, uint8_t out[32]);

#ifdef __cplusplus
}
#endif
#endif
