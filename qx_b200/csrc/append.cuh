// append.cuh — the K new cache rows of a speculative verify step.
//
// The reference verifies K candidate tokens in one pass
// (qx-runtime-v2 lib.rs:3722-3760: encode_rope_kv_batch writes the rotated
// keys and the values of positions start..start+K-1 into the cache, then
// encode_attention_batch_with_plan lets token t attend positions
// [0, start + t], kernels/v2_decode.metal:632-685). Here one CTA per (token,
// layer) writes the token's row exactly as the decode kernel writes a new row
// (same RoPE, same rounding to the cache type, so the rows are bit-identical
// to K successive decodes); the attention is then one decode launch with K
// causal entries.
#pragma once
#include "decode.cuh"

namespace qx {

struct AppendParams {
  char* k_region;
  char* v_region;
  int capacity;      // rows per (sequence, layer) of a contiguous arena
  KvPaging paging;   // or the page map of a paged one
  int layers, layer_begin, layer_count;
  int seq;     // sequence index in the arena
  int start;   // cache row of token 0
  int tokens;
  const void* k;  // [tokens][layer_count][HKV * D]
  const void* v;
  const float* k_norm;        // Qwen: RMSNorm weights of k, or null (1.0)
  const float2* rope_table;   // Qwen: [absolute position][64] (cos, sin)
  int in_dtype;
  unsigned* err;
};

template <class M, typename KT, typename VT>
__global__ void __launch_bounds__(128) qx_append_rows_kernel(const __grid_constant__ AppendParams p) {
  constexpr int D = M::D, HKV = M::HKV;
  const int t = blockIdx.x / p.layer_count, l = blockIdx.x - t * p.layer_count;
  const int row = p.start + t;
  const long long src = ((long long)t * p.layer_count + l) * HKV * D;
  const int tid = threadIdx.x;
  bool bad = false;
  pdl_wait();  // the page table and the rows may come from the previous launch
  const long long arow = kv_row(p.paging, p.capacity, p.layers, p.seq, p.layer_begin + l, row);
  KT* kdst = reinterpret_cast<KT*>(p.k_region) + arow * HKV * D;
  VT* vdst = reinterpret_cast<VT*>(p.v_region) + arow * HKV * D;
  if constexpr (!M::QWEN) {
    // rotate-half RoPE with qx's pinned sin/cos (granite_rope_pair,
    // qx-consensus-math lib.rs:199-207), as the decode kernel's new row
    for (int i = tid; i < HKV * (D / 2); i += 128) {
      const int h = i / (D / 2), pair = i - h * (D / 2);
      const float left = load_any(p.k, src + h * D + pair, p.in_dtype);
      const float right = load_any(p.k, src + h * D + pair + D / 2, p.in_dtype);
      float sn, cs, a = 0.f, b = 0.f;
      bad |= !(granite_sin_cos((uint32_t)row, pair, &sn, &cs) && granite_rotate(left, right, sn, cs, &a, &b));
      kdst[h * D + pair] = Elem<KT>::from_f32(a);
      kdst[h * D + pair + D / 2] = Elem<KT>::from_f32(b);
    }
  } else {
    // per-head RMSNorm with the reference's sequential sum of squares, then
    // rotate-half RoPE from the cos/sin table (qx-qwen-parity main.rs:1170-1210)
    __shared__ float raw[HKV * D];
    __shared__ float inv[HKV];
    for (int i = tid; i < HKV * D; i += 128) raw[i] = load_any(p.k, src + i, p.in_dtype);
    __syncthreads();
    if (tid < HKV) {
      float sum = 0.0f;
      for (int i = 0; i < D; ++i) sum = __fadd_rn(sum, __fmul_rn(raw[tid * D + i], raw[tid * D + i]));
      inv[tid] = __frcp_rn(__fsqrt_rn(__fadd_rn(__fdiv_rn(sum, (float)D), 1.0e-6f)));
    }
    __syncthreads();
    const float2* tab = p.rope_table + (long long)row * (D / 2);
    for (int i = tid; i < HKV * (D / 2); i += 128) {
      const int h = i / (D / 2), pair = i - h * (D / 2);
      const float x = raw[h * D + pair], y = raw[h * D + pair + D / 2];
      const float left = __fmul_rn(__fmul_rn(x, inv[h]), p.k_norm ? p.k_norm[pair] : 1.0f);
      const float right = __fmul_rn(__fmul_rn(y, inv[h]), p.k_norm ? p.k_norm[D / 2 + pair] : 1.0f);
      const float2 c = tab[pair];
      const float a = __fsub_rn(__fmul_rn(left, c.x), __fmul_rn(right, c.y));
      const float b = __fadd_rn(__fmul_rn(right, c.x), __fmul_rn(left, c.y));
      bad |= !(isfinite(a) && isfinite(b));
      kdst[h * D + pair] = Elem<KT>::from_f32(a);
      kdst[h * D + pair + D / 2] = Elem<KT>::from_f32(b);
    }
  }
  for (int i = tid; i < HKV * D; i += 128) vdst[i] = Elem<VT>::from_f32(load_any(p.v, src + i, p.in_dtype));
  if (bad) flag_error(p.err, QX_ERR_BIT_NONFINITE);
}

}  // namespace qx
