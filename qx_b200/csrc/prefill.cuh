// prefill.cuh — causal GQA prompt prefill for Granite (bf16 in, f32 acc).
//
// The reference has no dense prefill: a prompt is fed one token at a time
// through granite_attention_decode (qx-runtime-v2 lib.rs:4152-4187 loops
// `step`). Running the decode at positions 0..L-1 is exactly causal
// attention over a cache whose rows are the RoPE'd keys, so prefill here is
//   1. qx_prefill_rope_kv_kernel: RoPE (qx's pinned sin/cos) on every key
//      row, written as bf16 into the cache, values copied, cursor -> L;
//   2. causal attention of the RoPE'd queries against the cache.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "qx_math.cuh"
#include "qx_ptx.cuh"

namespace qx {

struct PrefillParams {
  const __nv_bfloat16* q;  // [L][16][64]
  const __nv_bfloat16* k;  // [L][8][64]
  const __nv_bfloat16* v;  // [L][8][64]
  __nv_bfloat16* k_cache;  // [capacity][8][64]
  __nv_bfloat16* v_cache;
  void* out;  // [L][16][64]
  int out_dtype;
  int length;
  int pinned_exp;
  unsigned* err;
};

// One CTA per position: 8 key heads x 32 pairs rotated, values copied.
__global__ void __launch_bounds__(256) qx_prefill_rope_kv_kernel(const PrefillParams p) {
  const int pos = blockIdx.x;
  const int head = threadIdx.x >> 5, pair = threadIdx.x & 31;
  const long long base = ((long long)pos * 8 + head) * 64;
  const float left = __bfloat162float(p.k[base + pair]);
  const float right = __bfloat162float(p.k[base + pair + 32]);
  float sn, cs, a = 0.f, b = 0.f;
  const bool ok = granite_sin_cos((uint32_t)pos, pair, &sn, &cs) && granite_rotate(left, right, sn, cs, &a, &b);
  if (!ok) flag_error(p.err, QX_ERR_BIT_NONFINITE);
  p.k_cache[base + pair] = __float2bfloat16_rn(a);
  p.k_cache[base + pair + 32] = __float2bfloat16_rn(b);
  p.v_cache[base + pair] = p.v[base + pair];
  p.v_cache[base + pair + 32] = p.v[base + pair + 32];
}

// Causal attention on CUDA cores: one CTA per (64-query tile, query head);
// one thread per query row with an online softmax over 64-key tiles.
__global__ void __launch_bounds__(64) qx_prefill_attn_simt_kernel(const PrefillParams p) {
  __shared__ float ks[64][65];
  __shared__ float vs[64][65];
  const int tile = blockIdx.x, qh = blockIdx.y, kvh = qh >> 1;
  const int row = tile * 64 + threadIdx.x;
  const bool live = row < p.length;
  const bool pinned = p.pinned_exp != 0;
  float q[64];
  if (live) {
    const long long qb = ((long long)row * 16 + qh) * 64;
    for (int pr = 0; pr < 32; ++pr) {
      float sn, cs, a = 0.f, b = 0.f;
      const float l = __bfloat162float(p.q[qb + pr]), r = __bfloat162float(p.q[qb + pr + 32]);
      if (!(granite_sin_cos((uint32_t)row, pr, &sn, &cs) && granite_rotate(l, r, sn, cs, &a, &b)))
        flag_error(p.err, QX_ERR_BIT_NONFINITE);
      q[pr] = a;
      q[pr + 32] = b;
    }
  }
  float acc[64];
  for (int d = 0; d < 64; ++d) acc[d] = 0.f;
  float m = -INFINITY, l = 0.f;
  const int last_key = min(p.length, (tile + 1) * 64);
  for (int k0 = 0; k0 < last_key; k0 += 64) {
    __syncthreads();
    for (int i = threadIdx.x; i < 64 * 64; i += 64) {
      const int r = i >> 6, d = i & 63;
      const int key = k0 + r;
      const long long off = ((long long)key * 8 + kvh) * 64 + d;
      ks[r][d] = key < p.length ? __bfloat162float(p.k_cache[off]) : 0.f;
      vs[r][d] = key < p.length ? __bfloat162float(p.v_cache[off]) : 0.f;
    }
    __syncthreads();
    if (!live) continue;
    const int nk = min(64, row - k0 + 1);  // causal: keys <= row
    for (int j = 0; j < nk; ++j) {
      float s = 0.f;
#pragma unroll 16
      for (int d = 0; d < 64; ++d) s = fmaf(q[d], ks[j][d], s);
      s *= 0.015625f;
      const float mn = fmaxf(m, s);
      const float alpha = m == -INFINITY ? 0.f : softmax_exp(m - mn, pinned);
      const float pw = softmax_exp(s - mn, pinned);
      l = fmaf(l, alpha, pw);
#pragma unroll 16
      for (int d = 0; d < 64; ++d) acc[d] = fmaf(pw, vs[j][d], acc[d] * alpha);
      m = mn;
    }
  }
  if (!live) return;
  const long long ob = ((long long)row * 16 + qh) * 64;
  const float inv = 1.0f / l;
  for (int d = 0; d < 64; ++d) store_any(p.out, ob + d, p.out_dtype, acc[d] * inv);
}

inline cudaError_t launch_prefill(const PrefillParams& p, cudaStream_t stream, int* launches) {
  qx_prefill_rope_kv_kernel<<<p.length, 256, 0, stream>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  dim3 grid((p.length + 63) / 64, 16);
  qx_prefill_attn_simt_kernel<<<grid, 64, 0, stream>>>(p);
  *launches = 2;
  return cudaGetLastError();
}

}  // namespace qx
