// prefill.cuh — causal GQA prompt prefill for Granite on tcgen05 tensor
// cores (bf16 operands, f32 accumulation in TMEM).
//
// The reference has no dense prefill: a prompt is fed one token at a time
// through granite_attention_decode (qx-runtime-v2 lib.rs:4152-4187 loops
// `step`). Running the decode at positions 0..L-1 is exactly causal
// attention over a cache of RoPE'd keys, so prefill here is
//   1. qx_prefill_rope_kernel: one CTA per position evaluates qx's pinned
//      sin/cos for the 32 rotation pairs once and applies them to all 16
//      query and 8 key heads (same operations as rotate_heads, qx-runtime
//      lib.rs:2439-2453); keys go into the cache as bf16 (bit-identical to
//      the oracle), values are copied, rotated queries go to a bf16 scratch;
//   2. qx_prefill_attn_tc_kernel: one CTA per (64-position query block,
//      chunk of at most kc of its causal key tiles, kv head); the chunks of a
//      block merge by log-sum-exp in the last one to finish (atomic ticket). Its 128 accumulator rows are the kv head's two query heads x
//      64 positions, so both heads of the GQA group share every K/V tile.
//      TMA brings 128-byte-swizzled Q, K and V tiles into shared memory;
//      one thread issues tcgen05.mma for S = Q K^T (M=128, N=64, K=64) into
//      TMEM; every thread owns one row: tcgen05.ld of its 64 scores, causal
//      mask, online softmax in registers, P written as bf16 into a swizzled
//      K-major tile; a second tcgen05.mma computes P V (V consumed MN-major
//      straight from its TMA tile) into TMEM, read back and accumulated.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "qx_math.cuh"
#include "qx_ptx.cuh"
#include "qx_tc.cuh"

namespace qx {

struct PrefillParams {
  CUtensorMap tmq;  // rotated queries [L][16][64] bf16: box {64, 1, 64}, 128-byte swizzle
  CUtensorMap tmk;  // key cache [L][8][64] bf16, same box
  CUtensorMap tmv;  // value cache [L][8][64] bf16, same box
  const __nv_bfloat16* q;  // [L][16][64]
  const __nv_bfloat16* k;  // [L][8][64]
  const __nv_bfloat16* v;  // [L][8][64]
  __nv_bfloat16* q_rot;    // scratch [L][16][64]
  __nv_bfloat16* k_cache;  // [capacity][8][64]
  __nv_bfloat16* v_cache;
  void* out;  // [L][16][64]
  int out_dtype;
  int length;
  unsigned* err;
  // split of the key range: a query block's key tiles 0..qb are cut into
  // chunks of at most kc tiles, one CTA each; several chunks merge through
  // partials [item][8 heads][128 rows][68] (O[64], m, l, 2 pad: rows stay
  // 16-byte aligned for the float4 accesses) and a ticket per block
  int kc;
  float* partials;
  int* tickets;
  // diagnostics only (QXC_PREFILL_TRACE): per CTA, %globaltimer at stage
  // boundaries, kTraceSlots entries, written by thread 0
  unsigned long long* trace;
};

constexpr int kTraceSlots = 32;

// One CTA per position: sin/cos of the 32 pairs once, 24 heads rotated.
__global__ void __launch_bounds__(256) qx_prefill_rope_kernel(const __grid_constant__ PrefillParams p) {
  __shared__ float s_sin[32], s_cos[32];
  const int pos = blockIdx.x, tid = threadIdx.x;
  if (tid < 32) {
    float sn = 0.f, cs = 0.f;
    if (!granite_sin_cos((uint32_t)pos, tid, &sn, &cs)) flag_error(p.err, QX_ERR_BIT_NONFINITE);
    s_sin[tid] = sn;
    s_cos[tid] = cs;
  }
  __syncthreads();
  for (int idx = tid; idx < 24 * 32; idx += 256) {
    const int head = idx >> 5, pair = idx & 31;
    const __nv_bfloat16* src = head < 16 ? p.q + ((long long)pos * 16 + head) * 64
                                         : p.k + ((long long)pos * 8 + head - 16) * 64;
    __nv_bfloat16* dst = head < 16 ? p.q_rot + ((long long)pos * 16 + head) * 64
                                   : p.k_cache + ((long long)pos * 8 + head - 16) * 64;
    float a = 0.f, b = 0.f;
    if (!granite_rotate(__bfloat162float(src[pair]), __bfloat162float(src[pair + 32]), s_sin[pair], s_cos[pair], &a,
                        &b))
      flag_error(p.err, QX_ERR_BIT_NONFINITE);
    dst[pair] = __float2bfloat16_rn(a);
    dst[pair + 32] = __float2bfloat16_rn(b);
  }
  const uint4* vs = reinterpret_cast<const uint4*>(p.v + (long long)pos * 512);
  uint4* vd = reinterpret_cast<uint4*>(p.v_cache + (long long)pos * 512);
  if (tid < 64) vd[tid] = vs[tid];
}

struct PrefillCfg {
  static constexpr int NT = 128;
  static constexpr int TILE = 8192;               // [64 rows][128 B]
  static constexpr int OFF_Q = 0;                 // [128 rows][128 B]: rows 0-63 head 2h, 64-127 head 2h+1
  static constexpr int OFF_K = OFF_Q + 2 * TILE;  // 2 stages
  static constexpr int OFF_V = OFF_K + 2 * TILE;  // 2 stages
  static constexpr int OFF_P = OFF_V + 2 * TILE;  // [128 rows][128 B] bf16 probabilities
  static constexpr int OFF_BAR = OFF_P + 2 * TILE;
  static constexpr int SMEM = OFF_BAR + 64 + 1024;  // + slack to align the base to 1024
  static constexpr uint32_t TMEM_COLS = 128;        // S in [0,64), P.V in [64,128)
};

__global__ void __launch_bounds__(128) qx_prefill_attn_tc_kernel(const __grid_constant__ PrefillParams p) {
  using C = PrefillCfg;
  extern __shared__ __align__(1024) unsigned char sm_raw[];
  unsigned char* sm = sm_raw + ((1024u - (smem_addr(sm_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + C::OFF_BAR);  // [2] K/V stages
  uint64_t* qbar = full + 2;
  uint64_t* mbar = full + 3;  // tcgen05.commit target
  uint32_t* tslot = reinterpret_cast<uint32_t*>(full + 4);
  const int tid = threadIdx.x, warp = tid >> 5;
  const int h = blockIdx.y;
  // work item -> (query block qb, chunk c of its key tiles 0..qb)
  int qb = 0, c = blockIdx.x;
  for (;;) {
    const int n = (qb + p.kc) / p.kc;
    if (c < n) break;
    c -= n;
    ++qb;
  }
  const int nc = (qb + p.kc) / p.kc;      // chunks of this query block
  const int item0 = blockIdx.x - c;       // its first chunk's item
  const int j0 = c * p.kc;                // key tiles [j0, j1)
  const int j1 = min(j0 + p.kc, qb + 1);
  const uint32_t sQ = smem_addr(sm + C::OFF_Q), sK = smem_addr(sm + C::OFF_K), sV = smem_addr(sm + C::OFF_V),
                 sP = smem_addr(sm + C::OFF_P);

  if (tid == 0) {
    mbar_init(&full[0], 1);
    mbar_init(&full[1], 1);
    mbar_init(qbar, 1);
    mbar_init(mbar, 1);
    fence_barrier_init();
  }
  if (warp == 0) {
    tmem_alloc(tslot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  unsigned long long* tr = p.trace ? p.trace + ((long long)blockIdx.y * gridDim.x + blockIdx.x) * kTraceSlots : nullptr;
  int tn = 0;
  auto mark = [&]() {
    if (tr && tid == 0 && tn < kTraceSlots) tr[tn++] = global_ns();
  };
  mark();  // 0: after TMEM allocation

  if (tid == 0) {
    mbar_arrive_expect_tx(qbar, 2 * C::TILE);
    tma_load_3d(sm + C::OFF_Q, &p.tmq, 0, 2 * h, 64 * qb, qbar);
    tma_load_3d(sm + C::OFF_Q + C::TILE, &p.tmq, 0, 2 * h + 1, 64 * qb, qbar);
    for (int t = 0; t < 2 && j0 + t < j1; ++t) {
      mbar_arrive_expect_tx(&full[t], 2 * C::TILE);
      tma_load_3d(sm + C::OFF_K + t * C::TILE, &p.tmk, 0, h, 64 * (j0 + t), &full[t]);
      tma_load_3d(sm + C::OFF_V + t * C::TILE, &p.tmv, 0, h, 64 * (j0 + t), &full[t]);
    }
  }

  const int r = tid;                       // accumulator row == TMEM lane
  const int pos = 64 * qb + (r & 63);      // query position of this row
  const int qh = 2 * h + (r >> 6);         // query head of this row
  const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
  constexpr uint32_t IDESC_S = umma_idesc_bf16_f32(128, 64, false);
  constexpr uint32_t IDESC_PV = umma_idesc_bf16_f32(128, 64, true);
  // scores arrive as q.k; softmax runs in base 2 on q.k * (1/64) * log2(e)
  constexpr float SCALE_LOG2 = 0.015625f * 1.4426950408889634f;

  bool ok = mbar_wait_bounded(qbar, 0, p.err);
  mark();  // 1: Q landed
  float m = -INFINITY, l = 0.0f, O[64];
#pragma unroll
  for (int i = 0; i < 64; ++i) O[i] = 0.0f;
  uint32_t mphase = 0;

  for (int j = j0; j < j1; ++j) {
    const int s = (j - j0) & 1;
    ok &= mbar_wait_bounded(&full[s], (uint32_t)((j - j0) >> 1) & 1u, p.err);
    mark();  // tile: K/V landed
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        tc_mma_bf16(tbase, umma_desc_sw128(sQ + kk * 32, 16, 1024),
                    umma_desc_sw128(sK + s * C::TILE + kk * 32, 16, 1024), IDESC_S, kk > 0);
      tc_commit(mbar);
    }
    ok &= mbar_wait_bounded(mbar, mphase, p.err);
    mphase ^= 1u;
    mark();  // tile: S MMA done
    tc_fence_after();
    float sv[64];
    tmem_ld32(tbase + lane_base, sv);
    tmem_ld32(tbase + lane_base + 32, sv + 32);
    tmem_wait_ld();
    // causal mask on the diagonal tile (earlier tiles are entirely visible)
    float mx = -INFINITY;
#pragma unroll
    for (int c = 0; c < 64; ++c) {
      float x = sv[c] * SCALE_LOG2;
      if (j == qb && c > (r & 63)) x = -INFINITY;
      sv[c] = x;
      mx = fmaxf(mx, x);
    }
    const float mnew = fmaxf(m, mx);
    const float alpha = (m == -INFINITY) ? 0.0f : fast_exp2(m - mnew);
    m = mnew;
    float rs = 0.0f;
    uint32_t pk[32];
#pragma unroll
    for (int c = 0; c < 64; c += 2) {
      const float p0 = fast_exp2(sv[c] - mnew), p1 = fast_exp2(sv[c + 1] - mnew);
      rs += p0 + p1;
      const __nv_bfloat162 b2 = __floats2bfloat162_rn(p0, p1);
      pk[c >> 1] = *reinterpret_cast<const uint32_t*>(&b2);
    }
    l = fmaf(l, alpha, rs);
#pragma unroll
    for (int i = 0; i < 64; ++i) O[i] *= alpha;
    // P row r, K-major 128-byte swizzle: 16-byte chunk c at (c ^ (r & 7))
    unsigned char* prow = sm + C::OFF_P + r * 128;
#pragma unroll
    for (int c = 0; c < 8; ++c)
      *reinterpret_cast<uint4*>(prow + ((c ^ (r & 7)) << 4)) =
          make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
    fence_proxy_async_shared();  // generic-proxy stores -> tensor-core reads
    tc_fence_before();
    __syncthreads();
    mark();  // tile: softmax + P written
    if (tid == 0) {
      tc_fence_after();
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        tc_mma_bf16(tbase + 64, umma_desc_sw128(sP + kk * 32, 16, 1024),
                    umma_desc_sw128(sV + s * C::TILE + kk * 2048, C::TILE, 1024), IDESC_PV, kk > 0);
      tc_commit(mbar);
    }
    ok &= mbar_wait_bounded(mbar, mphase, p.err);
    mphase ^= 1u;
    mark();  // tile: P.V MMA done
    tc_fence_after();
    if (tid == 0 && j + 2 < j1) {  // both MMAs reading stage s are done
      mbar_arrive_expect_tx(&full[s], 2 * C::TILE);
      tma_load_3d(sm + C::OFF_K + s * C::TILE, &p.tmk, 0, h, 64 * (j + 2), &full[s]);
      tma_load_3d(sm + C::OFF_V + s * C::TILE, &p.tmv, 0, h, 64 * (j + 2), &full[s]);
    }
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      float pv[32];
      tmem_ld32(tbase + lane_base + 64 + 32 * half, pv);
      tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 32; ++i) O[32 * half + i] += pv[i];
    }
    tc_fence_before();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, C::TMEM_COLS);
  }
  mark();  // loop done, TMEM freed
  bool nonfinite = !ok;
  const long long ob = ((long long)pos * 16 + qh) * 64;
  if (nc > 1) {
    // this chunk's row partial: O (relative to m), m (base-2 units), l
    float* prow = p.partials + (((long long)(blockIdx.x) * 8 + h) * 128 + r) * 68;
#pragma unroll
    for (int i = 0; i < 16; ++i)
      reinterpret_cast<float4*>(prow)[i] = make_float4(O[4 * i], O[4 * i + 1], O[4 * i + 2], O[4 * i + 3]);
    prow[64] = m;
    prow[65] = l;
    __threadfence();
    __syncthreads();
    int* ticket = p.tickets + qb * 8 + h;
    __shared__ int last;
    if (tid == 0) last = (atomicAdd(ticket, 1) == nc - 1);
    __syncthreads();
    if (!last) return;
    __threadfence();
    // merge the nc chunks of this row by log-sum-exp
    float M = -INFINITY;
    for (int cc = 0; cc < nc; ++cc)
      M = fmaxf(M, __ldcg(p.partials + (((long long)(item0 + cc) * 8 + h) * 128 + r) * 68 + 64));
    l = 0.0f;
#pragma unroll
    for (int i = 0; i < 64; ++i) O[i] = 0.0f;
    for (int cc = 0; cc < nc; ++cc) {
      const float* pc = p.partials + (((long long)(item0 + cc) * 8 + h) * 128 + r) * 68;
      const float w = fast_exp2(__ldcg(pc + 64) - M);
      l = fmaf(w, __ldcg(pc + 65), l);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float4 v4 = __ldcg(reinterpret_cast<const float4*>(pc) + i);
        O[4 * i] = fmaf(w, v4.x, O[4 * i]);
        O[4 * i + 1] = fmaf(w, v4.y, O[4 * i + 1]);
        O[4 * i + 2] = fmaf(w, v4.z, O[4 * i + 2]);
        O[4 * i + 3] = fmaf(w, v4.w, O[4 * i + 3]);
      }
    }
    if (tid == 0) *ticket = 0;  // ready for the next call
    mark();  // merge done
  }
  if (pos < p.length) {
    const float inv = 1.0f / l;
    if (p.out_dtype == 0) {
      float4* o4 = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + ob);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float4 v4 = make_float4(O[4 * i] * inv, O[4 * i + 1] * inv, O[4 * i + 2] * inv, O[4 * i + 3] * inv);
        nonfinite |= !(isfinite(v4.x) && isfinite(v4.y) && isfinite(v4.z) && isfinite(v4.w));
        o4[i] = v4;
      }
    } else {
#pragma unroll
      for (int i = 0; i < 64; ++i) store_any(p.out, ob + i, p.out_dtype, O[i] * inv);
    }
    if (nonfinite) flag_error(p.err, ok ? QX_ERR_BIT_NONFINITE : QX_ERR_BIT_TIMEOUT);
  }
}

}  // namespace qx
