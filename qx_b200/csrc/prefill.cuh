// prefill.cuh — causal GQA prompt prefill for Granite on tcgen05 tensor
// cores (bf16 operands, f32 accumulation in TMEM).
//
// The reference has no dense prefill: a prompt is fed one token at a time
// through granite_attention_decode (qx-runtime-v2 lib.rs:4152-4187 loops
// `step`). Running the decode at positions 0..L-1 is exactly causal
// attention over a cache of RoPE'd keys, so prefill here is
//   1. qx_prefill_rope_kernel: four positions per CTA; qx's pinned sin/cos
//      of the 32 rotation pairs is evaluated once per position and applied
//      to all 16 query and 8 key heads with 16-byte loads and stores (same
//      operations as rotate_heads, qx-runtime lib.rs:2439-2453); keys go
//      into the cache as bf16 (bit-identical to the oracle), values are
//      copied, rotated queries go to a bf16 scratch;
//   2. qx_prefill_attn_tc_kernel, launched as a programmatic dependent of
//      (1) so its set-up overlaps (1)'s tail: one CTA per (64-position query
//      block, kv head), longest blocks first, one CTA per SM. Its 128
//      accumulator rows are the kv head's two query heads x 64 positions, so
//      both heads of the GQA group share every K/V tile. Warp roles:
//        warp 8     TMA producers: lane 0 streams Q and the K tiles, lane 1
//                   the V tiles, each through a four-stage ring (128-byte
//                   swizzle);
//        warps 9-10 MMA issuers, one per softmax group: S(t) = Q K_t^T
//                   (M=128, N=64, K=64) into a TMEM score buffer, then
//                   O += P(t) V_t and l += P(t) 1 with P read from TMEM;
//        warps 0-7  two softmax groups of four warps; key tile t belongs to
//                   group t & 1, so the groups' tiles overlap and a block's
//                   critical path is half its tiles. A thread owns one
//                   accumulator row of its group: scores by tcgen05.ld,
//                   causal mask on the diagonal tile, P = 2^(s - m) in base 2
//                   (a third of the exponentials on the FMA pipe) written
//                   back over the scores as bf16 pairs by tcgen05.st. The max
//                   m moves only when a row's max exceeds it by 2^8, the rare
//                   case in which the warp rescales its O and l in TMEM. At
//                   the end group 1 hands (m, l, O) to group 0 through shared
//                   memory and group 0 writes the merged rows.
//      Every hand-off is an mbarrier with its own phase sequence: full and
//      empty per K and V stage, full per score buffer, and done per P (the
//      P.V that read it completed, so the buffer may take new scores).
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
  int nqb;  // query blocks of 64 positions
  int early_trigger;  // the RoPE grid is resident all at once: let the attention grid launch at its start
  const float2* rope;  // pinned (sin, cos) [4096 positions][32 pairs]
  unsigned* err;
  unsigned long long* trace;  // stage timeline (diagnostics), or null
};

constexpr int kRopePositions = 4;  // positions per RoPE CTA
constexpr int kGraniteRopePositions = 4096;  // Granite MAX_CONTEXT

// qx's pinned (sin, cos) of every Granite position and rotation pair,
// evaluated once per context with the routine the decode kernels run inline
// (granite_rope_sin_cos, qx-consensus-math lib.rs:192-195).
__global__ void qx_granite_rope_table_kernel(float2* tab, unsigned* err) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= kGraniteRopePositions * 32) return;
  float s = 0.f, c = 0.f;
  if (!granite_sin_cos((uint32_t)(i >> 5), i & 31, &s, &c)) flag_error(err, QX_ERR_BIT_NONFINITE);
  tab[i] = make_float2(s, c);
}

// Four positions per CTA, 160 work items per position: 24 heads x 4 groups
// of 8 pairs (16-byte halves x[i..i+7] and x[i+32..i+39]) and the 64
// 16-byte chunks of its values. Every thread issues its loads (and the
// first 128 threads the positions' rows of the sin/cos table) before the
// CTA synchronises once.
__global__ void __launch_bounds__(256) qx_prefill_rope_kernel(const __grid_constant__ PrefillParams p) {
  constexpr int ITEMS = kRopePositions * 160;
  constexpr int PER_THREAD = (ITEMS + 255) / 256;
  __shared__ float s_sin[kRopePositions][32], s_cos[kRopePositions][32];
  // With every RoPE CTA resident at once, the attention grid may launch now:
  // its CTAs take each SM as its RoPE CTAs drain and wait for this grid in
  // griddepcontrol.wait (L = 2048: 31.4 -> 30.9 us per call; 512: 13.1 -> 12.5).
  if (p.early_trigger) pdl_launch_dependents();
  const int tid = threadIdx.x;
  const int pos0 = blockIdx.x * kRopePositions;
  uint4 lo[PER_THREAD], hi[PER_THREAD];
#pragma unroll
  for (int k = 0; k < PER_THREAD; ++k) {
    const int idx = tid + 256 * k, pp = idx / 160, w = idx - pp * 160, pos = pos0 + pp;
    lo[k] = hi[k] = make_uint4(0u, 0u, 0u, 0u);
    if (idx >= ITEMS || pos >= p.length) continue;
    if (w < 96) {
      const int head = w >> 2, i0 = (w & 3) * 8;
      const __nv_bfloat16* src = head < 16 ? p.q + ((long long)pos * 16 + head) * 64
                                           : p.k + ((long long)pos * 8 + head - 16) * 64;
      lo[k] = *reinterpret_cast<const uint4*>(src + i0);
      hi[k] = *reinterpret_cast<const uint4*>(src + 32 + i0);
    } else {
      lo[k] = reinterpret_cast<const uint4*>(p.v + (long long)pos * 512)[w - 96];
    }
  }
  if (tid < kRopePositions * 32) {
    const int pp = tid >> 5, pair = tid & 31, pos = pos0 + pp;
    const float2 sc = pos < p.length ? p.rope[pos * 32 + pair] : make_float2(0.f, 0.f);
    s_sin[pp][pair] = sc.x;
    s_cos[pp][pair] = sc.y;
  }
  __syncthreads();
#pragma unroll
  for (int k = 0; k < PER_THREAD; ++k) {
    const int idx = tid + 256 * k, pp = idx / 160, w = idx - pp * 160, pos = pos0 + pp;
    if (idx >= ITEMS || pos >= p.length) continue;
    if (w < 96) {
      const int head = w >> 2, i0 = (w & 3) * 8;
      __nv_bfloat16* dst = head < 16 ? p.q_rot + ((long long)pos * 16 + head) * 64
                                     : p.k_cache + ((long long)pos * 8 + head - 16) * 64;
      const __nv_bfloat16* x = reinterpret_cast<const __nv_bfloat16*>(&lo[k]);
      const __nv_bfloat16* y = reinterpret_cast<const __nv_bfloat16*>(&hi[k]);
      uint4 olo, ohi;
      __nv_bfloat16* a = reinterpret_cast<__nv_bfloat16*>(&olo);
      __nv_bfloat16* b = reinterpret_cast<__nv_bfloat16*>(&ohi);
      bool good = true;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float ra = 0.f, rb = 0.f;
        good &= granite_rotate(__bfloat162float(x[e]), __bfloat162float(y[e]), s_sin[pp][i0 + e], s_cos[pp][i0 + e],
                               &ra, &rb);
        a[e] = __float2bfloat16_rn(ra);
        b[e] = __float2bfloat16_rn(rb);
      }
      if (!good) flag_error(p.err, QX_ERR_BIT_NONFINITE);
      *reinterpret_cast<uint4*>(dst + i0) = olo;
      *reinterpret_cast<uint4*>(dst + 32 + i0) = ohi;
    } else {
      reinterpret_cast<uint4*>(p.v_cache + (long long)pos * 512)[w - 96] = lo[k];
    }
  }
  // Otherwise only now: the attention CTAs fill every SM's registers, so an
  // earlier start would starve the RoPE CTAs not yet resident.
  if (!p.early_trigger) pdl_launch_dependents();
}

struct PrefillCfg {
  // softmax groups 0 and 1 (warps 0-3 and 4-7), TMA warp 8, MMA issuers:
  // warp 9 for group 0, warp 10 for group 1
  static constexpr int NT = 352;
  static constexpr int NSK = 4, NSV = 4;               // K and V ring stages
  static constexpr int TILE = 8192;                    // [64 rows][128 B]
  static constexpr int OFF_Q = 0;                      // [128 rows][128 B]: rows 0-63 head 2h, 64-127 head 2h+1
  static constexpr int OFF_K = OFF_Q + 2 * TILE;       // NSK stages
  static constexpr int OFF_V = OFF_K + NSK * TILE;     // NSV stages
  static constexpr int OFF_ONES = OFF_V + NSV * TILE;  // [16 rows][128 B] bf16 1.0: row sums by MMA
  static constexpr int OFF_BAR = OFF_ONES + 2048;
  static constexpr int NBAR = 1 + 2 * NSK + 2 * NSV + 12 + 2;
  static constexpr int SMEM = OFF_BAR + NBAR * 8 + 16 + 1024;  // + TMEM slot, + slack to align the base
  // per group g (base 256 g): scores in columns +0 and +64 (two buffers;
  // P overwrites the first 32 columns of its scores as packed bf16 pairs and
  // is the TMEM A operand of P.V), O = sum P.V at +128 (64 columns),
  // l = sum P.1 at +192 (16 equal columns)
  static constexpr uint32_t TMEM_COLS = 512;
  // the running max a group's P is taken against moves only when a row's
  // max exceeds it by more than TAU (base 2): P <= 2^TAU, and the rescale of
  // O and l in TMEM is rare
  static constexpr float TAU = 8.0f;
  static_assert((NSK + NSV) * TILE >= 66 * 128 * 4, "group merge staging fits the K/V rings");
};

// One CTA per (query block qb, kv head h), longest blocks first; key tiles
// 0..qb alternate between the two softmax groups (tile t -> group t & 1),
// each with its own running max and its own O and l accumulators in TMEM,
// merged at the end.
__global__ void __launch_bounds__(352, 1) qx_prefill_attn_tc_kernel(const __grid_constant__ PrefillParams p) {
  using C = PrefillCfg;
  constexpr int NSK = C::NSK, NSV = C::NSV;
  extern __shared__ __align__(1024) unsigned char sm_raw[];
  unsigned char* sm = sm_raw + ((1024u - (smem_addr(sm_raw) & 1023u)) & 1023u);
  uint64_t* qfull = reinterpret_cast<uint64_t*>(sm + C::OFF_BAR);
  uint64_t* kfull = qfull + 1;      // [NSK] K tile landed
  uint64_t* kempty = kfull + NSK;   // [NSK] S MMA done with the K stage
  uint64_t* vfull = kempty + NSK;   // [NSV] V tile landed
  uint64_t* vempty = vfull + NSV;   // [NSV] P.V MMA done with the V stage
  uint64_t* sfull = vempty + NSV;   // [group][buffer] scores in TMEM
  uint64_t* pfull = sfull + 4;      // [group][buffer] P written over the scores by the group's four warps
  uint64_t* pdone = pfull + 4;      // [group][buffer] P.V and P.1 of that P completed: buffer free
  uint64_t* mdone = pdone + 4;      // [issuer] every MMA it issued completed
  uint32_t* tslot = reinterpret_cast<uint32_t*>(mdone + 2);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int qb = p.nqb - 1 - (int)(blockIdx.x >> 3);  // longest query blocks first
  const int h = blockIdx.x & 7;
  const int ntiles = qb + 1;
  const uint32_t sQ = smem_addr(sm + C::OFF_Q), sK = smem_addr(sm + C::OFF_K), sV = smem_addr(sm + C::OFF_V),
                 sOnes = smem_addr(sm + C::OFF_ONES);

  if (tid == 0) {
    mbar_init(qfull, 1);
    for (int s = 0; s < NSK; ++s) {
      mbar_init(&kfull[s], 1);
      mbar_init(&kempty[s], 1);
    }
    for (int s = 0; s < NSV; ++s) {
      mbar_init(&vfull[s], 1);
      mbar_init(&vempty[s], 1);
    }
    for (int i = 0; i < 4; ++i) {
      mbar_init(&sfull[i], 1);
      mbar_init(&pfull[i], 4);
      mbar_init(&pdone[i], 1);
    }
    mbar_init(&mdone[0], 1);
    mbar_init(&mdone[1], 1);
    fence_barrier_init();
  }
  for (int i = tid; i < 2048 / 16; i += C::NT)  // bf16 1.0 everywhere: no swizzle to mind
    reinterpret_cast<uint4*>(sm + C::OFF_ONES)[i] = make_uint4(0x3f803f80u, 0x3f803f80u, 0x3f803f80u, 0x3f803f80u);
  fence_proxy_async_shared();
  if (warp == 0) {
    tmem_alloc(tslot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tslot;
  bool ok = true;

  if (warp == 8) {
    // ---- TMA producers: lane 0 streams Q and K, lane 1 streams V ------------
    if (lane == 0) {
      prefetch_tmap(&p.tmq);
      prefetch_tmap(&p.tmk);
      pdl_wait();  // rotated queries and the key cache come from the RoPE grid
      mbar_arrive_expect_tx(qfull, 2 * C::TILE);
      tma_load_3d(sm + C::OFF_Q, &p.tmq, 0, 2 * h, 64 * qb, qfull);
      tma_load_3d(sm + C::OFF_Q + C::TILE, &p.tmq, 0, 2 * h + 1, 64 * qb, qfull);
      for (int t = 0; t < ntiles; ++t) {
        const int s = t % NSK;
        if (t >= NSK) ok &= mbar_wait_bounded(&kempty[s], (uint32_t)(t / NSK - 1) & 1u, p.err);
        mbar_arrive_expect_tx(&kfull[s], C::TILE);
        tma_load_3d(sm + C::OFF_K + s * C::TILE, &p.tmk, 0, h, 64 * t, &kfull[s]);
      }
      // no copy may still be landing when the CTA exits
      for (int t = ntiles > NSK ? ntiles - NSK : 0; t < ntiles; ++t)
        ok &= mbar_wait_bounded(&kfull[t % NSK], (uint32_t)(t / NSK) & 1u, p.err);
    } else if (lane == 1) {
      prefetch_tmap(&p.tmv);
      pdl_wait();  // the value cache comes from the RoPE grid
      for (int t = 0; t < ntiles; ++t) {
        const int s = t % NSV;
        if (t >= NSV) ok &= mbar_wait_bounded(&vempty[s], (uint32_t)(t / NSV - 1) & 1u, p.err);
        mbar_arrive_expect_tx(&vfull[s], C::TILE);
        tma_load_3d(sm + C::OFF_V + s * C::TILE, &p.tmv, 0, h, 64 * t, &vfull[s]);
      }
      for (int t = ntiles > NSV ? ntiles - NSV : 0; t < ntiles; ++t)
        ok &= mbar_wait_bounded(&vfull[t % NSV], (uint32_t)(t / NSV) & 1u, p.err);
    }
  } else if (warp >= 9) {
    // ---- MMA issuers: warp 9 serves group 0 (even tiles), warp 10 group 1 ---
    const int g = warp - 9;
    if (lane == 0) {
      StageTrace mtrace(p.trace, (long long)(1 + g) * gridDim.x + blockIdx.x, true);
      constexpr uint32_t IDESC_S = umma_idesc_bf16_f32(128, 64, false);
      constexpr uint32_t IDESC_PV = umma_idesc_bf16_f32(128, 64, true);
      constexpr uint32_t IDESC_SUM = umma_idesc_bf16_f32(128, 16, false);
      const uint32_t tg = tbase + 256 * g;
      ok &= mbar_wait_bounded(qfull, 0, p.err);
      // S(t) -> buffer (t >> 1) & 1 of group t & 1
      auto issue_s = [&](int t) {
        const int s = t % NSK, b = (t >> 1) & 1;
        ok &= mbar_wait_bounded(&kfull[s], (uint32_t)(t / NSK) & 1u, p.err);
        // the buffer held P(t-4) until P(t-4).V completed
        if (t >= 4) ok &= mbar_wait_bounded(&pdone[2 * g + b], (uint32_t)((t >> 2) - 1) & 1u, p.err);
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          tc_mma_bf16(tg + 64 * b, umma_desc_sw128(sQ + kk * 32, 16, 1024),
                      umma_desc_sw128(sK + s * C::TILE + kk * 32, 16, 1024), IDESC_S, kk > 0);
        tc_commit(&sfull[2 * g + b]);
        tc_commit(&kempty[s]);
        mtrace.mark();  // S(t) issued
      };
      // O += P(t).V and l += P(t).1 (the group's first tile starts them)
      auto issue_pv = [&](int t) {
        const int s = t % NSV, b = (t >> 1) & 1;
        ok &= mbar_wait_bounded(&pfull[2 * g + b], (uint32_t)(t >> 2) & 1u, p.err);
        mtrace.mark();  // P(t) seen
        ok &= mbar_wait_bounded(&vfull[s], (uint32_t)(t / NSV) & 1u, p.err);
        tc_fence_after();
        const uint32_t pa = tg + 64 * b;  // P: 128 lanes x 32 columns of bf16 pairs
        const uint32_t acc = t > g ? 1u : 0u;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          tc_mma_ts_bf16(tg + 128, pa + 8 * kk, umma_desc_sw128(sV + s * C::TILE + kk * 2048, C::TILE, 1024),
                         IDESC_PV, acc | (kk > 0));
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          tc_mma_ts_bf16(tg + 192, pa + 8 * kk, umma_desc_sw128(sOnes + kk * 32, 16, 1024), IDESC_SUM,
                         acc | (kk > 0));
        tc_commit(&pdone[2 * g + b]);
        tc_commit(&vempty[s]);
      };
      if (g < ntiles) issue_s(g);
      if (g + 2 < ntiles) issue_s(g + 2);
      for (int t = g; t < ntiles; t += 2) {
        issue_pv(t);
        if (t + 4 < ntiles) issue_s(t + 4);
      }
      tc_commit(&mdone[g]);  // TMEM is released only after every MMA completed
      ok &= mbar_wait_bounded(&mdone[g], 0, p.err);
    }
  } else {
    // ---- softmax groups: thread owns accumulator row r = 32 (warp % 4) + lane --
    const int g = warp >> 2;
    const int r = ((warp & 3) << 5) | lane;
    StageTrace trace(p.trace, blockIdx.x, tid == 0);
    trace.mark();  // set-up done
    const int pos = 64 * qb + (r & 63);  // query position of this row
    const int qh = 2 * h + (r >> 6);     // query head of this row
    const uint32_t trow = tbase + ((uint32_t)((warp & 3) * 32) << 16) + 256 * g;
    // scores arrive as q.k; the softmax runs in base 2 on q.k * (1/64) * log2(e)
    constexpr float SCALE_LOG2 = 0.015625f * 1.4426950408889634f;
    float m = -INFINITY;  // the max this row's P is taken against
    for (int t = g; t < ntiles; t += 2) {
      const int b = (t >> 1) & 1;
      ok &= mbar_wait_bounded(&sfull[2 * g + b], (uint32_t)(t >> 2) & 1u, p.err);
      __syncwarp();
      tc_fence_after();
      float sv[64];
      tmem_ld32_sync(trow + 64 * b, sv);
      tmem_ld32_sync(trow + 64 * b + 32, sv + 32);
      trace.mark();  // tile: scores read
      // causal mask on the diagonal tile (earlier tiles are entirely visible)
      if (t == qb) {
#pragma unroll
        for (int c = 0; c < 64; ++c)
          if (c > (r & 63)) sv[c] = -INFINITY;
      }
      float m4[4] = {sv[0], sv[1], sv[2], sv[3]};
#pragma unroll
      for (int c = 4; c < 64; ++c) m4[c & 3] = fmaxf(m4[c & 3], sv[c]);
      const float mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])) * SCALE_LOG2;
      const bool raise = mx > m + C::TAU;  // true on the group's first tile (m = -inf)
      trace.mark();  // tile: row max
      if (__any_sync(0xffffffffu, raise) && t > g) {
        // rescale this warp's rows of O and l once their last P.V landed
        const int u = t - 2;
        ok &= mbar_wait_bounded(&pdone[2 * g + ((u >> 1) & 1)], (uint32_t)(u >> 2) & 1u, p.err);
        __syncwarp();
        tc_fence_after();
        const float alpha = raise ? fast_exp2(m - mx) : 1.0f;
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          float o[32];
          tmem_ld32_sync(trow + 128 + 32 * half, o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] *= alpha;
          tmem_st32(trow + 128 + 32 * half, o);
        }
        tmem_st1(trow + 192, tmem_ld1_sync(trow + 192) * alpha);
        tmem_wait_st();
        tc_fence_before();
        trace.mark();  // tile: O and l rescaled
      }
      if (raise) m = mx;
      // P = 2^(s * scale - m) rounded to bf16 pairs, exactly the operand of
      // P.V; their row sums come from the P.1 MMA, so l and O see the same P
      // (every third pair on the FMA pipe, the rest on the special-function
      // unit, which the exponentials of both groups would otherwise saturate)
      uint32_t pk[32];
#pragma unroll
      for (int c = 0; c < 64; c += 2) {
        const float a0 = fmaf(sv[c], SCALE_LOG2, -m), a1 = fmaf(sv[c + 1], SCALE_LOG2, -m);
        const bool poly = ((c >> 1) % 3) == 2;
        const __nv_bfloat162 b2 = poly ? __floats2bfloat162_rn(exp2_poly(a0), exp2_poly(a1))
                                       : __floats2bfloat162_rn(fast_exp2(a0), fast_exp2(a1));
        pk[c >> 1] = *reinterpret_cast<const uint32_t*>(&b2);
      }
      trace.mark();  // tile: P evaluated
      // P over the scores it came from: row r = TMEM lane r, columns 0..31
      tmem_st32u(trow + 64 * b, pk);
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&pfull[2 * g + b]);
      trace.mark();  // tile: P written
    }
    // this group's accumulators, once its last P.V landed
    const int last = ntiles - 1 - ((ntiles - 1 - g) & 1);  // the group's last tile (or < 0)
    float O[64], l = 0.0f;
    if (last >= 0) {
      ok &= mbar_wait_bounded(&pdone[2 * g + ((last >> 1) & 1)], (uint32_t)(last >> 2) & 1u, p.err);
      __syncwarp();
      tc_fence_after();
      tmem_ld32_sync(trow + 128, O);
      tmem_ld32_sync(trow + 160, O + 32);
      l = tmem_ld1_sync(trow + 192);
    } else {
#pragma unroll
      for (int i = 0; i < 64; ++i) O[i] = 0.0f;
    }
    trace.mark();  // group done
    // merge the two groups: group 1 stages (m, l, O) column-major in the K/V
    // rings (every copy into them has landed and every MMA reading them has
    // completed once both groups read their accumulators)
    float* stage = reinterpret_cast<float*>(sm + C::OFF_K);  // [66][128]
    named_sync(1, 256);
    if (g == 1) {
      stage[64 * 128 + r] = m;
      stage[65 * 128 + r] = l;
#pragma unroll
      for (int i = 0; i < 64; ++i) stage[i * 128 + r] = O[i];
    }
    named_sync(1, 256);
    if (g == 0 && pos < p.length) {
      const float m1 = stage[64 * 128 + r], l1 = stage[65 * 128 + r];
      const float M = fmaxf(m, m1);
      const float w0 = fast_exp2(m - M), w1 = (m1 == -INFINITY) ? 0.0f : fast_exp2(m1 - M);
      const float inv = 1.0f / fmaf(w0, l, w1 * l1);
      bool nonfinite = false;
      const long long ob = ((long long)pos * 16 + qh) * 64;
      if (p.out_dtype == 0) {
        float4* o4 = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + ob);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float v[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) v[j] = fmaf(w0, O[4 * i + j], w1 * stage[(4 * i + j) * 128 + r]) * inv;
          nonfinite |= !(isfinite(v[0]) && isfinite(v[1]) && isfinite(v[2]) && isfinite(v[3]));
          o4[i] = make_float4(v[0], v[1], v[2], v[3]);
        }
      } else {
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          const float v = fmaf(w0, O[i], w1 * stage[i * 128 + r]) * inv;
          nonfinite |= !isfinite(v);
          store_any(p.out, ob + i, p.out_dtype, v);
        }
      }
      if (nonfinite && ok) flag_error(p.err, QX_ERR_BIT_NONFINITE);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tbase, C::TMEM_COLS);
  }
}

}  // namespace qx
