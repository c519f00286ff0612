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
//      (1) so its set-up overlaps (1)'s tail, one CTA per SM. A work item is
//      a (64-position query block, kv head); its 128 accumulator rows are the
//      kv head's two query heads x 64 positions, so both heads of the GQA
//      group share every K/V tile. A CTA runs one item, longest first, or,
//      when that takes two waves of CTAs and pairs fit in one, two items
//      (blocks nqb-1-j and j of one kv head) back to back. Warp roles:
//        warp 12    TMA producer: one thread streams the query tiles, then
//                   the K and V tiles, tile by tile, each through a
//                   six-stage ring (128-byte swizzle);
//        warps 13-15 MMA issuers, one per softmax group: the group's next
//                   scores S(T+3) = Q K_{T+3}^T (M=128, N=64, K=64) as soon
//                   as it holds S(T) in registers, then O += P(T) V_T (P
//                   read from TMEM) once it has written P(T);
//        warps 0-11 three softmax groups of four warps; key tile T belongs
//                   to group T % 3, so three tiles are in the softmax at
//                   once. A thread owns one accumulator row of its group:
//                   scores by tcgen05.ld, causal mask on the diagonal tile,
//                   P = 2^(s - m) in base 2 (a quarter of the exponentials on
//                   the FMA pipe) written to the group's P columns as bf16
//                   pairs by tcgen05.st, and summed (in f32) into the row's
//                   l. The max m moves only when a row's max exceeds it by
//                   2^8, the rare case in which the warp rescales its O in
//                   TMEM. At the end of an item every group publishes (m, l)
//                   in shared memory and group 0 merges the three O from
//                   TMEM and writes the rows.
//      Every hand-off is an mbarrier with its own phase sequence: full and
//      empty per K and V stage; per group scores full, scores read, P full,
//      and P done (the P.V that read it completed, so P's columns may take
//      the next P and O is settled); and, between two items, O read.
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
  int paired;  // attention CTA j takes query blocks nqb-1-j/8 and j/8 (one wave of CTAs instead of two)
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
  // softmax groups 0-2 (warps 4g..4g+3), TMA warp 12, MMA issuers warps 13-15
  static constexpr int NGROUP = 3;
  static constexpr int NT = 512;
  static constexpr int NSK = 6, NSV = 6;               // K and V ring stages
  static constexpr int TILE = 8192;                    // [64 rows][128 B]
  // two query tiles, one per work item, each [128 rows][128 B]: rows 0-63
  // head 2h, 64-127 head 2h+1
  static constexpr int OFF_Q = 0;
  static constexpr int OFF_K = OFF_Q + 4 * TILE;       // NSK stages
  static constexpr int OFF_V = OFF_K + NSK * TILE;     // NSV stages
  static constexpr int OFF_ML = OFF_V + NSV * TILE;    // [item][group][m, l][128 rows] f32
  static constexpr int OFF_BAR = OFF_ML + 2 * NGROUP * 2 * 128 * 4;
  // qfull[2]; K full/empty; V full/empty; per group sfull, sfree, pfull,
  // pdone, ofree, mdone
  static constexpr int NBAR = 2 + 2 * NSK + 2 * NSV + 6 * NGROUP;
  static constexpr int SMEM = OFF_BAR + NBAR * 8 + 16 + 1024;  // + TMEM slot, + slack to align the base
  // TMEM columns of group g: scores at COL_S + 64 g, O = sum P.V at
  // COL_O + 64 g, P (packed bf16 pairs, the A operand of P.V) at COL_P + 32 g
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t COL_S = 0, COL_O = 192, COL_P = 384;
  // the running max a group's P is taken against moves only when a row's
  // max exceeds it by more than TAU (base 2): P <= 2^TAU, and the rescale of
  // O in TMEM is rare
  static constexpr float TAU = 8.0f;
  // exponent pairs c with c % POLY_EVERY == POLY_EVERY - 1 run on the FMA
  // pipe, the others on the special-function unit
  static constexpr int POLY_EVERY = 4;
  static_assert(COL_P + 32 * NGROUP <= TMEM_COLS, "TMEM layout");
};

// CTA j takes kv head h = j % 8 and one or two query blocks (work items):
// qb = nqb-1-j/8, and when paired also qb = j/8, so every CTA attends
// about nqb+1 key tiles. The items' key tiles form one stream T = 0..ntot-1
// through the rings and TMEM buffers; tile T belongs to softmax group T % 3,
// which keeps its own running max, O and l per item; group 0 merges the
// three at the end of each item.
__global__ void __maxnreg__(128) qx_prefill_attn_tc_kernel(const __grid_constant__ PrefillParams p) {
  using C = PrefillCfg;
  constexpr int NSK = C::NSK, NSV = C::NSV, NG = C::NGROUP;
  extern __shared__ __align__(1024) unsigned char sm_raw[];
  unsigned char* sm = sm_raw + ((1024u - (smem_addr(sm_raw) & 1023u)) & 1023u);
  uint64_t* qfull = reinterpret_cast<uint64_t*>(sm + C::OFF_BAR);  // [item] query tile landed
  uint64_t* kfull = qfull + 2;      // [NSK] K tile landed
  uint64_t* kempty = kfull + NSK;   // [NSK] S MMA done with the K stage
  uint64_t* vfull = kempty + NSK;   // [NSV] V tile landed
  uint64_t* vempty = vfull + NSV;   // [NSV] P.V MMA done with the V stage
  uint64_t* sfull = vempty + NSV;   // [group] the group's scores in TMEM
  uint64_t* sfree = sfull + NG;     // [group] its four warps hold the scores in registers: the buffer may take the next
  uint64_t* pfull = sfree + NG;     // [group] P written to TMEM by its four warps
  uint64_t* pdone = pfull + NG;     // [group] P.V of that P completed: P buffer free, O settled
  uint64_t* ofree = pdone + NG;     // [group] group 0 read the group's O of the first item: the next may start
  uint64_t* mdone = ofree + NG;     // [issuer] every MMA it issued completed
  uint32_t* tslot = reinterpret_cast<uint32_t*>(mdone + NG);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int h = blockIdx.x & 7;
  const int qbA = p.nqb - 1 - (int)(blockIdx.x >> 3);  // longest query blocks first
  const int qbB = p.paired && (int)(blockIdx.x >> 3) < qbA ? (int)(blockIdx.x >> 3) : -1;
  const int nA = qbA + 1;
  const int nitems = qbB >= 0 ? 2 : 1;
  const int ntot = nA + qbB + 1;  // key tiles of both items (qbB + 1 = 0 when unpaired)
  const uint32_t sQ = smem_addr(sm + C::OFF_Q), sK = smem_addr(sm + C::OFF_K), sV = smem_addr(sm + C::OFF_V);

  if (tid == 0) {
    mbar_init(&qfull[0], 1);
    mbar_init(&qfull[1], 1);
    for (int s = 0; s < NSK; ++s) {
      mbar_init(&kfull[s], 1);
      mbar_init(&kempty[s], 1);
    }
    for (int s = 0; s < NSV; ++s) {
      mbar_init(&vfull[s], 1);
      mbar_init(&vempty[s], 1);
    }
    for (int g = 0; g < NG; ++g) {
      mbar_init(&sfull[g], 1);
      mbar_init(&sfree[g], 4);
      mbar_init(&pfull[g], 4);
      mbar_init(&pdone[g], 1);
      mbar_init(&ofree[g], 4);
    }
    for (int g = 0; g < NG; ++g) mbar_init(&mdone[g], 1);
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
  bool ok = true;

  if (warp == 4 * NG) {
    // ---- TMA producer: one thread streams Q, then K and V tile by tile -------
    // (one thread, not one lane each for K and V: two lanes of a warp that
    // wait on different barriers run their paths one at a time, and a lane
    // held in its wait delays the other's copies)
    if (lane == 0) {
      static_assert(NSK == NSV, "K and V stages advance together");
      prefetch_tmap(&p.tmq);
      prefetch_tmap(&p.tmk);
      prefetch_tmap(&p.tmv);
      pdl_wait();  // rotated queries and the key and value cache come from the RoPE grid
      for (int it = 0; it < nitems; ++it) {
        const int qb = it ? qbB : qbA;
        mbar_arrive_expect_tx(&qfull[it], 2 * C::TILE);
        tma_load_3d(sm + C::OFF_Q + it * 2 * C::TILE, &p.tmq, 0, 2 * h, 64 * qb, &qfull[it]);
        tma_load_3d(sm + C::OFF_Q + it * 2 * C::TILE + C::TILE, &p.tmq, 0, 2 * h + 1, 64 * qb, &qfull[it]);
      }
      for (int T = 0; T < ntot; ++T) {
        const int s = T % NSK, t = T < nA ? T : T - nA;
        const uint32_t ph = (uint32_t)(T / NSK - 1) & 1u;
        if (T >= NSK) ok &= mbar_wait_bounded(&kempty[s], ph, p.err);
        mbar_arrive_expect_tx(&kfull[s], C::TILE);
        tma_load_3d(sm + C::OFF_K + s * C::TILE, &p.tmk, 0, h, 64 * t, &kfull[s]);
        if (T >= NSV) ok &= mbar_wait_bounded(&vempty[s], ph, p.err);
        mbar_arrive_expect_tx(&vfull[s], C::TILE);
        tma_load_3d(sm + C::OFF_V + s * C::TILE, &p.tmv, 0, h, 64 * t, &vfull[s]);
      }
      // no copy may still be landing when the CTA exits
      for (int T = ntot > NSK ? ntot - NSK : 0; T < ntot; ++T) {
        ok &= mbar_wait_bounded(&kfull[T % NSK], (uint32_t)(T / NSK) & 1u, p.err);
        ok &= mbar_wait_bounded(&vfull[T % NSV], (uint32_t)(T / NSV) & 1u, p.err);
      }
    }
  } else if (warp > 4 * NG) {
    // ---- MMA issuers, one per softmax group: warp 13 + g serves group g -----
    const int gi = warp - 4 * NG - 1;
    if (lane == 0) {
      StageTrace mtrace(p.trace, (long long)gridDim.x + blockIdx.x, gi == 0);
      constexpr uint32_t IDESC_S = umma_idesc_bf16_f32(128, 64, false);
      constexpr uint32_t IDESC_PV = umma_idesc_bf16_f32(128, 64, true);
      // tile T is the (T / 3)-th tile of group T % 3
      auto issue_s = [&](int T) {
        const int s = T % NSK, g = T % NG, k = T / NG, it = T < nA ? 0 : 1;
        ok &= mbar_wait_bounded(&qfull[it], 0, p.err);
        ok &= mbar_wait_bounded(&kfull[s], (uint32_t)(T / NSK) & 1u, p.err);
        // the group holds its previous scores in registers
        if (k >= 1) ok &= mbar_wait_bounded(&sfree[g], (uint32_t)(k - 1) & 1u, p.err);
        tc_fence_after();
        const uint32_t q = sQ + it * 2 * C::TILE;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          tc_mma_bf16(tbase + C::COL_S + 64 * g, umma_desc_sw128(q + kk * 32, 16, 1024),
                      umma_desc_sw128(sK + s * C::TILE + kk * 32, 16, 1024), IDESC_S, kk > 0);
        tc_commit(&sfull[g]);
        tc_commit(&kempty[s]);
        mtrace.mark();  // S(T) issued
      };
      auto issue_pv = [&](int T) {
        const int g = T % NG, k = T / NG, sv = T % NSV;
        // the group's first tile of an item starts its O afresh; in the
        // second item only once group 0 has read the first item's O
        const bool first = T - NG < (T < nA ? 0 : nA);
        ok &= mbar_wait_bounded(&pfull[g], (uint32_t)k & 1u, p.err);
        mtrace.mark();  // P(T) seen
        ok &= mbar_wait_bounded(&vfull[sv], (uint32_t)(T / NSV) & 1u, p.err);
        if (first && T >= nA) ok &= mbar_wait_bounded(&ofree[g], 0, p.err);
        tc_fence_after();
        const uint32_t pa = tbase + C::COL_P + 32 * g;  // P: 128 lanes x 32 columns of bf16 pairs
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          tc_mma_ts_bf16(tbase + C::COL_O + 64 * g, pa + 8 * kk,
                         umma_desc_sw128(sV + sv * C::TILE + kk * 2048, C::TILE, 1024), IDESC_PV,
                         (first ? 0u : 1u) | (kk > 0 ? 1u : 0u));
        tc_commit(&pdone[g]);
        tc_commit(&vempty[sv]);
        mtrace.mark();  // P(T).V issued
      };
      // the group's next scores as soon as it holds S(T) in registers, so
      // they are ready when it has finished P(T)
      if (gi < ntot) issue_s(gi);
      for (int T = gi; T < ntot; T += NG) {
        if (T + NG < ntot) issue_s(T + NG);
        issue_pv(T);
      }
      tc_commit(&mdone[gi]);  // TMEM is released only after every MMA completed
      ok &= mbar_wait_bounded(&mdone[gi], 0, p.err);
    }
  } else {
    // ---- softmax groups: thread owns accumulator row r = 32 (warp % 4) + lane --
    const int g = warp >> 2;
    const int r = ((warp & 3) << 5) | lane;
    StageTrace trace(p.trace, g == 0 ? (long long)blockIdx.x : 2LL * gridDim.x + blockIdx.x,
                     tid == 0 || tid == 128);
    trace.mark();  // set-up done
    const uint32_t trow = tbase + ((uint32_t)((warp & 3) * 32) << 16);
    const uint32_t tS = trow + C::COL_S + 64 * g, tP = trow + C::COL_P + 32 * g;
    float* ml = reinterpret_cast<float*>(sm + C::OFF_ML);
    // scores arrive as q.k; the softmax runs in base 2 on q.k * (1/64) * log2(e)
    constexpr float SCALE_LOG2 = 0.015625f * 1.4426950408889634f;
    int T = g;  // this group's next tile of the stream
    for (int it = 0; it < nitems; ++it) {
      const int qb = it ? qbB : qbA;
      const int start = it ? nA : 0, end = start + qb + 1;
      float m = -INFINITY;  // the max this row's P is taken against
      // l = sum of this row's P (the f32 values before their rounding to the
      // bf16 operand of P.V), two packed partial sums
      float2 lsum[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
      for (; T < end; T += NG) {
        const int t = T - start, k = T / NG;
        ok &= mbar_wait_bounded(&sfull[g], (uint32_t)k & 1u, p.err);
        __syncwarp();
        tc_fence_after();
        float sv[64];
        tmem_ld32_sync(tS, sv);
        tmem_ld32_sync(tS + 32, sv + 32);
        // the scores are in registers: the group's next S may be computed
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&sfree[g]);
        trace.mark();  // tile: scores read
        // causal mask on the diagonal tile (earlier tiles are entirely visible)
        if (t == qb) {
#pragma unroll
          for (int c = 0; c < 64; ++c)
            if (c > (r & 63)) sv[c] = -INFINITY;
        }
        float m3[3] = {sv[0], sv[1], sv[2]};
#pragma unroll
        for (int c = 3; c < 63; c += 6) {
          m3[0] = fmax3f(m3[0], sv[c], sv[c + 1]);
          m3[1] = fmax3f(m3[1], sv[c + 2], sv[c + 3]);
          m3[2] = fmax3f(m3[2], sv[c + 4], sv[c + 5]);
        }
        const float mx = fmax3f(m3[0], fmaxf(m3[1], sv[63]), m3[2]) * SCALE_LOG2;
        const bool raise = mx > m + C::TAU;  // true on the group's first tile of the item (m = -inf)
        bool settled = false;                // P.V of the group's previous tile waited for
        if (__any_sync(0xffffffffu, raise) && T - NG >= start) {
          // rescale this warp's rows of O once their last P.V landed
          ok &= mbar_wait_bounded(&pdone[g], (uint32_t)(k - 1) & 1u, p.err);
          __syncwarp();
          tc_fence_after();
          settled = true;
          const float alpha = raise ? fast_exp2(m - mx) : 1.0f;
          const uint32_t tO = trow + C::COL_O + 64 * g;
#pragma unroll
          for (int c0 = 0; c0 < 64; c0 += 16) {
            float o[16];
            uint32_t ob[16];
            tmem_ld16_sync(tO + c0, o);
#pragma unroll
            for (int i = 0; i < 16; i += 2) {
              const float2 s2 = __fmul2_rn(make_float2(o[i], o[i + 1]), make_float2(alpha, alpha));
              ob[i] = __float_as_uint(s2.x);
              ob[i + 1] = __float_as_uint(s2.y);
            }
            tmem_st16u(tO + c0, ob);
          }
          tmem_wait_st();
          tc_fence_before();
        }
        if (raise) {
          const float alpha = fast_exp2(m - mx);  // 0 on the group's first tile (m = -inf)
          lsum[0] = __fmul2_rn(lsum[0], make_float2(alpha, alpha));
          lsum[1] = __fmul2_rn(lsum[1], make_float2(alpha, alpha));
          m = mx;
        }
        trace.mark();  // tile: row max
        // the P columns held the group's previous P until its P.V completed
        // (long since, as a rule)
        if (k > 0 && !settled) {
          ok &= mbar_wait_bounded(&pdone[g], (uint32_t)(k - 1) & 1u, p.err);
          __syncwarp();
          tc_fence_after();
        }
        // P = 2^(s * scale - m) rounded to bf16 pairs, the operand of P.V,
        // in two halves of 16 pairs
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint32_t pk[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int c = 32 * half + 2 * j;
            const float2 a = __ffma2_rn(make_float2(sv[c], sv[c + 1]), make_float2(SCALE_LOG2, SCALE_LOG2),
                                        make_float2(-m, -m));
            const float2 e = (j % C::POLY_EVERY) == C::POLY_EVERY - 1 ? exp2_poly2(a)
                                                                      : make_float2(fast_exp2(a.x), fast_exp2(a.y));
            const __nv_bfloat162 b2 = __floats2bfloat162_rn(e.x, e.y);
            pk[j] = *reinterpret_cast<const uint32_t*>(&b2);
            lsum[j & 1] = __fadd2_rn(lsum[j & 1], e);
          }
          tmem_st16u(tP + 16 * half, pk);
        }
        trace.mark();  // tile: P evaluated
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&pfull[g]);
        trace.mark();  // tile: P written
      }
      // publish (m, l) of this item; group 0 merges the groups' O from TMEM
      ml[((it * NG + g) * 2 + 0) * 128 + r] = m;
      ml[((it * NG + g) * 2 + 1) * 128 + r] = (lsum[0].x + lsum[0].y) + (lsum[1].x + lsum[1].y);
      named_sync(1, 128 * NG);
      trace.mark();  // item done
      if (g == 0) {
        float w[NG];
        bool has[NG];
        float M = -INFINITY, den = 0.0f;
#pragma unroll
        for (int u = 0; u < NG; ++u) M = fmaxf(M, ml[((it * NG + u) * 2) * 128 + r]);  // finite: group 0 has tile 0
#pragma unroll
        for (int u = 0; u < NG; ++u) {
          // group u's last tile of the item (none when the item has fewer than u + 1 tiles)
          const int last = end - 1 - (((end - 1 - u) % NG) + NG) % NG;
          has[u] = last >= start;
          const float mu = ml[((it * NG + u) * 2) * 128 + r];
          w[u] = has[u] ? fast_exp2(mu - M) : 0.0f;
          den = fmaf(w[u], ml[((it * NG + u) * 2 + 1) * 128 + r], den);
          if (has[u]) ok &= mbar_wait_bounded(&pdone[u], (uint32_t)(last / NG) & 1u, p.err);
        }
        __syncwarp();
        tc_fence_after();
        const float inv = 1.0f / den;
        const int pos = 64 * qb + (r & 63);  // query position of this row
        const int qh = 2 * h + (r >> 6);     // query head of this row
        const long long ob = ((long long)pos * 16 + qh) * 64;
        bool nonfinite = false;
#pragma unroll
        for (int c0 = 0; c0 < 64; c0 += 16) {
          float acc[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) acc[i] = 0.0f;
#pragma unroll
          for (int u = 0; u < NG; ++u) {
            if (!has[u]) continue;  // warp-uniform
            float o[16];
            tmem_ld16_sync(trow + C::COL_O + 64 * u + c0, o);
#pragma unroll
            for (int i = 0; i < 16; ++i) acc[i] = fmaf(w[u], o[i], acc[i]);
          }
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            acc[i] *= inv;
            nonfinite |= !isfinite(acc[i]);
          }
          if (pos < p.length) {
            if (p.out_dtype == 0) {
              float4* o4 = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + ob + c0);
#pragma unroll
              for (int i = 0; i < 4; ++i) o4[i] = make_float4(acc[4 * i], acc[4 * i + 1], acc[4 * i + 2], acc[4 * i + 3]);
            } else {
#pragma unroll
              for (int i = 0; i < 16; ++i) store_any(p.out, ob + c0 + i, p.out_dtype, acc[i]);
            }
          }
        }
        if (nonfinite && pos < p.length && ok) flag_error(p.err, QX_ERR_BIT_NONFINITE);
        if (it + 1 < nitems) {
          // every group's O of this item is in registers: the next item's P.V may start
          tc_fence_before();
          __syncwarp();
          if (lane == 0) {
#pragma unroll
            for (int u = 0; u < NG; ++u) mbar_arrive(&ofree[u]);
          }
        }
      }
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
