// decode_tc.cuh — Qwen3 split-KV decode on tcgen05 tensor cores.
//
// Qwen3-30B-A3B attention has 8 query heads per kv head and head_dim 128:
// every cached row meets 8 queries, 2 x 8 x 128 multiply-adds per row, which
// CUDA cores cannot issue as fast as HBM delivers the row. Both contractions
// therefore run on the tensor cores, per 128-row tile of the kv head:
//
//   S^T [128 rows x 16]  = K [128 rows x 128 dims] . Q^T      (tcgen05.mma
//       M=128, N=16 = the 8 query heads padded with zero rows, K=128;
//       K straight from its TMA tile, 128-byte swizzle, K-major)
//   O^T [128 dims x 16] = V^T [128 dims x 128 rows] . P^T      (M=128 dims,
//       V consumed MN-major from the same kind of tile, P^T K-major)
//
// Accumulators live in TMEM (32 columns). Thread t of the four consumer
// warps owns TMEM lane t: position t of S^T (its 8 head scores) and dim t
// of O^T. The softmax is per head over the tile's 128 positions: warp
// shuffles plus a four-warp shared-memory step. A producer warp streams K
// and V (32 KB each per tile) into one buffer each: K is released once the
// S MMA has read it, so the next tile's K loads during this tile's softmax
// and P.V; V is released once the P.V MMA has read it.
//
// Prologue (RMSNorm with the reference's sequential sum, rotate-half RoPE
// from the host cos/sin table, the appended row) and the split merge are
// those of qx_decode_kernel (tools/qx-qwen-parity/src/main.rs:1170-1258).
#pragma once
#include <type_traits>

#include "decode.cuh"
#include "qx_tc.cuh"

namespace qx {

template <typename KT>
struct TcCfg {
  static constexpr int T = 128;  // cache rows per tile
  static constexpr int D = 128, G = 8, HKV = 4, HQ = 32;
  static constexpr int NPAD = 16;       // MMA N (8 heads + 8 zero rows)
  static constexpr int BLK = T * 128;   // one 64-dim column block [128 rows][128 B]
  static constexpr int STAGE = 2 * BLK;  // K (or V) of one tile: 32 KB
  // One K buffer and one V buffer (78 KB per CTA, two CTAs per SM). The
  // next tile's K streams in as soon as the S MMA has consumed the current
  // one, overlapping the softmax and the P.V MMA; V follows after P.V.
  static constexpr int OFF_K = 0;
  static constexpr int OFF_V = OFF_K + STAGE;
  static constexpr int OFF_Q = OFF_V + STAGE;            // 2 blocks [16 rows][128 B]
  static constexpr int OFF_P = OFF_Q + 2 * NPAD * 128;   // 2 blocks [16 rows][128 B]
  static constexpr int OFF_RAW = OFF_P + 2 * NPAD * 128;  // f32 [(G + 1)][D]
  static constexpr int OFF_NEWK = OFF_RAW + (G + 1) * D * 4;
  static constexpr int OFF_NEWV = OFF_NEWK + D * 2;
  static constexpr int OFF_RED = OFF_NEWV + D * 2;  // f32 [2][4 warps][G]
  static constexpr int OFF_STAT = OFF_RED + 2 * 4 * G * 4;  // f32 [2 * G]; inv [G + 1]
  static constexpr int OFF_BAR = ((OFF_STAT + 4 * (3 * G + 1) + 15) / 16) * 16;
  static constexpr int SMEM = OFF_BAR + 64 + 1024;  // + slack to align the base to 1024
  static constexpr int NT = 160;                     // 4 consumer warps + 1 producer warp
  static constexpr uint32_t TMEM_COLS = 32;          // S^T in [0,16), O^T tile in [16,32)
  static constexpr int FMT = std::is_same<KT, __nv_bfloat16>::value ? 1 : 0;  // MMA operand format
  static constexpr int MAX_SPLITS = (2 * STAGE) / (8 * G);
};

template <typename KT>
__global__ void __launch_bounds__(160) qx_decode_tc_kernel(const __grid_constant__ DecodeParams p) {
  using C = TcCfg<KT>;
  constexpr int D = C::D, G = C::G, HKV = C::HKV, HQ = C::HQ, T = C::T;
  extern __shared__ __align__(1024) unsigned char sm_raw[];
  unsigned char* sm = sm_raw + ((1024u - (smem_addr(sm_raw) & 1023u)) & 1023u);
  float* raw = reinterpret_cast<float*>(sm + C::OFF_RAW);
  KT* newk = reinterpret_cast<KT*>(sm + C::OFF_NEWK);
  KT* newv = reinterpret_cast<KT*>(sm + C::OFF_NEWV);
  float* red_max = reinterpret_cast<float*>(sm + C::OFF_RED);  // [4][G]
  float* red_sum = red_max + 4 * G;                              // [4][G]
  float* stat = reinterpret_cast<float*>(sm + C::OFF_STAT);     // [2G] merge stats
  float* st_inv = stat + 2 * G;                                  // [G + 1]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + C::OFF_BAR);
  uint64_t* fullK = bars + 0;   // TMA landed
  uint64_t* fullV = bars + 1;
  uint64_t* emptyK = bars + 2;  // buffer free again (its MMA completed)
  uint64_t* emptyV = bars + 3;
  uint64_t* mbarS = bars + 4;   // tcgen05.commit of the S MMAs
  uint64_t* mbarPV = bars + 5;  // tcgen05.commit of the P.V MMAs
  uint32_t* tslot = reinterpret_cast<uint32_t*>(bars + 6);
  int* s_flag = reinterpret_cast<int*>(bars + 7);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  SeqInfo si;
  const int slot = find_slot(p, &si);
  const int nsplit = (si.attend + p.chunk - 1) / p.chunk;
  int r = blockIdx.x - si.item_begin;
  const int lloc = r / (HKV * nsplit);
  r -= lloc * HKV * nsplit;
  const int h = r / nsplit;
  const int s = r - h * nsplit;
  const int layer = p.layer_begin + lloc;
  const long long unit = (long long)si.seq_id * p.layers + layer;
  const char* kunit = p.k_region + unit * p.k_unit_bytes;
  const char* vunit = p.v_region + unit * p.v_unit_bytes;
  const int begin = s * p.chunk;
  const int end = min(begin + p.chunk, si.attend);
  const bool has_new = si.new_slot >= begin && si.new_slot < end;
  const int ntiles = (end - begin + T - 1) / T;
  const long long cu = (long long)slot * p.layer_count + lloc;
  const bool last_split = (s == nsplit - 1);

  if (tid == 0) {
    for (int i = 0; i < 6; ++i) mbar_init(&bars[i], 1);
    s_flag[1] = 0;
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
  StageTrace trace(p.trace, blockIdx.x, tid == 0);
  trace.mark();  // TMEM allocated

  if (warp == 4) {
    // ---- producer: K and V tiles, 4 TMA boxes each ([64 rows][128 B]) ------
    if (lane == 0) {
      prefetch_tmap(&p.tmk);
      prefetch_tmap(&p.tmv);
      const int z0 = (int)(unit * p.capacity) + begin;
      unsigned char* kt = sm + C::OFF_K;
      unsigned char* vt = sm + C::OFF_V;
      for (int tile = 0; tile < ntiles; ++tile) {
        const uint32_t prev = (uint32_t)(tile - 1) & 1u;
        const int z = z0 + tile * T;
        if (tile >= 1 && !mbar_wait_bounded(emptyK, prev, p.err)) {
          s_flag[1] = 1;
          break;
        }
        mbar_arrive_expect_tx(fullK, (uint32_t)C::STAGE);
#pragma unroll
        for (int b = 0; b < 2; ++b)
#pragma unroll
          for (int half = 0; half < 2; ++half)
            tma_load_3d(kt + b * C::BLK + half * 8192, &p.tmk, b * 64, h, z + half * 64, fullK);
        if (tile >= 1 && !mbar_wait_bounded(emptyV, prev, p.err)) {
          s_flag[1] = 1;
          break;
        }
        mbar_arrive_expect_tx(fullV, (uint32_t)C::STAGE);
#pragma unroll
        for (int b = 0; b < 2; ++b)
#pragma unroll
          for (int half = 0; half < 2; ++half)
            tma_load_3d(vt + b * C::BLK + half * 8192, &p.tmv, b * 64, h, z + half * 64, fullV);
      }
    }
  } else {
    // ---- consumers: prologue ------------------------------------------------
    const long long qbase = (cu * HQ + (long long)h * G) * D;
    const long long kvbase = (cu * HKV + h) * D;
    bool bad = false;
    for (int i = tid; i < (G + 1) * D; i += 128) {
      const int g = i / D, e = i - g * D;
      raw[i] = g < G ? load_any(p.q, qbase + g * D + e, p.q_dtype)
                     : (has_new ? load_any(p.k, kvbase + e, p.in_dtype) : 0.0f);
    }
    // zero the padding rows 8..15 of Q and P (both column blocks)
    for (int i = tid; i < 4 * 128; i += 128) {
      const int blk = i >> 7, j = i & 127;  // blk 0,1: Q blocks; 2,3: P blocks
      unsigned char* base = sm + (blk < 2 ? C::OFF_Q : C::OFF_P) + (blk & 1) * 2048 + 1024;
      reinterpret_cast<uint2*>(base)[j] = make_uint2(0u, 0u);
    }
    consumers_sync(128);
    if (tid < G || (tid == G && has_new)) {
      const float* row = raw + tid * D;
      float sum = 0.0f;
#pragma unroll
      for (int i = 0; i < D; ++i) sum = __fadd_rn(sum, __fmul_rn(row[i], row[i]));
      st_inv[tid] = __frcp_rn(__fsqrt_rn(__fadd_rn(__fdiv_rn(sum, 128.0f), 1.0e-6f)));
    }
    consumers_sync(128);
    const float2* tab = p.rope_table + (long long)si.rope_pos * 64;
    for (int idx = tid; idx < (G + 1) * 64; idx += 128) {
      const int g = idx >> 6, i = idx & 63;
      if (g == G && !has_new) break;
      const bool is_q = g < G;
      const float inv = st_inv[g];
      const float* wn = is_q ? p.q_norm : p.k_norm;
      const float x = raw[g * D + i], y = raw[g * D + i + 64];
      const float left = __fmul_rn(__fmul_rn(x, inv), wn ? wn[i] : 1.0f);
      const float right = __fmul_rn(__fmul_rn(y, inv), wn ? wn[64 + i] : 1.0f);
      const float2 cssn = tab[i];
      const float a = __fsub_rn(__fmul_rn(left, cssn.x), __fmul_rn(right, cssn.y));
      const float b = __fadd_rn(__fmul_rn(right, cssn.x), __fmul_rn(left, cssn.y));
      bad |= !(isfinite(a) && isfinite(b));
      const KT ka = Elem<KT>::from_f32(a), kb = Elem<KT>::from_f32(b);
      if (is_q) {
        // Q row g (K-major, 128-byte swizzle): dims i and i+64 in blocks 0 and 1
        const int c = (i & 63) >> 3, off = (i & 7) * 2;
        *reinterpret_cast<KT*>(sm + C::OFF_Q + g * 128 + ((c ^ (g & 7)) << 4) + off) = ka;
        *reinterpret_cast<KT*>(sm + C::OFF_Q + 2048 + g * 128 + ((c ^ (g & 7)) << 4) + off) = kb;
        if (p.q_rot_out && last_split) {
          p.q_rot_out[qbase + g * D + i] = Elem<KT>::to_f32(ka);
          p.q_rot_out[qbase + g * D + i + 64] = Elem<KT>::to_f32(kb);
        }
      } else {
        newk[i] = ka;
        newk[i + 64] = kb;
      }
    }
    if (has_new)
      for (int i = tid; i < D; i += 128) newv[i] = Elem<KT>::from_f32(load_any(p.v, kvbase + i, p.in_dtype));
    if (bad) flag_error(p.err, QX_ERR_BIT_NONFINITE);
    consumers_sync(128);
    if (has_new) {
      char* kdst = const_cast<char*>(kunit) + ((long long)si.new_slot * HKV + h) * (D * 2);
      char* vdst = const_cast<char*>(vunit) + ((long long)si.new_slot * HKV + h) * (D * 2);
      if (tid < 16) reinterpret_cast<uint4*>(kdst)[tid] = reinterpret_cast<const uint4*>(newk)[tid];
      else if (tid < 32) reinterpret_cast<uint4*>(vdst)[tid - 16] = reinterpret_cast<const uint4*>(newv)[tid - 16];
    }
    fence_proxy_async_shared();  // Q / P padding written by threads, read by tcgen05.mma
    trace.mark();  // prologue done

    // ---- consumers: tiles ----------------------------------------------------
    const bool pinned = p.pinned_exp != 0;
    constexpr float SCALE_LOG2 = 0.08838834764831845f * 1.4426950408889634f;  // 1/sqrt(128) * log2(e)
    constexpr uint32_t IDESC_S = umma_idesc_16bit(128, C::NPAD, C::FMT, false, false);
    constexpr uint32_t IDESC_PV = umma_idesc_16bit(128, C::NPAD, C::FMT, true, false);
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    const uint32_t sQ = smem_addr(sm + C::OFF_Q), sP = smem_addr(sm + C::OFF_P);
    float m_run[G], l_run[G], O[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      m_run[g] = -INFINITY;
      l_run[g] = 0.0f;
      O[g] = 0.0f;
    }
    bool ok = true;
    // every consumer runs every iteration (the named barriers need all 128);
    // after a timed-out wait a thread stops waiting and the result is discarded
    unsigned char* kt = sm + C::OFF_K;
    unsigned char* vt = sm + C::OFF_V;
    const uint32_t sK = smem_addr(kt), sV = smem_addr(vt);
    for (int tile = 0; tile < ntiles; ++tile) {
      const uint32_t ph = (uint32_t)tile & 1u;
      const int rows = min(T, end - (begin + tile * T));
      const bool last = has_new && tile == ntiles - 1;
      if (ok) ok = mbar_wait_bounded(fullK, ph, p.err);
      trace.mark();  // tile: K landed
      if (last && tid < 16)  // the appended key comes from registers, not from the copy
        *reinterpret_cast<uint4*>(kt + swz<C::BLK>(rows - 1, tid * 16)) = reinterpret_cast<const uint4*>(newk)[tid];
      fence_proxy_async_shared();
      tc_fence_before();
      consumers_sync(128);
      if (tid == 0) {
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          tc_mma_bf16(tbase, umma_desc_sw128(sK + (kk >> 2) * C::BLK + (kk & 3) * 32, 16, 1024),
                      umma_desc_sw128(sQ + (kk >> 2) * 2048 + (kk & 3) * 32, 16, 1024), IDESC_S, kk > 0);
        tc_commit(mbarS);
      }
      if (ok) ok = mbar_wait_bounded(mbarS, ph, p.err);
      trace.mark();  // tile: S MMA done
      tc_fence_after();
      if (tid == 0) mbar_arrive(emptyK);  // the S MMAs are done with K
      float x[G];
      tmem_ld8(tbase + lane_base, x);
      tmem_wait_ld();
#pragma unroll
      for (int g = 0; g < G; ++g) {
        x[g] = tid < rows ? x[g] * SCALE_LOG2 : -INFINITY;
        const float wm = warp_max(x[g]);
        if (lane == 0) red_max[warp * G + g] = wm;
      }
      consumers_sync(128);
      float alpha[G];
      const int pb = tid >> 6, pc = (tid & 63) >> 3, poff = (tid & 7) * 2;
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float tmax = fmaxf(fmaxf(red_max[g], red_max[G + g]), fmaxf(red_max[2 * G + g], red_max[3 * G + g]));
        const float mnew = fmaxf(m_run[g], tmax);
        alpha[g] = (m_run[g] == -INFINITY) ? 0.0f : fast_exp2(m_run[g] - mnew);
        const float pw = fast_exp2(x[g] - mnew);
        m_run[g] = mnew;
        // P^T row g (a head), column tid (a position): K-major, 128-byte swizzle
        *reinterpret_cast<KT*>(sm + C::OFF_P + pb * 2048 + g * 128 + ((pc ^ (g & 7)) << 4) + poff) =
            Elem<KT>::from_f32(pw);
        const float ws = warp_sum(pw);
        if (lane == 0) red_sum[warp * G + g] = ws;
      }
      if (ok) ok = mbar_wait_bounded(fullV, ph, p.err);
      trace.mark();  // tile: softmax done, V landed
      if (last && tid < 16)
        *reinterpret_cast<uint4*>(vt + swz<C::BLK>(rows - 1, tid * 16)) = reinterpret_cast<const uint4*>(newv)[tid];
      // rows past the cache end carry zero probability; zero their values so
      // the tensor core never multiplies 0 by a stale non-finite element
      for (int i = tid; i < (T - rows) * 16; i += 128) {
        const int rr = rows + (i >> 4);
        *reinterpret_cast<uint4*>(vt + swz<C::BLK>(rr, (i & 15) * 16)) = make_uint4(0u, 0u, 0u, 0u);
      }
      fence_proxy_async_shared();
      tc_fence_before();
      consumers_sync(128);
      if (tid == 0) {
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          tc_mma_bf16(tbase + 16, umma_desc_sw128(sV + kk * 2048, C::BLK, 1024),
                      umma_desc_sw128(sP + (kk >> 2) * 2048 + (kk & 3) * 32, 16, 1024), IDESC_PV, kk > 0);
        tc_commit(mbarPV);
      }
#pragma unroll
      for (int g = 0; g < G; ++g)
        l_run[g] = fmaf(l_run[g], alpha[g],
                        (red_sum[g] + red_sum[G + g]) + (red_sum[2 * G + g] + red_sum[3 * G + g]));
      if (ok) ok = mbar_wait_bounded(mbarPV, ph, p.err);
      trace.mark();  // tile: P.V MMA done
      tc_fence_after();
      if (tid == 0) mbar_arrive(emptyV);  // the P.V MMAs are done with V
      float pv[G];
      tmem_ld8(tbase + lane_base + 16, pv);
      tmem_wait_ld();
#pragma unroll
      for (int g = 0; g < G; ++g) O[g] = fmaf(O[g], alpha[g], pv[g]);
      tc_fence_before();
    }
    if (!ok) s_flag[1] = 1;
    // thread tid = dim, k = head for finish_outputs
    float Mg[G], Lg[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      Mg[g] = m_run[g] / 1.4426950408889634f;  // back to the natural-log domain of the partials
      Lg[g] = l_run[g];
    }
    tc_fence_before();
    cta_sync();  // (A) with the producer warp
    if (warp == 0) {
      tc_fence_after();
      tmem_dealloc(tbase, C::TMEM_COLS);
    }
    if (s_flag[1]) return;
    trace.mark();  // tiles done
    finish_outputs<G, D, HKV, HQ, G>(p, O, Mg, Lg, nsplit, s, cu, h, tid, warp, lane, pinned,
                                     reinterpret_cast<float*>(sm + C::OFF_K), stat, s_flag);
    trace.mark();  // outputs (or partials) written
    return;
  }
  cta_sync();  // (A) for the producer warp
}

}  // namespace qx
