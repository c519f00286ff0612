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
//   O^T [128 dims x 16] += V^T [128 dims x 128 rows] . P^T     (M=128 dims,
//       V consumed MN-major from the same kind of tile, P^T K-major)
//
// One CTA per SM streams its split through a three-stage ring of K tiles and
// one of V tiles (warp 4: lane 0 loads K, lane 1 loads V). Warp 5 issues the
// MMAs: S(t+1) goes out before P(t).V, so the scores of the next tile are
// ready when the softmax of this one ends. O^T accumulates in TMEM across
// the whole split. The softmax (warps 0-3, thread t = cache row t of the
// tile) keeps one max per head for the CTA and takes P = 2^(s - m) against
// it; m moves only when some row exceeds it by 2^8, and only then does the
// CTA reduce the tile's max and rescale O^T in TMEM and its row-sum
// partials. Each thread sums its own rows' P per head; the sums meet once,
// after the last tile.
//
// Prologue (RMSNorm with the reference's sequential sum, rotate-half RoPE
// from the host cos/sin table, the appended row) and the split merge are
// those of qx_decode_kernel (tools/qx-qwen-parity/src/main.rs:1170-1258).
//
// Granite with a 16-bit cache (group 2, head_dim 64) runs the same kernel
// on a pair of adjacent kv heads as one 128-dim unit: the K tile holds head
// 2u in dims 0-63 and head 2u+1 in dims 64-127, and Q^T is block-diagonal
// (query heads 4u, 4u+1 nonzero in dims 0-63 only, 4u+2, 4u+3 in dims
// 64-127 only), so one S^T MMA gives each query head its own kv head's
// scores. O^T = V^T.P^T then holds every (dim, head) product; each head's
// output is its own kv head's half of the dims and the rest is never read.
// The prologue is Granite's: qx's pinned RoPE (granite_rotate) on q and k,
// q rounded to the operand type for the MMA. This takes both contractions
// off the CUDA cores for every Granite cache whose keys and values are both
// bf16 or both f16; fp32 and mixed caches stay on qx_decode_kernel.
#pragma once
#include <type_traits>

#include "decode.cuh"
#include "qx_tc.cuh"

namespace qx {

// One work unit's geometry. D: dims of a unit's K/V row (MMA K of S, M of
// P.V); G: query heads per unit; UNITS: units per layer; HEAD_D: dims of
// one head; KV_PER_UNIT: kv heads in a unit.
struct TcQwen {
  static constexpr bool GRANITE = false;
  static constexpr int D = 128, G = 8, UNITS = 4, HQ = 32, HEAD_D = 128, KV_PER_UNIT = 1;
  static constexpr float SCALE_LOG2 = 0.08838834764831845f * 1.4426950408889634f;  // 1/sqrt(128) * log2(e)
};
struct TcGranitePair {
  static constexpr bool GRANITE = true;
  static constexpr int D = 128, G = 4, UNITS = 4, HQ = 16, HEAD_D = 64, KV_PER_UNIT = 2;
  static constexpr float SCALE_LOG2 = 0.015625f * 1.4426950408889634f;  // 1/64 * log2(e)
};

template <typename KT, class TM = TcQwen>
struct TcCfg {
  static constexpr int T = 128;  // cache rows per tile
  static constexpr int D = TM::D, G = TM::G, HKV = TM::UNITS, HQ = TM::HQ;
  static constexpr int NPAD = 16;        // MMA N (8 heads + 8 zero rows)
  static constexpr int BLK = T * 128;    // one 64-dim column block [128 rows][128 B]
  static constexpr int STAGE = 2 * BLK;  // K (or V) of one tile: 32 KB
  static constexpr int NS = 3;           // ring stages of K and of V
  static constexpr int OFF_K = 0;
  static constexpr int OFF_V = OFF_K + NS * STAGE;
  static constexpr int OFF_Q = OFF_V + NS * STAGE;             // 2 blocks [16 rows][128 B]
  static constexpr int OFF_P = OFF_Q + 2 * NPAD * 128;         // 2 buffers x 2 blocks [16 rows][128 B]
  static constexpr int OFF_RAW = OFF_P + 2 * 2 * NPAD * 128;   // f32 [(G + 1)][D]
  static constexpr int OFF_NEWK = OFF_RAW + (G + 1) * D * 4;
  static constexpr int OFF_NEWV = OFF_NEWK + D * 2;
  static constexpr int OFF_RED = OFF_NEWV + D * 2;         // f32 [4 warps][G], then u32 [2][4] flags
  static constexpr int OFF_STAT = OFF_RED + 4 * G * 4 + 32;  // f32 [2 * G]; inv [G + 1]
  static constexpr int OFF_BAR = ((OFF_STAT + 4 * (3 * G + 1) + 15) / 16) * 16;
  static constexpr int NBAR = 4 * NS + 2 + 2 + 2 + 4;
  static constexpr int SMEM = OFF_BAR + (NBAR + 2) * 8 + 1024;  // + TMEM slot and flags, + slack to align
  static constexpr int NT = 192;  // consumer warps 0-3, TMA warp 4, MMA warp 5
  static constexpr uint32_t TMEM_COLS = 64;  // S^T buffers [0,16) [16,32); O^T [32,48)
  static constexpr int FMT = std::is_same<KT, __nv_bfloat16>::value ? 1 : 0;  // MMA operand format
  static constexpr int MAX_SPLITS = 1024;
  static constexpr float TAU = 8.0f;  // base-2 headroom of the lazily moved max
  // Tiles (K and V) a CTA streams before griddepcontrol.wait. One tile pair,
  // 64 KB per SM, lands while the previous grids drain; with two or three the
  // prologue's loads after the wait queue behind the rest (config 3 on B200:
  // 17.3 us per call with one, 17.5 with two, 18.3 with none).
  static constexpr int PRE = 1;
};

template <typename KT, class TM = TcQwen>
__global__ void __launch_bounds__(192, 1) qx_decode_tc_kernel(const __grid_constant__ DecodeParams p) {
  using C = TcCfg<KT, TM>;
  constexpr int D = C::D, G = C::G, HKV = C::HKV, HQ = C::HQ, T = C::T, NS = C::NS;
  extern __shared__ __align__(1024) unsigned char sm_raw[];
  unsigned char* sm = sm_raw + ((1024u - (smem_addr(sm_raw) & 1023u)) & 1023u);
  float* raw = reinterpret_cast<float*>(sm + C::OFF_RAW);
  KT* newk = reinterpret_cast<KT*>(sm + C::OFF_NEWK);
  KT* newv = reinterpret_cast<KT*>(sm + C::OFF_NEWV);
  float* red = reinterpret_cast<float*>(sm + C::OFF_RED);  // [4][G]
  uint32_t* red_flag = reinterpret_cast<uint32_t*>(red + 4 * G);  // [tile parity][4 warps]
  float* stat = reinterpret_cast<float*>(sm + C::OFF_STAT);      // [2G] merge stats
  float* st_inv = stat + 2 * G;                                   // [G + 1]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + C::OFF_BAR);
  uint64_t* kfull = bars;           // [NS] K tile landed
  uint64_t* kempty = kfull + NS;    // [NS] S MMA done with the K stage
  uint64_t* vfull = kempty + NS;    // [NS] V tile landed
  uint64_t* vempty = vfull + NS;    // [NS] P.V MMA done with the V stage
  uint64_t* sfull = vempty + NS;    // [2] S^T in TMEM
  uint64_t* pfull = sfull + 2;      // [2] P^T written by the four consumer warps
  uint64_t* pdone = pfull + 2;      // [2] P.V of that P^T completed (buffer free, O^T current)
  uint64_t* qready = pdone + 2;     // Q in shared memory
  uint64_t* kpatch = qready + 1;    // the appended key is in its K stage
  uint64_t* mdone = kpatch + 1;     // every MMA completed
  uint64_t* loaded = mdone + 1;     // the prologue's global loads landed (the ring may start)
  uint32_t* tslot = reinterpret_cast<uint32_t*>(loaded + 1);
  int* s_flag = reinterpret_cast<int*>(loaded + 2);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  if (tid == 0) {
    for (int i = 0; i < 4 * NS; ++i) mbar_init(&bars[i], 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sfull[i], 1);
      mbar_init(&pfull[i], 4);
      mbar_init(&pdone[i], 1);
    }
    mbar_init(qready, 1);
    mbar_init(kpatch, 1);
    mbar_init(mdone, 1);
    mbar_init(loaded, 4);
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

  // Tile t of this CTA's split, K (lane 0) or V (lane 1): 4 boxes of
  // [64 rows][128 B] into ring stage t % NS, completing on its full barrier.
  auto issue_tile = [&](int t, int seq_id, int layer, int h, int begin, int end) {
    const CUtensorMap* map = lane == 0 ? &p.tmk : &p.tmv;
    uint64_t* full = lane == 0 ? kfull : vfull;
    unsigned char* ring = sm + (lane == 0 ? C::OFF_K : C::OFF_V);
    const int st = t % NS;
    mbar_arrive_expect_tx(&full[st], (uint32_t)C::STAGE);
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      // a box with no row of the split (the second half of a last tile of at
      // most 64 rows) reads the fill value from outside the tensor instead of
      // looking up a page past the sequence's block table
      const int slot = begin + t * T + half * 64;
      const int z = slot < end ? (int)kv_row(p.paging, p.capacity, p.layers, seq_id, layer, slot) : -128;
#pragma unroll
      for (int b = 0; b < 2; ++b) {
        // column block b: dims 64b.. of the kv head (Qwen), or kv head 2h+b (Granite pair)
        const int x = TM::KV_PER_UNIT == 1 ? b * 64 : 0, y = TM::KV_PER_UNIT == 1 ? h : 2 * h + b;
        tma_load_3d(ring + st * C::STAGE + b * C::BLK + half * 8192, map, x, y, z, &full[st]);
      }
    }
  };
  // The first C::PRE tiles, if all their rows lie below pre_rows, stream
  // before the wait while the previous grids drain (single-sequence calls:
  // the work item comes from the parameters, no memory read).
  int npre = 0;
  if (warp == 4 && lane < 2 && p.seq_table == nullptr && p.paging.table == nullptr && p.pre_rows > 0) {
    const SeqInfo& s0 = p.single;
    const int ns = (s0.attend + p.chunk - 1) / p.chunk;
    int r0 = blockIdx.x - s0.item_begin;
    const int l0 = r0 / (HKV * ns);
    r0 -= l0 * HKV * ns;
    const int h0 = r0 / ns, b0 = (r0 - h0 * ns) * p.chunk;
    const int e0 = min(b0 + p.chunk, s0.attend);
    const int n0 = (e0 - b0 + T - 1) / T;
    prefetch_tmap(lane == 0 ? &p.tmk : &p.tmv);
    while (npre < C::PRE && npre < n0 && min(b0 + (npre + 1) * T, e0) <= p.pre_rows) {
      issue_tile(npre, s0.seq_id, p.layer_begin + l0, h0, b0, e0);
      ++npre;
    }
  }
  // launched as a programmatic dependent: everything above overlapped the
  // previous grid; from here on its memory is visible
  pdl_wait();
  // the merge grid (or the next call) may get resident meanwhile; only now,
  // so that a grid launched early never overlaps one that still writes rows
  if (p.early_trigger) pdl_launch_dependents();
  SeqInfo si;
  const int slot = find_slot(p, &si);
  const int nsplit = (si.attend + p.chunk - 1) / p.chunk;
  int r = blockIdx.x - si.item_begin;
  const int lloc = r / (HKV * nsplit);
  r -= lloc * HKV * nsplit;
  const int h = r / nsplit;
  const int s = r - h * nsplit;
  const int layer = p.layer_begin + lloc;
  const int begin = s * p.chunk;
  const int end = min(begin + p.chunk, si.attend);
  const bool has_new = si.new_slot >= begin && si.new_slot < end;
  const int ntiles = (end - begin + T - 1) / T;
  const long long cu = (long long)slot * p.layer_count + lloc;
  const bool last_split = (s == nsplit - 1);
  const int last_rows = end - (begin + (ntiles - 1) * T);  // rows of the last tile

  const uint32_t tbase = *tslot;
  StageTrace trace(p.trace, blockIdx.x, tid == 0);
  trace.mark();  // TMEM allocated
  bool ok = true;

  if (warp == 4) {
    // ---- TMA producers: lane 0 streams K tiles, lane 1 V tiles (4 boxes of [64 rows][128 B] each)
    if (lane < 2) {
      uint64_t* full = lane == 0 ? kfull : vfull;
      uint64_t* empty = lane == 0 ? kempty : vempty;
      if (npre == 0) prefetch_tmap(lane == 0 ? &p.tmk : &p.tmv);
      // the prologue's few loads go first: behind the ring's ~200 KB per SM
      // they would wait for most of it
      ok &= mbar_wait_bounded(loaded, 0, p.err);
      for (int t = npre; t < ntiles; ++t) {
        if (t >= NS) ok &= mbar_wait_bounded(&empty[t % NS], (uint32_t)(t / NS - 1) & 1u, p.err);
        issue_tile(t, si.seq_id, layer, h, begin, end);
      }
      // no copy may still be landing when the CTA exits
      for (int t = ntiles > NS ? ntiles - NS : 0; t < ntiles; ++t)
        ok &= mbar_wait_bounded(&full[t % NS], (uint32_t)(t / NS) & 1u, p.err);
    }
  } else if (warp == 5) {
    // ---- MMA issuer ----------------------------------------------------------
    if (lane == 0) {
      constexpr uint32_t IDESC_S = umma_idesc_16bit(128, C::NPAD, C::FMT, false, false);
      constexpr uint32_t IDESC_PV = umma_idesc_16bit(128, C::NPAD, C::FMT, true, false);
      const uint32_t sQ = smem_addr(sm + C::OFF_Q), sP = smem_addr(sm + C::OFF_P);
      const uint32_t sK = smem_addr(sm + C::OFF_K), sV = smem_addr(sm + C::OFF_V);
      ok &= mbar_wait_bounded(qready, 0, p.err);
      // S^T(t) into buffer t & 1: its previous reader, the softmax of t-2,
      // finished before P(t-2) was handed over, i.e. before P(t-2).V issued
      auto issue_s = [&](int t) {
        const int st = t % NS, b = t & 1;
        ok &= mbar_wait_bounded(&kfull[st], (uint32_t)(t / NS) & 1u, p.err);
        if (has_new && t == ntiles - 1) ok &= mbar_wait_bounded(kpatch, 0, p.err);
        tc_fence_after();
        const uint32_t kb = sK + st * C::STAGE;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          tc_mma_bf16(tbase + 16 * b, umma_desc_sw128(kb + (kk >> 2) * C::BLK + (kk & 3) * 32, 16, 1024),
                      umma_desc_sw128(sQ + (kk >> 2) * 2048 + (kk & 3) * 32, 16, 1024), IDESC_S, kk > 0);
        tc_commit(&sfull[b]);
        tc_commit(&kempty[st]);
      };
      // O^T += V^T(t) . P^T(t)
      auto issue_pv = [&](int t) {
        const int st = t % NS, b = t & 1;
        ok &= mbar_wait_bounded(&pfull[b], (uint32_t)(t >> 1) & 1u, p.err);
        ok &= mbar_wait_bounded(&vfull[st], (uint32_t)(t / NS) & 1u, p.err);
        tc_fence_after();
        const uint32_t vb = sV + st * C::STAGE, pb = sP + b * 2 * 2048;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          tc_mma_bf16(tbase + 32, umma_desc_sw128(vb + kk * 2048, C::BLK, 1024),
                      umma_desc_sw128(pb + (kk >> 2) * 2048 + (kk & 3) * 32, 16, 1024), IDESC_PV,
                      (t > 0 || kk > 0) ? 1u : 0u);
        tc_commit(&pdone[b]);
        tc_commit(&vempty[st]);
      };
      issue_s(0);
      for (int t = 0; t < ntiles; ++t) {
        if (t + 1 < ntiles) issue_s(t + 1);
        issue_pv(t);
      }
      tc_commit(mdone);  // TMEM is released only after every MMA completed
      ok &= mbar_wait_bounded(mdone, 0, p.err);
    }
    if (!ok) s_flag[1] = 1;
  } else {
    // ---- consumers: prologue, one round of global loads --------------------
    const long long qbase = (cu * HQ + (long long)h * G) * TM::HEAD_D;
    const long long kvbase = (cu * HKV + h) * D;  // the unit's new k/v row
    bool bad = false;
    if constexpr (TM::GRANITE) {
      // thread t: rotation pair i of query head slot j (and of kv head slot
      // j < 2 of the new key); dim t of the new value row
      const int j = tid >> 5, i = tid & 31;
      const long long qa = qbase + j * 64 + i;
      const float ql = load_any(p.q, qa, p.q_dtype), qr = load_any(p.q, qa + 32, p.q_dtype);
      float kl = 0.0f, kr = 0.0f, vnew = 0.0f;
      if (has_new) {
        if (tid < 64) {
          kl = load_any(p.k, kvbase + j * 64 + i, p.in_dtype);
          kr = load_any(p.k, kvbase + j * 64 + i + 32, p.in_dtype);
        }
        vnew = load_any(p.v, kvbase + tid, p.in_dtype);
      }
      {
        const float sink = ql + qr + kl + kr + vnew;  // every load above has landed
        asm volatile("" ::"f"(sink));
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(loaded);
      trace.mark();  // prologue loads landed
      // Q^T is block-diagonal: zero all of it, and the padding rows G..15 of
      // both P^T buffers (both column blocks)
      for (int w = tid; w < 256 + 4 * (16 - G) * 8; w += 128) {
        unsigned char* dst = w < 256 ? sm + C::OFF_Q + w * 16
                                     : sm + C::OFF_P + ((w - 256) / ((16 - G) * 8)) * 2048 + G * 128 +
                                           ((w - 256) % ((16 - G) * 8)) * 16;
        *reinterpret_cast<uint4*>(dst) = make_uint4(0u, 0u, 0u, 0u);
      }
      consumers_sync(128);
      trace.mark();  // (no norms)
      float sn = 0.f, cs = 0.f, a = 0.f, b = 0.f;
      bool ok = granite_sin_cos((uint32_t)si.rope_pos, i, &sn, &cs) && granite_rotate(ql, qr, sn, cs, &a, &b);
      bad |= !ok;
      // query head slot j is row j of Q^T, in column block j >> 1 (its kv head's dims)
      unsigned char* qrow = sm + C::OFF_Q + (j >> 1) * 2048 + j * 128;
      *reinterpret_cast<KT*>(qrow + (((i >> 3) ^ j) << 4) + (i & 7) * 2) = Elem<KT>::from_f32(a);
      *reinterpret_cast<KT*>(qrow + ((((i >> 3) + 4) ^ j) << 4) + (i & 7) * 2) = Elem<KT>::from_f32(b);
      if (p.q_rot_out && last_split) {
        p.q_rot_out[qa] = a;
        p.q_rot_out[qa + 32] = b;
      }
      if (has_new) {
        if (tid < 64) {
          ok = granite_rotate(kl, kr, sn, cs, &a, &b);
          bad |= !ok;
          newk[j * 64 + i] = Elem<KT>::from_f32(a);
          newk[j * 64 + i + 32] = Elem<KT>::from_f32(b);
        }
        newv[tid] = Elem<KT>::from_f32(vnew);
      }
    } else {
      const int pi = tid & 63;  // the rotation pair of every prologue item of this thread
      // all of this thread's prologue inputs in flight at once: dim tid of the
      // G query rows (and of the new key row), its RoPE pair, norm weights, new v
      float qv[G], kn = 0.0f, vnew = 0.0f;
      load_any_n<G>(p.q, qbase + tid, D, p.q_dtype, qv);
      if (has_new) {
        load_any_n<1>(p.k, kvbase + tid, 0, p.in_dtype, &kn);
        load_any_n<1>(p.v, kvbase + tid, 0, p.in_dtype, &vnew);
      }
      const float2 cssn = p.rope_table[(long long)si.rope_pos * 64 + pi];
      const float wq0 = p.q_norm ? p.q_norm[pi] : 1.0f, wq1 = p.q_norm ? p.q_norm[64 + pi] : 1.0f;
      const float wk0 = p.k_norm ? p.k_norm[pi] : 1.0f, wk1 = p.k_norm ? p.k_norm[64 + pi] : 1.0f;
#pragma unroll
      for (int g = 0; g < G; ++g) raw[g * D + tid] = qv[g];
      raw[G * D + tid] = kn;
      {
        // every load above has landed once its value is used
        const float sink = cssn.x + wq0 + wq1 + wk0 + wk1 + vnew;
        asm volatile("" ::"f"(sink));
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(loaded);
      trace.mark();  // prologue loads landed
      // zero the padding rows 8..15 of Q and of both P^T buffers (both column blocks)
      for (int i = tid; i < 6 * 128; i += 128) {
        const int blk = i >> 7, j = i & 127;  // blk 0,1: Q blocks; 2..5: P blocks
        unsigned char* base = sm + (blk < 2 ? C::OFF_Q + blk * 2048 : C::OFF_P + (blk - 2) * 2048) + 1024;
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
      trace.mark();  // RMS norms
      for (int idx = tid; idx < (G + 1) * 64; idx += 128) {
        const int g = idx >> 6;
        if (g == G && !has_new) break;
        const bool is_q = g < G;
        const float inv = st_inv[g];
        const float x = raw[g * D + pi], y = raw[g * D + pi + 64];
        const float left = __fmul_rn(__fmul_rn(x, inv), is_q ? wq0 : wk0);
        const float right = __fmul_rn(__fmul_rn(y, inv), is_q ? wq1 : wk1);
        const float a = __fsub_rn(__fmul_rn(left, cssn.x), __fmul_rn(right, cssn.y));
        const float b = __fadd_rn(__fmul_rn(right, cssn.x), __fmul_rn(left, cssn.y));
        bad |= !(isfinite(a) && isfinite(b));
        const KT ka = Elem<KT>::from_f32(a), kb = Elem<KT>::from_f32(b);
        if (is_q) {
          // Q row g (K-major, 128-byte swizzle): dims pi and pi+64 in blocks 0 and 1
          const int c = pi >> 3, off = (pi & 7) * 2;
          *reinterpret_cast<KT*>(sm + C::OFF_Q + g * 128 + ((c ^ (g & 7)) << 4) + off) = ka;
          *reinterpret_cast<KT*>(sm + C::OFF_Q + 2048 + g * 128 + ((c ^ (g & 7)) << 4) + off) = kb;
          if (p.q_rot_out && last_split) {
            p.q_rot_out[qbase + g * D + pi] = Elem<KT>::to_f32(ka);
            p.q_rot_out[qbase + g * D + pi + 64] = Elem<KT>::to_f32(kb);
          }
        } else {
          newk[pi] = ka;
          newk[pi + 64] = kb;
        }
      }
      if (has_new) newv[tid] = Elem<KT>::from_f32(vnew);
    }
    if (bad) flag_error(p.err, QX_ERR_BIT_NONFINITE);
    fence_proxy_async_shared();  // Q and the P padding are read by tcgen05.mma
    consumers_sync(128);
    if (tid == 0) mbar_arrive(qready);
    if (has_new) {
      const long long row = kv_row(p.paging, p.capacity, p.layers, si.seq_id, layer, si.new_slot);
      char* kdst = p.k_region + (row * HKV + h) * (D * 2);
      char* vdst = p.v_region + (row * HKV + h) * (D * 2);
      if (tid < 16) reinterpret_cast<uint4*>(kdst)[tid] = reinterpret_cast<const uint4*>(newk)[tid];
      else if (tid < 32) reinterpret_cast<uint4*>(vdst)[tid - 16] = reinterpret_cast<const uint4*>(newv)[tid - 16];
    }
    trace.mark();  // prologue done

    // ---- consumers: tiles ----------------------------------------------------
    const bool pinned = p.pinned_exp != 0;
    constexpr float SCALE_LOG2 = TM::SCALE_LOG2;
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    unsigned char* kring = sm + C::OFF_K;
    unsigned char* vring = sm + C::OFF_V;
    float m_run[G], l_part[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      m_run[g] = -INFINITY;
      l_part[g] = 0.0f;
    }
    // P^T column tid (a cache row) of head g: K-major, 128-byte swizzle
    const int pb = tid >> 6, pc = (tid & 63) >> 3, poff = (tid & 7) * 2;
    for (int t = 0; t < ntiles; ++t) {
      const int b = t & 1, st = t % NS;
      const bool last = t == ntiles - 1;
      const int rows = last ? last_rows : T;
      if (last && has_new) {
        // the appended key comes from registers, not from the copy
        ok &= mbar_wait_bounded(&kfull[st], (uint32_t)(t / NS) & 1u, p.err);
        if (tid < 16)
          *reinterpret_cast<uint4*>(kring + st * C::STAGE + swz<C::BLK>(rows - 1, tid * 16)) =
              reinterpret_cast<const uint4*>(newk)[tid];
        fence_proxy_async_shared();
        consumers_sync(128);
        if (tid == 0) mbar_arrive(kpatch);
      }
      ok &= mbar_wait_bounded(&sfull[b], (uint32_t)(t >> 1) & 1u, p.err);
      __syncwarp();
      tc_fence_after();
      float x[8];  // columns G..7 hold zero-padding scores
      tmem_ld8_sync(tbase + lane_base + 16 * b, x);
#pragma unroll
      for (int g = 0; g < G; ++g) x[g] = tid < rows ? x[g] * SCALE_LOG2 : -INFINITY;
      trace.mark();  // tile: scores read
      // does any row raise a head's max past its headroom?
      uint32_t raise = 0;
#pragma unroll
      for (int g = 0; g < G; ++g) raise |= (x[g] > m_run[g] + C::TAU ? 1u : 0u) << g;
      raise = __reduce_or_sync(0xffffffffu, raise);
      // (two flag sets: a warp may write tile t+1's while another still reads tile t's)
      uint32_t* flags = red_flag + 4 * b;
      if (lane == 0) flags[warp] = raise;
      consumers_sync(128);
      raise = flags[0] | flags[1] | flags[2] | flags[3];
      if (raise) {
        // the tile's max of the raised heads, then O^T and the row sums
        // rescaled to it (once the previous P.V has landed in O^T)
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float wm = warp_max(x[g]);
          if (lane == 0) red[warp * G + g] = wm;
        }
        consumers_sync(128);
        float alpha[G];
#pragma unroll
        for (int g = 0; g < G; ++g) {
          alpha[g] = 1.0f;
          if (raise & (1u << g)) {
            const float tmax = fmaxf(fmaxf(red[g], red[G + g]), fmaxf(red[2 * G + g], red[3 * G + g]));
            alpha[g] = m_run[g] == -INFINITY ? 0.0f : fast_exp2(m_run[g] - tmax);
            m_run[g] = tmax;
          }
          l_part[g] *= alpha[g];
        }
        if (t > 0) {
          ok &= mbar_wait_bounded(&pdone[(t - 1) & 1], (uint32_t)((t - 1) >> 1) & 1u, p.err);
          __syncwarp();
          tc_fence_after();
          float o[8];
          tmem_ld8_sync(tbase + lane_base + 32, o);  // thread tid = dim tid of the unit, 8 columns
#pragma unroll
          for (int g = 0; g < G; ++g) o[g] *= alpha[g];
          tmem_st8(tbase + lane_base + 32, o);
          tmem_wait_st();
          tc_fence_before();
        }
        consumers_sync(128);  // red[] is rewritten by the next raise
      }
      // P^T buffer b was last read by P(t-2).V
      if (t >= 2) ok &= mbar_wait_bounded(&pdone[b], (uint32_t)((t - 2) >> 1) & 1u, p.err);
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const KT pw = Elem<KT>::from_f32(fast_exp2(x[g] - m_run[g]));
        l_part[g] += Elem<KT>::to_f32(pw);  // the sum of exactly the P the MMA sees
        *reinterpret_cast<KT*>(sm + C::OFF_P + b * 4096 + pb * 2048 + g * 128 + ((pc ^ (g & 7)) << 4) + poff) = pw;
      }
      if (last) {
        // rows past the cache end carry zero probability; zero their values
        // so the tensor core never multiplies 0 by a stale non-finite element
        ok &= mbar_wait_bounded(&vfull[st], (uint32_t)(t / NS) & 1u, p.err);
        unsigned char* vt = vring + st * C::STAGE;
        if (has_new && tid < 16)
          *reinterpret_cast<uint4*>(vt + swz<C::BLK>(rows - 1, tid * 16)) = reinterpret_cast<const uint4*>(newv)[tid];
        for (int i = tid; i < (T - rows) * 16; i += 128) {
          const int rr = rows + (i >> 4);
          *reinterpret_cast<uint4*>(vt + swz<C::BLK>(rr, (i & 15) * 16)) = make_uint4(0u, 0u, 0u, 0u);
        }
      }
      fence_proxy_async_shared();  // P^T (and the patched V) are read by tcgen05.mma
      __syncwarp();
      if (lane == 0) mbar_arrive(&pfull[b]);
      trace.mark();  // tile: P written
    }
    // O^T of the split (thread tid = dim tid, 8 heads) once the last P.V landed
    ok &= mbar_wait_bounded(&pdone[(ntiles - 1) & 1], (uint32_t)((ntiles - 1) >> 1) & 1u, p.err);
    __syncwarp();
    tc_fence_after();
    float O[8];
    tmem_ld8_sync(tbase + lane_base + 32, O);
    // the row-sum partials of the four warps
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float ws = warp_sum(l_part[g]);
      if (lane == 0) red[warp * G + g] = ws;
    }
    consumers_sync(128);
    float Mg[G], Lg[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      Mg[g] = m_run[g] / 1.4426950408889634f;  // back to the natural-log domain of the partials
      Lg[g] = (red[g] + red[G + g]) + (red[2 * G + g] + red[3 * G + g]);
    }
    if (!ok) s_flag[1] = 1;
    tc_fence_before();
    cta_sync();  // (A) with the TMA and MMA warps
    if (warp == 0) {
      tc_fence_after();
      tmem_dealloc(tbase, C::TMEM_COLS);
    }
    if (s_flag[1]) return;
    trace.mark();  // tiles done
    if constexpr (TM::GRANITE) {
      // Lane tid of O^T holds dim tid & 63 of kv head slot a = tid >> 6 for
      // query head slots 2a and 2a+1 (its own kv head's heads; the other
      // columns are cross products). finish_outputs wants thread tid to hold
      // dim tid & 63 of heads a and a + 2: trade through shared memory.
      float* xs = raw;  // [G][64]
      const int a = tid >> 6, d = tid & 63;
      xs[(2 * a) * 64 + d] = a ? O[2] : O[0];
      xs[(2 * a + 1) * 64 + d] = a ? O[3] : O[1];
      consumers_sync(128);
      float O2[2], M2[2], L2[2];
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int g = a + 2 * k;
        O2[k] = xs[g * 64 + d];
        M2[k] = a ? Mg[1 + 2 * k] : Mg[2 * k];
        L2[k] = a ? Lg[1 + 2 * k] : Lg[2 * k];
      }
      finish_outputs<G, TM::HEAD_D, HKV, HQ, 2>(p, O2, M2, L2, nsplit, s, cu, h, tid, warp, lane, pinned,
                                                reinterpret_cast<float*>(sm + C::OFF_K), stat, s_flag);
    } else if (p.slice_merge && nsplit > 1) {
      slice_merge<G, D, HQ>(p, O, Mg, Lg, nsplit, s, cu, h, tid, pinned, reinterpret_cast<float*>(sm + C::OFF_K));
    } else {
      finish_outputs<G, D, HKV, HQ, G>(p, O, Mg, Lg, nsplit, s, cu, h, tid, warp, lane, pinned,
                                       reinterpret_cast<float*>(sm + C::OFF_K), stat, s_flag);
    }
    trace.mark();  // outputs (or partials) written
    return;
  }
  tc_fence_before();
  cta_sync();  // (A) for the TMA and MMA warps
}

}  // namespace qx
