// decode.cuh — split-KV flash decode for qx's GQA attention on sm_100a.
//
// One CTA per work item (sequence, layer, kv head, split of the cache). The
// CTA
//   1. issues TMA bulk copies (cp.async.bulk, one per cache row of its kv
//      head; the cache keeps the reference's position-major layout
//      [pos][kv_head][head_dim]) into a multi-stage shared-memory ring, with
//      an mbarrier per stage, before doing anything else;
//   2. meanwhile applies RoPE to the G query heads that share this kv head
//      (Granite: qx's pinned sin/cos and FMA order, qx-consensus-math
//      lib.rs:148-207; Qwen: per-head RMSNorm then rotate-half RoPE,
//      qx-qwen-parity main.rs:1177-1204), and, on the split that owns the
//      new token, RoPE on k, writing k and v into slot `position` and into
//      its own last tile (so no CTA ever reads the slot being written);
//   3. streams tiles of 64 positions: scores for all G heads against each
//      key row held once in shared memory, a tile-wise online softmax with
//      warp-shuffle max/sum, and P.V accumulation in registers;
//   4. writes its (m, l, O) partial; the last CTA of the (sequence, layer,
//      kv head) to finish (atomic ticket, no spinning) merges the partials
//      with a log-sum-exp combine and writes the output.
//
// Reference semantics: crates/qx-runtime/src/lib.rs:464-552
// (granite_attention_decode_with_profile) for Granite, and
// tools/qx-qwen-parity/src/main.rs:1170-1258 for Qwen3.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "qx_math.cuh"
#include "qx_ptx.cuh"

namespace qx {

struct Granite {
  static constexpr int HQ = 16, HKV = 8, D = 64, G = 2;
  static constexpr bool QWEN = false;
  static constexpr float SCALE = 0.015625f;  // ATTENTION_MULTIPLIER, qx-model lib.rs:20
};
struct Qwen3 {
  static constexpr int HQ = 32, HKV = 4, D = 128, G = 8;
  static constexpr bool QWEN = true;
  static constexpr float SCALE = 0.08838834764831845f;  // 1/sqrt(128)
};

// Per-sequence entry of one call.
struct SeqInfo {
  int seq_id;      // sequence index in the arena
  int attend;      // slots attended: [0, attend)
  int new_slot;    // slot receiving the new token (== attend-1), or -1
  int rope_pos;    // absolute position used for the RoPE angle
  int item_begin;  // first work item of this sequence in the grid
  int pad[3];
};

struct DecodeParams {
  // arena
  char* k_region;
  char* v_region;
  long long k_unit_bytes;  // one (sequence, layer) key cache
  long long v_unit_bytes;
  int layers;
  // call
  int layer_begin, layer_count, n_seq;
  const SeqInfo* seq_table;  // device [n_seq], or nullptr to use `single`
  SeqInfo single;
  int chunk;  // positions per split, multiple of 64
  const void* q;
  const void* k;
  const void* v;
  void* out;
  float* q_rot_out;
  const float* q_norm;
  const float* k_norm;
  const float2* rope_table;  // Qwen: [absolute position][64] (cos, sin)
  int q_dtype, in_dtype, out_dtype;
  int pinned_exp;
  int emit_partials;  // write (O, m, l) per query head instead of O / l
  float* partials;    // scratch [items][G][D+2]
  int* tickets;       // scratch [n_seq][layer_count][HKV], zero between calls
  unsigned* err;
};

template <class M, typename KT, typename VT>
struct DecodeCfg {
  static constexpr int T = 64, NT = 128;
  static constexpr int D = M::D, G = M::G;
  static constexpr int KROW = D * (int)sizeof(KT), VROW = D * (int)sizeof(VT);
  // 16-byte row padding: consecutive rows start 4 banks apart, so the
  // 8 rows a 128-bit shared load wavefront touches never collide.
  static constexpr int KSTR = KROW + 16, VSTR = VROW + 16;
  static constexpr int STAGE_BYTES = T * (KSTR + VSTR);
  static constexpr int STAGES = STAGE_BYTES <= 20480 ? 4 : 3;
  static constexpr int OFF_K = 0;
  static constexpr int OFF_V = OFF_K + STAGES * T * KSTR;
  static constexpr int OFF_Q = OFF_V + STAGES * T * VSTR;   // float [G][D]
  static constexpr int OFF_S = OFF_Q + G * D * 4;            // float [T][G]
  static constexpr int OFF_NEWK = OFF_S + T * G * 4;         // KT [D]
  static constexpr int OFF_NEWV = OFF_NEWK + ((KROW + 15) / 16) * 16;
  static constexpr int OFF_STAT = OFF_NEWV + ((VROW + 15) / 16) * 16;  // float m[G], l[G], a[G], inv[G+1]
  static constexpr int OFF_BAR = ((OFF_STAT + 4 * (4 * G + 1) + 15) / 16) * 16;
  static constexpr int SMEM = OFF_BAR + 8 * STAGES + 16;
  static constexpr int HPT = G / 2;   // query heads per thread in QK and PV
  static constexpr int DPT = D / 64;  // dims per thread in PV
};

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Locate this CTA's sequence entry (binary search over item_begin).
__device__ __forceinline__ int find_slot(const DecodeParams& p, SeqInfo* info) {
  if (p.seq_table == nullptr) {
    *info = p.single;
    return 0;
  }
  int lo = 0, hi = p.n_seq - 1;
  const int item = blockIdx.x;
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if (p.seq_table[mid].item_begin <= item) lo = mid;
    else hi = mid - 1;
  }
  *info = p.seq_table[lo];
  return lo;
}

template <class M, typename KT, typename VT>
__global__ void __launch_bounds__(128) qx_decode_kernel(const DecodeParams p) {
  using C = DecodeCfg<M, KT, VT>;
  constexpr int D = M::D, G = M::G, HKV = M::HKV, HQ = M::HQ, T = C::T, NT = C::NT;
  constexpr int HPT = C::HPT, DPT = C::DPT, STAGES = C::STAGES;
  extern __shared__ __align__(128) unsigned char sm[];
  unsigned char* ktiles = sm + C::OFF_K;
  unsigned char* vtiles = sm + C::OFF_V;
  float* q_s = reinterpret_cast<float*>(sm + C::OFF_Q);
  float* S = reinterpret_cast<float*>(sm + C::OFF_S);
  KT* newk = reinterpret_cast<KT*>(sm + C::OFF_NEWK);
  VT* newv = reinterpret_cast<VT*>(sm + C::OFF_NEWV);
  float* st_m = reinterpret_cast<float*>(sm + C::OFF_STAT);
  float* st_l = st_m + G;
  float* st_a = st_l + G;
  float* st_inv = st_a + G;  // [G + 1]: Qwen inverse RMS of q heads, then k
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + C::OFF_BAR);
  int* s_flag = reinterpret_cast<int*>(bars + STAGES);

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  // ---- work item ---------------------------------------------------------
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
  const bool has_new = si.new_slot >= begin && si.new_slot < end;  // last split only
  const int ntiles = (end - begin + T - 1) / T;
  const long long cu = (long long)slot * p.layer_count + lloc;  // packed q/k/v/out index
  const bool last_split = (s == nsplit - 1);

  // ---- barriers, then the first tiles in flight ----------------------------
  if (tid == 0) {
#pragma unroll
    for (int i = 0; i < STAGES; ++i) mbar_init(&bars[i], 1);
    fence_barrier_init();
  }
  __syncthreads();

  auto issue = [&](int tile) {  // warp 0
    const int st = tile % STAGES;
    const int t0 = begin + tile * T;
    const int rows = min(T, end - t0);
    const int fetch = rows - ((has_new && tile == ntiles - 1) ? 1 : 0);
    if (lane == 0) mbar_arrive_expect_tx(&bars[st], (uint32_t)fetch * (C::KROW + C::VROW));
    __syncwarp();
    unsigned char* kt = ktiles + st * T * C::KSTR;
    unsigned char* vt = vtiles + st * T * C::VSTR;
    for (int rr = lane; rr < fetch; rr += 32) {
      const long long row = (long long)(t0 + rr) * HKV + h;
      bulk_copy_g2s(kt + rr * C::KSTR, kunit + row * C::KROW, C::KROW, &bars[st]);
      bulk_copy_g2s(vt + rr * C::VSTR, vunit + row * C::VROW, C::VROW, &bars[st]);
    }
  };
  if (warp == 0) {
    const int first = min(STAGES, ntiles);
    for (int i = 0; i < first; ++i) issue(i);
  }

  // ---- prologue: RoPE (and the new k/v row on the owning split) -------------
  const long long qbase = (cu * HQ + (long long)h * G) * D;  // first query element of this group
  const long long kvbase = (cu * HKV + h) * D;
  bool bad = false;
  if constexpr (!M::QWEN) {
    // 32 rotation pairs per head; warps 0-1 take the G=2 query heads, warp 2 k.
    if (tid < G * 32) {
      const int g = tid >> 5, pair = tid & 31;
      float left = load_any(p.q, qbase + g * D + pair, p.q_dtype);
      float right = load_any(p.q, qbase + g * D + pair + 32, p.q_dtype);
      float sn, cs, a = 0.f, b = 0.f;
      bool ok = granite_sin_cos((uint32_t)si.rope_pos, pair, &sn, &cs) && granite_rotate(left, right, sn, cs, &a, &b);
      bad |= !ok;
      q_s[g * D + pair] = a;
      q_s[g * D + pair + 32] = b;
      if (p.q_rot_out && last_split) {
        p.q_rot_out[qbase + g * D + pair] = a;
        p.q_rot_out[qbase + g * D + pair + 32] = b;
      }
    } else if (has_new && tid < G * 32 + 32) {
      const int pair = tid - G * 32;
      float left = load_any(p.k, kvbase + pair, p.in_dtype);
      float right = load_any(p.k, kvbase + pair + 32, p.in_dtype);
      float sn, cs, a = 0.f, b = 0.f;
      bool ok = granite_sin_cos((uint32_t)si.rope_pos, pair, &sn, &cs) && granite_rotate(left, right, sn, cs, &a, &b);
      bad |= !ok;
      newk[pair] = Elem<KT>::from_f32(a);
      newk[pair + 32] = Elem<KT>::from_f32(b);
    }
  } else {
    // Per-head RMSNorm needs the reference's sequential sum of squares
    // (bit-exact K); one thread per head.
    if (tid < G || (tid == G && has_new)) {
      const bool is_q = tid < G;
      float sum = 0.0f;
      for (int i = 0; i < D; ++i) {
        float x = is_q ? load_any(p.q, qbase + tid * D + i, p.q_dtype) : load_any(p.k, kvbase + i, p.in_dtype);
        sum = __fadd_rn(sum, __fmul_rn(x, x));
      }
      st_inv[tid] = __frcp_rn(__fsqrt_rn(__fadd_rn(__fdiv_rn(sum, 128.0f), 1.0e-6f)));
    }
    __syncthreads();
    const float2* tab = p.rope_table + (long long)si.rope_pos * 64;
    for (int idx = tid; idx < (G + 1) * 64; idx += NT) {
      const int g = idx >> 6, i = idx & 63;
      if (g == G && !has_new) break;
      const bool is_q = g < G;
      const float inv = st_inv[g];
      const float* wn = is_q ? p.q_norm : p.k_norm;
      float x = is_q ? load_any(p.q, qbase + g * D + i, p.q_dtype) : load_any(p.k, kvbase + i, p.in_dtype);
      float y = is_q ? load_any(p.q, qbase + g * D + i + 64, p.q_dtype) : load_any(p.k, kvbase + i + 64, p.in_dtype);
      float left = __fmul_rn(__fmul_rn(x, inv), wn ? wn[i] : 1.0f);
      float right = __fmul_rn(__fmul_rn(y, inv), wn ? wn[64 + i] : 1.0f);
      const float2 cssn = tab[i];
      float a = __fsub_rn(__fmul_rn(left, cssn.x), __fmul_rn(right, cssn.y));
      float b = __fadd_rn(__fmul_rn(right, cssn.x), __fmul_rn(left, cssn.y));
      bad |= !(isfinite(a) && isfinite(b));
      if (is_q) {
        // the reference rounds the rotated query to its 16-bit type
        a = Elem<KT>::to_f32(Elem<KT>::from_f32(a));
        b = Elem<KT>::to_f32(Elem<KT>::from_f32(b));
        q_s[g * D + i] = a;
        q_s[g * D + i + 64] = b;
        if (p.q_rot_out && last_split) {
          p.q_rot_out[qbase + g * D + i] = a;
          p.q_rot_out[qbase + g * D + i + 64] = b;
        }
      } else {
        newk[i] = Elem<KT>::from_f32(a);
        newk[i + 64] = Elem<KT>::from_f32(b);
      }
    }
  }
  if (has_new) {
    for (int i = tid; i < D; i += NT) newv[i] = Elem<VT>::from_f32(load_any(p.v, kvbase + i, p.in_dtype));
  }
  if (tid < G) {
    st_m[tid] = -INFINITY;
    st_l[tid] = 0.0f;
  }
  if (bad) flag_error(p.err, QX_ERR_BIT_NONFINITE);
  __syncthreads();
  if (has_new) {
    // Append: slot new_slot of this kv head, same bits the tile will use.
    char* kdst = const_cast<char*>(kunit) + ((long long)si.new_slot * HKV + h) * C::KROW;
    char* vdst = const_cast<char*>(vunit) + ((long long)si.new_slot * HKV + h) * C::VROW;
    for (int i = tid; i < C::KROW / 16; i += NT)
      reinterpret_cast<uint4*>(kdst)[i] = reinterpret_cast<const uint4*>(newk)[i];
    for (int i = tid; i < C::VROW / 16; i += NT)
      reinterpret_cast<uint4*>(vdst)[i] = reinterpret_cast<const uint4*>(newv)[i];
  }

  // ---- main loop over tiles -------------------------------------------------
  const int hg = tid >> 6, t_own = tid & 63, dg = tid & 63;
  float acc[HPT][DPT];
#pragma unroll
  for (int j = 0; j < HPT; ++j)
#pragma unroll
    for (int e = 0; e < DPT; ++e) acc[j][e] = 0.0f;
  const bool pinned = p.pinned_exp != 0;

  for (int tile = 0; tile < ntiles; ++tile) {
    const int st = tile % STAGES;
    const uint32_t parity = (uint32_t)(tile / STAGES) & 1u;
    const bool ok = mbar_wait_bounded(&bars[st], parity, p.err);
    if (__syncthreads_or(!ok)) return;  // bounded wait gave up; error recorded
    const int t0 = begin + tile * T;
    const int rows = min(T, end - t0);
    unsigned char* kt = ktiles + st * T * C::KSTR;
    unsigned char* vt = vtiles + st * T * C::VSTR;
    if (has_new && tile == ntiles - 1) {
      for (int i = tid; i < C::KROW / 16; i += NT)
        reinterpret_cast<uint4*>(kt + (rows - 1) * C::KSTR)[i] = reinterpret_cast<const uint4*>(newk)[i];
      for (int i = tid; i < C::VROW / 16; i += NT)
        reinterpret_cast<uint4*>(vt + (rows - 1) * C::VSTR)[i] = reinterpret_cast<const uint4*>(newv)[i];
      __syncthreads();
    }
    // scores: thread (position t_own, heads hg*HPT .. +HPT)
    {
      float sc[HPT];
#pragma unroll
      for (int j = 0; j < HPT; ++j) sc[j] = 0.0f;
      if (t_own < rows) {
        const KT* krow = reinterpret_cast<const KT*>(kt + t_own * C::KSTR);
        constexpr int VEC = Vec16<KT>::N;
#pragma unroll 2
        for (int d0 = 0; d0 < D; d0 += VEC) {
          float kf[VEC];
          Vec16<KT>::load(krow + d0, kf);
#pragma unroll
          for (int j = 0; j < HPT; ++j) {
            const float* qrow = &q_s[(hg * HPT + j) * D + d0];
#pragma unroll
            for (int v4 = 0; v4 < VEC; v4 += 4) {
              const float4 qv = *reinterpret_cast<const float4*>(qrow + v4);
              sc[j] = fmaf(qv.x, kf[v4], sc[j]);
              sc[j] = fmaf(qv.y, kf[v4 + 1], sc[j]);
              sc[j] = fmaf(qv.z, kf[v4 + 2], sc[j]);
              sc[j] = fmaf(qv.w, kf[v4 + 3], sc[j]);
            }
          }
        }
#pragma unroll
        for (int j = 0; j < HPT; ++j) sc[j] *= M::SCALE;
      } else {
#pragma unroll
        for (int j = 0; j < HPT; ++j) sc[j] = -INFINITY;
      }
#pragma unroll
      for (int j = 0; j < HPT; ++j) S[t_own * G + hg * HPT + j] = sc[j];
    }
    __syncthreads();
    // tile-wise online softmax: warp w owns heads w, w+4, ...
    for (int g = warp; g < G; g += 4) {
      const float s0 = S[lane * G + g], s1 = S[(lane + 32) * G + g];
      const float mt = warp_max(fmaxf(s0, s1));
      const float mold = st_m[g];
      const float mnew = fmaxf(mold, mt);
      const float alpha = (mold == -INFINITY) ? 0.0f : softmax_exp(mold - mnew, pinned);
      const float p0 = lane < rows ? softmax_exp(s0 - mnew, pinned) : 0.0f;
      const float p1 = lane + 32 < rows ? softmax_exp(s1 - mnew, pinned) : 0.0f;
      S[lane * G + g] = p0;
      S[(lane + 32) * G + g] = p1;
      const float sum = warp_sum(p0 + p1);
      if (lane == 0) {
        st_l[g] = fmaf(st_l[g], alpha, sum);
        st_m[g] = mnew;
        st_a[g] = alpha;
      }
    }
    __syncthreads();
    // P.V: thread owns heads hg*HPT.. and dims dg*DPT..
    {
#pragma unroll
      for (int j = 0; j < HPT; ++j) {
        const float a = st_a[hg * HPT + j];
#pragma unroll
        for (int e = 0; e < DPT; ++e) acc[j][e] *= a;
      }
#pragma unroll 4
      for (int tt = 0; tt < rows; ++tt) {
        const VT* vrow = reinterpret_cast<const VT*>(vt + tt * C::VSTR);
        float vv[DPT];
#pragma unroll
        for (int e = 0; e < DPT; ++e) vv[e] = Elem<VT>::to_f32(vrow[dg * DPT + e]);
        const float* prow = &S[tt * G + hg * HPT];
#pragma unroll
        for (int j = 0; j < HPT; ++j) {
          const float pw = prow[j];
#pragma unroll
          for (int e = 0; e < DPT; ++e) acc[j][e] = fmaf(pw, vv[e], acc[j][e]);
        }
      }
    }
    __syncthreads();  // stage `st` and S are free again
    if (warp == 0 && tile + STAGES < ntiles) issue(tile + STAGES);
  }

  // ---- finish: direct output, or partial + last-CTA merge -------------------
  const long long obase = (cu * HQ + (long long)h * G) * D;
  if (nsplit == 1) {
    bool nonfinite = false;
#pragma unroll
    for (int j = 0; j < HPT; ++j) {
      const int g = hg * HPT + j;
      const float l = st_l[g];
      if (p.emit_partials) {
        float* part = reinterpret_cast<float*>(p.out) + (cu * HQ + (long long)h * G + g) * (D + 2);
#pragma unroll
        for (int e = 0; e < DPT; ++e) part[dg * DPT + e] = acc[j][e];
        if (dg == 0) {
          part[D] = st_m[g];
          part[D + 1] = l;
        }
      } else {
        const float inv = 1.0f / l;
#pragma unroll
        for (int e = 0; e < DPT; ++e) {
          const float o = acc[j][e] * inv;
          nonfinite |= !isfinite(o);
          store_any(p.out, obase + g * D + dg * DPT + e, p.out_dtype, o);
        }
      }
    }
    if (nonfinite) flag_error(p.err, QX_ERR_BIT_NONFINITE);
    return;
  }

  float* part = p.partials + (long long)blockIdx.x * G * (D + 2);
#pragma unroll
  for (int j = 0; j < HPT; ++j)
#pragma unroll
    for (int e = 0; e < DPT; ++e) part[(hg * HPT + j) * (D + 2) + dg * DPT + e] = acc[j][e];
  if (tid < G) {
    part[tid * (D + 2) + D] = st_m[tid];
    part[tid * (D + 2) + D + 1] = st_l[tid];
  }
  __threadfence();
  __syncthreads();
  int* ticket = p.tickets + cu * HKV + h;
  if (tid == 0) s_flag[0] = (atomicAdd(ticket, 1) == nsplit - 1);
  __syncthreads();
  if (!s_flag[0]) return;
  __threadfence();

  const float* first = p.partials + (long long)(blockIdx.x - s) * G * (D + 2);
  bool nonfinite = false;
#pragma unroll
  for (int j = 0; j < HPT; ++j) {
    const int g = hg * HPT + j;
    float mx = -INFINITY;
    for (int i = 0; i < nsplit; ++i) mx = fmaxf(mx, __ldcg(first + ((long long)i * G + g) * (D + 2) + D));
    float L = 0.0f, O[DPT];
#pragma unroll
    for (int e = 0; e < DPT; ++e) O[e] = 0.0f;
    for (int i = 0; i < nsplit; ++i) {
      const float* pi = first + ((long long)i * G + g) * (D + 2);
      const float w = softmax_exp(__ldcg(pi + D) - mx, pinned);
      L = fmaf(w, __ldcg(pi + D + 1), L);
#pragma unroll
      for (int e = 0; e < DPT; ++e) O[e] = fmaf(w, __ldcg(pi + dg * DPT + e), O[e]);
    }
    if (p.emit_partials) {
      float* dst = reinterpret_cast<float*>(p.out) + (cu * HQ + (long long)h * G + g) * (D + 2);
#pragma unroll
      for (int e = 0; e < DPT; ++e) dst[dg * DPT + e] = O[e];
      if (dg == 0) {
        dst[D] = mx;
        dst[D + 1] = L;
      }
    } else {
      const float inv = 1.0f / L;
#pragma unroll
      for (int e = 0; e < DPT; ++e) {
        const float o = O[e] * inv;
        nonfinite |= !isfinite(o);
        store_any(p.out, obase + g * D + dg * DPT + e, p.out_dtype, o);
      }
    }
  }
  if (nonfinite) flag_error(p.err, QX_ERR_BIT_NONFINITE);
  if (tid == 0) *ticket = 0;  // ready for the next call
}

// ---- log-sum-exp merge of partial sets (KV-length split across GPUs) -------
// partials [n_parts][HQ][D+2] -> out [HQ][D]. One CTA per query head.
template <int HQ, int D>
__global__ void qx_lse_merge_kernel(const float* __restrict__ partials, int n_parts, void* out, int out_dtype,
                                    int pinned, unsigned* err) {
  const int qh = blockIdx.x;
  float mx = -INFINITY;
  for (int i = 0; i < n_parts; ++i) mx = fmaxf(mx, partials[((long long)i * HQ + qh) * (D + 2) + D]);
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float L = 0.0f, O = 0.0f;
    for (int i = 0; i < n_parts; ++i) {
      const float* pi = partials + ((long long)i * HQ + qh) * (D + 2);
      if (pi[D] == -INFINITY) continue;  // empty shard
      const float w = softmax_exp(pi[D] - mx, pinned != 0);
      L = fmaf(w, pi[D + 1], L);
      O = fmaf(w, pi[d], O);
    }
    const float o = O / L;
    if (!isfinite(o)) flag_error(err, QX_ERR_BIT_NONFINITE);
    store_any(out, (long long)qh * D + d, out_dtype, o);
  }
}

// ---- standalone RoPE (apply_granite_rope, qx-runtime lib.rs:434-442) -------
// q [16][64] and k [8][64] f32 in place; one thread per rotation pair.
__global__ void qx_granite_rope_kernel(float* q, float* k, int position, unsigned* err) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;  // 0 .. 24*32-1
  if (idx >= 24 * 32) return;
  const int head = idx >> 5, pair = idx & 31;
  float* base = head < 16 ? q + head * 64 : k + (head - 16) * 64;
  float sn, cs, a = 0.f, b = 0.f;
  bool ok = granite_sin_cos((uint32_t)position, pair, &sn, &cs) && granite_rotate(base[pair], base[pair + 32], sn, cs, &a, &b);
  if (!ok) {
    flag_error(err, QX_ERR_BIT_NONFINITE);
    return;
  }
  base[pair] = a;
  base[pair + 32] = b;
}

}  // namespace qx
