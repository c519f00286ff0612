// decode.cuh — split-KV flash decode for qx's GQA attention on sm_100a.
//
// One CTA per work item (sequence, layer, kv head, split of the cache). The
// CTA
//   1. dedicates one producer warp to TMA: 3-D tensor-map boxes of 64 cache
//      rows of its kv head (the cache keeps the reference's position-major
//      layout [pos][kv_head][head_dim]) into a multi-stage shared-memory
//      ring guarded by full/empty mbarriers;
//   2. meanwhile the four consumer warps apply RoPE to the G query heads that share this kv head
//      (Granite: qx's pinned sin/cos and FMA order, qx-consensus-math
//      lib.rs:148-207; Qwen: per-head RMSNorm then rotate-half RoPE,
//      qx-qwen-parity main.rs:1177-1204), and, on the split that owns the
//      new token, RoPE on k, writing k and v into slot `position` and into
//      its own last tile (so no CTA ever reads the slot being written);
//   3. each consumer warp owns 16 rows of every stage and keeps its own
//      online-softmax state (scores for all G query heads against each key
//      row held once in shared memory, 16-lane shuffle max/sum, P.V in
//      registers), so the loop has no block-wide barrier; the four warp
//      states merge once at the end;
//   4. writes its (m, l, O) partial; the last CTA of the (sequence, layer,
//      kv head) to finish (atomic ticket, no spinning) merges the partials
//      with a log-sum-exp combine and writes the output.
//
// Reference semantics: crates/qx-runtime/src/lib.rs:464-552
// (granite_attention_decode_with_profile) for Granite, and
// tools/qx-qwen-parity/src/main.rs:1170-1258 for Qwen3.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "qx_math.cuh"
#include "qx_ptx.cuh"

namespace qx {

// G query rows per kv head in a work item: NTOK tokens x G0 query heads.
struct Granite {
  static constexpr int HQ = 16, HKV = 8, D = 64, G = 2, NTOK = 1, G0 = 2;
  static constexpr bool QWEN = false;
  static constexpr float SCALE = 0.015625f;  // ATTENTION_MULTIPLIER, qx-model lib.rs:20
};
struct Qwen3 {
  static constexpr int HQ = 32, HKV = 4, D = 128, G = 8, NTOK = 1, G0 = 8;
  static constexpr bool QWEN = true;
  static constexpr float SCALE = 0.08838834764831845f;  // 1/sqrt(128)
};
// Speculative verify of up to 4 candidate tokens of one sequence: every
// cache tile is scored against the 4 tokens' queries at once, token t
// seeing rows [0, start + t] (HQ counts the 4 tokens' heads).
struct GraniteVerify4 {
  static constexpr int HQ = 64, HKV = 8, D = 64, G = 8, NTOK = 4, G0 = 2;
  static constexpr bool QWEN = false;
  static constexpr float SCALE = Granite::SCALE;
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

// How a (sequence, layer, slot) finds its cache row in the arena's regions
// (rows of [kv_heads][head_dim]). A contiguous arena keeps each (sequence,
// layer) cache as `capacity` consecutive rows. A paged arena keeps, per
// layer, a pool of pages of 2^shift rows; a sequence's block table (shared
// by all layers, as in vLLM) maps its logical page to a physical page.
struct KvPaging {
  const int* table;  // device [sequences][stride] physical page per logical page; null: contiguous
  int stride;        // logical pages per sequence
  int shift;         // log2 of rows per page (>= 6: a 64-row TMA box never straddles pages)
  int pool;          // physical pages per layer
};

__device__ __forceinline__ long long kv_row(const KvPaging& pg, int capacity, int layers, int seq, int layer,
                                            int slot) {
  if (!pg.table) return ((long long)seq * layers + layer) * capacity + slot;
  const int page = __ldg(pg.table + (long long)seq * pg.stride + (slot >> pg.shift));
  return (((long long)layer * pg.pool + page) << pg.shift) + (slot & ((1 << pg.shift) - 1));
}

struct DecodeParams {
  // 3-D tensor maps over the key / value regions of the arena:
  // dims {head_dim, kv_heads, sequences*layers*capacity}, box
  // {128 bytes of head_dim, 1, 64 positions}, 128-byte swizzle.
  CUtensorMap tmk;
  CUtensorMap tmv;
  int capacity;  // rows per (sequence, layer) in the tensor maps (contiguous arenas)
  KvPaging paging;
  // arena
  char* k_region;
  char* v_region;
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
  int external_merge;  // splits only store partials; qx_split_merge_kernel merges them
  // One-wave tensor-core decode with 2..64 splits: the splits of each (unit,
  // kv head) store their partials tagged and merge them among themselves
  // (slice_merge) instead of in qx_split_merge_kernel.
  int slice_merge;
  unsigned merge_tag;  // this call's tag for those partials (never 0)
  uint2* tpartials;    // scratch [items][G][D+2] {value bits, tag}
  int early_trigger;   // one-wave grid: let the next grid launch early (griddepcontrol)
  // Single-sequence calls (seq_table == nullptr) on a contiguous arena:
  // cache rows [0, pre_rows) of the sequence were written by grids that have
  // completed, so the tensor-core decode may stream them before
  // griddepcontrol.wait (0: none). The host derives it from the launches it
  // made on the stream (note_rows_written).
  int pre_rows;
  float* partials;    // scratch [items][G][D+2]
  int* tickets;       // scratch [n_seq][layer_count][HKV], zero between calls
  unsigned* err;
  unsigned long long* trace;  // stage timeline (diagnostics), or null
  // KV-length split across GPUs, merged by qx_split_merge_kernel itself
  // (xworld > 0): every rank's inbox of [2][xworld][HQ * D/32][34] tagged
  // values (32 dims of O, m, l per query head and 32-dim slice) and this
  // rank's step counter per (query head, slice); see exchange.cuh
  uint2* xinbox[8];
  unsigned* xstep;
  unsigned* xfailed;       // the peer group's failed word (device), see mark_peer_group_failed
  unsigned* xfailed_host;  // and its pinned host copy
  int xrank, xworld;
  void* xout;  // final output [HQ][D]
  int xout_dtype;
  int ntok;  // candidate tokens of a multi-token item (GraniteVerify4), <= its NTOK
};

// Element d of output row g (of the G rows of kv head h) of unit cu. One
// token per item: [unit][HQ][D]. NTOK tokens per item (one sequence): row g
// is token g / G0's query head h * G0 + g % G0, stored [token][layer][HQ / NTOK][D]
// like the q and out tensors of a verify call; cu is then the layer within it.
template <int G, int D, int HQ, int NTOK, int G0>
__device__ __forceinline__ long long out_elem(const DecodeParams& p, long long cu, int h, int g, int d) {
  if constexpr (NTOK == 1) {
    return (cu * HQ + (long long)h * G + g) * D + d;
  } else {
    const int t = g / G0;
    return (((long long)t * p.layer_count + cu) * (HQ / NTOK) + h * G0 + g % G0) * D + d;
  }
}

template <class M, typename KT, typename VT>
struct DecodeCfg {
  static constexpr int T = 64;             // positions per pipeline stage
  // Consumer warps come in groups of four; group g takes stages g, g+NGROUP,
  // ... and warp w of a group owns rows [16w, 16w+16) of each of them.
  // Granite runs two groups (more resident warps to hide shared-memory
  // latency); Qwen's 8-head state needs the registers of one group.
  static constexpr int NWC = M::QWEN ? 4 : 8;  // consumer warps
  static constexpr int NGROUP = NWC / 4;
  static constexpr int NT = 32 * NWC + 32;     // + one producer warp
  static constexpr int WT = T / 4;             // rows per consumer warp per stage
  static constexpr int D = M::D, G = M::G;
  static constexpr int QPL = G * WT / 32;      // query heads per lane in QK (Granite 1, Qwen 4)
  // P.V: Granite lanes of each half-warp take alternate rows and 4 dims each
  // (one 128-bit load of V per row); Qwen lanes take D/32 dims of every row.
  static constexpr bool PVH = !M::QWEN;
  static constexpr int DPL = PVH ? D / 16 : D / 32;
  static constexpr int KROW = D * (int)sizeof(KT), VROW = D * (int)sizeof(VT);
  // A stage arrives as 128-byte-wide TMA boxes ([64 rows][128 B], 128-byte
  // swizzle: chunk c of row t sits at chunk c ^ (t & 7)), so 128-bit shared
  // loads by 8 consecutive rows never hit the same bank twice.
  static constexpr int KB = KROW / 128, VB = VROW / 128;  // boxes per row
  static constexpr int BOX = T * 128;
  static constexpr int STAGE_K = KB * BOX, STAGE_V = VB * BOX;
  // Tile t lives in stage t % STAGES and is consumed by group t % NGROUP.
  // STAGES must be a multiple of NGROUP: then a stage is always consumed by
  // the same group, which finished the stage's previous tile before waiting
  // for the next one, so a full/empty barrier is never more than one phase
  // ahead of its waiter (mbarrier parity only tells two phases apart).
  static constexpr int STAGES = NGROUP == 2 ? ((STAGE_K + STAGE_V) <= 16384 ? 4 : 2)
                                            : ((STAGE_K + STAGE_V) <= 16384 ? 4 : 3);
  static_assert(STAGES % NGROUP == 0, "each stage must belong to one consumer group");
  static constexpr int OFF_K = 0;                         // 1024-aligned
  static constexpr int OFF_V = OFF_K + STAGES * STAGE_K;  // 1024-aligned
  static constexpr int OFF_Q = OFF_V + STAGES * STAGE_V;  // float [G][D]
  static constexpr int OFF_P = OFF_Q + G * D * 4;         // float [NWC][WT][G]
  // Qwen: raw q heads and the k head staged as f32 for the RMSNorm prologue
  static constexpr int RAW_FLOATS = M::QWEN ? (G + 1) * D : 0;
  static constexpr int OFF_RAW = OFF_P + NWC * WT * G * 4;
  static constexpr int OFF_NEWK = OFF_RAW + RAW_FLOATS * 4;
  static constexpr int OFF_NEWV = OFF_NEWK + ((KROW + 15) / 16) * 16;
  static constexpr int OFF_STAT = OFF_NEWV + ((VROW + 15) / 16) * 16;  // float [NWC][G][2], inv[G+1]
  static constexpr int OFF_BAR = ((OFF_STAT + 4 * (NWC * G * 2 + G + 1) + 15) / 16) * 16;
  static constexpr int SMEM = OFF_BAR + 16 * STAGES + 16 + 1024;  // + slack to align the base to 1024
  // after the main loop the stage buffers hold the per-warp merge [NWC][G][D]
  static_assert(NWC * G * D * 4 <= STAGES * (STAGE_K + STAGE_V), "merge buffer must fit the stages");
  // the last CTA's split merge stages 2 x G x nsplit floats there too
  static constexpr int MAX_SPLITS = (STAGES * (STAGE_K + STAGE_V)) / (8 * G);
};

// Byte offset of byte `b` of row `t` inside a swizzled [64][128 B] box stack.
template <int BOX>
__device__ __forceinline__ int swz(int t, int b) {
  const int w = b & 127;
  return (b >> 7) * BOX + t * 128 + ((((w >> 4) ^ (t & 7))) << 4) + (w & 15);
}

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
// Reductions within each 16-lane half of a warp.
__device__ __forceinline__ float half_max(float v) {
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float half_sum(float v) {
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Barrier 1 over the consumer threads only (the producer warp is busy).
__device__ __forceinline__ void consumers_sync(int n) { asm volatile("bar.sync 1, %0;" ::"r"(n) : "memory"); }
// Barrier 2 over the first 128 threads (the output combine).
__device__ __forceinline__ void combine_sync() { asm volatile("bar.sync 2, 128;" ::: "memory"); }
// Barrier 0 over the whole CTA, reached from the producer and the consumer
// branches (PTX counts arrivals, wherever they come from).
__device__ __forceinline__ void cta_sync() { asm volatile("bar.sync 0;" ::: "memory"); }

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

// Outputs of one work item, then (when the cache was split) the split merge.
// Thread tid < 128 holds outputs idx = tid + k*128 (head g = idx / D, dim
// d = idx % D) as unnormalised O[k] with head max Mg[k] and sum Lg[k].
// One split: O / L goes straight to `out` (or (O, m, l) when emitting
// partials). Several: every split stores its (O, m, l) partial; the last
// CTA of the (sequence, layer, kv head) to finish (atomic ticket, no
// spinning) merges them by log-sum-exp and resets the ticket.
// merge_smem must hold 2 * G * nsplit floats, stat_smem 2 * G floats.
template <int G, int D, int HKV, int HQ, int OPT, int NTOK = 1, int G0 = G>
__device__ __forceinline__ void finish_outputs(const DecodeParams& p, const float* O, const float* Mg, const float* Lg,
                                               int nsplit, int s, long long cu, int h, int tid, int warp, int lane,
                                               bool pinned, float* merge_smem, float* stat_smem, int* s_flag) {
  // (with an exchange across GPUs even one split goes to qx_split_merge_kernel,
  // which pushes it to the peers)
  if (nsplit == 1 && !p.xworld) {
    bool nonfinite = false;
#pragma unroll
    for (int k = 0; k < OPT; ++k) {
      const int idx = tid + k * 128, g = idx / D, d = idx % D;
      if (p.emit_partials) {
        float* part = reinterpret_cast<float*>(p.out) + (cu * HQ + (long long)h * G + g) * (D + 2);
        part[d] = O[k];
        if (d == 0) {
          part[D] = Mg[k];
          part[D + 1] = Lg[k];
        }
      } else if (NTOK == 1 || g / G0 < p.ntok) {
        const float o = O[k] / Lg[k];
        nonfinite |= !isfinite(o);
        store_any(p.out, out_elem<G, D, HQ, NTOK, G0>(p, cu, h, g, d), p.out_dtype, o);
      }
    }
    if (nonfinite) flag_error(p.err, QX_ERR_BIT_NONFINITE);
    return;
  }

  float* part = p.partials + (long long)blockIdx.x * G * (D + 2);
#pragma unroll
  for (int k = 0; k < OPT; ++k) {
    const int idx = tid + k * 128, g = idx / D, d = idx % D;
    part[g * (D + 2) + d] = O[k];
    if (d == 0) {
      part[g * (D + 2) + D] = Mg[k];
      part[g * (D + 2) + D + 1] = Lg[k];
    }
  }
  if (p.external_merge) return;  // qx_split_merge_kernel, launched next, merges
  __threadfence();
  combine_sync();
  int* ticket = p.tickets + cu * HKV + h;
  if (tid == 0) s_flag[0] = (atomicAdd(ticket, 1) == nsplit - 1);
  combine_sync();
  if (!s_flag[0]) return;
  __threadfence();

  // Merge the nsplit partials of this (sequence, layer, kv head) in three
  // parallel steps: stage every split's (m, l) in shared memory; one warp
  // per head reduces M = max m_i and L = sum e^(m_i - M) l_i and leaves the
  // weights e^(m_i - M); every output then sums nsplit weighted partials
  // with independent loads (4 accumulators).
  const float* first = p.partials + (long long)(blockIdx.x - s) * G * (D + 2);
  float* wts = merge_smem;  // [G][nsplit] m_i, then weights
  float* lsp = wts + G * nsplit;                          // [G][nsplit] l_i
  float* hml = stat_smem;  // [G] M, [G] L
  for (int i = tid; i < nsplit * G; i += 128) {
    const int sp = i / G, g = i - sp * G;
    const float* pi = first + ((long long)sp * G + g) * (D + 2);
    wts[g * nsplit + sp] = __ldcg(pi + D);
    lsp[g * nsplit + sp] = __ldcg(pi + D + 1);
  }
  combine_sync();
  for (int g = warp; g < G; g += 4) {
    float mx = -INFINITY;
    for (int i = lane; i < nsplit; i += 32) mx = fmaxf(mx, wts[g * nsplit + i]);
    mx = warp_max(mx);
    float L = 0.0f;
    for (int i = lane; i < nsplit; i += 32) {
      const float w = softmax_exp(wts[g * nsplit + i] - mx, pinned);
      wts[g * nsplit + i] = w;
      L = fmaf(w, lsp[g * nsplit + i], L);
    }
    L = warp_sum(L);
    if (lane == 0) {
      hml[g] = mx;
      hml[G + g] = L;
    }
  }
  combine_sync();
  // splits outer, outputs inner: every iteration has OPT independent loads,
  // and unrolling by 4 keeps 4 x OPT of them in flight
  const long long stride = (long long)G * (D + 2);
  float o[OPT];
#pragma unroll
  for (int k = 0; k < OPT; ++k) o[k] = 0.0f;
#pragma unroll 4
  for (int i = 0; i < nsplit; ++i) {
    const float* pi = first + i * stride;
#pragma unroll
    for (int k = 0; k < OPT; ++k) {
      const int idx = tid + k * 128, g = idx / D, d = idx % D;
      o[k] = fmaf(wts[g * nsplit + i], __ldcg(pi + g * (D + 2) + d), o[k]);
    }
  }
  bool nonfinite = false;
#pragma unroll
  for (int k = 0; k < OPT; ++k) {
    const int idx = tid + k * 128, g = idx / D, d = idx % D;
    const float mx = hml[g], L = hml[G + g];
    if (p.emit_partials) {
      float* dst = reinterpret_cast<float*>(p.out) + (cu * HQ + (long long)h * G + g) * (D + 2);
      dst[d] = o[k];
      if (d == 0) {
        dst[D] = mx;
        dst[D + 1] = L;
      }
    } else if (NTOK == 1 || g / G0 < p.ntok) {
      const float v = o[k] / L;
      nonfinite |= !isfinite(v);
      store_any(p.out, out_elem<G, D, HQ, NTOK, G0>(p, cu, h, g, d), p.out_dtype, v);
    }
  }
  if (nonfinite) flag_error(p.err, QX_ERR_BIT_NONFINITE);
  if (tid == 0) *ticket = 0;  // ready for the next call
}

template <class M, typename KT, typename VT>
__device__ __forceinline__ void decode_body(const DecodeParams& p) {
  using C = DecodeCfg<M, KT, VT>;
  // A one-wave grid lets the next grid (the merge, or the next call) get
  // resident at once. Launches on the stream after this grid may therefore
  // overlap the grids before it; the host knows (note_rows_written).
  if (p.early_trigger) pdl_launch_dependents();
  constexpr int D = M::D, G = M::G, HKV = M::HKV, HQ = M::HQ, T = C::T, NWC = C::NWC, WT = C::WT;
  constexpr int QPL = C::QPL, DPL = C::DPL, STAGES = C::STAGES;
  extern __shared__ __align__(1024) unsigned char sm_raw[];
  unsigned char* sm = sm_raw + ((1024u - (smem_addr(sm_raw) & 1023u)) & 1023u);
  unsigned char* ktiles = sm + C::OFF_K;
  unsigned char* vtiles = sm + C::OFF_V;
  float* q_s = reinterpret_cast<float*>(sm + C::OFF_Q);
  float* P_s = reinterpret_cast<float*>(sm + C::OFF_P);
  KT* newk = reinterpret_cast<KT*>(sm + C::OFF_NEWK);
  VT* newv = reinterpret_cast<VT*>(sm + C::OFF_NEWV);
  float* stat = reinterpret_cast<float*>(sm + C::OFF_STAT);  // [NWC][G][2]
  float* st_inv = stat + NWC * G * 2;                         // [G + 1]
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + C::OFF_BAR);
  uint64_t* empty = full + STAGES;
  int* s_flag = reinterpret_cast<int*>(empty + STAGES);  // [0] last-CTA flag, [1] abort

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid == 0) {
#pragma unroll
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 4);  // the four warps of the group that consumes the stage
    }
    s_flag[1] = 0;
    fence_barrier_init();
  }
  __syncthreads();
  // launched as a programmatic dependent: everything above overlapped the
  // previous grid; from here on its memory is visible
  pdl_wait();

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
  const int begin = s * p.chunk;
  const int end = min(begin + p.chunk, si.attend);
  const bool has_new = si.new_slot >= begin && si.new_slot < end;  // last split only
  const int ntiles = (end - begin + T - 1) / T;
  const long long cu = (long long)slot * p.layer_count + lloc;  // packed q/k/v/out index
  const bool last_split = (s == nsplit - 1);


  if (warp == NWC) {
    // ---- producer warp: TMA boxes into the stage ring -----------------------
    if (lane == 0) {
      prefetch_tmap(&p.tmk);
      prefetch_tmap(&p.tmv);
      for (int tile = 0; tile < ntiles; ++tile) {
        const int st = tile % STAGES;
        const int z = (int)kv_row(p.paging, p.capacity, p.layers, si.seq_id, layer, begin + tile * T);
        if (tile >= STAGES && !mbar_wait_bounded(&empty[st], (uint32_t)((tile / STAGES) - 1) & 1u, p.err)) {
          s_flag[1] = 1;
          break;
        }
        unsigned char* kt = ktiles + st * C::STAGE_K;
        unsigned char* vt = vtiles + st * C::STAGE_V;
        mbar_arrive_expect_tx(&full[st], (uint32_t)(C::STAGE_K + C::STAGE_V));
#pragma unroll
        for (int b = 0; b < C::KB; ++b)
          tma_load_3d(kt + b * C::BOX, &p.tmk, b * (128 / (int)sizeof(KT)), h, z, &full[st]);
#pragma unroll
        for (int b = 0; b < C::VB; ++b)
          tma_load_3d(vt + b * C::BOX, &p.tmv, b * (128 / (int)sizeof(VT)), h, z, &full[st]);
      }
    }
  } else {
    // ---- consumers: prologue (RoPE; the new k/v row on the owning split) -----
    const long long qbase = (cu * HQ + (long long)h * G) * D;  // first query element of this group
    const long long kvbase = (cu * HKV + h) * D;
    bool bad = false;
    if constexpr (!M::QWEN) {
      // 32 rotation pairs per head: warps 0-1 the G=2 query heads, warp 2 k.
      if (tid < G * 32) {
        const int g = tid >> 5, pair = tid & 31;
        // several candidate tokens per item: row g is token g / G0 at its own position
        const int tok = g / M::G0;
        const bool live = M::NTOK == 1 || tok < p.ntok;
        const long long qa = M::NTOK == 1 ? qbase + g * D : out_elem<G, D, HQ, M::NTOK, M::G0>(p, cu, h, g, 0);
        float left = live ? load_any(p.q, qa + pair, p.q_dtype) : 0.0f;
        float right = live ? load_any(p.q, qa + pair + 32, p.q_dtype) : 0.0f;
        float sn, cs, a = 0.f, b = 0.f;
        bool ok = granite_sin_cos((uint32_t)(si.rope_pos + tok), pair, &sn, &cs) &&
                  granite_rotate(left, right, sn, cs, &a, &b);
        bad |= live && !ok;
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
        bool ok = granite_sin_cos((uint32_t)si.rope_pos, pair, &sn, &cs) &&
                  granite_rotate(left, right, sn, cs, &a, &b);
        bad |= !ok;
        newk[pair] = Elem<KT>::from_f32(a);
        newk[pair + 32] = Elem<KT>::from_f32(b);
      }
    } else {
      // Stage the raw q heads (and k) in shared memory with parallel loads,
      // then per-head RMSNorm with the reference's sequential sum of squares
      // (bit-exact K); one thread per head sums from shared memory.
      float* raw = reinterpret_cast<float*>(sm + C::OFF_RAW);  // [G + 1][D]
      for (int i = tid; i < (G + 1) * D; i += 32 * NWC) {
        const int g = i / D, e = i - g * D;
        raw[i] = g < G ? load_any(p.q, qbase + g * D + e, p.q_dtype)
                       : (has_new ? load_any(p.k, kvbase + e, p.in_dtype) : 0.0f);
      }
      consumers_sync(32 * NWC);
      if (tid < G || (tid == G && has_new)) {
        const float* row = raw + tid * D;
        float sum = 0.0f;
#pragma unroll
        for (int i = 0; i < D; ++i) sum = __fadd_rn(sum, __fmul_rn(row[i], row[i]));
        st_inv[tid] = __frcp_rn(__fsqrt_rn(__fadd_rn(__fdiv_rn(sum, 128.0f), 1.0e-6f)));
      }
      consumers_sync(32 * NWC);
      const float2* tab = p.rope_table + (long long)si.rope_pos * 64;
      for (int idx = tid; idx < (G + 1) * 64; idx += 32 * NWC) {
        const int g = idx >> 6, i = idx & 63;
        if (g == G && !has_new) break;
        const bool is_q = g < G;
        const float inv = st_inv[g];
        const float* wn = is_q ? p.q_norm : p.k_norm;
        const float x = raw[g * D + i], y = raw[g * D + i + 64];
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
    if (has_new)
      for (int i = tid; i < D; i += 32 * NWC) newv[i] = Elem<VT>::from_f32(load_any(p.v, kvbase + i, p.in_dtype));
    if (bad) flag_error(p.err, QX_ERR_BIT_NONFINITE);
    consumers_sync(32 * NWC);
    if (has_new) {
      // Append: slot new_slot of this kv head.
      const long long row = kv_row(p.paging, p.capacity, p.layers, si.seq_id, layer, si.new_slot);
      char* kdst = p.k_region + (row * HKV + h) * C::KROW;
      char* vdst = p.v_region + (row * HKV + h) * C::VROW;
      for (int i = tid; i < C::KROW / 16; i += 32 * NWC)
        reinterpret_cast<uint4*>(kdst)[i] = reinterpret_cast<const uint4*>(newk)[i];
      for (int i = tid; i < C::VROW / 16; i += 32 * NWC)
        reinterpret_cast<uint4*>(vdst)[i] = reinterpret_cast<const uint4*>(newv)[i];
    }

    // ---- consumers: main loop; warp w owns rows [16w, 16w+16) of each stage --
    const bool pinned = p.pinned_exp != 0;
    const int trow = lane & 15;              // QK: row within my 16
    const int hq0 = (lane >> 4) * QPL;       // QK: first query head of this lane
    float m_run[G], l_run[G], acc[G][DPL];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      m_run[g] = -INFINITY;
      l_run[g] = 0.0f;
#pragma unroll
      for (int e = 0; e < DPL; ++e) acc[g][e] = 0.0f;
    }
    float* Pw = P_s + warp * WT * G;
    const int wg = warp & 3;
    for (int tile = warp >> 2; tile < ntiles; tile += C::NGROUP) {
      const int st = tile % STAGES;
      if (!mbar_wait_bounded(&full[st], (uint32_t)(tile / STAGES) & 1u, p.err)) {
        s_flag[1] = 1;
        break;
      }
      unsigned char* kt = ktiles + st * C::STAGE_K;
      unsigned char* vt = vtiles + st * C::STAGE_V;
      const int rows = min(T, end - (begin + tile * T));
      const int r0 = wg * WT;
      const int mine = max(0, min(WT, rows - r0));
      if (has_new && tile == ntiles - 1 && rows - 1 >= r0 && rows - 1 < r0 + WT) {
        // the appended slot comes from registers, not from the copy
        for (int i = lane; i < C::KROW / 16; i += 32)
          *reinterpret_cast<uint4*>(kt + swz<C::BOX>(rows - 1, i * 16)) = reinterpret_cast<const uint4*>(newk)[i];
        for (int i = lane; i < C::VROW / 16; i += 32)
          *reinterpret_cast<uint4*>(vt + swz<C::BOX>(rows - 1, i * 16)) = reinterpret_cast<const uint4*>(newv)[i];
        __syncwarp();
      }
      if (mine > 0) {
        // scores: lane (row r0+trow, heads hq0..hq0+QPL-1), 4 partial sums
        float sc[QPL];
        if constexpr (G == 2) {
          // a group of two heads: each half-warp takes half the dims of its
          // 16 rows for both heads, so a K element is loaded (and widened
          // from 16 bits) once instead of once per head; one shuffle joins
          // the halves, after which lane (row, half) keeps head `half`
          const int dh = lane >> 4;
          float part[2][4];
#pragma unroll
          for (int j = 0; j < 2; ++j)
#pragma unroll
            for (int u = 0; u < 4; ++u) part[j][u] = 0.0f;
          if (trow < mine) {
            constexpr int VEC = Vec16<KT>::N;
#pragma unroll
            for (int i = 0; i < D / 2; i += VEC) {
              const int d0 = dh * (D / 2) + i;
              float kf[VEC];
              Vec16<KT>::load(reinterpret_cast<const KT*>(kt + swz<C::BOX>(r0 + trow, d0 * (int)sizeof(KT))), kf);
#pragma unroll
              for (int j = 0; j < 2; ++j) {
                const float* qrow = &q_s[j * D + d0];
#pragma unroll
                for (int v4 = 0; v4 < VEC; v4 += 4) {
                  // the four chains in pairs, one packed fma per pair (same roundings)
                  const float4 qv = *reinterpret_cast<const float4*>(qrow + v4);
                  const float2 lo = __ffma2_rn(make_float2(qv.x, qv.y), make_float2(kf[v4], kf[v4 + 1]),
                                               make_float2(part[j][0], part[j][1]));
                  const float2 hi = __ffma2_rn(make_float2(qv.z, qv.w), make_float2(kf[v4 + 2], kf[v4 + 3]),
                                               make_float2(part[j][2], part[j][3]));
                  part[j][0] = lo.x;
                  part[j][1] = lo.y;
                  part[j][2] = hi.x;
                  part[j][3] = hi.y;
                }
              }
            }
          }
          float s2[2];
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const float h = (part[j][0] + part[j][1]) + (part[j][2] + part[j][3]);
            s2[j] = h + __shfl_xor_sync(0xffffffffu, h, 16);  // dims of both halves: same sum in both lanes
          }
          sc[0] = trow < mine ? (dh == 0 ? s2[0] : s2[1]) * M::SCALE : -INFINITY;
        } else if (trow < mine) {
          float part[QPL][4];
#pragma unroll
          for (int j = 0; j < QPL; ++j)
#pragma unroll
            for (int u = 0; u < 4; ++u) part[j][u] = 0.0f;
          constexpr int VEC = Vec16<KT>::N;
#pragma unroll
          for (int d0 = 0; d0 < D; d0 += VEC) {
            float kf[VEC];
            Vec16<KT>::load(reinterpret_cast<const KT*>(kt + swz<C::BOX>(r0 + trow, d0 * (int)sizeof(KT))), kf);
#pragma unroll
            for (int j = 0; j < QPL; ++j) {
              const float* qrow = &q_s[(hq0 + j) * D + d0];
#pragma unroll
              for (int v4 = 0; v4 < VEC; v4 += 4) {
                const float4 qv = *reinterpret_cast<const float4*>(qrow + v4);
                const float2 lo = __ffma2_rn(make_float2(qv.x, qv.y), make_float2(kf[v4], kf[v4 + 1]),
                                             make_float2(part[j][0], part[j][1]));
                const float2 hi = __ffma2_rn(make_float2(qv.z, qv.w), make_float2(kf[v4 + 2], kf[v4 + 3]),
                                             make_float2(part[j][2], part[j][3]));
                part[j][0] = lo.x;
                part[j][1] = lo.y;
                part[j][2] = hi.x;
                part[j][3] = hi.y;
              }
            }
          }
#pragma unroll
          for (int j = 0; j < QPL; ++j) sc[j] = ((part[j][0] + part[j][1]) + (part[j][2] + part[j][3])) * M::SCALE;
          if constexpr (M::NTOK > 1) {
            // candidate t sees rows [0, start + t]: attend = start + ntok
            const int row = begin + tile * T + r0 + trow;
#pragma unroll
            for (int j = 0; j < QPL; ++j)
              if (row > si.attend - p.ntok + (hq0 + j) / M::G0) sc[j] = -INFINITY;
          }
        } else {
#pragma unroll
          for (int j = 0; j < QPL; ++j) sc[j] = -INFINITY;
        }
        // online softmax per head over this warp's rows (16-lane halves)
        float a_l[QPL], s_l[QPL], m_l[QPL];
#pragma unroll
        for (int j = 0; j < QPL; ++j) {
          const int g = hq0 + j;
          const float mt = half_max(sc[j]);
          float mold = m_run[0];
#pragma unroll
          for (int gg = 1; gg < G; ++gg)
            if (gg == g) mold = m_run[gg];
          const float mnew = fmaxf(mold, mt);
          a_l[j] = (mold == -INFINITY) ? 0.0f : softmax_exp(mold - mnew, pinned);
          // (a candidate may see none of these rows yet: then mnew is -inf too)
          const bool seen = M::NTOK == 1 ? trow < mine : (trow < mine && sc[j] != -INFINITY);
          const float pw = seen ? softmax_exp(sc[j] - mnew, pinned) : 0.0f;
          Pw[trow * G + g] = pw;
          s_l[j] = half_sum(pw);
          m_l[j] = mnew;
        }
        __syncwarp();
        // every lane needs (alpha, tile sum, new max) of all G heads; head g
        // lives in slot g % QPL of the lanes of half g / QPL.
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const int src = (g / QPL) * 16;
          const float a = __shfl_sync(0xffffffffu, a_l[g % QPL], src);
          const float ts = __shfl_sync(0xffffffffu, s_l[g % QPL], src);
          m_run[g] = __shfl_sync(0xffffffffu, m_l[g % QPL], src);
          l_run[g] = fmaf(l_run[g], a, ts);
#pragma unroll
          for (int e = 0; e < DPL; ++e) acc[g][e] *= a;
        }
        if constexpr (C::PVH) {
          // P.V: half-warp h2 takes rows h2, h2+2, ...; lane owns 4 dims of all G heads
          const int h2 = lane >> 4, dl = lane & 15;
          for (int tt = h2; tt < mine; tt += 2) {
            const float4 v4 = lds4<VT>(reinterpret_cast<const VT*>(vt + swz<C::BOX>(r0 + tt, dl * 4 * (int)sizeof(VT))));
            const float* prow = &Pw[tt * G];
#pragma unroll
            for (int g = 0; g < G; ++g) {
              const float2 pw = make_float2(prow[g], prow[g]);
              const float2 lo = __ffma2_rn(pw, make_float2(v4.x, v4.y), make_float2(acc[g][0], acc[g][1]));
              const float2 hi = __ffma2_rn(pw, make_float2(v4.z, v4.w), make_float2(acc[g][2], acc[g][3]));
              acc[g][0] = lo.x;
              acc[g][1] = lo.y;
              acc[g][2] = hi.x;
              acc[g][3] = hi.y;
            }
          }
        } else
        // P.V: lane owns dims [lane*DPL, lane*DPL + DPL) of all G heads
        for (int tt = 0; tt < mine; ++tt) {
          float vv[DPL];
          const VT* vrow = reinterpret_cast<const VT*>(vt + swz<C::BOX>(r0 + tt, lane * DPL * (int)sizeof(VT)));
#pragma unroll
          for (int e = 0; e < DPL; ++e) vv[e] = Elem<VT>::to_f32(vrow[e]);
          const float* prow = &Pw[tt * G];
#pragma unroll
          for (int g = 0; g < G; ++g) {
            const float pw = prow[g];
#pragma unroll
            for (int e = 0; e < DPL; ++e) acc[g][e] = fmaf(pw, vv[e], acc[g][e]);
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
    }
    // per-warp state for the merge
    if (lane == 0) {
#pragma unroll
      for (int g = 0; g < G; ++g) {
        stat[(warp * G + g) * 2] = m_run[g];
        stat[(warp * G + g) * 2 + 1] = l_run[g];
      }
    }
    if constexpr (C::PVH) {
      // fold the two half-warps (alternate rows) together
#pragma unroll
      for (int g = 0; g < G; ++g)
#pragma unroll
        for (int e = 0; e < DPL; ++e) acc[g][e] += __shfl_xor_sync(0xffffffffu, acc[g][e], 16);
    }
    // stash acc once every warp has left the stage buffers
    cta_sync();  // (A) whole CTA
    if (!s_flag[1]) {
      float* mbuf = reinterpret_cast<float*>(sm + C::OFF_K);  // [NWC][G][D]
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float mx = -INFINITY;
#pragma unroll
        for (int w = 0; w < NWC; ++w) mx = fmaxf(mx, stat[(w * G + g) * 2]);
        const float sc_w = (m_run[g] == -INFINITY) ? 0.0f : softmax_exp(m_run[g] - mx, pinned);
        if (!C::PVH || lane < 16) {
#pragma unroll
          for (int e = 0; e < DPL; ++e) mbuf[(warp * G + g) * D + (C::PVH ? (lane & 15) : lane) * DPL + e] = acc[g][e] * sc_w;
        }
      }
    }
  }
  if (warp == NWC) cta_sync();  // (A) for the producer warp
  cta_sync();                  // (B) merge buffer complete
  if (s_flag[1]) return;             // a bounded wait gave up; error recorded
  if (tid >= 128) return;             // the combine runs on the first 128 threads

  // ---- combine the warps: thread -> outputs (g, d) = idx / D, idx % D --------
  constexpr int OPT = G * D / 128;  // outputs per consumer thread
  const bool pinned = p.pinned_exp != 0;
  const float* mbuf = reinterpret_cast<const float*>(sm + C::OFF_K);
  float O[OPT], Mg[OPT], Lg[OPT];
#pragma unroll
  for (int k = 0; k < OPT; ++k) {
    const int idx = tid + k * 128, g = idx / D, d = idx % D;
    float mx = -INFINITY;
#pragma unroll
    for (int w = 0; w < NWC; ++w) mx = fmaxf(mx, stat[(w * G + g) * 2]);
    float L = 0.0f, o = 0.0f;
#pragma unroll
    for (int w = 0; w < NWC; ++w) {
      const float mw = stat[(w * G + g) * 2];
      if (mw != -INFINITY) L = fmaf(stat[(w * G + g) * 2 + 1], softmax_exp(mw - mx, pinned), L);
      o += mbuf[(w * G + g) * D + d];
    }
    O[k] = o;
    Mg[k] = mx;
    Lg[k] = L;
  }

  finish_outputs<G, D, HKV, HQ, OPT, M::NTOK, M::G0>(p, O, Mg, Lg, nsplit, s, cu, h, tid, warp, lane, pinned,
                                                    reinterpret_cast<float*>(sm + C::OFF_K), stat, s_flag);
}

template <class M, typename KT, typename VT>
__global__ void __launch_bounds__(DecodeCfg<M, KT, VT>::NT) qx_decode_kernel(const __grid_constant__ DecodeParams p) {
  decode_body<M, KT, VT>(p);
}

// The multi-token verify variant: its group of 8 query rows would hold one
// CTA per SM by registers; two resident CTAs keep more loads in flight.
template <typename KT, typename VT>
__global__ void __launch_bounds__(DecodeCfg<GraniteVerify4, KT, VT>::NT, 2)
    qx_verify_kernel(const __grid_constant__ DecodeParams p) {
  decode_body<GraniteVerify4, KT, VT>(p);
}

// ---- split merge as its own kernel (many splits) ----------------------------
// When a cache is cut into many splits, merging them in the last CTA of each
// kv head serialises a long chain of L2 reads on one CTA. Here four lanes
// share each output dim: lane q of the quad loads (m_i, l_i, O_i[d]) of
// splits i = q, q + 4, ... (kMergeLoads of them per pass, all in flight at
// once), and the quad combines its log-sum-exp terms with shuffles. The
// kernel has no shared memory and little code, so its CTAs can be resident
// beside the decode CTAs: it is launched as a programmatic dependent of the
// decode grid and waits for it (and its memory) in griddepcontrol.wait.
// Grid: one CTA per 32 output dims of one (call unit cu, kv head h, query
// head g of the group): blockIdx.x = ((cu * HKV + h) * G + g) * (D / 32) +
// dim block. The (cu, h) partial rows are found from the same sequence table
// the decode kernel used.
constexpr int kMergeLoads = 16;

// One pass of a quad's log-sum-exp merge: (mv, lv, ov)[k] are split
// q + 4k's (m, l, O[d]) of this pass (m = -inf, l = O = 0 past the last
// split); the quad's running (M, L, o) absorb them. The split merge kernel
// and the decode kernels' slice merge (tc_slice_merge) both run this, so
// they produce the same bits.
__device__ __forceinline__ void merge_quad_pass(const float* mv, const float* lv, const float* ov, bool pinned,
                                                float& M, float& L, float& o) {
  float mx = mv[0];
#pragma unroll
  for (int k = 1; k < kMergeLoads; ++k) mx = fmaxf(mx, mv[k]);
  mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
  mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
  const float Mn = fmaxf(M, mx);
  const float a = M == -INFINITY ? 0.0f : softmax_exp(M - Mn, pinned);
  float Ls = 0.0f, os = 0.0f;
#pragma unroll
  for (int k = 0; k < kMergeLoads; ++k) {
    const float w = mv[k] == -INFINITY ? 0.0f : softmax_exp(mv[k] - Mn, pinned);
    Ls = fmaf(w, lv[k], Ls);
    os = fmaf(w, ov[k], os);
  }
  Ls += __shfl_xor_sync(0xffffffffu, Ls, 1);
  os += __shfl_xor_sync(0xffffffffu, os, 1);
  Ls += __shfl_xor_sync(0xffffffffu, Ls, 2);
  os += __shfl_xor_sync(0xffffffffu, os, 2);
  L = fmaf(L, a, Ls);
  o = fmaf(o, a, os);
  M = Mn;
}

// KV-length split across GPUs: slice `slice` (32 dims) of query head qh of
// this rank's merged partial (quad lane 0 of quad dl holds o of dim
// slice * 32 + dl; every lane holds M and L) goes tagged into every rank's
// inbox; then the slices of all ranks are merged in rank order
// (qx_lse_merge's arithmetic) straight into p.xout. The peers' matching
// slices are being merged by grids that are one wave, so they are running
// too. Run by 128 threads whose barrier is `sync`; xs is 17 floats of
// shared memory. A CTA whose own merge gave up (local_ok false on any
// thread) pushes nothing and fails the peer group, as a timed-out exchange
// does (mark_peer_group_failed).
template <int D, int HQ, class Sync>
__device__ __forceinline__ void exchange_slice(const DecodeParams& p, long long cu, long long qh, int slice, float o,
                                               float M, float L, bool local_ok, int tid, bool pinned, float* xs,
                                               Sync sync) {
  constexpr int S = D / 32, ROW = 34;
  const int q = tid & 3, dl = tid >> 2;
  float* xml = xs;  // m_r, l_r of up to 8 ranks
  volatile int* xok = reinterpret_cast<volatile int*>(xs + 16);
  // an earlier exchange on this group timed out: push nothing (one thread
  // reads the word, so the whole CTA takes one branch)
  if (tid == 0) *xok = peer_group_failed(p.xfailed) ? 0 : 1;
  sync();
  if (!local_ok) *xok = 0;
  sync();
  if (!*xok) {
    if (tid == 0) {
      flag_error(p.err, QX_ERR_BIT_TIMEOUT | QX_ERR_BIT_PEER);
      mark_peer_group_failed(p.xfailed, p.xfailed_host);
    }
    return;
  }
  const int W = p.xworld;
  unsigned* stp = p.xstep + qh * S + slice;
  const unsigned st = *stp, tag = st + 1u, half = st & 1u;
  const long long rows = (long long)HQ * S;
  const long long mine = ((long long)half * W + p.xrank) * rows + qh * S + slice;
  if (q == 0)
    for (int r = 0; r < W; ++r) st_tagged(p.xinbox[r] + mine * ROW + dl, o, tag);
  if (tid == 0)
    for (int r = 0; r < W; ++r) {
      st_tagged(p.xinbox[r] + mine * ROW + 32, M, tag);
      st_tagged(p.xinbox[r] + mine * ROW + 33, L, tag);
    }
  const uint2* in = p.xinbox[p.xrank] + ((long long)half * W * rows + qh * S + slice) * ROW;
  bool ok = true;
  float ov[8];
#pragma unroll
  for (int r = 0; r < 8; ++r) ov[r] = 0.0f;
  if (tid < 32) {
    // dim tid of every rank's slice, and lanes 0 .. 2W-1 also (m, l) of
    // rank tid / 2, all polled together
    float v = 0.0f;
    const uint2* ml = tid < 2 * W ? in + (tid >> 1) * rows * ROW + 32 + (tid & 1) : nullptr;
    ok = wait_tagged_n<8>(in + tid, rows * ROW, W, ml, tag, ov, &v);
    if (tid < 2 * W) xml[tid] = v;
  }
  if (!ok) {
    flag_error(p.err, QX_ERR_BIT_TIMEOUT | QX_ERR_BIT_PEER);
    mark_peer_group_failed(p.xfailed, p.xfailed_host);
    *xok = 0;
  }
  sync();
  if (!*xok) return;
  if (tid < 32) {
    float mx = -INFINITY;
    for (int r = 0; r < W; ++r) mx = fmaxf(mx, xml[2 * r]);
    float Lt = 0.0f, Ot = 0.0f;
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      if (r >= W) break;
      const float m = xml[2 * r];
      if (m == -INFINITY) continue;  // empty shard
      const float w = softmax_exp(m - mx, pinned);
      Lt = fmaf(w, xml[2 * r + 1], Lt);
      Ot = fmaf(w, ov[r], Ot);
    }
    const float v = Ot / Lt;
    if (!isfinite(v)) flag_error(p.err, QX_ERR_BIT_NONFINITE);
    store_any(p.xout, (cu * HQ + qh) * D + slice * 32 + tid, p.xout_dtype, v);
  }
  if (tid == 0) *stp = st + 1u;
}

// The splits of one (unit cu, kv head h) merge their partials among
// themselves, with no second grid: every split stores its (O, m, l) as tagged
// values (st_tagged), then split s takes the 32-dim output slices s,
// s + nsplit, ... of the group's G x D outputs and merges each as
// qx_split_merge_kernel does (four lanes per dim, one merge_quad_pass over
// at most 4 x kMergeLoads splits), polling the tagged values it reads; the
// outputs equal that kernel's bit for bit. On a KV length split across GPUs
// (p.xworld) each merged slice then goes through exchange_slice, as in that
// kernel, with xs (17 floats of shared memory) as its scratch. A split
// waits for the others, so every CTA of the grid must be resident at once:
// the host takes this path only for a grid of one wave. Each wait is
// bounded (kMaxWaitNs); a timeout sets QX_ERR_BIT_TIMEOUT and leaves the
// slice unwritten. Run by 128 threads (barrier 1), thread t holding dim t
// of every head (O[k], and Mg[k], Lg[k] of head k).
template <int G, int D, int HQ>
__device__ __forceinline__ void slice_merge(const DecodeParams& p, const float* O, const float* Mg, const float* Lg,
                                            int nsplit, int s, long long cu, int h, int tid, bool pinned, float* xs) {
  static_assert(D == 128, "thread t holds dim t of every head");
  const unsigned tag = p.merge_tag;
  const long long stride = (long long)G * (D + 2);
  uint2* mine = p.tpartials + (long long)blockIdx.x * stride;
#pragma unroll
  for (int k = 0; k < G; ++k) st_tagged(mine + k * (D + 2) + tid, O[k], tag);
  if (tid < G) {
    float m = Mg[0], l = Lg[0];
#pragma unroll
    for (int k = 1; k < G; ++k)
      if (k == tid) {
        m = Mg[k];
        l = Lg[k];
      }
    st_tagged(mine + tid * (D + 2) + D, m, tag);
    st_tagged(mine + tid * (D + 2) + D + 1, l, tag);
  }
  const uint2* first = p.tpartials + (long long)(blockIdx.x - s) * stride;
  const int q = tid & 3, dl = tid >> 2;
  constexpr int SLICES = G * (D / 32);
  bool failed = false;
  for (int j = s; j < SLICES; j += nsplit) {
    const int g = j / (D / 32), d = (j % (D / 32)) * 32 + dl;
    const uint2* base = first + (long long)g * (D + 2);
    uint2 mt[kMergeLoads], lt[kMergeLoads], ot[kMergeLoads];
#pragma unroll
    for (int k = 0; k < kMergeLoads; ++k) {
      const int i = q + 4 * k;
      if (i < nsplit && !failed) {
        mt[k] = ld_tagged(base + i * stride + D);
        lt[k] = ld_tagged(base + i * stride + D + 1);
        ot[k] = ld_tagged(base + i * stride + d);
      } else {
        mt[k] = make_uint2(__float_as_uint(-INFINITY), tag);
        lt[k] = ot[k] = make_uint2(0u, tag);
      }
    }
    // every value still missing is loaded again, all in flight together
    unsigned long long t0 = 0;
    for (unsigned spins = 0;; ++spins) {
      bool all = true;
#pragma unroll
      for (int k = 0; k < kMergeLoads; ++k) all &= mt[k].y == tag && lt[k].y == tag && ot[k].y == tag;
      if (all || failed) break;
#pragma unroll
      for (int k = 0; k < kMergeLoads; ++k) {
        const int i = q + 4 * k;  // (values past the last split carry the tag already)
        if (mt[k].y != tag) mt[k] = ld_tagged(base + i * stride + D);
        if (lt[k].y != tag) lt[k] = ld_tagged(base + i * stride + D + 1);
        if (ot[k].y != tag) ot[k] = ld_tagged(base + i * stride + d);
      }
      if ((spins & 15u) == 0u) {
        const unsigned long long now = global_ns();
        if (t0 == 0) t0 = now;
        else if (now - t0 > kMaxWaitNs) failed = true;
      }
    }
    float mv[kMergeLoads], lv[kMergeLoads], ov[kMergeLoads];
#pragma unroll
    for (int k = 0; k < kMergeLoads; ++k) {
      mv[k] = __uint_as_float(mt[k].x);
      lv[k] = __uint_as_float(lt[k].x);
      ov[k] = __uint_as_float(ot[k].x);
    }
    float M = -INFINITY, L = 0.0f, o = 0.0f;
    merge_quad_pass(mv, lv, ov, pinned, M, L, o);
    if (p.xworld) {
      // KV-length split across GPUs: this slice of this rank's merge goes
      // to every rank and the ranks' slices are merged into p.xout
      exchange_slice<D, HQ>(p, cu, (long long)h * G + g, j % (D / 32), o, M, L, !failed, tid, pinned, xs,
                            [] { consumers_sync(128); });
      consumers_sync(128);  // xs is free for the next slice
    } else if (failed) {
      flag_error(p.err, QX_ERR_BIT_TIMEOUT);
    } else if (q == 0) {
      const float v = o / L;
      if (!isfinite(v)) flag_error(p.err, QX_ERR_BIT_NONFINITE);
      store_any(p.out, out_elem<G, D, HQ, 1, G>(p, cu, h, g, d), p.out_dtype, v);
    }
  }
}

template <int G, int D, int HKV, int HQ, int NTOK = 1, int G0 = G>
__global__ void __launch_bounds__(128) qx_split_merge_kernel(const __grid_constant__ DecodeParams p) {
  const int tid = threadIdx.x, q = tid & 3;
  const int blk = blockIdx.x;
  const int d = (blk % (D / 32)) * 32 + (tid >> 2);
  const int row = blk / (D / 32);
  const int g = row % G, uh = row / G;
  const int h = uh % HKV;
  const long long cu = uh / HKV;
  StageTrace trace(p.trace, blk, tid == 0);
  pdl_launch_dependents();  // the next grid may get resident meanwhile
  pdl_wait();  // the decode grid's partials
  trace.mark();  // start
  const int slot = (int)(cu / p.layer_count), lloc = (int)(cu % p.layer_count);
  const SeqInfo si = p.seq_table ? p.seq_table[slot] : p.single;
  const int n = (si.attend + p.chunk - 1) / p.chunk;
  if (n <= 1 && !p.xworld) return;  // the decode kernel wrote this head's output itself
  const long long item0 = si.item_begin + (long long)(lloc * HKV + h) * n;
  const float* first = p.partials + item0 * G * (D + 2) + (long long)g * (D + 2);
  const long long stride = (long long)G * (D + 2);
  const bool pinned = p.pinned_exp != 0;
  float M = -INFINITY, L = 0.0f, o = 0.0f;
  for (int base = 0; base < n; base += 4 * kMergeLoads) {
    float mv[kMergeLoads], lv[kMergeLoads], ov[kMergeLoads];
#pragma unroll
    for (int k = 0; k < kMergeLoads; ++k) {
      const int i = base + q + 4 * k;
      const float* pi = first + (long long)i * stride;
      mv[k] = i < n ? __ldcg(pi + D) : -INFINITY;
      lv[k] = i < n ? __ldcg(pi + D + 1) : 0.0f;
      ov[k] = i < n ? __ldcg(pi + d) : 0.0f;
    }
    merge_quad_pass(mv, lv, ov, pinned, M, L, o);
  }
  if (p.xworld) {
    __shared__ float xml[17];  // m_r, l_r of up to 8 ranks; [16]: the CTA's go-ahead
    exchange_slice<D, HQ>(p, cu, (long long)h * G + g, blk % (D / 32), o, M, L, true, tid, pinned, xml,
                          [] { __syncthreads(); });
    return;
  }
  if (q == 0) {
    const long long qh = (long long)h * G + g;
    if (p.emit_partials) {
      float* dst = reinterpret_cast<float*>(p.out) + (cu * HQ + qh) * (D + 2);
      dst[d] = o;
      if (d == 0) {
        dst[D] = M;
        dst[D + 1] = L;
      }
    } else if (NTOK == 1 || g / G0 < p.ntok) {
      const float v = o / L;
      if (!isfinite(v)) flag_error(p.err, QX_ERR_BIT_NONFINITE);
      store_any(p.out, out_elem<G, D, HQ, NTOK, G0>(p, cu, h, g, d), p.out_dtype, v);
    }
  }
  trace.mark();  // done
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
static __global__ void qx_granite_rope_kernel(float* q, float* k, int position, unsigned* err) {
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
