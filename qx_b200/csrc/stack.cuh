// stack.cuh — the attention sub-layers of a stack of Granite layers with Q4
// weights, for one token, in ONE persistent kernel.
//
// Per layer the reference runs (PreparedAttentionStack::encode,
// crates/qx-runtime-v2/src/lib.rs:1793-1821, each layer
// GpuRuntimeBuffers::encode_attention_layer :6916-6994):
//
//   x         = cpu_rms_norm_simd(hidden, input_norm)
//   q, k, v   = Q4 mat-vecs of x (mat_vec_simd32 lane order)
//   attention = RoPE (the fma pair), KV append at `position`, GQA attention
//   hidden'   = fma(0.22, o_proj(attention), hidden)
//
// Every step needs the whole result of the one before (the RMS all of
// hidden, the o-projection all 16 heads), so as separate launches the chain
// is four small latency-bound grids per layer. Here one CTA per SM (a
// cooperative launch: every CTA is resident) walks all the layers, and the
// CTAs hand their results to one another through global memory:
//
//   A  CTAs with q/k/v rows: RMSNorm of hidden(i) (each computes it, in the
//      reference's order), then their contiguous slice of the 2048 q/k/v
//      rows from Q4 weights staged in shared memory (bulk copies issued two
//      layers ahead into a double buffer).
//   B  CTAs with an attention item (kv head h, split s of the cache, at
//      most 256 rows): every lane takes its row's key into registers while
//      q is on its way; RoPE of q (and, on the split holding the new slot,
//      of k); append the new row; (m, l, O) of both query heads. A ticket per
//      kv head, counted up for good, elects the last of the head's items to
//      finish, which merges the head's splits into 128 values of the
//      attention vector.
//   C  CTAs with o-projection rows: the attention vector, their rows of the
//      o-projection and the residual: their part of hidden(i + 1). The
//      residual's input rows come from the CTA's own copy of hidden(i) in
//      shared memory (taken in A), not from a second global load.
//
// The next layer's cache rows (16.8 MB of fp32 KV at 4096 positions) are
// prefetched from HBM into L2 as soon as a layer's attention is done and
// copied on into shared memory (TMA) in two parts, a quarter at the layer's
// end and the rest once the next hidden state has arrived, so the HBM
// stream runs under the dependent steps. Only L2-to-SM bytes, not HBM-to-SM
// ones, then queue ahead of the hand-off loads on the same SM, and few of
// them ahead of the hidden-state poll.
//
// Hand-offs carry no fence and no counter: every 32-bit value travels with a
// 32-bit tag (this launch's generation and the layer) in one 8-byte store,
// which a reader sees whole or not at all, and the reader polls the value
// itself until its tag is the expected one: the poll is the load of the
// data. (A fence here would wait behind the CTA's own bulk copies in
// flight: microseconds.) A buffer is only rewritten (the next layer's tag)
// once every reader of its current contents has passed a point the writer
// depends on, so a reader never sees a later tag than the one it waits for.
// Every poll is bounded: after kMaxWaitNs, or once another CTA has raised
// the shared abort word, the CTA records QX_ERR_BIT_TIMEOUT, raises the
// word, waits (bounded) for its own copies in flight and leaves; the host
// clears the word (and the tickets) when it reports the error.
//
// Arithmetic: RMSNorm, q/k/v and the o-projection are bit-identical to the
// reference's CPU routines (layer.cuh's order); RoPE is qx's pinned sin/cos
// with the fma pair, bit-identical; the attention and the split merge are
// fp32 with qx's pinned exp (the decode kernel's tolerance, 1e-5 normwise).
#pragma once
#include "decode.cuh"
#include "layer.cuh"

namespace qx {

constexpr int kStackThreads = 256;
constexpr int kStackMaxLayers = 32;    // layers per launch (the host chains launches beyond)
constexpr int kStackTileRows = 64;
constexpr int kStackMaxTiles = 4;      // cached rows per attention item <= 256
constexpr int kStackMaxSplits = 16;    // items = 8 kv heads x splits <= 128
constexpr int kStackMaxQkvRows = 16;   // q/k/v rows per CTA (2048 / CTAs, at least 128 CTAs)
constexpr int kStackMaxORows = 8;      // o-projection rows per CTA (one per warp)
constexpr int kStackPartial = 2 * 66;  // values per item: (O[64], m, l) for both query heads

struct StackLayerW {
  const float* norm;           // [1024] input RMSNorm weight
  const uint8_t* codes[4];     // q [1024], k [512], v [512], o [1024] rows x 512 bytes
  const uint16_t* scales[4];   // rows x 32 FP16
};

struct StackParams {
  CUtensorMap tmk, tmv;  // the arena's key / value maps (decode.cuh layout)
  char* k_region;
  char* v_region;
  int capacity, arena_layers, seq;
  int layer_begin, n_layers;
  int position;           // the new token's slot in every layer; attend = position + 1
  int chunk, nsplit;      // cached rows per attention item (multiple of 64), splits per kv head
  unsigned gen;           // this launch's generation: tag of layer i = gen * 64 + i + 1
  const float* hidden_in;
  float* hidden_out;
  // tagged exchange buffers ({value bits, tag})
  uint2* hx;              // [2][1024] hidden between layers
  uint2* qx;              // [2048] q, k, v
  uint2* px;              // [8 * nsplit][kStackPartial] tagged split partials
  unsigned* tickets;      // [8] per kv head: items done, counted up for good (never reset)
  unsigned ticket_base;   // every head's ticket count when this launch starts
  uint2* ax;              // [1024] the merged attention vector
  unsigned* abort;        // raised by a CTA whose wait gave up
  int pinned_exp;
  unsigned* err;
  unsigned long long* trace;
  StackLayerW w[kStackMaxLayers];
};

struct StackCfg {
  static constexpr int BOX = kStackTileRows * 128;      // one [64 rows][128 B] swizzled box
  static constexpr int TILE = 2 * BOX;                  // 64 fp32 dims of 64 rows
  static constexpr int OFF_K = 0;
  static constexpr int OFF_V = OFF_K + kStackMaxTiles * TILE;
  static constexpr int QKV_CODES = kStackMaxQkvRows * 512, O_CODES = kStackMaxORows * 512;
  static constexpr int QKV_SCALES = kStackMaxQkvRows * 64, O_SCALES = kStackMaxORows * 64;
  static constexpr int NORM = 1024 * 4;
  static constexpr int WBUF = QKV_CODES + O_CODES + QKV_SCALES + O_SCALES + NORM;  // one layer's weights of a CTA
  static constexpr int OFF_W = OFF_V + kStackMaxTiles * TILE;
  static constexpr int OFF_X = OFF_W + 2 * WBUF;        // float [1024]: normalized hidden, then attention
  static constexpr int OFF_Q = OFF_X + 1024 * 4;        // float [2][64] rotated q; [64] new k; [64] new v
  static constexpr int OFF_WO = OFF_Q + 256 * 4;        // float [8 warps][2][64] warp partial O
  static constexpr int OFF_WML = OFF_WO + 8 * 2 * 64 * 4;  // float [8][2][2] warp (m, l), then weights, M, L
  static constexpr int OFF_MW = OFF_WML + 64 * 4;       // float [2][16] merge weights, [2] L
  static constexpr int OFF_RED = OFF_MW + 64 * 4;       // float [8] warp sums, [1] scale
  static constexpr int OFF_ROPE = OFF_RED + 64;         // float [32][2] (sin, cos) at the position, int ok, KV counts
  static constexpr int OFF_H = OFF_ROPE + 288;          // float [1024] this layer's input hidden (the residual)
  static constexpr int OFF_BAR = OFF_H + 1024 * 4;      // 3 mbarriers: KV, weights 0, weights 1
  static constexpr int SMEM = OFF_BAR + 32 + 1024;      // + slack to align the base to 1024
};
static_assert(StackCfg::SMEM <= 227 * 1024, "the stack kernel's shared memory must fit one SM");

// 1-D bulk copy global -> shared (16-byte aligned addresses, size a
// multiple of 16), completing on `bar`'s transaction count.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_addr(dst)),
               "l"(src), "r"(bytes), "r"(smem_addr(bar))
               : "memory");
}

// Poll state of one thread: when it first had to wait, and how often.
struct StackPoll {
  unsigned long long t0 = 0;
  unsigned spins = 0;
  bool failed = false;
};

// Wait until the tagged value at `x` carries `tag`; its value. On a timeout
// (or the abort word raised by another CTA) marks the poll failed, raises
// the abort word and returns 0.
__device__ __forceinline__ float stack_take(const StackParams& p, const uint2* x, unsigned tag, StackPoll& st) {
  uint2 v = ld_tagged(x);
  while (v.y != tag && !st.failed) {
    if ((++st.spins & 63u) == 0u) {
      const unsigned long long now = global_ns();
      if (st.t0 == 0) st.t0 = now;
      if (*reinterpret_cast<volatile unsigned*>(p.abort) != 0u) {
        st.failed = true;
      } else if (now - st.t0 > kMaxWaitNs) {
        *reinterpret_cast<volatile unsigned*>(p.abort) = 1u;
        flag_error(p.err, QX_ERR_BIT_TIMEOUT);
        st.failed = true;
      }
    }
    v = ld_tagged(x);
  }
  return st.failed ? 0.0f : __uint_as_float(v.x);
}

// N tagged values x[0], x[stride], ... (the first `count` of them): every
// load is issued before the first is tested, so values that are already
// there cost one round trip together; only those not yet tagged are polled
// again. Values past `count` read as 0.
template <int N>
__device__ __forceinline__ void stack_take_n(const StackParams& p, const uint2* x, long long stride, int count,
                                             unsigned tag, float* out, StackPoll& st) {
  uint2 v[N];
#pragma unroll
  for (int k = 0; k < N; ++k) v[k] = k < count ? ld_tagged(x + k * stride) : make_uint2(0u, tag);
  for (;;) {
    bool all = true;
#pragma unroll
    for (int k = 0; k < N; ++k) all &= v[k].y == tag;
    if (all || st.failed) break;
    // every value still missing is loaded again, all in flight together
#pragma unroll
    for (int k = 0; k < N; ++k)
      if (v[k].y != tag) v[k] = ld_tagged(x + k * stride);
    if ((++st.spins & 15u) == 0u) {
      const unsigned long long now = global_ns();
      if (st.t0 == 0) st.t0 = now;
      if (*reinterpret_cast<volatile unsigned*>(p.abort) != 0u) {
        st.failed = true;
      } else if (now - st.t0 > kMaxWaitNs) {
        *reinterpret_cast<volatile unsigned*>(p.abort) = 1u;
        flag_error(p.err, QX_ERR_BIT_TIMEOUT);
        st.failed = true;
      }
    }
  }
#pragma unroll
  for (int k = 0; k < N; ++k) out[k] = st.failed ? 0.0f : __uint_as_float(v[k].x);
}

// One Q4 row (1024 columns) of shared-memory codes/scales against x (shared),
// by a warp in mat_vec_simd32's order: lane l accumulates columns l, l + 32,
// ... by fma and the lanes reduce as (16, 8, 4, 2, 1). Sum in lane 0.
__device__ __forceinline__ float q4_row_dot_smem(const uint8_t* codes, const uint16_t* scales, const float* x,
                                                 int lane) {
  float acc = 0.0f;
  const int byte = lane >> 1, shift = (lane & 1) * 4;
#pragma unroll 8
  for (int j = 0; j < 32; ++j) {
    const float sc = __half2float(__ushort_as_half(scales[j]));
    const int code = (codes[j * 16 + byte] >> shift) & 0xF;
    const float value = __fmul_rn((float)(code - 7), sc);
    acc = __fmaf_rn(value, x[j * 32 + lane], acc);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, off));
  return acc;
}

// Two rows at once (two independent chains, the same order for each).
__device__ __forceinline__ void q4_row_dot2_smem(const uint8_t* c0, const uint16_t* s0, const uint8_t* c1,
                                                 const uint16_t* s1, const float* x, int lane, float* y0,
                                                 float* y1) {
  float a0 = 0.0f, a1 = 0.0f;
  const int byte = lane >> 1, shift = (lane & 1) * 4;
#pragma unroll 8
  for (int j = 0; j < 32; ++j) {
    const float xv = x[j * 32 + lane];
    const float v0 =
        __fmul_rn((float)(((c0[j * 16 + byte] >> shift) & 0xF) - 7), __half2float(__ushort_as_half(s0[j])));
    const float v1 =
        __fmul_rn((float)(((c1[j * 16 + byte] >> shift) & 0xF) - 7), __half2float(__ushort_as_half(s1[j])));
    a0 = __fmaf_rn(v0, xv, a0);
    a1 = __fmaf_rn(v1, xv, a1);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    a0 = __fadd_rn(a0, __shfl_down_sync(0xffffffffu, a0, off));
    a1 = __fadd_rn(a1, __shfl_down_sync(0xffffffffu, a1, off));
  }
  *y0 = a0;
  *y1 = a1;
}

// Byte offset of fp32 dim d of row r inside a [2 boxes][64 rows][128 B]
// swizzled tile (chunk c of row r sits at chunk c ^ (r & 7) of its box).
__device__ __forceinline__ int stack_swz(int r, int d) {
  const int b = d * 4;
  return (b >> 7) * StackCfg::BOX + r * 128 + ((((b & 127) >> 4) ^ (r & 7)) << 4) + (b & 15);
}

__device__ __forceinline__ void stack_raise(const StackParams& p, StackPoll& poll) {
  *reinterpret_cast<volatile unsigned*>(p.abort) = 1u;
  poll.failed = true;
}

__global__ void __launch_bounds__(kStackThreads, 1) qx_attention_stack_kernel(const __grid_constant__ StackParams p) {
  using C = StackCfg;
  extern __shared__ __align__(1024) unsigned char sm_raw[];
  unsigned char* sm = sm_raw + ((1024u - (smem_addr(sm_raw) & 1023u)) & 1023u);
  unsigned char* ks = sm + C::OFF_K;
  unsigned char* vs = sm + C::OFF_V;
  float* xs = reinterpret_cast<float*>(sm + C::OFF_X);
  float* hs = reinterpret_cast<float*>(sm + C::OFF_H);
  float* qs = reinterpret_cast<float*>(sm + C::OFF_Q);  // [2][64]
  float* newk = qs + 128;
  float* newv = qs + 192;
  float* wo = reinterpret_cast<float*>(sm + C::OFF_WO);
  float* wml = reinterpret_cast<float*>(sm + C::OFF_WML);
  float* mw = reinterpret_cast<float*>(sm + C::OFF_MW);  // [2][16], then L [2]
  float* red = reinterpret_cast<float*>(sm + C::OFF_RED);
  float* rope = reinterpret_cast<float*>(sm + C::OFF_ROPE);  // [32][2] sin, cos
  int* rope_ok = reinterpret_cast<int*>(rope + 64);
  uint64_t* bar_kv = reinterpret_cast<uint64_t*>(sm + C::OFF_BAR);
  uint64_t* bar_w = bar_kv + 1;  // [2]

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int NB = gridDim.x, b = blockIdx.x;
  const int n = p.n_layers;
  const int attend = p.position + 1;
  const bool pinned = p.pinned_exp != 0;
  StageTrace trace(p.trace, b, tid == 0);

  // this CTA's rows: q/k/v [rq0, rq1) of 2048, o [ro0, ro1) of 1024
  const int rq_per = (2048 + NB - 1) / NB, ro_per = (1024 + NB - 1) / NB;
  const int rq0 = min(2048, b * rq_per), rq1 = min(2048, rq0 + rq_per);
  const int ro0 = min(1024, b * ro_per), ro1 = min(1024, ro0 + ro_per);
  const bool has_q = rq1 > rq0, has_o = ro1 > ro0;
  // attention item: kv head h, split s
  const int items = 8 * p.nsplit;
  const bool has_item = b < items;
  const int h = has_item ? b / p.nsplit : 0, s = has_item ? b % p.nsplit : 0;
  const int begin = s * p.chunk, end = min(begin + p.chunk, attend);
  const int ntiles = has_item ? (end - begin + kStackTileRows - 1) / kStackTileRows : 0;
  const bool owner = has_item && p.position >= begin && p.position < end;
  if (!has_q && !has_o && !has_item) return;  // no part in any hand-off

  if (tid == 0) {
    mbar_init(bar_kv, 1);
    mbar_init(&bar_w[0], 1);
    mbar_init(&bar_w[1], 1);
    fence_barrier_init();
    *rope_ok = 1;
  }
  __syncthreads();
  if (tid < 32) {
    // qx's pinned sin/cos of the 32 rotation pairs at the token's position
    // (the same for every layer)
    float sn = 0.f, cs = 0.f;
    if (!granite_sin_cos((uint32_t)p.position, tid, &sn, &cs)) *rope_ok = 0;
    rope[2 * tid] = sn;
    rope[2 * tid + 1] = cs;
  }
  pdl_wait();  // (a programmatic dependent launch: earlier grids' memory is visible from here)
  trace.mark();

  // copies in flight: KV fills are issued by thread kKvIssuer and waited
  // for by thread 0 (the counts meet in shared memory at the end); weight
  // fills per buffer are issued and waited for by thread 0
  constexpr int kKvIssuer = 224;  // warp 7: idle while the merge and the partial run
  int* kv_count = reinterpret_cast<int*>(rope_ok + 1);  // [0] issued, [1] waited
  int kv_issued = 0, kv_waited = 0;
  int w_issued[2] = {0, 0}, w_waited[2] = {0, 0};

  // This item's rows of layer i into shared memory, in one barrier phase.
  // part 0: every K and V tile. part 1 (issued at the end of layer i - 1):
  // the first kStackEarlyKTiles K tiles, and the expected byte count of the
  // whole phase. part 2 (issued once layer i's hidden state has arrived):
  // the other K tiles and all V tiles. Each part's L2-to-shared bytes queue
  // ahead of the hand-off loads the CTA issues next: a quarter of the rows
  // ahead of the hidden-state poll, the rest beside the q/k/v mat-vec.
  constexpr int kStackEarlyKTiles = 2;
  auto issue_kv = [&](int i, int part) {
    if (!has_item) return;
    fence_proxy_async_shared();  // generic writes to the tiles (the appended row) before the async ones
    const int layer = p.layer_begin + i;
    if (part != 2) mbar_arrive_expect_tx(bar_kv, (uint32_t)(ntiles * 2 * C::TILE));
    for (int t = 0; t < ntiles; ++t) {
      const int z = (int)(((long long)p.seq * p.arena_layers + layer) * p.capacity + begin + t * kStackTileRows);
      const bool k_now = part == 0 || (part == 1) == (t < kStackEarlyKTiles);
#pragma unroll
      for (int bx = 0; bx < 2; ++bx) {
        if (k_now) tma_load_3d(ks + t * C::TILE + bx * C::BOX, &p.tmk, bx * 32, h, z, bar_kv);
        if (part != 1) tma_load_3d(vs + t * C::TILE + bx * C::BOX, &p.tmv, bx * 32, h, z, bar_kv);
      }
    }
    if (part != 2) ++kv_issued;
  };
  auto prefetch_kv = [&](int i) {  // this item's rows of layer i into L2
    if (!has_item) return;
    const int layer = p.layer_begin + i;
    for (int t = 0; t < ntiles; ++t) {
      const int z = (int)(((long long)p.seq * p.arena_layers + layer) * p.capacity + begin + t * kStackTileRows);
#pragma unroll
      for (int bx = 0; bx < 2; ++bx) {
        tma_prefetch_3d(&p.tmk, bx * 32, h, z);
        tma_prefetch_3d(&p.tmv, bx * 32, h, z);
      }
    }
  };
  auto issue_w = [&](int i) {  // thread 0: this CTA's norm, q/k/v and o rows of layer i into buffer i & 1
    if (!has_q && !has_o) return;
    unsigned char* wb = sm + C::OFF_W + (i & 1) * C::WBUF;
    const StackLayerW& lw = p.w[i];
    fence_proxy_async_shared();
    mbar_arrive_expect_tx(&bar_w[i & 1], (uint32_t)((rq1 - rq0) + (ro1 - ro0)) * 576u + (has_q ? C::NORM : 0u));
    // q/k/v rows: up to two matrices (q: rows 0-1023, k: 1024-1535, v: 1536-2047)
    for (int r = rq0; r < rq1;) {
      const int m = r < 1024 ? 0 : (r < 1536 ? 1 : 2);
      const int base = m == 0 ? 0 : (m == 1 ? 1024 : 1536);
      const int lim = m == 0 ? 1024 : (m == 1 ? 1536 : 2048);
      const int e = min(rq1, lim);
      bulk_load(wb + (r - rq0) * 512, lw.codes[m] + (size_t)(r - base) * 512, (uint32_t)(e - r) * 512u,
                &bar_w[i & 1]);
      bulk_load(wb + C::QKV_CODES + C::O_CODES + (r - rq0) * 64, lw.scales[m] + (size_t)(r - base) * 32,
                (uint32_t)(e - r) * 64u, &bar_w[i & 1]);
      r = e;
    }
    if (has_o) {
      bulk_load(wb + C::QKV_CODES, lw.codes[3] + (size_t)ro0 * 512, (uint32_t)(ro1 - ro0) * 512u, &bar_w[i & 1]);
      bulk_load(wb + C::QKV_CODES + C::O_CODES + C::QKV_SCALES, lw.scales[3] + (size_t)ro0 * 32,
                (uint32_t)(ro1 - ro0) * 64u, &bar_w[i & 1]);
    }
    if (has_q)
      bulk_load(wb + C::QKV_CODES + C::O_CODES + C::QKV_SCALES + C::O_SCALES, lw.norm, C::NORM, &bar_w[i & 1]);
    ++w_issued[i & 1];
  };
  // thread 0: the next weight fill of buffer j (bounded); false on timeout
  auto wait_w = [&](int j) -> bool {
    if (!has_q && !has_o) return true;
    if (!mbar_wait_bounded(&bar_w[j], (uint32_t)(w_waited[j] & 1), p.err)) return false;
    ++w_waited[j];
    return true;
  };

  if (tid == kKvIssuer) issue_kv(0, 0);
  if (tid == 0) {
    issue_w(0);
    if (n > 1) issue_w(1);
  }

  StackPoll poll;
  bool ok = true;  // uniform across the CTA
  for (int i = 0; i < n && ok; ++i) {
    const unsigned tag = p.gen * 64u + (unsigned)i + 1u;
    const uint2* hin_x = p.hx + ((i - 1) & 1) * 1024;  // tagged input hidden (layers after the first)
    uint2* hout_x = p.hx + (i & 1) * 1024;
    unsigned char* wb = sm + C::OFF_W + (i & 1) * C::WBUF;
    const uint8_t* wq_codes = wb;
    const uint8_t* wo_codes = wb + C::QKV_CODES;
    const uint16_t* wq_scales = reinterpret_cast<const uint16_t*>(wb + C::QKV_CODES + C::O_CODES);
    const uint16_t* wo_scales = wq_scales + C::QKV_SCALES / 2;
    const float* norm_s =
        reinterpret_cast<const float*>(wb + C::QKV_CODES + C::O_CODES + C::QKV_SCALES + C::O_SCALES);

    // ---- A: RMSNorm and this CTA's q/k/v rows --------------------------------
    if (has_q || has_o) {
      if (tid == 0 && !wait_w(i & 1)) stack_raise(p, poll);
      if (!has_q && __syncthreads_or(poll.failed)) {
        ok = false;
        break;
      }
    }
    if (has_q) {
      float hv[4];
      if (i == 0) {
#pragma unroll
        for (int k = 0; k < 4; ++k) hv[k] = __ldg(p.hidden_in + tid + 256 * k);
      } else {
        stack_take_n<4>(p, hin_x + tid, 256, 4, tag - 1u, hv, poll);
      }
      if (__syncthreads_or(poll.failed)) {
        ok = false;
        break;
      }
      if (tid == kKvIssuer && i > 0) issue_kv(i, 2);  // the rest of this layer's rows
#pragma unroll
      for (int k = 0; k < 4; ++k) hs[tid + 256 * k] = hv[k];  // the residual's input, for C
      trace.mark();
      // cpu_rms_norm_simd: thread t sums x[t], x[t + 256], ... by fma; the
      // warps, then the 8 warp sums, reduce as reduce_simd32
      float sum = 0.0f;
#pragma unroll
      for (int k = 0; k < 4; ++k) sum = __fmaf_rn(hv[k], hv[k], sum);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) sum = __fadd_rn(sum, __shfl_down_sync(0xffffffffu, sum, off));
      if (lane == 0) red[warp] = sum;
      __syncthreads();
      if (warp == 0) {
        float g = lane < 8 ? red[lane] : 0.0f;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) g = __fadd_rn(g, __shfl_down_sync(0xffffffffu, g, off));
        if (lane == 0) {
          float scale = 0.0f;
          if (!pinned_rsqrt(__fadd_rn(__fdiv_rn(g, (float)kHidden), kRmsEpsilon), &scale))
            flag_error(p.err, QX_ERR_BIT_NONFINITE);
          red[8] = scale;
        }
      }
      __syncthreads();
      const float scale = red[8];
#pragma unroll
      for (int k = 0; k < 4; ++k) xs[tid + 256 * k] = __fmul_rn(__fmul_rn(hv[k], scale), norm_s[tid + 256 * k]);
      __syncthreads();
      // rows: warp w takes local rows w and w + 8 together
      const int r0 = rq0 + warp, r1 = rq0 + warp + 8;
      if (r1 < rq1) {
        float y0, y1;
        q4_row_dot2_smem(wq_codes + warp * 512, wq_scales + warp * 32, wq_codes + (warp + 8) * 512,
                         wq_scales + (warp + 8) * 32, xs, lane, &y0, &y1);
        if (lane == 0) {
          if (!isfinite(y0) || !isfinite(y1)) flag_error(p.err, QX_ERR_BIT_NONFINITE);
          st_tagged(p.qx + r0, y0, tag);
          st_tagged(p.qx + r1, y1, tag);
        }
      } else if (r0 < rq1) {
        const float y = q4_row_dot_smem(wq_codes + warp * 512, wq_scales + warp * 32, xs, lane);
        if (lane == 0) {
          if (!isfinite(y)) flag_error(p.err, QX_ERR_BIT_NONFINITE);
          st_tagged(p.qx + r0, y, tag);
        }
      }
      trace.mark();
    }

    // ---- B: the attention item --------------------------------------------------
    if (has_item) {
      if (!has_q && tid == kKvIssuer && i > 0) issue_kv(i, 2);
      // the split's rows, copied since the previous layer's end
      if (tid == 0) {
        if (mbar_wait_bounded(bar_kv, (uint32_t)(kv_waited & 1), p.err)) ++kv_waited;
        else stack_raise(p, poll);
      }
      if (__syncthreads_or(poll.failed)) {
        ok = false;
        break;
      }
      // each lane takes its row's key into registers while q is on its way
      const int rr = warp * 32 + lane;
      const bool valid = begin + rr < end;
      const bool warp_rows = warp * 32 < end - begin;
      float kreg[64];
      if (warp_rows) {
        const unsigned char* krow = ks + (rr >> 6) * C::TILE;
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          const float4 kv4 = *reinterpret_cast<const float4*>(krow + stack_swz(rr & 63, c * 4));
          kreg[4 * c] = kv4.x;
          kreg[4 * c + 1] = kv4.y;
          kreg[4 * c + 2] = kv4.z;
          kreg[4 * c + 3] = kv4.w;
        }
      }
      bool bad = false;
      if (tid < 64) {
        // q heads 2h, 2h + 1: the pinned RoPE pair (rotate_heads' arithmetic)
        const int g = tid >> 5, pair = tid & 31;
        float lr[2];
        stack_take_n<2>(p, p.qx + (2 * h + g) * 64 + pair, 32, 2, tag, lr, poll);
        const float left = lr[0], right = lr[1];
        float a = 0.f, c2 = 0.f;
        bad |= !poll.failed &&
               !(*rope_ok && granite_rotate(left, right, rope[2 * pair], rope[2 * pair + 1], &a, &c2));
        qs[g * 64 + pair] = a;
        qs[g * 64 + pair + 32] = c2;
      } else if (owner && tid < 96) {
        const int pair = tid - 64;
        float lr[2];
        stack_take_n<2>(p, p.qx + 1024 + h * 64 + pair, 32, 2, tag, lr, poll);
        const float left = lr[0], right = lr[1];
        float a = 0.f, c2 = 0.f;
        bad |= !poll.failed &&
               !(*rope_ok && granite_rotate(left, right, rope[2 * pair], rope[2 * pair + 1], &a, &c2));
        newk[pair] = a;
        newk[pair + 32] = c2;
      } else if (owner && tid >= 128 && tid < 192) {
        newv[tid - 128] = stack_take(p, p.qx + 1536 + h * 64 + (tid - 128), tag, poll);
      }
      if (bad) flag_error(p.err, QX_ERR_BIT_NONFINITE);
      if (__syncthreads_or(poll.failed)) {
        ok = false;
        break;
      }
      if (owner && tid < 32) {
        // append: the cache row in HBM, and the copy in this CTA's tile
        const int layer = p.layer_begin + i;
        const long long row = ((long long)p.seq * p.arena_layers + layer) * p.capacity + p.position;
        float* kd = reinterpret_cast<float*>(p.k_region) + (row * 8 + h) * 64;
        float* vd = reinterpret_cast<float*>(p.v_region) + (row * 8 + h) * 64;
        const int d = tid * 2;
        *reinterpret_cast<float2*>(kd + d) = make_float2(newk[d], newk[d + 1]);
        *reinterpret_cast<float2*>(vd + d) = make_float2(newv[d], newv[d + 1]);
        const int nr = p.position - begin, t = nr >> 6, r = nr & 63;
        *reinterpret_cast<float2*>(ks + t * C::TILE + stack_swz(r, d)) = make_float2(newk[d], newk[d + 1]);
        *reinterpret_cast<float2*>(vs + t * C::TILE + stack_swz(r, d)) = make_float2(newv[d], newv[d + 1]);
      }
      if (owner && begin + rr == p.position) {
        // the lane of the new slot: its key is the rotated new one
#pragma unroll
        for (int c = 0; c < 64; ++c) kreg[c] = newk[c];
      }
      __syncthreads();
      trace.mark();
      // warp w scores rows [32w, 32w + 32) of the item, one row per lane,
      // the key from registers and q broadcast from shared memory
      {
        float s0 = -INFINITY, s1 = -INFINITY;
        if (warp_rows) {
          float2 a0 = make_float2(0.f, 0.f), a0b = make_float2(0.f, 0.f);
          float2 a1 = make_float2(0.f, 0.f), a1b = make_float2(0.f, 0.f);
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            const float4 q0 = *reinterpret_cast<const float4*>(qs + c * 4);
            const float4 q1 = *reinterpret_cast<const float4*>(qs + 64 + c * 4);
            const float2 k01 = make_float2(kreg[4 * c], kreg[4 * c + 1]);
            const float2 k23 = make_float2(kreg[4 * c + 2], kreg[4 * c + 3]);
            a0 = __ffma2_rn(make_float2(q0.x, q0.y), k01, a0);
            a0b = __ffma2_rn(make_float2(q0.z, q0.w), k23, a0b);
            a1 = __ffma2_rn(make_float2(q1.x, q1.y), k01, a1);
            a1b = __ffma2_rn(make_float2(q1.z, q1.w), k23, a1b);
          }
          float a0v[4] = {a0.x, a0.y, a0b.x, a0b.y}, a1v[4] = {a1.x, a1.y, a1b.x, a1b.y};
          if (valid) {
            s0 = ((a0v[0] + a0v[1]) + (a0v[2] + a0v[3])) * Granite::SCALE;
            s1 = ((a1v[0] + a1v[1]) + (a1v[2] + a1v[3])) * Granite::SCALE;
          }
        }
        const float m0 = warp_max(s0), m1 = warp_max(s1);
        const float p0 = valid ? softmax_exp(s0 - m0, pinned) : 0.0f;
        const float p1 = valid ? softmax_exp(s1 - m1, pinned) : 0.0f;
        const float l0 = warp_sum(p0), l1 = warp_sum(p1);
        // P.V: lane owns dims 2 lane, 2 lane + 1 of both heads
        float o00 = 0.f, o01 = 0.f, o10 = 0.f, o11 = 0.f;
        const int nrows = max(0, min(32, end - begin - warp * 32));
        const int d = lane * 2;
#pragma unroll 8
        for (int j = 0; j < nrows; ++j) {
          const float pj0 = __shfl_sync(0xffffffffu, p0, j);
          const float pj1 = __shfl_sync(0xffffffffu, p1, j);
          const int rj = warp * 32 + j;
          const float2 v2 = *reinterpret_cast<const float2*>(vs + (rj >> 6) * C::TILE + stack_swz(rj & 63, d));
          const float2 a = __ffma2_rn(make_float2(pj0, pj0), v2, make_float2(o00, o01));
          const float2 c = __ffma2_rn(make_float2(pj1, pj1), v2, make_float2(o10, o11));
          o00 = a.x;
          o01 = a.y;
          o10 = c.x;
          o11 = c.y;
        }
        *reinterpret_cast<float2*>(wo + (warp * 2 + 0) * 64 + d) = make_float2(o00, o01);
        *reinterpret_cast<float2*>(wo + (warp * 2 + 1) * 64 + d) = make_float2(o10, o11);
        if (lane == 0) {
          wml[(warp * 2 + 0) * 2] = m0;
          wml[(warp * 2 + 0) * 2 + 1] = l0;
          wml[(warp * 2 + 1) * 2] = m1;
          wml[(warp * 2 + 1) * 2 + 1] = l1;
        }
      }
      __syncthreads();
      trace.mark();
      if (warp == 0 && lane < 16) {
        // combine weights of the 8 warps: lane = 2 w + head
        const float m = wml[lane * 2], l = wml[lane * 2 + 1];
        float M = m;
#pragma unroll
        for (int o = 2; o < 16; o <<= 1) M = fmaxf(M, __shfl_xor_sync(0x0000ffffu, M, o));
        const float wgt = m == -INFINITY ? 0.0f : softmax_exp(m - M, pinned);
        float L = wgt * l;
#pragma unroll
        for (int o = 2; o < 16; o <<= 1) L += __shfl_xor_sync(0x0000ffffu, L, o);
        wml[32 + lane] = wgt;
        if (lane < 2) {
          wml[48 + lane] = M;
          wml[50 + lane] = L;
        }
      }
      __syncthreads();
      if (tid < 128) {
        const int g = tid >> 6, d = tid & 63;
        float o = 0.0f;
#pragma unroll
        for (int w = 0; w < 8; ++w) o = fmaf(wml[32 + w * 2 + g], wo[(w * 2 + g) * 64 + d], o);
        uint2* part = p.px + (long long)b * kStackPartial + g * 66;
        st_tagged(part + d, o, tag);
        if (d == 0) {
          st_tagged(part + 64, wml[48 + g], tag);
          st_tagged(part + 65, wml[50 + g], tag);
        }
      }
      // the next layer's rows start their way from HBM into L2 now; they
      // move on into this CTA's shared memory later (issue_kv's parts 1 and
      // 2), so that the bulk of them does not queue ahead of the hand-off
      // loads
      if (tid == kKvIssuer && i + 1 < n) prefetch_kv(i + 1);
      // the last of this head's items to finish merges them: a ticket,
      // counted up for good, elects it (no fence: the partials carry their
      // tags, and it polls them like any hand-off)
      if (tid == 0) {
        const unsigned t = atomicAdd(p.tickets + h, 1u);
        const unsigned last = p.ticket_base + (unsigned)i * (unsigned)p.nsplit + (unsigned)p.nsplit - 1u;
        red[9] = __int_as_float(t == last ? 1 : 0);
      }
      __syncthreads();
      trace.mark();
      if (__float_as_int(red[9])) {
        // this head's splits -> 128 values of the attention vector: thread
        // (g, d) = (tid >> 6, tid & 63) of the first 128 loads every split's
        // O[d] at once; warp 4 takes every split's (m, l)
        const uint2* first = p.px + (long long)h * p.nsplit * kStackPartial;
        float v[kStackMaxSplits];
        const int g = (tid >> 6) & 1, d = tid & 63;
        if (tid < 128) {
          stack_take_n<kStackMaxSplits>(p, first + g * 66 + d, kStackPartial, p.nsplit, tag, v, poll);
        } else if (warp == 4) {
          // lane = (head g2, split sp) = (lane >> 4, lane & 15)
          const int g2 = lane >> 4, sp = lane & 15;
          float mm = -INFINITY, ll = 0.0f;
          if (sp < p.nsplit) {
            float ml[2];
            stack_take_n<2>(p, first + (long long)sp * kStackPartial + g2 * 66 + 64, 1, 2, tag, ml, poll);
            mm = poll.failed ? -INFINITY : ml[0];
            ll = ml[1];
          }
          const float M = half_max(mm);
          const float wgt = mm == -INFINITY ? 0.0f : softmax_exp(mm - M, pinned);
          const float L = half_sum(wgt * ll);
          mw[g2 * 16 + sp] = wgt;
          if (sp == 0) mw[32 + g2] = L;
        }
        if (__syncthreads_or(poll.failed)) {
          ok = false;
          break;
        }
        if (tid < 128) {
          float o = 0.0f;
#pragma unroll
          for (int sp = 0; sp < kStackMaxSplits; ++sp) o = fmaf(mw[g * 16 + sp], v[sp], o);
          const float a = o / mw[32 + g];
          if (!isfinite(a)) flag_error(p.err, QX_ERR_BIT_NONFINITE);
          st_tagged(p.ax + h * 128 + tid, a, tag);
        }
      }
      trace.mark();
    }

    // ---- C: o-projection rows and the residual ------------------------------------
    __syncthreads();  // every warp is done with xs (the normalized hidden)
    if (has_o) {
      {
        float av[4];
        stack_take_n<4>(p, p.ax + tid, 256, 4, tag, av, poll);
#pragma unroll
        for (int k = 0; k < 4; ++k) xs[tid + 256 * k] = av[k];
      }
      if (__syncthreads_or(poll.failed)) {
        ok = false;
        break;
      }
      trace.mark();
      if (ro0 + warp < ro1) {
        const int r = ro0 + warp;
        // the residual: this layer's input row r (kept from A's hidden-state
        // poll on a CTA with q/k/v rows)
        const float hr = lane != 0 ? 0.0f
                         : has_q  ? hs[r]
                         : (i == 0 ? __ldg(p.hidden_in + r) : stack_take(p, hin_x + r, tag - 1u, poll));
        const float y = q4_row_dot_smem(wo_codes + warp * 512, wo_scales + warp * 32, xs, lane);
        if (lane == 0 && !poll.failed) {
          const float v = __fmaf_rn(kResidualMultiplier, y, hr);
          if (!isfinite(v)) flag_error(p.err, QX_ERR_BIT_NONFINITE);
          if (i == n - 1) p.hidden_out[r] = v;
          else st_tagged(hout_x + r, v, tag);
        }
      }
      if (__syncthreads_or(poll.failed)) {
        ok = false;
        break;
      }
      trace.mark();
    }
    __syncthreads();  // every warp is done with this layer's weights
    if (tid == 0 && i + 2 < n) issue_w(i + 2);  // their buffer takes layer i + 2's
    // the first of the next layer's rows (in L2 since the attention) into shared memory
    if (tid == kKvIssuer && i + 1 < n) issue_kv(i + 1, 1);
  }

  // ---- leave: copies in flight first (bounded) ---------------------------------------
  if (tid == kKvIssuer) kv_count[0] = kv_issued;
  __syncthreads();
  if (tid == 0) {
    kv_issued = kv_count[0];
    while (kv_waited < kv_issued) {
      if (!mbar_wait_bounded(bar_kv, (uint32_t)(kv_waited & 1), p.err)) break;
      ++kv_waited;
    }
#pragma unroll
    for (int j = 0; j < 2; ++j)
      while (w_waited[j] < w_issued[j]) {
        if (!mbar_wait_bounded(&bar_w[j], (uint32_t)(w_waited[j] & 1), p.err)) break;
        ++w_waited[j];
      }
    if (!ok) *reinterpret_cast<volatile unsigned*>(p.abort) = 1u;
  }
}

}  // namespace qx
