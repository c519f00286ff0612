// qxcuda.cu — host side of libqxcuda: contexts, KV arenas, argument
// validation with the reference's error behaviour, and kernel dispatch.
//
// Error behaviour mirrors crates/qx-runtime/src/lib.rs:382-405
// (KvCache::append: "KV position {p} does not follow cache length {len}",
// "KV position {p} exceeds context {max}") and
// crates/qx-runtime-v2/src/lib.rs:6587-6589 ("context {c} must be in
// 1..=4096"). Nothing is launched when validation fails, so a rejected call
// leaves the cache untouched, as the reference's Err return does.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <new>
#include <string>
#include <vector>

#include "../../include/qxcuda.h"
#include "decode.cuh"
#include "decode_tc.cuh"
#include "append.cuh"
#include "layer.cuh"
#include "prefill.cuh"
#include "commit.cuh"
#include "pages.cuh"
#include "exchange.cuh"
#include "stack.cuh"

using namespace qx;

struct qxc_ctx {
  int device = 0;
  int sm_count = 148;
  cudaStream_t own_stream = nullptr;
  cudaStream_t stream = nullptr;
  std::string err;
  unsigned* err_host = nullptr;  // mapped pinned error word
  unsigned* err_dev = nullptr;
  // scratch (grown on demand)
  float* partials = nullptr;
  size_t partials_cap = 0;  // floats
  int* tickets = nullptr;
  size_t tickets_cap = 0;  // ints
  // tagged partials of the slice merge (zeroed when allocated: tag 0 is no
  // call's) and the last call's tag
  uint2* tpartials = nullptr;
  size_t tpartials_cap = 0;  // uint2
  unsigned merge_gen = 0;
  // per-call sequence tables: device ring + pinned host ring
  static constexpr int kRing = 8;
  SeqInfo* seq_dev[kRing] = {};
  SeqInfo* seq_host[kRing] = {};
  cudaEvent_t seq_ev[kRing] = {};
  size_t seq_cap[kRing] = {};
  int seq_next = 0;
  // device staging for host-pointer entry points
  char* stage_dev = nullptr;
  size_t stage_cap = 0;
  unsigned long long launches = 0;
  int last_split = 0;
  // Which cache rows a grid launched now may find still being written.
  // A grid that triggers its dependents only after its own
  // griddepcontrol.wait (or at its end) has all grids before it complete by
  // the time any later grid starts. Since the last such grid on the stream:
  // kvw_open = some grid that writes rows triggered early (any row may still
  // be written); else kvw_arena = the arena written (null: none), kvw_seq
  // its sequence (-1: several) and kvw_row the lowest row written.
  bool kvw_open = false;
  const void* kvw_arena = nullptr;
  int kvw_seq = -1;
  int kvw_row = 0;
  // Qwen RoPE (cos, sin) for every position 0..kQwenMaxPositions-1, shared
  // by all Qwen arenas of this context (created with the first one).
  float2* qwen_rope = nullptr;
  float2* granite_rope = nullptr;  // pinned (sin, cos) [4096][32], built on first prefill
  float* layer_scratch = nullptr;   // attention layer: q[1024] k[512] v[512] attention[1024]
  // attention stack (stack.cuh): tagged exchange buffers hx [2][1024],
  // qx [2048], ax [1024]; split partials [128][132] floats and chain
  // [2][1024] floats (between launches of > 32 layers); the words: [0] abort,
  // [1..8] merge tickets; the launch generation
  uint2* stack_x = nullptr;
  float* stack_f = nullptr;
  unsigned* stack_words = nullptr;
  unsigned stack_gen = 0;
  unsigned stack_tickets = 0;  // every head's merge-ticket count after the launches so far
  // prefill's rotated-query scratch (bf16 elements)
  unsigned short* prefill_q = nullptr;
  size_t prefill_q_cap = 0;
};

constexpr int kQwenMaxPositions = 40960;  // max_position_embeddings, qx-model lib.rs:308

static constexpr int kExchHeads = 32, kExchRow = 130;

// One rank's exchange area and the views of every rank's (see exchange.cuh),
// sized for the largest model (Qwen3: 32 query heads, head_dim 128):
//   inbox  [2][world][32][130] {value, tag}     qx_exchange_merge_kernel
//   xinbox [2][world][32 * 4][34] {value, tag}  qx_split_merge_kernel's exchange
//   steps  [32] u32, then [32][4] u32           one counter per writer
struct qxc_peer_group {
  qxc_ctx* ctx = nullptr;
  int rank = 0, world = 1;
  char* base = nullptr;
  size_t bytes = 0, off_xinbox = 0, off_step = 0;
  char* peer[kMaxPeers] = {};    // every rank's base as seen from this device
  bool opened[kMaxPeers] = {};   // opened through CUDA IPC (closed on destroy)
  // Set (by the device) once an exchange on this group has timed out; from
  // then on every exchange call on it fails (see mark_peer_group_failed).
  unsigned* failed_host = nullptr;  // mapped pinned word
  unsigned* failed_mapped = nullptr;  // its device address
  unsigned* failed_dev() const { return reinterpret_cast<unsigned*>(base + off_step + 768); }
  bool failed() const { return *reinterpret_cast<volatile unsigned*>(failed_host) != 0u; }
};

struct qxc_kv {
  qxc_ctx* ctx = nullptr;
  qxc_kv_desc desc{};
  int hq = 0, hkv = 0, d = 0;
  size_t kes = 0, ves = 0;
  char* base = nullptr;
  char* k_region = nullptr;
  char* v_region = nullptr;
  size_t k_unit = 0, v_unit = 0;  // bytes per (sequence, layer)
  std::vector<int> len;
  float2* rope_table = nullptr;  // Qwen (cos, sin) per absolute position (owned by ctx)
  CUtensorMap tmk, tmv;          // tensor maps over the key / value regions
  // paged arenas (page_shift > 0): per layer a pool of pool_pages pages of
  // 2^page_shift rows; a sequence's logical pages [0, mapped[seq]) map to
  // physical pages through table (host mirror of table_dev, -1 unmapped)
  int page_shift = 0;
  int pool_pages = 0;
  int table_stride = 0;  // logical pages per sequence
  int* table_dev = nullptr;
  std::vector<int> table;
  std::vector<int> mapped;
  std::vector<int> free_pages;  // a stack: the next page to hand out is at the back
  bool paged() const { return page_shift != 0; }
  int pages_for(long long rows) const { return (int)((rows + (1ll << page_shift) - 1) >> page_shift); }
};

// The row map the kernels use for this arena (null table: contiguous).
static KvPaging kv_paging(const qxc_kv* kv) {
  KvPaging g;
  memset(&g, 0, sizeof(g));
  if (kv->paged()) {
    g.table = kv->table_dev;
    g.stride = kv->table_stride;
    g.shift = kv->page_shift;
    g.pool = kv->pool_pages;
  }
  return g;
}

namespace {

qxc_status fail(qxc_ctx* ctx, qxc_status st, const char* fmt, ...) {
  if (ctx) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    ctx->err = buf;
  }
  return st;
}

#define QXC_CUDA(ctx, call)                                                                          \
  do {                                                                                               \
    cudaError_t e_ = (call);                                                                         \
    if (e_ != cudaSuccess)                                                                           \
      return fail((ctx), e_ == cudaErrorMemoryAllocation ? QXC_ERR_OUT_OF_MEMORY : QXC_ERR_CUDA,     \
                  "%s: %s", #call, cudaGetErrorString(e_));                                          \
  } while (0)

size_t dtype_size(int dt) { return dt == QXC_F32 ? 4 : 2; }
bool valid_dtype(int dt) { return dt == QXC_F32 || dt == QXC_BF16 || dt == QXC_F16; }

void model_shape(int model, int* hq, int* hkv, int* d) {
  if (model == QXC_MODEL_QWEN3) {
    *hq = 32, *hkv = 4, *d = 128;
  } else {
    *hq = 16, *hkv = 8, *d = 64;
  }
}

qxc_status check_desc(qxc_ctx* ctx, const qxc_kv_desc* d) {
  if (!d) return fail(ctx, QXC_ERR_INVALID_ARG, "null KV descriptor");
  if (d->model != QXC_MODEL_GRANITE && d->model != QXC_MODEL_QWEN3)
    return fail(ctx, QXC_ERR_INVALID_ARG, "unknown model %d", d->model);
  if (d->layers < 1 || d->sequences < 1)
    return fail(ctx, QXC_ERR_INVALID_ARG, "layers and sequences must be >= 1");
  if (!valid_dtype(d->key_dtype) || !valid_dtype(d->value_dtype))
    return fail(ctx, QXC_ERR_INVALID_ARG, "unknown KV dtype");
  if (d->first_position < 0) return fail(ctx, QXC_ERR_INVALID_ARG, "first_position must be >= 0");
  if (d->model == QXC_MODEL_GRANITE) {
    // ExecutionPlan::granite_with_kv_element_bytes (qx-runtime-v2 lib.rs:6587-6589)
    if (d->capacity == 0 || d->capacity < 0 || d->first_position + d->capacity > 4096)
      return fail(ctx, QXC_ERR_INVALID_ARG, "context %d must be in 1..=4096", d->first_position + d->capacity);
  } else {
    // Qwen3-30B-A3B max_position_embeddings 40960 (qx-model lib.rs:308); the
    // decode kernel supports 16-bit KV only.
    if (d->capacity < 1 || d->first_position + d->capacity > 40960)
      return fail(ctx, QXC_ERR_INVALID_ARG, "context %d must be in 1..=40960", d->first_position + d->capacity);
    if (d->key_dtype == QXC_F32 || d->value_dtype != d->key_dtype)
      return fail(ctx, QXC_ERR_UNSUPPORTED, "Qwen KV must be bf16 or f16 for both keys and values");
  }
  if (d->model == QXC_MODEL_GRANITE && d->key_dtype != d->value_dtype) {
    const bool ok = (d->key_dtype == QXC_F32 && d->value_dtype == QXC_F16) ||
                    (d->key_dtype == QXC_F16 && d->value_dtype == QXC_F32);
    if (!ok) return fail(ctx, QXC_ERR_UNSUPPORTED, "mixed KV precision must be f32/f16");
  }
  if (d->model == QXC_MODEL_GRANITE && d->key_dtype == QXC_F32 && d->value_dtype == QXC_BF16)
    return fail(ctx, QXC_ERR_UNSUPPORTED, "unsupported KV precision");
  return QXC_OK;
}

template <typename T>
qxc_status grow(qxc_ctx* ctx, T** ptr, size_t* cap, size_t need, bool zero) {
  if (need <= *cap) return QXC_OK;
  size_t n = std::max(need, *cap * 2);
  if (*ptr) {
    QXC_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
    cudaFree(*ptr);
    *ptr = nullptr;
    *cap = 0;
  }
  QXC_CUDA(ctx, cudaMalloc(reinterpret_cast<void**>(ptr), n * sizeof(T)));
  if (zero) QXC_CUDA(ctx, cudaMemsetAsync(*ptr, 0, n * sizeof(T), ctx->stream));
  *cap = n;
  return QXC_OK;
}

// Resident CTAs per SM of one decode instantiation (occupancy API).
template <class M, typename KT, typename VT>
int blocks_per_sm() {
  using C = DecodeCfg<M, KT, VT>;
  cudaFuncSetAttribute(qx_decode_kernel<M, KT, VT>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  int n = 1;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, qx_decode_kernel<M, KT, VT>, C::NT, C::SMEM) != cudaSuccess)
    n = 1;
  return n > 0 ? n : 1;
}

template <typename KT, class TM>
int tc_blocks_per_sm() {
  using C = TcCfg<KT, TM>;
  cudaFuncSetAttribute(qx_decode_tc_kernel<KT, TM>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  int n = 1;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, qx_decode_tc_kernel<KT, TM>, C::NT, C::SMEM) != cudaSuccess)
    n = 1;
  return n > 0 ? n : 1;
}

// A Granite arena whose keys and values share one 16-bit type decodes on the
// tensor cores, a pair of kv heads per work unit (TcGranitePair).
bool granite_pair_tc(const qxc_kv* kv) {
  const int kd = kv->desc.key_dtype, vd = kv->desc.value_dtype;
  return kv->desc.model == QXC_MODEL_GRANITE && kd == vd && (kd == QXC_BF16 || kd == QXC_F16);
}

// The decode kernel's grid runs on tcgen05 (Qwen, 16-bit Granite).
bool decode_on_tc(const qxc_kv* kv) { return kv->desc.model == QXC_MODEL_QWEN3 || granite_pair_tc(kv); }

// Work units per layer of the decode kernels: kv heads, or kv-head pairs.
int decode_units(const qxc_kv* kv) { return granite_pair_tc(kv) ? kv->hkv / 2 : kv->hkv; }

int decode_blocks_per_sm(const qxc_kv* kv) {
  const int kd = kv->desc.key_dtype, vd = kv->desc.value_dtype;
  if (kv->desc.model == QXC_MODEL_QWEN3)
    return kd == QXC_BF16 ? tc_blocks_per_sm<__nv_bfloat16, TcQwen>() : tc_blocks_per_sm<__half, TcQwen>();
  if (granite_pair_tc(kv))
    return kd == QXC_BF16 ? tc_blocks_per_sm<__nv_bfloat16, TcGranitePair>()
                          : tc_blocks_per_sm<__half, TcGranitePair>();
  if (kd == QXC_F32 && vd == QXC_F32) return blocks_per_sm<Granite, float, float>();
  if (kd == QXC_F32 && vd == QXC_F16) return blocks_per_sm<Granite, float, __half>();
  if (kd == QXC_F16 && vd == QXC_F32) return blocks_per_sm<Granite, __half, float>();
  if (kd == QXC_F16 && vd == QXC_F16) return blocks_per_sm<Granite, __half, __half>();
  return blocks_per_sm<Granite, __nv_bfloat16, __nv_bfloat16>();
}

// Cache rows per pipeline tile: 128 for the tensor-core kernels, else 64.
int decode_tile(const qxc_kv* kv) { return decode_on_tc(kv) ? 128 : 64; }

// A split must be a multiple of this many rows: 64 for Granite (the
// tensor-core kernel masks the rest of a 128-row tile), 128 for Qwen.
int split_unit(const qxc_kv* kv) { return kv->desc.model == QXC_MODEL_QWEN3 ? 128 : 64; }

int decode_max_splits(const qxc_kv* kv) {
  const int kd = kv->desc.key_dtype, vd = kv->desc.value_dtype;
  if (decode_on_tc(kv)) return TcCfg<__nv_bfloat16>::MAX_SPLITS;
  if (kd == QXC_F32 && vd == QXC_F32) return DecodeCfg<Granite, float, float>::MAX_SPLITS;
  if (kd == QXC_F32 && vd == QXC_F16) return DecodeCfg<Granite, float, __half>::MAX_SPLITS;
  if (kd == QXC_F16 && vd == QXC_F32) return DecodeCfg<Granite, __half, float>::MAX_SPLITS;
  if (kd == QXC_F16 && vd == QXC_F16) return DecodeCfg<Granite, __half, __half>::MAX_SPLITS;
  return DecodeCfg<Granite, __nv_bfloat16, __nv_bfloat16>::MAX_SPLITS;
}

// Positions per split (a multiple of 64). Split-KV exists to fill 148 SMs
// at small batch; too many splits add per-CTA overhead, and a grid that
// leaves the last wave nearly empty wastes the tail. Model the time as
// waves x (64-row tiles per CTA + a fixed per-CTA cost) and take the
// cheapest split, preferring fewer splits on ties.
int auto_chunk(int slots, const int* attend, int n, int units_per_seq, int max_splits, int tile) {
  int max_attend = 1;
  for (int i = 0; i < n; ++i) max_attend = std::max(max_attend, attend[i]);
  const int top = ((max_attend + tile - 1) / tile) * tile;
  // A batch whose unsplit work already fills every CTA slot a few times
  // over gains nothing from splitting; each extra CTA only adds its fixed
  // cost (the tensor-core kernel on config 4: 48.1k tok/s at splits of 1024
  // rows, 62.1k unsplit; its first 8 sequences: 45.1k and 54.4k). Unsplit
  // when the work per slot is at least twice the longest item.
  {
    double work = 0.0;
    for (int i = 0; i < n; ++i) work += (double)units_per_seq * ((double)(attend[i] + tile - 1) / tile + 3.0);
    const double longest = (double)top / tile + 3.0;
    if (work / slots >= 2.0 * longest && (max_attend + top - 1) / top <= max_splits) return top;
  }
  double best = 1e300;
  int best_c = top;
  for (int c = top; c >= tile; c -= tile) {
    if ((max_attend + c - 1) / c > max_splits) break;
    long long items = 0;
    for (int i = 0; i < n; ++i) items += (long long)units_per_seq * ((attend[i] + c - 1) / c);
    const long long waves = (items + slots - 1) / slots;
    // + the merge, which grows with the split count (weighted so that the
    // measured optima stay chosen: config 1 at 2048 rows, config 3 at 896,
    // the Q4 layer's single-layer decode at 256 rather than 128)
    const double cost = (double)waves * ((double)c / tile + 3.0) * tile / 64.0 + 0.2 * ((max_attend + c - 1) / c);
    if (cost < best - 1e-9) {
      best = cost;
      best_c = c;
    }
  }
  return best_c;
}

using KernelFn = void (*)(DecodeParams);

// Launch a DecodeParams kernel as a programmatic dependent of the stream's
// previous kernel: its CTAs may become resident and set up (barriers, TMEM)
// while that kernel drains, and wait for it in griddepcontrol.wait.
cudaError_t launch_pdl(qxc_ctx* ctx, KernelFn fn, int grid, int threads, int smem, const DecodeParams& p) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = ctx->stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, fn, p);
}

// Diagnostics: with QXC_TRACE set in the environment, a launch gets a zeroed
// stage-timeline buffer (kTraceSlots per CTA) and, once it completes, one
// line per CTA goes to stderr: "<kernel> trace cta N: t0 t1 ..." in absolute
// %globaltimer nanoseconds. Tracing synchronises the stream after every
// launch and allocates, so it cannot run under stream capture.
struct TraceRun {
  qxc_ctx* ctx;
  const char* name;
  size_t ctas;
  unsigned long long* buf = nullptr;
  TraceRun(qxc_ctx* c, const char* n, size_t k) : ctx(c), name(n), ctas(k) {
    static const bool on = getenv("QXC_TRACE") != nullptr;
    if (!on) return;
    if (cudaMalloc(&buf, ctas * kTraceSlots * sizeof(unsigned long long)) != cudaSuccess) {
      buf = nullptr;
      return;
    }
    cudaMemsetAsync(buf, 0, ctas * kTraceSlots * sizeof(unsigned long long), ctx->stream);
  }
  ~TraceRun() {
    if (!buf) return;
    std::vector<unsigned long long> h(ctas * kTraceSlots);
    cudaMemcpyAsync(h.data(), buf, h.size() * sizeof(unsigned long long), cudaMemcpyDeviceToHost, ctx->stream);
    cudaStreamSynchronize(ctx->stream);
    cudaFree(buf);
    for (size_t cta = 0; cta < ctas; ++cta) {
      fprintf(stderr, "%s trace cta %zu:", name, cta);
      for (int i = 0; i < kTraceSlots && h[cta * kTraceSlots + i]; ++i) fprintf(stderr, " %llu", h[cta * kTraceSlots + i]);
      fprintf(stderr, "\n");
    }
  }
};

template <class M, typename KT, typename VT>
qxc_status launch_typed(qxc_ctx* ctx, const DecodeParams& p, int items) {
  using C = DecodeCfg<M, KT, VT>;
  static unsigned long long configured = 0;  // one bit per device ordinal
  const unsigned long long bit = 1ull << (ctx->device & 63);
  if (!(configured & bit)) {
    QXC_CUDA(ctx, cudaFuncSetAttribute(qx_decode_kernel<M, KT, VT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       C::SMEM));
    configured |= bit;
  }
  QXC_CUDA(ctx, launch_pdl(ctx, qx_decode_kernel<M, KT, VT>, items, C::NT, C::SMEM, p));
  ctx->launches++;
  return QXC_OK;
}

template <typename KT, class TM>
qxc_status launch_tc(qxc_ctx* ctx, const DecodeParams& p, int items) {
  using C = TcCfg<KT, TM>;
  static unsigned long long configured = 0;
  const unsigned long long bit = 1ull << (ctx->device & 63);
  if (!(configured & bit)) {
    QXC_CUDA(ctx, cudaFuncSetAttribute(qx_decode_tc_kernel<KT, TM>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       C::SMEM));
    configured |= bit;
  }
  QXC_CUDA(ctx, launch_pdl(ctx, qx_decode_tc_kernel<KT, TM>, items, C::NT, C::SMEM, p));
  ctx->launches++;
  return QXC_OK;
}

qxc_status launch_decode_kernel(qxc_ctx* ctx, const qxc_kv* kv, const DecodeParams& p, int items);

// Splits beyond which the merge runs as its own kernel.
constexpr int kInKernelMergeMaxSplits = 8;

// The merge grid is a programmatic dependent of the decode grid: it may be
// launched while the decode runs and waits for it in griddepcontrol.wait.
qxc_status launch_split_merge(qxc_ctx* ctx, const qxc_kv* kv, const DecodeParams& p) {
  const int grid = p.n_seq * p.layer_count * kv->hq * (kv->d / 32);
  if (kv->desc.model == QXC_MODEL_QWEN3)
    QXC_CUDA(ctx, launch_pdl(ctx, qx_split_merge_kernel<8, 128, 4, 32>, grid, 128, 0, p));
  else if (granite_pair_tc(kv))
    QXC_CUDA(ctx, launch_pdl(ctx, qx_split_merge_kernel<4, 64, 4, 16>, grid, 128, 0, p));
  else
    QXC_CUDA(ctx, launch_pdl(ctx, qx_split_merge_kernel<2, 64, 8, 16>, grid, 128, 0, p));
  ctx->launches++;
  return QXC_OK;
}

qxc_status launch_decode(qxc_ctx* ctx, const qxc_kv* kv, const DecodeParams& p0, int items) {
  DecodeParams p = p0;
  qxc_status st;
  {
    TraceRun tr(ctx, "decode", items);
    p.trace = tr.buf;
    st = launch_decode_kernel(ctx, kv, p, items);
  }
  if (st != QXC_OK || !p.external_merge) return st;
  TraceRun tr(ctx, "merge", (size_t)p.n_seq * p.layer_count * kv->hq * (kv->d / 32));
  p.trace = tr.buf;
  return launch_split_merge(ctx, kv, p);
}

qxc_status launch_decode_kernel(qxc_ctx* ctx, const qxc_kv* kv, const DecodeParams& p, int items) {
  const int kd = kv->desc.key_dtype, vd = kv->desc.value_dtype;
  if (kv->desc.model == QXC_MODEL_QWEN3) {
    // group-8 attention runs on the tensor cores (decode_tc.cuh)
    if (kd == QXC_BF16) return launch_tc<__nv_bfloat16, TcQwen>(ctx, p, items);
    return launch_tc<__half, TcQwen>(ctx, p, items);
  }
  if (granite_pair_tc(kv)) {
    if (kd == QXC_BF16) return launch_tc<__nv_bfloat16, TcGranitePair>(ctx, p, items);
    return launch_tc<__half, TcGranitePair>(ctx, p, items);
  }
  if (kd == QXC_F32 && vd == QXC_F32) return launch_typed<Granite, float, float>(ctx, p, items);
  if (kd == QXC_F32 && vd == QXC_F16) return launch_typed<Granite, float, __half>(ctx, p, items);
  if (kd == QXC_F16 && vd == QXC_F32) return launch_typed<Granite, __half, float>(ctx, p, items);
  if (kd == QXC_F16 && vd == QXC_F16) return launch_typed<Granite, __half, __half>(ctx, p, items);
  return launch_typed<Granite, __nv_bfloat16, __nv_bfloat16>(ctx, p, items);
}

// Upload a sequence table through the pinned ring (host slot reuse waits on
// the event of the copy that last read it).
qxc_status upload_seq_table(qxc_ctx* ctx, const std::vector<SeqInfo>& tab, const SeqInfo** dev) {
  const int i = ctx->seq_next;
  ctx->seq_next = (i + 1) % qxc_ctx::kRing;
  const size_t need = tab.size();
  if (ctx->seq_ev[i]) QXC_CUDA(ctx, cudaEventSynchronize(ctx->seq_ev[i]));
  if (need > ctx->seq_cap[i]) {
    if (ctx->seq_dev[i]) {
      QXC_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
      cudaFree(ctx->seq_dev[i]);
      cudaFreeHost(ctx->seq_host[i]);
    }
    size_t n = std::max<size_t>(need, 256);
    QXC_CUDA(ctx, cudaMalloc(&ctx->seq_dev[i], n * sizeof(SeqInfo)));
    QXC_CUDA(ctx, cudaMallocHost(&ctx->seq_host[i], n * sizeof(SeqInfo)));
    ctx->seq_cap[i] = n;
  }
  if (!ctx->seq_ev[i]) QXC_CUDA(ctx, cudaEventCreateWithFlags(&ctx->seq_ev[i], cudaEventDisableTiming));
  memcpy(ctx->seq_host[i], tab.data(), need * sizeof(SeqInfo));
  QXC_CUDA(ctx, cudaMemcpyAsync(ctx->seq_dev[i], ctx->seq_host[i], need * sizeof(SeqInfo), cudaMemcpyHostToDevice,
                                ctx->stream));
  QXC_CUDA(ctx, cudaEventRecord(ctx->seq_ev[i], ctx->stream));
  *dev = ctx->seq_dev[i];
  return QXC_OK;
}

struct CallPlan {
  std::vector<SeqInfo> tab;
  int items = 0;
  int chunk = 0;
  int units = 0;  // work units per layer (kv heads, or kv-head pairs)
};

// Build the work decomposition of one call. `attend[i]`, `new_slot[i]`,
// `rope_pos[i]` per sequence entry.
// `units`: work units per layer of the kernel that will run (0: the decode
// kernels' decode_units).
qxc_status plan_call(qxc_ctx* ctx, const qxc_kv* kv, int seq_count, const int* seq_ids, const int* attend,
                     const int* new_slot, const int* rope_pos, int layer_count, int split, CallPlan* out,
                     int units = 0) {
  if (units == 0) units = decode_units(kv);
  out->units = units;
  int chunk = split;
  if (chunk == 0) {
    static int cached_slots[64][8] = {};  // [device][arena type] resident CTAs on the GPU
    const int kd = kv->desc.key_dtype, vd = kv->desc.value_dtype;
    const int type = kv->desc.model == QXC_MODEL_QWEN3 ? (kd == QXC_BF16 ? 5 : 6)
                     : kd == QXC_BF16                  ? 4
                                                       : (kd == QXC_F16 ? 2 : 0) + (vd == QXC_F16 ? 1 : 0);
    int& slots = cached_slots[ctx->device & 63][type];
    if (!slots) slots = ctx->sm_count * decode_blocks_per_sm(kv);
    chunk = auto_chunk(slots, attend, seq_count, layer_count * units, decode_max_splits(kv), decode_tile(kv));
  }
  {
    int max_attend = 1;
    for (int i = 0; i < seq_count; ++i) max_attend = std::max(max_attend, attend[i]);
    if ((max_attend + chunk - 1) / chunk > decode_max_splits(kv))
      return fail(ctx, QXC_ERR_INVALID_ARG, "split %d gives %d splits; at most %d fit the merge", chunk,
                  (max_attend + chunk - 1) / chunk, decode_max_splits(kv));
  }
  if (chunk <= 0 || chunk % split_unit(kv) != 0)
    return fail(ctx, QXC_ERR_INVALID_ARG, "split %d must be a positive multiple of %d", split, split_unit(kv));
  out->chunk = chunk;
  ctx->last_split = chunk;
  out->tab.resize(seq_count);
  long long items = 0;
  for (int i = 0; i < seq_count; ++i) {
    SeqInfo& s = out->tab[i];
    s.seq_id = seq_ids ? seq_ids[i] : i;
    s.attend = attend[i];
    s.new_slot = new_slot[i];
    s.rope_pos = rope_pos[i];
    s.item_begin = (int)items;
    s.pad[0] = s.pad[1] = s.pad[2] = 0;
    const long long nsplit = (attend[i] + chunk - 1) / chunk;
    items += nsplit * layer_count * units;
  }
  if (items > 0x7fffffffLL) return fail(ctx, QXC_ERR_INVALID_ARG, "too much work in one call");
  out->items = (int)items;
  return QXC_OK;
}

// Rows [0, result) of `seq` no running grid can be writing.
int rows_settled(const qxc_ctx* ctx, const qxc_kv* kv, int seq) {
  if (ctx->kvw_open) return 0;
  if (ctx->kvw_arena != kv || (ctx->kvw_seq >= 0 && ctx->kvw_seq != seq)) return kv->desc.capacity;
  return ctx->kvw_row;
}

// Record a grid that triggers its dependents only after its wait (or at its
// end) and wrote rows >= row_lo of `seq` (-1: several) of kv (kv null: none).
void note_rows_written(qxc_ctx* ctx, const qxc_kv* kv, int seq, int row_lo) {
  ctx->kvw_open = false;
  ctx->kvw_arena = kv;
  ctx->kvw_seq = seq;
  ctx->kvw_row = row_lo;
}

// Record a grid that may write rows and triggers its dependents before its
// wait: until the next grid that waits first, any row may be in flight.
void note_rows_open(qxc_ctx* ctx) { ctx->kvw_open = true; }

qxc_status fill_params(qxc_ctx* ctx, qxc_kv* kv, const CallPlan& plan, int layer_begin, int layer_count,
                       DecodeParams* p) {
  memset(p, 0, sizeof(*p));
  p->tmk = kv->tmk;
  p->tmv = kv->tmv;
  p->capacity = kv->desc.capacity;
  p->paging = kv_paging(kv);
  p->k_region = kv->k_region;
  p->v_region = kv->v_region;
  p->layers = kv->desc.layers;
  p->layer_begin = layer_begin;
  p->layer_count = layer_count;
  p->n_seq = (int)plan.tab.size();
  p->chunk = plan.chunk;
  p->rope_table = kv->rope_table;
  p->err = ctx->err_dev;
  if (plan.tab.size() == 1) {
    p->seq_table = nullptr;
    p->single = plan.tab[0];
  } else {
    qxc_status st = upload_seq_table(ctx, plan.tab, &p->seq_table);
    if (st != QXC_OK) return st;
  }
  const int G = kv->hq / plan.units;
  qxc_status st = grow(ctx, &ctx->partials, &ctx->partials_cap, (size_t)plan.items * G * (kv->d + 2), false);
  if (st != QXC_OK) return st;
  st = grow(ctx, &ctx->tickets, &ctx->tickets_cap, (size_t)plan.tab.size() * layer_count * plan.units, true);
  if (st != QXC_OK) return st;
  p->partials = ctx->partials;
  p->tickets = ctx->tickets;
  int max_split = 1;
  for (const SeqInfo& si : plan.tab) max_split = std::max(max_split, (si.attend + plan.chunk - 1) / plan.chunk);
  const bool one_wave = plan.items <= decode_blocks_per_sm(kv) * ctx->sm_count;
  p->external_merge = max_split > kInKernelMergeMaxSplits ? 1 : 0;
  // a one-wave grid lets the next grid (the merge, or the next call) get
  // resident while it runs
  p->early_trigger = one_wave ? 1 : 0;
  // a single contiguous sequence may stream its settled rows before the wait
  if (plan.tab.size() == 1 && !kv->paged()) p->pre_rows = rows_settled(ctx, kv, plan.tab[0].seq_id);
  if (!decode_on_tc(kv)) {
    // the CUDA-core kernels trigger at their start (measured faster for
    // them) and stream nothing before their wait
    note_rows_open(ctx);
  } else {
    // the tensor-core decode triggers after its wait: it is now the only
    // grid that may still write rows (its new slots), or none
    int lo = kv->desc.capacity;
    for (const SeqInfo& si : plan.tab)
      if (si.new_slot >= 0) lo = std::min(lo, si.new_slot);
    if (lo < kv->desc.capacity) note_rows_written(ctx, kv, plan.tab.size() == 1 ? plan.tab[0].seq_id : -1, lo);
    else note_rows_written(ctx, nullptr, -1, 0);
  }
  return QXC_OK;
}

// A Qwen decode whose grid is one wave, with 2 to 64 splits of some (unit,
// kv head), merges its splits inside the decode grid (slice_merge in
// decode.cuh) instead of a second grid: the splits wait for one another,
// which a one-wave grid allows, and the merge kernel's launch and its wait
// for the decode grid's end drop out of the call. On a KV length split
// across GPUs (qxc_decode_exchange) the merged slices then go through the
// same exchange as in the merge kernel.
qxc_status use_slice_merge(qxc_ctx* ctx, const qxc_kv* kv, const CallPlan& plan, DecodeParams* p) {
  if (kv->desc.model != QXC_MODEL_QWEN3) return QXC_OK;
  int max_split = 1;
  for (const SeqInfo& si : plan.tab) max_split = std::max(max_split, (si.attend + plan.chunk - 1) / plan.chunk);
  if (max_split < 2 || max_split > 4 * kMergeLoads) return QXC_OK;
  if (plan.items > decode_blocks_per_sm(kv) * ctx->sm_count) return QXC_OK;
  const size_t need = (size_t)plan.items * kv->hq / plan.units * (kv->d + 2);
  if (need > ctx->tpartials_cap) {
    if (ctx->tpartials) {
      QXC_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
      cudaFree(ctx->tpartials);
      ctx->tpartials = nullptr;
      ctx->tpartials_cap = 0;
    }
    QXC_CUDA(ctx, cudaMalloc(&ctx->tpartials, need * sizeof(uint2)));
    QXC_CUDA(ctx, cudaMemsetAsync(ctx->tpartials, 0, need * sizeof(uint2), ctx->stream));
    ctx->tpartials_cap = need;
  }
  ctx->merge_gen += 1u;
  if (ctx->merge_gen == 0u) ctx->merge_gen = 1u;
  p->slice_merge = 1;
  p->external_merge = 0;
  p->merge_tag = ctx->merge_gen;
  p->tpartials = ctx->tpartials;
  return QXC_OK;
}

bool default_pinned(const qxc_kv* kv, int flags) {
  if (flags & QXC_DECODE_NATIVE_EXP) return false;
  if (flags & QXC_DECODE_PINNED_EXP) return true;
  return kv->desc.model == QXC_MODEL_GRANITE;
}

qxc_status check_seq(qxc_ctx* ctx, const qxc_kv* kv, int seq) {
  if (seq < 0 || seq >= kv->desc.sequences)
    return fail(ctx, QXC_ERR_INVALID_ARG, "sequence %d is outside the arena (%d sequences)", seq, kv->desc.sequences);
  return QXC_OK;
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// 3-D map over one region: {head_dim, kv_heads, rows}, box {128 B of
// head_dim, 1 head, 64 rows}, 128-byte swizzle. Rows past the region read
// as zero.
qxc_status encode_kv_map(qxc_ctx* ctx, CUtensorMap* map, void* base, int dtype, int hkv, int d, size_t rows) {
  auto fn = encode_fn();
  if (!fn) return fail(ctx, QXC_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  const size_t es = dtype_size(dtype);
  const CUtensorMapDataType t = dtype == QXC_F32    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                : dtype == QXC_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                    : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  cuuint64_t dims[3] = {(cuuint64_t)d, (cuuint64_t)hkv, (cuuint64_t)rows};
  cuuint64_t strides[2] = {(cuuint64_t)(d * es), (cuuint64_t)(hkv * d * es)};
  cuuint32_t box[3] = {(cuuint32_t)(128 / es), 1, 64};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, t, 3, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(ctx, QXC_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return QXC_OK;
}

// 3-D map {inner, heads, rows} with box {box_inner, 1, box_rows}, 128-byte swizzle.
qxc_status encode_tile_map(qxc_ctx* ctx, CUtensorMap* map, void* base, int dtype, int heads, int inner, size_t rows,
                           int box_rows) {
  auto fn = encode_fn();
  if (!fn) return fail(ctx, QXC_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  const size_t es = dtype_size(dtype);
  const CUtensorMapDataType t = dtype == QXC_F32    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                : dtype == QXC_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                    : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  cuuint64_t dims[3] = {(cuuint64_t)inner, (cuuint64_t)heads, (cuuint64_t)rows};
  cuuint64_t strides[2] = {(cuuint64_t)(inner * es), (cuuint64_t)(heads * inner * es)};
  cuuint32_t box[3] = {(cuuint32_t)(128 / es), 1, (cuuint32_t)box_rows};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, t, 3, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(ctx, QXC_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return QXC_OK;
}

qxc_status ensure_granite_rope(qxc_ctx* ctx) {
  if (ctx->granite_rope) return QXC_OK;
  float2* tab = nullptr;
  QXC_CUDA(ctx, cudaMalloc(&tab, (size_t)kGraniteRopePositions * 32 * sizeof(float2)));
  qx_granite_rope_table_kernel<<<kGraniteRopePositions * 32 / 256, 256, 0, ctx->stream>>>(tab, ctx->err_dev);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    cudaFree(tab);
    return fail(ctx, QXC_ERR_CUDA, "CUDA error: %s", cudaGetErrorString(e));
  }
  ctx->launches++;
  ctx->granite_rope = tab;
  return QXC_OK;
}

qxc_status ensure_qwen_rope(qxc_ctx* ctx) {
  if (ctx->qwen_rope) return QXC_OK;
  // cos/sin of position * 1e6^(-i/64) with the platform's single-precision
  // powf/sinf/cosf, as tools/qx-qwen-parity/src/main.rs:1193-1195 evaluates
  // them; computed once on the host so the device never evaluates
  // transcendental RoPE and every position's values equal the host's.
  std::vector<float2> tab((size_t)kQwenMaxPositions * 64);
  float inv[64];
  for (int i = 0; i < 64; ++i) inv[i] = powf(1000000.0f, -(float)i / 64.0f);
  for (int pos = 0; pos < kQwenMaxPositions; ++pos)
    for (int i = 0; i < 64; ++i) {
      volatile float angle = (float)pos * inv[i];
      tab[(size_t)pos * 64 + i] = make_float2(cosf(angle), sinf(angle));
    }
  QXC_CUDA(ctx, cudaMalloc(&ctx->qwen_rope, tab.size() * sizeof(float2)));
  QXC_CUDA(ctx, cudaMemcpy(ctx->qwen_rope, tab.data(), tab.size() * sizeof(float2), cudaMemcpyHostToDevice));
  return QXC_OK;
}

}  // namespace

// ============================================================================
// Q4 mat-vec kernel, a programmatic dependent like the decode.
qxc_status launch_matvec(qxc_ctx* ctx, const LayerParams& p) {
  int rows = 0;
  for (int m = 0; m < p.nmat; ++m) rows += p.w[m].rows;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(std::min(1024, (rows + 7) / 8));
  cfg.blockDim = dim3(256);
  cfg.stream = ctx->stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  QXC_CUDA(ctx, cudaLaunchKernelEx(&cfg, qx_q4_matvec_kernel, p));
  ctx->launches++;
  return QXC_OK;
}

qxc_status check_q4(qxc_ctx* ctx, const qxc_q4_matrix* w, int rows, int cols, const char* name) {
  if (!w->codes || !w->scales) return fail(ctx, QXC_ERR_INVALID_ARG, "%s: null Q4 data", name);
  if ((rows && w->rows != rows) || (cols && w->cols != cols))
    return fail(ctx, QXC_ERR_INVALID_ARG, "%s must be %d x %d, got %d x %d", name, rows, cols, w->rows, w->cols);
  if (w->rows < 1 || w->cols < 32 || w->cols % 32 != 0 || w->cols > 4 * kHidden)
    return fail(ctx, QXC_ERR_INVALID_ARG, "%s: %d x %d is not a Q4 shape (cols a multiple of 32, at most %d)", name,
                w->rows, w->cols, 4 * kHidden);
  return QXC_OK;
}

Q4Ref q4ref(const qxc_q4_matrix& w) {
  Q4Ref r;
  r.codes = w.codes;
  r.scales = w.scales;
  r.rows = w.rows;
  r.cols = w.cols;
  return r;
}

// Append kernel of qxc_decode_verify, a programmatic dependent like the decode.
template <class M, typename KT, typename VT>
qxc_status launch_append(qxc_ctx* ctx, const AppendParams& a, int grid) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(128);
  cfg.stream = ctx->stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  QXC_CUDA(ctx, cudaLaunchKernelEx(&cfg, qx_append_rows_kernel<M, KT, VT>, a));
  ctx->launches++;
  return QXC_OK;
}

// ---- paged arenas ----------------------------------------------------------------
// Send new block-table entries to the device in stream order.
qxc_status push_table(qxc_ctx* ctx, qxc_kv* kv, const std::vector<int>& idx, const std::vector<int>& val) {
  for (size_t at = 0; at < idx.size(); at += kPageUpdates) {
    PageUpdates u;
    u.table = kv->table_dev;
    u.n = (int)std::min<size_t>(kPageUpdates, idx.size() - at);
    for (int i = 0; i < u.n; ++i) {
      u.index[i] = idx[at + i];
      u.page[i] = val[at + i];
    }
    qx_page_table_kernel<<<1, 128, 0, ctx->stream>>>(u);
    QXC_CUDA(ctx, cudaGetLastError());
    ctx->launches++;
  }
  return QXC_OK;
}

// Map pages so that rows [0, rows[i]) of sequence seqs[i] exist, all or
// nothing: when the pool cannot cover every request, nothing is mapped.
qxc_status ensure_pages(qxc_ctx* ctx, qxc_kv* kv, int n, const int* seqs, const int* rows) {
  if (!kv->paged()) return QXC_OK;
  long long need = 0;
  for (int i = 0; i < n; ++i) need += std::max(0, kv->pages_for(rows[i]) - kv->mapped[seqs[i]]);
  if (need == 0) return QXC_OK;
  if (need > (long long)kv->free_pages.size())
    return fail(ctx, QXC_ERR_OUT_OF_MEMORY, "KV page pool exhausted: %lld more pages needed, %zu of %d free", need,
                kv->free_pages.size(), kv->pool_pages);
  std::vector<int> idx, val;
  for (int i = 0; i < n; ++i) {
    const int seq = seqs[i], want = kv->pages_for(rows[i]);
    while (kv->mapped[seq] < want) {
      const int page = kv->free_pages.back();
      kv->free_pages.pop_back();
      const int e = seq * kv->table_stride + kv->mapped[seq];
      kv->table[e] = page;
      idx.push_back(e);
      val.push_back(page);
      kv->mapped[seq]++;
    }
  }
  return push_table(ctx, kv, idx, val);
}

// Return the pages of `seq` past its first `keep` logical pages to the pool.
// Their device table entries stay as they were: nothing reads them until the
// pages are mapped again, which sends fresh entries.
void release_pages(qxc_kv* kv, int seq, int keep) {
  while (kv->mapped[seq] > keep) {
    const int e = seq * kv->table_stride + --kv->mapped[seq];
    kv->free_pages.push_back(kv->table[e]);
    kv->table[e] = -1;
  }
}

// Hash kernel, a programmatic dependent like the decode (it waits for the
// stream's previous kernel before reading rows).
qxc_status launch_hash(qxc_ctx* ctx, const HashParams& p, int ctas, void (*fn)(HashParams) = qx_kv_hash_kernel,
                       int smem = 0, int warps_per_cta = kHashWarps) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ctas);
  cfg.blockDim = dim3(32 * warps_per_cta);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = ctx->stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  QXC_CUDA(ctx, cudaLaunchKernelEx(&cfg, fn, p));
  ctx->launches++;
  return QXC_OK;
}

// Row geometry shared by both hash entry points: rows of 1, 2, 4 or 8
// 256-byte chunks (encode_verification_hashes' rule, qx-metal lib.rs:9288-9302).
qxc_status hash_params(qxc_ctx* ctx, const qxc_kv* kv, int seq, HashParams* p) {
  memset(p, 0, sizeof(*p));
  const long long krow = (long long)kv->hkv * kv->d * (long long)kv->kes;
  const long long vrow = (long long)kv->hkv * kv->d * (long long)kv->ves;
  for (long long b : {krow, vrow}) {
    const long long c = b / 256;
    if (b % 256 != 0 || c < 1 || c > 8 || (c & (c - 1)) != 0)
      return fail(ctx, QXC_ERR_UNSUPPORTED, "KV row of %lld bytes is not 1, 2, 4 or 8 chunks of 256", b);
  }
  p->k_region = kv->k_region;
  p->v_region = kv->v_region;
  p->capacity = kv->desc.capacity;
  p->paging = kv_paging(kv);
  p->key_row_bytes = (int)krow;
  p->value_row_bytes = (int)vrow;
  p->layers = kv->desc.layers;
  p->seq = seq;
  p->checkpoint_interval = 1;
  // hash_domain's framing of a chunk leaf up to the chunk bytes (qx-commit
  // state.rs:225-233): domain, u64 4, u32 index (zero here), u64 256
  const char* domains[3] = {"QX:STATE:CHUNK:V1", "QX:KV:KEY:CHUNK:V1", "QX:KV:VALUE:CHUNK:V1"};
  for (int r = 0; r < 3; ++r) {
    unsigned char b[48] = {0};
    const size_t n = strlen(domains[r]);
    memcpy(b, domains[r], n);
    b[n] = 4;          // u64 4
    b[n + 12 + 1] = 1;  // u64 256 = 00 01 00 ...
    p->prefix_len[r] = (int)n + 20;
    for (int w = 0; w < 12; ++w)
      p->prefix[r][w] = (uint32_t)b[4 * w] | (uint32_t)b[4 * w + 1] << 8 | (uint32_t)b[4 * w + 2] << 16 |
                        (uint32_t)b[4 * w + 3] << 24;
  }
  return QXC_OK;
}

// Speculative verify of 2..4 Granite candidates with shared tiles
// (GraniteVerify4): one work item per (layer, kv head, split) scores each
// cache tile against all candidates' query rows, so the cache is read once
// per call instead of once per candidate.
template <typename KT, typename VT>
qxc_status launch_verify_typed(qxc_ctx* ctx, qxc_kv* kv, const qxc_verify_args* a) {
  using C = DecodeCfg<GraniteVerify4, KT, VT>;
  static int slots_cache[64] = {};
  int& slots = slots_cache[ctx->device & 63];
  if (!slots) {
    QXC_CUDA(ctx, cudaFuncSetAttribute(qx_verify_kernel<KT, VT>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
    int n = 1;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, qx_verify_kernel<KT, VT>, C::NT, C::SMEM) != cudaSuccess || n < 1)
      n = 1;
    slots = ctx->sm_count * n;
  }
  int attend = a->start + a->tokens, none = -1, rope = a->start, seq = a->seq;
  const int split = a->split ? a->split : auto_chunk(slots, &attend, 1, a->layer_count * kv->hkv, C::MAX_SPLITS, 64);
  if ((attend + split - 1) / split > C::MAX_SPLITS)
    return fail(ctx, QXC_ERR_INVALID_ARG, "split %d gives %d splits; at most %d fit the merge", split,
                (attend + split - 1) / split, C::MAX_SPLITS);
  CallPlan plan;
  qxc_status st = plan_call(ctx, kv, 1, &seq, &attend, &none, &rope, a->layer_count, split, &plan, kv->hkv);
  if (st != QXC_OK) return st;
  DecodeParams p;
  st = fill_params(ctx, kv, plan, a->layer_begin, a->layer_count, &p);
  if (st != QXC_OK) return st;
  note_rows_open(ctx);  // the verify kernel triggers its dependents at its start
  st = grow(ctx, &ctx->partials, &ctx->partials_cap, (size_t)plan.items * C::G * (C::D + 2), false);
  if (st != QXC_OK) return st;
  p.partials = ctx->partials;
  p.early_trigger = plan.items <= slots ? 1 : 0;
  p.q = a->q;
  p.k = a->k;  // not read: the rows were appended already
  p.v = a->v;
  p.out = a->out;
  p.q_dtype = a->q_dtype;
  p.in_dtype = a->in_dtype;
  p.out_dtype = a->out_dtype;
  p.pinned_exp = default_pinned(kv, a->flags) ? 1 : 0;
  p.ntok = a->tokens;
  {
    TraceRun tr(ctx, "verify", plan.items);
    p.trace = tr.buf;
    QXC_CUDA(ctx, launch_pdl(ctx, qx_verify_kernel<KT, VT>, plan.items, C::NT, C::SMEM, p));
    ctx->launches++;
  }
  if (!p.external_merge) return QXC_OK;
  p.trace = nullptr;
  const int grid = a->layer_count * GraniteVerify4::HQ * (GraniteVerify4::D / 32);
  QXC_CUDA(ctx, launch_pdl(ctx, qx_split_merge_kernel<8, 64, 8, 64, 4, 2>, grid, 128, 0, p));
  ctx->launches++;
  return QXC_OK;
}

qxc_status launch_verify_shared(qxc_ctx* ctx, qxc_kv* kv, const qxc_verify_args* a) {
  const int kd = kv->desc.key_dtype, vd = kv->desc.value_dtype;
  if (kd == QXC_F32 && vd == QXC_F32) return launch_verify_typed<float, float>(ctx, kv, a);
  if (kd == QXC_F32 && vd == QXC_F16) return launch_verify_typed<float, __half>(ctx, kv, a);
  if (kd == QXC_F16 && vd == QXC_F32) return launch_verify_typed<__half, float>(ctx, kv, a);
  if (kd == QXC_F16 && vd == QXC_F16) return launch_verify_typed<__half, __half>(ctx, kv, a);
  return launch_verify_typed<__nv_bfloat16, __nv_bfloat16>(ctx, kv, a);
}

extern "C" {

int qxc_abi_version(void) { return QXC_ABI_VERSION; }

const char* qxc_status_string(qxc_status s) {
  switch (s) {
    case QXC_OK: return "ok";
    case QXC_ERR_INVALID_ARG: return "invalid argument";
    case QXC_ERR_POSITION: return "KV position error";
    case QXC_ERR_NONFINITE: return "non-finite value";
    case QXC_ERR_CUDA: return "CUDA error";
    case QXC_ERR_NCCL: return "NCCL error";
    case QXC_ERR_TIMEOUT: return "device wait timed out";
    case QXC_ERR_UNSUPPORTED: return "unsupported";
    case QXC_ERR_OUT_OF_MEMORY: return "out of device memory";
  }
  return "unknown status";
}

qxc_status qxc_init(int device, qxc_ctx** out) {
  if (!out) return QXC_ERR_INVALID_ARG;
  *out = nullptr;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) return QXC_ERR_CUDA;
  qxc_ctx* ctx = new (std::nothrow) qxc_ctx();
  if (!ctx) return QXC_ERR_OUT_OF_MEMORY;
  ctx->device = device;
  if (cudaSetDevice(device) != cudaSuccess) {
    delete ctx;
    return QXC_ERR_CUDA;
  }
  cudaDeviceGetAttribute(&ctx->sm_count, cudaDevAttrMultiProcessorCount, device);
  if (cudaStreamCreateWithFlags(&ctx->own_stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaHostAlloc(reinterpret_cast<void**>(&ctx->err_host), sizeof(unsigned), cudaHostAllocMapped) != cudaSuccess ||
      cudaHostGetDevicePointer(reinterpret_cast<void**>(&ctx->err_dev), ctx->err_host, 0) != cudaSuccess) {
    qxc_destroy(ctx);
    return QXC_ERR_CUDA;
  }
  *ctx->err_host = 0;
  ctx->stream = ctx->own_stream;
  *out = ctx;
  return QXC_OK;
}

void qxc_destroy(qxc_ctx* ctx) {
  if (!ctx) return;
  cudaSetDevice(ctx->device);
  if (ctx->stream) cudaStreamSynchronize(ctx->stream);
  cudaFree(ctx->partials);
  cudaFree(ctx->tpartials);
  cudaFree(ctx->tickets);
  for (int i = 0; i < qxc_ctx::kRing; ++i) {
    cudaFree(ctx->seq_dev[i]);
    if (ctx->seq_host[i]) cudaFreeHost(ctx->seq_host[i]);
    if (ctx->seq_ev[i]) cudaEventDestroy(ctx->seq_ev[i]);
  }
  cudaFree(ctx->stage_dev);
  cudaFree(ctx->qwen_rope);
  cudaFree(ctx->granite_rope);
  cudaFree(ctx->layer_scratch);
  cudaFree(ctx->stack_x);
  cudaFree(ctx->stack_f);
  cudaFree(ctx->stack_words);
  cudaFree(ctx->prefill_q);
  if (ctx->err_host) cudaFreeHost(ctx->err_host);
  if (ctx->own_stream) cudaStreamDestroy(ctx->own_stream);
  delete ctx;
}

qxc_status qxc_set_stream(qxc_ctx* ctx, void* stream) {
  if (!ctx) return QXC_ERR_INVALID_ARG;
  ctx->stream = stream ? static_cast<cudaStream_t>(stream) : ctx->own_stream;
  return QXC_OK;
}

void* qxc_get_stream(qxc_ctx* ctx) { return ctx ? static_cast<void*>(ctx->stream) : nullptr; }

qxc_status qxc_sync(qxc_ctx* ctx) {
  if (!ctx) return QXC_ERR_INVALID_ARG;
  QXC_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  const unsigned e = *reinterpret_cast<volatile unsigned*>(ctx->err_host);
  if (e) {
    *reinterpret_cast<volatile unsigned*>(ctx->err_host) = 0;
    // a kernel that stopped early may have left split tickets raised
    if (ctx->tickets) {
      cudaMemsetAsync(ctx->tickets, 0, ctx->tickets_cap * sizeof(int), ctx->stream);
      cudaStreamSynchronize(ctx->stream);
    }
    // and a stack launch that gave up has raised its abort word and may
    // have left merge tickets raised
    if (ctx->stack_words) {
      cudaMemsetAsync(ctx->stack_words, 0, 16 * sizeof(unsigned), ctx->stream);
      cudaStreamSynchronize(ctx->stream);
      ctx->stack_tickets = 0;
    }
    if (e & QX_ERR_BIT_PEER)
      return fail(ctx, QXC_ERR_TIMEOUT,
                  "a bounded device-side wait gave up: an exchange with a peer rank timed out, and its peer group "
                  "is failed (destroy and re-create the groups on every rank)");
    if (e & QX_ERR_BIT_TIMEOUT) return fail(ctx, QXC_ERR_TIMEOUT, "a bounded device-side wait gave up");
    return fail(ctx, QXC_ERR_NONFINITE, "non-finite value in RoPE or attention (the reference panics here)");
  }
  return QXC_OK;
}

const char* qxc_last_error(const qxc_ctx* ctx) { return ctx ? ctx->err.c_str() : "null context"; }

uint64_t qxc_launch_count(const qxc_ctx* ctx) { return ctx ? ctx->launches : 0; }

int32_t qxc_last_split(const qxc_ctx* ctx) { return ctx ? ctx->last_split : 0; }

int32_t qxc_auto_split(int32_t slots, const int32_t* attend, int32_t n, int32_t units, int32_t max_splits,
                       int32_t tile) {
  if (slots < 1 || !attend || n < 1 || units < 1 || max_splits < 1 || tile < 1) return 0;
  for (int i = 0; i < n; ++i)
    if (attend[i] < 1) return 0;
  return auto_chunk(slots, attend, n, units, max_splits, tile);
}

// ---- KV arena ---------------------------------------------------------------
qxc_status qxc_kv_bytes(const qxc_kv_desc* d, size_t* key_bytes, size_t* value_bytes) {
  qxc_status st = check_desc(nullptr, d);
  if (st != QXC_OK) return st;
  int hq, hkv, hd;
  model_shape(d->model, &hq, &hkv, &hd);
  const size_t per = (size_t)d->capacity * hkv * hd * (size_t)d->layers * d->sequences;
  if (key_bytes) *key_bytes = per * dtype_size(d->key_dtype);
  if (value_bytes) *value_bytes = per * dtype_size(d->value_dtype);
  return QXC_OK;
}

static qxc_status check_paging(qxc_ctx* ctx, const qxc_kv_desc* d, const qxc_kv_paging* pg) {
  if (!pg) return fail(ctx, QXC_ERR_INVALID_ARG, "null paging descriptor");
  if (pg->page_size < 64 || pg->page_size > 4096 || (pg->page_size & (pg->page_size - 1)) != 0)
    return fail(ctx, QXC_ERR_INVALID_ARG, "page size %d must be a power of two in 64..=4096", pg->page_size);
  if (pg->pool_pages < 1) return fail(ctx, QXC_ERR_INVALID_ARG, "the page pool needs at least one page");
  if (d->first_position != 0) return fail(ctx, QXC_ERR_UNSUPPORTED, "a paged arena cannot be a KV-length shard");
  // TMA row coordinates are 32-bit
  if ((long long)d->layers * pg->pool_pages * pg->page_size > 0x7fffffffLL)
    return fail(ctx, QXC_ERR_INVALID_ARG, "%d layers x %d pages x %d rows exceed 2^31 rows", d->layers,
                pg->pool_pages, pg->page_size);
  return QXC_OK;
}

// One allocation: keys [layers][pool][page][kv_heads][head_dim] (paged) or
// [sequences][layers][capacity][kv_heads][head_dim] (contiguous), then values.
static qxc_status kv_create(qxc_ctx* ctx, const qxc_kv_desc* desc, const qxc_kv_paging* paging, qxc_kv** out) {
  if (!ctx || !out) return QXC_ERR_INVALID_ARG;
  *out = nullptr;
  qxc_status st = check_desc(ctx, desc);
  if (st != QXC_OK) return st;
  if (paging) {
    st = check_paging(ctx, desc, paging);
    if (st != QXC_OK) return st;
  }
  QXC_CUDA(ctx, cudaSetDevice(ctx->device));
  qxc_kv* kv = new (std::nothrow) qxc_kv();
  if (!kv) return fail(ctx, QXC_ERR_OUT_OF_MEMORY, "host allocation failed");
  kv->ctx = ctx;
  kv->desc = *desc;
  model_shape(desc->model, &kv->hq, &kv->hkv, &kv->d);
  kv->kes = dtype_size(desc->key_dtype);
  kv->ves = dtype_size(desc->value_dtype);
  kv->k_unit = (size_t)desc->capacity * kv->hkv * kv->d * kv->kes;
  kv->v_unit = (size_t)desc->capacity * kv->hkv * kv->d * kv->ves;
  size_t rows = (size_t)desc->layers * desc->sequences * desc->capacity;
  if (paging) {
    for (int s2 = 1; (1 << s2) <= paging->page_size; ++s2) kv->page_shift = s2;
    kv->pool_pages = paging->pool_pages;
    kv->table_stride = kv->pages_for(desc->capacity);
    kv->table.assign((size_t)desc->sequences * kv->table_stride, -1);
    kv->mapped.assign(desc->sequences, 0);
    for (int pg = paging->pool_pages - 1; pg >= 0; --pg) kv->free_pages.push_back(pg);
    rows = (size_t)desc->layers * paging->pool_pages * paging->page_size;
  }
  const size_t kbytes = rows * kv->hkv * kv->d * kv->kes, vbytes = rows * kv->hkv * kv->d * kv->ves;
  const size_t koff_v = ((kbytes + 255) / 256) * 256;
  cudaError_t e = cudaMalloc(&kv->base, koff_v + vbytes);
  if (e == cudaSuccess && paging) {
    e = cudaMalloc(&kv->table_dev, kv->table.size() * sizeof(int));
    if (e != cudaSuccess) cudaFree(kv->base);
  }
  if (e != cudaSuccess) {
    delete kv;
    return fail(ctx, e == cudaErrorMemoryAllocation ? QXC_ERR_OUT_OF_MEMORY : QXC_ERR_CUDA,
                "KV arena of %zu bytes: %s", koff_v + vbytes, cudaGetErrorString(e));
  }
  // Zero-initialised like KvCache::new (qx-runtime lib.rs:359-368).
  cudaMemsetAsync(kv->base, 0, koff_v + vbytes, ctx->stream);
  if (kv->table_dev) cudaMemsetAsync(kv->table_dev, 0xff, kv->table.size() * sizeof(int), ctx->stream);  // -1
  kv->k_region = kv->base;
  kv->v_region = kv->base + koff_v;
  kv->len.assign(desc->sequences, 0);
  qxc_status mst = encode_kv_map(ctx, &kv->tmk, kv->k_region, desc->key_dtype, kv->hkv, kv->d, rows);
  if (mst == QXC_OK) mst = encode_kv_map(ctx, &kv->tmv, kv->v_region, desc->value_dtype, kv->hkv, kv->d, rows);
  if (mst == QXC_OK && desc->model == QXC_MODEL_QWEN3) mst = ensure_qwen_rope(ctx);
  if (mst != QXC_OK) {
    cudaFree(kv->base);
    if (kv->table_dev) cudaFree(kv->table_dev);
    delete kv;
    return mst;
  }
  kv->rope_table = ctx->qwen_rope;
  QXC_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  *out = kv;
  return QXC_OK;
}

qxc_status qxc_kv_create(qxc_ctx* ctx, const qxc_kv_desc* desc, qxc_kv** out) {
  return kv_create(ctx, desc, nullptr, out);
}

qxc_status qxc_kv_create_paged(qxc_ctx* ctx, const qxc_kv_desc* desc, const qxc_kv_paging* paging, qxc_kv** out) {
  if (!paging) return fail(ctx, QXC_ERR_INVALID_ARG, "null paging descriptor");
  return kv_create(ctx, desc, paging, out);
}

qxc_status qxc_kv_paged_bytes(const qxc_kv_desc* d, const qxc_kv_paging* pg, size_t* key_bytes, size_t* value_bytes) {
  qxc_status st = check_desc(nullptr, d);
  if (st != QXC_OK) return st;
  st = check_paging(nullptr, d, pg);
  if (st != QXC_OK) return st;
  int hq, hkv, hd;
  model_shape(d->model, &hq, &hkv, &hd);
  const size_t per = (size_t)d->layers * pg->pool_pages * pg->page_size * hkv * hd;
  if (key_bytes) *key_bytes = per * dtype_size(d->key_dtype);
  if (value_bytes) *value_bytes = per * dtype_size(d->value_dtype);
  return QXC_OK;
}

qxc_status qxc_kv_page_stats(const qxc_kv* kv, int32_t seq, int32_t* mapped_pages, int32_t* free_pages) {
  if (!kv) return QXC_ERR_INVALID_ARG;
  if (!kv->paged()) return fail(kv->ctx, QXC_ERR_UNSUPPORTED, "the arena is not paged");
  if (seq >= kv->desc.sequences) return fail(kv->ctx, QXC_ERR_INVALID_ARG, "sequence %d out of range", seq);
  if (mapped_pages) *mapped_pages = seq < 0 ? kv->pool_pages - (int)kv->free_pages.size() : kv->mapped[seq];
  if (free_pages) *free_pages = (int)kv->free_pages.size();
  return QXC_OK;
}

qxc_status qxc_kv_pool_buffer(qxc_kv* kv, int32_t key, void** ptr, size_t* bytes) {
  if (!kv || !ptr) return QXC_ERR_INVALID_ARG;
  if (!kv->paged()) return fail(kv->ctx, QXC_ERR_UNSUPPORTED, "the arena is not paged");
  const size_t rows = (size_t)kv->desc.layers * kv->pool_pages << kv->page_shift;
  *ptr = key ? kv->k_region : kv->v_region;
  if (bytes) *bytes = rows * kv->hkv * kv->d * (key ? kv->kes : kv->ves);
  return QXC_OK;
}

qxc_status qxc_kv_trim(qxc_kv* kv, int32_t seq) {
  if (!kv) return QXC_ERR_INVALID_ARG;
  qxc_status st = check_seq(kv->ctx, kv, seq);
  if (st != QXC_OK) return st;
  if (kv->paged()) release_pages(kv, seq, kv->pages_for(kv->len[seq]));
  return QXC_OK;
}

void qxc_kv_destroy(qxc_kv* kv) {
  if (!kv) return;
  cudaSetDevice(kv->ctx->device);
  cudaStreamSynchronize(kv->ctx->stream);
  cudaFree(kv->base);
  if (kv->table_dev) cudaFree(kv->table_dev);
  delete kv;
}

qxc_status qxc_kv_len(const qxc_kv* kv, int32_t seq, int32_t* length) {
  if (!kv || !length) return QXC_ERR_INVALID_ARG;
  if (seq < 0 || seq >= kv->desc.sequences) return QXC_ERR_INVALID_ARG;
  *length = kv->len[seq];
  return QXC_OK;
}

// A reset sequence's pages go back to the pool (paged arenas).
qxc_status qxc_kv_reset(qxc_kv* kv, int32_t seq) {
  if (!kv) return QXC_ERR_INVALID_ARG;
  if (seq < 0) {
    std::fill(kv->len.begin(), kv->len.end(), 0);
    if (kv->paged())
      for (int i = 0; i < kv->desc.sequences; ++i) release_pages(kv, i, 0);
    return QXC_OK;
  }
  if (seq >= kv->desc.sequences) return fail(kv->ctx, QXC_ERR_INVALID_ARG, "sequence %d out of range", seq);
  kv->len[seq] = 0;
  if (kv->paged()) release_pages(kv, seq, 0);
  return QXC_OK;
}

qxc_status qxc_kv_set_len(qxc_kv* kv, int32_t seq, int32_t length) {
  if (!kv) return QXC_ERR_INVALID_ARG;
  qxc_status st = check_seq(kv->ctx, kv, seq);
  if (st != QXC_OK) return st;
  if (length < 0 || length > kv->desc.capacity)
    return fail(kv->ctx, QXC_ERR_POSITION, "KV length %d is outside capacity %d", length, kv->desc.capacity);
  st = ensure_pages(kv->ctx, kv, 1, &seq, &length);
  if (st != QXC_OK) return st;
  kv->len[seq] = length;
  return QXC_OK;
}

qxc_status qxc_kv_checkpoint(const qxc_kv* kv, int32_t seq, int32_t* sequence_len) {
  return qxc_kv_len(kv, seq, sequence_len);
}

// rollback_kv (qx-runtime-v2 lib.rs:3273-3286)
qxc_status qxc_kv_rollback(qxc_kv* kv, int32_t seq, int32_t sequence_len) {
  if (!kv) return QXC_ERR_INVALID_ARG;
  qxc_status st = check_seq(kv->ctx, kv, seq);
  if (st != QXC_OK) return st;
  if (sequence_len < 0 || sequence_len > kv->len[seq] || sequence_len > kv->desc.capacity)
    return fail(kv->ctx, QXC_ERR_POSITION, "KV rollback checkpoint %d is outside current position %d / context %d",
                sequence_len, kv->len[seq], kv->desc.capacity);
  kv->len[seq] = sequence_len;
  return QXC_OK;
}

// commit_kv (qx-runtime-v2 lib.rs:3291-3310)
qxc_status qxc_kv_commit(qxc_kv* kv, int32_t seq, int32_t sequence_len, int32_t accepted_prefix) {
  if (!kv) return QXC_ERR_INVALID_ARG;
  qxc_status st = check_seq(kv->ctx, kv, seq);
  if (st != QXC_OK) return st;
  if (sequence_len < 0 || accepted_prefix < 0 || (long long)sequence_len + accepted_prefix > 0x7fffffffLL)
    return fail(kv->ctx, QXC_ERR_POSITION, "KV commit position overflow");
  const int end = sequence_len + accepted_prefix;
  const int position = kv->len[seq];
  if (sequence_len > position || end > position || end > kv->desc.capacity)
    return fail(kv->ctx, QXC_ERR_POSITION, "KV commit [%d, %d) is outside current speculative range ending at %d",
                sequence_len, end, position);
  kv->len[seq] = end;
  return QXC_OK;
}

static qxc_status kv_view(qxc_kv* kv, int32_t seq, int32_t layer, bool key, void** ptr, size_t* bytes) {
  if (!kv || !ptr) return QXC_ERR_INVALID_ARG;
  if (seq < 0 || seq >= kv->desc.sequences) return fail(kv->ctx, QXC_ERR_INVALID_ARG, "sequence %d out of range", seq);
  if (layer < 0 || layer >= kv->desc.layers)
    return fail(kv->ctx, QXC_ERR_INVALID_ARG, "KV layer %d is outside the plan", layer);
  if (kv->paged())
    return fail(kv->ctx, QXC_ERR_UNSUPPORTED, "a paged arena has no contiguous view of one cache");
  const size_t unit = (size_t)seq * kv->desc.layers + layer;
  *ptr = key ? kv->k_region + unit * kv->k_unit : kv->v_region + unit * kv->v_unit;
  if (bytes) *bytes = key ? kv->k_unit : kv->v_unit;
  return QXC_OK;
}

qxc_status qxc_kv_key_buffer(qxc_kv* kv, int32_t seq, int32_t layer, void** p, size_t* bytes) {
  return kv_view(kv, seq, layer, true, p, bytes);
}
qxc_status qxc_kv_value_buffer(qxc_kv* kv, int32_t seq, int32_t layer, void** p, size_t* bytes) {
  return kv_view(kv, seq, layer, false, p, bytes);
}

static qxc_status kv_copy(qxc_kv* kv, int32_t seq, int32_t layer, int32_t begin, int32_t count, void* hk,
                          void* hv, bool to_host) {
  if (!kv) return QXC_ERR_INVALID_ARG;
  qxc_ctx* ctx = kv->ctx;
  qxc_status st = check_seq(ctx, kv, seq);
  if (st != QXC_OK) return st;
  if (layer < 0 || layer >= kv->desc.layers)
    return fail(ctx, QXC_ERR_INVALID_ARG, "KV layer %d is outside the plan", layer);
  if (begin < 0 || count < 0 || (long long)begin + count > kv->desc.capacity)
    return fail(ctx, QXC_ERR_INVALID_ARG, "slots [%d, %d) outside capacity %d", begin, begin + count, kv->desc.capacity);
  QXC_CUDA(ctx, cudaSetDevice(ctx->device));
  if (kv->paged()) {
    const int end = begin + count;
    if (to_host) {
      if (kv->pages_for(end) > kv->mapped[seq])
        return fail(ctx, QXC_ERR_INVALID_ARG, "slots [%d, %d) are not all mapped (%d pages of %d rows)", begin, end,
                    kv->mapped[seq], 1 << kv->page_shift);
    } else {
      st = ensure_pages(ctx, kv, 1, &seq, &end);
      if (st != QXC_OK) return st;
    }
  }
  QXC_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
  const size_t krow = (size_t)kv->hkv * kv->d * kv->kes, vrow = (size_t)kv->hkv * kv->d * kv->ves;
  const KvPaging pg = kv_paging(kv);
  // runs of rows contiguous in the arena: the whole range, or one page at a time
  for (int r = begin; r < begin + count;) {
    int n = begin + count - r;
    long long arow;
    if (kv->paged()) {
      const int page_rows = 1 << kv->page_shift;
      n = std::min(n, page_rows - (r & (page_rows - 1)));
      arow = ((long long)layer * pg.pool + kv->table[seq * pg.stride + (r >> pg.shift)]) * page_rows +
             (r & (page_rows - 1));
    } else {
      arow = ((long long)seq * kv->desc.layers + layer) * kv->desc.capacity + r;
    }
    char* kdev = kv->k_region + arow * krow;
    char* vdev = kv->v_region + arow * vrow;
    char* kh = hk ? static_cast<char*>(hk) + (size_t)(r - begin) * krow : nullptr;
    char* vh = hv ? static_cast<char*>(hv) + (size_t)(r - begin) * vrow : nullptr;
    if (kh) {
      if (to_host) QXC_CUDA(ctx, cudaMemcpy(kh, kdev, (size_t)n * krow, cudaMemcpyDeviceToHost));
      else QXC_CUDA(ctx, cudaMemcpy(kdev, kh, (size_t)n * krow, cudaMemcpyHostToDevice));
    }
    if (vh) {
      if (to_host) QXC_CUDA(ctx, cudaMemcpy(vh, vdev, (size_t)n * vrow, cudaMemcpyDeviceToHost));
      else QXC_CUDA(ctx, cudaMemcpy(vdev, vh, (size_t)n * vrow, cudaMemcpyHostToDevice));
    }
    r += n;
  }
  return QXC_OK;
}

qxc_status qxc_kv_read(qxc_kv* kv, int32_t seq, int32_t layer, int32_t begin, int32_t count, void* hk, void* hv) {
  return kv_copy(kv, seq, layer, begin, count, hk, hv, true);
}
qxc_status qxc_kv_write(qxc_kv* kv, int32_t seq, int32_t layer, int32_t begin, int32_t count, const void* hk,
                        const void* hv) {
  return kv_copy(kv, seq, layer, begin, count, const_cast<void*>(hk), const_cast<void*>(hv), false);
}

// ---- decode -------------------------------------------------------------------
qxc_status qxc_decode(qxc_ctx* ctx, qxc_kv* kv, const qxc_decode_args* a) {
  if (!ctx || !kv || !a) return fail(ctx, QXC_ERR_INVALID_ARG, "null argument");
  if (kv->ctx != ctx) return fail(ctx, QXC_ERR_INVALID_ARG, "KV arena belongs to another context");
  if (a->seq_count < 1 || !a->positions) return fail(ctx, QXC_ERR_INVALID_ARG, "seq_count >= 1 and positions required");
  if (a->layer_count < 1 || a->layer_begin < 0 || a->layer_begin + a->layer_count > kv->desc.layers)
    return fail(ctx, QXC_ERR_INVALID_ARG, "layers [%d, %d) outside the arena's %d layers", a->layer_begin,
                a->layer_begin + a->layer_count, kv->desc.layers);
  if (!a->q || !a->k || !a->v || !a->out) return fail(ctx, QXC_ERR_INVALID_ARG, "null tensor pointer");
  if (!valid_dtype(a->q_dtype) || !valid_dtype(a->in_dtype) || !valid_dtype(a->out_dtype))
    return fail(ctx, QXC_ERR_INVALID_ARG, "unknown tensor dtype");
  if (kv->desc.model == QXC_MODEL_QWEN3 && (a->q_dtype != kv->desc.key_dtype || a->in_dtype != kv->desc.key_dtype))
    return fail(ctx, QXC_ERR_INVALID_ARG, "Qwen q/k/v must use the KV cache's 16-bit type");
  if (kv->desc.first_position != 0)
    return fail(ctx, QXC_ERR_INVALID_ARG, "a KV-length shard decodes through qxc_decode_partials");
  std::vector<int> attend(a->seq_count), new_slot(a->seq_count), rope(a->seq_count);
  std::vector<char> seen(kv->desc.sequences, 0);
  for (int i = 0; i < a->seq_count; ++i) {
    const int seq = a->seq_ids ? a->seq_ids[i] : i;
    qxc_status st = check_seq(ctx, kv, seq);
    if (st != QXC_OK) return st;
    if (seen[seq]) return fail(ctx, QXC_ERR_INVALID_ARG, "sequence %d appears twice in one call", seq);
    seen[seq] = 1;
    const int position = a->positions[i];
    // KvCache::append (qx-runtime lib.rs:385-398)
    if (position != kv->len[seq])
      return fail(ctx, QXC_ERR_POSITION, "KV position %d does not follow cache length %d", position, kv->len[seq]);
    if (position >= kv->desc.capacity)
      return fail(ctx, QXC_ERR_POSITION, "KV position %d exceeds context %d", position, kv->desc.capacity);
    attend[i] = position + 1;
    new_slot[i] = position;
    rope[i] = position;
  }
  QXC_CUDA(ctx, cudaSetDevice(ctx->device));
  {
    std::vector<int> ids(a->seq_count);
    for (int i = 0; i < a->seq_count; ++i) ids[i] = a->seq_ids ? a->seq_ids[i] : i;
    qxc_status st = ensure_pages(ctx, kv, a->seq_count, ids.data(), attend.data());
    if (st != QXC_OK) return st;
  }
  CallPlan plan;
  qxc_status st = plan_call(ctx, kv, a->seq_count, a->seq_ids, attend.data(), new_slot.data(), rope.data(),
                            a->layer_count, a->split, &plan);
  if (st != QXC_OK) return st;
  DecodeParams p;
  st = fill_params(ctx, kv, plan, a->layer_begin, a->layer_count, &p);
  if (st != QXC_OK) return st;
  p.q = a->q;
  p.k = a->k;
  p.v = a->v;
  p.out = a->out;
  p.q_rot_out = a->q_rot_out;
  p.q_norm = a->q_norm;
  p.k_norm = a->k_norm;
  p.q_dtype = a->q_dtype;
  p.in_dtype = a->in_dtype;
  p.out_dtype = a->out_dtype;
  p.pinned_exp = default_pinned(kv, a->flags) ? 1 : 0;
  p.emit_partials = 0;
  st = use_slice_merge(ctx, kv, plan, &p);
  if (st != QXC_OK) return st;
  st = launch_decode(ctx, kv, p, plan.items);
  if (st != QXC_OK) return st;
  if (!(a->flags & QXC_DECODE_NO_ADVANCE))
    for (int i = 0; i < a->seq_count; ++i) kv->len[a->seq_ids ? a->seq_ids[i] : i] += 1;
  return QXC_OK;
}

// ---- Q4 projections around attention ------------------------------------------
qxc_status qxc_q4_mat_vec(qxc_ctx* ctx, const qxc_q4_matrix* w, const float* x, const float* rms_weight,
                          float* y) {
  if (!ctx || !w || !x || !y) return fail(ctx, QXC_ERR_INVALID_ARG, "null argument");
  qxc_status st = check_q4(ctx, w, 0, rms_weight ? kHidden : 0, "matrix");
  if (st != QXC_OK) return st;
  QXC_CUDA(ctx, cudaSetDevice(ctx->device));
  LayerParams p;
  memset(&p, 0, sizeof(p));
  p.hidden = x;
  p.norm = rms_weight;
  p.normalize = rms_weight ? 1 : 0;
  p.w[0] = q4ref(*w);
  p.y[0] = y;
  p.nmat = 1;
  p.err = ctx->err_dev;
  return launch_matvec(ctx, p);
}

qxc_status qxc_attention_layer(qxc_ctx* ctx, qxc_kv* kv, const qxc_layer_args* a) {
  if (!ctx || !kv || !a) return fail(ctx, QXC_ERR_INVALID_ARG, "null argument");
  if (kv->ctx != ctx) return fail(ctx, QXC_ERR_INVALID_ARG, "KV arena belongs to another context");
  if (kv->desc.model != QXC_MODEL_GRANITE) return fail(ctx, QXC_ERR_UNSUPPORTED, "the Q4 layer is Granite's");
  if (!a->hidden_in || !a->hidden_out || !a->input_norm) return fail(ctx, QXC_ERR_INVALID_ARG, "null tensor pointer");
  qxc_status st = check_q4(ctx, &a->q_proj, kHidden, kHidden, "q_proj");
  if (st == QXC_OK) st = check_q4(ctx, &a->k_proj, 512, kHidden, "k_proj");
  if (st == QXC_OK) st = check_q4(ctx, &a->v_proj, 512, kHidden, "v_proj");
  if (st == QXC_OK) st = check_q4(ctx, &a->o_proj, kHidden, kHidden, "o_proj");
  if (st == QXC_OK) st = check_seq(ctx, kv, a->seq);
  if (st != QXC_OK) return st;
  if (a->layer < 0 || a->layer >= kv->desc.layers) return fail(ctx, QXC_ERR_INVALID_ARG, "layer %d out of range", a->layer);
  // KvCache::append (qx-runtime lib.rs:385-398), checked before any launch
  if (a->position != kv->len[a->seq])
    return fail(ctx, QXC_ERR_POSITION, "KV position %d does not follow cache length %d", a->position,
                kv->len[a->seq]);
  if (a->position >= kv->desc.capacity)
    return fail(ctx, QXC_ERR_POSITION, "KV position %d exceeds context %d", a->position, kv->desc.capacity);
  QXC_CUDA(ctx, cudaSetDevice(ctx->device));
  if (!ctx->layer_scratch) QXC_CUDA(ctx, cudaMalloc(&ctx->layer_scratch, 3072 * sizeof(float)));
  float* q = ctx->layer_scratch;
  float* k = q + 1024;
  float* v = k + 512;
  float* att = a->attention_out ? a->attention_out : v + 512;
  // 1. RMSNorm + q/k/v projections
  LayerParams p;
  memset(&p, 0, sizeof(p));
  p.hidden = a->hidden_in;
  p.norm = a->input_norm;
  p.normalize = 1;
  p.w[0] = q4ref(a->q_proj);
  p.w[1] = q4ref(a->k_proj);
  p.w[2] = q4ref(a->v_proj);
  p.y[0] = q;
  p.y[1] = k;
  p.y[2] = v;
  p.nmat = 3;
  p.err = ctx->err_dev;
  st = launch_matvec(ctx, p);
  if (st != QXC_OK) return st;
  // 2. RoPE, append, attention
  qxc_decode_args d;
  memset(&d, 0, sizeof(d));
  const int32_t seq = a->seq, pos = a->position;
  d.layer_begin = a->layer;
  d.layer_count = 1;
  d.seq_count = 1;
  d.seq_ids = &seq;
  d.positions = &pos;
  d.q = q;
  d.k = k;
  d.v = v;
  d.out = att;
  d.q_dtype = d.in_dtype = d.out_dtype = QXC_F32;
  d.flags = a->flags;
  d.split = a->split;
  st = qxc_decode(ctx, kv, &d);
  if (st != QXC_OK) return st;
  // 3. o-projection and residual
  LayerParams o;
  memset(&o, 0, sizeof(o));
  o.hidden = att;
  o.w[0] = q4ref(a->o_proj);
  o.y[0] = a->hidden_out;
  o.nmat = 1;
  o.residual = a->hidden_in;
  o.err = ctx->err_dev;
  return launch_matvec(ctx, o);
}

// ---- the attention sub-layers of a layer stack in one launch (stack.cuh) ------
namespace {

constexpr int kStackHx = 0, kStackQx = 2048, kStackAx = 4096, kStackPx = 5120;
constexpr int kStackTagged = kStackPx + 8 * kStackMaxSplits * kStackPartial;  // uint2 values
constexpr int kStackChain = 0;  // floats: the chain between launches
constexpr int kStackFloats = 2048;

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Cached rows per attention item of a fused launch: the fewest rows (a
// multiple of 64) that cover the attended rows with at most min(16, CTAs/8)
// splits per kv head; 0 when that exceeds the 256 rows a CTA stages.
int stack_chunk(int attend, int ctas, int split) {
  const int max_splits = std::min(kStackMaxSplits, ctas / 8);
  if (max_splits < 1) return 0;
  int chunk = split;
  if (chunk == 0) chunk = ((attend + max_splits - 1) / max_splits + 63) / 64 * 64;
  if (chunk < 64 || chunk % 64 || chunk > kStackMaxTiles * kStackTileRows) return 0;
  if ((attend + chunk - 1) / chunk > max_splits) return 0;
  return chunk;
}

// The fused kernel applies to fp32 contiguous Granite arenas on a GPU whose
// every SM takes one CTA (at least 128, so a CTA's q/k/v and o rows fit its
// buffers) with 16-byte aligned Q4 rows.
bool stack_fusable(qxc_ctx* ctx, const qxc_kv* kv, const qxc_stack_args* a, int chunk) {
  if (kv->desc.key_dtype != QXC_F32 || kv->desc.value_dtype != QXC_F32 || kv->paged() || chunk == 0) return false;
  if (ctx->sm_count < 128 || (2048 + ctx->sm_count - 1) / ctx->sm_count > kStackMaxQkvRows) return false;
  int coop = 0;
  cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, ctx->device);
  if (!coop) return false;
  for (int l = 0; l < a->layer_count; ++l) {
    const qxc_layer_weights& w = a->layers[l];
    for (const qxc_q4_matrix* m : {&w.q_proj, &w.k_proj, &w.v_proj, &w.o_proj})
      if (!aligned16(m->codes) || !aligned16(m->scales)) return false;
  }
  return true;
}

qxc_status launch_stack(qxc_ctx* ctx, const StackParams& p) {
  static unsigned long long configured = 0;
  const unsigned long long bit = 1ull << (ctx->device & 63);
  if (!(configured & bit)) {
    QXC_CUDA(ctx, cudaFuncSetAttribute(qx_attention_stack_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       StackCfg::SMEM));
    int per_sm = 0;
    QXC_CUDA(ctx, cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, qx_attention_stack_kernel, kStackThreads,
                                                                StackCfg::SMEM));
    if (per_sm < 1) return fail(ctx, QXC_ERR_UNSUPPORTED, "the attention stack kernel does not fit an SM");
    configured |= bit;
  }
  TraceRun tr(ctx, "stack", (size_t)ctx->sm_count);
  StackParams q = p;
  q.trace = tr.buf;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ctx->sm_count);
  cfg.blockDim = dim3(kStackThreads);
  cfg.dynamicSmemBytes = StackCfg::SMEM;
  cfg.stream = ctx->stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident: they wait on one another
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  QXC_CUDA(ctx, cudaLaunchKernelEx(&cfg, qx_attention_stack_kernel, q));
  ctx->launches++;
  return QXC_OK;
}

}  // namespace

qxc_status qxc_attention_stack(qxc_ctx* ctx, qxc_kv* kv, const qxc_stack_args* a) {
  if (!ctx || !kv || !a) return fail(ctx, QXC_ERR_INVALID_ARG, "null argument");
  if (kv->ctx != ctx) return fail(ctx, QXC_ERR_INVALID_ARG, "KV arena belongs to another context");
  if (kv->desc.model != QXC_MODEL_GRANITE) return fail(ctx, QXC_ERR_UNSUPPORTED, "the Q4 layer is Granite's");
  if (!a->hidden_in || !a->hidden_out || !a->layers) return fail(ctx, QXC_ERR_INVALID_ARG, "null tensor pointer");
  qxc_status st = check_seq(ctx, kv, a->seq);
  if (st != QXC_OK) return st;
  if (a->layer_count < 1 || a->layer_begin < 0 || a->layer_begin + a->layer_count > kv->desc.layers)
    return fail(ctx, QXC_ERR_INVALID_ARG, "layers [%d, %d) outside the arena's %d layers", a->layer_begin,
                a->layer_begin + a->layer_count, kv->desc.layers);
  for (int l = 0; l < a->layer_count && st == QXC_OK; ++l) {
    const qxc_layer_weights& w = a->layers[l];
    if (!w.input_norm) return fail(ctx, QXC_ERR_INVALID_ARG, "layer %d: null input_norm", l);
    st = check_q4(ctx, &w.q_proj, kHidden, kHidden, "q_proj");
    if (st == QXC_OK) st = check_q4(ctx, &w.k_proj, 512, kHidden, "k_proj");
    if (st == QXC_OK) st = check_q4(ctx, &w.v_proj, 512, kHidden, "v_proj");
    if (st == QXC_OK) st = check_q4(ctx, &w.o_proj, kHidden, kHidden, "o_proj");
  }
  if (st != QXC_OK) return st;
  // KvCache::append (qx-runtime lib.rs:385-398), checked before any launch
  if (a->position != kv->len[a->seq])
    return fail(ctx, QXC_ERR_POSITION, "KV position %d does not follow cache length %d", a->position,
                kv->len[a->seq]);
  if (a->position >= kv->desc.capacity)
    return fail(ctx, QXC_ERR_POSITION, "KV position %d exceeds context %d", a->position, kv->desc.capacity);
  if (a->split < 0 || a->split % 64 != 0)
    return fail(ctx, QXC_ERR_INVALID_ARG, "split %d must be 0 or a positive multiple of 64", a->split);
  QXC_CUDA(ctx, cudaSetDevice(ctx->device));
  if (!ctx->stack_x) {
    // zeroed: tag 0 is never a launch's tag (those start at 65)
    QXC_CUDA(ctx, cudaMalloc(&ctx->stack_x, kStackTagged * sizeof(uint2)));
    QXC_CUDA(ctx, cudaMemsetAsync(ctx->stack_x, 0, kStackTagged * sizeof(uint2), ctx->stream));
    QXC_CUDA(ctx, cudaMalloc(&ctx->stack_f, kStackFloats * sizeof(float)));
    QXC_CUDA(ctx, cudaMalloc(&ctx->stack_words, 16 * sizeof(unsigned)));
    QXC_CUDA(ctx, cudaMemsetAsync(ctx->stack_words, 0, 16 * sizeof(unsigned), ctx->stream));
  }
  const int attend = a->position + 1;
  const int chunk = stack_chunk(attend, ctx->sm_count, a->split);
  if (a->split && !chunk)
    return fail(ctx, QXC_ERR_INVALID_ARG, "split %d: at most %d splits of at most %d rows per kv head", a->split,
                std::min(kStackMaxSplits, ctx->sm_count / 8), kStackMaxTiles * kStackTileRows);
  if (!stack_fusable(ctx, kv, a, chunk)) {
    // one qxc_attention_layer per layer, the hidden state through the chain buffers
    float* chain = ctx->stack_f + kStackChain;
    for (int l = 0; l < a->layer_count; ++l) {
      const qxc_layer_weights& w = a->layers[l];
      qxc_layer_args la;
      memset(&la, 0, sizeof(la));
      la.seq = a->seq;
      la.layer = a->layer_begin + l;
      la.position = a->position;
      la.hidden_in = l == 0 ? a->hidden_in : chain + ((l - 1) & 1) * 1024;
      la.hidden_out = l == a->layer_count - 1 ? a->hidden_out : chain + (l & 1) * 1024;
      la.input_norm = w.input_norm;
      la.q_proj = w.q_proj;
      la.k_proj = w.k_proj;
      la.v_proj = w.v_proj;
      la.o_proj = w.o_proj;
      la.flags = (a->flags & ~QXC_DECODE_NO_ADVANCE) | QXC_DECODE_NO_ADVANCE;
      st = qxc_attention_layer(ctx, kv, &la);
      if (st != QXC_OK) return st;
    }
  } else {
    StackParams p;
    memset(&p, 0, sizeof(p));
    p.tmk = kv->tmk;
    p.tmv = kv->tmv;
    p.k_region = kv->k_region;
    p.v_region = kv->v_region;
    p.capacity = kv->desc.capacity;
    p.arena_layers = kv->desc.layers;
    p.seq = a->seq;
    p.position = a->position;
    p.chunk = chunk;
    p.nsplit = (attend + chunk - 1) / chunk;
    p.hx = ctx->stack_x + kStackHx;
    p.qx = ctx->stack_x + kStackQx;
    p.ax = ctx->stack_x + kStackAx;
    p.px = ctx->stack_x + kStackPx;
    p.abort = ctx->stack_words;
    p.tickets = ctx->stack_words + 1;
    p.pinned_exp = (a->flags & QXC_DECODE_NATIVE_EXP) ? 0 : 1;
    p.err = ctx->err_dev;
    float* chain = ctx->stack_f + kStackChain;
    // at most kStackMaxLayers layers per launch; longer stacks chain launches
    for (int l0 = 0, part = 0; l0 < a->layer_count; l0 += kStackMaxLayers, ++part) {
      const int n = std::min(kStackMaxLayers, a->layer_count - l0);
      p.layer_begin = a->layer_begin + l0;
      p.n_layers = n;
      p.hidden_in = l0 == 0 ? a->hidden_in : chain + ((part - 1) & 1) * 1024;
      p.hidden_out = l0 + n == a->layer_count ? a->hidden_out : chain + (part & 1) * 1024;
      for (int l = 0; l < n; ++l) {
        const qxc_layer_weights& w = a->layers[l0 + l];
        p.w[l].norm = w.input_norm;
        const qxc_q4_matrix* m[4] = {&w.q_proj, &w.k_proj, &w.v_proj, &w.o_proj};
        for (int j = 0; j < 4; ++j) {
          p.w[l].codes[j] = m[j]->codes;
          p.w[l].scales[j] = m[j]->scales;
        }
      }
      // the launch's tags: gen * 64 + layer + 1, never 0 (gen wraps at 2^26)
      ctx->stack_gen = (ctx->stack_gen + 1u) & 0x3ffffffu;
      if (ctx->stack_gen == 0u) ctx->stack_gen = 1u;
      p.gen = ctx->stack_gen;
      p.ticket_base = ctx->stack_tickets;
      st = launch_stack(ctx, p);
      if (st != QXC_OK) return st;
      ctx->stack_tickets += (unsigned)n * (unsigned)p.nsplit;  // (mod 2^32, as the kernel counts)
    }
    // the kernel writes row `position` of every layer and waits for nothing
    // after its end: later grids see complete rows
    note_rows_written(ctx, nullptr, -1, 0);
  }
  if (!(a->flags & QXC_DECODE_NO_ADVANCE)) kv->len[a->seq] += 1;
  return QXC_OK;
}

// ---- speculative verify ----------------------------------------------------
qxc_status qxc_decode_verify(qxc_ctx* ctx, qxc_kv* kv, const qxc_verify_args* a) {
  if (!ctx || !kv || !a) return fail(ctx, QXC_ERR_INVALID_ARG, "null argument");
  if (kv->ctx != ctx) return fail(ctx, QXC_ERR_INVALID_ARG, "KV arena belongs to another context");
  qxc_status st = check_seq(ctx, kv, a->seq);
  if (st != QXC_OK) return st;
  if (a->tokens < 1) return fail(ctx, QXC_ERR_INVALID_ARG, "batched attention requires at least one token");
  if (a->layer_count < 1 || a->layer_begin < 0 || a->layer_begin + a->layer_count > kv->desc.layers)
    return fail(ctx, QXC_ERR_INVALID_ARG, "layers [%d, %d) outside the arena's %d layers", a->layer_begin,
                a->layer_begin + a->layer_count, kv->desc.layers);
  if (!a->q || !a->k || !a->v || !a->out) return fail(ctx, QXC_ERR_INVALID_ARG, "null tensor pointer");
  if (!valid_dtype(a->q_dtype) || !valid_dtype(a->in_dtype) || !valid_dtype(a->out_dtype))
    return fail(ctx, QXC_ERR_INVALID_ARG, "unknown tensor dtype");
  if (kv->desc.model == QXC_MODEL_QWEN3 && (a->q_dtype != kv->desc.key_dtype || a->in_dtype != kv->desc.key_dtype))
    return fail(ctx, QXC_ERR_INVALID_ARG, "Qwen q/k/v must use the KV cache's 16-bit type");
  if (kv->desc.first_position != 0)
    return fail(ctx, QXC_ERR_INVALID_ARG, "a KV-length shard decodes through qxc_decode_partials");
  // KvCache::append for every candidate (qx-runtime lib.rs:385-398)
  if (a->start != kv->len[a->seq])
    return fail(ctx, QXC_ERR_POSITION, "KV position %d does not follow cache length %d", a->start, kv->len[a->seq]);
  if (a->start + a->tokens > kv->desc.capacity)
    return fail(ctx, QXC_ERR_POSITION, "KV position %d exceeds context %d", a->start + a->tokens - 1,
                kv->desc.capacity);
  QXC_CUDA(ctx, cudaSetDevice(ctx->device));
  {
    const int rows = a->start + a->tokens;
    st = ensure_pages(ctx, kv, 1, &a->seq, &rows);
    if (st != QXC_OK) return st;
  }
  // 1. the candidates' rows
  AppendParams ap;
  memset(&ap, 0, sizeof(ap));
  ap.k_region = kv->k_region;
  ap.v_region = kv->v_region;
  ap.capacity = kv->desc.capacity;
  ap.paging = kv_paging(kv);
  ap.layers = kv->desc.layers;
  ap.layer_begin = a->layer_begin;
  ap.layer_count = a->layer_count;
  ap.seq = a->seq;
  ap.start = a->start;
  ap.tokens = a->tokens;
  ap.k = a->k;
  ap.v = a->v;
  ap.k_norm = a->k_norm;
  ap.rope_table = kv->rope_table;
  ap.in_dtype = a->in_dtype;
  ap.err = ctx->err_dev;
  const int grid = a->tokens * a->layer_count;
  const int kd = kv->desc.key_dtype, vd = kv->desc.value_dtype;
  if (kv->desc.model == QXC_MODEL_QWEN3)
    st = kd == QXC_BF16 ? launch_append<Qwen3, __nv_bfloat16, __nv_bfloat16>(ctx, ap, grid)
                        : launch_append<Qwen3, __half, __half>(ctx, ap, grid);
  else if (kd == QXC_F32 && vd == QXC_F32) st = launch_append<Granite, float, float>(ctx, ap, grid);
  else if (kd == QXC_F32 && vd == QXC_F16) st = launch_append<Granite, float, __half>(ctx, ap, grid);
  else if (kd == QXC_F16 && vd == QXC_F32) st = launch_append<Granite, __half, float>(ctx, ap, grid);
  else if (kd == QXC_F16 && vd == QXC_F16) st = launch_append<Granite, __half, __half>(ctx, ap, grid);
  else st = launch_append<Granite, __nv_bfloat16, __nv_bfloat16>(ctx, ap, grid);
  if (st != QXC_OK) return st;
  note_rows_written(ctx, kv, a->seq, a->start);
  // 2. token t attends [0, start + t]
  if (kv->desc.model == QXC_MODEL_GRANITE && a->tokens >= 2 && a->tokens <= GraniteVerify4::NTOK &&
      !(a->flags & QXC_VERIFY_PER_TOKEN)) {
    st = launch_verify_shared(ctx, kv, a);
    if (st != QXC_OK) return st;
    if (!(a->flags & QXC_DECODE_NO_ADVANCE)) kv->len[a->seq] += a->tokens;
    return QXC_OK;
  }
  // one decode launch with one causal entry per token
  std::vector<int> ids(a->tokens, a->seq), attend(a->tokens), none(a->tokens, -1), rope(a->tokens);
  for (int t = 0; t < a->tokens; ++t) {
    attend[t] = a->start + t + 1;
    rope[t] = a->start + t;
  }
  CallPlan plan;
  st = plan_call(ctx, kv, a->tokens, ids.data(), attend.data(), none.data(), rope.data(), a->layer_count, a->split,
                 &plan);
  if (st != QXC_OK) return st;
  DecodeParams p;
  st = fill_params(ctx, kv, plan, a->layer_begin, a->layer_count, &p);
  if (st != QXC_OK) return st;
  p.q = a->q;
  p.k = a->k;
  p.v = a->v;
  p.out = a->out;
  p.q_norm = a->q_norm;
  p.k_norm = a->k_norm;
  p.q_dtype = a->q_dtype;
  p.in_dtype = a->in_dtype;
  p.out_dtype = a->out_dtype;
  p.pinned_exp = default_pinned(kv, a->flags) ? 1 : 0;
  st = launch_decode(ctx, kv, p, plan.items);
  if (st != QXC_OK) return st;
  if (!(a->flags & QXC_DECODE_NO_ADVANCE)) kv->len[a->seq] += a->tokens;
  return QXC_OK;
}

static qxc_status stage_reserve(qxc_ctx* ctx, size_t bytes) {
  if (bytes > ctx->stage_cap) {
    QXC_CUDA(ctx, cudaStreamSynchronize(ctx->stream));
    cudaFree(ctx->stage_dev);
    ctx->stage_dev = nullptr;
    ctx->stage_cap = 0;
    QXC_CUDA(ctx, cudaMalloc(&ctx->stage_dev, bytes));
    ctx->stage_cap = bytes;
  }
  return QXC_OK;
}

qxc_status qxc_decode_host(qxc_ctx* ctx, qxc_kv* kv, const qxc_decode_args* a) {
  if (!ctx || !kv || !a) return fail(ctx, QXC_ERR_INVALID_ARG, "null argument");
  if (!a->q || !a->k || !a->v || !a->out) return fail(ctx, QXC_ERR_INVALID_ARG, "null tensor pointer");
  const size_t units = (size_t)std::max(a->seq_count, 0) * std::max(a->layer_count, 0);
  const size_t qb = units * kv->hq * kv->d * dtype_size(a->q_dtype);
  const size_t kb = units * kv->hkv * kv->d * dtype_size(a->in_dtype);
  const size_t ob = units * kv->hq * kv->d * dtype_size(a->out_dtype);
  const size_t rb = a->q_rot_out ? units * kv->hq * kv->d * 4 : 0;
  auto al = [](size_t x) { return ((x + 255) / 256) * 256; };
  const size_t off_k = al(qb), off_v = off_k + al(kb), off_o = off_v + al(kb), off_r = off_o + al(ob);
  const size_t total = off_r + al(rb);
  // Pinned host buffers that the device can address (cudaHostAlloc, which
  // maps them under unified addressing, or cudaHostRegister with the mapped
  // flag; torch's pin_memory is the former): the kernels read q/k/v over
  // PCIe in their prologue, while the KV stream starts, and write the
  // outputs straight back, so no copy is queued before or after them.
  {
    auto mapped = [](const void* h, void** d) {
      cudaPointerAttributes at;
      if (cudaPointerGetAttributes(&at, h) != cudaSuccess) {
        cudaGetLastError();
        return false;
      }
      if (at.type != cudaMemoryTypeHost || !at.devicePointer) return false;
      *d = at.devicePointer;
      return true;
    };
    void *dq, *dk, *dv, *dout, *drot = nullptr;
    QXC_CUDA(ctx, cudaSetDevice(ctx->device));
    if (mapped(a->q, &dq) && mapped(a->k, &dk) && mapped(a->v, &dv) && mapped(a->out, &dout) &&
        (!a->q_rot_out || mapped(a->q_rot_out, &drot))) {
      qxc_decode_args d = *a;
      d.q = dq;
      d.k = dk;
      d.v = dv;
      d.out = dout;
      d.q_rot_out = static_cast<float*>(drot);
      qxc_status st = qxc_decode(ctx, kv, &d);
      if (st != QXC_OK) return st;
      return qxc_sync(ctx);
    }
  }
  qxc_status st = stage_reserve(ctx, total);
  if (st != QXC_OK) return st;
  // Other host memory: copies from the caller's buffers (pinned memory goes
  // by DMA with no host-side copy; pageable memory is staged by the driver;
  // either way the copy completes in stream order).
  QXC_CUDA(ctx, cudaMemcpyAsync(ctx->stage_dev, a->q, qb, cudaMemcpyHostToDevice, ctx->stream));
  QXC_CUDA(ctx, cudaMemcpyAsync(ctx->stage_dev + off_k, a->k, kb, cudaMemcpyHostToDevice, ctx->stream));
  QXC_CUDA(ctx, cudaMemcpyAsync(ctx->stage_dev + off_v, a->v, kb, cudaMemcpyHostToDevice, ctx->stream));
  qxc_decode_args d = *a;
  d.q = ctx->stage_dev;
  d.k = ctx->stage_dev + off_k;
  d.v = ctx->stage_dev + off_v;
  d.out = ctx->stage_dev + off_o;
  d.q_rot_out = a->q_rot_out ? reinterpret_cast<float*>(ctx->stage_dev + off_r) : nullptr;
  st = qxc_decode(ctx, kv, &d);
  if (st != QXC_OK) return st;
  QXC_CUDA(ctx, cudaMemcpyAsync(a->out, ctx->stage_dev + off_o, ob, cudaMemcpyDeviceToHost, ctx->stream));
  if (a->q_rot_out)
    QXC_CUDA(ctx, cudaMemcpyAsync(a->q_rot_out, ctx->stage_dev + off_r, rb, cudaMemcpyDeviceToHost, ctx->stream));
  return qxc_sync(ctx);
}

qxc_status qxc_granite_attention_decode(qxc_ctx* ctx, qxc_kv* kv, const float* q, const float* k, const float* v,
                                        int32_t position, float* out) {
  if (!kv) return fail(ctx, QXC_ERR_INVALID_ARG, "null KV cache");
  if (kv->desc.model != QXC_MODEL_GRANITE) return fail(ctx, QXC_ERR_INVALID_ARG, "not a Granite KV arena");
  qxc_decode_args a;
  memset(&a, 0, sizeof(a));
  const int32_t pos = position;
  a.layer_begin = 0;
  a.layer_count = 1;
  a.seq_count = 1;
  a.positions = &pos;
  a.q = q;
  a.k = k;
  a.v = v;
  a.out = out;
  a.q_dtype = a.in_dtype = a.out_dtype = QXC_F32;
  return qxc_decode_host(ctx, kv, &a);
}

qxc_status qxc_apply_granite_rope(qxc_ctx* ctx, float* q, float* k, int32_t position) {
  if (!ctx || !q || !k) return fail(ctx, QXC_ERR_INVALID_ARG, "null argument");
  if (position < 0) return fail(ctx, QXC_ERR_INVALID_ARG, "negative position");
  qxc_status st = stage_reserve(ctx, 1536 * sizeof(float));
  if (st != QXC_OK) return st;
  float* dq = reinterpret_cast<float*>(ctx->stage_dev);
  QXC_CUDA(ctx, cudaMemcpyAsync(dq, q, 1024 * sizeof(float), cudaMemcpyHostToDevice, ctx->stream));
  QXC_CUDA(ctx, cudaMemcpyAsync(dq + 1024, k, 512 * sizeof(float), cudaMemcpyHostToDevice, ctx->stream));
  qx_granite_rope_kernel<<<6, 128, 0, ctx->stream>>>(dq, dq + 1024, position, ctx->err_dev);
  QXC_CUDA(ctx, cudaGetLastError());
  ctx->launches++;
  QXC_CUDA(ctx, cudaMemcpyAsync(q, dq, 1024 * sizeof(float), cudaMemcpyDeviceToHost, ctx->stream));
  QXC_CUDA(ctx, cudaMemcpyAsync(k, dq + 1024, 512 * sizeof(float), cudaMemcpyDeviceToHost, ctx->stream));
  return qxc_sync(ctx);
}

// ---- KV-length split ---------------------------------------------------------
// qxc_decode_partials, and with a peer group the fused exchange: every
// split partial, even a lone one, goes through the split merge kernel, which
// pushes this rank's merged partials to every rank and merges all ranks'
// into xout. So the path does not depend on a rank's split count, and every
// rank takes it.
static qxc_status decode_partials_impl(qxc_ctx* ctx, qxc_kv* kv, const qxc_partial_args* a, qxc_peer_group* g,
                                       void* xout, int xout_dtype) {
  if (!ctx || !kv || !a) return fail(ctx, QXC_ERR_INVALID_ARG, "null argument");
  if (kv->ctx != ctx) return fail(ctx, QXC_ERR_INVALID_ARG, "KV arena belongs to another context");
  qxc_status st = check_seq(ctx, kv, a->seq);
  if (st != QXC_OK) return st;
  if (a->layer < 0 || a->layer >= kv->desc.layers) return fail(ctx, QXC_ERR_INVALID_ARG, "layer %d out of range", a->layer);
  if (!a->q || (!a->partials && !g) || (a->append && (!a->k || !a->v)))
    return fail(ctx, QXC_ERR_INVALID_ARG, "null tensor pointer");
  if (kv->desc.model == QXC_MODEL_QWEN3 && (a->q_dtype != kv->desc.key_dtype || (a->append && a->in_dtype != kv->desc.key_dtype)))
    return fail(ctx, QXC_ERR_INVALID_ARG, "Qwen q/k/v must use the KV cache's 16-bit type");
  const int first = kv->desc.first_position;
  const int len = kv->len[a->seq];
  int attend, new_slot;
  if (a->append) {
    const int local = a->position - first;
    if (local != len)
      return fail(ctx, QXC_ERR_POSITION, "KV position %d does not follow cache length %d", a->position, first + len);
    if (local >= kv->desc.capacity)
      return fail(ctx, QXC_ERR_POSITION, "KV position %d exceeds context %d", a->position, first + kv->desc.capacity);
    attend = local + 1;
    new_slot = local;
  } else {
    if (len < 1) return fail(ctx, QXC_ERR_INVALID_ARG, "a shard without the new token needs cached rows");
    if (a->position < first + len)
      return fail(ctx, QXC_ERR_POSITION, "position %d precedes this shard's slots", a->position);
    attend = len;
    new_slot = -1;
  }
  if (kv->desc.model == QXC_MODEL_GRANITE && a->position >= 4096)
    return fail(ctx, QXC_ERR_POSITION, "KV position %d exceeds context 4096", a->position);
  if (kv->desc.model == QXC_MODEL_QWEN3 && a->position >= kQwenMaxPositions)
    return fail(ctx, QXC_ERR_POSITION, "KV position %d exceeds context %d", a->position, kQwenMaxPositions);
  QXC_CUDA(ctx, cudaSetDevice(ctx->device));
  CallPlan plan;
  const int seq = a->seq, rope = a->position;
  st = ensure_pages(ctx, kv, 1, &seq, &attend);
  if (st != QXC_OK) return st;
  // With a peer group a one-wave Qwen grid merges and exchanges inside the
  // decode grid, one NVLink round trip per 32-dim output slice a split
  // takes (exchange_slice). The automatic split then gives every kv head at
  // least one split per slice (32: 8 query heads x 4 slices) while the grid
  // stays one wave: with fewer, some splits take two slices one after the
  // other and the step pays the round trip twice (config 3 at N = 4: 22
  // splits of 384 rows, 21.4 us per step).
  int split = a->split;
  if (g && split == 0 && kv->desc.model == QXC_MODEL_QWEN3) {
    const int unit = split_unit(kv), slices = kv->hq / kv->hkv * (kv->d / 32);
    const int chunk = std::max(unit, attend / slices / unit * unit);
    const int nsplit = (attend + chunk - 1) / chunk;
    if (nsplit >= slices && nsplit <= 4 * kMergeLoads && nsplit * kv->hkv <= decode_blocks_per_sm(kv) * ctx->sm_count)
      split = chunk;
  }
  st = plan_call(ctx, kv, 1, &seq, &attend, &new_slot, &rope, 1, split, &plan);
  if (st != QXC_OK) return st;
  DecodeParams p;
  st = fill_params(ctx, kv, plan, a->layer, 1, &p);
  if (st != QXC_OK) return st;
  p.q = a->q;
  p.k = a->k ? a->k : a->q;
  p.v = a->v ? a->v : a->q;
  p.out = a->partials;
  p.q_norm = a->q_norm;
  p.k_norm = a->k_norm;
  p.q_dtype = a->q_dtype;
  p.in_dtype = a->in_dtype;
  p.out_dtype = QXC_F32;
  p.pinned_exp = default_pinned(kv, a->flags) ? 1 : 0;
  p.emit_partials = 1;
  if (g) {
    p.external_merge = 1;
    for (int r = 0; r < g->world; ++r) p.xinbox[r] = reinterpret_cast<uint2*>(g->peer[r] + g->off_xinbox);
    p.xstep = reinterpret_cast<unsigned*>(g->base + g->off_step) + kExchHeads;
    p.xfailed = g->failed_dev();
    p.xfailed_host = g->failed_mapped;
    p.xrank = g->rank;
    p.xworld = g->world;
    p.xout = xout;
    p.xout_dtype = xout_dtype;
    // a one-wave Qwen grid merges its splits and exchanges the result with
    // the peers itself (exchange_slice), with no merge grid
    st = use_slice_merge(ctx, kv, plan, &p);
    if (st != QXC_OK) return st;
  }
  st = launch_decode(ctx, kv, p, plan.items);
  if (st != QXC_OK) return st;
  if (a->append) kv->len[a->seq] += 1;
  return QXC_OK;
}

qxc_status qxc_decode_partials(qxc_ctx* ctx, qxc_kv* kv, const qxc_partial_args* a) {
  return decode_partials_impl(ctx, kv, a, nullptr, nullptr, 0);
}

qxc_status qxc_lse_merge(qxc_ctx* ctx, int32_t model, int32_t n_parts, const float* partials, void* out,
                         int32_t out_dtype) {
  if (!ctx || !partials || !out || n_parts < 1) return fail(ctx, QXC_ERR_INVALID_ARG, "invalid merge arguments");
  if (!valid_dtype(out_dtype)) return fail(ctx, QXC_ERR_INVALID_ARG, "unknown dtype");
  QXC_CUDA(ctx, cudaSetDevice(ctx->device));
  const int pinned = model == QXC_MODEL_GRANITE ? 1 : 0;
  if (model == QXC_MODEL_QWEN3)
    qx_lse_merge_kernel<32, 128><<<32, 128, 0, ctx->stream>>>(partials, n_parts, out, out_dtype, pinned, ctx->err_dev);
  else if (model == QXC_MODEL_GRANITE)
    qx_lse_merge_kernel<16, 64><<<16, 64, 0, ctx->stream>>>(partials, n_parts, out, out_dtype, pinned, ctx->err_dev);
  else
    return fail(ctx, QXC_ERR_INVALID_ARG, "unknown model %d", model);
  QXC_CUDA(ctx, cudaGetLastError());
  ctx->launches++;
  return QXC_OK;
}

// ---- exchange over NVLink (KV-length split across GPUs) --------------------------

static qxc_status peer_group_failed_error(qxc_ctx* ctx) {
  return fail(ctx, QXC_ERR_TIMEOUT,
              "peer group failed: an earlier exchange on it timed out (destroy and re-create the groups on every "
              "rank)");
}

qxc_status qxc_peer_group_create(qxc_ctx* ctx, int32_t rank, int32_t world, qxc_peer_group** out) {
  if (!ctx || !out) return fail(ctx, QXC_ERR_INVALID_ARG, "null argument");
  *out = nullptr;
  if (world < 1 || world > kMaxPeers || rank < 0 || rank >= world)
    return fail(ctx, QXC_ERR_INVALID_ARG, "rank %d of world %d (at most %d ranks)", rank, world, kMaxPeers);
  QXC_CUDA(ctx, cudaSetDevice(ctx->device));
  qxc_peer_group* g = new (std::nothrow) qxc_peer_group();
  if (!g) return fail(ctx, QXC_ERR_OUT_OF_MEMORY, "host allocation failed");
  g->ctx = ctx;
  g->rank = rank;
  g->world = world;
  const size_t inbox = (size_t)2 * world * kExchHeads * kExchRow * sizeof(uint2);
  const size_t xinbox = (size_t)2 * world * kExchHeads * 4 * 34 * sizeof(uint2);
  g->off_xinbox = (inbox + 255) / 256 * 256;
  g->off_step = g->off_xinbox + (xinbox + 255) / 256 * 256;
  // [32] exchange-kernel steps, then [32][4] split-merge steps, then (at
  // byte 768) the group-failed word
  g->bytes = g->off_step + 1024;
  const size_t bytes = g->bytes;
  cudaError_t e = cudaHostAlloc(reinterpret_cast<void**>(&g->failed_host), sizeof(unsigned), cudaHostAllocMapped);
  if (e != cudaSuccess) {
    delete g;
    return fail(ctx, QXC_ERR_OUT_OF_MEMORY, "pinned group word: %s", cudaGetErrorString(e));
  }
  *g->failed_host = 0u;
  e = cudaHostGetDevicePointer(reinterpret_cast<void**>(&g->failed_mapped), g->failed_host, 0);
  if (e == cudaSuccess) e = cudaMalloc(&g->base, bytes);
  if (e != cudaSuccess) {
    cudaFreeHost(g->failed_host);
    delete g;
    return fail(ctx, QXC_ERR_OUT_OF_MEMORY, "exchange area of %zu bytes: %s", bytes, cudaGetErrorString(e));
  }
  e = cudaMemset(g->base, 0, g->bytes);
  if (e != cudaSuccess) {
    cudaFree(g->base);
    cudaFreeHost(g->failed_host);
    delete g;
    return fail(ctx, QXC_ERR_CUDA, "cudaMemset: %s", cudaGetErrorString(e));
  }
  g->peer[rank] = g->base;
  *out = g;
  return QXC_OK;
}

void qxc_peer_group_destroy(qxc_peer_group* g) {
  if (!g) return;
  cudaSetDevice(g->ctx->device);
  cudaStreamSynchronize(g->ctx->stream);
  for (int r = 0; r < g->world; ++r)
    if (g->opened[r]) cudaIpcCloseMemHandle(g->peer[r]);
  cudaFree(g->base);
  cudaFreeHost(g->failed_host);
  delete g;
}

qxc_status qxc_peer_group_handle(const qxc_peer_group* g, void* handle) {
  if (!g || !handle) return QXC_ERR_INVALID_ARG;
  qxc_ctx* ctx = g->ctx;
  QXC_CUDA(ctx, cudaSetDevice(ctx->device));
  cudaIpcMemHandle_t h;
  QXC_CUDA(ctx, cudaIpcGetMemHandle(&h, g->base));
  static_assert(sizeof(cudaIpcMemHandle_t) == QXC_PEER_HANDLE_BYTES, "IPC handle size");
  memcpy(handle, &h, sizeof(h));
  return QXC_OK;
}

qxc_status qxc_peer_group_base(const qxc_peer_group* g, void** base) {
  if (!g || !base) return QXC_ERR_INVALID_ARG;
  *base = g->base;
  return QXC_OK;
}

qxc_status qxc_peer_group_open(qxc_peer_group* g, int32_t peer, const void* handle) {
  if (!g || !handle) return QXC_ERR_INVALID_ARG;
  qxc_ctx* ctx = g->ctx;
  if (peer < 0 || peer >= g->world || peer == g->rank)
    return fail(ctx, QXC_ERR_INVALID_ARG, "peer %d is not another rank of world %d", peer, g->world);
  if (g->peer[peer]) return fail(ctx, QXC_ERR_INVALID_ARG, "peer %d is already attached", peer);
  QXC_CUDA(ctx, cudaSetDevice(ctx->device));
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  QXC_CUDA(ctx, cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  g->peer[peer] = static_cast<char*>(p);
  g->opened[peer] = true;
  return QXC_OK;
}

qxc_status qxc_peer_group_set_peer(qxc_peer_group* g, int32_t peer, void* base) {
  if (!g || !base) return QXC_ERR_INVALID_ARG;
  qxc_ctx* ctx = g->ctx;
  if (peer < 0 || peer >= g->world || peer == g->rank)
    return fail(ctx, QXC_ERR_INVALID_ARG, "peer %d is not another rank of world %d", peer, g->world);
  if (g->peer[peer]) return fail(ctx, QXC_ERR_INVALID_ARG, "peer %d is already attached", peer);
  QXC_CUDA(ctx, cudaSetDevice(ctx->device));
  cudaPointerAttributes attr;
  QXC_CUDA(ctx, cudaPointerGetAttributes(&attr, base));
  if (attr.type != cudaMemoryTypeDevice) return fail(ctx, QXC_ERR_INVALID_ARG, "peer base is not device memory");
  if (attr.device != ctx->device) {
    int ok = 0;
    QXC_CUDA(ctx, cudaDeviceCanAccessPeer(&ok, ctx->device, attr.device));
    if (!ok) return fail(ctx, QXC_ERR_UNSUPPORTED, "device %d cannot access device %d", ctx->device, attr.device);
    cudaError_t e = cudaDeviceEnablePeerAccess(attr.device, 0);
    if (e == cudaErrorPeerAccessAlreadyEnabled) cudaGetLastError();
    else if (e != cudaSuccess) return fail(ctx, QXC_ERR_CUDA, "cudaDeviceEnablePeerAccess: %s", cudaGetErrorString(e));
  }
  g->peer[peer] = static_cast<char*>(base);
  return QXC_OK;
}

qxc_status qxc_exchange_merge(qxc_ctx* ctx, qxc_peer_group* g, int32_t model, const float* partials, void* out,
                              int32_t out_dtype) {
  if (!ctx || !g || !partials || !out) return fail(ctx, QXC_ERR_INVALID_ARG, "null argument");
  if (g->ctx != ctx) return fail(ctx, QXC_ERR_INVALID_ARG, "peer group belongs to another context");
  if (!valid_dtype(out_dtype)) return fail(ctx, QXC_ERR_INVALID_ARG, "unknown dtype");
  if (model != QXC_MODEL_QWEN3 && model != QXC_MODEL_GRANITE)
    return fail(ctx, QXC_ERR_INVALID_ARG, "unknown model %d", model);
  if (g->failed()) return peer_group_failed_error(ctx);
  ExchangeParams p;
  memset(&p, 0, sizeof(p));
  for (int r = 0; r < g->world; ++r) {
    if (!g->peer[r]) return fail(ctx, QXC_ERR_INVALID_ARG, "peer %d is not attached", r);
    p.inbox[r] = reinterpret_cast<uint2*>(g->peer[r]);
  }
  p.step = reinterpret_cast<unsigned*>(g->base + g->off_step);
  p.failed = g->failed_dev();
  p.failed_host = g->failed_mapped;
  p.rank = g->rank;
  p.world = g->world;
  p.hq = model == QXC_MODEL_QWEN3 ? 32 : 16;
  p.d = model == QXC_MODEL_QWEN3 ? 128 : 64;
  p.partials = partials;
  p.out = out;
  p.out_dtype = out_dtype;
  p.pinned = model == QXC_MODEL_GRANITE ? 1 : 0;
  p.err = ctx->err_dev;
  QXC_CUDA(ctx, cudaSetDevice(ctx->device));
  TraceRun tr(ctx, "exchange", (size_t)p.hq);
  p.trace = tr.buf;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.hq);
  cfg.blockDim = dim3(kExchThreads);
  cfg.stream = ctx->stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  QXC_CUDA(ctx, cudaLaunchKernelEx(&cfg, qx_exchange_merge_kernel, p));
  ctx->launches++;
  return QXC_OK;
}

qxc_status qxc_decode_exchange(qxc_ctx* ctx, qxc_kv* kv, const qxc_partial_args* a, qxc_peer_group* g, void* out,
                               int32_t out_dtype) {
  if (!ctx || !kv || !a || !g || !out) return fail(ctx, QXC_ERR_INVALID_ARG, "null argument");
  if (g->ctx != ctx) return fail(ctx, QXC_ERR_INVALID_ARG, "peer group belongs to another context");
  if (!valid_dtype(out_dtype)) return fail(ctx, QXC_ERR_INVALID_ARG, "unknown dtype");
  for (int r = 0; r < g->world; ++r)
    if (!g->peer[r]) return fail(ctx, QXC_ERR_INVALID_ARG, "peer %d is not attached", r);
  if (g->failed()) return peer_group_failed_error(ctx);
  if ((kv->desc.model == QXC_MODEL_QWEN3 ? 32 : 16) * (kv->d / 32) > ctx->sm_count * 8)
    return fail(ctx, QXC_ERR_UNSUPPORTED, "the merge grid must fit one wave");
  return decode_partials_impl(ctx, kv, a, g, out, out_dtype);
}

// ---- prefill -------------------------------------------------------------------
qxc_status qxc_prefill(qxc_ctx* ctx, qxc_kv* kv, const qxc_prefill_args* a) {
  if (!ctx || !kv || !a) return fail(ctx, QXC_ERR_INVALID_ARG, "null argument");
  if (kv->ctx != ctx) return fail(ctx, QXC_ERR_INVALID_ARG, "KV arena belongs to another context");
  if (kv->desc.model != QXC_MODEL_GRANITE) return fail(ctx, QXC_ERR_UNSUPPORTED, "prefill supports Granite only");
  if (kv->paged()) return fail(ctx, QXC_ERR_UNSUPPORTED, "prefill needs a contiguous arena");
  if (kv->desc.key_dtype != QXC_BF16 || kv->desc.value_dtype != QXC_BF16)
    return fail(ctx, QXC_ERR_UNSUPPORTED, "prefill requires a bf16 KV arena");
  if (a->in_dtype != QXC_BF16) return fail(ctx, QXC_ERR_UNSUPPORTED, "prefill inputs must be bf16");
  if (a->out_dtype != QXC_F32 && a->out_dtype != QXC_BF16)
    return fail(ctx, QXC_ERR_INVALID_ARG, "prefill output must be f32 or bf16");
  qxc_status st = check_seq(ctx, kv, a->seq);
  if (st != QXC_OK) return st;
  if (a->layer < 0 || a->layer >= kv->desc.layers) return fail(ctx, QXC_ERR_INVALID_ARG, "layer %d out of range", a->layer);
  if (!a->q || !a->k || !a->v || !a->out) return fail(ctx, QXC_ERR_INVALID_ARG, "null tensor pointer");
  // the prefill kernels move q/k/v rows and output rows with 16-byte accesses
  if (((uintptr_t)a->q | (uintptr_t)a->k | (uintptr_t)a->v | (uintptr_t)a->out) & 15u)
    return fail(ctx, QXC_ERR_INVALID_ARG, "prefill tensors must be 16-byte aligned");
  if (kv->len[a->seq] != 0)
    return fail(ctx, QXC_ERR_POSITION, "KV position 0 does not follow cache length %d", kv->len[a->seq]);
  if (a->length < 1 || a->length > kv->desc.capacity)
    return fail(ctx, QXC_ERR_POSITION, "KV position %d exceeds context %d", a->length - 1, kv->desc.capacity);
  if (kv->desc.first_position != 0) return fail(ctx, QXC_ERR_INVALID_ARG, "prefill needs an unsharded arena");
  QXC_CUDA(ctx, cudaSetDevice(ctx->device));
  void *kc, *vc;
  kv_view(kv, a->seq, a->layer, true, &kc, nullptr);
  kv_view(kv, a->seq, a->layer, false, &vc, nullptr);
  // rotated-query scratch, L x 16 x 64 bf16
  st = grow(ctx, &ctx->prefill_q, &ctx->prefill_q_cap, (size_t)a->length * 1024, false);
  if (st != QXC_OK) return st;
  st = ensure_granite_rope(ctx);
  if (st != QXC_OK) return st;
  PrefillParams p;
  memset(&p, 0, sizeof(p));
  p.rope = ctx->granite_rope;
  st = encode_tile_map(ctx, &p.tmq, ctx->prefill_q, QXC_BF16, 16, 64, a->length, 64);
  if (st == QXC_OK) st = encode_tile_map(ctx, &p.tmk, kc, QXC_BF16, 8, 64, a->length, 64);
  if (st == QXC_OK) st = encode_tile_map(ctx, &p.tmv, vc, QXC_BF16, 8, 64, a->length, 64);
  if (st != QXC_OK) return st;
  p.q = static_cast<const __nv_bfloat16*>(a->q);
  p.k = static_cast<const __nv_bfloat16*>(a->k);
  p.v = static_cast<const __nv_bfloat16*>(a->v);
  p.q_rot = reinterpret_cast<__nv_bfloat16*>(ctx->prefill_q);
  p.k_cache = static_cast<__nv_bfloat16*>(kc);
  p.v_cache = static_cast<__nv_bfloat16*>(vc);
  p.out = a->out;
  p.out_dtype = a->out_dtype;
  p.length = a->length;
  p.err = ctx->err_dev;
  const int nqb = (a->length + 63) / 64;
  p.nqb = nqb;
  static unsigned long long configured = 0;
  const unsigned long long bit = 1ull << (ctx->device & 63);
  if (!(configured & bit)) {
    QXC_CUDA(ctx, cudaFuncSetAttribute(qx_prefill_attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       PrefillCfg::SMEM));
    configured |= bit;
  }
  const int rope_grid = (a->length + kRopePositions - 1) / kRopePositions;
  {
    static int rope_slots[64] = {};  // resident RoPE CTAs per SM, by device
    int& per_sm = rope_slots[ctx->device & 63];
    if (!per_sm && (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, qx_prefill_rope_kernel, 256, 0) !=
                        cudaSuccess || per_sm < 1))
      per_sm = 1;
    p.early_trigger = rope_grid <= per_sm * ctx->sm_count ? 1 : 0;
  }
  // Query block qb attends qb + 1 key tiles. When one CTA per (block, kv
  // head) leaves a second wave of at least half the SMs but pairs of blocks
  // fit in one wave, CTA j takes blocks nqb-1-j/8 and j/8 (nqb + 1 tiles
  // each). A smaller second wave costs less than a pair's item boundary
  // (L = 1216, 19 blocks: 18.0 us unpaired against 20.5 us paired; L = 2048,
  // 32 blocks: 28.0 against 27.5).
  const int paired_grid = (nqb + 1) / 2 * 8;
  p.paired = (2 * nqb * 8 >= 3 * ctx->sm_count && paired_grid <= ctx->sm_count) ? 1 : 0;
  const int attn_grid = p.paired ? paired_grid : nqb * 8;
  TraceRun tr(ctx, "prefill", (size_t)nqb * 8 * 3);  // softmax timeline, then the two MMA issuers'
  p.trace = tr.buf;
  qx_prefill_rope_kernel<<<rope_grid, 256, 0, ctx->stream>>>(p);
  QXC_CUDA(ctx, cudaGetLastError());
  note_rows_written(ctx, kv, a->seq, 0);
  // the attention grid is a programmatic dependent of the RoPE grid: its CTAs
  // initialise barriers and TMEM while the RoPE grid drains, and wait for it
  // (griddepcontrol.wait) before the first TMA load
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(attn_grid);
  cfg.blockDim = dim3(PrefillCfg::NT);
  cfg.dynamicSmemBytes = PrefillCfg::SMEM;
  cfg.stream = ctx->stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  QXC_CUDA(ctx, cudaLaunchKernelEx(&cfg, qx_prefill_attn_tc_kernel, p));
  ctx->launches += 2;
  if (!(a->flags & QXC_DECODE_NO_ADVANCE)) kv->len[a->seq] = a->length;
  return QXC_OK;
}

// ---- commitments -----------------------------------------------------------------
qxc_status qxc_verification_hashes(qxc_ctx* ctx, qxc_kv* kv, const qxc_verification_hash_args* a) {
  if (!ctx || !kv || !a) return fail(ctx, QXC_ERR_INVALID_ARG, "null argument");
  if (kv->ctx != ctx) return fail(ctx, QXC_ERR_INVALID_ARG, "KV arena belongs to another context");
  qxc_status st = check_seq(ctx, kv, a->seq);
  if (st != QXC_OK) return st;
  if (!a->residuals || !a->digests) return fail(ctx, QXC_ERR_INVALID_ARG, "null tensor pointer");
  const int layers = kv->desc.layers;
  // the reference's own limits (qx-metal lib.rs:9262-9302)
  if (a->checkpoint_interval < 1 || a->checkpoint_interval > layers)
    return fail(ctx, QXC_ERR_INVALID_ARG, "verification checkpoint interval %d is outside 1..=%d",
                a->checkpoint_interval, layers);
  const long long chunks = a->residual_stride / 256;
  if (a->residual_stride <= 0 || a->residual_stride % 256 != 0 || chunks > 16 || (chunks & (chunks - 1)) != 0)
    return fail(ctx, QXC_ERR_INVALID_ARG, "verification residual size %lld is not 1..16 (a power of two) chunks of 256",
                (long long)a->residual_stride);
  if ((uintptr_t)a->residuals & 15u) return fail(ctx, QXC_ERR_INVALID_ARG, "residual snapshots must be 16-byte aligned");
  if (a->token < 0 || a->token >= kv->len[a->seq])
    return fail(ctx, QXC_ERR_POSITION, "token %d is not below cache length %d", a->token, kv->len[a->seq]);
  HashParams p;
  st = hash_params(ctx, kv, a->seq, &p);
  if (st != QXC_OK) return st;
  p.mode = kHashModeVerify;
  p.token = a->token;
  p.residuals = static_cast<const char*>(a->residuals);
  p.residual_stride = a->residual_stride;
  p.checkpoint_interval = a->checkpoint_interval;
  p.out = a->digests;
  QXC_CUDA(ctx, cudaSetDevice(ctx->device));
  return launch_hash(ctx, p, (layers + 1 + kHashWarps - 1) / kHashWarps);
}

qxc_status qxc_kv_slot_hashes(qxc_ctx* ctx, qxc_kv* kv, int32_t seq, int32_t layer_begin, int32_t layer_count,
                              int32_t token_begin, int32_t token_count, uint8_t* digests, int32_t flags) {
  if (!ctx || !kv) return fail(ctx, QXC_ERR_INVALID_ARG, "null argument");
  if (kv->ctx != ctx) return fail(ctx, QXC_ERR_INVALID_ARG, "KV arena belongs to another context");
  qxc_status st = check_seq(ctx, kv, seq);
  if (st != QXC_OK) return st;
  if (!digests) return fail(ctx, QXC_ERR_INVALID_ARG, "null tensor pointer");
  if (layer_count < 1 || layer_begin < 0 || layer_begin + layer_count > kv->desc.layers)
    return fail(ctx, QXC_ERR_INVALID_ARG, "layers [%d, %d) outside the arena's %d layers", layer_begin,
                layer_begin + layer_count, kv->desc.layers);
  if (token_count < 1 || token_begin < 0 || token_begin + token_count > kv->len[seq])
    return fail(ctx, QXC_ERR_POSITION, "tokens [%d, %d) are not below cache length %d", token_begin,
                token_begin + token_count, kv->len[seq]);
  HashParams p;
  st = hash_params(ctx, kv, seq, &p);
  if (st != QXC_OK) return st;
  p.mode = kHashModeSlots;
  p.layer_begin = layer_begin;
  p.layer_count = layer_count;
  p.token_begin = token_begin;
  p.token_count = token_count;
  const int chunks = std::max(p.key_row_bytes, p.value_row_bytes) / 256;
  p.seg = chunks;  // a power of two <= 8
  p.out = digests;
  const long long slots = (long long)layer_count * token_count;
  if (slots > (1ll << 31) - 1) return fail(ctx, QXC_ERR_INVALID_ARG, "too many slots");
  if (flags < QXC_HASH_AUTO || flags > QXC_HASH_PER_SLOT) return fail(ctx, QXC_ERR_INVALID_ARG, "unknown hash flags");
  QXC_CUDA(ctx, cudaSetDevice(ctx->device));
  // a lane pair per slot once the range gives every SM at least 8 full warps
  bool serial = flags == QXC_HASH_PER_SLOT;
  if (flags == QXC_HASH_AUTO) serial = slots >= 16ll * 8 * ctx->sm_count;
  if (!serial) {
    const long long per_cta = 32 / (2 * p.seg) * kHashWarps;
    return launch_hash(ctx, p, (int)((slots + per_cta - 1) / per_cta));
  }
  static unsigned long long configured = 0;
  const unsigned long long bit = 1ull << (ctx->device & 63);
  if (!(configured & bit)) {
    QXC_CUDA(ctx, cudaFuncSetAttribute(qx_kv_hash_serial_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       kHashSerialSmem));
    configured |= bit;
  }
  const long long per_cta = 16ll * kHashSerialWarps;  // a lane pair per slot
  return launch_hash(ctx, p, (int)((slots + per_cta - 1) / per_cta), qx_kv_hash_serial_kernel, kHashSerialSmem,
                     kHashSerialWarps);
}

// One thread per input: the pinned exp, rsqrt and Granite RoPE (sin, cos)
// of the input as raw bits, the RoPE position being the input truncated to
// an unsigned integer and the pair the thread index mod 32. Quiet NaN
// (0x7fc00000) where the pinned function has no value.
static __global__ void qx_consensus_math_kernel(const float* in, int n, uint4* out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float x = in[i];
  const unsigned nan_bits = 0x7fc00000u;
  uint4 r;
  r.x = isfinite(x) ? __float_as_uint(qx::pinned_exp(x)) : nan_bits;
  float v = 0.0f;
  r.y = qx::pinned_rsqrt(x, &v) ? __float_as_uint(v) : nan_bits;
  float s = 0.0f, c = 0.0f;
  if (qx::granite_sin_cos(__float2uint_rz(x), i & 31, &s, &c)) {
    r.z = __float_as_uint(s);
    r.w = __float_as_uint(c);
  } else {
    r.z = r.w = nan_bits;
  }
  out[i] = r;
}

qxc_status qxc_consensus_math_conformance(qxc_ctx* ctx, const float* inputs, int32_t n, uint32_t* out) {
  if (!ctx || n < 0 || (n > 0 && (!inputs || !out))) return fail(ctx, QXC_ERR_INVALID_ARG, "null argument");
  if (n == 0) return QXC_OK;
  QXC_CUDA(ctx, cudaSetDevice(ctx->device));
  float* din = nullptr;
  uint4* dout = nullptr;
  QXC_CUDA(ctx, cudaMalloc(&din, sizeof(float) * n));
  cudaError_t e = cudaMalloc(&dout, sizeof(uint4) * n);
  if (e == cudaSuccess) e = cudaMemcpyAsync(din, inputs, sizeof(float) * n, cudaMemcpyHostToDevice, ctx->stream);
  if (e == cudaSuccess) {
    qx_consensus_math_kernel<<<(n + 255) / 256, 256, 0, ctx->stream>>>(din, n, dout);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) e = cudaMemcpyAsync(out, dout, sizeof(uint4) * n, cudaMemcpyDeviceToHost, ctx->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
  cudaFree(din);
  cudaFree(dout);
  QXC_CUDA(ctx, e);
  return QXC_OK;
}

qxc_status qxc_blake3_compress_rate(qxc_ctx* ctx, double* per_second) {
  if (!ctx || !per_second) return fail(ctx, QXC_ERR_INVALID_ARG, "null argument");
  QXC_CUDA(ctx, cudaSetDevice(ctx->device));
  int sms = 0;
  QXC_CUDA(ctx, cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, ctx->device));
  int per_sm = 0;
  QXC_CUDA(ctx, cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, qx_b3_compress_rate_kernel, 256, 0));
  const int grid = sms * std::max(per_sm, 1), iters = 2048;
  cudaEvent_t e0, e1;
  QXC_CUDA(ctx, cudaEventCreate(&e0));
  QXC_CUDA(ctx, cudaEventCreate(&e1));
  float best = 1e30f;
  for (int rep = 0; rep < 4; ++rep) {  // the first is warm-up
    cudaEventRecord(e0, ctx->stream);
    qx_b3_compress_rate_kernel<<<grid, 256, 0, ctx->stream>>>(iters);
    cudaEventRecord(e1, ctx->stream);
    cudaEventSynchronize(e1);
    float ms = 0.f;
    cudaEventElapsedTime(&ms, e0, e1);
    if (rep > 0) best = std::min(best, ms);
  }
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  QXC_CUDA(ctx, cudaGetLastError());
  *per_second = (double)grid * 256 * iters / (best * 1e-3);
  return QXC_OK;
}

}  // extern "C"
