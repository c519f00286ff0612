// exchange.cuh — the KV-length split's exchange and merge over NVLink in one
// kernel: each rank pushes its per-query-head partials (O, m, l) straight
// into every rank's inbox with peer stores, then waits for every rank's
// partial of its head and merges.
//
// This replaces the all-gather + merge of the split (the combine of
// qx-runtime-v2's split attention, re-derived for a KV split across GPUs:
// M = max m_r, O = sum e^(m_r - M) O_r / sum e^(m_r - M) l_r), with the
// ranks in a fixed order, so every rank's output is bit-identical to
// qx_lse_merge_kernel over the all-gathered partials.
//
// No memory fence: every 32-bit value travels with a 32-bit tag in one
// 8-byte store, which a reader sees whole or not at all; the reader polls
// each value until its tag is the step's. A system-scope fence costs a few
// microseconds on B200, several times the whole exchange.
//
// Memory of one rank's exchange area (device, opened by the peers through
// CUDA IPC): inbox [2][world][HQ][D+2] of {value, tag}, and the local step
// counters [HQ]. Step s of head h uses tag s+1 and half s & 1 of the inbox,
// so a rank pushing step s+2 into the same half never overwrites what a peer
// still reads of step s: that push follows this rank's merge of step s+1,
// which needed the peer's step s+1 push, which followed the peer's merge of
// step s (every rank runs the same steps in the same stream order). Tags
// never repeat within 2^32 steps, so a stale value is never taken for the
// current one.
//
// Waits are bounded (kMaxWaitNs of %globaltimer): a missing peer turns into
// QX_ERR_BIT_TIMEOUT | QX_ERR_BIT_PEER, and the CTA returns without merging
// and marks the peer group failed. Every later exchange on a failed group
// returns at once with the same error, before it pushes anything: the step
// counters of the heads that timed out did not advance while the others'
// did, so the tags no longer tell one step from the next (a slow peer's
// next push carries the tag this rank still waits for).
#pragma once
#include "decode.cuh"

namespace qx {

constexpr int kMaxPeers = 8;
constexpr int kExchThreads = 128;

struct ExchangeParams {
  uint2* inbox[kMaxPeers];  // every rank's inbox base (index = rank), this rank's own included
  unsigned* step;           // this rank's [HQ] step counters
  unsigned* failed;         // this rank's group-failed word (device)
  unsigned* failed_host;    // the same fact for the host (mapped pinned memory)
  int rank, world;
  int hq, d;                // query heads and head dim of the model (d <= kExchThreads)
  const float* partials;    // this rank's [HQ][D+2]
  void* out;                // [HQ][D]
  int out_dtype;
  int pinned;
  unsigned* err;
  unsigned long long* trace;  // stage timeline (diagnostics), or null
};

// One CTA per query head.
__global__ void __launch_bounds__(kExchThreads) qx_exchange_merge_kernel(const __grid_constant__ ExchangeParams p) {
  __shared__ float ml[2 * kMaxPeers];  // m_r, l_r
  __shared__ int s_ok;
  const int h = blockIdx.x, tid = threadIdx.x;
  const int HQ = p.hq, D = p.d, W = p.world;
  StageTrace trace(p.trace, h, tid == 0);
  trace.mark();  // resident
  // the next grid may get resident and set up meanwhile: this grid's CTAs
  // are all resident already (one per query head), and the next grid waits
  // for this one's completion before it touches anything
  pdl_launch_dependents();
  pdl_wait();  // the partials come from the previous grid
  trace.mark();  // partials ready
  // one thread reads the failed word, so the whole CTA takes one branch
  if (tid == 0) s_ok = peer_group_failed(p.failed) ? 0 : 1;
  __syncthreads();
  if (!s_ok) {
    if (tid == 0) flag_error(p.err, QX_ERR_BIT_TIMEOUT | QX_ERR_BIT_PEER);
    return;
  }
  const unsigned s = p.step[h], tag = s + 1u, half = s & 1u;
  // 1. push this rank's head-h partial into every rank's inbox [half][rank][h]
  const long long slot = (((long long)half * W + p.rank) * HQ + h) * (D + 2);
  for (int i = tid; i < D + 2; i += kExchThreads) {
    const float v = __ldcg(p.partials + (long long)h * (D + 2) + i);
    for (int r = 0; r < W; ++r) st_tagged(p.inbox[r] + slot + i, v, tag);
  }
  trace.mark();  // pushed
  // 2. collect every rank's head-h partial: thread d takes O[d] of each rank,
  //    threads 0 .. 2W-1 also take (m, l)
  const uint2* in = p.inbox[p.rank] + ((long long)half * W * HQ + h) * (D + 2);
  const long long rs = (long long)HQ * (D + 2);
  bool ok = true;
  float o[kMaxPeers];
#pragma unroll
  for (int r = 0; r < kMaxPeers; ++r) o[r] = 0.0f;
  {
    // O[tid] of every rank (tid < D) and, on threads 0 .. 2W-1, (m, l) of
    // rank tid / 2, all polled together
    float v = 0.0f;
    const uint2* mlp = tid < 2 * W ? in + (tid >> 1) * rs + D + (tid & 1) : nullptr;
    ok = wait_tagged_n<kMaxPeers>(in + tid, rs, tid < D ? W : 0, mlp, tag, o, &v);
    if (tid < 2 * W) ml[tid] = v;
  }
  if (!ok) {
    flag_error(p.err, QX_ERR_BIT_TIMEOUT | QX_ERR_BIT_PEER);
    mark_peer_group_failed(p.failed, p.failed_host);
    s_ok = 0;
  }
  __syncthreads();
  trace.mark();  // every rank's partial is here
  if (!s_ok) return;
  // 3. merge in rank order (qx_lse_merge_kernel's arithmetic)
  if (tid < D) {
    float mx = -INFINITY;
    for (int r = 0; r < W; ++r) mx = fmaxf(mx, ml[2 * r]);
    float L = 0.0f, O = 0.0f;
#pragma unroll
    for (int r = 0; r < kMaxPeers; ++r) {
      if (r >= W) break;
      const float m = ml[2 * r];
      if (m == -INFINITY) continue;  // empty shard
      const float w = softmax_exp(m - mx, p.pinned != 0);
      L = fmaf(w, ml[2 * r + 1], L);
      O = fmaf(w, o[r], O);
    }
    const float v = O / L;
    if (!isfinite(v)) flag_error(p.err, QX_ERR_BIT_NONFINITE);
    store_any(p.out, (long long)h * D + tid, p.out_dtype, v);
  }
  if (tid == 0) p.step[h] = s + 1u;
  trace.mark();  // merged
}

}  // namespace qx
