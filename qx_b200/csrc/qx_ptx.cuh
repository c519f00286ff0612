// qx_ptx.cuh — hand-written PTX for sm_100a: mbarriers, TMA bulk copies,
// and bounded waits.
//
// Every wait on an mbarrier is bounded: after kMaxWaitNs it gives up,
// records QX_ERR_BIT_TIMEOUT in the context's error word and returns
// false, so a kernel never spins forever. No copy issued here is
// broadcast to other CTAs.
#pragma once
#include <stdint.h>

namespace qx {

// Error-word bits (qxc_sync maps them to status codes).
constexpr unsigned QX_ERR_BIT_NONFINITE = 0x1u;
constexpr unsigned QX_ERR_BIT_TIMEOUT = 0x2u;
// An exchange with peer ranks gave up (or found its peer group already
// failed): qxc_sync reports QXC_ERR_TIMEOUT and names the peer group.
constexpr unsigned QX_ERR_BIT_PEER = 0x4u;

// A peer group that has seen a timed-out exchange is failed for good. Its
// ranks' step counters no longer agree (the heads that timed out did not
// advance, the others did), so a later exchange could take a peer's earlier
// push, which carries the same tag, for the current one. The first CTA to
// give up stores 1 into the group's device word (read by every later
// exchange kernel before it pushes anything) and into its pinned host word
// (read by the host before every later exchange call).
__device__ __forceinline__ bool peer_group_failed(const unsigned* failed) {
  return failed && *reinterpret_cast<const volatile unsigned*>(failed) != 0u;
}
__device__ __forceinline__ void mark_peer_group_failed(unsigned* failed, unsigned* failed_host) {
  if (failed) *reinterpret_cast<volatile unsigned*>(failed) = 1u;
  if (failed_host) *reinterpret_cast<volatile unsigned*>(failed_host) = 1u;
}

// Record a device-side error. The word lives in mapped pinned host memory;
// a plain volatile store (no read-modify-write) is enough because the host
// only needs "some error happened, of this kind".
__device__ __forceinline__ void flag_error(unsigned* err, unsigned bit) {
  if (err) *reinterpret_cast<volatile unsigned*>(err) = bit;
}

// Bound on any device-side wait, in nanoseconds of %globaltimer: far beyond
// a legitimate copy latency (microseconds), short enough that a stuck wait
// returns an error to the host instead of holding the GPU.
constexpr unsigned long long kMaxWaitNs = 1000000000ull;

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Tagged values for exchanges between GPUs without a memory fence: a 32-bit
// value and a 32-bit tag travel in one 8-byte store, which a reader sees
// whole or not at all, so a reader that polls until the tag is the one it
// expects has the value that came with it.
__device__ __forceinline__ void st_tagged(uint2* p, float v, unsigned tag) {
  asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(__float_as_uint(v)), "r"(tag) : "memory");
}
__device__ __forceinline__ uint2 ld_tagged(const uint2* p) {
  uint2 v;
  asm volatile("ld.volatile.global.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p) : "memory");
  return v;
}

// Poll `count` <= N tagged values p[k * stride] (and `extra`, if not null)
// until every one carries `tag`. All loads are in flight together and only
// the values still missing are loaded again, so waiting for N peers costs one
// round trip after the last one arrived, not N. v[k] is 0 for k >= count.
// False after kMaxWaitNs.
template <int N>
__device__ __forceinline__ bool wait_tagged_n(const uint2* p, long long stride, int count, const uint2* extra,
                                              unsigned tag, float* v, float* vextra) {
  uint2 x[N];
#pragma unroll
  for (int k = 0; k < N; ++k) x[k] = k < count ? ld_tagged(p + k * stride) : make_uint2(0u, tag);
  uint2 e = extra ? ld_tagged(extra) : make_uint2(0u, tag);
  unsigned long long t0 = 0;
  for (unsigned spins = 0;; ++spins) {
    bool all = e.y == tag;
#pragma unroll
    for (int k = 0; k < N; ++k) all &= x[k].y == tag;
    if (all) break;
#pragma unroll
    for (int k = 0; k < N; ++k)
      if (x[k].y != tag) x[k] = ld_tagged(p + k * stride);
    if (e.y != tag) e = ld_tagged(extra);
    if ((spins & 15u) == 0u) {
      const unsigned long long now = global_ns();
      if (t0 == 0) {
        t0 = now;
      } else if (now - t0 > kMaxWaitNs) {
        return false;
      }
    }
  }
#pragma unroll
  for (int k = 0; k < N; ++k) v[k] = __uint_as_float(x[k].x);
  if (vextra) *vextra = __uint_as_float(e.x);
  return true;
}

// Stage timeline for diagnostics (host switch QXC_TRACE): one writer thread
// per CTA stores %globaltimer at stage boundaries into kTraceSlots slots of a
// per-launch buffer; a null buffer makes every mark a no-op.
constexpr int kTraceSlots = 48;

struct StageTrace {
  unsigned long long* slot;
  int n;
  __device__ __forceinline__ StageTrace(unsigned long long* base, long long cta, bool writer)
      : slot(base && writer ? base + cta * kTraceSlots : nullptr), n(0) {}
  __device__ __forceinline__ void mark() {
    if (slot && n < kTraceSlots) slot[n++] = global_ns();
  }
};

// Programmatic dependent launch: the running grid lets the next grid in the
// stream start its prologue; the dependent grid waits for this grid's
// completion (and its memory) before touching what it produced.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Named barrier `id` among the `n` threads (a multiple of 32) that execute
// it; id 0 is the one __syncthreads uses.
__device__ __forceinline__ void named_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

// Make mbarrier initialisation visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Bounded wait for phase `parity` of `bar`. Returns false (and flags the
// error word) if the phase never completed within the poll budget.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, unsigned* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long start = global_ns();
  for (;;) {
    if (mbar_try_wait(bar, parity)) return true;
    if (global_ns() - start > kMaxWaitNs) break;
  }
  flag_error(err, QX_ERR_BIT_TIMEOUT);
  return false;
}

// TMA tensor-tile copy (3-D tensor map) global -> this CTA's shared memory.
// The innermost coordinate x must be a multiple of 16 bytes' worth of
// elements; callers only pass x = 0 or a multiple of a 128-byte box.
__device__ __forceinline__ void tma_load_3d(void* dst, const void* tmap, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(smem_addr(dst)),
      "l"(tmap), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar))
      : "memory");
}

// Prefetch of a TMA tile into L2 only: nothing lands in shared memory and
// no barrier completes (a plain copy for this CTA). L2 stays coherent with later
// writes, so any rows may be prefetched, settled or not.
__device__ __forceinline__ void tma_prefetch_3d(const void* tmap, int x, int y, int z) {
  asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(tmap), "r"(x), "r"(y),
               "r"(z)
               : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

}  // namespace qx
