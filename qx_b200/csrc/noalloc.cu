// noalloc.cu — qxc_granite_decode_static_scratch: one Granite decode step
// that allocates no device memory at call time.
//
// Who needs it: callers that own every byte of device memory themselves and
// must not have a library allocate behind their back. Examples are a host
// runtime that, like qx's static execution plan, sizes one arena before
// token generation and forbids allocation afterwards; code running under a
// memory pool or budget that cudaMalloc would bypass; and hosts whose
// allocator is not the CUDA runtime's. The regular qxc_decode grows its
// split-KV scratch (partials and merge tickets) with cudaMalloc on demand,
// which such callers cannot allow.
//
// Here that scratch is a file-scope static __device__ array of
// kStaticScratchBytes (128 KiB). Every GPU that loads libqxcuda holds one
// copy of it until the process exits. The caller passes the KV cache and the
// q/k/v/out tensors as device pointers; the call itself performs no
// cudaMalloc, cudaFree or other allocating routine.
//
// Rules that come with a shared static buffer:
//  - The first call on each device does a one-time set-up with that device
//    current: it looks up the array's device address (cudaGetSymbolAddress)
//    and, per KV precision, sets the kernel's shared-memory attribute. Make
//    that first call before any stream capture on the device. The set-up
//    runs once per device even when several host threads call at once.
//  - With split 0 the split comes from the wave model of qxc_decode
//    (qxc_auto_split), limited to the splits whose partials fit the array
//    (30 for one Granite layer). The merge of the splits always runs inside
//    the decode kernel (the last CTA of each kv head), whatever their number.
//  - All calls on a device share the one array and it keeps the last call's
//    contents. The merge tickets that must start at zero are cleared by each
//    call (an asynchronous memset on the caller's stream). Two calls whose
//    kernels overlap on the GPU (different streams, no ordering between
//    them) race on the array and may produce wrong results: order them.
//  - A request whose split-KV partials would not fit in the array is
//    rejected with QXC_ERR_INVALID_ARG and a message naming both sizes.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "../../include/qxcuda.h"
#include "decode.cuh"

using namespace qx;

namespace {

constexpr size_t kStaticScratchBytes = 128 * 1024;
constexpr size_t kTicketBytes = 256;  // 8 kv-head tickets, padded to the alignment
constexpr size_t kPartialBytes = 2 * (64 + 2) * sizeof(float);  // one work item's (O, m, l) for 2 query heads
// Splits of the one (sequence, layer) a call decodes that fit the array:
// 8 kv-head work items per split.
constexpr int kStaticMaxSplits = (int)((kStaticScratchBytes - kTicketBytes) / (8 * kPartialBytes));

// The scratch: [0, kTicketBytes) merge tickets, then split partials.
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

constexpr int kMaxDevices = 64;
constexpr int kPairs = 5;  // accepted (key, value) dtype pairs

// One-time set-up, race-free when several host threads make their first
// call at once: std::call_once per device (the scratch address, the SM
// count) and per (device, dtype pair) (the kernel's shared-memory attribute
// and its resident CTAs per SM). Each slot is written inside its call_once
// and only read after it, which call_once orders.
struct DeviceSetup {
  std::once_flag once;
  cudaError_t status = cudaSuccess;
  void* scratch = nullptr;
  int sm_count = 0;
};
struct KernelSetup {
  std::once_flag once;
  cudaError_t status = cudaSuccess;
  int blocks_per_sm = 1;
};
DeviceSetup g_device[kMaxDevices];
KernelSetup g_kernel[kMaxDevices][kPairs];

qxc_status say(char* msg, size_t len, qxc_status st, const char* text) {
  if (msg && len) snprintf(msg, len, "%s", text);
  return st;
}

size_t esize(int dt) { return dt == QXC_F32 ? 4 : 2; }

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

qxc_status encode_map(CUtensorMap* map, void* base, int dtype, int capacity, char* msg, size_t len) {
  const PFN_cuTensorMapEncodeTiled_v12000 fn = encode_fn();
  if (!fn) return say(msg, len, QXC_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  const size_t es = esize(dtype);
  const CUtensorMapDataType t = dtype == QXC_F32    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                : dtype == QXC_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                    : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  cuuint64_t dims[3] = {64, 8, (cuuint64_t)capacity};
  cuuint64_t strides[2] = {(cuuint64_t)(64 * es), (cuuint64_t)(8 * 64 * es)};
  cuuint32_t box[3] = {(cuuint32_t)(128 / es), 1, 64};
  cuuint32_t estr[3] = {1, 1, 1};
  if (fn(map, t, 3, base, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return say(msg, len, QXC_ERR_INVALID_ARG, "cache pointer or capacity not usable for a TMA tensor map");
  return QXC_OK;
}

// The kernel's set-up on this device (with it current): shared-memory
// attribute, then resident CTAs per SM for the split model.
template <typename KT, typename VT>
const KernelSetup& kernel_setup(int dev, int pair) {
  KernelSetup& k = g_kernel[dev][pair];
  std::call_once(k.once, [&k] {
    using C = DecodeCfg<Granite, KT, VT>;
    k.status = cudaFuncSetAttribute(qx_decode_kernel<Granite, KT, VT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    C::SMEM);
    int n = 1;
    if (k.status == cudaSuccess)
      k.status = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, qx_decode_kernel<Granite, KT, VT>, C::NT, C::SMEM);
    k.blocks_per_sm = n > 0 ? n : 1;
  });
  return k;
}

template <typename KT, typename VT>
qxc_status launch(DecodeParams& p, int attend, int split, const DeviceSetup& ds, int dev, int pair,
                  cudaStream_t stream, char* msg, size_t len) {
  using C = DecodeCfg<Granite, KT, VT>;
  const KernelSetup& ks = kernel_setup<KT, VT>(dev, pair);
  if (ks.status != cudaSuccess) return say(msg, len, QXC_ERR_CUDA, cudaGetErrorString(ks.status));
  const int max_splits = std::min(kStaticMaxSplits, C::MAX_SPLITS);
  // the split: the same wave model qxc_decode uses (qxc_auto_split), over
  // the splits that fit the array
  int chunk = split;
  if (chunk == 0) chunk = qxc_auto_split(ds.sm_count * ks.blocks_per_sm, &attend, 1, 8, max_splits, C::T);
  if (chunk <= 0) return say(msg, len, QXC_ERR_INVALID_ARG, "no split fits the static scratch");
  const int nsplit = (attend + chunk - 1) / chunk;
  const int items = nsplit * 8;
  const size_t need = kTicketBytes + (size_t)items * kPartialBytes;
  if (need > kStaticScratchBytes) {
    char buf[160];
    snprintf(buf, sizeof(buf),
             "split-KV scratch of %zu bytes exceeds the static scratch of %zu bytes; use a larger split",
             need, kStaticScratchBytes);
    return say(msg, len, QXC_ERR_INVALID_ARG, buf);
  }
  p.chunk = chunk;
  // Tickets must start at zero; the array keeps whatever the last call left.
  if (cudaMemsetAsync(p.tickets, 0, kTicketBytes, stream) != cudaSuccess)
    return say(msg, len, QXC_ERR_CUDA, "clearing the static scratch failed");
  qx_decode_kernel<Granite, KT, VT><<<items, C::NT, C::SMEM, stream>>>(p);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return say(msg, len, QXC_ERR_CUDA, cudaGetErrorString(e));
  return QXC_OK;
}

}  // namespace

extern "C" qxc_status qxc_granite_decode_static_scratch(const qxc_static_decode_args* a, void* cuda_stream,
                                                        char* msg, size_t len) {
  if (msg && len) msg[0] = '\0';
  if (!a) return say(msg, len, QXC_ERR_INVALID_ARG, "null arguments");
  if (!a->key_cache || !a->value_cache || !a->q || !a->k || !a->v || !a->out)
    return say(msg, len, QXC_ERR_INVALID_ARG, "null tensor pointer");
  if (a->capacity < 1 || a->capacity > 4096)
    return say(msg, len, QXC_ERR_INVALID_ARG, "capacity must be in 1..=4096");
  if (a->position < 0 || a->position >= a->capacity) {
    char buf[96];
    snprintf(buf, sizeof(buf), "KV position %d exceeds context %d", a->position, a->capacity);
    return say(msg, len, QXC_ERR_POSITION, buf);
  }
  const int kd = a->key_dtype, vd = a->value_dtype;
  const bool kv_ok = (kd == QXC_F32 && vd == QXC_F32) || (kd == QXC_F32 && vd == QXC_F16) ||
                     (kd == QXC_F16 && vd == QXC_F32) || (kd == QXC_F16 && vd == QXC_F16) ||
                     (kd == QXC_BF16 && vd == QXC_BF16);
  if (!kv_ok) return say(msg, len, QXC_ERR_UNSUPPORTED, "unsupported KV precision");
  auto dt_ok = [](int d) { return d == QXC_F32 || d == QXC_BF16 || d == QXC_F16; };
  if (!dt_ok(a->q_dtype) || !dt_ok(a->in_dtype) || !dt_ok(a->out_dtype))
    return say(msg, len, QXC_ERR_INVALID_ARG, "unknown tensor dtype");
  if (a->split < 0 || a->split % 64 != 0)
    return say(msg, len, QXC_ERR_INVALID_ARG, "split must be 0 or a positive multiple of 64");

  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return say(msg, len, QXC_ERR_CUDA, "no current CUDA device");

  // One-time set-up on this device (with it current): the device address of
  // the static scratch and the SM count used to size the split.
  DeviceSetup& ds = g_device[dev];
  std::call_once(ds.once, [&ds, dev] {
    void* ptr = nullptr;
    ds.status = cudaGetSymbolAddress(&ptr, g_static_scratch);
    int sms = 0;
    if (ds.status == cudaSuccess) ds.status = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    ds.scratch = ptr;
    ds.sm_count = sms > 0 ? sms : 1;
  });
  if (ds.status != cudaSuccess) return say(msg, len, QXC_ERR_CUDA, cudaGetErrorString(ds.status));

  const int attend = a->position + 1;
  DecodeParams p;
  memset(&p, 0, sizeof(p));
  qxc_status st = encode_map(&p.tmk, a->key_cache, kd, a->capacity, msg, len);
  if (st != QXC_OK) return st;
  st = encode_map(&p.tmv, a->value_cache, vd, a->capacity, msg, len);
  if (st != QXC_OK) return st;
  p.capacity = a->capacity;
  p.k_region = static_cast<char*>(a->key_cache);
  p.v_region = static_cast<char*>(a->value_cache);
  p.layers = 1;
  p.layer_begin = 0;
  p.layer_count = 1;
  p.n_seq = 1;
  p.seq_table = nullptr;
  p.single.seq_id = 0;
  p.single.attend = attend;
  p.single.new_slot = a->position;
  p.single.rope_pos = a->position;
  p.single.item_begin = 0;
  p.q = a->q;
  p.k = a->k;
  p.v = a->v;
  p.out = a->out;
  p.q_dtype = a->q_dtype;
  p.in_dtype = a->in_dtype;
  p.out_dtype = a->out_dtype;
  p.pinned_exp = (a->flags & QXC_DECODE_NATIVE_EXP) ? 0 : 1;
  p.emit_partials = 0;
  unsigned char* scratch = static_cast<unsigned char*>(ds.scratch);
  p.tickets = reinterpret_cast<int*>(scratch);
  p.partials = reinterpret_cast<float*>(scratch + kTicketBytes);
  p.err = a->device_error;

  cudaStream_t stream = static_cast<cudaStream_t>(cuda_stream);
  const int split = a->split;
  if (kd == QXC_F32 && vd == QXC_F32) return launch<float, float>(p, attend, split, ds, dev, 0, stream, msg, len);
  if (kd == QXC_F32 && vd == QXC_F16) return launch<float, __half>(p, attend, split, ds, dev, 1, stream, msg, len);
  if (kd == QXC_F16 && vd == QXC_F32) return launch<__half, float>(p, attend, split, ds, dev, 2, stream, msg, len);
  if (kd == QXC_F16 && vd == QXC_F16) return launch<__half, __half>(p, attend, split, ds, dev, 3, stream, msg, len);
  return launch<__nv_bfloat16, __nv_bfloat16>(p, attend, split, ds, dev, 4, stream, msg, len);
}
