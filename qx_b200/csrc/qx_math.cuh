// qx_math.cuh — qx's pinned binary32 math on the device, bit-identical to
// crates/qx-consensus-math/src/lib.rs (same constants, same operation order).
//
// Every multiply, add and fused multiply-add is an explicit round-to-nearest
// intrinsic (__fmul_rn, __fadd_rn, __fmaf_rn), so nvcc cannot contract or
// reorder them whatever -fmad is set to. These are qx's own published
// polynomials; no CUDA math-library routine is involved.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace qx {

// Granite inverse frequencies for theta=1e4, head_dim 64
// (GRANITE_ROPE_INVERSE_FREQUENCY_BITS, qx-consensus-math lib.rs:28-61).
__constant__ uint32_t kGraniteInvFreqBits[32] = {
    0x3f800000u, 0x3f3ff911u, 0x3f0ff59au, 0x3ed7e89bu, 0x3ea1e89bu, 0x3e72d424u,
    0x3e361887u, 0x3e088d77u, 0x3dcccccdu, 0x3d99940eu, 0x3d6655c3u, 0x3d2cba15u,
    0x3d0186e2u, 0x3cc24350u, 0x3c91ad39u, 0x3c5a7bf1u, 0x3c23d70au, 0x3bf5b9b0u,
    0x3bb8449cu, 0x3b8a2e77u, 0x3b4f3e37u, 0x3b1b690du, 0x3ae91528u, 0x3aaec98eu,
    0x3a83126fu, 0x3a44948cu, 0x3a136a16u, 0x39dd1726u, 0x39a5cb5fu, 0x3978a814u,
    0x393a7753u, 0x390bd472u};

__device__ __forceinline__ float fbits(uint32_t b) { return __uint_as_float(b); }

// exp_f32 (lib.rs:70-110). Caller guarantees a finite argument; the clamps
// are kept. Returns +inf-free results for the attention domain (x <= 0).
__device__ __forceinline__ float pinned_exp(float x) {
  if (x < -87.0f) return 0.0f;
  if (x > 88.0f) return fbits(0x7f7fffffu);
  float scaled = __fmaf_rn(x, fbits(0x3fb8aa3bu), 0.0f);
  float rounded = scaled >= 0.0f ? __fadd_rn(scaled, 0.5f) : __fsub_rn(scaled, 0.5f);
  int exponent = __float2int_rz(rounded);
  float ef = __int2float_rn(exponent);
  float r = __fmaf_rn(-ef, fbits(0x3f317200u), x);
  r = __fmaf_rn(-ef, fbits(0x35bfbe8eu), r);
  float p = fbits(0x39500d01u);
  p = __fmaf_rn(p, r, fbits(0x3ab60b61u));
  p = __fmaf_rn(p, r, fbits(0x3c088889u));
  p = __fmaf_rn(p, r, fbits(0x3d2aaaabu));
  p = __fmaf_rn(p, r, fbits(0x3e2aaaabu));
  p = __fmaf_rn(p, r, fbits(0x3f000000u));
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  float pow2 = fbits((uint32_t)(exponent + 127) << 23);
  return __fmul_rn(p, pow2);
}

// Hardware base-2 exponential (MUFU.EX2) of x*log2(e); ablation / Qwen path.
__device__ __forceinline__ float native_exp(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x * 1.4426950408889634f));
  return y;
}

// Hardware base-2 exponential (MUFU.EX2); exp2(-inf) = +0.
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x for x <= 0 on the FMA pipe, for kernels whose exponentials would
// otherwise all queue on the special-function unit. Cody-Waite split
// x = n + f with n = round(x) (adding and removing 1.5 * 2^23 rounds to an
// integer held in the low mantissa bits) and f in [-0.5, 0.5]; 2^f from a
// degree-3 polynomial fitted here for minimum relative error on that
// interval (max relative error 7.5e-5, far below the bf16 rounding of its
// callers); 2^n joins through the exponent field. 0 below 2^-125.
__device__ __forceinline__ float exp2_poly(float x) {
  const float xc = fmaxf(x, -125.0f);
  const float j = __fadd_rn(xc, 12582912.0f);
  const float n = __fsub_rn(j, 12582912.0f);
  const float f = __fsub_rn(xc, n);
  float p = __fmaf_rn(0.05517132207751274f, f, 0.24261054396629333f);
  p = __fmaf_rn(p, f, 0.6932609677314758f);
  p = __fmaf_rn(p, f, 0.9999281167984009f);
  const float r = __int_as_float(__float_as_int(p) + (__float_as_int(j) << 23));
  return x < -125.0f ? 0.0f : r;
}

// exp2_poly of two arguments with the packed f32 operations of sm_100 (one
// instruction per pair for each add and FMA); bit-identical to two calls of
// exp2_poly, since every packed lane rounds like its scalar twin and
// xc - n is exact.
__device__ __forceinline__ float2 exp2_poly2(float2 x) {
  const float2 xc = make_float2(fmaxf(x.x, -125.0f), fmaxf(x.y, -125.0f));
  const float2 j = __fadd2_rn(xc, make_float2(12582912.0f, 12582912.0f));
  const float2 n = __fadd2_rn(j, make_float2(-12582912.0f, -12582912.0f));
  const float2 f = __ffma2_rn(n, make_float2(-1.0f, -1.0f), xc);
  float2 p = __ffma2_rn(make_float2(0.05517132207751274f, 0.05517132207751274f), f,
                        make_float2(0.24261054396629333f, 0.24261054396629333f));
  p = __ffma2_rn(p, f, make_float2(0.6932609677314758f, 0.6932609677314758f));
  p = __ffma2_rn(p, f, make_float2(0.9999281167984009f, 0.9999281167984009f));
  const float rx = __int_as_float(__float_as_int(p.x) + (__float_as_int(j.x) << 23));
  const float ry = __int_as_float(__float_as_int(p.y) + (__float_as_int(j.y) << 23));
  return make_float2(x.x < -125.0f ? 0.0f : rx, x.y < -125.0f ? 0.0f : ry);
}

// max of three f32 values in one instruction (sm_100's three-input max)
__device__ __forceinline__ float fmax3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

__device__ __forceinline__ float softmax_exp(float x, bool pinned) {
  return pinned ? pinned_exp(x) : native_exp(x);
}

// sin_cos_f32 (lib.rs:148-189). Returns false where the reference returns
// None (non-finite or |angle| > 4096).
__device__ __forceinline__ bool pinned_sin_cos(float angle, float* s, float* c) {
  if (!isfinite(angle) || fabsf(angle) > 4096.0f) return false;
  float scaled = __fmaf_rn(angle, fbits(0x3e22f983u), 0.0f);
  float rounded = scaled >= 0.0f ? __fadd_rn(scaled, 0.5f) : __fsub_rn(scaled, 0.5f);
  int turns = __float2int_rz(rounded);
  float tf = __int2float_rn(turns);
  float r = __fmaf_rn(-tf, fbits(0x40c90fdbu), angle);
  r = __fmaf_rn(-tf, fbits(0xb43bbd2eu), r);
  float sign = 1.0f;
  if (r > fbits(0x3fc90fdbu)) {
    r = __fsub_rn(fbits(0x40490fdbu), r);
    sign = -1.0f;
  } else if (r < -fbits(0x3fc90fdbu)) {
    r = __fsub_rn(-fbits(0x40490fdbu), r);
    sign = -1.0f;
  }
  float sq = __fmul_rn(r, r);
  float sp = fbits(0x2f309231u);
  sp = __fmaf_rn(sp, sq, fbits(0xb2d7322bu));
  sp = __fmaf_rn(sp, sq, fbits(0x3638ef1du));
  sp = __fmaf_rn(sp, sq, fbits(0xb9500d01u));
  sp = __fmaf_rn(sp, sq, fbits(0x3c088889u));
  sp = __fmaf_rn(sp, sq, fbits(0xbe2aaaabu));
  *s = __fmaf_rn(__fmul_rn(sp, sq), r, r);
  float cp = fbits(0x310f76c7u);
  cp = __fmaf_rn(cp, sq, fbits(0xb493f27eu));
  cp = __fmaf_rn(cp, sq, fbits(0x37d00d01u));
  cp = __fmaf_rn(cp, sq, fbits(0xbab60b61u));
  cp = __fmaf_rn(cp, sq, fbits(0x3d2aaaabu));
  cp = __fmaf_rn(cp, sq, fbits(0xbf000000u));
  *c = __fmul_rn(__fmaf_rn(cp, sq, 1.0f), sign);
  return true;
}

// rsqrt_f32 (qx-consensus-math lib.rs:114-128): integer seed and four fixed
// Newton steps; false for a non-positive or non-finite input or result.
__device__ __forceinline__ bool pinned_rsqrt(float x, float* out) {
  if (!isfinite(x) || x <= 0.0f) return false;
  const float half = __fmul_rn(x, 0.5f);
  float e = __uint_as_float(0x5f375a86u - (__float_as_uint(x) >> 1));
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float square = __fmul_rn(e, e);
    const float correction = __fmaf_rn(-half, square, 1.5f);
    e = __fmul_rn(e, correction);
  }
  *out = e;
  return isfinite(e);
}

// granite_rope_sin_cos (lib.rs:192-195).
__device__ __forceinline__ bool granite_sin_cos(uint32_t position, int pair, float* s, float* c) {
  float angle = __fmul_rn(__uint2float_rn(position), fbits(kGraniteInvFreqBits[pair]));
  return pinned_sin_cos(angle, s, c);
}

// granite_rope_pair (lib.rs:199-207) with (sin, cos) already evaluated.
__device__ __forceinline__ bool granite_rotate(float left, float right, float s, float c,
                                               float* first, float* second) {
  if (!isfinite(left) || !isfinite(right)) return false;
  float a = __fmaf_rn(-right, s, __fmul_rn(left, c));
  float b = __fmaf_rn(right, c, __fmul_rn(left, s));
  *first = a;
  *second = b;
  return isfinite(a) && isfinite(b);
}

// ---- element conversions ------------------------------------------------
template <typename T> struct Elem;
template <> struct Elem<float> {
  static __device__ __forceinline__ float to_f32(float x) { return x; }
  static __device__ __forceinline__ float from_f32(float x) { return x; }
};
template <> struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }
  static __device__ __forceinline__ __nv_bfloat16 from_f32(float x) { return __float2bfloat16_rn(x); }
};
template <> struct Elem<__half> {
  static __device__ __forceinline__ float to_f32(__half x) { return __half2float(x); }
  static __device__ __forceinline__ __half from_f32(float x) { return __float2half_rn(x); }
};

// Load element i of a runtime-typed array (0 f32, 1 bf16, 2 f16).
__device__ __forceinline__ float load_any(const void* base, long long i, int dtype) {
  if (dtype == 1) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(base)[i]);
  if (dtype == 2) return __half2float(reinterpret_cast<const __half*>(base)[i]);
  return reinterpret_cast<const float*>(base)[i];
}
// N elements base[i0 + stride * j] (j < N) of a runtime dtype, every load
// issued before the first is used (a loop of load_any that stores each
// value to shared memory would wait for each load in turn: the generic
// source pointer might alias the shared destination).
template <int N>
__device__ __forceinline__ void load_any_n(const void* base, long long i0, int stride, int dtype, float* out) {
  if (dtype == 1) {
    const __nv_bfloat16* b = reinterpret_cast<const __nv_bfloat16*>(base) + i0;
    __nv_bfloat16 r[N];
#pragma unroll
    for (int j = 0; j < N; ++j) r[j] = b[(long long)stride * j];
#pragma unroll
    for (int j = 0; j < N; ++j) out[j] = __bfloat162float(r[j]);
  } else if (dtype == 2) {
    const __half* b = reinterpret_cast<const __half*>(base) + i0;
    __half r[N];
#pragma unroll
    for (int j = 0; j < N; ++j) r[j] = b[(long long)stride * j];
#pragma unroll
    for (int j = 0; j < N; ++j) out[j] = __half2float(r[j]);
  } else {
    const float* b = reinterpret_cast<const float*>(base) + i0;
#pragma unroll
    for (int j = 0; j < N; ++j) out[j] = b[(long long)stride * j];
  }
}

__device__ __forceinline__ void store_any(void* base, long long i, int dtype, float v) {
  if (dtype == 1) reinterpret_cast<__nv_bfloat16*>(base)[i] = __float2bfloat16_rn(v);
  else if (dtype == 2) reinterpret_cast<__half*>(base)[i] = __float2half_rn(v);
  else reinterpret_cast<float*>(base)[i] = v;
}

// Four consecutive elements from shared memory as f32.
template <typename T> __device__ __forceinline__ float4 lds4(const T* p);
template <> __device__ __forceinline__ float4 lds4<float>(const float* p) {
  return *reinterpret_cast<const float4*>(p);
}
template <> __device__ __forceinline__ float4 lds4<__nv_bfloat16>(const __nv_bfloat16* p) {
  uint2 u = *reinterpret_cast<const uint2*>(p);
  return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u),
                     __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xffff0000u));
}
template <> __device__ __forceinline__ float4 lds4<__half>(const __half* p) {
  uint2 u = *reinterpret_cast<const uint2*>(p);
  __half2 a = *reinterpret_cast<__half2*>(&u.x), b = *reinterpret_cast<__half2*>(&u.y);
  float2 fa = __half22float2(a), fb2 = __half22float2(b);
  return make_float4(fa.x, fa.y, fb2.x, fb2.y);
}

// Sixteen bytes of shared memory (4 f32 or 8 16-bit elements) as f32.
template <typename T> struct Vec16;
template <> struct Vec16<float> {
  static constexpr int N = 4;
  static __device__ __forceinline__ void load(const float* p, float* o) {
    const float4 v = *reinterpret_cast<const float4*>(p);
    o[0] = v.x; o[1] = v.y; o[2] = v.z; o[3] = v.w;
  }
};
template <> struct Vec16<__nv_bfloat16> {
  static constexpr int N = 8;
  static __device__ __forceinline__ void load(const __nv_bfloat16* p, float* o) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      o[2 * i] = __uint_as_float(w[i] << 16);
      o[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  }
};
template <> struct Vec16<__half> {
  static constexpr int N = 8;
  static __device__ __forceinline__ void load(const __half* p, float* o) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
      o[2 * i] = f.x;
      o[2 * i + 1] = f.y;
    }
  }
};

}  // namespace qx
