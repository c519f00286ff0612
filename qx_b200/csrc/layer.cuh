// layer.cuh — the projections around attention in a Granite layer with Q4
// weights (the reference's attention sub-layer, qx-runtime-v2
// CpuQ4Reference::step lib.rs:4680-4706, GPU stage encode_attention_layer
// :6916-6994):
//
//   normalized = cpu_rms_norm_simd(hidden, input_norm)          (:4924-4946)
//   q, k, v    = Q4 mat-vecs of normalized                      (qx-quant :892-933)
//   attention  = the decode kernel (RoPE, append, GQA attention)
//   out        = fma(RESIDUAL_MULTIPLIER, o_proj(attention), hidden)
//
// Q4 here is the reference's row-major layout with group 32: per row and
// group an FP16 scale and 16 bytes of codes, low nibble first, value =
// (code - 7) * scale. The reference's mat-vec accumulates column c into lane
// c % 32 with fma and reduces the 32 lanes as (16, 8, 4, 2, 1) — exactly a
// warp with one row per warp and a shuffle-down tree, so the projections
// below are bit-identical to it; the RMSNorm keeps its 256 fma partials and
// two 32-lane trees the same way.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

#include "qx_math.cuh"
#include "qx_ptx.cuh"

namespace qx {

constexpr int kHidden = 1024;
constexpr float kResidualMultiplier = 0.22f;  // qx-model lib.rs:22
constexpr float kRmsEpsilon = 1e-6f;          // qx-model lib.rs:24

struct Q4Ref {
  const uint8_t* codes;    // [rows][cols / 32][16]
  const uint16_t* scales;  // [rows][cols / 32] FP16 bits
  int rows, cols;
};

struct LayerParams {
  const float* hidden;  // [1024] layer input
  const float* norm;    // [1024] input RMSNorm weight
  Q4Ref w[3];           // q, k, v projections (or one matrix for qxc_q4_mat_vec)
  float* y[3];          // their outputs
  int nmat;             // matrices in w / y
  int normalize;        // RMSNorm the input first (else the input is used as is)
  const float* residual;  // o-projection: out = fma(0.22, W x, residual) when non-null
  unsigned* err;
  unsigned long long* trace;
};

// One row of a Q4 matrix against x (shared memory), by the warp; the sum is
// returned in lane 0. Lane l owns columns l, l + 32, ... — nibble l of every
// group. The row's codes arrive as one 16-byte load per lane (group l) and
// pass through the warp's shared staging slice, from which lane l reads byte
// l / 2 of each group; group j's scale comes from lane j by a shuffle.
__device__ __forceinline__ float q4_row_dot(const uint8_t* __restrict__ codes, const uint16_t* __restrict__ scales,
                                            int groups, const float* x, uint8_t* stage, int lane) {
  float acc = 0.0f;
  for (int g0 = 0; g0 < groups; g0 += 32) {
    const bool mine = g0 + lane < groups;
    const uint4 c = mine ? __ldg(reinterpret_cast<const uint4*>(codes) + g0 + lane) : make_uint4(0u, 0u, 0u, 0u);
    const float sc_l = mine ? __half2float(__ushort_as_half(__ldg(scales + g0 + lane))) : 0.0f;
    __syncwarp();
    reinterpret_cast<uint4*>(stage)[lane] = c;
    __syncwarp();
    const int n = min(32, groups - g0);
#pragma unroll 8
    for (int j = 0; j < n; ++j) {
      const float sc = __shfl_sync(0xffffffffu, sc_l, j);
      const int code = (stage[j * 16 + (lane >> 1)] >> ((lane & 1) * 4)) & 0xF;
      const float value = __fmul_rn((float)(code - 7), sc);
      acc = __fmaf_rn(value, x[(g0 + j) * 32 + lane], acc);
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, off));
  return acc;
}

// RMSNorm (optional), then every row of the nmat matrices, one row per warp;
// 256 threads. With `residual`, row r's output is fma(0.22, dot, residual[r]).
__global__ void __launch_bounds__(256) qx_q4_matvec_kernel(const __grid_constant__ LayerParams p) {
  __shared__ float xs[kHidden * 4];  // the input vector (up to 4096 columns)
  __shared__ __align__(16) uint8_t stage[8][512];
  __shared__ float part[8];
  __shared__ float s_scale;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  pdl_launch_dependents();  // the next kernel may get resident and wait for this one
  pdl_wait();
  const int cols = p.w[0].cols;
  if (p.normalize) {
    // every input and weight element of this thread in flight at once
    float hv[kHidden / 256], wv[kHidden / 256];
#pragma unroll
    for (int k = 0; k < kHidden / 256; ++k) {
      hv[k] = p.hidden[tid + 256 * k];
      wv[k] = p.norm[tid + 256 * k];
    }
    // cpu_rms_norm_simd: thread t sums x[t], x[t + 256], ... by fma; warps
    // and then the 8 warp sums reduce as reduce_simd32
    float sum = 0.0f;
#pragma unroll
    for (int k = 0; k < kHidden / 256; ++k) sum = __fmaf_rn(hv[k], hv[k], sum);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) sum = __fadd_rn(sum, __shfl_down_sync(0xffffffffu, sum, off));
    if (lane == 0) part[warp] = sum;
    __syncthreads();
    if (warp == 0) {
      float g = lane < 8 ? part[lane] : 0.0f;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) g = __fadd_rn(g, __shfl_down_sync(0xffffffffu, g, off));
      if (lane == 0) {
        float scale = 0.0f;
        if (!pinned_rsqrt(__fadd_rn(__fdiv_rn(g, (float)kHidden), kRmsEpsilon), &scale))
          flag_error(p.err, QX_ERR_BIT_NONFINITE);
        s_scale = scale;
      }
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < kHidden / 256; ++k) xs[tid + 256 * k] = __fmul_rn(__fmul_rn(hv[k], s_scale), wv[k]);
  } else {
    for (int i = tid; i < cols; i += 256) xs[i] = p.hidden[i];
  }
  __syncthreads();
  int total = 0;
  for (int m = 0; m < p.nmat; ++m) total += p.w[m].rows;
  for (int row = blockIdx.x * 8 + warp; row < total; row += gridDim.x * 8) {
    int m = 0, r = row;
    while (r >= p.w[m].rows) r -= p.w[m].rows, ++m;
    const Q4Ref w = p.w[m];
    const int groups = w.cols / 32;
    const float y = q4_row_dot(w.codes + (long long)r * groups * 16, w.scales + (long long)r * groups, groups, xs,
                               stage[warp], lane);
    if (lane == 0) {
      float v = p.residual ? __fmaf_rn(kResidualMultiplier, y, p.residual[r]) : y;
      if (!isfinite(v)) flag_error(p.err, QX_ERR_BIT_NONFINITE);
      p.y[m][r] = v;
    }
  }
}

}  // namespace qx
