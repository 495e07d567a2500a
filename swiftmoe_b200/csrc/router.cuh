// Router kernels: gate logits (fp32 accumulation), top-k with lower-index ties, softmax
// over the selected logits.
//
// Reference behaviour restated: models/baseline_moe.py:56-67 (nn.Linear gate -> topk ->
// softmax over the k logits) and models/ultimate_moe.py:288-293 (same via matmul).
// The reference's Triton kernel (models/ultimate_moe.py:34-101) only scans 128 columns
// and fills absent experts with 0.0 logits; this router scans exactly E experts.
#pragma once
#include "common.cuh"

namespace smoe {

// Select the top-k of the E logits held one per lane (lanes >= E hold nothing) and
// write indices / softmax weights for one token.  All lanes take part.
__device__ __forceinline__ void warp_topk_softmax_lane_values(float mine, int lane, int E, int k, int32_t* idx_out,
                                                              float* w_out) {
  float v = lane < E ? mine : -INFINITY;
  int i = lane < E ? lane : 0x7fffffff;
  // k <= E <= 32 on this path.  Lane j keeps the j-th selected value; the first
  // selection is the maximum, so exp(v - first) is the max-shifted softmax numerator.
  float first = 0.f, sum = 0.f, my_ex = 0.f;
  int my_idx = 0;
  for (int j = 0; j < k; ++j) {
    float bv = v;
    int bi = i;
    warp_argbest(bv, bi);
    if (j == 0) first = bv;
    const float ex = expf(bv - first);
    sum += ex;
    if (lane == j) { my_ex = ex; my_idx = bi; }
    if (i == bi) { v = -INFINITY; i = 0x7fffffff; }
  }
  if (lane < k) {
    idx_out[lane] = my_idx;
    w_out[lane] = my_ex / sum;
  }
}

// Small-E fused router.  One warp handles TOK tokens at a time; the gate matrix sits in
// shared memory (E*d elements); every lane streams 16-byte vectors of x.
template <typename T, int EMAX, int TOK, int VEC>
__global__ void __launch_bounds__(256) router_small_kernel(const T* __restrict__ x, const T* __restrict__ wg,
                                                           const float* __restrict__ bias, int T_, int d, int E,
                                                           int k, int32_t* __restrict__ idx, float* __restrict__ w,
                                                           float* __restrict__ logits_out) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  T* s_wg = reinterpret_cast<T*>(smem_raw);
  // stage the gate matrix once per block
  {
    const int n = E * d;
    if constexpr (VEC > 1) {
      const uint4* src = reinterpret_cast<const uint4*>(wg);
      uint4* dst = reinterpret_cast<uint4*>(s_wg);
      for (int i = threadIdx.x; i < n / VEC; i += blockDim.x) dst[i] = src[i];
    } else {
      for (int i = threadIdx.x; i < n; i += blockDim.x) s_wg[i] = wg[i];
    }
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int warps_total = gridDim.x * (blockDim.x >> 5);
  const int groups = (T_ + TOK - 1) / TOK;
  for (int gi = blockIdx.x * (blockDim.x >> 5) + warp; gi < groups; gi += warps_total) {
    const int t0 = gi * TOK;
    float acc[TOK][EMAX];
#pragma unroll
    for (int a = 0; a < TOK; ++a)
#pragma unroll
      for (int e = 0; e < EMAX; ++e) acc[a][e] = 0.f;
    for (int base = lane * VEC; base < d; base += 32 * VEC) {
      float xv[TOK][VEC];
#pragma unroll
      for (int a = 0; a < TOK; ++a) {
        if (t0 + a < T_) load_vec_f<T, VEC>(x + (size_t)(t0 + a) * d + base, xv[a]);
        else {
#pragma unroll
          for (int q = 0; q < VEC; ++q) xv[a][q] = 0.f;
        }
      }
#pragma unroll
      for (int e = 0; e < EMAX; ++e) {
        if (e < E) {
          float gv[VEC];
          load_vec_f<T, VEC>(s_wg + (size_t)e * d + base, gv);
#pragma unroll
          for (int a = 0; a < TOK; ++a)
#pragma unroll
            for (int q = 0; q < VEC; ++q) acc[a][e] = fmaf(xv[a][q], gv[q], acc[a][e]);
        }
      }
    }
#pragma unroll
    for (int a = 0; a < TOK; ++a) {
      const int t = t0 + a;
      float mine = 0.f;
#pragma unroll
      for (int e = 0; e < EMAX; ++e) {
        float s = warp_sum(acc[a][e]);
        if (lane == e) mine = s;
      }
      if (t >= T_) continue;  // warp-uniform
      if (logits_out != nullptr && lane < E) logits_out[(size_t)t * E + lane] = mine;
      if (bias != nullptr && lane < E) mine += bias[lane];
      warp_topk_softmax_lane_values(mine, lane, E, k, idx + (size_t)t * k, w + (size_t)t * k);
    }
  }
}

// Top-k + softmax from fp32 logits [T, E] (any E), one warp per row.
__global__ void __launch_bounds__(256) topk_from_logits_kernel(const float* __restrict__ logits,
                                                               const float* __restrict__ bias, int T_, int E, int k,
                                                               int32_t* __restrict__ idx, float* __restrict__ w) {
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= T_) return;
  const float* lg = logits + (size_t)row * E;
  // taken[] bit j of lane l marks expert l + 32*j as already selected (E <= 1024).
  uint32_t taken = 0;
  float first = 0.f, sum = 0.f, my_ex = 0.f;
  int my_idx = 0;
  for (int j = 0; j < k; ++j) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int s = 0; s * 32 + lane < E; ++s) {
      if (taken & (1u << s)) continue;
      const int e = s * 32 + lane;
      float v = lg[e];
      if (bias != nullptr) v += bias[e];
      if (ranks_before(v, e, bv, bi)) { bv = v; bi = e; }
    }
    warp_argbest(bv, bi);
    if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
    if (j == 0) first = bv;
    // the first selected value is the maximum (NaN ranks first and poisons the sum,
    // as torch.softmax does)
    const float ex = expf(bv - first);
    sum += ex;
    if (lane == j) { my_ex = ex; my_idx = bi; }
  }
  if (lane < k) {
    idx[(size_t)row * k + lane] = my_idx;
    w[(size_t)row * k + lane] = my_ex / sum;
  }
}

}  // namespace smoe
