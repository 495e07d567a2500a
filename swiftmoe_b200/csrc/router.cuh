// Router kernels: gate logits (fp32 accumulation), top-k with lower-index ties, softmax
// over the selected logits.
//
// Reference behaviour restated: models/baseline_moe.py:56-67 (nn.Linear gate -> topk ->
// softmax over the k logits) and models/ultimate_moe.py:288-293 (same via matmul).
// The reference's Triton kernel (models/ultimate_moe.py:34-101) only scans 128 columns
// and fills absent experts with 0.0 logits; this router scans exactly E experts.
#pragma once
#include <type_traits>

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
  pdl_wait_and_release();
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

// 16-byte loads kept in program order with the MMAs (volatile asm), so a whole batch of
// loads is in flight before the first MMA that consumes it.  x is streamed (no L1
// allocation); the small gate matrix is read through L1, where it stays resident.
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ uint4 ldg_keep(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
  return v;
}

// Two m16n8k16 MMAs (fp32 accumulate) over one 32-column step: fragment pairs .x/.y
// then .z/.w of the 16-byte chunks (see router_mma_kernel for the column order).
template <typename T>
__device__ __forceinline__ void mma_step(float (&c)[4], const uint4& a0, const uint4& a1, const uint4& b) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0.x), "r"(a1.x), "r"(a0.y), "r"(a1.y), "r"(b.x), "r"(b.y));
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0.z), "r"(a1.z), "r"(a0.w), "r"(a1.w), "r"(b.z), "r"(b.w));
  } else {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0.x), "r"(a1.x), "r"(a0.y), "r"(a1.y), "r"(b.x), "r"(b.y));
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0.z), "r"(a1.z), "r"(a0.w), "r"(a1.w), "r"(b.z), "r"(b.w));
  }
}

// Router for 16-bit x with E <= 32 on the warp-level tensor-core MMA
// (mma.sync m16n8k16, fp32 accumulate).  KSPLIT warps of a block share 16 tokens, each
// taking one slice of the d columns (4 slices when d % 128 == 0, else 2).  Per
// step of 32 columns a lane loads two 16-byte chunks of x (its token rows g and g+8) and,
// per 8 experts, one 16-byte chunk of the gate (read through L1, where the whole gate
// stays resident), and issues two MMAs per 8 experts; 8 steps are unrolled so 8 KB of x
// per warp is in flight.  The reduction index is permuted identically in both operands
// (lane quad q supplies columns 8q..8q+7 of the step as its fragment pairs), which leaves
// each dot product unchanged and makes every fragment one contiguous 16-byte load.  The
// slice sums meet in shared memory (added in a fixed order) and one lane per token does
// top-k + softmax.  The router reads x once: it is bound by HBM bandwidth.
// WARPS = 16, KSPLIT = 16 (d % 512 == 0) serves decode-sized batches: one block per 16
// tokens with 16 warps on the d columns, so a single token's router is one batch of loads
// per warp instead of four.
template <typename T, int NT, int KSPLIT, int WARPS = 4>  // E <= 8 * NT; KSPLIT warps share 16 tokens
__global__ void __launch_bounds__(WARPS * 32) router_mma_kernel(const T* __restrict__ x, const T* __restrict__ wg,
                                                                const float* __restrict__ bias, int T_, int d, int E,
                                                                int k, int32_t* __restrict__ idx,
                                                                float* __restrict__ w,
                                                                float* __restrict__ logits_out) {
  pdl_wait_and_release();
  constexpr int GROUPS = WARPS / KSPLIT;       // 16-token groups per block
  __shared__ float s_part[WARPS][16][8 * NT];  // per warp: partial logits of its 16 tokens
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, q = lane & 3;
  const int part = warp % KSPLIT;          // which slice of the d columns
  const int t0 = blockIdx.x * 16 * GROUPS + (warp / KSPLIT) * 16;
  const int r0 = min(t0 + g, T_ - 1), r1 = min(t0 + g + 8, T_ - 1);
  const int dh = d / KSPLIT;               // a multiple of 32 on this path
  const T* x0 = x + (size_t)r0 * d + part * dh + q * 8;
  const T* x1 = x + (size_t)r1 * d + part * dh + q * 8;
  const T* gq = wg + part * dh + q * 8;
  float acc[NT][4];
#pragma unroll
  for (int n = 0; n < NT; ++n)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[n][j] = 0.f;
  // batches of UNR steps: all loads of a batch are issued before its MMAs, so a warp keeps
  // UNR * 1 KB of x in flight
  constexpr int UNR = 8;
  int kb = 0;
  for (; kb + 32 * UNR <= dh; kb += 32 * UNR) {
    uint4 A0[UNR], A1[UNR], Bv[UNR][NT];
#pragma unroll
    for (int u = 0; u < UNR; ++u) {
      A0[u] = ldg_stream(x0 + kb + 32 * u);
      A1[u] = ldg_stream(x1 + kb + 32 * u);
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        const int e = min(n * 8 + g, E - 1);  // rows >= E are multiplied by zero below
        Bv[u][n] = ldg_keep(gq + (size_t)e * d + kb + 32 * u);
        if (n * 8 + g >= E) Bv[u][n] = make_uint4(0, 0, 0, 0);
      }
    }
#pragma unroll
    for (int u = 0; u < UNR; ++u)
#pragma unroll
      for (int n = 0; n < NT; ++n) mma_step<T>(acc[n], A0[u], A1[u], Bv[u][n]);
  }
  for (; kb < dh; kb += 32) {
    const uint4 a0 = __ldg(reinterpret_cast<const uint4*>(x0 + kb));
    const uint4 a1 = __ldg(reinterpret_cast<const uint4*>(x1 + kb));
#pragma unroll
    for (int n = 0; n < NT; ++n) {
      const int e = n * 8 + g;
      const uint4 b = e < E ? __ldg(reinterpret_cast<const uint4*>(gq + (size_t)e * d + kb)) : make_uint4(0, 0, 0, 0);
      mma_step<T>(acc[n], a0, a1, b);
    }
  }
  // D fragment: acc[n][0..1] = token g, experts 8n+2q..+1; acc[n][2..3] = token g+8
#pragma unroll
  for (int n = 0; n < NT; ++n) {
    s_part[warp][g][n * 8 + 2 * q] = acc[n][0];
    s_part[warp][g][n * 8 + 2 * q + 1] = acc[n][1];
    s_part[warp][g + 8][n * 8 + 2 * q] = acc[n][2];
    s_part[warp][g + 8][n * 8 + 2 * q + 1] = acc[n][3];
  }
  __syncthreads();
  if (part == 0 && lane < 16 && t0 + lane < T_) {
    const int t = t0 + lane;
    float row[8 * NT];
#pragma unroll
    for (int e = 0; e < 8 * NT; ++e) {
      float v = s_part[warp][lane][e];
#pragma unroll
      for (int p = 1; p < KSPLIT; ++p) v += s_part[warp + p][lane][e];  // fixed order
      row[e] = v;
    }
    if (logits_out != nullptr)
      for (int e = 0; e < E; ++e) logits_out[(size_t)t * E + e] = row[e];
    if (bias != nullptr)
      for (int e = 0; e < E; ++e) row[e] += bias[e];
    // top-k by repeated selection, ties -> lower index, NaN first
    uint32_t taken = 0;
    float first = 0.f, sum = 0.f;
    for (int j = 0; j < k; ++j) {
      float bv = -INFINITY;
      int bi = 0x7fffffff;
#pragma unroll
      for (int e = 0; e < 8 * NT; ++e) {
        if (e >= E || (taken & (1u << e))) continue;
        if (ranks_before(row[e], e, bv, bi)) { bv = row[e]; bi = e; }
      }
      taken |= 1u << bi;
      if (j == 0) first = bv;
      const float ex = expf(bv - first);
      sum += ex;
      idx[(size_t)t * k + j] = bi;
      w[(size_t)t * k + j] = ex;
    }
    for (int j = 0; j < k; ++j) w[(size_t)t * k + j] /= sum;
  }
}

// Top-k + softmax from fp32 logits [T, E] (any E), one warp per row.
__global__ void __launch_bounds__(256) topk_from_logits_kernel(const float* __restrict__ logits,
                                                               const float* __restrict__ bias, int T_, int E, int k,
                                                               int32_t* __restrict__ idx, float* __restrict__ w) {
  pdl_wait_and_release();
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
