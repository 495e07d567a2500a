// fp32 grouped GEMM on the FFMA pipes (SIMT).  Used for fp32 layers, where the reference
// computes in full fp32 (models/ultimate_moe.py:187 with use_fp16=False) and the 1e-5
// max-abs tolerance rules out TF32 tensor cores.
//
// Same grouping contract as the tensor-core kernel: group g owns rows
// [offsets[g], ends ? ends[g] : offsets[g+1]) of A [rows, K]; B is [G, N, K].  Block tile 64 x 64,
// K step 16, 256 threads with a 4 x 4 register tile each.  For the SwiGLU epilogue a
// block computes 32 gate columns and the 32 matching up columns and stores
// silu(gate) * up.
#pragma once
#include "common.cuh"

namespace smoe {
namespace simt {

constexpr int BM = 64, BN = 64, BK = 16, THREADS = 256, MAX_GROUPS = 1024;

template <int EPI>
__global__ void __launch_bounds__(THREADS) grouped_gemm_f32_kernel(const float* __restrict__ A,
                                                                   const float* __restrict__ B,
                                                                   const float* __restrict__ B3, float* __restrict__ C,
                                                                   int64_t ldc, const uint64_t* __restrict__ row_ptrs,
                                                                   const int32_t* __restrict__ offsets,
                                                                   const int32_t* __restrict__ ends, int G, int N,
                                                                   int K, int rows_cap) {
  __shared__ int s_beg[MAX_GROUPS], s_fin[MAX_GROUPS];
  __shared__ int s_ts[MAX_GROUPS + 1];
  __shared__ float As[BK][BM + 4];
  __shared__ float Bs[BK][BN + 4];
  if (threadIdx.x == 0) {  // row ranges clamped into [0, rows_cap]
    int acc = 0;
    for (int g = 0; g < G; ++g) {
      const int b = min(max(offsets[g], 0), rows_cap);
      const int f = min(max(ends != nullptr ? ends[g] : offsets[g + 1], b), rows_cap);
      s_beg[g] = b;
      s_fin[g] = f;
      s_ts[g] = acc;
      acc += (f - b + BM - 1) / BM;
    }
    s_ts[G] = acc;
  }
  __syncthreads();
  const int mt = blockIdx.x;
  if (mt >= s_ts[G]) return;
  int lo = 0, hi = G - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (s_ts[mid] <= mt) lo = mid; else hi = mid - 1;
  }
  const int g = lo;
  const int row0 = s_beg[g] + (mt - s_ts[g]) * BM;
  const int row_end = s_fin[g];
  // column layout of the block: STORE -> output columns n0 .. n0+63;
  // SWIGLU -> smem columns 0..31 = gate rows n0.., 32..63 = up rows n0..
  const int n0 = (EPI == SMOE_EPI_SWIGLU) ? blockIdx.y * 32 : blockIdx.y * BN;
  const float* Bg = B + (size_t)g * N * K;
  const float* B3g = (EPI == SMOE_EPI_SWIGLU) ? B3 + (size_t)g * N * K : nullptr;

  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  float acc[4][4] = {};
  const int lr = threadIdx.x >> 2;         // 0..63 : tile row loaded by this thread
  const int lk = (threadIdx.x & 3) * 4;    // 0,4,8,12
  for (int k0 = 0; k0 < K; k0 += BK) {
    {
      const int row = row0 + lr;
      float v[4] = {0.f, 0.f, 0.f, 0.f};
      if (row < row_end) {
        const float* p = A + (size_t)row * K + k0 + lk;
#pragma unroll
        for (int i = 0; i < 4; ++i)
          if (k0 + lk + i < K) v[i] = p[i];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) As[lk + i][lr] = v[i];
    }
    {
      const float* src;
      int n;
      if (EPI == SMOE_EPI_SWIGLU) {
        src = lr < 32 ? Bg : B3g;
        n = n0 + (lr & 31);
      } else {
        src = Bg;
        n = n0 + lr;
      }
      float v[4] = {0.f, 0.f, 0.f, 0.f};
      if (n < N) {
        const float* p = src + (size_t)n * K + k0 + lk;
#pragma unroll
        for (int i = 0; i < 4; ++i)
          if (k0 + lk + i < K) v[i] = p[i];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) Bs[lk + i][lr] = v[i];
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      float a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx + 16 * j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int row = row0 + ty * 4 + i;
    if (row >= row_end) continue;
    float* crow = row_ptrs ? reinterpret_cast<float*>(row_ptrs[row]) : C + (int64_t)row * ldc;
    if (crow == nullptr) continue;
    if (EPI == SMOE_EPI_SWIGLU) {
      // columns tx and tx+16 are gate; tx+32, tx+48 the matching up columns
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int n = n0 + tx + 16 * j;
        if (n < N) {
          const float gt = acc[i][j], up = acc[i][j + 2];
          crow[n] = gt / (1.0f + expf(-gt)) * up;
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int n = n0 + tx + 16 * j;
        if (n < N) crow[n] = acc[i][j];
      }
    }
  }
  if (row_ptrs) __threadfence_system();  // rows in another GPU's memory: visible before exit
}

}  // namespace simt
}  // namespace smoe
