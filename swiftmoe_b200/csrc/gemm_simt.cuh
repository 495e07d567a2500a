// fp32 grouped GEMM on the FFMA pipes (SIMT).  Used for fp32 layers, where the reference
// computes in full fp32 (models/ultimate_moe.py:187 with use_fp16=False) and the 1e-5
// max-abs tolerance rules out TF32 tensor cores.
//
// Same grouping contract as the tensor-core kernel: group g owns rows
// [offsets[g], ends ? ends[g] : offsets[g+1]) of A [rows, K]; B is [G, N, K].
// Block tile 128 x 128, K step 8, 256 threads with an 8 x 8 register tile each (rows
// ty*4 + {0..3} and 64 + ty*4 + {0..3}, columns tx*4 + {0..3} and 64 + tx*4 + {0..3}), so
// every k step costs four 16-byte shared-memory loads for 64 FMAs.  The next K slice is
// loaded from global memory into registers while the current one is multiplied, and
// the shared tiles are double-buffered (one barrier per K step).  For the SwiGLU
// epilogue the block's first 64 B-columns are gate rows n0.. and the last 64 the
// matching up rows, so each thread holds both halves of its four output columns and
// stores silu(gate) * up.
#pragma once
#include "common.cuh"

namespace smoe {
namespace simt {

constexpr int BM = 128, BN = 128, BK = 8, THREADS = 256, MAX_GROUPS = 1024, PAD = 4;

// Four consecutive K elements of one row (zeros past K or for a missing row).
__device__ __forceinline__ void load_k4(const float* __restrict__ row, int k, int K, bool vec, float (&v)[4]) {
  if (row != nullptr && vec && k + 3 < K) {
    const float4 t = *reinterpret_cast<const float4*>(row + k);
    v[0] = t.x;
    v[1] = t.y;
    v[2] = t.z;
    v[3] = t.w;
    return;
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = (row != nullptr && k + i < K) ? row[k + i] : 0.0f;
}

template <int EPI>
__global__ void __launch_bounds__(THREADS, 2) grouped_gemm_f32_kernel(const float* __restrict__ A,
                                                                      const float* __restrict__ B,
                                                                      const float* __restrict__ B3,
                                                                      float* __restrict__ C, int64_t ldc,
                                                                      const uint64_t* __restrict__ row_ptrs,
                                                                      const int32_t* __restrict__ offsets,
                                                                      const int32_t* __restrict__ ends, int G, int N,
                                                                      int K, int rows_cap) {
  pdl_wait();
  __shared__ int s_beg[MAX_GROUPS], s_fin[MAX_GROUPS];
  __shared__ int s_ts[MAX_GROUPS + 1];
  __shared__ __align__(16) float As[2][BK][BM + PAD];
  __shared__ __align__(16) float Bs[2][BK][BN + PAD];
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
  // STORE: output columns n0 .. n0+127.  SWIGLU: output columns n0 .. n0+63, B-tile
  // columns 0..63 = gate rows n0.., 64..127 = up rows n0..
  const int n0 = (EPI == SMOE_EPI_SWIGLU) ? blockIdx.y * (BN / 2) : blockIdx.y * BN;
  const float* Bg = B + (size_t)g * N * K;
  const float* B3g = (EPI == SMOE_EPI_SWIGLU) ? B3 + (size_t)g * N * K : nullptr;

  // loader: each thread brings 4 consecutive K elements of one A row and one B row
  const int lrow = threadIdx.x >> 1;       // 0..127
  const int lk = (threadIdx.x & 1) * 4;    // 0 or 4
  const float* ap = row0 + lrow < row_end ? A + (size_t)(row0 + lrow) * K : nullptr;
  const float* bp;
  {
    const int n = (EPI == SMOE_EPI_SWIGLU) ? n0 + (lrow & 63) : n0 + lrow;
    const float* src = (EPI == SMOE_EPI_SWIGLU && lrow >= 64) ? B3g : Bg;
    bp = n < N ? src + (size_t)n * K : nullptr;
  }
  const bool vec = (K & 3) == 0 && ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(B) |
                                     reinterpret_cast<uintptr_t>(B3)) & 15) == 0;
  float ra[4], rb[4];
  load_k4(ap, lk, K, vec, ra);
  load_k4(bp, lk, K, vec, rb);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    As[0][lk + i][lrow] = ra[i];
    Bs[0][lk + i][lrow] = rb[i];
  }
  __syncthreads();

  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;
  int buf = 0;
  for (int k0 = 0; k0 < K; k0 += BK) {
    const bool more = k0 + BK < K;
    if (more) {  // next K slice into registers while this one is multiplied
      load_k4(ap, k0 + BK + lk, K, vec, ra);
      load_k4(bp, k0 + BK + lk, K, vec, rb);
    }
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      const float4 a0 = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 4]);
      const float4 a1 = *reinterpret_cast<const float4*>(&As[buf][kk][64 + ty * 4]);
      const float4 b0 = *reinterpret_cast<const float4*>(&Bs[buf][kk][tx * 4]);
      const float4 b1 = *reinterpret_cast<const float4*>(&Bs[buf][kk][64 + tx * 4]);
      const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float b[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    if (more) {  // the other buffer was last read before the previous barrier
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        As[buf ^ 1][lk + i][lrow] = ra[i];
        Bs[buf ^ 1][lk + i][lrow] = rb[i];
      }
      __syncthreads();
      buf ^= 1;
    }
  }

#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int row = row0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
    if (row >= row_end) continue;
    float* crow = row_ptrs ? reinterpret_cast<float*>(row_ptrs[row]) : C + (int64_t)row * ldc;
    if (crow == nullptr) continue;
    if (EPI == SMOE_EPI_SWIGLU) {
      // column tx*4 + j: gate in acc[i][j], the matching up column in acc[i][j + 4]
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int n = n0 + tx * 4 + j;
        if (n < N) {
          const float gt = acc[i][j], up = acc[i][j + 4];
          crow[n] = gt / (1.0f + expf(-gt)) * up;
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int n = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + (j - 4));
        if (n < N) crow[n] = acc[i][j];
      }
    }
  }
  if (row_ptrs) __threadfence_system();  // rows in another GPU's memory: visible before exit
}

}  // namespace simt
}  // namespace smoe
