// Grouped GEMM for decode-sized batches (at most MAX_ROWS rows in all groups together),
// 16-bit inputs.  With a handful of rows the layer is a stream of expert weights: the
// tensor-core kernel's 128-row tiles would give the down projection of one token
// 2 experts x 16 column tiles = 32 CTAs for 148 SMs.  Here one warp owns one output
// column n of one group: its lanes read the weight row B[g][n][:] (and B3[g][n][:] for
// SwiGLU) in 16-byte pieces, 8 pieces per matrix in flight per lane, multiply them with
// every row of the group (A rows stay in L1/L2) and reduce across the warp.  Groups
// without rows read nothing, so a token routed to 2 of 8 experts streams 2 experts'
// weights, and the warps stride over the (group with rows, column) pairs only.
//
// (A ring of 1-D bulk copies into shared memory, consumed by 8 warps behind a named
// barrier, measured slower on the Mixtral decode shapes: 70 / 146 us for the down and
// gate/up projections against 60 / 83 us here; the per-stage barrier and reduction cost
// more than the deeper copies save.)
//
// Same grouping contract as the other grouped GEMMs: group g owns rows
// [offsets[g], ends ? ends[g] : offsets[g+1]) of A [rows, K], clamped to rows_cap;
// B is [G, N, K].  K % 8 == 0, A and B 16-byte aligned.  With a_index, row r of the
// groups reads row a_index[r] of A (the dispatch plan's row_token: the layer's first GEMM
// gathers the token rows itself, no permuted copy); an index outside [0, a_rows) reads
// zeros.
#pragma once
#include "common.cuh"

namespace smoe {
namespace gemv {

constexpr int THREADS = 256, MAX_ROWS = 2, MAX_GROUPS = 1024;
// 16-byte weight loads in flight per lane, per matrix.  16 for the one-matrix kernel
// measured slower on the Mixtral down projection (67 vs 60 us): it fits 2 blocks per SM
// instead of 3, and more warps beat more bytes per warp here.
constexpr int UNROLL = 8;
// Batches this small take this kernel.  Measured on the Mixtral layer (1 B200, 1965 MHz):
// one token (2 rows, one per expert) runs gate/up in 92 us and down in 62 us against 119
// and 95 us on the tensor cores.  An earlier build of this kernel for up to 16 rows took
// 553 + 546 us at 8 tokens (2 rows per expert) against 322 + 146 us on the tensor cores,
// its per-row work outgrowing the weight stream, hence the 2-row limit.
constexpr int DISPATCH_ROWS = MAX_ROWS;

template <typename T>
__device__ __forceinline__ void fma8(const uint4& a, const uint4& b, float& acc) {
  const T* x = reinterpret_cast<const T*>(&a);
  const T* y = reinterpret_cast<const T*>(&b);
#pragma unroll
  for (int i = 0; i < 8; ++i) acc = fmaf(Num<T>::to_f(x[i]), Num<T>::to_f(y[i]), acc);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// KS warps share one column: warp part p of a column reads the p-th of KS equal slices of
// K, and the slices' sums are added in slice order (deterministic).  KS = 2 for long rows
// (the down projection's 28 KB rows): half the load rounds per task and twice the tasks,
// so the last wave of tasks is shorter.
template <int EPI, typename T, typename OutT, int KS>
__global__ void __launch_bounds__(THREADS, 2) grouped_gemv_kernel(const T* __restrict__ A, const T* __restrict__ B,
                                                               const T* __restrict__ B3, OutT* __restrict__ C,
                                                               int64_t ldc, const uint64_t* __restrict__ row_ptrs,
                                                               const int32_t* __restrict__ offsets,
                                                               const int32_t* __restrict__ ends, int G, int N, int K,
                                                               int rows_cap, const int32_t* __restrict__ a_index,
                                                               int a_rows) {
  pdl_wait_and_release();
  constexpr int CPB = (THREADS / 32) / KS;   // columns per block and step
  constexpr int H = EPI == SMOE_EPI_SWIGLU ? 2 : 1;
  // Groups with rows, compacted: the warps stride over (active group, column) tasks only,
  // so a token routed to 2 of 8 experts keeps every warp on a weight row of those 2.
  __shared__ int s_beg[MAX_GROUPS], s_fin[MAX_GROUPS], s_act[MAX_GROUPS];
  __shared__ int s_nact;
  __shared__ float s_part[CPB][KS][MAX_ROWS][H];
  for (int g = threadIdx.x; g < G; g += blockDim.x) {
    const int b = min(max(offsets[g], 0), rows_cap);
    s_beg[g] = b;
    s_fin[g] = min(max(ends != nullptr ? ends[g] : offsets[g + 1], b), min(rows_cap, b + MAX_ROWS));
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int n = 0;
    for (int g = 0; g < G; ++g)
      if (s_fin[g] > s_beg[g]) s_act[n++] = g;
    s_nact = n;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int wib = threadIdx.x >> 5;          // warp in block
  const int slot = wib / KS, part = wib - (wib / KS) * KS;
  const int64_t tasks = (int64_t)s_nact * N;
  const int chunks = K / 8;                  // 16-byte pieces per row
  const int per = (chunks + KS - 1) / KS;
  const int c_lo = min(chunks, part * per), c_hi = min(chunks, c_lo + per);
  for (int64_t base = (int64_t)blockIdx.x * CPB; base < tasks; base += (int64_t)gridDim.x * CPB) {
    const int64_t task = base + slot;
    const bool have = task < tasks;
    const int a = have ? (int)(task / N) : 0;
    const int g = s_act[a];
    const int n = have ? (int)(task - (int64_t)a * N) : 0;
    const int b = s_beg[g], nr = have ? s_fin[g] - b : 0;
    const uint4* brow = reinterpret_cast<const uint4*>(B + ((int64_t)g * N + n) * K);
    const uint4* b3row = EPI == SMOE_EPI_SWIGLU ? reinterpret_cast<const uint4*>(B3 + ((int64_t)g * N + n) * K)
                                                : nullptr;
    float acc[MAX_ROWS], acc3[MAX_ROWS];
#pragma unroll
    for (int r = 0; r < MAX_ROWS; ++r) acc[r] = acc3[r] = 0.0f;
    for (int c0 = c_lo + lane; have && c0 < c_hi; c0 += 32 * UNROLL) {
      uint4 wv[UNROLL], w3[UNROLL];
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) {
        const int c = c0 + u * 32;
        wv[u] = c < c_hi ? __ldcs(brow + c) : make_uint4(0u, 0u, 0u, 0u);  // weights: streamed once
        if (EPI == SMOE_EPI_SWIGLU) w3[u] = c < c_hi ? __ldcs(b3row + c) : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int r = 0; r < MAX_ROWS; ++r) {
        const int src = r < nr ? (a_index != nullptr ? a_index[b + r] : b + r) : -1;
        if (src >= 0 && src < a_rows) {
          const uint4* arow = reinterpret_cast<const uint4*>(A + (int64_t)src * K);
#pragma unroll
          for (int u = 0; u < UNROLL; ++u) {
            const int c = c0 + u * 32;
            if (c < c_hi) {
              const uint4 av = __ldg(arow + c);
              fma8<T>(av, wv[u], acc[r]);
              if (EPI == SMOE_EPI_SWIGLU) fma8<T>(av, w3[u], acc3[r]);
            }
          }
        }
      }
    }
    float v[MAX_ROWS][H];
#pragma unroll
    for (int r = 0; r < MAX_ROWS; ++r) {
      v[r][0] = warp_sum(acc[r]);
      if (EPI == SMOE_EPI_SWIGLU) v[r][H - 1] = warp_sum(acc3[r]);
    }
    if (KS > 1) {                            // slice sums meet in shared memory
      if (lane == 0)
#pragma unroll
        for (int r = 0; r < MAX_ROWS; ++r)
#pragma unroll
          for (int h = 0; h < H; ++h) s_part[slot][part][r][h] = v[r][h];
      __syncthreads();
      if (part == 0)
#pragma unroll
        for (int r = 0; r < MAX_ROWS; ++r)
#pragma unroll
          for (int h = 0; h < H; ++h) {
            float t = s_part[slot][0][r][h];
#pragma unroll
            for (int q = 1; q < KS; ++q) t += s_part[slot][q][r][h];
            v[r][h] = t;
          }
    }
    if (part == 0 && lane == 0) {
#pragma unroll
      for (int r = 0; r < MAX_ROWS; ++r) {
        if (r < nr) {
          float out = v[r][0];
          if (EPI == SMOE_EPI_SWIGLU) out = out / (1.0f + __expf(-out)) * v[r][H - 1];
          const int row = b + r;
          OutT* crow = row_ptrs ? reinterpret_cast<OutT*>(row_ptrs[row]) : C + (int64_t)row * ldc;
          if (crow != nullptr) crow[n] = Num<OutT>::from_f(out);
        }
      }
    }
    if (KS > 1) __syncthreads();             // s_part is reused by the next step
  }
  if (row_ptrs) __threadfence_system();  // rows in another GPU's memory: visible before exit
}

}  // namespace gemv
}  // namespace smoe
