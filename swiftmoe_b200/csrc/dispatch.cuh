// Dispatch plan (histogram -> scan -> stable scatter), row permutation, combine and a
// batched transpose.
//
// The reference groups the T*2 (token, slot) pairs by target rank with an unstable
// argsort (models/ultimate_moe.py:120), replicates tokens with repeat_interleave
// (:123) and groups again by local expert (:224-231).  Here the plan is built in one
// pass over the routing indices: per-block histograms, a scan over (expert, block) and
// a scatter that numbers the pairs of each expert in (token, slot) order using warp
// match/ballot ranks, so the result is deterministic and bit-exact across runs.
#pragma once
#include "common.cuh"

namespace smoe {

constexpr int kPlanThreads = 256;                  // 8 warps
constexpr int kPlanWarps = kPlanThreads / 32;
constexpr int kPlanSlotsPerWarp = 256;             // 8 steps of 32 slots
constexpr int kPlanChunk = kPlanWarps * kPlanSlotsPerWarp;  // slots per block

// Per-warp counts of each expert over the warp's slot range; cnt is [kPlanWarps][E].
__device__ __forceinline__ void plan_warp_counts(const int32_t* __restrict__ idx, int64_t n_slots, int E,
                                                 int64_t slot0, int* cnt) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  int* my = cnt + warp * E;
  for (int step = 0; step < kPlanSlotsPerWarp / 32; ++step) {
    const int64_t s = slot0 + warp * kPlanSlotsPerWarp + step * 32 + lane;
    int e = -1;
    if (s < n_slots) {
      e = idx[s];
      if (e != -1 && (e < 0 || e >= E)) {  // -1 marks a slot to skip
        set_device_error(kErrBadExpertIndex);
        e = -1;
      }
    }
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    if (e >= 0 && lane == __ffs(peers) - 1) my[e] += __popc(peers);
    __syncwarp();
  }
}

// Kernel 1: hist[b][e] = number of slots of block b routed to expert e.
__global__ void __launch_bounds__(kPlanThreads) plan_count_kernel(const int32_t* __restrict__ idx, int64_t n_slots,
                                                                  int E, int32_t* __restrict__ hist) {
  pdl_wait_and_release();
  extern __shared__ int cnt[];  // [kPlanWarps][E]
  for (int i = threadIdx.x; i < kPlanWarps * E; i += blockDim.x) cnt[i] = 0;
  __syncthreads();
  const int64_t slot0 = (int64_t)blockIdx.x * kPlanChunk;
  plan_warp_counts(idx, n_slots, E, slot0, cnt);
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int s = 0;
    for (int w = 0; w < kPlanWarps; ++w) s += cnt[w * E + e];
    hist[(size_t)blockIdx.x * E + e] = s;
  }
}

// Kernel 2 (one block): per-expert running base over blocks, totals, capacity cut and
// the exclusive scan of aligned kept counts into expert_offsets.
__global__ void __launch_bounds__(1024) plan_scan_kernel(const int32_t* __restrict__ hist, int nblocks, int E,
                                                         int capacity, int row_align, int32_t* __restrict__ base,
                                                         int32_t* __restrict__ counts, int32_t* __restrict__ offsets,
                                                         int32_t* __restrict__ row_token) {
  pdl_wait_and_release();
  extern __shared__ int s_kept[];  // [E] aligned kept counts, then scanned in place
  __shared__ int s_warp[32];
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int run = 0;
    for (int b = 0; b < nblocks; ++b) {
      base[(size_t)b * E + e] = run;
      run += hist[(size_t)b * E + e];
    }
    counts[e] = run;
    const int kept = capacity > 0 ? min(run, capacity) : run;
    s_kept[e] = ((kept + row_align - 1) / row_align) * row_align;
  }
  __syncthreads();
  // block-wide exclusive scan of s_kept[0..E): each thread owns a contiguous strip
  const int per = (E + blockDim.x - 1) / blockDim.x;
  const int lo = min(E, (int)threadIdx.x * per), hi = min(E, lo + per);
  int local = 0;
  for (int e = lo; e < hi; ++e) local += s_kept[e];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) s_warp[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    int v = lane < nw ? s_warp[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int u = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v += u;
    }
    if (lane < nw) s_warp[lane] = v;  // inclusive per-warp totals
  }
  __syncthreads();
  int run = (incl - local) + (warp > 0 ? s_warp[warp - 1] : 0);
  for (int e = lo; e < hi; ++e) {
    const int a = s_kept[e];
    offsets[e] = run;
    run += a;
  }
  if (threadIdx.x == blockDim.x - 1) offsets[E] = run;  // last strip ends at the total
  if (E == 0 && threadIdx.x == 0) offsets[0] = 0;
  __syncthreads();
  // alignment padding rows carry token -1
  if (row_align > 1) {
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
      const int kept = capacity > 0 ? min(counts[e], capacity) : counts[e];
      for (int r = offsets[e] + kept; r < offsets[e + 1]; ++r) row_token[r] = -1;
    }
  }
}

// Kernel 3: stable scatter.  Slot s of expert e gets row offsets[e] + (number of
// earlier slots of e); slots at or beyond the capacity are dropped (-1).
__global__ void __launch_bounds__(kPlanThreads) plan_scatter_kernel(const int32_t* __restrict__ idx, int64_t n_slots,
                                                                    int k, int E, int capacity,
                                                                    const int32_t* __restrict__ base,
                                                                    const int32_t* __restrict__ offsets,
                                                                    int32_t* __restrict__ slot_row,
                                                                    int32_t* __restrict__ row_token) {
  pdl_wait_and_release();
  extern __shared__ int cnt[];  // [kPlanWarps][E], turned into per-warp running positions
  for (int i = threadIdx.x; i < kPlanWarps * E; i += blockDim.x) cnt[i] = 0;
  __syncthreads();
  const int64_t slot0 = (int64_t)blockIdx.x * kPlanChunk;
  plan_warp_counts(idx, n_slots, E, slot0, cnt);
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int run = base[(size_t)blockIdx.x * E + e];
    for (int w = 0; w < kPlanWarps; ++w) {
      const int c = cnt[w * E + e];
      cnt[w * E + e] = run;
      run += c;
    }
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  int* pos = cnt + warp * E;
  const unsigned lt = (1u << lane) - 1u;
  for (int step = 0; step < kPlanSlotsPerWarp / 32; ++step) {
    const int64_t s = slot0 + warp * kPlanSlotsPerWarp + step * 32 + lane;
    int e = -1;
    if (s < n_slots) {
      e = idx[s];
      if (e < 0 || e >= E) e = -1;
    }
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    int p = 0;
    if (e >= 0) p = pos[e] + __popc(peers & lt);
    __syncwarp();
    if (e >= 0 && lane == __ffs(peers) - 1) pos[e] += __popc(peers);
    __syncwarp();
    if (s < n_slots) {
      if (e < 0 || (capacity > 0 && p >= capacity)) {
        slot_row[s] = -1;
      } else {
        const int row = offsets[e] + p;
        slot_row[s] = row;
        row_token[row] = (int32_t)(s / k);
      }
    }
  }
}

// The three plan kernels in one launch for plans of one block (n_slots <= kPlanChunk,
// decode-sized batches): the single block's base is 0 for every expert, so counting,
// the capacity cut, the scan and the stable scatter run back to back in shared memory
// and give the same arrays as plan_count -> plan_scan -> plan_scatter.
__global__ void __launch_bounds__(kPlanThreads) plan_small_kernel(const int32_t* __restrict__ idx, int64_t n_slots,
                                                                  int k, int E, int capacity, int row_align,
                                                                  int32_t* __restrict__ counts,
                                                                  int32_t* __restrict__ offsets,
                                                                  int32_t* __restrict__ slot_row,
                                                                  int32_t* __restrict__ row_token) {
  pdl_wait_and_release();
  extern __shared__ int sm_plan[];
  int* cnt = sm_plan;                    // [kPlanWarps][E]: counts, then running positions
  int* s_off = cnt + kPlanWarps * E;     // [E + 1]: aligned kept rows, then their exclusive scan
  __shared__ int s_warp[kPlanWarps];
  for (int i = threadIdx.x; i < kPlanWarps * E; i += blockDim.x) cnt[i] = 0;
  __syncthreads();
  plan_warp_counts(idx, n_slots, E, 0, cnt);
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int run = 0;
    for (int w = 0; w < kPlanWarps; ++w) {
      const int c = cnt[w * E + e];
      cnt[w * E + e] = run;              // warp w's first position among expert e's slots
      run += c;
    }
    counts[e] = run;
    const int kept = capacity > 0 ? min(run, capacity) : run;
    s_off[e] = ((kept + row_align - 1) / row_align) * row_align;
  }
  __syncthreads();
  // exclusive scan of s_off[0..E) over contiguous per-thread strips
  const int per = (E + blockDim.x - 1) / blockDim.x;
  const int lo = min(E, (int)threadIdx.x * per), hi = min(E, lo + per);
  int local = 0;
  for (int e = lo; e < hi; ++e) local += s_off[e];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) s_warp[warp] = incl;
  __syncthreads();
  int run = incl - local;
  for (int w = 0; w < warp; ++w) run += s_warp[w];
  __syncthreads();                       // every strip has read its s_off entries
  for (int e = lo; e < hi; ++e) {
    const int a = s_off[e];
    s_off[e] = run;
    offsets[e] = run;
    run += a;
  }
  if (threadIdx.x == blockDim.x - 1) {   // the last strip ends at the total
    s_off[E] = run;
    offsets[E] = run;
  }
  __syncthreads();
  if (row_align > 1) {                   // alignment padding rows carry token -1
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
      const int c = counts[e];           // written by this thread above
      const int kept = capacity > 0 ? min(c, capacity) : c;
      for (int r = s_off[e] + kept; r < s_off[e + 1]; ++r) row_token[r] = -1;
    }
  }
  int* pos = cnt + warp * E;
  const unsigned lt = (1u << lane) - 1u;
  for (int step = 0; step < kPlanSlotsPerWarp / 32; ++step) {
    const int64_t s = warp * kPlanSlotsPerWarp + step * 32 + lane;
    int e = -1;
    if (s < n_slots) {
      e = idx[s];
      if (e < 0 || e >= E) e = -1;
    }
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    int p = 0;
    if (e >= 0) p = pos[e] + __popc(peers & lt);
    __syncwarp();
    if (e >= 0 && lane == __ffs(peers) - 1) pos[e] += __popc(peers);
    __syncwarp();
    if (s < n_slots) {
      if (e < 0 || (capacity > 0 && p >= capacity)) {
        slot_row[s] = -1;
      } else {
        const int row = s_off[e] + p;
        slot_row[s] = row;
        row_token[row] = (int32_t)(s / k);
      }
    }
  }
}

// rows[r,:] = x[row_token[r],:] for offsets[0] <= r < offsets[E] (a plan's offsets start
// at 0; a slice of them selects a range of experts); one warp per row, 16-byte vectors
// when every row starts on a 16-byte boundary.
__global__ void __launch_bounds__(256) permute_rows_kernel(const unsigned char* __restrict__ x, int64_t row_bytes,
                                                           bool vec, const int32_t* __restrict__ row_token,
                                                           const int32_t* __restrict__ offsets, int E,
                                                           unsigned char* __restrict__ rows) {
  pdl_wait_and_release();
  const int lane = threadIdx.x & 31;
  const int64_t first = offsets[0];
  const int64_t total = offsets[E];
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t r = first + (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < total; r += warps) {
    const int t = row_token[r];
    unsigned char* dst = rows + r * row_bytes;
    if (vec) {
      const int nv = (int)(row_bytes >> 4);
      uint4* d4 = reinterpret_cast<uint4*>(dst);
      if (t >= 0) {
        const uint4* s4 = reinterpret_cast<const uint4*>(x + (int64_t)t * row_bytes);
        int i = lane;
        for (; i + 96 < nv; i += 128) {   // four 16-byte loads in flight per lane
          const uint4 a = s4[i], b = s4[i + 32], c = s4[i + 64], e = s4[i + 96];
          d4[i] = a;
          d4[i + 32] = b;
          d4[i + 64] = c;
          d4[i + 96] = e;
        }
        for (; i < nv; i += 32) d4[i] = s4[i];
      } else {
        for (int i = lane; i < nv; i += 32) d4[i] = make_uint4(0, 0, 0, 0);
      }
    } else {
      const unsigned char* src = x + (int64_t)(t >= 0 ? t : 0) * row_bytes;
      for (int64_t i = lane; i < row_bytes; i += 32) dst[i] = t >= 0 ? src[i] : 0;
    }
  }
}

// out[t, c..c+VEC) = sum_j w[t,j] * y[slot_row[t,j], c..] (+ shared[t, c..]).
// Each product is rounded to fp32 before it is added (no fused multiply-add), in slot
// order: the same arithmetic as weighting the expert rows first and summing the k
// weighted fp32 rows afterwards, which is how the stage-by-stage API (expert outputs
// weighted in _expert_forward, slots summed in _combine_tokens) computes the layer.
template <typename T, int VEC>
__global__ void __launch_bounds__(256) combine_kernel(const T* __restrict__ y, const int32_t* __restrict__ slot_row,
                                                      const float* __restrict__ w, int T_, int k, int d,
                                                      const T* __restrict__ shared, T* __restrict__ out) {
  pdl_wait_and_release();
  const int per_row = d / VEC;
  const int64_t total = (int64_t)T_ * per_row;
  for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < total; g += (int64_t)gridDim.x * blockDim.x) {
    const int t = (int)(g / per_row);
    const int c = (int)(g - (int64_t)t * per_row) * VEC;
    float acc[VEC];
#pragma unroll
    for (int q = 0; q < VEC; ++q) acc[q] = 0.f;
    for (int j = 0; j < k; ++j) {
      const int r = slot_row[(size_t)t * k + j];
      if (r < 0) continue;
      const float wj = w[(size_t)t * k + j];
      float v[VEC];
      load_vec_f<T, VEC>(y + (size_t)r * d + c, v);
#pragma unroll
      for (int q = 0; q < VEC; ++q) acc[q] = __fadd_rn(acc[q], __fmul_rn(wj, v[q]));
    }
    if (shared != nullptr) {
      float v[VEC];
      load_vec_f<T, VEC>(shared + (size_t)t * d + c, v);
#pragma unroll
      for (int q = 0; q < VEC; ++q) acc[q] = __fadd_rn(acc[q], v[q]);
    }
    if constexpr (VEC == 1) {
      out[(size_t)t * d + c] = Num<T>::from_f(acc[0]);
    } else {
      union {
        uint4 u;
        T e[VEC];
      } o;
#pragma unroll
      for (int q = 0; q < VEC; ++q) o.e[q] = Num<T>::from_f(acc[q]);
      *reinterpret_cast<uint4*>(out + (size_t)t * d + c) = o.u;
    }
  }
}

// combine_kernel for 16-byte-aligned rows, one warp per token: the token's k row indices
// and weights are read once (lane j holds slot j) and shared by shuffles, and each lane
// keeps 4 column pieces x 2 slots = 8 16-byte loads in flight.  Same arithmetic, in the
// same order, as combine_kernel: acc = fl(acc + fl(w_j * y_j)) over j, then + shared.
template <typename T, int VEC>
__global__ void __launch_bounds__(256) combine_warp_kernel(const T* __restrict__ y, const int32_t* __restrict__ slot_row,
                                                           const float* __restrict__ w, int T_, int k, int d,
                                                           const T* __restrict__ shared, T* __restrict__ out) {
  pdl_wait_and_release();
  constexpr int U = 4;
  const int lane = threadIdx.x & 31;
  const int nv = d / VEC;                       // 16-byte pieces per row
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < T_; t += warps) {
    const int my_r = lane < k ? slot_row[t * k + lane] : -1;
    const float my_w = lane < k ? w[t * k + lane] : 0.f;
    for (int c0 = lane; c0 < nv; c0 += 32 * U) {
      float acc[U][VEC];
#pragma unroll
      for (int u = 0; u < U; ++u)
#pragma unroll
        for (int q = 0; q < VEC; ++q) acc[u][q] = 0.f;
      for (int j = 0; j < k; j += 2) {
        const int r0 = __shfl_sync(0xffffffffu, my_r, j);
        const int r1 = j + 1 < k ? __shfl_sync(0xffffffffu, my_r, j + 1) : -1;
        const float w0 = __shfl_sync(0xffffffffu, my_w, j);
        const float w1 = __shfl_sync(0xffffffffu, my_w, (j + 1) & 31);
        uint4 v0[U], v1[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int c = c0 + u * 32;
          v0[u] = (r0 >= 0 && c < nv) ? *reinterpret_cast<const uint4*>(y + (int64_t)r0 * d + (int64_t)c * VEC)
                                      : make_uint4(0u, 0u, 0u, 0u);
          v1[u] = (r1 >= 0 && c < nv) ? *reinterpret_cast<const uint4*>(y + (int64_t)r1 * d + (int64_t)c * VEC)
                                      : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const T* e0 = reinterpret_cast<const T*>(&v0[u]);
          const T* e1 = reinterpret_cast<const T*>(&v1[u]);
          if (r0 >= 0) {
#pragma unroll
            for (int q = 0; q < VEC; ++q) acc[u][q] = __fadd_rn(acc[u][q], __fmul_rn(w0, Num<T>::to_f(e0[q])));
          }
          if (r1 >= 0) {
#pragma unroll
            for (int q = 0; q < VEC; ++q) acc[u][q] = __fadd_rn(acc[u][q], __fmul_rn(w1, Num<T>::to_f(e1[q])));
          }
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int c = c0 + u * 32;
        if (c >= nv) continue;
        if (shared != nullptr) {
          const uint4 sv = *reinterpret_cast<const uint4*>(shared + t * d + (int64_t)c * VEC);
          const T* es = reinterpret_cast<const T*>(&sv);
#pragma unroll
          for (int q = 0; q < VEC; ++q) acc[u][q] = __fadd_rn(acc[u][q], Num<T>::to_f(es[q]));
        }
        union {
          uint4 u4;
          T e[VEC];
        } o;
#pragma unroll
        for (int q = 0; q < VEC; ++q) o.e[q] = Num<T>::from_f(acc[u][q]);
        *reinterpret_cast<uint4*>(out + t * d + (int64_t)c * VEC) = o.u4;
      }
    }
  }
}

// The permutation read token by token: x row t is read once and stored to each of its
// k kept rows (slot_row[t*k + j] >= 0).  One warp per token, 16-byte vectors, 8 loads in
// flight per lane.  Writes the same rows as permute_rows_kernel for a plan without
// alignment padding (every row of [0, offsets[E]) is some slot's row).
__global__ void __launch_bounds__(256) permute_tokens_kernel(const unsigned char* __restrict__ x, int64_t row_bytes,
                                                             const int32_t* __restrict__ slot_row, int T_, int k,
                                                             unsigned char* __restrict__ rows) {
  pdl_wait_and_release();
  constexpr int U = 8;
  const int lane = threadIdx.x & 31;
  const int nv = (int)(row_bytes >> 4);
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t t = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < T_; t += warps) {
    const int my_r = lane < k ? slot_row[t * k + lane] : -1;
    const unsigned live = __ballot_sync(0xffffffffu, my_r >= 0);
    if (live == 0) continue;
    const uint4* src = reinterpret_cast<const uint4*>(x + t * row_bytes);
    for (int c0 = lane; c0 < nv; c0 += 32 * U) {
      uint4 v[U];
#pragma unroll
      for (int u = 0; u < U; ++u) v[u] = c0 + u * 32 < nv ? src[c0 + u * 32] : make_uint4(0u, 0u, 0u, 0u);
      for (unsigned m = live; m != 0; m &= m - 1) {
        const int j = __ffs(m) - 1;
        const int r = __shfl_sync(0xffffffffu, my_r, j);
        uint4* dst = reinterpret_cast<uint4*>(rows + (int64_t)r * row_bytes);
#pragma unroll
        for (int u = 0; u < U; ++u)
          if (c0 + u * 32 < nv) dst[c0 + u * 32] = v[u];
      }
    }
  }
}

// dst[r,:] = src[index[r],:] for r < n_rows (zero rows where index is -1).
__global__ void __launch_bounds__(256) gather_rows_kernel(const unsigned char* __restrict__ src, int64_t row_bytes,
                                                          bool vec, const int32_t* __restrict__ index, int64_t n_rows,
                                                          unsigned char* __restrict__ dst) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  for (int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < n_rows; r += warps) {
    const int i = index[r];
    unsigned char* o = dst + r * row_bytes;
    if (vec) {
      const int nv = (int)(row_bytes >> 4);
      uint4* o4 = reinterpret_cast<uint4*>(o);
      if (i >= 0) {
        const uint4* s4 = reinterpret_cast<const uint4*>(src + (int64_t)i * row_bytes);
        for (int j = lane; j < nv; j += 32) o4[j] = s4[j];
      } else {
        for (int j = lane; j < nv; j += 32) o4[j] = make_uint4(0, 0, 0, 0);
      }
    } else {
      const unsigned char* s = src + (int64_t)(i >= 0 ? i : 0) * row_bytes;
      for (int64_t j = lane; j < row_bytes; j += 32) o[j] = i >= 0 ? s[j] : 0;
    }
  }
}

// Block-wide exclusive scan of data[0..n) in shared memory (in place); returns the total
// to every thread.  scratch holds 32 ints.
__device__ int block_exclusive_scan(int* data, int n, int* scratch) {
  const int per = (n + blockDim.x - 1) / blockDim.x;
  const int lo = min(n, (int)threadIdx.x * per), hi = min(n, lo + per);
  int local = 0;
  for (int e = lo; e < hi; ++e) local += data[e];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  __syncthreads();
  if (lane == 31) scratch[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    int v = lane < nw ? scratch[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int u = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v += u;
    }
    if (lane < nw) scratch[lane] = v;
  }
  __syncthreads();
  int run = (incl - local) + (warp > 0 ? scratch[warp - 1] : 0);
  for (int e = lo; e < hi; ++e) {
    const int a = data[e];
    data[e] = run;
    run += a;
  }
  const int total = scratch[(blockDim.x >> 5) - 1];
  __syncthreads();
  return total;
}

// Expert-parallel receive plan, part 1 (one block).  rc is recv_counts [ws][El].
// Writes seg_start[ws*El+1] (receive row where segment (s, le) starts), src_base[ws*El]
// (position inside expert le of the segment's first row), expert counts and offsets.
__global__ void __launch_bounds__(1024) ep_regroup_scan_kernel(const int32_t* __restrict__ rc, int ws, int El,
                                                               int capacity, const int32_t* __restrict__ pos_base,
                                                               int32_t* __restrict__ counts,
                                                               int32_t* __restrict__ offsets,
                                                               int32_t* __restrict__ seg_start,
                                                               int32_t* __restrict__ src_base,
                                                               int32_t* __restrict__ kept_base) {
  extern __shared__ int sh[];  // [El] kept counts, then [ws] row totals
  __shared__ int scratch[32];
  int* s_kept = sh;
  int* s_row = sh + El;
  for (int le = threadIdx.x; le < El; le += blockDim.x) {
    // src_base: global position of the segment's first row (capacity test);
    // kept_base: rows of this call already kept for le before the segment (layout)
    int run = 0, kept = 0;
    for (int s = 0; s < ws; ++s) {
      const int c = rc[s * El + le];
      const int pos = pos_base != nullptr ? pos_base[s * El + le] : run;
      src_base[s * El + le] = pos;
      kept_base[s * El + le] = kept;
      run += c;
      kept += capacity > 0 ? max(0, min(c, capacity - pos)) : c;
    }
    counts[le] = run;
    s_kept[le] = kept;
  }
  for (int s = threadIdx.x; s < ws; s += blockDim.x) {
    int run = 0;
    for (int le = 0; le < El; ++le) {
      seg_start[s * El + le] = run;  // row-local prefix for now
      run += rc[s * El + le];
    }
    s_row[s] = run;
  }
  __syncthreads();
  const int kept_total = block_exclusive_scan(s_kept, El, scratch);
  const int recv_total = block_exclusive_scan(s_row, ws, scratch);
  for (int le = threadIdx.x; le < El; le += blockDim.x) offsets[le] = s_kept[le];
  if (threadIdx.x == 0) {
    offsets[El] = kept_total;
    seg_start[ws * El] = recv_total;
  }
  for (int i = threadIdx.x; i < ws * El; i += blockDim.x) seg_start[i] += s_row[i / El];
}

// Part 2: one thread per received row.
__global__ void __launch_bounds__(256) ep_regroup_rows_kernel(const int32_t* __restrict__ seg_start,
                                                              const int32_t* __restrict__ src_base,
                                                              const int32_t* __restrict__ kept_base,
                                                              const int32_t* __restrict__ offsets, int nseg, int El,
                                                              int capacity, int64_t n_recv,
                                                              int32_t* __restrict__ row_src,
                                                              int32_t* __restrict__ recv_dst) {
  for (int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r < n_recv; r += (int64_t)gridDim.x * blockDim.x) {
    int lo = 0, hi = nseg - 1;  // last segment whose start <= r
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (seg_start[mid] <= r) lo = mid; else hi = mid - 1;
    }
    const int le = lo % El;
    const int i = (int)(r - seg_start[lo]);
    if (capacity > 0 && src_base[lo] + i >= capacity) {
      recv_dst[r] = -1;
    } else {
      const int dst = offsets[le] + kept_base[lo] + i;
      recv_dst[r] = dst;
      row_src[dst] = (int32_t)r;
    }
  }
}

// Expert-parallel return addresses.  seg[0..nsrc] are the first received row of each
// source segment (seg[nsrc] = n_recv); seg[nsrc+1+s] is the address of source s's
// return region.  Received row r goes back to row r - seg[s] of it.
__device__ __forceinline__ uint64_t ep_return_addr(int64_t r, const int64_t* __restrict__ seg, int nsrc,
                                                   int64_t row_bytes) {
  int lo = 0, hi = nsrc - 1;  // last segment whose start <= r
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (seg[mid] <= r) lo = mid; else hi = mid - 1;
  }
  return (uint64_t)seg[nsrc + 1 + lo] + (uint64_t)((r - seg[lo]) * row_bytes);
}

// row_ptrs[i] for every expert row i < rows_cap (0 past the kept rows), and zero rows,
// one warp per row, at the return addresses of received rows the capacity dropped.
// row_src NULL: expert row i is received row i; recv_dst NULL: nothing was dropped.
__global__ void __launch_bounds__(256) ep_return_rows_kernel(const int32_t* __restrict__ row_src,
                                                             const int32_t* __restrict__ offsets, int El,
                                                             const int32_t* __restrict__ recv_dst, int64_t n_recv,
                                                             const int64_t* __restrict__ seg, int nsrc,
                                                             int64_t row_bytes, uint64_t* __restrict__ row_ptrs,
                                                             int64_t rows_cap) {
  const int64_t kept = offsets[El];
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t nth = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = tid; i < rows_cap; i += nth) {
    const int64_t r = i < kept ? (row_src != nullptr ? (int64_t)row_src[i] : i) : -1;
    uint64_t p = (r >= 0 && r < n_recv) ? ep_return_addr(r, seg, nsrc, row_bytes) : 0;
    if (p & 15) {
      set_device_error(kErrBadRowAddress);
      p = 0;
    }
    row_ptrs[i] = p;
  }
  if (recv_dst == nullptr) return;  // nothing dropped
  const int lane = threadIdx.x & 31;
  bool wrote = false;
  for (int64_t r = tid >> 5; r < n_recv; r += nth >> 5) {
    if (recv_dst[r] >= 0) continue;
    const uint64_t p = ep_return_addr(r, seg, nsrc, row_bytes);
    if (p & 15) {
      if (lane == 0) set_device_error(kErrBadRowAddress);
      continue;
    }
    uint4* dst = reinterpret_cast<uint4*>(p);
    for (int64_t j = lane; j < row_bytes / 16; j += 32) dst[j] = make_uint4(0u, 0u, 0u, 0u);
    wrote = true;
  }
  if (wrote) __threadfence_system();  // rows in another GPU's memory: visible before exit
}

// Expert-parallel token dedup.  A token whose k slots go to several experts of one rank
// travels to that rank once.  ridx[t][j] = the destination rank of slot j in this rank's
// rotated order ((e / El - me + ws) % ws, so this rank's own rows come first) for the
// first slot of token t bound for that rank, -1 for its later slots to the same rank;
// a dispatch plan over ridx with ws "experts" then lays out one row per (token, rank).
__global__ void __launch_bounds__(256) ep_dedup_ranks_kernel(const int32_t* __restrict__ idx, int64_t T, int k,
                                                             int El, int ws, int me, int32_t* __restrict__ ridx) {
  const int E = El * ws;
  for (int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; t < T; t += (int64_t)gridDim.x * blockDim.x) {
    const int32_t* it = idx + t * k;
    for (int j = 0; j < k; ++j) {
      const int e = it[j];
      if (e < 0 || e >= E) {
        set_device_error(kErrBadExpertIndex);
        ridx[t * k + j] = -1;
        continue;
      }
      const int r = e / El;
      bool first = true;
      for (int jj = 0; jj < j; ++jj) {
        const int e2 = it[jj];
        if (e2 >= 0 && e2 < E && e2 / El == r) first = false;
      }
      ridx[t * k + j] = first ? (r - me + ws) % ws : -1;
    }
  }
}

// Per sent (token, rank) row p = slot_row[t][j] of a first slot j: the local expert
// (-1 if the slot goes elsewhere) and the gate weight of each of the token's k slots, in
// slot order, for the receiver's expansion and its weighted partial sum.  own_e holds
// the same for this rank's own rows (rows [0, own_count[0]) of the rotated send layout)
// and -1 in rows [own_count[0], T), so that a plan over own_e [T, k] covers exactly them.
__global__ void __launch_bounds__(256) ep_dedup_meta_kernel(const int32_t* __restrict__ idx,
                                                            const float* __restrict__ w,
                                                            const int32_t* __restrict__ ridx,
                                                            const int32_t* __restrict__ slot_row,
                                                            const int32_t* __restrict__ own_count, int64_t T,
                                                            int k, int El, int ws, int32_t* __restrict__ meta_e,
                                                            float* __restrict__ meta_w, int32_t* __restrict__ own_e) {
  const int E = El * ws;
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t nth = (int64_t)gridDim.x * blockDim.x;
  for (int64_t t = tid; t < T; t += nth) {
    const int32_t* it = idx + t * k;
    for (int j = 0; j < k; ++j) {
      const int rr = ridx[t * k + j];
      const int64_t p = slot_row[t * k + j];
      if (rr < 0 || p < 0) continue;
      const int r = it[j] / El;
      for (int jj = 0; jj < k; ++jj) {
        const int e2 = it[jj];
        const bool same = e2 >= 0 && e2 < E && e2 / El == r;
        meta_e[p * k + jj] = same ? e2 % El : -1;
        meta_w[p * k + jj] = same ? w[t * k + jj] : 0.0f;
        if (rr == 0) own_e[p * k + jj] = same ? e2 % El : -1;
      }
    }
  }
  const int64_t own = own_count[0];
  for (int64_t i = own * k + tid; i < T * k; i += nth) own_e[i] = -1;
}

// dst[g][c][r] = src[g][r][c]; 32x32 tiles through shared memory.
template <typename T>
__global__ void __launch_bounds__(256) transpose_batched_kernel(const T* __restrict__ src, T* __restrict__ dst, int R,
                                                                int C) {
  __shared__ T tile[32][33];
  const int g = blockIdx.z;
  const int r0 = blockIdx.y * 32, c0 = blockIdx.x * 32;
  const T* s = src + (size_t)g * R * C;
  T* o = dst + (size_t)g * R * C;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int r = r0 + i, c = c0 + threadIdx.x;
    if (r < R && c < C) tile[i][threadIdx.x] = s[(size_t)r * C + c];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int c = c0 + i, r = r0 + threadIdx.x;
    if (r < R && c < C) o[(size_t)c * R + r] = tile[threadIdx.x][i];
  }
}

}  // namespace smoe
