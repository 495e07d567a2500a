// Layer backward (SwiGLU experts, post-weighting): the element-wise and routing pieces
// between the grouped GEMMs.  The reference is forward-only; the gradients are those of
// its forward (models/baseline_moe.py:56-189 with SwiGLU experts):
//   out_t = sum_j w_tj * y_tj (+ shared(x_t)),  y = W2 (silu(W1 x) * (W3 x)),
//   w_t = softmax of the k selected logits, logits = x Wg^T (+ offsets).
// Routed rows r carry one (token, slot); a = W1 x_r, b = W3 x_r, h = silu(a) * b,
// g_r = W2^T dout_t (the gradient reaching h before the gate weight w_r):
//   dh = w_r g_r,  da = dh * b * silu'(a),  db = dh * silu(a),  dw_r = <g_r, h>,
//   dW2 += dout_t^T (w_r h),  dW1 += da^T x_r,  dW3 += db^T x_r,  dx_t += W1^T da + W3^T db;
// router: dsel_tj = w_tj (dw_tj - sum_j' w_tj' dw_tj') on the selected logits (dw = 0 for
// slots the capacity cut dropped), dx_t += sum_j dsel_tj Wg[e_tj], dWg[e] += dsel x_t.
#pragma once
#include "common.cuh"

namespace smoe {

// row_w[slot_row[s]] = w[s] for every kept slot; rows without a slot keep their value
// (the caller zeroes them first).
__global__ void __launch_bounds__(256) slot_weights_to_rows_kernel(const int32_t* __restrict__ slot_row,
                                                                   const float* __restrict__ w, int64_t n_slots,
                                                                   float* __restrict__ row_w) {
  for (int64_t s = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; s < n_slots; s += (int64_t)gridDim.x * blockDim.x) {
    const int r = slot_row[s];
    if (r >= 0) row_w[r] = w[s];
  }
}

// One block per row r < *n_rows (device count; rows_cap bounds the grid): in place,
//   ab[r] = [a | b] -> [da | db],   g[r] -> w_r * h,   dw_row[r] = sum_f g * h (fp32).
// row_w == NULL means w_r = 1 (the shared expert); dw_row may be NULL.  F % 8 == 0.
template <typename T>
__global__ void __launch_bounds__(256) swiglu_bwd_kernel(T* __restrict__ ab, T* __restrict__ g,
                                                         const float* __restrict__ row_w,
                                                         const int32_t* __restrict__ n_rows, int64_t rows_cap,
                                                         int F, float* __restrict__ dw_row) {
  __shared__ float red[8];
  const int64_t rows = n_rows != nullptr ? ((int64_t)*n_rows < rows_cap ? (int64_t)*n_rows : rows_cap) : rows_cap;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float wr = row_w != nullptr ? row_w[r] : 1.0f;
    T* pa = ab + r * 2 * (int64_t)F;
    T* pb = pa + F;
    T* pg = g + r * (int64_t)F;
    float dw = 0.f;
    for (int f = threadIdx.x * 8; f < F; f += blockDim.x * 8) {
      float a[8], b[8], gg[8];
      load_vec_f<T, 8>(pa + f, a);
      load_vec_f<T, 8>(pb + f, b);
      load_vec_f<T, 8>(pg + f, gg);
      union {
        uint4 u;
        T e[8];
      } da, db, hw;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float sg = 1.0f / (1.0f + __expf(-a[i]));
        const float si = a[i] * sg;
        const float h = si * b[i];
        const float dh = wr * gg[i];
        dw = fmaf(gg[i], h, dw);
        da.e[i] = Num<T>::from_f(dh * b[i] * sg * (1.0f + a[i] * (1.0f - sg)));
        db.e[i] = Num<T>::from_f(dh * si);
        hw.e[i] = Num<T>::from_f(wr * h);
      }
      *reinterpret_cast<uint4*>(pa + f) = da.u;
      *reinterpret_cast<uint4*>(pb + f) = db.u;
      *reinterpret_cast<uint4*>(pg + f) = hw.u;
    }
    if (dw_row != nullptr) {
      dw = warp_sum(dw);
      if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = dw;
      __syncthreads();
      if (threadIdx.x == 0) {
        float s = 0.f;
        for (int i = 0; i < (int)(blockDim.x >> 5); ++i) s += red[i];
        dw_row[r] = s;
      }
      __syncthreads();
    }
  }
}

// Linear experts (y = x Wl^T): one block per row r < *n_rows, in place,
//   dw_row[r] = sum_i g[r,i] * x[r,i]   (g = dout_r Wl, so that <g, x> = <dout_r, y_r>),
//   g[r] -> w_r * g[r]   (the input gradient of the row),   dr[r] -> w_r * dr[r]   (dy_r).
template <typename T>
__global__ void __launch_bounds__(256) linear_bwd_kernel(T* __restrict__ g, const T* __restrict__ xr,
                                                         T* __restrict__ dr, const float* __restrict__ row_w,
                                                         const int32_t* __restrict__ n_rows, int64_t rows_cap, int d,
                                                         float* __restrict__ dw_row) {
  __shared__ float red[8];
  const int64_t rows = (int64_t)*n_rows < rows_cap ? (int64_t)*n_rows : rows_cap;
  for (int64_t r = blockIdx.x; r < rows; r += gridDim.x) {
    const float wr = row_w[r];
    T* pg = g + r * (int64_t)d;
    const T* px = xr + r * (int64_t)d;
    T* pd = dr + r * (int64_t)d;
    float dw = 0.f;
    for (int c = threadIdx.x * 8; c < d; c += blockDim.x * 8) {
      float gg[8], xx[8], dd[8];
      load_vec_f<T, 8>(pg + c, gg);
      load_vec_f<T, 8>(px + c, xx);
      load_vec_f<T, 8>(pd + c, dd);
      union {
        uint4 u;
        T e[8];
      } og, od;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        dw = fmaf(gg[i], xx[i], dw);
        og.e[i] = Num<T>::from_f(wr * gg[i]);
        od.e[i] = Num<T>::from_f(wr * dd[i]);
      }
      *reinterpret_cast<uint4*>(pg + c) = og.u;
      *reinterpret_cast<uint4*>(pd + c) = od.u;
    }
    dw = warp_sum(dw);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = dw;
    __syncthreads();
    if (threadIdx.x == 0) {
      float s = 0.f;
      for (int i = 0; i < (int)(blockDim.x >> 5); ++i) s += red[i];
      dw_row[r] = s;
    }
    __syncthreads();
  }
}

// dx[t, c] = sum_j dxr[slot_row[t,j], c] (kept slots) + dxs[t, c] (shared expert, may be
// NULL) + sum_j dsel_tj * wg[idx[t,j], c], accumulated in fp32 and rounded once.
// dsel_tj = w_tj (dw_tj - sum_j' w_tj' dw_tj'), dw_tj = dw_row[slot_row[t,j]] (0 when the
// slot was dropped).  The thread that owns column 0 of token t also writes dsel_tj to
// dsel_row[slot_row_full[t,j]] (a plan over every slot, for the gate weight gradient).
template <typename T, int VEC>
__global__ void __launch_bounds__(256) moe_bwd_dx_kernel(const T* __restrict__ dxr, const int32_t* __restrict__ slot_row,
                                                         const int32_t* __restrict__ idx, const float* __restrict__ w,
                                                         const float* __restrict__ dw_row, const T* __restrict__ wg,
                                                         const T* __restrict__ dxs, int T_, int k, int d,
                                                         T* __restrict__ dx, const int32_t* __restrict__ slot_row_full,
                                                         float* __restrict__ dsel_row) {
  const int per_row = d / VEC;
  const int64_t total = (int64_t)T_ * per_row;
  for (int64_t gi = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; gi < total;
       gi += (int64_t)gridDim.x * blockDim.x) {
    const int t = (int)(gi / per_row);
    const int c = (int)(gi - (int64_t)t * per_row) * VEC;
    const int32_t* sr = slot_row + (size_t)t * k;
    const float* wt = w + (size_t)t * k;
    float sdw = 0.f;
    for (int j = 0; j < k; ++j) {
      const float dwj = sr[j] >= 0 ? dw_row[sr[j]] : 0.f;
      sdw = fmaf(wt[j], dwj, sdw);
    }
    float acc[VEC];
#pragma unroll
    for (int q = 0; q < VEC; ++q) acc[q] = 0.f;
    for (int j = 0; j < k; ++j) {
      float v[VEC];
      if (sr[j] >= 0) {
        load_vec_f<T, VEC>(dxr + (size_t)sr[j] * d + c, v);
#pragma unroll
        for (int q = 0; q < VEC; ++q) acc[q] += v[q];
      }
      const float dwj = sr[j] >= 0 ? dw_row[sr[j]] : 0.f;
      const float ds = wt[j] * (dwj - sdw);
      load_vec_f<T, VEC>(wg + (size_t)idx[(size_t)t * k + j] * d + c, v);
#pragma unroll
      for (int q = 0; q < VEC; ++q) acc[q] = fmaf(ds, v[q], acc[q]);
      if (c == 0 && dsel_row != nullptr) {
        const int rf = slot_row_full[(size_t)t * k + j];
        if (rf >= 0) dsel_row[rf] = ds;
      }
    }
    if (dxs != nullptr) {
      float v[VEC];
      load_vec_f<T, VEC>(dxs + (size_t)t * d + c, v);
#pragma unroll
      for (int q = 0; q < VEC; ++q) acc[q] += v[q];
    }
    if constexpr (VEC == 1) {
      dx[(size_t)t * d + c] = Num<T>::from_f(acc[0]);
    } else {
      union {
        uint4 u;
        T e[VEC];
      } o;
#pragma unroll
      for (int q = 0; q < VEC; ++q) o.e[q] = Num<T>::from_f(acc[q]);
      *reinterpret_cast<uint4*>(dx + (size_t)t * d + c) = o.u;
    }
  }
}

// Partial gate-weight gradient: part[z][e][c] = sum over the z-th of gridDim.z slices of
// the rows of expert e in a plan over every slot (offsets [E+1], row_token) of
// dsel_row[r] * x[row_token[r], c], in row order.  Grid: (ceil(d / 256), E, slices);
// router_dwg_reduce_kernel adds the slices in order (deterministic).
template <typename T>
__global__ void __launch_bounds__(256) router_dwg_kernel(const T* __restrict__ x, const int32_t* __restrict__ row_token,
                                                         const int32_t* __restrict__ offsets,
                                                         const float* __restrict__ dsel_row, int d, int E,
                                                         float* __restrict__ part) {
  const int e = blockIdx.y;
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= d) return;
  const int e0 = offsets[e], e1 = offsets[e + 1];
  const int len = (e1 - e0 + (int)gridDim.z - 1) / (int)gridDim.z;
  const int r0 = min(e1, e0 + (int)blockIdx.z * len), r1 = min(e1, r0 + len);
  float* dwg = part + (size_t)blockIdx.z * E * d;
  float acc = 0.f;
  int r = r0;
  for (; r + 4 <= r1; r += 4) {
    const float v0 = Num<T>::to_f(x[(size_t)row_token[r] * d + c]);
    const float v1 = Num<T>::to_f(x[(size_t)row_token[r + 1] * d + c]);
    const float v2 = Num<T>::to_f(x[(size_t)row_token[r + 2] * d + c]);
    const float v3 = Num<T>::to_f(x[(size_t)row_token[r + 3] * d + c]);
    acc = fmaf(dsel_row[r], v0, acc);
    acc = fmaf(dsel_row[r + 1], v1, acc);
    acc = fmaf(dsel_row[r + 2], v2, acc);
    acc = fmaf(dsel_row[r + 3], v3, acc);
  }
  for (; r < r1; ++r) acc = fmaf(dsel_row[r], Num<T>::to_f(x[(size_t)row_token[r] * d + c]), acc);
  dwg[(size_t)e * d + c] = acc;
}

__global__ void __launch_bounds__(256) router_dwg_reduce_kernel(const float* __restrict__ part, int slices,
                                                                int64_t n, float* __restrict__ dwg) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float s = 0.f;
    for (int z = 0; z < slices; ++z) s += part[(size_t)z * n + i];
    dwg[i] = s;
  }
}


}  // namespace smoe
