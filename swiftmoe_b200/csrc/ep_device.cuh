// Expert-parallel exchange laid out on the device: no host round trip per forward.
//
// The reference learns the per-rank counts on the host (`.item()` / `.tolist()`,
// models/ultimate_moe.py:128-137) to size and address its three payload all-to-alls
// (:139-141).  Here every rank all-gathers the per-expert counts of every rank into
// device memory G[ws][E] (NCCL), and
//   * ep_layout_kernel turns G into this rank's addresses: where each of its expert
//     segments lands in the destination's receive buffer (expert-major: local expert,
//     then source rank, then token / slot), the kept prefix of every segment under the
//     capacity cut, the expert offsets of its own receive buffer and the return address
//     of every received segment (the source's return buffer, in the source's send
//     layout);
//   * ep_send_rows_kernel reads each routed row straight from x (by row_token) and
//     stores it into the destination GPU's receive buffer over NVLink (plain 16-byte
//     stores to CUDA-IPC peer memory; no TMA, no multicast);
//   * ep_drop_slots_kernel marks the sender's slots that the capacity cut dropped, so
//     its combine skips them.
// Every rank computes the same G, so all ranks take the same decisions, including the
// overflow guard: if any receive buffer would overflow, nothing is sent or computed
// and the device error word says so.
#pragma once
#include "common.cuh"

namespace smoe {

constexpr int kErrExchangeOverflow = 4;  // a receive buffer of the exchange would overflow
constexpr int kLayoutMaxCells = 8192;    // ws * E handled by the one-block layout kernel

// One block.  G [ws][E] row counts (source rank s -> global expert e, before the cut).
// Outputs:
//   send_addr[E]   byte address in the destination's receive buffer of this rank's first
//                  row for expert e (0 for this rank's own experts and on overflow)
//   keep[E]        rows of this rank's segment for expert e kept by the capacity cut
//   recv_off[El+1] expert offsets of this rank's receive buffer ([El] = rows received)
//   seg[2*El*ws+1] return table of the received segments in (local expert, source) order:
//                  first receive row of each segment, the row total, then the byte
//                  address of each segment's first row in the source's return buffer
//
// rotated != 0 (token dedup: one "expert" per rank, E == ws): every source lays its rows
// out in ITS rotated rank order (its own rank first), G[s][g] counts source s's group g
// = destination (s + g) % ws, and send_addr / keep are written in this rank's rotated
// group order; everything else is in rank order.
__device__ __forceinline__ int layout_count(const int32_t* G, int ws, int E, bool rotated, int s, int e) {
  return rotated ? G[s * E + (e - s + ws) % ws] : G[s * E + e];
}

__global__ void __launch_bounds__(256) ep_layout_kernel(const int32_t* __restrict__ G, int ws, int E, int me,
                                                        int capacity, const uint64_t* __restrict__ recv_base,
                                                        const uint64_t* __restrict__ ret_base, int64_t row_bytes,
                                                        int64_t recv_rows_max, uint64_t* __restrict__ send_addr,
                                                        int32_t* __restrict__ keep, int32_t* __restrict__ recv_off,
                                                        int64_t* __restrict__ seg, int rotated) {
  extern __shared__ int lay_sh[];
  int* Kp = lay_sh;                  // [ws][E] kept rows of each (source, expert) segment
  int* per_exp = Kp + ws * E;        // [E] rows expert e receives from other ranks
  int* eo = per_exp + E;             // [E] start of expert e's region in its owner's buffer
  __shared__ int s_overflow;
  const int El = E / ws;
  const bool rot = rotated != 0 && El == 1;
  if (threadIdx.x == 0) s_overflow = 0;
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    const int owner = e / El;
    int before = 0, recv = 0;
    for (int s = 0; s < ws; ++s) {
      const int c = layout_count(G, ws, E, rot, s, e);
      const int kp = capacity > 0 ? max(0, min(c, capacity - before)) : c;
      Kp[s * E + e] = kp;
      before += c;
      if (s != owner) recv += kp;
    }
    per_exp[e] = recv;
  }
  __syncthreads();
  for (int r = threadIdx.x; r < ws; r += blockDim.x) {   // receive layout of every rank
    int64_t run = 0;
    for (int le = 0; le < El; ++le) {
      eo[r * El + le] = (int)run;
      run += per_exp[r * El + le];
    }
    if (run > recv_rows_max) atomicExch(&s_overflow, 1);
  }
  __syncthreads();
  const bool overflow = s_overflow != 0;
  if (overflow && threadIdx.x == 0) set_device_error(kErrExchangeOverflow);
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    const int owner = e / El;
    int so = 0;                       // rows of lower ranks (other than the owner) before mine
    for (int s = 0; s < me; ++s)
      if (s != owner) so += Kp[s * E + e];
    const int64_t row = (int64_t)eo[e] + so;
    const int o = rot ? (e - me + ws) % ws : e;        // output slot: this rank's send layout order
    send_addr[o] = (owner == me || overflow) ? 0ull : recv_base[owner] + (uint64_t)(row * row_bytes);
    keep[o] = overflow ? 0 : Kp[me * E + e];
  }
  const int nseg = El * ws;
  for (int i = threadIdx.x; i < nseg; i += blockDim.x) {
    const int le = i / ws, s = i % ws;
    const int e = me * El + le;
    int so = 0;
    for (int q = 0; q < s; ++q)
      if (q != me) so += Kp[q * E + e];
    seg[i] = overflow ? 0 : (int64_t)eo[e] + so;
    int64_t src_off = 0;              // the segment's first row in source s's send layout
    const int pos = rot ? (e - s + ws) % ws : e;
    for (int f = 0; f < pos; ++f) src_off += G[s * E + f];
    seg[nseg + 1 + i] = (int64_t)(ret_base[s] + (uint64_t)(src_off * row_bytes));
  }
  for (int le = threadIdx.x; le < El; le += blockDim.x) recv_off[le] = overflow ? 0 : eo[me * El + le];
  if (threadIdx.x == 0) {
    int64_t total = 0;
    for (int le = 0; le < El; ++le) total += per_exp[me * El + le];
    recv_off[El] = overflow ? 0 : (int32_t)total;
    seg[nseg] = overflow ? 0 : total;
  }
}

// Send every routed row of the other ranks' experts: row i of the send layout (plan
// offsets [E+1], rows grouped by global expert) holds x[row_token[i]]; it goes to
// send_addr[e] + p * row_bytes for its expert e and position p in e's segment, when
// p < keep[e].  One warp per row, 16-byte vectors (row_bytes % 16 == 0), four in flight
// per lane.  The last fence makes the peer stores visible before the kernel ends; the
// caller orders the receivers after it (a collective on the same stream).
__global__ void __launch_bounds__(256) ep_send_rows_kernel(const unsigned char* __restrict__ x, int64_t row_bytes,
                                                           const int32_t* __restrict__ row_token,
                                                           const int32_t* __restrict__ offsets, int E, int own_lo,
                                                           int own_hi, const uint64_t* __restrict__ send_addr,
                                                           const int32_t* __restrict__ keep) {
  const int lane = threadIdx.x & 31;
  const int64_t total = offsets[E];
  const int64_t own_a = offsets[own_lo], own_b = offsets[own_hi];
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int nv = (int)(row_bytes >> 4);
  bool wrote = false;
  for (int64_t i = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); i < total; i += warps) {
    if (i >= own_a && i < own_b) continue;     // this rank's own experts stay here
    int lo = 0, hi = E - 1;                    // last expert whose first row <= i
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (offsets[mid] <= i) lo = mid; else hi = mid - 1;
    }
    const int64_t p = i - offsets[lo];
    const uint64_t base = send_addr[lo];
    if (p >= keep[lo] || base == 0) continue;
    const int t = row_token[i];
    if (t < 0) continue;
    const uint4* src = reinterpret_cast<const uint4*>(x + (int64_t)t * row_bytes);
    uint4* dst = reinterpret_cast<uint4*>(base + (uint64_t)(p * row_bytes));
    int j = lane;
    for (; j + 96 < nv; j += 128) {
      const uint4 a = src[j], b = src[j + 32], c = src[j + 64], d = src[j + 96];
      dst[j] = a;
      dst[j + 32] = b;
      dst[j + 64] = c;
      dst[j + 96] = d;
    }
    for (; j < nv; j += 32) dst[j] = src[j];
    wrote = true;
  }
  if (wrote) __threadfence_system();
}

// idx[r][j] = -1 for the received rows r >= *n_rows (their slots hold stale metadata).
__global__ void __launch_bounds__(256) ep_clear_tail_kernel(int32_t* __restrict__ idx, const int32_t* __restrict__ n_rows,
                                                            int64_t rows_cap, int k) {
  const int64_t first = (int64_t)(*n_rows) * k;
  for (int64_t i = first + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < rows_cap * k;
       i += (int64_t)gridDim.x * blockDim.x)
    idx[i] = -1;
}

// Row r of src (r < n_rows) to the address row_ptrs[r] (0: skipped); one warp per row,
// 16-byte vectors (row_bytes % 16 == 0).  The addresses may be in other GPUs' memory.
__global__ void __launch_bounds__(256) store_rows_kernel(const unsigned char* __restrict__ src, int64_t row_bytes,
                                                         const uint64_t* __restrict__ row_ptrs, int64_t n_rows) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int nv = (int)(row_bytes >> 4);
  bool wrote = false;
  for (int64_t r = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < n_rows; r += warps) {
    const uint64_t p = row_ptrs[r];
    if (p == 0 || (p & 15)) continue;
    const uint4* s4 = reinterpret_cast<const uint4*>(src + r * row_bytes);
    uint4* d4 = reinterpret_cast<uint4*>(p);
    for (int j = lane; j < nv; j += 32) d4[j] = s4[j];
    wrote = true;
  }
  if (wrote) __threadfence_system();
}

// dst rows [0, *n_rows) = src rows [0, *n_rows) (n_rows in device memory, <= rows_cap).
__global__ void __launch_bounds__(256) copy_rows_count_kernel(unsigned char* __restrict__ dst,
                                                              const unsigned char* __restrict__ src, int64_t row_bytes,
                                                              const int32_t* __restrict__ n_rows, int64_t rows_cap) {
  const int64_t n = min((int64_t)(*n_rows), rows_cap) * (row_bytes >> 4);
  const uint4* s4 = reinterpret_cast<const uint4*>(src);
  uint4* d4 = reinterpret_cast<uint4*>(dst);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    d4[i] = s4[i];
}

// slot_row[s] = -1 for every slot whose row lies past the kept prefix of its expert's
// segment (keep[e], positions counted from offsets[e]).
__global__ void __launch_bounds__(256) ep_drop_slots_kernel(const int32_t* __restrict__ idx, int64_t n_slots,
                                                            const int32_t* __restrict__ offsets, int E,
                                                            const int32_t* __restrict__ keep,
                                                            int32_t* __restrict__ slot_row) {
  for (int64_t s = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; s < n_slots;
       s += (int64_t)gridDim.x * blockDim.x) {
    const int e = idx[s];
    const int r = slot_row[s];
    if (e < 0 || e >= E || r < 0) continue;
    if (r - offsets[e] >= keep[e]) slot_row[s] = -1;
  }
}

}  // namespace smoe
