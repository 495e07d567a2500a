// Grouped GEMM on the sm_100a 5th-generation tensor cores.
//
// Replaces the reference's per-expert host loop of torch.mm (models/ultimate_moe.py:237-250)
// and the nn.Linear experts (models/baseline_moe.py:151-162) with ONE persistent kernel over
// all experts' tiles:
//   * tiles of 128 rows x 256 accumulator columns, K in steps of 64 (one 128-byte swizzle
//     row of 16-bit elements);
//   * warp 0: one thread issues TMA loads (A rows of the group, B rows of the group's
//     weights through a 3-D tensor map so ragged N never reads the next expert) into a
//     4-stage shared-memory ring guarded by mbarriers;
//   * warp 1: one thread issues tcgen05.mma (M=128, N=256, K=16) into one of two TMEM
//     accumulators (2 x 256 columns = all 512), committing each stage back to the
//     producer and each finished tile to the epilogue;
//   * warps 2-5: read the accumulator with tcgen05.ld, apply the epilogue (plain store,
//     or SwiGLU silu(gate) * up on the fused [gate | up] halves of the tile) and store to
//     global memory while the tensor cores already work on the next tile.
// Every mbarrier wait is bounded (see mbar_wait); on a timeout the kernel records the
// error, drains its in-flight copies and MMAs and frees its TMEM before returning.
#pragma once
#include "common.cuh"

namespace smoe {
namespace tc {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int BN = 256;  // accumulator columns per tile
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;
constexpr int B_BYTES = BN * BK * 2;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int THREADS = 192;
constexpr int MAX_GROUPS = 1024;
constexpr int GM_DEFAULT = 16;  // m-tiles per rasterisation band unless the launch asks otherwise
constexpr int NUM_BARS = 2 * STAGES + 5;
constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + NUM_BARS * 8 + 16 + 3 * (MAX_GROUPS + 1) * 4;
// Internal epilogue kind (not in the C ABI): store 16-bit rows at per-row addresses,
// staged through shared memory so that every warp store writes 128 contiguous bytes
// of 4 rows (expert-parallel return into other GPUs' buffers).
constexpr int EPI_ROWS = 2;
// Public epilogue SMOE_EPI_GATEUP (3): the SwiGLU GEMM's two pre-activations stored
// side by side, C[r, n] = A B1_g^T and C[r, N + n] = A B3_g^T (C is [rows_cap, 2N]);
// the backward pass recomputes them instead of keeping them from the forward.
constexpr int EPI_GATEUP = SMOE_EPI_GATEUP;
template <int EPI> struct EpiTraits {
  static constexpr bool kPair = EPI == SMOE_EPI_SWIGLU || EPI == EPI_GATEUP;  // [gate | up] tiles
};
constexpr int ROWS_STAGE_BYTES = 32 * 128;  // per epilogue warp: 32 rows x 64 16-bit columns
constexpr int SMEM_BYTES_ROWS = SMEM_BYTES + 16 + 4 * ROWS_STAGE_BYTES;
constexpr uint64_t kDrainLimitNs = 200000000ull;  // 200 ms

// Wait used while draining on the way out: ignores the error word, bounded by time.
__device__ __forceinline__ void mbar_wait_drain(uint32_t bar, uint32_t parity) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > kDrainLimitNs) {
      set_device_error(kErrWaitTimeout);
      return;
    }
  }
}

struct TileCoord {
  int g, row0, rows_valid, nb;
};

// Per-launch group table, built by one thread: group g covers rows
// [s_beg[g], s_fin[g]) -- offsets[g] .. (ends ? ends[g] : offsets[g+1]) clamped into
// [0, rows_cap] so that no tile can touch rows outside the buffers whatever the caller
// passed -- and its tiles are numbered from s_ts[g]; s_ts[G] is the total.
template <int BM_>
__device__ __forceinline__ void build_group_table(const int32_t* offsets, const int32_t* ends, int G, int rows_cap,
                                                  int NB, int* s_beg, int* s_fin, int* s_ts) {
  int acc = 0;
  for (int g = 0; g < G; ++g) {
    const int b = min(max(offsets[g], 0), rows_cap);
    const int f = min(max(ends != nullptr ? ends[g] : offsets[g + 1], b), rows_cap);
    s_beg[g] = b;
    s_fin[g] = f;
    s_ts[g] = acc;
    acc += ((f - b + BM_ - 1) / BM_) * NB;
  }
  s_ts[G] = acc;
}

// Tile L -> (group, first row, valid rows, n-block).  Inside a group the tiles are
// rasterised in bands of GM_ m-tiles, m fastest, so concurrently running CTAs share the
// weight tiles of a few n-blocks and the rows of a few m-tiles.  A band as tall as the
// group reads every weight tile from DRAM once, provided the group's rows fit in L2.
template <int BM_>
__device__ __forceinline__ TileCoord decode_tile_t(int L, const int* s_ts, const int* s_beg, const int* s_fin, int G,
                                                   int NB, int GM_) {
  int lo = 0, hi = G - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (s_ts[mid] <= L) lo = mid; else hi = mid - 1;
  }
  TileCoord t;
  t.g = lo;
  const int local = L - s_ts[lo];
  const int rows = s_fin[lo] - s_beg[lo];
  const int mt_g = (rows + BM_ - 1) / BM_;
  const int band = local / (GM_ * NB);
  const int m_first = band * GM_;
  const int gm = min(mt_g - m_first, GM_);
  const int r = local - band * GM_ * NB;
  const int mt = m_first + r % gm;
  t.nb = r / gm;
  t.row0 = s_beg[lo] + mt * BM_;
  t.rows_valid = min(BM_, s_fin[lo] - t.row0);
  return t;
}

template <typename OutT> struct Store;
template <> struct Store<float> {
  // 32 fp32 columns starting at col0 (N % 4 == 0)
  static __device__ __forceinline__ void cols32(float* row, int col0, int N, const uint32_t (&v)[32]) {
#pragma unroll
    for (int j = 0; j < 8; ++j)
      if (col0 + 4 * j < N)
        *reinterpret_cast<uint4*>(row + col0 + 4 * j) = make_uint4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
  }
};
template <typename H> struct Store16 {
  static __device__ __forceinline__ void cols32(H* row, int col0, int N, const float (&f)[32]) {
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (col0 + 8 * j < N) {
        uint4 u;
        u.x = pack2<H>(f[8 * j + 0], f[8 * j + 1]);
        u.y = pack2<H>(f[8 * j + 2], f[8 * j + 3]);
        u.z = pack2<H>(f[8 * j + 4], f[8 * j + 5]);
        u.w = pack2<H>(f[8 * j + 6], f[8 * j + 7]);
        *reinterpret_cast<uint4*>(row + col0 + 8 * j) = u;
      }
  }
};

// Destination of one accumulator row: C + row * ldc, or the address held in row_ptrs
// (for the expert-parallel return, a row of another GPU's buffer); a null address
// skips the row.
template <typename OutT>
__device__ __forceinline__ OutT* out_row(OutT* C, int64_t ldc, const uint64_t* row_ptrs, int row, bool& row_ok) {
  if (!row_ok) return C;
  if (row_ptrs == nullptr) return C + (int64_t)row * ldc;
  const uint64_t p = row_ptrs[row];
  row_ok = p != 0;
  return reinterpret_cast<OutT*>(p);
}

// EPI_ROWS: drain this warp's 32 accumulator rows, 64 columns at a time.  Each thread
// holds one row (tcgen05.ld 32x32b); the 128-byte row pieces go through a
// 4 KB shared-memory stage (16-byte chunks XOR-swizzled by row, conflict-free both
// ways) and leave as warp stores of 4 rows x 128 contiguous bytes.  row_addr: this
// thread's row address (0 = skip the row); the other rows' addresses come by shuffle.
template <typename OutT>
__device__ __forceinline__ void epilogue_rows(uint32_t tbase, uint64_t row_addr, int col0, int N,
                                              unsigned char* stage, int lane) {
#pragma unroll 1
  for (int c = 0; c < BN / 64; ++c) {
    uint32_t v0[32], v1[32];
    tmem_ld32(tbase + c * 64, v0);
    tmem_ld32(tbase + c * 64 + 32, v1);
    tmem_ld_wait();
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t* v = j < 4 ? v0 : v1;
      const int b = (j & 3) * 8;
      uint4 u;
      u.x = pack2<OutT>(__uint_as_float(v[b + 0]), __uint_as_float(v[b + 1]));
      u.y = pack2<OutT>(__uint_as_float(v[b + 2]), __uint_as_float(v[b + 3]));
      u.z = pack2<OutT>(__uint_as_float(v[b + 4]), __uint_as_float(v[b + 5]));
      u.w = pack2<OutT>(__uint_as_float(v[b + 6]), __uint_as_float(v[b + 7]));
      *reinterpret_cast<uint4*>(stage + lane * 128 + ((j ^ (lane & 7)) << 4)) = u;
    }
    __syncwarp();
    const int j = lane & 7;
    const int col = col0 + c * 64 + j * 8;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int row = i * 4 + (lane >> 3);
      const uint64_t dst = __shfl_sync(0xffffffffu, row_addr, row);
      const uint4 u = *reinterpret_cast<const uint4*>(stage + row * 128 + ((j ^ (row & 7)) << 4));
      if (dst != 0 && col < N) *reinterpret_cast<uint4*>(reinterpret_cast<OutT*>(dst) + col) = u;
    }
    __syncwarp();
  }
}

// Drain one 128-row accumulator (this warp's 32 TMEM lanes) into rows of C: SwiGLU on
// the [gate | up] halves, or a plain store of all BN columns.
template <int EPI, typename OutT>
__device__ __forceinline__ void epilogue_tile(uint32_t tbase, OutT* crow, bool row_ok, int col0, int N) {
  if constexpr (EPI == EPI_GATEUP) {
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      uint32_t gv[32], uv[32];
      tmem_ld32(tbase + c * 32, gv);
      tmem_ld32(tbase + 128 + c * 32, uv);
      tmem_ld_wait();
      float g[32], u[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        g[j] = __uint_as_float(gv[j]);
        u[j] = __uint_as_float(uv[j]);
      }
      if (row_ok) {
        Store16<OutT>::cols32(crow, col0 + c * 32, N, g);
        Store16<OutT>::cols32(crow + N, col0 + c * 32, N, u);
      }
    }
  } else if constexpr (EPI == SMOE_EPI_SWIGLU) {
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      uint32_t gv[32], uv[32];
      tmem_ld32(tbase + c * 32, gv);
      tmem_ld32(tbase + 128 + c * 32, uv);
      tmem_ld_wait();
      float h[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float g = __uint_as_float(gv[j]);
        const float u = __uint_as_float(uv[j]);
        h[j] = g / (1.0f + __expf(-g)) * u;
      }
      if (row_ok) {
        if constexpr (sizeof(OutT) == 4) {
          uint32_t hb[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) hb[j] = __float_as_uint(h[j]);
          Store<float>::cols32(reinterpret_cast<float*>(crow), col0 + c * 32, N, hb);
        } else {
          Store16<OutT>::cols32(crow, col0 + c * 32, N, h);
        }
      }
    }
  } else {
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      uint32_t v[32];
      tmem_ld32(tbase + c * 32, v);
      tmem_ld_wait();
      if (row_ok) {
        if constexpr (sizeof(OutT) == 4) {
          Store<float>::cols32(reinterpret_cast<float*>(crow), col0 + c * 32, N, v);
        } else {
          float f[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) f[j] = __uint_as_float(v[j]);
          Store16<OutT>::cols32(crow, col0 + c * 32, N, f);
        }
      }
    }
  }
}

// -------------------------------------------------------------- fp32 on tf32 tensor cores
// An fp32 product a*b on tf32 tensor cores to about fp32 accuracy ("3xTF32"): with
// hi(v) = v rounded to tf32 (10 explicit mantissa bits, to nearest, ties away from zero)
// and lo(v) = v - hi(v) (exact in fp32), a*b = hi(a)hi(b) + hi(a)lo(b) + lo(a)hi(b) up to
// lo(a)lo(b) and the tf32 truncation of the lo terms, both below 2^-21 |a b|.  The three
// products are one tf32 GEMM over a K axis three times as long: every row of A becomes
// [hi | lo | hi] and every weight row [lo | hi | hi], so the two small cross terms are
// accumulated first and hi(a)hi(b) last.  The tensor cores' fp32 accumulation loses up
// to an ulp of the running sum per step, so steps taken while the sum is still small
// (2^-11 of the result) cost almost nothing and the error grows with K/8 steps, not 3K/8.
// This kernel writes those rows (lo_pos = 1 for A, 0 for B); K % 4 == 0, 16-byte aligned
// rows.
__device__ __forceinline__ float tf32_hi(float v) {
  const uint32_t u = __float_as_uint(v);
  if ((u & 0x7f800000u) == 0x7f800000u) return v;  // inf / nan as they are
  return __uint_as_float((u + 0x1000u) & 0xffffe000u);
}

__global__ void tf32_split3_kernel(const float* __restrict__ src, float* __restrict__ dst, int64_t rows, int K,
                                   int lo_pos) {
  pdl_wait();
  const int q = K / 4;  // float4 pieces per row
  const int64_t n = rows * q;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / q;
    const int c = (int)(i - r * q);
    const float4 v = *reinterpret_cast<const float4*>(src + r * K + 4 * c);
    const float4 h = make_float4(tf32_hi(v.x), tf32_hi(v.y), tf32_hi(v.z), tf32_hi(v.w));
    const float4 l = make_float4(v.x - h.x, v.y - h.y, v.z - h.z, v.w - h.w);
    float* row = dst + r * 3 * (int64_t)K + 4 * c;
#pragma unroll
    for (int seg = 0; seg < 3; ++seg) *reinterpret_cast<float4*>(row + seg * (int64_t)K) = seg == lo_pos ? l : h;
  }
}

// ---------------------------------------------------------------------------- split-K
// A launch with few tiles -- decode-sized groups in a large row buffer: the down
// projection of one expert is 16 tiles of 256 columns for 148 SMs -- leaves most SMs idle
// while a few stream the weights.  The kernel decides on the device, from the tile count
// of the group table it builds, whether to cut every tile's K range into ksplit slices
// (at least SPLIT_MIN_KB k-blocks each), one work unit per slice: only when at least
// twice as many scratch units as tiles exist, so each unit still runs on its own CTA.
// A unit stores its fp32 partial tile (valid rows and columns only) into its slot of the
// launch's scratch; the last unit of a tile to finish -- found with the tile's arrival
// counter, which it resets to zero for the next launch -- sums the partials in slice
// order (a fixed order: the result does not depend on which unit finishes last) and
// applies the epilogue.
constexpr int SPLIT_MIN_KB = 4, MAX_SPLIT = 16;

__device__ __forceinline__ int split_count(int tiles, int KB, int units) {
  if (tiles <= 0 || 2 * tiles > units) return 1;
  return max(1, min(min(units / tiles, KB / SPLIT_MIN_KB), MAX_SPLIT));
}

// The four epilogue warps (128 threads) meet on hardware barrier 1.
__device__ __forceinline__ void epi_bar_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// This warp's 32 accumulator rows (one per thread) into the unit's fp32 slot, laid out
// piece-major: the 4-column piece p (columns 4p .. 4p+3) of row r at float (p * BM + r) * 4,
// so the 32 lanes of a warp store 512 contiguous bytes.  Only accumulator columns below
// `valid` (per [gate | up] half for the paired epilogues) are stored.  tcgen05.ld is
// warp-wide, so every lane loads and row_ok masks the stores.
template <bool kPair>
__device__ __forceinline__ void split_store_partial(uint32_t tbase, float* slot, int r, bool row_ok, int valid) {
#pragma unroll 1
  for (int c = 0; c < BN / 32; ++c) {
    const int cc = kPair ? (c * 32) % 128 : c * 32;
    if (cc >= valid) continue;  // warp-uniform
    uint32_t v[32];
    tmem_ld32(tbase + c * 32, v);
    tmem_ld_wait();
    if (row_ok)
#pragma unroll
      for (int j = 0; j < 8; ++j)
        *reinterpret_cast<uint4*>(slot + ((int64_t)(c * 8 + j) * BM + r) * 4) =
            make_uint4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
  }
}

template <typename OutT> __device__ __forceinline__ void store4(OutT* p, float a, float b, float c, float d) {
  *reinterpret_cast<uint2*>(p) = make_uint2(pack2<OutT>(a, b), pack2<OutT>(c, d));
}
template <> __device__ __forceinline__ void store4<float>(float* p, float a, float b, float c, float d) {
  *reinterpret_cast<float4*>(p) = make_float4(a, b, c, d);
}

// The last unit of a tile: partial sums of the ks_n slots starting at tile_ws, in slot
// order (from zero: the first add is exact), then the epilogue; et = this thread's index
// among the 128 epilogue threads.  Consecutive threads take consecutive rows of one
// piece, so the slot reads coalesce; each thread keeps U items x 4 slots of loads in
// flight, since a full tile is 64 items per thread and L2 latency would otherwise
// serialise them.
template <int EPI, typename OutT>
__device__ __forceinline__ void split_fixup(const float* tile_ws, int ks_n, const TileCoord& t, OutT* C, int64_t ldc,
                                            const uint64_t* row_ptrs, int N, int et) {
  constexpr bool kPair = EpiTraits<EPI>::kPair;
  constexpr int U = kPair ? 4 : 8, QB = 4;
  const int col0 = kPair ? t.nb * 128 : t.nb * BN;
  // output pieces of the tile that lie below N (N % 8 == 0: a piece is all in or all out)
  const int np = min((kPair ? 128 : BN) / 4, (N - col0) / 4);
  const int rows = t.rows_valid;
  const int total = np * rows;
  const int64_t slot = (int64_t)BM * BN;
  for (int i0 = et; i0 < total; i0 += 128 * U) {
    float4 a[U], b[U];
    int off[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int i = i0 + u * 128;
      const int p = i / rows, row = i - p * rows;
      off[u] = i < total ? (p * BM + row) * 4 : -1;
      a[u] = b[u] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    for (int q0 = 0; q0 < ks_n; q0 += QB) {
      float4 la[U][QB], lb[U][QB];
#pragma unroll
      for (int u = 0; u < U; ++u)
#pragma unroll
        for (int qq = 0; qq < QB; ++qq)
          if (off[u] >= 0 && q0 + qq < ks_n) {
            const float* pq = tile_ws + (q0 + qq) * slot + off[u];
            la[u][qq] = __ldcg(reinterpret_cast<const float4*>(pq));
            if (kPair) lb[u][qq] = __ldcg(reinterpret_cast<const float4*>(pq + 32 * BM * 4));  // the up piece
          }
#pragma unroll
      for (int u = 0; u < U; ++u)
#pragma unroll
        for (int qq = 0; qq < QB; ++qq)
          if (off[u] >= 0 && q0 + qq < ks_n) {
            a[u].x += la[u][qq].x;
            a[u].y += la[u][qq].y;
            a[u].z += la[u][qq].z;
            a[u].w += la[u][qq].w;
            if (kPair) {
              b[u].x += lb[u][qq].x;
              b[u].y += lb[u][qq].y;
              b[u].z += lb[u][qq].z;
              b[u].w += lb[u][qq].w;
            }
          }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (off[u] < 0) continue;
      const int i = i0 + u * 128;
      const int p = i / rows, row = i - p * rows, c = 4 * p;
      bool ok = true;
      OutT* dst = out_row(C, ldc, row_ptrs, t.row0 + row, ok);
      if (!ok) continue;
      const float4 x = a[u], y = b[u];
      if constexpr (EPI == SMOE_EPI_SWIGLU) {
        store4<OutT>(dst + col0 + c, x.x / (1.0f + __expf(-x.x)) * y.x, x.y / (1.0f + __expf(-x.y)) * y.y,
                     x.z / (1.0f + __expf(-x.z)) * y.z, x.w / (1.0f + __expf(-x.w)) * y.w);
      } else if constexpr (EPI == EPI_GATEUP) {
        store4<OutT>(dst + col0 + c, x.x, x.y, x.z, x.w);
        store4<OutT>(dst + N + col0 + c, y.x, y.y, y.z, y.w);
      } else {
        store4<OutT>(dst + col0 + c, x.x, x.y, x.z, x.w);
      }
    }
  }
}

// EPI: SMOE_EPI_STORE or SMOE_EPI_SWIGLU.  OutT: float, __nv_bfloat16 or __half.
// split_ws / split_cnt: split-K scratch of split_units fp32 [BM, BN] slots and as many
// counters (all zero between launches), or null for no split; a split launch has at most
// split_units tiles x slices, so each of its tiles has a counter.  min_split: at least that
// many K slices per tile (a bound on the length of each accumulation chain), as far as
// the scratch holds them.
// ES: operand element size -- 2 for bf16/fp16 (kind::f16, 64 elements per 128-byte
// swizzle row), 4 for tf32 (fp32 operands, kind::tf32, 32 elements per row); either way a
// k-block is one 128-byte row per operand row and 4 MMAs of 32 bytes of K.
template <int EPI, typename OutT, int ES = 2>
__global__ void __launch_bounds__(THREADS, 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmB3, OutT* __restrict__ C, int64_t ldc, const uint64_t* __restrict__ row_ptrs,
                        const int32_t* __restrict__ offsets, const int32_t* __restrict__ ends, int G, int N,
                        int K, int rows_cap, int gm, uint32_t idesc, float* __restrict__ split_ws,
                        int* __restrict__ split_cnt, int split_units, int min_split) {
  pdl_wait();
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* sA = smem;
  unsigned char* sB = smem + STAGES * A_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sB + STAGES * B_BYTES);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bars + NUM_BARS);
  volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);  // set when a wait gives up
  volatile int* s_last = reinterpret_cast<volatile int*>(s_tmem + 2);   // split-K: 1 last unit, -1 abort
  int* s_beg = reinterpret_cast<int*>(s_tmem + 4);
  int* s_fin = s_beg + (MAX_GROUPS + 1);
  int* s_ts = s_fin + (MAX_GROUPS + 1);
  // EPI_ROWS only (its launches request SMEM_BYTES_ROWS): the epilogue warps' stages
  unsigned char* s_stage =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(s_ts + MAX_GROUPS + 1) + 15) & ~uintptr_t(15));

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  constexpr bool kPair = EpiTraits<EPI>::kPair;
  const int NB = kPair ? (N + 127) / 128 : (N + BN - 1) / BN;
  constexpr int BKE = 128 / ES;  // K elements per k-block
  const int KB = (K + BKE - 1) / BKE;

  auto full_bar = [&](int s) { return smem_u32(bars + s); };
  auto empty_bar = [&](int s) { return smem_u32(bars + STAGES + s); };
  auto tfull_bar = [&](int a) { return smem_u32(bars + 2 * STAGES + a); };
  auto tempty_bar = [&](int a) { return smem_u32(bars + 2 * STAGES + 2 + a); };
  const uint32_t mma_done_bar = smem_u32(bars + 2 * STAGES + 4);

  if (threadIdx.x == 0) {
    *s_abort = 0;
    build_group_table<BM>(offsets, ends, G, rows_cap, NB, s_beg, s_fin, s_ts);
  }
  if (warp == 0 && lane == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), 4);  // one arrive per epilogue warp
    }
    mbar_init(mma_done_bar, 1);
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (kPair) tma_prefetch_desc(&tmB3);
  }
  if (warp == 1) tmem_alloc(smem_u32(s_tmem), 2 * BN);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *s_tmem;
  const int tiles = s_ts[G];
  int ks_n = 1;
  if (split_ws != nullptr && split_cnt != nullptr && tiles > 0) {
    ks_n = max(split_count(tiles, KB, min(split_units, (int)gridDim.x)), min(min_split, KB));
    if ((int64_t)tiles * ks_n > split_units) ks_n = max(1, split_units / tiles);  // never past the scratch
  }
  const int total = tiles * ks_n;  // work units: (tile, K slice), slices of a tile adjacent

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------- TMA producer
      int stage = 0;
      uint32_t phase = 0;
      int64_t issued = 0;
      bool ok = true;
      for (int L = blockIdx.x; L < total && ok; L += gridDim.x) {
        const int tile = L / ks_n, ks = L - tile * ks_n;
        const TileCoord t = decode_tile_t<BM>(tile, s_ts, s_beg, s_fin, G, NB, gm);
        const int n0 = kPair ? t.nb * 128 : t.nb * BN;
        const int kb_lo = ks * KB / ks_n, kb_hi = (ks + 1) * KB / ks_n;
        for (int kb = kb_lo; kb < kb_hi; ++kb) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1, s_abort)) { ok = false; break; }
          const uint32_t fb = full_bar(stage);
          mbar_arrive_expect_tx(fb, STAGE_BYTES);
          const uint32_t a_dst = smem_u32(sA + stage * A_BYTES);
          const uint32_t b_dst = smem_u32(sB + stage * B_BYTES);
          tma_load_2d(a_dst, &tmA, fb, kb * BKE, t.row0);
          tma_load_3d(b_dst, &tmB, fb, kb * BKE, n0, t.g);
          if (kPair) tma_load_3d(b_dst + B_BYTES / 2, &tmB3, fb, kb * BKE, n0, t.g);
          else tma_load_3d(b_dst + B_BYTES / 2, &tmB, fb, kb * BKE, n0 + 128, t.g);
          ++issued;
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      // drain: the last armed phase of every stage must have landed before exit
      for (int s = 0; s < STAGES; ++s) {
        const int64_t cnt = issued / STAGES + (s < issued % STAGES ? 1 : 0);
        if (cnt > 0) mbar_wait_drain(full_bar(s), (uint32_t)((cnt - 1) & 1));
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------- MMA issuer
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int L = blockIdx.x; L < total && ok; L += gridDim.x) {
        const int ks = L % ks_n;
        const int kb_lo = ks * KB / ks_n, kb_hi = (ks + 1) * KB / ks_n;
        if (!mbar_wait(tempty_bar(acc), acc_phase ^ 1, s_abort)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        for (int kb = kb_lo; kb < kb_hi; ++kb) {
          if (!mbar_wait(full_bar(stage), phase, s_abort)) { ok = false; break; }
          tc_fence_after();
          const uint64_t a_desc = umma_desc_sw128(smem_u32(sA + stage * A_BYTES));
          const uint64_t b_desc = umma_desc_sw128(smem_u32(sB + stage * B_BYTES));
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {  // 32 bytes of K each: 16 f16 or 8 tf32 elements
            if constexpr (ES == 4)
              umma_tf32(d_tmem, a_desc + 2 * kk, b_desc + 2 * kk, idesc, (kb != kb_lo || kk != 0) ? 1u : 0u);
            else
              umma_f16(d_tmem, a_desc + 2 * kk, b_desc + 2 * kk, idesc, (kb != kb_lo || kk != 0) ? 1u : 0u);
          }
          umma_commit(empty_bar(stage));
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        umma_commit(tfull_bar(acc));
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
      umma_commit(mma_done_bar);
      mbar_wait_drain(mma_done_bar, 0);
    }
  } else {
    // --------------------------------------------------------------- epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int r = q * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int L = blockIdx.x; L < total; L += gridDim.x) {
      const int tile = L / ks_n;
      const TileCoord t = decode_tile_t<BM>(tile, s_ts, s_beg, s_fin, G, NB, gm);
      bool row_ok = r < t.rows_valid;
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN);
      const int col0 = kPair ? t.nb * 128 : t.nb * BN;
      if (ks_n > 1) {
        // every epilogue warp reaches both barriers of every unit, whether its wait
        // succeeded or not, and leaves the loop on the decision published between them
        if (mbar_wait(tfull_bar(acc), acc_phase, s_abort)) {
          tc_fence_after();
          split_store_partial<kPair>(tbase, split_ws + (int64_t)L * BM * BN, r, row_ok, N - col0);
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(tempty_bar(acc));
        }
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
        __threadfence();
        epi_bar_sync();
        if (threadIdx.x == 64) {
          int last = -1;
          if (!*s_abort) {
            last = atomicAdd(split_cnt + tile, 1) == ks_n - 1 ? 1 : 0;
            if (last) split_cnt[tile] = 0;
          }
          *s_last = last;
        }
        epi_bar_sync();
        const int last = *s_last;
        if (last < 0) break;
        if (last) {
          __threadfence();
          split_fixup<EPI, OutT>(split_ws + (int64_t)tile * ks_n * BM * BN, ks_n, t, C, ldc, row_ptrs, N,
                                 (int)threadIdx.x - 64);
        }
        continue;
      }
      if (!mbar_wait(tfull_bar(acc), acc_phase, s_abort)) break;
      tc_fence_after();
      if constexpr (EPI == EPI_ROWS) {
        const uint64_t addr = row_ok ? row_ptrs[t.row0 + r] : 0;
        epilogue_rows<OutT>(tbase, addr, col0, N, s_stage + q * ROWS_STAGE_BYTES, lane);
      } else {
        OutT* crow = out_row(C, ldc, row_ptrs, t.row0 + r, row_ok);
        epilogue_tile<EPI, OutT>(tbase, crow, row_ok, col0, N);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty_bar(acc));
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
    if (row_ptrs) __threadfence_system();  // rows in another GPU's memory: visible before exit
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 2 * BN);
  }
}

// ============================================================================ K-grouped GEMM
// Weight gradients of the grouped GEMMs: for every group g,
//   C[g][m][n] = sum over k in [koff[g], koff[g+1]) of A[m][k] * B[n][k],
// where A [M, Ktot] and B [N, Ktot] are K-major (the transposed routed rows: K runs over
// the rows of all groups, grouped by expert).  Same pipeline as grouped_gemm_kernel
// (TMA producer, single-thread tcgen05.mma issuer, double-buffered TMEM accumulators,
// four epilogue warps); the tiles are 128 (M) x 256 (N) of one group, n fastest within
// an m-tile, so a group's B rows (its K range of B) stay in L2 while the A rows stream
// once.  Group starts must be multiples of BK (the dispatch plan's row_align 64): the
// K tiles of a group then never reach into the next group, and every TMA K coordinate is
// 16-byte aligned.  A start that is not is rounded down (wrong sums, no fault) and
// reported in the device error word.  A group without rows gets zeros.
// Tile L -> (group, m0, n0).  n_fast: the n-tiles of one m-tile run back to back, so a
// group's B rows stay in L2 while A streams once (B the smaller operand); otherwise the
// m-tiles of one n-tile do, keeping A resident instead.
constexpr uint32_t kMnBox = 64 * BK * 2;  // one 64 x 64 MN-major box: 8 KB

__device__ __forceinline__ void wgrad_tile(int L, int MT, int NB, bool n_fast, int& g, int& m0, int& n0) {
  const int per = MT * NB;
  g = L / per;
  const int local = L - g * per;
  if (n_fast) {
    m0 = (local / NB) * BM;
    n0 = (local % NB) * BN;
  } else {
    m0 = (local % MT) * BM;
    n0 = (local / MT) * BN;
  }
}

// fp32 tile rows through a 4 KB shared-memory stage per epilogue warp: each thread
// holds one accumulator row (tcgen05.ld 32x32b), 32 columns (128 bytes) at a time; the
// 16-byte pieces are XOR-swizzled by row in the stage and leave as warp stores of 4 rows
// x 128 contiguous bytes.  Rows at or past M and columns at or past N are not written;
// zero: store zeros instead of reading the accumulator (a group without rows).
__device__ __forceinline__ void epilogue_f32_staged(uint32_t tbase, float* __restrict__ C, int64_t row_base, int M,
                                                    int N, int m0_warp, int n0, unsigned char* stage, int lane,
                                                    bool zero) {
#pragma unroll 1
  for (int c = 0; c < BN / 32; ++c) {
    uint32_t v[32];
    if (zero) {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = 0u;
    } else {
      tmem_ld32(tbase + c * 32, v);
      tmem_ld_wait();
    }
#pragma unroll
    for (int j = 0; j < 8; ++j)
      *reinterpret_cast<uint4*>(stage + lane * 128 + ((j ^ (lane & 7)) << 4)) =
          make_uint4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
    __syncwarp();
    const int j = lane & 7;
    const int col = n0 + c * 32 + j * 4;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int rr = i * 4 + (lane >> 3);
      const int row = m0_warp + rr;
      const uint4 u = *reinterpret_cast<const uint4*>(stage + rr * 128 + ((j ^ (rr & 7)) << 4));
      if (row < M && col < N) *reinterpret_cast<uint4*>(C + (row_base + row) * (int64_t)N + col) = u;
    }
    __syncwarp();
  }
}

// MN = true: A and B are given as rows of K ([K, M] and [K, N], M / N contiguous: the
// routed rows as they are) and are read as MN-major tiles -- TMA boxes of 64 MN-elements x
// 64 K-rows, two for the 128 A columns and four for the 256 B columns of a tile, each box
// one 8 KB region of 8 swizzle atoms along K -- instead of K-major boxes of transposed
// copies.  MN = false: A [M, K] and B [N, K], K-major.
template <typename OutT, bool MN>
__global__ void __launch_bounds__(THREADS, 1)
    wgrad_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      OutT* __restrict__ C, const int32_t* __restrict__ koff, int G, int M, int N, uint32_t idesc,
                      bool n_fast) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* sA = smem;
  unsigned char* sB = smem + STAGES * A_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sB + STAGES * B_BYTES);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bars + NUM_BARS);
  volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);
  int* s_kb0 = reinterpret_cast<int*>(s_tmem + 4);  // first K tile of each group
  int* s_kb1 = s_kb0 + (MAX_GROUPS + 1);            // end K tile of each group
  // the epilogue warps' output stages (the launch requests SMEM_BYTES_ROWS)
  unsigned char* s_stage =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(s_kb1 + 2 * (MAX_GROUPS + 1)) + 15) & ~uintptr_t(15));

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int MT = (M + BM - 1) / BM;
  const int NB = (N + BN - 1) / BN;
  const int total = G * MT * NB;

  auto full_bar = [&](int s) { return smem_u32(bars + s); };
  auto empty_bar = [&](int s) { return smem_u32(bars + STAGES + s); };
  auto tfull_bar = [&](int a) { return smem_u32(bars + 2 * STAGES + a); };
  auto tempty_bar = [&](int a) { return smem_u32(bars + 2 * STAGES + 2 + a); };
  const uint32_t mma_done_bar = smem_u32(bars + 2 * STAGES + 4);

  if (threadIdx.x == 0) {
    *s_abort = 0;
    bool misaligned = false;
    for (int g = 0; g < G; ++g) {
      const int a = max(koff[g], 0), b = max(koff[g + 1], a);
      misaligned |= (a % BK) != 0;
      s_kb0[g] = a / BK;                    // rounded down: a K coordinate stays aligned
      s_kb1[g] = (b + BK - 1) / BK;
    }
    if (misaligned) set_device_error(kErrBadGroupStart);
  }
  if (warp == 0 && lane == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), 4);
    }
    mbar_init(mma_done_bar, 1);
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) tmem_alloc(smem_u32(s_tmem), 2 * BN);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *s_tmem;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------- TMA producer
      int stage = 0;
      uint32_t phase = 0;
      int64_t issued = 0;
      bool ok = true;
      for (int L = blockIdx.x; L < total && ok; L += gridDim.x) {
        int g, m0, n0;
        wgrad_tile(L, MT, NB, n_fast, g, m0, n0);
        for (int kb = s_kb0[g]; kb < s_kb1[g]; ++kb) {
          if (!mbar_wait(empty_bar(stage), phase ^ 1, s_abort)) { ok = false; break; }
          const uint32_t fb = full_bar(stage);
          mbar_arrive_expect_tx(fb, STAGE_BYTES);
          const uint32_t a_dst = smem_u32(sA + stage * A_BYTES);
          const uint32_t b_dst = smem_u32(sB + stage * B_BYTES);
          if constexpr (MN) {
            tma_load_2d(a_dst, &tmA, fb, m0, kb * BK);
            tma_load_2d(a_dst + kMnBox, &tmA, fb, m0 + 64, kb * BK);
#pragma unroll
            for (int i = 0; i < 4; ++i) tma_load_2d(b_dst + i * kMnBox, &tmB, fb, n0 + 64 * i, kb * BK);
          } else {
            tma_load_2d(a_dst, &tmA, fb, kb * BK, m0);
            tma_load_2d(b_dst, &tmB, fb, kb * BK, n0);
            tma_load_2d(b_dst + B_BYTES / 2, &tmB, fb, kb * BK, n0 + 128);
          }
          ++issued;
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      for (int s = 0; s < STAGES; ++s) {
        const int64_t cnt = issued / STAGES + (s < issued % STAGES ? 1 : 0);
        if (cnt > 0) mbar_wait_drain(full_bar(s), (uint32_t)((cnt - 1) & 1));
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------- MMA issuer
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int L = blockIdx.x; L < total && ok; L += gridDim.x) {
        int g, m0, n0;
        wgrad_tile(L, MT, NB, n_fast, g, m0, n0);
        const int kb0 = s_kb0[g], kb1 = s_kb1[g];
        if (kb1 <= kb0) continue;           // no rows: the epilogue writes zeros
        if (!mbar_wait(tempty_bar(acc), acc_phase ^ 1, s_abort)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(full_bar(stage), phase, s_abort)) { ok = false; break; }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            uint64_t a_desc, b_desc;
            if constexpr (MN) {   // K step of 16 rows = two 1 KB atoms along K
              a_desc = umma_desc_mn_sw128(smem_u32(sA + stage * A_BYTES) + kk * 2048, kMnBox, 1024);
              b_desc = umma_desc_mn_sw128(smem_u32(sB + stage * B_BYTES) + kk * 2048, kMnBox, 1024);
            } else {              // K step of 16 elements = 32 bytes inside the 128-byte rows
              a_desc = umma_desc_sw128(smem_u32(sA + stage * A_BYTES)) + 2 * kk;
              b_desc = umma_desc_sw128(smem_u32(sB + stage * B_BYTES)) + 2 * kk;
            }
            umma_f16(d_tmem, a_desc, b_desc, idesc, (kb > kb0 || kk != 0) ? 1u : 0u);
          }
          umma_commit(empty_bar(stage));
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        umma_commit(tfull_bar(acc));
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
      umma_commit(mma_done_bar);
      mbar_wait_drain(mma_done_bar, 0);
    }
  } else {
    // --------------------------------------------------------------- epilogue
    static_assert(sizeof(OutT) == 4, "the weight gradients are stored in fp32");
    const int q = warp & 3;
    unsigned char* stage = s_stage + q * ROWS_STAGE_BYTES;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int L = blockIdx.x; L < total; L += gridDim.x) {
      int g, m0, n0;
      wgrad_tile(L, MT, NB, n_fast, g, m0, n0);
      const uint32_t tq = tmem_base + ((uint32_t)(q * 32) << 16);
      if (s_kb1[g] <= s_kb0[g]) {           // empty group: zero tile, no accumulator used
        epilogue_f32_staged(tq, reinterpret_cast<float*>(C), (int64_t)g * M, M, N, m0 + q * 32, n0, stage, lane,
                            true);
        continue;
      }
      if (!mbar_wait(tfull_bar(acc), acc_phase, s_abort)) break;
      tc_fence_after();
      const uint32_t tbase = tq + (uint32_t)(acc * BN);
      epilogue_f32_staged(tbase, reinterpret_cast<float*>(C), (int64_t)g * M, M, N, m0 + q * 32, n0, stage, lane,
                          false);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty_bar(acc));
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 2 * BN);
  }
}

// ============================================================================ CTA pairs
// The same grouped GEMM on pairs of CTAs (a cluster of 2 on neighbouring SMs) issuing
// tcgen05.mma.cta_group::2: one 256 x 256 tile per pair, M split across the two CTAs
// (128 rows each, accumulated in each CTA's own TMEM) and the B operand split along N
// (each CTA stages 128 of the 256 weight rows).  Per FLOP every SM moves a third less
// data from L2 into shared memory than the single-CTA kernel, and the 32 KB stages
// allow a 6-deep ring.  The even CTA issues the MMAs; each CTA's TMA loads count their
// bytes on the even CTA's "full" barrier; the MMA thread's commits arrive on the
// "empty" / "accumulator full" barriers of both CTAs; both CTAs' epilogue warps arrive
// on the even CTA's "accumulator empty" barrier.
namespace pair {
constexpr int BM = 256;  // rows per pair tile
constexpr int BMC = 128; // rows per CTA
constexpr int STAGES = 6;
constexpr int A_BYTES = BMC * BK * 2;
constexpr int B_BYTES = (BN / 2) * BK * 2;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int PAIR_STAGE_BYTES = 2 * STAGE_BYTES;
constexpr int NUM_BARS = 2 * STAGES + 5;
constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + NUM_BARS * 8 + 16 + 3 * (MAX_GROUPS + 1) * 4;
}  // namespace pair

__device__ __forceinline__ void mbar_wait_drain_cluster(uint32_t bar, uint32_t parity) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait_cluster(bar, parity)) {
    if (globaltimer_ns() - t0 > kDrainLimitNs) {
      set_device_error(kErrWaitTimeout);
      return;
    }
  }
}

template <int EPI, typename OutT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(THREADS, 1)
    grouped_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                             const __grid_constant__ CUtensorMap tmB3, OutT* __restrict__ C, int64_t ldc, const uint64_t* __restrict__ row_ptrs,
                             const int32_t* __restrict__ offsets, const int32_t* __restrict__ ends, int G, int N,
                             int K, int rows_cap, int gm, uint32_t idesc) {
  constexpr int BM = pair::BM, BMC = pair::BMC, STAGES = pair::STAGES;
  constexpr int A_BYTES = pair::A_BYTES, B_BYTES = pair::B_BYTES, NUM_BARS = pair::NUM_BARS;
  constexpr int PAIR_STAGE_BYTES = pair::PAIR_STAGE_BYTES;
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char* sA = smem;
  unsigned char* sB = smem + STAGES * A_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sB + STAGES * B_BYTES);
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bars + NUM_BARS);
  volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);
  int* s_beg = reinterpret_cast<int*>(s_tmem + 4);
  int* s_fin = s_beg + (MAX_GROUPS + 1);
  int* s_ts = s_fin + (MAX_GROUPS + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();  // 0: issues the MMAs for the pair
  const int pair_id = blockIdx.x >> 1;
  const int npairs = gridDim.x >> 1;
  const int NB = (EPI == SMOE_EPI_SWIGLU) ? (N + 127) / 128 : (N + BN - 1) / BN;
  const int KB = (K + BK - 1) / BK;

  auto full_bar = [&](int s) { return smem_u32(bars + s); };
  auto empty_bar = [&](int s) { return smem_u32(bars + STAGES + s); };
  auto tfull_bar = [&](int a) { return smem_u32(bars + 2 * STAGES + a); };
  auto tempty_bar = [&](int a) { return smem_u32(bars + 2 * STAGES + 2 + a); };
  const uint32_t mma_done_bar = smem_u32(bars + 2 * STAGES + 4);

  if (threadIdx.x == 0) {
    *s_abort = 0;
    build_group_table<BM>(offsets, ends, G, rows_cap, NB, s_beg, s_fin, s_ts);
  }
  if (warp == 0 && lane == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(tfull_bar(a), 1);
      mbar_init(tempty_bar(a), 8);  // four epilogue warps in each CTA of the pair
    }
    mbar_init(mma_done_bar, 1);
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
    if (EPI == SMOE_EPI_SWIGLU) tma_prefetch_desc(&tmB3);
  }
  if (warp == 1) tmem_alloc_pair(smem_u32(s_tmem), 2 * BN);
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers exist before any cross-CTA arrive
  tc_fence_after();
  const uint32_t tmem_base = *s_tmem;
  const int total = s_ts[G];

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------- TMA producer
      int stage = 0;
      uint32_t phase = 0;
      int64_t issued = 0;
      bool ok = true;
      for (int L = pair_id; L < total && ok; L += npairs) {
        const TileCoord t = decode_tile_t<BM>(L, s_ts, s_beg, s_fin, G, NB, gm);
        const int a_row = t.row0 + (int)rank * BMC;
        const int n0 = (EPI == SMOE_EPI_SWIGLU) ? t.nb * 128 : t.nb * BN + (int)rank * 128;
        const void* bmap = (EPI == SMOE_EPI_SWIGLU && rank == 1) ? (const void*)&tmB3 : (const void*)&tmB;
        for (int kb = 0; kb < KB; ++kb) {
          if (!mbar_wait_cluster(empty_bar(stage), phase ^ 1, s_abort)) { ok = false; break; }
          if (rank == 0) mbar_arrive_expect_tx(full_bar(stage), PAIR_STAGE_BYTES);
          const uint32_t fb = mapa_shared(full_bar(stage), 0);
          tma_load_2d_pair(smem_u32(sA + stage * A_BYTES), &tmA, fb, kb * BK, a_row);
          tma_load_3d_pair(smem_u32(sB + stage * B_BYTES), bmap, fb, kb * BK, n0, t.g);
          ++issued;
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      // drain: every issued stage must have been consumed (its loads landed) before exit
      for (int s = 0; s < STAGES; ++s) {
        const int64_t cnt = issued / STAGES + (s < issued % STAGES ? 1 : 0);
        if (cnt > 0) mbar_wait_drain_cluster(empty_bar(s), (uint32_t)((cnt - 1) & 1));
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      // ------------------------------------------------------------- MMA issuer (even CTA)
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int L = pair_id; L < total && ok; L += npairs) {
        if (!mbar_wait_cluster(tempty_bar(acc), acc_phase ^ 1, s_abort)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        for (int kb = 0; kb < KB; ++kb) {
          if (!mbar_wait_cluster(full_bar(stage), phase, s_abort)) { ok = false; break; }
          tc_fence_after();
          const uint64_t a_desc = umma_desc_sw128(smem_u32(sA + stage * A_BYTES));
          const uint64_t b_desc = umma_desc_sw128(smem_u32(sB + stage * B_BYTES));
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk)
            umma_f16_pair(d_tmem, a_desc + 2 * kk, b_desc + 2 * kk, idesc, (kb | kk) != 0 ? 1u : 0u);
          umma_commit_pair(mapa_shared(empty_bar(stage), 0));
          umma_commit_pair(mapa_shared(empty_bar(stage), 1));
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        umma_commit_pair(mapa_shared(tfull_bar(acc), 0));
        umma_commit_pair(mapa_shared(tfull_bar(acc), 1));
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
      umma_commit_pair(mapa_shared(mma_done_bar, 0));
      mbar_wait_drain_cluster(mma_done_bar, 0);
    }
  } else {
    // --------------------------------------------------------------- epilogue (both CTAs)
    const int q = warp & 3;
    const int r = q * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int L = pair_id; L < total; L += npairs) {
      const TileCoord t = decode_tile_t<BM>(L, s_ts, s_beg, s_fin, G, NB, gm);
      if (!mbar_wait_cluster(tfull_bar(acc), acc_phase, s_abort)) break;
      tc_fence_after();
      const int row_base = t.row0 + (int)rank * BMC;
      const int rows_valid = min(BMC, t.rows_valid - (int)rank * BMC);
      bool row_ok = r < rows_valid;
      OutT* crow = out_row(C, ldc, row_ptrs, row_base + r, row_ok);
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN);
      const int col0 = (EPI == SMOE_EPI_SWIGLU) ? t.nb * 128 : t.nb * BN;
      epilogue_tile<EPI, OutT>(tbase, crow, row_ok, col0, N);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(mapa_shared(tempty_bar(acc), 0));
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
    if (row_ptrs) __threadfence_system();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // the pair's MMAs into this CTA's TMEM are complete
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, 2 * BN);
  }
}

}  // namespace tc
}  // namespace smoe
