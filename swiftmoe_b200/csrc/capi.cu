// libswiftmoe.so: the C ABI declared in include/swiftmoe.h.
//
// Single translation unit: the kernels live in the *.cuh files included below so that
// one device-side error word is shared by all of them without relocatable device code.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <utility>

#include "common.cuh"
#include "dispatch.cuh"
#include "ep_device.cuh"
#include "backward.cuh"
#include "gemm_simt.cuh"
#include "gemv.cuh"
#include "gemm_tc.cuh"
#include "router.cuh"

using namespace smoe;

namespace {

#define SMOE_CK(expr)                                   \
  do {                                                  \
    cudaError_t e_ = (expr);                            \
    if (e_ != cudaSuccess) {                            \
      report_cuda_error(e_, #expr, __FILE__, __LINE__); \
      return SMOE_ERR_CUDA;                             \
    }                                                   \
  } while (0)

void report_cuda_error(cudaError_t e, const char* what, const char* file, int line) {
  if (getenv("SMOE_VERBOSE")) fprintf(stderr, "swiftmoe: %s failed: %s (%s:%d)\n", what, cudaGetErrorString(e), file, line);
}

inline int elt_size(int dtype) {
  switch (dtype) {
    case SMOE_F32: return 4;
    case SMOE_F16:
    case SMOE_BF16: return 2;
    default: return 0;
  }
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }
inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

constexpr int kMaxDevices = 64;

int device_sms() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
  static int cache[kMaxDevices] = {0};
  if (cache[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n > 0 ? n : 148;
  }
  return cache[dev];
}

// Programmatic dependent launch for the layer forward's chain of kernels: while
// smoe_layer_fwd runs a decode-sized batch on this thread, launch_k() gives every launch the
// programmatic-serialization attribute, so a kernel is scheduled while its predecessor
// finishes and waits inside (pdl_wait_and_release) for the predecessor's writes; every
// kernel launched through launch_k calls that wait before its first global access.  Other
// entry points launch the ordinary way.  SMOE_NO_PDL=1 turns it off (for measurements).
thread_local bool t_pdl = false;

bool pdl_enabled() {
  static const bool off = getenv("SMOE_NO_PDL") != nullptr && strcmp(getenv("SMOE_NO_PDL"), "0") != 0;
  return !off;
}

struct PdlScope {
  bool prev;
  explicit PdlScope(bool on) : prev(t_pdl) { t_pdl = on && pdl_enabled(); }
  ~PdlScope() { t_pdl = prev; }
};

template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args&&... args) {
  if (!t_pdl) {
    kernel<<<grid, block, smem, st>>>(std::forward<Args>(args)...);
    return cudaGetLastError();
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Per-device record of the dynamic shared-memory limit already granted to one kernel.
struct SmemGrant {
  int bytes[kMaxDevices] = {0};
};

// Raise (never lower) a kernel's dynamic shared-memory limit on the current device.
template <typename K>
cudaError_t ensure_smem(K kernel, int bytes, SmemGrant* grant) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  if (grant->bytes[dev] >= bytes) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) grant->bytes[dev] = bytes;
  return e;
}

// ------------------------------------------------------------------ tensor maps
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 2-D map over a row-major [rows, K] 16-bit matrix; box = 64 (K) x 128 rows, 128 B swizzle.
bool make_map_2d(CUtensorMap* m, const void* base, CUtensorMapDataType dt, int64_t rows, int64_t K, int es = 2) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)K * es};
  cuuint32_t box[2] = {(cuuint32_t)(128 / es), 128};  // one 128-byte swizzle row of K
  cuuint32_t estr[2] = {1, 1};
  return enc(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 2-D map over the first K columns of a row-major [rows, ld] 16-bit matrix (ld >= K,
// ld * 2 bytes a multiple of 16): columns from K on read as zeros.
bool make_map_2d_ld(CUtensorMap* m, const void* base, CUtensorMapDataType dt, int64_t rows, int64_t K, int64_t ld) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {64, 128};
  cuuint32_t estr[2] = {1, 1};
  return enc(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 2-D map over a row-major [rows, ld] 16-bit matrix whose first `cols` columns are used,
// box = 64 columns x `box_rows` rows, 128 B swizzle (MN-major operand tiles: the columns
// are the M or N elements, the rows the K index).  Rows from `rows` on read as zeros.
bool make_map_2d_box(CUtensorMap* m, const void* base, CUtensorMapDataType dt, int64_t rows, int64_t cols, int64_t ld,
                     int box_rows) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  return enc(m, dt, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 3-D map over [G, N, K] weights; box = one 128-byte row of K (64 16-bit or 32 fp32
// elements) x 128 (N) x 1 group.
bool make_map_3d(CUtensorMap* m, const void* base, CUtensorMapDataType dt, int64_t G, int64_t N, int64_t K,
                 int es = 2) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return false;
  cuuint64_t dims[3] = {(cuuint64_t)K, (cuuint64_t)N, (cuuint64_t)G};
  cuuint64_t strides[2] = {(cuuint64_t)K * es, (cuuint64_t)N * K * es};
  cuuint32_t box[3] = {(cuuint32_t)(128 / es), 128, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  return enc(m, dt, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
             CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

__global__ void fill_two_kernel(int32_t* p, int32_t a, int32_t b) {
  pdl_wait_and_release();
  p[0] = a;
  p[1] = b;
}

// ------------------------------------------------------------------ grouped GEMM
// Raster band height (m-tiles) of the tensor-core GEMMs.  The SwiGLU gate/up GEMM
// (K = d_model, short rows) uses bands of 32 m-tiles: with the Mixtral shape that is a
// whole expert, whose 32 MB of rows stay in L2 while every weight tile is read from DRAM
// once.  The down GEMM (K = d_ff, 3.7 MB per row tile) keeps bands of 16.
// SMOE_RASTER_BAND overrides both (measurements).
int raster_band(int epi) {
  static const char* forced = getenv("SMOE_RASTER_BAND");
  if (forced) {
    const int v = atoi(forced);
    if (v > 0) return v;
  }
  return (epi == SMOE_EPI_SWIGLU || epi == SMOE_EPI_GATEUP) ? 32 : tc::GM_DEFAULT;
}

// Split-K scratch of the tensor-core GEMM (its kernel decides on the device whether to
// split): one per (device, stream), so launches on different streams never share one --
// device_sms() fp32 [BM, BN] slots and as many arrival counters, zero between launches.
// Allocated at the first launch on the stream, in relaxed capture mode so that a stream
// being captured into a CUDA graph may allocate it too; the counters are zeroed on a
// private stream that is never captured.  SMOE_SPLITK=0 turns the split off.
struct SplitScratch {
  float* ws = nullptr;
  int* cnt = nullptr;
  int units = 0;
};
std::mutex g_split_mu;
std::map<std::pair<int, cudaStream_t>, SplitScratch> g_split;

SplitScratch split_scratch(cudaStream_t st) {
  static const bool off = getenv("SMOE_SPLITK") != nullptr && strcmp(getenv("SMOE_SPLITK"), "0") == 0;
  int dev = 0;
  if (off || cudaGetDevice(&dev) != cudaSuccess) return {};
  std::lock_guard<std::mutex> lk(g_split_mu);
  const auto key = std::make_pair(dev, st);
  const auto it = g_split.find(key);
  if (it != g_split.end()) return it->second;
  SplitScratch s;
  s.units = device_sms();
  const size_t ws_bytes = (size_t)s.units * tc::BM * tc::BN * sizeof(float);
  const size_t cnt_bytes = (size_t)s.units * sizeof(int);
  cudaStreamCaptureMode mode = cudaStreamCaptureModeRelaxed;
  cudaThreadExchangeStreamCaptureMode(&mode);
  void* p = nullptr;
  cudaStream_t init = nullptr;
  bool ok = cudaMalloc(&p, ws_bytes + cnt_bytes) == cudaSuccess;
  ok = ok && cudaStreamCreateWithFlags(&init, cudaStreamNonBlocking) == cudaSuccess;
  ok = ok && cudaMemsetAsync(static_cast<char*>(p) + ws_bytes, 0, cnt_bytes, init) == cudaSuccess;
  ok = ok && cudaStreamSynchronize(init) == cudaSuccess;
  if (init) cudaStreamDestroy(init);
  cudaThreadExchangeStreamCaptureMode(&mode);
  if (!ok) {  // no scratch: this stream's launches run unsplit
    if (p) cudaFree(p);
    cudaGetLastError();
    s = SplitScratch{};
  } else {
    s.ws = static_cast<float*>(p);
    s.cnt = reinterpret_cast<int*>(static_cast<char*>(p) + ws_bytes);
  }
  g_split[key] = s;
  return s;
}

// After a device wait gave up, a split launch may have left tile counters part-counted.
void reset_split_counters(int dev) {
  std::lock_guard<std::mutex> lk(g_split_mu);
  for (auto& kv : g_split)
    if (kv.first.first == dev && kv.second.cnt) cudaMemset(kv.second.cnt, 0, (size_t)kv.second.units * sizeof(int));
}

// Scratch of the fp32 GEMMs on tf32 tensor cores (the [hi | lo | hi] rows of A and
// [lo | hi | hi] rows of the weights), one per (device, stream), grown to the largest
// request.  A stream being captured into a CUDA graph never allocates or grows it: that
// call runs on the FFMA kernel instead.  SMOE_FP32_GEMM=simt keeps every fp32 GEMM on
// the FFMA kernel.
struct Tf32Scratch {
  void* p = nullptr;
  size_t bytes = 0;
};
std::mutex g_tf32_mu;
std::map<std::pair<int, cudaStream_t>, Tf32Scratch> g_tf32;

void* tf32_scratch(cudaStream_t st, size_t bytes) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
  std::lock_guard<std::mutex> lk(g_tf32_mu);
  Tf32Scratch& s = g_tf32[std::make_pair(dev, st)];
  if (s.bytes >= bytes) return s.p;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(st, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) return nullptr;
  // relaxed capture mode: another thread may be capturing a graph on another stream
  cudaStreamCaptureMode mode = cudaStreamCaptureModeRelaxed;
  cudaThreadExchangeStreamCaptureMode(&mode);
  if (s.p) {
    cudaFree(s.p);  // waits for the device: no launch still reads the old buffer
    s = Tf32Scratch{};
  }
  void* p = nullptr;
  const bool ok = cudaMalloc(&p, bytes) == cudaSuccess;
  cudaThreadExchangeStreamCaptureMode(&mode);
  if (!ok) {
    cudaGetLastError();
    return nullptr;
  }
  s.p = p;
  s.bytes = bytes;
  return p;
}

// forced: a split-K scratch of the caller's with at least min_split slices per tile;
// otherwise the stream's own (the kernel then splits only launches with few tiles).
template <int EPI, typename OutT, int ES = 2>
int launch_tc(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mb3, void* C, int64_t ldc,
              const uint64_t* row_ptrs, const int32_t* offsets, const int32_t* ends, int G, int64_t rows_cap, int N, int K, uint32_t idesc,
              cudaStream_t st, const SplitScratch* forced = nullptr, int min_split = 1) {
  static SmemGrant done;
  auto kern = tc::grouped_gemm_kernel<EPI, OutT, ES>;
  constexpr int smem = EPI == tc::EPI_ROWS ? tc::SMEM_BYTES_ROWS : tc::SMEM_BYTES;
  SMOE_CK(ensure_smem(kern, smem, &done));
  const SplitScratch sc = forced ? *forced : split_scratch(st);
  SMOE_CK(launch_k(kern, device_sms(), tc::THREADS, smem, st, ma, mb, mb3, reinterpret_cast<OutT*>(C), ldc, row_ptrs, offsets, ends, G, N,
                                                         K, (int)rows_cap, raster_band(EPI), idesc, sc.ws, sc.cnt, sc.units,
                                                         forced ? min_split : 1));
  SMOE_CK(cudaGetLastError());
  return SMOE_OK;
}

template <int EPI, typename OutT>
int launch_tc_pair(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mb3, void* C, int64_t ldc,
                   const uint64_t* row_ptrs, const int32_t* offsets, const int32_t* ends, int G, int64_t rows_cap, int N, int K, uint32_t idesc,
              cudaStream_t st) {
  static SmemGrant done;
  auto kern = tc::grouped_gemm_pair_kernel<EPI, OutT>;
  SMOE_CK(ensure_smem(kern, tc::pair::SMEM_BYTES, &done));
  const int grid = device_sms() & ~1;  // whole CTA pairs
  kern<<<grid, tc::THREADS, tc::pair::SMEM_BYTES, st>>>(ma, mb, mb3, reinterpret_cast<OutT*>(C), ldc, row_ptrs, offsets, ends, G, N,
                                                        K, (int)rows_cap, raster_band(EPI) / 2, idesc);
  SMOE_CK(cudaGetLastError());
  return SMOE_OK;
}

template <bool MN>
int launch_wgrad(const CUtensorMap& ma, const CUtensorMap& mb, float* C, const int32_t* koff, int G, int M, int N,
                 uint32_t idesc, cudaStream_t st) {
  static SmemGrant done;
  auto kern = tc::wgrad_gemm_kernel<float, MN>;
  SMOE_CK(ensure_smem(kern, tc::SMEM_BYTES_ROWS, &done));
  const int64_t tiles = (int64_t)G * cdiv(M, tc::BM) * cdiv(N, tc::BN);
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(tiles, device_sms()));
  // keep the smaller operand (per group: N rows of B against M rows of A) in L2
  kern<<<grid, tc::THREADS, tc::SMEM_BYTES_ROWS, st>>>(ma, mb, C, koff, G, M, N, idesc, N <= M);
  SMOE_CK(cudaGetLastError());
  return SMOE_OK;
}

template <int EPI, typename T, typename OutT>
int launch_gemv_t(const void* A, const void* B, const void* B3, void* C, const uint64_t* row_ptrs,
                  const int32_t* offsets, const int32_t* ends, int G, int64_t rows_cap, int N, int K,
                  cudaStream_t st, const int32_t* a_index, int a_rows) {
  // one warp (two for rows of 8192 or more elements) per (group with rows, column); at
  // most min(G, rows_cap) groups have rows.  Measured on the Mixtral decode shapes: two
  // warps take the 14336-element down rows in 54 us (one: 60, four: 57); the 4096-element
  // gate/up rows stay on one warp (two: 97 us against 84).
  const int64_t cols = std::min<int64_t>(G, std::max<int64_t>(rows_cap, 1)) * N;
  if (K >= 8192) {
    constexpr int CPB = gemv::THREADS / 32 / 2;
    const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>(cdiv(cols, CPB), 65535));
    SMOE_CK(launch_k(gemv::grouped_gemv_kernel<EPI, T, OutT, 2>, grid, gemv::THREADS, 0, st, 
        (const T*)A, (const T*)B, (const T*)B3, (OutT*)C, N, row_ptrs, offsets, ends, G, N, K, (int)rows_cap, a_index,
        a_rows));
  } else {
    const unsigned grid = (unsigned)std::max<int64_t>(
        1, std::min<int64_t>(cdiv(cols * 32, gemv::THREADS), (int64_t)device_sms() * 8));
    SMOE_CK(launch_k(gemv::grouped_gemv_kernel<EPI, T, OutT, 1>, grid, gemv::THREADS, 0, st, 
        (const T*)A, (const T*)B, (const T*)B3, (OutT*)C, N, row_ptrs, offsets, ends, G, N, K, (int)rows_cap, a_index,
        a_rows));
  }
  SMOE_CK(cudaGetLastError());
  return SMOE_OK;
}

int launch_gemv(const void* A, const void* B, const void* B3, void* C, const uint64_t* row_ptrs, int dtype,
                int out_dtype, int epi, const int32_t* offsets, const int32_t* ends, int G, int64_t rows_cap, int N,
                int K, cudaStream_t st, const int32_t* a_index = nullptr, int a_rows = -1) {
  const bool bf = dtype == SMOE_BF16;
  if (a_index == nullptr) a_rows = (int)rows_cap;
  if (epi == SMOE_EPI_SWIGLU)
    return bf ? launch_gemv_t<SMOE_EPI_SWIGLU, __nv_bfloat16, __nv_bfloat16>(A, B, B3, C, row_ptrs, offsets, ends,
                                                                             G, rows_cap, N, K, st, a_index, a_rows)
              : launch_gemv_t<SMOE_EPI_SWIGLU, __half, __half>(A, B, B3, C, row_ptrs, offsets, ends, G, rows_cap, N,
                                                               K, st, a_index, a_rows);
  if (out_dtype == SMOE_F32)
    return bf ? launch_gemv_t<SMOE_EPI_STORE, __nv_bfloat16, float>(A, B, B3, C, row_ptrs, offsets, ends, G,
                                                                    rows_cap, N, K, st, a_index, a_rows)
              : launch_gemv_t<SMOE_EPI_STORE, __half, float>(A, B, B3, C, row_ptrs, offsets, ends, G, rows_cap, N, K,
                                                             st, a_index, a_rows);
  return bf ? launch_gemv_t<SMOE_EPI_STORE, __nv_bfloat16, __nv_bfloat16>(A, B, B3, C, row_ptrs, offsets, ends, G,
                                                                          rows_cap, N, K, st, a_index, a_rows)
            : launch_gemv_t<SMOE_EPI_STORE, __half, __half>(A, B, B3, C, row_ptrs, offsets, ends, G, rows_cap, N, K,
                                                            st, a_index, a_rows);
}

// A 16-bit grouped GEMM that the decode kernels take: at most gemv::DISPATCH_ROWS rows.
bool gemv_eligible(const void* A, const void* B, const void* B3, int dtype, int out_dtype, int epi, int G,
                   int64_t rows_cap, int K) {
  return dtype != SMOE_F32 && epi != SMOE_EPI_GATEUP && rows_cap <= gemv::DISPATCH_ROWS && G <= gemv::MAX_GROUPS &&
         K % 8 == 0 && aligned16(A) && aligned16(B) && (!B3 || aligned16(B3)) &&
         (epi == SMOE_EPI_STORE || out_dtype == dtype) && (out_dtype == SMOE_F32 || out_dtype == dtype);
}

// Which tensor-core kernel runs a grouped GEMM.  Measured on the Mixtral-shaped layer
// (power-capped B200, 16384 tokens): the CTA-pair kernel takes 6.37 ms for the gate/up
// GEMM against 6.03 ms for single CTAs -- the tensor pipe is power-bound, so the
// shared-memory traffic it saves buys no clock, while its 256-row tiles double the
// per-expert tail waste.  Single CTAs are therefore the default; SMOE_GEMM_VARIANT=2sm
// selects the pair kernel (and =1sm the default) for measurements.
bool use_pair_kernel(int64_t rows_cap, int G) {
  static const char* forced = getenv("SMOE_GEMM_VARIANT");
  (void)rows_cap;
  (void)G;
  return forced != nullptr && strcmp(forced, "2sm") == 0;
}

// The fp32 grouped GEMM on tf32 tensor cores (3xTF32, see tc::tf32_split3_kernel):
// SMOE_ERR_WORKSPACE when no scratch could be had (the caller then uses the FFMA kernel).
// b_split: B (and B3) are already the [G, N, 3K] rows [lo | hi | hi] of
// smoe_tf32_split_weights, so only A is split here.
int tf32x3_gemm(const void* A, const void* B, const void* B3, void* C, const uint64_t* row_ptrs, int epi,
                const int32_t* offsets, const int32_t* ends, int G, int64_t rows_cap, int N, int K, cudaStream_t st,
                bool b_split = false) {
  const int64_t K3 = 3 * (int64_t)K;
  const size_t a_el = (size_t)rows_cap * K3, b_el = (size_t)G * N * K3;
  // Accumulation chains of at most kTf32ChainKb k-blocks (48 x 32 tf32 elements of the
  // tripled K): the error of the tensor cores' fp32 accumulation grows with the chain --
  // measured on unit-scale outputs, 2e-6 at 4-6 k-blocks, 5e-6 at 12, 1.0e-5 at 24,
  // 1.7e-5 at 48, 2.9e-5 at 84, 8.6e-5 at 336 -- against the fp32 bar of 1e-5 x the
  // output scale (~4.4e-5 here), so longer K is cut into split-K slices that the last
  // slice sums in fp32, rounding to nearest.
  constexpr int64_t kTf32ChainKb = 48;
  const int min_split = (int)cdiv(cdiv(K3, 32), kTf32ChainKb);
  const int64_t nb = epi == SMOE_EPI_SWIGLU ? cdiv(N, 128) : cdiv(N, tc::BN);
  const int64_t tiles_max = min_split > 1 ? (cdiv(rows_cap, tc::BM) + G) * nb : 0;
  const size_t slot_el = (size_t)tiles_max * min_split * tc::BM * tc::BN;
  if (tiles_max * min_split > INT32_MAX) return SMOE_ERR_WORKSPACE;
  // one counter per slot: the kernel splits only while tiles x slices fit the slots, so
  // every tile index of a split launch has a counter, overlapping row ranges included
  const size_t cnt_bytes = (size_t)tiles_max * min_split * sizeof(int);
  const size_t b_own = b_split ? 0 : b_el * (epi == SMOE_EPI_SWIGLU ? 2 : 1);
  const size_t bytes = (a_el + b_own + slot_el) * sizeof(float) + cnt_bytes;
  float* s = static_cast<float*>(tf32_scratch(st, bytes));
  if (!s) return SMOE_ERR_WORKSPACE;
  float* a3 = s;
  float* b3 = b_split ? static_cast<float*>(const_cast<void*>(B)) : a3 + a_el;
  float* b33 = b_split ? static_cast<float*>(const_cast<void*>(B3)) : b3 + b_el;
  SplitScratch chain;
  if (min_split > 1) {
    chain.ws = a3 + a_el + b_own;
    chain.cnt = reinterpret_cast<int*>(chain.ws + slot_el);
    chain.units = (int)(tiles_max * min_split);
    SMOE_CK(cudaMemsetAsync(chain.cnt, 0, cnt_bytes, st));
  }
  const SplitScratch* forced = min_split > 1 ? &chain : nullptr;
  auto split = [&](const void* src, float* dst, int64_t rows, int lo_pos) {
    const int64_t n = rows * (K / 4);
    const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>(cdiv(n, 256), (int64_t)device_sms() * 16));
    return launch_k(tc::tf32_split3_kernel, grid, 256, 0, st, static_cast<const float*>(src), dst, rows, K, lo_pos);
  };
  SMOE_CK(split(A, a3, rows_cap, 1));  // [hi | lo | hi]
  if (!b_split) {
    SMOE_CK(split(B, b3, (int64_t)G * N, 0));  // [lo | hi | hi]
    if (epi == SMOE_EPI_SWIGLU) SMOE_CK(split(B3, b33, (int64_t)G * N, 0));
  }
  CUtensorMap ma, mb, mb3;
  if (!make_map_2d(&ma, a3, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, rows_cap, K3, 4)) return SMOE_ERR_CUDA;
  if (!make_map_3d(&mb, b3, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, G, N, K3, 4)) return SMOE_ERR_CUDA;
  if (epi == SMOE_EPI_SWIGLU) {
    if (!make_map_3d(&mb3, b33, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, G, N, K3, 4)) return SMOE_ERR_CUDA;
  } else {
    mb3 = mb;
  }
  const uint32_t idesc = umma_idesc_f16(2u, tc::BM, tc::BN);  // a/b format 2: tf32
  if (epi == SMOE_EPI_SWIGLU)
    return launch_tc<SMOE_EPI_SWIGLU, float, 4>(ma, mb, mb3, C, N, row_ptrs, offsets, ends, G, rows_cap, N, (int)K3,
                                                idesc, st, forced, min_split);
  return launch_tc<SMOE_EPI_STORE, float, 4>(ma, mb, mb3, C, N, row_ptrs, offsets, ends, G, rows_cap, N, (int)K3,
                                             idesc, st, forced, min_split);
}

bool tf32x3_enabled() {
  static const bool off = getenv("SMOE_FP32_GEMM") != nullptr && strcmp(getenv("SMOE_FP32_GEMM"), "simt") == 0;
  return !off;
}

// C [rows_cap, N] (ldc = N), or, when row_ptrs is given, output row r at the address
// row_ptrs[r] (null: row skipped) and C unused.
int grouped_gemm_impl(const void* A, const void* B, const void* B3, void* C, int dtype, int out_dtype, int epi,
                      const int32_t* offsets, const int32_t* ends, int G, int64_t rows_cap, int N, int K,
                      cudaStream_t st, const uint64_t* row_ptrs = nullptr, bool b_split = false) {
  if (row_ptrs) C = nullptr;
  if (!A || !B || (!C && !row_ptrs) || !offsets || G < 1 || N < 1 || K < 1 || rows_cap < 0) return SMOE_ERR_INVALID;
  if (epi != SMOE_EPI_STORE && epi != SMOE_EPI_SWIGLU && epi != SMOE_EPI_GATEUP) return SMOE_ERR_INVALID;
  if ((epi == SMOE_EPI_SWIGLU || epi == SMOE_EPI_GATEUP) && !B3) return SMOE_ERR_INVALID;
  if (epi == SMOE_EPI_GATEUP && (row_ptrs || dtype == SMOE_F32 || out_dtype != dtype)) return SMOE_ERR_UNSUPPORTED;
  if (elt_size(dtype) == 0 || elt_size(out_dtype) == 0) return SMOE_ERR_INVALID;
  if (rows_cap == 0) return SMOE_OK;
  if (rows_cap > INT32_MAX) return SMOE_ERR_UNSUPPORTED;
  if (dtype == SMOE_F32) {
    if (out_dtype != SMOE_F32) return SMOE_ERR_UNSUPPORTED;
    // fp32 on the tensor cores where the shapes allow (3xTF32), else FFMA
    const bool tc_ok = tf32x3_enabled() && K % 4 == 0 && N % 8 == 0 && G <= tc::MAX_GROUPS &&
                       (int64_t)3 * K <= INT32_MAX && aligned16(A) && aligned16(B) && (!C || aligned16(C)) &&
                       (!B3 || aligned16(B3));
    if (b_split && !tc_ok) return SMOE_ERR_UNSUPPORTED;  // split weights fit the tensor-core path only
    if (tc_ok) {
      const int rc = tf32x3_gemm(A, B, B3, C, row_ptrs, epi, offsets, ends, G, rows_cap, N, K, st, b_split);
      if (rc != SMOE_ERR_WORKSPACE || b_split) return rc;
    }
    if (G > simt::MAX_GROUPS) return SMOE_ERR_UNSUPPORTED;
    dim3 grid((unsigned)(cdiv(rows_cap, simt::BM) + G), (unsigned)(epi == SMOE_EPI_SWIGLU ? cdiv(N, simt::BN / 2) : cdiv(N, simt::BN)));
    if (epi == SMOE_EPI_SWIGLU)
      SMOE_CK(launch_k(simt::grouped_gemm_f32_kernel<SMOE_EPI_SWIGLU>, grid, simt::THREADS, 0, st, 
          (const float*)A, (const float*)B, (const float*)B3, (float*)C, N, row_ptrs, offsets, ends, G, N, K,
          (int)rows_cap));
    else
      SMOE_CK(launch_k(simt::grouped_gemm_f32_kernel<SMOE_EPI_STORE>, grid, simt::THREADS, 0, st, 
          (const float*)A, (const float*)B, nullptr, (float*)C, N, row_ptrs, offsets, ends, G, N, K, (int)rows_cap));
    SMOE_CK(cudaGetLastError());
    return SMOE_OK;
  }
  // 16-bit inputs: decode-sized batches stream the weights on the SIMT pipes, the rest
  // runs on tensor cores
  if (gemv_eligible(A, B, B3, dtype, out_dtype, epi, G, rows_cap, K))
    return launch_gemv(A, B, B3, C, row_ptrs, dtype, out_dtype, epi, offsets, ends, G, rows_cap, N, K, st);
  if (G > tc::MAX_GROUPS) return SMOE_ERR_UNSUPPORTED;
  if (K % 8 != 0 || N % 8 != 0) return SMOE_ERR_UNSUPPORTED;
  if (!aligned16(A) || !aligned16(B) || (C && !aligned16(C)) || (B3 && !aligned16(B3))) return SMOE_ERR_UNSUPPORTED;
  if (epi == SMOE_EPI_SWIGLU && out_dtype != dtype) return SMOE_ERR_UNSUPPORTED;
  if (out_dtype != SMOE_F32 && out_dtype != dtype) return SMOE_ERR_UNSUPPORTED;
  const CUtensorMapDataType dt = dtype == SMOE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap ma, mb, mb3;
  if (!make_map_2d(&ma, A, dt, rows_cap, K)) return SMOE_ERR_CUDA;
  if (!make_map_3d(&mb, B, dt, G, N, K)) return SMOE_ERR_CUDA;
  if (epi == SMOE_EPI_SWIGLU || epi == SMOE_EPI_GATEUP) {
    if (!make_map_3d(&mb3, B3, dt, G, N, K)) return SMOE_ERR_CUDA;
  } else {
    mb3 = mb;
  }
  if (epi == SMOE_EPI_GATEUP) {  // [gate | up] pre-activations, rows of 2N
    const uint32_t idesc = umma_idesc_f16(dtype == SMOE_BF16 ? 1u : 0u, tc::BM, tc::BN);
    return dtype == SMOE_BF16
               ? launch_tc<tc::EPI_GATEUP, __nv_bfloat16>(ma, mb, mb3, C, 2 * (int64_t)N, nullptr, offsets, ends, G,
                                                          rows_cap, N, K, idesc, st)
               : launch_tc<tc::EPI_GATEUP, __half>(ma, mb, mb3, C, 2 * (int64_t)N, nullptr, offsets, ends, G,
                                                   rows_cap, N, K, idesc, st);
  }
  if (row_ptrs && epi == SMOE_EPI_STORE && out_dtype == dtype) {  // rows staged, 128-byte stores
    const uint32_t idesc = umma_idesc_f16(dtype == SMOE_BF16 ? 1u : 0u, tc::BM, tc::BN);
    return dtype == SMOE_BF16
               ? launch_tc<tc::EPI_ROWS, __nv_bfloat16>(ma, mb, mb3, C, N, row_ptrs, offsets, ends, G, rows_cap, N, K,
                                                        idesc, st)
               : launch_tc<tc::EPI_ROWS, __half>(ma, mb, mb3, C, N, row_ptrs, offsets, ends, G, rows_cap, N, K, idesc,
                                                 st);
  }
  if (use_pair_kernel(rows_cap, G)) {
    const uint32_t idesc2 = umma_idesc_f16(dtype == SMOE_BF16 ? 1u : 0u, tc::pair::BM, tc::BN);
    if (epi == SMOE_EPI_SWIGLU)
      return dtype == SMOE_BF16
                 ? launch_tc_pair<SMOE_EPI_SWIGLU, __nv_bfloat16>(ma, mb, mb3, C, N, row_ptrs, offsets, ends, G, rows_cap, N, K, idesc2, st)
                 : launch_tc_pair<SMOE_EPI_SWIGLU, __half>(ma, mb, mb3, C, N, row_ptrs, offsets, ends, G, rows_cap, N, K, idesc2, st);
    if (out_dtype == SMOE_F32)
      return launch_tc_pair<SMOE_EPI_STORE, float>(ma, mb, mb3, C, N, row_ptrs, offsets, ends, G, rows_cap, N, K, idesc2, st);
    return dtype == SMOE_BF16
               ? launch_tc_pair<SMOE_EPI_STORE, __nv_bfloat16>(ma, mb, mb3, C, N, row_ptrs, offsets, ends, G, rows_cap, N, K, idesc2, st)
               : launch_tc_pair<SMOE_EPI_STORE, __half>(ma, mb, mb3, C, N, row_ptrs, offsets, ends, G, rows_cap, N, K, idesc2, st);
  }
  const uint32_t idesc = umma_idesc_f16(dtype == SMOE_BF16 ? 1u : 0u, tc::BM, tc::BN);
  if (epi == SMOE_EPI_SWIGLU) {
    return dtype == SMOE_BF16 ? launch_tc<SMOE_EPI_SWIGLU, __nv_bfloat16>(ma, mb, mb3, C, N, row_ptrs, offsets, ends, G, rows_cap, N, K, idesc, st)
                              : launch_tc<SMOE_EPI_SWIGLU, __half>(ma, mb, mb3, C, N, row_ptrs, offsets, ends, G, rows_cap, N, K, idesc, st);
  }
  if (out_dtype == SMOE_F32) return launch_tc<SMOE_EPI_STORE, float>(ma, mb, mb3, C, N, row_ptrs, offsets, ends, G, rows_cap, N, K, idesc, st);
  return dtype == SMOE_BF16 ? launch_tc<SMOE_EPI_STORE, __nv_bfloat16>(ma, mb, mb3, C, N, row_ptrs, offsets, ends, G, rows_cap, N, K, idesc, st)
                            : launch_tc<SMOE_EPI_STORE, __half>(ma, mb, mb3, C, N, row_ptrs, offsets, ends, G, rows_cap, N, K, idesc, st);
}

// ------------------------------------------------------------------ router
enum RouterPath { kRouterMma, kRouterSmall, kRouterGemm, kRouterGeneric };

int router_mma_tiles(int E) { return E <= 8 ? 1 : (E <= 16 ? 2 : 4); }

RouterPath router_path(int d, int E, int dtype) {
  if (dtype != SMOE_F32 && E <= 32 && d % 64 == 0) return kRouterMma;
  const size_t smem = (size_t)E * d * elt_size(dtype);
  if (E <= 32 && smem <= 200 * 1024) return kRouterSmall;
  if (dtype == SMOE_F32) return kRouterGemm;
  if (E % 8 == 0 && d % 8 == 0) return kRouterGemm;
  return kRouterGeneric;
}

template <typename T, int EMAX, int TOK, int VEC>
int launch_router_small(const void* x, const void* wg, const float* bias, int T_, int d, int E, int k, int32_t* idx,
                        float* w, float* logits, cudaStream_t st) {
  static SmemGrant done;
  auto kern = router_small_kernel<T, EMAX, TOK, VEC>;
  const int smem = E * d * (int)sizeof(T);
  SMOE_CK(ensure_smem(kern, std::max(smem, 1), &done));
  int per_sm = 1;
  SMOE_CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, 256, smem));
  per_sm = std::max(per_sm, 1);
  const int64_t groups = cdiv(T_, TOK);
  const int64_t want = cdiv(groups, 8);
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(want, (int64_t)device_sms() * per_sm));
  SMOE_CK(launch_k(kern, grid, 256, smem, st, (const T*)x, (const T*)wg, bias, T_, d, E, k, idx, w, logits));
  SMOE_CK(cudaGetLastError());
  return SMOE_OK;
}

template <typename T, int VEC>
int router_small_dispatch_e(const void* x, const void* wg, const float* bias, int T_, int d, int E, int k,
                            int32_t* idx, float* w, float* logits, cudaStream_t st) {
  if (E <= 8) return launch_router_small<T, 8, 4, VEC>(x, wg, bias, T_, d, E, k, idx, w, logits, st);
  if (E <= 16) return launch_router_small<T, 16, 2, VEC>(x, wg, bias, T_, d, E, k, idx, w, logits, st);
  return launch_router_small<T, 32, 1, VEC>(x, wg, bias, T_, d, E, k, idx, w, logits, st);
}

template <typename T>
int router_small_dispatch(const void* x, const void* wg, const float* bias, int T_, int d, int E, int k, int32_t* idx,
                          float* w, float* logits, cudaStream_t st) {
  constexpr int V = 16 / sizeof(T);
  if (d % V == 0 && aligned16(x) && aligned16(wg))
    return router_small_dispatch_e<T, V>(x, wg, bias, T_, d, E, k, idx, w, logits, st);
  return router_small_dispatch_e<T, 1>(x, wg, bias, T_, d, E, k, idx, w, logits, st);
}

template <typename T, int NT>
int launch_router_mma(const void* x, const void* wg, const float* bias, int T_, int d, int E, int k, int32_t* idx,
                      float* w, float* logits, cudaStream_t st) {
  if (T_ <= 64 && d % 512 == 0) {  // decode-sized: sixteen warps per 16 tokens
    SMOE_CK(launch_k(router_mma_kernel<T, NT, 16, 16>, (unsigned)cdiv(T_, 16), 512, 0, st, (const T*)x, (const T*)wg, bias, T_, d,
                                                                              E, k, idx, w, logits));
    SMOE_CK(cudaGetLastError());
    return SMOE_OK;
  }
  if (d % 128 == 0) {  // four warps per 16 tokens
    const int64_t blocks = cdiv(T_, 16);
    if (blocks > INT32_MAX) return SMOE_ERR_UNSUPPORTED;
    SMOE_CK(launch_k(router_mma_kernel<T, NT, 4>, (unsigned)blocks, 128, 0, st, (const T*)x, (const T*)wg, bias, T_, d, E, k, idx,
                                                                   w, logits));
    SMOE_CK(cudaGetLastError());
    return SMOE_OK;
  }
  const int64_t blocks = cdiv(T_, 32);  // two warps per 16 tokens
  if (blocks > INT32_MAX) return SMOE_ERR_UNSUPPORTED;
  SMOE_CK(launch_k(router_mma_kernel<T, NT, 2>, (unsigned)blocks, 128, 0, st, (const T*)x, (const T*)wg, bias, T_, d, E, k, idx, w,
                                                                 logits));
  SMOE_CK(cudaGetLastError());
  return SMOE_OK;
}

template <typename T>
int router_mma_dispatch(const void* x, const void* wg, const float* bias, int T_, int d, int E, int k, int32_t* idx,
                        float* w, float* logits, cudaStream_t st) {
  switch (router_mma_tiles(E)) {
    case 1: return launch_router_mma<T, 1>(x, wg, bias, T_, d, E, k, idx, w, logits, st);
    case 2: return launch_router_mma<T, 2>(x, wg, bias, T_, d, E, k, idx, w, logits, st);
    default: return launch_router_mma<T, 4>(x, wg, bias, T_, d, E, k, idx, w, logits, st);
  }
}

// Generic fallback router kernel for shapes the other two paths do not take
// (16-bit, E > 32 with E or d not a multiple of 8): one warp per token, one dot
// product per expert, fp32 logits into the workspace.
template <typename T>
__global__ void __launch_bounds__(256) router_logits_generic_kernel(const T* __restrict__ x, const T* __restrict__ wg,
                                                                    int T_, int d, int E, float* __restrict__ logits) {
  pdl_wait_and_release();
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (t >= T_) return;
  for (int e = 0; e < E; ++e) {
    float s = 0.f;
    for (int i = lane; i < d; i += 32) s = fmaf(Num<T>::to_f(x[(size_t)t * d + i]), Num<T>::to_f(wg[(size_t)e * d + i]), s);
    s = warp_sum(s);
    if (lane == 0) logits[(size_t)t * E + e] = s;
  }
}

// Self-test of the bounded wait: one thread waits for phase 0 of an mbarrier that
// expects one arrival and gets none, giving up after limit_ns.  *gave_up = 1 when the
// wait returned without the phase completing (the normal outcome).
__global__ void selftest_wait_kernel(uint64_t limit_ns, int* gave_up) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_word;
  if (threadIdx.x == 0) {
    abort_word = 0;
    mbar_init(smem_u32(&bar), 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const bool completed = mbar_wait(smem_u32(&bar), 0, &abort_word, limit_ns);
    *gave_up = completed ? 0 : 1;
  }
}

}  // namespace

// =============================================================================== C ABI
extern "C" {

const char* smoe_version(void) { return "swiftmoe-b200 0.1 (sm_100a)"; }

const char* smoe_status_string(int s) {
  switch (s) {
    case SMOE_OK: return "ok";
    case SMOE_ERR_INVALID: return "invalid argument";
    case SMOE_ERR_CUDA: return "CUDA error";
    case SMOE_ERR_TIMEOUT: return "device wait timed out";
    case SMOE_ERR_UNSUPPORTED: return "unsupported shape or dtype";
    case SMOE_ERR_WORKSPACE: return "workspace too small";
    case SMOE_ERR_TOO_LARGE: return "size beyond the fixed maximum of this entry point";
    default: return "unknown status";
  }
}

int smoe_device_sm_count(void) { return device_sms(); }

int smoe_read_device_error(int* flag, smoe_stream_t stream) {
  if (!flag) return SMOE_ERR_INVALID;
  SMOE_CK(cudaStreamSynchronize((cudaStream_t)stream));
  int v = 0;
  SMOE_CK(cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int)));
  const int zero = 0;
  SMOE_CK(cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int)));
  if (v != 0) {
    int dev = 0;
    SMOE_CK(cudaDeviceSynchronize());
    SMOE_CK(cudaGetDevice(&dev));
    reset_split_counters(dev);
  }
  *flag = v;
  return SMOE_OK;
}

int smoe_selftest_wait_timeout(uint64_t limit_ns, int* gave_up, smoe_stream_t stream) {
  if (!gave_up || limit_ns == 0 || limit_ns > 1000000000ull) return SMOE_ERR_INVALID;
  selftest_wait_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(limit_ns, gave_up);
  SMOE_CK(cudaGetLastError());
  return SMOE_OK;
}

size_t smoe_router_workspace_size(int T, int d, int E, int dtype) {
  if (T <= 0 || E <= 0 || elt_size(dtype) == 0) return 0;
  const RouterPath p = router_path(d, E, dtype);
  if (p == kRouterSmall || p == kRouterMma) return 0;
  return align_up((size_t)T * E * sizeof(float), 256) + 256;
}

int smoe_router_fwd(const void* x, const void* wg, int dtype, const float* logit_bias, int T, int d, int E, int k,
                    int32_t* idx, float* w, float* logits_out, void* workspace, size_t workspace_bytes,
                    smoe_stream_t stream) {
  cudaStream_t st = (cudaStream_t)stream;
  if (T < 0 || d < 1 || E < 1 || k < 1 || k > E || k > 32 || E > 32 * 32 || elt_size(dtype) == 0)
    return SMOE_ERR_INVALID;
  if (T == 0) return SMOE_OK;
  if (!x || !wg || !idx || !w) return SMOE_ERR_INVALID;
  RouterPath path = router_path(d, E, dtype);
  if (path == kRouterMma && (!aligned16(x) || !aligned16(wg))) path = kRouterSmall;
  if (path == kRouterMma) {
    return dtype == SMOE_F16 ? router_mma_dispatch<__half>(x, wg, logit_bias, T, d, E, k, idx, w, logits_out, st)
                             : router_mma_dispatch<__nv_bfloat16>(x, wg, logit_bias, T, d, E, k, idx, w, logits_out, st);
  }
  if (path == kRouterSmall) {
    switch (dtype) {
      case SMOE_F32: return router_small_dispatch<float>(x, wg, logit_bias, T, d, E, k, idx, w, logits_out, st);
      case SMOE_F16: return router_small_dispatch<__half>(x, wg, logit_bias, T, d, E, k, idx, w, logits_out, st);
      default: return router_small_dispatch<__nv_bfloat16>(x, wg, logit_bias, T, d, E, k, idx, w, logits_out, st);
    }
  }
  // logits through a GEMM (or the generic kernel), then top-k
  float* logits = logits_out;
  int32_t* offs = nullptr;
  const size_t need = smoe_router_workspace_size(T, d, E, dtype);
  if (!workspace || workspace_bytes < need) return SMOE_ERR_WORKSPACE;
  unsigned char* wsb = static_cast<unsigned char*>(workspace);
  if (!logits) logits = reinterpret_cast<float*>(wsb);
  offs = reinterpret_cast<int32_t*>(wsb + align_up((size_t)T * E * sizeof(float), 256));
  if (path == kRouterGemm) {
    SMOE_CK(launch_k(fill_two_kernel, 1, 1, 0, st, offs, 0, T));
    SMOE_CK(cudaGetLastError());
    const int rc = grouped_gemm_impl(x, wg, nullptr, logits, dtype, SMOE_F32, SMOE_EPI_STORE, offs, nullptr, 1, T, E, d, st);
    if (rc != SMOE_OK) return rc;
  } else {
    const unsigned grid = (unsigned)cdiv(T, 8);
    if (dtype == SMOE_F16)
      SMOE_CK(launch_k(router_logits_generic_kernel<__half>, grid, 256, 0, st, (const __half*)x, (const __half*)wg, T, d, E, logits));
    else
      SMOE_CK(launch_k(router_logits_generic_kernel<__nv_bfloat16>, grid, 256, 0, st, (const __nv_bfloat16*)x,
                       (const __nv_bfloat16*)wg, T, d, E, logits));
    SMOE_CK(cudaGetLastError());
  }
  SMOE_CK(launch_k(topk_from_logits_kernel, (unsigned)cdiv(T, 8), 256, 0, st, logits, logit_bias, T, E, k, idx, w));
  SMOE_CK(cudaGetLastError());
  return SMOE_OK;
}

int smoe_topk_from_logits(const float* logits, int T, int E, int k, int32_t* idx, float* w, smoe_stream_t stream) {
  if (T < 0 || E < 1 || k < 1 || k > E || k > 32 || E > 32 * 32) return SMOE_ERR_INVALID;
  if (T == 0) return SMOE_OK;
  if (!logits || !idx || !w) return SMOE_ERR_INVALID;
  SMOE_CK(launch_k(topk_from_logits_kernel, (unsigned)cdiv(T, 8), 256, 0, (cudaStream_t)stream, logits, nullptr, T, E, k, idx, w));
  SMOE_CK(cudaGetLastError());
  return SMOE_OK;
}

// ------------------------------------------------------------------ dispatch plan
size_t smoe_plan_workspace_size(int T, int k, int E) {
  if (T < 0 || k < 1 || E < 1) return 0;
  const int64_t nb = std::max<int64_t>(1, cdiv((int64_t)T * k, kPlanChunk));
  return 2 * align_up((size_t)nb * E * sizeof(int32_t), 256);
}

int64_t smoe_plan_rows_cap(int T, int k, int E, int capacity, int row_align) {
  if (T < 0 || k < 1 || E < 1 || row_align < 1) return 0;
  int64_t kept = (int64_t)T * k;
  if (capacity > 0) kept = std::min<int64_t>(kept, (int64_t)capacity * E);
  return kept + (int64_t)E * (row_align - 1);
}

int smoe_dispatch_plan(const int32_t* idx, int T, int k, int E, int capacity, int row_align, int32_t* expert_counts,
                       int32_t* expert_offsets, int32_t* slot_row, int32_t* row_token, int64_t rows_cap,
                       void* workspace, size_t workspace_bytes, smoe_stream_t stream) {
  cudaStream_t st = (cudaStream_t)stream;
  if (T < 0 || k < 1 || E < 1 || E > 4096 || row_align < 1 || row_align > 1024) return SMOE_ERR_INVALID;
  if (!expert_counts || !expert_offsets) return SMOE_ERR_INVALID;
  if (rows_cap < smoe_plan_rows_cap(T, k, E, capacity, row_align)) return SMOE_ERR_INVALID;
  if (T > 0 && (!idx || !slot_row || !row_token)) return SMOE_ERR_INVALID;
  const size_t need = smoe_plan_workspace_size(T, k, E);
  if (!workspace || workspace_bytes < need) return SMOE_ERR_WORKSPACE;
  const int64_t n_slots = (int64_t)T * k;
  if (n_slots > INT32_MAX) return SMOE_ERR_UNSUPPORTED;
  const int nb = (int)std::max<int64_t>(1, cdiv(n_slots, kPlanChunk));
  int32_t* hist = static_cast<int32_t*>(workspace);
  int32_t* base = reinterpret_cast<int32_t*>(static_cast<unsigned char*>(workspace) +
                                             align_up((size_t)nb * E * sizeof(int32_t), 256));
  const int smem_w = kPlanWarps * E * (int)sizeof(int);
  if (nb == 1) {  // one block: count, scan and scatter in one launch
    static SmemGrant done_1;
    const int smem_1 = smem_w + (E + 1) * (int)sizeof(int);
    SMOE_CK(ensure_smem(plan_small_kernel, smem_1, &done_1));
    SMOE_CK(launch_k(plan_small_kernel, 1, kPlanThreads, smem_1, st, idx, n_slots, k, E, capacity, row_align, expert_counts,
                                                       expert_offsets, slot_row, row_token));
    SMOE_CK(cudaGetLastError());
    return SMOE_OK;
  }
  static SmemGrant done_c, done_s;
  SMOE_CK(ensure_smem(plan_count_kernel, smem_w, &done_c));
  SMOE_CK(ensure_smem(plan_scatter_kernel, smem_w, &done_s));
  SMOE_CK(launch_k(plan_count_kernel, nb, kPlanThreads, smem_w, st, idx, n_slots, E, hist));
  SMOE_CK(cudaGetLastError());
  SMOE_CK(launch_k(plan_scan_kernel, 1, 1024, E * sizeof(int), st, hist, nb, E, capacity, row_align, base, expert_counts,
                                                     expert_offsets, row_token));
  SMOE_CK(cudaGetLastError());
  if (n_slots > 0) {
    SMOE_CK(launch_k(plan_scatter_kernel, nb, kPlanThreads, smem_w, st, idx, n_slots, k, E, capacity, base, expert_offsets,
                                                          slot_row, row_token));
    SMOE_CK(cudaGetLastError());
  }
  return SMOE_OK;
}

int smoe_permute_rows(const void* x, int dtype, int T, int d, const int32_t* row_token, const int32_t* expert_offsets,
                      int E, int64_t rows_cap, void* rows, smoe_stream_t stream) {
  const int es = elt_size(dtype);
  if (es == 0 || T < 0 || d < 1 || E < 1 || rows_cap < 0) return SMOE_ERR_INVALID;
  if (rows_cap == 0) return SMOE_OK;
  if (!row_token || !expert_offsets || !rows || (T > 0 && !x)) return SMOE_ERR_INVALID;
  const int64_t row_bytes = (int64_t)d * es;
  const bool vec = row_bytes % 16 == 0 && aligned16(x) && aligned16(rows);
  const int64_t blocks = std::min<int64_t>(cdiv(rows_cap, 8), (int64_t)device_sms() * 16);
  SMOE_CK(launch_k(permute_rows_kernel, (unsigned)blocks, 256, 0, (cudaStream_t)stream, 
      static_cast<const unsigned char*>(x), row_bytes, vec, row_token, expert_offsets, E,
      static_cast<unsigned char*>(rows)));
  SMOE_CK(cudaGetLastError());
  return SMOE_OK;
}

int smoe_combine(const void* y, int dtype, const int32_t* slot_row, const float* w, int T, int k, int d,
                 const void* shared, void* out, smoe_stream_t stream) {
  const int es = elt_size(dtype);
  if (es == 0 || T < 0 || k < 1 || d < 1) return SMOE_ERR_INVALID;
  if (T == 0) return SMOE_OK;
  if (!slot_row || !w || !out || !y) return SMOE_ERR_INVALID;
  cudaStream_t st = (cudaStream_t)stream;
  const int V = 16 / es;
  const bool vec = d % V == 0 && aligned16(y) && aligned16(out) && (!shared || aligned16(shared));
  if (vec && k <= 32) {  // one warp per token
    const unsigned grid = (unsigned)std::min<int64_t>(cdiv(T, 8), (int64_t)device_sms() * 8);
#define SMOE_COMBINE_W(TY, VV)                                                                                 \
  SMOE_CK(launch_k(combine_warp_kernel<TY, VV>, grid, 256, 0, st, (const TY*)y, slot_row, w, T, k, d, (const TY*)shared, (TY*)out))
    switch (dtype) {
      case SMOE_F32: SMOE_COMBINE_W(float, 4); break;
      case SMOE_F16: SMOE_COMBINE_W(__half, 8); break;
      default: SMOE_COMBINE_W(__nv_bfloat16, 8);
    }
#undef SMOE_COMBINE_W
    SMOE_CK(cudaGetLastError());
    return SMOE_OK;
  }
  const int64_t items = (int64_t)T * (vec ? d / V : d);
  const unsigned grid = (unsigned)std::min<int64_t>(cdiv(items, 256), (int64_t)device_sms() * 32);
#define SMOE_COMBINE(TY, VV)                                                                                  \
  SMOE_CK(launch_k(combine_kernel<TY, VV>, grid, 256, 0, st, (const TY*)y, slot_row, w, T, k, d, (const TY*)shared, (TY*)out))
  switch (dtype) {
    case SMOE_F32:
      if (vec) SMOE_COMBINE(float, 4); else SMOE_COMBINE(float, 1);
      break;
    case SMOE_F16:
      if (vec) SMOE_COMBINE(__half, 8); else SMOE_COMBINE(__half, 1);
      break;
    default:
      if (vec) SMOE_COMBINE(__nv_bfloat16, 8); else SMOE_COMBINE(__nv_bfloat16, 1);
  }
#undef SMOE_COMBINE
  SMOE_CK(cudaGetLastError());
  return SMOE_OK;
}

int smoe_grouped_gemm(const void* A, const void* B, const void* B3, void* C, int dtype, int out_dtype, int epilogue,
                      const int32_t* offsets, const int32_t* ends, int G, int64_t rows_cap, int N, int K,
                      smoe_stream_t stream) {
  return grouped_gemm_impl(A, B, B3, C, dtype, out_dtype, epilogue, offsets, ends, G, rows_cap, N, K,
                           (cudaStream_t)stream);
}

int smoe_grouped_gemm_rows(const void* A, const void* B, const void* B3, const uint64_t* row_ptrs, int dtype,
                           int out_dtype, int epilogue, const int32_t* offsets, const int32_t* ends, int G,
                           int64_t rows_cap, int N, int K, smoe_stream_t stream) {
  if (!row_ptrs) return SMOE_ERR_INVALID;
  if (out_dtype != SMOE_F32 && (N * (int64_t)elt_size(out_dtype)) % 16 != 0) return SMOE_ERR_UNSUPPORTED;
  return grouped_gemm_impl(A, B, B3, nullptr, dtype, out_dtype, epilogue, offsets, ends, G, rows_cap, N, K,
                           (cudaStream_t)stream, row_ptrs);
}

int smoe_tf32_split_weights(const float* w, float* out, int64_t rows, int K, smoe_stream_t stream) {
  if (!w || !out || rows < 0 || K < 4 || K % 4 != 0) return SMOE_ERR_INVALID;
  if (!aligned16(w) || !aligned16(out)) return SMOE_ERR_UNSUPPORTED;
  if (rows == 0) return SMOE_OK;
  const int64_t n = rows * (K / 4);
  const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>(cdiv(n, 256), (int64_t)device_sms() * 16));
  SMOE_CK(launch_k(tc::tf32_split3_kernel, grid, 256, 0, (cudaStream_t)stream, w, out, rows, K, 0));
  SMOE_CK(cudaGetLastError());
  return SMOE_OK;
}

int smoe_transpose_batched(const void* src, void* dst, int dtype, int G, int R, int C, smoe_stream_t stream) {
  const int es = elt_size(dtype);
  if (es == 0 || G < 0 || R < 0 || C < 0) return SMOE_ERR_INVALID;
  if ((int64_t)G * R * C == 0) return SMOE_OK;
  if (!src || !dst || src == dst) return SMOE_ERR_INVALID;
  dim3 grid((unsigned)cdiv(C, 32), (unsigned)cdiv(R, 32), (unsigned)G), block(32, 8);
  if (es == 4)
    transpose_batched_kernel<float><<<grid, block, 0, (cudaStream_t)stream>>>((const float*)src, (float*)dst, R, C);
  else
    transpose_batched_kernel<unsigned short>
        <<<grid, block, 0, (cudaStream_t)stream>>>((const unsigned short*)src, (unsigned short*)dst, R, C);
  SMOE_CK(cudaGetLastError());
  return SMOE_OK;
}

int smoe_gather_rows(const void* src, int dtype, int d, const int32_t* index, int64_t n_rows, void* dst,
                     smoe_stream_t stream) {
  const int es = elt_size(dtype);
  if (es == 0 || d < 1 || n_rows < 0) return SMOE_ERR_INVALID;
  if (n_rows == 0) return SMOE_OK;
  if (!src || !index || !dst) return SMOE_ERR_INVALID;
  const int64_t row_bytes = (int64_t)d * es;
  const bool vec = row_bytes % 16 == 0 && aligned16(src) && aligned16(dst);
  const int64_t blocks = std::min<int64_t>(cdiv(n_rows, 8), (int64_t)device_sms() * 16);
  gather_rows_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(
      static_cast<const unsigned char*>(src), row_bytes, vec, index, n_rows, static_cast<unsigned char*>(dst));
  SMOE_CK(cudaGetLastError());
  return SMOE_OK;
}

size_t smoe_ep_regroup_workspace_size(int ws, int E_l) {
  if (ws < 1 || E_l < 1) return 0;
  return 3 * align_up(((size_t)ws * E_l + 1) * sizeof(int32_t), 256);
}

int smoe_ep_regroup_plan(const int32_t* recv_counts, int ws, int E_l, int capacity, const int32_t* pos_base,
                         int64_t n_recv, int32_t* expert_counts, int32_t* expert_offsets, int32_t* row_src,
                         int32_t* recv_dst, void* workspace, size_t workspace_bytes, smoe_stream_t stream) {
  cudaStream_t st = (cudaStream_t)stream;
  if (ws < 1 || E_l < 1 || n_recv < 0 || n_recv > INT32_MAX || (int64_t)ws * E_l > (1 << 20)) return SMOE_ERR_INVALID;
  if (!recv_counts || !expert_counts || !expert_offsets) return SMOE_ERR_INVALID;
  if (n_recv > 0 && (!row_src || !recv_dst)) return SMOE_ERR_INVALID;
  if (!workspace || workspace_bytes < smoe_ep_regroup_workspace_size(ws, E_l)) return SMOE_ERR_WORKSPACE;
  const size_t slab = align_up(((size_t)ws * E_l + 1) * sizeof(int32_t), 256);
  int32_t* seg_start = static_cast<int32_t*>(workspace);
  int32_t* src_base = reinterpret_cast<int32_t*>(static_cast<unsigned char*>(workspace) + slab);
  int32_t* kept_base = reinterpret_cast<int32_t*>(static_cast<unsigned char*>(workspace) + 2 * slab);
  const int smem = (E_l + ws) * (int)sizeof(int);
  static SmemGrant done;
  SMOE_CK(ensure_smem(ep_regroup_scan_kernel, smem, &done));
  ep_regroup_scan_kernel<<<1, 1024, smem, st>>>(recv_counts, ws, E_l, capacity, pos_base, expert_counts,
                                                expert_offsets, seg_start, src_base, kept_base);
  SMOE_CK(cudaGetLastError());
  if (n_recv > 0) {
    const unsigned grid = (unsigned)std::min<int64_t>(cdiv(n_recv, 256), (int64_t)device_sms() * 8);
    ep_regroup_rows_kernel<<<grid, 256, 0, st>>>(seg_start, src_base, kept_base, expert_offsets, ws * E_l, E_l,
                                                 capacity, n_recv, row_src, recv_dst);
    SMOE_CK(cudaGetLastError());
  }
  return SMOE_OK;
}

int smoe_ep_dedup_ranks(const int32_t* idx, int64_t T, int k, int E_l, int ws, int rank, int32_t* ridx,
                        smoe_stream_t stream) {
  if (T < 0 || k < 1 || E_l < 1 || ws < 1 || rank < 0 || rank >= ws) return SMOE_ERR_INVALID;
  if (T == 0) return SMOE_OK;
  if (!idx || !ridx) return SMOE_ERR_INVALID;
  const unsigned grid = (unsigned)std::min<int64_t>(cdiv(T, 256), (int64_t)device_sms() * 8);
  ep_dedup_ranks_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(idx, T, k, E_l, ws, rank, ridx);
  SMOE_CK(cudaGetLastError());
  return SMOE_OK;
}

int smoe_ep_dedup_meta(const int32_t* idx, const float* w, const int32_t* ridx, const int32_t* slot_row,
                       const int32_t* own_count, int64_t T, int k, int E_l, int ws, int32_t* meta_e, float* meta_w,
                       int32_t* own_e, smoe_stream_t stream) {
  if (T < 0 || k < 1 || E_l < 1 || ws < 1) return SMOE_ERR_INVALID;
  if (T == 0) return SMOE_OK;
  if (!idx || !w || !ridx || !slot_row || !own_count || !meta_e || !meta_w || !own_e) return SMOE_ERR_INVALID;
  const unsigned grid = (unsigned)std::min<int64_t>(cdiv(T * k, 256), (int64_t)device_sms() * 8);
  ep_dedup_meta_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(idx, w, ridx, slot_row, own_count, T, k, E_l, ws,
                                                               meta_e, meta_w, own_e);
  SMOE_CK(cudaGetLastError());
  return SMOE_OK;
}

int smoe_ep_return_rows(const int32_t* row_src, const int32_t* expert_offsets, int E_l, const int32_t* recv_dst,
                        int64_t n_recv, const int64_t* seg_table, int n_src, int64_t row_bytes, uint64_t* row_ptrs,
                        int64_t rows_cap, smoe_stream_t stream) {
  if (E_l < 1 || n_src < 1 || n_recv < 0 || rows_cap < 0 || row_bytes <= 0 || row_bytes % 16 != 0)
    return SMOE_ERR_INVALID;
  if (!expert_offsets || !seg_table || (rows_cap > 0 && !row_ptrs)) return SMOE_ERR_INVALID;
  if (!row_src && rows_cap > n_recv) return SMOE_ERR_INVALID;
  if (rows_cap == 0 && n_recv == 0) return SMOE_OK;
  const int64_t work = std::max<int64_t>(rows_cap, recv_dst ? n_recv * 32 : 0);
  const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>(cdiv(work, 256), (int64_t)device_sms() * 8));
  ep_return_rows_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(row_src, expert_offsets, E_l, recv_dst, n_recv,
                                                                seg_table, n_src, row_bytes, row_ptrs, rows_cap);
  SMOE_CK(cudaGetLastError());
  return SMOE_OK;
}

int smoe_ep_layout(const int32_t* counts_all, int ws, int E, int rank, int capacity, const uint64_t* recv_base,
                   const uint64_t* ret_base, int64_t row_bytes, int64_t recv_rows_max, uint64_t* send_addr,
                   int32_t* keep, int32_t* recv_offsets, int64_t* seg_table, int flags, smoe_stream_t stream) {
  if (ws < 1 || E < 1 || E % ws != 0 || rank < 0 || rank >= ws || capacity < 0) return SMOE_ERR_INVALID;
  if (flags & ~SMOE_EP_LAYOUT_ROTATED) return SMOE_ERR_INVALID;
  if ((flags & SMOE_EP_LAYOUT_ROTATED) && (E != ws || capacity != 0)) return SMOE_ERR_INVALID;
  if (row_bytes <= 0 || row_bytes % 16 != 0 || recv_rows_max < 0 || recv_rows_max > INT32_MAX) return SMOE_ERR_INVALID;
  if (!counts_all || !recv_base || !ret_base || !send_addr || !keep || !recv_offsets || !seg_table)
    return SMOE_ERR_INVALID;
  if ((int64_t)ws * E > kLayoutMaxCells) return SMOE_ERR_UNSUPPORTED;
  const int smem = (ws * E + 2 * E) * (int)sizeof(int);
  static SmemGrant done;
  SMOE_CK(ensure_smem(ep_layout_kernel, smem, &done));
  ep_layout_kernel<<<1, 256, smem, (cudaStream_t)stream>>>(counts_all, ws, E, rank, capacity, recv_base, ret_base,
                                                           row_bytes, recv_rows_max, send_addr, keep, recv_offsets,
                                                           seg_table, flags & SMOE_EP_LAYOUT_ROTATED);
  SMOE_CK(cudaGetLastError());
  return SMOE_OK;
}

int smoe_ep_send_rows(const void* x, int64_t row_bytes, const int32_t* row_token, const int32_t* expert_offsets,
                      int E, int own_first, int own_count, const uint64_t* send_addr, const int32_t* keep,
                      int64_t rows_cap, smoe_stream_t stream) {
  if (row_bytes <= 0 || row_bytes % 16 != 0 || E < 1 || own_first < 0 || own_count < 0 || own_first + own_count > E ||
      rows_cap < 0)
    return SMOE_ERR_INVALID;
  if (rows_cap == 0) return SMOE_OK;
  if (!x || !row_token || !expert_offsets || !send_addr || !keep || !aligned16(x)) return SMOE_ERR_INVALID;
  const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>(cdiv(rows_cap, 8), (int64_t)device_sms() * 2));
  ep_send_rows_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(
      static_cast<const unsigned char*>(x), row_bytes, row_token, expert_offsets, E, own_first,
      own_first + own_count, send_addr, keep);
  SMOE_CK(cudaGetLastError());
  return SMOE_OK;
}

int smoe_ep_clear_tail(int32_t* idx, const int32_t* n_rows, int64_t rows_cap, int k, smoe_stream_t stream) {
  if (rows_cap < 0 || k < 1) return SMOE_ERR_INVALID;
  if (rows_cap == 0) return SMOE_OK;
  if (!idx || !n_rows) return SMOE_ERR_INVALID;
  const unsigned grid = (unsigned)std::min<int64_t>(cdiv(rows_cap * k, 256), (int64_t)device_sms() * 8);
  ep_clear_tail_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(idx, n_rows, rows_cap, k);
  SMOE_CK(cudaGetLastError());
  return SMOE_OK;
}

int smoe_store_rows(const void* src, int64_t row_bytes, const uint64_t* row_ptrs, int64_t n_rows,
                    smoe_stream_t stream) {
  if (row_bytes <= 0 || row_bytes % 16 != 0 || n_rows < 0) return SMOE_ERR_INVALID;
  if (n_rows == 0) return SMOE_OK;
  if (!src || !row_ptrs || !aligned16(src)) return SMOE_ERR_INVALID;
  const int64_t blocks = std::max<int64_t>(1, std::min<int64_t>(cdiv(n_rows, 8), (int64_t)device_sms() * 4));
  store_rows_kernel<<<(unsigned)blocks, 256, 0, (cudaStream_t)stream>>>(static_cast<const unsigned char*>(src),
                                                                         row_bytes, row_ptrs, n_rows);
  SMOE_CK(cudaGetLastError());
  return SMOE_OK;
}

int smoe_copy_rows_count(void* dst, const void* src, int64_t row_bytes, const int32_t* n_rows, int64_t rows_cap,
                         smoe_stream_t stream) {
  if (row_bytes <= 0 || row_bytes % 16 != 0 || rows_cap < 0) return SMOE_ERR_INVALID;
  if (rows_cap == 0) return SMOE_OK;
  if (!dst || !src || !n_rows || !aligned16(dst) || !aligned16(src)) return SMOE_ERR_INVALID;
  const unsigned grid = (unsigned)std::min<int64_t>(cdiv(rows_cap * (row_bytes >> 4), 256), (int64_t)device_sms() * 8);
  copy_rows_count_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(static_cast<unsigned char*>(dst),
                                                                 static_cast<const unsigned char*>(src), row_bytes,
                                                                 n_rows, rows_cap);
  SMOE_CK(cudaGetLastError());
  return SMOE_OK;
}

int smoe_ep_drop_slots(const int32_t* idx, int64_t n_slots, const int32_t* expert_offsets, int E, const int32_t* keep,
                       int32_t* slot_row, smoe_stream_t stream) {
  if (n_slots < 0 || E < 1) return SMOE_ERR_INVALID;
  if (n_slots == 0) return SMOE_OK;
  if (!idx || !expert_offsets || !keep || !slot_row) return SMOE_ERR_INVALID;
  const unsigned grid = (unsigned)std::min<int64_t>(cdiv(n_slots, 256), (int64_t)device_sms() * 8);
  ep_drop_slots_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(idx, n_slots, expert_offsets, E, keep, slot_row);
  SMOE_CK(cudaGetLastError());
  return SMOE_OK;
}

// ------------------------------------------------------------------ whole layer
namespace {
struct LayerPlan {
  size_t off_idx, off_w, off_counts, off_offsets, off_slot_row, off_row_token, off_plan_ws, off_router_ws, off_xrows,
      off_h, off_y, off_hs, off_ys, off_soff, total;
  size_t plan_ws, router_ws;
  int64_t rows_cap;
};

bool layer_plan(const smoe_layer_args* a, LayerPlan* p) {
  const int es = elt_size(a->dtype);
  if (es == 0) return false;
  const int64_t T = a->tokens, d = a->d_model, E = a->num_experts, k = a->top_k;
  const int64_t F = a->expert_type == SMOE_EXPERT_SWIGLU ? a->d_ff : 0;
  const int64_t Fs = a->num_shared > 0 ? a->d_ff_shared : 0;
  p->rows_cap = smoe_plan_rows_cap((int)T, (int)k, (int)E, a->capacity, 1);
  p->plan_ws = smoe_plan_workspace_size((int)T, (int)k, (int)E);
  p->router_ws = smoe_router_workspace_size((int)T, (int)d, (int)E, a->dtype);
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o = align_up(o + bytes, 256);
    return at;
  };
  p->off_idx = take(T * k * 4);
  p->off_w = take(T * k * 4);
  p->off_counts = take(E * 4);
  p->off_offsets = take((E + 1) * 4);
  p->off_slot_row = take(T * k * 4);
  p->off_row_token = take(std::max<int64_t>(p->rows_cap, 1) * 4);
  p->off_plan_ws = take(p->plan_ws);
  p->off_router_ws = take(p->router_ws);
  p->off_xrows = take(p->rows_cap * d * es);
  p->off_h = take(p->rows_cap * F * es);
  p->off_y = take(p->rows_cap * d * es);
  p->off_hs = take(T * Fs * es);
  p->off_ys = take(Fs > 0 ? T * d * es : 0);
  p->off_soff = take(16);
  p->total = o;
  return true;
}
}  // namespace

int smoe_ep_buffer_create(size_t bytes, void** dev_ptr, void* ipc_handle) {
  if (!dev_ptr || !ipc_handle || bytes == 0) return SMOE_ERR_INVALID;
  static_assert(sizeof(cudaIpcMemHandle_t) == SMOE_IPC_HANDLE_BYTES, "IPC handle size");
  void* p = nullptr;
  SMOE_CK(cudaMalloc(&p, bytes));
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    report_cuda_error(e, "cudaIpcGetMemHandle", __FILE__, __LINE__);
    return SMOE_ERR_CUDA;
  }
  memcpy(ipc_handle, &h, sizeof(h));
  *dev_ptr = p;
  return SMOE_OK;
}

int smoe_ep_buffer_destroy(void* dev_ptr) {
  if (!dev_ptr) return SMOE_ERR_INVALID;
  SMOE_CK(cudaFree(dev_ptr));
  return SMOE_OK;
}

int smoe_ep_peer_open(const void* ipc_handle, void** peer_ptr) {
  if (!ipc_handle || !peer_ptr) return SMOE_ERR_INVALID;
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  void* p = nullptr;
  SMOE_CK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  *peer_ptr = p;
  return SMOE_OK;
}

int smoe_ep_peer_close(void* peer_ptr) {
  if (!peer_ptr) return SMOE_ERR_INVALID;
  SMOE_CK(cudaIpcCloseMemHandle(peer_ptr));
  return SMOE_OK;
}

int smoe_copy_segments(void* const* dst, const void* const* src, const size_t* bytes, int n, smoe_stream_t stream) {
  if (n < 0 || (n > 0 && (!dst || !src || !bytes))) return SMOE_ERR_INVALID;
  for (int i = 0; i < n; ++i) {
    if (bytes[i] == 0) continue;
    if (!dst[i] || !src[i]) return SMOE_ERR_INVALID;
    SMOE_CK(cudaMemcpyAsync(dst[i], src[i], bytes[i], cudaMemcpyDeviceToDevice, (cudaStream_t)stream));
  }
  return SMOE_OK;
}

int smoe_event_create(void** event) {
  if (!event) return SMOE_ERR_INVALID;
  cudaEvent_t e;
  SMOE_CK(cudaEventCreate(&e));
  *event = e;
  return SMOE_OK;
}

int smoe_event_destroy(void* event) {
  if (!event) return SMOE_ERR_INVALID;
  SMOE_CK(cudaEventDestroy((cudaEvent_t)event));
  return SMOE_OK;
}

int smoe_event_record(void* event, smoe_stream_t stream) {
  if (!event) return SMOE_ERR_INVALID;
  SMOE_CK(cudaEventRecord((cudaEvent_t)event, (cudaStream_t)stream));
  return SMOE_OK;
}

int smoe_event_elapsed(void* start, void* end, float* ms) {
  if (!start || !end || !ms) return SMOE_ERR_INVALID;
  SMOE_CK(cudaEventSynchronize((cudaEvent_t)end));
  SMOE_CK(cudaEventElapsedTime(ms, (cudaEvent_t)start, (cudaEvent_t)end));
  return SMOE_OK;
}

size_t smoe_layer_workspace_size(const smoe_layer_args* a) {
  LayerPlan p;
  if (a && a->dtype == SMOE_F32_SPLITW) {
    smoe_layer_args b = *a;
    b.dtype = SMOE_F32;
    return layer_plan(&b, &p) ? p.total : 0;
  }
  if (!a || !layer_plan(a, &p)) return 0;
  return p.total;
}

static int layer_fwd_impl(const smoe_layer_args* a, smoe_stream_t stream, bool split_w);

// dtype SMOE_F32_SPLITW: an fp32 layer whose routed expert weights come split
int smoe_layer_fwd(const smoe_layer_args* a, smoe_stream_t stream) {
  if (a && a->dtype == SMOE_F32_SPLITW) {
    smoe_layer_args b = *a;
    b.dtype = SMOE_F32;
    return layer_fwd_impl(&b, stream, true);
  }
  return layer_fwd_impl(a, stream, false);
}

static int layer_fwd_impl(const smoe_layer_args* a, smoe_stream_t stream, bool split_w) {
  if (!a) return SMOE_ERR_INVALID;
  // Decode-sized batches (a one-block dispatch plan) launch the chain below with
  // programmatic dependent launch: measured 0.158 -> 0.147 ms for one token of the
  // Mixtral-shaped layer.  At 16384 tokens it measured 5 % slower, so larger batches
  // launch the ordinary way.
  const PdlScope pdl(a->tokens >= 0 && (int64_t)a->tokens * a->top_k <= kPlanChunk);
  cudaStream_t st = (cudaStream_t)stream;
  const int T = a->tokens, d = a->d_model, E = a->num_experts, k = a->top_k;
  if (T < 0 || d < 1 || E < 1 || k < 1 || k > E || elt_size(a->dtype) == 0) return SMOE_ERR_INVALID;
  if (a->expert_type != SMOE_EXPERT_LINEAR && a->expert_type != SMOE_EXPERT_SWIGLU) return SMOE_ERR_INVALID;
  if (a->expert_type == SMOE_EXPERT_SWIGLU && (a->d_ff < 1 || !a->w1 || !a->w3 || !a->w2)) return SMOE_ERR_INVALID;
  if (a->expert_type == SMOE_EXPERT_LINEAR && !a->w_lin) return SMOE_ERR_INVALID;
  if (a->num_shared < 0 || a->num_shared > 1) return SMOE_ERR_UNSUPPORTED;
  if (a->num_shared == 1 && (a->d_ff_shared < 1 || !a->sw1 || !a->sw3 || !a->sw2)) return SMOE_ERR_INVALID;
  if (!a->gate_w || (T > 0 && (!a->x || !a->out))) return SMOE_ERR_INVALID;
  LayerPlan p;
  layer_plan(a, &p);
  if (!a->workspace || a->workspace_bytes < p.total) return SMOE_ERR_WORKSPACE;
  if (T == 0) {
    for (int i = 0; i < 6; ++i)
      if (a->stage_events[i]) SMOE_CK(cudaEventRecord((cudaEvent_t)a->stage_events[i], st));
    return SMOE_OK;
  }
  unsigned char* ws = static_cast<unsigned char*>(a->workspace);
  int32_t* idx = a->topk_idx ? a->topk_idx : reinterpret_cast<int32_t*>(ws + p.off_idx);
  float* w = a->topk_w ? a->topk_w : reinterpret_cast<float*>(ws + p.off_w);
  int32_t* counts = a->expert_counts ? a->expert_counts : reinterpret_cast<int32_t*>(ws + p.off_counts);
  int32_t* offsets = reinterpret_cast<int32_t*>(ws + p.off_offsets);
  int32_t* slot_row = reinterpret_cast<int32_t*>(ws + p.off_slot_row);
  int32_t* row_token = reinterpret_cast<int32_t*>(ws + p.off_row_token);
  void* xrows = ws + p.off_xrows;
  void* h = ws + p.off_h;
  void* y = ws + p.off_y;
  const int dt = a->dtype;
  const int F = a->d_ff;
  auto mark = [&](int i) -> int {
    if (a->stage_events[i]) SMOE_CK(cudaEventRecord((cudaEvent_t)a->stage_events[i], st));
    return SMOE_OK;
  };
  int rc;
  if ((rc = mark(0))) return rc;
  rc = smoe_router_fwd(a->x, a->gate_w, dt, a->logit_bias, T, d, E, k, idx, w, nullptr, ws + p.off_router_ws,
                       p.router_ws, stream);
  if (rc) return rc;
  if ((rc = mark(1))) return rc;
  rc = smoe_dispatch_plan(idx, T, k, E, a->capacity, 1, counts, offsets, slot_row, row_token, p.rows_cap,
                          ws + p.off_plan_ws, p.plan_ws, stream);
  if (rc) return rc;
  // decode-sized SwiGLU layers: the first GEMM reads the token rows through row_token
  const bool gather = a->expert_type == SMOE_EXPERT_SWIGLU &&
                      gemv_eligible(a->x, a->w1, a->w3, dt, dt, SMOE_EPI_SWIGLU, E, p.rows_cap, d);
  if (!gather) {
    const int64_t row_bytes = (int64_t)d * elt_size(dt);
    if (row_bytes % 16 == 0 && aligned16(a->x) && aligned16(xrows) && k <= 32) {
      // token by token: each x row is read once for its k rows
      const unsigned grid = (unsigned)std::min<int64_t>(cdiv(T, 8), (int64_t)device_sms() * 8);
      SMOE_CK(launch_k(permute_tokens_kernel, grid, 256, 0, st, static_cast<const unsigned char*>(a->x), row_bytes, slot_row, T, k,
                                                  static_cast<unsigned char*>(xrows)));
      SMOE_CK(cudaGetLastError());
    } else {
      rc = smoe_permute_rows(a->x, dt, T, d, row_token, offsets, E, p.rows_cap, xrows, stream);
      if (rc) return rc;
    }
  }
  if ((rc = mark(2))) return rc;
  if (a->expert_type == SMOE_EXPERT_SWIGLU) {
    rc = gather ? launch_gemv(a->x, a->w1, a->w3, h, nullptr, dt, dt, SMOE_EPI_SWIGLU, offsets, nullptr, E,
                              p.rows_cap, F, d, st, row_token, T)
                : grouped_gemm_impl(xrows, a->w1, a->w3, h, dt, dt, SMOE_EPI_SWIGLU, offsets, nullptr, E, p.rows_cap,
                                    F, d, st, nullptr, split_w);
    if (rc) return rc;
    if ((rc = mark(3))) return rc;
    rc = grouped_gemm_impl(h, a->w2, nullptr, y, dt, dt, SMOE_EPI_STORE, offsets, nullptr, E, p.rows_cap, d, F, st,
                           nullptr, split_w);
    if (rc) return rc;
  } else {
    rc = grouped_gemm_impl(xrows, a->w_lin, nullptr, y, dt, dt, SMOE_EPI_STORE, offsets, nullptr, E, p.rows_cap, d, d, st,
                           nullptr, split_w);
    if (rc) return rc;
    if ((rc = mark(3))) return rc;
  }
  void* ys = nullptr;
  if (a->num_shared == 1) {
    int32_t* soff = reinterpret_cast<int32_t*>(ws + p.off_soff);
    SMOE_CK(launch_k(fill_two_kernel, 1, 1, 0, st, soff, 0, T));
    SMOE_CK(cudaGetLastError());
    void* hs = ws + p.off_hs;
    ys = ws + p.off_ys;
    rc = grouped_gemm_impl(a->x, a->sw1, a->sw3, hs, dt, dt, SMOE_EPI_SWIGLU, soff, nullptr, 1, T, a->d_ff_shared, d, st);
    if (rc) return rc;
    rc = grouped_gemm_impl(hs, a->sw2, nullptr, ys, dt, dt, SMOE_EPI_STORE, soff, nullptr, 1, T, d, a->d_ff_shared, st);
    if (rc) return rc;
  }
  if ((rc = mark(4))) return rc;
  rc = smoe_combine(y, dt, slot_row, w, T, k, d, ys, a->out, stream);
  if (rc) return rc;
  return mark(5);
}

int smoe_wgrad_gemm(const void* A, int64_t lda, const void* B, int64_t ldb, int dtype, const int32_t* k_offsets, int G,
                    int M, int N, int64_t K, float* C, smoe_stream_t stream) {
  if (!A || !B || !k_offsets || !C || G < 1 || G > tc::MAX_GROUPS || M < 1 || N < 1 || K < 0) return SMOE_ERR_INVALID;
  if (dtype != SMOE_BF16 && dtype != SMOE_F16) return SMOE_ERR_UNSUPPORTED;
  if (lda < K || ldb < K || lda % 8 != 0 || ldb % 8 != 0 || N % 4 != 0) return SMOE_ERR_UNSUPPORTED;
  if (!aligned16(A) || !aligned16(B) || !aligned16(C)) return SMOE_ERR_UNSUPPORTED;
  const CUtensorMapDataType dt = dtype == SMOE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap ma, mb;
  // an empty K range still needs a valid map: one column wide, never loaded
  if (!make_map_2d_ld(&ma, A, dt, M, std::max<int64_t>(K, 1), lda)) return SMOE_ERR_CUDA;
  if (!make_map_2d_ld(&mb, B, dt, N, std::max<int64_t>(K, 1), ldb)) return SMOE_ERR_CUDA;
  const uint32_t idesc = umma_idesc_f16(dtype == SMOE_BF16 ? 1u : 0u, tc::BM, tc::BN);
  return launch_wgrad<false>(ma, mb, C, k_offsets, G, M, N, idesc, (cudaStream_t)stream);
}

int smoe_wgrad_gemm_rows(const void* A, int64_t lda, const void* B, int64_t ldb, int dtype, const int32_t* k_offsets,
                         int G, int M, int N, int64_t K, float* C, smoe_stream_t stream) {
  if (!A || !B || !k_offsets || !C || G < 1 || G > tc::MAX_GROUPS || M < 1 || N < 1 || K < 0) return SMOE_ERR_INVALID;
  if (dtype != SMOE_BF16 && dtype != SMOE_F16) return SMOE_ERR_UNSUPPORTED;
  if (lda < M || ldb < N || lda % 8 != 0 || ldb % 8 != 0 || M % 8 != 0 || N % 8 != 0) return SMOE_ERR_UNSUPPORTED;
  if (!aligned16(A) || !aligned16(B) || !aligned16(C)) return SMOE_ERR_UNSUPPORTED;
  const CUtensorMapDataType dt = dtype == SMOE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUtensorMap ma, mb;
  // an empty K range still needs a valid map: one row, never loaded
  if (!make_map_2d_box(&ma, A, dt, std::max<int64_t>(K, 1), M, lda, tc::BK)) return SMOE_ERR_CUDA;
  if (!make_map_2d_box(&mb, B, dt, std::max<int64_t>(K, 1), N, ldb, tc::BK)) return SMOE_ERR_CUDA;
  const uint32_t idesc = umma_idesc_f16_mn(dtype == SMOE_BF16 ? 1u : 0u, tc::BM, tc::BN);
  return launch_wgrad<true>(ma, mb, C, k_offsets, G, M, N, idesc, (cudaStream_t)stream);
}

}  // extern "C"

// ------------------------------------------------------------------ layer backward
namespace {
constexpr int64_t kDwgSlices = 32;  // row slices of the gate-gradient kernel, at most

struct BwdPlan {
  int64_t S, rows_cap_full;
  size_t o_idx, o_w, o_cnt, o_off, o_sr, o_rt, o_pws, o_cntf, o_offf, o_srf, o_rtf, o_rws, o_xr, o_dr, o_roww,
      o_dwr, o_dsel, o_ab, o_g, o_dxr, o_abs, o_gs, o_dxs, o_soff, o_dwgp, total;
  size_t plan_ws, router_ws;
};

bool bwd_plan(const smoe_layer_bwd_args* a, BwdPlan* p) {
  const int es = elt_size(a->dtype);
  if (es != 2) return false;
  const bool lin = a->expert_type == SMOE_EXPERT_LINEAR;
  const int64_t T = a->tokens, d = a->d_model, E = a->num_experts, k = a->top_k, F = lin ? 0 : a->d_ff;
  const int64_t Fs = a->num_shared > 0 ? a->d_ff_shared : 0;
  p->S = smoe_plan_rows_cap((int)T, (int)k, (int)E, a->capacity, 64);
  p->rows_cap_full = smoe_plan_rows_cap((int)T, (int)k, (int)E, 0, 1);
  p->plan_ws = smoe_plan_workspace_size((int)T, (int)k, (int)E);
  p->router_ws = smoe_router_workspace_size((int)T, (int)d, (int)E, a->dtype);
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o = align_up(o + bytes, 256);
    return at;
  };
  const int64_t S = p->S;
  p->o_idx = take(T * k * 4);
  p->o_w = take(T * k * 4);
  p->o_cnt = take(E * 4);
  p->o_off = take((E + 1) * 4);
  p->o_sr = take(T * k * 4);
  p->o_rt = take(std::max<int64_t>(S, 1) * 4);
  p->o_pws = take(p->plan_ws);
  p->o_cntf = take(E * 4);
  p->o_offf = take((E + 1) * 4);
  p->o_srf = take(T * k * 4);
  p->o_rtf = take(std::max<int64_t>(p->rows_cap_full, 1) * 4);
  p->o_rws = take(p->router_ws);
  p->o_xr = take(S * d * es);
  p->o_dr = take(S * d * es);
  p->o_roww = take(S * 4);
  p->o_dwr = take(S * 4);
  p->o_dsel = take(std::max<int64_t>(p->rows_cap_full, 1) * 4);
  p->o_ab = take(S * 2 * F * es);
  p->o_g = take(S * (lin ? d : F) * es);   // linear experts: dout_r Wl, then the rows' input gradient
  p->o_dxr = take(lin ? 0 : S * d * es);
  p->o_abs = take(T * 2 * Fs * es);
  p->o_gs = take(T * Fs * es);
  p->o_dxs = take(Fs > 0 ? T * d * es : 0);
  p->o_soff = take(16);
  p->o_dwgp = take(kDwgSlices * E * d * 4);
  p->total = o;
  return true;
}

template <typename T>
int swiglu_bwd_launch(void* ab, void* g, const float* row_w, const int32_t* n_rows, int64_t rows_cap, int F,
                      float* dw_row, cudaStream_t st) {
  if (rows_cap == 0) return SMOE_OK;
  const unsigned grid = (unsigned)std::min<int64_t>(rows_cap, (int64_t)device_sms() * 16);
  swiglu_bwd_kernel<T><<<grid, 256, 0, st>>>((T*)ab, (T*)g, row_w, n_rows, rows_cap, F, dw_row);
  SMOE_CK(cudaGetLastError());
  return SMOE_OK;
}

template <typename T>
int linear_bwd_launch(void* g, const void* xr, void* dr, const float* row_w, const int32_t* n_rows, int64_t rows_cap,
                      int d, float* dw_row, cudaStream_t st) {
  if (rows_cap == 0) return SMOE_OK;
  const unsigned grid = (unsigned)std::min<int64_t>(rows_cap, (int64_t)device_sms() * 16);
  linear_bwd_kernel<T><<<grid, 256, 0, st>>>((T*)g, (const T*)xr, (T*)dr, row_w, n_rows, rows_cap, d, dw_row);
  SMOE_CK(cudaGetLastError());
  return SMOE_OK;
}

template <typename T>
int bwd_tail(const smoe_layer_bwd_args* a, const BwdPlan& p, unsigned char* ws, const void* dxr_rows, cudaStream_t st) {
  const int64_t T_ = a->tokens, d = a->d_model, k = a->top_k;
  const int E = a->num_experts;
  const int32_t* idx = reinterpret_cast<const int32_t*>(ws + p.o_idx);
  const float* w = reinterpret_cast<const float*>(ws + p.o_w);
  const bool vec = d % 8 == 0 && aligned16(a->dx) && aligned16(a->gate_w) && aligned16(dxr_rows);
  const T* dxs = a->num_shared > 0 ? reinterpret_cast<const T*>(ws + p.o_dxs) : nullptr;
  const int64_t items = T_ * (vec ? d / 8 : d);
  const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>(cdiv(items, 256), (int64_t)device_sms() * 32));
  if (T_ > 0) {
    if (vec)
      moe_bwd_dx_kernel<T, 8><<<grid, 256, 0, st>>>(
          reinterpret_cast<const T*>(dxr_rows), reinterpret_cast<const int32_t*>(ws + p.o_sr), idx, w,
          reinterpret_cast<const float*>(ws + p.o_dwr), (const T*)a->gate_w, dxs, (int)T_, (int)k, (int)d, (T*)a->dx,
          reinterpret_cast<const int32_t*>(ws + p.o_srf), reinterpret_cast<float*>(ws + p.o_dsel));
    else
      moe_bwd_dx_kernel<T, 1><<<grid, 256, 0, st>>>(
          reinterpret_cast<const T*>(dxr_rows), reinterpret_cast<const int32_t*>(ws + p.o_sr), idx, w,
          reinterpret_cast<const float*>(ws + p.o_dwr), (const T*)a->gate_w, dxs, (int)T_, (int)k, (int)d, (T*)a->dx,
          reinterpret_cast<const int32_t*>(ws + p.o_srf), reinterpret_cast<float*>(ws + p.o_dsel));
    SMOE_CK(cudaGetLastError());
  }
  // gate gradient: row slices of every expert in parallel, then an in-order sum of the slices
  const int64_t cols = cdiv(d, 256);
  const int slices = (int)std::max<int64_t>(1, std::min<int64_t>(kDwgSlices, cdiv((int64_t)device_sms() * 8, cols * E)));
  dim3 g2((unsigned)cols, (unsigned)E, (unsigned)slices);
  float* part = reinterpret_cast<float*>(ws + p.o_dwgp);
  router_dwg_kernel<T><<<g2, 256, 0, st>>>((const T*)a->x, reinterpret_cast<const int32_t*>(ws + p.o_rtf),
                                           reinterpret_cast<const int32_t*>(ws + p.o_offf),
                                           reinterpret_cast<const float*>(ws + p.o_dsel), (int)d, E, part);
  SMOE_CK(cudaGetLastError());
  const int64_t n = (int64_t)E * d;
  router_dwg_reduce_kernel<<<(unsigned)std::min<int64_t>(cdiv(n, 256), (int64_t)device_sms() * 8), 256, 0, st>>>(
      part, slices, n, a->dgate);
  SMOE_CK(cudaGetLastError());
  return SMOE_OK;
}
}  // namespace

namespace {
// Shared expert backward: one group of all T rows with weight 1; its input gradient
// goes to the dxs slab of the workspace, its weight gradients to dsw13 / dsw2.
int bwd_shared(const smoe_layer_bwd_args* a, const BwdPlan& p, unsigned char* ws, cudaStream_t st) {
  const int Fs = a->num_shared ? a->d_ff_shared : 0;
  if (!Fs) return SMOE_OK;
  const int T = a->tokens, d = a->d_model, dt = a->dtype;
  smoe_stream_t stream = (smoe_stream_t)st;
  int rc;
  int32_t* soff = reinterpret_cast<int32_t*>(ws + p.o_soff);
  SMOE_CK(launch_k(fill_two_kernel, 1, 1, 0, st, soff, 0, T));
  SMOE_CK(cudaGetLastError());
  void* abs_ = ws + p.o_abs;
  void* gs = ws + p.o_gs;
  if ((rc = grouped_gemm_impl(a->x, a->sw1, a->sw3, abs_, dt, dt, SMOE_EPI_GATEUP, soff, nullptr, 1, T, Fs, d, st)))
    return rc;
  if ((rc = grouped_gemm_impl(a->dout, a->sw2t, nullptr, gs, dt, dt, SMOE_EPI_STORE, soff, nullptr, 1, T, Fs, d, st)))
    return rc;
  rc = dt == SMOE_BF16 ? swiglu_bwd_launch<__nv_bfloat16>(abs_, gs, nullptr, nullptr, T, Fs, nullptr, st)
                       : swiglu_bwd_launch<__half>(abs_, gs, nullptr, nullptr, T, Fs, nullptr, st);
  if (rc) return rc;
  if ((rc = grouped_gemm_impl(abs_, a->sw13t, nullptr, ws + p.o_dxs, dt, dt, SMOE_EPI_STORE, soff, nullptr, 1, T, d,
                              2 * Fs, st)))
    return rc;
  // weight gradients of the shared expert: K = the T tokens, rows read as they are
  if ((rc = smoe_wgrad_gemm_rows(abs_, 2 * Fs, a->x, d, dt, soff, 1, 2 * Fs, d, T, a->dsw13, stream))) return rc;
  if ((rc = smoe_wgrad_gemm_rows(a->dout, d, gs, Fs, dt, soff, 1, d, Fs, T, a->dsw2, stream))) return rc;
  return SMOE_OK;
}

}  // namespace

extern "C" {

size_t smoe_layer_bwd_workspace_size(const smoe_layer_bwd_args* a) {
  BwdPlan p;
  if (!a || !bwd_plan(a, &p)) return 0;
  return p.total;
}

int smoe_layer_bwd(const smoe_layer_bwd_args* a, smoe_stream_t stream) {
  if (!a) return SMOE_ERR_INVALID;
  cudaStream_t st = (cudaStream_t)stream;
  const bool lin = a->expert_type == SMOE_EXPERT_LINEAR;
  if (!lin && a->expert_type != SMOE_EXPERT_SWIGLU) return SMOE_ERR_INVALID;
  const int T = a->tokens, d = a->d_model, E = a->num_experts, k = a->top_k, F = lin ? 0 : a->d_ff, dt = a->dtype;
  if (T < 0 || d < 1 || E < 1 || k < 1 || k > E || (!lin && F < 1)) return SMOE_ERR_INVALID;
  if (dt != SMOE_BF16 && dt != SMOE_F16) return SMOE_ERR_UNSUPPORTED;
  if (d % 8 != 0 || F % 8 != 0 || E > tc::MAX_GROUPS) return SMOE_ERR_UNSUPPORTED;
  if (a->num_shared < 0 || a->num_shared > 1) return SMOE_ERR_UNSUPPORTED;
  const int Fs = a->num_shared ? a->d_ff_shared : 0;
  if (a->num_shared && (Fs < 1 || Fs % 8 != 0 || !a->sw1 || !a->sw3 || !a->sw2t || !a->sw13t || !a->dsw13 || !a->dsw2))
    return SMOE_ERR_INVALID;
  if (!a->gate_w || !a->dgate) return SMOE_ERR_INVALID;
  if (lin ? (!a->w_lin_t || !a->dw_lin) : (!a->w1 || !a->w3 || !a->w2t || !a->w13t || !a->dw13 || !a->dw2))
    return SMOE_ERR_INVALID;
  if (T > 0 && (!a->x || !a->dout || !a->dx)) return SMOE_ERR_INVALID;
  BwdPlan p;
  bwd_plan(a, &p);
  if (!a->workspace || a->workspace_bytes < p.total) return SMOE_ERR_WORKSPACE;
  if (T == 0) {  // no tokens: every gradient is zero
    SMOE_CK(cudaMemsetAsync(a->dgate, 0, (size_t)E * d * 4, st));
    if (lin) {
      SMOE_CK(cudaMemsetAsync(a->dw_lin, 0, (size_t)E * d * d * 4, st));
    } else {
      SMOE_CK(cudaMemsetAsync(a->dw13, 0, (size_t)E * 2 * F * d * 4, st));
      SMOE_CK(cudaMemsetAsync(a->dw2, 0, (size_t)E * d * F * 4, st));
    }
    if (Fs) {
      SMOE_CK(cudaMemsetAsync(a->dsw13, 0, (size_t)2 * Fs * d * 4, st));
      SMOE_CK(cudaMemsetAsync(a->dsw2, 0, (size_t)d * Fs * 4, st));
    }
    return SMOE_OK;
  }
  unsigned char* ws = static_cast<unsigned char*>(a->workspace);
  int32_t* idx = reinterpret_cast<int32_t*>(ws + p.o_idx);
  float* w = reinterpret_cast<float*>(ws + p.o_w);
  int32_t* offsets = reinterpret_cast<int32_t*>(ws + p.o_off);
  int32_t* slot_row = reinterpret_cast<int32_t*>(ws + p.o_sr);
  int32_t* row_token = reinterpret_cast<int32_t*>(ws + p.o_rt);
  float* row_w = reinterpret_cast<float*>(ws + p.o_roww);
  float* dw_row = reinterpret_cast<float*>(ws + p.o_dwr);
  void* xr = ws + p.o_xr;
  void* dr = ws + p.o_dr;
  void* ab = ws + p.o_ab;
  void* g = ws + p.o_g;
  void* dxr = ws + p.o_dxr;
  const int64_t S = p.S;
  int rc;
  // routing and dispatch, as in the forward (rows padded to 64 per expert for the K groups)
  rc = smoe_router_fwd(a->x, a->gate_w, dt, a->logit_bias, T, d, E, k, idx, w, nullptr, ws + p.o_rws, p.router_ws,
                       stream);
  if (rc) return rc;
  rc = smoe_dispatch_plan(idx, T, k, E, a->capacity, 64, reinterpret_cast<int32_t*>(ws + p.o_cnt), offsets, slot_row,
                          row_token, S, ws + p.o_pws, p.plan_ws, stream);
  if (rc) return rc;
  rc = smoe_dispatch_plan(idx, T, k, E, 0, 1, reinterpret_cast<int32_t*>(ws + p.o_cntf),
                          reinterpret_cast<int32_t*>(ws + p.o_offf), reinterpret_cast<int32_t*>(ws + p.o_srf),
                          reinterpret_cast<int32_t*>(ws + p.o_rtf), p.rows_cap_full, ws + p.o_pws, p.plan_ws, stream);
  if (rc) return rc;
  if ((rc = smoe_permute_rows(a->x, dt, T, d, row_token, offsets, E, S, xr, stream))) return rc;
  if ((rc = smoe_permute_rows(a->dout, dt, T, d, row_token, offsets, E, S, dr, stream))) return rc;
  SMOE_CK(cudaMemsetAsync(row_w, 0, (size_t)S * 4, st));
  slot_weights_to_rows_kernel<<<(unsigned)std::min<int64_t>(cdiv((int64_t)T * k, 256), (int64_t)device_sms() * 8), 256,
                                0, st>>>(slot_row, w, (int64_t)T * k, row_w);
  SMOE_CK(cudaGetLastError());
  if (lin) {  // g = dout_r Wl; the element-wise step turns it into the rows' input gradient
    if ((rc = grouped_gemm_impl(dr, a->w_lin_t, nullptr, g, dt, dt, SMOE_EPI_STORE, offsets, nullptr, E, S, d, d, st)))
      return rc;
    rc = dt == SMOE_BF16 ? linear_bwd_launch<__nv_bfloat16>(g, xr, dr, row_w, offsets + E, S, d, dw_row, st)
                         : linear_bwd_launch<__half>(g, xr, dr, row_w, offsets + E, S, d, dw_row, st);
    if (rc) return rc;
    if ((rc = bwd_shared(a, p, ws, st))) return rc;
    rc = dt == SMOE_BF16 ? bwd_tail<__nv_bfloat16>(a, p, ws, g, st) : bwd_tail<__half>(a, p, ws, g, st);
    if (rc) return rc;
    return a->dw_lin_transposed ? smoe_wgrad_gemm_rows(xr, d, dr, d, dt, offsets, E, d, d, S, a->dw_lin, stream)
                                : smoe_wgrad_gemm_rows(dr, d, xr, d, dt, offsets, E, d, d, S, a->dw_lin, stream);
  }
  // recomputed pre-activations, the gradient reaching h, the element-wise backward
  if ((rc = grouped_gemm_impl(xr, a->w1, a->w3, ab, dt, dt, SMOE_EPI_GATEUP, offsets, nullptr, E, S, F, d, st))) return rc;
  if ((rc = grouped_gemm_impl(dr, a->w2t, nullptr, g, dt, dt, SMOE_EPI_STORE, offsets, nullptr, E, S, F, d, st))) return rc;
  rc = dt == SMOE_BF16 ? swiglu_bwd_launch<__nv_bfloat16>(ab, g, row_w, offsets + E, S, F, dw_row, st)
                       : swiglu_bwd_launch<__half>(ab, g, row_w, offsets + E, S, F, dw_row, st);
  if (rc) return rc;
  // input gradient of the routed rows: [da | db] against [W1 | W3]
  if ((rc = grouped_gemm_impl(ab, a->w13t, nullptr, dxr, dt, dt, SMOE_EPI_STORE, offsets, nullptr, E, S, d, 2 * F, st)))
    return rc;
  if ((rc = bwd_shared(a, p, ws, st))) return rc;
  // dx (routed rows + shared expert + router) and the gate's gradient
  rc = dt == SMOE_BF16 ? bwd_tail<__nv_bfloat16>(a, p, ws, dxr, st) : bwd_tail<__half>(a, p, ws, dxr, st);
  if (rc) return rc;
  // expert weight gradients: K runs over the routed rows, grouped by expert (rows read as
  // they are, as MN-major tiles)
  if ((rc = smoe_wgrad_gemm_rows(ab, 2 * F, xr, d, dt, offsets, E, 2 * F, d, S, a->dw13, stream))) return rc;
  return smoe_wgrad_gemm_rows(dr, d, g, F, dt, offsets, E, d, F, S, a->dw2, stream);
}

// ---- the layer backward in pieces, for expert parallelism: the routed rows' part runs on
// the rank that owns their experts, the tokens' part on the tokens' own rank.

int smoe_swiglu_bwd(void* ab, void* g, const float* row_w, const int32_t* n_rows, int64_t rows_cap, int F, int dtype,
                    float* dw_row, smoe_stream_t stream) {
  if (rows_cap < 0 || F < 1) return SMOE_ERR_INVALID;
  if (dtype != SMOE_BF16 && dtype != SMOE_F16) return SMOE_ERR_UNSUPPORTED;
  if (F % 8 != 0) return SMOE_ERR_UNSUPPORTED;
  if (rows_cap == 0) return SMOE_OK;
  if (!ab || !g) return SMOE_ERR_INVALID;
  if (!aligned16(ab) || !aligned16(g)) return SMOE_ERR_UNSUPPORTED;
  cudaStream_t st = (cudaStream_t)stream;
  return dtype == SMOE_BF16 ? swiglu_bwd_launch<__nv_bfloat16>(ab, g, row_w, n_rows, rows_cap, F, dw_row, st)
                            : swiglu_bwd_launch<__half>(ab, g, row_w, n_rows, rows_cap, F, dw_row, st);
}

int smoe_linear_bwd(void* g, const void* xr, void* dr, const float* row_w, const int32_t* n_rows, int64_t rows_cap,
                    int d, int dtype, float* dw_row, smoe_stream_t stream) {
  if (rows_cap < 0 || d < 1) return SMOE_ERR_INVALID;
  if (dtype != SMOE_BF16 && dtype != SMOE_F16) return SMOE_ERR_UNSUPPORTED;
  if (d % 8 != 0) return SMOE_ERR_UNSUPPORTED;
  if (rows_cap == 0) return SMOE_OK;
  if (!g || !xr || !dr || !row_w || !n_rows || !dw_row) return SMOE_ERR_INVALID;
  if (!aligned16(g) || !aligned16(xr) || !aligned16(dr)) return SMOE_ERR_UNSUPPORTED;
  cudaStream_t st = (cudaStream_t)stream;
  return dtype == SMOE_BF16 ? linear_bwd_launch<__nv_bfloat16>(g, xr, dr, row_w, n_rows, rows_cap, d, dw_row, st)
                            : linear_bwd_launch<__half>(g, xr, dr, row_w, n_rows, rows_cap, d, dw_row, st);
}

int smoe_moe_bwd_dx(const void* dxr, const int32_t* slot_row, const int32_t* idx, const float* w, const float* dw_row,
                    const void* gate_w, const void* dxs, int T, int k, int d, int dtype, void* dx,
                    const int32_t* slot_row_full, float* dsel_row, smoe_stream_t stream) {
  if (T < 0 || k < 1 || d < 1) return SMOE_ERR_INVALID;
  if (dtype != SMOE_BF16 && dtype != SMOE_F16) return SMOE_ERR_UNSUPPORTED;
  if (T == 0) return SMOE_OK;
  if (!dxr || !slot_row || !idx || !w || !dw_row || !gate_w || !dx) return SMOE_ERR_INVALID;
  if (dsel_row && !slot_row_full) return SMOE_ERR_INVALID;
  cudaStream_t st = (cudaStream_t)stream;
  const bool vec = d % 8 == 0 && aligned16(dx) && aligned16(gate_w) && aligned16(dxr) && (!dxs || aligned16(dxs));
  const int64_t items = (int64_t)T * (vec ? d / 8 : d);
  const unsigned grid = (unsigned)std::max<int64_t>(1, std::min<int64_t>(cdiv(items, 256), (int64_t)device_sms() * 32));
#define SMOE_BWD_DX(TY, VV)                                                                                          \
  moe_bwd_dx_kernel<TY, VV><<<grid, 256, 0, st>>>((const TY*)dxr, slot_row, idx, w, dw_row, (const TY*)gate_w,        \
                                                  (const TY*)dxs, T, k, d, (TY*)dx, slot_row_full, dsel_row)
  if (dtype == SMOE_BF16) {
    if (vec) SMOE_BWD_DX(__nv_bfloat16, 8); else SMOE_BWD_DX(__nv_bfloat16, 1);
  } else {
    if (vec) SMOE_BWD_DX(__half, 8); else SMOE_BWD_DX(__half, 1);
  }
#undef SMOE_BWD_DX
  SMOE_CK(cudaGetLastError());
  return SMOE_OK;
}

size_t smoe_router_dwg_workspace_size(int d, int E) {
  if (d < 1 || E < 1) return 0;
  return (size_t)kDwgSlices * E * d * sizeof(float);
}

int smoe_router_dwg(const void* x, const int32_t* row_token_full, const int32_t* offsets_full, const float* dsel_row,
                    int d, int E, int dtype, float* dgate, void* workspace, size_t workspace_bytes,
                    smoe_stream_t stream) {
  if (d < 1 || E < 1) return SMOE_ERR_INVALID;
  if (dtype != SMOE_BF16 && dtype != SMOE_F16) return SMOE_ERR_UNSUPPORTED;
  if (!x || !row_token_full || !offsets_full || !dsel_row || !dgate) return SMOE_ERR_INVALID;
  if (!workspace || workspace_bytes < smoe_router_dwg_workspace_size(d, E)) return SMOE_ERR_WORKSPACE;
  cudaStream_t st = (cudaStream_t)stream;
  const int64_t cols = cdiv(d, 256);
  const int slices = (int)std::max<int64_t>(1, std::min<int64_t>(kDwgSlices, cdiv((int64_t)device_sms() * 8, cols * E)));
  dim3 g2((unsigned)cols, (unsigned)E, (unsigned)slices);
  float* part = static_cast<float*>(workspace);
  if (dtype == SMOE_BF16)
    router_dwg_kernel<__nv_bfloat16><<<g2, 256, 0, st>>>((const __nv_bfloat16*)x, row_token_full, offsets_full, dsel_row,
                                                         d, E, part);
  else
    router_dwg_kernel<__half><<<g2, 256, 0, st>>>((const __half*)x, row_token_full, offsets_full, dsel_row, d, E, part);
  SMOE_CK(cudaGetLastError());
  const int64_t n = (int64_t)E * d;
  router_dwg_reduce_kernel<<<(unsigned)std::min<int64_t>(cdiv(n, 256), (int64_t)device_sms() * 8), 256, 0, st>>>(
      part, slices, n, dgate);
  SMOE_CK(cudaGetLastError());
  return SMOE_OK;
}

}  // extern "C"

// Allocation-free dispatch plan (static device scratch); see noalloc_plan.cu.
#include "noalloc_plan.cu"
