// Dispatch plan with its scratch in a fixed, file-scope device array: an entry point for
// callers that cannot allocate device memory.
//
// Some hosts of this library own every byte of device memory themselves: an inference
// server that carves one arena at start-up, or a framework whose caching allocator must
// be the only allocator in the process.  Such a caller cannot let a library call
// cudaMalloc (it would go around the arena, and cudaMalloc/cudaFree also synchronise
// the device in the middle of a step), and it may not be able to hand out a scratch
// buffer either, because its arena is sized for the tensors it knows about.
// smoe_dispatch_plan_noalloc() needs neither: the per-block histograms and bases live in
// g_plan_scratch below, which every GPU that loads the library keeps until the process
// exits (512 KiB per device).
//
// This file is compiled as part of capi.cu's translation unit (it is #included there),
// so the kernels it launches and the static array are in the same module.
#pragma once

#include <mutex>

namespace smoe {
namespace noalloc {

constexpr int kMaxSlots = SMOE_NOALLOC_PLAN_MAX_SLOTS;     // T * k
constexpr int kMaxExperts = SMOE_NOALLOC_PLAN_MAX_EXPERTS;  // E
constexpr int kMaxBlocks = kMaxSlots / kPlanChunk;          // plan blocks at most
// A call at the slot limit launches cdiv(kMaxSlots, kPlanChunk) plan blocks; the scratch
// holds histograms for kMaxBlocks of them, so the limit must be a whole number of chunks.
static_assert(kMaxSlots % kPlanChunk == 0, "SMOE_NOALLOC_PLAN_MAX_SLOTS must be a multiple of the plan chunk");
constexpr size_t kWords = 2ull * kMaxBlocks * kMaxExperts;  // hist + base

// The scratch: [0, kMaxBlocks*kMaxExperts) histograms, then the per-block bases.
// Every launch writes all the entries it later reads, so nothing has to start at zero;
// the contents left by the previous call are simply overwritten.
static __device__ __align__(256) int32_t g_plan_scratch[kWords];

// Device address of g_plan_scratch per device.  In host code the name g_plan_scratch is
// only a host-side shadow, not a device address, so it is resolved once per device with
// that device current.
int32_t* g_scratch_ptr[kMaxDevices] = {nullptr};
std::mutex g_scratch_mu;

int scratch_for_current_device(int32_t** out) {
  int dev = 0;
  SMOE_CK(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return SMOE_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    SMOE_CK(cudaGetSymbolAddress(&p, g_plan_scratch));
    if (p == nullptr) return SMOE_ERR_CUDA;
    g_scratch_ptr[dev] = static_cast<int32_t*>(p);
  }
  *out = g_scratch_ptr[dev];
  return SMOE_OK;
}

}  // namespace noalloc
}  // namespace smoe

extern "C" int smoe_dispatch_plan_noalloc(const int32_t* idx, int T, int k, int E, int capacity, int row_align,
                                          int32_t* expert_counts, int32_t* expert_offsets, int32_t* slot_row,
                                          int32_t* row_token, int64_t rows_cap, smoe_stream_t stream) {
  using namespace smoe;
  cudaStream_t st = (cudaStream_t)stream;
  if (T < 0 || k < 1 || E < 1 || row_align < 1 || row_align > 1024) return SMOE_ERR_INVALID;
  if (E > noalloc::kMaxExperts || (int64_t)T * k > noalloc::kMaxSlots) return SMOE_ERR_TOO_LARGE;
  if (!expert_counts || !expert_offsets) return SMOE_ERR_INVALID;
  if (rows_cap < smoe_plan_rows_cap(T, k, E, capacity, row_align)) return SMOE_ERR_INVALID;
  if (T > 0 && (!idx || !slot_row || !row_token)) return SMOE_ERR_INVALID;
  int32_t* scratch = nullptr;
  const int rc = noalloc::scratch_for_current_device(&scratch);
  if (rc != SMOE_OK) return rc;
  const int64_t n_slots = (int64_t)T * k;
  const int nb = (int)std::max<int64_t>(1, cdiv(n_slots, kPlanChunk));
  int32_t* hist = scratch;
  int32_t* base = scratch + (size_t)noalloc::kMaxBlocks * noalloc::kMaxExperts;
  // E <= 256: the counting kernels need at most 8 KiB of shared memory (default limit)
  const int smem_w = kPlanWarps * E * (int)sizeof(int);
  plan_count_kernel<<<nb, kPlanThreads, smem_w, st>>>(idx, n_slots, E, hist);
  SMOE_CK(cudaGetLastError());
  plan_scan_kernel<<<1, 1024, E * sizeof(int), st>>>(hist, nb, E, capacity, row_align, base, expert_counts,
                                                     expert_offsets, row_token);
  SMOE_CK(cudaGetLastError());
  if (n_slots > 0) {
    plan_scatter_kernel<<<nb, kPlanThreads, smem_w, st>>>(idx, n_slots, k, E, capacity, base, expert_offsets,
                                                          slot_row, row_token);
    SMOE_CK(cudaGetLastError());
  }
  return SMOE_OK;
}
