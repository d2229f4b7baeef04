// Allocation-free C entry point for the MoE dispatch plan.
//
// This entry point has no counterpart in the reference; it is an addition of
// this library.
//
// Who it is for: callers that cannot allocate device memory at the moment they
// need a dispatch plan.  Examples are an inference or serving engine that
// reserves one fixed device arena at start-up and forbids any later
// allocation (an allocation in the middle of a request could fail or stall
// behind other tenants), and plain C/C++ programs that load this library with
// dlopen and have no PyTorch caching allocator at all.  The PyTorch entry point
// `moe_plan` allocates its outputs and a per-block count table on every call;
// this one writes into buffers the caller already owns and keeps its scratch
// in a fixed device array compiled into the library.
//
//   The exported prototypes and return codes are declared in csrc/pm_noalloc.h.
//
// Inputs and outputs have the meaning and shapes of `moe_plan`:
//   idx [n] int32 (n = tokens * k, top-k expert ids), lut optional (logical ->
//   slot), weights optional fp32 [n]; outputs offsets [num_slots + 1],
//   counts [num_slots], row_of [n], row_token [capacity], row_scale [capacity].
//   The padded segments end at offsets[num_slots] <= n + num_slots * (align - 1), and
//   the kernels write row_token / row_scale up to that row, so a capacity below that
//   bound is rejected with PM_NOALLOC_BAD_ARGS before anything is launched.
// Returns 0 on success, otherwise a nonzero code (see pm_moe_plan_noalloc_error).
//
// Limits: the scratch array holds kNoAllocScratchInts = 262144 int32 (1 MiB) of
// per-block slot counts, so ceil(n / 2048) * num_slots must not exceed 262144
// (for 64 slots: up to 8,388,608 assignments); num_slots <= 1024.  Larger
// requests are rejected with PM_NOALLOC_TOO_LARGE and nothing is launched.
//
// Set-up: the first call on a device looks up the device address of the
// scratch array with cudaGetSymbolAddress (with that device current) and
// caches it per device ordinal.  Make that first call before any stream capture
// on the device.  Every device that loads the library holds the 1 MiB array
// until the process exits.  The address belongs to the device's primary
// context (the one the CUDA runtime uses): use the entry point from the
// runtime's primary context only, and not after cudaDeviceReset() on that
// device, which destroys the context the cached address refers to.  The
// first-call look-up is serialised by a mutex, so threads may race to make it.
//
// Sharing: all calls on one device share the one scratch array, and the array
// keeps the contents of the last call.  The count kernel writes every scratch
// entry it later reads, so nothing needs clearing between calls.  Two calls
// whose kernels overlap on the GPU (different streams without ordering between
// them) race on the array and produce wrong plans: order them on one stream or
// with events.
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "common.cuh"
#include "pm_noalloc.h"

namespace pm {
// Kernels of the allocating entry point (moe_route.cu), reused unchanged.
constexpr int kPlanChunkNA = 2048;
constexpr int kPlanWarpsNA = 8;
__global__ void __launch_bounds__(256) plan_count_kernel(const int* __restrict__ idx, const int* __restrict__ lut, int n, int num_slots,
                                  int* __restrict__ block_counts);
__global__ void __launch_bounds__(1024) plan_scan_kernel(int* __restrict__ block_counts, int nblocks, int num_slots, int align,
                                 int* __restrict__ offsets, int* __restrict__ counts);
__global__ void __launch_bounds__(256) plan_scatter_kernel(const int* __restrict__ idx, const int* __restrict__ lut,
                                    const float* __restrict__ w, int n, int K, int num_slots,
                                    const int* __restrict__ block_base, const int* __restrict__ offsets,
                                    int* __restrict__ row_of, int* __restrict__ row_token,
                                    float* __restrict__ row_scale);
__global__ void plan_pad_kernel(const int* __restrict__ offsets, const int* __restrict__ counts, int num_slots,
                                int* __restrict__ row_token, float* __restrict__ row_scale);
}  // namespace pm

namespace {

constexpr int kNoAllocScratchInts = 262144;  // 1 MiB
constexpr int kMaxDevices = 64;

// The scratch array.  In host code `g_noalloc_scratch` is only a host-side
// stand-in for the symbol: its device address comes from cudaGetSymbolAddress.
static __device__ __align__(256) int g_noalloc_scratch[kNoAllocScratchInts];

int* g_scratch_ptr[kMaxDevices] = {nullptr};
std::mutex g_scratch_mu;

thread_local const char* g_last_error = "ok";

int fail(int code, const char* msg) {
  g_last_error = msg;
  return code;
}

// Records the CUDA error name of a failed launch; returns true on failure.
bool launch_status(cudaError_t e) {
  if (e == cudaSuccess) return false;
  g_last_error = cudaGetErrorName(e);
  return true;
}

}  // namespace

extern "C" {

// Message of the last failing call on this thread (a CUDA error name for launch failures).
const char* pm_moe_plan_noalloc_error(void) { return g_last_error; }

// Scratch capacity in int32 entries (the limit on ceil(n / 2048) * num_slots).
int pm_moe_plan_noalloc_scratch_ints(void) { return kNoAllocScratchInts; }

int pm_moe_plan_noalloc(const int* idx, const int* lut, const float* weights, int n, int k, int num_slots,
                        int capacity, int align, int* offsets, int* counts, int* row_of, int* row_token,
                        float* row_scale, cudaStream_t stream) {
  if (n < 0 || k <= 0 || num_slots <= 0 || num_slots > 1024 || align <= 0 || capacity < 0)
    return fail(PM_NOALLOC_BAD_ARGS, "invalid size arguments (need n >= 0, k > 0, 0 < num_slots <= 1024, align > 0)");
  if (!idx || !offsets || !counts || !row_of || !row_token || !row_scale)
    return fail(PM_NOALLOC_BAD_ARGS, "a required pointer is null");
  int nblocks = n > 0 ? (n + pm::kPlanChunkNA - 1) / pm::kPlanChunkNA : 1;
  if ((long long)nblocks * num_slots > kNoAllocScratchInts)
    return fail(PM_NOALLOC_TOO_LARGE,
                "request exceeds the fixed scratch: ceil(n / 2048) * num_slots must be <= 262144");
  // the padded plan ends at offsets[num_slots] <= n + num_slots * (align - 1)
  if ((long long)capacity < (long long)n + (long long)num_slots * (align - 1))
    return fail(PM_NOALLOC_BAD_ARGS, "capacity below n + num_slots * (align - 1) rows");
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return fail(PM_NOALLOC_SYMBOL, "cudaGetDevice failed or device index out of range");
  int* block_counts = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (g_scratch_ptr[dev] == nullptr) {
      void* ptr = nullptr;
      const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
      if (e != cudaSuccess || ptr == nullptr) return fail(PM_NOALLOC_SYMBOL, "cudaGetSymbolAddress(scratch) failed");
      g_scratch_ptr[dev] = static_cast<int*>(ptr);
    }
    block_counts = g_scratch_ptr[dev];
  }
  // cudaLaunchKernel reports the status of each launch itself, independent of any
  // error state left in the runtime by earlier, unrelated calls of the process.
  {
    void* args[] = {&idx, &lut, &n, &num_slots, &block_counts};
    if (launch_status(cudaLaunchKernel((const void*)pm::plan_count_kernel, dim3(nblocks), dim3(256), args,
                                       num_slots * sizeof(int), stream)))
      return PM_NOALLOC_LAUNCH;
  }
  {
    void* args[] = {&block_counts, (void*)&nblocks, &num_slots, &align, &offsets, &counts};
    if (launch_status(cudaLaunchKernel((const void*)pm::plan_scan_kernel, dim3(1), dim3(1024), args, 0, stream)))
      return PM_NOALLOC_LAUNCH;
  }
  const size_t smem = (size_t)pm::kPlanWarpsNA * num_slots * sizeof(int);
  // The scatter kernel's dynamic shared-memory limit is a per-function attribute that
  // other callers of the same kernel may have lowered; raise it to the largest request
  // this entry point can make (1024 slots) before every launch.
  if (launch_status(cudaFuncSetAttribute((const void*)pm::plan_scatter_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         pm::kPlanWarpsNA * 1024 * (int)sizeof(int))))
    return PM_NOALLOC_LAUNCH;
  {
    const int* bb = block_counts;
    void* args[] = {&idx, &lut, &weights, &n, &k, &num_slots, &bb, &offsets, &row_of, &row_token, &row_scale};
    if (launch_status(cudaLaunchKernel((const void*)pm::plan_scatter_kernel, dim3(nblocks), dim3(256), args, smem,
                                       stream)))
      return PM_NOALLOC_LAUNCH;
  }
  {
    void* args[] = {&offsets, &counts, &num_slots, &row_token, &row_scale};
    if (launch_status(cudaLaunchKernel((const void*)pm::plan_pad_kernel, dim3(num_slots), dim3(128), args, 0,
                                       stream)))
      return PM_NOALLOC_LAUNCH;
  }
  g_last_error = "ok";
  return PM_NOALLOC_OK;
}

}  // extern "C"
