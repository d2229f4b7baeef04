// Public C interface of the allocation-free MoE dispatch-plan entry point
// (kernels/moe_plan_noalloc.cu, exported from the pm_kernels shared library).
//
// This entry point has no counterpart in the reference; it is an addition of
// this library for callers that cannot allocate device memory when they need
// a dispatch plan (a serving engine that reserves one fixed device arena at
// start-up, a C program without PyTorch's caching allocator).  Semantics,
// limits and the sharing rules of its fixed scratch array are documented at
// the definition.
#pragma once

#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

// Return codes of pm_moe_plan_noalloc.
#define PM_NOALLOC_OK 0
#define PM_NOALLOC_BAD_ARGS 1    // a size or pointer argument is invalid (nothing launched)
#define PM_NOALLOC_TOO_LARGE 2   // the request needs more than the fixed scratch (nothing launched)
#define PM_NOALLOC_SYMBOL 3      // the scratch array's device address could not be obtained
#define PM_NOALLOC_LAUNCH 4      // a kernel launch failed (message: pm_moe_plan_noalloc_error)

// Dispatch plan of n = tokens * k assignments into `num_slots` expert segments padded to
// `align` rows.  Outputs are caller-owned device buffers: offsets [num_slots + 1],
// counts [num_slots], row_of [n], row_token [capacity], row_scale [capacity], with
// capacity >= n + num_slots * (align - 1).  `lut` (logical -> slot) and `weights` may be NULL.
int pm_moe_plan_noalloc(const int* idx, const int* lut, const float* weights, int n, int k, int num_slots,
                        int capacity, int align, int* offsets, int* counts, int* row_of, int* row_token,
                        float* row_scale, cudaStream_t stream);

// Message of the last failing call on the calling thread ("ok" after a success).
const char* pm_moe_plan_noalloc_error(void);

// Size of the fixed scratch array in int32 entries: ceil(n / 2048) * num_slots must not exceed it.
int pm_moe_plan_noalloc_scratch_ints(void);

#ifdef __cplusplus
}
#endif
