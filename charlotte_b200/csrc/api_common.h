// Shared host-side plumbing of the C ABI: status codes, the thread-local
// error message, device facts.
#pragma once

#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <string>

#include "charlotte_b200.h"

namespace cb {

// Records `message` as the calling thread's last error and returns `status`.
int fail(int status, const char* format, ...);

// A CUDA error as a status: a sticky device error is CB_ERROR_DEVICE_LOST
// (the context is unusable, as WebGPU's lost device is), any other
// CB_ERROR_STEP; the message names `what`.
int fail_cuda(cudaError_t e, const char* what);

// The current device's SM count (cached per device).
int sm_count();

// The current device's fault word: kernels whose bounded waits run out set
// bits in it; cb_fault_check reads and clears it.
unsigned int* fault_word();

// cb_select's preconditions, shared by cb_select_run and
// cb_select_run_static: `who` names the entry point in the message; with
// own_scratch the caller's partials and ticket are not required (the entry
// point brings its own). CB_OK or CB_ERROR_INVALID.
int select_arguments(const cb_select* s, const char* who, bool own_scratch);

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace cb
