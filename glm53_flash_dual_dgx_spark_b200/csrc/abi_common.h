// Host-side helpers shared by the C-ABI launchers: per-thread error messages and
// per-device attribute caches.  No torch types appear anywhere in this library.
#pragma once

#include <cuda_runtime.h>
#include <stdarg.h>
#include <stdio.h>

#include "../../include/nvfp4kv.h"

namespace nvfp4kv {

// Records a formatted message for nvfp4kv_last_error() and returns `code`.
int fail(int code, const char* fmt, ...);

// Returns NVFP4KV_ECUDA with the runtime's message when the last launch failed.
int check_launch(const char* what);

// Number of SMs of the current device (cached per device).
int device_sm_count();

// Measurement hook (nvfp4kv_set_kernel_events): events to record around the next main
// attention kernel launched by the calling thread.  Returns them and clears the hook.
void take_kernel_events(cudaEvent_t* start, cudaEvent_t* stop);

}  // namespace nvfp4kv
