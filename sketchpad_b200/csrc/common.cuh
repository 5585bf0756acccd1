// common.cuh -- host-side helpers shared by the C-ABI entry points: status/error reporting,
// dtype sizes, the TMA descriptor encoder (fetched from the driver at run time), and
// launch checking.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/sketchpad_b200.h"

namespace sp {

// Records a printf-style message for sp_last_error() and returns `status`.
int set_error(int status, const char* fmt, ...);
void clear_error();

inline int dtype_size(int dt) {
  switch (dt) {
    case SP_F32: return 4;
    case SP_F16: return 2;
    case SP_BF16: return 2;
    default: return 0;
  }
}

inline bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Checks cudaGetLastError after a launch; returns SP_OK or SP_ERR_LAUNCH with a message.
int check_launch(const char* what);

// Returns SP_OK if the current device is sm_100 (B200/GB200 class), else SP_ERR_DEVICE.
int require_sm100();

// SM count of the current device (cached per device).
int num_sms();

// Current device index (cudaGetDevice; 0 on failure).
int current_device();

// True once per (flag, device): lets a launcher set a kernel attribute the first time it
// runs on a device instead of on every call.
bool first_time_on_device(unsigned long long* flag_bits);
cudaMemPool_t scratch_pool();

// cuTensorMapEncodeTiled obtained through cudaGetDriverEntryPoint (no libcuda link).
int encode_tiled(CUtensorMap* map, CUtensorMapDataType dt, uint32_t rank, const void* base,
                 const uint64_t* dims, const uint64_t* strides_bytes, const uint32_t* box,
                 CUtensorMapSwizzle swizzle);

// Channels-last GroupNorm (groupnorm_nhwc.cu).
bool gn_nhwc_applicable(int64_t B, int64_t C, int64_t H, int64_t W, const int64_t* x_strides, int es,
                        int64_t groups);
size_t gn_nhwc_workspace_bytes(int64_t B, int64_t C, int64_t H, int64_t W, int es, int64_t groups);
int gn_nhwc_launch(const void* x, const void* x_add, const void* gamma, const void* beta, void* y,
                   int64_t B, int64_t C, int64_t H, int64_t W, int64_t groups, float eps, int act,
                   int dtype, void* workspace, size_t workspace_bytes, cudaStream_t s);

}  // namespace sp
