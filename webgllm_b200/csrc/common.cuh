// Shared host/device helpers of the Q4 library.
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <string>

#include "../../include/webgllm_q4.h"

namespace wg {

// Number of SMs of a B200 (2 dies x 74); the launch heuristics read the
// device's own count and fall back to this.
constexpr int kB200Sms = 148;

// Status of a CUDA runtime call as a WG_* code.
inline int status_of(cudaError_t e) {
  switch (e) {
    case cudaSuccess:
      return WG_OK;
    case cudaErrorMemoryAllocation:
      return WG_OUT_OF_MEMORY;
    case cudaErrorNoDevice:
    case cudaErrorInvalidDevice:
    case cudaErrorInsufficientDriver:
      return WG_NO_DEVICE;
    case cudaErrorIllegalAddress:
    case cudaErrorLaunchFailure:
    case cudaErrorIllegalInstruction:
    case cudaErrorMisalignedAddress:
    case cudaErrorHardwareStackError:
    case cudaErrorInvalidPc:
    case cudaErrorAssert:
    case cudaErrorECCUncorrectable:
      return WG_DEVICE_LOST;
    default:
      return WG_CUDA_ERROR;
  }
}

// Device-side error flags written by kernels that wait with a bound (set
// bits are reported by wg_sync as WG_TIMEOUT).
enum DeviceFlag : unsigned {
  kFlagTimeout = 1u,
  kFlagBadArgument = 2u,
};

__device__ __forceinline__ void raise_flag(unsigned *flags, unsigned bit) {
  if (flags) atomicOr(flags, bit);
}

}  // namespace wg
