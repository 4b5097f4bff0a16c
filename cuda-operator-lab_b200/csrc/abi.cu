// Library-level exports: error strings and device/build information.
#include "common.cuh"

#ifndef COL_BUILD_TAG
#define COL_BUILD_TAG "dev"
#endif

COL_API const char* cuda_operator_error_string(int code) {
  switch (code) {
    case col::kErrNoTensorMapEncoder:
      return "the CUDA driver does not provide cuTensorMapEncodeTiled";
    case col::kErrTensorMapEncode:
      return "cuTensorMapEncodeTiled rejected a GEMM operand layout";
    case col::kErrDeviceNotSupported:
      return "the tensor-core GEMM needs a compute capability 10.x (sm_100) device";
    case col::kErrNoAllocCapacity:
      return "cuda_operator_lab_reduction_noalloc accepts at most 268435456 (2^28) elements";
    case col::kErrGatherLayout:
      return "the gathering GEMM needs k a multiple of 8 and 16-byte aligned x and weight";
    default:
      return cudaGetErrorString(static_cast<cudaError_t>(code));
  }
}

COL_API int cuda_operator_lab_device_info(int* sm_count, int* cc_major, int* cc_minor) {
  if (!sm_count || !cc_major || !cc_minor) return static_cast<int>(cudaErrorInvalidValue);
  int count = 0;
  const cudaError_t e = cudaGetDeviceCount(&count);
  if (e != cudaSuccess) return static_cast<int>(e);
  const col::DeviceInfo& info = col::device_info();
  *sm_count = info.sm_count;
  *cc_major = info.cc_major;
  *cc_minor = info.cc_minor;
  return 0;
}

COL_API const char* cuda_operator_lab_build_tag(void) { return "cuda-operator-lab-b200 sm_100a " COL_BUILD_TAG; }
