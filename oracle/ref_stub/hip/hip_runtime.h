/*
 * Stub of the HIP runtime header, just enough for the reference's host file
 * (fmha_host.cpp) to compile with g++ on a machine without ROCm. Only the
 * reference's CPU functions (FMHAConfig, do_validation) are ever called from
 * oracle/ref_shim.cpp; every runtime entry point here is an inert template
 * that is compiled but never executed. Test infrastructure only.
 */
#pragma once
#include <cstddef>
#include <stdexcept>

typedef int hipError_t;
static const hipError_t hipSuccess = 0;
typedef void* hipStream_t;
typedef void* hipEvent_t;
enum hipMemcpyKind { hipMemcpyHostToDevice = 1, hipMemcpyDeviceToHost = 2 };
struct dim3 {
  unsigned x, y, z;
  dim3(unsigned a = 1, unsigned b = 1, unsigned c = 1) : x(a), y(b), z(c) {}
};
struct hipDeviceProp_t {
  char name[256];
  int major, minor;
  std::size_t totalGlobalMem;
};
inline const char* hipGetErrorString(hipError_t) { return "hip stub"; }
#define FMHA_REF_STUB(name) \
  template <class... A> inline hipError_t name(A...) { throw std::logic_error(#name " is a stub"); }
FMHA_REF_STUB(hipMalloc)
FMHA_REF_STUB(hipFree)
FMHA_REF_STUB(hipMemcpy)
FMHA_REF_STUB(hipMemset)
FMHA_REF_STUB(hipEventCreate)
FMHA_REF_STUB(hipEventRecord)
FMHA_REF_STUB(hipEventSynchronize)
FMHA_REF_STUB(hipEventElapsedTime)
FMHA_REF_STUB(hipEventDestroy)
FMHA_REF_STUB(hipDeviceSynchronize)
FMHA_REF_STUB(hipGetDeviceCount)
FMHA_REF_STUB(hipGetDeviceProperties)
#undef FMHA_REF_STUB
