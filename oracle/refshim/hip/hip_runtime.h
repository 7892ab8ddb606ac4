/*
 * Host-memory stand-in for the HIP runtime API, used only to compile the
 * reference's device headers as plain C++ for the CPU oracle.
 *
 * The reference selects its HIP macro layer with CARL_USE_HIP
 * (include/Cuda/Common.cuh:6-35), which renames every cuda* call it makes to a
 * hip* call.  This header supplies those hip* names over malloc/memcpy/memset so
 * that `DeviceArray<T>` (include/Cuda/DeviceArray.cuh) allocates host memory.
 * TEST INFRASTRUCTURE: only tests, smoke() and bench.py's CPU baseline use it.
 */
#pragma once

#include <cstddef>
#include <cstdlib>
#include <cstring>

typedef int hipError_t;
typedef void* hipEvent_t;
typedef void* hipStream_t;

enum { hipSuccess = 0, hipErrorNotReady = 600, hipErrorMemoryAllocation = 2 };
enum hipMemcpyKind {
    hipMemcpyHostToHost = 0,
    hipMemcpyHostToDevice = 1,
    hipMemcpyDeviceToHost = 2,
    hipMemcpyDeviceToDevice = 3
};

struct hipDeviceProp_t { int multiProcessorCount; };

template <class T>
inline hipError_t hipMalloc(T** ptr, size_t bytes)
{
    *ptr = static_cast<T*>(std::calloc(bytes ? bytes : 1, 1));
    return *ptr ? hipSuccess : hipErrorMemoryAllocation;
}
inline hipError_t hipFree(void* ptr) { std::free(ptr); return hipSuccess; }
inline hipError_t hipMemcpy(void* dst, const void* src, size_t bytes, hipMemcpyKind)
{
    if (bytes) std::memcpy(dst, src, bytes);
    return hipSuccess;
}
inline hipError_t hipMemcpyAsync(void* dst, const void* src, size_t bytes, hipMemcpyKind k,
                                 hipStream_t = nullptr)
{
    return hipMemcpy(dst, src, bytes, k);
}
inline hipError_t hipMemset(void* dst, int value, size_t bytes)
{
    if (bytes) std::memset(dst, value, bytes);
    return hipSuccess;
}
inline const char* hipGetErrorString(hipError_t) { return "host oracle error"; }
inline hipError_t hipGetLastError() { return hipSuccess; }
inline hipError_t hipGetDeviceProperties(hipDeviceProp_t* p, int)
{
    p->multiProcessorCount = 1;
    return hipSuccess;
}
inline hipError_t hipStreamCreate(hipStream_t* s) { *s = nullptr; return hipSuccess; }
inline hipError_t hipStreamDestroy(hipStream_t) { return hipSuccess; }
inline hipError_t hipStreamSynchronize(hipStream_t) { return hipSuccess; }
inline hipError_t hipEventCreate(hipEvent_t* e) { *e = nullptr; return hipSuccess; }
inline hipError_t hipEventCreateWithFlags(hipEvent_t* e, unsigned) { *e = nullptr; return hipSuccess; }
inline hipError_t hipEventDestroy(hipEvent_t) { return hipSuccess; }
inline hipError_t hipEventRecord(hipEvent_t, hipStream_t = nullptr) { return hipSuccess; }
inline hipError_t hipEventQuery(hipEvent_t) { return hipSuccess; }
inline hipError_t hipEventSynchronize(hipEvent_t) { return hipSuccess; }
inline hipError_t hipEventElapsedTime(float* ms, hipEvent_t, hipEvent_t) { *ms = 0.f; return hipSuccess; }
enum { hipEventDisableTiming = 2 };
