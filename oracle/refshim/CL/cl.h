/* Compile-only stand-in for <CL/cl.h>.
 *
 * Test infrastructure: it lets the reference drivers (<variant>/main.cpp,
 * int2_moe/prefill.cpp) compile on a machine without an OpenCL SDK so that their
 * host-gold functions (compute_gold, compute_scale_a, to_sel_layout, ...) can be
 * called from oracle/ref_*.cpp.  Every entry point fails; none is ever called,
 * because the drivers' main() is renamed and never run. */
#pragma once
#include <cstddef>
#include <cstdint>

typedef int32_t cl_int;
typedef uint32_t cl_uint;
typedef uint64_t cl_ulong;
typedef uint8_t cl_uchar;
typedef uint64_t cl_bitfield;
typedef cl_bitfield cl_queue_properties;
typedef cl_bitfield cl_mem_flags;
typedef cl_bitfield cl_device_type;
typedef cl_uint cl_device_info;
typedef cl_uint cl_profiling_info;
typedef cl_uint cl_program_build_info;
typedef cl_uint cl_bool;
typedef struct _cl_platform_id *cl_platform_id;
typedef struct _cl_device_id *cl_device_id;
typedef struct _cl_context *cl_context;
typedef struct _cl_command_queue *cl_command_queue;
typedef struct _cl_mem *cl_mem;
typedef struct _cl_program *cl_program;
typedef struct _cl_kernel *cl_kernel;
typedef struct _cl_event *cl_event;
typedef intptr_t cl_context_properties;

#define CL_SUCCESS 0
#define CL_TRUE 1
#define CL_FALSE 0
#define CL_DEVICE_TYPE_GPU (1 << 2)
#define CL_DEVICE_NAME 0x102B
#define CL_MEM_READ_WRITE (1 << 0)
#define CL_MEM_READ_ONLY (1 << 2)
#define CL_MEM_COPY_HOST_PTR (1 << 5)
#define CL_QUEUE_PROPERTIES 0x1093
#define CL_QUEUE_PROFILING_ENABLE (1 << 1)
#define CL_PROFILING_COMMAND_START 0x1282
#define CL_PROFILING_COMMAND_END 0x1283
#define CL_PROGRAM_BUILD_LOG 0x1183

#define TERNOCL_CL_STUB_FAIL { return -1; }
#define TERNOCL_CL_STUB_NULL { if (e) *e = -1; return nullptr; }
inline cl_int clGetPlatformIDs(cl_uint, cl_platform_id *, cl_uint *) TERNOCL_CL_STUB_FAIL
inline cl_int clGetDeviceIDs(cl_platform_id, cl_device_type, cl_uint, cl_device_id *, cl_uint *) TERNOCL_CL_STUB_FAIL
inline cl_int clGetDeviceInfo(cl_device_id, cl_device_info, size_t, void *, size_t *) TERNOCL_CL_STUB_FAIL
inline cl_context clCreateContext(const cl_context_properties *, cl_uint, const cl_device_id *, void *, void *, cl_int *e) TERNOCL_CL_STUB_NULL
inline cl_command_queue clCreateCommandQueueWithProperties(cl_context, cl_device_id, const cl_queue_properties *, cl_int *e) TERNOCL_CL_STUB_NULL
inline cl_program clCreateProgramWithSource(cl_context, cl_uint, const char **, const size_t *, cl_int *e) TERNOCL_CL_STUB_NULL
inline cl_int clBuildProgram(cl_program, cl_uint, const cl_device_id *, const char *, void *, void *) TERNOCL_CL_STUB_FAIL
inline cl_int clGetProgramBuildInfo(cl_program, cl_device_id, cl_program_build_info, size_t, void *, size_t *) TERNOCL_CL_STUB_FAIL
inline cl_kernel clCreateKernel(cl_program, const char *, cl_int *e) TERNOCL_CL_STUB_NULL
inline cl_mem clCreateBuffer(cl_context, cl_mem_flags, size_t, void *, cl_int *e) TERNOCL_CL_STUB_NULL
inline cl_int clEnqueueFillBuffer(cl_command_queue, cl_mem, const void *, size_t, size_t, size_t, cl_uint, const cl_event *, cl_event *) TERNOCL_CL_STUB_FAIL
inline cl_int clEnqueueNDRangeKernel(cl_command_queue, cl_kernel, cl_uint, const size_t *, const size_t *, const size_t *, cl_uint, const cl_event *, cl_event *) TERNOCL_CL_STUB_FAIL
inline cl_int clEnqueueReadBuffer(cl_command_queue, cl_mem, cl_bool, size_t, size_t, void *, cl_uint, const cl_event *, cl_event *) TERNOCL_CL_STUB_FAIL
inline cl_int clSetKernelArg(cl_kernel, cl_uint, size_t, const void *) TERNOCL_CL_STUB_FAIL
inline cl_int clWaitForEvents(cl_uint, const cl_event *) TERNOCL_CL_STUB_FAIL
inline cl_int clFinish(cl_command_queue) TERNOCL_CL_STUB_FAIL
inline cl_int clGetEventProfilingInfo(cl_event, cl_profiling_info, size_t, void *, size_t *) TERNOCL_CL_STUB_FAIL
inline cl_int clReleaseEvent(cl_event) TERNOCL_CL_STUB_FAIL
inline cl_int clReleaseMemObject(cl_mem) TERNOCL_CL_STUB_FAIL
inline cl_int clReleaseKernel(cl_kernel) TERNOCL_CL_STUB_FAIL
inline cl_int clReleaseProgram(cl_program) TERNOCL_CL_STUB_FAIL
inline cl_int clReleaseCommandQueue(cl_command_queue) TERNOCL_CL_STUB_FAIL
inline cl_int clReleaseContext(cl_context) TERNOCL_CL_STUB_FAIL
