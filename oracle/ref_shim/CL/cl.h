/* Minimal OpenCL 1.1 host API declarations for building the reference's
 * main.c against the CPU shim in ../cl_cpu.cpp.
 *
 * TEST INFRASTRUCTURE ONLY.  Written from the public OpenCL 1.1
 * specification: the types, the entry points main.c calls and the constants
 * it names.  The numeric values only have to agree with ../cl_cpu.cpp.
 */
#ifndef REF_SHIM_CL_H
#define REF_SHIM_CL_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int32_t cl_int;
typedef uint32_t cl_uint;
typedef uint64_t cl_ulong;
typedef cl_uint cl_bool;
typedef float cl_float;
typedef struct { float s[4]; } __attribute__((aligned(16))) cl_float4;
typedef cl_ulong cl_bitfield;
typedef cl_bitfield cl_device_type;
typedef cl_bitfield cl_mem_flags;
typedef cl_bitfield cl_command_queue_properties;
typedef cl_uint cl_device_info;
typedef cl_uint cl_platform_info;
typedef cl_uint cl_program_build_info;
typedef intptr_t cl_context_properties;

typedef struct _cl_platform_id *cl_platform_id;
typedef struct _cl_device_id *cl_device_id;
typedef struct _cl_context *cl_context;
typedef struct _cl_command_queue *cl_command_queue;
typedef struct _cl_mem *cl_mem;
typedef struct _cl_program *cl_program;
typedef struct _cl_kernel *cl_kernel;
typedef struct _cl_event *cl_event;

#define CL_SUCCESS 0
#define CL_DEVICE_NOT_FOUND -1
#define CL_MEM_OBJECT_ALLOCATION_FAILURE -4
#define CL_OUT_OF_HOST_MEMORY -6
#define CL_BUILD_PROGRAM_FAILURE -11
#define CL_INVALID_VALUE -30
#define CL_INVALID_MEM_OBJECT -38
#define CL_INVALID_KERNEL_NAME -46
#define CL_INVALID_ARG_INDEX -49
#define CL_INVALID_KERNEL_ARGS -52
#define CL_INVALID_WORK_GROUP_SIZE -54

#define CL_FALSE 0
#define CL_TRUE 1

#define CL_DEVICE_TYPE_GPU (1 << 2)

#define CL_MEM_READ_WRITE (1 << 0)
#define CL_MEM_WRITE_ONLY (1 << 1)
#define CL_MEM_READ_ONLY (1 << 2)

#define CL_PLATFORM_NAME 0x0902
#define CL_DEVICE_MAX_COMPUTE_UNITS 0x1002
#define CL_DEVICE_MAX_WORK_GROUP_SIZE 0x1004
#define CL_DEVICE_MAX_CLOCK_FREQUENCY 0x100C
#define CL_DEVICE_GLOBAL_MEM_SIZE 0x101F
#define CL_DEVICE_LOCAL_MEM_SIZE 0x1023
#define CL_DEVICE_NAME 0x102B
#define CL_DEVICE_VENDOR 0x102C
#define CL_DEVICE_EXTENSIONS 0x1030
#define CL_PROGRAM_BUILD_LOG 0x1183

cl_int clGetPlatformIDs(cl_uint num_entries, cl_platform_id *platforms, cl_uint *num_platforms);
cl_int clGetPlatformInfo(cl_platform_id platform, cl_platform_info name, size_t size, void *value,
                         size_t *size_ret);
cl_int clGetDeviceIDs(cl_platform_id platform, cl_device_type type, cl_uint num_entries,
                      cl_device_id *devices, cl_uint *num_devices);
cl_int clGetDeviceInfo(cl_device_id device, cl_device_info name, size_t size, void *value,
                       size_t *size_ret);
cl_context clCreateContext(const cl_context_properties *props, cl_uint num_devices,
                           const cl_device_id *devices,
                           void (*notify)(const char *, const void *, size_t, void *),
                           void *user_data, cl_int *errcode_ret);
cl_command_queue clCreateCommandQueue(cl_context context, cl_device_id device,
                                      cl_command_queue_properties props, cl_int *errcode_ret);
cl_program clCreateProgramWithSource(cl_context context, cl_uint count, const char **strings,
                                     const size_t *lengths, cl_int *errcode_ret);
cl_int clBuildProgram(cl_program program, cl_uint num_devices, const cl_device_id *devices,
                      const char *options, void (*notify)(cl_program, void *), void *user_data);
cl_int clGetProgramBuildInfo(cl_program program, cl_device_id device, cl_program_build_info name,
                             size_t size, void *value, size_t *size_ret);
cl_kernel clCreateKernel(cl_program program, const char *name, cl_int *errcode_ret);
cl_int clSetKernelArg(cl_kernel kernel, cl_uint index, size_t size, const void *value);
cl_int clEnqueueNDRangeKernel(cl_command_queue queue, cl_kernel kernel, cl_uint work_dim,
                              const size_t *global_offset, const size_t *global_size,
                              const size_t *local_size, cl_uint num_events,
                              const cl_event *wait_list, cl_event *event);
cl_int clFinish(cl_command_queue queue);
cl_mem clCreateBuffer(cl_context context, cl_mem_flags flags, size_t size, void *host_ptr,
                      cl_int *errcode_ret);
cl_int clEnqueueWriteBuffer(cl_command_queue queue, cl_mem buffer, cl_bool blocking, size_t offset,
                            size_t size, const void *ptr, cl_uint num_events,
                            const cl_event *wait_list, cl_event *event);
cl_int clEnqueueReadBuffer(cl_command_queue queue, cl_mem buffer, cl_bool blocking, size_t offset,
                           size_t size, void *ptr, cl_uint num_events, const cl_event *wait_list,
                           cl_event *event);
cl_int clEnqueueWriteBufferRect(cl_command_queue queue, cl_mem buffer, cl_bool blocking,
                                const size_t *buffer_origin, const size_t *host_origin,
                                const size_t *region, size_t buffer_row_pitch,
                                size_t buffer_slice_pitch, size_t host_row_pitch,
                                size_t host_slice_pitch, const void *ptr, cl_uint num_events,
                                const cl_event *wait_list, cl_event *event);
cl_int clEnqueueCopyBuffer(cl_command_queue queue, cl_mem src, cl_mem dst, size_t src_offset,
                           size_t dst_offset, size_t size, cl_uint num_events,
                           const cl_event *wait_list, cl_event *event);
cl_int clReleaseMemObject(cl_mem mem);
cl_int clReleaseKernel(cl_kernel kernel);
cl_int clReleaseProgram(cl_program program);
cl_int clReleaseCommandQueue(cl_command_queue queue);
cl_int clReleaseContext(cl_context context);

#ifdef __cplusplus
}
#endif
#endif
