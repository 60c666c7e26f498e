/* Prelude that lets OpenCL C kernel sources compile as C++ for the host CPU.
 *
 * TEST INFRASTRUCTURE ONLY.  oracle/Makefile force-includes this before the
 * reference's math.cl (and before the matmul source main.c generates at run
 * time) so those kernels build unchanged from the reference's own files:
 *
 *   __kernel  -> extern "C" function     __global -> nothing
 *   __local   -> static thread_local (each OS thread runs one work-group at a
 *                time, its work-items as fibers, so they share it as local
 *                memory is shared, and groups on other threads have their own)
 *   float4    -> struct with .s0-.s3 and the scalar*vector / vector+vector
 *                operators the kernels use
 *   get_*_id, barrier -> the work-item executor in cl_cpu.cpp
 *
 * Arithmetic is ordinary IEEE float; the build uses -ffp-contract=off.
 */
#ifndef MATHCL_PRELUDE_H
#define MATHCL_PRELUDE_H
#include <math.h>
#include <stddef.h>

#define __kernel extern "C"
#define __global
#define __local static thread_local
#define CLK_LOCAL_MEM_FENCE 1
#define CLK_GLOBAL_MEM_FENCE 2

struct alignas(16) float4 {
    float s0, s1, s2, s3;
    float4() = default;
    float4(float v) : s0(v), s1(v), s2(v), s3(v) {}
    float4 &operator+=(const float4 &o) {
        s0 += o.s0; s1 += o.s1; s2 += o.s2; s3 += o.s3;
        return *this;
    }
};
static inline float4 operator*(float a, const float4 &b) {
    float4 r;
    r.s0 = a * b.s0; r.s1 = a * b.s1; r.s2 = a * b.s2; r.s3 = a * b.s3;
    return r;
}
static inline float4 operator+(const float4 &a, const float4 &b) {
    float4 r;
    r.s0 = a.s0 + b.s0; r.s1 = a.s1 + b.s1; r.s2 = a.s2 + b.s2; r.s3 = a.s3 + b.s3;
    return r;
}

extern "C" size_t get_global_id(unsigned dim);
extern "C" size_t get_local_id(unsigned dim);
extern "C" size_t get_group_id(unsigned dim);
extern "C" size_t get_local_size(unsigned dim);
extern "C" size_t get_global_size(unsigned dim);
extern "C" void barrier(int flags);

#endif
