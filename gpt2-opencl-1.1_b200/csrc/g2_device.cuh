// g2_device.cuh -- device helpers shared by the kernel files: element
// conversion, the tanh GELU (math.cl:21-23) and the GEMM epilogue.
#pragma once
#include <cuda_fp16.h>

#include "g2_internal.h"

namespace g2 {

// Programmatic dependent launch: a kernel launched with it may start while
// the previous kernel of the stream is still running.  pdl_wait() returns once
// that kernel has completed and its writes are visible (a no-op for a normal
// launch); every such kernel calls it before reading anything a previous
// kernel wrote, and before writing anything a previous kernel reads.
// pdl_launch() lets the next kernel start launching.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch() { asm volatile("griddepcontrol.launch_dependents;" :::); }

__device__ __forceinline__ float tof(float v) { return v; }
__device__ __forceinline__ float tof(__half v) { return __half2float(v); }
template <typename T>
__device__ __forceinline__ T fromf(float v);
template <>
__device__ __forceinline__ float fromf<float>(float v) { return v; }
template <>
__device__ __forceinline__ __half fromf<__half>(float v) { return __float2half_rn(v); }

// tanh-form GELU (math.cl:21-23, HF "gelu_new").
__device__ __forceinline__ float gelu_f(float v) {
    return 0.5f * v * (1.0f + tanhf(0.7978845608f * (v + 0.044715f * v * v * v)));
}

// Store v as element i of a GEMM operand (OperandOut): tf32 hi / lo, or fp16.
__device__ __forceinline__ void put_operand(const OperandOut &o, size_t i, float v) {
    if (o.kind == 1) {
        unsigned t;
        asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(t) : "f"(v));
        const float h = __uint_as_float(t);
        asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(t) : "f"(v - h));
        o.hi[i] = h;
        o.lo[i] = __uint_as_float(t);
    } else if (o.kind == 0) {
        o.h16[i] = __float2half_rn(v);
    }
}

// Epilogue shared by gemv and gemm: v = acc (+bias) (GELU) (+resid), stored to
// out[r][n]; with EPI_KV the K and V thirds of a qkv row are also appended to
// the cache at (slot[r], layer, head, pos[r]) -- split_kv (math.cl:367-383).
template <typename WT>
struct Epi {
    const WT *bias;
    const float *resid;
    float *out;
    int N, epi;
    KVLayout kv;
    int layer;
    const int *pos;
    const int *slot;
    int E;

    // Returns the value stored to out[r][n].
    __device__ __forceinline__ float apply(int r, int n, float v) const {
        if (epi & EPI_BIAS) v += tof(bias[n]);
        if (epi & EPI_GELU) v = gelu_f(v);
        if (epi & EPI_RESID) v = resid[(size_t)r * N + n] + v;
        if (!(epi & EPI_NOSTORE)) out[(size_t)r * N + n] = v;
        if ((epi & EPI_KV) && n >= E) {
            const float stored = v;
            int m = n - E;
            const bool isv = m >= E;
            if (isv) m -= E;
            const int h = m >> 6, d = m & 63;
            const int p = pos[r];
            const int sl = slot[r];
            // positions and slots are validated on the host; never write outside (reported when checked)
            if (!G2_BOUNDS(p >= 0 && p < kv.max_seq && sl >= 0 && sl < kv.n_slots, 103)) return stored;
            const long long off = (long long)sl * kv.slot_stride + (long long)layer * kv.layer_stride +
                                  ((long long)h * kv.max_seq + p) * kHeadDim + d;
            WT *base = reinterpret_cast<WT *>(isv ? kv.v : kv.k);
            base[off] = fromf<WT>(v);
        }
        return v;
    }
};

}  // namespace g2
